"""In-process binding of the C ABI (include/cpde_b200.h) with ctypes.

The engine runs inside the calling process, on the device it was created on.
Importing this module never falls back to anything: if libcpde_b200.so is
missing or fails to load, ``load()`` raises.
"""
import ctypes
from pathlib import Path

import numpy as np

from .wire import Reader, Writer, decode_state, encode_state

LIBRARY = Path(__file__).resolve().parent / 'libcpde_b200.so'
SERVER = Path(__file__).resolve().parent / 'bin' / 'cpde_server'

OK, REJECTED, DEVICE_ERROR = 0, 1, 2

SINK = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t)
EVENT = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t)

_lib = None

# name -> (restype, argtypes); mirrors include/cpde_b200.h
P, U64, I32, SZ = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int32, ctypes.c_size_t
PI32, PF32, PF64, PU64 = (ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float),
                          ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint64))
SIGNATURES = {
    'cpde_engine_create': (I32, [I32, ctypes.POINTER(P)]),
    'cpde_engine_create_sharded': (I32, [I32, I32, I32, P, ctypes.POINTER(P)]),
    'cpde_sharding_id': (I32, [P, SZ]),
    'cpde_shard_range': (I32, [ctypes.c_int64, I32, I32, ctypes.POINTER(ctypes.c_int64),
                               ctypes.POINTER(ctypes.c_int64)]),
    'cpde_engine_destroy': (None, [P]),
    'cpde_last_error': (ctypes.c_char_p, [P]),
    'cpde_hello': (I32, [P, SINK, P]),
    'cpde_data_create': (I32, [P, I32, I32, I32, I32, PI32, SZ, PF32, SZ, PU64]),
    'cpde_data_shape': (I32, [P, U64, PI32, PI32, PI32]),
    'cpde_data_download': (I32, [P, U64, PF32, SZ]),
    'cpde_data_replace': (I32, [P, U64, PF32, SZ]),
    'cpde_net_create': (I32, [P, PI32, PI32, I32, ctypes.POINTER(PF32), ctypes.POINTER(SZ), PU64]),
    'cpde_net_evaluate': (I32, [P, U64, U64, I32, PU64]),
    'cpde_net_snapshot': (I32, [P, U64, SINK, P]),
    'cpde_net_restore': (I32, [P, U64, P, SZ]),
    'cpde_cost_matching': (I32, [P, U64, U64, U64, I32, PI32, SZ, PI32, SZ, I32, PF32, SZ, PU64]),
    'cpde_cost_polynomial': (I32, [P, U64, U64, I32, PI32, SZ, I32, PI32, SZ, PF32, SZ, PF32, SZ, PF32, SZ, PU64]),
    'cpde_cost_integral': (I32, [P, U64, U64, I32, I32, PI32, SZ, PF64, SZ, I32, PF64, SZ, PF64, SZ, PU64]),
    'cpde_cost_source': (I32, [P, U64, I32, SINK, SINK, P]),
    'cpde_release': (I32, [P, I32, U64]),
    'cpde_train': (I32, [P, I32, P, SZ, EVENT, P, PI32]),
    'cpde_graph_evaluate': (I32, [P, P, SZ, SINK, P]),
    'cpde_benchmark': (I32, [P, U64, U64, I32, I32, I32, SINK, P]),
    'cpde_epoch': (I32, [P, U64, PU64, SZ]),
    'cpde_epoch_result': (I32, [P, U64, PF64, PF32, SZ]),
    'cpde_engine_stream': (I32, [P, ctypes.POINTER(P)]),
    'cpde_kernel_timing': (I32, [P, I32]),
    'cpde_kernel_timing_report': (I32, [P, SINK, P]),
    'cpde_set_tier': (I32, [P, I32]),
    'cpde_jet_plan': (I32, [PI32, I32, I32, PI32, SZ, ctypes.POINTER(SZ)]),
    'cpde_layer_gradient_static': (I32, [P, P, P, I32, I32, ctypes.c_int64, I32, P, P]),
}


def load():
    """Load libcpde_b200.so and declare every entry point; raises if absent."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise RuntimeError(f'{LIBRARY} is not built; run python -m cpde_b200.build')
        lib = ctypes.CDLL(str(LIBRARY))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class EngineError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


def _ptr(a, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def _i32(a):
    return np.ascontiguousarray(a, np.int32)


def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def _f64(a):
    return np.ascontiguousarray(a, np.float64)


class _Collector:
    """Accumulates sink callbacks into bytes objects."""

    def __init__(self):
        self.parts = []
        self.cb = SINK(self._sink)

    def _sink(self, _ctx, data, length):
        self.parts.append(ctypes.string_at(data, length) if length else b'')


def jet_plan(counts):
    """Host-only schema compiler; returns the packed int32 table."""
    lib = load()
    c = _i32(counts)
    n = ctypes.c_size_t()
    if lib.cpde_jet_plan(_ptr(c, ctypes.c_int32), c.shape[0], c.shape[1], None, 0, ctypes.byref(n)) != OK:
        raise ValueError('invalid derivative schema')
    out = np.zeros(n.value, np.int32)
    lib.cpde_jet_plan(_ptr(c, ctypes.c_int32), c.shape[0], c.shape[1], _ptr(out, ctypes.c_int32), out.size,
                      ctypes.byref(n))
    return out


def sharding_id():
    """A fresh 128-byte NCCL group id (rank 0 creates it, every rank joins with it)."""
    lib = load()
    buf = ctypes.create_string_buffer(128)
    status = lib.cpde_sharding_id(buf, 128)
    if status != OK:
        raise EngineError(status, 'NCCL is unavailable for sharded engines')
    return buf.raw


def shard_range(total, rank, world):
    """(first sample, sample count) of rank's shard of ``total`` samples."""
    lo, count = ctypes.c_int64(), ctypes.c_int64()
    if load().cpde_shard_range(total, rank, world, ctypes.byref(lo), ctypes.byref(count)) != OK:
        raise ValueError('invalid shard request')
    return lo.value, count.value


class Engine:
    """One engine on one CUDA device, driven through the C ABI. With
    ``world > 1`` it is rank ``rank`` of a point-sharded group joined through
    ``unique_id`` (from :func:`sharding_id` on rank 0): every rank receives the
    same requests, keeps its own shard of each Data object and sums gradients
    and cost totals over the group once per epoch."""

    def __init__(self, device=0, rank=0, world=1, unique_id=None):
        self.lib = load()
        handle = ctypes.c_void_p()
        if world > 1:
            uid = ctypes.create_string_buffer(bytes(unique_id), 128)
            status = self.lib.cpde_engine_create_sharded(device, rank, world, uid, ctypes.byref(handle))
        else:
            status = self.lib.cpde_engine_create(device, ctypes.byref(handle))
        self.handle = handle
        if status != OK:
            message = self.lib.cpde_last_error(handle).decode() if handle else 'engine creation failed'
            if handle:
                self.lib.cpde_engine_destroy(handle)
            self.handle = None
            raise EngineError(status, message)

    def close(self):
        if self.handle:
            self.lib.cpde_engine_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, status):
        if status != OK:
            raise EngineError(status, self.lib.cpde_last_error(self.handle).decode())

    # --- objects ---------------------------------------------------------
    def data(self, samples, table):
        """``samples`` in client layout (derivative, channel, sample)."""
        a = _f32(np.asarray(samples, np.float32).transpose(0, 2, 1))
        t = _i32(table)
        out = ctypes.c_uint64()
        d, n, c = a.shape
        self._check(self.lib.cpde_data_create(self.handle, d, c, n, t.shape[1] - 1, _ptr(t, ctypes.c_int32), t.size,
                                              _ptr(a, ctypes.c_float), a.size, ctypes.byref(out)))
        return out.value

    def download(self, handle):
        d, c, s = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        self._check(self.lib.cpde_data_shape(self.handle, handle, ctypes.byref(d), ctypes.byref(c), ctypes.byref(s)))
        a = np.zeros((d.value, s.value, c.value), np.float32)
        self._check(self.lib.cpde_data_download(self.handle, handle, _ptr(a, ctypes.c_float), a.size))
        return a.transpose(0, 2, 1).copy()

    def replace(self, handle, samples):
        a = _f32(np.asarray(samples, np.float32).transpose(0, 2, 1))
        self._check(self.lib.cpde_data_replace(self.handle, handle, _ptr(a, ctypes.c_float), a.size))

    def replace_raw(self, handle, address, count):
        """Replace values from host memory already in the engine's
        (derivative, sample, channel) layout, e.g. a pinned buffer."""
        self._check(self.lib.cpde_data_replace(self.handle, handle, ctypes.cast(address, PF32), count))

    def network(self, layers, weights, linear=None):
        linear = [1] + [0] * (len(layers) - 2) + [1] if linear is None else list(linear)
        ns, ls = _i32(layers), _i32(linear)
        arrays = [_f32(w) for w in weights]
        ptrs = (PF32 * len(arrays))(*[_ptr(a, ctypes.c_float) for a in arrays])
        counts = (ctypes.c_size_t * len(arrays))(*[a.size for a in arrays])
        out = ctypes.c_uint64()
        self._check(self.lib.cpde_net_create(self.handle, _ptr(ns, ctypes.c_int32), _ptr(ls, ctypes.c_int32), len(ns),
                                             ptrs, counts, ctypes.byref(out)))
        return out.value

    def evaluate(self, net, data, chunk=0):
        out = ctypes.c_uint64()
        self._check(self.lib.cpde_net_evaluate(self.handle, net, data, chunk, ctypes.byref(out)))
        return out.value

    def snapshot(self, net):
        col = _Collector()
        self._check(self.lib.cpde_net_snapshot(self.handle, net, col.cb, None))
        return b''.join(col.parts)

    def state(self, net):
        return decode_state(self.snapshot(net))

    def restore(self, net, blob):
        buf = ctypes.create_string_buffer(blob, len(blob))
        self._check(self.lib.cpde_net_restore(self.handle, net, buf, len(blob)))

    def set_weights(self, net, arrays):
        meta, layers = self.state(net)
        for layer, a in zip(layers, arrays):
            layer['buffers'][0] = np.asarray(a, np.float32)
        self.restore(net, encode_state(meta, layers))

    def matching(self, net, inputs, targets, rows, target_rows, weight_samples, weights, chunk=0):
        r, tr, w = _i32(rows), _i32(target_rows), _f32(weights)
        out = ctypes.c_uint64()
        self._check(self.lib.cpde_cost_matching(self.handle, net, inputs, targets, chunk, _ptr(r, ctypes.c_int32),
                                                r.size, _ptr(tr, ctypes.c_int32), tr.size, weight_samples,
                                                _ptr(w, ctypes.c_float), w.size, ctypes.byref(out)))
        return out.value

    def polynomial(self, net, inputs, rows, equations, terms, coefficients, rhs, weights, chunk=0):
        r, t = _i32(rows), _i32(np.asarray(terms, np.int32).reshape(-1))
        co, rh, w = _f32(coefficients).reshape(-1), _f32(rhs).reshape(-1), _f32(weights).reshape(-1)
        out = ctypes.c_uint64()
        self._check(self.lib.cpde_cost_polynomial(self.handle, net, inputs, chunk, _ptr(r, ctypes.c_int32), r.size,
                                                  equations, _ptr(t, ctypes.c_int32), t.size,
                                                  _ptr(co, ctypes.c_float), co.size, _ptr(rh, ctypes.c_float), rh.size,
                                                  _ptr(w, ctypes.c_float), w.size, ctypes.byref(out)))
        return out.value

    def integral(self, net, inputs, samples, nodes, constants, fields, weights, chunk=0):
        nd = _i32(np.asarray(nodes, np.int32).reshape(-1))
        c, f, w = _f64(constants), _f64(fields).reshape(-1), _f64(weights)
        nfields = 0 if f.size == 0 else int(np.asarray(fields).shape[0])
        out = ctypes.c_uint64()
        self._check(self.lib.cpde_cost_integral(self.handle, net, inputs, chunk, samples, _ptr(nd, ctypes.c_int32),
                                                nd.size, _ptr(c, ctypes.c_double), c.size, nfields,
                                                _ptr(f, ctypes.c_double), f.size, _ptr(w, ctypes.c_double), w.size,
                                                ctypes.byref(out)))
        return out.value

    def source(self, cost, compile=True):
        col = _Collector()
        self._check(self.lib.cpde_cost_source(self.handle, cost, int(compile), col.cb, col.cb, None))
        return col.parts[0].decode(), col.parts[1].decode()

    def release(self, kind, handle):
        self._check(self.lib.cpde_release(self.handle, kind, handle))

    # --- epochs ----------------------------------------------------------
    def graph_evaluate(self, net, costs, graph, gradient=True):
        body = Writer().put('Q', net).array(list(costs), 'u8').put('i', int(gradient)).raw(graph).bytes()
        col = _Collector()
        buf = ctypes.create_string_buffer(body, len(body))
        self._check(self.lib.cpde_graph_evaluate(self.handle, buf, len(body), col.cb, None))
        r = Reader(b''.join(col.parts))
        value = r.get('d')
        if not gradient:
            return value, None
        count = r.get('i')
        grads = [r.array('f4') for _ in range(count)]
        r.end()
        return value, grads

    def train(self, body, graph_mode=False, stop=None):
        events = []

        def on_event(_ctx, kind, data, length):
            events.append((kind, ctypes.string_at(data, length) if length else b''))

        cb = EVENT(on_event)
        buf = ctypes.create_string_buffer(body, len(body))
        flag = stop if stop is not None else ctypes.c_int32(0)
        self._check(self.lib.cpde_train(self.handle, int(graph_mode), buf, len(body), cb, None, ctypes.byref(flag)))
        return events

    def epoch(self, net, costs):
        ids = np.ascontiguousarray(costs, np.uint64)
        self._check(self.lib.cpde_epoch(self.handle, net, _ptr(ids, ctypes.c_uint64), ids.size))

    def epoch_result(self, net, params):
        value = ctypes.c_double()
        g = np.zeros(params, np.float32)
        self._check(self.lib.cpde_epoch_result(self.handle, net, ctypes.byref(value), _ptr(g, ctypes.c_float), g.size))
        return value.value, g

    def benchmark(self, net, cost, warm, iterations, batches, layers):
        col = _Collector()
        self._check(self.lib.cpde_benchmark(self.handle, net, cost, warm, iterations, batches, col.cb, None))
        r = Reader(b''.join(col.parts))
        wall, device, loss = r.array('f8'), r.array('f8'), r.get('d')
        grads = [r.array('f4') for _ in range(layers)]
        r.end()
        return wall, device, loss, grads

    def stream(self):
        s = ctypes.c_void_p()
        self._check(self.lib.cpde_engine_stream(self.handle, ctypes.byref(s)))
        return s.value

    def timing(self, enable):
        self._check(self.lib.cpde_kernel_timing(self.handle, int(enable)))

    def timing_report(self):
        col = _Collector()
        self._check(self.lib.cpde_kernel_timing_report(self.handle, col.cb, None))
        out = {}
        for line in b''.join(col.parts).decode().splitlines():
            name, launches, ms = line.split()
            out[name] = (int(launches), float(ms))
        return out

    def set_tier(self, tier):
        self._check(self.lib.cpde_set_tier(self.handle, tier))
