"""Python client for any server that speaks the cPDE wire protocol.

It drives both the reference server (the oracle build under ``oracle/_ref``)
and this package's ``cpde_server`` with identical requests, which is how the
parity tests and the benchmark compare them. Names follow the reference front
end (cpde/api.py: ``Session`` :28, ``Data`` :153, ``Network`` :259) and the
request layouts follow the server (cuda/cpde_server.cu:436-555); the class
bodies are this package's own.
"""
import queue
import struct
import subprocess
import threading

import numpy as np

from .wire import FRAME_LIMIT, Reader, Writer, decode_state, encode_state, read_metadata

OP_QUIT, OP_HELLO, OP_DATA, OP_NET, OP_EVAL, OP_DOWNLOAD, OP_REPLACE, OP_COST = range(8)
OP_TRAIN, OP_SNAPSHOT, OP_RESTORE, OP_RELEASE, OP_INTEGRAL, OP_INSPECT, OP_GRAPH_EVAL, OP_GRAPH_TRAIN = range(8, 16)
OP_BENCH, OP_STOP = 90, 99


class ServerError(RuntimeError):
    """A kind-1 reply: the server rejected the command and stays usable."""


class Session:
    """One server process; requests are serialised, replies read by a thread."""

    def __init__(self, executable, *, device=0, args=None, env=None):
        cmd = [str(executable)] + (list(args) if args is not None else ['--device', str(device)])
        self.process = subprocess.Popen(cmd, stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                        stderr=subprocess.PIPE, bufsize=0, env=env)
        self.diagnostics = []
        self._replies = queue.Queue()
        self._lock = threading.RLock()
        self._closed = False
        threading.Thread(target=self._read_stderr, daemon=True).start()
        threading.Thread(target=self._read_stdout, daemon=True).start()
        r = self.request(OP_HELLO)
        self.protocol = r.string()
        self.version = r.get('i')
        self.capabilities = r.get('I')
        r.end()
        if self.protocol != 'CPDE/3' or self.version != 6:
            raise RuntimeError('incompatible server')

    def _read_stderr(self):
        for line in iter(self.process.stderr.readline, b''):
            self.diagnostics.append(line.decode('utf-8', 'replace').rstrip())

    def _exact(self, n):
        parts = []
        while n:
            chunk = self.process.stdout.read(n)
            if not chunk:
                raise RuntimeError('server stopped: ' + '\n'.join(self.diagnostics[-20:]))
            parts.append(chunk)
            n -= len(chunk)
        return b''.join(parts)

    def _read_stdout(self):
        try:
            while True:
                size = struct.unpack('<Q', self._exact(8))[0]
                if not 4 <= size <= FRAME_LIMIT:
                    raise RuntimeError('invalid reply frame')
                payload = self._exact(size)
                self._replies.put((struct.unpack_from('<I', payload)[0], Reader(payload[4:])))
        except BaseException as e:  # delivered to the waiting request
            self._replies.put(e)

    def send(self, op, body=b''):
        if self._closed:
            raise RuntimeError('session is closed')
        frame = struct.pack('<QI', len(body) + 4, op) + body
        self.process.stdin.write(frame)
        self.process.stdin.flush()

    def receive(self):
        item = self._replies.get()
        if isinstance(item, BaseException):
            raise item
        return item

    def request(self, op, body=b''):
        with self._lock:
            self.send(op, body)
            kind, r = self.receive()
            if kind == 1:
                raise ServerError(r.string())
            if kind != 0:
                raise RuntimeError(f'unexpected reply kind {kind}')
            return r

    def stop(self):
        self.send(OP_STOP)

    def release(self, kind, handle):
        self.request(OP_RELEASE, Writer().put('i', kind).put('Q', handle).bytes()).end()

    def close(self):
        if self._closed:
            return
        try:
            self.request(OP_QUIT)
        finally:
            self._closed = True
            self.process.stdin.close()
            self.process.wait(timeout=120)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Data:
    """Samples laid out (derivative, channel, sample) on the client; the server
    stores (derivative, sample, channel) (cpde/api.py:167)."""

    def __init__(self, session, samples, table, handle=None, shape=None):
        self.session = session
        self.table = np.asarray(table, np.int32)
        if handle is not None:
            self.handle, self.shape = handle, shape
            return
        a = np.asarray(samples, np.float32)
        if a.ndim != 3 or a.shape[0] != len(self.table):
            raise ValueError('samples must be (derivative, channel, sample)')
        self.shape = a.shape
        w = Writer()
        for x in (*a.shape, self.table.shape[1] - 1):
            w.put('i', x)
        w.array(self.table, 'i4').array(a.transpose(0, 2, 1), 'f4')
        r = session.request(OP_DATA, w.bytes())
        self.handle = r.get('Q')
        r.end()

    @property
    def samples(self):
        return self.shape[2]

    def to_numpy(self):
        r = self.session.request(OP_DOWNLOAD, Writer().put('Q', self.handle).bytes())
        a = r.array('f4')
        r.end()
        d, c, n = self.shape
        return a.reshape(d, n, c).transpose(0, 2, 1).copy()

    def replace(self, samples):
        a = np.asarray(samples, np.float32)
        if a.shape != self.shape:
            raise ValueError('replacement must keep the data shape')
        body = Writer().put('Q', self.handle).array(a.transpose(0, 2, 1), 'f4').bytes()
        self.session.request(OP_REPLACE, body).end()

    def close(self):
        self.session.release(0, self.handle)


class Cost:
    def __init__(self, net, handle, rows, kind):
        self.net, self.handle, self.rows, self.kind = net, handle, rows, kind

    def close(self):
        self.net.session.release(2, self.handle)


def graph_bytes(nodes, constants, root):
    return Writer().array(np.asarray(nodes, np.int32).reshape(-1, 3), 'i4').array(
        np.asarray(constants, np.float64), 'f8').put('i', int(root)).bytes()


def sum_graph(count):
    """Cost graph that adds ``count`` leaves: leaf nodes first, then a running
    sum (the shape cpde/cost.py:99-103 emits for a CostSum)."""
    nodes = [[1, i, -1] for i in range(count)]
    total = 0
    for i in range(1, count):
        nodes.append([3, total, i])
        total = len(nodes) - 1
    return graph_bytes(nodes, [0.0] * len(nodes), total)


class Network:
    """An MLP held by the server. ``weights`` is a list of per-layer flat arrays:
    column-major W (n_l x n_{l-1}) followed by the bias (cpde/api.py:278-283)."""

    def __init__(self, session, layers, *, weights, linear=None):
        self.session = session
        self.layers = [int(x) for x in layers]
        self.linear = [1] + [0] * (len(layers) - 2) + [1] if linear is None else [int(x) for x in linear]
        w = Writer().array(self.layers, 'i4').array(self.linear, 'i4')
        for values in weights:
            w.array(values, 'f4')
        r = session.request(OP_NET, w.bytes())
        self.handle = r.get('Q')
        r.end()

    # --- state ---------------------------------------------------------
    def snapshot(self):
        r = self.session.request(OP_SNAPSHOT, Writer().put('Q', self.handle).bytes())
        return r.data

    def state(self):
        return decode_state(self.snapshot())

    def restore(self, meta, layers):
        body = Writer().put('Q', self.handle).raw(encode_state(meta, layers)).bytes()
        self.session.request(OP_RESTORE, body).end()

    def weights(self):
        return [layer['buffers'][0] for layer in self.state()[1]]

    def set_weights(self, arrays):
        meta, layers = self.state()
        for layer, a in zip(layers, arrays):
            layer['buffers'][0] = np.asarray(a, np.float32)
        self.restore(meta, layers)

    def gradients(self):
        """Active gradient buffer of each layer (the last backward's result)."""
        return [layer['buffers'][layer['active']] for layer in self.state()[1]]

    # --- evaluation ----------------------------------------------------
    def eval(self, data, chunk=0):
        body = Writer().put('Q', self.handle).put('Q', data.handle).put('i', chunk).bytes()
        r = self.session.request(OP_EVAL, body)
        handle = r.get('Q')
        r.end()
        return Data(self.session, None, data.table, handle=handle,
                    shape=(data.shape[0], self.layers[-1], data.shape[2]))

    # --- costs ---------------------------------------------------------
    def matching(self, inputs, targets, weights, chunk=0):
        """Kind-0 squared-error matching (cpde/api.py:346-363 encoding)."""
        from .expressions import closure
        outputs = self.layers[-1]
        d, n = len(inputs.table), inputs.samples
        w = np.asarray(weights, np.float32)
        active = np.any(w != 0, axis=0)
        if active.ndim == 2:
            active = active.any(axis=1)
        rows = closure(inputs.table, np.flatnonzero(active))
        weight_samples = 1 if w.ndim == 2 else n
        packed = w[:, rows].T[:, None, :] if w.ndim == 2 else w[:, rows, :].transpose(1, 2, 0)
        keys = {tuple(int(x) for x in row): i for i, row in enumerate(targets.table)}
        target_rows = [keys[tuple(int(x) for x in inputs.table[i])] for i in rows]
        body = (Writer().put('Q', self.handle).put('Q', inputs.handle).put('Q', targets.handle)
                .put('i', 0).put('i', chunk).array(rows, 'i4').array(target_rows, 'i4')
                .put('i', weight_samples).array(packed, 'f4').bytes())
        r = self.session.request(OP_COST, body)
        c = Cost(self, r.get('Q'), rows, 0)
        r.end()
        return c

    def polynomial(self, inputs, polynomials, *, rhs=None, weights=None, chunk=0):
        """Kind-1 residuals; ``polynomials`` is a list (one per equation) of
        ``{(a,) or (a, b): coefficients}`` over data-table component indices."""
        from .expressions import closure
        outputs = self.layers[-1]
        n = inputs.samples
        e = len(polynomials)
        rv = np.zeros((e, n), np.float32) if rhs is None else np.asarray(rhs, np.float32).reshape(e, n)
        wv = np.ones((e, n), np.float32) if weights is None else np.asarray(weights, np.float32).reshape(e, n)
        used = {i // outputs for k, poly in enumerate(polynomials) if np.any(wv[k] != 0)
                for mono, co in poly.items() if np.any(co != 0) for i in mono}
        rows = closure(inputs.table, used)
        remap = {old: new for new, old in enumerate(rows)}
        terms, coeffs = [], []
        for k, poly in enumerate(polynomials):
            if not np.any(wv[k] != 0):
                continue
            for mono, co in poly.items():
                if not np.any(co != 0):
                    continue
                idx = [remap[x // outputs] * outputs + x % outputs for x in mono]
                terms.append((k, idx[0], idx[1] if len(idx) == 2 else -1))
                coeffs.append(np.broadcast_to(np.asarray(co, np.float32), (n,)))
        body = (Writer().put('Q', self.handle).put('Q', inputs.handle).put('Q', 0).put('i', 1)
                .put('i', chunk).array(rows, 'i4').put('i', e).array(np.asarray(terms, np.int32).reshape(-1, 3), 'i4')
                .array(np.asarray(coeffs, np.float32).reshape(-1), 'f4').array(rv, 'f4').array(wv, 'f4').bytes())
        r = self.session.request(OP_COST, body)
        c = Cost(self, r.get('Q'), rows, 1)
        r.end()
        return c

    def integral(self, inputs, expression, *, weights=None, chunk=0):
        """Kind-2 compiled integral: ``expression`` is an expressions.Expression
        bound to ``inputs``' table; ``weights`` are per-sample quadrature weights."""
        n = inputs.samples if inputs is not None else expression.count
        qw = np.ones(n) if weights is None else np.broadcast_to(np.asarray(weights, np.float64), (n,))
        fields = expression.field_array()
        body = (Writer().put('Q', self.handle).put('Q', inputs.handle if inputs is not None else 0)
                .put('i', chunk).put('i', n).array(np.asarray(expression.nodes, np.int32).reshape(-1, 3), 'i4')
                .array(np.asarray(expression.constants, np.float64), 'f8').put('i', len(fields))
                .array(fields, 'f8').array(qw, 'f8').bytes())
        r = self.session.request(OP_INTEGRAL, body)
        c = Cost(self, r.get('Q'), None, 2)
        r.end()
        return c

    # --- training / evaluation of objectives ------------------------------
    def evaluate(self, costs, *, graph=None, gradient=False):
        """Op 14: value of the cost graph (default: sum of leaves), optionally
        with per-layer weight gradients. Optimizer state is left untouched."""
        graph = sum_graph(len(costs)) if graph is None else graph
        body = (Writer().put('Q', self.handle).array([c.handle for c in costs], 'u8')
                .put('i', int(gradient)).raw(graph).bytes())
        r = self.session.request(OP_GRAPH_EVAL, body)
        value = r.get('d')
        if not gradient:
            r.end()
            return value
        count = r.get('i')
        grads = [r.array('f4') for _ in range(count)]
        r.end()
        return value, grads

    def train(self, costs, epochs, *, optimizer='rprop', reset=False, steps=0.0, moments=False, lr=0.0,
              log_every=1, eval_every=0, print_outputs=False, save_every=0, stage='', diagnostics=0,
              graph=None, restore_every=0, restore_step=0.0, on_event=None):
        """Op 8 (plain sum of costs) or op 15 (with ``graph``). Returns
        (completed, stopped, metadata, events)."""
        w = (Writer().put('Q', self.handle).array([c.handle for c in costs], 'u8').put('Q', epochs)
             .put('i', int(optimizer == 'adam')).put('i', int(reset)).put('f', steps).put('i', int(moments))
             .put('f', lr))
        for value in (1, log_every, eval_every, int(print_outputs), save_every):
            w.put('i', value)
        w.string(stage).put('i', diagnostics)
        if graph is not None:
            w.raw(graph)
        if restore_every:
            w.put('Q', restore_every).put('f', restore_step)
        events = []
        with self.session._lock:
            self.session.send(OP_GRAPH_TRAIN if graph is not None else OP_TRAIN, w.bytes())
            while True:
                kind, r = self.session.receive()
                if kind == 1:
                    raise ServerError(r.string())
                if kind == 0:
                    completed, stopped = r.get('Q'), bool(r.get('i'))
                    meta = read_metadata(Reader(r.take(r.get('Q'))))
                    r.end()
                    return dict(completed=completed, stopped=stopped, metadata=meta, events=events)
                event = self._decode_event(kind, r)
                events.append(event)
                if on_event is not None:
                    on_event(event)

    def _decode_event(self, kind, r):
        if kind in (2, 6):
            ev = dict(kind=kind, epoch=r.get('Q'), update=r.get('Q'), after=r.get('i'), values=r.array('f8'))
            if kind == 6:
                ev['total'] = r.get('d')
            r.end()
            return ev
        if kind == 3:
            return dict(kind=3, blob=r.data)
        if kind == 4:
            ev = dict(kind=4, cost=r.get('Q'), outputs=r.array('f4'))
            r.end()
            return ev
        if kind == 5:
            ev = dict(kind=5, epoch=r.get('Q'), update=r.get('Q'))
            count = r.get('i')
            ev['layers'] = [dict(squared_norm=r.get('d'), max_abs=r.get('d'), nonfinite=r.get('Q'),
                                 first=r.get('i')) for _ in range(count)]
            r.end()
            return ev
        raise RuntimeError(f'unexpected training event kind {kind}')

    def benchmark(self, cost, warm=3, iterations=10, batches=3):
        """Op 90: fixed-weight epochs (forward + loss + weight gradients) timed
        inside the server. Returns (wall ms, device ms, loss, gradients)."""
        body = (Writer().put('Q', self.handle).put('Q', cost.handle).put('i', warm).put('i', iterations)
                .put('i', batches).bytes())
        r = self.session.request(OP_BENCH, body)
        wall, device, loss = r.array('f8'), r.array('f8'), r.get('d')
        grads = [r.array('f4') for _ in range(len(self.layers) - 1)]
        r.end()
        return wall, device, loss, grads

    def close(self):
        self.session.release(1, self.handle)
