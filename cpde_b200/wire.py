"""Little-endian framed wire format of the cPDE server protocol.

A frame is ``u64 length`` (4 + payload bytes, 4 <= length <= 4 GiB), ``u32 kind``
and the payload. Arrays are a ``u64`` element count followed by the raw
elements; strings are byte arrays. This restates the contract of the reference
(cuda/protocol.hpp:10-51, cpde/_wire.py:4-26) in code written for this package.
"""
import struct

import numpy as np

FRAME_LIMIT = 4 * 1024 ** 3


class Writer:
    """Accumulates one payload."""

    def __init__(self):
        self._parts = []

    def put(self, fmt, value):
        self._parts.append(struct.pack('<' + fmt, value))
        return self

    def array(self, values, dtype):
        a = np.ascontiguousarray(values, dtype=np.dtype(dtype).newbyteorder('<'))
        self._parts.append(struct.pack('<Q', a.size))
        self._parts.append(a.tobytes())
        return self

    def string(self, text):
        raw = text.encode('utf-8') if isinstance(text, str) else bytes(text)
        self._parts.append(struct.pack('<Q', len(raw)))
        self._parts.append(raw)
        return self

    def raw(self, payload):
        self._parts.append(bytes(payload))
        return self

    def bytes(self):
        return b''.join(self._parts)


class Reader:
    """Consumes one payload; every accessor checks the remaining length."""

    def __init__(self, payload):
        self.data = payload
        self.pos = 0

    def take(self, n):
        if self.pos + n > len(self.data):
            raise RuntimeError('truncated server reply')
        out = self.data[self.pos:self.pos + n]
        self.pos += n
        return out

    def get(self, fmt):
        size = struct.calcsize('<' + fmt)
        return struct.unpack('<' + fmt, self.take(size))[0]

    def array(self, dtype):
        dt = np.dtype(dtype).newbyteorder('<')
        count = self.get('Q')
        return np.frombuffer(self.take(count * dt.itemsize), dtype=dt).copy()

    def string(self):
        return self.take(self.get('Q')).decode('utf-8')

    def remaining(self):
        return len(self.data) - self.pos

    def end(self):
        if self.pos != len(self.data):
            raise RuntimeError('unexpected trailing reply fields')


OPTIMIZERS = {-1: None, 0: 'rprop', 1: 'adam'}


def read_metadata(r):
    """State metadata v1 (cuda/cpde_server.cu:193-198)."""
    if r.get('I') != 1:
        raise ValueError('unsupported state version')
    meta = dict(neurons=r.array('i4').tolist(), linear=r.array('i4').tolist())
    meta['optimizer'] = OPTIMIZERS[r.get('i')]
    for key in ('updates', 'adam_step', 'stage_completed', 'remaining'):
        meta[key] = r.get('Q')
    meta['learning_rate'] = r.get('f')
    meta['initial_step'] = r.get('f')
    meta['stage'] = r.string()
    return meta


def decode_state(blob):
    """Snapshot blob: metadata then, per layer, i32 active buffer and 4 f32 arrays
    {W, g1, g2, steps-or-moment} (cuda/cpde_server.cu:199-206)."""
    r = Reader(blob)
    meta = read_metadata(r)
    layers = []
    ns = meta['neurons']
    for width, height in zip(ns[:-1], ns[1:]):
        active = r.get('i')
        buffers = [r.array('f4') for _ in range(4)]
        if active not in (1, 2) or any(len(b) != height * (width + 1) for b in buffers):
            raise ValueError('invalid state buffers')
        layers.append(dict(active=active, buffers=buffers))
    r.end()
    return meta, layers


def encode_state(meta, layers):
    """Inverse of decode_state (the op-10 restore payload)."""
    w = Writer().put('I', 1).array(meta['neurons'], 'i4').array(meta['linear'], 'i4')
    w.put('i', {None: -1, 'rprop': 0, 'adam': 1}[meta['optimizer']])
    for key in ('updates', 'adam_step', 'stage_completed', 'remaining'):
        w.put('Q', meta[key])
    w.put('f', meta['learning_rate']).put('f', meta['initial_step']).string(meta['stage'])
    for layer in layers:
        w.put('i', layer['active'])
        for b in layer['buffers']:
            w.array(b, 'f4')
    return w.bytes()
