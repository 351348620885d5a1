"""Shared access to the golden fixtures and the oracle's answers for them.

Tolerances (stated once, used by every parity test): per-row normwise relative
error ||a-b||_2/||b||_2 of output jets and per-layer normwise relative error of
weight gradients against the float64 oracle must stay below 1e-5 when the
highest derivative order is <= 3 and 1e-4 for orders 4-6 (the north-star
bound). The reference's own float32 results sit about 2e-6 from the oracle.
"""
from pathlib import Path

import numpy as np

from oracle import jets

GOLDEN = Path(__file__).resolve().parent / 'golden'


def names():
    return sorted(p.stem for p in GOLDEN.glob('*.npz'))


def load(name):
    with np.load(GOLDEN / f'{name}.npz') as f:
        return {k: f[k] for k in f.files}


def tolerance(table):
    return 1e-5 if int(np.max(table[:, 0])) <= 3 else 1e-4


def weights_of(case, prefix='w'):
    count = len(case['layers']) - 1
    return [case[f'{prefix}{i}'] for i in range(count)]


def rowwise_error(actual, expected):
    a = np.asarray(actual, np.float64).reshape(len(expected), -1)
    b = np.asarray(expected, np.float64).reshape(len(expected), -1)
    norm = np.linalg.norm(b, axis=1)
    return np.linalg.norm(a - b, axis=1) / np.where(norm > 0, norm, 1.0)


def layer_error(actual, expected):
    return max(float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-300))
               for a, b in zip(actual, expected))


def oracle_outputs(case):
    schema = jets.Schema(case['table'][:, 1:])
    layers = [int(x) for x in case['layers']]
    linear = [int(x) for x in case['linear']]
    pre, acts = jets.forward(schema, weights_of(case), layers, linear, case['inputs'])
    return schema, layers, linear, pre, acts


def oracle_cost(case, y):
    """(loss, dE/dy) of the case's cost on output jets y (R, outputs, P)."""
    if 'targets' in case:
        w = case['match_weights'].T[:, :, None]
        return jets.matching(y, case['targets'], w)
    if 'poly_weights' in case:
        P = y.shape[2]
        comps = [int(c) for c in case['poly_components']]
        terms = [(0, c, -1) for c in comps]
        coeffs = [np.ones(P) for _ in comps]
        return jets.polynomial(y, terms, coeffs, np.zeros((1, P)), case['poly_weights'])
    nodes = [tuple(int(v) for v in n) for n in case['nodes']]
    return jets.expression(y, nodes, case['constants'], np.zeros((0, y.shape[2])), case['quad_weights'])


def oracle_gradients(case):
    schema, layers, linear, pre, acts = oracle_outputs(case)
    loss, dout = oracle_cost(case, acts[-1])
    grads = jets.backward(schema, weights_of(case), layers, linear, pre, acts, dout)
    return loss, grads, acts[-1]


def oracle_training(case, optimizer, epochs=4):
    """Float32 optimizer trajectory driven by float64 oracle gradients."""
    weights = [w.astype(np.float32).copy() for w in weights_of(case)]
    schema = jets.Schema(case['table'][:, 1:])
    layers = [int(x) for x in case['layers']]
    linear = [int(x) for x in case['linear']]
    state = [dict(steps=np.full_like(w, np.float32(0.002)), prev=np.zeros_like(w), m=np.zeros_like(w),
                  v=np.zeros_like(w)) for w in weights]
    for epoch in range(1, epochs + 1):
        pre, acts = jets.forward(schema, weights, layers, linear, case['inputs'])
        _, dout = oracle_cost(case, acts[-1])
        grads = jets.backward(schema, weights, layers, linear, pre, acts, dout)
        for w, g, st in zip(weights, grads, state):
            g32 = g.astype(np.float32)
            if optimizer == 'rprop':
                jets.rprop(w, st['steps'], g32, st['prev'])
                st['prev'] = g32
            else:
                jets.adam(w, g32, st['m'], st['v'], epoch, 0.001)
    return weights, [st['steps'] if optimizer == 'rprop' else st['m'] for st in state]
