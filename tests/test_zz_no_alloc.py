"""The allocation-free layer-gradient entry point (cpde_layer_gradient_static).

It exists for callers that cannot allocate device memory: hosts whose own
allocator owns the GPU's memory, and latency-bound code that must not take
cudaMalloc's implicit synchronisation. Its answer must equal the weight
gradient the engine's regular objective entry point (op 14,
cpde_graph_evaluate) reports for the same layer, within the parity tests'
1e-5 normwise bound, on two calls in a row, since both calls share the
library's static scratch array: one layer inside a single 128 x 128 tile with
two column splits, and one of 2 x 2 tiles whose many splits fill most of the
array. This file is collected last on purpose; it also passes alone in a fresh
process.
"""
import ctypes

import numpy as np
import pytest

import golden_cases as gc
from cpde_b200 import native
from cpde_b200.client import sum_graph
from cpde_b200.expressions import all_mixed

pytestmark = pytest.mark.gpu


def linear_case(engine, seed, inputs=8, outputs=4, points=300):
    """Linear layer inputs -> outputs with a matching cost; returns the
    interleaved dZ and inputs and the gradient op 14 reports."""
    rng = np.random.default_rng(seed)
    t = all_mixed(2, 'xy')
    R = len(t)
    x = rng.normal(size=(R, inputs, points)).astype(np.float32)
    w = rng.normal(size=outputs * (inputs + 1)).astype(np.float32) * 0.3
    net = engine.network([inputs, outputs], [w], [1, 1])
    data = engine.data(x, t)
    targets = rng.normal(size=(R, outputs, points)).astype(np.float32)
    tgt = engine.data(targets, t)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, outputs), np.float32))
    _, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
    z = engine.download(engine.evaluate(net, data))
    dz = (np.float32(2.0) * (z - targets)).astype(np.float32)  # matching adjoint, unit weights
    dz_il = np.ascontiguousarray(dz.transpose(2, 0, 1)).reshape(-1)  # (point, row, output)
    x_il = np.ascontiguousarray(x.transpose(2, 0, 1)).reshape(-1)    # (point, row, input)
    return dz_il, x_il, grads[0], R, points


@pytest.mark.parametrize('inputs,outputs,points', [(8, 4, 300), (192, 256, 40000)], ids=['one_tile', 'many_splits'])
def test_static_scratch_gradient_matches_graph_evaluate_twice(inputs, outputs, points):
    import torch
    torch.cuda.init()
    with native.Engine(0) as engine:
        for seed in (1, 2):  # two calls in a row share the static scratch
            dz, x, expected, R, P = linear_case(engine, seed, inputs, outputs, points)
            d_dz = torch.from_numpy(dz).cuda()
            d_x = torch.from_numpy(x).cuda()
            d_g = torch.full((outputs * (inputs + 1),), float('nan'), device='cuda')
            torch.cuda.synchronize()
            status = engine.lib.cpde_layer_gradient_static(engine.handle, ctypes.c_void_p(d_dz.data_ptr()),
                                                           ctypes.c_void_p(d_x.data_ptr()), outputs, inputs, P, R,
                                                           ctypes.c_void_p(d_g.data_ptr()), None)
            engine._check(status)
            torch.cuda.synchronize()  # device-wide: covers the engine stream the call used
            got = d_g.cpu().numpy()
            assert gc.layer_error([got], [expected.astype(np.float64)]) < 1e-5


def test_static_scratch_rejects_oversized_layers():
    with native.Engine(0) as engine:
        status = engine.lib.cpde_layer_gradient_static(engine.handle, ctypes.c_void_p(16), ctypes.c_void_p(16),
                                                       4096, 4096, 10, 1, ctypes.c_void_p(16), None)
        assert status == native.REJECTED
        assert 'static scratch' in engine.lib.cpde_last_error(engine.handle).decode()
