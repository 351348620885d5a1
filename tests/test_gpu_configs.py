"""The benchmarked configurations' kernels against the float64 oracle.

Each case is one of bench.py's workloads (configs 2-5: same network widths,
activations, derivative rows and cost kind) cut to a point count the oracle
finishes in seconds but still large enough to take the kernels the full-size
bench takes; the per-kernel timing report proves which kernels ran. Outputs
(op 4, every data row), the objective and the weight gradients (op 14) are
compared with the oracle. Tolerances, as everywhere: per-row normwise
relative error of the outputs and per-layer normwise relative error of the
weight gradients below 1e-5 when the highest order is <= 3 and 1e-4 for
orders 4-6; objectives within the same relative bound. B200 only.
"""
import pytest

import bench
import golden_cases as gc
from cpde_b200 import native
from cpde_b200.client import sum_graph
from oracle import jets

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def engine():
    with native.Engine(0) as e:
        yield e


def oracle_epoch(w):
    """(outputs, loss, gradients) of the workload from the float64 oracle."""
    schema = jets.Schema(w.t[:, 1:])
    pre, acts = jets.forward(schema, w.weights, w.layers, w.linear, w.x)
    y = acts[-1]
    kind, *a = w.cost
    if kind == 'matching':
        loss, dout = jets.matching(y, a[0], a[1].transpose(0, 2, 1))
    elif kind == 'integral':
        loss, dout = jets.expression(y, [tuple(int(v) for v in n) for n in a[0]], a[1], a[2], a[3])
    else:
        loss, dout = jets.polynomial(y, a[0], a[1], a[2], a[3][None, :])
    return y, loss, jets.backward(schema, w.weights, w.layers, w.linear, pre, acts, dout)


def check(engine, w, kernels, tol):
    net, data, cost = w.own(engine)
    out = engine.download(engine.evaluate(net, data, chunk=w.chunk))
    engine.timing(True)
    engine.timing_report()
    try:
        value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
        report = engine.timing_report()
    finally:
        engine.timing(False)
    missing = [k for k in kernels if k not in report]
    assert not missing, f'kernels {missing} did not run; ran {sorted(report)}'
    y, loss, expected = oracle_epoch(w)
    assert gc.rowwise_error(out, y).max() < tol
    assert abs(value - loss) <= tol * abs(loss)
    assert gc.layer_error(grads, expected) < tol
    for kind, h in ((2, cost), (0, data), (1, net)):
        engine.release(kind, h)


def test_config2_kernels(engine):
    """2 -> 128^4 -> 1 sigmoid, order 6 all mixed, matching: the
    warp-specialised tensor-core layers and the fused matching head (the
    point count is above the point-tile epoch's limit)."""
    w = bench.config2_workload(1024)
    check(engine, w, ['input_forward', 'forward_ws', 'head_matching', 'weight_gradient_ws', 'backward_ws',
                      'backward_input_ws'], 1e-4)


@pytest.mark.parametrize('tier', [0, 2, 4], ids=['auto', 'tensor', 'ffma'])
def test_config3_kernels(engine, tier):
    """2 -> 64^3 -> 1 sigmoid, rows u, u_x, u_y, u_xx, u_yy, compiled integral
    of (u_xx + u_yy + 1)^2 over points in the disk: the tensor-core layers
    (64 neurons: paired column tiles, lo-first term order, 64-neuron
    weight-gradient slices), which the automatic tier takes at orders <= 3
    when no hidden layer is wider than 64, and the exact-FP32 FFMA layers
    (tier 4), both at 1e-5."""
    w = bench.config3_workload(2048)
    kernels = (['input_forward', 'forward', 'head_expression', 'weight_gradient', 'backward', 'backward_input']
               if tier == 4 else
               ['input_forward', 'forward_ws', 'head_expression', 'weight_gradient_ws', 'backward_ws',
                'backward_input_ws'])
    engine.set_tier(tier)
    try:
        check(engine, w, kernels, 1e-5)
    finally:
        engine.set_tier(0)


def test_config4_kernels(engine):
    """3 -> 256^3 -> 1 tanh (config 4's width, activation, rows and cost with
    two hidden layers fewer), the biharmonic residual integral over the 25-row
    closure, two chunks of several column tiles per CTA."""
    w = bench.config4_workload(2000, chunk=1100)
    w.layers = [3, 256, 256, 256, 1]
    w.linear = [1, 2, 2, 2, 1]
    w.weights = w.weights[:3] + w.weights[-1:]
    check(engine, w, ['input_forward', 'forward_wide', 'cost_integral', 'output_backward', 'weight_gradient_ws',
                      'backward_wide', 'backward_input_wide'], 1e-4)


def test_config5_kernels(engine):
    """4 -> 512^3 -> 1 sigmoid (config 5's width and rows with three hidden
    layers fewer), pure order-6 rows along 4 axes, polynomial residual with
    per-point weights, two chunks of several column tiles per CTA."""
    w = bench.config5_workload(600, chunk=350)
    w.layers = [4, 512, 512, 512, 1]
    w.linear = [1, 0, 0, 0, 1]
    w.weights = w.weights[:3] + w.weights[-1:]
    check(engine, w, ['input_forward', 'forward_wide', 'cost_polynomial', 'output_backward', 'weight_gradient_ws',
                      'backward_wide', 'backward_input_wide'], 1e-4)
