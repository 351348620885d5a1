"""Cost graphs, gradient reports and the fast tier's integral and polynomial
costs against the float64 oracle, through the C ABI. B200 only.

* A quotient of two integral costs (interior residual over boundary term) is
  a graph whose leaf multipliers depend on the leaf values
  (cuda/graph_schedule.hpp:18-55 of the reference): both leaves' forward
  values are needed before either backward pass. Checked through op 14
  (value and weight gradients) over several chunks, and through op 15
  (three RPROP epochs) against an oracle-driven float32 RPROP trajectory.
* The kind-5 gradient report of training (squared L2 norm, max |g|,
  non-finite count and first index per layer,
  cuda/reduction_kernels.cuh:81-98) against numpy on the gradient buffers.
* Integral and polynomial costs on fast-tier networks of widths 32, 64, 96
  and 128: the fused expression head (integral costs, last hidden layer of
  32, 64 or 128 neurons) and the separate output-layer kernels (the other
  cases); at orders <= 3 the automatic tier runs widths 32 and 64 on the
  3xTF32 tensor cores (lo-first term order) and 96 and 128 on exact-FP32 FFMA.

Tolerances as in tests/golden_cases.py (1e-5 for orders <= 3, 1e-4 above).
"""
import numpy as np
import pytest

import golden_cases as gc
from cpde_b200 import codegen, native
from cpde_b200.client import graph_bytes, sum_graph
from cpde_b200.expressions import DIV, COMPONENT, Expression, glorot_like, quadrature_inputs, table
from cpde_b200.wire import Reader, Writer
from oracle import jets

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def engine():
    with native.Engine(0) as e:
        yield e


def disk_problem(interior=700, boundary=90, layers=(2, 32, 32, 1), seed=5):
    """Interior residual (u_xx + u_yy + 1)^2 on points in the unit disk and
    u^2 on its boundary circle."""
    rng = np.random.default_rng(seed)
    r, th = np.sqrt(rng.uniform(size=interior)), 2 * np.pi * rng.uniform(size=interior)
    t_in = table(['xx', 'yy'], 'xy')
    x_in = quadrature_inputs(np.stack([r * np.cos(th), r * np.sin(th)], 1), t_in)
    phi = 2 * np.pi * np.arange(boundary) / boundary
    t_bd = table([''], 'xy')
    x_bd = quadrature_inputs(np.stack([np.cos(phi), np.sin(phi)], 1), t_bd)
    e_in = Expression('(u_xx+u_yy+1)**2', table=t_in, variables='xy', outputs='u', count=interior)
    e_bd = Expression('u**2', table=t_bd, variables='xy', outputs='u', count=boundary)
    w_in, w_bd = np.full(interior, np.pi / interior), np.full(boundary, 2 * np.pi / boundary)
    weights = [a + np.float32(0.05) * np.random.default_rng(seed + 1).normal(size=a.shape).astype(np.float32)
               for a in glorot_like(list(layers), seed=0)]
    return (t_in, x_in, e_in, w_in), (t_bd, x_bd, e_bd, w_bd), list(layers), weights


def oracle_leaf(weights, layers, t, x, expr, qw):
    linear = [1] + [0] * (len(layers) - 2) + [1]
    schema = jets.Schema(t[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    loss, dout = jets.expression(acts[-1], [tuple(int(v) for v in n) for n in expr.nodes], expr.constants,
                                 expr.field_array(), qw)
    return loss, jets.backward(schema, weights, layers, linear, pre, acts, dout)


def oracle_quotient(weights, layers, interior, boundary):
    a, ga = oracle_leaf(weights, layers, *interior)
    b, gb = oracle_leaf(weights, layers, *boundary)
    return a / b, [x / b - a * y / (b * b) for x, y in zip(ga, gb)]


QUOTIENT = graph_bytes([[COMPONENT, 0, -1], [COMPONENT, 1, -1], [DIV, 0, 1]], [0.0, 0.0, 0.0], 2)


def make_leaves(engine, net, interior, boundary, chunks=(128, 40)):
    costs = []
    for (t, x, expr, qw), chunk in zip((interior, boundary), chunks):
        data = engine.data(x, t)
        costs.append(engine.integral(net, data, len(qw), np.asarray(expr.nodes, np.int32),
                                     np.asarray(expr.constants), expr.field_array(), qw, chunk=chunk))
    return costs


def test_quotient_graph_value_and_gradient(engine):
    interior, boundary, layers, weights = disk_problem()
    net = engine.network(layers, weights)
    costs = make_leaves(engine, net, interior, boundary)
    value, grads = engine.graph_evaluate(net, costs, QUOTIENT)
    expected_value, expected = oracle_quotient(weights, layers, interior, boundary)
    assert abs(value - expected_value) <= 1e-5 * abs(expected_value)
    assert gc.layer_error(grads, expected) < 1e-5
    # the leaves alone, through the plain sum graph, agree with the oracle too
    for cost, leaf in zip(costs, (interior, boundary)):
        v, g = engine.graph_evaluate(net, [cost], sum_graph(1))
        lv, lg = oracle_leaf(weights, layers, *leaf)
        assert abs(v - lv) <= 1e-5 * abs(lv) and gc.layer_error(g, lg) < 1e-5


def graph_train_body(net, costs, epochs, graph, diagnostics=0, optimizer=0):
    w = (Writer().put('Q', net).array(costs, 'u8').put('Q', epochs).put('i', optimizer).put('i', 1)
         .put('f', 0.0).put('i', 0).put('f', 0.0))
    for value in (0, 1, 0, 0, 0):  # verbose, log every, eval every, print outputs, save every
        w.put('i', value)
    w.string('').put('i', diagnostics)
    if graph is not None:
        w.raw(graph)
    return w.bytes()


def test_quotient_graph_training_matches_oracle_rprop(engine):
    interior, boundary, layers, weights = disk_problem(seed=9)
    net = engine.network(layers, weights)
    costs = make_leaves(engine, net, interior, boundary)
    events = engine.train(graph_train_body(net, costs, 3, QUOTIENT), graph_mode=True)
    assert events[-1][0] == 0
    w = [a.astype(np.float32).copy() for a in weights]
    steps = [np.full_like(a, np.float32(0.002)) for a in w]
    prev = [np.zeros_like(a) for a in w]
    for _ in range(3):
        _, g = oracle_quotient(w, layers, interior, boundary)
        for i in range(len(w)):
            g32 = g[i].astype(np.float32)
            jets.rprop(w[i], steps[i], g32, prev[i])
            prev[i] = g32
    _, state = engine.state(net)
    for layer, expected in zip(state, w):
        np.testing.assert_allclose(layer['buffers'][0], expected, rtol=0, atol=2e-5)
    # the leaf values of the last epoch are reported as graph events (kind 6)
    assert any(kind == 6 for kind, _ in events)


def decode_gradient_report(payload):
    r = Reader(payload)
    epoch, update, count = r.get('Q'), r.get('Q'), r.get('i')
    layers = [dict(squared_norm=r.get('d'), max_abs=r.get('d'), nonfinite=r.get('Q'), first=r.get('i'))
              for _ in range(count)]
    r.end()
    return epoch, update, layers


def test_gradient_report_matches_gradient_buffers(engine):
    interior, _, layers, weights = disk_problem(layers=(2, 64, 64, 1), seed=3)
    net = engine.network(layers, weights)
    cost = make_leaves(engine, net, interior, interior)[0]
    events = engine.train(graph_train_body(net, [cost], 1, None, diagnostics=1, optimizer=1))
    reports = [decode_gradient_report(p) for kind, p in events if kind == 5]
    assert len(reports) == 1
    epoch, update, stats = reports[0]
    assert epoch == 1 and update == 0
    _, state = engine.state(net)
    for layer, s in zip(state, stats):
        g = np.asarray(layer['buffers'][layer['active']], np.float64)  # Adam leaves the gradient as computed
        np.testing.assert_allclose(s['squared_norm'], np.dot(g, g), rtol=1e-9)
        assert s['max_abs'] == np.abs(g).max()
        assert s['nonfinite'] == 0 and s['first'] == -1
    # the reported gradient is the oracle's at the initial weights
    _, expected = oracle_leaf(weights, layers, *interior)
    for s, e in zip(stats, expected):
        assert abs(np.sqrt(s['squared_norm']) - np.linalg.norm(e)) <= 1e-5 * np.linalg.norm(e)


SCHEMA_CASES = [2, 4, 7]  # full 2D order 2, full 2D order 4, pure 2D order 2


@pytest.mark.parametrize('sid', SCHEMA_CASES, ids=[codegen.SCHEMAS[i][0] for i in SCHEMA_CASES])
@pytest.mark.parametrize('width', [32, 64, 96, 128])
@pytest.mark.parametrize('kind', ['integral', 'polynomial'])
def test_fast_tier_integral_and_polynomial_costs(engine, sid, width, kind):
    rows = codegen.SCHEMAS[sid][1]
    t = np.array([(sum(r), *r) for r in rows], np.int32)
    R, P = len(t), 517
    rng = np.random.default_rng(sid + width)
    x = quadrature_inputs(rng.uniform(-1, 1, (P, 2)), t)
    layers = [2, width, width, width, 1]
    weights = [(rng.normal(size=h * (w + 1)) / np.sqrt(w)).astype(np.float32) for w, h in zip(layers[:-1], layers[1:])]
    net = engine.network(layers, weights)
    data = engine.data(x, t)
    top = [i for i in range(R) if t[i, 0] == t[:, 0].max()]
    qw = rng.uniform(0.5, 1.5, P)
    if kind == 'integral':
        names = ['u_' + 'x' * int(t[i, 1]) + 'y' * int(t[i, 2]) for i in top]
        expr = Expression('(' + '+'.join(names) + '+u-1)**2', table=t, variables='xy', outputs='u', count=P)
        cost = engine.integral(net, data, P, np.asarray(expr.nodes, np.int32), np.asarray(expr.constants),
                               expr.field_array(), qw, chunk=200)
    else:
        terms = [(0, i, -1) for i in top] + [(0, 0, 0)]
        coeffs = rng.uniform(0.5, 1.5, (len(terms), P)).astype(np.float32)
        rhs = np.ones((1, P), np.float32)
        cost = engine.polynomial(net, data, list(range(R)), 1, terms, coeffs, rhs, qw.astype(np.float32)[None],
                                 chunk=200)
    engine.timing(True)
    engine.timing_report()
    try:
        value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
        report = engine.timing_report()
    finally:
        engine.timing(False)
    # integral costs on a last hidden layer of 32, 64 or 128 neurons take the
    # fused expression head; the others the fast tier's separate output layer
    fused = kind == 'integral' and width in (32, 64, 128)
    assert ('head_expression' if fused else 'output_backward') in report
    schema = jets.Schema(t[:, 1:])
    linear = [1, 0, 0, 0, 1]
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    if kind == 'integral':
        loss, dout = jets.expression(acts[-1], [tuple(int(v) for v in n) for n in expr.nodes], expr.constants,
                                     expr.field_array(), qw)
    else:
        loss, dout = jets.polynomial(acts[-1], terms, coeffs, rhs, qw.astype(np.float32)[None])
    expected = jets.backward(schema, weights, layers, linear, pre, acts, dout)
    tol = gc.tolerance(t)
    assert abs(value - loss) <= tol * abs(loss)
    assert gc.layer_error(grads, expected) < tol
