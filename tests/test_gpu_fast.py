"""Fast-tier kernels (fused GEMM + register jets) against the oracle and the
generic tier, for every schema with generated jet code. B200 only.

Tolerances: per-row normwise relative error of outputs and per-layer normwise
relative error of weight gradients vs the float64 oracle, 1e-5 for orders <= 3
and 1e-4 for orders 4-6 (same rule as tests/golden_cases.py)."""
import numpy as np
import pytest

import golden_cases as gc
from cpde_b200 import codegen, native
from cpde_b200.client import sum_graph
from cpde_b200.expressions import quadrature_inputs
from oracle import jets

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def engine():
    with native.Engine(0) as e:
        yield e


def schema_table(rows):
    return np.array([(sum(r), *r) for r in rows], np.int32)


def setup(engine, rows, layers, linear, points, seed):
    rng = np.random.default_rng(seed)
    t = schema_table(rows)
    V = t.shape[1] - 1
    pts = rng.uniform(-1, 1, (points, V))
    x = quadrature_inputs(pts, t)
    x[2 * V + 1:] = rng.normal(size=x[2 * V + 1:].shape) * 0.1 if len(t) > 2 * V + 1 else x[2 * V + 1:]
    weights = [(rng.normal(size=h * (w + 1)) * (1.0 / np.sqrt(w))).astype(np.float32)
               for w, h in zip(layers[:-1], layers[1:])]
    net = engine.network(layers, weights, linear)
    data = engine.data(x, t)
    return t, x, weights, net, data


CASES = [(sid, name, rows) for sid, (name, rows) in enumerate(codegen.SCHEMAS)]


@pytest.mark.parametrize('sid,name,rows', CASES, ids=[c[1] for c in CASES])
@pytest.mark.parametrize('act', [0, 2], ids=['sigmoid', 'tanh'])
@pytest.mark.parametrize('tier', [0, 2, 4], ids=['auto', 'tensor', 'ffma'])
def test_fast_tier_matches_oracle(engine, sid, name, rows, act, tier):
    V = len(rows[0])
    engine.set_tier(tier)
    layers = [V, 128, 128, 128, 2] if tier == 2 else [V, 64, 32, 64, 2]
    linear = [1, act, act, act, 1]
    P = 203  # not a multiple of any tile's point count
    t, x, weights, net, data = setup(engine, rows, layers, linear, P, sid + 10 * act)
    out = engine.download(engine.evaluate(net, data, chunk=97))
    schema = jets.Schema(t[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    tol = gc.tolerance(t)
    assert gc.rowwise_error(out, acts[-1]).max() < tol
    targets = (acts[-1] * 0.5).astype(np.float32)
    tgt = engine.data(targets, t)
    R = len(t)
    mw = np.random.default_rng(1).uniform(0.5, 1.5, (R, 1, 2)).astype(np.float32)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, mw, chunk=120)
    value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
    loss, dout = jets.matching(acts[-1], targets, mw.transpose(0, 2, 1))
    expected = jets.backward(schema, weights, layers, linear, pre, acts, dout)
    assert abs(value - loss) <= tol * abs(loss)
    assert gc.layer_error(grads, expected) < tol
    engine.set_tier(1)
    try:
        gen_value, gen_grads = engine.graph_evaluate(net, [cost], sum_graph(1))
    finally:
        engine.set_tier(0)
    if tier == 2:
        engine.set_tier(2)
        tc_out = engine.download(engine.evaluate(net, data, chunk=97))
        engine.set_tier(0)
        assert gc.rowwise_error(tc_out, acts[-1]).max() < tol
    assert abs(value - gen_value) <= tol * abs(gen_value)
    assert gc.layer_error(grads, gen_grads) < tol


def test_fast_tier_wide_layers_and_single_output(engine):
    """Config-style shapes: 2 -> 256 -> 128 -> 256 -> 1, order 4, many points."""
    rows = codegen.SCHEMAS[4][1]
    layers = [2, 256, 128, 256, 1]
    linear = [1, 0, 0, 0, 1]
    t, x, weights, net, data = setup(engine, rows, layers, linear, 1500, 3)
    schema = jets.Schema(t[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    out = engine.download(engine.evaluate(net, data))
    assert gc.rowwise_error(out, acts[-1]).max() < 1e-4
    R = len(t)
    tgt = engine.data(np.zeros_like(out), t)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32))
    value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
    loss, dout = jets.matching(acts[-1], np.zeros_like(out), 1.0)
    expected = jets.backward(schema, weights, layers, linear, pre, acts, dout)
    assert abs(value - loss) <= 1e-4 * loss
    assert gc.layer_error(grads, expected) < 1e-4


@pytest.mark.parametrize('sid', [8, 9, 10], ids=[codegen.SCHEMAS[i][0] for i in (8, 9, 10)])
def test_tensor_tier_many_tiles_per_cta(engine, sid):
    """Warp-specialised layers with several column tiles per CTA, for the
    schemas whose backward ring has no more stages than a tile has K slabs
    (25 and 35 rows at 128 neurons): one MMA issuer takes every tile there.
    The network mixes 128-wide and 256-wide layers, so the wide kernels and
    the wider weight gradient run the same way."""
    rows = codegen.SCHEMAS[sid][1]
    V = len(rows[0])
    layers = [V, 128, 128, 256, 128, 1]
    linear = [1, 0, 0, 0, 0, 1]
    t, x, weights, net, data = setup(engine, rows, layers, linear, 1200, 60 + sid)
    schema = jets.Schema(t[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    engine.set_tier(2)
    try:
        out = engine.download(engine.evaluate(net, data))
        R = len(t)
        tgt = engine.data(np.zeros_like(out), t)
        cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32))
        engine.timing(True)
        engine.timing_report()
        value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
        report = engine.timing_report()
    finally:
        engine.timing(False)
        engine.set_tier(0)
    for k in ('forward_ws', 'forward_wide', 'backward_ws', 'backward_wide', 'weight_gradient_ws'):
        assert k in report, (k, sorted(report))
    assert gc.rowwise_error(out, acts[-1]).max() < 1e-4
    loss, dout = jets.matching(acts[-1], np.zeros_like(out), 1.0)
    expected = jets.backward(schema, weights, layers, linear, pre, acts, dout)
    assert abs(value - loss) <= 1e-4 * loss
    assert gc.layer_error(grads, expected) < 1e-4


@pytest.mark.parametrize('width', [128, 512])
def test_tensor_weight_gradient_over_many_columns(engine, width):
    """The tensor-core weight gradient sums hundreds of thousands of columns
    per layer; its accumulators are folded into round-to-nearest FP32 sums
    every few chunks, so the result stays as close to the exact-FP32 FFMA
    kernels' as a short sum would (without the folding the drift grew with
    the column count: 3e-5 on config 2, 6e-4 on config 5). Order 3 (tier 0
    runs FFMA there), 65,536 and 16,384 points."""
    rows = codegen.SCHEMAS[3][1]
    layers = [2, width, width, width, 1]
    linear = [1, 0, 0, 0, 1]
    P = 65536 if width == 128 else 16384
    t, x, weights, net, data = setup(engine, rows, layers, linear, P, 5)
    R = len(t)
    tgt = engine.data(np.zeros((R, 1, P), np.float32), t)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32))
    engine.set_tier(4)
    try:
        exact_value, exact = engine.graph_evaluate(net, [cost], sum_graph(1))
        engine.set_tier(2)
        value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
    finally:
        engine.set_tier(0)
    err = [float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b)) for a, b in zip(grads, exact)]
    assert abs(value - exact_value) <= 1e-5 * abs(exact_value)
    # what remains is the GEMMs' own 3xTF32 error (accumulation over K = 512
    # inputs in the wide layers), not the length of the column sums
    assert max(err) < (5e-6 if width == 128 else 2e-5), err


@pytest.mark.parametrize('sid', [2, 3, 7], ids=[codegen.SCHEMAS[i][0] for i in (2, 3, 7)])
@pytest.mark.parametrize('width', [32, 64, 96])
def test_tensor_tier_narrow_layers(engine, sid, width):
    """Tensor-core (3xTF32) layers narrower than the 128-row tile: the rows
    past the layer's width are zero weights, not stored; layers of at most 64
    neurons and inputs pair two column tiles per accumulator (an odd tile
    count leaves the last pair's second tile empty: 12,001 points of 5 rows
    are 481 tiles). Orders <= 3, so the exact-FP32 tolerance 1e-5 applies;
    several tiles per CTA."""
    rows = codegen.SCHEMAS[sid][1]
    layers = [2, width, width, width, 1]
    linear = [1, 0, 0, 0, 1]
    t, x, weights, net, data = setup(engine, rows, layers, linear, 12001, 80 + sid + width)
    schema = jets.Schema(t[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    R = len(t)
    targets = (acts[-1] * 0.5).astype(np.float32)
    tgt = engine.data(targets, t)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32))
    engine.set_tier(2)
    try:
        out = engine.download(engine.evaluate(net, data))
        engine.timing(True)
        engine.timing_report()
        value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
        report = engine.timing_report()
    finally:
        engine.timing(False)
        engine.set_tier(0)
    for k in ('forward_ws', 'backward_ws', 'backward_input_ws', 'weight_gradient_ws'):
        assert k in report, (k, sorted(report))
    assert gc.rowwise_error(out, acts[-1]).max() < 1e-5
    loss, dout = jets.matching(acts[-1], targets, 1.0)
    expected = jets.backward(schema, weights, layers, linear, pre, acts, dout)
    assert abs(value - loss) <= 1e-5 * abs(loss)
    assert gc.layer_error(grads, expected) < 1e-5


@pytest.mark.parametrize('sid', [1, 3, 11], ids=[codegen.SCHEMAS[i][0] for i in (1, 3, 11)])
def test_ffma_tier_wide_tiles(engine, sid):
    """Exact-FP32 FFMA layers (orders <= 3 at tier 0) with 128-neuron tiles
    and a 160-neuron layer (a full and a 32-row slice), 6,001 points (above
    the automatic tier's point-tile epoch limit of 16,384 columns) over many
    column tiles, against the float64 oracle at 1e-5."""
    rows = codegen.SCHEMAS[sid][1]
    V = len(rows[0])
    layers = [V, 128, 160, 128, 1]
    linear = [1, 0, 0, 0, 1]
    t, x, weights, net, data = setup(engine, rows, layers, linear, 6001, 90 + sid)
    schema = jets.Schema(t[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    out = engine.download(engine.evaluate(net, data))
    assert gc.rowwise_error(out, acts[-1]).max() < 1e-5
    R = len(t)
    targets = (acts[-1] * 0.5).astype(np.float32)
    tgt = engine.data(targets, t)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32))
    engine.timing(True)
    engine.timing_report()
    try:
        value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
        report = engine.timing_report()
    finally:
        engine.timing(False)
    for k in ('forward', 'backward', 'backward_input', 'weight_gradient'):
        assert k in report, (k, sorted(report))
    loss, dout = jets.matching(acts[-1], targets, 1.0)
    expected = jets.backward(schema, weights, layers, linear, pre, acts, dout)
    assert abs(value - loss) <= 1e-5 * abs(loss)
    assert gc.layer_error(grads, expected) < 1e-5


@pytest.mark.parametrize('sid', [2, 6])
@pytest.mark.parametrize('width,outputs', [(32, 1), (64, 3), (96, 2), (128, 3)])
def test_output_layer_widths(engine, sid, width, outputs):
    """The separate output-layer kernels (every cost except a matching cost on
    a 128- or 256-wide last layer with few outputs): last hidden widths that
    divide 128 (one neuron slice per CTA, several point lanes), one that does
    not, and several outputs; the point count is not a multiple of any lane
    count."""
    rows = codegen.SCHEMAS[sid][1]
    V = len(rows[0])
    layers = [V, 64, width, outputs]
    linear = [1, 0, 0, 1]
    t, x, weights, net, data = setup(engine, rows, layers, linear, 1001, 40 + sid + width)
    schema = jets.Schema(t[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    tol = gc.tolerance(t)
    out = engine.download(engine.evaluate(net, data))
    assert gc.rowwise_error(out, acts[-1]).max() < tol
    R = len(t)
    targets = (acts[-1] * 0.5).astype(np.float32)
    tgt = engine.data(targets, t)
    mw = np.random.default_rng(2).uniform(0.5, 1.5, (R, 1, outputs)).astype(np.float32)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, mw)
    value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
    loss, dout = jets.matching(acts[-1], targets, mw.transpose(0, 2, 1))
    expected = jets.backward(schema, weights, layers, linear, pre, acts, dout)
    assert abs(value - loss) <= tol * abs(loss)
    assert gc.layer_error(grads, expected) < tol


POINT_SHAPES = {'o1': [128, 64, 128, 1], 'o2': [128, 128, 2], 'wide': [96, 256, 1]}


@pytest.mark.parametrize('sid,name,rows', CASES, ids=[c[1] for c in CASES])
@pytest.mark.parametrize('act', [0, 2], ids=['sigmoid', 'tanh'])
@pytest.mark.parametrize('shape', sorted(POINT_SHAPES))
def test_point_epoch_matches_oracle(engine, sid, name, rows, act, shape):
    """Tier 3: the single-launch point-tile epoch (matching costs), over
    several chunks with a ragged tail, against the float64 oracle."""
    V = len(rows[0])
    layers = [V] + POINT_SHAPES[shape]
    linear = [1] + [act] * (len(layers) - 2) + [1]
    P = 157
    t, x, weights, net, data = setup(engine, rows, layers, linear, P, 100 + sid + 10 * act)
    schema = jets.Schema(t[:, 1:])
    pre, acts = jets.forward(schema, weights, layers, linear, x)
    targets = (acts[-1] * 0.5).astype(np.float32)
    tgt = engine.data(targets, t)
    R, O = len(t), layers[-1]
    mw = np.random.default_rng(2).uniform(0.5, 1.5, (R, 1, O)).astype(np.float32)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, mw, chunk=64)
    engine.set_tier(3)
    try:
        value, grads = engine.graph_evaluate(net, [cost], sum_graph(1))
    finally:
        engine.set_tier(0)
    loss, dout = jets.matching(acts[-1], targets, mw.transpose(0, 2, 1))
    expected = jets.backward(schema, weights, layers, linear, pre, acts, dout)
    tol = gc.tolerance(t)
    assert abs(value - loss) <= tol * abs(loss)
    assert gc.layer_error(grads, expected) < tol


def test_point_epoch_is_the_launched_kernel(engine):
    """Tier 3 runs the point-tile epoch and its partial sum, nothing per layer."""
    rows = codegen.SCHEMAS[3][1]
    layers = [2, 128, 128, 128, 1]
    t, x, weights, net, data = setup(engine, rows, layers, [1, 0, 0, 0, 1], 300, 7)
    R = len(t)
    tgt = engine.data(np.zeros((R, 1, 300), np.float32), t)
    cost = engine.matching(net, data, tgt, list(range(R)), list(range(R)), 1, np.ones((R, 1, 1), np.float32))
    engine.set_tier(3)
    try:
        engine.timing(True)
        engine.timing_report()
        engine.epoch(net, [cost])
        report = engine.timing_report()
    finally:
        engine.timing(False)
        engine.set_tier(0)
    assert report['point_epoch'][0] == 1
    assert not any(k in report for k in ('forward', 'backward', 'weight_gradient', 'head_matching'))
