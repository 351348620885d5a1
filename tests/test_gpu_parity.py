"""CUDA engine parity against the oracle and the reference's golden outputs.

Runs on a B200 only. Everything goes through the C ABI (in-process via
cpde_b200.native) or through bin/cpde_server. Tolerances are those of
tests/golden_cases.py: per-row normwise relative error 1e-5 (orders <= 3) or
1e-4 (orders 4-6) against the float64 oracle.
"""
import numpy as np
import pytest

import golden_cases as gc
from cpde_b200 import native
from cpde_b200.client import Data, Network, Session, sum_graph
from cpde_b200.wire import Writer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def engine():
    with native.Engine(0) as e:
        yield e


def load_case(engine, case):
    layers = [int(x) for x in case['layers']]
    linear = [int(x) for x in case['linear']]
    net = engine.network(layers, gc.weights_of(case), linear)
    data = engine.data(case['inputs'], case['table'])
    return net, data, layers, linear


def make_cost(engine, case, net, data, layers):
    t = case['table']
    R = len(t)
    outputs = layers[-1]
    if 'targets' in case:
        tgt = engine.data(case['targets'], t)
        mw = case['match_weights']
        rows = list(range(R))  # every row carries weight in the fixtures
        packed = mw[:, rows].T[:, None, :]
        return engine.matching(net, data, tgt, rows, rows, 1, packed)
    P = case['inputs'].shape[2]
    if 'poly_weights' in case:
        comps = [int(c) for c in case['poly_components']]
        terms = [(0, c, -1) for c in comps]
        coeffs = np.ones((len(comps), P), np.float32)
        return engine.polynomial(net, data, list(range(R)), 1, terms, coeffs, np.zeros((1, P)),
                                 case['poly_weights'])
    return engine.integral(net, data, P, case['nodes'], case['constants'], np.zeros((0, P)), case['quad_weights'],
                           chunk=16)


@pytest.mark.parametrize('name', gc.names())
def test_output_jets(engine, name):
    case = gc.load(name)
    net, data, layers, _ = load_case(engine, case)
    out = engine.download(engine.evaluate(net, data, chunk=7))
    _, _, _, _, acts = gc.oracle_outputs(case)
    tol = gc.tolerance(case['table'])
    assert gc.rowwise_error(out, acts[-1]).max() < tol
    assert gc.rowwise_error(out, case['outputs']).max() < tol


@pytest.mark.parametrize('name', gc.names())
def test_objective_and_gradients(engine, name):
    case = gc.load(name)
    net, data, layers, _ = load_case(engine, case)
    cost = make_cost(engine, case, net, data, layers)
    value, grads = engine.graph_evaluate(net, [cost], sum_graph(1), gradient=True)
    loss, expected, _ = gc.oracle_gradients(case)
    tol = gc.tolerance(case['table'])
    assert abs(value - loss) <= 10 * tol * abs(loss) + 1e-12
    assert gc.layer_error(grads, expected) < tol
    assert gc.layer_error(grads, gc.weights_of(case, 'g')) < 2 * tol


def train_body(net, costs, epochs, optimizer):
    w = (Writer().put('Q', net).array(costs, 'u8').put('Q', epochs).put('i', int(optimizer == 'adam'))
         .put('i', 1).put('f', 0.0).put('i', 0).put('f', 0.0))
    for value in (0, 1, 0, 0, 0):
        w.put('i', value)
    return w.string('').put('i', 0).bytes()


@pytest.mark.parametrize('name', ['fourier_order2', 'fourier_order3', 'chunked_multioutput', 'linear_hidden'])
@pytest.mark.parametrize('optimizer', ['rprop', 'adam'])
def test_training_trajectory_matches_reference(engine, name, optimizer):
    case = gc.load(name)
    net, data, layers, _ = load_case(engine, case)
    cost = make_cost(engine, case, net, data, layers)
    events = engine.train(train_body(net, [cost], 4, optimizer))
    assert events[-1][0] == 0
    _, state = engine.state(net)
    for i, layer in enumerate(state):
        np.testing.assert_allclose(layer['buffers'][0], case[f'{optimizer}_w{i}'], rtol=0, atol=2e-5)


def test_chunking_is_invisible(engine):
    case = gc.load('fourier_order4')
    net, data, layers, _ = load_case(engine, case)
    full = engine.download(engine.evaluate(net, data))
    for chunk in (1, 3, 17, 48, 49, 1000):
        np.testing.assert_array_equal(engine.download(engine.evaluate(net, data, chunk=chunk)), full)


def test_generic_and_automatic_tiers_agree(engine):
    case = gc.load('fourier_order6')
    net, data, layers, _ = load_case(engine, case)
    cost = make_cost(engine, case, net, data, layers)
    auto = engine.graph_evaluate(net, [cost], sum_graph(1))
    engine.set_tier(1)
    try:
        generic = engine.graph_evaluate(net, [cost], sum_graph(1))
    finally:
        engine.set_tier(0)
    assert abs(auto[0] - generic[0]) <= 1e-5 * abs(generic[0])
    assert gc.layer_error(auto[1], generic[1]) < 1e-5


def test_server_drop_in_matches_golden():
    """bin/cpde_server answers the reference's requests with the same results."""
    case = gc.load('fourier_order3')
    with Session(native.SERVER) as s:
        assert s.protocol == 'CPDE/3' and s.capabilities & 31 == 31
        layers = [int(x) for x in case['layers']]
        net = Network(s, layers, weights=gc.weights_of(case))
        inp = Data(s, case['inputs'], case['table'])
        out = net.eval(inp, chunk=5).to_numpy()
        assert gc.rowwise_error(out, case['outputs']).max() < 1e-5
        tgt = Data(s, case['targets'], case['table'])
        cost = net.matching(inp, tgt, case['match_weights'])
        value, grads = net.evaluate([cost], gradient=True)
        assert abs(value - case['loss']) <= 1e-5 * abs(case['loss'])
        assert gc.layer_error(grads, gc.weights_of(case, 'g')) < 1e-5
        wall, device, loss, g90 = net.benchmark(cost, 1, 2, 1)
        assert abs(loss - case['loss']) <= 1e-5 * abs(case['loss']) and device[0] > 0
        result = net.train([cost], 4, optimizer='rprop', reset=True, log_every=1)
        assert result['completed'] == 4 and result['metadata']['updates'] == 4
        for i, w in enumerate(net.weights()):
            np.testing.assert_allclose(w, case[f'rprop_w{i}'], rtol=0, atol=2e-5)
