"""The float64 oracle reproduces the reference server's own results (CPU)."""
import numpy as np
import pytest

import golden_cases as gc


@pytest.mark.parametrize('name', gc.names())
def test_output_jets_match_reference(name):
    case = gc.load(name)
    _, _, _, _, acts = gc.oracle_outputs(case)
    err = gc.rowwise_error(case['outputs'], acts[-1])
    assert err.max() < gc.tolerance(case['table']), err


@pytest.mark.parametrize('name', gc.names())
def test_objective_and_gradients_match_reference(name):
    case = gc.load(name)
    loss, grads, _ = gc.oracle_gradients(case)
    assert abs(case['loss'] - loss) <= 1e-5 * abs(loss) + 1e-12
    assert gc.layer_error(gc.weights_of(case, 'g'), grads) < gc.tolerance(case['table'])


@pytest.mark.parametrize('name', [n for n in gc.names() if n.startswith('fourier') or n in (
    'chunked_multioutput', 'linear_hidden', 'mixed3d_order4')])
@pytest.mark.parametrize('optimizer', ['rprop', 'adam'])
def test_optimizer_trajectories_match_reference(name, optimizer):
    case = gc.load(name)
    weights, aux = gc.oracle_training(case, optimizer)
    for i, (w, a) in enumerate(zip(weights, aux)):
        np.testing.assert_allclose(w, case[f'{optimizer}_w{i}'], rtol=0, atol=2e-5)
        np.testing.assert_allclose(a, case[f'{optimizer}_s{i}'], rtol=1e-3, atol=1e-6)


BLAS_SERVER = gc.GOLDEN.parents[1] / 'oracle' / '_ref' / 'cpde_ref_cpu_server_blas'


@pytest.mark.skipif(not BLAS_SERVER.exists(), reason='BLAS-linked reference CPU server not built')
@pytest.mark.parametrize('name', ['fourier_order3', 'chunked_multioutput', 'mixed3d_order4'])
def test_blas_reference_server_matches_golden(name):
    """The CPU baseline's server (the reference built with its CBLAS option
    against numpy's OpenBLAS) gives the golden fixtures' objective and weight
    gradients, which the portable serial build of the same sources wrote:
    both are the reference."""
    from cpde_b200.client import Data, Network, Session
    case = gc.load(name)
    layers = [int(v) for v in case['layers']]
    t = case['table']
    with Session(BLAS_SERVER) as s:
        net = Network(s, layers, weights=gc.weights_of(case), linear=[int(v) for v in case['linear']])
        inp = Data(s, case['inputs'], t)
        tgt = Data(s, case['targets'], t)
        cost = net.matching(inp, tgt, case['match_weights'])
        value, grads = net.evaluate([cost], gradient=True)
    assert abs(value - float(case['loss'])) <= 1e-5 * abs(float(case['loss']))
    assert gc.layer_error(grads, gc.weights_of(case, 'g')) < gc.tolerance(t)
