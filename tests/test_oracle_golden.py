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
