"""C ABI library and host logic, without a GPU."""
import re
from pathlib import Path

import numpy as np
import pytest

from cpde_b200 import native
from cpde_b200.expressions import all_mixed, pure, table
from oracle import jets

HEADER = Path(__file__).resolve().parents[1] / 'include' / 'cpde_b200.h'


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r'^\s*(?:int|void|const char\*)\s+(cpde_\w+)\(', text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = native.load()
    names = declared()
    assert len(names) >= 25
    for name in names:
        assert hasattr(lib, name), name
        assert name in native.SIGNATURES, name


def evaluate_plan(packed, R, z, kind):
    """Run the packed Leibniz tables in float64 (the CUDA kernels' recurrence)."""
    fwd = packed[:R + 1]
    sq = packed[R + 1:2 * (R + 1)]
    adj = packed[2 * (R + 1):3 * (R + 1)]
    coef = lambda i: np.int32(packed[i]).view(np.float32).item()
    y = np.zeros_like(z)
    s = np.zeros_like(z)
    if kind == 'sigmoid':
        y[0] = 1 / (1 + np.exp(-z[0]))
        s[0] = y[0] * (1 - y[0])
        lead = 1 - 2 * y[0]
    else:
        y[0] = np.tanh(z[0])
        s[0] = 1 - y[0] ** 2
        lead = -2 * y[0]
    for r in range(1, R):
        for t in range(fwd[r], fwd[r + 1], 3):
            y[r] += coef(t) * s[packed[t + 1]] * z[packed[t + 2]]
        s[r] = lead * y[r]
        for t in range(sq[r], sq[r + 1], 3):
            s[r] -= coef(t) * y[packed[t + 1]] * y[packed[t + 2]]
    return y, s, adj, coef


@pytest.mark.parametrize('kind', ['sigmoid', 'tanh'])
@pytest.mark.parametrize('schema', [all_mixed(6, 'xy'), all_mixed(4, 'xyz'), pure(6, 'wxyz'), pure(2, 'xy'),
                                    table(['xxxxxx'], 'x'), table(['xyzabc'], 'xyzabc'), all_mixed(0, 'xy')],
                         ids=['2d-o6', '3d-o4', '4d-pure6', '2d-pure2', '1d-o6', '6d-mixed', 'value'])
def test_leibniz_tables_match_set_partition_jets(schema, kind):
    counts = schema[:, 1:]
    R = len(counts)
    packed = native.jet_plan(counts)
    rng = np.random.default_rng(R)
    z = rng.normal(size=(R, 50)) * 0.7
    sch = jets.Schema(counts)
    expected = jets.jet_forward(sch, z, kind)
    y, s, adj, coef = evaluate_plan(packed, R, z, kind)
    np.testing.assert_allclose(y, expected, rtol=1e-10, atol=1e-12)
    dy = rng.normal(size=z.shape)
    dz = np.zeros_like(z)
    for t in range(R):
        for i in range(adj[t], adj[t + 1], 3):
            dz[t] += coef(i) * s[packed[i + 1]] * dy[packed[i + 2]]
    np.testing.assert_allclose(dz, jets.jet_adjoint(sch, z, dy, kind), rtol=1e-9, atol=1e-11)


def test_jet_plan_rejects_unclosed_and_unsorted_schemas():
    with pytest.raises(ValueError):
        native.jet_plan([[0, 0], [2, 0]])  # missing (1, 0)
    with pytest.raises(ValueError):
        native.jet_plan([[1, 0], [0, 0]])  # value row not first
