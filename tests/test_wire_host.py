"""Wire encodings and host-side cost builders (no GPU)."""
import numpy as np

from cpde_b200.client import sum_graph
from cpde_b200.expressions import Expression, Polynomial, all_mixed, closure, pure, quadrature_inputs, table
from cpde_b200.wire import Reader, decode_state, encode_state


def test_state_blob_round_trip():
    meta = dict(neurons=[2, 3, 1], linear=[1, 0, 1], optimizer='rprop', updates=5, adam_step=0,
                stage_completed=2, remaining=7, learning_rate=np.float32(0.001), initial_step=np.float32(0.002),
                stage='abc|def')
    rng = np.random.default_rng(0)
    layers = [dict(active=a, buffers=[rng.normal(size=n).astype(np.float32) for _ in range(4)])
              for a, n in ((1, 9), (2, 4))]
    m2, l2 = decode_state(encode_state(meta, layers))
    assert m2['stage'] == 'abc|def' and m2['updates'] == 5 and m2['optimizer'] == 'rprop'
    for a, b in zip(layers, l2):
        assert a['active'] == b['active']
        for x, y in zip(a['buffers'], b['buffers']):
            np.testing.assert_array_equal(x, y)


def test_tables_closures_and_row_counts():
    assert [len(all_mixed(k, 'xy')) for k in range(7)] == [1, 3, 6, 10, 15, 21, 28]
    assert len(all_mixed(4, 'xyz')) == 35 and len(pure(6, 'wxyz')) == 25 and len(table(['xx', 'yy'], 'xy')) == 5
    t = all_mixed(3, 'xy')
    rows = closure(t, [len(t) - 1])  # rows sort by (order, counts): the last is x^3
    assert [tuple(int(v) for v in t[r, 1:]) for r in rows] == [(0, 0), (1, 0), (2, 0), (3, 0)]


def test_sum_graph_layout():
    r = Reader(sum_graph(3))
    nodes = r.array('i4').reshape(-1, 3)
    assert nodes[:3, 0].tolist() == [1, 1, 1] and nodes[-1].tolist() == [3, 3, 2]


def test_expression_and_polynomial_builders():
    t = table(['xx', 'yy'], 'xy')
    e = Expression('(u_xx+u_yy+1)**2', table=t, variables='xy', outputs='u', count=4)
    ops = [n[0] for n in e.nodes]
    assert ops == [1, 1, 3, 0, 3, 7] and e.constants[-1] == 2
    p = Polynomial(table=t, variables='xy', outputs='u', count=4).parse('u_xx+u_yy')
    assert sorted(p) == [(3,), (4,)] or len(p) == 2
    x = quadrature_inputs(np.array([[.1, .2], [.3, .4]]), t)
    assert x.shape == (5, 2, 2) and x[1].sum() == 2 and x[3].sum() == 0
