"""Generate the golden fixtures in this folder by running the reference server.

The reference cPDE server is built from its own sources by ``make -C oracle``
(oracle/_ref/cpde_ref_cpu_server). This script drives it through
cpde_b200.client on small seeded cases and stores, per case, the inputs, the
evaluated output jets (op 4), the objective and weight gradients (op 14) and
short RPROP/Adam trajectories (op 8). The fixtures pin oracle/jets.py
(tests/test_oracle_golden.py) and the CUDA engine (tests/test_gpu_parity.py)
without needing the reference at test time.

    python tests/golden/make_golden.py [path/to/cpde_ref_cpu_server] [--only-tanh]
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from cpde_b200.client import Data, Network, Session  # noqa: E402
from cpde_b200.expressions import (Expression, Polynomial, all_mixed, glorot_like,  # noqa: E402
                                   pure, quadrature_inputs, table)

OUT = Path(__file__).resolve().parent


def points_in(rng, count, dims, low=0.0, high=1.0):
    return rng.uniform(low, high, (count, dims))


def fourier_targets(pts, t):
    """sin(pi x) cos(pi y) and its derivatives (2D) - the config-1 target."""
    out = np.zeros((len(t), 1, len(pts)), np.float32)
    for i, (_, a, b) in enumerate(t):
        out[i, 0] = (np.pi ** (a + b) * np.sin(np.pi * pts[:, 0] + a * np.pi / 2)
                     * np.cos(np.pi * pts[:, 1] + b * np.pi / 2))
    return out


def random_weights(rng, layers, scale=0.6):
    return [rng.uniform(-scale, scale, h * (w + 1)).astype(np.float32) for w, h in zip(layers[:-1], layers[1:])]


def run_matching(s, name, t, pts, layers, weights, rng, linear=None, chunk=0, epochs=4):
    x = quadrature_inputs(pts, t)
    outputs = layers[-1]
    net = Network(s, layers, weights=weights, linear=linear)
    inp = Data(s, x, t)
    y = net.eval(inp).to_numpy()
    if outputs == 1 and t.shape[1] == 3:
        targets = fourier_targets(pts, t)
    else:
        targets = (rng.normal(size=y.shape) * 0.1 + y).astype(np.float32)
    tgt = Data(s, targets, t)
    mw = rng.uniform(0.5, 1.5, (outputs, len(t))).astype(np.float32)
    cost = net.matching(inp, tgt, mw, chunk=chunk)
    value, grads = net.evaluate([cost], gradient=True)
    record = dict(table=t, points=pts, inputs=x, layers=np.array(layers), linear=np.array(net.linear),
                  targets=targets, match_weights=mw, outputs=y, loss=np.float64(value))
    for i, w in enumerate(weights):
        record[f'w{i}'] = w
    for i, g in enumerate(grads):
        record[f'g{i}'] = g
    # short training trajectories from the same start, both optimizers
    for opt in ('rprop', 'adam'):
        net.set_weights(weights)
        net.train([cost], epochs, optimizer=opt, reset=True, log_every=1)
        meta, state = net.state()
        for i, layer in enumerate(state):
            record[f'{opt}_w{i}'] = layer['buffers'][0]
            record[f'{opt}_s{i}'] = layer['buffers'][3]
    np.savez_compressed(OUT / f'{name}.npz', **record)
    print(name, 'rows', len(t), 'loss', value)


def run_polynomial(s, name, rng):
    """Config-5 style: 4D pure derivatives through order 6, weighted linear
    combination of the sixth-order pure derivatives, per-point weights."""
    variables = 'wxyz'
    t = pure(6, variables)
    pts = points_in(rng, 24, 4, -1, 1)
    layers = [4, 12, 12, 1]
    weights = random_weights(rng, layers, 0.5)
    net = Network(s, layers, weights=weights)
    x = quadrature_inputs(pts, t)
    inp = Data(s, x, t)
    y = net.eval(inp).to_numpy()
    parser = Polynomial(table=t, variables=variables, outputs='u', count=len(pts))
    poly = parser.parse('+'.join(f'u_{v * 6}' for v in variables))
    pw = rng.uniform(0, 1, (1, len(pts))).astype(np.float32)
    cost = net.polynomial(inp, [poly], weights=pw)
    value, grads = net.evaluate([cost], gradient=True)
    terms = sorted(poly)
    record = dict(table=t, points=pts, inputs=x, layers=np.array(layers), linear=np.array(net.linear),
                  outputs=y, loss=np.float64(value), poly_weights=pw,
                  poly_components=np.array([k[0] for k in terms]))
    for i, w in enumerate(weights):
        record[f'w{i}'] = w
    for i, g in enumerate(grads):
        record[f'g{i}'] = g
    np.savez_compressed(OUT / f'{name}.npz', **record)
    print(name, 'rows', len(t), 'loss', value)


def run_integral(s, name, rng):
    """Config-3 style: (u_xx+u_yy+1)**2 on disk points with weight pi/N."""
    t = table(['xx', 'yy'], 'xy')
    n = 40
    r = np.sqrt(rng.uniform(0, 1, n))
    th = 2 * np.pi * rng.uniform(0, 1, n)
    pts = np.column_stack([r * np.cos(th), r * np.sin(th)])
    layers = [2, 10, 10, 10, 1]
    weights = random_weights(rng, layers, 0.7)
    net = Network(s, layers, weights=weights)
    x = quadrature_inputs(pts, t)
    inp = Data(s, x, t)
    y = net.eval(inp).to_numpy()
    expr = Expression('(u_xx+u_yy+1)**2', table=t, variables='xy', outputs='u', count=n)
    qw = np.full(n, np.pi / n)
    cost = net.integral(inp, expr, weights=qw, chunk=16)
    value, grads = net.evaluate([cost], gradient=True)
    record = dict(table=t, points=pts, inputs=x, layers=np.array(layers), linear=np.array(net.linear),
                  outputs=y, loss=np.float64(value), quad_weights=qw,
                  nodes=np.array(expr.nodes, np.int32), constants=np.array(expr.constants))
    for i, w in enumerate(weights):
        record[f'w{i}'] = w
    for i, g in enumerate(grads):
        record[f'g{i}'] = g
    np.savez_compressed(OUT / f'{name}.npz', **record)
    print(name, 'rows', len(t), 'loss', value)


def run_tanh(s, name, rng, t, pts, layers, expression=None, chunk=0):
    """A network with tanh hidden layers. The reference server has no tanh
    (cuda/cpde_server.cu:457), so it evaluates the exact reparametrisation
    tanh(z) = 2 sigma(2z) - 1 (cpde_b200.expressions.tanh_as_sigmoid): same
    outputs and derivative rows; its weight gradients are mapped back through
    the transpose of that linear map. Matching cost, or an integral cost when
    `expression` is given. No optimizer trajectories: RPROP and Adam do not
    commute with the reparametrisation."""
    from cpde_b200.expressions import sigmoid_gradients_to_tanh, tanh_as_sigmoid
    linear = [1] + [2] * (len(layers) - 2) + [1]
    weights = random_weights(rng, layers, 0.6)
    sig_linear, sig_weights = tanh_as_sigmoid(layers, linear, weights)
    net = Network(s, layers, weights=sig_weights, linear=sig_linear)
    x = quadrature_inputs(pts, t)
    inp = Data(s, x, t)
    y = net.eval(inp).to_numpy()
    record = dict(table=t, points=pts, inputs=x, layers=np.array(layers), linear=np.array(linear), outputs=y)
    if expression is None:
        targets = (rng.normal(size=y.shape) * 0.1 + y).astype(np.float32)
        mw = rng.uniform(0.5, 1.5, (layers[-1], len(t))).astype(np.float32)
        cost = net.matching(inp, Data(s, targets, t), mw, chunk=chunk)
        record.update(targets=targets, match_weights=mw)
    else:
        expr = Expression(expression, table=t, variables='xyz'[:t.shape[1] - 1], outputs='u', count=len(pts))
        qw = np.full(len(pts), 1.0 / len(pts))
        cost = net.integral(inp, expr, weights=qw, chunk=chunk)
        record.update(quad_weights=qw, nodes=np.array(expr.nodes, np.int32), constants=np.array(expr.constants))
    value, grads = net.evaluate([cost], gradient=True)
    record['loss'] = np.float64(value)
    for i, w in enumerate(weights):
        record[f'w{i}'] = w
    for i, g in enumerate(sigmoid_gradients_to_tanh(layers, linear, grads)):
        record[f'g{i}'] = g
    np.savez_compressed(OUT / f'{name}.npz', **record)
    print(name, 'rows', len(t), 'loss', value)


def tanh_cases(s):
    rng = np.random.default_rng(20261202)
    run_tanh(s, 'tanh_mixed2d_order4', rng, all_mixed(4, 'xy'), points_in(rng, 17, 2, -1, 1), [2, 12, 10, 2],
             chunk=6)
    run_tanh(s, 'tanh_biharmonic3d', rng, all_mixed(4, 'xyz'), points_in(rng, 11, 3), [3, 10, 8, 1],
             expression='(u_xxxx+u_yyyy+u_zzzz+2*u_xxyy+2*u_xxzz+2*u_yyzz-1)**2', chunk=4)


def main(exe, only=None):
    if only == 'tanh':
        with Session(exe) as s:
            tanh_cases(s)
        return
    rng = np.random.default_rng(20261201)
    with Session(exe) as s:
        grid = np.linspace(0, 1, 7)
        gx, gy = np.meshgrid(grid, grid, indexing='ij')
        grid_pts = np.column_stack([gx.ravel(), gy.ravel()])
        for order in range(7):
            layers = [2, 16, 16, 16, 1]
            run_matching(s, f'fourier_order{order}', all_mixed(order, 'xy'), grid_pts, layers,
                         glorot_like(layers, seed=order), rng)
        run_matching(s, 'chunked_multioutput', all_mixed(2, 'xy'), points_in(rng, 23, 2), [2, 9, 7, 3],
                     random_weights(rng, [2, 9, 7, 3]), rng, chunk=5)
        run_matching(s, 'linear_hidden', all_mixed(3, 'xy'), points_in(rng, 11, 2), [2, 6, 5, 4, 1],
                     random_weights(rng, [2, 6, 5, 4, 1]), rng, linear=[1, 0, 1, 0, 1])
        run_matching(s, 'mixed3d_order4', all_mixed(4, 'xyz'), points_in(rng, 9, 3), [3, 8, 8, 1],
                     random_weights(rng, [3, 8, 8, 1], 0.5), rng)
        run_matching(s, 'one_direction_order6', table(['xxxxxx'], 'x'), points_in(rng, 13, 1, -1, 1),
                     [1, 5, 4, 1], random_weights(rng, [1, 5, 4, 1]), rng)
        run_matching(s, 'six_variables_mixed', table(['xyzabc'], 'xyzabc'), points_in(rng, 5, 6, -.2, .2),
                     [6, 4, 3, 1], random_weights(rng, [6, 4, 3, 1], 0.6), rng)
        run_polynomial(s, 'pure4d_order6_polynomial', rng)
        run_integral(s, 'disk_poisson_integral', rng)
        tanh_cases(s)


if __name__ == '__main__':
    args = [a for a in sys.argv[1:] if not a.startswith('--')]
    main(args[0] if args else ROOT / 'oracle' / '_ref' / 'cpde_ref_cpu_server',
         only='tanh' if '--only-tanh' in sys.argv else None)
