"""TEST INFRASTRUCTURE ONLY: CPU restatement of the reference cPDE hot path.

This module is the checker for the CUDA engine. Only ``tests/``, the
``smoke()`` entry point and ``bench.py``'s CPU-baseline leg may import it; the
engine never does. Everything is float64 NumPy, vectorised over
(neuron, point) and organised like the reference algorithm, with the reference
file:line each function restates:

* derivative rows and the per-row subset stacks (cuda/cpde_engine.cuh:213-340,
  391-469): every row S is a multiset of k directions; its 2^k position subsets
  are ordered by size then lexicographically and resolved to rows;
* the forward sigmoid jet (cuda/derivative_kernels_v4.cu:382-745): y_S is the
  sum over set partitions of the k positions of sigma^(|partition|)(z) times
  the product of the z rows of the blocks (Faa di Bruno), with tanh added the
  same way (tanh does not exist in the reference; its jet uses the same
  partition sum with tanh's derivatives);
* the backward jet adjoint (cuda/derivative_kernels_v4.cu:339-380): rows
  ascending, dE/dZ_i = sum_{S_j >= S_i} C(S_j,S_i) * D^{S_j-S_i}[sigma'(z)] *
  dE/dY_j, where the D term is the same partition sum with sigma shifted by one
  order;
* the per-layer linear maps, bias on the value row only, and the weight
  gradients of network::feedforward/backprop (cuda/cpde_engine.cuh:889-991);
* matching and polynomial costs (cuda/cost_kernels.cuh:6-90), the scalar
  expression IR and cost graph (cuda/expression_program.hpp:31-93,
  cuda/cost_graph.cuh:6-27, cuda/scalar_ops.cuh:4-27);
* RPROP and Adam (cuda/derivative_kernels_v4.cu:752-832), in float32 like the
  reference.

Parity pin: tests/test_oracle_golden.py checks this module against outputs of
the reference server built from its own sources (oracle/Makefile) that are
committed under tests/golden/.
"""
import itertools
import math
from functools import lru_cache

import numpy as np

# ---------------------------------------------------------------------------
# activation derivatives


@lru_cache(maxsize=None)
def _sigmoid_polynomials(n):
    """Coefficients of sigma^(k) as polynomials in s=sigma, k = 0..n.

    d/dz P(s) = P'(s) * s * (1 - s)."""
    polys = [np.array([0.0, 1.0])]  # s
    for _ in range(n):
        p = polys[-1]
        dp = np.polynomial.polynomial.polyder(p) if len(p) > 1 else np.array([0.0])
        polys.append(np.polynomial.polynomial.polymul(dp, [0.0, 1.0, -1.0]))
    return polys


@lru_cache(maxsize=None)
def _tanh_polynomials(n):
    """tanh^(k) as polynomials in t=tanh: d/dz P(t) = P'(t) * (1 - t^2)."""
    polys = [np.array([0.0, 1.0])]
    for _ in range(n):
        p = polys[-1]
        dp = np.polynomial.polynomial.polyder(p) if len(p) > 1 else np.array([0.0])
        polys.append(np.polynomial.polynomial.polymul(dp, [1.0, 0.0, -1.0]))
    return polys


def activation_derivatives(z, n, kind):
    """[f(z), f'(z), ..., f^(n)(z)] for kind 'sigmoid' or 'tanh'."""
    if kind == 'sigmoid':
        base = 0.5 * (1.0 + np.tanh(0.5 * z))  # overflow-free logistic
        polys = _sigmoid_polynomials(n)
    else:
        base = np.tanh(z)
        polys = _tanh_polynomials(n)
    return [np.polynomial.polynomial.polyval(base, p) for p in polys]


# ---------------------------------------------------------------------------
# schema tables


def directions(counts):
    """Multiset of variable indices of one row (cuda/cpde_engine.cuh:425-429)."""
    out = []
    for v, c in enumerate(counts):
        out.extend([v] * int(c))
    return out


@lru_cache(maxsize=None)
def set_partitions(k):
    """All set partitions of range(k), each a tuple of blocks (tuples)."""
    if k == 0:
        return ((),)
    out = []
    for part in set_partitions(k - 1):
        # put element k-1 into an existing block or a new one
        for i in range(len(part)):
            blocks = list(part)
            blocks[i] = blocks[i] + (k - 1,)
            out.append(tuple(blocks))
        out.append(part + ((k - 1,),))
    return tuple(out)


def subset_row(counts, positions, index):
    """Row index of the sub-multi-index made of the chosen positions
    (cuda/cpde_engine.cuh:313-340 resolve)."""
    dirs = directions(counts)
    sub = [0] * len(counts)
    for p in positions:
        sub[dirs[p]] += 1
    return index[tuple(sub)]


class Schema:
    """Rows of one derivative context: list of count tuples, value row first,
    orders non-decreasing (cuda/cpde_server.cu:113-123)."""

    def __init__(self, counts):
        self.counts = [tuple(int(x) for x in c) for c in counts]
        self.index = {c: i for i, c in enumerate(self.counts)}
        if self.counts[0] != (0,) * len(self.counts[0]):
            raise ValueError('value row must come first')
        orders = [sum(c) for c in self.counts]
        if orders != sorted(orders) or max(orders) > 6:
            raise ValueError('rows must be sorted by order, orders 0..6')
        self.orders = orders
        # partition terms per row: list of (number of blocks, [row of each block])
        self.terms = []
        for c in self.counts:
            k = sum(c)
            terms = []
            for part in set_partitions(k):
                terms.append((len(part), [subset_row(c, b, self.index) for b in part]))
            self.terms.append(terms)
        # difference table and coefficients (cuda/cpde_engine.cuh:476-498)
        self.pairs = []  # (i, j, row of S_j - S_i, C(S_j, S_i))
        for i, a in enumerate(self.counts):
            for j, b in enumerate(self.counts):
                if j <= i or any(x > y for x, y in zip(a, b)):
                    continue
                diff = tuple(y - x for x, y in zip(a, b))
                coef = math.prod(math.comb(y, x) for x, y in zip(a, b))
                self.pairs.append((i, j, self.index[diff], coef))

    @property
    def rows(self):
        return len(self.counts)


def jet_forward(schema, z, kind):
    """y[r] = d^{S_r} f(z) by the set-partition sum; z has shape (R, ...)."""
    n = max(schema.orders)
    f = activation_derivatives(z[0], n, kind)
    y = np.empty_like(z)
    y[0] = f[0]
    for r in range(1, schema.rows):
        acc = 0.0
        for blocks, members in schema.terms[r]:
            prod = f[blocks]
            for m in members:
                prod = prod * z[m]
            acc = acc + prod
        y[r] = acc
    return y


def shifted_jet(schema, z, f, row):
    """D^{S_row}[f'(z)] by the partition sum with derivatives shifted by one
    (cuda/derivative_kernels_v4.cu:12-347 d1p..d6p)."""
    if row == 0:
        return f[1]
    acc = 0.0
    for blocks, members in schema.terms[row]:
        prod = f[blocks + 1]
        for m in members:
            prod = prod * z[m]
        acc = acc + prod
    return acc


def jet_adjoint(schema, z, dy, kind):
    """dE/dZ from dE/dY through the jet map (back_step,
    cuda/derivative_kernels_v4.cu:349-380)."""
    n = max(schema.orders) + 1
    f = activation_derivatives(z[0], n, kind)
    d = [shifted_jet(schema, z, f, r) for r in range(schema.rows)]
    dz = dy * d[0]
    for i, j, diff, coef in schema.pairs:
        dz[i] = dz[i] + coef * d[diff] * dy[j]
    return dz


# ---------------------------------------------------------------------------
# network


def split_layer(flat, width, height):
    """Column-major W (height x width) then bias (tests/network_reference.py:18-19)."""
    flat = np.asarray(flat, np.float64)
    return flat[:width * height].reshape((height, width), order='F'), flat[width * height:]


ACTIVATIONS = {0: 'sigmoid', 2: 'tanh'}


def forward(schema, weights, layers, linear, x, activation='sigmoid'):
    """Jets of every layer. ``x`` has shape (R, n0, P). Returns the list of
    pre-activations Z_l (l >= 1) and post-activation jets A_l (A_0 = x).
    Layer flags: 1 linear, 0 sigmoid, 2 tanh (tanh is an extension: the
    reference knows only 0 and 1, cuda/cpde_server.cu:457)."""
    acts = [np.asarray(x, np.float64)]
    pre = [None]
    for l in range(1, len(layers)):
        w, b = split_layer(weights[l - 1], layers[l - 1], layers[l])
        z = np.einsum('mk,rkp->rmp', w, acts[-1])
        z[0] += b[:, None]
        pre.append(z)
        if linear[l] == 1:
            acts.append(z)
        else:
            acts.append(jet_forward(schema, z, ACTIVATIONS.get(linear[l], activation)))
    return pre, acts


def backward(schema, weights, layers, linear, pre, acts, dout, activation='sigmoid'):
    """Weight gradients (flat, like the weights) from dE/dZ of the output layer."""
    grads = [None] * (len(layers) - 1)
    dz = np.asarray(dout, np.float64)
    for l in range(len(layers) - 1, 0, -1):
        w, _ = split_layer(weights[l - 1], layers[l - 1], layers[l])
        gw = np.einsum('rmp,rkp->mk', dz, acts[l - 1])
        gb = dz[0].sum(axis=1)
        grads[l - 1] = np.concatenate([gw.ravel(order='F'), gb])
        if l == 1:
            break
        dy = np.einsum('mk,rmp->rkp', w, dz)
        dz = dy if linear[l - 1] == 1 else jet_adjoint(schema, pre[l - 1], dy,
                                                        ACTIVATIONS.get(linear[l - 1], activation))
    return grads


# ---------------------------------------------------------------------------
# costs


def matching(y, target, weights):
    """Kind-0 cost (cuda/cost_kernels.cuh:6-35): y, target (R, outputs, P),
    weights broadcastable to it. Returns (loss, dE/dy)."""
    r = y - target
    w = np.broadcast_to(weights, y.shape)
    return float(np.sum(w * r * r)), 2.0 * w * r


def polynomial(y, terms, coefficients, rhs, weights):
    """Kind-1 cost (cuda/cost_kernels.cuh:37-90); ``y`` (R, outputs, P), terms
    (eq, a, b) over component index row*outputs+output, coefficients (T, P),
    rhs and weights (E, P)."""
    R, outputs, P = y.shape
    flat = np.asarray(y, np.float64).reshape(R * outputs, P)
    g = np.zeros_like(flat)
    loss = 0.0
    for e in range(rhs.shape[0]):
        res = -np.asarray(rhs[e], np.float64).copy()
        mine = [(t, c) for t, c in zip(terms, coefficients) if t[0] == e]
        for (eq, a, b), c in mine:
            res += c * flat[a] * (1.0 if b < 0 else flat[b])
        w = np.asarray(weights[e], np.float64)
        loss += float(np.sum(w * res * res))
        scale = 2.0 * w * res
        for (eq, a, b), c in mine:
            if b < 0:
                g[a] += scale * c
            else:
                g[a] += scale * c * flat[b]
                g[b] += scale * c * flat[a]
    return loss, g.reshape(R, outputs, P)


def scalar_value(op, a, b, p):
    """cuda/scalar_ops.cuh:6-16."""
    with np.errstate(all='ignore'):
        if op == 0:
            return np.full_like(np.asarray(a, np.float64), p)
        if op == 3:
            return a + b
        if op == 4:
            return a - b
        if op == 5:
            return a * b
        if op == 6:
            return np.where(b == 0, np.nan, a / np.where(b == 0, 1, b))
        if op == 7:
            bad = ((a < 0) & (math.floor(p) != p)) | ((a == 0) & (p < 0))
            return np.where(bad, np.nan, np.power(np.where(bad, 1.0, a), p))
        if op == 8:
            return -a
        if op == 9:
            return np.exp(a)
        if op == 10:
            return np.where(a > 0, np.log(np.where(a > 0, a, 1.0)), np.nan)
        if op == 11:
            return np.where(a >= 0, np.sqrt(np.abs(a)), np.nan)
        if op == 12:
            return np.sin(a)
        if op == 13:
            return np.cos(a)
        if op == 14:
            return np.tanh(a)
        if op == 15:
            return a
    raise ValueError(op)


def scalar_partials(op, a, b, v, p):
    """cuda/scalar_ops.cuh:17-26."""
    one = np.ones_like(np.asarray(v, np.float64))
    zero = np.zeros_like(one)
    with np.errstate(all='ignore'):
        if op in (3, 15):
            return one, one
        if op == 4:
            return one, -one
        if op == 5:
            return b * one, a * one
        if op == 6:
            return 1 / b, -v / b
        if op == 7:
            return (zero if p == 0 else one if p == 1 else p * np.power(a, p - 1)), zero
        if op == 8:
            return -one, zero
        if op == 9:
            return v, zero
        if op == 10:
            return 1 / a, zero
        if op == 11:
            return 0.5 / v, zero
        if op == 12:
            return np.cos(a), zero
        if op == 13:
            return -np.sin(a), zero
        if op == 14:
            return 1 - v * v, zero
    return zero, zero


def expression(y, nodes, constants, fields, weights):
    """Kind-2 integral (cuda/expression_program.hpp:71-93 semantics, float64):
    returns (sum of weights*value, dE/dy) for y of shape (R, outputs, P);
    ``nodes`` component indices are already mapped to this y's rows."""
    R, outputs, P = y.shape
    vals = []
    active = []
    for i, (op, a, b) in enumerate(nodes):
        if op == 1:
            vals.append(np.asarray(y[a // outputs, a % outputs], np.float64))
            active.append(b == 0)
        elif op == 2:
            vals.append(np.asarray(fields[a], np.float64))
            active.append(False)
        elif op == 0:
            vals.append(np.full(P, constants[i]))
            active.append(False)
        else:
            binary = op <= 6
            vals.append(scalar_value(op, vals[a], vals[b] if binary else 0.0, constants[i]))
            active.append(active[a] or (binary and active[b]))
    w = np.asarray(weights, np.float64)
    loss = float(np.sum(w * vals[-1]))
    adj = [np.zeros(P) for _ in nodes]
    adj[-1] = np.ones(P)
    for i in range(len(nodes) - 1, -1, -1):
        op, a, b = nodes[i]
        if op <= 2 or not active[i]:
            continue
        da, db = scalar_partials(op, vals[a], vals[b] if op <= 6 else 0.0, vals[i], constants[i])
        if active[a]:
            adj[a] = adj[a] + adj[i] * da
        if op <= 6 and active[b]:
            adj[b] = adj[b] + adj[i] * db
    g = np.zeros((R * outputs, P))
    for i, (op, a, b) in enumerate(nodes):
        if op == 1 and b == 0:
            g[a] += adj[i]
    g *= w
    return loss, g.reshape(R, outputs, P)


# ---------------------------------------------------------------------------
# optimizers (float32 like the reference kernels)


def rprop(w, steps, current, previous):
    """One Resile_k update (cuda/derivative_kernels_v4.cu:752-778); arrays are
    float32 and modified in place. The caller swaps current/previous after."""
    f32 = np.float32
    prod = current * previous
    grow = prod > 0
    steps[grow] = steps[grow] * f32(1.2)
    nw = (w - np.copysign(steps, current)).astype(f32)
    back = prod < 0
    w[back] = w[back] + np.copysign(steps[back], previous[back])
    steps[back] = steps[back] * f32(0.5)
    current[back] = 0
    move = (~back) & (current != 0)
    ok = move & (np.abs(nw) <= 20)
    w[ok] = nw[ok]
    rej = move & ~ok
    steps[rej] = f32(0.1)
    current[rej] = 0


def adam(w, grad, m, v, step, lr):
    """ADAM_k (cuda/derivative_kernels_v4.cu:780-799) with the host's float32
    pow(beta, step) (cuda/cpde_engine.cuh:1010)."""
    f32 = np.float32
    b1, b2 = f32(0.9), f32(0.999)
    b1t, b2t = f32(np.float32(0.9) ** np.float32(step)), f32(np.float32(0.999) ** np.float32(step))
    m[:] = b1 * m + (f32(1) - b1) * grad
    v[:] = b2 * v + (f32(1) - b2) * grad * grad
    mh = m / (f32(1) - b1t)
    vh = v / (f32(1) - b2t)
    nw = (w.astype(np.float64) - (f32(lr) * mh).astype(np.float64) / (np.sqrt(vh).astype(np.float64) + 1e-8)).astype(f32)
    ok = np.abs(nw) <= 20
    w[ok] = nw[ok]
