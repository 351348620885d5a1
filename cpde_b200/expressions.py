"""Host-side builders for the cost encodings the server accepts.

These are independent implementations of the encodings the reference's Python
front end produces, so that tests and benchmarks can drive a server without the
reference package:

* derivative tables and closures (cpde/quadrature.py:16-38, cpde/_prepare.py:84-90,
  cpde/_prepare.py:132-138);
* the scalar expression IR of integral costs (cpde/_expressions.py:7-104,
  opcode numbering of cuda/scalar_ops.cuh:4);
* sparse linear/quadratic polynomial residuals (cpde/_prepare.py:160-223).
"""
import ast
import itertools
import math
import re

import numpy as np

CONSTANT, COMPONENT, FIELD, ADD, SUB, MUL, DIV, POWER, NEG, EXP, LOG, SQRT, SIN, COS, TANH, ATTACH = range(16)
FUNCTIONS = dict(exp=EXP, log=LOG, sqrt=SQRT, sin=SIN, cos=COS, tanh=TANH)
MAX_ORDER = 6


def table(derivatives, variables):
    """Derivative table rows ``(order, counts...)`` for the requested suffixes plus
    every lower dependency, sorted by total order then by the count tuple."""
    if not isinstance(variables, str) or not 1 <= len(variables) <= 26 or len(set(variables)) != len(variables):
        raise ValueError('variables must be 1..26 unique letters')
    counts = {(0,) * len(variables)}
    for suffix in derivatives:
        if any(ch not in variables for ch in suffix) or len(suffix) > MAX_ORDER:
            raise ValueError(f'invalid derivative suffix {suffix!r}')
        top = tuple(suffix.count(v) for v in variables)
        counts.update(itertools.product(*(range(c + 1) for c in top)))
    rows = sorted(counts, key=lambda c: (sum(c), c))
    return np.array([(sum(c), *c) for c in rows], dtype=np.int32)


def all_mixed(order, variables):
    """Every pure and mixed derivative through ``order``."""
    suffixes = []
    for k in range(order + 1):
        for combo in itertools.combinations_with_replacement(variables, k):
            suffixes.append(''.join(combo))
    return table(suffixes, variables)


def pure(order, variables):
    """Value plus pure derivatives of each variable through ``order``."""
    return table([v * order for v in variables], variables)


def closure(t, selected):
    """Rows needed to propagate the selected rows: value row, every sub-index of
    each selected row, sorted by (order, original position)."""
    keys = {tuple(int(x) for x in row[1:]): i for i, row in enumerate(t)}
    wanted = {keys[(0,) * (t.shape[1] - 1)]}
    for i in selected:
        for sub in itertools.product(*(range(int(x) + 1) for x in t[i, 1:])):
            wanted.add(keys[sub])
    return sorted(wanted, key=lambda i: (int(t[i, 0]), i))


def component_index(name, t, variables, outputs):
    """``u`` / ``u_xy`` -> row * outputs + output in derivative table ``t``."""
    if not re.fullmatch(r'[A-Za-z](?:_[A-Za-z]+)?', name) or name[0] not in outputs:
        raise ValueError(f'unknown component {name!r}')
    suffix = name[2:] if len(name) > 1 else ''
    if any(ch not in variables for ch in suffix):
        raise ValueError(f'unknown derivative variable in {name!r}')
    counts = tuple(suffix.count(v) for v in variables)
    rows = {tuple(int(x) for x in r[1:]): i for i, r in enumerate(t)}
    if counts not in rows:
        raise ValueError(f'derivative {name!r} not present in the data table')
    return rows[counts] * len(outputs) + outputs.index(name[0])


class Expression:
    """Compile a restricted arithmetic expression into the scalar IR.

    Node ``[op, a, b]`` with a parallel ``constants`` array; children precede
    parents. Components carry the data-table component index in ``a`` and a
    stop-gradient flag in ``b``. Fields are per-sample float64 vectors.
    """

    def __init__(self, text, *, table, variables, outputs, parameters=None, freeze=(), count=None,
                 coordinates=None):
        self.table, self.variables, self.outputs = table, variables, outputs
        self.parameters = dict(parameters or {})
        self.coordinates = coordinates
        self.count = count
        self.nodes, self.constants, self.fields = [], [], []
        self._field_values = []
        self._freeze = {self._canonical(name) for name in freeze}
        tree = ast.parse('(' + text.strip() + '\n)', mode='eval').body
        self._visit(tree)

    def _canonical(self, name):
        suffix = name[2:] if len(name) > 1 else ''
        return name[0] + ('_' + ''.join(v * suffix.count(v) for v in self.variables) if suffix else '')

    def _emit(self, op, a=-1, b=-1, value=0.0):
        if len(self.nodes) >= 512:
            raise ValueError('expression exceeds 512 IR nodes')
        self.nodes.append([op, a, b])
        self.constants.append(float(value))
        return len(self.nodes) - 1

    def _field(self, key, values):
        if key not in self.fields:
            v = np.asarray(values, dtype=np.float64)
            if v.ndim == 0:
                v = np.full(self.count, float(v))
            self.fields.append(key)
            self._field_values.append(v)
        return self._emit(FIELD, self.fields.index(key))

    def _visit(self, node):
        if isinstance(node, ast.Constant) and type(node.value) in (int, float):
            return self._emit(CONSTANT, value=node.value)
        if isinstance(node, ast.Name):
            if node.id in self.parameters:
                return self._field(node.id, self.parameters[node.id])
            canonical = self._canonical(node.id)
            index = component_index(node.id, self.table, self.variables, self.outputs)
            return self._emit(COMPONENT, index, int(canonical in self._freeze))
        if isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name) and node.value.id == 'coord':
            axis = self.variables.index(node.attr)
            return self._field('coord.' + node.attr, self.coordinates[:, axis])
        if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.USub, ast.UAdd)):
            a = self._visit(node.operand)
            return self._emit(NEG, a) if isinstance(node.op, ast.USub) else a
        if isinstance(node, ast.BinOp):
            if isinstance(node.op, ast.Pow):
                exponent = node.right
                sign = 1
                if isinstance(exponent, ast.UnaryOp) and isinstance(exponent.op, ast.USub):
                    sign, exponent = -1, exponent.operand
                return self._emit(POWER, self._visit(node.left), value=sign * exponent.value)
            op = {ast.Add: ADD, ast.Sub: SUB, ast.Mult: MUL, ast.Div: DIV}[type(node.op)]
            return self._emit(op, self._visit(node.left), self._visit(node.right))
        if isinstance(node, ast.Call) and isinstance(node.func, ast.Name) and node.func.id in FUNCTIONS:
            return self._emit(FUNCTIONS[node.func.id], self._visit(node.args[0]))
        raise ValueError('unsupported expression syntax: ' + type(node).__name__)

    def field_array(self):
        if not self._field_values:
            return np.zeros((0, self.count), np.float64)
        return np.stack(self._field_values).astype(np.float64)


class Polynomial:
    """Sparse linear/quadratic monomials in output components with per-sample
    coefficient vectors: ``{(a,) or (a, b): coefficients[samples]}``."""

    def __init__(self, *, table, variables, outputs, count, parameters=None):
        self.table, self.variables, self.outputs, self.count = table, variables, outputs, count
        self.parameters = {k: np.broadcast_to(np.asarray(v, np.float32), (count,)).copy()
                           for k, v in (parameters or {}).items()}

    def parse(self, text):
        poly = self._visit(ast.parse('(' + text.strip() + '\n)', mode='eval').body)
        constant = poly.pop((), None)
        if constant is not None and np.any(constant != 0):
            raise ValueError('constant terms belong in rhs')
        return {k: v.astype(np.float32) for k, v in poly.items() if np.any(v != 0)}

    def _visit(self, node):
        ones = np.ones(self.count, np.float32)
        if isinstance(node, ast.Name):
            if node.id in self.parameters:
                return {(): self.parameters[node.id]}
            return {(component_index(node.id, self.table, self.variables, self.outputs),): ones}
        if isinstance(node, ast.Constant):
            return {(): ones * np.float32(node.value)}
        if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.USub, ast.UAdd)):
            sign = -1 if isinstance(node.op, ast.USub) else 1
            return {k: sign * v for k, v in self._visit(node.operand).items()}
        if isinstance(node, ast.BinOp):
            a = self._visit(node.left)
            if isinstance(node.op, ast.Pow):
                return self._mul(a, a)
            b = self._visit(node.right)
            if isinstance(node.op, ast.Add):
                return self._add(a, b, 1)
            if isinstance(node.op, ast.Sub):
                return self._add(a, b, -1)
            if isinstance(node.op, ast.Mult):
                return self._mul(a, b)
        raise ValueError('supported polynomial operations are +, -, * and **2')

    @staticmethod
    def _add(a, b, sign):
        out = dict(a)
        for k, v in b.items():
            out[k] = out.get(k, 0) + sign * v
        return out

    @staticmethod
    def _mul(a, b):
        out = {}
        for ka, va in a.items():
            for kb, vb in b.items():
                key = tuple(sorted(ka + kb))
                if len(key) > 2:
                    raise ValueError('only linear and quadratic monomials are supported')
                out[key] = out.get(key, 0) + va * vb
        return out


def quadrature_inputs(points, t):
    """Input jets of coordinate data: value row = coordinates, first-order rows =
    unit vectors, higher rows zero (cpde/quadrature.py:155-158).

    Returns an array (derivatives, channels, samples)."""
    points = np.asarray(points, np.float64)
    arrays = np.zeros((len(t), points.shape[1], len(points)), np.float32)
    arrays[0] = points.T
    for i, row in enumerate(t):
        if row[0] == 1:
            arrays[i, int(np.argmax(row[1:])), :] = 1
    return arrays


def tanh_as_sigmoid(layers, linear, weights):
    """Exact reparametrisation of a network with tanh layers as a sigmoid
    network, through tanh(z) = 2 sigma(2z) - 1, so that a server without tanh
    (the reference's, cuda/cpde_server.cu:457) computes the same outputs and
    every derivative row of them.

    Weight layer l maps layer l-1 to layer l; with c = 2 if layer l is tanh
    (else 1) and t = "layer l-1 is tanh": W' = c * (2W if t else W) and
    b' = c * (b - W 1 if t else b). Returns (linear', weights') with every
    tanh flag (2) replaced by sigmoid (0)."""
    out = []
    for l, (width, height) in enumerate(zip(layers[:-1], layers[1:]), start=1):
        flat = np.asarray(weights[l - 1], np.float64)
        W = flat[:width * height].reshape(width, height).T  # column-major storage
        b = flat[width * height:]
        c = 2.0 if linear[l] == 2 else 1.0
        if linear[l - 1] == 2:
            W, b = 2.0 * W, b - W.sum(axis=1)
        out.append(np.concatenate([(c * W).ravel(order='F'), c * b]).astype(np.float32))
    return [0 if a == 2 else a for a in linear], out


def sigmoid_gradients_to_tanh(layers, linear, gradients):
    """Maps per-layer gradients of the tanh_as_sigmoid network back to the
    tanh network's weights (the transpose of that linear map):
    dE/dW = c * (2 G_W - G_b 1^T if t else G_W), dE/db = c * G_b."""
    out = []
    for l, (width, height) in enumerate(zip(layers[:-1], layers[1:]), start=1):
        flat = np.asarray(gradients[l - 1], np.float64)
        G = flat[:width * height].reshape(width, height).T
        gb = flat[width * height:]
        c = 2.0 if linear[l] == 2 else 1.0
        if linear[l - 1] == 2:
            G = 2.0 * G - gb[:, None]
        out.append(np.concatenate([(c * G).ravel(order='F'), c * gb]))
    return out


def glorot_like(layers, seed=0):
    """Benchmark initialisation: per layer in order, N(0, 1/sqrt(fan_in)) weights
    stored column-major (Fortran ravel) followed by zero biases."""
    rng = np.random.default_rng(seed)
    out = []
    for width, height in zip(layers[:-1], layers[1:]):
        w = rng.normal(0.0, 1.0 / math.sqrt(width), (height, width)).astype(np.float32)
        out.append(np.concatenate([w.ravel(order='F'), np.zeros(height, np.float32)]))
    return out
