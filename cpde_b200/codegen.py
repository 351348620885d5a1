"""Generate csrc/generated/jets_static.cuh: register-resident jet code for the
derivative schemas the fast tier compiles ahead of time.

For each schema (a list of multi-indices in canonical order: by total order,
then by count tuple, the order cpde/quadrature.py:16-38 produces) this emits
straight-line CUDA with constant indices, so every jet value lives in a
register:

* ``forward<Act>(z, y)``: y = f(z) through the Leibniz recurrence
  y_S = sum_U C(T,U) s_U z_{T-U+e_v},  s_S = lead*y_S - sum C(S,V) y_V y_{S-V};
* ``adjoint<Act>(y, g)``: g <- dE/dZ from g = dE/dY and the stored y, with
  s rebuilt from y and dz_T = sum_{S>=T} C(S,T) s_{S-T} dy_S.

The recurrence and the adjoint identity are the ones csrc/schema.hpp tabulates
for the generic tier. ``python -m cpde_b200.codegen`` rewrites the header.
"""
import itertools
import math
from pathlib import Path

OUT = Path(__file__).resolve().parent / 'csrc' / 'generated' / 'jets_static.cuh'


def full(variables, order):
    rows = [c for c in itertools.product(range(order + 1), repeat=variables) if sum(c) <= order]
    return sorted(rows, key=lambda c: (sum(c), c))


def pure(variables, order):
    rows = {(0,) * variables}
    for v in range(variables):
        for k in range(1, order + 1):
            c = [0] * variables
            c[v] = k
            rows.add(tuple(c))
    return sorted(rows, key=lambda c: (sum(c), c))


def closure_of(tops):
    """Every sub-multi-index of the given rows (the closure a cost requesting
    exactly those derivatives propagates), in canonical order."""
    rows = set()
    for top in tops:
        rows.update(itertools.product(*(range(x + 1) for x in top)))
    return sorted(rows, key=lambda c: (sum(c), c))


# (name, rows) of every static schema; ids are positions in this list.
SCHEMAS = [(f'full{v}d_o{k}', full(v, k)) for v, k in [(2, 0), (2, 1), (2, 2), (2, 3), (2, 4), (2, 5), (2, 6)]]
SCHEMAS += [('pure2d_o2', pure(2, 2)), ('full3d_o4', full(3, 4)), ('pure4d_o6', pure(4, 6))]
# the rows a 3D biharmonic residual (u_xxxx + u_yyyy + u_zzzz + 2 u_xxyy +
# 2 u_xxzz + 2 u_yyzz) propagates, and the 3D Laplacian's
SCHEMAS += [('bih3d_o4', closure_of([(4, 0, 0), (0, 4, 0), (0, 0, 4), (2, 2, 0), (2, 0, 2), (0, 2, 2)])),
            ('pure3d_o2', pure(3, 2))]


def subs(s):
    return list(itertools.product(*(range(x + 1) for x in s)))


def coefficient(s, u):
    return math.prod(math.comb(a, b) for a, b in zip(s, u))


def term(coef, a, b):
    if coef == 1:
        return f'{a} * {b}'
    return f'{float(coef)!r}f * {a} * {b}'


def emit_schema(sid, name, rows):
    R = len(rows)
    index = {c: i for i, c in enumerate(rows)}
    V = len(rows[0])
    out = [f'// schema {sid}: {name}, {R} rows', 'template <>', f'struct StaticJet<{sid}> {{',
           f'    static constexpr int R = {R};', f'    static constexpr int V = {V};']
    # forward
    fwd = ['    template <class Act>',
           f'    __device__ __forceinline__ static void forward(const float (&z)[{R}], float (&y)[{R}]) {{',
           f'        float s[{R}];', '        Act::value(z[0], y[0], s[0]);', '        const float lead = Act::lead(y[0]);']
    for r in range(1, R):
        S = rows[r]
        v = next(i for i, x in enumerate(S) if x)
        T = list(S)
        T[v] -= 1
        parts = []
        for U in subs(T):
            W = [t - u for t, u in zip(T, U)]
            W[v] += 1
            parts.append(term(coefficient(T, U), f's[{index[tuple(U)]}]', f'z[{index[tuple(W)]}]'))
        fwd.append(f'        y[{r}] = ' + ' + '.join(parts) + ';')
        sq = []
        for Vv in subs(S):
            Vc = tuple(a - b for a, b in zip(S, Vv))
            a, b = index[tuple(Vv)], index[Vc]
            if a == 0 or b == 0 or a > b:
                continue
            sq.append(term(coefficient(S, Vv) * (1 if a == b else 2), f'y[{a}]', f'y[{b}]'))
        fwd.append(f'        s[{r}] = lead * y[{r}]' + ''.join(' - ' + t for t in sq) + ';')
    fwd.append('    }')
    # adjoint
    adj = ['    template <class Act>',
           f'    __device__ __forceinline__ static void adjoint(const float (&y)[{R}], float (&g)[{R}]) {{',
           f'        float s[{R}], dz[{R}];', '        s[0] = Act::slope_from_value(y[0]);',
           '        const float lead = Act::lead(y[0]);']
    for r in range(1, R):
        S = rows[r]
        sq = []
        for Vv in subs(S):
            Vc = tuple(a - b for a, b in zip(S, Vv))
            a, b = index[tuple(Vv)], index[Vc]
            if a == 0 or b == 0 or a > b:
                continue
            sq.append(term(coefficient(S, Vv) * (1 if a == b else 2), f'y[{a}]', f'y[{b}]'))
        adj.append(f'        s[{r}] = lead * y[{r}]' + ''.join(' - ' + t for t in sq) + ';')
    for t in range(R):
        T = rows[t]
        parts = []
        for s_idx in range(t, R):
            S = rows[s_idx]
            if any(a < b for a, b in zip(S, T)):
                continue
            D = tuple(a - b for a, b in zip(S, T))
            parts.append(term(coefficient(S, T), f's[{index[D]}]', f'g[{s_idx}]'))
        adj.append(f'        dz[{t}] = ' + ' + '.join(parts) + ';')
    adj.append(f'#pragma unroll\n        for (int i = 0; i < {R}; ++i) g[i] = dz[i];')
    adj.append('    }')
    out += fwd + adj + ['};', '']
    return out


def generate():
    lines = ['// GENERATED by cpde_b200/codegen.py - do not edit.',
             '// Register-resident derivative-jet code for the fast tier.', '#pragma once', '',
             'namespace cpde {', '', 'template <int SID>', 'struct StaticJet;', '']
    for sid, (name, rows) in enumerate(SCHEMAS):
        lines += emit_schema(sid, name, rows)
    # host registry: variables, rows, flattened counts
    lines.append(f'constexpr int kStaticSchemas = {len(SCHEMAS)};')
    flat, offs = [], []
    for name, rows in SCHEMAS:
        offs.append(len(flat))
        for r in rows:
            flat.extend(r)
    lines.append('struct StaticSchemaInfo { int variables, rows, offset; };')
    lines.append('constexpr StaticSchemaInfo kStaticSchemaInfo[] = {' + ', '.join(
        f'{{{len(rows[0])}, {len(rows)}, {o}}}' for (name, rows), o in zip(SCHEMAS, offs)) + '};')
    lines.append(f'constexpr int kStaticSchemaCounts[] = {{{", ".join(map(str, flat))}}};')
    lines += ['', '}  // namespace cpde', '']
    return '\n'.join(lines)


SOURCE_OUT = OUT.with_name('jets_static_source.cuh')


def generate_source_table():
    """The same StaticJet code as C++ string literals, one per schema, for the
    kernels the engine compiles at run time with NVRTC (the fused expression
    head): the run-time source then carries exactly the jet code the
    ahead-of-time kernels use."""
    lines = ['// GENERATED by cpde_b200/codegen.py - do not edit.',
             '// Source text of each StaticJet<SID> specialisation, for NVRTC-compiled kernels.', '#pragma once', '',
             'namespace cpde {', '', 'static const char* const kStaticJetSource[] = {']
    for sid, (name, rows) in enumerate(SCHEMAS):
        body = '\n'.join(emit_schema(sid, name, rows))
        lines.append(f'    R"JET({body})JET",')
    lines += ['};', '', '}  // namespace cpde', '']
    return '\n'.join(lines)


def write():
    OUT.parent.mkdir(parents=True, exist_ok=True)
    for path, text in ((OUT, generate()), (SOURCE_OUT, generate_source_table())):
        if not path.exists() or path.read_text() != text:
            path.write_text(text)
    return OUT


if __name__ == '__main__':
    print(write())
