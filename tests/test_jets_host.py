"""The generated register jet code (csrc/generated/jets_static.cuh, the
forward combine and adjoint fused into every fast-tier and tensor-core
kernel) against the float64 oracle, on the CPU.

The generated header is plain arithmetic, so it is compiled here as host C++
(g++) with host versions of the two activations, and each schema's forward
(y = f(z) as jets) and adjoint (dE/dZ from dE/dY and the stored y) is run on
seeded jets and compared with oracle/jets.py (the reference's set-partition
formulas, cuda/derivative_kernels_v4.cu:12-745). Tolerances as everywhere:
per-row normwise relative error below 1e-5 for orders <= 3 and 1e-4 for
orders 4-6.
"""
import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from cpde_b200 import codegen
from oracle import jets

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'cpde_b200' / 'csrc' / 'generated' / 'jets_static.cuh'

HARNESS = r'''
#include <cmath>
#define __device__
#define __forceinline__ inline
// host versions of the activations (same formulas as the device structs)
struct Sigmoid {
    static void value(float z, float& y, float& s) {
        float e = std::exp(-std::fabs(z));
        float big = 1.0f / (1.0f + e), small = e * big;
        y = z >= 0.f ? big : small;
        s = big * small;
    }
    static float slope_from_value(float y) { return y * (1.0f - y); }
    static float lead(float y) { return 1.0f - 2.0f * y; }
};
struct Tanh {
    static void value(float z, float& y, float& s) {
        y = std::tanh(z);
        s = (1.0f - y) * (1.0f + y);
    }
    static float slope_from_value(float y) { return (1.0f - y) * (1.0f + y); }
    static float lead(float y) { return -2.0f * y; }
};
#include "jets_static.cuh"
using namespace cpde;

template <int SID, class Act>
static void run(int adjoint, const float* a, float* b, int count) {
    constexpr int R = StaticJet<SID>::R;
    for (int p = 0; p < count; ++p) {
        float x[R], y[R];
        for (int r = 0; r < R; ++r) x[r] = a[p * R + r];
        if (adjoint) {
            for (int r = 0; r < R; ++r) y[r] = b[p * R + r];
            StaticJet<SID>::template adjoint<Act>(x, y);
        } else {
            StaticJet<SID>::template forward<Act>(x, y);
        }
        for (int r = 0; r < R; ++r) b[p * R + r] = y[r];
    }
}

template <int SID>
static int dispatch(int sid, int act, int adjoint, const float* a, float* b, int count) {
    if constexpr (SID < kStaticSchemas) {
        if (sid != SID) return dispatch<SID + 1>(sid, act, adjoint, a, b, count);
        if (act) run<SID, Tanh>(adjoint, a, b, count);
        else run<SID, Sigmoid>(adjoint, a, b, count);
        return StaticJet<SID>::R;
    }
    return -1;
}

// adjoint = 0: b = forward(a = z); adjoint = 1: b (dE/dY in) = adjoint(a = y, b)
extern "C" int jet_run(int sid, int act, int adjoint, const float* a, float* b, int count) {
    return dispatch<0>(sid, act, adjoint, a, b, count);
}
'''


@pytest.fixture(scope='module')
def harness(tmp_path_factory):
    gxx = shutil.which('g++')
    if not gxx:
        pytest.skip('g++ not available')
    d = tmp_path_factory.mktemp('jets')
    src = d / 'harness.cpp'
    src.write_text(HARNESS)
    lib = d / 'libjets.so'
    subprocess.run([gxx, '-std=c++17', '-O1', '-shared', '-fPIC', '-Wno-unknown-pragmas', f'-I{HEADER.parent}',
                    str(src), '-o', str(lib)], check=True)
    h = ctypes.CDLL(str(lib))
    h.jet_run.restype = ctypes.c_int
    h.jet_run.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    return h


def rowwise(a, b):
    return np.linalg.norm(a - b, axis=1) / np.maximum(np.linalg.norm(b, axis=1), 1e-300)


CASES = [(sid, name) for sid, (name, _) in enumerate(codegen.SCHEMAS)]


@pytest.mark.parametrize('sid,name', CASES, ids=[c[1] for c in CASES])
@pytest.mark.parametrize('kind', ['sigmoid', 'tanh'])
def test_generated_jets_match_oracle(harness, sid, name, kind):
    rows = codegen.SCHEMAS[sid][1]
    schema = jets.Schema(rows)
    R, P = len(rows), 257
    rng = np.random.default_rng(100 + sid)
    z = rng.normal(0, 0.5, (R, P))
    z[0] = rng.uniform(-3, 3, P)
    z = z.astype(np.float32).astype(np.float64)
    act = 0 if kind == 'sigmoid' else 1
    tol = 1e-5 if max(sum(r) for r in rows) <= 3 else 1e-4

    y_ref = jets.jet_forward(schema, z, kind)
    zin = np.ascontiguousarray(z.T, np.float32)  # (point, row)
    y = np.zeros_like(zin)
    assert harness.jet_run(sid, act, 0, zin.ctypes.data, y.ctypes.data, P) == R
    assert rowwise(y.T.astype(np.float64), y_ref).max() < tol

    g = rng.normal(0, 1, (R, P)).astype(np.float32).astype(np.float64)
    dz_ref = jets.jet_adjoint(schema, z, g, kind)
    yin = np.ascontiguousarray(y_ref.T, np.float32)  # the stored activations
    dz = np.ascontiguousarray(g.T, np.float32)
    assert harness.jet_run(sid, act, 1, yin.ctypes.data, dz.ctypes.data, P) == R
    assert rowwise(dz.T.astype(np.float64), dz_ref).max() < tol
