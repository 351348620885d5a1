// Scalar IR shared by compiled integral costs and cost graphs.
//
// Opcodes and their value/partial semantics follow the reference
// (cuda/scalar_ops.cuh:4-27): 0 constant, 1 leaf/component, 2 field, 3 add,
// 4 sub, 5 mul, 6 div, 7 power, 8 neg, 9 exp, 10 log, 11 sqrt, 12 sin, 13 cos,
// 14 tanh, 15 attach (graphs only: value of a, adjoint to both a and b).
#pragma once
#include <cmath>
#include <string>
#include <vector>

#include "common.hpp"

namespace cpde {

enum ScalarOp { kConstant, kLeaf, kField, kAdd, kSub, kMul, kDiv, kPower, kNeg, kExp, kLog, kSqrt, kSin, kCos,
                kTanh, kAttach };

struct ScalarNode {
    int op, a, b;
    double parameter;
};

__host__ __device__ inline double scalar_value(int op, double a, double b, double p) {
    switch (op) {
        case kConstant: return p;
        case kAdd: return a + b;
        case kSub: return a - b;
        case kMul: return a * b;
        case kDiv: return b == 0 ? NAN : a / b;
        case kPower: return (a < 0 && floor(p) != p) || (a == 0 && p < 0) ? NAN : pow(a, p);
        case kNeg: return -a;
        case kExp: return exp(a);
        case kLog: return a > 0 ? log(a) : NAN;
        case kSqrt: return a >= 0 ? sqrt(a) : NAN;
        case kSin: return sin(a);
        case kCos: return cos(a);
        case kTanh: return tanh(a);
        case kAttach: return a;
        default: return NAN;
    }
}

__host__ __device__ inline void scalar_partials(int op, double a, double b, double v, double p, double& da,
                                                double& db) {
    da = db = 0;
    switch (op) {
        case kAdd: case kAttach: da = db = 1; break;
        case kSub: da = 1; db = -1; break;
        case kMul: da = b; db = a; break;
        case kDiv: da = 1 / b; db = -v / b; break;
        case kPower: da = p == 0 ? 0 : (p == 1 ? 1 : p * pow(a, p - 1)); break;
        case kNeg: da = -1; break;
        case kExp: da = v; break;
        case kLog: da = 1 / a; break;
        case kSqrt: da = .5 / v; break;
        case kSin: da = cos(a); break;
        case kCos: da = -sin(a); break;
        case kTanh: da = 1 - v * v; break;
        default: break;
    }
}

inline bool scalar_binary(int op) { return (op >= kAdd && op <= kDiv) || op == kAttach; }

}  // namespace cpde
