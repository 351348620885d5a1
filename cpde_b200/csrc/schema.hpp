// Derivative schema compiler.
//
// A context's rows are multi-indices S (counts per input variable), value row
// first, orders 0..6, closed under taking sub-multi-indices (the closure the
// reference builds in cpde/_prepare.py:132-138 and checks in
// cuda/cpde_server.cu:113-123). Instead of the reference's per-row subset
// pointer stacks and set-partition expansions (cuda/cpde_engine.cuh:213-469,
// cuda/derivative_kernels_v4.cu:382-745), rows are propagated by a Leibniz
// recurrence on two jets:
//
//   y = f(z) (sigmoid or tanh), s = f'(z) as a jet.
//   y_S = sum_{U <= T} C(T,U) s_U z_{T-U+e_v}          with S = T + e_v
//   s_S = lead * y_S - sum_{0<V<S} C(S,V) y_V y_{S-V}   (f' = f - f^2 or 1 - f^2)
//   adjoint: dz_T = sum_{S >= T} C(S,T) s_{S-T} dy_S
//
// which costs O(#sub-index pairs) per element instead of O(Bell(k)) and needs
// only the value and the s-jet. The adjoint identity is the one the reference
// uses (cuda/derivative_kernels_v4.cu:349-380, dTab/Crs of
// cuda/cpde_engine.cuh:476-498).
#pragma once
#include <algorithm>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "common.hpp"

namespace cpde {

struct JetTerm {
    float coef;
    int32_t a, b;
};

struct JetPlan {
    int rows = 0, variables = 0, max_order = 0;
    std::vector<std::vector<int>> counts;
    // y_S += coef * s[a] * z[b]          (rows 1..R-1)
    std::vector<int> fwd_start;
    std::vector<JetTerm> fwd;
    // s_S -= coef * y[a] * y[b]          (rows 1..R-1; symmetric pairs merged)
    std::vector<int> sq_start;
    std::vector<JetTerm> sq;
    // dz_T += coef * s[a] * dy[b]        (rows 0..R-1; includes S = T)
    std::vector<int> adj_start;
    std::vector<JetTerm> adj;

    static long binom(int n, int k) {
        long r = 1;
        for (int i = 1; i <= k; ++i) r = r * (n - k + i) / i;
        return r;
    }

    static JetPlan build(const std::vector<std::vector<int>>& counts) {
        JetPlan p;
        require(!counts.empty(), "empty derivative closure");
        p.rows = int(counts.size());
        p.variables = int(counts[0].size());
        p.counts = counts;
        std::map<std::vector<int>, int> index;
        int previous = -1;
        for (int r = 0; r < p.rows; ++r) {
            const auto& c = counts[r];
            require(int(c.size()) == p.variables, "inconsistent derivative table");
            int order = 0;
            for (int x : c) {
                require(x >= 0 && x <= 6, "derivative counts must be 0..6");
                order += x;
            }
            require(order >= previous && order <= 6, "derivative closure must be sorted, orders 0..6");
            previous = order;
            p.max_order = std::max(p.max_order, order);
            require(index.emplace(c, r).second, "duplicate derivative row");
        }
        require(std::all_of(counts[0].begin(), counts[0].end(), [](int x) { return x == 0; }),
                "value derivative must come first");
        auto find = [&](const std::vector<int>& c) {
            auto it = index.find(c);
            require(it != index.end(), "derivative closure is missing a lower-order dependency");
            return it->second;
        };
        // Enumerate all U <= S.
        auto subs = [&](const std::vector<int>& s) {
            std::vector<std::vector<int>> out{std::vector<int>(s.size(), 0)};
            for (size_t v = 0; v < s.size(); ++v) {
                std::vector<std::vector<int>> next;
                for (auto& u : out)
                    for (int k = 0; k <= s[v]; ++k) {
                        auto w = u;
                        w[v] = k;
                        next.push_back(w);
                    }
                out.swap(next);
            }
            return out;
        };
        auto coefficient = [&](const std::vector<int>& s, const std::vector<int>& u) {
            long c = 1;
            for (size_t v = 0; v < s.size(); ++v) c *= binom(s[v], u[v]);
            return c;
        };
        p.fwd_start.assign(p.rows + 1, 0);
        p.sq_start.assign(p.rows + 1, 0);
        for (int r = 0; r < p.rows; ++r) {
            p.fwd_start[r] = int(p.fwd.size());
            p.sq_start[r] = int(p.sq.size());
            if (r == 0) continue;
            const auto& S = counts[r];
            int v = 0;
            while (S[v] == 0) ++v;
            auto T = S;
            T[v] -= 1;
            for (auto& U : subs(T)) {
                auto W = T;
                for (int i = 0; i < p.variables; ++i) W[i] -= U[i];
                W[v] += 1;
                p.fwd.push_back({float(coefficient(T, U)), find(U), find(W)});
            }
            for (auto& V : subs(S)) {
                auto Vc = S;
                for (int i = 0; i < p.variables; ++i) Vc[i] -= V[i];
                int a = find(V), b = find(Vc);
                if (a == 0 || b == 0 || a > b) continue;  // lead term and mirrored pairs
                long c = coefficient(S, V) * (a == b ? 1 : 2);
                p.sq.push_back({float(c), a, b});
            }
        }
        p.fwd_start[p.rows] = int(p.fwd.size());
        p.sq_start[p.rows] = int(p.sq.size());
        p.adj_start.assign(p.rows + 1, 0);
        for (int t = 0; t < p.rows; ++t) {
            p.adj_start[t] = int(p.adj.size());
            const auto& T = counts[t];
            for (int s = t; s < p.rows; ++s) {
                const auto& S = counts[s];
                bool above = true;
                for (int i = 0; i < p.variables; ++i) above = above && S[i] >= T[i];
                if (!above) continue;
                auto D = S;
                for (int i = 0; i < p.variables; ++i) D[i] -= T[i];
                p.adj.push_back({float(coefficient(S, T)), find(D), s});
            }
        }
        p.adj_start[p.rows] = int(p.adj.size());
        return p;
    }

    // Packed device table: [3 x (R+1) starts][fwd][sq][adj] as int32 words,
    // each term 3 words (coef bits, a, b).
    std::vector<int32_t> pack() const {
        const int header = 3 * (rows + 1);
        const int fwd_base = header, sq_base = fwd_base + 3 * int(fwd.size());
        const int adj_base = sq_base + 3 * int(sq.size());
        std::vector<int32_t> out(header);
        for (int i = 0; i <= rows; ++i) {
            out[i] = fwd_base + 3 * fwd_start[i];
            out[rows + 1 + i] = sq_base + 3 * sq_start[i];
            out[2 * (rows + 1) + i] = adj_base + 3 * adj_start[i];
        }
        for (const auto* ts : {&fwd, &sq, &adj})
            for (const auto& t : *ts) {
                int32_t bits;
                std::memcpy(&bits, &t.coef, 4);
                out.push_back(bits);
                out.push_back(t.a);
                out.push_back(t.b);
            }
        return out;
    }

    std::string key() const {
        std::string k;
        for (auto& c : counts) {
            for (int x : c) k.push_back(char('0' + x));
            k.push_back(',');
        }
        return k;
    }
};

}  // namespace cpde
