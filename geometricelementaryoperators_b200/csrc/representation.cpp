// representation.cpp -- search for signed-Pauli-string representations of
// Cl(p,q), n <= 6 (see representation.h for the math).
#include "representation.h"

#include <cstring>
#include <utility>
#include <vector>

#include "geo_internal.h"

namespace geo {
namespace {

int popc(unsigned v) { return __builtin_popcount(v); }

struct Str {
    unsigned x, z;
};

// Square sign of a string and commutation parity of two strings.
int square_sign(Str s) { return (popc(s.x & s.z) & 1) ? -1 : 1; }
bool anticommute(Str a, Str b) { return ((popc(a.z & b.x) + popc(b.z & a.x)) & 1) != 0; }

// Product of two signed strings: (s1 P1)(s2 P2) = s1 s2 (-1)^popc(z1 & x2) P(x1^x2, z1^z2).
void multiply(int &sign, Str &acc, Str g) {
    if (popc(acc.z & g.x) & 1) sign = -sign;
    acc.x ^= g.x;
    acc.z ^= g.z;
}

// Gaussian elimination over GF(2) on 2d-bit vectors: true if v is independent of basis.
bool independent(std::vector<unsigned> &basis, unsigned v) {
    for (unsigned b : basis) {
        const unsigned top = 31u - (unsigned)__builtin_clz(b);
        if ((v >> top) & 1u) v ^= b;
    }
    if (v == 0) return false;
    // keep basis in reduced form ordered by leading bit
    basis.push_back(v);
    for (size_t i = basis.size() - 1; i > 0; --i) {
        const unsigned ti = 31u - (unsigned)__builtin_clz(basis[i]);
        const unsigned tp = 31u - (unsigned)__builtin_clz(basis[i - 1]);
        if (ti > tp) std::swap(basis[i], basis[i - 1]);
    }
    return true;
}

struct Search {
    int n, d;
    const int8_t *sig;
    std::vector<Str> chosen;
    RepPlan *out;
    int side;

    bool finish() {
        const int N = 1 << n, D = 1 << d;
        // Blade strings.
        for (int A = 0; A < N; ++A) {
            int sign = 1;
            Str acc{0, 0};
            for (int a = 0; a < n; ++a)
                if ((A >> a) & 1) multiply(sign, acc, chosen[a]);
            out->xm[A] = (uint8_t)acc.x;
            out->zm[A] = (uint8_t)acc.z;
            out->sg[A] = (int8_t)sign;
        }
        // The x-masks must cover all of Z_2^d so that S * D == N.
        unsigned span_x = 0;
        std::vector<unsigned> xb;
        for (int a = 0; a < n; ++a)
            if (independent(xb, chosen[a].x)) ++span_x;
        if ((int)span_x != d) return false;
        const int S = N / D;
        out->D = D;
        out->S = S;
        out->c = S;
        // Try row (column) subsets of size S until P^T P == S I.
        std::vector<int> pick(S);
        for (int i = 0; i < S; ++i) pick[i] = i;
        for (;;) {
            if (try_rows(pick)) return true;
            int i = S - 1;
            while (i >= 0 && pick[i] == D - S + i) --i;
            if (i < 0) return false;
            ++pick[i];
            for (int j = i + 1; j < S; ++j) pick[j] = pick[j - 1] + 1;
        }
    }

    bool try_rows(const std::vector<int> &pick) {
        const int N = 1 << n, D = out->D, S = out->S;
        // Dense kept-entry matrix P[e][A] with e = r*D + k.
        std::vector<int> P((size_t)N * N, 0);
        for (int r = 0; r < S; ++r) {
            for (int k = 0; k < D; ++k) {
                const int e = r * D + k;
                for (int A = 0; A < N; ++A) {
                    // right: rho(e_A)[rows[r]][k];  left: rho(e_A)[k][rows[r]]
                    const int i = side == 0 ? pick[r] : k;
                    const int j = side == 0 ? k : pick[r];
                    if (i != (j ^ out->xm[A])) continue;
                    P[(size_t)e * N + A] = out->sg[A] * ((popc(out->zm[A] & j) & 1) ? -1 : 1);
                }
            }
        }
        for (int A = 0; A < N; ++A)
            for (int B = 0; B < N; ++B) {
                long dot = 0;
                for (int e = 0; e < N; ++e) dot += (long)P[(size_t)e * N + A] * P[(size_t)e * N + B];
                if (dot != (A == B ? S : 0)) return false;
            }
        for (int r = 0; r < S; ++r) out->rows[r] = (uint8_t)pick[r];
        for (int e = 0; e < N; ++e) {
            int t = 0;
            for (int A = 0; A < N; ++A) {
                const int v = P[(size_t)e * N + A];
                if (v == 0) continue;
                if (t >= 8) return false;
                out->gb[e][t] = (uint8_t)A;
                out->gs[e][t] = (int8_t)v;
                ++t;
            }
            if (t != S) return false;
        }
        return true;
    }

    bool dfs(int axis, std::vector<unsigned> &basis) {
        if (axis == n) return finish();
        const unsigned limit = 1u << (2 * d);
        for (unsigned v = 1; v < limit; ++v) {
            const Str s{v & ((1u << d) - 1u), v >> d};
            if (square_sign(s) != sig[axis]) continue;
            bool ok = true;
            for (const Str &c : chosen) ok = ok && anticommute(c, s);
            if (!ok) continue;
            std::vector<unsigned> b2 = basis;
            if (!independent(b2, v)) continue;
            chosen.push_back(s);
            if (dfs(axis + 1, b2)) return true;
            chosen.pop_back();
        }
        return false;
    }
};

}  // namespace

int rep_entry(const RepPlan &p, int blade, int i, int j) {
    if (i != (j ^ p.xm[blade])) return 0;
    return p.sg[blade] * ((__builtin_popcount(p.zm[blade] & j) & 1) ? -1 : 1);
}

bool make_rep_plan(RepPlan *out, uint8_t dimension, const int8_t *signature, int side) {
    if (out == nullptr || !signature_valid(signature, dimension)) return false;
    std::memset(out, 0, sizeof(*out));
    const int n = dimension;
    out->dimension = n;
    out->blades = 1 << n;
    out->side = side ? 1 : 0;
    for (int d = (n + 1) / 2; d <= 4 && d <= n; ++d) {
        Search s{n, d, signature, {}, out, out->side};
        std::vector<unsigned> basis;
        if (!s.dfs(0, basis)) continue;
        // Self-check: rho(e_A) rho(e_B) == s(A, B) rho(e_{A^B}) for all blade pairs.
        const int N = 1 << n, D = 1 << d;
        bool good = true;
        for (int A = 0; A < N && good; ++A)
            for (int B = 0; B < N && good; ++B) {
                const int s_ref = sign_rule((uint8_t)A, (uint8_t)B, signature, (uint8_t)n);
                for (int i = 0; i < D && good; ++i) {
                    // (rho_A rho_B)[i][j] has one non-zero column j
                    const int mid = i ^ out->xm[A];  // rho_A[i][mid] != 0
                    const int j = mid ^ out->xm[B];
                    const int prod = rep_entry(*out, A, i, mid) * rep_entry(*out, B, mid, j);
                    good = prod == s_ref * rep_entry(*out, A ^ B, i, j);
                }
            }
        if (!good) continue;
        out->valid = 1;
        return true;
    }
    std::memset(out, 0, sizeof(*out));
    return false;
}

namespace {

// Perfect matching on a bipartite graph (left = lanes, right = bank classes)
// by augmenting paths; adj[l] lists candidate edges as (class, edge id).
bool augment(int l, const std::vector<std::vector<std::pair<int, int>>> &adj, std::vector<int> &match_r,
             std::vector<int> &edge_of_r, std::vector<char> &seen) {
    for (const auto &ce : adj[l]) {
        const int r = ce.first;
        if (seen[r]) continue;
        seen[r] = 1;
        if (match_r[r] < 0 || augment(match_r[r], adj, match_r, edge_of_r, seen)) {
            match_r[r] = l;
            edge_of_r[r] = ce.second;
            return true;
        }
    }
    return false;
}

}  // namespace

bool make_rep_device(RepDevice *out, const RepPlan &p) {
    if (!p.valid || p.S > 8 || p.D > 16) return false;
    std::memset(out, 0, sizeof(*out));
    for (int A = 0; A < 64; ++A) {
        out->xm[A] = p.xm[A];
        out->zm[A] = p.zm[A];
        out->sg[A] = p.sg[A];
    }
    const int D = p.D, S = p.S, N = p.blades, c = p.c;
    out->blades = N;
    out->D = D;
    out->S = S;
    out->side = p.side;
    // Bank classes: a warp's gather load covers 32 / D samples. Raw rows are
    // unpadded; for D = 8 odd samples are stored with their 64-byte halves
    // swapped (blade A at column A ^ 8), so four samples spread over all 16
    // double-banks when the D lanes of one sample load blades distinct modulo 8.
    // For D = 16 the 16 lanes of one sample need blades distinct modulo 16.
    const int mod = D >= 16 ? 16 : 8;
    out->raw_stride = N;
    // Group members and their signs from the kept-entry gather table.
    std::vector<std::vector<int>> members(D);
    for (int A = 0; A < N; ++A) members[p.xm[A]].push_back(A);
    for (int m = 0; m < D; ++m)
        if ((int)members[m].size() != c) return false;
    // Edge-colour the c-regular bipartite multigraph (group m) x (blade mod `mod`)
    // into c perfect matchings: matching t gives every group its load at step t.
    std::vector<std::vector<int>> remaining = members;
    for (int t = 0; t < c; ++t) {
        std::vector<std::vector<std::pair<int, int>>> adj(D);
        for (int m = 0; m < D; ++m)
            for (int i = 0; i < (int)remaining[m].size(); ++i) adj[m].push_back({remaining[m][i] % mod, i});
        std::vector<int> match_r(mod, -1), edge_of_r(mod, -1);
        for (int m = 0; m < D; ++m) {
            std::vector<char> seen(mod, 0);
            if (!augment(m, adj, match_r, edge_of_r, seen)) return false;
        }
        std::vector<int> take(D, -1);
        for (int r = 0; r < mod; ++r)
            if (match_r[r] >= 0) take[match_r[r]] = edge_of_r[r];
        for (int m = 0; m < D; ++m) {
            if (take[m] < 0) return false;
            out->grp_blade[m][t] = (uint8_t)remaining[m][take[m]];
            remaining[m].erase(remaining[m].begin() + take[m]);
        }
    }
    for (int m = 0; m < D; ++m) {
        uint64_t neg = 0;
        for (int r = 0; r < S; ++r) {
            const int k = p.rows[r] ^ m;
            out->grp_col[m][r] = (uint8_t)k;
            const int e = r * D + k;
            for (int t = 0; t < c; ++t) {
                const int A = out->grp_blade[m][t];
                int sign = 0;
                for (int u = 0; u < c; ++u)
                    if (p.gb[e][u] == A) sign = p.gs[e][u];
                if (sign == 0) return false;
                if (sign < 0) neg |= (uint64_t)1 << (r * 8 + t);
            }
        }
        out->grp_neg[m] = neg;
    }
    return true;
}

}  // namespace geo
