// representation.cpp -- search for signed-Pauli-string representations of
// Cl(p,q), n <= 6 (see representation.h for the math).
#include "representation.h"

#include <cstring>
#include <mutex>
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

// Edge-colours the bipartite multigraph (lane L) x (blade mod `mod`), where
// lane L may load any blade of lanes[L], into `steps` perfect matchings:
// matching t gives every lane its load at step t. The graph is regular, so a
// perfect matching exists at every step (Koenig).
bool colour_loads(const std::vector<std::vector<int>> &lanes, int mod, int steps, uint8_t (*order)[8]) {
    std::vector<std::vector<int>> remaining = lanes;
    const int L = (int)lanes.size();
    for (int t = 0; t < steps; ++t) {
        std::vector<std::vector<std::pair<int, int>>> adj(L);
        for (int l = 0; l < L; ++l)
            for (int i = 0; i < (int)remaining[l].size(); ++i) adj[l].push_back({remaining[l][i] % mod, i});
        std::vector<int> match_r(mod, -1), edge_of_r(mod, -1);
        for (int l = 0; l < L; ++l) {
            std::vector<char> seen(mod, 0);
            if (!augment(l, adj, match_r, edge_of_r, seen)) return false;
        }
        std::vector<int> take(L, -1);
        for (int r = 0; r < mod; ++r)
            if (match_r[r] >= 0) take[match_r[r]] = edge_of_r[r];
        for (int l = 0; l < L; ++l) {
            if (take[l] < 0) return false;
            order[l][t] = (uint8_t)remaining[l][take[l]];
            remaining[l].erase(remaining[l].begin() + take[l]);
        }
    }
    return true;
}

// Sign bits of group m's gather for a load order: bit (r * 8 + t) set when
// kept entry (r, rows[r] ^ m) takes blade order[t] with a minus sign.
bool gather_signs(const RepPlan &p, int m, const uint8_t *order, uint64_t *neg_out) {
    uint64_t neg = 0;
    for (int r = 0; r < p.S; ++r) {
        const int e = r * p.D + (p.rows[r] ^ m);
        for (int t = 0; t < p.c; ++t) {
            int sign = 0;
            for (int u = 0; u < p.c; ++u)
                if (p.gb[e][u] == order[t]) sign = p.gs[e][u];
            if (sign == 0) return false;
            if (sign < 0) neg |= (uint64_t)1 << (r * 8 + t);
        }
    }
    *neg_out = neg;
    return true;
}

// Coordinates of a group's blades: all groups share the subspace V of z-masks
// of group 0 (the blades with x-mask 0), and group m's blades are
// A(m, c) = A(m, 0) ^ sum_i c_i a_i with a_i the blade of group 0 whose z-mask
// is the i-th basis vector of V.
bool make_ws_tables(RepDevice *out, const RepPlan &p, const std::vector<std::vector<int>> &members) {
    const int D = p.D, S = p.S;
    int d = 0;
    while ((1 << d) < S) ++d;
    // Basis of V from group 0 (which contains the scalar blade, z = 0).
    std::vector<int> basis_blade;
    {
        std::vector<unsigned> ech;
        for (int A : members[0]) {
            if (p.zm[A] == 0) continue;
            std::vector<unsigned> e2 = ech;
            if (independent(e2, p.zm[A])) {
                ech = e2;
                basis_blade.push_back(A);
            }
        }
        if ((int)basis_blade.size() != d) return false;
    }
    auto blade_at = [&](int m, int c) {
        int A = members[m][0];
        for (int i = 0; i < d; ++i)
            if ((c >> i) & 1) A ^= basis_blade[i];
        return A;
    };
    auto sign_in_entry = [&](int r, int k, int A) {
        const int e = r * D + k;
        for (int u = 0; u < p.c; ++u)
            if (p.gb[e][u] == A) return (int)p.gs[e][u];
        return 0;
    };
    // Per group: alpha(r), beta(c), phi(r) with s(r, c) = alpha beta (-1)^{c . phi}.
    std::vector<std::vector<int>> alpha(D, std::vector<int>(S)), beta(D, std::vector<int>(S)),
        phi(D, std::vector<int>(S));
    for (int m = 0; m < D; ++m) {
        std::vector<std::vector<int>> s(S, std::vector<int>(S));
        for (int c = 0; c < S; ++c) {
            const int A = blade_at(m, c);
            if (p.xm[A] != m) return false;
            for (int r = 0; r < S; ++r) {
                s[r][c] = sign_in_entry(r, p.rows[r] ^ m, A);
                if (s[r][c] == 0) return false;
            }
        }
        std::vector<char> seen(S, 0);
        for (int r = 0; r < S; ++r) {
            alpha[m][r] = s[r][0];
            int f = 0;
            for (int i = 0; i < d; ++i) {
                const int chi = s[r][1 << i] * s[r][0] * s[0][1 << i] * s[0][0];
                if (chi < 0) f |= 1 << i;
            }
            phi[m][r] = f;
            if (seen[f]) return false;
            seen[f] = 1;
        }
        for (int c = 0; c < S; ++c) beta[m][c] = s[0][c] * s[0][0];
        for (int r = 0; r < S; ++r)
            for (int c = 0; c < S; ++c) {
                const int ch = (__builtin_popcount(c & phi[m][r]) & 1) ? -1 : 1;
                if (alpha[m][r] * beta[m][c] * ch != s[r][c]) return false;
            }
    }
    // delta per lane: 16 lanes of a half-warp need distinct banks (blade mod 16)
    // at step 0; the loads of step t differ from step 0 by one common XOR, so
    // every step is then conflict-free.
    const int lanes = D == 8 ? 16 : D;
    std::vector<std::vector<std::pair<int, int>>> adj(lanes);
    for (int L = 0; L < lanes; ++L)
        for (int delta = 0; delta < S; ++delta) adj[L].push_back({blade_at(L % D, delta) % 16, delta});
    std::vector<int> match_r(16, -1), edge_of_r(16, -1);
    for (int L = 0; L < lanes; ++L) {
        std::vector<char> seen(16, 0);
        if (!augment(L, adj, match_r, edge_of_r, seen)) return false;
    }
    std::vector<int> delta(lanes, -1);
    for (int b = 0; b < 16; ++b)
        if (match_r[b] >= 0) delta[match_r[b]] = edge_of_r[b];
    for (int L = 0; L < lanes; ++L) {
        if (delta[L] < 0) return false;
        const int m = L % D;
        uint8_t in_neg = 0, out_neg = 0;
        for (int t = 0; t < S; ++t) {
            const int c = t ^ delta[L];
            out->ws_blade[L][t] = (uint8_t)blade_at(m, c);
            if (beta[m][c] < 0) in_neg |= (uint8_t)(1u << t);
        }
        for (int r = 0; r < S; ++r) {
            const int f = phi[m][r];
            out->ws_out_row[L][f] = (uint8_t)r;
            const int sg = alpha[m][r] * ((__builtin_popcount(delta[L] & f) & 1) ? -1 : 1);
            if (sg < 0) out_neg |= (uint8_t)(1u << f);
        }
        out->ws_in_neg[L] = in_neg;
        out->ws_out_neg[L] = out_neg;
    }
    return true;
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
    out->raw_stride = N;
    std::vector<std::vector<int>> members(D);
    for (int A = 0; A < N; ++A) members[p.xm[A]].push_back(A);
    for (int m = 0; m < D; ++m)
        if ((int)members[m].size() != c) return false;
    for (int m = 0; m < D; ++m)
        for (int r = 0; r < S; ++r) out->grp_col[m][r] = (uint8_t)(p.rows[r] ^ m);
    // Synchronous kernel: a warp's gather load covers 32 / D samples. For D = 8
    // odd samples are staged with their 64-byte halves swapped (blade A at
    // column A ^ 8), so the D lanes of one sample need blades distinct modulo 8;
    // for D = 16 the 16 lanes of one sample need blades distinct modulo 16.
    if (!colour_loads(members, D >= 16 ? 16 : 8, c, out->grp_blade)) return false;
    for (int m = 0; m < D; ++m)
        if (!gather_signs(p, m, out->grp_blade[m], &out->grp_neg[m])) return false;
    // Warp-specialised kernel: butterfly tables (the kernel exists for
    // D = 16, S >= 2 and D = 8, S >= 4; without tables the synchronous kernel runs).
    if ((D == 16 && S >= 2) || (D == 8 && S >= 4)) out->ws_ready = make_ws_tables(out, p, members) ? 1 : 0;
    // Complex structure J = P(12, 4): it commutes with P(x_A, z_A) when
    // popc(z_J & x_A) + popc(z_A & x_J) is even, for every blade A.
    bool commutes = D == 16 && S == 4;
    for (int A = 0; commutes && A < N; ++A)
        commutes = ((__builtin_popcount(4u & p.xm[A]) + __builtin_popcount(12u & p.zm[A])) & 1) == 0;
    out->cplx = commutes ? 1 : 0;
    return true;
}

bool rep_supported(const RepDevice &rep) {
    return (rep.D == 16 && rep.S == 4) || (rep.D == 8 && rep.S == 8) || (rep.D == 8 && rep.S == 4) ||
           (rep.D == 16 && rep.S == 2);
}

namespace {
// Index: dimension (5, 6) x signature bit pattern (bit a set = axis a is -1) x side.
struct RepSlot {
    bool tried = false;
    bool usable = false;
    RepDevice rep;
};
RepSlot g_rep_slots[2][64][2];
std::mutex g_rep_mutex;
}  // namespace

const RepDevice *cached_rep_device(uint8_t dimension, const int8_t *signature, bool parameter_on_left) {
    if (dimension < 5 || dimension > kMaxDim || !signature_valid(signature, dimension)) return nullptr;
    unsigned mask = 0;
    for (unsigned a = 0; a < dimension; ++a)
        if (signature[a] < 0) mask |= 1u << a;
    RepSlot &slot = g_rep_slots[dimension - 5][mask][parameter_on_left ? 1 : 0];
    std::lock_guard<std::mutex> lock(g_rep_mutex);
    if (!slot.tried) {
        slot.tried = true;
        RepPlan rp;
        slot.usable = make_rep_plan(&rp, dimension, signature, parameter_on_left ? 1 : 0) &&
                      make_rep_device(&slot.rep, rp) && rep_supported(slot.rep) && slot.rep.ws_ready;
    }
    return slot.usable ? &slot.rep : nullptr;
}

}  // namespace geo

namespace geo {

bool make_pair_tables(const RepPlan &p, const int8_t *signature, bool rev_a, bool rev_b, PairTables *out) {
    std::memset(out, 0, sizeof(*out));
    if (!p.valid || p.dimension != 6 || p.D != 16 || p.S != 4 || p.side != 0) return false;
    int kern[4], nk = 0;  // the blades with x-mask 0
    for (int A = 0; A < 64; ++A)
        if (p.xm[A] == 0) {
            if (nk == 4) return false;
            kern[nk++] = A;
        }
    if (nk != 4 || kern[0] != 0) return false;
    const int k1 = kern[1];
    int k2 = -1;
    for (int i = 2; i < 4; ++i)
        if (p.zm[kern[i]] != p.zm[k1]) {
            k2 = kern[i];
            break;
        }
    if (k2 < 0) return false;
    unsigned z[4] = {p.zm[k1], p.zm[k2], 0, 0};
    if (z[0] == 0 || z[1] == 0 || z[0] == z[1]) return false;
    auto spans = [&](unsigned v, int n) {
        for (unsigned c = 0; c < (1u << n); ++c) {
            unsigned acc = 0;
            for (int i = 0; i < n; ++i)
                if ((c >> i) & 1u) acc ^= z[i];
            if (acc == v) return true;
        }
        return false;
    };
    int nz = 2;  // extend {z1, z2} to a basis with unit vectors
    for (unsigned e = 1; e < 16 && nz < 4; e <<= 1)
        if (!spans(e, nz)) z[nz++] = e;
    if (nz != 4) return false;
    int coord[16];  // z -> its coordinates in the basis z[0..3]
    for (int v = 0; v < 16; ++v) coord[v] = -1;
    for (unsigned c = 0; c < 16; ++c) {
        unsigned acc = 0;
        for (int i = 0; i < 4; ++i)
            if ((c >> i) & 1u) acc ^= z[i];
        coord[acc] = (int)c;
    }
    for (int v = 0; v < 16; ++v)
        if (coord[v] < 0) return false;
    auto T = [&](unsigned x) {
        unsigned u = 0;
        for (int i = 0; i < 4; ++i) u |= (unsigned)(popc(z[i] & x) & 1) << i;
        return u;
    };
    auto kappa = [&](int c) { return ((c & 1) ? k1 : 0) ^ ((c & 2) ? k2 : 0); };
    auto par = [](unsigned v) { return (popc(v) & 1) != 0; };
    const uint32_t NEG = 0x80000000u;
    bool seen[16] = {};
    for (int A = 0; A < 64; ++A) {
        const unsigned g = T(p.xm[A]);
        if (seen[g]) continue;
        seen[g] = true;
        const int B0 = A ^ kappa(coord[p.zm[A]] & 3);
        const unsigned zb = (unsigned)coord[p.zm[B0]];
        if ((zb & 3u) != 0u || T(p.xm[B0]) != g) return false;
        for (int c = 0; c < 4; ++c) {
            const int B = B0 ^ kappa(c);
            if (T(p.xm[B]) != g || (unsigned)coord[p.zm[B]] != (zb ^ (unsigned)c)) return false;
            out->blade[g][c] = (uint8_t)B;
            const bool sneg = p.sg[B] < 0;
            const bool self = sign_rule((uint8_t)B, (uint8_t)B, signature, 6) < 0;
            out->xa[g][c] = (sneg != (rev_a && self)) != (par((unsigned)c & (g & 3u)) != par(zb & g)) ? NEG : 0u;
            out->xb[g][c] = (sneg != (rev_b && self)) ? NEG : 0u;
            out->post[g][c] = (sneg != par(zb & g)) != par((unsigned)c & (g & 3u)) ? NEG : 0u;
        }
        const uint32_t h1 = (zb & 4u) ? NEG : 0u, h2 = (zb & 8u) ? NEG : 0u;
        out->chi[g][0] = h1;
        out->chi[g][1] = h2;
        out->chi[g][2] = h1 ^ h2;
    }
    for (int g = 0; g < 16; ++g)
        if (!seen[g]) return false;
    return true;
}

void pair_product_host(const PairTables &t, const double *a, const double *b, double *y) {
    double yh[4][16];
    auto flip = [](double v, uint32_t m) { return m ? -v : v; };
    for (int l = 0; l < 4; ++l) {
        uint32_t xl[4];
        for (int c = 0; c < 4; ++c) xl[c] = (popc((unsigned)(c & l)) & 1) ? 0x80000000u : 0u;
        double ah[16];
        for (int m = 0; m < 16; ++m) {
            double w[4];
            for (int c = 0; c < 4; ++c) w[c] = flip(a[t.blade[m][c]], t.xa[m][c] ^ xl[c]);
            ah[m] = (w[0] + w[1]) + (w[2] + w[3]);
        }
        for (int u = 0; u < 16; ++u) yh[l][u] = 0.0;
        for (int g = 0; g < 16; ++g) {
            double w[4];
            for (int c = 0; c < 4; ++c) w[c] = flip(b[t.blade[g][c]], t.xb[g][c] ^ xl[c]);
            for (int h = 1; h < 4; h <<= 1)
                for (int c = 0; c < 4; ++c)
                    if (!(c & h)) {
                        const double u0 = w[c], v0 = w[c | h];
                        w[c] = u0 + v0;
                        w[c | h] = u0 - v0;
                    }
            for (int u = 0; u < 16; ++u) {
                const int uh = u >> 2;
                const double bv = uh == 0 ? w[u & 3] : flip(w[u & 3], t.chi[g][uh - 1]);
                yh[l][u] += ah[g ^ u] * bv;
            }
        }
    }
    for (int g = 0; g < 16; ++g) {
        double w[4] = {yh[0][g], yh[1][g], yh[2][g], yh[3][g]};
        for (int h = 1; h < 4; h <<= 1)
            for (int c = 0; c < 4; ++c)
                if (!(c & h)) {
                    const double u0 = w[c], v0 = w[c | h];
                    w[c] = u0 + v0;
                    w[c | h] = u0 - v0;
                }
        for (int c = 0; c < 4; ++c) y[t.blade[g][c]] = flip(w[c], t.post[g][c]) * 0.25;
    }
}

}  // namespace geo
