// Host check of the Pauli-string representation search: for every canonical
// signature and both sides, the plan must exist for n >= 2, satisfy the
// Clifford relations (checked inside make_rep_plan) and reproduce the direct
// product y = x*W / W*x through X' W' and the scatter back.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "representation.h"
#include "geo_internal.h"
#include "rep_layout.h"

using namespace geo;

// 16 lanes of a half-warp hit 16 distinct double-banks (8-byte words mod 16).
static bool distinct_banks(const int *addr) {
    unsigned used = 0;
    for (int l = 0; l < 16; ++l) used |= 1u << (addr[l] & 15);
    return __builtin_popcount(used) == 16;
}

// Replays every shared-memory access of rep_ws_kernel<D, S> (producer raw
// reads and in-place writes, consumer fragment loads) per half-warp, and checks
// that the producers' writes cover each transformed entry exactly once.
template <int D, int S>
static const char *check_ws_layout(const RepDevice &dev) {
    using G = WsGeo<D, S>;
    constexpr int N = G::N;
    std::vector<int> hits(G::TILE, 0);
    for (int w = 0; w < kWsProducers / 32; ++w)
        for (int i = 0; i < G::PER; ++i)
            for (int h = 0; h < 2; ++h) {
                for (int t = 0; t < S; ++t) {
                    int rd[16], wr[16];
                    for (int l = 0; l < 16; ++l) {
                        const int tid = 32 * w + 16 * h + l;
                        const int m = tid % D, slot = tid / D;
                        const int L = D == 8 ? (slot & 1) * 8 + m : m;
                        const int sm = slot + G::SLOTS * i;
                        rd[l] = sm * N + dev.ws_blade[L][t];
                        const int r = dev.ws_out_row[L][t];  // transform output t goes to kept row r
                        wr[l] = ws_index<D>(sm * S + r, dev.grp_col[m][r]);
                        if (wr[l] < 0 || wr[l] >= G::TILE) return "write outside the tile";
                        hits[wr[l]] += 1;
                        // The kernel writes at sm * N + (offset computed for i = 0).
                        const int sm0 = slot;
                        if (wr[l] - sm * N != ws_index<D>(sm0 * S + r, dev.grp_col[m][r]) - sm0 * N)
                            return "write offset depends on the sample";
                    }
                    if (!distinct_banks(rd)) return "producer raw read conflicts";
                    if (!distinct_banks(wr)) return "producer write conflicts";
                }
            }
    for (int e = 0; e < G::TILE; ++e)
        if (hits[e] != 1) return "producer writes do not cover the tile once";
    for (int cw = 0; cw < 4; ++cw)
        for (int j = 0; j < G::GPW; ++j) {
            const int n0 = (cw * G::GPW + j) * 8;
            for (int h = 0; h < 2; ++h) {
                for (int kk = 0; kk < D / 4; ++kk) {
                    int a[16];
                    for (int l = 0; l < 16; ++l) {
                        const int lane = 16 * h + l, g = lane >> 2, t = lane & 3;
                        a[l] = ws_index<D>(n0 + g, 4 * kk + t);
                    }
                    if (!distinct_banks(a)) return "GEMM 1 operand conflicts";
                }
                for (int hh = 0; hh < 2; ++hh)
                    for (int off = 0; off < D; off += 8) {
                        int a[16];
                        for (int l = 0; l < 16; ++l) {
                            const int lane = 16 * h + l, g = lane >> 2, t = lane & 3;
                            a[l] = ws_index<D>(n0 + 2 * t + hh, g + off);
                        }
                        if (!distinct_banks(a)) return "epilogue / GEMM 2 operand conflicts";
                    }
                // The complex (3M) consumer of D = 16: GEMM 1 reads columns m = t + 4 kk and
                // m ^ 12 of row n0 + g; T' and GEMM 2 read columns g and g ^ 12 of rows n0 + 2 t + hh.
                for (int kk = 0; D == 16 && kk < 2; ++kk)
                    for (int pair = 0; pair < 2; ++pair) {
                        int a[16];
                        for (int l = 0; l < 16; ++l) {
                            const int lane = 16 * h + l, g = lane >> 2, t = lane & 3;
                            a[l] = ws_index<D>(n0 + g, (t + 4 * kk) ^ (pair ? 12 : 0));
                        }
                        if (!distinct_banks(a)) return "3M GEMM 1 operand conflicts";
                    }
                for (int hh = 0; D == 16 && hh < 2; ++hh)
                    for (int pair = 0; pair < 2; ++pair) {
                        int a[16];
                        for (int l = 0; l < 16; ++l) {
                            const int lane = 16 * h + l, g = lane >> 2, t = lane & 3;
                            a[l] = ws_index<D>(n0 + 2 * t + hh, g ^ (pair ? 12 : 0));
                        }
                        if (!distinct_banks(a)) return "3M T' / GEMM 2 operand conflicts";
                    }
            }
        }
    // rep_fwd_kernel: the consumers' Y' writes (the epilogue positions above)
    // cover every transformed entry of the tile exactly once.
    std::vector<int> ywrites(G::TILE, 0);
    for (int cw = 0; cw < 4; ++cw)
        for (int j = 0; j < G::GPW; ++j) {
            const int n0 = (cw * G::GPW + j) * 8;
            for (int lane = 0; lane < 32; ++lane)
                for (int hh = 0; hh < 2; ++hh)
                    for (int off = 0; off < D; off += 8) {
                        const int g = lane >> 2, t = lane & 3;
                        ywrites[ws_index<D>(n0 + 2 * t + hh, g + off)] += 1;
                    }
        }
    for (int e = 0; e < G::TILE; ++e)
        if (ywrites[e] != 1) return "forward Y' writes do not cover the tile once";
    return nullptr;
}

// The forward kernel's pipeline (rep_fwd_kernel, FwdPipe):
// producer iteration k issues the load of tile k + AHEAD (after waiting until
// at most STORE_PENDING bulk stores are pending), gathers tile k and scatters
// + stores tile k - LAG. Replays the order for many tile counts and checks that
// every load goes into a stage whose previous tile was already stored, and
// that the stores still pending at that moment are all later tiles.
static const char *check_forward_pipeline() {
    using P = FwdPipe;
    for (int K = 1; K <= 64; ++K) {
        std::vector<int> stored;  // tiles in store-issue order
        std::vector<bool> issued(K, false);
        for (int k = 0; k < K && k < P::AHEAD; ++k) issued[k] = true;  // prologue
        for (int k = 0; k < K + P::LAG; ++k) {
            if (k < K) {
                const int ahead = k + P::AHEAD;
                if (ahead < K) {
                    const int prev = ahead - P::STAGES;  // tile that last used the stage
                    if (prev >= 0) {
                        // wait_group.read STORE_PENDING: all but the newest STORE_PENDING stores are done
                        int pos = -1;
                        for (int i = 0; i < (int)stored.size(); ++i)
                            if (stored[i] == prev) pos = i;
                        if (pos < 0) return "stage reloaded before its store was issued";
                        if ((int)stored.size() - pos <= P::STORE_PENDING)
                            return "stage reloaded while its store may still read it";
                    }
                    issued[ahead] = true;
                }
                if (!issued[k]) return "tile gathered before its load was issued";
            }
            const int j = k - P::LAG;
            if (j >= 0 && j < K) stored.push_back(j);
        }
        if ((int)stored.size() != K) return "not every tile stored";
    }
    return nullptr;
}

// Replays the handoffs of the fused MSE-SGD kernel (SgdPipe) for every tile
// count up to 64 as two agents (the producer warps, with thread 0's loads and
// stores, and the consumer warps), each blocking exactly where the kernel
// waits. Two schedules are replayed: producers run as far as they can before
// the consumers move, and the reverse. Checks: no deadlock; every phase finds
// its stage holding its own tile (so no mbarrier phase of a stage is overtaken
// by a later tile before its wait); a stage is reloaded only after GEMM 2 of
// its previous tile and after the residual store reading it has been retired
// by wait_group.read (stores retire only when a wait forces them).
static const char *check_sgd_pipeline() {
    using P = SgdPipe;
    const int NST = P::STAGES;
    for (int K = 1; K <= 64; ++K) {
        for (int policy = 0; policy < 2; ++policy) {
            std::vector<int> issued(K, 0), full(K, 0), done(K, 0), resid(K, 0), freed(K, 0);
            std::vector<int> stores;  // tiles whose residual store may still read shared memory
            std::vector<int> stage_tile(NST, -1);
            int pk = 0, pphase = 0;   // producer iteration; phase 0 gather, 1 residual, 2 issue
            int ck = 0, cphase = 0;   // consumer iteration; phase 0 GEMM 1, 1 GEMM 2
            for (int k = 0; k < K && k < P::AHEAD; ++k) {
                issued[k] = 1;
                stage_tile[k % NST] = k;
            }
            auto owns = [&](int tile) { return stage_tile[tile % NST] == tile; };
            // 1 progressed, 0 blocked, -1 finished, -2 stage misuse
            auto producer_step = [&]() -> int {
                if (pk >= K + P::LAG) return -1;
                if (pphase == 0) {
                    if (pk < K) {
                        if (!issued[pk]) return 0;
                        if (!owns(pk)) return -2;
                        full[pk] = 1;
                    }
                    pphase = 1;
                    return 1;
                }
                if (pphase == 1) {
                    const int j = pk - P::LAG;
                    if (j >= 0) {
                        if (!done[j]) return 0;
                        if (!owns(j)) return -2;
                        resid[j] = 1;
                        stores.push_back(j);
                    }
                    pphase = 2;
                    return 1;
                }
                const int ahead = pk + P::AHEAD;
                if (ahead < K) {
                    const int prev = ahead - NST;
                    if (prev >= 0) {
                        if (!freed[prev]) return 0;
                        // wait_group.read STORE_PENDING retires all but the newest STORE_PENDING stores
                        while ((int)stores.size() > P::STORE_PENDING) stores.erase(stores.begin());
                        for (int s : stores)
                            if (s % NST == ahead % NST) return -2;  // a store still reads the stage
                    }
                    issued[ahead] = 1;
                    stage_tile[ahead % NST] = ahead;
                }
                ++pk;
                pphase = 0;
                return 1;
            };
            auto consumer_step = [&]() -> int {
                if (ck >= K + P::LAG) return -1;
                if (cphase == 0) {
                    if (ck < K) {
                        if (!full[ck]) return 0;
                        if (!owns(ck)) return -2;
                        done[ck] = 1;
                    }
                    cphase = 1;
                    return 1;
                }
                const int j = ck - P::LAG;
                if (j >= 0) {
                    if (!resid[j]) return 0;
                    if (!owns(j)) return -2;
                    freed[j] = 1;
                }
                ++ck;
                cphase = 0;
                return 1;
            };
            for (;;) {
                int a, b;
                if (policy == 0) {
                    while ((a = producer_step()) == 1) {}
                    b = consumer_step();
                } else {
                    while ((b = consumer_step()) == 1) {}
                    a = producer_step();
                }
                if (a == -2 || b == -2) return "a stage was used by a tile that does not own it";
                if (a == -1 && b == -1) break;
                if (a != 1 && b != 1) {
                    a = producer_step();
                    b = consumer_step();
                    if (a == -2 || b == -2) return "a stage was used by a tile that does not own it";
                    if (a == -1 && b == -1) break;
                    if (a != 1 && b != 1) return "deadlock";
                }
            }
            for (int k = 0; k < K; ++k)
                if (!freed[k] || !resid[k]) return "not every tile completed";
        }
    }
    return nullptr;
}

// Inverse butterfly of the forward kernel's scatter: from a group's kept
// entries back to its blades, y_t = in_sign_t * (1/S) * sum_f H[t][f] out_sign_f Y_f.
static bool check_scatter(const RepDevice &dev, const double *x, const double *Xp) {
    const int D = dev.D, S = dev.S;
    for (int L = 0; L < (D == 8 ? 16 : D); ++L) {
        const int m = L % D;
        double v[8];
        for (int f = 0; f < S; ++f) {
            const int r = dev.ws_out_row[L][f];
            const double e = Xp[r * D + dev.grp_col[m][r]];
            v[f] = ((dev.ws_out_neg[L] >> f) & 1) ? -e : e;
        }
        for (int hs = 1; hs < S; hs <<= 1)
            for (int a = 0; a < S; ++a)
                if (!(a & hs)) {
                    const double u = v[a], w = v[a | hs];
                    v[a] = u + w;
                    v[a | hs] = u - w;
                }
        for (int t = 0; t < S; ++t) {
            const double got = (((dev.ws_in_neg[L] >> t) & 1) ? -v[t] : v[t]) * (1.0 / S);
            if (std::fabs(got - x[dev.ws_blade[L][t]]) > 1e-12) return false;
        }
    }
    return true;
}

static const char *check_ws(const RepDevice &dev) {
    if (!dev.ws_ready) return nullptr;
    if (dev.D == 16 && dev.S == 4) return check_ws_layout<16, 4>(dev);
    if (dev.D == 16 && dev.S == 2) return check_ws_layout<16, 2>(dev);
    if (dev.D == 8 && dev.S == 8) return check_ws_layout<8, 8>(dev);
    if (dev.D == 8 && dev.S == 4) return check_ws_layout<8, 4>(dev);
    return nullptr;  // no warp-specialised kernel for this shape
}

int main() {
    std::mt19937_64 rng(5);
    std::uniform_real_distribution<double> U(-1.0, 1.0);
    int cases = 0;
    if (const char *why = check_forward_pipeline()) {
        printf("FAIL forward pipeline: %s\n", why);
        return 1;
    }
    if (const char *why = check_sgd_pipeline()) {
        printf("FAIL mse-sgd pipeline: %s\n", why);
        return 1;
    }
    for (int n = 1; n <= 6; ++n) {
        for (int q = 0; q <= n; ++q) {
            int8_t sig[6] = {0};
            for (int a = 0; a < n; ++a) sig[a] = a < n - q ? 1 : -1;
            for (int side = 0; side <= 1; ++side) {
                RepPlan p;
                if (!make_rep_plan(&p, (uint8_t)n, sig, side)) {
                    if (n >= 2) { printf("FAIL no plan n=%d q=%d side=%d\n", n, q, side); return 1; }
                    continue;
                }
                const int N = 1 << n, D = p.D, S = p.S;
                double x[64], w[64], y_ref[64], Wp[16][16], Xp[64], Yp[64], y[64];
                for (int i = 0; i < N; ++i) { x[i] = U(rng); w[i] = U(rng); }
                for (int o = 0; o < N; ++o) {
                    double acc = 0;
                    for (int i = 0; i < N; ++i) {
                        const int pb = i ^ o;
                        const int s = side ? sign_rule((uint8_t)pb, (uint8_t)i, sig, (uint8_t)n)
                                           : sign_rule((uint8_t)i, (uint8_t)pb, sig, (uint8_t)n);
                        acc += x[i] * w[pb] * s;
                    }
                    y_ref[o] = acc;
                }
                // W' = rho(W) (right) or rho(W)^T (left)
                for (int k = 0; k < D; ++k)
                    for (int j = 0; j < D; ++j) {
                        double acc = 0;
                        for (int A = 0; A < N; ++A)
                            acc += w[A] * (side ? rep_entry(p, A, j, k) : rep_entry(p, A, k, j));
                        Wp[k][j] = acc;
                    }
                for (int e = 0; e < N; ++e) {
                    double acc = 0;
                    for (int t = 0; t < p.c; ++t) acc += p.gs[e][t] * x[p.gb[e][t]];
                    Xp[e] = acc;
                }
                for (int r = 0; r < S; ++r)
                    for (int j = 0; j < D; ++j) {
                        double acc = 0;
                        for (int k = 0; k < D; ++k) acc += Xp[r * D + k] * Wp[k][j];
                        Yp[r * D + j] = acc;
                    }
                for (int A = 0; A < N; ++A) y[A] = 0;
                for (int e = 0; e < N; ++e)
                    for (int t = 0; t < p.c; ++t) y[p.gb[e][t]] += p.gs[e][t] * Yp[e] / S;
                double err = 0;
                for (int o = 0; o < N; ++o) err = std::fmax(err, std::fabs(y[o] - y_ref[o]));
                if (err > 1e-12) { printf("FAIL n=%d q=%d side=%d err=%g\n", n, q, side, err); return 1; }
                RepDevice dev;
                if (!make_rep_device(&dev, p)) { printf("FAIL device tables n=%d q=%d side=%d\n", n, q, side); return 1; }
                // Grouped gather == entry gather, and every warp load step hits distinct bank classes.
                double Xg[64] = {0};
                for (int m = 0; m < D; ++m)
                    for (int r = 0; r < S; ++r) {
                        double acc = 0;
                        for (int t = 0; t < S; ++t) {
                            const double v = x[dev.grp_blade[m][t]];
                            acc += ((dev.grp_neg[m] >> (r * 8 + t)) & 1) ? -v : v;
                        }
                        Xg[r * D + dev.grp_col[m][r]] = acc;
                    }
                for (int e = 0; e < N; ++e)
                    if (std::fabs(Xg[e] - Xp[e]) > 1e-12) { printf("FAIL grouped gather n=%d q=%d\n", n, q); return 1; }
                const int mod = D >= 16 ? 16 : 8;
                for (int t = 0; t < S; ++t) {
                    unsigned used = 0;
                    for (int m = 0; m < D; ++m) used |= 1u << (dev.grp_blade[m][t] % mod);
                    if (__builtin_popcount(used) != D) { printf("FAIL bank classes n=%d q=%d\n", n, q); return 1; }
                }
                // The warp-specialised kernel's butterfly gather gives the same entries.
                if (((D == 8 && S >= 4) || (D == 16 && S >= 2)) && !dev.ws_ready) {
                    printf("FAIL no butterfly tables n=%d q=%d side=%d\n", n, q, side);
                    return 1;
                }
                for (int L = 0; dev.ws_ready && L < (D == 8 ? 16 : D); ++L) {
                    const int m = L % D;
                    double w[8];
                    for (int t = 0; t < S; ++t) {
                        const double v = x[dev.ws_blade[L][t]];
                        w[t] = ((dev.ws_in_neg[L] >> t) & 1) ? -v : v;
                    }
                    for (int hs = 1; hs < S; hs <<= 1)
                        for (int a = 0; a < S; ++a)
                            if (!(a & hs)) {
                                const double u = w[a], v = w[a | hs];
                                w[a] = u + v;
                                w[a | hs] = u - v;
                            }
                    for (int f = 0; f < S; ++f) {
                        const int r = dev.ws_out_row[L][f];
                        const double got = ((dev.ws_out_neg[L] >> f) & 1) ? -w[f] : w[f];
                        if (std::fabs(got - Xp[r * D + dev.grp_col[m][r]]) > 1e-12) {
                            printf("FAIL ws butterfly n=%d q=%d side=%d\n", n, q, side);
                            return 1;
                        }
                    }
                }
                if (const char *why = check_ws(dev)) {
                    printf("FAIL ws layout n=%d q=%d side=%d: %s\n", n, q, side, why);
                    return 1;
                }
                if (dev.ws_ready && !check_scatter(dev, x, Xp)) {
                    printf("FAIL forward scatter n=%d q=%d side=%d\n", n, q, side);
                    return 1;
                }
                printf("n=%d q=%d side=%d D=%d S=%d err=%.1e\n", n, q, side, D, S, err);
                ++cases;
            }
        }
    }
    printf("REP_CHECK: PASS cases=%d\n", cases);
    return 0;
}
