// Host check of the Pauli-string representation search: for every canonical
// signature and both sides, the plan must exist for n >= 2, satisfy the
// Clifford relations (checked inside make_rep_plan) and reproduce the direct
// product y = x*W / W*x through X' W' and the scatter back.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>

#include "representation.h"
#include "geo_internal.h"

using namespace geo;

int main() {
    std::mt19937_64 rng(5);
    std::uniform_real_distribution<double> U(-1.0, 1.0);
    int cases = 0;
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
                printf("n=%d q=%d side=%d D=%d S=%d err=%.1e\n", n, q, side, D, S, err);
                ++cases;
            }
        }
    }
    printf("REP_CHECK: PASS cases=%d\n", cases);
    return 0;
}
