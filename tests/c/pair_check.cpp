// Host check of the pairwise representation tables (geo::make_pair_tables):
// for every n = 6 signature whose representation has D = 16, S = 4, and every
// operand reversal, the table-driven product (geo::pair_product_host, the
// kernel's arithmetic) equals the direct product sum_{l,r} s(l, r) a_l b_r e_{l^r}
// (operand blade m multiplied by s(m, m) where reversed) to 1e-12.
#include <math.h>
#include <stdio.h>

#include <random>

#include "geo_internal.h"
#include "representation.h"

int main() {
    std::mt19937_64 gen(7);
    std::uniform_real_distribution<double> U(-1.0, 1.0);
    int cases = 0, skipped = 0, bad = 0;
    double worst = 0.0;
    for (int mask = 0; mask < 64; ++mask) {
        int8_t sig[6];
        for (int a = 0; a < 6; ++a) sig[a] = ((mask >> a) & 1) ? -1 : 1;
        geo::RepPlan rp;
        if (!geo::make_rep_plan(&rp, 6, sig, 0) || rp.D != 16) {
            ++skipped;
            continue;
        }
        for (int rev = 0; rev < 4; ++rev) {
            geo::PairTables t;
            if (!geo::make_pair_tables(rp, sig, rev & 1, rev & 2, &t)) {
                printf("tables failed: mask=%d rev=%d\n", mask, rev);
                ++bad;
                continue;
            }
            for (int trial = 0; trial < 20; ++trial) {
                double a[64], b[64], y[64], d[64] = {};
                for (int i = 0; i < 64; ++i) {
                    a[i] = U(gen);
                    b[i] = U(gen);
                }
                geo::pair_product_host(t, a, b, y);
                for (int l = 0; l < 64; ++l)
                    for (int r = 0; r < 64; ++r) {
                        double al = a[l], br = b[r];
                        if ((rev & 1) && geo::sign_rule((uint8_t)l, (uint8_t)l, sig, 6) < 0) al = -al;
                        if ((rev & 2) && geo::sign_rule((uint8_t)r, (uint8_t)r, sig, 6) < 0) br = -br;
                        d[l ^ r] += geo::sign_rule((uint8_t)l, (uint8_t)r, sig, 6) * al * br;
                    }
                for (int i = 0; i < 64; ++i) {
                    const double e = fabs(y[i] - d[i]);
                    if (e > worst) worst = e;
                    if (e > 1e-12 * (1.0 + fabs(d[i]))) ++bad;
                }
            }
            ++cases;
        }
    }
    printf("PAIR_CHECK: %s cases=%d skipped_signatures=%d worst=%.3g\n", bad ? "FAIL" : "PASS", cases, skipped, worst);
    return bad ? 1 : 0;
}
