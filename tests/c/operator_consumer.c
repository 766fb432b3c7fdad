/*
 * A C11 caller of the reference's per-multivector operator calls
 * (reference include/geo/operator_kernel.h): every geo_operator_*_f64 symbol,
 * resolved from libgeo_b200.so (GPU), compared bit for bit with the oracle's
 * restatement of the reference (oracle/liboracle.so, orc_* symbols) on every
 * canonical signature. Prints GEO_B200_OPERATOR_CONSUMER: PASS on success.
 */
#include <stdio.h>
#include <string.h>

#include "geo/operator_kernel.h"
#include "geo_oracle.h"

#define CHECK(c) do { if (!(c)) { fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #c); return 1; } } while (0)

static double value(unsigned seed, unsigned k) {
    unsigned h = (seed * 2654435761u) ^ (k * 40503u + 977u);
    h ^= h >> 13;
    h *= 0x5bd1e995u;
    h ^= h >> 15;
    return (double)((int)(h % 2001u) - 1000) / 997.0;
}

static void fill(geo_operator_mv_f64_t *v, uint8_t n, const int8_t *sig, unsigned seed) {
    unsigned k;
    memset(v, 0, sizeof(*v));
    v->dimension = n;
    memcpy(v->signature, sig, n);
    for (k = 0; k < (1u << n); ++k) v->coefficients[k] = value(seed, k);
}

static int same(const double *a, const double *b, unsigned count) { return memcmp(a, b, count * sizeof(double)) == 0; }

int main(void) {
    unsigned n, q;
    for (n = 1; n <= 6; ++n) {
        for (q = 0; q <= n; ++q) {
            int8_t sig[6];
            unsigned i, N = 1u << n;
            geo_operator_mv_f64_t a, b, c, d, out, out2;
            double want[64], want2[64];
            for (i = 0; i < n; ++i) sig[i] = (int8_t)(i < n - q ? 1 : -1);
            fill(&a, (uint8_t)n, sig, 11 + n + 7 * q);
            fill(&b, (uint8_t)n, sig, 23 + n + 7 * q);
            fill(&c, (uint8_t)n, sig, 37 + n + 7 * q);
            fill(&d, (uint8_t)n, sig, 41 + n + 7 * q);
            a.coefficients[0] = 0.0; /* a skipped left coefficient */
            CHECK(geo_operator_gp_f64(&a, &b, &out) == GEO_OPERATOR_OK);
            CHECK(orc_gp_f64((uint8_t)n, sig, a.coefficients, b.coefficients, want) == 0);
            CHECK(same(out.coefficients, want, N) && out.dimension == n);
            CHECK(geo_operator_gp_f64_jvp(&a, &b, &c, &d, &out) == GEO_OPERATOR_OK);
            CHECK(orc_gp_f64_jvp((uint8_t)n, sig, a.coefficients, b.coefficients, c.coefficients, d.coefficients,
                                 want) == 0);
            CHECK(same(out.coefficients, want, N));
            CHECK(geo_operator_gp_f64_vjp(&a, &b, &c, &out, &out2) == GEO_OPERATOR_OK);
            CHECK(orc_gp_f64_vjp((uint8_t)n, sig, a.coefficients, b.coefficients, c.coefficients, want, want2) == 0);
            CHECK(same(out.coefficients, want, N) && same(out2.coefficients, want2, N));
            {
                geo_operator_plan_i32_t plan;
                geo_operator_term_i32_t terms[3];
                uint8_t blades[3];
                int32_t coeffs[3];
                double params[3] = {0.5, -1.25, 2.0}, pc[3], wpc[3];
                unsigned t, count = N >= 3 ? 3 : N, side;
                for (t = 0; t < count; ++t) {
                    blades[t] = (uint8_t)((t * 5 + q) % N);
                    coeffs[t] = (int32_t)t * 2 - 3;
                    terms[t].blade = blades[t];
                    terms[t].coefficient = coeffs[t];
                }
                for (side = 0; side < 2; ++side) {
                    CHECK(geo_operator_plan_sparse_i32(&plan, (uint8_t)n, sig, (geo_operator_side_t)side, terms,
                                                       count) == GEO_OPERATOR_OK);
                    CHECK(geo_operator_apply_f64(&plan, &b, &out) == GEO_OPERATOR_OK);
                    CHECK(orc_sparse_apply((uint8_t)n, sig, (int)side, blades, coeffs, count, b.coefficients,
                                           want) == 0);
                    CHECK(same(out.coefficients, want, N));
                    CHECK(geo_operator_apply_parametric_f64(&plan, params, count, &b, &out) == GEO_OPERATOR_OK);
                    CHECK(orc_sparse_apply_parametric((uint8_t)n, sig, (int)side, blades, params, count,
                                                      b.coefficients, want) == 0);
                    CHECK(same(out.coefficients, want, N));
                    CHECK(geo_operator_apply_f64_vjp(&plan, &c, &out) == GEO_OPERATOR_OK);
                    CHECK(orc_sparse_apply_vjp((uint8_t)n, sig, (int)side, blades, coeffs, count, c.coefficients,
                                               want) == 0);
                    CHECK(same(out.coefficients, want, N));
                    CHECK(geo_operator_apply_parametric_f64_vjp(&plan, params, count, &b, &c, &out, pc, count) ==
                          GEO_OPERATOR_OK);
                    CHECK(orc_sparse_apply_parametric_vjp((uint8_t)n, sig, (int)side, blades, params, count,
                                                          b.coefficients, c.coefficients, want, wpc) == 0);
                    CHECK(same(out.coefficients, want, N) && same(pc, wpc, count));
                }
            }
        }
    }
    puts("GEO_B200_OPERATOR_CONSUMER: PASS");
    return 0;
}
