/*
 * A C11 program that uses the library exactly as it would use the reference:
 * plan_init + the host-pointer batch API (reference include/geo/batch_gp.h),
 * then the additive trainer. Built and linked on any machine; run on a GPU.
 * Prints GEO_B200_CONSUMER: PASS on success.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

#include "geo/batch_gp.h"
#include "geo/geo_b200.h"

#define CHECK(c) do { if (!(c)) { fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #c); return 1; } } while (0)

int main(void) {
    const int8_t sig[6] = {1, 1, 1, -1, -1, -1};
    geo_batch_gp_plan_t plan;
    enum { B = 1000, N = 64 };
    static double x[B * N], y[B * N], t[B * N];
    double w[N], g[N], w2[N], loss = -1.0;
    size_t i;
    CHECK(geo_batch_gp_abi_version() == GEO_BATCH_GP_ABI_VERSION);
    CHECK(geo_batch_gp_plan_init(&plan, 6, sig) == GEO_BATCH_GP_OK);
    for (i = 0; i < B * N; ++i) x[i] = (double)((int)(i * 7919u % 2001u) - 1000) / 1000.0;
    for (i = 0; i < N; ++i) w[i] = w2[i] = (double)((int)(i * 31u % 17u) - 8) / 16.0;
    CHECK(geo_batch_gp_right_forward_f64(&plan, x, B, w, y) == GEO_BATCH_GP_OK);
    for (i = 0; i < B * N; ++i) t[i] = y[i];
    CHECK(geo_batch_gp_right_vjp_parameter_f64(&plan, x, y, B, g) == GEO_BATCH_GP_OK);
    CHECK(geo_batch_gp_right_mse_sgd_step_f64(&plan, x, t, B, 0.01, w2, &loss) == GEO_BATCH_GP_OK);
    CHECK(loss == 0.0);
    for (i = 0; i < N; ++i) CHECK(w2[i] == w[i]);
    {
        geo_b200_trainer_t *tr = NULL;
        geo_b200_optimizer_config_t cfg = {GEO_B200_OPTIMIZER_ADAM, 1e-3, 0.9, 0.999, 1e-8};
        double ls = -1.0;
        CHECK(geo_b200_trainer_create(&tr, 6, sig, 0, w, &cfg) == GEO_B200_OK);
        CHECK(geo_b200_trainer_step_host(tr, x, t, B, 1.0 / B, &ls) == GEO_B200_OK);
        /* targets are this library's own forward outputs: the loss is rounding-level */
        CHECK(ls >= 0.0 && ls < 1e-20 * B);
        geo_b200_trainer_destroy(tr);
    }
    puts("GEO_B200_CONSUMER: PASS");
    return 0;
}
