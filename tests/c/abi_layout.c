/*
 * Layout pins for the public headers: every caller-owned struct must keep the
 * reference's byte layout (reference include/geo/batch_gp.h:23-33,
 * include/geo/batch_gp_cuda.h:23-34, include/geo/operator_kernel.h:37-63).
 * Compiled with -std=c11; a failing _Static_assert fails the build.
 */
#include <stddef.h>
#include <stdio.h>

#include "geo/batch_gp.h"
#include "geo/batch_gp_cuda.h"
#include "geo/geo_b200.h"
#include "geo/hand_cuda_comparator.h"
#include "geo/operator_kernel.h"

_Static_assert(sizeof(geo_batch_gp_plan_t) == 16400, "batch plan size");
_Static_assert(offsetof(geo_batch_gp_plan_t, dimension) == 4, "dimension");
_Static_assert(offsetof(geo_batch_gp_plan_t, signature) == 5, "signature");
_Static_assert(offsetof(geo_batch_gp_plan_t, blade_count) == 12, "blade_count");
_Static_assert(offsetof(geo_batch_gp_plan_t, term_count) == 14, "term_count");
_Static_assert(offsetof(geo_batch_gp_plan_t, left_blade) == 16, "left_blade");
_Static_assert(offsetof(geo_batch_gp_plan_t, right_blade) == 4112, "right_blade");
_Static_assert(offsetof(geo_batch_gp_plan_t, output_blade) == 8208, "output_blade");
_Static_assert(offsetof(geo_batch_gp_plan_t, sign) == 12304, "sign");
_Static_assert(sizeof(geo_batch_gp_cuda_plan_t) == 56, "cuda plan size");
_Static_assert(offsetof(geo_batch_gp_cuda_plan_t, blade_count) == 4, "cuda blade_count");
_Static_assert(offsetof(geo_batch_gp_cuda_plan_t, term_count) == 6, "cuda term_count");
_Static_assert(offsetof(geo_batch_gp_cuda_plan_t, dimension) == 8, "cuda dimension");
_Static_assert(offsetof(geo_batch_gp_cuda_plan_t, signature) == 9, "cuda signature");
_Static_assert(offsetof(geo_batch_gp_cuda_plan_t, device_signature) == 16, "device_signature");
_Static_assert(offsetof(geo_batch_gp_cuda_plan_t, device_sign) == 48, "device_sign");
_Static_assert(sizeof(geo_operator_term_i32_t) == 8, "term size");
_Static_assert(sizeof(geo_operator_plan_i32_t) == 528, "operator plan size");
_Static_assert(offsetof(geo_operator_plan_i32_t, kind) == 11, "kind");
_Static_assert(offsetof(geo_operator_plan_i32_t, terms) == 16, "terms");
_Static_assert(sizeof(geo_operator_mv_f64_t) == 520, "mv f64 size");
_Static_assert(offsetof(geo_operator_mv_f64_t, coefficients) == 8, "mv coefficients");
_Static_assert(sizeof(geo_operator_mv_i32_t) == 264, "mv i32 size");
_Static_assert(GEO_BATCH_GP_ABI_VERSION == 0x00010000u, "batch abi");
_Static_assert(GEO_BATCH_GP_CUDA_ABI_VERSION == 0x00010001u, "cuda abi");
_Static_assert(GEO_OPERATOR_ABI_VERSION == 0x00050100u, "operator abi");
_Static_assert(GEO_BATCH_GP_NUMERIC_FAILURE == 3 && GEO_BATCH_GP_CUDA_NUMERIC_FAILURE == 4, "status values");

int main(void) {
    printf("%zu %zu %zu %zu\n", sizeof(geo_batch_gp_plan_t), sizeof(geo_batch_gp_cuda_plan_t),
           sizeof(geo_operator_plan_i32_t), sizeof(geo_operator_mv_f64_t));
    return 0;
}
