/*
 * geo/operator_kernel.h -- constants, status codes and value types shared by the
 * batched geometric-product path.
 *
 * Drop-in for the reference header include/geo/operator_kernel.h. The type
 * layouts (geo_operator_term_i32_t, geo_operator_plan_i32_t,
 * geo_operator_mv_f64_t, geo_operator_mv_i32_t), the enum values and the
 * macros must match it byte for byte, because C callers allocate these types
 * themselves and hand them across the ABI. tests/c/abi_layout.c pins every
 * offset with _Static_assert.
 *
 * Exported here (host side, integer plan logic, bit-exact with the reference):
 *   geo_operator_abi_version          reference src/operator_kernel.c:98-100
 *   geo_operator_gradient_abi_version reference src/operator_kernel.c:102-104
 *   geo_operator_blade_count          reference src/operator_kernel.c:106-109
 *   geo_operator_gp_sign              reference src/operator_kernel.c:111-135
 *   geo_operator_plan_fixed_blade_i32 reference src/operator_kernel.c:137-149
 *   geo_operator_plan_sparse_i32      reference src/operator_kernel.c:151-189
 *
 * Exported here (per-multivector float64 arithmetic, computed on the GPU by
 * one small launch per call on the caller's current device, bit-identical to
 * the reference; synchronous, like the reference):
 *   geo_operator_apply_f64                 reference src/operator_kernel.c:191-220
 *   geo_operator_apply_parametric_f64      reference src/operator_kernel.c:222-254
 *   geo_operator_apply_f64_vjp             reference src/operator_kernel.c:256-278
 *   geo_operator_apply_parametric_f64_vjp  reference src/operator_kernel.c:280-334
 *   geo_operator_gp_f64                    reference src/operator_kernel.c:412-447
 *   geo_operator_gp_f64_jvp                reference src/operator_kernel.c:449-492
 *   geo_operator_gp_f64_vjp                reference src/operator_kernel.c:494-539
 * Their statuses are the reference's, plus GEO_OPERATOR_B200_DEVICE_FAILURE
 * (geo/geo_b200.h) when the GPU call itself fails. The batched,
 * device-resident forms are in geo/geo_b200.h (geo_b200_pairwise_*,
 * geo_b200_sparse_*). The modular and Q-format integer paths of the
 * reference (geo_operator_apply_mod_i32, geo_operator_apply_q_i32) are
 * embedded-only and are not part of this library.
 */
#ifndef GEO_OPERATOR_KERNEL_H
#define GEO_OPERATOR_KERNEL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GEO_OPERATOR_MAX_DIMENSION 6u
#define GEO_OPERATOR_MAX_BLADES 64u
#define GEO_OPERATOR_MAX_TERMS 64u
#define GEO_OPERATOR_ABI_VERSION 0x00050100u
#define GEO_OPERATOR_GRADIENT_ABI_VERSION 0x00010000u

typedef enum {
    GEO_OPERATOR_OK = 0,
    GEO_OPERATOR_INVALID_ARGUMENT = 1,
    GEO_OPERATOR_UNSUPPORTED_DIMENSION = 2,
    GEO_OPERATOR_TOO_MANY_TERMS = 3,
    GEO_OPERATOR_ZERO_MODULUS = 4,
    GEO_OPERATOR_OVERFLOW = 5,
    GEO_OPERATOR_BAD_PLAN = 6
} geo_operator_status_t;

typedef enum {
    GEO_OPERATOR_SIDE_RIGHT = 0,
    GEO_OPERATOR_SIDE_LEFT = 1
} geo_operator_side_t;

typedef enum {
    GEO_OPERATOR_PLAN_FIXED_BLADE = 1,
    GEO_OPERATOR_PLAN_SPARSE_FIXED_MULTIVECTOR = 2
} geo_operator_plan_kind_t;

/* One (blade, integer coefficient) term of a fixed multivector. */
typedef struct {
    uint8_t blade;
    int32_t coefficient;
} geo_operator_term_i32_t;

/* Fixed-blade or sparse fixed-multivector operator plan (one side). */
typedef struct {
    uint32_t abi_version;
    uint8_t dimension;
    int8_t signature[GEO_OPERATOR_MAX_DIMENSION];
    uint8_t kind;
    uint8_t side;
    uint8_t term_count;
    uint8_t reserved;
    geo_operator_term_i32_t terms[GEO_OPERATOR_MAX_TERMS];
} geo_operator_plan_i32_t;

/* Dense multivector: coefficient k belongs to the blade whose axis bitmask is k. */
typedef struct {
    uint8_t dimension;
    int8_t signature[GEO_OPERATOR_MAX_DIMENSION];
    double coefficients[GEO_OPERATOR_MAX_BLADES];
} geo_operator_mv_f64_t;

typedef struct {
    uint8_t dimension;
    int8_t signature[GEO_OPERATOR_MAX_DIMENSION];
    int32_t coefficients[GEO_OPERATOR_MAX_BLADES];
} geo_operator_mv_i32_t;

uint32_t geo_operator_abi_version(void);
uint32_t geo_operator_gradient_abi_version(void);

/* 2^dimension for dimension in 1..6, else 0. */
size_t geo_operator_blade_count(uint8_t dimension);

/*
 * Sign s in e_left * e_right = s * e_(left XOR right) for the diagonal metric
 * `signature` (entries +1/-1). Returns 0 when the signature is invalid.
 */
int geo_operator_gp_sign(
    uint8_t left_blade,
    uint8_t right_blade,
    const int8_t *signature,
    uint8_t dimension
);

geo_operator_status_t geo_operator_plan_fixed_blade_i32(
    geo_operator_plan_i32_t *plan,
    uint8_t dimension,
    const int8_t *signature,
    geo_operator_side_t side,
    uint8_t blade,
    int32_t coefficient
);

geo_operator_status_t geo_operator_plan_sparse_i32(
    geo_operator_plan_i32_t *plan,
    uint8_t dimension,
    const int8_t *signature,
    geo_operator_side_t side,
    const geo_operator_term_i32_t *terms,
    size_t term_count
);

/* output = input * plan (right side) or plan * input (left side). */
geo_operator_status_t geo_operator_apply_f64(
    const geo_operator_plan_i32_t *plan,
    const geo_operator_mv_f64_t *input,
    geo_operator_mv_f64_t *output
);

/* As geo_operator_apply_f64 with parameters[i] in place of the plan's integer
 * coefficient of term i (parameter_count must equal the term count). */
geo_operator_status_t geo_operator_apply_parametric_f64(
    const geo_operator_plan_i32_t *plan,
    const double *parameters,
    size_t parameter_count,
    const geo_operator_mv_f64_t *input,
    geo_operator_mv_f64_t *output
);

/* input_cotangent = M^T output_cotangent for the plan's operator M. */
geo_operator_status_t geo_operator_apply_f64_vjp(
    const geo_operator_plan_i32_t *plan,
    const geo_operator_mv_f64_t *output_cotangent,
    geo_operator_mv_f64_t *input_cotangent
);

/* Cotangents of the input and of every parameter of the parametric apply. */
geo_operator_status_t geo_operator_apply_parametric_f64_vjp(
    const geo_operator_plan_i32_t *plan,
    const double *parameters,
    size_t parameter_count,
    const geo_operator_mv_f64_t *input,
    const geo_operator_mv_f64_t *output_cotangent,
    geo_operator_mv_f64_t *input_cotangent,
    double *parameter_cotangents,
    size_t parameter_cotangent_count
);

/* output = left * right (dense geometric product; zero left coefficients are skipped). */
geo_operator_status_t geo_operator_gp_f64(
    const geo_operator_mv_f64_t *left,
    const geo_operator_mv_f64_t *right,
    geo_operator_mv_f64_t *output
);

/* Forward-mode derivative: output_tangent = left_tangent * right + left * right_tangent. */
geo_operator_status_t geo_operator_gp_f64_jvp(
    const geo_operator_mv_f64_t *left,
    const geo_operator_mv_f64_t *right,
    const geo_operator_mv_f64_t *left_tangent,
    const geo_operator_mv_f64_t *right_tangent,
    geo_operator_mv_f64_t *output_tangent
);

/* Reverse-mode derivative of the geometric product (the two outputs must differ). */
geo_operator_status_t geo_operator_gp_f64_vjp(
    const geo_operator_mv_f64_t *left,
    const geo_operator_mv_f64_t *right,
    const geo_operator_mv_f64_t *output_cotangent,
    geo_operator_mv_f64_t *left_cotangent,
    geo_operator_mv_f64_t *right_cotangent
);

#ifdef __cplusplus
}
#endif

#endif
