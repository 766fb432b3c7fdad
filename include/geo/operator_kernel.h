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
 * The per-multivector arithmetic of the reference (geo_operator_gp_f64, its
 * JVP/VJP, geo_operator_apply_*_f64 and their VJPs) is provided in batched,
 * device-resident form by geo/geo_b200.h (geo_b200_pairwise_*,
 * geo_b200_sparse_*). The modular and Q-format integer paths of the
 * reference are embedded-only and are not part of this library.
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

#ifdef __cplusplus
}
#endif

#endif
