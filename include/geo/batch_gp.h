/*
 * geo/batch_gp.h -- batched geometric product, host-pointer API.
 *
 * Drop-in for the reference header include/geo/batch_gp.h (ABI 0x00010000).
 * Same symbols, same plan struct, same status codes, same argument meaning:
 *
 *   geo_batch_gp_abi_version              reference src/batch_gp.c:65-67
 *   geo_batch_gp_plan_init                reference src/batch_gp.c:69-105
 *   geo_batch_gp_{right,left}_forward_f64 reference src/batch_gp.c:107-161
 *   geo_batch_gp_{right,left}_vjp_parameter_f64
 *                                         reference src/batch_gp.c:163-235
 *   geo_batch_gp_{right,left}_mse_sgd_step_f64
 *                                         reference src/batch_gp.c:237-350
 *
 * What changes behind the symbols: the arithmetic runs on the current CUDA
 * device. Arrays may be pageable host memory (staged through pinned buffers
 * in pipelined chunks), pinned host memory (copied asynchronously) or device
 * memory (used in place). Every call is synchronous, like the reference, and
 * outputs are overwritten, not accumulated.
 *
 * Status semantics follow the reference exactly: non-finite inputs or
 * parameters give GEO_BATCH_GP_INVALID_ARGUMENT with outputs untouched;
 * non-finite results give GEO_BATCH_GP_NUMERIC_FAILURE; the SGD step leaves
 * the parameter unchanged unless every candidate coefficient is finite.
 * Floating-point results agree with the reference to 1e-12 relative
 * (|a-b| <= 1e-12 (1+|a|+|b|)); the summation order differs.
 */
#ifndef GEO_BATCH_GP_H
#define GEO_BATCH_GP_H

#include "geo/operator_kernel.h"

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GEO_BATCH_GP_ABI_VERSION 0x00010000u
#define GEO_BATCH_GP_MAX_TERMS (GEO_OPERATOR_MAX_BLADES * GEO_OPERATOR_MAX_BLADES)

typedef enum {
    GEO_BATCH_GP_OK = 0,
    GEO_BATCH_GP_INVALID_ARGUMENT = 1,
    GEO_BATCH_GP_UNSUPPORTED_DIMENSION = 2,
    GEO_BATCH_GP_NUMERIC_FAILURE = 3
} geo_batch_gp_status_t;

/*
 * All 4^n (left, right) blade pairs in lexicographic order with their output
 * blade left^right and sign. Caller-owned; 16400 bytes.
 */
typedef struct {
    uint32_t abi_version;
    uint8_t dimension;
    int8_t signature[GEO_OPERATOR_MAX_DIMENSION];
    uint16_t blade_count;
    uint16_t term_count;
    uint8_t left_blade[GEO_BATCH_GP_MAX_TERMS];
    uint8_t right_blade[GEO_BATCH_GP_MAX_TERMS];
    uint8_t output_blade[GEO_BATCH_GP_MAX_TERMS];
    int8_t sign[GEO_BATCH_GP_MAX_TERMS];
} geo_batch_gp_plan_t;

uint32_t geo_batch_gp_abi_version(void);

geo_batch_gp_status_t geo_batch_gp_plan_init(
    geo_batch_gp_plan_t *plan,
    uint8_t dimension,
    const int8_t *signature
);

/* outputs[s] = inputs[s] * right_parameter for every sample s. */
geo_batch_gp_status_t geo_batch_gp_right_forward_f64(
    const geo_batch_gp_plan_t *plan,
    const double *inputs,
    size_t batch_size,
    const double *right_parameter,
    double *outputs
);

/* outputs[s] = left_parameter * inputs[s] for every sample s. */
geo_batch_gp_status_t geo_batch_gp_left_forward_f64(
    const geo_batch_gp_plan_t *plan,
    const double *left_parameter,
    const double *inputs,
    size_t batch_size,
    double *outputs
);

/* parameter_cotangent = sum over samples of d<outputs, cotangents>/d(parameter). */
geo_batch_gp_status_t geo_batch_gp_right_vjp_parameter_f64(
    const geo_batch_gp_plan_t *plan,
    const double *inputs,
    const double *output_cotangents,
    size_t batch_size,
    double *parameter_cotangent
);

geo_batch_gp_status_t geo_batch_gp_left_vjp_parameter_f64(
    const geo_batch_gp_plan_t *plan,
    const double *inputs,
    const double *output_cotangents,
    size_t batch_size,
    double *parameter_cotangent
);

/*
 * One step of w -= learning_rate * grad / batch_size on the loss
 * sum_s 0.5 |x_s * w - t_s|^2; mean_loss = loss / batch_size.
 */
geo_batch_gp_status_t geo_batch_gp_right_mse_sgd_step_f64(
    const geo_batch_gp_plan_t *plan,
    const double *inputs,
    const double *targets,
    size_t batch_size,
    double learning_rate,
    double *right_parameter,
    double *mean_loss
);

geo_batch_gp_status_t geo_batch_gp_left_mse_sgd_step_f64(
    const geo_batch_gp_plan_t *plan,
    const double *inputs,
    const double *targets,
    size_t batch_size,
    double learning_rate,
    double *left_parameter,
    double *mean_loss
);

#ifdef __cplusplus
}
#endif

#endif
