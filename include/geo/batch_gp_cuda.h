/*
 * geo/batch_gp_cuda.h -- batched geometric product, device-pointer API.
 *
 * Drop-in for the reference header include/geo/batch_gp_cuda.h
 * (ABI 0x00010001). Same symbols, same plan struct layout, same status codes:
 *
 *   geo_batch_gp_cuda_abi_version          reference src/batch_gp_cuda.cu:200-202
 *   geo_batch_gp_cuda_plan_upload/destroy  reference src/batch_gp_cuda.cu:204-250
 *   geo_batch_gp_cuda_{reference_,planned_}forward_f64
 *                                          reference src/batch_gp_cuda.cu:252-286
 *   geo_batch_gp_cuda_{reference_,}parameter_vjp_f64
 *                                          reference src/batch_gp_cuda.cu:288-320
 *   geo_batch_gp_cuda_{reference_,}mse_sgd_step_f64
 *                                          reference src/batch_gp_cuda.cu:322-354
 *   geo_batch_gp_cuda_status_string        reference src/batch_gp_cuda.cu:356-365
 *
 * All compute calls take device pointers, are asynchronous on `stream`, and
 * return only host-side argument and launch status, as in the reference.
 * `device_loss` receives the SUM of 0.5 r^2 over the batch (not the mean) and
 * `device_residuals` receives r = x*w - t (or w*x - t), as in the reference.
 * The "reference_" and "planned" variants are kept as separate symbols for
 * source compatibility; both run this library's sm_100a kernels.
 *
 * The library owns the plan's device arrays. Besides the reference's
 * signature/left/right/output/sign arrays (same contents), the same
 * allocation holds this library's baked tables and a reduction scratch area,
 * so calls that share one plan must be ordered on one stream (or use one
 * plan per stream).
 */
#ifndef GEO_BATCH_GP_CUDA_H
#define GEO_BATCH_GP_CUDA_H

#include "geo/batch_gp.h"
#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GEO_BATCH_GP_CUDA_ABI_VERSION 0x00010001u

typedef enum {
    GEO_BATCH_GP_CUDA_OK = 0,
    GEO_BATCH_GP_CUDA_INVALID_ARGUMENT = 1,
    GEO_BATCH_GP_CUDA_ALLOCATION_FAILURE = 2,
    GEO_BATCH_GP_CUDA_RUNTIME_FAILURE = 3,
    GEO_BATCH_GP_CUDA_NUMERIC_FAILURE = 4
} geo_batch_gp_cuda_status_t;

typedef struct {
    uint32_t abi_version;
    uint16_t blade_count;
    uint16_t term_count;
    uint8_t dimension;
    int8_t signature[GEO_OPERATOR_MAX_DIMENSION];
    int8_t *device_signature;
    uint8_t *device_left_blade;
    uint8_t *device_right_blade;
    uint8_t *device_output_blade;
    int8_t *device_sign;
} geo_batch_gp_cuda_plan_t;

uint32_t geo_batch_gp_cuda_abi_version(void);
geo_batch_gp_cuda_status_t geo_batch_gp_cuda_plan_upload(geo_batch_gp_cuda_plan_t *device_plan, const geo_batch_gp_plan_t *host_plan);
void geo_batch_gp_cuda_plan_destroy(geo_batch_gp_cuda_plan_t *plan);
geo_batch_gp_cuda_status_t geo_batch_gp_cuda_reference_forward_f64(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, size_t batch_size, const double *device_parameter, int parameter_on_left, double *device_outputs, cudaStream_t stream);
geo_batch_gp_cuda_status_t geo_batch_gp_cuda_planned_forward_f64(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, size_t batch_size, const double *device_parameter, int parameter_on_left, double *device_outputs, cudaStream_t stream);
geo_batch_gp_cuda_status_t geo_batch_gp_cuda_reference_parameter_vjp_f64(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_output_cotangents, size_t batch_size, int parameter_on_left, double *device_parameter_cotangent, cudaStream_t stream);
geo_batch_gp_cuda_status_t geo_batch_gp_cuda_parameter_vjp_f64(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_output_cotangents, size_t batch_size, int parameter_on_left, double *device_parameter_cotangent, cudaStream_t stream);
geo_batch_gp_cuda_status_t geo_batch_gp_cuda_reference_mse_sgd_step_f64(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_targets, size_t batch_size, double learning_rate, int parameter_on_left, double *device_parameter, double *device_residuals, double *device_gradient, double *device_loss, cudaStream_t stream);
geo_batch_gp_cuda_status_t geo_batch_gp_cuda_mse_sgd_step_f64(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_targets, size_t batch_size, double learning_rate, int parameter_on_left, double *device_parameter, double *device_residuals, double *device_gradient, double *device_loss, cudaStream_t stream);
const char *geo_batch_gp_cuda_status_string(geo_batch_gp_cuda_status_t status);

#ifdef __cplusplus
}
#endif

#endif
