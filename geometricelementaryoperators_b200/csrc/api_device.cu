// api_device.cu -- the device-pointer C ABI (geo/batch_gp_cuda.h and
// geo/hand_cuda_comparator.h), implemented on this library's sm_100a kernels.
//
// Reference interfaces replaced (file:line in the reference tree):
//   geo_batch_gp_cuda_plan_upload/destroy     src/batch_gp_cuda.cu:204-250
//   geo_batch_gp_cuda_*forward_f64            src/batch_gp_cuda.cu:252-286
//   geo_batch_gp_cuda_*parameter_vjp_f64      src/batch_gp_cuda.cu:288-320
//   geo_batch_gp_cuda_*mse_sgd_step_f64       src/batch_gp_cuda.cu:322-354 (+ :152-196)
//   geo_batch_gp_cuda_status_string           src/batch_gp_cuda.cu:356-365
//   geo_hand_cuda_*                           src/hand_cuda_comparator.cu:107-211
// Argument checks, status codes and the asynchronous contract are the
// reference's: a call returns after enqueueing work on `stream` and reports
// only argument errors and launch errors.
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include "geo/batch_gp_cuda.h"
#include "geo/hand_cuda_comparator.h"
#include "geo_runtime.h"

using geo::DevicePlanLayout;

namespace {

bool plan_usable(const geo_batch_gp_cuda_plan_t *plan) {
    if (plan == nullptr || plan->abi_version != GEO_BATCH_GP_CUDA_ABI_VERSION || plan->blade_count == 0 ||
        plan->term_count != plan->blade_count * plan->blade_count || plan->device_signature == nullptr ||
        plan->device_sign == nullptr) {
        return false;
    }
    // The scratch area lives in the same allocation: only plans made by
    // geo_batch_gp_cuda_plan_upload carry it.
    const uint8_t *base = reinterpret_cast<const uint8_t *>(plan->device_signature);
    return plan->device_left_blade == base + DevicePlanLayout::kLeft &&
           plan->device_right_blade == base + DevicePlanLayout::kRight &&
           plan->device_output_blade == base + DevicePlanLayout::kOutput &&
           reinterpret_cast<const uint8_t *>(plan->device_sign) == base + DevicePlanLayout::kSign &&
           plan->blade_count == (1u << plan->dimension);
}

double *plan_records(const geo_batch_gp_cuda_plan_t *plan) {
    return reinterpret_cast<double *>(reinterpret_cast<uint8_t *>(plan->device_signature) +
                                      DevicePlanLayout::kRecords);
}

geo_batch_gp_cuda_status_t launch_status(cudaError_t e) {
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_BATCH_GP_CUDA_RUNTIME_FAILURE;
    }
    return GEO_BATCH_GP_CUDA_OK;
}

geo_batch_gp_cuda_status_t forward(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs,
                                   size_t batch_size, const double *device_parameter, int parameter_on_left,
                                   double *device_outputs, cudaStream_t stream) {
    geo::NvtxRange range("geo_batch_gp_cuda.forward");
    if (!plan_usable(plan) || device_inputs == nullptr || device_parameter == nullptr ||
        device_outputs == nullptr || batch_size == 0) {
        return GEO_BATCH_GP_CUDA_INVALID_ARGUMENT;
    }
    const geo::SignPlan *sp = geo::cached_sign_plan(plan->dimension, plan->signature, parameter_on_left != 0);
    if (sp == nullptr) return GEO_BATCH_GP_CUDA_INVALID_ARGUMENT;
    // n = 5, 6 with 16-byte aligned operands: the representation forward on the
    // FP64 tensor cores (the MSE-SGD step below computes its outputs with the same
    // arithmetic); otherwise the Cayley kernel.
    const geo::RepDevice *rep = geo::cached_rep_device(plan->dimension, plan->signature, parameter_on_left != 0);
    if (rep != nullptr && geo::rep_forward_supported(*rep, device_inputs, device_outputs))
        return launch_status(
            geo::launch_rep_forward(*rep, device_inputs, device_parameter, device_outputs, batch_size, stream));
    return launch_status(geo::launch_forward(*sp, device_inputs, device_parameter, device_outputs, batch_size, stream));
}

geo_batch_gp_cuda_status_t vjp(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs,
                               const double *device_output_cotangents, size_t batch_size, int parameter_on_left,
                               double *device_parameter_cotangent, cudaStream_t stream) {
    geo::NvtxRange range("geo_batch_gp_cuda.parameter_vjp");
    if (!plan_usable(plan) || device_inputs == nullptr || device_output_cotangents == nullptr ||
        device_parameter_cotangent == nullptr || batch_size == 0) {
        return GEO_BATCH_GP_CUDA_INVALID_ARGUMENT;
    }
    const geo::SignPlan *sp = geo::cached_sign_plan(plan->dimension, plan->signature, parameter_on_left != 0);
    if (sp == nullptr) return GEO_BATCH_GP_CUDA_INVALID_ARGUMENT;
    double *records = plan_records(plan);
    int ctas = 0;
    // n = 5, 6 with 16-byte aligned operands: the representation kernel on the
    // FP64 tensor cores; otherwise the Cayley kernel.
    const geo::RepDevice *rep = geo::cached_rep_device(plan->dimension, plan->signature, parameter_on_left != 0);
    cudaError_t e = (rep != nullptr && geo::rep_vjp_supported(*rep, device_inputs, device_output_cotangents))
                        ? geo::launch_rep_vjp(*rep, device_inputs, device_output_cotangents, batch_size, records,
                                              &ctas, stream)
                        : geo::launch_cycle(*sp, geo::kVjp, device_inputs, device_output_cotangents, nullptr, nullptr,
                                            batch_size, records, &ctas, stream);
    if (e != cudaSuccess) return launch_status(e);
    geo::OptimizerArgs opt{};
    opt.kind = geo::kOptNone;
    opt.blades = plan->blade_count;
    e = geo::launch_finalize(records, ctas, opt, device_parameter_cotangent, nullptr, nullptr, nullptr, nullptr,
                             nullptr, stream);
    return launch_status(e);
}

// Forward -> residual (stored) -> loss sum -> VJP -> SGD, as the reference's
// five-launch sequence (src/batch_gp_cuda.cu:152-196). n = 5, 6 with 16-byte
// aligned operands: one representation pass stores r = y - t (y exactly as the
// forward above computes it, so targets equal to its outputs give zero
// residuals, loss and gradient, as in the reference) and reduces the parameter
// VJP of r with 0.5 |r|^2, then the update; otherwise the fused Cayley cycle
// kernel and the update.
geo_batch_gp_cuda_status_t sgd_step(const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs,
                                    const double *device_targets, size_t batch_size, double learning_rate,
                                    int parameter_on_left, double *device_parameter, double *device_residuals,
                                    double *device_gradient, double *device_loss, cudaStream_t stream) {
    geo::NvtxRange range("geo_batch_gp_cuda.mse_sgd_step");
    if (!plan_usable(plan) || device_inputs == nullptr || device_targets == nullptr || device_parameter == nullptr ||
        device_residuals == nullptr || device_gradient == nullptr || device_loss == nullptr || batch_size == 0 ||
        !isfinite(learning_rate) || learning_rate <= 0.0) {
        return GEO_BATCH_GP_CUDA_INVALID_ARGUMENT;
    }
    const geo::SignPlan *sp = geo::cached_sign_plan(plan->dimension, plan->signature, parameter_on_left != 0);
    if (sp == nullptr) return GEO_BATCH_GP_CUDA_INVALID_ARGUMENT;
    double *records = plan_records(plan);
    int ctas = 0;
    const geo::RepDevice *rep = geo::cached_rep_device(plan->dimension, plan->signature, parameter_on_left != 0);
    cudaError_t e;
    if (rep != nullptr && geo::rep_sgd_supported(*rep, device_inputs, device_targets, device_residuals)) {
        e = geo::launch_rep_mse_pass(*rep, device_inputs, device_parameter, device_targets, device_residuals,
                                     batch_size, records, &ctas, stream);
    } else {
        e = geo::launch_cycle(*sp, geo::kCycle, device_inputs, device_targets, device_parameter, device_residuals,
                              batch_size, records, &ctas, stream);
    }
    if (e != cudaSuccess) return launch_status(e);
    geo::OptimizerArgs opt{};
    opt.kind = geo::kOptSgdScaled;
    opt.blades = plan->blade_count;
    opt.learning_rate = learning_rate / (double)batch_size;  // the reference's scale, src/batch_gp_cuda.cu:194
    e = geo::launch_finalize(records, ctas, opt, device_gradient, device_loss, device_parameter, nullptr, nullptr,
                             nullptr, stream);
    return launch_status(e);
}

}  // namespace

extern "C" uint32_t geo_batch_gp_cuda_abi_version(void) { return GEO_BATCH_GP_CUDA_ABI_VERSION; }

extern "C" geo_batch_gp_cuda_status_t geo_batch_gp_cuda_plan_upload(geo_batch_gp_cuda_plan_t *device_plan,
                                                                    const geo_batch_gp_plan_t *host_plan) {
    if (device_plan == nullptr || host_plan == nullptr || host_plan->abi_version != GEO_BATCH_GP_ABI_VERSION ||
        host_plan->blade_count == 0 || host_plan->term_count != host_plan->blade_count * host_plan->blade_count ||
        !geo::signature_valid(host_plan->signature, host_plan->dimension) ||
        host_plan->blade_count != (1u << host_plan->dimension)) {
        return GEO_BATCH_GP_CUDA_INVALID_ARGUMENT;
    }
    memset(device_plan, 0, sizeof(*device_plan));
    device_plan->abi_version = GEO_BATCH_GP_CUDA_ABI_VERSION;
    device_plan->blade_count = host_plan->blade_count;
    device_plan->term_count = host_plan->term_count;
    device_plan->dimension = host_plan->dimension;
    memcpy(device_plan->signature, host_plan->signature, sizeof(device_plan->signature));

    uint8_t *base = nullptr;
    if (cudaMalloc((void **)&base, DevicePlanLayout::kTotal) != cudaSuccess) {
        (void)cudaGetLastError();
        memset(device_plan, 0, sizeof(*device_plan));
        return GEO_BATCH_GP_CUDA_ALLOCATION_FAILURE;
    }
    // Same contents as the reference upload: signature bytes and the four term arrays.
    uint8_t staging[DevicePlanLayout::kRecords];
    memset(staging, 0, sizeof(staging));
    memcpy(staging + DevicePlanLayout::kSignature, host_plan->signature, host_plan->dimension);
    const size_t terms = host_plan->term_count;
    memcpy(staging + DevicePlanLayout::kLeft, host_plan->left_blade, terms);
    memcpy(staging + DevicePlanLayout::kRight, host_plan->right_blade, terms);
    memcpy(staging + DevicePlanLayout::kOutput, host_plan->output_blade, terms);
    memcpy(staging + DevicePlanLayout::kSign, host_plan->sign, terms);
    if (cudaMemcpy(base, staging, sizeof(staging), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(base + DevicePlanLayout::kRecords, 0, DevicePlanLayout::kRecordBytes) != cudaSuccess) {
        (void)cudaGetLastError();
        cudaFree(base);
        memset(device_plan, 0, sizeof(*device_plan));
        return GEO_BATCH_GP_CUDA_RUNTIME_FAILURE;
    }
    device_plan->device_signature = reinterpret_cast<int8_t *>(base + DevicePlanLayout::kSignature);
    device_plan->device_left_blade = base + DevicePlanLayout::kLeft;
    device_plan->device_right_blade = base + DevicePlanLayout::kRight;
    device_plan->device_output_blade = base + DevicePlanLayout::kOutput;
    device_plan->device_sign = reinterpret_cast<int8_t *>(base + DevicePlanLayout::kSign);
    // Warm the sign-plan cache for both sides so compute calls stay cheap.
    (void)geo::cached_sign_plan(host_plan->dimension, host_plan->signature, 0);
    (void)geo::cached_sign_plan(host_plan->dimension, host_plan->signature, 1);
    return GEO_BATCH_GP_CUDA_OK;
}

extern "C" void geo_batch_gp_cuda_plan_destroy(geo_batch_gp_cuda_plan_t *plan) {
    if (plan == nullptr) return;
    if (plan->device_signature != nullptr) cudaFree(plan->device_signature);
    memset(plan, 0, sizeof(*plan));
}

extern "C" geo_batch_gp_cuda_status_t geo_batch_gp_cuda_reference_forward_f64(
    const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, size_t batch_size,
    const double *device_parameter, int parameter_on_left, double *device_outputs, cudaStream_t stream) {
    return forward(plan, device_inputs, batch_size, device_parameter, parameter_on_left, device_outputs, stream);
}

extern "C" geo_batch_gp_cuda_status_t geo_batch_gp_cuda_planned_forward_f64(
    const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, size_t batch_size,
    const double *device_parameter, int parameter_on_left, double *device_outputs, cudaStream_t stream) {
    return forward(plan, device_inputs, batch_size, device_parameter, parameter_on_left, device_outputs, stream);
}

extern "C" geo_batch_gp_cuda_status_t geo_batch_gp_cuda_reference_parameter_vjp_f64(
    const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_output_cotangents,
    size_t batch_size, int parameter_on_left, double *device_parameter_cotangent, cudaStream_t stream) {
    return vjp(plan, device_inputs, device_output_cotangents, batch_size, parameter_on_left,
               device_parameter_cotangent, stream);
}

extern "C" geo_batch_gp_cuda_status_t geo_batch_gp_cuda_parameter_vjp_f64(
    const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_output_cotangents,
    size_t batch_size, int parameter_on_left, double *device_parameter_cotangent, cudaStream_t stream) {
    return vjp(plan, device_inputs, device_output_cotangents, batch_size, parameter_on_left,
               device_parameter_cotangent, stream);
}

extern "C" geo_batch_gp_cuda_status_t geo_batch_gp_cuda_reference_mse_sgd_step_f64(
    const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_targets,
    size_t batch_size, double learning_rate, int parameter_on_left, double *device_parameter,
    double *device_residuals, double *device_gradient, double *device_loss, cudaStream_t stream) {
    return sgd_step(plan, device_inputs, device_targets, batch_size, learning_rate, parameter_on_left,
                    device_parameter, device_residuals, device_gradient, device_loss, stream);
}

extern "C" geo_batch_gp_cuda_status_t geo_batch_gp_cuda_mse_sgd_step_f64(
    const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_targets,
    size_t batch_size, double learning_rate, int parameter_on_left, double *device_parameter,
    double *device_residuals, double *device_gradient, double *device_loss, cudaStream_t stream) {
    return sgd_step(plan, device_inputs, device_targets, batch_size, learning_rate, parameter_on_left,
                    device_parameter, device_residuals, device_gradient, device_loss, stream);
}

extern "C" const char *geo_batch_gp_cuda_status_string(geo_batch_gp_cuda_status_t status) {
    switch (status) {
        case GEO_BATCH_GP_CUDA_OK: return "ok";
        case GEO_BATCH_GP_CUDA_INVALID_ARGUMENT: return "invalid_argument";
        case GEO_BATCH_GP_CUDA_ALLOCATION_FAILURE: return "allocation_failure";
        case GEO_BATCH_GP_CUDA_RUNTIME_FAILURE: return "runtime_failure";
        case GEO_BATCH_GP_CUDA_NUMERIC_FAILURE: return "numeric_failure";
        default: return "unknown";
    }
}

// Hand-written control path of the reference: same contract, same kernels here.
extern "C" geo_batch_gp_cuda_status_t geo_hand_cuda_forward_f64(const geo_batch_gp_cuda_plan_t *plan,
                                                               const double *device_inputs, size_t batch_size,
                                                               const double *device_parameter,
                                                               int parameter_on_left, double *device_outputs,
                                                               cudaStream_t stream) {
    return forward(plan, device_inputs, batch_size, device_parameter, parameter_on_left, device_outputs, stream);
}

extern "C" geo_batch_gp_cuda_status_t geo_hand_cuda_parameter_vjp_f64(
    const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_output_cotangents,
    size_t batch_size, int parameter_on_left, double *device_parameter_cotangent, cudaStream_t stream) {
    return vjp(plan, device_inputs, device_output_cotangents, batch_size, parameter_on_left,
               device_parameter_cotangent, stream);
}

extern "C" geo_batch_gp_cuda_status_t geo_hand_cuda_mse_sgd_step_f64(
    const geo_batch_gp_cuda_plan_t *plan, const double *device_inputs, const double *device_targets,
    size_t batch_size, double learning_rate, int parameter_on_left, double *device_parameter,
    double *device_residuals, double *device_gradient, double *device_loss, cudaStream_t stream) {
    return sgd_step(plan, device_inputs, device_targets, batch_size, learning_rate, parameter_on_left,
                    device_parameter, device_residuals, device_gradient, device_loss, stream);
}
