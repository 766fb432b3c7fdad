// api_host.cu -- the host-pointer C ABI of geo/batch_gp.h on the GPU.
//
// Reference interfaces replaced (reference tree file:line):
//   geo_batch_gp_{right,left}_forward_f64        src/batch_gp.c:107-161
//   geo_batch_gp_{right,left}_vjp_parameter_f64  src/batch_gp.c:163-235
//   geo_batch_gp_{right,left}_mse_sgd_step_f64   src/batch_gp.c:237-350
//
// Each call is synchronous, like the reference. Arrays may live in pageable or
// pinned host memory or in device memory; they are copied into a per-device
// workspace, processed by the sm_100a kernels and copied back. The reference's
// status rules are reproduced exactly:
//   * a non-finite input, cotangent, target or parameter -> INVALID_ARGUMENT,
//     outputs untouched (the kernels probe their results; only when a probe
//     fires are the inputs scanned, so the common path reads them once);
//   * a non-finite forward output or gradient -> NUMERIC_FAILURE with the
//     outputs written, as the reference writes them before its final check;
//   * SGD: a residual that overflows -> INVALID_ARGUMENT (the reference's VJP
//     rejects non-finite cotangents), a non-finite candidate parameter ->
//     NUMERIC_FAILURE with the parameter unchanged, a non-finite mean loss ->
//     NUMERIC_FAILURE after the update (src/batch_gp.c:294-307).
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <mutex>

#include "geo/batch_gp.h"
#include "geo_runtime.h"

namespace {

constexpr int kMaxDevices = 64;

struct Workspace {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    double *a = nullptr;  // inputs
    double *b = nullptr;  // targets / cotangents
    double *c = nullptr;  // outputs
    size_t cap = 0;       // doubles per large buffer
    double *small = nullptr;     // [0,64) parameter, [64,128) gradient, [128] loss sum
    double *records = nullptr;   // kMaxCtas * kRecStride
    uint32_t *status = nullptr;  // device status word
};

Workspace g_ws[kMaxDevices];

bool plan_valid(const geo_batch_gp_plan_t *plan) {
    if (plan == nullptr) return false;
    const size_t blades = (size_t)1u << plan->dimension;
    return plan->abi_version == GEO_BATCH_GP_ABI_VERSION && geo::signature_valid(plan->signature, plan->dimension) &&
           plan->blade_count == blades && plan->term_count == blades * blades;
}

// Returns false on allocation or runtime failure.
bool workspace_ready(Workspace &ws, size_t values, bool need_b, bool need_c) {
    if (ws.stream == nullptr) {
        if (cudaStreamCreateWithFlags(&ws.stream, cudaStreamNonBlocking) != cudaSuccess) return false;
        if (cudaMalloc((void **)&ws.small, 256 * sizeof(double)) != cudaSuccess) return false;
        if (cudaMalloc((void **)&ws.records, (size_t)geo::kMaxCtas * geo::kRecStride * sizeof(double)) != cudaSuccess)
            return false;
        if (cudaMalloc((void **)&ws.status, 64) != cudaSuccess) return false;
    }
    if (ws.cap < values) {
        cudaFree(ws.a);
        cudaFree(ws.b);
        cudaFree(ws.c);
        ws.a = ws.b = ws.c = nullptr;
        ws.cap = 0;
        if (cudaMalloc((void **)&ws.a, values * sizeof(double)) != cudaSuccess) return false;
        if (cudaMalloc((void **)&ws.b, values * sizeof(double)) != cudaSuccess) return false;
        if (cudaMalloc((void **)&ws.c, values * sizeof(double)) != cudaSuccess) return false;
        ws.cap = values;
    }
    (void)need_b;
    (void)need_c;
    return true;
}

Workspace *current_workspace() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    return &g_ws[dev];
}

bool host_finite(const double *values, size_t count, Workspace &ws) {
    // `values` may be device memory; fetch N <= 64 values to the host first.
    double local[64];
    if (count > 64) return false;
    if (geo::copy_any(local, values, count * sizeof(double), ws.stream) != cudaSuccess) return false;
    for (size_t i = 0; i < count; ++i)
        if (!isfinite(local[i])) return false;
    return true;
}

// Scan device arrays; true when every value is finite.
bool device_finite(Workspace &ws, const double *a, const double *b, size_t count) {
    uint32_t bits = 0;
    if (cudaMemsetAsync(ws.status, 0, sizeof(uint32_t), ws.stream) != cudaSuccess) return false;
    if (a && geo::launch_check_finite(a, count, 1u, ws.status, ws.stream) != cudaSuccess) return false;
    if (b && geo::launch_check_finite(b, count, 1u, ws.status, ws.stream) != cudaSuccess) return false;
    if (geo::copy_any(&bits, ws.status, sizeof(bits), ws.stream) != cudaSuccess) return false;
    return bits == 0u;
}

geo_batch_gp_status_t forward_impl(const geo_batch_gp_plan_t *plan, const double *inputs, size_t batch_size,
                                   const double *parameter, int on_left, double *outputs) {
    if (!plan_valid(plan) || batch_size == 0u || outputs == nullptr || inputs == nullptr || parameter == nullptr)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    const size_t blades = plan->blade_count;
    const size_t values = batch_size * blades;
    Workspace *wsp = current_workspace();
    if (wsp == nullptr) return GEO_BATCH_GP_INVALID_ARGUMENT;
    Workspace &ws = *wsp;
    std::lock_guard<std::mutex> lock(ws.mu);
    if (!workspace_ready(ws, values, false, true)) return GEO_BATCH_GP_INVALID_ARGUMENT;
    if (!host_finite(parameter, blades, ws)) return GEO_BATCH_GP_INVALID_ARGUMENT;
    const geo::SignPlan *sp = geo::cached_sign_plan(plan->dimension, plan->signature, on_left);
    if (sp == nullptr) return GEO_BATCH_GP_INVALID_ARGUMENT;
    if (geo::copy_any(ws.small, parameter, blades * sizeof(double), ws.stream) != cudaSuccess ||
        geo::copy_any(ws.a, inputs, values * sizeof(double), ws.stream) != cudaSuccess)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    uint32_t bits = 0;
    if (cudaMemsetAsync(ws.status, 0, sizeof(uint32_t), ws.stream) != cudaSuccess ||
        geo::launch_forward(*sp, ws.a, ws.small, ws.c, batch_size, ws.stream) != cudaSuccess ||
        geo::launch_check_finite(ws.c, values, geo::kDevOutputNonFinite, ws.status, ws.stream) != cudaSuccess ||
        geo::copy_any(&bits, ws.status, sizeof(bits), ws.stream) != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    }
    if (bits != 0u && !device_finite(ws, ws.a, nullptr, values)) return GEO_BATCH_GP_INVALID_ARGUMENT;
    if (geo::copy_any(outputs, ws.c, values * sizeof(double), ws.stream) != cudaSuccess)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    return bits != 0u ? GEO_BATCH_GP_NUMERIC_FAILURE : GEO_BATCH_GP_OK;
}

geo_batch_gp_status_t vjp_impl(const geo_batch_gp_plan_t *plan, const double *inputs, const double *cotangents,
                               size_t batch_size, int on_left, double *parameter_cotangent) {
    if (!plan_valid(plan) || batch_size == 0u || parameter_cotangent == nullptr || inputs == nullptr ||
        cotangents == nullptr)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    const size_t blades = plan->blade_count;
    const size_t values = batch_size * blades;
    Workspace *wsp = current_workspace();
    if (wsp == nullptr) return GEO_BATCH_GP_INVALID_ARGUMENT;
    Workspace &ws = *wsp;
    std::lock_guard<std::mutex> lock(ws.mu);
    if (!workspace_ready(ws, values, true, false)) return GEO_BATCH_GP_INVALID_ARGUMENT;
    const geo::SignPlan *sp = geo::cached_sign_plan(plan->dimension, plan->signature, on_left);
    if (sp == nullptr) return GEO_BATCH_GP_INVALID_ARGUMENT;
    if (geo::copy_any(ws.a, inputs, values * sizeof(double), ws.stream) != cudaSuccess ||
        geo::copy_any(ws.b, cotangents, values * sizeof(double), ws.stream) != cudaSuccess)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    geo::OptimizerArgs opt{};
    opt.kind = geo::kOptNone;
    opt.blades = (int32_t)blades;
    int ctas = 0;
    uint32_t bits = 0;
    double gradient[64];
    const geo::RepDevice *rep = geo::cached_rep_device(plan->dimension, plan->signature, on_left != 0);
    const bool use_rep = rep != nullptr && geo::rep_vjp_supported(*rep, ws.a, ws.b);
    if (cudaMemsetAsync(ws.status, 0, sizeof(uint32_t), ws.stream) != cudaSuccess ||
        (use_rep ? geo::launch_rep_vjp(*rep, ws.a, ws.b, batch_size, ws.records, &ctas, ws.stream)
                 : geo::launch_cycle(*sp, geo::kVjp, ws.a, ws.b, nullptr, nullptr, batch_size, ws.records, &ctas,
                                     ws.stream)) != cudaSuccess ||
        geo::launch_finalize(ws.records, ctas, opt, ws.small + 64, nullptr, nullptr, nullptr, nullptr, ws.status,
                             ws.stream) != cudaSuccess ||
        geo::copy_any(&bits, ws.status, sizeof(bits), ws.stream) != cudaSuccess ||
        geo::copy_any(gradient, ws.small + 64, blades * sizeof(double), ws.stream) != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    }
    if (bits != 0u && !device_finite(ws, ws.a, ws.b, values)) return GEO_BATCH_GP_INVALID_ARGUMENT;
    if (geo::copy_any(parameter_cotangent, gradient, blades * sizeof(double), ws.stream) != cudaSuccess)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    return bits != 0u ? GEO_BATCH_GP_NUMERIC_FAILURE : GEO_BATCH_GP_OK;
}

geo_batch_gp_status_t sgd_impl(const geo_batch_gp_plan_t *plan, const double *inputs, const double *targets,
                               size_t batch_size, double learning_rate, int on_left, double *parameter,
                               double *mean_loss) {
    if (!plan_valid(plan) || batch_size == 0u || !isfinite(learning_rate) || learning_rate <= 0.0 ||
        mean_loss == nullptr || inputs == nullptr || targets == nullptr || parameter == nullptr)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    const size_t blades = plan->blade_count;
    const size_t values = batch_size * blades;
    Workspace *wsp = current_workspace();
    if (wsp == nullptr) return GEO_BATCH_GP_INVALID_ARGUMENT;
    Workspace &ws = *wsp;
    std::lock_guard<std::mutex> lock(ws.mu);
    if (!workspace_ready(ws, values, true, false)) return GEO_BATCH_GP_INVALID_ARGUMENT;
    if (!host_finite(parameter, blades, ws)) return GEO_BATCH_GP_INVALID_ARGUMENT;
    const geo::SignPlan *sp = geo::cached_sign_plan(plan->dimension, plan->signature, on_left);
    if (sp == nullptr) return GEO_BATCH_GP_INVALID_ARGUMENT;
    if (geo::copy_any(ws.small, parameter, blades * sizeof(double), ws.stream) != cudaSuccess ||
        geo::copy_any(ws.a, inputs, values * sizeof(double), ws.stream) != cudaSuccess ||
        geo::copy_any(ws.b, targets, values * sizeof(double), ws.stream) != cudaSuccess)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    geo::OptimizerArgs opt{};
    opt.kind = geo::kOptSgdBatchGp;
    opt.blades = (int32_t)blades;
    opt.learning_rate = learning_rate;
    opt.batch_divisor = (double)batch_size;
    int ctas = 0;
    uint32_t bits = 0;
    double loss_sum = 0.0;
    double updated[64];
    if (cudaMemsetAsync(ws.status, 0, sizeof(uint32_t), ws.stream) != cudaSuccess ||
        geo::launch_cycle(*sp, geo::kCycle, ws.a, ws.b, ws.small, nullptr, batch_size, ws.records, &ctas,
                          ws.stream) != cudaSuccess ||
        geo::launch_finalize(ws.records, ctas, opt, ws.small + 64, ws.small + 128, ws.small, nullptr, nullptr,
                             ws.status, ws.stream) != cudaSuccess ||
        geo::copy_any(&bits, ws.status, sizeof(bits), ws.stream) != cudaSuccess ||
        geo::copy_any(&loss_sum, ws.small + 128, sizeof(double), ws.stream) != cudaSuccess ||
        geo::copy_any(updated, ws.small, blades * sizeof(double), ws.stream) != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    }
    const uint32_t pre_update =
        geo::kDevOutputNonFinite | geo::kDevResidualNonFinite | geo::kDevGradientNonFinite;
    if ((bits & pre_update) != 0u) {
        if (!device_finite(ws, ws.a, ws.b, values)) return GEO_BATCH_GP_INVALID_ARGUMENT;
        if (bits & geo::kDevOutputNonFinite) return GEO_BATCH_GP_NUMERIC_FAILURE;
        if (bits & geo::kDevResidualNonFinite) return GEO_BATCH_GP_INVALID_ARGUMENT;
        return GEO_BATCH_GP_NUMERIC_FAILURE;
    }
    if (bits & geo::kDevCandidateNonFinite) return GEO_BATCH_GP_NUMERIC_FAILURE;
    if (geo::copy_any(parameter, updated, blades * sizeof(double), ws.stream) != cudaSuccess)
        return GEO_BATCH_GP_INVALID_ARGUMENT;
    *mean_loss = loss_sum / (double)batch_size;
    return isfinite(*mean_loss) ? GEO_BATCH_GP_OK : GEO_BATCH_GP_NUMERIC_FAILURE;
}

}  // namespace

extern "C" geo_batch_gp_status_t geo_batch_gp_right_forward_f64(const geo_batch_gp_plan_t *plan,
                                                                const double *inputs, size_t batch_size,
                                                                const double *right_parameter, double *outputs) {
    return forward_impl(plan, inputs, batch_size, right_parameter, 0, outputs);
}

extern "C" geo_batch_gp_status_t geo_batch_gp_left_forward_f64(const geo_batch_gp_plan_t *plan,
                                                               const double *left_parameter, const double *inputs,
                                                               size_t batch_size, double *outputs) {
    return forward_impl(plan, inputs, batch_size, left_parameter, 1, outputs);
}

extern "C" geo_batch_gp_status_t geo_batch_gp_right_vjp_parameter_f64(const geo_batch_gp_plan_t *plan,
                                                                      const double *inputs,
                                                                      const double *output_cotangents,
                                                                      size_t batch_size,
                                                                      double *parameter_cotangent) {
    return vjp_impl(plan, inputs, output_cotangents, batch_size, 0, parameter_cotangent);
}

extern "C" geo_batch_gp_status_t geo_batch_gp_left_vjp_parameter_f64(const geo_batch_gp_plan_t *plan,
                                                                     const double *inputs,
                                                                     const double *output_cotangents,
                                                                     size_t batch_size,
                                                                     double *parameter_cotangent) {
    return vjp_impl(plan, inputs, output_cotangents, batch_size, 1, parameter_cotangent);
}

extern "C" geo_batch_gp_status_t geo_batch_gp_right_mse_sgd_step_f64(const geo_batch_gp_plan_t *plan,
                                                                     const double *inputs, const double *targets,
                                                                     size_t batch_size, double learning_rate,
                                                                     double *right_parameter, double *mean_loss) {
    return sgd_impl(plan, inputs, targets, batch_size, learning_rate, 0, right_parameter, mean_loss);
}

extern "C" geo_batch_gp_status_t geo_batch_gp_left_mse_sgd_step_f64(const geo_batch_gp_plan_t *plan,
                                                                    const double *inputs, const double *targets,
                                                                    size_t batch_size, double learning_rate,
                                                                    double *left_parameter, double *mean_loss) {
    return sgd_impl(plan, inputs, targets, batch_size, learning_rate, 1, left_parameter, mean_loss);
}
