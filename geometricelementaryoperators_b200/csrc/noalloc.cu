// noalloc.cu -- geo_b200_parameter_vjp_noalloc_f64: the parameter VJP with its
// reduction scratch in a fixed array compiled into the library, for callers
// that cannot allocate device memory (see geo/geo_b200.h for the contract).
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

#include "geo/geo_b200.h"
#include "geo_runtime.h"

namespace {

constexpr int kRecords = (int)GEO_B200_NOALLOC_RECORDS;
static_assert(GEO_B200_NOALLOC_MAX_BATCH <= (size_t)GEO_B200_NOALLOC_RECORDS * 64u,
              "every dimension's tile holds at least 64 samples");

// The scratch: one record (kRecStride doubles) per CTA of a call. Each CTA
// overwrites every slot the finalize step reads, so nothing has to be cleared
// between calls; the array keeps the last call's contents.
static __device__ __align__(256) double g_noalloc_records[(size_t)kRecords * geo::kRecStride];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
double *g_records[kMaxDevices] = {};
CUcontext g_context[kMaxDevices] = {};  // the context the address belongs to

// The current driver context (null when the driver entry point is missing).
CUcontext current_context() {
    using Fn = CUresult (*)(CUcontext *);
    static Fn fn = []() -> Fn {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<Fn>(p);
    }();
    CUcontext ctx = nullptr;
    if (fn != nullptr && fn(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    return ctx;
}

// Device address of the array on the current device (host code cannot use the
// symbol's name as a pointer). Looked up once per device, and again only when
// the device's context is no longer the one the address was taken in (after a
// cudaDeviceReset the module is loaded anew and the old address is stale).
geo_b200_status_t records_for_current_device(double **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        (void)cudaGetLastError();
        return GEO_B200_RUNTIME_FAILURE;
    }
    std::lock_guard<std::mutex> lock(g_mutex);
    const CUcontext ctx = g_records[dev] != nullptr ? current_context() : nullptr;
    if (g_records[dev] == nullptr || ctx != g_context[dev]) {
        double *ptr = nullptr;
        if (cudaGetSymbolAddress((void **)&ptr, g_noalloc_records) != cudaSuccess || ptr == nullptr) {
            (void)cudaGetLastError();
            return GEO_B200_RUNTIME_FAILURE;
        }
        g_records[dev] = ptr;
        g_context[dev] = current_context();
    }
    *out = g_records[dev];
    return GEO_B200_OK;
}

}  // namespace

extern "C" geo_b200_status_t geo_b200_parameter_vjp_noalloc_f64(uint8_t dimension, const int8_t *signature,
                                                                int parameter_on_left, const double *device_inputs,
                                                                const double *device_output_cotangents,
                                                                size_t batch_size, double *device_parameter_cotangent,
                                                                cudaStream_t stream) {
    if (!geo::dimension_valid(dimension)) return GEO_B200_UNSUPPORTED_DIMENSION;
    if (!geo::signature_valid(signature, dimension) || device_inputs == nullptr ||
        device_output_cotangents == nullptr || device_parameter_cotangent == nullptr || batch_size == 0 ||
        batch_size > GEO_B200_NOALLOC_MAX_BATCH)
        return GEO_B200_INVALID_ARGUMENT;
    const geo::SignPlan *sp = geo::cached_sign_plan(dimension, signature, parameter_on_left != 0);
    if (sp == nullptr) return GEO_B200_INVALID_ARGUMENT;
    double *records = nullptr;
    const geo_b200_status_t st = records_for_current_device(&records);
    if (st != GEO_B200_OK) return st;
    int ctas = 0;
    cudaError_t e = geo::launch_vjp_per_tile(*sp, device_inputs, device_output_cotangents, batch_size, records,
                                             kRecords, &ctas, stream);
    if (e == cudaSuccess) {
        geo::OptimizerArgs opt{};
        opt.kind = geo::kOptNone;
        opt.blades = sp->blades;
        e = geo::launch_finalize(records, ctas, opt, device_parameter_cotangent, nullptr, nullptr, nullptr, nullptr,
                                 nullptr, stream);
    }
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_B200_RUNTIME_FAILURE;
    }
    return GEO_B200_OK;
}
