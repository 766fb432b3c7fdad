// crmath.cu -- the graph runtime's correctly rounded exp and tanh (crmath.h)
// over a device array (geo_b200_cr_math_f64).
#include <cuda_runtime.h>
#include <stdint.h>

#include "crmath.h"
#include "geo/geo_b200.h"

namespace {

__global__ void cr_math_kernel(int fn, const double *x, double *y, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const double v = x[i];
        double r;
        switch (fn) {
            case GEO_B200_CR_EXP: r = geo::cr::exp(v); break;
            case GEO_B200_CR_TANH: r = geo::cr::tanh(v); break;
            case GEO_B200_CR_EXP_EXACT_PATH: {
                const double a = fabs(v);
                r = (a >= 0x1p-54 && a < 746.0) ? geo::cr::exp_accurate(v) : geo::cr::exp(v);
                break;
            }
            default: {
                const double a = fabs(v);
                r = (a >= 0x1p-27 && a < 19.1) ? geo::cr::tanh_accurate(v) : geo::cr::tanh(v);
                break;
            }
        }
        y[i] = r;
    }
}

}  // namespace

extern "C" geo_b200_status_t geo_b200_cr_math_f64(int function, const double *device_in, double *device_out,
                                                  size_t count, cudaStream_t stream) {
    if (function < GEO_B200_CR_EXP || function > GEO_B200_CR_TANH_EXACT_PATH) return GEO_B200_INVALID_ARGUMENT;
    if (count == 0) return GEO_B200_OK;
    if (device_in == nullptr || device_out == nullptr) return GEO_B200_INVALID_ARGUMENT;
    const unsigned blocks = (unsigned)((count + 255) / 256 < 148 * 8 ? (count + 255) / 256 : 148 * 8);
    cr_math_kernel<<<blocks, 256, 0, stream>>>(function, device_in, device_out, count);
    return cudaGetLastError() == cudaSuccess ? GEO_B200_OK : GEO_B200_RUNTIME_FAILURE;
}
