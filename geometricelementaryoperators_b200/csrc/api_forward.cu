// api_forward.cu -- geo_b200_forward_f64: the fixed-parameter batched forward
// (the product of geo_batch_gp_cuda_planned_forward_f64, reference
// src/batch_gp_cuda.cu:252-286 and src/batch_gp.c:107-161) on the kernel
// family the caller picks, without a plan object.
#include <cuda_runtime.h>

#include "geo/geo_b200.h"
#include "geo_runtime.h"

extern "C" geo_b200_status_t geo_b200_forward_f64(uint8_t dimension, const int8_t *signature, int parameter_on_left,
                                                  geo_b200_algorithm_t algorithm, const double *device_inputs,
                                                  const double *device_parameter, double *device_outputs,
                                                  size_t batch_size, cudaStream_t stream) {
    geo::NvtxRange range("geo_b200.forward");
    if (!geo::dimension_valid(dimension)) return GEO_B200_UNSUPPORTED_DIMENSION;
    if (signature == nullptr || !geo::signature_valid(signature, dimension) || device_inputs == nullptr ||
        device_parameter == nullptr || device_outputs == nullptr || batch_size == 0)
        return GEO_B200_INVALID_ARGUMENT;
    if (algorithm != GEO_B200_ALGORITHM_AUTO && algorithm != GEO_B200_ALGORITHM_CAYLEY &&
        algorithm != GEO_B200_ALGORITHM_REPRESENTATION)
        return GEO_B200_INVALID_ARGUMENT;
    const geo::RepDevice *rep =
        algorithm == GEO_B200_ALGORITHM_CAYLEY ? nullptr
                                               : geo::cached_rep_device(dimension, signature, parameter_on_left != 0);
    const bool use_rep = rep != nullptr && geo::rep_forward_supported(*rep, device_inputs, device_outputs);
    if (algorithm == GEO_B200_ALGORITHM_REPRESENTATION && !use_rep) return GEO_B200_INVALID_ARGUMENT;
    cudaError_t e;
    if (use_rep) {
        e = geo::launch_rep_forward(*rep, device_inputs, device_parameter, device_outputs, batch_size, stream);
    } else {
        const geo::SignPlan *sp = geo::cached_sign_plan(dimension, signature, parameter_on_left != 0);
        if (sp == nullptr) return GEO_B200_INVALID_ARGUMENT;
        e = geo::launch_forward(*sp, device_inputs, device_parameter, device_outputs, batch_size, stream);
    }
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_B200_RUNTIME_FAILURE;
    }
    return GEO_B200_OK;
}
