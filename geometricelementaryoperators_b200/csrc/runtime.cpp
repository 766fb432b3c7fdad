// runtime.cpp -- sign-plan cache and pointer classification.
#include <cstring>
#include <mutex>

#include "geo_runtime.h"

namespace geo {

namespace {
// Index: dimension (1..6) x signature bit pattern (bit a set = axis a is -1) x side.
struct PlanSlot {
    bool ready = false;
    SignPlan plan;
};
PlanSlot g_slots[kMaxDim + 1][64][2];
std::mutex g_slots_mutex;
}  // namespace

const SignPlan *cached_sign_plan(uint8_t dimension, const int8_t *signature, int parameter_on_left) {
    if (!signature_valid(signature, dimension)) return nullptr;
    unsigned mask = 0;
    for (unsigned a = 0; a < dimension; ++a)
        if (signature[a] < 0) mask |= 1u << a;
    PlanSlot &slot = g_slots[dimension][mask][parameter_on_left ? 1 : 0];
    std::lock_guard<std::mutex> lock(g_slots_mutex);
    if (!slot.ready) {
        if (!make_sign_plan(&slot.plan, dimension, signature, parameter_on_left)) return nullptr;
        slot.ready = true;
    }
    return &slot.plan;
}

Residency classify_pointer(const void *ptr) {
    cudaPointerAttributes attr;
    std::memset(&attr, 0, sizeof(attr));
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
        (void)cudaGetLastError();
        return Residency::kPageableHost;
    }
    switch (attr.type) {
        case cudaMemoryTypeDevice:
        case cudaMemoryTypeManaged:
            return Residency::kDevice;
        case cudaMemoryTypeHost:
            return Residency::kPinnedHost;
        default:
            return Residency::kPageableHost;
    }
}

cudaError_t copy_any(void *dst, const void *src, size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return cudaSuccess;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(stream);
}

}  // namespace geo
