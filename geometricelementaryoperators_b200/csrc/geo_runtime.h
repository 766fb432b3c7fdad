// geo_runtime.h -- host runtime helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stddef.h>
#include <stdint.h>

#include "geo_internal.h"

namespace geo {

// Cached SignPlan for (dimension, signature, side); nullptr when invalid.
// Thread-safe; plans are built once and never freed.
const SignPlan *cached_sign_plan(uint8_t dimension, const int8_t *signature, int parameter_on_left);

// Byte layout of the single device allocation behind a geo_batch_gp_cuda_plan_t.
// The first five regions hold exactly what the reference uploads
// (reference src/batch_gp_cuda.cu:220-238); the rest is this library's.
struct DevicePlanLayout {
    static constexpr size_t kSignature = 0;
    static constexpr size_t kLeft = 64;
    static constexpr size_t kRight = kLeft + 4096;
    static constexpr size_t kOutput = kRight + 4096;
    static constexpr size_t kSign = kOutput + 4096;
    static constexpr size_t kRecords = 16640;  // 256-byte aligned
    static constexpr size_t kRecordBytes = (size_t)kMaxCtas * kRecStride * sizeof(double);
    static constexpr size_t kTotal = kRecords + kRecordBytes;
};

// Pointer residency as seen by the CUDA runtime.
enum class Residency { kDevice, kPinnedHost, kPageableHost };
Residency classify_pointer(const void *ptr);

// Copy helper that accepts any residency on either side (synchronous on `stream`).
cudaError_t copy_any(void *dst, const void *src, size_t bytes, cudaStream_t stream);

// Named host range for profilers (NVTX, header-only: a no-op unless a tool is
// attached): marks the enqueue of an entry point's launches.
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};

}  // namespace geo
