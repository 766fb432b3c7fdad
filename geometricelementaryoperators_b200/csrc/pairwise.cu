// pairwise.cu -- per-element geometric products where both operands vary
// (geo_b200_pairwise_*).
//
// Reference semantics batched here (reference tree file:line):
//   geo_operator_gp_f64       src/operator_kernel.c:412-447
//   geo_operator_gp_f64_jvp   src/operator_kernel.c:449-492
//   geo_operator_gp_f64_vjp   src/operator_kernel.c:494-539
//
// Layout: sample-major [batch][2^n]. The generic kernel stages a tile of
// samples into shared memory with coalesced loads; one thread computes one
// output blade of one sample, reading the sign of every term from a bit table
// (bit p of neg[l] set when e_l e_p = -e_(l^p)). The n = 6 forwards (float64
// and float32) have dedicated TMA-staged kernels with compile-time signs.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <utility>

#include "geo/geo_b200.h"
#include "geo_runtime.h"
#include "pair_tables_gen.h"

namespace {

constexpr int kThreads = 256;

geo_b200_status_t from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return GEO_B200_OK;
    (void)cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? GEO_B200_ALLOCATION_FAILURE : GEO_B200_RUNTIME_FAILURE;
}

__device__ __forceinline__ double apply_sign(double v, bool negative) { return negative ? -v : v; }
__device__ __forceinline__ float apply_sign(float v, bool negative) { return negative ? -v : v; }

// Rank of an even blade among the even blades in increasing order.
__device__ __forceinline__ int even_rank(int blade) { return blade >> 1; }

enum PairMode : int { kPairForward = 0, kPairVjp = 1, kPairJvp = 2 };

// Stage `rows` samples of width `width` starting at `first` into smem (zero-fill past batch).
template <typename T>
__device__ __forceinline__ void stage(T *dst, const T *__restrict__ src, size_t first, int rows, int width,
                                     size_t batch) {
    for (int i = threadIdx.x; i < rows * width; i += blockDim.x) {
        const int s = i / width;
        const size_t sample = first + (size_t)s;
        dst[i] = sample < batch ? src[sample * width + (i - s * width)] : T(0);
    }
}

// One CTA handles kThreads / N samples per pass; thread (s, b) owns blade b of sample s.
template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads)
pairwise_kernel(const geo::SignPlan plan, const T *__restrict__ left, int left_compact, const T *__restrict__ right,
                const T *__restrict__ aux0, const T *__restrict__ aux1, T *__restrict__ out0, T *__restrict__ out1,
                size_t batch) {
    const int N = plan.blades;
    const int per_pass = kThreads / N;
    const int lw = left_compact ? N / 2 : N;
    __shared__ uint64_t neg[64];
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *Ls = reinterpret_cast<T *>(smem_raw);
    T *Rs = Ls + per_pass * N;
    T *A0 = Rs + per_pass * N;
    T *A1 = A0 + per_pass * N;
    if (threadIdx.x < 64) neg[threadIdx.x] = plan.neg[threadIdx.x];
    const int s = threadIdx.x / N;
    const int b = threadIdx.x - s * N;
    const bool lane_ok = s < per_pass;
    for (size_t first = (size_t)blockIdx.x * per_pass; first < batch; first += (size_t)gridDim.x * per_pass) {
        __syncthreads();
        // Left operand, expanded to dense storage in shared memory.
        for (int i = threadIdx.x; i < per_pass * N; i += blockDim.x) {
            const int ss = i / N;
            const int bb = i - ss * N;
            const size_t sample = first + (size_t)ss;
            T v = T(0);
            if (sample < batch) {
                if (!left_compact) v = left[sample * N + bb];
                else if ((__popc(bb) & 1) == 0) v = left[sample * lw + even_rank(bb)];
            }
            Ls[i] = v;
        }
        stage(Rs, right, first, per_pass, N, batch);
        if (MODE != kPairForward) stage(A0, aux0, first, per_pass, N, batch);
        if (MODE == kPairJvp) stage(A1, aux1, first, per_pass, N, batch);
        __syncthreads();
        const size_t sample = first + (size_t)s;
        if (!lane_ok || sample >= batch) continue;
        const T *l = Ls + s * N;
        const T *r = Rs + s * N;
        if (MODE == kPairForward) {
            // y[b] = sum_l left[l] right[l^b] s(l, l^b)
            T acc = T(0);
            for (int k = 0; k < N; ++k) {
                const int p = k ^ b;
                acc = fma(l[k], apply_sign(r[p], (neg[k] >> p) & 1ull), acc);
            }
            out0[sample * N + b] = acc;
        } else if (MODE == kPairVjp) {
            // left_bar[b] = sum_r cot[b^r] s(b, r) right[r]; right_bar[b] = sum_l cot[l^b] s(l, b) left[l]
            const T *c = A0 + s * N;
            if (out0 != nullptr) {
                T acc = T(0);
                const uint64_t nb = neg[b];
                for (int k = 0; k < N; ++k) acc = fma(apply_sign(c[b ^ k], (nb >> k) & 1ull), r[k], acc);
                out0[sample * N + b] = acc;
            }
            if (out1 != nullptr) {
                T acc = T(0);
                for (int k = 0; k < N; ++k) acc = fma(apply_sign(c[k ^ b], (neg[k] >> b) & 1ull), l[k], acc);
                out1[sample * N + b] = acc;
            }
        } else {
            // out_t[b] = sum_l (lt[l] right[l^b] + left[l] rt[l^b]) s(l, l^b)
            const T *lt = A0 + s * N;
            const T *rt = A1 + s * N;
            T acc = T(0);
            for (int k = 0; k < N; ++k) {
                const int p = k ^ b;
                const T term = fma(lt[k], r[p], l[k] * rt[p]);
                acc += apply_sign(term, (neg[k] >> p) & 1ull);
            }
            out0[sample * N + b] = acc;
        }
    }
}

// ---- float32 n = 6 fast path ----------------------------------------------
// One thread per element; the 64 output blades accumulate in registers and the
// sign of every term is a compile-time constant of the canonical signature
// Cl(6-Q, Q), so each term is one FFMA with a free operand negation. Tiles of
// 64 elements are staged through padded shared memory with 16-byte copies
// (coalesced in both directions); a compact even-grade left operand (32
// floats per element) halves its read traffic.
__host__ __device__ constexpr int popc_c(int v) { return v == 0 ? 0 : (v & 1) + popc_c(v >> 1); }

// k-th even blade (increasing order) of a 6-dimensional algebra.
__host__ __device__ constexpr int even_blade_c(int k) { return (k << 1) | (popc_c(k << 1) & 1); }

__host__ __device__ constexpr int sign_c(int l, int r, int q) {
    int s = 1;
    for (int a = 0; a < 6; ++a) {
        if ((l >> a) & 1) {
            int lower = r & ((1 << a) - 1), c = 0;
            for (; lower; lower &= lower - 1) ++c;
            if (c & 1) s = -s;
            if (((r >> a) & 1) && a >= 6 - q) s = -s;
        }
    }
    return s;
}

// One term y[l^r] += +-a_l b_r with compile-time indices and sign; the whole
// product is a fold over an index sequence so every array index is constant
// (the operands stay in registers).
template <int Q, bool COMPACT, int I, int LW>
__device__ __forceinline__ void f32_term(const float (&a)[LW], const float (&b)[64], float (&y)[64]) {
    constexpr int li = I / 64, r = I % 64;
    constexpr int l = COMPACT ? even_blade_c(li) : li;
    constexpr int sg = sign_c(l, r, Q);
    y[l ^ r] = fmaf(sg > 0 ? a[li] : -a[li], b[r], y[l ^ r]);
}

template <int Q, bool COMPACT, int LW, int... I>
__device__ __forceinline__ void f32_product(const float (&a)[LW], const float (&b)[64], float (&y)[64],
                                            std::integer_sequence<int, I...>) {
    (f32_term<Q, COMPACT, I, LW>(a, b, y), ...);
}

constexpr int kF32Threads = 64;
constexpr int kF32LdR = 64 + 4;   // padded row stride (floats) of right / out tiles
constexpr int kF32LdL = 64 + 4;   // left tile (dense or compact uses the first 32)

template <int Q, bool COMPACT>
__global__ void __launch_bounds__(kF32Threads)
pairwise_f32_n6_kernel(const float *__restrict__ left, const float *__restrict__ right, float *__restrict__ out,
                       size_t batch) {
    constexpr int LW = COMPACT ? 32 : 64;
    __shared__ __align__(16) float Ls[kF32Threads * kF32LdL];
    __shared__ __align__(16) float Rs[kF32Threads * kF32LdR];
    const int tid = threadIdx.x;
    for (size_t first = (size_t)blockIdx.x * kF32Threads; first < batch; first += (size_t)gridDim.x * kF32Threads) {
        const int rows = (int)min((size_t)kF32Threads, batch - first);
        // stage: 16-byte chunks, consecutive threads take consecutive chunks
        for (int c = tid; c < rows * (LW / 4); c += kF32Threads) {
            const int s = c / (LW / 4), k = c - s * (LW / 4);
            *reinterpret_cast<float4 *>(&Ls[s * kF32LdL + 4 * k]) =
                *reinterpret_cast<const float4 *>(&left[(first + s) * LW + 4 * k]);
        }
        for (int c = tid; c < rows * 16; c += kF32Threads) {
            const int s = c / 16, k = c - s * 16;
            *reinterpret_cast<float4 *>(&Rs[s * kF32LdR + 4 * k]) =
                *reinterpret_cast<const float4 *>(&right[(first + s) * 64 + 4 * k]);
        }
        __syncthreads();
        float a[LW], b[64], y[64];
        if (tid < rows) {
#pragma unroll
            for (int k = 0; k < LW / 4; ++k) {
                const float4 v = *reinterpret_cast<const float4 *>(&Ls[tid * kF32LdL + 4 * k]);
                a[4 * k] = v.x; a[4 * k + 1] = v.y; a[4 * k + 2] = v.z; a[4 * k + 3] = v.w;
            }
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float4 v = *reinterpret_cast<const float4 *>(&Rs[tid * kF32LdR + 4 * k]);
                b[4 * k] = v.x; b[4 * k + 1] = v.y; b[4 * k + 2] = v.z; b[4 * k + 3] = v.w;
            }
#pragma unroll
            for (int o = 0; o < 64; ++o) y[o] = 0.0f;
            // y[l ^ r] += a_l b_r s(l, r); compact storage holds the even blades in increasing order
            f32_product<Q, COMPACT, LW>(a, b, y, std::make_integer_sequence<int, LW * 64>{});
        }
        __syncthreads();
        if (tid < rows) {
#pragma unroll
            for (int k = 0; k < 16; ++k)
                *reinterpret_cast<float4 *>(&Rs[tid * kF32LdR + 4 * k]) =
                    make_float4(y[4 * k], y[4 * k + 1], y[4 * k + 2], y[4 * k + 3]);
        }
        __syncthreads();
        for (int c = tid; c < rows * 16; c += kF32Threads) {
            const int s = c / 16, k = c - s * 16;
            *reinterpret_cast<float4 *>(&out[(first + s) * 64 + 4 * k]) =
                *reinterpret_cast<const float4 *>(&Rs[s * kF32LdR + 4 * k]);
        }
        __syncthreads();
    }
}


// ---- float32 n = 6, TMA-staged ---------------------------------------------
// Same arithmetic as pairwise_f32_n6_kernel; the data moves by TMA. Each CTA
// of 64 threads (one element each) runs a ring of kTmaStages stages: tensor
// loads of 64-row boxes of the left (32 or 64 floats per row) and right
// (64 floats) operands, 128-byte swizzled; outputs are written back over the
// right operand's rows and leave by tensor stores. At the top of iteration k
// the stage of tile k - 1 is refilled with tile k + kTmaStages - 1 once its
// store has read it. Two stages (one tile loading during each compute) keep
// four CTAs (eight warps) per SM for the compact left operand, which measured
// faster than three stages at three CTAs per SM. Rows past the batch read as
// zeros and are not stored.
constexpr int kTmaRows = 64;
constexpr int kTmaStages = 2;
constexpr int kTmaSub = kTmaRows * 32;  // floats of one [64][32] box (8 KB)
constexpr uint32_t kTmaWaitLimit = 1u << 22;

// Give-ups of the TMA kernels' bounded waits on this device (read and reset by
// geo_b200_pairwise_wait_failures). Such a CTA stops issuing loads,
// waits (bounded) for the loads it has in flight, writes NaN into every output
// row it had not yet stored and ends.
__device__ unsigned g_pairwise_tma_wait_failures;

template <bool COMPACT>
struct TmaTile {
    static constexpr int A_SUB = COMPACT ? 1 : 2;  // boxes of the left operand
    static constexpr int STAGE = (A_SUB + 2) * kTmaSub;
    static constexpr unsigned BYTES = STAGE * sizeof(float);
    static constexpr size_t SMEM = (size_t)kTmaStages * BYTES + 1024;  // + alignment slack
};

// Float offset of (row, 4-float chunk j) in a [64][32] box stored with the
// 128-byte swizzle: chunk j of row r sits at chunk j ^ (r & 7).
__device__ __forceinline__ int sw128(int row, int chunk) { return row * 32 + ((chunk ^ (row & 7)) << 2); }

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

// Waits for phase `parity` of an mbarrier for at most `limit` polls; false when it gave up.
__device__ __forceinline__ bool tma_bounded_wait(uint64_t *bar, unsigned parity, uint32_t limit) {
    const unsigned a = smem_u32(bar);
    for (uint32_t i = 0; i < limit; ++i) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];\n" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int x, int y, const void *src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(map),
                 "r"(x), "r"(y), "r"(smem_u32(src))
                 : "memory");
}

// STARVE (the wait self-test only): no load is ever issued, so the first wait
// runs out after `wait_limit` polls with nothing in flight.
template <int Q, bool COMPACT, bool STARVE = false>
__global__ void __launch_bounds__(kTmaRows)
pairwise_f32_n6_tma_kernel(const __grid_constant__ CUtensorMap map_left, const __grid_constant__ CUtensorMap map_right,
                           const __grid_constant__ CUtensorMap map_out, float *__restrict__ out, size_t batch,
                           uint32_t wait_limit) {
    using TT = TmaTile<COMPACT>;
    constexpr int LW = COMPACT ? 32 : 64;
    extern __shared__ unsigned char tma_raw[];
    __shared__ __align__(8) uint64_t bars[kTmaStages];
    float *base = reinterpret_cast<float *>(((uintptr_t)tma_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x;
    const size_t tiles = (batch + kTmaRows - 1) / kTmaRows;
    const int K = (size_t)blockIdx.x < tiles ? (int)((tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    if (tid == 0) {
        for (int s = 0; s < kTmaStages; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(&bars[s])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    auto issue = [&](int k) {
        const int s = k % kTmaStages;
        float *st = base + s * TT::STAGE;
        const int y = (int)((blockIdx.x + (size_t)k * gridDim.x) * kTmaRows);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(&bars[s])),
                     "r"(TT::BYTES)
                     : "memory");
        tma_load_2d(st, &map_left, 0, y, &bars[s]);
        if (!COMPACT) tma_load_2d(st + kTmaSub, &map_left, 32, y, &bars[s]);
        tma_load_2d(st + TT::A_SUB * kTmaSub, &map_right, 0, y, &bars[s]);
        tma_load_2d(st + (TT::A_SUB + 1) * kTmaSub, &map_right, 32, y, &bars[s]);
    };
    int issued = 0;  // tiles whose loads were issued (thread 0's count)
    if (tid == 0 && !STARVE)
        for (; issued < K && issued < kTmaStages; ++issued) issue(issued);
    for (int k = 0; k < K; ++k) {
        const int s = k % kTmaStages;
        if (!STARVE && tid == 0 && k >= 1 && k + kTmaStages - 1 < K) {
            // The stage of tile k + 2 last held tile k - 1, whose store (the
            // latest one) must have finished reading it.
            asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
            issue(k + kTmaStages - 1);
            issued = k + kTmaStages;
        }
        const bool ok = tma_bounded_wait(&bars[s], (unsigned)((k / kTmaStages) & 1), wait_limit);
        float *st = base + s * TT::STAGE;
        float *rb = st + TT::A_SUB * kTmaSub;
        float a[LW], b[64], y[64];
#pragma unroll
        for (int j = 0; j < LW / 4; ++j) {
            const float4 v = *reinterpret_cast<const float4 *>(&st[(j >> 3) * kTmaSub + sw128(tid, j & 7)]);
            a[4 * j] = v.x; a[4 * j + 1] = v.y; a[4 * j + 2] = v.z; a[4 * j + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float4 v = *reinterpret_cast<const float4 *>(&rb[(j >> 3) * kTmaSub + sw128(tid, j & 7)]);
            b[4 * j] = v.x; b[4 * j + 1] = v.y; b[4 * j + 2] = v.z; b[4 * j + 3] = v.w;
        }
#pragma unroll
        for (int o = 0; o < 64; ++o) y[o] = 0.0f;
        f32_product<Q, COMPACT, LW>(a, b, y, std::make_integer_sequence<int, LW * 64>{});
        // Each thread overwrites only its own row, which only it has read.
#pragma unroll
        for (int j = 0; j < 16; ++j)
            *reinterpret_cast<float4 *>(&rb[(j >> 3) * kTmaSub + sw128(tid, j & 7)]) =
                make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        if (__syncthreads_or(!ok)) {
            // Some thread's wait gave up: tiles k..K-1 are not stored from the
            // ring. Wait (bounded) for the loads still in flight, then write
            // NaN into their rows.
            if (tid == 0) {
                for (int j = k; j < issued; ++j)
                    (void)tma_bounded_wait(&bars[j % kTmaStages], (unsigned)((j / kTmaStages) & 1), wait_limit);
                asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
                atomicAdd(&g_pairwise_tma_wait_failures, 1u);
            }
            for (int j = k; j < K; ++j) {
                const size_t row = (blockIdx.x + (size_t)j * gridDim.x) * kTmaRows + (size_t)tid;
                if (row < batch)
                    for (int c = 0; c < 64; ++c) out[row * 64 + c] = __int_as_float(0x7fc00000);
            }
            return;
        }
        if (tid == 0) {
            const int row = (int)((blockIdx.x + (size_t)k * gridDim.x) * kTmaRows);
            tma_store_2d(&map_out, 0, row, rb);
            tma_store_2d(&map_out, 32, row, rb + kTmaSub);
            asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
        }
    }
    if (tid == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
}

// cuTensorMapEncodeTiled from the driver (resolved once; null when unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// [rows][cols] float32 tensor, 64 x 32 boxes, 128-byte swizzle, zero fill.
bool encode_rows(CUtensorMap *map, const float *ptr, int cols, size_t rows) {
    const auto encode = tensor_map_encoder();
    if (encode == nullptr || rows == 0 || rows > 0xffffffffull) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(float)};
    const cuuint32_t box[2] = {32, (cuuint32_t)kTmaRows};
    const cuuint32_t elem[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int Q, bool COMPACT, bool STARVE = false>
cudaError_t launch_f32_tma(const CUtensorMap &ml, const CUtensorMap &mr, const CUtensorMap &mo, float *out,
                           size_t batch, cudaStream_t stream, uint32_t wait_limit = kTmaWaitLimit) {
    auto kernel = pairwise_f32_n6_tma_kernel<Q, COMPACT, STARVE>;
    const size_t smem = TmaTile<COMPACT>::SMEM;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kTmaRows, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const size_t tiles = (batch + kTmaRows - 1) / kTmaRows;
    size_t grid = (size_t)geo::device_sm_count() * (size_t)per_sm;
    if (grid > tiles) grid = tiles;
    kernel<<<(unsigned)grid, kTmaRows, smem, stream>>>(ml, mr, mo, out, batch, wait_limit);
    return cudaGetLastError();
}

// Canonical signature q of a length-6 signature (first 6-q entries +1, rest -1), or -1.
int canonical_q6(const int8_t *sig) {
    int q = 0;
    while (q < 6 && sig[5 - q] == -1) ++q;
    for (int a = 0; a < 6 - q; ++a)
        if (sig[a] != 1) return -1;
    return q;
}

bool launch_pairwise_f32_fast(const int8_t *signature, const float *left, int compact, const float *right, float *out,
                              size_t batch, cudaStream_t stream, cudaError_t *err) {
    const int q = canonical_q6(signature);
    if (q < 0) return false;
    const uintptr_t bits = (uintptr_t)left | (uintptr_t)right | (uintptr_t)out;
    if (bits & 15u) return false;  // float4 paths need 16-byte alignment
    {
        CUtensorMap ml, mr, mo;
        if (encode_rows(&ml, left, compact ? 32 : 64, batch) && encode_rows(&mr, right, 64, batch) &&
            encode_rows(&mo, out, 64, batch)) {
#define GEO_F32_TMA_CASE(QQ)                                                                        \
    case QQ:                                                                                        \
        *err = compact ? launch_f32_tma<QQ, true>(ml, mr, mo, out, batch, stream)                  \
                       : launch_f32_tma<QQ, false>(ml, mr, mo, out, batch, stream);                \
        return true;
            switch (q) {
                GEO_F32_TMA_CASE(0) GEO_F32_TMA_CASE(1) GEO_F32_TMA_CASE(2) GEO_F32_TMA_CASE(3) GEO_F32_TMA_CASE(4)
                GEO_F32_TMA_CASE(5) GEO_F32_TMA_CASE(6)
                default: break;
            }
#undef GEO_F32_TMA_CASE
        }
    }
    size_t grid = (batch + kF32Threads - 1) / kF32Threads;
    const size_t cap = (size_t)geo::device_sm_count() * 8;
    if (grid > cap) grid = cap;
#define GEO_F32_CASE(QQ)                                                                                       \
    case QQ:                                                                                                   \
        if (compact) pairwise_f32_n6_kernel<QQ, true><<<(unsigned)grid, kF32Threads, 0, stream>>>(left, right, out, batch); \
        else pairwise_f32_n6_kernel<QQ, false><<<(unsigned)grid, kF32Threads, 0, stream>>>(left, right, out, batch); \
        break;
    switch (q) {
        GEO_F32_CASE(0) GEO_F32_CASE(1) GEO_F32_CASE(2) GEO_F32_CASE(3) GEO_F32_CASE(4) GEO_F32_CASE(5) GEO_F32_CASE(6)
        default: return false;
    }
#undef GEO_F32_CASE
    *err = cudaGetLastError();
    return true;
}

// ---- float64 n = 6, TMA-staged, compile-time signs --------------------------
// y_o = sum_l a_l b_{l^o} sigma(l, o), sigma(l, o) = s(l, l^o). The sign rule
// is a bilinear form over GF(2): s(l, m) = (-1)^(l^T M m) with
// M = (strictly lower ones) + diag(negative axes). Splitting blade indices into
// the high axes 4, 5 (block L0, O0 in 0..3) and the low axes 0..3 (i, k in
// 0..15), sigma((L0,i), (O0,k)) = alpha_{L0,O0}(i) beta_{L0,O0}(k) gamma(i, k)
// with gamma(i, k) = s_low(i, k), the sign rule of the low four axes alone. So
// per 16 x 16 block (L0, O0) the 256 terms have compile-time signs gamma (one
// DFMA with a free negation each); alpha flips the sign bits of the 16 a
// values and beta is applied by flipping the accumulators' sign bits before
// and after the block (exact). The host derives alpha and beta from the sign
// rule and verifies the factorisation for every (l, o) before launching.
//
// CTA of 4 compute warps and one producer warp on tiles of 32 pairs
// (lane = pair): compute warp w produces output blades 16w..16w+15 of the
// tile's pairs. Operands arrive by TMA in [32][16] float64 boxes with the
// 128-byte swizzle (one 16-byte read per lane hits a distinct bank group per
// quarter warp) into a 2-stage ring: `full` mbarriers carry the transaction
// bytes, `empty` mbarriers (one arrival per compute warp) release a stage to
// the producer, so compute warps never wait for one another. Each compute
// warp writes its outputs into its own swizzled box and stores it by TMA.
constexpr int kF64Rows = 32;
constexpr int kF64Compute = 4;                 // compute warps
constexpr int kF64Threads = 32 * (kF64Compute + 1);
constexpr int kF64Box = kF64Rows * 16;         // doubles of one [32][16] box (4 KB)
constexpr int kF64Stages = 2;
constexpr int kF64StageBoxes = 8;              // a: 4 boxes, b: 4 boxes
// + 1024 bytes to align the boxes to the 1024-byte period of the 128-byte swizzle
// Output area of a compute warp: the swizzled [32][16] box of the TMA store, or
// (accumulating launches) 32 per-lane slots of 16 doubles at an 18-double
// stride (16-byte aligned, conflict-free 16-byte writes); 5 KB keeps every box
// on the 1024-byte period of the swizzle.
constexpr int kF64OutArea = kF64Box;              // doubles per compute warp (one output box, 4 KB)
constexpr size_t kF64Smem =
    ((size_t)kF64Stages * kF64StageBoxes * kF64Box + (size_t)kF64Compute * kF64OutArea) * sizeof(double) + 1024;

struct F64BlockSigns {
    uint16_t alpha[4][4];  // [L0][O0] bit i: a_{16 L0 + i} enters block (L0, O0) negated
    uint16_t beta[4][4];   // [L0][O0] bit k: block (L0, O0) adds to y_{16 O0 + k} negated
    uint16_t bflip[4];     // [L0 ^ O0] bit j: b_{16 (L0 ^ O0) + j} is negated on load (VJP operands)
};

// Sign of e_i e_k over axes 0..3 with negative-metric mask NEG (bit a: axis a negative).
__host__ __device__ constexpr int low_sign(int i, int k, int neg) {
    int s = 1;
    for (int a = 0; a < 4; ++a) {
        if ((i >> a) & 1) {
            int lower = k & ((1 << a) - 1), c = 0;
            for (; lower; lower &= lower - 1) ++c;
            if (c & 1) s = -s;
            if (((k >> a) & 1) && ((neg >> a) & 1)) s = -s;
        }
    }
    return s;
}

// acc[k] += sum_i gamma(i, k) a[i] b[i ^ k] with compile-time indices and signs.
template <int NEG, int I>
__device__ __forceinline__ void f64_block_term(const double (&a)[16], const double (&b)[16], double (&acc)[16]) {
    constexpr int i = I / 16, k = I % 16;
    constexpr int sg = low_sign(i, k, NEG);
    acc[k] = fma(sg > 0 ? a[i] : -a[i], b[i ^ k], acc[k]);
}
template <int NEG, int... I>
__device__ __forceinline__ void f64_block(const double (&a)[16], const double (&b)[16], double (&acc)[16],
                                          std::integer_sequence<int, I...>) {
    (f64_block_term<NEG, I>(a, b, acc), ...);
}

__device__ __forceinline__ double flip_bit(double v, unsigned bit) {
    return __hiloint2double(__double2hiint(v) ^ (int)(bit << 31), __double2loint(v));
}

// Double offset of (row, 16-byte chunk j) in a [32][16] float64 box with the 128-byte swizzle.
__device__ __forceinline__ int sw128d(int row, int chunk) { return row * 16 + ((chunk ^ (row & 7)) << 1); }

// PRODUCTS = 1: y = a b. PRODUCTS = 2 (the JVP): y = a b + a2 b2 in one pass;
// the ring alternates (a, b) and (a2, b2) tiles of the same rows and the
// compute warps keep one accumulator across both before the single store.
// (A compile-time count: a run-time one cost the plain product 4%.)
//
// Every wait is bounded by `wait_limit` polls. A compute warp whose wait gives
// up (or that finds the CTA aborted) raises the CTA's abort flag, writes NaN
// into its 16 output columns of every row it has not stored and ends; the
// producer stops issuing once the flag is up or its own wait gives up, and
// before it ends waits (bounded) for the loads it issued, so no copy into the
// CTA's shared memory outlives the CTA. STARVE (the wait self-test only)
// issues no load at all.
template <int NEG, int PRODUCTS, bool STARVE = false>
__global__ void __launch_bounds__(kF64Threads, 2)
pairwise_f64_n6_tma_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                           const __grid_constant__ CUtensorMap map_a2, const __grid_constant__ CUtensorMap map_b2,
                           const __grid_constant__ CUtensorMap map_out, const F64BlockSigns signs,
                           double *__restrict__ out, size_t batch, uint32_t wait_limit) {
    constexpr int products = PRODUCTS;
    extern __shared__ unsigned char f64_raw[];
    __shared__ __align__(8) uint64_t full[kF64Stages], empty[kF64Stages];
    __shared__ F64BlockSigns sgn;
    __shared__ volatile int s_abort;
    double *base = reinterpret_cast<double *>(((uintptr_t)f64_raw + 1023) & ~(uintptr_t)1023);
    double *outbox = base + kF64Stages * kF64StageBoxes * kF64Box;  // one output area per compute warp
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t tiles = (batch + kF64Rows - 1) / kF64Rows;
    const int K = (size_t)blockIdx.x < tiles ? (int)((tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    if (tid == 0) {
        for (int s = 0; s < kF64Stages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(&full[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(&empty[s])), "r"(kF64Compute)
                         : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        sgn = signs;
        s_abort = 0;
    }
    __syncthreads();
    if (warp == kF64Compute) {
        // ---- producer: one thread keeps the ring full
        if (lane == 0 && !STARVE) {
            // stage loads v = 0, 1, ...: tile v / products, operand pair v % products
            int issued = 0;
            for (int v = 0; v < K * products; ++v) {
                const int s = v % kF64Stages;
                // the stage last held load v - kF64Stages: wait until all compute warps released it
                if (v >= kF64Stages &&
                    !tma_bounded_wait(&empty[s], (unsigned)((v / kF64Stages - 1) & 1), wait_limit)) {
                    s_abort = 1;
                    atomicAdd(&g_pairwise_tma_wait_failures, 1u);
                }
                if (s_abort) break;
                double *st = base + s * kF64StageBoxes * kF64Box;
                const int y = (int)((blockIdx.x + (size_t)(v / products) * gridDim.x) * kF64Rows);
                const bool second = v % products != 0;
                const CUtensorMap *ma = second ? &map_a2 : &map_a;
                const CUtensorMap *mb = second ? &map_b2 : &map_b;
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(&full[s])),
                             "r"((unsigned)(kF64StageBoxes * kF64Box * sizeof(double)))
                             : "memory");
                for (int c = 0; c < 4; ++c) {
                    tma_load_2d(st + c * kF64Box, ma, 16 * c, y, &full[s]);
                    tma_load_2d(st + (4 + c) * kF64Box, mb, 16 * c, y, &full[s]);
                }
                issued = v + 1;
            }
            // Every load before issued - kF64Stages completed before its stage was
            // reissued; wait for the last one of each stage.
            for (int v = issued > kF64Stages ? issued - kF64Stages : 0; v < issued; ++v)
                (void)tma_bounded_wait(&full[v % kF64Stages], (unsigned)((v / kF64Stages) & 1), wait_limit);
        }
        return;
    }
    // ---- compute warps
    double *ob = outbox + warp * kF64OutArea;
    for (int k = 0; k < K; ++k) {
        double acc[16];
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) acc[kk] = 0.0;
        unsigned prev = 0u;
        bool failed = false;
#pragma unroll 1
        for (int p = 0; p < products; ++p) {
            const int v = k * products + p;
            const int s = v % kF64Stages;
            const bool ok = tma_bounded_wait(&full[s], (unsigned)((v / kF64Stages) & 1), wait_limit);
            if (__any_sync(0xffffffffu, !ok) || s_abort) {
                failed = true;
                break;
            }
            const double *A = base + s * kF64StageBoxes * kF64Box;
            const double *Bm = A + 4 * kF64Box;
#pragma unroll
            for (int L0 = 0; L0 < 4; ++L0) {
                const unsigned am = sgn.alpha[L0][warp], bm = sgn.beta[L0][warp];
                double av[16], bv[16];
                const double *ab = A + L0 * kF64Box;
                const double *bb = Bm + (L0 ^ warp) * kF64Box;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const double2 u = *reinterpret_cast<const double2 *>(&ab[sw128d(lane, j)]);
                    const double2 v = *reinterpret_cast<const double2 *>(&bb[sw128d(lane, j)]);
                    av[2 * j] = u.x; av[2 * j + 1] = u.y;
                    bv[2 * j] = v.x; bv[2 * j + 1] = v.y;
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) av[i] = flip_bit(av[i], (am >> i) & 1u);
                const unsigned bf = sgn.bflip[L0 ^ warp];
                if (bf != 0u) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) bv[j] = flip_bit(bv[j], (bf >> j) & 1u);
                }
                const unsigned fm = bm ^ prev;
#pragma unroll
                for (int kk = 0; kk < 16; ++kk) acc[kk] = flip_bit(acc[kk], (fm >> kk) & 1u);
                prev = bm;
                f64_block<NEG>(av, bv, acc, std::make_integer_sequence<int, 256>{});
            }
            // The warp is done reading stage s.
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(&empty[s])) : "memory");
        }
        if (failed) {
            // Abort: NaN into this warp's columns of tiles k..K-1 (plain stores),
            // then let this warp's pending tensor stores finish.
            if (lane == 0) {
                s_abort = 1;
                atomicAdd(&g_pairwise_tma_wait_failures, 1u);
            }
            for (int j = k; j < K; ++j) {
                const size_t row = (blockIdx.x + (size_t)j * gridDim.x) * kF64Rows + (size_t)lane;
                if (row < batch)
                    for (int c = 0; c < 16; ++c) out[row * 64 + 16 * warp + c] = __longlong_as_double(0x7ff8000000000000ll);
            }
            break;
        }
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) acc[kk] = flip_bit(acc[kk], (prev >> kk) & 1u);
        const size_t row0 = (blockIdx.x + (size_t)k * gridDim.x) * kF64Rows;
        // The store of tile k - 1 from this warp's box must have finished reading it.
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
            *reinterpret_cast<double2 *>(&ob[sw128d(lane, j)]) = make_double2(acc[2 * j], acc[2 * j + 1]);
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(&map_out, 16 * warp, (int)row0, ob);
            asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
        }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
}

// [rows][64] float64 tensor, [32][16] boxes, 128-byte swizzle, zero fill.
bool encode_rows_f64(CUtensorMap *map, const double *ptr, size_t rows) {
    const auto encode = tensor_map_encoder();
    if (encode == nullptr || rows == 0 || rows > 0xffffffffull) return false;
    const cuuint64_t dims[2] = {64, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {64 * sizeof(double)};
    const cuuint32_t box[2] = {16, (cuuint32_t)kF64Rows};
    const cuuint32_t elem[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double *>(ptr), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// alpha / beta of the block factorisation for a 6-dimensional signature;
// false (use the generic kernel) if sigma does not factor as alpha beta gamma.
// rev_a / rev_b multiply operand blade m of a / b by s(m, m) (the operands of
// the VJP products).
bool f64_block_signs(const geo::SignPlan &plan, int neg_low, bool rev_a, bool rev_b, F64BlockSigns *out) {
    // plan.neg[l] bit p: s(l, p) = -1 (parameter-on-right plan: sigma(i, p) = s(i, p)).
    auto sigma = [&](int l, int o) { return ((plan.neg[l] >> (l ^ o)) & 1ull) ? -1 : 1; };
    auto self_negative = [&](int m) { return ((plan.neg[m] >> m) & 1ull) != 0; };  // s(m, m) = -1
    for (int c = 0; c < 4; ++c) {
        uint16_t f = 0;
        for (int j = 0; rev_b && j < 16; ++j)
            if (self_negative(16 * c + j)) f |= (uint16_t)(1u << j);
        out->bflip[c] = f;
    }
    for (int L0 = 0; L0 < 4; ++L0)
        for (int O0 = 0; O0 < 4; ++O0) {
            int alpha[16], beta[16];
            for (int i = 0; i < 16; ++i) alpha[i] = sigma(16 * L0 + i, 16 * O0);
            for (int k = 0; k < 16; ++k) beta[k] = sigma(16 * L0, 16 * O0 + k) * alpha[0];
            uint16_t am = 0, bm = 0;
            for (int i = 0; i < 16; ++i) {
                if ((alpha[i] < 0) != (rev_a && self_negative(16 * L0 + i))) am |= (uint16_t)(1u << i);
                for (int k = 0; k < 16; ++k)
                    if (sigma(16 * L0 + i, 16 * O0 + k) != alpha[i] * beta[k] * low_sign(i, k, neg_low)) return false;
            }
            for (int k = 0; k < 16; ++k)
                if (beta[k] < 0) bm |= (uint16_t)(1u << k);
            out->alpha[L0][O0] = am;
            out->beta[L0][O0] = bm;
        }
    return true;
}

template <int NEG, bool STARVE = false>
cudaError_t launch_f64_tma_neg(const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &ma2,
                               const CUtensorMap &mb2, const CUtensorMap &mo, const F64BlockSigns &signs, double *out,
                               size_t batch, int products, cudaStream_t stream, uint32_t wait_limit = kTmaWaitLimit) {
    auto kernel = products == 2 ? pairwise_f64_n6_tma_kernel<NEG, 2, STARVE> : pairwise_f64_n6_tma_kernel<NEG, 1, STARVE>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kF64Smem);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kF64Threads, kF64Smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const size_t tiles = (batch + kF64Rows - 1) / kF64Rows;
    size_t grid = (size_t)geo::device_sm_count() * (size_t)per_sm;
    if (grid > tiles) grid = tiles;
    kernel<<<(unsigned)grid, kF64Threads, kF64Smem, stream>>>(ma, mb, ma2, mb2, mo, signs, out, batch, wait_limit);
    return cudaGetLastError();
}

template <int... NEG>
cudaError_t launch_f64_tma_dispatch(int neg, const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &ma2,
                                    const CUtensorMap &mb2, const CUtensorMap &mo, const F64BlockSigns &signs,
                                    double *out, size_t batch, int products, cudaStream_t stream,
                                    std::integer_sequence<int, NEG...>) {
    cudaError_t e = cudaErrorInvalidValue;
    ((neg == NEG ? (e = launch_f64_tma_neg<NEG>(ma, mb, ma2, mb2, mo, signs, out, batch, products, stream), true)
                 : false) ||
     ...);
    return e;
}


// ---- float64 n = 6 through the matrix representation (canonical D = 16 algebras)
// y = a b as Y' = A' rho(b) (geo::make_pair_tables: 1024 multiply-adds per
// product instead of 4096) for Cl(6,0), Cl(5,1), Cl(2,4) and Cl(1,5), whose
// tables are compile-time data (pair_tables_gen.h, written by
// gen/gen_pair_tables.cpp from the same host code): blade offsets are immediates
// and signs are negations inside the multiply-adds. A product is handled by four
// lanes of a warp, lane l one kept row: it forms its 16 coefficients Ah[m] of a
// from broadcast reads of the raw row (the four lanes read the same words; the
// lane enters only through the signs (-1)^{popc(c & l)}, applied as exact +-1
// multiply-adds), then for every group g of b a Walsh transform of the
// lane-signed members and 16 multiply-adds into Yh[u]; a Walsh transform of
// Yh[g] across the four lanes (shfl.xor) leaves output blade[g][c] in lane c.
// Operand rows arrive by 512-byte bulk copies into rows of 66 doubles (528 B):
// the eight rows a warp reads at once fall in eight distinct bank pairs, so
// every broadcast read is one wavefront. The ring (2 stages, producer warp,
// full / empty mbarriers, bounded waits, abort protocol) is the one of
// pairwise_f64_n6_tma_kernel; outputs are written over the product's a row of
// the (last) stage and leave by one 512-byte bulk store per row.
struct PairTablesC {
    unsigned char blade[16][4], xa[16][4], xb[16][4], post[16][4], chi[16][2];
};
constexpr PairTablesC kPairTables[4][4] = GEO_PAIR_TABLES_INIT;

constexpr int kPrRows = 32;                  // products per tile
constexpr int kPrPitch = 66;                 // doubles per staged row
constexpr int kPrCompute = 4;                // compute warps, 8 products each
constexpr int kPrThreads = 32 * (kPrCompute + 1);
constexpr int kPrStages = 2;
constexpr int kPrStage = 2 * kPrRows * kPrPitch;   // doubles per stage (a rows, b rows)
constexpr size_t kPrSmem = (size_t)kPrStages * kPrStage * sizeof(double) + 16;

template <int... I, typename F>
__device__ __forceinline__ void static_for_seq(std::integer_sequence<int, I...>, F &&f) {
    (f(std::integral_constant<int, I>{}), ...);
}
template <int N, typename F>
__device__ __forceinline__ void static_for(F &&f) {
    static_for_seq(std::make_integer_sequence<int, N>{}, f);
}

__device__ __forceinline__ void bulk_load_1d(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void bulk_store_1d(void *dst, const void *src, unsigned bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst), "r"(smem_u32(src)),
                 "r"(bytes)
                 : "memory");
}

template <int SI, int REV, int PRODUCTS, bool STARVE = false>
__global__ void __launch_bounds__(kPrThreads, 3)
pairwise_rep_kernel(const double *__restrict__ a1, const double *__restrict__ b1, const double *__restrict__ a2,
                    const double *__restrict__ b2, double *__restrict__ out, size_t batch, uint32_t wait_limit) {
    extern __shared__ unsigned char pr_raw[];
    __shared__ __align__(8) uint64_t full[kPrStages], empty[kPrStages];
    __shared__ volatile int s_abort;
    double *base = reinterpret_cast<double *>(((uintptr_t)pr_raw + 15) & ~(uintptr_t)15);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t tiles = (batch + kPrRows - 1) / kPrRows;
    const int K = (size_t)blockIdx.x < tiles ? (int)((tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    if (tid == 0) {
        for (int st = 0; st < kPrStages; ++st) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(&full[st])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(&empty[st])), "r"(kPrCompute)
                         : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        s_abort = 0;
    }
    __syncthreads();
    if (warp == kPrCompute) {
        // ---- producer: one thread keeps the ring full (row copies of a and b)
        if (lane == 0 && !STARVE) {
            int issued = 0;
            for (int v = 0; v < K * PRODUCTS; ++v) {
                const int st = v % kPrStages;
                if (v >= kPrStages &&
                    !tma_bounded_wait(&empty[st], (unsigned)((v / kPrStages - 1) & 1), wait_limit)) {
                    s_abort = 1;
                    atomicAdd(&g_pairwise_tma_wait_failures, 1u);
                }
                if (s_abort) break;
                double *sa = base + st * kPrStage;
                const size_t row0 = (blockIdx.x + (size_t)(v / PRODUCTS) * gridDim.x) * kPrRows;
                const int rows = batch - row0 < (size_t)kPrRows ? (int)(batch - row0) : kPrRows;
                const bool second = v % PRODUCTS != 0;
                const double *ga = (second ? a2 : a1) + row0 * 64;
                const double *gb = (second ? b2 : b1) + row0 * 64;
                // (also orders the compute warps' writes of the stage before the reload)
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(&full[st])),
                             "r"((unsigned)(2 * rows * 512))
                             : "memory");
                for (int r = 0; r < rows; ++r) {
                    bulk_load_1d(sa + r * kPrPitch, ga + r * 64, 512u, &full[st]);
                    bulk_load_1d(sa + (kPrRows + r) * kPrPitch, gb + r * 64, 512u, &full[st]);
                }
                issued = v + 1;
            }
            for (int v = issued > kPrStages ? issued - kPrStages : 0; v < issued; ++v)
                (void)tma_bounded_wait(&full[v % kPrStages], (unsigned)((v / kPrStages) & 1), wait_limit);
        }
        return;
    }
    // ---- compute warps
    const int ps = lane >> 2, l = lane & 3;
    const int prow = warp * 8 + ps;  // product row within the tile
    // The lane's signs (-1)^{popc(c & l)}: member 1 by s1, member 2 by s2, member 3
    // by s1 s2, as multiplies by +-1 inside fused multiply-adds (exact: each sum
    // rounds as a plain add).
    const double s1 = (l & 1) ? -1.0 : 1.0, s2 = (l & 2) ? -1.0 : 1.0;
    for (int k = 0; k < K; ++k) {
        double yh[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) yh[u] = 0.0;
        bool failed = false;
        int last_st = 0;
#pragma unroll 1
        for (int pp = 0; pp < PRODUCTS; ++pp) {
            const int v = k * PRODUCTS + pp;
            const int st = v % kPrStages;
            const bool ok = tma_bounded_wait(&full[st], (unsigned)((v / kPrStages) & 1), wait_limit);
            if (__any_sync(0xffffffffu, !ok) || s_abort) {
                failed = true;
                break;
            }
            const double *ra = base + st * kPrStage + prow * kPrPitch;
            const double *rb = ra + kPrRows * kPrPitch;
            double ah[16];
            static_for<16>([&](auto mI) {
                constexpr int m = decltype(mI)::value;
                const double *pa = ra;
                double w[4];
                static_for<4>([&](auto cI) {
                    constexpr int c = decltype(cI)::value;
                    constexpr int blade = kPairTables[SI][REV].blade[m][c];
                    constexpr bool neg = kPairTables[SI][REV].xa[m][c] != 0;
                    const double x = pa[blade];
                    w[c] = neg ? -x : x;
                });
                // (w0 + s1 w1) + (s2 w2 + s1 s2 w3)
                ah[m] = fma(s2, fma(s1, w[3], w[2]), fma(s1, w[1], w[0]));
            });
            static_for<16>([&](auto gI) {
                constexpr int g = decltype(gI)::value;
                const double *pb = rb;
                double w[4];
                static_for<4>([&](auto cI) {
                    constexpr int c = decltype(cI)::value;
                    constexpr int blade = kPairTables[SI][REV].blade[g][c];
                    constexpr bool neg = kPairTables[SI][REV].xb[g][c] != 0;
                    const double x = pb[blade];
                    w[c] = neg ? -x : x;
                });
                // Walsh transform of (w0, s1 w1, s2 w2, s1 s2 w3)
                const double e0 = fma(s1, w[1], w[0]), f0 = fma(-s1, w[1], w[0]);
                const double e1 = fma(s1, w[3], w[2]), f1 = fma(-s1, w[3], w[2]);
                const double bt[4] = {fma(s2, e1, e0), fma(s2, f1, f0), fma(-s2, e1, e0), fma(-s2, f1, f0)};
                static_for<16>([&](auto uI) {
                    constexpr int u = decltype(uI)::value;
                    constexpr int uh = u >> 2;
                    constexpr bool h1 = kPairTables[SI][REV].chi[g][0] != 0;
                    constexpr bool h2 = kPairTables[SI][REV].chi[g][1] != 0;
                    constexpr bool neg = uh == 0 ? false : uh == 1 ? h1 : uh == 2 ? h2 : h1 != h2;
                    yh[u] = fma(ah[g ^ u], neg ? -bt[u & 3] : bt[u & 3], yh[u]);
                });
            });
            __syncwarp();
            last_st = st;
            if (pp + 1 < PRODUCTS && lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(&empty[st])) : "memory");
        }
        const size_t row0 = (blockIdx.x + (size_t)k * gridDim.x) * kPrRows;
        if (failed) {
            // Abort: NaN into this warp's product rows of tiles k..K-1 (plain stores).
            if (lane == 0) {
                s_abort = 1;
                atomicAdd(&g_pairwise_tma_wait_failures, 1u);
            }
            for (int j = k; j < K; ++j) {
                const size_t row = (blockIdx.x + (size_t)j * gridDim.x) * kPrRows + (size_t)prow;
                if (row < batch)
                    for (int c = 0; c < 16; ++c) out[row * 64 + 16 * l + c] = __longlong_as_double(0x7ff8000000000000ll);
            }
            break;
        }
        // Walsh transform of Yh[g] across the four lanes of the product.
#pragma unroll
        for (int h = 1; h < 4; h <<= 1) {
            const double sg = (l & h) ? -1.0 : 1.0;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const double o = __shfl_xor_sync(0xffffffffu, yh[u], h);
                yh[u] = fma(sg, yh[u], o);
            }
        }
        // Outputs over this product's a row of the last stage (no lane reads it any
        // more): lane l holds blade[g][l] of every group g.
        double *ro = base + last_st * kPrStage + prow * kPrPitch;
        static_for<16>([&](auto gI) {
            constexpr int g = decltype(gI)::value;
            constexpr int B0 = kPairTables[SI][REV].blade[g][0], B1 = kPairTables[SI][REV].blade[g][1];
            constexpr int B2 = kPairTables[SI][REV].blade[g][2], B3 = kPairTables[SI][REV].blade[g][3];
            constexpr bool P0 = kPairTables[SI][REV].post[g][0] != 0, P1 = kPairTables[SI][REV].post[g][1] != 0;
            constexpr bool P2 = kPairTables[SI][REV].post[g][2] != 0, P3 = kPairTables[SI][REV].post[g][3] != 0;
            const int bl = l == 0 ? B0 : l == 1 ? B1 : l == 2 ? B2 : B3;
            const bool pn = l == 0 ? P0 : l == 1 ? P1 : l == 2 ? P2 : P3;
            ro[bl] = (pn ? -yh[g] : yh[g]) * 0.25;  // exact
        });
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncwarp();
        if (lane == 0) {
            for (int q = 0; q < 8; ++q) {
                const size_t row = row0 + (size_t)(warp * 8 + q);
                if (row < batch)
                    bulk_store_1d(out + row * 64, base + last_st * kPrStage + (warp * 8 + q) * kPrPitch, 512u);
            }
            asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
            // The stage is reloaded only after the stores have read it.
            asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(&empty[last_st])) : "memory");
        }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
}

// Index of a canonical D = 16 signature in the generated tables, or -1.
int pair_table_index(const int8_t *signature) {
    unsigned mask = 0;
    for (unsigned a = 0; a < 6; ++a)
        if (signature[a] < 0) mask |= 1u << a;
    switch (mask) {
        case 0x00u: return 0;  // Cl(6,0)
        case 0x20u: return 1;  // Cl(5,1)
        case 0x3Cu: return 2;  // Cl(2,4)
        case 0x3Eu: return 3;  // Cl(1,5)
        default: return -1;
    }
}

template <int SI, int REV, int PRODUCTS, bool STARVE = false>
cudaError_t launch_pair_rep_t(const double *a1, const double *b1, const double *a2, const double *b2, double *out,
                              size_t batch, cudaStream_t stream, uint32_t wait_limit) {
    auto kernel = pairwise_rep_kernel<SI, REV, PRODUCTS, STARVE>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPrSmem);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kPrThreads, kPrSmem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const size_t tiles = (batch + kPrRows - 1) / kPrRows;
    size_t grid = (size_t)geo::device_sm_count() * (size_t)per_sm;
    if (grid > tiles) grid = tiles;
    kernel<<<(unsigned)grid, kPrThreads, kPrSmem, stream>>>(a1, b1, a2, b2, out, batch, wait_limit);
    return cudaGetLastError();
}

template <int SI>
cudaError_t launch_pair_rep_si(int rev, int products, const double *a1, const double *b1, const double *a2,
                               const double *b2, double *out, size_t batch, cudaStream_t stream) {
    if (products == 2) return launch_pair_rep_t<SI, 0, 2>(a1, b1, a2, b2, out, batch, stream, kTmaWaitLimit);
    switch (rev) {
        case 1: return launch_pair_rep_t<SI, 1, 1>(a1, b1, a2, b2, out, batch, stream, kTmaWaitLimit);
        case 2: return launch_pair_rep_t<SI, 2, 1>(a1, b1, a2, b2, out, batch, stream, kTmaWaitLimit);
        default: return launch_pair_rep_t<SI, 0, 1>(a1, b1, a2, b2, out, batch, stream, kTmaWaitLimit);
    }
}

// out = left right (or + left2 right2, the JVP) through the representation;
// false when it does not apply (a canonical D = 16 signature, 16-byte aligned
// operands; the JVP without operand reversal).
bool launch_pairwise_rep(const int8_t *signature, const double *left, const double *right, double *out, size_t batch,
                         cudaStream_t stream, cudaError_t *err, bool rev_left, bool rev_right, const double *left2,
                         const double *right2) {
    const bool two = left2 != nullptr && right2 != nullptr;
    if (((uintptr_t)left | (uintptr_t)right | (uintptr_t)out) & 15u) return false;
    if (two && (((uintptr_t)left2 | (uintptr_t)right2) & 15u || rev_left || rev_right)) return false;
    if (rev_left && rev_right) return false;
    const int si = pair_table_index(signature);
    if (si < 0) return false;
    const int rev = (rev_left ? 1 : 0) | (rev_right ? 2 : 0);
    const double *a2 = two ? left2 : left, *b2 = two ? right2 : right;
    const int products = two ? 2 : 1;
    switch (si) {
        case 0: *err = launch_pair_rep_si<0>(rev, products, left, right, a2, b2, out, batch, stream); break;
        case 1: *err = launch_pair_rep_si<1>(rev, products, left, right, a2, b2, out, batch, stream); break;
        case 2: *err = launch_pair_rep_si<2>(rev, products, left, right, a2, b2, out, batch, stream); break;
        default: *err = launch_pair_rep_si<3>(rev, products, left, right, a2, b2, out, batch, stream); break;
    }
    return true;
}

// float64 n = 6 forward on the TMA kernel, out = left right, or with left2 and
// right2 given out = left right + left2 right2 in one pass (the JVP); false when
// it does not apply (unaligned operands, no tensor-map encoder, sign table that
// does not factor).
bool launch_pairwise_f64_fast(const geo::SignPlan &plan, const int8_t *signature, const double *left,
                              const double *right, double *out, size_t batch, cudaStream_t stream, cudaError_t *err,
                              bool rev_left = false, bool rev_right = false, const double *left2 = nullptr,
                              const double *right2 = nullptr) {
    if (plan.blades == 64 && launch_pairwise_rep(signature, left, right, out, batch, stream, err, rev_left, rev_right,
                                                 left2, right2))
        return true;
    const bool two = left2 != nullptr && right2 != nullptr;
    if (plan.blades != 64 || ((uintptr_t)left | (uintptr_t)right | (uintptr_t)out) & 15u) return false;
    if (two && ((uintptr_t)left2 | (uintptr_t)right2) & 15u) return false;
    int neg_low = 0;
    for (int a = 0; a < 4; ++a)
        if (signature[a] < 0) neg_low |= 1 << a;
    F64BlockSigns signs;
    if (!f64_block_signs(plan, neg_low, rev_left, rev_right, &signs)) return false;
    CUtensorMap ma, mb, ma2, mb2, mo;
    if (!encode_rows_f64(&ma, left, batch) || !encode_rows_f64(&mb, right, batch) || !encode_rows_f64(&mo, out, batch))
        return false;
    if (two ? (!encode_rows_f64(&ma2, left2, batch) || !encode_rows_f64(&mb2, right2, batch)) : false) return false;
    if (!two) {
        ma2 = ma;
        mb2 = mb;
    }
    *err = launch_f64_tma_dispatch(neg_low, ma, mb, ma2, mb2, mo, signs, out, batch, two ? 2 : 1, stream,
                                   std::make_integer_sequence<int, 16>{});
    return true;
}

template <typename T, int MODE>
geo_b200_status_t launch_pairwise(uint8_t dimension, const int8_t *signature, const T *left, int left_compact,
                                  const T *right, const T *aux0, const T *aux1, T *out0, T *out1, size_t batch,
                                  cudaStream_t stream) {
    if (!geo::dimension_valid(dimension)) return GEO_B200_UNSUPPORTED_DIMENSION;
    const geo::SignPlan *plan = geo::cached_sign_plan(dimension, signature, 0);
    if (plan == nullptr || left == nullptr || right == nullptr || batch == 0) return GEO_B200_INVALID_ARGUMENT;
    if (left_compact && dimension < 1) return GEO_B200_INVALID_ARGUMENT;
    const int N = plan->blades;
    const int per_pass = kThreads / N;
    const size_t smem = (size_t)4 * per_pass * N * sizeof(T);
    size_t grid = (batch + per_pass - 1) / per_pass;
    const size_t cap = (size_t)geo::device_sm_count() * 8;
    if (grid > cap) grid = cap;
    pairwise_kernel<T, MODE><<<(unsigned)grid, kThreads, smem, stream>>>(*plan, left, left_compact, right, aux0,
                                                                         aux1, out0, out1, batch);
    return from_cuda(cudaGetLastError());
}

}  // namespace

extern "C" geo_b200_status_t geo_b200_pairwise_gp_f64(uint8_t dimension, const int8_t *signature,
                                                      const double *device_left, const double *device_right,
                                                      double *device_out, size_t batch, cudaStream_t stream) {
    if (device_out == nullptr) return GEO_B200_INVALID_ARGUMENT;
    if (dimension == 6 && device_left != nullptr && device_right != nullptr && batch > 0) {
        const geo::SignPlan *plan = geo::cached_sign_plan(6, signature, 0);
        cudaError_t e = cudaSuccess;
        if (plan != nullptr && launch_pairwise_f64_fast(*plan, signature, device_left, device_right, device_out,
                                                        batch, stream, &e))
            return from_cuda(e);
    }
    return launch_pairwise<double, kPairForward>(dimension, signature, device_left, 0, device_right, nullptr, nullptr,
                                                 device_out, nullptr, batch, stream);
}

extern "C" geo_b200_status_t geo_b200_pairwise_gp_vjp_f64(uint8_t dimension, const int8_t *signature,
                                                          const double *device_left, const double *device_right,
                                                          const double *device_out_cotangent,
                                                          double *device_left_cotangent,
                                                          double *device_right_cotangent, size_t batch,
                                                          cudaStream_t stream) {
    if (device_out_cotangent == nullptr || (device_left_cotangent == nullptr && device_right_cotangent == nullptr))
        return GEO_B200_INVALID_ARGUMENT;
    // n = 6: two forward products on the TMA kernel. With y = a b and
    // m~ = s(m, m) m per blade (the transpose of multiplication by e_m is s(m, m)
    // times itself): a_bar = y_bar b~ and b_bar = a~ y_bar.
    const geo::SignPlan *plan = dimension == 6 ? geo::cached_sign_plan(6, signature, 0) : nullptr;
    const bool al = ((uintptr_t)device_left | (uintptr_t)device_right | (uintptr_t)device_out_cotangent |
                     (uintptr_t)device_left_cotangent | (uintptr_t)device_right_cotangent) % 16u == 0u;
    if (plan != nullptr && al && device_left != nullptr && device_right != nullptr && batch > 0 &&
        tensor_map_encoder() != nullptr) {
        cudaError_t e = cudaSuccess;
        bool ran = true;
        if (device_left_cotangent != nullptr)
            ran = launch_pairwise_f64_fast(*plan, signature, device_out_cotangent, device_right, device_left_cotangent,
                                           batch, stream, &e, false, true);
        if (ran && e == cudaSuccess && device_right_cotangent != nullptr)
            ran = launch_pairwise_f64_fast(*plan, signature, device_left, device_out_cotangent,
                                           device_right_cotangent, batch, stream, &e, true, false);
        if (ran) return from_cuda(e);
    }
    return launch_pairwise<double, kPairVjp>(dimension, signature, device_left, 0, device_right, device_out_cotangent,
                                             nullptr, device_left_cotangent, device_right_cotangent, batch, stream);
}

extern "C" geo_b200_status_t geo_b200_pairwise_gp_jvp_f64(uint8_t dimension, const int8_t *signature,
                                                          const double *device_left, const double *device_right,
                                                          const double *device_left_tangent,
                                                          const double *device_right_tangent,
                                                          double *device_out_tangent, size_t batch,
                                                          cudaStream_t stream) {
    if (device_left_tangent == nullptr || device_right_tangent == nullptr || device_out_tangent == nullptr)
        return GEO_B200_INVALID_ARGUMENT;
    // n = 6: one pass of the TMA kernel over both products, out = a_dot b + a b_dot
    // (one accumulator per output across both).
    const geo::SignPlan *plan = dimension == 6 ? geo::cached_sign_plan(6, signature, 0) : nullptr;
    const bool al = ((uintptr_t)device_left | (uintptr_t)device_right | (uintptr_t)device_left_tangent |
                     (uintptr_t)device_right_tangent | (uintptr_t)device_out_tangent) % 16u == 0u;
    if (plan != nullptr && al && device_left != nullptr && device_right != nullptr && batch > 0 &&
        tensor_map_encoder() != nullptr) {
        cudaError_t e = cudaSuccess;
        if (launch_pairwise_f64_fast(*plan, signature, device_left_tangent, device_right, device_out_tangent, batch,
                                     stream, &e, false, false, device_left, device_right_tangent))
            return from_cuda(e);
    }
    return launch_pairwise<double, kPairJvp>(dimension, signature, device_left, 0, device_right, device_left_tangent,
                                             device_right_tangent, device_out_tangent, nullptr, batch, stream);
}

extern "C" geo_b200_status_t geo_b200_pairwise_gp_f32(uint8_t dimension, const int8_t *signature,
                                                      const float *device_left, int left_even_compact,
                                                      const float *device_right, float *device_out, size_t batch,
                                                      cudaStream_t stream) {
    if (device_out == nullptr) return GEO_B200_INVALID_ARGUMENT;
    if (dimension == 6 && signature != nullptr && device_left != nullptr && device_right != nullptr && batch > 0 &&
        geo::signature_valid(signature, 6)) {
        cudaError_t e = cudaSuccess;
        if (launch_pairwise_f32_fast(signature, device_left, left_even_compact != 0, device_right, device_out, batch,
                                     stream, &e))
            return from_cuda(e);
    }
    return launch_pairwise<float, kPairForward>(dimension, signature, device_left, left_even_compact != 0,
                                                device_right, nullptr, nullptr, device_out, nullptr, batch, stream);
}

extern "C" geo_b200_status_t geo_b200_pairwise_wait_failures(unsigned *count, int reset) {
    if (count == nullptr) return GEO_B200_INVALID_ARGUMENT;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(count, g_pairwise_tma_wait_failures, sizeof(unsigned));
    if (e == cudaSuccess && reset) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_pairwise_tma_wait_failures, &zero, sizeof(unsigned));
    }
    if (e != cudaSuccess) return from_cuda(e);
    return *count != 0 ? GEO_B200_TIMEOUT : GEO_B200_OK;
}

extern "C" geo_b200_status_t geo_b200_pairwise_wait_selftest(int precision, void *device_out, size_t batch,
                                                             uint32_t wait_limit, cudaStream_t stream) {
    if (device_out == nullptr || batch == 0 || wait_limit == 0 || (precision != 32 && precision != 64) ||
        ((uintptr_t)device_out & 15u) != 0 || tensor_map_encoder() == nullptr)
        return GEO_B200_INVALID_ARGUMENT;
    unsigned before = 0;
    geo_b200_status_t st = geo_b200_pairwise_wait_failures(&before, 1);
    if (st != GEO_B200_OK && st != GEO_B200_TIMEOUT) return st;
    cudaError_t e = cudaSuccess;
    if (precision == 64) {
        double *out = static_cast<double *>(device_out);
        // The representation kernel first (Cl(6,0) tables), then the direct one.
        e = launch_pair_rep_t<0, 0, 1, true>(out, out, out, out, out, batch, stream, wait_limit);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return from_cuda(e);
        unsigned first = 0;
        st = geo_b200_pairwise_wait_failures(&first, 1);
        if (st != GEO_B200_TIMEOUT) return st == GEO_B200_OK ? GEO_B200_RUNTIME_FAILURE : st;
        CUtensorMap m;
        if (!encode_rows_f64(&m, out, batch)) return GEO_B200_INVALID_ARGUMENT;
        F64BlockSigns signs;
        memset(&signs, 0, sizeof signs);
        e = launch_f64_tma_neg<0, true>(m, m, m, m, m, signs, out, batch, 1, stream, wait_limit);
    } else {
        float *out = static_cast<float *>(device_out);
        CUtensorMap m;
        if (!encode_rows(&m, out, 64, batch)) return GEO_B200_INVALID_ARGUMENT;
        e = launch_f32_tma<0, false, true>(m, m, m, out, batch, stream, wait_limit);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return from_cuda(e);
    unsigned count = 0;
    return geo_b200_pairwise_wait_failures(&count, 1);
}
