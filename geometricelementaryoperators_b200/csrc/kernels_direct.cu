// kernels_direct.cu -- sm_100a streaming kernels for the batched geometric
// product with a fixed parameter multivector W (any n = 1..6, any diagonal
// signature, parameter on either side).
//
// Math (reference src/batch_gp.c:107-201, written as matrices):
//   Y = X M          with M[i][o] = W[i^o] * sigma(i, i^o)
//   C = X^T R        (reduced over the batch)
//   g[p] = sum_i sigma(i, p) C[i][i^p]
// where X, Y, R are sample-major [batch][2^n] float64 arrays and sigma is the
// baked sign of SignPlan. A training step fuses Y, R = Y - T, the loss
// sum 0.5 r^2 and C into one pass over X and T (R never touches HBM unless the
// caller asks for it), so each step streams 2 x 8 x 2^n bytes per sample.
//
// Structure of the tiled kernels (2^n >= 8):
//   * persistent CTAs of 256 threads walk tiles of TS samples;
//   * each tile of X and T is staged into padded shared memory with 16-byte
//     cp.async copies, double-buffered so the next tile streams in while the
//     current one is computed;
//   * phase A: register-blocked FP64 GEMM Y = X M (M built once per CTA in
//     shared memory), then R = Y - T written back over T, loss and finiteness
//     probes accumulated in registers;
//   * phase B: register-blocked FP64 GEMM C += X^T R; C stays in registers for
//     the life of the CTA;
//   * epilogue: C copies summed in shared memory, folded into the per-CTA
//     gradient record g[p]; a finalize kernel sums records in CTA order, so
//     the result is deterministic (no floating-point atomics anywhere).
// Thread layout inside a warp: OG output groups x IG sample/row groups, chosen
// so every shared-memory read is either a broadcast or conflict-free.
#include <cuda_runtime.h>
#include <math.h>

#include "geo_internal.h"

namespace geo {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ void cp_async_16(void *smem, const void *gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_8(void *smem, const void *gmem, int src_bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int Pending>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(Pending) : "memory");
}

// Tile geometry for the register-blocked kernels.
template <int N>
struct Tiled {
    static_assert(N >= 8 && N <= 64, "tiled kernels cover 8..64 blades");
    static constexpr int OG = (N / 2 < 8) ? N / 2 : 8;  // output (column-pair) groups per warp
    static constexpr int IG = 32 / OG;                  // sample groups (A) / row groups (B)
    static constexpr int QC = N / (2 * OG);             // column pairs per thread
    static constexpr int TS = (N == 64) ? 64 : 128;     // samples per tile
    static constexpr int A = TS / (IG * kWarps);        // samples per thread in phase A
    static constexpr int RU = (N == 8) ? 1 : 4;         // rows per thread in phase B
    static constexpr int ROWS_PER_WARP = IG * RU;
    static constexpr int WARPS_PER_COPY = N / ROWS_PER_WARP;
    static constexpr int COPIES = kWarps / WARPS_PER_COPY;
    static constexpr int LD = N + 2;                    // padded row stride (doubles)
    static constexpr int TILE_DOUBLES = TS * LD;
    static_assert(A >= 1 && TS % (IG * kWarps) == 0, "phase A layout");
    static_assert(ROWS_PER_WARP <= N && N % ROWS_PER_WARP == 0, "phase B layout");
    static_assert(kWarps % WARPS_PER_COPY == 0 && TS % COPIES == 0, "phase B copies");
};

// Stage samples [first, first + TS) of a sample-major array into a padded tile.
template <int N, int TS, int LD, bool ALIGNED16>
__device__ __forceinline__ void stage_tile(double *tile, const double *__restrict__ src, size_t first,
                                           size_t batch) {
    if (ALIGNED16) {
        constexpr int CH = N / 2;  // 16-byte chunks per row
        for (int c = threadIdx.x; c < TS * CH; c += kThreads) {
            const int s = c / CH;
            const int k2 = c - s * CH;
            const size_t sample = first + (size_t)s;
            const bool ok = sample < batch;
            const double *g = ok ? src + sample * N + 2 * k2 : src;
            cp_async_16(tile + s * LD + 2 * k2, g, ok ? 16 : 0);
        }
    } else {
        for (int c = threadIdx.x; c < TS * N; c += kThreads) {
            const int s = c / N;
            const int k = c - s * N;
            const size_t sample = first + (size_t)s;
            const bool ok = sample < batch;
            const double *g = ok ? src + sample * N + k : src;
            cp_async_8(tile + s * LD + k, g, ok ? 8 : 0);
        }
    }
}

// M[i][o] = W[i^o] * sigma(i, i^o), row-major [N][N] in shared memory.
template <int N>
__device__ __forceinline__ void build_multiplier(double *Ms, const double *__restrict__ parameter,
                                                 const SignPlan &plan) {
    for (int idx = threadIdx.x; idx < N * N; idx += kThreads) {
        const int i = idx / N;
        const int o = idx - i * N;
        const int p = i ^ o;
        const double w = parameter[p];
        Ms[idx] = ((plan.neg[i] >> p) & 1ull) ? -w : w;
    }
}

// Deterministic block reduction of `count` per-thread values (count <= 8).
template <int COUNT>
__device__ __forceinline__ void block_sum(double (&v)[COUNT], double *scratch /* kThreads*COUNT */) {
    for (int c = 0; c < COUNT; ++c) scratch[c * kThreads + threadIdx.x] = v[c];
    __syncthreads();
    for (int width = kThreads / 2; width > 0; width >>= 1) {
        if (threadIdx.x < width) {
            for (int c = 0; c < COUNT; ++c) {
                scratch[c * kThreads + threadIdx.x] += scratch[c * kThreads + threadIdx.x + width];
            }
        }
        __syncthreads();
    }
    for (int c = 0; c < COUNT; ++c) v[c] = scratch[c * kThreads];
    __syncthreads();
}

enum KernelMode : int { kModeForward = 0, kModeCycle = 1, kModeVjp = 2 };

// ---------------------------------------------------------------------------
// Tiled kernel (N >= 8). MODE selects forward-only, full cycle or VJP-only.
//   forward: in = X, out = Y
//   cycle:   in = X, aux = T, out = residuals (optional), records
//   vjp:     in = X, aux = cotangents, records
template <int N, int MODE, bool ALIGNED16>
__global__ void __launch_bounds__(kThreads, 1)
tiled_kernel(const SignPlan plan, const double *__restrict__ in, const double *__restrict__ aux,
             const double *__restrict__ parameter, double *__restrict__ out, size_t batch,
             double *__restrict__ records) {
    using G = Tiled<N>;
    constexpr int TS = G::TS, LD = G::LD, OG = G::OG, IG = G::IG, QC = G::QC, A = G::A, RU = G::RU;
    constexpr bool kHasAux = MODE != kModeForward;
    constexpr bool kPhaseA = MODE != kModeVjp;
    constexpr bool kPhaseB = MODE != kModeForward;

    extern __shared__ __align__(16) double smem[];
    double *Ms = smem;                                   // N*N
    double *Xb = Ms + N * N;                             // 2 tiles
    double *Tb = Xb + 2 * G::TILE_DOUBLES;               // 2 tiles (T/cotangent, then R)

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int og = lane % OG;
    const int gq = lane / OG;  // sample group (phase A) / row group (phase B)

    if (kPhaseA) build_multiplier<N>(Ms, parameter, plan);

    const size_t tiles = (batch + TS - 1) / TS;
    size_t tile = blockIdx.x;
    int buf = 0;
    if (tile < tiles) {
        stage_tile<N, TS, LD, ALIGNED16>(Xb, in, tile * TS, batch);
        if (kHasAux) stage_tile<N, TS, LD, ALIGNED16>(Tb, aux, tile * TS, batch);
    }
    cp_async_commit();

    double loss = 0.0, check_y = 0.0, check_r = 0.0;
    double cacc[RU][QC][2];
#pragma unroll
    for (int u = 0; u < RU; ++u)
#pragma unroll
        for (int q = 0; q < QC; ++q) cacc[u][q][0] = cacc[u][q][1] = 0.0;

    for (; tile < tiles; tile += gridDim.x) {
        const size_t next = tile + gridDim.x;
        if (next < tiles) {
            stage_tile<N, TS, LD, ALIGNED16>(Xb + (buf ^ 1) * G::TILE_DOUBLES, in, next * TS, batch);
            if (kHasAux) stage_tile<N, TS, LD, ALIGNED16>(Tb + (buf ^ 1) * G::TILE_DOUBLES, aux, next * TS, batch);
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();

        double *Xs = Xb + buf * G::TILE_DOUBLES;
        double *Ts = Tb + buf * G::TILE_DOUBLES;
        const size_t first = tile * TS;

        if (kPhaseA) {
            // Phase A: Y = X M for samples s_j = warp*IG*A + gq + IG*j.
            double acc[A][QC][2];
#pragma unroll
            for (int j = 0; j < A; ++j)
#pragma unroll
                for (int q = 0; q < QC; ++q) acc[j][q][0] = acc[j][q][1] = 0.0;
            const int sbase = warp * IG * A + gq;
#pragma unroll 4
            for (int k = 0; k < N; ++k) {
                double xv[A];
#pragma unroll
                for (int j = 0; j < A; ++j) xv[j] = Xs[(sbase + IG * j) * LD + k];
                double2 mv[QC];
#pragma unroll
                for (int q = 0; q < QC; ++q)
                    mv[q] = *reinterpret_cast<const double2 *>(&Ms[k * N + 2 * og + 2 * OG * q]);
#pragma unroll
                for (int j = 0; j < A; ++j)
#pragma unroll
                    for (int q = 0; q < QC; ++q) {
                        acc[j][q][0] = fma(xv[j], mv[q].x, acc[j][q][0]);
                        acc[j][q][1] = fma(xv[j], mv[q].y, acc[j][q][1]);
                    }
            }
#pragma unroll
            for (int j = 0; j < A; ++j) {
                const int s = sbase + IG * j;
                const size_t sample = first + (size_t)s;
#pragma unroll
                for (int q = 0; q < QC; ++q) {
                    const int o = 2 * og + 2 * OG * q;
                    if (MODE == kModeForward) {
                        if (sample < batch) {
                            if (ALIGNED16) {
                                *reinterpret_cast<double2 *>(&out[sample * N + o]) =
                                    make_double2(acc[j][q][0], acc[j][q][1]);
                            } else {  // 8-byte aligned output: scalar stores only
                                out[sample * N + o] = acc[j][q][0];
                                out[sample * N + o + 1] = acc[j][q][1];
                            }
                        }
                    } else {
                        const double2 t = *reinterpret_cast<const double2 *>(&Ts[s * LD + o]);
                        double2 r;
                        r.x = acc[j][q][0] - t.x;
                        r.y = acc[j][q][1] - t.y;
                        // Padding samples have x = t = 0, hence y = r = 0: no effect on sums.
                        *reinterpret_cast<double2 *>(&Ts[s * LD + o]) = r;
                        loss = fma(0.5 * r.x, r.x, loss);
                        loss = fma(0.5 * r.y, r.y, loss);
                        check_y = fma(acc[j][q][0], 0.0, check_y);
                        check_y = fma(acc[j][q][1], 0.0, check_y);
                        check_r = fma(r.x, 0.0, check_r);
                        check_r = fma(r.y, 0.0, check_r);
                        if (out != nullptr && sample < batch) {
                            if (ALIGNED16) {
                                *reinterpret_cast<double2 *>(&out[sample * N + o]) = r;
                            } else {
                                out[sample * N + o] = r.x;
                                out[sample * N + o + 1] = r.y;
                            }
                        }
                    }
                }
            }
            if (kPhaseB) __syncthreads();
        }

        if (kPhaseB) {
            // Phase B: C += X^T R over this copy's share of the tile.
            constexpr int SPC = TS / G::COPIES;
            const int copy = warp / G::WARPS_PER_COPY;
            const int rbase = (warp % G::WARPS_PER_COPY) * G::ROWS_PER_WARP + gq;
            const int s0 = copy * SPC;
#pragma unroll 2
            for (int s = s0; s < s0 + SPC; ++s) {
                double xv[RU];
#pragma unroll
                for (int u = 0; u < RU; ++u) xv[u] = Xs[s * LD + rbase + IG * u];
                double2 rv[QC];
#pragma unroll
                for (int q = 0; q < QC; ++q)
                    rv[q] = *reinterpret_cast<const double2 *>(&Ts[s * LD + 2 * og + 2 * OG * q]);
#pragma unroll
                for (int u = 0; u < RU; ++u)
#pragma unroll
                    for (int q = 0; q < QC; ++q) {
                        cacc[u][q][0] = fma(xv[u], rv[q].x, cacc[u][q][0]);
                        cacc[u][q][1] = fma(xv[u], rv[q].y, cacc[u][q][1]);
                    }
            }
        }
        __syncthreads();
        buf ^= 1;
    }
    cp_async_wait<0>();
    __syncthreads();

    if (MODE == kModeForward) return;

    // Epilogue: sum the C copies in copy order, fold into g, reduce loss/probes.
    double *Cs = Xb;  // COPIES * N * N doubles; tile buffers are free now
    {
        const int copy = warp / G::WARPS_PER_COPY;
        const int rbase = (warp % G::WARPS_PER_COPY) * G::ROWS_PER_WARP + gq;
#pragma unroll
        for (int u = 0; u < RU; ++u)
#pragma unroll
            for (int q = 0; q < QC; ++q) {
                const int i = rbase + IG * u;
                const int o = 2 * og + 2 * OG * q;
                Cs[(copy * N + i) * N + o] = cacc[u][q][0];
                Cs[(copy * N + i) * N + o + 1] = cacc[u][q][1];
            }
    }
    __syncthreads();
    double *rec = records + (size_t)blockIdx.x * kRecStride;
    if (threadIdx.x < N) {
        const int p = threadIdx.x;
        double g = 0.0;
        for (int i = 0; i < N; ++i) {
            double c = 0.0;
            for (int copy = 0; copy < G::COPIES; ++copy) c += Cs[(copy * N + i) * N + (i ^ p)];
            g += ((plan.neg[i] >> p) & 1ull) ? -c : c;
        }
        rec[p] = g;
    }
    __syncthreads();
    double red[3] = {loss, check_y, check_r};
    block_sum<3>(red, Cs + G::COPIES * N * N);
    if (threadIdx.x == 0) {
        rec[kRecLoss] = red[0];
        rec[kRecCheckY] = red[1];
        rec[kRecCheckR] = red[2];
        rec[kRecCheckIn] = 0.0;
    }
}

// ---------------------------------------------------------------------------
// Small kernel (N = 2, 4): one thread per sample, everything in registers.
template <int N, int MODE>
__global__ void __launch_bounds__(kThreads)
small_kernel(const SignPlan plan, const double *__restrict__ in, const double *__restrict__ aux,
             const double *__restrict__ parameter, double *__restrict__ out, size_t batch,
             double *__restrict__ records) {
    __shared__ double Ms[N * N];
    __shared__ double scratch[kThreads * 4];
    if (MODE != kModeVjp) build_multiplier<N>(Ms, parameter, plan);
    __syncthreads();

    double cacc[N][N];
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
        for (int o = 0; o < N; ++o) cacc[i][o] = 0.0;
    double loss = 0.0, check_y = 0.0, check_r = 0.0;

    const size_t stride = (size_t)gridDim.x * kThreads;
    for (size_t s = (size_t)blockIdx.x * kThreads + threadIdx.x; s < batch; s += stride) {
        double x[N], r[N];
#pragma unroll
        for (int k = 0; k < N; ++k) x[k] = in[s * N + k];
        if (MODE == kModeVjp) {
#pragma unroll
            for (int k = 0; k < N; ++k) r[k] = aux[s * N + k];
        } else {
#pragma unroll
            for (int o = 0; o < N; ++o) {
                double y = 0.0;
#pragma unroll
                for (int i = 0; i < N; ++i) y = fma(x[i], Ms[i * N + o], y);
                if (MODE == kModeForward) {
                    out[s * N + o] = y;
                } else {
                    r[o] = y - aux[s * N + o];
                    loss = fma(0.5 * r[o], r[o], loss);
                    check_y = fma(y, 0.0, check_y);
                    check_r = fma(r[o], 0.0, check_r);
                    if (out != nullptr) out[s * N + o] = r[o];
                }
            }
        }
        if (MODE != kModeForward) {
#pragma unroll
            for (int i = 0; i < N; ++i)
#pragma unroll
                for (int o = 0; o < N; ++o) cacc[i][o] = fma(x[i], r[o], cacc[i][o]);
        }
    }
    if (MODE == kModeForward) return;

    double red[4];
    double *rec = records + (size_t)blockIdx.x * kRecStride;
    double g[N];
#pragma unroll
    for (int p = 0; p < N; ++p) {
        double acc = 0.0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const double c = cacc[i][i ^ p];
            acc += ((plan.neg[i] >> p) & 1ull) ? -c : c;
        }
        g[p] = acc;
    }
    static_assert(N <= 4, "small kernel reduction width");
#pragma unroll
    for (int p = 0; p < 4; ++p) red[p] = p < N ? g[p] : 0.0;
    block_sum<4>(red, scratch);
    if (threadIdx.x == 0) {
#pragma unroll
        for (int p = 0; p < N; ++p) rec[p] = red[p];
    }
    double red2[3] = {loss, check_y, check_r};
    block_sum<3>(red2, scratch);
    if (threadIdx.x == 0) {
        rec[kRecLoss] = red2[0];
        rec[kRecCheckY] = red2[1];
        rec[kRecCheckR] = red2[2];
        rec[kRecCheckIn] = 0.0;
    }
}

// ---------------------------------------------------------------------------
// Ordered sum of `count` records into totals[kRecStride] with kRecThreads
// threads: thread (slot, part) sums a contiguous chunk of records, then the
// kRecParts chunk sums are added in chunk order. Deterministic.
constexpr int kRecParts = 8;
constexpr int kRecThreads = kRecStride * kRecParts;  // 576

__device__ __forceinline__ void ordered_record_sum(const double *__restrict__ records, int count,
                                                   double *totals /* smem kRecStride */,
                                                   double *parts /* smem kRecThreads */) {
    const int t = threadIdx.x;
    if (t < kRecThreads) {
        const int slot = t % kRecStride;
        const int part = t / kRecStride;
        const int chunk = (count + kRecParts - 1) / kRecParts;
        const int lo = part * chunk;
        const int hi = min(count, lo + chunk);
        // Loads in batches of 8 (independent, in flight together); the sum
        // itself stays sequential in record order.
        double acc = 0.0;
        int c = lo;
        for (; c + 8 <= hi; c += 8) {
            double v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = records[(size_t)(c + u) * kRecStride + slot];
#pragma unroll
            for (int u = 0; u < 8; ++u) acc += v[u];
        }
        for (; c < hi; ++c) acc += records[(size_t)c * kRecStride + slot];
        parts[part * kRecStride + slot] = acc;
    }
    __syncthreads();
    if (t < kRecStride) {
        double acc = 0.0;
        for (int p = 0; p < kRecParts; ++p) acc += parts[p * kRecStride + t];
        totals[t] = acc;
    }
    __syncthreads();
}

// Finalize: ordered sum of CTA records, status probes, optimizer (transactional).
__global__ void __launch_bounds__(kRecThreads)
finalize_kernel(const double *__restrict__ records, int ctas, const OptimizerArgs opt,
                double *__restrict__ gradient_out, double *__restrict__ loss_sum_out,
                double *__restrict__ parameter, double *__restrict__ first_moment,
                double *__restrict__ second_moment, uint32_t *__restrict__ status,
                unsigned long long *__restrict__ step_counter) {
    __shared__ double totals[kRecStride];
    __shared__ double parts[kRecThreads];
    // A failure recorded by an earlier step on this stream blocks later updates
    // until the host clears the status word (transactional chain).
    const bool blocked = status != nullptr && opt.kind != kOptNone && opt.kind != kOptSgdScaled && *status != 0u;
    const int t = threadIdx.x;
    ordered_record_sum(records, ctas, totals, parts);
    const int blades = opt.blades;
    const double loss = totals[kRecLoss];
    const bool bad_y = !isfinite(totals[kRecCheckY]);
    const bool bad_r = !isfinite(totals[kRecCheckR]);
    const bool active = t < blades;
    const double g = active ? totals[t] : 0.0;
    const bool bad_g = __syncthreads_or(active && !isfinite(g)) != 0;
    if (active && gradient_out != nullptr) gradient_out[t] = g;
    if (t == 0 && loss_sum_out != nullptr) *loss_sum_out = loss;

    uint32_t bits = 0u;
    if (bad_y) bits |= kDevOutputNonFinite;
    if (bad_r) bits |= kDevResidualNonFinite;
    if (bad_g) bits |= kDevGradientNonFinite;

    if (opt.kind == kOptSgdScaled) {
        // Device ABI semantics: parameter -= scale * gradient with scale = lr / B
        // computed on the host; applied whatever the values, like the reference.
        if (active) parameter[t] = __dsub_rn(parameter[t], __dmul_rn(opt.learning_rate, g));
    } else if (opt.kind != kOptNone && bits == 0u && !blocked) {
        // Candidate update, mirrored operation for operation from the CPU path
        // (no FMA contraction: __dmul_rn/__dadd_rn keep each rounding separate).
        double w = active ? parameter[t] : 0.0;
        double m = 0.0, v = 0.0;
        bool bad = false;
        if (opt.kind == kOptSgdBatchGp) {
            // reference src/batch_gp.c:295-304: w - lr * g / B
            w = __dsub_rn(w, __ddiv_rn(__dmul_rn(opt.learning_rate, g), opt.batch_divisor));
        } else {
            const double gs = __dmul_rn(g, opt.gradient_scale);
            double update = gs;
            if (opt.kind == kOptAdamV8) {
                // reference src/full_cycle_v8.c:996-1008
                m = active ? first_moment[t] : 0.0;
                v = active ? second_moment[t] : 0.0;
                const double first = __dadd_rn(__dmul_rn(opt.beta1, m), __dmul_rn(__dsub_rn(1.0, opt.beta1), gs));
                const double second =
                    __dadd_rn(__dmul_rn(opt.beta2, v), __dmul_rn(__dmul_rn(__dsub_rn(1.0, opt.beta2), gs), gs));
                bad = !isfinite(first) || !isfinite(second);
                m = first;
                v = second;
                update = __ddiv_rn(__ddiv_rn(first, opt.bias1),
                                   __dadd_rn(__dsqrt_rn(__ddiv_rn(second, opt.bias2)), opt.epsilon));
            }
            w = __dsub_rn(w, __dmul_rn(opt.learning_rate, update));
        }
        bad = bad || !isfinite(w);
        const bool any_bad = __syncthreads_or(active && bad) != 0;
        if (any_bad) {
            bits |= kDevCandidateNonFinite;
        } else if (active) {
            parameter[t] = w;
            if (opt.kind == kOptAdamV8) {
                first_moment[t] = m;
                second_moment[t] = v;
            }
        }
        if (!any_bad && opt.kind == kOptSgdBatchGp && !isfinite(loss / opt.batch_divisor))
            bits |= kDevLossNonFinite;
        if (!any_bad && t == 0 && step_counter != nullptr) *step_counter += 1ull;
    }
    if (t == 0 && status != nullptr && bits != 0u) atomicOr(status, bits);
}

__global__ void __launch_bounds__(kRecThreads)
reduce_records_kernel(const double *__restrict__ records, int count, double *__restrict__ out, int accumulate) {
    __shared__ double totals[kRecStride];
    __shared__ double parts[kRecThreads];
    ordered_record_sum(records, count, totals, parts);
    const int t = threadIdx.x;
    if (t < kRecStride) out[t] = accumulate ? out[t] + totals[t] : totals[t];
}

__global__ void check_finite_kernel(const double *__restrict__ values, size_t count, uint32_t bit,
                                    uint32_t *__restrict__ status) {
    bool bad = false;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
        bad = bad || !isfinite(values[i]);
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(status, bit);
}

// ---------------------------------------------------------------------------
template <int N, int MODE, bool AL>
cudaError_t launch_tiled_impl(const SignPlan &plan, const double *in, const double *aux,
                              const double *parameter, double *out, size_t batch, double *records,
                              int *ctas_used, cudaStream_t stream) {
    using G = Tiled<N>;
    auto kernel = tiled_kernel<N, MODE, AL>;
    const size_t smem = (size_t)(N * N + 4 * G::TILE_DOUBLES) * sizeof(double);
    static bool configured[2] = {false, false};
    (void)configured;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const size_t tiles = (batch + G::TS - 1) / G::TS;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    size_t grid = (size_t)device_sm_count() * (size_t)per_sm;
    if (grid > (size_t)kMaxCtas) grid = kMaxCtas;
    if (grid > tiles) grid = tiles;
    if (grid < 1) grid = 1;
    kernel<<<(unsigned)grid, kThreads, smem, stream>>>(plan, in, aux, parameter, out, batch, records);
    if (ctas_used) *ctas_used = (int)grid;
    return cudaGetLastError();
}

template <int N, int MODE>
cudaError_t launch_small_impl(const SignPlan &plan, const double *in, const double *aux,
                              const double *parameter, double *out, size_t batch, double *records,
                              int *ctas_used, cudaStream_t stream) {
    size_t blocks = (batch + kThreads - 1) / kThreads;
    const size_t cap = (size_t)device_sm_count() * 4;
    if (blocks > cap) blocks = cap;
    if (blocks > (size_t)kMaxCtas) blocks = kMaxCtas;
    if (blocks < 1) blocks = 1;
    small_kernel<N, MODE><<<(unsigned)blocks, kThreads, 0, stream>>>(plan, in, aux, parameter, out, batch, records);
    if (ctas_used) *ctas_used = (int)blocks;
    return cudaGetLastError();
}

template <int MODE>
cudaError_t dispatch(const SignPlan &plan, const double *in, const double *aux, const double *parameter,
                     double *out, size_t batch, double *records, int *ctas_used, cudaStream_t stream) {
    uintptr_t bits = (uintptr_t)in | (uintptr_t)aux | (uintptr_t)out;
    const bool al = (bits & 15u) == 0u;
    switch (plan.blades) {
        case 2: return launch_small_impl<2, MODE>(plan, in, aux, parameter, out, batch, records, ctas_used, stream);
        case 4: return launch_small_impl<4, MODE>(plan, in, aux, parameter, out, batch, records, ctas_used, stream);
#define GEO_TILED_CASE(NB)                                                                                      \
    case NB:                                                                                                    \
        return al ? launch_tiled_impl<NB, MODE, true>(plan, in, aux, parameter, out, batch, records, ctas_used, \
                                                      stream)                                                   \
                  : launch_tiled_impl<NB, MODE, false>(plan, in, aux, parameter, out, batch, records,           \
                                                       ctas_used, stream);
        GEO_TILED_CASE(8)
        GEO_TILED_CASE(16)
        GEO_TILED_CASE(32)
        GEO_TILED_CASE(64)
#undef GEO_TILED_CASE
        default: return cudaErrorInvalidValue;
    }
}

// One CTA per tile (no persistent loop), so the record count is known from the
// batch alone; used when the caller supplies a fixed-size record buffer.
template <int N, bool AL>
cudaError_t launch_tiled_vjp_per_tile(const SignPlan &plan, const double *in, const double *aux, size_t batch,
                                      double *records, int max_records, int *ctas_used, cudaStream_t stream) {
    using G = Tiled<N>;
    auto kernel = tiled_kernel<N, kModeVjp, AL>;
    const size_t tiles = (batch + G::TS - 1) / G::TS;
    if (tiles < 1 || tiles > (size_t)max_records) return cudaErrorInvalidValue;
    const size_t smem = (size_t)(N * N + 4 * G::TILE_DOUBLES) * sizeof(double);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kernel<<<(unsigned)tiles, kThreads, smem, stream>>>(plan, in, aux, nullptr, nullptr, batch, records);
    if (ctas_used) *ctas_used = (int)tiles;
    return cudaGetLastError();
}

template <int N>
cudaError_t launch_small_vjp_per_tile(const SignPlan &plan, const double *in, const double *aux, size_t batch,
                                      double *records, int max_records, int *ctas_used, cudaStream_t stream) {
    const size_t blocks = (batch + kThreads - 1) / kThreads;
    if (blocks < 1 || blocks > (size_t)max_records) return cudaErrorInvalidValue;
    small_kernel<N, kModeVjp><<<(unsigned)blocks, kThreads, 0, stream>>>(plan, in, aux, nullptr, nullptr, batch,
                                                                         records);
    if (ctas_used) *ctas_used = (int)blocks;
    return cudaGetLastError();
}

}  // namespace

size_t vjp_tile_samples(int blades) {
    switch (blades) {
        case 2:
        case 4: return kThreads;
        case 8: return Tiled<8>::TS;
        case 16: return Tiled<16>::TS;
        case 32: return Tiled<32>::TS;
        case 64: return Tiled<64>::TS;
        default: return 0;
    }
}

cudaError_t launch_vjp_per_tile(const SignPlan &plan, const double *inputs, const double *cotangents, size_t batch,
                                double *records, int max_records, int *ctas_used, cudaStream_t stream) {
    const bool al = (((uintptr_t)inputs | (uintptr_t)cotangents) & 15u) == 0u;
    switch (plan.blades) {
        case 2: return launch_small_vjp_per_tile<2>(plan, inputs, cotangents, batch, records, max_records, ctas_used, stream);
        case 4: return launch_small_vjp_per_tile<4>(plan, inputs, cotangents, batch, records, max_records, ctas_used, stream);
#define GEO_TILE_CASE(NB)                                                                                         \
    case NB:                                                                                                      \
        return al ? launch_tiled_vjp_per_tile<NB, true>(plan, inputs, cotangents, batch, records, max_records,   \
                                                        ctas_used, stream)                                      \
                  : launch_tiled_vjp_per_tile<NB, false>(plan, inputs, cotangents, batch, records, max_records,  \
                                                         ctas_used, stream);
        GEO_TILE_CASE(8)
        GEO_TILE_CASE(16)
        GEO_TILE_CASE(32)
        GEO_TILE_CASE(64)
#undef GEO_TILE_CASE
        default: return cudaErrorInvalidValue;
    }
}

int device_sm_count() {
    int dev = 0, count = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || count <= 0)
        return 148;
    return count;
}

cudaError_t launch_forward(const SignPlan &plan, const double *inputs, const double *parameter, double *outputs,
                           size_t batch, cudaStream_t stream) {
    return dispatch<kModeForward>(plan, inputs, nullptr, parameter, outputs, batch, nullptr, nullptr, stream);
}

cudaError_t launch_cycle(const SignPlan &plan, CycleMode mode, const double *inputs,
                         const double *targets_or_cotangents, const double *parameter, double *residuals_out,
                         size_t batch, double *records, int *ctas_used, cudaStream_t stream) {
    if (mode == kCycle)
        return dispatch<kModeCycle>(plan, inputs, targets_or_cotangents, parameter, residuals_out, batch, records,
                                    ctas_used, stream);
    return dispatch<kModeVjp>(plan, inputs, targets_or_cotangents, parameter, nullptr, batch, records, ctas_used,
                              stream);
}

cudaError_t launch_finalize(const double *records, int ctas, const OptimizerArgs &opt, double *gradient_out,
                            double *loss_sum_out, double *parameter, double *first_moment, double *second_moment,
                            uint32_t *status, cudaStream_t stream, unsigned long long *step_counter) {
    finalize_kernel<<<1, kRecThreads, 0, stream>>>(records, ctas, opt, gradient_out, loss_sum_out, parameter, first_moment,
                                           second_moment, status, step_counter);
    return cudaGetLastError();
}

cudaError_t launch_reduce_records(const double *records, int count, double *out, cudaStream_t stream,
                                  int accumulate) {
    reduce_records_kernel<<<1, kRecThreads, 0, stream>>>(records, count, out, accumulate);
    return cudaGetLastError();
}

cudaError_t launch_check_finite(const double *values, size_t count, uint32_t bit, uint32_t *status,
                                cudaStream_t stream) {
    size_t blocks = (count + 255) / 256;
    const size_t cap = (size_t)device_sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    check_finite_kernel<<<(unsigned)blocks, 256, 0, stream>>>(values, count, bit, status);
    return cudaGetLastError();
}

}  // namespace geo
