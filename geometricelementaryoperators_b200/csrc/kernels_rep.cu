// kernels_rep.cu -- fused training pass on FP64 tensor cores through a real
// matrix representation of the algebra (see representation.h).
//
// Per sample s (2^n blades, S kept rows of a D x D representation, S*D = 2^n):
//   X'_s = P x_s,  T'_s = P t_s              signed gathers (S terms each)
//   Y'_s = X'_s W',  R'_s = Y'_s - T'_s       S x D times D x D   (GEMM 1)
//   loss += |R'_s|^2 / (2S)
//   G'  += X'_s^T R'_s                         D x D, reduced over the batch (GEMM 2)
// and once per CTA: g_A = <G', rho(e_A)> / S (or rho(e_A)^T for the left side).
// This is the reference's forward -> residual -> 0.5 r^2 -> parameter VJP
// (src/batch_gp.c:237-308) with the 4^n-term Cayley product replaced by an
// S*D*D GEMM: Cl(6,0)-type algebras use D = 16, S = 4 (1024 multiply-adds per
// GEMM per sample instead of 4096), Cl(3,3)-type D = 8, S = 8 (512).
//
// Data movement per tile of TS samples (HBM traffic = x and t read once):
//   * cp.async copies of the raw x and t rows into one of kStages shared-memory
//     stages, issued kStages-1 tiles ahead (two CTAs per SM keep ~128 KB of
//     loads in flight per SM);
//   * gather in place: each thread loads the S blades of its blade group for
//     its samples into registers, the CTA synchronises, then the S kept
//     entries are written over the raw rows (a transformed sample is again
//     2^n doubles), in an XOR-swizzled layout;
//   * per 16-row block, a warp runs GEMM 1 with mma.sync.m16n8k4.f64 (W'
//     fragments resident in registers), forms R' = Y' - T' in place, and GEMM 2
//     reading X'^T straight from shared memory as the A operand.
// The swizzles make every fragment load, every gather load and the epilogue
// accesses hit each shared-memory bank at most twice per warp instruction.
#include <cuda_runtime.h>
#include <math.h>

#include "geo_internal.h"
#include "rep_layout.h"
#include "representation.h"

namespace geo {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr int kStages = 3;

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

// D(16x8) += A(16x4) * B(4x8), float64 tensor cores.
// Fragments (g = lane / 4, t = lane % 4): a0 = A[g][t], a1 = A[g+8][t];
// b0 = B[t][g]; c0,c1 = C[g][2t, 2t+1], c2,c3 = C[g+8][2t, 2t+1].
__device__ __forceinline__ void mma_16x8x4(double (&c)[4], double a0, double a1, double b0) {
    asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
                 : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
                 : "d"(a0), "d"(a1), "d"(b0));
}

template <int D, int S>
struct RepGeo {
    static constexpr int N = D * S;         // blades (= doubles per sample, raw or transformed)
    static constexpr int TS = 32;           // samples per tile
    static constexpr int ROWS = TS * S;     // X' rows per tile
    static constexpr int BLOCKS = ROWS / 16;
    static constexpr int NT = D / 8;        // 8-column tiles of the D outputs
    static constexpr int KT = D / 4;        // k-steps of GEMM 1
    static constexpr int TILE = TS * N;     // doubles of one raw tile (x or t)
    static constexpr int STAGE = 2 * TILE;  // x tile + t tile
    static_assert(ROWS % 16 == 0 && D % 8 == 0, "tile shape");
};

// Column swizzle of the transformed (X', T', R') rows, keyed by the row within
// the tile: conflict-free GEMM-1 A loads (rows g, cols 4kt + t), GEMM-2 A/B
// loads (rows 4kk + t, cols g) and 16-byte epilogue accesses.
template <int D>
__device__ __forceinline__ int xsw(int row) {
    if (D == 16) return 4 * (2 * (row & 1) + ((row >> 2) & 1));
    return 4 * ((row >> 1) & 1);
}
// Raw-row swizzle: for D = 8 (four samples per gather load) odd samples swap
// their 64-byte halves so the four samples cover all 16 double-banks.
template <int D>
__device__ __forceinline__ int rsw(int sample) {
    return D == 8 ? 8 * (sample & 1) : 0;
}

template <int D, int S, bool AL>
__device__ __forceinline__ void stage_tile(double *dst, const double *__restrict__ src, size_t first, size_t batch) {
    using G = RepGeo<D, S>;
    constexpr int N = G::N;
    if (AL) {
        for (int c = threadIdx.x; c < G::TS * (N / 2); c += kThreads) {
            const int s = c / (N / 2);
            const int k = 2 * (c - s * (N / 2));
            const size_t sample = first + (size_t)s;
            const bool ok = sample < batch;
            const double *g = ok ? src + sample * N + k : src;
            cp_async_16(dst + s * N + (k ^ rsw<D>(s)), g, ok ? 16 : 0);
        }
    } else {
        for (int c = threadIdx.x; c < G::TS * N; c += kThreads) {
            const int s = c / N;
            const int k = c - s * N;
            const size_t sample = first + (size_t)s;
            const bool ok = sample < batch;
            const double *g = ok ? src + sample * N + k : src;
            cp_async_8(dst + s * N + (k ^ rsw<D>(s)), g, ok ? 8 : 0);
        }
    }
}

template <int D, int S, bool AL>
__global__ void __launch_bounds__(kThreads, 2)
rep_cycle_kernel(const RepDevice rep, const double *__restrict__ X, const double *__restrict__ T,
                 const double *__restrict__ W, size_t batch, double *__restrict__ records) {
    using G = RepGeo<D, S>;
    constexpr int N = G::N, TS = G::TS;
    extern __shared__ __align__(16) double smem[];
    double *Wp = smem;                     // D*D
    double *stages = Wp + D * D;           // kStages x (x tile, t tile)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;

    // This thread's blade group for the gathers, resident for the whole kernel.
    constexpr int SLICES = kThreads / D;
    const int gm = threadIdx.x % D;
    const int gslice = threadIdx.x / D;
    int gblade[S], gcol[S];
#pragma unroll
    for (int t = 0; t < S; ++t) {
        gblade[t] = rep.grp_blade[gm][t];
        gcol[t] = rep.grp_col[gm][t];
    }
    const uint64_t gneg = rep.grp_neg[gm];

    // W' = rho(W) (right) or rho(W)^T (left): W'[k][j] = sum_{A: x_A = k^j} W_A sg_A (-1)^{z_A . col}
    for (int idx = threadIdx.x; idx < D * D; idx += kThreads) {
        const int k = idx / D, j = idx - k * D;
        const int col = rep.side ? k : j;
        double acc = 0.0;
        for (int A = 0; A < N; ++A) {
            if (rep.xm[A] != (k ^ j)) continue;
            const double w = W[A];
            const bool neg = (rep.sg[A] < 0) != ((__popc(rep.zm[A] & col) & 1) != 0);
            acc += neg ? -w : w;
        }
        Wp[idx] = acc;
    }

    const size_t tiles = (batch + TS - 1) / TS;
    // Prologue: issue the first kStages-1 tiles of this CTA.
#pragma unroll
    for (int st = 0; st < kStages - 1; ++st) {
        const size_t tile = blockIdx.x + (size_t)st * gridDim.x;
        if (tile < tiles) {
            double *dst = stages + st * G::STAGE;
            stage_tile<D, S, AL>(dst, X, tile * TS, batch);
            stage_tile<D, S, AL>(dst + G::TILE, T, tile * TS, batch);
        }
        cp_async_commit();
    }
    __syncthreads();

    // W' fragments for GEMM 1 (B operand, k-steps x n-tiles), resident all kernel.
    double bw[G::KT][G::NT];
#pragma unroll
    for (int kt = 0; kt < G::KT; ++kt)
#pragma unroll
        for (int nt = 0; nt < G::NT; ++nt) bw[kt][nt] = Wp[(kt * 4 + t4) * D + nt * 8 + g];

    double gacc[G::NT][4];
#pragma unroll
    for (int nt = 0; nt < G::NT; ++nt) gacc[nt][0] = gacc[nt][1] = gacc[nt][2] = gacc[nt][3] = 0.0;
    double sq = 0.0, check_y = 0.0, check_r = 0.0;

    int stage = 0;
    for (size_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        // Issue the tile kStages-1 ahead into the stage freed at the end of the previous iteration.
        {
            const size_t ahead = tile + (size_t)(kStages - 1) * gridDim.x;
            const int st = (stage + kStages - 1) % kStages;
            if (ahead < tiles) {
                double *dst = stages + st * G::STAGE;
                stage_tile<D, S, AL>(dst, X, ahead * TS, batch);
                stage_tile<D, S, AL>(dst + G::TILE, T, ahead * TS, batch);
            }
            cp_async_commit();
        }
        cp_async_wait<kStages - 1>();
        __syncthreads();

        double *xs = stages + stage * G::STAGE;
        double *ts = xs + G::TILE;
        // Gather in place: load this thread's blades of its samples, synchronise,
        // write the kept entries over the same rows.
        constexpr int PER = (TS + SLICES - 1) / SLICES;
        double vx[PER][S], vt[PER][S];
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int s = gslice + SLICES * i;
            if (s < TS) {
#pragma unroll
                for (int t = 0; t < S; ++t) {
                    const int col = gblade[t] ^ rsw<D>(s);
                    vx[i][t] = xs[s * N + col];
                    vt[i][t] = ts[s * N + col];
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int s = gslice + SLICES * i;
            if (s < TS) {
#pragma unroll
                for (int r = 0; r < S; ++r) {
                    double ax = 0.0, at = 0.0;
#pragma unroll
                    for (int t = 0; t < S; ++t) {
                        const bool neg = (gneg >> (r * 8 + t)) & 1ull;
                        ax = neg ? ax - vx[i][t] : ax + vx[i][t];
                        at = neg ? at - vt[i][t] : at + vt[i][t];
                    }
                    const int row = s * S + r;
                    const int col = gcol[r] ^ xsw<D>(row);
                    xs[row * D + col] = ax;
                    ts[row * D + col] = at;
                }
            }
        }
        __syncthreads();

        for (int blk = warp; blk < G::BLOCKS; blk += kWarps) {
            const double *xb = xs + blk * 16 * D;
            double *tb = ts + blk * 16 * D;
            // GEMM 1: Y'(16 x D) = X'(16 x D) W'(D x D). Block rows start at a multiple of 16,
            // so the swizzle of local row r equals that of the tile row.
            double acc[G::NT][4];
#pragma unroll
            for (int nt = 0; nt < G::NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0;
#pragma unroll
            for (int kt = 0; kt < G::KT; ++kt) {
                const int c = kt * 4 + t4;
                const double a0 = xb[g * D + (c ^ xsw<D>(g))];
                const double a1 = xb[(g + 8) * D + (c ^ xsw<D>(g + 8))];
#pragma unroll
                for (int nt = 0; nt < G::NT; ++nt) mma_16x8x4(acc[nt], a0, a1, bw[kt][nt]);
            }
            // Epilogue: R' = Y' - T' in place over T'; loss and finiteness probes.
#pragma unroll
            for (int nt = 0; nt < G::NT; ++nt) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row = g + 8 * h;
                    double2 *p = reinterpret_cast<double2 *>(&tb[row * D + ((nt * 8 + 2 * t4) ^ xsw<D>(row))]);
                    const double2 tv = *p;
                    double2 r;
                    r.x = acc[nt][2 * h] - tv.x;
                    r.y = acc[nt][2 * h + 1] - tv.y;
                    *p = r;
                    sq = fma(r.x, r.x, sq);
                    sq = fma(r.y, r.y, sq);
                    check_y = fma(acc[nt][2 * h], 0.0, check_y);
                    check_y = fma(acc[nt][2 * h + 1], 0.0, check_y);
                    check_r = fma(r.x, 0.0, check_r);
                    check_r = fma(r.y, 0.0, check_r);
                }
            }
            __syncwarp();
            // GEMM 2: G'(D x D) += X'^T(D x 16) R'(16 x D); k runs over the 16 rows of the block.
            // D = 8 uses the top half of the 16-row M tile (rows 8..15 of A are zero).
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int row = kk * 4 + t4;
                const int sw = xsw<D>(row);
                const double a0 = xb[row * D + (g ^ sw)];
                const double a1 = (D >= 16) ? xb[row * D + ((g + 8) ^ sw)] : 0.0;
#pragma unroll
                for (int nt = 0; nt < G::NT; ++nt) {
                    const double b0 = tb[row * D + ((nt * 8 + g) ^ sw)];
                    mma_16x8x4(gacc[nt], a0, a1, b0);
                }
            }
        }
        __syncthreads();  // the stage is reloaded by the next iteration's issue
        stage = (stage + 1) % kStages;
    }
    cp_async_wait<0>();
    __syncthreads();

    // Reduce the warps' G' partials in warp order (deterministic) in shared memory.
    double *Gs = stages;                            // kWarps * D * D
    double *Gsum = Gs + kWarps * D * D;             // D * D
    double *red = Gsum + D * D;                     // 3 * kThreads
    static_assert(kWarps * D * D + D * D + 3 * kThreads <= kStages * G::STAGE, "epilogue scratch fits");
#pragma unroll
    for (int nt = 0; nt < G::NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = g + 8 * h;
            if (row < D) {
                Gs[(warp * D + row) * D + nt * 8 + 2 * t4] = gacc[nt][2 * h];
                Gs[(warp * D + row) * D + nt * 8 + 2 * t4 + 1] = gacc[nt][2 * h + 1];
            }
        }
    red[threadIdx.x] = sq;
    red[kThreads + threadIdx.x] = check_y;
    red[2 * kThreads + threadIdx.x] = check_r;
    __syncthreads();
    for (int idx = threadIdx.x; idx < D * D; idx += kThreads) {
        double acc = 0.0;
        for (int w = 0; w < kWarps; ++w) acc += Gs[w * D * D + idx];
        Gsum[idx] = acc;
    }
    for (int width = kThreads / 2; width > 0; width >>= 1) {
        __syncthreads();
        if (threadIdx.x < width) {
            red[threadIdx.x] += red[threadIdx.x + width];
            red[kThreads + threadIdx.x] += red[kThreads + threadIdx.x + width];
            red[2 * kThreads + threadIdx.x] += red[2 * kThreads + threadIdx.x + width];
        }
    }
    __syncthreads();
    double *rec = records + (size_t)blockIdx.x * kRecStride;
    const double inv_s = 1.0 / (double)S;  // exact: S is a power of two
    if (threadIdx.x < N) {
        // g_A = <G', rho(e_A)> / S (right) or <G', rho(e_A)^T> / S (left)
        const int A = threadIdx.x;
        const int xa = rep.xm[A], za = rep.zm[A];
        double acc = 0.0;
        for (int j = 0; j < D; ++j) {
            // right: entry (j ^ xa, j) with sign (-1)^{za . j}; left: entry (j, j ^ xa), same sign
            const double v = rep.side ? Gsum[j * D + (j ^ xa)] : Gsum[(j ^ xa) * D + j];
            acc += (__popc(za & j) & 1) ? -v : v;
        }
        rec[A] = (rep.sg[A] < 0 ? -acc : acc) * inv_s;
    }
    if (threadIdx.x == 0) {
        rec[kRecLoss] = 0.5 * red[0] * inv_s;
        rec[kRecCheckY] = red[kThreads];
        rec[kRecCheckR] = red[2 * kThreads];
        rec[kRecCheckIn] = 0.0;
    }
}

template <int D, int S, bool AL>
cudaError_t launch_rep_impl(const RepDevice &rep, const double *X, const double *T, const double *W, size_t batch,
                            double *records, int *ctas_used, cudaStream_t stream) {
    using G = RepGeo<D, S>;
    if (rep.raw_stride != G::N || rep.D != D || rep.S != S) return cudaErrorInvalidValue;
    auto kernel = rep_cycle_kernel<D, S, AL>;
    const size_t smem = (size_t)(D * D + kStages * G::STAGE) * sizeof(double);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const size_t tiles = (batch + G::TS - 1) / G::TS;
    size_t grid = (size_t)device_sm_count() * (size_t)per_sm;
    if (grid > (size_t)kMaxCtas) grid = kMaxCtas;
    if (grid > tiles) grid = tiles;
    if (grid < 1) grid = 1;
    kernel<<<(unsigned)grid, kThreads, smem, stream>>>(rep, X, T, W, batch, records);
    if (ctas_used) *ctas_used = (int)grid;
    return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// Warp-specialised kernel (16-byte aligned x and t).
//
// Warps 0-3 (producers) move data: one thread issues bulk copies
// (cp.async.bulk, completion on an mbarrier per stage) of the raw x and t rows
// of a tile, kWsStages - 2 tiles ahead; all producers then gather the tile in
// place into X' and T' (ws_index layout). Warps 4-7 (consumers) run the math
// on the previous tile meanwhile:
//   GEMM 1 transposed, Y'^T = W'^T X'^T (W'^T fragments resident as the A
//     operand), so each lane's accumulators hold Y'[n0 + 2t + h][g (+8)];
//   the accumulators start at -T' (the producers write T' negated), so GEMM 1
//     leaves R' = Y' - T' in registers: exactly the B fragment of GEMM 2 when
//     the k slots of an mma are the rows n0 + 2t + h;
//   GEMM 2, G' += X'^T R', with X'^T loaded as the A operand.
// Named barriers hand stages over (FULL: gathered, EMPTY: consumed); every
// wait on an mbarrier is bounded and a wait that gives up marks the record as
// failed (non-finite check value) while the barrier protocol carries on.
constexpr int kWsAhead = kWsStages - 2;
constexpr int kBarFull = 1;                          // + stage
constexpr int kBarEmpty = kBarFull + kWsStages;      // + stage
constexpr int kBarProducers = kBarEmpty + kWsStages;  // producers only
static_assert(kBarProducers < 16, "named barrier ids");
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Bounded wait for the completion of phase `parity`; false when it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity) {
    const unsigned a = smem_u32(bar);
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
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
__device__ __forceinline__ void bulk_load(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// D(16x8) += A(16x16) * B(16x8), float64: a[i] = A[g + 8 (i % 2)][t + 4 (i / 2)],
// b[j] = B[t + 4 j][g]; C as in mma_16x8x4.
__device__ __forceinline__ void mma_16x8x16(double (&c)[4], const double (&a)[8], const double (&b)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7,%8,%9,%10,%11}, "
        "{%12,%13,%14,%15}, {%0,%1,%2,%3};\n"
        : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
        : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]), "d"(b[0]),
          "d"(b[1]), "d"(b[2]), "d"(b[3]));
}

// D(8x8) += A(8x4) * B(4x8): a0 = A[g][t], b0 = B[t][g], c0,c1 = C[g][2t, 2t+1].
__device__ __forceinline__ void mma_8x8x4(double (&c)[2], double a0, double b0) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
                 : "+d"(c[0]), "+d"(c[1])
                 : "d"(a0), "d"(b0));
}

// Exponent field of v (0x7ff00000 exactly when v is not finite).
__device__ __forceinline__ unsigned exponent_bits(double v) { return (unsigned)__double2hiint(v) & 0x7ff00000u; }

// v with its sign bit XORed by `mask` (0 or 0x80000000): an integer operation.
__device__ __forceinline__ double flip_sign(double v, unsigned mask) {
    return __hiloint2double(__double2hiint(v) ^ (int)mask, __double2loint(v));
}

// In-place Walsh-Hadamard transform: w[f] <- sum_t (-1)^{popc(t & f)} w[t].
template <int S>
__device__ __forceinline__ void walsh(double (&w)[S]) {
#pragma unroll
    for (int h = 1; h < S; h <<= 1)
#pragma unroll
        for (int a = 0; a < S; ++a)
            if (!(a & h)) {
                const double u = w[a], v = w[a | h];
                w[a] = u + v;
                w[a | h] = u - v;
            }
}

// A producer thread's blade group in the warp-specialised kernels (thread tid
// handles group m = tid % D of the samples slot + SLOTS i, slot = tid / D):
// raw offsets of the S member blades within a stage (roff), offsets of the S
// kept entries in the ws_index layout (woff), and the sign masks of the gather
// X'_f = out_f sum_t H[f][t] in_t x_t (and of its inverse).
template <int D, int S>
struct GroupMap {
    int roff[S], woff[S];
    unsigned in_sign[S], out_sign[S];
    __device__ __forceinline__ GroupMap(const RepDevice &rep, int tid) {
        using G = WsGeo<D, S>;
        const int m = tid % D, slot = tid / D;
        const int L = D == 8 ? (slot & 1) * 8 + m : m;
#pragma unroll
        for (int t = 0; t < S; ++t) {
            roff[t] = slot * G::N + rep.ws_blade[L][t];
            in_sign[t] = ((rep.ws_in_neg[L] >> t) & 1u) << 31;
            const int r = rep.ws_out_row[L][t];
            woff[t] = ws_index<D>(slot * S + r, rep.grp_col[m][r]);
            out_sign[t] = ((rep.ws_out_neg[L] >> t) & 1u) << 31;
        }
    }
};

// W' = rho(W) (right) or rho(W)^T (left) of a dense parameter, built by the
// whole CTA into shared memory (entry (k, j) sums the S blades A with
// xm[A] = k ^ j, signed by the blade's sign and its Z mask on the column).
template <int D, int N>
__device__ __forceinline__ void build_wprime(const RepDevice &rep, const double *__restrict__ W, double *Wp) {
    for (int idx = threadIdx.x; idx < D * D; idx += kWsThreads) {
        const int k = idx / D, j = idx - k * D;
        const int col = rep.side ? k : j;
        double acc = 0.0;
        for (int A = 0; A < N; ++A) {
            if (rep.xm[A] != (k ^ j)) continue;
            const double w = W[A];
            const bool neg = (rep.sg[A] < 0) != ((__popc(rep.zm[A] & col) & 1) != 0);
            acc += neg ? -w : w;
        }
        Wp[idx] = acc;
    }
}

// Consumer-side G' accumulators of the warp-specialised kernels: D / 8
// 8-column tiles of G', two k halves, the mma C fragment.
template <int D>
using GAcc = double[D / 8][2][D == 16 ? 4 : 2];

// End of a warp-specialised training or VJP pass, called by every thread after
// a __syncthreads (all stage memory free): reduces the consumer warps' G'
// partials in warp order and the threads' sums of |R'|^2 (a fixed tree), and
// writes the CTA's record: g_A = <G', rho(e_A)> / S, loss 0.5 sum |R'|^2 / S,
// and the check value (NaN when some R' was not finite or a wait gave up).
// rep_ws_kernel carries the same reduction, W' build and group tables inline:
// moving them onto these helpers changes that kernel's register allocation,
// and its timing is the measured one.
// Consumer partials of the complex (3M) GEMM 2 written as the complex-linear
// part of G' in the original columns (see rep_ws_kernel's CPLX notes).
__device__ __forceinline__ void ws_store_complex_partials(const double (&c3)[3][2][2], double *gw) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int m = g, mp = 2 * t4 + i;
        const double m1 = c3[0][0][i] + c3[0][1][i], m2 = c3[1][0][i] + c3[1][1][i];
        const double m3 = c3[2][0][i] + c3[2][1][i];
        const double P = 0.5 * (m1 - m3), Q = 0.5 * (m1 - m2);
        const unsigned sm = (m & 4) ? 0x80000000u : 0u, sp = (mp & 4) ? 0x80000000u : 0u;
        gw[m * 16 + mp] = P;
        gw[m * 16 + (mp ^ 12)] = flip_sign(Q, sp ^ 0x80000000u);
        gw[(m ^ 12) * 16 + mp] = flip_sign(Q, sm);
        gw[(m ^ 12) * 16 + (mp ^ 12)] = flip_sign(P, sm ^ sp);
    }
}

template <int D, int S, bool CPLX = false>
__device__ __forceinline__ void ws_write_record(const RepDevice &rep, const GAcc<D> &gacc, const double (&c3)[3][2][2],
                                                double sq, unsigned worst_exp, const unsigned *gave_up,
                                                double *scratch, double *records) {
    constexpr int N = D * S, PT = D / 8;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    double *Gs = scratch;                // 4 * D * D
    double *Gsum = Gs + 4 * D * D;       // D * D
    double *red = Gsum + D * D;          // kWsThreads
    if (CPLX && warp >= kWsProducers / 32) {
        ws_store_complex_partials(c3, Gs + (warp - kWsProducers / 32) * D * D);
    } else if (warp >= kWsProducers / 32) {
        const int cw = warp - kWsProducers / 32;
        const int g = lane >> 2, t4 = lane & 3;
        double *gw = Gs + cw * D * D;
#pragma unroll
        for (int p = 0; p < PT; ++p)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                gw[g * D + p * 8 + 2 * t4 + i] = gacc[p][0][i] + gacc[p][1][i];
                if constexpr (D == 16) gw[(g + 8) * D + p * 8 + 2 * t4 + i] = gacc[p][0][2 + i] + gacc[p][1][2 + i];
            }
    }
    red[tid] = sq;
    const int bad = __syncthreads_or(worst_exp == 0x7ff00000u);
    for (int idx = tid; idx < D * D; idx += kWsThreads)
        Gsum[idx] = ((Gs[idx] + Gs[D * D + idx]) + Gs[2 * D * D + idx]) + Gs[3 * D * D + idx];
    for (int width = kWsThreads / 2; width > 0; width >>= 1) {
        __syncthreads();
        if (tid < width) red[tid] += red[tid + width];
    }
    __syncthreads();
    double *rec = records + (size_t)blockIdx.x * kRecStride;
    const double inv_s = 1.0 / (double)S;  // exact: S is a power of two
    if (tid < N) {
        const int A = tid;
        const int xa = rep.xm[A], za = rep.zm[A];
        double acc = 0.0;
        for (int j = 0; j < D; ++j) {
            const double v = rep.side ? Gsum[j * D + (j ^ xa)] : Gsum[(j ^ xa) * D + j];
            acc += (__popc(za & j) & 1) ? -v : v;
        }
        rec[A] = (rep.sg[A] < 0 ? -acc : acc) * inv_s;
    }
    if (tid == 0) {
        rec[kRecLoss] = 0.5 * red[0] * inv_s;
        rec[kRecCheckY] = 0.0;
        // Y' = R' + T' with T' finite, so a non-finite output shows in R'.
        rec[kRecCheckR] =
            (bad || *(volatile const unsigned *)gave_up) ? __longlong_as_double(0x7ff8000000000000ll) : 0.0;
        rec[kRecCheckIn] = 0.0;
    }
}

// VJP = false: training pass (x, targets t, parameter W). VJP = true: parameter
// VJP of given output cotangents c (in place of t, no W): the producers write
// C' = P c instead of -T', and GEMM 1 is skipped (R' := C').
//
// CPLX (D = 16, S = 4, RepDevice::cplx): the consumers use the complex
// structure J = P(12, 4). Column pair (m, m ^ 12), m < 8, of a row r of X' is
// the complex number u - i v with u = r[m], v = s_m r[m ^ 12] (s_m = -1 for
// m >= 4), and W' is the 8 x 8 complex matrix alpha + i beta with
// alpha[m][m'] = W'[m][m'], beta[m][m'] = s_m W'[m ^ 12][m']. GEMM 1 is then
// three real 8 x 8 products per row (Gauss's three-multiplication form):
//   K1 = (u - v) alpha,  K2 = u (beta - alpha),  K3 = v (alpha + beta),
//   R'[m'] = K1 + K3 - T'[m'],  R'[m' ^ 12] s_m' = -(K1 + K2) - s_m' T'[m' ^ 12],
// and GEMM 2 keeps only the complex-linear part of G' = X'^T R', which is all
// that <G', rho(e_A)> sees (rho(e_A) commutes with J): with p, q the pair of
// R' entries, P = sum u p + v q and Q = sum v p - u q are
//   M1 = (u + v) p,  M2 = u (p + q),  M3 = v (p - q),  P = M1 - M3,  Q = M1 - M2.
// 1536 instead of 2048 FP64 multiply-adds per sample (m8n8k4 tiles), for 192
// extra additions; the shared-memory access sets are the plain consumer's.
template <int D, int S, bool VJP, bool CPLX = false>
__global__ void __launch_bounds__(kWsThreads, 2)
rep_ws_kernel(const RepDevice rep, const double *__restrict__ X, const double *__restrict__ T,
              const double *__restrict__ W, size_t batch, double *__restrict__ records) {
    using G = WsGeo<D, S>;
    constexpr int N = G::N, TS = G::TS;
    extern __shared__ __align__(16) double smem[];
    double *Wp = smem;                    // D * D
    double *stages = Wp + D * D;          // kWsStages x (x tile, t tile)
    uint64_t *bars = reinterpret_cast<uint64_t *>(stages + kWsStages * G::STAGE);
    __shared__ unsigned s_gave_up;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t tiles = (batch + TS - 1) / TS;
    const int K = (size_t)blockIdx.x < tiles ? (int)((tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;

    if (tid == 0) {
        for (int s = 0; s < kWsStages; ++s) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        s_gave_up = 0u;
    }
    // W' = rho(W) (right) or rho(W)^T (left), as in rep_cycle_kernel.
    for (int idx = tid; !VJP && idx < D * D; idx += kWsThreads) {
        const int k = idx / D, j = idx - k * D;
        const int col = rep.side ? k : j;
        double acc = 0.0;
        for (int A = 0; A < N; ++A) {
            if (rep.xm[A] != (k ^ j)) continue;
            const double w = W[A];
            const bool neg = (rep.sg[A] < 0) != ((__popc(rep.zm[A] & col) & 1) != 0);
            acc += neg ? -w : w;
        }
        Wp[idx] = acc;
    }
    __syncthreads();

    // Consumer state (also declared, unused, in the producer warps).
    constexpr int PT = D / 8;  // 8-column tiles of G'
    double gacc[PT][2][D == 16 ? 4 : 2];
    double c3[3][2][2];  // CPLX: M1, M2, M3 per k slice parity h, the m8n8k4 C fragment
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int h = 0; h < 2; ++h) c3[a][h][0] = c3[a][h][1] = 0.0;
#pragma unroll
    for (int p = 0; p < PT; ++p)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < (D == 16 ? 4 : 2); ++i) gacc[p][h][i] = 0.0;
    double sq = 0.0;
    unsigned worst_exp = 0u;

    if (warp < kWsProducers / 32) {
        // ------------------------------------------------------------ producers
        const int m = tid % D, slot = tid / D;
        const int L = D == 8 ? (slot & 1) * 8 + m : m;
        // Offsets within a stage for this thread's first sample (slot); sample
        // slot + SLOTS * i adds SLOTS * i * N to both.
        int roff[S], woff[S];
        unsigned in_sign[S], out_sign[S];
#pragma unroll
        for (int t = 0; t < S; ++t) {
            roff[t] = slot * N + rep.ws_blade[L][t];
            in_sign[t] = ((rep.ws_in_neg[L] >> t) & 1u) << 31;
            const int r = rep.ws_out_row[L][t];
            woff[t] = ws_index<D>(slot * S + r, rep.grp_col[m][r]);
            out_sign[t] = ((rep.ws_out_neg[L] >> t) & 1u) << 31;
        }
        auto issue = [&](int k) {
            const size_t first = (blockIdx.x + (size_t)k * gridDim.x) * TS;
            const size_t count = batch - first < (size_t)TS ? batch - first : (size_t)TS;
            const unsigned bytes = (unsigned)(count * N * sizeof(double));
            double *dst = stages + (k % kWsStages) * G::STAGE;
            uint64_t *bar = &bars[k % kWsStages];
            mbar_expect_tx(bar, 2u * bytes);
            bulk_load(dst, X + first * N, bytes, bar);
            bulk_load(dst + G::TILE, T + first * N, bytes, bar);
        };
        if (tid == 0)
            for (int k = 0; k < K && k < kWsAhead; ++k) issue(k);
        for (int k = 0; k < K; ++k) {
            const int st = k % kWsStages;
            const int ahead = k + kWsAhead;
            if (ahead < K) {
                // The stage of `ahead` last held tile ahead - kWsStages: wait until it is consumed.
                if (ahead >= kWsStages) named_sync(kBarEmpty + ahead % kWsStages, kWsThreads);
                if (tid == 0) {
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    issue(ahead);
                }
            }
            if (!mbar_wait(&bars[st], (unsigned)((k / kWsStages) & 1))) atomicOr(&s_gave_up, 1u);
            const size_t first = (blockIdx.x + (size_t)k * gridDim.x) * TS;
            const int valid = batch - first < (size_t)TS ? (int)(batch - first) : TS;
            double *xs = stages + st * G::STAGE;
            double *ts = xs + G::TILE;
            double vx[G::PER][S], vt[G::PER][S];
#pragma unroll
            for (int i = 0; i < G::PER; ++i) {
                const bool ok = slot + G::SLOTS * i < valid;
#pragma unroll
                for (int t = 0; t < S; ++t) {
                    vx[i][t] = ok ? xs[G::SLOTS * i * N + roff[t]] : 0.0;
                    vt[i][t] = ok ? ts[G::SLOTS * i * N + roff[t]] : 0.0;
                }
            }
            named_sync(kBarProducers, kWsProducers);  // every raw read is done before the in-place writes
#pragma unroll
            for (int i = 0; i < G::PER; ++i) {
#pragma unroll
                for (int t = 0; t < S; ++t) {
                    vx[i][t] = flip_sign(vx[i][t], in_sign[t]);
                    vt[i][t] = flip_sign(vt[i][t], in_sign[t]);
                }
                walsh<S>(vx[i]);
                walsh<S>(vt[i]);
#pragma unroll
                for (int f = 0; f < S; ++f) {
                    xs[G::SLOTS * i * N + woff[f]] = flip_sign(vx[i][f], out_sign[f]);
                    ts[G::SLOTS * i * N + woff[f]] = flip_sign(vt[i][f], out_sign[f] ^ (VJP ? 0u : 0x80000000u));  // -T' or C'
                }
            }
            named_arrive(kBarFull + st, kWsThreads);
        }
    } else if constexpr (CPLX) {
        // ------------------------------------------------------ consumers (3M)
        // Software-pipelined: iteration k loads every operand of tile k from its
        // stage (GEMM 1 operands, T', GEMM 2's X' operands), issues GEMM 2 of tile
        // k - 1 from registers and GEMM 1 of tile k (independent streams), and
        // releases the stage. The accumulation order of GEMM 2 is tile by tile as
        // without the pipelining.
        static_assert(D == 16 && S == 4, "complex form of the n = 6 quaternionic algebras");
        constexpr int GP = G::GPW;
        const int cw = warp - kWsProducers / 32;
        const int g = lane >> 2, t4 = lane & 3;
        constexpr unsigned NEG = 0x80000000u;
        const unsigned sg_neg = (g & 4) ? NEG : 0u;  // s_g of complex column g
        // GEMM 1 A fragments (m8n8k4, A[m'][m], m' = g, m = t4 + 4 kk; s_m = -1 for kk = 1).
        double wk1[2], wk2[2], wk3[2];
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int m = t4 + 4 * kk;
            const double al = VJP ? 0.0 : Wp[m * 16 + g];
            const double be = VJP ? 0.0 : flip_sign(Wp[(m ^ 12) * 16 + g], kk ? NEG : 0u);
            wk1[kk] = al;
            wk2[kk] = be - al;
            wk3[kk] = al + be;
        }
        // GEMM 2 operands of the previous tile: R' pair (p, q) and X' pair (u, v) at
        // row n0 + 2 t4 + h, complex column g.
        double pp[GP][2], pq[GP][2], pu[GP][2], pv[GP][2];
        auto gemm2 = [&]() {
#pragma unroll
            for (int j = 0; j < GP; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    mma_8x8x4(c3[0][h], pu[j][h] + pv[j][h], pp[j][h]);
                    mma_8x8x4(c3[1][h], pu[j][h], pp[j][h] + pq[j][h]);
                    mma_8x8x4(c3[2][h], pv[j][h], pp[j][h] - pq[j][h]);
                }
        };
        for (int k = 0; k < K; ++k) {
            const int st = k % kWsStages;
            named_sync(kBarFull + st, kWsThreads);
            const double *xs = stages + st * G::STAGE;
            const double *ts = xs + G::TILE;
            double cu[GP][2], cv[GP][2], k1[GP][2], k2[GP][2], k3[GP][2], bu[GP][2], bv[GP][2];
#pragma unroll
            for (int j = 0; j < GP; ++j) {
                const int n0 = (cw * GP + j) * 8;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row = n0 + 2 * t4 + h;
                    cu[j][h] = xs[ws_index<16>(row, g)];
                    cv[j][h] = flip_sign(xs[ws_index<16>(row, g ^ 12)], sg_neg);
                    // K3 starts at -T'[.][g] (stored negated), K2 at +s_g T'[.][g ^ 12]; in
                    // VJP mode these are C' itself: p = C'[.][g], q = s_g C'[.][g ^ 12].
                    k3[j][h] = ts[ws_index<16>(row, g)];
                    k2[j][h] = flip_sign(ts[ws_index<16>(row, g ^ 12)], VJP ? sg_neg : (sg_neg ^ NEG));
                    k1[j][h] = 0.0;
                }
#pragma unroll
                for (int kk = 0; kk < 2 && !VJP; ++kk) {
                    const int m = t4 + 4 * kk;
                    bu[j][kk] = xs[ws_index<16>(n0 + g, m)];
                    bv[j][kk] = flip_sign(xs[ws_index<16>(n0 + g, m ^ 12)], kk ? NEG : 0u);
                }
            }
            if (k > 0) gemm2();
            // GEMM 1 transposed of tile k: K[m' = g][row n0 + 2 t4 + h].
#pragma unroll
            for (int j = 0; j < GP && !VJP; ++j)
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    mma_8x8x4(k1[j], wk1[kk], bu[j][kk] - bv[j][kk]);
                    mma_8x8x4(k2[j], wk2[kk], bu[j][kk]);
                    mma_8x8x4(k3[j], wk3[kk], bv[j][kk]);
                }
#pragma unroll
            for (int j = 0; j < GP; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const double r0 = VJP ? k3[j][h] : k1[j][h] + k3[j][h];
                    const double r1 = VJP ? k2[j][h] : -(k1[j][h] + k2[j][h]);
                    sq = fma(r0, r0, sq);
                    sq = fma(r1, r1, sq);
                    worst_exp = max(worst_exp, max(exponent_bits(r0), exponent_bits(r1)));
                    pp[j][h] = r0;
                    pq[j][h] = r1;
                    pu[j][h] = cu[j][h];
                    pv[j][h] = cv[j][h];
                }
            // Every value read from the stage has been used: release it.
            if (k + kWsStages < K) named_arrive(kBarEmpty + st, kWsThreads);
        }
        if (K > 0) gemm2();
    } else {
        // ------------------------------------------------------------ consumers
        const int cw = warp - kWsProducers / 32;
        const int g = lane >> 2, t4 = lane & 3;
        constexpr int KT = D / 4;
        // W'^T as the A operand: D = 16 one m16n8k16 fragment, wa[i] = W'[t + 4 (i / 2)][g + 8 (i % 2)];
        // D = 8 the m8n8k4 fragments wa[kk] = W'[4 kk + t][g].
        double wa[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (VJP) wa[i] = 0.0;
            else if (D == 16) wa[i] = Wp[(t4 + 4 * (i / 2)) * D + g + 8 * (i % 2)];
            else wa[i] = i < KT ? Wp[(4 * i + t4) * D + g] : 0.0;
        }
        for (int k = 0; k < K; ++k) {
            const int st = k % kWsStages;
            named_sync(kBarFull + st, kWsThreads);
            const double *xs = stages + st * G::STAGE;
            const double *ts = xs + G::TILE;
#pragma unroll
            for (int j = 0; j < G::GPW; j += 2) {
                int n0[2];
                n0[0] = (cw * G::GPW + j) * 8;
                n0[1] = n0[0] + 8;
                if constexpr (D == 16) {
                    // GEMM 1 per row group: one m16n8k16 (M = output column j, N = 8 rows, K = 16).
                    double c[2][4];
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        double b[4];
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) b[kk] = xs[ws_index<D>(n0[q] + g, 4 * kk + t4)];
                        // accumulate onto -T': the result is R' = Y' - T'
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            c[q][h] = ts[ws_index<D>(n0[q] + 2 * t4 + h, g)];
                            c[q][2 + h] = ts[ws_index<D>(n0[q] + 2 * t4 + h, g + 8)];
                        }
                        if constexpr (!VJP) mma_16x8x16(c[q], wa, b);
                    }
                    // Epilogue in registers; GEMM 2 over both row groups as one m16n8k16 per
                    // 8-column tile of G', k slot t + 4 j <-> row n0[j / 2] + 2 t + j % 2.
                    double ax[8], rlo[4], rhi[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int q = j >> 1, h = j & 1;
                        const int row = n0[q] + 2 * t4 + h;
                        const int plo = ws_index<D>(row, g), phi = ws_index<D>(row, g + 8);
                        rlo[j] = c[q][h];
                        rhi[j] = c[q][2 + h];
                        sq = fma(rlo[j], rlo[j], sq);
                        sq = fma(rhi[j], rhi[j], sq);
                        worst_exp = max(worst_exp, max(exponent_bits(rlo[j]), exponent_bits(rhi[j])));
                        ax[2 * j] = xs[plo];
                        ax[2 * j + 1] = xs[phi];
                    }
                    mma_16x8x16(gacc[0][0], ax, rlo);
                    mma_16x8x16(gacc[PT - 1][0], ax, rhi);
                } else {
                    double c[2][2];  // start at -T' (R' = Y' - T' after GEMM 1)
#pragma unroll
                    for (int q = 0; q < 2; ++q)
#pragma unroll
                        for (int h = 0; h < 2; ++h) c[q][h] = ts[ws_index<D>(n0[q] + 2 * t4 + h, g)];
#pragma unroll
                    for (int kk = 0; !VJP && kk < KT; ++kk)
#pragma unroll
                        for (int q = 0; q < 2; ++q) mma_8x8x4(c[q], wa[kk], xs[ws_index<D>(n0[q] + g, 4 * kk + t4)]);
#pragma unroll
                    for (int q = 0; q < 2; ++q)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int row = n0[q] + 2 * t4 + h;
                            const int pos = ws_index<D>(row, g);
                            const double r = c[q][h];
                            sq = fma(r, r, sq);
                            worst_exp = max(worst_exp, exponent_bits(r));
                            mma_8x8x4(gacc[0][h], xs[pos], r);
                        }
                }
            }
            if (k + kWsStages < K) named_arrive(kBarEmpty + st, kWsThreads);
        }
    }
    __syncthreads();

    // Reduce the consumer warps' G' partials in warp order (deterministic).
    double *Gs = stages;                 // 4 * D * D
    double *Gsum = Gs + 4 * D * D;       // D * D
    double *red = Gsum + D * D;          // kWsThreads
    static_assert(5 * D * D + kWsThreads <= kWsStages * G::STAGE, "epilogue scratch fits");
    if (CPLX && warp >= kWsProducers / 32) {
        // The complex-linear part of G' in the original columns: entry (m, m')
        // carries P / 2, (m, m' ^ 12) -s_m' Q / 2, (m ^ 12, m') s_m Q / 2 and
        // (m ^ 12, m' ^ 12) s_m s_m' P / 2 (halving is exact).
        ws_store_complex_partials(c3, Gs + (warp - kWsProducers / 32) * D * D);
    } else if (warp >= kWsProducers / 32) {
        const int cw = warp - kWsProducers / 32;
        const int g = lane >> 2, t4 = lane & 3;
        double *gw = Gs + cw * D * D;
#pragma unroll
        for (int p = 0; p < PT; ++p)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                gw[g * D + p * 8 + 2 * t4 + i] = gacc[p][0][i] + gacc[p][1][i];
                if constexpr (D == 16) gw[(g + 8) * D + p * 8 + 2 * t4 + i] = gacc[p][0][2 + i] + gacc[p][1][2 + i];
            }
    }
    red[tid] = sq;
    const int bad = __syncthreads_or(worst_exp == 0x7ff00000u);
    for (int idx = tid; idx < D * D; idx += kWsThreads)
        Gsum[idx] = ((Gs[idx] + Gs[D * D + idx]) + Gs[2 * D * D + idx]) + Gs[3 * D * D + idx];
    for (int width = kWsThreads / 2; width > 0; width >>= 1) {
        __syncthreads();
        if (tid < width) red[tid] += red[tid + width];
    }
    __syncthreads();
    double *rec = records + (size_t)blockIdx.x * kRecStride;
    const double inv_s = 1.0 / (double)S;  // exact: S is a power of two
    if (tid < N) {
        const int A = tid;
        const int xa = rep.xm[A], za = rep.zm[A];
        double acc = 0.0;
        for (int j = 0; j < D; ++j) {
            const double v = rep.side ? Gsum[j * D + (j ^ xa)] : Gsum[(j ^ xa) * D + j];
            acc += (__popc(za & j) & 1) ? -v : v;
        }
        rec[A] = (rep.sg[A] < 0 ? -acc : acc) * inv_s;
    }
    if (tid == 0) {
        rec[kRecLoss] = 0.5 * red[0] * inv_s;
        rec[kRecCheckY] = 0.0;
        // Y' = R' + T' with T' finite, so a non-finite output shows in R'.
        rec[kRecCheckR] = (bad || s_gave_up) ? __longlong_as_double(0x7ff8000000000000ll) : 0.0;
        rec[kRecCheckIn] = 0.0;
    }
}

template <int D, int S, bool VJP>
cudaError_t launch_rep_ws(const RepDevice &rep, const double *X, const double *T, const double *W, size_t batch,
                          double *records, int *ctas_used, cudaStream_t stream) {
    using G = WsGeo<D, S>;
    if (rep.raw_stride != G::N || rep.D != D || rep.S != S) return cudaErrorInvalidValue;
    auto kernel = rep_ws_kernel<D, S, VJP>;
    if constexpr (D == 16 && S == 4)
        if (rep.cplx) kernel = rep_ws_kernel<16, 4, VJP, true>;
    const size_t smem = (size_t)(D * D + kWsStages * G::STAGE) * sizeof(double) + kWsStages * sizeof(uint64_t);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kWsThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const size_t tiles = (batch + G::TS - 1) / G::TS;
    size_t grid = (size_t)device_sm_count() * (size_t)per_sm;
    if (grid > (size_t)kMaxCtas) grid = kMaxCtas;
    if (grid > tiles) grid = tiles;
    if (grid < 1) grid = 1;
    kernel<<<(unsigned)grid, kWsThreads, smem, stream>>>(rep, X, T, W, batch, records);
    if (ctas_used) *ctas_used = (int)grid;
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Forward through the representation (16-byte aligned x and y).
//
// Per sample: X' = P x, Y' = X' W', y = P^-1 Y'. P is block diagonal over the
// blade groups, and a group's S x S block is O H I (O, I diagonal signs, H the
// Walsh-Hadamard matrix, H H = S 1), so its inverse is I H O / S: the scatter
// runs the gather's butterfly backwards (read the kept entries, flip by the
// output signs, Walsh transform, flip by the input signs, scale by 1/S, which
// is exact).
//
// Warps 0-3 (producers): thread 0 keeps FwdPipe::AHEAD bulk loads of raw x
// tiles in flight (completion on one mbarrier per stage). For tile k all
// producers gather X' in place and arrive on full[stage]; then, once the
// consumers have arrived on done[] for tile k - FwdPipe::LAG, they scatter its
// Y' back to raw rows in place, and thread 0 stores the tile's rows with one
// bulk copy. A stage is reloaded only after its
// store has finished reading it (bulk wait_group.read).
// Warps 4-7 (consumers): GEMM 1 transposed with W'^T fragments resident, as in
// rep_ws_kernel, from zero accumulators; Y' is written over the X' rows the
// warp has just read.
// Every wait is bounded; a wait that gives up makes the CTA write NaN in place
// of its remaining outputs, and the kernel still ends.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_store(void *dst, const void *src, unsigned bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst), "r"(smem_u32(src)),
                 "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

template <int D, int S>
__global__ void __launch_bounds__(kWsThreads, FwdPipe::CTAS_PER_SM)
rep_fwd_kernel(const RepDevice rep, const double *__restrict__ X, const double *__restrict__ W,
               const TermParameter terms, size_t batch, double *Y) {
    using G = WsGeo<D, S>;
    using P = FwdPipe;
    constexpr int N = G::N, TS = G::TS, TILE = G::TILE;
    constexpr int NST = P::STAGES, STAGE = TILE;
    constexpr int kConsumers = kWsThreads - kWsProducers;
    constexpr int kBarScatter = 1;  // named barrier of the producer warps
    extern __shared__ __align__(16) double smem[];
    double *Wp = smem;                      // D * D
    double *stages = Wp + D * D;            // NST x tiles
    uint64_t *loaded = reinterpret_cast<uint64_t *>(stages + NST * STAGE);
    uint64_t *full = loaded + NST;          // producers -> consumers: X' ready
    uint64_t *done = full + NST;            // consumers -> producers: Y' ready
    __shared__ unsigned s_gave_up;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t tiles = (batch + TS - 1) / TS;
    const int K = (size_t)blockIdx.x < tiles ? (int)((tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&loaded[s], 1);
            mbar_init(&full[s], kWsProducers);
            mbar_init(&done[s], kConsumers);
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        s_gave_up = 0u;
    }
    // W' = rho(W) (right) or rho(W)^T (left), as in rep_cycle_kernel; W is a dense
    // device array, or (W == null) the term list sum_t value_t e_{blade_t}.
    for (int idx = tid; idx < D * D; idx += kWsThreads) {
        const int k = idx / D, j = idx - k * D;
        const int col = rep.side ? k : j;
        double acc = 0.0;
        if (W != nullptr) {
            for (int A = 0; A < N; ++A) {
                if (rep.xm[A] != (k ^ j)) continue;
                const double w = W[A];
                const bool neg = (rep.sg[A] < 0) != ((__popc(rep.zm[A] & col) & 1) != 0);
                acc += neg ? -w : w;
            }
        } else {
            for (int t = 0; t < terms.terms; ++t) {
                const int A = terms.blade[t];
                if (rep.xm[A] != (k ^ j)) continue;
                const double w = terms.values != nullptr ? terms.scale[t] * terms.values[t] : terms.coeff[t];
                const bool neg = (rep.sg[A] < 0) != ((__popc(rep.zm[A] & col) & 1) != 0);
                acc += neg ? -w : w;
            }
        }
        Wp[idx] = acc;
    }
    __syncthreads();

    if (warp < kWsProducers / 32) {
        // ------------------------------------------------------------ producers
        const int m = tid % D, slot = tid / D;
        const int L = D == 8 ? (slot & 1) * 8 + m : m;
        int roff[S], woff[S];
        unsigned in_sign[S], out_sign[S];
#pragma unroll
        for (int t = 0; t < S; ++t) {
            roff[t] = slot * N + rep.ws_blade[L][t];
            in_sign[t] = ((rep.ws_in_neg[L] >> t) & 1u) << 31;
            const int r = rep.ws_out_row[L][t];
            woff[t] = ws_index<D>(slot * S + r, rep.grp_col[m][r]);
            out_sign[t] = ((rep.ws_out_neg[L] >> t) & 1u) << 31;
        }
        const double inv_s = 1.0 / (double)S;  // exact: S is a power of two
        auto tile_rows = [&](int k, size_t *first) {
            *first = (blockIdx.x + (size_t)k * gridDim.x) * TS;
            return batch - *first < (size_t)TS ? (int)(batch - *first) : TS;
        };
        auto issue = [&](int k) {
            size_t first;
            const unsigned bytes = (unsigned)tile_rows(k, &first) * N * (unsigned)sizeof(double);
            uint64_t *bar = &loaded[k % NST];
            mbar_expect_tx(bar, bytes);
            bulk_load(stages + (k % NST) * STAGE, X + first * N, bytes, bar);
        };
        if (tid == 0)
            for (int k = 0; k < K && k < P::AHEAD; ++k) issue(k);
        for (int k = 0; k < K + P::LAG; ++k) {
            if (k < K) {
                const int ahead = k + P::AHEAD;
                if (tid == 0 && ahead < K) {
                    // The stage of `ahead` last held tile ahead - NST, whose store was
                    // issued STORE_PENDING stores ago at the latest.
                    if (ahead >= NST) bulk_wait_read<P::STORE_PENDING>();
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    issue(ahead);
                }
                const int st = k % NST;
                if (!mbar_wait(&loaded[st], (unsigned)((k / NST) & 1))) atomicOr(&s_gave_up, 1u);
                size_t first;
                const int valid = tile_rows(k, &first);
                double *xs = stages + st * STAGE;
                double v[G::PER][S];
#pragma unroll
                for (int i = 0; i < G::PER; ++i) {
                    const bool ok = slot + G::SLOTS * i < valid;
#pragma unroll
                    for (int t = 0; t < S; ++t) v[i][t] = ok ? xs[G::SLOTS * i * N + roff[t]] : 0.0;
                }
                named_sync(kBarScatter, kWsProducers);  // every raw read is done before the in-place writes
#pragma unroll
                for (int i = 0; i < G::PER; ++i) {
#pragma unroll
                    for (int t = 0; t < S; ++t) v[i][t] = flip_sign(v[i][t], in_sign[t]);
                    walsh<S>(v[i]);
#pragma unroll
                    for (int f = 0; f < S; ++f) xs[G::SLOTS * i * N + woff[f]] = flip_sign(v[i][f], out_sign[f]);
                }
                mbar_arrive(&full[st]);
            }
            const int j = k - P::LAG;
            if (j >= 0) {
                const int st = j % NST;
                if (!mbar_wait(&done[st], (unsigned)((j / NST) & 1))) atomicOr(&s_gave_up, 1u);
                double *xs = stages + st * STAGE;
                double v[G::PER][S];
#pragma unroll
                for (int i = 0; i < G::PER; ++i)
#pragma unroll
                    for (int f = 0; f < S; ++f) v[i][f] = flip_sign(xs[G::SLOTS * i * N + woff[f]], out_sign[f]);
                named_sync(kBarScatter, kWsProducers);  // every Y' read is done before the in-place writes
                const bool poison = *(volatile unsigned *)&s_gave_up != 0u;
#pragma unroll
                for (int i = 0; i < G::PER; ++i) {
                    walsh<S>(v[i]);
#pragma unroll
                    for (int t = 0; t < S; ++t) {
                        // the scaling by 1/S is exact (S is a power of two)
                        const double y = flip_sign(v[i][t], in_sign[t]) * inv_s;
                        xs[G::SLOTS * i * N + roff[t]] = poison ? __longlong_as_double(0x7ff8000000000000ll) : y;
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic writes -> bulk store
                named_sync(kBarScatter, kWsProducers);
                if (tid == 0) {
                    size_t first;
                    const int valid = tile_rows(j, &first);
                    bulk_store(Y + first * N, xs, (unsigned)valid * N * (unsigned)sizeof(double));
                }
            }
        }
        if (tid == 0) {
            asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
            // After a wait that gave up, bounded waits for loads that may still be in flight.
            if (*(volatile unsigned *)&s_gave_up != 0u)
                for (int k = K > NST ? K - NST : 0; k < K; ++k)
                    (void)mbar_wait(&loaded[k % NST], (unsigned)((k / NST) & 1));
        }
    } else {
        // ------------------------------------------------------------ consumers
        const int cw = warp - kWsProducers / 32;
        const int g = lane >> 2, t4 = lane & 3;
        constexpr int KT = D / 4;
        double wa[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (D == 16) wa[i] = Wp[(t4 + 4 * (i / 2)) * D + g + 8 * (i % 2)];
            else wa[i] = i < KT ? Wp[(4 * i + t4) * D + g] : 0.0;
        }
        for (int k = 0; k < K; ++k) {
            const int st = k % NST;
            if (!mbar_wait(&full[st], (unsigned)((k / NST) & 1))) atomicOr(&s_gave_up, 1u);
            double *xs = stages + st * STAGE;
#pragma unroll
            for (int j = 0; j < G::GPW; j += 2) {
                int n0[2];
                n0[0] = (cw * G::GPW + j) * 8;
                n0[1] = n0[0] + 8;
                if constexpr (D == 16) {
                    double c[2][4];
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        double b[4];
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) b[kk] = xs[ws_index<D>(n0[q] + g, 4 * kk + t4)];
                        c[q][0] = c[q][1] = c[q][2] = c[q][3] = 0.0;
                        mma_16x8x16(c[q], wa, b);
                    }
                    __syncwarp();  // the warp's X' reads of these rows are done before Y' overwrites them
#pragma unroll
                    for (int q = 0; q < 2; ++q)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            xs[ws_index<D>(n0[q] + 2 * t4 + h, g)] = c[q][h];
                            xs[ws_index<D>(n0[q] + 2 * t4 + h, g + 8)] = c[q][2 + h];
                        }
                } else {
                    double c[2][2] = {{0.0, 0.0}, {0.0, 0.0}};
#pragma unroll
                    for (int kk = 0; kk < KT; ++kk)
#pragma unroll
                        for (int q = 0; q < 2; ++q) mma_8x8x4(c[q], wa[kk], xs[ws_index<D>(n0[q] + g, 4 * kk + t4)]);
                    __syncwarp();
#pragma unroll
                    for (int q = 0; q < 2; ++q)
#pragma unroll
                        for (int h = 0; h < 2; ++h) xs[ws_index<D>(n0[q] + 2 * t4 + h, g)] = c[q][h];
                }
            }
            mbar_arrive(&done[st]);
        }
    }
}

template <int D, int S>
cudaError_t launch_rep_fwd(const RepDevice &rep, const double *X, const double *W, const TermParameter &terms,
                           double *Y, size_t batch, cudaStream_t stream) {
    using G = WsGeo<D, S>;
    using P = FwdPipe;
    if (rep.raw_stride != G::N || rep.D != D || rep.S != S) return cudaErrorInvalidValue;
    auto kernel = rep_fwd_kernel<D, S>;
    const size_t smem = (size_t)(D * D + P::STAGES * G::TILE) * sizeof(double) +
                        3 * P::STAGES * sizeof(uint64_t);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kWsThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const size_t tiles = (batch + G::TS - 1) / G::TS;
    size_t grid = (size_t)device_sm_count() * (size_t)per_sm;
    if (grid > tiles) grid = tiles;
    if (grid < 1) grid = 1;
    kernel<<<(unsigned)grid, kWsThreads, smem, stream>>>(rep, X, W, terms, batch, Y);
    return cudaGetLastError();
}

cudaError_t launch_rep_forward_impl(const RepDevice &rep, const double *X, const double *W,
                                    const TermParameter &terms, double *Y, size_t batch, cudaStream_t stream) {
    if (!rep_forward_supported(rep, X, Y)) return cudaErrorInvalidValue;
    if (rep.D == 16 && rep.S == 4) return launch_rep_fwd<16, 4>(rep, X, W, terms, Y, batch, stream);
    if (rep.D == 8 && rep.S == 8) return launch_rep_fwd<8, 8>(rep, X, W, terms, Y, batch, stream);
    if (rep.D == 8 && rep.S == 4) return launch_rep_fwd<8, 4>(rep, X, W, terms, Y, batch, stream);
    if (rep.D == 16 && rep.S == 2) return launch_rep_fwd<16, 2>(rep, X, W, terms, Y, batch, stream);
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// Fused MSE-SGD pass (16-byte aligned x, t and r): the reference device ABI's
// forward -> r = y - t (stored) -> 0.5 r^2 -> parameter VJP of r
// (src/batch_gp_cuda.cu:152-196) in one pass over x and t. Per tile:
//   producers, gather phase: X' = P x in place, as rep_fwd_kernel;
//   consumers, GEMM 1: Y' = X' W' (W'^T fragments resident) into the stage's
//     third tile;
//   producers, residual phase: y = P^-1 Y' exactly as rep_fwd_kernel computes
//     it, r = y - t over the raw target rows in place (one bulk copy stores
//     them), and R' = P r from the same registers into the third tile, as
//     rep_ws_kernel<VJP> gathers its cotangents;
//   consumers, GEMM 2: G' += X'^T R' and the sum of |R'|^2, as rep_ws_kernel<VJP>.
// y is computed by the same operations as rep_fwd_kernel and R' as
// rep_ws_kernel<VJP> computes it from a stored r, on the grid of that kernel,
// so the residuals are bitwise the forward's outputs minus t and the records
// bitwise those of the parameter VJP of the stored residuals, while x is read
// once and r is never read back.
// Handoffs (mbarriers, one phase per tile of a stage): loaded (bulk loads),
// full (X'), done (Y'), resid (R' and r), freed (GEMM 2 has read the stage;
// producer thread 0 waits on it before reloading the stage, together with
// bulk wait_group.read for the residual store). Every wait is bounded; a wait
// that gives up poisons the CTA's remaining residuals and its record.
// CPLX: GEMM 2 in the complex (3M) form, in the order of rep_ws_kernel<VJP, CPLX>.
template <int D, int S, bool CPLX = false>
__global__ void __launch_bounds__(kWsThreads, SgdPipe::CTAS_PER_SM)
rep_sgd_kernel(const RepDevice rep, const double *__restrict__ X, const double *__restrict__ T,
               const double *__restrict__ W, size_t batch, double *R, double *__restrict__ records) {
    using G = WsGeo<D, S>;
    using P = SgdPipe;
    constexpr int N = G::N, TS = G::TS, TILE = G::TILE;
    constexpr int NST = P::STAGES, STAGE = P::ARRAYS * TILE;
    constexpr int kConsumers = kWsThreads - kWsProducers;
    constexpr int kBarProducers = 1;  // named barrier of the producer warps
    static_assert(5 * D * D + kWsThreads <= NST * STAGE, "epilogue scratch fits");
    extern __shared__ __align__(16) double smem[];
    double *Wp = smem;                      // D * D
    double *stages = Wp + D * D;            // NST x (x tile, target tile, Y'/R' tile)
    uint64_t *loaded = reinterpret_cast<uint64_t *>(stages + NST * STAGE);
    uint64_t *full = loaded + NST;
    uint64_t *done = full + NST;
    uint64_t *resid = done + NST;
    uint64_t *freed = resid + NST;
    __shared__ unsigned s_gave_up;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t tiles = (batch + TS - 1) / TS;
    const int K = (size_t)blockIdx.x < tiles ? (int)((tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&loaded[s], 1);
            mbar_init(&full[s], kWsProducers);
            mbar_init(&done[s], kConsumers);
            mbar_init(&resid[s], kWsProducers);
            mbar_init(&freed[s], kConsumers);
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        s_gave_up = 0u;
    }
    build_wprime<D, N>(rep, W, Wp);
    __syncthreads();

    constexpr int PT = D / 8;
    GAcc<D> gacc;
#pragma unroll
    for (int p = 0; p < PT; ++p)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < (D == 16 ? 4 : 2); ++i) gacc[p][h][i] = 0.0;
    double c3[3][2][2];  // CPLX: M1, M2, M3 per k slice parity h
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int h = 0; h < 2; ++h) c3[a][h][0] = c3[a][h][1] = 0.0;
    double sq = 0.0;
    unsigned worst_exp = 0u;

    if (warp < kWsProducers / 32) {
        // ------------------------------------------------------------ producers
        const int slot = tid / D;
        const GroupMap<D, S> gm(rep, tid);
        const double inv_s = 1.0 / (double)S;  // exact: S is a power of two
        auto tile_rows = [&](int k, size_t *first) {
            *first = (blockIdx.x + (size_t)k * gridDim.x) * TS;
            return batch - *first < (size_t)TS ? (int)(batch - *first) : TS;
        };
        auto issue = [&](int k) {
            size_t first;
            const unsigned bytes = (unsigned)tile_rows(k, &first) * N * (unsigned)sizeof(double);
            uint64_t *bar = &loaded[k % NST];
            double *dst = stages + (k % NST) * STAGE;
            mbar_expect_tx(bar, 2u * bytes);
            bulk_load(dst, X + first * N, bytes, bar);
            bulk_load(dst + TILE, T + first * N, bytes, bar);
        };
        if (tid == 0)
            for (int k = 0; k < K && k < P::AHEAD; ++k) issue(k);
        for (int k = 0; k < K + P::LAG; ++k) {
            if (k < K) {
                // gather phase of tile k
                const int st = k % NST;
                if (!mbar_wait(&loaded[st], (unsigned)((k / NST) & 1))) atomicOr(&s_gave_up, 1u);
                size_t first;
                const int valid = tile_rows(k, &first);
                double *xs = stages + st * STAGE;
                double v[G::PER][S];
#pragma unroll
                for (int i = 0; i < G::PER; ++i) {
                    const bool ok = slot + G::SLOTS * i < valid;
#pragma unroll
                    for (int t = 0; t < S; ++t) v[i][t] = ok ? xs[G::SLOTS * i * N + gm.roff[t]] : 0.0;
                }
                named_sync(kBarProducers, kWsProducers);  // every raw read is done before the in-place writes
#pragma unroll
                for (int i = 0; i < G::PER; ++i) {
#pragma unroll
                    for (int t = 0; t < S; ++t) v[i][t] = flip_sign(v[i][t], gm.in_sign[t]);
                    walsh<S>(v[i]);
#pragma unroll
                    for (int f = 0; f < S; ++f)
                        xs[G::SLOTS * i * N + gm.woff[f]] = flip_sign(v[i][f], gm.out_sign[f]);
                }
                mbar_arrive(&full[st]);
            }
            const int j = k - P::LAG;
            if (j >= 0) {
                // residual phase of tile j: every access below is to this thread's own
                // kept entries (woff) and raw blades (roff), so reads and in-place writes
                // need no barrier between them
                const int st = j % NST;
                if (!mbar_wait(&done[st], (unsigned)((j / NST) & 1))) atomicOr(&s_gave_up, 1u);
                size_t first;
                const int valid = tile_rows(j, &first);
                double *ts = stages + st * STAGE + TILE;
                double *ys = ts + TILE;
                const bool poison = *(volatile unsigned *)&s_gave_up != 0u;
#pragma unroll
                for (int i = 0; i < G::PER; ++i) {
                    const bool ok = slot + G::SLOTS * i < valid;
                    double v[S];
#pragma unroll
                    for (int f = 0; f < S; ++f) v[f] = flip_sign(ys[G::SLOTS * i * N + gm.woff[f]], gm.out_sign[f]);
                    walsh<S>(v);
#pragma unroll
                    for (int t = 0; t < S; ++t) {
                        const int at = G::SLOTS * i * N + gm.roff[t];
                        // y exactly as the plain forward computes it (the scaling by 1/S is
                        // exact); rows past the batch contribute zero residuals
                        const double y = flip_sign(v[t], gm.in_sign[t]) * inv_s;
                        double r = ok ? __dsub_rn(y, ts[at]) : 0.0;
                        if (poison) r = __longlong_as_double(0x7ff8000000000000ll);
                        ts[at] = r;
                        v[t] = flip_sign(r, gm.in_sign[t]);
                    }
                    walsh<S>(v);
#pragma unroll
                    for (int f = 0; f < S; ++f) ys[G::SLOTS * i * N + gm.woff[f]] = flip_sign(v[f], gm.out_sign[f]);
                }
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic writes -> bulk store
                mbar_arrive(&resid[st]);
                named_sync(kBarProducers, kWsProducers);  // every residual is written before the store
                if (tid == 0) bulk_store(R + first * N, ts, (unsigned)valid * N * (unsigned)sizeof(double));
            }
            const int ahead = k + P::AHEAD;
            if (tid == 0 && ahead < K) {
                // The stage of `ahead` last held tile ahead - NST: its GEMM 2 is done and
                // its residual store (STORE_PENDING stores ago at most) has read it.
                const int prev = ahead - NST;
                if (prev >= 0) {
                    if (!mbar_wait(&freed[prev % NST], (unsigned)((prev / NST) & 1))) atomicOr(&s_gave_up, 1u);
                    bulk_wait_read<P::STORE_PENDING>();
                }
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                issue(ahead);
            }
        }
        if (tid == 0) {
            asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
            // After a wait that gave up, bounded waits for loads that may still be in flight.
            if (*(volatile unsigned *)&s_gave_up != 0u)
                for (int k = K > NST ? K - NST : 0; k < K; ++k)
                    (void)mbar_wait(&loaded[k % NST], (unsigned)((k / NST) & 1));
        }
    } else {
        // ------------------------------------------------------------ consumers
        const int cw = warp - kWsProducers / 32;
        const int g = lane >> 2, t4 = lane & 3;
        constexpr int KT = D / 4;
        double wa[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (D == 16) wa[i] = Wp[(t4 + 4 * (i / 2)) * D + g + 8 * (i % 2)];
            else wa[i] = i < KT ? Wp[(4 * i + t4) * D + g] : 0.0;
        }
        for (int k = 0; k < K + P::LAG; ++k) {
            if (k < K) {
                // GEMM 1 of tile k: Y' into the third tile
                const int st = k % NST;
                if (!mbar_wait(&full[st], (unsigned)((k / NST) & 1))) atomicOr(&s_gave_up, 1u);
                const double *xs = stages + st * STAGE;
                double *ys = stages + st * STAGE + 2 * TILE;
#pragma unroll
                for (int jj = 0; jj < G::GPW; jj += 2) {
                    int n0[2];
                    n0[0] = (cw * G::GPW + jj) * 8;
                    n0[1] = n0[0] + 8;
                    if constexpr (D == 16) {
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            double b[4], c[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) b[kk] = xs[ws_index<D>(n0[q] + g, 4 * kk + t4)];
                            mma_16x8x16(c, wa, b);
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                ys[ws_index<D>(n0[q] + 2 * t4 + h, g)] = c[h];
                                ys[ws_index<D>(n0[q] + 2 * t4 + h, g + 8)] = c[2 + h];
                            }
                        }
                    } else {
                        double c[2][2] = {{0.0, 0.0}, {0.0, 0.0}};
#pragma unroll
                        for (int kk = 0; kk < KT; ++kk)
#pragma unroll
                            for (int q = 0; q < 2; ++q) mma_8x8x4(c[q], wa[kk], xs[ws_index<D>(n0[q] + g, 4 * kk + t4)]);
#pragma unroll
                        for (int q = 0; q < 2; ++q)
#pragma unroll
                            for (int h = 0; h < 2; ++h) ys[ws_index<D>(n0[q] + 2 * t4 + h, g)] = c[q][h];
                    }
                }
                mbar_arrive(&done[st]);
            }
            const int j = k - P::LAG;
            if (j >= 0) {
                // GEMM 2 of tile j on X' and R', in the order of rep_ws_kernel<VJP>
                const int st = j % NST;
                if (!mbar_wait(&resid[st], (unsigned)((j / NST) & 1))) atomicOr(&s_gave_up, 1u);
                const double *xs = stages + st * STAGE;
                const double *rs = xs + 2 * TILE;
                if constexpr (CPLX) {
                    const unsigned sg_neg = (g & 4) ? 0x80000000u : 0u;
#pragma unroll
                    for (int jj = 0; jj < G::GPW; ++jj) {
                        const int n0 = (cw * G::GPW + jj) * 8;
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int row = n0 + 2 * t4 + h;
                            const double p = rs[ws_index<16>(row, g)];
                            const double q = flip_sign(rs[ws_index<16>(row, g ^ 12)], sg_neg);
                            const double u = xs[ws_index<16>(row, g)];
                            const double v = flip_sign(xs[ws_index<16>(row, g ^ 12)], sg_neg);
                            sq = fma(p, p, sq);
                            sq = fma(q, q, sq);
                            worst_exp = max(worst_exp, max(exponent_bits(p), exponent_bits(q)));
                            mma_8x8x4(c3[0][h], u + v, p);
                            mma_8x8x4(c3[1][h], u, p + q);
                            mma_8x8x4(c3[2][h], v, p - q);
                        }
                    }
                }
#pragma unroll
                for (int jj = 0; jj < G::GPW && !CPLX; jj += 2) {
                    int n0[2];
                    n0[0] = (cw * G::GPW + jj) * 8;
                    n0[1] = n0[0] + 8;
                    if constexpr (D == 16) {
                        double ax[8], rlo[4], rhi[4];
#pragma unroll
                        for (int m = 0; m < 4; ++m) {
                            const int row = n0[m >> 1] + 2 * t4 + (m & 1);
                            const int plo = ws_index<D>(row, g), phi = ws_index<D>(row, g + 8);
                            rlo[m] = rs[plo];
                            rhi[m] = rs[phi];
                            sq = fma(rlo[m], rlo[m], sq);
                            sq = fma(rhi[m], rhi[m], sq);
                            worst_exp = max(worst_exp, max(exponent_bits(rlo[m]), exponent_bits(rhi[m])));
                            ax[2 * m] = xs[plo];
                            ax[2 * m + 1] = xs[phi];
                        }
                        mma_16x8x16(gacc[0][0], ax, rlo);
                        mma_16x8x16(gacc[PT - 1][0], ax, rhi);
                    } else {
#pragma unroll
                        for (int q = 0; q < 2; ++q)
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int pos = ws_index<D>(n0[q] + 2 * t4 + h, g);
                                const double r = rs[pos];
                                sq = fma(r, r, sq);
                                worst_exp = max(worst_exp, exponent_bits(r));
                                mma_8x8x4(gacc[0][h], xs[pos], r);
                            }
                    }
                }
                mbar_arrive(&freed[st]);
            }
        }
    }
    __syncthreads();
    ws_write_record<D, S, CPLX>(rep, gacc, c3, sq, worst_exp, &s_gave_up, stages, records);
}

template <int D, int S>
cudaError_t launch_rep_sgd(const RepDevice &rep, const double *X, const double *T, const double *W, double *R,
                           size_t batch, double *records, int *ctas_used, cudaStream_t stream) {
    using G = WsGeo<D, S>;
    using P = SgdPipe;
    if (rep.raw_stride != G::N || rep.D != D || rep.S != S) return cudaErrorInvalidValue;
    auto kernel = rep_sgd_kernel<D, S>;
    if constexpr (D == 16 && S == 4)
        if (rep.cplx) kernel = rep_sgd_kernel<16, 4, true>;
    const size_t smem = (size_t)(D * D + P::STAGES * P::ARRAYS * G::TILE) * sizeof(double) +
                        5 * P::STAGES * sizeof(uint64_t);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kWsThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    // The grid of launch_rep_ws (two CTAs per SM there too), so that the records
    // partition the batch as the parameter VJP's do.
    const size_t tiles = (batch + G::TS - 1) / G::TS;
    size_t grid = (size_t)device_sm_count() * (size_t)per_sm;
    if (grid > (size_t)kMaxCtas) grid = kMaxCtas;
    if (grid > tiles) grid = tiles;
    if (grid < 1) grid = 1;
    kernel<<<(unsigned)grid, kWsThreads, smem, stream>>>(rep, X, T, W, batch, R, records);
    if (ctas_used) *ctas_used = (int)grid;
    return cudaGetLastError();
}

}  // namespace

bool rep_forward_supported(const RepDevice &rep, const double *X, const double *Y) {
    return rep.ws_ready && rep_supported(rep) && (((uintptr_t)X | (uintptr_t)Y) & 15u) == 0u;
}

cudaError_t launch_rep_forward(const RepDevice &rep, const double *X, const double *W, double *Y, size_t batch,
                               cudaStream_t stream) {
    if (W == nullptr) return cudaErrorInvalidValue;
    TermParameter none;
    none.terms = 0;
    none.values = nullptr;
    return launch_rep_forward_impl(rep, X, W, none, Y, batch, stream);
}

cudaError_t launch_rep_forward_terms(const RepDevice &rep, const double *X, const TermParameter &terms, double *Y,
                                     size_t batch, cudaStream_t stream) {
    if (terms.terms < 1 || terms.terms > 64) return cudaErrorInvalidValue;
    return launch_rep_forward_impl(rep, X, nullptr, terms, Y, batch, stream);
}

cudaError_t launch_rep_cycle(const RepDevice &rep, const double *X, const double *T, const double *W, size_t batch,
                             double *records, int *ctas_used, cudaStream_t stream) {
    const bool al = (((uintptr_t)X | (uintptr_t)T) & 15u) == 0u;
#define GEO_REP_CASE(DD, SS)                                                                             \
    if (rep.D == DD && rep.S == SS)                                                                      \
        return (al && rep.ws_ready) ? launch_rep_ws<DD, SS, false>(rep, X, T, W, batch, records, ctas_used, stream) \
                  : launch_rep_impl<DD, SS, false>(rep, X, T, W, batch, records, ctas_used, stream);
    GEO_REP_CASE(16, 4)
    GEO_REP_CASE(8, 8)
    GEO_REP_CASE(8, 4)
    GEO_REP_CASE(16, 2)
#undef GEO_REP_CASE
    return cudaErrorInvalidValue;
}


bool rep_sgd_supported(const RepDevice &rep, const double *X, const double *T, const double *R) {
    return rep.ws_ready && rep_supported(rep) && (((uintptr_t)X | (uintptr_t)T | (uintptr_t)R) & 15u) == 0u;
}

cudaError_t launch_rep_mse_pass(const RepDevice &rep, const double *X, const double *W, const double *T, double *R,
                                size_t batch, double *records, int *ctas_used, cudaStream_t stream) {
    if (W == nullptr || !rep_sgd_supported(rep, X, T, R)) return cudaErrorInvalidValue;
    if (rep.D == 16 && rep.S == 4) return launch_rep_sgd<16, 4>(rep, X, T, W, R, batch, records, ctas_used, stream);
    if (rep.D == 8 && rep.S == 8) return launch_rep_sgd<8, 8>(rep, X, T, W, R, batch, records, ctas_used, stream);
    if (rep.D == 8 && rep.S == 4) return launch_rep_sgd<8, 4>(rep, X, T, W, R, batch, records, ctas_used, stream);
    if (rep.D == 16 && rep.S == 2) return launch_rep_sgd<16, 2>(rep, X, T, W, R, batch, records, ctas_used, stream);
    return cudaErrorInvalidValue;
}

bool rep_vjp_supported(const RepDevice &rep, const double *X, const double *C) {
    return rep.ws_ready && rep_supported(rep) && (((uintptr_t)X | (uintptr_t)C) & 15u) == 0u;
}

cudaError_t launch_rep_vjp(const RepDevice &rep, const double *X, const double *C, size_t batch, double *records,
                           int *ctas_used, cudaStream_t stream) {
    if (!rep_vjp_supported(rep, X, C)) return cudaErrorInvalidValue;
    if (rep.D == 16 && rep.S == 4) return launch_rep_ws<16, 4, true>(rep, X, C, nullptr, batch, records, ctas_used, stream);
    if (rep.D == 8 && rep.S == 8) return launch_rep_ws<8, 8, true>(rep, X, C, nullptr, batch, records, ctas_used, stream);
    if (rep.D == 8 && rep.S == 4) return launch_rep_ws<8, 4, true>(rep, X, C, nullptr, batch, records, ctas_used, stream);
    if (rep.D == 16 && rep.S == 2) return launch_rep_ws<16, 2, true>(rep, X, C, nullptr, batch, records, ctas_used, stream);
    return cudaErrorInvalidValue;
}

}  // namespace geo
