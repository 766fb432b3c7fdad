// sparse.cu -- sparse fixed-multivector operator plans over a batch
// (geo_b200_sparse_*).
//
// Reference semantics batched here (reference tree file:line):
//   geo_operator_apply_f64, _apply_parametric_f64        src/operator_kernel.c:191-254
//   geo_operator_apply_f64_vjp, _parametric_f64_vjp      src/operator_kernel.c:256-334
// A plan is W = sum_t c_t e_{b_t} on one side (c_t the integer coefficients or
// the caller's parameters), and
//   apply:       out[s][src ^ b_t] += in[s][src] * sign_t(src) * c_t
//   input VJP:   in_bar[s][src]    += out_bar[s][src ^ b_t] * sign_t(src) * c_t
//   parameters:  c_bar[t]          += out_bar[s][src ^ b_t] * in[s][src] * sign_t(src)
// with sign_t(src) = s(src, b_t) (right side) or s(b_t, src) (left side).
//
// Kernel routes:
//  * sparse_stream_kernel (every n; plans of fewer than kDenseMinTerms terms
//    at n = 5, 6): rows stream through registers with coalesced loads and
//    stores. For 2^n >= 32 a warp holds one row (lane l owns blades l and
//    l + 32), otherwise 32 / 2^n rows; the source of term t for output blade o
//    is o ^ b_t, which is lane ^ (b_t mod 32) in the same or the other half, so
//    it is one shfl.bfly per value. One FMA per term and output, in term order:
//    a non-finite input reaches exactly the outputs its terms reach, as in the
//    reference.
//  * dense route (n = 5, 6, kDenseMinTerms terms or more, 16-byte aligned
//    rows): apply is the fixed-parameter product x W (or W x) on the
//    representation kernel (FP64 tensor cores). Right (left) multiplication by
//    a blade e_b is a signed permutation R_b with R_b R_b = s(b,b) 1, so
//    R_b^T = s(b,b) R_b and the input VJP is the same product with
//    W~ = sum_t s(b_t,b_t) c_t e_{b_t}. Finite inputs agree with the per-term
//    sums to rounding; a non-finite input coefficient makes every output
//    coefficient of its sample non-finite.
//  * parameter cotangents (n = 5, 6, 16-byte aligned rows): the batched
//    parameter VJP of the representation kernel, read at the plan's blades
//    (c_bar[t] is the parameter gradient g_{b_t}). Otherwise sparse_kernel.
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include "geo/geo_b200.h"
#include "geo_runtime.h"

namespace {

constexpr int kThreads = 256;
constexpr int kStreamThreads = 256;
// Row sets per warp iteration (loads in flight per warp): 16 measured 0.96 of the
// copy bandwidth for a one-blade plan at 2^22 rows, 4 gave 0.92 and 8 gave 0.93.
constexpr int kStreamSets = 16;
constexpr int kDenseMinTerms = 5;  // plans with this many terms take the dense route at n = 5, 6

geo_b200_status_t from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return GEO_B200_OK;
    (void)cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? GEO_B200_ALLOCATION_FAILURE : GEO_B200_RUNTIME_FAILURE;
}

__device__ __forceinline__ double apply_sign(double v, bool negative) { return negative ? -v : v; }

// v with its sign bit XORed by `mask` (0 or 0x80000000): an integer operation.
__device__ __forceinline__ double flip_sign(double v, unsigned mask) {
    return __hiloint2double(__double2hiint(v) ^ (int)mask, __double2loint(v));
}

struct SparsePlan {
    uint64_t negmask[64];  // bit src set when the sign of (src, blade_t) on the plan's side is -1
    double coeff[64];      // integer coefficients as doubles (ignored by parametric calls)
    uint8_t blade[64];
    int32_t terms;
    int32_t blades;
};

bool make_sparse_plan(const geo_operator_plan_i32_t *p, SparsePlan *out) {
    if (p == nullptr || p->abi_version != GEO_OPERATOR_ABI_VERSION || !geo::signature_valid(p->signature, p->dimension))
        return false;
    if (p->side != GEO_OPERATOR_SIDE_LEFT && p->side != GEO_OPERATOR_SIDE_RIGHT) return false;
    if (p->kind != GEO_OPERATOR_PLAN_FIXED_BLADE && p->kind != GEO_OPERATOR_PLAN_SPARSE_FIXED_MULTIVECTOR) return false;
    if (p->term_count == 0 || p->term_count > GEO_OPERATOR_MAX_TERMS) return false;
    if (p->kind == GEO_OPERATOR_PLAN_FIXED_BLADE && p->term_count != 1) return false;
    memset(out, 0, sizeof(*out));
    const unsigned blades = 1u << p->dimension;
    out->terms = p->term_count;
    out->blades = (int32_t)blades;
    for (unsigned t = 0; t < p->term_count; ++t) {
        if (p->terms[t].blade >= blades || p->terms[t].coefficient == 0) return false;
        out->blade[t] = p->terms[t].blade;
        out->coeff[t] = (double)p->terms[t].coefficient;
        uint64_t m = 0;
        for (unsigned src = 0; src < blades; ++src) {
            // reference src/operator_kernel.c:88-96: right side s(src, blade), left side s(blade, src)
            const int s = p->side == GEO_OPERATOR_SIDE_RIGHT
                              ? geo::sign_rule((uint8_t)src, p->terms[t].blade, p->signature, p->dimension)
                              : geo::sign_rule(p->terms[t].blade, (uint8_t)src, p->signature, p->dimension);
            if (s < 0) m |= (uint64_t)1 << src;
        }
        out->negmask[t] = m;
    }
    return true;
}

enum SparseMode : int { kSparseApply = 0, kSparseVjpInput = 1, kSparseParamVjp = 2 };

// ---- streaming per-term kernel ----------------------------------------------

// kSparseApply:    out[o]   = sum_t in[o ^ b_t]  c_t sign_t(o ^ b_t)
// kSparseVjpInput: out[src] = sum_t cot[src ^ b_t] c_t sign_t(src)
template <int N, int MODE>
__global__ void __launch_bounds__(kStreamThreads)
sparse_stream_kernel(const SparsePlan plan, const double *__restrict__ params, const double *in, double *out,
                     size_t batch) {
    constexpr int H = N >= 32 ? N / 32 : 1;  // blades per lane
    constexpr int R = N >= 32 ? 1 : 32 / N;  // rows per warp row set
    constexpr int U = kStreamSets;
    constexpr int kWarpsPerBlock = kStreamThreads / 32;
    __shared__ double coeff[64];
    if (threadIdx.x < plan.terms) coeff[threadIdx.x] = params != nullptr ? params[threadIdx.x] : plan.coeff[threadIdx.x];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int blade0 = N >= 32 ? lane : (lane & (N - 1));  // this lane's blade in half 0
    const int row_in_set = N >= 32 ? 0 : lane / N;
    // Bit t of sg[h]: term t enters this lane's output blade of half h with a negative sign.
    uint64_t sg[H];
#pragma unroll
    for (int h = 0; h < H; ++h) {
        sg[h] = 0;
        const int o = blade0 + 32 * h;
        for (int t = 0; t < plan.terms; ++t) {
            const int idx = MODE == kSparseApply ? (o ^ plan.blade[t]) : o;
            if ((plan.negmask[t] >> idx) & 1ull) sg[h] |= 1ull << t;
        }
    }
    const size_t sets = (batch + R - 1) / R;
    const size_t stride = (size_t)gridDim.x * kWarpsPerBlock * U;
    for (size_t s0 = ((size_t)blockIdx.x * kWarpsPerBlock + warp) * U; s0 < sets; s0 += stride) {
        double v[U][H], acc[U][H];
        size_t row[U];
        bool ok[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            row[u] = (s0 + u) * R + row_in_set;
            ok[u] = s0 + u < sets && row[u] < batch;
#pragma unroll
            for (int h = 0; h < H; ++h) {
                v[u][h] = ok[u] ? __ldcs(in + row[u] * N + blade0 + 32 * h) : 0.0;
                acc[u][h] = 0.0;
            }
        }
        for (int t = 0; t < plan.terms; ++t) {
            const int b = plan.blade[t];
            const int bl = N >= 32 ? (b & 31) : b;
            const int bh = N >= 64 ? (b >> 5) : 0;
            const double c = coeff[t];
#pragma unroll
            for (int h = 0; h < H; ++h) {
                const double ch = flip_sign(c, (unsigned)((sg[h] >> t) & 1ull) << 31);
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    // source half h ^ bh (bh is the same for the whole warp)
                    const double sv = (H == 2 && ((h ^ bh) & 1)) ? v[u][H - 1] : v[u][0];
                    acc[u][h] = fma(__shfl_xor_sync(0xffffffffu, sv, bl), ch, acc[u][h]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (ok[u])
#pragma unroll
                for (int h = 0; h < H; ++h) __stcs(out + row[u] * N + blade0 + 32 * h, acc[u][h]);
    }
}

template <int N, int MODE>
cudaError_t launch_stream_n(const SparsePlan &plan, const double *params, const double *in, double *out,
                            size_t batch, cudaStream_t stream) {
    auto kernel = sparse_stream_kernel<N, MODE>;
    int per_sm = 1;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kStreamThreads, 0);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    constexpr int R = N >= 32 ? 1 : 32 / N;
    const size_t sets = (batch + R - 1) / R;
    const size_t per_block = (size_t)(kStreamThreads / 32) * kStreamSets;
    size_t grid = (sets + per_block - 1) / per_block;
    const size_t cap = (size_t)geo::device_sm_count() * (size_t)per_sm;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    kernel<<<(unsigned)grid, kStreamThreads, 0, stream>>>(plan, params, in, out, batch);
    return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_stream(const SparsePlan &plan, const double *params, const double *in, double *out, size_t batch,
                          cudaStream_t stream) {
    switch (plan.blades) {
        case 2: return launch_stream_n<2, MODE>(plan, params, in, out, batch, stream);
        case 4: return launch_stream_n<4, MODE>(plan, params, in, out, batch, stream);
        case 8: return launch_stream_n<8, MODE>(plan, params, in, out, batch, stream);
        case 16: return launch_stream_n<16, MODE>(plan, params, in, out, batch, stream);
        case 32: return launch_stream_n<32, MODE>(plan, params, in, out, batch, stream);
        case 64: return launch_stream_n<64, MODE>(plan, params, in, out, batch, stream);
        default: return cudaErrorInvalidValue;
    }
}

// ---- per-element kernel for the parameter cotangents -------------------------

// Stage `rows` samples of width `width` starting at `first` into smem (zero-fill past batch).
__device__ __forceinline__ void stage(double *dst, const double *__restrict__ src, size_t first, int rows, int width,
                                     size_t batch) {
    for (int i = threadIdx.x; i < rows * width; i += blockDim.x) {
        const int s = i / width;
        const size_t sample = first + (size_t)s;
        dst[i] = sample < batch ? src[sample * width + (i - s * width)] : 0.0;
    }
}

// Thread (s, j) owns blade j of sample s of a pass: it writes the input
// cotangent of blade j (out may be null) and accumulates parameter term t = j
// (j < terms); records[cta][t] receives the CTA's sums in sample-slot order.
__global__ void __launch_bounds__(kThreads)
sparse_param_vjp_kernel(const SparsePlan plan, const double *__restrict__ params, const double *__restrict__ a,
                        const double *__restrict__ b, double *__restrict__ out, size_t batch,
                        double *__restrict__ records) {
    const int N = plan.blades;
    const int per_pass = kThreads / N;
    extern __shared__ __align__(16) double sm[];
    double *As = sm;                    // per_pass * N  (inputs)
    double *Bs = As + per_pass * N;     // per_pass * N  (output cotangents)
    __shared__ double coeff[64];
    __shared__ double pacc[kThreads];
    if (threadIdx.x < plan.terms) coeff[threadIdx.x] = params[threadIdx.x];
    const int s = threadIdx.x / N;
    const int j = threadIdx.x - s * N;
    const bool lane_ok = s < per_pass;
    double pa = 0.0;
    for (size_t first = (size_t)blockIdx.x * per_pass; first < batch; first += (size_t)gridDim.x * per_pass) {
        __syncthreads();
        stage(As, a, first, per_pass, N, batch);
        stage(Bs, b, first, per_pass, N, batch);
        __syncthreads();
        const size_t sample = first + (size_t)s;
        if (!lane_ok || sample >= batch) continue;
        const double *row = As + s * N;
        const double *cot = Bs + s * N;
        if (out != nullptr) {
            double acc = 0.0;
            for (int t = 0; t < plan.terms; ++t)
                acc = fma(cot[j ^ plan.blade[t]], apply_sign(coeff[t], (plan.negmask[t] >> j) & 1ull), acc);
            out[sample * N + j] = acc;
        }
        if (j < plan.terms) {
            const uint64_t m = plan.negmask[j];
            const int bt = plan.blade[j];
            double acc = 0.0;
            for (int src = 0; src < N; ++src) acc = fma(apply_sign(cot[src ^ bt], (m >> src) & 1ull), row[src], acc);
            pa += acc;
        }
    }
    pacc[threadIdx.x] = pa;
    __syncthreads();
    if (threadIdx.x < plan.terms) {
        double acc = 0.0;
        for (int ss = 0; ss < per_pass; ++ss) acc += pacc[ss * N + threadIdx.x];
        records[(size_t)blockIdx.x * geo::kRecStride + threadIdx.x] = acc;
    } else if (threadIdx.x < geo::kRecStride) {
        records[(size_t)blockIdx.x * geo::kRecStride + threadIdx.x] = 0.0;
    }
}

// dst[t] = src[index[t]] for t < count (index null: the identity).
__global__ void select_kernel(const double *__restrict__ src, const SparsePlan plan, int use_blades,
                              double *__restrict__ dst) {
    const int t = threadIdx.x;
    if (t < plan.terms) dst[t] = src[use_blades ? plan.blade[t] : t];
}

// ---- routing ------------------------------------------------------------------

// The representation tables for a plan at n = 5, 6, or null.
const geo::RepDevice *plan_rep(const geo_operator_plan_i32_t *p) {
    return geo::cached_rep_device(p->dimension, p->signature, p->side == GEO_OPERATOR_SIDE_LEFT);
}

// Term list of the plan (values = parameters when given); `vjp` multiplies term t by s(b_t, b_t).
geo::TermParameter term_parameter(const geo_operator_plan_i32_t *p, const SparsePlan &sp, const double *params,
                                  bool vjp) {
    geo::TermParameter tp;
    memset(&tp, 0, sizeof(tp));
    tp.terms = sp.terms;
    tp.values = params;
    for (int t = 0; t < sp.terms; ++t) {
        const int s = vjp ? geo::sign_rule(sp.blade[t], sp.blade[t], p->signature, p->dimension) : 1;
        tp.blade[t] = sp.blade[t];
        tp.scale[t] = (int8_t)s;
        tp.coeff[t] = s * sp.coeff[t];
    }
    return tp;
}

// apply (vjp = false) or input VJP (vjp = true) of a validated plan.
template <int MODE>
geo_b200_status_t per_element(const geo_operator_plan_i32_t *p, const SparsePlan &sp, const double *params,
                              const double *in, double *out, size_t batch, cudaStream_t stream) {
    const geo::RepDevice *rep = sp.terms >= kDenseMinTerms ? plan_rep(p) : nullptr;
    if (rep != nullptr && geo::rep_forward_supported(*rep, in, out)) {
        const geo::TermParameter tp = term_parameter(p, sp, params, MODE == kSparseVjpInput);
        return from_cuda(geo::launch_rep_forward_terms(*rep, in, tp, out, batch, stream));
    }
    return from_cuda(launch_stream<MODE>(sp, params, in, out, batch, stream));
}

geo_b200_status_t param_vjp(const geo_operator_plan_i32_t *p, const SparsePlan &sp, const double *params,
                            const double *in, const double *cot, double *in_cot, double *param_out, size_t batch,
                            cudaStream_t stream) {
    const geo::RepDevice *rep = plan_rep(p);
    const bool use_rep = rep != nullptr && geo::rep_vjp_supported(*rep, in, cot);
    size_t grid = 0;
    if (!use_rep) {
        const int per_pass = kThreads / sp.blades;
        grid = (batch + per_pass - 1) / per_pass;
        const size_t cap = (size_t)geo::device_sm_count() * 4;
        if (grid > cap) grid = cap;
        if (grid > (size_t)geo::kMaxCtas) grid = geo::kMaxCtas;
    }
    // Stream-ordered scratch for the per-CTA records and their sum (pool-cached after first use).
    const size_t slots = use_rep ? (size_t)geo::kMaxCtas : grid;
    double *records = nullptr;
    cudaError_t e = cudaMallocAsync((void **)&records, (slots + 1) * geo::kRecStride * sizeof(double), stream);
    if (e != cudaSuccess) return from_cuda(e);
    double *sum = records + slots * geo::kRecStride;
    int ctas = 0;
    if (use_rep) {
        e = geo::launch_rep_vjp(*rep, in, cot, batch, records, &ctas, stream);
    } else {
        const size_t smem = (size_t)2 * (kThreads / sp.blades) * sp.blades * sizeof(double);
        sparse_param_vjp_kernel<<<(unsigned)grid, kThreads, smem, stream>>>(sp, params, in, cot, in_cot, batch,
                                                                            records);
        e = cudaGetLastError();
        ctas = (int)grid;
    }
    if (e == cudaSuccess) e = geo::launch_reduce_records(records, ctas, sum, stream);
    if (e == cudaSuccess) {
        select_kernel<<<1, 64, 0, stream>>>(sum, sp, use_rep ? 1 : 0, param_out);
        e = cudaGetLastError();
    }
    cudaFreeAsync(records, stream);
    if (e != cudaSuccess) return from_cuda(e);
    if (use_rep && in_cot != nullptr) return per_element<kSparseVjpInput>(p, sp, params, cot, in_cot, batch, stream);
    return GEO_B200_OK;
}

}  // namespace

extern "C" geo_b200_status_t geo_b200_sparse_apply_f64(const geo_operator_plan_i32_t *plan, const double *device_in,
                                                       double *device_out, size_t batch, cudaStream_t stream) {
    SparsePlan sp;
    if (device_out == nullptr || device_in == nullptr || batch == 0 || !make_sparse_plan(plan, &sp))
        return GEO_B200_INVALID_ARGUMENT;
    return per_element<kSparseApply>(plan, sp, nullptr, device_in, device_out, batch, stream);
}

extern "C" geo_b200_status_t geo_b200_sparse_apply_parametric_f64(const geo_operator_plan_i32_t *plan,
                                                                  const double *device_parameters,
                                                                  const double *device_in, double *device_out,
                                                                  size_t batch, cudaStream_t stream) {
    SparsePlan sp;
    if (device_out == nullptr || device_parameters == nullptr || device_in == nullptr || batch == 0 ||
        !make_sparse_plan(plan, &sp))
        return GEO_B200_INVALID_ARGUMENT;
    return per_element<kSparseApply>(plan, sp, device_parameters, device_in, device_out, batch, stream);
}

extern "C" geo_b200_status_t geo_b200_sparse_apply_vjp_f64(const geo_operator_plan_i32_t *plan,
                                                           const double *device_out_cotangent,
                                                           double *device_in_cotangent, size_t batch,
                                                           cudaStream_t stream) {
    SparsePlan sp;
    if (device_in_cotangent == nullptr || device_out_cotangent == nullptr || batch == 0 ||
        !make_sparse_plan(plan, &sp))
        return GEO_B200_INVALID_ARGUMENT;
    return per_element<kSparseVjpInput>(plan, sp, nullptr, device_out_cotangent, device_in_cotangent, batch, stream);
}

extern "C" geo_b200_status_t geo_b200_sparse_apply_parametric_vjp_f64(
    const geo_operator_plan_i32_t *plan, const double *device_parameters, const double *device_in,
    const double *device_out_cotangent, double *device_in_cotangent, double *device_parameter_cotangent,
    size_t batch, cudaStream_t stream) {
    SparsePlan sp;
    if (device_parameters == nullptr || device_in == nullptr || device_out_cotangent == nullptr ||
        device_parameter_cotangent == nullptr || batch == 0 || !make_sparse_plan(plan, &sp))
        return GEO_B200_INVALID_ARGUMENT;
    return param_vjp(plan, sp, device_parameters, device_in, device_out_cotangent, device_in_cotangent,
                     device_parameter_cotangent, batch, stream);
}
