// operator_mv.cu -- the reference's per-multivector float64 operator calls on
// the GPU, under the reference's names and signatures (geo/operator_kernel.h):
//
//   geo_operator_gp_f64                     reference src/operator_kernel.c:412-447
//   geo_operator_gp_f64_jvp                 reference src/operator_kernel.c:449-492
//   geo_operator_gp_f64_vjp                 reference src/operator_kernel.c:494-539
//   geo_operator_apply_f64                  reference src/operator_kernel.c:191-220
//   geo_operator_apply_parametric_f64       reference src/operator_kernel.c:222-254
//   geo_operator_apply_f64_vjp              reference src/operator_kernel.c:256-278
//   geo_operator_apply_parametric_f64_vjp   reference src/operator_kernel.c:280-334
//
// Each call is one launch of one CTA (thread k owns output blade k, or term k
// for parameter cotangents) on a library stream of the caller's current
// device. The operands travel through a page-locked, device-mapped staging
// block (no device allocation per call); the CTA stages them into shared memory
// and writes its results back through the mapping. The host side validates the
// arguments with the reference's status rules and precedence before anything
// is launched, and returns the reference's output structs (dimension and
// signature copied, coefficients past 2^n zero).
//
// Every output coefficient accumulates its terms in the reference's order with
// explicitly rounded multiplies and adds (no contraction into FMA), and the
// reference's skips are kept (a zero left coefficient of the geometric
// product, a zero input coefficient of apply), so results are bit-identical
// to the reference's CPU code, non-finite operands included.
//
// Calls are synchronous and thread-safe (calls on one device are serialised on
// its staging block). A CUDA failure returns GEO_OPERATOR_B200_DEVICE_FAILURE
// (a status outside the reference's enum; there is no CPU fallback).
#include <cuda_runtime.h>
#include <string.h>

#include <mutex>

#include "geo/geo_b200.h"
#include "geo/operator_kernel.h"
#include "geo_runtime.h"

namespace {

enum MvMode : int {
    kMvGp = 0,
    kMvGpJvp = 1,
    kMvGpVjp = 2,
    kMvApply = 3,
    kMvApplyParametric = 4,
    kMvApplyVjp = 5,
    kMvApplyParametricVjp = 6,
};

constexpr int kMvSlots = 5;  // operand slots of 64 doubles

// Kernel parameter block: the sign tables and the plan's terms.
struct MvArgs {
    uint64_t neg[64];        // geometric product: bit r of neg[l] set when s(l, r) = -1
    uint64_t term_neg[64];   // apply: bit src of term_neg[t] set when the plan's sign of (src, b_t) is -1
    double term_pos[64];     // apply: (double)(+1 * c_t)
    double term_negv[64];    // apply: (double)(-1 * c_t), wrapped as the reference's int product
    uint8_t blade[64];
    int32_t blades;
    int32_t terms;
};

// Staging block (page-locked, mapped): operand slots in, results out.
struct MvBlock {
    double in[kMvSlots][64];
    double out[2][64];
    double pout[64];
};

__device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double sgn(uint64_t mask, int bit) { return ((mask >> bit) & 1ull) ? -1.0 : 1.0; }

template <int MODE>
__global__ void __launch_bounds__(64) operator_mv_kernel(const MvArgs args, MvBlock *block) {
    __shared__ double v[kMvSlots][64];
    const int k = threadIdx.x, N = args.blades, T = args.terms;
    for (int s = 0; s < kMvSlots; ++s) v[s][k] = block->in[s][k];
    __syncthreads();
    if (MODE == kMvGp) {
        // out[o] = sum over left blades l (skipping a zero left coefficient) of (a_l b_(l^o)) s(l, l^o)
        if (k < N) {
            double acc = 0.0;
            for (int l = 0; l < N; ++l) {
                if (v[0][l] == 0.0) continue;
                const int r = l ^ k;
                acc = add(acc, mul(mul(v[0][l], v[1][r]), sgn(args.neg[l], r)));
            }
            block->out[0][k] = acc;
        }
    } else if (MODE == kMvGpJvp) {
        // out[o] = sum_l (ta_l b_r + a_l tb_r) s(l, r), r = l ^ o
        if (k < N) {
            double acc = 0.0;
            for (int l = 0; l < N; ++l) {
                const int r = l ^ k;
                acc = add(acc, mul(add(mul(v[2][l], v[1][r]), mul(v[0][l], v[3][r])), sgn(args.neg[l], r)));
            }
            block->out[0][k] = acc;
        }
    } else if (MODE == kMvGpVjp) {
        // c = cot[l ^ r] s(l, r); left_bar[l] += c b_r (r order), right_bar[r] += c a_l (l order)
        if (k < N) {
            double lacc = 0.0, racc = 0.0;
            for (int j = 0; j < N; ++j) {
                lacc = add(lacc, mul(mul(v[2][k ^ j], sgn(args.neg[k], j)), v[1][j]));
                racc = add(racc, mul(mul(v[2][j ^ k], sgn(args.neg[j], k)), v[0][j]));
            }
            block->out[0][k] = lacc;
            block->out[1][k] = racc;
        }
    } else if (MODE == kMvApply || MODE == kMvApplyParametric) {
        // out[o] += value(src, t) for src ascending (zero inputs skipped), the one
        // term t with src ^ b_t = o; integer plans: src (sign c_t), parametric: (src p_t) sign.
        if (k < N) {
            double acc = 0.0;
            for (int src = 0; src < N; ++src) {
                if (v[0][src] == 0.0) continue;
                for (int t = 0; t < T; ++t) {
                    if ((src ^ args.blade[t]) != k) continue;
                    const bool neg = (args.term_neg[t] >> src) & 1ull;
                    const double term = MODE == kMvApply ? mul(v[0][src], neg ? args.term_negv[t] : args.term_pos[t])
                                                         : mul(mul(v[0][src], v[1][t]), neg ? -1.0 : 1.0);
                    acc = add(acc, term);
                }
            }
            block->out[0][k] = acc;
        }
    } else if (MODE == kMvApplyVjp) {
        // in_bar[src] = sum_t cot[src ^ b_t] (sign c_t), term order
        if (k < N) {
            double acc = 0.0;
            for (int t = 0; t < T; ++t) {
                const bool neg = (args.term_neg[t] >> k) & 1ull;
                acc = add(acc, mul(v[0][k ^ args.blade[t]], neg ? args.term_negv[t] : args.term_pos[t]));
            }
            block->out[0][k] = acc;
        }
    } else {  // kMvApplyParametricVjp: slots 0 = input, 1 = cotangent, 2 = parameters
        if (k < N) {
            double acc = 0.0;
            for (int t = 0; t < T; ++t)
                acc = add(acc, mul(mul(v[1][k ^ args.blade[t]], v[2][t]), sgn(args.term_neg[t], k)));
            block->out[0][k] = acc;
        }
        if (k < T) {
            double acc = 0.0;
            const int b = args.blade[k];
            for (int src = 0; src < N; ++src)
                acc = add(acc, mul(mul(v[1][src ^ b], v[0][src]), sgn(args.term_neg[k], src)));
            block->pout[k] = acc;
        }
    }
}

// ---- per-device staging -------------------------------------------------------
constexpr int kMaxDevices = 64;

struct MvDevice {
    std::mutex mutex;
    MvBlock *host = nullptr;    // page-locked, mapped
    MvBlock *device = nullptr;  // its device address
    cudaStream_t stream = nullptr;
};

MvDevice g_devices[kMaxDevices];
std::mutex g_init;

MvDevice *current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        (void)cudaGetLastError();
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_init);
    MvDevice &d = g_devices[dev];
    if (d.host == nullptr) {
        void *h = nullptr;
        if (cudaHostAlloc(&h, sizeof(MvBlock), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        void *dp = nullptr;
        cudaStream_t s = nullptr;
        if (cudaHostGetDevicePointer(&dp, h, 0) != cudaSuccess ||
            cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
            (void)cudaGetLastError();
            cudaFreeHost(h);
            return nullptr;
        }
        d.device = static_cast<MvBlock *>(dp);
        d.stream = s;
        d.host = static_cast<MvBlock *>(h);
    }
    return &d;
}

template <int MODE>
geo_operator_status_t run(const MvArgs &args, const double *const *in, int slots, double *out0, double *out1,
                          double *pout) {
    MvDevice *d = current_device();
    if (d == nullptr) return (geo_operator_status_t)GEO_OPERATOR_B200_DEVICE_FAILURE;
    std::lock_guard<std::mutex> lock(d->mutex);
    memset(d->host, 0, sizeof(MvBlock));
    for (int s = 0; s < slots; ++s)
        if (in[s] != nullptr) memcpy(d->host->in[s], in[s], 64 * sizeof(double));
    operator_mv_kernel<MODE><<<1, 64, 0, d->stream>>>(args, d->device);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return (geo_operator_status_t)GEO_OPERATOR_B200_DEVICE_FAILURE;
    }
    const int N = args.blades;
    if (out0 != nullptr) memcpy(out0, d->host->out[0], N * sizeof(double));
    if (out1 != nullptr) memcpy(out1, d->host->out[1], N * sizeof(double));
    if (pout != nullptr) memcpy(pout, d->host->pout, args.terms * sizeof(double));
    return GEO_OPERATOR_OK;
}

// ---- the reference's argument rules ------------------------------------------
bool same_metric(uint8_t dimension, const int8_t *a, const int8_t *b) {
    for (unsigned i = 0; i < dimension; ++i)
        if (a[i] != b[i]) return false;
    return true;
}

bool mv_matches(const geo_operator_mv_f64_t *v, uint8_t dimension, const int8_t *signature) {
    return v != nullptr && v->dimension == dimension && same_metric(dimension, v->signature, signature);
}

// Zeroed multivector carrying the metric (the reference's result initialisation).
void mv_init(geo_operator_mv_f64_t *v, uint8_t dimension, const int8_t *signature) {
    memset(v, 0, sizeof(*v));
    v->dimension = dimension;
    memcpy(v->signature, signature, dimension);
}

// reference src/operator_kernel.c:70-86
geo_operator_status_t validate_plan(const geo_operator_plan_i32_t *plan) {
    if (plan == nullptr) return GEO_OPERATOR_INVALID_ARGUMENT;
    const unsigned blades = geo::dimension_valid(plan->dimension) ? 1u << plan->dimension : 0u;
    if (plan->abi_version != GEO_OPERATOR_ABI_VERSION) return GEO_OPERATOR_BAD_PLAN;
    if (!geo::signature_valid(plan->signature, plan->dimension)) return GEO_OPERATOR_BAD_PLAN;
    if (plan->side != GEO_OPERATOR_SIDE_LEFT && plan->side != GEO_OPERATOR_SIDE_RIGHT) return GEO_OPERATOR_BAD_PLAN;
    if (plan->kind != GEO_OPERATOR_PLAN_FIXED_BLADE && plan->kind != GEO_OPERATOR_PLAN_SPARSE_FIXED_MULTIVECTOR)
        return GEO_OPERATOR_BAD_PLAN;
    if (plan->term_count == 0u || plan->term_count > GEO_OPERATOR_MAX_TERMS) return GEO_OPERATOR_BAD_PLAN;
    if (plan->kind == GEO_OPERATOR_PLAN_FIXED_BLADE && plan->term_count != 1u) return GEO_OPERATOR_BAD_PLAN;
    for (unsigned t = 0; t < plan->term_count; ++t)
        if ((unsigned)plan->terms[t].blade >= blades || plan->terms[t].coefficient == 0) return GEO_OPERATOR_BAD_PLAN;
    return GEO_OPERATOR_OK;
}

// Sign tables of a validated plan; the coefficient products are the reference's
// int multiply sign * c_t (two's-complement wrap for c_t = INT32_MIN).
MvArgs plan_args(const geo_operator_plan_i32_t *plan) {
    MvArgs a;
    memset(&a, 0, sizeof a);
    a.blades = 1 << plan->dimension;
    a.terms = plan->term_count;
    for (int t = 0; t < a.terms; ++t) {
        const uint8_t b = plan->terms[t].blade;
        a.blade[t] = b;
        a.term_pos[t] = (double)plan->terms[t].coefficient;
        a.term_negv[t] = (double)(int32_t)(0u - (uint32_t)plan->terms[t].coefficient);
        uint64_t m = 0;
        for (int src = 0; src < a.blades; ++src) {
            const int s = plan->side == GEO_OPERATOR_SIDE_RIGHT
                              ? geo::sign_rule((uint8_t)src, b, plan->signature, plan->dimension)
                              : geo::sign_rule(b, (uint8_t)src, plan->signature, plan->dimension);
            if (s < 0) m |= 1ull << src;
        }
        a.term_neg[t] = m;
    }
    return a;
}

MvArgs product_args(uint8_t dimension, const int8_t *signature) {
    MvArgs a;
    memset(&a, 0, sizeof a);
    a.blades = 1 << dimension;
    for (int l = 0; l < a.blades; ++l) {
        uint64_t m = 0;
        for (int r = 0; r < a.blades; ++r)
            if (geo::sign_rule((uint8_t)l, (uint8_t)r, signature, dimension) < 0) m |= 1ull << r;
        a.neg[l] = m;
    }
    return a;
}

// Common checks of the geometric-product family (reference :421-428).
geo_operator_status_t check_pair(const geo_operator_mv_f64_t *left, const geo_operator_mv_f64_t *right) {
    if (!geo::dimension_valid(left->dimension) || left->dimension != right->dimension)
        return GEO_OPERATOR_UNSUPPORTED_DIMENSION;
    if (!geo::signature_valid(left->signature, left->dimension) ||
        !same_metric(left->dimension, left->signature, right->signature))
        return GEO_OPERATOR_INVALID_ARGUMENT;
    return GEO_OPERATOR_OK;
}

}  // namespace

extern "C" geo_operator_status_t geo_operator_gp_f64(const geo_operator_mv_f64_t *left,
                                                     const geo_operator_mv_f64_t *right,
                                                     geo_operator_mv_f64_t *output) {
    if (left == nullptr || right == nullptr || output == nullptr) return GEO_OPERATOR_INVALID_ARGUMENT;
    geo_operator_status_t st = check_pair(left, right);
    if (st != GEO_OPERATOR_OK) return st;
    geo::NvtxRange range("geo_operator_gp_f64");
    const MvArgs args = product_args(left->dimension, left->signature);
    const double *in[2] = {left->coefficients, right->coefficients};
    geo_operator_mv_f64_t result;
    mv_init(&result, left->dimension, left->signature);
    st = run<kMvGp>(args, in, 2, result.coefficients, nullptr, nullptr);
    if (st == GEO_OPERATOR_OK) *output = result;
    return st;
}

extern "C" geo_operator_status_t geo_operator_gp_f64_jvp(const geo_operator_mv_f64_t *left,
                                                         const geo_operator_mv_f64_t *right,
                                                         const geo_operator_mv_f64_t *left_tangent,
                                                         const geo_operator_mv_f64_t *right_tangent,
                                                         geo_operator_mv_f64_t *output_tangent) {
    if (left == nullptr || right == nullptr || left_tangent == nullptr || right_tangent == nullptr ||
        output_tangent == nullptr)
        return GEO_OPERATOR_INVALID_ARGUMENT;
    geo_operator_status_t st = check_pair(left, right);
    if (st != GEO_OPERATOR_OK) return st;
    if (!mv_matches(left_tangent, left->dimension, left->signature) ||
        !mv_matches(right_tangent, left->dimension, left->signature))
        return GEO_OPERATOR_INVALID_ARGUMENT;
    geo::NvtxRange range("geo_operator_gp_f64_jvp");
    const MvArgs args = product_args(left->dimension, left->signature);
    const double *in[4] = {left->coefficients, right->coefficients, left_tangent->coefficients,
                           right_tangent->coefficients};
    geo_operator_mv_f64_t result;
    mv_init(&result, left->dimension, left->signature);
    st = run<kMvGpJvp>(args, in, 4, result.coefficients, nullptr, nullptr);
    if (st == GEO_OPERATOR_OK) *output_tangent = result;
    return st;
}

extern "C" geo_operator_status_t geo_operator_gp_f64_vjp(const geo_operator_mv_f64_t *left,
                                                         const geo_operator_mv_f64_t *right,
                                                         const geo_operator_mv_f64_t *output_cotangent,
                                                         geo_operator_mv_f64_t *left_cotangent,
                                                         geo_operator_mv_f64_t *right_cotangent) {
    if (left == nullptr || right == nullptr || output_cotangent == nullptr || left_cotangent == nullptr ||
        right_cotangent == nullptr || left_cotangent == right_cotangent)
        return GEO_OPERATOR_INVALID_ARGUMENT;
    geo_operator_status_t st = check_pair(left, right);
    if (st != GEO_OPERATOR_OK) return st;
    if (!mv_matches(output_cotangent, left->dimension, left->signature)) return GEO_OPERATOR_INVALID_ARGUMENT;
    geo::NvtxRange range("geo_operator_gp_f64_vjp");
    const MvArgs args = product_args(left->dimension, left->signature);
    const double *in[3] = {left->coefficients, right->coefficients, output_cotangent->coefficients};
    geo_operator_mv_f64_t lres, rres;
    mv_init(&lres, left->dimension, left->signature);
    mv_init(&rres, left->dimension, left->signature);
    st = run<kMvGpVjp>(args, in, 3, lres.coefficients, rres.coefficients, nullptr);
    if (st == GEO_OPERATOR_OK) {
        *left_cotangent = lres;
        *right_cotangent = rres;
    }
    return st;
}

extern "C" geo_operator_status_t geo_operator_apply_f64(const geo_operator_plan_i32_t *plan,
                                                        const geo_operator_mv_f64_t *input,
                                                        geo_operator_mv_f64_t *output) {
    geo_operator_status_t st = validate_plan(plan);
    if (st != GEO_OPERATOR_OK) return st;
    if (input == nullptr || output == nullptr) return GEO_OPERATOR_INVALID_ARGUMENT;
    if (!mv_matches(input, plan->dimension, plan->signature)) return GEO_OPERATOR_INVALID_ARGUMENT;
    geo::NvtxRange range("geo_operator_apply_f64");
    const MvArgs args = plan_args(plan);
    const double *in[1] = {input->coefficients};
    geo_operator_mv_f64_t result;
    mv_init(&result, plan->dimension, plan->signature);
    st = run<kMvApply>(args, in, 1, result.coefficients, nullptr, nullptr);
    if (st == GEO_OPERATOR_OK) *output = result;
    return st;
}

extern "C" geo_operator_status_t geo_operator_apply_parametric_f64(const geo_operator_plan_i32_t *plan,
                                                                   const double *parameters, size_t parameter_count,
                                                                   const geo_operator_mv_f64_t *input,
                                                                   geo_operator_mv_f64_t *output) {
    geo_operator_status_t st = validate_plan(plan);
    if (st != GEO_OPERATOR_OK) return st;
    if (parameters == nullptr || input == nullptr || output == nullptr) return GEO_OPERATOR_INVALID_ARGUMENT;
    if (parameter_count != (size_t)plan->term_count) return GEO_OPERATOR_INVALID_ARGUMENT;
    if (!mv_matches(input, plan->dimension, plan->signature)) return GEO_OPERATOR_INVALID_ARGUMENT;
    geo::NvtxRange range("geo_operator_apply_parametric_f64");
    const MvArgs args = plan_args(plan);
    double p[64] = {0.0};
    memcpy(p, parameters, parameter_count * sizeof(double));
    const double *in[2] = {input->coefficients, p};
    geo_operator_mv_f64_t result;
    mv_init(&result, plan->dimension, plan->signature);
    st = run<kMvApplyParametric>(args, in, 2, result.coefficients, nullptr, nullptr);
    if (st == GEO_OPERATOR_OK) *output = result;
    return st;
}

extern "C" geo_operator_status_t geo_operator_apply_f64_vjp(const geo_operator_plan_i32_t *plan,
                                                            const geo_operator_mv_f64_t *output_cotangent,
                                                            geo_operator_mv_f64_t *input_cotangent) {
    geo_operator_status_t st = validate_plan(plan);
    if (st != GEO_OPERATOR_OK) return st;
    if (output_cotangent == nullptr || input_cotangent == nullptr) return GEO_OPERATOR_INVALID_ARGUMENT;
    if (!mv_matches(output_cotangent, plan->dimension, plan->signature)) return GEO_OPERATOR_INVALID_ARGUMENT;
    geo::NvtxRange range("geo_operator_apply_f64_vjp");
    const MvArgs args = plan_args(plan);
    const double *in[1] = {output_cotangent->coefficients};
    geo_operator_mv_f64_t result;
    mv_init(&result, plan->dimension, plan->signature);
    st = run<kMvApplyVjp>(args, in, 1, result.coefficients, nullptr, nullptr);
    if (st == GEO_OPERATOR_OK) *input_cotangent = result;
    return st;
}

extern "C" geo_operator_status_t geo_operator_apply_parametric_f64_vjp(
    const geo_operator_plan_i32_t *plan, const double *parameters, size_t parameter_count,
    const geo_operator_mv_f64_t *input, const geo_operator_mv_f64_t *output_cotangent,
    geo_operator_mv_f64_t *input_cotangent, double *parameter_cotangents, size_t parameter_cotangent_count) {
    geo_operator_status_t st = validate_plan(plan);
    if (st != GEO_OPERATOR_OK) return st;
    if (parameters == nullptr || input == nullptr || output_cotangent == nullptr || input_cotangent == nullptr ||
        parameter_cotangents == nullptr)
        return GEO_OPERATOR_INVALID_ARGUMENT;
    if (parameter_count != (size_t)plan->term_count || parameter_cotangent_count < (size_t)plan->term_count)
        return GEO_OPERATOR_INVALID_ARGUMENT;
    if (!mv_matches(input, plan->dimension, plan->signature) ||
        !mv_matches(output_cotangent, plan->dimension, plan->signature))
        return GEO_OPERATOR_INVALID_ARGUMENT;
    geo::NvtxRange range("geo_operator_apply_parametric_f64_vjp");
    const MvArgs args = plan_args(plan);
    double p[64] = {0.0};
    memcpy(p, parameters, parameter_count * sizeof(double));
    const double *in[3] = {input->coefficients, output_cotangent->coefficients, p};
    geo_operator_mv_f64_t result;
    mv_init(&result, plan->dimension, plan->signature);
    double pc[64];
    st = run<kMvApplyParametricVjp>(args, in, 3, result.coefficients, nullptr, pc);
    if (st == GEO_OPERATOR_OK) {
        *input_cotangent = result;
        memcpy(parameter_cotangents, pc, (size_t)plan->term_count * sizeof(double));
    }
    return st;
}
