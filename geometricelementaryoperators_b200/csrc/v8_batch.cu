// v8_batch.cu -- batched execution of a compiled V8 program of any shape over a
// device-resident minibatch (the general path of geo_b200_v8_batch_train_step
// and geo_b200_v8_batch_forward).
//
// The reference trains a V8 graph one sample at a time: set INPUT and TARGET,
// geo_v8_forward, geo_v8_backward(accumulate) (src/full_cycle_v8.c:569-692,
// 717-940). Here one warp runs that per-sample forward and backward for its
// samples (lane l owns blades l and l + 32), with every multiply and add
// explicitly rounded in the reference's operation order, and sums by blade
// sequentially in one lane where the reference does; each sample's values and
// cotangents are therefore those of the reference. Leaf gradients and the loss
// are summed per warp over its samples, then over warps in warp order
// (deterministic); only this order of the sum over samples differs from the
// reference's sample-by-sample accumulation.
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "crmath.h"
#include "geo_internal.h"
#include "v8_internal.h"

namespace geo {
namespace v8 {
namespace {

constexpr int kBatchThreads = 256;
constexpr int kBatchCtasPerSm = 2;  // 16 warps per SM hide the latency of the per-sample chains

struct BatchNode {
    int32_t kind, left, right, grade;
    double scalar;
    int32_t requires_grad;
    int32_t grad_slot;  // >= 0 for leaves whose gradient is accumulated
    int32_t source;     // 0: the leaf's own value; 1 / 2: row s of row source a / b
    int32_t column;     // first column of the leaf's coefficients in that row
    int32_t invariant;  // the value does not depend on the per-sample rows
    int32_t reserved;
};

struct BatchArgs {
    const BatchNode *nodes;
    const double *leaf_values;  // [count][64]: values of the leaves that do not vary per sample
    const double *rows_a;       // per-sample rows, row s at rows_a + s * stride_a
    const double *rows_b;
    size_t stride_a, stride_b;
    double *outputs;            // forward-only: [batch][blades] of output_node
    double *scratch;            // [warps][2][count][64]: values, cotangents
    double *partials;           // [warps][grad_slots + 1][64]; row grad_slots holds the loss at [0]
    int *status;                // first failure (geo_v8_status_t), 0 while none
    int *failed_node;
    size_t batch;
    int count, blades, loss_node, output_node, grad_slots, backward;
    uint64_t neg[64];  // bit r of neg[l]: e_l e_r = -e_(l^r)
};

__device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ int map_sign(int mode, int blade) {
    const unsigned g = __popc(blade);
    if (mode == 0) return ((g * (g - 1u) / 2u) & 1u) ? -1 : 1;  // reverse
    if (mode == 1) return (g & 1u) ? -1 : 1;                    // grade involution
    return ((g * (g + 1u) / 2u) & 1u) ? -1 : 1;                 // Clifford conjugate
}
__device__ __forceinline__ bool warp_any(bool v) { return __any_sync(0xffffffffu, v); }

// v * (bit `bit` of `word` set ? -1 : 1): multiplying by -1 is exact, so the
// sign bit is flipped with an integer operation instead of an FP64 multiply.
__device__ __forceinline__ double signed_by(double v, uint64_t word, int bit) {
    const int flip = (int)((word >> bit) & 1ull) << 31;
    return __hiloint2double(__double2hiint(v) ^ flip, __double2loint(v));
}

// Sequential sums over the blades in blade order (the reference's loops),
// computed identically on every lane from the node values in the warp's
// scratch: each load reads one address for the whole warp (a broadcast), two
// blades at a time, so only the chain of adds is serial.
template <int N>
__device__ __forceinline__ double blade_dot(const double *x, const double *y) {
    double acc = 0.0;
#pragma unroll 8
    for (int q = 0; q < N; q += 2) {
        const double2 u = *reinterpret_cast<const double2 *>(x + q);
        const double2 v = *reinterpret_cast<const double2 *>(y + q);
        acc = add(acc, mul(u.x, v.x));
        acc = add(acc, mul(u.y, v.y));
    }
    return acc;
}
template <int N>
__device__ __forceinline__ double half_squared_norm(const double *x) {
    double acc = 0.0;
#pragma unroll 8
    for (int q = 0; q < N; q += 2) {
        const double2 u = *reinterpret_cast<const double2 *>(x + q);
        acc = add(acc, mul(mul(0.5, u.x), u.x));
        acc = add(acc, mul(mul(0.5, u.y), u.y));
    }
    return acc;
}

__device__ void record_failure(const BatchArgs &a, int status, int node) {
    if ((threadIdx.x & 31) == 0 && atomicCAS(a.status, 0, status) == 0) *a.failed_node = node;
}

// dest[b] += src_b * scale for this lane's blades, with the reference's rule
// (src/full_cycle_v8.c:117-130): nothing is written if any result is not finite.
__device__ bool accumulate2(const BatchArgs &a, double *dest, double s0, double s1, double scale, int b0, int b1) {
    const bool l0 = b0 < a.blades, l1 = b1 < a.blades;
    const double n0 = l0 ? add(dest[b0], mul(s0, scale)) : 0.0;
    const double n1 = l1 ? add(dest[b1], mul(s1, scale)) : 0.0;
    if (warp_any((l0 && !isfinite(n0)) || (l1 && !isfinite(n1)))) return false;
    if (l0) dest[b0] = n0;
    if (l1) dest[b1] = n1;
    __syncwarp();
    return true;
}

// NB = 2^n blades, a compile-time constant so every loop over blades has a fixed trip count.
template <int NB>
__global__ void __launch_bounds__(kBatchThreads, kBatchCtasPerSm) batch_kernel(const BatchArgs a) {
    const int lane = threadIdx.x & 31;
    const size_t warp = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const size_t warps = ((size_t)gridDim.x * blockDim.x) >> 5;
    constexpr int N = NB;
    const int C = a.count;
    double *vals = a.scratch + warp * 2 * (size_t)C * 64;
    double *cots = vals + (size_t)C * 64;
    double *part = a.partials + warp * (size_t)(a.grad_slots + 1) * 64;
    for (int i = lane; i < (a.grad_slots + 1) * 64; i += 32) part[i] = 0.0;
    __syncwarp();
    const int b0 = lane, b1 = lane + 32;
    const bool l0 = b0 < N, l1 = b1 < N;
    // Per-lane sign masks of the geometric-product terms, built once: bit l of
    // gp_sign[0 / 1] is the sign of the forward term (l, l ^ b) for output b =
    // b0 / b1 (bit l ^ b of neg[l]); bit q of gp_sign[2 / 3] is the sign of the
    // right-cotangent term e_q e_b (bit b of neg[q]). With the term loops fully
    // unrolled each sign is a constant-bit extract. Layout [mask][thread]: a
    // warp's 8-byte loads are conflict-free.
    __shared__ uint64_t gp_sign[4][kBatchThreads];
    {
        uint64_t f0 = 0, f1 = 0, r0 = 0, r1 = 0;
        for (int l = 0; l < N; ++l) {
            const uint64_t w = a.neg[l];
            f0 |= ((w >> ((l ^ b0) & 63)) & 1ull) << l;
            f1 |= ((w >> ((l ^ b1) & 63)) & 1ull) << l;
            r0 |= ((w >> (b0 & 63)) & 1ull) << l;
            r1 |= ((w >> (b1 & 63)) & 1ull) << l;
        }
        gp_sign[0][threadIdx.x] = f0;
        gp_sign[1][threadIdx.x] = f1;
        gp_sign[2][threadIdx.x] = r0;
        gp_sign[3][threadIdx.x] = r1;
    }

    for (size_t s = warp; s < a.batch; s += warps) {
        if (*(volatile int *)a.status != 0) break;
        // ---------------------------------------------------------------- forward
        int fail = 0, fnode = -1;
        for (int i = 0; i < C && !fail; ++i) {
            const BatchNode nd = a.nodes[i];
            // A value that no per-sample row reaches is computed for the warp's
            // first sample and stays in its scratch for the others.
            if (nd.invariant && s != warp) continue;
            double *v = vals + (size_t)i * 64;
            const int k = nd.kind;
            if (k >= GEO_V8_NODE_INPUT && k <= GEO_V8_NODE_STATE) {
                const double *src = nd.source == 1   ? a.rows_a + s * a.stride_a + nd.column
                                    : nd.source == 2 ? a.rows_b + s * a.stride_b + nd.column
                                                     : a.leaf_values + (size_t)i * 64;
                const double x0 = l0 ? src[b0] : 0.0, x1 = l1 ? src[b1] : 0.0;
                if (warp_any(!isfinite(x0) || !isfinite(x1))) {
                    // per-sample rows go through geo_v8_set_value in the reference, which rejects them
                    fail = nd.source != 0 ? GEO_V8_INVALID_ARGUMENT : GEO_V8_NUMERIC_FAILURE;
                    fnode = i;
                    break;
                }
                v[b0] = x0;
                v[b1] = x1;
                __syncwarp();
                continue;
            }
            const double *L = nd.left >= 0 ? vals + (size_t)nd.left * 64 : nullptr;
            const double *R = nd.right >= 0 ? vals + (size_t)nd.right * 64 : nullptr;
            double o0 = 0.0, o1 = 0.0;
            switch (k) {
                case GEO_V8_NODE_ADD: o0 = add(L[b0], R[b0]); o1 = add(L[b1], R[b1]); break;
                case GEO_V8_NODE_SCALE: o0 = mul(L[b0], nd.scalar); o1 = mul(L[b1], nd.scalar); break;
                case GEO_V8_NODE_GEOMETRIC_PRODUCT: {
                    // reference src/operator_kernel.c:412-447: left-blade-major, zero left coefficients skipped;
                    // left blade l by a broadcast load, right blade l ^ b by a per-lane load (both in L1)
                    double c0 = 0.0, c1 = 0.0;
                    const uint64_t f0 = gp_sign[0][threadIdx.x], f1 = gp_sign[1][threadIdx.x];
#pragma unroll
                    for (int l = 0; l < N; ++l) {
                        const double lv = L[l];
                        if (lv == 0.0) continue;
                        if (l0) c0 = add(c0, signed_by(mul(lv, R[l ^ b0]), f0, l));
                        if (l1) c1 = add(c1, signed_by(mul(lv, R[l ^ b1]), f1, l));
                    }
                    o0 = c0;
                    o1 = c1;
                    break;
                }
                case GEO_V8_NODE_REVERSE: o0 = mul(L[b0], (double)map_sign(0, b0)); o1 = mul(L[b1], (double)map_sign(0, b1)); break;
                case GEO_V8_NODE_GRADE_INVOLUTION: o0 = mul(L[b0], (double)map_sign(1, b0)); o1 = mul(L[b1], (double)map_sign(1, b1)); break;
                case GEO_V8_NODE_CLIFFORD_CONJUGATE: o0 = mul(L[b0], (double)map_sign(2, b0)); o1 = mul(L[b1], (double)map_sign(2, b1)); break;
                case GEO_V8_NODE_GRADE_PROJECT:
                    o0 = __popc(b0) == nd.grade ? L[b0] : 0.0;
                    o1 = __popc(b1) == nd.grade ? L[b1] : 0.0;
                    break;
                case GEO_V8_NODE_HADAMARD: o0 = mul(L[b0], R[b0]); o1 = mul(L[b1], R[b1]); break;
                case GEO_V8_NODE_TANH: o0 = geo::cr::tanh(L[b0]); o1 = geo::cr::tanh(L[b1]); break;
                case GEO_V8_NODE_SIGMOID: {
                    // reference src/full_cycle_v8.c:181-190
                    const double x[2] = {L[b0], L[b1]};
                    double y[2];
                    for (int h = 0; h < 2; ++h) {
                        if (x[h] >= 0.0) y[h] = __ddiv_rn(1.0, add(1.0, geo::cr::exp(-x[h])));
                        else { const double z = geo::cr::exp(x[h]); y[h] = __ddiv_rn(z, add(1.0, z)); }
                    }
                    o0 = y[0];
                    o1 = y[1];
                    break;
                }
                case GEO_V8_NODE_EUCLIDEAN_NORMALIZE: {
                    const double n2 = blade_dot<N>(L, L);
                    const double floor_value = nd.scalar > 0.0 ? nd.scalar : 1e-12;
                    if (!isfinite(n2) || n2 <= mul(floor_value, floor_value)) { fail = GEO_V8_NUMERIC_FAILURE; fnode = i; break; }
                    const double inverse = __ddiv_rn(1.0, __dsqrt_rn(n2));
                    o0 = mul(L[b0], inverse);
                    o1 = mul(L[b1], inverse);
                    break;
                }
                case GEO_V8_NODE_SQUARED_NORM: {
                    const double sum = half_squared_norm<N>(L);
                    o0 = lane == 0 ? sum : 0.0;
                    o1 = 0.0;
                    break;
                }
                default: fail = GEO_V8_BAD_PROGRAM; fnode = i; break;
            }
            if (fail) break;
            if (!l0) o0 = 0.0;
            if (!l1) o1 = 0.0;
            if (warp_any(!isfinite(o0) || !isfinite(o1))) { fail = GEO_V8_NUMERIC_FAILURE; fnode = i; break; }
            v[b0] = o0;
            v[b1] = o1;
            __syncwarp();
        }
        if (!fail) {
            // the loss must be a finite scalar (reference loss check before backward)
            const double *lv = vals + (size_t)a.loss_node * 64;
            const bool bad = (lane == 0 && !isfinite(lv[0])) || (l0 && b0 >= 1 && lv[b0] != 0.0) ||
                             (l1 && lv[b1] != 0.0);
            if (a.backward && warp_any(bad)) { fail = GEO_V8_NON_SCALAR_LOSS; fnode = a.loss_node; }
        }
        if (fail) { record_failure(a, fail, fnode); break; }
        if (!a.backward) {
            const double *ov = vals + (size_t)a.output_node * 64;
            if (l0) a.outputs[s * N + b0] = ov[b0];
            if (l1) a.outputs[s * N + b1] = ov[b1];
            continue;
        }
        // --------------------------------------------------------------- backward
        for (int i = 0; i < C; ++i) {
            cots[(size_t)i * 64 + b0] = 0.0;
            cots[(size_t)i * 64 + b1] = 0.0;
        }
        __syncwarp();
        if (lane == 0) cots[(size_t)a.loss_node * 64] = 1.0;
        __syncwarp();
        for (int cursor = C - 1; cursor >= 0 && !fail; --cursor) {
            const BatchNode nd = a.nodes[cursor];
            const int k = nd.kind;
            if (!nd.requires_grad || (k >= GEO_V8_NODE_INPUT && k <= GEO_V8_NODE_STATE)) continue;
            const double *cot = cots + (size_t)cursor * 64;
            const BatchNode *ln = nd.left >= 0 ? &a.nodes[nd.left] : nullptr;
            const BatchNode *rn = nd.right >= 0 ? &a.nodes[nd.right] : nullptr;
            double *lc = nd.left >= 0 ? cots + (size_t)nd.left * 64 : nullptr;
            double *rc = nd.right >= 0 ? cots + (size_t)nd.right * 64 : nullptr;
            const double *lvv = nd.left >= 0 ? vals + (size_t)nd.left * 64 : nullptr;
            const double *rvv = nd.right >= 0 ? vals + (size_t)nd.right * 64 : nullptr;
            const double c0 = l0 ? cot[b0] : 0.0, c1 = l1 ? cot[b1] : 0.0;
            bool ok = true;
            switch (k) {
                case GEO_V8_NODE_ADD:
                    if (ln->requires_grad) ok = accumulate2(a, lc, c0, c1, 1.0, b0, b1);
                    if (ok && rn->requires_grad) ok = accumulate2(a, rc, c0, c1, 1.0, b0, b1);
                    break;
                case GEO_V8_NODE_SCALE:
                    if (ln->requires_grad) ok = accumulate2(a, lc, c0, c1, nd.scalar, b0, b1);
                    break;
                case GEO_V8_NODE_GEOMETRIC_PRODUCT: {
                    // reference src/operator_kernel.c:494-539; blade q of the operands by broadcast
                    // loads, cotangent blade b ^ q by a per-lane load (all in L1)
                    const uint64_t neg0 = a.neg[b0 & 63], neg1 = a.neg[b1 & 63];
                    const uint64_t r0 = gp_sign[2][threadIdx.x], r1 = gp_sign[3][threadIdx.x];
                    double la0 = 0.0, la1 = 0.0, ra0 = 0.0, ra1 = 0.0;
#pragma unroll
                    for (int q = 0; q < N; ++q) {
                        const double rq = rvv[q], lq = lvv[q];
                        if (l0) {
                            const double cq0 = cot[b0 ^ q];
                            la0 = add(la0, mul(signed_by(cq0, neg0, q), rq));
                            ra0 = add(ra0, mul(signed_by(cq0, r0, q), lq));
                        }
                        if (l1) {
                            const double cq1 = cot[b1 ^ q];
                            la1 = add(la1, mul(signed_by(cq1, neg1, q), rq));
                            ra1 = add(ra1, mul(signed_by(cq1, r1, q), lq));
                        }
                    }
                    if (ln->requires_grad) ok = accumulate2(a, lc, la0, la1, 1.0, b0, b1);
                    if (ok && rn->requires_grad) ok = accumulate2(a, rc, ra0, ra1, 1.0, b0, b1);
                    break;
                }
                case GEO_V8_NODE_REVERSE:
                case GEO_V8_NODE_GRADE_INVOLUTION:
                case GEO_V8_NODE_CLIFFORD_CONJUGATE: {
                    const int mode = k == GEO_V8_NODE_REVERSE ? 0 : (k == GEO_V8_NODE_GRADE_INVOLUTION ? 1 : 2);
                    if (ln->requires_grad)
                        ok = accumulate2(a, lc, mul(c0, (double)map_sign(mode, b0)), mul(c1, (double)map_sign(mode, b1)),
                                         1.0, b0, b1);
                    break;
                }
                case GEO_V8_NODE_GRADE_PROJECT:
                    if (ln->requires_grad)
                        ok = accumulate2(a, lc, __popc(b0) == nd.grade ? c0 : 0.0, __popc(b1) == nd.grade ? c1 : 0.0,
                                         1.0, b0, b1);
                    break;
                case GEO_V8_NODE_HADAMARD: {
                    // both partials read values, not cotangents
                    if (ln->requires_grad) {
                        const double n0 = l0 ? add(lc[b0], mul(c0, rvv[b0])) : 0.0;
                        const double n1 = l1 ? add(lc[b1], mul(c1, rvv[b1])) : 0.0;
                        if (warp_any((l0 && !isfinite(n0)) || (l1 && !isfinite(n1)))) { ok = false; break; }
                        if (l0) lc[b0] = n0;
                        if (l1) lc[b1] = n1;
                        __syncwarp();
                    }
                    if (rn->requires_grad) {
                        const double n0 = l0 ? add(rc[b0], mul(c0, lvv[b0])) : 0.0;
                        const double n1 = l1 ? add(rc[b1], mul(c1, lvv[b1])) : 0.0;
                        if (warp_any((l0 && !isfinite(n0)) || (l1 && !isfinite(n1)))) { ok = false; break; }
                        if (l0) rc[b0] = n0;
                        if (l1) rc[b1] = n1;
                        __syncwarp();
                    }
                    break;
                }
                case GEO_V8_NODE_TANH:
                case GEO_V8_NODE_SIGMOID:
                    if (ln->requires_grad) {
                        const double *ov = vals + (size_t)cursor * 64;
                        double d0 = 0.0, d1 = 0.0;
                        if (k == GEO_V8_NODE_TANH) {
                            d0 = __dsub_rn(1.0, mul(ov[b0], ov[b0]));
                            d1 = __dsub_rn(1.0, mul(ov[b1], ov[b1]));
                        } else {
                            d0 = mul(ov[b0], __dsub_rn(1.0, ov[b0]));
                            d1 = mul(ov[b1], __dsub_rn(1.0, ov[b1]));
                        }
                        const double n0 = l0 ? add(lc[b0], mul(c0, d0)) : 0.0;
                        const double n1 = l1 ? add(lc[b1], mul(c1, d1)) : 0.0;
                        if (warp_any((l0 && !isfinite(n0)) || (l1 && !isfinite(n1)))) { ok = false; break; }
                        if (l0) lc[b0] = n0;
                        if (l1) lc[b1] = n1;
                        __syncwarp();
                    }
                    break;
                case GEO_V8_NODE_EUCLIDEAN_NORMALIZE: {
                    const double *ov = vals + (size_t)cursor * 64;
                    const double n2 = blade_dot<N>(lvv, lvv);
                    const double dot = blade_dot<N>(ov, cot);
                    if (!isfinite(n2) || n2 <= 0.0 || !isfinite(dot)) { ok = false; break; }
                    if (ln->requires_grad) {
                        const double inverse = __ddiv_rn(1.0, __dsqrt_rn(n2));
                        const double n0 = l0 ? add(lc[b0], mul(inverse, __dsub_rn(c0, mul(ov[b0], dot)))) : 0.0;
                        const double n1 = l1 ? add(lc[b1], mul(inverse, __dsub_rn(c1, mul(ov[b1], dot)))) : 0.0;
                        if (warp_any((l0 && !isfinite(n0)) || (l1 && !isfinite(n1)))) { ok = false; break; }
                        if (l0) lc[b0] = n0;
                        if (l1) lc[b1] = n1;
                        __syncwarp();
                    }
                    break;
                }
                case GEO_V8_NODE_SQUARED_NORM: {
                    if (warp_any((l0 && b0 >= 1 && c0 != 0.0) || (l1 && c1 != 0.0))) {
                        fail = GEO_V8_NON_SCALAR_LOSS;
                        fnode = cursor;
                        break;
                    }
                    const double seed = __shfl_sync(0xffffffffu, c0, 0);
                    if (ln->requires_grad)
                        ok = accumulate2(a, lc, l0 ? lvv[b0] : 0.0, l1 ? lvv[b1] : 0.0, seed, b0, b1);
                    break;
                }
                default: fail = GEO_V8_BAD_PROGRAM; fnode = cursor; break;
            }
            if (!fail && !ok) { fail = GEO_V8_NUMERIC_FAILURE; fnode = cursor; }
        }
        if (fail) { record_failure(a, fail, fnode); break; }
        // Leaf gradients and the loss, summed over this warp's samples.
        for (int i = 0; i < C; ++i) {
            const BatchNode nd = a.nodes[i];
            if (nd.grad_slot < 0) continue;
            double *g = part + (size_t)nd.grad_slot * 64;
            const double *cot = cots + (size_t)i * 64;
            const double n0 = l0 ? add(g[b0], cot[b0]) : 0.0;
            const double n1 = l1 ? add(g[b1], cot[b1]) : 0.0;
            if (warp_any((l0 && !isfinite(n0)) || (l1 && !isfinite(n1)))) { fail = GEO_V8_NUMERIC_FAILURE; fnode = i; break; }
            if (l0) g[b0] = n0;
            if (l1) g[b1] = n1;
        }
        if (fail) { record_failure(a, fail, fnode); break; }
        if (lane == 0) part[(size_t)a.grad_slots * 64] = add(part[(size_t)a.grad_slots * 64], vals[(size_t)a.loss_node * 64]);
        __syncwarp();
    }
}

// out[r][b] = sum over warps (in warp order) of partials[w][r][b]; rows = grad_slots + 1.
// One warp per entry: the lanes load 32 warps' partials at a time (the next
// 32 are loaded while these are summed) and the sum runs through shuffles in
// warp order, so the result is the sequential sum.
__global__ void reduce_partials_kernel(const double *__restrict__ partials, size_t warps, int rows,
                                       double *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const size_t entry = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (entry >= (size_t)rows * 64) return;  // whole warps
    const size_t stride = (size_t)rows * 64;
    double acc = 0.0;
    double next = (size_t)lane < warps ? partials[(size_t)lane * stride + entry] : 0.0;
    for (size_t w0 = 0; w0 < warps; w0 += 32) {
        const double cur = next;
        const size_t w1 = w0 + 32 + (size_t)lane;
        next = w1 < warps ? partials[w1 * stride + entry] : 0.0;
        const int m = warps - w0 < 32 ? (int)(warps - w0) : 32;
        for (int j = 0; j < m; ++j) acc = add(acc, __shfl_sync(0xffffffffu, cur, j));
    }
    if (lane == 0) out[entry] = acc;
}

struct Workspace {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    void *buffer = nullptr;
    size_t bytes = 0;
};
Workspace g_batch_ws[64];

}  // namespace

geo_v8_status_t run_batch(geo_v8_program_t *p, const std::vector<RowLeaf> &row_leaves, const RowSource &a_rows,
                          const RowSource &b_rows, uint32_t output_node, double *device_outputs, size_t batch,
                          int backward, double *loss_sum, std::vector<double> *gradients) {
    const int count = (int)p->node_count;
    const int blades = 1 << p->dimension;
    std::vector<BatchNode> nodes((size_t)count);
    std::vector<double> leaf_values((size_t)count * 64, 0.0);
    int slots = 0;
    for (int i = 0; i < count; ++i) {
        const geo_v8_node_t &n = p->nodes[i];
        BatchNode &b = nodes[(size_t)i];
        b.kind = n.kind;
        b.left = n.left == GEO_V8_INVALID_NODE ? -1 : (int32_t)n.left;
        b.right = n.right == GEO_V8_INVALID_NODE ? -1 : (int32_t)n.right;
        b.grade = n.grade;
        b.scalar = n.scalar;
        b.requires_grad = n.requires_grad;
        b.grad_slot = -1;
        b.source = 0;
        b.column = 0;
    }
    for (const RowLeaf &r : row_leaves) {
        if (r.node >= (uint32_t)count || !leaf_kind(p->nodes[r.node].kind) || (r.source != 1 && r.source != 2))
            return GEO_V8_BAD_PROGRAM;
        nodes[r.node].source = r.source;
        nodes[r.node].column = (int32_t)r.column;
    }
    for (int i = 0; i < count; ++i) {
        const geo_v8_node_t &n = p->nodes[i];
        BatchNode &b = nodes[(size_t)i];
        if (leaf_kind(n.kind)) {
            if (b.source == 0) {
                if (!mv_valid(&n.value, p->dimension, p->signature)) return GEO_V8_NUMERIC_FAILURE;
                memcpy(&leaf_values[(size_t)i * 64], n.value.coefficients, 64 * sizeof(double));
            }
            if (backward && n.requires_grad) b.grad_slot = slots++;
        }
        b.invariant = leaf_kind(n.kind) ? (b.source == 0)
                                        : (b.left >= 0 && nodes[(size_t)b.left].invariant &&
                                           (b.right < 0 || nodes[(size_t)b.right].invariant));
        b.reserved = 0;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GEO_V8_ALLOCATION_FAILURE;
    const int sms = device_sm_count();
    size_t warps = (size_t)sms * kBatchCtasPerSm * (kBatchThreads / 32);
    const size_t needed_warps = batch;
    if (warps > needed_warps) warps = needed_warps;
    if (warps < 1) warps = 1;
    const size_t ctas = (warps + (kBatchThreads / 32) - 1) / (kBatchThreads / 32);
    warps = ctas * (kBatchThreads / 32);
    const int rows = slots + 1;
    const size_t node_bytes = (size_t)count * sizeof(BatchNode);
    const size_t leaf_bytes = (size_t)count * 64 * sizeof(double);
    const size_t scratch_bytes = warps * 2 * (size_t)count * 64 * sizeof(double);
    const size_t partial_bytes = warps * (size_t)rows * 64 * sizeof(double);
    const size_t out_bytes = (size_t)rows * 64 * sizeof(double);
    auto align = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t total = align(node_bytes) + align(leaf_bytes) + align(scratch_bytes) + align(partial_bytes) +
                         align(out_bytes) + 256;

    Workspace &ws = g_batch_ws[dev];
    std::lock_guard<std::mutex> lock(ws.mu);
    if (ws.stream == nullptr && cudaStreamCreateWithFlags(&ws.stream, cudaStreamNonBlocking) != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_V8_ALLOCATION_FAILURE;
    }
    if (ws.bytes < total) {
        if (ws.buffer) cudaFree(ws.buffer);
        ws.buffer = nullptr;
        ws.bytes = 0;
        if (cudaMalloc(&ws.buffer, total) != cudaSuccess) {
            (void)cudaGetLastError();
            return GEO_V8_ALLOCATION_FAILURE;
        }
        ws.bytes = total;
    }
    char *cur = (char *)ws.buffer;
    auto take = [&](size_t bytes) {
        char *r = cur;
        cur += align(bytes);
        return r;
    };
    BatchArgs a{};
    a.nodes = (const BatchNode *)take(node_bytes);
    a.leaf_values = (const double *)take(leaf_bytes);
    a.scratch = (double *)take(scratch_bytes);
    a.partials = (double *)take(partial_bytes);
    double *sums = (double *)take(out_bytes);
    int *flags = (int *)take(256);
    a.status = flags;
    a.failed_node = flags + 1;
    a.rows_a = a_rows.base;
    a.stride_a = a_rows.stride;
    a.rows_b = b_rows.base;
    a.stride_b = b_rows.stride;
    a.outputs = device_outputs;
    a.batch = batch;
    a.count = count;
    a.blades = blades;
    a.loss_node = (int)p->loss_node;
    a.output_node = output_node == GEO_V8_INVALID_NODE ? -1 : (int)output_node;
    a.grad_slots = slots;
    a.backward = backward;
    for (int l = 0; l < 64; ++l) {
        uint64_t neg = 0;
        for (int r = 0; r < blades; ++r)
            if (sign_rule((uint8_t)l, (uint8_t)r, p->signature, p->dimension) < 0) neg |= 1ull << r;
        a.neg[l] = l < blades ? neg : 0ull;
    }
    cudaError_t e = cudaMemcpyAsync((void *)a.nodes, nodes.data(), node_bytes, cudaMemcpyHostToDevice, ws.stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync((void *)a.leaf_values, leaf_values.data(), leaf_bytes, cudaMemcpyHostToDevice, ws.stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(flags, 0, 256, ws.stream);
    if (e == cudaSuccess) {
        switch (blades) {
            case 2: batch_kernel<2><<<(unsigned)ctas, kBatchThreads, 0, ws.stream>>>(a); break;
            case 4: batch_kernel<4><<<(unsigned)ctas, kBatchThreads, 0, ws.stream>>>(a); break;
            case 8: batch_kernel<8><<<(unsigned)ctas, kBatchThreads, 0, ws.stream>>>(a); break;
            case 16: batch_kernel<16><<<(unsigned)ctas, kBatchThreads, 0, ws.stream>>>(a); break;
            case 32: batch_kernel<32><<<(unsigned)ctas, kBatchThreads, 0, ws.stream>>>(a); break;
            default: batch_kernel<64><<<(unsigned)ctas, kBatchThreads, 0, ws.stream>>>(a); break;
        }
        e = cudaGetLastError();
    }
    std::vector<double> host_sums((size_t)rows * 64, 0.0);
    int host_flags[2] = {0, -1};
    if (e == cudaSuccess && backward) {
        reduce_partials_kernel<<<(unsigned)((rows * 64 * 32 + 255) / 256), 256, 0, ws.stream>>>(a.partials, warps, rows,
                                                                                         sums);
        e = cudaGetLastError();
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(host_sums.data(), sums, out_bytes, cudaMemcpyDeviceToHost, ws.stream);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(host_flags, flags, sizeof(host_flags), cudaMemcpyDeviceToHost, ws.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ws.stream);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_V8_ALLOCATION_FAILURE;
    }
    if (host_flags[0] != 0) return (geo_v8_status_t)host_flags[0];
    if (backward) {
        if (loss_sum) *loss_sum = host_sums[(size_t)slots * 64];
        if (gradients) {
            gradients->assign((size_t)count * 64, 0.0);
            for (int i = 0; i < count; ++i)
                if (nodes[(size_t)i].grad_slot >= 0)
                    memcpy(&(*gradients)[(size_t)i * 64], &host_sums[(size_t)nodes[(size_t)i].grad_slot * 64],
                           (size_t)blades * sizeof(double));
        }
    }
    return GEO_V8_OK;
}

}  // namespace v8
}  // namespace geo
