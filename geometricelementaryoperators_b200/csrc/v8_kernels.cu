// v8_kernels.cu -- device interpreter for V8 programs (geo/full_cycle_v8.h).
//
// One CTA of 64 threads walks the program's nodes in order; thread b owns
// blade b of every multivector. Node storage is the program's mapped
// page-locked allocation, read and written in place. Arithmetic mirrors the
// reference operation for operation (src/full_cycle_v8.c:569-692 forward,
// :717-940 backward, :942-1041 optimizer, :192-281 constraints), with
// explicitly rounded multiplies and adds so that no FMA contraction changes
// a result; sums the reference runs sequentially over blades are run
// sequentially by one thread. The GP sign comes from the baked sign table of
// the program's signature (reference src/operator_kernel.c:111-135).
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

#include "crmath.h"
#include "geo_internal.h"
#include "v8_internal.h"

namespace geo {
namespace v8 {
namespace {

constexpr int kThreads = 64;

struct Ctx {
    geo_v8_node_t *nodes;
    Control *control;
    Candidate *cand;
    uint32_t count;
    uint32_t loss_node;
    int32_t n;
    int32_t blades;
    int8_t signature[8];
    uint64_t neg[64];  // bit r of neg[l]: e_l e_r = -e_(l^r)
};

// Node kinds 1..5 (INPUT, TARGET, PARAMETER, CONSTANT, STATE) are leaves.
__device__ __forceinline__ bool leaf_kind_device(int k) { return k >= GEO_V8_NODE_INPUT && k <= GEO_V8_NODE_STATE; }

__device__ __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double gsign(const Ctx &c, int l, int r) { return ((c.neg[l] >> r) & 1ull) ? -1.0 : 1.0; }

__device__ __forceinline__ int map_sign(int mode, int blade) {
    const unsigned g = __popc(blade);
    if (mode == 0) return ((g * (g - 1u) / 2u) & 1u) ? -1 : 1;  // reverse
    if (mode == 1) return (g & 1u) ? -1 : 1;                    // grade involution
    return ((g * (g + 1u) / 2u) & 1u) ? -1 : 1;                 // Clifford conjugate
}

// mv layout helpers: every written multivector carries the program's dimension/signature.
__device__ __forceinline__ void set_header(const Ctx &c, geo_operator_mv_f64_t *mv) {
    if (threadIdx.x == 0) {
        mv->dimension = (uint8_t)c.n;
        for (int a = 0; a < 6; ++a) mv->signature[a] = a < c.n ? c.signature[a] : 0;
    }
}

__device__ bool header_ok(const Ctx &c, const geo_operator_mv_f64_t *mv) {
    if (mv->dimension != c.n) return false;
    for (int a = 0; a < c.n; ++a)
        if (mv->signature[a] != c.signature[a]) return false;
    return true;
}

// Block-uniform: true when any thread's flag is set.
__device__ __forceinline__ bool any(bool flag) { return __syncthreads_or(flag) != 0; }

__device__ void fail(const Ctx &c, int status, int node) {
    if (threadIdx.x == 0) {
        c.control->status = status;
        c.control->failed_node = node;
    }
}

// GP of two multivectors, output blade o (reference src/operator_kernel.c:412-447:
// left-blade-major, zero left coefficients skipped).
__device__ double gp_out(const Ctx &c, const double *L, const double *R, int o) {
    double acc = 0.0;
    for (int l = 0; l < c.blades; ++l) {
        const double lv = L[l];
        if (lv == 0.0) continue;
        acc = add(acc, mul(mul(lv, R[l ^ o]), gsign(c, l, l ^ o)));
    }
    return acc;
}

__global__ void __launch_bounds__(kThreads) forward_kernel(const Ctx c) {
    __shared__ double serial;
    const int b = threadIdx.x;
    const bool lane = b < c.blades;
    if (b == 0) {
        c.control->status = GEO_V8_OK;
        c.control->failed_node = -1;
    }
    for (uint32_t i = 0; i < c.count; ++i) {
        geo_v8_node_t *node = &c.nodes[i];
        const int kind = node->kind;
        if (leaf_kind_device(kind)) {
            const bool bad = !header_ok(c, &node->value) || (lane && !isfinite(node->value.coefficients[b]));
            if (any(bad)) { fail(c, GEO_V8_NUMERIC_FAILURE, (int)i); return; }
            continue;
        }
        const double *L = node->left != GEO_V8_INVALID_NODE ? c.nodes[node->left].value.coefficients : nullptr;
        const double *R = node->right != GEO_V8_INVALID_NODE ? c.nodes[node->right].value.coefficients : nullptr;
        double out = 0.0;
        bool bad = false;
        switch (kind) {
            case GEO_V8_NODE_ADD: if (lane) out = add(L[b], R[b]); break;
            case GEO_V8_NODE_SCALE: if (lane) out = mul(L[b], node->scalar); break;
            case GEO_V8_NODE_GEOMETRIC_PRODUCT: if (lane) out = gp_out(c, L, R, b); break;
            case GEO_V8_NODE_REVERSE: if (lane) out = mul(L[b], (double)map_sign(0, b)); break;
            case GEO_V8_NODE_GRADE_INVOLUTION: if (lane) out = mul(L[b], (double)map_sign(1, b)); break;
            case GEO_V8_NODE_CLIFFORD_CONJUGATE: if (lane) out = mul(L[b], (double)map_sign(2, b)); break;
            case GEO_V8_NODE_GRADE_PROJECT: if (lane) out = (__popc(b) == (int)node->grade) ? L[b] : 0.0; break;
            case GEO_V8_NODE_HADAMARD: if (lane) out = mul(L[b], R[b]); break;
            case GEO_V8_NODE_TANH: if (lane) out = geo::cr::tanh(L[b]); break;
            case GEO_V8_NODE_SIGMOID:
                if (lane) {
                    // reference src/full_cycle_v8.c:181-190
                    const double v = L[b];
                    if (v >= 0.0) out = __ddiv_rn(1.0, add(1.0, geo::cr::exp(-v)));
                    else { const double z = geo::cr::exp(v); out = __ddiv_rn(z, add(1.0, z)); }
                }
                break;
            case GEO_V8_NODE_EUCLIDEAN_NORMALIZE: {
                if (b == 0) {
                    double n2 = 0.0;
                    for (int k = 0; k < c.blades; ++k) n2 = add(n2, mul(L[k], L[k]));
                    serial = n2;
                }
                __syncthreads();
                const double floor_value = node->scalar > 0.0 ? node->scalar : 1e-12;
                const double n2 = serial;
                if (!isfinite(n2) || n2 <= mul(floor_value, floor_value)) { fail(c, GEO_V8_NUMERIC_FAILURE, (int)i); return; }
                const double inverse = __ddiv_rn(1.0, __dsqrt_rn(n2));
                if (lane) out = mul(L[b], inverse);
                break;
            }
            case GEO_V8_NODE_SQUARED_NORM: {
                if (b == 0) {
                    double s = 0.0;
                    for (int k = 0; k < c.blades; ++k) s = add(s, mul(mul(0.5, L[k]), L[k]));
                    serial = s;
                }
                __syncthreads();
                out = b == 0 ? serial : 0.0;
                break;
            }
            default: fail(c, GEO_V8_BAD_PROGRAM, (int)i); return;
        }
        bad = lane && !isfinite(out);
        if (any(bad)) { fail(c, GEO_V8_NUMERIC_FAILURE, (int)i); return; }
        set_header(c, &node->value);
        node->value.coefficients[b] = lane ? out : 0.0;
        __syncthreads();
    }
}

// dest += src * scale with the reference's finiteness rule (src/full_cycle_v8.c:117-130).
__device__ bool accumulate(const Ctx &c, double *dest, const double *src, double scale) {
    const int b = threadIdx.x;
    double next = 0.0;
    const bool lane = b < c.blades;
    if (lane) next = add(dest[b], mul(src[b], scale));
    const bool bad = any(lane && !isfinite(next));
    if (!bad && lane) dest[b] = next;
    __syncthreads();
    return !bad;
}

__global__ void __launch_bounds__(kThreads) backward_kernel(const Ctx c, int accumulate_gradients) {
    __shared__ double tmp_a[64];
    __shared__ double tmp_b[64];
    __shared__ double serial[2];
    const int b = threadIdx.x;
    const bool lane = b < c.blades;
    if (b == 0) {
        c.control->status = GEO_V8_OK;
        c.control->failed_node = -1;
    }
    for (uint32_t i = 0; i < c.count; ++i) {
        geo_v8_node_t *node = &c.nodes[i];
        if (!accumulate_gradients) {
            set_header(c, &node->gradient);
            node->gradient.coefficients[b] = 0.0;
        }
        set_header(c, &node->cotangent);
        node->cotangent.coefficients[b] = 0.0;
    }
    __syncthreads();
    if (b == 0) c.nodes[c.loss_node].cotangent.coefficients[0] = 1.0;
    __syncthreads();
    for (uint32_t cursor = c.count; cursor > 0;) {
        --cursor;
        geo_v8_node_t *node = &c.nodes[cursor];
        if (!node->requires_grad) continue;
        const int kind = node->kind;
        if (leaf_kind_device(kind)) continue;
        geo_v8_node_t *left = node->left != GEO_V8_INVALID_NODE ? &c.nodes[node->left] : nullptr;
        geo_v8_node_t *right = node->right != GEO_V8_INVALID_NODE ? &c.nodes[node->right] : nullptr;
        const double *cot = node->cotangent.coefficients;
        bool ok = true;
        switch (kind) {
            case GEO_V8_NODE_ADD:
                if (left->requires_grad) ok = accumulate(c, left->cotangent.coefficients, cot, 1.0);
                if (ok && right->requires_grad) ok = accumulate(c, right->cotangent.coefficients, cot, 1.0);
                break;
            case GEO_V8_NODE_SCALE:
                if (left->requires_grad) ok = accumulate(c, left->cotangent.coefficients, cot, node->scalar);
                break;
            case GEO_V8_NODE_GEOMETRIC_PRODUCT: {
                // reference src/operator_kernel.c:494-539: c = cot[l^r] s(l,r);
                // left_bar[l] += c R[r] (r ascending); right_bar[r] += c L[l] (l ascending)
                const double *L = left->value.coefficients;
                const double *R = right->value.coefficients;
                if (lane) {
                    double la = 0.0, ra = 0.0;
                    for (int k = 0; k < c.blades; ++k) {
                        la = add(la, mul(mul(cot[b ^ k], gsign(c, b, k)), R[k]));
                        ra = add(ra, mul(mul(cot[k ^ b], gsign(c, k, b)), L[k]));
                    }
                    tmp_a[b] = la;
                    tmp_b[b] = ra;
                }
                __syncthreads();
                if (left->requires_grad) ok = accumulate(c, left->cotangent.coefficients, tmp_a, 1.0);
                if (ok && right->requires_grad) ok = accumulate(c, right->cotangent.coefficients, tmp_b, 1.0);
                break;
            }
            case GEO_V8_NODE_REVERSE:
            case GEO_V8_NODE_GRADE_INVOLUTION:
            case GEO_V8_NODE_CLIFFORD_CONJUGATE: {
                const int mode = kind == GEO_V8_NODE_REVERSE ? 0 : (kind == GEO_V8_NODE_GRADE_INVOLUTION ? 1 : 2);
                if (lane) tmp_a[b] = mul(cot[b], (double)map_sign(mode, b));
                __syncthreads();
                if (left->requires_grad) ok = accumulate(c, left->cotangent.coefficients, tmp_a, 1.0);
                break;
            }
            case GEO_V8_NODE_GRADE_PROJECT:
                if (lane) tmp_a[b] = (__popc(b) == (int)node->grade) ? cot[b] : 0.0;
                __syncthreads();
                if (left->requires_grad) ok = accumulate(c, left->cotangent.coefficients, tmp_a, 1.0);
                break;
            case GEO_V8_NODE_HADAMARD: {
                // Both partials read the values, not the cotangents: order of updates is immaterial.
                if (left->requires_grad) {
                    const double next = lane ? add(left->cotangent.coefficients[b], mul(cot[b], right->value.coefficients[b])) : 0.0;
                    if (any(lane && !isfinite(next))) { ok = false; break; }
                    if (lane) left->cotangent.coefficients[b] = next;
                    __syncthreads();
                }
                if (right->requires_grad) {
                    const double next = lane ? add(right->cotangent.coefficients[b], mul(cot[b], left->value.coefficients[b])) : 0.0;
                    if (any(lane && !isfinite(next))) { ok = false; break; }
                    if (lane) right->cotangent.coefficients[b] = next;
                    __syncthreads();
                }
                break;
            }
            case GEO_V8_NODE_TANH:
            case GEO_V8_NODE_SIGMOID:
                if (left->requires_grad) {
                    double next = 0.0;
                    if (lane) {
                        const double o = node->value.coefficients[b];
                        const double d = kind == GEO_V8_NODE_TANH ? __dsub_rn(1.0, mul(o, o)) : mul(o, __dsub_rn(1.0, o));
                        next = add(left->cotangent.coefficients[b], mul(cot[b], d));
                    }
                    if (any(lane && !isfinite(next))) { ok = false; break; }
                    if (lane) left->cotangent.coefficients[b] = next;
                    __syncthreads();
                }
                break;
            case GEO_V8_NODE_EUCLIDEAN_NORMALIZE: {
                const double *in = left->value.coefficients;
                if (b == 0) {
                    double n2 = 0.0, dot = 0.0;
                    for (int k = 0; k < c.blades; ++k) {
                        n2 = add(n2, mul(in[k], in[k]));
                        dot = add(dot, mul(node->value.coefficients[k], cot[k]));
                    }
                    serial[0] = n2;
                    serial[1] = dot;
                }
                __syncthreads();
                const double n2 = serial[0], dot = serial[1];
                if (!isfinite(n2) || n2 <= 0.0 || !isfinite(dot)) { ok = false; break; }
                if (left->requires_grad) {
                    const double inverse = __ddiv_rn(1.0, __dsqrt_rn(n2));
                    double next = 0.0;
                    if (lane) {
                        const double contribution =
                            mul(inverse, __dsub_rn(cot[b], mul(node->value.coefficients[b], dot)));
                        next = add(left->cotangent.coefficients[b], contribution);
                    }
                    if (any(lane && !isfinite(next))) { ok = false; break; }
                    if (lane) left->cotangent.coefficients[b] = next;
                    __syncthreads();
                }
                break;
            }
            case GEO_V8_NODE_SQUARED_NORM: {
                const bool nonscalar = lane && b >= 1 && cot[b] != 0.0;
                if (any(nonscalar)) { fail(c, GEO_V8_NON_SCALAR_LOSS, (int)cursor); return; }
                if (left->requires_grad)
                    ok = accumulate(c, left->cotangent.coefficients, left->value.coefficients, cot[0]);
                break;
            }
            default: fail(c, GEO_V8_BAD_PROGRAM, (int)cursor); return;
        }
        if (!ok) { fail(c, GEO_V8_NUMERIC_FAILURE, (int)cursor); return; }
    }
    for (uint32_t i = 0; i < c.count; ++i) {
        geo_v8_node_t *node = &c.nodes[i];
        if (leaf_kind_device(node->kind) && node->requires_grad) {
            if (!accumulate(c, node->gradient.coefficients, node->cotangent.coefficients, 1.0)) {
                fail(c, GEO_V8_NUMERIC_FAILURE, (int)i);
                return;
            }
        }
    }
}

// Constraint projection of a candidate value (reference src/full_cycle_v8.c:192-281).
// Returns GEO_V8_OK or GEO_V8_CONSTRAINT_FAILURE; block-uniform.
__device__ int project(const Ctx &c, int constraint, double *v /* smem[64] */, double *scratch /* smem[64] */,
                       double *serial) {
    const int b = threadIdx.x;
    const bool lane = b < c.blades;
    const double tiny = 1e-14;
    if (constraint == GEO_V8_CONSTRAINT_NONE) return GEO_V8_OK;
    if (constraint == GEO_V8_CONSTRAINT_UNIT_EUCLIDEAN) {
        if (b == 0) {
            double n2 = 0.0;
            for (int k = 0; k < c.blades; ++k) n2 = add(n2, mul(v[k], v[k]));
            serial[0] = n2;
        }
        __syncthreads();
        const double n2 = serial[0];
        if (!isfinite(n2) || n2 <= tiny) return GEO_V8_CONSTRAINT_FAILURE;
        const double inverse = __ddiv_rn(1.0, __dsqrt_rn(n2));
        if (lane) v[b] = mul(v[b], inverse);
        __syncthreads();
        return GEO_V8_OK;
    }
    if (constraint == GEO_V8_CONSTRAINT_UNIT_VECTOR_METRIC) {
        if (lane && __popc(b) != 1) v[b] = 0.0;
        __syncthreads();
        if (b == 0) {
            double m = 0.0;
            for (int a = 0; a < c.n; ++a) {
                const double x = v[1 << a];
                m = add(m, mul(mul((double)c.signature[a], x), x));
            }
            serial[0] = m;
        }
        __syncthreads();
        const double m = serial[0];
        if (!isfinite(m) || fabs(m) <= tiny) return GEO_V8_CONSTRAINT_FAILURE;
        const double inverse = __ddiv_rn(1.0, __dsqrt_rn(fabs(m)));
        if (lane && __popc(b) == 1) v[b] = mul(v[b], inverse);
        __syncthreads();
        return GEO_V8_OK;
    }
    if (constraint == GEO_V8_CONSTRAINT_EVEN_VERSOR) {
        if (lane && (__popc(b) & 1)) v[b] = 0.0;
        __syncthreads();
        if (lane) scratch[b] = mul(v[b], (double)map_sign(0, b));  // reverse
        __syncthreads();
        // product = v * reverse(v); only its scalar part and squared residual are needed
        double p = lane ? gp_out(c, v, scratch, b) : 0.0;
        __syncthreads();
        if (lane) scratch[b] = p;
        __syncthreads();
        if (b == 0) {
            double r2 = 0.0;
            for (int k = 1; k < c.blades; ++k) r2 = add(r2, mul(scratch[k], scratch[k]));
            serial[0] = scratch[0];
            serial[1] = r2;
        }
        __syncthreads();
        const double ns = serial[0], r2 = serial[1];
        if (!isfinite(ns) || !isfinite(r2) || fabs(ns) <= tiny || r2 > mul(1e-12, add(1.0, mul(ns, ns))))
            return GEO_V8_CONSTRAINT_FAILURE;
        const double inverse = __ddiv_rn(1.0, __dsqrt_rn(fabs(ns)));
        if (lane) v[b] = mul(v[b], inverse);
        __syncthreads();
        return GEO_V8_OK;
    }
    return GEO_V8_CONSTRAINT_FAILURE;
}

struct OptArgs {
    int32_t optimizer;
    double lr, beta1, beta2, epsilon, scale, bias1, bias2;
};

__global__ void __launch_bounds__(kThreads) optimizer_kernel(const Ctx c, const OptArgs o) {
    __shared__ double v[64];
    __shared__ double scratch[64];
    __shared__ double serial[2];
    const int b = threadIdx.x;
    const bool lane = b < c.blades;
    if (b == 0) {
        c.control->status = GEO_V8_OK;
        c.control->failed_node = -1;
    }
    __syncthreads();
    // Candidates (reference src/full_cycle_v8.c:986-1019), nothing is committed until all pass.
    for (uint32_t i = 0; i < c.count; ++i) {
        geo_v8_node_t *node = &c.nodes[i];
        if (node->kind != GEO_V8_NODE_PARAMETER) continue;
        double m = lane ? node->first_moment[b] : 0.0;
        double s = lane ? node->second_moment[b] : 0.0;
        double w = lane ? node->value.coefficients[b] : 0.0;
        bool bad = false;
        if (lane) {
            const double g = mul(node->gradient.coefficients[b], o.scale);
            double update = g;
            if (o.optimizer == GEO_V8_OPTIMIZER_ADAM) {
                const double first = add(mul(o.beta1, m), mul(__dsub_rn(1.0, o.beta1), g));
                const double second = add(mul(o.beta2, s), mul(mul(__dsub_rn(1.0, o.beta2), g), g));
                bad = !isfinite(first) || !isfinite(second);
                m = first;
                s = second;
                update = __ddiv_rn(__ddiv_rn(first, o.bias1), add(__dsqrt_rn(__ddiv_rn(second, o.bias2)), o.epsilon));
            }
            w = __dsub_rn(w, mul(o.lr, update));
            bad = bad || !isfinite(w);
        }
        if (any(bad)) { fail(c, GEO_V8_NUMERIC_FAILURE, (int)i); return; }
        if (lane) v[b] = w;
        __syncthreads();
        if (project(c, node->constraint, v, scratch, serial) != GEO_V8_OK) {
            fail(c, GEO_V8_CONSTRAINT_FAILURE, (int)i);
            return;
        }
        Candidate *cd = &c.cand[i];
        cd->value[b] = lane ? v[b] : node->value.coefficients[b];
        cd->first[b] = lane ? m : node->first_moment[b];
        cd->second[b] = lane ? s : node->second_moment[b];
        __syncthreads();
    }
    // Commit.
    for (uint32_t i = 0; i < c.count; ++i) {
        geo_v8_node_t *node = &c.nodes[i];
        if (node->kind != GEO_V8_NODE_PARAMETER) continue;
        const Candidate *cd = &c.cand[i];
        node->value.coefficients[b] = cd->value[b];
        node->first_moment[b] = cd->first[b];
        node->second_moment[b] = cd->second[b];
    }
}

std::mutex g_stream_mutex;
cudaStream_t g_streams[64] = {};

cudaStream_t stream_for_current_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_stream_mutex);
    if (g_streams[dev] == nullptr) cudaStreamCreateWithFlags(&g_streams[dev], cudaStreamNonBlocking);
    return g_streams[dev];
}

bool make_ctx(geo_v8_program_t *p, Ctx *c) {
    geo_v8_node_t *dev_nodes = nullptr;
    if (cudaHostGetDevicePointer((void **)&dev_nodes, p->nodes, 0) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    c->nodes = dev_nodes;
    c->cand = candidates(dev_nodes, p->node_capacity);
    c->control = control(dev_nodes, p->node_capacity);
    c->count = p->node_count;
    c->loss_node = p->loss_node;
    c->n = p->dimension;
    c->blades = 1 << p->dimension;
    for (int a = 0; a < 8; ++a) c->signature[a] = a < p->dimension ? p->signature[a] : 0;
    SignPlan sp;
    if (!make_sign_plan(&sp, p->dimension, p->signature, 0)) return false;
    for (int l = 0; l < 64; ++l) c->neg[l] = sp.neg[l];
    return true;
}

geo_v8_status_t finish(geo_v8_program_t *p, cudaStream_t s) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return GEO_V8_BAD_PROGRAM;
    if (cudaStreamSynchronize(s) != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_V8_BAD_PROGRAM;
    }
    return (geo_v8_status_t)control(p->nodes, p->node_capacity)->status;
}

}  // namespace

geo_v8_status_t run_forward(geo_v8_program_t *p) {
    Ctx c;
    if (!make_ctx(p, &c)) return GEO_V8_ALLOCATION_FAILURE;
    cudaStream_t s = stream_for_current_device();
    forward_kernel<<<1, kThreads, 0, s>>>(c);
    return finish(p, s);
}

geo_v8_status_t run_backward(geo_v8_program_t *p, int accumulate_gradients) {
    Ctx c;
    if (!make_ctx(p, &c)) return GEO_V8_ALLOCATION_FAILURE;
    cudaStream_t s = stream_for_current_device();
    backward_kernel<<<1, kThreads, 0, s>>>(c, accumulate_gradients);
    return finish(p, s);
}

geo_v8_status_t run_optimizer(geo_v8_program_t *p, int optimizer, double lr, double beta1, double beta2,
                              double epsilon, double scale, double bias1, double bias2) {
    Ctx c;
    if (!make_ctx(p, &c)) return GEO_V8_ALLOCATION_FAILURE;
    OptArgs o{optimizer, lr, beta1, beta2, epsilon, scale, bias1, bias2};
    cudaStream_t s = stream_for_current_device();
    optimizer_kernel<<<1, kThreads, 0, s>>>(c, o);
    return finish(p, s);
}

}  // namespace v8
}  // namespace geo
