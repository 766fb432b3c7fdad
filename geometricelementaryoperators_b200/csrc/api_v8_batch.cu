// api_v8_batch.cu -- batched training of a pattern-matched V8 program
// (geo_b200_v8_batch_train_step, declared in geo/geo_b200.h).
//
// The per-sample loop of the reference (benchmarks/bench_v8_full_cycle.c:207-219,
// tools/geo_cycle_io.c:194-323) over the graph x*w -> add(., scale(t, -1)) ->
// squared_norm is replaced by one fused streaming pass (kernels_direct.cu or
// kernels_rep.cu) that sums the parameter gradient and the loss over the
// minibatch, and the V8 optimizer update (reference src/full_cycle_v8.c:942-1041)
// applied by the finalize kernel directly on the program's mapped node memory.
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "geo/full_cycle_v8.h"
#include "geo/geo_b200.h"
#include "geo_runtime.h"
#include "representation.h"
#include "v8_internal.h"

namespace {

struct Match {
    geo_v8_node_id_t param, gp, loss;
    int parameter_on_left;
};

bool is_kind(const geo_v8_program_t *p, geo_v8_node_id_t id, int kind) {
    return id < p->node_count && p->nodes[id].kind == kind;
}

// Recognise gp = GP(input, w) | GP(w, input); neg = SCALE(target, -1);
// residual = ADD(gp, neg) | ADD(neg, gp); loss = SQUARED_NORM(residual).
bool match(const geo_v8_program_t *p, geo_v8_node_id_t input, geo_v8_node_id_t target, Match *m) {
    if (!is_kind(p, input, GEO_V8_NODE_INPUT) || !is_kind(p, target, GEO_V8_NODE_TARGET)) return false;
    const geo_v8_node_id_t loss = p->loss_node;
    if (!is_kind(p, loss, GEO_V8_NODE_SQUARED_NORM)) return false;
    const geo_v8_node_id_t res = p->nodes[loss].left;
    if (!is_kind(p, res, GEO_V8_NODE_ADD)) return false;
    geo_v8_node_id_t a = p->nodes[res].left, b = p->nodes[res].right;
    if (is_kind(p, a, GEO_V8_NODE_SCALE)) {
        const geo_v8_node_id_t t = a;
        a = b;
        b = t;
    }
    if (!is_kind(p, a, GEO_V8_NODE_GEOMETRIC_PRODUCT) || !is_kind(p, b, GEO_V8_NODE_SCALE)) return false;
    if (p->nodes[b].left != target || p->nodes[b].scalar != -1.0) return false;
    const geo_v8_node_id_t l = p->nodes[a].left, r = p->nodes[a].right;
    geo_v8_node_id_t param;
    int on_left;
    if (l == input && is_kind(p, r, GEO_V8_NODE_PARAMETER)) {
        param = r;
        on_left = 0;
    } else if (r == input && is_kind(p, l, GEO_V8_NODE_PARAMETER)) {
        param = l;
        on_left = 1;
    } else {
        return false;
    }
    if (p->nodes[param].constraint != GEO_V8_CONSTRAINT_NONE) return false;
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i)
        if (p->nodes[i].kind == GEO_V8_NODE_PARAMETER && i != param) return false;
    m->param = param;
    m->gp = a;
    m->loss = loss;
    m->parameter_on_left = on_left;
    return true;
}

struct Workspace {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    double *records = nullptr;
    double *scratch = nullptr;  // [0] loss sum, [8, 72) device copy of W
    uint32_t *status = nullptr;
};
Workspace g_ws[64];

// Any other graph: per-sample forward/backward on the GPU (v8_batch.cu), the
// summed leaf gradients written into the program, then the program's own
// optimizer step (constraints and transactionality included).
int general_step(geo_v8_program_t *p, uint32_t input_node, uint32_t target_node, const double *device_inputs,
                 const double *device_targets, size_t batch, int optimizer, double learning_rate, double beta1,
                 double beta2, double epsilon, double gradient_scale, double *loss_sum) {
    if (!is_kind(p, input_node, GEO_V8_NODE_INPUT)) return GEO_V8_BAD_PROGRAM;
    if (target_node != GEO_V8_INVALID_NODE && !is_kind(p, target_node, GEO_V8_NODE_TARGET)) return GEO_V8_BAD_PROGRAM;
    (void)geo_v8_zero_grad(p);
    double loss = 0.0;
    std::vector<double> grads;
    const size_t blades = (size_t)1 << p->dimension;
    std::vector<geo::v8::RowLeaf> leaves{{input_node, 1, 0}};
    if (target_node != GEO_V8_INVALID_NODE) leaves.push_back({target_node, 2, 0});
    const geo_v8_status_t st =
        geo::v8::run_batch(p, leaves, {device_inputs, blades}, {device_targets, blades}, GEO_V8_INVALID_NODE,
                           nullptr, batch, 1, &loss, &grads);
    if (st != GEO_V8_OK) return st;
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i)
        if (geo::v8::leaf_kind(p->nodes[i].kind) && p->nodes[i].requires_grad)
            memcpy(p->nodes[i].gradient.coefficients, &grads[(size_t)i * 64], blades * sizeof(double));
    p->gradient_samples = batch > 0xffffffffull ? 0xffffffffu : (uint32_t)batch;
    p->forward_valid = 1u;
    p->backward_valid = 1u;
    if (loss_sum) *loss_sum = loss;
    return geo_v8_optimizer_step(p, (geo_v8_optimizer_t)optimizer, learning_rate, beta1, beta2, epsilon,
                                 gradient_scale);
}

}  // namespace

extern "C" int geo_b200_v8_batch_forward(void *program_ptr, uint32_t input_node, const double *device_inputs,
                                         size_t batch, uint32_t output_node, double *device_outputs) {
    geo_v8_program_t *p = (geo_v8_program_t *)program_ptr;
    if (!geo::v8::program_valid(p)) return GEO_V8_BAD_PROGRAM;
    if (!p->compiled) return GEO_V8_NOT_COMPILED;
    if (device_inputs == nullptr || device_outputs == nullptr || batch == 0) return GEO_V8_INVALID_ARGUMENT;
    if (!is_kind(p, input_node, GEO_V8_NODE_INPUT) || output_node >= p->node_count) return GEO_V8_BAD_PROGRAM;
    const size_t blades = (size_t)1 << p->dimension;
    return geo::v8::run_batch(p, {{input_node, 1, 0}}, {device_inputs, blades}, {nullptr, 0}, output_node,
                              device_outputs, batch, 0, nullptr, nullptr);
}

extern "C" int geo_b200_v8_batch_train_step(void *program_ptr, uint32_t input_node, uint32_t target_node,
                                            const double *device_inputs, const double *device_targets,
                                            size_t batch, int optimizer, double learning_rate, double beta1,
                                            double beta2, double epsilon, double gradient_scale, double *loss_sum) {
    geo_v8_program_t *p = (geo_v8_program_t *)program_ptr;
    if (!geo::v8::program_valid(p)) return GEO_V8_BAD_PROGRAM;
    if (!p->compiled) return GEO_V8_NOT_COMPILED;
    if (device_inputs == nullptr || batch == 0 || (device_targets == nullptr && target_node != GEO_V8_INVALID_NODE))
        return GEO_V8_INVALID_ARGUMENT;
    if ((optimizer != GEO_V8_OPTIMIZER_SGD && optimizer != GEO_V8_OPTIMIZER_ADAM) || !isfinite(learning_rate) ||
        learning_rate <= 0.0 || !isfinite(gradient_scale) || gradient_scale <= 0.0 || !isfinite(beta1) ||
        beta1 < 0.0 || beta1 >= 1.0 || !isfinite(beta2) || beta2 < 0.0 || beta2 >= 1.0 || !isfinite(epsilon) ||
        epsilon <= 0.0)
        return GEO_V8_INVALID_ARGUMENT;
    Match m;
    if (!match(p, input_node, target_node, &m))
        return general_step(p, input_node, target_node, device_inputs, device_targets, batch, optimizer,
                            learning_rate, beta1, beta2, epsilon, gradient_scale, loss_sum);
    geo_v8_node_t *param = &p->nodes[m.param];
    if (!geo::v8::mv_valid(&param->value, p->dimension, p->signature)) return GEO_V8_NUMERIC_FAILURE;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GEO_V8_BAD_PROGRAM;
    Workspace &ws = g_ws[dev];
    std::lock_guard<std::mutex> lock(ws.mu);
    if (ws.stream == nullptr) {
        if (cudaStreamCreateWithFlags(&ws.stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaMalloc((void **)&ws.records, (size_t)geo::kMaxCtas * geo::kRecStride * sizeof(double)) !=
                cudaSuccess ||
            cudaMalloc((void **)&ws.scratch, 128 * sizeof(double)) != cudaSuccess ||
            cudaMalloc((void **)&ws.status, 64) != cudaSuccess) {
            (void)cudaGetLastError();
            return GEO_V8_ALLOCATION_FAILURE;
        }
    }
    // Device views of the parameter's value and moments in the mapped node memory.
    geo_v8_node_t *dev_nodes = nullptr;
    if (cudaHostGetDevicePointer((void **)&dev_nodes, p->nodes, 0) != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_V8_ALLOCATION_FAILURE;
    }
    geo_v8_node_t *dparam = dev_nodes + m.param;

    const uint64_t step = p->optimizer_step + 1u;
    geo::OptimizerArgs opt{};
    opt.kind = optimizer == GEO_V8_OPTIMIZER_ADAM ? geo::kOptAdamV8 : geo::kOptSgdV8;
    opt.blades = 1 << p->dimension;
    opt.learning_rate = learning_rate;
    opt.beta1 = beta1;
    opt.beta2 = beta2;
    opt.epsilon = epsilon;
    opt.gradient_scale = gradient_scale;
    opt.batch_divisor = 1.0;
    opt.bias1 = 1.0;
    opt.bias2 = 1.0;
    if (optimizer == GEO_V8_OPTIMIZER_ADAM) {
        opt.bias1 = 1.0 - pow(beta1, (double)step);  // reference src/full_cycle_v8.c:976-984
        opt.bias2 = 1.0 - pow(beta2, (double)step);
        if (!isfinite(opt.bias1) || !isfinite(opt.bias2) || opt.bias1 <= 0.0 || opt.bias2 <= 0.0)
            return GEO_V8_NUMERIC_FAILURE;
    }
    // The streaming kernels read W from a device copy (every CTA reads it);
    // only the optimizer writes back into the mapped node.
    double *w = ws.scratch + 8;
    int ctas = 0;
    cudaError_t e = cudaMemsetAsync(ws.status, 0, sizeof(uint32_t), ws.stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(w, param->value.coefficients, (size_t)opt.blades * sizeof(double), cudaMemcpyHostToDevice,
                            ws.stream);
    geo::RepPlan rp;
    geo::RepDevice rd;
    const bool use_rep = p->dimension >= 5 && geo::make_rep_plan(&rp, p->dimension, p->signature, m.parameter_on_left) &&
                         geo::make_rep_device(&rd, rp) && geo::rep_supported(rd);
    if (e == cudaSuccess) {
        if (use_rep) {
            e = geo::launch_rep_cycle(rd, device_inputs, device_targets, w, batch, ws.records, &ctas, ws.stream);
        } else {
            const geo::SignPlan *sp = geo::cached_sign_plan(p->dimension, p->signature, m.parameter_on_left);
            e = sp == nullptr ? cudaErrorInvalidValue
                              : geo::launch_cycle(*sp, geo::kCycle, device_inputs, device_targets, w, nullptr, batch,
                                                  ws.records, &ctas, ws.stream);
        }
    }
    if (e == cudaSuccess)
        e = geo::launch_finalize(ws.records, ctas, opt, nullptr, ws.scratch, dparam->value.coefficients,
                                 dparam->first_moment, dparam->second_moment, ws.status, ws.stream);
    uint32_t bits = 0;
    double loss = 0.0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&bits, ws.status, sizeof(bits), cudaMemcpyDeviceToHost, ws.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&loss, ws.scratch, sizeof(loss), cudaMemcpyDeviceToHost, ws.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ws.stream);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_V8_BAD_PROGRAM;
    }
    if (loss_sum) *loss_sum = loss;
    if (bits & (geo::kDevOutputNonFinite | geo::kDevResidualNonFinite)) {
        // A non-finite sample would have been rejected by geo_v8_set_value.
        uint32_t in_bits = 0;
        if (cudaMemsetAsync(ws.status, 0, sizeof(uint32_t), ws.stream) == cudaSuccess &&
            geo::launch_check_finite(device_inputs, batch << p->dimension, 1u, ws.status, ws.stream) == cudaSuccess &&
            geo::launch_check_finite(device_targets, batch << p->dimension, 1u, ws.status, ws.stream) == cudaSuccess &&
            cudaMemcpyAsync(&in_bits, ws.status, sizeof(in_bits), cudaMemcpyDeviceToHost, ws.stream) == cudaSuccess &&
            cudaStreamSynchronize(ws.stream) == cudaSuccess && in_bits != 0u)
            return GEO_V8_INVALID_ARGUMENT;
        return GEO_V8_NUMERIC_FAILURE;
    }
    if (bits != 0u) return GEO_V8_NUMERIC_FAILURE;
    p->optimizer_step = step;
    p->forward_valid = 0u;
    p->backward_valid = 0u;
    (void)geo_v8_zero_grad(p);
    return GEO_V8_OK;
}
