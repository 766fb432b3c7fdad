// v8_host.cpp -- V8 graph construction and bookkeeping (geo/full_cycle_v8.h).
//
// Graph structure, validation and status rules restate the reference
// (src/full_cycle_v8.c:7-130 helpers, :283-567 construction, :694-715
// zero_grad, :942-1041 optimizer bookkeeping, :1043-1098 states and
// accessors). Node storage is one mapped page-locked allocation so that the
// forward, backward and optimizer kernels (v8_kernels.cu) work on the very
// memory the caller reads through geo_v8_value / program->nodes.
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <cstdlib>

#include "v8_internal.h"

namespace geo {
namespace v8 {

size_t allocation_bytes(size_t capacity) {
    return capacity * (sizeof(geo_v8_node_t) + sizeof(Candidate)) + sizeof(Control);
}
Candidate *candidates(geo_v8_node_t *nodes, size_t capacity) {
    return reinterpret_cast<Candidate *>(nodes + capacity);
}
Control *control(geo_v8_node_t *nodes, size_t capacity) {
    return reinterpret_cast<Control *>(candidates(nodes, capacity) + capacity);
}

bool dimension_valid(unsigned n) { return n >= 1u && n <= GEO_OPERATOR_MAX_DIMENSION; }

bool signature_valid(const int8_t *signature, unsigned n) {
    if (signature == nullptr || !dimension_valid(n)) return false;
    for (unsigned i = 0; i < n; ++i)
        if (signature[i] != 1 && signature[i] != -1) return false;
    return true;
}

static bool same_signature(unsigned n, const int8_t *a, const int8_t *b) {
    if (a == nullptr || b == nullptr) return false;
    for (unsigned i = 0; i < n; ++i)
        if (a[i] != b[i]) return false;
    return true;
}

void mv_zero(geo_operator_mv_f64_t *value, unsigned n, const int8_t *signature) {
    memset(value, 0, sizeof(*value));
    value->dimension = (uint8_t)n;
    memcpy(value->signature, signature, n);
}

bool mv_valid(const geo_operator_mv_f64_t *value, unsigned n, const int8_t *signature) {
    if (value == nullptr || value->dimension != n || !same_signature(n, value->signature, signature)) return false;
    for (unsigned b = 0; b < (1u << n); ++b)
        if (!isfinite(value->coefficients[b])) return false;
    return true;
}

bool program_valid(const geo_v8_program_t *p) {
    return p != nullptr && p->abi_version == GEO_V8_ABI_VERSION && signature_valid(p->signature, p->dimension) &&
           p->pairing == GEO_V8_PAIRING_COEFFICIENT_EUCLIDEAN && p->node_count <= p->node_capacity &&
           (p->node_capacity == 0u || p->nodes != nullptr);
}

bool node_exists(const geo_v8_program_t *p, geo_v8_node_id_t id) { return program_valid(p) && id < p->node_count; }

bool leaf_kind(int k) {
    return k == GEO_V8_NODE_INPUT || k == GEO_V8_NODE_TARGET || k == GEO_V8_NODE_PARAMETER ||
           k == GEO_V8_NODE_CONSTANT || k == GEO_V8_NODE_STATE;
}
bool unary_kind(int k) {
    return k == GEO_V8_NODE_SCALE || k == GEO_V8_NODE_REVERSE || k == GEO_V8_NODE_GRADE_PROJECT ||
           k == GEO_V8_NODE_GRADE_INVOLUTION || k == GEO_V8_NODE_CLIFFORD_CONJUGATE || k == GEO_V8_NODE_TANH ||
           k == GEO_V8_NODE_SIGMOID || k == GEO_V8_NODE_EUCLIDEAN_NORMALIZE || k == GEO_V8_NODE_SQUARED_NORM;
}
bool binary_kind(int k) {
    return k == GEO_V8_NODE_ADD || k == GEO_V8_NODE_GEOMETRIC_PRODUCT || k == GEO_V8_NODE_HADAMARD;
}

}  // namespace v8
}  // namespace geo

using namespace geo::v8;

namespace {

bool name_valid(const char *name) {
    const size_t len = name == nullptr ? 0u : strlen(name);
    return len > 0u && len < GEO_V8_NAME_MAX;
}

bool name_unique(const geo_v8_program_t *p, const char *name) {
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i)
        if (strcmp(p->nodes[i].name, name) == 0) return false;
    return true;
}

geo_v8_status_t reserve_one(geo_v8_program_t *p, const char *name, geo_v8_node_id_t *id) {
    if (!program_valid(p) || id == nullptr || !name_valid(name)) return GEO_V8_INVALID_ARGUMENT;
    if (p->compiled) return GEO_V8_BAD_PROGRAM;
    if (!name_unique(p, name)) return GEO_V8_DUPLICATE_NAME;
    if (p->node_count == p->node_capacity) {
        const size_t next = p->node_capacity == 0u ? 16u : (size_t)p->node_capacity * 2u;
        if (next <= (size_t)p->node_capacity || next > (size_t)UINT32_MAX) return GEO_V8_ALLOCATION_FAILURE;
        const geo_v8_status_t st = geo_v8_program_reserve(p, next);
        if (st != GEO_V8_OK) return st;
    }
    *id = p->node_count;
    ++p->node_count;
    return GEO_V8_OK;
}

bool loss_scalar(const geo_v8_program_t *p) {
    const geo_operator_mv_f64_t *loss = &p->nodes[p->loss_node].value;
    if (!isfinite(loss->coefficients[0])) return false;
    for (unsigned b = 1; b < (1u << p->dimension); ++b)
        if (loss->coefficients[b] != 0.0) return false;
    return true;
}

}  // namespace

extern "C" uint32_t geo_v8_abi_version(void) { return GEO_V8_ABI_VERSION; }

extern "C" geo_v8_status_t geo_v8_program_init(geo_v8_program_t *p, uint8_t dimension, const int8_t *signature,
                                               geo_v8_pairing_t pairing, size_t initial_capacity) {
    if (p == nullptr || signature == nullptr) return GEO_V8_INVALID_ARGUMENT;
    if (!dimension_valid(dimension)) return GEO_V8_UNSUPPORTED_DIMENSION;
    if (!signature_valid(signature, dimension) || pairing != GEO_V8_PAIRING_COEFFICIENT_EUCLIDEAN ||
        initial_capacity > (size_t)UINT32_MAX)
        return GEO_V8_INVALID_ARGUMENT;
    memset(p, 0, sizeof(*p));
    p->abi_version = GEO_V8_ABI_VERSION;
    p->dimension = dimension;
    memcpy(p->signature, signature, dimension);
    p->pairing = (uint8_t)pairing;
    p->loss_node = GEO_V8_INVALID_NODE;
    if (initial_capacity != 0u) return geo_v8_program_reserve(p, initial_capacity);
    return GEO_V8_OK;
}

extern "C" void geo_v8_program_free(geo_v8_program_t *p) {
    if (p == nullptr) return;
    if (p->nodes != nullptr) cudaFreeHost(p->nodes);
    memset(p, 0, sizeof(*p));
}

extern "C" geo_v8_status_t geo_v8_program_reserve(geo_v8_program_t *p, size_t capacity) {
    if (!program_valid(p) || capacity > (size_t)UINT32_MAX) return GEO_V8_INVALID_ARGUMENT;
    if (p->compiled) return GEO_V8_BAD_PROGRAM;
    if (capacity <= (size_t)p->node_capacity) return GEO_V8_OK;
    geo_v8_node_t *fresh = nullptr;
    if (cudaHostAlloc((void **)&fresh, allocation_bytes(capacity), cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
        (void)cudaGetLastError();
        return GEO_V8_ALLOCATION_FAILURE;
    }
    memset(fresh, 0, allocation_bytes(capacity));
    if (p->nodes != nullptr) {
        memcpy(fresh, p->nodes, (size_t)p->node_count * sizeof(geo_v8_node_t));
        cudaFreeHost(p->nodes);
    }
    p->nodes = fresh;
    p->node_capacity = (geo_v8_node_id_t)capacity;
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_add_leaf(geo_v8_program_t *p, geo_v8_node_kind_t kind, const char *name,
                                           const geo_operator_mv_f64_t *initial_value, int requires_grad,
                                           geo_v8_constraint_t constraint, geo_v8_node_id_t *id) {
    if (!program_valid(p) || !leaf_kind(kind) || constraint < GEO_V8_CONSTRAINT_NONE ||
        constraint > GEO_V8_CONSTRAINT_EVEN_VERSOR || !mv_valid(initial_value, p->dimension, p->signature))
        return GEO_V8_INVALID_ARGUMENT;
    if (kind != GEO_V8_NODE_PARAMETER && constraint != GEO_V8_CONSTRAINT_NONE) return GEO_V8_INVALID_ARGUMENT;
    const geo_v8_status_t st = reserve_one(p, name, id);
    if (st != GEO_V8_OK) return st;
    geo_v8_node_t *node = &p->nodes[*id];
    memset(node, 0, sizeof(*node));
    node->kind = (uint8_t)kind;
    node->requires_grad = (requires_grad != 0 || kind == GEO_V8_NODE_PARAMETER) ? 1u : 0u;
    node->constraint = (uint8_t)constraint;
    node->left = node->right = node->state_update = GEO_V8_INVALID_NODE;
    memcpy(node->name, name, strlen(name) + 1u);
    node->value = *initial_value;
    mv_zero(&node->cotangent, p->dimension, p->signature);
    mv_zero(&node->gradient, p->dimension, p->signature);
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_add_unary(geo_v8_program_t *p, geo_v8_node_kind_t kind, const char *name,
                                            geo_v8_node_id_t input, double scalar, uint8_t grade,
                                            geo_v8_node_id_t *id) {
    if (!program_valid(p) || !unary_kind(kind) || !node_exists(p, input) || !isfinite(scalar) ||
        (kind == GEO_V8_NODE_GRADE_PROJECT && grade > p->dimension))
        return GEO_V8_INVALID_ARGUMENT;
    const geo_v8_status_t st = reserve_one(p, name, id);
    if (st != GEO_V8_OK) return st;
    geo_v8_node_t *node = &p->nodes[*id];
    memset(node, 0, sizeof(*node));
    node->kind = (uint8_t)kind;
    node->requires_grad = p->nodes[input].requires_grad;
    node->grade = grade;
    node->left = input;
    node->right = node->state_update = GEO_V8_INVALID_NODE;
    node->scalar = scalar;
    memcpy(node->name, name, strlen(name) + 1u);
    mv_zero(&node->value, p->dimension, p->signature);
    mv_zero(&node->cotangent, p->dimension, p->signature);
    mv_zero(&node->gradient, p->dimension, p->signature);
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_add_binary(geo_v8_program_t *p, geo_v8_node_kind_t kind, const char *name,
                                             geo_v8_node_id_t left, geo_v8_node_id_t right, geo_v8_node_id_t *id) {
    if (!program_valid(p) || !binary_kind(kind) || !node_exists(p, left) || !node_exists(p, right))
        return GEO_V8_INVALID_ARGUMENT;
    const geo_v8_status_t st = reserve_one(p, name, id);
    if (st != GEO_V8_OK) return st;
    geo_v8_node_t *node = &p->nodes[*id];
    memset(node, 0, sizeof(*node));
    node->kind = (uint8_t)kind;
    node->requires_grad = (p->nodes[left].requires_grad || p->nodes[right].requires_grad) ? 1u : 0u;
    node->left = left;
    node->right = right;
    node->state_update = GEO_V8_INVALID_NODE;
    memcpy(node->name, name, strlen(name) + 1u);
    mv_zero(&node->value, p->dimension, p->signature);
    mv_zero(&node->cotangent, p->dimension, p->signature);
    mv_zero(&node->gradient, p->dimension, p->signature);
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_bind_state_update(geo_v8_program_t *p, geo_v8_node_id_t state,
                                                    geo_v8_node_id_t source) {
    if (!node_exists(p, state) || !node_exists(p, source)) return GEO_V8_BAD_NODE;
    if (p->compiled || p->nodes[state].kind != GEO_V8_NODE_STATE) return GEO_V8_BAD_PROGRAM;
    p->nodes[state].state_update = source;
    return GEO_V8_OK;
}

extern "C" geo_v8_node_id_t geo_v8_find_node(const geo_v8_program_t *p, const char *name) {
    if (!program_valid(p) || !name_valid(name)) return GEO_V8_INVALID_NODE;
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i)
        if (strcmp(p->nodes[i].name, name) == 0) return i;
    return GEO_V8_INVALID_NODE;
}

extern "C" geo_v8_status_t geo_v8_compile(geo_v8_program_t *p, geo_v8_node_id_t loss_node) {
    if (!program_valid(p)) return GEO_V8_BAD_PROGRAM;
    if (p->node_count == 0u || loss_node >= p->node_count) return GEO_V8_BAD_NODE;
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i) {
        const geo_v8_node_t *node = &p->nodes[i];
        const int kind = node->kind;
        if (!name_valid(node->name)) return GEO_V8_BAD_PROGRAM;
        if (leaf_kind(kind)) {
            if (node->left != GEO_V8_INVALID_NODE || node->right != GEO_V8_INVALID_NODE ||
                !mv_valid(&node->value, p->dimension, p->signature))
                return GEO_V8_BAD_PROGRAM;
            if (kind == GEO_V8_NODE_STATE && node->state_update != GEO_V8_INVALID_NODE &&
                node->state_update >= p->node_count)
                return GEO_V8_BAD_PROGRAM;
        } else if (unary_kind(kind)) {
            if (node->left >= i || node->right != GEO_V8_INVALID_NODE) return GEO_V8_BAD_PROGRAM;
        } else if (binary_kind(kind)) {
            if (node->left >= i || node->right >= i) return GEO_V8_BAD_PROGRAM;
        } else {
            return GEO_V8_BAD_PROGRAM;
        }
    }
    p->compiled = 1u;
    p->forward_valid = 0u;
    p->backward_valid = 0u;
    p->loss_node = loss_node;
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_set_value(geo_v8_program_t *p, geo_v8_node_id_t id,
                                            const geo_operator_mv_f64_t *value) {
    if (!node_exists(p, id)) return GEO_V8_BAD_NODE;
    if (!mv_valid(value, p->dimension, p->signature)) return GEO_V8_INVALID_ARGUMENT;
    geo_v8_node_t *node = &p->nodes[id];
    if (!leaf_kind(node->kind)) return GEO_V8_BAD_NODE;
    node->value = *value;
    if (node->kind == GEO_V8_NODE_PARAMETER) {
        memset(node->first_moment, 0, sizeof(node->first_moment));
        memset(node->second_moment, 0, sizeof(node->second_moment));
        p->optimizer_step = 0u;
    }
    p->forward_valid = 0u;
    p->backward_valid = 0u;
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_forward(geo_v8_program_t *p) {
    if (!program_valid(p)) return GEO_V8_BAD_PROGRAM;
    if (!p->compiled) return GEO_V8_NOT_COMPILED;
    p->forward_valid = 0u;
    p->backward_valid = 0u;
    const geo_v8_status_t st = run_forward(p);
    if (st == GEO_V8_OK) p->forward_valid = 1u;
    return st;
}

extern "C" geo_v8_status_t geo_v8_zero_grad(geo_v8_program_t *p) {
    if (!program_valid(p)) return GEO_V8_BAD_PROGRAM;
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i) {
        mv_zero(&p->nodes[i].cotangent, p->dimension, p->signature);
        mv_zero(&p->nodes[i].gradient, p->dimension, p->signature);
    }
    p->gradient_samples = 0u;
    p->backward_valid = 0u;
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_backward(geo_v8_program_t *p, int accumulate) {
    if (!program_valid(p)) return GEO_V8_BAD_PROGRAM;
    if (!p->compiled) return GEO_V8_NOT_COMPILED;
    if (!p->forward_valid) return GEO_V8_FORWARD_REQUIRED;
    if (!loss_scalar(p)) return GEO_V8_NON_SCALAR_LOSS;
    if (!accumulate) p->gradient_samples = 0u;
    const geo_v8_status_t st = run_backward(p, accumulate);
    if (st != GEO_V8_OK) return st;
    ++p->gradient_samples;
    p->backward_valid = 1u;
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_optimizer_step(geo_v8_program_t *p, geo_v8_optimizer_t optimizer,
                                                 double learning_rate, double beta1, double beta2, double epsilon,
                                                 double gradient_scale) {
    if (!program_valid(p)) return GEO_V8_BAD_PROGRAM;
    if (!p->compiled) return GEO_V8_NOT_COMPILED;
    if (!p->backward_valid || p->gradient_samples == 0u) return GEO_V8_BACKWARD_REQUIRED;
    if ((optimizer != GEO_V8_OPTIMIZER_SGD && optimizer != GEO_V8_OPTIMIZER_ADAM) || !isfinite(learning_rate) ||
        learning_rate <= 0.0 || !isfinite(gradient_scale) || gradient_scale <= 0.0 || !isfinite(beta1) ||
        beta1 < 0.0 || beta1 >= 1.0 || !isfinite(beta2) || beta2 < 0.0 || beta2 >= 1.0 || !isfinite(epsilon) ||
        epsilon <= 0.0)
        return GEO_V8_INVALID_ARGUMENT;
    const uint64_t step = p->optimizer_step + 1u;
    double bias1 = 1.0, bias2 = 1.0;
    if (optimizer == GEO_V8_OPTIMIZER_ADAM) {
        // reference src/full_cycle_v8.c:976-984, host libm pow
        bias1 = 1.0 - pow(beta1, (double)step);
        bias2 = 1.0 - pow(beta2, (double)step);
        if (!isfinite(bias1) || !isfinite(bias2) || bias1 <= 0.0 || bias2 <= 0.0) return GEO_V8_NUMERIC_FAILURE;
    }
    const geo_v8_status_t st =
        run_optimizer(p, optimizer, learning_rate, beta1, beta2, epsilon, gradient_scale, bias1, bias2);
    if (st != GEO_V8_OK) return st;
    p->optimizer_step = step;
    p->forward_valid = 0u;
    p->backward_valid = 0u;
    (void)geo_v8_zero_grad(p);
    return GEO_V8_OK;
}

extern "C" geo_v8_status_t geo_v8_commit_states(geo_v8_program_t *p) {
    if (!program_valid(p)) return GEO_V8_BAD_PROGRAM;
    if (!p->compiled) return GEO_V8_NOT_COMPILED;
    if (!p->forward_valid) return GEO_V8_FORWARD_REQUIRED;
    // Two phases (gather, then write) so states that read other states see old values.
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i)
        if (p->nodes[i].kind == GEO_V8_NODE_STATE && p->nodes[i].state_update == GEO_V8_INVALID_NODE)
            return GEO_V8_STATE_UPDATE_REQUIRED;
    geo_operator_mv_f64_t *updates =
        (geo_operator_mv_f64_t *)calloc(p->node_count ? p->node_count : 1u, sizeof(geo_operator_mv_f64_t));
    if (updates == nullptr) return GEO_V8_ALLOCATION_FAILURE;
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i)
        if (p->nodes[i].kind == GEO_V8_NODE_STATE) updates[i] = p->nodes[p->nodes[i].state_update].value;
    for (geo_v8_node_id_t i = 0; i < p->node_count; ++i)
        if (p->nodes[i].kind == GEO_V8_NODE_STATE) p->nodes[i].value = updates[i];
    free(updates);
    p->forward_valid = 0u;
    return GEO_V8_OK;
}

extern "C" const geo_operator_mv_f64_t *geo_v8_value(const geo_v8_program_t *p, geo_v8_node_id_t id) {
    if (!node_exists(p, id)) return nullptr;
    return &p->nodes[id].value;
}

extern "C" const geo_operator_mv_f64_t *geo_v8_gradient(const geo_v8_program_t *p, geo_v8_node_id_t id) {
    if (!node_exists(p, id) || p->gradient_samples == 0u) return nullptr;
    return &p->nodes[id].gradient;
}
