// v8_internal.h -- shared pieces of the V8 graph runtime (v8_host.cpp, v8_kernels.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "geo/full_cycle_v8.h"

namespace geo {
namespace v8 {

// The node array of a program is one mapped, page-locked host allocation:
//   [ node_capacity x geo_v8_node_t | node_capacity x Candidate | Control ]
// Callers see only `nodes`; the trailing area holds the optimizer's
// transactional candidates and the device-written status word.
struct Candidate {
    double value[64];
    double first[64];
    double second[64];
};

struct Control {
    int32_t status;      // geo_v8_status_t written by the kernels
    int32_t failed_node; // first node that failed (diagnostics)
    int32_t pad[14];
};

size_t allocation_bytes(size_t capacity);
Candidate *candidates(geo_v8_node_t *nodes, size_t capacity);
Control *control(geo_v8_node_t *nodes, size_t capacity);

// Validation helpers with the reference's rules (src/full_cycle_v8.c:7-130).
bool dimension_valid(unsigned n);
bool signature_valid(const int8_t *signature, unsigned n);
bool mv_valid(const geo_operator_mv_f64_t *value, unsigned n, const int8_t *signature);
bool program_valid(const geo_v8_program_t *program);
bool node_exists(const geo_v8_program_t *program, geo_v8_node_id_t id);
bool leaf_kind(int kind);
bool unary_kind(int kind);
bool binary_kind(int kind);
void mv_zero(geo_operator_mv_f64_t *value, unsigned n, const int8_t *signature);

// Device execution (v8_kernels.cu); each call launches and waits.
geo_v8_status_t run_forward(geo_v8_program_t *program);
geo_v8_status_t run_backward(geo_v8_program_t *program, int accumulate);
geo_v8_status_t run_optimizer(geo_v8_program_t *program, int optimizer, double learning_rate, double beta1,
                              double beta2, double epsilon, double gradient_scale, double bias1, double bias2);

// Batched execution of a compiled program over device-resident rows
// (v8_batch.cu). Each RowLeaf takes, for sample s, its coefficients from row s
// of row source 1 (a) or 2 (b), starting at `column`; every other leaf keeps
// its value. backward != 0: per-sample forward + backward, *loss_sum = sum of
// the loss node over the batch, (*gradients)[i * 64 + b] = gradient of leaf i
// summed over the batch. backward == 0: forward only, row s of device_outputs
// ([batch][2^n]) receives output_node's value. Synchronous; returns the first
// failure (a non-finite row value gives GEO_V8_INVALID_ARGUMENT, as
// geo_v8_set_value would).
struct RowLeaf {
    uint32_t node;
    int source;
    size_t column;
};
struct RowSource {
    const double *base;
    size_t stride;  // doubles per row
};
geo_v8_status_t run_batch(geo_v8_program_t *program, const std::vector<RowLeaf> &row_leaves, const RowSource &a,
                          const RowSource &b, uint32_t output_node, double *device_outputs, size_t batch,
                          int backward, double *loss_sum, std::vector<double> *gradients);

}  // namespace v8
}  // namespace geo
