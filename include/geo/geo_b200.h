/*
 * geo/geo_b200.h -- additive C ABI of libgeo_b200.so (no reference header has
 * these symbols; each block names the reference code whose semantics it
 * batches).
 *
 *  1. Trainer: a parameter multivector and its optimizer state resident on one
 *     GPU, trained by the fused full cycle (forward -> residual -> 0.5|r|^2 ->
 *     parameter VJP -> optimizer) in one streaming pass per minibatch.
 *     Optimizer semantics are the reference V8 graph runtime's for the graph
 *     x*w (or w*x) -> add(., scale(t, -1)) -> squared_norm
 *     (reference src/full_cycle_v8.c:942-1041): g = sum_s grad_s * scale,
 *     SGD w -= lr g, Adam m = b1 m + (1-b1) g, v = b2 v + (1-b2) g^2,
 *     w -= lr (m / (1-b1^t)) / (sqrt(v / (1-b2^t)) + eps); transactional
 *     (nothing changes when any candidate value is non-finite).
 *  2. Data parallelism: one process (or thread) per GPU; each rank trains on
 *     its own slice of the global batch and the per-rank gradient/loss record
 *     (2^n + 8 doubles) is all-gathered over NCCL and summed in rank order, so
 *     every rank applies the identical update to its replica.
 *  3. Pairwise products with both operands varying per element (reference
 *     src/operator_kernel.c:412-539, geo_operator_gp_f64 and its JVP/VJP),
 *     float64, plus a float32 build of the forward.
 *  4. Sparse fixed-multivector operators over a batch (reference
 *     src/operator_kernel.c:191-334, geo_operator_apply_*_f64 and VJPs).
 *
 * All device-pointer calls are asynchronous on the given stream; host-pointer
 * calls are synchronous. Arrays are sample-major [batch][2^n].
 */
#ifndef GEO_B200_H
#define GEO_B200_H

#include "geo/operator_kernel.h"

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GEO_B200_ABI_VERSION 0x00010000u

/* Status of the per-multivector geo_operator_*_f64 calls (geo/operator_kernel.h)
 * when the GPU call itself fails (no device, launch or copy error); the
 * reference's geo_operator_status_t has no such value. */
#define GEO_OPERATOR_B200_DEVICE_FAILURE 100

typedef enum {
    GEO_B200_OK = 0,
    GEO_B200_INVALID_ARGUMENT = 1,
    GEO_B200_UNSUPPORTED_DIMENSION = 2,
    GEO_B200_NUMERIC_FAILURE = 3,
    GEO_B200_RUNTIME_FAILURE = 4,
    GEO_B200_ALLOCATION_FAILURE = 5,
    GEO_B200_COMM_FAILURE = 6,
    GEO_B200_TIMEOUT = 7
} geo_b200_status_t;

typedef enum {
    GEO_B200_OPTIMIZER_SGD = 1,  /* same values as GEO_V8_OPTIMIZER_* */
    GEO_B200_OPTIMIZER_ADAM = 2
} geo_b200_optimizer_t;

typedef struct {
    uint32_t optimizer;      /* geo_b200_optimizer_t */
    double learning_rate;
    double beta1;
    double beta2;
    double epsilon;
} geo_b200_optimizer_config_t;

typedef struct geo_b200_trainer geo_b200_trainer_t;
typedef struct geo_b200_comm geo_b200_comm_t;

uint32_t geo_b200_abi_version(void);
const char *geo_b200_status_string(geo_b200_status_t status);

/* ---- 1. trainer ------------------------------------------------------- */

/* Creates the trainer on the current CUDA device. initial_parameter is a host
 * array of 2^dimension doubles; moments start at zero and the step count at 0
 * (like geo_v8_set_value on a PARAMETER, reference src/full_cycle_v8.c:559-563). */
geo_b200_status_t geo_b200_trainer_create(geo_b200_trainer_t **trainer, uint8_t dimension,
                                          const int8_t *signature, int parameter_on_left,
                                          const double *initial_parameter,
                                          const geo_b200_optimizer_config_t *config);
void geo_b200_trainer_destroy(geo_b200_trainer_t *trainer);

/* One training step on a device-resident minibatch (inputs/targets
 * [batch][2^n] in device memory). gradient_scale multiplies the summed
 * gradient (1/global_batch gives the mean, as geo_v8_optimizer_step's
 * gradient_scale). Asynchronous on `stream`; numeric status accumulates until
 * geo_b200_trainer_sync. With a communicator attached, every rank must call it
 * the same number of times. */
geo_b200_status_t geo_b200_trainer_step_device(geo_b200_trainer_t *trainer, const double *device_inputs,
                                               const double *device_targets, size_t batch,
                                               double gradient_scale, cudaStream_t stream);

/* The two halves of a step, for gradient accumulation over micro-batches
 * (the batched form of geo_v8_backward(accumulate) + geo_v8_optimizer_step):
 * accumulate adds the micro-batch's gradient and loss sums to the trainer's
 * running record; apply reduces the record across ranks (when a communicator
 * is attached), applies the optimizer with `gradient_scale` and clears the
 * record. step_device == accumulate + apply. */
geo_b200_status_t geo_b200_trainer_accumulate_device(geo_b200_trainer_t *trainer, const double *device_inputs,
                                                     const double *device_targets, size_t batch,
                                                     cudaStream_t stream);
geo_b200_status_t geo_b200_trainer_apply(geo_b200_trainer_t *trainer, double gradient_scale, cudaStream_t stream);

/* Same step from host (pageable or pinned) buffers: copies in, trains, waits,
 * and returns the step's status; *loss_sum receives sum_s 0.5 |r_s|^2 over
 * the global batch (may be NULL). */
geo_b200_status_t geo_b200_trainer_step_host(geo_b200_trainer_t *trainer, const double *inputs,
                                             const double *targets, size_t batch, double gradient_scale,
                                             double *loss_sum);

/* Waits for all queued steps (bounded by the communicator timeout when one is
 * attached) and returns the first failure since the previous sync.
 * *loss_sum (may be NULL) receives the last step's global loss sum. */
geo_b200_status_t geo_b200_trainer_sync(geo_b200_trainer_t *trainer, double *loss_sum);

/* Host copies of the parameter and Adam moments (any pointer may be NULL). */
geo_b200_status_t geo_b200_trainer_get_state(geo_b200_trainer_t *trainer, double *parameter,
                                             double *first_moment, double *second_moment,
                                             uint64_t *step_count);
/* Replaces the parameter and resets moments and step count. */
geo_b200_status_t geo_b200_trainer_set_parameter(geo_b200_trainer_t *trainer, const double *parameter);
/* Restores a full optimizer state (checkpoint resume). */
geo_b200_status_t geo_b200_trainer_set_state(geo_b200_trainer_t *trainer, const double *parameter,
                                             const double *first_moment, const double *second_moment,
                                             uint64_t step_count);
/* Kernel family used by the trainer's streaming pass.
 *  CAYLEY: the 2^n x 2^n sign-folded Cayley matrix on FP64 FMA units (any n).
 *  REPRESENTATION: a D x D real matrix representation of Cl(p,q) (D = 8 or 16
 *    for n = 5, 6) on FP64 tensor cores; S*D*D instead of 4^n multiply-adds.
 *  AUTO (default): REPRESENTATION where available for n >= 5, else CAYLEY.
 * Both are parity-checked against the reference to 1e-12. */
typedef enum {
    GEO_B200_ALGORITHM_AUTO = 0,
    GEO_B200_ALGORITHM_CAYLEY = 1,
    GEO_B200_ALGORITHM_REPRESENTATION = 2
} geo_b200_algorithm_t;

/* Selects the kernel family; INVALID_ARGUMENT when REPRESENTATION is not
 * available for this algebra and side. */
geo_b200_status_t geo_b200_trainer_set_algorithm(geo_b200_trainer_t *trainer, geo_b200_algorithm_t algorithm);
/* The family the next step will use (never AUTO). */
geo_b200_algorithm_t geo_b200_trainer_algorithm(const geo_b200_trainer_t *trainer);

/* Device pointer to the resident parameter (2^n doubles). */
const double *geo_b200_trainer_device_parameter(const geo_b200_trainer_t *trainer);

/* ---- 1b. fixed-parameter forward on a chosen kernel family ------------ */

/* outputs[s] = inputs[s] * parameter (parameter_on_left = 0) or
 * parameter * inputs[s]: the product of geo_batch_gp_cuda_planned_forward_f64
 * (reference src/batch_gp_cuda.cu:252-286, src/batch_gp.c:107-161) without a
 * plan object. All arrays are device memory; asynchronous on `stream`;
 * reports argument and launch errors only, like the device ABI.
 *  CAYLEY: the 2^n x 2^n sign-folded Cayley matrix on FP64 FMA units (any n).
 *  REPRESENTATION (n = 5, 6; inputs and outputs 16-byte aligned): X' = P x,
 *    Y' = X' W' on FP64 tensor cores, y = P^-1 Y'. Equal to the Cayley product
 *    up to rounding (within 1e-12 relative); INVALID_ARGUMENT where it is not
 *    available.
 *  AUTO: REPRESENTATION where available, else CAYLEY; bit-identical to
 *    geo_batch_gp_cuda_planned_forward_f64 on the same arrays (the same kernel).
 * device_parameter may be geo_b200_trainer_device_parameter(). Outputs may be
 * the inputs (in place) but must not overlap them otherwise. A non-finite
 * input coefficient makes every output coefficient of its sample non-finite
 * on both families, as in the reference (which of Inf and NaN may differ). */
geo_b200_status_t geo_b200_forward_f64(uint8_t dimension, const int8_t *signature, int parameter_on_left,
                                       geo_b200_algorithm_t algorithm, const double *device_inputs,
                                       const double *device_parameter, double *device_outputs, size_t batch_size,
                                       cudaStream_t stream);

/* ---- 2. data parallelism ---------------------------------------------- */

#define GEO_B200_COMM_ID_BYTES 128

/* Rank 0 creates the id and shares the bytes with the other ranks out of band. */
geo_b200_status_t geo_b200_comm_unique_id(unsigned char id[GEO_B200_COMM_ID_BYTES]);
/* Collective over `world` ranks; uses the current CUDA device. Returns
 * GEO_B200_TIMEOUT if the ranks have not all joined within timeout_ms. */
geo_b200_status_t geo_b200_comm_create(geo_b200_comm_t **comm, int rank, int world,
                                       const unsigned char id[GEO_B200_COMM_ID_BYTES], int timeout_ms);
void geo_b200_comm_destroy(geo_b200_comm_t *comm);
/* Aborts in-flight collectives (use after a peer failed). */
void geo_b200_comm_abort(geo_b200_comm_t *comm);
geo_b200_status_t geo_b200_trainer_attach_comm(geo_b200_trainer_t *trainer, geo_b200_comm_t *comm);

/* ---- 2b. batched V8 programs ------------------------------------------ */

/* One optimizer step of a compiled V8 program over a device-resident
 * minibatch, equal to: geo_v8_zero_grad; for every sample s: set the INPUT
 * node `input_node` to inputs[s] and the TARGET node `target_node` to
 * targets[s], geo_v8_forward, geo_v8_backward(accumulate = s != 0); then
 * geo_v8_optimizer_step(optimizer, ..., gradient_scale)
 * (reference src/full_cycle_v8.c:569-1041, per sample). Any compiled program:
 *   - the graph gp = GEOMETRIC_PRODUCT(input, w) or (w, input);
 *     neg = SCALE(target, -1); residual = ADD(gp, neg) (either order);
 *     loss = SQUARED_NORM(residual), with `w` its only PARAMETER and no
 *     constraint, runs as one fused streaming pass on the tensor cores;
 *   - every other graph (all node kinds, constraints, several parameters,
 *     STATE leaves held fixed across the batch) runs per sample on the GPU with
 *     the reference's arithmetic, gradients summed over the batch.
 * target_node may be GEO_V8_INVALID_NODE (device_targets then unused) for the
 * general path. Parameters and Adam moments are updated in place
 * (transactional), the step count advances, gradients are cleared; node
 * values other than the parameters are left unchanged. *loss_sum (may be
 * NULL) receives the sum over the batch of the loss node's value.
 * Synchronous; returns geo_v8_status_t values (declared in
 * geo/full_cycle_v8.h, passed here as int to keep this header independent). */
int geo_b200_v8_batch_train_step(void *program, uint32_t input_node, uint32_t target_node,
                                 const double *device_inputs, const double *device_targets, size_t batch,
                                 int optimizer, double learning_rate, double beta1, double beta2, double epsilon,
                                 double gradient_scale, double *loss_sum);

/* Batched inference: for every sample s, set `input_node` to inputs[s], run
 * geo_v8_forward and write the value of `output_node` to outputs[s]
 * ([batch][2^n] device arrays). Every other leaf keeps its value; node values
 * in the program are not modified. Synchronous; geo_v8_status_t values. */
int geo_b200_v8_batch_forward(void *program, uint32_t input_node, const double *device_inputs, size_t batch,
                              uint32_t output_node, double *device_outputs);

/* The graph runtime's exp and tanh (TANH nodes; SIGMOID nodes through exp,
 * reference src/full_cycle_v8.c:181-190, 651) are correctly rounded (round to
 * nearest, ties to even) for every binary64 argument: a table-driven
 * double-double evaluation with Ziv's rounding test, and an exact 256-bit
 * fixed-point evaluation when that test cannot decide. The reference calls the
 * C library's exp and tanh; wherever those are correctly rounded the results
 * agree bit for bit, elsewhere the value here is the closer one.
 * geo_b200_cr_math_f64 applies one of them to `count` doubles of a device array
 * (device_out may equal device_in), asynchronously on `stream`; the *_EXACT_PATH
 * values run the fixed-point evaluation for every argument it covers (a check
 * of that path). */
typedef enum {
    GEO_B200_CR_EXP = 0,
    GEO_B200_CR_TANH = 1,
    GEO_B200_CR_EXP_EXACT_PATH = 2,
    GEO_B200_CR_TANH_EXACT_PATH = 3
} geo_b200_cr_function_t;
geo_b200_status_t geo_b200_cr_math_f64(int function, const double *device_in, double *device_out, size_t count,
                                       cudaStream_t stream);

/* ---- 2c. parameter VJP that allocates nothing -------------------------- */

/* This entry point has no counterpart in the reference.
 *
 * Same result as geo_batch_gp_cuda_parameter_vjp_f64 (the summed parameter
 * cotangent of the batched geometric product), for callers that cannot call
 * cudaMalloc: hosts whose own allocator has reserved the device memory up
 * front (so a further cudaMalloc fails), latency-critical loops that must not
 * take the implicit device synchronisation of cudaMalloc/cudaFree, and plugin
 * hosts that forbid device allocation after start-up. It takes no plan (a plan
 * upload allocates); dimension and signature are given directly, all arrays
 * are device memory supplied by the caller, and the call is asynchronous on
 * `stream`.
 *
 * Its reduction scratch is one fixed array compiled into the library
 * (GEO_B200_NOALLOC_RECORDS records of 576 bytes, about 1.2 MB), which every
 * GPU that loads the library holds until the process exits. That bounds the
 * batch: batch_size must not exceed GEO_B200_NOALLOC_MAX_BATCH (131072
 * samples, any dimension); larger batches are rejected with
 * GEO_B200_INVALID_ARGUMENT before anything is launched. The first call on each
 * device looks up the array's device address (a one-time set-up per device,
 * repeated only if the device's context was recreated, e.g. after
 * cudaDeviceReset); make that first call before any stream capture. All calls share the one
 * array and every call overwrites the part it uses, so calls whose kernels
 * overlap on the GPU (different streams without ordering) race; order them on
 * one stream. */
#define GEO_B200_NOALLOC_RECORDS 2048u
#define GEO_B200_NOALLOC_MAX_BATCH 131072u
geo_b200_status_t geo_b200_parameter_vjp_noalloc_f64(uint8_t dimension, const int8_t *signature,
                                                     int parameter_on_left, const double *device_inputs,
                                                     const double *device_output_cotangents, size_t batch_size,
                                                     double *device_parameter_cotangent, cudaStream_t stream);

/* ---- 3. pairwise products (both operands vary per element) ------------ */

/* out[s] = left[s] * right[s]. */
geo_b200_status_t geo_b200_pairwise_gp_f64(uint8_t dimension, const int8_t *signature, const double *device_left,
                                           const double *device_right, double *device_out, size_t batch,
                                           cudaStream_t stream);
/* Per-element VJP: left_bar[s], right_bar[s] from out_bar[s]
 * (reference src/operator_kernel.c:494-539). Either output may be NULL. */
geo_b200_status_t geo_b200_pairwise_gp_vjp_f64(uint8_t dimension, const int8_t *signature,
                                               const double *device_left, const double *device_right,
                                               const double *device_out_cotangent, double *device_left_cotangent,
                                               double *device_right_cotangent, size_t batch, cudaStream_t stream);
/* Per-element JVP (reference src/operator_kernel.c:449-492). */
geo_b200_status_t geo_b200_pairwise_gp_jvp_f64(uint8_t dimension, const int8_t *signature,
                                               const double *device_left, const double *device_right,
                                               const double *device_left_tangent, const double *device_right_tangent,
                                               double *device_out_tangent, size_t batch, cudaStream_t stream);
/* float32 build of the forward. When left_even_compact is non-zero, `left`
 * holds only the 2^(n-1) even-grade coefficients of each element, in
 * increasing blade order (compact storage); otherwise 2^n dense values. */
geo_b200_status_t geo_b200_pairwise_gp_f32(uint8_t dimension, const int8_t *signature, const float *device_left,
                                           int left_even_compact, const float *device_right, float *device_out,
                                           size_t batch, cudaStream_t stream);

/* Bounded waits of the n = 6 TMA pairwise kernels (no counterpart in the
 * reference, whose products run on the CPU). Every wait of those kernels on a
 * load or on a ring stage gives up after a fixed number of polls; a CTA whose
 * wait gave up stops loading, waits (bounded) for its loads in flight, writes
 * NaN into every output row it had not stored and ends, so the context stays
 * usable. This call synchronizes the current device and reports how many
 * give-ups (one per CTA of the float32 kernel, one per warp of the float64
 * kernel) were recorded since the last reset (*count); reset != 0 clears it.
 * Returns GEO_B200_TIMEOUT when the count is non-zero. */
geo_b200_status_t geo_b200_pairwise_wait_failures(unsigned *count, int reset);
/* Self-test of that failure path: runs the float64 (precision 64) or float32
 * (precision 32) TMA pairwise kernel over `batch` rows of device_out with no
 * load issued at all, so every first wait runs out after wait_limit polls with
 * no copy in flight. Synchronizes the stream; returns GEO_B200_TIMEOUT when the
 * kernel reported its give-up (device_out then holds NaN in every row). */
geo_b200_status_t geo_b200_pairwise_wait_selftest(int precision, void *device_out, size_t batch,
                                                  uint32_t wait_limit, cudaStream_t stream);

/* ---- 4. sparse fixed-multivector plans over a batch ------------------- */

/* out[s] = plan applied to in[s] (integer coefficients of the plan). */
geo_b200_status_t geo_b200_sparse_apply_f64(const geo_operator_plan_i32_t *plan, const double *device_in,
                                            double *device_out, size_t batch, cudaStream_t stream);
/* Coefficients replaced by real parameters[term_count] (device array). */
geo_b200_status_t geo_b200_sparse_apply_parametric_f64(const geo_operator_plan_i32_t *plan,
                                                       const double *device_parameters, const double *device_in,
                                                       double *device_out, size_t batch, cudaStream_t stream);
/* in_bar[s] = M^T out_bar[s] (integer plan). */
geo_b200_status_t geo_b200_sparse_apply_vjp_f64(const geo_operator_plan_i32_t *plan,
                                                const double *device_out_cotangent, double *device_in_cotangent,
                                                size_t batch, cudaStream_t stream);
/* Parametric VJP: per-element input cotangents (may be NULL) and the
 * parameter cotangents summed over the batch (term_count doubles, device). */
geo_b200_status_t geo_b200_sparse_apply_parametric_vjp_f64(const geo_operator_plan_i32_t *plan,
                                                           const double *device_parameters, const double *device_in,
                                                           const double *device_out_cotangent,
                                                           double *device_in_cotangent,
                                                           double *device_parameter_cotangent, size_t batch,
                                                           cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif
