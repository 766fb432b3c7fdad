/*
 * geo_oracle.h -- CPU oracle for the batched geometric-product path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference
 * CPU algorithm, used by tests/, by __graft_entry__.smoke() and by the
 * cpu_baseline leg of bench.py as the checker. The product library
 * (libgeo_b200.so) never links, loads or calls it.
 *
 * Every function follows the reference operation for operation (same loop
 * order, same accumulation order, same status rules), so that, compiled with
 * gcc without FMA contraction, it reproduces the reference bit for bit. That
 * claim is pinned by tests/test_oracle.py against the reference compiled from
 * its own sources (oracle/_ref, see oracle/Makefile) and against the committed
 * golden vectors in tests/golden/.
 *
 * Status codes are the reference's integer values
 * (OK=0, INVALID_ARGUMENT=1, UNSUPPORTED_DIMENSION=2, NUMERIC_FAILURE=3 for
 * the batch path; the operator path uses its own enum values).
 */
#ifndef GEO_ORACLE_H
#define GEO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* reference src/batch_gp.c:29-45 and src/operator_kernel.c:111-135 */
int orc_gp_sign(uint8_t left, uint8_t right, const int8_t *signature, uint8_t dimension);

/*
 * reference src/batch_gp.c:69-105. Writes the 16400-byte plan layout of
 * geo_batch_gp_plan_t into `plan_bytes` (which must hold 16400 bytes).
 */
int orc_batch_plan_init(void *plan_bytes, uint8_t dimension, const int8_t *signature);

/* reference src/batch_gp.c:107-141 (parameter_on_left selects the side) */
int orc_batch_forward(const void *plan_bytes, const double *inputs, size_t batch_size,
                      const double *parameter, int parameter_on_left, double *outputs);

/* reference src/batch_gp.c:163-201 */
int orc_batch_vjp(const void *plan_bytes, const double *inputs, const double *cotangents,
                  size_t batch_size, int parameter_on_left, double *parameter_cotangent);

/* reference src/batch_gp.c:237-308 */
int orc_batch_mse_sgd_step(const void *plan_bytes, const double *inputs, const double *targets,
                           size_t batch_size, double learning_rate, int parameter_on_left,
                           double *parameter, double *mean_loss);

/* reference src/operator_kernel.c:412-447 (dense coefficient arrays of 2^n) */
int orc_gp_f64(uint8_t dimension, const int8_t *signature, const double *left,
               const double *right, double *output);

/* reference src/operator_kernel.c:449-492 */
int orc_gp_f64_jvp(uint8_t dimension, const int8_t *signature, const double *left,
                   const double *right, const double *left_tangent,
                   const double *right_tangent, double *output_tangent);

/* reference src/operator_kernel.c:494-539 */
int orc_gp_f64_vjp(uint8_t dimension, const int8_t *signature, const double *left,
                   const double *right, const double *output_cotangent,
                   double *left_cotangent, double *right_cotangent);

/*
 * Sparse fixed-multivector operators. `blades`/`coefficients` are the plan's
 * terms (term_count <= 64), `side` 0 = right (input * plan), 1 = left.
 * reference src/operator_kernel.c:191-220 (apply), :222-254 (parametric),
 * :256-278 (apply VJP), :280-334 (parametric VJP).
 */
int orc_sparse_apply(uint8_t dimension, const int8_t *signature, int side,
                     const uint8_t *blades, const int32_t *coefficients, size_t term_count,
                     const double *input, double *output);
int orc_sparse_apply_parametric(uint8_t dimension, const int8_t *signature, int side,
                                const uint8_t *blades, const double *parameters,
                                size_t term_count, const double *input, double *output);
int orc_sparse_apply_vjp(uint8_t dimension, const int8_t *signature, int side,
                         const uint8_t *blades, const int32_t *coefficients, size_t term_count,
                         const double *output_cotangent, double *input_cotangent);
int orc_sparse_apply_parametric_vjp(uint8_t dimension, const int8_t *signature, int side,
                                    const uint8_t *blades, const double *parameters,
                                    size_t term_count, const double *input,
                                    const double *output_cotangent, double *input_cotangent,
                                    double *parameter_cotangent);

/*
 * One optimizer update of a single PARAMETER node with no constraint,
 * following reference src/full_cycle_v8.c:942-1041 operation for operation:
 * g = gradient_sum[b] * gradient_scale; SGD: w -= lr * g; Adam:
 * m = b1 m + (1-b1) g, v = b2 v + (1-b2) g g, w -= lr (m/bias1)/(sqrt(v/bias2)+eps)
 * with bias_k = 1 - pow(beta_k, step). `step` is the step number being taken
 * (optimizer_step + 1). optimizer: 1 = SGD, 2 = Adam (GEO_V8_OPTIMIZER_*).
 * Transactional: on failure nothing is written. Returns GEO_V8 status values
 * (OK=0, INVALID_ARGUMENT=1, NUMERIC_FAILURE=11).
 */
int orc_v8_optimizer_update(size_t count, int optimizer, double learning_rate, double beta1,
                            double beta2, double epsilon, double gradient_scale,
                            uint64_t step, const double *gradient_sum, double *value,
                            double *first_moment, double *second_moment);

#ifdef __cplusplus
}
#endif

#endif
