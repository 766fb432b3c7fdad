// geo_internal.h -- internal declarations shared by the sm_100a kernels and the
// C-ABI translation units of libgeo_b200.so. Nothing here is exported.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "geo/batch_gp.h"
#include "geo/operator_kernel.h"

namespace geo {

constexpr int kMaxDim = 6;
constexpr int kMaxBlades = 64;

// Baked routing/sign plan for one (dimension, signature, side) triple.
// neg[i] bit p is set when sigma(i, p) = -1, where sigma is the sign of the
// term that pairs input blade i with parameter blade p:
//   parameter on the right: sigma(i, p) = s(i, p)  (term left=i, right=p)
//   parameter on the left:  sigma(i, p) = s(p, i)  (term left=p, right=i)
// and the output blade is always i ^ p (reference src/batch_gp.c:127-137).
// Passed to kernels by value (kernel parameter space, 528 bytes).
struct SignPlan {
    uint64_t neg[kMaxBlades];
    int32_t dimension;
    int32_t blades;
    int32_t parameter_on_left;
    int32_t reserved;
};

// Sign rule of the reference (src/batch_gp.c:29-45): each axis of `left`
// flips the sign once per lower axis set in `right`; a shared axis multiplies
// by its metric entry. Bit-exact integer arithmetic.
int sign_rule(uint8_t left, uint8_t right, const int8_t *signature, uint8_t dimension);
bool dimension_valid(unsigned dimension);
bool signature_valid(const int8_t *signature, unsigned dimension);

// Build the baked plan; returns false for an invalid dimension/signature.
bool make_sign_plan(SignPlan *out, uint8_t dimension, const int8_t *signature,
                    int parameter_on_left);

// ---------------------------------------------------------------------------
// Reduction record written by every CTA of the streaming kernels. The
// finalize kernel sums records in CTA order, so results are deterministic.
// Layout per CTA: [0, blades) parameter gradient partial, then:
constexpr int kRecLoss = 64;      // sum of 0.5 r^2
constexpr int kRecCheckY = 65;    // sum of 0*y  (NaN iff some y is non-finite)
constexpr int kRecCheckR = 66;    // sum of 0*r  (NaN iff some r is non-finite)
constexpr int kRecCheckIn = 67;   // sum of 0*x + 0*t (NaN iff some input is non-finite)
constexpr int kRecStride = 72;    // doubles per CTA record (576 B, 64-B multiple)
constexpr int kMaxCtas = 1184;    // 148 SMs x 8

// Status word written by device code (bit flags).
enum DeviceStatusBits : uint32_t {
    kDevOk = 0u,
    kDevInputNonFinite = 1u,     // inputs/targets/parameter not finite
    kDevOutputNonFinite = 2u,    // forward outputs not finite
    kDevResidualNonFinite = 4u,  // residual overflowed
    kDevGradientNonFinite = 8u,  // parameter gradient not finite
    kDevCandidateNonFinite = 16u,// updated parameter not finite (update not committed)
    kDevLossNonFinite = 32u,     // mean loss not finite (update committed)
    kDevBiasInvalid = 64u,       // Adam bias correction not positive/finite
};

// Optimizer description consumed by the finalize kernel.
enum OptimizerKind : int32_t {
    kOptNone = 0,        // gradient + loss only
    kOptSgdBatchGp = 1,  // w -= lr * g / B        (reference src/batch_gp.c:302-304)
    kOptSgdV8 = 2,       // w -= lr * (g * scale)  (reference src/full_cycle_v8.c:991,1008)
    kOptAdamV8 = 3,      // Adam, reference src/full_cycle_v8.c:976-1008
    kOptSgdScaled = 4,   // w -= (lr / B) * g, unconditional (reference src/batch_gp_cuda.cu:137-140,193-194)
};

struct OptimizerArgs {
    int32_t kind;
    int32_t blades;
    double learning_rate;
    double beta1;
    double beta2;
    double epsilon;
    double gradient_scale;   // multiplies the summed gradient (V8 semantics)
    double batch_divisor;    // B for kOptSgdBatchGp and for the mean loss
    double bias1;            // 1 - beta1^step, computed on the host with libm pow
    double bias2;            // 1 - beta2^step
};

// ---------------------------------------------------------------------------
// Kernel launchers (kernels_direct.cu). All are asynchronous on `stream` and
// return the launch error. `records` points to kMaxCtas * kRecStride doubles.

// y = x * W (or W * x): inputs/outputs sample-major [batch][blades].
cudaError_t launch_forward(const SignPlan &plan, const double *inputs, const double *parameter,
                           double *outputs, size_t batch, cudaStream_t stream);

// Streaming full cycle. When `targets` is null the kernel only reduces the
// parameter VJP of `cotangents` (= the r of the loss) against `inputs`.
//   mode kCycle: r = fwd(x) - t (optionally stored to residuals_out), loss, VJP.
//   mode kVjp:   VJP of the given cotangents.
enum CycleMode : int32_t { kCycle = 0, kVjp = 1 };
cudaError_t launch_cycle(const SignPlan &plan, CycleMode mode, const double *inputs,
                         const double *targets_or_cotangents, const double *parameter,
                         double *residuals_out, size_t batch, double *records, int *ctas_used,
                         cudaStream_t stream);

// Sum `ctas` records in order; write gradient (may be null), loss sum (may be
// null), apply the optimizer to `parameter` (+ moments for Adam) transactionally
// and OR status bits into *status (may be null).
// A non-zero *status on entry blocks the optimizer update (failures chain);
// `step_counter` (may be null) is incremented on every committed update.
cudaError_t launch_finalize(const double *records, int ctas, const OptimizerArgs &opt,
                            double *gradient_out, double *loss_sum_out, double *parameter,
                            double *first_moment, double *second_moment, uint32_t *status,
                            cudaStream_t stream, unsigned long long *step_counter = nullptr);

// out[k] = sum over `count` records of record[k], in record order
// (accumulate != 0: out[k] += that sum).
cudaError_t launch_reduce_records(const double *records, int count, double *out, cudaStream_t stream,
                                  int accumulate = 0);

// Parameter VJP with one CTA per tile of vjp_tile_samples(blades) samples, so
// it needs exactly ceil(batch / tile) records; fails with cudaErrorInvalidValue
// (launching nothing) when that exceeds max_records.
size_t vjp_tile_samples(int blades);
cudaError_t launch_vjp_per_tile(const SignPlan &plan, const double *inputs, const double *cotangents, size_t batch,
                                double *records, int max_records, int *ctas_used, cudaStream_t stream);

// Finite check of a device array; ORs `bit` into *status when a value is not finite.
cudaError_t launch_check_finite(const double *values, size_t count, uint32_t bit,
                                uint32_t *status, cudaStream_t stream);

int device_sm_count();

// ---------------------------------------------------------------------------
// Representation path (kernels_rep.cu, representation.h): fused training pass
// through a D x D real matrix representation on FP64 tensor cores.
struct RepPlan;
struct RepDevice {
    uint8_t xm[64];
    uint8_t zm[64];
    int8_t sg[64];
    // Gather by blade group: the thread of group m (blades with x-mask m, c of
    // them) loads grp_blade[m][t] at step t and writes kept row r, column
    // grp_col[m][r], with input t negated when bit (r * 8 + t) of grp_neg[m] is
    // set. The load order is an edge colouring of (lane, bank) so each load
    // instruction of a warp touches distinct shared-memory banks.
    uint8_t grp_blade[16][8];
    uint8_t grp_col[16][8];
    uint64_t grp_neg[16];
    // Butterfly gather of the warp-specialised kernel. A group's S x S sign
    // block is a signed Walsh-Hadamard matrix: kept entry r of group m is
    //   alpha(r) * sum_c beta(c) (-1)^{c . phi(r)} x[A(m, c)]
    // over the coordinates c of the group's blades. Lane L (L = m for D = 16;
    // L = 8 * parity + m for D = 8, parity = sample & 1) loads blade
    // ws_blade[L][t] = A(m, t ^ delta_L) at step t, negates it when bit t of
    // ws_in_neg[L] is set, runs the in-register Walsh transform, and writes
    // transform output f to kept row ws_out_row[L][f], negated when bit f of
    // ws_out_neg[L] is set. delta_L is chosen so that every load step of a
    // half-warp covers 16 distinct double-banks of the unswizzled raw rows.
    uint8_t ws_blade[16][8];
    uint8_t ws_out_row[16][8];
    uint8_t ws_in_neg[16];
    uint8_t ws_out_neg[16];
    int32_t blades, D, S, side;
    int32_t raw_stride;  // row stride (doubles) of the staged raw tiles (= blades, unpadded)
    int32_t ws_ready;    // butterfly tables present (warp-specialised kernel usable)
    // D = 16, S = 4: the signed Pauli string J = P(x = 12, z = 4) (J^2 = -1)
    // commutes with every rho(e_A). J is then a complex structure on the D
    // columns (pairs m, m ^ 12, m < 8, sign -1 for m >= 4) that every W' and
    // every rho(e_A) respects, so the GEMMs are 8 x 8 complex products and the
    // warp-specialised kernel runs them as three real products each (3M).
    int32_t cplx;
};
bool make_rep_device(RepDevice *out, const RepPlan &plan);
// True when a tensor-core kernel exists for the plan's (D, S).
bool rep_supported(const RepDevice &rep);
// Same record contract as launch_cycle(kCycle) without residual output.
cudaError_t launch_rep_cycle(const RepDevice &rep, const double *inputs, const double *targets,
                             const double *parameter, size_t batch, double *records, int *ctas_used,
                             cudaStream_t stream);
// Parameter VJP of output cotangents through the representation (record
// contract of launch_cycle(kVjp)); needs 16-byte aligned inputs and cotangents.
bool rep_vjp_supported(const RepDevice &rep, const double *inputs, const double *cotangents);
cudaError_t launch_rep_vjp(const RepDevice &rep, const double *inputs, const double *cotangents, size_t batch,
                           double *records, int *ctas_used, cudaStream_t stream);
// Forward y = x W (or W x) through the representation; needs 16-byte aligned
// inputs and outputs (outputs may equal inputs, but must not overlap them otherwise).
bool rep_forward_supported(const RepDevice &rep, const double *inputs, const double *outputs);
cudaError_t launch_rep_forward(const RepDevice &rep, const double *inputs, const double *parameter, double *outputs,
                               size_t batch, cudaStream_t stream);
// A parameter multivector given as a term list, W = sum_t value_t e_{blade[t]}
// (repeated blades add up): value_t = coeff[t] when `values` is null, else
// scale[t] * values[t] with `values` a device array of `terms` doubles.
// Passed to kernels by value.
struct TermParameter {
    double coeff[64];
    const double *values;
    int8_t scale[64];
    uint8_t blade[64];
    int32_t terms;
};
cudaError_t launch_rep_forward_terms(const RepDevice &rep, const double *inputs, const TermParameter &parameter,
                                     double *outputs, size_t batch, cudaStream_t stream);
// One pass of the MSE-SGD step: residuals[s] = (x_s W or W x_s) - targets[s],
// the product computed with the arithmetic of launch_rep_forward (so targets
// equal to its outputs give exactly zero), and the records of launch_rep_vjp
// applied to those residuals (the same values, bit for bit); inputs, targets
// and residuals 16-byte aligned.
bool rep_sgd_supported(const RepDevice &rep, const double *inputs, const double *targets, const double *residuals);
cudaError_t launch_rep_mse_pass(const RepDevice &rep, const double *inputs, const double *parameter,
                                const double *targets, double *residuals, size_t batch, double *records,
                                int *ctas_used, cudaStream_t stream);
// Representation tables for (dimension, signature, side), built once and cached;
// null when the algebra has no warp-specialised representation kernel (n < 5).
const RepDevice *cached_rep_device(uint8_t dimension, const int8_t *signature, bool parameter_on_left);

}  // namespace geo
