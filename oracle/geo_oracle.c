/*
 * geo_oracle.c -- CPU oracle (test infrastructure only; see geo_oracle.h).
 *
 * A restatement, in this project's own code, of the reference CPU path for
 * batched geometric products (reference src/batch_gp.c), the dense and sparse
 * per-multivector operators (reference src/operator_kernel.c) and the V8
 * optimizer update (reference src/full_cycle_v8.c). The loop nests and the
 * accumulation order mirror the reference so that results are bit-identical
 * when both are compiled by gcc for x86-64 without FMA contraction.
 */
#include "geo_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define ORC_MAX_DIM 6u
#define ORC_MAX_BLADES 64u
#define ORC_MAX_TERMS 4096u
#define ORC_BATCH_ABI 0x00010000u

enum { ORC_OK = 0, ORC_INVALID = 1, ORC_UNSUPPORTED = 2, ORC_NUMERIC = 3 };

/* Same byte layout as geo_batch_gp_plan_t (reference include/geo/batch_gp.h:23-33). */
typedef struct {
    uint32_t abi_version;
    uint8_t dimension;
    int8_t signature[ORC_MAX_DIM];
    uint16_t blade_count;
    uint16_t term_count;
    uint8_t left_blade[ORC_MAX_TERMS];
    uint8_t right_blade[ORC_MAX_TERMS];
    uint8_t output_blade[ORC_MAX_TERMS];
    int8_t sign[ORC_MAX_TERMS];
} orc_plan_t;

_Static_assert(sizeof(orc_plan_t) == 16400u, "plan layout must match the reference ABI");

static int dim_ok(uint8_t n) { return n >= 1u && n <= ORC_MAX_DIM; }

static int sig_ok(const int8_t *s, uint8_t n) {
    uint8_t a;
    if (s == NULL || !dim_ok(n)) return 0;
    for (a = 0u; a < n; ++a) {
        if (s[a] != 1 && s[a] != -1) return 0;
    }
    return 1;
}

static unsigned bits_set(unsigned v) {
    unsigned c = 0u;
    for (; v != 0u; v &= v - 1u) ++c;
    return c;
}

/*
 * Sign of e_left e_right: moving each basis vector of `left` past the lower
 * basis vectors of `right` flips the sign once per crossing; a shared axis
 * contracts with its metric entry. reference src/batch_gp.c:29-45.
 */
static int sign_rule(uint8_t left, uint8_t right, const int8_t *signature, uint8_t n) {
    int s = 1;
    uint8_t a;
    for (a = 0u; a < n; ++a) {
        if ((left >> a) & 1u) {
            if (bits_set((unsigned)right & ((1u << a) - 1u)) & 1u) s = -s;
            if ((right >> a) & 1u) s *= signature[a];
        }
    }
    return s;
}

int orc_gp_sign(uint8_t left, uint8_t right, const int8_t *signature, uint8_t dimension) {
    /* reference src/operator_kernel.c:119 returns 0 for an invalid signature */
    if (!sig_ok(signature, dimension)) return 0;
    return sign_rule(left, right, signature, dimension);
}

static int finite_all(const double *v, size_t count) {
    size_t i;
    if (v == NULL) return 0;
    for (i = 0u; i < count; ++i) {
        if (!isfinite(v[i])) return 0;
    }
    return 1;
}

static int plan_ok(const orc_plan_t *p) {
    size_t blades;
    if (p == NULL) return 0;
    blades = (size_t)1u << p->dimension;
    return p->abi_version == ORC_BATCH_ABI && sig_ok(p->signature, p->dimension) &&
        p->blade_count == blades && p->term_count == blades * blades;
}

/* reference src/batch_gp.c:69-105 */
int orc_batch_plan_init(void *plan_bytes, uint8_t dimension, const int8_t *signature) {
    orc_plan_t *p = (orc_plan_t *)plan_bytes;
    size_t l, r, t = 0u, blades;
    if (p == NULL || signature == NULL) return ORC_INVALID;
    if (!dim_ok(dimension)) return ORC_UNSUPPORTED;
    if (!sig_ok(signature, dimension)) return ORC_INVALID;
    blades = (size_t)1u << dimension;
    memset(p, 0, sizeof(*p));
    p->abi_version = ORC_BATCH_ABI;
    p->dimension = dimension;
    memcpy(p->signature, signature, dimension);
    p->blade_count = (uint16_t)blades;
    p->term_count = (uint16_t)(blades * blades);
    for (l = 0u; l < blades; ++l) {
        for (r = 0u; r < blades; ++r, ++t) {
            p->left_blade[t] = (uint8_t)l;
            p->right_blade[t] = (uint8_t)r;
            p->output_blade[t] = (uint8_t)(l ^ r);
            p->sign[t] = (int8_t)sign_rule((uint8_t)l, (uint8_t)r, signature, dimension);
        }
    }
    return ORC_OK;
}

/*
 * Term-major batched product: for every plan term, multiplier = w[param] *
 * sign, then out[s, o] += in[s, i] * multiplier over all samples.
 * reference src/batch_gp.c:107-141.
 */
int orc_batch_forward(const void *plan_bytes, const double *inputs, size_t batch_size,
                      const double *parameter, int parameter_on_left, double *outputs) {
    const orc_plan_t *p = (const orc_plan_t *)plan_bytes;
    size_t t, s, blades, values;
    if (!plan_ok(p) || batch_size == 0u || outputs == NULL) return ORC_INVALID;
    blades = p->blade_count;
    values = batch_size * blades;
    if (!finite_all(inputs, values) || !finite_all(parameter, blades)) return ORC_INVALID;
    memset(outputs, 0, values * sizeof(double));
    for (t = 0u; t < p->term_count; ++t) {
        const size_t in_b = parameter_on_left ? p->right_blade[t] : p->left_blade[t];
        const size_t par_b = parameter_on_left ? p->left_blade[t] : p->right_blade[t];
        const size_t out_b = p->output_blade[t];
        const double mult = parameter[par_b] * (double)p->sign[t];
        for (s = 0u; s < batch_size; ++s) {
            outputs[s * blades + out_b] += inputs[s * blades + in_b] * mult;
        }
    }
    return finite_all(outputs, values) ? ORC_OK : ORC_NUMERIC;
}

/*
 * Per term: sequential batch sum of in[s, i] * cot[s, o] from 0, then
 * g[param] += sign * sum. reference src/batch_gp.c:163-201.
 */
int orc_batch_vjp(const void *plan_bytes, const double *inputs, const double *cotangents,
                  size_t batch_size, int parameter_on_left, double *parameter_cotangent) {
    const orc_plan_t *p = (const orc_plan_t *)plan_bytes;
    size_t t, s, blades, values;
    if (!plan_ok(p) || batch_size == 0u || parameter_cotangent == NULL) return ORC_INVALID;
    blades = p->blade_count;
    values = batch_size * blades;
    if (!finite_all(inputs, values) || !finite_all(cotangents, values)) return ORC_INVALID;
    memset(parameter_cotangent, 0, blades * sizeof(double));
    for (t = 0u; t < p->term_count; ++t) {
        const size_t in_b = parameter_on_left ? p->right_blade[t] : p->left_blade[t];
        const size_t par_b = parameter_on_left ? p->left_blade[t] : p->right_blade[t];
        const size_t out_b = p->output_blade[t];
        const double sg = (double)p->sign[t];
        double acc = 0.0;
        for (s = 0u; s < batch_size; ++s) {
            acc += inputs[s * blades + in_b] * cotangents[s * blades + out_b];
        }
        parameter_cotangent[par_b] += sg * acc;
    }
    return finite_all(parameter_cotangent, blades) ? ORC_OK : ORC_NUMERIC;
}

/*
 * forward -> r = y - t, loss += 0.5 r r -> VJP(r) -> transactional candidate
 * check -> w -= lr * g / B -> mean_loss = loss / B (status NUMERIC if that is
 * not finite, after the update). reference src/batch_gp.c:237-308.
 */
int orc_batch_mse_sgd_step(const void *plan_bytes, const double *inputs, const double *targets,
                           size_t batch_size, double learning_rate, int parameter_on_left,
                           double *parameter, double *mean_loss) {
    const orc_plan_t *p = (const orc_plan_t *)plan_bytes;
    double grad[ORC_MAX_BLADES];
    double loss = 0.0;
    double *res;
    size_t i, blades, values;
    int st;
    if (!plan_ok(p) || batch_size == 0u || !isfinite(learning_rate) || learning_rate <= 0.0 ||
        mean_loss == NULL) {
        return ORC_INVALID;
    }
    blades = p->blade_count;
    values = batch_size * blades;
    if (!finite_all(inputs, values) || !finite_all(targets, values) ||
        !finite_all(parameter, blades)) {
        return ORC_INVALID;
    }
    res = (double *)malloc(values * sizeof(double));
    if (res == NULL) return ORC_INVALID;
    st = orc_batch_forward(p, inputs, batch_size, parameter, parameter_on_left, res);
    if (st != ORC_OK) { free(res); return st; }
    for (i = 0u; i < values; ++i) {
        res[i] -= targets[i];
        loss += 0.5 * res[i] * res[i];
    }
    st = orc_batch_vjp(p, inputs, res, batch_size, parameter_on_left, grad);
    if (st != ORC_OK) { free(res); return st; }
    for (i = 0u; i < blades; ++i) {
        const double cand = parameter[i] - learning_rate * grad[i] / (double)batch_size;
        if (!isfinite(cand)) { free(res); return ORC_NUMERIC; }
    }
    for (i = 0u; i < blades; ++i) {
        parameter[i] -= learning_rate * grad[i] / (double)batch_size;
    }
    *mean_loss = loss / (double)batch_size;
    free(res);
    return isfinite(*mean_loss) ? ORC_OK : ORC_NUMERIC;
}

/* reference src/operator_kernel.c:412-447: left-blade-major, zero left terms skipped */
int orc_gp_f64(uint8_t dimension, const int8_t *signature, const double *left,
               const double *right, double *output) {
    double acc[ORC_MAX_BLADES];
    size_t l, r, blades;
    if (left == NULL || right == NULL || output == NULL) return 1;
    if (!dim_ok(dimension)) return 2;
    if (!sig_ok(signature, dimension)) return 1;
    blades = (size_t)1u << dimension;
    memset(acc, 0, sizeof(acc));
    for (l = 0u; l < blades; ++l) {
        if (left[l] == 0.0) continue;
        for (r = 0u; r < blades; ++r) {
            const int s = sign_rule((uint8_t)l, (uint8_t)r, signature, dimension);
            acc[l ^ r] += left[l] * right[r] * (double)s;
        }
    }
    memcpy(output, acc, blades * sizeof(double));
    return 0;
}

/* reference src/operator_kernel.c:449-492 */
int orc_gp_f64_jvp(uint8_t dimension, const int8_t *signature, const double *left,
                   const double *right, const double *left_tangent,
                   const double *right_tangent, double *output_tangent) {
    double acc[ORC_MAX_BLADES];
    size_t l, r, blades;
    if (left == NULL || right == NULL || left_tangent == NULL || right_tangent == NULL ||
        output_tangent == NULL) {
        return 1;
    }
    if (!dim_ok(dimension)) return 2;
    if (!sig_ok(signature, dimension)) return 1;
    blades = (size_t)1u << dimension;
    memset(acc, 0, sizeof(acc));
    for (l = 0u; l < blades; ++l) {
        for (r = 0u; r < blades; ++r) {
            const int s = sign_rule((uint8_t)l, (uint8_t)r, signature, dimension);
            acc[l ^ r] += (left_tangent[l] * right[r] + left[l] * right_tangent[r]) * (double)s;
        }
    }
    memcpy(output_tangent, acc, blades * sizeof(double));
    return 0;
}

/* reference src/operator_kernel.c:494-539 */
int orc_gp_f64_vjp(uint8_t dimension, const int8_t *signature, const double *left,
                   const double *right, const double *output_cotangent,
                   double *left_cotangent, double *right_cotangent) {
    double lacc[ORC_MAX_BLADES];
    double racc[ORC_MAX_BLADES];
    size_t l, r, blades;
    if (left == NULL || right == NULL || output_cotangent == NULL || left_cotangent == NULL ||
        right_cotangent == NULL || left_cotangent == right_cotangent) {
        return 1;
    }
    if (!dim_ok(dimension)) return 2;
    if (!sig_ok(signature, dimension)) return 1;
    blades = (size_t)1u << dimension;
    memset(lacc, 0, sizeof(lacc));
    memset(racc, 0, sizeof(racc));
    for (l = 0u; l < blades; ++l) {
        for (r = 0u; r < blades; ++r) {
            const int s = sign_rule((uint8_t)l, (uint8_t)r, signature, dimension);
            const double c = output_cotangent[l ^ r] * (double)s;
            lacc[l] += c * right[r];
            racc[r] += c * left[l];
        }
    }
    memcpy(left_cotangent, lacc, blades * sizeof(double));
    memcpy(right_cotangent, racc, blades * sizeof(double));
    return 0;
}

/* Sign of (source, fixed) on the plan's side. reference src/operator_kernel.c:88-96 */
static int side_sign(int side, uint8_t source, uint8_t fixed, const int8_t *sig, uint8_t n) {
    return side == 0 ? sign_rule(source, fixed, sig, n) : sign_rule(fixed, source, sig, n);
}

static int sparse_ok(uint8_t n, const int8_t *sig, int side, const uint8_t *blades,
                     size_t terms) {
    size_t i, j;
    if (!dim_ok(n) || !sig_ok(sig, n) || (side != 0 && side != 1) || blades == NULL) return 0;
    if (terms == 0u || terms > ORC_MAX_BLADES) return 0;
    for (i = 0u; i < terms; ++i) {
        if ((size_t)blades[i] >= ((size_t)1u << n)) return 0;
        for (j = 0u; j < i; ++j) {
            if (blades[j] == blades[i]) return 0;
        }
    }
    return 1;
}

/* reference src/operator_kernel.c:191-220 */
int orc_sparse_apply(uint8_t n, const int8_t *sig, int side, const uint8_t *blades,
                     const int32_t *coefficients, size_t terms, const double *input,
                     double *output) {
    double acc[ORC_MAX_BLADES];
    size_t src, t, count;
    if (!sparse_ok(n, sig, side, blades, terms) || coefficients == NULL || input == NULL ||
        output == NULL) {
        return 1;
    }
    count = (size_t)1u << n;
    memset(acc, 0, sizeof(acc));
    for (src = 0u; src < count; ++src) {
        const double v = input[src];
        if (v == 0.0) continue;
        for (t = 0u; t < terms; ++t) {
            const int s = side_sign(side, (uint8_t)src, blades[t], sig, n);
            acc[src ^ blades[t]] += v * (double)(s * coefficients[t]);
        }
    }
    memcpy(output, acc, count * sizeof(double));
    return 0;
}

/* reference src/operator_kernel.c:222-254 */
int orc_sparse_apply_parametric(uint8_t n, const int8_t *sig, int side, const uint8_t *blades,
                                const double *parameters, size_t terms, const double *input,
                                double *output) {
    double acc[ORC_MAX_BLADES];
    size_t src, t, count;
    if (!sparse_ok(n, sig, side, blades, terms) || parameters == NULL || input == NULL ||
        output == NULL) {
        return 1;
    }
    count = (size_t)1u << n;
    memset(acc, 0, sizeof(acc));
    for (src = 0u; src < count; ++src) {
        const double v = input[src];
        if (v == 0.0) continue;
        for (t = 0u; t < terms; ++t) {
            const int s = side_sign(side, (uint8_t)src, blades[t], sig, n);
            acc[src ^ blades[t]] += v * parameters[t] * (double)s;
        }
    }
    memcpy(output, acc, count * sizeof(double));
    return 0;
}

/* reference src/operator_kernel.c:256-278 */
int orc_sparse_apply_vjp(uint8_t n, const int8_t *sig, int side, const uint8_t *blades,
                         const int32_t *coefficients, size_t terms,
                         const double *output_cotangent, double *input_cotangent) {
    double acc[ORC_MAX_BLADES];
    size_t src, t, count;
    if (!sparse_ok(n, sig, side, blades, terms) || coefficients == NULL ||
        output_cotangent == NULL || input_cotangent == NULL) {
        return 1;
    }
    count = (size_t)1u << n;
    memset(acc, 0, sizeof(acc));
    for (src = 0u; src < count; ++src) {
        for (t = 0u; t < terms; ++t) {
            const int s = side_sign(side, (uint8_t)src, blades[t], sig, n);
            acc[src] += output_cotangent[src ^ blades[t]] * (double)(s * coefficients[t]);
        }
    }
    memcpy(input_cotangent, acc, count * sizeof(double));
    return 0;
}

/* reference src/operator_kernel.c:280-334 */
int orc_sparse_apply_parametric_vjp(uint8_t n, const int8_t *sig, int side,
                                    const uint8_t *blades, const double *parameters,
                                    size_t terms, const double *input,
                                    const double *output_cotangent, double *input_cotangent,
                                    double *parameter_cotangent) {
    double iacc[ORC_MAX_BLADES];
    double pacc[ORC_MAX_BLADES];
    size_t src, t, count;
    if (!sparse_ok(n, sig, side, blades, terms) || parameters == NULL || input == NULL ||
        output_cotangent == NULL || input_cotangent == NULL || parameter_cotangent == NULL) {
        return 1;
    }
    count = (size_t)1u << n;
    memset(iacc, 0, sizeof(iacc));
    memset(pacc, 0, sizeof(pacc));
    for (src = 0u; src < count; ++src) {
        for (t = 0u; t < terms; ++t) {
            const int s = side_sign(side, (uint8_t)src, blades[t], sig, n);
            const double c = output_cotangent[src ^ blades[t]];
            iacc[src] += c * parameters[t] * (double)s;
            pacc[t] += c * input[src] * (double)s;
        }
    }
    memcpy(input_cotangent, iacc, count * sizeof(double));
    memcpy(parameter_cotangent, pacc, terms * sizeof(double));
    return 0;
}

/* reference src/full_cycle_v8.c:942-1041 (single parameter node, no constraint) */
int orc_v8_optimizer_update(size_t count, int optimizer, double learning_rate, double beta1,
                            double beta2, double epsilon, double gradient_scale,
                            uint64_t step, const double *gradient_sum, double *value,
                            double *first_moment, double *second_moment) {
    double w[ORC_MAX_BLADES], m[ORC_MAX_BLADES], v[ORC_MAX_BLADES];
    double bias1 = 1.0, bias2 = 1.0;
    size_t b;
    if (count == 0u || count > ORC_MAX_BLADES || gradient_sum == NULL || value == NULL ||
        first_moment == NULL || second_moment == NULL) {
        return 1;
    }
    if ((optimizer != 1 && optimizer != 2) || !isfinite(learning_rate) || learning_rate <= 0.0 ||
        !isfinite(gradient_scale) || gradient_scale <= 0.0 ||
        !isfinite(beta1) || beta1 < 0.0 || beta1 >= 1.0 ||
        !isfinite(beta2) || beta2 < 0.0 || beta2 >= 1.0 ||
        !isfinite(epsilon) || epsilon <= 0.0) {
        return 1;
    }
    memcpy(w, value, count * sizeof(double));
    memcpy(m, first_moment, count * sizeof(double));
    memcpy(v, second_moment, count * sizeof(double));
    if (optimizer == 2) {
        bias1 = 1.0 - pow(beta1, (double)step);
        bias2 = 1.0 - pow(beta2, (double)step);
        if (!isfinite(bias1) || !isfinite(bias2) || bias1 <= 0.0 || bias2 <= 0.0) return 11;
    }
    for (b = 0u; b < count; ++b) {
        const double g = gradient_sum[b] * gradient_scale;
        double update;
        if (optimizer == 1) {
            update = g;
        } else {
            const double first = beta1 * m[b] + (1.0 - beta1) * g;
            const double second = beta2 * v[b] + (1.0 - beta2) * g * g;
            if (!isfinite(first) || !isfinite(second)) return 11;
            m[b] = first;
            v[b] = second;
            update = (first / bias1) / (sqrt(second / bias2) + epsilon);
        }
        w[b] -= learning_rate * update;
        if (!isfinite(w[b])) return 11;
    }
    memcpy(value, w, count * sizeof(double));
    memcpy(first_moment, m, count * sizeof(double));
    memcpy(second_moment, v, count * sizeof(double));
    return 0;
}
