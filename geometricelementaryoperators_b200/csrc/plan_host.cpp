// plan_host.cpp -- host-side routing/sign plans (integer, bit-exact).
//
// Exported C entry points:
//   geo_batch_gp_abi_version, geo_batch_gp_plan_init      (reference src/batch_gp.c:65-105)
//   geo_operator_abi_version, geo_operator_gradient_abi_version,
//   geo_operator_blade_count, geo_operator_gp_sign,
//   geo_operator_plan_fixed_blade_i32, geo_operator_plan_sparse_i32
//                                                          (reference src/operator_kernel.c:98-189)
// Internal: the baked SignPlan consumed by the sm_100a kernels.
#include <cstring>

#include "geo_internal.h"

namespace geo {

bool dimension_valid(unsigned dimension) {
    return dimension >= 1u && dimension <= (unsigned)kMaxDim;
}

bool signature_valid(const int8_t *signature, unsigned dimension) {
    if (signature == nullptr || !dimension_valid(dimension)) return false;
    for (unsigned a = 0; a < dimension; ++a) {
        if (signature[a] != 1 && signature[a] != -1) return false;
    }
    return true;
}

int sign_rule(uint8_t left, uint8_t right, const int8_t *signature, uint8_t dimension) {
    int s = 1;
    for (unsigned a = 0; a < dimension; ++a) {
        if ((left >> a) & 1u) {
            const unsigned lower = (unsigned)right & ((1u << a) - 1u);
            if (__builtin_popcount(lower) & 1) s = -s;
            if ((right >> a) & 1u) s *= signature[a];
        }
    }
    return s;
}

bool make_sign_plan(SignPlan *out, uint8_t dimension, const int8_t *signature,
                    int parameter_on_left) {
    if (out == nullptr || !signature_valid(signature, dimension)) return false;
    std::memset(out, 0, sizeof(*out));
    const unsigned blades = 1u << dimension;
    out->dimension = dimension;
    out->blades = (int32_t)blades;
    out->parameter_on_left = parameter_on_left != 0;
    for (unsigned i = 0; i < blades; ++i) {
        uint64_t bits = 0;
        for (unsigned p = 0; p < blades; ++p) {
            const int s = parameter_on_left ? sign_rule((uint8_t)p, (uint8_t)i, signature, dimension)
                                            : sign_rule((uint8_t)i, (uint8_t)p, signature, dimension);
            if (s < 0) bits |= (uint64_t)1 << p;
        }
        out->neg[i] = bits;
    }
    return true;
}

}  // namespace geo

using geo::dimension_valid;
using geo::signature_valid;

extern "C" uint32_t geo_batch_gp_abi_version(void) { return GEO_BATCH_GP_ABI_VERSION; }

extern "C" geo_batch_gp_status_t geo_batch_gp_plan_init(geo_batch_gp_plan_t *plan, uint8_t dimension,
                                                        const int8_t *signature) {
    if (plan == nullptr || signature == nullptr) return GEO_BATCH_GP_INVALID_ARGUMENT;
    if (!dimension_valid(dimension)) return GEO_BATCH_GP_UNSUPPORTED_DIMENSION;
    if (!signature_valid(signature, dimension)) return GEO_BATCH_GP_INVALID_ARGUMENT;
    std::memset(plan, 0, sizeof(*plan));
    const unsigned blades = 1u << dimension;
    plan->abi_version = GEO_BATCH_GP_ABI_VERSION;
    plan->dimension = dimension;
    std::memcpy(plan->signature, signature, dimension);
    plan->blade_count = (uint16_t)blades;
    plan->term_count = (uint16_t)(blades * blades);
    unsigned term = 0;
    for (unsigned l = 0; l < blades; ++l) {
        for (unsigned r = 0; r < blades; ++r, ++term) {
            plan->left_blade[term] = (uint8_t)l;
            plan->right_blade[term] = (uint8_t)r;
            plan->output_blade[term] = (uint8_t)(l ^ r);
            plan->sign[term] = (int8_t)geo::sign_rule((uint8_t)l, (uint8_t)r, signature, dimension);
        }
    }
    return GEO_BATCH_GP_OK;
}

extern "C" uint32_t geo_operator_abi_version(void) { return GEO_OPERATOR_ABI_VERSION; }
extern "C" uint32_t geo_operator_gradient_abi_version(void) { return GEO_OPERATOR_GRADIENT_ABI_VERSION; }

extern "C" size_t geo_operator_blade_count(uint8_t dimension) {
    return dimension_valid(dimension) ? (size_t)1u << dimension : 0u;
}

extern "C" int geo_operator_gp_sign(uint8_t left_blade, uint8_t right_blade, const int8_t *signature,
                                    uint8_t dimension) {
    if (!signature_valid(signature, dimension)) return 0;
    return geo::sign_rule(left_blade, right_blade, signature, dimension);
}

extern "C" geo_operator_status_t geo_operator_plan_sparse_i32(geo_operator_plan_i32_t *plan, uint8_t dimension,
                                                             const int8_t *signature, geo_operator_side_t side,
                                                             const geo_operator_term_i32_t *terms,
                                                             size_t term_count) {
    if (plan == nullptr || terms == nullptr) return GEO_OPERATOR_INVALID_ARGUMENT;
    if (!dimension_valid(dimension)) return GEO_OPERATOR_UNSUPPORTED_DIMENSION;
    if (!signature_valid(signature, dimension)) return GEO_OPERATOR_INVALID_ARGUMENT;
    if (side != GEO_OPERATOR_SIDE_LEFT && side != GEO_OPERATOR_SIDE_RIGHT) return GEO_OPERATOR_INVALID_ARGUMENT;
    if (term_count == 0u || term_count > GEO_OPERATOR_MAX_TERMS) return GEO_OPERATOR_TOO_MANY_TERMS;
    const size_t blades = (size_t)1u << dimension;
    std::memset(plan, 0, sizeof(*plan));
    plan->abi_version = GEO_OPERATOR_ABI_VERSION;
    plan->dimension = dimension;
    std::memcpy(plan->signature, signature, dimension);
    plan->kind = term_count == 1u ? GEO_OPERATOR_PLAN_FIXED_BLADE : GEO_OPERATOR_PLAN_SPARSE_FIXED_MULTIVECTOR;
    plan->side = (uint8_t)side;
    plan->term_count = (uint8_t)term_count;
    for (size_t t = 0; t < term_count; ++t) {
        bool bad = (size_t)terms[t].blade >= blades || terms[t].coefficient == 0;
        for (size_t u = 0; u < t && !bad; ++u) bad = terms[u].blade == terms[t].blade;
        if (bad) {
            std::memset(plan, 0, sizeof(*plan));
            return GEO_OPERATOR_INVALID_ARGUMENT;
        }
        plan->terms[t] = terms[t];
    }
    return GEO_OPERATOR_OK;
}

extern "C" geo_operator_status_t geo_operator_plan_fixed_blade_i32(geo_operator_plan_i32_t *plan, uint8_t dimension,
                                                                  const int8_t *signature, geo_operator_side_t side,
                                                                  uint8_t blade, int32_t coefficient) {
    geo_operator_term_i32_t term;
    term.blade = blade;
    term.coefficient = coefficient;
    return geo_operator_plan_sparse_i32(plan, dimension, signature, side, &term, 1u);
}
