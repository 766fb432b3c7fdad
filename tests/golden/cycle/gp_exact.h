#ifndef gp_exact_GEO_V8_MODEL_H
#define gp_exact_GEO_V8_MODEL_H

#include <stddef.h>
#include <stdint.h>

#define gp_exact_DIMENSION 2u
#define gp_exact_BLADE_COUNT 4u
#define gp_exact_PARAMETER_COUNT 1u

static const int8_t gp_exact_signature[2] = {1, 1};
static const double gp_exact_w[4] = {
    0.75,
    -1.25,
    0.5,
    1
};

#endif
