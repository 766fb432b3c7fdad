#ifndef recurrent_GEO_V8_MODEL_H
#define recurrent_GEO_V8_MODEL_H

#include <stddef.h>
#include <stdint.h>

#define recurrent_DIMENSION 2u
#define recurrent_BLADE_COUNT 4u
#define recurrent_PARAMETER_COUNT 2u

static const int8_t recurrent_signature[2] = {1, -1};
static const double recurrent_w[4] = {
    0.090929590749565053,
    0.067404152162525599,
    0.015890604531590004,
    -0.11044291555602335
};
static const double recurrent_u[4] = {
    -0.30382702918499926,
    -0.067457989245481423,
    -0.094732199145225571,
    -0.15517016121305366
};

#endif
