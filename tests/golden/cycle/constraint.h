#ifndef constraint_GEO_V8_MODEL_H
#define constraint_GEO_V8_MODEL_H

#include <stddef.h>
#include <stdint.h>

#define constraint_DIMENSION 3u
#define constraint_BLADE_COUNT 8u
#define constraint_PARAMETER_COUNT 1u

static const int8_t constraint_signature[3] = {1, 1, 1};
static const double constraint_r[8] = {
    0.87353138610459513,
    0.35738594577629013,
    -0.073306437871328414,
    -0.10300100827128782,
    -0.21969405412218032,
    0.084013140852192886,
    -0.19299110870148919,
    0.025805201475018382
};

#endif
