// The runtime's correctly rounded exp and tanh (geometricelementaryoperators_b200/
// csrc/crmath.h) under the C library's names. Linked (with -Bsymbolic) into
// oracle/_ref/libgeo_ref_crmath.so, a second build of the reference's own CPU
// sources whose graph nonlinearities call these instead of the C library's:
// the test comparison that separates the C library's rounding from everything
// else. Test infrastructure only.
#include "crmath.h"

extern "C" double exp(double x) noexcept { return geo::cr::exp(x); }
extern "C" double tanh(double x) noexcept { return geo::cr::tanh(x); }
