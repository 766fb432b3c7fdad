// Host build of the graph runtime's correctly rounded exp and tanh (crmath.h):
// reads binary64 arguments from argv[1], writes four results per argument to
// argv[2]: exp, tanh, exp on its fixed-point path, tanh on its fixed-point path
// (the latter two only where that path applies, else the plain function).
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

#include "crmath.h"

int main(int argc, char **argv) {
    if (argc != 3) return 2;
    FILE *f = fopen(argv[1], "rb");
    if (!f) return 2;
    fseek(f, 0, SEEK_END);
    const long n = ftell(f) / 8;
    fseek(f, 0, SEEK_SET);
    double *x = (double *)malloc((size_t)(n > 0 ? n : 1) * 8);
    if ((long)fread(x, 8, (size_t)n, f) != n) return 2;
    fclose(f);
    FILE *o = fopen(argv[2], "wb");
    if (!o) return 2;
    for (long i = 0; i < n; ++i) {
        const double a = fabs(x[i]);
        double r[4] = {geo::cr::exp(x[i]), geo::cr::tanh(x[i]), 0.0, 0.0};
        r[2] = (a >= 0x1p-54 && a < 746.0) ? geo::cr::exp_accurate(x[i]) : r[0];
        r[3] = (a >= 0x1p-27 && a < 19.1) ? geo::cr::tanh_accurate(x[i]) : r[1];
        fwrite(r, 8, 4, o);
    }
    fclose(o);
    free(x);
    return 0;
}
