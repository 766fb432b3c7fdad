// geo_cycle_b200 -- command line of the geo_cycle model runner on libgeo_b200
// (same commands and output as the reference tool tools/geo_cycle.c).
#include "geo/geo_cycle_b200.h"

int main(int argc, char **argv) { return geo_b200_cycle_main(argc, argv); }
