// rep_layout.h -- tile geometry and shared-memory layout of the
// warp-specialised representation kernel (kernels_rep.cu). Shared with the
// host-side layout check (tests/c/rep_check.cpp), which replays every shared
// memory access pattern of the kernel and requires 16 distinct double-banks
// per half-warp (a warp's 8-byte access is served as two half-warps).
#pragma once

#if defined(__CUDACC__)
#define GEO_LAYOUT_FN __host__ __device__ __forceinline__
#else
#define GEO_LAYOUT_FN inline
#endif

namespace geo {

constexpr int kWsThreads = 256;    // 8 warps per CTA
constexpr int kWsProducers = 128;  // warps 0-3: bulk loads and gathers
constexpr int kWsStages = 6;       // shared-memory stages per CTA

// Forward kernel (rep_fwd_kernel): a stage holds one x tile (8 KB), which is
// gathered in place, overwritten by Y', scattered back to raw y rows and
// stored from the same stage.
struct FwdPipe {
    static constexpr int STAGES = 8;        // shared-memory stages per CTA
    static constexpr int AHEAD = 4;         // tiles whose bulk loads are in flight
    // CTAs per SM (the 66 KB ring fits three; measured faster than 12 stages at
    // two CTAs per SM)
    static constexpr int CTAS_PER_SM = 3;
    static constexpr int LAG = 2;           // the scatter of tile k - LAG follows the gather of tile k
    // Bulk stores that may still be reading shared memory when a stage is
    // reloaded: the load of tile k + AHEAD reuses the stage of tile
    // k + AHEAD - STAGES, whose store was issued this many stores ago.
    static constexpr int STORE_PENDING = STAGES - 1 - LAG - AHEAD;
    static_assert(STORE_PENDING >= 0, "a stage is reloaded only after its store was issued");
};

// Fused MSE-SGD pass (rep_sgd_kernel): a stage holds the x tile (gathered to
// X' in place), the target tile (replaced in place by r = y - t, which a bulk
// copy stores) and a third tile that takes Y' from the consumers and then
// R' = P r from the producers. Iteration k of the producers gathers tile k,
// runs the residual phase of tile k - LAG and then issues the loads of tile
// k + AHEAD; iteration k of the consumers runs GEMM 1 of tile k and GEMM 2 of
// tile k - LAG.
struct SgdPipe {
    static constexpr int ARRAYS = 3;
    static constexpr int STAGES = 4;       // 24 KB stages: two CTAs per SM
    static constexpr int AHEAD = 2;        // tiles whose bulk loads are in flight
    static constexpr int LAG = 1;
    static constexpr int CTAS_PER_SM = 2;
    // The load of tile k + AHEAD (issued at the end of iteration k) reuses the
    // stage of tile k + AHEAD - STAGES, whose residual store was issued in
    // iteration k + AHEAD - STAGES + LAG: this many stores ago at most.
    static constexpr int STORE_PENDING = STAGES - AHEAD - LAG;
    static_assert(STORE_PENDING >= 0, "a stage is reloaded only after its store was issued");
};

template <int D, int S>
struct WsGeo {
    static constexpr int N = D * S;                // blades = doubles per sample
    static constexpr int ROWS = D == 16 ? 64 : 128;  // X' rows per tile
    static constexpr int TS = ROWS / S;            // samples per tile
    static constexpr int TILE = ROWS * D;          // doubles of one array (x or t) per stage
    static constexpr int STAGE = 2 * TILE;         // x tile + t tile (16 KB)
    static constexpr int GROUPS = ROWS / 8;        // 8-row groups of the GEMMs
    static constexpr int GPW = GROUPS / 4;         // groups per consumer warp
    static constexpr int SLOTS = kWsProducers / D; // sample slots of the producer threads
    static constexpr int PER = TS / SLOTS;         // samples per producer thread per tile
    static_assert(TILE == TS * N && PER * SLOTS == TS && GPW % 2 == 0, "tile shape");
};

// Position of entry (row, col) of a transformed tile (X' or T', D doubles per
// row). D = 16: the 4-column blocks of a row are XOR-permuted by
// f(row) = (row & 3) ^ ((row >> 2) & 1). D = 8: pairs of rows form 16-double
// units whose entries are XOR-permuted by 4 * (unit & 3) ^ 8 * ((unit >> 2) & 1),
// which may move an entry into the other row of its unit; the second term puts
// consecutive samples of S = 8 rows (four units each) in opposite halves.
template <int D>
GEO_LAYOUT_FN int ws_index(int row, int col) {
    if (D == 16) return row * 16 + (col ^ (4 * ((row & 3) ^ ((row >> 2) & 1))));
    const int unit = row >> 1;
    return 16 * unit + ((8 * (row & 1) + col) ^ (4 * (unit & 3)) ^ (8 * ((unit >> 2) & 1)));
}

}  // namespace geo
