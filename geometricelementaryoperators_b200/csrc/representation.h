// representation.h -- real matrix representations of Cl(p,q) built from
// signed Pauli strings, used to turn a fixed-parameter geometric product into
// a small dense GEMM.
//
// A Pauli string (x, z) on d qubits is the 2^d x 2^d matrix
//   P(x, z)[i][j] = [i == j ^ x] * (-1)^popcount(z & j)
// (a signed permutation). P(x,z)^2 = (-1)^popcount(x & z) I, and two strings
// anticommute iff popcount(z1 & x2) + popcount(z2 & x1) is odd. Choosing n
// pairwise-anticommuting, independent strings gamma_k with gamma_k^2 =
// signature[k] gives a faithful representation rho of Cl(p,q); the blade e_A
// (axes in increasing order) maps to rho(e_A) = gamma_a1 gamma_a2 ... =
// sign_A P(x_A, z_A).
//
// Right product y = x W:  rho(y) = rho(x) rho(W). Keeping only a set R of S
// rows of rho(x) loses nothing when the S*D kept entries determine x; the
// search below picks strings whose x-masks span all of Z_2^d, so S*D = 2^n and
// the map P: x -> rows R of rho(x) is square with P^T P = S I (every blade
// lands once in every kept row with sign +-1). Then per sample
//   Y' = X' W'   (S x D times D x D),   W' = rho(W)
// replaces the 2^n x 2^n Cayley product, and the training step only needs
//   R' = Y' - P(t),   loss = |R'|^2 / (2S),   G' = sum_s X'^T R',
//   g_A = <G', rho(e_A)> / S.
// Left product y = W x uses columns instead of rows: X'_L = (rho(x)[:, R])^T,
// W'_L = rho(W)^T, g_A = <G', rho(e_A)^T> / S.
//
// Cost per sample: S*D*D multiply-adds per GEMM (Cl(3,3): 8*8*8 = 512,
// Cl(6,0): 4*16*16 = 1024) instead of 4^n = 4096, plus the signed gathers.
#pragma once

#include <stdint.h>

namespace geo {

struct RepPlan {
    int32_t valid;
    int32_t dimension;
    int32_t blades;      // N = 2^n
    int32_t D;           // matrix size 2^d
    int32_t S;           // kept rows (right) / columns (left); S * D == N
    int32_t c;           // blades per kept entry (== S)
    int32_t side;        // 0: parameter on the right, 1: on the left
    int32_t reserved;
    uint8_t xm[64];      // blade -> x-mask of its Pauli string
    uint8_t zm[64];      // blade -> z-mask
    int8_t sg[64];       // blade -> overall sign
    uint8_t rows[16];    // kept rows (right) / columns (left)
    // Gather table: kept entry e = r * D + k receives sum_t gs[e][t] * x[gb[e][t]]
    uint8_t gb[64][8];
    int8_t gs[64][8];
};

// Builds the representation for (dimension, signature, side). Returns false
// when no string set with S * D == 2^n is found (the caller then uses the
// direct Cayley-matrix kernels). Self-checks the Clifford relations against
// the reference sign rule and P^T P = S I before returning true.
bool make_rep_plan(RepPlan *out, uint8_t dimension, const int8_t *signature, int side);

// Host-side reference of the representation maps (used by the self-check and
// by tests): dense rho(e_A) entry, the kept-entry matrix P, and W'.
int rep_entry(const RepPlan &p, int blade, int i, int j);

// Tables of the pairwise product y = a b (both operands vary) through the
// representation, for the n = 6 algebras with D = 16, S = 4 (right-side plan):
// Y' = A' rho(b), A' = S kept rows of rho(a), 1024 multiply-adds instead of 4096.
//
// The blades with x-mask 0 form K = {0, k1, k2, k1 ^ k2}; with z1, z2 their z-masks
// extended to a basis z1..z4 of GF(2)^4, the index space is relabelled by
// u = T j, (T j)_i = popc(z_i & j) mod 2, so z . j = z' . u with z' the
// coordinates of z in that basis. Then k1, k2 have z' = e0, e1, a group g (the
// four blades of one x-mask, relabelled g = T x) is B0 ^ {0, k1, k2, k1 ^ k2} with
// z'(B0) chosen free of the low two bits, and member c has z' = z'(B0) ^ c. The
// kept rows are T^-1 {0, 1, 2, 3}. Lane l (kept row l) of a product forms
//   Ah[m] = sum_c (-1)^{xa[m][c] + popc(c & l)} a[blade[m][c]]
//   bt_g  = Walsh transform over c of (-1)^{xb[g][c] + popc(c & l)} b[blade[g][c]]
//   Yh[u] = sum_g Ah[g ^ u] (-1)^{chi(g, u >> 2)} bt_g[u & 3]
// and a Walsh transform of Yh[g] over the four lanes leaves in lane c
// 4 (-1)^{post[g][c]} y[blade[g][c]] (sign words: bit 31).
struct PairTables {
    uint8_t blade[16][4];
    uint32_t xa[16][4], xb[16][4], post[16][4];
    uint32_t chi[16][3];  // sign words for u's high bits 1, 2, 3
};
// rev_a / rev_b multiply operand blade m by s(m, m) (the operands of the VJP products).
bool make_pair_tables(const RepPlan &p, const int8_t *signature, bool rev_a, bool rev_b, PairTables *out);
// The same arithmetic on the host (the check of the tables; y = a b).
void pair_product_host(const PairTables &t, const double *a, const double *b, double *y);

}  // namespace geo
