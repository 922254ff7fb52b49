// skinny.cuh — the tensor-core GEMM of multi-stream decode: up to 64 token
// rows against BF16 weight matrices, Y[token][feature] = x_token . W[feature].
//
// Roles are swapped with respect to the prefill GEMM: the weight rows are
// the MMA's A operand (M = 128 features per tile, streamed from HBM once per
// step), the tokens are B (N = 128 = 64 token rows hi + the same 64 rows lo,
// the F32 activations split into two BF16 planes, re-read from L2). The
// accumulator column j holds x_hi[j].W and column 64 + j holds x_lo[j].W.
#pragma once
#include <cstdint>
#include <vector>
#include <cuda.h>

namespace ds {

constexpr int SK_TOK = 64;  // token rows per tile (B = 2 x 64 rows)

// A plane tensor holds hi rows [0, lo_off) and lo rows [lo_off, 2 lo_off);
// a tile reads hi rows b_row .. b_row+63 and lo rows lo_off + b_row ...
struct SkTile {
    int amap;    // weight map (and output slot) index, 0..3
    int a_row;   // first weight row (SwiGLU: first gate row)
    int a_row2;  // SwiGLU: first up row (in map amap2)
    int amap2;   // SwiGLU: weight map of the up rows
    int kind;    // activation plane map 0/1 (and SwiGLU output slot)
    int b_row;   // first token row in the plane
    int n_tok;   // valid token rows (<= 64)
    int out_col; // first output feature (PLAIN) / intermediate index (SwiGLU)
    int kb;      // K blocks of 64 in this tile
    // split K (PLAIN only): this tile covers K blocks k0 .. k0+kb-1 and
    // writes part `split` of nsplit of output tile `otile` to the part
    // buffer; the kernel that reads the output sums the parts in order
    int k0, split, nsplit, otile;
};

struct SkGemm {
    CUtensorMap a[4];  // weights, box 64 x 128 (PLAIN) or 64 x 64 (SwiGLU halves)
    CUtensorMap b[2];  // activation planes, box 64 x 64
    int lo_off[2];
    const SkTile *tiles;
    const int *n_tiles;
    // PLAIN: out[amap][(b_row + j) * out_ld + out_col + r] (+ resid, same index)
    float *out[4];
    const float *resid[4];
    int out_ld[4], out_n[4];
    // SwiGLU: h planes [kind] rows b_row + j, columns out_col + i (hi, lo)
    uint16_t *h_hi[2], *h_lo[2];
    int h_ld[2];
    // split K: parts [otile][split][64 tokens][128 rows]
    float *ws;
    int max_split;
    unsigned *err;
};

constexpr int SK_MAX_SPLIT = 20;

// Output (token, feature) of a split-K GEMM: the sum of its parts in split
// order (feature = output tile * 128 + row).
__device__ __forceinline__ float sk_part_sum(const float *ws, int max_split, int nsplit, int tok, int f) {
    const float *p = ws + ((size_t)(f >> 7) * max_split * 64 + tok) * 128 + (f & 127);
    float v = p[0];
    for (int s = 1; s < nsplit; s++) v = __fadd_rn(v, p[(size_t)s * 64 * 128]);
    return v;
}

// Appends tile t split into nsplit K ranges (output tile id otile).
inline void sk_push_split(std::vector<SkTile> &v, SkTile t, int nsplit, int otile) {
    if (nsplit > t.kb) nsplit = t.kb;
    if (nsplit <= 1) {
        v.push_back(t);
        return;
    }
    const int kb = t.kb;
    for (int s = 0; s < nsplit; s++) {
        SkTile u = t;
        u.k0 = kb * s / nsplit;
        u.kb = kb * (s + 1) / nsplit - u.k0;
        u.split = s;
        u.nsplit = nsplit;
        u.otile = otile;
        v.push_back(u);
    }
}

}  // namespace ds
