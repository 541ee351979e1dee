// Shared declarations of the MoE (SwitchGLU) path.
#pragma once

#include "q38_internal.h"

namespace q38 {

// One tile of a grouped expert product: expert, block of weight rows, and a run of up to
// 32, 64 or 128 consecutive expert-sorted (token, slot) pairs starting at p0.
struct MoeTile {
    int e, rb, p0, np;
};

struct GroupedProblem {
    const void* x;       // activations in sorted pair order, permuted for the weights' bits, [pairs, K]
    int pairs, K;
    const uint32_t* w0;  // codes of the first 64-row box of a tile (gate, or down)
    const uint32_t* w1;  // codes of the second box (up, or down again)
    const void *s0, *s1, *b0, *b1;
    int E, rows_per_expert;
    const MoeTile* tiles;
    const int* ntiles;   // device
    int max_tiles;       // host bound on *ntiles
    void* out;
    int out_ld;
    int xr;              // longest run of pairs in a tile: 32, 64 or 128
};

q38_status grouped_gate_up(q38_ctx* ctx, const GroupedProblem& p, int bits);
q38_status grouped_down(q38_ctx* ctx, const GroupedProblem& p, int bits);
// xs[j] = permute(x[perm[j] / top_k]) for j < min(pairs, *valid) (valid: device count of
// pairs with an expert, i.e. offsets[E] of the sort).
q38_status moe_gather_launch(q38_ctx* ctx, const void* x, int H, const int32_t* perm, int pairs, int top_k,
                             const int32_t* valid, void* xs, int bits);

}  // namespace q38
