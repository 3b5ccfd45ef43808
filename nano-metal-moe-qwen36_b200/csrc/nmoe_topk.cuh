// nmoe_topk.cuh -- warp-level top-k of 256 router logits.
#pragma once
#include <math.h>
#include <stdint.h>

#include "nmoe_common.cuh"

namespace nmoe {

struct TopkScratch {
    __align__(16) float cval[kExperts + 4];
    __align__(16) int cidx[kExperts + 4];
    uint32_t idx[kMaxK];
    float sel_v[kMaxK];
};

// Top-k of the 256 logits held 8 per lane (lane l: experts 8l..8l+7), one warp.
// Rule of nmoe_cpu_topk (src/math.m:95-132) on the logits: descending, lower expert id
// first on ties. Writes S->idx[0..k) and S->sel_v[0..k) (the selected logits).
// Candidates are the logits >= min over 8 groups (4 lanes, 32 logits) of the group
// maximum -- at least 8 logits qualify, so the top-k (k <= 8) are among them -- ranked
// against each other.
__device__ __forceinline__ void warp_topk(const float *v, int k, TopkScratch *S, int lane) {
    float m = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, v[i]);
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    float thr = m;
    thr = fminf(thr, __shfl_xor_sync(0xffffffffu, thr, 4));
    thr = fminf(thr, __shfl_xor_sync(0xffffffffu, thr, 8));
    thr = fminf(thr, __shfl_xor_sync(0xffffffffu, thr, 16));
    // candidate positions from 8 ballots (value slot j major, lane minor)
    const uint32_t lt = (1u << lane) - 1u;
    int base = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const bool cand = !(v[j] < thr);
        const uint32_t b = __ballot_sync(0xffffffffu, cand);
        if (cand) {
            S->cval[base + __popc(b & lt)] = v[j];
            S->cidx[base + __popc(b & lt)] = 8 * lane + j;
        }
        base += __popc(b);
    }
    const int nc = base;
    const int ncp = (nc + 3) & ~3;   // pad to a multiple of 4 with entries that never win
    if (lane < ncp - nc) {
        S->cval[nc + lane] = -INFINITY;
        S->cidx[nc + lane] = 1 << 20;
    }
    __syncwarp();
    for (int q = lane; q < nc; q += 32) {
        const float vi = S->cval[q];
        const int ii = S->cidx[q];
        int rank = 0;
        for (int j = 0; j < ncp; j += 4) {
            const float4 u = *reinterpret_cast<const float4 *>(&S->cval[j]);
            const int4 ui = *reinterpret_cast<const int4 *>(&S->cidx[j]);
            rank += (u.x > vi) | ((u.x == vi) & (ui.x < ii));
            rank += (u.y > vi) | ((u.y == vi) & (ui.y < ii));
            rank += (u.z > vi) | ((u.z == vi) & (ui.z < ii));
            rank += (u.w > vi) | ((u.w == vi) & (ui.w < ii));
        }
        if (rank < k) {
            S->idx[rank] = (uint32_t)ii;
            S->sel_v[rank] = vi;
        }
    }
    __syncwarp();
}


// Renormalised top-k weights: exp(l_s - l_0) / sum_{t<k} exp(l_t - l_0) -- the
// softmax-then-renormalise of src/runtime.m:1498-1511, whose full denominator cancels.
__device__ __forceinline__ float topk_weight(const TopkScratch *S, int k, int s) {
    const float l0 = S->sel_v[0];
    float sum = 0.f;
    for (int t = 0; t < k; ++t) sum += expf(S->sel_v[t] - l0);
    return s < k ? expf(S->sel_v[s] - l0) / sum : 0.f;
}

}  // namespace nmoe
