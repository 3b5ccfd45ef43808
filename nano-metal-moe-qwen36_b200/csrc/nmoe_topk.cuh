// nmoe_topk.cuh -- warp-level top-k of 256 router logits.
#pragma once
#include <math.h>
#include <stdint.h>

#include "nmoe_common.cuh"

namespace nmoe {

struct TopkScratch {
    uint32_t idx[kMaxK];
    float sel_v[kMaxK];
};

// Order-preserving key of a float: unsigned comparison of keys is float comparison
// (-0 and +0 map to one key, as they compare equal).
__device__ __forceinline__ uint32_t topk_key(float f) {
    const uint32_t u = __float_as_uint(f + 0.0f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float topk_val(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

// Top-k of the 256 logits held 8 per lane (lane l: experts 8l..8l+7), one warp.
// Rule of nmoe_cpu_topk (src/math.m:95-132) on the logits: descending, lower expert id
// first on ties. Writes S->idx[0..k) and S->sel_v[0..k) (the selected logits).
// Each lane keeps the best of its remaining logits (first position on ties); a round is
// one warp max of those heads, and the lowest lane holding it -- the lowest expert id --
// gives up its head. Registers only, k rounds of a few instructions: the routing sits
// on the decode kernel's serial path, where every instruction is a fetch.
__device__ __forceinline__ void warp_topk(const float *v, int k, TopkScratch *S, int lane) {
    uint32_t key[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) key[j] = topk_key(v[j]);
    auto head = [&](uint32_t &hk, int &hj) {
        hk = key[0];
        hj = 0;
#pragma unroll
        for (int j = 1; j < 8; ++j)
            if (key[j] > hk) { hk = key[j]; hj = j; }
    };
    uint32_t hk;
    int hj;
    head(hk, hj);
#pragma unroll 1
    for (int r = 0; r < k; ++r) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, hk);
        const int w = __ffs(__ballot_sync(0xffffffffu, hk == m)) - 1;
        if (lane == w) {
            S->idx[r] = (uint32_t)(8 * lane + hj);
            S->sel_v[r] = topk_val(m);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j == hj) key[j] = 0u;   // below every finite key: never picked again
            head(hk, hj);
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
