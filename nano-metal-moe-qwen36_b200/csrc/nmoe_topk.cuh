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
// (-0 and +0 map to one key, as they compare equal). NaN maps to 1, below every other
// key (-inf is 0x007FFFFF) and above the popped-head sentinel 0: the reference's strict
// `>` never prefers a NaN (src/math.m:112-117), so a NaN logit is taken only once no
// other logit is left, lowest expert id first.
__device__ __forceinline__ uint32_t topk_key(float f) {
    const uint32_t u = __float_as_uint(f + 0.0f);
    if (f != f) return 1u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float topk_val(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

// Top-k of the 256 logits held 8 per lane (lane l: experts 8l..8l+7), one warp.
// Rule of nmoe_cpu_topk (src/math.m:95-132) on the logits: descending, lower expert id
// first on ties. Each lane sorts its 8 logits once (stable odd-even transposition: ties
// keep the lower position first); a round is one warp max of the lanes' heads, and the
// lowest lane holding it -- the lowest expert id -- pops its head. Registers only, one
// short dependency chain per round. Lane r < k returns the r-th selection; every lane
// returns the largest logit (l0).
struct TopkLane {
    uint32_t idx;
    float val, l0;
};
__device__ __forceinline__ TopkLane warp_topk_lane(const float *v, int k, int lane) {
    uint32_t key[8], id[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        key[j] = topk_key(v[j]);
        id[j] = (uint32_t)(8 * lane + j);
    }
#pragma unroll
    for (int ph = 0; ph < 8; ++ph)
#pragma unroll
        for (int j = ph & 1; j + 1 < 8; j += 2) {
            const bool sw = key[j + 1] > key[j];
            const uint32_t ka = key[j], kb = key[j + 1], ia = id[j], ib = id[j + 1];
            key[j] = sw ? kb : ka;
            key[j + 1] = sw ? ka : kb;
            id[j] = sw ? ib : ia;
            id[j + 1] = sw ? ia : ib;
        }
    TopkLane out{0u, 0.f, 0.f};
#pragma unroll 1
    for (int r = 0; r < k; ++r) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, key[0]);
        const int w = __ffs(__ballot_sync(0xffffffffu, key[0] == m)) - 1;
        const uint32_t wid = __shfl_sync(0xffffffffu, id[0], w);
        const float mv = topk_val(m);
        if (r == 0) out.l0 = mv;
        if (lane == r) {
            out.idx = wid;
            out.val = mv;
        }
        const bool me = lane == w;   // pop the head; 0 is below every finite key
#pragma unroll
        for (int j = 0; j < 7; ++j) {
            key[j] = me ? key[j + 1] : key[j];
            id[j] = me ? id[j + 1] : id[j];
        }
        key[7] = me ? 0u : key[7];
    }
    return out;
}

// The same selection with a shorter chain per round: the winning lane writes its id to
// sidx[r] and every lane writes sval[r] = the round's maximum (shared memory, read after
// a __syncwarp), so a round is one warp max, one ballot and the pop; the winner is the
// lowest lane holding the maximum (no lane index is moved between lanes). Returns the
// largest logit (l0) on every lane.
// tl (diagnostic timeline, may be null): lane 0 stamps %globaltimer after the per-lane
// sort (tl[0]) and after the first round (tl[1]).
__device__ __forceinline__ float warp_topk_smem(const float *v, int k, int lane, uint32_t *sidx, float *sval,
                                               uint32_t *tl = nullptr) {
    uint32_t key[8], id[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        key[j] = topk_key(v[j]);
        id[j] = (uint32_t)(8 * lane + j);
    }
#pragma unroll
    for (int ph = 0; ph < 8; ++ph)
#pragma unroll
        for (int j = ph & 1; j + 1 < 8; j += 2) {
            const bool sw = key[j + 1] > key[j];
            const uint32_t ka = key[j], kb = key[j + 1], ia = id[j], ib = id[j + 1];
            key[j] = sw ? kb : ka;
            key[j + 1] = sw ? ka : kb;
            id[j] = sw ? ib : ia;
            id[j + 1] = sw ? ia : ib;
        }
    uint32_t lt;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
    if (tl != nullptr && lane == 0) {
        uint64_t t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : "r"(key[7]), "r"(key[0]));
        tl[0] = (uint32_t)t;
    }
    float l0 = 0.f;
#pragma unroll 1
    for (int r = 0; r < k; ++r) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, key[0]);
        const bool eq = key[0] == m;
        const uint32_t bal = __ballot_sync(0xffffffffu, eq);
        const bool me = eq && (bal & lt) == 0u;   // lowest lane holding the maximum
        const float mv = topk_val(m);
        if (me) sidx[r] = id[0];
        if (lane == 0) sval[r] = mv;
        if (r == 0) l0 = mv;
#pragma unroll
        for (int j = 0; j < 7; ++j) {   // pop the head; 0 is below every other key
            key[j] = me ? key[j + 1] : key[j];
            id[j] = me ? id[j + 1] : id[j];
        }
        key[7] = me ? 0u : key[7];
        if (r == 0 && tl != nullptr && lane == 0) {
            uint64_t t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : "r"(key[0]));
            tl[1] = (uint32_t)t;
        }
    }
    __syncwarp();
    return l0;
}

// Same selection, written to S->idx[0..k) and S->sel_v[0..k).
__device__ __forceinline__ void warp_topk(const float *v, int k, TopkScratch *S, int lane) {
    const TopkLane t = warp_topk_lane(v, k, lane);
    if (lane < k) {
        S->idx[lane] = t.idx;
        S->sel_v[lane] = t.val;
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
