// nmoe_decode.cu -- batch-1 routed-MoE block, staged kernels.
//
// Four launches per layer:
//   route_shared  router logits + shared SiLU(gate)*up + shared-gate score
//                 (the work of nmoe_route_shared_q4, metal/kernels.metal:384-514)
//   route_topk    top-k of 256 + renormalised weights (nmoe_route_topk,
//                 metal/kernels.metal:1715-1776; selection rule of src/math.m:95-132)
//   gate_up       SiLU(gate_e x) * (up_e x) for the k routed experts
//                 (nmoe_expert_gate_up_q4_routed, metal/kernels.metal:716-788; q2 path
//                 src/runtime.m:2862-2877)
//   down_combine  h_mid + sum_s w_s down_e(act_s) + sigmoid(score) shared_down(shared_act)
//                 (nmoe_expert_down_combine_q4, metal/kernels.metal:1456-1542;
//                 nmoe_weighted_expert_sum, metal/kernels.metal:1394-1423)
// Every kernel is a warp-per-row GEMV with 128-bit streaming loads of the packed
// weights; the affine dequant is factored per 32/64-column chunk as
// s*sum(q*x) + b*sum(x). Scratch between launches lives in a DecodeScratch block.
#include "nmoe_decode.cuh"

namespace nmoe {

__device__ __forceinline__ void stage_x(const void *x, int x_f32, float *xs, float *xsum32) {
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x)
        xs[i] = x_f32 ? static_cast<const float *>(x)[i] : bf16_to_f32(static_cast<const uint16_t *>(x)[i]);
    __syncthreads();
    for (int c = threadIdx.x; c < kHidden / 32; c += blockDim.x) {
        float s = 0.f;
        for (int i = 0; i < 32; ++i) s += xs[32 * c + i];
        xsum32[c] = s;
    }
    __syncthreads();
}

// ---------------------------------------------------------------- route_shared --
// Warp jobs: [0,256) router rows, [256,768) shared gate/up rows, 768 shared-gate score.
template <bool kRouterQ4, bool kSharedQ4>
__global__ void __launch_bounds__(256) k_route_shared(LayerDev L, const void *x, int x_f32, DecodeScratch *ws) {
    __shared__ float xs[kHidden];
    __shared__ float xsum32[kHidden / 32];
    stage_x(x, x_f32, xs, xsum32);
    const int lane = threadIdx.x & 31;
    const int job = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (job < kExperts) {
        float v = warp_sum(dense_row_partial<kRouterQ4>(L.router, job, kHidden, xs, xsum32, lane));
        if (lane == 0) ws->logits[job] = v;
    } else if (job < kExperts + kInter) {
        const int r = job - kExperts;
        float g = warp_sum(dense_row_partial<kSharedQ4>(L.sgate, r, kHidden, xs, xsum32, lane));
        float u = warp_sum(dense_row_partial<kSharedQ4>(L.sup, r, kHidden, xs, xsum32, lane));
        if (lane == 0) ws->shared_act[r] = siluf_(g) * u;
    } else if (job == kExperts + kInter) {
        float v = warp_sum(dense_row_partial<kSharedQ4>(L.gvec, 0, kHidden, xs, xsum32, lane));
        if (lane == 0) ws->score = v;
    }
}

// ------------------------------------------------------------------ route_topk --
// 256 threads; thread i ranks logit i against all others: rank = #{j: l_j > l_i or
// (l_j == l_i and j < i)}. Picks with rank < k land in slot `rank`, i.e. descending
// order with the lower expert id first on a tie -- the selection of nmoe_cpu_topk
// (src/math.m:95-132) applied to the logits (softmax is monotone).
// Weight of slot s: exp(l_s - l_0) / sum_{t<k} exp(l_t - l_0), which equals the
// reference's renormalised softmax probability (the full-softmax denominator cancels).
__device__ void block_topk256(const float *lg, int k, uint32_t *idx_s, float *val_s) {
    const int i = threadIdx.x;
    const float v = lg[i];
    int rank = 0;
#pragma unroll 8
    for (int j = 0; j < kExperts; ++j) {
        const float u = lg[j];
        rank += (u > v) | ((u == v) & (j < i));
    }
    if (rank < k) {
        idx_s[rank] = (uint32_t)i;
        val_s[rank] = v;
    }
}

__global__ void __launch_bounds__(256) k_route_topk(const float *logits_in, int k, DecodeScratch *ws,
                                                    uint32_t *idx_out, float *w_out, float *logits_out) {
    __shared__ float lg[kExperts];
    __shared__ uint32_t idx_s[kMaxK];
    __shared__ float val_s[kMaxK];
    lg[threadIdx.x] = logits_in[threadIdx.x];
    if (logits_out) logits_out[threadIdx.x] = lg[threadIdx.x];
    __syncthreads();
    block_topk256(lg, k, idx_s, val_s);
    __syncthreads();
    if (threadIdx.x < kMaxK) {
        const int s = threadIdx.x;
        float e = s < k ? expf(val_s[s] - val_s[0]) : 0.f;
        float sum = 0.f;
        for (int t = 0; t < k; ++t) sum += expf(val_s[t] - val_s[0]);
        const float w = s < k ? e / sum : 0.f;
        const uint32_t id = s < k ? idx_s[s] : 0u;
        ws->idx[s] = id;
        ws->w[s] = w;
        if (idx_out) idx_out[s] = id;
        if (w_out) w_out[s] = w;
    }
}

// --------------------------------------------------------------------- gate_up --
// grid (rows/8, k); warp = one intermediate row r of slot s: act[s][r] = SiLU(g)*u.
template <int kBits>
__global__ void __launch_bounds__(256) k_expert_gate_up(LayerDev L, const void *x, int x_f32,
                                                        DecodeScratch *ws, int num_experts, int *err) {
    __shared__ float xs[kHidden];
    __shared__ float xsum32[kHidden / 32];
    stage_x(x, x_f32, xs, xsum32);
    const int lane = threadIdx.x & 31;
    const int s = blockIdx.y;
    const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const uint32_t e = ws->idx[s];
    if (e >= (uint32_t)num_experts) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicCAS(err, 0, kErrExpertRange);
        if (lane == 0) ws->act[s * kInter + r] = 0.f;
        return;
    }
    const ExpertOffsets o = expert_offsets(kBits);
    const uint8_t *blob = L.experts + (size_t)e * o.size;
    constexpr int kWordsPerRow = kHidden * kBits / 32;   // 256 (q4) / 128 (q2)
    constexpr int kChunks = kWordsPerRow / 4;            // uint4 chunks per row
    const uint4 *gw = reinterpret_cast<const uint4 *>(blob + o.gw) + (size_t)r * kChunks;
    const uint4 *uw = reinterpret_cast<const uint4 *>(blob + o.uw) + (size_t)r * kChunks;
    const uint16_t *gs = reinterpret_cast<const uint16_t *>(blob + o.gs) + r * (kHidden / kGroup);
    const uint16_t *gb = reinterpret_cast<const uint16_t *>(blob + o.gb) + r * (kHidden / kGroup);
    const uint16_t *us = reinterpret_cast<const uint16_t *>(blob + o.us) + r * (kHidden / kGroup);
    const uint16_t *ub = reinterpret_cast<const uint16_t *>(blob + o.ub) + r * (kHidden / kGroup);
    float ga = 0.f, ua = 0.f;
#pragma unroll
    for (int c = lane; c < kChunks; c += 32) {
        const uint4 wg = ldg_stream(gw + c), wu = ldg_stream(uw + c);
        if (kBits == 4) {
            const int g = c >> 1;
            const float *xc = xs + 32 * c;
            ga = fmaf(bf16_to_f32(gs[g]), dot_q4_32(wg, xc), fmaf(bf16_to_f32(gb[g]), xsum32[c], ga));
            ua = fmaf(bf16_to_f32(us[g]), dot_q4_32(wu, xc), fmaf(bf16_to_f32(ub[g]), xsum32[c], ua));
        } else {
            const int g = c;
            const float *xc = xs + 64 * c;
            const float sx = xsum32[2 * c] + xsum32[2 * c + 1];
            ga = fmaf(bf16_to_f32(gs[g]), dot_q2_64(wg, xc), fmaf(bf16_to_f32(gb[g]), sx, ga));
            ua = fmaf(bf16_to_f32(us[g]), dot_q2_64(wu, xc), fmaf(bf16_to_f32(ub[g]), sx, ua));
        }
    }
    ga = warp_sum(ga);
    ua = warp_sum(ua);
    if (lane == 0) ws->act[s * kInter + r] = siluf_(ga) * ua;
}

// ---------------------------------------------------------------- down_combine --
// grid 2048/8; warp = one output row. Experts are split across lane groups
// (q4: 16 lanes x 16 chunks of 32 columns per slot; q2: 8 lanes x 8 chunks of 64).
template <int kBits, bool kSharedQ4>
__global__ void __launch_bounds__(256) k_down_combine(LayerDev L, DecodeScratch *ws, int k, const float *h_mid,
                                                      float *out, int num_experts) {
    __shared__ float act[kMaxK][kInter];
    __shared__ float asum[kMaxK][kInter / 32];
    __shared__ float sact[kInter];
    __shared__ float ssum[kInter / 32];
    for (int i = threadIdx.x; i < k * kInter; i += blockDim.x) act[i / kInter][i % kInter] = ws->act[i];
    for (int i = threadIdx.x; i < kInter; i += blockDim.x) sact[i] = ws->shared_act[i];
    __syncthreads();
    for (int i = threadIdx.x; i < (k + 1) * (kInter / 32); i += blockDim.x) {
        const int s = i / (kInter / 32), c = i % (kInter / 32);
        const float *src = s < k ? &act[s][32 * c] : &sact[32 * c];
        float t = 0.f;
        for (int j = 0; j < 32; ++j) t += src[j];
        if (s < k) asum[s][c] = t;
        else ssum[c] = t;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const ExpertOffsets o = expert_offsets(kBits);
    constexpr int kLanesPerSlot = kBits == 4 ? 16 : 8;
    constexpr int kSlotsPerPass = 32 / kLanesPerSlot;
    const int sub = lane / kLanesPerSlot, c = lane % kLanesPerSlot;
    float moe = 0.f;
    for (int s0 = 0; s0 < k; s0 += kSlotsPerPass) {
        const int s = s0 + sub;
        if (s >= k) continue;
        const uint32_t e = ws->idx[s];
        if (e >= (uint32_t)num_experts) continue;
        const uint8_t *blob = L.experts + (size_t)e * o.size;
        const uint4 w = ldg_stream(reinterpret_cast<const uint4 *>(blob + o.dw) + (size_t)row * kLanesPerSlot + c);
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(blob + o.ds) + row * (kInter / kGroup);
        const uint16_t *bi = reinterpret_cast<const uint16_t *>(blob + o.db) + row * (kInter / kGroup);
        float part;
        if (kBits == 4) {
            part = fmaf(bf16_to_f32(sc[c >> 1]), dot_q4_32(w, &act[s][32 * c]), bf16_to_f32(bi[c >> 1]) * asum[s][c]);
        } else {
            part = fmaf(bf16_to_f32(sc[c]), dot_q2_64(w, &act[s][64 * c]),
                        bf16_to_f32(bi[c]) * (asum[s][2 * c] + asum[s][2 * c + 1]));
        }
        moe = fmaf(ws->w[s], part, moe);
    }
    float sh = dense_row_partial<kSharedQ4>(L.sdown, row, kInter, sact, ssum, lane);
    moe = warp_sum(moe);
    sh = warp_sum(sh);
    if (lane == 0) {
        const float hm = h_mid ? h_mid[row] : 0.f;
        out[row] = hm + moe + sigmoidf_(ws->score) * sh;
    }
}

// ------------------------------------------------------------------- launchers --
cudaError_t launch_route(const DecodeArgs &a, cudaStream_t st, float *logits_out) {
    dim3 blk(256);
    const int jobs = kExperts + kInter + 1;
    dim3 grd((jobs + 7) / 8);
    if (a.router_q4 && a.shared_q4) k_route_shared<true, true><<<grd, blk, 0, st>>>(a.L, a.x, a.x_f32, a.ws);
    else if (a.router_q4) k_route_shared<true, false><<<grd, blk, 0, st>>>(a.L, a.x, a.x_f32, a.ws);
    else if (a.shared_q4) k_route_shared<false, true><<<grd, blk, 0, st>>>(a.L, a.x, a.x_f32, a.ws);
    else k_route_shared<false, false><<<grd, blk, 0, st>>>(a.L, a.x, a.x_f32, a.ws);
    k_route_topk<<<1, 256, 0, st>>>(a.ws->logits, a.k, a.ws, a.idx_out, a.w_out, logits_out);
    return cudaGetLastError();
}

cudaError_t launch_decode_staged(const DecodeArgs &a, cudaStream_t st) {
    cudaError_t e = launch_route(a, st, nullptr);
    if (e != cudaSuccess) return e;
    dim3 blk(256);
    dim3 g2(kInter / 8, a.k);
    if (a.bits == 4) k_expert_gate_up<4><<<g2, blk, 0, st>>>(a.L, a.x, a.x_f32, a.ws, a.num_experts, a.err);
    else k_expert_gate_up<2><<<g2, blk, 0, st>>>(a.L, a.x, a.x_f32, a.ws, a.num_experts, a.err);
    dim3 g3(kHidden / 8);
    if (a.bits == 4) {
        if (a.shared_q4) k_down_combine<4, true><<<g3, blk, 0, st>>>(a.L, a.ws, a.k, a.h_mid, a.out, a.num_experts);
        else k_down_combine<4, false><<<g3, blk, 0, st>>>(a.L, a.ws, a.k, a.h_mid, a.out, a.num_experts);
    } else {
        if (a.shared_q4) k_down_combine<2, true><<<g3, blk, 0, st>>>(a.L, a.ws, a.k, a.h_mid, a.out, a.num_experts);
        else k_down_combine<2, false><<<g3, blk, 0, st>>>(a.L, a.ws, a.k, a.h_mid, a.out, a.num_experts);
    }
    return cudaGetLastError();
}

}  // namespace nmoe
