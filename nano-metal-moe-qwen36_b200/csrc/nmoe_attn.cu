// nmoe_attn.cu -- full-attention decode step (Qwen3.6 full layers), one launch.
//
// Replaces, in NMOEFullAttentionStepMetal (src/runtime.m:3040-3095): nmoe_full_qk_prep
// (metal/kernels.metal:1006-1058: per-head RMS norm with weight + 1, rotate-half RoPE on
// dims 0..63, sigmoid of the query gate), the two copy kernels that append k and v to the
// caches, and nmoe_attn_decode_fused (kernels.metal:1119-1194: one threadgroup per query
// head, online softmax over all positions, output times the gate).
//
// Geometry: 16 query heads, 2 KV heads (8 query heads share one), head dim 256, caches
// f32 [position][2][256] (the reference's layout and type).
//
// Work split (split-K flash decode): the positions 0..position are cut into S slices per
// KV head (S up to 74, so at most 148 CTAs); a CTA reads each K and V row of its slice
// once and uses it for all 8 query heads of the KV head (the reference reads every row
// once per query head). Warp w of a CTA takes positions w, w+8, ...; lane l holds dims
// l + 32 j of a row. Each CTA writes its (max, sum, weighted values) per head to the
// workspace; a second launch merges the S slices of each (KV head, query head) in one CTA
// and applies the gate. The CTA whose slice holds `position` normalises and rotates the
// new k and appends k and v to the caches.
#include <cuda_runtime.h>
#include <math.h>

#include "nmoe/moe_cuda.h"

namespace {

constexpr int kHeads = 16, kKV = 2, kDim = 256, kGroup = kHeads / kKV;   // 8 query heads per KV head
constexpr int kThreads = 256, kWarps = kThreads / 32;
constexpr int kMaxSplit = 74;
constexpr int kPart = kDim + 4;   // weighted values, max, sum, 2 pad (rows of 16-byte units)
constexpr float kTheta = 10000000.0f;

struct FaArgs {
    const float *q, *k_new, *v_new;
    const uint16_t *q_norm, *k_norm;
    void *k_cache, *v_cache;   // f32 or bf16 [batch][cap][2][256]
    float *out;
    float *part;          // [batch][kKV][kMaxSplit][kGroup][kPart]
    int position, splits, cap;
    const int *d_position;   // when set: sequence b's position is d_position[b], read on the device
                             // (graph replays, batches), and the grid holds kMaxSplit slices per
                             // KV head, the unused ones exit
    float freq[32];       // RoPE frequencies theta^(-2t/64), correctly rounded to float
};

// ~64 positions (64 KB of K and V) per slice, 1 to kMaxSplit slices
__host__ __device__ __forceinline__ int slices_for(int position) {
    const int s = (position + 64) / 64;
    return s < 1 ? 1 : (s > kMaxSplit ? kMaxSplit : s);
}

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// cache elements: f32 (the reference's cache) or bf16 (uint16_t, round to nearest even)
__device__ __forceinline__ float kv_load(const float *p) { return __ldcs(p); }
__device__ __forceinline__ float kv_load(const uint16_t *p) { return bf16f(__ldcs(reinterpret_cast<const unsigned short *>(p))); }
__device__ __forceinline__ void kv_store(float *p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(uint16_t *p, float v) {
    const uint32_t u = __float_as_uint(v);
    *p = (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// RMS norm (eps 1e-6, weight + 1) and rotate-half RoPE of one 256-vector held by a warp,
// lane l: dims l + 32 j (kernels.metal:1006-1053).
__device__ __forceinline__ void prep_vec(float *v, const uint16_t *w, int position, int lane, const float *freq) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)kDim + 1e-6f);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = v[j] * inv * (bf16f(w[lane + 32 * j]) + 1.0f);
    // rotary dims 0..63: pair (t, t + 32), t = lane: elements j = 0 and j = 1 of this lane
    // the angle position * freq is ill-conditioned at long positions (one ulp of freq
    // moves it by position ulps), so freq is the correctly rounded value, from the host
    const float ang = (float)position * freq[lane];
    float s, c;
    sincosf(ang, &s, &c);
    const float v0 = v[0], v1 = v[1];
    v[0] = v0 * c - v1 * s;
    v[1] = v0 * s + v1 * c;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_full_attn_step(const FaArgs a) {
    extern __shared__ float smf[];
    float *qs = smf;                             // [8][256] prepared queries
    float *tacc = qs + kGroup * kDim;            // [8 warps][8 heads][256]
    float *tm = tacc + kWarps * kGroup * kDim;   // [8 warps][8 heads]
    float *tl = tm + kWarps * kGroup;            // [8 warps][8 heads]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.y;   // sequence
    const int position = a.d_position ? a.d_position[b] : a.position;
    if (position < 0 || position >= a.cap) return;   // the merge writes zeros for it
    const float *Q = a.q + (size_t)b * kHeads * 2 * kDim;
    const float *KN = a.k_new + (size_t)b * kKV * kDim, *VN = a.v_new + (size_t)b * kKV * kDim;
    T *KC = static_cast<T *>(a.k_cache) + (size_t)b * a.cap * kKV * kDim;
    T *VC = static_cast<T *>(a.v_cache) + (size_t)b * a.cap * kKV * kDim;
    const int splits = a.d_position ? slices_for(position) : a.splits;
    const int grid_splits = a.d_position ? kMaxSplit : a.splits;
    const int kvh = blockIdx.x / grid_splits, split = blockIdx.x % grid_splits;
    if (split >= splits) return;   // uniform over the CTA, before any barrier
    const int seq = position + 1;
    const int P = (seq + splits - 1) / splits;
    const int p0 = min(seq, split * P), p1 = min(seq, p0 + P);
    const bool holds_new = p0 <= position && position < p1;

    // ---- queries of the 8 heads (warp w: head 8 kvh + w)
    {
        const int h = kGroup * kvh + warp;
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = Q[h * 2 * kDim + lane + 32 * j];
        prep_vec(v, a.q_norm, position, lane, a.freq);
#pragma unroll
        for (int j = 0; j < 8; ++j) qs[warp * kDim + lane + 32 * j] = v[j];
    }
    // ---- the new position: k prepared, k and v appended to the caches (one CTA per KV head)
    if (holds_new && warp == 0) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = KN[kvh * kDim + lane + 32 * j];
        prep_vec(v, a.k_norm, position, lane, a.freq);
        const size_t row = ((size_t)position * kKV + kvh) * kDim;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            kv_store(KC + row + lane + 32 * j, v[j]);
            kv_store(VC + row + lane + 32 * j, VN[kvh * kDim + lane + 32 * j]);
        }
    }
    __syncthreads();

    // ---- online softmax over the slice (warp w: positions p0 + w, p0 + w + 8, ...)
    float qr[kGroup][8];
#pragma unroll
    for (int h = 0; h < kGroup; ++h)
#pragma unroll
        for (int j = 0; j < 8; ++j) qr[h][j] = qs[h * kDim + lane + 32 * j];
    float m[kGroup], l[kGroup], acc[kGroup][8];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
        m[h] = -1e30f;
        l[h] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[h][j] = 0.f;
    }
    const float inv_scale = 1.0f / 16.0f;   // 1 / sqrt(256)
    // rows of the next two positions of this warp are in flight while one is processed
    float kr[8], vr[8], k1[8], v1[8], k2[8], v2[8];
    auto load_row = [&](int p, float *kx, float *vx) {
        if (p < p1) {
            const T *kp = KC + ((size_t)p * kKV + kvh) * kDim;
            const T *vp = VC + ((size_t)p * kKV + kvh) * kDim;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                kx[j] = kv_load(kp + lane + 32 * j);
                vx[j] = kv_load(vp + lane + 32 * j);
            }
        }
    };
    load_row(p0 + warp, kr, vr);
    load_row(p0 + warp + kWarps, k1, v1);
    for (int p = p0 + warp; p < p1; p += kWarps) {
        load_row(p + 2 * kWarps, k2, v2);
        float s[kGroup];
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            float d = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) d = fmaf(qr[h][j], kr[j], d);
            s[h] = d;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int h = 0; h < kGroup; ++h) s[h] += __shfl_xor_sync(0xffffffffu, s[h], o);
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            const float sc = s[h] * inv_scale;
            const float mn = fmaxf(m[h], sc);
            const float c = __expf(m[h] - mn), w = __expf(sc - mn);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[h][j] = fmaf(w, vr[j], acc[h][j] * c);
            l[h] = fmaf(l[h], c, w);
            m[h] = mn;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            kr[j] = k1[j];
            vr[j] = v1[j];
            k1[j] = k2[j];
            v1[j] = v2[j];
        }
    }
    // ---- merge the 8 warps, then this CTA's slice into the workspace
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
#pragma unroll
        for (int j = 0; j < 8; ++j) tacc[(warp * kGroup + h) * kDim + lane + 32 * j] = acc[h][j];
        if (lane == 0) {
            tm[warp * kGroup + h] = m[h];
            tl[warp * kGroup + h] = l[h];
        }
    }
    __syncthreads();
    {
        const int d = tid;   // one dim per thread, all 8 heads
        float *pb = a.part + (((size_t)b * kKV + kvh) * kMaxSplit + split) * kGroup * kPart;
#pragma unroll 1
        for (int h = 0; h < kGroup; ++h) {
            float M = -1e30f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) M = fmaxf(M, tm[w * kGroup + h]);
            float L = 0.f, A = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float e = __expf(tm[w * kGroup + h] - M);
                L = fmaf(tl[w * kGroup + h], e, L);
                A = fmaf(tacc[(w * kGroup + h) * kDim + d], e, A);
            }
            pb[h * kPart + d] = A;
            if (d == 0) {
                pb[h * kPart + kDim] = M;
                pb[h * kPart + kDim + 1] = L;
            }
        }
    }
}

// Merge of the S slices of one (KV head, query head) per CTA, one dim per thread, then the
// gate. A second launch on the stream: it starts after every slice has been written.
__global__ void __launch_bounds__(kThreads) k_full_attn_merge(const FaArgs a) {
    __shared__ float sm_m[kMaxSplit], sm_l[kMaxSplit];
    const int tid = threadIdx.x;
    const int b = blockIdx.y;   // sequence
    const int position = a.d_position ? a.d_position[b] : a.position;
    const int kvh = blockIdx.x / kGroup, h = blockIdx.x % kGroup;
    const int hq = kGroup * kvh + h;
    float *out = a.out + (size_t)b * kHeads * kDim;
    if (position < 0 || position >= a.cap) {   // a position outside the cache: zeros
        out[hq * kDim + tid] = 0.f;
        return;
    }
    const int splits = a.d_position ? slices_for(position) : a.splits;
    const float *pb = a.part + ((size_t)b * kKV + kvh) * kMaxSplit * kGroup * kPart + (size_t)h * kPart;
    const size_t sstride = (size_t)kGroup * kPart;
    if (tid < splits) {
        sm_m[tid] = pb[tid * sstride + kDim];
        sm_l[tid] = pb[tid * sstride + kDim + 1];
    }
    __syncthreads();
    float M = -1e30f;
    for (int sI = 0; sI < splits; ++sI) M = fmaxf(M, sm_m[sI]);
    float L = 0.f, A = 0.f;
#pragma unroll 8
    for (int sI = 0; sI < splits; ++sI) {
        const float e = __expf(sm_m[sI] - M);
        L = fmaf(sm_l[sI], e, L);
        A = fmaf(pb[sI * sstride + tid], e, A);
    }
    const float gate = 1.0f / (1.0f + expf(-a.q[(size_t)b * kHeads * 2 * kDim + hq * 2 * kDim + kDim + tid]));
    out[hq * kDim + tid] = (L > 0.f ? A / L : 0.f) * gate;
}

constexpr size_t kSmem = (size_t)(kGroup * kDim + kWarps * kGroup * kDim + 2 * kWarps * kGroup) * 4;

}  // namespace

extern "C" size_t nmoe_full_attn_workspace_bytes(void) {
    return (size_t)kKV * kMaxSplit * kGroup * kPart * 4 + 256;
}

extern "C" size_t nmoe_full_attn_batched_workspace_bytes(int batch) {
    return batch < 1 ? 0 : (size_t)batch * kKV * kMaxSplit * kGroup * kPart * 4 + 256;
}

namespace {

template <typename T>
int launch_full_attn(const nmoe_full_attn_weights *w, int batch, const float *q, const float *k_new,
                     const float *v_new, T *k_cache, T *v_cache, int cap, int position, const int *d_position,
                     float *out, void *workspace, cudaStream_t st) {
    static bool attr_set = false;   // per process and element type; a function property
    if (!attr_set) {
        if (cudaFuncSetAttribute(k_full_attn_step<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) !=
            cudaSuccess)
            return NMOE_ECUDA;
        attr_set = true;
    }
    FaArgs a;
    a.q = q;
    a.k_new = k_new;
    a.v_new = v_new;
    a.q_norm = w->q_norm;
    a.k_norm = w->k_norm;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.out = out;
    a.part = static_cast<float *>(workspace);
    a.position = position;
    a.splits = slices_for(position);
    a.cap = cap;
    a.d_position = d_position;
    for (int t = 0; t < 32; ++t) a.freq[t] = (float)pow((double)kTheta, -2.0 * t / 64.0);
    const dim3 grid(kKV * (d_position ? kMaxSplit : a.splits), batch);
    k_full_attn_step<T><<<grid, kThreads, kSmem, st>>>(a);
    k_full_attn_merge<<<dim3(kKV * kGroup, batch), kThreads, 0, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? NMOE_OK : NMOE_ECUDA;
}

}  // namespace

extern "C" int nmoe_full_attn_step(const nmoe_full_attn_weights *w, const float *q, const float *k_new,
                                   const float *v_new, float *k_cache, float *v_cache, int position,
                                   int max_positions, float *out, void *workspace, void *stream) {
    if (w == nullptr || w->q_norm == nullptr || w->k_norm == nullptr || q == nullptr || k_new == nullptr ||
        v_new == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr || workspace == nullptr)
        return NMOE_EINVAL;
    if (position < 0 || position >= max_positions) return NMOE_EINVAL;
    if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return NMOE_EINVAL;
    return launch_full_attn<float>(w, 1, q, k_new, v_new, k_cache, v_cache, max_positions, position, nullptr, out,
                                   workspace, static_cast<cudaStream_t>(stream));
}

extern "C" int nmoe_full_attn_step_batched(const nmoe_full_attn_weights *w, int batch, const float *q,
                                           const float *k_new, const float *v_new, uint16_t *k_cache,
                                           uint16_t *v_cache, const int32_t *d_positions, int max_positions,
                                           float *out, void *workspace, void *stream) {
    if (w == nullptr || w->q_norm == nullptr || w->k_norm == nullptr || q == nullptr || k_new == nullptr ||
        v_new == nullptr || k_cache == nullptr || v_cache == nullptr || d_positions == nullptr || out == nullptr ||
        workspace == nullptr)
        return NMOE_EINVAL;
    if (batch < 1 || batch > 65535 || max_positions < 1) return NMOE_EINVAL;
    if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return NMOE_EINVAL;
    return launch_full_attn<uint16_t>(w, batch, q, k_new, v_new, k_cache, v_cache, max_positions, 0, d_positions,
                                      out, workspace, static_cast<cudaStream_t>(stream));
}

namespace nmoe {
// The same step with the position read on the device from *d_position (checked by the
// caller to lie in [0, max_positions)): one launch shape for every position, so that a
// captured graph of decode steps replays at any position.
int full_attn_step_dev(const nmoe_full_attn_weights *w, const float *q, const float *k_new, const float *v_new,
                       float *k_cache, float *v_cache, int max_positions, const int *d_position, float *out,
                       void *workspace, cudaStream_t st) {
    return launch_full_attn<float>(w, 1, q, k_new, v_new, k_cache, v_cache, max_positions, 0, d_position, out,
                                   workspace, st);
}
}  // namespace nmoe
