// nmoe_gdn.cu -- the GatedDeltaNet (linear-attention) core of one decode step, one launch.
//
// Replaces five reference kernels run back to back in NMOELinearAttentionStepMetal
// (src/runtime.m:3390-3478): nmoe_conv1d_step (metal/kernels.metal:1275-1295),
// nmoe_rms_norm_qk (1780-1821), nmoe_compute_decay_beta (1823-1839),
// nmoe_gated_delta_net_step (1300-1346) and nmoe_gated_rms_norm (1841-1873). The
// projections before (qkv / z / beta / alpha) and the output projection after are plain
// GEMVs and stay outside.
//
// Geometry (Qwen3.6): 16 key heads and 32 value heads of 128; value head vh reads key
// head vh / 2; conv over 8192 channels (q 0..2047, k 2048..4095, v 4096..8191), width 4.
//
// Work split: 16 clusters of 8 CTAs, one cluster per key head. CTA r of cluster kh serves
// value head 2 kh + r / 4, value rows 32 (r % 4) .. +31, i.e. 16 KB of the 2 MB recurrent
// state, read and written once. The q and k channels of the key head are convolved once:
// CTA r owns 16 q and 16 k channels (and its 32 v channels), updates their conv state, and
// the cluster exchanges the convolved q, k through distributed shared memory. The gated
// RMS norm needs the sum of squares over a value head's 128 outputs: the 4 CTAs of the
// head exchange their partial sums the same way. No CTA waits on memory another CTA
// writes through global memory, and every channel's conv state has exactly one writer.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "nmoe/moe_cuda.h"

namespace cg = cooperative_groups;

namespace {

constexpr int kKH = 16, kVH = 32, kD = 128, kConv = 8192;
constexpr int kCluster = 8, kThreads = 128, kRows = 32;   // value rows per CTA

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }
__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu(float x) { return x * sigm(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

struct GdnArgs {
    const float *qkv, *z, *alpha, *beta;
    const uint16_t *conv_w, *dt_bias, *norm_w;
    const float *A_log;
    float *conv_state, *delta_state, *out;
};

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads, 1) k_linear_attn_step(const GdnArgs a) {
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ float qk_part[32];        // this CTA's 16 q and 16 k channels, convolved
    __shared__ float qs[kD], ks[kD];     // the key head's q and k, gathered and normalised
    __shared__ float vloc[kRows], oloc[kRows];
    __shared__ float red[2][4];
    __shared__ float ss_part;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = (int)cluster.block_rank();
    // sequence blockIdx.y of a batch: its inputs, states and output
    const size_t sq = blockIdx.y;
    const float *qkv = a.qkv + sq * kConv, *zin = a.z + sq * kVH * kD;
    const float *alpha = a.alpha + sq * kVH, *beta = a.beta + sq * kVH;
    float *conv_state = a.conv_state + sq * 3 * kConv, *out = a.out + sq * kVH * kD;
    const int kh = blockIdx.x / kCluster;
    const int vh = 2 * kh + (r >> 2), split = r & 3;

    // the 32 state rows are issued first: their HBM latency overlaps the conv, the
    // exchanges and the norms (warp w rows 8w..8w+7, lane l keys 4l..4l+3)
    float4 *S = reinterpret_cast<float4 *>(a.delta_state + sq * kVH * kD * kD + ((size_t)vh * kD + kRows * split + 8 * warp) * kD);
    float4 st[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) st[i] = __ldcs(S + i * (kD / 4) + lane);

    // ---- conv step of the 64 channels this CTA owns (kernels.metal:1275-1295)
    if (tid < 64) {
        int ch;
        if (tid < 16) ch = kh * kD + 16 * r + tid;                           // q
        else if (tid < 32) ch = 2048 + kh * kD + 16 * r + (tid - 16);        // k
        else ch = 4096 + vh * kD + kRows * split + (tid - 32);               // v
        const uint2 wv = *reinterpret_cast<const uint2 *>(a.conv_w + 4 * ch);
        const float s0 = conv_state[ch], s1 = conv_state[kConv + ch], s2 = conv_state[2 * kConv + ch];
        const float inp = qkv[ch];
        float acc = 0.0f;
        acc += s0 * bf16f((uint16_t)(wv.x & 0xFFFFu));
        acc += s1 * bf16f((uint16_t)(wv.x >> 16));
        acc += s2 * bf16f((uint16_t)(wv.y & 0xFFFFu));
        acc += inp * bf16f((uint16_t)(wv.y >> 16));
        const float c = silu(acc);
        conv_state[ch] = s1;
        conv_state[kConv + ch] = s2;
        conv_state[2 * kConv + ch] = inp;
        if (tid < 32) qk_part[tid] = c;
        else vloc[tid - 32] = c;
    }
    cluster.sync();
    // ---- gather q, k of the key head from the 8 CTAs (distributed shared memory)
    {
        const float *src = cluster.map_shared_rank(qk_part, tid >> 4);
        qs[tid] = src[tid & 15];
        ks[tid] = src[16 + (tid & 15)];
    }
    __syncthreads();
    // ---- q/k RMS norm (kernels.metal:1780-1821: eps 1e-12, inv_scale = 1/sqrt(128))
    {
        const float q = qs[tid], k = ks[tid];
        float sq = warp_sum(q * q), sk = warp_sum(k * k);
        if (lane == 0) {
            red[0][warp] = sq;
            red[1][warp] = sk;
        }
        __syncthreads();
        sq = (red[0][0] + red[0][1]) + (red[0][2] + red[0][3]);
        sk = (red[1][0] + red[1][1]) + (red[1][2] + red[1][3]);
        const float inv_scale = rsqrtf((float)kD);
        qs[tid] = q * rsqrtf(sq / (float)kD + 1e-12f) * inv_scale * inv_scale;
        ks[tid] = k * rsqrtf(sk / (float)kD + 1e-12f) * inv_scale;
    }
    __syncthreads();
    // ---- decay and beta of the value head (kernels.metal:1823-1839)
    const float A = expf(a.A_log[vh]);
    const float sp = logf(1.0f + expf(alpha[vh] + bf16f(a.dt_bias[vh])));
    const float g = expf(-A * sp);
    const float b = sigm(beta[vh]);
    // ---- delta rule on the 32 state rows (kernels.metal:1300-1346)
    {
        const float4 k4 = reinterpret_cast<const float4 *>(ks)[lane];
        const float4 q4 = reinterpret_cast<const float4 *>(qs)[lane];
        float kv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            st[i].x *= g;
            st[i].y *= g;
            st[i].z *= g;
            st[i].w *= g;
            kv[i] = (st[i].x * k4.x + st[i].y * k4.y) + (st[i].z * k4.z + st[i].w * k4.w);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int i = 0; i < 8; ++i) kv[i] += __shfl_xor_sync(0xffffffffu, kv[i], o);
        float ov[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float d = (vloc[8 * warp + i] - kv[i]) * b;
            st[i].x += k4.x * d;
            st[i].y += k4.y * d;
            st[i].z += k4.z * d;
            st[i].w += k4.w * d;
            __stcs(S + i * (kD / 4) + lane, st[i]);
            ov[i] = (st[i].x * q4.x + st[i].y * q4.y) + (st[i].z * q4.z + st[i].w * q4.w);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int i = 0; i < 8; ++i) ov[i] += __shfl_xor_sync(0xffffffffu, ov[i], o);
        if (lane < 8) {
            float v = ov[0];
#pragma unroll
            for (int i = 1; i < 8; ++i) v = lane == i ? ov[i] : v;
            oloc[8 * warp + lane] = v;
        }
    }
    __syncthreads();
    // ---- gated RMS norm over the value head's 128 outputs (kernels.metal:1841-1873)
    if (warp == 0) {
        const float o = oloc[lane];
        const float s = warp_sum(o * o);
        if (lane == 0) ss_part = s;
    }
    cluster.sync();
    if (tid < kRows) {
        const int base = r & 4;   // the 4 CTAs of this value head
        float tot = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) tot += *cluster.map_shared_rank(&ss_part, base + j);
        const float inv = rsqrtf(tot / (float)kD + 1e-6f);
        const int vi = kRows * split + tid;
        out[vh * kD + vi] = oloc[tid] * inv * silu(zin[vh * kD + vi]) * bf16f(a.norm_w[vi]);
    }
    cluster.sync();   // no CTA leaves while another still reads its shared memory
}

}  // namespace

namespace {

int launch_gdn(const nmoe_linear_attn_weights *w, int batch, const float *qkv, const float *z, const float *alpha,
               const float *beta, float *conv_state, float *delta_state, float *out, void *stream) {
    if (w == nullptr || w->conv_w == nullptr || w->A_log == nullptr || w->dt_bias == nullptr ||
        w->norm_w == nullptr || qkv == nullptr || z == nullptr || alpha == nullptr || beta == nullptr ||
        conv_state == nullptr || delta_state == nullptr || out == nullptr)
        return NMOE_EINVAL;
    if (batch < 1 || batch > 65535) return NMOE_EINVAL;
    if ((reinterpret_cast<uintptr_t>(delta_state) & 15u) != 0 || (reinterpret_cast<uintptr_t>(w->conv_w) & 7u) != 0)
        return NMOE_EINVAL;
    GdnArgs a{qkv, z, alpha, beta, w->conv_w, w->dt_bias, w->norm_w, w->A_log, conv_state, delta_state, out};
    k_linear_attn_step<<<dim3(kKH * kCluster, batch), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    return cudaGetLastError() == cudaSuccess ? NMOE_OK : NMOE_ECUDA;
}

}  // namespace

extern "C" int nmoe_linear_attn_step(const nmoe_linear_attn_weights *w, const float *qkv, const float *z,
                                     const float *alpha, const float *beta, float *conv_state, float *delta_state,
                                     float *out, void *stream) {
    return launch_gdn(w, 1, qkv, z, alpha, beta, conv_state, delta_state, out, stream);
}

extern "C" int nmoe_linear_attn_step_batched(const nmoe_linear_attn_weights *w, int batch, const float *qkv,
                                             const float *z, const float *alpha, const float *beta,
                                             float *conv_state, float *delta_state, float *out, void *stream) {
    return launch_gdn(w, batch, qkv, z, alpha, beta, conv_state, delta_state, out, stream);
}
