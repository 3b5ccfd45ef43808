// nmoe_batched.cu -- the T-token routed-MoE block: nmoe_moe_forward_batched.
//
// The reference runs prefill token by token through the batch-1 kernels
// (src/runtime.m:3816); this path computes the same block for T tokens at once:
//
//   k_prep      x -> bf16 hi (and lo, for f32 x) planes in the K order of the GEMM
//   GEMM        router logits [T][256] (hi/lo split operands: fp32-accurate)
//   k_route     per token: top-k of 256 + renormalised weights (src/runtime.m:1498-1511),
//               shared-gate score, per-expert counts and ranks
//   k_scatter   positions: tokens grouped by expert (offset[e] + rank)
//   GEMM        gate/up + SwiGLU for every (token, expert) position and for the shared
//               expert over all T tokens -> act
//   GEMM        down -> Y per position
//   k_combine   out = h_mid + sum_s w_s Y[pos(t,s)] + sigmoid(score) * Y[shared(t)]
//               (nmoe_expert_down_combine_q4, metal/kernels.metal:1497-1541)
// Every launch is asynchronous on the caller's stream; nothing is allocated per call.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "nmoe_batched.cuh"
#include "nmoe_gemm.cuh"
#include "nmoe_pack.cuh"
#include "nmoe_topk.cuh"

using namespace nmoe;

namespace nmoe {

struct BatchedState {
    int t_max = 0;
    uint16_t *xh = nullptr, *xl = nullptr;   // [t_max][2048] K-permuted bf16 planes
    float *logits = nullptr;                 // [t_max][256]
    float *score = nullptr;                  // [t_max]
    float *w = nullptr;                      // [t_max][8]
    uint32_t *idx = nullptr;                 // [t_max][8]
    int *rank = nullptr, *inv = nullptr;     // [t_max][8]
    int *perm = nullptr;                     // [t_max * 8]
    int *cnt = nullptr;                      // [256]
    uint16_t *act = nullptr;                 // [t_max * 9][512]  (routed positions, then shared)
    uint16_t *y = nullptr;                   // [t_max * 9][2048]
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    uint64_t timeout_ns = 1000000000ull;
    int last_T = 0;
};

}  // namespace nmoe

// ------------------------------------------------------------------ kernels ----

// x [T][2048] (bf16 or f32) -> xh (bf16(x)) and xl (bf16(x - xh), f32 input only), each
// 8-column group stored in the order [0,4,1,5,2,6,3,7]. Block 0 also clears the counts.
__global__ void k_prep(const void *x, int x_f32, int T, uint16_t *xh, uint16_t *xl, int *cnt) {
    if (blockIdx.x == 0 && threadIdx.x < kExperts) cnt[threadIdx.x] = 0;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // 8-column group
    if (i >= T * (kHidden / 8)) return;
    float v[8];
    if (x_f32) {
        const float4 a = reinterpret_cast<const float4 *>(x)[2 * i], b = reinterpret_cast<const float4 *>(x)[2 * i + 1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 a = reinterpret_cast<const uint4 *>(x)[i];
        const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) { v[2 * j] = bf16_lo(u[j]); v[2 * j + 1] = bf16_hi(u[j]); }
    }
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        h[j] = pack_bf16x2(v[j], v[j + 4]);
        l[j] = pack_bf16x2(v[j] - __uint_as_float(h[j] << 16), v[j + 4] - __uint_as_float(h[j] & 0xFFFF0000u));
    }
    reinterpret_cast<uint4 *>(xh)[i] = make_uint4(h[0], h[1], h[2], h[3]);
    if (x_f32) reinterpret_cast<uint4 *>(xl)[i] = make_uint4(l[0], l[1], l[2], l[3]);
}

// One warp per token: top-k of the 256 logits, renormalised weights, shared-gate score
// (fp32, from the unpermuted x), ranks within each expert's group.
struct RouteArgs {
    const float *logits;
    const void *x;
    int x_f32;
    const uint8_t *gvec;
    int gvec_q4;
    int T, k, num_experts;
    int expert_lo, n_local;
    uint32_t *idx;
    float *w, *score;
    int *rank, *cnt;
    uint32_t *idx_out;
    float *w_out;
    int *err;
};

constexpr int kRouteWarps = 8;

__global__ void __launch_bounds__(kRouteWarps * 32) k_route(const RouteArgs a) {
    __shared__ TopkScratch tk[kRouteWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kRouteWarps + warp;
    if (t >= a.T) return;
    TopkScratch *S = &tk[warp];
    float v[8];
    const float4 *lg = reinterpret_cast<const float4 *>(a.logits + (size_t)t * kExperts + 8 * lane);
    const float4 l0 = lg[0], l1 = lg[1];
    v[0] = l0.x; v[1] = l0.y; v[2] = l0.z; v[3] = l0.w; v[4] = l1.x; v[5] = l1.y; v[6] = l1.z; v[7] = l1.w;
    warp_topk(v, a.k, S, lane);

    // shared-gate score: lane covers columns 64*lane .. 64*lane+63
    float xs[64];
    if (a.x_f32) {
        const float4 *xp = reinterpret_cast<const float4 *>(static_cast<const float *>(a.x) + (size_t)t * kHidden + 64 * lane);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float4 q = xp[j];
            xs[4 * j] = q.x; xs[4 * j + 1] = q.y; xs[4 * j + 2] = q.z; xs[4 * j + 3] = q.w;
        }
    } else {
        const uint4 *xp = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.x) + (size_t)t * kHidden + 64 * lane);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint4 q = xp[j];
            const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) { xs[8 * j + 2 * i] = bf16_lo(u[i]); xs[8 * j + 2 * i + 1] = bf16_hi(u[i]); }
        }
    }
    float acc = 0.f;
    if (a.gvec_q4) {
        const uint32_t *gw = reinterpret_cast<const uint32_t *>(a.gvec) + 8 * lane;
        const uint16_t *gs = reinterpret_cast<const uint16_t *>(a.gvec + 1024);
        const float s = __uint_as_float((uint32_t)gs[lane] << 16), b = __uint_as_float((uint32_t)gs[32 + lane] << 16);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t q = gw[j];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = fmaf(fmaf((float)((q >> (4 * i)) & 15u), s, b), xs[8 * j + i], acc);
        }
    } else {
        const uint4 *gp = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(a.gvec) + 64 * lane);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint4 q = gp[j];
            const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc = fmaf(bf16_lo(u[i]), xs[8 * j + 2 * i], acc);
                acc = fmaf(bf16_hi(u[i]), xs[8 * j + 2 * i + 1], acc);
            }
        }
    }
    acc = warp_sum(acc);

    if (lane < kMaxK) {
        const int s = lane;
        const uint32_t e = s < a.k ? S->idx[s] : 0u;
        const float wt = topk_weight(S, a.k, s);
        const bool valid = s < a.k && e < (uint32_t)a.num_experts;
        if (s < a.k && !valid) atomicCAS(a.err, 0, kErrExpertRange);
        const int le = (int)e - a.expert_lo;
        int rk = -1;
        if (valid && le >= 0 && le < a.n_local) rk = atomicAdd(&a.cnt[le], 1);
        a.idx[(size_t)t * kMaxK + s] = e;
        a.w[(size_t)t * kMaxK + s] = valid ? wt : 0.f;
        a.rank[(size_t)t * kMaxK + s] = rk;
        if (a.idx_out) a.idx_out[(size_t)t * kMaxK + s] = e;
        if (a.w_out) a.w_out[(size_t)t * kMaxK + s] = wt;
    }
    if (lane == 0) a.score[t] = acc;
}

// Position of (t, s) = exclusive prefix of counts over the experts before e + rank.
__global__ void k_scatter(const uint32_t *idx, const int *rank, const int *cnt, int T, int k, int expert_lo,
                          int n_local, int *perm, int *inv) {
    __shared__ int off[kExperts];
    __shared__ int wsum[8];
    const int tid = threadIdx.x;   // 256 threads
    const int c = tid < n_local ? cnt[tid] : 0;
    int x = c;
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    int base = 0;
    for (int i = 0; i < warp; ++i) base += wsum[i];
    off[tid] = base + x - c;
    __syncthreads();
    const int i = blockIdx.x * blockDim.x + tid;
    if (i >= T * k) return;
    const int t = i / k, s = i - t * k;
    const int rk = rank[(size_t)t * kMaxK + s];
    int pos = -1;
    if (rk >= 0) {
        pos = off[(int)idx[(size_t)t * kMaxK + s] - expert_lo] + rk;
        perm[pos] = t;
    }
    inv[(size_t)t * kMaxK + s] = pos;
}

// out[t][c..c+8) = h_mid + sum_s w_s * Y[pos(t,s)] + sigmoid(score_t) * Y[shared(t)]
__global__ void k_combine(const uint16_t *y, const float *w, const int *inv, const float *score, const float *h_mid,
                          int T, int k, int shared_base, void *out, int out_bf16) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // 8-column chunk
    if (i >= T * (kHidden / 8)) return;
    const int t = i >> 8, c = (i & 255) * 8;
    float moe[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < k; ++s) {
        const int p = inv[(size_t)t * kMaxK + s];
        if (p < 0) continue;
        const float ws = w[(size_t)t * kMaxK + s];
        const uint4 q = *reinterpret_cast<const uint4 *>(y + (size_t)p * kHidden + c);
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            moe[2 * j] += ws * bf16_lo(u[j]);
            moe[2 * j + 1] += ws * bf16_hi(u[j]);
        }
    }
    const float sg = 1.f / (1.f + expf(-score[t]));
    const uint4 q = *reinterpret_cast<const uint4 *>(y + (size_t)(shared_base + t) * kHidden + c);
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
    float o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        o[2 * j] = sg * bf16_lo(u[j]);
        o[2 * j + 1] = sg * bf16_hi(u[j]);
    }
    float hm[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (h_mid) {
        const float4 a = reinterpret_cast<const float4 *>(h_mid + (size_t)t * kHidden + c)[0];
        const float4 b = reinterpret_cast<const float4 *>(h_mid + (size_t)t * kHidden + c)[1];
        hm[0] = a.x; hm[1] = a.y; hm[2] = a.z; hm[3] = a.w; hm[4] = b.x; hm[5] = b.y; hm[6] = b.z; hm[7] = b.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = hm[j] + moe[j] + o[j];
    if (out_bf16) {
        reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out) + (size_t)t * kHidden + c)[0] =
            make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
    } else {
        float4 *op = reinterpret_cast<float4 *>(static_cast<float *>(out) + (size_t)t * kHidden + c);
        op[0] = make_float4(o[0], o[1], o[2], o[3]);
        op[1] = make_float4(o[4], o[5], o[6], o[7]);
    }
}

// ------------------------------------------------------------- host side ----

namespace {

struct Guard {
    int prev = -1;
    explicit Guard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~Guard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

constexpr int kGemmSmemMax = 227 * 1024;

// 4D tiled map: (inner elements, 16 rows, bands, groups); box (box0, 16, 8, 1).
bool make_map(BatchedState *B, CUtensorMap *m, const void *base, bool u32, uint64_t d0, uint64_t row_stride,
              uint64_t bands, uint64_t band_stride, uint64_t groups, uint64_t group_stride, uint32_t box0) {
    const cuuint64_t dims[4] = {d0, 16, bands, groups};
    const cuuint64_t strides[3] = {row_stride, band_stride, group_stride};
    const cuuint32_t box[4] = {box0, 16, 8, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    const CUresult r = B->encode(m, u32 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 4,
                                 const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Weight (+ scale/bias) maps of one q4/q2/bf16 matrix whose rows are `row_stride` bytes
// apart inside bands of 16 rows `band_stride` apart, groups (experts) `group_stride`
// apart. s_off/b_off: byte offsets of the scales / biases from `base`; their rows are
// s_row_stride bytes apart (the weight row stride for row-interleaved dense matrices).
bool make_matrix_maps(BatchedState *B, GemmProblem &pr, int m, const uint8_t *base, int fmt, int cols,
                      uint64_t row_stride, uint64_t bands, uint64_t band_stride, uint64_t groups, uint64_t group_stride,
                      size_t s_off, size_t b_off, uint64_t s_row_stride) {
    if (fmt == kAFmtBf16)
        return make_map(B, &pr.tw[m], base, false, cols, row_stride, bands, band_stride, groups, group_stride, 64);
    const int vpw = fmt == kAFmtQ4 ? 8 : 16;
    const int ng = cols / 64;
    return make_map(B, &pr.tw[m], base, true, cols / vpw, row_stride, bands, band_stride, groups, group_stride,
                    64 / vpw) &&
           make_map(B, &pr.ts[m], base + s_off, false, ng, s_row_stride, bands, band_stride, groups, group_stride, 8) &&
           make_map(B, &pr.tb[m], base + b_off, false, ng, s_row_stride, bands, band_stride, groups, group_stride, 8);
}

cudaError_t launch_gemm(nmoe_moe_ctx *ctx, GemmParams &P, cudaStream_t st) {
    int raw = 0;
    for (int i = 0; i < P.n_prob; ++i) raw = max(raw, P.prob[i].n_mat * raw_mat_bytes(P.prob[i].fmt));
    P.raw_stage = raw;
    P.sr = std::min(8, std::max(2, 65536 / raw));
    P.err = ctx->d_err;
    P.timeout_ns = ctx->batched->timeout_ns;
    const size_t smem = 1024 + kGemmSA * 2 * kGemmAStage + kGemmSB * kGemmBStage + kGemmSS * 2 * kGemmScStage +
                        (size_t)P.sr * raw + sizeof(GemmSmem);
    k_moe_gemm<<<ctx->num_sms, kGemmThreads, smem, st>>>(P);
    return cudaGetLastError();
}

}  // namespace

int nmoe_batched_init(nmoe_moe_ctx *ctx) {
    BatchedState *B = new (std::nothrow) BatchedState();
    if (B == nullptr) return NMOE_ENOMEM;
    ctx->batched = B;
    if (const char *t = getenv("NMOE_WAIT_TIMEOUT_MS")) B->timeout_ns = (uint64_t)atoll(t) * 1000000ull;
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr) {
        nmoe_ctx_set_error(ctx, "cuTensorMapEncodeTiled unavailable");
        return NMOE_ECUDA;
    }
    B->encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    cudaError_t e = cudaFuncSetAttribute(k_moe_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmemMax);
    if (e != cudaSuccess) {
        nmoe_ctx_set_error(ctx, "gemm smem attribute: %s", cudaGetErrorString(e));
        return NMOE_ECUDA;
    }
    const int tm = ctx->cfg.t_max;
    B->t_max = tm;
    if (tm <= 0) return NMOE_OK;
    const size_t T = (size_t)tm;
    struct { void **p; size_t bytes; } al[] = {
        {(void **)&B->xh, T * kHidden * 2},       {(void **)&B->xl, T * kHidden * 2},
        {(void **)&B->logits, T * kExperts * 4},  {(void **)&B->score, T * 4},
        {(void **)&B->w, T * kMaxK * 4},          {(void **)&B->idx, T * kMaxK * 4},
        {(void **)&B->rank, T * kMaxK * 4},       {(void **)&B->inv, T * kMaxK * 4},
        {(void **)&B->perm, T * kMaxK * 4},       {(void **)&B->cnt, kExperts * 4},
        {(void **)&B->act, T * 9 * kInter * 2},   {(void **)&B->y, T * 9 * kHidden * 2},
    };
    for (auto &a : al) {
        e = cudaMalloc(a.p, a.bytes);
        if (e == cudaSuccess) e = cudaMemset(*a.p, 0, a.bytes);
        if (e != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "batched workspace (t_max=%d): %s", tm, cudaGetErrorString(e));
            return e == cudaErrorMemoryAllocation ? NMOE_ENOMEM : NMOE_ECUDA;
        }
    }
    return NMOE_OK;
}

void nmoe_batched_destroy(nmoe_moe_ctx *ctx) {
    BatchedState *B = ctx->batched;
    if (B == nullptr) return;
    void *ps[] = {B->xh, B->xl, B->logits, B->score, B->w, B->idx, B->rank, B->inv, B->perm, B->cnt, B->act, B->y};
    for (void *p : ps)
        if (p) cudaFree(p);
    delete B;
    ctx->batched = nullptr;
}

extern "C" int nmoe_moe_forward_batched(nmoe_moe_ctx *ctx, int layer, int T, int k, const void *x, int x_dtype,
                                        const float *h_mid, void *out, int out_dtype, uint32_t *idx_out,
                                        float *w_out, void *stream) {
    int rc = nmoe_ctx_check_call(ctx, layer, k, x_dtype);
    if (rc != NMOE_OK) return rc;
    BatchedState *B = ctx->batched;
    if (T < 0 || T > B->t_max) {
        nmoe_ctx_set_error(ctx, "T=%d outside [0, t_max=%d]", T, B->t_max);
        return NMOE_EINVAL;
    }
    if (out_dtype != NMOE_DTYPE_F32 && out_dtype != NMOE_DTYPE_BF16) {
        nmoe_ctx_set_error(ctx, "out_dtype must be NMOE_DTYPE_F32 or NMOE_DTYPE_BF16");
        return NMOE_EINVAL;
    }
    if (T > 0 && (x == nullptr || out == nullptr)) {
        nmoe_ctx_set_error(ctx, "x and out are required");
        return NMOE_EINVAL;
    }
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16 ||
        reinterpret_cast<uintptr_t>(h_mid) % 16) {
        nmoe_ctx_set_error(ctx, "x, out and h_mid must be 16-byte aligned");
        return NMOE_EINVAL;
    }
    if (ctx->cfg.world_size > 1) {
        nmoe_ctx_set_error(ctx, "expert-parallel forward_batched is not available in this build");
        return NMOE_EINVAL;
    }
    B->last_T = T;
    if (T == 0) return NMOE_OK;
    Guard guard(ctx->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool xf32 = x_dtype == NMOE_DTYPE_F32;
    const int bits = ctx->cfg.quant_bits;
    const int rfmt = ctx->cfg.router_dtype == NMOE_DTYPE_Q4 ? kAFmtQ4 : kAFmtBf16;
    const int sfmt = ctx->cfg.shared_dtype == NMOE_DTYPE_Q4 ? kAFmtQ4 : kAFmtBf16;
    const DenseArena DA = dense_arena(ctx->cfg.router_dtype, ctx->cfg.shared_dtype);
    const uint8_t *dense = ctx->d_dense + (size_t)layer * ctx->dense_layer_bytes;
    const uint8_t *experts = ctx->d_experts + (size_t)layer * ctx->expert_layer_bytes;
    const PackGeo pg = pack_geo(bits);
    cudaError_t e;

    // 1. x planes, counts cleared
    k_prep<<<(T * 256 + 255) / 256, 256, 0, st>>>(x, xf32, T, B->xh, B->xl, B->cnt);

    // 2. router logits
    {
        GemmParams P;
        memset(&P, 0, sizeof P);
        P.n_prob = 1;
        GemmProblem &r = P.prob[0];
        r.fmt = rfmt;
        r.n_mat = 1;
        r.K = kHidden;
        r.m_tiles = 2;
        r.n_groups = 1;
        r.cnt_const = T;
        r.b_hi = B->xh;
        r.b_lo = B->xl;
        r.passes = kPassHiHi | (xf32 ? kPassHiLo : 0) | (rfmt == kAFmtQ4 ? kPassLoHi : 0);
        r.split = 1;
        r.epi = kEpiF32;
        r.ld_out = kExperts;
        r.out = B->logits;
        const uint8_t *rb = dense + DA.router;
        if (!make_matrix_maps(B, r, 0, rb, rfmt, kHidden, DA.rrow, 16, 16ull * DA.rrow, 1, 256ull * DA.rrow, 1024, 1088, DA.rrow)) {
            nmoe_ctx_set_error(ctx, "router tensor map");
            return NMOE_ECUDA;
        }
        if ((e = launch_gemm(ctx, P, st)) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "router gemm launch: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
    }

    // 3. routing
    {
        RouteArgs a;
        a.logits = B->logits;
        a.x = x;
        a.x_f32 = xf32;
        a.gvec = dense + DA.gvec;
        a.gvec_q4 = sfmt == kAFmtQ4;
        a.T = T;
        a.k = k;
        a.num_experts = ctx->cfg.num_experts;
        a.expert_lo = ctx->expert_lo;
        a.n_local = ctx->n_local;
        a.idx = B->idx;
        a.w = B->w;
        a.score = B->score;
        a.rank = B->rank;
        a.cnt = B->cnt;
        a.idx_out = idx_out;
        a.w_out = w_out;
        a.err = ctx->d_err;
        k_route<<<(T + kRouteWarps - 1) / kRouteWarps, kRouteWarps * 32, 0, st>>>(a);
        k_scatter<<<(T * k + 255) / 256, 256, 0, st>>>(B->idx, B->rank, B->cnt, T, k, ctx->expert_lo, ctx->n_local,
                                                       B->perm, B->inv);
    }
    const int shared_base = T * k;

    // 4. gate/up + SwiGLU: routed positions and the shared expert
    {
        GemmParams P;
        memset(&P, 0, sizeof P);
        P.n_prob = 2;
        GemmProblem &r = P.prob[0];
        r.fmt = bits;
        r.n_mat = 2;
        r.K = kHidden;
        r.m_tiles = 4;
        r.n_groups = ctx->n_local;
        r.cnt = B->cnt;
        r.perm = B->perm;
        r.b_hi = B->xh;
        r.passes = kPassHiHi;
        r.epi = kEpiSwiGLU;
        r.ld_out = kInter;
        r.out = B->act;
        const uint32_t rowb = pg.wgu * 4;
        bool ok = make_matrix_maps(B, r, 0, experts, bits, kHidden, rowb, 32, pg.bp, ctx->n_local, pg.esz,
                                   2 * pg.tile_band_gu, 2 * pg.tile_band_gu + 1024, 64);
        ok = ok && make_matrix_maps(B, r, 1, experts + pg.tile_band_gu, bits, kHidden, rowb, 32, pg.bp, ctx->n_local,
                                    pg.esz, pg.tile_band_gu + 2048, pg.tile_band_gu + 3072, 64);
        GemmProblem &s = P.prob[1];
        s.fmt = sfmt;
        s.n_mat = 2;
        s.K = kHidden;
        s.m_tiles = 4;
        s.n_groups = 1;
        s.cnt_const = T;
        s.b_hi = B->xh;
        s.passes = kPassHiHi;
        s.epi = kEpiSwiGLU;
        s.ld_out = kInter;
        s.out = B->act;
        s.out_base = shared_base;
        const uint8_t *sp = dense + DA.spairs;
        const uint64_t ps = 2ull * DA.srow;   // pair stride
        if (sfmt == kAFmtQ4) {
            ok = ok && make_matrix_maps(B, s, 0, sp, sfmt, kHidden, ps, 32, 16 * ps, 1, 512 * ps, 2048, 2112, ps);
            ok = ok && make_matrix_maps(B, s, 1, sp + 1024, sfmt, kHidden, ps, 32, 16 * ps, 1, 512 * ps, 2176 - 1024,
                                        2240 - 1024, ps);
        } else {
            ok = ok && make_matrix_maps(B, s, 0, sp, sfmt, kHidden, ps, 32, 16 * ps, 1, 512 * ps, 0, 0, ps);
            ok = ok && make_matrix_maps(B, s, 1, sp + DA.srow, sfmt, kHidden, ps, 32, 16 * ps, 1, 512 * ps, 0, 0, ps);
        }
        if (!ok) {
            nmoe_ctx_set_error(ctx, "gate/up tensor maps");
            return NMOE_ECUDA;
        }
        if ((e = launch_gemm(ctx, P, st)) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "gate/up gemm launch: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
    }

    // 5. down: routed positions and the shared expert
    {
        GemmParams P;
        memset(&P, 0, sizeof P);
        P.n_prob = 2;
        GemmProblem &r = P.prob[0];
        r.fmt = bits;
        r.n_mat = 1;
        r.K = kInter;
        r.m_tiles = 16;
        r.n_groups = ctx->n_local;
        r.cnt = B->cnt;
        r.b_hi = B->act;
        r.passes = kPassHiHi;
        r.epi = kEpiBf16;
        r.ld_out = kHidden;
        r.out = B->y;
        bool ok = make_matrix_maps(B, r, 0, experts + pg.gu_bytes, bits, kInter, pg.wd * 4, 128, pg.db, ctx->n_local,
                                   pg.esz, pg.tile_band_d, pg.tile_band_d + 256, 16);
        GemmProblem &s = P.prob[1];
        s.fmt = sfmt;
        s.n_mat = 1;
        s.K = kInter;
        s.m_tiles = 16;
        s.n_groups = 1;
        s.cnt_const = T;
        s.in_base = shared_base;
        s.out_base = shared_base;
        s.b_hi = B->act;
        s.passes = kPassHiHi;
        s.epi = kEpiBf16;
        s.ld_out = kHidden;
        s.out = B->y;
        const uint64_t rs = DA.sdrow;
        ok = ok && make_matrix_maps(B, s, 0, dense + DA.sdown, sfmt, kInter, rs, 128, 16 * rs, 1, 2048 * rs, 256, 272, rs);
        if (!ok) {
            nmoe_ctx_set_error(ctx, "down tensor maps");
            return NMOE_ECUDA;
        }
        if ((e = launch_gemm(ctx, P, st)) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "down gemm launch: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
    }

    // 6. combine
    k_combine<<<(T * 256 + 255) / 256, 256, 0, st>>>(B->y, B->w, B->inv, B->score, h_mid, T, k, shared_base, out,
                                                     out_dtype == NMOE_DTYPE_BF16);
    if ((e = cudaGetLastError()) != cudaSuccess) {
        nmoe_ctx_set_error(ctx, "batched launch: %s", cudaGetErrorString(e));
        return NMOE_ECUDA;
    }
    return NMOE_OK;
}

extern "C" int nmoe_moe_debug_logits(nmoe_moe_ctx *ctx, float *out, int T) {
    if (ctx == nullptr || ctx->batched == nullptr || out == nullptr || T < 0 || T > ctx->batched->last_T) {
        if (ctx) nmoe_ctx_set_error(ctx, "debug_logits: bad arguments (T must be <= the last forward_batched T)");
        return NMOE_EINVAL;
    }
    Guard guard(ctx->device);
    const cudaError_t e = cudaMemcpy(out, ctx->batched->logits, (size_t)T * kExperts * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        nmoe_ctx_set_error(ctx, "debug_logits: %s", cudaGetErrorString(e));
        return NMOE_ECUDA;
    }
    return NMOE_OK;
}
