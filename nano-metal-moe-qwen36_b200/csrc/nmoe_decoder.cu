// nmoe_decoder.cu -- one whole decode step on the GPU.
//
// The C restatement of NMOEProcessToken (src/runtime.m:3712-3805) and of the two layer
// steps it calls, NMOELinearAttentionStepMetal (src/runtime.m:3335-3500) and
// NMOEFullAttentionStepMetal (src/runtime.m:3001-3180): embedding row, 40 layers (full
// attention when (l + 1) % 4 == 0, src/runtime.m:2373), final RMSNorm and LM head. The
// per-layer pieces are this library's kernels: q4 matrix-vector products (below) for the
// projections, nmoe_linear_attn_step / nmoe_full_attn_step for the attention cores,
// nmoe_moe_forward for the MoE block (the residual as h_mid), nmoe_lm_head_argmax.
//
// The matrix-vector product follows the reference's dequant matvec (form 0,
// metal/kernels.metal:192-238): acc += fma(q, scale, bias) * x, fp32. One warp per row;
// lane l takes 16-byte chunks l, l + 32, ... of the row (coalesced), x from shared memory.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "nmoe/moe_cuda.h"

namespace nmoe {
int full_attn_step_dev(const nmoe_full_attn_weights *w, const float *q, const float *k_new, const float *v_new,
                       float *k_cache, float *v_cache, int max_positions, const int *d_position, float *out,
                       void *workspace, cudaStream_t st);
}

namespace {

constexpr int kHidden = 2048;
constexpr int kMvWarps = 8;

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }
// exact float of a nibble (0..15) without a conversion instruction
__device__ __forceinline__ float nib(uint32_t w, int i) {
    return __int_as_float(0x4B000000 | ((w >> (4 * i)) & 0xFu)) - 8388608.0f;
}

// out = x * rsqrt(mean(x^2) + 1e-6) * (w + 1) over 2048 (the reference's input / post
// norms: NMOEEncodeRMSNormTensor(..., YES, 1e-6f), metal/kernels.metal:862-900).
__global__ void __launch_bounds__(256) k_rmsnorm(const float *x, const uint16_t *w, float *out) {
    __shared__ float red[8];
    const int tid = threadIdx.x;
    float v[8], ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        v[j] = x[tid + 256 * j];
        ss += v[j] * v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    const float inv = rsqrtf(t / (float)kHidden + 1e-6f);
#pragma unroll
    for (int j = 0; j < 8; ++j) out[tid + 256 * j] = v[j] * inv * (bf16f(w[tid + 256 * j]) + 1.0f);
}

// Up to four q4 matrices over one x, one launch: y_m[r] = sum_c fma(q, s, b) * x[c]
// (+ resid[r] for a single matrix), K columns (2048 or 4096). With norm_w set, x is first
// replaced by its RMSNorm (weight + 1, eps 1e-6) computed in every CTA exactly as
// k_rmsnorm does (same thread split and summation order: the same floats), so the input
// norm of a layer costs no launch of its own. x sits in shared memory in 32-column pieces
// padded to 36 floats: lane l reads the piece of its chunk l + 32 c as eight float4, and
// the 8 lanes of each quarter-warp phase hit 8 different 16-byte bank groups (piece stride
// 9 units), where an unpadded layout (stride 8 units) puts them all on one.
struct MvSeg {
    const uint32_t *w;
    const uint16_t *s, *b;
    float *y;
    int row_end;   // cumulative rows through this matrix
};
struct MvArgs {
    MvSeg seg[4];
    int nseg;
    const float *x, *resid;
    const uint16_t *norm_w;
};

template <int K>
__global__ void __launch_bounds__(kMvWarps * 32) k_q4_matvec(const MvArgs a) {
    __shared__ __align__(16) float xs[K / 32 * 36];
    __shared__ float red[kMvWarps];
    const int tid = threadIdx.x;
    if (a.norm_w != nullptr) {   // K == kHidden, 256 threads: k_rmsnorm's arithmetic
        float v[8], ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[j] = a.x[tid + 256 * j];
            ss += v[j] * v[j];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) t += red[i];
        const float inv = rsqrtf(t / (float)kHidden + 1e-6f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = tid + 256 * j;
            xs[(i >> 5) * 36 + (i & 31)] = v[j] * inv * (bf16f(a.norm_w[i]) + 1.0f);
        }
    } else {
        for (int i = tid; i < K; i += kMvWarps * 32) xs[(i >> 5) * 36 + (i & 31)] = a.x[i];
    }
    __syncthreads();
    const int warp = tid >> 5, lane = tid & 31;
    constexpr int kChunks = K / 32 / 32;   // 16-byte chunks (32 columns) per lane
    const int rows = a.seg[a.nseg - 1].row_end;
    for (int gr = blockIdx.x * kMvWarps + warp; gr < rows; gr += gridDim.x * kMvWarps) {
        int m = 0;
        while (m + 1 < a.nseg && gr >= a.seg[m].row_end) ++m;
        const MvSeg &sg = a.seg[m];
        const int r = m ? gr - a.seg[m - 1].row_end : gr;
        const uint4 *wr = reinterpret_cast<const uint4 *>(sg.w + (size_t)r * (K / 8));
        const uint16_t *sr = sg.s + (size_t)r * (K / 64), *br = sg.b + (size_t)r * (K / 64);
        uint4 u[kChunks];
#pragma unroll
        for (int c = 0; c < kChunks; ++c) u[c] = __ldcs(wr + lane + 32 * c);
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
            const int chunk = lane + 32 * c, g = chunk >> 1;   // 32 columns, half a group
            const float sv = bf16f(sr[g]), bv = bf16f(br[g]);
            const uint32_t ws[4] = {u[c].x, u[c].y, u[c].z, u[c].w};
            const float4 *xp = reinterpret_cast<const float4 *>(xs + 36 * chunk);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 xv = xp[q];
                const uint32_t wd = ws[q >> 1];
                const int i0 = 4 * (q & 1);
                acc = fmaf(fmaf(nib(wd, i0), sv, bv), xv.x, acc);
                acc = fmaf(fmaf(nib(wd, i0 + 1), sv, bv), xv.y, acc);
                acc = fmaf(fmaf(nib(wd, i0 + 2), sv, bv), xv.z, acc);
                acc = fmaf(fmaf(nib(wd, i0 + 3), sv, bv), xv.w, acc);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) sg.y[r] = acc + (a.resid ? a.resid[r] : 0.f);
    }
}

// Embedding row of *token (q4: dequant_row, metal/kernels.metal nmoe_dequant_row; bf16:
// widened), 256 threads x 8 columns.
__global__ void __launch_bounds__(256) k_embed(const uint32_t *tok, int vocab, int q4, const void *w, const uint16_t *s,
                                               const uint16_t *b, float *out) {
    uint32_t t = *tok;
    if (t >= (uint32_t)vocab) t = 0;
    const int c0 = 8 * threadIdx.x;
    if (q4) {
        const uint32_t word = static_cast<const uint32_t *>(w)[(size_t)t * (kHidden / 8) + threadIdx.x];
        const float sv = bf16f(s[(size_t)t * (kHidden / 64) + c0 / 64]), bv = bf16f(b[(size_t)t * (kHidden / 64) + c0 / 64]);
#pragma unroll
        for (int i = 0; i < 8; ++i) out[c0 + i] = fmaf(nib(word, i), sv, bv);
    } else {
        const uint16_t *row = static_cast<const uint16_t *>(w) + (size_t)t * kHidden;
#pragma unroll
        for (int i = 0; i < 8; ++i) out[c0 + i] = bf16f(row[c0 + i]);
    }
}

}  // namespace

// ------------------------------------------------------------------ host side ----

namespace {

struct DevQ4 {   // a q4 matrix in device memory
    uint32_t *w = nullptr;
    uint16_t *s = nullptr, *b = nullptr;
    int rows = 0, cols = 0;
};

struct LinearLayer {
    uint16_t *in_norm = nullptr, *post_norm = nullptr, *conv_w = nullptr, *dt_bias = nullptr, *norm_w = nullptr;
    float *A_log = nullptr;
    DevQ4 qkv, z, beta, alpha, out;
    float *conv_state = nullptr, *delta_state = nullptr;
    bool set = false;
};

struct FullLayer {
    uint16_t *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    DevQ4 q, k, v, o;
    float *k_cache = nullptr, *v_cache = nullptr;
    bool set = false;
};

bool is_full(int l) { return ((l + 1) % 4) == 0; }

__global__ void k_set_position(int *p, int v) { *p = v; }

}  // namespace

struct nmoe_decoder {
    nmoe_moe_ctx *moe = nullptr;
    int num_layers = 0, k = 8, max_pos = 0, device = 0;
    std::vector<LinearLayer> lin;
    std::vector<FullLayer> full;
    // globals
    int vocab = 0, embed_q4 = 0, head_dtype = NMOE_DTYPE_Q4;
    void *embed_w = nullptr;
    uint16_t *embed_s = nullptr, *embed_b = nullptr, *final_norm = nullptr;
    void *head_w = nullptr;
    uint16_t *head_s = nullptr, *head_b = nullptr;
    bool globals = false;
    // activations
    float *h0 = nullptr, *h1 = nullptr, *xn = nullptr, *h2 = nullptr, *qkv = nullptr, *z = nullptr, *beta = nullptr,
          *alpha = nullptr, *attn = nullptr, *q = nullptr, *kk = nullptr, *vv = nullptr;
    void *fa_ws = nullptr, *lm_ws = nullptr;
    int *d_pos = nullptr;   // the step's position, written by a one-thread launch before the step
    // the step as one CUDA graph, captured for one (token, next, hidden) pointer triple
    cudaGraphExec_t graph = nullptr;
    cudaStream_t cap = nullptr;
    const void *g_token = nullptr, *g_next = nullptr, *g_hidden = nullptr;
    bool use_graph = true;
    std::vector<void *> allocs;
    char err[512] = {0};
};

namespace {

void drop_graph(nmoe_decoder *d) {
    if (d->graph) cudaGraphExecDestroy(d->graph);
    d->graph = nullptr;
}

int dfail(nmoe_decoder *d, int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(d->err, sizeof d->err, fmt, ap);
    va_end(ap);
    return code;
}

template <class T>
bool dalloc(nmoe_decoder *d, T **p, size_t bytes) {
    void *v = nullptr;
    if (cudaMalloc(&v, bytes) != cudaSuccess) return false;
    d->allocs.push_back(v);
    *p = static_cast<T *>(v);
    return true;
}

template <class T>
bool dcopy(nmoe_decoder *d, T **p, const void *host, size_t bytes) {
    if (host == nullptr) return false;
    if (*p == nullptr && !dalloc(d, p, bytes)) return false;
    return cudaMemcpy(*p, host, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
}

bool q4copy(nmoe_decoder *d, DevQ4 &m, const nmoe_tensor &t, int rows, int cols) {
    m.rows = rows;
    m.cols = cols;
    return dcopy(d, &m.w, t.weight, (size_t)rows * cols / 2) && dcopy(d, &m.s, t.scales, (size_t)rows * cols / 64 * 2) &&
           dcopy(d, &m.b, t.biases, (size_t)rows * cols / 64 * 2);
}

// One launch of k_q4_matvec over n (<= 4) matrices of the same width; x normalised
// first when norm_w is set (then the width is kHidden); resid only with n == 1.
cudaError_t matvec(const DevQ4 *const *m, float *const *y, int n, const float *x, const uint16_t *norm_w,
                   const float *resid, cudaStream_t st) {
    MvArgs a{};
    int rows = 0;
    for (int i = 0; i < n; ++i) {
        rows += m[i]->rows;
        a.seg[i] = MvSeg{m[i]->w, m[i]->s, m[i]->b, y[i], rows};
    }
    a.nseg = n;
    a.x = x;
    a.resid = resid;
    a.norm_w = norm_w;
    const int blocks = (rows + kMvWarps - 1) / kMvWarps;
    if (m[0]->cols == 2048) k_q4_matvec<2048><<<blocks, kMvWarps * 32, 0, st>>>(a);
    else k_q4_matvec<4096><<<blocks, kMvWarps * 32, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t matvec(const DevQ4 &m, const float *x, const float *resid, float *y, cudaStream_t st) {
    const DevQ4 *mm[1] = {&m};
    float *yy[1] = {y};
    return matvec(mm, yy, 1, x, nullptr, resid, st);
}

}  // namespace

extern "C" const char *nmoe_decoder_error(const nmoe_decoder *d) { return d ? d->err : "null decoder"; }

extern "C" nmoe_decoder *nmoe_decoder_create(nmoe_moe_ctx *moe, int num_layers, int k, int max_positions, int *status) {
    auto fail_create = [&](int code) -> nmoe_decoder * {
        if (status) *status = code;
        return nullptr;
    };
    if (moe == nullptr || num_layers < 1 || num_layers > 64 || k < 1 || k > NMOE_MAX_K || max_positions < 1)
        return fail_create(NMOE_EINVAL);
    nmoe_decoder *d = new nmoe_decoder();
    d->moe = moe;
    d->num_layers = num_layers;
    d->k = k;
    d->max_pos = max_positions;
    cudaGetDevice(&d->device);
    d->lin.resize(num_layers);
    d->full.resize(num_layers);
    bool ok = dalloc(d, &d->h0, kHidden * 4) && dalloc(d, &d->h1, kHidden * 4) && dalloc(d, &d->xn, kHidden * 4) &&
              dalloc(d, &d->h2, kHidden * 4) && dalloc(d, &d->qkv, 8192 * 4) && dalloc(d, &d->z, 4096 * 4) &&
              dalloc(d, &d->beta, 32 * 4) && dalloc(d, &d->alpha, 32 * 4) && dalloc(d, &d->attn, 4096 * 4) &&
              dalloc(d, &d->q, 8192 * 4) && dalloc(d, &d->kk, 512 * 4) && dalloc(d, &d->vv, 512 * 4) &&
              dalloc(d, &d->fa_ws, nmoe_full_attn_workspace_bytes()) && dalloc(d, &d->lm_ws, nmoe_lm_head_workspace_bytes()) &&
              dalloc(d, &d->d_pos, 16);
    if (ok) ok = cudaStreamCreateWithFlags(&d->cap, cudaStreamNonBlocking) == cudaSuccess;
    const char *ge = getenv("NMOE_DECODER_GRAPH");
    d->use_graph = !(ge && ge[0] == '0');
    for (int l = 0; ok && l < num_layers; ++l) {
        if (is_full(l)) {
            const size_t cache = (size_t)max_positions * 2 * 256 * 4;
            ok = dalloc(d, &d->full[l].k_cache, cache) && dalloc(d, &d->full[l].v_cache, cache);
        } else {
            ok = dalloc(d, &d->lin[l].conv_state, 3 * 8192 * 4) && dalloc(d, &d->lin[l].delta_state, 32 * 128 * 128 * 4);
        }
    }
    if (ok) ok = cudaMemset(d->lm_ws, 0, nmoe_lm_head_workspace_bytes()) == cudaSuccess;
    if (ok) ok = nmoe_decoder_reset(d, nullptr) == NMOE_OK;
    if (!ok) {
        nmoe_decoder_destroy(d);
        return fail_create(NMOE_ENOMEM);
    }
    if (status) *status = NMOE_OK;
    return d;
}

extern "C" void nmoe_decoder_destroy(nmoe_decoder *d) {
    if (d == nullptr) return;
    if (d->graph) cudaGraphExecDestroy(d->graph);
    if (d->cap) cudaStreamDestroy(d->cap);
    for (void *p : d->allocs) cudaFree(p);
    delete d;
}

extern "C" int nmoe_decoder_reset(nmoe_decoder *d, void *stream) {
    if (d == nullptr) return NMOE_EINVAL;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int l = 0; l < d->num_layers; ++l) {
        if (is_full(l)) continue;   // the caches are written before they are read
        if (cudaMemsetAsync(d->lin[l].conv_state, 0, 3 * 8192 * 4, st) != cudaSuccess ||
            cudaMemsetAsync(d->lin[l].delta_state, 0, 32 * 128 * 128 * 4, st) != cudaSuccess)
            return dfail(d, NMOE_ECUDA, "state reset");
    }
    return NMOE_OK;
}

extern "C" int nmoe_decoder_set_linear_layer(nmoe_decoder *d, int l, const nmoe_linear_layer_host *w) {
    if (d == nullptr || w == nullptr || l < 0 || l >= d->num_layers) return NMOE_EINVAL;
    drop_graph(d);
    if (is_full(l)) return dfail(d, NMOE_EINVAL, "layer %d is a full-attention layer", l);
    LinearLayer &L = d->lin[l];
    const bool ok = dcopy(d, &L.in_norm, w->input_norm, kHidden * 2) && dcopy(d, &L.post_norm, w->post_norm, kHidden * 2) &&
                    q4copy(d, L.qkv, w->qkv, 8192, 2048) && q4copy(d, L.z, w->z, 4096, 2048) &&
                    q4copy(d, L.beta, w->beta, 32, 2048) && q4copy(d, L.alpha, w->alpha, 32, 2048) &&
                    q4copy(d, L.out, w->out, 2048, 4096) && dcopy(d, &L.conv_w, w->conv_w, 8192 * 4 * 2) &&
                    dcopy(d, &L.A_log, w->A_log, 32 * 4) && dcopy(d, &L.dt_bias, w->dt_bias, 32 * 2) &&
                    dcopy(d, &L.norm_w, w->norm_w, 128 * 2);
    if (!ok) return dfail(d, NMOE_EINVAL, "layer %d: a weight is missing or the copy failed", l);
    L.set = true;
    return NMOE_OK;
}

extern "C" int nmoe_decoder_set_full_layer(nmoe_decoder *d, int l, const nmoe_full_layer_host *w) {
    if (d == nullptr || w == nullptr || l < 0 || l >= d->num_layers) return NMOE_EINVAL;
    drop_graph(d);
    if (!is_full(l)) return dfail(d, NMOE_EINVAL, "layer %d is a linear-attention layer", l);
    FullLayer &F = d->full[l];
    const bool ok = dcopy(d, &F.in_norm, w->input_norm, kHidden * 2) && dcopy(d, &F.post_norm, w->post_norm, kHidden * 2) &&
                    q4copy(d, F.q, w->q, 8192, 2048) && q4copy(d, F.k, w->k, 512, 2048) &&
                    q4copy(d, F.v, w->v, 512, 2048) && q4copy(d, F.o, w->o, 2048, 4096) &&
                    dcopy(d, &F.q_norm, w->q_norm, 256 * 2) && dcopy(d, &F.k_norm, w->k_norm, 256 * 2);
    if (!ok) return dfail(d, NMOE_EINVAL, "layer %d: a weight is missing or the copy failed", l);
    F.set = true;
    return NMOE_OK;
}

extern "C" int nmoe_decoder_set_globals(nmoe_decoder *d, int vocab, int embed_dtype, const nmoe_tensor *embed,
                                        const uint16_t *final_norm, int head_dtype, const nmoe_tensor *lm_head) {
    if (d == nullptr || embed == nullptr || lm_head == nullptr || vocab < 1) return NMOE_EINVAL;
    drop_graph(d);
    if ((embed_dtype != NMOE_DTYPE_Q4 && embed_dtype != NMOE_DTYPE_BF16) ||
        (head_dtype != NMOE_DTYPE_Q4 && head_dtype != NMOE_DTYPE_BF16))
        return dfail(d, NMOE_EINVAL, "embedding and head dtypes: NMOE_DTYPE_Q4 or NMOE_DTYPE_BF16");
    d->vocab = vocab;
    d->embed_q4 = embed_dtype == NMOE_DTYPE_Q4;
    d->head_dtype = head_dtype;
    const size_t V = (size_t)vocab;
    bool ok;
    if (d->embed_q4)
        ok = dcopy(d, &d->embed_w, embed->weight, V * 1024) && dcopy(d, &d->embed_s, embed->scales, V * 64) &&
             dcopy(d, &d->embed_b, embed->biases, V * 64);
    else
        ok = dcopy(d, &d->embed_w, embed->weight, V * 4096);
    ok = ok && dcopy(d, &d->final_norm, final_norm, kHidden * 2);
    if (head_dtype == NMOE_DTYPE_Q4)
        ok = ok && dcopy(d, &d->head_w, lm_head->weight, V * 1024) && dcopy(d, &d->head_s, lm_head->scales, V * 64) &&
             dcopy(d, &d->head_b, lm_head->biases, V * 64);
    else
        ok = ok && dcopy(d, &d->head_w, lm_head->weight, V * 4096);
    if (!ok) return dfail(d, NMOE_ENOMEM, "globals: a weight is missing or the copy failed");
    d->globals = true;
    return NMOE_OK;
}

namespace {

// Every launch of one step on st; the position is read on the device from d->d_pos.
int enqueue_step(nmoe_decoder *d, const uint32_t *d_token, uint32_t *d_next, float *d_hidden, cudaStream_t st) {
    k_embed<<<1, 256, 0, st>>>(d_token, d->vocab, d->embed_q4, d->embed_w, d->embed_s, d->embed_b, d->h0);
    float *h = d->h0, *hn = d->h1;
    for (int l = 0; l < d->num_layers; ++l) {
        if (is_full(l)) {
            FullLayer &F = d->full[l];
            const DevQ4 *mm[3] = {&F.q, &F.k, &F.v};
            float *yy[3] = {d->q, d->kk, d->vv};
            if (matvec(mm, yy, 3, h, F.in_norm, nullptr, st) != cudaSuccess)
                return dfail(d, NMOE_ECUDA, "layer %d projections", l);
            nmoe_full_attn_weights aw{F.q_norm, F.k_norm};
            int rc = nmoe::full_attn_step_dev(&aw, d->q, d->kk, d->vv, F.k_cache, F.v_cache, d->max_pos, d->d_pos, d->attn,
                                              d->fa_ws, st);
            if (rc != NMOE_OK) return dfail(d, rc, "layer %d attention", l);
            if (matvec(F.o, d->attn, h, d->h2, st) != cudaSuccess) return dfail(d, NMOE_ECUDA, "layer %d o_proj", l);
            k_rmsnorm<<<1, 256, 0, st>>>(d->h2, F.post_norm, d->xn);
        } else {
            LinearLayer &L = d->lin[l];
            const DevQ4 *mm[4] = {&L.qkv, &L.z, &L.beta, &L.alpha};
            float *yy[4] = {d->qkv, d->z, d->beta, d->alpha};
            if (matvec(mm, yy, 4, h, L.in_norm, nullptr, st) != cudaSuccess)
                return dfail(d, NMOE_ECUDA, "layer %d projections", l);
            nmoe_linear_attn_weights lw{L.conv_w, L.A_log, L.dt_bias, L.norm_w};
            int rc = nmoe_linear_attn_step(&lw, d->qkv, d->z, d->alpha, d->beta, L.conv_state, L.delta_state, d->attn,
                                           st);
            if (rc != NMOE_OK) return dfail(d, rc, "layer %d linear attention", l);
            if (matvec(L.out, d->attn, h, d->h2, st) != cudaSuccess) return dfail(d, NMOE_ECUDA, "layer %d out_proj", l);
            k_rmsnorm<<<1, 256, 0, st>>>(d->h2, L.post_norm, d->xn);
        }
        int rc = nmoe_moe_forward(d->moe, l, d->k, d->xn, NMOE_DTYPE_F32, d->h2, hn, nullptr, nullptr, st);
        if (rc != NMOE_OK) return dfail(d, rc, "layer %d moe: %s", l, nmoe_moe_last_error(d->moe));
        float *t = h;
        h = hn;
        hn = t;
    }
    if (d_hidden && cudaMemcpyAsync(d_hidden, h, kHidden * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return dfail(d, NMOE_ECUDA, "hidden copy");
    nmoe_tensor head{d->head_w, d->head_s, d->head_b};
    int rc = nmoe_lm_head_argmax(&head, d->head_dtype, d->vocab, kHidden, h, NMOE_DTYPE_F32, d->final_norm, 1e-6f, 1,
                                 nullptr, d_next, d->lm_ws, st);
    if (rc != NMOE_OK) return dfail(d, rc, "lm head: %s", nmoe_lm_head_error());
    return cudaGetLastError() == cudaSuccess ? NMOE_OK : dfail(d, NMOE_ECUDA, "decode step launch");
}

}  // namespace

extern "C" int nmoe_decoder_step(nmoe_decoder *d, const uint32_t *d_token, int position, uint32_t *d_next,
                                 float *d_hidden, void *stream) {
    if (d == nullptr || d_token == nullptr || d_next == nullptr) return NMOE_EINVAL;
    if (position < 0 || position >= d->max_pos) return dfail(d, NMOE_EINVAL, "position %d outside [0, %d)", position, d->max_pos);
    if (!d->globals) return dfail(d, NMOE_EINVAL, "globals not set");
    for (int l = 0; l < d->num_layers; ++l)
        if (!(is_full(l) ? d->full[l].set : d->lin[l].set)) return dfail(d, NMOE_EINVAL, "layer %d not set", l);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    k_set_position<<<1, 1, 0, st>>>(d->d_pos, position);
    if (d->graph && d->g_token == d_token && d->g_next == d_next && d->g_hidden == d_hidden) {
        if (cudaGraphLaunch(d->graph, st) != cudaSuccess) return dfail(d, NMOE_ECUDA, "decode step graph launch");
        return NMOE_OK;
    }
    // first step with these buffers: run it directly, then capture the same launches
    // (nothing runs during a capture) for the steps after it
    drop_graph(d);
    int rc = enqueue_step(d, d_token, d_next, d_hidden, st);
    if (rc != NMOE_OK || !d->use_graph) return rc;
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(d->cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return dfail(d, NMOE_ECUDA, "decode step capture");
    rc = enqueue_step(d, d_token, d_next, d_hidden, d->cap);
    const cudaError_t ce = cudaStreamEndCapture(d->cap, &g);
    if (rc != NMOE_OK || ce != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return rc != NMOE_OK ? rc : dfail(d, NMOE_ECUDA, "decode step capture: %s", cudaGetErrorString(ce));
    }
    const cudaError_t ie = cudaGraphInstantiate(&d->graph, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
        d->graph = nullptr;
        return dfail(d, NMOE_ECUDA, "decode step graph: %s", cudaGetErrorString(ie));
    }
    d->g_token = d_token;
    d->g_next = d_next;
    d->g_hidden = d_hidden;
    return NMOE_OK;
}
