/*
 * nmoe/moe_cuda.h -- C ABI of the B200 (sm_100a) routed-MoE block for nmoe.
 *
 * This is the drop-in seam for nmoe's host (src/runtime.m): everything between the
 * post-attention RMSNorm output (`normBuffer`) and the layer output is one call here.
 * It replaces, in the reference:
 *   - the router + shared-expert encoders  NMOEEncodeRouteSharedQ4Tensors
 *     (src/runtime.m:970-1038) and the q2-mode dequant/gate-up encoders
 *     (src/runtime.m:3151-3166, 3498-3513);
 *   - routing  NMOESelectRouteTopKCPU (src/runtime.m:1498-1511) / NMOEEncodeRouteTopK
 *     (src/runtime.m:1403-1424);
 *   - the expert phase  NMOEEncodeExpertPhase (src/runtime.m:2778-2903) and its
 *     pipelined tail NMOEPipelinedExpertTail (src/runtime.m:2908-2999);
 *   - the SSD expert loader  nmoe_expert_store_open / NMOEAsyncReadExpertsRange
 *     (include/nmoe/expert_io.h:22-26, src/runtime.m:1588-1634) -- expert packs are
 *     uploaded once and stay resident in HBM.
 *
 * Conventions (mirroring include/nmoe/expert_io.h and include/nmoe/backend.h):
 *   - plain C: no CUDA or C++ types; a CUDA stream is passed as `void *` (cudaStream_t);
 *   - every call returns an int status (NMOE_OK == 0), detail in nmoe_moe_last_error();
 *   - tensors passed to forward calls are DEVICE pointers owned by the caller;
 *     weights passed to load/set calls are HOST pointers, copied into the context;
 *   - one host thread per context (the reference has one Metal queue,
 *     src/backend/metal_backend.m:271); contexts on different devices are independent.
 */
#ifndef NMOE_MOE_CUDA_H
#define NMOE_MOE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (reference: BOOL + NSError, src/expert_io.m:52-65) ---------- */
#define NMOE_OK 0
#define NMOE_EINVAL 1   /* bad argument: k outside [1,k_max], layer/expert out of range, dtype */
#define NMOE_ESIZE 2    /* pack or layout size mismatch (src/runtime.m:2445 check)            */
#define NMOE_ECUDA 3    /* CUDA runtime error (no device, launch failure, ...)                 */
#define NMOE_ENCCL 4    /* NCCL error in the expert-parallel path                              */
#define NMOE_ETIMEOUT 5 /* a bounded device-side wait expired (never traps)                   */
#define NMOE_EDEVICE 6  /* the device error word was set (e.g. routed expert id >= experts)   */
#define NMOE_EIO 7      /* file open/read error                                               */
#define NMOE_ENOMEM 8   /* allocation failure                                                 */
#define NMOE_ECHECKSUM 9 /* an expert pack's CRC-32C differs from the expected one          */

/* ---- dtypes ------------------------------------------------------------------- */
#define NMOE_DTYPE_F32 0
#define NMOE_DTYPE_BF16 1
#define NMOE_DTYPE_Q2 2
#define NMOE_DTYPE_Q4 4

/* ---- fixed Qwen3.6-35B-A3B MoE geometry (src/runtime.m:31-44, convert_qwen36.py:31-36) */
#define NMOE_HIDDEN 2048
#define NMOE_INTER 512
#define NMOE_NUM_EXPERTS 256
#define NMOE_GROUP 64
#define NMOE_MAX_K 8 /* include/nmoe/expert_io.h:11 */

typedef struct nmoe_moe_ctx nmoe_moe_ctx;

typedef struct nmoe_moe_config {
    int quant_bits;    /* expert packs: 4 (packed_experts) or 2 (packed_experts_2bit)        */
    int num_layers;    /* 40 for the full model; any >= 1                                    */
    int num_experts;   /* 256                                                                */
    int k_max;         /* largest k a forward call may use, 1..8 (--experts, app_config.m)   */
    int router_dtype;  /* NMOE_DTYPE_BF16 or NMOE_DTYPE_Q4 (reference model_weights: q4)     */
    int shared_dtype;  /* NMOE_DTYPE_BF16 or NMOE_DTYPE_Q4 (shared expert + its gate vector)  */
    int t_max;         /* largest T of nmoe_moe_forward_batched (workspace is sized at create) */
    int world_size;    /* expert-parallel ranks (1 = single GPU)                             */
    int rank;          /* this process's rank, 0..world_size-1                               */
    const void *nccl_unique_id; /* 128-byte ncclUniqueId shared by all ranks (world_size>1)  */
    int flags;         /* NMOE_FLAG_* bits, 0 for the defaults                                */
} nmoe_moe_config;

/* Opt-in behaviour (nmoe_moe_config.flags). */
/* Layers are called in order 0, 1, ... (a decode step): each batch-1 call also pulls the
 * next layer's router and shared-expert weights into L2 during its tail, so the next call
 * starts from L2. Harmless but useless for other call orders. */
#define NMOE_FLAG_PREFETCH_NEXT_LAYER 1
/* Routed-expert dot products in fp32 (about 1e-6 relative) instead of the default half2
 * products with fp32 flushes (about 3e-4 relative, twice the throughput). */
#define NMOE_FLAG_EXPERT_FP32 2

/* A matrix given to nmoe_moe_set_dense: bf16 uses `weight` only ([rows][cols] u16);
 * q4 uses weight ([rows][cols/8] u32), scales and biases ([rows][cols/64] bf16), the
 * layout written by quantize_matrix_to_weights (scripts/convert_qwen36.py:214-263). */
typedef struct nmoe_tensor {
    const void *weight;
    const void *scales;
    const void *biases;
} nmoe_tensor;

/* The per-layer non-expert MoE weights, named as in model_weights.json
 * (src/runtime.m:2357-2371). */
typedef struct nmoe_moe_dense_weights {
    nmoe_tensor router;          /* model.layers.N.mlp.gate                    [256][2048] */
    nmoe_tensor shared_gate;     /* model.layers.N.mlp.shared_expert.gate_proj [512][2048] */
    nmoe_tensor shared_up;       /* model.layers.N.mlp.shared_expert.up_proj   [512][2048] */
    nmoe_tensor shared_down;     /* model.layers.N.mlp.shared_expert.down_proj [2048][512] */
    nmoe_tensor shared_gate_vec; /* model.layers.N.mlp.shared_expert_gate      [1][2048]   */
} nmoe_moe_dense_weights;

/* ---- host-only pack/layout helpers (no GPU needed) ------------------------------ */

/* Bytes of one expert blob: 1,769,472 (q4) / 983,040 (q2). Replaces
 * nmoe_expert_active_size (include/nmoe/expert_io.h:28). 0 for other bits. */
size_t nmoe_moe_expert_size(int quant_bits);

/* The nine component offsets of an expert blob, in EXPERT_LAYOUT order
 * (scripts/convert_qwen36.py:38-64; NMOEExpertOffsetsForBits, src/runtime.m:2240-2252). */
int nmoe_moe_expert_offsets(int quant_bits, size_t offsets[9]);

/* Validate a converter-written layout.json (scripts/convert_qwen36.py:351-359: keys
 * expert_size, num_layers, num_experts, components[{name,offset,size}]) against the
 * built-in layout for `quant_bits`. Accepts, unlike the reference's never-called
 * validator (src/expert_io.m:274-316), the keys the converter actually writes; optional
 * dtype/shape keys are checked when present. Message (if any) goes to err[errlen]. */
int nmoe_moe_validate_layout_json(const char *path, int quant_bits, char *err, size_t errlen);

const char *nmoe_moe_strerror(int status);

/* ---- context ------------------------------------------------------------------ */

/* Create a context on CUDA device `device` (replaces nmoe_backend_create +
 * NMOEInitExpertIOBuffers, src/runtime.m:2664, 1542). Device memory for all layers'
 * expert packs and dense weights plus every workspace is reserved here; forward calls
 * allocate nothing. With world_size > 1 the context owns an NCCL communicator and holds
 * only its 1/world_size share of each layer's experts. */
nmoe_moe_ctx *nmoe_moe_create(const nmoe_moe_config *cfg, int device, int *status);
void nmoe_moe_destroy(nmoe_moe_ctx *ctx);
/* Message of the last failed nmoe_moe_create on this host thread (no context exists). */
const char *nmoe_moe_create_error(void);
const char *nmoe_moe_last_error(const nmoe_moe_ctx *ctx);

/* Upload one layer's expert packs from a host image of layer_XX.bin: exactly
 * num_experts * expert_size bytes (the size check of NMOELoadExpertLayer,
 * src/runtime.m:2445, made exact). Replaces the per-token pread loader. */
int nmoe_moe_load_layer(nmoe_moe_ctx *ctx, int layer, const void *layer_bin, size_t bytes);
/* Same, reading the file at `path` (e.g. packed_experts/layer_07.bin). */
int nmoe_moe_load_layer_file(nmoe_moe_ctx *ctx, int layer, const char *path);
/* No counterpart in the reference (its loader checks sizes only, src/expert_io.m:52-65).
 * The loads above with an integrity check: the CRC-32C (Castagnoli, reflected 0x82F63B78,
 * init and final xor 0xFFFFFFFF) of every expert blob this context holds is computed on
 * the device while the image is staged, before it is repacked. expected_crc[num_experts]
 * (global expert ids, may be NULL): on the first mismatch nothing is loaded and the call
 * returns NMOE_ECHECKSUM, naming the expert in nmoe_moe_last_error(). crc_out[num_experts]
 * (may be NULL) receives the CRCs (entries of experts an expert-parallel rank does not
 * hold are left untouched). nmoe_crc32c() gives the same values on the host. */
int nmoe_moe_load_layer_checked(nmoe_moe_ctx *ctx, int layer, const void *layer_bin, size_t bytes,
                                const uint32_t *expected_crc, uint32_t *crc_out);
int nmoe_moe_load_layer_file_checked(nmoe_moe_ctx *ctx, int layer, const char *path,
                                     const uint32_t *expected_crc, uint32_t *crc_out);
/* Host CRC-32C, continuing from `crc` (0 to start): nmoe_crc32c(0, blob, n) is the value
 * the checked loads compute for a blob. SSE4.2 instruction where the CPU has it. */
uint32_t nmoe_crc32c(uint32_t crc, const void *data, size_t n);
/* Device CRC-32C of nblobs consecutive blobs of blob_bytes each (a multiple of 8192;
 * expert blobs are) in caller-owned DEVICE memory (8-byte aligned) into d_crc_out[nblobs]
 * (device). Asynchronous on `stream`, allocates nothing: e.g. to verify the device copy of
 * a layer image that nmoe_moe_forward_static reads. One CTA per blob. */
int nmoe_crc32c_device(const void *d_data, size_t blob_bytes, int nblobs, uint32_t *d_crc_out, void *stream);
/* CRC-32C of A followed by B from crc(A), crc(B) and the length of B in bytes. */
uint32_t nmoe_crc32c_combine(uint32_t crc_a, uint32_t crc_b, size_t len_b);
/* Upload one layer's router + shared-expert weights (dtypes from the config). */
int nmoe_moe_set_dense(nmoe_moe_ctx *ctx, int layer, const nmoe_moe_dense_weights *w);

/* ---- forward ------------------------------------------------------------------ */

/* One token through layer `layer`'s routed-MoE block, asynchronous on `stream`:
 *   out[r] = h_mid[r] + sum_{s<k} w_s * down_{e_s}(SiLU(gate_{e_s} x) * up_{e_s} x)
 *            + sigmoid(gvec . x) * shared_down(SiLU(shared_gate x) * shared_up x)
 * with (e_s, w_s) the top-k of softmax(router x) renormalised over the k picks
 * (NMOESelectRouteTopKCPU semantics: descending, lower expert id wins a tie).
 *   x      device [2048], x_dtype NMOE_DTYPE_BF16 or NMOE_DTYPE_F32
 *   h_mid  device fp32 [2048] residual, or NULL for the bare block output
 *   out    device fp32 [2048]
 *   idx_out/w_out  device [8] (uint32 / fp32), optional; slots >= k are (0, 0.0)
 *                  as in nmoe_route_topk (metal/kernels.metal:1767-1775)
 * k must be in [1, k_max] (the reference clamps --experts to 1..8, app_config.m:215-226;
 * the library rejects instead of clamping). Replaces src/runtime.m:3151-3201. */
int nmoe_moe_forward(nmoe_moe_ctx *ctx, int layer, int k, const void *x, int x_dtype,
                     const float *h_mid, float *out, uint32_t *idx_out, float *w_out, void *stream);

/* Routing only: router logits (device fp32 [256], optional), top-k ids and renormalised
 * weights (device [8], optional). Same rule as nmoe_moe_forward. The GPU counterpart of
 * NMOEEncodeRouteTopK + nmoe_route_topk (src/runtime.m:1403-1424, kernels.metal:1715-1776). */
int nmoe_moe_route(nmoe_moe_ctx *ctx, int layer, int k, const void *x, int x_dtype,
                   float *logits_out, uint32_t *idx_out, float *w_out, void *stream);

/* T tokens (prefill / batched decode) through one layer: x device [T][2048] (bf16 or
 * f32), h_mid device fp32 [T][2048] or NULL, out device [T][2048] in out_dtype
 * (F32 or BF16), idx_out/w_out device [T][8] optional. T <= t_max. With world_size > 1
 * every rank passes its own T tokens (0 allowed) and every rank must make the same calls
 * in the same order; experts are sharded num_experts/world_size per rank and token rows
 * travel by NVLink peer stores between the ranks' mapped buffers, on the stream, with no
 * host synchronisation (t_max and k_max must be equal on all ranks). No reference
 * counterpart (the reference runs prefill token by token, src/runtime.m:3816). */
int nmoe_moe_forward_batched(nmoe_moe_ctx *ctx, int layer, int T, int k, const void *x, int x_dtype,
                             const float *h_mid, void *out, int out_dtype, uint32_t *idx_out,
                             float *w_out, void *stream);

/* Diagnostics: device time (ms) of the last expert-parallel call's two exchanges:
 * ms[0] = dispatch of the token rows + wait for every source's rows, ms[1] = return of the
 * down outputs + wait for every owner's returns. Needs world_size > 1 and NMOE_EP_TIMING=1
 * in the environment at create. Synchronises on the last call. No reference counterpart. */
int nmoe_moe_debug_ep_times(nmoe_moe_ctx *ctx, float *ms);

/* Expert parallelism: fill `out` (>= 128 bytes) with a fresh NCCL unique id. One rank
 * calls it and hands the bytes to every rank's nmoe_moe_config.nccl_unique_id. No
 * reference counterpart (the reference runs on one device). */
int nmoe_moe_nccl_unique_id(void *out, size_t bytes);

/* Read and clear the device error word (synchronises the context's device). Returns
 * NMOE_OK or NMOE_EDEVICE and the first recorded code in *code (may be NULL). */
int nmoe_moe_device_status(nmoe_moe_ctx *ctx, int *code);

/* Diagnostics: copy and clear the single-launch decode kernel's per-CTA progress trail
 * (n <= 1024 entries; entry c = 100 + phase where a bounded wait of CTA c gave up; with
 * NMOE_TIMELINE=1 at context creation also the highest phase 1..7 reached since the last
 * read). Synchronises the device. No reference counterpart. */
int nmoe_moe_debug_trail(nmoe_moe_ctx *ctx, uint32_t *out, int n);
/* Diagnostics: per-CTA phase timestamps (globaltimer ns, low 32 bits, [n_ctas][32]) of
 * the last decode call, recorded when the context was created with NMOE_TIMELINE=1 in
 * the environment (slots a CTA did not reach in that call read 0). Synchronises the
 * device. No reference counterpart. */
int nmoe_moe_debug_timeline(nmoe_moe_ctx *ctx, uint32_t *out, int n_ctas);
/* Diagnostics: CTAs of the batch-1 decode kernel's grid (one per SM, at most 256), i.e.
 * the rows nmoe_moe_debug_timeline fills. No reference counterpart. */
int nmoe_moe_decode_grid(const nmoe_moe_ctx *ctx);

/* Diagnostics: copy the router logits [T][256] (fp32) of the last
 * nmoe_moe_forward_batched call to host memory (T <= that call's T). Synchronises the
 * device. */
int nmoe_moe_debug_logits(nmoe_moe_ctx *ctx, float *out, int T);
/* Diagnostics: per-role %clock timestamps of CTA 0 of one grouped-GEMM launch of
 * nmoe_moe_forward_batched ([13][1024] u32: producer slots, B stages, dequant start/end,
 * MMA issue, epilogue start/end, raw slot landed, MMA step issued, last dequant warp step end, dequant wait begin, A stage free, scales ready), recorded when the context was created with
 * NMOE_GEMM_TRACE=<0 router | 1 gate/up | 2 down> in the environment. */
int nmoe_moe_debug_gemm_trace(nmoe_moe_ctx *ctx, uint32_t *out, int n);

/* ---- forward without any allocation ------------------------------------------ */

/* No counterpart in the reference. The batch-1 block of nmoe_moe_forward for callers
 * that cannot allocate device memory when they call: hosts whose device memory belongs
 * to a preallocated pool they may not go around, code where cudaMalloc's implicit
 * synchronisation is not allowed, embedders that never create an nmoe_moe_ctx.
 * All weights are DEVICE pointers the caller owns, laid out as nmoe_moe_load_layer /
 * nmoe_moe_set_dense take them on the host: `experts` is a layer_XX.bin image of
 * num_experts expert blobs, `dense` holds the router/shared tensors. The call allocates
 * nothing: its scratch (19,712 bytes, nmoe_moe_static_scratch_bytes()) is one array
 * compiled into the library, held by every GPU that loads it until the process exits,
 * and shared by all calls on a device. It runs four fp32 kernels (router + shared
 * expert, top-k, routed gate/up, down + combine).
 * Limits: k in [1, 8] (the scratch holds 8 routed slots); larger k is rejected with
 * NMOE_EINVAL. The first call on a device (the current one) looks up that array's device
 * address; make that first call before any stream capture. Calls that overlap on the
 * GPU (different streams, or different host threads) race on the shared scratch: order
 * them. Routed ids >= num_experts contribute nothing and set the scratch's error word,
 * which nmoe_moe_static_status reads. Message of a failed call: nmoe_moe_static_error(). */
int nmoe_moe_forward_static(const void *experts, int num_experts, int quant_bits,
                            const nmoe_moe_dense_weights *dense, int router_dtype, int shared_dtype,
                            int k, const void *x, int x_dtype, const float *h_mid, float *out,
                            uint32_t *idx_out, float *w_out, void *stream);
const char *nmoe_moe_static_error(void);
/* No counterpart in the reference. Bytes of the static scratch array. */
size_t nmoe_moe_static_scratch_bytes(void);
/* No counterpart in the reference. Read and clear the error word that the last
 * nmoe_moe_forward_static call on the current device left in the static scratch (each
 * call clears it when it starts), waiting for `stream` first. Allocates nothing. Returns
 * NMOE_OK, NMOE_EDEVICE (routed expert id >= num_experts) or NMOE_ETIMEOUT, with the code
 * in *code (may be NULL). Races, like the calls, with static calls that overlap it. */
int nmoe_moe_static_status(int *code, void *stream);

/* ---- LM head: final RMSNorm + vocab GEMV + top-1 in one launch ------------------
 * Replaces NMOERunLmHeadArgmaxQ4Metal (src/runtime.m:1882-1948: kernels
 * nmoe_lm_head_argmax_q4 + nmoe_lm_head_argmax_reduce, metal/kernels.metal:1599-1713)
 * and the model.norm RMSNorm before it (src/runtime.m:3786, nmoe_rms_norm
 * metal/kernels.metal:862-900); with logits_out it also covers the fallback
 * (dequant matvec + nmoe_argmax_top1, src/runtime.m:3793-3794).
 *   head: DEVICE tensors. q4: weight u32 [vocab][256], scales/biases bf16 [vocab][32]
 *         (lm_head.weight/.scales/.biases, group 64); bf16: weight [vocab][2048].
 *         16-byte aligned.
 *   in_dim: must be 2048. x: DEVICE [2048] f32 or bf16 (x_dtype).
 *   norm_weight: DEVICE bf16 [2048] (model.norm.weight) or NULL to use x as given;
 *         x_n = x * rsqrt(mean(x^2) + norm_eps) * (w + (norm_add_one ? 1 : 0)).
 *   logits_out: DEVICE f32 [vocab] or NULL. token_out: DEVICE u32 [1].
 *   workspace: DEVICE, nmoe_lm_head_workspace_bytes() bytes, 8-byte aligned, zeroed
 *         by the caller ONCE; every call leaves it zeroed again. Calls that share a
 *         workspace must not overlap on the GPU.
 * Token rule (both reference kernels): lowest row index among the rows with the maximum
 * logit; NaN, -inf and -FLT_MAX never win; 0 if no row qualifies. A bounded device wait
 * that expired writes UINT32_MAX as the token (the reference's "no token" value,
 * src/runtime.m:3804). Asynchronous on `stream`; allocates nothing; capturable.
 * Message of a failed call: nmoe_lm_head_error(). */
int nmoe_lm_head_argmax(const nmoe_tensor *head, int head_dtype, int vocab, int in_dim, const void *x,
                        int x_dtype, const uint16_t *norm_weight, float norm_eps, int norm_add_one,
                        float *logits_out, uint32_t *token_out, void *workspace, void *stream);
size_t nmoe_lm_head_workspace_bytes(void);
const char *nmoe_lm_head_error(void);

/* ---- Linear attention (GatedDeltaNet) core of one decode step ---------------------
 * Replaces the five kernels of NMOELinearAttentionStepMetal between the fused
 * qkv/z/beta/alpha projection and the output projection (src/runtime.m:3390-3478):
 * conv1d step, per-head q/k RMS norm, decay/beta, the gated delta rule on the recurrent
 * state, and the z-gated RMS norm (metal/kernels.metal:1275-1346, 1780-1873). Qwen3.6
 * geometry: 16 key heads and 32 value heads of 128, conv width 4 over 8192 channels.
 * All pointers are DEVICE memory: qkv f32[8192] (q 0..2047, k 2048..4095, v 4096..8191),
 * z f32[4096], alpha f32[32], beta f32[32]; conv_state f32[3][8192] and delta_state
 * f32[32][128][128] (16-byte aligned) are updated in place; out f32[4096] feeds the output
 * projection. One launch of 16 clusters x 8 CTAs; allocates nothing; capturable. */
typedef struct nmoe_linear_attn_weights {
    const uint16_t *conv_w;   /* bf16 [8192][4]  linear_attn.conv1d.weight (8-byte aligned) */
    const float *A_log;       /* f32 [32]        linear_attn.A_log                          */
    const uint16_t *dt_bias;  /* bf16 [32]       linear_attn.dt_bias                        */
    const uint16_t *norm_w;   /* bf16 [128]      linear_attn.norm.weight                    */
} nmoe_linear_attn_weights;
int nmoe_linear_attn_step(const nmoe_linear_attn_weights *w, const float *qkv, const float *z,
                          const float *alpha, const float *beta, float *conv_state, float *delta_state,
                          float *out, void *stream);
/* The same step for a batch of sequences, one launch of batch x 128
 * CTAs: every pointer covers `batch` consecutive copies of the single-sequence layout
 * (qkv [batch][8192], z [batch][4096], alpha / beta [batch][32], conv_state
 * [batch][3][8192], delta_state [batch][32][128][128], out [batch][4096]). */
int nmoe_linear_attn_step_batched(const nmoe_linear_attn_weights *w, int batch, const float *qkv,
                                  const float *z, const float *alpha, const float *beta,
                                  float *conv_state, float *delta_state, float *out, void *stream);

/* ---- Full-attention decode step --------------------------------------------------
 * Replaces, in NMOEFullAttentionStepMetal (src/runtime.m:3040-3095), nmoe_full_qk_prep
 * (per-head RMS norm with weight + 1, rotate-half RoPE on dims 0..63 with theta 1e7,
 * sigmoid of the query gate; metal/kernels.metal:1006-1058), the copies of k and v into
 * the caches, and nmoe_attn_decode_fused (kernels.metal:1119-1194). Qwen3.6 geometry: 16
 * query heads, 2 KV heads, head dim 256. DEVICE pointers: q f32 [16][512] (query | gate
 * per head; not modified), k_new / v_new f32 [2][256] (the k / v projections of this
 * token), k_cache / v_cache f32 [max_positions][2][256] (row `position` is written),
 * out f32 [16][256] (attention times the gate, the input of o_proj). workspace: DEVICE,
 * nmoe_full_attn_workspace_bytes(), 16-byte aligned (the slices' partial results; calls
 * sharing a workspace must not overlap). Two launches: split-K over positions (up to 148
 * CTAs), then the merge of the slices; allocates nothing; capturable. */
typedef struct nmoe_full_attn_weights {
    const uint16_t *q_norm;   /* bf16 [256] self_attn.q_norm.weight */
    const uint16_t *k_norm;   /* bf16 [256] self_attn.k_norm.weight */
} nmoe_full_attn_weights;
int nmoe_full_attn_step(const nmoe_full_attn_weights *w, const float *q, const float *k_new,
                        const float *v_new, float *k_cache, float *v_cache, int position,
                        int max_positions, float *out, void *workspace, void *stream);
size_t nmoe_full_attn_workspace_bytes(void);

/* The same step for a batch of sequences over a bf16 KV cache (batch 64
 * at 32k context; the reference's cache is f32 and batch 1). DEVICE pointers: q f32
 * [batch][16][512], k_new / v_new f32 [batch][2][256], k_cache / v_cache bf16
 * [batch][max_positions][2][256] (sequence b's row d_positions[b] is written, rounded to
 * nearest even), d_positions int32 [batch] read on the device (a position outside
 * [0, max_positions) leaves that sequence's caches untouched and its out zero), out f32
 * [batch][16][256]. workspace: nmoe_full_attn_batched_workspace_bytes(batch), 16-byte
 * aligned. Two launches of batch x 148 and batch x 16 CTAs; allocates nothing;
 * capturable (positions on the device: one graph serves every step). */
int nmoe_full_attn_step_batched(const nmoe_full_attn_weights *w, int batch, const float *q,
                                const float *k_new, const float *v_new, uint16_t *k_cache,
                                uint16_t *v_cache, const int32_t *d_positions, int max_positions,
                                float *out, void *workspace, void *stream);
size_t nmoe_full_attn_batched_workspace_bytes(int batch);

/* ---- Whole decode step ------------------------------------------
 * The C restatement of NMOEProcessToken (src/runtime.m:3712-3805) on the GPU: embedding
 * row, 40 layers (layer l is full attention when (l + 1) % 4 == 0, else linear attention:
 * src/runtime.m:2373), each: input RMSNorm (weight + 1, eps 1e-6), attention (projections
 * as q4 matrix-vector products in the reference's dequant order, then
 * nmoe_linear_attn_step or nmoe_full_attn_step), output projection + residual, post
 * RMSNorm, and the routed-MoE block of the given context (nmoe_moe_forward with the
 * residual as h_mid); then the final RMSNorm and the LM head's top-1 (nmoe_lm_head_argmax).
 * Weights given to the set calls are HOST pointers, copied to the device. q4 matrices:
 * weight u32 [rows][cols/8], scales/biases bf16 [rows][cols/64] (nmoe_tensor). */
typedef struct nmoe_decoder nmoe_decoder;
typedef struct nmoe_linear_layer_host {
    const uint16_t *input_norm, *post_norm;   /* bf16 [2048] */
    nmoe_tensor qkv, z, beta, alpha;          /* q4 [8192|4096|32|32][2048]  in_proj_qkv / z / b / a */
    nmoe_tensor out;                          /* q4 [2048][4096]             out_proj               */
    const uint16_t *conv_w;                   /* bf16 [8192][4]  */
    const float *A_log;                       /* f32 [32]        */
    const uint16_t *dt_bias;                  /* bf16 [32]       */
    const uint16_t *norm_w;                   /* bf16 [128]      */
} nmoe_linear_layer_host;
typedef struct nmoe_full_layer_host {
    const uint16_t *input_norm, *post_norm;   /* bf16 [2048] */
    nmoe_tensor q, k, v;                      /* q4 [8192|512|512][2048] (q: per head 256 query + 256 gate) */
    nmoe_tensor o;                            /* q4 [2048][4096] */
    const uint16_t *q_norm, *k_norm;          /* bf16 [256] */
} nmoe_full_layer_host;
/* moe: a context with num_layers >= the decoder's, every layer loaded; k routed experts. */
nmoe_decoder *nmoe_decoder_create(nmoe_moe_ctx *moe, int num_layers, int k, int max_positions, int *status);
void nmoe_decoder_destroy(nmoe_decoder *dec);
const char *nmoe_decoder_error(const nmoe_decoder *dec);
int nmoe_decoder_set_linear_layer(nmoe_decoder *dec, int layer, const nmoe_linear_layer_host *w);
int nmoe_decoder_set_full_layer(nmoe_decoder *dec, int layer, const nmoe_full_layer_host *w);
/* embed / lm_head: NMOE_DTYPE_Q4 or NMOE_DTYPE_BF16, [vocab][2048]; final_norm bf16 [2048]. */
int nmoe_decoder_set_globals(nmoe_decoder *dec, int vocab, int embed_dtype, const nmoe_tensor *embed,
                             const uint16_t *final_norm, int head_dtype, const nmoe_tensor *lm_head);
/* Zero the recurrent and conv states (a new sequence). */
int nmoe_decoder_reset(nmoe_decoder *dec, void *stream);
/* One token: d_token (DEVICE u32) at `position` (< max_positions) -> d_next (DEVICE u32).
 * d_hidden (DEVICE f32 [2048], may be NULL) receives the last layer's output. */
int nmoe_decoder_step(nmoe_decoder *dec, const uint32_t *d_token, int position, uint32_t *d_next,
                      float *d_hidden, void *stream);

#ifdef __cplusplus
}
#endif
#endif
