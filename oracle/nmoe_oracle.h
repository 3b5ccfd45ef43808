/*
 * nmoe_oracle.h -- CPU restatement of nmoe's routed-MoE block (TEST INFRASTRUCTURE).
 *
 * This library is the checker for the CUDA path, never part of the product:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load it.  Every function cites the reference file:line it restates
 * (paths are relative to the nano-metal-moe-qwen36 project root).
 *
 * Parity pins: the quantiser is checked bit-exactly against fixtures produced by
 * importing the reference's scripts/convert_qwen36.py (tests/golden/make_golden.py);
 * the routing math (softmax / top-k / renormalise / SwiGLU / dequant matvec) is
 * checked bit-exactly against the reference's own src/math.m compiled as C into
 * oracle/_ref/ (oracle/Makefile, target `ref`).  The Metal kernels themselves
 * cannot run here (no Apple GPU); their fp32 math is restated below.
 */
#ifndef NMOE_ORACLE_H
#define NMOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_HIDDEN 2048
#define ORC_INTER 512
#define ORC_EXPERTS 256
#define ORC_GROUP 64
#define ORC_MAX_K 8

enum { ORC_DTYPE_BF16 = 1, ORC_DTYPE_Q4 = 4, ORC_DTYPE_Q2 = 2, ORC_DTYPE_F32 = 0 };

/* bf16 <-> f32 (src/math.m:7-19, scripts/convert_qwen36.py:147-155) */
float orc_bf16_to_f32(uint16_t v);
uint16_t orc_f32_to_bf16(float v);
void orc_f32_to_bf16_array(const float *in, uint16_t *out, size_t n);
void orc_bf16_to_f32_array(const uint16_t *in, float *out, size_t n);

/* Affine group-64 quantiser (scripts/convert_qwen36.py:158-211).
 * packed: rows x (in_dim*bits/32) u32, scales/biases: rows x (in_dim/64) bf16. */
int orc_quantize_rows(const uint16_t *rows_bf16, size_t rows, size_t in_dim, int bits,
                      uint32_t *packed, uint16_t *scales, uint16_t *biases);

/* Expert blob layout (scripts/convert_qwen36.py:38-64; src/runtime.m:2240-2252). */
size_t orc_expert_size(int bits);
int orc_expert_offsets(int bits, size_t off[9]);
/* gate_up_bf16: [1024][2048] (rows 0-511 gate, 512-1023 up), down_bf16: [2048][512]
 * (scripts/convert_qwen36.py:377-409). */
int orc_pack_expert(const uint16_t *gate_up_bf16, const uint16_t *down_bf16, int bits, uint8_t *blob);

/* src/math.m restatements */
float orc_sigmoid_cpu(float x);                                            /* math.m:21-28 */
float orc_sigmoid_kernel(float x);                                         /* kernels.metal:177-179 */
void orc_softmax(float *values, size_t count);                             /* math.m:67-93 */
size_t orc_topk(const float *values, size_t count, size_t k, uint32_t *indices,
                float *selected);                                          /* math.m:95-132 */
void orc_renormalize(float *values, size_t count);                         /* math.m:134-153 */
void orc_swiglu(const float *gate, const float *up, float *out, size_t n); /* kernels.metal:1352-1361 */
/* math.m:236-274: sequential fp32 accumulation, (q*scale + bias) * x. */
void orc_dequant_matvec_seq(const uint32_t *packed, const uint16_t *scales, const uint16_t *biases,
                            const float *x, float *y, size_t rows, size_t in_dim, int bits);

/* Kernel-form matvecs: 32 lane-strided fp32 partial sums (one per SIMD lane, as the
 * Metal kernels stride packed words by lane) reduced by a butterfly tree.
 * form 0: acc += fma(q, s, b) * x      (kernels.metal:192-238, 562-640, 642-714, 1456-1542)
 * form 1: acc += fma(q, s*x, b*x)      (kernels.metal:240-301, 384-514)                */
void orc_dequant_matvec(const uint32_t *packed, const uint16_t *scales, const uint16_t *biases,
                        const float *x, float *y, size_t rows, size_t in_dim, int bits, int form);
/* bf16 weights (no reference kernel): same lane-strided fp32 structure. */
void orc_bf16_matvec(const uint16_t *w, const float *x, float *y, size_t rows, size_t in_dim);

/* A dense (non-expert) matrix: bf16 [rows][cols] or q4 (weight u32, scales, biases). */
typedef struct orc_dense {
    int dtype;                 /* ORC_DTYPE_BF16 or ORC_DTYPE_Q4 */
    const void *weight;
    const uint16_t *scales;    /* q4 only */
    const uint16_t *biases;    /* q4 only */
} orc_dense;

typedef struct orc_layer {
    int bits;                  /* expert quantisation: 4 or 2 */
    const uint8_t *experts;    /* layer_XX.bin image: num_experts * expert_size bytes */
    size_t num_experts;
    orc_dense router;          /* [256][2048]  (model.layers.N.mlp.gate) */
    orc_dense shared_gate;     /* [512][2048]  (mlp.shared_expert.gate_proj) */
    orc_dense shared_up;       /* [512][2048]  (mlp.shared_expert.up_proj) */
    orc_dense shared_down;     /* [2048][512]  (mlp.shared_expert.down_proj) */
    orc_dense shared_gate_vec; /* [1][2048]    (mlp.shared_expert_gate) */
} orc_layer;

/* Per-expert products (kernels.metal:562-640 q4 / 192-238+1352-1361 q2, 642-714). */
void orc_expert_gate_up(const uint8_t *blob, int bits, const float *x, float *act);
void orc_expert_down(const uint8_t *blob, int bits, const float *act, float *out);

/* Router + shared gate/up + shared score (kernels.metal:384-514 for q4; bf16 analog). */
void orc_route_shared(const orc_layer *L, const float *x, float *logits, float *shared_act, float *score);

/* One routed-MoE block for one token, following the default q4 path
 * (src/runtime.m:3151-3166 -> 1498-1511 -> 2778-2903, 2976-2983) and the q2 path
 * (src/runtime.m:2841-2888).
 *   k: active experts 1..8 (src/runtime.m:2923 clamp; here out-of-range -> -1)
 *   x: fp32[2048]; h_mid: fp32[2048] or NULL (treated as zero)
 *   logits_override: if non-NULL, route on these 256 logits instead of the computed ones
 * Outputs (each may be NULL): out[2048], idx[8], w[8] (zero padded), logits[256],
 * shared_act[512], score[1]. Returns 0 on success. */
int orc_moe_block_forward(const orc_layer *L, int k, const float *x, const float *h_mid,
                          const float *logits_override, float *out, uint32_t *idx, float *w,
                          float *logits, float *shared_act, float *score);

/* Batched block: T tokens, each routed independently (same math as above per token). */
int orc_moe_block_forward_batched(const orc_layer *L, int T, int k, const float *x,
                                  const float *h_mid, float *out, uint32_t *idx, float *w);


/* RMSNorm as the reference's nmoe_rms_norm kernel computes it (metal/kernels.metal:862-900):
 * out = x * rsqrt(mean(x^2) + eps) * (w (+1 if add_one)); w NULL = unit weight. The sum of
 * squares is taken in double here. Cross-checked against the CPU form nmoe_cpu_rms_norm
 * (src/math.m:34-64, x / sqrt(mean + eps) * w). */
void orc_rms_norm(const float *x, const uint16_t *w_bf16, float *out, size_t n, float eps, int add_one);

/* Top-1 rule of nmoe_argmax_top1 / nmoe_lm_head_argmax_reduce (metal/kernels.metal:1562-1597,
 * 1668-1713): lowest index of the maximum among values > -FLT_MAX (NaN never wins); 0 if none. */
uint32_t orc_argmax_top1(const float *v, size_t n);

/* LM head of NMOERunLmHeadArgmaxQ4Metal (src/runtime.m:1882-1948; kernels.metal:1599-1713):
 * optional RMSNorm of x (norm_w non-NULL), logits[r] = kernel-form dequant matvec (form 0,
 * lane-strided, as nmoe_lm_head_argmax_q4 accumulates), token = orc_argmax_top1(logits).
 * dtype ORC_DTYPE_Q4 (w u32 [vocab][in/8], s/b bf16 [vocab][in/64]) or ORC_DTYPE_BF16
 * (w bf16 [vocab][in]). logits may be NULL only if the caller does not need them. */
uint32_t orc_lm_head_argmax(int dtype, const void *w, const uint16_t *s, const uint16_t *b, size_t vocab,
                            size_t in_dim, const float *x, const uint16_t *norm_w, float eps, int add_one,
                            float *logits);

/* CRC-32C (Castagnoli, reflected 0x82F63B78, init/final xor 0xFFFFFFFF), bit at a time:
 * the definition, for checking the library's table / SSE4.2 / device versions. Continues
 * from `crc` (0 to start). */
uint32_t orc_crc32c(uint32_t crc, const uint8_t *data, size_t n);

/* Linear-attention (GatedDeltaNet) core of one decode step, Qwen3.6 geometry: 16 key heads
 * x 128, 32 value heads x 128, conv width 4 over 8192 channels (q 0..2047, k 2048..4095,
 * v 4096..8191). The reference's sequence (src/runtime.m:3390-3478):
 *   nmoe_conv1d_step      (metal/kernels.metal:1275-1295): out = SiLU(sum of 4 taps),
 *                          conv_state shifted, the input appended;
 *   nmoe_rms_norm_qk      (kernels.metal:1780-1821): per key head, q * rsqrt(mean q^2 + 1e-12)
 *                          / key_dim, k * rsqrt(mean k^2 + 1e-12) / sqrt(key_dim);
 *   nmoe_compute_decay_beta (kernels.metal:1823-1839): g = exp(-exp(A_log) softplus(alpha +
 *                          dt_bias)), b = sigmoid(beta);
 *   nmoe_gated_delta_net_step (kernels.metal:1300-1346): S = g S; d = (v - S k) b; S += k d;
 *                          o = S q (value head vh reads key head vh / 2);
 *   nmoe_gated_rms_norm    (kernels.metal:1841-1873): o * rsqrt(mean o^2 + 1e-6) * SiLU(z) * w.
 * qkv[8192], z[4096], alpha[32], beta[32]; conv_w bf16 [8192][4], A_log f32[32], dt_bias
 * bf16[32], norm_w bf16[128]; conv_state f32 [3][8192] and delta_state f32 [32][128][128]
 * are updated in place; out[4096]. Sums run in the reference kernels' sequential order. */
void orc_linear_attn_step(const float *qkv, const float *z, const float *alpha, const float *beta,
                          const uint16_t *conv_w, const float *A_log, const uint16_t *dt_bias,
                          const uint16_t *norm_w, float *conv_state, float *delta_state, float *out);

/* Full-attention decode step (Qwen3.6: 16 query heads, 2 KV heads, head dim 256, partial
 * rotary 64, RoPE theta 1e7), the reference's sequence (src/runtime.m:3040-3095):
 *   nmoe_full_qk_prep (metal/kernels.metal:1006-1058): per head RMS norm (eps 1e-6, weight
 *     + 1), rotate-half RoPE on dims 0..63 at `position`, sigmoid of the q gate half;
 *   k, v of the position copied into the caches ([pos][2][256] f32);
 *   nmoe_attn_decode_fused (kernels.metal:1119-1194): softmax(q k / 16) v over positions
 *     0..position, times the gate.
 * q f32 [16][512] (query | gate per head), k_new/v_new f32 [2][256]; q_norm/k_norm bf16
 * [256]; caches updated at `position`; out f32 [16][256]. q is not modified. */
void orc_full_attn_step(const float *q, const float *k_new, const float *v_new, const uint16_t *q_norm,
                        const uint16_t *k_norm, float *k_cache, float *v_cache, int position, float *out);
/* The same step over a bf16 KV cache (the reference's cache is f32):
 * the caches are f32 arrays holding bf16 values, and the appended k (after norm and RoPE)
 * and v rows are rounded to bf16 (nearest even) before the attention reads them. */
void orc_full_attn_step_bf16kv(const float *q, const float *k_new, const float *v_new, const uint16_t *q_norm,
                               const uint16_t *k_norm, float *k_cache, float *v_cache, int position, float *out);

/* Set the OpenMP thread count used by the matvecs (0 = library default). */
void orc_set_threads(int n);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
