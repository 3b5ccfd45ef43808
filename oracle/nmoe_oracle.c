/*
 * nmoe_oracle.c -- CPU restatement of nmoe's routed-MoE block.
 *
 * TEST INFRASTRUCTURE ONLY: this is the checker the CUDA path is compared with
 * (tests/, __graft_entry__.smoke(), bench.py cpu_baseline / reference arm).  The
 * product library never links or calls it.
 *
 * Reference citations are file:line within the nano-metal-moe-qwen36 project.
 * Parity of this restatement is pinned by tests/test_oracle.py: bit-exact against
 * fixtures generated from the reference's own quantiser (tests/golden/) and against
 * the reference's src/math.m compiled unchanged as C (oracle/_ref/).
 *
 * Build: oracle/Makefile (gcc -O3 -march=native -fopenmp -ffp-contract=off).
 * -ffp-contract=off keeps every multiply and add separately rounded exactly where
 * the restated source writes them separately; fused operations are written as fmaf().
 */
#include "nmoe_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void orc_set_threads(int n) {
    g_threads = n;
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------------------- bf16 ---- */

/* src/math.m:7-12 */
float orc_bf16_to_f32(uint16_t v) {
    uint32_t bits = ((uint32_t)v) << 16;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* src/math.m:14-19 and scripts/convert_qwen36.py:151-155: round-to-nearest-even on the
 * upper 16 bits (u + 0x7FFF + lsb). */
uint16_t orc_f32_to_bf16(float v) {
    uint32_t u;
    memcpy(&u, &v, sizeof u);
    uint32_t r = u + 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(r >> 16);
}

void orc_f32_to_bf16_array(const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = orc_f32_to_bf16(in[i]);
}

void orc_bf16_to_f32_array(const uint16_t *in, float *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = orc_bf16_to_f32(in[i]);
}

/* ----------------------------------------------------------- quantiser ---- */

/* scripts/convert_qwen36.py:167-183 (2-bit) and 195-211 (4-bit):
 *   mn, mx = min/max over each group of 64 (fp32)
 *   scale = (mx - mn) / levels            (fp32; levels = 15 or 3)
 *   safe  = scale == 0 ? 1 : scale
 *   q     = clip(rint((x - mn) / safe), 0, levels)   rint = round half to even
 *   stored scale = bf16(scale), stored bias = bf16(mn)
 * Packing (py:158-164, 186-192): value at column vpw*j + i goes to word j, bits bits*i. */
int orc_quantize_rows(const uint16_t *rows_bf16, size_t rows, size_t in_dim, int bits,
                      uint32_t *packed, uint16_t *scales, uint16_t *biases) {
    if (bits != 2 && bits != 4) return -1;
    if (in_dim % ORC_GROUP != 0) return -1;
    const size_t vpw = 32u / (size_t)bits;
    const size_t words = in_dim / vpw;
    const size_t groups = in_dim / ORC_GROUP;
    const float levels = bits == 4 ? 15.0f : 3.0f;
    const uint32_t qmax = bits == 4 ? 15u : 3u;
    for (size_t r = 0; r < rows; r++) {
        const uint16_t *row = rows_bf16 + r * in_dim;
        uint32_t *prow = packed + r * words;
        memset(prow, 0, words * sizeof(uint32_t));
        for (size_t g = 0; g < groups; g++) {
            float mn = orc_bf16_to_f32(row[g * ORC_GROUP]);
            float mx = mn;
            for (size_t c = 1; c < ORC_GROUP; c++) {
                float v = orc_bf16_to_f32(row[g * ORC_GROUP + c]);
                if (v < mn) mn = v;
                if (v > mx) mx = v;
            }
            float scale = (mx - mn) / levels;
            float safe = scale == 0.0f ? 1.0f : scale;
            for (size_t c = 0; c < ORC_GROUP; c++) {
                size_t col = g * ORC_GROUP + c;
                float v = orc_bf16_to_f32(row[col]);
                float qf = rintf((v - mn) / safe);
                if (qf < 0.0f) qf = 0.0f;
                if (qf > (float)qmax) qf = (float)qmax;
                uint32_t q = (uint32_t)qf;
                prow[col / vpw] |= q << ((col % vpw) * (size_t)bits);
            }
            scales[r * groups + g] = orc_f32_to_bf16(scale);
            biases[r * groups + g] = orc_f32_to_bf16(mn);
        }
    }
    return 0;
}

/* ------------------------------------------------------------- layout ---- */

/* EXPERT_LAYOUT / EXPERT_LAYOUT_2BIT (scripts/convert_qwen36.py:38-64); identical to
 * NMOEExpertOffsetsForBits (src/runtime.m:2240-2252). Component order:
 * gate.w, gate.s, gate.b, up.w, up.s, up.b, down.w, down.s, down.b. */
size_t orc_expert_size(int bits) {
    if (bits == 4) return 1769472u;
    if (bits == 2) return 983040u;
    return 0;
}

int orc_expert_offsets(int bits, size_t off[9]) {
    if (bits != 2 && bits != 4) return -1;
    const size_t vpw = 32u / (size_t)bits;
    const size_t w_gu = (size_t)ORC_INTER * (ORC_HIDDEN / vpw) * 4u;   /* gate/up weight bytes */
    const size_t sb_gu = (size_t)ORC_INTER * (ORC_HIDDEN / ORC_GROUP) * 2u;
    const size_t w_d = (size_t)ORC_HIDDEN * (ORC_INTER / vpw) * 4u;
    const size_t sb_d = (size_t)ORC_HIDDEN * (ORC_INTER / ORC_GROUP) * 2u;
    const size_t sizes[9] = {w_gu, sb_gu, sb_gu, w_gu, sb_gu, sb_gu, w_d, sb_d, sb_d};
    size_t o = 0;
    for (int i = 0; i < 9; i++) {
        off[i] = o;
        o += sizes[i];
    }
    return o == orc_expert_size(bits) ? 0 : -1;
}

/* scripts/convert_qwen36.py:377-409: gate = gate_up rows 0..511, up = rows 512..1023,
 * each quantised row-wise, written at the layout offsets as little-endian arrays. */
int orc_pack_expert(const uint16_t *gate_up_bf16, const uint16_t *down_bf16, int bits, uint8_t *blob) {
    size_t off[9];
    if (orc_expert_offsets(bits, off) != 0) return -1;
    memset(blob, 0, orc_expert_size(bits));
    const uint16_t *mats[3] = {gate_up_bf16, gate_up_bf16 + (size_t)ORC_INTER * ORC_HIDDEN, down_bf16};
    const size_t rows[3] = {ORC_INTER, ORC_INTER, ORC_HIDDEN};
    const size_t cols[3] = {ORC_HIDDEN, ORC_HIDDEN, ORC_INTER};
    for (int m = 0; m < 3; m++) {
        int rc = orc_quantize_rows(mats[m], rows[m], cols[m], bits,
                                   (uint32_t *)(blob + off[3 * m]),
                                   (uint16_t *)(blob + off[3 * m + 1]),
                                   (uint16_t *)(blob + off[3 * m + 2]));
        if (rc != 0) return rc;
    }
    return 0;
}

/* ---------------------------------------------------------- math.m ---- */

/* src/math.m:21-28 */
float orc_sigmoid_cpu(float x) {
    if (x >= 0.0f) {
        float z = expf(-x);
        return 1.0f / (1.0f + z);
    }
    float z = expf(x);
    return z / (1.0f + z);
}

/* metal/kernels.metal:177-179 */
float orc_sigmoid_kernel(float x) { return 1.0f / (1.0f + expf(-x)); }

static float orc_silu_kernel(float x) { return x * orc_sigmoid_kernel(x); } /* kernels.metal:181-183 */

/* src/math.m:67-93: max, expf(v - max), long-double sum, multiply by 1/(float)sum. */
void orc_softmax(float *values, size_t count) {
    if (values == NULL || count == 0) return;
    float maxv = values[0];
    for (size_t i = 1; i < count; i++)
        if (values[i] > maxv) maxv = values[i];
    long double sum = 0.0;
    for (size_t i = 0; i < count; i++) {
        values[i] = expf(values[i] - maxv);
        sum += values[i];
    }
    if (sum == 0.0) {
        float uniform = 1.0f / (float)count;
        for (size_t i = 0; i < count; i++) values[i] = uniform;
        return;
    }
    float inv = 1.0f / (float)sum;
    for (size_t i = 0; i < count; i++) values[i] *= inv;
}

/* src/math.m:95-132: k passes, each picks the largest untaken value; strict '>' and the
 * lower index wins a tie. Output order = selection order (descending). */
size_t orc_topk(const float *values, size_t count, size_t k, uint32_t *indices, float *selected) {
    if (values == NULL || count == 0 || indices == NULL || k == 0) return 0;
    if (k > count) k = count;
    uint8_t *taken = calloc(count, 1);
    if (taken == NULL) return 0;
    size_t produced = 0;
    while (produced < k) {
        size_t best_index = 0;
        float best_value = -INFINITY;
        for (size_t i = 0; i < count; i++) {
            if (taken[i]) continue;
            float v = values[i];
            if (v > best_value || (v == best_value && i < best_index)) {
                best_value = v;
                best_index = i;
            }
        }
        taken[best_index] = 1;
        indices[produced] = (uint32_t)best_index;
        if (selected != NULL) selected[produced] = best_value;
        produced++;
    }
    free(taken);
    return produced;
}

/* src/math.m:134-153 (float sum, multiply by 1/sum). */
void orc_renormalize(float *values, size_t count) {
    if (values == NULL || count == 0) return;
    float sum = 0.0f;
    for (size_t i = 0; i < count; i++) sum += values[i];
    if (sum == 0.0f) {
        float uniform = 1.0f / (float)count;
        for (size_t i = 0; i < count; i++) values[i] = uniform;
        return;
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < count; i++) values[i] *= inv;
}

/* metal/kernels.metal:1352-1361 */
void orc_swiglu(const float *gate, const float *up, float *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = orc_silu_kernel(gate[i]) * up[i];
}

/* src/math.m:236-274 */
void orc_dequant_matvec_seq(const uint32_t *packed, const uint16_t *scales, const uint16_t *biases,
                            const float *x, float *y, size_t rows, size_t in_dim, int bits) {
    const size_t vpw = 32u / (size_t)bits;
    const size_t pcols = in_dim / vpw;
    const size_t groups = in_dim / ORC_GROUP;
    const size_t wpg = ORC_GROUP / vpw;
    const uint32_t mask = bits == 2 ? 0x3u : 0xFu;
    for (size_t r = 0; r < rows; r++) {
        float acc = 0.0f;
        for (size_t g = 0; g < groups; g++) {
            float s = orc_bf16_to_f32(scales[r * groups + g]);
            float b = orc_bf16_to_f32(biases[r * groups + g]);
            for (size_t w = 0; w < wpg; w++) {
                uint32_t word = packed[r * pcols + g * wpg + w];
                for (size_t v = 0; v < vpw; v++) {
                    size_t col = g * ORC_GROUP + w * vpw + v;
                    uint32_t q = (word >> (v * (size_t)bits)) & mask;
                    acc += ((float)q * s + b) * x[col];
                }
            }
        }
        y[r] = acc;
    }
}

/* simd_sum over 32 lane partials: fixed butterfly tree. */
static float orc_lane_sum(const float *lanes) {
    float t[32];
    memcpy(t, lanes, sizeof t);
    for (int off = 16; off >= 1; off >>= 1)
        for (int l = 0; l < off; l++) t[l] = t[l] + t[l + off];
    return t[0];
}

static float orc_dequant_row(const uint32_t *prow, const uint16_t *srow, const uint16_t *brow,
                             const float *x, size_t in_dim, int bits, int form) {
    const size_t vpw = 32u / (size_t)bits;
    const size_t pcols = in_dim / vpw;
    const uint32_t mask = bits == 2 ? 0x3u : 0xFu;
    float lanes[32] = {0};
    for (size_t pi = 0; pi < pcols; pi++) {
        uint32_t word = prow[pi];
        size_t base = pi * vpw;
        size_t g = base / ORC_GROUP;
        float s = orc_bf16_to_f32(srow[g]);
        float b = orc_bf16_to_f32(brow[g]);
        float acc = lanes[pi & 31u];
        for (size_t v = 0; v < vpw; v++) {
            float q = (float)((word >> (v * (size_t)bits)) & mask);
            float xv = x[base + v];
            if (form == 0) acc += fmaf(q, s, b) * xv;
            else acc += fmaf(q, s * xv, b * xv);
        }
        lanes[pi & 31u] = acc;
    }
    return orc_lane_sum(lanes);
}

void orc_dequant_matvec(const uint32_t *packed, const uint16_t *scales, const uint16_t *biases,
                        const float *x, float *y, size_t rows, size_t in_dim, int bits, int form) {
    const size_t pcols = in_dim / (32u / (size_t)bits);
    const size_t groups = in_dim / ORC_GROUP;
    long long n = (long long)rows;
#pragma omp parallel for schedule(static) if (n >= 64)
    for (long long r = 0; r < n; r++)
        y[r] = orc_dequant_row(packed + (size_t)r * pcols, scales + (size_t)r * groups,
                               biases + (size_t)r * groups, x, in_dim, bits, form);
}

/* bf16 weights: lane-strided over 8-column chunks, fp32 multiply-add. */
static float orc_bf16_row(const uint16_t *w, const float *x, size_t in_dim) {
    float lanes[32] = {0};
    for (size_t pi = 0; pi < in_dim / 8u; pi++) {
        float acc = lanes[pi & 31u];
        for (size_t v = 0; v < 8; v++) acc += orc_bf16_to_f32(w[pi * 8 + v]) * x[pi * 8 + v];
        lanes[pi & 31u] = acc;
    }
    return orc_lane_sum(lanes);
}

void orc_bf16_matvec(const uint16_t *w, const float *x, float *y, size_t rows, size_t in_dim) {
    long long n = (long long)rows;
#pragma omp parallel for schedule(static) if (n >= 64)
    for (long long r = 0; r < n; r++) y[r] = orc_bf16_row(w + (size_t)r * in_dim, x, in_dim);
}

/* --------------------------------------------------------- block parts ---- */

static void orc_dense_matvec(const orc_dense *d, const float *x, float *y, size_t rows, size_t in_dim,
                             int form) {
    if (d->dtype == ORC_DTYPE_BF16)
        orc_bf16_matvec((const uint16_t *)d->weight, x, y, rows, in_dim);
    else
        orc_dequant_matvec((const uint32_t *)d->weight, d->scales, d->biases, x, y, rows, in_dim, 4, form);
}

/* q4: nmoe_expert_gate_up_q4_batched (kernels.metal:562-640), form 0, SiLU(gate)*up.
 * q2: two nmoe_dequant_matvec_q2 (kernels.metal:192-238, 303-319) then
 *     nmoe_moe_expert_gate_up (kernels.metal:1352-1361) (src/runtime.m:2862-2877). */
void orc_expert_gate_up(const uint8_t *blob, int bits, const float *x, float *act) {
    size_t off[9];
    orc_expert_offsets(bits, off);
    float gate[ORC_INTER], up[ORC_INTER];
    orc_dequant_matvec((const uint32_t *)(blob + off[0]), (const uint16_t *)(blob + off[1]),
                       (const uint16_t *)(blob + off[2]), x, gate, ORC_INTER, ORC_HIDDEN, bits, 0);
    orc_dequant_matvec((const uint32_t *)(blob + off[3]), (const uint16_t *)(blob + off[4]),
                       (const uint16_t *)(blob + off[5]), x, up, ORC_INTER, ORC_HIDDEN, bits, 0);
    orc_swiglu(gate, up, act, ORC_INTER);
}

/* kernels.metal:642-714 (q4) / 192-238 (q2): down [2048][512] applied to act[512]. */
void orc_expert_down(const uint8_t *blob, int bits, const float *act, float *out) {
    size_t off[9];
    orc_expert_offsets(bits, off);
    orc_dequant_matvec((const uint32_t *)(blob + off[6]), (const uint16_t *)(blob + off[7]),
                       (const uint16_t *)(blob + off[8]), act, out, ORC_HIDDEN, ORC_INTER, bits, 0);
}

/* q4 reference path: nmoe_route_shared_q4 (kernels.metal:384-514): rows 0-511 shared
 * SiLU(gate)*up, rows 512-767 router logits, row 768 shared-gate score; all form 1.
 * q2 path (src/runtime.m:3158-3165): router and score by nmoe_dequant_matvec_q4 (form 1),
 * shared gate/up by nmoe_expert_gate_up_q4 (kernels.metal:321-382, form 0).
 * bf16 weights: plain bf16 matvecs. */
void orc_route_shared(const orc_layer *L, const float *x, float *logits, float *shared_act, float *score) {
    const int gu_form = L->bits == 2 ? 0 : 1;
    float gate[ORC_INTER], up[ORC_INTER];
    orc_dense_matvec(&L->router, x, logits, ORC_EXPERTS, ORC_HIDDEN, 1);
    orc_dense_matvec(&L->shared_gate, x, gate, ORC_INTER, ORC_HIDDEN, gu_form);
    orc_dense_matvec(&L->shared_up, x, up, ORC_INTER, ORC_HIDDEN, gu_form);
    orc_swiglu(gate, up, shared_act, ORC_INTER);
    orc_dense_matvec(&L->shared_gate_vec, x, score, 1, ORC_HIDDEN, 1);
}

int orc_moe_block_forward(const orc_layer *L, int k, const float *x, const float *h_mid,
                          const float *logits_override, float *out, uint32_t *idx, float *w,
                          float *logits, float *shared_act, float *score) {
    if (L == NULL || x == NULL || k < 1 || k > ORC_MAX_K) return -1;
    if (L->bits != 2 && L->bits != 4) return -1;
    const size_t esz = orc_expert_size(L->bits);

    float lg[ORC_EXPERTS], sact[ORC_INTER], sc = 0.0f;
    orc_route_shared(L, x, lg, sact, &sc);
    if (logits) memcpy(logits, lg, sizeof lg);
    if (shared_act) memcpy(shared_act, sact, sizeof sact);
    if (score) *score = sc;

    /* NMOESelectRouteTopKCPU (src/runtime.m:1498-1511) */
    float probs[ORC_EXPERTS];
    memcpy(probs, logits_override ? logits_override : lg, sizeof probs);
    orc_softmax(probs, ORC_EXPERTS);
    uint32_t sel[ORC_MAX_K] = {0};
    float vals[ORC_MAX_K] = {0};
    size_t n = orc_topk(probs, ORC_EXPERTS, (size_t)k, sel, vals);
    orc_renormalize(vals, n);

    /* params packing (src/runtime.m:2976-2983): [0..7] weights, [8] raw shared score */
    float params[16] = {0};
    for (size_t i = 0; i < n && i < 8; i++) params[i] = vals[i];
    params[8] = sc;
    if (idx) {
        for (int i = 0; i < ORC_MAX_K; i++) idx[i] = i < (int)n ? sel[i] : 0u;
    }
    if (w) {
        for (int i = 0; i < ORC_MAX_K; i++) w[i] = i < (int)n ? vals[i] : 0.0f;
    }
    if (out == NULL) return 0;

    static __thread float act[ORC_MAX_K][ORC_INTER];
    static __thread float dout[ORC_MAX_K][ORC_HIDDEN];
    float sdown[ORC_HIDDEN];
    for (size_t s = 0; s < n; s++) {
        if (sel[s] >= L->num_experts) return -2;
        const uint8_t *blob = L->experts + (size_t)sel[s] * esz;
        orc_expert_gate_up(blob, L->bits, x, act[s]);
        orc_expert_down(blob, L->bits, act[s], dout[s]);
    }
    /* shared down: q4 fused combine uses form 0 (kernels.metal:1519-1530); the q2 path
     * runs it through nmoe_dequant_matvec_q4 (form 1, src/runtime.m:2798-2800). */
    orc_dense_matvec(&L->shared_down, sact, sdown, ORC_HIDDEN, ORC_INTER, L->bits == 4 ? 0 : 1);

    /* nmoe_expert_down_combine_q4 (kernels.metal:1497-1541) / nmoe_weighted_expert_sum
     * (kernels.metal:1394-1423): h_mid + sum_s params[s]*down_s + sigmoid(params[8])*shared */
    const float sg = orc_sigmoid_kernel(params[8]);
    for (size_t r = 0; r < ORC_HIDDEN; r++) {
        float moe = 0.0f;
        for (size_t s = 0; s < n; s++) moe += params[s] * dout[s][r];
        float hm = h_mid ? h_mid[r] : 0.0f;
        out[r] = hm + moe + sg * sdown[r];
    }
    return 0;
}

int orc_moe_block_forward_batched(const orc_layer *L, int T, int k, const float *x,
                                  const float *h_mid, float *out, uint32_t *idx, float *w) {
    if (T < 0) return -1;
    int rc = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : rc)
    for (int t = 0; t < T; t++) {
        rc |= orc_moe_block_forward(L, k, x + (size_t)t * ORC_HIDDEN,
                                    h_mid ? h_mid + (size_t)t * ORC_HIDDEN : NULL, NULL,
                                    out + (size_t)t * ORC_HIDDEN, idx ? idx + (size_t)t * ORC_MAX_K : NULL,
                                    w ? w + (size_t)t * ORC_MAX_K : NULL, NULL, NULL, NULL);
    }
    return rc;
}

/* ------------------------------------------------------------- LM head ---- */

void orc_rms_norm(const float *x, const uint16_t *w_bf16, float *out, size_t n, float eps, int add_one) {
    double ss = 0.0;
    for (size_t i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    const float inv = 1.0f / sqrtf((float)(ss / (double)n) + eps);
    for (size_t i = 0; i < n; i++) {
        float w = 1.0f;
        if (w_bf16 != NULL) {
            w = orc_bf16_to_f32(w_bf16[i]);
            if (add_one) w += 1.0f;
        }
        out[i] = x[i] * inv * w;
    }
}

uint32_t orc_argmax_top1(const float *v, size_t n) {
    float best = -FLT_MAX;
    uint32_t idx = 0;
    for (size_t i = 0; i < n; i++)
        if (v[i] > best) {   /* strict: the earlier index keeps a tie; NaN compares false */
            best = v[i];
            idx = (uint32_t)i;
        }
    return idx;
}

uint32_t orc_lm_head_argmax(int dtype, const void *w, const uint16_t *s, const uint16_t *b, size_t vocab,
                            size_t in_dim, const float *x, const uint16_t *norm_w, float eps, int add_one,
                            float *logits) {
    float *xn = (float *)malloc(in_dim * sizeof(float));
    float *lg = logits != NULL ? logits : (float *)malloc(vocab * sizeof(float));
    if (norm_w != NULL)
        orc_rms_norm(x, norm_w, xn, in_dim, eps, add_one);
    else
        memcpy(xn, x, in_dim * sizeof(float));
    if (dtype == ORC_DTYPE_BF16)
        orc_bf16_matvec((const uint16_t *)w, xn, lg, vocab, in_dim);
    else
        orc_dequant_matvec((const uint32_t *)w, s, b, xn, lg, vocab, in_dim, 4, 0);
    const uint32_t tok = orc_argmax_top1(lg, vocab);
    if (lg != logits) free(lg);
    free(xn);
    return tok;
}

/* ------------------------------------------------------------- CRC-32C ---- */

uint32_t orc_crc32c(uint32_t crc, const uint8_t *data, size_t n) {
    crc = ~crc;
    for (size_t i = 0; i < n; i++) {
        crc ^= data[i];
        for (int b = 0; b < 8; b++) crc = (crc & 1u) ? (crc >> 1) ^ 0x82F63B78u : crc >> 1;
    }
    return ~crc;
}

/* ------------------------------------------------- linear attention step ---- */

#define ORC_LA_KH 16
#define ORC_LA_VH 32
#define ORC_LA_D 128
#define ORC_LA_CONV 8192

void orc_linear_attn_step(const float *qkv, const float *z, const float *alpha, const float *beta,
                          const uint16_t *conv_w, const float *A_log, const uint16_t *dt_bias,
                          const uint16_t *norm_w, float *conv_state, float *delta_state, float *out) {
    float *cv = (float *)malloc(ORC_LA_CONV * sizeof(float));
    /* kernels.metal:1275-1295 */
    for (int i = 0; i < ORC_LA_CONV; i++) {
        float acc = 0.0f;
        acc += conv_state[0 * ORC_LA_CONV + i] * orc_bf16_to_f32(conv_w[4 * i + 0]);
        acc += conv_state[1 * ORC_LA_CONV + i] * orc_bf16_to_f32(conv_w[4 * i + 1]);
        acc += conv_state[2 * ORC_LA_CONV + i] * orc_bf16_to_f32(conv_w[4 * i + 2]);
        const float inp = qkv[i];
        acc += inp * orc_bf16_to_f32(conv_w[4 * i + 3]);
        cv[i] = orc_silu_kernel(acc);
        conv_state[0 * ORC_LA_CONV + i] = conv_state[1 * ORC_LA_CONV + i];
        conv_state[1 * ORC_LA_CONV + i] = conv_state[2 * ORC_LA_CONV + i];
        conv_state[2 * ORC_LA_CONV + i] = inp;
    }
    /* kernels.metal:1780-1821, inv_scale = 1/sqrt(128), eps 1e-12 (src/runtime.m:3360, 3410) */
    const float inv_scale = 1.0f / sqrtf((float)ORC_LA_D);
    for (int h = 0; h < ORC_LA_KH; h++) {
        float *q = cv + h * ORC_LA_D, *k = cv + 2048 + h * ORC_LA_D;
        float sq = 0.0f, sk = 0.0f;
        for (int i = 0; i < ORC_LA_D; i++) sq += q[i] * q[i];
        const float qi = 1.0f / sqrtf(sq / (float)ORC_LA_D + 1e-12f);
        for (int i = 0; i < ORC_LA_D; i++) q[i] = q[i] * qi * inv_scale * inv_scale;
        for (int i = 0; i < ORC_LA_D; i++) sk += k[i] * k[i];
        const float ki = 1.0f / sqrtf(sk / (float)ORC_LA_D + 1e-12f);
        for (int i = 0; i < ORC_LA_D; i++) k[i] = k[i] * ki * inv_scale;
    }
    for (int vh = 0; vh < ORC_LA_VH; vh++) {
        /* kernels.metal:1823-1839 */
        const float A = expf(A_log[vh]);
        const float sp = logf(1.0f + expf(alpha[vh] + orc_bf16_to_f32(dt_bias[vh])));
        const float g = expf(-A * sp);
        const float b = orc_sigmoid_kernel(beta[vh]);
        const int kh = vh / 2;
        const float *q = cv + kh * ORC_LA_D, *k = cv + 2048 + kh * ORC_LA_D, *v = cv + 4096 + vh * ORC_LA_D;
        float o[ORC_LA_D];
        /* kernels.metal:1300-1346 */
        for (int vi = 0; vi < ORC_LA_D; vi++) {
            float *S = delta_state + ((size_t)vh * ORC_LA_D + vi) * ORC_LA_D;
            float kv = 0.0f;
            for (int i = 0; i < ORC_LA_D; i++) {
                const float s = S[i] * g;
                S[i] = s;
                kv += s * k[i];
            }
            const float d = (v[vi] - kv) * b;
            for (int i = 0; i < ORC_LA_D; i++) S[i] += k[i] * d;
            float ov = 0.0f;
            for (int i = 0; i < ORC_LA_D; i++) ov += S[i] * q[i];
            o[vi] = ov;
        }
        /* kernels.metal:1841-1873, eps 1e-6 */
        float ss = 0.0f;
        for (int vi = 0; vi < ORC_LA_D; vi++) ss += o[vi] * o[vi];
        const float inv = 1.0f / sqrtf(ss / (float)ORC_LA_D + 1e-6f);
        for (int vi = 0; vi < ORC_LA_D; vi++)
            out[vh * ORC_LA_D + vi] = o[vi] * inv * orc_silu_kernel(z[vh * ORC_LA_D + vi]) *
                                      orc_bf16_to_f32(norm_w[vi]);
    }
    free(cv);
}

/* --------------------------------------------------- full attention step ---- */

static void orc_fa_prep(float *vec, const uint16_t *w, int position) {
    float ss = 0.0f;
    for (int i = 0; i < 256; i++) ss += vec[i] * vec[i];
    const float inv = 1.0f / sqrtf(ss / 256.0f + 1e-6f);
    for (int i = 0; i < 256; i++) vec[i] = vec[i] * inv * (orc_bf16_to_f32(w[i]) + 1.0f);
    for (int t = 0; t < 32; t++) {   /* kernels.metal:1042-1053, rotary_dim 64 */
        /* theta^(-2t/64) correctly rounded to float (the kernel's pow in float can differ
         * by an ulp, and at position p the angle moves by p ulps of freq) */
        const float freq = (float)pow(10000000.0, -2.0 * (double)t / 64.0);
        const float ang = (float)position * freq;
        const float c = cosf(ang), s = sinf(ang);
        const float v0 = vec[t], v1 = vec[t + 32];
        vec[t] = v0 * c - v1 * s;
        vec[t + 32] = v0 * s + v1 * c;
    }
}

static void fa_step(const float *q, const float *k_new, const float *v_new, const uint16_t *q_norm,
                    const uint16_t *k_norm, float *k_cache, float *v_cache, int position, float *out, int bf16_kv) {
    for (int kh = 0; kh < 2; kh++) {
        float kv[256], vv[256];
        memcpy(kv, k_new + kh * 256, sizeof kv);
        memcpy(vv, v_new + kh * 256, sizeof vv);
        orc_fa_prep(kv, k_norm, position);
        if (bf16_kv)   /* the rows as a bf16 cache stores them (round to nearest even) */
            for (int i = 0; i < 256; i++) {
                kv[i] = orc_bf16_to_f32(orc_f32_to_bf16(kv[i]));
                vv[i] = orc_bf16_to_f32(orc_f32_to_bf16(vv[i]));
            }
        memcpy(k_cache + ((size_t)position * 2 + kh) * 256, kv, sizeof kv);
        memcpy(v_cache + ((size_t)position * 2 + kh) * 256, vv, sizeof vv);
    }
    const int seq = position + 1;
    float *sc = (float *)malloc((size_t)seq * sizeof(float));
    for (int h = 0; h < 16; h++) {
        float qh[256];
        memcpy(qh, q + h * 512, sizeof qh);
        orc_fa_prep(qh, q_norm, position);
        const int kh = h / 8;
        float m = -1e30f;
        for (int p = 0; p < seq; p++) {
            const float *kp = k_cache + ((size_t)p * 2 + kh) * 256;
            float d = 0.0f;
            for (int i = 0; i < 256; i++) d += qh[i] * kp[i];
            sc[p] = d * (1.0f / 16.0f);
            if (sc[p] > m) m = sc[p];
        }
        double l = 0.0;
        for (int p = 0; p < seq; p++) l += exp((double)(sc[p] - m));
        for (int i = 0; i < 256; i++) {
            double a = 0.0;
            for (int p = 0; p < seq; p++) a += exp((double)(sc[p] - m)) * v_cache[((size_t)p * 2 + kh) * 256 + i];
            out[h * 256 + i] = (float)(a / l) * orc_sigmoid_kernel(q[h * 512 + 256 + i]);
        }
    }
    free(sc);
}

void orc_full_attn_step(const float *q, const float *k_new, const float *v_new, const uint16_t *q_norm,
                        const uint16_t *k_norm, float *k_cache, float *v_cache, int position, float *out) {
    fa_step(q, k_new, v_new, q_norm, k_norm, k_cache, v_cache, position, out, 0);
}

void orc_full_attn_step_bf16kv(const float *q, const float *k_new, const float *v_new, const uint16_t *q_norm,
                               const uint16_t *k_norm, float *k_cache, float *v_cache, int position, float *out) {
    fa_step(q, k_new, v_new, q_norm, k_norm, k_cache, v_cache, position, out, 1);
}
