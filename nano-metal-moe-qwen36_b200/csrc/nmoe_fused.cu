// nmoe_fused.cu -- batch-1 routed-MoE block in ONE persistent launch (sm_100a).
//
// Grid = one 512-thread CTA per SM, launched cooperatively so that every CTA is
// resident and the bounded cross-CTA wait cannot deadlock. Work per CTA c of G:
//   router rows      [c*256/G, (c+1)*256/G)            -> logits (published)
//   shared rows      [c*512/G, (c+1)*512/G)            -> shared act (kept local)
//   gate vector      every CTA                          -> score (kept local)
//   routed units     u = c, c+G, ... < 32k              (unit = slot u/32, 16-row band u%32)
//   output rows      [c*2048/G, (c+1)*2048/G)           initialised to h_mid (or 0)
// The block output is accumulated split-K over the intermediate dimension: a CTA that
// holds intermediate rows (a shared row, or one routed unit's 16 rows) also holds the
// matching COLUMNS of the down matrix (nmoe_pack.cuh: down group slabs; the dense
// arena's column copy of the shared down), so it turns its activations into a partial
// 2048-row output without seeing anyone else's. Each thread keeps 4 output rows in
// registers across its CTA's shared and routed partials and adds them into `out` with
// one red.global.add.v4.f32 at the end. The only cross-CTA exchange left is the router
// logits: every CTA needs all 256 of them for the top-k. Their publication doubles as
// the barrier that orders every CTA's output-row initialisation before anyone's add.
// The adds are fp32 reductions in arrival order: the output is reproducible to fp32
// rounding of the sum order, not bitwise.
//
// Weight bytes move by cp.async.bulk straight into shared memory (one copy per slice):
// the routing-independent ones (router rows, shared rows and columns, gate vector) are
// issued before the programmatic-dependent-launch wait, the routed ones as soon as this
// CTA knows the top-k. While the router runs, each CTA touches the first and last line
// of its share of the layer's 256 expert blobs, so that the address translations of
// whichever experts win are warm when their copies go out.
// Routed gate/up dots use the packed values in place as exact subnormal halves against
// a per-call scaled half2 table of x, flushed to fp32 once per word (or fp32 FFMA2 with
// NMOE_FLAG_EXPERT_FP32); the affine dequantisation is applied per 64-column group as
// s * sum(q*x) + b * sum(x). Router, shared-expert and all down products are fp32.
// The logits are published as 64-bit words {launch tag, value}; a consumer polls the
// words it needs until all carry this launch's tag -- one L2 round trip after the last
// producer, no separate counter. The tag is epoch + 1, and the last CTA to finish
// advances the epoch for the next launch. Every wait is bounded (timer and iteration
// cap) and reports NMOE_ETIMEOUT through the device error word.
//
// Reference math: router/shared (metal/kernels.metal:384-514), top-k on the logits with
// the selection rule of src/math.m:95-132 and weights exp(l_s - l_0)/sum_t exp(l_t - l_0)
// (the renormalised softmax, src/runtime.m:1498-1511), SwiGLU gate/up
// (kernels.metal:716-788), down + sigmoid-gated shared expert + combine
// (kernels.metal:1456-1542).
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>

#include <cuda_fp16.h>

#include "nmoe_fused.cuh"
#include "nmoe_pack.cuh"
#include "nmoe_sm100.cuh"
#include "nmoe_topk.cuh"

namespace nmoe {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kXP = 36;   // padded floats per 32 columns (conflict-free 16-byte lane reads)
constexpr int kMaxUnits = 4;
constexpr uint32_t kUnset = 0xFFFFFFFFu;   // top-k slot not decided yet
constexpr int kTlSlots = 32;
constexpr int kLogitCopies = 8;
// mbarriers: router rows, shared expert, then per routed unit its gate/up part (band pair
// + scales) and its down part (word columns + group scales/biases)
constexpr int kBarRouter = 0, kBarShared = 1, kBarGu0 = 2, kBarD0 = kBarGu0 + kMaxUnits, kNumBars = kBarD0 + kMaxUnits;

struct FusedSync {
    uint32_t epoch, done_cnt;
    uint32_t pad[30];
    uint32_t arrive;                 // logits publications of all launches (+G per launch)
    uint32_t pad1[31];
    uint32_t inited;                 // output-row initialisations of all launches (+G per launch)
    uint32_t pad3[31];
    // tagged {tag, value} logits in kLogitCopies copies: CTA c reads copy c % kLogitCopies,
    // so that the 148 reads that follow the last publication spread over 8x the L2 lines
    uint64_t logits[kLogitCopies][kExperts];
    uint32_t diag[1024];             // per CTA: highest phase reached; 100+phase where a wait gave up
    uint32_t tl[1024][kTlSlots];     // per CTA phase timestamps (globaltimer low 32 bits)
};

struct FusedLayout {
    uint32_t bars, ctl, xs, xsum, xh, rw, gv, sp, sdt, dsp, sact, uact, atab, units, total;
    uint32_t unit_bytes;   // one routed unit: band pair | down word columns | group scales+biases
    int nRmax, nSmax, nUmax, kmax;
};

struct FusedParams {
    const uint8_t *experts;   // repacked expert blobs of this layer
    const uint8_t *router, *spairs, *gvec, *sdown_t;   // repacked dense regions
    const uint8_t *next_dense;   // dense arena to prefetch into L2 during the tail, or null
    uint32_t next_dense_bytes;
    const void *x;
    int x_f32;
    const float *h_mid;
    float *out;
    uint32_t *idx_out;
    float *w_out;
    float *logits_out;
    int k, num_experts, route_only;
    int stall;   // test hook: the logits wait looks for a tag that is never written
    FusedSync *sy;
    int *err;
    FusedLayout lay;
    uint64_t timeout_ns;
};

struct Ctl {
    uint32_t xmax_bits;           // max |x| (float bits; non-negative floats order as ints)
    int abort;
    int rdone, sdone;
    uint32_t armed;               // barriers with a transaction count posted (teardown drain)
    uint32_t idx[kMaxK];
    float w[kMaxK];
    int valid[kMaxK];
    float score;
    uint32_t sidx[kMaxK], dsidx[kMaxK];   // top-k ids (real / warm-up pass)
    float sval[kMaxK], dsval[kMaxK];      // top-k logits (real / warm-up pass)
    float sink[kWarps];                   // results of the warm-up passes
    uint32_t amax_bits[kMaxUnits];        // max |act| per routed unit (float bits)
};

__device__ __forceinline__ void st_tagged(uint64_t *p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// Poll 8 consecutive tagged words (64-byte aligned): all four loads of an attempt are in
// flight together, so a successful attempt costs one L2 round trip.
__device__ __forceinline__ bool poll_tagged8(const uint64_t *p, uint32_t tag, float *v, uint64_t deadline) {
    for (uint32_t it = 0;; ++it) {
        uint64_t a[8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(a[2 * j]), "=l"(a[2 * j + 1]) : "l"(p + 2 * j) : "memory");
        bool all = true;
#pragma unroll
        for (int j = 0; j < 8; ++j) all &= (uint32_t)(a[j] >> 32) == tag;
        if (all) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __uint_as_float((uint32_t)a[j]);
            return true;
        }
        if (it >= kMaxSpins || globaltimer_ns() > deadline) return false;
    }
}

// total * i < 2^32 for every split here (total <= 2048, i <= grid <= 1024): 32-bit unsigned
// division, inline (a 64-bit division is a called routine, slow on a cold instruction cache)
__device__ __forceinline__ int split_lo(int total, int parts, int i) {
    return (int)(((uint32_t)total * (uint32_t)i) / (uint32_t)parts);
}
__device__ __forceinline__ void set_err(int *err, int code) { atomicCAS(err, 0, code); }

__device__ __forceinline__ void red_add_v4(float *p, float a, float b, float c, float d) {
    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// ---------------------------------------------------------------- FFMA dense path ----
__device__ __forceinline__ float mant(uint32_t bits) { return __uint_as_float(bits | 0x3F800000u); }
// 32 q4 columns: nibble q placed in mantissa bits [15,18] reads 1 + q/256, in [19,22]
// 1 + q/16; removing sum(x) per column parity leaves sum(q*x).
__device__ __forceinline__ float q4_dot32(const uint4 w, const float *xr, float xe, float xo) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    float al = 0.f, ah = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t a = ws[j] << 15, b = ws[j] << 7, c = ws[j] >> 1, d = ws[j] >> 9;
        al = fmaf(mant(a & 0x00078000u), xr[8 * j + 0], al);
        ah = fmaf(mant(a & 0x00780000u), xr[8 * j + 1], ah);
        al = fmaf(mant(b & 0x00078000u), xr[8 * j + 2], al);
        ah = fmaf(mant(b & 0x00780000u), xr[8 * j + 3], ah);
        al = fmaf(mant(c & 0x00078000u), xr[8 * j + 4], al);
        ah = fmaf(mant(c & 0x00780000u), xr[8 * j + 5], ah);
        al = fmaf(mant(d & 0x00078000u), xr[8 * j + 6], al);
        ah = fmaf(mant(d & 0x00780000u), xr[8 * j + 7], ah);
    }
    return 256.f * (al - xe) + 16.f * (ah - xo);
}

__device__ __forceinline__ void load_x32(const float *xs, int c32, float *xr) {
    const float *p = xs + c32 * kXP;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = lds128f(p + 4 * i);
        xr[4 * i] = v.x; xr[4 * i + 1] = v.y; xr[4 * i + 2] = v.z; xr[4 * i + 3] = v.w;
    }
}
__device__ __forceinline__ void load_x8(const float *xs, int c8, float *xr) {
    const float *p = xs + (c8 >> 2) * kXP + (c8 & 3) * 8;
    const float4 a = lds128f(p), b = lds128f(p + 4);
    xr[0] = a.x; xr[1] = a.y; xr[2] = a.z; xr[3] = a.w; xr[4] = b.x; xr[5] = b.y; xr[6] = b.z; xr[7] = b.w;
}

// Lane partials of NR dense rows (smem): q4 rows (w, s, b) or bf16 rows (w).
// Lane handles 16-byte chunks c = c0, c0 + cstep, ... < c1.
template <bool kQ4, int NR>
__device__ __forceinline__ void dense_dot(const uint8_t *const *w, const uint16_t *const *s, const uint16_t *const *b,
                                          const float *xs, const float *xsum, int c0, int cstep, int c1, float *acc) {
    // one or two trips per lane at the kernel's shapes: no unrolling (code size is latency)
    if (kQ4) {
#pragma unroll 1
        for (int c = c0; c < c1; c += cstep) {
            float xr[32];
            load_x32(xs, c, xr);
            const float xe = xsum[3 * c], xo = xsum[3 * c + 1], xa = xsum[3 * c + 2];
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const float sc = bf16_to_f32(s[r][c >> 1]), bi = bf16_to_f32(b[r][c >> 1]);
                acc[r] = fmaf(sc, q4_dot32(lds128(w[r] + 16 * c), xr, xe, xo), fmaf(bi, xa, acc[r]));
            }
        }
    } else {
#pragma unroll 1
        for (int c = c0; c < c1; c += cstep) {
            float xr[8];
            load_x8(xs, c, xr);
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] += bf16_dot8(lds128(w[r] + 16 * c), xr);
        }
    }
}

// Warp-reduced dot products with x of one dense row ([w | s | b], NR = 1: a router row or
// the gate vector) or one shared gate/up pair (NR = 2) over chunks [c0, c1) (noinline:
// one copy of the code, warmed before the dependency wait).
template <bool kQ4, int NR>
__device__ __noinline__ float2 dense_seg(const uint8_t *base, const float *xs, const float *xsum, int c0, int c1,
                                         int lane) {
    const uint8_t *w[2] = {base, base + (kQ4 ? 1024 : 4096)};
    const uint16_t *sp[2] = {reinterpret_cast<const uint16_t *>(base + (NR == 1 ? 1024 : 2048)),
                             reinterpret_cast<const uint16_t *>(base + 2176)};
    const uint16_t *bp[2] = {reinterpret_cast<const uint16_t *>(base + (NR == 1 ? 1088 : 2112)),
                             reinterpret_cast<const uint16_t *>(base + 2240)};
    float acc[2] = {0.f, 0.f};
    dense_dot<kQ4, NR>(w, sp, bp, xs, xsum, c0 + lane, 32, c1, acc);
    return make_float2(warp_sum(acc[0]), NR == 2 ? warp_sum(acc[1]) : 0.f);
}

// ------------------------------------------------------- routed experts: f32x2 ----
// Blackwell's packed fp32 FMA (fma.rn.f32x2) over a conversion-free dequant: one shift
// of a packed word puts an even-column value in mantissa bits [15,18] (q4: reads
// 1 + q/256) and the next odd-column value in [19,22] (1 + q/16); two LOP3s make the fp32
// pair, one FFMA2 accumulates both against (v_even, v_odd). q2 words use bits [19,20]
// (1 + q/16) and [21,22] (1 + q/4). 2 instructions per weight, fp32 math.
__device__ __forceinline__ uint64_t u64_of(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }
__device__ __forceinline__ void ffma2(uint64_t &acc, uint64_t a, uint64_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// sum(q*v) over NW packed words (q4: 8 columns each, q2: 16); x2[i] = (v[2i], v[2i+1]),
// ve / vo = the sums of the even / odd columns.
template <int kBits, int NW>
__device__ __forceinline__ float qdot_f32(const uint32_t *ws, const uint64_t *x2, float ve, float vo) {
    uint64_t acc = 0ull;
    if (kBits == 4) {
#pragma unroll
        for (int j = 0; j < NW; ++j) {
            const uint32_t sh[4] = {ws[j] << 15, ws[j] << 7, ws[j] >> 1, ws[j] >> 9};
#pragma unroll
            for (int p = 0; p < 4; ++p)
                ffma2(acc, u64_of((sh[p] & 0x00078000u) | 0x3F800000u, (sh[p] & 0x00780000u) | 0x3F800000u),
                      x2[4 * j + p]);
        }
        return 256.f * (lo_f(acc) - ve) + 16.f * (hi_f(acc) - vo);
    } else {
#pragma unroll
        for (int j = 0; j < NW; ++j) {
#pragma unroll
            for (int p = 0; p < 8; ++p) {
                const int sft = 19 - 4 * p;
                const uint32_t v = sft >= 0 ? (ws[j] << sft) : (ws[j] >> (-sft));
                ffma2(acc, u64_of((v & 0x00180000u) | 0x3F800000u, (v & 0x00600000u) | 0x3F800000u), x2[8 * j + p]);
            }
        }
        return 16.f * (lo_f(acc) - ve) + 4.f * (hi_f(acc) - vo);
    }
}

// Lane's x chunk: 32 (q4) or 64 (q2) columns from the padded fp32 layout as fp32 pairs,
// plus the chunk's even/odd column sums.
template <int kBits>
__device__ __forceinline__ void load_chunk_x2(const float *vpad, const float *vsum, int chunk, uint64_t *x2, float &xe,
                                              float &xo) {
    constexpr int n32 = kBits == 4 ? 1 : 2;
#pragma unroll
    for (int q = 0; q < n32; ++q) {
        const float *p = vpad + (n32 * chunk + q) * kXP;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = lds128f(p + 4 * i);
            x2[16 * q + 2 * i] = u64_of(__float_as_uint(v.x), __float_as_uint(v.y));
            x2[16 * q + 2 * i + 1] = u64_of(__float_as_uint(v.z), __float_as_uint(v.w));
        }
    }
    xe = vsum[3 * n32 * chunk] + (n32 == 2 ? vsum[3 * (2 * chunk + 1)] : 0.f);
    xo = vsum[3 * n32 * chunk + 1] + (n32 == 2 ? vsum[3 * (2 * chunk + 1) + 1] : 0.f);
}

// ---------------------------------------------- routed experts: half2 (default) ----
// Packed values used in place as exact subnormal halves: in each 16-bit half of a word,
// (w & 0x000F << 4p) reads q * 2^(4p-24) for p in {0,1} (q2: 0x0003 << 2p, p < 4); a
// single w >> 8 brings the other positions down. Multiplied by v * 2^(E - 4p) (the pair
// table below) every product is q * v * 2^(E-24), accumulated 4 (q4) / 8 (q2) deep in
// half2 and flushed to fp32 once per word: 0.6 integer and ~1 FP16 instruction per
// weight, about twice the rate of the fp32 path, ~3e-4 relative error per dot.
template <int kBits, int NW>
__device__ __forceinline__ float qdot_h2(const uint32_t *ws, const __half2 *xh) {
    constexpr int kFlush = 1;   // words per half2 accumulation
    float acc = 0.f;
    __half2 h = __float2half2_rn(0.f);
#pragma unroll
    for (int j = 0; j < NW; ++j) {
        const uint32_t w8 = ws[j] >> 8;
        if (kBits == 4) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint32_t q = (i < 2 ? ws[j] : w8) & (0x000F000Fu << (4 * (i & 1)));
                h = __hfma2(*reinterpret_cast<const __half2 *>(&q), xh[4 * j + i], h);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint32_t q = (i < 4 ? ws[j] : w8) & (0x00030003u << (2 * (i & 3)));
                h = __hfma2(*reinterpret_cast<const __half2 *>(&q), xh[8 * j + i], h);
            }
        }
        if ((j + 1) % kFlush == 0 || j + 1 == NW) {
            const float2 f = __half22float2(h);
            acc += f.x + f.y;
            h = __float2half2_rn(0.f);
        }
    }
    return acc;
}

// Scale exponent of a vector with max |v| = vmax: vmax * 2^E <= 2^15 (half range).
__device__ __forceinline__ int half_exp(float vmax) {
    if (!(vmax > 0.f) || !isfinite(vmax)) return 0;
    return 15 - (int)ceilf(log2f(vmax));
}

// Pair entry k (0..15 for q4, 0..31 for q2) of one 16-byte chunk of a vector v (read
// through vat(column)): q4 entry 4j+i = (v[8j+i], v[8j+i+4]) * 2^(E-4(i&1));
// q2 entry 8j+i = (v[16j+i], v[16j+i+8]) * 2^(E-2(i&3)).
template <int kBits, class F>
__device__ __forceinline__ __half2 pair_of(F vat, int k, int E) {
    constexpr int half_span = kBits == 4 ? 4 : 8, wcols = kBits == 4 ? 8 : 16;
    const int j = k / half_span, i = k % half_span;
    const int c0 = wcols * j + i;
    const float sc = exp2f((float)(E - (kBits == 4 ? 4 * (i & 1) : 2 * (i & 3))));
    return __floats2half2_rn(vat(c0) * sc, vat(c0 + half_span) * sc);
}
// The x pair table: 64 (q4) / 32 (q2) chunks of 16 / 32 entries, stored
// [entry / 4][chunk][4] so that the 32 lanes of a warp, reading chunks lane and
// lane + 32, read consecutive 16-byte cells (no bank conflicts).
template <int kBits>
__device__ __forceinline__ int xtab_pos(int chunk, int k) {
    constexpr int nch = kBits == 4 ? 64 : 32;
    return ((k >> 2) * nch + chunk) * 4 + (k & 3);
}

// ------------------------------------------------------------- routed units ----
// 2^n as a float, n in [-126, 127]: built from the exponent field, no MUFU.
__device__ __forceinline__ float pow2i(int n) { return __int_as_float((127 + n) << 23); }
// half_exp(vmax) from the float bits of vmax >= 0: 15 - ceil(log2(vmax)), integer only.
__device__ __forceinline__ int half_exp_bits(uint32_t b) {
    if (b == 0u || b >= 0x7F800000u) return 0;
    int e = (int)(b >> 23) - 127;
    if (b & 0x007FFFFFu) e += 1;   // ceil of log2 of a non-power of two
    e = 15 - e;
    return e < -100 ? -100 : (e > 100 ? 100 : e);
}

// SiLU(gate . x) * (up . x) of row pair `warp` of NU routed units at once (their band
// pairs at up[n]); the lane's x chunks (xhr: pair-table entries, x2: fp32 pairs) are
// loaded once for all units, and the units' dot products interleave. act[n] on every lane.
template <int kBits, bool kHalf, int NU>
__device__ __forceinline__ void units_act(const uint8_t *const *up, const __half2 *xtab, const float *xs,
                                          const float *xsum, float hscale, int warp, int lane, float *act) {
    const PackGeo pg = pack_geo(kBits);
    constexpr int kChunksPerLane = kBits == 4 ? 2 : 1;   // 64 (q4) / 32 (q2) chunks per row
    constexpr int kPairs = kBits == 4 ? 16 : 32;         // pair-table entries per chunk
    float g[NU], uu[NU];
#pragma unroll
    for (int n = 0; n < NU; ++n) g[n] = uu[n] = 0.f;
#pragma unroll
    for (int q = 0; q < kChunksPerLane; ++q) {
        const int ch = lane + 32 * q, grp = kBits == 4 ? ch >> 1 : ch;
        const int n32 = kBits == 4 ? 1 : 2;
        float xe = xsum[3 * n32 * ch] + (n32 == 2 ? xsum[3 * (2 * ch + 1)] : 0.f);
        float xo = xsum[3 * n32 * ch + 1] + (n32 == 2 ? xsum[3 * (2 * ch + 1) + 1] : 0.f);
        __half2 xhr[kHalf ? kPairs : 1];
        uint64_t x2[kHalf ? 1 : 16 * (kBits == 4 ? 1 : 2)];
        if (kHalf) {
#pragma unroll
            for (int e = 0; e < kPairs; e += 4) {
                const uint4 t4 = *reinterpret_cast<const uint4 *>(xtab + xtab_pos<kBits>(ch, e));
                xhr[e] = *reinterpret_cast<const __half2 *>(&t4.x);
                xhr[e + 1] = *reinterpret_cast<const __half2 *>(&t4.y);
                xhr[e + 2] = *reinterpret_cast<const __half2 *>(&t4.z);
                xhr[e + 3] = *reinterpret_cast<const __half2 *>(&t4.w);
            }
        } else {
            load_chunk_x2<kBits>(xs, xsum, ch, x2, xe, xo);
        }
        const float xa = xe + xo;
#pragma unroll
        for (int n = 0; n < NU; ++n) {
            const uint8_t *gw = up[n] + warp * pg.wgu * 4, *uw = gw + pg.tile_band_gu;
            const uint16_t *gs = reinterpret_cast<const uint16_t *>(up[n] + 2 * pg.tile_band_gu) + warp * 32;
            const uint4 wg4 = lds128(gw + 16 * ch), wu4 = lds128(uw + 16 * ch);
            const uint32_t wg[4] = {wg4.x, wg4.y, wg4.z, wg4.w}, wu[4] = {wu4.x, wu4.y, wu4.z, wu4.w};
            float dg, du;
            if (kHalf) {
                dg = qdot_h2<kBits, 4>(wg, xhr) * hscale;
                du = qdot_h2<kBits, 4>(wu, xhr) * hscale;
            } else {
                dg = qdot_f32<kBits, 4>(wg, x2, xe, xo);
                du = qdot_f32<kBits, 4>(wu, x2, xe, xo);
            }
            g[n] = fmaf(bf16_to_f32(gs[grp]), dg, fmaf(bf16_to_f32(gs[512 + grp]), xa, g[n]));
            uu[n] = fmaf(bf16_to_f32(gs[1024 + grp]), du, fmaf(bf16_to_f32(gs[1536 + grp]), xa, uu[n]));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int n = 0; n < NU; ++n) {
            g[n] += __shfl_xor_sync(0xffffffffu, g[n], o);
            uu[n] += __shfl_xor_sync(0xffffffffu, uu[n], o);
        }
#pragma unroll
    for (int n = 0; n < NU; ++n) act[n] = siluf_(g[n]) * uu[n];
}

// Per-unit activation state for the down product: the half2 pair table of the unit's 16
// activations (8 entries), its scale 2^(24-E), and the sums of the even / odd activations.
struct UnitAct {
    __half2 tab[8];
    float ascale, ae, ao, pad;
};

// Warp 0, lanes 16n + r (r < 16) for unit n < NU: from the unit's activations uact[n][16],
// its pair table (entry k = r < 8: q4 (a[8j+i], a[8j+i+4]) * 2^(E-4(i&1)), k = 4j+i; q2
// (a[k], a[k+8]) * 2^(E-2(k&3)); E from max |a|) and its even / odd sums.
template <int kBits, int NU>
__device__ __forceinline__ void units_tables(const float *uact, UnitAct *ua, int lane) {
    const int n = lane >> 4, r = lane & 15;
    const float a = n < NU ? uact[n * 16 + r] : 0.f;
    float mx = fabsf(a), ev = (r & 1) ? 0.f : a, od = (r & 1) ? a : 0.f;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        ev += __shfl_xor_sync(0xffffffffu, ev, o);
        od += __shfl_xor_sync(0xffffffffu, od, o);
    }
    const int E = half_exp_bits(__float_as_uint(mx));
    const int k = r & 7;
    const int c0 = kBits == 4 ? 8 * (k >> 2) + (k & 3) : k, span = kBits == 4 ? 4 : 8;
    const float lo = __shfl_sync(0xffffffffu, a, (lane & 16) + c0);
    const float hi = __shfl_sync(0xffffffffu, a, (lane & 16) + c0 + span);
    const float sc = pow2i(E - (kBits == 4 ? 4 * (k & 1) : 2 * (k & 3)));
    if (n < NU) {
        if (r < 8) ua[n].tab[r] = __floats2half2_rn(lo * sc, hi * sc);
        if (r == 0) {
            ua[n].ascale = pow2i(24 - E);
            ua[n].ae = ev;
            ua[n].ao = od;
        }
    }
}

// Down partials of NU units: acc[i] += wgt[n] * (s_i * sum_v q[i][v] a[v] + b_i * sum_v a[v])
// for this thread's 4 output rows 4t..4t+3 and each unit's 16 activations a. q4: two word
// columns (8 activations each), q2: one (16 activations); wc[n] = the unit's word columns
// ([col][2048] u32), sb[n] = its group's scales [2048] then biases [2048]; ua[n] = the
// unit's pair table and sums. Units with live[n] false contribute nothing.
template <int kBits, bool kHalf, int NU>
__device__ __forceinline__ void down_units(const uint8_t *const *wc, const uint16_t *const *sb, const float *uact,
                                           const UnitAct *ua, const float *wgt, const bool *live, int t, float *acc) {
    constexpr int NW = kBits == 4 ? 2 : 1;
#pragma unroll
    for (int n = 0; n < NU; ++n) {
        uint32_t ws[4][NW];
        {
            const uint4 w0 = lds128(wc[n] + 16 * t);
            ws[0][0] = w0.x; ws[1][0] = w0.y; ws[2][0] = w0.z; ws[3][0] = w0.w;
            if (NW == 2) {
                const uint4 w1 = lds128(wc[n] + 2048 * 4 + 16 * t);
                ws[0][NW - 1] = w1.x; ws[1][NW - 1] = w1.y; ws[2][NW - 1] = w1.z; ws[3][NW - 1] = w1.w;
            }
        }
        const uint2 s4 = *reinterpret_cast<const uint2 *>(sb[n] + 4 * t);
        const uint2 b4 = *reinterpret_cast<const uint2 *>(sb[n] + 2048 + 4 * t);
        const float sc[4] = {bf16_lo(s4.x), bf16_hi(s4.x), bf16_lo(s4.y), bf16_hi(s4.y)};
        const float bi[4] = {bf16_lo(b4.x), bf16_hi(b4.x), bf16_lo(b4.y), bf16_hi(b4.y)};
        const float ae = ua[n].ae, ao = ua[n].ao;
        float d[4];
        if (kHalf) {
            __half2 ah[8];
            const uint4 t0 = *reinterpret_cast<const uint4 *>(&ua[n].tab[0]);
            const uint4 t1 = *reinterpret_cast<const uint4 *>(&ua[n].tab[4]);
            const uint32_t tw[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) ah[k] = *reinterpret_cast<const __half2 *>(&tw[k]);
            const float ascale = ua[n].ascale;
#pragma unroll
            for (int i = 0; i < 4; ++i) d[i] = qdot_h2<kBits, NW>(ws[i], ah) * ascale;
        } else {
            uint64_t x2[8];
#pragma unroll
            for (int v = 0; v < 16; v += 4) {
                const float4 f = lds128f(uact + 16 * n + v);
                x2[v / 2] = u64_of(__float_as_uint(f.x), __float_as_uint(f.y));
                x2[v / 2 + 1] = u64_of(__float_as_uint(f.z), __float_as_uint(f.w));
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) d[i] = qdot_f32<kBits, NW>(ws[i], x2, ae, ao);
        }
        const float asum = ae + ao;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float r = fmaf(wgt[n], fmaf(sc[i], d[i], bi[i] * asum), acc[i]);
            acc[i] = live[n] ? r : acc[i];
        }
    }
}

// The routing selection (one copy: run dry by warp 4, then for real by warp 0; warps 0
// and 4 share an SM sub-partition and its instruction cache).
__device__ __noinline__ float route_topk(float v0, float v1, float v2, float v3, float v4, float v5, float v6,
                                         float v7, int k, int lane, uint32_t *sidx, float *sval,
                                         uint32_t *tl) {
    const float v[8] = {v0, v1, v2, v3, v4, v5, v6, v7};
    return warp_topk_smem(v, k, lane, sidx, sval, tl);
}

#define NMOE_STAMP(slot)                                                    \
    do {                                                                    \
        if (kTL) P.sy->tl[c & 1023][(slot)] = (uint32_t)globaltimer_ns();   \
    } while (0)
#define NMOE_PHASE(v)                                         \
    do {                                                      \
        if (kTL && tid == 0) {                                \
            atomicMax(&P.sy->diag[c & 1023], (uint32_t)(v)); \
            NMOE_STAMP(v);                                    \
        }                                                     \
    } while (0)
#define NMOE_GIVEUP(v)                                        \
    do {                                                      \
        set_err(P.err, kErrTimeout);                          \
        S->abort = 1;                                         \
        atomicMax(&P.sy->diag[c & 1023], 100u + (v));         \
    } while (0)

// kTL: record the per-CTA phase timeline and trail (diagnostic build, NMOE_TIMELINE=1).
template <int kBits, bool kRQ4, bool kSQ4, bool kHalf, bool kTL>
__global__ void __launch_bounds__(kThreads, 1) k_moe_decode_fused(const FusedParams P) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const PackGeo pg = pack_geo(kBits);
    const FusedLayout &Y = P.lay;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int k = P.k;
    FusedSync *sy = P.sy;
    const uint64_t t_start = globaltimer_ns();
    const uint64_t deadline = t_start + P.timeout_ns;

    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + Y.bars);
    Ctl *S = reinterpret_cast<Ctl *>(sm + Y.ctl);
    float *xs = reinterpret_cast<float *>(sm + Y.xs);
    float *xsum = reinterpret_cast<float *>(sm + Y.xsum);

    constexpr uint32_t RW = kRQ4 ? 1152u : 4096u;           // router row bytes
    constexpr uint32_t SRW = kSQ4 ? 1152u : 4096u;          // shared gate/up row bytes
    constexpr uint32_t SPW = 2 * SRW;                       // shared pair bytes
    constexpr uint32_t SDC = kSQ4 ? 1024u : 4096u;          // shared down column bytes

    const int r0 = split_lo(kExperts, G, c), nR = split_lo(kExperts, G, c + 1) - r0;
    const int s0 = split_lo(kInter, G, c), nS = split_lo(kInter, G, c + 1) - s0;
    const int o0 = split_lo(kHidden, G, c), nO = split_lo(kHidden, G, c + 1) - o0;
    const int nU = P.route_only ? 0 : ((32 * k > c) ? (32 * k - c + G - 1) / G : 0);
    const bool do_shared = !P.route_only && nS > 0;
    // q4 shared down: the groups of 64 columns that rows [s0, s0+nS) fall in
    const int sg0 = s0 >> 6, nsg = nS > 0 ? ((s0 + nS - 1) >> 6) - sg0 + 1 : 0;
    uint32_t tl_a = 0, tl_b = 0, tl_c = 0;
    if (kTL) tl_a = (uint32_t)globaltimer_ns();
    // Programmatic dependent launch: the next call on this stream may start launching now;
    // its CTAs become resident as this call's CTAs exit.
    if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0) {
        for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
        S->abort = 0;
        S->rdone = 0;
        S->sdone = 0;
        S->xmax_bits = 0;
        S->armed = 0;
        for (int i = 0; i < kMaxK; ++i) S->sidx[i] = kUnset;
        for (int i = 0; i < kMaxUnits; ++i) S->amax_bits[i] = 0;
    }
    if (kTL && tid < kTlSlots) sy->tl[c & 1023][tid] = 0;   // this launch's stamps only
    __syncthreads();
    if (kTL) tl_b = (uint32_t)globaltimer_ns();

    // ---- 0. routing-independent copies ------------------------------------------------
    // Weights depend on nothing the previous call on this stream produces: the router rows
    // go out before the dependency wait, the shared-expert rows and columns right after
    // the x request. x, h_mid, out and the sync state are touched only after the wait.
    const uint64_t pol0 = policy_evict_first();
    auto issue_shared = [&]() {
        if (do_shared) {
            mbar_arrive_expect_tx(&bars[kBarShared], nS * SPW + SRW + nS * SDC + (kSQ4 ? 2u * nsg * 4096u : 0u));
            bulk_g2s(sm + Y.sp, P.spairs + (size_t)s0 * SPW, nS * SPW, &bars[kBarShared], pol0);
            bulk_g2s(sm + Y.gv, P.gvec, SRW, &bars[kBarShared], pol0);
            bulk_g2s(sm + Y.sdt, P.sdown_t + (size_t)s0 * SDC, nS * SDC, &bars[kBarShared], pol0);
            if (kSQ4) {   // scales then biases of the groups: [nsg][2048] each
                const uint8_t *sb = P.sdown_t + 512 * 1024;
                bulk_g2s(sm + Y.sdt + 4 * 1024, sb + (size_t)sg0 * 4096, nsg * 4096, &bars[kBarShared], pol0);
                bulk_g2s(sm + Y.sdt + 4 * 1024 + 2 * 4096, sb + 8 * 4096 + (size_t)sg0 * 4096, nsg * 4096,
                         &bars[kBarShared], pol0);
            }
        }
    };
    if (tid == 0) {
        mbar_arrive_expect_tx(&bars[kBarRouter], nR * RW);
        if (nR) bulk_g2s(sm + Y.rw, P.router + (size_t)r0 * RW, nR * RW, &bars[kBarRouter], pol0);
        S->armed = (1u << kBarRouter) | (do_shared ? 1u << kBarShared : 0u);
    }
    if (kTL) tl_c = (uint32_t)globaltimer_ns();
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (kTL && tid == 0) {
        NMOE_STAMP(16);
        sy->tl[c & 1023][29] = tl_a;
        sy->tl[c & 1023][30] = tl_b;
        sy->tl[c & 1023][31] = tl_c;
    }
    uint32_t tag;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(tag) : "l"(&sy->epoch) : "memory");
    tag += 1u;
    // x: each thread loads its 4 columns straight into registers (one L2 round trip)
    uint4 xr4 = make_uint4(0u, 0u, 0u, 0u);
    if (P.x_f32) {
        xr4 = __ldcg(reinterpret_cast<const uint4 *>(P.x) + tid);
    } else {
        const uint2 u = __ldcg(reinterpret_cast<const uint2 *>(P.x) + tid);
        xr4.x = u.x;
        xr4.y = u.y;
    }
    // the shared expert's 6 MB go out behind the x request, not ahead of it (x gates the
    // router dots; the shared rows are needed only after them)
    if (tid == 0) issue_shared();
    // this CTA's output rows start at h_mid (or 0); every CTA adds its partials once all
    // logits are published, i.e. after every CTA has written its rows
    if (kTL && tid == 0) sy->tl[c & 1023][0] = (uint32_t)t_start;

    // ---- 1. x: fp32 padded + per-32-column parity sums ---------------------------------
    {
        const int col0 = 4 * tid;   // 512 threads x 4 columns
        float v[4];
        if (P.x_f32) {
            v[0] = __uint_as_float(xr4.x); v[1] = __uint_as_float(xr4.y);
            v[2] = __uint_as_float(xr4.z); v[3] = __uint_as_float(xr4.w);
        } else {
            v[0] = bf16_lo(xr4.x); v[1] = bf16_hi(xr4.x); v[2] = bf16_lo(xr4.y); v[3] = bf16_hi(xr4.y);
        }
        *reinterpret_cast<float4 *>(xs + (col0 >> 5) * kXP + (col0 & 31)) = make_float4(v[0], v[1], v[2], v[3]);
        float e = v[0] + v[2], o = v[1] + v[3];
#pragma unroll
        for (int m = 1; m < 8; m <<= 1) {
            e += __shfl_xor_sync(0xffffffffu, e, m);
            o += __shfl_xor_sync(0xffffffffu, o, m);
        }
        if (kHalf) {
            float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o2));
            if (lane == 0) atomicMax(&S->xmax_bits, __float_as_uint(m));
        }
        if (kTL && tid == 0) NMOE_STAMP(21);
        if ((tid & 7) == 0) {
            const int cc = col0 >> 5;
            xsum[3 * cc] = e;
            xsum[3 * cc + 1] = o;
            xsum[3 * cc + 2] = e + o;
        }
    }
    __syncthreads();
    NMOE_PHASE(1);
    if (warp == kWarps - 1) {
        // warp 15 (no router rows) writes this CTA's output rows, then (fenced) counts them
        // as done; every CTA acquires the full count before its adds (warp 1, phase 4)
        if (!P.route_only && lane < nO) P.out[o0 + lane] = P.h_mid ? __ldcg(P.h_mid + o0 + lane) : 0.f;
        __syncwarp();
        if (lane == 0) {
            __threadfence();
            asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(&sy->inited) : "memory");
        }
    }

    // ---- 2. router / shared rows (FFMA), router first; last finisher completes --------
    // Units: (row, 1/8 of the columns). The last warp to finish a group's units sums the
    // 8 partials per row in a fixed order: router rows are published, shared rows
    // (SiLU(gate) * up) and the score stay in this CTA.
    constexpr int kSeg = 8;    // shared rows: 8 column segments
    constexpr int kRSeg = 4;   // router rows: 4 column segments (warps 0-7 at 2 rows a CTA)
    constexpr int kRChunks = kHidden / (kRQ4 ? 32 : 8), kSChunks = kHidden / (kSQ4 ? 32 : 8);
    float *rpart = reinterpret_cast<float *>(sm + Y.dsp);
    float *spart = rpart + Y.nRmax * kSeg, *gpart = spart + Y.nSmax * 2 * kSeg;
    float *sact = reinterpret_cast<float *>(sm + Y.sact);
    const int uR = nR * kRSeg, uS = do_shared ? nS * kSeg : 0, uG = do_shared ? kSeg : 0;
    bool r_ready = false, s_ready = false;
    auto do_unit = [&](int u) -> bool {
        if (u < uR) {
            if (!r_ready && !(r_ready = mbar_wait_warp(&bars[kBarRouter], 0, deadline))) return false;
            if (kTL && warp == 0 && lane == 0) NMOE_STAMP(18);
            const int row = u / kRSeg, seg = u % kRSeg, len = kRChunks / kRSeg;
            const float v = dense_seg<kRQ4, 1>(sm + Y.rw + row * RW, xs, xsum, seg * len, (seg + 1) * len, lane).x;
            if (kTL && warp == 0 && lane == 0) NMOE_STAMP(19);
            if (lane == 0) {
                rpart[u] = v;
                __threadfence_block();
                if (atomicAdd(&S->rdone, 1) == uR - 1) {
                    __threadfence_block();   // the other warps' partials, read below
                    if (kTL) NMOE_STAMP(20);
                    for (int r = 0; r < nR; ++r) {
                        float t = 0.f;
                        for (int q = 0; q < kRSeg; ++q) t += rpart[r * kRSeg + q];
#pragma unroll
                        for (int cp = 0; cp < kLogitCopies; ++cp) st_tagged(&sy->logits[cp][r0 + r], t, tag);
                    }
                    // a count of the publications, for the pollers (the tags above stay the
                    // authority: a poller that reads the count early re-reads the words)
                    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(&sy->arrive) : "memory");
                    NMOE_STAMP(8);
                }
            }
        } else {
            if (!s_ready && !(s_ready = mbar_wait_warp(&bars[kBarShared], 0, deadline))) return false;
            if (u < uR + uS) {
                const int pr = (u - uR) / kSeg, seg = (u - uR) % kSeg, len = kSChunks / kSeg;
                const float2 gu = dense_seg<kSQ4, 2>(sm + Y.sp + pr * SPW, xs, xsum, seg * len, (seg + 1) * len, lane);
                const float g = gu.x, uu = gu.y;
                if (lane == 0) {
                    spart[2 * (u - uR)] = g;
                    spart[2 * (u - uR) + 1] = uu;
                }
            } else {
                const int seg = u - uR - uS, len = kSChunks / kSeg;
                const float v = dense_seg<kSQ4, 1>(sm + Y.gv, xs, xsum, seg * len, (seg + 1) * len, lane).x;
                if (lane == 0) gpart[seg] = v;
            }
            if (lane == 0) {
                __threadfence_block();
                if (atomicAdd(&S->sdone, 1) == uS + uG - 1) {
                    __threadfence_block();
                    for (int r = 0; r < nS; ++r) {
                        float tg = 0.f, tu = 0.f;
                        for (int q = 0; q < kSeg; ++q) {
                            tg += spart[2 * (r * kSeg + q)];
                            tu += spart[2 * (r * kSeg + q) + 1];
                        }
                        sact[r] = siluf_(tg) * tu;
                    }
                    float t = 0.f;
                    for (int q = 0; q < kSeg; ++q) t += gpart[q];
                    S->score = t;
                }
            }
        }
        return true;
    };
    {
        // warp 0 takes router units only (it runs the top-k next); the shared units go to
        // warps 1..15 once their router units are done. One loop, so that the unit code is
        // emitted once: the kernel's serial path is sensitive to instruction-fetch misses.
        bool ok = !S->abort;
        const int uEnd = warp == 0 ? uR : uR + uS + uG;
        for (int u = warp < uR ? warp : (warp == 0 ? uEnd : uR + warp - 1); ok && u < uEnd;) {
            ok = do_unit(u);
            if (u < uR) {
                u += kWarps;
                if (u >= uR && warp != 0) {
                    u = uR + warp - 1;   // first shared unit of this warp
                    if (warp == 4) {
                        // Warm-up pass of the top-k (result discarded): the instruction
                        // caches start every launch cold; warp 4 shares warp 0's SM
                        // sub-partition, so warp 0's real pass finds the code cached.
                        const float *d = xs + 8 * lane;
                        const float l0 = route_topk(d[0], d[1], d[2], d[3], d[4], d[5], d[6], d[7], k, lane,
                                                    S->dsidx, S->dsval, nullptr);
                        if (lane == 0) S->sink[warp] = l0;
                    }
                }
            } else {
                u += kWarps - 1;
            }
        }
        if (!ok && lane == 0) NMOE_GIVEUP(2);
    }

    // x pair table of the half2 routed-unit path (off the critical path: routing in flight)
    if (kHalf && warp != 0 && nU > 0) {
        const int E = half_exp_bits(S->xmax_bits);
        __half2 *xh = reinterpret_cast<__half2 *>(sm + Y.xh);
        constexpr int kPairs = kBits == 4 ? 16 : 32, half_span = kBits == 4 ? 4 : 8, wcols = kBits == 4 ? 8 : 16;
#pragma unroll 1
        for (int e = tid - 32; e < 1024; e += kThreads - 32) {
            const int ch = e / kPairs, kk = e % kPairs;
            const int j = kk / half_span, i = kk % half_span;
            const int c0 = (kBits == 4 ? 32 : 64) * ch + wcols * j + i, c1 = c0 + half_span;
            const float sc = pow2i(E - (kBits == 4 ? 4 * (i & 1) : 2 * (i & 3)));
            const float v0 = xs[(c0 >> 5) * kXP + (c0 & 31)] * sc, v1 = xs[(c1 >> 5) * kXP + (c1 & 31)] * sc;
            xh[xtab_pos<kBits>(ch, kk)] = __floats2half2_rn(v0, v1);
        }
    }
    NMOE_PHASE(2);

    // ---- 3. routing: all 256 logits -> top-k (warp 0); routed copies (warp 1) ---------
    // One lane polls the publication count; the warp then reads the 256 tagged words once.
    if (warp == 0) {
        // lane holds experts 8*lane .. 8*lane+7
        float v[8];
        bool ok = !S->abort;
        const uint32_t want = P.stall ? tag + 1u : tag;
        if (kTL && lane == 0) NMOE_STAMP(13);
        if (ok && lane == 0) {
            const uint32_t target = want * (uint32_t)G;
            for (uint32_t it = 0; (int)(ld_relaxed_u32(&sy->arrive) - target) < 0; ++it)
                if (it >= kMaxSpins || globaltimer_ns() > deadline) break;
        }
        if (kTL && lane == 0) NMOE_STAMP(22);
        __syncwarp();
        // normally one read: every tag is already this launch's
        if (ok) ok = poll_tagged8(&sy->logits[c % kLogitCopies][8 * lane], want, v, deadline);
        ok = __all_sync(0xffffffffu, ok);
        if (kTL && lane == 0) NMOE_STAMP(15);
        if (!ok) {
            if (lane == 0 && !S->abort) NMOE_GIVEUP(3);
        } else {
            if (c == 0 && P.logits_out) {
                reinterpret_cast<float4 *>(P.logits_out)[2 * lane] = make_float4(v[0], v[1], v[2], v[3]);
                reinterpret_cast<float4 *>(P.logits_out)[2 * lane + 1] = make_float4(v[4], v[5], v[6], v[7]);
            }
            // each round's winner writes S->sidx[r]; warp 1 issues a unit's copies as soon
            // as its slot is decided
            if (kTL && lane == 0) NMOE_STAMP(23);
            const float l0 = route_topk(v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], k, lane, S->sidx, S->sval,
                                        kTL ? &sy->tl[c & 1023][24] : nullptr);
            if (kTL && lane == 0) NMOE_STAMP(6);
            const uint32_t e = lane < k ? S->sidx[lane & 7] : 0u;
            const int valid = lane < k && e < (uint32_t)P.num_experts;
            if (lane < kMaxK) {
                S->idx[lane] = e;
                S->valid[lane] = valid;
            }
            // renormalised weight of selection s (lane s): exp(l_s - l_0) / sum_t exp(l_t - l_0),
            // the sum taken in selection order
            const float ex = lane < k ? expf(S->sval[lane & 7] - l0) : 0.f;
            float sum = 0.f;
#pragma unroll 1
            for (int t = 0; t < k; ++t) sum += __shfl_sync(0xffffffffu, ex, t);
            if (lane < kMaxK) {
                const float w = lane < k ? ex / sum : 0.f;
                if (lane < k && !valid) set_err(P.err, kErrExpertRange);
                S->w[lane] = valid ? w : 0.f;
                if (c == 0) {
                    if (P.idx_out) P.idx_out[lane] = e;
                    if (P.w_out) P.w_out[lane] = w;
                }
            }
            if (kTL && lane == 0) NMOE_STAMP(9);
        }
    } else if (warp == 1 && nU > 0 && lane == 0) {
        uint32_t armed = 0;
        for (int i = 0; i < nU; ++i) {
            const int u = c + i * G, slot = u >> 5, band = u & 31;
            uint32_t e = kUnset;
            for (uint32_t it = 0; it < kMaxSpins; ++it) {
                e = *reinterpret_cast<volatile uint32_t *>(&S->sidx[slot]);
                if (e != kUnset || *reinterpret_cast<volatile int *>(&S->abort) || globaltimer_ns() > deadline) break;
            }
            if (e == kUnset) break;   // warp 0 gave up: nothing of this unit is issued
            const bool vs = e < (uint32_t)P.num_experts;
            uint8_t *dst = sm + Y.units + i * Y.unit_bytes;
            mbar_arrive_expect_tx(&bars[kBarGu0 + i], vs ? pg.bp : 0u);
            mbar_arrive_expect_tx(&bars[kBarD0 + i], vs ? pg.dunit + 8192u : 0u);
            armed |= (1u << (kBarGu0 + i)) | (1u << (kBarD0 + i));
            if (vs) {
                const uint8_t *ex = P.experts + (size_t)e * pg.esz;
                const uint8_t *slab = ex + pg.gu_bytes + (size_t)(band >> 2) * pg.dslab;
                bulk_g2s(dst, ex + (size_t)band * pg.bp, pg.bp, &bars[kBarGu0 + i], pol0);
                bulk_g2s(dst + pg.bp, slab + (size_t)(band & 3) * pg.dunit, pg.dunit, &bars[kBarD0 + i], pol0);
                bulk_g2s(dst + pg.bp + pg.dunit, slab + pg.dslab_w, 8192u, &bars[kBarD0 + i], pol0);
            }
            if (kTL && i == 0) NMOE_STAMP(17);
        }
        atomicOr(&S->armed, armed);
        if (kTL) NMOE_STAMP(10);
    }
    __syncthreads();
    NMOE_PHASE(3);

    if (!S->abort && !P.route_only) {
        // this thread's 4 output rows, across all of the CTA's partials
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int t = tid;
        if (warp == 1 && lane == 0) {
            // every CTA's output rows are initialised before this CTA's adds: acquire the count
            // (normally complete long before; read while the routed copies land)
            const uint32_t target = tag * (uint32_t)G;
            bool got = false;
            for (uint32_t it = 0; it < kMaxSpins; ++it) {
                if ((int)(ld_acquire_u32(&sy->inited) - target) >= 0) { got = true; break; }
                if (globaltimer_ns() > deadline) break;
            }
            if (!got) NMOE_GIVEUP(5);
        }

        // ---- 4. shared expert: sigmoid(score) * D_sh[:, s0:s0+nS] . sact ---------------
        // (its columns landed with the shared rows; runs while the routed copies fly)
        if (do_shared) {
            const float gsc = sigmoidf_(S->score);
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            const uint8_t *cols = sm + Y.sdt;
            if (!kSQ4) {
#pragma unroll 1
                for (int j = 0; j < nS; ++j) {
                    const float a = sact[j];
                    const uint2 wv = *reinterpret_cast<const uint2 *>(cols + j * 4096 + 8 * t);
                    d[0] = fmaf(bf16_lo(wv.x), a, d[0]);
                    d[1] = fmaf(bf16_hi(wv.x), a, d[1]);
                    d[2] = fmaf(bf16_lo(wv.y), a, d[2]);
                    d[3] = fmaf(bf16_hi(wv.y), a, d[3]);
                }
            } else {
                const uint16_t *ss = reinterpret_cast<const uint16_t *>(cols + 4 * 1024);
                const uint16_t *sb = ss + 2 * 2048;
#pragma unroll 1
                for (int j = 0; j < nS; ++j) {
                    const float a = sact[j];
                    const int g = ((s0 + j) >> 6) - sg0;
                    const uint32_t w = *reinterpret_cast<const uint32_t *>(cols + j * 1024 + 4 * (t >> 1)) >>
                                       (16 * (t & 1));
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float q = small_u2f((w >> (4 * i)) & 0xFu);
                        const float sv = bf16_to_f32(ss[g * 2048 + 4 * t + i]), bv = bf16_to_f32(sb[g * 2048 + 4 * t + i]);
                        d[i] = fmaf(fmaf(q, sv, bv), a, d[i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = gsc * d[i];
        }
        if (tid == 0) NMOE_STAMP(12);

        // ---- 5. routed units: gate/up -> act (16 rows) -> down partial ---------------
        // warp w computes row pair w of the unit's band; the warp's x chunks stay in
        // registers across the units.
        if (nU > 0) {
            float *uact = reinterpret_cast<float *>(sm + Y.uact);   // [nU][16]
            UnitAct *uas = reinterpret_cast<UnitAct *>(sm + Y.atab);
            const float hscale = pow2i(24 - half_exp_bits(S->xmax_bits));
            // units two at a time (both usually land together): one pass over x for both
            for (int i = 0; i < nU; i += 2) {
                const int nb = nU - i >= 2 ? 2 : 1;
                bool ok = true;
                for (int n = 0; n < nb; ++n) ok &= mbar_wait_warp(&bars[kBarGu0 + i + n], 0, deadline);
                if (!ok && lane == 0) NMOE_GIVEUP(4);
                if (i == 0 && tid == 0) NMOE_STAMP(11);
                const uint8_t *up[2];
                bool live[2];
                float wgt[2], act[2] = {0.f, 0.f};
                for (int n = 0; n < 2; ++n) {
                    const int ui = i + (n < nb ? n : 0), slot = (c + ui * G) >> 5;
                    up[n] = sm + Y.units + ui * Y.unit_bytes;
                    live[n] = ok && n < nb && S->valid[slot] && !S->abort;
                    wgt[n] = S->w[slot];
                }
                const __half2 *xth = reinterpret_cast<const __half2 *>(sm + Y.xh);
                if (ok) {
                    if (nb == 2) units_act<kBits, kHalf, 2>(up, xth, xs, xsum, hscale, warp, lane, act);
                    else units_act<kBits, kHalf, 1>(up, xth, xs, xsum, hscale, warp, lane, act);
                }
                if (lane == 0)
                    for (int n = 0; n < nb; ++n) uact[(i + n) * 16 + warp] = live[n] ? act[n] : 0.f;
                if (i == 0 && tid == 0) NMOE_STAMP(27);
                __syncthreads();
                if (i == 0 && tid == 0) NMOE_STAMP(28);
                if (warp == 0) {
                    if (nb == 2) units_tables<kBits, 2>(uact + i * 16, uas + i, lane);
                    else units_tables<kBits, 1>(uact + i * 16, uas + i, lane);
                }
                bool okd = true;
                for (int n = 0; n < nb; ++n) okd &= mbar_wait_warp(&bars[kBarD0 + i + n], 0, deadline);
                if (!okd && lane == 0) NMOE_GIVEUP(4);
                if (i == 0 && tid == 0) NMOE_STAMP(26);
                __syncthreads();
                if (i == 0 && tid == 0) NMOE_STAMP(14);
                const uint8_t *wc[2] = {up[0] + pg.bp, up[1] + pg.bp};
                const uint16_t *sb[2] = {reinterpret_cast<const uint16_t *>(up[0] + pg.bp + pg.dunit),
                                         reinterpret_cast<const uint16_t *>(up[1] + pg.bp + pg.dunit)};
                bool dl[2] = {live[0] && okd, live[1] && okd};
                if (nb == 2) down_units<kBits, kHalf, 2>(wc, sb, uact + i * 16, uas + i, wgt, dl, t, acc);
                else down_units<kBits, kHalf, 1>(wc, sb, uact + i * 16, uas + i, wgt, dl, t, acc);
            }
        }
        if (tid == 0) NMOE_STAMP(5);

        // ---- 6. one vector add of this thread's 4 output rows -------------------------
        __syncthreads();   // the output-row count acquired above (warp 1) precedes every add
        if (!S->abort && (do_shared || nU > 0)) red_add_v4(P.out + 4 * t, acc[0], acc[1], acc[2], acc[3]);
        // The next layer's routing-independent weights (router + shared expert) do not
        // depend on this call: start pulling them into L2 now, so that its head reads L2.
        if (tid == 0 && P.next_dense) {
            const uint32_t lo = (uint32_t)(((uint64_t)P.next_dense_bytes * c / G) & ~15ull);
            const uint32_t hi = (uint32_t)(((uint64_t)P.next_dense_bytes * (c + 1) / G) & ~15ull);
            if (hi > lo)
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(P.next_dense + lo), "r"(hi - lo) : "memory");
        }
    }

    // ---- 7. teardown -----------------------------------------------------------------
    __syncthreads();
    if (S->abort) {
        // let issued copies land (bounded) before this CTA's shared memory is released
        const uint64_t dl2 = globaltimer_ns() + 50000000ull;
        if (tid < kNumBars && (S->armed >> tid & 1u)) mbar_wait(&bars[tid], 0, dl2);
        __syncthreads();
    }
    NMOE_PHASE(7);
    if (tid == 0) {
        __threadfence();
        const uint32_t prev = atomicAdd(&sy->done_cnt, 1u);
        if (prev == (uint32_t)G - 1) {
            // every CTA's counts are in: re-base them (a launch that gave up may have
            // skipped some), so that the next launch waits for exactly G of each
            sy->arrive = tag * (uint32_t)G;
            sy->inited = tag * (uint32_t)G;
            sy->done_cnt = 0;
            sy->epoch = tag;   // next launch publishes with tag + 1
            __threadfence();
        }
    }
}

}  // namespace nmoe

using namespace nmoe;

struct nmoe::FusedState {
    FusedSync *sy = nullptr;
    int grid = 0;
    FusedLayout lay{};
    bool ok = false;
    uint64_t timeout_ns = 1000000000ull;
    int timeline = 0;
    int stall = 0;   // NMOE_TEST_STALL_WAIT=1 (tests): one cross-CTA wait can never complete
    int pdl = 1;   // launch with programmatic dependent launch (NMOE_PDL=0 turns it off)
    int expert_fp32 = 0;   // NMOE_EXPERT_FP32=1: fp32 routed-expert dots (slower, ~1e-6)
};

static FusedLayout make_layout(int bits, bool rq4, bool sq4, int G, int kmax) {
    FusedLayout Y{};
    const PackGeo pg = pack_geo(bits);
    auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
    Y.nRmax = cdiv(kExperts, G);
    Y.nSmax = cdiv(kInter, G);
    Y.nUmax = cdiv(32 * kmax, G);
    Y.kmax = kmax;
    const uint32_t RW = rq4 ? 1152 : 4096, SRW = sq4 ? 1152 : 4096, SDC = sq4 ? 1024 : 4096;
    uint32_t off = 0;
    auto take = [&](uint32_t bytes) {
        const uint32_t o = off;
        off += (bytes + 127) & ~127u;
        return o;
    };
    Y.bars = take(kNumBars * 8);
    Y.ctl = take(sizeof(Ctl));
    Y.xs = take(kHidden / 32 * kXP * 4);
    Y.xsum = take(kHidden / 32 * 3 * 4);
    Y.xh = take(1024 * 4);
    Y.rw = take(Y.nRmax * RW);
    Y.gv = take(SRW);
    Y.sp = take(Y.nSmax * 2 * SRW);
    // q4: the columns, then scales and biases of up to two groups ([2][2048] bf16 each)
    Y.sdt = take(sq4 ? 4 * 1024 + 4 * 4096 : Y.nSmax * SDC);
    Y.dsp = take((Y.nRmax * 8 + Y.nSmax * 16 + 8) * 4);
    Y.sact = take(Y.nSmax * 4);
    Y.uact = take(Y.nUmax * 16 * 4);
    Y.atab = take(Y.nUmax * (uint32_t)sizeof(UnitAct));
    // routed units last: [band pair | down word columns | group scales + biases 8 KB]
    Y.unit_bytes = (pg.bp + pg.dunit + 8192 + 127) & ~127u;
    Y.units = take(Y.nUmax * Y.unit_bytes);
    Y.total = off;
    return Y;
}

template <int kBits, bool kRQ4, bool kSQ4>
static cudaError_t set_attr(int smem) {
    cudaError_t e = cudaFuncSetAttribute(k_moe_decode_fused<kBits, kRQ4, kSQ4, true, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_decode_fused<kBits, kRQ4, kSQ4, false, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_moe_decode_fused<kBits, kRQ4, kSQ4, true, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    return e;
}

int nmoe_fused_init(nmoe_moe_ctx *ctx) {
    FusedState *F = new FusedState();
    ctx->fused = F;
    if (cudaMalloc(&F->sy, sizeof(FusedSync)) != cudaSuccess) return NMOE_ENOMEM;
    if (cudaMemset(F->sy, 0, sizeof(FusedSync)) != cudaSuccess) return NMOE_ECUDA;
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device);
    // every CTA holds at least one router row: its logits publication orders its output
    // rows' initialisation before the other CTAs' adds
    F->grid = std::min(ctx->num_sms, kExperts);
    if (const char *t = getenv("NMOE_WAIT_TIMEOUT_MS")) F->timeout_ns = (uint64_t)atoll(t) * 1000000ull;
    if (const char *t = getenv("NMOE_TIMELINE")) F->timeline = atoi(t) != 0;
    if (const char *t = getenv("NMOE_PDL")) F->pdl = atoi(t) != 0;
    if (const char *t = getenv("NMOE_TEST_STALL_WAIT")) F->stall = atoi(t) != 0;
    F->expert_fp32 = (ctx->cfg.flags & NMOE_FLAG_EXPERT_FP32) != 0;
    if (const char *t = getenv("NMOE_EXPERT_FP32")) F->expert_fp32 = atoi(t) != 0;
    const int bits = ctx->cfg.quant_bits;
    const bool rq4 = ctx->cfg.router_dtype == NMOE_DTYPE_Q4, sq4 = ctx->cfg.shared_dtype == NMOE_DTYPE_Q4;
    F->lay = make_layout(bits, rq4, sq4, F->grid, ctx->cfg.k_max);
    if ((int)F->lay.total > max_smem || F->lay.nUmax > kMaxUnits || (sq4 && F->lay.nSmax > 4)) {
        nmoe_ctx_set_error(ctx, "decode kernel needs %u B of shared memory and %d routed units per CTA on %d SMs "
                           "(device max %d B, %d units)", F->lay.total, F->lay.nUmax, F->grid, max_smem, kMaxUnits);
        return NMOE_ECUDA;
    }
    cudaError_t e = cudaErrorInvalidValue;
#define NMOE_SET(B, R, S) \
    if (bits == B && rq4 == R && sq4 == S) e = set_attr<B, R, S>(max_smem);
    NMOE_SET(4, false, false) NMOE_SET(4, true, false) NMOE_SET(4, false, true) NMOE_SET(4, true, true)
    NMOE_SET(2, false, false) NMOE_SET(2, true, false) NMOE_SET(2, false, true) NMOE_SET(2, true, true)
#undef NMOE_SET
    if (e != cudaSuccess) {
        nmoe_ctx_set_error(ctx, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        return NMOE_ECUDA;
    }
    F->ok = true;
    return NMOE_OK;
}

void nmoe_fused_destroy(nmoe_moe_ctx *ctx) {
    if (ctx->fused == nullptr) return;
    if (ctx->fused->sy) cudaFree(ctx->fused->sy);
    delete ctx->fused;
    ctx->fused = nullptr;
}

template <int kBits, bool kRQ4, bool kSQ4>
static cudaError_t launch(const FusedParams &p, int grid, cudaStream_t st, bool half, bool pdl, bool tl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.lay.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    if (!half) return cudaLaunchKernelEx(&cfg, k_moe_decode_fused<kBits, kRQ4, kSQ4, false, false>, p);
    if (tl) return cudaLaunchKernelEx(&cfg, k_moe_decode_fused<kBits, kRQ4, kSQ4, true, true>, p);
    return cudaLaunchKernelEx(&cfg, k_moe_decode_fused<kBits, kRQ4, kSQ4, true, false>, p);
}

cudaError_t nmoe_fused_launch(nmoe_moe_ctx *ctx, const FusedCall &a, cudaStream_t st) {
    FusedState *F = ctx->fused;
    FusedParams p;
    p.experts = a.experts;
    p.router = a.router;
    p.spairs = a.spairs;
    p.gvec = a.gvec;
    p.sdown_t = a.sdown_t;
    p.x = a.x;
    p.x_f32 = a.x_f32;
    p.h_mid = a.h_mid;
    p.out = a.out;
    p.idx_out = a.idx_out;
    p.w_out = a.w_out;
    p.logits_out = a.logits_out;
    p.k = a.k;
    p.num_experts = a.num_experts;
    p.route_only = a.route_only;
    p.next_dense = a.next_dense;
    p.next_dense_bytes = a.next_dense_bytes;
    p.stall = F->stall;
    p.sy = F->sy;
    p.err = a.err;
    p.lay = F->lay;
    p.timeout_ns = F->timeout_ns;
    const int bits = ctx->cfg.quant_bits;
    const bool rq4 = ctx->cfg.router_dtype == NMOE_DTYPE_Q4, sq4 = ctx->cfg.shared_dtype == NMOE_DTYPE_Q4;
    const bool tl = F->timeline != 0;
#define NMOE_L(B, R, S) \
    if (bits == B && rq4 == R && sq4 == S) return launch<B, R, S>(p, F->grid, st, !F->expert_fp32, F->pdl, tl);
    NMOE_L(4, false, false) NMOE_L(4, true, false) NMOE_L(4, false, true) NMOE_L(4, true, true)
    NMOE_L(2, false, false) NMOE_L(2, true, false) NMOE_L(2, false, true) NMOE_L(2, true, true)
#undef NMOE_L
    return cudaErrorInvalidValue;
}

extern "C" int nmoe_moe_debug_trail(nmoe_moe_ctx *ctx, uint32_t *out, int n) {
    if (ctx == nullptr || ctx->fused == nullptr || ctx->fused->sy == nullptr || out == nullptr || n < 0) return NMOE_EINVAL;
    n = n > 1024 ? 1024 : n;
    cudaSetDevice(ctx->device);
    if (cudaDeviceSynchronize() != cudaSuccess) return NMOE_ECUDA;
    if (cudaMemcpy(out, ctx->fused->sy->diag, n * sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess) return NMOE_ECUDA;
    if (cudaMemset(ctx->fused->sy->diag, 0, sizeof(ctx->fused->sy->diag)) != cudaSuccess) return NMOE_ECUDA;
    return NMOE_OK;
}

extern "C" int nmoe_moe_debug_timeline(nmoe_moe_ctx *ctx, uint32_t *out, int n_ctas) {
    if (ctx == nullptr || ctx->fused == nullptr || out == nullptr || n_ctas < 0) return NMOE_EINVAL;
    n_ctas = n_ctas > 1024 ? 1024 : n_ctas;
    cudaSetDevice(ctx->device);
    if (cudaDeviceSynchronize() != cudaSuccess) return NMOE_ECUDA;
    if (cudaMemcpy(out, ctx->fused->sy->tl, (size_t)n_ctas * kTlSlots * sizeof(uint32_t), cudaMemcpyDeviceToHost) !=
        cudaSuccess)
        return NMOE_ECUDA;
    return NMOE_OK;
}

extern "C" int nmoe_moe_decode_grid(const nmoe_moe_ctx *ctx) {
    return (ctx == nullptr || ctx->fused == nullptr) ? 0 : ctx->fused->grid;
}
