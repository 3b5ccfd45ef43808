// nmoe_fused.cu -- batch-1 routed-MoE block in ONE persistent launch (sm_100a).
//
// Grid = one 512-thread CTA per SM, launched cooperatively so that every CTA is
// resident and the bounded cross-CTA waits cannot deadlock. Work per CTA c of G:
//   router rows      [c*256/G, (c+1)*256/G)          -> logits
//   shared pairs     [c*512/G, (c+1)*512/G)          -> shared act
//   gate vector      CTA G-1                         -> score
//   routed gate/up   units u = c, c+G, ... < 32k     (unit = slot u/32, 16-row band u%32)
//                                                    -> act
//   output bands     b with (G-1-b) mod G == c       (16 output rows: k expert down
//                                                    bands + shared down + combine)
// Weight bytes move by cp.async.bulk straight into shared memory, each slice in one
// copy thanks to the repacked HBM layout (nmoe_pack.cuh): the routing-independent ones
// at kernel start, the routed ones as soon as this CTA knows the top-k. Routed gate/up
// and down dots use the packed values in place as exact subnormal halves against a
// per-call scaled half2 table of x (or act), flushed to fp32 once per word; the affine
// dequantisation is applied per 64-column group as  s * sum(q*x) + b * sum(x).
// Router and shared-expert rows (bf16 or q4) use an fp32 FFMA path.
// Cross-CTA results (logits, shared act, score, act) are published as 64-bit words
// {launch tag, value}; a consumer polls the words it needs until all carry this launch's
// tag -- one L2 round trip after the last producer, no separate counter. The tag is
// epoch + 1, and the last CTA to finish advances the epoch for the next launch.
// Every wait is bounded (timer and iteration cap) and reports NMOE_ETIMEOUT through the
// device error word.
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
constexpr int kMaxBars = 16;
constexpr int kBarX = 0, kBarRouter = 1, kBarShared = 2, kBarSDown = 3, kBarUnit0 = 4, kBarBand0 = 10;
constexpr int kMaxUnits = 6, kMaxBands = 6;

struct FusedSync {
    uint32_t epoch, done_cnt;
    uint32_t pad[30];
    uint64_t logits[kExperts];       // tagged {tag, value}
    uint64_t shared_act[kInter];
    uint64_t score;
    uint64_t pad2[15];
    float act[kMaxK * kInter];       // plain; readiness is per unit in uflag
    uint32_t uflag[32 * kMaxK];      // tag of the launch whose unit u act rows are written
    uint32_t diag[1024];        // per CTA: highest phase reached; 100+phase where a wait gave up
    uint32_t tl[1024][16];      // per CTA phase timestamps (globaltimer low 32 bits)
};

struct FusedLayout {
    uint32_t bars, ctl, xs, xsum, rw, sp, gv, sdn, units, bands, part, dsp, sred, total;
    // aliases inside `units` (dead once the routed gate/up is done)
    uint32_t sact, ssum, actf, ag, acth;
    uint32_t xh;
    int nUmax, nBmax, nR, nS, kmax;
};

struct FusedParams {
    const uint8_t *experts;   // repacked expert blobs of this layer
    const uint8_t *router, *spairs, *gvec, *sdown;   // repacked dense regions
    const uint8_t *next_dense;   // dense arena to prefetch into L2 during the tail, or null
    uint32_t next_dense_bytes;
    const void *x;
    int x_f32;
    const float *h_mid;
    float *out;
    uint32_t *idx_out;
    float *w_out;
    float *logits_out;
    int k, num_experts, route_only, timeline;
    int stall;   // test hook: the logits poll waits for a tag that is never written
    FusedSync *sy;
    int *err;
    FusedLayout lay;
    uint64_t timeout_ns;
};

struct Ctl {
    uint32_t xmax_bits;           // max |x| (float bits; non-negative floats order as ints)
    uint32_t amax_bits[kMaxK];    // max |act| per slot
    int abort;
    int rdone, sdone;
    uint32_t idx[kMaxK];
    float w[kMaxK];
    int valid[kMaxK];
    float score;

};

__device__ __forceinline__ void st_tagged(uint64_t *p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// Poll 4 consecutive tagged words (32-byte aligned) until all carry `tag`.
__device__ __forceinline__ bool poll_tagged4(const uint64_t *p, uint32_t tag, float *v, uint64_t deadline) {
    for (uint32_t it = 0;; ++it) {
        uint64_t a0, a1, b0, b1;
        asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(a0), "=l"(a1) : "l"(p) : "memory");
        asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(b0), "=l"(b1) : "l"(p + 2) : "memory");
        if ((uint32_t)(a0 >> 32) == tag && (uint32_t)(a1 >> 32) == tag && (uint32_t)(b0 >> 32) == tag &&
            (uint32_t)(b1 >> 32) == tag) {
            v[0] = __uint_as_float((uint32_t)a0);
            v[1] = __uint_as_float((uint32_t)a1);
            v[2] = __uint_as_float((uint32_t)b0);
            v[3] = __uint_as_float((uint32_t)b1);
            return true;
        }
        if (it >= kMaxSpins || globaltimer_ns() > deadline) return false;
        __nanosleep(64);
    }
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
        __nanosleep(64);
    }
}
__device__ __forceinline__ bool poll_tagged1(const uint64_t *p, uint32_t tag, float *v, uint64_t deadline) {
    for (uint32_t it = 0;; ++it) {
        uint64_t a;
        asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
        if ((uint32_t)(a >> 32) == tag) {
            *v = __uint_as_float((uint32_t)a);
            return true;
        }
        if (it >= kMaxSpins || globaltimer_ns() > deadline) return false;
        __nanosleep(64);
    }
}

__device__ __forceinline__ int split_lo(int total, int parts, int i) { return (int)((long long)total * i / parts); }
__device__ __forceinline__ void set_err(int *err, int code) { atomicCAS(err, 0, code); }

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

// ------------------------------------------------------- routed experts: f32x2 ----
// Blackwell's packed fp32 FMA (fma.rn.f32x2) over the same conversion-free dequant:
// one shift of a packed word puts an even-column value in mantissa bits [15,18]
// (q4: reads 1 + q/256) and the next odd-column value in [19,22] (1 + q/16); two LOP3s
// make the fp32 pair, one FFMA2 accumulates both against (x_even, x_odd). q2 words use
// bits [19,20] (1 + q/16) and [21,22] (1 + q/4). 2 instructions per weight, fp32 math.
__device__ __forceinline__ uint64_t u64_of(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }
__device__ __forceinline__ void ffma2(uint64_t &acc, uint64_t a, uint64_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

// sum(q*x) over one 16-byte chunk (q4: 32 columns, q2: 64); x2[i] = (x[2i], x[2i+1]).
template <int kBits>
__device__ __forceinline__ float qdot_chunk(const uint4 w, const uint64_t *x2, float xe, float xo) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint64_t acc = 0ull;
    if (kBits == 4) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t sh[4] = {ws[j] << 15, ws[j] << 7, ws[j] >> 1, ws[j] >> 9};
#pragma unroll
            for (int p = 0; p < 4; ++p)
                ffma2(acc, u64_of((sh[p] & 0x00078000u) | 0x3F800000u, (sh[p] & 0x00780000u) | 0x3F800000u),
                      x2[4 * j + p]);
        }
        return 256.f * (lo_f(acc) - xe) + 16.f * (hi_f(acc) - xo);
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int p = 0; p < 8; ++p) {
                const int sft = 19 - 4 * p;
                const uint32_t v = sft >= 0 ? (ws[j] << sft) : (ws[j] >> (-sft));
                ffma2(acc, u64_of((v & 0x00180000u) | 0x3F800000u, (v & 0x00600000u) | 0x3F800000u), x2[8 * j + p]);
            }
        }
        return 16.f * (lo_f(acc) - xe) + 4.f * (hi_f(acc) - xo);
    }
}

// Lane's x (or act) chunk: 32 (q4) or 64 (q2) columns from the padded fp32 layout as
// fp32 pairs, plus the chunk's even/odd column sums.
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
// single w >> 8 brings the other positions down. Multiplied by x * 2^(E - 4p) (the pair
// table below) every product is q * x * 2^(E-24), accumulated 4 (q4) / 8 (q2) deep in
// half2 and flushed to fp32 once per word: 0.6 integer and ~1 FP16 instruction per
// weight, about twice the rate of the fp32 path, ~3e-4 relative error per dot.
template <int kBits>
__device__ __forceinline__ float qdot_h2(const uint4 w, const __half2 *xh) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        __half2 h = __float2half2_rn(0.f);
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
        const float2 f = __half22float2(h);
        acc += f.x + f.y;
    }
    return acc;
}

// Scale exponent of a vector with max |v| = vmax: vmax * 2^E <= 2^15 (half range).
__device__ __forceinline__ int half_exp(float vmax) {
    if (!(vmax > 0.f) || !isfinite(vmax)) return 0;
    return 15 - (int)ceilf(log2f(vmax));
}

// Pair-table entry e of a padded fp32 vector (16 (q4) / 32 (q2) entries per chunk):
// q4: entry 4j+i of chunk c = (v[32c+8j+i], v[32c+8j+i+4]) * 2^(E-4(i&1))
// q2: entry 8j+i of chunk c = (v[64c+16j+i], v[64c+16j+i+8]) * 2^(E-2(i&3))
template <int kBits>
__device__ __forceinline__ __half2 pair_entry(const float *vpad, int e, int E) {
    constexpr int per = kBits == 4 ? 16 : 32, half_span = kBits == 4 ? 4 : 8, wcols = kBits == 4 ? 8 : 16;
    const int cch = e / per, k = e % per;
    const int j = k / half_span, i = k % half_span;
    const int c0 = (kBits == 4 ? 32 : 64) * cch + wcols * j + i, c1 = c0 + half_span;
    const float sc = exp2f((float)(E - (kBits == 4 ? 4 * (i & 1) : 2 * (i & 3))));
    return __floats2half2_rn(vpad[(c0 >> 5) * kXP + (c0 & 31)] * sc, vpad[(c1 >> 5) * kXP + (c1 & 31)] * sc);
}

#define NMOE_STAMP(slot)                                                             \
    do {                                                                             \
        if (P.timeline) P.sy->tl[c & 1023][(slot)] = (uint32_t)globaltimer_ns();    \
    } while (0)
#define NMOE_PHASE(v)                                         \
    do {                                                      \
        if (tid == 0) {                                       \
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

template <int kBits, bool kRQ4, bool kSQ4, bool kHalf>
__global__ void __launch_bounds__(kThreads, 1) k_moe_decode_fused(const FusedParams P) {
    extern __shared__ __align__(1024) uint8_t sm[];
    constexpr int vpw = 32 / kBits;
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
    constexpr uint32_t SDW = kSQ4 ? 288u : 1024u;           // shared down row bytes

    const int r0 = split_lo(kExperts, G, c), nR = split_lo(kExperts, G, c + 1) - r0;
    const int s0 = split_lo(kInter, G, c), nS = split_lo(kInter, G, c + 1) - s0;
    const bool has_gvec = (c == G - 1);
    const int nU = (32 * k > c) ? (32 * k - c + G - 1) / G : 0;
    const int nB = (128 > (G - 1 - c)) ? (128 - (G - 1 - c) + G - 1) / G : 0;   // bands b = G-1-c + i*G
    const int band0 = G - 1 - c;
    // Programmatic dependent launch: the next call on this stream may start launching now;
    // its CTAs become resident as this call's CTAs exit.
    if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0) {
        for (int i = 0; i < kMaxBars; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
        S->abort = 0;
        S->rdone = 0;
        S->sdone = 0;
        S->xmax_bits = 0;
        for (int i = 0; i < kMaxK; ++i) S->amax_bits[i] = 0;
    }
    __syncthreads();

    // ---- 0. routing-independent copies ------------------------------------------------
    // The router rows depend on nothing the previous call on this stream produces: they
    // go out before the dependency wait. x, h_mid and the shared sync state (the epoch
    // word and the exchange buffers) are read only after it.
    if (tid == 0) {
        const uint64_t pol = policy_evict_first();
        mbar_arrive_expect_tx(&bars[kBarRouter], nR * RW);
        if (nR) bulk_g2s(sm + Y.rw, P.router + (size_t)r0 * RW, nR * RW, &bars[kBarRouter], pol);
        mbar_arrive_expect_tx(&bars[kBarShared], nS * SPW + (has_gvec ? SRW : 0));
        mbar_arrive_expect_tx(&bars[kBarSDown], P.route_only ? 0u : nB * 16 * SDW);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
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
    // residual rows this thread combines at the end: load early, latency hidden
    float hm_reg = 0.f;
    if (!P.route_only && P.h_mid && tid < nB * 16)   // volatile: keep the load here, not at its use
        asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(hm_reg) : "l"(P.h_mid + (band0 + (tid >> 4) * G) * 16 + (tid & 15)));
    if (tid == 0) {
        if (P.timeline) sy->tl[c & 1023][0] = (uint32_t)t_start;
        mbar_arrive_expect_tx(&bars[kBarX], 0u);   // unused: x is loaded by the threads
    }
    // The shared-expert copies go out only once the router rows have landed (see phase
    // 2), so that the router bytes do not queue behind them in this SM's copy engine.
    auto issue_shared = [&]() {
        const uint64_t pol = policy_evict_first();
        if (nS) bulk_g2s(sm + Y.sp, P.spairs + (size_t)s0 * SPW, nS * SPW, &bars[kBarShared], pol);
        if (has_gvec) bulk_g2s(sm + Y.gv, P.gvec, SRW, &bars[kBarShared], pol);
        if (!P.route_only)
            for (int i = 0; i < nB; ++i)
                bulk_g2s(sm + Y.sdn + i * 16 * SDW, P.sdown + (size_t)(band0 + i * G) * 16 * SDW, 16 * SDW,
                         &bars[kBarSDown], pol);
    };
    if (tid == 0 && nR == 0) issue_shared();
    // The routed down bands are only needed after the act exchange: they go out once this
    // CTA's first gate/up unit has landed, so that the gate/up bytes are not interleaved
    // with them in HBM.
    auto issue_bands = [&]() {
        const uint64_t pol = policy_evict_first();
        for (int i = 0; i < nB; ++i) {
            const int band = band0 + i * G;
            for (int s = 0; s < k; ++s)
                if (S->valid[s])
                    bulk_g2s(sm + Y.bands + (i * Y.kmax + s) * pg.db,
                             P.experts + (size_t)S->idx[s] * pg.esz + pg.gu_bytes + (size_t)band * pg.db, pg.db,
                             &bars[kBarBand0 + i], pol);
        }
    };

    // ---- 1. x: fp32 padded + per-32-column parity sums + per-64-column group sums -----
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
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) atomicMax(&S->xmax_bits, __float_as_uint(m));
        }
        if ((tid & 7) == 0) {
            const int cc = col0 >> 5;
            xsum[3 * cc] = e;
            xsum[3 * cc + 1] = o;
            xsum[3 * cc + 2] = e + o;
        }
    }
    __syncthreads();
    NMOE_PHASE(1);

    // ---- 2. router / shared rows (FFMA), router first; last finisher publishes --------
    // Units: (row, 1/8 of the columns). The last warp to finish a group's units sums the
    // 8 partials per row in a fixed order and publishes them.
    constexpr int kSeg = 8;
    constexpr int kRChunks = kHidden / (kRQ4 ? 32 : 8), kSChunks = kHidden / (kSQ4 ? 32 : 8);
    float *rpart = reinterpret_cast<float *>(sm + Y.dsp);
    float *spart = rpart + nR * kSeg, *gpart = spart + nS * 2 * kSeg;
    const int uR = nR * kSeg, uS = nS * kSeg, uG = has_gvec ? kSeg : 0;
    bool r_ready = false, s_ready = false;
    auto do_unit = [&](int u) -> bool {
            if (u < uR) {
                if (!r_ready) {
                    if (!(r_ready = mbar_wait_warp(&bars[kBarRouter], 0, deadline))) return false;
                    if (u == 0 && lane == 0) issue_shared();
                }
                const int row = u / kSeg, seg = u % kSeg, len = kRChunks / kSeg;
                const uint8_t *base = sm + Y.rw + row * RW;
                const uint8_t *w[1] = {base};
                const uint16_t *sp[1] = {reinterpret_cast<const uint16_t *>(base + 1024)};
                const uint16_t *bp[1] = {reinterpret_cast<const uint16_t *>(base + 1088)};
                float acc[1] = {0.f};
                dense_dot<kRQ4, 1>(w, sp, bp, xs, xsum, seg * len + lane, 32, (seg + 1) * len, acc);
                const float v = warp_sum(acc[0]);
                if (lane == 0) {
                    rpart[u] = v;
                    __threadfence_block();
                    if (atomicAdd(&S->rdone, 1) == uR - 1) {
                        __threadfence_block();
                        for (int r = 0; r < nR; ++r) {
                            float t = 0.f;
                            for (int q = 0; q < kSeg; ++q) t += rpart[r * kSeg + q];
                            st_tagged(&sy->logits[r0 + r], t, tag);
                        }
                        NMOE_STAMP(8);
                    }
                }
            } else {
                if (!s_ready && !(s_ready = mbar_wait_warp(&bars[kBarShared], 0, deadline))) return false;
                if (u < uR + uS) {
                    const int pr = (u - uR) / kSeg, seg = (u - uR) % kSeg, len = kSChunks / kSeg;
                    const uint8_t *base = sm + Y.sp + pr * SPW;
                    const uint8_t *w[2] = {base, base + (kSQ4 ? 1024 : 4096)};
                    const uint16_t *sp[2] = {reinterpret_cast<const uint16_t *>(base + 2048),
                                             reinterpret_cast<const uint16_t *>(base + 2176)};
                    const uint16_t *bp[2] = {reinterpret_cast<const uint16_t *>(base + 2112),
                                             reinterpret_cast<const uint16_t *>(base + 2240)};
                    float acc[2] = {0.f, 0.f};
                    dense_dot<kSQ4, 2>(w, sp, bp, xs, xsum, seg * len + lane, 32, (seg + 1) * len, acc);
                    const float g = warp_sum(acc[0]), uu = warp_sum(acc[1]);
                    if (lane == 0) {
                        spart[2 * (u - uR)] = g;
                        spart[2 * (u - uR) + 1] = uu;
                    }
                } else {
                    const int seg = u - uR - uS, len = kSChunks / kSeg;
                    const uint8_t *base = sm + Y.gv;
                    const uint8_t *w[1] = {base};
                    const uint16_t *sp[1] = {reinterpret_cast<const uint16_t *>(base + 1024)};
                    const uint16_t *bp[1] = {reinterpret_cast<const uint16_t *>(base + 1088)};
                    float acc[1] = {0.f};
                    dense_dot<kSQ4, 1>(w, sp, bp, xs, xsum, seg * len + lane, 32, (seg + 1) * len, acc);
                    const float v = warp_sum(acc[0]);
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
                            st_tagged(&sy->shared_act[s0 + r], siluf_(tg) * tu, tag);
                        }
                        if (has_gvec) {
                            float t = 0.f;
                            for (int q = 0; q < kSeg; ++q) t += gpart[q];
                            st_tagged(&sy->score, t, tag);
                        }
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
                if (u >= uR && warp != 0) u = uR + warp - 1;   // first shared unit of this warp
            } else {
                u += kWarps - 1;
            }
        }
        if (!ok && lane == 0) NMOE_GIVEUP(2);
    }

    // x pair table for the half2 expert path (off the critical path: routing in flight)
    if (kHalf && warp != 0) {
        const int E = half_exp(__uint_as_float(S->xmax_bits));
        __half2 *xh = reinterpret_cast<__half2 *>(sm + Y.xh);
#pragma unroll 1
        for (int e = tid - 32; e < 1024; e += kThreads - 32) xh[e] = pair_entry<kBits>(xs, e, E);
    }
    NMOE_PHASE(2);

    // ---- 3. routing: all 256 logits -> top-k (warp 0) -> routed copies -----------------
    if (warp == 0) {
        // lane holds experts 8*lane .. 8*lane+7
        float v[8];
        bool ok = !S->abort;
        const uint32_t want = P.stall ? tag + 1u : tag;
        if (ok) ok = poll_tagged8(&sy->logits[8 * lane], want, v, deadline);
        ok = __all_sync(0xffffffffu, ok);
        if (lane == 0) NMOE_STAMP(15);
        if (!ok) {
            if (lane == 0 && !S->abort) NMOE_GIVEUP(3);
        } else {
            if (c == 0 && P.logits_out) {
                reinterpret_cast<float4 *>(P.logits_out)[2 * lane] = make_float4(v[0], v[1], v[2], v[3]);
                reinterpret_cast<float4 *>(P.logits_out)[2 * lane + 1] = make_float4(v[4], v[5], v[6], v[7]);
            }
            const TopkLane tk = warp_topk_lane(v, k, lane);
            const uint32_t e = lane < k ? tk.idx : 0u;
            const int valid = lane < k && e < (uint32_t)P.num_experts;
            if (lane < kMaxK) {
                S->idx[lane] = e;
                S->valid[lane] = valid;
            }
            __syncwarp();
            // routed copies first (gate/up units, then the band expectations); the weights
            // are only needed at the combine
            if (lane == 0 && !P.route_only) {
                const uint64_t pol = policy_evict_first();
                for (int i = 0; i < nU; ++i) {
                    const int u = c + i * G, slot = u >> 5, band = u & 31;
                    const bool vs = S->valid[slot];
                    mbar_arrive_expect_tx(&bars[kBarUnit0 + i], vs ? pg.bp : 0u);
                    if (vs)
                        bulk_g2s(sm + Y.units + i * pg.bp, P.experts + (size_t)S->idx[slot] * pg.esz + (size_t)band * pg.bp,
                                 pg.bp, &bars[kBarUnit0 + i], pol);
                }
                for (int i = 0; i < nB; ++i) {
                    uint32_t bytes = 0;
                    for (int s = 0; s < k; ++s) bytes += S->valid[s] ? pg.db : 0u;
                    mbar_arrive_expect_tx(&bars[kBarBand0 + i], bytes);
                }
                if (nU == 0) issue_bands();
                NMOE_STAMP(10);
            }
            // renormalised weight of selection s (lane s): exp(l_s - l_0) / sum_t exp(l_t - l_0),
            // the sum taken in selection order
            const float ex = lane < k ? expf(tk.val - tk.l0) : 0.f;
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
            if (lane == 0) NMOE_STAMP(9);
        }
    }
    __syncthreads();
    NMOE_PHASE(3);

    if (!S->abort && !P.route_only) {
        // ---- 4. routed gate/up: warp w computes row pair w of each of this CTA's units ----
        // The warp's x chunks stay in registers across its rows; each row is finished by
        // one warp, so no cross-warp reduction.
        {
            constexpr int kChunksPerLane = kBits == 4 ? 2 : 1;   // 64 (q4) / 32 (q2) chunks per row
            constexpr int kPairs = kBits == 4 ? 16 : 32;         // pair-table entries per chunk
            uint64_t x2[kHalf ? 1 : kChunksPerLane][kHalf ? 1 : 16 * (kBits == 4 ? 1 : 2)];
            __half2 xhr[kHalf ? kChunksPerLane : 1][kHalf ? kPairs : 1];
            float xe[kChunksPerLane], xo[kChunksPerLane];
            const float hscale = exp2f((float)(24 - half_exp(__uint_as_float(S->xmax_bits))));
#pragma unroll
            for (int q = 0; q < kChunksPerLane; ++q) {
                const int ch = lane + 32 * q;
                if (kHalf) {
                    const __half2 *src = reinterpret_cast<const __half2 *>(sm + Y.xh) + ch * kPairs;
#pragma unroll
                    for (int e = 0; e < kPairs; ++e) xhr[q][e] = src[e];
                    const int n32 = kBits == 4 ? 1 : 2;
                    xe[q] = xsum[3 * n32 * ch] + (n32 == 2 ? xsum[3 * (2 * ch + 1)] : 0.f);
                    xo[q] = xsum[3 * n32 * ch + 1] + (n32 == 2 ? xsum[3 * (2 * ch + 1) + 1] : 0.f);
                } else {
                    load_chunk_x2<kBits>(xs, xsum, ch, x2[q], xe[q], xo[q]);
                }
            }
            auto qd = [&](const uint8_t *row, int q) -> float {
                const uint4 wv = lds128(row + 16 * (lane + 32 * q));
                if (kHalf) return qdot_h2<kBits>(wv, xhr[q]) * hscale;
                return qdot_chunk<kBits>(wv, x2[kHalf ? 0 : q], xe[q], xo[q]);
            };
            for (int i = 0; i < nU; ++i) {
                const int u = c + i * G, slot = u >> 5, band = u & 31;
                if (!mbar_wait_warp(&bars[kBarUnit0 + i], 0, deadline)) {
                    if (lane == 0) NMOE_GIVEUP(4);
                    break;
                }
                if (i == 0 && tid == 0) {
                    NMOE_STAMP(11);
                    issue_bands();
                }
                float g = 0.f, uu = 0.f;
                if (S->valid[slot]) {
                    const uint8_t *up0 = sm + Y.units + i * pg.bp;
                    const uint8_t *gw = up0 + warp * pg.wgu * 4, *uw = gw + pg.tile_band_gu;
                    const uint16_t *gs = reinterpret_cast<const uint16_t *>(up0 + 2 * pg.tile_band_gu) + warp * 32;
                    const uint16_t *gb = gs + 512, *us = gs + 1024, *ub = gs + 1536;
#pragma unroll
                    for (int q = 0; q < kChunksPerLane; ++q) {
                        const int ch = lane + 32 * q, grp = kBits == 4 ? ch >> 1 : ch;
                        const float xa = xe[q] + xo[q];
                        g = fmaf(bf16_to_f32(gs[grp]), qd(gw, q), fmaf(bf16_to_f32(gb[grp]), xa, g));
                        uu = fmaf(bf16_to_f32(us[grp]), qd(uw, q), fmaf(bf16_to_f32(ub[grp]), xa, uu));
                    }
                }
                g = warp_sum(g);
                uu = warp_sum(uu);
                if (lane == 0) sy->act[slot * kInter + band * 16 + warp] = S->valid[slot] ? siluf_(g) * uu : 0.f;
            }
        }
        __syncthreads();
        // The next layer's routing-independent weights (router + shared expert) do not
        // depend on this call: start pulling them into L2 now, so that its head reads L2.
        if (tid == 0 && P.next_dense) {
            const uint32_t lo = (uint32_t)(((uint64_t)P.next_dense_bytes * c / G) & ~15ull);
            const uint32_t hi = (uint32_t)(((uint64_t)P.next_dense_bytes * (c + 1) / G) & ~15ull);
            if (hi > lo)
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(P.next_dense + lo), "r"(hi - lo) : "memory");
        }
        // publish: the CTA's act stores happen-before (barrier + fence) the unit flags
        if (tid < nU) {
            __threadfence();
            asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&sy->uflag[c + tid * G]), "r"(tag) : "memory");
        }
        NMOE_PHASE(4);

        // ---- 5. output bands: shared down + k expert downs + combine -----------------
        if (nB > 0 && !S->abort) {
            float *sact = reinterpret_cast<float *>(sm + Y.sact);
            float *ssum = reinterpret_cast<float *>(sm + Y.ssum);
            float *actf = reinterpret_cast<float *>(sm + Y.actf);   // [k][16 chunks][kXP]
            float *ag = reinterpret_cast<float *>(sm + Y.ag);       // [k][8] group sums
            float *sred = reinterpret_cast<float *>(sm + Y.sred);   // [nB][16]
            {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (tid < 128 && !poll_tagged4(&sy->shared_act[4 * tid], tag, &v.x, deadline)) NMOE_GIVEUP(5);
                if (tid == 128 && !poll_tagged1(&sy->score, tag, &S->score, deadline)) NMOE_GIVEUP(5);
                __syncthreads();
                if (tid < 128 && !S->abort) {
                    const int col = 4 * tid;
                    *reinterpret_cast<float4 *>(sact + (col >> 5) * kXP + (col & 31)) = v;
                    float e = v.x + v.z, o = v.y + v.w;
#pragma unroll
                    for (int m = 1; m < 8; m <<= 1) {
                        e += __shfl_xor_sync(0xffffffffu, e, m);
                        o += __shfl_xor_sync(0xffffffffu, o, m);
                    }
                    if ((tid & 7) == 0) {
                        ssum[3 * (col >> 5)] = e;
                        ssum[3 * (col >> 5) + 1] = o;
                        ssum[3 * (col >> 5) + 2] = e + o;
                    }
                }
                __syncthreads();
            }
            if (!S->abort) {
                // shared down: warp per output row (16 rows per band)
                if (mbar_wait_warp(&bars[kBarSDown], 0, deadline)) {
#pragma unroll 1
                    for (int rr = warp; rr < nB * 16; rr += kWarps) {
                        const uint8_t *base = sm + Y.sdn + rr * SDW;
                        const uint8_t *w[1] = {base};
                        const uint16_t *sp[1] = {reinterpret_cast<const uint16_t *>(base + 256)};
                        const uint16_t *bp[1] = {reinterpret_cast<const uint16_t *>(base + 272)};
                        float acc[1] = {0.f};
                        dense_dot<kSQ4, 1>(w, sp, bp, sact, ssum, lane, 32, kInter / (kSQ4 ? 32 : 8), acc);
                        const float v = warp_sum(acc[0]);
                        if (lane == 0) sred[rr] = v;
                    }
                } else if (lane == 0) {
                    NMOE_GIVEUP(5);
                }
                if (tid == 0) NMOE_STAMP(12);
            }
            __syncthreads();
            if (!S->abort) {
                // act, slot by slot: the wps warps of slot s wait for that slot's 32 unit
                // flags, stage its act (fp32 padded + parity sums) and its half2 pair table,
                // then run its down dots. Slots are ready at different times (first units
                // before second units), so no slot waits for the others; the group syncs on
                // its own named barrier.
                float *asum = reinterpret_cast<float *>(sm + Y.ag);   // [k*16 chunks][3]
                const int wps = max(1, kWarps / k);
                const int s = warp / wps, part = warp % wps;
                const int gn = wps * 32, gt = tid - s * gn;
                auto gsync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + s), "r"(gn) : "memory"); };
                bool bands_ok = true;
                if (s < k) {
                    if (gt < 32) {
                        bool got = false;
                        for (uint32_t it = 0; it < kMaxSpins; ++it) {
                            if (ld_acquire_u32(&sy->uflag[32 * s + gt]) == tag) { got = true; break; }
                            if (globaltimer_ns() > deadline) break;
                            __nanosleep(32);
                        }
                        if (!got) NMOE_GIVEUP(6);
                    }
                    gsync();
#pragma unroll 1
                    for (int i = gt; i < kInter / 4; i += gn) {   // uniform within a warp
                        const int ii = s * (kInter / 4) + i;
                        const float4 v = __ldcg(reinterpret_cast<const float4 *>(sy->act) + ii);
                        const int e = 4 * ii;
                        *reinterpret_cast<float4 *>(actf + (e >> 5) * kXP + (e & 31)) = v;
                        if (kHalf) {
                            float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                            if (lane == 0) atomicMax(&S->amax_bits[s], __float_as_uint(m));
                        }
                        float e2 = v.x + v.z, o2 = v.y + v.w;
#pragma unroll
                        for (int m = 1; m < 8; m <<= 1) {
                            e2 += __shfl_xor_sync(0xffffffffu, e2, m);
                            o2 += __shfl_xor_sync(0xffffffffu, o2, m);
                        }
                        if ((ii & 7) == 0) {
                            asum[3 * (ii >> 3)] = e2;
                            asum[3 * (ii >> 3) + 1] = o2;
                            asum[3 * (ii >> 3) + 2] = e2 + o2;
                        }
                    }
                    gsync();
                    if (kHalf) {
                        __half2 *ah = reinterpret_cast<__half2 *>(sm + Y.acth) + s * 256;
                        const int E = half_exp(__uint_as_float(S->amax_bits[s]));
#pragma unroll 1
                        for (int e = gt; e < 256; e += gn) ah[e] = pair_entry<kBits>(actf + s * (kInter / 32) * kXP, e, E);
                        gsync();
                    }
                    if (tid == 0) NMOE_STAMP(6);
                    for (int i = 0; i < nB; ++i) bands_ok &= mbar_wait_warp(&bars[kBarBand0 + i], 0, deadline);
                    if (!bands_ok && lane == 0) NMOE_GIVEUP(7);
                    if (tid == 0) NMOE_STAMP(14);
                }
                float *dpart = reinterpret_cast<float *>(sm + Y.part);   // [band][slot][16 rows]
                if (bands_ok) {
                    // warp -> (slot, part); lane -> (chunk of the 512 columns, row subgroup);
                    // the lane's act chunk stays in registers across its rows
                    constexpr int kLanesPer = kBits == 4 ? 16 : 8;   // chunks per down row
                    constexpr int kSubs = 32 / kLanesPer;
                    const int cc = lane % kLanesPer, sub = lane / kLanesPer;
                    const int stride = kSubs * wps;
                    const int npass = (16 + stride - 1) / stride;
                    if (s < k && S->valid[s]) {
                        uint64_t x2[kHalf ? 1 : 16 * (kBits == 4 ? 1 : 2)];
                        constexpr int kPairs = kBits == 4 ? 16 : 32;
                        __half2 ahr[kHalf ? kPairs : 1];
                        float xe, xo;
                        const float ascale = exp2f((float)(24 - half_exp(__uint_as_float(S->amax_bits[s]))));
                        if (kHalf) {
                            const __half2 *src = reinterpret_cast<const __half2 *>(sm + Y.acth) + s * 256 + cc * kPairs;
#pragma unroll
                            for (int e = 0; e < kPairs; ++e) ahr[e] = src[e];
                            const float *vs = asum + s * (kInter / 32) * 3;
                            const int n32 = kBits == 4 ? 1 : 2;
                            xe = vs[3 * n32 * cc] + (n32 == 2 ? vs[3 * (2 * cc + 1)] : 0.f);
                            xo = vs[3 * n32 * cc + 1] + (n32 == 2 ? vs[3 * (2 * cc + 1) + 1] : 0.f);
                        } else {
                            load_chunk_x2<kBits>(actf + s * (kInter / 32) * kXP, asum + s * (kInter / 32) * 3, cc, x2, xe, xo);
                        }
                        for (int i = 0; i < nB; ++i) {
                            const uint8_t *bd = sm + Y.bands + (i * Y.kmax + s) * pg.db;
                            const uint16_t *ds = reinterpret_cast<const uint16_t *>(bd + pg.tile_band_d);
                            const uint16_t *dbi = ds + 16 * 8;
                            const int grp = kBits == 4 ? cc >> 1 : cc;
                            for (int pss = 0; pss < npass; ++pss) {   // warp-uniform trip count
                                const int r = part + wps * sub + stride * pss;
                                float v = 0.f;
                                if (r < 16)
                                    v = fmaf(bf16_to_f32(ds[r * 8 + grp]),
                                             kHalf ? qdot_h2<kBits>(lds128(bd + r * pg.wd * 4 + 16 * cc), ahr) * ascale
                                                   : qdot_chunk<kBits>(lds128(bd + r * pg.wd * 4 + 16 * cc), x2, xe, xo),
                                             bf16_to_f32(dbi[r * 8 + grp]) * (xe + xo));
#pragma unroll
                                for (int o = kLanesPer / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                                if (cc == 0 && r < 16) dpart[(i * kMaxK + s) * 16 + r] = v;
                            }
                        }
                    }
                }
                if (tid == 0) NMOE_STAMP(5);
                __syncthreads();
                if (tid < nB * 16 && !S->abort) {
                    const int i = tid >> 4, row = tid & 15;
                    const int o = (band0 + i * G) * 16 + row;
                    float moe = 0.f;
                    for (int s = 0; s < k; ++s)
                        if (S->valid[s]) moe += S->w[s] * dpart[(i * kMaxK + s) * 16 + row];
                    P.out[o] = hm_reg + moe + sigmoidf_(S->score) * sred[tid];
                }
            }
        }
    }

    // ---- 7. teardown -----------------------------------------------------------------
    __syncthreads();
    if (S->abort) {
        // let issued copies land (bounded) before this CTA's shared memory is released
        const uint64_t dl2 = globaltimer_ns() + 50000000ull;
        if (tid < kMaxBars) mbar_wait(&bars[tid], 0, dl2);
        __syncthreads();
    }
    NMOE_PHASE(7);
    if (tid == 0) {
        __threadfence();
        const uint32_t prev = atomicAdd(&sy->done_cnt, 1u);
        if (prev == (uint32_t)G - 1) {
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
    Y.nR = cdiv(kExperts, G);
    Y.nS = cdiv(kInter, G);
    Y.nUmax = cdiv(32 * kmax, G);
    Y.nBmax = cdiv(128, G);
    Y.kmax = kmax;
    const uint32_t RW = rq4 ? 1152 : 4096, SRW = sq4 ? 1152 : 4096, SDW = sq4 ? 288 : 1024;
    uint32_t off = 0;
    auto take = [&](uint32_t bytes) {
        const uint32_t o = off;
        off += (bytes + 127) & ~127u;
        return o;
    };
    Y.bars = take(kMaxBars * 8);
    Y.ctl = take(sizeof(Ctl));
    Y.xs = take(kHidden / 32 * kXP * 4);
    Y.xsum = take(kHidden / 32 * 3 * 4);
    Y.rw = take(Y.nR * RW);
    Y.sp = take(Y.nS * 2 * SRW);
    Y.gv = take(SRW);
    Y.sdn = take(Y.nBmax * 16 * SDW);
    Y.bands = take(Y.nBmax * kmax * pg.db);
    Y.part = take(Y.nBmax * kMaxK * 16 * 4);
    Y.dsp = take((Y.nR * 8 + Y.nS * 16 + 8) * 4);
    Y.sred = take(Y.nBmax * 16 * 4);
    Y.xh = take(1024 * 4);
    // `units` last; the act buffers alias it (act is staged after the routed gate/up
    // is done)
    Y.units = take(0);
    uint32_t ua = 0;
    auto utake = [&](uint32_t bytes) {
        const uint32_t o = Y.units + ua;
        ua += (bytes + 127) & ~127u;
        return o;
    };
    Y.sact = utake((kInter / 32) * kXP * 4);
    Y.ssum = utake((kInter / 32) * 3 * 4);
    Y.actf = utake(kmax * (kInter / 32) * kXP * 4);
    Y.ag = utake(kmax * (kInter / 32) * 3 * 4);
    Y.acth = utake(kmax * 256 * 4);
    const uint32_t unit_bytes = std::max(Y.nUmax * pg.bp, ua);
    Y.total = Y.units + unit_bytes;
    return Y;
}

template <int kBits, bool kRQ4, bool kSQ4>
static cudaError_t set_attr(int smem) {
    cudaError_t e = cudaFuncSetAttribute(k_moe_decode_fused<kBits, kRQ4, kSQ4, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_moe_decode_fused<kBits, kRQ4, kSQ4, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem);
}

int nmoe_fused_init(nmoe_moe_ctx *ctx) {
    FusedState *F = new FusedState();
    ctx->fused = F;
    if (cudaMalloc(&F->sy, sizeof(FusedSync)) != cudaSuccess) return NMOE_ENOMEM;
    if (cudaMemset(F->sy, 0, sizeof(FusedSync)) != cudaSuccess) return NMOE_ECUDA;
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device);
    F->grid = ctx->num_sms;
    if (const char *t = getenv("NMOE_WAIT_TIMEOUT_MS")) F->timeout_ns = (uint64_t)atoll(t) * 1000000ull;
    if (const char *t = getenv("NMOE_TIMELINE")) F->timeline = atoi(t) != 0;
    if (const char *t = getenv("NMOE_PDL")) F->pdl = atoi(t) != 0;
    if (const char *t = getenv("NMOE_TEST_STALL_WAIT")) F->stall = atoi(t) != 0;
    F->expert_fp32 = (ctx->cfg.flags & NMOE_FLAG_EXPERT_FP32) != 0;
    if (const char *t = getenv("NMOE_EXPERT_FP32")) F->expert_fp32 = atoi(t) != 0;
    const int bits = ctx->cfg.quant_bits;
    const bool rq4 = ctx->cfg.router_dtype == NMOE_DTYPE_Q4, sq4 = ctx->cfg.shared_dtype == NMOE_DTYPE_Q4;
    F->lay = make_layout(bits, rq4, sq4, F->grid, ctx->cfg.k_max);
    if ((int)F->lay.total > max_smem || F->lay.nUmax > kMaxUnits || F->lay.nBmax > kMaxBands) {
        nmoe_ctx_set_error(ctx, "decode kernel needs %u B of shared memory per CTA on %d SMs (device max %d)",
                           F->lay.total, F->grid, max_smem);
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
static cudaError_t launch(const FusedParams &p, int grid, cudaStream_t st, bool half, bool pdl) {
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
    if (half) return cudaLaunchKernelEx(&cfg, k_moe_decode_fused<kBits, kRQ4, kSQ4, true>, p);
    return cudaLaunchKernelEx(&cfg, k_moe_decode_fused<kBits, kRQ4, kSQ4, false>, p);
}

cudaError_t nmoe_fused_launch(nmoe_moe_ctx *ctx, const FusedCall &a, cudaStream_t st) {
    FusedState *F = ctx->fused;
    FusedParams p;
    p.experts = a.experts;
    p.router = a.router;
    p.spairs = a.spairs;
    p.gvec = a.gvec;
    p.sdown = a.sdown;
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
    p.timeline = F->timeline;
    p.stall = F->stall;
    p.sy = F->sy;
    p.err = a.err;
    p.lay = F->lay;
    p.timeout_ns = F->timeout_ns;
    const int bits = ctx->cfg.quant_bits;
    const bool rq4 = ctx->cfg.router_dtype == NMOE_DTYPE_Q4, sq4 = ctx->cfg.shared_dtype == NMOE_DTYPE_Q4;
#define NMOE_L(B, R, S) \
    if (bits == B && rq4 == R && sq4 == S) return launch<B, R, S>(p, F->grid, st, !F->expert_fp32, F->pdl);
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
    if (cudaMemcpy(out, ctx->fused->sy->tl, (size_t)n_ctas * 16 * sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
        return NMOE_ECUDA;
    return NMOE_OK;
}
