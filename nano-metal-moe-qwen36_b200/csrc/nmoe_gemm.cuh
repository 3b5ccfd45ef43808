// nmoe_gemm.cuh -- grouped GEMM for the T-token MoE block on 5th-generation tensor cores.
//
// D[m][n] = sum_k A[m][k] * B[n][k] per work item, where
//   A = 128 rows of a weight matrix (an expert's gate/up or down rows, the router, the
//       shared expert), read from HBM in its stored format (q4 / q2 / bf16) by TMA and
//       dequantised to bf16 in shared memory by a dequant warpgroup;
//   B = up to 128 token rows (the tokens routed to one expert, in position order),
//       gathered with cp.async into 128B-swizzled shared memory;
//   D = fp32 in tensor memory (TMEM), double-buffered so the epilogue of one item
//       overlaps the main loop of the next.
// This is the swap-AB form of the reference's per-token expert matvecs
// (nmoe_expert_gate_up_q4_batched, metal/kernels.metal:562-640; expert down,
// kernels.metal:642-714): weights are the MMA's M side, tokens its N side, so a group of
// a handful of tokens still fills the 128-row MMA.
//
// K order: every 8-column group is held in the order [0,4,1,5,2,6,3,7] in shared memory
// (A and B alike, so the products are unchanged). That order lets a q4 word's nibble
// pairs (v_i, v_{i+4}) become one bf16x2 with a single LOP3. Token activations are
// stored in that order by the producer kernels (prep for x, the SwiGLU epilogue for act).
//
// Warp roles (512 threads, one CTA per SM, persistent over the item list):
//   warp 0      TMA producer: raw weight tiles + scale/bias tiles
//   warp 1      MMA issuer (one thread) and TMEM owner
//   warps 2-3   B loader: cp.async gather of token rows
//   warps 4-11  dequant: raw tile -> bf16 swizzled A tile
//   warps 12-15 epilogue: TMEM -> registers -> SwiGLU / store
// Every mbarrier wait is bounded; on timeout the CTA records kErrTimeout, drains what it
// has in flight (bounded), frees TMEM and exits.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "nmoe_sm100.cuh"

namespace nmoe {

enum : int { kAFmtQ4 = 4, kAFmtQ2 = 2, kAFmtBf16 = 16 };
enum : int { kEpiSwiGLU = 0, kEpiBf16 = 1, kEpiF32 = 2 };
enum : int { kPassHiHi = 1, kPassHiLo = 2, kPassLoHi = 4 };

constexpr int kGemmThreads = 512;
constexpr int kGemmNChunk = 128;       // tokens per item (MMA N <= 128)
constexpr int kGemmMaxGroups = 256;
constexpr int kGemmMaxProblems = 2;
constexpr int kGemmSA = 2, kGemmSB = 4, kGemmSS = 2;
constexpr int kGemmAStage = 16384;     // one matrix's 128 x 64 bf16 tile
constexpr int kGemmBStage = 16384;     // 128 tokens x 64 bf16
constexpr int kGemmScStage = 4096;     // one matrix's scales + biases, 128 rows x 8 groups

struct alignas(64) GemmProblem {
    CUtensorMap tw[2];        // weights (4D: inner, 16 rows, bands, group)
    CUtensorMap ts[2];        // scales  (4D: groups, 16 rows, bands, group)
    CUtensorMap tb[2];        // biases
    int fmt;                  // kAFmt*
    int n_mat;                // 2 = gate+up (SwiGLU epilogue), 1 otherwise
    int K;                    // 2048 or 512
    int m_tiles;              // rows / 128
    int n_groups;             // experts (or 1)
    int cnt_const;            // group size when cnt == nullptr
    const int *cnt;           // [n_groups] tokens per group
    const int *perm;          // B row of position p, or nullptr (identity)
    int in_base;              // added to the position before perm / identity
    int out_base;             // output row = out_base + position
    const uint16_t *b_hi;     // B rows [.][K] bf16, K-permuted
    const uint16_t *b_lo;     // low plane for kPassHiLo
    int passes;               // kPass* bits
    int split;                // A in fp32-exact hi/lo planes (router)
    int epi;                  // kEpi*
    int ld_out;
    void *out;
};

struct GemmParams {
    GemmProblem prob[kGemmMaxProblems];
    int n_prob;
    int sr;                   // raw stages
    int raw_stage;            // bytes per raw stage
    int *err;
    uint64_t timeout_ns;
};

// ------------------------------------------------------------------ helpers ----

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;             // LBO (unused for 128B-swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;   // SBO: 8 rows x 128 B
    d |= (uint64_t)1 << 46;             // descriptor version
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}
__device__ __forceinline__ uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ uint32_t sw128_off(int r, int chunk) { return r * 128 + (((chunk ^ (r & 7))) << 4); }

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
// (hi, lo) bf16 planes of an fp32 value pair: hi = bf16(v), lo = bf16(v - hi).
__device__ __forceinline__ uint32_t split_pair(float a, float b, bool lo) {
    const uint32_t h = pack_bf16x2(a, b);
    if (!lo) return h;
    return pack_bf16x2(a - __uint_as_float(h << 16), b - __uint_as_float(h & 0xFFFF0000u));
}

// ----------------------------------------------------------- work items ----

struct GemmTables {
    int ipre[kGemmMaxProblems][kGemmMaxGroups + 1];   // item prefix per group
    int goff[kGemmMaxProblems][kGemmMaxGroups + 1];   // position prefix per group
    int total[kGemmMaxProblems + 1];                  // item prefix per problem
};

struct GemmItem {
    int p, g, mt, c0, n, pos0;
};

__device__ __forceinline__ int gemm_group_count(const GemmProblem &pr, int g) {
    return pr.cnt ? pr.cnt[g] : pr.cnt_const;
}

// One warp per problem: prefix sums over groups of positions and of items.
__device__ __forceinline__ void gemm_build_tables(const GemmParams &P, GemmTables *T, int warp, int lane) {
    if (warp < P.n_prob) {
        const GemmProblem &pr = P.prob[warp];
        int c[8], it[8], sc = 0, si = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int g = 8 * lane + j;
            c[j] = g < pr.n_groups ? gemm_group_count(pr, g) : 0;
            it[j] = (c[j] + kGemmNChunk - 1) / kGemmNChunk * pr.m_tiles;
            sc += c[j];
            si += it[j];
        }
        int xc = sc, xi = si;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, xc, o), b = __shfl_up_sync(0xffffffffu, xi, o);
            if (lane >= o) { xc += a; xi += b; }
        }
        int pc = xc - sc, pi = xi - si;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            T->goff[warp][8 * lane + j] = pc;
            T->ipre[warp][8 * lane + j] = pi;
            pc += c[j];
            pi += it[j];
        }
        if (lane == 31) {
            T->goff[warp][kGemmMaxGroups] = pc;
            T->ipre[warp][kGemmMaxGroups] = pi;
        }
    }
}

__device__ __forceinline__ GemmItem gemm_item(const GemmParams &P, const GemmTables *T, int it) {
    GemmItem w;
    w.p = it >= T->total[1] ? 1 : 0;
    int li = it - T->total[w.p];
    const int *ip = T->ipre[w.p];
    int lo = 0, hi = kGemmMaxGroups;   // largest g with ip[g] <= li
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (ip[mid] <= li) lo = mid; else hi = mid;
    }
    w.g = lo;
    li -= ip[lo];
    const GemmProblem &pr = P.prob[w.p];
    const int cnt = gemm_group_count(pr, w.g);
    const int chunks = (cnt + kGemmNChunk - 1) / kGemmNChunk;
    w.mt = li / chunks;
    const int ch = li - w.mt * chunks;
    w.c0 = ch * kGemmNChunk;
    w.n = min(kGemmNChunk, cnt - w.c0);
    w.pos0 = T->goff[w.p][w.g] + w.c0;
    return w;
}

__device__ __forceinline__ int gemm_steps(const GemmProblem &pr) {
    return __popc(pr.passes) * (pr.K / 64);
}
// pass of step s: the (s / kb)-th set bit of passes
__device__ __forceinline__ int gemm_pass(const GemmProblem &pr, int s) {
    int q = s / (pr.K / 64);
    uint32_t b = (uint32_t)pr.passes;
    while (q-- > 0) b &= b - 1;
    return __ffs(b) - 1;   // 0: hi.hi  1: hi.lo  2: lo.hi
}

__host__ __device__ __forceinline__ int raw_mat_bytes(int fmt) {
    return fmt == kAFmtQ4 ? 4096 : fmt == kAFmtQ2 ? 2048 : 16384;
}

// ------------------------------------------------------------------ kernel ----

struct GemmSmem {
    uint64_t raw_full[8], raw_empty[8];
    uint64_t sc_full[kGemmSS], sc_empty[kGemmSS];
    uint64_t a_full[kGemmSA], a_empty[kGemmSA];
    uint64_t b_full[kGemmSB], b_empty[kGemmSB];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    GemmTables T;
};

__device__ __forceinline__ void gemm_fail(GemmSmem *S, int *err) {
    S->abort = 1;
    atomicCAS(err, 0, kErrTimeout);
}

// K-permuted slot order within an 8-column group: slot s holds column kPermCol[s].
__device__ __forceinline__ int kperm_pos(int col) {   // position of column col (within its group of 8)
    const int j = col & 7;
    return (col & ~7) | (j < 4 ? 2 * j : 2 * (j - 4) + 1);
}

__global__ void __launch_bounds__(kGemmThreads, 1) k_moe_gemm(const __grid_constant__ GemmParams P) {
    extern __shared__ __align__(1024) uint8_t smraw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = sm;                                  // kGemmSA x 2 x 16 KB
    uint8_t *sB = sA + kGemmSA * 2 * kGemmAStage;      // kGemmSB x 16 KB
    uint8_t *sSc = sB + kGemmSB * kGemmBStage;         // kGemmSS x 2 x 4 KB
    uint8_t *sRaw = sSc + kGemmSS * 2 * kGemmScStage;  // sr x raw_stage
    GemmSmem *S = reinterpret_cast<GemmSmem *>(sRaw + P.sr * P.raw_stage);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t deadline = globaltimer_ns() + P.timeout_ns;

    if (tid == 0) {
        for (int i = 0; i < P.sr; ++i) { mbar_init(&S->raw_full[i], 1); mbar_init(&S->raw_empty[i], 8); }
        for (int i = 0; i < kGemmSS; ++i) { mbar_init(&S->sc_full[i], 1); mbar_init(&S->sc_empty[i], 8); }
        for (int i = 0; i < kGemmSA; ++i) { mbar_init(&S->a_full[i], 8); mbar_init(&S->a_empty[i], 1); }
        for (int i = 0; i < kGemmSB; ++i) { mbar_init(&S->b_full[i], 64); mbar_init(&S->b_empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&S->acc_full[i], 1); mbar_init(&S->acc_empty[i], 4); }
        mbar_init(&S->drain, 1);
        S->abort = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&S->tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    gemm_build_tables(P, &S->T, warp - 2 >= 0 ? warp - 2 : 99, lane);
    __syncthreads();
    if (tid == 0) {
        S->T.total[0] = 0;
        S->T.total[1] = S->T.ipre[0][kGemmMaxGroups];
        S->T.total[2] = S->T.total[1] + (P.n_prob > 1 ? S->T.ipre[1][kGemmMaxGroups] : 0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S->tmem_base;
    const int n_items = S->T.total[P.n_prob > 1 ? 2 : 1];

    if (warp == 0) {
        // ------------------------------------------------ TMA producer ----
        if (lane == 0) {
            uint32_t rit = 0, sit = 0;
            for (int it = blockIdx.x; it < n_items && !S->abort; it += gridDim.x) {
                const GemmItem w = gemm_item(P, &S->T, it);
                const GemmProblem &pr = P.prob[w.p];
                const bool q = pr.fmt != kAFmtBf16;
                const int kb = pr.K / 64, steps = gemm_steps(pr);
                const int rawm = raw_mat_bytes(pr.fmt);
                const int wpk = pr.fmt == kAFmtQ4 ? 8 : pr.fmt == kAFmtQ2 ? 4 : 64;
                for (int s = 0; s < steps; ++s) {
                    const int ks = s % kb;
                    if (q && (ks & 7) == 0) {
                        const int st = sit % kGemmSS;
                        if (!mbar_wait(&S->sc_empty[st], ((sit / kGemmSS) & 1) ^ 1, deadline)) { gemm_fail(S, P.err); break; }
                        mbar_arrive_expect_tx(&S->sc_full[st], pr.n_mat * kGemmScStage);
                        for (int m = 0; m < pr.n_mat; ++m) {
                            uint8_t *d = sSc + (st * 2 + m) * kGemmScStage;
                            tma_load_4d(d, &pr.ts[m], ks, 0, w.mt * 8, w.g, &S->sc_full[st]);
                            tma_load_4d(d + 2048, &pr.tb[m], ks, 0, w.mt * 8, w.g, &S->sc_full[st]);
                        }
                        ++sit;
                    }
                    const int st = rit % P.sr;
                    if (!mbar_wait(&S->raw_empty[st], ((rit / P.sr) & 1) ^ 1, deadline)) { gemm_fail(S, P.err); break; }
                    mbar_arrive_expect_tx(&S->raw_full[st], pr.n_mat * rawm);
                    for (int m = 0; m < pr.n_mat; ++m)
                        tma_load_4d(sRaw + st * P.raw_stage + m * rawm, &pr.tw[m], ks * wpk, 0, w.mt * 8, w.g,
                                    &S->raw_full[st]);
                    ++rit;
                }
            }
            // drain: the last fill of every stage has landed before the CTA may exit
            for (uint32_t j = rit > (uint32_t)P.sr ? rit - P.sr : 0; j < rit; ++j)
                if (!mbar_wait(&S->raw_full[j % P.sr], (j / P.sr) & 1, deadline)) break;
            for (uint32_t j = sit > (uint32_t)kGemmSS ? sit - kGemmSS : 0; j < sit; ++j)
                if (!mbar_wait(&S->sc_full[j % kGemmSS], (j / kGemmSS) & 1, deadline)) break;
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer ----
        if (lane == 0) {
            uint32_t ait = 0, bit = 0, tile = 0;
            bool issued = false;
            for (int it = blockIdx.x; it < n_items && !S->abort; it += gridDim.x, ++tile) {
                const GemmItem w = gemm_item(P, &S->T, it);
                const GemmProblem &pr = P.prob[w.p];
                const int steps = gemm_steps(pr);
                const int ab = tile & 1;
                if (!mbar_wait(&S->acc_empty[ab], ((tile >> 1) & 1) ^ 1, deadline)) { gemm_fail(S, P.err); break; }
                tc_fence_after();
                const uint32_t idesc = idesc_bf16((w.n + 15) & ~15);
                bool ok = true;
                for (int s = 0; s < steps; ++s) {
                    const int sa = ait % kGemmSA, sb = bit % kGemmSB;
                    if (!mbar_wait(&S->a_full[sa], (ait / kGemmSA) & 1, deadline) ||
                        !mbar_wait(&S->b_full[sb], (bit / kGemmSB) & 1, deadline)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t bsa = smem_u32(sB + sb * kGemmBStage);
                    for (int kk = 0; kk < 4; ++kk)
                        for (int m = 0; m < pr.n_mat; ++m)
                            tc_mma(tmem + ab * 256 + m * 128, sw128_desc(smem_u32(sA + (sa * 2 + m) * kGemmAStage)) + 2 * kk,
                                   sw128_desc(bsa) + 2 * kk, idesc, (s | kk) ? 1u : 0u);
                    issued = true;
                    tc_commit(&S->a_empty[sa]);
                    tc_commit(&S->b_empty[sb]);
                    ++ait;
                    ++bit;
                }
                if (!ok) { gemm_fail(S, P.err); break; }
                tc_commit(&S->acc_full[ab]);
            }
            if (issued) {   // every MMA issued has completed before TMEM is freed
                tc_commit(&S->drain);
                mbar_wait(&S->drain, 0, deadline + 100000000ull);
            }
        }
    } else if (warp < 4) {
        // ------------------------------------------------ B loader (64 threads) ----
        const int lt = tid - 64;
        uint32_t bit = 0;
        uint32_t pending = 0;   // committed groups not yet signalled (0 or 1)
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const GemmItem w = gemm_item(P, &S->T, it);
            const GemmProblem &pr = P.prob[w.p];
            const int kb = pr.K / 64, steps = gemm_steps(pr);
            const int n16 = (w.n + 15) & ~15;
            for (int s = 0; s < steps; ++s) {
                const int st = bit % kGemmSB;
                const bool wait_ok = __all_sync(0xffffffffu, mbar_wait(&S->b_empty[st], ((bit / kGemmSB) & 1) ^ 1, deadline));
                if (!wait_ok || S->abort) { ok = false; break; }
                const int pass = gemm_pass(pr, s), ks = s % kb;
                const uint16_t *src = pass == 1 ? pr.b_lo : pr.b_hi;
                uint8_t *dst = sB + st * kGemmBStage;
                for (int c = lt; c < n16 * 8; c += 64) {
                    const int r = c >> 3, ch = c & 7;
                    if (r < w.n) {
                        const int p = pr.in_base + w.pos0 + r;
                        const int row = pr.perm ? pr.perm[p] : p;
                        cp_async16(dst + sw128_off(r, ch), src + (size_t)row * pr.K + ks * 64 + ch * 8);
                    }
                }
                cp_async_commit();
                if (pending) {   // the previous stage is complete: publish it
                    cp_async_wait<1>();
                    fence_async_smem();
                    mbar_arrive(&S->b_full[(bit - 1) % kGemmSB]);
                }
                pending = 1;
                ++bit;
            }
        }
        cp_async_wait<0>();
        if (pending && ok) {
            fence_async_smem();
            mbar_arrive(&S->b_full[(bit - 1) % kGemmSB]);
        }
        if (!ok) gemm_fail(S, P.err);
    } else if (warp < 12) {
        // ------------------------------------------------ dequant (256 threads) ----
        const int dt = tid - 128, r = dt & 127, h = dt >> 7;
        uint32_t rit = 0, sit = 0, ait = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const GemmItem w = gemm_item(P, &S->T, it);
            const GemmProblem &pr = P.prob[w.p];
            const bool q = pr.fmt != kAFmtBf16;
            const int kb = pr.K / 64, steps = gemm_steps(pr);
            const int rawm = raw_mat_bytes(pr.fmt);
            for (int s = 0; s < steps; ++s) {
                const int ks = s % kb;
                const int lo = gemm_pass(pr, s) == 2;
                const int ss = sit % kGemmSS;
                if (q && (ks & 7) == 0)
                    if (!mbar_wait_warp(&S->sc_full[ss], (sit / kGemmSS) & 1, deadline)) { ok = false; break; }
                const int sr = rit % P.sr, sa = ait % kGemmSA;
                if (!mbar_wait_warp(&S->raw_full[sr], (rit / P.sr) & 1, deadline) ||
                    !mbar_wait_warp(&S->a_empty[sa], ((ait / kGemmSA) & 1) ^ 1, deadline)) {
                    ok = false;
                    break;
                }
                if (S->abort) { ok = false; break; }
                for (int m = 0; m < pr.n_mat; ++m) {
                    const uint8_t *raw = sRaw + sr * P.raw_stage + m * rawm;
                    uint8_t *a = sA + (sa * 2 + m) * kGemmAStage + r * 128;
                    const int rx = r & 7;
                    if (!q) {
                        // bf16 rows: 4 groups of 8 columns, pair (v_j, v_{j+4}) per word
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint4 v = lds128(raw + r * 128 + h * 64 + j * 16);
                            uint4 o;
                            if (pr.split && lo) {
                                o = make_uint4(0, 0, 0, 0);
                            } else {
                                o.x = prmt(v.x, v.z, 0x5410);
                                o.y = prmt(v.x, v.z, 0x7632);
                                o.z = prmt(v.y, v.w, 0x5410);
                                o.w = prmt(v.y, v.w, 0x7632);
                            }
                            *reinterpret_cast<uint4 *>(a + (((4 * h + j) ^ rx) << 4)) = o;
                        }
                        continue;
                    }
                    const uint8_t *sc = sSc + (ss * 2 + m) * kGemmScStage;
                    const uint16_t s16 = reinterpret_cast<const uint16_t *>(sc)[r * 8 + (ks & 7)];
                    const uint16_t b16 = reinterpret_cast<const uint16_t *>(sc + 2048)[r * 8 + (ks & 7)];
                    // 4 words of 8 q4 values, or 2 words of 16 q2 values: 4 groups of 8
                    uint32_t gw[4];   // per group: values at bits [0,16) (q4: 8 x 4 bits)
                    int sh = 4;       // bit step between consecutive values of a group
                    if (pr.fmt == kAFmtQ4) {
                        const uint4 v = lds128(raw + r * 32 + h * 16);
                        gw[0] = v.x; gw[1] = v.y; gw[2] = v.z; gw[3] = v.w;
                    } else {
                        const uint2 v = *reinterpret_cast<const uint2 *>(raw + r * 16 + h * 8);
                        // 8 q2 values of a group in bits [0,16): spread so (v_i, v_{i+4}) sit 16 apart
                        const uint32_t g0 = v.x & 0xFFFFu, g1 = v.x >> 16, g2 = v.y & 0xFFFFu, g3 = v.y >> 16;
                        gw[0] = g0 | (g0 << 8); gw[1] = g1 | (g1 << 8);
                        gw[2] = g2 | (g2 << 8); gw[3] = g3 | (g3 << 8);
                        sh = 2;
                    }
                    const uint32_t mask = pr.fmt == kAFmtQ4 ? 0x000F000Fu : 0x00030003u;
                    if (!pr.split) {
                        const uint32_t s2 = (uint32_t)s16 | ((uint32_t)s16 << 16);
                        const uint32_t b2 = (uint32_t)b16 | ((uint32_t)b16 << 16);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint32_t o[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t qq = ((gw[j] >> (sh * i)) & mask) | 0x43004300u;
                                o[i] = bf16x2_fma(bf16x2_sub(qq, 0x43004300u), s2, b2);
                            }
                            *reinterpret_cast<uint4 *>(a + (((4 * h + j) ^ rx) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    } else {
                        const float sf = __uint_as_float((uint32_t)s16 << 16), bf = __uint_as_float((uint32_t)b16 << 16);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint32_t o[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t qq = (gw[j] >> (sh * i)) & mask;
                                const float va = fmaf((float)(qq & 0xFFFFu), sf, bf);
                                const float vb = fmaf((float)(qq >> 16), sf, bf);
                                o[i] = split_pair(va, vb, lo);
                            }
                            *reinterpret_cast<uint4 *>(a + (((4 * h + j) ^ rx) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&S->raw_empty[sr]);
                    mbar_arrive(&S->a_full[sa]);
                    if (q && ((ks & 7) == 7 || ks == kb - 1)) mbar_arrive(&S->sc_empty[ss]);
                }
                if (q && ((ks & 7) == 7 || ks == kb - 1)) ++sit;
                ++rit;
                ++ait;
            }
        }
        if (!ok && lane == 0) gemm_fail(S, P.err);
    } else {
        // ------------------------------------------------ epilogue (128 threads) ----
        const int eq = warp & 3, row = 32 * eq + lane;
        uint32_t tile = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++tile) {
            const GemmItem w = gemm_item(P, &S->T, it);
            const GemmProblem &pr = P.prob[w.p];
            const int ab = tile & 1;
            const bool ok = mbar_wait_warp(&S->acc_full[ab], (tile >> 1) & 1, deadline);
            if (!ok || S->abort) {
                if (!ok && lane == 0) gemm_fail(S, P.err);
                break;
            }
            tc_fence_after();
            const int m = w.mt * 128 + row;
            const uint32_t tbase = tmem + ((uint32_t)(32 * eq) << 16) + ab * 256;
            const int obase = pr.out_base + w.pos0;
            for (int c0 = 0; c0 < w.n; c0 += 8) {
                uint32_t g[8], u[8];
                tc_ld8(tbase + c0, g);
                if (pr.n_mat == 2) tc_ld8(tbase + 128 + c0, u);
                tc_wait_ld();
                const int nc = min(8, w.n - c0);
                if (pr.epi == kEpiSwiGLU) {
                    uint16_t *o = static_cast<uint16_t *>(pr.out);
                    const int col = kperm_pos(m);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j < nc) {
                            const float gv = __uint_as_float(g[j]), uv = __uint_as_float(u[j]);
                            const float a = gv / (1.f + expf(-gv)) * uv;
                            o[(size_t)(obase + c0 + j) * pr.ld_out + col] = (uint16_t)(pack_bf16x2(a, 0.f) & 0xFFFFu);
                        }
                } else if (pr.epi == kEpiBf16) {
                    uint16_t *o = static_cast<uint16_t *>(pr.out);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j < nc)
                            o[(size_t)(obase + c0 + j) * pr.ld_out + m] =
                                (uint16_t)(pack_bf16x2(__uint_as_float(g[j]), 0.f) & 0xFFFFu);
                } else {
                    float *o = static_cast<float *>(pr.out);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j < nc) o[(size_t)(obase + c0 + j) * pr.ld_out + m] = __uint_as_float(g[j]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S->acc_empty[ab]);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

}  // namespace nmoe
