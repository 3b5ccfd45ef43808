// nmoe_gemm.cuh -- grouped GEMM for the T-token MoE block on 5th-generation tensor cores.
//
// D[m][n] = sum_k A[m][k] * B[n][k] per work item, where
//   A = 128 rows of a weight matrix (an expert's gate/up or down rows, the router, the
//       shared expert), read from HBM in its stored format (q4 / q2 / bf16) by TMA,
//       dequantised to bf16 by two dequant warpgroups and written straight into tensor
//       memory (tcgen05.st), where the MMA reads it: no bf16 tile crosses shared memory;
//   B = up to 128 token rows (the tokens routed to one expert, contiguous in position
//       order), loaded by TMA into 128B-swizzled shared memory;
//   D = fp32 in tensor memory (TMEM columns 0-255): one buffer for gate+up items, two
//       (so the epilogue overlaps the next item) for single-matrix items. Columns 256-511
//       hold four A stages of 2 x 32 columns.
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
//   warp 1      MMA issuer for matrix 0 (one thread) and TMEM owner
//   warp 2      B loader: TMA tiles of token rows (16 rows x 64 columns)
//   warp 3      MMA issuer for matrix 1 (one thread)
//   warps 4-11  dequant: raw tile -> bf16 A rows in TMEM
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
constexpr int kGemmMaxPeers = 8;       // expert parallelism: ranks whose return buffers an epilogue writes
constexpr int kGemmSA = 4, kGemmSB = kGemmSA, kGemmSS = 2;   // kGemmSS scale stages per dequant group
// A step's A stage (TMEM) and B stage (shared memory) share one ring position: one MMA
// commit frees both, and the B tile's TMA completes on the stage's a_full barrier, so the
// MMA issuer waits on a single barrier per step.
constexpr int kGemmMaxSlots = 16;
constexpr uint32_t kGemmAccCols = 256; // accumulators: TMEM columns [0, 256)
constexpr uint32_t kGemmACols = 64;    // one A stage: 2 matrices x 32 columns (bf16 pairs)
constexpr int kGemmBStage = 16384;     // 128 tokens x 64 bf16
constexpr int kGemmScStage = 4096;     // one matrix's scales + biases, 128 rows x 8 groups
constexpr int kGemmSlot = 8192;        // raw weight slot
// Raw weight slots: a q4/q2 slot holds one 64-column step of all 128 rows (8 KB for q4
// gate+up, less otherwise); a bf16 step spans `nslot` slots, each holding a block of rows
// (gate+up: 4 x 32 rows, single: 2 x 64).

struct alignas(64) GemmProblem {
    CUtensorMap tw[2];        // weights (4D: inner, 16 rows, bands, group)
    CUtensorMap ts[2];        // scales  (4D: groups, 16 rows, bands, group)
    CUtensorMap tb[2];        // biases
    CUtensorMap tx[2];        // B rows (2D: K columns, rows; box 64 x 16, 128B swizzle): hi, lo
    int fmt;                  // kAFmt*
    int a_cm;                 // weights in down group slabs: tiles [wpg words][128 rows]
                              // (column-major), scales/biases [8 groups][128 rows]
    int n_mat;                // 2 = gate+up, 1 otherwise
    int K;                    // 2048 or 512
    int m_tiles;              // rows / 128
    int ksplit;               // K slices per tile (partial sums, kEpiF32 only)
    int n_groups;             // experts (or 1)
    int cnt_const;            // group size when cnt == nullptr
    const int *cnt;           // [n_groups] tokens per group
    int group_mod;            // weight group of group g = g % group_mod (0: g); expert
                              // parallelism orders groups (source rank, local expert)
    int slab_groups;          // expert parallelism: groups come in slabs of slab_groups (one
    int slab_rows;            // per source rank) whose rows start at slab * slab_rows (0: the
                              // groups' rows are contiguous)
    int in_base;              // B row of position p = in_base + p
    int out_base;             // output row = out_base + position (+ split * split_rows)
    int split_rows;
    const uint16_t *b_hi;     // B rows [.][K] bf16, K-permuted (tx[0])
    const uint16_t *b_lo;     // low plane for kPassHiLo (tx[1])
    int passes;               // kPass* bits
    int split;                // A in fp32-exact hi/lo planes (router)
    int epi;                  // kEpi*
    int ld_out;
    int mat_col;              // kEpiF32 with two matrices: column offset of the second
    void *out;
    // expert parallelism, kEpiBf16: the rows of slab r go straight to rank r's return
    // buffer ret_base[r] (peer memory over NVLink), at row ret_meta[r] + (position -
    // r * slab_rows); nullptr: rows go to `out`
    const int *ret_meta;
    uint8_t *ret_base[kGemmMaxPeers];
};

struct GemmParams {
    GemmProblem prob[kGemmMaxProblems];
    int n_prob;
    int sr;                   // raw slots
    int acc_bufs;             // accumulator buffers: 1 when a problem has two matrices, else 2
    int *err;
    uint64_t timeout_ns;
    uint32_t *trace;          // diagnostics: CTA 0 role timestamps (%clock), or nullptr
};

// Trace rows (1024 entries each): 0 producer slot acquired, 1 B stage issued, 2 dequant
// step start, 3 dequant step end, 4 MMA step committed (matrix 0 issuer), 5 epilogue item
// start, 6 item end, 7 raw slot data landed, 8 MMA step's A and B ready, 9 SwiGLU epilogue
// chunk before / after its TMEM loads, 10 dequant step begins waiting, 11 A stage free,
// 12 scales ready.
constexpr int kTraceRow = 1024;
constexpr int kTraceRows = 13;
__device__ __forceinline__ void trace_put(const GemmParams &P, int row, uint32_t i) {
    if (P.trace != nullptr && blockIdx.x == 0 && i < (uint32_t)kTraceRow) {
        uint32_t c;
        asm volatile("mov.u32 %0, %%clock;" : "=r"(c));
        P.trace[row * kTraceRow + i] = c;
    }
}

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
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
// Four rows (r0..r3) of 64 columns starting at column c of a 2D map, one row high box.
__device__ __forceinline__ void tma_gather4(void *dst, const CUtensorMap *map, int c, int r0, int r1, int r2, int r3,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(c), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_n(uint64_t *bar, uint32_t n) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(n) : "memory");
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
// D[tmem] (+)= A[tmem] * B[smem desc]^T; A: lane = row, column = a bf16 pair along K.
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

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


// ------------------------------------------------------------ geometry ----

struct StepGeo {
    int kb;      // steps per pass of one item (K / 64 / ksplit)
    int sps;     // q formats: steps per raw slot
    int nslot;   // bf16: raw slots per step
    int wpk;     // q formats: words per row per step
    int rowb;    // q formats: bytes per row in a slot
    int rawm;    // q formats: bytes per matrix in a slot
};

__host__ __device__ __forceinline__ StepGeo step_geo(int fmt, int n_mat, int K, int ksplit) {
    StepGeo g;
    g.kb = K / 64 / ksplit;
    if (fmt == kAFmtBf16) {
        g.sps = 1;
        g.nslot = 2 * n_mat;
        g.wpk = 64;
        g.rowb = 128;
        g.rawm = kGemmSlot / n_mat;
    } else {
        g.wpk = fmt == kAFmtQ4 ? 8 : 4;
        g.sps = 1;
        g.nslot = 1;
        g.rowb = g.wpk * 4 * g.sps;
        g.rawm = 128 * g.rowb;
    }
    return g;
}

// ----------------------------------------------------------- work items ----

struct GemmTables {
    int ipre[kGemmMaxProblems][kGemmMaxGroups + 1];   // item prefix per group
    int goff[kGemmMaxProblems][kGemmMaxGroups + 1];   // position prefix per group
    int total[kGemmMaxProblems + 1];                  // item prefix per problem
};

struct GemmItem {
    int p, g, e, mt, sp, n, pos0;   // e: weight group (expert) of group g
};

__device__ __forceinline__ int gemm_group_count(const GemmProblem &pr, int g) {
    return pr.cnt ? pr.cnt[g] : pr.cnt_const;
}

// One warp per problem: prefix sums over groups of positions and of items.
__device__ __forceinline__ void gemm_build_tables(const GemmParams &P, GemmTables *T, int prob, int lane) {
    if (prob < P.n_prob) {
        const GemmProblem &pr = P.prob[prob];
        int c[8], it[8], sc = 0, si = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int g = 8 * lane + j;
            c[j] = g < pr.n_groups ? gemm_group_count(pr, g) : 0;
            it[j] = (c[j] + kGemmNChunk - 1) / kGemmNChunk * pr.m_tiles * pr.ksplit;
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
        if (pr.slab_groups > 0) {
            // rows of slab r (groups [r*G, (r+1)*G), lanes [r*G/8, (r+1)*G/8)) start at r*slab_rows
            const int lanes = pr.slab_groups / 8, r = lane / lanes;
            const int base = __shfl_sync(0xffffffffu, pc, r * lanes);
            pc = pc - base + r * pr.slab_rows;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            T->goff[prob][8 * lane + j] = pc;
            T->ipre[prob][8 * lane + j] = pi;
            pc += c[j];
            pi += it[j];
        }
        if (lane == 31) {
            T->goff[prob][kGemmMaxGroups] = pc;
            T->ipre[prob][kGemmMaxGroups] = pi;
        }
    }
}

// Items of a group in the order (m tile, K slice, token chunk): consecutive items share
// the weight tile, so the CTAs working on the chunks of one expert read it from L2.
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
    w.e = pr.group_mod ? w.g % pr.group_mod : w.g;
    const int cnt = gemm_group_count(pr, w.g);
    const int chunks = (cnt + kGemmNChunk - 1) / kGemmNChunk;
    const int per_mt = chunks * pr.ksplit;
    w.mt = li / per_mt;
    li -= w.mt * per_mt;
    w.sp = li / chunks;
    const int c0 = (li - w.sp * chunks) * kGemmNChunk;
    w.n = min(kGemmNChunk, cnt - c0);
    w.pos0 = T->goff[w.p][w.g] + c0;
    return w;
}

// pass of pass index q: the q-th set bit of passes (0: hi.hi  1: hi.lo  2: lo.hi)
__device__ __forceinline__ int gemm_pass(int passes, int q) {
    uint32_t b = (uint32_t)passes;
    while (q-- > 0) b &= b - 1;
    return __ffs(b) - 1;
}

// ------------------------------------------------------------- dequant ----
// One thread converts row r, columns [32h, 32h+32) of a 64-column step (four groups of
// 8) and stores them as 16 bf16 pairs into its TMEM lane (tcgen05.st, 16 columns), each
// group as (v0,v4)(v1,v5)(v2,v6)(v3,v7): the K order [0,4,1,5,2,6,3,7].

// gw[g]: group g's 8 values, value i at bit sh*i and value i+4 at bit sh*i + 16.
template <int kFmt>
__device__ __forceinline__ void dq_load(const uint8_t *raw, int h, uint32_t *gw) {
    if (kFmt == kAFmtQ4) {
        const uint4 v = lds128(raw + h * 16);
        gw[0] = v.x; gw[1] = v.y; gw[2] = v.z; gw[3] = v.w;
    } else {
        const uint2 v = *reinterpret_cast<const uint2 *>(raw + h * 8);
        const uint32_t g0 = v.x & 0xFFFFu, g1 = v.x >> 16, g2 = v.y & 0xFFFFu, g3 = v.y >> 16;
        gw[0] = g0 | (g0 << 8); gw[1] = g1 | (g1 << 8);
        gw[2] = g2 | (g2 << 8); gw[3] = g3 | (g3 << 8);
    }
}

// Same groups from a column-major tile ([word column][128 rows] u32, row r).
template <int kFmt>
__device__ __forceinline__ void dq_load_cm(const uint8_t *raw, int r, int h, uint32_t *gw) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(raw) + r;
    if (kFmt == kAFmtQ4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) gw[i] = w[(4 * h + i) * 128];
    } else {
        const uint32_t a = w[(2 * h) * 128], b = w[(2 * h + 1) * 128];
        const uint32_t g0 = a & 0xFFFFu, g1 = a >> 16, g2 = b & 0xFFFFu, g3 = b >> 16;
        gw[0] = g0 | (g0 << 8); gw[1] = g1 | (g1 << 8);
        gw[2] = g2 | (g2 << 8); gw[3] = g3 | (g3 << 8);
    }
}

// taddr: this thread's lane, column of matrix 0's half h; matrix m at +32 m.
// kCM: single-matrix column-major tile (raw = the slot, cm_r = the row).
template <int kFmt, int kNMat, bool kCM = false>
__device__ __forceinline__ void dq_step_q(const uint8_t *raw, int rawm, const uint8_t *sc, int sidx, uint32_t taddr,
                                          int h, int cm_r = 0) {
    constexpr int sh = kFmt == kAFmtQ4 ? 4 : 2;
    constexpr uint32_t mask = kFmt == kAFmtQ4 ? 0x000F000Fu : 0x00030003u;
    uint32_t gw[kNMat][4], s2[kNMat], b2[kNMat];
#pragma unroll
    for (int m = 0; m < kNMat; ++m) {
        if (kCM) dq_load_cm<kFmt>(raw, cm_r, h, gw[m]);
        else dq_load<kFmt>(raw + m * rawm, h, gw[m]);
        const uint32_t s16 = reinterpret_cast<const uint16_t *>(sc + m * kGemmScStage)[sidx];
        const uint32_t b16 = reinterpret_cast<const uint16_t *>(sc + m * kGemmScStage + 2048)[sidx];
        s2[m] = s16 | (s16 << 16);
        b2[m] = b16 | (b16 << 16);
    }
#pragma unroll
    for (int m = 0; m < kNMat; ++m) {
        uint32_t o[16];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t qq = ((gw[m][jj] >> (sh * i)) & mask) | 0x43004300u;
                o[4 * jj + i] = bf16x2_fma(bf16x2_sub(qq, 0x43004300u), s2[m], b2[m]);
            }
        tc_st16(taddr + 32 * m, o);
    }
}

// fp32-exact planes (router): hi = bf16(q*s + b), lo = bf16(q*s + b - hi).
template <int kFmt>
__device__ __forceinline__ void dq_step_split(const uint8_t *raw, const uint8_t *sc, int sidx, uint32_t taddr, int h,
                                              bool lo) {
    constexpr int sh = kFmt == kAFmtQ4 ? 4 : 2;
    constexpr uint32_t mask = kFmt == kAFmtQ4 ? 0x000F000Fu : 0x00030003u;
    uint32_t gw[4];
    dq_load<kFmt>(raw, h, gw);
    const float sf = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(sc)[sidx] << 16);
    const float bf = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(sc + 2048)[sidx] << 16);
    uint32_t o[16];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t qq = (gw[jj] >> (sh * i)) & mask;
            o[4 * jj + i] = split_pair(fmaf((float)(qq & 0xFFFFu), sf, bf), fmaf((float)(qq >> 16), sf, bf), lo);
        }
    tc_st16(taddr, o);
}

// bf16 rows: the four words of a group are (v0,v1)(v2,v3)(v4,v5)(v6,v7).
template <int kNMat>
__device__ __forceinline__ void dq_step_bf16(const uint8_t *raw, int rawm, uint32_t taddr, bool zero) {
    uint4 v[kNMat][4];
#pragma unroll
    for (int m = 0; m < kNMat; ++m)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) v[m][jj] = lds128(raw + m * rawm + jj * 16);
#pragma unroll
    for (int m = 0; m < kNMat; ++m) {
        uint32_t o[16];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            o[4 * jj + 0] = zero ? 0u : prmt(v[m][jj].x, v[m][jj].z, 0x5410);
            o[4 * jj + 1] = zero ? 0u : prmt(v[m][jj].x, v[m][jj].z, 0x7632);
            o[4 * jj + 2] = zero ? 0u : prmt(v[m][jj].y, v[m][jj].w, 0x5410);
            o[4 * jj + 3] = zero ? 0u : prmt(v[m][jj].y, v[m][jj].w, 0x7632);
        }
        tc_st16(taddr + 32 * m, o);
    }
}

// ------------------------------------------------------------------ kernel ----

struct GemmSmem {
    uint64_t raw_full[kGemmMaxSlots], raw_empty[kGemmMaxSlots];
    uint64_t sc_full[2 * kGemmSS], sc_empty[2 * kGemmSS];   // [group][stage]
    uint64_t a_full[kGemmSA], a_empty[kGemmSA];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t drain[2];
    uint32_t tmem_base;
    int abort;
    GemmTables T;
};

constexpr int kGemmEpiStage = 4 * 32 * 64;   // SwiGLU epilogue: 4 warps x 32 tokens x 32 bf16
__host__ __device__ constexpr size_t gemm_smem_bytes(int sr) {
    return 1024 + (size_t)kGemmSB * kGemmBStage + (size_t)2 * kGemmSS * 2 * kGemmScStage +
           (size_t)sr * kGemmSlot + kGemmEpiStage + sizeof(GemmSmem);
}

// Position in a ring of mbarrier-guarded stages: index, phase parity, total advances.
struct Ring {
    uint32_t idx = 0, phase = 0, count = 0, n;
    __device__ explicit Ring(int n_) : n((uint32_t)n_) {}
    __device__ __forceinline__ void next() {
        ++count;
        if (++idx == n) { idx = 0; phase ^= 1; }
    }
    // wait (bounded) for the last fill of every stage to complete
    __device__ void drain(uint64_t *full, uint64_t deadline) const {
        const uint32_t k = count < n ? count : n;
        for (uint32_t i = 0; i < k; ++i) {
            const uint32_t back = i + 1;   // the back-th most recent fill
            const uint32_t st = (idx + n - back % n) % n;
            const uint32_t ph = back > idx ? phase ^ 1 : phase;
            if (!mbar_wait_sleep(&full[st], ph, deadline)) return;
        }
    }
};

__device__ __forceinline__ void gemm_fail(GemmSmem *S, int *err) {
    S->abort = 1;
    atomicCAS(err, 0, kErrTimeout);
}

// Position of column `col` inside its 8-column group in the K order [0,4,1,5,2,6,3,7].
__host__ __device__ __forceinline__ int kperm_pos(int col) {
    const int j = col & 7;
    return (col & ~7) | (j < 4 ? 2 * j : 2 * (j - 4) + 1);
}

// State of one dequant thread across items: ring positions and its place in the CTA.
struct DqCtx {
    GemmSmem *S;
    uint8_t *sRaw, *sSc;
    int SR, grp, r;
    uint32_t tlane;          // TMEM lane of row r, first A-stage column
    uint64_t deadline;
    uint32_t *trace_a;       // trace rows for one thread, or nullptr
    Ring raw{kGemmMaxSlots}, sc{kGemmSS}, a{kGemmSA};
    uint32_t gstep = 0;      // steps seen so far (both groups): parity picks the group
};

__device__ __forceinline__ void dq_trace(const DqCtx &D, int row, uint32_t i) {
    if (D.trace_a != nullptr && blockIdx.x == 0 && i < (uint32_t)kTraceRow) {
        uint32_t c;
        asm volatile("mov.u32 %0, %%clock;" : "=r"(c));
        D.trace_a[row * kTraceRow + i] = c;
    }
}

// The step's A stage is free (the MMAs that read it have completed): lane 0 waits, the
// warp follows it.
__device__ __forceinline__ bool dq_wait_a_free(const DqCtx &D) {
    const int lane = threadIdx.x & 31;
    bool ok = true;
    if (lane == 0) ok = mbar_wait_sleep(&D.S->a_empty[D.a.idx], D.a.phase ^ 1, D.deadline);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    return ok;
}

// One pass over the steps [ks0, ks0 + kb) of an item, q4/q2 weights.
template <int kFmt, int kNMat, bool kSplit, bool kCM = false>
__device__ bool dq_run_q(DqCtx &D, const StepGeo &G, int ks0, bool lo) {
    GemmSmem *S = D.S;
    const int lane = threadIdx.x & 31;
    int lastw = -1;
    for (int j = 0; j < G.kb; ++j, ++D.gstep) {
        if ((int)(D.gstep & 1) != D.grp) {   // the other group's step: advance the rings
            D.raw.next();
            D.a.next();
            continue;
        }
        const int ks = ks0 + j;
        dq_trace(D, 10, D.a.count);
        if (!dq_wait_a_free(D)) return false;
        dq_trace(D, 11, D.a.count);
        const int si = D.grp * kGemmSS + D.sc.idx;
        if ((ks >> 3) != lastw) {
            lastw = ks >> 3;
            if (!__all_sync(0xffffffffu, mbar_wait_sleep(&S->sc_full[si], D.sc.phase, D.deadline))) return false;
        }
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(&S->raw_full[D.raw.idx], D.raw.phase, D.deadline))) return false;
        if (S->abort) return false;
        dq_trace(D, 2, D.a.count);
        const uint8_t *src = D.sRaw + D.raw.idx * kGemmSlot + (kCM ? 0 : D.r * G.rowb);
        const uint8_t *scp = D.sSc + si * 2 * kGemmScStage;
        const int sidx = kCM ? (ks & 7) * 128 + D.r : D.r * 8 + (ks & 7);
        const uint32_t ta = D.tlane + D.a.idx * kGemmACols;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            if (kSplit) dq_step_split<kFmt>(src, scp, sidx, ta + 16 * hh, hh, lo);
            else dq_step_q<kFmt, kNMat, kCM>(src, G.rawm, scp, sidx, ta + 16 * hh, hh, D.r);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        // last step of this group in the scale window: the group's next step is 2 on
        const bool rel_sc = ((ks + 2) >> 3) != (ks >> 3) || j + 2 >= G.kb;
        dq_trace(D, 3, D.a.count);
        if (lane == 0) {
            mbar_arrive(&S->a_full[D.a.idx]);
            mbar_arrive(&S->raw_empty[D.raw.idx]);
            if (rel_sc) mbar_arrive(&S->sc_empty[si]);
        }
        if (rel_sc) {
            D.sc.next();
            lastw = -1;
        }
        D.raw.next();
        D.a.next();
    }
    return true;
}

// One pass over an item's steps, bf16 weights (nslot raw slots a step; this thread's
// rows sit in slot r / rows-per-slot).
template <int kNMat>
__device__ bool dq_run_bf16(DqCtx &D, const StepGeo &G, int ks0, bool zero) {
    GemmSmem *S = D.S;
    const int lane = threadIdx.x & 31;
    const int rps = 128 / G.nslot, qs = D.r / rps;
    for (int j = 0; j < G.kb; ++j, ++D.gstep) {
        if ((int)(D.gstep & 1) != D.grp) {
            for (int k = 0; k < G.nslot; ++k) D.raw.next();
            D.a.next();
            continue;
        }
        if (!dq_wait_a_free(D)) return false;
        const uint32_t slot = D.raw.idx + qs < (uint32_t)D.SR ? D.raw.idx + qs : D.raw.idx + qs - D.SR;
        const uint32_t ph = D.raw.idx + qs < (uint32_t)D.SR ? D.raw.phase : D.raw.phase ^ 1;
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(&S->raw_full[slot], ph, D.deadline))) return false;
        if (S->abort) return false;
        const uint8_t *src = D.sRaw + slot * kGemmSlot + (D.r - qs * rps) * 128;
        const uint32_t ta = D.tlane + D.a.idx * kGemmACols;
        dq_step_bf16<kNMat>(src, G.rawm, ta, zero);
        dq_step_bf16<kNMat>(src + 64, G.rawm, ta + 16, zero);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive_n(&S->raw_empty[slot], 4 * 32 / rps);   // four arrivals complete a slot
            mbar_arrive(&S->a_full[D.a.idx]);
        }
        for (int k = 0; k < G.nslot; ++k) D.raw.next();
        D.a.next();
    }
    return true;
}

// One dequant pass of a problem whose (format, matrices, split) are compile-time: each
// kernel instantiation carries only the conversion code its problems use.
// Problem 0 of a single-matrix q-format non-split launch is the routed down product,
// whose weights are the column-major group slabs (kCM).
template <int kFmt, int kNMat, int kSplit, bool kCM = false>
__device__ __forceinline__ bool dq_pass(DqCtx &D, const StepGeo &G, int ks0, bool lo) {
    if constexpr (kFmt == kAFmtBf16) return dq_run_bf16<kNMat>(D, G, ks0, kSplit && lo);
    else return dq_run_q<kFmt, kNMat, kSplit != 0, kCM && kNMat == 1 && kSplit == 0>(D, G, ks0, lo);
}

// Template parameters: (format, matrices, split) of problem 0 and of problem 1.
template <int F0, int M0, int S0, int F1, int M1, int S1>
__global__ void __launch_bounds__(kGemmThreads, 1) k_moe_gemm(const __grid_constant__ GemmParams P) {
    extern __shared__ __align__(1024) uint8_t smraw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
    uint8_t *sB = sm;                                  // kGemmSB x 16 KB
    uint8_t *sSc = sB + kGemmSB * kGemmBStage;         // 2 groups x kGemmSS x 2 x 4 KB
    uint8_t *sRaw = sSc + 2 * kGemmSS * 2 * kGemmScStage;  // sr x 8 KB
    uint8_t *sEpi = sRaw + P.sr * kGemmSlot;               // kGemmEpiStage
    GemmSmem *S = reinterpret_cast<GemmSmem *>(sEpi + kGemmEpiStage);
    const int SR = P.sr;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t deadline = globaltimer_ns() + P.timeout_ns;

    if (tid == 0) {
        for (int i = 0; i < SR; ++i) { mbar_init(&S->raw_full[i], 1); mbar_init(&S->raw_empty[i], 4); }
        for (int i = 0; i < 2 * kGemmSS; ++i) { mbar_init(&S->sc_full[i], 1); mbar_init(&S->sc_empty[i], 4); }
        // a_empty / acc_full: one commit from each of the two MMA issuers
        // a_full: four dequant warps + the B loader's expect_tx (its TMA tiles complete on
        // the same barrier), so a full stage has its A rows in TMEM and its B tile landed
        for (int i = 0; i < kGemmSA; ++i) { mbar_init(&S->a_full[i], 5); mbar_init(&S->a_empty[i], 2); }
        for (int i = 0; i < 2; ++i) { mbar_init(&S->acc_full[i], 2); mbar_init(&S->acc_empty[i], 4); }
        mbar_init(&S->drain[0], 1);
        mbar_init(&S->drain[1], 1);
        S->abort = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&S->tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    gemm_build_tables(P, &S->T, warp >= 2 ? warp - 2 : kGemmMaxProblems, lane);
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
            Ring raw(SR), sc0(kGemmSS), sc1(kGemmSS);
            uint32_t gstep = 0;   // steps issued so far: step parity picks the dequant group
            bool ok = true;
            for (int it = blockIdx.x; it < n_items && ok && !S->abort; it += gridDim.x) {
                const GemmItem w = gemm_item(P, &S->T, it);
                const GemmProblem &pr = P.prob[w.p];
                const StepGeo G = step_geo(pr.fmt, pr.n_mat, pr.K, pr.ksplit);
                const bool q = pr.fmt != kAFmtBf16;
                const int npass = __popc(pr.passes), ks0 = w.sp * G.kb;
                for (int ps = 0; ps < npass && ok; ++ps) {
                    int lastw[2] = {-1, -1};   // scale window last loaded for each group
                    for (int j = 0; j < G.kb; ++j, ++gstep) {
                        const int ks = ks0 + j, grp = gstep & 1;
                        if (q) {
                            if ((ks >> 3) != lastw[grp]) {
                                lastw[grp] = ks >> 3;
                                Ring &sc = grp ? sc1 : sc0;
                                const int si = grp * kGemmSS + sc.idx;
                                if (!mbar_wait_sleep(&S->sc_empty[si], sc.phase ^ 1, deadline)) { ok = false; break; }
                                mbar_arrive_expect_tx(&S->sc_full[si], pr.n_mat * kGemmScStage);
                                for (int m = 0; m < pr.n_mat; ++m) {
                                    uint8_t *d = sSc + (si * 2 + m) * kGemmScStage;
                                    if (pr.a_cm) {
                                        tma_load_4d(d, &pr.ts[m], w.mt * 128, 0, ks & ~7, w.e, &S->sc_full[si]);
                                        tma_load_4d(d + 2048, &pr.tb[m], w.mt * 128, 0, ks & ~7, w.e, &S->sc_full[si]);
                                    } else {
                                        tma_load_4d(d, &pr.ts[m], ks & ~7, 0, w.mt * 8, w.e, &S->sc_full[si]);
                                        tma_load_4d(d + 2048, &pr.tb[m], ks & ~7, 0, w.mt * 8, w.e, &S->sc_full[si]);
                                    }
                                }
                                sc.next();
                            }
                            if (!mbar_wait_sleep(&S->raw_empty[raw.idx], raw.phase ^ 1, deadline)) { ok = false; break; }
                            trace_put(P, 0, raw.count);
                            mbar_arrive_expect_tx(&S->raw_full[raw.idx], pr.n_mat * G.rawm);
                            for (int m = 0; m < pr.n_mat; ++m) {
                                if (pr.a_cm)
                                    tma_load_4d(sRaw + raw.idx * kGemmSlot, &pr.tw[m], w.mt * 128, 0, ks, w.e,
                                                &S->raw_full[raw.idx]);
                                else
                                    tma_load_4d(sRaw + raw.idx * kGemmSlot + m * G.rawm, &pr.tw[m], ks * G.wpk, 0,
                                                w.mt * 8, w.e, &S->raw_full[raw.idx]);
                            }
                            raw.next();
                        } else {
                            const int bands = 8 / G.nslot;
                            for (int qs = 0; qs < G.nslot; ++qs) {
                                if (!mbar_wait_sleep(&S->raw_empty[raw.idx], raw.phase ^ 1, deadline)) { ok = false; break; }
                                mbar_arrive_expect_tx(&S->raw_full[raw.idx], kGemmSlot);
                                for (int m = 0; m < pr.n_mat; ++m)
                                    tma_load_4d(sRaw + raw.idx * kGemmSlot + m * G.rawm, &pr.tw[m], ks * 64, 0,
                                                w.mt * 8 + qs * bands, w.e, &S->raw_full[raw.idx]);
                                raw.next();
                            }
                            if (!ok) break;
                        }
                    }
                }
            }
            if (!ok) gemm_fail(S, P.err);
            // drain: the last fill of every slot has landed before the CTA may exit
            raw.drain(S->raw_full, deadline);
            sc0.drain(S->sc_full, deadline);
            sc1.drain(S->sc_full + kGemmSS, deadline);
        } else if (lane == 1 && P.trace != nullptr && blockIdx.x == 0) {
            // diagnostics only: record when each raw slot's data lands
            Ring raw(SR);
            for (int it = blockIdx.x; it < n_items && !S->abort; it += gridDim.x) {
                const GemmItem w = gemm_item(P, &S->T, it);
                const GemmProblem &pr = P.prob[w.p];
                const StepGeo G = step_geo(pr.fmt, pr.n_mat, pr.K, pr.ksplit);
                const int slots = __popc(pr.passes) * G.kb * G.nslot;
                for (int q = 0; q < slots; ++q) {
                    if (!mbar_wait_sleep(&S->raw_full[raw.idx], raw.phase, deadline)) break;
                    trace_put(P, 7, raw.count);
                    raw.next();
                }
            }
        }
    } else if (warp == 1 || warp == 3) {
        // ------------------------------------------------ MMA issuers ----
        // A thread issues ~one tcgen05.mma every 46 cycles, so two threads share the work:
        // warp 1 issues matrix 0 (gate), warp 3 matrix 1 (up). Both commit every stage
        // release; for single-matrix problems warp 3 only adds its arrivals.
        const int mat = warp == 1 ? 0 : 1;
        if (lane == 0) {
            Ring a(kGemmSA);
            uint32_t tile = 0;
            bool issued = false, ok = true;
            for (int it = blockIdx.x; it < n_items && ok && !S->abort; it += gridDim.x, ++tile) {
                const GemmItem w = gemm_item(P, &S->T, it);
                const GemmProblem &pr = P.prob[w.p];
                const StepGeo G = step_geo(pr.fmt, pr.n_mat, pr.K, pr.ksplit);
                const int steps = __popc(pr.passes) * G.kb;
                const bool mine = mat < pr.n_mat;
                const int ab = tile % P.acc_bufs;
                if (!mbar_wait_sleep(&S->acc_empty[ab], ((tile / P.acc_bufs) & 1) ^ 1, deadline)) { ok = false; break; }
                tc_fence_after();
                const uint32_t idesc = idesc_bf16((w.n + 15) & ~15);
                const uint32_t d = tmem + ab * 128 + mat * 128;   // this issuer's accumulator
                for (int s = 0; s < steps; ++s) {
                    // a_full: the A rows are in TMEM and the B tile has landed
                    if (!mbar_wait_sleep(&S->a_full[a.idx], a.phase, deadline)) { ok = false; break; }
                    tc_fence_after();
                    if (mat == 0) trace_put(P, 8, a.count);
                    if (mine) {
                        const uint64_t bd = sw128_desc(smem_u32(sB + a.idx * kGemmBStage));
                        const uint32_t a0 = tmem + kGemmAccCols + a.idx * kGemmACols + mat * 32;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) tc_mma_ts(d, a0 + 8 * kk, bd + 2 * kk, idesc, (s | kk) ? 1u : 0u);
                        issued = true;
                    }
                    tc_commit(&S->a_empty[a.idx]);   // frees the A and the B stage
                    if (mat == 0) trace_put(P, 4, a.count);
                    a.next();
                }
                if (!ok) break;
                tc_commit(&S->acc_full[ab]);
            }
            if (!ok) gemm_fail(S, P.err);
            if (issued) {   // every MMA this thread issued has completed before TMEM is freed
                tc_commit(&S->drain[mat]);
                mbar_wait_sleep(&S->drain[mat], 0, deadline + 100000000ull);
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------ B loader (TMA, 16-row tiles) ----
        if (lane == 0) {
            Ring b(kGemmSB);
            bool ok = true;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                const GemmItem w = gemm_item(P, &S->T, it);
                const GemmProblem &pr = P.prob[w.p];
                const StepGeo G = step_geo(pr.fmt, pr.n_mat, pr.K, pr.ksplit);
                const int npass = __popc(pr.passes), ks0 = w.sp * G.kb;
                const int nt = (w.n + 15) >> 4, row0 = pr.in_base + w.pos0;
                for (int ps = 0; ps < npass && ok; ++ps) {
                    const CUtensorMap *map = &pr.tx[gemm_pass(pr.passes, ps) == 1 ? 1 : 0];
                    for (int j = 0; j < G.kb; ++j) {
                        if (!mbar_wait_sleep(&S->a_empty[b.idx], b.phase ^ 1, deadline) || S->abort) { ok = false; break; }
                        uint8_t *dst = sB + b.idx * kGemmBStage;
                        trace_put(P, 1, b.count);
                        mbar_arrive_expect_tx(&S->a_full[b.idx], nt * 2048);
                        for (int i = 0; i < nt; ++i)
                            tma_load_2d(dst + i * 2048, map, (ks0 + j) * 64, row0 + 16 * i, &S->a_full[b.idx]);
                        b.next();
                    }
                }
            }
            if (!ok) gemm_fail(S, P.err);
            b.drain(S->a_full, deadline);
        }
    } else if (warp < 12) {
        // ------------------------------------------------ dequant (2 x 128 threads) ----
        // Two groups of four warps take alternate steps, so one group's barrier waits
        // overlap the other's conversion. A thread converts one full row of a step.
        const int grp = (warp - 4) >> 2, r = 32 * (warp & 3) + lane;
        DqCtx D;
        D.S = S;
        D.sRaw = sRaw;
        D.sSc = sSc;
        D.SR = SR;
        D.grp = grp;
        D.r = r;
        D.tlane = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + kGemmAccCols;
        D.deadline = deadline;
        D.trace_a = (warp == 4 && lane == 0) ? P.trace : nullptr;
        D.raw.n = (uint32_t)SR;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const GemmItem w = gemm_item(P, &S->T, it);
            const GemmProblem &pr = P.prob[w.p];
            const StepGeo G = step_geo(pr.fmt, pr.n_mat, pr.K, pr.ksplit);
            const int npass = __popc(pr.passes), ks0 = w.sp * G.kb;
            for (int ps = 0; ps < npass && ok; ++ps) {
                const bool lo = gemm_pass(pr.passes, ps) == 2;
                ok = w.p == 0 ? dq_pass<F0, M0, S0, true>(D, G, ks0, lo) : dq_pass<F1, M1, S1>(D, G, ks0, lo);
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
            const int ab = tile % P.acc_bufs;
            const bool ok = __all_sync(0xffffffffu, mbar_wait_sleep(&S->acc_full[ab], (tile / P.acc_bufs) & 1, deadline));
            if (!ok || S->abort) {
                if (!ok && lane == 0) gemm_fail(S, P.err);
                break;
            }
            tc_fence_after();
            if (tid == 384) trace_put(P, 5, tile);
            const int m = w.mt * 128 + row;
            const uint32_t tbase = tmem + ((uint32_t)(32 * eq) << 16) + ab * 128;
            const int obase = pr.out_base + w.sp * pr.split_rows + w.pos0;
            if (pr.epi == kEpiSwiGLU) {
                // 32 tokens a round: one wait per 64 columns read (gate and up). SiLU(g) * u
                // with the hardware exponential and reciprocal (a few ulp of fp32; the result
                // is rounded to bf16): one epilogue warp per sub-partition runs this for every
                // token, and the IEEE division and expf (tens of instructions each) had made
                // the epilogue as long as the item's main loop. All 32 values are computed
                // before any store, with no branch between them, so their latencies overlap.
                uint16_t *o = static_cast<uint16_t *>(pr.out);
                const int cbase = w.mt * 128 + 32 * eq;           // the warp's 32 act columns
                const int lcol = kperm_pos(m) - cbase;            // this lane's, K-permuted
                for (int c0 = 0; c0 < w.n; c0 += 32) {
                    uint32_t g[32], u[32];
                    if (tid == 384) trace_put(P, 9, 8 * tile + 2 * (c0 >> 5));
                    tc_ld32(tbase + c0, g);
                    tc_ld32(tbase + 128 + c0, u);
                    tc_wait_ld();
                    if (tid == 384) trace_put(P, 9, 8 * tile + 2 * (c0 >> 5) + 1);
                    const int nc = min(32, w.n - c0);
                    uint32_t av[16];
#pragma unroll
                    for (int jj = 0; jj < 32; jj += 2) {
                        const float g0 = __uint_as_float(g[jj]), u0 = __uint_as_float(u[jj]);
                        const float g1 = __uint_as_float(g[jj + 1]), u1 = __uint_as_float(u[jj + 1]);
                        av[jj / 2] = pack_bf16x2(__fdividef(g0, 1.f + __expf(-g0)) * u0,
                                                 __fdividef(g1, 1.f + __expf(-g1)) * u1);
                    }
                    // through shared memory, so that each store is 16 bytes of one token's
                    // row instead of 2 bytes: the warp's [32 tokens][32 columns] tile
                    uint16_t *tile16 = reinterpret_cast<uint16_t *>(sEpi + eq * 2048);
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) tile16[jj * 32 + lcol] = (uint16_t)(av[jj / 2] >> (16 * (jj & 1)));
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int q = lane + 32 * i, tk = q >> 2, part = q & 3;
                        if (tk < nc) {
                            const uint4 v = *reinterpret_cast<const uint4 *>(tile16 + tk * 32 + part * 8);
                            *reinterpret_cast<uint4 *>(o + (size_t)(obase + c0 + tk) * pr.ld_out + cbase + part * 8) = v;
                        }
                    }
                    __syncwarp();
                }
            }
            if (pr.epi == kEpiBf16) {
                // 32 tokens a round through shared memory: 16-byte stores of one token's row
                // (a peer's memory under expert parallelism: 2-byte stores over NVLink were
                // the slow part of an earlier version)
                const int cbase = w.mt * 128 + 32 * eq;
                uint16_t *dst0;
                if (pr.ret_meta != nullptr) {
                    const int r = w.g / pr.slab_groups;
                    dst0 = reinterpret_cast<uint16_t *>(pr.ret_base[r]) +
                           (size_t)(pr.ret_meta[r] + w.pos0 - r * pr.slab_rows) * pr.ld_out;
                } else {
                    dst0 = static_cast<uint16_t *>(pr.out) + (size_t)obase * pr.ld_out;
                }
                uint16_t *tile16 = reinterpret_cast<uint16_t *>(sEpi + eq * 2048);
                for (int c0 = 0; c0 < w.n; c0 += 32) {
                    uint32_t g[32];
                    tc_ld32(tbase + c0, g);
                    tc_wait_ld();
                    const int nc = min(32, w.n - c0);
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj)
                        tile16[jj * 32 + lane] = (uint16_t)(pack_bf16x2(__uint_as_float(g[jj]), 0.f) & 0xFFFFu);
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int q = lane + 32 * i, tk = q >> 2, part = q & 3;
                        if (tk < nc) {
                            const uint4 v = *reinterpret_cast<const uint4 *>(tile16 + tk * 32 + part * 8);
                            *reinterpret_cast<uint4 *>(dst0 + (size_t)(c0 + tk) * pr.ld_out + cbase + part * 8) = v;
                        }
                    }
                    __syncwarp();
                }
            }
            for (int c0 = 0; pr.epi == kEpiF32 && c0 < w.n; c0 += 8) {
                uint32_t g[8], u[8];
                tc_ld8(tbase + c0, g);
                if (pr.n_mat == 2) tc_ld8(tbase + 128 + c0, u);
                tc_wait_ld();
                const int nc = min(8, w.n - c0);
                float *o = static_cast<float *>(pr.out);
#pragma unroll
                for (int jj = 0; jj < 8; ++jj)
                    if (jj < nc) {
                        o[(size_t)(obase + c0 + jj) * pr.ld_out + m] = __uint_as_float(g[jj]);
                        if (pr.n_mat == 2)
                            o[(size_t)(obase + c0 + jj) * pr.ld_out + pr.mat_col + m] = __uint_as_float(u[jj]);
                    }
            }
            tc_fence_before();
            __syncwarp();
            if (tid == 384) trace_put(P, 6, tile);
            if (lane == 0) mbar_arrive(&S->acc_empty[ab]);
        }
        // rows written to peers' return buffers: visible system-wide before the kernel
        // ends (the signal kernel that follows announces them)
        if (P.prob[0].ret_meta != nullptr) __threadfence_system();
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
