// nmoe_batched.cu -- the T-token routed-MoE block: nmoe_moe_forward_batched.
//
// The reference runs prefill token by token through the batch-1 kernels
// (src/runtime.m:3816); this path computes the same block for T tokens at once:
//
//   k_prep      x -> bf16 hi (and lo, for f32 x) planes in the K order of the GEMM
//   GEMM        router logits [T][256] (hi/lo split operands: fp32-accurate), K-slice
//               partial sums when T is small so that the router spreads over the SMs
//   k_route     per token: top-k of 256 + renormalised weights (src/runtime.m:1498-1511),
//               shared-gate score, per-expert counts and ranks
//   k_scatter   positions: tokens grouped by expert (offset[e] + rank)
//   GEMM        gate/up + SwiGLU for every (token, expert) position -> act; the shared
//               expert's gate/up over all T tokens as K-slice partials
//   k_shared_act  shared SiLU(gate) * up -> act
//   GEMM        down -> Y per routed position; shared down as K-slice partials
//   k_combine   out = h_mid + sum_s w_s Y[pos(t,s)] + sigmoid(score) * Y[shared(t)]
//               (nmoe_expert_down_combine_q4, metal/kernels.metal:1497-1541)
// Every launch is asynchronous on the caller's stream; nothing is allocated per call.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include <nccl.h>

#include "nmoe_batched.cuh"
#include "nmoe_gemm.cuh"
#include "nmoe_pack.cuh"
#include "nmoe_topk.cuh"

using namespace nmoe;

namespace nmoe {

struct BatchedState {
    int t_max = 0;
    uint16_t *xh = nullptr, *xl = nullptr;   // [t_max][2048] K-permuted bf16 planes
    uint16_t *xp = nullptr;                  // [t_max * 8][2048] xh rows in position order
    float *logits = nullptr;                 // [t_max][256]
    float *score = nullptr;                  // [t_max]
    float *w = nullptr;                      // [t_max][8]
    uint32_t *idx = nullptr;                 // [t_max][8]
    int *rank = nullptr, *inv = nullptr;     // [t_max][8]
    int *perm = nullptr;                     // [t_max * 8]
    int *cnt = nullptr;                      // [256]
    int *eoff = nullptr;                     // [256] first position of each expert's rows
    uint16_t *act = nullptr;                 // [t_max * 9][512]  (routed positions, then shared)
    uint16_t *y = nullptr;                   // [t_max * 8][2048] routed down outputs
    int rows_cap = 0;                        // rows of each partial-sum buffer
    float *p_router = nullptr;               // [rows_cap][256]   router K-slice partials
    float *p_sgu = nullptr;                  // [rows_cap][1024]  shared gate|up partials
    float *p_sdown = nullptr;                // [rows_cap][2048]  shared down partials
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    uint64_t timeout_ns = 1000000000ull;
    int last_T = 0;
    int trace_launch = -1;                   // NMOE_GEMM_TRACE=<0 router | 1 gate/up | 2 down>
    uint32_t *trace = nullptr;               // [kTraceRows][1024]
    int launch_no = 0;
};

// Expert parallelism (world_size > 1): this rank holds experts [expert_lo, expert_lo +
// n_local) and exchanges token rows with the other ranks by NVLink peer stores into a
// symmetric arena that every rank maps (CUDA IPC). Per call, on the device only:
//   dispatch: rows go into slab `rank` of each destination's xr (fixed capacity C =
//             t_max * k_max rows, so no sizes travel to the host first), with the counts
//             per local expert and this rank's segment offset; a flag with the call's tag
//             follows the rows;
//   wait:     the receiver waits (bounded) for every source's flag;
//   compute:  the grouped GEMMs read the slabs (groups (source, local expert));
//   return:   down outputs go back into the source's yret, at the positions the rows left
//             from; a second flag follows; the source waits for every receiver's flag and
//             combines.
// Calls alternate between two sets of buffers: a rank writes set (call & 1) of a peer only
// after that peer returned this rank's rows of the call two back, so nothing overwrites
// data still being read.
constexpr int kEpMaxWorld = 8;
static_assert(kEpMaxWorld <= kGemmMaxPeers, "GEMM return pointers per rank");
struct EpLayout {              // offsets inside each rank's arena
    size_t flags;              // arrive[kEpMaxWorld], ret[kEpMaxWorld]: u32, 64 bytes apart
    size_t rcnt;               // [2][W][n_local] int: rows per (source, local expert)
    size_t rmeta;              // [2][W] int: the source's position of its first row here
    size_t xr;                 // [2][W][C][2048] bf16: received rows, slab per source
    size_t yret;               // [2][C][2048] bf16: this rank's rows' down outputs, position order
    size_t total;
};
struct EpState {
    ncclComm_t comm = nullptr;   // set-up only (handle exchange, barriers)
    int world = 1, rank = 0;
    size_t C = 0;                // slab rows: t_max * k_max
    EpLayout L{};
    uint8_t *arena = nullptr;    // this rank's arena (exported)
    uint8_t *peer[kEpMaxWorld] = {};   // every rank's arena as mapped here (peer[rank] = arena)
    uint8_t **d_peer = nullptr;  // device copy of peer[]
    uint16_t *yr = nullptr;      // [W * C][2048] down outputs of the received rows (slab order)
    int return_kernel = 0;       // NMOE_EP_RETURN_KERNEL=1: a separate return kernel instead of
                                 // the down epilogue's peer stores
    unsigned *done = nullptr;    // [2] grid completion counters (dispatch, return)
    uint32_t call = 0;           // calls so far; the tag of a call is call + 1
    bool timing = false;         // NMOE_EP_TIMING=1: events around the exchanges
    cudaEvent_t ev[4] = {};
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
    const float *part;        // router partial sums [nsplit][T][256]
    int nsplit;
    float *logits;            // their sum [T][256]
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
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int sp = 0; sp < a.nsplit; ++sp) {   // K slices summed in a fixed order
        const float4 *lg = reinterpret_cast<const float4 *>(a.part + ((size_t)sp * a.T + t) * kExperts + 8 * lane);
        const float4 l0 = lg[0], l1 = lg[1];
        v[0] += l0.x; v[1] += l0.y; v[2] += l0.z; v[3] += l0.w; v[4] += l1.x; v[5] += l1.y; v[6] += l1.z; v[7] += l1.w;
    }
    float4 *lo = reinterpret_cast<float4 *>(a.logits + (size_t)t * kExperts + 8 * lane);
    lo[0] = make_float4(v[0], v[1], v[2], v[3]);
    lo[1] = make_float4(v[4], v[5], v[6], v[7]);
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
                          int n_local, int *perm, int *inv, int *eoff) {
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
    if (blockIdx.x == 0 && eoff) eoff[tid] = off[tid];   // first position of each expert's rows
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

// xp[pos] = xh[perm[pos]]: each routed token's row at its position, 16 bytes a thread.
// Positions past the routed total (possible only after an out-of-range expert id) copy
// a stale but in-range row that no item reads.
__global__ void k_gather_rows(const uint16_t *xh, const int *perm, int T, int k, uint16_t *xp) {
    const int pos = blockIdx.x, c = threadIdx.x;
    if (pos >= T * k) return;
    reinterpret_cast<uint4 *>(xp + (size_t)pos * kHidden)[c] =
        reinterpret_cast<const uint4 *>(xh + (size_t)perm[pos] * kHidden)[c];
}

// Shared expert: act[shared_base + t] = SiLU(gate) * up from the K-slice partial sums
// [nsplit][T][gate 512 | up 512], written in the GEMM's K order.
__global__ void k_shared_act(const float *part, int nsplit, int T, uint16_t *act, int shared_base) {
    // four lanes per (token, 8-row group) share the K slices, then add in a fixed order
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int q = i & 3, grp = i >> 2;
    const bool live = grp < T * (kInter / 8);
    const int t = live ? grp / (kInter / 8) : 0, j0 = live ? (grp % (kInter / 8)) * 8 : 0;
    float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, u[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) {
#pragma unroll 4
        for (int sp = q; sp < nsplit; sp += 4) {
            const float4 *r = reinterpret_cast<const float4 *>(part + ((size_t)sp * T + t) * (2 * kInter) + j0);
            const float4 a = r[0], b = r[1], c = r[kInter / 4], d = r[kInter / 4 + 1];
            g[0] += a.x; g[1] += a.y; g[2] += a.z; g[3] += a.w; g[4] += b.x; g[5] += b.y; g[6] += b.z; g[7] += b.w;
            u[0] += c.x; u[1] += c.y; u[2] += c.z; u[3] += c.w; u[4] += d.x; u[5] += d.y; u[6] += d.z; u[7] += d.w;
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        g[j] += __shfl_xor_sync(0xffffffffu, g[j], 1);
        u[j] += __shfl_xor_sync(0xffffffffu, u[j], 1);
        g[j] += __shfl_xor_sync(0xffffffffu, g[j], 2);
        u[j] += __shfl_xor_sync(0xffffffffu, u[j], 2);
    }
    if (!live || q != 0) return;
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = g[j] / (1.f + expf(-g[j])) * u[j];
    // K order [0,4,1,5,2,6,3,7]
    reinterpret_cast<uint4 *>(act + (size_t)(shared_base + t) * kInter + j0)[0] =
        make_uint4(pack_bf16x2(a[0], a[4]), pack_bf16x2(a[1], a[5]), pack_bf16x2(a[2], a[6]), pack_bf16x2(a[3], a[7]));
}

// out[t][c..c+8) = h_mid + sum_s w_s * Y[pos(t,s)] + sigmoid(score_t) * shared_down(t), the
// shared down from its K-slice partial sums [nsplit][T][2048].
__global__ void k_combine(const uint16_t *y, const float *w, const int *inv, const float *score, const float *h_mid,
                          const float *sdown, int nsplit, int T, int k, void *out, int out_bf16) {
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
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int sp = 0; sp < nsplit; ++sp) {
        const float4 *r = reinterpret_cast<const float4 *>(sdown + ((size_t)sp * T + t) * kHidden + c);
        const float4 a = r[0], b = r[1];
        o[0] += a.x; o[1] += a.y; o[2] += a.z; o[3] += a.w; o[4] += b.x; o[5] += b.y; o[6] += b.z; o[7] += b.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] *= sg;
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

// ------------------------------------------------------ expert parallelism ----

__device__ __forceinline__ void st_release_sys_u32(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct EpArgs {
    uint8_t *const *peer;        // arenas of every rank
    EpLayout L;
    int world, rank, n_local, set;
    size_t C;
    uint32_t tag;
    unsigned *done;
};

// The last block of a grid to finish (after every block's stores, made visible system-wide)
// raises flag `which` (0 arrive, 1 ret) of this rank in every peer's arena.
__device__ __forceinline__ void ep_signal_last(const EpArgs &a, int which, unsigned *done) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0;
            __threadfence_system();
            for (int p = 0; p < a.world; ++p)
                st_release_sys_u32(reinterpret_cast<uint32_t *>(a.peer[p] + a.L.flags) + (which * kEpMaxWorld + a.rank) * 16,
                                   a.tag);
        }
    }
}

// Dispatch: rows (t, s) of xh (grid-stride, one row per block iteration) go into slab
// `rank` of the owner of their expert, at (position - first position of that owner's
// experts, eoff); blocks b < world also write that destination's counts and this rank's
// segment offset. Grid: at least `world` blocks of 256 threads.
__global__ void __launch_bounds__(256) k_ep_dispatch(EpArgs a, const uint16_t *xh, const uint32_t *idx,
                                                     const int *inv, const int *cnt, const int *eoff, int T, int k) {
    const int tid = threadIdx.x, nl = a.n_local;
    for (int q = blockIdx.x; q < T * k; q += gridDim.x) {
        const int t = q / k, s = q - t * k;
        const int pos = inv[(size_t)t * kMaxK + s];
        if (pos < 0) continue;
        const int p = (int)idx[(size_t)t * kMaxK + s] / nl;
        const size_t row = ((size_t)a.set * a.world + a.rank) * a.C + (size_t)(pos - eoff[p * nl]);
        uint4 *dst = reinterpret_cast<uint4 *>(a.peer[p] + a.L.xr) + row * (kHidden / 8);
        dst[tid] = reinterpret_cast<const uint4 *>(xh + (size_t)t * kHidden)[tid];
    }
    const int b = blockIdx.x;
    if (b < a.world) {
        int *rc = reinterpret_cast<int *>(a.peer[b] + a.L.rcnt) + ((size_t)a.set * a.world + a.rank) * nl;
        if (tid < nl) rc[tid] = cnt[b * nl + tid];
        if (tid == 0) reinterpret_cast<int *>(a.peer[b] + a.L.rmeta)[a.set * a.world + a.rank] = eoff[b * nl];
    }
    ep_signal_last(a, 0, a.done);
}

// Raise this rank's flag `which` in every arena (one block; the stores it announces were
// made by earlier kernels on the stream, each fenced system-wide by its writer).
__global__ void k_ep_signal(EpArgs a, int which) {
    __threadfence_system();
    const int p = threadIdx.x;
    if (p < a.world)
        st_release_sys_u32(reinterpret_cast<uint32_t *>(a.peer[p] + a.L.flags) + (which * kEpMaxWorld + a.rank) * 16,
                           a.tag);
}

// Wait (bounded) until every rank's flag `which` in this rank's arena carries the tag.
__global__ void k_ep_wait(EpArgs a, int which, int *err, uint64_t timeout_ns) {
    const int p = threadIdx.x;
    if (p >= a.world) return;
    const uint32_t *f = reinterpret_cast<const uint32_t *>(a.peer[a.rank] + a.L.flags) + (which * kEpMaxWorld + p) * 16;
    const uint64_t deadline = globaltimer_ns() + timeout_ns;
    for (uint32_t it = 0;; ++it) {
        if ((int)(ld_acquire_sys_u32(f) - a.tag) >= 0) return;
        if (it >= kMaxSpins || globaltimer_ns() > deadline) {
            atomicCAS(err, 0, kErrTimeout);
            return;
        }
    }
}

// Return: every received row's down output (yr, slab order) goes back into its source's
// yret at the source's position; then the ret flags. Grid-stride over the received rows.
__global__ void __launch_bounds__(256) k_ep_return(EpArgs a, const uint16_t *yr) {
    __shared__ int tot[kEpMaxWorld + 1];
    __shared__ int meta[kEpMaxWorld];
    const int tid = threadIdx.x, nl = a.n_local;
    const int *rc = reinterpret_cast<const int *>(a.peer[a.rank] + a.L.rcnt) + (size_t)a.set * a.world * nl;
    if (tid < a.world) {
        int n = 0;
        for (int j = 0; j < nl; ++j) n += rc[tid * nl + j];
        tot[tid + 1] = n;
        meta[tid] = reinterpret_cast<const int *>(a.peer[a.rank] + a.L.rmeta)[a.set * a.world + tid];
    }
    if (tid == 0) tot[0] = 0;
    __syncthreads();
    if (tid == 0)
        for (int r = 0; r < a.world; ++r) tot[r + 1] += tot[r];
    __syncthreads();
    for (int q = blockIdx.x; q < tot[a.world]; q += gridDim.x) {
        int r = 0;
        while (q >= tot[r + 1]) ++r;
        const int i = q - tot[r];
        const uint4 *src = reinterpret_cast<const uint4 *>(yr + ((size_t)r * a.C + i) * kHidden);
        uint4 *dst = reinterpret_cast<uint4 *>(a.peer[r] + a.L.yret) + ((size_t)a.set * a.C + meta[r] + i) * (kHidden / 8);
        dst[tid] = src[tid];
    }
    ep_signal_last(a, 1, a.done + 1);
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

// 4D tiled map: (inner elements, 16 rows, bands, groups); box (box0, 16, box2, 1).
bool make_map(BatchedState *B, CUtensorMap *m, const void *base, bool u32, uint64_t d0, uint64_t row_stride,
              uint64_t bands, uint64_t band_stride, uint64_t groups, uint64_t group_stride, uint32_t box0,
              uint32_t box2 = 8) {
    const cuuint64_t dims[4] = {d0, 16, bands, groups};
    const cuuint64_t strides[3] = {row_stride, band_stride, group_stride};
    const cuuint32_t box[4] = {box0, 16, box2, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    const CUresult r = B->encode(m, u32 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 4,
                                 const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// B rows: 2D (K columns, rows) bf16, box 64 columns x 16 rows, 128B swizzle.
bool make_bmap(BatchedState *B, CUtensorMap *m, const uint16_t *base, int K, int rows) {
    if (base == nullptr) return true;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {64, 16};
    const cuuint32_t es[2] = {1, 1};
    return B->encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t *>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_bmaps(BatchedState *B, GemmProblem &pr, int rows) {
    return make_bmap(B, &pr.tx[0], pr.b_hi, pr.K, rows) && make_bmap(B, &pr.tx[1], pr.b_lo, pr.K, rows);
}

// Weight (+ scale/bias) maps of one q4/q2/bf16 matrix whose rows are `row_stride` bytes
// apart inside bands of 16 rows `band_stride` apart, groups (experts) `group_stride`
// apart. s_off/b_off: byte offsets of the scales / biases from `base`; their rows are
// s_row_stride bytes apart (the weight row stride for row-interleaved dense matrices).
bool make_matrix_maps(BatchedState *B, GemmProblem &pr, int m, const uint8_t *base, int fmt, int cols,
                      uint64_t row_stride, uint64_t bands, uint64_t band_stride, uint64_t groups, uint64_t group_stride,
                      size_t s_off, size_t b_off, uint64_t s_row_stride) {
    // box: one raw slot (step_geo): q formats sps steps x 128 rows, bf16 a block of rows
    const StepGeo G = step_geo(fmt, pr.n_mat, cols, 1);
    if (fmt == kAFmtBf16)
        return make_map(B, &pr.tw[m], base, false, cols, row_stride, bands, band_stride, groups, group_stride, 64,
                        8 / G.nslot);
    const int vpw = fmt == kAFmtQ4 ? 8 : 16;
    const int ng = cols / 64;
    return make_map(B, &pr.tw[m], base, true, cols / vpw, row_stride, bands, band_stride, groups, group_stride,
                    G.wpk * G.sps) &&
           make_map(B, &pr.ts[m], base + s_off, false, ng, s_row_stride, bands, band_stride, groups, group_stride, 8) &&
           make_map(B, &pr.tb[m], base + b_off, false, ng, s_row_stride, bands, band_stride, groups, group_stride, 8);
}

// Column-major maps of the routed down matrices (down group slabs, nmoe_pack.cuh):
// weights (2048 rows, wpg word columns, 8 slabs, experts), box 128 rows x wpg words;
// scales / biases (2048 rows, 1, 8 slabs, experts), box 128 rows x 8 slabs.
bool make_cm_maps(BatchedState *B, GemmProblem &pr, const uint8_t *down, const PackGeo &pg, int n_experts) {
    pr.a_cm = 1;
    {
        const cuuint64_t dims[4] = {2048, pg.wpg, 8, (cuuint64_t)n_experts};
        const cuuint64_t strides[3] = {2048 * 4, pg.dslab, pg.esz};
        const cuuint32_t box[4] = {128, pg.wpg, 1, 1};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        if (B->encode(&pr.tw[0], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, const_cast<uint8_t *>(down), dims, strides, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    for (int which = 0; which < 2; ++which) {
        const cuuint64_t dims[4] = {2048, 1, 8, (cuuint64_t)n_experts};
        const cuuint64_t strides[3] = {4096, pg.dslab, pg.esz};
        const cuuint32_t box[4] = {128, 1, 8, 1};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        CUtensorMap *m = which ? &pr.tb[0] : &pr.ts[0];
        if (B->encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<uint8_t *>(down + pg.dslab_w + which * 4096),
                      dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

// The kernel instantiation for the problems of a launch (see k_moe_gemm's parameters).
using GemmKernel = void (*)(const GemmParams);
#define NMOE_GEMM_KINDS(X)                                                      \
    X(kAFmtBf16, 1, 1, kAFmtBf16, 1, 1) X(kAFmtQ4, 1, 1, kAFmtQ4, 1, 1)           \
    X(kAFmtQ4, 2, 0, kAFmtBf16, 2, 0) X(kAFmtQ4, 2, 0, kAFmtQ4, 2, 0)             \
    X(kAFmtQ2, 2, 0, kAFmtBf16, 2, 0) X(kAFmtQ2, 2, 0, kAFmtQ4, 2, 0)             \
    X(kAFmtQ4, 1, 0, kAFmtBf16, 1, 0) X(kAFmtQ4, 1, 0, kAFmtQ4, 1, 0)             \
    X(kAFmtQ2, 1, 0, kAFmtBf16, 1, 0) X(kAFmtQ2, 1, 0, kAFmtQ4, 1, 0)

GemmKernel gemm_kernel(const GemmParams &P) {
    const GemmProblem &a = P.prob[0];
    const GemmProblem &b = P.n_prob > 1 ? P.prob[1] : P.prob[0];
    // a single problem reuses an instantiation whose second problem is never reached;
    // with two problems the shared expert is bf16 or q4
    const int bf = P.n_prob > 1 ? b.fmt : (a.split ? a.fmt : kAFmtBf16);
#define NMOE_GEMM_PICK(f0, m0, s0, f1, m1, s1)                                                   \
    if (a.fmt == f0 && a.n_mat == m0 && (a.split != 0) == (s0 != 0) && bf == f1)                 \
        return k_moe_gemm<f0, m0, s0, f1, m1, s1>;
    NMOE_GEMM_KINDS(NMOE_GEMM_PICK)
#undef NMOE_GEMM_PICK
    return nullptr;
}

cudaError_t launch_gemm(nmoe_moe_ctx *ctx, GemmParams &P, cudaStream_t st) {
    int sr = kGemmMaxSlots;
    while (sr > 2 && gemm_smem_bytes(sr) > (size_t)kGemmSmemMax) --sr;
    P.sr = sr;
    P.acc_bufs = 2;
    for (int i = 0; i < P.n_prob; ++i)
        if (P.prob[i].n_mat == 2) P.acc_bufs = 1;
    P.err = ctx->d_err;
    P.timeout_ns = ctx->batched->timeout_ns;
    BatchedState *B = ctx->batched;
    P.trace = (B->trace && B->launch_no == B->trace_launch) ? B->trace : nullptr;
    ++B->launch_no;
    const GemmKernel kern = gemm_kernel(P);
    if (kern == nullptr) return cudaErrorInvalidValue;
    kern<<<ctx->num_sms, kGemmThreads, gemm_smem_bytes(sr), st>>>(P);
    return cudaGetLastError();
}

// K slices for a dense problem over T tokens: enough items to cover the SMs, within
// the partial-sum buffer (rows_cap rows) and the slot geometry.
int pick_ksplit(int fmt, int n_mat, int K, int m_tiles, int T, int rows_cap, int target) {
    const int chunks = (T + kGemmNChunk - 1) / kGemmNChunk;
    int best = 1;
    for (int S = 2; S <= 32; S *= 2) {
        if ((K / 64) % S) break;
        const StepGeo G = step_geo(fmt, n_mat, K, S);
        if (G.kb < 1 || G.kb % G.sps || (long)S * T > rows_cap) break;
        if (m_tiles * chunks * best >= target) break;
        best = S;
    }
    return best;
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
    cudaError_t e = cudaSuccess;
#define NMOE_GEMM_ATTR(f0, m0, s0, f1, m1, s1)                                                           \
    if (e == cudaSuccess)                                                                                \
        e = cudaFuncSetAttribute(k_moe_gemm<f0, m0, s0, f1, m1, s1>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 kGemmSmemMax);
    NMOE_GEMM_KINDS(NMOE_GEMM_ATTR)
#undef NMOE_GEMM_ATTR
    if (e != cudaSuccess) {
        nmoe_ctx_set_error(ctx, "gemm smem attribute: %s", cudaGetErrorString(e));
        return NMOE_ECUDA;
    }
    if (const char *t = getenv("NMOE_GEMM_TRACE")) {
        B->trace_launch = atoi(t);
        if (cudaMalloc(&B->trace, kTraceRows * kTraceRow * 4) != cudaSuccess) B->trace = nullptr;
        else cudaMemset(B->trace, 0, kTraceRows * kTraceRow * 4);
    }
    const int tm = ctx->cfg.t_max;
    B->t_max = tm;
    if (tm <= 0) return NMOE_OK;
    const size_t T = (size_t)tm;
    B->rows_cap = std::max(4 * tm, 1024);
    const size_t R = (size_t)B->rows_cap;
    const int W = ctx->cfg.world_size;
    size_t act_rows = T * 9;
    if (W > 1) {
        if (W > kEpMaxWorld || kExperts / W < 8) {
            nmoe_ctx_set_error(ctx, "expert parallelism supports 2..%d ranks", kEpMaxWorld);
            return NMOE_EINVAL;
        }
        EpState *E = new (std::nothrow) EpState();
        if (E == nullptr) return NMOE_ENOMEM;
        ctx->ep = E;
        E->world = W;
        E->rank = ctx->cfg.rank;
        E->C = T * (size_t)ctx->cfg.k_max;
        ncclUniqueId id;
        memcpy(&id, ctx->cfg.nccl_unique_id, sizeof id);
        const ncclResult_t nr = ncclCommInitRank(&E->comm, W, id, E->rank);
        if (nr != ncclSuccess) {
            E->comm = nullptr;
            nmoe_ctx_set_error(ctx, "ncclCommInitRank: %s", ncclGetErrorString(nr));
            return NMOE_ENCCL;
        }
        const int nl = ctx->n_local;
        auto al256 = [](size_t v) { return (v + 255) & ~size_t(255); };
        EpLayout &L = E->L;
        L.flags = 0;
        L.rcnt = al256(2 * kEpMaxWorld * 64);
        L.rmeta = al256(L.rcnt + (size_t)2 * W * nl * 4);
        L.xr = al256(L.rmeta + (size_t)2 * W * 4);
        L.yret = al256(L.xr + (size_t)2 * W * E->C * kHidden * 2);
        L.total = al256(L.yret + (size_t)2 * E->C * kHidden * 2);
        act_rows = (size_t)W * E->C + T;
        e = cudaMalloc(&E->arena, L.total);
        if (e == cudaSuccess) e = cudaMemset(E->arena, 0, L.xr);   // flags, counts, offsets
        if (e == cudaSuccess) e = cudaMalloc(&E->yr, (size_t)W * E->C * kHidden * 2);
        if (e == cudaSuccess) e = cudaMalloc(&E->done, 2 * sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemset(E->done, 0, 2 * sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMalloc(&E->d_peer, kEpMaxWorld * sizeof(uint8_t *));
        if (e != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "expert-parallel buffers: %s", cudaGetErrorString(e));
            return e == cudaErrorMemoryAllocation ? NMOE_ENOMEM : NMOE_ECUDA;
        }
        // Every rank's (t_max, k_max, n_local) and arena handle, gathered once: the slabs have
        // one capacity on all ranks, so the sizes must agree (checked here, on every rank).
        struct Rec {
            int t_max, k_max, n_local, device;
            cudaIpcMemHandle_t h;
        };
        Rec mine{};
        mine.t_max = tm;
        mine.k_max = ctx->cfg.k_max;
        mine.n_local = nl;
        mine.device = ctx->device;
        if ((e = cudaIpcGetMemHandle(&mine.h, E->arena)) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
        Rec *d_recs = nullptr;
        std::vector<Rec> recs(W);
        e = cudaMalloc(&d_recs, sizeof(Rec) * W);
        if (e == cudaSuccess) e = cudaMemcpy(d_recs + E->rank, &mine, sizeof mine, cudaMemcpyHostToDevice);
        ncclResult_t gr = ncclSuccess;
        if (e == cudaSuccess) gr = ncclAllGather(d_recs + E->rank, d_recs, sizeof(Rec), ncclChar, E->comm, 0);
        if (e == cudaSuccess && gr == ncclSuccess) e = cudaMemcpy(recs.data(), d_recs, sizeof(Rec) * W, cudaMemcpyDeviceToHost);
        if (d_recs) cudaFree(d_recs);
        if (gr != ncclSuccess || e != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "expert-parallel set-up exchange: %s",
                               gr != ncclSuccess ? ncclGetErrorString(gr) : cudaGetErrorString(e));
            return gr != ncclSuccess ? NMOE_ENCCL : NMOE_ECUDA;
        }
        for (int p = 0; p < W; ++p)
            if (recs[p].t_max != tm || recs[p].k_max != ctx->cfg.k_max || recs[p].n_local != nl) {
                nmoe_ctx_set_error(ctx, "rank %d has t_max=%d k_max=%d, rank %d t_max=%d k_max=%d: expert parallelism "
                                   "needs the same t_max and k_max on every rank", p, recs[p].t_max, recs[p].k_max,
                                   E->rank, tm, ctx->cfg.k_max);
                return NMOE_EINVAL;
            }
        for (int p = 0; p < W; ++p) {
            if (p == E->rank) {
                E->peer[p] = E->arena;
                continue;
            }
            void *ptr = nullptr;
            if ((e = cudaIpcOpenMemHandle(&ptr, recs[p].h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) {
                nmoe_ctx_set_error(ctx, "cudaIpcOpenMemHandle (rank %d): %s", p, cudaGetErrorString(e));
                return NMOE_ECUDA;
            }
            E->peer[p] = static_cast<uint8_t *>(ptr);
        }
        if ((e = cudaMemcpy(E->d_peer, E->peer, kEpMaxWorld * sizeof(uint8_t *), cudaMemcpyHostToDevice)) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "expert-parallel peers: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
        if (const char *t = getenv("NMOE_EP_TIMING")) E->timing = atoi(t) != 0;
        if (const char *t = getenv("NMOE_EP_RETURN_KERNEL")) E->return_kernel = atoi(t) != 0;
        if (E->timing)
            for (auto &ev : E->ev) cudaEventCreate(&ev);
        // every rank has mapped every arena before any rank's first dispatch writes into one
        int *d_one = nullptr;
        e = cudaMalloc(&d_one, sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(d_one, 0, sizeof(int));
        if (e == cudaSuccess) gr = ncclAllReduce(d_one, d_one, 1, ncclInt32, ncclSum, E->comm, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (d_one) cudaFree(d_one);
        if (gr != ncclSuccess || e != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "expert-parallel set-up barrier failed");
            return gr != ncclSuccess ? NMOE_ENCCL : NMOE_ECUDA;
        }
    }
    struct { void **p; size_t bytes; } al[] = {
        {(void **)&B->xh, T * kHidden * 2},       {(void **)&B->xl, T * kHidden * 2},
        {(void **)&B->xp, T * kMaxK * kHidden * 2},
        {(void **)&B->logits, T * kExperts * 4},  {(void **)&B->score, T * 4},
        {(void **)&B->w, T * kMaxK * 4},          {(void **)&B->idx, T * kMaxK * 4},
        {(void **)&B->rank, T * kMaxK * 4},       {(void **)&B->inv, T * kMaxK * 4},
        {(void **)&B->perm, T * kMaxK * 4},       {(void **)&B->cnt, kExperts * 4},
        {(void **)&B->eoff, kExperts * 4},
        {(void **)&B->act, act_rows * kInter * 2}, {(void **)&B->y, T * 8 * kHidden * 2},
        {(void **)&B->p_router, R * kExperts * 4}, {(void **)&B->p_sgu, R * 2 * kInter * 4},
        {(void **)&B->p_sdown, R * kHidden * 4},
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
    void *ps[] = {B->xh,   B->xl,  B->xp,  B->logits, B->score, B->w,        B->idx,  B->rank,
                  B->inv,  B->perm, B->cnt, B->eoff,   B->act,   B->y,        B->p_router, B->p_sgu, B->p_sdown,
                  B->trace};
    for (void *p : ps)
        if (p) cudaFree(p);
    delete B;
    ctx->batched = nullptr;
    if (EpState *E = ctx->ep) {
        // no rank may still write into this arena: a barrier over all ranks before unmapping
        if (E->comm && E->d_peer) {
            int *d_one = nullptr;
            if (cudaMalloc(&d_one, sizeof(int)) == cudaSuccess) {
                cudaMemset(d_one, 0, sizeof(int));
                ncclAllReduce(d_one, d_one, 1, ncclInt32, ncclSum, E->comm, 0);
                cudaDeviceSynchronize();
                cudaFree(d_one);
            }
        }
        for (int p = 0; p < E->world; ++p)
            if (E->peer[p] && p != E->rank) cudaIpcCloseMemHandle(E->peer[p]);
        if (E->comm) ncclCommDestroy(E->comm);
        if (E->arena) cudaFree(E->arena);
        if (E->yr) cudaFree(E->yr);
        if (E->done) cudaFree(E->done);
        if (E->d_peer) cudaFree(E->d_peer);
        for (auto ev : E->ev)
            if (ev) cudaEventDestroy(ev);
        delete E;
        ctx->ep = nullptr;
    }
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
    EpState *E = ctx->ep;
    if (ctx->cfg.world_size > 1 && E == nullptr) {
        nmoe_ctx_set_error(ctx, "expert parallelism needs t_max > 0 at create");
        return NMOE_EINVAL;
    }
    B->last_T = T;
    B->launch_no = 0;
    if (T == 0 && E == nullptr) return NMOE_OK;   // with EP, the rank still serves its experts
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
    if (T > 0) k_prep<<<(T * 256 + 255) / 256, 256, 0, st>>>(x, xf32, T, B->xh, B->xl, B->cnt);
    else cudaMemsetAsync(B->cnt, 0, kExperts * sizeof(int), st);

    // K slices of the dense problems (router, shared gate/up, shared down)
    // a quarter of the SMs' worth of items: more K slices leave each item a step or two and
    // the consumers (k_route, k_shared_act, k_combine) more partials to add (measured)
    const int target = ctx->num_sms / 4;
    const int nsplit_r = pick_ksplit(rfmt, 1, kHidden, 2, T, B->rows_cap, target);
    const int nsplit_g = pick_ksplit(sfmt, 2, kHidden, 4, T, B->rows_cap, target);
    const int nsplit_d = pick_ksplit(sfmt, 1, kInter, 16, T, B->rows_cap, target);

    // 2. router logits (K-slice partials)
    if (T > 0) {
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
        r.out = B->p_router;
        r.ksplit = nsplit_r;
        r.split_rows = T;
        const uint8_t *rb = dense + DA.router;
        if (!make_matrix_maps(B, r, 0, rb, rfmt, kHidden, DA.rrow, 16, 16ull * DA.rrow, 1, 256ull * DA.rrow, 1024, 1088,
                              DA.rrow) ||
            !make_bmaps(B, r, B->t_max)) {
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
        a.part = B->p_router;
        a.nsplit = nsplit_r;
        a.logits = B->logits;
        a.x = x;
        a.x_f32 = xf32;
        a.gvec = dense + DA.gvec;
        a.gvec_q4 = sfmt == kAFmtQ4;
        a.T = T;
        a.k = k;
        a.num_experts = ctx->cfg.num_experts;
        // with EP every rank routes over all experts; positions then group the rows by
        // destination rank
        a.expert_lo = E ? 0 : ctx->expert_lo;
        a.n_local = E ? kExperts : ctx->n_local;
        a.idx = B->idx;
        a.w = B->w;
        a.score = B->score;
        a.rank = B->rank;
        a.cnt = B->cnt;
        a.idx_out = idx_out;
        a.w_out = w_out;
        a.err = ctx->d_err;
        if (T > 0) {
            k_route<<<(T + kRouteWarps - 1) / kRouteWarps, kRouteWarps * 32, 0, st>>>(a);
            k_scatter<<<(T * k + 255) / 256, 256, 0, st>>>(B->idx, B->rank, B->cnt, T, k, a.expert_lo, a.n_local,
                                                           B->perm, B->inv, B->eoff);
            if (E == nullptr) k_gather_rows<<<T * k, 256, 0, st>>>(B->xh, B->perm, T, k, B->xp);
        }
    }
    int shared_base = T * k;

    // 3b. expert parallelism: rows into the owners' slabs (peer stores), then wait for
    // every source's rows (all on the stream: no host synchronisation)
    EpArgs ea{};
    if (E != nullptr) {
        ea.peer = E->d_peer;
        ea.L = E->L;
        ea.world = E->world;
        ea.rank = E->rank;
        ea.n_local = ctx->n_local;
        ea.set = (int)(E->call & 1u);
        ea.C = E->C;
        ea.tag = E->call + 1u;
        ea.done = E->done;
        ++E->call;
        if (E->timing) cudaEventRecord(E->ev[0], st);
        if (T == 0) cudaMemsetAsync(B->eoff, 0, kExperts * sizeof(int), st);
        k_ep_dispatch<<<std::max(std::min(T * k, 16 * ctx->num_sms), E->world), 256, 0, st>>>(ea, B->xh, B->idx, B->inv,
                                                                                          B->cnt, B->eoff, T, k);
        k_ep_wait<<<1, 32, 0, st>>>(ea, 0, ctx->d_err, B->timeout_ns);
        if (E->timing) cudaEventRecord(E->ev[1], st);
        if ((e = cudaGetLastError()) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "token dispatch: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
        shared_base = (int)((size_t)E->world * E->C);
    }
    const int n_groups = E ? E->world * ctx->n_local : ctx->n_local;
    const int *gcnt = E ? reinterpret_cast<const int *>(E->arena + E->L.rcnt) + (size_t)ea.set * E->world * ctx->n_local
                        : B->cnt;
    const int group_mod = E ? ctx->n_local : 0;
    const uint16_t *xrows = E ? reinterpret_cast<const uint16_t *>(E->arena + E->L.xr) +
                                    (size_t)ea.set * E->world * E->C * kHidden
                              : B->xp;
    const size_t act_rows = E ? (size_t)E->world * E->C + (size_t)B->t_max : (size_t)B->t_max * 9;

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
        r.ksplit = 1;
        r.n_groups = n_groups;
        r.cnt = gcnt;
        r.group_mod = group_mod;
        r.slab_groups = E ? ctx->n_local : 0;
        r.slab_rows = E ? (int)E->C : 0;
        r.b_hi = xrows;
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
        s.ksplit = nsplit_g;
        s.n_groups = 1;
        s.cnt_const = T;
        s.b_hi = B->xh;
        s.passes = kPassHiHi;
        s.epi = kEpiF32;
        s.ld_out = 2 * kInter;
        if (T == 0) P.n_prob = 1;
        s.mat_col = kInter;
        s.split_rows = T;
        s.out = B->p_sgu;
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
        ok = ok && make_bmaps(B, r, E ? (int)(E->world * E->C) : kMaxK * B->t_max) && make_bmaps(B, s, B->t_max);
        if (!ok) {
            nmoe_ctx_set_error(ctx, "gate/up tensor maps");
            return NMOE_ECUDA;
        }
        if ((e = launch_gemm(ctx, P, st)) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "gate/up gemm launch: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
    }

    // shared expert activations from the gate/up partials
    if (T > 0)
        k_shared_act<<<(T * (kInter / 8) * 4 + 255) / 256, 256, 0, st>>>(B->p_sgu, nsplit_g, T, B->act, shared_base);

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
        r.ksplit = 1;
        r.n_groups = n_groups;
        r.cnt = gcnt;
        r.group_mod = group_mod;
        r.slab_groups = E ? ctx->n_local : 0;
        r.slab_rows = E ? (int)E->C : 0;
        r.b_hi = B->act;
        r.passes = kPassHiHi;
        r.epi = kEpiBf16;
        r.ld_out = kHidden;
        r.out = E ? E->yr : B->y;
        if (E != nullptr && !E->return_kernel) {
            // the down epilogue writes each output row into its source's return buffer
            r.ret_meta = reinterpret_cast<const int *>(E->arena + E->L.rmeta) + (size_t)ea.set * E->world;
            for (int p = 0; p < E->world; ++p)
                r.ret_base[p] = E->peer[p] + E->L.yret + (size_t)ea.set * E->C * kHidden * 2;
        }
        bool ok = make_cm_maps(B, r, experts + pg.gu_bytes, pg, ctx->n_local);
        GemmProblem &s = P.prob[1];
        s.fmt = sfmt;
        s.n_mat = 1;
        s.K = kInter;
        s.m_tiles = 16;
        s.ksplit = nsplit_d;
        s.n_groups = 1;
        s.cnt_const = T;
        s.in_base = shared_base;
        s.b_hi = B->act;
        s.passes = kPassHiHi;
        s.epi = kEpiF32;
        s.ld_out = kHidden;
        s.split_rows = T;
        s.out = B->p_sdown;
        if (T == 0) P.n_prob = 1;
        const uint64_t rs = DA.sdrow;
        ok = ok && make_matrix_maps(B, s, 0, dense + DA.sdown, sfmt, kInter, rs, 128, 16 * rs, 1, 2048 * rs, 256, 272, rs);
        ok = ok && make_bmaps(B, r, (int)act_rows) && make_bmaps(B, s, (int)act_rows);
        if (!ok) {
            nmoe_ctx_set_error(ctx, "down tensor maps");
            return NMOE_ECUDA;
        }
        if ((e = launch_gemm(ctx, P, st)) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "down gemm launch: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
    }

    // 5b. expert parallelism: down outputs back to their sources (peer stores), then wait
    // for every owner's returns
    const uint16_t *ysrc = B->y;
    if (E != nullptr) {
        if (E->timing) cudaEventRecord(E->ev[2], st);
        if (E->return_kernel) k_ep_return<<<16 * ctx->num_sms, 256, 0, st>>>(ea, E->yr);
        else k_ep_signal<<<1, 32, 0, st>>>(ea, 1);   // the down epilogue already wrote the rows
        k_ep_wait<<<1, 32, 0, st>>>(ea, 1, ctx->d_err, B->timeout_ns);
        if (E->timing) cudaEventRecord(E->ev[3], st);
        if ((e = cudaGetLastError()) != cudaSuccess) {
            nmoe_ctx_set_error(ctx, "combine exchange: %s", cudaGetErrorString(e));
            return NMOE_ECUDA;
        }
        if (T == 0) return NMOE_OK;
        ysrc = reinterpret_cast<const uint16_t *>(E->arena + E->L.yret) + (size_t)ea.set * E->C * kHidden;
    }

    // 6. combine
    k_combine<<<(T * 256 + 255) / 256, 256, 0, st>>>(ysrc, B->w, B->inv, B->score, h_mid, B->p_sdown, nsplit_d, T, k,
                                                     out, out_dtype == NMOE_DTYPE_BF16);
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

extern "C" int nmoe_moe_debug_gemm_trace(nmoe_moe_ctx *ctx, uint32_t *out, int n) {
    if (ctx == nullptr || ctx->batched == nullptr || ctx->batched->trace == nullptr || out == nullptr || n < 0 ||
        n > kTraceRows * kTraceRow) {
        if (ctx) nmoe_ctx_set_error(ctx, "debug_gemm_trace: tracing is off (NMOE_GEMM_TRACE) or bad arguments");
        return NMOE_EINVAL;
    }
    Guard guard(ctx->device);
    if (cudaMemcpy(out, ctx->batched->trace, (size_t)n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return NMOE_ECUDA;
    return NMOE_OK;
}

extern "C" int nmoe_moe_debug_ep_times(nmoe_moe_ctx *ctx, float *ms) {
    if (ctx == nullptr || ms == nullptr || ctx->ep == nullptr || !ctx->ep->timing) {
        if (ctx) nmoe_ctx_set_error(ctx, "debug_ep_times: needs world_size > 1 and NMOE_EP_TIMING=1 at create");
        return NMOE_EINVAL;
    }
    Guard guard(ctx->device);
    EpState *E = ctx->ep;
    if (cudaEventSynchronize(E->ev[3]) != cudaSuccess) return NMOE_ECUDA;
    if (cudaEventElapsedTime(&ms[0], E->ev[0], E->ev[1]) != cudaSuccess) return NMOE_ECUDA;
    if (cudaEventElapsedTime(&ms[1], E->ev[2], E->ev[3]) != cudaSuccess) return NMOE_ECUDA;
    return NMOE_OK;
}

extern "C" int nmoe_moe_nccl_unique_id(void *out, size_t bytes) {
    if (out == nullptr || bytes < sizeof(ncclUniqueId)) return NMOE_EINVAL;
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return NMOE_ENCCL;
    memcpy(out, &id, sizeof id);
    return NMOE_OK;
}
