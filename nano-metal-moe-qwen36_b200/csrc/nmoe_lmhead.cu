// nmoe_lmhead.cu -- the LM head as one launch: final RMSNorm, vocab GEMV and top-1.
//
// Replaces, in the reference, the model.norm RMSNorm before the head
// (src/runtime.m:3786, kernel nmoe_rms_norm metal/kernels.metal:862-900) and the two-kernel
// head NMOERunLmHeadArgmaxQ4Metal (src/runtime.m:1882-1948): nmoe_lm_head_argmax_q4
// (metal/kernels.metal:1599-1666: one simdgroup per vocab row, acc += fma(q, scale, bias) * x,
// per-threadgroup best) and nmoe_lm_head_argmax_reduce (metal/kernels.metal:1668-1713).
// It also covers the reference's fallback (dequant matvec into logits + nmoe_argmax_top1,
// src/runtime.m:3793-3794, metal/kernels.metal:1562-1597) when the caller asks for logits.
//
// Selection rule (both reference kernels): the token is the lowest row index among the
// rows whose logit equals the maximum; a NaN logit, -inf and -FLT_MAX never win; if no
// row qualifies the token is 0. -0.0 and +0.0 compare equal.
//
// Layout of the work. The head is 248,320 rows x 2048 columns: 286 MB in q4 (1 KB of
// packed words + 64 B of scales + 64 B of biases per row), 1.02 GB in bf16 (4 KB per row),
// well above L2, so the launch is an HBM stream. One persistent CTA per SM owns a
// contiguous range of 16-row tiles. Rows are contiguous in HBM, so a tile is one bulk copy
// (plus one each for its scales and biases) into a shared-memory ring that a producer warp
// keeps full; the 16 compute warps take one row each per tile. The copies of the first
// tiles are issued before the programmatic-dependent-launch wait (the weights do not
// depend on the previous kernel), so the stream starts while the previous kernel drains.
// Each lane keeps its 64 columns of the normalised x in registers for the whole launch:
// q4 lane l owns scale group l (columns 64l..64l+63), bf16 lane l owns the 8-column chunks
// 32j+l (j = 0..7), which makes every shared-memory read of a row conflict-free.
// Top-1: each warp keeps its best (value, row); the CTA folds them into one 64-bit key
// (order-preserving value bits << 32 | ~row) and one atomicMax; the last CTA to finish
// writes the token and zeroes the workspace for the next call.
#include <cuda_runtime.h>
#include <float.h>
#include <stdio.h>

#include <mutex>

#include "nmoe/moe_cuda.h"
#include "nmoe_sm100.cuh"

using namespace nmoe;

namespace {

constexpr int kComputeWarps = 16;
constexpr int kThreads = (kComputeWarps + 1) * 32;   // + one producer warp
constexpr int kCols = NMOE_HIDDEN;                    // 2048
constexpr int kGroups = kCols / NMOE_GROUP;          // 32 scale groups per row

// Ring geometry per weight type: rows per tile, stage bytes and stage count.
template <int kDtype> struct Ring;
template <> struct Ring<NMOE_DTYPE_Q4> {
    static constexpr int kTileRows = 2 * kComputeWarps;               // 32: two rows per warp
    static constexpr int kRowBytes = kCols / 2;                       // 1024
    static constexpr int kSBytes = kGroups * 2;                       // 64 (scales; biases same)
    static constexpr int kStageBytes = kTileRows * (kRowBytes + 2 * kSBytes);   // 36 KB
    static constexpr int kStages = 5;
};
template <> struct Ring<NMOE_DTYPE_BF16> {
    static constexpr int kTileRows = kComputeWarps;                   // 16
    static constexpr int kRowBytes = kCols * 2;                       // 4096
    static constexpr int kSBytes = 0;
    static constexpr int kStageBytes = kTileRows * kRowBytes;        // 64 KB
    static constexpr int kStages = 3;
};
template <int kDtype>
constexpr int smem_bytes() {
    return Ring<kDtype>::kStages * Ring<kDtype>::kStageBytes + kCols * 4 + 2 * 64 * 8 + 1024;
}

struct LmArgs {
    const uint8_t *w;      // q4 packed words [vocab][256] u32, or bf16 [vocab][2048]
    const uint8_t *s;      // q4 scales bf16 [vocab][32]
    const uint8_t *b;      // q4 biases bf16 [vocab][32]
    const void *x;         // [2048] f32 or bf16
    const uint16_t *norm;  // bf16 [2048] RMSNorm weight, or null (x used as given)
    float eps;
    int add_one;
    int x_bf16;
    int vocab;
    int ntiles;
    float *logits;         // [vocab] or null
    uint32_t *token;       // [1]
    unsigned long long *ws;   // workspace: [0] best key, [1] low = CTA count, high = error word
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

__device__ __forceinline__ uint64_t pair64(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
// acc += (lo, hi) * b as one f32x2 FMA; lo/hi are 32-bit words joined as a register pair.
__device__ __forceinline__ void ffma2(uint64_t &acc, uint32_t lo, uint32_t hi, uint64_t b) {
    asm("{\n\t.reg .b64 t;\n\tmov.b64 t, {%1, %2};\n\tfma.rn.f32x2 %0, t, %3, %0;\n\t}"
        : "+l"(acc)
        : "r"(lo), "r"(hi), "l"(b));
}
__device__ __forceinline__ float pair_sum(uint64_t v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return lo + hi;
}

// q4 products without integer-to-float conversion: a nibble masked in place at bits
// k..k+3 (k = 0, 4, 8, 12) of an otherwise zero word is the subnormal float n * 2^(k-149).
// Column c of x is pre-scaled by 2^(E+19-k_c), k_c its nibble's bit position (E chosen per
// call so that every scaled |x| < 2^124), so every product is n * x * 2^(E-130), exact,
// and the fp32 sum of a row's products is sum(n x) * 2^(E-130): one AND per column (nibbles
// 4-7 of a word after one shift by 16), one f32x2 FMA per two columns, no constant term.
// Four packed words = 32 consecutive columns; nibble i of word j is column 8j+i.
__device__ __forceinline__ void q4_acc32(uint64_t &acc, const uint4 w, const uint64_t *x2) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t hi = ws[j] >> 16;
        ffma2(acc, ws[j] & 0xFu, ws[j] & 0xF0u, x2[4 * j]);
        ffma2(acc, ws[j] & 0xF00u, ws[j] & 0xF000u, x2[4 * j + 1]);
        ffma2(acc, hi & 0xFu, hi & 0xF0u, x2[4 * j + 2]);
        ffma2(acc, hi & 0xF00u, hi & 0xF000u, x2[4 * j + 3]);
    }
}

// Eight bf16 columns: the high half of a word is a float as it stands, the low half
// shifted up by 16.
__device__ __forceinline__ void bf16_acc8(uint64_t &acc, const uint4 w, const uint64_t *x2) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int p = 0; p < 4; ++p) ffma2(acc, u[p] << 16, u[p] & 0xFFFF0000u, x2[p]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Order-preserving key of a candidate; 0 = not a candidate (NaN, <= -FLT_MAX).
__device__ __forceinline__ unsigned long long cand_key(float v, uint32_t row) {
    if (!(v > -FLT_MAX)) return 0ull;
    if (v == 0.f) v = 0.f;   // -0.0 ties with +0.0
    const uint32_t u = __float_as_uint(v);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - row);
}

constexpr int kErrTimeout = 2;

template <int kDtype>
__global__ void __launch_bounds__(kThreads, 1) k_lm_head(const LmArgs a) {
    using R = Ring<kDtype>;
    constexpr int kTileRows = R::kTileRows;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *ring = smem;
    float *xs = reinterpret_cast<float *>(smem + R::kStages * R::kStageBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(xs + kCols);
    uint64_t *empty = full + 64;
    __shared__ float red[kComputeWarps];
    __shared__ unsigned long long best_keys[kComputeWarps];
    __shared__ int cta_err;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int t0 = (int)((long long)a.ntiles * c / G), t1 = (int)((long long)a.ntiles * (c + 1) / G);
    const int n = t1 - t0;
    const uint64_t deadline = globaltimer_ns() + 1000000000ull;   // 1 s; a launch takes < 1 ms

    if (tid == 0) {
        for (int s = 0; s < R::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kComputeWarps);
        }
        cta_err = 0;
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == kComputeWarps) {
        // ---- producer: keep the ring full (weights only: no dependency on the previous kernel)
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int issued = 0;
            for (int i = 0; i < n; ++i) {
                const int s = i % R::kStages;
                if (i >= R::kStages && !mbar_wait(&empty[s], ((i / R::kStages) - 1) & 1, deadline)) {
                    atomicExch(&cta_err, kErrTimeout);
                    break;
                }
                if (*(volatile int *)&cta_err) break;
                const int row0 = (t0 + i) * kTileRows;
                const int rows = min(kTileRows, a.vocab - row0);
                uint8_t *st = ring + s * R::kStageBytes;
                const uint32_t wb = (uint32_t)rows * R::kRowBytes;
                mbar_arrive_expect_tx(&full[s], wb + 2u * rows * R::kSBytes);
                bulk_g2s(st, a.w + (size_t)row0 * R::kRowBytes, wb, &full[s], pol);
                if (R::kSBytes) {
                    uint8_t *ss = st + kTileRows * R::kRowBytes;
                    bulk_g2s(ss, a.s + (size_t)row0 * R::kSBytes, rows * R::kSBytes, &full[s], pol);
                    bulk_g2s(ss + kTileRows * R::kSBytes, a.b + (size_t)row0 * R::kSBytes, rows * R::kSBytes,
                             &full[s], pol);
                }
                issued = i + 1;
            }
            // Copies still in flight (only after an error: normally every tile was consumed)
            // must land before this CTA's shared memory is released.
            for (int i = max(0, issued - R::kStages); i < issued; ++i)
                (void)mbar_wait(&full[i % R::kStages], (i / R::kStages) & 1, deadline + 100000000ull);
        }
        __syncwarp();
    } else {
        // ---- compute warps: x (after the previous kernel), optional RMSNorm, rows
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int ct = tid;   // 0..511
        float ss = 0.f;
        for (int i = ct; i < kCols; i += kComputeWarps * 32) {
            const float v = a.x_bf16 ? bf16f(reinterpret_cast<const uint16_t *>(a.x)[i])
                                     : reinterpret_cast<const float *>(a.x)[i];
            xs[i] = v;
            ss += v * v;
        }
        if (a.norm != nullptr) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            asm volatile("bar.sync 1, %0;" ::"r"(kComputeWarps * 32) : "memory");
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < kComputeWarps; ++w) tot += red[w];
            const float inv = rsqrtf(tot / (float)kCols + a.eps);
            for (int i = ct; i < kCols; i += kComputeWarps * 32) {
                float wgt = bf16f(a.norm[i]);
                if (a.add_one) wgt += 1.0f;
                xs[i] = xs[i] * inv * wgt;
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kComputeWarps * 32) : "memory");

        unsigned long long best = 0ull;
        uint64_t x2[32];
        if (kDtype == NMOE_DTYPE_Q4) {
            // Scale exponent E for the subnormal-product form (max |x| < 2^e -> E = 104 - e).
            float m = 0.f;
            for (int i = ct; i < kCols; i += kComputeWarps * 32) m = fmaxf(m, fabsf(xs[i]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            asm volatile("bar.sync 1, %0;" ::"r"(kComputeWarps * 32) : "memory");   // red[] reuse
            if (lane == 0) red[warp] = m;
            asm volatile("bar.sync 1, %0;" ::"r"(kComputeWarps * 32) : "memory");
            float mx = 0.f;
#pragma unroll
            for (int w = 0; w < kComputeWarps; ++w) mx = fmaxf(mx, red[w]);
            int e = 0;
            if (mx > 0.f && isfinite(mx)) (void)frexpf(mx, &e);
            const int E = 104 - e;
            // sum(n x) = acc * 2^(130-E), applied as two exact power-of-two multiplies
            const int bk = 130 - E, bk1 = bk / 2;
            const float back1 = ldexpf(1.f, bk1), back2 = ldexpf(1.f, bk - bk1);
            // Lane l owns scale group l (columns 64l..64l+63: 16-byte chunks 2l and 2l+1 of a
            // row). It reads chunk 2l+sw first and 2l+1-sw second, sw = bit 2 of the lane, so
            // that the eight lanes of each quarter-warp hit eight different bank groups in
            // both reads (no shared-memory conflicts).
            const int sw = (lane >> 2) & 1;
            const int cfirst = 2 * lane + sw, csecond = 2 * lane + 1 - sw;
            float xsum = 0.f;
            // Registers: x2[16h + 4j + p] = columns 8j+2p, 8j+2p+1 of the chunk read h-th
            // (chunk c = words 4c..4c+3 = columns 32c..32c+31), scaled for their nibble slots.
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int c = h == 0 ? cfirst : csecond;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 v0 = lds128f(xs + 32 * c + 8 * j);
                    const float4 v1 = lds128f(xs + 32 * c + 8 * j + 4);
                    xsum += ((v0.x + v0.y) + (v0.z + v0.w)) + ((v1.x + v1.y) + (v1.z + v1.w));
                    x2[16 * h + 4 * j] = pair64(ldexpf(v0.x, E + 19), ldexpf(v0.y, E + 15));
                    x2[16 * h + 4 * j + 1] = pair64(ldexpf(v0.z, E + 11), ldexpf(v0.w, E + 7));
                    x2[16 * h + 4 * j + 2] = pair64(ldexpf(v1.x, E + 19), ldexpf(v1.y, E + 15));
                    x2[16 * h + 4 * j + 3] = pair64(ldexpf(v1.z, E + 11), ldexpf(v1.w, E + 7));
                }
            }
            const bool upper = (lane & 16) != 0;

            int s = 0;
            uint32_t ph = 0;
            for (int i = 0; i < n; ++i) {
                if (!mbar_wait_warp(&full[s], ph, deadline)) {
                    if (lane == 0) atomicExch(&cta_err, kErrTimeout);
                    break;
                }
                const uint8_t *st = ring + s * R::kStageBytes;
                const int r0 = 2 * warp;                        // rows r0, r0+1 of the tile
                const int row = (t0 + i) * kTileRows + r0;      // first of the two
                if (row < a.vocab) {
                    const uint16_t *sc = reinterpret_cast<const uint16_t *>(st + kTileRows * R::kRowBytes);
                    const uint16_t *bi = sc + kTileRows * kGroups;
                    float v[2];
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const uint8_t *wr = st + (r0 + r) * R::kRowBytes;
                        const uint4 wa = lds128(wr + 16 * cfirst), wb = lds128(wr + 16 * csecond);
                        uint64_t acc_a = 0ull, acc_b = 0ull;
                        q4_acc32(acc_a, wa, x2);
                        q4_acc32(acc_b, wb, x2 + 16);
                        const int so = (r0 + r) * kGroups + lane;
                        const float sv = bf16f(sc[so]) * back1 * back2;
                        v[r] = fmaf(sv, pair_sum(acc_a) + pair_sum(acc_b), bf16f(bi[so]) * xsum);
                    }
                    // Two rows reduced together: after the first exchange lanes 0-15 hold row
                    // r0's partials and lanes 16-31 row r0+1's.
                    float keep = upper ? v[1] : v[0];
                    keep += __shfl_xor_sync(0xffffffffu, upper ? v[0] : v[1], 16);
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
                    const int my_row = row + (upper ? 1 : 0);
                    const unsigned long long k = cand_key(keep, (uint32_t)my_row);
                    const bool mine = (lane & 15) == 0 && my_row < a.vocab;
                    if (mine && a.logits != nullptr) a.logits[my_row] = keep;
                    best = (mine && k > best) ? k : best;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                if (++s == R::kStages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 v0 = lds128f(xs + 8 * (32 * j + lane));
                const float4 v1 = lds128f(xs + 8 * (32 * j + lane) + 4);
                x2[4 * j] = pair64(v0.x, v0.y);
                x2[4 * j + 1] = pair64(v0.z, v0.w);
                x2[4 * j + 2] = pair64(v1.x, v1.y);
                x2[4 * j + 3] = pair64(v1.z, v1.w);
            }
            int s = 0;
            uint32_t ph = 0;
            for (int i = 0; i < n; ++i) {
                if (!mbar_wait_warp(&full[s], ph, deadline)) {
                    if (lane == 0) atomicExch(&cta_err, kErrTimeout);
                    break;
                }
                const int row = (t0 + i) * kTileRows + warp;
                const uint8_t *wr = ring + s * R::kStageBytes + warp * R::kRowBytes;
                if (row < a.vocab) {
                    uint64_t acc = 0ull;
#pragma unroll
                    for (int j = 0; j < 8; ++j) bf16_acc8(acc, lds128(wr + 16 * (32 * j + lane)), x2 + 4 * j);
                    const float v = warp_sum(pair_sum(acc));
                    if (lane == 0) {
                        if (a.logits != nullptr) a.logits[row] = v;
                        const unsigned long long k = cand_key(v, (uint32_t)row);
                        best = k > best ? k : best;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                if (++s == R::kStages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) best_keys[warp] = best;
    }
    __syncthreads();

    if (tid == 0) {
        unsigned long long k = 0ull;
        for (int w = 0; w < kComputeWarps; ++w) k = best_keys[w] > k ? best_keys[w] : k;
        if (k != 0ull) atomicMax(&a.ws[0], k);
        if (cta_err) atomicOr(&a.ws[1], (unsigned long long)cta_err << 32);
        __threadfence();
        const unsigned long long prev = atomicAdd(&a.ws[1], 1ull);
        if ((uint32_t)prev == (uint32_t)(G - 1)) {
            __threadfence();
            const unsigned long long key = atomicExch(&a.ws[0], 0ull);
            const unsigned long long cnt = atomicExch(&a.ws[1], 0ull);
            const uint32_t err = (uint32_t)(cnt >> 32);
            *a.token = err ? 0xFFFFFFFFu : (key ? 0xFFFFFFFFu - (uint32_t)key : 0u);
        }
    }
}

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int g_sms[kMaxDevices] = {};   // 0 = device not set up yet
thread_local char g_err[256];

int fail(int code, const char *msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
    return code;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace

extern "C" const char *nmoe_lm_head_error(void) { return g_err; }

extern "C" size_t nmoe_lm_head_workspace_bytes(void) { return 16; }

extern "C" int nmoe_lm_head_argmax(const nmoe_tensor *head, int head_dtype, int vocab, int in_dim, const void *x,
                                   int x_dtype, const uint16_t *norm_weight, float norm_eps, int norm_add_one,
                                   float *logits_out, uint32_t *token_out, void *workspace, void *stream) {
    g_err[0] = 0;
    if (head == nullptr || head->weight == nullptr) return fail(NMOE_EINVAL, "head weight is null");
    if (head_dtype != NMOE_DTYPE_Q4 && head_dtype != NMOE_DTYPE_BF16)
        return fail(NMOE_EINVAL, "head_dtype must be NMOE_DTYPE_Q4 or NMOE_DTYPE_BF16");
    if (head_dtype == NMOE_DTYPE_Q4 && (head->scales == nullptr || head->biases == nullptr))
        return fail(NMOE_EINVAL, "q4 head needs scales and biases");
    if (in_dim != kCols) return fail(NMOE_EINVAL, "in_dim must be 2048 (NMOE_HIDDEN)");
    if (vocab < 1 || vocab > (1 << 30)) return fail(NMOE_EINVAL, "vocab out of range");
    if (x == nullptr || token_out == nullptr || workspace == nullptr) return fail(NMOE_EINVAL, "x, token_out and workspace are required");
    if (x_dtype != NMOE_DTYPE_F32 && x_dtype != NMOE_DTYPE_BF16) return fail(NMOE_EINVAL, "x_dtype must be F32 or BF16");
    if (!aligned(head->weight, 16) || (head_dtype == NMOE_DTYPE_Q4 && (!aligned(head->scales, 16) || !aligned(head->biases, 16))))
        return fail(NMOE_EINVAL, "head tensors must be 16-byte aligned");
    if (!aligned(workspace, 8) || !aligned(x, x_dtype == NMOE_DTYPE_F32 ? 4 : 2))
        return fail(NMOE_EINVAL, "misaligned x or workspace");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return fail(NMOE_ECUDA, "no usable current CUDA device");
    int sms;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (g_sms[dev] == 0) {
            int v = 0;
            cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(k_lm_head<NMOE_DTYPE_Q4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes<NMOE_DTYPE_Q4>());
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(k_lm_head<NMOE_DTYPE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes<NMOE_DTYPE_BF16>());
            if (e != cudaSuccess) return fail(NMOE_ECUDA, cudaGetErrorString(e));
            g_sms[dev] = v;
        }
        sms = g_sms[dev];
    }

    const int tile_rows = head_dtype == NMOE_DTYPE_Q4 ? Ring<NMOE_DTYPE_Q4>::kTileRows : Ring<NMOE_DTYPE_BF16>::kTileRows;
    LmArgs a;
    a.w = static_cast<const uint8_t *>(head->weight);
    a.s = static_cast<const uint8_t *>(head->scales);
    a.b = static_cast<const uint8_t *>(head->biases);
    a.x = x;
    a.norm = norm_weight;
    a.eps = norm_eps;
    a.add_one = norm_add_one ? 1 : 0;
    a.x_bf16 = x_dtype == NMOE_DTYPE_BF16;
    a.vocab = vocab;
    a.ntiles = (vocab + tile_rows - 1) / tile_rows;
    a.logits = logits_out;
    a.token = token_out;
    a.ws = static_cast<unsigned long long *>(workspace);

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.ntiles < sms ? a.ntiles : sms);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (head_dtype == NMOE_DTYPE_Q4) {
        cfg.dynamicSmemBytes = smem_bytes<NMOE_DTYPE_Q4>();
        e = cudaLaunchKernelEx(&cfg, k_lm_head<NMOE_DTYPE_Q4>, a);
    } else {
        cfg.dynamicSmemBytes = smem_bytes<NMOE_DTYPE_BF16>();
        e = cudaLaunchKernelEx(&cfg, k_lm_head<NMOE_DTYPE_BF16>, a);
    }
    if (e != cudaSuccess) return fail(NMOE_ECUDA, cudaGetErrorString(e));
    return NMOE_OK;
}
