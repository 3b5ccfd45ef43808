// nmoe_common.cuh -- shared device helpers and the device-side view of one MoE layer.
//
// Data layout in HBM (per layer, all resident):
//   experts : num_experts x expert_size bytes, byte-identical to layer_XX.bin
//             (EXPERT_LAYOUT, scripts/convert_qwen36.py:38-64). Each blob holds
//             gate.w [512][2048/vpw] u32 | gate.s [512][32] bf16 | gate.b | up.(w,s,b) |
//             down.w [2048][512/vpw] u32 | down.s [2048][8] bf16 | down.b
//             (vpw = 8 values per word for q4, 16 for q2).
//   dense   : router [256][2048], shared gate/up [512][2048], shared down [2048][512],
//             shared gate vector [1][2048]; bf16 row-major, or q4 (w, s, b) as written by
//             quantize_matrix_to_weights (scripts/convert_qwen36.py:214-263).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nmoe {

constexpr int kHidden = 2048;
constexpr int kInter = 512;
constexpr int kExperts = 256;
constexpr int kGroup = 64;
constexpr int kMaxK = 8;

// Device error word codes (read back by nmoe_moe_device_status).
constexpr int kErrExpertRange = 1;
constexpr int kErrTimeout = 2;

struct DenseDev {
    const void *w;        // bf16 [rows][cols] or q4 u32 [rows][cols/8]
    const uint16_t *s;    // q4 scales [rows][cols/64]
    const uint16_t *b;    // q4 biases
};

struct LayerDev {
    const uint8_t *experts;  // this rank's experts (expert_lo .. expert_lo + n_local - 1)
    DenseDev router, sgate, sup, sdown, gvec;
};

struct ExpertOffsets {
    uint32_t gw, gs, gb, uw, us, ub, dw, ds, db, size;
};

__host__ __device__ inline ExpertOffsets expert_offsets(int bits) {
    // EXPERT_LAYOUT / EXPERT_LAYOUT_2BIT (scripts/convert_qwen36.py:38-64).
    if (bits == 2) return {0u, 262144u, 294912u, 327680u, 589824u, 622592u, 655360u, 917504u, 950272u, 983040u};
    return {0u, 524288u, 557056u, 589824u, 1114112u, 1146880u, 1179648u, 1703936u, 1736704u, 1769472u};
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_to_f32(uint16_t v) { return __uint_as_float(((uint32_t)v) << 16); }

// Exact small integer -> float without I2F: 2^23 + q has q in the low mantissa bits.
__device__ __forceinline__ float small_u2f(uint32_t q) {
    return __uint_as_float(0x4B000000u | q) - 8388608.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x * sigmoidf_(x); }

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    // Weights are read once per call: skip L1 allocation.
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// sum_{i<32} q_i * x_i for the 32 nibbles of a q4 uint4 (word j nibble i = column 8j+i).
__device__ __forceinline__ float dot_q4_32(const uint4 w, const float *xs) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            a0 = fmaf(small_u2f((ws[j] >> (4 * i)) & 0xFu), xs[8 * j + i], a0);
            a1 = fmaf(small_u2f((ws[j] >> (4 * i + 4)) & 0xFu), xs[8 * j + i + 1], a1);
        }
    }
    return a0 + a1;
}

// sum_{i<64} q_i * x_i for the 64 crumbs of a q2 uint4 (word j crumb i = column 16j+i).
__device__ __forceinline__ float dot_q2_64(const uint4 w, const float *xs) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            a0 = fmaf(small_u2f((ws[j] >> (2 * i)) & 0x3u), xs[16 * j + i], a0);
            a1 = fmaf(small_u2f((ws[j] >> (2 * i + 2)) & 0x3u), xs[16 * j + i + 1], a1);
        }
    }
    return a0 + a1;
}

// sum_{i<8} w_i * x_i for 8 bf16 weights.
__device__ __forceinline__ float dot_bf16_8(const uint4 w, const float *xs) {
    float a = 0.f;
    a = fmaf(bf16_lo(w.x), xs[0], a);
    a = fmaf(bf16_hi(w.x), xs[1], a);
    a = fmaf(bf16_lo(w.y), xs[2], a);
    a = fmaf(bf16_hi(w.y), xs[3], a);
    a = fmaf(bf16_lo(w.z), xs[4], a);
    a = fmaf(bf16_hi(w.z), xs[5], a);
    a = fmaf(bf16_lo(w.w), xs[6], a);
    a = fmaf(bf16_hi(w.w), xs[7], a);
    return a;
}

// One warp: dot of a dense row (bf16 or q4, `cols` wide) with xs (fp32 in shared memory).
// xsum32[c] = sum of xs[32c .. 32c+31] (used by the q4 affine factorisation
// sum (q*s+b)*x = s*sum(q*x) + b*sum(x) per 32-column chunk). Lane partial, not reduced.
template <bool kQ4>
__device__ __forceinline__ float dense_row_partial(const DenseDev &d, int row, int cols, const float *xs,
                                                   const float *xsum32, int lane) {
    float acc = 0.f;
    if (kQ4) {
        const uint4 *wr = reinterpret_cast<const uint4 *>(static_cast<const uint32_t *>(d.w) + (size_t)row * (cols / 8));
        const uint16_t *sr = d.s + (size_t)row * (cols / kGroup);
        const uint16_t *br = d.b + (size_t)row * (cols / kGroup);
        for (int c = lane; c < cols / 32; c += 32) {
            uint4 w = ldg_stream(wr + c);
            float s = bf16_to_f32(sr[c >> 1]), b = bf16_to_f32(br[c >> 1]);
            acc = fmaf(s, dot_q4_32(w, xs + 32 * c), fmaf(b, xsum32[c], acc));
        }
    } else {
        const uint4 *wr = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(d.w) + (size_t)row * cols);
        for (int c = lane; c < cols / 8; c += 32) acc += dot_bf16_8(ldg_stream(wr + c), xs + 8 * c);
    }
    return acc;
}

}  // namespace nmoe
