// nmoe_crc.cu -- CRC-32C of expert packs: on the device while a layer image is staged for
// loading, and on the host for writing manifests.
//
// CRC-32C (Castagnoli): reflected polynomial 0x82F63B78, initial value and final xor
// 0xFFFFFFFF (the iSCSI / SSE4.2 `crc32` checksum). The reference's loader has no
// checksum (include/nmoe/expert_io.h:22-26 only checks sizes, src/expert_io.m:52-65);
// this is the integrity check of a layer_XX.bin image that the B200 loader adds.
//
// Device layout of the work: one CTA per expert blob, 1024 threads; thread i computes the
// CRC of bytes [i S, (i + 1) S) of the blob (S = blob / 1024, a multiple of 8) with
// slice-by-8 tables in shared memory, and the 1024 CRCs are folded pairwise in 10 levels
// with the linear combination rule crc(A B) = x^(8 |B|) * crc(A) + crc(B) mod P (the
// published zlib crc32_combine method: GF(2) polynomial products in reflected order).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "nmoe/moe_cuda.h"

namespace {

constexpr uint32_t kPoly = 0x82F63B78u;   // reflected Castagnoli polynomial
constexpr int kThreads = 1024;

// a * b mod P, reflected representation (bit 31 = x^0).
__host__ __device__ inline uint32_t multmodp(uint32_t a, uint32_t b) {
    uint32_t m = 1u << 31, p = 0u;
    for (;;) {
        if (a & m) {
            p ^= b;
            if ((a & (m - 1u)) == 0u) break;
        }
        m >>= 1;
        b = (b & 1u) ? (b >> 1) ^ kPoly : b >> 1;
    }
    return p;
}

// x^(8 n) mod P by square-and-multiply over x^(2^k).
__host__ __device__ inline uint32_t x8nmodp(uint64_t n) {
    uint32_t p = 1u << 31;          // x^0
    uint32_t sq = 1u << 23;         // x^8 (bit 31 - k holds x^k): the power for one byte
    while (n) {
        if (n & 1u) p = multmodp(sq, p);
        sq = multmodp(sq, sq);
        n >>= 1;
    }
    return p;
}

// crc(A B) from crc(A), crc(B) and |B| bytes.
__host__ __device__ inline uint32_t crc_combine(uint32_t ca, uint32_t cb, uint64_t len_b) {
    return multmodp(x8nmodp(len_b), ca) ^ cb;
}

}  // namespace

namespace nmoe {
struct FoldPowers {
    uint32_t x[10];   // x^(8 S 2^j) mod P, S = blob / 1024: the shift of fold level j
};
}  // namespace nmoe
using nmoe::FoldPowers;

namespace {

__global__ void __launch_bounds__(kThreads, 1)
    k_crc32c_blobs(const uint8_t *base, size_t blob, uint32_t *out, const FoldPowers fp) {
    __shared__ uint32_t T[8][256];
    __shared__ uint32_t crcs[kThreads];
    const int tid = threadIdx.x;
    // byte table, then the 7 slice tables level by level
    if (tid < 256) {
        uint32_t c = (uint32_t)tid;
        for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ kPoly : c >> 1;
        T[0][tid] = c;
    }
    __syncthreads();
    for (int s = 1; s < 8; ++s) {
        if (tid < 256) T[s][tid] = (T[s - 1][tid] >> 8) ^ T[0][T[s - 1][tid] & 0xFFu];
        __syncthreads();
    }
    const size_t seg = blob / kThreads;
    const uint8_t *p = base + (size_t)blockIdx.x * blob + (size_t)tid * seg;
    uint32_t crc = 0xFFFFFFFFu;
    for (size_t o = 0; o < seg; o += 8) {
        const uint2 w = __ldg(reinterpret_cast<const uint2 *>(p + o));
        const uint32_t lo = w.x ^ crc, hi = w.y;
        crc = T[7][lo & 0xFFu] ^ T[6][(lo >> 8) & 0xFFu] ^ T[5][(lo >> 16) & 0xFFu] ^ T[4][lo >> 24] ^
              T[3][hi & 0xFFu] ^ T[2][(hi >> 8) & 0xFFu] ^ T[1][(hi >> 16) & 0xFFu] ^ T[0][hi >> 24];
    }
    crcs[tid] = crc ^ 0xFFFFFFFFu;
    __syncthreads();
    // fold: at level j, segment i (i a multiple of 2^(j+1)) absorbs segment i + 2^j
    for (int j = 0; (1 << j) < kThreads; ++j) {
        const int step = 1 << j;
        if ((tid & (2 * step - 1)) == 0) crcs[tid] = multmodp(fp.x[j], crcs[tid]) ^ crcs[tid + step];
        __syncthreads();
    }
    if (tid == 0) out[blockIdx.x] = crcs[0];
}

// ---------------------------------------------------------------- host ----

struct HostTables {
    uint32_t t[8][256];
    HostTables() {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ kPoly : c >> 1;
            t[0][i] = c;
        }
        for (int s = 1; s < 8; ++s)
            for (uint32_t i = 0; i < 256; ++i) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xFFu];
    }
};
const HostTables g_tab;

#if defined(__x86_64__)
__attribute__((target("sse4.2"))) uint32_t crc_hw(uint32_t crc, const uint8_t *p, size_t n) {
    uint64_t c = crc;
    for (; n >= 8; n -= 8, p += 8) {
        uint64_t v;
        memcpy(&v, p, 8);
        c = __builtin_ia32_crc32di(c, v);
    }
    uint32_t c32 = (uint32_t)c;
    for (; n; --n, ++p) c32 = __builtin_ia32_crc32qi(c32, *p);
    return c32;
}
#endif

uint32_t crc_sw(uint32_t crc, const uint8_t *p, size_t n) {
    for (; n >= 8; n -= 8, p += 8) {
        uint32_t lo, hi;
        memcpy(&lo, p, 4);
        memcpy(&hi, p + 4, 4);
        lo ^= crc;
        crc = g_tab.t[7][lo & 0xFFu] ^ g_tab.t[6][(lo >> 8) & 0xFFu] ^ g_tab.t[5][(lo >> 16) & 0xFFu] ^
              g_tab.t[4][lo >> 24] ^ g_tab.t[3][hi & 0xFFu] ^ g_tab.t[2][(hi >> 8) & 0xFFu] ^
              g_tab.t[1][(hi >> 16) & 0xFFu] ^ g_tab.t[0][hi >> 24];
    }
    for (; n; --n, ++p) crc = (crc >> 8) ^ g_tab.t[0][(crc ^ *p) & 0xFFu];
    return crc;
}

}  // namespace

extern "C" uint32_t nmoe_crc32c(uint32_t crc, const void *data, size_t n) {
    const uint8_t *p = static_cast<const uint8_t *>(data);
    if (p == nullptr || n == 0) return crc;
    crc = ~crc;
#if defined(__x86_64__)
    if (__builtin_cpu_supports("sse4.2")) return ~crc_hw(crc, p, n);
#endif
    return ~crc_sw(crc, p, n);
}

extern "C" uint32_t nmoe_crc32c_combine(uint32_t crc_a, uint32_t crc_b, size_t len_b) {
    return crc_combine(crc_a, crc_b, len_b);
}

namespace nmoe {
FoldPowers fold_powers(size_t blob);
}

extern "C" int nmoe_crc32c_device(const void *d_data, size_t blob_bytes, int nblobs, uint32_t *d_crc_out,
                                  void *stream) {
    if (d_data == nullptr || d_crc_out == nullptr || nblobs < 0) return NMOE_EINVAL;
    if (nblobs == 0) return NMOE_OK;
    if (blob_bytes == 0 || blob_bytes % (8u * kThreads) != 0 || (reinterpret_cast<uintptr_t>(d_data) & 7u) != 0)
        return NMOE_EINVAL;
    k_crc32c_blobs<<<nblobs, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t *>(d_data), blob_bytes, d_crc_out, nmoe::fold_powers(blob_bytes));
    return cudaGetLastError() == cudaSuccess ? NMOE_OK : NMOE_ECUDA;
}

namespace nmoe {

FoldPowers fold_powers(size_t blob) {
    FoldPowers f;
    for (int j = 0; j < 10; ++j) f.x[j] = x8nmodp((uint64_t)(blob / kThreads) << j);
    return f;
}

// CRC-32C of n consecutive blobs of `blob` bytes (a multiple of 8 * 1024) at d_base,
// into d_out[n]; asynchronous on st.
cudaError_t crc32c_blobs(const uint8_t *d_base, size_t blob, int n, uint32_t *d_out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (blob == 0 || blob % (8u * kThreads) != 0) return cudaErrorInvalidValue;
    k_crc32c_blobs<<<n, kThreads, 0, st>>>(d_base, blob, d_out, fold_powers(blob));
    return cudaGetLastError();
}

}  // namespace nmoe
