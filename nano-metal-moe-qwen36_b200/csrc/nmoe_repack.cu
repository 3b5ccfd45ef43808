// nmoe_repack.cu -- converter layout (EXPERT_LAYOUT, scripts/convert_qwen36.py:38-64)
// -> the kernel layout of nmoe_pack.cuh (gate/up band pairs, down group slabs). One
// thread per 32-bit word of the destination; a pure permutation (same byte count).
#include "nmoe_fused.cuh"
#include "nmoe_pack.cuh"

namespace nmoe {

__global__ void k_repack(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int n_experts, int bits) {
    const PackGeo pg = pack_geo(bits);
    const ExpertOffsets eo = expert_offsets(bits);
    const size_t words = (size_t)n_experts * pg.esz / 4;
    for (size_t wi = blockIdx.x * (size_t)blockDim.x + threadIdx.x; wi < words; wi += (size_t)gridDim.x * blockDim.x) {
        const size_t e = wi * 4 / pg.esz;
        const uint32_t d = (uint32_t)(wi * 4 - e * pg.esz);
        uint32_t s;   // source byte offset within the blob
        if (d < pg.gu_bytes) {
            const uint32_t bp = d / pg.bp, r = d % pg.bp;
            if (r < 2 * pg.tile_band_gu) {   // 16 gate rows then 16 up rows, row-major
                const uint32_t mat = r / pg.tile_band_gu, q = r % pg.tile_band_gu;
                s = (mat ? eo.uw : eo.gw) + 16 * bp * pg.wgu * 4 + q;
            } else {                          // gs, gb, us, ub: [16][32] bf16 each
                const uint32_t r2 = r - 2 * pg.tile_band_gu, which = r2 / 1024, q = r2 % 1024;
                const uint32_t comp[4] = {eo.gs, eo.gb, eo.us, eo.ub};
                s = comp[which] + 16 * bp * 64 + q;
            }
        } else {   // down group slab g: word columns [j][2048 rows], then s[2048], b[2048]
            const uint32_t d2 = d - pg.gu_bytes, g = d2 / pg.dslab, r = d2 % pg.dslab;
            if (r < pg.dslab_w) {
                const uint32_t j = r / (2048 * 4), row = (r % (2048 * 4)) / 4;
                s = eo.dw + (row * pg.wd + g * pg.wpg + j) * 4;
            } else {   // two bf16 of consecutive rows: assembled from the [2048][8] tables
                const uint32_t r2 = r - pg.dslab_w, which = r2 / 4096, row = (r2 % 4096) / 2;
                const uint8_t *base = src + e * pg.esz + (which ? eo.db : eo.ds);
                const uint32_t lo = *reinterpret_cast<const uint16_t *>(base + (row * 8 + g) * 2);
                const uint32_t hi = *reinterpret_cast<const uint16_t *>(base + ((row + 1) * 8 + g) * 2);
                reinterpret_cast<uint32_t *>(dst)[wi] = lo | (hi << 16);
                continue;
            }
        }
        reinterpret_cast<uint32_t *>(dst)[wi] = *reinterpret_cast<const uint32_t *>(src + e * pg.esz + s);
    }
}

cudaError_t repack_experts(const uint8_t *src, uint8_t *dst, int n_experts, int bits, cudaStream_t st) {
    k_repack<<<1184, 256, 0, st>>>(src, dst, n_experts, bits);
    return cudaGetLastError();
}

}  // namespace nmoe
