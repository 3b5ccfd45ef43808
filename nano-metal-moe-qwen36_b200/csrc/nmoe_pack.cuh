// nmoe_pack.cuh -- the HBM layout the batch-1 decode kernel and the grouped GEMM read.
//
// nmoe_moe_load_layer accepts the converter's layer_XX.bin image (EXPERT_LAYOUT,
// scripts/convert_qwen36.py:38-64) and stores each expert blob regrouped, same size:
//
//   GU region : 32 "band pairs" of 16 intermediate rows each:
//               [gate.w rows | up.w rows | gate.s | gate.b | up.s | up.b]
//               (rows row-major as in the converter; scales/biases [16 rows][32] bf16)
//   D region  : 8 "group slabs", one per 64-column group of the down matrix's input
//               (intermediate) dimension: [word column j][2048 output rows] u32 for the
//               group's wpg word columns (q4: 8, q2: 4), then down.s [2048] and down.b
//               [2048] bf16 of that group.
// A batch-1 unit (one expert, one 16-row band of the intermediate dimension) is then
// three contiguous copies: its gate/up band pair, the 2 (q4) / 1 (q2) word columns of
// the down matrix that the band's activations multiply, and its group's scales/biases.
// The grouped GEMM reads the band pairs through 4D tensor maps and the down slabs as
// [128 rows x wpg words] column-major tiles.
// Sizes: q4 band pair 36,864 B, down slab 73,728 B; q2 20,480 B and 40,960 B; the blob
// stays 1,769,472 (q4) / 983,040 (q2) bytes.
//
// Dense (router / shared) weights are stored row-interleaved so one CTA's slice is one
// contiguous copy: router rows [w | s | b] (q4) or [w] (bf16); shared gate/up pairs
// [gate.w | up.w | gate.s | gate.b | up.s | up.b]; shared down rows [w | s | b] (the
// grouped GEMM's copy) and the shared down again by columns (the batch-1 kernel's
// copy, `sdown_t`): bf16 [512 columns][2048 rows]; q4 [512 columns][256 words], each
// word 8 consecutive output rows of one column (row 8m+i in bits 4i..4i+3), then the
// scales [8 groups][2048] and biases [8 groups][2048] bf16.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace nmoe {

struct PackGeo {
    int bits, vpw;            // values per 32-bit word
    uint32_t wgu, wd;         // words per gate/up row (2048 cols) and per down row (512)
    uint32_t tile_band_gu;    // bytes of one matrix's 16 rows in a band
    uint32_t bp;              // band-pair bytes
    uint32_t wpg;             // down words per row per 64-column group (q4 8, q2 4)
    uint32_t dslab_w, dslab;  // down slab: word bytes / whole slab bytes
    uint32_t dunit;           // down word bytes of one 16-column band (2 / 1 word columns)
    uint32_t gu_bytes;        // 32 band pairs
    uint32_t esz;
};

__host__ __device__ inline PackGeo pack_geo(int bits) {
    PackGeo p;
    p.bits = bits;
    p.vpw = 32 / bits;
    p.wgu = 2048 / p.vpw;
    p.wd = 512 / p.vpw;
    p.tile_band_gu = 16 * p.wgu * 4;
    p.bp = 2 * p.tile_band_gu + 4 * 16 * 32 * 2;
    p.wpg = 64 / p.vpw;
    p.dslab_w = p.wpg * 2048 * 4;
    p.dslab = p.dslab_w + 2 * 2048 * 2;
    p.dunit = (16 / p.vpw) * 2048 * 4;
    p.gu_bytes = 32 * p.bp;
    p.esz = p.gu_bytes + 8 * p.dslab;
    return p;
}

// Dense row/pair strides in the repacked dense arena.
__host__ __device__ inline uint32_t dense_row_bytes(bool q4, int cols) {
    return q4 ? (uint32_t)(cols / 2 + 2 * (cols / 64) * 2) : (uint32_t)(cols * 2);
}

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Dense arena of one layer, row-interleaved as above: router rows, shared
// gate/up pairs, gate vector, shared down rows; each region 256-byte aligned.
struct DenseArena {
    size_t router, spairs, gvec, sdown, sdown_t, total;
    uint32_t rrow, srow, sdrow;   // row bytes (router, shared gate/up, shared down)
};
inline DenseArena dense_arena(int router_dtype, int shared_dtype) {
    DenseArena a;
    a.rrow = dense_row_bytes(router_dtype == 4, 2048);
    a.srow = dense_row_bytes(shared_dtype == 4, 2048);
    a.sdrow = dense_row_bytes(shared_dtype == 4, 512);
    a.router = 0;
    a.spairs = align256(a.router + (size_t)256 * a.rrow);
    a.gvec = align256(a.spairs + (size_t)512 * 2 * a.srow);
    a.sdown = align256(a.gvec + a.srow);
    a.sdown_t = align256(a.sdown + (size_t)2048 * a.sdrow);
    a.total = align256(a.sdown_t + (shared_dtype == 4 ? (size_t)512 * 1024 + 2 * 8 * 2048 * 2 : (size_t)512 * 2048 * 2));
    return a;
}

}  // namespace nmoe
