// nmoe_pack.cuh -- the HBM layout the single-launch decode kernel reads.
//
// nmoe_moe_load_layer accepts the converter's layer_XX.bin image (EXPERT_LAYOUT,
// scripts/convert_qwen36.py:38-64) and stores each expert blob regrouped by 16-row
// bands, same size, so that one CTA's routed slice is a single contiguous copy:
//
//   GU region : 32 "band pairs" of 16 intermediate rows each:
//               [gate.w rows | up.w rows | gate.s | gate.b | up.s | up.b]
//               (rows row-major as in the converter; scales/biases [16 rows][32] bf16)
//   D region  : 128 bands of 16 output rows: [down.w rows | down.s | down.b] ([16][8]).
// Sizes: q4 band pair 36,864 B, down band 4,608 B; q2 20,480 B and 2,560 B; the blob
// stays 1,769,472 (q4) / 983,040 (q2) bytes.
//
// Dense (router / shared) weights are stored row-interleaved so one CTA's slice is one
// contiguous copy: router rows [w | s | b] (q4) or [w] (bf16); shared gate/up pairs
// [gate.w | up.w | gate.s | gate.b | up.s | up.b]; shared down rows [w | s | b].
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace nmoe {

struct PackGeo {
    int bits, vpw;            // values per 32-bit word
    uint32_t wgu, wd;         // words per gate/up row (2048 cols) and per down row (512)
    uint32_t tile_band_gu;    // bytes of one matrix's 16 rows in a band
    uint32_t bp;              // band-pair bytes
    uint32_t tile_band_d, db; // down band tiles / whole band bytes
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
    p.tile_band_d = 16 * p.wd * 4;
    p.db = p.tile_band_d + 2 * 16 * 8 * 2;
    p.gu_bytes = 32 * p.bp;
    p.esz = p.gu_bytes + 128 * p.db;
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
    size_t router, spairs, gvec, sdown, total;
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
    a.total = align256(a.sdown + (size_t)2048 * a.sdrow);
    return a;
}

}  // namespace nmoe
