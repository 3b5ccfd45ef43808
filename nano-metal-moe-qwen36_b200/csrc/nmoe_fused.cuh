// nmoe_fused.cuh -- single-launch batch-1 decode (persistent kernel) and the repack of
// expert packs into the layout it reads (nmoe_pack.cuh).
#pragma once
#include "nmoe_ctx.cuh"

namespace nmoe {
struct FusedCall {
    const uint8_t *experts;                          // repacked blobs of this layer (this rank's)
    const uint8_t *router, *spairs, *gvec, *sdown_t;   // repacked dense regions of this layer
    const uint8_t *next_dense;                       // next layer's dense arena (L2 prefetch) or null
    uint32_t next_dense_bytes;
    const void *x;
    int x_f32;
    const float *h_mid;
    float *out;
    uint32_t *idx_out;
    float *w_out;
    float *logits_out;
    int k, num_experts, route_only;
    int *err;
};
// Repack n_experts blobs from the converter layout (src) into the kernel layout (dst).
cudaError_t repack_experts(const uint8_t *src, uint8_t *dst, int n_experts, int bits, cudaStream_t st);
}  // namespace nmoe

int nmoe_fused_init(nmoe_moe_ctx *ctx);
void nmoe_fused_destroy(nmoe_moe_ctx *ctx);
cudaError_t nmoe_fused_launch(nmoe_moe_ctx *ctx, const nmoe::FusedCall &a, cudaStream_t st);
