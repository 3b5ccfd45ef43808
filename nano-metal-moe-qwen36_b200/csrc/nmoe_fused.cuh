// nmoe_fused.cuh -- single-launch batch-1 decode (persistent kernel).
#pragma once
#include "nmoe_ctx.cuh"
#include "nmoe_decode.cuh"

cudaError_t nmoe_fused_init(nmoe_moe_ctx *ctx);
void nmoe_fused_destroy(nmoe_moe_ctx *ctx);
cudaError_t nmoe_fused_launch(nmoe_moe_ctx *ctx, const nmoe::DecodeArgs &a, cudaStream_t st);
