// nmoe_batched.cuh -- T-token routed-MoE block (permutation + grouped GEMM + combine).
#pragma once
#include "nmoe_ctx.cuh"

int nmoe_batched_init(nmoe_moe_ctx *ctx);
void nmoe_batched_destroy(nmoe_moe_ctx *ctx);
