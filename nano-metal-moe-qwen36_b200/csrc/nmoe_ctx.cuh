// nmoe_ctx.cuh -- the context behind the opaque nmoe_moe_ctx handle.
#pragma once
#include <vector>

#include "nmoe/moe_cuda.h"
#include "nmoe_common.cuh"

namespace nmoe {
struct DecodeScratch;
struct FusedState;
struct BatchedState;
struct EpState;
}  // namespace nmoe

struct nmoe_moe_ctx {
    nmoe_moe_config cfg;
    int device = 0;
    int num_sms = 0;
    size_t esz = 0;                 // bytes per expert blob
    int n_local = 0;                // experts held by this rank
    int expert_lo = 0;              // first global expert id held by this rank
    size_t expert_layer_bytes = 0;  // n_local * esz
    size_t dense_layer_bytes = 0;
    uint8_t *d_experts = nullptr;   // [num_layers][n_local * esz]
    uint8_t *d_dense = nullptr;     // [num_layers][dense_layer_bytes]
    int *d_err = nullptr;           // device error word (+3 spare ints)
    std::vector<char> loaded, dense_set;
    int prefetch_next = 0;          // NMOE_PREFETCH_NEXT=1: prefetch layer+1's dense weights to L2
    nmoe::FusedState *fused = nullptr;
    nmoe::BatchedState *batched = nullptr;
    nmoe::EpState *ep = nullptr;
    char last_error[512] = {0};
};

void nmoe_ctx_set_error(nmoe_moe_ctx *ctx, const char *fmt, ...);
int nmoe_ctx_check_call(nmoe_moe_ctx *ctx, int layer, int k, int x_dtype);
