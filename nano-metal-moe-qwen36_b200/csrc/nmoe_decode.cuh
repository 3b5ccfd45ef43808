// nmoe_decode.cuh -- batch-1 decode launch interface.
#pragma once
#include "nmoe_common.cuh"

namespace nmoe {

// Device scratch shared by the staged batch-1 kernels of one call.
struct DecodeScratch {
    float logits[kExperts];
    float shared_act[kInter];
    float score;
    uint32_t idx[kMaxK];
    float w[kMaxK];
    float act[kMaxK * kInter];
};

struct DecodeArgs {
    LayerDev L;
    int bits;          // expert quantisation (4 / 2)
    bool router_q4, shared_q4;
    int num_experts;   // experts addressable in L.experts
    int k;
    const void *x;
    int x_f32;
    const float *h_mid;
    float *out;
    uint32_t *idx_out;
    float *w_out;
    DecodeScratch *ws;
    int *err;          // device error word
};

cudaError_t launch_route(const DecodeArgs &a, cudaStream_t st, float *logits_out);
cudaError_t launch_decode_staged(const DecodeArgs &a, cudaStream_t st);

}  // namespace nmoe
