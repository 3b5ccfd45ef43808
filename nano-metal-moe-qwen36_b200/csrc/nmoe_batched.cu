// nmoe_batched.cu -- placeholder until the batched path lands.
#include "nmoe_batched.cuh"

int nmoe_batched_init(nmoe_moe_ctx *) { return NMOE_OK; }
void nmoe_batched_destroy(nmoe_moe_ctx *) {}
extern "C" int nmoe_moe_forward_batched(nmoe_moe_ctx *ctx, int, int, int, const void *, int, const float *, void *,
                                        int, uint32_t *, float *, void *) {
    nmoe_ctx_set_error(ctx, "forward_batched not available in this build");
    return NMOE_EINVAL;
}
