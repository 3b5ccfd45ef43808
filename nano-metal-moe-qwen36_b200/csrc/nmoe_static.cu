// nmoe_static.cu -- a batch-1 forward that allocates nothing.
//
// nmoe_moe_forward_static runs the staged batch-1 kernels (nmoe_decode.cu) on layer
// weights the caller already holds in device memory, with the kernels' scratch in a
// file-scope device array instead of memory from cudaMalloc. It exists for callers that
// cannot allocate device memory at the point of the call: hosts whose memory is owned by
// a preallocated pool or arena they may not bypass, code running where cudaMalloc's
// implicit device synchronisation is not allowed, or embedders that create no
// nmoe_moe_ctx at all.
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>

#include "nmoe/moe_cuda.h"
#include "nmoe_decode.cuh"

using namespace nmoe;

namespace {

// Scratch of one call: the staged kernels' DecodeScratch (router logits, shared
// activation, score, routed ids/weights, act for up to kMaxK = 8 slots) + error word.
struct StaticScratch {
    DecodeScratch ws;
    int err[4];
};
constexpr size_t kStaticScratchBytes = (sizeof(StaticScratch) + 255) & ~size_t(255);

// Every GPU that loads this library holds this array until the process exits.
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
StaticScratch *g_scratch_ptr[kMaxDevices] = {};   // device address per device (set once)

thread_local char g_static_error[256];

int fail(int code, const char *msg) {
    snprintf(g_static_error, sizeof g_static_error, "%s", msg);
    return code;
}

}  // namespace

extern "C" const char *nmoe_moe_static_error(void) { return g_static_error; }

extern "C" size_t nmoe_moe_static_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" int nmoe_moe_static_status(int *code, void *stream) {
    g_static_error[0] = 0;
    if (code) *code = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return fail(NMOE_ECUDA, "no usable current CUDA device");
    StaticScratch *scr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        scr = g_scratch_ptr[dev];
    }
    if (scr == nullptr) return NMOE_OK;   // no call has run on this device
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int h = 0;   // the word is read into this stack variable: nothing is allocated
    cudaError_t e = cudaMemcpyAsync(&h, scr->err, sizeof h, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = cudaMemsetAsync(scr->err, 0, sizeof(int), st);
    if (e != cudaSuccess) return fail(NMOE_ECUDA, cudaGetErrorString(e));
    if (code) *code = h;
    if (h == 0) return NMOE_OK;
    snprintf(g_static_error, sizeof g_static_error, "device error word = %d (%s)", h,
             h == kErrExpertRange ? "routed expert id out of range" : h == kErrTimeout ? "bounded wait expired" : "unknown");
    return h == kErrTimeout ? NMOE_ETIMEOUT : NMOE_EDEVICE;
}

extern "C" int nmoe_moe_forward_static(const void *experts, int num_experts, int quant_bits,
                                       const nmoe_moe_dense_weights *dense, int router_dtype, int shared_dtype,
                                       int k, const void *x, int x_dtype, const float *h_mid, float *out,
                                       uint32_t *idx_out, float *w_out, void *stream) {
    g_static_error[0] = 0;
    if (quant_bits != 2 && quant_bits != 4) return fail(NMOE_EINVAL, "quant_bits must be 2 or 4");
    if (k < 1 || k > kMaxK)
        return fail(NMOE_EINVAL, "k must be in [1, 8]: the static scratch holds activations for at most 8 routed experts");
    if (num_experts < 1 || num_experts > NMOE_NUM_EXPERTS) return fail(NMOE_EINVAL, "num_experts must be in [1, 256]");
    for (int d : {router_dtype, shared_dtype})
        if (d != NMOE_DTYPE_BF16 && d != NMOE_DTYPE_Q4) return fail(NMOE_EINVAL, "router/shared dtype must be BF16 or Q4");
    if (x_dtype != NMOE_DTYPE_BF16 && x_dtype != NMOE_DTYPE_F32) return fail(NMOE_EINVAL, "x_dtype must be BF16 or F32");
    if (experts == nullptr || dense == nullptr || x == nullptr || out == nullptr)
        return fail(NMOE_EINVAL, "experts, dense, x and out are required");
    const nmoe_tensor *t[5] = {&dense->router, &dense->shared_gate, &dense->shared_up, &dense->shared_down,
                               &dense->shared_gate_vec};
    for (int m = 0; m < 5; ++m) {
        const bool q4 = (m == 0 ? router_dtype : shared_dtype) == NMOE_DTYPE_Q4;
        if (t[m]->weight == nullptr || (q4 && (t[m]->scales == nullptr || t[m]->biases == nullptr)))
            return fail(NMOE_EINVAL, "a dense tensor is missing its weight/scales/biases pointer");
    }

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(NMOE_ECUDA, "no usable current CUDA device");
    StaticScratch *scr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (g_scratch_ptr[dev] == nullptr) {
            // One-time set-up on this device (the current one): the device address of the
            // file-scope array. The host-side symbol is not a device address.
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
            if (e != cudaSuccess) {
                snprintf(g_static_error, sizeof g_static_error, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
                return NMOE_ECUDA;
            }
            g_scratch_ptr[dev] = static_cast<StaticScratch *>(p);
        }
        scr = g_scratch_ptr[dev];
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The error word must start at zero; everything else is written before it is read.
    cudaError_t e = cudaMemsetAsync(scr->err, 0, sizeof scr->err, st);
    if (e != cudaSuccess) return fail(NMOE_ECUDA, cudaGetErrorString(e));

    DecodeArgs a;
    a.L.experts = static_cast<const uint8_t *>(experts);
    DenseDev *dst[5] = {&a.L.router, &a.L.sgate, &a.L.sup, &a.L.sdown, &a.L.gvec};
    for (int m = 0; m < 5; ++m) {
        dst[m]->w = t[m]->weight;
        dst[m]->s = static_cast<const uint16_t *>(t[m]->scales);
        dst[m]->b = static_cast<const uint16_t *>(t[m]->biases);
    }
    a.bits = quant_bits;
    a.router_q4 = router_dtype == NMOE_DTYPE_Q4;
    a.shared_q4 = shared_dtype == NMOE_DTYPE_Q4;
    a.num_experts = num_experts;
    a.k = k;
    a.x = x;
    a.x_f32 = x_dtype == NMOE_DTYPE_F32;
    a.h_mid = h_mid;
    a.out = out;
    a.idx_out = idx_out;
    a.w_out = w_out;
    a.ws = &scr->ws;
    a.err = scr->err;
    e = launch_decode_staged(a, st);
    if (e != cudaSuccess) return fail(NMOE_ECUDA, cudaGetErrorString(e));
    return NMOE_OK;
}
