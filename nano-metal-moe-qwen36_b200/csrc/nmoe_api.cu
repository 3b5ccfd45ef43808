// nmoe_api.cu -- the C ABI (include/nmoe/moe_cuda.h): context, HBM-resident packs,
// layout validation and the forward entry points.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "nmoe/moe_cuda.h"
#include "nmoe_batched.cuh"
#include "nmoe_ctx.cuh"
#include "nmoe_decode.cuh"
#include "nmoe_fused.cuh"
#include "nmoe_pack.cuh"

using namespace nmoe;

namespace nmoe {
cudaError_t crc32c_blobs(const uint8_t *d_base, size_t blob, int n, uint32_t *d_out, cudaStream_t st);
}

// ------------------------------------------------------------------ helpers ----

void nmoe_ctx_set_error(nmoe_moe_ctx *ctx, const char *fmt, ...) {
    if (ctx == nullptr) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(ctx->last_error, sizeof ctx->last_error, fmt, ap);
    va_end(ap);
}

static int cuda_fail(nmoe_moe_ctx *ctx, cudaError_t e, const char *what) {
    nmoe_ctx_set_error(ctx, "%s: %s", what, cudaGetErrorString(e));
    return NMOE_ECUDA;
}

#define NMOE_CUDA_TRY(ctx, call)                           \
    do {                                                   \
        cudaError_t _e = (call);                           \
        if (_e != cudaSuccess) return cuda_fail(ctx, _e, #call); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// ------------------------------------------------------------- host helpers ----

extern "C" size_t nmoe_moe_expert_size(int quant_bits) {
    if (quant_bits != 2 && quant_bits != 4) return 0;
    return expert_offsets(quant_bits).size;
}

extern "C" int nmoe_moe_expert_offsets(int quant_bits, size_t offsets[9]) {
    if ((quant_bits != 2 && quant_bits != 4) || offsets == nullptr) return NMOE_EINVAL;
    const ExpertOffsets o = expert_offsets(quant_bits);
    const uint32_t v[9] = {o.gw, o.gs, o.gb, o.uw, o.us, o.ub, o.dw, o.ds, o.db};
    for (int i = 0; i < 9; ++i) offsets[i] = v[i];
    return NMOE_OK;
}

extern "C" const char *nmoe_moe_strerror(int status) {
    switch (status) {
        case NMOE_OK: return "ok";
        case NMOE_EINVAL: return "invalid argument";
        case NMOE_ESIZE: return "size or layout mismatch";
        case NMOE_ECUDA: return "CUDA error";
        case NMOE_ENCCL: return "NCCL error";
        case NMOE_ETIMEOUT: return "device wait timed out";
        case NMOE_EDEVICE: return "device error word set";
        case NMOE_EIO: return "I/O error";
        case NMOE_ENOMEM: return "out of memory";
        case NMOE_ECHECKSUM: return "checksum mismatch";
        default: return "unknown status";
    }
}

extern "C" const char *nmoe_moe_last_error(const nmoe_moe_ctx *ctx) {
    return ctx ? ctx->last_error : "null context";
}

// ------------------------------------------------------------------ create ----

static int validate_config(const nmoe_moe_config *c, char *msg, size_t n) {
    if (c == nullptr) { snprintf(msg, n, "null config"); return NMOE_EINVAL; }
    if (c->quant_bits != 2 && c->quant_bits != 4) { snprintf(msg, n, "quant_bits must be 2 or 4"); return NMOE_EINVAL; }
    if (c->num_layers < 1) { snprintf(msg, n, "num_layers must be >= 1"); return NMOE_EINVAL; }
    if (c->num_experts < 1 || c->num_experts > NMOE_NUM_EXPERTS) {
        snprintf(msg, n, "num_experts must be in [1, %d]", NMOE_NUM_EXPERTS); return NMOE_EINVAL;
    }
    if (c->k_max < 1 || c->k_max > NMOE_MAX_K) { snprintf(msg, n, "k_max must be in [1, 8]"); return NMOE_EINVAL; }
    if (c->k_max > c->num_experts) { snprintf(msg, n, "k_max exceeds num_experts"); return NMOE_EINVAL; }
    for (int d : {c->router_dtype, c->shared_dtype})
        if (d != NMOE_DTYPE_BF16 && d != NMOE_DTYPE_Q4) {
            snprintf(msg, n, "router/shared dtype must be NMOE_DTYPE_BF16 or NMOE_DTYPE_Q4"); return NMOE_EINVAL;
        }
    if (c->t_max < 0) { snprintf(msg, n, "t_max must be >= 0"); return NMOE_EINVAL; }
    const int ws = c->world_size < 1 ? 1 : c->world_size;
    if (c->rank < 0 || c->rank >= ws) { snprintf(msg, n, "rank out of range"); return NMOE_EINVAL; }
    if (ws > 1 && (c->num_experts % ws != 0)) { snprintf(msg, n, "num_experts must divide by world_size"); return NMOE_EINVAL; }
    if (ws > 1 && c->nccl_unique_id == nullptr) { snprintf(msg, n, "nccl_unique_id required when world_size > 1"); return NMOE_EINVAL; }
    return NMOE_OK;
}

static thread_local char g_create_error[512];

extern "C" const char *nmoe_moe_create_error(void) { return g_create_error; }

extern "C" nmoe_moe_ctx *nmoe_moe_create(const nmoe_moe_config *cfg, int device, int *status) {
    int st_dummy;
    int *st = status ? status : &st_dummy;
    g_create_error[0] = 0;
    *st = validate_config(cfg, g_create_error, sizeof g_create_error);
    if (*st != NMOE_OK) return nullptr;

    int ndev = 0;
    cudaError_t ce = cudaGetDeviceCount(&ndev);
    if (ce != cudaSuccess || device < 0 || device >= ndev) {
        snprintf(g_create_error, sizeof g_create_error, "no CUDA device %d (%s)", device,
                 ce != cudaSuccess ? cudaGetErrorString(ce) : "out of range");
        *st = NMOE_ECUDA;
        return nullptr;
    }
    DeviceGuard guard(device);
    nmoe_moe_ctx *ctx = new (std::nothrow) nmoe_moe_ctx();
    if (ctx == nullptr) { *st = NMOE_ENOMEM; return nullptr; }
    ctx->cfg = *cfg;
    if (ctx->cfg.world_size < 1) ctx->cfg.world_size = 1;
    ctx->device = device;
    ctx->esz = nmoe_moe_expert_size(cfg->quant_bits);
    ctx->n_local = cfg->num_experts / ctx->cfg.world_size;
    ctx->expert_lo = ctx->cfg.rank * ctx->n_local;
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, device);
    ctx->num_sms = prop.multiProcessorCount;

    const size_t per_layer = dense_arena(cfg->router_dtype, cfg->shared_dtype).total;
    ctx->dense_layer_bytes = per_layer;
    ctx->expert_layer_bytes = (size_t)ctx->n_local * ctx->esz;

    auto fail = [&](cudaError_t e, const char *what) -> nmoe_moe_ctx * {
        snprintf(g_create_error, sizeof g_create_error, "%s: %s", what, cudaGetErrorString(e));
        *st = (e == cudaErrorMemoryAllocation) ? NMOE_ENOMEM : NMOE_ECUDA;
        nmoe_moe_destroy(ctx);
        return nullptr;
    };
    if ((ce = cudaMalloc(&ctx->d_experts, ctx->expert_layer_bytes * cfg->num_layers)) != cudaSuccess)
        return fail(ce, "cudaMalloc(experts)");
    if ((ce = cudaMemset(ctx->d_experts, 0, ctx->expert_layer_bytes * cfg->num_layers)) != cudaSuccess)
        return fail(ce, "cudaMemset(experts)");
    if ((ce = cudaMalloc(&ctx->d_dense, per_layer * cfg->num_layers)) != cudaSuccess)
        return fail(ce, "cudaMalloc(dense)");
    if ((ce = cudaMemset(ctx->d_dense, 0, per_layer * cfg->num_layers)) != cudaSuccess)
        return fail(ce, "cudaMemset(dense)");
    if ((ce = cudaMalloc(&ctx->d_err, sizeof(int) * 4)) != cudaSuccess) return fail(ce, "cudaMalloc(err)");
    if ((ce = cudaMemset(ctx->d_err, 0, sizeof(int) * 4)) != cudaSuccess) return fail(ce, "cudaMemset(err)");
    ctx->loaded.assign(cfg->num_layers, 0);
    ctx->dense_set.assign(cfg->num_layers, 0);
    int bst = nmoe_fused_init(ctx);
    if (bst != NMOE_OK) {
        snprintf(g_create_error, sizeof g_create_error, "decode kernel init: %.400s", ctx->last_error);
        *st = bst;
        nmoe_moe_destroy(ctx);
        return nullptr;
    }
    bst = nmoe_batched_init(ctx);
    if (bst != NMOE_OK) {
        snprintf(g_create_error, sizeof g_create_error, "batched init: %.400s", ctx->last_error);
        *st = bst;
        nmoe_moe_destroy(ctx);
        return nullptr;
    }
    ctx->prefetch_next = (cfg->flags & NMOE_FLAG_PREFETCH_NEXT_LAYER) != 0;
    if (const char *pf = getenv("NMOE_PREFETCH_NEXT")) ctx->prefetch_next = atoi(pf) != 0;
    *st = NMOE_OK;
    return ctx;
}

extern "C" void nmoe_moe_destroy(nmoe_moe_ctx *ctx) {
    if (ctx == nullptr) return;
    DeviceGuard guard(ctx->device);
    nmoe_batched_destroy(ctx);
    nmoe_fused_destroy(ctx);
    if (ctx->d_experts) cudaFree(ctx->d_experts);
    if (ctx->d_dense) cudaFree(ctx->d_dense);
    if (ctx->d_err) cudaFree(ctx->d_err);
    delete ctx;
}

// ---------------------------------------------------------------- loading ----

// Converter-layout blobs in device memory -> this layer's kernel-layout slot.
static cudaError_t repack_layer(nmoe_moe_ctx *ctx, int layer, const uint8_t *stage) {
    cudaError_t e = repack_experts(stage, ctx->d_experts + (size_t)layer * ctx->expert_layer_bytes, ctx->n_local,
                                   ctx->cfg.quant_bits, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    return e;
}

// CRC-32C of this rank's staged experts, checked against expected[] (global expert ids)
// and written to crc_out[] (global ids; entries of experts this rank does not hold are
// left as they are). NMOE_ECHECKSUM names the first mismatching expert.
static int check_staged(nmoe_moe_ctx *ctx, int layer, const uint8_t *d_stage, const uint32_t *expected,
                        uint32_t *crc_out) {
    if (expected == nullptr && crc_out == nullptr) return NMOE_OK;
    uint32_t *d_crc = nullptr;
    NMOE_CUDA_TRY(ctx, cudaMalloc(&d_crc, (size_t)ctx->n_local * sizeof(uint32_t)));
    std::vector<uint32_t> h(ctx->n_local);
    cudaError_t e = crc32c_blobs(d_stage, ctx->esz, ctx->n_local, d_crc, 0);
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), d_crc, h.size() * sizeof(uint32_t), cudaMemcpyDeviceToHost);
    cudaFree(d_crc);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "crc32c");
    for (int i = 0; i < ctx->n_local; ++i) {
        const int ge = ctx->expert_lo + i;
        if (crc_out) crc_out[ge] = h[i];
    }
    if (expected)
        for (int i = 0; i < ctx->n_local; ++i) {
            const int ge = ctx->expert_lo + i;
            if (h[i] != expected[ge]) {
                nmoe_ctx_set_error(ctx, "layer %d expert %d: CRC-32C 0x%08x, expected 0x%08x", layer, ge, h[i],
                                   expected[ge]);
                return NMOE_ECHECKSUM;
            }
        }
    return NMOE_OK;
}

extern "C" int nmoe_moe_load_layer_checked(nmoe_moe_ctx *ctx, int layer, const void *layer_bin, size_t bytes,
                                           const uint32_t *expected_crc, uint32_t *crc_out) {
    if (ctx == nullptr) return NMOE_EINVAL;
    if (layer < 0 || layer >= ctx->cfg.num_layers) {
        nmoe_ctx_set_error(ctx, "layer %d out of range [0, %d)", layer, ctx->cfg.num_layers);
        return NMOE_EINVAL;
    }
    const size_t want = (size_t)ctx->cfg.num_experts * ctx->esz;
    if (layer_bin == nullptr || bytes != want) {
        nmoe_ctx_set_error(ctx, "layer %d pack has %zu bytes, expected %d experts x %zu = %zu", layer, bytes,
                           ctx->cfg.num_experts, ctx->esz, want);
        return NMOE_ESIZE;
    }
    DeviceGuard guard(ctx->device);
    const uint8_t *src = static_cast<const uint8_t *>(layer_bin) + (size_t)ctx->expert_lo * ctx->esz;
    uint8_t *stage = nullptr;
    NMOE_CUDA_TRY(ctx, cudaMalloc(&stage, ctx->expert_layer_bytes));
    cudaError_t e = cudaMemcpy(stage, src, ctx->expert_layer_bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(stage);
        return cuda_fail(ctx, e, "load_layer");
    }
    int rc = check_staged(ctx, layer, stage, expected_crc, crc_out);
    if (rc == NMOE_OK) {
        e = repack_layer(ctx, layer, stage);
        if (e != cudaSuccess) rc = cuda_fail(ctx, e, "load_layer");
    }
    cudaFree(stage);
    if (rc == NMOE_OK) ctx->loaded[layer] = 1;
    return rc;
}

extern "C" int nmoe_moe_load_layer(nmoe_moe_ctx *ctx, int layer, const void *layer_bin, size_t bytes) {
    return nmoe_moe_load_layer_checked(ctx, layer, layer_bin, bytes, nullptr, nullptr);
}

extern "C" int nmoe_moe_load_layer_file_checked(nmoe_moe_ctx *ctx, int layer, const char *path,
                                                const uint32_t *expected_crc, uint32_t *crc_out) {
    if (ctx == nullptr || path == nullptr) return NMOE_EINVAL;
    if (layer < 0 || layer >= ctx->cfg.num_layers) {
        nmoe_ctx_set_error(ctx, "layer %d out of range [0, %d)", layer, ctx->cfg.num_layers);
        return NMOE_EINVAL;
    }
    FILE *f = fopen(path, "rb");
    if (f == nullptr) { nmoe_ctx_set_error(ctx, "cannot open %s", path); return NMOE_EIO; }
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    const size_t want = (size_t)ctx->cfg.num_experts * ctx->esz;
    if (sz < 0 || (size_t)sz != want) {
        fclose(f);
        nmoe_ctx_set_error(ctx, "%s has %ld bytes, expected %zu", path, sz, want);
        return NMOE_ESIZE;
    }
    // Stream this rank's slice through a pinned staging buffer.
    DeviceGuard guard(ctx->device);
    const size_t chunk = 64u << 20;
    void *stage = nullptr;
    if (cudaMallocHost(&stage, chunk) != cudaSuccess) { fclose(f); nmoe_ctx_set_error(ctx, "pinned alloc"); return NMOE_ENOMEM; }
    int rc = NMOE_OK;
    fseek(f, (long)((size_t)ctx->expert_lo * ctx->esz), SEEK_SET);
    uint8_t *dst = nullptr;
    if (cudaMalloc(&dst, ctx->expert_layer_bytes) != cudaSuccess) {
        cudaFreeHost(stage);
        fclose(f);
        nmoe_ctx_set_error(ctx, "device staging alloc");
        return NMOE_ENOMEM;
    }
    for (size_t done = 0; done < ctx->expert_layer_bytes && rc == NMOE_OK;) {
        const size_t n = std::min(chunk, ctx->expert_layer_bytes - done);
        if (fread(stage, 1, n, f) != n) { nmoe_ctx_set_error(ctx, "short read of %s", path); rc = NMOE_EIO; break; }
        cudaError_t e = cudaMemcpy(dst + done, stage, n, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) rc = cuda_fail(ctx, e, "cudaMemcpy(layer file)");
        done += n;
    }
    cudaFreeHost(stage);
    fclose(f);
    if (rc == NMOE_OK) rc = check_staged(ctx, layer, dst, expected_crc, crc_out);
    if (rc == NMOE_OK) {
        cudaError_t e = repack_layer(ctx, layer, dst);
        if (e != cudaSuccess) rc = cuda_fail(ctx, e, "repack");
    }
    cudaFree(dst);
    if (rc == NMOE_OK) ctx->loaded[layer] = 1;
    return rc;
}

extern "C" int nmoe_moe_load_layer_file(nmoe_moe_ctx *ctx, int layer, const char *path) {
    return nmoe_moe_load_layer_file_checked(ctx, layer, path, nullptr, nullptr);
}

extern "C" int nmoe_moe_set_dense(nmoe_moe_ctx *ctx, int layer, const nmoe_moe_dense_weights *w) {
    if (ctx == nullptr) return NMOE_EINVAL;
    if (w == nullptr || layer < 0 || layer >= ctx->cfg.num_layers) {
        nmoe_ctx_set_error(ctx, "set_dense: bad layer %d or null weights", layer);
        return NMOE_EINVAL;
    }
    const bool rq4 = ctx->cfg.router_dtype == NMOE_DTYPE_Q4, sq4 = ctx->cfg.shared_dtype == NMOE_DTYPE_Q4;
    const nmoe_tensor *src[5] = {&w->router, &w->shared_gate, &w->shared_up, &w->shared_down, &w->shared_gate_vec};
    for (int m = 0; m < 5; ++m) {
        const bool q4 = m == 0 ? rq4 : sq4;
        if (src[m]->weight == nullptr || (q4 && (src[m]->scales == nullptr || src[m]->biases == nullptr))) {
            nmoe_ctx_set_error(ctx, "set_dense: tensor %d missing weight/scales/biases", m);
            return NMOE_EINVAL;
        }
    }
    const DenseArena A = dense_arena(ctx->cfg.router_dtype, ctx->cfg.shared_dtype);
    std::vector<uint8_t> h(A.total, 0);
    // one row of a [rows][cols] matrix as [w | s | b] (q4) or [w] (bf16)
    auto put_row = [&](uint8_t *dst, const nmoe_tensor *t, bool q4, int row, int cols) {
        if (!q4) {
            memcpy(dst, static_cast<const uint8_t *>(t->weight) + (size_t)row * cols * 2, (size_t)cols * 2);
            return;
        }
        const size_t wb = cols / 2, sb = (cols / 64) * 2;
        memcpy(dst, static_cast<const uint8_t *>(t->weight) + row * wb, wb);
        memcpy(dst + wb, static_cast<const uint8_t *>(t->scales) + row * sb, sb);
        memcpy(dst + wb + sb, static_cast<const uint8_t *>(t->biases) + row * sb, sb);
    };
    for (int r = 0; r < NMOE_NUM_EXPERTS; ++r) put_row(&h[A.router + (size_t)r * A.rrow], src[0], rq4, r, NMOE_HIDDEN);
    for (int r = 0; r < NMOE_INTER; ++r) {
        uint8_t *pr = &h[A.spairs + (size_t)r * 2 * A.srow];
        if (!sq4) {
            put_row(pr, src[1], false, r, NMOE_HIDDEN);
            put_row(pr + A.srow, src[2], false, r, NMOE_HIDDEN);
        } else {   // [gate.w | up.w | gate.s | gate.b | up.s | up.b]
            memcpy(pr, static_cast<const uint8_t *>(src[1]->weight) + (size_t)r * 1024, 1024);
            memcpy(pr + 1024, static_cast<const uint8_t *>(src[2]->weight) + (size_t)r * 1024, 1024);
            memcpy(pr + 2048, static_cast<const uint8_t *>(src[1]->scales) + (size_t)r * 64, 64);
            memcpy(pr + 2112, static_cast<const uint8_t *>(src[1]->biases) + (size_t)r * 64, 64);
            memcpy(pr + 2176, static_cast<const uint8_t *>(src[2]->scales) + (size_t)r * 64, 64);
            memcpy(pr + 2240, static_cast<const uint8_t *>(src[2]->biases) + (size_t)r * 64, 64);
        }
    }
    put_row(&h[A.gvec], src[4], sq4, 0, NMOE_HIDDEN);
    for (int r = 0; r < NMOE_HIDDEN; ++r) put_row(&h[A.sdown + (size_t)r * A.sdrow], src[3], sq4, r, NMOE_INTER);
    // the shared down again by columns for the batch-1 kernel (nmoe_pack.cuh, sdown_t)
    if (!sq4) {
        const uint16_t *dw = static_cast<const uint16_t *>(src[3]->weight);
        uint16_t *t = reinterpret_cast<uint16_t *>(&h[A.sdown_t]);
        for (int r = 0; r < NMOE_HIDDEN; ++r)
            for (int c = 0; c < NMOE_INTER; ++c) t[(size_t)c * NMOE_HIDDEN + r] = dw[(size_t)r * NMOE_INTER + c];
    } else {
        const uint32_t *dw = static_cast<const uint32_t *>(src[3]->weight);   // [2048][64] words
        uint32_t *t = reinterpret_cast<uint32_t *>(&h[A.sdown_t]);             // [512][256] words
        for (int r = 0; r < NMOE_HIDDEN; ++r)
            for (int c = 0; c < NMOE_INTER; ++c) {
                const uint32_t q = (dw[(size_t)r * 64 + c / 8] >> (4 * (c % 8))) & 0xFu;
                t[(size_t)c * 256 + r / 8] |= q << (4 * (r % 8));
            }
        const uint16_t *ss = static_cast<const uint16_t *>(src[3]->scales);
        const uint16_t *sb = static_cast<const uint16_t *>(src[3]->biases);
        uint16_t *ts = reinterpret_cast<uint16_t *>(&h[A.sdown_t + 512 * 1024]);
        for (int g = 0; g < 8; ++g)
            for (int r = 0; r < NMOE_HIDDEN; ++r) {
                ts[g * NMOE_HIDDEN + r] = ss[r * 8 + g];
                ts[8 * NMOE_HIDDEN + g * NMOE_HIDDEN + r] = sb[r * 8 + g];
            }
    }
    DeviceGuard guard(ctx->device);
    NMOE_CUDA_TRY(ctx, cudaMemcpy(ctx->d_dense + (size_t)layer * ctx->dense_layer_bytes, h.data(), A.total,
                                  cudaMemcpyHostToDevice));
    ctx->dense_set[layer] = 1;
    return NMOE_OK;
}

// ---------------------------------------------------------------- forward ----

int nmoe_ctx_check_call(nmoe_moe_ctx *ctx, int layer, int k, int x_dtype) {
    if (ctx == nullptr) return NMOE_EINVAL;
    if (layer < 0 || layer >= ctx->cfg.num_layers) {
        nmoe_ctx_set_error(ctx, "layer %d out of range [0, %d)", layer, ctx->cfg.num_layers);
        return NMOE_EINVAL;
    }
    if (k < 1 || k > ctx->cfg.k_max) {
        nmoe_ctx_set_error(ctx, "k=%d outside [1, k_max=%d]", k, ctx->cfg.k_max);
        return NMOE_EINVAL;
    }
    if (x_dtype != NMOE_DTYPE_BF16 && x_dtype != NMOE_DTYPE_F32) {
        nmoe_ctx_set_error(ctx, "x_dtype must be NMOE_DTYPE_BF16 or NMOE_DTYPE_F32");
        return NMOE_EINVAL;
    }
    if (!ctx->loaded[layer] || !ctx->dense_set[layer]) {
        nmoe_ctx_set_error(ctx, "layer %d weights not uploaded (load_layer / set_dense)", layer);
        return NMOE_EINVAL;
    }
    return NMOE_OK;
}

static FusedCall make_call(nmoe_moe_ctx *ctx, int layer, int k, const void *x, int x_dtype, const float *h_mid,
                           float *out, uint32_t *idx_out, float *w_out, float *logits_out, int route_only) {
    const DenseArena A = dense_arena(ctx->cfg.router_dtype, ctx->cfg.shared_dtype);
    const uint8_t *d = ctx->d_dense + (size_t)layer * ctx->dense_layer_bytes;
    FusedCall a;
    a.experts = ctx->d_experts + (size_t)layer * ctx->expert_layer_bytes;
    a.router = d + A.router;
    a.spairs = d + A.spairs;
    a.gvec = d + A.gvec;
    a.sdown_t = d + A.sdown_t;
    a.x = x;
    a.x_f32 = x_dtype == NMOE_DTYPE_F32;
    a.h_mid = h_mid;
    a.out = out;
    a.idx_out = idx_out;
    a.w_out = w_out;
    a.logits_out = logits_out;
    a.k = k;
    a.num_experts = ctx->cfg.num_experts;
    a.route_only = route_only;
    a.err = ctx->d_err;
    a.next_dense = nullptr;
    a.next_dense_bytes = 0;
    if (ctx->prefetch_next && !route_only) {
        const int nl = (layer + 1) % ctx->cfg.num_layers;
        a.next_dense = ctx->d_dense + (size_t)nl * ctx->dense_layer_bytes;
        a.next_dense_bytes = (uint32_t)ctx->dense_layer_bytes;
    }
    return a;
}

extern "C" int nmoe_moe_forward(nmoe_moe_ctx *ctx, int layer, int k, const void *x, int x_dtype,
                                const float *h_mid, float *out, uint32_t *idx_out, float *w_out, void *stream) {
    int rc = nmoe_ctx_check_call(ctx, layer, k, x_dtype);
    if (rc != NMOE_OK) return rc;
    if (x == nullptr || out == nullptr) { nmoe_ctx_set_error(ctx, "x and out are required"); return NMOE_EINVAL; }
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0) { nmoe_ctx_set_error(ctx, "x must be 16-byte aligned"); return NMOE_EINVAL; }
    if (ctx->cfg.world_size > 1) {
        nmoe_ctx_set_error(ctx, "batch-1 decode runs on replicas (world_size 1); use forward_batched for EP");
        return NMOE_EINVAL;
    }
    DeviceGuard guard(ctx->device);
    cudaError_t e = nmoe_fused_launch(ctx, make_call(ctx, layer, k, x, x_dtype, h_mid, out, idx_out, w_out, nullptr, 0),
                                      static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "decode launch");
    return NMOE_OK;
}

extern "C" int nmoe_moe_route(nmoe_moe_ctx *ctx, int layer, int k, const void *x, int x_dtype, float *logits_out,
                              uint32_t *idx_out, float *w_out, void *stream) {
    int rc = nmoe_ctx_check_call(ctx, layer, k, x_dtype);
    if (rc != NMOE_OK) return rc;
    if (x == nullptr) { nmoe_ctx_set_error(ctx, "x is required"); return NMOE_EINVAL; }
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0) { nmoe_ctx_set_error(ctx, "x must be 16-byte aligned"); return NMOE_EINVAL; }
    DeviceGuard guard(ctx->device);
    // the same kernel, stopped after routing: the same fp32 logits as nmoe_moe_forward
    cudaError_t e = nmoe_fused_launch(ctx, make_call(ctx, layer, k, x, x_dtype, nullptr, nullptr, idx_out, w_out,
                                                     logits_out, 1),
                                      static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "route launch");
    return NMOE_OK;
}

extern "C" int nmoe_moe_device_status(nmoe_moe_ctx *ctx, int *code) {
    if (ctx == nullptr) return NMOE_EINVAL;
    DeviceGuard guard(ctx->device);
    int h[4] = {0, 0, 0, 0};
    NMOE_CUDA_TRY(ctx, cudaDeviceSynchronize());
    NMOE_CUDA_TRY(ctx, cudaMemcpy(h, ctx->d_err, sizeof h, cudaMemcpyDeviceToHost));
    NMOE_CUDA_TRY(ctx, cudaMemset(ctx->d_err, 0, sizeof h));
    if (code) *code = h[0];
    if (h[0] != 0) {
        nmoe_ctx_set_error(ctx, "device error word = %d (%s)", h[0],
                           h[0] == kErrExpertRange ? "routed expert id out of range" :
                           h[0] == kErrTimeout ? "bounded wait expired" : "unknown");
        return h[0] == kErrTimeout ? NMOE_ETIMEOUT : NMOE_EDEVICE;
    }
    return NMOE_OK;
}
