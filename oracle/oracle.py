"""ctypes bindings for the CPU oracle (oracle/libnmoe_oracle.so) -- TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline and the reference
arm) may import this module; the product path never does.  It also wraps the
reference's own src/math.m compiled unchanged into oracle/_ref/ when that library
exists (built in the development container by `make -C oracle ref`).

Also holds the seeded synthetic-weight generators shared by tests and bench.py:
weights are drawn bf16 ~N(0, 0.02) and quantised by the restated
scripts/convert_qwen36.py quantiser (orc_quantize_rows).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnmoe_oracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libnmoe_math_ref.so")

HIDDEN, INTER, EXPERTS, GROUP, MAX_K = 2048, 512, 256, 64, 8
DTYPE_BF16, DTYPE_Q4, DTYPE_Q2 = 1, 4, 2

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build(quiet: bool = True) -> None:
    """Compile the oracle (and the reference math.m when the reference tree exists)."""
    out = subprocess.DEVNULL if quiet else None
    subprocess.run(["make", "-C", HERE, "all"], check=True, stdout=out)
    ref_root = os.environ.get("NMOE_REF_ROOT", "/root/reference")
    if os.path.isfile(os.path.join(ref_root, "src", "math.m")):
        subprocess.run(["make", "-C", HERE, "ref", f"REF_ROOT={ref_root}"], check=True, stdout=out)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_bf16_to_f32.restype = C.c_float
        L.orc_bf16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_f32_to_bf16.argtypes = [C.c_float]
        L.orc_f32_to_bf16_array.argtypes = [_f32p, _u16p, C.c_size_t]
        L.orc_quantize_rows.restype = C.c_int
        L.orc_quantize_rows.argtypes = [_u16p, C.c_size_t, C.c_size_t, C.c_int, _u32p, _u16p, _u16p]
        L.orc_expert_size.restype = C.c_size_t
        L.orc_expert_size.argtypes = [C.c_int]
        L.orc_expert_offsets.restype = C.c_int
        L.orc_expert_offsets.argtypes = [C.c_int, C.POINTER(C.c_size_t)]
        L.orc_pack_expert.restype = C.c_int
        L.orc_pack_expert.argtypes = [_u16p, _u16p, C.c_int, _u8p]
        L.orc_sigmoid_cpu.restype = C.c_float
        L.orc_sigmoid_cpu.argtypes = [C.c_float]
        L.orc_sigmoid_kernel.restype = C.c_float
        L.orc_sigmoid_kernel.argtypes = [C.c_float]
        L.orc_softmax.argtypes = [_f32p, C.c_size_t]
        L.orc_topk.restype = C.c_size_t
        L.orc_topk.argtypes = [_f32p, C.c_size_t, C.c_size_t, _u32p, _f32p]
        L.orc_renormalize.argtypes = [_f32p, C.c_size_t]
        L.orc_swiglu.argtypes = [_f32p, _f32p, _f32p, C.c_size_t]
        L.orc_dequant_matvec_seq.argtypes = [_u32p, _u16p, _u16p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_int]
        L.orc_dequant_matvec.argtypes = [_u32p, _u16p, _u16p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_int, C.c_int]
        L.orc_bf16_matvec.argtypes = [_u16p, _f32p, _f32p, C.c_size_t, C.c_size_t]
        L.orc_expert_gate_up.argtypes = [_u8p, C.c_int, _f32p, _f32p]
        L.orc_expert_down.argtypes = [_u8p, C.c_int, _f32p, _f32p]
        L.orc_moe_block_forward.restype = C.c_int
        L.orc_moe_block_forward.argtypes = [C.POINTER(OrcLayer), C.c_int, _f32p, C.c_void_p, C.c_void_p,
                                            C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_moe_block_forward_batched.restype = C.c_int
        L.orc_moe_block_forward_batched.argtypes = [C.POINTER(OrcLayer), C.c_int, C.c_int, _f32p, C.c_void_p,
                                                    _f32p, C.c_void_p, C.c_void_p]
        L.orc_rms_norm.argtypes = [_f32p, C.c_void_p, _f32p, C.c_size_t, C.c_float, C.c_int]
        L.orc_argmax_top1.restype = C.c_uint32
        L.orc_argmax_top1.argtypes = [_f32p, C.c_size_t]
        L.orc_lm_head_argmax.restype = C.c_uint32
        L.orc_lm_head_argmax.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t,
                                         _f32p, C.c_void_p, C.c_float, C.c_int, C.c_void_p]
        L.orc_crc32c.restype = C.c_uint32
        L.orc_crc32c.argtypes = [C.c_uint32, C.c_void_p, C.c_size_t]
        L.orc_linear_attn_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _u16p, _f32p, _u16p, _u16p, _f32p, _f32p,
                                           _f32p]
        L.orc_full_attn_step.argtypes = [_f32p, _f32p, _f32p, _u16p, _u16p, _f32p, _f32p, C.c_int, _f32p]
        L.orc_full_attn_step_bf16kv.argtypes = L.orc_full_attn_step.argtypes
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        _lib = L
    return _lib


def ref_lib():
    """The reference's src/math.m compiled as C, or None when it was not built here."""
    if not os.path.exists(REF_LIB_PATH):
        return None
    L = C.CDLL(REF_LIB_PATH)
    L.nmoe_cpu_softmax.argtypes = [_f32p, C.c_size_t]
    L.nmoe_cpu_topk.restype = C.c_size_t
    L.nmoe_cpu_topk.argtypes = [_f32p, C.c_size_t, C.c_size_t, np.ctypeslib.ndpointer(np.uint64), _f32p]
    L.nmoe_cpu_renormalize.argtypes = [_f32p, C.c_size_t]
    L.nmoe_cpu_swiglu.argtypes = [_f32p, _f32p, _f32p, C.c_size_t]
    L.nmoe_cpu_sigmoid.restype = C.c_float
    L.nmoe_cpu_sigmoid.argtypes = [C.c_float]
    L.nmoe_cpu_dequant_matvec.argtypes = [_u32p, _u16p, _u16p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_int]
    L.nmoe_cpu_rms_norm.argtypes = [_f32p, C.c_void_p, _f32p, C.c_size_t, C.c_float, C.c_int]
    L.nmoe_f32_to_bf16.restype = C.c_uint16
    L.nmoe_f32_to_bf16.argtypes = [C.c_float]
    return L


class OrcDense(C.Structure):
    _fields_ = [("dtype", C.c_int), ("weight", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p)]


class OrcLayer(C.Structure):
    _fields_ = [("bits", C.c_int), ("experts", C.c_void_p), ("num_experts", C.c_size_t),
                ("router", OrcDense), ("shared_gate", OrcDense), ("shared_up", OrcDense),
                ("shared_down", OrcDense), ("shared_gate_vec", OrcDense)]


# ------------------------------------------------------------------ helpers ----

def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def quantize_rows(rows_bf16: np.ndarray, bits: int):
    rows_bf16 = np.ascontiguousarray(rows_bf16, dtype=np.uint16)
    r, c = rows_bf16.shape
    packed = np.zeros((r, c * bits // 32), np.uint32)
    scales = np.zeros((r, c // GROUP), np.uint16)
    biases = np.zeros((r, c // GROUP), np.uint16)
    rc = lib().orc_quantize_rows(rows_bf16, r, c, bits, packed, scales, biases)
    if rc != 0:
        raise ValueError("orc_quantize_rows failed")
    return packed, scales, biases


def expert_size(bits: int) -> int:
    return int(lib().orc_expert_size(bits))


def expert_offsets(bits: int):
    arr = (C.c_size_t * 9)()
    if lib().orc_expert_offsets(bits, arr) != 0:
        raise ValueError(bits)
    return [int(v) for v in arr]


def pack_expert(gate_up_bf16: np.ndarray, down_bf16: np.ndarray, bits: int) -> np.ndarray:
    blob = np.zeros(expert_size(bits), np.uint8)
    rc = lib().orc_pack_expert(np.ascontiguousarray(gate_up_bf16, np.uint16),
                               np.ascontiguousarray(down_bf16, np.uint16), bits, blob)
    if rc != 0:
        raise ValueError("orc_pack_expert failed")
    return blob


def randn_bf16(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    return f32_to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def _dense_bf16_or_q4(rng, shape, dtype, std=0.02):
    w = randn_bf16(rng, shape, std)
    if dtype == DTYPE_BF16:
        return {"dtype": DTYPE_BF16, "weight": w}
    p, s, b = quantize_rows(w, 4)
    return {"dtype": DTYPE_Q4, "weight": p, "scales": s, "biases": b}


@dataclass
class LayerWeights:
    """One synthetic MoE layer: expert packs (layer_XX.bin image) + router/shared weights."""
    bits: int
    experts: np.ndarray          # uint8 [num_experts * expert_size]
    num_experts: int
    router: dict
    shared_gate: dict
    shared_up: dict
    shared_down: dict
    shared_gate_vec: dict
    router_bias: np.ndarray | None = None   # optional per-expert logit offset (skewed routing)
    _keep: list = field(default_factory=list)

    def orc(self) -> OrcLayer:
        def dense(d):
            out = OrcDense(d["dtype"], d["weight"].ctypes.data, 0, 0)
            if d["dtype"] == DTYPE_Q4:
                out.scales = d["scales"].ctypes.data
                out.biases = d["biases"].ctypes.data
            return out
        L = OrcLayer(self.bits, self.experts.ctypes.data, self.num_experts, dense(self.router),
                     dense(self.shared_gate), dense(self.shared_up), dense(self.shared_down),
                     dense(self.shared_gate_vec))
        return L


def make_layer(seed: int, bits: int = 4, router_dtype: int = DTYPE_BF16, shared_dtype: int = DTYPE_BF16,
               num_experts: int = EXPERTS, distinct_experts: int | None = None) -> LayerWeights:
    """Seeded synthetic layer (BASELINE config 0/1 distributions).

    Experts: gate_up [1024,2048] and down [2048,512] bf16 ~N(0,0.02) quantised by the
    restated convert_qwen36.py quantiser.  `distinct_experts` (default: all) bounds the
    host cost: expert e reuses the pack of e % distinct_experts (tests use this to stay
    fast; routing still addresses all `num_experts` slots).
    """
    rng = np.random.default_rng(seed)
    esz = expert_size(bits)
    nd = num_experts if distinct_experts is None else max(1, min(distinct_experts, num_experts))
    packs = []
    for _ in range(nd):
        gu = randn_bf16(rng, (2 * INTER, HIDDEN), 0.02)
        dn = randn_bf16(rng, (HIDDEN, INTER), 0.02)
        packs.append(pack_expert(gu, dn, bits))
    experts = np.empty(num_experts * esz, np.uint8)
    for e in range(num_experts):
        experts[e * esz:(e + 1) * esz] = packs[e % nd]
    return LayerWeights(
        bits=bits, experts=experts, num_experts=num_experts,
        router=_dense_bf16_or_q4(rng, (EXPERTS, HIDDEN), router_dtype),
        shared_gate=_dense_bf16_or_q4(rng, (INTER, HIDDEN), shared_dtype),
        shared_up=_dense_bf16_or_q4(rng, (INTER, HIDDEN), shared_dtype),
        shared_down=_dense_bf16_or_q4(rng, (HIDDEN, INTER), shared_dtype),
        shared_gate_vec=_dense_bf16_or_q4(rng, (1, HIDDEN), shared_dtype),
    )


def block_forward(layer: LayerWeights, k: int, x: np.ndarray, h_mid: np.ndarray | None = None,
                  logits_override: np.ndarray | None = None):
    """One token through the oracle block. Returns dict(out, idx, w, logits, shared_act, score)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(HIDDEN, np.float32)
    idx = np.zeros(MAX_K, np.uint32)
    w = np.zeros(MAX_K, np.float32)
    logits = np.zeros(EXPERTS, np.float32)
    sact = np.zeros(INTER, np.float32)
    score = np.zeros(1, np.float32)
    hm = None if h_mid is None else np.ascontiguousarray(h_mid, np.float32)
    lo = None if logits_override is None else np.ascontiguousarray(logits_override, np.float32)
    L = layer.orc()
    rc = lib().orc_moe_block_forward(C.byref(L), k, x, None if hm is None else hm.ctypes.data,
                                     None if lo is None else lo.ctypes.data, out.ctypes.data,
                                     idx.ctypes.data, w.ctypes.data, logits.ctypes.data,
                                     sact.ctypes.data, score.ctypes.data)
    if rc != 0:
        raise ValueError(f"orc_moe_block_forward rc={rc}")
    return {"out": out, "idx": idx, "w": w, "logits": logits, "shared_act": sact, "score": float(score[0])}


def block_forward_batched(layer: LayerWeights, k: int, x: np.ndarray, h_mid: np.ndarray | None = None):
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    out = np.zeros((T, HIDDEN), np.float32)
    idx = np.zeros((T, MAX_K), np.uint32)
    w = np.zeros((T, MAX_K), np.float32)
    hm = None if h_mid is None else np.ascontiguousarray(h_mid, np.float32)
    L = layer.orc()
    rc = lib().orc_moe_block_forward_batched(C.byref(L), T, k, x, None if hm is None else hm.ctypes.data,
                                             out, idx.ctypes.data, w.ctypes.data)
    if rc != 0:
        raise ValueError(f"orc_moe_block_forward_batched rc={rc}")
    return {"out": out, "idx": idx, "w": w}


def route_reference(logits: np.ndarray, k: int):
    """Softmax -> top-k -> renormalise exactly as NMOESelectRouteTopKCPU (src/runtime.m:1498-1511)."""
    p = np.array(logits, np.float32, copy=True)
    L = lib()
    L.orc_softmax(p, p.size)
    idx = np.zeros(k, np.uint32)
    vals = np.zeros(k, np.float32)
    n = L.orc_topk(p, p.size, k, idx, vals)
    L.orc_renormalize(vals, n)
    return idx[:n], vals[:n]


# ------------------------------------------------------------------ LM head ----

def rms_norm(x: np.ndarray, w_bf16: np.ndarray | None, eps: float = 1e-6, add_one: bool = True) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    w = None if w_bf16 is None else np.ascontiguousarray(w_bf16, np.uint16)
    lib().orc_rms_norm(x, None if w is None else w.ctypes.data, out, x.size, eps, int(add_one))
    return out


def argmax_top1(v: np.ndarray) -> int:
    return int(lib().orc_argmax_top1(np.ascontiguousarray(v, np.float32), v.size))


@dataclass
class LmHead:
    """Synthetic LM head (lm_head.weight [vocab][2048]) in the converter's q4 form or bf16."""
    dtype: int
    vocab: int
    weight: np.ndarray                 # q4: u32 [vocab][256]; bf16: u16 [vocab][2048]
    scales: np.ndarray | None = None   # q4: u16 [vocab][32]
    biases: np.ndarray | None = None


def make_lm_head(seed: int, vocab: int, dtype: int = DTYPE_Q4, std: float = 0.02) -> LmHead:
    rng = np.random.default_rng(seed)
    w = randn_bf16(rng, (vocab, HIDDEN), std)
    if dtype == DTYPE_BF16:
        return LmHead(dtype, vocab, w)
    p, sc, b = quantize_rows(w, 4)
    return LmHead(dtype, vocab, p, sc, b)


def lm_head_argmax(head: LmHead, x: np.ndarray, norm_w: np.ndarray | None = None, eps: float = 1e-6,
                   add_one: bool = True):
    """(token, logits fp32[vocab]) by the reference's head and top-1 rule."""
    x = np.ascontiguousarray(x, np.float32)
    logits = np.empty(head.vocab, np.float32)
    nw = None if norm_w is None else np.ascontiguousarray(norm_w, np.uint16)
    tok = lib().orc_lm_head_argmax(head.dtype, head.weight.ctypes.data,
                                   None if head.scales is None else head.scales.ctypes.data,
                                   None if head.biases is None else head.biases.ctypes.data,
                                   head.vocab, HIDDEN, x, None if nw is None else nw.ctypes.data, eps,
                                   int(add_one), logits.ctypes.data)
    return int(tok), logits


def crc32c(data, crc: int = 0) -> int:
    """CRC-32C of a bytes-like / numpy buffer (bitwise definition)."""
    a = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray)) else data).view(np.uint8)
    return int(lib().orc_crc32c(crc, a.ctypes.data, a.nbytes))


# ------------------------------------------------------- linear attention ----

def make_linear_attn(seed: int):
    """Seeded linear-attention weights and step inputs at Qwen3.6 geometry."""
    rng = np.random.default_rng(seed)
    w = {"conv_w": randn_bf16(rng, (8192, 4), 0.3),
         "A_log": (rng.standard_normal(32) * 0.5).astype(np.float32),
         "dt_bias": randn_bf16(rng, (32,), 0.5),
         "norm_w": f32_to_bf16(1.0 + rng.standard_normal(128).astype(np.float32) * 0.1)}
    return w


def linear_attn_inputs(rng):
    return {"qkv": rng.standard_normal(8192).astype(np.float32),
            "z": rng.standard_normal(4096).astype(np.float32),
            "alpha": rng.standard_normal(32).astype(np.float32),
            "beta": rng.standard_normal(32).astype(np.float32)}


def linear_attn_step(w, inp, conv_state, delta_state):
    """One step by the reference kernels' sequence; states updated in place; returns out[4096]."""
    out = np.zeros(4096, np.float32)
    lib().orc_linear_attn_step(inp["qkv"], inp["z"], inp["alpha"], inp["beta"], w["conv_w"].reshape(-1),
                               w["A_log"], w["dt_bias"], w["norm_w"], conv_state.reshape(-1),
                               delta_state.reshape(-1), out)
    return out


def full_attn_step(q, k_new, v_new, q_norm, k_norm, k_cache, v_cache, position, bf16_kv: bool = False):
    """One full-attention decode step by the reference's sequence; caches updated. bf16_kv:
    the caches hold bf16 values (f32 arrays) and the appended rows are rounded to bf16."""
    out = np.zeros(16 * 256, np.float32)
    fn = lib().orc_full_attn_step_bf16kv if bf16_kv else lib().orc_full_attn_step
    fn(np.ascontiguousarray(q, np.float32).reshape(-1), k_new.reshape(-1), v_new.reshape(-1),
                             q_norm, k_norm, k_cache.reshape(-1), v_cache.reshape(-1), int(position), out)
    return out


# ------------------------------------------------------------ whole decode step ----

def _q4(rng, rows, cols, std=0.02):
    p, s, b = quantize_rows(randn_bf16(rng, (rows, cols), std), 4)
    return {"weight": p, "scales": s, "biases": b, "rows": rows, "cols": cols}


def make_decoder_weights(seed: int, num_layers: int, vocab: int, head_dtype: int = DTYPE_Q4,
                         embed_dtype: int = DTYPE_Q4):
    """Seeded synthetic attention / norm / embedding / head weights of the 40-layer model
    (all weights ~N(0, 0.02), projections q4 as the reference's converter
    writes them); layer l is full attention when (l + 1) % 4 == 0."""
    rng = np.random.default_rng(seed)
    layers = []
    for l in range(num_layers):
        norms = {"input_norm": randn_bf16(rng, (HIDDEN,), 0.02), "post_norm": randn_bf16(rng, (HIDDEN,), 0.02)}
        if (l + 1) % 4 == 0:
            layers.append({"kind": "full", **norms, "q": _q4(rng, 8192, 2048), "k": _q4(rng, 512, 2048),
                           "v": _q4(rng, 512, 2048), "o": _q4(rng, 2048, 4096),
                           "q_norm": randn_bf16(rng, (256,), 0.02), "k_norm": randn_bf16(rng, (256,), 0.02)})
        else:
            la = make_linear_attn(int(rng.integers(1 << 30)))
            layers.append({"kind": "linear", **norms, "qkv": _q4(rng, 8192, 2048), "z": _q4(rng, 4096, 2048),
                           "beta": _q4(rng, 32, 2048), "alpha": _q4(rng, 32, 2048), "out": _q4(rng, 2048, 4096),
                           **la})
    def table(dtype):
        w = randn_bf16(rng, (vocab, HIDDEN), 0.02)
        if dtype == DTYPE_BF16:
            return {"dtype": DTYPE_BF16, "weight": w}
        p, s, b = quantize_rows(w, 4)
        return {"dtype": DTYPE_Q4, "weight": p, "scales": s, "biases": b}
    g = {"vocab": vocab, "embed": table(embed_dtype), "final_norm": randn_bf16(rng, (HIDDEN,), 0.02),
         "lm_head": table(head_dtype)}
    return layers, g


def _matvec(m, x):
    y = np.zeros(m["rows"], np.float32)
    lib().orc_dequant_matvec(m["weight"].reshape(-1), m["scales"].reshape(-1), m["biases"].reshape(-1),
                             np.ascontiguousarray(x, np.float32), y, m["rows"], m["cols"], 4, 0)
    return y


class DecoderOracle:
    """NMOEProcessToken (src/runtime.m:3712-3805) restated with the oracle's pieces:
    embedding row, per layer input RMSNorm -> attention (linear_attn_step / full_attn_step,
    projections by the reference's dequant matvec, form 0) -> output projection + residual
    -> post RMSNorm -> MoE block (block_forward with h_mid), final RMSNorm + LM head."""

    def __init__(self, layers, g, moe_layers, k: int = 8, max_positions: int = 64):
        self.layers, self.g, self.moe, self.k = layers, g, moe_layers, k
        self.conv = [np.zeros((3, 8192), np.float32) for _ in layers]
        self.S = [np.zeros((32, 128, 128), np.float32) for _ in layers]
        self.kc = [np.zeros((max_positions, 2, 256), np.float32) for _ in layers]
        self.vc = [np.zeros((max_positions, 2, 256), np.float32) for _ in layers]

    def _embed(self, t):
        e = self.g["embed"]
        if e["dtype"] == DTYPE_BF16:
            return bf16_to_f32(e["weight"][t])
        q = np.stack([(e["weight"][t] >> (4 * i)) & 0xF for i in range(8)], 1).reshape(-1).astype(np.float32)
        s = np.repeat(bf16_to_f32(e["scales"][t]), 64)
        b = np.repeat(bf16_to_f32(e["biases"][t]), 64)
        return (q * s + b).astype(np.float32)

    def step(self, token: int, position: int):
        h = self._embed(token)
        for l, w in enumerate(self.layers):
            xn = rms_norm(h, w["input_norm"])
            if w["kind"] == "full":
                q, kk, vv = _matvec(w["q"], xn), _matvec(w["k"], xn), _matvec(w["v"], xn)
                a = full_attn_step(q, kk, vv, w["q_norm"], w["k_norm"], self.kc[l], self.vc[l], position)
                h2 = _matvec(w["o"], a) + h
            else:
                inp = {"qkv": _matvec(w["qkv"], xn), "z": _matvec(w["z"], xn), "beta": _matvec(w["beta"], xn),
                       "alpha": _matvec(w["alpha"], xn)}
                a = linear_attn_step(w, inp, self.conv[l], self.S[l])
                h2 = _matvec(w["out"], a) + h
            xn2 = rms_norm(h2, w["post_norm"])
            h = block_forward(self.moe[l], self.k, xn2, h_mid=h2)["out"]
        head = self.g["lm_head"]
        lh = LmHead(head["dtype"], self.g["vocab"], head["weight"], head.get("scales"), head.get("biases"))
        tok, logits = lm_head_argmax(lh, h, self.g["final_norm"])
        return tok, h, logits
