"""Python host binding of libnmoe_cuda.so (the C ABI declared in include/nmoe/moe_cuda.h).

The reference's host is Objective-C/C calling Metal; here the host-facing surface is
the C ABI, and this module is a thin ctypes mirror of it for Python callers (tests,
bench.py). Tensors passed to forward calls are device pointers (ints) or torch CUDA
tensors; weights passed to load/set calls are host numpy arrays.

There is no fallback: if the CUDA library is missing, `lib()` raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("NMOE_LIB") or os.path.join(HERE, "libnmoe_cuda.so")   # NMOE_LIB: another build

OK, EINVAL, ESIZE, ECUDA, ENCCL, ETIMEOUT, EDEVICE, EIO, ENOMEM, ECHECKSUM = range(10)
DTYPE_F32, DTYPE_BF16, DTYPE_Q2, DTYPE_Q4 = 0, 1, 2, 4
HIDDEN, INTER, NUM_EXPERTS, GROUP, MAX_K = 2048, 512, 256, 64, 8

# Every symbol include/nmoe/moe_cuda.h declares.
ABI_SYMBOLS = (
    "nmoe_moe_expert_size", "nmoe_moe_expert_offsets", "nmoe_moe_validate_layout_json",
    "nmoe_moe_strerror", "nmoe_moe_create", "nmoe_moe_destroy", "nmoe_moe_create_error", "nmoe_moe_last_error",
    "nmoe_moe_load_layer", "nmoe_moe_load_layer_file", "nmoe_moe_set_dense",
    "nmoe_moe_forward", "nmoe_moe_route", "nmoe_moe_forward_batched", "nmoe_moe_device_status",
    "nmoe_moe_forward_static", "nmoe_moe_static_error", "nmoe_moe_debug_trail", "nmoe_moe_debug_timeline",
    "nmoe_moe_debug_logits", "nmoe_moe_debug_gemm_trace", "nmoe_moe_nccl_unique_id", "nmoe_moe_decode_grid",
    "nmoe_moe_static_scratch_bytes", "nmoe_moe_static_status", "nmoe_moe_debug_ep_times",
    "nmoe_lm_head_argmax", "nmoe_lm_head_workspace_bytes", "nmoe_lm_head_error",
    "nmoe_moe_load_layer_checked", "nmoe_moe_load_layer_file_checked", "nmoe_crc32c", "nmoe_crc32c_combine",
    "nmoe_crc32c_device", "nmoe_linear_attn_step", "nmoe_full_attn_step", "nmoe_full_attn_workspace_bytes",
    "nmoe_full_attn_step_batched", "nmoe_linear_attn_step_batched", "nmoe_full_attn_batched_workspace_bytes",
    "nmoe_decoder_create", "nmoe_decoder_destroy", "nmoe_decoder_error", "nmoe_decoder_set_linear_layer",
    "nmoe_decoder_set_full_layer", "nmoe_decoder_set_globals", "nmoe_decoder_reset", "nmoe_decoder_step",
)


class NmoeError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"nmoe status {status}: {msg}")
        self.status = status


class Config(C.Structure):
    _fields_ = [("quant_bits", C.c_int), ("num_layers", C.c_int), ("num_experts", C.c_int),
                ("k_max", C.c_int), ("router_dtype", C.c_int), ("shared_dtype", C.c_int),
                ("t_max", C.c_int), ("world_size", C.c_int), ("rank", C.c_int),
                ("nccl_unique_id", C.c_void_p), ("flags", C.c_int)]

FLAG_PREFETCH_NEXT_LAYER, FLAG_EXPERT_FP32 = 1, 2


class Tensor(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p)]


class DenseWeights(C.Structure):
    _fields_ = [("router", Tensor), ("shared_gate", Tensor), ("shared_up", Tensor),
                ("shared_down", Tensor), ("shared_gate_vec", Tensor)]


class LinearAttnWeights(C.Structure):
    _fields_ = [("conv_w", C.c_void_p), ("A_log", C.c_void_p), ("dt_bias", C.c_void_p), ("norm_w", C.c_void_p)]


class FullAttnWeights(C.Structure):
    _fields_ = [("q_norm", C.c_void_p), ("k_norm", C.c_void_p)]


class LinearLayerHost(C.Structure):
    _fields_ = [("input_norm", C.c_void_p), ("post_norm", C.c_void_p), ("qkv", Tensor), ("z", Tensor),
                ("beta", Tensor), ("alpha", Tensor), ("out", Tensor), ("conv_w", C.c_void_p), ("A_log", C.c_void_p),
                ("dt_bias", C.c_void_p), ("norm_w", C.c_void_p)]


class FullLayerHost(C.Structure):
    _fields_ = [("input_norm", C.c_void_p), ("post_norm", C.c_void_p), ("q", Tensor), ("k", Tensor), ("v", Tensor),
                ("o", Tensor), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p)]


def build(quiet: bool = True) -> str:
    out = subprocess.DEVNULL if quiet else None
    subprocess.run(["make", "-C", HERE, "-j8", "all"], check=True, stdout=out)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` "
                           "(or __graft_entry__.build()); there is no CPU fallback")
    L = C.CDLL(LIB_PATH)
    vp, i, sz = C.c_void_p, C.c_int, C.c_size_t
    L.nmoe_moe_expert_size.restype = sz
    L.nmoe_moe_expert_size.argtypes = [i]
    L.nmoe_moe_expert_offsets.restype = i
    L.nmoe_moe_expert_offsets.argtypes = [i, C.POINTER(sz)]
    L.nmoe_moe_validate_layout_json.restype = i
    L.nmoe_moe_validate_layout_json.argtypes = [C.c_char_p, i, C.c_char_p, sz]
    L.nmoe_moe_strerror.restype = C.c_char_p
    L.nmoe_moe_strerror.argtypes = [i]
    L.nmoe_moe_create.restype = vp
    L.nmoe_moe_create.argtypes = [C.POINTER(Config), i, C.POINTER(i)]
    L.nmoe_moe_create_error.restype = C.c_char_p
    L.nmoe_moe_destroy.argtypes = [vp]
    L.nmoe_moe_last_error.restype = C.c_char_p
    L.nmoe_moe_last_error.argtypes = [vp]
    L.nmoe_moe_load_layer.restype = i
    L.nmoe_moe_load_layer.argtypes = [vp, i, vp, sz]
    L.nmoe_moe_load_layer_file.restype = i
    L.nmoe_moe_load_layer_file.argtypes = [vp, i, C.c_char_p]
    L.nmoe_moe_set_dense.restype = i
    L.nmoe_moe_set_dense.argtypes = [vp, i, C.POINTER(DenseWeights)]
    L.nmoe_moe_forward.restype = i
    L.nmoe_moe_forward.argtypes = [vp, i, i, vp, i, vp, vp, vp, vp, vp]
    L.nmoe_moe_route.restype = i
    L.nmoe_moe_route.argtypes = [vp, i, i, vp, i, vp, vp, vp, vp]
    L.nmoe_moe_forward_batched.restype = i
    L.nmoe_moe_forward_batched.argtypes = [vp, i, i, i, vp, i, vp, vp, i, vp, vp, vp]
    L.nmoe_moe_device_status.restype = i
    L.nmoe_moe_device_status.argtypes = [vp, C.POINTER(i)]
    L.nmoe_moe_forward_static.restype = i
    L.nmoe_moe_forward_static.argtypes = [vp, i, i, C.POINTER(DenseWeights), i, i, i, vp, i, vp, vp, vp, vp, vp]
    L.nmoe_moe_static_error.restype = C.c_char_p
    L.nmoe_moe_static_scratch_bytes.restype = sz
    L.nmoe_moe_static_status.restype = i
    L.nmoe_moe_static_status.argtypes = [C.POINTER(i), vp]
    L.nmoe_moe_debug_trail.restype = i
    L.nmoe_moe_debug_trail.argtypes = [vp, vp, i]
    L.nmoe_moe_debug_timeline.restype = i
    L.nmoe_moe_debug_timeline.argtypes = [vp, vp, i]
    L.nmoe_moe_decode_grid.restype = i
    L.nmoe_moe_decode_grid.argtypes = [vp]
    L.nmoe_moe_debug_ep_times.restype = i
    L.nmoe_moe_debug_ep_times.argtypes = [vp, vp]
    L.nmoe_moe_debug_logits.restype = i
    L.nmoe_moe_debug_logits.argtypes = [vp, vp, i]
    L.nmoe_moe_nccl_unique_id.restype = i
    L.nmoe_moe_nccl_unique_id.argtypes = [vp, sz]
    L.nmoe_moe_debug_gemm_trace.restype = i
    L.nmoe_moe_debug_gemm_trace.argtypes = [vp, vp, i]
    L.nmoe_moe_load_layer_checked.restype = i
    L.nmoe_moe_load_layer_checked.argtypes = [vp, i, vp, sz, vp, vp]
    L.nmoe_moe_load_layer_file_checked.restype = i
    L.nmoe_moe_load_layer_file_checked.argtypes = [vp, i, C.c_char_p, vp, vp]
    L.nmoe_crc32c.restype = C.c_uint32
    L.nmoe_crc32c.argtypes = [C.c_uint32, vp, sz]
    L.nmoe_crc32c_device.restype = i
    L.nmoe_crc32c_device.argtypes = [vp, sz, i, vp, vp]
    L.nmoe_crc32c_combine.restype = C.c_uint32
    L.nmoe_crc32c_combine.argtypes = [C.c_uint32, C.c_uint32, sz]
    L.nmoe_linear_attn_step.restype = i
    L.nmoe_linear_attn_step.argtypes = [C.POINTER(LinearAttnWeights), vp, vp, vp, vp, vp, vp, vp, vp]
    L.nmoe_full_attn_step.restype = i
    L.nmoe_full_attn_step.argtypes = [C.POINTER(FullAttnWeights), vp, vp, vp, vp, vp, i, i, vp, vp, vp]
    L.nmoe_full_attn_workspace_bytes.restype = sz
    L.nmoe_linear_attn_step_batched.restype = i
    L.nmoe_linear_attn_step_batched.argtypes = [C.POINTER(LinearAttnWeights), i, vp, vp, vp, vp, vp, vp, vp, vp]
    L.nmoe_full_attn_step_batched.restype = i
    L.nmoe_full_attn_step_batched.argtypes = [C.POINTER(FullAttnWeights), i, vp, vp, vp, vp, vp, vp, i, vp, vp, vp]
    L.nmoe_full_attn_batched_workspace_bytes.restype = sz
    L.nmoe_full_attn_batched_workspace_bytes.argtypes = [i]
    L.nmoe_decoder_create.restype = vp
    L.nmoe_decoder_create.argtypes = [vp, i, i, i, C.POINTER(i)]
    L.nmoe_decoder_destroy.argtypes = [vp]
    L.nmoe_decoder_error.restype = C.c_char_p
    L.nmoe_decoder_error.argtypes = [vp]
    L.nmoe_decoder_set_linear_layer.restype = i
    L.nmoe_decoder_set_linear_layer.argtypes = [vp, i, C.POINTER(LinearLayerHost)]
    L.nmoe_decoder_set_full_layer.restype = i
    L.nmoe_decoder_set_full_layer.argtypes = [vp, i, C.POINTER(FullLayerHost)]
    L.nmoe_decoder_set_globals.restype = i
    L.nmoe_decoder_set_globals.argtypes = [vp, i, i, C.POINTER(Tensor), vp, i, C.POINTER(Tensor)]
    L.nmoe_decoder_reset.restype = i
    L.nmoe_decoder_reset.argtypes = [vp, vp]
    L.nmoe_decoder_step.restype = i
    L.nmoe_decoder_step.argtypes = [vp, vp, i, vp, vp, vp]
    L.nmoe_lm_head_argmax.restype = i
    L.nmoe_lm_head_argmax.argtypes = [C.POINTER(Tensor), i, i, i, vp, i, vp, C.c_float, i, vp, vp, vp, vp]
    L.nmoe_lm_head_workspace_bytes.restype = sz
    L.nmoe_lm_head_error.restype = C.c_char_p
    _lib = L
    return L


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id for Context(world_size > 1, nccl_unique_id=...)."""
    buf = C.create_string_buffer(128)
    rc = lib().nmoe_moe_nccl_unique_id(buf, 128)
    if rc != OK:
        raise NmoeError(rc, "ncclGetUniqueId failed")
    return buf.raw


def expert_size(bits: int) -> int:
    return int(lib().nmoe_moe_expert_size(bits))


def expert_offsets(bits: int):
    arr = (C.c_size_t * 9)()
    rc = lib().nmoe_moe_expert_offsets(bits, arr)
    if rc != OK:
        raise NmoeError(rc, "bad quant_bits")
    return [int(v) for v in arr]


def validate_layout_json(path: str, bits: int):
    """Returns (status, message)."""
    buf = C.create_string_buffer(512)
    rc = lib().nmoe_moe_validate_layout_json(path.encode(), bits, buf, 512)
    return rc, buf.value.decode()


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _np_ptr(a) -> int | None:
    return None if a is None else a.ctypes.data


# Stamp slots of the batch-1 kernel's timeline (k_moe_decode_fused, NMOE_TIMELINE=1).
TIMELINE_WIDTH = 32
TIMELINE_SLOTS = {
    29: "prologue: indices computed", 30: "prologue: barriers initialised", 31: "prologue: copies issued",
    16: "dependency wait done",
    21: "x loaded (tid 0)",
    1: "x staged",
    18: "router rows ready (warp 0)",
    19: "router dot done (warp 0)",
    20: "last router unit done",
    8: "logits published",
    2: "router and shared rows done",
    13: "logits poll starts",
    22: "publication count complete",
    15: "logits seen",
    23: "top-k starts",
    24: "top-k lane sort done",
    25: "top-k round 0 done",
    6: "top-k ids done",
    17: "unit 0 copies issued",
    10: "routed copies issued",
    9: "top-k weights done",
    3: "routing barrier",
    12: "shared down done",
    11: "first unit landed",
    27: "warp 0 gate/up dots done (units 0-1)",
    28: "all warps' gate/up dots done (units 0-1)",
    26: "down columns landed (units 0-1)",
    14: "unit 0 gate/up done",
    5: "routed units done",
    7: "end",
}


def summarize_timeline(tl):
    """Decode a [CTA][slots] table of %globaltimer low words (slot 0 = CTA start, 0 = not
    reached) into {phase name: (min, median, max)} microseconds after the earliest start."""
    t = np.asarray(tl, np.int64)
    ref = t[:, 0][t[:, 0] > 0][0]

    def rel(v):   # signed difference of 32-bit stamp words (they wrap every ~4.3 s)
        d = (v - ref) & 0xFFFFFFFF
        return np.where(d >= 2**31, d - 2**32, d)

    t0 = rel(t[:, 0][t[:, 0] > 0]).min()
    out = {}
    for slot, name in TIMELINE_SLOTS.items():
        if slot >= t.shape[1]:
            continue
        v = t[:, slot]
        v = rel(v[v > 0]) - t0
        if v.size:
            out[name] = (v.min() / 1e3, float(np.median(v)) / 1e3, v.max() / 1e3)
    return out


class Context:
    """One nmoe_moe_ctx on one CUDA device."""

    def __init__(self, quant_bits=4, num_layers=1, num_experts=NUM_EXPERTS, k_max=8,
                 router_dtype=DTYPE_BF16, shared_dtype=DTYPE_BF16, t_max=0, device=0,
                 world_size=1, rank=0, nccl_unique_id: bytes | None = None, flags=0):
        self._L = lib()
        self._id_buf = None
        if nccl_unique_id is not None:
            self._id_buf = C.create_string_buffer(bytes(nccl_unique_id), 128)
        self.cfg = Config(quant_bits, num_layers, num_experts, k_max, router_dtype, shared_dtype, t_max,
                          world_size, rank, C.cast(self._id_buf, C.c_void_p) if self._id_buf else None, flags)
        st = C.c_int(0)
        h = self._L.nmoe_moe_create(C.byref(self.cfg), device, C.byref(st))
        if not h:
            raise NmoeError(st.value, self._L.nmoe_moe_create_error().decode())
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            self._L.nmoe_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc != OK:
            raise NmoeError(rc, self._L.nmoe_moe_last_error(self.h).decode())

    def load_layer(self, layer: int, layer_bin: np.ndarray):
        a = np.ascontiguousarray(layer_bin).view(np.uint8)
        self._check(self._L.nmoe_moe_load_layer(self.h, layer, a.ctypes.data, a.nbytes))

    def load_layer_file(self, layer: int, path: str):
        self._check(self._L.nmoe_moe_load_layer_file(self.h, layer, path.encode()))

    def load_layer_checked(self, layer: int, layer_bin: np.ndarray, expected=None):
        """Load with the device CRC-32C check; returns the per-expert CRCs (uint32[num_experts])."""
        a = np.ascontiguousarray(layer_bin).view(np.uint8)
        out = np.zeros(self.cfg.num_experts, np.uint32)
        exp = None if expected is None else np.ascontiguousarray(expected, np.uint32)
        self._check(self._L.nmoe_moe_load_layer_checked(self.h, layer, a.ctypes.data, a.nbytes,
                                                        _np_ptr(exp), out.ctypes.data))
        return out

    def load_layer_file_checked(self, layer: int, path: str, expected=None):
        out = np.zeros(self.cfg.num_experts, np.uint32)
        exp = None if expected is None else np.ascontiguousarray(expected, np.uint32)
        self._check(self._L.nmoe_moe_load_layer_file_checked(self.h, layer, path.encode(), _np_ptr(exp),
                                                             out.ctypes.data))
        return out

    def set_dense(self, layer: int, router: dict, shared_gate: dict, shared_up: dict, shared_down: dict,
                  shared_gate_vec: dict):
        """Each dict: {"weight": ndarray, ["scales": ndarray, "biases": ndarray]}."""
        keep = []

        def t(d):
            w = np.ascontiguousarray(d["weight"])
            s = np.ascontiguousarray(d["scales"]) if d.get("scales") is not None else None
            b = np.ascontiguousarray(d["biases"]) if d.get("biases") is not None else None
            keep.extend([w, s, b])
            return Tensor(w.ctypes.data, _np_ptr(s), _np_ptr(b))

        dw = DenseWeights(t(router), t(shared_gate), t(shared_up), t(shared_down), t(shared_gate_vec))
        self._check(self._L.nmoe_moe_set_dense(self.h, layer, C.byref(dw)))

    def forward(self, layer, k, x, out, x_dtype=DTYPE_BF16, h_mid=None, idx_out=None, w_out=None, stream=0):
        self._check(self._L.nmoe_moe_forward(self.h, layer, k, _ptr(x), x_dtype, _ptr(h_mid), _ptr(out),
                                             _ptr(idx_out), _ptr(w_out), stream))

    def route(self, layer, k, x, x_dtype=DTYPE_BF16, logits_out=None, idx_out=None, w_out=None, stream=0):
        self._check(self._L.nmoe_moe_route(self.h, layer, k, _ptr(x), x_dtype, _ptr(logits_out), _ptr(idx_out),
                                           _ptr(w_out), stream))

    def forward_batched(self, layer, T, k, x, out, x_dtype=DTYPE_BF16, out_dtype=DTYPE_F32, h_mid=None,
                        idx_out=None, w_out=None, stream=0):
        self._check(self._L.nmoe_moe_forward_batched(self.h, layer, T, k, _ptr(x), x_dtype, _ptr(h_mid), _ptr(out),
                                                     out_dtype, _ptr(idx_out), _ptr(w_out), stream))

    def debug_logits(self, T):
        """Router logits [T][256] of the last forward_batched call."""
        out = np.zeros((T, 256), np.float32)
        self._check(self._L.nmoe_moe_debug_logits(self.h, out.ctypes.data, T))
        return out

    def debug_ep_times(self):
        """(dispatch + wait, return + wait) device ms of the last expert-parallel call
        (context created with NMOE_EP_TIMING=1)."""
        ms = np.zeros(2, np.float32)
        self._check(self._L.nmoe_moe_debug_ep_times(self.h, ms.ctypes.data))
        return float(ms[0]), float(ms[1])

    def debug_gemm_trace(self):
        """[13][1024] %clock stamps of CTA 0 of the traced grouped-GEMM launch."""
        out = np.zeros((13, 1024), np.uint32)
        self._check(self._L.nmoe_moe_debug_gemm_trace(self.h, out.ctypes.data, out.size))
        return out

    def debug_trail(self, n=1024):
        out = np.zeros(n, np.uint32)
        self._check(self._L.nmoe_moe_debug_trail(self.h, out.ctypes.data, n))
        return out

    def decode_grid(self) -> int:
        """CTAs of the batch-1 decode kernel's grid (one per SM)."""
        return int(self._L.nmoe_moe_decode_grid(self.h))

    def debug_timeline(self, n_ctas=None):
        n_ctas = self.decode_grid() if n_ctas is None else n_ctas
        out = np.zeros((n_ctas, TIMELINE_WIDTH), np.uint32)
        self._check(self._L.nmoe_moe_debug_timeline(self.h, out.ctypes.data, n_ctas))
        return out

    def timeline_phases(self, n_ctas=None):
        """Per-phase times of the last batch-1 launch, in microseconds after the earliest
        CTA start: {phase name: (min, median, max) over the CTAs that reached it}.
        Needs a context created with NMOE_TIMELINE=1 in the environment."""
        return summarize_timeline(self.debug_timeline(n_ctas))

    def device_status(self):
        code = C.c_int(0)
        rc = self._L.nmoe_moe_device_status(self.h, C.byref(code))
        return rc, code.value


def forward_static(experts, num_experts, quant_bits, dense, router_dtype, shared_dtype, k, x, out,
                   x_dtype=DTYPE_BF16, h_mid=None, idx_out=None, w_out=None, stream=0):
    """nmoe_moe_forward_static: batch-1 block over caller-owned DEVICE weights, allocating
    nothing. `dense` maps router/shared_gate/shared_up/shared_down/shared_gate_vec to
    dicts of device tensors/pointers {"weight", ["scales", "biases"]}."""
    def t(d):
        return Tensor(_ptr(d["weight"]), _ptr(d.get("scales")), _ptr(d.get("biases")))
    dw = DenseWeights(t(dense["router"]), t(dense["shared_gate"]), t(dense["shared_up"]),
                      t(dense["shared_down"]), t(dense["shared_gate_vec"]))
    L = lib()
    rc = L.nmoe_moe_forward_static(_ptr(experts), num_experts, quant_bits, C.byref(dw), router_dtype, shared_dtype,
                                   k, _ptr(x), x_dtype, _ptr(h_mid), _ptr(out), _ptr(idx_out), _ptr(w_out), stream)
    if rc != OK:
        raise NmoeError(rc, L.nmoe_moe_static_error().decode())


def static_status(stream=0):
    """nmoe_moe_static_status: (status, code) of the last static call on this device."""
    L = lib()
    code = C.c_int(0)
    rc = L.nmoe_moe_static_status(C.byref(code), stream)
    return rc, code.value


def lm_head_workspace_bytes() -> int:
    return int(lib().nmoe_lm_head_workspace_bytes())


def lm_head_argmax(head: dict, head_dtype: int, vocab: int, x, token_out, workspace, x_dtype=DTYPE_F32,
                   norm_weight=None, norm_eps=1e-6, norm_add_one=True, logits_out=None, stream=0):
    """nmoe_lm_head_argmax: final RMSNorm + LM head GEMV + top-1 in one launch.
    `head` = {"weight", ["scales", "biases"]} device tensors/pointers; `token_out` a device
    u32 [1]; `workspace` device memory of lm_head_workspace_bytes(), zeroed once."""
    t = Tensor(_ptr(head["weight"]), _ptr(head.get("scales")), _ptr(head.get("biases")))
    L = lib()
    rc = L.nmoe_lm_head_argmax(C.byref(t), head_dtype, vocab, HIDDEN, _ptr(x), x_dtype, _ptr(norm_weight),
                               norm_eps, int(bool(norm_add_one)), _ptr(logits_out), _ptr(token_out),
                               _ptr(workspace), stream)
    if rc != OK:
        raise NmoeError(rc, L.nmoe_lm_head_error().decode())


def crc32c(data, crc: int = 0) -> int:
    """nmoe_crc32c: host CRC-32C of a bytes-like / numpy buffer."""
    a = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray)) else data)
    return int(lib().nmoe_crc32c(crc, a.ctypes.data, a.nbytes))


def expert_crcs(layer_bin: np.ndarray, bits: int):
    """Per-expert CRC-32C of a layer_XX.bin image (host): the values the checked loads
    compute on the device, e.g. to write a manifest next to the file."""
    a = np.ascontiguousarray(layer_bin).view(np.uint8)
    esz = expert_size(bits)
    if esz == 0 or a.nbytes % esz:
        raise ValueError("image size is not a whole number of expert blobs")
    return np.array([crc32c(a[i * esz:(i + 1) * esz]) for i in range(a.nbytes // esz)], np.uint32)


def crc32c_device(data, blob_bytes: int, nblobs: int, out, stream=0):
    """nmoe_crc32c_device: CRC-32C of nblobs device blobs into the device uint32 tensor `out`."""
    rc = lib().nmoe_crc32c_device(_ptr(data), blob_bytes, nblobs, _ptr(out), stream)
    if rc != OK:
        raise NmoeError(rc, "nmoe_crc32c_device")


def linear_attn_step(weights: dict, qkv, z, alpha, beta, conv_state, delta_state, out, stream=0):
    """nmoe_linear_attn_step: GatedDeltaNet core of one decode step (device tensors);
    `weights` = {"conv_w", "A_log", "dt_bias", "norm_w"}. States are updated in place."""
    w = LinearAttnWeights(_ptr(weights["conv_w"]), _ptr(weights["A_log"]), _ptr(weights["dt_bias"]),
                          _ptr(weights["norm_w"]))
    rc = lib().nmoe_linear_attn_step(C.byref(w), _ptr(qkv), _ptr(z), _ptr(alpha), _ptr(beta), _ptr(conv_state),
                                     _ptr(delta_state), _ptr(out), stream)
    if rc != OK:
        raise NmoeError(rc, "nmoe_linear_attn_step")


def linear_attn_step_batched(weights: dict, qkv, z, alpha, beta, conv_state, delta_state, out, stream=0):
    """nmoe_linear_attn_step_batched: the step for a batch of sequences (leading dimension
    of every tensor = the batch)."""
    w = LinearAttnWeights(_ptr(weights["conv_w"]), _ptr(weights["A_log"]), _ptr(weights["dt_bias"]),
                          _ptr(weights["norm_w"]))
    rc = lib().nmoe_linear_attn_step_batched(C.byref(w), int(qkv.shape[0]), _ptr(qkv), _ptr(z), _ptr(alpha),
                                             _ptr(beta), _ptr(conv_state), _ptr(delta_state), _ptr(out), stream)
    if rc != OK:
        raise NmoeError(rc, "nmoe_linear_attn_step_batched")


def full_attn_workspace_bytes() -> int:
    return int(lib().nmoe_full_attn_workspace_bytes())


def full_attn_step(weights: dict, q, k_new, v_new, k_cache, v_cache, position: int, max_positions: int, out,
                   workspace, stream=0):
    """nmoe_full_attn_step: full-attention decode step (device tensors); `weights` =
    {"q_norm", "k_norm"}; row `position` of the caches is written."""
    w = FullAttnWeights(_ptr(weights["q_norm"]), _ptr(weights["k_norm"]))
    rc = lib().nmoe_full_attn_step(C.byref(w), _ptr(q), _ptr(k_new), _ptr(v_new), _ptr(k_cache), _ptr(v_cache),
                                   position, max_positions, _ptr(out), _ptr(workspace), stream)
    if rc != OK:
        raise NmoeError(rc, "nmoe_full_attn_step")


def full_attn_batched_workspace_bytes(batch: int) -> int:
    return int(lib().nmoe_full_attn_batched_workspace_bytes(batch))


def full_attn_step_batched(weights: dict, q, k_new, v_new, k_cache, v_cache, positions, max_positions: int, out,
                           workspace, stream=0):
    """nmoe_full_attn_step_batched: the step for a batch of sequences over bf16 caches
    (device tensors; caches int16/bf16 [B][max_positions][2][256], positions int32 [B] on
    the device)."""
    w = FullAttnWeights(_ptr(weights["q_norm"]), _ptr(weights["k_norm"]))
    rc = lib().nmoe_full_attn_step_batched(C.byref(w), int(q.shape[0]), _ptr(q), _ptr(k_new), _ptr(v_new),
                                           _ptr(k_cache), _ptr(v_cache), _ptr(positions), max_positions, _ptr(out),
                                           _ptr(workspace), stream)
    if rc != OK:
        raise NmoeError(rc, "nmoe_full_attn_step_batched")


def _q4t(m):
    return Tensor(_np_ptr(m["weight"]), _np_ptr(m["scales"]), _np_ptr(m["biases"]))


class Decoder:
    """nmoe_decoder: the whole decode step over a loaded Context (one layer per model layer).
    Layer weights are host numpy arrays (see oracle.make_decoder_weights for the keys)."""

    def __init__(self, moe: Context, num_layers: int, k: int = 8, max_positions: int = 4096):
        self._L = lib()
        st = C.c_int(0)
        h = self._L.nmoe_decoder_create(moe.h, num_layers, k, max_positions, C.byref(st))
        if not h:
            raise NmoeError(st.value, "nmoe_decoder_create")
        self.h, self.moe, self.num_layers = h, moe, num_layers

    def _check(self, rc):
        if rc != OK:
            raise NmoeError(rc, self._L.nmoe_decoder_error(self.h).decode())

    def set_layer(self, l: int, w: dict):
        if w["kind"] == "full":
            hw = FullLayerHost(_np_ptr(w["input_norm"]), _np_ptr(w["post_norm"]), _q4t(w["q"]), _q4t(w["k"]),
                               _q4t(w["v"]), _q4t(w["o"]), _np_ptr(w["q_norm"]), _np_ptr(w["k_norm"]))
            self._check(self._L.nmoe_decoder_set_full_layer(self.h, l, C.byref(hw)))
        else:
            hw = LinearLayerHost(_np_ptr(w["input_norm"]), _np_ptr(w["post_norm"]), _q4t(w["qkv"]), _q4t(w["z"]),
                                 _q4t(w["beta"]), _q4t(w["alpha"]), _q4t(w["out"]), _np_ptr(w["conv_w"]),
                                 _np_ptr(w["A_log"]), _np_ptr(w["dt_bias"]), _np_ptr(w["norm_w"]))
            self._check(self._L.nmoe_decoder_set_linear_layer(self.h, l, C.byref(hw)))

    def set_globals(self, g: dict):
        emb, head = g["embed"], g["lm_head"]
        et = Tensor(_np_ptr(emb["weight"]), _np_ptr(emb.get("scales")), _np_ptr(emb.get("biases")))
        ht = Tensor(_np_ptr(head["weight"]), _np_ptr(head.get("scales")), _np_ptr(head.get("biases")))
        self._check(self._L.nmoe_decoder_set_globals(self.h, g["vocab"], emb["dtype"], C.byref(et),
                                                     _np_ptr(g["final_norm"]), head["dtype"], C.byref(ht)))

    def reset(self, stream=0):
        self._check(self._L.nmoe_decoder_reset(self.h, stream))

    def step(self, d_token, position: int, d_next, d_hidden=None, stream=0):
        self._check(self._L.nmoe_decoder_step(self.h, _ptr(d_token), position, _ptr(d_next), _ptr(d_hidden), stream))

    def close(self):
        if getattr(self, "h", None):
            self._L.nmoe_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
