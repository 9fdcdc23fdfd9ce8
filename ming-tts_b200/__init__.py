"""mingtts_b200 -- Python bindings of libmingcuda.so (the B200 hot path of Ming-3.0-tts-0.5B).

The library is a C ABI (include/mingcuda.h); this module declares its prototypes with ctypes and
mirrors its structs. Torch tensors are accepted wherever the ABI takes a device pointer; the
current torch stream is passed as the CUDA stream. There is no CPU fallback: every compute call
goes to the CUDA library, and importing fails loudly if the library has not been built.

The directory is named ``ming-tts_b200``; import it with ``load_package()`` from ``_loader.py`` or
register it under the module name ``mingtts_b200``.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_size_t, c_uint32, c_uint64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmingcuda.so")

MT_OK, MT_ERR_ARG, MT_ERR_SHAPE, MT_ERR_CAPACITY, MT_ERR_CUDA, MT_ERR_TIMEOUT, MT_ERR_NOMEM, MT_ERR_STATE = range(8)
STATUS_NAMES = ["MT_OK", "MT_ERR_ARG", "MT_ERR_SHAPE", "MT_ERR_CAPACITY", "MT_ERR_CUDA", "MT_ERR_TIMEOUT",
                "MT_ERR_NOMEM", "MT_ERR_STATE"]

BIAS, ACCUM, GELU, SILU_GATE, SILU = 1, 2, 4, 8, 16


class MingError(RuntimeError):
    """A non-zero mt_status; .status holds the code."""

    def __init__(self, status: int, message: str):
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"{name}: {message}")
        self.status = status


# ------------------------------------------------------------------------------------------------
# Struct mirrors of include/mingcuda.h
# ------------------------------------------------------------------------------------------------
class QwenConfig(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("heads", c_int), ("kv_heads", c_int), ("intermediate", c_int),
                ("layers", c_int), ("window", c_int), ("rope_theta", c_float), ("eps", c_float)]


class QwenLayer(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("norm1", "qkv_w", "qkv_b", "o_w", "norm2", "gate_w", "up_w", "down_w")]


class QwenWeights(ctypes.Structure):
    _fields_ = [("cfg", QwenConfig), ("layers", POINTER(QwenLayer)), ("final_norm", c_void_p)]


class DitConfig(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("heads", c_int), ("depth", c_int), ("ff", c_int), ("out_dim", c_int),
                ("eps", c_float)]


class DitBlock(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("norm1", "qkv_w", "qkv_b", "out_w", "out_b", "norm2", "ff1_w", "ff1_b",
                                        "ff2_w", "ff2_b")]


class DitWeights(ctypes.Structure):
    _fields_ = [("cfg", DitConfig), ("blocks", POINTER(DitBlock)), ("final_norm", c_void_p), ("final_w", c_void_p),
                ("final_b", c_void_p), ("inv_freq", c_void_p)]


class ModelConfig(ctypes.Structure):
    _fields_ = [("llm", QwenConfig), ("vae", QwenConfig), ("flow", DitConfig), ("agg", DitConfig),
                ("latent_dim", c_int), ("time_dim", c_int), ("vocab", c_int), ("nfft", c_int), ("hop", c_int),
                ("flow_steps", c_int), ("llm_capacity", c_int)]


class ModelWeights(ctypes.Structure):
    _fields_ = [("llm", QwenWeights), ("stop_w", c_void_p), ("stop_b", c_void_p),
                ("flow_x_w", c_void_p), ("flow_x_b", c_void_p), ("flow_c_w", c_void_p), ("flow_c_b", c_void_p),
                ("flow_t1_w", c_void_p), ("flow_t1_b", c_void_p), ("flow_t2_w", c_void_p), ("flow_t2_b", c_void_p),
                ("flow", DitWeights),
                ("agg_x_w", c_void_p), ("agg_x_b", c_void_p), ("agg_cls", c_void_p), ("agg", DitWeights),
                ("vae_fc1_w", c_void_p), ("vae_fc1_b", c_void_p), ("vae", QwenWeights),
                ("vae_head_w", c_void_p), ("vae_head_b", c_void_p), ("vae_window", c_void_p),
                ("embed_tokens", c_void_p)]


# ------------------------------------------------------------------------------------------------
# Library loading and prototypes
# ------------------------------------------------------------------------------------------------
_P = c_void_p
PROTOTYPES = {
    # name: (restype, argtypes)
    "mt_ctx_create": (c_int, [c_int, POINTER(c_void_p)]),
    "mt_ctx_destroy": (None, [_P]),
    "mt_last_error": (c_char_p, [_P]),
    "mt_version": (c_char_p, []),
    "mt_ctx_check": (c_int, [_P, _P]),
    "mt_linear_route": (c_int, [c_int, c_int, c_int]),
    "mt_linear": (c_int, [_P, _P, _P, c_int, c_int, _P, _P, _P, c_int, c_int, _P, c_int, c_uint32]),
    "mt_rmsnorm": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P, _P, c_int, c_float]),
    "mt_copy": (c_int, [_P, _P, _P, c_int, _P]),
    "mt_rope_cache": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P, _P, c_int, _P]),
    "mt_attention": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, c_int, _P, c_int]),
    "mt_dit_attention": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, _P, _P, c_int]),
    "mt_flow_assemble": (c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_int, c_int, _P]),
    "mt_flow_euler": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_float, c_float, _P]),
    "mt_upsample4": (c_int, [_P, _P, _P, _P, _P, c_int, _P]),
    "mt_istft_frames": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P, _P, _P, c_int, c_int]),
    "mt_istft_emit": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P]),
    "mt_gaussian_noise_host": (None, [_P, c_size_t, c_uint64]),
    "mt_randn_bf16_host": (None, [_P, c_size_t, c_uint64, c_float]),
    "mt_randn_bf16": (c_int, [_P, _P, _P, c_size_t, c_uint64, c_float]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded libmingcuda.so with prototypes declared. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C ming-tts_b200/csrc` "
                              "or __graft_entry__.build()")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def ptr(t) -> int | None:
    """Device/host address of a torch tensor or numpy array (None passes through)."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    return int(t)


def current_stream() -> int:
    import torch
    return torch.cuda.current_stream().cuda_stream


class Context:
    """An mt_ctx bound to one CUDA device. Every op call raises MingError on a non-zero status."""

    def __init__(self, device: int = 0):
        self._ctx = c_void_p()
        st = lib().mt_ctx_create(device, ctypes.byref(self._ctx))
        if st != MT_OK:
            raise MingError(st, f"mt_ctx_create(device={device}) failed")
        self.device = device

    @property
    def handle(self) -> c_void_p:
        return self._ctx

    def close(self):
        if self._ctx:
            lib().mt_ctx_destroy(self._ctx)
            self._ctx = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int, what: str):
        if st != MT_OK:
            msg = lib().mt_last_error(self._ctx)
            raise MingError(st, f"{what}: {msg.decode() if msg else ''}")

    def check(self, stream=None):
        self._check(lib().mt_ctx_check(self._ctx, stream if stream is not None else current_stream()), "mt_ctx_check")

    def call(self, name: str, *args, stream=None):
        """Calls mt_<name>(ctx, stream, *args) with tensors converted to pointers."""
        fn = getattr(lib(), "mt_" + name)
        conv = [ptr(a) if (hasattr(a, "data_ptr") or hasattr(a, "ctypes")) else a for a in args]
        st = fn(self._ctx, stream if stream is not None else current_stream(), *conv)
        self._check(st, "mt_" + name)

    # Thin wrappers with the reference's argument order (Kernels.swift:132-281).
    def linear(self, x, ldx, m, w, w2, bias, n, k, y, ldy, flags):
        self.call("linear", x, ldx, m, w, w2, bias, n, k, y, ldy, flags)

    def rmsnorm(self, x, ldx, rows, width, w, y, ldy, eps=1e-6):
        self.call("rmsnorm", x, ldx, rows, width, w, y, ldy, eps)

    def rope_cache(self, qkv, ldq, m, hq, hkv, pos0, kc, vc, cap, inv_freq):
        self.call("rope_cache", qkv, ldq, m, hq, hkv, pos0, kc, vc, cap, inv_freq)

    def attention(self, q, ldq, m, hq, hkv, pos0, window, kc, vc, cap, out, ldo):
        self.call("attention", q, ldq, m, hq, hkv, pos0, window, kc, vc, cap, out, ldo)

    def dit_attention(self, qkv, ld, batch, seq, heads, inv_freq, out, ldo):
        self.call("dit_attention", qkv, ld, batch, seq, heads, inv_freq, out, ldo)


def version() -> str:
    return lib().mt_version().decode()
