"""CPU oracle of the Ming-TTS hot path -- TEST INFRASTRUCTURE ONLY.

ctypes bindings of oracle/_build/liboracle.so (oracle.c / oracle_engine.c, a plain-C restatement
of the reference's Metal kernels and generation loop). Only tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference arm may import this module, and only as the checker or the
timed CPU baseline; the product (libmingcuda.so) never uses it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_float, c_int, c_long, c_size_t, c_uint16, c_uint32, c_uint64, c_void_p

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

_P = c_void_p


class GenerateIO(ctypes.Structure):
    _fields_ = [("prompt_rows", c_int), ("embeds", _P), ("steps", c_int), ("cfg", c_float), ("obey_stop", c_int),
                ("noise", _P), ("initial_history", _P),
                ("stop_logits", _P), ("llm_hidden", _P), ("latents", _P), ("agg_out", _P), ("velocity0", _P),
                ("vae_hidden", _P), ("layer0_prefill", _P), ("layer_last_prefill", _P), ("pcm", _P),
                ("pcm_cap", c_long), ("chunk_counts", _P), ("step_seconds", _P),
                ("steps_run", c_int), ("stopped", c_int), ("pcm_count", c_long), ("chunks", c_int)]


PROTOTYPES = {
    "or_bf16_bits": (c_uint16, [c_float]),
    "or_bf16_to_f32": (c_float, [c_uint16]),
    "or_lcg_floats": (None, [POINTER(c_uint64), _P, c_size_t, c_float]),
    "or_gaussian_noise": (None, [_P, c_size_t, c_uint64]),
    "or_randn_bf16": (None, [_P, c_size_t, c_uint64, c_float]),
    "or_linear": (None, [_P, c_int, c_int, _P, _P, _P, c_int, c_int, _P, c_int, c_uint32]),
    "or_rmsnorm": (None, [_P, c_int, c_int, c_int, _P, _P, c_int, c_float]),
    "or_rope_cache": (None, [_P, c_int, c_int, c_int, c_int, c_int, _P, _P, c_int, _P]),
    "or_attention": (None, [_P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, c_int, _P, c_int]),
    "or_dit_attention": (None, [_P, c_int, c_int, c_int, c_int, _P, _P, c_int]),
    "or_flow_assemble": (None, [_P, _P, _P, _P, _P, _P, _P, c_int, c_int, _P]),
    "or_flow_euler": (None, [_P, _P, c_int, c_int, c_int, c_int, c_float, c_float, _P]),
    "or_upsample4": (None, [_P, _P, _P, c_int, _P]),
    "or_istft_frames": (None, [_P, c_int, c_int, c_int, _P, _P, c_int, c_int]),
    "or_istft_emit": (None, [_P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P]),
    "or_flow_timesteps": (None, [c_int, _P]),
    "or_sinusoid": (None, [c_float, _P]),
    "or_generate": (c_int, [_P, _P, POINTER(GenerateIO)]),
    "or_llm_decode": (c_int, [_P, _P, c_int, c_int, _P, c_int, _P]),
    "or_flow_patch": (c_int, [_P, _P, _P, _P, _P, c_float, _P]),
    "or_vae_decode_clip": (ctypes.c_long, [_P, _P, _P, c_int, _P, ctypes.c_long]),
    "or_vae_encode": (c_int, [_P, _P, _P, ctypes.c_long, _P, _P]),
    "or_aggregate_latents": (c_int, [_P, _P, _P, c_int, _P]),
}

_lib = None


def build() -> None:
    """Compiles liboracle.so with the committed Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def _p(a):
    if a is None:
        return None
    assert isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous numpy"
    return a.ctypes.data


def lcg_floats(seed: int, n: int, scale: float = 1.0) -> np.ndarray:
    """KernelTests.swift:21-28 LCG stream (returns n floats)."""
    state = c_uint64(seed)
    out = np.empty(n, np.float32)
    lib().or_lcg_floats(ctypes.byref(state), _p(out), n, scale)
    return out


def gaussian_noise(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_gaussian_noise(_p(out), n, seed)
    return out


def randn_bf16(n: int, seed: int, std: float) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().or_randn_bf16(_p(out), n, seed, std)
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (KernelTests.swift:30-34), vectorised."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def linear(x, ldx, m, w, w2, bias, n, k, y, ldy, flags):
    lib().or_linear(_p(x), ldx, m, _p(w), _p(w2), _p(bias), n, k, _p(y), ldy, flags)


def rmsnorm(x, ldx, rows, width, w, y, ldy, eps=1e-6):
    lib().or_rmsnorm(_p(x), ldx, rows, width, _p(w), _p(y), ldy, eps)


def rope_cache(qkv, ldq, m, hq, hkv, pos0, kc, vc, cap, inv_freq):
    lib().or_rope_cache(_p(qkv), ldq, m, hq, hkv, pos0, _p(kc), _p(vc), cap, _p(inv_freq))


def attention(q, ldq, m, hq, hkv, pos0, window, kc, vc, cap, out, ldo):
    lib().or_attention(_p(q), ldq, m, hq, hkv, pos0, window, _p(kc), _p(vc), cap, _p(out), ldo)


def dit_attention(qkv, ld, batch, seq, heads, inv_freq, out, ldo):
    lib().or_dit_attention(_p(qkv), ld, batch, seq, heads, _p(inv_freq), _p(out), ldo)


def flow_assemble(y, history, cemb, cbias, temb, xw, xb, hidden, latent, x):
    lib().or_flow_assemble(_p(y), _p(history), _p(cemb), _p(cbias), _p(temb), _p(xw), _p(xb), hidden, latent, _p(x))


def flow_euler(y, pred, ldp, pred_row, null_row, latent, cfg, dt, capture):
    lib().or_flow_euler(_p(y), _p(pred), ldp, pred_row, null_row, latent, cfg, dt, _p(capture))


def upsample4(prev, cur, nxt, hidden, frames):
    lib().or_upsample4(_p(prev), _p(cur), _p(nxt), hidden, _p(frames))


def istft_frames(spec, ld_spec, count, nfft, window, frames, frame0, ring):
    lib().or_istft_frames(_p(spec), ld_spec, count, nfft, _p(window), _p(frames), frame0, ring)


def istft_emit(frames, window, nfft, hop, s0, count, last_frame, ring, out):
    lib().or_istft_emit(_p(frames), _p(window), nfft, hop, s0, count, last_frame, ring, _p(out))


def flow_timesteps(steps: int) -> np.ndarray:
    out = np.empty(steps + 1, np.float32)
    lib().or_flow_timesteps(steps, _p(out))
    return out


def sinusoid(t: float) -> np.ndarray:
    out = np.empty(256, np.float32)
    lib().or_sinusoid(t, _p(out))
    return out
