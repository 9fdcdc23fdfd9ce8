"""mingtts_b200 -- Python bindings of libmingcuda.so (the B200 hot path of Ming-3.0-tts-0.5B).

The library is a C ABI (include/mingcuda.h); this module declares its prototypes with ctypes and
mirrors its structs. Torch tensors are accepted wherever the ABI takes a device pointer; the
current torch stream is passed as the CUDA stream. There is no CPU fallback: every compute call
goes to the CUDA library, and importing fails loudly if the library has not been built.

The directory is named ``ming-tts_b200``; tests/conftest.py, bench.py and __graft_entry__.py import it
under the module name ``mingtts_b200`` with importlib.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_size_t, c_uint32, c_uint64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmingcuda.so")

(MT_OK, MT_ERR_ARG, MT_ERR_SHAPE, MT_ERR_CAPACITY, MT_ERR_CUDA, MT_ERR_TIMEOUT, MT_ERR_NOMEM, MT_ERR_STATE,
 MT_ERR_CHECKPOINT) = range(9)
STATUS_NAMES = ["MT_OK", "MT_ERR_ARG", "MT_ERR_SHAPE", "MT_ERR_CAPACITY", "MT_ERR_CUDA", "MT_ERR_TIMEOUT",
                "MT_ERR_NOMEM", "MT_ERR_STATE", "MT_ERR_CHECKPOINT"]

BIAS, ACCUM, GELU, SILU_GATE, SILU = 1, 2, 4, 8, 16
SAMPLE_RATE = 44100  # MingTTSModel.sampleRate: hop 882 samples per 20 ms frame


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


class TensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 96), ("offset", c_size_t), ("numel", c_size_t), ("dtype", c_int),
                ("init", c_int), ("std", c_float), ("seed", c_uint64)]


class EncoderWeights(ctypes.Structure):
    _fields_ = [("frame", c_int), ("padded_frame", c_int), ("patch", c_int), ("max_frames", c_int),
                ("fc1_w", c_void_p), ("fc2_w", c_void_p), ("fc2_b", c_void_p), ("stack", QwenWeights),
                ("aggregator", QwenWeights), ("cls", c_void_p), ("fc3_w", c_void_p), ("fc3_b", c_void_p)]


class EngineOptions(ctypes.Structure):
    _fields_ = [("max_requests", c_int), ("max_prompt", c_int), ("max_steps", c_int), ("vae_ring", c_int),
                ("use_graphs", c_int), ("groups", c_int)]


class ConvDecConfig(ctypes.Structure):
    _fields_ = [("latent_dim", c_int), ("channels", c_int * 5), ("strides", c_int * 4), ("kernel", c_int)]


class ConvDecWeights(ctypes.Structure):
    _fields_ = [("in_w", c_void_p), ("in_b", c_void_p), ("up_w", c_void_p * 4), ("up_b", c_void_p * 4),
                ("a_w", c_void_p * 4), ("a_b", c_void_p * 4), ("b_w", c_void_p * 4), ("b_b", c_void_p * 4),
                ("out_w", c_void_p), ("out_b", c_void_p)]


MT_DTYPE_BF16, MT_DTYPE_F32 = 0, 1
BUF_Z, BUF_STOP_LOGITS, BUF_LATENTS, BUF_AGG_OUT, BUF_VELOCITY0, BUF_VAE_HIDDEN, BUF_PCM = range(7)


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
    "mt_ctx_set_gemm_pairs": (c_int, [_P, c_int]),
    "mt_ctx_set_wait_limit": (c_int, [_P, c_uint32]),
    "mt_ctx_set_persistent": (c_int, [_P, c_int]),
    "mt_ctx_wait_probe": (c_int, [_P, _P]),
    "mt_linear": (c_int, [_P, _P, _P, c_int, c_int, _P, _P, _P, c_int, c_int, _P, c_int, c_uint32]),
    "mt_linear_split": (c_int, [_P, _P, _P, _P, c_int, c_int, _P, _P, _P, c_int, c_int, _P, c_int, _P, _P, c_int,
                                c_uint32]),
    "mt_linear_static": (c_int, [_P, _P, c_int, c_int, _P, _P, _P, c_int, c_int, _P, c_int, c_uint32]),
    "mt_linear_static_status": (c_int, [_P]),
    "mt_rmsnorm": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P, _P, c_int, c_float]),
    "mt_rope_attention": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, c_int, _P, _P, c_int,
                                  c_int]),
    "mt_copy": (c_int, [_P, _P, _P, c_int, _P]),
    "mt_qwen_decode": (c_int, [_P, _P, _P, c_int, c_int, _P, _P, ctypes.c_longlong, c_int, _P, _P]),
    "mt_rope_cache": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P, _P, c_int, _P]),
    "mt_attention": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, c_int, _P, c_int]),
    "mt_dit_attention": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, _P, _P, c_int]),
    "mt_flow_assemble": (c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_int, c_int, _P]),
    "mt_flow_euler": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_float, c_float, _P]),
    "mt_upsample4": (c_int, [_P, _P, _P, _P, _P, c_int, _P]),
    "mt_istft_frames": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P, _P, _P, c_int, c_int]),
    "mt_istft_emit": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P]),
    "mt_model_config_default": (None, [POINTER(ModelConfig)]),
    "mt_model_tensors": (c_int, [POINTER(ModelConfig), c_uint64, c_int, _P, c_int]),
    "mt_model_arena_bytes": (c_size_t, [POINTER(ModelConfig), c_int]),
    "mt_model_create_random": (c_int, [_P, POINTER(ModelConfig), c_uint64, c_int, POINTER(c_void_p)]),
    "mt_model_create_from_arena": (c_int, [_P, POINTER(ModelConfig), _P, c_int, POINTER(c_void_p)]),
    "mt_model_get_weights": (_P, [_P]),
    "mt_model_get_config": (_P, [_P]),
    "mt_model_arena": (c_int, [_P, POINTER(c_void_p), POINTER(c_size_t)]),
    "mt_model_destroy": (None, [_P]),
    "mt_checkpoint_fill_arena": (c_int, [ctypes.c_char_p, POINTER(ModelConfig), c_int, _P, c_size_t, ctypes.c_char_p,
                                         c_size_t]),
    "mt_model_load_safetensors": (c_int, [_P, POINTER(ModelConfig), ctypes.c_char_p, c_int, POINTER(c_void_p)]),
    "mt_engine_create": (c_int, [_P, _P, POINTER(EngineOptions), POINTER(c_void_p)]),
    "mt_engine_destroy": (None, [_P]),
    "mt_engine_begin": (c_int, [_P, _P, c_int, c_int, _P, _P, _P, _P, c_int, c_float]),
    "mt_engine_prefill": (c_int, [_P, _P]),
    "mt_engine_step": (c_int, [_P, _P, POINTER(c_int)]),
    "mt_engine_flush": (c_int, [_P, _P, POINTER(c_int)]),
    "mt_engine_buffer": (c_int, [_P, c_int, POINTER(c_void_p), POINTER(ctypes.c_longlong)]),
    "mt_engine_steps_done": (c_int, [_P]),
    "mt_engine_step_kernels": (c_int, [_P]),
    "mt_engine_set_stage_timing": (c_int, [_P, c_int]),
    "mt_engine_set_stop_rule": (c_int, [_P, c_int]),
    "mt_engine_stage_ms": (c_int, [_P, _P]),
    "mt_engine_generate": (c_int, [_P, _P, c_int, c_int, _P, _P, _P, c_int, c_float, _P, ctypes.c_longlong,
                                   POINTER(ctypes.c_longlong), _P]),
    "mt_encoder_tensors": (c_int, [POINTER(ModelConfig), c_uint64, _P, c_int]),
    "mt_encoder_arena_bytes": (c_size_t, [POINTER(ModelConfig)]),
    "mt_encoder_create_random": (c_int, [_P, POINTER(ModelConfig), c_uint64, POINTER(c_void_p)]),
    "mt_encoder_create_from_arena": (c_int, [_P, POINTER(ModelConfig), _P, POINTER(c_void_p)]),
    "mt_checkpoint_fill_encoder_arena": (c_int, [ctypes.c_char_p, POINTER(ModelConfig), _P, c_size_t,
                                                 ctypes.c_char_p, c_size_t]),
    "mt_encoder_load_safetensors": (c_int, [_P, POINTER(ModelConfig), ctypes.c_char_p, POINTER(c_void_p)]),
    "mt_encoder_get_weights": (_P, [_P]),
    "mt_encoder_arena": (c_int, [_P, POINTER(c_void_p), POINTER(c_size_t)]),
    "mt_encoder_destroy": (None, [_P]),
    "mt_vae_encode": (c_int, [_P, _P, _P, ctypes.c_longlong, _P, _P]),
    "mt_aggregate_latents": (c_int, [_P, _P, _P, _P, c_int, _P]),
    "mt_engine_generate_stream": (c_int, [_P, _P, c_int, c_int, _P, _P, _P, c_int, c_float, _P, _P,
                                          POINTER(ctypes.c_longlong), _P]),
    "mt_write_wav_f32": (c_int, [ctypes.c_char_p, _P, ctypes.c_longlong, c_int]),
    "mt_gaussian_noise_host": (None, [_P, c_size_t, c_uint64]),
    "mt_randn_bf16_host": (None, [_P, c_size_t, c_uint64, c_float]),
    "mt_randn_bf16": (c_int, [_P, _P, _P, c_size_t, c_uint64, c_float]),
    "mt_convdec_samples": (ctypes.c_longlong, [POINTER(ConvDecConfig), c_int]),
    "mt_convdec_create": (c_int, [_P, POINTER(ConvDecConfig), POINTER(ConvDecWeights), c_int, POINTER(c_void_p)]),
    "mt_convdec_decode": (c_int, [_P, _P, _P, c_int, _P]),
    "mt_convdec_destroy": (None, [_P]),
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

    def set_persistent(self, mode: int):
        """Small-batch stacks: 1 the persistent stack kernel where it fits, 0 one launch per op (default),
        2 the persistent kernel required."""
        self._check(lib().mt_ctx_set_persistent(self._ctx, mode), "mt_ctx_set_persistent")

    def set_wait_limit(self, microseconds: int):
        """Wall-time limit of the kernels' bounded waits (0 = the default 2 s)."""
        self._check(lib().mt_ctx_set_wait_limit(self._ctx, microseconds), "mt_ctx_set_wait_limit")

    def wait_probe(self, stream=None):
        """Enqueues a kernel whose bounded wait runs out; the next check() raises MT_ERR_TIMEOUT."""
        self._check(lib().mt_ctx_wait_probe(self._ctx, stream if stream is not None else current_stream()),
                    "mt_ctx_wait_probe")

    def set_gemm_pairs(self, mode: int):
        """Tensor-core GEMM tiling for later plans: -1 automatic, 0 single-CTA tiles, 1 CTA pairs."""
        self._check(lib().mt_ctx_set_gemm_pairs(self._ctx, mode), "mt_ctx_set_gemm_pairs")

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


# ------------------------------------------------------------------------------------------------
# Model and engine
# ------------------------------------------------------------------------------------------------
def default_config() -> ModelConfig:
    c = ModelConfig()
    lib().mt_model_config_default(ctypes.byref(c))
    return c


def small_config() -> ModelConfig:
    """A reduced model with the same block structure, for fast CPU-oracle parity runs."""
    c = default_config()
    c.llm.hidden, c.llm.heads, c.llm.kv_heads, c.llm.intermediate, c.llm.layers = 128, 2, 1, 256, 2
    c.vae.hidden, c.vae.heads, c.vae.kv_heads, c.vae.intermediate, c.vae.layers = 128, 2, 1, 256, 2
    c.flow.hidden, c.flow.heads, c.flow.depth, c.flow.ff = 128, 2, 2, 256
    c.agg.hidden, c.agg.heads, c.agg.depth, c.agg.ff, c.agg.out_dim = 128, 2, 2, 256, 128
    c.vocab, c.nfft, c.hop = 1000, 256, 64
    return c


def tensor_table(cfg: ModelConfig, seed: int = 0, with_embeddings: bool = True) -> list[TensorInfo]:
    n = lib().mt_model_tensors(ctypes.byref(cfg), seed, int(with_embeddings), None, 0)
    arr = (TensorInfo * n)()
    lib().mt_model_tensors(ctypes.byref(cfg), seed, int(with_embeddings), arr, n)
    return list(arr)


def weights_struct(cfg: ModelConfig, base: int, tensors: list[TensorInfo]):
    """mt_model_weights over an arena at address `base` (device or host) laid out as `tensors`.
    Returns (struct, keepalive) -- keep both alive while the struct is in use."""
    off = {t.name.decode(): t.offset for t in tensors}

    def at(name):
        return base + off[name] if name in off else None

    keep = []

    def qwen(prefix, qc):
        layers = (QwenLayer * qc.layers)()
        for l in range(qc.layers):
            p = f"{prefix}.layers.{l}"
            layers[l] = QwenLayer(at(p + ".input_layernorm.weight"), at(p + ".self_attn.qkv_proj.weight"),
                                  at(p + ".self_attn.qkv_proj.bias"), at(p + ".self_attn.o_proj.weight"),
                                  at(p + ".post_attention_layernorm.weight"), at(p + ".mlp.gate_proj.weight"),
                                  at(p + ".mlp.up_proj.weight"), at(p + ".mlp.down_proj.weight"))
        keep.append(layers)
        return QwenWeights(qc, ctypes.cast(layers, POINTER(QwenLayer)), at(prefix + ".norm.weight"))

    def dit(prefix, dc):
        blocks = (DitBlock * dc.depth)()
        for i in range(dc.depth):
            p = f"{prefix}.blocks.{i}"
            blocks[i] = DitBlock(at(p + ".norm1.weight"), at(p + ".attn.to_qkv.weight"), at(p + ".attn.to_qkv.bias"),
                                 at(p + ".attn.to_out.0.weight"), at(p + ".attn.to_out.0.bias"),
                                 at(p + ".norm2.weight"), at(p + ".mlp.ff.0.0.weight"), at(p + ".mlp.ff.0.0.bias"),
                                 at(p + ".mlp.ff.2.weight"), at(p + ".mlp.ff.2.bias"))
        keep.append(blocks)
        return DitWeights(dc, ctypes.cast(blocks, POINTER(DitBlock)), at(prefix + ".final_layer.norm_final.weight"),
                          at(prefix + ".final_layer.linear.weight"), at(prefix + ".final_layer.linear.bias"),
                          at(prefix + ".rotary_embed.inv_freq"))

    f, a, v = "flowloss.cfm.model", "linear_proj_audio", "audio.decoder"
    w = ModelWeights()
    w.llm = qwen("model.model", cfg.llm)
    w.stop_w, w.stop_b = at("stop_head.weight"), at("stop_head.bias")
    w.flow_x_w, w.flow_x_b = at(f + ".x_embedder.weight"), at(f + ".x_embedder.bias")
    w.flow_c_w, w.flow_c_b = at(f + ".c_embedder.cond_embedder.weight"), at(f + ".c_embedder.cond_embedder.bias")
    w.flow_t1_w, w.flow_t1_b = at(f + ".t_embedder.time_mlp.0.weight"), at(f + ".t_embedder.time_mlp.0.bias")
    w.flow_t2_w, w.flow_t2_b = at(f + ".t_embedder.time_mlp.2.weight"), at(f + ".t_embedder.time_mlp.2.bias")
    w.flow = dit(f, cfg.flow)
    w.agg_x_w, w.agg_x_b, w.agg_cls = at(a + ".x_embedder.weight"), at(a + ".x_embedder.bias"), at(a + ".word_embedder.weight")
    w.agg = dit(a, cfg.agg)
    w.vae_fc1_w, w.vae_fc1_b = at(v + ".fc1.weight"), at(v + ".fc1.bias")
    w.vae = qwen(v + ".decoder", cfg.vae)
    w.vae_head_w, w.vae_head_b = at(v + ".head.out.weight"), at(v + ".head.out.bias")
    w.vae_window = at(v + ".head.istft.window")
    w.embed_tokens = at("model.model.embed_tokens.weight")
    return w, keep


class CheckpointError(MingError):
    """A safetensors file the loader cannot use (MT_ERR_CHECKPOINT)."""


def checkpoint_fill_arena(path: str, cfg: ModelConfig | None = None, with_embeddings: bool = True):
    """Host numpy uint8 arena (mt_model_tensors layout) filled from a safetensors file. No GPU."""
    import numpy as np
    cfg = cfg if cfg is not None else default_config()
    nbytes = lib().mt_model_arena_bytes(ctypes.byref(cfg), int(with_embeddings))
    arena = np.empty(nbytes, np.uint8)
    err = ctypes.create_string_buffer(512)
    st = lib().mt_checkpoint_fill_arena(str(path).encode(), ctypes.byref(cfg), int(with_embeddings),
                                        arena.ctypes.data, nbytes, err, len(err))
    if st != MT_OK:
        raise (CheckpointError if st == MT_ERR_CHECKPOINT else MingError)(st, f"mt_checkpoint_fill_arena: {err.value.decode()}")
    return arena


class Model:
    """An mt_model with a device arena: random-init from `seed`, or a checkpoint (Model.load)."""

    def __init__(self, ctx: Context, cfg: ModelConfig | None = None, seed: int = 1, with_embeddings: bool = True,
                 _handle=None):
        self.ctx = ctx
        self.cfg = cfg if cfg is not None else default_config()
        self.seed = seed
        self.with_embeddings = with_embeddings
        self._m = c_void_p()
        if _handle is not None:
            self._m = _handle
            return
        ctx._check(lib().mt_model_create_random(ctx.handle, ctypes.byref(self.cfg), seed, int(with_embeddings),
                                                ctypes.byref(self._m)), "mt_model_create_random")

    @classmethod
    def load(cls, ctx: Context, path: str, cfg: ModelConfig | None = None, with_embeddings: bool = True) -> "Model":
        """A model whose arena is filled from a safetensors checkpoint (mt_model_load_safetensors)."""
        cfg = cfg if cfg is not None else default_config()
        h = c_void_p()
        st = lib().mt_model_load_safetensors(ctx.handle, ctypes.byref(cfg), str(path).encode(), int(with_embeddings),
                                             ctypes.byref(h))
        if st != MT_OK:
            msg = lib().mt_last_error(ctx.handle).decode()
            raise (CheckpointError if st == MT_ERR_CHECKPOINT else MingError)(st, f"mt_model_load_safetensors: {msg}")
        return cls(ctx, cfg, seed=0, with_embeddings=with_embeddings, _handle=h)

    @property
    def handle(self):
        return self._m

    def arena(self):
        p, n = c_void_p(), c_size_t()
        lib().mt_model_arena(self._m, ctypes.byref(p), ctypes.byref(n))
        return p.value, n.value

    def tensors(self):
        return tensor_table(self.cfg, self.seed, self.with_embeddings)

    def arena_to_host(self):
        """Host numpy uint8 copy of the device arena."""
        import numpy as np
        p, nbytes = self.arena()
        return device_to_numpy(p, (nbytes,), np.uint8)

    def close(self):
        if self._m:
            lib().mt_model_destroy(self._m)
            self._m = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def encoder_tensor_table(cfg: ModelConfig, seed: int = 0) -> list[TensorInfo]:
    n = lib().mt_encoder_tensors(ctypes.byref(cfg), seed, None, 0)
    arr = (TensorInfo * n)()
    lib().mt_encoder_tensors(ctypes.byref(cfg), seed, arr, n)
    return list(arr)


def encoder_weights_struct(cfg: ModelConfig, base: int, tensors: list[TensorInfo]):
    """mt_encoder_weights over an arena at `base` (device or host) laid out as `tensors`.
    Returns (struct, keepalive)."""
    off = {t.name.decode(): t.offset for t in tensors}
    at = lambda name: base + off[name]
    keep = []

    def qwen(prefix, qc):
        layers = (QwenLayer * qc.layers)()
        for l in range(qc.layers):
            p = f"{prefix}.layers.{l}"
            layers[l] = QwenLayer(at(p + ".input_layernorm.weight"), at(p + ".self_attn.qkv_proj.weight"),
                                  at(p + ".self_attn.qkv_proj.bias"), at(p + ".self_attn.o_proj.weight"),
                                  at(p + ".post_attention_layernorm.weight"), at(p + ".mlp.gate_proj.weight"),
                                  at(p + ".mlp.up_proj.weight"), at(p + ".mlp.down_proj.weight"))
        keep.append(layers)
        return QwenWeights(qc, ctypes.cast(layers, POINTER(QwenLayer)), at(prefix + ".norm.weight"))

    e = "audio.encoder"
    agg_cfg = QwenConfig.from_buffer_copy(cfg.vae)
    agg_cfg.layers = 4
    w = EncoderWeights()
    w.frame, w.padded_frame, w.patch, w.max_frames = cfg.hop, (cfg.hop + 63) // 64 * 64, 4, 1600
    w.fc1_w, w.fc2_w, w.fc2_b = at(e + ".fc1.weight"), at(e + ".fc2.weight"), at(e + ".fc2.bias")
    w.stack = qwen(e + ".encoder", cfg.vae)
    w.aggregator = qwen(e + ".aggregator", agg_cfg)
    w.cls, w.fc3_w, w.fc3_b = at(e + ".cls_embed"), at(e + ".fc3.weight"), at(e + ".fc3.bias")
    return w, keep


def checkpoint_fill_encoder_arena(path: str, cfg: ModelConfig | None = None):
    """Host numpy uint8 encoder arena filled from a safetensors file. No GPU."""
    import numpy as np
    cfg = cfg if cfg is not None else default_config()
    nbytes = lib().mt_encoder_arena_bytes(ctypes.byref(cfg))
    arena = np.empty(nbytes, np.uint8)
    err = ctypes.create_string_buffer(512)
    st = lib().mt_checkpoint_fill_encoder_arena(str(path).encode(), ctypes.byref(cfg), arena.ctypes.data, nbytes, err,
                                                len(err))
    if st != MT_OK:
        raise (CheckpointError if st == MT_ERR_CHECKPOINT else MingError)(
            st, f"mt_checkpoint_fill_encoder_arena: {err.value.decode()}")
    return arena


class Encoder:
    """mt_encoder: the audio VAE encoder of the clone path (random-init from `seed`, or Encoder.load)."""

    def __init__(self, ctx: Context, cfg: ModelConfig | None = None, seed: int = 1, _handle=None):
        self.ctx = ctx
        self.cfg = cfg if cfg is not None else default_config()
        self.seed = seed
        self._e = c_void_p()
        if _handle is not None:
            self._e = _handle
            return
        ctx._check(lib().mt_encoder_create_random(ctx.handle, ctypes.byref(self.cfg), seed, ctypes.byref(self._e)),
                   "mt_encoder_create_random")

    @classmethod
    def load(cls, ctx: Context, path: str, cfg: ModelConfig | None = None) -> "Encoder":
        cfg = cfg if cfg is not None else default_config()
        h = c_void_p()
        st = lib().mt_encoder_load_safetensors(ctx.handle, ctypes.byref(cfg), str(path).encode(), ctypes.byref(h))
        if st != MT_OK:
            msg = lib().mt_last_error(ctx.handle).decode()
            raise (CheckpointError if st == MT_ERR_CHECKPOINT else MingError)(st, f"mt_encoder_load_safetensors: {msg}")
        return cls(ctx, cfg, seed=0, _handle=h)

    def tensors(self):
        return encoder_tensor_table(self.cfg, self.seed)

    def arena(self):
        p, n = c_void_p(), c_size_t()
        lib().mt_encoder_arena(self._e, ctypes.byref(p), ctypes.byref(n))
        return p.value, n.value

    def arena_to_host(self):
        import numpy as np
        p, nbytes = self.arena()
        return device_to_numpy(p, (nbytes,), np.uint8)

    def encode(self, samples, stream=None):
        """VAEEncoder.encode: posterior (mean, std), each [latents, latent_dim]."""
        import numpy as np
        x = np.ascontiguousarray(samples, np.float32)
        frames_per_latent = 4 * self.cfg.hop
        latents = x.size // frames_per_latent
        mean = np.zeros((latents, self.cfg.latent_dim), np.float32)
        std = np.zeros_like(mean)
        self.ctx._check(lib().mt_vae_encode(self._e, stream if stream is not None else current_stream(), x.ctypes.data,
                                            x.size, mean.ctypes.data, std.ctypes.data), "mt_vae_encode")
        return mean, std

    def close(self):
        if self._e:
            lib().mt_encoder_destroy(self._e)
            self._e = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------------------------------------
# 1-D convolutional waveform decoder (mt_convdec_*)
# ------------------------------------------------------------------------------------------------
def default_convdec_config() -> ConvDecConfig:
    """The decoder of BASELINE config 4: 64 latent channels, 512 -> 256 -> 128 -> 64 -> 64 channels,
    upsampling strides 8, 8, 4, 8 (2048 samples per latent frame), kernel 7."""
    c = ConvDecConfig()
    c.latent_dim = 64
    c.channels[:] = [512, 256, 128, 64, 64]
    c.strides[:] = [8, 8, 4, 8]
    c.kernel = 7
    return c


def convdec_shapes(cfg: ConvDecConfig):
    """(name, PyTorch-layout shape, fan_in) of every decoder tensor, in a fixed order."""
    C, S, K, L = list(cfg.channels), list(cfg.strides), cfg.kernel, cfg.latent_dim
    out = [("in_w", (C[0], L, K), L * K), ("in_b", (C[0],), 0)]
    for i in range(4):
        out += [(f"up_w{i}", (C[i], C[i + 1], 2 * S[i]), 2 * C[i]), (f"up_b{i}", (C[i + 1],), 0),
                (f"a_w{i}", (C[i + 1], C[i + 1], K), C[i + 1] * K), (f"a_b{i}", (C[i + 1],), 0),
                (f"b_w{i}", (C[i + 1], C[i + 1], K), C[i + 1] * K), (f"b_b{i}", (C[i + 1],), 0)]
    out += [("out_w", (1, C[4], K), C[4] * K), ("out_b", (1,), 0)]
    return out


def convdec_random_weights(cfg: ConvDecConfig, seed: int = 4):
    """Seeded random-init weights as bf16 bits (uint16) in PyTorch layouts: N(0, 1 / fan_in) for
    convolution weights (activations keep unit scale through the stack), N(0, 0.02^2) for biases;
    tensor i draws from the SplitMix stream seeded seed * 1000 + i."""
    import numpy as np
    out = {}
    for i, (name, shape, fan_in) in enumerate(convdec_shapes(cfg)):
        n = int(np.prod(shape))
        bits = np.zeros(n, np.uint16)
        std = (1.0 / fan_in) ** 0.5 if fan_in else 0.02
        lib().mt_randn_bf16_host(bits.ctypes.data, n, seed * 1000 + i, std)
        out[name] = bits.reshape(shape)
    return out


class ConvDecoder:
    """mt_convdec: latents [frames, latent_dim] -> PCM [frames * prod(strides)] on the tensor cores."""

    def __init__(self, ctx: Context, weights: dict, cfg: ConvDecConfig | None = None, max_frames: int = 216):
        import torch
        self.ctx = ctx
        self.cfg = cfg if cfg is not None else default_convdec_config()
        self.max_frames = max_frames
        dev = {k: torch.from_numpy(v.astype("uint16").view("int16").copy()).cuda() for k, v in weights.items()}
        w = ConvDecWeights()
        w.in_w, w.in_b, w.out_w, w.out_b = (dev[k].data_ptr() for k in ("in_w", "in_b", "out_w", "out_b"))
        for i in range(4):
            w.up_w[i], w.up_b[i] = dev[f"up_w{i}"].data_ptr(), dev[f"up_b{i}"].data_ptr()
            w.a_w[i], w.a_b[i] = dev[f"a_w{i}"].data_ptr(), dev[f"a_b{i}"].data_ptr()
            w.b_w[i], w.b_b[i] = dev[f"b_w{i}"].data_ptr(), dev[f"b_b{i}"].data_ptr()
        self._d = c_void_p()
        ctx._check(lib().mt_convdec_create(ctx.handle, ctypes.byref(self.cfg), ctypes.byref(w), max_frames,
                                           ctypes.byref(self._d)), "mt_convdec_create")
        del dev  # the decoder holds its own repacked copies

    def samples(self, frames: int) -> int:
        return int(lib().mt_convdec_samples(ctypes.byref(self.cfg), frames))

    def decode(self, latents, pcm=None, stream=None):
        """latents: CUDA fp32 tensor [frames, latent_dim]; returns (or fills) the CUDA fp32 PCM tensor."""
        import torch
        frames = latents.shape[0]
        if pcm is None:
            pcm = torch.empty(self.samples(frames), device=latents.device, dtype=torch.float32)
        self.ctx._check(lib().mt_convdec_decode(self._d, stream if stream is not None else current_stream(),
                                                latents.data_ptr(), frames, pcm.data_ptr()), "mt_convdec_decode")
        return pcm

    def close(self):
        if self._d:
            lib().mt_convdec_destroy(self._d)
            self._d = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def aggregate_latents(ctx: Context, model: "Model", latents, stream=None):
    """MingEngine.aggregate: [count, latent_dim] reference latents -> [count, llm.hidden] LLM input rows."""
    import numpy as np
    x = np.ascontiguousarray(latents, np.float32)
    count = x.shape[0]
    rows = np.zeros((count, model.cfg.llm.hidden), np.float32)
    ctx._check(lib().mt_aggregate_latents(ctx.handle, model.handle, stream if stream is not None else current_stream(),
                                          x.ctypes.data, count, rows.ctypes.data), "mt_aggregate_latents")
    return rows


class _DeviceView:
    """Exposes a raw device pointer through __cuda_array_interface__ (zero-copy view for torch)."""

    def __init__(self, address: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (address, False),
                                         "version": 3, "strides": None}


def device_view(address: int, shape, dtype="float32"):
    """A torch CUDA tensor viewing library-owned device memory (no copy)."""
    import numpy as np
    import torch
    return torch.as_tensor(_DeviceView(address, shape, np.dtype(dtype).str), device="cuda")


def device_to_numpy(address: int, shape, dtype="float32"):
    """Copies library-owned device memory into a new numpy array."""
    import torch
    torch.cuda.synchronize()
    return device_view(address, shape, dtype).cpu().numpy().copy()


PCM_CHUNK_FN = ctypes.CFUNCTYPE(c_int, c_void_p, c_int, c_int, c_int, c_void_p, ctypes.c_longlong)


def write_wav(path: str, samples, sample_rate: int = SAMPLE_RATE) -> None:
    """Mono float32 WAV, by default at the model's 44.1 kHz (mt_write_wav_f32; main.swift:134-144)."""
    import numpy as np
    x = np.ascontiguousarray(samples, np.float32)
    st = lib().mt_write_wav_f32(str(path).encode(), x.ctypes.data, x.size, sample_rate)
    if st != MT_OK:
        raise MingError(st, f"mt_write_wav_f32: cannot write {path}")


class Engine:
    """mt_engine: the generation loop for R concurrent requests."""

    def __init__(self, ctx: Context, model: Model, max_requests: int, max_prompt: int, max_steps: int,
                 use_graphs: bool = True, vae_ring: int = 0, groups: int = 0):
        self.ctx, self.model = ctx, model
        self.opt = EngineOptions(max_requests, max_prompt, max_steps, vae_ring, int(use_graphs), groups)
        self._e = c_void_p()
        ctx._check(lib().mt_engine_create(ctx.handle, model.handle, ctypes.byref(self.opt), ctypes.byref(self._e)),
                   "mt_engine_create")

    @property
    def handle(self):
        return self._e

    def begin(self, requests, prompt_rows, embeds=None, token_ids=None, noise=None, initial_history=None, steps=1,
              cfg=2.0, stream=None):
        self.ctx._check(lib().mt_engine_begin(self._e, stream if stream is not None else current_stream(), requests,
                                              prompt_rows, ptr(embeds), ptr(token_ids), ptr(noise),
                                              ptr(initial_history), steps, cfg), "mt_engine_begin")

    def prefill(self, stream=None):
        self.ctx._check(lib().mt_engine_prefill(self._e, stream if stream is not None else current_stream()),
                        "mt_engine_prefill")

    def step(self, stream=None) -> int:
        cnt = c_int()
        self.ctx._check(lib().mt_engine_step(self._e, stream if stream is not None else current_stream(),
                                             ctypes.byref(cnt)), "mt_engine_step")
        return cnt.value

    def flush(self, stream=None) -> int:
        cnt = c_int()
        self.ctx._check(lib().mt_engine_flush(self._e, stream if stream is not None else current_stream(),
                                              ctypes.byref(cnt)), "mt_engine_flush")
        return cnt.value

    def stage_timing(self, on: bool = True):
        self.ctx._check(lib().mt_engine_set_stage_timing(self._e, int(on)), "mt_engine_set_stage_timing")

    def stop_rule(self, on: bool = True):
        """mt_engine_set_stop_rule: generate/generate_stream end once every request has met
        p > 0.5 with n > 3 (Engine.swift:347-355); steps_done() then gives the steps run."""
        self.ctx._check(lib().mt_engine_set_stop_rule(self._e, int(on)), "mt_engine_set_stop_rule")

    def steps_done(self) -> int:
        return lib().mt_engine_steps_done(self._e)

    def stage_ms(self):
        """[llm, flow, agg, vae] GPU milliseconds of the last timed step."""
        out = (c_float * 4)()
        self.ctx._check(lib().mt_engine_stage_ms(self._e, out), "mt_engine_stage_ms")
        return list(out)

    def buffer(self, which: int):
        p, stride = c_void_p(), ctypes.c_longlong()
        self.ctx._check(lib().mt_engine_buffer(self._e, which, ctypes.byref(p), ctypes.byref(stride)),
                        "mt_engine_buffer")
        return p.value, stride.value

    def read(self, which: int, requests: int, count: int | None = None):
        """Host copy [requests, count] of an engine buffer (count defaults to the request stride)."""
        import numpy as np
        p, stride = self.buffer(which)
        full = device_to_numpy(p, (requests, stride))
        return full if count is None else np.ascontiguousarray(full[:, :count])

    def generate(self, requests, prompt_rows, noise_host, steps, cfg=2.0, embeds_host=None, ids_host=None,
                 stream=None):
        import numpy as np
        c = self.model.cfg
        stride = 4 * c.hop * steps
        pcm = np.zeros((requests, stride), np.float32)
        stop = np.zeros((requests, steps), np.float32)
        cnt = ctypes.c_longlong()
        self.ctx._check(lib().mt_engine_generate(self._e, stream if stream is not None else current_stream(), requests,
                                                 prompt_rows, ptr(embeds_host), ptr(ids_host), ptr(noise_host), steps,
                                                 cfg, ptr(pcm), stride, ctypes.byref(cnt), ptr(stop)),
                        "mt_engine_generate")
        return pcm[:, :cnt.value], stop

    def generate_stream(self, requests, prompt_rows, noise_host, steps, on_chunk, cfg=2.0, embeds_host=None,
                        ids_host=None, stream=None):
        """mt_engine_generate_stream: on_chunk(index, pcm[requests, count]) gets each PCM chunk (a
        numpy copy) as soon as it reaches the host; a truthy return cancels (MingError MT_ERR_STATE).
        Returns (samples per request, stop probabilities [requests, steps])."""
        import numpy as np
        stop = np.zeros((requests, steps), np.float32)
        cnt = ctypes.c_longlong()
        errors = []

        def trampoline(user, chunk, reqs, count, pcm, request_stride):
            try:
                view = np.ctypeslib.as_array(ctypes.cast(pcm, POINTER(c_float)), shape=(reqs * request_stride,))
                block = view.reshape(reqs, request_stride)[:, :count].copy()
                return 1 if on_chunk(chunk, block) else 0
            except BaseException as exc:  # surface callback errors after the C call returns
                errors.append(exc)
                return 1

        cb = PCM_CHUNK_FN(trampoline)
        st = lib().mt_engine_generate_stream(self._e, stream if stream is not None else current_stream(), requests,
                                             prompt_rows, ptr(embeds_host), ptr(ids_host), ptr(noise_host), steps,
                                             cfg, ctypes.cast(cb, c_void_p), None, ctypes.byref(cnt), ptr(stop))
        if errors:
            raise errors[0]
        self.ctx._check(st, "mt_engine_generate_stream")
        return cnt.value, stop

    def close(self):
        if self._e:
            lib().mt_engine_destroy(self._e)
            self._e = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
