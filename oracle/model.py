"""Host model for the CPU oracle -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Builds the seeded random-init weights of Ming-3.0-tts-0.5B in host memory without the product
library: the tensor list (checkpoint names and shapes of Sources/MingTTS/Engine/Weights.swift:81-263,
q/k/v concatenated as Weights.swift:121-125, 158-159 do), the synthetic-data convention of the
product's model table (tensor i of the table draws bf16 N(0, 0.02) from SplitMix64 stream
seed * 1000003 + i; norm gains 1.0; DiT rotary inv_freq 1/10000^(2i/64); periodic Hann ISTFT window),
and ctypes mirrors of the mt_model_config / mt_model_weights structs of include/mingcuda.h that the
oracle's C code takes. bench.py's reference arm and CPU baseline use this, so that timing the CPU
restatement loads liboracle.so only; tests/test_oracle_model.py checks the table against the
product's mt_model_tensors.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_void_p

import numpy as np

from . import bf16_to_f32, randn_bf16

BF16, F32 = 0, 1
NORMAL, ONES, INV_FREQ, HANN = 0, 1, 2, 3


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


def default_config() -> ModelConfig:
    """Ming-3.0-tts-0.5B dimensions: QwenConfig (Weights.swift:81-92), the VAE decoder's 65-key window
    (:216-217), DiT 1024/16/8/4096 (:146-189), latent 64, nfft 3528 / hop 882, 10 flow steps, 512 positions."""
    c = ModelConfig()
    c.llm = QwenConfig(896, 14, 2, 4864, 24, 0, 1e6, 1e-6)
    c.vae = QwenConfig(896, 14, 2, 4864, 24, 65, 1e6, 1e-6)
    c.flow = DitConfig(1024, 16, 8, 4096, 64, 1e-6)
    c.agg = DitConfig(1024, 16, 8, 4096, 896, 1e-6)
    c.latent_dim, c.time_dim, c.vocab, c.nfft, c.hop, c.flow_steps, c.llm_capacity = 64, 256, 151936, 3528, 882, 10, 512
    return c


def tensor_list(cfg: ModelConfig, with_embeddings: bool = True):
    """[(name, numel, dtype, init)] in table order (the order fixes each tensor's seed)."""
    out = []

    def bf(name, n):
        out.append((name, int(n), BF16, NORMAL))

    def ones(name, n):
        out.append((name, int(n), BF16, ONES))

    def qwen(prefix, c):
        h, qkv, inter = c.hidden, (c.heads + 2 * c.kv_heads) * 64, c.intermediate
        for l in range(c.layers):
            p = f"{prefix}.layers.{l}"
            ones(p + ".input_layernorm.weight", h)
            bf(p + ".self_attn.qkv_proj.weight", qkv * h)
            bf(p + ".self_attn.qkv_proj.bias", qkv)
            bf(p + ".self_attn.o_proj.weight", h * c.heads * 64)
            ones(p + ".post_attention_layernorm.weight", h)
            bf(p + ".mlp.gate_proj.weight", inter * h)
            bf(p + ".mlp.up_proj.weight", inter * h)
            bf(p + ".mlp.down_proj.weight", h * inter)
        ones(prefix + ".norm.weight", h)

    def dit(prefix, c):
        h, ff = c.hidden, c.ff
        for i in range(c.depth):
            p = f"{prefix}.blocks.{i}"
            ones(p + ".norm1.weight", h)
            bf(p + ".attn.to_qkv.weight", 3 * h * h)
            bf(p + ".attn.to_qkv.bias", 3 * h)
            bf(p + ".attn.to_out.0.weight", h * h)
            bf(p + ".attn.to_out.0.bias", h)
            ones(p + ".norm2.weight", h)
            bf(p + ".mlp.ff.0.0.weight", ff * h)
            bf(p + ".mlp.ff.0.0.bias", ff)
            bf(p + ".mlp.ff.2.weight", h * ff)
            bf(p + ".mlp.ff.2.bias", h)
        ones(prefix + ".final_layer.norm_final.weight", h)
        bf(prefix + ".final_layer.linear.weight", c.out_dim * h)
        bf(prefix + ".final_layer.linear.bias", c.out_dim)
        out.append((prefix + ".rotary_embed.inv_freq", 32, F32, INV_FREQ))

    qwen("model.model", cfg.llm)
    bf("stop_head.weight", 2 * cfg.llm.hidden)
    bf("stop_head.bias", 2)
    f = "flowloss.cfm.model"
    bf(f + ".x_embedder.weight", cfg.flow.hidden * cfg.latent_dim)
    bf(f + ".x_embedder.bias", cfg.flow.hidden)
    bf(f + ".c_embedder.cond_embedder.weight", cfg.flow.hidden * cfg.llm.hidden)
    bf(f + ".c_embedder.cond_embedder.bias", cfg.flow.hidden)
    bf(f + ".t_embedder.time_mlp.0.weight", cfg.flow.hidden * cfg.time_dim)
    bf(f + ".t_embedder.time_mlp.0.bias", cfg.flow.hidden)
    bf(f + ".t_embedder.time_mlp.2.weight", cfg.flow.hidden * cfg.flow.hidden)
    bf(f + ".t_embedder.time_mlp.2.bias", cfg.flow.hidden)
    dit(f, cfg.flow)
    a = "linear_proj_audio"
    bf(a + ".x_embedder.weight", cfg.agg.hidden * cfg.latent_dim)
    bf(a + ".x_embedder.bias", cfg.agg.hidden)
    out.append((a + ".word_embedder.weight", cfg.agg.hidden, F32, NORMAL))
    dit(a, cfg.agg)
    v = "audio.decoder"
    bf(v + ".fc1.weight", cfg.vae.hidden * cfg.latent_dim)
    bf(v + ".fc1.bias", cfg.vae.hidden)
    qwen(v + ".decoder", cfg.vae)
    bf(v + ".head.out.weight", (cfg.nfft + 2) * cfg.vae.hidden)
    bf(v + ".head.out.bias", cfg.nfft + 2)
    out.append((v + ".head.istft.window", cfg.nfft, F32, HANN))
    if with_embeddings:
        bf("model.model.embed_tokens.weight", cfg.vocab * cfg.llm.hidden)
    return out


def tensor_seed(seed: int, index: int) -> int:
    return (seed * 1000003 + index) & 0xFFFFFFFFFFFFFFFF


def fill(numel: int, dtype: int, init: int, seed: int, std: float = 0.02) -> np.ndarray:
    """One tensor's values: uint16 bf16 bits or float32."""
    if dtype == BF16:
        if init == ONES:
            return np.full(numel, 0x3F80, np.uint16)
        return randn_bf16(numel, seed, std)
    if init == NORMAL:
        return bf16_to_f32(randn_bf16(numel, seed, std)).astype(np.float32)
    if init == INV_FREQ:
        return (1.0 / np.power(10000.0, 2 * np.arange(numel) / 64.0)).astype(np.float32)
    return (0.5 - 0.5 * np.cos(2 * np.pi * np.arange(numel) / numel)).astype(np.float32)


class HostModel:
    """Every tensor as its own host array and the ModelWeights struct pointing at them."""

    def __init__(self, cfg: ModelConfig | None = None, seed: int = 1, with_embeddings: bool = True):
        self.cfg = cfg if cfg is not None else default_config()
        self.arrays = {}
        for i, (name, numel, dtype, init) in enumerate(tensor_list(self.cfg, with_embeddings)):
            self.arrays[name] = fill(numel, dtype, init, tensor_seed(seed, i))
        self._keep = []
        self.weights = self._struct()

    def at(self, name):
        a = self.arrays.get(name)
        return None if a is None else a.ctypes.data

    def _struct(self) -> ModelWeights:
        at, keep = self.at, self._keep

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
                blocks[i] = DitBlock(at(p + ".norm1.weight"), at(p + ".attn.to_qkv.weight"),
                                     at(p + ".attn.to_qkv.bias"), at(p + ".attn.to_out.0.weight"),
                                     at(p + ".attn.to_out.0.bias"), at(p + ".norm2.weight"),
                                     at(p + ".mlp.ff.0.0.weight"), at(p + ".mlp.ff.0.0.bias"),
                                     at(p + ".mlp.ff.2.weight"), at(p + ".mlp.ff.2.bias"))
            keep.append(blocks)
            return DitWeights(dc, ctypes.cast(blocks, POINTER(DitBlock)), at(prefix + ".final_layer.norm_final.weight"),
                              at(prefix + ".final_layer.linear.weight"), at(prefix + ".final_layer.linear.bias"),
                              at(prefix + ".rotary_embed.inv_freq"))

        c = self.cfg
        f, a, v = "flowloss.cfm.model", "linear_proj_audio", "audio.decoder"
        w = ModelWeights()
        w.llm = qwen("model.model", c.llm)
        w.stop_w, w.stop_b = at("stop_head.weight"), at("stop_head.bias")
        w.flow_x_w, w.flow_x_b = at(f + ".x_embedder.weight"), at(f + ".x_embedder.bias")
        w.flow_c_w, w.flow_c_b = at(f + ".c_embedder.cond_embedder.weight"), at(f + ".c_embedder.cond_embedder.bias")
        w.flow_t1_w, w.flow_t1_b = at(f + ".t_embedder.time_mlp.0.weight"), at(f + ".t_embedder.time_mlp.0.bias")
        w.flow_t2_w, w.flow_t2_b = at(f + ".t_embedder.time_mlp.2.weight"), at(f + ".t_embedder.time_mlp.2.bias")
        w.flow = dit(f, c.flow)
        w.agg_x_w, w.agg_x_b = at(a + ".x_embedder.weight"), at(a + ".x_embedder.bias")
        w.agg_cls = at(a + ".word_embedder.weight")
        w.agg = dit(a, c.agg)
        w.vae_fc1_w, w.vae_fc1_b = at(v + ".fc1.weight"), at(v + ".fc1.bias")
        w.vae = qwen(v + ".decoder", c.vae)
        w.vae_head_w, w.vae_head_b = at(v + ".head.out.weight"), at(v + ".head.out.bias")
        w.vae_window = at(v + ".head.istft.window")
        w.embed_tokens = at("model.model.embed_tokens.weight")
        return w

    def embed(self, ids: np.ndarray) -> np.ndarray:
        """Prompt embeddings: rows of embed_tokens widened to fp32 (Engine.swift:204-222)."""
        H = self.cfg.llm.hidden
        table = self.arrays["model.model.embed_tokens.weight"].reshape(-1, H)
        return np.ascontiguousarray(bf16_to_f32(table[ids]), np.float32)
