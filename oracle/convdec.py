"""fp64 host restatement of the 1-D convolutional waveform decoder -- TEST INFRASTRUCTURE ONLY.

The decoder (mt_convdec_* in include/mingcuda.h) has no counterpart in the reference, whose VAE
decoder is the windowed Qwen stack + ISTFT (Sources/MingTTS/Engine/VAEDecoder.swift:1-108); this
file is the checker for the convolution stack that BASELINE config 4 describes, so its parity is
UNPINNED to the reference. What it does pin: conv1d and conv_transpose1d are restated here from
their textbook definitions (PyTorch semantics: cross-correlation, zero padding, ConvTranspose
output index i * stride - padding + k), and tests/test_convdec.py checks both against
torch.nn.functional in float64.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline may use this module.
"""
from __future__ import annotations

import numpy as np


class Config:
    """The decoder's shape (mirrors mt_convdec_config)."""

    def __init__(self, latent_dim=64, channels=(512, 256, 128, 64, 64), strides=(8, 8, 4, 8), kernel=7):
        self.latent_dim, self.channels, self.strides, self.kernel = latent_dim, list(channels), list(strides), kernel


def default_config() -> Config:
    return Config()


def shapes(cfg):
    """(name, PyTorch-layout shape, fan_in) of every tensor, in the order the seeds are assigned."""
    C, S, K, L = list(cfg.channels), list(cfg.strides), cfg.kernel, cfg.latent_dim
    out = [("in_w", (C[0], L, K), L * K), ("in_b", (C[0],), 0)]
    for i in range(4):
        out += [(f"up_w{i}", (C[i], C[i + 1], 2 * S[i]), 2 * C[i]), (f"up_b{i}", (C[i + 1],), 0),
                (f"a_w{i}", (C[i + 1], C[i + 1], K), C[i + 1] * K), (f"a_b{i}", (C[i + 1],), 0),
                (f"b_w{i}", (C[i + 1], C[i + 1], K), C[i + 1] * K), (f"b_b{i}", (C[i + 1],), 0)]
    out += [("out_w", (1, C[4], K), C[4] * K), ("out_b", (1,), 0)]
    return out


def random_weights(cfg, seed: int = 4) -> dict:
    """The seeded random init as real values: tensor i is N(0, 1 / fan_in) (weights) or N(0, 0.02^2)
    (biases) from the SplitMix stream seeded seed * 1000 + i, rounded to bf16."""
    import oracle
    out = {}
    for i, (name, shape, fan_in) in enumerate(shapes(cfg)):
        n = int(np.prod(shape))
        std = (1.0 / fan_in) ** 0.5 if fan_in else 0.02
        out[name] = oracle.bf16_to_f32(oracle.randn_bf16(n, seed * 1000 + i, std)).reshape(shape)
    return out


def silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


def conv1d(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """y[t, co] = b[co] + sum_{ci, k} w[co, ci, k] x[t + k - (K - 1) / 2, ci] (zero outside).
    x: [T, C_in] time-major; w: [C_out, C_in, K] (K odd)."""
    T, K = x.shape[0], w.shape[2]
    half = (K - 1) // 2
    xp = np.zeros((T + 2 * half, x.shape[1]), np.float64)
    xp[half:half + T] = x
    y = np.tile(b.astype(np.float64), (T, 1))
    for k in range(K):
        y += xp[k:k + T] @ w[:, :, k].T.astype(np.float64)
    return y


def conv_transpose1d(x: np.ndarray, w: np.ndarray, b: np.ndarray, stride: int) -> np.ndarray:
    """out[o, co] = b[co] + sum_{i, k: o = i * stride - p + k} w[ci, co, k] x[i, ci], p = stride / 2,
    kernel 2 * stride: T * stride outputs. x: [T, C_in]; w: [C_in, C_out, 2 * stride]."""
    T, Kt = x.shape[0], w.shape[2]
    p = stride // 2
    full = (T - 1) * stride + Kt
    acc = np.zeros((full, w.shape[1]), np.float64)
    for k in range(Kt):
        acc[k:k + (T - 1) * stride + 1:stride] += x.astype(np.float64) @ w[:, :, k].astype(np.float64)
    return acc[p:p + T * stride] + b.astype(np.float64)


def decode(cfg, weights: dict, latents: np.ndarray) -> np.ndarray:
    """The whole decoder in fp64: latents [frames, latent_dim] -> PCM [frames * prod(strides)].
    `weights` maps the names of mingtts_b200.convdec_shapes to real-valued arrays (bf16 values)."""
    W = {k: np.asarray(v, np.float64) for k, v in weights.items()}
    x = conv1d(np.asarray(latents, np.float64), W["in_w"], W["in_b"])
    for i in range(4):
        u = conv_transpose1d(silu(x), W[f"up_w{i}"], W[f"up_b{i}"], int(cfg.strides[i]))
        h = conv1d(silu(u), W[f"a_w{i}"], W[f"a_b{i}"])
        x = u + conv1d(silu(h), W[f"b_w{i}"], W[f"b_b{i}"])
    return np.tanh(conv1d(silu(x), W["out_w"], W["out_b"])[:, 0])
