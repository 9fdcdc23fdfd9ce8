"""Generates tests/golden/golden.npz: known-answer vectors for the oracle, computed with
implementations that share no code with it (pure Python integers, numpy float64, torch).

Each case follows a CPU reference of the reference's kernel tests
(maralski/ming-tts Tests/MingTTSTests/KernelTests.swift) or a published algorithm:
  lcg        KernelTests.swift:21-28 LCG (pure Python ints)
  splitmix   SplitMix64 (Vigna) -- published vector for seed 1234567 -- and the
             gaussianNoise Box-Muller of Engine.swift:433-453 (pure Python, math module)
  bf16       float32 -> bfloat16 round-to-nearest-even (torch's own conversion)
  linear_*   y = epi(x W^T) in numpy float64 (KernelTests.swift:86-101)
  rmsnorm    torch float64 (KernelTests.swift:195-201)
  attn_*     NeoX RoPE + causal/windowed GQA softmax attention in numpy float64
             (KernelTests.swift:207-266)
  dit_attn   interleaved RoPE full attention in numpy float64 (KernelTests.swift:282-322)
  istft      numpy.fft.irfft per frame, window, overlap-add, envelope (KernelTests.swift:327-379)
  upsample   torch.nn.functional.interpolate(linear, x4, align_corners=False) (KernelTests.swift:383-403)
  timesteps  EPSS-10 + sway (DiT.swift:56-65) in numpy float32
  sinusoid   SinusPositionEmbedding(256, scale 1000) in torch float32 (DiT.swift:68-79)

Inputs are not stored: tests regenerate them from the same LCG seeds (the LCG itself is pinned
by lcg_seed12345). Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import math
import os

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
M64 = (1 << 64) - 1


def lcg(seed: int, n: int, scale: float = 1.0) -> np.ndarray:
    s = seed
    out = np.empty(n, np.float32)
    for i in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & M64
        out[i] = np.float32(np.float32(s >> 40) / np.float32(1 << 24) * np.float32(2) - np.float32(1)) * np.float32(scale)
    return out


def splitmix_outputs(x: int, n: int) -> list[int]:
    out = []
    for _ in range(n):
        x = (x + 0x9E3779B97F4A7C15) & M64
        z = x
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
        out.append(z ^ (z >> 31))
    return out


def gaussian_noise(n: int, seed: int) -> np.ndarray:
    # state starts at seed + golden; each draw first advances by golden (Engine.swift:434-442).
    draws = splitmix_outputs((seed + 0x9E3779B97F4A7C15) & M64, n + 2)
    u = [(d >> 11) / float(1 << 53) for d in draws]
    out = np.empty(n, np.float32)
    i = 0
    while i < n:
        u1, u2 = max(u[i], 1e-300), u[i + 1]
        r = math.sqrt(-2.0 * math.log(u1))
        out[i] = np.float32(r * math.cos(2.0 * math.pi * u2))
        if i + 1 < n:
            out[i + 1] = np.float32(r * math.sin(2.0 * math.pi * u2))
        i += 2
    return out


def bf16_bits_torch(x: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16).copy()


def bf16_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def gelu_tanh(v):
    u = np.clip(np.float32(0.7978845608028654) * (v + np.float32(0.044715) * v * v * v), -15, 15)
    return (np.float32(0.5) * v * (np.float32(1) + np.tanh(u))).astype(np.float32)


def silu(v):
    return (v / (np.float32(1) + np.exp(-v))).astype(np.float32)


def linear_case(m, n, k, flags, seed):
    x = lcg(seed, m * k).reshape(m, k)
    w = bf16_bits_torch(lcg(seed + 1, n * k, 0.1)).reshape(n, k)
    w2 = bf16_bits_torch(lcg(seed + 2, n * k, 0.1)).reshape(n, k)
    b = bf16_bits_torch(lcg(seed + 3, n))
    y0 = lcg(seed + 4, m * n).reshape(m, n)
    acc = (x.astype(np.float64) @ bf16_f32(w).astype(np.float64).T).astype(np.float32)
    acc2 = (x.astype(np.float64) @ bf16_f32(w2).astype(np.float64).T).astype(np.float32)
    v = acc + (bf16_f32(b)[None, :] if flags & 1 else np.float32(0))
    if flags & 8:
        v = silu(v) * acc2
    if flags & 4:
        v = gelu_tanh(v)
    if flags & 16:
        v = silu(v)
    if flags & 2:
        v = v + y0
    return dict(want=v.astype(np.float32), shape=np.array([m, n, k, flags]))


def neox(v, pos, inv):
    a = (np.float32(pos) * inv).astype(np.float32).astype(np.float64)
    c, s = np.cos(a), np.sin(a)
    out = v.astype(np.float64).copy()
    out[:32] = v[:32] * c - v[32:] * s
    out[32:] = v[32:] * c + v[:32] * s
    return out


def attention_case(t0, m, window, seed):
    hq, hkv = 14, 2
    ld = (hq + 2 * hkv) * 64
    total = t0 + m
    qkv = lcg(seed, total * ld).reshape(total, ld)
    inv = (1.0 / np.power(np.float32(1e6), np.arange(32, dtype=np.float32) * 2 / 64)).astype(np.float32)
    ks = [[neox(qkv[p, (hq + h) * 64:(hq + h + 1) * 64], p, inv) for p in range(total)] for h in range(hkv)]
    want = np.zeros((total, hq * 64))
    for p in range(total):
        j0 = p + 1 - window if (window > 0 and p + 1 > window) else 0
        for h in range(hq):
            q = neox(qkv[p, h * 64:(h + 1) * 64], p, inv)
            g = h // (hq // hkv)
            sc = np.array([q @ ks[g][j] for j in range(j0, p + 1)]) / 8.0
            e = np.exp(sc - sc.max())
            e /= e.sum()
            vs = np.stack([qkv[j, (hq + hkv + g) * 64:(hq + hkv + g + 1) * 64].astype(np.float64) for j in range(j0, p + 1)])
            want[p, h * 64:(h + 1) * 64] = e @ vs
    return dict(want=want.astype(np.float32), shape=np.array([t0, m, window, hq, hkv]))


def dit_attention_case(seed):
    B, S, H = 2, 3, 16
    D = H * 64
    ld = 3 * D
    qkv = lcg(seed, B * S * ld).reshape(B * S, ld)
    inv = (1.0 / np.power(np.float32(1e4), np.arange(32, dtype=np.float32) * 2 / 64)).astype(np.float32)

    def rope(v, pos):
        a = (np.float32(pos) * inv).astype(np.float32).astype(np.float64)
        c, s = np.cos(a), np.sin(a)
        o = v.astype(np.float64).copy()
        o[0::2] = v[0::2] * c - v[1::2] * s
        o[1::2] = v[1::2] * c + v[0::2] * s
        return o

    want = np.zeros((B * S, D))
    for b in range(B):
        for h in range(H):
            for i in range(S):
                q = rope(qkv[b * S + i, h * 64:(h + 1) * 64], i)
                sc = np.array([q @ rope(qkv[b * S + j, D + h * 64:D + (h + 1) * 64], j) for j in range(S)]) / 8.0
                e = np.exp(sc - sc.max())
                e /= e.sum()
                want[b * S + i, h * 64:(h + 1) * 64] = sum(e[j] * qkv[b * S + j, 2 * D + h * 64:2 * D + (h + 1) * 64].astype(np.float64) for j in range(S))
    return dict(want=want.astype(np.float32), shape=np.array([B, S, H]))


def istft_case(seed):
    nfft, hop, frames = 3528, 882, 8
    bins = nfft // 2 + 1
    r = lcg(seed, frames * bins * 2)
    spec = np.zeros((frames, 2 * bins), np.float32)
    it = iter(range(0, len(r), 2))
    for f in range(frames):
        for k in range(bins):
            i = next(it)
            spec[f, k] = r[i] * 2 - 1
            spec[f, bins + k] = r[i + 1] * 3
    window = (0.5 - 0.5 * np.cos(2 * np.pi * np.arange(nfft) / nfft)).astype(np.float32)
    mag = np.minimum(np.exp(spec[:, :bins].astype(np.float64)), 100.0)
    ph = spec[:, bins:].astype(np.float64)
    X = mag * np.exp(1j * ph)
    X[:, 0] = X[:, 0].real  # irfft ignores the imaginary parts of DC and Nyquist, as the direct sum does
    X[:, -1] = X[:, -1].real
    fr = np.fft.irfft(X, n=nfft, axis=1) * window.astype(np.float64)[None, :]
    full = (frames - 1) * hop + nfft
    y = np.zeros(full)
    env = np.zeros(full)
    for f in range(frames):
        y[f * hop:f * hop + nfft] += fr[f]
        env[f * hop:f * hop + nfft] += window.astype(np.float64) ** 2
    pad = (nfft - hop) // 2
    total = frames * hop
    want = (y[pad:pad + total] / env[pad:pad + total]).astype(np.float32)
    return dict(want=want, shape=np.array([nfft, hop, frames]))


def upsample_case(seed):
    hidden, n = 896, 5
    h = lcg(seed, n * hidden).reshape(n, hidden)
    t = torch.from_numpy(h.T.copy()).double()[None]  # [1, C, n]
    up = torch.nn.functional.interpolate(t, scale_factor=4, mode="linear", align_corners=False)
    return dict(want=up[0].T.float().numpy().copy(), shape=np.array([hidden, n]))


def timesteps():
    base = np.array([0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32], np.float32) / np.float32(32)
    return (base - (np.cos(np.float32(np.pi / 2) * base).astype(np.float32) - np.float32(1) + base)).astype(np.float32)


def sinusoid(t: float) -> np.ndarray:
    half = 128
    emb = math.log(10000) / (half - 1)
    emb = torch.exp(torch.arange(half, dtype=torch.float32) * -emb)
    emb = 1000.0 * torch.tensor([t], dtype=torch.float32)[:, None] * emb[None, :]
    return torch.cat((emb.sin(), emb.cos()), dim=-1)[0].numpy()


def main():
    g = {}
    g["lcg_seed12345"] = lcg(12345, 64)
    g["splitmix_1234567"] = np.array(splitmix_outputs(1234567, 5), np.uint64)
    g["gauss_seed0"] = gaussian_noise(64, 0)
    g["gauss_seed3"] = gaussian_noise(64, 3)
    xs = np.concatenate([lcg(7, 4096, 50.0), np.array([0.0, -0.0, 1.0, 65504.0, 1e-40, -3.3895314e38], np.float32)])
    g["bf16_in"] = xs
    g["bf16_out"] = bf16_bits_torch(xs)
    for name, (m, n, k, flags) in {
        "linear_a": (1, 384, 896, 1), "linear_b": (2, 2, 896, 1), "linear_c": (4, 96, 512, 2),
        "linear_d": (6, 128, 256, 5), "linear_e": (3, 64, 1024, 1), "linear_f": (5, 64, 896, 8),
        "linear_g": (1, 64, 896, 16), "linear_h": (21, 40, 128, 0),
    }.items():
        for key, v in linear_case(m, n, k, flags, seed=m * 1000 + n * 7 + k).items():
            g[f"{name}_{key}"] = v
    x = lcg(3, 5 * 896, 3.0).reshape(5, 896)
    w = bf16_bits_torch(lcg(4, 896))
    xt = torch.from_numpy(x).double()
    g["rms_want"] = (xt * torch.rsqrt(xt.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(bf16_f32(w)).double()).float().numpy()
    for name, (t0, m, window) in {"attn_a": (37, 1, 0), "attn_b": (20, 4, 0), "attn_c": (70, 4, 64)}.items():
        for key, v in attention_case(t0, m, window, seed=t0 * 31 + m + window).items():
            g[f"{name}_{key}"] = v
    for key, v in dit_attention_case(11).items():
        g[f"dit_{key}"] = v
    for key, v in istft_case(5).items():
        g[f"istft_{key}"] = v
    for key, v in upsample_case(9).items():
        g[f"up_{key}"] = v
    g["timesteps10"] = timesteps()
    g["sinusoid_t"] = np.array([0.0, 0.0302, 0.5, 1.0], np.float32)
    g["sinusoid_want"] = np.stack([sinusoid(float(t)) for t in g["sinusoid_t"]])
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT}: {len(g)} arrays, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
