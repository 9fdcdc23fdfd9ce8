"""CPU checks of the oracle's generation loop and of the model tensor table (no GPU)."""
from __future__ import annotations

import ctypes

import numpy as np

from test_engine_gpu import oracle_generate


def host_arena(mt, oracle, cfg, seed):
    """Builds the model arena on the host from the tensor table, with the oracle's generator."""
    tensors = mt.tensor_table(cfg, seed)
    nbytes = mt.lib().mt_model_arena_bytes(ctypes.byref(cfg), 1)
    arena = np.zeros(nbytes, np.uint8)
    for t in tensors:
        if t.dtype == mt.MT_DTYPE_BF16:
            view = arena[t.offset:t.offset + 2 * t.numel].view(np.uint16)
            view[:] = 0x3F80 if t.init == 1 else oracle.randn_bf16(t.numel, t.seed, t.std)
        else:
            view = arena[t.offset:t.offset + 4 * t.numel].view(np.float32)
            if t.init == 0:
                view[:] = oracle.bf16_to_f32(oracle.randn_bf16(t.numel, t.seed, t.std))
            elif t.init == 2:
                view[:] = (1.0 / np.power(10000.0, 2 * np.arange(t.numel) / 64.0)).astype(np.float32)
            elif t.init == 3:
                view[:] = (0.5 - 0.5 * np.cos(2 * np.pi * np.arange(t.numel) / t.numel)).astype(np.float32)
    return arena, tensors


def test_tensor_table_layout(mt):
    cfg = mt.default_config()
    t = mt.tensor_table(cfg)
    names = [x.name.decode() for x in t]
    assert len(names) == len(set(names))
    assert all(x.offset % 256 == 0 for x in t)
    assert all(a.offset + a.numel * (2 if a.dtype == 0 else 4) <= b.offset for a, b in zip(t, t[1:]))
    # The per-step weights of Ming-3.0-tts-0.5B (LLM + flow + aggregator + VAE decoder): ~0.92 B parameters.
    per_step = sum(x.numel for x in t if not x.name.startswith(b"model.model.embed_tokens"))
    assert 0.90e9 < per_step < 0.95e9
    qkv = next(x for x in t if x.name == b"model.model.layers.0.self_attn.qkv_proj.weight")
    assert qkv.numel == (14 + 2 * 2) * 64 * 896


def test_oracle_generation_bookkeeping(mt, oracle):
    cfg = mt.small_config()
    arena, tensors = host_arena(mt, oracle, cfg, seed=3)
    w, keep = mt.weights_struct(cfg, arena.ctypes.data, tensors)
    steps, T = 5, 4
    rs = np.random.default_rng(0)
    embeds = (0.5 * rs.standard_normal((T, cfg.llm.hidden))).astype(np.float32)
    noise = oracle.gaussian_noise(steps * cfg.latent_dim, 7).reshape(steps, cfg.latent_dim)
    a = oracle_generate(oracle, cfg, w, embeds, noise, steps)
    b = oracle_generate(oracle, cfg, w, embeds, noise, steps)
    hop, pad = cfg.hop, (cfg.nfft - cfg.hop) // 2
    # Emissions: latent 0 at step 2 (4 hops minus the pad), then 4 hops each, the last adds the pad
    # (VAEDecoder.swift:93-99); total = 4 hops per latent.
    assert list(a["chunks"]) == [4 * hop - pad] + [4 * hop] * (steps - 2) + [4 * hop + pad]
    assert a["pcm"].size == 4 * hop * steps
    np.testing.assert_array_equal(a["pcm"], b["pcm"])
    np.testing.assert_array_equal(a["latents"], b["latents"])
    assert np.isfinite(a["pcm"]).all() and np.abs(a["pcm"]).max() > 0
    # The latent history feeds the next step: different noise at step 1 changes latent 1 only from there on.
    noise2 = noise.copy()
    noise2[1] += 1.0
    c = oracle_generate(oracle, cfg, w, embeds, noise2, steps)
    np.testing.assert_array_equal(a["latents"][0], c["latents"][0])
    assert not np.allclose(a["latents"][1], c["latents"][1])


def test_oracle_stop_rule(mt, oracle):
    """obey_stop (Engine.swift:347-367): with the stop bias pinned so p ~ 1 the loop ends after step
    n = 4 (the rule needs n > 3) and flushes, which is exactly a 5-step run on the same noise; with
    p ~ 0 every step runs."""
    cfg = mt.small_config()
    arena, tensors = host_arena(mt, oracle, cfg, seed=5)
    off = {t.name.decode(): t.offset for t in tensors}["stop_head.bias"]
    bias = arena[off:off + 4].view(np.uint16)
    w, keep = mt.weights_struct(cfg, arena.ctypes.data, tensors)
    steps, T = 9, 3
    rs = np.random.default_rng(5)
    embeds = (0.5 * rs.standard_normal((T, cfg.llm.hidden))).astype(np.float32)
    noise = oracle.gaussian_noise(steps * cfg.latent_dim, 11).reshape(steps, cfg.latent_dim)
    bias[:] = [0xC180, 0x4180]  # bf16 -16, +16
    stopped = oracle_generate(oracle, cfg, w, embeds, noise, steps, obey_stop=1)
    fixed = oracle_generate(oracle, cfg, w, embeds, np.ascontiguousarray(noise[:5]), 5)
    assert stopped["stopped"] == 1 and stopped["steps_run"] == 5
    assert list(stopped["chunks"]) == list(fixed["chunks"])
    np.testing.assert_array_equal(stopped["pcm"], fixed["pcm"])
    bias[:] = [0x4180, 0xC180]
    never = oracle_generate(oracle, cfg, w, embeds, noise, steps, obey_stop=1)
    assert never["stopped"] == 0 and never["steps_run"] == steps and never["pcm"].size == 4 * cfg.hop * steps


def test_oracle_initial_history(mt, oracle):
    """The history buffer is zeroed and then overwritten by initialHistory when one is given
    (Engine.swift:314-315): an all-zero history gives exactly the run without one, a reference
    voice's latent changes the generation from step 0 on."""
    cfg = mt.small_config()
    arena, tensors = host_arena(mt, oracle, cfg, seed=8)
    w, keep = mt.weights_struct(cfg, arena.ctypes.data, tensors)
    steps, T = 4, 3
    rs = np.random.default_rng(8)
    embeds = (0.5 * rs.standard_normal((T, cfg.llm.hidden))).astype(np.float32)
    noise = oracle.gaussian_noise(steps * cfg.latent_dim, 13).reshape(steps, cfg.latent_dim)
    plain = oracle_generate(oracle, cfg, w, embeds, noise, steps)
    zeros = oracle_generate(oracle, cfg, w, embeds, noise, steps,
                            initial_history=np.zeros(cfg.latent_dim, np.float32))
    voice = oracle_generate(oracle, cfg, w, embeds, noise, steps,
                            initial_history=rs.standard_normal(cfg.latent_dim).astype(np.float32))
    np.testing.assert_array_equal(zeros["latents"], plain["latents"])
    np.testing.assert_array_equal(zeros["pcm"], plain["pcm"])
    assert np.abs(voice["latents"][0] - plain["latents"][0]).max() > 1e-3


def test_oracle_stage_helpers_match_generation(mt, oracle):
    """or_flow_patch and or_vae_decode_clip (the CPU legs of BASELINE configs 3 and 4) reproduce the
    generation loop's own stages: step 0's latent from z with a zero history, and the whole waveform
    from the loop's latents."""
    cfg = mt.small_config()
    arena, tensors = host_arena(mt, oracle, cfg, seed=5)
    w, keep = mt.weights_struct(cfg, arena.ctypes.data, tensors)
    steps, T, L = 5, 4, cfg.latent_dim
    rs = np.random.default_rng(1)
    embeds = (0.5 * rs.standard_normal((T, cfg.llm.hidden))).astype(np.float32)
    noise = oracle.gaussian_noise(steps * L, 8).reshape(steps, L)
    g = oracle_generate(oracle, cfg, w, embeds, noise, steps)
    y = np.zeros(L, np.float32)
    z0 = np.ascontiguousarray(g["z"][0])
    hist = np.zeros(L, np.float32)
    n0 = np.ascontiguousarray(noise[0])
    assert oracle.lib().or_flow_patch(ctypes.addressof(cfg), ctypes.addressof(w), z0.ctypes.data, hist.ctypes.data,
                                      n0.ctypes.data, 2.0, y.ctypes.data) == 0
    np.testing.assert_array_equal(y, g["latents"][0])
    lat = np.ascontiguousarray(g["latents"])
    pcm = np.zeros(4 * cfg.hop * (steps + 1), np.float32)
    n = oracle.lib().or_vae_decode_clip(ctypes.addressof(cfg), ctypes.addressof(w), lat.ctypes.data, steps,
                                        pcm.ctypes.data, pcm.size)
    assert n == g["pcm"].size
    np.testing.assert_array_equal(pcm[:n], g["pcm"])
