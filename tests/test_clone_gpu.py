"""Clone path on the GPU against the CPU oracle: the audio VAE encoder (VAEEncoder.encode,
VAEEncoder.swift:56-107) and the aggregator over reference latents (MingEngine.aggregate,
Engine.swift:236-256), both composed from the operator entry points.

Bar: the posterior mean and std, and the aggregated LLM rows, within 1e-3 of the oracle
(max |err| / max |ref|), on the same weights (host copies of the device arenas).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def oracle_encode(oracle, mt, cfg, enc, samples):
    host = enc.arena_to_host()
    w, keep = mt.encoder_weights_struct(cfg, host.ctypes.data, enc.tensors())
    latents = samples.size // (4 * cfg.hop)
    mean = np.zeros((latents, cfg.latent_dim), np.float32)
    std = np.zeros_like(mean)
    assert oracle.lib().or_vae_encode(ctypes.addressof(cfg), ctypes.addressof(w), samples.ctypes.data, samples.size,
                                      mean.ctypes.data, std.ctypes.data) == 0
    return mean, std


def oracle_aggregate(oracle, mt, cfg, model, latents):
    host = model.arena_to_host()
    w, keep = mt.weights_struct(cfg, host.ctypes.data, model.tensors())
    rows = np.zeros((latents.shape[0], cfg.llm.hidden), np.float32)
    assert oracle.lib().or_aggregate_latents(ctypes.addressof(cfg), ctypes.addressof(w), latents.ctypes.data,
                                             latents.shape[0], rows.ctypes.data) == 0
    return rows


@pytest.mark.parametrize("full,latents", [(False, 6), (False, 1), (True, 4)])
def test_vae_encode_matches_oracle(ctx, mt, oracle, full, latents):
    cfg = mt.default_config() if full else mt.small_config()
    enc = mt.Encoder(ctx, cfg, seed=11)
    rng = np.random.default_rng(latents + 17 * full)
    samples = (0.3 * rng.standard_normal(4 * cfg.hop * latents)).astype(np.float32)
    mean, std = enc.encode(samples)
    want_mean, want_std = oracle_encode(oracle, mt, cfg, enc, samples)
    assert mean.shape == (latents, cfg.latent_dim)
    assert np.all(std > 0)
    assert rel_err(mean, want_mean) <= 1e-3, rel_err(mean, want_mean)
    assert rel_err(std, want_std) <= 1e-3, rel_err(std, want_std)
    enc.close()


def test_vae_encode_rejects_partial_patches(ctx, mt):
    cfg = mt.small_config()
    enc = mt.Encoder(ctx, cfg, seed=1)
    with pytest.raises(mt.MingError) as e:
        enc.encode(np.zeros(4 * cfg.hop + 3, np.float32))
    assert e.value.status == mt.MT_ERR_SHAPE
    with pytest.raises(mt.MingError) as e:
        enc.encode(np.zeros(4 * cfg.hop * 401, np.float32))  # 1604 frames > 1600
    assert e.value.status == mt.MT_ERR_CAPACITY
    enc.close()


@pytest.mark.parametrize("full,count", [(False, 7), (True, 5)])
def test_aggregate_latents_matches_oracle(ctx, mt, oracle, full, count):
    cfg = mt.default_config() if full else mt.small_config()
    model = mt.Model(ctx, cfg, seed=12, with_embeddings=False)
    latents = np.random.default_rng(count).standard_normal((count, cfg.latent_dim)).astype(np.float32)
    rows = mt.aggregate_latents(ctx, model, latents)
    want = oracle_aggregate(oracle, mt, cfg, model, latents)
    assert rows.shape == (count, cfg.llm.hidden)
    assert rel_err(rows, want) <= 1e-3, rel_err(rows, want)
    model.close()


def test_encoder_load_safetensors_device_arena(ctx, mt, tmp_path):
    from test_checkpoint import build_encoder_checkpoint
    import safetensors_io as sio
    cfg = mt.small_config()
    tensors, want = build_encoder_checkpoint(mt, cfg, seed=5)
    sio.write(tmp_path / "model.safetensors", tensors)
    enc = mt.Encoder.load(ctx, tmp_path / "model.safetensors", cfg)
    assert np.array_equal(enc.arena_to_host(), want)
    enc.close()
