"""the whole 24-layer LLM decode step against the oracle, through mt_qwen_decode.

Qwen2-0.5B dimensions with random-init weights (seed 1), the KV cache of every layer pre-filled to
256 (and 500) of 512 positions with bf16-representable N(0,1) values, one new row per sequence:
M = 1 (the reference's decode, Engine.swift:381-385) and M = 2 (the config's CFG pair as two
sequences with their own caches), and 8 sequences (the most the small-batch path takes). Two steps
in a row, so the second attends to the row the first appended. Each case runs on both paths of
mt_qwen_decode: the persistent stack kernel (one launch per pass) and one launch per operation. The oracle restates QwenForward.dispatches (Qwen.swift:72-97) with fp64 dot products.
Bar: residual stream and final-norm rows within 1e-3 relative (max |err| / max |ref|), appended
cache rows within 1e-4.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def llm(ctx, mt):
    cfg = mt.default_config()
    model = mt.Model(ctx, cfg, seed=1, with_embeddings=False)
    host = model.arena_to_host()
    w_host, keep = mt.weights_struct(cfg, host.ctypes.data, model.tensors())
    w_dev = ctypes.cast(mt.lib().mt_model_get_weights(model.handle), ctypes.POINTER(mt.ModelWeights)).contents
    yield cfg, model, w_dev, w_host, (host, keep)
    model.close()


def prefilled_cache(oracle, cfg, cap, length, seed):
    c = cfg.llm
    cache = np.zeros((c.layers, 2, c.kv_heads, cap, 64), np.float32)
    vals = oracle.bf16_to_f32(oracle.randn_bf16(c.layers * 2 * c.kv_heads * length * 64, seed, 1.0))
    cache[:, :, :, :length, :] = vals.reshape(c.layers, 2, c.kv_heads, length, 64)
    return cache


@pytest.fixture(params=[2, 0], ids=["persistent", "per-op"])
def path(request, ctx):
    """Both implementations of mt_qwen_decode: the persistent stack kernel (required: an error if it
    cannot run) and one launch per op."""
    ctx.set_persistent(request.param)
    yield request.param
    ctx.set_persistent(0)


@pytest.mark.parametrize("requests,length", [(1, 256), (2, 256), (1, 500), (2, 500), (8, 300)])
def test_llm_decode_step_matches_oracle(ctx, mt, oracle, llm, path, requests, length):
    import torch
    cfg, model, w_dev, w_host, _ = llm
    if path == 2 and requests * 1 * cfg.llm.intermediate * 4 > 80 * 1024:
        pytest.skip("the persistent kernel stages at most 80 KB of a Qwen pass's input rows")
    c, H, cap = cfg.llm, cfg.llm.hidden, cfg.llm_capacity
    rs = np.random.default_rng(length + requests)
    caches = np.stack([prefilled_cache(oracle, cfg, cap, length, 100 + r) for r in range(requests)])
    kv = torch.from_numpy(caches.copy()).cuda()
    stride = caches[0].size
    pos = torch.tensor([length] * requests, dtype=torch.int32, device="cuda")
    want_cache = [np.ascontiguousarray(caches[r]) for r in range(requests)]
    for step in range(2):
        x0 = (0.5 * rs.standard_normal((requests, H))).astype(np.float32)
        x = torch.from_numpy(x0.copy()).cuda()
        z = torch.zeros(requests, H, device="cuda")
        ctx.call("qwen_decode", ctypes.byref(w_dev.llm), requests, 1, x, kv, stride, cap, pos, z)
        ctx.check()
        got_x, got_z = x.cpu().numpy(), z.cpu().numpy()
        for r in range(requests):
            xr = np.ascontiguousarray(x0[r:r + 1])
            zr = np.zeros((1, H), np.float32)
            # or_llm_decode advances the oracle's own copy of this request's cache in place
            assert oracle.lib().or_llm_decode(ctypes.addressof(w_host.llm), want_cache[r].ctypes.data, cap,
                                              length + step, xr.ctypes.data, 1, zr.ctypes.data) == 0
            what = f"config 2 M={requests} length {length} step {step} request {r}"
            assert rel_err(got_z[r], zr[0]) < 1e-3, f"{what}: final norm rel {rel_err(got_z[r], zr[0])}"
        pos += 1
    got_cache = kv.cpu().numpy().reshape(requests, c.layers, 2, c.kv_heads, cap, 64)
    for r in range(requests):
        want = want_cache[r].reshape(c.layers, 2, c.kv_heads, cap, 64)
        new = slice(length, length + 2)
        assert rel_err(got_cache[r][:, :, :, new], want[:, :, :, new]) < 1e-4, "appended cache rows"
        np.testing.assert_array_equal(got_cache[r][:, :, :, :length], want[:, :, :, :length])


def test_decode_rejects_bad_shapes(ctx, mt, llm):
    import torch
    cfg, model, w_dev, _, _ = llm
    H = cfg.llm.hidden
    x = torch.zeros(16, H, device="cuda")
    kv = torch.zeros(8, device="cuda")
    pos = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(mt.MingError) as e:  # more than 8 rows in all
        ctx.call("qwen_decode", ctypes.byref(w_dev.llm), 9, 1, x, kv, 10 ** 9, 512, pos, x)
    assert e.value.status == mt.MT_ERR_SHAPE
    with pytest.raises(mt.MingError) as e:  # request stride smaller than one cache
        ctx.call("qwen_decode", ctypes.byref(w_dev.llm), 1, 1, x, kv, 8, 512, pos, x)
    assert e.value.status == mt.MT_ERR_CAPACITY


def test_vae_style_decode_matches_oracle(ctx, mt, oracle, path):
    """Four rows per sequence over a 65-key window in a 128-slot ring (the VAE decoder's shape,
    VAEDecoder.swift:86-107), reduced dimensions, two sequences, positions past the ring's wrap."""
    import torch
    cfg = mt.small_config()
    model = mt.Model(ctx, cfg, seed=4, with_embeddings=False)
    host = model.arena_to_host()
    w_host, keep = mt.weights_struct(cfg, host.ctypes.data, model.tensors())
    w_dev = ctypes.cast(mt.lib().mt_model_get_weights(model.handle), ctypes.POINTER(mt.ModelWeights)).contents
    c, H, cap, S, R = cfg.vae, cfg.vae.hidden, 128, 4, 2
    rs = np.random.default_rng(4)
    # the oracle keeps every position; the device cache is a ring of `cap` slots
    full = [np.zeros((c.layers, 2, c.kv_heads, 512, 64), np.float32) for _ in range(R)]
    ring = torch.zeros(R * c.layers * 2 * c.kv_heads * cap * 64, device="cuda")
    stride = c.layers * 2 * c.kv_heads * cap * 64
    pos = torch.zeros(R, dtype=torch.int32, device="cuda")
    for step in range(40):  # 160 positions: the ring wraps after 128
        x0 = (0.5 * rs.standard_normal((R * S, H))).astype(np.float32)
        x = torch.from_numpy(x0.copy()).cuda()
        z = torch.zeros(R * S, H, device="cuda")
        ctx.call("qwen_decode", ctypes.byref(w_dev.vae), R, S, x, ring, stride, cap, pos, z)
        ctx.check()
        got = z.cpu().numpy()
        for r in range(R):
            zr = np.zeros((S, H), np.float32)
            xr = np.ascontiguousarray(x0[r * S:(r + 1) * S])
            assert oracle.lib().or_llm_decode(ctypes.addressof(w_host.vae), full[r].ctypes.data, 512, 4 * step,
                                              xr.ctypes.data, S, zr.ctypes.data) == 0
            assert rel_err(got[r * S:(r + 1) * S], zr) < 1e-3, f"step {step} sequence {r}"
        pos += S
    model.close()
