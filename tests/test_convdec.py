"""The 1-D convolutional waveform decoder (mt_convdec_* in include/mingcuda.h).

It has no counterpart in the reference (whose decoder is the windowed Qwen stack + ISTFT), so its
oracle (oracle/convdec.py, fp64) is pinned here to torch.nn.functional's conv1d /
conv_transpose1d in float64 instead: the CPU tests check the oracle's convolutions and the whole
decoder composition against torch; the GPU tests check the tensor-core decoder against the oracle.
Bar (north star): waveform cosine >= 0.999 for the same latents; here also max |error| <= 1e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import cosine

torch = pytest.importorskip("torch")


def _oracle():
    from oracle import convdec
    return convdec


def _torch_decode(cfg, W, latents):
    """The decoder with torch.nn.functional in float64 ([1, C, T] layout)."""
    F = torch.nn.functional
    t = {k: torch.from_numpy(np.asarray(v, np.float64)) for k, v in W.items()}
    K = cfg.kernel
    x = F.conv1d(torch.from_numpy(latents.T[None].astype(np.float64)), t["in_w"], t["in_b"], padding=(K - 1) // 2)
    for i in range(4):
        s = int(cfg.strides[i])
        u = F.conv_transpose1d(F.silu(x), t[f"up_w{i}"], t[f"up_b{i}"], stride=s, padding=s // 2)
        h = F.conv1d(F.silu(u), t[f"a_w{i}"], t[f"a_b{i}"], padding=(K - 1) // 2)
        x = u + F.conv1d(F.silu(h), t[f"b_w{i}"], t[f"b_b{i}"], padding=(K - 1) // 2)
    return torch.tanh(F.conv1d(F.silu(x), t["out_w"], t["out_b"], padding=(K - 1) // 2))[0, 0].numpy()


def _weights_f32(mt, cfg, seed):
    import oracle
    bits = mt.convdec_random_weights(cfg, seed)
    return bits, {k: oracle.bf16_to_f32(v.reshape(-1)).reshape(v.shape) for k, v in bits.items()}


@pytest.mark.parametrize("cin,cout,k", [(64, 128, 7), (96, 32, 3), (8, 8, 1)])
def test_oracle_conv1d_matches_torch(cin, cout, k):
    rs = np.random.default_rng(cin + k)
    x = rs.standard_normal((37, cin))
    w = rs.standard_normal((cout, cin, k))
    b = rs.standard_normal(cout)
    want = torch.nn.functional.conv1d(torch.from_numpy(x.T[None]), torch.from_numpy(w), torch.from_numpy(b),
                                      padding=(k - 1) // 2)[0].numpy().T
    np.testing.assert_allclose(_oracle().conv1d(x, w, b), want, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("stride", [2, 4, 8])
def test_oracle_conv_transpose1d_matches_torch(stride):
    rs = np.random.default_rng(stride)
    x = rs.standard_normal((11, 24))
    w = rs.standard_normal((24, 16, 2 * stride))
    b = rs.standard_normal(16)
    want = torch.nn.functional.conv_transpose1d(torch.from_numpy(x.T[None]), torch.from_numpy(w), torch.from_numpy(b),
                                                stride=stride, padding=stride // 2)[0].numpy().T
    got = _oracle().conv_transpose1d(x, w, b, stride)
    assert got.shape == (11 * stride, 16)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


def test_oracle_decoder_matches_torch(mt):
    cfg = mt.default_convdec_config()
    _, W = _weights_f32(mt, cfg, 4)
    latents = np.random.default_rng(3).standard_normal((2, cfg.latent_dim))
    got = _oracle().decode(cfg, W, latents)
    assert got.shape == (2 * 2048,)
    np.testing.assert_allclose(got, _torch_decode(cfg, W, latents), rtol=1e-9, atol=1e-9)
    assert 0.01 < np.abs(got).mean() < 0.99  # the random init keeps the signal off zero and off saturation


def test_oracle_weights_equal_library_init(mt):
    """The host restatement's init draws the same bf16 bits as mingtts_b200.convdec_random_weights."""
    cfg = mt.default_convdec_config()
    _, W = _weights_f32(mt, cfg, 4)
    Wo = _oracle().random_weights(_oracle().default_config(), 4)
    assert W.keys() == Wo.keys()
    for k in W:
        np.testing.assert_array_equal(W[k], Wo[k])


def test_convdec_samples_and_config_checks(mt):
    import ctypes
    cfg = mt.default_convdec_config()
    assert mt.lib().mt_convdec_samples(ctypes.byref(cfg), 216) == 216 * 2048
    assert mt.lib().mt_convdec_samples(None, 4) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("frames", [3, 8])
def test_convdec_matches_oracle(ctx, mt, frames):
    cfg = mt.default_convdec_config()
    bits, W = _weights_f32(mt, cfg, 4)
    dec = mt.ConvDecoder(ctx, bits, cfg, max_frames=16)
    latents = np.random.default_rng(frames).standard_normal((frames, cfg.latent_dim)).astype(np.float32)
    pcm = dec.decode(torch.from_numpy(latents).cuda()).cpu().numpy()
    ctx.check()
    want = _oracle().decode(cfg, W, latents)
    assert pcm.shape == want.shape
    assert np.abs(pcm - want).max() <= 1e-3 and cosine(pcm, want) >= 0.999
    dec.close()


@pytest.mark.gpu
def test_convdec_shorter_call_after_longer(ctx, mt):
    """Rows a longer call left behind must read as zero padding in a shorter one."""
    cfg = mt.default_convdec_config()
    bits, W = _weights_f32(mt, cfg, 5)
    dec = mt.ConvDecoder(ctx, bits, cfg, max_frames=12)
    rs = np.random.default_rng(7)
    long_lat = rs.standard_normal((12, cfg.latent_dim)).astype(np.float32)
    dec.decode(torch.from_numpy(long_lat).cuda())
    short = rs.standard_normal((5, cfg.latent_dim)).astype(np.float32)
    pcm = dec.decode(torch.from_numpy(short).cuda()).cpu().numpy()
    ctx.check()
    want = _oracle().decode(cfg, W, short)
    assert np.abs(pcm - want).max() <= 1e-3 and cosine(pcm, want) >= 0.999
    with pytest.raises(mt.MingError) as e:  # more frames than the decoder was created for
        dec.decode(torch.from_numpy(rs.standard_normal((13, cfg.latent_dim)).astype(np.float32)).cuda())
    assert e.value.status == mt.MT_ERR_CAPACITY
    dec.close()
