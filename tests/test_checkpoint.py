"""Safetensors checkpoint loading (mt_checkpoint_fill_arena / mt_model_load_safetensors).

The reference reads checkpoint tensors by name (SafeTensors.swift:7-87) and packs each module's
bf16 tensors, concatenating q/k/v along their first axis and checking element counts
(WeightArena, Weights.swift:32-62, names :116-263). These tests write checkpoints with the
reference's tensor names (q/k/v separate) for the reduced test configuration and check the
arena the loader builds byte for byte, then each failure the reference reports.
"""
from __future__ import annotations

import numpy as np
import pytest

import safetensors_io as sio


def qkv_parts(name: str, numel: int, cfg):
    """The checkpoint tensors a table entry is gathered from, with their element counts."""
    if ".self_attn.qkv_proj." in name:
        qc = cfg.vae if name.startswith("audio.") else cfg.llm
        unit = numel // (qc.heads + 2 * qc.kv_heads)
        return [(name.replace(".qkv_proj.", f".{p}_proj."), unit * c)
                for p, c in (("q", qc.heads), ("k", qc.kv_heads), ("v", qc.kv_heads))]
    if ".attn.to_qkv." in name:
        return [(name.replace(".to_qkv.", f".to_{p}."), numel // 3) for p in "qkv"]
    return [(name, numel)]


def build_checkpoint(mt, cfg, seed=0, with_embeddings=True, f32_as_bf16=("linear_proj_audio.word_embedder.weight",)):
    """(tensors for the file, expected host arena)."""
    rng = np.random.default_rng(seed)
    table = mt.tensor_table(cfg, 0, with_embeddings)
    arena = np.zeros(mt.lib().mt_model_arena_bytes(mt.ctypes.byref(cfg), int(with_embeddings)), np.uint8)
    tensors = {}
    for t in table:
        name = t.name.decode()
        if t.dtype == mt.MT_DTYPE_BF16:
            parts = []
            for src, n in qkv_parts(name, t.numel, cfg):
                bits = sio.bf16_bits(rng, n)
                tensors[src] = ("BF16", [n], bits.tobytes())
                parts.append(bits)
            raw = np.concatenate(parts).view(np.uint8)
            arena[t.offset:t.offset + raw.size] = raw
        else:
            vals = (rng.standard_normal(t.numel) * 0.5).astype(np.float32)
            if name in f32_as_bf16:
                bits = (vals.view(np.uint32) >> 16).astype(np.uint16)
                tensors[name] = ("BF16", [t.numel], bits.tobytes())
                vals = (bits.astype(np.uint32) << 16).view(np.float32)
            else:
                tensors[name] = ("F32", [t.numel], vals.tobytes())
            raw = vals.view(np.uint8)
            arena[t.offset:t.offset + raw.size] = raw
    # a tensor the per-step path does not use (the VAE encoder's) is ignored
    tensors["audio.encoder.fc1.weight"] = ("BF16", [4, 8], sio.bf16_bits(rng, 32).tobytes())
    return tensors, arena


def build_encoder_checkpoint(mt, cfg, seed=0):
    """(tensors for the file, expected host encoder arena): fc1 stored [hidden, frame] as in the
    checkpoint, the arena holding it [hidden, padded_frame] with zero columns."""
    rng = np.random.default_rng(seed)
    table = mt.encoder_tensor_table(cfg, 0)
    arena = np.zeros(mt.lib().mt_encoder_arena_bytes(mt.ctypes.byref(cfg)), np.uint8)
    tensors = {}
    h, frame, padded = cfg.vae.hidden, cfg.hop, (cfg.hop + 63) // 64 * 64
    for t in table:
        name = t.name.decode()
        if name == "audio.encoder.fc1.weight":
            bits = sio.bf16_bits(rng, h * frame).reshape(h, frame)
            tensors[name] = ("BF16", [h, frame], bits.tobytes())
            full = np.zeros((h, padded), np.uint16)
            full[:, :frame] = bits
            raw = full.view(np.uint8).ravel()
            arena[t.offset:t.offset + raw.size] = raw
        elif t.dtype == mt.MT_DTYPE_BF16:
            parts = []
            for src, n in qkv_parts(name, t.numel, cfg):
                bits = sio.bf16_bits(rng, n)
                tensors[src] = ("BF16", [n], bits.tobytes())
                parts.append(bits)
            raw = np.concatenate(parts).view(np.uint8)
            arena[t.offset:t.offset + raw.size] = raw
        else:
            vals = (rng.standard_normal(t.numel) * 0.5).astype(np.float32)
            tensors[name] = ("F32", [t.numel], vals.tobytes())
            raw = vals.view(np.uint8)
            arena[t.offset:t.offset + raw.size] = raw
    return tensors, arena


@pytest.fixture(scope="module")
def small(mt):
    return mt.small_config()


def test_fill_arena_matches_reference_packing(mt, small, tmp_path):
    tensors, want = build_checkpoint(mt, small)
    path = tmp_path / "model.safetensors"
    sio.write(path, tensors, metadata={"format": "pt"})
    got = mt.checkpoint_fill_arena(path, small, with_embeddings=True)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


def test_fill_arena_without_embeddings(mt, small, tmp_path):
    """The embedding table is the table's last tensor: without it the arena is the same bytes minus
    that tail, whether or not the file holds the table."""
    tensors, want_full = build_checkpoint(mt, small, seed=3, with_embeddings=True)
    path = tmp_path / "model.safetensors"
    sio.write(path, tensors)
    got = mt.checkpoint_fill_arena(path, small, with_embeddings=False)
    assert got.size == mt.lib().mt_model_arena_bytes(mt.ctypes.byref(small), 0) < want_full.size
    assert np.array_equal(got, want_full[:got.size])


def _expect_error(mt, small, path, fragment):
    with pytest.raises(mt.CheckpointError) as e:
        mt.checkpoint_fill_arena(path, small, with_embeddings=True)
    assert e.value.status == mt.MT_ERR_CHECKPOINT
    assert fragment in str(e.value), str(e.value)


def test_missing_tensor(mt, small, tmp_path):
    tensors, _ = build_checkpoint(mt, small)
    del tensors["stop_head.bias"]
    sio.write(tmp_path / "m.safetensors", tensors)
    _expect_error(mt, small, tmp_path / "m.safetensors", "missing tensor stop_head.bias")


def test_missing_qkv_part(mt, small, tmp_path):
    tensors, _ = build_checkpoint(mt, small)
    del tensors["model.model.layers.1.self_attn.k_proj.weight"]
    sio.write(tmp_path / "m.safetensors", tensors)
    _expect_error(mt, small, tmp_path / "m.safetensors", "missing tensor model.model.layers.1.self_attn.k_proj.weight")


def test_wrong_dtype(mt, small, tmp_path):
    tensors, _ = build_checkpoint(mt, small)
    _, shape, raw = tensors["stop_head.weight"]
    n = len(raw) // 2
    tensors["stop_head.weight"] = ("F32", [n], np.zeros(n, np.float32).tobytes())
    sio.write(tmp_path / "m.safetensors", tensors)
    _expect_error(mt, small, tmp_path / "m.safetensors", "stop_head.weight is F32, expected BF16")


def test_wrong_element_count(mt, small, tmp_path):
    tensors, _ = build_checkpoint(mt, small)
    _, shape, raw = tensors["stop_head.weight"]
    tensors["stop_head.weight"] = ("BF16", [len(raw) // 2 - 2], raw[:-4])
    sio.write(tmp_path / "m.safetensors", tensors)
    _expect_error(mt, small, tmp_path / "m.safetensors", "stop_head.weight has")


def test_truncated_file(mt, small, tmp_path):
    tensors, _ = build_checkpoint(mt, small)
    blob = sio.encode(tensors)
    (tmp_path / "m.safetensors").write_bytes(blob[:-100])
    _expect_error(mt, small, tmp_path / "m.safetensors", "download incomplete?")


def _blob(header: bytes) -> bytes:
    return len(header).to_bytes(8, "little") + header


@pytest.mark.parametrize("blob,fragment", [
    (b"\x01\x02\x03", "file too small"),
    ((10**6).to_bytes(8, "little") + b"{}", "exceeds file"),
    (_blob(b"[1,2]"), "header is not a JSON object"),
    (_blob(b'{"a": {"dtype": 1}}'), "malformed entry a"),
    (_blob(b'{"a": {"dtype": "BF16", "shape": [2], "data_offsets": [4, 0]}}'), "malformed entry a"),
    (_blob(b'{"a": {"dtype": "BF16", "shape"'), "header is not a JSON object"),
])
def test_malformed_files(mt, small, tmp_path, blob, fragment):
    (tmp_path / "m.safetensors").write_bytes(blob)
    _expect_error(mt, small, tmp_path / "m.safetensors", fragment)


def test_unreadable_path(mt, small, tmp_path):
    _expect_error(mt, small, tmp_path / "absent.safetensors", "cannot open")


def test_json_escapes_in_names(mt, small, tmp_path):
    """Tensor names are JSON strings: escaped characters in an unrelated name do not disturb parsing."""
    tensors, want = build_checkpoint(mt, small)
    tensors['odd "name" \\ é'] = ("BF16", [2], b"\x00\x00\x00\x00")
    sio.write(tmp_path / "m.safetensors", tensors, metadata={"note": "tab\there"})
    assert np.array_equal(mt.checkpoint_fill_arena(tmp_path / "m.safetensors", small, True), want)


@pytest.mark.gpu
def test_model_load_safetensors_device_arena(mt, ctx, small, tmp_path):
    tensors, want = build_checkpoint(mt, small, seed=7)
    path = tmp_path / "model.safetensors"
    sio.write(path, tensors)
    model = mt.Model.load(ctx, path, small, with_embeddings=True)
    try:
        got = model.arena_to_host()
        assert np.array_equal(got, want)
    finally:
        model.close()
    with pytest.raises(mt.CheckpointError):
        mt.Model.load(ctx, tmp_path / "absent.safetensors", small)


def test_encoder_fill_arena_pads_fc1(mt, small, tmp_path):
    for cfg in (small, mt.default_config()):
        if cfg is not small:  # the full encoder table only: names, offsets and fc1 padding of 882 -> 896
            t = {x.name.decode(): x for x in mt.encoder_tensor_table(cfg, 0)}
            assert t["audio.encoder.fc1.weight"].numel == 896 * 896
            assert t["audio.encoder.fc3.weight"].numel == 128 * 896
            assert "audio.encoder.aggregator.layers.3.mlp.down_proj.weight" in t
            assert "audio.encoder.aggregator.layers.4.mlp.down_proj.weight" not in t
            assert "audio.encoder.encoder.layers.23.self_attn.qkv_proj.bias" in t
            continue
        tensors, want = build_encoder_checkpoint(mt, cfg, seed=4)
        sio.write(tmp_path / "m.safetensors", tensors)
        got = mt.checkpoint_fill_encoder_arena(tmp_path / "m.safetensors", cfg)
        assert np.array_equal(got, want)


def test_encoder_fc1_shape_is_checked(mt, small, tmp_path):
    tensors, _ = build_encoder_checkpoint(mt, small, seed=4)
    _, shape, raw = tensors["audio.encoder.fc1.weight"]
    tensors["audio.encoder.fc1.weight"] = ("BF16", [shape[1], shape[0]], raw)
    sio.write(tmp_path / "m.safetensors", tensors)
    with pytest.raises(mt.CheckpointError) as e:
        mt.checkpoint_fill_encoder_arena(tmp_path / "m.safetensors", small)
    assert "audio.encoder.fc1.weight is BF16" in str(e.value)
