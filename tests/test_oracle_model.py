"""The oracle's host model (oracle/model.py) against the product's model table, on CPU.

bench.py's CPU legs build the weights with oracle.model so that they load liboracle.so only; these
tests pin that restatement to libmingcuda.so's mt_model_tensors (host code, no GPU): the same names,
sizes, dtypes, init kinds and per-tensor seeds in the same order, the same default dimensions, and
struct mirrors with the same layout as the package's.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest


@pytest.fixture(scope="module")
def om():
    import oracle.model as m
    return m


def as_oracle_config(om, cfg):
    return om.ModelConfig.from_buffer_copy(cfg)


@pytest.mark.parametrize("which", ["default", "small"])
def test_tensor_list_matches_product_table(mt, om, which):
    cfg = mt.default_config() if which == "default" else mt.small_config()
    want = mt.tensor_table(cfg, seed=7)
    got = om.tensor_list(as_oracle_config(om, cfg))
    assert len(got) == len(want)
    for i, ((name, numel, dtype, init), t) in enumerate(zip(got, want)):
        assert name == t.name.decode() and numel == t.numel and dtype == t.dtype and init == t.init, name
        assert om.tensor_seed(7, i) == t.seed, name


def test_default_config_matches_product(mt, om):
    a, b = om.default_config(), mt.default_config()
    assert ctypes.sizeof(a) == ctypes.sizeof(b)
    assert bytes(a) == bytes(b)


@pytest.mark.parametrize("pair", ["QwenConfig", "QwenLayer", "QwenWeights", "DitConfig", "DitBlock", "DitWeights",
                                  "ModelConfig", "ModelWeights"])
def test_struct_mirrors_have_the_same_layout(mt, om, pair):
    a, b = getattr(om, pair), getattr(mt, pair)
    assert ctypes.sizeof(a) == ctypes.sizeof(b)
    assert [f[0] for f in a._fields_] == [f[0] for f in b._fields_]
    for (name, _), _ in zip(a._fields_, b._fields_):
        assert getattr(a, name).offset == getattr(b, name).offset, name


def test_host_model_values_match_product_generators(mt, om, oracle):
    """A few tensors filled by the oracle's host model equal the product's host generator draws."""
    cfg = mt.small_config()
    hm = om.HostModel(as_oracle_config(om, cfg), seed=3, with_embeddings=False)
    table = {t.name.decode(): t for t in mt.tensor_table(cfg, seed=3, with_embeddings=False)}
    for name in ("model.model.layers.0.self_attn.qkv_proj.weight", "stop_head.bias",
                 "flowloss.cfm.model.blocks.1.mlp.ff.2.weight"):
        t = table[name]
        ref = np.empty(t.numel, np.uint16)
        mt.lib().mt_randn_bf16_host(ref.ctypes.data, t.numel, t.seed, t.std)
        np.testing.assert_array_equal(hm.arrays[name], ref, err_msg=name)
    assert np.all(hm.arrays["model.model.layers.1.input_layernorm.weight"] == 0x3F80)
    cls = hm.arrays["linear_proj_audio.word_embedder.weight"]
    assert cls.dtype == np.float32 and np.all(oracle.bf16_to_f32(oracle.bf16_bits(cls)) == cls)
