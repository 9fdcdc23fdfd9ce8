"""The C ABI without a GPU: the library loads, exports every function include/*.h declares, and its
host-only logic (routing, argument checks, the host generators) behaves. No compute call here."""
from __future__ import annotations

import ctypes
import glob
import os
import re

import numpy as np

from conftest import ROOT


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(mt_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_every_declared_symbol_is_exported(mt):
    lib = mt.lib()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_prototypes_cover_the_header(mt):
    missing = [n for n in declared_functions() if n not in mt.PROTOTYPES]
    assert not missing, f"no ctypes prototype for {missing}"


def test_version(mt):
    assert "sm_100a" in mt.version()


def test_linear_route(mt):
    lib = mt.lib()
    # Decode rows stay on CUDA cores, batched rows go to the tensor cores (Kernels.usesGemm analogue).
    assert lib.mt_linear_route(1, 1152, 896) == 0
    assert lib.mt_linear_route(8, 896, 4864) == 0
    assert lib.mt_linear_route(9, 896, 4864) == 1
    assert lib.mt_linear_route(174, 1152, 896) == 1


def test_null_context_is_an_error_not_a_crash(mt):
    lib = mt.lib()
    assert lib.mt_linear(None, None, None, 896, 1, None, None, None, 8, 896, None, 8, 0) == mt.MT_ERR_ARG
    assert lib.mt_rmsnorm(None, None, None, 896, 1, 896, None, None, 896, 1e-6) == mt.MT_ERR_ARG
    assert lib.mt_attention(None, None, None, 1152, 1, 14, 2, 0, 0, None, None, 512, None, 896) == mt.MT_ERR_ARG
    assert lib.mt_last_error(None) == b"no context"


def test_host_generators_match_oracle(mt, oracle):
    lib = mt.lib()
    out = np.empty(1001, np.float32)
    lib.mt_gaussian_noise_host(out.ctypes.data, out.size, 42)
    np.testing.assert_array_equal(out, oracle.gaussian_noise(1001, 42))
    bits = np.empty(100_001, np.uint16)
    lib.mt_randn_bf16_host(bits.ctypes.data, bits.size, 7, ctypes.c_float(0.02))
    np.testing.assert_array_equal(bits, oracle.randn_bf16(100_001, 7, 0.02))
