"""mt_linear_static -- the linear for callers that cannot allocate device memory.

Hosts that cannot call cudaMalloc (a framework that owns all device memory through its own pool, a
real-time audio thread that must not block on an allocation) get one entry point that needs no
context and uses a scratch array compiled into the library.
This file checks it through the C ABI against the CPU oracle (fp64 dot products, the reference's
epilogue order) and against the allocating entry point (mt_linear), on two calls in a row (the
second reuses the array the first left behind), with strided activations and outputs, at the size
limit, and checks that its device status word stays clear. It is named so that pytest collects it
last; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close, rel_err

pytestmark = pytest.mark.gpu

MAX_ACTIVATIONS = 1 << 20  # m * k limit of the static scratch array


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def case(rs, oracle, m, n, k, ldx, ldy):
    x = np.zeros((m, ldx), np.float32)
    x[:, :k] = rs.standard_normal((m, k))
    x[:, k:] = np.nan  # columns past k must never be read
    w = oracle.bf16_bits(0.05 * rs.standard_normal((n, k)).astype(np.float32))
    w2 = oracle.bf16_bits(0.05 * rs.standard_normal((n, k)).astype(np.float32))
    b = oracle.bf16_bits(0.05 * rs.standard_normal(n).astype(np.float32))
    y0 = rs.standard_normal((m, ldy)).astype(np.float32)
    return x, w, w2, b, y0


def check(got, want, k, ldy, n, what):
    assert_close(got[:, :n], want[:, :n], atol=2e-4 * np.sqrt(k) / 30, rtol=1e-4, what=what)
    assert rel_err(got[:, :n], want[:, :n]) <= 1e-3, what
    if ldy > n:  # columns past n are left as they were
        np.testing.assert_array_equal(got[:, n:], want[:, n:], err_msg=what)


@pytest.mark.parametrize("m,n,k,flags,ldx_pad,ldy_pad", [
    (64, 896, 4864, 2, 0, 0),    # accumulate (LLM down projection shape)
    (384, 1024, 1024, 5, 0, 0),  # bias + GELU (flow DiT rows)
    (9, 200, 136, 8, 0, 0),      # SiLU gate, ragged tiles
    (3, 64, 1024, 17, 0, 0),     # few rows: the static entry stays on the tensor cores
    (40, 320, 512, 3, 4, 12),    # strided x (ldx = k + 4) and y (ldy = n + 12), bias + accumulate
    (17, 128, 256, 8, 8, 4),     # strided, SiLU gate
])
def test_static_linear_matches_oracle_twice(ctx, mt, oracle, m, n, k, flags, ldx_pad, ldy_pad):
    import torch
    lib = mt.lib()
    rs = np.random.default_rng(m * 7 + n)
    gated = bool(flags & mt.SILU_GATE)
    ldx, ldy = k + ldx_pad, n + ldy_pad
    for call in range(2):
        x, w, w2, b, y0 = case(rs, oracle, m, n, k, ldx, ldy)
        want = y0.copy()
        oracle.linear(x, ldx, m, w, w2 if gated else None, b, n, k, want, ldy, flags)
        xd, wd, w2d, bd = dev(x), dev(w), dev(w2), dev(b)
        alloc = dev(y0)
        ctx.linear(xd, ldx, m, wd, w2d if gated else None, bd, n, k, alloc, ldy, flags)
        got = dev(y0)
        st = lib.mt_linear_static(mt.current_stream(), xd.data_ptr(), ldx, m, wd.data_ptr(),
                                  w2d.data_ptr() if gated else None, bd.data_ptr(), n, k, got.data_ptr(), ldy, flags)
        assert st == mt.MT_OK, f"mt_linear_static returned {st}"
        assert lib.mt_linear_static_status(mt.current_stream()) == mt.MT_OK
        torch.cuda.synchronize()
        g = got.cpu().numpy()
        what = f"static linear m{m} n{n} k{k} ldx {ldx} ldy {ldy} flags {flags} call {call}"
        check(g, want, k, ldy, n, what + " vs oracle")
        check(g, alloc.cpu().numpy(), k, ldy, n, what + " vs mt_linear")


def test_static_linear_size_limit(ctx, mt, oracle):
    import torch
    lib = mt.lib()
    k, n = 1024, 64
    m = MAX_ACTIVATIONS // k + 1
    rs = np.random.default_rng(5)
    x = rs.standard_normal((m, k)).astype(np.float32)
    w = oracle.bf16_bits(0.05 * rs.standard_normal((n, k)).astype(np.float32))
    xd, wd = dev(x), dev(w)
    y = torch.zeros(m, n, device="cuda")
    st = lib.mt_linear_static(mt.current_stream(), xd.data_ptr(), k, m, wd.data_ptr(), None, None, n, k,
                              y.data_ptr(), n, 0)
    assert st == mt.MT_ERR_CAPACITY
    # The largest size that fits is accepted and computed in full.
    m_ok = MAX_ACTIVATIONS // k
    st = lib.mt_linear_static(mt.current_stream(), xd.data_ptr(), k, m_ok, wd.data_ptr(), None, None, n, k,
                              y.data_ptr(), n, 0)
    assert st == mt.MT_OK
    assert lib.mt_linear_static_status(mt.current_stream()) == mt.MT_OK
    want = np.zeros((m_ok, n), np.float32)
    oracle.linear(np.ascontiguousarray(x[:m_ok]), k, m_ok, w, None, None, n, k, want, n, 0)
    got = y.cpu().numpy()
    check(got[:m_ok], want, k, n, n, "static linear at the size limit")
    assert np.all(got[m_ok:] == 0)  # the row past the limit was not written
