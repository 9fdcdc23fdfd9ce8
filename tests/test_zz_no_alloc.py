"""mt_linear_static -- the linear for callers that cannot allocate device memory.

Hosts that cannot call cudaMalloc (a framework that owns all device memory through its own pool, a
real-time audio thread that must not block on an allocation) get one entry point that needs no
context and uses a scratch array compiled into the library.
This file checks it against the allocating entry point (mt_linear) through the C ABI, on two calls
in a row (the second reuses the array the first left behind), and checks the size limit. It is
named so that pytest collects it last; it also passes on its own in a fresh process.
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


def case(rs, oracle, m, n, k):
    x = rs.standard_normal((m, k)).astype(np.float32)
    w = oracle.bf16_bits(0.05 * rs.standard_normal((n, k)).astype(np.float32))
    w2 = oracle.bf16_bits(0.05 * rs.standard_normal((n, k)).astype(np.float32))
    b = oracle.bf16_bits(0.05 * rs.standard_normal(n).astype(np.float32))
    y0 = rs.standard_normal((m, n)).astype(np.float32)
    return x, w, w2, b, y0


@pytest.mark.parametrize("m,n,k,flags", [
    (64, 896, 4864, 2),    # accumulate (LLM down projection shape)
    (384, 1024, 1024, 5),  # bias + GELU (flow DiT rows)
    (9, 200, 136, 8),      # SiLU gate, ragged tiles
    (3, 64, 1024, 17),     # few rows: the static entry stays on the tensor cores
])
def test_static_linear_matches_linear_twice(ctx, mt, oracle, m, n, k, flags):
    import torch
    lib = mt.lib()
    rs = np.random.default_rng(m * 7 + n)
    gated = bool(flags & mt.SILU_GATE)
    for call in range(2):
        x, w, w2, b, y0 = case(rs, oracle, m, n, k)
        xd, wd, w2d, bd = dev(x), dev(w), dev(w2), dev(b)
        want = dev(y0)
        ctx.linear(xd, k, m, wd, w2d if gated else None, bd, n, k, want, n, flags)
        got = dev(y0)
        st = lib.mt_linear_static(mt.current_stream(), xd.data_ptr(), k, m, wd.data_ptr(),
                                  w2d.data_ptr() if gated else None, bd.data_ptr(), n, k, got.data_ptr(), n, flags)
        assert st == mt.MT_OK, f"mt_linear_static returned {st}"
        torch.cuda.synchronize()
        g, ref = got.cpu().numpy(), want.cpu().numpy()
        what = f"static linear m{m} n{n} k{k} flags {flags} call {call}"
        assert_close(g, ref, atol=2e-4 * np.sqrt(k) / 30, rtol=1e-4, what=what)
        assert rel_err(g, ref) <= 1e-3, what


def test_static_linear_rejects_sizes_beyond_the_array(ctx, mt):
    import torch
    lib = mt.lib()
    k = 1024
    m = MAX_ACTIVATIONS // k + 1
    x = torch.zeros(m, k, device="cuda")
    w = torch.zeros(64, k, dtype=torch.int16, device="cuda")
    y = torch.zeros(m, 64, device="cuda")
    st = lib.mt_linear_static(mt.current_stream(), x.data_ptr(), k, m, w.data_ptr(), None, None, 64, k,
                              y.data_ptr(), 64, 0)
    assert st == mt.MT_ERR_CAPACITY
    # The largest size that fits is accepted.
    m_ok = MAX_ACTIVATIONS // k
    st = lib.mt_linear_static(mt.current_stream(), x.data_ptr(), k, m_ok, w.data_ptr(), None, None, 64, k,
                              y.data_ptr(), 64, 0)
    assert st == mt.MT_OK
    torch.cuda.synchronize()
