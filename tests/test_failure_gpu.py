"""Failure detection on the GPU without a fault: a bounded device wait that runs out.

The reference surfaces GPU failures as command-buffer errors at StepRecorder.finish
(Sources/MingTTS/Engine/Engine.swift:70-85, `gpuFailure`). Here every mbarrier wait of the kernels
is bounded by a wall-time limit; one that gives up records MT_ERR_TIMEOUT in the context's status
word, its kernel returns, and mt_ctx_check reports it. This test shortens the limit to 1 ms, runs
the library's probe kernel (a wait on a shared-memory barrier that nothing arrives on, with no copy
in flight), and checks that the timeout is reported once, is cleared by the check, and that the
context still computes correct results afterwards.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_recovers(ctx, mt, oracle):
    import torch
    ctx.set_wait_limit(1000)  # 1 ms
    try:
        ctx.wait_probe()
        with pytest.raises(mt.MingError) as e:
            ctx.check()
        assert e.value.status == mt.MT_ERR_TIMEOUT
        assert "site 90" in str(e.value)
        ctx.check()  # the check cleared the status word
    finally:
        ctx.set_wait_limit(0)
    # The context keeps working: a tensor-core linear (which itself uses bounded waits) against the oracle.
    m, n, k = 24, 256, 512
    rs = np.random.default_rng(90)
    x = rs.standard_normal((m, k)).astype(np.float32)
    w = oracle.bf16_bits(0.05 * rs.standard_normal((n, k)).astype(np.float32))
    b = oracle.bf16_bits(0.05 * rs.standard_normal(n).astype(np.float32))
    want = np.zeros((m, n), np.float32)
    oracle.linear(x, k, m, w, None, b, n, k, want, n, mt.BIAS | mt.GELU)
    xd, wd, bd = (torch.from_numpy(a).cuda() for a in (x, w, b))
    yd = torch.zeros(m, n, device="cuda")
    ctx.linear(xd, k, m, wd, None, bd, n, k, yd, n, mt.BIAS | mt.GELU)
    ctx.check()
    assert_close(yd.cpu().numpy(), want, atol=2e-4 * np.sqrt(k) / 30, rtol=1e-4, what="linear after a timeout")

