"""Multi-rank host logic of bench.py on CPU: two gloo ranks (the GPU run uses one NCCL rank per GPU
with the same helpers). Checks the max-over-ranks timing reduction, the barrier, and that the
replicas draw disjoint, reproducible request inputs."""
from __future__ import annotations

import datetime
import importlib.util
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _load_bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        bench = _load_bench()
        mt = bench.load_package()
        cfg = mt.small_config()
        t = bench.dist_max(float(rank + 1) * 0.5, world, device="cpu")
        bench.barrier(world, device="cpu")
        first, count = bench.rank_requests(rank, 3)
        ids, noise = bench.request_inputs(bench.product_noise(mt), cfg.vocab, cfg.latent_dim, count, 4, 2, first)
        # config 5's strong-scaling partition: 64 requests in all, 32 per rank
        strong_first, strong_count = bench.rank_requests(rank, 64 // world)
        out[rank] = (t, first, ids, noise, strong_first, strong_count)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks():
    import torch.multiprocessing as mp
    world = 2
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, join=True, start_method="spawn")
    assert sorted(out.keys()) == [0, 1]
    for r in range(world):
        assert out[r][0] == pytest.approx(1.0)  # max over ranks of 0.5 and 1.0
    assert out[0][1] == 0 and out[1][1] == 3
    assert [(out[r][4], out[r][5]) for r in range(world)] == [(0, 32), (32, 32)]
    assert not np.array_equal(out[0][2], out[1][2])
    assert not np.array_equal(out[0][3], out[1][3])
    # Reproducible: rank 1's inputs are the global requests 3..5 drawn in one process.
    bench = _load_bench()
    mt = bench.load_package()
    cfg = mt.small_config()
    ids, noise = bench.request_inputs(bench.product_noise(mt), cfg.vocab, cfg.latent_dim, 6, 4, 2, 0)
    np.testing.assert_array_equal(out[1][2], ids[3:])
    np.testing.assert_array_equal(out[1][3], noise[3:])
