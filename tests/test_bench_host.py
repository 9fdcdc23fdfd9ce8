"""Host-side contract of bench.py on CPU (no GPU): the reference arm's JSON line, its rank handling
under torchrun, and the time-to-first-audio helper's timing rule."""
from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _load_bench():
    spec = importlib.util.spec_from_file_location("bench_host_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _run_bench(args, env_extra=None, timeout=600):
    env = dict(os.environ, **(env_extra or {}))
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          env=env, timeout=timeout, cwd=ROOT)


def test_reference_arm_line():
    """`--impl reference` times the CPU oracle of the full model and prints one JSON line with the
    arm's keys; its value, cpu_baseline and e2e agree, with no host-device bytes."""
    r = _run_bench(["--impl", "reference", "--steps", "1", "--warmup", "3", "--prompt", "8"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "audio-s/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    cb, e2e = d["cpu_baseline"], d["e2e"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == e2e["value"] == d["value"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"]


def test_reference_arm_loads_only_the_oracle():
    """The reference arm times the oracle without the product library: after a run, the process has
    mapped liboracle.so and not libmingcuda.so, and has not imported the product package."""
    code = ("import sys, json; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3', "
            "'--prompt', '4']; sys.path.insert(0, '.'); import bench; bench.main(); "
            "maps = open('/proc/self/maps').read(); "
            "print(json.dumps({'oracle': 'liboracle.so' in maps, 'product': 'libmingcuda' in maps, "
            "'package': 'mingtts_b200' in sys.modules}))")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d == {"oracle": True, "product": False, "package": False}


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun only rank 0 runs the CPU arm; the other ranks print nothing and exit 0."""
    r = _run_bench(["--impl", "reference", "--steps", "1", "--warmup", "3"],
                   {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


class _FakeEngine:
    """Stands in for Engine.generate_stream: the first chunk after `first_s`, a later one after more."""

    def __init__(self, first_s):
        self.first_s, self.calls = first_s, 0

    def generate_stream(self, requests, prompt_rows, noise_host, steps, on_chunk, ids_host=None):
        self.calls += 1
        time.sleep(self.first_s)
        on_chunk(0, None)
        time.sleep(0.05)
        on_chunk(1, None)
        return 0, None


def test_time_to_first_audio_times_the_first_chunk():
    bench = _load_bench()
    eng = _FakeEngine(0.02)
    t, calls = bench.time_to_first_audio(eng, 1, 4, None, None, 3, world=1, reps=3)
    assert calls == 3 and eng.calls == 3
    assert 0.02 <= t < 0.06  # the later chunk (0.07 s) does not count
