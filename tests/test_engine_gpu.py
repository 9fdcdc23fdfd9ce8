"""GPU parity of the batched generation engine against the CPU oracle's reference loop.

The engine runs R requests at once (stacked rows, tensor cores above 8 rows, two streams, CUDA
graphs); the oracle restates MingEngine.generate (Engine.swift:302-415) for one request at a time on
the same weights (a host copy of the engine's arena). Per request and step: LLM output z, stop
logits, aggregator output, step-0 velocities, every latent, and the streamed waveform.
Bar (north star): latents and waveform cosine >= 0.999 for the same noise; here also
max|latent error| <= 1e-3 * max|latent| and per-step stop logits within 1e-3.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import cosine, rel_err

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def oracle_generate(oracle, cfg, w_host, embeds, noise, steps, cfg_scale=2.0, obey_stop=0, initial_history=None):
    L, H, Hv = cfg.latent_dim, cfg.llm.hidden, cfg.vae.hidden
    T = embeds.shape[0]
    out = dict(stop=np.zeros((steps, 2), np.float32), z=np.zeros((steps, H), np.float32),
               latents=np.zeros((steps, L), np.float32), agg=np.zeros((steps, H), np.float32),
               vel0=np.zeros((cfg.flow_steps, 2, L), np.float32), vae_hidden=np.zeros((steps, 4, Hv), np.float32),
               pcm=np.zeros(4 * cfg.hop * (steps + 1), np.float32), chunks=np.zeros(steps + 2, np.int32))
    io = oracle.GenerateIO()
    io.prompt_rows, io.embeds, io.steps, io.cfg, io.obey_stop = T, embeds.ctypes.data, steps, cfg_scale, obey_stop
    io.noise = noise.ctypes.data
    io.initial_history = None if initial_history is None else initial_history.ctypes.data
    io.stop_logits, io.llm_hidden, io.latents = out["stop"].ctypes.data, out["z"].ctypes.data, out["latents"].ctypes.data
    io.agg_out, io.velocity0, io.vae_hidden = out["agg"].ctypes.data, out["vel0"].ctypes.data, out["vae_hidden"].ctypes.data
    io.pcm, io.pcm_cap, io.chunk_counts = out["pcm"].ctypes.data, out["pcm"].size, out["chunks"].ctypes.data
    assert oracle.lib().or_generate(ctypes.addressof(cfg), ctypes.addressof(w_host), ctypes.byref(io)) == 0
    out["pcm"] = out["pcm"][:io.pcm_count]
    out["chunks"] = out["chunks"][:io.chunks]
    out["steps_run"], out["stopped"] = io.steps_run, io.stopped
    return out


def engine_generate(mt, eng, cfg, embeds=None, ids=None, noise=None, steps=1, cfg_scale=2.0, initial_history=None):
    import torch
    R, T = (embeds.shape[0], embeds.shape[1]) if embeds is not None else ids.shape
    H, L = cfg.llm.hidden, cfg.latent_dim
    eng.begin(R, T, embeds=dev(embeds) if embeds is not None else None,
              token_ids=dev(ids) if ids is not None else None, noise=dev(noise),
              initial_history=dev(initial_history) if initial_history is not None else None, steps=steps, cfg=cfg_scale)
    eng.prefill()
    res = dict(stop=[], z=[], agg=[], pcm=[[] for _ in range(R)], chunks=[], vae_hidden=[], kernels=0)
    for n in range(steps):
        count = eng.step()
        res["kernels"] = max(res["kernels"], mt.lib().mt_engine_step_kernels(eng.handle))
        torch.cuda.synchronize()
        res["stop"].append(eng.read(mt.BUF_STOP_LOGITS, R))
        res["z"].append(eng.read(mt.BUF_Z, R))
        res["agg"].append(eng.read(mt.BUF_AGG_OUT, R))
        if count:
            res["chunks"].append(count)
            res["vae_hidden"].append(eng.read(mt.BUF_VAE_HIDDEN, R))
            pcm = eng.read(mt.BUF_PCM, R, count)
            for r in range(R):
                res["pcm"][r].append(pcm[r])
    while True:
        count = eng.flush()
        if not count:
            break
        torch.cuda.synchronize()
        res["chunks"].append(count)
        res["vae_hidden"].append(eng.read(mt.BUF_VAE_HIDDEN, R))
        pcm = eng.read(mt.BUF_PCM, R, count)
        for r in range(R):
            res["pcm"][r].append(pcm[r])
    res["latents"] = eng.read(mt.BUF_LATENTS, R).reshape(R, -1, L)[:, :steps]
    res["vel0"] = eng.read(mt.BUF_VELOCITY0, R).reshape(R, cfg.flow_steps, 2, L)
    res["stop"] = np.stack(res["stop"], 1)
    res["z"] = np.stack(res["z"], 1)
    res["agg"] = np.stack(res["agg"], 1)
    res["pcm"] = [np.concatenate(p) for p in res["pcm"]]
    res["vae_hidden"] = np.stack(res["vae_hidden"], 1).reshape(R, -1, 4, cfg.vae.hidden)
    return res


def compare(mt, oracle, ctx, cfg, R, T, steps, seed, use_graphs=True, use_ids=False, lat_rel=1e-3, groups=0,
            with_history=False, check=None):
    """Runs R requests through the engine and checks requests `check` (default: all) against the
    oracle's one-request loop."""
    model = mt.Model(ctx, cfg, seed=seed)
    host = model.arena_to_host()
    tensors = model.tensors()
    w_host, keep = mt.weights_struct(cfg, host.ctypes.data, tensors)
    H, L = cfg.llm.hidden, cfg.latent_dim
    rs = np.random.default_rng(seed)
    noise = np.stack([oracle.gaussian_noise(steps * L, 1000 + r).reshape(steps, L) for r in range(R)])
    if use_ids:
        ids = rs.integers(0, cfg.vocab, size=(R, T), dtype=np.int32)
        off = {t.name.decode(): t.offset for t in tensors}["model.model.embed_tokens.weight"]
        table = host[off:off + cfg.vocab * H * 2].view(np.uint16).reshape(cfg.vocab, H)
        embeds = oracle.bf16_to_f32(table[ids]).astype(np.float32)
    else:
        ids = None
        embeds = (0.5 * rs.standard_normal((R, T, H))).astype(np.float32)
    # a cloned voice's starting history: the reference clip's last latent (MingTTS.swift:105, 112-114)
    hist = rs.standard_normal((R, L)).astype(np.float32) if with_history else None
    eng = mt.Engine(ctx, model, R, T, steps, use_graphs=use_graphs, groups=groups)
    got = engine_generate(mt, eng, cfg, embeds=None if use_ids else embeds, ids=ids, noise=noise, steps=steps,
                          initial_history=hist)
    for r in (range(R) if check is None else check):
        want = oracle_generate(oracle, cfg, w_host, np.ascontiguousarray(embeds[r]), np.ascontiguousarray(noise[r]), steps,
                               initial_history=None if hist is None else np.ascontiguousarray(hist[r]))
        tag = f"R{R} request {r}"
        assert list(got["chunks"]) == list(want["chunks"]), f"{tag}: emission counts"
        assert rel_err(got["z"][r], want["z"]) < 1e-3, f"{tag}: llm hidden rel {rel_err(got['z'][r], want['z'])}"
        assert np.abs(got["stop"][r] - want["stop"]).max() < 1e-3, f"{tag}: stop logits"
        assert rel_err(got["vel0"][r], want["vel0"]) < 1e-3, f"{tag}: step-0 velocity"
        assert rel_err(got["agg"][r], want["agg"]) < 1e-3, f"{tag}: aggregator out"
        lat_c = cosine(got["latents"][r], want["latents"])
        lat_e = rel_err(got["latents"][r], want["latents"])
        assert lat_c >= 0.9999 and lat_e <= lat_rel, f"{tag}: latents cosine {lat_c} rel {lat_e}"
        vh = got["vae_hidden"][r]
        assert rel_err(vh, want["vae_hidden"][:vh.shape[0]]) < 2e-3, f"{tag}: vae hidden"
        pc = cosine(got["pcm"][r], want["pcm"])
        assert got["pcm"][r].shape == want["pcm"].shape and pc >= 0.999, f"{tag}: waveform cosine {pc}"
    eng.close()
    model.close()
    return got


def test_small_model_mixed_routes(ctx, mt, oracle):
    # R = 3: LLM and aggregator rows on the GEMV, flow (18) and VAE (12) rows on the tensor cores.
    compare(mt, oracle, ctx, mt.small_config(), R=3, T=5, steps=7, seed=3)


def test_small_model_all_tensor_core(ctx, mt, oracle):
    compare(mt, oracle, ctx, mt.small_config(), R=12, T=6, steps=6, seed=4, use_ids=True)


@pytest.mark.parametrize("R,groups", [(12, 3), (11, 2)])
def test_small_model_request_groups(ctx, mt, oracle, R, groups):
    # Requests split into groups stepped on their own streams (11 = 6 + 5: uneven groups).
    compare(mt, oracle, ctx, mt.small_config(), R=R, T=5, steps=6, seed=7, groups=groups)


def test_initial_history_matches_oracle(ctx, mt, oracle):
    """mt_engine_begin's initial_history (Options.initialHistory, Engine.swift:315): per-request
    starting latent history of the flow head, as a cloned voice sets it."""
    got = compare(mt, oracle, ctx, mt.small_config(), R=3, T=4, steps=4, seed=21, with_history=True)
    plain = compare(mt, oracle, ctx, mt.small_config(), R=3, T=4, steps=4, seed=21)
    assert rel_err(got["latents"], plain["latents"]) > 1e-2  # the history reaches the flow head


def test_graph_replay_matches_eager(ctx, mt, oracle):
    cfg = mt.small_config()
    model = mt.Model(ctx, cfg, seed=5)
    R, T, steps = 9, 4, 6
    rs = np.random.default_rng(5)
    embeds = (0.5 * rs.standard_normal((R, T, cfg.llm.hidden))).astype(np.float32)
    noise = rs.standard_normal((R, steps, cfg.latent_dim)).astype(np.float32)
    outs = []
    for graphs, groups in ((False, 1), (True, 1), (True, 3)):
        eng = mt.Engine(ctx, model, R, T, steps, use_graphs=graphs, groups=groups)
        outs.append(engine_generate(mt, eng, cfg, embeds=embeds, noise=noise, steps=steps))
        eng.close()
    # Split-K reductions add partial sums in arrival order, so replays agree to rounding, not bits;
    # groups change the tile shapes and therefore the rounding too.
    for o in outs[1:]:
        assert rel_err(o["latents"], outs[0]["latents"]) < 1e-5
        for a, b in zip(outs[0]["pcm"], o["pcm"]):
            assert cosine(a, b) > 0.999999


def test_generate_host_api_matches_steps(ctx, mt, oracle):
    cfg = mt.small_config()
    model = mt.Model(ctx, cfg, seed=6)
    R, T, steps = 4, 5, 5
    rs = np.random.default_rng(6)
    embeds = (0.5 * rs.standard_normal((R, T, cfg.llm.hidden))).astype(np.float32)
    noise = rs.standard_normal((R, steps, cfg.latent_dim)).astype(np.float32)
    eng = mt.Engine(ctx, model, R, T, steps)
    pcm, stop = eng.generate(R, T, noise, steps, embeds_host=embeds)
    ref = engine_generate(mt, eng, cfg, embeds=embeds, noise=noise, steps=steps)
    assert pcm.shape == (R, 4 * cfg.hop * steps)
    for r in range(R):
        assert cosine(pcm[r], ref["pcm"][r]) > 0.999999 and rel_err(pcm[r], ref["pcm"][r]) < 1e-4
        p = 1.0 / (1.0 + np.exp(ref["stop"][r][:, 0] - ref["stop"][r][:, 1]))
        np.testing.assert_allclose(stop[r], p, atol=1e-5)


def test_generate_stream_delivers_generate_chunks(ctx, mt, oracle):
    """mt_engine_generate_stream hands over the same PCM as mt_engine_generate, chunk by chunk in
    order (4 hop-sized frames per step from step 2 on, then the flush), and a truthy callback
    return cancels with MT_ERR_STATE leaving the engine usable."""
    cfg = mt.small_config()
    model = mt.Model(ctx, cfg, seed=9)
    R, T, steps = 3, 4, 6
    rs = np.random.default_rng(9)
    embeds = (0.5 * rs.standard_normal((R, T, cfg.llm.hidden))).astype(np.float32)
    noise = rs.standard_normal((R, steps, cfg.latent_dim)).astype(np.float32)
    eng = mt.Engine(ctx, model, R, T, steps)
    pcm, stop = eng.generate(R, T, noise, steps, embeds_host=embeds)
    chunks = []
    count, stop_s = eng.generate_stream(R, T, noise, steps, lambda i, block: chunks.append((i, block)),
                                        embeds_host=embeds)
    assert [i for i, _ in chunks] == list(range(len(chunks)))
    assert all(b.shape[0] == R for _, b in chunks)
    streamed = np.concatenate([b for _, b in chunks], axis=1)
    assert count == streamed.shape[1] == pcm.shape[1]
    for r in range(R):
        assert cosine(streamed[r], pcm[r]) > 0.999999 and rel_err(streamed[r], pcm[r]) < 1e-4
    np.testing.assert_allclose(stop_s, stop, atol=1e-5)
    seen = []
    with pytest.raises(mt.MingError) as e:
        eng.generate_stream(R, T, noise, steps, lambda i, block: seen.append(i) or i == 1, embeds_host=embeds)
    assert e.value.status == mt.MT_ERR_STATE and seen == [0, 1]
    pcm2, _ = eng.generate(R, T, noise, steps, embeds_host=embeds)
    for r in range(R):
        assert rel_err(pcm2[r], pcm[r]) < 1e-4


def pin_stop_bias(mt, model, l0, l1):
    """Writes the stop head's bias (bf16 [2], exact for these values) on the device, so that the
    stop probability 1/(1+exp(l0-l1)) sits far from 0.5 whatever the random stop weights give."""
    import torch
    base, _ = model.arena()
    off = {t.name.decode(): t.offset for t in model.tensors()}["stop_head.bias"]
    bits = (np.array([l0, l1], np.float32).view(np.uint32) >> 16).astype(np.uint16).view(np.int16)
    mt.device_view(base + off, (2,), "int16").copy_(torch.from_numpy(bits))
    torch.cuda.synchronize()


@pytest.mark.parametrize("R", [1, 2])
def test_stop_rule_matches_reference_loop(ctx, mt, oracle, R):
    """mt_engine_set_stop_rule against the oracle's loop with the stop obeyed (Engine.swift:347-367):
    with p pinned near 1 every request meets the rule at n = 4, so 5 steps run and the flush follows;
    the waveform, emission counts and steps run match the oracle's, through both host APIs."""
    cfg = mt.small_config()
    model = mt.Model(ctx, cfg, seed=13)
    pin_stop_bias(mt, model, -16.0, 16.0)
    host = model.arena_to_host()
    w_host, keep = mt.weights_struct(cfg, host.ctypes.data, model.tensors())
    T, steps = 4, 9
    rs = np.random.default_rng(13)
    embeds = (0.5 * rs.standard_normal((R, T, cfg.llm.hidden))).astype(np.float32)
    noise = rs.standard_normal((R, steps, cfg.latent_dim)).astype(np.float32)
    eng = mt.Engine(ctx, model, R, T, steps)
    eng.stop_rule(True)
    pcm, stop = eng.generate(R, T, noise, steps, embeds_host=embeds)
    assert eng.steps_done() == 5
    assert np.all(stop[:, :5] > 0.5) and np.all(stop[:, 5:] == 0)
    chunks = []
    count, _ = eng.generate_stream(R, T, noise, steps, lambda i, b: chunks.append(b), embeds_host=embeds)
    assert eng.steps_done() == 5 and count == pcm.shape[1]
    for r in range(R):
        want = oracle_generate(oracle, cfg, w_host, np.ascontiguousarray(embeds[r]), np.ascontiguousarray(noise[r]),
                               steps, obey_stop=1)
        assert want["stopped"] == 1 and want["steps_run"] == 5
        assert [b.shape[1] for b in chunks] == list(want["chunks"])
        assert pcm[r].shape == want["pcm"].shape and cosine(pcm[r], want["pcm"]) >= 0.999
        streamed = np.concatenate([b[r] for b in chunks])
        assert rel_err(streamed, pcm[r]) < 1e-4
    # p pinned near 0: the rule never holds and every step runs, as without the rule
    eng.close()
    pin_stop_bias(mt, model, 16.0, -16.0)
    eng = mt.Engine(ctx, model, R, T, steps)
    eng.stop_rule(True)
    pcm_all, stop_all = eng.generate(R, T, noise, steps, embeds_host=embeds)
    assert eng.steps_done() == steps and np.all(stop_all < 0.5)
    eng.stop_rule(False)
    pcm_off, _ = eng.generate(R, T, noise, steps, embeds_host=embeds)
    assert pcm_all.shape == pcm_off.shape == (R, 4 * cfg.hop * steps)
    for r in range(R):
        assert rel_err(pcm_all[r], pcm_off[r]) < 1e-4
    eng.close()
    model.close()


def test_full_model_parity(ctx, mt, oracle):
    # Reference dimensions (Ming-3.0-tts-0.5B), two requests, four steps and the flush.
    compare(mt, oracle, ctx, mt.default_config(), R=2, T=8, steps=4, seed=1, use_ids=True)


def test_full_model_batched_parity(ctx, mt, oracle):
    # Enough requests that every stack (LLM 12 rows, flow 72, aggregator 24, VAE 48) is on the tensor cores.
    compare(mt, oracle, ctx, mt.default_config(), R=12, T=4, steps=3, seed=2, use_ids=True)


def test_full_model_two_groups_parity(ctx, mt, oracle):
    # Two request groups of 10 (LLM 10 rows, flow 60, aggregator 20 each) on concurrent streams.
    compare(mt, oracle, ctx, mt.default_config(), R=20, T=4, steps=3, seed=8, use_ids=True, groups=2)


def test_serving_config_parity(ctx, mt, oracle):
    """The benchmarked configuration (64 requests, 128-token prompts) for 40 steps: LLM 64-row tiles,
    flow 384-row plans with split-K, aggregator 128 rows, VAE 256-row plans, an 8192-row prefill,
    and the VAE ring of 128 positions wrapping after latent 32. Three requests spread over the
    tiles are checked against the oracle."""
    compare(mt, oracle, ctx, mt.default_config(), R=64, T=128, steps=40, seed=11, use_ids=True, check=[0, 33, 63])


@pytest.mark.parametrize("R", [2, 9])
def test_long_cache_parity(ctx, mt, oracle, R):
    """Positions 424..447 of the 512-entry cache: the decode attention stages more keys than its
    shared memory holds (chunks of 416 keys) and merges them with the online softmax, inside the
    engine; R = 2 runs the LLM rows on the CUDA-core GEMV, R = 9 on the tensor cores."""
    compare(mt, oracle, ctx, mt.default_config(), R=R, T=424, steps=24, seed=12, use_ids=True, check=[0, R - 1])


def test_alternate_dit_dims_parity(ctx, mt, oracle):
    """BASELINE config 3's DiT dimensions (hidden 512, 8 heads, 6 blocks, MLP 2048) in the reference's
    block structure (DiT.swift:35-52) for the flow head; the kernels are shape-generic."""
    cfg = mt.default_config()
    cfg.flow.hidden, cfg.flow.heads, cfg.flow.depth, cfg.flow.ff = 512, 8, 6, 2048
    compare(mt, oracle, ctx, cfg, R=12, T=4, steps=3, seed=14, use_ids=True, check=[0, 5, 11])
    compare(mt, oracle, ctx, cfg, R=1, T=4, steps=3, seed=15, use_ids=True)


@pytest.mark.parametrize("R", [1, 2, 4])
def test_persistent_stacks_match_per_op(ctx, mt, oracle, R):
    """With few requests the engine runs the LLM token (R <= 8 rows), the VAE decode (4R <= 8),
    the flow DiT pass (6R <= 8) and the aggregator (2R <= 8) as persistent stack launches; the
    per-op path (one launch per kernel) gives the same generation, and both match the oracle."""
    cfg = mt.small_config()
    ctx.set_persistent(0)
    off = compare(mt, oracle, ctx, cfg, R=R, T=5, steps=6, seed=30 + R)
    try:
        ctx.set_persistent(1)
        on = compare(mt, oracle, ctx, cfg, R=R, T=5, steps=6, seed=30 + R)
    finally:
        ctx.set_persistent(0)
    assert on["kernels"] < off["kernels"]  # some stacks ran as single launches
    assert rel_err(on["latents"], off["latents"]) < 1e-5
    for a, b in zip(on["pcm"], off["pcm"]):
        assert cosine(a, b) > 0.999999


def test_single_request_full_model_parity(ctx, mt, oracle):
    """One request at the reference dimensions (the reference's own use): every stack of the step
    runs as a persistent launch (LLM 1 row, flow 6 rows, aggregator 2 rows, VAE 4 rows)."""
    try:
        ctx.set_persistent(1)
        compare(mt, oracle, ctx, mt.default_config(), R=1, T=12, steps=5, seed=16, use_ids=True)
    finally:
        ctx.set_persistent(0)
