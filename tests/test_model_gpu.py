"""Model-level parity of the CUDA runtime (C ABI, include/plamo.h) against the CPU restatement.

Acceptance: next-token logits within RMSE <= 1e-2 and max-abs <= 5e-2
of the restatement at every step, identical greedy ids, .p12 runs bit-identical to bf16 runs.
Greedy ids are compared under teacher forcing (both sides consume the oracle's ids), so one
near-tie cannot cascade; an argmax disagreement is accepted only where the oracle's own top-2
logits are within TIE (two bf16 ulps at the logit scale), and such steps are counted.

The small test models (d 256, 4 layers) amplify fp32 reordering more than the reference dims: two
correct CPU implementations that differ only in summation order already drift by RMSE ~0.03 there.
Their tolerance is therefore max(north-star bound, 2x the restatement's own measured noise floor
on the same prompt and steps, oracle.noise_floor); the reference-dims case uses the bound as is.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RMSE_TOL = 1e-2
MAXABS_TOL = 5e-2
TIE = 0.0625


@pytest.fixture(scope="module")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch


def compare(gpu, ora, prompt, steps):
    """Teacher-forced comparison; returns per-step stats and the oracle's greedy ids."""
    g = gpu.prefill(prompt)
    o = ora.prefill(prompt)
    stats = []
    ids = [o]
    for i in range(steps + 1):
        lg, lo = gpu.logits(), ora.logits()
        err = lg - lo
        top2 = np.sort(lo)[-2:]
        stats.append(dict(rmse=float(np.sqrt(np.mean(err * err))), maxabs=float(np.max(np.abs(err))),
                          same=g == o, near_tie=bool(lo[g] >= lo[o] - TIE), margin=float(top2[1] - top2[0]),
                          bitwise=bool(np.array_equal(lg.view(np.uint32), lo.view(np.uint32)))))
        if i == steps:
            break
        g = gpu.forward([o])
        o = ora.forward([o])
        ids.append(o)
    return stats, ids


def tolerances(floor=None):
    if floor is None:
        return RMSE_TOL, MAXABS_TOL
    return max(RMSE_TOL, 2 * floor["rmse"]), max(MAXABS_TOL, 2 * floor["maxabs"])


def check(stats, floor=None):
    rmse_tol, max_tol = tolerances(floor)
    worst = max(range(len(stats)), key=lambda i: stats[i]["rmse"])
    first_bad = next((i for i, s in enumerate(stats) if s["rmse"] > rmse_tol or s["maxabs"] > max_tol), None)
    detail = dict(worst_step=worst, worst=stats[worst], first_bad=first_bad, floor=floor,
                  first_rmse=[round(s["rmse"], 5) for s in stats[:12]])
    assert max(s["rmse"] for s in stats) <= rmse_tol, detail
    assert max(s["maxabs"] for s in stats) <= max_tol, detail
    for i, s in enumerate(stats):
        assert s["same"] or s["near_tie"], (i, s)


def check_bitwise(stats):
    """The batch-1 / 16-token-chunk CUDA path sums in the restatement's order: every logit of every
    step must be bit-identical (and therefore every greedy id)."""
    first = next((i for i, s in enumerate(stats) if not s["bitwise"]), None)
    assert first is None, dict(first_mismatch=first, stat=stats[first], steps=len(stats))
    assert all(s["same"] for s in stats)


def test_tiny_model_matches_oracle(cuda, pkg, oracle, tiny_dir):
    """Window 32 / ring 48: prefill chunks cross the window and the local rings wrap during decode."""
    rt = pkg.Runtime(tiny_dir, context=200)
    ora = oracle.OracleRuntime(tiny_dir, context=200)
    prompt = pkg.synthetic.seeded_tokens(70, rt.vocab, seed=1)
    stats, _ = compare(rt, ora, prompt, 120)
    check_bitwise(stats)
    # state after the run: KV caches equal the restatement's (local raw keys, global rotated keys)
    for layer in range(rt.layers):
        gk, gv = rt.debug_kv(layer)
        ok, ov = ora.kv(layer)
        assert np.array_equal(gk, ok) and np.array_equal(gv, ov), layer


def test_tiny_packed_equals_raw(cuda, pkg, tiny_dir):
    """PackedTests.swift:6-45: .p12 weights give bit-identical logits and ids."""
    raw = pkg.Runtime(tiny_dir, context=160)
    packed = pkg.Runtime(tiny_dir, context=160, packed=True)
    prompt = pkg.synthetic.seeded_tokens(40, raw.vocab, seed=2)
    a, b = raw.prefill(prompt), packed.prefill(prompt)
    for _ in range(60):
        assert a == b
        assert np.array_equal(raw.logits().view(np.uint32), packed.logits().view(np.uint32))
        a, b = raw.forward([a]), packed.forward([b])
    assert packed.weight_bytes < raw.weight_bytes


def test_gqa_example_dims_match_oracle(cuda, pkg, oracle, example_dir):
    """Grouped-query attention (4 KV heads, 4 query heads each) at BASELINE's example dims: the
    multi-kernel path (hidden 2048 is outside the persistent kernel's plan) bit for bit against the
    restatement through a prefill that crosses the window and decode steps that wrap the rings,
    raw and .p12, with every KV cache compared at the end."""
    rt = pkg.Runtime(example_dir, context=160)
    assert not rt.persistent and rt.kv_heads == 4
    ora = oracle.OracleRuntime(example_dir, context=160)
    prompt = pkg.synthetic.seeded_tokens(45, rt.vocab, seed=8)
    stats, ids = compare(rt, ora, prompt, 40)
    check_bitwise(stats)
    for layer in range(rt.layers):
        gk, gv = rt.debug_kv(layer)
        ok, ov = ora.kv(layer)
        assert np.array_equal(gk, ok) and np.array_equal(gv, ov), layer
    packed = pkg.Runtime(example_dir, context=160, packed=True)
    got = [packed.prefill(prompt)] + [packed.forward([i]) for i in ids[:-1]]
    assert got == ids
    assert np.array_equal(packed.logits().view(np.uint32), rt.logits().view(np.uint32))


def test_p12_bound_to_reference_digest_by_default(cuda, pkg, tiny_dir, monkeypatch):
    """Packed.swift:35-38: an archive whose source digest is not the reference checkpoint's is
    refused unless PLAMO_P12_LOCAL_SOURCE=1 accepts one bound to the safetensors file beside it."""
    monkeypatch.delenv("PLAMO_P12_LOCAL_SOURCE", raising=False)
    with pytest.raises(pkg.PlamoError, match="Incompatible packed archive"):
        pkg.Runtime(tiny_dir, context=64, packed=True)
    monkeypatch.setenv("PLAMO_P12_LOCAL_SOURCE", "1")
    pkg.Runtime(tiny_dir, context=64, packed=True).close()


def test_decode_chain_equals_forward_loop(cuda, pkg, tiny_dir):
    rt = pkg.Runtime(tiny_dir, context=200)
    prompt = pkg.synthetic.seeded_tokens(30, rt.vocab, seed=3)
    nxt = rt.prefill(prompt)
    ids = []
    for _ in range(50):
        nxt = rt.forward([nxt]); ids.append(nxt)
    rt.reset()
    rt.prefill(prompt)
    chained = rt.decode_chain(50)
    assert chained == ids
    assert rt.position == len(prompt) + 50


@pytest.mark.parametrize("packed", [False, True])
def test_persistent_equals_multikernel(cuda, pkg, tiny_dir, monkeypatch, packed):
    """The persistent decode kernel (one cooperative launch per token) against the multi-kernel
    graph of the same runtime: ids, logits, final hidden rows and KV caches bit-identical, through
    prefill (multi-kernel chunks) followed by per-token steps and device-chained steps."""
    mega = pkg.Runtime(tiny_dir, context=240, packed=packed)
    monkeypatch.setenv("PLAMO_PERSISTENT", "0")
    multi = pkg.Runtime(tiny_dir, context=240, packed=packed)
    monkeypatch.delenv("PLAMO_PERSISTENT")
    assert mega.persistent and not multi.persistent
    assert mega.step_launches() == 1 and multi.step_launches() > 1
    prompt = pkg.synthetic.seeded_tokens(45, mega.vocab, seed=4)
    a, b = mega.prefill(prompt), multi.prefill(prompt)
    for step in range(90):
        assert a == b, step
        assert np.array_equal(mega.logits().view(np.uint32), multi.logits().view(np.uint32)), step
        assert np.array_equal(mega.hidden().view(np.uint32), multi.hidden().view(np.uint32)), step
        a, b = mega.forward([a]), multi.forward([b])
    assert mega.decode_chain(60) == multi.decode_chain(60)
    for layer in range(mega.layers):
        mk, mv = mega.debug_kv(layer)
        gk, gv = multi.debug_kv(layer)
        assert np.array_equal(mk, gk) and np.array_equal(mv, gv), layer
    prof = mega.profile_decode(4)
    assert set(prof) == {"persistent"} and prof["persistent"]["launches"] == 4


def test_persistent_long_context_multi_tile(cuda, pkg, tiny_dir, monkeypatch):
    """Global-layer splits wider than one 64-key tile (a 2100-token history over 32 splits gives
    96-key splits): the persistent kernel stages several key and value tiles per split and must
    still equal the multi-kernel path bit for bit."""
    mega = pkg.Runtime(tiny_dir, context=2304)
    monkeypatch.setenv("PLAMO_PERSISTENT", "0")
    multi = pkg.Runtime(tiny_dir, context=2304)
    monkeypatch.delenv("PLAMO_PERSISTENT")
    assert mega.persistent and not multi.persistent
    prompt = pkg.synthetic.seeded_tokens(2100, mega.vocab, seed=5)
    a, b = mega.prefill(prompt), multi.prefill(prompt)
    for step in range(12):
        assert a == b, step
        assert np.array_equal(mega.logits().view(np.uint32), multi.logits().view(np.uint32)), step
        a, b = mega.forward([a]), multi.forward([b])
    for layer in range(mega.layers):
        mk, mv = mega.debug_kv(layer)
        gk, gv = multi.debug_kv(layer)
        assert np.array_equal(mk, gk) and np.array_equal(mv, gv), layer


def test_bounded_wait_timeout_fails_the_call_and_recovers(cuda, pkg, tiny_dir):
    """The failure path of the persistent kernel's bounded waits (Runtime.swift:462 throws on a
    failed command buffer): a device poll on a word that nothing sets gives up after 20 us instead
    of hanging, the call fails with the decode step's timeout message, and the runtime's later
    steps are bit-identical to those of a runtime that never failed."""
    import time
    rt = pkg.Runtime(tiny_dir, context=200)
    twin = pkg.Runtime(tiny_dir, context=200)
    assert rt.persistent and twin.persistent
    prompt = pkg.synthetic.seeded_tokens(30, rt.vocab, seed=6)
    a, b = rt.prefill(prompt), twin.prefill(prompt)
    for _ in range(4):
        a, b = rt.forward([a]), twin.forward([b])
    for _ in range(2):
        t0 = time.perf_counter()
        with pytest.raises(pkg.PlamoError, match="bounded device wait timed out"):
            rt.debug_wait_timeout(20_000)
        assert time.perf_counter() - t0 < 1.0
    assert rt.position == twin.position
    for step in range(24):
        assert a == b, step
        assert np.array_equal(rt.logits().view(np.uint32), twin.logits().view(np.uint32)), step
        a, b = rt.forward([a]), twin.forward([b])
    assert rt.decode_chain(16) == twin.decode_chain(16)


def test_reset_and_errors(cuda, pkg, tiny_dir):
    """PlamoTests.swift:204-209 (reset gives bit-identical logits) and the API edge validation
    (Runtime.swift:328-330, :474)."""
    rt = pkg.Runtime(tiny_dir, context=64)
    prompt = [1] + list(range(500, 532))
    rt.prefill(prompt)
    first = rt.logits().copy()
    rt.reset()
    rt.prefill(prompt)
    assert np.array_equal(first.view(np.uint32), rt.logits().view(np.uint32))
    with pytest.raises(pkg.PlamoError, match="Invalid tokens or context exhausted"):
        rt.forward(list(range(17)))
    with pytest.raises(pkg.PlamoError, match="Invalid tokens or context exhausted"):
        rt.forward([rt.vocab])
    with pytest.raises(pkg.PlamoError, match="Input exceeds context"):
        rt.prefill(list(range(64)))
    with pytest.raises(pkg.PlamoError):
        pkg.Runtime(tiny_dir, context=0)


def test_tiny_batch_matches_scalar_bitwise(cuda, pkg, tiny_dir):
    """BatchMapTests.swift:186-224: after a batched step every active lane holds exactly the scalar
    runtime's state (hidden, logits, KV rows, prediction); inactive lanes are untouched."""
    context = 120
    rt = pkg.Runtime(tiny_dir, context=context)
    prompts = [[1] + [(1000 + j * 17) % rt.vocab for j in range(1, n)] for n in (2, 3, 5, 60)]
    tokens, nxt, state = [], [], []
    for p in prompts:
        rt.reset()
        t = rt.prefill(p); tokens.append(t)
        nxt.append(rt.forward([t]))
        kv = [rt.debug_kv(i) for i in range(rt.layers)]
        state.append((rt.hidden().copy(), rt.logits().copy(), kv))
    batch = pkg.Batch(rt, lanes=4)
    for mask in range(1, 16):
        lanes = [i for i in range(4) if mask & (1 << i)]
        batch.prefill(prompts)
        frozen = {l: (batch.hidden(l).copy(), batch.logits(l).copy()) for l in range(4)}
        out = batch.step([tokens[i] if i in lanes else None for i in range(4)])
        for lane in range(4):
            if lane in lanes:
                hid, log, kv = state[lane]
                assert out[lane] == nxt[lane]
                assert np.array_equal(batch.hidden(lane).view(np.uint32), hid.view(np.uint32))
                assert np.array_equal(batch.logits(lane).view(np.uint32), log.view(np.uint32))
                n = len(prompts[lane]) + 1
                for i in range(rt.layers):
                    bk, bv = batch.debug_kv(i, lane)
                    cap = context if i % rt.pattern == rt.pattern - 1 else min(context, rt.window + 16)
                    rows = min(n, cap) * 128
                    assert np.array_equal(bk[:rows], kv[i][0][:rows]) and np.array_equal(bv[:rows], kv[i][1][:rows])
            else:
                assert np.array_equal(batch.hidden(lane).view(np.uint32), frozen[lane][0].view(np.uint32))


def test_tiny_batch_generate_wraps_ring(cuda, pkg, oracle, tiny_dir):
    """Batch decode past the 48-slot local ring (the C4 situation at tiny scale), lanes vs the
    restatement's Batch under teacher forcing, and decodeBatch stop/length bookkeeping."""
    context = 180
    rt = pkg.Runtime(tiny_dir, context=context)
    ora = oracle.OracleRuntime(tiny_dir, context=context)
    prompts = [pkg.synthetic.seeded_tokens(n, rt.vocab, seed=10 + n) for n in (20, 33, 50, 7)]
    b = pkg.Batch(rt, lanes=4)
    ob = oracle.OracleBatch(ora, lanes=4)
    g = b.prefill(prompts)
    o = ob.prefill(prompts)
    for step in range(100):
        for lane in range(4):
            lg = b.logits(lane); lo = oracle.bf16_to_f32(ob.logits_bits(lane))
            assert np.array_equal(lg.view(np.uint32), lo.view(np.uint32)), (step, lane, float(np.abs(lg - lo).max()))
        assert g == o, (step, g, o)
        active = [o[l] if step < 100 - 10 * l else None for l in range(4)]
        if all(a is None for a in active):
            break
        g = b.step(active)
        o = ob.step(active)
    # decodeBatch: a lane whose prediction is a stop id ends with "stop"; limits end with "length"
    res = b.generate(prompts[:3], [5, 0, 7])
    assert [r[1] for r in res][1] == "length" and len(res[1][0]) == 0
    for ids, reason in res:
        assert reason in ("stop", "length")
        assert all(t not in (1, 16) for t in ids)


@pytest.mark.slow
def test_reference_dims_c2_matches_oracle(cuda, pkg, oracle, reference_dir):
    """512-token seeded prompt, 256 greedy steps, plain bf16 weights, logits
    compared every step; then the .p12 archive (config 3) must reproduce every logit bit for bit."""
    prompt = pkg.synthetic.seeded_tokens(512, 107520, seed=1)
    rt = pkg.Runtime(reference_dir, context=1024)
    ora = oracle.OracleRuntime(reference_dir, context=1024)
    stats, ids = compare(rt, ora, prompt, 256)
    check_bitwise(stats)
    del ora
    # free-running greedy decode on the GPU (device-chained) reproduces the oracle's greedy ids
    rt.reset()
    gpu_ids = [rt.prefill(prompt)] + rt.decode_chain(256)
    assert gpu_ids == ids
    packed = pkg.Runtime(reference_dir, context=1024, packed=True)
    rt.reset()
    a, b = rt.prefill(prompt), packed.prefill(prompt)
    for _ in range(32):
        assert a == b and np.array_equal(rt.logits().view(np.uint32), packed.logits().view(np.uint32))
        a, b = rt.forward([a]), packed.forward([b])
