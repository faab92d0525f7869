"""Pins the CPU restatement (oracle/) against the reference's own known-answer tests."""
import json

import numpy as np
import pytest

from conftest import GOLDEN


def bf(x):
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint32) << 16).view(np.float32)


def test_argmax_cases(oracle):
    """ArgmaxTests.swift:13-64: -inf, NaN, +-0 and inf patterns; first index of the maximum."""
    cases = json.loads((GOLDEN / "argmax_cases.json").read_text())
    for c in cases:
        count, batch, pattern = c["count"], c["batch"], c["pattern"]
        values = np.array([float(((j * 17) % 4093) - 2046) / 32 for j in range(count * batch)], dtype=np.float32)
        for row in range(batch):
            s = row * count
            if pattern == 1: values[s:s + count] = -np.inf
            elif pattern == 2: values[s:s + count] = np.nan
            elif pattern == 3: values[s:s + count] = np.where(np.arange(count) % 2 == 0, -0.0, 0.0)
            elif pattern == 4:
                values[s] = np.nan
                if count > 1: values[s + count - 1] = np.inf
                if count > 257: values[s + 257] = np.inf
        for row in range(batch):
            v = values[row * count:(row + 1) * count]
            got = oracle.argmax_bits(oracle.f32_to_bf16(v)) if c["compact"] else oracle.argmax_f32(v)
            assert got == c["expected"][row], c


def test_linear_pattern(oracle):
    """PlamoTests.swift:327-364: m=35, n=128, several batches, tolerance 1e-4 of the bf16 result."""
    for batch in [1, 3, 16, 32, 33, 64]:
        n, m = 128, 35
        w = oracle.f32_to_bf16(np.array([((i % 17) - 8) / 16 for i in range(n * m)], dtype=np.float32))
        x = bf(np.array([((i % 11) - 5) / 8 for i in range(n * batch)], dtype=np.float32)).reshape(batch, n)
        y = oracle.linear(w.reshape(m, n), x)
        ref = bf((x.astype(np.float64) @ oracle.bf16_to_f32(w).reshape(m, n).T.astype(np.float64)).astype(np.float32))
        assert np.max(np.abs(y - ref)) <= 1e-4


def test_fused_norm_matches_separate(oracle):
    """PlamoTests.swift:288-325: residual norm + fused next norm == two separate norms, bitwise."""
    w = oracle.f32_to_bf16(np.array([((i % 31) - 15) / 64 for i in range(3072)], dtype=np.float32))
    for batch in [1, 3, 16]:
        x = np.array([((i % 37) - 18) / 16 for i in range(batch * 1536)], dtype=np.float32).reshape(batch, 1536)
        residual = x / 2
        y1, nxt = oracle.norm(w[:1536], x, 0.2, residual=residual, next_w=w[1536:])
        y2, _ = oracle.norm(w[:1536], x, 0.2, residual=residual)
        sep, _ = oracle.norm(w[1536:], y2, 1.0)
        assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
        assert np.array_equal(nxt.view(np.uint32), sep.view(np.uint32))


def test_attention_window_and_ring_mean(oracle):
    """PlamoTests.swift:156-194: with uniform scores the output is the mean of V over the window
    (local base 2043 in a 2064-slot ring, and a global layer), tolerance 3e-4."""
    inv = np.array([1e4 ** (-2 * i / 128) for i in range(64)], dtype=np.float32)
    for full in [True, False]:
        start, base = (65, 0) if full else (4090, 2043)
        count = start + 2 - base
        cap = count if full else 2064
        keys = np.zeros(cap * 128, dtype=np.uint16)
        values = np.zeros(cap * 128, dtype=np.uint16)
        for pos in range(base, start + 2):
            values[(pos % cap) * 128:(pos % cap + 1) * 128] = oracle.f32_to_bf16(np.float32(pos % 17 - 8))
        q = np.zeros(16 * 128, dtype=np.float32)  # zero queries -> uniform scores
        for token in range(2):
            end = start + token - base + 1
            begin = 0 if full else max(0, end - 2048)
            out = oracle.attention(keys, values, q, 16, 1, cap, base, count, begin, end, full, inv, 2064)
            lo = 0 if full else start + token - 2047
            expected = np.mean([p % 17 - 8 for p in range(lo, start + token + 1)])
            assert np.max(np.abs(out - expected)) <= 3e-4


def test_split_attention_matches_unfused(oracle):
    """AttentionTests.swift:16-65: 256-key split-K + merge vs the unfused softmax path, <= 2e-3."""
    rng = np.random.default_rng(0)
    inv = np.array([1e4 ** (-2 * i / 128) for i in range(64)], dtype=np.float32)
    for count in [19, 513, 2048, 4096, 32768]:
        keys = oracle.f32_to_bf16(((np.arange(count * 128) * 17) % 43 - 21).astype(np.float32) / 32)
        values = oracle.f32_to_bf16(((np.arange(count * 128) * 13) % 41 - 20).astype(np.float32) / 32)
        q = bf(((np.arange(2048) * 7) % 47 - 23).astype(np.float32) / 32)
        a = oracle.attention(keys, values, q, 16, 1, count, 0, count, 0, count, True, inv, 1)
        b = oracle.attention(keys, values, q, 16, 1, count, 0, count, 0, count, True, inv, 1, split=256)
        assert np.max(np.abs(a - b)) <= 2e-3 and np.isfinite(b).all()


def test_tiny_model_packed_equals_raw(oracle, tiny_dir):
    """PackedTests.swift:6-45 invariant: the .p12 weights decode bit-identical, so every logit of a
    packed run equals the raw run's."""
    raw = oracle.OracleRuntime(tiny_dir, context=96)
    packed = oracle.OracleRuntime(tiny_dir, context=96, packed=True)
    prompt = list(range(5, 40))
    a = raw.prefill(prompt); b = packed.prefill(prompt)
    assert a == b
    assert np.array_equal(raw.logits_bits(), packed.logits_bits())
    for _ in range(8):
        a = raw.forward([a]); b = packed.forward([b])
        assert a == b and np.array_equal(raw.logits_bits(), packed.logits_bits())


def test_tiny_model_reset_is_stable(oracle, tiny_dir):
    """PlamoTests.swift:204-209: logits after reset + identical prefill are bit-identical."""
    rt = oracle.OracleRuntime(tiny_dir, context=64)
    prompt = [1] + list(range(500 % 2048, 532 % 2048))
    rt.prefill(prompt)
    first = rt.logits_bits()
    rt.reset()
    rt.prefill(prompt)
    assert np.array_equal(first, rt.logits_bits())
    with pytest.raises(RuntimeError, match="context"):
        rt.forward(list(range(40)))  # more than one 16-token chunk


def test_tiny_batch_matches_scalar(oracle, tiny_dir):
    """BatchMapTests.swift:186-224: a batched step leaves exactly the scalar state for every
    active-lane mask (hidden, logits and predictions), here with window 32 so rings wrap."""
    context = 120
    rt = oracle.OracleRuntime(tiny_dir, context=context)
    prompts = [[1] + [(1000 + j * 17) % 2048 for j in range(1, n)] for n in (2, 3, 5, 60)]
    tokens, nxt, hid, logits = [], [], [], []
    for p in prompts:
        rt.reset()
        t = rt.prefill(p); tokens.append(t)
        nxt.append(rt.forward([t])); hid.append(rt.hidden_state()); logits.append(rt.logits_bits())
    batch = oracle.OracleBatch(rt, lanes=4)
    for mask in range(1, 16):
        lanes = [i for i in range(4) if mask & (1 << i)]
        batch.prefill(prompts)
        out = batch.step([tokens[i] if i in lanes else None for i in range(4)])
        for lane in lanes:
            assert out[lane] == nxt[lane]
            assert np.array_equal(batch.logits_bits(lane), logits[lane])
            assert np.array_equal(batch.hidden_state(lane).view(np.uint32), hid[lane].view(np.uint32))


def test_noise_floor_twins(oracle, micro_dir):
    """The restatement's two twins (sums reordered; each dot product summed exactly and rounded
    once) run on the micro model and report finite, non-negative drift; the tensor-mode tests
    measure against them."""
    import numpy as np
    prompt = [1] + [(7 * i) % 200 + 2 for i in range(11)]
    for mode in ("reverse", "exact"):
        f = oracle.noise_floor(micro_dir, 64, prompt, 2, mode=mode)
        assert set(f) == {"rmse", "maxabs", "rmse_mean"}
        assert all(np.isfinite(v) and v >= 0 for v in f.values()), (mode, f)
