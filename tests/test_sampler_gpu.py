"""Sampler.select on the device (plamo_k_select, plamo_select) against the CPU restatement
(oracle.sampler_select, Sampler.swift:9-31): the reference's own known answers, seeded full-vocabulary
cases with NaN, +-inf, +-0, repeated and out-of-range history ids, and the runtime entry point on the
logits a prefill left on the device. Integer counts and one IEEE operation per adjustment: the
selected ids must be identical."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch


def device_select(torch, rt, logits_f32, history, penalty, ngram, frequency=0.0, presence=0.0):
    V = len(logits_f32)
    bits = (np.asarray(logits_f32, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    lg = torch.from_numpy(bits.view(np.int16)).cuda()
    hist = torch.tensor(list(history) or [0], dtype=torch.int32, device="cuda")
    counts = torch.zeros(V, dtype=torch.int32, device="cuda")
    flags = torch.zeros(V, dtype=torch.uint8, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    rt.k_select(lg.data_ptr(), V, hist.data_ptr(), len(history), penalty, ngram, frequency, presence,
                counts.data_ptr(), flags.data_ptr(), key.data_ptr())
    torch.cuda.synchronize()
    return rt.select_key_to_id(int(key.cpu().numpy().view(np.uint64)[0]))


def bf16(a):
    a = np.asarray(a, dtype=np.float32)
    return ((a.view(np.uint32) >> 16) << 16).view(np.float32)


def test_k_select_sampler_tests(cuda, pkg, oracle):
    rt = pkg.runtime
    cases = [([1, 2, 2, 0], [], 1, 0, 0, 0), ([1, 5, 4], [1], 2, 0, 0, 0), ([-1, -5, -4], [1], 2, 0, 0, 0),
             ([0, 5, 4], [1], 1, 0, 0.5, 0), ([0, 5, 4], [1, 1, 1], 1, 0, 0.5, 0),
             ([0, 0, 0, 0, 0, 9], [0, 2, 3, 5, 2, 3], 1, 3, 0, 0),
             ([np.nan, -np.inf, np.nan], [], 1, 0, 0, 0), ([-0.0, 0.0], [], 1, 0, 0, 0),
             ([3, 2], [0, 0, 9999, -5], 1, 0, 0, 1.5)]
    for logits, hist, pen, ng, fr, pr in cases:
        want = oracle.sampler_select(bf16(logits), hist, pen, ng, fr, pr)
        assert device_select(cuda, rt, bf16(logits), hist, pen, ng, fr, pr) == want, (logits, hist)


@pytest.mark.parametrize("penalty,ngram,frequency,presence", [(1.0, 0, 0.0, 0.0), (1.3, 0, 0.0, 0.0),
                                                              (0.8, 3, 0.5, 0.0), (1.0, 2, 0.0, 0.0),
                                                              (1.2, 4, 0.25, 0.75)])
def test_k_select_full_vocabulary(cuda, pkg, oracle, penalty, ngram, frequency, presence):
    rt = pkg.runtime
    rng = np.random.default_rng(int(penalty * 100) + ngram)
    V = 107520
    for trial in range(4):
        logits = bf16(rng.normal(0, 2, size=V).astype(np.float32))
        logits[rng.integers(0, V, 8)] = np.nan
        logits[rng.integers(0, V, 4)] = -np.inf
        logits[rng.integers(0, V, 4)] = -0.0
        if trial == 3:
            logits[rng.integers(0, V, 2)] = np.inf
        top = np.argsort(np.nan_to_num(logits, nan=-1e30))[-50:]
        # history: mostly the top logits (so the penalties move the choice), with repeats and
        # out-of-range ids, long enough for n-gram matches
        hist = rng.choice(top, size=300).tolist() + [V + 5, -1]
        hist += hist[-6:-3] * 3
        want = oracle.sampler_select(logits, hist, penalty, ngram, frequency, presence)
        got = device_select(cuda, rt, logits, hist, penalty, ngram, frequency, presence)
        assert got == want, (trial, got, want)


def test_runtime_select_on_device_logits(cuda, pkg, oracle, tiny_dir):
    rt = pkg.Runtime(tiny_dir, context=128)
    prompt = pkg.synthetic.seeded_tokens(40, rt.vocab, seed=7)
    greedy = rt.prefill(prompt)
    assert rt.select([]) == greedy
    generated = [greedy]
    for _ in range(12):
        logits = rt.logits()
        for args in [(1.0, 0, 0.0, 0.0), (1.5, 0, 0.0, 0.0), (1.1, 2, 0.3, 0.2), (1.0, 3, 0.0, 0.0)]:
            want = oracle.sampler_select(logits, generated, *args)
            assert rt.select(generated, *args) == want, args
        nxt = rt.select(generated, 1.3, 2, 0.2, 0.0)
        generated.append(nxt)
        rt.forward([nxt])
    assert pkg.runtime.library().plamo_select(rt._h, None, 3, 1.0, 0, 0.0, 0.0, None) == 1  # invalid arguments
