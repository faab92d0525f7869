"""BASELINE configs 4 and 5a under parity: the batch4 ring wrap at the reference dims, and the
32k-context long-sequence path (global layers over the full history, split-K flash-decode).

C4 (Batch.swift:40,116-128; Runtime.swift:239-247): four lanes whose prompts overrun the
2,064-slot local ring and nearly fill the library's longer physical ring, so both wrap within the
first decoded steps. Every lane's
logits after every batched step must equal the scalar runtime's bit for bit (the scalar path is
itself bit-identical to the CPU restatement), and lane 0 is also checked against the restatement
directly across the wrap.

C5a (Runtime.swift:131,424-430; Kernels.metal:440-562): a 28,672-token prompt in a 32,768-token
context on the committed MICRO model, whose global layer then splits 28.7k-32.7k keys over 128
partitions. The persistent decode kernel and the multi-kernel graph must equal the restatement bit
for bit for the first 64 decoded tokens, then equal each other (ids, logits, global-layer caches)
for the remaining 4,032 tokens up to the end of the context.
"""
import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.fixture(scope="module")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch


def bits(a):
    return a.view(np.uint32)


def test_c4_batch4_rings_wrap_at_reference_dims(cuda, pkg, oracle, reference_dir):
    lens = [2550, 2556, 2562, 2568]
    # positions reach 2590-2608: past the reference's 2,064-slot local ring and past the library's
    # own ring of window + 512 = 2,560 slots, so both wrap during the batched steps
    steps = 40
    context = 2624
    prompts = [pkg.synthetic.seeded_tokens(n, 107520, seed=40 + i) for i, n in enumerate(lens)]
    rt = pkg.Runtime(reference_dir, context=context)
    # the scalar runtime, lane by lane: greedy ids and every step's logits
    want_ids, want_logits, want_kv = [], [], []
    for p in prompts:
        rt.reset()
        ids = [rt.prefill(p)]
        logs = [rt.logits().copy()]
        for _ in range(steps):
            ids.append(rt.forward([ids[-1]]))
            logs.append(rt.logits().copy())
        want_ids.append(ids)
        want_logits.append(logs)
        want_kv.append(rt.debug_kv(0))
    # lane 0 against the CPU restatement across the wrap (teacher forcing by the restatement's ids)
    ora = oracle.OracleRuntime(reference_dir, context=context)
    o = ora.prefill(prompts[0])
    for step in range(steps + 1):
        assert np.array_equal(bits(want_logits[0][step]), bits(ora.logits())), step
        assert want_ids[0][step] == o, step
        if step < steps:
            o = ora.forward([o])
    del ora
    # the batch: one weight pass for the four lanes per step
    b = pkg.Batch(rt, lanes=4)
    got = b.prefill(prompts)
    for step in range(steps + 1):
        for lane in range(4):
            assert got[lane] == want_ids[lane][step], (step, lane)
            assert np.array_equal(bits(b.logits(lane)), bits(want_logits[lane][step])), (step, lane)
        if step < steps:
            got = b.step([want_ids[lane][step] for lane in range(4)])
    for lane in range(4):  # the wrapped local ring of layer 0, slot for slot
        bk, bv = b.debug_kv(0, lane)
        assert np.array_equal(bk, want_kv[lane][0]) and np.array_equal(bv, want_kv[lane][1]), lane
    b.close()
    rt.close()


def test_c5a_long_context_32k(cuda, pkg, oracle, micro_dir, monkeypatch):
    context, prompt_len, checked = 32768, 28672, 64
    prompt = pkg.synthetic.seeded_tokens(prompt_len, 512, seed=7)
    mega = pkg.Runtime(micro_dir, context=context)
    monkeypatch.setenv("PLAMO_PERSISTENT", "0")
    multi = pkg.Runtime(micro_dir, context=context)
    monkeypatch.delenv("PLAMO_PERSISTENT")
    assert mega.persistent and not multi.persistent
    ora = oracle.OracleRuntime(micro_dir, context=context)
    a, b, o = mega.prefill(prompt), multi.prefill(prompt), ora.prefill(prompt)
    for step in range(checked + 1):
        lo = bits(ora.logits())
        assert np.array_equal(bits(mega.logits()), lo), step
        assert np.array_equal(bits(multi.logits()), lo), step
        assert a == o and b == o, step
        if step < checked:  # every side consumes the restatement's id (teacher forcing)
            a, b, o = mega.forward([o]), multi.forward([o]), ora.forward([o])
    del ora
    # to the end of the context: device-chained greedy decode on both paths
    rest = context - mega.position - 1
    assert rest > 4000
    assert mega.decode_chain(rest) == multi.decode_chain(rest)
    assert mega.position == context - 1
    assert np.array_equal(bits(mega.logits()), bits(multi.logits()))
    for layer in range(mega.layers):
        mk, mv = mega.debug_kv(layer)
        gk, gv = multi.debug_kv(layer)
        assert np.array_equal(mk, gk) and np.array_equal(mv, gv), layer
