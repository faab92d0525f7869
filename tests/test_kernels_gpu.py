"""Kernel-level parity of the CUDA path (through the C ABI of include/plamo_kernels.h) against the
CPU restatement and the reference's known-answer vectors."""
import json

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("CUDA device required")
    return t


@pytest.fixture(scope="module")
def rt(pkg):
    return pkg.runtime


# Device buffers handed to the C ABI as raw pointers must outlive the kernels that use them: a
# temporary tensor whose only use is `.data_ptr()` is released to torch's caching allocator at
# once and its memory can be handed to the next temporary. Every buffer made by dev() is kept
# alive until the end of the test (after a device synchronisation).
_ALIVE = []


@pytest.fixture(autouse=True)
def _keep_device_buffers_alive():
    yield
    import torch as t
    if t.cuda.is_available():
        t.cuda.synchronize()
    _ALIVE.clear()


def dev(torch, a):
    """numpy -> CUDA tensor with the same bytes (kept alive for the rest of the test)."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        t = torch.from_numpy(a.view(np.int16)).cuda()
    elif a.dtype == np.uint32:
        t = torch.from_numpy(a.view(np.int32)).cuda()
    elif a.dtype == np.uint64:
        t = torch.from_numpy(a.view(np.int64)).cuda()
    else:
        t = torch.from_numpy(a).cuda()
    _ALIVE.append(t)
    return t


def host(t, dtype):
    return t.cpu().numpy().view(dtype)


def bf16_bits(oracle, x):
    return oracle.f32_to_bf16(np.asarray(x, dtype=np.float32))


def bf16_ulp(x):
    """Spacing of bf16 numbers at magnitude x (x >= 0): 2^(exponent(x) - 7)."""
    e = np.floor(np.log2(np.maximum(x, 2.0 ** -126)))
    return np.exp2(e - 7)


def test_packed_decode_golden(torch, rt):
    """All 323,584 words of PackedDecodeTests.swift:8-31 (every raw pattern, every (min, sm, code))."""
    g = np.load(GOLDEN / "packed_decode.npz")
    data, entries, expected = dev(torch, g["payload"]), dev(torch, g["entries"]), g["expected"]
    out = torch.zeros(expected.size, dtype=torch.int16, device="cuda")
    rt.k_packed_decode(data.data_ptr(), entries.data_ptr(), expected.size, out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(host(out, np.uint16), expected)


def test_packed_decode_fast_path(torch, rt, pkg):
    """Blocks without signed-zero codes take the paired decode path; must be bit-exact too."""
    gen = torch.Generator().manual_seed(3)
    for std in (0.02, 1.0, 3e-4):
        vals = (torch.randn(256 * 128, generator=gen) * std).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        data, offsets, minima = pkg.packing.pack(vals)
        entries = pkg.packing.tag(offsets, minima)
        out = torch.zeros(vals.size, dtype=torch.int16, device="cuda")
        rt.k_packed_decode(dev(torch, data).data_ptr(), dev(torch, entries).data_ptr(), vals.size, out.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(host(out, np.uint16), vals), std


@pytest.mark.parametrize("rows", [1, 3, 16, 33, 64, 100])
def test_linear_matches_oracle_and_packed_equals_raw(torch, rt, pkg, oracle, rows):
    """linear/matrix (Kernels.metal:92-200) vs the CPU restatement, bit for bit; packed == raw
    bit for bit (PackedTests.swift:6-45). Above 16 rows raw weights go through the tiled GEMM
    and packed weights through the GEMV in 16-row passes, so this also pins GEMM == GEMV."""
    gen = torch.Generator().manual_seed(rows)
    for M, K in [(35, 128), (2304, 1536), (96, 2048), (64, 6144)]:
        w = (torch.randn(M * K, generator=gen) * 0.02).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        x16 = (torch.randn(rows * K, generator=gen)).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        x = oracle.bf16_to_f32(x16).reshape(rows, K)
        ref = oracle.linear(w.reshape(M, K), x, logits=True)
        y = torch.zeros(rows * M, dtype=torch.int16, device="cuda")
        rt.k_linear(dev(torch, w).data_ptr(), 0, dev(torch, x16).data_ptr(), rows, K, M, 0, y.data_ptr())
        data, offsets, minima = pkg.packing.pack(w)
        yp = torch.zeros(rows * M, dtype=torch.int16, device="cuda")
        rt.k_linear(dev(torch, data).data_ptr(), dev(torch, pkg.packing.tag(offsets, minima)).data_ptr(),
                    dev(torch, x16).data_ptr(), rows, K, M, 0, yp.data_ptr())
        torch.cuda.synchronize()
        got, gotp = host(y, np.uint16).reshape(rows, M), host(yp, np.uint16).reshape(rows, M)
        assert np.array_equal(got, gotp), (M, K)
        # the restatement sums in the kernel's order: bit-identical
        bad = got != ref
        assert not bad.any(), (M, K, int(bad.sum()), got[bad][:4], ref[bad][:4])


def test_linear_reference_pattern(torch, rt, oracle):
    """PlamoTests.swift:327-364: m=35, n=128, batch 1..64, within 1e-4 of the bf16-rounded dot."""
    for batch in [1, 3, 16, 32, 33, 64]:
        n, m = 128, 35
        w = bf16_bits(oracle, [((i % 17) - 8) / 16 for i in range(n * m)])
        x16 = bf16_bits(oracle, [((i % 11) - 5) / 8 for i in range(n * batch)])
        y = torch.zeros(batch * m, dtype=torch.int16, device="cuda")
        rt.k_linear(dev(torch, w).data_ptr(), 0, dev(torch, x16).data_ptr(), batch, n, m, 0, y.data_ptr())
        torch.cuda.synchronize()
        got = oracle.bf16_to_f32(host(y, np.uint16)).reshape(batch, m)
        exact = oracle.bf16_to_f32(x16).reshape(batch, n).astype(np.float64) @ oracle.bf16_to_f32(w).reshape(m, n).T
        ref = oracle.bf16_to_f32(oracle.f32_to_bf16(exact.astype(np.float32)))
        assert np.max(np.abs(got - ref)) <= 1e-4


@pytest.mark.parametrize("rows", [3, 40])
def test_swiglu_and_logits_modes(torch, rt, oracle, rows):
    """gate_up + swiglu epilogue (Kernels.metal:202-210) and lm_head + argmax (:704-729); 40 rows
    run the tiled GEMM's epilogues."""
    gen = torch.Generator().manual_seed(11)
    F, K = 518, 1536
    w = (torch.randn(2 * F * K, generator=gen) * 0.02).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    x16 = torch.randn(rows * K, generator=gen).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    x = oracle.bf16_to_f32(x16).reshape(rows, K)
    gates = oracle.linear(w.reshape(2 * F, K), x)
    ref = np.empty((rows, F), dtype=np.float32)
    oracle.lib().oracle_swiglu(gates.ctypes.data_as(oracle._f32p), ref.ctypes.data_as(oracle._f32p), rows, F)
    y = torch.zeros(rows * F, dtype=torch.int16, device="cuda")
    rt.k_linear(dev(torch, w).data_ptr(), 0, dev(torch, x16).data_ptr(), rows, K, 2 * F, 1, y.data_ptr())
    torch.cuda.synchronize()
    got = oracle.bf16_to_f32(host(y, np.uint16)).reshape(rows, F)
    assert np.max(np.abs(got - ref) / (np.abs(ref) + 1e-6)) <= 2 ** -6
    # logits + argmax
    V = 4096
    wl = (torch.randn(V * K, generator=gen) * 0.02).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    yl = torch.zeros(rows * V, dtype=torch.int16, device="cuda")
    keys = torch.zeros(rows, dtype=torch.int64, device="cuda")
    idx = torch.zeros(rows, dtype=torch.int32, device="cuda")
    rt.k_linear(dev(torch, wl).data_ptr(), 0, dev(torch, x16).data_ptr(), rows, K, V, 2, yl.data_ptr(), keys.data_ptr())
    rt.k_argmax_keys(keys.data_ptr(), rows, idx.data_ptr())
    torch.cuda.synchronize()
    logits = host(yl, np.uint16).reshape(rows, V)
    assert np.array_equal(logits, oracle.linear(wl.reshape(V, K), x, logits=True))
    for r in range(rows):
        assert host(idx, np.uint32)[r] == oracle.argmax_bits(logits[r])


def test_argmax_cases(torch, rt, oracle):
    """ArgmaxTests.swift:13-64 (bf16 rows): -inf, NaN, +-0, inf; first index of the maximum."""
    cases = [c for c in json.loads((GOLDEN / "argmax_cases.json").read_text()) if c["compact"]]
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
        bits = oracle.f32_to_bf16(values)
        scratch = torch.zeros(batch, dtype=torch.int64, device="cuda")
        out = torch.zeros(batch, dtype=torch.int32, device="cuda")
        rt.k_argmax(dev(torch, bits).data_ptr(), batch, count, scratch.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        assert host(out, np.uint32).tolist() == c["expected"], c


def test_norm_fused_matches_separate_and_oracle(torch, rt, oracle):
    """PlamoTests.swift:288-325: fused residual + next norm == separate norms bit for bit; and the
    CUDA norm within one bf16 ulp of the CPU restatement."""
    w = bf16_bits(oracle, [((i % 31) - 15) / 64 for i in range(3072)])
    for batch in [1, 3, 16]:
        x = bf16_bits(oracle, [((i % 37) - 18) / 16 for i in range(batch * 1536)])
        res = bf16_bits(oracle, oracle.bf16_to_f32(x) / 2)
        dw = dev(torch, w)
        r1, n1 = dev(torch, res), torch.zeros(batch * 1536, dtype=torch.int16, device="cuda")
        rt.k_norm(dw.data_ptr(), dev(torch, x).data_ptr(), r1.data_ptr(), batch, 1536, 0.2, 1, dw.data_ptr() + 3072, n1.data_ptr())
        r2 = dev(torch, res)
        rt.k_norm(dw.data_ptr(), dev(torch, x).data_ptr(), r2.data_ptr(), batch, 1536, 0.2, 1)
        n2 = torch.zeros(batch * 1536, dtype=torch.int16, device="cuda")
        rt.k_norm(dw.data_ptr() + 3072, r2.data_ptr(), n2.data_ptr(), batch, 1536, 1.0, 0)
        torch.cuda.synchronize()
        assert torch.equal(r1, r2) and torch.equal(n1, n2)
        ref_x, ref_next = oracle.norm(w[:1536], oracle.bf16_to_f32(x).reshape(batch, 1536), 0.2,
                                      residual=oracle.bf16_to_f32(res).reshape(batch, 1536), next_w=w[1536:])
        got = oracle.bf16_to_f32(host(n1, np.uint16)).reshape(batch, 1536)
        got_x = oracle.bf16_to_f32(host(r1, np.uint16)).reshape(batch, 1536)
        assert np.array_equal(got.view(np.uint32), ref_next.view(np.uint32))
        assert np.array_equal(got_x.view(np.uint32), ref_x.view(np.uint32))


def _rope_local(oracle, rows):
    inv = np.array([1e4 ** (-2 * i / 128) for i in range(64)], dtype=np.float32)
    lo, _ = oracle.rope_tables(inv, inv, rows, 1)
    return inv, lo.view(np.uint32)


def test_attention_window_and_ring_mean(torch, rt, oracle):
    """PlamoTests.swift:156-194: uniform scores (zero queries) give the window mean of V; local base
    2043 in a 2064-slot ring and a global layer; tolerance 3e-4."""
    inv, table = _rope_local(oracle, 2064)
    dtable = dev(torch, table)
    for full in [True, False]:
        start, base = (65, 0) if full else (4090, 2043)
        count = start + 2 - base
        cap = count if full else 2064
        keys = np.zeros(cap * 128, dtype=np.uint16)
        values = np.zeros(cap * 128, dtype=np.uint16)
        for pos in range(base, start + 2):
            values[(pos % cap) * 128:(pos % cap + 1) * 128] = oracle.f32_to_bf16(np.float32(pos % 17 - 8))
        q = torch.zeros(16 * 128, dtype=torch.int16, device="cuda")
        dk, dv = dev(torch, keys), dev(torch, values)
        for token in range(2):
            end = start + token - base + 1
            begin = 0 if full else max(0, end - 2048)
            out = torch.zeros(16 * 128, dtype=torch.int16, device="cuda")
            rt.k_attention(q.data_ptr(), dk.data_ptr(), dv.data_ptr(), 16, 1, cap, base, count, begin, end, full,
                           dtable.data_ptr(), 8, out.data_ptr())
            got = oracle.bf16_to_f32(host(out, np.uint16))
            lo = 0 if full else start + token - 2047
            expected = np.mean([p % 17 - 8 for p in range(lo, start + token + 1)])
            assert np.max(np.abs(got - expected)) <= 3e-4


@pytest.mark.parametrize("count,full,splits", [(19, True, 1), (513, True, 4), (2048, False, 32), (2063, False, 32),
                                               (4096, True, 32), (32768, True, 128)])
def test_attention_matches_oracle(torch, rt, oracle, count, full, splits):
    """AttentionTests.swift:16-65 shapes: split-K CUDA attention vs the unfused CPU restatement,
    max-abs <= 2e-3; local rows re-rotate raw keys in a wrapped ring."""
    rng = np.random.default_rng(count)
    cap = count if full else 2064
    first = 0 if full else 2043
    inv, table = _rope_local(oracle, 2064)
    keys = oracle.f32_to_bf16(rng.standard_normal(cap * 128).astype(np.float32))
    values = oracle.f32_to_bf16(rng.standard_normal(cap * 128).astype(np.float32))
    q = oracle.f32_to_bf16(rng.standard_normal(16 * 128).astype(np.float32) * 0.3)
    end = count
    begin = 0 if full else max(0, end - 2048)
    ref = oracle.attention(keys, values, oracle.bf16_to_f32(q), 16, 1, cap, first, count, begin, end, full, inv, 2064)
    out = torch.zeros(16 * 128, dtype=torch.int16, device="cuda")
    rt.k_attention(dev(torch, q).data_ptr(), dev(torch, keys).data_ptr(), dev(torch, values).data_ptr(), 16, 1, cap,
                   first, count, begin, end, full, dev(torch, table).data_ptr(), splits, out.data_ptr())
    torch.cuda.synchronize()
    got = oracle.bf16_to_f32(host(out, np.uint16))
    assert np.isfinite(got).all()
    assert np.max(np.abs(got - ref)) <= 2e-3
    # and bit for bit against the split-K restatement with the same partitioning
    ref_split = oracle.attention(keys, values, oracle.bf16_to_f32(q), 16, 1, cap, first, count, begin, end, full, inv,
                                 2064, split=splits)
    assert np.array_equal(got.view(np.uint32), ref_split.view(np.uint32))


def test_exp_matches_restatement(torch, rt, oracle):
    """The software exp used by softmax and SwiGLU: bit-identical to the restatement's and within
    one ulp of the exact exponential over the float range (specials included)."""
    x = np.concatenate([np.linspace(-110, 90, 400001, dtype=np.float32),
                        np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 88.72283935546875, -103.972084], np.float32)])
    dx = dev(torch, x)
    y = torch.zeros_like(dx)
    rt.k_exp(dx.data_ptr(), y.data_ptr(), x.size)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    ref = oracle.exp(x)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    exact = np.exp(x.astype(np.float64))
    fin = np.isfinite(exact) & (exact > 1e-37) & (exact < 3e38)
    assert np.max(np.abs(got[fin] - exact[fin]) / np.spacing(exact[fin].astype(np.float32))) < 1.0
