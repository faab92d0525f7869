"""plamo_k_attention_static (fixed device scratch, no allocation) against plamo_k_attention on the
same inputs: two calls in a row through the C ABI, the first with more splits than the second, so
the second runs on scratch that still holds the first call's partials."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _case(oracle, torch, keep, count, full, seed):
    rng = np.random.default_rng(seed)
    cap = count if full else 2064
    first = 0 if full else 2043
    inv = np.array([1e4 ** (-2 * i / 128) for i in range(64)], dtype=np.float32)
    table = oracle.rope_tables(inv, inv, 2064, 1)[0].view(np.uint32)
    keys = oracle.f32_to_bf16(rng.standard_normal(cap * 128).astype(np.float32))
    values = oracle.f32_to_bf16(rng.standard_normal(cap * 128).astype(np.float32))
    q = oracle.f32_to_bf16(rng.standard_normal(16 * 128).astype(np.float32) * 0.3)
    end = count
    begin = 0 if full else max(0, end - 2048)

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16 if a.dtype == np.uint16 else np.int32)).cuda()
        keep.append(t)
        return t.data_ptr()

    return (dev(q), dev(keys), dev(values), 16, 1, cap, first, count, begin, end, full, dev(table))


def test_static_scratch_attention_matches_allocating_entry_point(pkg, oracle):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    rt = pkg.runtime
    keep = []
    for count, full, splits, seed in [(32768, True, 128, 11), (2063, False, 32, 12)]:
        args = _case(oracle, torch, keep, count, full, seed)
        ref = torch.zeros(16 * 128, dtype=torch.int16, device="cuda")
        got = torch.full((16 * 128,), -1, dtype=torch.int16, device="cuda")
        rt.k_attention(*args, splits, ref.data_ptr())
        rt.k_attention_static(*args, splits, got.data_ptr())
        torch.cuda.synchronize()
        r = oracle.bf16_to_f32(ref.cpu().numpy().view(np.uint16))
        g = oracle.bf16_to_f32(got.cpu().numpy().view(np.uint16))
        assert np.isfinite(g).all()
        # the same kernels on the same inputs: identical bits (well inside the 2e-3 attention tolerance)
        assert np.array_equal(g.view(np.uint32), r.view(np.uint32)), (count, splits)
    with pytest.raises(pkg.PlamoError, match="static 2 MiB buffer"):
        rt.k_attention_static(*args, 4096, got.data_ptr())
    torch.cuda.synchronize()
    keep.clear()
