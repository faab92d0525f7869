"""The tensor-core prefill attention (tensor mode) against the CUDA-core split-K attention on the
same inputs, through plamo_k_attention_rows: many query rows of chunked prefill geometry
(Runtime.swift:389-395; Kernels.metal:301-562), global and local (window re-rotation, a wrapped
ring) layers, windows longer than one tensor-core split (2,048 keys) and 8-row groups that span two
chunks. The CUDA-core kernels are bit-identical to the CPU restatement (test_kernels_gpu.py); the
tensor-core kernel sums in the tensor core's order and carries P as a bf16 hi/lo pair, so it is
held to rounding: every output within 4e-3 (two bf16 ulps at the outputs' magnitude) and nearly all
outputs identical. A wrong row, head, key tile or mask fails by O(1)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, W = 16, 2048


def geometry(chunks, p0, cap, full):
    """[rows][4] {first, count, begin, end} of consecutive prefill chunks starting at p0."""
    geo, pos = [], p0
    for n in chunks:
        cstart = pos
        for j in range(n):
            p = cstart + j
            if full:
                geo.append((0, cstart + n, 0, p + 1))
            else:
                first = max(0, cstart - (W - 1))
                end = p - first + 1
                geo.append((first, cstart + n - first, max(0, end - W), end))
        pos += n
    assert all(g[1] <= cap for g in geo)
    return np.array(geo, dtype=np.int32)


@pytest.mark.parametrize("full,cap,p0,chunks,splits", [
    (1, 4096, 3900, [12, 16, 16, 16, 4], 32),    # global: keys 3.9k-4k, two tensor splits
    (0, 2064, 3000, [12, 16, 16, 16, 4], 33),    # local: ring wrapped, 2,048-key windows
    (0, 2064, 0, [16, 16, 8], 33),               # local from position 0: short, causal windows
    (1, 32768, 28660, [4, 16, 16], 128),         # global at the end of a 32k context (C5a)
])
def test_tensor_attention_matches_cuda_core(pkg, oracle, full, cap, p0, chunks, splits):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    rt = pkg.runtime
    rng = np.random.default_rng(1000 + p0 + full)
    geo = geometry(chunks, p0, cap, full)
    rows = len(geo)
    inv = np.array([1e4 ** (-2 * i / 128) for i in range(64)], dtype=np.float32)
    table = oracle.rope_tables(inv, inv, 2064, 1)[0].view(np.uint32)
    keys = oracle.f32_to_bf16(rng.standard_normal(cap * 128).astype(np.float32))
    values = oracle.f32_to_bf16(rng.standard_normal(cap * 128).astype(np.float32))
    q = oracle.f32_to_bf16(rng.standard_normal(rows * H * 128).astype(np.float32))

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16 if a.dtype == np.uint16 else np.int32)).cuda()

    tq, tk, tv, tt, tg = dev(q), dev(keys), dev(values), dev(table), dev(geo)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    outs = {}
    for tensor in (0, 1):
        out = torch.full((rows * H * 128,), -1, dtype=torch.int16, device="cuda")
        rt.k_attention_rows(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), H, 1, cap, tg.data_ptr(), rows, full,
                            tt.data_ptr(), splits, tensor, out.data_ptr(), ws.data_ptr(), ws.numel())
        torch.cuda.synchronize()
        outs[tensor] = oracle.bf16_to_f32(out.cpu().numpy().view(np.uint16)).reshape(rows, H, 128)
    exact, tc = outs[0], outs[1]
    assert np.isfinite(exact).all() and np.isfinite(tc).all()
    diff = np.abs(tc - exact)
    worst = np.unravel_index(diff.argmax(), diff.shape)
    same = float(np.mean(tc == exact))
    assert diff.max() <= 4e-3, dict(worst=worst, diff=float(diff.max()), same=same)
    assert same >= 0.9, same
    print(f"rows {rows} cap {cap}: max |diff| {diff.max():.2e}, identical {same:.4f}")


def test_tensor_attention_rejects_other_head_layouts(pkg):
    """The tensor-core kernel takes 16 query heads over one KV head; other layouts report an error
    (the runtime keeps them on the CUDA-core kernel)."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    with pytest.raises(pkg.PlamoError, match="16 query heads over one KV head"):
        pkg.runtime.k_attention_rows(p, p, p, 16, 4, 64, p, 1, 1, 0, 4, 1, p, p, buf.numel())


@pytest.mark.parametrize("full,cap,p0,rows,splits", [
    (0, 2064, 500, 32, 33),       # batched step after 512-token prompts: short local windows
    (0, 2064, 3000, 32, 33),      # local, ring wrapped, full 2,048-key windows
    (1, 4096, 3990, 16, 32),      # global: 128-key splits, two key tiles per split
    (1, 32768, 32700, 16, 128),   # global at the end of a 32k context: 256-key splits
])
def test_decode_row_tensor_attention_matches_cuda_core(pkg, oracle, full, cap, p0, rows, splits):
    """Tensor mode's decode-row kernel (tensor == 2: one row per lane of a batched step, 16 heads as
    the 16 rows of warp-level bf16 MMAs, P as a bf16 hi / lo pair) against the CUDA-core kernels on
    the same rows and the same splits: held to rounding like the prefill kernel above."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    rt = pkg.runtime
    rng = np.random.default_rng(2000 + p0 + full)
    geo = geometry([1] * rows, p0, cap, full)
    inv = np.array([1e4 ** (-2 * i / 128) for i in range(64)], dtype=np.float32)
    table = oracle.rope_tables(inv, inv, 2064, 1)[0].view(np.uint32)
    keys = oracle.f32_to_bf16(rng.standard_normal(cap * 128).astype(np.float32))
    values = oracle.f32_to_bf16(rng.standard_normal(cap * 128).astype(np.float32))
    q = oracle.f32_to_bf16(rng.standard_normal(rows * H * 128).astype(np.float32))

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16 if a.dtype == np.uint16 else np.int32)).cuda()

    tq, tk, tv, tt, tg = dev(q), dev(keys), dev(values), dev(table), dev(geo)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    outs = {}
    for tensor in (0, 2):
        out = torch.full((rows * H * 128,), -1, dtype=torch.int16, device="cuda")
        rt.k_attention_rows(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), H, 1, cap, tg.data_ptr(), rows, full,
                            tt.data_ptr(), splits, tensor, out.data_ptr(), ws.data_ptr(), ws.numel())
        torch.cuda.synchronize()
        outs[tensor] = oracle.bf16_to_f32(out.cpu().numpy().view(np.uint16)).reshape(rows, H, 128)
    exact, mma = outs[0], outs[2]
    assert np.isfinite(exact).all() and np.isfinite(mma).all()
    diff = np.abs(mma - exact)
    worst = np.unravel_index(diff.argmax(), diff.shape)
    same = float(np.mean(mma == exact))
    assert diff.max() <= 4e-3, dict(worst=worst, diff=float(diff.max()), same=same)
    assert same >= 0.9, same
    print(f"decode rows {rows} cap {cap}: max |diff| {diff.max():.2e}, identical {same:.4f}")


def test_decode_row_tensor_attention_rejects_other_head_layouts(pkg):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    with pytest.raises(pkg.PlamoError, match="16 query heads over one KV head"):
        pkg.runtime.k_attention_rows(p, p, p, 16, 4, 64, p, 1, 1, 0, 4, 2, p, p, buf.numel())
