"""The tcgen05 tensor-core GEMM (gemm_tc.cu, plamo_k_linear_tc) and the runtime's tensor-core mode
(plamo_set_tensor_gemm).

Kernel level: outputs against a float64 PyTorch reference of the same op (then rounded to bf16 as
the kernel rounds); the tensor core accumulates in fp32 in its own order, so a result may sit one
bf16 ulp from the rounded exact sum, rarely more than that.

Model level: the tensor-core prefill and batched steps against the CPU restatement. The seeded
random-init models amplify any change of summation order: the restatement with its dot products
reordered, or rounded exactly once, already drifts from itself by RMSE 0.34 / max |diff| 1.6 at the
reference dims after the 512-token prompt, far outside the north-star bound (RMSE <= 1e-2, max
|diff| <= 5e-2), which only the bit-exact default path meets. The tensor path is therefore held to
max(north-star bound, 4 x that drift on the same prompt and steps), and each greedy pick to within
the same distance of the restatement's top logit.
"""
import numpy as np
import pytest


pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch


def _reference(torch, x, w, mode):
    """float64 sums, then the kernel's epilogue rounding (bf16 outputs; SwiGLU on bf16 g and u)."""
    y = (x.double() @ w.double().T).float()
    if mode == 1:
        F = w.shape[0] // 2
        g = y[:, :F].bfloat16().float()
        u = y[:, F:].bfloat16().float()
        act = (g / (1.0 + torch.exp(-g))).bfloat16().float()
        return (act * u).bfloat16()
    return y.bfloat16()


CASES = [
    # rows, K, M, mode (0 plain, 1 SwiGLU, 2 logits), splits (0 = launcher's choice)
    (16, 1536, 2304, 0, 0),
    (100, 2048, 1536, 0, 0),
    (512, 1536, 2304, 0, 0),
    (300, 6144, 1536, 0, 0),
    (32, 6144, 1536, 0, 0),
    (32, 6144, 1536, 0, 4),
    (7, 128, 300, 0, 2),
    (200, 1536, 1000, 1, 0),
    (32, 1536, 12288, 1, 0),
    (32, 2048, 1536, 1, 8),
    (48, 1536, 4000, 2, 0),
    (32, 1536, 2000, 2, 4),
    # enough tiles for 128-row activation tiles (BN = 128)
    (512, 1536, 12288, 1, 0),
    (300, 1536, 24576, 0, 0),
    (256, 1536, 40000, 2, 0),
    # long K over few tiles: 256-row activation tiles with K split over the idle SMs
    (512, 6144, 1536, 0, 0),
]


@pytest.mark.parametrize("rows,K,M,mode,splits", CASES)
def test_linear_tc_matches_float64_reference(cuda, pkg, rows, K, M, mode, splits):
    torch = cuda
    rt = pkg.runtime
    g = torch.Generator(device="cpu").manual_seed(rows * 7 + K + M + mode)
    w = (torch.randn(M, K, generator=g) * 0.02).bfloat16().cuda()
    x = torch.randn(rows, K, generator=g).bfloat16().cuda()
    Mout = M // 2 if mode == 1 else M
    y = torch.zeros(rows, Mout, dtype=torch.bfloat16, device="cuda")
    keys = torch.zeros(rows, dtype=torch.int64, device="cuda")
    ws = torch.zeros(16 * rows * M + 1, dtype=torch.float32, device="cuda")
    rt.k_linear_tc(w.data_ptr(), x.data_ptr(), rows, K, M, mode, y.data_ptr(), keys.data_ptr() if mode == 2 else 0,
                   splits, ws.data_ptr(), ws.numel())
    torch.cuda.synchronize()
    ref = _reference(torch, x, w, mode).float().cpu().numpy()
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    # one bf16 ulp of the reference value; SwiGLU rounds g, g*sigmoid(g), u and the product, so an
    # ulp in g or u can grow to a few ulps of the output
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
    diff = np.abs(got - ref)
    allowed = (4 if mode == 1 else 1) * ulp + 1e-6 * np.abs(ref).max()
    assert (diff <= allowed).all(), (float(diff.max()), int((diff > allowed).sum()))
    assert (diff == 0).mean() >= (0.95 if mode == 1 else 0.98), float((diff == 0).mean())
    if mode == 2:
        idx = torch.zeros(rows, dtype=torch.int32, device="cuda")
        rt.k_argmax_keys(keys.data_ptr(), rows, idx.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(idx.cpu().numpy(), got.argmax(axis=1).astype(np.int32))


def test_linear_tc_agrees_with_exact_path(cuda, pkg):
    """Same inputs through the order-exact CUDA-core GEMM: one bf16 ulp apart at most (outputs near
    zero after cancellation: within fp32 accumulation noise of the largest output)."""
    torch = cuda
    rt = pkg.runtime
    rows, K, M = 64, 1536, 2304
    g = torch.Generator(device="cpu").manual_seed(5)
    w = (torch.randn(M, K, generator=g) * 0.02).bfloat16().cuda()
    x = torch.randn(rows, K, generator=g).bfloat16().cuda()
    a = torch.zeros(rows, M, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros_like(a)
    rt.k_linear(w.data_ptr(), 0, x.data_ptr(), rows, K, M, 0, a.data_ptr())
    rt.k_linear_tc(w.data_ptr(), x.data_ptr(), rows, K, M, 0, b.data_ptr())
    torch.cuda.synchronize()
    af, bf = a.float().cpu().numpy(), b.float().cpu().numpy()
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(af), 1e-30))) - 7)
    assert (np.abs(af - bf) <= ulp + 1e-6 * np.abs(af).max()).all()
    assert (af == bf).mean() >= 0.98


def test_linear_tc_argument_checks(pkg):
    rt = pkg.runtime
    with pytest.raises(pkg.PlamoError):
        rt.k_linear_tc(1, 1, 4, 100, 64, 0, 1)  # K not a multiple of 64
    with pytest.raises(pkg.PlamoError):
        rt.k_linear_tc(1, 1, 4, 128, 64, 0, 1, splits=4)  # split partials need a workspace


def floor_of(oracle, directory, context, prompt, steps, model=None):
    """The restatement's own drift on this prompt: the larger of its reordered twin and its
    correctly rounded twin (each dot product summed exactly, rounded once)."""
    a = oracle.noise_floor(directory, context, prompt, steps, model=model)
    b = oracle.noise_floor(directory, context, prompt, steps, model=model, mode="exact")
    return {k: max(a[k], b[k]) for k in a}


def check_noise(stats, floor, factor=4.0):
    """Logits within max(north-star bound, factor x the restatement's own drift), and every greedy
    pick within that drift of the restatement's top logit. The tensor core accumulates in fp32 but
    not with a round-to-nearest after every add, so it moves more outputs across a bf16 rounding
    boundary than either twin; measured: 1.6-1.9x the floor at the reference dims after the
    512-token prefill, up to 3.0x on single lanes of the small model (short prompts, where the
    floor itself is small)."""
    rmse_tol = max(1e-2, factor * floor["rmse"])
    max_tol = max(5e-2, factor * floor["maxabs"])
    detail = dict(floor=floor, rmse=[round(s["rmse"], 4) for s in stats], maxabs=[round(s["maxabs"], 3) for s in stats])
    assert max(s["rmse"] for s in stats) <= rmse_tol, detail
    assert max(s["maxabs"] for s in stats) <= max_tol, detail
    for i, s in enumerate(stats):
        assert s["same"] or s["pick_gap"] <= max_tol, (i, s)
    return dict(same=sum(s["same"] for s in stats), steps=len(stats))


def compare_gap(gpu, ora, prompt, steps):
    """compare() plus, per step, how far the GPU's greedy pick sits below the restatement's top."""
    g = gpu.prefill(prompt)
    o = ora.prefill(prompt)
    stats = []
    for i in range(steps + 1):
        lg, lo = gpu.logits(), ora.logits()
        e = lg - lo
        stats.append(dict(rmse=float(np.sqrt(np.mean(e * e))), maxabs=float(np.abs(e).max()), same=g == o,
                          pick_gap=float(lo[o] - lo[g])))
        if i == steps:
            break
        g = gpu.forward([o])
        o = ora.forward([o])
    return stats


def test_tensor_mode_tiny_prefill(cuda, pkg, oracle, tiny_dir):
    """A 70-token prefill (one call of 70 rows, so every projection runs on the tensor cores) and
    40 batch-1 steps over the KV it wrote."""
    rt = pkg.Runtime(tiny_dir, context=200)
    rt.set_tensor_gemm(True)
    ora = oracle.OracleRuntime(tiny_dir, context=200)
    prompt = pkg.synthetic.seeded_tokens(70, rt.vocab, seed=1)
    stats = compare_gap(rt, ora, prompt, 40)
    check_noise(stats, floor_of(oracle, tiny_dir, 200, prompt, 40))


def test_tensor_mode_tiny_batch(cuda, pkg, oracle, tiny_dir):
    """16 lanes (the smallest batch the tensor path takes): batched prefill and 12 batched steps
    against the restatement's Batch under teacher forcing. One lane's drift is a single sample of a
    chaotic process, so the comparison is over the population: the mean logit RMSE over all lanes
    and steps against the mean drift of the restatement's twins on the same prompts, and every
    logit and greedy pick against the largest drift the twins show."""
    context = 160
    rt = pkg.Runtime(tiny_dir, context=context)
    rt.set_tensor_gemm(True)
    ora = oracle.OracleRuntime(tiny_dir, context=context)
    lanes, steps = 16, 12
    prompts = [pkg.synthetic.seeded_tokens(8 + 3 * i, rt.vocab, seed=40 + i) for i in range(lanes)]
    b = pkg.Batch(rt, lanes=lanes)
    ob = oracle.OracleBatch(ora, lanes=lanes)
    g = b.prefill(prompts)
    o = ob.prefill(prompts)
    rmse, maxabs, gaps = [], [], []
    for step in range(steps + 1):
        for lane in range(lanes):
            lg = b.logits(lane)
            lo = oracle.bf16_to_f32(ob.logits_bits(lane))
            e = lg - lo
            rmse.append(float(np.sqrt(np.mean(e * e))))
            maxabs.append(float(np.abs(e).max()))
            gaps.append(float(lo[o[lane]] - lo[g[lane]]))
        if step == steps:
            break
        g = b.step(o)
        o = ob.step(o)
    model = oracle.Model(tiny_dir)
    floors = [floor_of(oracle, tiny_dir, context, p, steps, model=model) for p in prompts]
    floor_mean = float(np.mean([f["rmse_mean"] for f in floors]))
    floor_max = max(f["maxabs"] for f in floors)
    detail = dict(rmse_mean=float(np.mean(rmse)), floor_mean=floor_mean, maxabs=max(maxabs), floor_maxabs=floor_max)
    assert np.mean(rmse) <= max(1e-2, 4.0 * floor_mean), detail
    assert max(maxabs) <= max(5e-2, 4.0 * floor_max), detail
    assert max(gaps) <= max(5e-2, 4.0 * floor_max), detail


@pytest.mark.slow
def test_tensor_mode_reference_dims_prefill(cuda, pkg, oracle, reference_dir):
    """BASELINE config 2 shape: the 512-token prompt prefilled on the tensor cores, then 4 batch-1
    steps, against the restatement's own drift on the same prompt and steps."""
    prompt = pkg.synthetic.seeded_tokens(512, 107520, seed=1)
    rt = pkg.Runtime(reference_dir, context=1024)
    rt.set_tensor_gemm(True)
    ora = oracle.OracleRuntime(reference_dir, context=1024)
    stats = compare_gap(rt, ora, prompt, 4)
    del ora
    check_noise(stats, floor_of(oracle, reference_dir, 1024, prompt, 4))


@pytest.mark.slow
def test_tensor_mode_layer0_cache_against_float64(cuda, pkg, oracle, reference_dir):
    """The tcgen05 path's contract at the model level, element by element: after the 512-token
    prompt prefilled on the tensor cores at the reference dims, layer 0's value cache holds
    bf16(h . W_v) for every row, where h is the pre-mixer norm of the embedding rows (no earlier
    tensor-core result feeds it). Against that product in float64 every cached value must lie
    within one bf16 ulp and nearly all must be identical, so a wrong row, lane or tile mapping of
    the qkv GEMM (or its epilogue) fails here, although the logits downstream are only held to the
    accumulation-order drift. The key cache (QK-norm of the same GEMM's key rows, stored
    unrotated) is held to the bound after its extra roundings (Kernels.metal:223-259)."""
    prompt = np.array(pkg.synthetic.seeded_tokens(512, 107520, seed=1))
    rt = pkg.Runtime(reference_dir, context=1024)
    rt.set_tensor_gemm(True)
    rt.prefill(list(prompt))
    gk, gv = rt.debug_kv(0)
    model = oracle.Model(reference_dir)
    t = model.tensors
    emb = oracle.bf16_to_f32(t["model.embed_tokens.weight"][prompt])
    h, _ = oracle.norm(t["model.layers.layers.0.pre_mixer_norm.weight"], emb, 1.0)
    w = oracle.bf16_to_f32(t["model.layers.layers.0.mixer.qkv_proj.weight"])
    exact = h.astype(np.float64) @ w.astype(np.float64).T  # [512, 2304]
    rounded = oracle.bf16_to_f32(oracle.f32_to_bf16(exact.astype(np.float32)))

    def excess(got_bits, ref, n_ulps, slack):
        """How far each cached value lies outside n_ulps bf16 ulps of `ref` plus an absolute
        slack for results that cancel (their fp32 accumulation error is absolute, not relative);
        > 0 flags an element. A mis-mapped row or lane is off by O(1)."""
        got = oracle.bf16_to_f32(got_bits).astype(np.float64)
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
        return np.abs(got - ref) - (n_ulps * ulp + slack)

    v_ref = rounded[:, 2176:2304]
    v_got = gv.reshape(-1, 128)[:512]
    same_v = float(np.mean(oracle.bf16_to_f32(v_got) == v_ref))
    ev = excess(v_got, exact[:, 2176:2304], 1.0, 1e-4)
    assert ev.max() <= 0, (np.unravel_index(ev.argmax(), ev.shape), float(ev.max()))
    assert same_v >= 0.995, same_v
    # keys: per-row RMSNorm with k_norm + 1 of the bf16 GEMM rows (layer 0 is local: unrotated)
    k_ref, _ = oracle.norm(t["model.layers.layers.0.mixer.k_norm.weight"], rounded[:, 2048:2176].astype(np.float32), 1.0)
    k_got = oracle.bf16_to_f32(gk.reshape(-1, 128)[:512])
    same_k = float(np.mean(k_got == k_ref))
    ek = excess(gk.reshape(-1, 128)[:512], k_ref.astype(np.float64), 2.0, 1e-3)
    assert ek.max() <= 0, (np.unravel_index(ek.argmax(), ek.shape), float(ek.max()))
    assert same_k >= 0.99, same_k
    print(f"layer-0 cache: values identical {same_v:.5f}, keys identical {same_k:.5f}")
