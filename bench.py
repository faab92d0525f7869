#!/usr/bin/env python
"""Benchmark: batch-1 greedy decode of the PLaMo-3 0.8B decoder on B200.

Workload (per GPU): the reference-dims model (d 1536, 16 layers, 16 q-heads / 1 KV head, FFN 6144,
vocab 107520) with random-init weights (seed 0, normal std 0.02 in bf16, norms 1.0) written to a
model directory on the box, a 512-token seeded-uniform prompt (seed 1 + rank), prefill, then greedy
decode. One step = one decoded token (one pass of the decoder over one token, weights streamed
from HBM; the 1.45 GB of weights are far larger than the 126 MB L2, so no flush is needed).

  value  tokens/s over exactly K device-chained steps (inputs resident, each step's argmax feeds
         the next on the device), timed with CUDA events on the runtime's stream; N GPUs run
         independent replicas (weak scaling), max time over ranks, value = N*K / time.
  e2e    the same metric through the public C ABI (plamo_forward per token: host id in via a
         pinned H2D copy, next id out via D2H), wall clock per call sequence.
  roofline  the dominant kernel timed live with CUDA events around every launch: the persistent
         decode kernel (one launch per token) when it is active, else the projection GEMVs;
         algorithmic bytes = weight bytes streamed per launch.
  cpu_baseline  the CPU restatement of the same forward (oracle/, OpenMP on all host cores) on a
         bounded sample of the same workload (rank 0, N=1).
  segments  aggregate throughput of independent segments (BASELINE config 5b shape): 32 seeded
         512-token segments per GPU, batched prefill, then batched greedy decode steps (device
         time, max over ranks); reported beside the bs1 headline, not folded into `value`.
         `segments` runs the order-exact CUDA-core projections, `segments_tensor` the tcgen05
         tensor-core GEMM (plamo_set_tensor_gemm).
  prefill  the 512-token prompt prefilled on both paths (device time, median of 5, max over
         ranks), with its algorithmic FLOPs against the measured dense bf16 tensor peak.

--impl reference runs the reference arm: the reference (Swift + Metal) cannot run on Linux, so its
CPU path is the restatement in oracle/, timed on the host cores.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PROMPT = 512
# the synthetic checkpoint's .p12 archive is bound to the safetensors file beside it (opt-in)
os.environ.setdefault("PLAMO_P12_LOCAL_SOURCE", "1")


def _load(name, path, package=False):
    if name in sys.modules:
        return sys.modules[name]
    kw = {"submodule_search_locations": [str(path.parent)]} if package else {}
    spec = importlib.util.spec_from_file_location(name, path, **kw)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pkg():
    return _load("plamo_b200", REPO / "plamo3-0.8b-runtime_b200" / "__init__.py", package=True)


def oracle_mod():
    return _load("plamo_oracle", REPO / "oracle" / "oracle.py")


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm=float(d["hbm_gbs"]), bf16=float(d["bf16_tflops"]), source="measured")
    return dict(hbm=6650.0, bf16=1590.0, source="fallback")


class Clocks:
    """Samples SM clock, max clock and throttle reasons with NVML while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle"}

    def __init__(self, device: int):
        self.samples, self.reasons, self.stop_flag = [], set(), False
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            idx = device
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            if vis:
                idx = int(vis.split(",")[device])
            self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # pragma: no cover - no NVML
            self.nv = None
            self.error = str(e)

    def _run(self):
        while not self.stop_flag:
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self.stop_flag = True
        if self.nv:
            self.t.join()

    def summary(self):
        if not self.nv:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "error", "no nvml")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def ensure_model(root: Path, packed: bool, rank: int, dist) -> Path:
    P = pkg()
    d = root / "reference"
    marker = d / (".ready_packed" if packed else ".ready")
    if rank == 0 and not marker.exists():
        if not (d / ".ready").exists():
            P.synthetic.write_model(d, P.synthetic.REFERENCE, seed=0)
            (d / ".ready").write_text("ok")
        if packed:
            P.runtime.pack_p12(d)  # the library's C++ writer: pack_weights.py's archive bytes
            marker.write_text("ok")
    if dist is not None:
        dist.barrier()
    return d


def segment_block(rank: int, world: int, total: int) -> range:
    """Indices of the independent segments rank `rank` of `world` decodes: one contiguous block,
    ranks' blocks disjoint and together covering all `total` (no exchange between ranks)."""
    return range(total * rank // world, total * (rank + 1) // world)


def segment_seed(index: int) -> int:
    """Seed of segment `index`'s 512-token prompt (segment k uses seed 1000 + k)."""
    return 1000 + index


def aggregate_rate(units_per_rank: int, world: int, max_seconds: float) -> float:
    """Whole-job throughput of `world` ranks that each processed `units_per_rank` units, timed as
    the slowest rank's device time."""
    return world * units_per_rank / max_seconds


def linear_bytes(model_dir: Path, packed: bool) -> int:
    """Algorithmic weight bytes streamed per decode token by the projection GEMVs."""
    P = pkg()
    if not packed:
        return 2 * P.synthetic.REFERENCE.linear_params()
    manifest, _ = P.packing.read_p12(model_dir / "model.p12")
    total = 0
    for rec in manifest["tensors"].values():
        if "offsets" in rec:
            total += rec["offsets"][1] - rec["offsets"][0] + rec["data"][1] - rec["data"][0]
    return total


def cpu_baseline(model_dir: Path, prompt, budget_s: float, max_steps: int):
    """CPU restatement: prefill the prompt (untimed), then time decode steps for ~budget_s."""
    O = oracle_mod()
    O.set_threads(os.cpu_count() or 1)
    ora = O.OracleRuntime(model_dir, context=len(prompt) + max_steps + 8)
    nxt = ora.prefill(prompt)
    t0 = time.perf_counter()
    nxt = ora.forward([nxt])
    one = time.perf_counter() - t0
    n = max(2, min(max_steps, int(budget_s / max(one, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(n):
        nxt = ora.forward([nxt])
    el = time.perf_counter() - t0
    import platform
    cpu = platform.processor() or ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                cpu = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return dict(value=n / el, unit="tok/s", cores=O.threads(), kind="port",
                sample=f"{n} greedy decode steps at positions {len(prompt) + 1}..{len(prompt) + n} after a "
                       f"{len(prompt)}-token prefill of the reference-dims model (CPU restatement, fp32 "
                       f"accumulation, {O.threads()} OpenMP threads, {cpu})")


def run_reference(args):
    """Reference arm: the reference's CPU path (restated in oracle/) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    root = Path(args.model_root)
    model = ensure_model(root, args.packed, 0, None)
    P = pkg()
    prompt = P.synthetic.seeded_tokens(PROMPT, 107520, seed=1)
    steps = max(1, min(args.steps, args.reference_max_steps))
    O = oracle_mod()
    O.set_threads(os.cpu_count() or 1)
    ora = O.OracleRuntime(model, context=PROMPT + args.warmup + steps + 8, packed=args.packed)
    nxt = ora.prefill(prompt)
    for _ in range(args.warmup):
        nxt = ora.forward([nxt])
    t0 = time.perf_counter()
    for _ in range(steps):
        nxt = ora.forward([nxt])
    el = time.perf_counter() - t0
    value = steps / el
    line = dict(metric="decode tok/s (bs1)", value=value, unit="tok/s", n_gpus=args.gpus, steps=args.steps,
                warmup=args.warmup, ms_per_step=1e3 * el / steps, higher_is_better=True, scaling="weak",
                vs_baseline=None, dtype="bf16 weights, fp32 accumulate", data="synthetic", impl="reference",
                config=workload_config(args),
                cpu_baseline=dict(value=value, unit="tok/s", cores=O.threads(), kind="port",
                                  sample=f"{steps} of {args.steps} requested decode steps (bounded) after a {PROMPT}-token "
                                         f"prefill; CPU restatement of the reference forward"),
                e2e=dict(value=value, unit="tok/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)
    return 0


def prefill_flop(tokens: int, layers: int = 16, window: int = 2048, linear_params: int = 725_090_304,
                 head_params: int = 165_150_720) -> float:
    """Algorithmic FLOPs of prefilling `tokens` prompt tokens at the reference dims: every non-head
    projection on every token, q.k and p.v over each token's visible keys (8192 FLOP per key and
    layer: 16 heads x 128 x 2 x 2), and the lm_head on the last row."""
    attn = 0
    for layer in range(layers):
        full = layer % 8 == 7
        attn += sum(t + 1 if full else min(t + 1, window) for t in range(tokens))
    return 2.0 * (linear_params - head_params) * tokens + 8192.0 * attn + 2.0 * head_params


def kv_read_bytes(p: int, layers: int = 16, window: int = 2048, pattern: int = 8) -> int:
    """K+V bytes a decode row at position p reads (512 per visible key and layer: one KV head of
    128 bf16 keys and values); local layers see min(p + 1, window) keys, global ones p + 1."""
    n_global = layers // pattern
    return 512 * ((layers - n_global) * min(p + 1, window) + n_global * (p + 1))


def decode_row_bytes(p: int) -> int:
    """Per-row bytes of a decode step beyond the shared weights (SURVEY 8(d) formula): KV reads at
    position p, the 16 layers' KV writes, the embedding row and the bf16 logits."""
    return kv_read_bytes(p) + 16 * 512 + 3072 + 215_040


NORM_BYTES = 207_872  # every norm vector read once per step


def decode_step_bytes(weight_bytes: int, positions) -> int:
    """Algorithmic HBM bytes of one decode step over rows at `positions` (one weight pass)."""
    return weight_bytes + NORM_BYTES + sum(decode_row_bytes(p) for p in positions)


def workload_config(args):
    return {"workload": "BASELINE config 2: reference-dims PLaMo-3 0.8B (d1536 L16 H16/KV1 F6144 V107520), "
                        f"{PROMPT}-token seeded prompt, prefill then greedy bs1 decode"
                        + (" from the .p12 packed archive (config 3)" if args.packed else ", bf16 weights"),
            "prompt_tokens": PROMPT, "batch": 1, "weights": "p12" if args.packed else "bf16",
            "parallelism": f"replicas x{args.gpus} (weights broadcast by NCCL at load)" if args.gpus > 1 else "single GPU",
            "l2": "weights (1.45 GB) exceed L2 (126 MB): no flush needed"}


def kernel_case(args):
    """One projection (rows x K activations, M x K seeded weights; mode 0 plain, 1 SwiGLU, 2 logits)
    on the tcgen05 GEMM and on the order-exact CUDA-core path: CUDA-event time per call over
    --steps calls after --warmup, achieved TFLOP/s against the measured bf16 peak. Used for kernel
    profiles (a small case that ncu captures in seconds)."""
    import torch
    rows, K, M, mode = (int(v) for v in args.kernel_case.split(","))
    R = pkg().runtime
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(M, K, generator=g) * 0.02).bfloat16().cuda()
    x = torch.randn(rows, K, generator=g).bfloat16().cuda()
    y = torch.zeros(rows, M // 2 if mode == 1 else M, dtype=torch.bfloat16, device="cuda")
    keys = torch.zeros(rows, dtype=torch.int64, device="cuda")
    ws = torch.zeros(8 << 20, dtype=torch.float32, device="cuda")
    pk = peaks()
    out = dict(case=dict(rows=rows, K=K, M=M, mode=mode), flop=2.0 * rows * K * M, weight_bytes=2 * K * M)
    calls = {
        "tcgen05": lambda: R.k_linear_tc(w.data_ptr(), x.data_ptr(), rows, K, M, mode, y.data_ptr(), keys.data_ptr(),
                                         0, ws.data_ptr(), ws.numel()),
        "exact": lambda: R.k_linear(w.data_ptr(), 0, x.data_ptr(), rows, K, M, mode, y.data_ptr(), keys.data_ptr()),
    }
    for name, fn in calls.items():
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        tf = out["flop"] / us / 1e6
        out[name] = dict(us=us, tflops=tf, tensor_frac=tf / pk["bf16"], weight_gbs=out["weight_bytes"] / us / 1e3)
    print(json.dumps(out), flush=True)
    return 0


def prefill_case(args):
    """One 512-token prefill of BASELINE config 2 on one path (exact or tensor), after a warm-up
    prefill: device time of the second. A short case for kernel profiles and launch lists."""
    import torch
    P = pkg()
    model = ensure_model(Path(args.model_root), False, 0, None)
    rt = P.Runtime(model, context=PROMPT + 16)
    rt.set_tensor_gemm(args.prefill_case == "tensor")
    prompt = P.synthetic.seeded_tokens(PROMPT, rt.vocab, seed=1)
    rt.prefill(prompt)
    rt.reset()
    torch.cuda.synchronize()
    g0 = rt.gpu_seconds
    rt.prefill(prompt)
    torch.cuda.synchronize()
    print(json.dumps(dict(case="prefill", path=args.prefill_case, tokens=PROMPT, ms=1e3 * (rt.gpu_seconds - g0))), flush=True)
    return 0


def attention_case(args):
    """plamo_k_attention_rows on chunked-prefill geometry (full,cap,p0,rows: rows consecutive
    positions from p0 in 16-token chunks, a global layer when full else a local one with the
    2,048-key window): CUDA-event time per call of the CUDA-core and the tensor-core kernels over
    --steps calls after --warmup, on seeded random queries, keys and values."""
    import numpy as np
    import torch
    R = pkg().runtime
    full, cap, p0, rows = (int(v) for v in args.attention_case.split(","))
    H, W = 16, 2048
    geo, pos = [], p0
    while len(geo) < rows:
        cstart, n = pos, min(16, rows - len(geo))
        for j in range(n):
            p = cstart + j
            if full:
                geo.append((0, cstart + n, 0, p + 1))
            else:
                first = max(0, cstart - (W - 1))
                end = p - first + 1
                geo.append((first, cstart + n - first, max(0, end - W), end))
        pos += n
    g = torch.Generator().manual_seed(0)
    keys = torch.randn(cap * 128, generator=g).bfloat16().cuda()
    values = torch.randn(cap * 128, generator=g).bfloat16().cuda()
    q = torch.randn(rows * H * 128, generator=g).bfloat16().cuda()
    inv = torch.tensor([1e4 ** (-2 * i / 128) for i in range(64)], dtype=torch.float64)
    ang = (torch.arange(2064, dtype=torch.float64)[:, None] * inv[None, :]).float().double()
    cs = torch.cos(ang).float().bfloat16().view(torch.int16).int() & 0xFFFF
    sn = torch.sin(ang).float().bfloat16().view(torch.int16).int() & 0xFFFF
    table = (cs | (sn << 16)).cuda()
    tgeo = torch.tensor(np.array(geo, dtype=np.int32)).cuda()
    out = torch.zeros(rows * H * 128, dtype=torch.bfloat16, device="cuda")
    splits = max(32, (cap + 255) // 256) if full else (min(cap, 2064) + 63) // 64
    ws = torch.zeros(rows * max(splits, 16) * H * (128 * 4 + 8) + rows * 16 + (1 << 20), dtype=torch.uint8, device="cuda")
    res = dict(case=dict(full=full, cap=cap, p0=p0, rows=rows, exact_splits=splits))
    for name, tensor in (("exact", 0), ("tensor", 1)):
        fn = lambda: R.k_attention_rows(q.data_ptr(), keys.data_ptr(), values.data_ptr(), H, 1, cap, tgeo.data_ptr(), rows,
                                        full, table.data_ptr(), splits, tensor, out.data_ptr(), ws.data_ptr(), ws.numel())
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        res[name] = dict(us=e0.elapsed_time(e1) * 1e3 / args.steps)
    print(json.dumps(res), flush=True)
    return 0


def select_case(args):
    """plamo_k_select (Sampler.select on the device) over a reference-size vocabulary of seeded
    random logits with a 256-token history: CUDA-event time per call."""
    import torch
    R = pkg().runtime
    V = 107520
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(V, generator=g).bfloat16().cuda()
    hist = torch.randint(0, V, (256,), generator=g, dtype=torch.int32).cuda()
    counts = torch.zeros(V, dtype=torch.int32, device="cuda")
    flags = torch.zeros(V, dtype=torch.uint8, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    fn = lambda: R.k_select(logits.data_ptr(), V, hist.data_ptr(), 256, 1.3, 3, 0.2, 0.1, counts.data_ptr(),
                            flags.data_ptr(), key.data_ptr())
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    print(json.dumps(dict(case="select", vocab=V, history=256, us=e0.elapsed_time(e1) * 1e3 / args.steps)), flush=True)
    return 0


def measure_batch4(P, model, local, dist, args, pk, wbytes):
    """four independent 512-token segments (seeds 2000 + lane) prefilled
    together, then 2,048 batched greedy steps each, so every lane's 2,064-slot local ring wraps
    (Batch.swift:109-179, the --batch4 mode). Device time of the steps (CUDA events per call),
    wall time of the whole call sequence beside it; HBM roofline of the batched step."""
    import torch
    lanes, steps = 4, args.batch4_steps
    rt = P.Runtime(model, context=PROMPT + steps + 8, device=local)
    b = P.Batch(rt, lanes=lanes)
    prompts = [P.synthetic.seeded_tokens(PROMPT, rt.vocab, seed=2000 + lane) for lane in range(lanes)]
    p0 = b.gpu_seconds
    nxt = b.prefill(prompts)
    prefill_s = b.gpu_seconds - p0
    if dist: dist.barrier()
    torch.cuda.synchronize()
    g0, w0 = b.gpu_seconds, time.perf_counter()
    for _ in range(steps):
        nxt = b.step(nxt)
    wall = time.perf_counter() - w0
    dev = b.gpu_seconds - g0
    b.close()
    rt.close()
    t = torch.tensor([dev, wall, prefill_s], device="cuda", dtype=torch.float64)
    if dist: dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev, wall, prefill_s = (float(x) for x in t.tolist())
    nbytes = sum(decode_step_bytes(wbytes, [PROMPT + i] * lanes) for i in range(steps))
    return dict(lanes=lanes, prompt_tokens=PROMPT, steps=steps, ring_wraps=PROMPT + steps > 2064,
                decode_tok_s=lanes * steps / dev, step_ms=1e3 * dev / steps,
                e2e_tok_s=lanes * steps / wall, prefill_ms=1e3 * prefill_s,
                hbm_frac=nbytes / dev / 1e9 / pk["hbm"],
                path="order-exact CUDA-core projections (bit-identical to the restatement); one weight pass per step")


def measure_packed(P, root, local, rank, dist, args, pk, prompt):
    """the C2 decode from the lossless .p12 archive (the library's C++ packer
    writes it from the same weights; Packed.swift:12-91, Kernels.metal:23-44). Device-chained
    greedy steps after the 512-token prefill, CUDA events, max over ranks; roofline of the
    persistent kernel against the archive's streamed bytes (data regions + block tables)."""
    import torch
    d = ensure_model(root, True, rank, dist)
    steps = args.packed_steps
    rt = P.Runtime(d, context=PROMPT + args.warmup + steps + args.profile_steps + 16, packed=True, device=local)
    rt.prefill(prompt)
    rt.decode_chain(args.warmup)
    if dist: dist.barrier()
    torch.cuda.synchronize()
    g0 = rt.gpu_seconds
    rt.decode_chain(steps)
    torch.cuda.synchronize()
    t = torch.tensor([rt.gpu_seconds - g0], device="cuda", dtype=torch.float64)
    if dist: dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed = float(t.item())
    prof = rt.profile_decode(args.profile_steps)
    rt.close()
    key = "persistent" if "persistent" in prof else "gemv"
    pbytes = linear_bytes(d, True)
    per_launch_bytes = pbytes * args.profile_steps / max(1, prof[key]["launches"])
    per_launch_s = prof[key]["ms"] * 1e-3 / max(1, prof[key]["launches"])
    achieved = per_launch_bytes / per_launch_s / 1e9
    tf = REPO / "profiles" / f"{key}_decode_traffic_p12.json"
    traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch") if tf.exists() else None
    world = dist.get_world_size() if dist else 1
    return dict(steps=steps, tok_s=aggregate_rate(steps, world, elapsed), ms_per_step=1e3 * elapsed / steps,
                bytes_per_token=pbytes,
                roofline=dict(bound="hbm", kernel="k_decode_mega<packed>" if key == "persistent" else "k_gemv<packed>",
                              achieved=achieved, peak=pk["hbm"], unit="GB/s", frac=achieved / pk["hbm"],
                              traffic=traffic, bytes_per_launch=per_launch_bytes, launch_us=per_launch_s * 1e6),
                path="persistent decode from the .p12 archive, decoded in registers (ids identical to bf16)")


def measure_long(P, model, local, dist, args, pk, wbytes):
    """BASELINE config 5a: one 28,672-token prompt in a 32,768-token context (global layers keep
    the full history; split-K flash-decode), prefilled on the order-exact path and on the tcgen05
    path (device time), then greedy decode of the remaining 4,096 - 1 tokens device-chained on the
    persistent kernel: tok/s and the HBM roofline including the growing KV reads."""
    import torch
    prompt_len, context = args.long_prompt, 32768
    rt = P.Runtime(model, context=context, device=local)
    prompt = P.synthetic.seeded_tokens(prompt_len, rt.vocab, seed=5)
    out = dict(prompt_tokens=prompt_len, context=context, flop=prefill_flop(prompt_len))
    for mode in ("tensor", "exact"):  # the decode below continues from the order-exact prefill
        rt.set_tensor_gemm(mode == "tensor")
        rt.reset()
        if dist: dist.barrier()
        g0 = rt.gpu_seconds
        rt.prefill(prompt)
        t_s = rt.gpu_seconds - g0
        tt = torch.tensor([t_s], device="cuda", dtype=torch.float64)
        if dist: dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_s = float(tt.item())
        out["prefill_" + mode] = dict(ms=1e3 * t_s, tok_s=prompt_len / t_s, tflops=out["flop"] / t_s / 1e12,
                                      tensor_frac=out["flop"] / t_s / 1e12 / pk["bf16"])
    steps = context - prompt_len - 1
    if dist: dist.barrier()
    g0 = rt.gpu_seconds
    rt.decode_chain(steps)
    dev = rt.gpu_seconds - g0
    tt = torch.tensor([dev], device="cuda", dtype=torch.float64)
    if dist: dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    dev = float(tt.item())
    rt.close()
    nbytes = sum(decode_step_bytes(wbytes, [prompt_len + i]) for i in range(steps))
    out["decode"] = dict(steps=steps, positions=[prompt_len, prompt_len + steps - 1], tok_s=steps / dev,
                         ms_per_token=1e3 * dev / steps, gb_per_token=nbytes / steps / 1e9,
                         hbm_frac=nbytes / dev / 1e9 / pk["hbm"])
    return out


def measure_segment_job(P, model, local, rank, world, dist, args, pk, wbytes):
    """BASELINE config 5b, the whole fixed job: 256 independent 512-token segments (segment k seeded
    1000 + k) partitioned into contiguous blocks over the ranks (no exchange), each rank running
    waves of 32 lanes: batched prefill of the wave, then 512 batched greedy steps. Device time of
    the rank's whole job (prefill + steps), max over ranks, so the rate is strong-scaled: the same
    256 x 512 tokens whatever the GPU count. Roofline: sum of the waves' prefill FLOP at the bf16
    peak plus their decode-step bytes at the HBM peak, over the measured time."""
    import torch
    total, lanes, steps = args.job_segments, args.segment_lanes, args.job_steps
    mine = list(segment_block(rank, world, total))
    rt = P.Runtime(model, context=PROMPT + steps + 8, device=local)
    b = P.Batch(rt, lanes=lanes)
    roof_s, waves, dev = 0.0, 0, 0.0
    prompts = {k: P.synthetic.seeded_tokens(PROMPT, rt.vocab, seed=segment_seed(k)) for k in mine}
    if dist: dist.barrier()
    torch.cuda.synchronize()
    for w0 in range(0, len(mine), lanes):
        wave = mine[w0:w0 + lanes]
        b.reset()
        nxt = b.prefill([prompts[k] for k in wave])  # the batch's device clock restarts here
        for _ in range(steps - 1):
            nxt = b.step(nxt)
        dev += b.gpu_seconds
        waves += 1
        roof_s += len(wave) * prefill_flop(PROMPT) / (pk["bf16"] * 1e12)
        roof_s += sum(decode_step_bytes(wbytes, [PROMPT + i] * len(wave)) for i in range(steps - 1)) / (pk["hbm"] * 1e9)
    b.close()
    rt.close()
    t = torch.tensor([dev, roof_s], device="cuda", dtype=torch.float64)
    if dist: dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_max, roof_max = (float(x) for x in t.tolist())
    return dict(segments=total, segments_per_gpu=len(mine), lanes=lanes, waves_per_gpu=waves,
                prompt_tokens=PROMPT, new_tokens=steps, job_s=dev_max,
                segment_tok_s=total * steps / dev_max, total_tok_s=total * (PROMPT + steps) / dev_max,
                roofline_frac=roof_max / dev_max, scaling="strong (fixed 256-segment job)",
                path="order-exact CUDA-core projections (bit-identical to the restatement); tokens = greedy "
                     "tokens generated (the first comes from the prefill)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--packed", action="store_true")
    ap.add_argument("--model-root", default=os.environ.get("PLAMO_BENCH_MODELS", "/tmp/plamo_bench"))
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-steps", type=int, default=16)
    ap.add_argument("--reference-max-steps", type=int, default=64)
    ap.add_argument("--segment-lanes", type=int, default=32)
    ap.add_argument("--segment-steps", type=int, default=32)
    ap.add_argument("--prefill-reps", type=int, default=5)
    ap.add_argument("--packed-steps", type=int, default=1024, help="config 3 (.p12) decode steps (0: skip)")
    ap.add_argument("--batch4-steps", type=int, default=2048, help="config 4 decode steps per lane (0: skip)")
    ap.add_argument("--long-prompt", type=int, default=28672, help="config 5a prompt tokens (0: skip)")
    ap.add_argument("--job-segments", type=int, default=256, help="config 5b segments in the fixed job (0: skip)")
    ap.add_argument("--job-steps", type=int, default=512, help="config 5b greedy tokens per segment")
    ap.add_argument("--kernel-case", default=None,
                    help="rows,K,M,mode: time one projection on the tcgen05 GEMM and the exact GEMM, then exit")
    ap.add_argument("--prefill-case", default=None, choices=["exact", "tensor"],
                    help="one 512-token prefill on that path after a warm-up, then exit (profiles)")
    ap.add_argument("--attention-case", default=None,
                    help="full,cap,p0,rows: time the multi-row attention kernels, then exit")
    ap.add_argument("--select-case", action="store_true", help="time the device sampler, then exit")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    if args.kernel_case:
        return kernel_case(args)
    if args.prefill_case:
        return prefill_case(args)
    if args.attention_case:
        return attention_case(args)
    if args.select_case:
        return select_case(args)

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    P = pkg()
    model = ensure_model(Path(args.model_root), args.packed, rank, dist)
    context = PROMPT + 2 * (args.warmup + args.steps) + args.profile_steps + 16
    if context > 32768:
        raise SystemExit("steps too large for the 32768-token context")
    if world > 1:
        uid = [P.Runtime.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        rt = P.Runtime.broadcast(model, context, args.packed, local, uid[0], rank, world)
    else:
        rt = P.Runtime(model, context=context, packed=args.packed, device=local)
    prompt = P.synthetic.seeded_tokens(PROMPT, rt.vocab, seed=1 + rank)

    # ---- value: device-chained decode, K timed steps ---------------------------------------
    rt.prefill(prompt)
    rt.decode_chain(args.warmup)
    launches = rt.step_launches()
    if dist: dist.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    g0 = rt.gpu_seconds
    with clocks:
        rt.decode_chain(args.steps)
    torch.cuda.synchronize()
    elapsed = rt.gpu_seconds - g0
    if dist: dist.barrier()
    t = torch.tensor([elapsed], device="cuda", dtype=torch.float64)
    if dist: dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_max = float(t.item())

    # ---- roofline of the dominant kernel class, timed live ---------------------------------
    prof = rt.profile_decode(args.profile_steps)
    wbytes = linear_bytes(model, args.packed)
    # persistent path: one kernel per token streams every weight; multi-kernel path: the GEMVs
    dom_key = "persistent" if "persistent" in prof else "gemv"
    dom = prof[dom_key]
    dom_name = ("k_decode_mega (persistent decode step: every projection, attention, norms, lm_head)"
                if dom_key == "persistent" else "k_gemv (all projection GEMVs of a decode step)")
    per_launch_bytes = (wbytes * args.profile_steps) / max(1, dom["launches"])
    per_launch_s = dom["ms"] * 1e-3 / max(1, dom["launches"])
    pk = peaks()
    achieved = per_launch_bytes / per_launch_s / 1e9
    total_ms = sum(v["ms"] for v in prof.values())
    traffic = None
    tf = REPO / "profiles" / f"{dom_key}_decode_traffic{'_p12' if args.packed else ''}.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")

    # ---- e2e through the public API ---------------------------------------------------------
    rt.reset()
    nxt = rt.prefill(prompt)
    for _ in range(args.warmup):
        nxt = rt.forward([nxt])
    if dist: dist.barrier()
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        nxt = rt.forward([nxt])
    w1 = time.perf_counter()
    torch.cuda.synchronize()
    e2e_t = torch.tensor([w1 - w0], device="cuda", dtype=torch.float64)
    if dist:
        dist.barrier()
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_elapsed = float(e2e_t.item())
    bcast = rt.broadcast_seconds
    rt_arena_bytes = rt.weight_bytes
    rt.close()

    # ---- aggregate segment throughput (BASELINE config 5b shape): independent 512-token segments
    # decoded together on each GPU (batched prefill, then batched greedy steps); the steps are
    # timed with CUDA events on the runtime's stream (device time), max over ranks. Measured on the
    # order-exact CUDA-core path and with the projections on the tcgen05 tensor cores.
    def segments(tensor: bool):
        srt = P.Runtime(model, context=PROMPT + args.segment_steps + 8, device=local)
        srt.set_tensor_gemm(tensor)
        sb = P.Batch(srt, lanes=args.segment_lanes)
        segs = [P.synthetic.seeded_tokens(PROMPT, srt.vocab, seed=segment_seed(k))
                for k in segment_block(rank, world, world * args.segment_lanes)]
        p0 = sb.gpu_seconds
        nxt = sb.prefill(segs)
        prefill_s = sb.gpu_seconds - p0
        for _ in range(2):
            nxt = sb.step(nxt)
        if dist: dist.barrier()
        torch.cuda.synchronize()
        s0 = sb.gpu_seconds
        torch.cuda.nvtx.range_push("segment_steps_" + ("tensor" if tensor else "exact"))  # ncu --nvtx-include
        for _ in range(args.segment_steps):
            nxt = sb.step(nxt)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        st = torch.tensor([sb.gpu_seconds - s0, prefill_s], device="cuda", dtype=torch.float64)
        if dist: dist.all_reduce(st, op=dist.ReduceOp.MAX)
        sb.close()
        srt.close()
        return dict(lanes_per_gpu=args.segment_lanes, prompt_tokens=PROMPT, steps=args.segment_steps,
                    decode_tok_s=aggregate_rate(args.segment_lanes * args.segment_steps, world, float(st[0])),
                    step_ms=1e3 * float(st[0]) / args.segment_steps,
                    prefill_tok_s=aggregate_rate(args.segment_lanes * PROMPT, world, float(st[1])),
                    path=("tcgen05 tensor-core projections, tcgen05 prefill attention, decode-row attention on "
                          "warp-level bf16 MMAs (fp32 accumulate, within the restatement's reordering drift)"
                          if tensor else "order-exact CUDA-core projections (bit-identical to the restatement)")
                    + "; one weight pass for all lanes per step")

    seg = seg_tc = None
    if args.segment_lanes > 0:
        seg = segments(False)
        seg_tc = segments(True)

    # ---- prefill of the 512-token prompt, device time, max over ranks: the
    # order-exact path and the tcgen05 path, against the dense bf16 tensor roofline
    pre = None
    if args.prefill_reps > 0:
        prt = P.Runtime(model, context=PROMPT + 16, device=local)
        pre = dict(tokens=PROMPT, flop=prefill_flop(PROMPT))
        for mode in ("exact", "tensor"):
            prt.set_tensor_gemm(mode == "tensor")
            times = []
            for i in range(args.prefill_reps + 1):  # the first run warms up
                prt.reset()
                g0 = prt.gpu_seconds
                if i == 1:
                    torch.cuda.nvtx.range_push("prefill_" + mode)  # one timed prefill, for ncu --nvtx-include
                prt.prefill(prompt)
                if i == 1:
                    torch.cuda.nvtx.range_pop()
                if i:
                    times.append(prt.gpu_seconds - g0)
            tt = torch.tensor([sorted(times)[len(times) // 2]], device="cuda", dtype=torch.float64)
            if dist: dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t_s = float(tt.item())
            tflops = pre["flop"] / t_s / 1e12
            pre[mode] = dict(ms=1e3 * t_s, tok_s=aggregate_rate(PROMPT, world, t_s), tflops=tflops,
                             tensor_frac=tflops / pk["bf16"])
        pre["peak_tflops"] = pk["bf16"]
        pre["note"] = ("flop = 2 x non-head linear params x tokens + 8192 x visible keys per layer and token + "
                       "last-row lm_head; tensor_frac against the measured bf16 burst peak")
        prt.close()

    packed = (measure_packed(P, Path(args.model_root), local, rank, dist, args, pk, prompt)
              if args.packed_steps > 0 and not args.packed else None)
    job = measure_segment_job(P, model, local, rank, world, dist, args, pk, wbytes) if args.job_segments > 0 else None
    b4 = measure_batch4(P, model, local, dist, args, pk, wbytes) if args.batch4_steps > 0 else None
    long_ctx = measure_long(P, model, local, dist, args, pk, wbytes) if args.long_prompt > 0 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(model, prompt, args.cpu_budget, 64)

    if rank == 0:
        value = aggregate_rate(args.steps, world, elapsed_max)
        tok_bytes = wbytes
        line = dict(
            metric="decode tok/s (bs1)", value=value, unit="tok/s", n_gpus=world, steps=args.steps,
            warmup=args.warmup, ms_per_step=1e3 * elapsed_max / args.steps, higher_is_better=True, scaling="weak",
            vs_baseline=None, dtype="bf16 weights, fp32 accumulate", data="synthetic (seeded random-init weights and ids)",
            config=workload_config(args),
            e2e=dict(value=world * args.steps / e2e_elapsed, unit="tok/s", h2d_bytes_per_step=24, d2h_bytes_per_step=4),
            gpu_launches=launches * args.steps,
            roofline=dict(bound="hbm", kernel=dom_name, achieved=achieved,
                          peak=pk["hbm"], unit="GB/s", frac=achieved / pk["hbm"], traffic=traffic,
                          peak_source=pk["source"], bytes_per_launch=per_launch_bytes,
                          launch_us=per_launch_s * 1e6,
                          step_hbm_frac=(tok_bytes / (elapsed_max / args.steps)) / 1e9 / pk["hbm"],
                          class_share={k: round(v["ms"] / total_ms, 4) for k, v in prof.items()}),
            clocks=clocks.summary(),
        )
        if cpu:
            line["cpu_baseline"] = cpu
        if world > 1:
            line["weight_broadcast_s"] = bcast
            arena = rt_arena_bytes
            line["weight_broadcast_gbs"] = arena / bcast / 1e9 if bcast > 0 else None
        if seg:
            line["segments"] = seg
        if seg_tc:
            line["segments_tensor"] = seg_tc
        if pre:
            line["prefill"] = pre
        if packed:
            line["packed"] = packed
        if job:
            line["segments_job"] = job
        if b4:
            line["batch4"] = b4
        if long_ctx:
            line["long"] = long_ctx
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
