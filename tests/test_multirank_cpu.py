"""The multi-GPU path on CPU: two `gloo` ranks split a set of independent segments the way
bench.py does on GPUs (one contiguous block per rank, no exchange on the data path), each decodes
its block with the CPU restatement, and the whole-job figures come from the slowest rank.

What is checked:
- the blocks are disjoint and cover every segment;
- every rank's greedy ids equal a single-process decode of the same segments;
- the reported rate is the units of all ranks over the slowest rank's time (the MAX reduction the
  GPU run performs with NCCL is done here with gloo).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

SEGMENTS = 6
PROMPT = 24
STEPS = 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode(model_dir, indices):
    """Greedy ids of the given segments, decoded together with the CPU restatement."""
    from conftest import load_oracle, load_package
    import bench
    o, p = load_oracle(), load_package()
    rt = o.OracleRuntime(model_dir, context=PROMPT + STEPS + 8)
    if not indices:
        return []
    b = o.OracleBatch(rt, lanes=len(indices))
    prompts = [p.synthetic.seeded_tokens(PROMPT, rt.vocab, seed=bench.segment_seed(k)) for k in indices]
    ids = [b.prefill(prompts)]
    for _ in range(STEPS):
        ids.append(b.step(ids[-1]))
    return [[step[i] for step in ids] for i in range(len(indices))]


def _rank(rank, world, port, model_dir, out_dir):
    import sys
    from pathlib import Path
    here = Path(__file__).resolve().parent
    sys.path[:0] = [str(here), str(here.parent)]
    import time
    import torch
    import torch.distributed as dist
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        block = list(bench.segment_block(rank, world, SEGMENTS))
        t0 = time.perf_counter()
        ids = _decode(model_dir, block)
        elapsed = torch.tensor([time.perf_counter() - t0 + 0.01 * rank], dtype=torch.float64)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        units = torch.tensor([len(block) * (STEPS + 1)], dtype=torch.int64)
        dist.all_reduce(units, op=dist.ReduceOp.SUM)
        np.save(Path(out_dir) / f"rank{rank}.npy",
                np.array(dict(block=block, ids=ids, max_s=float(elapsed.item()), units=int(units.item()),
                              rate=bench.aggregate_rate(len(block) * (STEPS + 1), world, float(elapsed.item()))),
                         dtype=object))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_split_segments(tiny_dir, tmp_path):
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp
    import bench
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, world, port, str(tiny_dir), str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [np.load(tmp_path / f"rank{r}.npy", allow_pickle=True).item() for r in range(world)]
    blocks = [r["block"] for r in res]
    assert sorted(sum(blocks, [])) == list(range(SEGMENTS))
    assert not set(blocks[0]) & set(blocks[1])
    single = _decode(tiny_dir, list(range(SEGMENTS)))
    assert sum((r["ids"] for r in res), []) == single
    # every rank reports the same whole-job figures: all units over the slowest rank's time
    assert res[0]["units"] == res[1]["units"] == SEGMENTS * (STEPS + 1)
    assert res[0]["max_s"] == res[1]["max_s"]
    assert res[0]["rate"] == pytest.approx(world * len(blocks[0]) * (STEPS + 1) / res[0]["max_s"])
    assert bench.aggregate_rate(10, 4, 2.0) == 20.0
