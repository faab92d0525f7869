"""The data-parallel open on two GPUs (needs two; skipped otherwise), as child processes with
NVLS off: plamo_open_broadcast replicates rank 0's weight arena over NCCL, and a rank whose peer
never joins gets an error within the NCCL limit instead of waiting forever.

What is checked:
- both ranks, with weights received by broadcast, decode the same greedy ids as a runtime that
  read the weights from disk;
- when rank 1 fails before the collective (it never calls the open), rank 0's open fails with
  "NCCL communicator setup timed out" within PLAMO_NCCL_TIMEOUT_MS plus a margin, the aborted
  communicator leaves the device usable, and a plain open on it then decodes the same ids.
No kernel waits on another rank here: the only cross-rank steps are NCCL's own setup and
broadcast, bounded by the library's limit.
"""
from __future__ import annotations

import os
import socket
import time

import pytest

pytestmark = pytest.mark.gpu

STEPS = 8
LIMIT_MS = 3000


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, model_dir, scenario, out_dir):
    import sys
    from pathlib import Path
    here = Path(__file__).resolve().parent
    sys.path[:0] = [str(here), str(here.parent)]
    os.environ.update(NCCL_NVLS_ENABLE="0", PLAMO_NCCL_TIMEOUT_MS=str(LIMIT_MS),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    from conftest import load_package
    P = load_package()
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    result = {}
    try:
        uid = [P.Runtime.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        prompt = P.synthetic.seeded_tokens(20, 256, seed=7)
        t0 = time.perf_counter()
        try:
            if scenario == "peer-fails" and rank == 1:
                raise RuntimeError("rank 1 failed before the collective")
            rt = P.Runtime.broadcast(model_dir, 64, False, rank, uid[0], rank, world)
            ids = [rt.prefill(prompt)] + rt.decode_chain(STEPS)
            rt.close()
            result["broadcast"] = ids
        except Exception as e:  # noqa: BLE001 - the outcome is what the test checks
            result["error"] = f"{type(e).__name__}: {e}"
        result["seconds"] = time.perf_counter() - t0
        if rank == 0:  # the device is usable afterwards: a plain open decodes
            rt = P.Runtime(model_dir, 64, device=0)
            result["plain"] = [rt.prefill(prompt)] + rt.decode_chain(STEPS)
            rt.close()
        (Path(out_dir) / f"rank{rank}.txt").write_text(repr(result))
    finally:
        dist.destroy_process_group()


def _run(tmp_path, model_dir, scenario):
    import ast
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, world, port, str(model_dir), scenario, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [ast.literal_eval((tmp_path / f"rank{r}.txt").read_text()) for r in range(world)]


@pytest.fixture(scope="module")
def two_gpus():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("two CUDA devices required")


def test_broadcast_open_decodes_like_a_disk_open(two_gpus, tiny_dir, tmp_path):
    r0, r1 = _run(tmp_path, tiny_dir, "ok")
    assert "error" not in r0 and "error" not in r1, (r0, r1)
    assert r0["broadcast"] == r1["broadcast"] == r0["plain"]


def test_peer_that_never_joins_fails_the_open_in_bounded_time(two_gpus, tiny_dir, tmp_path):
    r0, r1 = _run(tmp_path, tiny_dir, "peer-fails")
    assert "NCCL communicator setup timed out" in r0.get("error", ""), r0
    assert LIMIT_MS / 1e3 <= r0["seconds"] < LIMIT_MS / 1e3 + 30, r0
    assert "rank 1 failed before the collective" in r1["error"]
    assert len(r0["plain"]) == STEPS + 1
