"""Failure paths of the data-parallel open, on CPU: the library's NCCL communicator setup (the
first step of plamo_open_broadcast, run alone by plamo_debug_nccl_init) between two `gloo` ranks,
with NCCL replaced by a fake (tests/fake_nccl/fake_nccl.c, loaded through PLAMO_NCCL_LIBRARY)
whose setup completes, never completes (a peer that never joins), or fails at once.

What is checked:
- a rank whose peer never joins (the peer failed before the collective, or its setup failed) gets
  "NCCL communicator setup timed out" within the limit instead of waiting forever, and the
  communicator it was handed is aborted: none is left alive;
- a rank whose own setup fails reports NCCL's error, and no communicator is created;
- when every rank's setup completes, each communicator is destroyed again;
- every rank learns the outcome of every other rank over gloo, so no rank proceeds alone.
"""
from __future__ import annotations

import os
import shutil
import socket
import subprocess
import time

import pytest

LIMIT_MS = 400


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def fake_nccl(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    src = os.path.join(os.path.dirname(__file__), "fake_nccl", "fake_nccl.c")
    out = tmp_path_factory.mktemp("fake_nccl") / "libfake_nccl.so"
    subprocess.run([cc, "-std=c11", "-O1", "-shared", "-fPIC", src, "-o", str(out)], check=True)
    return out


def _rank(rank, world, port, lib, modes, behaviour, out_dir):
    """One rank: `behaviour` is "join" (run the communicator setup) or "fail-before" (raise before
    the collective, as a rank whose model failed to load would)."""
    import sys
    from pathlib import Path
    here = Path(__file__).resolve().parent
    sys.path[:0] = [str(here), str(here.parent)]
    os.environ.update(PLAMO_NCCL_LIBRARY=str(lib), FAKE_NCCL_MODE=modes[rank],
                      FAKE_NCCL_LOG=str(Path(out_dir) / f"fake{rank}.log"),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from conftest import load_package
    P = load_package()
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = [P.Runtime.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        t0 = time.perf_counter()
        try:
            if behaviour[rank] == "fail-before":
                raise RuntimeError("model files missing on this rank")
            P.runtime.debug_nccl_init(uid[0], rank, world, LIMIT_MS)
            outcome = "ok"
        except Exception as e:  # noqa: BLE001 - the outcome is what the test checks
            outcome = f"{type(e).__name__}: {e}"
        elapsed = time.perf_counter() - t0
        outcomes = [None] * world
        dist.all_gather_object(outcomes, (outcome, elapsed))
        (Path(out_dir) / f"rank{rank}.txt").write_text(repr(outcomes))
    finally:
        dist.destroy_process_group()


def _run(tmp_path, lib, modes, behaviour):
    import ast
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, world, port, lib, modes, behaviour, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    views = [ast.literal_eval((tmp_path / f"rank{r}.txt").read_text()) for r in range(world)]
    assert views[0] == views[1]  # every rank saw every rank's outcome
    logs = {}
    for r in range(world):
        f = tmp_path / f"fake{r}.log"
        logs[r] = tuple(int(v) for v in f.read_text().split()) if f.exists() else (0, 0, 0)
    return views[0], logs


def test_peer_that_never_joins_times_out_and_aborts(fake_nccl, tmp_path):
    pytest.importorskip("torch")
    outcomes, logs = _run(tmp_path, fake_nccl, ["never", "never"], ["join", "fail-before"])
    (o0, t0), (o1, _) = outcomes
    assert "NCCL communicator setup timed out" in o0, o0
    assert LIMIT_MS / 1e3 <= t0 < LIMIT_MS / 1e3 + 5.0, t0
    assert "model files missing" in o1
    assert logs[0] == (1, 0, 1)  # created, destroyed, aborted: nothing left alive
    assert logs[1] == (0, 0, 0)


def test_failed_setup_on_one_rank(fake_nccl, tmp_path):
    pytest.importorskip("torch")
    outcomes, logs = _run(tmp_path, fake_nccl, ["never", "error"], ["join", "join"])
    (o0, _), (o1, _) = outcomes
    assert "NCCL communicator setup timed out" in o0, o0
    assert "ncclCommInitRankConfig failed: unhandled system error (fake)" in o1, o1
    assert logs[0] == (1, 0, 1)
    assert logs[1] == (0, 0, 0)


def test_completed_setup_destroys_its_communicator(fake_nccl, tmp_path):
    pytest.importorskip("torch")
    outcomes, logs = _run(tmp_path, fake_nccl, ["ok", "ok"], ["join", "join"])
    assert [o for o, _ in outcomes] == ["ok", "ok"]
    assert logs[0] == logs[1] == (1, 1, 0)


def test_debug_nccl_init_argument_checks(pkg):
    with pytest.raises(pkg.PlamoError, match="Invalid broadcast arguments"):
        pkg.runtime.debug_nccl_init(b"\0" * 128, 2, 2, 100)
    with pytest.raises(pkg.PlamoError, match="Invalid broadcast arguments"):
        pkg.runtime.debug_nccl_init(b"\0" * 128, 0, 1, 0)
