"""bench.py's host-side arithmetic, without a GPU: the prefill FLOP count against the closed form
of the reference dims (2 x non-head linear params x tokens + 8192 FLOP per visible key, layer and
token + the last row's lm_head), the segment partition and the whole-job rate."""
import pytest

import bench


def test_prefill_flop_closed_form():
    T = 512
    linear = 16 * 34_996_224  # per-layer qkv + o + gate_up + down at d 1536 / F 6144 / 16 q-heads + 1 kv-head
    head = 165_150_720
    visible = 16 * T * (T + 1) // 2  # every layer sees every earlier key below the 2048 window
    want = 2 * linear * T + 8192 * visible + 2 * head
    assert bench.prefill_flop(T) == pytest.approx(want, rel=0, abs=0.5)
    assert round(bench.prefill_flop(T) / 1e9, 1) == 590.9


def test_prefill_flop_window():
    # past the 2048-token window only the two global layers keep growing
    T = 3000
    local = sum(min(t + 1, 2048) for t in range(T))
    full = T * (T + 1) // 2
    want = 2 * (725_090_304 - 165_150_720) * T + 8192 * (14 * local + 2 * full) + 2 * 165_150_720
    assert bench.prefill_flop(T) == pytest.approx(want, rel=0, abs=0.5)


def test_segment_partition_and_rate():
    for world in (1, 2, 4, 8):
        blocks = [list(bench.segment_block(r, world, 256)) for r in range(world)]
        assert sorted(sum(blocks, [])) == list(range(256))
        assert all(len(b) == 256 // world for b in blocks)
    assert bench.segment_seed(7) == 1007
    assert bench.aggregate_rate(32 * 512, 8, 2.0) == 8 * 32 * 512 / 2.0
