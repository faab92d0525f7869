"""Tensor mode: a tcgen05 projection whose K is split over several CTAs leaves its fp32 partials to
the kernel that reads its output (k_qkv after q/k/v, the norms after o_proj and down_proj), which
adds them in split order itself instead of reading the bf16 output of a separate finish launch.
The sums are the same, so the results must be the same bits: a subprocess runs the same batched
prefill and steps with PLAMO_SPLIT_FINISH=1 (the finish launches kept), and every lane's logits
must equal the default path's. Tiny dims split o_proj and down_proj; the GQA example dims (d 2048,
4 KV heads) split q/k/v as well, so the value heads of k_qkv's partial path are covered.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TESTS = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("CUDA device required")
    return t


_RUN = r"""
import sys
import numpy as np
from conftest import load_package
pkg = load_package()
model, out = sys.argv[1], sys.argv[2]
rt = pkg.Runtime(model, context=160)
rt.set_tensor_gemm(3)
lanes = 32
prompts = [pkg.synthetic.seeded_tokens(20 + 3 * i, rt.vocab, seed=70 + i) for i in range(lanes)]
b = pkg.Batch(rt, lanes=lanes)
ids = b.prefill(prompts)
logits = []
for step in range(6):
    logits.append(np.stack([b.logits(l) for l in range(lanes)]))
    ids = b.step(ids)
logits.append(np.stack([b.logits(l) for l in range(lanes)]))
np.save(out, np.stack(logits).astype(np.float32))
"""


@pytest.mark.parametrize("dims", ["tiny_dir", "example_dir"])
def test_split_sums_in_consumers_match_finish_kernel(torch, request, dims, tmp_path):
    model = request.getfixturevalue(dims)
    results = []
    for name, extra in (("fused", {}), ("finish", {"PLAMO_SPLIT_FINISH": "1"})):
        env = dict(os.environ)
        env.pop("PLAMO_SPLIT_FINISH", None)
        env.update(extra)
        out = tmp_path / f"{name}.npy"
        p = subprocess.run([sys.executable, "-c", _RUN, str(model), str(out)], cwd=TESTS, env=env,
                           capture_output=True, text=True, timeout=600)
        assert p.returncode == 0, p.stderr[-2000:]
        results.append(np.load(out))
    assert results[0].shape == results[1].shape
    assert np.isfinite(results[0]).all()
    assert np.array_equal(results[0].view(np.uint32), results[1].view(np.uint32))
