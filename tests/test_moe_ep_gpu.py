"""Expert-parallel MoE block (NCCL all-to-all, one process per GPU, ranks with
different token counts) against the single-GPU MoELayer on the same weights.
Skipped when fewer GPUs are visible."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_moe_ep_matches_single_gpu(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "ep.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(HERE, "moe_ep_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    rep = json.loads(out.read_text())
    assert rep["repeat_equal"]
    assert len(rep["ranks"]) == world
    for s in rep["ranks"]:
        assert s["rel_err"] < 1e-5, s
