"""Tensor-parallel decoder (one process per GPU; partial sums exchanged over
NVLink peer memory or over NCCL) against the unsharded
decoder on the same weights: logits within tolerance at every step, identical
tokens on every rank.  Skipped when fewer GPUs are visible."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("collective", ["p2p", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decoder_matches_single_gpu(world, collective, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29531",
           os.path.join(HERE, "tp_worker.py"), str(out), "2", collective]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    rep = json.loads(out.read_text())
    assert rep["ranks_agree"] and rep["collective"] == collective
    assert len(rep["steps"]) == 6
    for s in rep["steps"]:
        assert s["rel_err"] < 2e-3, s
