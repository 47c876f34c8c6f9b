"""The N-stage pipeline on GPUs: configuration 1 as stages 0-1 | 2-3 on two
B200s with the F16 boundary over NCCL and the sampled tokens fed back to
stage 0 (tests/gpu_pipeline_rank.py, one process per GPU).  Needs two GPUs;
skipped on a one-GPU box (the pipeline's host logic is covered on CPU by
tests/test_pipeline_cpu.py)."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_gpu_pipeline_over_nccl_matches_the_reference(tmp_path):
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    out = tmp_path / "verdict.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={port}", os.path.join(ROOT, "tests", "gpu_pipeline_rank.py"), str(out)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    verdict = json.loads(out.read_text())
    assert verdict["ok"], verdict["detail"][:10]
