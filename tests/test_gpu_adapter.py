"""The B200 stage behind hLLM's own C++ runtime types (see
tests/cpp/adapter_contract.cpp): the reference's decode-batch contract and its
StageScheduler driving the backend from concurrent request threads."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BINARY = os.path.join(ROOT, "_build", "adapter_contract")

pytestmark = pytest.mark.gpu


def test_reference_scheduler_and_decode_batch_contract_over_the_c_abi():
    from tests.gpu_util import torch_cuda
    torch_cuda()
    if not os.path.exists(BINARY):
        pytest.skip("adapter contract not built (needs the reference tree at build time)")
    r = subprocess.run([BINARY], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "adapter contract: ok" in r.stdout
