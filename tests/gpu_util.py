"""Shared helpers for the GPU tests: device tensors (torch is plumbing only)
and calls through the C ABI."""

import numpy as np
import pytest

from hllm_b200 import _lib


def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def dev(a: np.ndarray):
    torch = torch_cuda()
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    return torch.from_numpy(a).cuda()


def host(t, dtype=None) -> np.ndarray:
    a = t.detach().cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a


def ptr(t) -> int:
    return t.data_ptr()


def stream():
    torch = torch_cuda()
    return torch.cuda.current_stream().cuda_stream


def sync():
    torch_cuda().cuda.synchronize()


def check(st):
    _lib.check(st)


def f16_bits(x: np.ndarray) -> np.ndarray:
    import oracle
    return oracle.f16_encode(x)


def f16_vals(bits: np.ndarray) -> np.ndarray:
    import oracle
    return oracle.f16_decode(bits)
