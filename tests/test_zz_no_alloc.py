"""The allocation-free GEMM entry point (hllm_b200_gemm_noalloc).

Some callers cannot let a library allocate device memory: a serving process
that fixes its device budget when it starts and admits requests against it
(hLLM's worker reserves each request's bytes before it runs), or a host that
owns all of a plugin's device memory.  For them the GEMM has a variant whose
split-K scratch is a static device array of fixed size.

This test calls it through the C ABI on two calls in a row -- the second call
finds the scratch as the first one left it -- and checks each result against
the allocating entry point (hllm_b200_gemm), within the GEMM tolerance the
kernel tests use (1e-4 for F32 outputs, 2e-3 for F16) and also bit for bit,
since both run the same plan and sum partial tiles in the same fixed order;
and against the float64 product of the same F16 inputs.  A split too large
for the static array is refused with a clear error.

It lives in a file of its own that pytest collects last, and passes both on
its own in a fresh process and after the other tests.
"""
import numpy as np
import pytest

from hllm_b200 import _lib
from tests.gpu_util import dev, f16_bits, f16_vals, host, ptr, stream, sync, torch_cuda

pytestmark = pytest.mark.gpu


def padded(a, k_pad):
    out = np.zeros((a.shape[0], k_pad), a.dtype)
    out[:, :a.shape[1]] = a
    return out


def call(fn, W, X, m, k_pad, n, pair, epi, Y, bn=0, grid=0):
    return fn(ptr(W), m, k_pad, pair, m if pair == 2 else 0, ptr(X), n, epi, ptr(Y), Y.shape[1],
              bn, grid, stream())


@pytest.mark.parametrize("m,k,n,pair,epi", [
    (2560, 4096, 64, 1, 2),    # o_proj at decode width: stream-K, residual epilogue
    (6144, 2560, 16, 1, 0),    # QKV at 16 tokens: stream-K, F32 store
    (9728, 2560, 64, 2, 3),    # gate/up pair: stream-K, SwiGLU
    (1000, 688, 33, 1, 1),     # ragged sizes, F16 store
    (40960, 2560, 64, 1, 0),   # direct plan (>= 2 tiles per SM, no scratch)
])
def test_noalloc_matches_allocating_entry_point_on_two_calls(m, k, n, pair, epi):
    torch = torch_cuda()
    L = _lib.lib()
    rng = np.random.default_rng(m + n)
    k_pad = (k + 63) // 64 * 64
    Wb = f16_bits(rng.standard_normal((m * pair, k)).astype(np.float32) * 0.03)
    Xb = f16_bits(rng.standard_normal((n, k)).astype(np.float32))
    W, X = dev(padded(Wb, k_pad)), dev(padded(Xb, k_pad))
    f16_out = epi in (1, 3)
    base = rng.standard_normal((n, m)).astype(np.float32)

    full = f16_vals(Xb).astype(np.float64) @ f16_vals(Wb).astype(np.float64).T
    if epi == 3:
        g, u = full[:, :m], full[:, m:]
        exact, tol64 = g / (1.0 + np.exp(-g)) * u, 3e-3
    elif epi == 2:
        exact, tol64 = base + full, 1e-4
    else:
        exact, tol64 = full, 2e-3 if f16_out else 1e-4

    def fresh():
        if f16_out:
            return torch.zeros((n, m), dtype=torch.int16, device="cuda")
        return dev(base.copy())

    def read(Y):
        return f16_vals(host(Y, np.uint16)) if f16_out else host(Y)

    Y_ref = fresh()
    _lib.check(call(L.hllm_b200_gemm, W, X, m, k_pad, n, pair, epi, Y_ref))
    sync()
    expected = read(Y_ref)
    np.testing.assert_allclose(expected, exact, rtol=tol64, atol=tol64)
    tol = 2e-3 if f16_out else 1e-4
    for _ in range(2):
        Y = fresh()
        _lib.check(call(L.hllm_b200_gemm_noalloc, W, X, m, k_pad, n, pair, epi, Y))
        sync()
        got = read(Y)
        np.testing.assert_allclose(got, expected, rtol=tol, atol=tol)
        assert np.array_equal(got, expected)
        np.testing.assert_allclose(got, exact, rtol=tol64, atol=tol64)


def test_noalloc_refuses_a_split_beyond_its_static_scratch():
    torch = torch_cuda()
    L = _lib.lib()
    m, k, n = 2560, 4096, 256
    W = torch.zeros((m, k), dtype=torch.float16, device="cuda")
    X = torch.zeros((n, k), dtype=torch.float16, device="cuda")
    Y = torch.zeros((n, m), dtype=torch.float32, device="cuda")
    st = call(L.hllm_b200_gemm_noalloc, W, X, m, k, n, 1, 0, Y, bn=256, grid=148)
    assert st == _lib.RESOURCE_EXHAUSTED
    assert "at most" in _lib.last_error()
