"""bm_gemm_run_noalloc: the GEMM entry point that allocates no device memory.

It serves callers that cannot call cudaMalloc (device memory owned by another
allocator, no allocation allowed after start-up, or no tolerance for
cudaMalloc/cudaFree's device-wide synchronisation). Its output must match
the regular prepare/launch entry point within the suite's tolerance, on two
calls in a row (the second call reuses the shared static scratch array,
which must be cleared again). Collected last on purpose: a failure here
leaves every other test already run. It passes alone in a fresh process and
after the rest of the suite.
"""
from __future__ import annotations

import numpy as np
import pytest

RTOL, ATOL = 1e-2, 2e-3


def test_noalloc_symbol_declared_and_exported(bm):
    assert "bm_gemm_run_noalloc" in bm.header_functions()
    assert hasattr(bm.load(), "bm_gemm_run_noalloc")


def test_noalloc_rejects_bad_problems_before_any_gpu_work(bm):
    # stream 0 (legacy default): validation fails before any CUDA call
    assert bm.run_noalloc(64, 64, 64, "NN", 16, 16, 16, stream=0)[0] == bm.BM_ERR_UNSUPPORTED_LAYOUT
    assert bm.run_noalloc(0, 64, 64, "NT", 16, 16, 16, stream=0)[0] == bm.BM_ERR_INVALID_ARGUMENT
    assert bm.run_noalloc(100, 64, 64, "NT", 16, 16, 16, stream=0)[0] == bm.BM_ERR_ALIGNMENT
    assert bm.error_string(10).startswith("call needs more scratch")


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_noalloc_matches_regular_entry_point(bm, cuda, layout):
    torch = cuda
    m, n, k = 1024, 768, 512
    a, b, c_ref = bm.alloc_operands(m, n, k, layout, mode=4, seed=21)
    with bm.Gemm.from_tensors(a, b, c_ref, layout) as g:
        g.launch()
        assert g.status() == (bm.BM_OK, 0)
    ref = c_ref.double().cpu().numpy()
    tol = RTOL * np.abs(ref) + ATOL * np.sqrt(k / 4096)
    for call in range(2):
        c = torch.full((n, m), float("nan"), dtype=torch.float16, device="cuda")
        rc, bits = bm.run_noalloc(m, n, k, layout, a.data_ptr(), b.data_ptr(), c.data_ptr())
        assert (rc, bits) == (bm.BM_OK, 0), f"call {call}: rc {rc} bits {bits:#x}"
        got = c.double().cpu().numpy()
        assert np.all(np.abs(got - ref) <= tol), f"call {call}: outside tolerance"


@pytest.mark.gpu
def test_noalloc_async_then_sync_calls(bm, cuda):
    torch = cuda
    m = n = k = 512
    a, b, c1 = bm.alloc_operands(m, n, k, "TN", mode=1)
    c2 = torch.empty_like(c1)
    s = torch.cuda.Stream()
    rc, _ = bm.run_noalloc(m, n, k, "TN", a.data_ptr(), b.data_ptr(), c1.data_ptr(), stream=s,
                           wait=False)
    assert rc == bm.BM_OK
    rc, bits = bm.run_noalloc(m, n, k, "TN", a.data_ptr(), b.data_ptr(), c2.data_ptr(), stream=s)
    assert (rc, bits) == (bm.BM_OK, 0)
    s.synchronize()
    assert torch.all(c1 == float(k)).item() and torch.all(c2 == float(k)).item()
