"""GPU parity of hc_fp8_gemv (the decode step's attention projections).

The reference casts its FP8-at-rest q/k/v/o weights to fp16 and calls
F.linear (engine.py:77-82, :100-123); the kernel reads the e4m3 bytes
directly.  Against an fp64 product of the same decoded weights: products are
exact, sums fp32, output rounded once to fp16."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import hc_native
    return hc_native


@pytest.mark.parametrize("rows", [1, 7, 4096, 6144, 4097])
def test_fp8_gemv_matches_fp64(N, rows):
    g = torch.Generator(device="cuda").manual_seed(rows)
    w = (torch.randn(rows, 4096, generator=g, device="cuda") * 0.02).to(torch.float8_e4m3fn)
    x = torch.randn(4096, generator=g, device="cuda").half()
    y = torch.empty(rows, dtype=torch.float16, device="cuda")
    N.check(N.lib.hc_fp8_gemv(N.ptr(w.view(torch.uint8)), None, rows, 4096, N.ptr(x), N.ptr(y), N.stream_handle()),
            "hc_fp8_gemv")
    ref = w.double() @ x.double()
    err = (y.double() - ref).abs()
    # fp16 output rounding (2^-11 relative) plus fp32 summation of 4096 terms
    assert float((err / ref.abs().clamp(min=1e-3)).max()) < 2e-3
    assert float(err.norm() / ref.norm()) < 1e-3


def test_fp8_gemv_row_scales_and_arguments(N):
    g = torch.Generator(device="cuda").manual_seed(9)
    rows = 300
    w = (torch.randn(rows, 4096, generator=g, device="cuda") * 0.02).to(torch.float8_e4m3fn)
    sc = torch.rand(rows, generator=g, device="cuda") + 0.5
    x = torch.randn(4096, generator=g, device="cuda").half()
    y = torch.empty(rows, dtype=torch.float16, device="cuda")
    N.check(N.lib.hc_fp8_gemv(N.ptr(w.view(torch.uint8)), N.ptr(sc), rows, 4096, N.ptr(x), N.ptr(y),
                              N.stream_handle()), "hc_fp8_gemv")
    ref = (w.double() @ x.double()) * sc.double()
    assert float((y.double() - ref).norm() / ref.norm()) < 1e-3
    assert N.lib.hc_fp8_gemv(N.ptr(w.view(torch.uint8)), None, rows, 2048, N.ptr(x), N.ptr(y),
                             N.stream_handle()) == N.HC_ERR_ARG
    assert N.lib.hc_fp8_gemv(N.ptr(w.view(torch.uint8)) + 8, None, rows, 4096, N.ptr(x), N.ptr(y),
                             N.stream_handle()) == N.HC_ERR_ARG
