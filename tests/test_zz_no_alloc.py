"""The allocation-free FP8 linear (sa3_fp8_linear_noalloc) against the regular FP8 path.

sa3_fp8_linear_noalloc serves callers that cannot allocate device memory: a
TensorRT plugin's enqueue (TensorRT plans all device memory ahead of time),
or a host with a fixed device-memory budget. It keeps its scratch (max|x|, the
activation scale and the e4m3 copy of the activation) in a file-scope device
array instead of caller-allocated buffers. This test calls it twice in a row
through the C ABI, with different inputs (the second with a smaller max|x|,
so a maximum left over from the first call would show), and checks each result
against the existing entry points (sa3_quantize_e4m3 twice + sa3_gemm) within
the FP8 GEMM tolerance the other tests use. It also checks that an activation
beyond the stated limit is refused before anything is launched.

The file name sorts last so a run that stops at the first failure has already
run every other test.
"""
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu


def _regular_fp8_linear(x, wq, sw, bias):
    from sa3_b200 import ops

    amax = torch.zeros(1, device=x.device)
    scale = torch.zeros(1, device=x.device)
    ops.absmax(x, amax)
    xq = ops.quantize_e4m3(x, amax, scale_out=scale)
    return ops.gemm(xq, wq, a_scale=scale, b_scale=sw, bias=bias)


def _noalloc_fp8_linear(x, wq, sw, bias, out):
    from sa3_b200 import _lib

    M, K = x.shape
    N = wq.shape[0]
    rc = _lib.load().sa3_fp8_linear_noalloc(x.data_ptr(), wq.data_ptr(), sw.data_ptr(),
                                            None if bias is None else bias.data_ptr(), out.data_ptr(), M, N, K,
                                            x.stride(0), wq.stride(0), out.stride(0),
                                            torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "sa3_fp8_linear_noalloc")
    return out


def test_fp8_linear_noalloc_matches_regular_path_twice(cuda):
    g = torch.Generator().manual_seed(42)
    M, N, K = 1000, 768, 1536
    w = torch.randn(N, K, generator=g) * 0.02
    wq, sw = oq.quantize_weight_e4m3(w)
    wq, sw = wq.to(cuda), sw.to(cuda)
    bias = (torch.randn(N, generator=g) * 0.1).to(cuda)
    inputs = [(torch.randn(M, K, generator=g) * 3.0).bfloat16().to(cuda),
              (torch.randn(M, K, generator=g) * 0.5).bfloat16().to(cuda)]
    for x in inputs:
        out = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
        _noalloc_fp8_linear(x, wq, sw, bias, out)
        ref = _regular_fp8_linear(x, wq, sw, bias)
        torch.cuda.synchronize()
        err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        assert err < 5e-3, err


@pytest.mark.parametrize("strided,with_bias", [(True, True), (False, False)])
def test_fp8_linear_noalloc_strided_input_and_no_bias(cuda, strided, with_bias):
    """x as a column slice of a wider bf16 tensor (row stride > K: the e4m3 copy's stride K differs from x's),
    and a call without bias, each against the regular path."""
    g = torch.Generator().manual_seed(7)
    M, N, K = 640, 512, 1024
    wq, sw = oq.quantize_weight_e4m3(torch.randn(N, K, generator=g) * 0.02)
    wq, sw = wq.to(cuda), sw.to(cuda)
    bias = (torch.randn(N, generator=g) * 0.1).to(cuda) if with_bias else None
    wide = (torch.randn(M, K + 256, generator=g) * 2.0).bfloat16().to(cuda)
    x = wide[:, 128:128 + K] if strided else wide[:, :K].contiguous()
    assert (x.stride(0) != K) == strided
    out = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    _noalloc_fp8_linear(x, wq, sw, bias, out)
    ref = _regular_fp8_linear(x, wq, sw, bias)
    torch.cuda.synchronize()
    err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
    assert err < 5e-3, err


def test_fp8_linear_noalloc_bad_arguments_touch_nothing(cuda):
    """A weight row stride that is not a multiple of 16 bytes is refused on the host, before the scratch or
    the output is touched."""
    from sa3_b200 import _lib

    M, N, K = 64, 256, 512
    x = torch.ones(M, K, device=cuda, dtype=torch.bfloat16)
    w = torch.zeros(N, K + 8, device=cuda, dtype=torch.float8_e4m3fn)
    out = torch.full((M, N), 7.0, device=cuda, dtype=torch.bfloat16)
    rc = _lib.load().sa3_fp8_linear_noalloc(x.data_ptr(), w.data_ptr(), None, None, out.data_ptr(), M, N, K, K,
                                            K + 8, N, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == -2  # SA3_ERR_ALIGN
    assert bool((out == 7.0).all())


def test_fp8_linear_noalloc_rejects_oversize(cuda):
    from sa3_b200 import _lib

    limit = (16 << 20) - 256
    K, N = 1536, 256
    M = limit // K + 1  # one row past the scratch capacity
    x = torch.zeros(M, K, device=cuda, dtype=torch.bfloat16)
    w = torch.zeros(N, K, device=cuda, dtype=torch.float8_e4m3fn)
    out = torch.full((M, N), 7.0, device=cuda, dtype=torch.bfloat16)
    rc = _lib.load().sa3_fp8_linear_noalloc(x.data_ptr(), w.data_ptr(), None, None, out.data_ptr(), M, N, K, K, K, N,
                                            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == -5  # SA3_ERR_UNSUPPORTED, refused on the host
    assert bool((out == 7.0).all())  # nothing was launched
