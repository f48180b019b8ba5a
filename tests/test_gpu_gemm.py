"""The tcgen05 GEMM (gemm_tc.cuh) that runs the Main Decoder's projections and
the EOS projection, checked through its C-ABI test hook against a plain
PyTorch fp32 product of the same bf16 inputs: Y = bf16(X W^T) within one bf16
rounding of the fp32 result (summation order differs), GELU-tanh of the
bf16-rounded product, and the split-K partial sums whose total is the fp32
product."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(x, w, y, rows, n, k, gelu=0, splits=1, partial=None):
    from magpie_tts_rt_b200 import _lib as L
    ptr = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return L.lib.mtt_b200_launch_test_gemm(ptr(x), ptr(w), ptr(y), rows, n, k, gelu, splits, ptr(partial), st)


def _inputs(rows, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) * k ** -0.5).to(torch.bfloat16)
    return x, w


def _close(got, ref):
    # one bf16 rounding of the fp32 product apart, plus summation-order noise
    err = (got.float() - ref).abs()
    tol = ref.abs() * 2.0 ** -7 + 1e-3 * ref.pow(2).mean().sqrt()
    assert bool((err <= tol).all()), float((err - tol).max())


@pytest.mark.parametrize("rows,n,k", [(512, 2304, 768), (512, 768, 768), (512, 128, 768), (512, 768, 128),
                                      (2, 128, 768), (130, 256, 128), (64, 3072, 768), (300, 384, 192)])
def test_gemm_matches_torch(rows, n, k):
    x, w = _inputs(rows, n, k, rows + n + k)
    y = torch.full((rows, n), 7.0, device="cuda", dtype=torch.bfloat16)
    assert _call(x, w, y, rows, n, k) == 0
    torch.cuda.synchronize()
    _close(y, x.float() @ w.float().t())


def test_gemm_gelu_epilogue():
    rows, n, k = 200, 3072, 768
    x, w = _inputs(rows, n, k, 5)
    y = torch.empty(rows, n, device="cuda", dtype=torch.bfloat16)
    assert _call(x, w, y, rows, n, k, gelu=1) == 0
    torch.cuda.synchronize()
    pre = (x.float() @ w.float().t()).to(torch.bfloat16).float()
    ref = torch.nn.functional.gelu(pre, approximate="tanh")
    err = (y.float() - ref).abs()
    assert bool((err <= ref.abs() * 2.0 ** -6 + 2e-3).all()), float(err.max())


@pytest.mark.parametrize("rows,splits", [(512, 4), (96, 4), (512, 2)])
def test_gemm_split_k_partials(rows, splits):
    n, k = 768, 3072
    x, w = _inputs(rows, n, k, 9 + rows)
    part = torch.full((splits, rows, n), float("nan"), device="cuda")
    assert _call(x, w, None, rows, n, k, splits=splits, partial=part) == 0
    torch.cuda.synchronize()
    kk = k // splits
    for s in range(splits):
        ref = x[:, s * kk:(s + 1) * kk].float() @ w[:, s * kk:(s + 1) * kk].float().t()
        torch.testing.assert_close(part[s], ref, rtol=1e-4, atol=1e-4)


def test_gemm_rejects_bad_shapes():
    x, w = _inputs(8, 128, 128, 1)
    y = torch.empty(8, 128, device="cuda", dtype=torch.bfloat16)
    assert _call(x, w, y, 8, 100, 128) == -1      # n not a multiple of 128
    assert _call(x, w, y, 8, 128, 96) == -1       # k not a multiple of 64
    assert _call(x, w, None, 8, 128, 128) == -1   # no output
