"""MagpieLayerNorm / MagpieGeluTanh / MagpieSoftmax (mode 0) drop-in kernels.

Known-answer tests of the reference (tests/plugins/local_ar_plugin_tests.cu:280-408)
bit for bit, the launchers' argument checks, and random inputs against
PyTorch's bf16 results (the reference's oracle for these plugins,
docs/engine-contracts.md:231-246): every element within one bf16 step, and
the large majority identical.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def ulp_diff(a, b):
    """Distance in bf16 steps between two bf16 tensors (same sign region)."""
    ai = bits(a).astype(np.int32)
    bi = bits(b).astype(np.int32)
    ka = np.where(ai & 0x8000, 0x8000 - (ai & 0x7FFF), 0x8000 + ai)
    kb = np.where(bi & 0x8000, 0x8000 - (bi & 0x7FFF), 0x8000 + bi)
    return np.abs(ka - kb)


def test_layer_norm_kat_and_arguments():
    from magpie_tts_rt_b200 import local_ar
    rows = 3
    x = torch.tensor([-1.0 if i % 2 == 0 else 1.0 for i in range(rows * 768)], dtype=torch.bfloat16).cuda()
    w = torch.ones(768, dtype=torch.bfloat16, device="cuda")
    out = torch.full_like(x, 9.0)
    assert local_ar.launch_layer_norm(x, w, out, rows) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(out), bits(x))
    assert local_ar.launch_layer_norm(None, w, out, rows) == -1
    assert local_ar.launch_layer_norm(x, w, out, 0) == -1
    assert local_ar.launch_layer_norm(x, w, out, 1025) == -1


def test_layer_norm_random_against_torch():
    from magpie_tts_rt_b200 import local_ar
    g = torch.Generator().manual_seed(3)
    rows = 200
    x = (torch.randn(rows, 768, generator=g) * 2 + 0.5).to(torch.bfloat16)
    w = (torch.randn(768, generator=g) * 0.3 + 1).to(torch.bfloat16)
    ref = torch.nn.functional.layer_norm(x.float(), (768,), w.float(), None, 1e-5).to(torch.bfloat16)
    xd, wd = x.cuda(), w.cuda()
    out = torch.empty_like(xd)
    assert local_ar.launch_layer_norm(xd, wd, out, rows) == 0
    torch.cuda.synchronize()
    d = ulp_diff(out.cpu(), ref)
    assert d.max() <= 1, d.max()
    assert (d == 0).mean() > 0.98


def test_gelu_kat_and_random():
    from magpie_tts_rt_b200 import local_ar
    n = 3 * 3072
    x = torch.tensor([float(i % 9 - 4) for i in range(n)], dtype=torch.bfloat16).cuda()
    out = torch.full_like(x, 9.0)
    assert local_ar.launch_gelu_tanh(x, out, n) == 0
    torch.cuda.synchronize()
    xf = x.cpu().float().numpy()
    beta, kappa = np.float32(0.7978845608028654), np.float32(0.044715)
    inner = beta * (xf + kappa * (xf * xf * xf))
    expect = torch.from_numpy((np.float32(0.5) * xf * (np.float32(1) + np.tanh(inner))).astype(np.float32))
    np.testing.assert_array_equal(bits(out), bits(expect.to(torch.bfloat16)))
    assert local_ar.launch_gelu_tanh(None, out, n) == -1
    assert local_ar.launch_gelu_tanh(x, out, 0) == -1
    assert local_ar.launch_gelu_tanh(x, out, 3072 * 512 + 1) == -1
    # random inputs against PyTorch's CUDA GELU (f32 math, bf16 store).  Where
    # 1 + tanh cancels (x < -4) the tiny results differ between tanh
    # implementations by more than a bf16 step but by less than 1e-6.
    g = torch.Generator().manual_seed(4)
    y = (torch.randn(100_000, generator=g) * 3).to(torch.bfloat16)
    yd = y.cuda()
    ref = torch.nn.functional.gelu(yd.float(), approximate="tanh").to(torch.bfloat16).cpu()
    o2 = torch.empty_like(yd)
    assert local_ar.launch_gelu_tanh(yd, o2, y.numel()) == 0
    torch.cuda.synchronize()
    a, b = o2.cpu().float().numpy(), ref.float().numpy()
    assert (np.abs(a - b) <= np.maximum(np.abs(b) * 2.0 ** -8, 1e-6)).all()
    assert (bits(o2) == bits(ref)).mean() > 0.99


@pytest.mark.parametrize("n", [1, 2, 3, 16, 17, 128, 129, 218, 467, 512])
def test_softmax_kat_uniform(n):
    from magpie_tts_rt_b200 import local_ar
    b = 3
    x = torch.zeros(b * 512, dtype=torch.bfloat16, device="cuda")
    out = torch.full_like(x, 9.0)
    assert local_ar.launch_softmax(x, out, b, n) == 0
    torch.cuda.synchronize()
    expect = torch.tensor(1.0 / n, dtype=torch.float32).to(torch.bfloat16)
    np.testing.assert_array_equal(bits(out[: b * n]), np.full(b * n, bits(expect.reshape(1))[0]))
    assert (bits(out[b * n:]) == bits(torch.tensor([9.0], dtype=torch.bfloat16))[0]).all()


def test_softmax_arguments_and_random():
    from magpie_tts_rt_b200 import local_ar
    x = torch.zeros(3 * 512, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    assert local_ar.launch_softmax(None, out, 3, 16) == -1
    assert local_ar.launch_softmax(x, out, 3, 513) == -1
    assert local_ar.launch_softmax(x, out, 0, 16) == -1
    g = torch.Generator().manual_seed(5)
    for n in (5, 16, 100, 467):
        rows = 37
        y = (torch.randn(rows, n, generator=g) * 4).to(torch.bfloat16)
        ref = torch.softmax(y.float(), dim=-1).to(torch.bfloat16)
        yd = y.cuda()
        o = torch.empty_like(yd)
        assert local_ar.launch_softmax(yd, o, rows, n) == 0
        torch.cuda.synchronize()
        d = ulp_diff(o.cpu(), ref)
        assert d.max() <= 1, (n, d.max())
