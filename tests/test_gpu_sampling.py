"""GPU parity of the sampling launcher against the C oracle and the
reference's known answers (tests/plugins/local_ar_plugin_tests.cu:136-278)."""
import os

import numpy as np
import pytest
import torch

from oracle import sampler as S

pytestmark = pytest.mark.gpu

VOCAB, EMBED = 2024, 768
MAX_COUNTER = S.MAX_COUNTER


@pytest.fixture(scope="module")
def la():
    from magpie_tts_rt_b200 import local_ar
    return local_ar


def _bf(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


class Buffers:
    def __init__(self):
        d = "cuda"
        self.emb = ((torch.arange(VOCAB * EMBED) % 251).float().to(torch.bfloat16)).reshape(VOCAB, EMBED).to(d)
        self.unfinished = torch.ones(1, dtype=torch.bool, device=d)
        self.finished = torch.zeros(1, dtype=torch.bool, device=d)
        self.forbid = torch.ones(1, dtype=torch.bool, device=d)
        self.seed = torch.tensor([20260729], dtype=torch.int64, device=d)
        self.counter = torch.zeros(1, dtype=torch.int64, device=d)
        self.sampled = torch.full((1,), -1, dtype=torch.int64, device=d)
        self.next = torch.zeros(2, EMBED, dtype=torch.bfloat16, device=d)
        self.updated = torch.full((1,), -1, dtype=torch.int64, device=d)
        self.invalid = torch.full((1,), -1, dtype=torch.int32, device=d)


def run(la, b, logits_bits, uf, fi, fb, seed, counter):
    b.unfinished.fill_(bool(uf)); b.finished.fill_(bool(fi)); b.forbid.fill_(bool(fb))
    b.seed.fill_(int(seed)); b.counter.fill_(int(counter))
    lg = _bf(logits_bits).reshape(2, VOCAB).cuda()
    rc = la.launch_local_ar_sampling(lg, b.unfinished, b.finished, b.forbid, b.seed, b.counter, b.emb,
                                     b.sampled, b.next, b.updated, b.invalid)
    assert rc == 0
    torch.cuda.synchronize()
    return int(b.sampled.item()), int(b.updated.item()), int(b.invalid.item())


def test_sampling_kats(la):
    b = Buffers()
    zeros = np.zeros((2, VOCAB), np.uint16)
    tok, ctr, inv = run(la, b, zeros, 1, 0, 1, 20260729, 0)
    assert (tok, ctr, inv) == (1871, 1, 0)
    torch.testing.assert_close(b.next[0], b.emb[1871], rtol=0, atol=0)
    torch.testing.assert_close(b.next[1], b.emb[1871], rtol=0, atol=0)
    dom = S.f32_to_bf16_bits(np.full((2, VOCAB), -1000.0, np.float32))
    dom[:, 7] = S.f32_to_bf16_bits(np.array([1000.0], np.float32))[0]
    assert run(la, b, dom, 1, 0, 1, 20260729, 0)[0] == 7
    tok, _, inv = run(la, b, zeros, 0, 1, 0, 20260729, 0)
    assert tok == 2017 and inv == 0
    assert run(la, b, zeros, 1, 1, 1, 20260729, 0)[2] != 0
    _, ctr, inv = run(la, b, zeros, 1, 0, 1, -1, 0)
    assert inv != 0 and ctr == 1
    _, ctr, inv = run(la, b, zeros, 1, 0, 1, 20260729, MAX_COUNTER + 1)
    assert inv != 0 and ctr == MAX_COUNTER + 1
    nan = np.full((2, VOCAB), 0x7FC0, np.uint16)
    assert run(la, b, nan, 1, 0, 1, 20260729, 0)[2] != 0
    # null input is rejected
    assert la.launch_local_ar_sampling(None, b.unfinished, b.finished, b.forbid, b.seed, b.counter,
                                       b.emb, b.sampled, b.next, b.updated, b.invalid) == -1


def test_golden_sweep(la, golden_dir):
    z = np.load(os.path.join(golden_dir, "sampling_sweep.npz"))
    b = Buffers()
    for i in range(z["logits"].shape[0]):
        m = z["meta"][i]
        got = run(la, b, z["logits"][i], m[0], m[1], m[2], m[3], m[4])
        assert got == tuple(int(v) for v in z["result"][i]), i


def test_random_sweep_matches_oracle(la):
    rng = np.random.default_rng(7)
    b = Buffers()
    n = 600
    for i in range(n):
        scale = rng.choice([0.05, 0.5, 2.0, 8.0])
        x = rng.standard_normal((2, VOCAB)).astype(np.float32) * scale
        if i % 5 == 0:
            x = np.round(x * 4) / 4  # ties
        if i % 17 == 0:
            x[:, rng.integers(0, VOCAB, 5)] = np.inf
        bits = S.f32_to_bf16_bits(x)
        uf, fi, fb = [(0, 0, 0), (1, 0, 0), (0, 0, 1), (0, 1, 0), (1, 1, 0), (0, 1, 1), (1, 0, 1)][i % 7]
        seed = int(rng.integers(0, 1 << 32)) if i % 23 else int(rng.choice([-5, 1 << 32, (1 << 32) - 1]))
        counter = int(rng.integers(0, 1 << 30)) if i % 29 else int(rng.choice([MAX_COUNTER, MAX_COUNTER + 1, -1]))
        got = run(la, b, bits, uf, fi, fb, seed, counter)
        tok, ctr, inv = S.sample(bits[None], uf, fi, fb, seed, counter)
        exp = (int(tok[0]), int(ctr[0]), int(inv[0]))
        assert got == exp, (i, got, exp)
        torch.testing.assert_close(b.next[0], b.emb[got[0]], rtol=0, atol=0)


def test_device_log_is_correctly_rounded(la):
    from magpie_tts_rt_b200 import _lib as L
    import ctypes
    rng = np.random.default_rng(3)
    lo, hi = np.float32(6e-8).view(np.uint32), np.float32(16.7).view(np.uint32)
    bits = np.concatenate([rng.integers(lo, hi, 8_000_000, dtype=np.uint32),
                           np.arange(lo, lo + 100_000, dtype=np.uint32),
                           np.arange(np.float32(0.999).view(np.uint32), np.float32(1.0).view(np.uint32),
                                     dtype=np.uint32)])
    x = bits.view(np.float32)
    ref = np.log(x.astype(np.float64)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    assert L.lib.mtt_b200_launch_test_log(ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(yd.data_ptr()),
                                          x.size, None) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(yd.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_gumbel_clamp_endpoints(la):
    from magpie_tts_rt_b200 import _lib as L
    import ctypes
    u = torch.tensor([0.0, 0.00000006, 1.0, 0.99999994, 0.5, 1e-3], device="cuda")
    g = torch.empty_like(u)
    assert L.lib.mtt_b200_launch_test_clamped_gumbel(ctypes.c_void_p(u.data_ptr()), ctypes.c_void_p(g.data_ptr()),
                                                     6, None) == 0
    torch.cuda.synchronize()
    g = g.cpu().numpy()
    assert g[0] == g[1] and g[2] == g[3] and np.isfinite(g).all()
    for i, v in enumerate(u.cpu().numpy()):
        assert g[i] == np.float32(S.clamped_gumbel(float(v)))
