"""GPU parity of the EOS launcher (tests/plugins/local_ar_plugin_tests.cu:
1359-1399 known answers, golden cases from the reference's _reference_eos,
random cases against the C oracle) and of launch_finalize_local_step
(tests/runtime/synthesis_kernels_gpu_tests.cu:120-270)."""
import numpy as np
import pytest
import torch

from oracle import sampler as S

pytestmark = pytest.mark.gpu

POS, VOCAB, EMBED = 16, 2024, 768


@pytest.fixture(scope="module")
def la():
    from magpie_tts_rt_b200 import local_ar
    return local_ar


def _inputs(case):
    if case["weights_seed"] is None:
        w = torch.zeros(POS * VOCAB, EMBED, dtype=torch.bfloat16)
        b = torch.zeros(POS * VOCAB, dtype=torch.bfloat16)
        h = torch.zeros(2, EMBED, dtype=torch.bfloat16)
    else:
        g = torch.Generator().manual_seed(case["weights_seed"])
        w = (torch.randn(POS * VOCAB, EMBED, generator=g) * 0.02).to(torch.bfloat16)
        b = (torch.randn(POS * VOCAB, generator=g) * 0.02).to(torch.bfloat16)
        h = torch.randn(2, EMBED, generator=g).to(torch.bfloat16)
    b = b.clone()
    for idx, val in case["bias_edits"]:
        b[idx] = val
    return h, w, b


def run_eos(la, h, w, b, codes, uf, fi, fb):
    d = "cuda"
    ws = torch.empty(la.local_ar_eos_workspace_size(), dtype=torch.uint8, device=d)
    out = torch.full((1,), -2, dtype=torch.int32, device=d)
    flag = lambda v: torch.tensor([bool(v)], device=d)
    rc = la.launch_local_ar_eos(h.to(d), torch.as_tensor(codes, dtype=torch.int64).reshape(1, 8, 2).to(d),
                                flag(uf), flag(fi), flag(fb), w.to(d), b.to(d), ws, out)
    assert rc == 0
    torch.cuda.synchronize()
    return int(out.item())


def test_eos_golden_cases(la, golden):
    for case in golden["eos_cases"]:
        h, w, b = _inputs(case)
        got = run_eos(la, h, w, b, case["codes"], case["unfinished"], case["finished"], case["forbid_eos"])
        assert got == case["end_frame"], case["name"]


def test_eos_random_vs_oracle(la):
    rng = np.random.default_rng(5)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    for k in range(6):
        g = torch.Generator().manual_seed(500 + k)
        w = (torch.randn(POS * VOCAB, EMBED, generator=g) * 0.03).to(torch.bfloat16)
        b = (torch.randn(POS * VOCAB, generator=g) * 0.5).to(torch.bfloat16)
        h = torch.randn(2, EMBED, generator=g).to(torch.bfloat16)
        # push EOS near the top at a few positions so both outcomes occur
        for p in rng.choice(16, 3, replace=False):
            b[p * VOCAB + 2017] = float(rng.choice([1.0, 2.0, 3.0]))
        codes = rng.integers(0, 2016, 16)
        if k == 3:
            codes[9] = 2017
        guided = S.eos_guided(bits(h), bits(w), bits(b))
        exp = S.eos_end_frame(guided, codes, 0, 0, 0)
        # decisions must agree unless a position is within one bf16 ulp of a tie
        margin = np.abs(guided[:, 2016] - guided[:, :2016].max(axis=1))
        got = run_eos(la, h, w, b, codes, 0, 0, 0)
        if (margin > 0.05 * np.abs(guided[:, 2016]) + 1e-3).all():
            assert got == exp, k


def test_finalize_local_step(la):
    d = "cuda"
    step = torch.arange(16, dtype=torch.int64, device=d) + 100
    agg = torch.full((8, 8), -1, dtype=torch.int64, device=d)
    ci = torch.tensor([3], dtype=torch.int32, device=d)
    ce = torch.tensor([1], dtype=torch.int32, device=d)
    si = torch.zeros(1, dtype=torch.int32, device=d)
    se = torch.zeros(1, dtype=torch.int32, device=d)
    upd = torch.tensor([48], dtype=torch.int64, device=d)
    ctr = torch.tensor([32], dtype=torch.int64, device=d)
    fin = torch.zeros(1, dtype=torch.bool, device=d)
    assert la.launch_finalize_local_step(step, agg, 4, ci, ce, si, se, upd, ctr, fin) == 0
    torch.cuda.synchronize()
    exp_agg, exp_si, exp_se, exp_ctr, exp_fin = S.finalize_local_step(
        step.cpu().numpy(), np.full((8, 8), -1, np.int64), 4, 3, 1, 48)
    np.testing.assert_array_equal(agg.cpu().numpy(), exp_agg)
    assert (int(si.item()), int(se.item()), int(ctr.item()), bool(fin.item())) == (exp_si, exp_se, exp_ctr, exp_fin)
    # bad frame offset rejected
    assert la.launch_finalize_local_step(step, agg, 3, ci, ce, si, se, upd, ctr, fin) == -1
    assert la.launch_finalize_local_step(step, agg, 8, ci, ce, si, se, upd, ctr, fin) == -1
