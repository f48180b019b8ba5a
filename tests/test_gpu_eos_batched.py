"""The frame's EOS projection on the tensor cores, at 1, 64 and 512 sessions
with EOS enabled in one frame call.

The frame gathers the enabled sessions' conditional / unconditional hidden
rows and multiplies them by the whole [16 x 2024][768] final projection in one
tcgen05 GEMM whose epilogue forms the guided logits with the reference's
roundings and keeps, per session and position, the largest code logit and the
EOS logit (local_ar_plugins.cu:1372-1495).  Each session's end_frame_index must
equal the C oracle's decision (oracle/csrc/oracle.c eos_guided + eos decision)
on the same hidden rows and the GPU's own tokens.

The EOS bias is raised so that about half of the positions sit near the
decision boundary and the three outcomes (-1, 0, 1) all occur.  The GPU sums
the 768-long dot products in another order than the oracle, so a position
whose guided EOS logit and best code logit are within 2 bf16 ulps of each
other may legitimately decide either way: sessions whose decision hinges on
such a near-tie are reported and skipped (at most 10% of the checked ones).
"""
import numpy as np
import pytest
import torch

from magpie_tts_rt_b200.model import EMBED, POSITIONS, SHAPE_BASELINE, VOCAB, make_weights
from oracle import sampler as S

from test_gpu_frame import bits, run_gpu

pytestmark = pytest.mark.gpu

_cache = {}


def eos_weights():
    if "w" not in _cache:
        w = make_weights(SHAPE_BASELINE, seed=41, dtype=torch.bfloat16, profile="parity", with_final=True)
        fb = w.final_b.view(POSITIONS, VOCAB)
        fb[:8, S.EOS_ID] += 4.0   # frame 0 positions: EOS wins for some sessions
        fb[8:, S.EOS_ID] += 4.5   # frame 1 positions: a little more often
        _cache["w"] = w
    return _cache["w"]


def decide(guided, tokens):
    """Oracle decision plus whether it hinges on a near-tie (2 bf16 ulps)."""
    votes, fragile = [False, False], [False, False]
    for p in range(POSITIONS):
        eos = float(guided[p, 2016])  # compact rows: codes 0..2015, then EOS
        best = float(np.max(guided[p, :2016]))
        frame = p // 8
        if tokens[p] == S.EOS_ID:
            votes[frame] = True
            continue
        if eos > best:
            votes[frame] = True
        if abs(eos - best) <= 2.0 * 2.0 ** -7 * max(abs(eos), abs(best), 1e-30):
            fragile[frame] = True
    end = 0 if votes[0] else (1 if votes[1] else -1)
    # the decision is fragile if a frame's vote can flip and that changes the result
    hinge = (fragile[0]) or (not votes[0] and fragile[1])
    return end, hinge


@pytest.mark.parametrize("n_enabled,cfg", [(1, True), (64, True), (512, True), (64, False)])
def test_frame_eos_projection_batched(n_enabled, cfg):
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    w = eos_weights()
    n = n_enabled + 8
    eng = LocalArEngine(w, max_streams=n, cfg=cfg)
    g = torch.Generator().manual_seed(500 + n_enabled)
    rows = 2 if cfg else 1
    hidden = torch.randn(n, rows, EMBED, generator=g).to(torch.bfloat16)
    if not cfg:
        hidden = hidden.reshape(n, EMBED)
    # the last 8 sessions: unfinished, finished, forbid_eos (no projection for them)
    uf = np.zeros(n, bool); fi = np.zeros(n, bool); fb = np.zeros(n, bool)
    uf[n_enabled:n_enabled + 3] = True
    fi[n_enabled + 3:n_enabled + 5] = True
    fb[n_enabled + 5:] = True
    seed = np.arange(n) + 11
    counter = np.zeros(n, np.int64)
    gpu = run_gpu(eng, hidden, (uf, fi, fb), seed, counter)
    assert (gpu["invalid"] == 0).all()
    np.testing.assert_array_equal(gpu["end"][n_enabled:n_enabled + 3], -1)
    np.testing.assert_array_equal(gpu["end"][n_enabled + 3:n_enabled + 5], 0)
    np.testing.assert_array_equal(gpu["end"][n_enabled + 5:], -1)
    fw, fbias = bits(w.final_w), bits(w.final_b)
    check = list(range(n_enabled)) if n_enabled <= 64 else list(range(0, n_enabled, 8)) + [n_enabled - 1]
    outcomes, skipped = set(), []
    for s in check:
        hb = bits(hidden[s].reshape(rows, EMBED))
        if not cfg:
            hb = np.concatenate([hb, hb])
        guided = S.eos_guided(hb, fw, fbias, 2.5 if cfg else 1.0)
        exp_end, hinge = decide(guided, gpu["tokens"][s])
        assert exp_end == S.eos_end_frame(guided, S.codec_layout(gpu["tokens"][s]), False, False, False)
        outcomes.add(exp_end)
        if hinge and gpu["end"][s] != exp_end:
            skipped.append(s)
            continue
        assert gpu["end"][s] == exp_end, (s, gpu["end"][s], exp_end)
    assert len(skipped) <= max(1, len(check) // 10), skipped
    if cfg and len(check) >= 64:
        assert outcomes == {-1, 0, 1}, outcomes
