"""GPU parity at the batch sizes the benchmark times, and over a long sequence.

`bench.py` times config 4 with 1024 / 512 / 256 / 128 sessions per GPU (1, 2,
4, 8 GPUs), config 3 with 64, and config 2 as 1000 consecutive frames of one
session.  These tests run exactly those batches through the AUTO frame path
(the one the bench takes) on the bench's own weights (seed 0, N(0, 0.02)) and
check a spread of sessions against the oracle with the criteria of
test_gpu_frame.py: logits within 1e-2 relative L2 per row of the teacher-forced
oracle, tokens / counters / invalid flags / end-frame index / next embedding
bit-exact against the C oracle sampler applied to the GPU's logits.

Flags follow config 4 at one frame (`bench.py` flag_tables): sessions whose
forced EOS frame has passed are inactive (outputs untouched), the ones forced
at this frame are `finished`, the rest `unfinished`; a few sessions have EOS
enabled (no flag set) so the EOS projection also runs at these sizes.
"""
import numpy as np
import pytest
import torch

from magpie_tts_rt_b200.model import EMBED, POSITIONS, SHAPE_BASELINE, VOCAB, make_weights
from oracle import lt_oracle
from oracle import sampler as S

from test_gpu_frame import bits, check_frame, check_logits, run_gpu

pytestmark = pytest.mark.gpu

_cache = {}


def bench_weights():
    if "w" not in _cache:
        _cache["w"] = make_weights(SHAPE_BASELINE, seed=0, dtype=torch.bfloat16, profile="baseline")
    return _cache["w"]


def spread(n, tile, want=64):
    """Sessions to check: first and last, and at least `want` more spread over
    every tile of `tile` sessions (a different offset inside each tile)."""
    tiles = (n + tile - 1) // tile
    per = max(1, -(-want // tiles))
    sel = {0, n - 1}
    for t in range(tiles):
        for j in range(per):
            s = t * tile + (7 * t + 5 * j) % tile
            if s < n:
                sel.add(s)
    return sorted(sel)


def config4_flags(n, frame=60, seed=2024):
    rng = np.random.default_rng(seed + n)
    eos = np.full(n, 10_000)
    k = max(4, n // 20)  # 5% forced EOS, as config 4
    chosen = rng.choice(n, k, replace=False)
    eos[chosen] = rng.integers(frame - 10, frame + 11, k)
    eos[chosen[:2]] = frame  # at least two finished at this frame
    eos[chosen[2:4]] = frame - 5  # and two already masked out
    active = frame <= eos
    unfinished = frame < eos
    finished = frame == eos
    forbid = np.zeros(n, bool)
    # EOS enabled (no flag) on a few active sessions, forbid_eos on a few others
    free = np.nonzero(unfinished)[0]
    unfinished[free[3::97]] = False
    forbid[free[5::89]] = True
    unfinished[free[5::89]] = False
    return active, unfinished, finished, forbid


QUAD, OCTO = 10, 11


@pytest.mark.parametrize("n,path", [(1024, 0), (512, 0), (256, 0), (128, 0), (64, 0), (512, QUAD), (1024, QUAD),
                                    (128, OCTO), (64, OCTO)],
                         ids=["1024-auto", "512-auto", "256-auto", "128-auto", "64-auto", "512-quad", "1024-quad",
                              "128-octo", "64-octo"])
def test_auto_frame_at_bench_batch(n, path):
    """The AUTO path at each bench batch, the quad kernel (explicit path) at
    config 4's one- and two-GPU batches (one wave of 4-CTA clusters at 512
    sessions, two waves at 1024), and the octo kernel at config 4's
    eight-GPU batch and config 3's."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    w = bench_weights()
    eng = LocalArEngine(w, max_streams=n, path=path)
    assert path == 0 or eng.path == path
    tile = {2: 8, 3: 8, 4: 16, 9: 16, QUAD: 16, OCTO: 16}.get(eng.path, 8)
    g = torch.Generator().manual_seed(1000 + n)
    hidden = torch.randn(n, 2, EMBED, generator=g).to(torch.bfloat16)
    active, uf, fi, fb = config4_flags(n)
    seed = np.arange(n, dtype=np.int64)
    counter = np.full(n, 16 * 60, np.int64)
    gpu = run_gpu(eng, hidden, (uf, fi, fb), seed, counter, active=active, sentinel=True)
    for s in np.nonzero(~active)[0]:
        assert (gpu["codec"][s] == -7).all() and gpu["invalid"][s] == -7 and gpu["end"][s] == -7, s
        assert gpu["counter"][s] == counter[s], s
    sel = [s for s in spread(n, tile) if active[s]]
    sel += [s for s in np.nonzero(active & ~uf & ~fi)[0] if s not in sel]  # every EOS-enabled / forbid session
    if n <= 128:
        sel = list(np.nonzero(active)[0])  # every active session
    assert len(sel) >= min(64, int(active.sum()))
    check_frame(w, hidden, (uf, fi, fb), seed, counter, gpu, streams=sorted(sel))
    assert (gpu["invalid"][active] == 0).all()
    assert (gpu["end"][fi & active] == 0).all()


def test_config2_sequence_of_240_frames():
    """Config 2's stream: one session x CFG, seed 1234, a new hidden state each
    frame, 240 consecutive frames on the latency path.  The RNG counter
    advances by 16 per frame (sequence_contract.py:95-160); every frame's
    tokens equal the oracle sampler's on the GPU's logits at that frame's
    counter, and every frame's logits match the oracle teacher-forced on the
    GPU's tokens."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    w = bench_weights()
    eng = LocalArEngine(w, max_streams=1)
    frames = 240
    g = torch.Generator().manual_seed(77)
    hidden = torch.randn(frames, 2, EMBED, generator=g).to(torch.bfloat16)
    b = StreamBatch.allocate(1)
    b.rng_seed.fill_(1234)
    b.unfinished.fill_(True)
    b.logits_out = torch.zeros(1, POSITIONS, 2, VOCAB, dtype=torch.bfloat16, device="cuda")
    logits = np.zeros((frames, POSITIONS, 2, VOCAB), np.uint16)
    tokens = np.zeros((frames, POSITIONS), np.int64)
    counters = np.zeros(frames + 1, np.int64)
    for f in range(frames):
        b.decoder_hidden.copy_(hidden[f:f + 1])
        b.forbid_eos.fill_(f < 2)
        eng.frame(b)
        torch.cuda.synchronize()
        logits[f] = bits(b.logits_out)[0]
        tokens[f] = b.codec_tokens.cpu().numpy()[0].T.reshape(-1)
        counters[f + 1] = int(b.rng_counter.item())
        assert int(b.invalid_rows.item()) == 0, f
        assert int(b.end_frame_index.item()) == -1, f
    np.testing.assert_array_equal(counters, 16 * np.arange(frames + 1))
    # tokens: the C oracle sampler on the GPU's logits, frame by frame
    for f in range(frames):
        ctr = int(counters[f])
        for p in range(POSITIONS):
            tok, c2, iv = S.sample(logits[f, p][None], True, False, f < 2, 1234, ctr, S.SamplingParams())
            assert tok[0] == tokens[f, p], (f, p)
            assert iv[0] == 0
            ctr = int(c2[0])
    # logits: the oracle teacher-forced on the GPU's tokens, all frames as one batch
    n = frames
    r = lt_oracle.run_frame(w, hidden, np.ones(n, bool), np.zeros(n, bool), np.arange(n) < 2,
                            np.full(n, 1234), counters[:-1], S.SamplingParams(), teacher_tokens=tokens,
                            record_logits=True, eos=False)
    check_logits(logits, r.logits.reshape(n, POSITIONS, 2, VOCAB), "config-2 sequence")
    # the next-frame embedding of the last frame
    emb = bits(b.next_embedding)[0]
    np.testing.assert_array_equal(emb, S.embedding_sum(bits(w.emb), tokens[-1]))
