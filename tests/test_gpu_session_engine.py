"""The per-GPU session engine (C++ host side, include/magpie_tts_rt_b200.h
section 6) against the same per-step sequence driven launch by launch from
Python: alignment gate -> Local AR frame, and with the Main Decoder in front
of it.  The engine's first step runs eagerly, its second is captured as a
CUDA graph and launched, later steps replay the graph; every step's codec
tokens, end-frame indices, invalid flags, RNG counters and embedding sums
must be bit-identical to the Python-driven sequence, closed slots untouched.
This replaces the reference's per-session run_local sequence
(src/runtime/synthesis_pipeline.cpp:511-569)."""
import numpy as np
import pytest
import torch

from magpie_tts_rt_b200.model import EMBED, SHAPE_BASELINE, make_weights

pytestmark = pytest.mark.gpu


def _scores(n, S, texts, gen):
    """Alignment scores with a clear peak that walks forward, bf16."""
    x = torch.randn(n, 2, S, generator=gen) * 0.1
    for s, T in enumerate(texts):
        x[s, :, min(T - 1, int(torch.randint(0, T, (1,), generator=gen)))] += 3.0
    return x.to(torch.bfloat16)


def test_session_engine_gate_and_frame_match_the_launch_sequence():
    from magpie_tts_rt_b200.local_ar import AlignmentBatch, LocalArEngine, StreamBatch
    from magpie_tts_rt_b200.session_engine import SessionEngine
    w = make_weights(SHAPE_BASELINE, seed=21, profile="parity", with_final=True)
    n, S = 6, 64
    lar = LocalArEngine(w, max_streams=n)
    opened = {0: (1234, 40), 1: (7, 5), 2: (0, 64), 4: (99, 12)}
    texts = [opened.get(s, (0, 1))[1] for s in range(n)]
    hidden = torch.zeros(n, 2, EMBED, dtype=torch.bfloat16, device="cuda")
    scores = torch.zeros(n, 2, S, dtype=torch.bfloat16, device="cuda")
    emb = torch.zeros(n, EMBED, dtype=torch.bfloat16, device="cuda")
    eng = SessionEngine(lar, n, S, decoder_hidden=hidden, alignment_scores=scores, next_embedding=emb)
    for s, (seed, T) in opened.items():
        eng.open(s, seed, T)
    eng.synchronize()
    # the same state, driven from Python
    gate = AlignmentBatch.allocate(texts, token_stride=S)
    gate.next_prior.fill_(1.0)
    fb = StreamBatch.allocate(n)
    fb.rng_seed.copy_(torch.tensor([opened.get(s, (0, 0))[0] for s in range(n)]))
    fb.active = torch.tensor([s in opened for s in range(n)], device="cuda")
    fb.end_frame_index.fill_(-1)
    fb.finished_latch = fb.finished
    gen = torch.Generator().manual_seed(3)
    for step in range(4):
        h = torch.randn(n, 2, EMBED, generator=gen).to(torch.bfloat16)
        sc = _scores(n, S, texts, gen)
        hidden.copy_(h)
        scores.copy_(sc)
        fb.decoder_hidden.copy_(h)
        gate.alignment_scores.copy_(sc)
        torch.cuda.synchronize()
        eng.step()
        gate.gate(fb)
        lar.frame(fb)
        torch.cuda.synchronize()
        codes, end, inv = eng.collect()
        np.testing.assert_array_equal(codes, fb.codec_tokens.cpu().numpy(), err_msg=f"step {step}")
        np.testing.assert_array_equal(end, fb.end_frame_index.cpu().numpy(), err_msg=f"step {step}")
        np.testing.assert_array_equal(inv, fb.invalid_rows.cpu().numpy(), err_msg=f"step {step}")
        assert torch.equal(emb, fb.next_embedding), step
        assert (inv[list(opened)] == 0).all()
        assert (codes[[3, 5]] == 0).all()  # closed slots
    # a session closed between steps is skipped from then on
    eng.close(1)
    before = eng.collect()[0][1].copy()
    eng.step()
    assert (eng.collect()[0][1] == before).all()
    eng.close_engine()


def test_session_engine_with_the_decoder_matches_the_launch_sequence():
    from magpie_tts_rt_b200.local_ar import AlignmentBatch, LocalArEngine, StreamBatch
    from magpie_tts_rt_b200.main_decoder import (CROSS_DIM, LAYERS, MainDecoderBatch, MainDecoderEngine,
                                                 make_main_decoder_weights)
    from magpie_tts_rt_b200.session_engine import SessionEngine
    n, S, cap = 3, 32, 16
    wl = make_weights(SHAPE_BASELINE, seed=0, profile="baseline", with_final=True)
    lar = LocalArEngine(wl, max_streams=n)
    wd = make_main_decoder_weights(5, positions=cap)
    dec = MainDecoderEngine(wd, max_sessions=n, token_stride=S)
    texts = [20, 32, 9]
    seeds = [11, 12, 13]
    gen = torch.Generator().manual_seed(9)
    ck = [torch.randn(LAYERS, 2, T, CROSS_DIM, generator=gen).to(torch.bfloat16).cuda() for T in texts]
    cv = [torch.randn(LAYERS, 2, T, CROSS_DIM, generator=gen).to(torch.bfloat16).cuda() for T in texts]
    cm = [torch.ones(2, T, dtype=torch.bool, device="cuda") for T in texts]
    for m in cm:
        m[1, 1:] = False
    e0 = [(torch.randn(EMBED, generator=gen) * 0.05).to(torch.bfloat16).cuda() for _ in texts]
    eng = SessionEngine(lar, n, S, decoder=dec, cache_capacity=cap)
    for s in range(n):
        eng.open(s, seeds[s], texts[s], ck[s], cv[s], cm[s], e0[s])
    eng.synchronize()
    # Python-driven reference
    db = MainDecoderBatch.allocate(n, cap=cap, token_stride=S)
    for s, T in enumerate(texts):
        db.cross_k[s, :, :, :T] = ck[s]
        db.cross_v[s, :, :, :T] = cv[s]
        db.cond_mask[s, :, :T] = cm[s]
        db.embedded[s] = e0[s]
    db.text_length.copy_(torch.tensor(texts, dtype=torch.int32))
    db.prior.fill_(1.0)
    gate = AlignmentBatch.allocate(texts, token_stride=S)
    fb = StreamBatch.allocate(n)
    fb.rng_seed.copy_(torch.tensor(seeds))
    fb.end_frame_index.fill_(-1)
    fb.finished_latch = fb.finished
    fb.decoder_hidden = db.hidden
    fb.next_embedding = db.embedded
    gate.alignment_scores = db.alignment
    gate.next_prior = db.prior
    for step in range(3):
        eng.step()
        dec.step(db)
        gate.gate(fb)
        lar.frame(fb)
        db.position += 1
        torch.cuda.synchronize()
        eng.synchronize()
        codes, end, inv = eng.collect()
        np.testing.assert_array_equal(codes, fb.codec_tokens.cpu().numpy(), err_msg=f"step {step}")
        np.testing.assert_array_equal(end, fb.end_frame_index.cpu().numpy(), err_msg=f"step {step}")
        np.testing.assert_array_equal(inv, fb.invalid_rows.cpu().numpy(), err_msg=f"step {step}")
        assert (inv == 0).all()
    eng.close_engine()
