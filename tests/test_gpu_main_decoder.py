"""GPU parity of the batched Main Decoder step against the oracle (which is
pinned bit-exact to the reference's wrapper).

Tolerance.  Twelve bf16 layers put the reference's own result about 1.2-1.3%
(relative L2 per row) from an f32 evaluation of the same bf16 weights and
inputs, and merely summing its GEMMs in another order moves it 0.6-1.2%; so
no implementation that does not repeat the CPU library's summation order
bit for bit can be held to 1e-2 of it.  The criterion is the one the Local AR
frame's test_gpu_no_further_from_exact_than_oracle uses: per output (hidden
state, alignment scores, the key / value rows written) the GPU is no further
from the f32 evaluation than 1.25 x the oracle's own distance (floor 1e-2),
and within 3e-2 of the oracle.  The cache outside the written position and
the key mask are checked exactly.
Also: ragged text lengths and positions in one batch, inactive and
out-of-range sessions, and the device-side decoder loop (Main Decoder step ->
alignment gate -> Local AR frame -> next step) sharing its buffers."""
import os

import numpy as np
import pytest
import torch

from magpie_tts_rt_b200.main_decoder import (
    LAYERS, WIDTH, MainDecoderBatch, MainDecoderEngine, make_main_decoder_weights,
)
from oracle import main_decoder as OMD

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "main_decoder.npz")
FLOOR = 1e-2      # relative L2 per row
SLACK = 1.25      # x the oracle's own distance from the f32 evaluation
TO_ORACLE = 3e-2  # relative L2 per row, GPU vs the bf16 oracle


def rel_l2(got, ref):
    g = got.float().reshape(got.shape[0], -1).double()
    r = ref.float().reshape(ref.shape[0], -1).double()
    return ((g - r).norm(dim=1) / r.norm(dim=1).clamp_min(1e-30)).max().item()


def load_session(b: MainDecoderBatch, s: int, inp: OMD.StepInputs):
    T = inp.prior.shape[1]
    b.embedded[s] = inp.embedded.cuda()
    b.position[s] = inp.position
    b.text_length[s] = T
    b.self_k[s] = inp.self_k.cuda()
    b.self_v[s] = inp.self_v.cuda()
    b.self_mask[s] = inp.self_mask.cuda()
    b.cross_k[s, :, :, :T] = inp.cross_k.cuda()
    b.cross_v[s, :, :, :T] = inp.cross_v.cuda()
    b.cond_mask[s].zero_()
    b.cond_mask[s, :, :T] = inp.cond_mask.cuda()
    b.prior[s, :, :T] = inp.prior.cuda()


def snapshot(b: MainDecoderBatch, s: int) -> OMD.StepInputs:
    T = int(b.text_length[s])
    return OMD.StepInputs(
        embedded=b.embedded[s].cpu(), position=int(b.position[s]), prior=b.prior[s, :, :T].cpu(),
        cond_mask=b.cond_mask[s, :, :T].cpu(), self_k=b.self_k[s].cpu(), self_v=b.self_v[s].cpu(),
        self_mask=b.self_mask[s].cpu(), cross_k=b.cross_k[s, :, :, :T].cpu(), cross_v=b.cross_v[s, :, :, :T].cpu())


def f32_reference(w, inp: OMD.StepInputs) -> OMD.StepOutputs:
    """The oracle's operations evaluated in f32 on the same bf16 numbers."""
    wf = type(w)(**{n: t.float() for n, t in w.tensors()})
    fields = {k: (v.float() if torch.is_tensor(v) and v.dtype == torch.bfloat16 else v)
              for k, v in inp.__dict__.items()}
    return OMD.step(wf, OMD.StepInputs(**fields))


def close(got, ref, exact, what):
    """got (GPU), ref (bf16 oracle), exact (f32): rows of each output."""
    d_ref = rel_l2(ref, exact)
    d_got = rel_l2(got, exact)
    assert d_got <= max(FLOOR, SLACK * d_ref), f"{what}: GPU {d_got:.4g} vs oracle {d_ref:.4g} from f32"
    assert rel_l2(got, ref) <= TO_ORACLE, f"{what}: GPU vs oracle {rel_l2(got, ref):.4g}"


def check_session(b: MainDecoderBatch, s: int, inp: OMD.StepInputs, ref: OMD.StepOutputs, w, what=""):
    T = inp.prior.shape[1]
    p = inp.position
    exact = f32_reference(w, inp)
    assert int(b.status[s]) == 0, what
    close(b.hidden[s].cpu(), ref.hidden, exact.hidden, what + " hidden")
    close(b.alignment[s, :, :T].cpu(), ref.alignment, exact.alignment, what + " alignment")
    k_new = b.self_k[s, :, :, :, p].reshape(LAYERS * 2, WIDTH).cpu()
    v_new = b.self_v[s, :, :, :, p].reshape(LAYERS * 2, WIDTH).cpu()
    close(k_new, ref.k_new.reshape(-1, WIDTH), exact.k_new.reshape(-1, WIDTH), what + " k_new")
    close(v_new, ref.v_new.reshape(-1, WIDTH), exact.v_new.reshape(-1, WIDTH), what + " v_new")
    # the rest of the cache is untouched, the mask gains the position
    keep = torch.ones(b.cap, dtype=torch.bool)
    keep[p] = False
    assert torch.equal(b.self_k[s][:, :, :, keep].cpu(), inp.self_k[:, :, :, keep]), what
    assert torch.equal(b.self_v[s][:, :, :, keep].cpu(), inp.self_v[:, :, :, keep]), what
    mask = inp.self_mask.clone()
    mask[:, p] = True
    assert torch.equal(b.self_mask[s].cpu(), mask), what


@pytest.fixture(scope="module")
def golden_engine():
    z = np.load(GOLDEN)
    cap = int(z["cap"])
    w = make_main_decoder_weights(int(z["weight_seed"]), positions=cap)
    return z, w, MainDecoderEngine(w, max_sessions=8, token_stride=512)


def test_golden_steps_in_one_batch(golden_engine):
    """The four golden steps (text lengths 40 / 128 / 7 / 512, positions 300 /
    466 / 218 / 350) as four sessions of one launch, against the reference
    wrapper's own outputs."""
    z, w, eng = golden_engine
    cap = int(z["cap"])
    b = MainDecoderBatch.allocate(4, cap=cap, token_stride=512)
    cases = []
    for i in range(4):
        seed, T, pos = (int(v) for v in z[f"c{i}_case"])
        inp = OMD.make_step_inputs(seed, T, pos, cap)
        load_session(b, i, inp)
        cases.append(inp)
    eng.step(b)
    torch.cuda.synchronize()

    def f(bits):
        return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)

    for i, inp in enumerate(cases):
        ref = OMD.StepOutputs(hidden=f(z[f"c{i}_hidden"]), alignment=f(z[f"c{i}_alignment"]),
                              k_new=f(z[f"c{i}_k_new"]), v_new=f(z[f"c{i}_v_new"]))
        check_session(b, i, inp, ref, w, f"golden case {i}")


def test_ragged_batch_inactive_and_out_of_range(golden_engine):
    z, w, eng = golden_engine
    cap = int(z["cap"])
    n = 8
    rng = np.random.default_rng(5)
    b = MainDecoderBatch.allocate(n, cap=cap, token_stride=512)
    cases = {}
    for s in range(n):
        T = int(rng.integers(1, 513))
        pos = int(rng.integers(0, cap))
        inp = OMD.make_step_inputs(100 + s, T, pos, cap)
        load_session(b, s, inp)
        cases[s] = inp
    b.active = torch.ones(n, dtype=torch.bool, device="cuda")
    b.active[3] = False
    b.position[5] = cap  # out of range: status 1, nothing written for it
    b.status.fill_(-7)
    b.hidden.fill_(7.0)
    eng.step(b)
    torch.cuda.synchronize()
    for s, inp in cases.items():
        if s == 3:
            assert int(b.status[s]) == -7 and bool((b.hidden[s] == 7.0).all())
            continue
        if s == 5:
            assert int(b.status[s]) == 1 and bool((b.hidden[s] == 7.0).all())
            assert torch.equal(b.self_k[s].cpu(), inp.self_k)
            continue
        check_session(b, s, inp, OMD.step(w, inp), w, f"session {s}")


def test_device_decoder_loop():
    """Three decoder steps with every buffer on the device and shared: the
    decoder writes the hidden state the Local AR frame reads and the
    alignment scores the gate reads; the gate writes the prior the next step
    reads and the frame's unfinished / forbid_eos; the frame writes the
    embedding sum the next step reads.  Each stage is checked against its
    oracle on the inputs it actually received."""
    from magpie_tts_rt_b200.local_ar import AlignmentBatch, LocalArEngine, StreamBatch
    from magpie_tts_rt_b200.model import SHAPE_BASELINE, make_weights
    from oracle import alignment as A
    n, cap, S = 4, 300, 64
    wd = make_main_decoder_weights(3, positions=cap)
    dec = MainDecoderEngine(wd, max_sessions=n, token_stride=S)
    wl = make_weights(SHAPE_BASELINE, seed=21, dtype=torch.bfloat16, profile="parity", with_final=False)
    lar = LocalArEngine(wl, max_streams=n)
    db = MainDecoderBatch.allocate(n, cap=cap, token_stride=S)
    T = [12, 40, 64, 33]
    for s in range(n):
        load_session(db, s, OMD.make_step_inputs(200 + s, T[s], 220 + s, cap))
    gate = AlignmentBatch.allocate(T, token_stride=S)
    fb = StreamBatch.allocate(n)
    fb.rng_seed.copy_(torch.arange(n))
    fb.end_frame_index.fill_(-1)
    # shared buffers: no copies between the stages
    fb.decoder_hidden = db.hidden
    fb.next_embedding = db.embedded
    gate.alignment_scores = db.alignment
    gate.next_prior = db.prior
    u16 = lambda t: t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    for k in range(3):
        before = {s: snapshot(db, s) for s in range(n)}
        dec.step(db)
        torch.cuda.synchronize()
        for s in range(n):
            check_session(db, s, before[s], OMD.step(wd, before[s]), wd, f"step {k} session {s}")
        st = dict(text_length=np.array(T, np.uint32), constants=(3, 5, 6, 4), scores=u16(db.alignment),
                  counters=gate.counters.cpu().numpy().view(np.uint32).copy(),
                  last_attended=gate.last_attended.cpu().numpy().view(np.uint32).copy(), prior=u16(db.prior),
                  attended=np.zeros(n, np.int64), unfinished=np.zeros(n, bool), invalid=np.zeros(n, np.int32),
                  decoder_steps=gate.decoder_steps.cpu().numpy().copy(), forbid_eos=np.zeros(n, bool))
        gate.gate(fb)
        A.gate_step(st)
        torch.cuda.synchronize()
        assert np.array_equal(gate.attended_token_index.cpu().numpy(), st["attended"])
        assert np.array_equal(u16(db.prior), st["prior"])
        assert np.array_equal(fb.unfinished.cpu().numpy(), st["unfinished"])
        assert np.array_equal(fb.forbid_eos.cpu().numpy(), st["forbid_eos"])
        lar.frame(fb)
        db.position += 1
        torch.cuda.synchronize()
        assert int(fb.invalid_rows.sum()) == 0


def _loop_state(seed_base: int):
    """One decoder-loop pool (4 sessions) with its own engines and shared
    buffers wired as in test_device_decoder_loop."""
    from magpie_tts_rt_b200.local_ar import AlignmentBatch, LocalArEngine, StreamBatch
    from magpie_tts_rt_b200.model import SHAPE_BASELINE, make_weights
    n, cap, S = 4, 300, 64
    wd = make_main_decoder_weights(3, positions=cap)
    wl = make_weights(SHAPE_BASELINE, seed=21, dtype=torch.bfloat16, profile="parity", with_final=True)
    dec = MainDecoderEngine(wd, max_sessions=n, token_stride=S)
    lar = LocalArEngine(wl, max_streams=n)
    db = MainDecoderBatch.allocate(n, cap=cap, token_stride=S)
    T = [12, 40, 64, 33]
    for s in range(n):
        load_session(db, s, OMD.make_step_inputs(seed_base + s, T[s], 220 + s, cap))
    gate = AlignmentBatch.allocate(T, token_stride=S)
    fb = StreamBatch.allocate(n)
    fb.rng_seed.copy_(torch.arange(n))
    fb.end_frame_index.fill_(-1)
    fb.decoder_hidden = db.hidden
    fb.next_embedding = db.embedded
    gate.alignment_scores = db.alignment
    gate.next_prior = db.prior

    def frame_step():
        dec.step(db)
        gate.gate(fb)
        lar.frame(fb)
        db.position += 1

    return frame_step, db, gate, fb


def test_decoder_loop_graph_replay_matches_eager():
    """The per-frame loop captured once as a CUDA graph (decoder step, gate,
    frame with its EOS kernels, position advance) and replayed, as the bench's
    config-5 loop runs it, leaves exactly the state that the same launches
    made one by one leave: cache, hidden state, scores, prior, counters,
    tokens, end-frame indices."""
    eager_step, e_db, e_gate, e_fb = _loop_state(200)
    graph_step, g_db, g_gate, g_fb = _loop_state(200)
    eager_step()  # also the library's one-time set-up (tensor maps, kernel attributes)
    graph_step()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    cuda_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(cuda_graph, stream=stream):
        graph_step()
    for _ in range(4):
        eager_step()
        cuda_graph.replay()
    torch.cuda.synchronize()
    pairs = [(e_db.self_k, g_db.self_k), (e_db.self_v, g_db.self_v), (e_db.self_mask, g_db.self_mask),
             (e_db.hidden, g_db.hidden), (e_db.embedded, g_db.embedded), (e_db.alignment, g_db.alignment),
             (e_db.prior, g_db.prior), (e_db.position, g_db.position), (e_db.status, g_db.status),
             (e_gate.counters, g_gate.counters), (e_gate.last_attended, g_gate.last_attended),
             (e_gate.decoder_steps, g_gate.decoder_steps), (e_fb.codec_tokens, g_fb.codec_tokens),
             (e_fb.rng_counter, g_fb.rng_counter), (e_fb.end_frame_index, g_fb.end_frame_index),
             (e_fb.invalid_rows, g_fb.invalid_rows), (e_fb.finished, g_fb.finished)]
    for i, (a, b) in enumerate(pairs):
        assert torch.equal(a, b), f"state {i} differs between graph replay and eager launches"
    assert int(e_db.position[0]) == 220 + 5
    assert int(e_fb.invalid_rows.sum()) == 0 and int((e_db.status != 0).sum()) == 0
    del cuda_graph


def _key_value(keys):
    """Order-preserving 32-bit keys (0: none) back to floats."""
    k = keys.astype(np.uint32)
    neg = (k & 0x80000000) == 0
    bits = np.where(neg, ~k, k & 0x7FFFFFFF).astype(np.uint32)
    vals = bits.view(np.float32).copy()
    vals[k == 0] = -np.inf
    return vals


def test_eos_projection_in_the_decoder_step(golden_engine):
    """The EOS projection folded into the decoder step (the reference runs it
    as a per-session GEMV inside the Local AR step, local_ar_plugins.cu:
    1372-1432, on the hidden state the decoder has just produced): for every
    session the step leaves the largest guided code logit and the guided EOS
    logit of each position.  They match the C oracle's guided logits of the
    step's own hidden state within one bf16 rounding (the 768-long dot
    products are summed in another order), and a frame handed this
    projection decides EOS exactly as a frame that computes its own."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    from magpie_tts_rt_b200.model import POSITIONS, SHAPE_BASELINE, VOCAB, make_weights
    from oracle import sampler as S
    z, w, _ = golden_engine
    cap = int(z["cap"])
    lw = make_weights(SHAPE_BASELINE, seed=41, profile="parity", with_final=True)
    fbias = lw.final_b.view(POSITIONS, VOCAB)
    fbias[:8, S.EOS_ID] += 4.0
    fbias[8:, S.EOS_ID] += 4.5
    eng = MainDecoderEngine(w, max_sessions=8, token_stride=512, final_w=lw.final_w, final_b=lw.final_b)
    n = 6
    rng = np.random.default_rng(17)
    b = MainDecoderBatch.allocate(n, cap=cap, token_stride=512)
    for s in range(n):
        load_session(b, s, OMD.make_step_inputs(300 + s, int(rng.integers(8, 200)), int(rng.integers(0, cap)), cap))
    b.eos_projection = torch.zeros(n, 32, dtype=torch.int32, device="cuda")
    eng.step(b)
    torch.cuda.synchronize()
    assert (b.status.cpu() == 0).all()
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    proj = b.eos_projection.cpu().numpy().view(np.uint32)
    got_max, got_eos = _key_value(proj[:, :16]), proj[:, 16:].copy().view(np.float32)
    fw, fb = bits(lw.final_w), bits(lw.final_b)
    exact = 0
    for s in range(n):
        guided = S.eos_guided(bits(b.hidden[s]), fw, fb, 2.5)
        exp_max, exp_eos = guided[:, :2016].max(axis=1), guided[:, 2016]
        for got, exp in ((got_max[s], exp_max), (got_eos[s], exp_eos)):
            assert np.all(np.abs(got - exp) <= 2.0 ** -7 * np.abs(exp) + 1e-6), (s, got, exp)
            exact += int(np.sum(got == exp))
    assert exact >= 0.9 * 2 * n * POSITIONS
    # the frame with the decoder's projection decides as the frame with its own
    leng = LocalArEngine(lw, max_streams=n)
    out = []
    for pre in (b.eos_projection, None):
        fbatch = StreamBatch.allocate(n)
        fbatch.decoder_hidden.copy_(b.hidden)
        fbatch.rng_seed.copy_(torch.arange(n) + 5)
        fbatch.eos_projection = pre
        leng.frame(fbatch)
        torch.cuda.synchronize()
        out.append((fbatch.end_frame_index.cpu().clone(), fbatch.codec_tokens.cpu().clone(),
                    fbatch.invalid_rows.cpu().clone()))
    assert torch.equal(out[0][1], out[1][1]) and torch.equal(out[0][2], out[1][2])
    assert torch.equal(out[0][0], out[1][0]), (out[0][0], out[1][0])
    assert (out[0][2] == 0).all()
