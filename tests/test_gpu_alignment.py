"""GPU parity of the alignment controller (per-utterance drop-in and the
batched gate) against the oracle: bit-exact attended index, unfinished flag,
prior, counters, last_attended and invalid flag on every step; the
reference's own GPU tests (tests/runtime/alignment_kernel_gpu_tests.cu:
75-256), the golden step sequences of the reference's host controller, the
in-band error cases, ragged batches of 1024 sessions, and the fold into the
Local AR frame (the gate's device-written flags give the same frame as flags
set from the oracle on the host)."""
import os

import numpy as np
import pytest
import torch

from oracle import alignment as A

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "alignment.npz")
SENT16 = 0x7777  # prior sentinel (bf16 bits)


def _u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _bf16(bits_np):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(bits_np, np.uint16)).view(np.int16)).view(
        torch.bfloat16)


class Single:
    """Device buffers of one utterance for the drop-in launcher."""

    def __init__(self, T, initial=1, alloc_T=None):
        n = max(T, 1) if alloc_T is None else alloc_T
        self.T = T
        self.scores = torch.zeros(2, n, dtype=torch.bfloat16, device="cuda")
        self.counters = torch.zeros(n, dtype=torch.int32, device="cuda")
        self.last = torch.full((1,), initial, dtype=torch.int32, device="cuda")
        self.prior = _bf16(np.full((2, n), SENT16, np.uint16)).cuda()
        self.attended = torch.full((1,), -7, dtype=torch.int64, device="cuda")
        self.unfinished = torch.zeros(1, dtype=torch.bool, device="cuda")
        self.invalid = torch.full((1,), -7, dtype=torch.int32, device="cuda")

    def step(self, row_bits, contract):
        from magpie_tts_rt_b200 import local_ar as la
        self.scores[0, :len(row_bits)] = _bf16(row_bits).cuda()
        rc = la.launch_alignment_controller(self.scores, contract, self.counters, self.last, self.prior,
                                            self.attended, self.unfinished, self.invalid)
        assert rc == 0
        torch.cuda.synchronize()
        return dict(invalid=int(self.invalid.item()), attended=int(self.attended.item()),
                    unfinished=bool(self.unfinished.item()), prior=_u16(self.prior).reshape(-1),
                    counters=self.counters.cpu().numpy().view(np.uint32), last=int(self.last.item()))


def _contract(T, ign=3, smax=5, la_=6, sink=4):
    from magpie_tts_rt_b200 import local_ar as la
    return la.AlignmentKernelContract(T, ign, smax, la_, sink)


def test_reference_gpu_test_sequence():
    """alignment_kernel_gpu_tests.cu:75-196 (T = 39: odd rows, element path)."""
    T = 39
    d = Single(T)
    host = A.AlignmentController(T)
    for step in range(12):
        s = np.full(T, -2.0, np.float32)
        peak = min(2 + step // 2, 30)
        s[peak] = 4.0
        s[min(peak + 1, T - 1)] = 3.0
        b = A.bf16_bits(s)
        g = d.step(b, _contract(T))
        e = host.advance(A.bf16_to_f32(b))
        assert g["invalid"] == 0 and g["attended"] == e.attended and g["unfinished"] == e.unfinished
        np.testing.assert_array_equal(g["prior"], A.bf16_bits(e.next_prior))


def test_reference_non_finite_fails_closed():
    """alignment_kernel_gpu_tests.cu:198-256, and the state the kernel still
    advances (counter, last_attended) with the prior left unwritten."""
    T = 8
    d = Single(T)
    b = A.bf16_bits(np.zeros(T, np.float32))
    b[7] = A.bf16_bits(np.array([np.nan], np.float32))[0]
    g = d.step(b, _contract(T))
    exp = A.kernel_step(b, A.KernelContract(T), np.zeros(T, np.uint32), np.array([1], np.uint32))
    assert g["invalid"] == 1 and g["attended"] == exp.attended == 1 and g["last"] == 1
    assert g["counters"][1] == 1 and (g["prior"] == SENT16).all()


@pytest.mark.parametrize("case", list(range(11)))
def test_golden_sequences(case):
    z = np.load(GOLDEN)
    g = {k[len(f"c{case}_"):]: z[k] for k in z.files if k.startswith(f"c{case}_")}
    T, ign, smax, la_, sink, init = (int(v) for v in g["contract"])
    d = Single(T, init)
    for k in range(g["scores"].shape[0]):
        out = d.step(g["scores"][k], _contract(T, ign, smax, la_, sink))
        assert out["invalid"] == 0, k
        assert (out["attended"], out["unfinished"]) == (g["attended"][k], g["unfinished"][k]), k
        np.testing.assert_array_equal(out["prior"], g["prior"][k])
    np.testing.assert_array_equal(out["counters"], g["counters"])
    assert out["last"] == int(g["last_attended"])


@pytest.mark.parametrize("T,kw", [(0, {}), (513, {}), (3, {}), (12, dict(la_=0)), (12, dict(sink=0))])
def test_rejected_contract_writes_only_invalid(T, kw):
    d = Single(T, alloc_T=600)
    g = d.step(A.bf16_bits(np.ones(600, np.float32)), _contract(T, **kw))
    assert g["invalid"] == 1 and g["attended"] == -7 and g["last"] == 1
    assert not g["counters"].any() and (g["prior"] == SENT16).all()


def test_non_finite_first_window_entry_and_overflows():
    T = 16
    for bad in (np.nan, np.inf, -np.inf):
        s = np.zeros(T, np.float32)
        s[3] = 5.0
        s[1] = bad
        b = A.bf16_bits(s)
        d = Single(T)
        g = d.step(b, _contract(T))
        e = A.kernel_step(b, A.KernelContract(T), np.zeros(T, np.uint32), np.array([1], np.uint32))
        assert (g["invalid"], g["attended"]) == (e.invalid, e.attended), bad
    # counter overflow at the attended token
    d = Single(T)
    d.counters[4] = -1  # 0xFFFFFFFF
    s = np.zeros(T, np.float32)
    s[4] = 2.0
    g = d.step(A.bf16_bits(s), _contract(T))
    assert g["invalid"] == 1 and g["counters"][4] == A.U32_MAX and (g["prior"] == SENT16).all()
    # search-start overflow: last_attended = UINT32_MAX with a sunk last token
    d = Single(T)
    d.last.fill_(-1)
    d.counters[T - 1] = 4
    g = d.step(A.bf16_bits(s), _contract(T))
    assert g["invalid"] == 1 and g["attended"] == T - 1 and not g["unfinished"]


def test_ties_and_signed_zero_pick_the_left_most():
    T = 24
    s = np.zeros(T, np.float32)
    s[1] = -0.0
    s[3] = 2.0
    s[5] = 2.0
    d = Single(T)
    g = d.step(A.bf16_bits(s), _contract(T))
    assert g["attended"] == 3
    d = Single(T, initial=2)
    s = np.full(T, -1.0, np.float32)
    s[2] = -0.0
    s[4] = 0.0
    g = d.step(A.bf16_bits(s), _contract(T))
    assert g["attended"] == 2


def _batch_state(n, S, seed, inactive_every=0):
    rng = np.random.default_rng(seed)
    T = rng.integers(4, S + 1, n).astype(np.uint32)
    T[::97] = 2  # rejected: shorter than the ignored tail
    T[5::211] = S  # the full stride
    st = dict(text_length=T, constants=(3, 5, 6, 4),
              scores=np.zeros((n, 2, S), np.uint16),
              counters=rng.integers(0, 3, (n, S)).astype(np.uint32),
              last_attended=np.minimum(rng.integers(0, 40, n), np.maximum(T.astype(np.int64) - 1, 0)).astype(np.uint32),
              prior=np.full((n, 2, S), SENT16, np.uint16),
              attended=np.full(n, -7, np.int64), unfinished=np.zeros(n, bool),
              invalid=np.full(n, -7, np.int32), decoder_steps=rng.integers(0, 4, n).astype(np.int64),
              forbid_eos=np.zeros(n, bool), end_frame_index=rng.integers(-1, 2, n).astype(np.int32),
              finished=np.zeros(n, bool))
    st["counters"][:, :] *= (np.arange(S)[None, :] < T[:, None])
    active = np.ones(n, bool)
    if inactive_every:
        active[::inactive_every] = False
    return st, active, rng


def _to_dev(st, active, S):
    from magpie_tts_rt_b200.local_ar import AlignmentBatch
    n = len(st["text_length"])
    ab = AlignmentBatch.allocate(st["text_length"].astype(np.int64).tolist(), token_stride=S)
    ab.counters.copy_(torch.from_numpy(st["counters"].view(np.int32)))
    ab.last_attended.copy_(torch.from_numpy(st["last_attended"].view(np.int32)))
    ab.next_prior.copy_(_bf16(st["prior"]))
    ab.attended_token_index.fill_(-7)
    ab.invalid_state.fill_(-7)
    ab.decoder_steps.copy_(torch.from_numpy(st["decoder_steps"]))
    outs = dict(unfinished=torch.zeros(n, dtype=torch.bool, device="cuda"),
                forbid_eos=torch.zeros(n, dtype=torch.bool, device="cuda"),
                finished=torch.zeros(n, dtype=torch.bool, device="cuda"),
                end_frame_index=torch.from_numpy(st["end_frame_index"]).cuda(),
                active=torch.from_numpy(active).cuda())
    return ab, outs


def _compare(ab, outs, st):
    np.testing.assert_array_equal(ab.invalid_state.cpu().numpy(), st["invalid"])
    np.testing.assert_array_equal(ab.attended_token_index.cpu().numpy(), st["attended"])
    np.testing.assert_array_equal(outs["unfinished"].cpu().numpy(), st["unfinished"])
    np.testing.assert_array_equal(outs["forbid_eos"].cpu().numpy(), st["forbid_eos"])
    np.testing.assert_array_equal(outs["finished"].cpu().numpy(), st["finished"])
    np.testing.assert_array_equal(ab.decoder_steps.cpu().numpy(), st["decoder_steps"])
    np.testing.assert_array_equal(ab.counters.cpu().numpy().view(np.uint32), st["counters"])
    np.testing.assert_array_equal(ab.last_attended.cpu().numpy().view(np.uint32), st["last_attended"])
    np.testing.assert_array_equal(_u16(ab.next_prior).reshape(st["prior"].shape), st["prior"])


@pytest.mark.parametrize("n,S,steps", [(1024, 512, 6), (300, 136, 8), (37, 37, 10), (5, 13, 12)])
def test_batch_matches_oracle(n, S, steps):
    """Ragged text lengths up to the stride, rejected contracts, inactive
    sessions, random prior state; strides 512 / 136 take the 16-byte path,
    37 / 13 the element path."""
    st, active, rng = _batch_state(n, S, seed=n + S, inactive_every=13)
    ab, outs = _to_dev(st, active, S)
    for k in range(steps):
        pos = (k + 1) * 1.5 + rng.uniform(0, 3, n)
        sc = rng.standard_normal((n, S)).astype(np.float32)
        sc += 4.0 * np.exp(-0.5 * ((np.arange(S)[None, :] - pos[:, None]) / 1.5) ** 2)
        if k % 3 == 2:
            sc = np.round(sc)  # ties
        bits = A.bf16_bits(sc)
        if k == 4:
            bits[min(7, n - 1), min(3, S - 1)] = 0x7FC0  # a NaN: that session fails closed this step
        st["scores"][:, 0] = bits
        st["scores"][:, 1] = A.bf16_bits(rng.standard_normal((n, S)).astype(np.float32))
        ab.alignment_scores.copy_(_bf16(st["scores"]))
        ab.gate(**outs)
        A.gate_step(st, active)
        torch.cuda.synchronize()
        _compare(ab, outs, st)


def test_batch_argument_checks():
    from magpie_tts_rt_b200 import _lib as L
    from magpie_tts_rt_b200.local_ar import AlignmentBatch
    import ctypes
    ab = AlignmentBatch.allocate([12, 12], token_stride=16)
    cb = ab.c_struct(unfinished=torch.zeros(2, dtype=torch.bool, device="cuda"))
    cb.decoder_steps = ab.decoder_steps.data_ptr()  # forbid_eos missing
    assert L.lib.mtt_b200_launch_alignment_batch(ctypes.byref(cb), None) == L.STATUS_INVALID_ARGUMENT
    cb.decoder_steps = None
    cb.token_stride = 0
    assert L.lib.mtt_b200_launch_alignment_batch(ctypes.byref(cb), None) == L.STATUS_INVALID_ARGUMENT


def test_gate_drives_the_local_ar_frame():
    """Three decoder steps of [alignment gate -> Local AR frame] on 24
    sessions: the frame inputs the gate writes on the device (unfinished,
    forbid_eos, finished from the previous frame's end_frame_index) equal
    the oracle's, and the frame's tokens, counters and EOS equal those of a
    frame whose flags were set on the host."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    from magpie_tts_rt_b200.model import EMBED, SHAPE_BASELINE, make_weights
    n, S = 24, 64
    w = make_weights(SHAPE_BASELINE, seed=21, dtype=torch.bfloat16, profile="parity", with_final=True)
    eng = LocalArEngine(w, max_streams=n)
    st, active, rng = _batch_state(n, S, seed=3)
    st["text_length"][:] = np.maximum(st["text_length"], 8)
    st["last_attended"][::2] = st["text_length"][::2] - 1  # text done: EOS is evaluated from step 2
    st["end_frame_index"][:] = -1
    st["decoder_steps"][:] = 0
    ab, _ = _to_dev(st, active, S)
    fb = StreamBatch.allocate(n)
    fb.end_frame_index.fill_(-1)
    fb.rng_seed.copy_(torch.arange(n, dtype=torch.int64))
    host = StreamBatch.allocate(n)
    host.end_frame_index.fill_(-1)
    host.rng_seed.copy_(fb.rng_seed)
    for k in range(3):
        g = torch.Generator().manual_seed(100 + k)
        hidden = torch.randn(n, 2, EMBED, generator=g).to(torch.bfloat16).cuda()
        fb.decoder_hidden.copy_(hidden)
        host.decoder_hidden.copy_(hidden)
        sc = A.bf16_bits(rng.standard_normal((n, S)).astype(np.float32) * 2)
        st["scores"][:, 0] = sc
        ab.alignment_scores.copy_(_bf16(st["scores"]))
        st["end_frame_index"] = host.end_frame_index.cpu().numpy()
        A.gate_step(st, None)
        ab.gate(fb)
        eng.frame(fb)
        host.unfinished.copy_(torch.from_numpy(st["unfinished"]))
        host.forbid_eos.copy_(torch.from_numpy(st["forbid_eos"]))
        host.finished.copy_(torch.from_numpy(st["finished"]))
        eng.frame(host)
        torch.cuda.synchronize()
        for name in ("unfinished", "forbid_eos", "finished"):
            np.testing.assert_array_equal(getattr(fb, name).cpu().numpy(), st[name], err_msg=name)
        for name in ("codec_tokens", "rng_counter", "invalid_rows", "end_frame_index"):
            assert torch.equal(getattr(fb, name), getattr(host, name)), name
