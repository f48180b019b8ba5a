"""The alignment-controller oracle on CPU: the reference's own known-answer
tests (tests/runtime/alignment_controller_tests.cpp:40-114), the golden step
sequences produced by the reference's compiled host controller
(tests/golden/alignment.npz), the CUDA kernel's in-band error behaviour
(src/runtime/alignment_kernel.cu:29-114) and the batched gate's EOS inputs."""
import os

import numpy as np
import pytest

from oracle import alignment as A
from oracle import alignment_ref as R

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "alignment.npz")


def golden_cases():
    z = np.load(GOLDEN)
    for i in range(int(z["n_cases"])):
        yield {k[len(f"c{i}_"):]: z[k] for k in z.files if k.startswith(f"c{i}_")}


# --------------------------------------------------- reference KATs (host class)

def test_window_sink_and_prior():
    """alignment_controller_tests.cpp:40-67."""
    c = A.AlignmentController(12)
    s = np.zeros(12, np.float32)
    s[4] = 2.0
    r = c.advance(s)
    assert r.attended == 4 and r.unfinished and r.next_prior.size == 24
    assert r.next_prior[3] == 1.0 and r.next_prior[4] == 1.0 and r.next_prior[9] == 1.0
    assert r.next_prior[12] == np.float32(0.1)
    s[:] = 0.0
    s[4] = 3.0
    for _ in range(3):
        assert c.advance(s).attended == 4
    s[5] = 4.0
    r = c.advance(s)
    assert r.attended == 5
    assert (r.next_prior[:5] == np.float32(0.1)).all()


def test_short_text_and_terminal_window():
    """alignment_controller_tests.cpp:69-90."""
    r = A.AlignmentController(5).advance([0.0, 3.0, 1.0, 0.0, 0.0])
    assert (r.next_prior[:5] == 1.0).all()
    c = A.AlignmentController(8)
    s = np.zeros(8, np.float32)
    s[4] = 2.0
    assert c.advance(s).attended == 4
    s[:] = 0.0
    s[4] = 1.0
    r = c.advance(s)
    assert r.attended == 4 and r.unfinished


def test_invalid_input_fails_closed():
    """alignment_controller_tests.cpp:92-114."""
    with pytest.raises(A.AlignmentControllerError) as e:
        A.AlignmentController(3)
    assert e.value.code == "invalid_text_length"
    c = A.AlignmentController(8)
    with pytest.raises(A.AlignmentControllerError) as e:
        c.advance([1.0])
    assert e.value.code == "invalid_score_count"
    with pytest.raises(A.AlignmentControllerError) as e:
        c.advance([0, 0, 0, np.nan, 0, 0, 0, 0])
    assert e.value.code == "non_finite_score"


def test_kernel_gpu_test_sequence():
    """tests/runtime/alignment_kernel_gpu_tests.cu:75-196: twelve steps of a
    travelling peak, the kernel's outputs equal the host class's (prior
    compared after bf16 rounding)."""
    T = 39
    host = A.AlignmentController(T)
    counters = np.zeros(T, np.uint32)
    last = np.array([1], np.uint32)
    for step in range(12):
        s = np.full(T, -2.0, np.float32)
        peak = min(2 + step // 2, 30)
        s[peak] = 4.0
        s[min(peak + 1, T - 1)] = 3.0
        bits = A.bf16_bits(s)
        out = A.kernel_step(bits, A.KernelContract(T), counters, last)
        exp = host.advance(A.bf16_to_f32(bits))
        assert out.invalid == 0 and out.attended == exp.attended and out.unfinished == exp.unfinished
        np.testing.assert_array_equal(out.prior, A.bf16_bits(exp.next_prior))


def test_bf16_helpers():
    x = np.array([0.1, 1.0, -2.0, 3.0, 4.0, np.inf, -np.inf], np.float32)
    b = A.bf16_bits(x)
    assert b[0] == A.EPSILON_BF16 and b[1] == A.ONE_BF16
    np.testing.assert_array_equal(A.bf16_to_f32(b)[1:], x[1:])
    assert np.isnan(A.bf16_to_f32(A.bf16_bits(np.array([np.nan], np.float32))))[0]


# --------------------------------------------------- golden step sequences

@pytest.mark.parametrize("case", list(range(11)))
def test_oracle_matches_reference_golden(case):
    g = list(golden_cases())[case]
    T, ign, smax, la, sink, init = (int(v) for v in g["contract"])
    host = A.AlignmentController(T, 0.1, init, ign, smax, la, sink)
    contract = A.KernelContract(T, ign, smax, la, sink)
    counters = np.zeros(T, np.uint32)
    last = np.array([init], np.uint32)
    for k in range(g["scores"].shape[0]):
        bits = g["scores"][k]
        r = host.advance(A.bf16_to_f32(bits))
        assert (r.attended, r.unfinished) == (g["attended"][k], g["unfinished"][k])
        np.testing.assert_array_equal(A.bf16_bits(r.next_prior), g["prior"][k])
        out = A.kernel_step(bits, contract, counters, last)
        assert out.invalid == 0
        assert (out.attended, out.unfinished) == (g["attended"][k], g["unfinished"][k])
        np.testing.assert_array_equal(out.prior, g["prior"][k])
    np.testing.assert_array_equal(counters, g["counters"])
    np.testing.assert_array_equal(host.counters.astype(np.uint32), g["counters"])
    assert int(last[0]) == int(g["last_attended"])


@pytest.mark.skipif(not os.path.exists(R.REF_SOURCE) and not os.path.exists(R.LIBRARY),
                    reason="the reference controller is only built where the reference tree is")
def test_oracle_matches_live_reference_random():
    """Fresh seeded sequences through the compiled reference class."""
    rng = np.random.default_rng(77)
    for trial in range(20):
        T = int(rng.integers(4, 300))
        ign = int(rng.integers(0, min(T, 8)))
        la = int(rng.integers(1, 20))
        sink = int(rng.integers(1, 6))
        smax = int(rng.integers(0, 12))
        ref = R.RefController(T, 0.1, 1, ign, smax, la, sink)
        if T <= ign:
            assert ref.status == 1
            continue
        host = A.AlignmentController(T, 0.1, 1, ign, smax, la, sink)
        for k in range(40):
            s = A.bf16_to_f32(A.bf16_bits(np.round(rng.standard_normal(T) * 2) / 2))
            rc, att, unf, prior = ref.advance(s)
            r = host.advance(s)
            assert rc == 0 and (att, unf) == (r.attended, r.unfinished), (trial, k)
            np.testing.assert_array_equal(prior, r.next_prior)
        np.testing.assert_array_equal(ref.counters(), host.counters.astype(np.uint32))


# --------------------------------------------------- kernel in-band errors

def _row(T, peak=4):
    s = np.zeros(T, np.float32)
    s[peak] = 2.0
    return A.bf16_bits(s)


@pytest.mark.parametrize("bad", [dict(text_length=0), dict(text_length=513), dict(text_length=3),
                                 dict(lookahead=0), dict(sink_threshold=0)])
def test_kernel_rejects_contract(bad):
    c = A.KernelContract(**{**dict(text_length=12), **bad})
    counters = np.zeros(600, np.uint32)
    last = np.array([1], np.uint32)
    out = A.kernel_step(_row(600), c, counters, last)
    assert out.invalid == 1 and out.attended is None and out.prior is None
    assert not counters.any() and last[0] == 1


def test_kernel_non_finite_advances_state_without_prior():
    """alignment_kernel_gpu_tests.cu:198-256: a NaN outside the window is
    still rejected; the kernel has already counted the step."""
    T = 8
    bits = A.bf16_bits(np.zeros(T, np.float32))
    bits[7] = A.bf16_bits(np.array([np.nan], np.float32))[0]
    counters = np.zeros(T, np.uint32)
    last = np.array([1], np.uint32)
    out = A.kernel_step(bits, A.KernelContract(T), counters, last)
    assert out.invalid == 1 and out.prior is None
    assert out.attended == 1 and counters[1] == 1 and last[0] == 1


def test_kernel_non_finite_first_window_entry_holds():
    T = 16
    s = np.zeros(T, np.float32)
    s[3] = 5.0
    bits = A.bf16_bits(s)
    for bad in (np.nan, np.inf):
        b = bits.copy()
        b[1] = A.bf16_bits(np.array([bad], np.float32))[0]
        out = A.kernel_step(b, A.KernelContract(T), np.zeros(T, np.uint32), np.array([1], np.uint32))
        assert out.invalid == 1 and out.attended == 1
    b = bits.copy()
    b[1] = A.bf16_bits(np.array([-np.inf], np.float32))[0]
    out = A.kernel_step(b, A.KernelContract(T), np.zeros(T, np.uint32), np.array([1], np.uint32))
    assert out.invalid == 1 and out.attended == 3


def test_kernel_counter_and_search_overflow():
    T = 12
    counters = np.zeros(T, np.uint32)
    counters[4] = A.U32_MAX
    out = A.kernel_step(_row(T), A.KernelContract(T), counters, np.array([1], np.uint32))
    assert out.invalid == 1 and counters[4] == A.U32_MAX and out.prior is None
    counters = np.zeros(T, np.uint32)
    counters[T - 1] = 4
    last = np.array([A.U32_MAX], np.uint32)
    out = A.kernel_step(_row(T), A.KernelContract(T), counters, last)
    assert out.invalid == 1 and out.attended == T - 1 and not out.unfinished


def test_kernel_last_attended_beyond_text():
    T = 12
    last = np.array([40], np.uint32)
    out = A.kernel_step(_row(T), A.KernelContract(T), np.zeros(T, np.uint32), last)
    assert out.invalid == 0 and out.attended == T - 1 and not out.unfinished


# --------------------------------------------------- batched gate (host logic)

def test_gate_step_eos_inputs():
    n, S = 4, 16
    st = dict(text_length=np.array([12, 12, 2, 12], np.uint32), constants=(3, 5, 6, 4),
              scores=np.zeros((n, 2, S), np.uint16), counters=np.zeros((n, S), np.uint32),
              last_attended=np.ones(n, np.uint32), prior=np.zeros((n, 2, S), np.uint16),
              attended=np.full(n, -7, np.int64), unfinished=np.zeros(n, bool),
              invalid=np.full(n, -7, np.int32), decoder_steps=np.array([0, 1, 2, 5], np.int64),
              forbid_eos=np.zeros(n, bool), end_frame_index=np.array([-1, 0, 1, -1], np.int32),
              finished=np.zeros(n, bool))
    st["scores"][:, 0] = _row(S)
    active = np.array([True, True, True, False])
    A.gate_step(st, active)
    assert st["forbid_eos"].tolist() == [True, True, False, False]
    assert st["decoder_steps"].tolist() == [1, 2, 3, 5]
    assert st["finished"].tolist() == [False, True, True, False]
    assert st["invalid"].tolist() == [0, 0, 1, -7]  # session 2: text shorter than the ignored tail
    assert st["attended"].tolist() == [4, 4, -7, -7] and st["unfinished"].tolist() == [True, True, False, False]
    assert (st["prior"][3] == 0).all() and (st["prior"][2] == 0).all()
