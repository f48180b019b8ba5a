"""CPU restatement of the reference's alignment (attention-prior) controller.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg as the checker.  The product library never
imports this module.

Once per Main Decoder step the controller picks the text token the decoder
attends to (a windowed argmax over the conditional row of the step's bf16
alignment scores), counts visits per token ("sinks"), reports whether text is
left (the Local AR's ``unfinished`` input) and writes the next step's
attention prior.  Two reference statements exist and both are restated here:

* ``AlignmentController`` follows the host reference class
  ``src/runtime/alignment_controller.cpp:57-185``: errors raise
  ``AlignmentControllerError`` (codes of ``alignment_controller.hpp:12-17``)
  and leave the state untouched.
* ``kernel_step`` follows the CUDA kernel
  ``src/runtime/alignment_kernel.cu:16-154`` that the runtime actually runs:
  errors are in-band (``invalid_state``), a rejected contract writes nothing
  else, and non-finite scores still advance the state (counters and
  last_attended) but leave the prior unwritten.

On valid inputs the two agree; the tests check that against the reference's
own known-answer tests and against golden vectors produced by compiling the
host reference class (``oracle/alignment_ref.py``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

MAX_TEXT_TOKENS = 512          # alignment_kernel.cu:12
U32_MAX = 0xFFFFFFFF           # alignment_kernel.cu:14
EPSILON_BF16 = 0x3DCD          # bf16 round-to-nearest-even of 0.1f (alignment_kernel.cu:115)
ONE_BF16 = 0x3F80              # 1.0

# the manifest values of the reference's tests (alignment_controller_tests.cpp:23-38)
TEST_CONTRACT = dict(ignored_terminal_tokens=3, short_text_no_prior_max_tokens=5, lookahead=6,
                     sink_threshold=4)
INITIAL_ATTENDED = 1


class AlignmentControllerError(RuntimeError):
    """alignment_controller.hpp:12-31; ``code`` is one of the four names."""

    def __init__(self, code: str, detail: str):
        super().__init__(f"alignment controller failed [code={code}]: {detail}")
        self.code = code


def bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN kept NaN)."""
    f = np.ascontiguousarray(np.asarray(x, np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class StepResult:
    attended: int
    unfinished: bool
    next_prior: np.ndarray  # [2*T] float32: conditional row, unconditional row


class AlignmentController:
    """alignment_controller.cpp:57-185 (the host reference the CUDA kernel is
    validated against)."""

    def __init__(self, text_length: int, prior_epsilon: float = 0.1,
                 initial_attended: int = INITIAL_ATTENDED, ignored_terminal_tokens: int = 3,
                 short_text_no_prior_max_tokens: int = 5, lookahead: int = 6, sink_threshold: int = 4):
        # alignment_controller.cpp:69-75
        if text_length == 0 or text_length <= ignored_terminal_tokens or initial_attended >= text_length:
            raise AlignmentControllerError(
                "invalid_text_length",
                "text must contain the initial attended token and all ignored terminal tokens")
        self.T = int(text_length)
        self.eps = np.float32(prior_epsilon)
        self.ignored = int(ignored_terminal_tokens)
        self.short_max = int(short_text_no_prior_max_tokens)
        self.lookahead = int(lookahead)
        self.sink = int(sink_threshold)
        self.last_attended = int(initial_attended)
        self.counters = np.zeros(self.T, np.uint64)

    def advance(self, scores) -> StepResult:
        s = np.asarray(scores, np.float32)
        T = self.T
        if s.shape != (T,):  # :80-84
            raise AlignmentControllerError("invalid_score_count",
                                           "alignment score length differs from the prepared token length")
        if not np.isfinite(s).all():  # :85-91
            raise AlignmentControllerError("non_finite_score", "alignment scores must all be finite")
        last = min(self.last_attended, T - 1)  # :93-104
        search_start = self.last_attended
        if self.counters[last] >= self.sink:
            if search_start == U32_MAX:
                raise AlignmentControllerError("state_overflow", "alignment search position overflowed")
            search_start += 1
        search_start = min(search_start, T)
        content_end = T - self.ignored  # :105-114
        window_end = min(min(search_start + self.lookahead, U32_MAX), content_end)
        attended = T - 1  # :116-130: strict '>' keeps the left-most maximum
        if window_end > search_start:
            attended = search_start
            best = s[search_start]
            for i in range(search_start + 1, window_end):
                if s[i] > best:
                    attended, best = i, s[i]
        self.last_attended = attended  # :131-138
        if self.counters[attended] == U32_MAX:
            raise AlignmentControllerError("state_overflow", "alignment sink counter overflowed")
        self.counters[attended] += 1
        prior = np.full(2 * T, self.eps, np.float32)  # :140-165
        if T <= self.short_max:
            prior[:T] = 1.0
        else:
            history = min(max(attended - 1 if attended else 0, min(1, T - 1)), T - 1)
            prior[history] = 1.0
            prior[attended] = 1.0
            for off in range(1, self.lookahead + 1):
                prior[min(attended + off, T - 1)] = 1.0
        sinks = np.flatnonzero(self.counters >= self.sink)  # :167-178
        if sinks.size:
            prior[:int(sinks[-1]) + 1] = self.eps
        return StepResult(attended, attended < content_end, prior)


@dataclass
class KernelContract:
    """AlignmentKernelContract (alignment_kernel.hpp:9-15)."""
    text_length: int
    ignored_terminal_tokens: int = 3
    short_text_no_prior_max_tokens: int = 5
    lookahead: int = 6
    sink_threshold: int = 4


@dataclass
class KernelOutputs:
    invalid: int
    attended: Optional[int]      # None: not written
    unfinished: Optional[bool]   # None: not written
    prior: Optional[np.ndarray]  # [2*T] bf16 bits, None: not written


def kernel_step(scores_bf16, contract: KernelContract, counters: np.ndarray, last_attended: np.ndarray) -> KernelOutputs:
    """One launch of alignment_controller_kernel (alignment_kernel.cu:16-154).

    ``scores_bf16``: the conditional row's bf16 bits (at least T entries; the
    unconditional row is never read).  ``counters`` (uint32 [>=T]) and
    ``last_attended`` (uint32 [1]) are updated in place as the kernel does."""
    T = int(contract.text_length)
    if (T == 0 or T > MAX_TEXT_TOKENS or T <= contract.ignored_terminal_tokens
            or contract.lookahead == 0 or contract.sink_threshold == 0):  # :33-37
        return KernelOutputs(1, None, None, None)
    bits = np.asarray(scores_bf16, np.uint16)[:T]
    vals = bf16_to_f32(bits)
    finite = (bits & 0x7F80) != 0x7F80
    invalid = 0
    la = int(last_attended[0])
    search_start = la  # :39-49
    if int(counters[min(la, T - 1)]) >= contract.sink_threshold:
        if search_start == U32_MAX:
            invalid = 1
        else:
            search_start += 1
    search_start = min(search_start, T)
    content_end = T - contract.ignored_terminal_tokens  # :50-59
    window_end = min(min(search_start + contract.lookahead, U32_MAX), content_end)
    attended = T - 1  # :61-81: the first window entry seeds 'best' even when
    if window_end > search_start:  # non-finite; later non-finite entries are skipped
        attended = search_start
        best = vals[search_start]
        for i in range(search_start + 1, window_end):
            if finite[i] and vals[i] > best:
                attended, best = i, vals[i]
    if not finite.all():  # :82-88 (the whole conditional row)
        invalid = 1
    if int(counters[attended]) == U32_MAX:  # :90-94
        invalid = 1
    else:
        counters[attended] += 1
    last_attended[0] = attended
    unfinished = attended < content_end
    if invalid:  # :106-114: nothing further is written
        return KernelOutputs(1, attended, unfinished, None)
    c = np.asarray(counters[:T], np.uint64)  # :99-104
    sinks = np.flatnonzero(c >= contract.sink_threshold)
    msp = int(sinks[-1]) if sinks.size else -1
    prior = np.full(2 * T, EPSILON_BF16, np.uint16)  # :115-153
    idx = np.arange(T)
    if T <= contract.short_text_no_prior_max_tokens:
        one = np.ones(T, bool)
    else:
        history = max(attended - 1 if attended else 0, min(1, T - 1))
        hi = min(attended + contract.lookahead, T - 1)
        one = (idx == history) | ((idx >= attended) & (idx <= hi))
    prior[:T][one & (idx > msp)] = ONE_BF16
    return KernelOutputs(0, attended, unfinished, prior)


def gate_step(state: dict, active: Optional[np.ndarray] = None) -> None:
    """One launch of the batched gate (``mtt_b200_launch_alignment_batch``) on
    a dict of numpy arrays, updated in place:

    per active session s, ``kernel_step`` on its row (text_length[s], the
    shared contract constants), its outputs written where the kernel writes
    them; then the Local AR EOS inputs the reference's pipeline prepares
    before each Local AR step (synthesis_pipeline.cpp:511-569):
    ``forbid_eos = decoder_steps < 2`` and ``decoder_steps += 1`` (the host's
    generated_decoder_steps_), and ``finished |= end_frame_index in {0, 1}``
    (the latch of launch_finalize_local_step, synthesis_kernels.cu:79-84,
    applied to the previous frame's result)."""
    for s in range(len(state["text_length"])):
        if active is not None and not active[s]:
            continue
        c = KernelContract(int(state["text_length"][s]), *state["constants"])
        cnt = state["counters"][s]
        la = state["last_attended"][s:s + 1]
        out = kernel_step(state["scores"][s, 0], c, cnt, la)
        state["invalid"][s] = out.invalid
        if out.attended is not None:
            state["attended"][s] = out.attended
            state["unfinished"][s] = out.unfinished
        if out.prior is not None:
            T = c.text_length
            state["prior"][s, 0, :T] = out.prior[:T]
            state["prior"][s, 1, :T] = out.prior[T:]
        if state.get("decoder_steps") is not None:
            state["forbid_eos"][s] = state["decoder_steps"][s] < 2
            state["decoder_steps"][s] += 1
        if state.get("end_frame_index") is not None:
            if state["end_frame_index"][s] in (0, 1):
                state["finished"][s] = True
