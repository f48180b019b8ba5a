"""Generate ``tests/golden/alignment.npz``: step sequences of the reference's
own host alignment controller (src/runtime/alignment_controller.cpp, compiled
by ``oracle/alignment_ref.py``) on seeded synthetic alignment scores.

Run where the reference tree is present:  python tests/golden/make_alignment_golden.py

Each case is one utterance: a contract, K steps of conditional-row scores
(bf16 bit patterns; the reference class sees their float values, as the
kernel does), and per step the attended token, the unfinished flag, the next
prior (bf16 bits of the reference's float prior); the counters and
last_attended after the last step.  Scores are a travelling peak over N(0, 1)
noise; some cases quantise to coarse steps so that ties exercise the left-most rule, some hold the peak
so that sinks form, one case is the reference's own GPU test sequence
(tests/runtime/alignment_kernel_gpu_tests.cu:103-112), restated as a formula.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import alignment as A  # noqa: E402
from oracle import alignment_ref as R  # noqa: E402

OUT = os.path.join(HERE, "alignment.npz")

# (text_length, ignored, short_max, lookahead, sink, steps, quantum, hold_prob, seed)
CASES = [
    (5, 3, 5, 6, 4, 12, 0.0, 0.3, 1),       # short text: prior all ones
    (8, 3, 5, 6, 4, 20, 0.0, 0.5, 2),       # terminal window
    (12, 3, 5, 6, 4, 40, 0.5, 0.5, 3),      # ties
    (39, 3, 5, 6, 4, 12, None, 0.0, 0),     # the reference GPU test's sequence
    (64, 3, 5, 6, 4, 200, 0.0, 0.6, 4),
    (64, 0, 5, 1, 1, 80, 0.0, 0.2, 5),      # lookahead 1, sink 1, no ignored tail
    (128, 2, 10, 12, 3, 200, 0.25, 0.5, 6),
    (257, 3, 5, 6, 4, 100, 0.0, 0.7, 7),
    (511, 3, 5, 40, 6, 120, 1.0, 0.4, 8),
    (512, 3, 5, 6, 4, 120, 0.0, 0.5, 9),
    (512, 5, 600, 6, 4, 30, 0.0, 0.5, 10),  # short-text rule with a long text
]


def scores_for(T, K, quantum, hold, seed):
    if quantum is None:  # alignment_kernel_gpu_tests.cu:103-112
        rows = []
        for step in range(K):
            s = np.full(T, -2.0, np.float32)
            peak = min(2 + step // 2, 30)
            s[peak] = 4.0
            s[min(peak + 1, T - 1)] = 3.0
            rows.append(s)
        return np.stack(rows)
    rng = np.random.default_rng(seed)
    pos = 1.0
    rows = []
    for _ in range(K):
        if rng.random() > hold:
            pos = min(pos + rng.uniform(0.2, 2.0), T + 2)
        s = rng.standard_normal(T).astype(np.float32)
        s += 4.0 * np.exp(-0.5 * ((np.arange(T) - pos) / 1.5) ** 2).astype(np.float32)
        if quantum:
            s = np.round(s / quantum) * quantum
        rows.append(s.astype(np.float32))
    return np.stack(rows)


def main():
    if R.build() is None:
        raise SystemExit("the reference tree is not present: cannot generate")
    out = {"n_cases": np.int32(len(CASES))}
    for i, (T, ign, smax, la, sink, K, q, hold, seed) in enumerate(CASES):
        raw = scores_for(T, K, q, hold, seed)
        bits = A.bf16_bits(raw)
        vals = A.bf16_to_f32(bits)
        ref = R.RefController(T, 0.1, 1, ign, smax, la, sink)
        assert ref.status == 0
        att = np.zeros(K, np.int64)
        unf = np.zeros(K, bool)
        prior = np.zeros((K, 2 * T), np.uint16)
        for k in range(K):
            rc, a, u, p = ref.advance(vals[k])
            assert rc == 0, rc
            att[k], unf[k] = a, u
            prior[k] = A.bf16_bits(p)
        out[f"c{i}_contract"] = np.array([T, ign, smax, la, sink, 1], np.int64)
        out[f"c{i}_scores"] = bits
        out[f"c{i}_attended"] = att
        out[f"c{i}_unfinished"] = unf
        out[f"c{i}_prior"] = prior
        out[f"c{i}_counters"] = ref.counters()
        out[f"c{i}_last_attended"] = np.uint32(ref.last_attended())
    np.savez_compressed(OUT, **out)
    print(OUT, os.path.getsize(OUT))


if __name__ == "__main__":
    main()
