"""The Main Decoder one-step oracle on CPU against the golden steps the
reference's own wrapper produced (tests/golden/main_decoder.npz, made by
tests/golden/make_main_decoder_golden.py from
tools/export/main_decoder_wrapper.py on NeMo's transformer_2501): bit-exact
hidden state, alignment scores and the key / value rows written."""
import os

import numpy as np
import pytest
import torch

from magpie_tts_rt_b200.main_decoder import make_main_decoder_weights
from oracle import main_decoder as OMD

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "main_decoder.npz")


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def golden():
    z = np.load(GOLDEN)
    w = make_main_decoder_weights(int(z["weight_seed"]), positions=int(z["cap"]))
    return z, w


@pytest.mark.parametrize("case", range(4))
def test_oracle_matches_reference_wrapper(golden, case):
    z, w = golden
    seed, T, pos = (int(v) for v in z[f"c{case}_case"])
    inp = OMD.make_step_inputs(seed, T, pos, int(z["cap"]))
    out = OMD.step(w, inp)
    np.testing.assert_array_equal(_bits(out.hidden), z[f"c{case}_hidden"])
    np.testing.assert_array_equal(_bits(out.alignment), z[f"c{case}_alignment"])
    np.testing.assert_array_equal(_bits(out.k_new), z[f"c{case}_k_new"])
    np.testing.assert_array_equal(_bits(out.v_new), z[f"c{case}_v_new"])


def test_alignment_is_a_distribution_on_the_conditional_row(golden):
    """Each alignment layer's probabilities sum to ~1 over the unmasked text
    (renormalised by the prior), so their mean does too; the unconditional
    row keeps only its first token (make_step_example's condition mask)."""
    z, w = golden
    seed, T, pos = (int(v) for v in z["c0_case"])
    out = OMD.step(w, OMD.make_step_inputs(seed, T, pos, int(z["cap"])))
    a = out.alignment.float()
    assert abs(float(a[0].sum()) - 1.0) < 0.02
    assert float(a[1, 0]) == 1.0 and float(a[1, 1:].abs().sum()) == 0.0
