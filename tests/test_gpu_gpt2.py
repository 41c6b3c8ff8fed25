"""Whole-model GPT-2 small forward on the device (Gpt2Session: embed, 12
layers, final LN, logits through the seam's fixed-point entry points)
against the reference's NumPy mirror (scripts/gpt2_fixed.py forward_model)
at T = 16 and at the benchmark's T = 1024, through the recorded digests of
every layer output, every wire of the first and last layer, the final LN
row and the logits."""

import numpy as np
import pytest

from tests.test_gpt2_model import golden, mismatches

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


@pytest.fixture(scope="module")
def model():
    from volta_zk_b200 import gpt2

    return gpt2.synthetic_model()


@pytest.mark.parametrize("t", [16, 1024])
def test_device_forward_matches_reference_mirror(prover, model, t):
    from volta_zk_b200 import gpt2

    with gpt2.Gpt2Session(prover, model, t) as s:
        tokens = gpt2.prefill_tokens(t)
        s.forward(tokens)
        assert s.error_word() == 0 and s.layer_errors() == [0] * gpt2.LAYERS
        bad = mismatches(golden(t), s.embed_out(), lambda l, k: s.wire(l, k), s.final_ln_out(), s.logits())
        assert not bad, bad
        # a second forward on the resident tokens gives the same logits
        first = s.logits()
        s.forward()
        assert np.array_equal(s.logits(), first)


def test_device_forward_without_stable_softmax_reports_saturation(prover, model):
    """LutParams::default (no row shift) at T = 1024: the reciprocal index
    leaves its u16 domain, which the reference asserts on (layer.rs:782);
    the device reports it through the sticky error word instead of
    faulting."""
    from volta_zk_b200 import gpt2

    with gpt2.Gpt2Session(prover, model, 1024, params=gpt2.LutParams(softmax_row_shift=False)) as s:
        s.forward(gpt2.prefill_tokens(1024))
        assert any(e != 0 for e in s.layer_errors())
