"""The GPT-2 prefill proof schedule on the device (Gpt2Prover over a
Gpt2Session's witness) against its CPU oracle composition
(oracle/gpt2.py) on the same model and tokens, word for word:
every layer's 14 LogUp instances, four GEMM sumchecks, the A.V, softmax-norm
and Q.K^T sumchecks and the two LayerNorm products; the boundary
corrections; the weight commitment's root.  A power-of-two prefill (T = 16)
and the reference's measured prefill length (T = 100, padded to 128)."""

import numpy as np
import pytest

from oracle.gpt2 import OracleOps, Schedule, forward_model, pcs_root

pytestmark = pytest.mark.gpu
SEED, MAC_SEED, PAD_SEED = bytes([0x50] * 32), bytes([0x4D] * 32), bytes([0x11] * 32)


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


@pytest.mark.parametrize("t,layers", [(16, 2), (100, 2)])
def test_proof_matches_oracle_composition(prover, oracle, t, layers):
    from volta_zk_b200 import gpt2

    model = gpt2.synthetic_model(n_layers=layers)
    luts = gpt2.build_luts()
    tokens = gpt2.prefill_tokens(t)
    with gpt2.Gpt2Session(prover, model, t) as s, gpt2.Gpt2Prover(s) as gp:
        s.forward(tokens)
        words, per_layer, root = gp.prove(SEED, MAC_SEED, PAD_SEED)
        corr = [[gp.correction(l, w) for w in range(5)] for l in range(layers)]
        # a second proof of the same witness is the same proof
        again, _, root2 = gp.prove(SEED, MAC_SEED, PAD_SEED)
        assert np.array_equal(again, words) and root2 == root
    res = forward_model(OracleOps(oracle), tokens, model, luts, row_shift=1)
    sch = Schedule(oracle, luts, t)
    assert per_layer * layers == words.shape[0]
    for l in range(layers):
        exp = sch.layer(res["layers"][l], model.layers[l], SEED, l)
        got = words[l * per_layer:(l + 1) * per_layer]
        assert got.shape == exp.shape, (l, got.shape, exp.shape)
        bad = np.nonzero(np.any(got != exp, axis=1))[0]
        assert bad.size == 0, f"layer {l}: first differing word {bad[:8]}"
        for w, e in enumerate(sch.corrections(res["layers"][l], MAC_SEED, l)):
            assert np.array_equal(corr[l][w], e), (l, w)
    assert root == pcs_root(oracle, model, PAD_SEED)


def test_proof_needs_the_stable_softmax(prover):
    from volta_zk_b200 import accel, gpt2

    model = gpt2.synthetic_model(n_layers=1)
    with gpt2.Gpt2Session(prover, model, 8, params=gpt2.LutParams(softmax_row_shift=False)) as s:
        with pytest.raises(accel.AccelError):
            gpt2.Gpt2Prover(s)
