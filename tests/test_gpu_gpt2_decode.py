"""Decode bands and KV-cached decoding on the device (config 4's witness):
the band witness of a forward against the oracle's band_witness
(rust/volta-gpt2/src/band.rs:77-196), greedy KV-cached decoding against the
oracle's decode_step / generate (decode.rs:137-300), and, at the
configuration's size (960-token prefill, 64 steps, 12 layers), decoding
against the band of the full 1024-token forward over the same tokens, as the
reference's own tests tie the two."""

import numpy as np
import pytest

from oracle.gpt2 import OracleOps, argmax_last, band_witness, forward_model, generate

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


@pytest.fixture(scope="module")
def model2():
    from volta_zk_b200 import gpt2

    return gpt2.synthetic_model(n_layers=2)


def test_band_witness_matches_oracle(prover, oracle, model2):
    from volta_zk_b200 import gpt2

    t, t0 = 16, 10
    luts = gpt2.build_luts()
    tokens = gpt2.prefill_tokens(t)
    full = forward_model(OracleOps(oracle), tokens, model2, luts, row_shift=1)
    exp = band_witness(OracleOps(oracle), full, model2, luts, t0)
    with gpt2.Gpt2Session(prover, model2, t) as s:
        s.forward(tokens)
        with s.band(t0) as band:
            for l in range(2):
                for name in gpt2.WIRES[:-1]:
                    got = band.wire(l, name)
                    want = np.asarray(exp["layers"][l][name]).reshape(-1)
                    assert np.array_equal(got.astype(np.int64), want.astype(np.int64)), (l, name)
            for k in range(6):
                assert np.array_equal(band.final_ln(k).astype(np.int64),
                                      np.asarray(exp["fin"][k]).reshape(-1).astype(np.int64)), k
            assert np.array_equal(band.logits(), exp["logits"])
            assert band.error_word() == 0
            # the band's last logits row is the full forward's last-position logits
            assert np.array_equal(band.logits()[-1], s.logits())


def test_band_rejects_improper_suffix(prover, model2):
    from volta_zk_b200 import accel, gpt2

    with gpt2.Gpt2Session(prover, model2, 8) as s:
        s.forward(gpt2.prefill_tokens(8))
        for t0 in (0, 8):
            with pytest.raises(accel.AccelError, match="proper suffix"):
                s.band(t0)


def test_decode_matches_oracle(prover, oracle, model2):
    from volta_zk_b200 import gpt2

    t0, n = 12, 4
    luts = gpt2.build_luts()
    tokens = gpt2.prefill_tokens(t0)
    with gpt2.Gpt2Session(prover, model2, t0) as s:
        s.forward(tokens)
        k_rows = [s.wire(l, "k") for l in range(2)]
        v_rows = [s.wire(l, "v") for l in range(2)]
        with s.decoder(n) as dec:
            dec.generate(2)
            dec.generate(n - 2)  # steps continue across calls
            got_tokens, got_rows = dec.tokens(), dec.logits()
            caches = [dec.cache(l, 0, t0 + n) for l in range(2)], [dec.cache(l, 1, t0 + n) for l in range(2)]
            assert dec.error_word() == 0
        exp_tokens, exp_rows, cache, errs = generate(OracleOps(oracle), model2, luts, k_rows, v_rows, t0,
                                                     s.logits(), n)
    assert list(got_tokens) == exp_tokens
    assert np.array_equal(got_rows, exp_rows)
    for l in range(2):
        assert np.array_equal(caches[0][l], cache["k"][l])
        assert np.array_equal(caches[1][l], cache["v"][l])
    assert all(e == 0 for e in errs)


def test_decode_960_plus_64_equals_band_of_full_forward(prover, oracle):
    """Config 4's witness at size: 64 greedy KV-cached steps after a
    960-token prefill (12 layers) give the logits rows and K/V rows of the
    band 960 .. 1023 of one full 1024-token forward over the same tokens; the
    first two steps also equal the oracle's decode from the device's caches."""
    from volta_zk_b200 import gpt2

    t0, n = 960, 64
    model = gpt2.synthetic_model()
    luts = gpt2.build_luts()
    tokens = gpt2.prefill_tokens(t0)
    with gpt2.Gpt2Session(prover, model, t0) as s:
        s.forward(tokens)
        pre_logits = s.logits()
        k0 = [s.wire(l, "k") for l in range(gpt2.LAYERS)]
        v0 = [s.wire(l, "v") for l in range(gpt2.LAYERS)]
        with s.decoder(n) as dec:
            dec.generate(n)
            gen, rows = dec.tokens(), dec.logits()
            kc = [dec.cache(l, 0, t0 + n) for l in range(gpt2.LAYERS)]
            vc = [dec.cache(l, 1, t0 + n) for l in range(gpt2.LAYERS)]
            assert dec.error_word() == 0
    assert gen[0] == argmax_last(pre_logits)
    assert all(gen[i + 1] == argmax_last(rows[i]) for i in range(n - 1))
    with gpt2.Gpt2Session(prover, model, t0 + n) as s2:
        s2.forward(np.concatenate([tokens, gen]).astype(np.uint32))
        assert s2.error_word() == 0
        with s2.band(t0) as band:
            assert np.array_equal(band.logits(), rows)
            for l in range(gpt2.LAYERS):
                assert np.array_equal(band.wire(l, "k"), kc[l][t0 * gpt2.D:]), l
                assert np.array_equal(band.wire(l, "v"), vc[l][t0 * gpt2.D:]), l
    exp_tokens, exp_rows, _, errs = generate(OracleOps(oracle), model, luts, k0, v0, t0, pre_logits, 2)
    assert exp_tokens == list(gen[:2]) and np.array_equal(exp_rows, rows[:2])
    assert all(e == 0 for e in errs)
