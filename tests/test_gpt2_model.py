"""GPT-2 small synthetic model (config 0/3): the package's input synthesis
and the oracle's whole-model forward against the reference's own NumPy
mirror (scripts/gpt2_fixed.py forward_model), through the digests that
tests/golden/make_model_golden.py recorded from it."""

import hashlib
import os

import numpy as np
import pytest

from oracle.gpt2 import OracleOps, forward_model

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LAYER_KEYS = ["row_shift", "ln1_out", "qkv_acc", "q", "k", "v", "scores_acc", "scores_q", "exp_out", "denoms",
              "recips", "av_acc", "av_q", "proj_acc", "attn_proj_q", "attn_block_out", "ln2_out", "ffn_up_acc",
              "ffn_up_q", "gelu_out", "ffn_down_acc", "ffn_down_q", "ffn_block_out"]
DTYPES = {"row_shift": np.int64, "denoms": np.int64, "recips": np.int16, "logits": np.int64}


def digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def golden(t):
    return np.load(os.path.join(GOLDEN_DIR, f"gpt2_model_t{t}.npz"))


def mismatches(g, embed_out, layers, final_ln_out, logits):
    """Names whose digest differs from the fixture.  `layers` maps a layer
    index to a callable name -> array (int64 accumulators, int16 wires)."""
    bad = []
    if digest(np.asarray(embed_out, np.int16)) != str(g["embed_out"]):
        bad.append("embed_out")
    n_layers = sum(1 for k in g.files if k.endswith("_ffn_block_out"))
    for layer in range(n_layers):
        keys = LAYER_KEYS if f"l{layer}_ln1_out" in g.files else ["attn_block_out", "ffn_block_out"]
        for k in keys:
            a = layers(layer, k)
            dt = DTYPES.get(k, np.int64 if k.endswith("_acc") else np.int16)
            if digest(np.asarray(a).astype(dt)) != str(g[f"l{layer}_{k}"]):
                bad.append(f"l{layer}_{k}")
    if digest(np.asarray(final_ln_out, np.int16)) != str(g["final_ln_out"]):
        bad.append("final_ln_out")
    if digest(np.asarray(logits, np.int64)) != str(g["logits"]):
        bad.append("logits")
    return bad


@pytest.fixture(scope="module")
def model():
    from volta_zk_b200 import gpt2

    return gpt2.synthetic_model()


def test_synthetic_model_matches_reference_generators(model, package_built):
    from volta_zk_b200 import gpt2

    g = golden(16)
    cat = np.concatenate([np.concatenate([lw[k].ravel() for k in ("c_attn", "attn_proj", "ffn_up", "ffn_down",
                                                                   "ln1_gain", "ln1_bias", "ln2_gain", "ln2_bias")])
                          for lw in model.layers])
    assert digest(cat) == str(g["weights_digest"])
    assert digest(model.wte) == str(g["wte_digest"])
    assert digest(model.wpe) == str(g["wpe_digest"])
    assert digest(gpt2.prefill_tokens(16)) == str(g["tokens_digest"])
    assert digest(gpt2.prefill_tokens(1024)) == str(golden(1024)["tokens_digest"])


def test_luts_match_reference_tables():
    from volta_zk_b200 import gpt2

    fx = np.load(os.path.join(GOLDEN_DIR, "fixed_layer_t8.npz"))
    luts = gpt2.build_luts()
    for k in ("exp", "gelu", "ln_rsqrt", "softmax_recip"):
        assert np.array_equal(luts[k], fx[k]), k


def test_reference_needs_the_stable_softmax_at_1024():
    """The recorded mirror run at T = 1024 is strict-clean with the P5 stable
    softmax; with LutParams::default the reference stops there (layer.rs:782)."""
    g = golden(1024)
    assert bool(g["strict_ok"]) and bool(g["softmax_row_shift"])


def test_oracle_forward_matches_reference_mirror_t16(oracle, model, package_built):
    from volta_zk_b200 import gpt2

    t = 16
    tokens = gpt2.prefill_tokens(t)
    res = forward_model(OracleOps(oracle), tokens, model, gpt2.build_luts(), row_shift=1)
    assert all(e == 0 for e in res["errors"])
    bad = mismatches(golden(t), res["embed_out"], lambda l, k: res["layers"][l][k], res["final_ln_out"],
                     res["logits"])
    assert not bad, bad


@pytest.fixture(scope="module")
def model2():
    from volta_zk_b200 import gpt2

    return gpt2.synthetic_model(n_layers=2)


def test_oracle_decode_equals_the_full_forward(oracle, model2, package_built):
    """decode.rs's own invariant (decode_matches_full_forward) on the oracle:
    greedy KV-cached steps after a prefill give the same logits rows and K/V
    rows as full forwards over the growing sequence (2-layer synthetic model)."""
    from oracle.gpt2 import argmax_last, generate
    from volta_zk_b200 import gpt2

    ops, luts = OracleOps(oracle), gpt2.build_luts()
    t0, n = 6, 3
    tokens = list(gpt2.prefill_tokens(t0))
    pre = forward_model(ops, np.array(tokens, np.uint32), model2, luts, row_shift=1)
    gen, rows, cache, errs = generate(ops, model2, luts, [r["k"] for r in pre["layers"]],
                                      [r["v"] for r in pre["layers"]], t0, pre["logits"], n)
    assert all(e == 0 for e in errs)
    assert gen[0] == argmax_last(pre["logits"])
    seq = tokens
    for i in range(n):
        seq = seq + [gen[i]]
        full = forward_model(ops, np.array(seq, np.uint32), model2, luts, row_shift=1)
        assert np.array_equal(np.asarray(full["logits"]).reshape(-1), rows[i]), i
        for l in range(2):
            assert np.array_equal(cache["k"][l][:len(seq) * 768], np.asarray(full["layers"][l]["k"]).reshape(-1))
            assert np.array_equal(cache["v"][l][:len(seq) * 768], np.asarray(full["layers"][l]["v"]).reshape(-1))
        if i + 1 < n:
            assert gen[i + 1] == argmax_last(rows[i])


def test_oracle_band_witness_invariants(oracle, model2, package_built):
    """band.rs's band_extraction_consistency on the oracle: band windows, and
    the band's last logits / final-LN row equal the full forward's."""
    from oracle.gpt2 import band_witness
    from volta_zk_b200 import gpt2

    ops, luts = OracleOps(oracle), gpt2.build_luts()
    t, t0 = 9, 5
    full = forward_model(ops, gpt2.prefill_tokens(t), model2, luts, row_shift=1)
    band = band_witness(ops, full, model2, luts, t0)
    q = t - t0
    assert band["layers"][0]["scores_q"].size == 12 * sum(t0 + r + 1 for r in range(q))
    assert np.array_equal(band["logits"][-1], np.asarray(full["logits"]).reshape(-1))
    assert np.array_equal(band["fin"][5][-768:], np.asarray(full["final_ln_out"]).reshape(-1))
    assert np.array_equal(band["layers"][1]["k"], np.asarray(full["layers"][1]["k"]).reshape(-1)[t0 * 768:])


def test_argmax_keeps_the_last_maximum():
    from oracle.gpt2 import argmax_last

    assert argmax_last([1, 5, 3, 5, 2]) == 3
    assert argmax_last([7]) == 0
    assert argmax_last([-4, -4]) == 1


def test_oracle_band_av_factors_evaluate_the_band_contraction(oracle, model2, package_built):
    """The band schedule's A.V factors: sum over (head, key) of A B C equals
    the multilinear value of the band's attention-value accumulators
    av_acc(r_i, r_h, r_c) (band rows i, heads h, head dimensions c), so the
    band packing (row i: window t0 + i + 1 at i t0 + i (i + 1) / 2) and the
    key range (all t0 + q cached V rows) are consistent with the forward."""
    from oracle.gpt2 import P, Schedule, band_witness, fp2_mul
    from volta_zk_b200 import gpt2

    ops, luts = OracleOps(oracle), gpt2.build_luts()
    t, t0 = 11, 6
    full = forward_model(ops, gpt2.prefill_tokens(t), model2, luts, row_shift=1)
    band = band_witness(ops, full, model2, luts, t0)
    q = t - t0
    sch = Schedule(oracle, luts, q, t0, chunk=1)
    assert (sch.tp, sch.sp, sch.rect) == (8, 16, 16 * 8 * 16)
    stream = oracle.FpStream(bytes([0x33] * 32), 7)
    rc = [stream.next_fp2() for _ in range(6)]
    rh = [stream.next_fp2() for _ in range(4)]
    ri = [stream.next_fp2() for _ in range(3)]
    eq_c, eq_h, eq_i = sch.eq(rc), sch.eq(rh), sch.eq(ri)
    lay = band["layers"][1]
    A, B, C = sch.av_factors(lay["weights"], full["layers"][1]["v"], eq_i, eq_c, eq_h)
    total = (0, 0)
    for a, b, c in zip(A, B, C):
        x = fp2_mul(fp2_mul(a, b), c)
        total = ((total[0] + x[0]) % P, (total[1] + x[1]) % P)
    acc = np.asarray(lay["av_acc"], np.int64).reshape(q, 768)
    want = (0, 0)
    for i in range(q):
        for h in range(12):
            for c in range(64):
                v = int(acc[i, h * 64 + c]) % P
                e = fp2_mul(fp2_mul(eq_i[i], eq_h[h]), eq_c[c])
                want = ((want[0] + e[0] * v) % P, (want[1] + e[1] * v) % P)
    assert total == want
