"""VOLE-MAC correlations of the mock backend, prover and verifier halves
(oracle/blind.py): prover tags (draw_sub_tags, rust/volta-mac/src/corr.rs:
1896-1915), verifier keys (expand_sub_keys / auth_verifier, corr.rs:2343-2357
and auth.rs:35-69), full-field draws and keys (corr.rs:1930-1978, 2480-2486).

The FpStream these draw from is pinned to the reference's ChaCha8 goldens in
test_oracle_golden.py; here the halves are checked against each other
through the MAC relation k = m + delta x of every authenticated value, on
random values and on the GPT-2 boundary corrections the prover emits."""

import numpy as np
import pytest

from oracle import blind as ob

P = 0xFFFFFFFF00000001
SEED = bytes([0x4D] * 32)
DELTA = (0x1234_5678_9ABC_DEF0 % P, 0x0FED_CBA9_8765_4321)


def test_sub_masks_are_the_epilogue_mask_rows(oracle):
    dom = (7 << 32) | 3
    assert ob.sub_masks(oracle, SEED, dom, 40) == [int(x) for x in oracle.chacha_fp_rows(SEED, dom, 1, 40)[0]]


def test_sub_tags_live_in_the_tag_domain(oracle):
    dom = (9 << 32) | 1
    tags = ob.sub_tags(oracle, SEED, dom, 5)
    s = oracle.FpStream(SEED, dom | ob.TAG_BIT)
    assert tags == [s.next_fp2() for _ in range(5)]
    assert tags != ob.full_corrs(oracle, SEED, dom, 5)


def test_auth_verifier_keys_satisfy_the_mac_relation(oracle):
    """auth_prover publishes c = x - r; the verifier's key k_r + delta c then
    satisfies k = m + delta x for the prover's tag m of the same slot."""
    rng = np.random.default_rng(5)
    dom, n = (3 << 32) | 11, 64
    x = [int(v) for v in rng.integers(-32768, 32768, size=n)]
    r = ob.sub_masks(oracle, SEED, dom, n)
    corr = [(xi - ri) % P for xi, ri in zip(x, r)]
    tags = ob.sub_tags(oracle, SEED, dom, n)
    keys = ob.auth_verifier(oracle, SEED, dom, corr, DELTA)
    assert ob.mac_holds(tags, keys, x, DELTA)
    # a wrong correction, a wrong value or another delta breaks it
    bad = list(corr)
    bad[17] = (bad[17] + 1) % P
    assert not ob.mac_holds(tags, ob.auth_verifier(oracle, SEED, dom, bad, DELTA), x, DELTA)
    assert not ob.mac_holds(tags, keys, x[:5] + [x[5] + 1] + x[6:], DELTA)
    assert not ob.mac_holds(tags, ob.auth_verifier(oracle, SEED, dom, corr, (DELTA[0], DELTA[1] + 1)), x, DELTA)


def test_full_field_keys_authenticate_corrected_values(oracle):
    """A full-field correction v - x (the blind LogUp corrections) moves the
    key by delta (v - x): k_v = m + delta v for the tag m of the draw."""
    dom, n = 0x5_0000_0021, 6
    corrs = ob.full_corrs(oracle, SEED, dom, n)
    keys = ob.full_keys(oracle, SEED, dom, n, DELTA)
    rng = np.random.default_rng(9)
    for (x, m), k in zip(corrs, keys):
        assert k == ob.add(ob.f2(m), ob.mul(DELTA, x))
        v = tuple(int(a) for a in rng.integers(0, P, size=2, dtype=np.uint64))
        c = ob.sub(v, x)
        assert ob.add(k, ob.mul(DELTA, c)) == ob.add(ob.f2(m), ob.mul(DELTA, v))


def test_gpt2_boundary_corrections_verify(oracle, package_built):
    """The GPT-2 layer proof's boundary corrections (x_in, k, v, attention
    and FFN block outputs, mask domain ((layer * 8 + w) << 32) | row) are
    accepted by the verifier half against the forward's wire values.  The
    device emits the same corrections word for word (test_gpu_gpt2_proof)."""
    from oracle.gpt2 import OracleOps, Schedule, forward_model
    from volta_zk_b200 import gpt2

    t = 4
    model = gpt2.synthetic_model(n_layers=1)
    luts = gpt2.build_luts()
    res = forward_model(OracleOps(oracle), gpt2.prefill_tokens(t), model, luts, row_shift=1)
    lay = res["layers"][0]
    corr = Schedule(oracle, luts, t).corrections(lay, SEED, 0)
    names = ("x_in", "k", "v", "attn_block_out", "ffn_block_out")
    for w, name in enumerate(names):
        x = np.asarray(lay[name]).reshape(t, 768)
        for row in (0, t - 1):
            dom = (w << 32) | row
            c = [int(v) for v in corr[w].reshape(t, 768)[row]]
            tags = ob.sub_tags(oracle, SEED, dom, 768)
            keys = ob.auth_verifier(oracle, SEED, dom, c, DELTA)
            assert ob.mac_holds(tags, keys, [int(v) for v in x[row]], DELTA), (name, row)
