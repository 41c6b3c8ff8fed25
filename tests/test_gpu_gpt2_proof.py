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


@pytest.mark.parametrize("t,t0,chunk", [(16, 10, 1), (100, 93, 3)])
def test_band_proof_matches_oracle_composition(prover, oracle, t, t0, chunk):
    """A decode band's proof (rows t0 .. t-1 of a t-token forward, attention
    over all t keys) against the oracle's band schedule over the oracle's
    band witness, with the full forward's K and V as the cache: every word
    and every boundary correction.  Non-power-of-two q and s included."""
    from oracle.gpt2 import band_witness
    from volta_zk_b200 import gpt2

    layers = 2
    model = gpt2.synthetic_model(n_layers=layers)
    luts = gpt2.build_luts()
    tokens = gpt2.prefill_tokens(t)
    with gpt2.Gpt2Session(prover, model, t) as s, gpt2.Gpt2Prover(s) as gp:
        s.forward(tokens)
        pre, _, root = gp.prove(SEED, MAC_SEED, PAD_SEED)
        with s.band(t0) as band:
            words, per_layer = gp.prove_band(band, chunk, SEED, MAC_SEED)
            corr = [[gp.correction(l, w) for w in range(5)] for l in range(layers)]
            other, _ = gp.prove_band(band, chunk + 1, SEED, MAC_SEED)
            half, _ = gp.prove_band(band, chunk, SEED, MAC_SEED, first=1, stride=2)
        # the prefill proof is untouched by the band proofs
        again, _, root2 = gp.prove(SEED, MAC_SEED, PAD_SEED)
        assert np.array_equal(again, pre) and root2 == root
    assert not np.array_equal(other, words)  # chunks have their own transcripts
    assert np.array_equal(half, words[per_layer:2 * per_layer])
    ops = OracleOps(oracle)
    full = forward_model(ops, tokens, model, luts, row_shift=1)
    bw = band_witness(ops, full, model, luts, t0)
    sch = Schedule(oracle, luts, t - t0, t0, chunk)
    assert per_layer * layers == words.shape[0]
    for l in range(layers):
        kv = (full["layers"][l]["k"], full["layers"][l]["v"])
        exp = sch.layer(bw["layers"][l], model.layers[l], SEED, l, kv=kv)
        got = words[l * per_layer:(l + 1) * per_layer]
        assert got.shape == exp.shape, (l, got.shape, exp.shape)
        bad = np.nonzero(np.any(got != exp, axis=1))[0]
        assert bad.size == 0, f"layer {l}: first differing word {bad[:8]}"
        for w, e in enumerate(sch.corrections(bw["layers"][l], MAC_SEED, l)):
            assert np.array_equal(corr[l][w], e), (l, w)


def test_band_proof_rejects_bad_chunk_and_foreign_band(prover):
    from volta_zk_b200 import accel, gpt2

    model = gpt2.synthetic_model(n_layers=1)
    with gpt2.Gpt2Session(prover, model, 8) as s, gpt2.Gpt2Session(prover, model, 8) as s2, \
            gpt2.Gpt2Prover(s) as gp:
        s.forward(gpt2.prefill_tokens(8))
        s2.forward(gpt2.prefill_tokens(8))
        with s.band(4) as band, s2.band(4) as foreign:
            with pytest.raises(accel.AccelError, match="chunk"):
                gp.prove_band(band, 0, SEED, MAC_SEED)
            with pytest.raises(accel.AccelError, match="session"):
                gp.prove_band(foreign, 1, SEED, MAC_SEED)


@pytest.mark.parametrize("split", ["world2", "world8", "parts", "sites"])
def test_site_units_reassemble_the_proof(prover, split):
    """A proof split over GPUs by (layer, site) units (the ranks taking turns
    on one device): gpt2.split_sites' splits, a split into layer parts and
    one into single sites.  The units' words reassemble to the one-GPU proof,
    the committing rank's root is the one-GPU root, and each layer's
    corrections come from the rank holding its site 0."""
    from volta_zk_b200 import gpt2

    t, layers = 16, 2
    model = gpt2.synthetic_model(n_layers=layers)
    with gpt2.Gpt2Session(prover, model, t) as s, gpt2.Gpt2Prover(s) as gp:
        s.forward(gpt2.prefill_tokens(t))
        full, _, root = gp.prove(SEED, MAC_SEED, PAD_SEED)
        corr = [[gp.correction(l, w) for w in range(5)] for l in range(layers)]
        if split.startswith("world"):
            per_rank, commit = gpt2.split_sites(int(split[5:]), t, layers=layers)
        elif split == "parts":
            per_rank = [[(0, gpt2.ALL_SITES), (1, gpt2.PART_REST)], [(1, gpt2.PART_ATTENTION)], []]
            commit = 2
        else:  # every site of layer 1 its own unit on its own rank, layer 0 whole
            per_rank = [[(0, gpt2.ALL_SITES)]] + [[(1, 1 << k)] for k in [0] + gpt2.SITE_ORDER]
            commit = 1
        pieces = []
        for g, units in enumerate(per_rank):
            words, sites, r = gp.prove_units(SEED, MAC_SEED, PAD_SEED, units, g == commit)
            if g == commit:
                assert r == root
            pieces.append((units, words, sites))
            for l, m in units:
                if m & 1:
                    for w in range(5):
                        assert np.array_equal(gp.correction(l, w), corr[l][w])
    assert np.array_equal(gpt2.assemble_units(pieces, layers=layers), full)


def test_correction_sink_receives_every_correction(prover):
    """With a correction sink the proof copies every boundary correction to
    pinned host memory while later layers compute (download_async on the
    second copy stream); after prove returns the sink equals the resident
    corrections, proof after proof, and the words are unchanged."""
    import torch

    from volta_zk_b200 import gpt2

    t, layers = 16, 2
    model = gpt2.synthetic_model(n_layers=layers)
    with gpt2.Gpt2Session(prover, model, t) as s, gpt2.Gpt2Prover(s) as gp:
        s.forward(gpt2.prefill_tokens(t))
        plain, _, _ = gp.prove(SEED, MAC_SEED, PAD_SEED)
        sink = torch.zeros(layers * 5 * t * gpt2.D, dtype=torch.int64).pin_memory().numpy().view(np.uint64)
        gp.set_correction_sink(sink)
        for mac in (MAC_SEED, bytes([0x4E] * 32)):
            sink[:] = 0
            words, _, _ = gp.prove(SEED, mac, PAD_SEED)
            assert np.array_equal(words, plain)
            got = sink.reshape(layers, 5, -1)
            for l in range(layers):
                for w in range(5):
                    assert np.array_equal(got[l, w], gp.correction(l, w)), (l, w)
        gp.set_correction_sink(None)
