"""The scaled synthetic shape of the decode/scaling configuration (24
layers, d_model 1024, 16 heads of 64, MLP 4096; gpt2.GPT2_SCALED) through
the same device session and proof schedule as GPT-2 small, against the
oracle: the witness forward wire for wire, the proof word for word, the
boundary corrections and the weight commitment's root, including a
commitment past GPT2_FULL's 8192 rows (the rows grow to the next power of
two that holds the weights)."""

import numpy as np
import pytest

from oracle.gpt2 import OracleOps, Schedule, forward_model, pcs_root, pcs_rows

pytestmark = pytest.mark.gpu
SEED, MAC_SEED, PAD_SEED = bytes([0x50] * 32), bytes([0x4D] * 32), bytes([0x11] * 32)


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


@pytest.mark.parametrize("t", [16, 100])
def test_scaled_forward_and_proof_match_oracle(prover, oracle, t):
    from volta_zk_b200 import gpt2

    layers = 2
    model = gpt2.synthetic_model(n_layers=layers, shape=gpt2.GPT2_SCALED)
    assert model.shape.d == 1024 and model.shape.heads == 16 and model.shape.dff == 4096
    luts = gpt2.build_luts()
    tokens = gpt2.prefill_tokens(t)
    res = forward_model(OracleOps(oracle), tokens, model, luts, row_shift=1)
    assert not any(int(np.asarray(e).reshape(-1)[0]) for e in res["errors"] if np.size(e))
    with gpt2.Gpt2Session(prover, model, t) as s, gpt2.Gpt2Prover(s) as gp:
        s.forward(tokens)
        assert s.error_word() == 0
        assert np.array_equal(s.logits(), np.asarray(res["logits"]).reshape(-1))
        for l in range(layers):
            for name in gpt2.WIRES:
                if name in res["layers"][l]:
                    exp = np.asarray(res["layers"][l][name]).reshape(-1)
                    got = s.wire(l, name)
                    assert np.array_equal(got.astype(np.int64), exp.astype(np.int64)), (l, name)
        words, per_layer, root = gp.prove(SEED, MAC_SEED, PAD_SEED)
        corr = [[gp.correction(l, w) for w in range(5)] for l in range(layers)]
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


def test_scaled_commitment_past_8192_rows(prover, oracle):
    """Eight scaled layers hold 153 M weights: 16384 rows of 2^14.  The
    commitment alone (no layer units) equals the oracle's root."""
    from volta_zk_b200 import gpt2

    model = gpt2.synthetic_model(n_layers=8, shape=gpt2.GPT2_SCALED)
    total = sum(w.size for lw in model.layers for w in lw.values()) + model.wte.size + model.wpe.size + 2 * 1024
    assert pcs_rows(total) == 16384
    t = 8
    with gpt2.Gpt2Session(prover, model, t) as s, gpt2.Gpt2Prover(s) as gp:
        s.forward(gpt2.prefill_tokens(t))
        words, sites, root = gp.prove_units(SEED, MAC_SEED, PAD_SEED, [], True)
        assert words.shape[0] == 0 and sites == []
    assert root == pcs_root(oracle, model, PAD_SEED)


def test_too_many_heads_rejected(prover):
    """The attention sumchecks pad heads to 16: a 32-head model is refused
    when the prover opens, before any launch."""
    from volta_zk_b200 import accel, gpt2

    shape = gpt2.Gpt2Shape(layers=1, d=2048, heads=32, dff=256, vocab=64, positions=16)
    model = gpt2.synthetic_model(shape=shape)
    with gpt2.Gpt2Session(prover, model, 4) as s:
        with pytest.raises(accel.AccelError, match="16 heads"):
            gpt2.Gpt2Prover(s)


@pytest.mark.parametrize("shape,layers,world", [("small", 2, 2), ("small", 2, 8), ("scaled", 8, 4)])
def test_row_split_commitment_equals_the_whole(prover, shape, layers, world):
    """The weight commitment split by rows over `world` GPUs (the ranks take
    turns on one device; the all-to-all and all-gather are array moves):
    each rank's column chaining values, its slab subtree and the top levels
    give the one-GPU root."""
    from volta_zk_b200 import gpt2, sharded

    sh = gpt2.GPT2_SCALED if shape == "scaled" else gpt2.GPT2_SMALL
    model = gpt2.synthetic_model(n_layers=layers, shape=sh)
    be = prover.backend
    with gpt2.Gpt2Session(prover, model, 8) as s, gpt2.Gpt2Prover(s) as gp:
        s.forward(gpt2.prefill_tokens(8))
        _, _, whole = gp.prove_units(SEED, MAC_SEED, PAD_SEED, [], True)
        rows, code_len = gp.pcs_rows(), 1 << 15
        rl, slab = rows // world, code_len // world
        cvs = [gp.commit_rows(PAD_SEED, g * rl, rl).reshape(world, slab, 32) for g in range(world)]
        roots = []
        for g in range(world):
            recv = np.stack([cvs[src][g] for src in range(world)])
            tree, root = sharded.ligero_shard_tree(be, recv, world, slab)
            be.free(tree)
            roots.append(np.frombuffer(root.tobytes(), np.uint8))
        top = sharded.ligero_top_tree(be, np.stack(roots))
        assert top[-1].tobytes() == whole
        with pytest.raises(Exception, match="row block"):
            gp.commit_rows(PAD_SEED, 64, 128)
