"""The scaled synthetic shape (gpt2.GPT2_SCALED: 24 layers, d_model 1024,
16 heads of 64, MLP 4096) on the CPU: the package's synthetic weights and
the oracle's forward against the reference's own NumPy mirror run at that
shape (tests/golden/make_model_golden.py --scaled: the first 2 layers at
T = 16, every wire of both), the oracle decode invariant at that shape, the
weight-commitment row rule, and the split of its 24 layers over GPUs."""

import numpy as np
import pytest

from oracle.gpt2 import OracleOps, forward_model, pcs_rows
from tests.test_gpt2_model import GOLDEN_DIR, digest, mismatches


@pytest.fixture(scope="module")
def scaled2():
    from volta_zk_b200 import gpt2

    return gpt2.synthetic_model(n_layers=2, shape=gpt2.GPT2_SCALED)


def golden():
    import os

    return np.load(os.path.join(GOLDEN_DIR, "gpt2_scaled_t16.npz"))


def test_scaled_weights_match_reference_generators(scaled2):
    from volta_zk_b200 import gpt2

    g = golden()
    sh = scaled2.shape
    assert (sh.layers, sh.d, sh.heads, sh.head_dim, sh.dff, sh.vocab, sh.positions) == (2, 1024, 16, 64, 4096,
                                                                                        50257, 1024)
    cat = np.concatenate([np.concatenate([lw[k].ravel() for k in ("c_attn", "attn_proj", "ffn_up", "ffn_down",
                                                                   "ln1_gain", "ln1_bias", "ln2_gain", "ln2_bias")])
                          for lw in scaled2.layers])
    assert digest(cat) == str(g["weights_digest"])
    assert digest(scaled2.wte) == str(g["wte_digest"])
    assert digest(scaled2.wpe) == str(g["wpe_digest"])


def test_oracle_scaled_forward_matches_reference_mirror(oracle, scaled2, package_built):
    from volta_zk_b200 import gpt2

    g = golden()
    assert bool(g["strict_ok"])
    tokens = gpt2.prefill_tokens(16)
    res = forward_model(OracleOps(oracle), tokens, scaled2, gpt2.build_luts(), row_shift=1)
    assert all(e == 0 for e in res["errors"])
    bad = mismatches(g, res["embed_out"], lambda l, k: res["layers"][l][k], res["final_ln_out"], res["logits"])
    assert not bad, bad


def test_weight_commitment_rows():
    """8192 rows (GPT2_FULL) while the weights fit; past that the power of
    two they fill: 8 scaled layers -> 16384, the whole scaled model (355 M
    weights) -> 32768."""
    from volta_zk_b200 import gpt2

    def total(shape, layers):
        d, f = shape.d, shape.dff
        return layers * (4 * d * d + 2 * d * f + 4 * d) + (shape.vocab + shape.positions) * d + 2 * d

    assert pcs_rows(total(gpt2.GPT2_SMALL, 12)) == 8192
    assert pcs_rows(8192 << 14) == 8192 and pcs_rows((8192 << 14) + 1) == 16384
    assert pcs_rows(total(gpt2.GPT2_SCALED, 8)) == 16384
    assert pcs_rows(total(gpt2.GPT2_SCALED, 24)) == 32768


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_scaled_split_covers_24_layers(world):
    from volta_zk_b200 import gpt2

    per_rank, commit = gpt2.split_sites(world, layers=24, costs=gpt2.SCALED_COSTS)
    assert len(per_rank) == world and 0 <= commit < world
    seen = set()
    for units in per_rank:
        for l, m in units:
            for k in [gpt2.SITE_CORRECTIONS] + gpt2.SITE_ORDER:
                if (m >> k) & 1:
                    assert (l, k) not in seen
                    seen.add((l, k))
    assert len(seen) == 24 * (1 + len(gpt2.SITE_ORDER))
