"""Splitting one GPT-2 proof over GPUs by (layer, site) units
(gpt2.split_sites / assemble_units, the host side of bench.py's config-3
multi-GPU step): every sub-proof is dealt to exactly one GPU, the loads
balance, and the units' words reassemble to the one-GPU word order.  The
device side (prove_units against the one-GPU proof) is in
tests/test_gpu_gpt2_proof.py."""

import numpy as np
import pytest


def _span(per_rank, commit):
    from volta_zk_b200 import gpt2

    cost = {gpt2.ALL_SITES: gpt2.LAYER_COST, **gpt2.PART_COSTS}
    loads = []
    for g, units in enumerate(per_rank):
        load = gpt2.COMMIT_COST if g == commit else 0.0
        for _, m in units:
            # a rank holding both parts of a layer proves the whole layer
            load += cost[m]
        loads.append(load)
    return max(loads)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 5, 8, 12])
def test_split_covers_every_site_once_and_beats_the_layer_split(world):
    from volta_zk_b200 import gpt2

    per_rank, commit = gpt2.split_sites(world)
    assert len(per_rank) == world and 0 <= commit < world
    seen = {}
    for g, units in enumerate(per_rank):
        assert [l for l, _ in units] == sorted({l for l, _ in units})  # one unit per layer, in layer order
        for l, m in units:
            assert m in (gpt2.ALL_SITES, gpt2.PART_ATTENTION, gpt2.PART_REST)
            for k in [gpt2.SITE_CORRECTIONS] + gpt2.SITE_ORDER:
                if (m >> k) & 1:
                    assert (l, k) not in seen
                    seen[(l, k)] = g
    assert len(seen) == gpt2.LAYERS * (1 + len(gpt2.SITE_ORDER))
    # never slower (by the cost model) than whole layers round-robin with the
    # commitment on the least-loaded rank
    layers = [[(l, gpt2.ALL_SITES) for l in range(g, gpt2.LAYERS, world)] for g in range(world)]
    plain = _span(layers, min(range(world), key=lambda g: (len(layers[g]), -g)))
    assert _span(per_rank, commit) <= plain + 1e-9
    if world == 1:
        assert per_rank[0] == [(l, gpt2.ALL_SITES) for l in range(gpt2.LAYERS)]
    if world == 8:  # 12 layers: the commitment goes to a rank with one layer
        assert len(per_rank[commit]) == 1


def test_assemble_restores_layer_and_site_order():
    from volta_zk_b200 import gpt2

    rng = np.random.default_rng(5)
    n_words = {k: int(rng.integers(1, 6)) for k in gpt2.SITE_ORDER}

    def site_words(l, k):
        return np.full((n_words[k], 2), l * 100 + k, dtype=np.uint64)

    full = np.concatenate([site_words(l, k) for l in range(gpt2.LAYERS) for k in gpt2.SITE_ORDER])
    per_rank, _ = gpt2.split_sites(5)
    assert any(m != gpt2.ALL_SITES for units in per_rank for _, m in units)  # some layers in parts
    pieces = []
    for units in per_rank[::-1]:  # any order of the pieces
        words, sites = [], []
        for l, m in units:
            us = [(k, n_words[k]) for k in gpt2.SITE_ORDER if (m >> k) & 1]
            sites.append(us)
            words += [site_words(l, k) for k, _ in us]
        pieces.append((units, np.concatenate(words) if words else np.zeros((0, 2), np.uint64), sites))
    assert np.array_equal(gpt2.assemble_units(pieces), full)


def _rank_gather(rank, world, port, q):
    """Each gloo rank holds the words of its units (synthetic words that name
    their layer and site); sharded.gather_units rebuilds the whole proof in
    layer and site order on every rank."""
    import os

    import torch
    import torch.distributed as dist

    from volta_zk_b200 import gpt2, sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        n_words = {k: 1 + (k % 4) for k in gpt2.SITE_ORDER}
        split, _ = gpt2.split_sites(world)
        words, sites = [], []
        for l, m in split[rank]:
            us = [(k, n_words[k]) for k in gpt2.SITE_ORDER if (m >> k) & 1]
            sites.append(us)
            words += [np.full((n, 2), l * 100 + k, np.uint64) for k, n in us]
        mine = np.concatenate(words) if words else np.zeros((0, 2), np.uint64)
        got = sharded.gather_units(mine, sites, split, rank, world, dist, torch.device("cpu"), gpt2.LAYERS)
        full = np.concatenate([np.full((n_words[k], 2), l * 100 + k, np.uint64)
                               for l in range(gpt2.LAYERS) for k in gpt2.SITE_ORDER])
        q.put((rank, bool(np.array_equal(got, full))))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_units():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_gather, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_split_plan_never_slower_than_the_unit_commitment(world):
    """split_plan keeps the commitment on one GPU unless splitting it by rows
    is faster by the cost model; with it split, no rank commits alone."""
    from volta_zk_b200 import gpt2

    for layers, costs in ((gpt2.LAYERS, None), (24, gpt2.SCALED_COSTS)):
        per_rank, commit = gpt2.split_plan(world, layers, costs)
        unit, unit_commit = gpt2.split_sites(world, layers=layers, costs=costs)
        c = costs or (gpt2.LAYER_COST, gpt2.PART_COSTS, gpt2.COMMIT_COST)
        span = gpt2.split_span(per_rank, commit, c) + (c[2] / world + 1.0 if commit is None else 0.0)
        assert span <= gpt2.split_span(unit, unit_commit, c) + 1e-9
        if world & (world - 1):
            assert commit is not None
