"""Load-balanced expert placement for expert parallelism (host logic, CPU):
the placement is a permutation with E / world experts per rank, it lowers
the largest per-rank load under skewed (Zipf) routing, and the renumbered
layer computes the same outputs as the original through the CPU oracle."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for _p in (os.path.join(ROOT, "burn-extended_b200"), os.path.join(ROOT, "oracle"), HERE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import oracle  # noqa: E402
from mxmoe import ep, synth  # noqa: E402
from moe_testutil import assert_close  # noqa: E402


def _rank_loads(loads, order, world):
    per = len(order) // world
    return np.array([loads[order[r * per:(r + 1) * per]].sum() for r in range(world)])


def test_placement_is_balanced_permutation():
    inp = synth.make_inputs(256, 256, 128, 4, 2048, True, seed=5, zipf_router_bias=1.1)
    loads = ep.expert_loads(inp.x, inp.gamma, inp.gate_w, inp.gate_b, inp.k)
    assert loads.sum() == inp.n * inp.k
    for world in (2, 4, 8):
        order = ep.balanced_placement(loads, world)
        assert sorted(order.tolist()) == list(range(inp.E))
        per = inp.E // world
        for r in range(world):
            part = order[r * per:(r + 1) * per]
            assert list(part) == sorted(part)
        contiguous = _rank_loads(loads, np.arange(inp.E), world).max()
        balanced = _rank_loads(loads, order, world)
        # no rank above the mean by more than the largest single expert
        assert balanced.max() <= loads.sum() / world + loads.max()
        assert balanced.max() < contiguous


def test_placement_uniform_loads_keeps_equal_shares():
    order = ep.balanced_placement(np.full(32, 7), 4)
    assert sorted(order.tolist()) == list(range(32))
    assert (_rank_loads(np.full(32, 7), order, 4) == 56).all()


def test_renumbered_layer_same_outputs():
    inp = synth.make_inputs(128, 64, 8, 2, 24, True, seed=9, zipf_router_bias=1.1)
    c = oracle.cfg(inp.d, inp.f, inp.E, inp.k)
    want, idx, _ = oracle.moe_forward(c, inp.x, inp.gamma, inp.gate_w, inp.gate_b, inp.host.w1_blocks,
                                      inp.host.w1_scales, inp.b1, inp.host.w2_blocks, inp.host.w2_scales, inp.b2)
    order = ep.balanced_placement(ep.expert_loads(inp.x, inp.gamma, inp.gate_w, inp.gate_b, inp.k), 2)
    gw, gb, h, b1, b2 = ep.renumber_experts(order, inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2)
    got, idx2, _ = oracle.moe_forward(c, inp.x, inp.gamma, gw, gb, h.w1_blocks, h.w1_scales, b1, h.w2_blocks,
                                      h.w2_scales, b2)
    # the renumbered router picks the same experts under their new ids
    assert (np.sort(order[idx2], axis=1) == np.sort(idx, axis=1)).all()
    assert_close(got, want, "renumbered layer")


def test_replica_plan_and_replicated_layer():
    loads = np.array([100, 40, 10, 10, 0, 0, 0, 0])
    src = ep.plan_replicas(loads, 4)
    assert list(src[:8]) == list(range(8))
    # copies go to the largest load per copy: 100 -> 50 -> 40 (expert 1) -> 33.3 -> ...
    assert sorted(src[8:].tolist()) == [0, 0, 0, 1]
    groups = ep.replica_groups(src)
    assert sorted(sum(groups, [])) == list(range(12))
    order = ep.balanced_placement(np.array([loads[e] / np.count_nonzero(src == e) for e in src]), 4)
    g2 = ep.replica_groups(src, order)
    inv = np.argsort(order)
    assert sorted(g2[0]) == sorted(int(inv[s]) for s in np.flatnonzero(src == 0))
    # copy slots never win the router: the replicated layer routes and computes as the original
    inp = synth.make_inputs(128, 64, 8, 2, 24, True, seed=11, zipf_router_bias=1.1)
    c = oracle.cfg(inp.d, inp.f, inp.E, inp.k)
    want, idx, _ = oracle.moe_forward(c, inp.x, inp.gamma, inp.gate_w, inp.gate_b, inp.host.w1_blocks,
                                      inp.host.w1_scales, inp.b1, inp.host.w2_blocks, inp.host.w2_scales, inp.b2)
    src = ep.plan_replicas(ep.expert_loads(inp.x, inp.gamma, inp.gate_w, inp.gate_b, inp.k), 2)
    gw, gb, h, b1, b2 = ep.replicate_experts(src, inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2)
    c2 = oracle.cfg(inp.d, inp.f, len(src), inp.k)
    got, idx2, _ = oracle.moe_forward(c2, inp.x, inp.gamma, gw, gb, h.w1_blocks, h.w1_scales, b1, h.w2_blocks,
                                      h.w2_scales, b2)
    assert (idx2 < inp.E).all() and (idx2 == idx).all()
    assert_close(got, want, "replicated layer")


def test_replica_remap_gives_canonical_maps():
    import torch
    src = np.array([0, 1, 2, 3, 0, 0, 1, 2])
    rm = ep.ReplicaRemap(ep.replica_groups(src), "cpu")
    rng = np.random.default_rng(3)
    idx = torch.from_numpy(np.stack([rng.permutation(4)[:3] for _ in range(50)]).astype(np.int32))
    out = rm.apply(ep.Routed(None, idx, None, None, None, None))
    new = out.topk_idx.numpy()
    assert (src[new] == idx.numpy()).all()  # every pair stays on a copy of its expert
    for e, n_copies in ((0, 3), (1, 2), (2, 2), (3, 1)):
        used = np.unique(new[src[new] == e])
        assert len(used) == n_copies
    offs, perm, inv = oracle.permute(new, len(src))
    assert np.array_equal(offs, out.offsets.numpy())
    assert np.array_equal(perm, out.perm.numpy())
    assert np.array_equal(inv, out.inv.numpy())


def test_c_abi_placement_matches_python():
    """mxmoe_ep_plan_replicas / mxmoe_ep_balanced_placement (host-only C
    entry points, no GPU needed) give the Python mirror's results."""
    from mxmoe import _lib
    lib = _lib.lib()
    rng = np.random.default_rng(7)
    for E, world, extra in ((128, 8, 8), (32, 4, 4), (8, 2, 0), (12, 3, 3)):
        loads = rng.zipf(1.5, E).astype(np.float64)
        loads[::5] = loads[1]  # ties
        src = np.empty(E + extra, dtype=np.int32)
        assert lib.mxmoe_ep_plan_replicas(loads.ctypes.data, E, extra, src.ctypes.data) == 0
        assert np.array_equal(src, ep.plan_replicas(loads, extra))
        S = E + extra
        if S % world:
            continue
        sl = np.array([loads[e] / np.count_nonzero(src == e) for e in src], dtype=np.float64)
        order = np.empty(S, dtype=np.int32)
        assert lib.mxmoe_ep_balanced_placement(sl.ctypes.data, S, world, order.ctypes.data) == 0
        assert np.array_equal(order, ep.balanced_placement(sl, world))
    bad = np.empty(7, dtype=np.int32)
    assert lib.mxmoe_ep_balanced_placement(np.ones(7).ctypes.data, 7, 2, bad.ctypes.data) != 0
