"""Expert-parallel entry points on one GPU: the layer's experts split over
several shard layers on the same device, the dispatch emulated by slicing
(no collective), against the single-layer forward and the oracle."""
import pytest

import mxmoe
from moe_testutil import assert_close, make_layer, oracle_forward, to_device_x
from mxmoe import synth
from mxmoe.ep import CudaExpertBackend, shard_bounds

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,n", [(2, 200), (4, 200), (2, 1), (4, 1)])
def test_sharded_layers_match_full_layer(world, n):
    """n = 1: every shard runs at most four routed pairs through the
    dequant-GEMV's non-fused mode (permutation maps in, y_pair rows out),
    the full layer through its fused mode."""
    import torch
    inp = synth.make_inputs(1024, 512, 8, 4, n, True, seed=21)
    full = make_layer(inp)
    x = to_device_x(inp)
    y_full = full.forward(x, out_dtype=torch.float32)
    cfg = mxmoe.MoeConfig(inp.d, inp.f, inp.E, inp.k)
    shards = []
    for r in range(world):
        b, c = shard_bounds(inp.E, world, r)
        shards.append(CudaExpertBackend(cfg, "cuda:0", b, c, inp.gamma, inp.gate_w, inp.gate_b, inp.host,
                                        inp.b1, inp.b2, pair_dtype=torch.float32))
    src = shards[0]
    routed = src.route(x)
    xs, meta = src.gather(x, routed)
    offs = routed.offsets.cpu().numpy()
    Eg = inp.E // world
    outs = [shards[r].local(xs[offs[r * Eg]:offs[(r + 1) * Eg]].contiguous(),
                            meta[offs[r * Eg]:offs[(r + 1) * Eg]].contiguous()) for r in range(world)]
    y = src.combine(x, routed, torch.cat(outs, 0), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), y_full.cpu().numpy(), "sharded vs full")
    want, _, _ = oracle_forward(inp)
    assert_close(y.cpu().numpy(), want, "sharded vs oracle")
    rr = full.routing_results(inp.n)
    assert torch.equal(rr["perm"], routed.perm)
    assert torch.equal(rr["inv"], routed.inv)
    full.close()


def test_forward_local_rejects_foreign_expert():
    import torch
    inp = synth.make_inputs(256, 256, 4, 2, 8, True, seed=2)
    cfg = mxmoe.MoeConfig(inp.d, inp.f, inp.E, inp.k)
    be = CudaExpertBackend(cfg, "cuda:0", 2, 2, inp.gamma, inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2)
    meta = torch.zeros(inp.n, 3, dtype=torch.int32, device="cuda:0")
    meta[:, 1] = 0  # expert 0 lives on another shard
    be.local(to_device_x(inp), meta)
    with pytest.raises(mxmoe.MxMoeError):
        be.layer.sync_status()


@pytest.mark.parametrize("world,n_per,E,k,flags", [(2, 100, 8, 4, 0), (4, 64, 8, 2, 0), (4, 300, 16, 4, 0),
                                                    (2, 100, 8, 4, 1), (4, 300, 16, 4, 1)])
def test_peer_dispatch_emulated_on_one_gpu(world, n_per, E, k, flags):
    """The peer-memory expert-parallel step with `world` ranks emulated on one
    GPU: each rank's receive / return buffers are plain device buffers whose
    pointers stand in for the IPC-opened peers; the ranks' dispatch, expert
    and combine phases run in turn, as the two barriers order them across
    GPUs.  Every rank's output must match the single-layer forward."""
    import torch
    from mxmoe.ep import PeerExpertParallelMoe
    inp = synth.make_inputs(512, 384, E, k, world * n_per, True, seed=31 + world)
    full = make_layer(inp)
    x_all = to_device_x(inp)
    cfg = mxmoe.MoeConfig(inp.d, inp.f, inp.E, inp.k)
    bufs = [(torch.zeros(world * n_per * k, inp.d, dtype=torch.bfloat16, device="cuda:0"),
             torch.zeros(world * n_per * k, 4, dtype=torch.int32, device="cuda:0"),
             torch.zeros(n_per * k, inp.d, dtype=torch.bfloat16, device="cuda:0")) for _ in range(world)]
    peers = [tuple(b.data_ptr() for b in bb) for bb in bufs]
    ranks = []
    for r in range(world):
        b, c = shard_bounds(inp.E, world, r)
        be = CudaExpertBackend(cfg, "cuda:0", b, c, inp.gamma, inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2)
        ranks.append(PeerExpertParallelMoe(be, world, r, n_per, peers=peers))
        ranks[-1].return_flags = flags  # 1: the W2 epilogue stores to the source directly
    xs = [x_all[r * n_per:(r + 1) * n_per].contiguous() for r in range(world)]
    routes = [m.backend.route(x) for m, x in zip(ranks, xs)]
    allc = torch.cat([m.send_counts(rt) for m, rt in zip(ranks, routes)])
    host = allc.cpu().tolist()
    for m, x, rt in zip(ranks, xs, routes):
        m.dispatch(x, rt, allc)
    for r, m in enumerate(ranks):
        m.experts(sum(host[s * world + r] for s in range(world)))
    ys = [m.combine(x, rt, out_dtype=torch.float32) for m, x, rt in zip(ranks, xs, routes)]
    torch.cuda.synchronize()
    for r in range(world):
        assert int(ranks[r].err.item()) == 0
        ranks[r].backend.layer.sync_status()
        want = full.forward(xs[r], out_dtype=torch.float32)
        assert_close(ys[r].cpu().numpy(), want.cpu().numpy(), f"peer EP rank {r}/{world}")
    full.close()


@pytest.mark.parametrize("world,n_per,E,k,zipf", [(2, 100, 8, 4, None), (4, 64, 8, 2, None), (4, 300, 16, 4, None),
                                                  (2, 40, 4, 2, None), (4, 96, 128, 4, 1.1), (8, 48, 128, 4, 1.1)])
def test_quantized_dispatch_emulated_on_one_gpu(world, n_per, E, k, zipf):
    """Quantized dispatch into the owners' layouts with `world` ranks emulated
    on one GPU (each rank its own layer and workspace; the pointer tables
    stand in for the IPC-opened peers).  Every rank's output must match the
    single-layer forward.  The 128-expert cases carry the Zipf(1.1) router
    bias of the GPT-OSS-120B-shaped workload: owners get very uneven loads and
    some experts none."""
    import torch
    from mxmoe.ep import QuantizedPeerMoe
    from mxmoe.ep import balanced_placement, expert_loads, renumber_experts
    inp = synth.make_inputs(512, 384, E, k, world * n_per, True, seed=41 + world + E, zipf_router_bias=zipf)
    full = make_layer(inp)
    x_all = to_device_x(inp)
    cfg = mxmoe.MoeConfig(inp.d, inp.f, inp.E, inp.k)
    rets = [torch.zeros(n_per * k, inp.d, dtype=torch.bfloat16, device="cuda:0") for _ in range(world)]
    gate_w, gate_b, host, b1, b2 = inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2
    if zipf is not None:
        # skewed routing: the ranks hold load-balanced renumbered shards, the
        # reference layer keeps the original numbering
        order = balanced_placement(expert_loads(inp.x, inp.gamma, gate_w, gate_b, k), world)
        gate_w, gate_b, host, b1, b2 = renumber_experts(order, gate_w, gate_b, host, b1, b2)
    ranks = []
    for r in range(world):
        b, c = shard_bounds(inp.E, world, r)
        be = CudaExpertBackend(cfg, "cuda:0", b, c, inp.gamma, gate_w, gate_b, host, b1, b2)
        ranks.append(QuantizedPeerMoe(be, world, r, n_per, peers=[]))
    table = [(m.local_peers()[0], rets[r].data_ptr()) for r, m in enumerate(ranks)]
    for m in ranks:
        m.set_peers(table)
    xs = [x_all[r * n_per:(r + 1) * n_per].contiguous() for r in range(world)]
    for _ in range(2):  # a second step reuses the layouts
        routes = [m.backend.route(x) for m, x in zip(ranks, xs)]
        allc = torch.cat([m.counts(rt) for m, rt in zip(ranks, routes)])
        for m, x, rt in zip(ranks, xs, routes):
            m.dispatch(x, rt, allc)
        for m in ranks:
            m.experts()
        ys = [m.combine(x, rt, out_dtype=torch.float32) for m, x, rt in zip(ranks, xs, routes)]
        torch.cuda.synchronize()
        for r in range(world):
            ranks[r].backend.layer.sync_status()
            want = full.forward(xs[r], out_dtype=torch.float32)
            assert_close(ys[r].cpu().numpy(), want.cpu().numpy(), f"quantized EP rank {r}/{world}")
    full.close()


@pytest.mark.parametrize("world,n_per,E,extra", [(4, 96, 16, 4), (2, 120, 32, 2)])
def test_replicated_hot_experts_emulated_on_one_gpu(world, n_per, E, extra):
    """Hot experts copied into extra slots (plan_replicas), the slots placed
    by load (balanced_placement), and each replicated expert's pairs spread
    over its copies by token (ReplicaRemap); ranks emulated on one GPU.  Every
    rank's output must match the original single layer."""
    import numpy as np
    import torch
    from mxmoe import ep
    k = 4
    inp = synth.make_inputs(512, 384, E, k, world * n_per, True, seed=61 + world + E, zipf_router_bias=1.1)
    full = make_layer(inp)
    x_all = to_device_x(inp)
    loads = ep.expert_loads(inp.x, inp.gamma, inp.gate_w, inp.gate_b, k)
    src = ep.plan_replicas(loads, extra)
    slot_loads = np.array([loads[e] / np.count_nonzero(src == e) for e in src])
    order = ep.balanced_placement(slot_loads, world)
    gw, gb, host, b1, b2 = ep.replicate_experts(src, inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2)
    gw, gb, host, b1, b2 = ep.renumber_experts(order, gw, gb, host, b1, b2)
    S = len(src)
    cfg = mxmoe.MoeConfig(inp.d, inp.f, S, k)
    rets = [torch.zeros(n_per * k, inp.d, dtype=torch.bfloat16, device="cuda:0") for _ in range(world)]
    ranks = []
    for r in range(world):
        b, c = shard_bounds(S, world, r)
        be = CudaExpertBackend(cfg, "cuda:0", b, c, inp.gamma, gw, gb, host, b1, b2)
        m = ep.QuantizedPeerMoe(be, world, r, n_per, peers=[])
        m.remap = ep.ReplicaRemap(ep.replica_groups(src, order), "cuda:0")
        ranks.append(m)
    table = [(m.local_peers()[0], rets[r].data_ptr()) for r, m in enumerate(ranks)]
    for m in ranks:
        m.set_peers(table)
    xs = [x_all[r * n_per:(r + 1) * n_per].contiguous() for r in range(world)]
    for _ in range(2):
        routes = [m.route(x) for m, x in zip(ranks, xs)]
        # the copies receive pairs
        cnt = sum(m.counts(rt).cpu().numpy() for m, rt in zip(ranks, routes))
        copies = [int(np.argsort(order)[s]) for s in range(E, S)]
        assert cnt[copies].sum() > 0
        allc = torch.cat([m.counts(rt) for m, rt in zip(ranks, routes)])
        for m, x, rt in zip(ranks, xs, routes):
            m.dispatch(x, rt, allc)
        for m in ranks:
            m.experts()
        ys = [m.combine(x, rt, out_dtype=torch.float32) for m, x, rt in zip(ranks, xs, routes)]
        torch.cuda.synchronize()
        for r in range(world):
            ranks[r].backend.layer.sync_status()
            want = full.forward(xs[r], out_dtype=torch.float32)
            assert_close(ys[r].cpu().numpy(), want.cpu().numpy(), f"replicated EP rank {r}/{world}")
    full.close()
