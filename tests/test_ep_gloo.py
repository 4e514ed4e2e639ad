"""Expert-parallel dispatch / combine on gloo ranks (CPU), with the oracle as
the rank-local compute: every rank's output must equal the single-process
oracle forward of its own tokens bit for bit.  Also the host-side failure
path: a rank that dies between steps makes its peer's next collective fail
within the process-group timeout instead of hanging."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _paths():
    for p in (os.path.join(ROOT, "burn-extended_b200"), os.path.join(ROOT, "oracle"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, case, result_q):
    _paths()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        import oracle
        from ep_oracle_backend import OracleExpertBackend
        from mxmoe import synth
        from mxmoe.ep import ExpertParallelMoe
        d, f, E, k, n, skew = case[:6]
        extra = case[6] if len(case) > 6 else 0
        inp = synth.make_inputs(d, f, E, k, n, bf16=True, seed=100, zipf_router_bias=skew)
        # every rank holds the same weights and its own tokens
        inp.x = synth.make_inputs(d, f, E, k, n, bf16=True, seed=200 + rank, zipf_router_bias=skew).x
        if extra:
            # copies of the hottest experts in extra slots, slots placed by load
            from dataclasses import replace
            from mxmoe import ep as epm
            cal = synth.make_inputs(d, f, E, k, 64, bf16=True, seed=300, zipf_router_bias=skew)
            loads = epm.expert_loads(cal.x, inp.gamma, inp.gate_w, inp.gate_b, k)
            src = epm.plan_replicas(loads, extra)
            order = epm.balanced_placement([loads[e] / np.count_nonzero(src == e) for e in src], world)
            t = epm.renumber_experts(order, *epm.replicate_experts(src, inp.gate_w, inp.gate_b, inp.host, inp.b1,
                                                                   inp.b2))
            slots = replace(inp, E=len(src), gate_w=t[0], gate_b=t[1], host=t[2], b1=t[3], b2=t[4])
            ep = ExpertParallelMoe(OracleExpertBackend(slots, world, rank), len(src), world, rank)
            ep.remap = epm.ReplicaRemap(epm.replica_groups(src, order), "cpu")
        else:
            ep = ExpertParallelMoe(OracleExpertBackend(inp, world, rank), E, world, rank)
        y = ep.forward(torch.from_numpy(inp.x)).numpy()
        want, _, _ = oracle.moe_forward(oracle.cfg(d, f, E, k), inp.x, inp.gamma, inp.gate_w, inp.gate_b,
                                        inp.host.w1_blocks, inp.host.w1_scales, inp.b1, inp.host.w2_blocks,
                                        inp.host.w2_scales, inp.b2)
        # with copies only the order of a token's k terms in the combine may change
        exact = (np.array_equal(y.view(np.uint32), want.view(np.uint32)) if not extra else
                 bool(np.abs(y - want).max() <= 1e-5 * np.abs(want).max()))
        result_q.put((rank, exact, float(np.abs(y - want).max())))
    finally:
        dist.destroy_process_group()


def _run(world, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = [q.get(timeout=5) for _ in range(world)]
    for p in procs:
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("world,case", [
    (2, (64, 64, 4, 2, 6, None)),
    (2, (64, 96, 4, 4, 9, None)),   # k = E: every token visits every rank
    (4, (64, 64, 8, 2, 5, 1.1)),    # Zipf-skewed router: some ranks get few pairs
    (2, (64, 64, 2, 1, 7, 8.0)),    # heavy skew: rank 1 receives nothing
    (2, (64, 64, 6, 2, 24, 1.5, 2)),  # copies of the hot experts in 2 extra slots
    (4, (64, 64, 8, 2, 16, 1.1, 4)),
])
def test_ep_matches_single_process_oracle(world, case):
    for rank, exact, err in _run(world, case):
        assert exact, f"rank {rank}: max abs diff {err}"


def _dying_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(3)  # leaves between steps, nothing in flight
    t0 = datetime.datetime.now()
    try:
        out = torch.empty(2)
        dist.all_to_all_single(out, torch.ones(2))
        result_q.put(("no-error", 0.0))
    except Exception as exc:  # the survivor learns of the failure from its collective
        result_q.put((type(exc).__name__, (datetime.datetime.now() - t0).total_seconds()))


def test_peer_failure_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    kind, secs = q.get(timeout=5)
    assert kind != "no-error"
    assert secs < 30
