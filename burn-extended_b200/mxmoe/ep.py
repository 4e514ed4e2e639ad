"""Expert-parallel MoE layer: one process per GPU, experts split into
contiguous shards, routed pairs moved by all-to-all (NCCL over NVLink on the
GPU path, gloo in the CPU tests).

The reference is single-rank (docs/gpt-oss-architecture.md:22 leaves
world_size sharding out); this module adds the expert-parallel form of
MoeGatedSwiGLU::forward (src/moe/mod.rs:99-115):

  1. every rank routes its own tokens with the full router (RmsNorm, gate,
     top-k, softmax) and sorts its (token, slot) pairs by expert -- pairs of
     one destination rank are then contiguous;
  2. the per-destination pair counts are exchanged, then the pairs' raw token
     rows and their (1/rms, expert, weight) metadata are dispatched;
  3. each rank runs its expert shard over the pairs it received;
  4. the per-pair outputs travel back on the reverse all-to-all and every rank
     combines its tokens' k contributions in increasing expert index and adds
     the residual.

The rank-local compute sits behind a backend object (route / gather / local /
combine): CudaExpertBackend runs libmxmoe's kernels; the CPU tests plug in
the oracle so that the dispatch logic is checked with gloo ranks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

from . import MoeConfig, MoeQuantLayerHost, QuantLinearMxFp4Desc, combine, gather_pairs


def shard_bounds(num_experts: int, world: int, rank: int):
    """Contiguous expert shard of `rank` (experts must divide evenly)."""
    if num_experts % world != 0:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    per = num_experts // world
    return rank * per, per


def slice_host(host: MoeQuantLayerHost, begin: int, count: int) -> MoeQuantLayerHost:
    """The expert shard [begin, begin + count) of a host weight payload."""
    d1, d2 = host.w1_desc, host.w2_desc
    return MoeQuantLayerHost(
        QuantLinearMxFp4Desc(count, d1.rows, d1.cols, d1.bpr, d1.gpr, d1.ue8_offset),
        QuantLinearMxFp4Desc(count, d2.rows, d2.cols, d2.bpr, d2.gpr, d2.ue8_offset),
        host.w1_blocks[begin:begin + count], host.w1_scales[begin:begin + count],
        host.w2_blocks[begin:begin + count], host.w2_scales[begin:begin + count])


def expert_loads(x, gamma, gate_w, gate_b, k: int, rms_eps: float = 1e-5):
    """Pairs per expert that the router (RmsNorm, gate, top-k) gives the
    tokens x [n, d] (numpy, f32 arithmetic).  A placement heuristic only: the
    layer's own router decides the real routing."""
    import numpy as np
    x = np.asarray(x, dtype=np.float32)
    xn = x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + rms_eps) * np.asarray(gamma, dtype=np.float32)
    logits = xn @ np.asarray(gate_w, dtype=np.float32).T + np.asarray(gate_b, dtype=np.float32)
    top = np.argpartition(-logits, k - 1, axis=1)[:, :k]
    return np.bincount(top.ravel(), minlength=logits.shape[1])


def balanced_placement(loads, world: int):
    """Expert order for load-balanced contiguous shards: rank r owns the
    experts order[r * E / world:(r + 1) * E / world].  Greedy longest-first:
    experts in decreasing load go to the rank with the least load that still
    has a free slot (ties to the lower rank), so that each rank gets E / world
    experts.  Within a rank the experts keep increasing id order."""
    import numpy as np
    loads = np.asarray(loads, dtype=np.float64)
    E = loads.shape[0]
    if E % world != 0:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    per = E // world
    total = np.zeros(world)
    slots = [[] for _ in range(world)]
    for e in sorted(range(E), key=lambda i: (-loads[i], i)):
        r = min((r for r in range(world) if len(slots[r]) < per), key=lambda r: (total[r], r))
        slots[r].append(e)
        total[r] += loads[e]
    return np.array([e for r in range(world) for e in sorted(slots[r])], dtype=np.int64)


def renumber_experts(order, gate_w, gate_b, host: MoeQuantLayerHost, b1, b2):
    """Layer tensors with expert i of the result = expert order[i] of the
    input: the gate rows, gate bias, MXFP4 blocks and scales and both biases
    are permuted together.  The renumbered layer computes the same function
    of x; only the combine's expert-order summation (and the top-k tie rule
    between exactly equal logits) follow the new ids, so outputs agree within
    f32 rounding.  The caller maps routing results back with order[id]."""
    import numpy as np
    o = np.asarray(order, dtype=np.int64)
    if sorted(o.tolist()) != list(range(host.w1_desc.experts)):
        raise ValueError("order must be a permutation of the experts")
    h = MoeQuantLayerHost(host.w1_desc, host.w2_desc, host.w1_blocks[o], host.w1_scales[o], host.w2_blocks[o],
                          host.w2_scales[o])
    return np.asarray(gate_w)[o], np.asarray(gate_b)[o], h, np.asarray(b1)[o], np.asarray(b2)[o]


def plan_replicas(loads, extra: int):
    """Hot-expert replication plan: `extra` additional expert slots, each a
    copy of an existing expert, handed out greedily to the expert with the
    largest load per copy.  Returns src, the original expert of every slot
    (slots 0 .. E - 1 are the experts themselves, E .. E + extra - 1 the
    copies)."""
    import numpy as np
    loads = np.asarray(loads, dtype=np.float64)
    copies = np.ones(loads.shape[0], dtype=np.int64)
    src = list(range(loads.shape[0]))
    for _ in range(extra):
        e = int(np.argmax(loads / copies))
        copies[e] += 1
        src.append(e)
    return np.array(src, dtype=np.int64)


def replicate_experts(src, gate_w, gate_b, host: MoeQuantLayerHost, b1, b2):
    """Layer tensors over the slots of plan_replicas: every slot gets its
    original expert's weights, scales and biases; copy slots get a zero gate
    row and a gate bias of -1e30, so that the router never picks them and
    top-k and softmax are those of the original experts.  ReplicaRemap then
    moves part of each hot expert's pairs onto its copies."""
    import numpy as np
    src = np.asarray(src, dtype=np.int64)
    E = np.asarray(gate_w).shape[0]
    gw = np.concatenate([np.asarray(gate_w, dtype=np.float32), np.zeros((len(src) - E, gate_w.shape[1]), np.float32)])
    gb = np.concatenate([np.asarray(gate_b, dtype=np.float32), np.full(len(src) - E, -1e30, np.float32)])
    d1, d2 = host.w1_desc, host.w2_desc
    h = MoeQuantLayerHost(QuantLinearMxFp4Desc(len(src), d1.rows, d1.cols, d1.bpr, d1.gpr, d1.ue8_offset),
                          QuantLinearMxFp4Desc(len(src), d2.rows, d2.cols, d2.bpr, d2.gpr, d2.ue8_offset),
                          host.w1_blocks[src], host.w1_scales[src], host.w2_blocks[src], host.w2_scales[src])
    return gw, gb, h, np.asarray(b1)[src], np.asarray(b2)[src]


class ReplicaRemap:
    """Moves the pairs of replicated experts onto their copies after the
    router: the pair of token t on expert e goes to copy t % c_e of e (c_e
    copies, the expert itself first), then the canonical maps are rebuilt
    for the remapped ids.  Stream-ordered torch and libmxmoe calls; nothing
    waits on the host.  groups: the slot ids of each original expert, after
    any renumbering (replica_groups)."""

    def __init__(self, groups, device):
        import torch
        self.torch = torch
        self.S = sum(len(g) for g in groups) if groups else 0
        width = max(len(g) for g in groups)
        table = torch.full((self.S, width), -1, dtype=torch.int64)
        ncopy = torch.ones(self.S, dtype=torch.int64)
        for g in groups:
            for sid in g:
                table[sid, :len(g)] = torch.tensor(g)
                ncopy[sid] = len(g)
        self.table = table.to(device)
        self.ncopy = ncopy.to(device)

    def apply(self, r: "Routed") -> "Routed":
        t = self.torch
        idx = r.topk_idx.to(t.int64)
        n = idx.shape[0]
        if n == 0:
            return r
        tok = t.arange(n, device=idx.device).unsqueeze(1)
        new = self.table[idx, tok % self.ncopy[idx]]
        flat = new.reshape(-1)
        # canonical maps: pairs sorted by expert, increasing pair index within one
        counts = t.zeros(self.S, dtype=t.int64, device=idx.device).scatter_add_(0, flat, t.ones_like(flat))
        offsets = t.zeros(self.S + 1, dtype=t.int32, device=idx.device)
        offsets[1:] = t.cumsum(counts, 0).to(t.int32)
        perm = t.sort(flat, stable=True).indices
        inv = t.empty_like(perm)
        inv[perm] = t.arange(perm.numel(), device=idx.device)
        return Routed(r.rscale, new.to(t.int32).contiguous(), r.topk_w, offsets, perm.to(t.int32), inv.to(t.int32))


def replica_groups(src, order=None):
    """Slot ids grouped by original expert, after the renumbering `order`
    (slot i of the renumbered layer = slot order[i] before it)."""
    import numpy as np
    src = np.asarray(src)
    new_of = np.arange(len(src)) if order is None else np.argsort(np.asarray(order))
    groups = {}
    for slot, e in enumerate(src.tolist()):
        groups.setdefault(e, []).append(int(new_of[slot]))
    return [groups[e] for e in sorted(groups)]


@dataclass
class Routed:
    rscale: object    # [n] 1 / rms per token
    topk_idx: object  # [n, k] global expert ids
    topk_w: object    # [n, k]
    offsets: object   # [E + 1] prefix sums of pairs per expert (canonical order)
    perm: object      # [n * k] sorted position -> pair
    inv: object       # [n * k] pair -> sorted position


class CudaExpertBackend:
    """Rank-local compute on libmxmoe: the full router plus this rank's
    expert shard."""

    def __init__(self, cfg: MoeConfig, device, begin: int, count: int, gamma, gate_w, gate_b,
                 host: MoeQuantLayerHost, b1, b2, pair_dtype=None):
        import torch
        self.torch = torch
        self.cfg = cfg
        self.device = torch.device(device)
        self.layer = cfg.init(self.device.index or 0)
        self.layer.set_router(gamma, gate_w, gate_b)
        self.layer.set_expert_shard(begin, count)
        self.layer.set_resident(slice_host(host, begin, count), b1[begin:begin + count], b2[begin:begin + count])
        # per-pair outputs travel back in bf16: half the combine traffic, and
        # the rounding (2^-9 relative per contribution) is far inside tolerance
        self.pair_dtype = pair_dtype or torch.bfloat16

    def route(self, x) -> Routed:
        t = self.torch
        n, k, E = x.shape[0], self.cfg.experts_per_token, self.cfg.num_experts
        dev = x.device
        r = Routed(t.empty(n, dtype=t.float32, device=dev), t.empty(n, k, dtype=t.int32, device=dev),
                   t.empty(n, k, dtype=t.float32, device=dev), t.empty(E + 1, dtype=t.int32, device=dev),
                   t.empty(n * k, dtype=t.int32, device=dev), t.empty(n * k, dtype=t.int32, device=dev))
        if n:
            self.layer.route(x, r.rscale, r.topk_idx, r.topk_w, r.offsets, r.perm, r.inv)
        else:
            r.offsets.zero_()
        return r

    def gather(self, x, r: Routed):
        t = self.torch
        P = r.perm.numel()
        out_x = t.empty(P, x.shape[1], dtype=x.dtype, device=x.device)
        meta = t.empty(P, 3, dtype=t.int32, device=x.device)  # (1/rms bits, expert, weight bits)
        if P:
            gather_pairs(x, self.cfg.experts_per_token, r.perm, r.rscale, r.topk_idx, r.topk_w, out_x, meta)
        return out_x, meta

    def local(self, xr, meta):
        t = self.torch
        out = t.empty(xr.shape[0], xr.shape[1], dtype=self.pair_dtype, device=xr.device)
        if xr.shape[0]:
            rs = meta[:, 0].contiguous().view(t.float32)
            ex = meta[:, 1].contiguous()
            w = meta[:, 2].contiguous().view(t.float32)
            self.layer.forward_local(xr, rs, ex, w, out)
        return out

    def combine(self, x, r: Routed, pair_out, out_dtype=None):
        t = self.torch
        y = t.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
        combine(x, self.cfg.experts_per_token, r.topk_idx, r.inv, pair_out, y, residual=self.cfg.residual)
        return y

    def empty(self, shape, dtype):
        return self.torch.empty(shape, dtype=dtype, device=self.device)

    def to_host_list(self, t) -> List[int]:
        return [int(v) for v in t.cpu().tolist()]


class ExpertParallelMoe:
    """One rank of the expert-parallel layer (see the module docstring)."""

    # rms, router logits, top-k, permute, gather, localize, permute, quantize,
    # W1, W2, un-permute, combine
    launches_per_step = 12

    def __init__(self, backend, num_experts: int, world: int, rank: int, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.backend = backend
        self.E = num_experts
        self.world = world
        self.rank = rank
        self.group = group
        self.Eg = num_experts // world

    def _a2a(self, out, inp, out_splits, in_splits):
        self.dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def _dispatch(self, x, r):
        import torch
        b = self.backend
        xs, meta = b.gather(x, r)  # enqueued before the host waits on the counts
        offs = b.to_host_list(r.offsets[:: self.Eg])  # world + 1 boundaries
        send = [offs[g + 1] - offs[g] for g in range(self.world)]
        send_t = b.empty((self.world,), torch.int64)
        send_t.copy_(torch.tensor(send, dtype=torch.int64))
        recv_t = b.empty((self.world,), torch.int64)
        self._a2a(recv_t, send_t, None, None)
        recv = b.to_host_list(recv_t)
        R = sum(recv)
        xr = b.empty((R, x.shape[1]), x.dtype)
        mr = b.empty((R, 3), torch.int32)
        self._a2a(xr, xs, recv, send)
        self._a2a(mr, meta, recv, send)
        return send, recv, xr, mr

    remap = None  # ReplicaRemap when hot experts are replicated

    def forward(self, x, out_dtype=None):
        b = self.backend
        r = b.route(x)
        if self.remap is not None:
            r = self.remap.apply(r)
        send, recv, xr, mr = self._dispatch(x, r)
        out = b.local(xr, mr)
        back = b.empty((sum(send), x.shape[1]), out.dtype)
        self._a2a(back, out, send, recv)
        return b.combine(x, r, back, out_dtype)

    def profile(self, x, steps: int = 3):
        """Per-phase device times in ms (CUDA events on the current stream)."""
        import torch
        b = self.backend
        names = ["route", "dispatch", "experts", "combine_a2a", "combine"]
        acc = {n: 0.0 for n in names}
        for _ in range(steps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            ev[0].record()
            r = b.route(x)
            ev[1].record()
            send, recv, xr, mr = self._dispatch(x, r)
            ev[2].record()
            out = b.local(xr, mr)
            ev[3].record()
            back = b.empty((sum(send), x.shape[1]), out.dtype)
            self._a2a(back, out, send, recv)
            ev[4].record()
            b.combine(x, r, back)
            ev[5].record()
            torch.cuda.synchronize()
            for i, n in enumerate(names):
                acc[n] += ev[i].elapsed_time(ev[i + 1]) / steps
        return acc


def build_cuda_rank(inp, world: int, rank: int, device, cfg: Optional[MoeConfig] = None, group=None):
    """ExpertParallelMoe over libmxmoe for synthetic inputs `inp` (mxmoe.synth)."""
    cfg = cfg or MoeConfig(inp.d, inp.f, inp.E, inp.k)
    begin, count = shard_bounds(inp.E, world, rank)
    be = CudaExpertBackend(cfg, device, begin, count, inp.gamma, inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2)
    return ExpertParallelMoe(be, inp.E, world, rank, group)


# ----------------------------------------------------------------------------
# Expert parallelism over peer memory (NVLink / NVSwitch).  The source rank's
# dispatch kernel writes every routed pair straight into the owning rank's
# receive buffers; the owner's W2 epilogue writes each pair's output straight
# into the source rank's return buffer (canonical order), so the step needs
# no gather copy, no data all-to-all and no un-permute pass.  Two collective
# barriers order the peer writes against their readers; the per-destination
# pair counts travel in one small all-gather.

class IpcBuffer:
    """Device buffer of this rank that peers open through CUDA IPC."""

    def __init__(self, nbytes: int, device: int):
        import ctypes
        from ._lib import IPC_HANDLE_BYTES, check, lib
        self.device = device
        self.nbytes = nbytes
        self.ptr = ctypes.c_void_p()
        self.handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(lib().mxmoe_ipc_alloc(nbytes, device, ctypes.byref(self.ptr), self.handle))

    def close(self):
        from ._lib import lib
        if self.ptr:
            lib().mxmoe_ipc_free(self.ptr, self.device)
            self.ptr = None


def open_peer(handle: bytes, device: int) -> int:
    import ctypes
    from ._lib import check, lib
    p = ctypes.c_void_p()
    check(lib().mxmoe_ipc_open(ctypes.create_string_buffer(handle, len(handle)), device, ctypes.byref(p)))
    return p.value


def return_slot(rank: int, q: int) -> int:
    """Return slot word of the pair at canonical position q of `rank`."""
    return (rank << 24) | q


def receive_rows(counts, world: int, src: int, dst: int, begin: int, end: int):
    """Rows [row0, row1) of dst's receive buffer that src fills with its
    canonical positions [begin, end) (its pairs for dst's experts);
    counts[s][g] = pairs s sends to g."""
    row0 = sum(counts[s][dst] for s in range(src))
    return row0, row0 + (end - begin)


class PeerExpertParallelMoe:
    """One rank of the expert-parallel layer over peer memory."""

    # rms, router logits, top-k, permute x2, dispatch, split meta, localize,
    # permute x2, quantize, W1, W2, combine
    launches_per_step = 14

    def __init__(self, backend: CudaExpertBackend, world: int, rank: int, max_tokens: int, x_dtype=None,
                 group=None, peers=None):
        """peers: optional list of (recv_x, recv_meta, ret) device pointers
        per rank, used instead of the IPC exchange (ranks emulated in one
        process on one GPU)."""
        import torch
        self.torch = torch
        self.backend = backend
        self.world, self.rank, self.group = world, rank, group
        cfg = backend.cfg
        self.d, self.k, self.E = cfg.d_model, cfg.experts_per_token, cfg.num_experts
        if self.E % world:
            raise ValueError(f"{self.E} experts do not split over {world} ranks")
        self.Eg = self.E // world
        self.max_tokens = max_tokens
        self.x_dtype = x_dtype or torch.bfloat16
        elem = torch.tensor([], dtype=self.x_dtype).element_size()
        dev = backend.device
        self.dev_index = dev.index or 0
        cap_local = max_tokens * self.k
        self.recv_cap = world * cap_local  # every pair of every rank could target one rank
        self.own = None
        if peers is None:
            import torch.distributed as dist
            self.own = [IpcBuffer(self.recv_cap * self.d * elem, self.dev_index),
                        IpcBuffer(self.recv_cap * 16, self.dev_index),
                        IpcBuffer(cap_local * self.d * 2, self.dev_index)]
            mine = [bytes(b.handle.raw) for b in self.own]
            allh = [None] * world
            dist.all_gather_object(allh, mine, group=group)
            self.opened = []
            peers = []
            for r in range(world):
                if r == rank:
                    peers.append(tuple(b.ptr.value for b in self.own))
                else:
                    ptrs = tuple(open_peer(h, self.dev_index) for h in allh[r])
                    self.opened.extend(ptrs)
                    peers.append(ptrs)
        self.peers = peers
        self.recv_x, self.recv_meta, self.ret = peers[rank]
        self.peer_x = torch.tensor([p[0] for p in peers], dtype=torch.int64, device=dev)
        self.peer_meta = torch.tensor([p[1] for p in peers], dtype=torch.int64, device=dev)
        self.peer_ret = torch.tensor([p[2] for p in peers], dtype=torch.int64, device=dev)
        self.tick = torch.zeros(1, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)  # dispatch bound violations (code 8)
        # 0: W2 writes locally, a copy pass pushes rows back; RETURN_FROM_EPILOGUE:
        # the W2 epilogue stores to the source ranks directly
        self.return_flags = 0

    # -- pieces of one step (the single-GPU emulation drives them directly)
    def send_counts(self, r):
        """Pairs this rank sends to each rank: [world] int32 on the device."""
        o = r.offsets
        return (o[self.Eg::self.Eg] - o[0:self.E:self.Eg]).to(self.torch.int32)

    def dispatch(self, x, r, counts_dev):
        from . import _dtype_code, _stream_ptr
        from ._lib import check, lib
        n = x.shape[0]
        if n == 0:
            return
        check(lib().mxmoe_dispatch_pairs(x.data_ptr(), _dtype_code(x), n, self.d, self.k, r.perm.data_ptr(),
                                         r.rscale.data_ptr(), r.topk_idx.data_ptr(), r.topk_w.data_ptr(),
                                         r.offsets.data_ptr(), self.Eg, self.world, self.rank,
                                         counts_dev.data_ptr(), self.peer_x.data_ptr(),
                                         self.peer_meta.data_ptr(), self.recv_cap, self.err.data_ptr(),
                                         _stream_ptr()))

    def experts(self, n_recv: int):
        from . import BF16, F32, _stream_ptr
        from ._lib import check, lib
        if n_recv == 0:
            return
        code = BF16 if self.x_dtype == self.torch.bfloat16 else F32
        check(lib().mxmoe_forward_local_meta(self.backend.layer._h, self.recv_x, code, self.recv_meta, n_recv,
                                             self.peer_ret.data_ptr(), self.world, self.max_tokens * self.k,
                                             self.return_flags, _stream_ptr()))

    def combine(self, x, r, out_dtype=None):
        from . import BF16, _dtype_code, _stream_ptr
        from ._lib import check, lib
        t = self.torch
        y = t.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
        n = x.shape[0]
        if n:
            check(lib().mxmoe_combine(x.data_ptr(), _dtype_code(x), n, self.d, self.k, r.topk_idx.data_ptr(),
                                      r.inv.data_ptr(), self.ret, BF16, 1 if self.backend.cfg.residual else 0,
                                      y.data_ptr(), _dtype_code(y), _stream_ptr()))
        return y

    def barrier(self):
        self.torch.distributed.all_reduce(self.tick, group=self.group)

    def exchange_counts(self, counts_dev):
        """All ranks' send counts [world][world] on the device and on the host."""
        t = self.torch
        allc = t.empty(self.world * self.world, dtype=t.int32, device=counts_dev.device)
        t.distributed.all_gather_into_tensor(allc, counts_dev, group=self.group)
        host = allc.cpu().tolist()
        return allc, [host[s * self.world:(s + 1) * self.world] for s in range(self.world)]

    def forward(self, x, out_dtype=None):
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"{x.shape[0]} tokens > max_tokens {self.max_tokens}")
        if x.dtype != self.x_dtype:
            raise ValueError(f"x dtype {x.dtype} != {self.x_dtype}")
        r = self.backend.route(x)
        allc, host = self.exchange_counts(self.send_counts(r))
        n_recv = sum(host[s][self.rank] for s in range(self.world))
        self.dispatch(x, r, allc)
        self.barrier()  # every rank's pairs are in its owners' receive buffers
        self.experts(n_recv)
        self.barrier()  # every pair's output is back in its source's return buffer
        return self.combine(x, r, out_dtype)

    def profile(self, x, steps: int = 3):
        """Per-phase device times in ms (CUDA events on the current stream)."""
        t = self.torch
        names = ["route", "counts", "dispatch", "experts", "combine"]
        acc = {nm: 0.0 for nm in names}
        for _ in range(steps):
            ev = [t.cuda.Event(enable_timing=True) for _ in range(6)]
            ev[0].record()
            r = self.backend.route(x)
            ev[1].record()
            allc, host = self.exchange_counts(self.send_counts(r))
            n_recv = sum(host[s][self.rank] for s in range(self.world))
            ev[2].record()
            self.dispatch(x, r, allc)
            self.barrier()
            ev[3].record()
            self.experts(n_recv)
            self.barrier()
            ev[4].record()
            self.combine(x, r)
            ev[5].record()
            t.cuda.synchronize()
            for i, nm in enumerate(names):
                acc[nm] += ev[i].elapsed_time(ev[i + 1]) / steps
        return acc

    def close(self):
        from ._lib import lib
        for p in getattr(self, "opened", []):
            lib().mxmoe_ipc_close(p, self.dev_index)
        self.opened = []
        for b in self.own or []:
            b.close()
        self.own = None


def build_peer_rank(inp, world: int, rank: int, device, cfg: Optional[MoeConfig] = None, group=None):
    """PeerExpertParallelMoe over libmxmoe for synthetic inputs `inp` (mxmoe.synth)."""
    cfg = cfg or MoeConfig(inp.d, inp.f, inp.E, inp.k)
    begin, count = shard_bounds(inp.E, world, rank)
    be = CudaExpertBackend(cfg, device, begin, count, inp.gamma, inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2)
    return PeerExpertParallelMoe(be, world, rank, inp.n, group=group)


class QuantizedPeerMoe:
    """One rank of the expert-parallel layer with quantized dispatch: this
    rank quantizes its own tokens once and writes every pair's codes, scales
    and row metadata straight into the owner's GEMM operand layout (peer
    memory); the owner runs W1/W2 on it and pushes the outputs back.  The
    pair counts travel in one all-gather on the device, so a step never
    waits on the host."""

    # rms, router logits, top-k, permute x2, layout, quantize-dispatch, W1, W2, return, combine
    launches_per_step = 11
    BUFS = 3  # activation codes, row-major scale bytes, row metadata (mxmoe_ep_reserve order)

    def __init__(self, backend: CudaExpertBackend, world: int, rank: int, max_tokens: int, x_dtype=None,
                 group=None, peers=None):
        """peers: for ranks emulated in one process, a list per rank of
        (3 layout buffer pointers, return buffer pointer) used instead of the
        IPC exchange; this rank's buffers are then exposed by .local_peers()
        before the list is complete (see the tests)."""
        import ctypes
        import torch
        from ._lib import IPC_HANDLE_BYTES, check, lib
        self.torch = torch
        self.backend = backend
        self.world, self.rank, self.group = world, rank, group
        cfg = backend.cfg
        self.d, self.k, self.E = cfg.d_model, cfg.experts_per_token, cfg.num_experts
        self.max_tokens = max_tokens
        self.x_dtype = x_dtype or torch.bfloat16
        self.dev = backend.device
        self.dev_index = self.dev.index or 0
        self.ret_rows = max_tokens * self.k
        handles = ctypes.create_string_buffer(self.BUFS * IPC_HANDLE_BYTES)
        check(lib().mxmoe_ep_reserve(backend.layer._h, max_tokens, world, handles))
        self.opened = []
        self.own_ret = None
        if peers is None:
            import torch.distributed as dist
            self.own_ret = IpcBuffer(self.ret_rows * self.d * 2, self.dev_index)
            mine = (bytes(handles.raw), bytes(self.own_ret.handle.raw))
            allh = [None] * world
            dist.all_gather_object(allh, mine, group=group)
            own = self.local_peers()[0]
            table = []
            for r in range(world):
                if r == rank:
                    table.append((own, self.own_ret.ptr.value))
                    continue
                hb, hr = allh[r]
                bufs = [open_peer(hb[i * IPC_HANDLE_BYTES:(i + 1) * IPC_HANDLE_BYTES], self.dev_index)
                        for i in range(self.BUFS)]
                ret = open_peer(hr, self.dev_index)
                self.opened.extend(bufs + [ret])
                table.append((bufs, ret))
            self.set_peers(table)

    def local_peers(self):
        """This rank's layout buffers as device pointers."""
        import ctypes
        from ._lib import check, lib
        arr = (ctypes.c_void_p * self.BUFS)()
        check(lib().mxmoe_ep_buffers(self.backend.layer._h, arr))
        return [int(arr[i]) for i in range(self.BUFS)], None

    def set_peers(self, table):
        """table[r] = (layout buffer pointers of rank r, its return buffer pointer)."""
        t = self.torch
        flat = [table[r][0][b] for b in range(self.BUFS) for r in range(self.world)]
        self.peer_bufs = t.tensor(flat, dtype=t.int64, device=self.dev)
        self.peer_ret = t.tensor([table[r][1] for r in range(self.world)], dtype=t.int64, device=self.dev)
        self.ret = table[self.rank][1]

    remap = None  # ReplicaRemap when hot experts are replicated

    def route(self, x):
        r = self.backend.route(x)
        return self.remap.apply(r) if self.remap is not None else r

    def counts(self, r):
        o = r.offsets
        return (o[1:] - o[:-1]).to(self.torch.int32)

    def all_counts(self, counts_dev):
        t = self.torch
        allc = t.empty(self.world * self.E, dtype=t.int32, device=counts_dev.device)
        t.distributed.all_gather_into_tensor(allc, counts_dev, group=self.group)
        return allc

    def dispatch(self, x, r, allc):
        from . import _dtype_code, _stream_ptr
        from ._lib import check, lib
        check(lib().mxmoe_ep_dispatch(self.backend.layer._h, x.data_ptr(), _dtype_code(x), x.shape[0],
                                      r.rscale.data_ptr(), r.topk_idx.data_ptr(), r.topk_w.data_ptr(),
                                      r.inv.data_ptr(), r.offsets.data_ptr(), allc.data_ptr(), self.rank,
                                      self.peer_bufs.data_ptr(), _stream_ptr()))

    def experts(self):
        from . import BF16, F32, _stream_ptr
        from ._lib import check, lib
        code = BF16 if self.x_dtype == self.torch.bfloat16 else F32
        check(lib().mxmoe_ep_experts(self.backend.layer._h, code, self.peer_ret.data_ptr(), self.ret_rows,
                                     _stream_ptr()))

    def combine(self, x, r, out_dtype=None):
        from . import BF16, _dtype_code, _stream_ptr
        from ._lib import check, lib
        y = self.torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
        if x.shape[0]:
            check(lib().mxmoe_combine(x.data_ptr(), _dtype_code(x), x.shape[0], self.d, self.k,
                                      r.topk_idx.data_ptr(), r.inv.data_ptr(), self.ret, BF16,
                                      1 if self.backend.cfg.residual else 0, y.data_ptr(), _dtype_code(y),
                                      _stream_ptr()))
        return y

    def barrier(self):
        if not hasattr(self, "tick"):
            self.tick = self.torch.zeros(1, dtype=self.torch.int32, device=self.dev)
        self.torch.distributed.all_reduce(self.tick, group=self.group)

    def forward(self, x, out_dtype=None):
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"{x.shape[0]} tokens > max_tokens {self.max_tokens}")
        if x.dtype != self.x_dtype:
            raise ValueError(f"x dtype {x.dtype} != {self.x_dtype}")
        r = self.route(x)
        allc = self.all_counts(self.counts(r))
        self.dispatch(x, r, allc)
        self.barrier()  # every pair is in its owner's layout
        self.experts()
        self.barrier()  # every output is back at its source
        return self.combine(x, r, out_dtype)

    def profile(self, x, steps: int = 3):
        t = self.torch
        names = ["route", "counts", "dispatch", "experts", "combine"]
        acc = {nm: 0.0 for nm in names}
        for _ in range(steps):
            ev = [t.cuda.Event(enable_timing=True) for _ in range(6)]
            ev[0].record()
            r = self.route(x)
            ev[1].record()
            allc = self.all_counts(self.counts(r))
            ev[2].record()
            self.dispatch(x, r, allc)
            self.barrier()
            ev[3].record()
            self.experts()
            self.barrier()
            ev[4].record()
            self.combine(x, r)
            ev[5].record()
            t.cuda.synchronize()
            for i, nm in enumerate(names):
                acc[nm] += ev[i].elapsed_time(ev[i + 1]) / steps
        return acc

    def close(self):
        from ._lib import lib
        for p in self.opened:
            lib().mxmoe_ipc_close(p, self.dev_index)
        self.opened = []
        if self.own_ret is not None:
            self.own_ret.close()
            self.own_ret = None


def build_quantized_peer_rank(inp, world: int, rank: int, device, cfg: Optional[MoeConfig] = None, group=None,
                              placement=None, replicas=None):
    """QuantizedPeerMoe over libmxmoe for synthetic inputs `inp` (mxmoe.synth).
    replicas: optional slot plan (plan_replicas) that copies hot experts into
    extra slots; placement: optional order of the (slot) experts
    (balanced_placement) applied before sharding.  Both identical on every
    rank."""
    from dataclasses import replace
    gate_w, gate_b, host, b1, b2 = inp.gate_w, inp.gate_b, inp.host, inp.b1, inp.b2
    S = inp.E
    if replicas is not None:
        gate_w, gate_b, host, b1, b2 = replicate_experts(replicas, gate_w, gate_b, host, b1, b2)
        S = len(replicas)
    cfg = cfg or MoeConfig(inp.d, inp.f, inp.E, inp.k)
    cfg = replace(cfg, num_experts=S)
    begin, count = shard_bounds(S, world, rank)
    if placement is not None:
        gate_w, gate_b, host, b1, b2 = renumber_experts(placement, gate_w, gate_b, host, b1, b2)
    be = CudaExpertBackend(cfg, device, begin, count, inp.gamma, gate_w, gate_b, host, b1, b2)
    m = QuantizedPeerMoe(be, world, rank, inp.n, group=group)
    if replicas is not None:
        m.remap = ReplicaRemap(replica_groups(replicas, placement), be.device)
    return m
