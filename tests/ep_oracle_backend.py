"""CPU stand-in for CudaExpertBackend (test infrastructure): the same
route / gather / local / combine contract computed by the CPU oracle, so that
the expert-parallel dispatch logic of mxmoe.ep runs on gloo ranks without a
GPU."""
import numpy as np
import torch

import oracle
from mxmoe.ep import Routed, shard_bounds, slice_host


class OracleExpertBackend:
    def __init__(self, inp, world, rank):
        self.inp = inp
        self.k = inp.k
        self.begin, self.count = shard_bounds(inp.E, world, rank)
        self.host = slice_host(inp.host, self.begin, self.count)
        self.b1 = inp.b1[self.begin:self.begin + self.count]
        self.b2 = inp.b2[self.begin:self.begin + self.count]

    def route(self, x):
        inp = self.inp
        r = oracle.route(oracle.cfg(inp.d, inp.f, inp.E, inp.k), x.numpy(), inp.gamma, inp.gate_w, inp.gate_b)
        offsets, perm, inv = oracle.permute(r["topk_idx"], inp.E)
        t = torch.from_numpy
        return Routed(t(r["rscale"]), t(r["topk_idx"]), t(r["topk_w"]), t(offsets), t(perm), t(inv))

    def gather(self, x, r):
        perm = r.perm.numpy()
        tok = perm // self.k
        xs = x[torch.from_numpy(tok).long()]
        rs = r.rscale.numpy()[tok]
        ex = r.topk_idx.numpy().ravel()[perm].astype(np.int32)
        w = r.topk_w.numpy().ravel()[perm]
        meta = np.stack([rs.view(np.int32), ex, w.view(np.int32)], axis=1).reshape(-1, 3)
        return xs.contiguous(), torch.from_numpy(np.ascontiguousarray(meta, dtype=np.int32))

    def local(self, xr, meta):
        inp = self.inp
        R = xr.shape[0]
        if R == 0:
            return torch.zeros(0, inp.d, dtype=torch.float32)
        m = meta.numpy()
        rs = np.ascontiguousarray(m[:, 0]).view(np.float32)
        ex = m[:, 1] - self.begin
        assert (ex >= 0).all() and (ex < self.count).all()
        w = np.ascontiguousarray(m[:, 2]).view(np.float32)
        x = xr.numpy()
        normed = ((x * rs[:, None]).astype(np.float32) * inp.gamma[None, :]).astype(np.float32)
        c = oracle.cfg(inp.d, inp.f, self.count, 1, flags=oracle.FLAG_NO_RESIDUAL)
        h = self.host
        out = oracle.moe_experts(c, x, normed, ex.reshape(R, 1).astype(np.int32), w.reshape(R, 1), h.w1_blocks,
                                 h.w1_scales, self.b1, h.w2_blocks, h.w2_scales, self.b2)
        return torch.from_numpy(out)

    def combine(self, x, r, pair_out, out_dtype=None):
        xn = x.numpy()
        idx = r.topk_idx.numpy()
        inv = r.inv.numpy().reshape(idx.shape)
        po = pair_out.numpy()
        y = np.empty_like(xn)
        for t in range(xn.shape[0]):
            acc = np.zeros(xn.shape[1], np.float32)
            for s in np.argsort(idx[t], kind="stable"):
                acc = (acc + po[inv[t, s]]).astype(np.float32)
            y[t] = (xn[t] + acc).astype(np.float32)
        return torch.from_numpy(y)

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype)

    def to_host_list(self, t):
        return [int(v) for v in t.tolist()]
