"""Worker of test_gpu_ep_multi: one rank per GPU (torchrun).  Runs the
quantized peer-memory expert-parallel layer and the full single-GPU layer on
this rank's tokens and checks them against each other; rank 0 prints one
JSON line with every rank's error."""
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, "..", "burn-extended_b200"), HERE]

import mxmoe  # noqa: E402
from mxmoe import ep, synth  # noqa: E402


def errors(y, ref):
    """(max |y - ref| / max |ref|, relative L2), as the parity tests measure."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    return np.abs(y - ref).max() / scale, np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    dist.init_process_group("nccl", device_id=dev)
    n, E, k = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3])
    # one model on every rank; each rank routes its own tokens
    inp = synth.rank_tokens(synth.make_inputs(512, 384, E, k, n, True, seed=100, zipf_router_bias=0.7), rank)
    m = ep.build_quantized_peer_rank(inp, world, rank, dev)
    full = mxmoe.MoeConfig(inp.d, inp.f, inp.E, inp.k).init(local)
    full.set_router(inp.gamma, inp.gate_w, inp.gate_b)
    full.set_resident(inp.host, inp.b1, inp.b2)
    x = torch.from_numpy(inp.x).to(torch.bfloat16).to(dev)
    res = []
    for _ in range(3):  # repeated steps reuse every buffer
        y = m.forward(x, out_dtype=torch.float32)
        want = full.forward(x, out_dtype=torch.float32)
        torch.cuda.synchronize()
        res.append(errors(y.cpu().numpy(), want.cpu().numpy()))
    m.backend.layer.sync_status()
    err = int(m.err.item()) if hasattr(m, "err") else 0
    out = [None] * world
    dist.all_gather_object(out, {"rank": rank, "errors": [list(map(float, r)) for r in res], "err": err})
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    m.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
