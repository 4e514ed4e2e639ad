"""mxmoe_permute_noalloc through the C ABI: the permutation entry point for
callers that cannot allocate device memory (for example code whose device
memory is all owned by an arena or caching allocator) must give exactly what
mxmoe_permute gives, call after call, while using only the library's fixed
scratch array."""
import ctypes

import numpy as np
import pytest

from mxmoe import _lib

pytestmark = pytest.mark.gpu


def _run(fn_name, topk, E):
    import torch
    L = _lib.lib()
    n, k = topk.shape
    t = torch.from_numpy(topk).cuda()
    offsets = torch.full((E + 1,), -1, dtype=torch.int32, device="cuda")
    perm = torch.full((n * k,), -1, dtype=torch.int32, device="cuda")
    inv = torch.full((n * k,), -1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(getattr(L, fn_name)(t.data_ptr(), n, k, E, offsets.data_ptr(), perm.data_ptr(), inv.data_ptr(),
                                   stream))
    torch.cuda.synchronize()
    return offsets.cpu().numpy(), perm.cpu().numpy(), inv.cpu().numpy()


def test_noalloc_permute_matches_permute_twice_in_a_row():
    rng = np.random.default_rng(7)
    # two consecutive calls with different shapes: the second must not see
    # anything left in the shared scratch by the first
    for n, k, E in ((4096, 4, 128), (300, 2, 8)):
        topk = np.stack([rng.permutation(E)[:k] for _ in range(n)]).astype(np.int32)
        want = _run("mxmoe_permute", topk, E)
        got = _run("mxmoe_permute_noalloc", topk, E)
        for w, g in zip(want, got):
            assert np.array_equal(g, w)


def test_noalloc_permute_rejects_too_many_experts():
    L = _lib.lib()
    rc = L.mxmoe_permute_noalloc(None, 0, 1, 1025, None, None, None, None)
    assert rc == 7  # MXMOE_ERR_TOO_LARGE
    assert "1024" in _lib.last_error()
