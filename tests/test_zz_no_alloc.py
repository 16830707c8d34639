"""The no-allocation decode entry point, checked against the regular one through the C ABI.

gpt2_attn_decode_b200_layers_noalloc exists for callers that cannot let a library allocate device
memory (a pool allocator that already owns all of HBM, a host that freezes allocations after
start-up, a latency-critical loop that cannot absorb a synchronising cudaMalloc). It runs the same
split-context kernel with its scratch in a fixed array inside the library. This file is named so
pytest collects it last; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import gpt2_b200 as G
from conftest import assert_close

pytestmark = pytest.mark.gpu
L_, H_, MAXT, E_, QKV_ = 12, 12, 1024, 768, 2304


def _setup(torch, seed):
    rng = np.random.default_rng(seed)
    arena = torch.from_numpy(
        rng.standard_normal((L_, 2, H_, MAXT, 64), dtype=np.float32).astype(np.float16)).cuda()
    q = torch.from_numpy(rng.standard_normal((L_, QKV_), dtype=np.float32).astype(np.float16)).cuda()
    return arena, q, G.cache_view(arena.data_ptr(), L_, MAXT)


def test_no_alloc_decode_matches_regular_entry_point_twice(cuda, lib):
    torch = cuda
    # two calls in a row, different caches and lengths: the second must not see the first's scratch
    for seed, length in ((1, 1023), (2, 300)):
        arena, q, kv = _setup(torch, seed)
        want = torch.empty((L_, E_), dtype=torch.float16, device="cuda")
        got = torch.full((L_, E_), 9.0, dtype=torch.float16, device="cuda")
        lib.check(lib.gpt2_attn_decode_b200_layers(want.data_ptr(), E_, q.data_ptr(), QKV_,
                                                   ctypes.byref(kv), 0, L_, None, length, length,
                                                   None), "regular decode")
        torch.cuda.synchronize()
        rc = lib.gpt2_attn_decode_b200_layers_noalloc(got.data_ptr(), E_, q.data_ptr(), QKV_,
                                                      ctypes.byref(kv), 0, L_, length, None)
        assert rc == G.OK, lib.gpt2_b200_strerror(rc)
        torch.cuda.synchronize()
        assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(),
                     f"no-alloc vs regular, len {length}")


def test_no_alloc_decode_refuses_requests_beyond_its_scratch(cuda, lib):
    kv = G.cache_view(1 << 20, 200, 2048)  # 200 layers x 12 heads: over the fixed limit
    rc = lib.gpt2_attn_decode_b200_layers_noalloc(1 << 20, E_, 1 << 20, QKV_, ctypes.byref(kv), 0, 200,
                                                  2048, None)
    assert rc == G.EINVAL
