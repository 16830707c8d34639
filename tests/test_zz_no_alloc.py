"""The no-allocation decode entry point, checked through the C ABI against the oracle and against the
regular entry point.

gpt2_attn_decode_b200_layers_noalloc exists for callers that cannot let a library allocate device
memory: a serving loop whose pool allocator already owns all of HBM, a host that freezes device
allocations once it has initialised, a latency-critical loop that cannot absorb a synchronising
cudaMalloc. It runs its own split-context kernel (k_decode_split) with the scratch in a fixed array
inside the library. This file is named so pytest collects it last; it also passes on its own in a
fresh process.
"""
import ctypes
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import gpt2_b200 as G
from conftest import assert_close

pytestmark = pytest.mark.gpu
L_, H_, MAXT, E_, QKV_ = 12, 12, 1024, 768, 2304
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _setup(torch, seed):
    rng = np.random.default_rng(seed)
    arena = rng.standard_normal((L_, 2, H_, MAXT, 64), dtype=np.float32).astype(np.float16)
    q = rng.standard_normal((L_, QKV_), dtype=np.float32).astype(np.float16)
    d_arena = torch.from_numpy(arena).cuda()
    d_q = torch.from_numpy(q).cuda()
    return arena.astype(np.float32), q.astype(np.float32), d_arena, d_q, G.cache_view(
        d_arena.data_ptr(), L_, MAXT)


def _noalloc(lib, out, q, kv, L0, nL, length):
    return lib.gpt2_attn_decode_b200_layers_noalloc(out.data_ptr(), E_, q.data_ptr(), QKV_,
                                                    ctypes.byref(kv), L0, nL, length, None)


def test_no_alloc_decode_matches_regular_entry_point_twice(cuda, lib, oracle):
    torch = cuda
    # two calls in a row, different caches and lengths: the second must not see the first's scratch
    for seed, length in ((1, 1023), (2, 300)):
        arena, qh, _, q, kv = _setup(torch, seed)
        want = torch.empty((L_, E_), dtype=torch.float16, device="cuda")
        got = torch.full((L_, E_), 9.0, dtype=torch.float16, device="cuda")
        lib.check(lib.gpt2_attn_decode_b200_layers(want.data_ptr(), E_, q.data_ptr(), QKV_,
                                                   ctypes.byref(kv), 0, L_, None, length, length,
                                                   None), "regular decode")
        torch.cuda.synchronize()
        rc = _noalloc(lib, got, q, kv, 0, L_, length)
        assert rc == G.OK, lib.gpt2_b200_strerror(rc)
        torch.cuda.synchronize()
        g = got.float().cpu().numpy()
        assert_close(g, want.float().cpu().numpy(), f"no-alloc vs regular, len {length}")
        for L in (0, 11):
            assert_close(g[L], oracle.decode(qh[L, :E_], arena[L, 0], arena[L, 1], length),
                         f"no-alloc vs oracle, len {length}, layer {L}")
    assert lib.status() == 0


@pytest.mark.parametrize("length", [1, 64, 128, 129, 1024])
@pytest.mark.parametrize("L0,nL", [(0, 12), (3, 4)])
def test_no_alloc_decode_lengths_and_layer_ranges(cuda, lib, oracle, length, L0, nL):
    """One split (len <= 128, output written directly) and several (a merge through the scratch),
    up to the whole cache; all layers, and a range that starts past layer 0."""
    torch = cuda
    arena, qh, _, q, kv = _setup(torch, 10 + length)
    got = torch.full((nL, E_), 9.0, dtype=torch.float16, device="cuda")
    qs = q[L0:]
    rc = lib.gpt2_attn_decode_b200_layers_noalloc(got.data_ptr(), E_, qs.data_ptr(), QKV_,
                                                  ctypes.byref(kv), L0, nL, length, None)
    assert rc == G.OK, lib.gpt2_b200_strerror(rc)
    want = torch.empty((nL, E_), dtype=torch.float16, device="cuda")
    lib.check(lib.gpt2_attn_decode_b200_layers(want.data_ptr(), E_, qs.data_ptr(), QKV_,
                                               ctypes.byref(kv), L0, nL, None, length, length, None),
              "regular decode")
    torch.cuda.synchronize()
    g = got.float().cpu().numpy()
    for i in range(nL):
        L = L0 + i
        assert_close(g[i], oracle.decode(qh[L, :E_], arena[L, 0], arena[L, 1], length),
                     f"len {length}, layer {L} vs oracle")
    assert_close(g, want.float().cpu().numpy(), f"len {length}, layers {L0}..{L0 + nL - 1} vs regular")
    assert lib.status() == 0


def test_no_alloc_decode_leaves_free_memory_unchanged(cuda, lib):
    """Once the library is on the device, calls of every size move no device memory."""
    torch = cuda
    _, _, _, q, kv = _setup(torch, 3)
    out = torch.empty((L_, E_), dtype=torch.float16, device="cuda")
    assert _noalloc(lib, out, q, kv, 0, 1, 5) == G.OK  # warm-up: the smallest request
    torch.cuda.synchronize()
    before = torch.cuda.mem_get_info()[0]
    for nL, length in ((1, 129), (12, 700), (12, 1024), (4, 1)):  # up to the largest scratch use
        assert _noalloc(lib, out, q, kv, 0, nL, length) == G.OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == before


_FRESH = r"""
import ctypes, json, sys
import numpy as np
from cuda.bindings import runtime as rt
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import gpt2_b200 as G
import oracle as O

def ok(r):
    err = r[0] if isinstance(r, tuple) else r
    assert err == rt.cudaError_t.cudaSuccess, err
    return r[1] if isinstance(r, tuple) and len(r) > 1 else None

L, H, T, E, QKV, n = 12, 12, 1024, 768, 2304, 1000
rng = np.random.default_rng(7)
arena = rng.standard_normal((L, 2, H, T, 64), dtype=np.float32).astype(np.float16)
q = rng.standard_normal((L, QKV), dtype=np.float32).astype(np.float16)
ok(rt.cudaSetDevice(0))
d_arena = ok(rt.cudaMalloc(arena.nbytes))
d_q = ok(rt.cudaMalloc(q.nbytes))
d_out = ok(rt.cudaMalloc(L * E * 2))
ok(rt.cudaMemcpy(d_arena, arena.ctypes.data, arena.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice))
ok(rt.cudaMemcpy(d_q, q.ctypes.data, q.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice))
lib = G.load()
# A refused cache plan: the library's runtime starts on this device (and, with eager module loading,
# places its module), but the refusal allocates nothing.
probe = G.GPT2KVCache()
assert lib.gpt2_kv_alloc_b200(ctypes.byref(probe), 1 << 30) == 1 and not probe.data
ok(rt.cudaDeviceSynchronize())
free0 = ok(rt.cudaMemGetInfo())
kv = G.cache_view(int(d_arena), L, T)
rc = lib.gpt2_attn_decode_b200_layers_noalloc(int(d_out), E, int(d_q), QKV, ctypes.byref(kv), 0, L, n, None)
ok(rt.cudaDeviceSynchronize())
free1 = ok(rt.cudaMemGetInfo())
out = np.empty((L, E), dtype=np.float16)
ok(rt.cudaMemcpy(out.ctypes.data, d_out, out.nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost))
a = arena.astype(np.float32)
orc = O.Oracle()
err = max(float(np.abs(out[l].astype(np.float64) - orc.decode(q[l, :E].astype(np.float32), a[l, 0], a[l, 1], n)).max())
          for l in range(L))
print(json.dumps({"rc": rc, "free_before": int(free0), "free_after": int(free1), "max_abs": err}))
"""


def test_no_alloc_first_call_on_a_fresh_device_allocates_nothing():
    """A fresh process with eager module loading (the library's code and fixed array are placed on the
    device when its runtime starts there) and no torch: the FIRST no-allocation call leaves the
    device's free memory unchanged, and its output matches the oracle."""
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER", CUDA_VISIBLE_DEVICES=os.environ.get(
        "CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    r = subprocess.run([sys.executable, "-c", _FRESH, os.path.join(ROOT, "bare-metal-gpt2_b200"),
                        os.path.join(ROOT, "oracle")], capture_output=True, text=True, timeout=300,
                       env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["rc"] == G.OK
    assert d["free_after"] == d["free_before"], d
    assert d["max_abs"] <= 2e-3, d


def test_no_alloc_decode_refuses_requests_beyond_its_scratch(cuda, lib):
    kv = G.cache_view(1 << 20, 200, 2048)  # 200 layers x 12 heads: over the fixed limit
    rc = lib.gpt2_attn_decode_b200_layers_noalloc(1 << 20, E_, 1 << 20, QKV_, ctypes.byref(kv), 0, 200,
                                                  2048, None)
    assert rc == G.EINVAL
    kv = G.cache_view(1 << 20, 16, 2048)  # 16 layers x 12 heads x 16 splits of 128 keys: too many
    rc = lib.gpt2_attn_decode_b200_layers_noalloc(1 << 20, E_, 1 << 20, QKV_, ctypes.byref(kv), 0, 16,
                                                  2048, None)
    assert rc == G.EINVAL
