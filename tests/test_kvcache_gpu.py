"""The KV-cache lifecycle on the GPU: gpt2_kv_alloc_b200 / _free / _reset / _step_bytes, the
replacements of the reference's planner (cuda/kvcache.cu:25-52), including its refusal to allocate a
plan that would leave less than 64 MiB of device memory free (cuda/kvcache.cu:31-35), and a cache
allocated by the library used end to end: filled by the prefill scatter and the append, read by the
decode attention, checked against the oracle."""
import ctypes

import numpy as np
import pytest

import gpt2_b200 as G
import oracle as O
from conftest import assert_close

pytestmark = pytest.mark.gpu
SLOT = 2 * 12 * 12 * 64 * 2  # bytes per cache position (K and V, 12 layers x 12 heads x 64 fp16)


def test_alloc_fills_the_descriptor_and_free_returns_the_memory(cuda, lib):
    torch = cuda
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    kv = G.GPT2KVCache()
    kv.len = 77
    assert lib.gpt2_kv_alloc_b200(ctypes.byref(kv), 1024) == 0
    assert kv.data and kv.data % 256 == 0
    assert (kv.maxT, kv.nLayer, kv.nHead, kv.headDim, kv.len) == (1024, 12, 12, 64, 0)
    assert kv.bytes == 1024 * SLOT == 37748736  # 37.7 MB, as the reference prints for maxT 1024
    assert free0 - torch.cuda.mem_get_info()[0] >= kv.bytes
    assert lib.gpt2_kv_step_bytes_b200(ctypes.byref(kv), 1023) == 2.0 * 12 * 12 * 1023 * 64 * 2
    kv.len = 5
    data = kv.data
    lib.gpt2_kv_reset_b200(ctypes.byref(kv))  # resets the length only, as the reference does
    assert kv.len == 0 and kv.data == data and kv.maxT == 1024
    lib.gpt2_kv_free_b200(ctypes.byref(kv))
    assert not kv.data
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] >= free0 - (2 << 20)
    lib.gpt2_kv_free_b200(ctypes.byref(kv))  # a second free of the same descriptor is a no-op
    lib.gpt2_kv_free_b200(None)


def test_alloc_refuses_a_plan_inside_the_64_MiB_headroom(cuda, lib):
    """A plan that fits in free memory but would leave less than 64 MiB is refused (returns 1) and
    allocates nothing; so is one larger than the device."""
    torch = cuda
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for max_t in ((free0 - (32 << 20)) // SLOT, (free0 - (63 << 20)) // SLOT, 4 * free0 // SLOT):
        kv = G.GPT2KVCache()
        assert lib.gpt2_kv_alloc_b200(ctypes.byref(kv), int(max_t)) == 1, max_t
        assert not kv.data
        assert kv.bytes == max_t * SLOT
    torch.cuda.synchronize()
    assert abs(torch.cuda.mem_get_info()[0] - free0) < (2 << 20)
    kv = G.GPT2KVCache()
    assert lib.gpt2_kv_alloc_b200(ctypes.byref(kv), 0) == 1  # no positions: refused, no allocation
    assert not kv.data


def test_library_allocated_cache_round_trip(cuda, lib, oracle):
    """Prefill scatter of T rows, one append at position T, then decode over T+1 keys, all through
    the library on a cache it allocated; compared with the oracle over the same fp16 values."""
    torch = cuda
    T, L = 300, 5
    rng = np.random.default_rng(9)
    x = rng.standard_normal((T + 1, O.QKV), dtype=np.float32).astype(np.float16)
    d_x = torch.from_numpy(x).cuda()
    kv = G.GPT2KVCache()
    assert lib.gpt2_kv_alloc_b200(ctypes.byref(kv), 512) == 0
    try:
        lib.gpt2_kv_scatter_prefill_b200(ctypes.byref(kv), L, d_x.data_ptr(), T)
        assert lib.gpt2_b200_last_error() == 0
        lib.gpt2_kv_append_one_b200(ctypes.byref(kv), L, d_x[T].data_ptr(), T)
        assert lib.gpt2_b200_last_error() == 0
        att = torch.empty((O.E,), dtype=torch.float16, device="cuda")
        lib.gpt2_attn_decode_b200(att.data_ptr(), d_x[T].data_ptr(), ctypes.byref(kv), L, T + 1)
        assert lib.gpt2_b200_last_error() == 0
        torch.cuda.synchronize()
        xf = x.astype(np.float32)
        k = np.zeros((O.H, 512, O.D), np.float32)
        v = np.zeros((O.H, 512, O.D), np.float32)
        k[:, :T + 1] = xf[:, O.E:2 * O.E].reshape(T + 1, O.H, O.D).transpose(1, 0, 2)
        v[:, :T + 1] = xf[:, 2 * O.E:].reshape(T + 1, O.H, O.D).transpose(1, 0, 2)
        want = oracle.decode(xf[T, :O.E], k, v, T + 1)
        assert_close(att.float().cpu().numpy(), want, "decode over a library-allocated cache")
        # the cache holds exactly the K/V rows written (bit-exact, reference layout)
        arena = np.empty(kv.bytes // 2, dtype=np.float16)
        from cuda.bindings import runtime as rt
        (err,) = rt.cudaMemcpy(arena.ctypes.data, kv.data, kv.bytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert err == rt.cudaError_t.cudaSuccess
        lay = arena.reshape(12, 2, 12, 512, 64)[L]
        assert np.array_equal(lay[0][:, :T + 1], x[:, O.E:2 * O.E].reshape(T + 1, 12, 64).transpose(1, 0, 2))
        assert np.array_equal(lay[1][:, :T + 1], x[:, 2 * O.E:].reshape(T + 1, 12, 64).transpose(1, 0, 2))
    finally:
        lib.gpt2_kv_free_b200(ctypes.byref(kv))
    assert lib.status() == 0
