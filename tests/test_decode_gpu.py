"""Decode parity on the GPU: split-context flash-decoding (through the C ABI) against the oracle
(cuda/kvcache.cu:88-129 restated in double) and the reference's own k_attn_decode compiled for
sm_100a, over the reference's [L][K|V][H][maxT][D] cache layout; plus the cache writers bit-exact
against the reference's k_kv_append / k_kv_scatter."""
import ctypes

import numpy as np
import pytest

import gpt2_b200 as G
import oracle as O
from conftest import assert_close

pytestmark = pytest.mark.gpu
L_, MAXT = 12, 1024


def host(t):
    return t.float().cpu().numpy()


@pytest.fixture(scope="module")
def cache(cuda):
    """A full GPT-2 cache (12 layers, maxT 1024) of seeded N(0,1) fp16 values, plus 12 queries."""
    rng = np.random.default_rng(123)
    arena = rng.standard_normal((L_, 2, O.H, MAXT, O.D), dtype=np.float32).astype(np.float16)
    q = rng.standard_normal((L_, O.QKV), dtype=np.float32).astype(np.float16)
    d_arena = cuda.from_numpy(arena).cuda()
    d_q = cuda.from_numpy(q).cuda()
    kv = G.cache_view(d_arena.data_ptr(), L_, MAXT)
    return dict(arena=arena.astype(np.float32), q=q.astype(np.float32), d_arena=d_arena, d_q=d_q,
                kv=kv)


@pytest.mark.parametrize("length", [1, 2, 15, 16, 17, 63, 64, 65, 127, 128, 129, 500, 1023, 1024])
def test_decode_one_layer_matches_oracle_and_reference(cuda, lib, oracle, ref_gpu, cache, length):
    kv = cache["kv"]
    for L in (0, 7, 11):
        att = cuda.empty((O.E,), dtype=cuda.float16, device="cuda")
        qrow = cache["d_q"][L]
        lib.gpt2_attn_decode_b200(att.data_ptr(), qrow.data_ptr(), ctypes.byref(kv), L, length)
        assert lib.gpt2_b200_last_error() == 0
        cuda.cuda.synchronize()
        got = host(att)
        want = oracle.decode(cache["q"][L, :O.E], cache["arena"][L, 0], cache["arena"][L, 1], length)
        assert_close(got, want, f"len={length} L={L} vs oracle")
        ref = cuda.empty_like(att)
        ref_gpu.attn_decode(ref.data_ptr(), qrow.data_ptr(), cache["d_arena"].data_ptr(), MAXT, L, length)
        assert_close(got, host(ref), f"len={length} L={L} vs reference k_attn_decode")
    assert lib.status() == 0


@pytest.mark.parametrize("ctx", [128, 512, 1023])
def test_decode_all_layers_one_launch(cuda, lib, oracle, cache, ctx):
    """Config 3's step: 12 layers of M=1 attention in a single launch."""
    att = cuda.empty((L_, O.E), dtype=cuda.float16, device="cuda")
    lib.decode_layers(att, O.E, cache["d_q"], O.QKV, cache["kv"], 0, L_, length=ctx)
    cuda.cuda.synchronize()
    got = host(att)
    for L in range(L_):
        want = oracle.decode(cache["q"][L, :O.E], cache["arena"][L, 0], cache["arena"][L, 1], ctx)
        assert_close(got[L], want, f"ctx={ctx} layer {L}")


def test_decode_graph_replay_with_device_length(cuda, lib, oracle, cache):
    """A captured CUDA graph reads the key count from device memory, so one graph serves every
    context length (the decode step is replayed as the context grows)."""
    torch = cuda
    lib.check(lib.gpt2_b200_reserve(L_, O.H, MAXT), "reserve")
    att = torch.empty((L_, O.E), dtype=torch.float16, device="cuda")
    d_len = torch.ones((1,), dtype=torch.int32, device="cuda")
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            lib.decode_layers(att, O.E, cache["d_q"], O.QKV, cache["kv"], 0, L_, d_len=d_len,
                              max_len=MAXT, stream=s.cuda_stream)
    torch.cuda.current_stream().wait_stream(s)
    for length in (1, 37, 128, 129, 1023, 1024, 5):
        d_len.fill_(length)
        g.replay()
        torch.cuda.synchronize()
        got = host(att)
        for L in (0, 11):
            want = oracle.decode(cache["q"][L, :O.E], cache["arena"][L, 0], cache["arena"][L, 1], length)
            assert_close(got[L], want, f"replay len={length} layer {L}")
    assert lib.status() == 0


def test_graph_survives_workspace_growth(cuda, lib, oracle, cache):
    """A graph captured with the split-context workspace keeps working after later calls grow the
    workspace (grown buffers are never freed while the process lives)."""
    torch = cuda
    lib.check(lib.gpt2_b200_reserve(1, O.H, MAXT), "reserve")
    att = torch.empty((O.E,), dtype=torch.float16, device="cuda")
    d_len = torch.full((1,), 700, dtype=torch.int32, device="cuda")
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):  # one layer: 12 (layer, head) pairs, split over the context
            lib.decode_layers(att, O.E, cache["d_q"][4], O.QKV, cache["kv"], 4, 1, d_len=d_len,
                              max_len=MAXT, stream=s.cuda_stream)
    torch.cuda.current_stream().wait_stream(s)
    # grow both the partials and the counters, and use the new buffers
    lib.check(lib.gpt2_b200_reserve(64, O.H, MAXT), "reserve")
    lib.check(lib.gpt2_b200_reserve(8192, O.H, MAXT), "reserve")
    other = torch.empty((3, O.E), dtype=torch.float16, device="cuda")
    lib.decode_layers(other, O.E, cache["d_q"], O.QKV, cache["kv"], 0, 3, length=999)
    for length in (700, 64, 1024):
        d_len.fill_(length)
        g.replay()
        torch.cuda.synchronize()
        want = oracle.decode(cache["q"][4, :O.E], cache["arena"][4, 0], cache["arena"][4, 1], length)
        assert_close(host(att), want, f"replay after growth, len={length}")
    assert lib.status() == 0


def test_decode_batched_sequences(cuda, lib, oracle, cache):
    """B independent caches (here: slabs of different layers) with per-sequence lengths."""
    torch = cuda
    lens = [1, 64, 65, 300, 1024, 999]
    B = len(lens)
    slab = O.H * MAXT * O.D
    base = cache["d_arena"].data_ptr()
    layers = [3, 0, 11, 5, 7, 3]
    kptr = torch.tensor([base + (2 * L) * slab * 2 for L in layers], dtype=torch.int64, device="cuda")
    vptr = torch.tensor([base + (2 * L + 1) * slab * 2 for L in layers], dtype=torch.int64, device="cuda")
    d_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = cache["d_q"][:B].contiguous()
    att = torch.empty((B, O.E), dtype=torch.float16, device="cuda")
    rc = lib.gpt2_attn_decode_b200_batched(att.data_ptr(), O.E, q.data_ptr(), O.QKV, kptr.data_ptr(),
                                           vptr.data_ptr(), d_lens.data_ptr(), B, O.H, MAXT, 0, None)
    lib.check(rc, "batched decode")
    torch.cuda.synchronize()
    got = host(att)
    for b, (L, n) in enumerate(zip(layers, lens)):
        want = oracle.decode(cache["q"][b, :O.E], cache["arena"][L, 0], cache["arena"][L, 1], n)
        assert_close(got[b], want, f"seq {b} (layer {L}, len {n})")


@pytest.mark.parametrize("B", [64, 8, 13, 16, 24, 40])
def test_decode_batched_many_sequences(cuda, lib, oracle, cache, B):
    """Batches of sequences, each (sequence, head) pair whole in one CTA: 64 x 12 heads takes the
    small-CTA shape (eight CTAs per SM), 13-40 sequences (156-480 pairs) the mid shape (up to four per
    SM), 8 sequences one CTA per SM. Lengths cover the stage edges of 32, 64 and 128 keys and the
    full cache."""
    torch = cuda
    rng = np.random.default_rng(77 + B)
    edges = [1, 2, 31, 32, 33, 63, 64, 65, 127, 128, 129, 1023, 1024]
    lens = (edges + [int(x) for x in rng.integers(1, MAXT + 1, size=max(0, B - len(edges)))])[:B]
    slab = O.H * MAXT * O.D
    base = cache["d_arena"].data_ptr()
    layers = [b % L_ for b in range(B)]
    kptr = torch.tensor([base + (2 * L) * slab * 2 for L in layers], dtype=torch.int64, device="cuda")
    vptr = torch.tensor([base + (2 * L + 1) * slab * 2 for L in layers], dtype=torch.int64, device="cuda")
    d_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.from_numpy(np.random.default_rng(78).standard_normal((B, O.QKV), dtype=np.float32)
                         .astype(np.float16)).cuda()
    att = torch.empty((B, O.E), dtype=torch.float16, device="cuda")
    rc = lib.gpt2_attn_decode_b200_batched(att.data_ptr(), O.E, q.data_ptr(), O.QKV, kptr.data_ptr(),
                                           vptr.data_ptr(), d_lens.data_ptr(), B, O.H, MAXT, 0, None)
    lib.check(rc, "batched decode")
    torch.cuda.synchronize()
    got = host(att)
    qf = host(q)
    for b, (L, n) in enumerate(zip(layers, lens)):
        want = oracle.decode(qf[b, :O.E], cache["arena"][L, 0], cache["arena"][L, 1], n)
        assert_close(got[b], want, f"seq {b} (layer {L}, len {n})")
    assert lib.status() == 0


def test_device_length_out_of_range_reports_status(cuda, lib, cache):
    torch = cuda
    att = torch.full((L_, O.E), 7.0, dtype=torch.float16, device="cuda")
    d_len = torch.zeros((1,), dtype=torch.int32, device="cuda")
    lib.decode_layers(att, O.E, cache["d_q"], O.QKV, cache["kv"], 0, L_, d_len=d_len, max_len=MAXT)
    st = lib.status(clear=True)
    assert st & G.ST_DECODE_BAD_LEN
    assert (host(att) == 7.0).all(), "no output may be written for an invalid length"
    assert lib.status() == 0


def test_scatter_and_append_bit_exact_vs_reference(cuda, lib, ref_gpu, oracle):
    torch = cuda
    T, maxt = 77, 96
    rng = np.random.default_rng(5)
    qkv = rng.standard_normal((T, O.QKV), dtype=np.float32).astype(np.float16)
    d_qkv = torch.from_numpy(qkv).cuda()
    mine = torch.zeros((L_, 2, O.H, maxt, O.D), dtype=torch.float16, device="cuda")
    ref = torch.zeros_like(mine)
    kv = G.cache_view(mine.data_ptr(), L_, maxt)
    for L in (0, 4, 11):
        lib.gpt2_kv_scatter_prefill_b200(ctypes.byref(kv), L, d_qkv.data_ptr(), T)
        assert lib.gpt2_b200_last_error() == 0
        ref_gpu.kv_scatter_prefill(ref.data_ptr(), maxt, L, d_qkv.data_ptr(), T)
        # decode-style append of row 40 at position T + 3
        lib.gpt2_kv_append_one_b200(ctypes.byref(kv), L, d_qkv[40].data_ptr(), T + 3)
        assert lib.gpt2_b200_last_error() == 0
        ref_gpu.kv_append_one(ref.data_ptr(), maxt, L, d_qkv[40].data_ptr(), T + 3)
    torch.cuda.synchronize()
    assert torch.equal(mine.view(torch.int16), ref.view(torch.int16))
    # and the oracle's restated scatter agrees
    k = np.zeros((O.H, maxt, O.D), np.uint16)
    v = np.zeros((O.H, maxt, O.D), np.uint16)
    oracle.kv_scatter(k, v, qkv.view(np.uint16))
    oracle.kv_scatter(k, v, qkv[40:41].view(np.uint16), pos0=T + 3)
    got = mine.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got[4, 0], k) and np.array_equal(got[4, 1], v)


def test_decode_attn_step_matches_reference_step(cuda, lib, ref_gpu):
    """Append-then-attend for all 12 layers (cuda/kvcache.cu:249-252), host and device position,
    against the reference's own append + decode kernels."""
    torch = cuda
    maxt, pos = 256, 200
    rng = np.random.default_rng(8)
    base = rng.standard_normal((L_, 2, O.H, maxt, O.D), dtype=np.float32).astype(np.float16)
    qkv = rng.standard_normal((L_, O.QKV), dtype=np.float32).astype(np.float16)
    d_qkv = torch.from_numpy(qkv).cuda()
    for use_dev in (False, True):
        mine = torch.from_numpy(base).cuda()
        ref = mine.clone()
        kv = G.cache_view(mine.data_ptr(), L_, maxt)
        att = torch.empty((L_, O.E), dtype=torch.float16, device="cuda")
        d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        lib.check(lib.gpt2_b200_reserve(L_, O.H, maxt), "reserve")
        rc = lib.gpt2_b200_decode_attn_step(att.data_ptr(), O.E, d_qkv.data_ptr(), O.QKV,
                                            ctypes.byref(kv), d_pos.data_ptr() if use_dev else None,
                                            pos, None)
        lib.check(rc, "decode_attn_step")
        ref_att = torch.empty_like(att)
        for L in range(L_):
            ref_gpu.kv_append_one(ref.data_ptr(), maxt, L, d_qkv[L].data_ptr(), pos)
            ref_gpu.attn_decode(ref_att[L].data_ptr(), d_qkv[L].data_ptr(), ref.data_ptr(), maxt, L,
                                pos + 1)
        torch.cuda.synchronize()
        assert torch.equal(mine.view(torch.int16), ref.view(torch.int16)), "cache after append"
        assert_close(host(att), host(ref_att), f"step attention (device pos={use_dev})")
    assert lib.status() == 0
