"""Prefill parity on the GPU: the tcgen05 kernel (through the C ABI) against the oracle (the
reference's cpu/forward_cpu.c attention restated, double precision) and against the reference's own
k_attention_flash (cuda/kernels_fused.cu:58-149) compiled for sm_100a, on the same seeded fp16 inputs.
Tolerance: max-abs 2e-3 and max|diff|/max|ref| 1e-2 (conftest.ABS_TOL / REL_TOL)."""
import os

import numpy as np
import pytest

import oracle as O
from conftest import assert_close

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SENTINEL = 12344.0  # exactly representable in fp16


def dev16(torch, x):
    return torch.from_numpy(np.ascontiguousarray(x).astype(np.float16)).cuda()


def host(t):
    return t.float().cpu().numpy()


# T values: 1, tile edges (127/128/129, 255/256/257), the reference's odd prompt length 161, 1024.
@pytest.mark.parametrize("T", [1, 2, 31, 32, 33, 127, 128, 129, 161, 255, 256, 257, 512, 1000, 1024])
def test_prefill_matches_oracle_and_reference_flash(cuda, lib, oracle, ref_gpu, T):
    x = O.seeded_qkv(2000 + T, T)
    qkv = dev16(cuda, x)
    att = cuda.full((T, O.E), SENTINEL, dtype=cuda.float16, device="cuda")
    lib.prefill(att, qkv, T)
    cuda.cuda.synchronize()
    assert lib.status() == 0
    got = host(att)
    assert_close(got, oracle.prefill(x), f"T={T} vs oracle")
    ref = cuda.empty_like(att)
    ref_gpu.attention_flash(ref.data_ptr(), qkv.data_ptr(), T)
    assert_close(got, host(ref), f"T={T} vs reference k_attention_flash")


def test_reference_signature_entry_point(cuda, lib, oracle, ref_gpu):
    """gpt2_attention_b200 has GPT2Backend.attention's exact signature (cuda/kernels.cuh:73)."""
    T = 155
    x = O.seeded_qkv(155, T)
    qkv = dev16(cuda, x)
    att = cuda.empty((T, O.E), dtype=cuda.float16, device="cuda")
    lib.gpt2_attention_b200(att.data_ptr(), qkv.data_ptr(), T, O.E, O.H, O.D)
    assert lib.gpt2_b200_last_error() == 0
    cuda.cuda.synchronize()
    assert_close(host(att), oracle.prefill(x), "void entry point")
    naive = cuda.empty_like(att)
    ref_gpu.attention_naive(naive.data_ptr(), qkv.data_ptr(), T)
    assert_close(host(att), host(naive), "vs reference k_attention (naive)")


def test_config1_golden_vector(cuda, lib):
    """Config 1 (B=1, P=128): GPU output against the reference-generated golden att."""
    g = np.load(os.path.join(GOLD, "prefill_T128_cfg1.npz"))
    x = O.seeded_qkv(int(g["seed"]), int(g["T"]))
    att = cuda.empty((128, O.E), dtype=cuda.float16, device="cuda")
    lib.prefill(att, dev16(cuda, x), 128)
    cuda.cuda.synchronize()
    assert_close(host(att), g["att"], "config 1 golden")


def test_golden_T40(cuda, lib):
    g = np.load(os.path.join(GOLD, "prefill_T40.npz"))
    qkv = cuda.from_numpy(g["qkv_f16"].view(np.float16).copy()).cuda()
    att = cuda.empty((40, O.E), dtype=cuda.float16, device="cuda")
    lib.prefill(att, qkv, 40)
    cuda.cuda.synchronize()
    assert_close(host(att), g["att"], "T40 golden")


def test_batched_twelve_layers_P1024(cuda, lib, oracle):
    """Config 2's shape: 12 independent layers of P=1024 in one launch."""
    B, T = 12, 1024
    xs = [O.seeded_qkv(3000 + b, T) for b in range(B)]
    qkv = dev16(cuda, np.stack(xs))
    att = cuda.empty((B, T, O.E), dtype=cuda.float16, device="cuda")
    lib.prefill(att, qkv, T, B=B)
    cuda.cuda.synchronize()
    assert lib.status() == 0
    got = host(att)
    for b in (0, 5, 11):
        assert_close(got[b], oracle.prefill(xs[b]), f"layer {b}")


def test_batched_strides_and_canaries(cuda, lib, oracle):
    """Padded per-sequence strides: the kernel reads only its rows and writes only its rows."""
    B, T, pad = 3, 200, 2
    xs = [O.seeded_qkv(4000 + b, T) for b in range(B)]
    qkv_full = np.zeros((B, T + 1, O.QKV), np.float32)
    qkv_full[:, :T] = np.stack(xs)
    qkv_full[:, T] = 60000.0  # poison row after each sequence: must never be read
    qkv = dev16(cuda, qkv_full)
    att = cuda.full((B, T + pad, O.E), SENTINEL, dtype=cuda.float16, device="cuda")
    lib.prefill(att, qkv, T, B=B, qkv_stride=(T + 1) * O.QKV, att_stride=(T + pad) * O.E)
    cuda.cuda.synchronize()
    got = host(att)
    assert (got[:, T:] == SENTINEL).all(), "write outside [0, T)"
    for b in range(B):
        assert_close(got[b, :T], oracle.prefill(xs[b]), f"seq {b}")


def test_deterministic(cuda, lib):
    T = 700
    qkv = dev16(cuda, O.seeded_qkv(9, T))
    a = cuda.empty((T, O.E), dtype=cuda.float16, device="cuda")
    b = cuda.empty_like(a)
    lib.prefill(a, qkv, T)
    lib.prefill(b, qkv, T)
    cuda.cuda.synchronize()
    assert cuda.equal(a, b)


def test_large_scores_stay_finite(cuda, lib, oracle):
    """Large |q.k| (values ~ N(0, 8^2)) exercises the running-max rescale path."""
    T = 384
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((T, O.QKV)) * 8).astype(np.float16).astype(np.float32)
    x[:, 2 * O.E:] /= 8  # keep v ~ N(0,1) so the abs tolerance stays meaningful
    att = cuda.empty((T, O.E), dtype=cuda.float16, device="cuda")
    lib.prefill(att, dev16(cuda, x), T)
    cuda.cuda.synchronize()
    assert_close(host(att), oracle.prefill(x), "large scores")


@pytest.mark.parametrize("T", [1, 129, 300, 1024])
def test_attention_with_kv_fill_matches_scatter_then_attention(cuda, lib, ref_gpu, T):
    """gpt2_attention_kv_b200_stream = the reference's gpt2_kv_scatter_prefill followed by attention
    (cuda/forward_cuda.cu:97-98), bit-exact: att equals the plain prefill's, and the whole cache arena
    equals the one the reference's own k_kv_scatter writes (rows >= T and other layers untouched).
    T = 1024 on one layer takes the split-unit path; the others keep whole pairs."""
    import ctypes
    import gpt2_b200 as G
    torch = cuda
    maxt, n_layer = 1024, 12
    x = O.seeded_qkv(900 + T, T)
    d_qkv = dev16(torch, x)
    mine = torch.full((n_layer, 2, O.H, maxt, O.D), -3.0, dtype=torch.float16, device="cuda")
    ref = mine.clone()
    kv = G.cache_view(mine.data_ptr(), n_layer, maxt)
    att = torch.empty((T, O.E), dtype=torch.float16, device="cuda")
    plain = torch.empty_like(att)
    for L in (0, 11):
        rc = lib.gpt2_attention_kv_b200_stream(att.data_ptr(), d_qkv.data_ptr(), ctypes.byref(kv), L, T,
                                               O.E, O.H, O.D, None)
        assert rc == 0
        ref_gpu.kv_scatter_prefill(ref.data_ptr(), maxt, L, d_qkv.data_ptr(), T)
        lib.prefill(plain, d_qkv, T)
        torch.cuda.synchronize()
        assert torch.equal(att.view(torch.int16), plain.view(torch.int16))
    assert torch.equal(mine.view(torch.int16), ref.view(torch.int16))
    assert lib.status() == 0


def test_attention_with_kv_fill_rejects_bad_cache(cuda, lib):
    import ctypes
    import gpt2_b200 as G
    torch = cuda
    T, maxt = 300, 256
    d_qkv = torch.zeros((T, O.QKV), dtype=torch.float16, device="cuda")
    arena = torch.zeros((12, 2, O.H, maxt, O.D), dtype=torch.float16, device="cuda")
    att = torch.empty((T, O.E), dtype=torch.float16, device="cuda")
    kv = G.cache_view(arena.data_ptr(), 12, maxt)
    # T beyond the cache's maxT, and a layer past nLayer: refused, nothing launched
    assert lib.gpt2_attention_kv_b200_stream(att.data_ptr(), d_qkv.data_ptr(), ctypes.byref(kv), 0, T,
                                             O.E, O.H, O.D, None) == G.EINVAL
    kv2 = G.cache_view(arena.data_ptr(), 12, maxt)
    assert lib.gpt2_attention_kv_b200_stream(att.data_ptr(), d_qkv.data_ptr(), ctypes.byref(kv2), 12, 100,
                                             O.E, O.H, O.D, None) == G.EINVAL
    assert lib.status() == 0


@pytest.mark.parametrize("T", [1400, 2048, 4096])
def test_single_layer_long_prompts_split_path(cuda, lib, oracle, T):
    """One layer of one long sequence. At T=1400 and 2048 there are too few whole pairs to fill the SMs,
    so the key ranges of the long query tiles are split into chunks run by the CTAs of a cluster and
    merged there (T=1400: chunks of single query tiles, an odd tile count; T=2048: chunks of pairs);
    T=4096 has enough whole pairs. Checked against the oracle on a sample of rows across the range,
    plus the last row."""
    torch = cuda
    x = O.seeded_qkv(4000 + T, T)
    att = torch.empty((T, O.E), dtype=torch.float16, device="cuda")
    lib.prefill(att, dev16(torch, x), T)
    torch.cuda.synchronize()
    assert lib.status() == 0
    got = host(att)
    rows = sorted(set(list(range(0, T, 97)) + [T - 1]))
    ref = oracle.prefill(x)
    assert_close(got[rows], ref[rows], f"T={T} sampled rows vs oracle")


# (B, T) of split launches. Single-query-tile units (the two softmax groups of a CTA take alternate
# key tiles and merge locally): in clusters of 3 chunks (T=640), of 2 (T=1152, B=2 at T=512 and 640)
# and unclustered (T=1536; B=2 at T=700, ragged last tile); chunks of pairs in clusters of 2 at
# T=1792 (7-tile chunks, ragged). B=3 at T=512 keeps whole pairs.
@pytest.mark.parametrize("B,T", [(1, 640), (1, 1152), (1, 1536), (1, 1792), (2, 512), (2, 640), (2, 700),
                                 (3, 512)])
def test_split_units_cluster_shapes(cuda, lib, oracle, B, T):
    torch = cuda
    xs = [O.seeded_qkv(6100 + 7 * b + T, T) for b in range(B)]
    att = torch.full((B, T, O.E), SENTINEL, dtype=torch.float16, device="cuda")
    lib.prefill(att, dev16(torch, np.stack(xs)), T, B=B)
    torch.cuda.synchronize()
    assert lib.status() == 0
    got = host(att)
    for b in range(B):
        assert_close(got[b], oracle.prefill(xs[b]), f"B={B} T={T} seq {b}")


def test_single_layer_prefill_in_cuda_graph(cuda, lib, oracle):
    """A one-layer launch takes the split-unit path (clusters of chunks of a pair). Captured in a graph,
    first before any eager call and then after one, it must reproduce the eager result across
    replays."""
    torch = cuda
    T = 1024
    x = O.seeded_qkv(5150, T)
    d_qkv = dev16(torch, x)
    ref = oracle.prefill(x)
    s = torch.cuda.Stream()
    outs = []
    for _ in range(2):  # the first capture precedes every eager split launch of this size
        att = torch.empty((T, O.E), dtype=torch.float16, device="cuda")
        g = torch.cuda.CUDAGraph()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g, stream=s):
            rc = lib.gpt2_attention_b200_stream(att.data_ptr(), d_qkv.data_ptr(), T, O.E, O.H, O.D,
                                                s.cuda_stream)
            assert rc == 0
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            att.fill_(0)
            g.replay()
            torch.cuda.synchronize()
            assert_close(host(att), ref, "graph-replayed one-layer prefill")
        outs.append(att.clone())
        eager = torch.empty_like(att)
        lib.prefill(eager, d_qkv, T)
        torch.cuda.synchronize()
        outs.append(eager)
        del g
    assert lib.status() == 0


def test_first_call_inside_graph_capture(cuda):
    """A fresh process whose first prefill call (one layer, so the split path with its one-time
    cluster occupancy query and kernel attribute set-up) is made while capturing a CUDA graph: the
    capture must stay valid and the replay must match an eager call."""
    import subprocess
    import sys
    code = r"""
import sys, numpy as np, torch
sys.path.insert(0, %r)
import gpt2_b200 as G
lib = G.load()
torch.cuda.set_device(0)
T = 1024
g = torch.Generator().manual_seed(7)
qkv = torch.randn(T, 2304, generator=g).half().cuda()
att = torch.empty(T, 768, dtype=torch.float16, device="cuda")
s = torch.cuda.Stream()
s.wait_stream(torch.cuda.current_stream())
graph = torch.cuda.CUDAGraph()
with torch.cuda.graph(graph, stream=s):
    assert lib.gpt2_attention_b200_stream(att.data_ptr(), qkv.data_ptr(), T, 768, 12, 64, s.cuda_stream) == 0
torch.cuda.current_stream().wait_stream(s)
graph.replay()
torch.cuda.synchronize()
eager = torch.empty_like(att)
lib.prefill(eager, qkv, T)
torch.cuda.synchronize()
assert lib.status() == 0
assert torch.equal(att, eager), "replayed graph differs from the eager call"
print("ok")
""" % (os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bare-metal-gpt2_b200"),)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
