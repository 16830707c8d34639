"""C ABI surface checks that need no GPU: exports, header validity, struct layouts, host logic and
argument validation (which happens before any CUDA call)."""
import ctypes
import os
import subprocess
import tempfile

import pytest

import gpt2_b200 as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# The reference tree (build container only): $GPT2_REFERENCE_DIR, else `reference` beside this repo.
REF_DIR = os.environ.get("GPT2_REFERENCE_DIR", os.path.join(os.path.dirname(ROOT), "reference"))


def test_library_exports_every_declared_function(lib):
    declared = G.header_functions()
    assert len(declared) >= 20
    missing = [n for n in declared if not hasattr(lib.lib, n)]
    assert not missing, f"declared in include/gpt2_b200.h but not exported: {missing}"
    # and the binding declares a signature for each
    assert sorted(G._SIGS) == declared


def _compile_c_probe(src: str) -> str:
    d = tempfile.mkdtemp()
    c = os.path.join(d, "probe.c")
    exe = os.path.join(d, "probe")
    open(c, "w").write(src)
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    "-I", "/usr/local/cuda/include", "-o", exe, c], check=True,
                   capture_output=True)
    return subprocess.run([exe], check=True, capture_output=True, text=True).stdout


def test_header_is_valid_c_and_struct_layouts_match_reference():
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "gpt2_b200.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu\n", sizeof(GPT2KVCache), offsetof(GPT2KVCache, bytes),
         offsetof(GPT2KVCache, maxT), offsetof(GPT2KVCache, len), sizeof(GPT2Backend),
         offsetof(GPT2Backend, attention));
  return 0;
}'''
    vals = [int(x) for x in _compile_c_probe(src).split()]
    # GPT2KVCache {half*; size_t; int x4; int len} (cuda/kvcache.cuh:39-44) on LP64
    assert vals[:4] == [40, 8, 16, 32]
    assert vals[0] == ctypes.sizeof(G.GPT2KVCache)
    # GPT2Backend: name + 9 function pointers (cuda/kernels.cuh:68-86); .attention is slot 4
    assert vals[4] == 80 and vals[5] == 32
    assert vals[4] == ctypes.sizeof(G.GPT2Backend)


def test_model_struct_layouts_match_reference():
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "gpt2_b200.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu\n", sizeof(GPT2LayerGPU), offsetof(GPT2LayerGPU, proj_b),
         sizeof(GPT2WeightsGPU), offsetof(GPT2WeightsGPU, layers), offsetof(GPT2WeightsGPU, lnf_g),
         offsetof(GPT2WeightsGPU, q), sizeof(GPT2ScratchGPU));
  return 0;
}'''
    vals = [int(x) for x in _compile_c_probe(src).split()]
    # GPT2LayerGPU: 12 half* (cuda/kernels.cuh:19-23); GPT2WeightsGPU {half*, size_t, wte, wpe,
    # layers[12], lnf_g, lnf_b, q} (kernels.cuh:41-48); GPT2ScratchGPU 7 half* + int (kernels.cuh:54)
    assert vals == [96, 88, 1208, 32, 1184, 1200, 64]
    assert vals[0] == ctypes.sizeof(G.GPT2LayerGPU) and vals[2] == ctypes.sizeof(G.GPT2WeightsGPU)


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF_DIR, "cuda")), reason="reference tree not present")
def test_header_compiles_after_the_reference_headers():
    """A reference translation unit includes its own kernels.cuh / kvcache.cuh first, then this
    header, and calls the drop-ins with the reference's own types (compile only)."""
    d = tempfile.mkdtemp()
    cu = os.path.join(d, "harness.cu")
    open(cu, "w").write(r'''
#include "kernels.cuh"
#include "kvcache.cuh"
#include "gpt2_b200.h"
void harness(const GPT2WeightsGPU *w, GPT2KVCache *kv, GPT2ScratchGPU *s, half *att, half *qkv,
             half *logits) {
    GPT2Backend b = GPT2_BACKEND_NAIVE;
    gpt2_b200_compose_backend(&b, &b);
    b.gemv = gpt2_gemv_b200;
    b.attention(att, qkv, 128, 768, 12, 64);
    gpt2_attention_kv_b200(att, qkv, kv, 0, 128, 768, 12, 64);
    gpt2_attn_decode_b200(att, qkv, kv, 0, 1);
    gpt2_decode_step_b200(&b, w, kv, 0, 0, s, logits, nullptr);
}
''')
    subprocess.run(["nvcc", "-std=c++17", "-c", "-o", os.path.join(d, "harness.o"),
                    "-I", os.path.join(REF_DIR, "cuda"), "-I", os.path.join(REF_DIR, "model"),
                    "-I", os.path.join(ROOT, "include"), cu], check=True, capture_output=True)


def test_compose_backend_the_reference_way(lib):
    base = G.GPT2Backend()
    base.name = b"gemv"
    for i, f in enumerate(("embed", "layernorm", "matmul", "attention", "gelu", "add", "matmul_q",
                           "gemv", "gemv_q")):
        setattr(base, f, 0x1000 + i)
    dst = G.GPT2Backend()
    lib.gpt2_b200_compose_backend(ctypes.byref(dst), ctypes.byref(base))
    assert dst.name == b"b200"
    attn_addr = ctypes.cast(lib.lib.gpt2_attention_b200, ctypes.c_void_p).value
    assert dst.attention == attn_addr
    assert (dst.embed, dst.matmul, dst.gemv, dst.gemv_q) == (0x1000, 0x1002, 0x1007, 0x1008)
    empty = G.GPT2Backend()
    lib.gpt2_b200_compose_backend(ctypes.byref(empty), None)
    assert empty.attention == attn_addr and empty.matmul is None


def test_kv_step_bytes_formula(lib):
    kv = G.cache_view(0, 12, 1024)
    for n in (1, 128, 512, 1023):
        assert lib.gpt2_kv_step_bytes_b200(ctypes.byref(kv), n) == 36864.0 * n


@pytest.mark.parametrize("T,E,H,D", [(4, 768, 12, 32), (4, 700, 12, 64), (-1, 768, 12, 64),
                                     (4, 768, 0, 64)])
def test_prefill_rejects_bad_shapes(lib, T, E, H, D):
    assert lib.gpt2_attention_b200_stream(16, 16, T, E, H, D, None) == G.EINVAL
    lib.gpt2_attention_b200(16, 16, T, E, H, D)
    assert lib.gpt2_b200_last_error() == G.EINVAL
    assert lib.gpt2_b200_last_error() == G.OK  # reading clears it


def test_prefill_rejects_misaligned_pointers(lib):
    assert lib.gpt2_attention_b200_stream(18, 16, 4, 768, 12, 64, None) == G.EINVAL
    assert lib.gpt2_attention_b200_stream(16, 0, 4, 768, 12, 64, None) == G.EINVAL
    assert lib.gpt2_attention_b200_batched(16, 16, 2, 4, 768, 12, 64, 13, 0, None) == G.EINVAL


def test_prefill_empty_is_a_no_op(lib):
    assert lib.gpt2_attention_b200_batched(None, None, 0, 4, 768, 12, 64, 0, 0, None) == G.OK
    assert lib.gpt2_attention_b200_batched(None, None, 3, 0, 768, 12, 64, 0, 0, None) == G.OK


def test_decode_rejects_bad_arguments(lib):
    kv = G.cache_view(0, 12, 1024)  # data == NULL
    assert lib.gpt2_attn_decode_b200_stream(16, 16, ctypes.byref(kv), 0, 5, None) == G.EINVAL
    assert lib.gpt2_attn_decode_b200_stream(16, 16, None, 0, 5, None) == G.EINVAL
    kv = G.cache_view(4096, 12, 1024)
    for L, n in ((0, 0), (0, 1025), (-1, 5), (12, 5)):
        assert lib.gpt2_attn_decode_b200_stream(16, 16, ctypes.byref(kv), L, n, None) == G.EINVAL
    bad = G.cache_view(4096, 12, 1024, head_dim=32)
    assert lib.gpt2_attn_decode_b200_stream(16, 16, ctypes.byref(bad), 0, 5, None) == G.EINVAL
    lib.gpt2_attn_decode_b200(16, 16, ctypes.byref(kv), 0, 0)
    assert lib.gpt2_b200_last_error() == G.EINVAL


def test_layer_batched_and_fixed_scratch_decode_reject_bad_arguments(lib):
    """The multi-layer, batched and no-allocation decode entry points refuse bad arguments before any
    CUDA call. Only refused cases appear here: a valid call would launch on these fake pointers."""
    kv = G.cache_view(4096, 12, 1024)
    ref = ctypes.byref(kv)
    layers = lib.gpt2_attn_decode_b200_layers
    assert layers(16, 768, 16, 2304, ref, 11, 2, None, 5, 0, None) == G.EINVAL   # layers 11..12
    assert layers(16, 769, 16, 2304, ref, 0, 2, None, 5, 0, None) == G.EINVAL    # stride % 8
    assert layers(16, 768, 16, 2304, ref, 0, 2, None, 0, 0, None) == G.EINVAL    # len 0
    assert layers(16, 768, 16, 2304, ref, 0, 2, None, 5, 1025, None) == G.EINVAL  # max_len > maxT
    assert layers(16, 768, 16, 2304, ref, 0, 2, None, 9, 8, None) == G.EINVAL    # len > max_len
    batched = lib.gpt2_attn_decode_b200_batched
    assert batched(16, 768, 16, 2304, 16, 16, 16, 0, 12, 1024, 0, None) == G.EINVAL  # B = 0
    assert batched(16, 770, 16, 2304, 16, 16, 16, 4, 12, 1024, 0, None) == G.EINVAL  # stride % 8
    assert batched(16, 768, 16, 2304, 16, 16, 16, 4, 12, 1024, 2048, None) == G.EINVAL  # max_len
    assert batched(16, 768, 16, 2304, None, 16, 16, 4, 12, 1024, 0, None) == G.EINVAL  # no slabs
    noalloc = lib.gpt2_attn_decode_b200_layers_noalloc
    assert noalloc(16, 768, 16, 2304, ref, 0, 12, 0, None) == G.EINVAL     # len 0
    assert noalloc(16, 768, 16, 2304, ref, 0, 12, 1025, None) == G.EINVAL  # len > maxT
    assert noalloc(18, 768, 16, 2304, ref, 0, 12, 5, None) == G.EINVAL     # misaligned att
    wide = G.cache_view(4096, 12, 1024, n_head=200)  # 2400 (layer, head) pairs > 2048
    assert noalloc(16, 12800, 16, 38400, ctypes.byref(wide), 0, 12, 5, None) == G.EINVAL
    long_ = G.cache_view(4096, 12, 4096)  # 144 pairs x 32 splits of 128 keys > 1985 partials
    assert noalloc(16, 768, 16, 2304, ctypes.byref(long_), 0, 12, 4096, None) == G.EINVAL


def test_prefill_with_cache_fill_rejects_a_mismatched_cache(lib):
    kv = G.cache_view(4096, 12, 64)
    ref = ctypes.byref(kv)
    fill = lib.gpt2_attention_kv_b200_stream
    assert fill(16, 16, ref, 0, 65, 768, 12, 64, None) == G.EINVAL   # T > maxT
    assert fill(16, 16, ref, 12, 8, 768, 12, 64, None) == G.EINVAL   # layer out of range
    other = G.cache_view(4096, 12, 64, n_head=6)
    assert fill(16, 16, ctypes.byref(other), 0, 8, 768, 12, 64, None) == G.EINVAL  # nHead != H
    assert fill(16, 16, None, 0, 8, 768, 12, 64, None) == G.EINVAL
    lib.gpt2_attention_kv_b200(16, 16, ref, 0, 65, 768, 12, 64)
    assert lib.gpt2_b200_last_error() == G.EINVAL


def test_step_attention_reserve_and_gemv_reject_bad_arguments(lib):
    kv = G.cache_view(4096, 12, 64)
    ref = ctypes.byref(kv)
    step = lib.gpt2_b200_decode_attn_step
    assert step(16, 768, 18, 2304, ref, None, 3, None) == G.EINVAL   # misaligned qkv
    assert step(16, 768, 16, 2301, ref, None, 3, None) == G.EINVAL   # qkv stride % 8
    assert step(16, 768, 16, 2304, ref, None, 64, None) == G.EINVAL  # pos >= maxT
    assert step(16, 765, 16, 2304, ref, None, 3, None) == G.EINVAL   # att stride % 8
    assert step(16, 768, 16, 2304, None, None, 3, None) == G.EINVAL
    for args in ((0, 12, 1024), (1, 0, 1024), (1, 12, 0)):
        assert lib.gpt2_b200_reserve(*args) == G.EINVAL
    lib.gpt2_gemv_b200(None, 16, 16, None, 768, 768)
    assert lib.gpt2_b200_last_error() == G.EINVAL


def test_model_entry_points_reject_bad_arguments(lib):
    """The decode-step and linear-layer entry points refuse bad arguments before any CUDA call."""
    w = G.GPT2WeightsGPU()  # every pointer NULL
    kvs = (G.GPT2KVCache * 2)(G.cache_view(4096, 12, 64), G.cache_view(8192, 12, 64))
    h = ctypes.c_void_p()
    assert lib.gpt2_b200_batch_create(ctypes.byref(h), ctypes.byref(w), kvs, 2) == G.EINVAL
    assert lib.gpt2_b200_batch_create(None, ctypes.byref(w), kvs, 2) == G.EINVAL
    assert lib.gpt2_b200_batch_create(ctypes.byref(h), None, kvs, 2) == G.EINVAL
    assert not h.value
    assert lib.gpt2_b200_batch_step(None, 16, 16, None, 0, None, None) == G.EINVAL
    assert lib.gpt2_b200_batch_generate(None, 16, 512, 16, 8, 16, 9, 0, None) == G.EINVAL
    assert lib.gpt2_b200_batch_launches_per_step(None, 0) == -1
    lib.gpt2_b200_batch_destroy(None)  # no-op
    # linear: unknown epilogue, output stride below N
    assert lib.gpt2_b200_linear(16, 768, 16, 768, 16, None, 4, 768, 768, 7, None) == G.EINVAL
    assert lib.gpt2_b200_linear(16, 100, 16, 768, 16, None, 4, 768, 768, 0, None) == G.EINVAL
    assert lib.gpt2_b200_linear(None, 768, 16, 768, 16, None, 4, 768, 768, 0, None) == G.EINVAL
    assert lib.gpt2_b200_linear_argmax(None, 0, 16, 768, 16, 4, 768, 768, None, None) == G.EINVAL
    # the decode-step drop-in: kv->len must equal pos (the reference's precondition)
    kv = G.cache_view(4096, 12, 64, length=3)
    lib.gpt2_decode_step_b200(None, ctypes.byref(w), ctypes.byref(kv), 1, 5, None, None, None)
    assert lib.gpt2_b200_last_error() == G.EINVAL
    lib.gpt2_decode_step_b200(None, ctypes.byref(w), ctypes.byref(kv), -1, 3, None, None, None)
    assert lib.gpt2_b200_last_error() == G.EINVAL


def test_kv_writers_reject_bad_positions(lib):
    kv = G.cache_view(4096, 12, 64)
    assert lib.gpt2_kv_append_b200_stream(ctypes.byref(kv), 0, 1, 16, 0, None, 64, None) == G.EINVAL
    assert lib.gpt2_kv_append_b200_stream(ctypes.byref(kv), 11, 2, 16, 0, None, 0, None) == G.EINVAL
    assert lib.gpt2_kv_scatter_prefill_b200_stream(ctypes.byref(kv), 0, 16, 65, None) == G.EINVAL
    lib.gpt2_kv_append_one_b200(ctypes.byref(kv), 0, 16, -1)
    assert lib.gpt2_b200_last_error() == G.EINVAL


def test_strerror_and_version(lib):
    assert lib.gpt2_b200_strerror(G.ETIMEOUT) == b"a kernel wait timed out"
    assert b"sm_100a" in lib.gpt2_b200_version()


def test_argmax_key_orders_like_an_argmax_over_fp16_logits():
    """The head's per-tile argmax keys (csrc/linear.cuh argmax_key): a larger fp16 value always wins,
    equal values go to the smaller index (first occurrence), and the index is recovered exactly.
    Checked on the host build of the same inline function over random and edge values."""
    import numpy as np
    d = tempfile.mkdtemp()
    src = os.path.join(d, "keys.cu")
    open(src, "w").write(r'''
#include <cstdio>
#include "linear.cuh"
int main() {
    float v; unsigned n;
    while (std::scanf("%f %u", &v, &n) == 2)
        std::printf("%llu %d\n", b200::lin::argmax_key(v, n), b200::lin::argmax_key_index(b200::lin::argmax_key(v, n)));
    return 0;
}
''')
    exe = os.path.join(d, "keys")
    subprocess.run(["nvcc", "-std=c++17", "-o", exe, "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(ROOT, "bare-metal-gpt2_b200", "csrc"), src], check=True,
                   capture_output=True)
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.standard_normal(400).astype(np.float16).astype(np.float32),
                           np.array([0.0, -0.0, 65504.0, -65504.0, 6e-8, -6e-8, 1.0, 1.0, -1.0, -1.0],
                                    dtype=np.float32)])
    idx = rng.permutation(50257)[:len(vals)].astype(np.uint32)
    inp = "".join(f"{v!r} {i}\n" for v, i in zip(vals.tolist(), idx.tolist()))
    out = subprocess.run([exe], input=inp, capture_output=True, text=True, check=True).stdout.split()
    keys = [int(x) for x in out[0::2]]
    back = [int(x) for x in out[1::2]]
    assert back == idx.tolist()
    # the winner of every pair is the argmax rule's winner (value first, then the lower index);
    # +0.0 and -0.0 compare by bit pattern here (+0 wins), which only matters for exact zeros
    for a in range(0, len(vals), 7):
        for b in range(len(vals)):
            va, vb = vals[a], vals[b]
            if va == vb and va == 0.0:
                continue
            want_a = va > vb or (va == vb and idx[a] < idx[b])
            if a == b:
                continue
            assert (keys[a] > keys[b]) == want_a, (va, vb, idx[a], idx[b])
