"""ctypes binding of libgpt2_b200.so (the C ABI declared in include/gpt2_b200.h).

This is plumbing for the tests and bench.py: it loads the in-tree shared library, declares every
entry point's signature, and offers thin helpers that pass torch tensors' device pointers. All work
happens in the CUDA kernels behind the C ABI; if the library is missing, loading raises instead of
falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "lib", "libgpt2_b200.so")
HEADER = os.path.join(ROOT, "include", "gpt2_b200.h")

OK, EINVAL, ECUDA, ENOMEM, EDEVICE, ETIMEOUT, ECAPTURE = range(7)

# Device status bits (bare-metal-gpt2_b200/csrc/common.cuh).
ST_PREFILL_LOAD_TIMEOUT = 1 << 0
ST_PREFILL_MMA_TIMEOUT = 1 << 1
ST_PREFILL_SOFTMAX_TIMEOUT = 1 << 2
ST_PREFILL_SMEM_ALIGN = 1 << 3
ST_PREFILL_DRAIN_TIMEOUT = 1 << 4
ST_DECODE_BAD_LEN = 1 << 8
ST_KV_BAD_POS = 1 << 9
ST_TEST_WAIT_TIMEOUT = 1 << 16


class GPT2KVCache(ctypes.Structure):
    """Same layout as GPT2KVCache in the reference's cuda/kvcache.cuh:39-44."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("bytes", ctypes.c_size_t),
        ("maxT", ctypes.c_int),
        ("nLayer", ctypes.c_int),
        ("nHead", ctypes.c_int),
        ("headDim", ctypes.c_int),
        ("len", ctypes.c_int),
    ]


class GPT2Backend(ctypes.Structure):
    """Same layout as GPT2Backend in the reference's cuda/kernels.cuh:68-86."""

    _fields_ = [("name", ctypes.c_char_p)] + [
        (n, ctypes.c_void_p)
        for n in ("embed", "layernorm", "matmul", "attention", "gelu", "add", "matmul_q", "gemv",
                  "gemv_q")
    ]


_vp, _ci, _cll, _cu, _cd = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_uint, ctypes.c_double
_kvp = ctypes.POINTER(GPT2KVCache)
_SIGS = {
    "gpt2_attention_b200": (None, [_vp, _vp, _ci, _ci, _ci, _ci]),
    "gpt2_attention_b200_stream": (_ci, [_vp, _vp, _ci, _ci, _ci, _ci, _vp]),
    "gpt2_attention_b200_batched": (_ci, [_vp, _vp, _ci, _ci, _ci, _ci, _ci, _cll, _cll, _vp]),
    "gpt2_attention_kv_b200": (None, [_vp, _vp, _kvp, _ci, _ci, _ci, _ci, _ci]),
    "gpt2_attention_kv_b200_stream": (_ci, [_vp, _vp, _kvp, _ci, _ci, _ci, _ci, _ci, _vp]),
    "gpt2_attn_decode_b200": (None, [_vp, _vp, _kvp, _ci, _ci]),
    "gpt2_attn_decode_b200_stream": (_ci, [_vp, _vp, _kvp, _ci, _ci, _vp]),
    "gpt2_attn_decode_b200_layers": (_ci, [_vp, _cll, _vp, _cll, _kvp, _ci, _ci, _vp, _ci, _ci, _vp]),
    "gpt2_attn_decode_b200_batched": (_ci, [_vp, _cll, _vp, _cll, _vp, _vp, _vp, _ci, _ci, _ci, _ci,
                                            _vp]),
    "gpt2_attn_decode_b200_layers_noalloc": (_ci, [_vp, _cll, _vp, _cll, _kvp, _ci, _ci, _ci, _vp]),
    "gpt2_b200_decode_attn_step": (_ci, [_vp, _cll, _vp, _cll, _kvp, _vp, _ci, _vp]),
    "gpt2_kv_alloc_b200": (_ci, [_kvp, _ci]),
    "gpt2_kv_alloc_shape_b200": (_ci, [_kvp, _ci, _ci, _ci, _ci]),
    "gpt2_kv_free_b200": (None, [_kvp]),
    "gpt2_kv_reset_b200": (None, [_kvp]),
    "gpt2_kv_step_bytes_b200": (_cd, [_kvp, _ci]),
    "gpt2_kv_append_one_b200": (None, [_kvp, _ci, _vp, _ci]),
    "gpt2_kv_append_b200_stream": (_ci, [_kvp, _ci, _ci, _vp, _cll, _vp, _ci, _vp]),
    "gpt2_kv_scatter_prefill_b200": (None, [_kvp, _ci, _vp, _ci]),
    "gpt2_kv_scatter_prefill_b200_stream": (_ci, [_kvp, _ci, _vp, _ci, _vp]),
    "gpt2_b200_compose_backend": (None, [ctypes.POINTER(GPT2Backend), ctypes.POINTER(GPT2Backend)]),
    "gpt2_b200_reserve": (_ci, [_ci, _ci, _ci]),
    "gpt2_b200_status": (_cu, [_ci]),
    "gpt2_b200_last_error": (_ci, []),
    "gpt2_b200_strerror": (ctypes.c_char_p, [_ci]),
    "gpt2_b200_selftest_wait_timeout": (_ci, [_cu]),
    "gpt2_b200_version": (ctypes.c_char_p, []),
}


def header_functions(path: str = HEADER) -> list[str]:
    """Names of every function the C header declares (for the export check)."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b(gpt2_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


class Lib:
    """The loaded library with typed entry points (attribute access = C function)."""

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(
                f"{path} is missing: build it with `make -C bare-metal-gpt2_b200` (there is no "
                "fallback implementation)")
        self.path = path
        self.lib = ctypes.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args

    def __getattr__(self, name):
        return getattr(self.lib, name)

    # -------------------------------------------------------------- checked helpers
    def check(self, rc: int, what: str) -> None:
        if rc != OK:
            raise RuntimeError(f"{what}: {self.lib.gpt2_b200_strerror(rc).decode()} ({rc})")

    def prefill(self, att, qkv, T: int, B: int = 1, stream: int = 0, qkv_stride: int = 0,
                att_stride: int = 0, E: int = 768, H: int = 12) -> None:
        rc = self.lib.gpt2_attention_b200_batched(att.data_ptr(), qkv.data_ptr(), B, T, E, H, 64,
                                                  qkv_stride, att_stride, stream)
        self.check(rc, "gpt2_attention_b200_batched")

    def decode_layers(self, att, att_stride: int, q, q_stride: int, kv: GPT2KVCache, L0: int,
                      nL: int, length: int = 0, d_len=None, max_len: int = 0,
                      stream: int = 0) -> None:
        rc = self.lib.gpt2_attn_decode_b200_layers(
            att.data_ptr(), att_stride, q.data_ptr(), q_stride, ctypes.byref(kv), L0, nL,
            d_len.data_ptr() if d_len is not None else None, length, max_len, stream)
        self.check(rc, "gpt2_attn_decode_b200_layers")

    def status(self, clear: bool = True) -> int:
        return int(self.lib.gpt2_b200_status(1 if clear else 0))


def cache_view(data_ptr: int, n_layer: int, max_t: int, n_head: int = 12, head_dim: int = 64,
               length: int = 0) -> GPT2KVCache:
    """A GPT2KVCache describing an existing device arena (e.g. a torch tensor's storage)."""
    kv = GPT2KVCache()
    kv.data = data_ptr
    kv.maxT = max_t
    kv.nLayer = n_layer
    kv.nHead = n_head
    kv.headDim = head_dim
    kv.bytes = 2 * n_layer * n_head * max_t * head_dim * 2
    kv.len = length
    return kv


_LIB: Lib | None = None


def load() -> Lib:
    global _LIB
    if _LIB is None:
        _LIB = Lib()
    return _LIB
