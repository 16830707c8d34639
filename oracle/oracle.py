"""TEST INFRASTRUCTURE ONLY — ctypes handles on the parity checkers.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs import this
module. The product library (bare-metal-gpt2_b200/) never does, and it has no CPU fallback.

Three checkers, all built by oracle/Makefile:
  * ``Oracle``      — oracle/attn_oracle.c, this repo's double-precision restatement of the reference's
                      prefill attention (cpu/forward_cpu.c:83-116) and M=1 decode attention
                      (cuda/kvcache.cu:88-129). Always available (built from this repo).
  * ``RefCPU``      — the reference's own attention() (cpu/forward_cpu.c:83-116), compiled from the
                      reference tree into oracle/_ref/libref_cpu.so. Used to pin ``Oracle`` and as the
                      timed CPU baseline.
  * ``RefGPU``      — the reference's own CUDA kernels (k_attention_flash, k_attention, k_attn_decode,
                      k_kv_append, k_kv_scatter) compiled for sm_100a into oracle/_ref/libref_gpu.so.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
REF_DIR = os.path.join(HERE, "_ref")

# GPT-2-124M attention shapes (model/config.h:11-19 of the reference).
E, H, D, QKV, N_CTX, N_LAYER = 768, 12, 64, 2304, 1024, 12

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def _fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f32p)


def _uptr(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_u16p)


class Oracle:
    """This repo's CPU restatement (oracle/attn_oracle.c)."""

    def __init__(self, path: str | None = None):
        path = path or os.path.join(BUILD_DIR, "libattn_oracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        lib = ctypes.CDLL(path)
        lib.oracle_prefill_attention.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_int, ctypes.c_long,
                                                 ctypes.c_long]
        lib.oracle_prefill_attention.restype = ctypes.c_int
        lib.oracle_decode_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.oracle_decode_attention.restype = ctypes.c_int
        lib.oracle_kv_scatter_u16.argtypes = [_u16p, _u16p, _u16p, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_long, ctypes.c_int]
        lib.oracle_kv_scatter_u16.restype = ctypes.c_int
        lib.oracle_num_threads.restype = ctypes.c_int
        self.lib = lib

    def threads(self) -> int:
        return int(self.lib.oracle_num_threads())

    def prefill(self, qkv: np.ndarray, e: int = E, h: int = H) -> np.ndarray:
        """qkv: float32 [T, >=3E] -> att float32 [T, E] (causal, scale 1/sqrt(D))."""
        qkv = np.ascontiguousarray(qkv, dtype=np.float32)
        t = qkv.shape[0]
        att = np.zeros((t, e), dtype=np.float32)
        rc = self.lib.oracle_prefill_attention(_fptr(att), _fptr(qkv), t, e, h, e // h,
                                               qkv.shape[1], e)
        if rc != 0:
            raise ValueError("oracle_prefill_attention rejected its arguments")
        return att

    def decode(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, length: int) -> np.ndarray:
        """q float32 [H*D]; k, v float32 [H, maxT, D] -> att float32 [H*D] over keys 0..length-1."""
        q = np.ascontiguousarray(q, dtype=np.float32)
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        h, max_t, d = k.shape
        att = np.zeros((h * d,), dtype=np.float32)
        rc = self.lib.oracle_decode_attention(_fptr(att), _fptr(q), _fptr(k), _fptr(v), h, max_t,
                                              d, length)
        if rc != 0:
            raise ValueError("oracle_decode_attention rejected its arguments")
        return att

    def kv_scatter(self, k: np.ndarray, v: np.ndarray, qkv_u16: np.ndarray, pos0: int = 0,
                   e: int = E, h: int = H) -> None:
        """Writes rows of qkv (uint16 words of fp16) into one layer's [H, maxT, D] K and V slabs."""
        t = qkv_u16.shape[0]
        max_t = k.shape[1]
        rc = self.lib.oracle_kv_scatter_u16(_uptr(k), _uptr(v), _uptr(qkv_u16), t, e, h, e // h,
                                            max_t, qkv_u16.shape[1], pos0)
        if rc != 0:
            raise ValueError("oracle_kv_scatter_u16 rejected its arguments")


_LAYER_NAMES = ("ln1_g", "ln1_b", "qkv_w", "qkv_b", "attn_proj_w", "attn_proj_b", "ln2_g", "ln2_b",
                "fc_w", "fc_b", "proj_w", "proj_b")


class _Layer(ctypes.Structure):
    """GPT2Layer (model/weights.h:8-15): fp32 host pointers."""
    _fields_ = [(n, ctypes.c_void_p) for n in _LAYER_NAMES]


class _Weights(ctypes.Structure):
    """GPT2Weights (model/weights.h:17-24)."""
    _fields_ = [("data", ctypes.c_void_p), ("n_floats", ctypes.c_size_t), ("wte", ctypes.c_void_p),
                ("wpe", ctypes.c_void_p), ("layers", _Layer * 12), ("lnf_g", ctypes.c_void_p),
                ("lnf_b", ctypes.c_void_p)]


class _Caps(ctypes.Structure):
    """GPT2Caps (cpu/forward_cpu.h:21-27)."""
    _fields_ = [("embed", ctypes.c_void_p), ("blocks", ctypes.c_void_p),
                ("final_ln", ctypes.c_void_p), ("logits", ctypes.c_void_p),
                ("logits_all", ctypes.c_int)]


class RefCPU:
    """The reference's own attention() (cpu/forward_cpu.c:83-116) and whole fp32 forward
    (gpt2_forward_cpu, cpu/forward_cpu.c:118), compiled from its source."""

    def __init__(self, path: str | None = None):
        path = path or os.path.join(REF_DIR, "libref_cpu.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref`")
        lib = ctypes.CDLL(path)
        lib.ref_cpu_attention.argtypes = [_f32p, _f32p, ctypes.c_int]
        lib.ref_cpu_attention.restype = ctypes.c_int
        lib.gpt2_forward_cpu.argtypes = [ctypes.POINTER(_Weights), ctypes.c_void_p, ctypes.c_int,
                                         ctypes.POINTER(_Caps)]
        lib.gpt2_forward_cpu.restype = None
        self.lib = lib

    def forward_logits(self, tensors: dict, ids) -> np.ndarray:
        """Logits [T, 50257] of the reference's fp32 forward over ids. tensors maps the names
        'wte', 'wpe', 'h{L}.{name}', 'lnf_g', 'lnf_b' to fp32 arrays of the reference's shapes."""
        keep = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in tensors.items()}
        w = _Weights()
        w.data = None
        w.n_floats = 0
        w.wte = keep["wte"].ctypes.data
        w.wpe = keep["wpe"].ctypes.data
        for L in range(12):
            for n in _LAYER_NAMES:
                setattr(w.layers[L], n, keep[f"h{L}.{n}"].ctypes.data)
        w.lnf_g = keep["lnf_g"].ctypes.data
        w.lnf_b = keep["lnf_b"].ctypes.data
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        logits = np.zeros((len(ids), keep["wte"].shape[0]), dtype=np.float32)
        caps = _Caps()
        caps.logits = logits.ctypes.data
        caps.logits_all = 1
        self.lib.gpt2_forward_cpu(ctypes.byref(w), ids.ctypes.data, len(ids), ctypes.byref(caps))
        return logits

    def prefill(self, qkv: np.ndarray) -> np.ndarray:
        qkv = np.ascontiguousarray(qkv, dtype=np.float32)
        assert qkv.shape[1] == QKV
        att = np.zeros((qkv.shape[0], E), dtype=np.float32)
        if self.lib.ref_cpu_attention(_fptr(att), _fptr(qkv), qkv.shape[0]) != 0:
            raise ValueError("ref_cpu_attention rejected T")
        return att


class RefGPU:
    """The reference's CUDA kernels (compiled for sm_100a). All pointers are device addresses."""

    def __init__(self, path: str | None = None):
        path = path or os.path.join(REF_DIR, "libref_gpu.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref`")
        lib = ctypes.CDLL(path)
        vp, ci = ctypes.c_void_p, ctypes.c_int
        for name, args in {
            "ref_gpu_attention_flash": [vp, vp, ci],
            "ref_gpu_attention_naive": [vp, vp, ci],
            "ref_gpu_attn_decode": [vp, vp, vp, ci, ci, ci],
            "ref_gpu_kv_append_one": [vp, ci, ci, vp, ci],
            "ref_gpu_kv_scatter_prefill": [vp, ci, ci, vp, ci],
            "ref_gpu_decode_step": [vp, vp, ci, ci, ci, vp, vp],
            "ref_gpu_prefill_fill_cache": [vp, vp, ci, vp, ci],
        }.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ci
        self.lib = lib

    def _ok(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what}: CUDA error {rc}")

    def attention_flash(self, att_ptr: int, qkv_ptr: int, t: int) -> None:
        self._ok(self.lib.ref_gpu_attention_flash(att_ptr, qkv_ptr, t), "ref flash attention")

    def attention_naive(self, att_ptr: int, qkv_ptr: int, t: int) -> None:
        self._ok(self.lib.ref_gpu_attention_naive(att_ptr, qkv_ptr, t), "ref naive attention")

    def attn_decode(self, att_ptr: int, qkv_ptr: int, kv_ptr: int, max_t: int, layer: int,
                    length: int) -> None:
        self._ok(self.lib.ref_gpu_attn_decode(att_ptr, qkv_ptr, kv_ptr, max_t, layer, length),
                 "ref decode attention")

    def kv_append_one(self, kv_ptr: int, max_t: int, layer: int, qkv_ptr: int, pos: int) -> None:
        self._ok(self.lib.ref_gpu_kv_append_one(kv_ptr, max_t, layer, qkv_ptr, pos), "ref append")

    def kv_scatter_prefill(self, kv_ptr: int, max_t: int, layer: int, qkv_ptr: int,
                           t: int) -> None:
        self._ok(self.lib.ref_gpu_kv_scatter_prefill(kv_ptr, max_t, layer, qkv_ptr, t),
                 "ref scatter")

    def prefill_fill_cache(self, weights_ptr: int, kv_ptr: int, max_t: int, ids_ptr: int, t: int) -> None:
        """The reference's gpt2_prefill_fill_cache for one sequence: rows 0..t-1 of every layer."""
        self._ok(self.lib.ref_gpu_prefill_fill_cache(weights_ptr, kv_ptr, max_t, ids_ptr, t),
                 "ref prefill fill cache")

    def decode_step(self, weights_ptr: int, kv_ptr: int, max_t: int, token: int, pos: int,
                    logits_ptr: int | None, caps_ptr: int | None = None) -> None:
        """The reference's gpt2_decode_step_cuda for one sequence (GEMV backend, fp16 path)."""
        self._ok(self.lib.ref_gpu_decode_step(weights_ptr, kv_ptr, max_t, token, pos, logits_ptr,
                                              caps_ptr), "ref decode step")


def seeded_qkv(seed: int, t: int, cols: int = QKV) -> np.ndarray:
    """N(0,1) fp32 values rounded through fp16 (what the GPU path stores), as float32 [t, cols]."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((t, cols), dtype=np.float32).astype(np.float16).astype(np.float32)
