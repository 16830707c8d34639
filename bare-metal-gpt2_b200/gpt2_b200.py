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
ST_DECODE_TIMEOUT = 1 << 10
ST_LINEAR_TIMEOUT = 1 << 11
ST_MODEL_BAD_TOKEN = 1 << 12
ST_TEST_WAIT_TIMEOUT = 1 << 16

LINEAR_STORE, LINEAR_GELU, LINEAR_RESID = 0, 1, 2
GEN_ATTENTION_ONLY = 1

# GPT-2-124M (the reference's model/config.h).
N_LAYER, N_HEAD, N_EMBD, VOCAB, N_CTX = 12, 12, 768, 50257, 1024
FFN, QKV_DIM = 4 * N_EMBD, 3 * N_EMBD
# Per-layer tensors in GPT2LayerGPU order (cuda/kernels.cuh:19-23) with their shapes.
LAYER_TENSORS = (
    ("ln1_g", (N_EMBD,)), ("ln1_b", (N_EMBD,)), ("qkv_w", (QKV_DIM, N_EMBD)), ("qkv_b", (QKV_DIM,)),
    ("attn_proj_w", (N_EMBD, N_EMBD)), ("attn_proj_b", (N_EMBD,)), ("ln2_g", (N_EMBD,)),
    ("ln2_b", (N_EMBD,)), ("fc_w", (FFN, N_EMBD)), ("fc_b", (FFN,)), ("proj_w", (N_EMBD, FFN)),
    ("proj_b", (N_EMBD,)),
)


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


class GPT2LayerGPU(ctypes.Structure):
    """Same layout as GPT2LayerGPU in the reference's cuda/kernels.cuh:19-23."""

    _fields_ = [(n, ctypes.c_void_p) for n, _ in LAYER_TENSORS]


class GPT2WeightsGPU(ctypes.Structure):
    """Same layout as GPT2WeightsGPU in the reference's cuda/kernels.cuh:41-48."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("n", ctypes.c_size_t),
        ("wte", ctypes.c_void_p),
        ("wpe", ctypes.c_void_p),
        ("layers", GPT2LayerGPU * N_LAYER),
        ("lnf_g", ctypes.c_void_p),
        ("lnf_b", ctypes.c_void_p),
        ("q", ctypes.c_void_p),
    ]


_vp, _ci, _cll, _cu, _cd = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_uint, ctypes.c_double
_kvp = ctypes.POINTER(GPT2KVCache)
_wp = ctypes.POINTER(GPT2WeightsGPU)
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
    "gpt2_decode_step_b200": (None, [_vp, _wp, _kvp, _ci, _ci, _vp, _vp, _vp]),
    "gpt2_b200_batch_create": (_ci, [ctypes.POINTER(_vp), _wp, _kvp, _ci]),
    "gpt2_b200_batch_destroy": (None, [_vp]),
    "gpt2_b200_batch_step": (_ci, [_vp, _vp, _vp, _vp, _cll, _vp, _vp]),
    "gpt2_b200_batch_generate": (_ci, [_vp, _vp, _cll, _vp, _ci, _vp, _cll, _ci, _vp]),
    "gpt2_b200_batch_launches_per_step": (_ci, [_vp, _ci]),
    "gpt2_b200_linear": (_ci, [_vp, _cll, _vp, _cll, _vp, _vp, _ci, _ci, _ci, _ci, _vp]),
    "gpt2_b200_linear_argmax": (_ci, [_vp, _cll, _vp, _cll, _vp, _ci, _ci, _ci, _vp, _vp]),
    "gpt2_gemv_b200": (None, [_vp, _vp, _vp, _vp, _ci, _ci]),
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
        """Raises RuntimeError with the library's message for any return code other than OK."""
        if rc != OK:
            raise RuntimeError(f"{what}: {self.lib.gpt2_b200_strerror(rc).decode()} ({rc})")

    def prefill(self, att, qkv, T: int, B: int = 1, stream: int = 0, qkv_stride: int = 0,
                att_stride: int = 0, E: int = 768, H: int = 12) -> None:
        """Causal prefill attention of B sequences (or layers) of T rows: att[b] from qkv[b] as the
        reference's attention slot computes it (cuda/kernels_fused.cu:145-149, one launch for all B).
        Strides are in elements, 0 for packed rows."""
        rc = self.lib.gpt2_attention_b200_batched(att.data_ptr(), qkv.data_ptr(), B, T, E, H, 64,
                                                  qkv_stride, att_stride, stream)
        self.check(rc, "gpt2_attention_b200_batched")

    def decode_layers(self, att, att_stride: int, q, q_stride: int, kv: GPT2KVCache, L0: int,
                      nL: int, length: int = 0, d_len=None, max_len: int = 0,
                      stream: int = 0) -> None:
        """M=1 decode attention of layers L0..L0+nL-1 over the first `length` cache positions (or the
        device int `d_len`), one launch: gpt2_attn_decode (cuda/kvcache.cu:207-210) for many layers."""
        rc = self.lib.gpt2_attn_decode_b200_layers(
            att.data_ptr(), att_stride, q.data_ptr(), q_stride, ctypes.byref(kv), L0, nL,
            d_len.data_ptr() if d_len is not None else None, length, max_len, stream)
        self.check(rc, "gpt2_attn_decode_b200_layers")

    def status(self, clear: bool = True) -> int:
        """The device's status word (bounded-wait timeouts and bad-input bits), cleared if asked."""
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


class ModelWeights:
    """Seeded random GPT-2-124M fp16 weights in one device buffer, described by a GPT2WeightsGPU.

    hf_init=True follows GPT-2's initialisation (linear weights and embeddings N(0, std), biases 0,
    LayerNorm gain 1 and bias 0); hf_init=False also randomises the biases and LayerNorm parameters
    so that every epilogue term is exercised (tests).
    """

    def __init__(self, torch, device, seed: int = 0, std: float = 0.02, hf_init: bool = True):
        shapes = [("wte", (VOCAB, N_EMBD)), ("wpe", (N_CTX, N_EMBD))]
        shapes += [(f"h{L}.{n}", sh) for L in range(N_LAYER) for n, sh in LAYER_TENSORS]
        shapes += [("lnf_g", (N_EMBD,)), ("lnf_b", (N_EMBD,))]
        total = sum(_numel(sh) for _, sh in shapes)
        self.buf = torch.empty(total, dtype=torch.float16, device=device)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.t = {}
        off = 0
        for name, sh in shapes:
            n = _numel(sh)
            v = self.buf[off:off + n].view(sh)
            off += n
            if name.endswith("_g"):
                v.fill_(1.0)
                if not hf_init:
                    v.add_(0.1 * torch.randn(sh, generator=gen, device=device))
            elif name.endswith("_b"):
                if hf_init:
                    v.zero_()
                else:
                    v.copy_(std * torch.randn(sh, generator=gen, device=device))
            else:
                v.copy_(std * torch.randn(sh, generator=gen, device=device))
            self.t[name] = v
        w = GPT2WeightsGPU()
        w.data = self.buf.data_ptr()
        w.n = total
        w.wte = self.t["wte"].data_ptr()
        w.wpe = self.t["wpe"].data_ptr()
        for L in range(N_LAYER):
            for n, _ in LAYER_TENSORS:
                setattr(w.layers[L], n, self.t[f"h{L}.{n}"].data_ptr())
        w.lnf_g = self.t["lnf_g"].data_ptr()
        w.lnf_b = self.t["lnf_b"].data_ptr()
        w.q = None
        self.struct = w


class DecodeBatch:
    """B sequences of GPT-2-124M decoded together (the gpt2_b200_batch_* entry points).

    caches: a torch fp16 tensor [B][12][2][12][maxT][64] (each sequence's arena in the reference
    layout) that stays alive as long as the batch. step() consumes one token per sequence at its
    position; generate() runs lock-step greedy generation (prompt tokens first) in a CUDA graph.
    """

    def __init__(self, lib: "Lib", weights: ModelWeights, caches):
        self.lib, self.weights, self.caches = lib, weights, caches
        self.B, max_t = int(caches.shape[0]), int(caches.shape[4])
        self.kvs = (GPT2KVCache * self.B)(*[cache_view(caches[b].data_ptr(), N_LAYER, max_t)
                                             for b in range(self.B)])
        self.h = ctypes.c_void_p()
        lib.check(lib.gpt2_b200_batch_create(ctypes.byref(self.h), ctypes.byref(weights.struct),
                                             self.kvs, self.B), "gpt2_b200_batch_create")

    def step(self, tokens, positions, logits=None, next_tokens=None, stream: int = 0) -> None:
        """tokens, positions: int32 device tensors [B]; logits: fp16 [B][>= VOCAB] or None;
        next_tokens: int32 [B] or None (argmax of each row)."""
        self.lib.check(self.lib.gpt2_b200_batch_step(
            self.h, tokens.data_ptr(), positions.data_ptr(),
            logits.data_ptr() if logits is not None else None,
            logits.stride(0) if logits is not None else 0,
            next_tokens.data_ptr() if next_tokens is not None else None, stream),
            "gpt2_b200_batch_step")

    def generate(self, prompt, prompt_len, n_steps: int, out, stream: int = 0) -> None:
        """prompt: int32 [B][P]; prompt_len: int32 [B] (1..P); out: int32 [B][>= n_steps+1]."""
        self.lib.check(self.lib.gpt2_b200_batch_generate(
            self.h, prompt.data_ptr(), prompt.stride(0), prompt_len.data_ptr(), n_steps,
            out.data_ptr(), out.stride(0), 0, stream), "gpt2_b200_batch_generate")

    def close(self) -> None:
        """Destroys the batch (the library synchronises the device first); safe to call twice."""
        if self.h:
            self.lib.gpt2_b200_batch_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


_LIB: Lib | None = None


def load() -> Lib:
    """The process-wide Lib; raises if lib/libgpt2_b200.so is missing (there is no fallback)."""
    global _LIB
    if _LIB is None:
        _LIB = Lib()
    return _LIB
