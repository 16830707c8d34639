"""The drop-in at run time: the reference's OWN prefill forward (gpt2_forward_cuda through
gpt2_prefill_fill_cache, cuda/forward_cuda.cu:77-116, cuda/kvcache.cu:271-277) and decode step
(gpt2_decode_step_cuda, cuda/kvcache.cu:233-269), compiled unmodified, with this library installed
behind them: the backend composed the reference's way with gpt2_attention_b200 / gpt2_gemv_b200,
and the reference's gpt2_kv_scatter_prefill / gpt2_kv_append_one / gpt2_attn_decode bound to the
library's replacements (oracle/ref_dropin_shim.cu). The same flow with the reference's stock GEMV
backend and cache functions is the expected result.

Each case runs in a fresh process: the shim must be loaded before the reference's library so that
the reference's calls bind to it.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "bare-metal-gpt2_b200")
ORACLE = os.path.join(ROOT, "oracle")
SHIM = os.path.join(ORACLE, "_ref", "libref_dropin.so")
LOGIT_TOL = 2e-2  # two fp16 pipelines, fp32 sums in a different order (as tests/test_model_gpu.py)
CACHE_TOL = 2e-2

_CHILD = r"""
import ctypes, json, os, sys
pkg, oracle_dir, T, N, MAXT = sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), int(sys.argv[5])
shim = ctypes.CDLL(os.path.join(oracle_dir, "_ref", "libref_dropin.so"), mode=ctypes.RTLD_GLOBAL)
sys.path[:0] = [pkg, oracle_dir]
import numpy as np
import torch
import gpt2_b200 as G
vp, ci = ctypes.c_void_p, ctypes.c_int
shim.dropin_generate.argtypes = [ci, vp, vp, ci, vp, ci, ci, vp, vp, vp]
shim.dropin_generate.restype = ci
shim.dropin_interposed.restype = ci
torch.cuda.set_device(0)
w = G.ModelWeights(torch, "cuda", seed=7, hf_init=False)
torch.cuda.synchronize()
rng = np.random.default_rng(T)
ids = rng.integers(0, G.VOCAB, size=T).astype(np.int32)
nxt = rng.integers(0, G.VOCAB, size=max(N, 1)).astype(np.int32)
out = {"interposed": shim.dropin_interposed()}
res = {}
for use in (0, 1):
    logits = np.zeros((N + 1, G.VOCAB), np.float16)
    cache = np.zeros((12, 2, 12, MAXT, 64), np.float16)
    calls = (ctypes.c_longlong * 4)()
    rc = shim.dropin_generate(use, ctypes.addressof(w.struct), ids.ctypes.data, T, nxt.ctypes.data, N,
                              MAXT, logits.ctypes.data, cache.ctypes.data, calls)
    res[use] = (logits.astype(np.float64), cache.astype(np.float64))
    out[f"rc{use}"] = rc
    out[f"calls{use}"] = list(calls)
(l0, c0), (l1, c1) = res[0], res[1]
n = T + N
out["logit_err"] = [float(np.abs(l1[i] - l0[i]).max()) for i in range(N + 1)]
out["argmax_equal"] = [bool(l1[i].argmax() == l0[i].argmax()) for i in range(N + 1)]
out["margin"] = [float(np.sort(l0[i])[-1] - np.sort(l0[i])[-2]) for i in range(N + 1)]
out["cache_err"] = float(np.abs(c1[:, :, :, :n] - c0[:, :, :, :n]).max())
out["cache_tail_zero"] = bool(np.all(c1[:, :, :, n:] == 0) and np.all(c0[:, :, :, n:] == 0))
out["finite"] = bool(np.isfinite(l1).all() and np.isfinite(c1).all())
out["lib_status"] = int(G.load().status())
print(json.dumps(out))
"""


@pytest.mark.gpu
@pytest.mark.parametrize("T,N,MAXT", [(200, 6, 256), (1000, 3, 1024)])
def test_reference_forward_and_decode_step_with_the_library_installed(T, N, MAXT):
    r = subprocess.run([sys.executable, "-c", _CHILD, PKG, ORACLE, str(T), str(N), str(MAXT)],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["interposed"] == 1
    assert d["rc0"] == 0 and d["rc1"] == 0, d
    # the stock run routes nothing; the B200 run routes every call of the reference's flow: the
    # prefill's 12 layer scatters and attentions, and per decode step 12 appends and 12 attentions
    assert d["calls0"] == [0, 0, 0, 0]
    assert d["calls1"] == [12 * N, 12 * N, 12, 12], d["calls1"]
    assert d["finite"] and d["lib_status"] == 0
    assert max(d["logit_err"]) <= LOGIT_TOL, d["logit_err"]
    for eq, margin in zip(d["argmax_equal"], d["margin"]):
        assert eq or margin < 0.1  # the same greedy token unless the top two are within noise
    assert d["cache_err"] <= CACHE_TOL, d["cache_err"]
    assert d["cache_tail_zero"]  # nothing written past the filled positions


@pytest.mark.skipif(not os.path.exists(SHIM), reason="reference not built (oracle/_ref)")
def test_dropin_shim_loads_ahead_of_the_reference():
    """CPU check of the arrangement: the shim loads with the reference's library and this library
    behind it, and finds the reference's stock definitions of the three cache functions."""
    code = ("import ctypes, sys; s = ctypes.CDLL(sys.argv[1], mode=ctypes.RTLD_GLOBAL); "
            "print(s.dropin_interposed())")
    r = subprocess.run([sys.executable, "-c", code, SHIM], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == "1"
