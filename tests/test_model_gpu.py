"""The decode step around the attention, on the GPU: the batched tcgen05 linear layers against fp64
torch math with the reference's rounding points; the batched step against the reference's own
decode step (gpt2_decode_step_cuda with its GEMV backend, cuda/kvcache.cu:233-269, compiled for
sm_100a from the reference's sources) sequence by sequence; the step's logits against the
reference's fp32 CPU forward (gpt2_forward_cpu, cpu/forward_cpu.c:118); and greedy lock-step
generation against the same step driven from the host."""
import ctypes

import numpy as np
import pytest

import gpt2_b200 as G

pytestmark = pytest.mark.gpu
V, E = G.VOCAB, G.N_EMBD


def ulp_check(got, want, scale, what, ulps=2.0, floor=1e-4):
    """|got - want| <= ulps * 2^-10 * scale + floor elementwise (fp16 has 10 fraction bits)."""
    got = got.double()
    err = (got - want).abs()
    lim = ulps * 2.0 ** -10 * scale + floor
    bad = err > lim
    assert not bool(bad.any()), (
        f"{what}: {int(bad.sum())} elements out of tolerance, worst err {float(err.max()):.3e}")


@pytest.fixture(scope="module")
def weights(cuda):
    return G.ModelWeights(cuda, "cuda", seed=7, hf_init=False)


def _gen(cuda, seed):
    g = cuda.Generator(device="cuda")
    g.manual_seed(seed)
    return g


@pytest.mark.parametrize("epi", [G.LINEAR_STORE, G.LINEAR_GELU, G.LINEAR_RESID])
@pytest.mark.parametrize("N,K", [(2304, 768), (768, 768), (3072, 768), (768, 3072), (40000, 768)])
@pytest.mark.parametrize("B", [1, 5, 16, 33, 64, 200, 256])
def test_linear_matches_fp64(cuda, lib, B, N, K, epi):
    torch = cuda
    g = _gen(torch, N * 31 + K * 7 + B)
    A = torch.randn(B, K, generator=g, device="cuda").half()
    W = (0.05 * torch.randn(N, K, generator=g, device="cuda")).half()
    bias = (0.1 * torch.randn(N, generator=g, device="cuda")).half()
    C0 = torch.randn(B, N, generator=g, device="cuda").half()
    C = C0.clone()
    rc = lib.gpt2_b200_linear(C.data_ptr(), N, A.data_ptr(), K, W.data_ptr(), bias.data_ptr(), B, N,
                              K, epi, None)
    assert rc == G.OK
    torch.cuda.synchronize()
    h = ((A.double() @ W.double().T) + bias.double()).half().double()  # k_gemv_fp16's rounding point
    if epi == G.LINEAR_STORE:
        want, scale = h, h.abs()
    elif epi == G.LINEAR_GELU:
        want = 0.5 * h * (1.0 + torch.tanh(0.7978845608028654 * (h + 0.044715 * h ** 3)))
        scale = h.abs() + want.abs()
    else:
        want = C0.double() + h
        scale = C0.double().abs() + h.abs()
    ulp_check(C, want, scale, f"linear B={B} N={N} K={K} epi={epi}")
    assert lib.status() == 0


@pytest.mark.parametrize("N,K", [(2304, 768), (768, 3072), (V, 768)])
def test_gemv_slot_matches_fp64(cuda, lib, N, K):
    """gpt2_gemv_b200 in the GPT2Backend.gemv slot's form: C[1,N] = A[1,K] W^T + bias (and
    bias NULL, as the reference's head call passes), repeated (cached plan) with new inputs."""
    torch = cuda
    g = _gen(torch, 500 + N + K)
    W = (0.05 * torch.randn(N, K, generator=g, device="cuda")).half()
    bias = (0.1 * torch.randn(N, generator=g, device="cuda")).half()
    A = torch.empty(1, K, dtype=torch.float16, device="cuda")
    C = torch.empty(1, N, dtype=torch.float16, device="cuda")
    for rep, b in enumerate((bias, None, bias)):
        A.copy_(torch.randn(1, K, generator=g, device="cuda").half())
        lib.gpt2_gemv_b200(C.data_ptr(), A.data_ptr(), W.data_ptr(),
                           b.data_ptr() if b is not None else None, N, K)
        assert lib.gpt2_b200_last_error() == G.OK
        torch.cuda.synchronize()
        want = A.double() @ W.double().T + (b.double() if b is not None else 0.0)
        want = want.half().double()
        ulp_check(C, want, want.abs(), f"gemv N={N} K={K} rep {rep}")


@pytest.mark.parametrize("B", [1, 3, 64])
def test_linear_argmax_matches_fp64_and_first_index_on_ties(cuda, lib, B):
    torch = cuda
    N, K = V, E
    g = _gen(torch, 1000 + B)
    A = torch.randn(B, K, generator=g, device="cuda").half()
    W = (0.02 * torch.randn(N, K, generator=g, device="cuda")).half()
    logits = torch.empty(B, N, dtype=torch.float16, device="cuda")
    nxt = torch.empty(B, dtype=torch.int32, device="cuda")

    def run():
        rc = lib.gpt2_b200_linear_argmax(logits.data_ptr(), N, A.data_ptr(), K, W.data_ptr(), B, N, K,
                                         nxt.data_ptr(), None)
        assert rc == G.OK
        torch.cuda.synchronize()

    run()
    want = (A.double() @ W.double().T).half().double()
    ulp_check(logits, want, want.abs(), f"head logits B={B}")
    assert torch.equal(nxt.long(), logits.float().argmax(dim=1)), "argmax of the written logits"
    # Plant exact ties: a copy of row 0's winning weight row at the last index keeps the first
    # index; a copy at index 0 moves the answer to 0.
    r = int(nxt[0])
    W[N - 1] = W[r]
    run()
    assert int(nxt[0]) == r
    if r != 0:
        W[0] = W[r]
        run()
        assert int(nxt[0]) == 0
    assert lib.status() == 0


def _caches(torch, B, max_t):
    arena = torch.zeros(B, G.N_LAYER, 2, G.N_HEAD, max_t, 64, dtype=torch.float16, device="cuda")
    kvs = (G.GPT2KVCache * B)()
    for b in range(B):
        kvs[b] = G.cache_view(arena[b].data_ptr(), G.N_LAYER, max_t)
    return arena, kvs


class Batch:
    def __init__(self, lib, weights, kvs, B):
        self.lib = lib
        self.h = ctypes.c_void_p()
        rc = lib.gpt2_b200_batch_create(ctypes.byref(self.h), ctypes.byref(weights.struct), kvs, B)
        assert rc == G.OK, rc

    def __del__(self):
        if self.h:
            self.lib.gpt2_b200_batch_destroy(self.h)


# Logit tolerance for two fp16 pipelines with fp32 accumulation in a different order (tcgen05 tiles
# and a tree LayerNorm here, per-warp GEMV sums and a strided LayerNorm in the reference): a one-ulp
# difference in an early activation propagates through 12 layers.
LOGIT_TOL = 2e-2
CACHE_TOL = 2e-2


def test_batch_step_matches_reference_step_lockstep(cuda, lib, ref_gpu, weights):
    torch = cuda
    B, T, MAXT = 3, 12, 64
    arena, kvs = _caches(torch, B, MAXT)
    ref_arena = torch.zeros_like(arena)
    bt = Batch(lib, weights, kvs, B)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, V, size=(B, T)).astype(np.int32)
    d_tok = torch.empty(B, dtype=torch.int32, device="cuda")
    d_pos = torch.empty(B, dtype=torch.int32, device="cuda")
    d_next = torch.empty(B, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, V, dtype=torch.float16, device="cuda")
    ref_logits = torch.empty(B, V, dtype=torch.float16, device="cuda")
    worst = 0.0
    for t in range(T):
        d_tok.copy_(torch.from_numpy(toks[:, t]))
        d_pos.fill_(t)
        rc = lib.gpt2_b200_batch_step(bt.h, d_tok.data_ptr(), d_pos.data_ptr(), logits.data_ptr(), V,
                                      d_next.data_ptr(), None)
        assert rc == G.OK
        for b in range(B):
            ref_gpu.decode_step(ctypes.addressof(weights.struct), ref_arena[b].data_ptr(), MAXT,
                                int(toks[b, t]), t, ref_logits[b].data_ptr())
        torch.cuda.synchronize()
        err = float((logits.float() - ref_logits.float()).abs().max())
        worst = max(worst, err)
        assert err <= LOGIT_TOL, f"step {t}: logits differ by {err:.3e}"
        assert torch.equal(d_next.long(), logits.float().argmax(dim=1))
    cerr = float((arena[:, :, :, :, :T].float() - ref_arena[:, :, :, :, :T].float()).abs().max())
    assert cerr <= CACHE_TOL, f"K/V appended to the caches differ by {cerr:.3e}"
    assert float(arena[:, :, :, :, T:].abs().max()) == 0.0, "wrote past the step positions"
    assert lib.status() == 0
    print(f"lockstep B={B}: worst logit diff {worst:.3e}, cache diff {cerr:.3e}")


def test_batch_step_with_different_positions(cuda, lib, ref_gpu, weights):
    """Each sequence at its own position: caches pre-filled by the reference's own step."""
    torch = cuda
    pos = [0, 7, 30, 63]
    B, MAXT = len(pos), 64
    arena, kvs = _caches(torch, B, MAXT)
    rng = np.random.default_rng(9)
    toks = rng.integers(0, V, size=(B, MAXT)).astype(np.int32)
    scratch = torch.empty(V, dtype=torch.float16, device="cuda")
    for b, p in enumerate(pos):
        for t in range(p):
            ref_gpu.decode_step(ctypes.addressof(weights.struct), arena[b].data_ptr(), MAXT,
                                int(toks[b, t]), t, scratch.data_ptr())
    ref_arena = arena.clone()
    ref_logits = torch.empty(B, V, dtype=torch.float16, device="cuda")
    for b, p in enumerate(pos):
        ref_gpu.decode_step(ctypes.addressof(weights.struct), ref_arena[b].data_ptr(), MAXT,
                            int(toks[b, p]), p, ref_logits[b].data_ptr())
    bt = Batch(lib, weights, kvs, B)
    d_tok = torch.tensor([int(toks[b, p]) for b, p in enumerate(pos)], dtype=torch.int32,
                         device="cuda")
    d_pos = torch.tensor(pos, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, V, dtype=torch.float16, device="cuda")
    rc = lib.gpt2_b200_batch_step(bt.h, d_tok.data_ptr(), d_pos.data_ptr(), logits.data_ptr(), V,
                                  None, None)
    assert rc == G.OK
    torch.cuda.synchronize()
    err = float((logits.float() - ref_logits.float()).abs().max())
    assert err <= LOGIT_TOL, f"logits differ by {err:.3e}"
    cerr = float((arena.float() - ref_arena.float()).abs().max())
    assert cerr <= CACHE_TOL, f"caches differ by {cerr:.3e}"
    assert lib.status() == 0


def test_batch_step_b64_matches_reference(cuda, lib, ref_gpu, weights):
    """The B=64 configuration (split-K clusters at their widest); sampled sequences vs reference."""
    torch = cuda
    B, T, MAXT = 64, 3, 16
    arena, kvs = _caches(torch, B, MAXT)
    ref_arena = torch.zeros_like(arena)
    bt = Batch(lib, weights, kvs, B)
    rng = np.random.default_rng(11)
    toks = rng.integers(0, V, size=(B, T)).astype(np.int32)
    d_tok = torch.empty(B, dtype=torch.int32, device="cuda")
    d_pos = torch.empty(B, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, V, dtype=torch.float16, device="cuda")
    ref_logits = torch.empty(V, dtype=torch.float16, device="cuda")
    sample = (0, 17, 40, 63)
    for t in range(T):
        d_tok.copy_(torch.from_numpy(toks[:, t]))
        d_pos.fill_(t)
        assert lib.gpt2_b200_batch_step(bt.h, d_tok.data_ptr(), d_pos.data_ptr(), logits.data_ptr(),
                                        V, None, None) == G.OK
        for b in sample:
            ref_gpu.decode_step(ctypes.addressof(weights.struct), ref_arena[b].data_ptr(), MAXT,
                                int(toks[b, t]), t, ref_logits.data_ptr())
            torch.cuda.synchronize()
            err = float((logits[b].float() - ref_logits.float()).abs().max())
            assert err <= LOGIT_TOL, f"step {t} seq {b}: logits differ by {err:.3e}"
    assert lib.status() == 0


@pytest.mark.parametrize("base", [500, 1000])
@pytest.mark.parametrize("B", [64, 16, 8])
def test_batch_step_long_context_b64_matches_reference(cuda, lib, ref_gpu, weights, base, B):
    """configs[4] at long context: B sequences whose caches were filled by the reference's own
    prefill forward (gpt2_prefill_fill_cache, cuda/kvcache.cu:271-277) to positions around `base`
    take one batched step; every sequence's logits and appended K/V are compared with the
    reference's own decode step (gpt2_decode_step_cuda) from the same cache, and two sequences
    also go through the single-sequence drop-in gpt2_decode_step_b200. B = 64 runs the step's
    attention in the small-CTA shape, 16 in the mid shape and 8 one CTA per (sequence, head); the
    last two as programmatic dependents that request the older K/V rows into L2 before their wait."""
    torch = cuda
    MAXT, NV = 1024, 8  # 8 distinct prompts (lengths base-4 .. base+3), each cache used B/8 times
    rng = np.random.default_rng(base)
    plen = [base - 4 + v for v in range(NV)]
    filled = torch.zeros(NV, G.N_LAYER, 2, G.N_HEAD, MAXT, 64, dtype=torch.float16, device="cuda")
    for v, n in enumerate(plen):
        ids = torch.from_numpy(rng.integers(0, V, size=n).astype(np.int32)).cuda()
        ref_gpu.prefill_fill_cache(ctypes.addressof(weights.struct), filled[v].data_ptr(), MAXT,
                                   ids.data_ptr(), n)
    arena, kvs = _caches(torch, B, MAXT)
    for b in range(B):
        arena[b].copy_(filled[b % NV])
    pos = [plen[b % NV] for b in range(B)]
    toks = rng.integers(0, V, size=B).astype(np.int32)
    bt = Batch(lib, weights, kvs, B)
    d_tok = torch.from_numpy(toks).cuda()
    d_pos = torch.tensor(pos, dtype=torch.int32, device="cuda")
    d_next = torch.empty(B, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, V, dtype=torch.float16, device="cuda")
    assert lib.gpt2_b200_batch_step(bt.h, d_tok.data_ptr(), d_pos.data_ptr(), logits.data_ptr(), V,
                                    d_next.data_ptr(), None) == G.OK
    torch.cuda.synchronize()
    assert torch.equal(d_next.long(), logits.float().argmax(dim=1))
    ref_arena = torch.empty_like(filled[0])
    ref_logits = torch.empty(V, dtype=torch.float16, device="cuda")
    worst, worst_kv = 0.0, 0.0
    for b in range(B):
        ref_arena.copy_(filled[b % NV])
        ref_gpu.decode_step(ctypes.addressof(weights.struct), ref_arena.data_ptr(), MAXT, int(toks[b]),
                            pos[b], ref_logits.data_ptr())
        torch.cuda.synchronize()
        err = float((logits[b].float() - ref_logits.float()).abs().max())
        worst = max(worst, err)
        assert err <= LOGIT_TOL, f"seq {b} at position {pos[b]}: logits differ by {err:.3e}"
        p = pos[b]
        kerr = float((arena[b, :, :, :, p].float() - ref_arena[:, :, :, p].float()).abs().max())
        worst_kv = max(worst_kv, kerr)
        assert kerr <= CACHE_TOL, f"seq {b}: K/V appended at {p} differ by {kerr:.3e}"
        # the step touched only position p
        assert torch.equal(arena[b, :, :, :, :p], filled[b % NV, :, :, :, :p])
        assert float(arena[b, :, :, :, p + 1:].abs().max()) == 0.0
    # the single-sequence drop-in from the same caches
    one = torch.empty(V, dtype=torch.float16, device="cuda")
    for b in (0, NV - 1):
        work = filled[b % NV].clone()
        kv = G.cache_view(work.data_ptr(), G.N_LAYER, MAXT, length=pos[b])
        lib.gpt2_decode_step_b200(None, ctypes.byref(weights.struct), ctypes.byref(kv), int(toks[b]),
                                  pos[b], None, one.data_ptr(), None)
        assert lib.gpt2_b200_last_error() == G.OK and kv.len == pos[b] + 1
        ref_arena.copy_(filled[b % NV])
        ref_gpu.decode_step(ctypes.addressof(weights.struct), ref_arena.data_ptr(), MAXT, int(toks[b]),
                            pos[b], ref_logits.data_ptr())
        torch.cuda.synchronize()
        err = float((one.float() - ref_logits.float()).abs().max())
        assert err <= LOGIT_TOL, f"drop-in step at {pos[b]}: logits differ by {err:.3e}"
    assert lib.status() == 0
    print(f"long context ~{base}: worst logit diff {worst:.3e}, appended K/V diff {worst_kv:.3e}")


@pytest.mark.parametrize("B", [100, 256])
def test_batch_step_large_batches_match_reference(cuda, lib, ref_gpu, weights, B):
    """Padded batches that do not split evenly over the cluster ranks (B = 100 -> 112 columns) and
    the largest batch (256); sampled sequences against the reference's own step."""
    torch = cuda
    T, MAXT = 2, 8
    arena, kvs = _caches(torch, B, MAXT)
    ref_arena = torch.zeros_like(arena)
    bt = Batch(lib, weights, kvs, B)
    rng = np.random.default_rng(B)
    toks = rng.integers(0, V, size=(B, T)).astype(np.int32)
    d_tok = torch.empty(B, dtype=torch.int32, device="cuda")
    d_pos = torch.empty(B, dtype=torch.int32, device="cuda")
    d_next = torch.empty(B, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, V, dtype=torch.float16, device="cuda")
    ref_logits = torch.empty(V, dtype=torch.float16, device="cuda")
    sample = (0, B // 3, B - 1)
    for t in range(T):
        d_tok.copy_(torch.from_numpy(toks[:, t]))
        d_pos.fill_(t)
        assert lib.gpt2_b200_batch_step(bt.h, d_tok.data_ptr(), d_pos.data_ptr(), logits.data_ptr(),
                                        V, d_next.data_ptr(), None) == G.OK
        torch.cuda.synchronize()
        assert torch.equal(d_next.long(), logits.float().argmax(dim=1))
        for b in sample:
            ref_gpu.decode_step(ctypes.addressof(weights.struct), ref_arena[b].data_ptr(), MAXT,
                                int(toks[b, t]), t, ref_logits.data_ptr())
            torch.cuda.synchronize()
            err = float((logits[b].float() - ref_logits.float()).abs().max())
            assert err <= LOGIT_TOL, f"B={B} step {t} seq {b}: logits differ by {err:.3e}"
    assert lib.status() == 0


def test_decode_step_dropin_matches_reference_with_captures(cuda, lib, ref_gpu, weights):
    torch = cuda
    MAXT, T = 32, 6
    arena, kvs = _caches(torch, 1, MAXT)
    ref_arena = torch.zeros_like(arena)
    kv = kvs[0]
    rng = np.random.default_rng(3)
    toks = rng.integers(0, V, size=T).astype(np.int32)
    logits = torch.empty(V, dtype=torch.float16, device="cuda")
    ref_logits = torch.empty(V, dtype=torch.float16, device="cuda")
    caps = torch.empty((G.N_LAYER + 2) * E, dtype=torch.float16, device="cuda")
    ref_caps = torch.empty_like(caps)
    for t in range(T):
        lib.gpt2_decode_step_b200(None, ctypes.byref(weights.struct), ctypes.byref(kv), int(toks[t]), t,
                                  None, logits.data_ptr(), caps.data_ptr())
        assert lib.gpt2_b200_last_error() == G.OK
        assert kv.len == t + 1
        ref_gpu.decode_step(ctypes.addressof(weights.struct), ref_arena[0].data_ptr(), MAXT,
                            int(toks[t]), t, ref_logits.data_ptr(), ref_caps.data_ptr())
        torch.cuda.synchronize()
        assert float((logits.float() - ref_logits.float()).abs().max()) <= LOGIT_TOL
        cap_err = (caps.float() - ref_caps.float()).abs().view(G.N_LAYER + 2, E).max(dim=1).values
        assert float(cap_err.max()) <= 5e-2, f"step {t}: captures differ {cap_err.tolist()}"
    # Wrong kv->len is refused without launching, as the reference requires len == pos on entry.
    lib.gpt2_decode_step_b200(None, ctypes.byref(weights.struct), ctypes.byref(kv), 1, 0, None, None,
                              None)
    assert lib.gpt2_b200_last_error() == G.EINVAL
    assert lib.status() == 0


def test_decode_step_logits_match_reference_cpu_forward(cuda, lib, weights):
    """Teacher-forced decode logits at positions 0..T-1 against the reference's fp32 CPU forward."""
    import oracle as O
    torch = cuda
    T, MAXT = 6, 16
    tensors = {k: v.float().cpu().numpy() for k, v in weights.t.items()}
    rng = np.random.default_rng(21)
    ids = rng.integers(0, V, size=T).astype(np.int32)
    want = O.RefCPU().forward_logits(tensors, ids)
    arena, kvs = _caches(torch, 1, MAXT)
    kv = kvs[0]
    logits = torch.empty(V, dtype=torch.float16, device="cuda")
    for t in range(T):
        lib.gpt2_decode_step_b200(None, ctypes.byref(weights.struct), ctypes.byref(kv), int(ids[t]), t,
                                  None, logits.data_ptr(), None)
        assert lib.gpt2_b200_last_error() == G.OK
        torch.cuda.synchronize()
        got = logits.float().cpu().numpy()
        err = float(np.abs(got - want[t]).max())
        assert err <= 5e-2, f"position {t}: logits differ from the fp32 forward by {err:.3e}"
        top = np.sort(want[t])[-2:]
        if top[1] - top[0] > 0.1:
            assert int(got.argmax()) == int(want[t].argmax())
    assert lib.status() == 0


def test_generate_matches_host_driven_steps(cuda, lib, weights):
    torch = cuda
    B, MAXT, N_STEPS = 4, 64, 40
    plen = np.array([1, 3, 8, 40], dtype=np.int32)
    rng = np.random.default_rng(17)
    prompt = rng.integers(0, V, size=(B, 48)).astype(np.int32)
    d_prompt = torch.from_numpy(prompt).cuda()
    d_plen = torch.from_numpy(plen).cuda()
    out = torch.full((B, N_STEPS + 1), -1, dtype=torch.int32, device="cuda")
    arena, kvs = _caches(torch, B, MAXT)
    bt = Batch(lib, weights, kvs, B)
    rc = lib.gpt2_b200_batch_generate(bt.h, d_prompt.data_ptr(), 48, d_plen.data_ptr(), N_STEPS,
                                      out.data_ptr(), N_STEPS + 1, 0, None)
    assert rc == G.OK
    torch.cuda.synchronize()
    gen = out.cpu().numpy()
    gen_arena = arena.clone()
    # The same steps driven from the host with the plain step entry point.
    arena.zero_()
    d_tok = torch.from_numpy(prompt[:, 0].copy()).cuda()
    d_pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    d_next = torch.empty(B, dtype=torch.int32, device="cuda")
    host = np.zeros((B, N_STEPS + 1), dtype=np.int32)
    host[:, 0] = prompt[:, 0]
    for t in range(N_STEPS):
        d_pos.fill_(t)
        assert lib.gpt2_b200_batch_step(bt.h, d_tok.data_ptr(), d_pos.data_ptr(), None, 0,
                                        d_next.data_ptr(), None) == G.OK
        nxt = d_next.cpu().numpy()
        for b in range(B):
            host[b, t + 1] = prompt[b, t + 1] if t + 1 < plen[b] else nxt[b]
        d_tok.copy_(torch.from_numpy(host[:, t + 1].copy()))
    assert np.array_equal(gen, host), "graph-driven generation differs from host-driven steps"
    for b in range(B):
        assert np.array_equal(gen[b, :plen[b]], prompt[b, :plen[b]])
    assert torch.equal(gen_arena, arena), "caches differ between the two drives"
    # Replaying (graph already built) gives the same tokens; attention-only replay runs clean.
    out2 = torch.full_like(out, -1)
    assert lib.gpt2_b200_batch_generate(bt.h, d_prompt.data_ptr(), 48, d_plen.data_ptr(), N_STEPS,
                                        out2.data_ptr(), N_STEPS + 1, 0, None) == G.OK
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    assert lib.gpt2_b200_batch_generate(bt.h, d_prompt.data_ptr(), 48, d_plen.data_ptr(), N_STEPS,
                                        out2.data_ptr(), N_STEPS + 1, G.GEN_ATTENTION_ONLY,
                                        None) == G.OK
    torch.cuda.synchronize()
    assert lib.status() == 0


def test_decode_batch_wrapper_generates_like_the_steps(cuda, lib, weights):
    """The Python DecodeBatch wrapper: generate() equals step() driven from the host."""
    torch = cuda
    B, MAXT, N_STEPS = 3, 32, 10
    caches = torch.zeros(B, G.N_LAYER, 2, G.N_HEAD, MAXT, 64, dtype=torch.float16, device="cuda")
    batch = G.DecodeBatch(lib, weights, caches)
    prompt = torch.randint(0, V, (B, 8), dtype=torch.int32, device="cuda")
    plen = torch.tensor([1, 4, 8], dtype=torch.int32, device="cuda")
    out = torch.empty(B, N_STEPS + 1, dtype=torch.int32, device="cuda")
    batch.generate(prompt, plen, N_STEPS, out)
    torch.cuda.synchronize()
    caches.zero_()
    tok = prompt[:, 0].clone()
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    nxt = torch.empty(B, dtype=torch.int32, device="cuda")
    want = [prompt[:, 0].cpu().tolist()]
    for t in range(N_STEPS):
        pos.fill_(t)
        batch.step(tok, pos, next_tokens=nxt)
        row = [int(prompt[b, t + 1]) if t + 1 < int(plen[b]) else int(nxt[b]) for b in range(B)]
        want.append(row)
        tok.copy_(torch.tensor(row, dtype=torch.int32))
    assert out.cpu().t().tolist() == want
    batch.close()
    assert lib.status() == 0


def test_batch_rejects_bad_arguments(cuda, lib, weights):
    torch = cuda
    arena, kvs = _caches(torch, 2, 32)
    h = ctypes.c_void_p()
    assert lib.gpt2_b200_batch_create(ctypes.byref(h), ctypes.byref(weights.struct), kvs, 0) == G.EINVAL
    assert lib.gpt2_b200_batch_create(ctypes.byref(h), ctypes.byref(weights.struct), kvs, 257) == G.EINVAL
    bad = (G.GPT2KVCache * 2)(kvs[0], G.cache_view(arena[1].data_ptr(), G.N_LAYER, 16))
    assert lib.gpt2_b200_batch_create(ctypes.byref(h), ctypes.byref(weights.struct), bad, 2) == G.EINVAL
    bt = Batch(lib, weights, kvs, 2)
    out = torch.empty(2, 40, dtype=torch.int32, device="cuda")
    pr = torch.zeros(2, 8, dtype=torch.int32, device="cuda")
    pl = torch.ones(2, dtype=torch.int32, device="cuda")
    # more steps than the cache holds
    assert lib.gpt2_b200_batch_generate(bt.h, pr.data_ptr(), 8, pl.data_ptr(), 33, out.data_ptr(), 40,
                                        0, None) == G.EINVAL
    # an out-of-range token id is clamped and flagged in the status word, not read out of bounds
    d_tok = torch.tensor([V + 5, 0], dtype=torch.int32, device="cuda")
    d_pos = torch.zeros(2, dtype=torch.int32, device="cuda")
    assert lib.gpt2_b200_batch_step(bt.h, d_tok.data_ptr(), d_pos.data_ptr(), None, 0, None,
                                    None) == G.OK
    st = lib.status(clear=True)
    assert st & G.ST_MODEL_BAD_TOKEN
    assert lib.status() == 0
