// model.cu — the GPT-2-124M decode step around the attention, for B sequences at once.
//
// The reference's step (gpt2_decode_step_cuda, cuda/kvcache.cu:233-269) decodes ONE sequence with
// 135 launches: embed; per layer LayerNorm, QKV GEMV, K/V append, attention, projection GEMV, add,
// LayerNorm, FC GEMV, GELU, projection GEMV, add; final LayerNorm; tied-head GEMV. Here one step
// serves B sequences and each layer is seven launches:
//   QKV linear   (bias; K/V appended to each sequence's cache at its position in the epilogue)
//   attention    (the batched decode kernel, one launch for all B x 12 heads)
//   projection   (bias + residual add into x)
//   LayerNorm 2
//   FC linear    (bias + GELU)
//   projection   (bias + residual add into x)
//   LayerNorm 1 of the next layer (or the final one)
// The embedding kernel also applies layer 0's LayerNorm, and the head's epilogue turns the logits
// into per-tile argmax keys that one small kernel reduces to the next token: 1 + 12 x 7 + 2 = 87
// launches per step (gpt2_b200_batch_launches_per_step reports the count). A lock-step greedy
// generator captures the whole step, token selection included, in one CUDA graph.
//
// Arithmetic follows the reference's fp16 path: activations stored in fp16, fp32 accumulation,
// LayerNorm statistics in fp32 over the fp16 row (k_layernorm, cuda/kernels_naive.cu:27-42: biased
// variance, eps 1e-5 inside the square root), embedding wte[token] + wpe[pos] summed in fp32 and
// rounded once (k_embed_one, kvcache.cu). Summation order differs (tree vs strided), so results
// agree to fp32 rounding before the fp16 store.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <new>

#include "common.cuh"
#include "linear.cuh"
#include "ptx.cuh"

namespace b200 {

int launch_decode(__half *out, long long out_stride, const __half *q, long long q_stride,
                  const __half *kbase, const __half *vbase, long long kv_stride,
                  const __half *const *k_ptrs, const __half *const *v_ptrs, const int *d_len,
                  int len_per_job, int len_add, int len, int max_len, int njobs, int H, int maxT,
                  cudaStream_t stream, bool pdl = false, bool l2_early = false);
int ensure_decode_workspace(DeviceContext *ctx, size_t floats, size_t words, cudaStream_t stream);
size_t decode_workspace_floats(int jobs, int H, int max_len, int num_sms, size_t *words);
int prepare_decode_stream();

namespace model {

constexpr int E = 768, NL = 12, NH = 12, HD = 64, F = 3072, Q = 2304, V = 50257;
constexpr int LN_THREADS = 256;  // 3 elements per thread
constexpr float LN_EPS = 1e-5f;

// Block-wide sum of one float per thread (LN_THREADS threads).
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // red may still be read from a previous call
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < LN_THREADS / 32; ++w) s += red[w];
    return s;
}

// LayerNorm of one fp16 row held as 3 floats per thread; writes fp16 out.
// This thread's 3 elements of the LayerNorm gain and bias. They are weights, which no kernel of the
// step writes, so the LayerNorm kernels load them before their grid dependency wait: only the row
// itself is then read after it.
__device__ __forceinline__ void ln_params(const __half *g, const __half *bta, float (&gv)[3], float (&bv)[3]) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const int e = threadIdx.x + i * LN_THREADS;
        gv[i] = __half2float(g[e]);
        bv[i] = __half2float(bta[e]);
    }
}

__device__ __forceinline__ void ln_row(const float (&xv)[3], __half *out, const float (&gv)[3],
                                       const float (&bv)[3], float *red) {
    const float mean = block_sum(xv[0] + xv[1] + xv[2], red) / E;
    float d2 = 0.0f;
#pragma unroll
    for (int i = 0; i < 3; ++i) d2 += (xv[i] - mean) * (xv[i] - mean);
    const float var = block_sum(d2, red) / E;
    const float inv = 1.0f / sqrtf(var + LN_EPS);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const int e = threadIdx.x + i * LN_THREADS;
        out[e] = __float2half_rn((xv[i] - mean) * inv * gv[i] + bv[i]);
    }
}

// x[b] = fp16(wte[tok[b]] + wpe[pos[b]]); ln[b] = LayerNorm(x[b]) with layer 0's ln_1.
__global__ void __launch_bounds__(LN_THREADS) k_embed_ln(__half *x, __half *ln, const __half *wte,
                                                         const __half *wpe, const __half *g,
                                                         const __half *bta, const int *tok,
                                                         const int *pos, int maxT, unsigned *status) {
    __shared__ float red[LN_THREADS / 32];
    float gv[3], bv[3];
    ln_params(g, bta, gv, bv);
    grid_dependency_wait();
    grid_launch_dependents();
    const int b = blockIdx.x;
    int t = tok[b], p = pos[b];
    if (t < 0 || t >= V || p < 0 || p >= maxT) {
        if (threadIdx.x == 0) atomicOr(status, ST_MODEL_BAD_TOKEN);
        t = min(max(t, 0), V - 1);
        p = min(max(p, 0), maxT - 1);
    }
    float xv[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const int e = threadIdx.x + i * LN_THREADS;
        const __half h = __float2half_rn(__half2float(wte[static_cast<long long>(t) * E + e]) +
                                         __half2float(wpe[static_cast<long long>(p) * E + e]));
        x[static_cast<long long>(b) * E + e] = h;
        xv[i] = __half2float(h);
    }
    ln_row(xv, ln + static_cast<long long>(b) * E, gv, bv, red);
}

__global__ void __launch_bounds__(LN_THREADS) k_layernorm(__half *ln, const __half *x,
                                                          const __half *g, const __half *bta) {
    __shared__ float red[LN_THREADS / 32];
    float gv[3], bv[3];
    ln_params(g, bta, gv, bv);
    grid_dependency_wait();
    grid_launch_dependents();
    const int b = blockIdx.x;
    float xv[3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
        xv[i] = __half2float(x[static_cast<long long>(b) * E + threadIdx.x + i * LN_THREADS]);
    ln_row(xv, ln + static_cast<long long>(b) * E, gv, bv, red);
}

// Best key of row b over the head's n_tiles tile keys (one block of 128 threads per row).
__device__ __forceinline__ unsigned long long row_best(const unsigned long long *amax, int n_tiles) {
    __shared__ unsigned long long red[4];
    const int b = blockIdx.x;
    unsigned long long k = 0;
    for (int i = threadIdx.x; i < n_tiles; i += blockDim.x)
        k = max(k, amax[static_cast<long long>(b) * n_tiles + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, k, o);
        k = max(k, other);
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = k;
    __syncthreads();
    return max(max(red[0], red[1]), max(red[2], red[3]));
}

__global__ void __launch_bounds__(128) k_argmax(int *next, const unsigned long long *amax,
                                                int n_tiles) {
    grid_dependency_wait();
    const unsigned long long k = row_best(amax, n_tiles);
    if (threadIdx.x == 0) next[blockIdx.x] = lin::argmax_key_index(k);
}

// Generation bookkeeping after a step at position pos[b]: next token = the prompt's while it lasts,
// else the argmax; record it; advance.
__global__ void __launch_bounds__(128) k_advance(int *tok, int *pos, int *out, long long out_stride,
                                                 const int *prompt, long long prompt_stride,
                                                 const int *plen, const unsigned long long *amax,
                                                 int n_tiles, int attention_only) {
    grid_dependency_wait();
    grid_launch_dependents();
    const unsigned long long k = attention_only ? 0ull : row_best(amax, n_tiles);
    if (threadIdx.x != 0) return;
    const int b = blockIdx.x;
    const int p = pos[b];
    // Prompt index clamped into the row (plen is the caller's, validated only here).
    const long long pi = min(static_cast<long long>(min(p + 1, max(plen[b] - 1, 0))), prompt_stride - 1);
    const int nxt = (p + 1 < plen[b] || attention_only) ? prompt[b * prompt_stride + pi]
                                                        : lin::argmax_key_index(k);
    out[b * out_stride + p + 1] = nxt;
    tok[b] = nxt;
    pos[b] = p + 1;
}

__global__ void k_gen_init(int *tok, int *pos, int *out, long long out_stride, const int *prompt,
                           long long prompt_stride, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int t = prompt[b * prompt_stride];
    tok[b] = t;
    pos[b] = 0;
    out[b * out_stride] = t;
}

// Kernel launch, optionally as a programmatic dependent of the previous kernel in the stream (the
// kernels above all wait for their predecessor before touching memory it writes).
template <typename... KArgs, typename... Args>
int launch(void (*kern)(KArgs...), int grid, int block, cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(block, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...) == cudaSuccess
               ? GPT2_B200_OK
               : GPT2_B200_ECUDA;
}

}  // namespace model
}  // namespace b200

using namespace b200;
using namespace b200::model;

struct gpt2_b200_batch {
    int B = 0, maxT = 0, device = 0;
    bool pdl = true;  // chain the step's kernels with programmatic dependent launch
    GPT2WeightsGPU w;
    void *arena = nullptr;  // device: activations, pointer arrays, generation state
    __half *x = nullptr, *ln = nullptr, *qkv = nullptr, *att = nullptr, *fc = nullptr;
    __half **kslab = nullptr, **vslab = nullptr;  // [NL][B]
    int *tok = nullptr, *pos = nullptr;           // generation state [B]
    unsigned long long *amax = nullptr;           // [B][head tiles]
    lin::Plan qkv_p[NL], proj_p[NL], fc_p[NL], proj2_p[NL], head_p;
    cudaGraphExec_t graph[2] = {nullptr, nullptr};  // generate step: full, attention only
    const int *g_prompt = nullptr, *g_plen = nullptr;
    int *g_out = nullptr;
    long long g_ps = 0, g_os = 0;
};

namespace {

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool weights_ok(const GPT2WeightsGPU *w) {
    if (!w || !w->wte || !w->wpe || !w->lnf_g || !w->lnf_b || !aligned16(w->wte)) return false;
    for (int L = 0; L < NL; ++L) {
        const GPT2LayerGPU &l = w->layers[L];
        if (!l.ln1_g || !l.ln1_b || !l.qkv_w || !l.qkv_b || !l.attn_proj_w || !l.attn_proj_b ||
            !l.ln2_g || !l.ln2_b || !l.fc_w || !l.fc_b || !l.proj_w || !l.proj_b)
            return false;
        if (!aligned16(l.qkv_w) || !aligned16(l.attn_proj_w) || !aligned16(l.fc_w) ||
            !aligned16(l.proj_w))
            return false;
    }
    return true;
}

// Enqueues one decode step for all B sequences (tokens/positions on the device).
int enqueue_step(gpt2_b200_batch *bt, const int *d_tok, const int *d_pos, __half *logits,
                 long long logits_stride, __half *caps, bool attention_only, cudaStream_t st) {
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_ECUDA;
    const int B = bt->B;
    const GPT2WeightsGPU &w = bt->w;
    if (!attention_only) {
        const int rc = launch(k_embed_ln, B, LN_THREADS, st, bt->pdl, bt->x, bt->ln, w.wte, w.wpe,
                              w.layers[0].ln1_g, w.layers[0].ln1_b, d_tok, d_pos, bt->maxT,
                              ctx->status);
        if (rc != GPT2_B200_OK) return rc;
        if (caps && cudaMemcpyAsync(caps + (NL + 1) * E, bt->x, E * sizeof(__half),
                                    cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return GPT2_B200_ECUDA;
    }
    for (int L = 0; L < NL; ++L) {
        int rc;
        if (!attention_only) {
            lin::Plan p = bt->qkv_p[L];
            p.p.d_pos = d_pos;
            if ((rc = lin::launch_linear(p, st)) != GPT2_B200_OK) return rc;
        }
        // The attention joins the launch chain only with few (sequence, head) pairs (one CTA per
        // pair per SM); with many pairs its small-CTA shape runs faster as an ordinary launch
        // (64 sequences: step 651 vs 663 us; 8 sequences chained: 422.5 vs 428 us). Chained, it
        // requests each sequence's older K/V rows into L2 while this layer's QKV projection runs.
        const bool attn_pdl = bt->pdl && static_cast<long long>(B) * NH < 2LL * ctx->num_sms;
        rc = launch_decode(bt->att, E, bt->qkv, Q, nullptr, nullptr, 0,
                           bt->kslab + static_cast<size_t>(L) * B,
                           bt->vslab + static_cast<size_t>(L) * B, d_pos, 1, 1, 0, bt->maxT, B, NH,
                           bt->maxT, st, attn_pdl, attn_pdl);
        if (rc != GPT2_B200_OK) return rc;
        if (attention_only) continue;
        if ((rc = lin::launch_linear(bt->proj_p[L], st)) != GPT2_B200_OK) return rc;
        if ((rc = launch(k_layernorm, B, LN_THREADS, st, bt->pdl, bt->ln, bt->x, w.layers[L].ln2_g,
                         w.layers[L].ln2_b)) != GPT2_B200_OK)
            return rc;
        if ((rc = lin::launch_linear(bt->fc_p[L], st)) != GPT2_B200_OK) return rc;
        if ((rc = lin::launch_linear(bt->proj2_p[L], st)) != GPT2_B200_OK) return rc;
        if (caps && cudaMemcpyAsync(caps + L * E, bt->x, E * sizeof(__half),
                                    cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return GPT2_B200_ECUDA;
        const __half *g = L + 1 < NL ? w.layers[L + 1].ln1_g : w.lnf_g;
        const __half *bb = L + 1 < NL ? w.layers[L + 1].ln1_b : w.lnf_b;
        if ((rc = launch(k_layernorm, B, LN_THREADS, st, bt->pdl, bt->ln, bt->x, g, bb)) !=
            GPT2_B200_OK)
            return rc;
    }
    if (attention_only) return cudaGetLastError() == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
    if (caps && cudaMemcpyAsync(caps + NL * E, bt->ln, E * sizeof(__half), cudaMemcpyDeviceToDevice,
                                st) != cudaSuccess)
        return GPT2_B200_ECUDA;
    lin::Plan hp = bt->head_p;
    hp.p.out = logits;
    hp.p.ldo = logits_stride;
    const int rc = lin::launch_linear(hp, st);
    if (rc != GPT2_B200_OK) return rc;
    return cudaGetLastError() == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}

int batch_init(gpt2_b200_batch *bt, const GPT2WeightsGPU *w, const GPT2KVCache *kvs, int B) {
    if (!weights_ok(w) || !kvs || B < 1 || B > lin::MAX_BPAD) return GPT2_B200_EINVAL;
    const int maxT = kvs[0].maxT;
    for (int b = 0; b < B; ++b) {
        const GPT2KVCache &kv = kvs[b];
        if (!kv.data || !aligned16(kv.data) || kv.nLayer != NL || kv.nHead != NH ||
            kv.headDim != HD || kv.maxT != maxT || maxT < 1)
            return GPT2_B200_EINVAL;
    }
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_EDEVICE;
    bt->B = B;
    bt->maxT = maxT;
    bt->device = ctx->device;
    bt->w = *w;
    const int head_tiles = (V + lin::BM - 1) / lin::BM;
    // One arena: activations (16-byte aligned rows), slab pointer arrays, state, argmax keys.
    auto up = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
    const size_t o_x = 0, o_ln = o_x + up(sizeof(__half) * B * E), o_qkv = o_ln + up(sizeof(__half) * B * E);
    const size_t o_att = o_qkv + up(sizeof(__half) * B * Q), o_fc = o_att + up(sizeof(__half) * B * E);
    const size_t o_ks = o_fc + up(sizeof(__half) * B * F), o_vs = o_ks + up(sizeof(void *) * NL * B);
    const size_t o_tok = o_vs + up(sizeof(void *) * NL * B), o_pos = o_tok + up(sizeof(int) * B);
    const size_t o_am = o_pos + up(sizeof(int) * B);
    const size_t total = o_am + up(sizeof(unsigned long long) * B * head_tiles);
    if (cudaMalloc(&bt->arena, total) != cudaSuccess) return GPT2_B200_ENOMEM;
    if (cudaMemset(bt->arena, 0, total) != cudaSuccess) return GPT2_B200_ECUDA;
    char *a = static_cast<char *>(bt->arena);
    bt->x = reinterpret_cast<__half *>(a + o_x);
    bt->ln = reinterpret_cast<__half *>(a + o_ln);
    bt->qkv = reinterpret_cast<__half *>(a + o_qkv);
    bt->att = reinterpret_cast<__half *>(a + o_att);
    bt->fc = reinterpret_cast<__half *>(a + o_fc);
    bt->kslab = reinterpret_cast<__half **>(a + o_ks);
    bt->vslab = reinterpret_cast<__half **>(a + o_vs);
    bt->tok = reinterpret_cast<int *>(a + o_tok);
    bt->pos = reinterpret_cast<int *>(a + o_pos);
    bt->amax = reinterpret_cast<unsigned long long *>(a + o_am);
    // Slab pointers: layer L of sequence b, K at (2L) and V at (2L+1) slabs (cuda/kvcache.cuh:61-66).
    const size_t slab = static_cast<size_t>(NH) * maxT * HD;
    __half **hk = new (std::nothrow) __half *[2 * NL * B];
    if (!hk) return GPT2_B200_ENOMEM;
    for (int L = 0; L < NL; ++L)
        for (int b = 0; b < B; ++b) {
            hk[L * B + b] = kvs[b].data + (2 * L) * slab;
            hk[NL * B + L * B + b] = kvs[b].data + (2 * L + 1) * slab;
        }
    const bool ok = cudaMemcpy(bt->kslab, hk, sizeof(void *) * NL * B, cudaMemcpyHostToDevice) ==
                        cudaSuccess &&
                    cudaMemcpy(bt->vslab, hk + NL * B, sizeof(void *) * NL * B,
                               cudaMemcpyHostToDevice) == cudaSuccess;
    delete[] hk;
    if (!ok) return GPT2_B200_ECUDA;
    const int sms = ctx->num_sms;
    for (int L = 0; L < NL; ++L) {
        const GPT2LayerGPU &l = w->layers[L];
        int rc = lin::plan_linear(&bt->qkv_p[L], lin::EPI_QKV, l.qkv_w, Q, E, bt->ln, E, B, l.qkv_b,
                                  bt->qkv, Q, 0, sms);
        if (rc) return rc;
        bt->qkv_p[L].p.k_dst = bt->kslab + static_cast<size_t>(L) * B;
        bt->qkv_p[L].p.v_dst = bt->vslab + static_cast<size_t>(L) * B;
        bt->qkv_p[L].p.maxT = maxT;
        bt->qkv_p[L].p.E = E;
        if ((rc = lin::plan_linear(&bt->proj_p[L], lin::EPI_RESID, l.attn_proj_w, E, E, bt->att, E, B,
                                   l.attn_proj_b, bt->x, E, 0, sms)))
            return rc;
        if ((rc = lin::plan_linear(&bt->fc_p[L], lin::EPI_GELU, l.fc_w, F, E, bt->ln, E, B, l.fc_b,
                                   bt->fc, F, 0, sms)))
            return rc;
        if ((rc = lin::plan_linear(&bt->proj2_p[L], lin::EPI_RESID, l.proj_w, E, F, bt->fc, F, B,
                                   l.proj_b, bt->x, E, 0, sms)))
            return rc;
    }
    int rc = lin::plan_linear(&bt->head_p, lin::EPI_HEAD, w->wte, V, E, bt->ln, E, B, nullptr,
                              nullptr, 0, 1, sms);
    if (rc) return rc;
    bt->head_p.p.amax = bt->amax;
    for (int L = 0; L < NL; ++L)
        bt->qkv_p[L].pdl = bt->proj_p[L].pdl = bt->fc_p[L].pdl = bt->proj2_p[L].pdl = bt->pdl;
    bt->head_p.pdl = bt->pdl;
    // Kernel attributes and the decode workspace for B sequences x 12 heads up to maxT keys, so
    // that a captured step makes no configuration call and never allocates.
    for (int L = 0; L < NL; ++L)
        if ((rc = lin::prepare_linear(bt->qkv_p[L])) || (rc = lin::prepare_linear(bt->proj_p[L])) ||
            (rc = lin::prepare_linear(bt->fc_p[L])) || (rc = lin::prepare_linear(bt->proj2_p[L])))
            return rc;
    if ((rc = lin::prepare_linear(bt->head_p)) || (rc = prepare_decode_stream())) return rc;
    size_t words = 0;
    const size_t floats = decode_workspace_floats(B, NH, maxT, sms, &words);
    return ensure_decode_workspace(ctx, floats, words, 0);
}

int check_device(const gpt2_b200_batch *bt) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return GPT2_B200_ECUDA;
    return dev == bt->device ? GPT2_B200_OK : GPT2_B200_EINVAL;
}

}  // namespace

extern "C" {

int gpt2_b200_batch_create(gpt2_b200_batch **out, const GPT2WeightsGPU *w, const GPT2KVCache *kvs,
                           int B) {
    if (!out) return GPT2_B200_EINVAL;
    *out = nullptr;
    gpt2_b200_batch *bt = new (std::nothrow) gpt2_b200_batch();
    if (!bt) return GPT2_B200_ENOMEM;
    const int rc = batch_init(bt, w, kvs, B);
    if (rc != GPT2_B200_OK) {
        gpt2_b200_batch_destroy(bt);
        return rc;
    }
    *out = bt;
    return GPT2_B200_OK;
}

void gpt2_b200_batch_destroy(gpt2_b200_batch *bt) {
    if (!bt) return;
    // replays queued on any stream may still be running: drain the device before releasing them
    int prev = -1;
    if (cudaGetDevice(&prev) == cudaSuccess && prev != bt->device) cudaSetDevice(bt->device);
    cudaDeviceSynchronize();
    for (cudaGraphExec_t &g : bt->graph)
        if (g) cudaGraphExecDestroy(g);
    if (bt->arena) cudaFree(bt->arena);
    if (prev >= 0 && prev != bt->device) cudaSetDevice(prev);
    delete bt;
}

int gpt2_b200_batch_step(gpt2_b200_batch *bt, const int *d_tokens, const int *d_pos,
                         gpt2_half *logits, long long logits_stride, int *d_next,
                         cudaStream_t stream) {
    if (!bt || !d_tokens || !d_pos) return GPT2_B200_EINVAL;
    if (logits && (logits_stride < V || !aligned16(logits))) return GPT2_B200_EINVAL;
    int rc = check_device(bt);
    if (rc) return rc;
    if ((rc = enqueue_step(bt, d_tokens, d_pos, logits, logits_stride, nullptr, false, stream)))
        return rc;
    if (d_next) {
        if ((rc = launch(k_argmax, bt->B, 128, stream, bt->pdl, d_next, bt->amax,
                         bt->head_p.p.n_tiles)) != GPT2_B200_OK)
            return rc;
    }
    return GPT2_B200_OK;
}

int gpt2_b200_batch_launches_per_step(const gpt2_b200_batch *bt, int flags) {
    if (!bt) return -1;
    // attention only: 12 attention launches + the bookkeeping kernel
    if (flags & GPT2_B200_GEN_ATTENTION_ONLY) return NL + 1;
    // embed+LN, 12 x (QKV, attention, proj, LN2, FC, proj2, LN), head, bookkeeping
    return 1 + NL * 7 + 1 + 1;
}

int gpt2_b200_batch_generate(gpt2_b200_batch *bt, const int *d_prompt, long long prompt_stride,
                             const int *d_plen, int n_steps, int *d_out, long long out_stride,
                             int flags, cudaStream_t stream) {
    if (!bt || !d_prompt || !d_plen || !d_out || n_steps < 1 || n_steps > bt->maxT ||
        out_stride < n_steps + 1 || prompt_stride < 1)
        return GPT2_B200_EINVAL;
    int rc = check_device(bt);
    if (rc) return rc;
    const bool attn_only = (flags & GPT2_B200_GEN_ATTENTION_ONLY) != 0;
    const int gi = attn_only ? 1 : 0;
    // The graph bakes in the generation buffers; re-capture when they change.
    if (bt->graph[gi] && (bt->g_prompt != d_prompt || bt->g_plen != d_plen || bt->g_out != d_out ||
                          bt->g_ps != prompt_stride || bt->g_os != out_stride)) {
        // earlier replays of these graphs may still be queued: let them finish first
        if (cudaDeviceSynchronize() != cudaSuccess) return GPT2_B200_ECUDA;
        for (cudaGraphExec_t &g : bt->graph)
            if (g) {
                cudaGraphExecDestroy(g);
                g = nullptr;
            }
    }
    bt->g_prompt = d_prompt;
    bt->g_plen = d_plen;
    bt->g_out = d_out;
    bt->g_ps = prompt_stride;
    bt->g_os = out_stride;
    const int head_tiles = bt->head_p.p.n_tiles;
    if (!bt->graph[gi]) {
        cudaStream_t cs;
        if (cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking) != cudaSuccess)
            return GPT2_B200_ECUDA;
        cudaGraph_t g = nullptr;
        rc = GPT2_B200_OK;
        if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            rc = GPT2_B200_ECUDA;
        } else {
            rc = enqueue_step(bt, bt->tok, bt->pos, nullptr, 0, nullptr, attn_only, cs);
            const int rc2 = launch(k_advance, bt->B, 128, cs, bt->pdl, bt->tok, bt->pos, d_out,
                                   out_stride, d_prompt, prompt_stride, d_plen, bt->amax,
                                   head_tiles, attn_only ? 1 : 0);
            if (rc == GPT2_B200_OK) rc = rc2;
            if (cudaStreamEndCapture(cs, &g) != cudaSuccess && rc == GPT2_B200_OK)
                rc = GPT2_B200_ECUDA;
        }
        if (rc == GPT2_B200_OK &&
            cudaGraphInstantiate(&bt->graph[gi], g, 0) != cudaSuccess)
            rc = GPT2_B200_ECUDA;
        if (g) cudaGraphDestroy(g);
        cudaStreamDestroy(cs);
        if (rc != GPT2_B200_OK) {
            bt->graph[gi] = nullptr;
            return rc;
        }
    }
    k_gen_init<<<(bt->B + 127) / 128, 128, 0, stream>>>(bt->tok, bt->pos, d_out, out_stride,
                                                         d_prompt, prompt_stride, bt->B);
    if (cudaGetLastError() != cudaSuccess) return GPT2_B200_ECUDA;
    for (int s = 0; s < n_steps; ++s)
        if (cudaGraphLaunch(bt->graph[gi], stream) != cudaSuccess) return GPT2_B200_ECUDA;
    return GPT2_B200_OK;
}

// ---------------------------------------------------------------- the linear layer alone
namespace {
// Per-device argmax key buffer for gpt2_b200_linear_argmax (grown on demand).
unsigned long long *g_keys[64] = {};
size_t g_keys_n[64] = {};
}  // namespace

namespace {
// Recently used plans of gpt2_b200_linear (a plan encodes two tensor maps and picks the split,
// which costs host time a per-token GEMV slot should not pay every call).
struct LinearCacheEntry {
    const void *C, *A, *W, *bias;
    long long ldc, lda;
    int B, N, K, epi, device;
    bool valid;
    lin::Plan plan;
};
constexpr int kLinearCache = 16;
thread_local LinearCacheEntry t_lin[kLinearCache];
thread_local int t_lin_next = 0;
}  // namespace

int gpt2_b200_linear(gpt2_half *C, long long ldc, const gpt2_half *A, long long lda,
                     const gpt2_half *W, const gpt2_half *bias, int B, int N, int K, int epi,
                     cudaStream_t stream) {
    if (epi < GPT2_B200_LINEAR_STORE || epi > GPT2_B200_LINEAR_RESID || !C || ldc < N)
        return GPT2_B200_EINVAL;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return GPT2_B200_ECUDA;
    for (const LinearCacheEntry &e : t_lin)
        if (e.valid && e.C == C && e.A == A && e.W == W && e.bias == bias && e.ldc == ldc &&
            e.lda == lda && e.B == B && e.N == N && e.K == K && e.epi == epi && e.device == dev)
            return lin::launch_linear(e.plan, stream);
    const int ep = epi == GPT2_B200_LINEAR_STORE ? lin::EPI_STORE
                   : epi == GPT2_B200_LINEAR_GELU ? lin::EPI_GELU
                                                  : lin::EPI_RESID;
    LinearCacheEntry &e = t_lin[t_lin_next];
    e.valid = false;
    int rc = lin::plan_linear(&e.plan, ep, W, N, K, A, lda, B, bias, C, ldc, 0, 0);
    if (rc != GPT2_B200_OK) return rc;
    e.C = C;
    e.A = A;
    e.W = W;
    e.bias = bias;
    e.ldc = ldc;
    e.lda = lda;
    e.B = B;
    e.N = N;
    e.K = K;
    e.epi = epi;
    e.device = dev;
    e.valid = true;
    t_lin_next = (t_lin_next + 1) % kLinearCache;
    return lin::launch_linear(e.plan, stream);
}

int gpt2_b200_linear_argmax(gpt2_half *logits, long long ldl, const gpt2_half *A, long long lda,
                            const gpt2_half *W, int B, int N, int K, int *d_next,
                            cudaStream_t stream) {
    if (!d_next || (logits && ldl < N)) return GPT2_B200_EINVAL;
    DeviceContext *ctx = device_context();
    if (!ctx || ctx->device < 0 || ctx->device >= 64) return GPT2_B200_ECUDA;
    lin::Plan pl;
    int rc = lin::plan_linear(&pl, lin::EPI_HEAD, W, N, K, A, lda, B, nullptr, logits, ldl, 1, 0);
    if (rc != GPT2_B200_OK) return rc;
    const size_t need = static_cast<size_t>(B) * pl.p.n_tiles;
    const int dev = ctx->device;
    if (g_keys_n[dev] < need) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone)
            return GPT2_B200_ECAPTURE;
        if (g_keys[dev] && cudaFree(g_keys[dev]) != cudaSuccess) return GPT2_B200_ECUDA;
        g_keys[dev] = nullptr;
        g_keys_n[dev] = 0;
        if (cudaMalloc(&g_keys[dev], need * sizeof(unsigned long long)) != cudaSuccess)
            return GPT2_B200_ENOMEM;
        g_keys_n[dev] = need;
    }
    pl.p.amax = g_keys[dev];
    if ((rc = lin::launch_linear(pl, stream)) != GPT2_B200_OK) return rc;
    k_argmax<<<B, 128, 0, stream>>>(d_next, pl.p.amax, pl.p.n_tiles);
    return cudaGetLastError() == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}

void gpt2_gemv_b200(gpt2_half *C, const gpt2_half *A, const gpt2_half *W, const gpt2_half *bias, int N,
                    int K) {
    b200::set_last_error(gpt2_b200_linear(C, N, A, K, W, bias, 1, N, K, GPT2_B200_LINEAR_STORE, 0));
}

// ---------------------------------------------------------------- the B = 1 drop-in
namespace {
struct StepCache {
    const void *w_data;
    const void *kv_data;
    int device;
    gpt2_b200_batch *bt;
    int *d_tp;  // token, position
};
constexpr int kStepCache = 4;
thread_local StepCache t_steps[kStepCache] = {};
thread_local int t_step_next = 0;
}  // namespace

void gpt2_decode_step_b200(const GPT2Backend *be, const GPT2WeightsGPU *w, GPT2KVCache *kv, int token,
                           int pos, GPT2ScratchGPU *s, gpt2_half *logits, gpt2_half *caps_blocks) {
    (void)be;
    (void)s;
    if (!w || !kv || !kv->data || pos < 0 || pos >= kv->maxT || kv->len != pos || token < 0 ||
        token >= V) {
        b200::set_last_error(GPT2_B200_EINVAL);
        return;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        b200::set_last_error(GPT2_B200_ECUDA);
        return;
    }
    StepCache *c = nullptr;
    for (StepCache &e : t_steps)
        if (e.bt && e.w_data == w->data && e.kv_data == kv->data && e.device == dev)
            c = &e;
    if (!c) {
        c = &t_steps[t_step_next];
        t_step_next = (t_step_next + 1) % kStepCache;
        if (c->bt) {
            gpt2_b200_batch_destroy(c->bt);
            cudaFree(c->d_tp);
            *c = StepCache{};
        }
        gpt2_b200_batch *bt = nullptr;
        int rc = gpt2_b200_batch_create(&bt, w, kv, 1);
        if (rc != GPT2_B200_OK) {
            b200::set_last_error(rc);
            return;
        }
        int *tp = nullptr;
        if (cudaMalloc(&tp, 2 * sizeof(int)) != cudaSuccess) {
            gpt2_b200_batch_destroy(bt);
            b200::set_last_error(GPT2_B200_ENOMEM);
            return;
        }
        *c = StepCache{w->data, kv->data, dev, bt, tp};
    }
    const int hv[2] = {token, pos};
    int rc = cudaMemcpyAsync(c->d_tp, hv, sizeof(hv), cudaMemcpyHostToDevice, 0) == cudaSuccess
                 ? GPT2_B200_OK
                 : GPT2_B200_ECUDA;
    if (rc == GPT2_B200_OK)
        rc = enqueue_step(c->bt, c->d_tp, c->d_tp + 1, logits, V, caps_blocks, false, 0);
    if (rc == GPT2_B200_OK) kv->len = pos + 1;
    b200::set_last_error(rc);
}

}  // extern "C"
