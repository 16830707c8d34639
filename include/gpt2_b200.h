/* gpt2_b200.h — C ABI of the B200 (sm_100a) causal self-attention library for GPT-2-124M.
 *
 * Drop-in replacements for the attention hot path of MatteoPhan926/bare-metal-gpt2:
 *   prefill : the GPT2Backend.attention slot          (cuda/kernels.cuh:73), implemented by
 *             gpt2_attention_flash in the reference   (cuda/kernels_fused.cu:145-149);
 *   decode  : gpt2_attn_decode over the KV cache      (cuda/kvcache.cuh:54, cuda/kvcache.cu:207-210);
 *   cache   : the GPT2KVCache arena, its alloc/free/reset/step-bytes helpers and the append / prefill
 *             scatter writers (cuda/kvcache.cuh:39-66, cuda/kvcache.cu:25-81,204-206).
 *
 * Conventions (same as the reference unless stated):
 *   - fp16 storage, fp32 accumulation; qkv rows are [q(E) | k(E) | v(E)], head h at h*D in each part;
 *     att rows are E wide. Causal: query i attends keys 0..i; scale 1/sqrt(D).
 *   - The cache layout is the reference's: per layer L, K at data + (2L)*H*maxT*D and V at
 *     data + (2L+1)*H*maxT*D, each [head][pos][dim] (cuda/kvcache.cuh:31-33,61-66).
 *   - All pointers are device pointers unless a parameter says "host". The caller owns every buffer.
 *   - The reference-signature entry points return void and launch on the legacy default stream, as the
 *     reference does; their argument / launch errors are kept in a per-thread "last error"
 *     (gpt2_b200_last_error). The _stream / _status variants return a GPT2_B200_* code.
 *   - Kernels never trap or spin forever: every wait is bounded, and a timeout sets a bit in a
 *     per-device status word read by gpt2_b200_status().
 *   - Shapes: D must be 64 (the reference's flash kernel has the same restriction, kernels_fused.cu:56);
 *     E = H*64; 16-byte aligned qkv / att / cache pointers.
 */
#ifndef GPT2_B200_H
#define GPT2_B200_H

#include <stddef.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
#include <cuda_fp16.h>
typedef __half gpt2_half; /* the reference's `half` */
extern "C" {
#else
typedef struct { unsigned short bits; } gpt2_half;
#endif

/* ---------------------------------------------------------------- status codes */
#define GPT2_B200_OK 0
#define GPT2_B200_EINVAL 1      /* bad argument (shape, alignment, length, null pointer) */
#define GPT2_B200_ECUDA 2       /* a CUDA runtime call failed */
#define GPT2_B200_ENOMEM 3      /* allocation refused (cache plan over budget, workspace) */
#define GPT2_B200_EDEVICE 4     /* the device is not compute capability 10.0, or the driver lacks TMA */
#define GPT2_B200_ETIMEOUT 5    /* a kernel's bounded wait expired (see gpt2_b200_status) */
#define GPT2_B200_ECAPTURE 6    /* would need to allocate while the stream is being captured */

/* ---------------------------------------------------------------- the KV cache (reference ABI)
 * Identical layout to GPT2KVCache in cuda/kvcache.cuh:39-44. If the reference's kvcache.cuh is
 * included first, its definition is used (include the reference headers before this one). */
#ifndef GPT2_KVCACHE_CUH
typedef struct GPT2KVCache {
    gpt2_half *data; /* owns the whole arena (device) */
    size_t bytes;
    int maxT, nLayer, nHead, headDim;
    int len;         /* positions currently cached [0, len) */
} GPT2KVCache;
#endif

/* ---------------------------------------------------------------- the backend table (reference ABI)
 * Identical layout to GPT2Backend in cuda/kernels.cuh:68-86 (opaque function pointers here, so this
 * header does not need the reference's weight types). */
#ifndef GPT2_KERNELS_CUH
typedef struct {
    const char *name;
    void (*embed)(void);
    void (*layernorm)(void);
    void (*matmul)(void);
    void (*attention)(gpt2_half *att, const gpt2_half *qkv, int T, int E, int H, int D);
    void (*gelu)(void);
    void (*add)(void);
    void (*matmul_q)(void);
    void (*gemv)(void);
    void (*gemv_q)(void);
} GPT2Backend;

/* fp16 device weights, identical layout to GPT2LayerGPU / GPT2WeightsGPU in cuda/kernels.cuh:19-48
 * (12 layers; every linear weight [out, in] row-major, model/weights.h:3-5). q is the reference's
 * optional INT8 attachment; it is not read here. */
typedef struct {
    gpt2_half *ln1_g, *ln1_b, *qkv_w, *qkv_b, *attn_proj_w, *attn_proj_b,
              *ln2_g, *ln2_b, *fc_w, *fc_b, *proj_w, *proj_b;
} GPT2LayerGPU;
typedef struct {
    gpt2_half *data; /* owns the whole fp16 body (device) */
    size_t n;
    gpt2_half *wte, *wpe; /* wte is also the tied output head */
    GPT2LayerGPU layers[12];
    gpt2_half *lnf_g, *lnf_b;
    const void *q;
} GPT2WeightsGPU;

/* Reusable device activation scratch, identical layout to GPT2ScratchGPU (cuda/kernels.cuh:54). */
typedef struct {
    gpt2_half *x, *ln, *qkv, *att, *ao, *fc, *ff;
    int maxT;
} GPT2ScratchGPU;
#endif

/* ================================================================ prefill attention */

/* Replaces GPT2Backend.attention / gpt2_attention_flash (cuda/kernels.cuh:73,
 * cuda/kernels_fused.cu:145-149): att[T,E] = causal softmax(q k^T / sqrt(D)) v for every head of
 * qkv[T,3E]. Same signature and semantics; runs the tcgen05/TMEM tensor-core kernel on the legacy
 * default stream. */
void gpt2_attention_b200(gpt2_half *att, const gpt2_half *qkv, int T, int E, int H, int D);

/* Stream variant of gpt2_attention_b200 (additive extension; no reference counterpart). */
int gpt2_attention_b200_stream(gpt2_half *att, const gpt2_half *qkv, int T, int E, int H, int D,
                               cudaStream_t stream);

/* Prefill attention that also fills the KV cache: the same att as gpt2_attention_b200, and rows
 * 0..T-1 of layer L of kv (K and V of every head) written exactly as gpt2_kv_scatter_prefill(kv, L,
 * qkv, T) writes them (cuda/kvcache.cu:67-81); rows >= T are left untouched and kv->len is not changed.
 * Replaces the reference's pair of calls in a prefill forward (cuda/forward_cuda.cu:97-98) with one
 * launch: the K/V tiles the attention loads anyway are stored to the cache from shared memory, so K
 * and V are read once. Requires kv->nHead == H and T <= kv->maxT. Additive extension; the reference
 * has no fused counterpart. */
void gpt2_attention_kv_b200(gpt2_half *att, const gpt2_half *qkv, const GPT2KVCache *kv, int L, int T,
                            int E, int H, int D);
int gpt2_attention_kv_b200_stream(gpt2_half *att, const gpt2_half *qkv, const GPT2KVCache *kv, int L,
                                  int T, int E, int H, int D, cudaStream_t stream);

/* Batched prefill: B independent sequences (or layers) in one launch. Sequence b reads
 * qkv + b*qkv_seq_stride and writes att + b*att_seq_stride (strides in elements; 0 = dense,
 * i.e. T*3E and T*E). Additive extension of cuda/kernels.cuh:73 for batch > 1. */
int gpt2_attention_b200_batched(gpt2_half *att, const gpt2_half *qkv, int B, int T, int E, int H,
                                int D, long long qkv_seq_stride, long long att_seq_stride,
                                cudaStream_t stream);

/* ================================================================ decode attention */

/* Replaces gpt2_attn_decode (cuda/kvcache.cuh:54, cuda/kvcache.cu:207-210): M=1 attention of the
 * step's query (the first E halves of qkv) over keys 0..len-1 of layer L of the cache; writes att[E].
 * Split-context flash-decoding with an in-kernel combine. Legacy default stream. */
void gpt2_attn_decode_b200(gpt2_half *att, const gpt2_half *qkv, const GPT2KVCache *kv, int L,
                           int len);

/* Stream variant (additive extension). */
int gpt2_attn_decode_b200_stream(gpt2_half *att, const gpt2_half *qkv, const GPT2KVCache *kv,
                                 int L, int len, cudaStream_t stream);

/* Decode attention for layers L0 .. L0+nL-1 of one cache in ONE launch. Layer l (relative) reads its
 * query at q + l*q_layer_stride and writes att + l*att_layer_stride (elements). The key count is
 * *d_len when d_len is not NULL (a device int, so a captured CUDA graph replays with a growing
 * context), else len. max_len bounds the split count (0 = kv->maxT). Additive extension. */
int gpt2_attn_decode_b200_layers(gpt2_half *att, long long att_layer_stride, const gpt2_half *q,
                                 long long q_layer_stride, const GPT2KVCache *kv, int L0, int nL,
                                 const int *d_len, int len, int max_len, cudaStream_t stream);

/* gpt2_attn_decode_b200_layers with a host length, for callers that must not have the library
 * allocate device memory (a pool allocator that owns all of HBM, a host that freezes allocations
 * after start-up, a latency-critical loop that cannot absorb a synchronising cudaMalloc). No
 * counterpart in the reference. It allocates nothing: its scratch is a fixed ~520 KiB array inside
 * the library image, one per GPU, held until the process exits. It runs k_decode_split (8 threads per
 * key row, split partials merged by the last CTA), not the regular entry point's k_decode_stream;
 * results agree within the library's parity tolerance. Limits: nL * nHead <= 2048 and
 * nL * nHead * ceil(len / 128) <= 1985 (all 12 GPT-2 layers up to 1024 keys); larger requests
 * return GPT2_B200_EINVAL before launching. The first call on a device looks up the array's device
 * address, and under CUDA's lazy module loading that is when the driver places the array in device
 * memory: make the first call on each device during initialisation, before allocations are frozen
 * and before any stream capture. Not valid after cudaDeviceReset. All calls on a device share the
 * array (its counters are cleared at the start of each call): calls that overlap on the GPU race,
 * so keep them ordered. Its status bits are reported by gpt2_b200_status(). */
int gpt2_attn_decode_b200_layers_noalloc(gpt2_half *att, long long att_layer_stride,
                                         const gpt2_half *q, long long q_layer_stride,
                                         const GPT2KVCache *kv, int L0, int nL, int len,
                                         cudaStream_t stream);

/* Decode attention for B independent sequences, one layer each, in ONE launch: sequence b attends
 * over the [H][maxT][D] K and V slabs at k_slabs[b] / v_slabs[b] (device arrays of device pointers)
 * for d_lens[b] keys (device ints), query q + b*q_stride, output att + b*att_stride. max_len bounds
 * the split count. Additive extension (batched decode over a [B] array of caches). */
int gpt2_attn_decode_b200_batched(gpt2_half *att, long long att_stride, const gpt2_half *q,
                                  long long q_stride, const gpt2_half *const *k_slabs,
                                  const gpt2_half *const *v_slabs, const int *d_lens, int B, int H,
                                  int maxT, int max_len, cudaStream_t stream);

/* The attention part of one decode step for every layer (the ordering of
 * gpt2_decode_step_cuda, cuda/kvcache.cu:249-252): append this step's K,V (from qkv rows
 * qkv + l*qkv_layer_stride) at position pos, then attend over len = pos+1 for all layers.
 * pos is *d_pos when d_pos is not NULL (graph replay), else the host value. Two launches.
 * Does not touch kv->len (the reference sets it on the host after the step, kvcache.cu:268). */
int gpt2_b200_decode_attn_step(gpt2_half *att, long long att_layer_stride, const gpt2_half *qkv,
                               long long qkv_layer_stride, GPT2KVCache *kv, const int *d_pos,
                               int pos, cudaStream_t stream);

/* ================================================================ the KV cache */

/* Replaces gpt2_kv_alloc (cuda/kvcache.cu:29-45): one arena of 2*L*H*maxT*D halves for the GPT-2-124M
 * shape (12 layers, 12 heads, D 64), refused (returns 1) when it would leave < 64 MiB free. 0 = ok. */
int gpt2_kv_alloc_b200(GPT2KVCache *kv, int maxT);
/* Same, for an explicit shape (additive extension). */
int gpt2_kv_alloc_shape_b200(GPT2KVCache *kv, int nLayer, int nHead, int headDim, int maxT);
/* Replaces gpt2_kv_free / gpt2_kv_reset / gpt2_kv_step_bytes (cuda/kvcache.cu:47-52). */
void gpt2_kv_free_b200(GPT2KVCache *kv);
void gpt2_kv_reset_b200(GPT2KVCache *kv);
double gpt2_kv_step_bytes_b200(const GPT2KVCache *kv, int len);

/* Replaces gpt2_kv_append_one (cuda/kvcache.cu:57-64,204-206): writes the K and V parts of qkv[3E]
 * into layer L at position pos, 16-byte vector stores. Legacy default stream. */
void gpt2_kv_append_one_b200(GPT2KVCache *kv, int L, const gpt2_half *qkv, int pos);
/* Append for layers L0..L0+nL-1 (rows qkv + l*qkv_layer_stride) on `stream`; position *d_pos if
 * d_pos != NULL (graph replay), else pos. Additive extension of gpt2_kv_append_one. */
int gpt2_kv_append_b200_stream(GPT2KVCache *kv, int L0, int nL, const gpt2_half *qkv,
                               long long qkv_layer_stride, const int *d_pos, int pos,
                               cudaStream_t stream);

/* Replaces gpt2_kv_scatter_prefill (cuda/kvcache.cu:67-81): rows 0..T-1 of qkv[T,3E] into layer L,
 * positions 0..T-1. Legacy default stream. */
void gpt2_kv_scatter_prefill_b200(GPT2KVCache *kv, int L, const gpt2_half *qkv, int T);
int gpt2_kv_scatter_prefill_b200_stream(GPT2KVCache *kv, int L, const gpt2_half *qkv, int T,
                                        cudaStream_t stream);

/* ================================================================ the decode step around attention
 * The reference's decode step (gpt2_decode_step_cuda, cuda/kvcache.cuh:74-76, cuda/kvcache.cu:233-269)
 * runs 135 launches per token for ONE sequence: embed, and per layer LayerNorm, QKV GEMV, K/V append,
 * attention, projection GEMV, add, LayerNorm, FC GEMV, GELU, projection GEMV, add; then the final
 * LayerNorm and the tied-head GEMV. The entry points below run the same step for B sequences at once:
 * every weight matmul is one tcgen05 pass over the weights for all B rows with bias, GELU, residual
 * add and the K/V append fused into its epilogue, the attention is the batched decode kernel above,
 * and the head's epilogue reduces the logits to per-sequence argmax keys. Four weight launches, one
 * attention launch and two LayerNorm launches per layer (87 per step with the embedding, the head and
 * the token bookkeeping). GPT-2-124M shapes only (E 768, 12 layers, 12 heads, vocabulary 50257). */

/* Drop-in for gpt2_decode_step_cuda on the fp16 path: consumes `token` at position `pos` of *kv
 * (kv->len must equal pos), appends every layer's K/V, writes logits[50257] when logits is not NULL
 * and captures the hidden states into caps_blocks when it is not NULL ((12+2)*768 halves: after
 * block L at L*768, final LayerNorm at 12*768, embedding at 13*768 — the reference's layout), then
 * sets kv->len = pos+1. be and s are accepted for signature compatibility and not used: the step's
 * activations live in a plan the library keeps per (weights, cache) pair, allocated by the first
 * call for that pair (about 10 KB plus tensor maps). Legacy default stream; errors go to
 * gpt2_b200_last_error(). */
void gpt2_decode_step_b200(const GPT2Backend *be, const GPT2WeightsGPU *w, GPT2KVCache *kv, int token,
                           int pos, GPT2ScratchGPU *s, gpt2_half *logits, gpt2_half *caps_blocks);

/* A batch of B (1..256) sequences decoded together, sequence b over the cache kvs[b] (host array of
 * B caches in the reference layout, all with the GPT-2-124M shape and the same maxT). Holds its own
 * activations, tensor maps and launch plans; the weights and caches stay owned by the caller. */
typedef struct gpt2_b200_batch gpt2_b200_batch;
int gpt2_b200_batch_create(gpt2_b200_batch **out, const GPT2WeightsGPU *w, const GPT2KVCache *kvs,
                           int B);
/* Releases the batch; synchronises its device first (replays may still be queued). */
void gpt2_b200_batch_destroy(gpt2_b200_batch *bt);

/* One decode step: sequence b consumes d_tokens[b] at position d_pos[b] (device ints), appends its
 * K/V at that position in every layer and attends over d_pos[b]+1 keys. Optional outputs: logits
 * ([B][logits_stride] halves, the fp16 logits) and d_next (B device ints: argmax of each row, the
 * first index on ties). Cache len fields are not touched. */
int gpt2_b200_batch_step(gpt2_b200_batch *bt, const int *d_tokens, const int *d_pos, gpt2_half *logits,
                         long long logits_stride, int *d_next, cudaStream_t stream);

/* Greedy generation in lock-step, one CUDA graph replay per step: at step t (0 <= t < n_steps) every
 * sequence consumes its token at position t; the token for position t+1 is d_prompt[b][t+1] while
 * t+1 < d_plen[b] (the prompt, fed one token per step) and the argmax of step t's logits after that.
 * d_out[b][0..n_steps] receives every sequence's tokens (prompt and generated; out_stride >=
 * n_steps+1). n_steps <= maxT. flags: 0, or GPT2_B200_GEN_ATTENTION_ONLY to replay only the
 * attention launches of each step (same lengths; a timing aid for the attention share). */
#define GPT2_B200_GEN_ATTENTION_ONLY 1
int gpt2_b200_batch_generate(gpt2_b200_batch *bt, const int *d_prompt, long long prompt_stride,
                             const int *d_plen, int n_steps, int *d_out, long long out_stride,
                             int flags, cudaStream_t stream);

/* The batched linear layer the step is built from (additive; the B-row counterpart of the GEMV slot
 * GPT2Backend.gemv / gpt2_gemv_fp16, cuda/kernels.cuh:94, cuda/kvcache.cu:212-214):
 * C[b, n] = epilogue(fp16(sum_k A[b, k] * W[n, k] + bias[n])) for b < B (1..256), W [N, K] row-major,
 * K a multiple of 64, bias may be NULL. epi: GPT2_B200_LINEAR_STORE writes the value, _GELU writes
 * gelu_new of it, _RESID adds it to C (the residual add). 16-byte aligned A and W, lda a multiple
 * of 8 (A's rows are read by TMA), ldc >= N. The plan of a call (tensor maps, split) is cached per
 * host thread for the last 16 argument sets, so a repeated call costs one launch. */
#define GPT2_B200_LINEAR_STORE 0
#define GPT2_B200_LINEAR_GELU 1
#define GPT2_B200_LINEAR_RESID 2
int gpt2_b200_linear(gpt2_half *C, long long ldc, const gpt2_half *A, long long lda,
                     const gpt2_half *W, const gpt2_half *bias, int B, int N, int K, int epi,
                     cudaStream_t stream);
/* The tied-head form: logits[b, n] = fp16(sum_k A[b, k] * W[n, k]) (written when logits is not NULL)
 * and d_next[b] = the first index of the row's maximum. Its per-tile argmax keys live in one buffer
 * per device (grown on demand, never inside a stream capture): calls on one device must not overlap
 * on the GPU. */
int gpt2_b200_linear_argmax(gpt2_half *logits, long long ldl, const gpt2_half *A, long long lda,
                            const gpt2_half *W, int B, int N, int K, int *d_next,
                            cudaStream_t stream);
/* Same signature and meaning as gpt2_gemv_fp16 (the GPT2Backend.gemv slot): C[1, N] = A[1, K] W^T + b,
 * legacy default stream. K must be a multiple of 64 (all GPT-2 weight matmuls). */
void gpt2_gemv_b200(gpt2_half *C, const gpt2_half *A, const gpt2_half *W, const gpt2_half *bias, int N,
                    int K);

/* Kernel launches one gpt2_b200_batch_step / one generate step makes (launch accounting). */
int gpt2_b200_batch_launches_per_step(const gpt2_b200_batch *bt, int flags);

/* ================================================================ backend, status, set-up */

/* Composes a backend the reference's way (cuda/kernels_fused.cu:157-164): copies *base and installs
 * gpt2_attention_b200 as .attention and "b200" as .name. base may be NULL (all other slots NULL). */
void gpt2_b200_compose_backend(GPT2Backend *dst, const GPT2Backend *base);

/* Reserves decode workspace on the current device for `jobs` (layer x sequence) decodes of up to
 * max_len keys, so that later calls (e.g. inside CUDA graph capture) do not allocate. */
int gpt2_b200_reserve(int jobs, int n_head, int max_len);

/* Synchronises the current device and returns the device status word (0 = healthy; bits name the
 * kernel and wait that timed out). clear != 0 resets it. */
unsigned gpt2_b200_status(int clear);

/* Last argument / launch error of a void entry point on this host thread (GPT2_B200_*); clears it. */
int gpt2_b200_last_error(void);
const char *gpt2_b200_strerror(int code);

/* Self-test of the bounded-wait path: launches one CTA that waits on an mbarrier nothing arrives on,
 * with a timeout of timeout_us microseconds. Returns GPT2_B200_ETIMEOUT when the wait expired and the
 * kernel returned cleanly (the expected result); the device context stays usable. */
int gpt2_b200_selftest_wait_timeout(unsigned timeout_us);

/* Library version string. */
const char *gpt2_b200_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif
#endif /* GPT2_B200_H */
