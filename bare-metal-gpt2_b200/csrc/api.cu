// api.cu — the C ABI (include/gpt2_b200.h): argument checks, per-device context, status word.
//
// Error behaviour: the reference's launchers return void and report nothing (cuda/kernels.cuh:73,
// cuda/kvcache.cuh:54); its harnesses find errors later through CUDA_CHECK(cudaGetLastError())
// (cuda/common.cuh:36). The void entry points here keep that signature, never launch on bad
// arguments, and leave a GPT2_B200_* code in a per-thread last-error slot. The _stream variants
// return the code directly.
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "ptx.cuh"

namespace b200 {

int launch_prefill(__half *att, const __half *qkv, int B, int T, int E, int H,
                   long long qkv_seq_stride, long long att_seq_stride, __half *kv_layer, int kv_maxT,
                   cudaStream_t stream);
int launch_decode(__half *out, long long out_stride, const __half *q, long long q_stride,
                  const __half *kbase, const __half *vbase, long long kv_stride,
                  const __half *const *k_ptrs, const __half *const *v_ptrs, const int *d_len,
                  int len_per_job, int len_add, int len, int max_len, int njobs, int H, int maxT,
                  cudaStream_t stream, bool pdl = false, bool l2_early = false);
int ensure_decode_workspace(DeviceContext *ctx, size_t floats, size_t words, cudaStream_t stream);
size_t decode_workspace_floats(int jobs, int H, int max_len, int num_sms, size_t *words);
int kv_alloc(GPT2KVCache *kv, int nLayer, int nHead, int headDim, int maxT);
int launch_kv_append(GPT2KVCache *kv, int L0, int nL, const __half *qkv, long long qkv_stride,
                     const int *d_pos, int pos, cudaStream_t stream);
int launch_kv_scatter(GPT2KVCache *kv, int L, const __half *qkv, int T, cudaStream_t stream);
unsigned noalloc_status(bool clear);

namespace {
constexpr int kMaxDevices = 64;
DeviceContext g_ctx[kMaxDevices];
bool g_ctx_ready[kMaxDevices] = {};
int g_ctx_err[kMaxDevices] = {};
std::mutex g_mu;
thread_local int t_last_error = GPT2_B200_OK;

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

EncodeTiledFn tensor_map_encoder() {
    // function-local static: initialised once, thread-safe
    static const EncodeTiledFn fn = [] {
        RelaxedCapture relaxed;  // a first call may come while this thread captures a graph
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(ptr);
        return static_cast<EncodeTiledFn>(nullptr);
    }();
    return fn;
}

DeviceContext *device_context() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    // A context never changes once created, so each host thread keeps its pointer (no lock).
    thread_local DeviceContext *t_ctx[kMaxDevices] = {};
    if (t_ctx[dev]) return t_ctx[dev];
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_ctx_ready[dev]) return t_ctx[dev] = &g_ctx[dev];
    if (g_ctx_err[dev]) return nullptr;
    cudaDeviceProp prop;
    // The library is built for sm_100a only: arch-specific code runs on compute capability 10.0
    // alone (not 10.3 and the like), so any other part fails here rather than at its first launch.
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess || prop.major != 10 || prop.minor != 0) {
        g_ctx_err[dev] = GPT2_B200_EDEVICE;
        return nullptr;
    }
    DeviceContext &c = g_ctx[dev];
    c.num_sms = prop.multiProcessorCount;
    c.device = dev;
    // The first call of a process may be made while its thread captures a CUDA graph: the status word
    // is allocated and zeroed on a private stream, which neither joins nor waits on a captured one.
    RelaxedCapture relaxed;
    cudaStream_t init = nullptr;
    bool ok = cudaStreamCreateWithFlags(&init, cudaStreamNonBlocking) == cudaSuccess &&
              cudaMalloc(&c.status, sizeof(unsigned)) == cudaSuccess &&
              cudaMemsetAsync(c.status, 0, sizeof(unsigned), init) == cudaSuccess &&
              cudaStreamSynchronize(init) == cudaSuccess;
    if (init) ok = cudaStreamDestroy(init) == cudaSuccess && ok;
    if (!ok) {
        g_ctx_err[dev] = GPT2_B200_ECUDA;
        return nullptr;
    }
    g_ctx_ready[dev] = true;
    return t_ctx[dev] = &c;
}

unsigned long long wait_timeout_ns() {
    static unsigned long long v = [] {
        const char *s = std::getenv("GPT2_B200_WAIT_TIMEOUT_MS");
        if (s && *s) {
            const long long ms = std::atoll(s);
            if (ms > 0) return static_cast<unsigned long long>(ms) * 1000000ull;
        }
        return kDefaultWaitTimeoutNs;
    }();
    return v;
}

void set_last_error(int code) { t_last_error = code; }

// ------------------------------------------------------------------ argument checks
static int check_prefill(const void *att, const void *qkv, int B, int T, int E, int H, int D,
                         long long qkv_seq_stride, long long att_seq_stride) {
    if (B < 0 || T < 0 || H < 1 || D != 64 || E != H * D) return GPT2_B200_EINVAL;
    if (B == 0 || T == 0) return GPT2_B200_OK;
    if (!att || !qkv || !aligned16(att) || !aligned16(qkv)) return GPT2_B200_EINVAL;
    if (qkv_seq_stride < 0 || att_seq_stride < 0 || (qkv_seq_stride & 7) || (att_seq_stride & 7))
        return GPT2_B200_EINVAL;
    return GPT2_B200_OK;
}

static int check_cache(const GPT2KVCache *kv) {
    if (!kv || !kv->data || !aligned16(kv->data) || kv->headDim != 64 || kv->nHead < 1 ||
        kv->nLayer < 1 || kv->maxT < 1)
        return GPT2_B200_EINVAL;
    return GPT2_B200_OK;
}

}  // namespace b200

using namespace b200;

extern "C" {

// ================================================================ prefill
int gpt2_attention_b200_batched(gpt2_half *att, const gpt2_half *qkv, int B, int T, int E, int H,
                                int D, long long qkv_seq_stride, long long att_seq_stride,
                                cudaStream_t stream) {
    int rc = check_prefill(att, qkv, B, T, E, H, D, qkv_seq_stride, att_seq_stride);
    if (rc != GPT2_B200_OK || B == 0 || T == 0) return rc;
    if (qkv_seq_stride == 0) qkv_seq_stride = static_cast<long long>(T) * 3 * E;
    if (att_seq_stride == 0) att_seq_stride = static_cast<long long>(T) * E;
    return launch_prefill(att, qkv, B, T, E, H, qkv_seq_stride, att_seq_stride, nullptr, 0, stream);
}

int gpt2_attention_b200_stream(gpt2_half *att, const gpt2_half *qkv, int T, int E, int H, int D,
                               cudaStream_t stream) {
    return gpt2_attention_b200_batched(att, qkv, 1, T, E, H, D, 0, 0, stream);
}

void gpt2_attention_b200(gpt2_half *att, const gpt2_half *qkv, int T, int E, int H, int D) {
    set_last_error(gpt2_attention_b200_batched(att, qkv, 1, T, E, H, D, 0, 0, 0));
}

int gpt2_attention_kv_b200_stream(gpt2_half *att, const gpt2_half *qkv, const GPT2KVCache *kv, int L,
                                  int T, int E, int H, int D, cudaStream_t stream) {
    int rc = check_prefill(att, qkv, 1, T, E, H, D, 0, 0);
    if (rc != GPT2_B200_OK) return rc;
    if (check_cache(kv) != GPT2_B200_OK || L < 0 || L >= kv->nLayer || kv->nHead != H || T > kv->maxT)
        return GPT2_B200_EINVAL;
    if (T == 0) return GPT2_B200_OK;
    __half *layer = reinterpret_cast<__half *>(kv->data) + static_cast<size_t>(2 * L) * H * kv->maxT * D;
    return launch_prefill(att, qkv, 1, T, E, H, static_cast<long long>(T) * 3 * E,
                          static_cast<long long>(T) * E, layer, kv->maxT, stream);
}

void gpt2_attention_kv_b200(gpt2_half *att, const gpt2_half *qkv, const GPT2KVCache *kv, int L, int T,
                            int E, int H, int D) {
    set_last_error(gpt2_attention_kv_b200_stream(att, qkv, kv, L, T, E, H, D, 0));
}

// ================================================================ decode
int gpt2_attn_decode_b200_layers(gpt2_half *att, long long att_layer_stride, const gpt2_half *q,
                                 long long q_layer_stride, const GPT2KVCache *kv, int L0, int nL,
                                 const int *d_len, int len, int max_len, cudaStream_t stream) {
    if (check_cache(kv) != GPT2_B200_OK) return GPT2_B200_EINVAL;
    if (nL < 1 || L0 < 0 || L0 + nL > kv->nLayer || !att || !q || !aligned16(att) || !aligned16(q))
        return GPT2_B200_EINVAL;
    if ((nL > 1) && ((att_layer_stride & 7) || (q_layer_stride & 7))) return GPT2_B200_EINVAL;
    if (max_len == 0) max_len = d_len ? kv->maxT : len;
    if (max_len < 1 || max_len > kv->maxT) return GPT2_B200_EINVAL;
    if (!d_len && (len < 1 || len > max_len)) return GPT2_B200_EINVAL;
    const long long slab = static_cast<long long>(kv->nHead) * kv->maxT * kv->headDim;
    const __half *kb = kv->data + 2LL * L0 * slab;
    return launch_decode(att, att_layer_stride, q, q_layer_stride, kb, kb + slab, 2 * slab, nullptr,
                         nullptr, d_len, 0, 0, len, max_len, nL, kv->nHead, kv->maxT, stream);
}

int gpt2_attn_decode_b200_stream(gpt2_half *att, const gpt2_half *qkv, const GPT2KVCache *kv,
                                 int L, int len, cudaStream_t stream) {
    if (check_cache(kv) != GPT2_B200_OK || len < 1 || len > kv->maxT) return GPT2_B200_EINVAL;
    return gpt2_attn_decode_b200_layers(att, 0, qkv, 0, kv, L, 1, nullptr, len, len, stream);
}

void gpt2_attn_decode_b200(gpt2_half *att, const gpt2_half *qkv, const GPT2KVCache *kv, int L,
                           int len) {
    set_last_error(gpt2_attn_decode_b200_stream(att, qkv, kv, L, len, 0));
}

int gpt2_attn_decode_b200_batched(gpt2_half *att, long long att_stride, const gpt2_half *q,
                                  long long q_stride, const gpt2_half *const *k_slabs,
                                  const gpt2_half *const *v_slabs, const int *d_lens, int B, int H,
                                  int maxT, int max_len, cudaStream_t stream) {
    if (B < 1 || H < 1 || maxT < 1 || !att || !q || !k_slabs || !v_slabs || !d_lens)
        return GPT2_B200_EINVAL;
    if (!aligned16(att) || !aligned16(q) || (att_stride & 7) || (q_stride & 7))
        return GPT2_B200_EINVAL;
    if (max_len == 0) max_len = maxT;
    if (max_len < 1 || max_len > maxT) return GPT2_B200_EINVAL;
    return launch_decode(att, att_stride, q, q_stride, nullptr, nullptr, 0, k_slabs, v_slabs,
                         d_lens, 1, 0, 0, max_len, B, H, maxT, stream);
}

int gpt2_b200_decode_attn_step(gpt2_half *att, long long att_layer_stride, const gpt2_half *qkv,
                               long long qkv_layer_stride, GPT2KVCache *kv, const int *d_pos,
                               int pos, cudaStream_t stream) {
    if (check_cache(kv) != GPT2_B200_OK || !qkv || !aligned16(qkv) || (qkv_layer_stride & 7))
        return GPT2_B200_EINVAL;
    if (!d_pos && (pos < 0 || pos >= kv->maxT)) return GPT2_B200_EINVAL;
    if (!att || !aligned16(att) || (att_layer_stride & 7)) return GPT2_B200_EINVAL;
    int rc = launch_kv_append(kv, 0, kv->nLayer, qkv, qkv_layer_stride, d_pos, pos, stream);
    if (rc != GPT2_B200_OK) return rc;
    // Attend over len = pos + 1 keys; with a device position the kernel adds the 1 itself, and the
    // split count is sized for the whole cache so a captured graph stays valid as pos grows.
    const long long slab = static_cast<long long>(kv->nHead) * kv->maxT * kv->headDim;
    const int max_len = d_pos ? kv->maxT : pos + 1;
    return launch_decode(att, att_layer_stride, qkv, qkv_layer_stride, kv->data, kv->data + slab,
                         2 * slab, nullptr, nullptr, d_pos, 0, 1, pos + 1, max_len, kv->nLayer,
                         kv->nHead, kv->maxT, stream);
}

// ================================================================ KV cache
int gpt2_kv_alloc_shape_b200(GPT2KVCache *kv, int nLayer, int nHead, int headDim, int maxT) {
    return kv_alloc(kv, nLayer, nHead, headDim, maxT);
}

int gpt2_kv_alloc_b200(GPT2KVCache *kv, int maxT) { return kv_alloc(kv, 12, 12, 64, maxT); }

void gpt2_kv_free_b200(GPT2KVCache *kv) {
    if (kv && kv->data) {
        cudaFree(kv->data);
        kv->data = nullptr;
    }
}

void gpt2_kv_reset_b200(GPT2KVCache *kv) {
    if (kv) kv->len = 0;
}

double gpt2_kv_step_bytes_b200(const GPT2KVCache *kv, int len) {
    return 2.0 * kv->nLayer * kv->nHead * static_cast<double>(len) * kv->headDim * sizeof(__half);
}

int gpt2_kv_append_b200_stream(GPT2KVCache *kv, int L0, int nL, const gpt2_half *qkv,
                               long long qkv_layer_stride, const int *d_pos, int pos,
                               cudaStream_t stream) {
    if (check_cache(kv) != GPT2_B200_OK || !qkv || !aligned16(qkv) || nL < 1 || L0 < 0 ||
        L0 + nL > kv->nLayer || (nL > 1 && (qkv_layer_stride & 7)))
        return GPT2_B200_EINVAL;
    if (!d_pos && (pos < 0 || pos >= kv->maxT)) return GPT2_B200_EINVAL;
    return launch_kv_append(kv, L0, nL, qkv, qkv_layer_stride, d_pos, pos, stream);
}

void gpt2_kv_append_one_b200(GPT2KVCache *kv, int L, const gpt2_half *qkv, int pos) {
    set_last_error(gpt2_kv_append_b200_stream(kv, L, 1, qkv, 0, nullptr, pos, 0));
}

int gpt2_kv_scatter_prefill_b200_stream(GPT2KVCache *kv, int L, const gpt2_half *qkv, int T,
                                        cudaStream_t stream) {
    if (check_cache(kv) != GPT2_B200_OK || L < 0 || L >= kv->nLayer || T < 0 || T > kv->maxT)
        return GPT2_B200_EINVAL;
    if (T > 0 && (!qkv || !aligned16(qkv))) return GPT2_B200_EINVAL;
    return launch_kv_scatter(kv, L, qkv, T, stream);
}

void gpt2_kv_scatter_prefill_b200(GPT2KVCache *kv, int L, const gpt2_half *qkv, int T) {
    set_last_error(gpt2_kv_scatter_prefill_b200_stream(kv, L, qkv, T, 0));
}

// ================================================================ backend, status, set-up
void gpt2_b200_compose_backend(GPT2Backend *dst, const GPT2Backend *base) {
    if (!dst) return;
    if (base) *dst = *base;
    else *dst = GPT2Backend{};
    dst->name = "b200";
    dst->attention = gpt2_attention_b200;
}

int gpt2_b200_reserve(int jobs, int n_head, int max_len) {
    if (jobs < 1 || n_head < 1 || max_len < 1) return GPT2_B200_EINVAL;
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_EDEVICE;
    size_t words = 0;
    const size_t floats = decode_workspace_floats(jobs, n_head, max_len, ctx->num_sms, &words);
    return ensure_decode_workspace(ctx, floats, words, 0);
}

unsigned gpt2_b200_status(int clear) {
    DeviceContext *ctx = device_context();
    if (!ctx) return 0xFFFFFFFFu;
    if (cudaDeviceSynchronize() != cudaSuccess) return 0xFFFFFFFFu;
    unsigned v = 0;
    if (cudaMemcpy(&v, ctx->status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0xFFFFFFFFu;
    v |= noalloc_status(clear != 0);  // the no-allocation decode keeps its word in its fixed scratch
    if (clear && v) {
        cudaMemset(ctx->status, 0, sizeof(unsigned));
        // A kernel that gave up may have left split-merge arrival counters part-way: re-arm them.
        if (ctx->counters) cudaMemset(ctx->counters, 0, ctx->counter_words * sizeof(unsigned));
        cudaDeviceSynchronize();
    }
    return v;
}

int gpt2_b200_last_error(void) {
    const int e = t_last_error;
    t_last_error = GPT2_B200_OK;
    return e;
}

const char *gpt2_b200_strerror(int code) {
    switch (code) {
        case GPT2_B200_OK: return "ok";
        case GPT2_B200_EINVAL: return "invalid argument";
        case GPT2_B200_ECUDA: return "CUDA runtime error";
        case GPT2_B200_ENOMEM: return "allocation refused";
        case GPT2_B200_EDEVICE: return "device is not compute capability 10.0 (sm_100) or lacks tensor-map support";
        case GPT2_B200_ETIMEOUT: return "a kernel wait timed out";
        case GPT2_B200_ECAPTURE: return "allocation needed while the stream is being captured";
        default: return "unknown";
    }
}

const char *gpt2_b200_version(void) { return "gpt2_b200 0.1 (sm_100a)"; }

}  // extern "C"

// ------------------------------------------------------------------ bounded-wait self-test
namespace b200 {
__global__ void k_wait_timeout_probe(unsigned *status, unsigned long long timeout_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    // Nothing arrives on this barrier: the wait must give up after timeout_ns and report it.
    const bool ok = mbar_wait(&bar, 0, timeout_ns);
    if (!ok && threadIdx.x == 0) atomicOr(status, ST_TEST_WAIT_TIMEOUT);
}
}  // namespace b200

extern "C" int gpt2_b200_selftest_wait_timeout(unsigned timeout_us) {
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_EDEVICE;
    if (timeout_us == 0 || timeout_us > 5000000u) return GPT2_B200_EINVAL;
    k_wait_timeout_probe<<<1, 32>>>(ctx->status, static_cast<unsigned long long>(timeout_us) * 1000ull);
    if (cudaGetLastError() != cudaSuccess) return GPT2_B200_ECUDA;
    const unsigned st = gpt2_b200_status(0);
    if (st == 0xFFFFFFFFu) return GPT2_B200_ECUDA;
    if (st & ST_TEST_WAIT_TIMEOUT) {
        unsigned keep = st & ~static_cast<unsigned>(ST_TEST_WAIT_TIMEOUT);
        cudaMemcpy(ctx->status, &keep, sizeof(keep), cudaMemcpyHostToDevice);
        return GPT2_B200_ETIMEOUT;
    }
    return GPT2_B200_OK;
}
