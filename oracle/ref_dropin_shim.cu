// ref_dropin_shim.cu — TEST INFRASTRUCTURE ONLY. Runs the reference's OWN forward pass and decode
// step (unmodified, from oracle/_ref/libref_gpu.so) with this library installed behind them the way a
// maintainer of the reference would install it, so a GPU test can show the drop-in at run time.
//
// What the reference's code calls, and what is swapped in:
//   - GPT2Backend.attention (cuda/kernels.cuh:73), called by gpt2_forward_cuda at
//     cuda/forward_cuda.cu:98: a backend composed the reference's way (cuda/kernels_fused.cu:157-164,
//     copy a backend, replace slots) with gpt2_attention_b200 and, for the decode GEMVs,
//     gpt2_gemv_b200 (the GPT2Backend.gemv slot, cuda/kernels.cuh:94);
//   - gpt2_kv_scatter_prefill (cuda/forward_cuda.cu:97), gpt2_kv_append_one and gpt2_attn_decode
//     (cuda/kvcache.cu:250-252): plain functions in the reference, not backend slots. A maintainer
//     edits their bodies to call the _b200 entry points; here the same effect is had
//     without touching the reference's sources: this library defines the three functions and is
//     loaded BEFORE libref_gpu.so, so the dynamic linker binds the reference's own calls to them
//     (the calls go through the PLT). With routing off they forward to the reference's definitions
//     (dlsym RTLD_NEXT), so the stock path runs in the same process for comparison.
//
// Every routed call is counted, so the test can check that the library really served them.
#include <dlfcn.h>

#include <cstring>
#include <vector>

#include "kernels.cuh"
#include "kvcache.cuh"
#include "gpt2_b200.h"

namespace {
int g_route = 0;           // 1: the reference's cache calls go to this library
long long g_calls[4] = {}; // routed: decode attention, append, scatter, prefill attention

template <typename F>
F next_definition(const char *mangled) {
    return reinterpret_cast<F>(dlsym(RTLD_NEXT, mangled));
}

void counted_attention(half *att, const half *qkv, int T, int E, int H, int D) {
    ++g_calls[3];
    gpt2_attention_b200(att, qkv, T, E, H, D);
}

// The B200 backend, composed at first use (never during static initialisation, the reference's
// own rule for GPT2_BACKEND_GEMV, cuda/kvcache.cu:280-290).
const GPT2Backend *b200_backend() {
    static GPT2Backend b;
    static bool made = false;
    if (!made) {
        gpt2_b200_compose_backend(&b, &GPT2_BACKEND_GEMV);
        b.attention = counted_attention;
        b.gemv = gpt2_gemv_b200;
        made = true;
    }
    return &b;
}
}  // namespace

// ---- the reference's cache functions, bound here first (same C++ signatures, kvcache.cuh:49-58)
void gpt2_attn_decode(half *att, const half *qkv, const GPT2KVCache *kv, int L, int len) {
    if (g_route) {
        ++g_calls[0];
        gpt2_attn_decode_b200(att, qkv, kv, L, len);
        return;
    }
    static auto stock = next_definition<void (*)(half *, const half *, const GPT2KVCache *, int, int)>(
        "_Z16gpt2_attn_decodeP6__halfPKS_PK11GPT2KVCacheii");
    stock(att, qkv, kv, L, len);
}

void gpt2_kv_append_one(GPT2KVCache *kv, int L, const half *qkv, int pos) {
    if (g_route) {
        ++g_calls[1];
        gpt2_kv_append_one_b200(kv, L, qkv, pos);
        return;
    }
    static auto stock = next_definition<void (*)(GPT2KVCache *, int, const half *, int)>(
        "_Z18gpt2_kv_append_oneP11GPT2KVCacheiPK6__halfi");
    stock(kv, L, qkv, pos);
}

void gpt2_kv_scatter_prefill(GPT2KVCache *kv, int L, const half *qkv, int T) {
    if (g_route) {
        ++g_calls[2];
        gpt2_kv_scatter_prefill_b200(kv, L, qkv, T);
        return;
    }
    static auto stock = next_definition<void (*)(GPT2KVCache *, int, const half *, int)>(
        "_Z23gpt2_kv_scatter_prefillP11GPT2KVCacheiPK6__halfi");
    stock(kv, L, qkv, T);
}

extern "C" {

// 1 when the three reference functions above are the ones the reference's code binds to and their
// stock definitions were found behind them.
int dropin_interposed(void) {
    return dlsym(RTLD_NEXT, "_Z16gpt2_attn_decodeP6__halfPKS_PK11GPT2KVCacheii") != nullptr &&
           dlsym(RTLD_NEXT, "_Z18gpt2_kv_append_oneP11GPT2KVCacheiPK6__halfi") != nullptr &&
           dlsym(RTLD_NEXT, "_Z23gpt2_kv_scatter_prefillP11GPT2KVCacheiPK6__halfi") != nullptr;
}

// The reference's prompt-then-generate flow on one sequence: gpt2_prefill_fill_cache over ids[0..T)
// (gpt2_forward_cuda with the cache capture, cuda/kvcache.cu:271-277), then n_decode calls of
// gpt2_decode_step_cuda (cuda/kvcache.cu:233-269) consuming next_ids[i] at position T+i.
// use_b200 = 0 runs the reference's stock GEMV backend and cache functions; 1 runs the B200 backend
// and routes the cache functions to this library. Outputs (host): logits [(n_decode+1)][50257] fp16
// (row 0 = the prompt's last position), cache = the final [L][K|V][H][maxT][D] arena, calls[4] =
// routed call counts. Returns a cudaError_t, or -1 for bad arguments.
int dropin_generate(int use_b200, const void *weights, const int *ids, int T, const int *next_ids,
                    int n_decode, int maxT, void *logits, void *cache, long long *calls) {
    if (!weights || !ids || T < 1 || n_decode < 0 || T + n_decode > maxT || !logits || !cache)
        return -1;
    const GPT2Backend *be = use_b200 ? b200_backend() : &GPT2_BACKEND_GEMV;
    const GPT2WeightsGPU *w = static_cast<const GPT2WeightsGPU *>(weights);
    GPT2KVCache kv;
    if (gpt2_kv_alloc(&kv, maxT) != 0) return -1;
    cudaMemset(kv.data, 0, kv.bytes);
    GPT2ScratchGPU s;
    gpt2_scratch_alloc(&s, maxT);
    int *d_ids = nullptr;
    half *d_logits = nullptr;
    cudaMalloc(&d_ids, sizeof(int) * T);
    cudaMalloc(&d_logits, sizeof(half) * GPT2_VOCAB);
    cudaMemcpy(d_ids, ids, sizeof(int) * T, cudaMemcpyHostToDevice);
    for (int i = 0; i < 4; ++i) g_calls[i] = 0;
    g_route = use_b200;

    GPT2CapsGPU caps;
    std::memset(&caps, 0, sizeof(caps));
    caps.logits = d_logits;  // the last position's logits (logits_all = 0)
    gpt2_prefill_fill_cache(be, w, &kv, d_ids, T, &s, &caps);
    half *out = static_cast<half *>(logits);
    cudaMemcpy(out, d_logits, sizeof(half) * GPT2_VOCAB, cudaMemcpyDeviceToHost);
    for (int i = 0; i < n_decode; ++i) {
        gpt2_decode_step_cuda(be, w, &kv, next_ids[i], T + i, &s, d_logits, nullptr);
        cudaMemcpy(out + static_cast<size_t>(i + 1) * GPT2_VOCAB, d_logits, sizeof(half) * GPT2_VOCAB,
                   cudaMemcpyDeviceToHost);
    }
    cudaError_t err = cudaDeviceSynchronize();
    if (kv.len != T + n_decode && err == cudaSuccess) err = cudaErrorUnknown;
    cudaMemcpy(cache, kv.data, kv.bytes, cudaMemcpyDeviceToHost);
    g_route = 0;
    if (calls)
        for (int i = 0; i < 4; ++i) calls[i] = g_calls[i];
    cudaFree(d_ids);
    cudaFree(d_logits);
    gpt2_scratch_free(&s);
    gpt2_kv_free(&kv);
    return err == cudaSuccess ? static_cast<int>(cudaGetLastError()) : static_cast<int>(err);
}

}  // extern "C"
