// ref_gpu_shim.cu — TEST INFRASTRUCTURE ONLY. extern "C" handles on the reference's CUDA kernels.
//
// oracle/Makefile compiles this file together with the reference's unmodified cuda/*.cu and
// model/weights.c (from where they lie in the reference tree) into oracle/_ref/libref_gpu.so for
// sm_100a. The reference's launchers have C++ linkage and run on the legacy default stream; these
// wrappers give the parity tests a C ABI to them and synchronise after each call.
//
// Wrapped entry points (reference file:line):
//   gpt2_attention_flash       cuda/kernels_fused.cu:145-149  (GPT2_BACKEND_FLASH.attention)
//   GPT2_BACKEND_NAIVE.attention cuda/kernels_naive.cu:109-111
//   gpt2_attn_decode           cuda/kvcache.cu:207-210
//   gpt2_kv_append_one         cuda/kvcache.cu:204-206
//   gpt2_kv_scatter_prefill    cuda/kvcache.cu:78-81
//   gpt2_decode_step_cuda      cuda/kvcache.cu:233-269 with GPT2_BACKEND_GEMV (kvcache.cu:280-290),
//                              the reference's fp16 decode path (M=1 GEMVs + its attention)
//   gpt2_prefill_fill_cache    cuda/kvcache.cu:271-277 (the prefill forward that fills the cache)
#include "kernels.cuh"
#include "kvcache.cuh"
#include <cuda_runtime.h>

static GPT2KVCache view(void *data, int maxT) {
    GPT2KVCache kv;
    kv.data = (half *)data;
    kv.maxT = maxT; kv.nLayer = GPT2_N_LAYER; kv.nHead = GPT2_N_HEAD; kv.headDim = GPT2_HEAD_DIM;
    kv.bytes = (size_t)2 * kv.nLayer * kv.nHead * maxT * kv.headDim * sizeof(half);
    kv.len = 0;
    return kv;
}

extern "C" {

int ref_gpu_attention_flash(void *att, const void *qkv, int T) {
    gpt2_attention_flash((half *)att, (const half *)qkv, T, GPT2_N_EMBD, GPT2_N_HEAD, GPT2_HEAD_DIM);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_attention_naive(void *att, const void *qkv, int T) {
    GPT2_BACKEND_NAIVE.attention((half *)att, (const half *)qkv, T, GPT2_N_EMBD, GPT2_N_HEAD,
                                 GPT2_HEAD_DIM);
    return (int)cudaDeviceSynchronize();
}

// kv_data: the [L][K|V][H][maxT][D] arena (kvcache.cuh:31-33); qkv: the step's [3E] row.
int ref_gpu_attn_decode(void *att, const void *qkv, void *kv_data, int maxT, int L, int len) {
    GPT2KVCache kv = view(kv_data, maxT);
    gpt2_attn_decode((half *)att, (const half *)qkv, &kv, L, len);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_kv_append_one(void *kv_data, int maxT, int L, const void *qkv, int pos) {
    GPT2KVCache kv = view(kv_data, maxT);
    gpt2_kv_append_one(&kv, L, (const half *)qkv, pos);
    return (int)cudaDeviceSynchronize();
}

int ref_gpu_kv_scatter_prefill(void *kv_data, int maxT, int L, const void *qkv, int T) {
    GPT2KVCache kv = view(kv_data, maxT);
    gpt2_kv_scatter_prefill(&kv, L, (const half *)qkv, T);
    return (int)cudaDeviceSynchronize();
}

// One decode step of ONE sequence through the reference's own step function. weights points at a
// GPT2WeightsGPU (cuda/kernels.cuh:41-48) whose fp16 tensors the caller owns (q must be NULL);
// kv_data is that sequence's [L][K|V][H][maxT][D] arena, holding positions 0..pos-1. logits [V]
// may be NULL; caps (14 x 768 halves) may be NULL.
int ref_gpu_decode_step(const void *weights, void *kv_data, int maxT, int token, int pos, void *logits,
                        void *caps) {
    static GPT2ScratchGPU s;
    static bool have = false;
    if (!have) {
        gpt2_scratch_alloc(&s, 1);
        have = true;
    }
    GPT2KVCache kv = view(kv_data, maxT);
    kv.len = pos;
    gpt2_decode_step_cuda(&GPT2_BACKEND_GEMV, static_cast<const GPT2WeightsGPU *>(weights), &kv,
                          token, pos, &s, static_cast<half *>(logits), static_cast<half *>(caps));
    return (int)cudaDeviceSynchronize();
}

// The reference's prefill that fills a sequence's cache (gpt2_prefill_fill_cache, cuda/kvcache.cu:
// 271-277: gpt2_forward_cuda over d_ids[0..T) with the cache capture, GEMV backend = tiled GEMM + its
// flash attention) into kv_data (rows 0..T-1 of every layer).
int ref_gpu_prefill_fill_cache(const void *weights, void *kv_data, int maxT, const int *d_ids, int T) {
    static GPT2ScratchGPU s;
    static int have = 0;
    if (T > maxT || T < 1) return -1;
    if (have < T) {
        if (have) gpt2_scratch_free(&s);
        gpt2_scratch_alloc(&s, T);
        have = T;
    }
    GPT2KVCache kv = view(kv_data, maxT);
    gpt2_prefill_fill_cache(&GPT2_BACKEND_GEMV, static_cast<const GPT2WeightsGPU *>(weights), &kv, d_ids,
                            T, &s, nullptr);
    if (kv.len != T) return -1;
    return (int)cudaDeviceSynchronize();
}

}  // extern "C"
