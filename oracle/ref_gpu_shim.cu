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

}  // extern "C"
