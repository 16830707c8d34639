// kvcache.cu — the KV cache arena and its writers, in the reference's layout.
//
// Layout (unchanged from cuda/kvcache.cuh:31-33 so either library can read the other's cache):
// one arena of [L][K|V][H][maxT][D] fp16; the decode attention reads K[h][0..len) as one contiguous
// slab per head, the append writes one position of every head (strided by maxT*D).
//
// The reference writes one half per thread (cuda/kvcache.cu:57-76). Here each thread moves one
// 16-byte vector (8 halves of one head row), so an append of all 12 heads of K and V is 192 threads
// and a prefill scatter of T rows is T*192 threads.
#include <cstdio>

#include "common.cuh"

namespace b200 {
namespace kv {

constexpr int VEC = 8;  // halves per 16-byte vector

// Append position pos (or *d_pos) of layers L0 + blockIdx.x from qkv rows qkv + l*qkv_stride.
// Threads [0, E/8) copy K vectors, [E/8, 2E/8) copy V vectors.
__global__ void k_kv_append(__half *data, int L0, const __half *qkv, long long qkv_stride,
                            const int *d_pos, int pos, int H, int maxT, int D, unsigned *status) {
    const int l = blockIdx.x;
    const int E = H * D;
    const int nvec = E / VEC;
    const int t = threadIdx.x;
    if (t >= 2 * nvec) return;
    if (d_pos) pos = *d_pos;
    if (pos < 0 || pos >= maxT) {
        if (t == 0) atomicOr(status, ST_KV_BAD_POS);
        return;
    }
    const int which = t / nvec;         // 0 = K, 1 = V
    const int e = (t - which * nvec) * VEC;
    const int h = e / D, d = e - h * D;
    const long long slab = static_cast<long long>(H) * maxT * D;
    __half *dst = data + (2LL * (L0 + l) + which) * slab + static_cast<long long>(h) * maxT * D +
                  static_cast<long long>(pos) * D + d;
    const __half *src = qkv + l * qkv_stride + (1 + which) * E + e;
    *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
}

// Prefill scatter: rows 0..T-1 of qkv[T, 3E] into positions 0..T-1 of layer L.
__global__ void k_kv_scatter(__half *K, __half *V, const __half *qkv, int T, int H, int maxT, int D) {
    const int E = H * D;
    const int nvec = E / VEC;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long total = 2LL * T * nvec;
    if (idx >= total) return;
    const int which = static_cast<int>(idx / (static_cast<long long>(T) * nvec));
    const long long r = idx - which * static_cast<long long>(T) * nvec;
    const int t = static_cast<int>(r / nvec);
    const int e = static_cast<int>(r - static_cast<long long>(t) * nvec) * VEC;
    const int h = e / D, d = e - h * D;
    __half *dst = (which ? V : K) + static_cast<long long>(h) * maxT * D + static_cast<long long>(t) * D + d;
    const __half *src = qkv + static_cast<long long>(t) * 3 * E + (1 + which) * E + e;
    *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
}

}  // namespace kv

int kv_alloc(GPT2KVCache *kv, int nLayer, int nHead, int headDim, int maxT) {
    if (!kv || nLayer < 1 || nHead < 1 || headDim < 1 || maxT < 1 || (nHead * headDim) % 8 != 0)
        return 1;
    kv->data = nullptr;
    kv->maxT = maxT;
    kv->nLayer = nLayer;
    kv->nHead = nHead;
    kv->headDim = headDim;
    kv->len = 0;
    kv->bytes = static_cast<size_t>(2) * nLayer * nHead * maxT * headDim * sizeof(__half);
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return 1;
    // The reference's refusal rule: the arena must leave at least 64 MiB of device memory free.
    const size_t headroom = static_cast<size_t>(64) << 20;
    if (kv->bytes + headroom > free_b) {
        fprintf(stderr,
                "[gpt2_b200] KV cache of %zu bytes not allocated: %zu bytes free on the device, and "
                "%zu must stay free after it\n",
                kv->bytes, free_b, headroom);
        return 1;
    }
    void *p = nullptr;
    if (cudaMalloc(&p, kv->bytes) != cudaSuccess) return 1;
    kv->data = static_cast<__half *>(p);
    return 0;
}

int launch_kv_append(GPT2KVCache *kv, int L0, int nL, const __half *qkv, long long qkv_stride,
                     const int *d_pos, int pos, cudaStream_t stream) {
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_ECUDA;
    const int E = kv->nHead * kv->headDim;
    kv::k_kv_append<<<nL, 2 * E / kv::VEC, 0, stream>>>(kv->data, L0, qkv, qkv_stride, d_pos, pos,
                                                        kv->nHead, kv->maxT, kv->headDim, ctx->status);
    return cudaGetLastError() == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}

int launch_kv_scatter(GPT2KVCache *kv, int L, const __half *qkv, int T, cudaStream_t stream) {
    if (T == 0) return GPT2_B200_OK;
    const int E = kv->nHead * kv->headDim;
    const long long slab = static_cast<long long>(kv->nHead) * kv->maxT * kv->headDim;
    __half *K = kv->data + 2LL * L * slab;
    __half *V = K + slab;
    const long long total = 2LL * T * (E / kv::VEC);
    const int nt = 256;
    kv::k_kv_scatter<<<static_cast<unsigned>((total + nt - 1) / nt), nt, 0, stream>>>(
        K, V, qkv, T, kv->nHead, kv->maxT, kv->headDim);
    return cudaGetLastError() == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}

}  // namespace b200
