// decode.cu — M=1 decode attention over the KV cache: split-context flash-decoding.
//
// Computes what the reference's k_attn_decode computes (cuda/kvcache.cu:88-129): for one query per
// (job, head) — a job is a layer of one cache or one sequence — att[h*64:(h+1)*64] =
// sum_{j<len} softmax_j(q.k_j / 8) v_j over the head-major [H][maxT][64] fp16 slabs.
//
// The reference uses one 64-thread block per head with three passes, per-thread 128-byte-strided K
// reads and block tree reductions, i.e. 12 blocks on the whole GPU. Here the context is split into
// chunks of `chunk` keys (16..128); each CTA of 128 threads owns one (split, head, job):
//   - thread t owns key group t/8 (keys k0 + t/8 + 16 i) and dims 8*(t%8) .. +7 of every key, so one
//     16-byte load per key per thread, 8 threads covering a 128-byte row: fully coalesced;
//   - all of the CTA's K and V rows are loaded (ld.global.nc, no L1 allocation) before any math, so
//     every thread has up to 16 independent 16-byte loads in flight;
//   - q.k partial dots are reduced across the 8 threads of a key with 3 xor-shuffles; the chunk max
//     and sum are warp-shuffle + one shared-memory step; scores live in the log2 domain (q pre-scaled
//     by log2(e)/8) and use the hardware ex2;
//   - the CTA's partial (o[64], m, l) goes to a workspace; the last CTA of a (job, head) to arrive
//     (an atomic counter) merges all partials and writes fp16, then re-arms the counter to zero.
// One launch therefore covers every layer / sequence of a decode step.
#include <cmath>
#include <cstdio>
#include <mutex>

#include <algorithm>

#include "common.cuh"
#include "ptx.cuh"

namespace b200 {
namespace decode {

constexpr int HD = 64;
constexpr int NT = 128;           // threads per CTA
constexpr int KEYS_PER_PASS = 16; // 128 threads / 8 threads per key row
constexpr int MAX_PASSES = 8;     // chunk <= 128 keys
constexpr int PART_STRIDE = HD + 2;  // o[64], m, l (floats)

struct Params {
    const __half *q;          // job j, head h query at q + j*q_stride + h*64
    long long q_stride;
    // K/V slabs of job j: either kbase + j*kv_stride (strided jobs) or k_ptrs[j] (pointer arrays)
    const __half *kbase;
    const __half *vbase;
    long long kv_stride;
    const __half *const *k_ptrs;
    const __half *const *v_ptrs;
    __half *out;              // job j output at out + j*out_stride
    long long out_stride;
    const int *d_len;         // device key count(s), or nullptr to use `len`
    int len_per_job;          // 1: d_len[j] per job; 0: d_len[0] for every job
    int len_add;              // added to a device length (1 turns an append position into a count)
    int len;
    int H, maxT, njobs;
    int chunk;                // keys per split (multiple of 16, <= 128)
    int nsplit_max;           // grid.x
    float scale_log2;         // log2(e) / sqrt(64)
    float *part;              // [njobs][H][nsplit_max][PART_STRIDE]
    unsigned *counters;       // [njobs][H], zero between calls
    unsigned *status;
};

__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float dot8(const float (&q)[8], const uint4 &k) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&k);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        s = fmaf(q[2 * i], f.x, s);
        s = fmaf(q[2 * i + 1], f.y, s);
    }
    return s;
}

__global__ void __launch_bounds__(NT) k_decode_split(const Params p) {
    const int split = blockIdx.x, h = blockIdx.y, job = blockIdx.z;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int kg = t >> 3;      // key group 0..15
    const int ds = t & 7;       // dim slice: dims 8*ds .. 8*ds+7

    int len = p.len;
    if (p.d_len) len = (p.len_per_job ? p.d_len[job] : p.d_len[0]) + p.len_add;
    if (len < 1 || len > p.maxT) {
        if (t == 0 && split == 0) atomicOr(p.status, ST_DECODE_BAD_LEN);
        return;
    }
    const int nsplit = (len + p.chunk - 1) / p.chunk;
    if (split >= nsplit) return;
    const int k0 = split * p.chunk;
    const int k1 = min(k0 + p.chunk, len);

    const __half *K = p.k_ptrs ? p.k_ptrs[job] : p.kbase + job * p.kv_stride;
    const __half *V = p.v_ptrs ? p.v_ptrs[job] : p.vbase + job * p.kv_stride;
    K += static_cast<long long>(h) * p.maxT * HD + ds * 8;
    V += static_cast<long long>(h) * p.maxT * HD + ds * 8;

    // Issue every K and V load of this thread before any arithmetic.
    uint4 kr[MAX_PASSES], vr[MAX_PASSES];
#pragma unroll
    for (int i = 0; i < MAX_PASSES; ++i) {
        const int key = k0 + kg + KEYS_PER_PASS * i;
        if (key < k1) kr[i] = ld_stream(K + static_cast<long long>(key) * HD);
        else kr[i] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < MAX_PASSES; ++i) {
        const int key = k0 + kg + KEYS_PER_PASS * i;
        if (key < k1) vr[i] = ld_stream(V + static_cast<long long>(key) * HD);
        else vr[i] = make_uint4(0, 0, 0, 0);
    }

    float qv[8];
    {
        const uint4 qr = *reinterpret_cast<const uint4 *>(p.q + job * p.q_stride + h * HD + ds * 8);
        const __half2 *q2 = reinterpret_cast<const __half2 *>(&qr);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(q2[i]);
            qv[2 * i] = f.x * p.scale_log2;
            qv[2 * i + 1] = f.y * p.scale_log2;
        }
    }

    float s[MAX_PASSES];
    float mloc = -INFINITY;
#pragma unroll
    for (int i = 0; i < MAX_PASSES; ++i) {
        float d = dot8(qv, kr[i]);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        d += __shfl_xor_sync(0xffffffffu, d, 4);
        const int key = k0 + kg + KEYS_PER_PASS * i;
        s[i] = key < k1 ? d : -INFINITY;
        mloc = fmaxf(mloc, s[i]);
    }
    __shared__ float red_m[NT / 32], red_l[NT / 32];
    __shared__ float red_o[NT / 32][HD];
    __shared__ int is_last;
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 8));
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 16));
    if (lane == 0) red_m[warp] = mloc;
    __syncthreads();
    const float m = fmaxf(fmaxf(red_m[0], red_m[1]), fmaxf(red_m[2], red_m[3]));

    float acc[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) acc[d] = 0.f;
    float lsum = 0.f;
#pragma unroll
    for (int i = 0; i < MAX_PASSES; ++i) {
        const float pr = ex2_approx(s[i] - m);  // 0 for keys outside [k0, k1)
        lsum += pr;
        const __half2 *v2 = reinterpret_cast<const __half2 *>(&vr[i]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(v2[e]);
            acc[2 * e] = fmaf(pr, f.x, acc[2 * e]);
            acc[2 * e + 1] = fmaf(pr, f.y, acc[2 * e + 1]);
        }
    }
    // Reduce over the 4 key groups of this warp that share the dim slice (lanes ds, ds+8, ...).
#pragma unroll
    for (int d = 0; d < 8; ++d) {
        acc[d] += __shfl_xor_sync(0xffffffffu, acc[d], 8);
        acc[d] += __shfl_xor_sync(0xffffffffu, acc[d], 16);
    }
    // lsum: every thread of a key group holds the same p values; count each key once (ds == 0).
    float lw = ds == 0 ? lsum : 0.f;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
    if (lane < 8) {
#pragma unroll
        for (int d = 0; d < 8; ++d) red_o[warp][lane * 8 + d] = acc[d];
    }
    if (lane == 0) red_l[warp] = lw;
    __syncthreads();

    const int jh = job * p.H + h;
    if (nsplit == 1) {
        if (t < HD / 2) {
            const float l = red_l[0] + red_l[1] + red_l[2] + red_l[3];
            const float inv = 1.f / l;
            const int d = 2 * t;
            const float o0 = (red_o[0][d] + red_o[1][d] + red_o[2][d] + red_o[3][d]) * inv;
            const float o1 = (red_o[0][d + 1] + red_o[1][d + 1] + red_o[2][d + 1] + red_o[3][d + 1]) * inv;
            reinterpret_cast<__half2 *>(p.out + job * p.out_stride + h * HD)[t] = __floats2half2_rn(o0, o1);
        }
        return;
    }

    float *mine = p.part + (static_cast<long long>(jh) * p.nsplit_max + split) * PART_STRIDE;
    if (t < HD) mine[t] = red_o[0][t] + red_o[1][t] + red_o[2][t] + red_o[3][t];
    if (t == HD) mine[HD] = m;
    if (t == HD + 1) mine[HD + 1] = red_l[0] + red_l[1] + red_l[2] + red_l[3];
    __threadfence();
    __syncthreads();
    if (t == 0) {
        const unsigned prev = atomicAdd(&p.counters[jh], 1u);
        is_last = (prev == static_cast<unsigned>(nsplit - 1));
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    // Merge the nsplit partials of this (job, head): O = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s.
    const float *base = p.part + static_cast<long long>(jh) * p.nsplit_max * PART_STRIDE;
    if (t < HD) {
        float M = -INFINITY;
        for (int sidx = 0; sidx < nsplit; ++sidx) M = fmaxf(M, __ldcg(base + sidx * PART_STRIDE + HD));
        float L = 0.f, O = 0.f;
        for (int sidx = 0; sidx < nsplit; ++sidx) {
            const float *ps = base + sidx * PART_STRIDE;
            const float w = ex2_approx(__ldcg(ps + HD) - M);
            L = fmaf(w, __ldcg(ps + HD + 1), L);
            O = fmaf(w, __ldcg(ps + t), O);
        }
        p.out[job * p.out_stride + h * HD + t] = __float2half_rn(O / L);
    }
    if (t == 0) p.counters[jh] = 0u;  // re-arm for the next call / graph replay
}

}  // namespace decode

// Ensures the workspace holds `floats` partial floats and `words` counters (zeroed). Refuses to
// allocate while `stream` is being captured.
int ensure_decode_workspace(DeviceContext *ctx, size_t floats, size_t words, cudaStream_t stream) {
    if (ctx->part_floats >= floats && ctx->counter_words >= words) return GPT2_B200_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) return GPT2_B200_ECUDA;
    if (cs != cudaStreamCaptureStatusNone) return GPT2_B200_ECAPTURE;
    if (cudaDeviceSynchronize() != cudaSuccess) return GPT2_B200_ECUDA;
    // A grown buffer replaces the old one but the old one is never freed: a CUDA graph captured
    // earlier keeps the address it was captured with. Growth at least doubles, so the retired
    // buffers together stay below the live one.
    if (ctx->part_floats < floats) {
        floats = std::max(floats, 2 * ctx->part_floats);
        ctx->part = nullptr;
        ctx->part_floats = 0;
        if (cudaMalloc(&ctx->part, floats * sizeof(float)) != cudaSuccess) return GPT2_B200_ENOMEM;
        ctx->part_floats = floats;
    }
    if (ctx->counter_words < words) {
        words = std::max(words, 2 * ctx->counter_words);
        ctx->counters = nullptr;
        ctx->counter_words = 0;
        if (cudaMalloc(&ctx->counters, words * sizeof(unsigned)) != cudaSuccess) return GPT2_B200_ENOMEM;
        if (cudaMemset(ctx->counters, 0, words * sizeof(unsigned)) != cudaSuccess) return GPT2_B200_ECUDA;
        ctx->counter_words = words;
    }
    return GPT2_B200_OK;
}

int decode_stream_splits(int max_len, long long pairs, int num_sms);
int launch_decode_stream(__half *out, long long out_stride, const __half *q, long long q_stride,
                         const __half *kbase, const __half *vbase, long long kv_stride,
                         const __half *const *k_ptrs, const __half *const *v_ptrs, const int *d_len,
                         int len_per_job, int len_add, int len, int max_len, int njobs, int H,
                         int maxT, cudaStream_t stream, bool pdl, bool l2_early = false);

// Workspace the decode launches need for `jobs` (layer x sequence) decodes of up to max_len keys.
size_t decode_workspace_floats(int jobs, int H, int max_len, int num_sms, size_t *words) {
    const int nsplit = decode_stream_splits(max_len, static_cast<long long>(jobs) * H, num_sms);
    if (words) *words = static_cast<size_t>(jobs) * H;
    return nsplit > 1 ? static_cast<size_t>(jobs) * H * nsplit * (decode::HD + 2) : 0;
}

// Decode for `njobs` jobs: the streamed kernel (decode_stream.cu). Exactly one of
// (kbase, vbase, kv_stride) or (k_ptrs, v_ptrs) describes the slabs. Arguments are validated by the
// caller.
int launch_decode(__half *out, long long out_stride, const __half *q, long long q_stride,
                  const __half *kbase, const __half *vbase, long long kv_stride,
                  const __half *const *k_ptrs, const __half *const *v_ptrs, const int *d_len,
                  int len_per_job, int len_add, int len, int max_len, int njobs, int H, int maxT,
                  cudaStream_t stream, bool pdl, bool l2_early) {
    return launch_decode_stream(out, out_stride, q, q_stride, kbase, vbase, kv_stride, k_ptrs,
                                v_ptrs, d_len, len_per_job, len_add, len, max_len, njobs, H, maxT,
                                stream, pdl, l2_early);
}

}  // namespace b200

// =====================================================================================
// Decode without any allocation by the library.
//
// Some callers cannot let a library call cudaMalloc: a serving loop that has handed all of HBM to
// its own pool allocator (a surprise cudaMalloc there fails or fragments the pool), a host that
// forbids device allocations once it has finished initialising so that memory use stays fixed and
// predictable, or a latency-critical path where cudaMalloc/cudaFree would synchronise the device.
// gpt2_attn_decode_b200_layers grows a per-device workspace on demand; the entry point below runs
// the same split-context kernel with its scratch (split partials, arrival counters, status word)
// in one fixed array that is part of the library image instead.
//
// Limits: at most NOALLOC_PARTIALS (layer, head, split) partial records and NOALLOC_COUNTERS
// (layer, head) pairs per call; splits are 128 keys. For GPT-2 (12 heads) that covers all 12
// layers up to 1024 keys. Larger requests are refused before anything is launched.
// =====================================================================================
namespace b200 {
namespace noalloc {

constexpr int CHUNK = decode::KEYS_PER_PASS * decode::MAX_PASSES;  // 128 keys per split
constexpr size_t NOALLOC_COUNTERS = 2048;                            // (layer, head) pairs
constexpr size_t NOALLOC_STATUS_WORDS = 64;                          // status word + padding
constexpr size_t NOALLOC_PARTIAL_FLOATS = 131072;                    // 512 KiB of partials
constexpr size_t NOALLOC_PARTIALS = NOALLOC_PARTIAL_FLOATS / decode::PART_STRIDE;
constexpr size_t NOALLOC_WORDS = NOALLOC_COUNTERS + NOALLOC_STATUS_WORDS + NOALLOC_PARTIAL_FLOATS;

// The scratch itself: [counters | status | partials], 4-byte words, about 520 KiB. Every GPU that
// loads this library holds one copy until the process exits. Device code could name it directly;
// host code only ever uses the device address looked up below.
static __device__ __align__(256) unsigned g_scratch[NOALLOC_WORDS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned *g_addr[kMaxDevices] = {};

// Looks up the device address of g_scratch for the current device, once per device. (In host code
// the name g_scratch is only a host-side stand-in; passing it to a kernel would be wrong.) The
// address is kept for the life of the process: after cudaDeviceReset, which unloads the library's
// module, it is stale and the entry point must not be called again.
unsigned *scratch_address(int *rc) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *rc = GPT2_B200_ECUDA;
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess || !p) {
            *rc = GPT2_B200_ECUDA;
            return nullptr;
        }
        g_addr[dev] = static_cast<unsigned *>(p);
    }
    *rc = GPT2_B200_OK;
    return g_addr[dev];
}

}  // namespace noalloc

// The status word inside the fixed scratch of the current device (0 when the no-allocation entry
// point has not run there), cleared when `clear`; gpt2_b200_status() ORs it into what it reports.
// The caller has synchronised the device.
unsigned noalloc_status(bool clear) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= noalloc::kMaxDevices) return 0;
    unsigned *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(noalloc::g_mu);
        base = noalloc::g_addr[dev];
    }
    if (!base) return 0;
    unsigned *status = base + noalloc::NOALLOC_COUNTERS;
    unsigned v = 0;
    if (cudaMemcpy(&v, status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return 0xFFFFFFFFu;
    if (clear && v) cudaMemset(status, 0, sizeof(unsigned));
    return v;
}

}  // namespace b200

// Same computation as gpt2_attn_decode_b200_layers with a host length, run by k_decode_split (an
// 8-threads-per-key split-context kernel with a last-CTA merge; the regular entry point runs
// k_decode_stream), but it allocates nothing: the scratch is the fixed array above. The first call
// on each device looks up that array's device address; with CUDA's lazy module loading that is also
// when the driver places the library module's globals, this array among them, in device memory.
// So make the first call on each device during initialisation: before a pool allocator takes the
// rest of HBM or allocations are frozen, and before any stream capture. Every call on a device
// shares the one array and leaves its contents behind; the arrival counters are cleared at the
// start of each call, so calls must not overlap on the GPU (issue them on one stream, or order
// them), or they race on the shared scratch. Its status word is reported by gpt2_b200_status().
extern "C" int gpt2_attn_decode_b200_layers_noalloc(gpt2_half *att, long long att_layer_stride,
                                                    const gpt2_half *q, long long q_layer_stride,
                                                    const GPT2KVCache *kv, int L0, int nL, int len,
                                                    cudaStream_t stream) {
    using namespace b200;
    const auto a16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
    if (!kv || !kv->data || !a16(kv->data) || kv->headDim != 64 || kv->nHead < 1 || kv->nLayer < 1 ||
        kv->maxT < 1)
        return GPT2_B200_EINVAL;
    if (nL < 1 || L0 < 0 || L0 + nL > kv->nLayer || !att || !q || !a16(att) || !a16(q))
        return GPT2_B200_EINVAL;
    if (nL > 1 && ((att_layer_stride & 7) || (q_layer_stride & 7))) return GPT2_B200_EINVAL;
    if (len < 1 || len > kv->maxT) return GPT2_B200_EINVAL;
    const int nsplit = (len + noalloc::CHUNK - 1) / noalloc::CHUNK;
    const size_t pairs = static_cast<size_t>(nL) * kv->nHead;
    if (pairs > noalloc::NOALLOC_COUNTERS || pairs * nsplit > noalloc::NOALLOC_PARTIALS) {
        fprintf(stderr,
                "[gpt2_b200] no-alloc decode: %zu (layer, head) pairs x %d splits exceeds the fixed "
                "scratch (%zu pairs, %zu partials); use gpt2_attn_decode_b200_layers\n",
                pairs, nsplit, noalloc::NOALLOC_COUNTERS, noalloc::NOALLOC_PARTIALS);
        return GPT2_B200_EINVAL;
    }
    int rc = GPT2_B200_OK;
    unsigned *base = noalloc::scratch_address(&rc);
    if (!base) return rc;
    unsigned *counters = base;
    unsigned *status = base + noalloc::NOALLOC_COUNTERS;
    float *part = reinterpret_cast<float *>(status + noalloc::NOALLOC_STATUS_WORDS);
    if (nsplit > 1 && cudaMemsetAsync(counters, 0, pairs * sizeof(unsigned), stream) != cudaSuccess)
        return GPT2_B200_ECUDA;

    const long long slab = static_cast<long long>(kv->nHead) * kv->maxT * kv->headDim;
    decode::Params p;
    p.q = q;
    p.q_stride = q_layer_stride;
    p.kbase = kv->data + 2LL * L0 * slab;
    p.vbase = p.kbase + slab;
    p.kv_stride = 2 * slab;
    p.k_ptrs = nullptr;
    p.v_ptrs = nullptr;
    p.out = att;
    p.out_stride = att_layer_stride;
    p.d_len = nullptr;
    p.len_per_job = 0;
    p.len_add = 0;
    p.len = len;
    p.H = kv->nHead;
    p.maxT = kv->maxT;
    p.njobs = nL;
    p.chunk = noalloc::CHUNK;
    p.nsplit_max = nsplit;
    p.scale_log2 = static_cast<float>(1.4426950408889634 / 8.0);
    p.part = part;
    p.counters = counters;
    p.status = status;
    dim3 grid(nsplit, kv->nHead, nL);
    decode::k_decode_split<<<grid, decode::NT, 0, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}
