// decode_stream.cu — M=1 decode attention over the KV cache, streamed through shared memory.
//
// Same operation as the reference's k_attn_decode (cuda/kvcache.cu:88-129): for one query per
// (job, head) — a job is a layer of one cache or one sequence — att[h*64:(h+1)*64] =
// sum_{j<len} softmax_j(q.k_j / 8) v_j over the head-major [H][maxT][64] fp16 K and V slabs.
//
// Decode is a pure HBM stream (36,864 bytes of K+V per key for the 12-layer step), so the kernel is
// built to keep every SM's share of HBM busy from start to finish:
//   - grid = (split, head, job), always one wave of CTAs (decode_stream_plan below); for the
//     12-layer GPT-2 step of one sequence that is one CTA per (layer, head) streaming its whole
//     context, so no cross-CTA merge is needed at all; batches of sequences use smaller CTAs
//     (the mid and small shapes below), several per SM, each (sequence, head) pair whole;
//   - warp 16 (one thread) issues cp.async.bulk copies of 128-key stages (16 KB of K + 16 KB of V,
//     the slabs are contiguous) into a 4-stage shared-memory ring, tracked by mbarriers (128 KB in
//     flight per SM: with more, the copies only queue longer in the memory system);
//   - warps 0-15 each own 8 keys of every stage: 4 lanes per key (16 dims each, q held pre-scaled by
//     log2(e)/8 in registers), two xor-shuffles per score, a warp-level online softmax (running max,
//     sum and 2 output dims per lane) with the hardware ex2, and V rows read as 128-byte lines;
//   - the 16 warps' (m, l, o) are merged once in shared memory; only when a (job, head) is split over
//     several CTAs (few jobs, e.g. one layer) do partials go through the workspace and the last CTA to
//     arrive merges them (atomic counter, re-armed to zero for the next call / graph replay).
// Every mbarrier wait is bounded; a timeout sets a status bit and the CTA unwinds after its own
// copies have landed.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "ptx.cuh"

namespace b200 {
namespace dstream {

constexpr int HD = 64;
constexpr int MAX_NSTAGE = 8;
constexpr int ROW_BYTES = HD * 2;            // 128 B per key row
constexpr int PART_STRIDE = HD + 2;

struct __align__(8) Bars {
    uint64_t full[MAX_NSTAGE];
    uint64_t empty[MAX_NSTAGE];
    int abort;
    int is_last;
};

// Shape of a CTA with NCW consumer warps (plus one producer warp): 8 keys per consumer warp per
// stage, so KPS = 8 * NCW keys and KPS * 128 bytes each of K and V per stage.
//   NCW = 16: 128-key stages, 128 KB ring, one CTA per SM (few (job, head) pairs: the GPT-2
//             12-layer step of one sequence, split over the context when pairs are fewer than SMs);
//   NCW = 4:  32-key stages, 3-stage 24 KB ring, eight CTAs per SM (many pairs: a batch of
//             sequences; the per-CTA ramp and tail of one pair overlap the others' streaming).
//             Measured at 64 sequences x 12 heads: 3 stages 5.17 / 5.96 TB/s at 512 / 1023 keys,
//             2 stages 5.02 / 5.73, 4 stages 4.89 / 5.56, 6 stages 3.99 / 4.58 (more CTAs per SM
//             beat a deeper ring per CTA); 2 or 8 consumer warps are slower.
//   NCW = 8:  64-key stages, 3-stage 48 KB ring, up to four CTAs per SM (between the two: one to
//             four SMs' worth of pairs, e.g. 13-49 sequences x 12 heads, where one CTA per pair
//             per SM would run a second, partial wave; each pair whole in one CTA, all in one wave).
template <int NCW, int NSTAGE>
struct Cfg {
    static constexpr int NT = 32 * (NCW + 1);
    static constexpr int KPS = 8 * NCW;
    static constexpr int STAGE_BYTES = KPS * ROW_BYTES;
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = OFF_K + NSTAGE * STAGE_BYTES;
    static constexpr int OFF_RED = OFF_V + NSTAGE * STAGE_BYTES;  // [NCW][64] o, [NCW] m, [NCW] l
    static constexpr int OFF_BAR = OFF_RED + (NCW * HD + 2 * NCW) * 4;
    static constexpr int SMEM_BYTES = OFF_BAR + static_cast<int>(sizeof(Bars));
    static_assert(NSTAGE >= 2 && NSTAGE <= MAX_NSTAGE, "ring depth");
    static_assert(OFF_BAR % 8 == 0, "mbarriers need 8-byte alignment");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};
constexpr int NCW_FEW = 16, NCW_MANY = 4, NCW_MID = 8;
constexpr int NSTAGE_FEW = 4, NSTAGE_MANY = 3, NSTAGE_MID = 3;
constexpr int MID_PER_SM = 4;  // resident CTAs of the mid shape per SM (shared memory, registers)
using CfgFew = Cfg<NCW_FEW, NSTAGE_FEW>;
using CfgMany = Cfg<NCW_MANY, NSTAGE_MANY>;
using CfgMid = Cfg<NCW_MID, NSTAGE_MID>;
static_assert(MID_PER_SM * (CfgMid::SMEM_BYTES + 1024) <= 228 * 1024, "mid shape: four CTAs per SM");

struct Params {
    const __half *q;
    long long q_stride;
    const __half *kbase;
    const __half *vbase;
    long long kv_stride;
    const __half *const *k_ptrs;
    const __half *const *v_ptrs;
    __half *out;
    long long out_stride;
    const int *d_len;
    int len_per_job;
    int len_add;
    int len;
    int H, maxT, njobs;
    int nsplit;               // grid.x: CTAs per (job, head) at most
    float scale_log2;
    float *part;              // [njobs][H][nsplit][PART_STRIDE] (used only when a pair is split)
    unsigned *counters;       // [njobs][H]
    unsigned *status;
    unsigned long long timeout_ns;
    // Inside a decode step only (0 elsewhere): bytes of K and of V per CTA that the producer requests
    // into L2 before the grid dependency wait (see the kernel).
    unsigned l2_early_bytes;
};

__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, unsigned long long to) {
    const bool ok = mbar_wait(bar, parity, to);
    return __all_sync(0xffffffffu, ok);
}

template <int NCW, int NSTAGE>
__global__ void __launch_bounds__(32 * (NCW + 1), NCW == NCW_MID ? MID_PER_SM : NCW == NCW_MANY ? 8 : 1)
    k_decode_stream(const Params p) {
    using C = Cfg<NCW, NSTAGE>;
    constexpr int KPS = C::KPS, STAGE_BYTES = C::STAGE_BYTES;
    constexpr int OFF_K = C::OFF_K, OFF_V = C::OFF_V, OFF_RED = C::OFF_RED, OFF_BAR = C::OFF_BAR;
    extern __shared__ __align__(128) uint8_t smem[];
    Bars *bars = reinterpret_cast<Bars *>(smem + OFF_BAR);
    float *red_o = reinterpret_cast<float *>(smem + OFF_RED);
    float *red_m = red_o + NCW * HD;
    float *red_l = red_m + NCW;
    const int split = blockIdx.x, h = blockIdx.y, job = blockIdx.z;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const unsigned long long to = p.timeout_ns;
    // Launched as a programmatic dependent (the batched decode step), the grid may start while its
    // predecessor finishes. Inside a decode step that predecessor is the QKV projection, which appends
    // each sequence's newest K/V row; the lengths were written by a kernel that completed before the
    // projection started, and every older row by an earlier step. So with l2_early_bytes set, the
    // producer first requests this CTA's older rows into L2 (a prefetch reads nothing into the CTA
    // and L2 is coherent), overlapping their HBM latency with the projection; everything the CTA
    // reads follows the wait.
    if (p.l2_early_bytes && t == NCW * 32) {
        int len0 = p.len;
        if (p.d_len) len0 = (p.len_per_job ? p.d_len[job] : p.d_len[0]) + p.len_add;
        if (len0 >= 2 && len0 <= p.maxT) {
            const int per0 = (len0 + p.nsplit - 1) / p.nsplit;
            const int chunk0 = ((per0 + KPS - 1) / KPS) * KPS;
            const int a = split * chunk0, b = min(a + chunk0, len0 - 1);  // rows before the newest
            if (b > a) {
                const uint32_t bytes = min(static_cast<uint32_t>(b - a) * ROW_BYTES, p.l2_early_bytes);
                const __half *K0 = p.k_ptrs ? p.k_ptrs[job] : p.kbase + job * p.kv_stride;
                const __half *V0 = p.v_ptrs ? p.v_ptrs[job] : p.vbase + job * p.kv_stride;
                const long long off = static_cast<long long>(h) * p.maxT * HD + static_cast<long long>(a) * HD;
                bulk_prefetch_l2(K0 + off, bytes);
                bulk_prefetch_l2(V0 + off, bytes);
            }
        }
    }
    grid_dependency_wait();
    grid_launch_dependents();

    int len = p.len;
    if (p.d_len) len = (p.len_per_job ? p.d_len[job] : p.d_len[0]) + p.len_add;
    if (len < 1 || len > p.maxT) {
        if (t == 0 && split == 0) atomicOr(p.status, ST_DECODE_BAD_LEN);
        return;
    }
    // Split of [0, len): chunks of whole stages; CTAs past the last chunk have nothing to do.
    const int per = (len + p.nsplit - 1) / p.nsplit;
    const int chunk = ((per + KPS - 1) / KPS) * KPS;
    const int nsplit = (len + chunk - 1) / chunk;
    if (split >= nsplit) return;
    const int k0 = split * chunk;
    const int k1 = min(k0 + chunk, len);
    const int nstages = (k1 - k0 + KPS - 1) / KPS;

    const __half *K = p.k_ptrs ? p.k_ptrs[job] : p.kbase + job * p.kv_stride;
    const __half *V = p.v_ptrs ? p.v_ptrs[job] : p.vbase + job * p.kv_stride;
    K += static_cast<long long>(h) * p.maxT * HD;
    V += static_cast<long long>(h) * p.maxT * HD;

    // The producer sets up the barriers and issues the first ring of copies before the block-wide
    // barrier; the consumers meanwhile bring their query into registers.
    const int first = min(nstages, NSTAGE);
    if (warp == NCW && lane == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], NCW);
        }
        bars->abort = 0;
        fence_mbar_init();
        for (int i = 0; i < first; ++i) {
            const int key = k0 + i * KPS;
            const uint32_t bytes = static_cast<uint32_t>(min(KPS, k1 - key)) * ROW_BYTES;
            mbar_arrive_expect_tx(&bars->full[i], 2 * bytes);
            bulk_load(smem + OFF_K + i * STAGE_BYTES, K + static_cast<long long>(key) * HD, bytes, &bars->full[i]);
            bulk_load(smem + OFF_V + i * STAGE_BYTES, V + static_cast<long long>(key) * HD, bytes, &bars->full[i]);
        }
    }
    const int kq = lane >> 2;        // key of this warp's 8 handled by this lane group
    const int dq = (lane & 3) * 16;  // 16 dims of that key handled by this lane
    float qv[16];
    if (warp < NCW) {
        const uint4 *q4 = reinterpret_cast<const uint4 *>(p.q + job * p.q_stride + h * HD + dq);
        const uint4 a = q4[0], b = q4[1];
        const __half2 *h2a = reinterpret_cast<const __half2 *>(&a);
        const __half2 *h2b = reinterpret_cast<const __half2 *>(&b);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 fa = __half22float2(h2a[i]);
            const float2 fb = __half22float2(h2b[i]);
            qv[2 * i] = fa.x * p.scale_log2;
            qv[2 * i + 1] = fa.y * p.scale_log2;
            qv[8 + 2 * i] = fb.x * p.scale_log2;
            qv[8 + 2 * i + 1] = fb.y * p.scale_log2;
        }
    }
    __syncthreads();

    if (warp == NCW) {
        // ------------------------------------------------------------ producer (one thread)
        if (lane == 0) {
            bool ok = true;
            int issued = first;
            for (int i = first; i < nstages; ++i) {
                const int s = i % NSTAGE;
                if (i >= NSTAGE) {
                    ok = mbar_wait(&bars->empty[s], ((i / NSTAGE) - 1) & 1, to);
                    if (!ok) break;
                }
                if (*reinterpret_cast<volatile int *>(&bars->abort)) break;
                const int key = k0 + i * KPS;
                const uint32_t bytes = static_cast<uint32_t>(min(KPS, k1 - key)) * ROW_BYTES;
                mbar_arrive_expect_tx(&bars->full[s], 2 * bytes);
                bulk_load(smem + OFF_K + s * STAGE_BYTES, K + static_cast<long long>(key) * HD, bytes,
                          &bars->full[s]);
                bulk_load(smem + OFF_V + s * STAGE_BYTES, V + static_cast<long long>(key) * HD, bytes,
                          &bars->full[s]);
                issued = i + 1;
            }
            if (!ok) {
                atomicOr(p.status, ST_DECODE_TIMEOUT);
                *reinterpret_cast<volatile int *>(&bars->abort) = 1;
            }
            // every issued copy lands before the CTA may exit
            bool drained = true;
            for (int i = (issued > NSTAGE ? issued - NSTAGE : 0); i < issued; ++i)
                drained = mbar_wait(&bars->full[i % NSTAGE], (i / NSTAGE) & 1, to) && drained;
            if (!drained) atomicOr(p.status, ST_DECODE_TIMEOUT);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ consumers (8 warps)
        float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;  // o: dims 2*lane, 2*lane+1
        bool ok = true;
        for (int i = 0; i < nstages; ++i) {
            const int s = i % NSTAGE;
            ok = warp_wait(&bars->full[s], (i / NSTAGE) & 1, to);
            if (!ok) break;
            const int rows = min(KPS, k1 - (k0 + i * KPS));
            const int krow = warp * 8 + kq;  // row of the stage this lane scores
            const bool valid = krow < rows;
            const uint8_t *kr = smem + OFF_K + s * STAGE_BYTES + krow * ROW_BYTES + dq * 2;
            float sc = -INFINITY;
            {
                const uint4 a = reinterpret_cast<const uint4 *>(kr)[0];
                const uint4 b = reinterpret_cast<const uint4 *>(kr)[1];
                const __half2 *h2a = reinterpret_cast<const __half2 *>(&a);
                const __half2 *h2b = reinterpret_cast<const __half2 *>(&b);
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 fa = __half22float2(h2a[e]);
                    const float2 fb = __half22float2(h2b[e]);
                    d = fmaf(qv[2 * e], fa.x, d);
                    d = fmaf(qv[2 * e + 1], fa.y, d);
                    d = fmaf(qv[8 + 2 * e], fb.x, d);
                    d = fmaf(qv[8 + 2 * e + 1], fb.y, d);
                }
                d += __shfl_xor_sync(0xffffffffu, d, 1);
                d += __shfl_xor_sync(0xffffffffu, d, 2);
                if (valid) sc = d;
            }
            float mt = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 4));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
            if (mt > m) {  // warp-uniform; m_t is finite whenever this warp has a valid key
                const float alpha = ex2_approx(m - mt);  // 0 on the first stage with keys
                l *= alpha;
                o0 *= alpha;
                o1 *= alpha;
                m = mt;
            }
            const float pk = valid ? ex2_approx(sc - m) : 0.f;
            float ps = pk;
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            ps += __shfl_xor_sync(0xffffffffu, ps, 8);
            ps += __shfl_xor_sync(0xffffffffu, ps, 16);
            l += ps;
            const uint8_t *vbase = smem + OFF_V + s * STAGE_BYTES + warp * 8 * ROW_BYTES + lane * 4;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float pkk = __shfl_sync(0xffffffffu, pk, 4 * k);
                if (warp * 8 + k < rows) {  // warp-uniform; never touch rows the copy did not fill
                    const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(vbase + k * ROW_BYTES));
                    o0 = fmaf(pkk, v.x, o0);
                    o1 = fmaf(pkk, v.y, o1);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->empty[s]);
        }
        if (!ok) {
            atomicOr(p.status, ST_DECODE_TIMEOUT);
            *reinterpret_cast<volatile int *>(&bars->abort) = 1;
            m = -INFINITY;
        }
        red_o[warp * HD + 2 * lane] = o0;
        red_o[warp * HD + 2 * lane + 1] = o1;
        if (lane == 0) {
            red_m[warp] = m;
            red_l[warp] = l;
        }
    }
    __syncthreads();
    if (*reinterpret_cast<volatile int *>(&bars->abort)) return;

    // ---------------------------------------------------------------- merge the 8 warps
    const int jh = job * p.H + h;
    float M = red_m[0];
#pragma unroll
    for (int w = 1; w < NCW; ++w) M = fmaxf(M, red_m[w]);
    if (nsplit == 1) {
        if (t < HD / 2) {
            float L = 0.f, a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int w = 0; w < NCW; ++w) {
                const float wt = red_m[w] == -INFINITY ? 0.f : ex2_approx(red_m[w] - M);
                L = fmaf(wt, red_l[w], L);
                a0 = fmaf(wt, red_o[w * HD + 2 * t], a0);
                a1 = fmaf(wt, red_o[w * HD + 2 * t + 1], a1);
            }
            const float inv = 1.f / L;
            reinterpret_cast<__half2 *>(p.out + job * p.out_stride + h * HD)[t] =
                __floats2half2_rn(a0 * inv, a1 * inv);
        }
        return;
    }
    float *mine = p.part + (static_cast<long long>(jh) * p.nsplit + split) * PART_STRIDE;
    if (t < HD) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; ++w)
            a = fmaf(red_m[w] == -INFINITY ? 0.f : ex2_approx(red_m[w] - M), red_o[w * HD + t], a);
        mine[t] = a;
    }
    if (t == HD) mine[HD] = M;
    if (t == HD + 1) {
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; ++w) L = fmaf(red_m[w] == -INFINITY ? 0.f : ex2_approx(red_m[w] - M), red_l[w], L);
        mine[HD + 1] = L;
    }
    __threadfence();
    __syncthreads();
    if (t == 0) {
        const unsigned prev = atomicAdd(&p.counters[jh], 1u);
        bars->is_last = (prev == static_cast<unsigned>(nsplit - 1));
    }
    __syncthreads();
    if (!bars->is_last) return;
    __threadfence();
    const float *base = p.part + static_cast<long long>(jh) * p.nsplit * PART_STRIDE;
    if (t < HD) {
        float MM = -INFINITY;
        for (int sidx = 0; sidx < nsplit; ++sidx) MM = fmaxf(MM, __ldcg(base + sidx * PART_STRIDE + HD));
        float L = 0.f, O = 0.f;
        for (int sidx = 0; sidx < nsplit; ++sidx) {
            const float *ps = base + sidx * PART_STRIDE;
            const float w = ex2_approx(__ldcg(ps + HD) - MM);
            L = fmaf(w, __ldcg(ps + HD + 1), L);
            O = fmaf(w, __ldcg(ps + t), O);
        }
        p.out[job * p.out_stride + h * HD + t] = __float2half_rn(O / L);
    }
    if (t == 0) p.counters[jh] = 0u;
}

}  // namespace dstream

struct DecodeStreamPlan {
    int shape;   // 0: one CTA per SM (16 consumer warps), 1: mid (8 warps), 2: many small CTAs (4 warps)
    int nsplit;  // CTAs per (job, head)
};

int ensure_decode_workspace(DeviceContext *ctx, size_t floats, size_t words, cudaStream_t stream);

// Shape and split of a launch over `pairs` (job, head) pairs of up to max_len keys, in one wave of
// CTAs. A split pair costs a merge of partial rows through global memory by the last CTA to finish
// (a chain of L2 round trips at the end of the launch), so pairs are split only when whole pairs
// would leave more than half of the SMs idle:
//   pairs <= SMs / 2       one CTA per SM, each pair split over floor(SMs / pairs) CTAs;
//   SMs / 2 < pairs <= SMs one CTA per SM, pairs whole;
//   SMs < pairs <= 4 SMs   the mid shape (up to four CTAs per SM), pairs whole: one wave, instead
//                          of a second, partial wave of one-per-SM CTAs;
//   pairs > 4 SMs          the small shape (eight CTAs per SM), pairs whole.
// Measured, 12-layer decode step at context 500-1023: 8 sequences (96 pairs) 69.6 us of attention
// with whole pairs against 135 us split in two (192 one-per-SM CTAs: a partial second wave) and
// 100 us split in three in the mid shape; 16 sequences 110.6 us in the mid shape against 127 us in
// two waves; 32 sequences (384 pairs) 140.6 us in the mid shape against 150.9 us in the small one.
DecodeStreamPlan decode_stream_plan(int max_len, long long pairs, int num_sms) {
    const int sms = num_sms > 0 ? num_sms : 148;
    DecodeStreamPlan plan{0, 1};
    if (pairs > 4LL * sms) {
        plan.shape = 2;
    } else if (pairs > sms) {
        plan.shape = 1;
    } else if (2 * pairs <= sms) {
        const long long max_n = std::max(1, (max_len + dstream::CfgFew::KPS - 1) / dstream::CfgFew::KPS);
        plan.nsplit = static_cast<int>(std::max(1LL, std::min(max_n, sms / pairs)));
    }
    return plan;
}

// CTAs per (job, head) of a launch (sizes the split workspace).
int decode_stream_splits(int max_len, long long pairs, int num_sms) {
    return decode_stream_plan(max_len, pairs, num_sms).nsplit;
}

// Sets the kernel's shared-memory attribute on the current device (once), so that a later launch
// inside a stream capture makes no configuration call.
int prepare_decode_stream() {
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_ECUDA;
    if (!ctx->decode_attr_done) {
        if (cudaFuncSetAttribute(dstream::k_decode_stream<dstream::NCW_FEW, dstream::NSTAGE_FEW>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 dstream::CfgFew::SMEM_BYTES) != cudaSuccess ||
            cudaFuncSetAttribute(dstream::k_decode_stream<dstream::NCW_MANY, dstream::NSTAGE_MANY>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 dstream::CfgMany::SMEM_BYTES) != cudaSuccess ||
            cudaFuncSetAttribute(dstream::k_decode_stream<dstream::NCW_MID, dstream::NSTAGE_MID>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 dstream::CfgMid::SMEM_BYTES) != cudaSuccess)
            return GPT2_B200_ECUDA;
        ctx->decode_attr_done = true;
    }
    return GPT2_B200_OK;
}

int launch_decode_stream(__half *out, long long out_stride, const __half *q, long long q_stride,
                         const __half *kbase, const __half *vbase, long long kv_stride,
                         const __half *const *k_ptrs, const __half *const *v_ptrs, const int *d_len,
                         int len_per_job, int len_add, int len, int max_len, int njobs, int H,
                         int maxT, cudaStream_t stream, bool pdl, bool l2_early) {
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_ECUDA;
    if (!ctx->decode_attr_done && prepare_decode_stream() != GPT2_B200_OK) return GPT2_B200_ECUDA;
    dstream::Params p;
    p.q = q;
    p.q_stride = q_stride;
    p.kbase = kbase;
    p.vbase = vbase;
    p.kv_stride = kv_stride;
    p.k_ptrs = k_ptrs;
    p.v_ptrs = v_ptrs;
    p.out = out;
    p.out_stride = out_stride;
    p.d_len = d_len;
    p.len_per_job = len_per_job;
    p.len_add = len_add;
    p.len = len;
    p.H = H;
    p.maxT = maxT;
    p.njobs = njobs;
    const DecodeStreamPlan plan = decode_stream_plan(max_len, static_cast<long long>(njobs) * H, ctx->num_sms);
    p.nsplit = plan.nsplit;
    p.scale_log2 = static_cast<float>(1.4426950408889634 / 8.0);
    p.status = ctx->status;
    p.timeout_ns = wait_timeout_ns();
    p.part = nullptr;
    p.counters = nullptr;
    if (p.nsplit > 1) {
        const size_t floats = static_cast<size_t>(njobs) * H * p.nsplit * dstream::PART_STRIDE;
        const size_t words = static_cast<size_t>(njobs) * H;
        const int rc = ensure_decode_workspace(ctx, floats, words, stream);
        if (rc != GPT2_B200_OK) return rc;
        p.part = ctx->part;
        p.counters = ctx->counters;
    }
    // At most ~40 MB requested into L2 per launch (of the 126 MB), 256 KB of K and of V per CTA.
    const long long ctas = static_cast<long long>(p.nsplit) * H * njobs;
    const long long cap = std::min(256LL << 10, (40LL << 20) / (2 * ctas)) & ~15LL;
    p.l2_early_bytes = (l2_early && pdl && d_len) ? static_cast<unsigned>(cap) : 0u;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nsplit, H, njobs);
    cfg.blockDim = dim3(plan.shape == 2 ? dstream::CfgMany::NT
                        : plan.shape == 1 ? dstream::CfgMid::NT : dstream::CfgFew::NT, 1, 1);
    cfg.dynamicSmemBytes = plan.shape == 2 ? dstream::CfgMany::SMEM_BYTES
                           : plan.shape == 1 ? dstream::CfgMid::SMEM_BYTES : dstream::CfgFew::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t err =
        plan.shape == 2 ? cudaLaunchKernelEx(&cfg, dstream::k_decode_stream<dstream::NCW_MANY, dstream::NSTAGE_MANY>, p)
        : plan.shape == 1 ? cudaLaunchKernelEx(&cfg, dstream::k_decode_stream<dstream::NCW_MID, dstream::NSTAGE_MID>, p)
                          : cudaLaunchKernelEx(&cfg, dstream::k_decode_stream<dstream::NCW_FEW, dstream::NSTAGE_FEW>, p);
    return err == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}

}  // namespace b200
