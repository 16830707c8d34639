// linear_tc.cu — the weight matmuls of a batched GPT-2 decode step on tcgen05 (sm_100a).
//
// The reference decodes one sequence at a time and computes every weight matmul as an M=1 GEMV, one
// warp per output row (k_gemv_fp16, cuda/kvcache.cu:150-170, dispatched at kvcache.cu:220-226 from
// the decode step kvcache.cu:233-269). For B sequences decoded together the same weights serve all B
// rows, so one pass over W computes the whole batch: D^T[n, b] = sum_k W[n, k] * x[b, k] with W as
// the MMA's A operand (M = 128 weight rows per tile) and the batch as its N (B rounded up to 16).
// At B = 64 the weights are read once per step for 64 tokens; the work stays bound by HBM reads
// of W, which is what this kernel is shaped for.
//
// One CTA = one 128-row tile of W and a contiguous range of 64-wide K atoms:
//   warp 0 lane 0  TMA producer: W atom (128 x 64, 128-byte swizzle) + x atom (bpad x 64) per stage;
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma (K = 16) per atom, accumulating in TMEM; each stage is
//                  released by tcgen05.commit to its "empty" mbarrier;
//   warps 0-3      epilogue: one thread per weight row (TMEM lane), tcgen05.ld of the batch columns.
// When the tiles alone would leave SMs idle, the K range of a tile is split across the CTAs of a
// thread-block cluster, CTA r owning batch columns [r*c, (r+1)*c). Small batches (padded B <= 32):
// each CTA stores its partial columns straight into the owners' receive buffers (plain distributed-
// shared-memory stores), one cluster barrier publishes them and each owner sums locally. Larger
// batches: each CTA stages its partial tile in its own shared memory, a cluster barrier publishes
// it, and the owners read their columns from the peers. Either way the ranks' partials are summed
// in rank order (deterministic) and nothing goes through global memory.
//
// Epilogues (fused, so no separate bias / GELU / residual / append launch): see lin::Epi. The
// rounding follows the reference: h = fp16(acc + bias) as k_gemv_fp16 writes it, then GELU (k_gelu,
// cuda/kernels_naive.cu:85-90) or the residual add (k_add, kernels_naive.cu:92-96) on h in fp32 with
// one more fp16 rounding. The QKV epilogue also writes the K and V columns into each sequence's
// cache at its position, which is what gpt2_kv_append_one does after the GEMV (kvcache.cu:57-65).
//
// Every wait is bounded (mbar_wait_spin: the stages land just in time, so the waiting threads poll
// rather than sleep); a timeout sets ST_LINEAR_TIMEOUT and the kernel unwinds.
// No TMA multicast.
#include <algorithm>
#include <cstring>

#include "linear.cuh"
#include "ptx.cuh"

namespace b200 {
namespace lin {

__device__ __forceinline__ float gelu_new(float v) {
    // gelu_new (tanh form): 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))).
    const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(inner));
}

// Per-sequence K/V destinations of the QKV epilogue, staged in shared memory at kernel start.
struct QkvMeta {
    __half *k[MAX_BPAD];
    __half *v[MAX_BPAD];
    int pos[MAX_BPAD];
};

// One output element of sequence b, feature n (both in range); acc includes the bias; xin is the
// residual input (EPI_RESID).
template <int EPI>
__device__ __forceinline__ void epi_elem(const Params &p, const QkvMeta *meta, int n, int b, float acc,
                                         float xin) {
    const __half h = __float2half_rn(acc);
    __half *o = p.out + static_cast<long long>(b) * p.ldo + n;
    if (EPI == EPI_GELU)
        *o = __float2half_rn(gelu_new(__half2float(h)));
    else if (EPI == EPI_RESID)
        *o = __float2half_rn(xin + __half2float(h));
    else
        *o = h;
    if (EPI == EPI_QKV && n >= p.E) {
        // K or V column: head (m >> 6), dim (m & 63) of this step's row in the sequence's cache.
        int m = n - p.E;
        const bool is_v = m >= p.E;
        if (is_v) m -= p.E;
        const int pos = meta->pos[b];
        if (pos < 0 || pos >= p.maxT) {
            atomicOr(p.status, ST_KV_BAD_POS);
            return;
        }
        (is_v ? meta->v[b] : meta->k[b])[(static_cast<long long>(m >> 6) * p.maxT + pos) * 64 +
                                         (m & 63)] = h;
    }
}

__device__ __forceinline__ void dsmem_st_v4(uint32_t cluster_saddr, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_saddr), "f"(v.x),
                 "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ float4 dsmem_ld_v4(uint32_t cluster_saddr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(cluster_saddr)
                 : "memory");
    return v;
}

template <int EPI>
__global__ void __launch_bounds__(NT, 1) k_linear_tc(const __grid_constant__ CUtensorMap tm_w,
                                                  const __grid_constant__ CUtensorMap tm_x,
                                                  const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stage_bytes = W_ATOM_BYTES + p.bpad * 128;
    // The stage ring; the pull reduction reuses it for the partial tile [bpad][128] after the MMAs.
    const int ring = max(p.nstage * stage_bytes, (p.cs > 1 && !p.push) ? p.bpad * BM * 4 : 0);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + ring);
    uint64_t *empty = full + MAX_STAGES;
    uint64_t *done = empty + MAX_STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    unsigned long long *red = reinterpret_cast<unsigned long long *>(smem + ring + 128);
    QkvMeta *meta = reinterpret_cast<QkvMeta *>(smem + ring + 128);
    // Split K, push reduction: partial columns received from every rank, [rank][128 rows][cpr4] fp32
    // (own slot too).
    float *recv = reinterpret_cast<float *>(smem + ring + 128 + p.extra_bytes);

    const int rank = static_cast<int>(cluster_rank());
    const int tile = blockIdx.y;
    const int n0 = tile * BM;
    const int a0 = (rank * p.atoms) / p.cs, a1 = ((rank + 1) * p.atoms) / p.cs;
    const int na = a1 - a0;
    // Split K: this rank reduces batch columns [my_lo, my_lo + my_w).
    const int my_lo = p.cs > 1 ? rank * p.cpr4 : 0;
    const int my_w = p.cs > 1 ? max(0, min(p.cpr4, p.bpad - my_lo)) : p.bpad;

    if (threadIdx.x == 0) {
        for (int s = 0; s < MAX_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_x);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, static_cast<uint32_t>(p.tcols));
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    // The next kernel of a chain may start launching now (it waits for this grid's completion
    // before it reads anything this grid writes).
    grid_launch_dependents();

    if (warp == 0) {
        // Producer: one W atom and one x atom per stage. The weights do not depend on the previous
        // kernel, so the first ring of W atoms is requested before waiting for it (programmatic
        // dependent launch: this overlaps the previous kernel's tail); x follows the wait. The whole
        // warp runs the loop (warp-uniform operands); one elected lane issues the copies.
        const bool leader = elect_one();
        const int pre = min(na, p.nstage);
        if (leader) {
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&full[i], static_cast<uint32_t>(stage_bytes));
                tma_load_2d(smem + i * stage_bytes, &tm_w, &full[i], (a0 + i) * KA, n0);
            }
        }
        grid_dependency_wait();
        if (leader)
            for (int i = 0; i < pre; ++i)
                tma_load_2d(smem + i * stage_bytes + W_ATOM_BYTES, &tm_x, &full[i], (a0 + i) * KA, 0);
        for (int i = pre; i < na; ++i) {
            const int s = i % p.nstage;
            const bool ok = mbar_wait_spin(&empty[s], ((i / p.nstage) - 1) & 1, p.timeout_ns);
            if (!__all_sync(0xffffffffu, ok)) {
                if (leader) atomicOr(p.status, ST_LINEAR_TIMEOUT);
                break;
            }
            if (leader) {
                uint8_t *st = smem + s * stage_bytes;
                mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(stage_bytes));
                tma_load_2d(st, &tm_w, &full[s], (a0 + i) * KA, n0);
                tma_load_2d(st + W_ATOM_BYTES, &tm_x, &full[s], (a0 + i) * KA, 0);
            }
            __syncwarp();
        }
    } else {
        grid_dependency_wait();
    }
    if (warp == 1) {
        // MMA issuer: the whole warp waits (warp-uniform descriptors, kept in uniform registers);
        // one elected lane issues. Descriptors are built once and advanced by 32-bit adds.
        const bool leader = elect_one();
        const uint32_t idesc = idesc_f16_f32(BM, p.bpad, 0, 0);
        const uint64_t dw0 = sdesc_sw128(smem_u32(smem), 16, 1024);
        const uint64_t dx0 = sdesc_sw128(smem_u32(smem + W_ATOM_BYTES), 16, 1024);
        const uint32_t w_lo = static_cast<uint32_t>(dw0), w_hi = static_cast<uint32_t>(dw0 >> 32);
        const uint32_t x_lo = static_cast<uint32_t>(dx0), x_hi = static_cast<uint32_t>(dx0 >> 32);
        for (int i = 0; i < na; ++i) {
            const int s = i % p.nstage;
            const bool ok = mbar_wait_spin(&full[s], (i / p.nstage) & 1, p.timeout_ns);
            if (!__all_sync(0xffffffffu, ok)) {
                if (leader) atomicOr(p.status, ST_LINEAR_TIMEOUT);
                break;
            }
            tc_fence_after();
            const uint32_t off = static_cast<uint32_t>((s * stage_bytes) >> 4);
            if (leader) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_f16_ss_lohi(tbase, w_lo + off + 2 * kk, w_hi, x_lo + off + 2 * kk, x_hi, idesc,
                                     (i > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (leader) umma_commit(done);  // arrives once every MMA issued above has completed
    }
    __syncwarp();

    // Inputs of the epilogue that do not depend on the accumulator, fetched while the MMAs run.
    const int row = warp * 32 + lane;  // TMEM lane = weight row within the tile
    const int n = n0 + row;
    const bool n_ok = n < p.N;
    const float bias_n = (p.bias != nullptr && n_ok) ? __half2float(p.bias[n]) : 0.0f;
    if (EPI == EPI_QKV) {
        for (int b = threadIdx.x; b < p.B; b += NT) {
            meta->pos[b] = p.d_pos[b];
            meta->k[b] = p.k_dst[b];
            meta->v[b] = p.v_dst[b];
        }
    }
    // Residual inputs of this thread's first 16 columns (whole K: columns 0..15; split K: this
    // rank's columns), prefetched.
    constexpr int XPRE = 16;
    float xin[XPRE];
#pragma unroll
    for (int j = 0; j < XPRE; ++j)
        xin[j] = (EPI == EPI_RESID && n_ok && j < my_w && my_lo + j < p.B)
                     ? __half2float(p.out[static_cast<long long>(my_lo + j) * p.ldo + n])
                     : 0.0f;
    if (EPI == EPI_QKV) __syncthreads();

    const bool have = mbar_wait_spin(done, 0, p.timeout_ns);
    if (!have && threadIdx.x == 0) atomicOr(p.status, ST_LINEAR_TIMEOUT);
    tc_fence_after();
    const uint32_t trow = tbase + (static_cast<uint32_t>(warp * 32) << 16);

    if (EPI == EPI_HEAD) {
        // Logits are fp16(acc); per batch column, the warp's best (value, index) key, then the CTA's.
        for (int c = 0; c < p.bpad; c += 16) {
            uint32_t r[16];
            tmem_ld16(trow + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int b = c + j;
                const __half h = __float2half_rn(__uint_as_float(r[j]) + bias_n);
                if (p.out != nullptr && n_ok && b < p.B)
                    p.out[static_cast<long long>(b) * p.ldo + n] = h;
                const unsigned long long key =
                    (n_ok && have) ? argmax_key(__half2float(h), static_cast<unsigned>(n)) : 0ull;
                const unsigned hi = static_cast<unsigned>(key >> 32);
                const unsigned mhi = __reduce_max_sync(0xFFFFFFFFu, hi);
                const unsigned mlo = __reduce_max_sync(
                    0xFFFFFFFFu, hi == mhi ? static_cast<unsigned>(key & 0xFFFFFFFFull) : 0u);
                if (lane == 0)
                    red[warp * p.bpad + b] = (static_cast<unsigned long long>(mhi) << 32) | mlo;
            }
        }
        __syncthreads();
        for (int b = threadIdx.x; b < p.B; b += NT) {
            unsigned long long k = red[b];
#pragma unroll
            for (int w = 1; w < 4; ++w) k = max(k, red[w * p.bpad + b]);
            p.amax[static_cast<long long>(b) * p.n_tiles + tile] = k;
        }
    } else if (p.cs == 1) {
        // Whole K in this CTA: straight from TMEM, 16 batch columns at a time.
        for (int c = 0; c < p.bpad; c += 16) {
            uint32_t r[16];
            tmem_ld16(trow + c, r);
            float xc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int b = c + j;
                xc[j] = c < XPRE ? xin[j]
                                 : ((EPI == EPI_RESID && n_ok && b < p.B)
                                        ? __half2float(p.out[static_cast<long long>(b) * p.ldo + n])
                                        : 0.0f);
            }
            tmem_wait_ld();
            if (have && n_ok) {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (c + j < p.B)
                        epi_elem<EPI>(p, meta, n, c + j, __uint_as_float(r[j]) + bias_n, xc[j]);
            }
        }
    } else {
        if (p.push) {
            // Split K: every rank owns the batch columns [r*cpr4, (r+1)*cpr4). Each CTA stores row `row`
            // of its partial for those columns straight into the owner's receive slot for this rank
            // (recv[rank][row][..], plain distributed-shared-memory stores; its own columns locally).
            // One cluster barrier (release / acquire) publishes every store; each owner then sums its
            // columns over the ranks in rank order (deterministic) from its own shared memory. Nothing
            // is read remotely, so no CTA has to wait for its peers again before exiting.
            const uint32_t recv_s = smem_u32(recv);
            for (int c = 0; c < p.bpad; c += 16) {
                uint32_t r[16];
                tmem_ld16(trow + c, r);
                tmem_wait_ld();
    #pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const int col = c + 4 * g;
                    const int q = col / p.cpr4;
                    const float4 v = make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                                                 __uint_as_float(r[4 * g + 2]),
                                                 __uint_as_float(r[4 * g + 3]));
                    const uint32_t off =
                        static_cast<uint32_t>(((rank * BM + row) * p.cpr4 + (col - q * p.cpr4)) * 4);
                    if (q == rank)
                        *reinterpret_cast<float4 *>(reinterpret_cast<uint8_t *>(recv) + off) = v;
                    else
                        dsmem_st_v4(dsmem_addr(recv_s + off, static_cast<uint32_t>(q)), v);
                }
            }
            cluster_sync_all();
            if (have && n_ok) {
    #pragma unroll
                for (int j = 0; j < XPRE; j += 4) {
                    if (j >= my_w) break;
                    float a4[4] = {bias_n, bias_n, bias_n, bias_n};
                    for (int q = 0; q < p.cs; ++q) {
                        const float4 v = *reinterpret_cast<const float4 *>(recv + (q * BM + row) * p.cpr4 + j);
                        a4[0] += v.x;
                        a4[1] += v.y;
                        a4[2] += v.z;
                        a4[3] += v.w;
                    }
    #pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (my_lo + j + i < p.B) epi_elem<EPI>(p, meta, n, my_lo + j + i, a4[i], xin[j + i]);
                }
                for (int j = XPRE; j < my_w; j += 4) {
                    float a4[4] = {bias_n, bias_n, bias_n, bias_n};
                    for (int q = 0; q < p.cs; ++q) {
                        const float4 v = *reinterpret_cast<const float4 *>(recv + (q * BM + row) * p.cpr4 + j);
                        a4[0] += v.x;
                        a4[1] += v.y;
                        a4[2] += v.z;
                        a4[3] += v.w;
                    }
    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int b = my_lo + j + i;
                        if (b >= p.B) break;
                        const float x = EPI == EPI_RESID
                                            ? __half2float(p.out[static_cast<long long>(b) * p.ldo + n])
                                            : 0.0f;
                        epi_elem<EPI>(p, meta, n, b, a4[i], x);
                    }
                }
            }
        } else {
            // Split K: publish this CTA's partial tile in shared memory as [bpad][128] fp32 (column b's
            // 128 rows at b*128), then rank r reduces its columns [my_lo, my_lo + my_w) over all ranks
            // in rank order through distributed shared memory (deterministic). Thread t owns rows
            // 4*(t % 32) .. +3 and the columns my_lo + t/32, +4, ...; two columns per pass, every load
            // of a pass issued before its first use.
            float *part = reinterpret_cast<float *>(smem);
            for (int c = 0; c < p.bpad; c += 16) {
                uint32_t r[16];
                tmem_ld16(trow + c, r);
                tmem_wait_ld();
    #pragma unroll
                for (int j = 0; j < 16; ++j) part[(c + j) * BM + row] = __uint_as_float(r[j]);
            }
            cluster_sync_all();
            const int q4 = (threadIdx.x & 31) * 4;
            const int nq = n0 + q4;
            float bq[4];
    #pragma unroll
            for (int i = 0; i < 4; ++i)
                bq[i] = (p.bias != nullptr && nq + i < p.N) ? __half2float(p.bias[nq + i]) : 0.0f;
            const uint32_t base = smem_u32(part) + static_cast<uint32_t>(q4 * 4);
            const int b1 = min(my_lo + my_w, p.B);
            constexpr int CG = 2;
            for (int b = my_lo + (threadIdx.x >> 5); b < b1; b += 4 * CG) {
                float xq[CG][4];
                float4 t[CG][MAX_CLUSTER];
    #pragma unroll
                for (int g = 0; g < CG; ++g) {
                    const int bb = b + 4 * g;
                    const bool valid = bb < b1;
    #pragma unroll
                    for (int i = 0; i < 4; ++i)
                        xq[g][i] = (EPI == EPI_RESID && valid && nq + i < p.N)
                                       ? __half2float(p.out[static_cast<long long>(bb) * p.ldo + nq + i])
                                       : 0.0f;
                    const uint32_t off = base + static_cast<uint32_t>(bb * BM * 4);
    #pragma unroll
                    for (int q = 0; q < MAX_CLUSTER; ++q)
                        t[g][q] = (valid && q < p.cs)
                                      ? dsmem_ld_v4(dsmem_addr(off, static_cast<uint32_t>(q)))
                                      : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
    #pragma unroll
                for (int g = 0; g < CG; ++g) {
                    const int bb = b + 4 * g;
                    if (bb >= b1 || !have) continue;
                    float acc[4] = {bq[0], bq[1], bq[2], bq[3]};
    #pragma unroll
                    for (int q = 0; q < MAX_CLUSTER; ++q) {
                        acc[0] += t[g][q].x;
                        acc[1] += t[g][q].y;
                        acc[2] += t[g][q].z;
                        acc[3] += t[g][q].w;
                    }
    #pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (nq + i < p.N) epi_elem<EPI>(p, meta, nq + i, bb, acc[i], xq[g][i]);
                }
            }
            cluster_sync_all();  // peers may still be reading this CTA's partial tile
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tbase, static_cast<uint32_t>(p.tcols));
}

// ---------------------------------------------------------------- host side
namespace {

// 2-D fp16 map over rows x cols (row stride ld elements), box 64 x box_rows, 128-byte swizzle.
// Rows past `rows` read as zero.
bool encode_rows(CUtensorMap *m, const __half *ptr, long long rows, int cols, long long ld,
                 int box_rows) {
    EncodeTiledFn fn = tensor_map_encoder();
    if (!fn) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(KA), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(ptr), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI>
void *kernel_of() {
    return reinterpret_cast<void *>(&k_linear_tc<EPI>);
}

void *kernel_for(int epi) {
    switch (epi) {
        case EPI_STORE: return kernel_of<EPI_STORE>();
        case EPI_GELU: return kernel_of<EPI_GELU>();
        case EPI_RESID: return kernel_of<EPI_RESID>();
        case EPI_QKV: return kernel_of<EPI_QKV>();
        case EPI_HEAD: return kernel_of<EPI_HEAD>();
        default: return nullptr;
    }
}

}  // namespace

int plan_linear(Plan *pl, int epi, const __half *W, int N, int K, const __half *X, long long ldx,
                int B, const __half *bias, __half *out, long long ldo, int cs, int num_sms) {
    if (!pl || !W || !X || N < 1 || K < KA || (K % KA) != 0 || B < 1 || B > MAX_BPAD)
        return GPT2_B200_EINVAL;
    if (epi < EPI_STORE || epi > EPI_HEAD) return GPT2_B200_EINVAL;
    if (epi != EPI_HEAD && !out) return GPT2_B200_EINVAL;
    if ((reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(X) & 15) ||
        (ldx & 7) || ldx < K)
        return GPT2_B200_EINVAL;
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_ECUDA;
    std::memset(pl, 0, sizeof(*pl));
    Params &p = pl->p;
    p.N = N;
    p.K = K;
    p.B = B;
    p.bpad = (B + 15) / 16 * 16;
    p.atoms = K / KA;
    p.n_tiles = (N + BM - 1) / BM;
    (void)num_sms;
    p.tcols = 32;
    while (p.tcols < p.bpad) p.tcols *= 2;
    p.bias = bias;
    p.out = out;
    p.ldo = ldo;
    p.status = ctx->status;
    p.timeout_ns = wait_timeout_ns();
    pl->epi = epi;
    if (!encode_rows(&pl->tm_w, W, N, K, K, BM)) return GPT2_B200_EDEVICE;
    if (!encode_rows(&pl->tm_x, X, B, K, ldx, p.bpad)) return GPT2_B200_EDEVICE;
    const int stage_bytes = W_ATOM_BYTES + p.bpad * 128;
    p.extra_bytes = epi == EPI_HEAD  ? 4 * p.bpad * 8
                    : epi == EPI_QKV ? static_cast<int>((sizeof(QkvMeta) + 15) / 16 * 16)
                                     : 0;
    int sm_smem = 0, reserved = 0;
    if (cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, ctx->device) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, ctx->device) !=
            cudaSuccess)
        return GPT2_B200_ECUDA;
    // Shared memory for a split of c: the ring (reused for the split-K partial tile), the barriers
    // and the epilogue's extra; the ring shrinks until it fits. Never more CTAs on an SM than its
    // 512 TMEM columns hold (a CTA whose allocation waited on another cluster's CTA could wait in
    // a cycle), so shared memory is padded to cap the CTAs per SM.
    const size_t limit = 227 * 1024;
    auto size_for = [&](int c, int *nstage) -> size_t {
        const int cpr4 = c > 1 ? ((p.bpad + c - 1) / c + 3) / 4 * 4 : p.bpad;
        const bool push = c > 1 && p.bpad <= PUSH_MAX_BPAD;
        const size_t recv = push ? static_cast<size_t>(c) * BM * cpr4 * 4 : 0;
        const size_t fixed = 1024 + 128 + p.extra_bytes + recv;
        // The head (393 tiles of the vocabulary, no split) streams through a 2-atom ring: four CTAs
        // fit per SM and all tiles run in one wave (20.2 -> 15.6 us for the 77 MB at B = 64).
        int ns = std::min(epi == EPI_HEAD ? HEAD_STAGES : MAX_STAGES, (p.atoms + c - 1) / c);
        while (ns > 1 && fixed + static_cast<size_t>(ns) * stage_bytes > limit) --ns;
        *nstage = ns;
        const size_t ring = std::max(static_cast<size_t>(ns) * stage_bytes,
                                     (c > 1 && !push) ? static_cast<size_t>(p.bpad) * BM * 4 : size_t{0});
        const int max_ctas = 512 / p.tcols;
        const size_t min_smem = static_cast<size_t>(sm_smem / (max_ctas + 1) - reserved + 1);
        return std::max(fixed + ring, min_smem);
    };
    void *fn = kernel_for(epi);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(limit)) != cudaSuccess)
        return GPT2_B200_ECUDA;
    if (epi == EPI_HEAD) cs = 1;  // the argmax keys are per tile; the head has tiles to spare
    if (cs <= 0) {
        // The widest split whose clusters all fit on the GPU at once (one wave): the K ranges
        // shrink with the split, but a second wave of clusters costs a whole kernel latency.
        // Without such a split, about one CTA per SM.
        const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
        const int fallback = std::max(1, sms / p.n_tiles);
        cs = 0;
        for (int c = std::min(MAX_CLUSTER, p.atoms); c >= 2; --c) {
            int ns = 0;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(c, p.n_tiles, 1);
            cfg.blockDim = dim3(NT, 1, 1);
            cfg.dynamicSmemBytes = size_for(c, &ns);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = static_cast<unsigned>(c);
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int active = 0;
            if (cudaOccupancyMaxActiveClusters(&active, fn, &cfg) != cudaSuccess) {
                cudaGetLastError();
                continue;
            }
            if (p.n_tiles <= active) {
                cs = c;
                break;
            }
        }
        if (cs == 0) cs = fallback;
    }
    cs = std::max(1, std::min(cs, std::min(MAX_CLUSTER, p.atoms)));
    p.cs = cs;
    p.cpr4 = cs > 1 ? ((p.bpad + cs - 1) / cs + 3) / 4 * 4 : p.bpad;
    p.push = cs > 1 && p.bpad <= PUSH_MAX_BPAD;
    pl->smem = size_for(cs, &p.nstage);
    if (pl->smem > limit) return GPT2_B200_EINVAL;
    pl->grid = dim3(cs, p.n_tiles, 1);
    return GPT2_B200_OK;
}

int prepare_linear(const Plan &pl) {
    void *fn = kernel_for(pl.epi);
    if (!fn) return GPT2_B200_EINVAL;
    // The attribute is per device; raise it once per (thread, device, epilogue) to the largest
    // plan seen.
    static thread_local int set_smem[64][EPI_HEAD + 1] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GPT2_B200_ECUDA;
    int &have = set_smem[dev][pl.epi];
    if (have < static_cast<int>(pl.smem)) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(pl.smem)) != cudaSuccess)
            return GPT2_B200_ECUDA;
        have = static_cast<int>(pl.smem);
    }
    return GPT2_B200_OK;
}

int launch_linear(const Plan &pl, cudaStream_t stream) {
    const int rc = prepare_linear(pl);
    if (rc != GPT2_B200_OK) return rc;
    void *fn = kernel_for(pl.epi);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = pl.grid;
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pl.pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (pl.p.cs > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = static_cast<unsigned>(pl.p.cs);
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    void *args[3] = {const_cast<CUtensorMap *>(&pl.tm_w), const_cast<CUtensorMap *>(&pl.tm_x),
                     const_cast<Params *>(&pl.p)};
    if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return GPT2_B200_ECUDA;
    return GPT2_B200_OK;
}

}  // namespace lin
}  // namespace b200
