// prefill_tc.cu — causal flash-attention prefill on the B200 tensor cores (tcgen05 + TMEM + TMA).
//
// Computes what the reference's k_attention_flash computes (cuda/kernels_fused.cu:58-140): for every
// head h of qkv[T, 3E] (q | k | v, head h at h*64), att[i, h*64:(h+1)*64] = sum_{j<=i} softmax_j(q_i.k_j
// / 8) v_j, fp16 in, fp32 accumulation, fp16 out. The reference runs one warp per query on CUDA cores
// with 32-key tiles; here one CTA owns a 128-query tile of one head and streams 128-key tiles:
//
//   warp 0  (1 thread)  TMA producer: Q tile once, then K_j / V_j tiles (128 x 64 fp16, 128-byte
//                       swizzle) straight out of the packed qkv rows into a 2-stage ring.
//   warp 1  (1 thread)  MMA issuer: S = Q K_j^T into TMEM (M128 N128 K64, 4 x tcgen05.mma K16), and
//                       O += P_j V_j into TMEM (M128 N64 K128, 8 x tcgen05.mma K16). S_{j+1} is issued
//                       as soon as the softmax warps have read S_j, so it overlaps their exp work.
//   warps 2-5 (128 thr) softmax: thread r owns query row r = TMEM lane r. Reads S_j (tcgen05.ld),
//                       applies the causal mask on the diagonal tile only, keeps a running max m and
//                       sum l in the log2 domain (scale folded into one FFMA), writes P_j = 2^(s-m) as
//                       fp16 into shared memory in the MMA's swizzled K-major layout, and rescales O in
//                       TMEM only when the running max grows by more than 2^8 (otherwise the stale max
//                       is kept for both l and O, which leaves the result unchanged). Epilogue: O / l
//                       -> fp16 -> att.
//
// TMEM: 256 columns per CTA (S: 128 fp32 columns, O: 64), so two CTAs share an SM (smem 112 KB each)
// and the tensor core alternates between them. Tiles are scheduled heaviest-first (the last query
// tile of a sequence has the most keys). No cluster, no multicast. Every mbarrier wait is bounded.
#include <cmath>
#include <cstdio>

#include "common.cuh"
#include "ptx.cuh"

namespace b200 {
namespace prefill {

constexpr int BM = 128;  // query rows per tile = TMEM lanes
constexpr int BN = 128;  // keys per KV tile
constexpr int HD = 64;   // head dim
constexpr int NSTAGE = 2;
constexpr int TILE_BYTES = BM * HD * 2;  // 16 KB: 128 rows x 128 B
constexpr int P_BLOCK_BYTES = BM * 64 * 2;  // P is two 64-key column blocks of 16 KB
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE_BYTES;
constexpr int OFF_V = OFF_K + NSTAGE * TILE_BYTES;
constexpr int OFF_P = OFF_V + NSTAGE * TILE_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * P_BLOCK_BYTES;
constexpr int SMEM_BYTES = OFF_BAR + 128;
constexpr int NTHREADS = 192;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t TCOL_S = 0;
constexpr uint32_t TCOL_O = 128;
constexpr uint32_t IDESC_S = idesc_f16_f32(BM, BN, 0, 0);  // Q K-major, K K-major
constexpr uint32_t IDESC_O = idesc_f16_f32(BM, HD, 0, 1);  // P K-major, V MN-major
constexpr float RESCALE_THRESHOLD = 8.0f;                  // log2 units: P stays <= 2^8

struct __align__(8) Bars {
    uint64_t q_full;
    uint64_t k_full[NSTAGE];
    uint64_t v_full[NSTAGE];
    uint64_t kv_empty[NSTAGE];
    uint64_t s_full;
    uint64_t s_free;
    uint64_t p_full;
    uint64_t o_done;
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Bars) <= 128, "barrier block");

struct Params {
    __half *att;
    long long att_seq_stride;  // elements between sequences of att
    int T, H, E, B;
    int n_qtiles;
    float scale_log2;          // log2(e) / sqrt(D)
    unsigned *status;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ void raise_abort(Bars *bars, unsigned *status, unsigned bit) {
    atomicOr(status, bit);
    *reinterpret_cast<volatile int *>(&bars->abort) = 1;
}

__device__ __forceinline__ bool aborted(Bars *bars) {
    return *reinterpret_cast<volatile int *>(&bars->abort) != 0;
}

// ------------------------------------------------------------------ producer (one thread)
__device__ void run_producer(const CUtensorMap *tm, uint8_t *smem, Bars *bars, const Params &p,
                             int b, int h, int qt, int nk) {
    const unsigned long long to = p.timeout_ns;
    mbar_arrive_expect_tx(&bars->q_full, TILE_BYTES);
    tma_load_3d(smem + OFF_Q, tm, &bars->q_full, h * HD, qt * BM, b);
    int last_issue[NSTAGE] = {-1, -1};
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
        const int st = j % NSTAGE;
        if (j >= NSTAGE) {
            ok = mbar_wait(&bars->kv_empty[st], ((j / NSTAGE) - 1) & 1, to);
            if (!ok) break;
        }
        if (aborted(bars)) break;
        mbar_arrive_expect_tx(&bars->k_full[st], TILE_BYTES);
        tma_load_3d(smem + OFF_K + st * TILE_BYTES, tm, &bars->k_full[st], p.E + h * HD, j * BN, b);
        mbar_arrive_expect_tx(&bars->v_full[st], TILE_BYTES);
        tma_load_3d(smem + OFF_V + st * TILE_BYTES, tm, &bars->v_full[st], 2 * p.E + h * HD,
                    j * BN, b);
        last_issue[st] = j;
    }
    if (!ok) raise_abort(bars, p.status, ST_PREFILL_LOAD_TIMEOUT);
    // Teardown guard: every copy this thread issued must have landed before the CTA exits.
    bool drained = mbar_wait(&bars->q_full, 0, to);
    for (int st = 0; st < NSTAGE; ++st) {
        if (last_issue[st] < 0) continue;
        const uint32_t par = (last_issue[st] / NSTAGE) & 1;
        drained = mbar_wait(&bars->k_full[st], par, to) && drained;
        drained = mbar_wait(&bars->v_full[st], par, to) && drained;
    }
    if (!drained) atomicOr(p.status, ST_PREFILL_DRAIN_TIMEOUT);
}

// ------------------------------------------------------------------ MMA issuer (one thread)
__device__ void run_mma(uint8_t *smem, Bars *bars, const Params &p, uint32_t tbase, int nk) {
    const unsigned long long to = p.timeout_ns;
    const uint32_t tS = tbase + TCOL_S, tO = tbase + TCOL_O;
    const uint32_t aQ = smem_u32(smem + OFF_Q);
    const uint32_t aK = smem_u32(smem + OFF_K);
    const uint32_t aV = smem_u32(smem + OFF_V);
    const uint32_t aP = smem_u32(smem + OFF_P);

    auto issue_qk = [&](int st) {
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t da = sdesc_sw128(aQ + kk * 32, 16, 1024);
            const uint64_t db = sdesc_sw128(aK + st * TILE_BYTES + kk * 32, 16, 1024);
            umma_f16_ss(tS, da, db, IDESC_S, kk > 0 ? 1u : 0u);
        }
    };
    auto issue_pv = [&](int st, bool first) {
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t da = sdesc_sw128(aP + (kk >> 2) * P_BLOCK_BYTES + (kk & 3) * 32, 16, 1024);
            const uint64_t db = sdesc_sw128(aV + st * TILE_BYTES + kk * 2048, TILE_BYTES, 1024);
            umma_f16_ss(tO, da, db, IDESC_O, (first && kk == 0) ? 0u : 1u);
        }
    };

    bool ok = mbar_wait(&bars->q_full, 0, to) && mbar_wait(&bars->k_full[0], 0, to);
    if (ok) {
        tc_fence_after();
        issue_qk(0);
        umma_commit(&bars->s_full);
    }
    for (int j = 0; ok && j < nk; ++j) {
        if (j + 1 < nk) {
            const int st1 = (j + 1) % NSTAGE;
            ok = mbar_wait(&bars->k_full[st1], ((j + 1) / NSTAGE) & 1, to) &&
                 mbar_wait(&bars->s_free, j & 1, to);
            if (!ok) break;
            tc_fence_after();
            issue_qk(st1);
            umma_commit(&bars->s_full);
        }
        const int st = j % NSTAGE;
        ok = mbar_wait(&bars->p_full, j & 1, to) && mbar_wait(&bars->v_full[st], (j / NSTAGE) & 1, to);
        if (!ok) break;
        tc_fence_after();
        issue_pv(st, j == 0);
        umma_commit(&bars->o_done);
        umma_commit(&bars->kv_empty[st]);
    }
    if (!ok) raise_abort(bars, p.status, ST_PREFILL_MMA_TIMEOUT);
    // Teardown guard: all MMAs issued by this thread complete before TMEM is released.
    umma_commit(&bars->drain);
    if (!mbar_wait(&bars->drain, 0, to)) atomicOr(p.status, ST_PREFILL_DRAIN_TIMEOUT);
}

// ------------------------------------------------------------------ softmax + epilogue (4 warps)
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity,
                                          unsigned long long to) {
    const bool ok = mbar_wait(bar, parity, to);
    return __all_sync(0xffffffffu, ok);
}

__device__ void run_softmax(uint8_t *smem, Bars *bars, const Params &p, uint32_t tbase, int warp,
                            int lane, int b, int h, int qt, int nk) {
    const unsigned long long to = p.timeout_ns;
    const int quarter = warp & 3;              // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;         // query row within the tile
    const uint32_t tl = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t tS = tl + TCOL_S, tO = tl + TCOL_O;
    const float c = p.scale_log2;
    uint8_t *sP = smem + OFF_P;

    float m_used = -INFINITY;  // running max (log2 units) used for the exponentials
    float l = 0.f;             // running sum of exponentials
    bool ok = true;

    for (int j = 0; j < nk; ++j) {
        ok = warp_wait(&bars->s_full, j & 1, to);
        if (!ok) break;
        tc_fence_after();
        float x[BN];
#pragma unroll
        for (int cb = 0; cb < BN / 32; ++cb) {
            uint32_t v[32];
            tmem_ld32(tS + cb * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) x[cb * 32 + i] = __uint_as_float(v[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->s_free);

        if (j == nk - 1) {  // diagonal tile (BM == BN): key c of this tile is visible iff c <= r
#pragma unroll
            for (int i = 0; i < BN; ++i)
                if (i > r) x[i] = -INFINITY;
        }
        float pm[8];  // 8 independent partial maxima (no 127-long dependency chain)
#pragma unroll
        for (int k = 0; k < 8; ++k) pm[k] = x[k];
#pragma unroll
        for (int i = 8; i < BN; ++i) pm[i & 7] = fmaxf(pm[i & 7], x[i]);
        const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                               fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        const float mt = mx * c;
        float alpha = 1.f;
        bool resc = false;
        if (mt > m_used + RESCALE_THRESHOLD) {
            alpha = ex2_approx(m_used - mt);  // 0 on the first tile (m_used = -inf)
            m_used = mt;
            l *= alpha;
            resc = true;
        }
        const float neg_m = -m_used;
        uint32_t pk[BN / 2];
        // The row sum adds the fp16-ROUNDED p values (the ones the PV MMA consumes), so numerator
        // and denominator see the same weights; 8 independent partial sums keep the adds parallel.
        float ps[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) ps[k] = 0.f;
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) {
            const float p0 = ex2_approx(fmaf(x[2 * i], c, neg_m));
            const float p1 = ex2_approx(fmaf(x[2 * i + 1], c, neg_m));
            pk[i] = pack_half2(p0, p1);
            ps[(2 * i) & 7] = add_f16lo_f32(pk[i], ps[(2 * i) & 7]);
            ps[(2 * i + 1) & 7] = add_f16hi_f32(pk[i], ps[(2 * i + 1) & 7]);
        }
        l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));

        if (j > 0) {  // PV_{j-1} must be done: it reads the P buffer and writes O
            ok = warp_wait(&bars->o_done, (j - 1) & 1, to);
            if (!ok) break;
            tc_fence_after();
        }
        // P row r -> two K-major SW128 blocks (keys 0-63, 64-127); 16-byte chunk g of the row lands
        // at chunk position (g ^ (r & 7)) of its 128-byte row, as TMA would have placed it.
#pragma unroll
        for (int g = 0; g < BN / 8; ++g) {
            uint8_t *dst = sP + (g >> 3) * P_BLOCK_BYTES + r * 128 + (((g & 7) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4 *>(dst) =
                make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
        }
        if (j > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll
            for (int cb = 0; cb < HD / 32; ++cb) {
                uint32_t v[32];
                tmem_ld32(tO + cb * 32, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                tmem_st32(tO + cb * 32, v);
            }
            tmem_wait_st();
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full);
    }
    if (!ok) {
        raise_abort(bars, p.status, ST_PREFILL_SOFTMAX_TIMEOUT);
        return;
    }
    ok = warp_wait(&bars->o_done, (nk - 1) & 1, to);
    if (!ok) {
        raise_abort(bars, p.status, ST_PREFILL_SOFTMAX_TIMEOUT);
        return;
    }
    tc_fence_after();
    const float inv_l = 1.f / l;
    const int row = qt * BM + r;
    __half *dst = p.att + static_cast<long long>(b) * p.att_seq_stride +
                  static_cast<long long>(row) * p.E + h * HD;
#pragma unroll
    for (int cb = 0; cb < HD / 32; ++cb) {
        uint32_t v[32];
        tmem_ld32(tO + cb * 32, v);
        tmem_wait_ld();
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
            o[i] = pack_half2(__uint_as_float(v[2 * i]) * inv_l, __uint_as_float(v[2 * i + 1]) * inv_l);
        if (row < p.T) {
            uint4 *d4 = reinterpret_cast<uint4 *>(dst + cb * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) d4[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        }
    }
}

__global__ void __launch_bounds__(NTHREADS, 2)
    k_flash_prefill_tc(const __grid_constant__ CUtensorMap tm_qkv, const Params p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    Bars *bars = reinterpret_cast<Bars *>(smem + OFF_BAR);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Heaviest tiles first: item i -> query tile (n_qtiles-1 - i / (H*B)), then head, then sequence.
    const int per = p.H * p.B;
    const int item = blockIdx.x;
    const int qt = p.n_qtiles - 1 - item / per;
    const int rem = item % per;
    const int h = rem % p.H;
    const int b = rem / p.H;
    const int nk = qt + 1;  // causal: KV tiles 0..qt

    if ((smem_u32(smem) & 1023u) != 0) {  // SW128 tiles need 1024-byte alignment; uniform exit
        if (threadIdx.x == 0) atomicOr(p.status, ST_PREFILL_SMEM_ALIGN);
        return;
    }
    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&bars->k_full[s], 1);
            mbar_init(&bars->v_full[s], 1);
            mbar_init(&bars->kv_empty[s], 1);
        }
        mbar_init(&bars->s_full, 1);
        mbar_init(&bars->s_free, 4);
        mbar_init(&bars->p_full, 4);
        mbar_init(&bars->o_done, 1);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_qkv);
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) run_producer(&tm_qkv, smem, bars, p, b, h, qt, nk);
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) run_mma(smem, bars, p, tbase, nk);
        __syncwarp();
    } else {
        run_softmax(smem, bars, p, tbase, warp, lane, b, h, qt, nk);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

}  // namespace prefill

// Launches the batched causal prefill. Arguments are validated by the caller (api.cu).
int launch_prefill(__half *att, const __half *qkv, int B, int T, int E, int H,
                   long long qkv_seq_stride, long long att_seq_stride, cudaStream_t stream) {
    using namespace prefill;
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_ECUDA;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return GPT2_B200_EDEVICE;
    if (!ctx->prefill_attr_done) {
        if (cudaFuncSetAttribute(k_flash_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SMEM_BYTES) != cudaSuccess)
            return GPT2_B200_ECUDA;
        cudaFuncSetAttribute(k_flash_prefill_tc, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
        ctx->prefill_attr_done = true;
    }
    CUtensorMap tm;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(3 * E), static_cast<cuuint64_t>(T),
                                static_cast<cuuint64_t>(B)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(3 * E) * 2,
                                   static_cast<cuuint64_t>(qkv_seq_stride) * 2};
    const cuuint32_t box[3] = {HD, BM, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult cr = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half *>(qkv), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return GPT2_B200_EINVAL;

    Params p;
    p.att = att;
    p.att_seq_stride = att_seq_stride;
    p.T = T;
    p.H = H;
    p.E = E;
    p.B = B;
    p.n_qtiles = (T + BM - 1) / BM;
    p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(HD)));
    p.status = ctx->status;
    p.timeout_ns = wait_timeout_ns();
    const long long grid = static_cast<long long>(p.n_qtiles) * H * B;
    if (grid <= 0) return GPT2_B200_OK;
    if (grid > 0x7fffffffLL) return GPT2_B200_EINVAL;
    k_flash_prefill_tc<<<static_cast<unsigned>(grid), NTHREADS, SMEM_BYTES, stream>>>(tm, p);
    return cudaGetLastError() == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}

}  // namespace b200
