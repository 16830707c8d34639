// prefill_tc.cu — causal flash-attention prefill on the B200 tensor cores (tcgen05 + TMEM + TMA).
//
// Computes what the reference's k_attention_flash computes (cuda/kernels_fused.cu:58-140): for every
// head h of qkv[T, 3E] (q | k | v, head h at h*64), att[i, h*64:(h+1)*64] = sum_{j<=i} softmax_j(q_i.k_j
// / 8) v_j, fp16 in, fp32 accumulation, fp16 out. The reference runs one warp per query on CUDA cores
// with 32-key tiles.
//
// Here a work item is a PAIR of 128-query tiles (A = tile 2p, B = tile 2p+1) of one head of one
// sequence, processed against 128-key tiles 0..2p+1 (A stops at its diagonal tile 2p). Each K/V tile
// is loaded once into shared memory and used by both query tiles, which halves the K/V traffic per
// FLOP. The kernel is persistent: one CTA per SM loops over its items (heavy and light pairs in a
// snake order), with TMEM and barriers set up once.
//
// The work of a CTA is a sequence of UNITS, one query tile against one K/V tile, in the order
// item by item, K/V tile by K/V tile, A before B. For head_dim 64 a unit's 16,384 exponentials cost
// each SM sub-partition 1,024 cycles of its MUFU (ex2) pipe against ~680 tensor cycles for the unit's
// two MMAs (QK at full rate, PV with N = 64 at ~60 %), so the kernel is built to keep the MUFU pipes
// busy: softmax warps never wait for anything but their next S, and two softmax warps share each
// sub-partition, their exponential phases overlapping (one warp alone issues ex2 at ~75 % of the
// pipe's rate, two reach ~90 %). Roles (16 warps, 4 warpgroups):
//
//   warp 0   (1 thread)  TMA producer: the two Q tiles of each item (double-buffered), then K(t) and
//                        V(t-1) tiles (128 x 64 fp16, 128-byte swizzle) straight out of the packed qkv
//                        rows into 4-stage K and V rings, running ahead across item boundaries.
//   warps 2, 1           MMA issuers for both query tiles, in unit order. Warp 2: S_u = Q K^T into one of
//                        three TMEM S buffers (M128 N128 K64, 4 x tcgen05.mma K16), issued as soon as
//                        the PV of unit u-3 (the buffer's previous user) has completed. Warp 1: O_x +=
//                        P_u V (M128 N64 K128, 8 x tcgen05.mma K16, P read from TMEM) once the softmax
//                        has written P_u.
//   warps 4-7, 8-11      softmax of query tile A, of B: one thread per query row (TMEM lane), all 128
//                        scores of a unit in registers. Log2 domain (1/8 * log2(e) folded into one
//                        FFMA, hardware ex2); causal mask on the diagonal tile only; P = 2^(s-m) written
//                        as packed fp16 over the first 64 columns of the unit's own S buffer; the row
//                        sum adds the fp16-rounded P values (numerator and denominator use identical
//                        weights); O is rescaled in TMEM only when the running max grows by more than
//                        2^8 (the stale max is otherwise kept for both l and O: exact, and P <= 256).
//   warps 12-15          epilogue of both query tiles: at the end of an item, O / l -> fp16 -> a
//                        swizzled 4 KB shared-memory slot per warp -> one TMA store of the warp's 32
//                        rows, so output rows leave as whole 128-byte lines; the split path's partial
//                        rows and merge (below) also run here.
//
// Launches with fewer whole pairs than SMs (one layer of one sequence) run the kSplit instantiation: a
// work unit is a chunk of a pair's key range; split units park unnormalised rows (o, m, l) in a
// workspace and the last chunk to arrive for a 32-row group merges them. With a KV-cache target the
// producer also stores the K/V tiles its unit owns into the cache, straight from the ring.
//
// TMEM: all 512 columns (S buffers at 0, 128, 256; O_A 384, O_B 448). Shared memory: Q 64 KB, K and V
// rings 128 KB, output slots 16 KB, row statistics 4 KB, barriers. No cluster, no multicast. Every
// mbarrier wait is bounded. Registers: the launch gives each of the 512 threads 128; the producer /
// MMA warpgroup and the epilogue warpgroup hand some back (setmaxnreg) so that the softmax warps hold
// their 128 scores without spilling.
//
// Launch: a programmatic dependent of the previous kernel in the stream. Barrier init, TMEM
// allocation and an L2 prefetch of the first item's Q, K and V tiles overlap that kernel's tail;
// every load, store and workspace access follows the grid dependency wait.
#include <algorithm>
#include <cmath>
#include <cstdio>

#include "common.cuh"
#include "ptx.cuh"

namespace b200 {
namespace prefill {

constexpr int BM = 128;  // query rows per tile = TMEM lanes
constexpr int BN = 128;  // keys per KV tile
constexpr int HD = 64;   // head dim
constexpr int NSTAGE = 4;  // K ring and V ring depth
constexpr int NQ = 2;      // Q buffers (each holds the two query tiles of an item)
constexpr int TILE_BYTES = BM * HD * 2;  // 16 KB: 128 rows x 128 B
constexpr int OFF_Q = 0;                                     // [NQ][2 tiles]
constexpr int OFF_K = OFF_Q + NQ * 2 * TILE_BYTES;
constexpr int OFF_V = OFF_K + NSTAGE * TILE_BYTES;
constexpr int OUT_ROWS = 32;                    // output rows per epilogue warp (one TMA store box)
constexpr int OUT_SLOT = OUT_ROWS * HD * 2;     // 4 KB: 32 rows x 128 B, 128-byte swizzle
constexpr int OFF_OUT = OFF_V + NSTAGE * TILE_BYTES;  // [4 epilogue warps] output slots
constexpr int OFF_STATS = OFF_OUT + 4 * OUT_SLOT;     // [2 tiles][2 item parities][m | l][128 rows] fp32
constexpr int OFF_BAR = OFF_STATS + 2 * 2 * 2 * BM * 4;
constexpr int SMEM_BYTES = OFF_BAR + 512;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
constexpr int NSOFT_WARPS = 4;  // per query tile: one warp per TMEM lane quarter
// Four warpgroups, one warp of each on every SM sub-partition: WG0 = warps 0-3 (producer, the two MMA
// issuers, one idle warp), WG1 = softmax of A, WG2 = softmax of B, WG3 = epilogue. The launch gives every
// thread LAUNCH_REGS registers; WG0 and WG3 give some back (setmaxnreg.dec) and the softmax groups
// take them (setmaxnreg.inc). The split adds up to the launch's pool exactly, and the host refuses to
// launch if ptxas gave the kernel another register count (an .inc could then never be satisfied).
constexpr int NTHREADS = 32 * 4 * 4;
constexpr int MMA_WARP = 1;      // query tile A's MMA issuer (and TMEM allocation)
constexpr int MMA_B_WARP = 2;    // query tile B's MMA issuer
constexpr int SOFT_WARP0 = 4;   // first softmax warp
constexpr int EPI_WARP0 = 12;   // first epilogue warp
constexpr int CTAS_PER_SM = 1;
constexpr int LAUNCH_REGS = 128;  // 65536 / (4 warps per sub-partition x 32)
constexpr int WG0_REGS = 64;
constexpr int EPI_REGS = 80;
constexpr int SOFTMAX_REGS = 184;
static_assert(128 * (WG0_REGS + EPI_REGS) + 256 * SOFTMAX_REGS == NTHREADS * LAUNCH_REGS, "register split");
static_assert(WG0_REGS + EPI_REGS + 2 * SOFTMAX_REGS <= 512, "one warp of each group per sub-partition");
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TCOL_S = 0;    // + 128 * query tile
constexpr uint32_t TCOL_O = 256;  // + 64 * query tile
constexpr uint32_t TCOL_P = 384;  // + 64 * query tile
constexpr uint32_t IDESC_S = idesc_f16_f32(BM, BN, 0, 0);  // Q K-major, K K-major
constexpr uint32_t IDESC_O = idesc_f16_f32(BM, HD, 0, 1);  // P K-major (TMEM), V MN-major
constexpr float RESCALE_THRESHOLD = 8.0f;                  // log2 units: P stays <= 2^8

struct Stream {  // per query tile of the pair
    uint64_t s_full;   // its QK of the current K/V tile has completed
    uint64_t s_free;   // its softmax warps have read S into registers
    uint64_t p_full;   // its softmax warps have written P (and rescaled O)
    uint64_t o_done;   // a PV of this query tile has completed (one phase per PV)
    uint64_t o_last;   // the item's last PV of this query tile has completed (one phase per item)
    uint64_t o_free;   // the epilogue has read O of the item
};

struct __align__(8) Bars {
    uint64_t q_full[NQ];
    uint64_t q_empty[NQ];      // the item's last QK has completed
    uint64_t k_full[NSTAGE];
    uint64_t k_empty[NSTAGE];  // the last QK reading this K stage has completed
    uint64_t v_full[NSTAGE];
    uint64_t v_empty[NSTAGE];  // the last PV reading this V stage has completed
    Stream st[2];              // per query tile
    uint64_t st_full[2][2];    // softmax of tile x wrote its item's row statistics (buffer = item parity)
    uint64_t st_free[2][2];    // the epilogue has read them
    uint64_t drain;            // teardown: every MMA of both issuers has completed
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Bars) <= 512, "barrier block");

struct Params {
    int T, H, E, B;
    unsigned hb_magic, h_magic;  // magic multipliers: item index / (H * B) and / H without division
    int hb_shift, h_shift;
    int n_qtiles;
    int n_pairs;               // ceil(n_qtiles / 2)
    int kv_chunk;              // K/V tiles per work unit (>= n_qtiles: a pair is never split)
    int units_per_hb;          // work units per (head, sequence): sum over pairs of their chunks
    int max_chunks;            // chunks of the longest pair (partial-row slots per query tile)
    int total_items;           // units_per_hb * H * B
    float scale_log2;          // log2(e) / sqrt(D)
    float *part;               // split units: partials [group][chunk][PART_COLS][128 rows]
    int kv_fill;               // also write K/V rows 0..T-1 into a KV-cache layer (B == 1)
    unsigned *counters;        // split units: arrivals per [group][lane quarter], re-armed to 0
    unsigned *status;
    unsigned long long timeout_ns;
    __half *att;               // split launches: output rows are stored directly (no TMA slot)
    long long att_seq_stride;  // elements between sequences of att
};
constexpr int PART_COLS = HD + 2;  // o[64], m, l of a row; stored column-major (coalesced)
constexpr int MAX_CHUNKS = 8;       // chunks per pair at most (the merge is unrolled over them)

struct Item {
    int pair, h, b;
    int kv0;             // first K/V tile of this unit (its chunk of the pair's key range)
    int chunk, nchunk;   // chunk index and chunks of this pair (nchunk > 1: partial rows + merge)
    int nk[2];  // K/V tiles of query tile A (2p) and of B (2p+1, none past T) in this unit: a prefix
    int nkv;    // K/V tiles loaded for the unit: max(nk)
    // nk[x] for a runtime x without a local-memory array access
    __device__ __forceinline__ int nk_of(int x) const { return x ? nk[1] : nk[0]; }
};

// n / d for any 32-bit unsigned n and 1 <= d < 2^31 with a precomputed magic (round-up method:
// l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1; q = (t + ((n - t) >> 1)) >> (l - 1) with
// t = mulhi(m, n); d == 1 is passed through).
__device__ __forceinline__ unsigned div_magic(unsigned n, unsigned d, unsigned m, int l) {
    if (d == 1) return n;
    const unsigned t = __umulhi(m, n);
    return (t + ((n - t) >> 1)) >> (l - 1);
}

// K/V tiles a pair's key range covers: through B's diagonal, or A's when B is past T.
__device__ __forceinline__ int pair_kv_tiles(const Params &p, int pair) {
    return (2 * pair + 1 < p.n_qtiles) ? 2 * pair + 2 : 2 * pair + 1;
}

// The r-th work unit of this CTA. A unit is one chunk of kv_chunk K/V tiles of a pair of query tiles
// (the whole key range unless the launch is too small to fill the SMs with whole pairs). Units are
// numbered heaviest pair first; rounds alternate direction (snake) so that each CTA gets a mix of
// heavy and light units. Returns false when this CTA has no r-th unit (nor any later one).
template <bool kSplit>
__device__ __forceinline__ bool get_item(const Params &p, int r, Item &it) {
    const int G = gridDim.x, c = blockIdx.x;
    const long long i = static_cast<long long>(r) * G + ((r & 1) ? (G - 1 - c) : c);
    if (i >= p.total_items) return false;
    const int per = p.H * p.B;
    const int idx = static_cast<int>(i);
    int u = static_cast<int>(div_magic(idx, per, p.hb_magic, p.hb_shift));  // unit in its (head, seq)
    const int rem = idx - u * per;
    it.b = static_cast<int>(div_magic(rem, p.H, p.h_magic, p.h_shift));
    it.h = rem - it.b * p.H;
    int pr = p.n_pairs - 1 - u, nc = 1;  // whole pairs: unit u is pair n_pairs-1-u, one chunk
    if (kSplit) {
        for (pr = p.n_pairs - 1; pr > 0; --pr) {
            nc = (pair_kv_tiles(p, pr) + p.kv_chunk - 1) / p.kv_chunk;
            if (u < nc) break;
            u -= nc;
        }
        if (pr == 0) nc = (pair_kv_tiles(p, 0) + p.kv_chunk - 1) / p.kv_chunk;
    } else {
        u = 0;
    }
    it.pair = pr;
    it.chunk = u;
    it.nchunk = nc;
    it.kv0 = u * p.kv_chunk;
    const int hi = min(it.kv0 + p.kv_chunk, pair_kv_tiles(p, pr));
    it.nk[0] = max(0, min(hi, 2 * pr + 1) - it.kv0);
    it.nk[1] = (2 * pr + 1 < p.n_qtiles) ? hi - it.kv0 : 0;
    it.nkv = hi - it.kv0;
    return true;
}

// A cursor over this CTA's K/V tiles in processing order (item by item).
template <bool kSplit>
struct Cursor {
    Item I;
    int it, j, g;  // item number, K/V tile within the item, K/V tile number over all items
    bool valid;
    __device__ __forceinline__ void start(const Params &p) {
        it = 0;
        j = 0;
        g = 0;
        valid = get_item<kSplit>(p, 0, I);
    }
    __device__ __forceinline__ void advance(const Params &p) {
        ++g;
        if (++j == I.nkv) {
            j = 0;
            ++it;
            valid = get_item<kSplit>(p, it, I);
        }
    }
};

__device__ __forceinline__ void raise_abort(Bars *bars, unsigned *status, unsigned bit) {
    atomicOr(status, bit);
    *reinterpret_cast<volatile int *>(&bars->abort) = 1;
}

__device__ __forceinline__ bool aborted(Bars *bars) {
    return *reinterpret_cast<volatile int *>(&bars->abort) != 0;
}

// ------------------------------------------------------------------ producer (one thread)
// Load order: the Q tiles of an item before its first K; then K(t), V(t-1), K(t+1), V(t), ... . K
// stages are released when their QKs complete and V stages when their PVs complete (later), so
// issuing V one tile behind K keeps the K loads from queueing behind a V wait.
template <bool kSplit>
__device__ void run_producer(const CUtensorMap *tm, const CUtensorMap *tm_kv, uint8_t *smem, Bars *bars,
                             const Params &p) {
    const unsigned long long to = p.timeout_ns;
    int last_q[NQ] = {-1, -1}, last_k[NSTAGE], last_v[NSTAGE];
    // KV-cache fill: the K/V tile each stage holds that this CTA must also store into the cache
    // (head << 16 | tile), -1 for none. A tile is stored by the unit of the pair whose top two tiles
    // it is (tiles 2p and 2p+1 are loaded by no lower pair), so each tile is written exactly once. It
    // is stored when its stage is about to be reused (it has landed and been consumed) or at teardown.
    int own_k[NSTAGE], own_v[NSTAGE];
    for (int s = 0; s < NSTAGE; ++s) last_k[s] = last_v[s] = own_k[s] = own_v[s] = -1;
    bool ok = true;
    Cursor<kSplit> kc, vc;  // next K tile to load; next V tile to load (never ahead of kc)
    kc.start(p);
    vc.start(p);
    auto owned = [&](const Cursor<kSplit> &c) -> int {
        const int tile = c.I.kv0 + c.j;
        return (p.kv_fill && tile >= 2 * c.I.pair) ? (c.I.h << 16) | tile : -1;
    };
    // z = head for K, nHead + head for V (the layer's K block is followed by its V block)
    auto store_tile = [&](const uint8_t *src, int own, int zoff) {
        tma_store_3d(tm_kv, src, 0, (own & 0xffff) * BN, zoff + (own >> 16));
        bulk_commit_group();
        bulk_wait_group_read0();  // the stage may be overwritten once the store has read it
    };
    auto load_v = [&]() -> bool {
        const int s = vc.g % NSTAGE;
        if (vc.g >= NSTAGE && !mbar_wait(&bars->v_empty[s], ((vc.g / NSTAGE) - 1) & 1, to)) return false;
        if (own_v[s] >= 0) store_tile(smem + OFF_V + s * TILE_BYTES, own_v[s], p.H);
        mbar_arrive_expect_tx(&bars->v_full[s], TILE_BYTES);
        tma_load_3d(smem + OFF_V + s * TILE_BYTES, tm, &bars->v_full[s], 2 * p.E + vc.I.h * HD,
                    (vc.I.kv0 + vc.j) * BN, vc.I.b);
        last_v[s] = vc.g;
        own_v[s] = owned(vc);
        vc.advance(p);
        return true;
    };
    while (ok && kc.valid) {
        if (aborted(bars)) {
            ok = false;
            break;
        }
        if (kc.j == 0) {  // new item: its two Q tiles (the buffer's previous item issued its last QK)
            const int qb = kc.it % NQ;
            if (kc.it >= NQ && !(ok = mbar_wait(&bars->q_empty[qb], ((kc.it / NQ) - 1) & 1, to))) break;
            const int ntiles = kc.I.nk[1] ? 2 : 1;
            mbar_arrive_expect_tx(&bars->q_full[qb], ntiles * TILE_BYTES);
            for (int t = 0; t < ntiles; ++t)
                tma_load_3d(smem + OFF_Q + (qb * 2 + t) * TILE_BYTES, tm, &bars->q_full[qb],
                            kc.I.h * HD, (2 * kc.I.pair + t) * BM, kc.I.b);
            last_q[qb] = kc.it;
        }
        const int s = kc.g % NSTAGE;
        if (kc.g >= NSTAGE && !(ok = mbar_wait(&bars->k_empty[s], ((kc.g / NSTAGE) - 1) & 1, to)))
            break;
        if (own_k[s] >= 0) store_tile(smem + OFF_K + s * TILE_BYTES, own_k[s], 0);
        mbar_arrive_expect_tx(&bars->k_full[s], TILE_BYTES);
        tma_load_3d(smem + OFF_K + s * TILE_BYTES, tm, &bars->k_full[s], p.E + kc.I.h * HD,
                    (kc.I.kv0 + kc.j) * BN, kc.I.b);
        last_k[s] = kc.g;
        own_k[s] = owned(kc);
        // Launch: every CTA asks for its first Q and K(0) alone, and only then for the rest of the
        // rings, so the first QK does not queue behind ~24 MB of later tiles requested by all SMs
        // at once (measured -2..3 % at P=1024).
        if (kc.g == 0 && !(ok = mbar_wait(&bars->k_full[0], 0, to))) break;
        kc.advance(p);
        if (vc.g + 1 < kc.g && !(ok = load_v())) break;  // V one tile behind K
    }
    while (ok && vc.valid && !aborted(bars)) ok = load_v();  // the remaining V tiles
    if (!ok && !aborted(bars)) raise_abort(bars, p.status, ST_PREFILL_LOAD_TIMEOUT);
    // Teardown guard: every copy this thread issued must have landed before the CTA exits.
    bool drained = true;
    for (int s = 0; s < NQ; ++s)
        if (last_q[s] >= 0) drained = mbar_wait(&bars->q_full[s], (last_q[s] / NQ) & 1, to) && drained;
    for (int s = 0; s < NSTAGE; ++s) {
        if (last_k[s] >= 0) drained = mbar_wait(&bars->k_full[s], (last_k[s] / NSTAGE) & 1, to) && drained;
        if (last_v[s] >= 0) drained = mbar_wait(&bars->v_full[s], (last_v[s] / NSTAGE) & 1, to) && drained;
    }
    if (!drained) atomicOr(p.status, ST_PREFILL_DRAIN_TIMEOUT);
    if (p.kv_fill) {  // the owned tiles still in the rings (their loads have landed)
        if (drained && !aborted(bars)) {
            for (int s = 0; s < NSTAGE; ++s) {
                if (own_k[s] >= 0) store_tile(smem + OFF_K + s * TILE_BYTES, own_k[s], 0);
                if (own_v[s] >= 0) store_tile(smem + OFF_V + s * TILE_BYTES, own_v[s], p.H);
            }
        }
        bulk_wait_group0();  // cache writes complete before the CTA's shared memory goes away
    }
}

// ------------------------------------------------------------------ MMA issuers (one warp per query tile)
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity,
                                          unsigned long long to) {
    const bool ok = mbar_wait(bar, parity, to);
    return __all_sync(0xffffffffu, ok);
}

struct Descs {
    uint32_t q_lo, q_hi, k_lo, k_hi, v_lo, v_hi;
    __device__ __forceinline__ explicit Descs(uint8_t *smem) {
        // Built once; an MMA then only adds a K-step offset to the start-address word (+32 B per K16
        // step inside a 128-byte swizzled row, +2 KB = 16 rows of V per K16 step).
        const uint64_t dq0 = sdesc_sw128(smem_u32(smem + OFF_Q), 16, 1024);
        const uint64_t dk0 = sdesc_sw128(smem_u32(smem + OFF_K), 16, 1024);
        const uint64_t dv0 = sdesc_sw128(smem_u32(smem + OFF_V), TILE_BYTES, 1024);
        q_lo = static_cast<uint32_t>(dq0);
        q_hi = static_cast<uint32_t>(dq0 >> 32);
        k_lo = static_cast<uint32_t>(dk0);
        k_hi = static_cast<uint32_t>(dk0 >> 32);
        v_lo = static_cast<uint32_t>(dv0);
        v_hi = static_cast<uint32_t>(dv0 >> 32);
    }
};
constexpr uint32_t TILE_DESC = TILE_BYTES >> 4;  // one 16 KB tile in start-address units

// Warp 1 issues query tile A's MMAs, warp 2 tile B's, each walking every K/V tile of every item: S_x =
// Q_x K^T once the softmax has read the previous S_x, O_x += P_x V once it has written P_x. Each issuer
// runs on its whole warp (every wait and all bookkeeping warp-uniform, so the MMA operands stay in
// uniform registers); one elected lane issues the MMAs and commits. The shared K, V and Q stages are
// released through two-arrival barriers: a tile's MMAs commit on them (or, for a tile it does not use,
// the issuer arrives after that tile has landed, so arrivals of different phases cannot mix).
template <bool kSplit>
__device__ void run_mma(uint8_t *smem, Bars *bars, const Params &p, uint32_t tbase, int x) {
    const unsigned long long to = p.timeout_ns;
    const Descs ds(smem);
    const bool leader = elect_one();
    Stream &S = bars->st[x];
    const uint32_t tS = tbase + TCOL_S + 128 * x, tO = tbase + TCOL_O + 64 * x;
    const uint32_t tP = tbase + TCOL_P + 64 * x;
    int gs = 0;   // this query tile's QKs issued (all items)
    int gp = 0;   // this query tile's PVs issued
    int itp = 0;  // items in which this query tile's PVs have started (for o_free)
    // S = Q K^T for the K/V tile under cursor q (or release of that tile if this query tile skips it).
    auto qk_step = [&](const Cursor<kSplit> &q) -> bool {
        const int qb = q.it % NQ, s = q.g % NSTAGE;
        const bool uses = q.j < q.I.nk_of(x);
        if (q.j == 0 && !warp_wait(&bars->q_full[qb], (q.it / NQ) & 1, to)) return false;
        if (!warp_wait(&bars->k_full[s], (q.g / NSTAGE) & 1, to)) return false;
        if (uses) {
            if (gs > 0 && !warp_wait(&S.s_free, (gs - 1) & 1, to)) return false;
            tc_fence_after();
            const uint32_t a = ds.q_lo + (qb * 2 + x) * TILE_DESC, b = ds.k_lo + s * TILE_DESC;
            if (leader) {
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    umma_f16_ss_lohi(tS, a + 2 * kk, ds.q_hi, b + 2 * kk, ds.k_hi, IDESC_S, kk > 0 ? 1u : 0u);
                umma_commit(&S.s_full);
                umma_commit(&bars->k_empty[s]);
            }
            ++gs;
        } else if (leader) {
            mbar_arrive(&bars->k_empty[s]);
        }
        // the Q buffer: released after this query tile's last QK of the item (or at once if it has none)
        const int last = q.I.nk_of(x) ? q.I.nk_of(x) - 1 : 0;
        if (q.j == last && leader) {
            if (uses) umma_commit(&bars->q_empty[qb]);
            else mbar_arrive(&bars->q_empty[qb]);
        }
        __syncwarp();
        return true;
    };
    // O += P V for the K/V tile under cursor v (or release of that tile).
    auto pv_step = [&](const Cursor<kSplit> &v) -> bool {
        const int s = v.g % NSTAGE;
        if (!warp_wait(&bars->v_full[s], (v.g / NSTAGE) & 1, to)) return false;
        if (v.j >= v.I.nk_of(x)) {
            if (leader) mbar_arrive(&bars->v_empty[s]);
            __syncwarp();
            return true;
        }
        if (!warp_wait(&S.p_full, gp & 1, to)) return false;
        if (v.j == 0) {  // the item's first PV overwrites O: the epilogue must have read it
            if (itp > 0 && !warp_wait(&S.o_free, (itp - 1) & 1, to)) return false;
            ++itp;
        }
        tc_fence_after();
        const uint32_t b = ds.v_lo + s * TILE_DESC;
        if (leader) {
            umma_f16_ts_lohi(tO, tP, b, ds.v_hi, IDESC_O, v.j == 0 ? 0u : 1u);
#pragma unroll
            for (int kk = 1; kk < BN / 16; ++kk)  // 16 keys = 8 packed TMEM columns of P per step
                umma_f16_ts_lohi(tO, tP + kk * 8, b + 128 * kk, ds.v_hi, IDESC_O, 1u);
            umma_commit(&S.o_done);
            if (v.j == v.I.nk_of(x) - 1) umma_commit(&S.o_last);
            umma_commit(&bars->v_empty[s]);
        }
        ++gp;
        __syncwarp();
        return true;
    };

    Cursor<kSplit> q, v;  // q: next K/V tile for QK; v: next tile for PV (one behind q)
    q.start(p);
    v.start(p);
    bool ok = true;
    if (q.valid) {
        ok = qk_step(q);
        q.advance(p);
    }
    while (ok && v.valid) {
        if (aborted(bars)) break;
        if (q.valid) {
            ok = qk_step(q);
            if (!ok) break;
            q.advance(p);
        }
        ok = pv_step(v);
        if (!ok) break;
        v.advance(p);
    }
    if (!ok && leader) raise_abort(bars, p.status, ST_PREFILL_MMA_TIMEOUT);
    // Teardown guard: all MMAs issued by this warp complete before TMEM is released.
    if (leader) umma_commit(&bars->drain);
    __syncwarp();
}

// ------------------------------------------------------------------ softmax

// End of an item in a split launch, run by the item's softmax warps (32 rows each): once the item's
// last PV of this query tile has completed, O / l goes straight to att when the item is a whole pair;
// a chunk of a pair parks its unnormalised rows (o, m, l) in the workspace and the last chunk to
// arrive for these 32 rows merges every chunk's partial. Rows are stored as whole 128-byte lines.
// Returns false when a wait expired.
__device__ __forceinline__ bool split_epilogue(Bars *bars, const Params &p, uint32_t tO, int x, int quarter,
                                            int lane, int row, int it, int g, float m_row, float l_row) {
    Stream &S = bars->st[x];
    if (!warp_wait(&S.o_done, (g - 1) & 1, p.timeout_ns)) return false;  // the item's last PV
    tc_fence_after();
    Item I;
    get_item<true>(p, it, I);
    const int qrow = (2 * I.pair + x) * BM + row;  // query index of this thread's row
    uint4 *dst = reinterpret_cast<uint4 *>(p.att + I.b * p.att_seq_stride +
                                           static_cast<long long>(qrow) * p.E + I.h * HD);
    auto store_row = [&](const float (&o)[32], int half) {  // 32 columns of this row, normalised
        if (qrow < p.T) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
                dst[4 * half + q] = make_uint4(pack_half2(o[8 * q], o[8 * q + 1]), pack_half2(o[8 * q + 2], o[8 * q + 3]),
                                               pack_half2(o[8 * q + 4], o[8 * q + 5]), pack_half2(o[8 * q + 6], o[8 * q + 7]));
        }
    };
    if (I.nchunk == 1) {
        const float inv_l = 1.f / l_row;
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
            uint32_t v[32];
            tmem_ld32(tO + 32 * cb, v);
            tmem_wait_ld();
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(v[i]) * inv_l;
            store_row(o, cb);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.o_free);
        return true;
    }
    const long long grp = ((static_cast<long long>(I.b) * p.H + I.h) * p.n_pairs + I.pair) * 2 + x;
    // column c of this row of chunk k at part[((grp * max_chunks + k) * PART_COLS + c) * 128 + row]
    float *mine = p.part + (grp * p.max_chunks + I.chunk) * (PART_COLS * BM) + row;
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
        uint32_t v[32];
        tmem_ld32(tO + 32 * cb, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) __stcg(mine + (32 * cb + i) * BM, __uint_as_float(v[i]));
    }
    __stcg(mine + HD * BM, m_row);
    __stcg(mine + (HD + 1) * BM, l_row);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.o_free);  // the next item's first PV may overwrite O
    // Publish the warp's 32 partial rows and count this chunk's arrival in one release-acquire atomic
    // (the warp barrier orders every lane's stores before lane 0's release; the last arrival's acquire
    // makes every chunk's rows visible to the merge below).
    unsigned *cnt = p.counters + grp * 4 + quarter;
    const int ncx = (2 * I.pair + x + p.kv_chunk) / p.kv_chunk;  // chunks with this tile's keys
    unsigned prev = 0;
    if (lane == 0)
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(cnt) : "memory");
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != static_cast<unsigned>(ncx - 1)) return true;
    // last chunk of these 32 rows: merge every chunk's partial row
    const float *base = p.part + grp * p.max_chunks * (PART_COLS * BM) + row;
    constexpr int CH = PART_COLS * BM;  // floats per chunk
    // Loads are predicated rather than branched so that each batch is one L2 round trip: (m, l) of
    // every chunk, then per 32-column half up to 4 chunks' values at once.
    float mk[MAX_CHUNKS], lk[MAX_CHUNKS], w[MAX_CHUNKS];
#pragma unroll
    for (int k = 0; k < MAX_CHUNKS; ++k) {
        mk[k] = -INFINITY;
        lk[k] = 0.f;
        if (k < ncx) {
            mk[k] = __ldcg(base + k * CH + HD * BM);
            lk[k] = __ldcg(base + k * CH + (HD + 1) * BM);
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < MAX_CHUNKS; ++k) M = fmaxf(M, k < ncx ? mk[k] : -INFINITY);
    float L = 0.f;
#pragma unroll
    for (int k = 0; k < MAX_CHUNKS; ++k) {
        w[k] = k < ncx ? ex2_approx(mk[k] - M) : 0.f;
        L = fmaf(w[k], lk[k], L);
    }
    const float inv_l = 1.f / L;
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
#pragma unroll
        for (int k0 = 0; k0 < MAX_CHUNKS; k0 += 4) {
            if (k0 < ncx) {
                float vals[4][32];
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float *pc = base + (k0 + kk) * CH + (32 * cb) * BM;
#pragma unroll
                    for (int i = 0; i < 32; ++i) vals[kk][i] = 0.f;
                    if (k0 + kk < ncx) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) vals[kk][i] = __ldcg(pc + i * BM);
                    }
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc[i] = fmaf(w[k0 + kk], vals[kk][i], acc[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] *= inv_l;
        store_row(acc, cb);
    }
    if (lane == 0) *cnt = 0u;  // re-armed for the next launch (every chunk has arrived)
    return true;
}

// Softmax of query tile x (0 = A, 1 = B) of every item: 4 warps, thread = one query row (TMEM lane),
// all 128 scores of a tile in registers. S is released as soon as it is in registers (the next QK
// runs while this tile is processed). The packed P values are kept in registers until every
// exponential is done; only then does the warp wait for the previous PV of its query tile (which read
// the P buffer, and after which O may be rescaled) -- by that time it has long completed. Every
// o_done phase is waited in order.
template <bool kSplit>
__device__ void run_softmax(uint8_t *smem, Bars *bars, const Params &p, uint32_t tbase, int x,
                            int warp, int lane) {
    const unsigned long long to = p.timeout_ns;
    Stream &S = bars->st[x];
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access (= SM sub-partition)
    const int row = quarter * 32 + lane;
    const uint32_t tl = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t tS = tl + TCOL_S + 128 * x;
    const uint32_t tO = tl + TCOL_O + 64 * x;
    const uint32_t tP = tl + TCOL_P + 64 * x;
    const float c = p.scale_log2;
    float *stats = reinterpret_cast<float *>(smem + OFF_STATS);
    int g = 0;   // this query tile's K/V tiles processed so far (all items)
    int kx = 0;  // items in which this query tile has keys (statistics buffer)
    bool ok = true;
    Item I;
    for (int it = 0; ok && get_item<kSplit>(p, it, I); ++it) {
        const int nk = I.nk_of(x);
        if (nk == 0) continue;     // this query tile has no keys in this unit of work
        const int diag_j = 2 * I.pair + x - I.kv0;  // K/V tile holding this tile's diagonal
        float m_used = -INFINITY;  // running max (log2 units) used for the exponentials
        float l = 0.f;             // running sum of the (fp16-rounded) exponentials
        for (int j = 0; j < nk; ++j, ++g) {
            ok = warp_wait(&S.s_full, g & 1, to);
            if (!ok) break;
            tc_fence_after();
            float xs[BN];
            {
                uint32_t v[4][32];
#pragma unroll
                for (int cb = 0; cb < 4; ++cb) tmem_ld32(tS + 32 * cb, v[cb]);
                tmem_wait_ld();
#pragma unroll
                for (int cb = 0; cb < 4; ++cb)
#pragma unroll
                    for (int i = 0; i < 32; ++i) xs[32 * cb + i] = __uint_as_float(v[cb][i]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.s_free);  // the next QK may overwrite S
            if (j == diag_j) {  // diagonal tile (BM == BN): key k is visible iff k <= r
#pragma unroll
                for (int i = 0; i < BN; ++i)
                    if (i > row) xs[i] = -INFINITY;
            }
            float pm[8];  // independent partial maxima, three-input max
#pragma unroll
            for (int k = 0; k < 8; ++k) pm[k] = fmaxf(xs[k], xs[8 + k]);
#pragma unroll
            for (int i = 16; i < BN; i += 16)
#pragma unroll
                for (int k = 0; k < 8; ++k) pm[k] = max3f(pm[k], xs[i + k], xs[i + 8 + k]);
            const float mt = max3f(max3f(pm[0], pm[1], pm[2]), max3f(pm[3], pm[4], pm[5]),
                                   fmaxf(pm[6], pm[7])) * c;
            float alpha = 1.f;
            bool resc = false;
            if (mt > m_used + RESCALE_THRESHOLD) {
                alpha = ex2_approx(m_used - mt);  // 0 on the first tile (m_used = -inf)
                m_used = mt;
                l *= alpha;
                resc = true;
            }
            const float neg_m = -m_used;
            // P = 2^(s - m) as packed fp16 (kept in registers). The row sum adds the fp16-ROUNDED values
            // (the ones the PV MMA consumes).
            uint32_t pk[4][16];
            float ps[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) ps[k] = 0.f;
#pragma unroll
            for (int cb = 0; cb < 4; ++cb) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = ex2_approx(fmaf(xs[32 * cb + 2 * i], c, neg_m));
                    const float p1 = ex2_approx(fmaf(xs[32 * cb + 2 * i + 1], c, neg_m));
                    pk[cb][i] = pack_half2(p0, p1);
                    ps[(2 * i) & 7] = add_f16lo_f32(pk[cb][i], ps[(2 * i) & 7]);
                    ps[(2 * i + 1) & 7] = add_f16hi_f32(pk[cb][i], ps[(2 * i + 1) & 7]);
                }
            }
            l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
            if (g > 0) {  // the previous PV of this query tile has read P and written O
                ok = warp_wait(&S.o_done, (g - 1) & 1, to);
                if (!ok) break;
                tc_fence_after();
            }
            if (j > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll
                for (int cb = 0; cb < 2; ++cb) {
                    uint32_t v[32];
                    tmem_ld32(tO + 32 * cb, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                    tmem_st32(tO + 32 * cb, v);
                }
            }
#pragma unroll
            for (int cb = 0; cb < 4; ++cb) tmem_st16(tP + 16 * cb, pk[cb]);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.p_full);
        }
        if (!ok) break;
        if (kSplit) {  // split launches: these warps finish their own rows (A and B in parallel)
            ok = split_epilogue(bars, p, tO, x, quarter, lane, row, it, g, m_used, l);
            if (!ok) break;
            continue;
        }
        // The item's row statistics for the epilogue (double-buffered by item parity).
        const int sb = kx & 1;
        if (kx >= 2) {
            ok = warp_wait(&bars->st_free[x][sb], ((kx >> 1) - 1) & 1, to);
            if (!ok) break;
        }
        float *st = stats + (x * 2 + sb) * 2 * BM;
        st[row] = m_used;
        st[BM + row] = l;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->st_full[x][sb]);
        ++kx;
    }
    if (!ok) raise_abort(bars, p.status, ST_PREFILL_SOFTMAX_TIMEOUT);
}

// ------------------------------------------------------------------ epilogue (4 warps, both tiles)
// At the end of each item, for A then B: O / l -> fp16 -> this warp's output slot -> one TMA store of
// its 32 rows (rows past T are clipped by the tensor map). A split unit first parks its unnormalised
// rows in the workspace; the last chunk to arrive for 32 rows merges them.
template <bool kSplit>
__device__ void run_epilogue(uint8_t *smem, Bars *bars, const Params &p, const CUtensorMap *tm_att,
                             uint32_t tbase, int warp, int lane) {
    const unsigned long long to = p.timeout_ns;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t tl = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
    const float *stats = reinterpret_cast<const float *>(smem + OFF_STATS);
    uint8_t *slot = smem + OFF_OUT + quarter * OUT_SLOT;
    // Row `lane` of the slot at lane * 128 B, 16-byte chunk k of a row at chunk position k ^ (row % 8)
    // (the TMA 128-byte swizzle, which also makes these writes bank-conflict-free).
    uint8_t *my_row = slot + lane * (HD * 2);
    auto put16 = [&](int c16, const uint32_t(&o)[8]) {  // fp16 columns 16 c16 .. 16 c16 + 15 of this row
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int chunk = (2 * c16 + q) ^ (lane & 7);
            *reinterpret_cast<uint4 *>(my_row + chunk * 16) =
                make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        }
    };
    if (kSplit) return;  // split launches: the softmax warps store their own rows
    int kx[2] = {0, 0};  // items of each query tile so far
    bool ok = true;
    Item I;
    for (int it = 0; ok && get_item<kSplit>(p, it, I); ++it) {
        for (int x = 0; x < 2; ++x) {
            if (I.nk_of(x) == 0) continue;
            const int sb = kx[x] & 1;
            ok = warp_wait(&bars->st[x].o_last, kx[x] & 1, to) &&
                 warp_wait(&bars->st_full[x][sb], (kx[x] >> 1) & 1, to);
            if (!ok) break;
            ++kx[x];
            tc_fence_after();
            const float *st = stats + (x * 2 + sb) * 2 * BM;
            const float l_row = st[BM + row];
            const uint32_t tO = tl + TCOL_O + 64 * x;
            // the slot's previous store has finished reading it (returns at once if none is pending)
            if (lane == 0) bulk_wait_group_read0();
            __syncwarp();
            {
                const float inv_l = 1.f / l_row;
#pragma unroll
                for (int c16 = 0; c16 < 4; ++c16) {  // 16 columns of O at a time (few registers)
                    uint32_t v[16];
                    tmem_ld16(tO + 16 * c16, v);
                    tmem_wait_ld();
                    uint32_t o[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        o[i] = pack_half2(__uint_as_float(v[2 * i]) * inv_l, __uint_as_float(v[2 * i + 1]) * inv_l);
                    put16(c16, o);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {  // O and the statistics have been read
                    mbar_arrive(&bars->st[x].o_free);
                    mbar_arrive(&bars->st_free[x][sb]);
                }
            }
            fence_proxy_async_smem();  // this thread's slot writes -> visible to the TMA engine
            __syncwarp();
            const int row0 = (2 * I.pair + x) * BM + quarter * OUT_ROWS;
            if (lane == 0 && row0 < p.T) {  // rows past T inside the box are clipped by the tensor map
                tma_store_3d(tm_att, slot, I.h * HD, row0, I.b);
                bulk_commit_group();
            }
        }
    }
    if (!ok) raise_abort(bars, p.status, ST_PREFILL_SOFTMAX_TIMEOUT);
    // The CTA's shared memory must outlive the stores that read it, and the launch ends with the
    // output written.
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
}

template <bool kSplit>
__global__ void __launch_bounds__(NTHREADS, CTAS_PER_SM)
    k_flash_prefill_tc(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_att,
                       const __grid_constant__ CUtensorMap tm_kv, const Params p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    Bars *bars = reinterpret_cast<Bars *>(smem + OFF_BAR);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if ((smem_u32(smem) & 1023u) != 0) {  // SW128 tiles need 1024-byte alignment; uniform exit
        if (threadIdx.x == 0) atomicOr(p.status, ST_PREFILL_SMEM_ALIGN);
        return;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < NQ; ++s) {
            mbar_init(&bars->q_full[s], 1);
            mbar_init(&bars->q_empty[s], 2);  // one release per query tile
        }
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&bars->k_full[s], 1);
            mbar_init(&bars->k_empty[s], 2);  // one release per query tile
            mbar_init(&bars->v_full[s], 1);
            mbar_init(&bars->v_empty[s], 2);
        }
        for (int x = 0; x < 2; ++x) {
            mbar_init(&bars->st[x].s_full, 1);
            mbar_init(&bars->st[x].s_free, NSOFT_WARPS);
            mbar_init(&bars->st[x].p_full, NSOFT_WARPS);
            mbar_init(&bars->st[x].o_done, 1);
            mbar_init(&bars->st[x].o_last, 1);
            mbar_init(&bars->st[x].o_free, 4);  // the epilogue warps
            for (int s = 0; s < 2; ++s) {
                mbar_init(&bars->st_full[x][s], NSOFT_WARPS);
                mbar_init(&bars->st_free[x][s], 4);
            }
        }
        mbar_init(&bars->drain, 2);  // one commit from each MMA issuer
        bars->abort = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_qkv);
        tma_prefetch_desc(&tm_att);
        if (p.kv_fill) tma_prefetch_desc(&tm_kv);
        // The first item's Q tiles and its first K and V tiles into L2 while the previous kernel
        // drains (the producer's first loads, issued after the dependency wait, then hit L2).
        Item i0;
        if (get_item<kSplit>(p, 0, i0)) {
            for (int t = 0; t < (i0.nk[1] ? 2 : 1); ++t)
                tma_prefetch_l2_3d(&tm_qkv, i0.h * HD, (2 * i0.pair + t) * BM, i0.b);
            tma_prefetch_l2_3d(&tm_qkv, p.E + i0.h * HD, i0.kv0 * BN, i0.b);
            tma_prefetch_l2_3d(&tm_qkv, 2 * p.E + i0.h * HD, i0.kv0 * BN, i0.b);
        }
    }
    if (warp == MMA_WARP) {
        tmem_alloc(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    // Launched as a programmatic dependent: the set-up above touches no global memory, so it overlaps
    // the previous kernel's tail; every global access (inputs, output, cache, workspace) follows this
    // wait. Dependents may start placing CTAs at once (they wait the same way before any access).
    grid_dependency_wait();
    grid_launch_dependents();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = bars->tmem_base;

    if (warp < SOFT_WARP0) {  // WG0: the whole warpgroup gives registers back, then takes its roles
        reg_dealloc<WG0_REGS>();
        if (warp == 0) {
            if (lane == 0) run_producer<kSplit>(&tm_qkv, &tm_kv, smem, bars, p);
        } else if (warp == MMA_WARP || warp == MMA_B_WARP) {
            run_mma<kSplit>(smem, bars, p, tbase, warp == MMA_WARP ? 0 : 1);
        }
        __syncwarp();
        // every MMA of both issuers has completed before TMEM is released (whole warp, converged)
        if (warp == MMA_WARP && !warp_wait(&bars->drain, 0, p.timeout_ns) && lane == 0)
            atomicOr(p.status, ST_PREFILL_DRAIN_TIMEOUT);
        __syncwarp();
    } else if (warp < EPI_WARP0) {  // WG1 / WG2: softmax of query tile A / B
        reg_alloc<SOFTMAX_REGS>();
        run_softmax<kSplit>(smem, bars, p, tbase, (warp - SOFT_WARP0) / NSOFT_WARPS, warp, lane);
    } else {  // WG3: epilogue
        reg_dealloc<EPI_REGS>();
        run_epilogue<kSplit>(smem, bars, p, &tm_att, tbase, warp, lane);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host side

// Chunk size (K/V tiles per work unit) for a launch of n_pairs pairs per (head, sequence) on `sms`
// SMs. Time model in units of one K/V tile step of a pair (both query tiles): a CTA's share of the
// total work, or the longest single unit, whichever is larger. A unit costs its tiles plus a fixed
// part measured on B200: ~2.2 steps for a whole pair (first loads, epilogue) and ~7 steps for a
// split one (the partial rows' write-out, fences and the merge are a chain of memory round trips).
// Large launches keep whole pairs; small ones (one layer of one sequence at P >= 1024) split the
// long key ranges when that clearly shortens the longest unit.
static int choose_kv_chunk(int n_qtiles, int n_pairs, long long hb, int sms) {
    int best = n_qtiles;
    double best_t = 1e300;
    const int cs_min = std::max(2, (n_qtiles + MAX_CHUNKS - 1) / MAX_CHUNKS);
    for (int cs = n_qtiles; cs >= cs_min; --cs) {
        long long units = 0, tiles = 0;
        for (int pr = 0; pr < n_pairs; ++pr) {
            const int nkv = (2 * pr + 1 < n_qtiles) ? 2 * pr + 2 : 2 * pr + 1;
            units += (nkv + cs - 1) / cs;
            tiles += nkv;
        }
        const bool split = units > n_pairs;
        const double ov = split ? 7.0 : 2.2;
        const double share = (static_cast<double>(tiles) * hb + units * hb * ov) / sms;
        const double longest = std::min(cs, n_qtiles) + ov;
        const double t = std::max(share, longest);
        if (t < best_t * 0.97) {  // prefer fewer, larger units unless splitting clearly pays
            best_t = t;
            best = cs;
        }
    }
    return best;
}

}  // namespace prefill

// Per-thread cache of recently encoded tensor maps (kind 0 = qkv load map, 1 = att store map).
namespace {
struct MapEntry {
    int kind, device, E, T, B;
    const void *ptr;
    long long seq_stride;
    bool valid;
    CUtensorMap map;
};
constexpr int kMapCache = 8;
thread_local MapEntry t_maps[kMapCache];
thread_local int t_map_next = 0;
}  // namespace

static bool cached_map(int kind, const void *ptr, int E, int T, int B, long long seq_stride, int device,
                       CUtensorMap *out) {
    for (const MapEntry &e : t_maps)
        if (e.valid && e.kind == kind && e.ptr == ptr && e.E == E && e.T == T && e.B == B &&
            e.seq_stride == seq_stride && e.device == device) {
            *out = e.map;
            return true;
        }
    return false;
}

static void remember_map(int kind, const void *ptr, int E, int T, int B, long long seq_stride, int device,
                         const CUtensorMap &map) {
    MapEntry &e = t_maps[t_map_next];
    t_map_next = (t_map_next + 1) % kMapCache;
    e = MapEntry{kind, device, E, T, B, ptr, seq_stride, true, map};
}

// Partial-row workspace of split prefill units (grown on demand, never while capturing).
static bool ensure_prefill_workspace(DeviceContext *ctx, size_t floats, size_t words, cudaStream_t stream) {
    if (ctx->pf_part_floats >= floats && ctx->pf_counter_words >= words) return true;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
    if (cudaDeviceSynchronize() != cudaSuccess) return false;
    // A grown buffer replaces the old one but the old one is never freed: a CUDA graph captured
    // earlier keeps the address it was captured with. Growth at least doubles, so the retired
    // buffers together stay below the live one.
    if (ctx->pf_part_floats < floats) {
        floats = std::max(floats, 2 * ctx->pf_part_floats);
        ctx->pf_part = nullptr;
        ctx->pf_part_floats = 0;
        if (cudaMalloc(&ctx->pf_part, floats * sizeof(float)) != cudaSuccess) return false;
        ctx->pf_part_floats = floats;
    }
    if (ctx->pf_counter_words < words) {
        words = std::max(words, 2 * ctx->pf_counter_words);
        ctx->pf_counters = nullptr;
        ctx->pf_counter_words = 0;
        if (cudaMalloc(&ctx->pf_counters, words * sizeof(unsigned)) != cudaSuccess) return false;
        if (cudaMemset(ctx->pf_counters, 0, words * sizeof(unsigned)) != cudaSuccess) return false;
        ctx->pf_counter_words = words;
    }
    return true;
}

// Launches the batched causal prefill. Arguments are validated by the caller (api.cu).
int launch_prefill(__half *att, const __half *qkv, int B, int T, int E, int H,
                   long long qkv_seq_stride, long long att_seq_stride, __half *kv_layer, int kv_maxT,
                   cudaStream_t stream) {
    using namespace prefill;
    DeviceContext *ctx = device_context();
    if (!ctx) return GPT2_B200_ECUDA;
    EncodeTiledFn enc = tensor_map_encoder();
    if (!enc) return GPT2_B200_EDEVICE;
    if (!ctx->prefill_attr_done) {
        for (auto fn : {k_flash_prefill_tc<false>, k_flash_prefill_tc<true>}) {
            // The warpgroups' register split is sized for exactly LAUNCH_REGS registers per thread at
            // launch; with any other count the softmax groups' setmaxnreg.inc could not be satisfied.
            cudaFuncAttributes fa;
            if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess) return GPT2_B200_ECUDA;
            if (fa.numRegs != LAUNCH_REGS) return GPT2_B200_EDEVICE;
            if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
                cudaSuccess)
                return GPT2_B200_ECUDA;
            cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
        }
        ctx->prefill_attr_done = true;
    }
    // qkv [B][T][3E] read as 64 x 128 boxes; att [B][T][E] written as 64 x 32 boxes (one per softmax
    // warp). Encoding is host work (microseconds), so the maps of recent calls are kept per thread:
    // the reference's forward pass calls attention on the same buffers for every layer.
    CUtensorMap tm, tm_att;
    if (!cached_map(0, qkv, E, T, B, qkv_seq_stride, ctx->device, &tm)) {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(3 * E), static_cast<cuuint64_t>(T),
                                    static_cast<cuuint64_t>(B)};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(3 * E) * 2,
                                       static_cast<cuuint64_t>(qkv_seq_stride) * 2};
        const cuuint32_t box[3] = {HD, BM, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half *>(qkv), dims, strides, box,
                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return GPT2_B200_EINVAL;
        remember_map(0, qkv, E, T, B, qkv_seq_stride, ctx->device, tm);
    }
    if (!cached_map(1, att, E, T, B, att_seq_stride, ctx->device, &tm_att)) {
        const cuuint64_t odims[3] = {static_cast<cuuint64_t>(E), static_cast<cuuint64_t>(T),
                                     static_cast<cuuint64_t>(B)};
        const cuuint64_t ostrides[2] = {static_cast<cuuint64_t>(E) * 2,
                                        static_cast<cuuint64_t>(att_seq_stride) * 2};
        const cuuint32_t obox[3] = {HD, OUT_ROWS, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (enc(&tm_att, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, att, odims, ostrides, obox, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return GPT2_B200_EINVAL;
        remember_map(1, att, E, T, B, att_seq_stride, ctx->device, tm_att);
    }

    // KV-cache layer (optional, B == 1): K block [H][maxT][64] then V block, rows 0..T-1 written
    CUtensorMap tm_kv = tm_att;  // unused unless kv_layer is set
    if (kv_layer) {
        if (B != 1 || kv_maxT < T) return GPT2_B200_EINVAL;
        if (!cached_map(2, kv_layer, E, T, kv_maxT, 0, ctx->device, &tm_kv)) {
            const cuuint64_t kdims[3] = {HD, static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(2 * H)};
            const cuuint64_t kstrides[2] = {HD * 2, static_cast<cuuint64_t>(kv_maxT) * HD * 2};
            const cuuint32_t kbox[3] = {HD, BN, 1};
            const cuuint32_t estr[3] = {1, 1, 1};
            if (enc(&tm_kv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, kv_layer, kdims, kstrides, kbox, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return GPT2_B200_EINVAL;
            remember_map(2, kv_layer, E, T, kv_maxT, 0, ctx->device, tm_kv);
        }
    }

    Params p;
    p.kv_fill = kv_layer != nullptr;
    p.att = att;
    p.att_seq_stride = att_seq_stride;
    p.T = T;
    auto magic = [](unsigned d, unsigned *m, int *l) {
        int sh = 0;
        while ((1ull << sh) < d) ++sh;
        *m = static_cast<unsigned>((((1ull << 32) * ((1ull << sh) - d)) / d + 1) & 0xffffffffull);
        *l = sh;
    };
    if (static_cast<long long>(H) * B >= (1ll << 31)) return GPT2_B200_EINVAL;
    magic(static_cast<unsigned>(H * B), &p.hb_magic, &p.hb_shift);
    magic(static_cast<unsigned>(H), &p.h_magic, &p.h_shift);
    p.H = H;
    p.E = E;
    p.B = B;
    p.n_qtiles = (T + BM - 1) / BM;
    p.n_pairs = (p.n_qtiles + 1) / 2;
    const long long hb = static_cast<long long>(H) * B;
    const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
    p.kv_chunk = p.n_qtiles;  // whole pairs
    p.units_per_hb = p.n_pairs;
    p.max_chunks = 1;
    p.part = nullptr;
    p.counters = nullptr;
    if (hb * p.n_pairs < sms) {
        const int cs = choose_kv_chunk(p.n_qtiles, p.n_pairs, hb, sms);
        int units = 0;
        for (int pr = 0; pr < p.n_pairs; ++pr)
            units += (((2 * pr + 1 < p.n_qtiles) ? 2 * pr + 2 : 2 * pr + 1) + cs - 1) / cs;
        const int max_chunks = (p.n_qtiles + cs - 1) / cs;
        const size_t groups = static_cast<size_t>(hb) * p.n_pairs * 2;
        if (units > p.n_pairs &&
            ensure_prefill_workspace(ctx, groups * max_chunks * BM * PART_COLS, groups * 4, stream)) {
            p.kv_chunk = cs;
            p.units_per_hb = units;
            p.max_chunks = max_chunks;
            p.part = ctx->pf_part;
            p.counters = ctx->pf_counters;
        }
    }
    const long long total = static_cast<long long>(p.units_per_hb) * hb;
    if (total <= 0) return GPT2_B200_OK;
    if (total > 0x7fffffffLL) return GPT2_B200_EINVAL;
    p.total_items = static_cast<int>(total);
    p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(HD)));
    p.status = ctx->status;
    p.timeout_ns = wait_timeout_ns();
    // Persistent: at most CTAS_PER_SM resident CTAs per SM, each looping over its share of items.
    const long long slots = static_cast<long long>(CTAS_PER_SM) * (ctx->num_sms > 0 ? ctx->num_sms : 148);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(total < slots ? total : slots));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = p.units_per_hb != p.n_pairs
                                ? cudaLaunchKernelEx(&cfg, k_flash_prefill_tc<true>, tm, tm_att, tm_kv, p)
                                : cudaLaunchKernelEx(&cfg, k_flash_prefill_tc<false>, tm, tm_att, tm_kv, p);
    return err == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}

}  // namespace b200
