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
// item by item, K/V tile by K/V tile. For head_dim 64 a unit's 16,384 exponentials cost each SM
// sub-partition 1,024 cycles of its MUFU (ex2) pipe against ~680 tensor cycles for the unit's two
// MMAs (QK at full rate, PV with N = 64 at ~60 %), so the kernel is built to keep the MUFU pipes busy:
// softmax warps never wait for anything but their next S, and two softmax warps share each
// sub-partition, their exponential phases overlapping (one warp alone issues ex2 at ~75 % of the
// pipe's rate, two reach ~90 %). Roles (16 warps, 4 warpgroups):
//
//   warp 0   (1 thread)  TMA producer: the two Q tiles of each item (double-buffered), then K(t) and
//                        V(t-1) tiles (128 x 64 fp16, 128-byte swizzle) straight out of the packed qkv
//                        rows into 4-stage K and V rings, running ahead across item boundaries.
//   warps 1, 2           MMA issuers of query tile A, of B, each on its whole warp with one elected
//                        lane: S_x = Q_x K^T (M128 N128 K64, 4 x tcgen05.mma K16) once the softmax has
//                        read the previous S_x, O_x += P_x V (M128 N64 K128, 8 x K16, P read from
//                        TMEM) once it has written P_x.
//   warps 4-7, 8-11      softmax of query tile A, of B: one thread per query row (TMEM lane), all 128
//                        scores of a unit in registers. Log2 domain (1/8 * log2(e) folded into one
//                        FFMA, hardware ex2); causal mask on the diagonal tile only; P = 2^(s-m) as
//                        packed fp16 kept in registers until the previous PV has completed, then
//                        written to the tile's P columns; the row sum adds the fp16-rounded P values
//                        (numerator and denominator use identical weights); O is rescaled in TMEM only
//                        when the running max grows by more than 2^8 (the stale max is otherwise kept
//                        for both l and O: exact, and P <= 256).
//   warps 12-15          epilogue of both query tiles: at the end of an item, O / l -> fp16 -> a
//                        swizzled 4 KB shared-memory slot per warp -> one TMA store of the warp's 32
//                        rows, so output rows leave as whole 128-byte lines.
//
// Launches with fewer whole pairs than SMs (one layer of one sequence) run the kSplit instantiation,
// one work unit per CTA (placed by the host), the chunks of a key range in one thread-block cluster
// (up to 4 CTAs). A unit is either a chunk of a pair's key range (both query tiles), or a chunk of ONE
// query tile's key range whose K/V tiles the two softmax groups take in turn (A the even ones, B the
// odd ones; they merge their rows locally at the end). Rows whose keys span several chunks are merged
// by one chunk: the others push their unnormalised rows (o, m, l) into its shared memory (remote
// st.async stores that complete on an mbarrier there), so no partial row goes through global memory.
// With a KV-cache target the producer also stores the K/V tiles its unit owns into the cache,
// straight from the ring.
//
// TMEM: all 512 columns (S_A at 0, S_B at 128, O_A 256, O_B 320, P_A 384, P_B 448). Shared memory:
// Q 64 KB, K and V rings 128 KB, output slots 16 KB, row statistics 4 KB (split launches receive the
// pushed partial rows there instead), barriers. No multicast. Every mbarrier wait is bounded.
// Registers: the launch gives each of the 512 threads 128; the producer / MMA warpgroup and the
// epilogue warpgroup hand some back (setmaxnreg) so that the softmax warps hold their 128 scores
// without spilling.
//
// Launch: a programmatic dependent of the previous kernel in the stream. Barrier init, TMEM
// allocation and an L2 prefetch of the first item's Q, K and V tiles overlap that kernel's tail;
// every global load and store follows the grid dependency wait.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <type_traits>

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
// Split launches: a softmax warp's 32 partial rows as pushed to the merging CTA: o as [16 column
// quads][32 rows] float4 (conflict-free for one row per lane on both sides), then (m, l) per row.
constexpr int MAX_CLUSTER = 4;  // chunks of one pair at most (= CTAs of a cluster)
constexpr int PART_O_BYTES = (HD / 4) * 32 * 16;
constexpr int PART_BYTES = PART_O_BYTES + 32 * 8;
// A split CTA has one unit, so it never uses the second Q buffer, the output slots and statistics,
// nor the K stages past its unit's K/V tiles: the pushed partials land there (see recv_slot).
constexpr int RECV_Q_SLOTS = 2 * TILE_BYTES / PART_BYTES;                   // 3
constexpr int RECV_OUT_SLOTS = (OFF_BAR - OFF_OUT) / PART_BYTES;            // 2
static_assert(RECV_Q_SLOTS == 3 && RECV_OUT_SLOTS == 2, "receive slots");
// Split launches of single-query-tile units: (m, l) of the B group's rows, handed to the A group
// (after the receive slots in the output-slot / statistics area).
constexpr int OFF_XCH = OFF_BAR - BM * 8;
static_assert(OFF_OUT + RECV_OUT_SLOTS * PART_BYTES <= OFF_XCH, "exchange area");
constexpr int MAX_SPLIT_CTAS = 160;  // CTAs of a split launch at most (one unit each, <= the SM count)
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
    uint64_t recv[2][4];       // split launches: the pushed partial rows of [query tile][lane quarter]
    uint64_t xm[4];            // single-query-tile split units: B's rows of a lane quarter are final
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
    int total_items;           // units_per_hb * H * B
    float scale_log2;          // log2(e) / sqrt(D)
    int kv_fill;               // also write K/V rows 0..T-1 into a KV-cache layer (B == 1)
    int intra;                 // split launches: a unit is a chunk of ONE query tile's keys (see Item)
    unsigned *status;
    unsigned long long timeout_ns;
    __half *att;               // split launches: output rows are stored directly (no TMA slot)
    long long att_seq_stride;  // elements between sequences of att
};

// Split launches: the work unit (item number) of each CTA, -1 for none. The host places the chunks of
// a pair in one cluster, chunk k at cluster rank (rank of chunk 0) + k. A separate kernel argument,
// absent (empty) from whole-pair launches.
struct SplitTable {
    short cta_item[MAX_SPLIT_CTAS];
};
struct NoSplitTable {};
template <bool kSplit>
using SplitArg = typename std::conditional<kSplit, SplitTable, NoSplitTable>::type;

// A unit of work. Pair units: query tiles A = 2 pair and B = 2 pair + 1, both against K/V tiles
// kv0 .. kv0 + nkv - 1 (A against a prefix). Single-query-tile units (split launches with
// Params::intra): query tile `pair` against those tiles, its two softmax groups taking alternate
// tiles (A the even ones, B the odd ones) and merging their rows at the end.
struct Item {
    int pair, h, b;
    int kv0;             // first K/V tile of this unit (its chunk of the key range)
    int chunk, nchunk;   // chunk index and chunks of this key range (nchunk > 1: partial rows + merge)
    int nk[2];  // K/V tiles group A and group B process in this unit
    int nkv;    // K/V tiles loaded for the unit
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

// Shared-memory offset of receive slot i of a split CTA whose unit loads at most kv_chunk K/V tiles.
__device__ __forceinline__ uint32_t recv_slot(int i, int kv_chunk) {
    if (i < RECV_Q_SLOTS) return OFF_Q + 2 * TILE_BYTES + i * PART_BYTES;
    if (i < RECV_Q_SLOTS + RECV_OUT_SLOTS) return OFF_OUT + (i - RECV_Q_SLOTS) * PART_BYTES;
    return OFF_K + kv_chunk * TILE_BYTES + (i - RECV_Q_SLOTS - RECV_OUT_SLOTS) * PART_BYTES;
}

// Chunks of a pair holding keys of its query tile x (its keys are K/V tiles 0 .. 2 pair + x: the
// first chunks), 0 when the tile is past T.
__device__ __forceinline__ int tile_chunks(const Params &p, int pair, int x) {
    return (2 * pair + x < p.n_qtiles) ? (2 * pair + x + p.kv_chunk) / p.kv_chunk : 0;
}

// Split launches: this CTA's unit (SplitTable::cta_item[blockIdx.x]), decoded once by thread 0 at
// launch (before the grid dependency wait) for every role.
__shared__ Item s_split_unit;
__shared__ int s_split_valid;

// Work unit number idx: unit idx / (H B) of (head, sequence) idx % (H B). A unit is one chunk of
// kv_chunk K/V tiles of a pair of query tiles (the whole key range unless the launch is too small to
// fill the SMs with whole pairs), or of one query tile (Params::intra); units are numbered heaviest
// pair (query tile) first.
template <bool kSplit>
__device__ __forceinline__ void decode_item(const Params &p, int idx, Item &it) {
    const int per = p.H * p.B;
    int u = static_cast<int>(div_magic(idx, per, p.hb_magic, p.hb_shift));  // unit in its (head, seq)
    const int rem = idx - u * per;
    it.b = static_cast<int>(div_magic(rem, p.H, p.h_magic, p.h_shift));
    it.h = rem - it.b * p.H;
    if (kSplit && p.intra) {  // query tiles from the last, each in ceil((qt + 1) / kv_chunk) chunks
        int qt = p.n_qtiles - 1, nc = (qt + p.kv_chunk) / p.kv_chunk;
        while (qt > 0 && u >= nc) {
            u -= nc;
            --qt;
            nc = (qt + p.kv_chunk) / p.kv_chunk;
        }
        it.pair = qt;
        it.chunk = u;
        it.nchunk = nc;
        it.kv0 = u * p.kv_chunk;
        it.nkv = min(it.kv0 + p.kv_chunk, qt + 1) - it.kv0;
        it.nk[0] = (it.nkv + 1) >> 1;
        it.nk[1] = it.nkv >> 1;
        return;
    }
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
}

// The r-th work unit of this CTA. Whole-pair launches are persistent: rounds of one unit per CTA
// alternate direction (snake) so that each CTA gets a mix of heavy and light units. Returns false
// when this CTA has no r-th unit (nor any later one).
template <bool kSplit>
__device__ __forceinline__ bool get_item(const Params &p, int r, Item &it) {
    if (kSplit) {  // one unit per CTA, placed by the host and decoded at launch
        if (r > 0 || !s_split_valid) return false;
        it = s_split_unit;
        return true;
    }
    const int G = gridDim.x, c = blockIdx.x;
    const long long i = static_cast<long long>(r) * G + ((r & 1) ? (G - 1 - c) : c);
    if (i >= p.total_items) return false;
    decode_item<kSplit>(p, static_cast<int>(i), it);
    return true;
}

// Whether query-tile group x processes K/V tile j of unit I, its first and last such tile (the last
// only when it has any), and the query tile it works on.
template <bool kSplit>
__device__ __forceinline__ bool item_uses(const Params &p, const Item &I, int j, int x) {
    return (kSplit && p.intra) ? ((j & 1) == x && j < I.nkv) : j < I.nk_of(x);
}
template <bool kSplit>
__device__ __forceinline__ int item_first(const Params &p, int x) {
    return (kSplit && p.intra) ? x : 0;
}
template <bool kSplit>
__device__ __forceinline__ int item_last(const Params &p, const Item &I, int x) {
    return (kSplit && p.intra) ? x + 2 * (I.nk_of(x) - 1) : I.nk_of(x) - 1;
}
template <bool kSplit>
__device__ __forceinline__ int item_qtile(const Params &p, const Item &I, int x) {
    return (kSplit && p.intra) ? I.pair : 2 * I.pair + x;
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
        const bool own = (kSplit && p.intra) ? tile == c.I.pair : tile >= 2 * c.I.pair;
        return (p.kv_fill && own) ? (c.I.h << 16) | tile : -1;
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
            const int ntiles = ((kSplit && p.intra) || !kc.I.nk[1]) ? 1 : 2;
            mbar_arrive_expect_tx(&bars->q_full[qb], ntiles * TILE_BYTES);
            for (int t = 0; t < ntiles; ++t)
                tma_load_3d(smem + OFF_Q + (qb * 2 + t) * TILE_BYTES, tm, &bars->q_full[qb],
                            kc.I.h * HD, item_qtile<kSplit>(p, kc.I, t) * BM, kc.I.b);
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
        // Launch: every CTA of a whole-pair launch asks for its first Q and K(0) alone, and only then
        // for the rest of the rings, so the first QK does not queue behind ~24 MB of later tiles
        // requested by all SMs at once (measured -2..3 % at P=1024). A split unit has only a few
        // tiles: it asks for all of them at once.
        if (!kSplit && kc.g == 0 && !(ok = mbar_wait(&bars->k_full[0], 0, to))) break;
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
        const bool uses = item_uses<kSplit>(p, q.I, q.j, x);
        if (q.j == 0 && !warp_wait(&bars->q_full[qb], (q.it / NQ) & 1, to)) return false;
        if (!warp_wait(&bars->k_full[s], (q.g / NSTAGE) & 1, to)) return false;
        if (uses) {
            if (gs > 0 && !warp_wait(&S.s_free, (gs - 1) & 1, to)) return false;
            tc_fence_after();
            const uint32_t a = ds.q_lo + (qb * 2 + ((kSplit && p.intra) ? 0 : x)) * TILE_DESC;
            const uint32_t b = ds.k_lo + s * TILE_DESC;
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
        const int last = q.I.nk_of(x) ? item_last<kSplit>(p, q.I, x) : 0;
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
        if (!item_uses<kSplit>(p, v.I, v.j, x)) {
            if (leader) mbar_arrive(&bars->v_empty[s]);
            __syncwarp();
            return true;
        }
        if (!warp_wait(&S.p_full, gp & 1, to)) return false;
        const bool first = v.j == item_first<kSplit>(p, x);
        if (first) {  // the item's first PV overwrites O: the epilogue must have read it
            if (itp > 0 && !warp_wait(&S.o_free, (itp - 1) & 1, to)) return false;
            ++itp;
        }
        tc_fence_after();
        const uint32_t b = ds.v_lo + s * TILE_DESC;
        if (leader) {
            umma_f16_ts_lohi(tO, tP, b, ds.v_hi, IDESC_O, first ? 0u : 1u);
#pragma unroll
            for (int kk = 1; kk < BN / 16; ++kk)  // 16 keys = 8 packed TMEM columns of P per step
                umma_f16_ts_lohi(tO, tP + kk * 8, b + 128 * kk, ds.v_hi, IDESC_O, 1u);
            umma_commit(&S.o_done);
            if (v.j == item_last<kSplit>(p, v.I, x)) umma_commit(&S.o_last);
            umma_commit(&bars->v_empty[s]);
        }
        ++gp;
        __syncwarp();
        return true;
    };

    Cursor<kSplit> q, v;  // q: next K/V tile for QK; v: next tile for PV (one behind q; two in
                          // single-query-tile units, where this query tile uses every other K/V tile)
    q.start(p);
    v.start(p);
    bool ok = true;
    for (int lead = (kSplit && p.intra) ? 2 : 1; ok && lead > 0 && q.valid; --lead) {
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

// The 32-row groups of a pair in a split launch: g = 4 x + lane quarter. Group g is merged by chunk
// g % nc (nc = chunks holding query tile x's keys), which receives the other nc - 1 chunks' partial
// rows of g in consecutive slots after those of the groups it merges before g.
__device__ __forceinline__ int merge_first_slot(const Params &p, int pair, int g, int km) {
    int slot = 0;
    for (int g2 = 0; g2 < g; ++g2) {
        const int n2 = tile_chunks(p, pair, g2 >> 2);
        if (n2 > 1 && g2 % n2 == km) slot += n2 - 1;
    }
    return slot;
}

// End of the unit of a split launch, run by each softmax warp for its 32 rows once the unit's last PV
// of its query tile has completed. Rows whose keys all lie in this chunk are normalised and stored;
// otherwise a chunk that does not merge these rows pushes its unnormalised rows (o, m, l) into the
// merging CTA (st.async, completing on that CTA's receive barrier), and the merging warp waits for
// the other chunks' rows, combines them with its own and stores the result. Output rows leave as
// whole 128-byte lines. Returns false when a wait expired.
__device__ __forceinline__ bool split_epilogue(uint8_t *smem, Bars *bars, const Params &p, const Item &I,
                                            uint32_t tO, int x, int quarter, int lane, int row, int g,
                                            float m_row, float l_row) {
    Stream &S = bars->st[x];
    if (!warp_wait(&S.o_done, (g - 1) & 1, p.timeout_ns)) return false;  // the unit's last PV
    tc_fence_after();
    float o[HD];
    {
        uint32_t v[2][32];
        tmem_ld32(tO, v[0]);
        tmem_ld32(tO + 32, v[1]);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = __uint_as_float(v[i >> 5][i & 31]);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.o_free);
    const int ncx = tile_chunks(p, I.pair, x);
    const int grp = 4 * x + quarter;
    const int km = ncx > 1 ? grp % ncx : I.chunk;  // the chunk that merges these rows
    if (I.chunk != km) {  // push this chunk's rows to the merging CTA (the same slots of its space)
        const int slot = merge_first_slot(p, I.pair, grp, km) + (I.chunk < km ? I.chunk : I.chunk - 1);
        const uint32_t rank = cluster_rank() - static_cast<uint32_t>(I.chunk) + static_cast<uint32_t>(km);
        const uint32_t dst = dsmem_addr(smem_u32(smem + recv_slot(slot, p.kv_chunk)), rank);
        const uint32_t bar = dsmem_addr(smem_u32(&bars->recv[x][quarter]), rank);
#pragma unroll
        for (int c4 = 0; c4 < HD / 4; ++c4)
            st_async_v4(dst + (c4 * 32 + lane) * 16, make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]),
                        bar);
        st_async_v2(dst + PART_O_BYTES + lane * 8, m_row, l_row, bar);
        return true;
    }
    float inv_l;
    if (ncx > 1) {  // merge the other chunks' rows into this one's
        if (!warp_wait(&bars->recv[x][quarter], 0, p.timeout_ns)) return false;
        const int s0 = merge_first_slot(p, I.pair, grp, km);
        const uint32_t in0 = smem_u32(smem) + static_cast<uint32_t>(lane) * 16u;
        float mk[MAX_CLUSTER - 1], lk[MAX_CLUSTER - 1];
        float M = m_row;
#pragma unroll
        for (int k = 0; k < MAX_CLUSTER - 1; ++k) {
            mk[k] = -INFINITY;
            lk[k] = 0.f;
            if (k < ncx - 1) {
                const float2 ml = lds_v2(smem_u32(smem) + recv_slot(s0 + k, p.kv_chunk) + PART_O_BYTES + lane * 8);
                mk[k] = ml.x;
                lk[k] = ml.y;
                M = fmaxf(M, ml.x);
            }
        }
        const float ws = ex2_approx(m_row - M);
        float L = ws * l_row;
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] *= ws;
#pragma unroll
        for (int k = 0; k < MAX_CLUSTER - 1; ++k) {
            if (k < ncx - 1) {
                const float w = ex2_approx(mk[k] - M);
                L = fmaf(w, lk[k], L);
                const uint32_t in = in0 + recv_slot(s0 + k, p.kv_chunk);
                float4 q[HD / 4];  // the whole partial row first: one round of shared-memory latency
#pragma unroll
                for (int c4 = 0; c4 < HD / 4; ++c4) q[c4] = lds_v4(in + c4 * 512);
#pragma unroll
                for (int c4 = 0; c4 < HD / 4; ++c4) {
                    o[4 * c4] = fmaf(w, q[c4].x, o[4 * c4]);
                    o[4 * c4 + 1] = fmaf(w, q[c4].y, o[4 * c4 + 1]);
                    o[4 * c4 + 2] = fmaf(w, q[c4].z, o[4 * c4 + 2]);
                    o[4 * c4 + 3] = fmaf(w, q[c4].w, o[4 * c4 + 3]);
                }
            }
        }
        inv_l = 1.f / L;
    } else {
        inv_l = 1.f / l_row;
    }
    const int qrow = (2 * I.pair + x) * BM + row;  // query index of this thread's row
    if (qrow < p.T) {
        uint4 *dst = reinterpret_cast<uint4 *>(p.att + I.b * p.att_seq_stride + static_cast<long long>(qrow) * p.E +
                                               I.h * HD);
#pragma unroll
        for (int q = 0; q < HD / 8; ++q)
            dst[q] = make_uint4(pack_half2(o[8 * q] * inv_l, o[8 * q + 1] * inv_l),
                                pack_half2(o[8 * q + 2] * inv_l, o[8 * q + 3] * inv_l),
                                pack_half2(o[8 * q + 4] * inv_l, o[8 * q + 5] * inv_l),
                                pack_half2(o[8 * q + 6] * inv_l, o[8 * q + 7] * inv_l));
    }
    return true;
}

// End of a single-query-tile unit of a split launch, run by each softmax warp for its 32 rows once its
// group's last PV has completed. Group B hands its (m, l) to group A's warp of the same lane quarter
// (its O stays in TMEM, which that warp can read); A combines both halves of the unit's key range.
// With several chunks of the query tile, the merged rows of lane quarter q are then merged across the
// cluster by chunk q % nchunk: the others push theirs into its shared memory (as the pair path does).
// Returns false when a wait expired.
__device__ __forceinline__ bool intra_epilogue(uint8_t *smem, Bars *bars, const Params &p, const Item &I,
                                            uint32_t tl, int x, int quarter, int lane, int row, int g,
                                            float m_row, float l_row) {
    Stream &S = bars->st[x];
    if (!warp_wait(&S.o_done, (g - 1) & 1, p.timeout_ns)) return false;  // this group's last PV
    tc_fence_after();
    float2 *xch = reinterpret_cast<float2 *>(smem + OFF_XCH);
    if (x == 1) {
        xch[row] = make_float2(m_row, l_row);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->xm[quarter]);
        return true;
    }
    float o[HD];
    {
        uint32_t v[2][32];
        tmem_ld32(tl + TCOL_O, v[0]);
        tmem_ld32(tl + TCOL_O + 32, v[1]);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = __uint_as_float(v[i >> 5][i & 31]);
    }
    float m = m_row, l = l_row;
    if (I.nk[1] > 0) {  // B's rows: wait for its hand-over, then combine
        if (!warp_wait(&bars->xm[quarter], 0, p.timeout_ns)) return false;
        tc_fence_after();
        const float2 mlb = xch[row];
        const float M = fmaxf(m, mlb.x);
        const float wa = ex2_approx(m - M), wb = ex2_approx(mlb.x - M);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t v[32];
            tmem_ld32(tl + TCOL_O + HD + 32 * h, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[32 * h + i] = fmaf(wb, __uint_as_float(v[i]), wa * o[32 * h + i]);
        }
        l = fmaf(wb, mlb.y, wa * l);
        m = M;
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.o_free);
    const int nc = I.nchunk;
    const int km = nc > 1 ? quarter % nc : I.chunk;  // the chunk that merges these rows
    int first = 0;  // the merging CTA's receive slots: after those of the quarters it merges before this one
    for (int q2 = 0; q2 < quarter; ++q2)
        if (q2 % nc == km) first += nc - 1;
    if (I.chunk != km) {
        const int slot = first + (I.chunk < km ? I.chunk : I.chunk - 1);
        const uint32_t rank = cluster_rank() - static_cast<uint32_t>(I.chunk) + static_cast<uint32_t>(km);
        const uint32_t dst = dsmem_addr(smem_u32(smem + recv_slot(slot, p.kv_chunk)), rank);
        const uint32_t bar = dsmem_addr(smem_u32(&bars->recv[0][quarter]), rank);
#pragma unroll
        for (int c4 = 0; c4 < HD / 4; ++c4)
            st_async_v4(dst + (c4 * 32 + lane) * 16, make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]),
                        bar);
        st_async_v2(dst + PART_O_BYTES + lane * 8, m, l, bar);
        return true;
    }
    if (nc > 1) {
        if (!warp_wait(&bars->recv[0][quarter], 0, p.timeout_ns)) return false;
        const uint32_t in0 = smem_u32(smem) + static_cast<uint32_t>(lane) * 16u;
        float mk[MAX_CLUSTER - 1], lk[MAX_CLUSTER - 1];
        float M = m;
#pragma unroll
        for (int k = 0; k < MAX_CLUSTER - 1; ++k) {
            mk[k] = -INFINITY;
            lk[k] = 0.f;
            if (k < nc - 1) {
                const float2 ml = lds_v2(smem_u32(smem) + recv_slot(first + k, p.kv_chunk) + PART_O_BYTES + lane * 8);
                mk[k] = ml.x;
                lk[k] = ml.y;
                M = fmaxf(M, ml.x);
            }
        }
        const float ws = ex2_approx(m - M);
        l *= ws;
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] *= ws;
#pragma unroll
        for (int k = 0; k < MAX_CLUSTER - 1; ++k) {
            if (k < nc - 1) {
                const float w = ex2_approx(mk[k] - M);
                l = fmaf(w, lk[k], l);
                const uint32_t in = in0 + recv_slot(first + k, p.kv_chunk);
                float4 q[HD / 4];
#pragma unroll
                for (int c4 = 0; c4 < HD / 4; ++c4) q[c4] = lds_v4(in + c4 * 512);
#pragma unroll
                for (int c4 = 0; c4 < HD / 4; ++c4) {
                    o[4 * c4] = fmaf(w, q[c4].x, o[4 * c4]);
                    o[4 * c4 + 1] = fmaf(w, q[c4].y, o[4 * c4 + 1]);
                    o[4 * c4 + 2] = fmaf(w, q[c4].z, o[4 * c4 + 2]);
                    o[4 * c4 + 3] = fmaf(w, q[c4].w, o[4 * c4 + 3]);
                }
            }
        }
    }
    const float inv_l = 1.f / l;
    const int qrow = I.pair * BM + row;
    if (qrow < p.T) {
        uint4 *dst = reinterpret_cast<uint4 *>(p.att + I.b * p.att_seq_stride + static_cast<long long>(qrow) * p.E +
                                               I.h * HD);
#pragma unroll
        for (int q = 0; q < HD / 8; ++q)
            dst[q] = make_uint4(pack_half2(o[8 * q] * inv_l, o[8 * q + 1] * inv_l),
                                pack_half2(o[8 * q + 2] * inv_l, o[8 * q + 3] * inv_l),
                                pack_half2(o[8 * q + 4] * inv_l, o[8 * q + 5] * inv_l),
                                pack_half2(o[8 * q + 6] * inv_l, o[8 * q + 7] * inv_l));
    }
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
    // Split launches: every peer of the cluster has initialised its receive barriers (the cluster
    // barrier's arrival follows the set-up of every CTA) before this warp pushes into one.
    if (kSplit) cluster_wait();
    Item I;
    for (int it = 0; ok && get_item<kSplit>(p, it, I); ++it) {
        const int nk = I.nk_of(x);
        if (nk == 0) continue;     // this query tile has no keys in this unit of work
        // this group's tile (in its own order) holding its query tile's diagonal, if any
        int diag_j = 2 * I.pair + x - I.kv0;
        if (kSplit && p.intra) {
            const int jd = I.pair - I.kv0;
            diag_j = (jd & 1) == x ? jd >> 1 : -1;
        }
        float m_used = -INFINITY;  // running max (log2 units) used for the exponentials
        float l = 0.f;             // running sum of the (fp16-rounded) exponentials
        for (int j = 0; j < nk; ++j, ++g) {
            ok = warp_wait(&S.s_full, g & 1, to);
            if (!ok) break;
            tc_fence_after();
            float xs[BN];
            {
                uint32_t v[4][32];
                if constexpr (kSplit) {  // (split launches measured faster with the narrow loads)
#pragma unroll
                    for (int cb = 0; cb < 4; ++cb) tmem_ld32(tS + 32 * cb, v[cb]);
                } else {
                    tmem_ld64(tS, *reinterpret_cast<uint32_t(*)[2][32]>(&v[0]));
                    tmem_ld64(tS + 64, *reinterpret_cast<uint32_t(*)[2][32]>(&v[2]));
                }
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
            // (the ones the PV MMA consumes: numerator and denominator use identical weights). The
            // scale-and-subtract runs two columns per instruction on the packed fp32 pipe; the block is
            // bound by instruction issue, not by the MUFU.
            uint32_t pk[4][16];
            float ps[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) ps[k] = 0.f;
            const uint64_t c2 = pair_f32(c, c), nm2 = pair_f32(neg_m, neg_m);
#pragma unroll
            for (int cb = 0; cb < 4; ++cb) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float e0, e1;
                    fma2_f32(e0, e1, xs[32 * cb + 2 * i], xs[32 * cb + 2 * i + 1], c2, nm2);
                    const float p0 = ex2_approx(e0);
                    const float p1 = ex2_approx(e1);
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
            if constexpr (kSplit) {
#pragma unroll
                for (int cb = 0; cb < 4; ++cb) tmem_st16(tP + 16 * cb, pk[cb]);
            } else {
                tmem_st64(tP, pk);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.p_full);
        }
        if (!ok) break;
        if (kSplit) {  // split launches: these warps finish their own rows (A and B in parallel)
            ok = p.intra ? intra_epilogue(smem, bars, p, I, tl, x, quarter, lane, row, g, m_used, l)
                         : split_epilogue(smem, bars, p, I, tO, x, quarter, lane, row, g, m_used, l);
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
// its 32 rows (rows past T are clipped by the tensor map). Split launches do not use these warps.
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
                       const __grid_constant__ CUtensorMap tm_kv, const Params p, const SplitArg<kSplit> tab) {
    extern __shared__ __align__(1024) uint8_t smem[];
    Bars *bars = reinterpret_cast<Bars *>(smem + OFF_BAR);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Split launches run in clusters: every thread takes part in both cluster barriers (the one after
    // set-up and the one before exit), also on the uniform early exits below.
    if constexpr (kSplit) {
        if (threadIdx.x == 0) {
            const int idx = tab.cta_item[blockIdx.x];
            s_split_valid = idx >= 0;
            if (idx >= 0) decode_item<true>(p, idx, s_split_unit);
        }
        __syncthreads();
    }
    const bool misaligned = (smem_u32(smem) & 1023u) != 0;  // SW128 tiles need 1024-byte alignment
    if (misaligned || (kSplit && !s_split_valid)) {
        if (misaligned && threadIdx.x == 0) atomicOr(p.status, ST_PREFILL_SMEM_ALIGN);
        if (kSplit) {
            cluster_sync_all();
            cluster_sync_all();
        }
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
        if (kSplit)
            for (int q = 0; q < 4; ++q) mbar_init(&bars->xm[q], 1);
        bars->abort = 0;
        if (kSplit)
            for (int x = 0; x < 2; ++x)
                for (int q = 0; q < 4; ++q) mbar_init(&bars->recv[x][q], 1);
        fence_mbar_init();
        tma_prefetch_desc(&tm_qkv);
        tma_prefetch_desc(&tm_att);
        if (p.kv_fill) tma_prefetch_desc(&tm_kv);
        // The first item's Q tiles and its first K and V tiles into L2 while the previous kernel
        // drains (the producer's first loads, issued after the dependency wait, then hit L2).
        Item i0;
        if (get_item<kSplit>(p, 0, i0)) {
            for (int t = 0; t < (((kSplit && p.intra) || !i0.nk[1]) ? 1 : 2); ++t)
                tma_prefetch_l2_3d(&tm_qkv, i0.h * HD, item_qtile<kSplit>(p, i0, t) * BM, i0.b);
            tma_prefetch_l2_3d(&tm_qkv, p.E + i0.h * HD, i0.kv0 * BN, i0.b);
            tma_prefetch_l2_3d(&tm_qkv, 2 * p.E + i0.h * HD, i0.kv0 * BN, i0.b);
        }
    }
    if (warp == MMA_WARP) {
        tmem_alloc(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    // Launched as a programmatic dependent: the set-up above touches no global memory, so it overlaps
    // the previous kernel's tail; every global access (inputs, output, cache) follows this
    // wait. Dependents may start placing CTAs at once (they wait the same way before any access).
    grid_dependency_wait();
    grid_launch_dependents();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (kSplit) {
        // A softmax warp whose 32 rows this CTA merges sets its receive barrier to expect the other
        // chunks' bytes; their pushes follow the cluster barrier (the fence orders this before it).
        if (warp >= SOFT_WARP0 && warp < EPI_WARP0 && lane == 0) {
            const int x = (warp - SOFT_WARP0) / NSOFT_WARPS, q = warp & 3;
            Item iu;
            if (get_item<true>(p, 0, iu)) {
                // pair units: group 4 x + q over the chunks holding x's keys; single-query-tile units:
                // lane quarter q (merged by group A's warps) over all chunks
                const int ncx = p.intra ? (x == 0 ? iu.nchunk : 0) : tile_chunks(p, iu.pair, x);
                if (ncx > 1 && (p.intra ? q : 4 * x + q) % ncx == iu.chunk) {
                    mbar_arrive_expect_tx(&bars->recv[x][q], (ncx - 1) * PART_BYTES);
                    fence_cluster();
                }
            }
        }
        __syncwarp();
        cluster_arrive_relaxed();  // waited for by the softmax warps before their first push
    }
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

    if (kSplit && (warp < SOFT_WARP0 || warp >= EPI_WARP0)) cluster_wait();  // (softmax warps waited)
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
    // No CTA of a cluster exits while a peer may still push into its shared memory.
    if (kSplit) cluster_sync_all();
}

// ------------------------------------------------------------------ host side

// Split launches. Time model in units of one step of a unit (both softmax groups each process one K/V
// tile, ~1.75 us): a unit costs its steps plus a fixed part fitted to back-to-back one-layer launches
// on B200 (first loads, epilogue, and for split units the cluster barriers and merges): ~2.2 steps for
// a whole pair, ~6 for a chunk of a pair, whose rows are pushed to and merged in its cluster, ~4.5 for
// a chunk of one query tile, whose two groups merge locally and push a quarter of the rows per other
// chunk. A split launch places every unit at once (one CTA each), so it costs its longest unit; it is
// used when that clearly beats the longest whole pair.
constexpr double WHOLE_OVERHEAD = 2.2;
constexpr double SPLIT_OVERHEAD = 6.0;
constexpr double INTRA_OVERHEAD = 4.5;

static int pair_kv_tiles_host(int n_qtiles, int pr) { return (2 * pr + 1 < n_qtiles) ? 2 * pr + 2 : 2 * pr + 1; }

// Receive slots a CTA needs at most with chunk size cs: over every chunk k of every pair, the
// partials of the other chunks for each 32-row group that k merges (group g of query tile x is merged
// by chunk g % nx, nx = chunks holding x's keys). Single-query-tile units: lane quarter q of a tile in
// nc chunks is merged by chunk q % nc.
static int recv_slots_needed(int n_qtiles, int n_pairs, int cs, bool intra) {
    int need = 0;
    if (intra) {
        const int nc = (n_qtiles - 1 + cs) / cs;  // the longest query tile's chunks
        for (int n = 2; n <= nc; ++n)
            for (int k = 0; k < n; ++k) need = std::max(need, ((3 - k) / n + 1) * (n - 1));
        return need;
    }
    for (int pr = 0; pr < n_pairs; ++pr) {
        int nx[2];
        for (int x = 0; x < 2; ++x) nx[x] = (2 * pr + x < n_qtiles) ? (2 * pr + x + cs) / cs : 0;
        for (int k = 0; k < std::max(nx[0], nx[1]); ++k) {
            int n = 0;
            for (int g = 0; g < 8; ++g) {
                const int c = nx[g >> 2];
                if (c > 1 && g % c == k) n += c - 1;
            }
            need = std::max(need, n);
        }
    }
    return need;
}

// Receive slots a split CTA has (recv_slot): the second Q buffer, the output slots and statistics, and
// the K stages past the unit's at most cs K/V tiles.
static int recv_slots_available(int cs) {
    return RECV_Q_SLOTS + RECV_OUT_SLOTS + std::max(0, NSTAGE - cs) * TILE_BYTES / PART_BYTES;
}

// Chunks of entry e of a (head, sequence) with chunk size cs: pair e, or query tile e of
// single-query-tile units.
static int entry_chunks(int n_qtiles, int e, int cs, bool intra) {
    return intra ? (e + cs) / cs : (pair_kv_tiles_host(n_qtiles, e) + cs - 1) / cs;
}

// Places the units of a split launch, entries (pairs, or query tiles) in decreasing size, each entry's
// chunks on consecutive ranks of one cluster of cl CTAs (first fit). Writes the CTA -> item table when
// `cta_item` is given (entries of unused ranks stay as they are). Returns the number of clusters, or
// -1 above max_clusters. Sets *units to the units per (head, sequence).
static int place_split_units(int n_qtiles, int n_pairs, int hb, int cs, int cl, bool intra, int max_clusters,
                             short *cta_item, int *units) {
    const int n_entries = intra ? n_qtiles : n_pairs;
    int nc[128], ubase[128];
    if (n_entries > 128) return -1;
    int u = 0;
    for (int pr = n_entries - 1; pr >= 0; --pr) {  // get_item's unit numbering: entries from the last
        nc[pr] = entry_chunks(n_qtiles, pr, cs, intra);
        ubase[pr] = u;
        u += nc[pr];
    }
    *units = u;
    int fill[MAX_SPLIT_CTAS];
    int clusters = 0;
    for (int pr = n_entries - 1; pr >= 0; --pr) {
        for (int b = 0; b < hb; ++b) {
            int c = 0;
            while (c < clusters && fill[c] + nc[pr] > cl) ++c;
            if (c == clusters) {
                if (clusters >= max_clusters || clusters >= MAX_SPLIT_CTAS) return -1;
                fill[clusters++] = 0;
            }
            if (cta_item)
                for (int k = 0; k < nc[pr]; ++k)
                    cta_item[c * cl + fill[c] + k] = static_cast<short>((ubase[pr] + k) * hb + b);
            fill[c] += nc[pr];
        }
    }
    return clusters;
}

// Clusters of cl split CTAs that fit on the device at once (cached per context; 0 when unknown).
static int max_active_clusters(DeviceContext *ctx, int cl) {
    if (cl < 1 || cl > MAX_CLUSTER) return 0;
    if (ctx->pf_active_clusters[cl] == 0) {
        RelaxedCapture relaxed;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(cl));
        cfg.blockDim = dim3(NTHREADS);
        cfg.dynamicSmemBytes = SMEM_BYTES;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(cl);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k_flash_prefill_tc<true>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = -1;
        }
        ctx->pf_active_clusters[cl] = n > 0 ? n : -1;
    }
    return std::max(0, ctx->pf_active_clusters[cl]);
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

// A launch's split plan (cs == 0: whole pairs) and its CTA -> unit table.
struct SplitPlan {
    int device, T, H, B;
    int cs, cl, clusters, units;
    bool intra;
    b200::prefill::SplitTable tab;
};
constexpr int kPlanCache = 8;
thread_local SplitPlan t_plans[kPlanCache];
thread_local bool t_plan_valid[kPlanCache];
thread_local int t_plan_next = 0;

const SplitPlan *cached_split_plan(const DeviceContext *ctx, int T, int H, int B) {
    for (int i = 0; i < kPlanCache; ++i)
        if (t_plan_valid[i] && t_plans[i].device == ctx->device && t_plans[i].T == T && t_plans[i].H == H &&
            t_plans[i].B == B)
            return &t_plans[i];
    return nullptr;
}

const SplitPlan *remember_split_plan(const SplitPlan &plan) {
    const int i = t_plan_next;
    t_plan_next = (t_plan_next + 1) % kPlanCache;
    t_plans[i] = plan;
    t_plan_valid[i] = true;
    return &t_plans[i];
}
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
        RelaxedCapture relaxed;
        for (const void *fn : {reinterpret_cast<const void *>(k_flash_prefill_tc<false>),
                               reinterpret_cast<const void *>(k_flash_prefill_tc<true>)}) {
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
    // Fewer whole pairs than SMs: split the longest key ranges into chunks when one wave of clusters
    // of the chunks clearly beats the longest whole pair: chunks of pairs, or chunks of single query
    // tiles whose two softmax groups take alternate K/V tiles (half the steps per chunk). The plan is
    // host work that a back-to-back stream of one-layer launches would notice, so recent plans are
    // kept per thread (the reference's forward pass calls attention with the same shape per layer).
    const SplitPlan *plan = cached_split_plan(ctx, T, H, B);
    if (!plan) {
        SplitPlan np{};
        np.device = ctx->device;
        np.T = T;
        np.H = H;
        np.B = B;
        if (hb * p.n_pairs < sms) {
            const int nkv_max = pair_kv_tiles_host(p.n_qtiles, p.n_pairs - 1);
            double best = (nkv_max + WHOLE_OVERHEAD) * 0.97;
            for (int intra = 0; intra < 2; ++intra) {
                const int longest = intra ? p.n_qtiles : nkv_max;  // K/V tiles of the longest entry
                for (int cs = longest - (intra ? 0 : 1); cs >= 1; --cs) {
                    const int cl = (longest + cs - 1) / cs;
                    if (cl > MAX_CLUSTER) break;
                    const double t = (intra ? (cs + 1) / 2 : cs) + (intra ? INTRA_OVERHEAD : SPLIT_OVERHEAD);
                    if (t >= best) continue;
                    if (recv_slots_needed(p.n_qtiles, p.n_pairs, cs, intra) > recv_slots_available(cs)) continue;
                    const int max_clusters =
                        std::min(max_active_clusters(ctx, cl), std::min(sms, MAX_SPLIT_CTAS) / cl);
                    int units = 0;
                    const int n = place_split_units(p.n_qtiles, p.n_pairs, static_cast<int>(hb), cs, cl,
                                                    intra != 0, max_clusters, nullptr, &units);
                    if (n <= 0) continue;
                    best = t;
                    np.cs = cs;
                    np.cl = cl;
                    np.clusters = n;
                    np.units = units;
                    np.intra = intra != 0;
                }
            }
        }
        if (np.cs > 0) {
            for (int i = 0; i < MAX_SPLIT_CTAS; ++i) np.tab.cta_item[i] = -1;
            int units = 0;
            place_split_units(p.n_qtiles, p.n_pairs, static_cast<int>(hb), np.cs, np.cl, np.intra, np.clusters,
                              np.tab.cta_item, &units);
        }
        plan = remember_split_plan(np);
    }
    const int split_cs = plan->cs, split_cl = plan->cl, split_clusters = plan->clusters;
    p.intra = plan->intra ? 1 : 0;
    if (split_cs > 0) {
        p.kv_chunk = split_cs;
        p.units_per_hb = plan->units;
    }
    const long long total = static_cast<long long>(p.units_per_hb) * hb;
    if (total <= 0) return GPT2_B200_OK;
    if (total > 0x7fffffffLL) return GPT2_B200_EINVAL;
    p.total_items = static_cast<int>(total);
    p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(HD)));
    p.status = ctx->status;
    p.timeout_ns = wait_timeout_ns();
    // Whole pairs: persistent, at most CTAS_PER_SM resident CTAs per SM, each looping over its share
    // of items. Split: one CTA per unit in clusters of split_cl.
    const long long slots = static_cast<long long>(CTAS_PER_SM) * sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(split_cs > 0 ? split_clusters * split_cl : (total < slots ? total : slots)));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(split_cl);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = split_cs > 0 ? 2 : 1;
    const cudaError_t err = split_cs > 0
                                ? cudaLaunchKernelEx(&cfg, k_flash_prefill_tc<true>, tm, tm_att, tm_kv, p, plan->tab)
                                : cudaLaunchKernelEx(&cfg, k_flash_prefill_tc<false>, tm, tm_att, tm_kv, p,
                                                     NoSplitTable{});
    return err == cudaSuccess ? GPT2_B200_OK : GPT2_B200_ECUDA;
}

}  // namespace b200
