// linear.cuh — batched linear layers of the GPT-2 decode step (internal interface).
//
// y[b, n] = epilogue( sum_k x[b, k] * W[n, k] + bias[n] ) for the B sequences of one decode step:
// W is a reference weight tensor [N, K] (row-major, cuda/kernels.cuh:19-23, model/weights.h:4-6),
// x is [B, K] fp16 activations. The reference computes each sequence with an M=1 GEMV
// (k_gemv_fp16, cuda/kvcache.cu:150-170); here the B rows share one pass over W on tcgen05.
#pragma once
#include "common.cuh"

namespace b200 {
namespace lin {

constexpr int BM = 128;                 // weight rows (output features) per tile: the MMA's M
constexpr int KA = 64;                  // K elements per atom: one 128-byte swizzle row
constexpr int MAX_STAGES = 4;           // atoms in flight per CTA
constexpr int HEAD_STAGES = 2;          // ... for the tied head (many tiles: occupancy matters more)
constexpr int NT = 128;                 // 4 warps (one per TMEM lane quarter)
constexpr int W_ATOM_BYTES = BM * 128;  // 16 KiB
constexpr int MAX_BPAD = 256;           // MMA N limit
constexpr int MAX_CLUSTER = 8;          // CTAs that split one tile's K range
// Split-K reduction: up to this padded batch each CTA pushes its partial columns into the owners'
// receive buffers (one cluster barrier, local sums); above it the owners pull them from the
// peers' staged tiles (no separate receive buffer, two barriers). Measured on B200: pushing wins
// at B = 8 (451 -> 421 us per decode step), pulling at B = 64 (669 vs 769 us).
constexpr int PUSH_MAX_BPAD = 32;

// What the epilogue does with h = fp16(acc + bias[n]) (the reference's GEMV rounding).
enum Epi : int {
    EPI_STORE = 0,  // out[b, n] = h
    EPI_GELU = 1,   // out[b, n] = fp16(gelu_new(h))          (be->gelu on the GEMV output)
    EPI_RESID = 2,  // out[b, n] = fp16(out[b, n] + h)        (be->add, the residual)
    EPI_QKV = 3,    // out[b, n] = h, and K/V columns appended to sequence b's cache at d_pos[b]
    EPI_HEAD = 4,   // logits (optional) and per-tile argmax keys of fp16(acc) (tied head, no bias)
};

struct Params {
    int N, K, B, bpad;      // output features, inner dim, sequences, MMA N (B rounded up to 16)
    int atoms, cs, n_tiles; // K / 64, CTAs per tile (cluster), ceil(N / 128)
    int nstage;             // ring depth in atoms
    int tcols;              // TMEM columns allocated (power of two >= 32)
    int cpr4;               // split K: batch columns reduced by each rank (multiple of 4)
    int push;               // split K: partials pushed to their owner (else pulled from peers)
    int extra_bytes;        // shared memory between the barriers and the receive buffer
    const __half *bias;     // [N] or null
    __half *out;            // [B][ldo] (EPI_HEAD: logits, may be null)
    long long ldo;
    // EPI_QKV
    __half *const *k_dst;   // [B] K slab base of this layer for each sequence ([H][maxT][D])
    __half *const *v_dst;   // [B] V slab base
    const int *d_pos;       // [B] position of this step
    int maxT, E;
    // EPI_HEAD
    unsigned long long *amax;  // [B][n_tiles] argmax keys
    unsigned *status;
    unsigned long long timeout_ns;
};

struct Plan {
    CUtensorMap tm_w, tm_x;
    Params p;
    int epi;
    dim3 grid;
    size_t smem;
    bool pdl;  // launch as a programmatic dependent of the previous kernel in the stream
};

// Builds a launch plan (tensor maps, tile split). cs = 0 picks the split from the grid size.
// Returns a GPT2_B200_* code.
int plan_linear(Plan *pl, int epi, const __half *W, int N, int K, const __half *X, long long ldx,
                int B, const __half *bias, __half *out, long long ldo, int cs, int num_sms);
int launch_linear(const Plan &pl, cudaStream_t stream);
// Applies the plan's kernel attributes on the current device without launching (call before a
// stream capture that will launch it).
int prepare_linear(const Plan &pl);

// Orderable 64-bit argmax key of an fp16-valued logit at vocabulary index n: larger value wins,
// ties go to the smaller index (first occurrence, as an argmax over the logits row).
__host__ __device__ inline unsigned long long argmax_key(float v, unsigned n) {
#ifdef __CUDA_ARCH__
    const unsigned u = __float_as_uint(v);
#else
    unsigned u;
    __builtin_memcpy(&u, &v, 4);
#endif
    const unsigned o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(o) << 32) | (0xFFFFFFFFu - n);
}
__host__ __device__ inline int argmax_key_index(unsigned long long key) {
    return static_cast<int>(0xFFFFFFFFu - static_cast<unsigned>(key & 0xFFFFFFFFull));
}

}  // namespace lin
}  // namespace b200
