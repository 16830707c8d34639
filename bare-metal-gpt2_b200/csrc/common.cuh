// common.cuh — shared definitions for the B200 attention library (internal).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gpt2_b200.h"

namespace b200 {

// Device status-word bits. Kernels OR these into a per-device word instead of trapping; the host
// reads them with gpt2_b200_status().
enum StatusBits : unsigned {
    ST_PREFILL_LOAD_TIMEOUT = 1u << 0,     // TMA producer gave up waiting for a free stage
    ST_PREFILL_MMA_TIMEOUT = 1u << 1,      // MMA issuer gave up waiting for data / softmax
    ST_PREFILL_SOFTMAX_TIMEOUT = 1u << 2,  // softmax warps gave up waiting for the MMA
    ST_PREFILL_SMEM_ALIGN = 1u << 3,       // dynamic shared memory not 1024-byte aligned
    ST_PREFILL_DRAIN_TIMEOUT = 1u << 4,    // teardown could not confirm in-flight copies / MMAs
    ST_DECODE_BAD_LEN = 1u << 8,           // device-side length outside [1, maxT]
    ST_DECODE_TIMEOUT = 1u << 10,          // a decode stage wait gave up
    ST_KV_BAD_POS = 1u << 9,               // device-side append position outside [0, maxT)
    ST_LINEAR_TIMEOUT = 1u << 11,          // a batched linear layer's stage wait gave up
    ST_MODEL_BAD_TOKEN = 1u << 12,         // a token id outside [0, vocab) reached the embedding
    ST_TEST_WAIT_TIMEOUT = 1u << 16,       // the wait-timeout self-test expired (expected)
};

// Default bound on any single mbarrier wait inside a kernel (wall clock). A correct kernel waits
// microseconds; the bound only matters when something is broken.
constexpr unsigned long long kDefaultWaitTimeoutNs = 2000000000ull;

struct DeviceContext {
    unsigned *status = nullptr;     // one word, zero = healthy
    float *part = nullptr;          // decode split partials
    unsigned *counters = nullptr;   // decode split-arrival counters (kept at zero between calls)
    size_t part_floats = 0;
    size_t counter_words = 0;
    int pf_active_clusters[5] = {0, 0, 0, 0, 0};  // prefill split clusters of n CTAs that fit (0 = not asked)
    bool prefill_attr_done = false;
    bool decode_attr_done = false;
    int num_sms = 0;
    int device = 0;                 // CUDA device ordinal of this context
};

// Returns the context of the current device (creating it on first use), or nullptr on CUDA error.
DeviceContext *device_context();

// Scope in which this thread's potentially unsafe CUDA calls (allocation, attribute set-up, occupancy
// queries: one-time host work that enqueues nothing on the caller's stream) do not invalidate a
// graph capture it may be running: the thread's capture mode is relaxed for the scope.
struct RelaxedCapture {
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    RelaxedCapture() { cudaThreadExchangeStreamCaptureMode(&mode); }
    ~RelaxedCapture() { cudaThreadExchangeStreamCaptureMode(&mode); }
    RelaxedCapture(const RelaxedCapture &) = delete;
    RelaxedCapture &operator=(const RelaxedCapture &) = delete;
};

// The driver's cuTensorMapEncodeTiled, looked up once through the runtime (nullptr when the driver
// lacks it). Shared by every kernel that builds TMA tensor maps.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encoder();
unsigned long long wait_timeout_ns();
void set_last_error(int code);

}  // namespace b200
