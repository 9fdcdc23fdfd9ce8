// linear_static.cu -- mt_linear_static: the tensor-core linear with its scratch in a static device
// array, for callers that cannot allocate device memory.
//
// Some hosts cannot call cudaMalloc at all: code that runs inside another framework's memory pool
// or arena (which owns every device allocation), or a plugin driven from a real-time or audio
// thread, where an allocation may block on a device-wide lock. The tensor-core route of mt_linear
// needs scratch for the bf16 hi/lo split of the fp32 activations and takes it from the context
// (cudaMalloc on first use). This entry point uses a fixed array compiled into the library instead,
// so it needs no context and allocates nothing.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace {

// Activations one call can hold: m * k <= 1,048,576 (for example 1024 rows of 1024). The hi and lo
// planes take 2 bytes each per activation: 4 MiB, held on every GPU that loads the library. No
// part of it has to start at zero: every call writes the m * k entries of both planes it then reads.
constexpr size_t kStaticMaxActivations = size_t(1) << 20;
static __device__ __align__(256) uint16_t g_static_scratch[2 * kStaticMaxActivations];
// Status word of these calls on this GPU, laid out as a context's ([0] code, [1] site, [2] detail,
// [3] wait limit, 0 = the default): a bounded wait of the GEMM that gives up records itself here.
static __device__ __align__(16) unsigned int g_static_status[4];

std::atomic<uint16_t*> g_scratch[mt::kMaxDevices];
std::atomic<unsigned int*> g_status[mt::kMaxDevices];
std::atomic<int> g_sm_count[mt::kMaxDevices];
std::mutex g_setup;

// The arrays' names are only host-side stand-ins in host code; their device addresses come from
// cudaGetSymbolAddress, resolved once per device with that device current.
mt_status device_scratch(int dev, uint16_t** out, unsigned int** status, int* sms) {
    uint16_t* p = g_scratch[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_setup);
        p = g_scratch[dev].load(std::memory_order_relaxed);
        if (!p) {
            void* addr = nullptr;
            void* st = nullptr;
            if (cudaGetSymbolAddress(&addr, g_static_scratch) != cudaSuccess || !addr) return MT_ERR_CUDA;
            if (cudaGetSymbolAddress(&st, g_static_status) != cudaSuccess || !st) return MT_ERR_CUDA;
            int count = 0;
            if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return MT_ERR_CUDA;
            g_sm_count[dev].store(count, std::memory_order_relaxed);
            g_status[dev].store(static_cast<unsigned int*>(st), std::memory_order_relaxed);
            p = static_cast<uint16_t*>(addr);
            g_scratch[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    *status = g_status[dev].load(std::memory_order_relaxed);
    *sms = g_sm_count[dev].load(std::memory_order_relaxed);
    return MT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

using namespace mt;

extern "C" mt_status mt_linear_static(void* stream, const float* x, int ldx, int m, const mt_bf16* w,
                                      const mt_bf16* w2, const mt_bf16* bias, int n, int k, float* y, int ldy,
                                      uint32_t flags) {
    if (!x || !w || !y) return MT_ERR_ARG;
    if ((flags & ~31u) != 0) return MT_ERR_ARG;
    if ((flags & MT_LINEAR_SILU_GATE) && !w2) return MT_ERR_ARG;
    if ((flags & MT_LINEAR_BIAS) && !bias) return MT_ERR_ARG;
    if (m < 0 || n <= 0 || k <= 0 || k % 8 != 0 || ldx < k || ldx % 4 != 0 || ldy < n) return MT_ERR_SHAPE;
    if (!aligned16(x) || !aligned16(w) || (w2 && !aligned16(w2))) return MT_ERR_ARG;
    if (m == 0) return MT_OK;
    if ((size_t)m * (size_t)k > kStaticMaxActivations) return MT_ERR_CAPACITY;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MT_ERR_CUDA;
    uint16_t* scratch = nullptr;
    unsigned int* status = nullptr;
    int sms = 0;
    mt_status st = device_scratch(dev, &scratch, &status, &sms);
    if (st != MT_OK) return st;
    cudaStream_t s = as_stream(stream);
    // The planes are rewritten in full for the m x k activations of this call before the GEMM
    // reads them, so nothing left by an earlier call is read.
    uint16_t* hi = scratch;
    uint16_t* lo = scratch + (size_t)m * k;
    launch_split(x, ldx, m, k, hi, lo, k, sms, s);
    LinearArgs a{};
    a.x_hi = hi; a.x_lo = lo; a.ld_split = k; a.m = m; a.n = n; a.k = k; a.w = w; a.w2 = w2; a.bias = bias;
    a.y = y; a.ldy = ldy; a.flags = flags; a.split_k = 1;
    GemmPlan plan;
    st = make_gemm_plan_bare(sms, a, &plan);
    if (st != MT_OK) return st;
    plan.e.status = status;
    run_gemm_plan(plan, s);
    // Peek, not get: the launches are checked without clearing an error that belongs to the caller.
    return cudaPeekAtLastError() == cudaSuccess ? MT_OK : MT_ERR_CUDA;
}

extern "C" mt_status mt_linear_static_status(void* stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MT_ERR_CUDA;
    if (cudaStreamSynchronize(as_stream(stream)) != cudaSuccess) return MT_ERR_CUDA;
    // Before the first mt_linear_static on this device nothing can have been recorded.
    if (!g_scratch[dev].load(std::memory_order_acquire)) return MT_OK;
    unsigned int word[3] = {0, 0, 0};
    if (cudaMemcpyFromSymbol(word, g_static_status, sizeof(word)) != cudaSuccess) return MT_ERR_CUDA;
    if (word[0] == DEV_OK) return MT_OK;
    const unsigned int zero[3] = {0, 0, 0};
    if (cudaMemcpyToSymbol(g_static_status, zero, sizeof(zero)) != cudaSuccess) return MT_ERR_CUDA;
    return word[0] == DEV_TIMEOUT ? MT_ERR_TIMEOUT : MT_ERR_ARG;
}
