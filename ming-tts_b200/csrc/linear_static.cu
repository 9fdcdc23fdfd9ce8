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

constexpr int kMaxDevices = 64;
std::atomic<uint16_t*> g_scratch[kMaxDevices];
std::atomic<int> g_sm_count[kMaxDevices];
std::mutex g_setup;

// The array's name is only a host-side stand-in in host code; the device address comes from
// cudaGetSymbolAddress, resolved once per device with that device current.
mt_status device_scratch(int dev, uint16_t** out, int* sms) {
    uint16_t* p = g_scratch[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_setup);
        p = g_scratch[dev].load(std::memory_order_relaxed);
        if (!p) {
            void* addr = nullptr;
            if (cudaGetSymbolAddress(&addr, g_static_scratch) != cudaSuccess || !addr) return MT_ERR_CUDA;
            int count = 0;
            if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return MT_ERR_CUDA;
            g_sm_count[dev].store(count, std::memory_order_relaxed);
            p = static_cast<uint16_t*>(addr);
            g_scratch[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
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
    int sms = 0;
    mt_status st = device_scratch(dev, &scratch, &sms);
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
    run_gemm_plan(plan, s);
    return cudaGetLastError() == cudaSuccess ? MT_OK : MT_ERR_CUDA;
}
