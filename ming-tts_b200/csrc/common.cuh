// common.cuh -- helpers shared by the sm_100a kernels and the C-ABI glue of libmingcuda.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <utility>

#include "../../include/mingcuda.h"

// ------------------------------------------------------------------------------------------------
// Context (host side). One per device; owns the device status word that bounded waits write and
// a scratch area for the fp32 -> bf16 hi/lo split of mt_linear's tensor-core route.
// ------------------------------------------------------------------------------------------------
struct mt_ctx {
    int device = 0;
    int sm_count = 0;
    unsigned int* d_status = nullptr;  // [0] = error code, [1] = site id, [2] = detail, [3] = wait limit (us)
    void* scratch = nullptr;           // grows on demand, see mt_scratch()
    size_t scratch_bytes = 0;
    int gemm_pairs = -1;               // tensor-core GEMM CTA pairs: -1 automatic, 0 never, 1 where valid
    int persistent = 0;                // small-batch stacks: 1 the persistent stack kernel where it fits, 0 never
    void* stack_area = nullptr;        // mt_qwen_decode's persistent-stack area (zeroed at allocation)
    size_t stack_area_bytes = 0;
    float* rope = nullptr;             // [32] NeoX rotation frequencies for rope_theta (mt_qwen_decode)
    float rope_theta = 0.f;
    std::string err;
};

namespace mt {

// Status word codes written by kernels (d_status[0]).
enum : unsigned int { DEV_OK = 0, DEV_TIMEOUT = 1, DEV_BAD_ARG = 2 };

mt_status fail(mt_ctx* ctx, mt_status code, const char* fmt, ...);
// Hands a model's arena (from mt_model_create_from_arena) to the model: mt_model_destroy frees it.
void model_own_arena(mt_model* m);
void encoder_own_arena(mt_encoder* e);
mt_ctx* encoder_ctx(const mt_encoder* e);
int encoder_latent_dim(const mt_encoder* e);
mt_status check_launch(mt_ctx* ctx, const char* what);
// Returns a device buffer of at least `bytes` owned by ctx. Grows (synchronising `stream` first)
// when too small.
mt_status scratch(mt_ctx* ctx, cudaStream_t stream, size_t bytes, void** out);
// Device table of the 32 NeoX inverse frequencies theta^(-2i/64) (Qwen.swift:60), computed on the
// host in fp32 as the reference does and kept by the context; uploads synchronously when theta
// changes (so the first call with a theta must not be inside a stream capture).
mt_status rope_table(mt_ctx* ctx, float theta, const float** out);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Runs a set-up step once per CUDA device, on the first call with that device current. Function
// attributes such as the dynamic shared-memory opt-in belong to the function in one device's
// context, so a process that drives several GPUs needs them set on each; several host threads
// may reach the first call at once.
constexpr int kMaxDevices = 64;
struct PerDeviceOnce {
    std::once_flag flags[kMaxDevices];
    template <typename F>
    void operator()(F&& f) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
            f();
            return;
        }
        std::call_once(flags[dev], std::forward<F>(f));
    }
};

}  // namespace mt

#define MT_REQUIRE(ctx, cond, code, ...)                          \
    do {                                                          \
        if (!(cond)) return mt::fail((ctx), (code), __VA_ARGS__); \
    } while (0)

// ------------------------------------------------------------------------------------------------
// Device helpers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// Round-to-nearest-even fp32 -> bf16 bits (the reference's host rounding, KernelTests.swift:30-34).
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float x) {
    uint32_t u = __float_as_uint(x);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// Hardware round-to-nearest-even fp32 -> bf16 (same result as f32_to_bf16_rne for finite values).
__device__ __forceinline__ uint16_t cvt_bf16_rn(float x) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x));
    return r;
}

// Two-term bf16 split of an fp32 value: x ~= hi + lo with |x - hi - lo| <= 2^-17 |x|. Integer
// rounding (the integer pipe has four times the throughput of the conversion unit).
__device__ __forceinline__ void split_bf16(float x, uint16_t& hi, uint16_t& lo) {
    hi = f32_to_bf16_rne(x);
    lo = f32_to_bf16_rne(x - bf16f(hi));
}

// The same split for two values with packed conversions (round to nearest even; bf16 bits of x0 in
// the low halves of hi2/lo2, of x1 in the high halves): one conversion per two values per term.
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t& hi2, uint32_t& lo2) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi2) : "f"(x1), "f"(x0));
    const float r0 = x0 - bf16_lo(hi2), r1 = x1 - bf16_hi(hi2);
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo2) : "f"(r1), "f"(r0));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// GELU (tanh form) with the reference's +-15 clamp (Shaders.swift:23-27), evaluated through the
// identity 0.5 (1 + tanh(u)) = 1 / (1 + exp(-2u)): one exponential, no cancellation for negative x,
// relative error a few fp32 ulps.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float k = 0.7978845608028654f;
    float u = k * (x + 0.044715f * x * x * x);
    u = fminf(fmaxf(u, -15.0f), 15.0f);
    return __fdividef(x, 1.0f + __expf(-2.0f * u));
}
// x * sigmoid(x); __fdividef returns 0 for denominators above 2^126, the right limit for x << 0.
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Streaming 16-byte weight load: read once, do not pollute L1.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Programmatic dependent launch. Every kernel of the library calls pdl_wait() before it touches
// global memory (it returns once the preceding kernel on the stream has completed and its writes
// are visible; a no-op without the launch attribute) and pdl_launch() to let the next kernel's
// CTAs be scheduled while this one drains.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launches `kernel` with the programmatic-stream-serialization attribute (see pdl_wait).
// Scheduling priority given to the kernels this thread launches (0: none, the stream's own). The
// engine raises its critical path (LLM token, flow, aggregator) above the concurrent VAE decode;
// captured launches keep it as a graph-node attribute.
inline int& launch_priority() {
    static thread_local int p = 0;
    return p;
}

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (launch_priority() != 0) {
        attr[1].id = cudaLaunchAttributePriority;
        attr[1].val.priority = launch_priority();
        cfg.numAttrs = 2;
    }
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// launch_k for kernels that run as clusters of two CTAs along x (grid.x even).
template <typename... KArgs, typename... Args>
inline void launch_k_pair(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[3];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (launch_priority() != 0) {
        attr[2].id = cudaLaunchAttributePriority;
        attr[2].val.priority = launch_priority();
        cfg.numAttrs = 3;
    }
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Records a device-side failure in the context status word (first writer wins).
__device__ __forceinline__ void report_status(unsigned int* status, unsigned int code,
                                              unsigned int site, unsigned int detail) {
    if (status && atomicCAS(status, 0u, code) == 0u) {
        status[1] = site;
        status[2] = detail;
    }
}

// ------------------------------------------------------------------------------------------------
// mbarrier helpers (shared memory barriers completed by arrivals and by async-copy byte counts).
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

constexpr uint64_t MBAR_WAIT_NS = 2000000000ull;  // 2 s per wait unless the status word sets a limit

// Wall-time limit of one bounded wait: word 3 of the status word holds it in microseconds
// (mt_ctx_set_wait_limit); 0 or no status word means MBAR_WAIT_NS.
__device__ __forceinline__ uint64_t wait_limit_ns(const unsigned int* status) {
    const unsigned int us = status ? *reinterpret_cast<const volatile unsigned int*>(status + 3) : 0u;
    return us ? (uint64_t)us * 1000ull : MBAR_WAIT_NS;
}

// Bounded wait on the phase with the given parity: gives up after the wait limit of wall time
// (checked every 256 polls) or as soon as another thread of the CTA has raised *abort; a wait that
// times out records the site in the status word, raises *abort and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* status, unsigned site,
                                          volatile int* abort) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0, limit = 0;
    for (uint32_t i = 0;; i++) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(addr), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 255u) == 255u) {
            if (*abort) return false;
            const uint64_t now = global_ns();
            if (t0 == 0) {
                t0 = now;
                limit = wait_limit_ns(status);
            } else if (now - t0 > limit) {
                break;
            }
        }
    }
    report_status(status, mt::DEV_TIMEOUT, site, blockIdx.x);
    *abort = 1;
    return false;
}

// Bulk (non-tensor) async copy global -> shared completing on an mbarrier; both addresses 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

