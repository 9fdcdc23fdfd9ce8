// common.cuh -- helpers shared by the sm_100a kernels and the C-ABI glue of libmingcuda.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/mingcuda.h"

// ------------------------------------------------------------------------------------------------
// Context (host side). One per device; owns the device status word that bounded waits write and
// a scratch area for the fp32 -> bf16 hi/lo split of mt_linear's tensor-core route.
// ------------------------------------------------------------------------------------------------
struct mt_ctx {
    int device = 0;
    int sm_count = 0;
    unsigned int* d_status = nullptr;  // [0] = error code, [1] = site id, [2] = detail
    void* scratch = nullptr;           // grows on demand, see mt_scratch()
    size_t scratch_bytes = 0;
    std::string err;
};

namespace mt {

// Status word codes written by kernels (d_status[0]).
enum : unsigned int { DEV_OK = 0, DEV_TIMEOUT = 1, DEV_BAD_ARG = 2 };

mt_status fail(mt_ctx* ctx, mt_status code, const char* fmt, ...);
mt_status check_launch(mt_ctx* ctx, const char* what);
// Returns a device buffer of at least `bytes` owned by ctx. Grows (synchronising `stream` first)
// when too small.
mt_status scratch(mt_ctx* ctx, cudaStream_t stream, size_t bytes, void** out);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

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
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
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
