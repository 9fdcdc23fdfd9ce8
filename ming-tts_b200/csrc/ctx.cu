// ctx.cu -- context, error reporting and the seeded synthetic-data generators of libmingcuda.so.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace mt {

mt_status fail(mt_ctx* ctx, mt_status code, const char* fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->err = buf;
    }
    return code;
}

mt_status check_launch(mt_ctx* ctx, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return MT_OK;
}

mt_status scratch(mt_ctx* ctx, cudaStream_t stream, size_t bytes, void** out) {
    if (bytes > ctx->scratch_bytes) {
        size_t want = bytes < (64u << 20) ? (64u << 20) : bytes;
        if (ctx->scratch) {
            cudaError_t e = cudaStreamSynchronize(stream);
            if (e != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "scratch grow sync: %s", cudaGetErrorString(e));
            cudaFree(ctx->scratch);
            ctx->scratch = nullptr;
            ctx->scratch_bytes = 0;
        }
        cudaError_t e = cudaMalloc(&ctx->scratch, want);
        if (e != cudaSuccess) return fail(ctx, MT_ERR_NOMEM, "scratch of %zu bytes: %s", want, cudaGetErrorString(e));
        ctx->scratch_bytes = want;
    }
    *out = ctx->scratch;
    return MT_OK;
}

// A bounded wait that nothing completes: one thread initialises a shared-memory barrier expecting
// one arrival, never arrives on it and waits for its first phase. The wait gives up after the
// context's wait limit and records DEV_TIMEOUT at site 90 in the status word; no asynchronous copy
// is in flight, so the kernel simply returns and the context stays usable.
__global__ void wait_probe_kernel(unsigned int* status) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    pdl_wait();
    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_wait(&bar, 0, status, 90, &abort_flag);
    }
}

mt_status rope_table(mt_ctx* ctx, float theta, const float** out) {
    if (!ctx->rope) {
        cudaError_t e = cudaMalloc(&ctx->rope, 32 * sizeof(float));
        if (e != cudaSuccess) return fail(ctx, MT_ERR_NOMEM, "rope table: %s", cudaGetErrorString(e));
        ctx->rope_theta = 0.f;
    }
    if (ctx->rope_theta != theta) {
        float inv[32];
        for (int i = 0; i < 32; i++) inv[i] = 1.0f / powf(theta, (float)(2 * i) / 64.0f);
        cudaError_t e = cudaMemcpy(ctx->rope, inv, sizeof(inv), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "rope table upload: %s", cudaGetErrorString(e));
        ctx->rope_theta = theta;
    }
    *out = ctx->rope;
    return MT_OK;
}

}  // namespace mt

extern "C" {

mt_status mt_ctx_create(int device, mt_ctx** out) {
    if (!out) return MT_ERR_ARG;
    *out = nullptr;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return MT_ERR_CUDA;
    mt_ctx* ctx = new mt_ctx();
    ctx->device = device;
    cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    e = cudaMalloc(&ctx->d_status, 4 * sizeof(unsigned int));
    if (e != cudaSuccess) {
        delete ctx;
        return MT_ERR_NOMEM;
    }
    cudaMemset(ctx->d_status, 0, 4 * sizeof(unsigned int));
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(ctx->d_status);
        delete ctx;
        return MT_ERR_CUDA;
    }
    *out = ctx;
    return MT_OK;
}

void mt_ctx_destroy(mt_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->stack_area) cudaFree(ctx->stack_area);
    if (ctx->rope) cudaFree(ctx->rope);
    if (ctx->d_status) cudaFree(ctx->d_status);
    delete ctx;
}

const char* mt_last_error(const mt_ctx* ctx) { return ctx ? ctx->err.c_str() : "no context"; }

const char* mt_version(void) { return "mingcuda 0.1.0 sm_100a"; }

mt_status mt_ctx_check(mt_ctx* ctx, void* stream) {
    if (!ctx) return MT_ERR_ARG;
    cudaError_t e = cudaStreamSynchronize(mt::as_stream(stream));
    if (e != cudaSuccess) return mt::fail(ctx, MT_ERR_CUDA, "stream: %s", cudaGetErrorString(e));
    unsigned int st[4];
    e = cudaMemcpy(st, ctx->d_status, sizeof(st), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return mt::fail(ctx, MT_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
    if (st[0] != mt::DEV_OK) {
        cudaMemset(ctx->d_status, 0, 3 * sizeof(unsigned int));  // word 3 (the wait limit) stays
        if (st[0] == mt::DEV_TIMEOUT)
            return mt::fail(ctx, MT_ERR_TIMEOUT, "device wait gave up (site %u, detail %u)", st[1], st[2]);
        return mt::fail(ctx, MT_ERR_ARG, "device check failed (code %u, site %u, detail %u)", st[0], st[1], st[2]);
    }
    return MT_OK;
}

mt_status mt_ctx_set_wait_limit(mt_ctx* ctx, unsigned int microseconds) {
    if (!ctx) return MT_ERR_ARG;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = cudaMemcpy(ctx->d_status + 3, &microseconds, sizeof(unsigned int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return mt::fail(ctx, MT_ERR_CUDA, "mt_ctx_set_wait_limit: %s", cudaGetErrorString(e));
    return MT_OK;
}

mt_status mt_ctx_set_persistent(mt_ctx* ctx, int mode) {
    if (!ctx || mode < 0 || mode > 2) return MT_ERR_ARG;
    ctx->persistent = mode;
    return MT_OK;
}

mt_status mt_ctx_wait_probe(mt_ctx* ctx, void* stream) {
    if (!ctx) return MT_ERR_ARG;
    launch_k(mt::wait_probe_kernel, 1, 32, 0, mt::as_stream(stream), ctx->d_status);
    return mt::check_launch(ctx, "mt_ctx_wait_probe");
}

mt_status mt_write_wav_f32(const char* path, const float* samples, long long count, int sample_rate) {
    if (!path || (!samples && count > 0) || count < 0 || sample_rate <= 0 || count * 4 > 0xFFFFFFFFLL - 36)
        return MT_ERR_ARG;
    FILE* f = fopen(path, "wb");
    if (!f) return MT_ERR_ARG;
    auto u32 = [&](uint32_t v) {
        const unsigned char b[4] = {(unsigned char)v, (unsigned char)(v >> 8), (unsigned char)(v >> 16),
                                    (unsigned char)(v >> 24)};
        fwrite(b, 1, 4, f);
    };
    auto u16 = [&](uint16_t v) {
        const unsigned char b[2] = {(unsigned char)v, (unsigned char)(v >> 8)};
        fwrite(b, 1, 2, f);
    };
    const uint32_t bytes = (uint32_t)(count * 4);
    fwrite("RIFF", 1, 4, f);
    u32(36 + bytes);
    fwrite("WAVEfmt ", 1, 8, f);
    u32(16);
    u16(3);  // IEEE float
    u16(1);  // mono
    u32((uint32_t)sample_rate);
    u32((uint32_t)sample_rate * 4);
    u16(4);
    u16(32);
    fwrite("data", 1, 4, f);
    u32(bytes);
    for (long long i = 0; i < count; i++) {  // little-endian fp32
        uint32_t u;
        memcpy(&u, &samples[i], 4);
        u32(u);
    }
    const bool ok = ferror(f) == 0;
    return fclose(f) == 0 && ok ? MT_OK : MT_ERR_ARG;
}

mt_status mt_ctx_set_gemm_pairs(mt_ctx* ctx, int mode) {
    if (!ctx) return MT_ERR_ARG;
    MT_REQUIRE(ctx, mode >= -1 && mode <= 1, MT_ERR_ARG, "mt_ctx_set_gemm_pairs: mode %d (-1, 0 or 1)", mode);
    ctx->gemm_pairs = mode;
    return MT_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Seeded generators. Draw j (1-based) of the SplitMix64 stream mixes seed + (j + 1) * golden, the
// sequence MingEngine.gaussianNoise walks (Engine.swift:433-453); pair p uses draws 2p+1, 2p+2 in a
// Box-Muller transform in double. Being counter-based, every pair is computed independently.
// ------------------------------------------------------------------------------------------------
namespace {

__host__ __device__ inline double sm64_draw(uint64_t seed, uint64_t j) {
    const uint64_t g = 0x9E3779B97F4A7C15ull;
    uint64_t z = seed + (j + 1) * g;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (double)(z >> 11) / (double)(1ull << 53);
}

__host__ __device__ inline void gauss_pair(uint64_t seed, uint64_t p, float* a, float* b) {
    double u1 = sm64_draw(seed, 2 * p + 1), u2 = sm64_draw(seed, 2 * p + 2);
    if (u1 < 1e-300) u1 = 1e-300;
    const double r = sqrt(-2.0 * log(u1));
    const double twopi = 6.283185307179586476925286766559;
    *a = (float)(r * cos(twopi * u2));
    *b = (float)(r * sin(twopi * u2));
}

__host__ __device__ inline uint16_t bf16_rne_bits(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

__global__ void randn_bf16_kernel(uint16_t* out, size_t count, uint64_t seed, float std) {
    const size_t pairs = (count + 1) / 2;
    for (size_t p = blockIdx.x * (size_t)blockDim.x + threadIdx.x; p < pairs; p += (size_t)gridDim.x * blockDim.x) {
        float a, b;
        gauss_pair(seed, p, &a, &b);
        out[2 * p] = bf16_rne_bits(a * std);
        if (2 * p + 1 < count) out[2 * p + 1] = bf16_rne_bits(b * std);
    }
}

}  // namespace

extern "C" {

void mt_gaussian_noise_host(float* out, size_t count, uint64_t seed) {
    for (size_t i = 0; i < count; i += 2) {
        float a, b;
        gauss_pair(seed, i / 2, &a, &b);
        out[i] = a;
        if (i + 1 < count) out[i + 1] = b;
    }
}

void mt_randn_bf16_host(mt_bf16* out, size_t count, uint64_t seed, float std) {
    const long long pairs = (long long)((count + 1) / 2);
#pragma omp parallel for schedule(static)
    for (long long p = 0; p < pairs; p++) {
        float a, b;
        gauss_pair(seed, (uint64_t)p, &a, &b);
        out[2 * p] = bf16_rne_bits(a * std);
        if ((size_t)(2 * p + 1) < count) out[2 * p + 1] = bf16_rne_bits(b * std);
    }
}

mt_status mt_randn_bf16(mt_ctx* ctx, void* stream, mt_bf16* out, size_t count, uint64_t seed, float std) {
    MT_REQUIRE(ctx, ctx && out, MT_ERR_ARG, "mt_randn_bf16: null argument");
    if (count == 0) return MT_OK;
    const size_t pairs = (count + 1) / 2;
    size_t blocks = (pairs + 255) / 256;
    if (blocks > (size_t)ctx->sm_count * 16) blocks = (size_t)ctx->sm_count * 16;
    randn_bf16_kernel<<<(unsigned)blocks, 256, 0, mt::as_stream(stream)>>>(out, count, seed, std);
    return mt::check_launch(ctx, "mt_randn_bf16");
}

}  // extern "C"
