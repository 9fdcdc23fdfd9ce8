// engine_kernels.cu -- batched kernels of the generation loop (R requests per launch).
//
// Each restates, for every request at once, a piece of MingEngine.encodeStep (Engine.swift:377-415)
// and VAEDecoder (VAEDecoder.swift:64-107). Step-dependent indices (step n, decoded latent d) are read
// from a device-resident step state, so a captured CUDA graph can replay the step unchanged.
#include "common.cuh"
#include "engine_kernels.cuh"

namespace mt {

// Prompt rows from the bf16 embedding table (promptEmbeddings, Engine.swift:204-212): row i of the
// batch is table[ids[i]] widened to fp32.
__global__ void embed_gather_kernel(const int32_t* __restrict__ ids, int rows, const uint16_t* __restrict__ table,
                                    int hidden, int vocab, float* __restrict__ x, unsigned int* status) {
    pdl_wait();
    pdl_launch();
    const int row = blockIdx.x;
    if (row >= rows) return;
    int id = ids[row];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) report_status(status, DEV_BAD_ARG, 10, (unsigned)row);
        id = 0;
    }
    const uint16_t* src = table + (size_t)id * hidden;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) x[(size_t)row * hidden + c] = bf16f(src[c]);
}

void launch_embed_gather(const int32_t* ids, int rows, const uint16_t* table, int hidden, int vocab, float* x,
                         unsigned int* status, cudaStream_t s) {
    launch_k(embed_gather_kernel, rows, 256, 0, s, ids, rows, table, hidden, vocab, x, status);
}

// history <- y (n > 0), y <- noise[n] (Engine.swift:389-393).
__global__ void flow_begin_kernel(float* __restrict__ y, float* __restrict__ hist, const float* __restrict__ noise,
                                  int latent, int steps_cap, const int* __restrict__ state) {
    pdl_wait();
    pdl_launch();
    const int r = blockIdx.x, d = threadIdx.x;
    if (d >= latent) return;
    const int n = state[ST_N];
    if (n > 0) hist[r * latent + d] = y[r * latent + d];
    y[r * latent + d] = noise[((size_t)r * steps_cap + n) * latent + d];
}

void launch_flow_begin(float* y, float* hist, const float* noise, int latent, int steps_cap, const int* state,
                       int requests, cudaStream_t s) {
    launch_k(flow_begin_kernel, requests, latent, 0, s, y, hist, noise, latent, steps_cap, state);
}

// x_emb of latent vectors: thread c keeps weight row c (latent bf16 values) in registers and
// applies it to the EMB_RB requests of its block (their vectors staged in shared memory), so each
// weight row is read once per block instead of once per request.
constexpr int EMB_THREADS = 128;
constexpr int EMB_RB = 8;          // requests per block
constexpr int EMB_MAX_LATENT = 64;

__device__ __forceinline__ void emb_load_row(const uint16_t* __restrict__ w, int c, int latent, uint32_t* wr) {
    const uint4* src = reinterpret_cast<const uint4*>(w + (size_t)c * latent);
#pragma unroll
    for (int i = 0; i < EMB_MAX_LATENT / 8; i++) {
        if (i * 8 < latent) {
            const uint4 v = src[i];
            wr[4 * i] = v.x; wr[4 * i + 1] = v.y; wr[4 * i + 2] = v.z; wr[4 * i + 3] = v.w;
        }
    }
}

__device__ __forceinline__ float emb_dot(const uint32_t* wr, const float* sv, int latent) {
    float e = 0.f;
#pragma unroll
    for (int i = 0; i < EMB_MAX_LATENT / 2; i++)
        if (2 * i < latent) e += bf16_lo(wr[i]) * sv[2 * i] + bf16_hi(wr[i]) * sv[2 * i + 1];
    return e;
}

// The six DiT input rows of every request (flow_assemble, Shaders.swift:654-677): x_emb(history)
// and x_emb(y) of column c are computed once and written to both halves.
__global__ void __launch_bounds__(EMB_THREADS) flow_assemble_batched_kernel(
    const float* __restrict__ y, const float* __restrict__ hist, const float* __restrict__ cemb,
    const uint16_t* __restrict__ cbias, const float* __restrict__ temb, const uint16_t* __restrict__ xw,
    const uint16_t* __restrict__ xb, int hidden, int latent, float* __restrict__ X, int requests) {
    __shared__ float sv[EMB_RB][2][EMB_MAX_LATENT];
    const int c = blockIdx.x * EMB_THREADS + threadIdx.x;
    const int r0 = blockIdx.y * EMB_RB;
    const int nr = min(EMB_RB, requests - r0);
    uint32_t wr[EMB_MAX_LATENT / 2];
    float b = 0.f, t = 0.f, tb = 0.f;
    if (c < hidden) {  // weights never depend on the previous kernel
        emb_load_row(xw, c, latent, wr);
        b = bf16f(xb[c]);
        tb = bf16f(cbias[c]);
    }
    pdl_wait();
    pdl_launch();
    for (int i = threadIdx.x; i < nr * latent; i += EMB_THREADS) {
        const int rr = i / latent, d = i % latent;
        sv[rr][0][d] = hist[(size_t)(r0 + rr) * latent + d];
        sv[rr][1][d] = y[(size_t)(r0 + rr) * latent + d];
    }
    if (c < hidden) t = temb[c];
    __syncthreads();
    if (c >= hidden) return;
    for (int rr = 0; rr < nr; rr++) {
        const int r = r0 + rr;
        const float eh = emb_dot(wr, sv[rr][0], latent) + b;
        const float ey = emb_dot(wr, sv[rr][1], latent) + b;
        float* base = X + (size_t)r * 6 * hidden + c;
        base[0] = t + cemb[(size_t)r * hidden + c];
        base[hidden] = eh;
        base[2 * hidden] = ey;
        base[3 * hidden] = t + tb;
        base[4 * hidden] = eh;
        base[5 * hidden] = ey;
    }
}

void launch_flow_assemble_batched(const float* y, const float* hist, const float* cemb, const uint16_t* cbias,
                                  const float* temb, const uint16_t* xw, const uint16_t* xb, int hidden, int latent,
                                  float* X, int requests, cudaStream_t s) {
    launch_k(flow_assemble_batched_kernel, dim3((hidden + EMB_THREADS - 1) / EMB_THREADS, (requests + EMB_RB - 1) / EMB_RB),
             EMB_THREADS, 0, s, y, hist, cemb, cbias, temb, xw, xb, hidden, latent, X, requests);
}

// Flow-head output and Euler step for every request, fused: RMSNorm of the rows whose predictions
// are used (row 2 = conditional, row 5 = unconditional, DiT.swift:50-51 over Engine.swift:398-401),
// the final linear (out_dim = latent) on those two rows, and y += (c + (c - u) cfg) dt
// (flow_euler, Shaders.swift:682-693). The reference norms and projects all six rows and reads
// rows 2 and 5; the other four never reach an output. Optional captures: the step-0 predictions
// and, after the last Euler step, the latent.
// One warp per (request, output): lane l holds columns 4l + 128t of both rows (t < hidden / 128),
// computes the two row norms with warp reductions and the two dot products; no shared memory.
constexpr int FF_WARPS = 8;
constexpr int FF_MAX_T = 8;  // hidden <= 1024

__global__ void __launch_bounds__(FF_WARPS * 32) flow_final_kernel(FlowFinalArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.y, o = blockIdx.x * FF_WARPS + warp;
    const int T = a.hidden / 128;
    uint2 g[FF_MAX_T], w[FF_MAX_T];
    const bool live = o < a.latent;
#pragma unroll
    for (int t = 0; t < FF_MAX_T; t++) {  // weights: before the dependency wait
        if (t < T && live) {
            g[t] = *reinterpret_cast<const uint2*>(a.norm_w + 4 * lane + 128 * t);
            w[t] = *reinterpret_cast<const uint2*>(a.final_w + (size_t)o * a.hidden + 4 * lane + 128 * t);
        }
    }
    pdl_wait();
    pdl_launch();
    if (!live) return;
    const float* rc = a.X + ((size_t)r * 6 + 2) * a.hidden;
    const float* ru = a.X + ((size_t)r * 6 + 5) * a.hidden;
    float4 xc[FF_MAX_T], xu[FF_MAX_T];
    float sc = 0.f, su = 0.f;
#pragma unroll
    for (int t = 0; t < FF_MAX_T; t++) {
        if (t < T) {
            xc[t] = *reinterpret_cast<const float4*>(rc + 4 * lane + 128 * t);
            xu[t] = *reinterpret_cast<const float4*>(ru + 4 * lane + 128 * t);
            sc += xc[t].x * xc[t].x + xc[t].y * xc[t].y + xc[t].z * xc[t].z + xc[t].w * xc[t].w;
            su += xu[t].x * xu[t].x + xu[t].y * xu[t].y + xu[t].z * xu[t].z + xu[t].w * xu[t].w;
        }
    }
    sc = warp_sum(sc);
    su = warp_sum(su);
    const float scale_c = rsqrtf(sc / (float)a.hidden + a.eps);
    const float scale_u = rsqrtf(su / (float)a.hidden + a.eps);
    float dc = 0.f, du = 0.f;
#pragma unroll
    for (int t = 0; t < FF_MAX_T; t++) {
        if (t < T) {
            const float g0 = bf16_lo(g[t].x), g1 = bf16_hi(g[t].x), g2 = bf16_lo(g[t].y), g3 = bf16_hi(g[t].y);
            const float w0 = bf16_lo(w[t].x), w1 = bf16_hi(w[t].x), w2 = bf16_lo(w[t].y), w3 = bf16_hi(w[t].y);
            dc += w0 * (xc[t].x * scale_c * g0) + w1 * (xc[t].y * scale_c * g1) + w2 * (xc[t].z * scale_c * g2) +
                  w3 * (xc[t].w * scale_c * g3);
            du += w0 * (xu[t].x * scale_u * g0) + w1 * (xu[t].y * scale_u * g1) + w2 * (xu[t].z * scale_u * g2) +
                  w3 * (xu[t].w * scale_u * g3);
        }
    }
    dc = warp_sum(dc);
    du = warp_sum(du);
    if (lane == 0) {
        const int n = a.state[ST_N];
        const float bo = bf16f(a.final_b[o]);
        const float c = dc + bo, u = du + bo;
        float* yp = a.y + (size_t)r * a.latent + o;
        const float yn = *yp + (c + (c - u) * a.cfg) * a.dt;
        *yp = yn;
        if (a.vel0 && n == 0) {
            float* v = a.vel0 + (((size_t)r * a.flow_steps + a.k) * 2) * a.latent;
            v[o] = c;
            v[a.latent + o] = u;
        }
        if (a.latents && a.k == a.flow_steps - 1) a.latents[((size_t)r * a.steps_cap + n) * a.latent + o] = yn;
    }
}

void launch_flow_final(const FlowFinalArgs& a, int requests, cudaStream_t s) {
    launch_k(flow_final_kernel, dim3((a.latent + FF_WARPS - 1) / FF_WARPS, requests), FF_WARPS * 32, 0, s, a);
}

// Aggregator input rows (Engine.swift:407-409): row 2r = cls, row 2r+1 = x_emb(latent of request r).
__global__ void __launch_bounds__(EMB_THREADS) agg_assemble_kernel(const float* __restrict__ y,
                                                                   const float* __restrict__ cls,
                                                                   const uint16_t* __restrict__ xw,
                                                                   const uint16_t* __restrict__ xb, int hidden,
                                                                   int latent, float* __restrict__ X, int requests) {
    __shared__ float sv[EMB_RB][EMB_MAX_LATENT];
    const int c = blockIdx.x * EMB_THREADS + threadIdx.x;
    const int r0 = blockIdx.y * EMB_RB;
    const int nr = min(EMB_RB, requests - r0);
    uint32_t wr[EMB_MAX_LATENT / 2];
    float b = 0.f, cl = 0.f;
    if (c < hidden) {
        emb_load_row(xw, c, latent, wr);
        b = bf16f(xb[c]);
        cl = cls[c];
    }
    pdl_wait();
    pdl_launch();
    for (int i = threadIdx.x; i < nr * latent; i += EMB_THREADS)
        sv[i / latent][i % latent] = y[(size_t)(r0 + i / latent) * latent + i % latent];
    __syncthreads();
    if (c >= hidden) return;
    for (int rr = 0; rr < nr; rr++) {
        const int r = r0 + rr;
        X[(size_t)(2 * r) * hidden + c] = cl;
        X[(size_t)(2 * r + 1) * hidden + c] = emb_dot(wr, sv[rr], latent) + b;
    }
}

void launch_agg_assemble(const float* y, const float* cls, const uint16_t* xw, const uint16_t* xb, int hidden,
                         int latent, float* X, int requests, cudaStream_t s) {
    launch_k(agg_assemble_kernel, dim3((hidden + EMB_THREADS - 1) / EMB_THREADS, (requests + EMB_RB - 1) / EMB_RB),
             EMB_THREADS, 0, s, y, cls, xw, xb, hidden, latent, X, requests);
}

// VAE fc1 of the new latent into ring slot n % VAE_H_RING of every request
// (VAEDecoder.encodeFc1, VAEDecoder.swift:64-67).
__global__ void __launch_bounds__(EMB_THREADS) vae_fc1_kernel(const float* __restrict__ y,
                                                              const uint16_t* __restrict__ w,
                                                              const uint16_t* __restrict__ b, int hidden, int latent,
                                                              float* __restrict__ h, const int* __restrict__ state,
                                                              int requests) {
    __shared__ float sv[EMB_RB][EMB_MAX_LATENT];
    const int c = blockIdx.x * EMB_THREADS + threadIdx.x;
    const int r0 = blockIdx.y * EMB_RB;
    const int nr = min(EMB_RB, requests - r0);
    uint32_t wr[EMB_MAX_LATENT / 2];
    float bc = 0.f;
    if (c < hidden) {
        emb_load_row(w, c, latent, wr);
        bc = bf16f(b[c]);
    }
    pdl_wait();
    pdl_launch();
    for (int i = threadIdx.x; i < nr * latent; i += EMB_THREADS)
        sv[i / latent][i % latent] = y[(size_t)(r0 + i / latent) * latent + i % latent];
    __syncthreads();
    if (c >= hidden) return;
    const int slot = state[ST_N] % VAE_H_RING;
    for (int rr = 0; rr < nr; rr++)
        h[((size_t)(r0 + rr) * VAE_H_RING + slot) * hidden + c] = emb_dot(wr, sv[rr], latent) + bc;
}

void launch_vae_fc1(const float* y, const uint16_t* w, const uint16_t* b, int hidden, int latent, float* h,
                    const int* state, int requests, cudaStream_t s) {
    launch_k(vae_fc1_kernel, dim3((hidden + EMB_THREADS - 1) / EMB_THREADS, (requests + EMB_RB - 1) / EMB_RB),
             EMB_THREADS, 0, s, y, w, b, hidden, latent, h, state, requests);
}

// The four upsampled frames of latent d for every request from ring slots d-1, d, d+1
// (upsample4, Shaders.swift:704-719; neighbours clamp to h[d] when absent).
__global__ void vae_upsample_kernel(const float* __restrict__ h, int hidden, const int* __restrict__ state,
                                    float* __restrict__ frames) {
    pdl_wait();
    pdl_launch();
    const int r = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= hidden) return;
    const int d = state[ST_D];
    const int has_prev = d >= 1, has_next = state[ST_HAS_NEXT];
    const float* base = h + (size_t)r * VAE_H_RING * hidden;
    const float cur = base[(size_t)(d % VAE_H_RING) * hidden + c];
    const float prev = has_prev ? base[(size_t)((d + VAE_H_RING - 1) % VAE_H_RING) * hidden + c] : cur;
    const float next = has_next ? base[(size_t)((d + 1) % VAE_H_RING) * hidden + c] : cur;
    float* out = frames + (size_t)r * 4 * hidden + c;
    out[0] = has_prev ? 0.625f * cur + 0.375f * prev : cur;
    out[hidden] = has_prev ? 0.875f * cur + 0.125f * prev : cur;
    out[2 * hidden] = has_next ? 0.875f * cur + 0.125f * next : cur;
    out[3 * hidden] = has_next ? 0.625f * cur + 0.375f * next : cur;
}

void launch_vae_upsample(const float* h, int hidden, const int* state, float* frames, int requests, cudaStream_t s) {
    launch_k(vae_upsample_kernel, dim3((hidden + 127) / 128, requests), 128, 0, s, h, hidden, state, frames);
}

}  // namespace mt
