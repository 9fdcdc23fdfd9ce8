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

// The six DiT input rows of every request (flow_assemble, Shaders.swift:654-677): thread c computes
// x_emb(history)[c] and x_emb(y)[c] once and writes all six rows of column c.
__global__ void flow_assemble_batched_kernel(const float* __restrict__ y, const float* __restrict__ hist,
                                             const float* __restrict__ cemb, const uint16_t* __restrict__ cbias,
                                             const float* __restrict__ temb, const uint16_t* __restrict__ xw,
                                             const uint16_t* __restrict__ xb, int hidden, int latent,
                                             float* __restrict__ X) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float sv[];  // [2][latent]
    const int r = blockIdx.y;
    for (int d = threadIdx.x; d < latent; d += blockDim.x) {
        sv[d] = hist[r * latent + d];
        sv[latent + d] = y[r * latent + d];
    }
    __syncthreads();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= hidden) return;
    const uint16_t* w = xw + (size_t)c * latent;
    const float b = bf16f(xb[c]);
    float eh = 0.f, ey = 0.f;
    for (int d = 0; d < latent; d += 2) {
        const uint32_t wv = *reinterpret_cast<const uint32_t*>(w + d);
        eh += bf16_lo(wv) * sv[d] + bf16_hi(wv) * sv[d + 1];
        ey += bf16_lo(wv) * sv[latent + d] + bf16_hi(wv) * sv[latent + d + 1];
    }
    eh += b;
    ey += b;
    float* base = X + (size_t)r * 6 * hidden + c;
    base[0] = temb[c] + cemb[(size_t)r * hidden + c];
    base[hidden] = eh;
    base[2 * hidden] = ey;
    base[3 * hidden] = temb[c] + bf16f(cbias[c]);
    base[4 * hidden] = eh;
    base[5 * hidden] = ey;
}

void launch_flow_assemble_batched(const float* y, const float* hist, const float* cemb, const uint16_t* cbias,
                                  const float* temb, const uint16_t* xw, const uint16_t* xb, int hidden, int latent,
                                  float* X, int requests, cudaStream_t s) {
    launch_k(flow_assemble_batched_kernel, dim3((hidden + 127) / 128, requests), 128, 2 * latent * sizeof(float), s, 
        y, hist, cemb, cbias, temb, xw, xb, hidden, latent, X);
}

// Flow-head output and Euler step for every request, fused: RMSNorm of the rows whose predictions
// are used (row 2 = conditional, row 5 = unconditional, DiT.swift:50-51 over Engine.swift:398-401),
// the final linear (out_dim = latent) on those two rows, and y += (c + (c - u) cfg) dt
// (flow_euler, Shaders.swift:682-693). The reference norms and projects all six rows and reads
// rows 2 and 5; the other four never reach an output. Optional captures: the step-0 predictions
// and, after the last Euler step, the latent.
__global__ void __launch_bounds__(256) flow_final_kernel(FlowFinalArgs a) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float sm[];
    float* xc = sm;                 // [hidden]
    float* xu = sm + a.hidden;      // [hidden]
    __shared__ float red[2][8];
    const int r = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float* rc = a.X + ((size_t)r * 6 + 2) * a.hidden;
    const float* ru = a.X + ((size_t)r * 6 + 5) * a.hidden;
    float sc = 0.f, su = 0.f;
    for (int i = tid; i < a.hidden; i += blockDim.x) {
        const float vc = rc[i], vu = ru[i];
        xc[i] = vc;
        xu[i] = vu;
        sc += vc * vc;
        su += vu * vu;
    }
    sc = warp_sum(sc);
    su = warp_sum(su);
    if (lane == 0) {
        red[0][warp] = sc;
        red[1][warp] = su;
    }
    __syncthreads();
    float tc = 0.f, tu = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
        tc += red[0][w];
        tu += red[1][w];
    }
    const float scale_c = rsqrtf(tc / (float)a.hidden + a.eps);
    const float scale_u = rsqrtf(tu / (float)a.hidden + a.eps);
    __syncthreads();
    for (int i = tid; i < a.hidden; i += blockDim.x) {
        const float g = bf16f(a.norm_w[i]);
        xc[i] = xc[i] * scale_c * g;
        xu[i] = xu[i] * scale_u * g;
    }
    __syncthreads();
    const int n = a.state[ST_N];
    for (int o = warp; o < a.latent; o += (int)(blockDim.x >> 5)) {
        const uint16_t* w = a.final_w + (size_t)o * a.hidden;
        float dc = 0.f, du = 0.f;
        for (int i = lane * 8; i < a.hidden; i += 256) {
            const uint4 wv = *reinterpret_cast<const uint4*>(w + i);
            const float w0 = bf16_lo(wv.x), w1 = bf16_hi(wv.x), w2 = bf16_lo(wv.y), w3 = bf16_hi(wv.y);
            const float w4 = bf16_lo(wv.z), w5 = bf16_hi(wv.z), w6 = bf16_lo(wv.w), w7 = bf16_hi(wv.w);
            dc += w0 * xc[i] + w1 * xc[i + 1] + w2 * xc[i + 2] + w3 * xc[i + 3] + w4 * xc[i + 4] + w5 * xc[i + 5] +
                  w6 * xc[i + 6] + w7 * xc[i + 7];
            du += w0 * xu[i] + w1 * xu[i + 1] + w2 * xu[i + 2] + w3 * xu[i + 3] + w4 * xu[i + 4] + w5 * xu[i + 5] +
                  w6 * xu[i + 6] + w7 * xu[i + 7];
        }
        dc = warp_sum(dc);
        du = warp_sum(du);
        if (lane == 0) {
            const float b = bf16f(a.final_b[o]);
            const float c = dc + b, u = du + b;
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
}

void launch_flow_final(const FlowFinalArgs& a, int requests, cudaStream_t s) {
    launch_k(flow_final_kernel, requests, 256, 2 * a.hidden * sizeof(float), s, a);
}

// Aggregator input rows (Engine.swift:407-409): row 2r = cls, row 2r+1 = x_emb(latent of request r).
__global__ void agg_assemble_kernel(const float* __restrict__ y, const float* __restrict__ cls,
                                    const uint16_t* __restrict__ xw, const uint16_t* __restrict__ xb, int hidden,
                                    int latent, float* __restrict__ X) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float sv[];
    const int r = blockIdx.y;
    for (int d = threadIdx.x; d < latent; d += blockDim.x) sv[d] = y[r * latent + d];
    __syncthreads();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= hidden) return;
    const uint16_t* w = xw + (size_t)c * latent;
    float e = 0.f;
    for (int d = 0; d < latent; d += 2) {
        const uint32_t wv = *reinterpret_cast<const uint32_t*>(w + d);
        e += bf16_lo(wv) * sv[d] + bf16_hi(wv) * sv[d + 1];
    }
    X[(size_t)(2 * r) * hidden + c] = cls[c];
    X[(size_t)(2 * r + 1) * hidden + c] = e + bf16f(xb[c]);
}

void launch_agg_assemble(const float* y, const float* cls, const uint16_t* xw, const uint16_t* xb, int hidden,
                         int latent, float* X, int requests, cudaStream_t s) {
    launch_k(agg_assemble_kernel, dim3((hidden + 127) / 128, requests), 128, latent * sizeof(float), s, y, cls, xw, xb,
                                                                                                hidden, latent, X);
}

// VAE fc1 of the new latent into ring slot n % VAE_H_RING of every request
// (VAEDecoder.encodeFc1, VAEDecoder.swift:64-67).
__global__ void vae_fc1_kernel(const float* __restrict__ y, const uint16_t* __restrict__ w,
                               const uint16_t* __restrict__ b, int hidden, int latent, float* __restrict__ h,
                               const int* __restrict__ state) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float sv[];
    const int r = blockIdx.y;
    for (int d = threadIdx.x; d < latent; d += blockDim.x) sv[d] = y[r * latent + d];
    __syncthreads();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= hidden) return;
    const int slot = state[ST_N] % VAE_H_RING;
    const uint16_t* wr = w + (size_t)c * latent;
    float e = 0.f;
    for (int d = 0; d < latent; d += 2) {
        const uint32_t wv = *reinterpret_cast<const uint32_t*>(wr + d);
        e += bf16_lo(wv) * sv[d] + bf16_hi(wv) * sv[d + 1];
    }
    h[((size_t)r * VAE_H_RING + slot) * hidden + c] = e + bf16f(b[c]);
}

void launch_vae_fc1(const float* y, const uint16_t* w, const uint16_t* b, int hidden, int latent, float* h,
                    const int* state, int requests, cudaStream_t s) {
    launch_k(vae_fc1_kernel, dim3((hidden + 127) / 128, requests), 128, latent * sizeof(float), s, y, w, b, hidden, latent,
                                                                                           h, state);
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
