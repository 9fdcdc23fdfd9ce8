// encoder.cu -- the clone path: the audio VAE encoder (VAEEncoder.encode, VAEEncoder.swift:56-107)
// and the aggregator over reference latents (MingEngine.aggregate, Engine.swift:236-256).
//
// These run once per reference voice, not per step, so they are composed from the operator entry
// points (mt_linear, mt_rmsnorm, mt_rope_cache, mt_attention, mt_dit_attention) on per-call device
// buffers; the large-M linears take the tensor-core route (frames of a clip: up to 1600 rows).
#include <math.h>
#include <string.h>

#include <vector>

#include "common.cuh"

namespace mt {

namespace {

#define TRY(x)                        \
    do {                              \
        const mt_status st_ = (x);    \
        if (st_ != MT_OK) return st_; \
    } while (0)

// One device allocation for all of a call's buffers, freed on scope exit. A slice that would not
// fit sets `overflow` (and returns the base, so no pointer leaves the allocation); callers check
// it before launching anything on their slices.
struct Scratch {
    uint8_t* base = nullptr;
    size_t used = 0, cap = 0;
    bool overflow = false;
    ~Scratch() {
        if (base) cudaFree(base);
    }
    bool reserve(size_t bytes) {
        cap = bytes;
        return cudaMalloc(&base, bytes) == cudaSuccess;
    }
    float* take(size_t floats) {  // 256-byte aligned slices
        const size_t bytes = (floats * 4 + 255) & ~size_t(255);
        if (used + bytes > cap) {
            overflow = true;
            return reinterpret_cast<float*>(base);
        }
        float* p = reinterpret_cast<float*>(base + used);
        used += bytes;
        return p;
    }
    static size_t size(size_t floats) { return (floats * 4 + 255) & ~size_t(255); }
};

// [patch frame rows | cls] per latent (VAEEncoder.swift:88-92).
__global__ void assemble_patches_kernel(const float* __restrict__ normed, const float* __restrict__ cls,
                                        float* __restrict__ patches, int latents, int patch, int h) {
    const long long total = (long long)latents * (patch + 1) * h;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int col = (int)(i % h);
        const long long row = i / h;
        const int p = (int)(row / (patch + 1)), j = (int)(row % (patch + 1));
        patches[i] = j < patch ? normed[((long long)p * patch + j) * h + col] : cls[col];
    }
}

// [cls, x_embedder(latent) + b] per latent: cls rows here, the x_embedder rows by mt_linear.
__global__ void cls_rows_kernel(const float* __restrict__ cls, float* __restrict__ x, int count, int h) {
    const long long total = (long long)count * h;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x)
        x[(i / h) * 2 * h + i % h] = cls[i % h];
}

size_t qwen_scratch_floats(const mt_qwen_config& c, int rows, int cap) {
    const size_t qkvw = (size_t)(c.heads + 2 * c.kv_heads) * 64;
    return Scratch::size((size_t)rows * c.hidden) + Scratch::size((size_t)rows * qkvw) +
           Scratch::size((size_t)rows * c.heads * 64) + Scratch::size((size_t)rows * c.intermediate) +
           Scratch::size((size_t)c.layers * 2 * c.kv_heads * cap * 64);
}

// QwenForward.dispatches (Qwen.swift:72-97) from an empty cache: every layer over `rows` rows at
// positions 0.., then the final norm of the last norm_rows rows into out.
mt_status qwen_prefill(mt_ctx* ctx, cudaStream_t s, const mt_qwen_weights& W, float* x, int rows, int norm_rows,
                       float* out, Scratch& sc, const float* inv_freq) {
    const mt_qwen_config& c = W.cfg;
    const int H = c.hidden, qkvw = (c.heads + 2 * c.kv_heads) * 64, cap = rows;
    float* normed = sc.take((size_t)rows * H);
    float* qkv = sc.take((size_t)rows * qkvw);
    float* attn = sc.take((size_t)rows * c.heads * 64);
    float* mlp = sc.take((size_t)rows * c.intermediate);
    float* kv = sc.take((size_t)c.layers * 2 * c.kv_heads * cap * 64);
    if (sc.overflow) return fail(ctx, MT_ERR_CAPACITY, "clone path: scratch sizing");
    const size_t per_tensor = (size_t)c.kv_heads * cap * 64;
    for (int l = 0; l < c.layers; l++) {
        const mt_qwen_layer& L = W.layers[l];
        float* kc = kv + (size_t)(2 * l) * per_tensor;
        float* vc = kc + per_tensor;
        TRY(mt_rmsnorm(ctx, s, x, H, rows, H, L.norm1, normed, H, c.eps));
        TRY(mt_linear(ctx, s, normed, H, rows, L.qkv_w, nullptr, L.qkv_b, qkvw, H, qkv, qkvw, MT_LINEAR_BIAS));
        TRY(mt_rope_cache(ctx, s, qkv, qkvw, rows, c.heads, c.kv_heads, 0, kc, vc, cap, inv_freq));
        TRY(mt_attention(ctx, s, qkv, qkvw, rows, c.heads, c.kv_heads, 0, c.window, kc, vc, cap, attn, c.heads * 64));
        TRY(mt_linear(ctx, s, attn, c.heads * 64, rows, L.o_w, nullptr, nullptr, H, c.heads * 64, x, H, MT_LINEAR_ACCUM));
        TRY(mt_rmsnorm(ctx, s, x, H, rows, H, L.norm2, normed, H, c.eps));
        TRY(mt_linear(ctx, s, normed, H, rows, L.gate_w, L.up_w, nullptr, c.intermediate, H, mlp, c.intermediate,
                      MT_LINEAR_SILU_GATE));
        TRY(mt_linear(ctx, s, mlp, c.intermediate, rows, L.down_w, nullptr, nullptr, H, c.intermediate, x, H,
                      MT_LINEAR_ACCUM));
    }
    return mt_rmsnorm(ctx, s, x + (size_t)(rows - norm_rows) * H, H, norm_rows, H, W.final_norm, out, H, c.eps);
}

// Round to nearest even bf16 and back (bf16Rounded, VAEEncoder.swift:110-114).
float bf16_rounded(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

// torch.nn.functional.softplus with its default threshold of 20 (VAEEncoder.swift:117).
float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

mt_status sync(mt_ctx* ctx, cudaStream_t s, const char* who) {
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "%s: %s", who, cudaGetErrorString(e));
    return check_launch(ctx, who);
}

}  // namespace

}  // namespace mt

using namespace mt;

extern "C" {

mt_status mt_vae_encode(mt_encoder* enc, void* stream, const float* samples, long long count, float* mean, float* stdv) {
    if (!enc) return MT_ERR_ARG;
    const mt_encoder_weights& W = *mt_encoder_get_weights(enc);
    mt_ctx* ctx = encoder_ctx(enc);  // the context the encoder was created on
    MT_REQUIRE(ctx, samples && mean && stdv, MT_ERR_ARG, "mt_vae_encode: null argument");
    const int frame = W.frame, patch = W.patch, pf = W.padded_frame, H = W.stack.cfg.hidden;
    const int L = encoder_latent_dim(enc);
    MT_REQUIRE(ctx, count > 0 && count % ((long long)frame * patch) == 0, MT_ERR_SHAPE,
               "mt_vae_encode: reference audio must be a whole number of %d-sample patches, got %lld", frame * patch,
               count);
    const int frames = (int)(count / frame);
    MT_REQUIRE(ctx, frames <= W.max_frames, MT_ERR_CAPACITY, "mt_vae_encode: %d frames, the encoder holds %d", frames,
               W.max_frames);
    const int latents = frames / patch, prow = latents * (patch + 1);
    cudaStream_t s = as_stream(stream);

    std::vector<float> padded((size_t)frames * pf, 0.0f);
    for (int f = 0; f < frames; f++)
        for (int i = 0; i < frame; i++) padded[(size_t)f * pf + i] = bf16_rounded(samples[(size_t)f * frame + i]);
    float inv_freq[32];
    for (int i = 0; i < 32; i++) inv_freq[i] = 1.0f / powf(W.stack.cfg.rope_theta, (float)(2 * i) / 64.0f);

    Scratch sc;
    const size_t need = Scratch::size((size_t)frames * pf) + 3 * Scratch::size((size_t)frames * H) +
                        2 * Scratch::size((size_t)prow * H) + Scratch::size((size_t)latents * H) +
                        Scratch::size((size_t)latents * 2 * L) + Scratch::size(32) +
                        qwen_scratch_floats(W.stack.cfg, frames, frames) +
                        qwen_scratch_floats(W.aggregator.cfg, prow, prow);
    if (!sc.reserve(need)) {
        cudaGetLastError();
        return fail(ctx, MT_ERR_NOMEM, "mt_vae_encode: %zu bytes of device memory", need);
    }
    float* d_frames = sc.take((size_t)frames * pf);
    float* proj = sc.take((size_t)frames * H);
    float* x = sc.take((size_t)frames * H);
    float* normed = sc.take((size_t)frames * H);
    float* patches = sc.take((size_t)prow * H);
    float* patches_normed = sc.take((size_t)prow * H);
    float* cls_rows = sc.take((size_t)latents * H);
    float* posterior = sc.take((size_t)latents * 2 * L);
    float* d_inv = sc.take(32);
    if (sc.overflow) return fail(ctx, MT_ERR_CAPACITY, "mt_vae_encode: scratch sizing");
    cudaMemcpyAsync(d_frames, padded.data(), padded.size() * 4, cudaMemcpyHostToDevice, s);
    cudaMemcpyAsync(d_inv, inv_freq, sizeof(inv_freq), cudaMemcpyHostToDevice, s);

    TRY(mt_linear(ctx, s, d_frames, pf, frames, W.fc1_w, nullptr, nullptr, H, pf, proj, H, 0));
    TRY(mt_linear(ctx, s, proj, H, frames, W.fc2_w, nullptr, W.fc2_b, H, H, x, H, MT_LINEAR_BIAS));
    TRY(qwen_prefill(ctx, s, W.stack, x, frames, frames, normed, sc, d_inv));
    assemble_patches_kernel<<<std::min(1184, (prow * H + 255) / 256), 256, 0, s>>>(normed, W.cls, patches, latents,
                                                                                  patch, H);
    TRY(qwen_prefill(ctx, s, W.aggregator, patches, prow, prow, patches_normed, sc, d_inv));
    // cls row of each patch (VAEEncoder.swift:94-96)
    cudaMemcpy2DAsync(cls_rows, (size_t)H * 4, patches_normed + (size_t)patch * H, (size_t)(patch + 1) * H * 4,
                      (size_t)H * 4, latents, cudaMemcpyDeviceToDevice, s);
    TRY(mt_linear(ctx, s, cls_rows, H, latents, W.fc3_w, nullptr, W.fc3_b, 2 * L, H, posterior, 2 * L, MT_LINEAR_BIAS));
    std::vector<float> raw((size_t)latents * 2 * L);
    cudaMemcpyAsync(raw.data(), posterior, raw.size() * 4, cudaMemcpyDeviceToHost, s);
    TRY(sync(ctx, s, "mt_vae_encode"));
    for (int p = 0; p < latents; p++)
        for (int i = 0; i < L; i++) {
            mean[(size_t)p * L + i] = raw[(size_t)p * 2 * L + i];
            stdv[(size_t)p * L + i] = softplus(raw[(size_t)p * 2 * L + L + i]) + 1e-4f;
        }
    return MT_OK;
}

mt_status mt_aggregate_latents(mt_ctx* ctx, const mt_model* model, void* stream, const float* latents_host, int count,
                               float* rows_host) {
    MT_REQUIRE(ctx, ctx && model && latents_host && rows_host, MT_ERR_ARG, "mt_aggregate_latents: null argument");
    const mt_model_config& c = *mt_model_get_config(model);
    const mt_model_weights& w = *mt_model_get_weights(model);
    MT_REQUIRE(ctx, count >= 1 && count <= c.llm_capacity, MT_ERR_CAPACITY,
               "mt_aggregate_latents: %d reference latents exceed the %d position cache", count, c.llm_capacity);
    const mt_dit_config& d = c.agg;
    const int h = d.hidden, L = c.latent_dim, rows = 2 * count, out_dim = d.out_dim;
    cudaStream_t s = as_stream(stream);
    Scratch sc;
    const size_t need = Scratch::size((size_t)count * L) + Scratch::size((size_t)rows * h) * 3 +
                        Scratch::size((size_t)rows * 3 * h) + Scratch::size((size_t)rows * d.ff) +
                        Scratch::size((size_t)rows * out_dim);
    if (!sc.reserve(need)) {
        cudaGetLastError();
        return fail(ctx, MT_ERR_NOMEM, "mt_aggregate_latents: %zu bytes of device memory", need);
    }
    float* lat = sc.take((size_t)count * L);
    float* x = sc.take((size_t)rows * h);
    float* normed = sc.take((size_t)rows * h);
    float* attn = sc.take((size_t)rows * h);
    float* qkv = sc.take((size_t)rows * 3 * h);
    float* ff = sc.take((size_t)rows * d.ff);
    float* out = sc.take((size_t)rows * out_dim);
    if (sc.overflow) return fail(ctx, MT_ERR_CAPACITY, "mt_aggregate_latents: scratch sizing");
    cudaMemcpyAsync(lat, latents_host, (size_t)count * L * 4, cudaMemcpyHostToDevice, s);
    cls_rows_kernel<<<std::min(1184, (count * h + 255) / 256), 256, 0, s>>>(w.agg_cls, x, count, h);
    TRY(mt_linear(ctx, s, lat, L, count, w.agg_x_w, nullptr, w.agg_x_b, h, L, x + h, 2 * h, MT_LINEAR_BIAS));
    // DiTForward.encode (DiT.swift:35-52), batch count, sequence 2, every row through the final layer.
    for (int b = 0; b < d.depth; b++) {
        const mt_dit_block& B = w.agg.blocks[b];
        TRY(mt_rmsnorm(ctx, s, x, h, rows, h, B.norm1, normed, h, d.eps));
        TRY(mt_linear(ctx, s, normed, h, rows, B.qkv_w, nullptr, B.qkv_b, 3 * h, h, qkv, 3 * h, MT_LINEAR_BIAS));
        TRY(mt_dit_attention(ctx, s, qkv, 3 * h, count, 2, d.heads, w.agg.inv_freq, attn, h));
        TRY(mt_linear(ctx, s, attn, h, rows, B.out_w, nullptr, B.out_b, h, h, x, h, MT_LINEAR_BIAS | MT_LINEAR_ACCUM));
        TRY(mt_rmsnorm(ctx, s, x, h, rows, h, B.norm2, normed, h, d.eps));
        TRY(mt_linear(ctx, s, normed, h, rows, B.ff1_w, nullptr, B.ff1_b, d.ff, h, ff, d.ff,
                      MT_LINEAR_BIAS | MT_LINEAR_GELU));
        TRY(mt_linear(ctx, s, ff, d.ff, rows, B.ff2_w, nullptr, B.ff2_b, h, d.ff, x, h, MT_LINEAR_BIAS | MT_LINEAR_ACCUM));
    }
    TRY(mt_rmsnorm(ctx, s, x, h, rows, h, w.agg.final_norm, normed, h, d.eps));
    TRY(mt_linear(ctx, s, normed, h, rows, w.agg.final_w, nullptr, w.agg.final_b, out_dim, h, out, out_dim,
                  MT_LINEAR_BIAS));
    // row 0 of each sequence (Engine.swift:252-254)
    cudaMemcpy2DAsync(rows_host, (size_t)out_dim * 4, out, (size_t)2 * out_dim * 4, (size_t)out_dim * 4, count,
                      cudaMemcpyDeviceToHost, s);
    return sync(ctx, s, "mt_aggregate_latents");
}

}  // extern "C"
