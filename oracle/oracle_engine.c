/*
 * oracle_engine.c -- CPU restatement of one generation (TEST INFRASTRUCTURE ONLY; see oracle.h).
 *
 * Follows, step for step, MingEngine.generate / encodeStep (Sources/MingTTS/Engine/Engine.swift:
 * 302-415), QwenForward.dispatches (Qwen.swift:72-97), DiTForward.encode (DiT.swift:35-52),
 * the temb precompute (Engine.swift:187-198) and the streaming VAEDecoder (VAEDecoder.swift:64-107),
 * built from the kernel restatements in oracle.c. One request, reference buffer layout (the VAE
 * KV cache keeps every position: capacity 4 * latents + 8).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "oracle.h"
#include "oracle_engine.h"

#define ALLOC(n) ((float*)calloc((size_t)(n) > 0 ? (size_t)(n) : 1, sizeof(float)))

typedef struct {
    const mt_qwen_weights* w;
    float* cache;  /* [layers][2][kv][cap][64] */
    int cap;
    int length;
    float inv_freq[32];
    float *normed, *qkv, *attn, *mlp;
} qwen_state;

static void qwen_init(qwen_state* s, const mt_qwen_weights* w, int cap, int max_rows) {
    const mt_qwen_config* c = &w->cfg;
    s->w = w;
    s->cap = cap;
    s->length = 0;
    s->cache = ALLOC((size_t)c->layers * 2 * c->kv_heads * cap * 64);
    for (int i = 0; i < 32; i++) s->inv_freq[i] = 1.0f / powf(c->rope_theta, (float)(2 * i) / 64.0f);
    const int qkvw = (c->heads + 2 * c->kv_heads) * 64;
    s->normed = ALLOC((size_t)max_rows * c->hidden);
    s->qkv = ALLOC((size_t)max_rows * qkvw);
    s->attn = ALLOC((size_t)max_rows * c->heads * 64);
    s->mlp = ALLOC((size_t)max_rows * c->intermediate);
}

static void qwen_free(qwen_state* s) {
    free(s->cache);
    free(s->normed);
    free(s->qkv);
    free(s->attn);
    free(s->mlp);
}

/* QwenForward.dispatches (Qwen.swift:72-97). capture(layer, x) is called after each layer. */
static void qwen_forward(qwen_state* s, float* x, int rows, int norm_rows, float* out,
                         float* cap0, float* cap_last) {
    const mt_qwen_config* c = &s->w->cfg;
    const int H = c->hidden, qkvw = (c->heads + 2 * c->kv_heads) * 64;
    const int pos0 = s->length;
    const size_t per_tensor = (size_t)c->kv_heads * s->cap * 64;
    for (int l = 0; l < c->layers; l++) {
        const mt_qwen_layer* L = &s->w->layers[l];
        float* kc = s->cache + (size_t)(2 * l) * per_tensor;
        float* vc = s->cache + (size_t)(2 * l + 1) * per_tensor;
        or_rmsnorm(x, H, rows, H, L->norm1, s->normed, H, c->eps);
        or_linear(s->normed, H, rows, L->qkv_w, NULL, L->qkv_b, qkvw, H, s->qkv, qkvw, MT_LINEAR_BIAS);
        or_rope_cache(s->qkv, qkvw, rows, c->heads, c->kv_heads, pos0, kc, vc, s->cap, s->inv_freq);
        or_attention(s->qkv, qkvw, rows, c->heads, c->kv_heads, pos0, c->window, kc, vc, s->cap, s->attn,
                     c->heads * 64);
        or_linear(s->attn, c->heads * 64, rows, L->o_w, NULL, NULL, H, c->heads * 64, x, H, MT_LINEAR_ACCUM);
        or_rmsnorm(x, H, rows, H, L->norm2, s->normed, H, c->eps);
        or_linear(s->normed, H, rows, L->gate_w, L->up_w, NULL, c->intermediate, H, s->mlp, c->intermediate,
                  MT_LINEAR_SILU_GATE);
        or_linear(s->mlp, c->intermediate, rows, L->down_w, NULL, NULL, H, c->intermediate, x, H, MT_LINEAR_ACCUM);
        if (l == 0 && cap0) memcpy(cap0, x, sizeof(float) * (size_t)rows * H);
        if (l == c->layers - 1 && cap_last) memcpy(cap_last, x, sizeof(float) * (size_t)rows * H);
    }
    or_rmsnorm(x + (size_t)(rows - norm_rows) * H, H, norm_rows, H, s->w->final_norm, out, H, c->eps);
    s->length += rows;
}

typedef struct {
    const mt_dit_weights* w;
    float *normed, *qkv, *attn, *ff;
} dit_state;

static void dit_init(dit_state* s, const mt_dit_weights* w, int max_rows) {
    s->w = w;
    s->normed = ALLOC((size_t)max_rows * w->cfg.hidden);
    s->qkv = ALLOC((size_t)max_rows * 3 * w->cfg.hidden);
    s->attn = ALLOC((size_t)max_rows * w->cfg.hidden);
    s->ff = ALLOC((size_t)max_rows * w->cfg.ff);
}

static void dit_free(dit_state* s) {
    free(s->normed);
    free(s->qkv);
    free(s->attn);
    free(s->ff);
}

/* DiTForward.encode (DiT.swift:35-52). */
static void dit_forward(dit_state* s, float* x, int batch, int seq, int out_rows, float* out) {
    const mt_dit_config* c = &s->w->cfg;
    const int h = c->hidden, rows = batch * seq;
    for (int b = 0; b < c->depth; b++) {
        const mt_dit_block* B = &s->w->blocks[b];
        or_rmsnorm(x, h, rows, h, B->norm1, s->normed, h, c->eps);
        or_linear(s->normed, h, rows, B->qkv_w, NULL, B->qkv_b, 3 * h, h, s->qkv, 3 * h, MT_LINEAR_BIAS);
        or_dit_attention(s->qkv, 3 * h, batch, seq, c->heads, s->w->inv_freq, s->attn, h);
        or_linear(s->attn, h, rows, B->out_w, NULL, B->out_b, h, h, x, h, MT_LINEAR_BIAS | MT_LINEAR_ACCUM);
        or_rmsnorm(x, h, rows, h, B->norm2, s->normed, h, c->eps);
        or_linear(s->normed, h, rows, B->ff1_w, NULL, B->ff1_b, c->ff, h, s->ff, c->ff, MT_LINEAR_BIAS | MT_LINEAR_GELU);
        or_linear(s->ff, c->ff, rows, B->ff2_w, NULL, B->ff2_b, h, c->ff, x, h, MT_LINEAR_BIAS | MT_LINEAR_ACCUM);
    }
    or_rmsnorm(x, h, out_rows, h, s->w->final_norm, s->normed, h, c->eps);
    or_linear(s->normed, h, out_rows, s->w->final_w, NULL, s->w->final_b, c->out_dim, h, out, c->out_dim,
              MT_LINEAR_BIAS);
}

typedef struct {
    const mt_model_config* cfg;
    const mt_model_weights* w;
    qwen_state stack;
    float *h, *frames, *hidden, *spec, *ring, *pcm;
    int latents, decoded, emitted;
} vae_state;

/* VAEDecoder.encodeFc1 (VAEDecoder.swift:64-67). */
static void vae_fc1(vae_state* v, const float* latent) {
    const int Hv = v->cfg->vae.hidden;
    or_linear(latent, v->cfg->latent_dim, 1, v->w->vae_fc1_w, NULL, v->w->vae_fc1_b, Hv, v->cfg->latent_dim,
              v->h + (size_t)(v->latents % 3) * Hv, Hv, MT_LINEAR_BIAS);
    v->latents++;
}

/* VAEDecoder.decodeDispatches (VAEDecoder.swift:86-107); returns the emitted count. */
static int vae_decode(vae_state* v, int n, int has_next, float* hidden_out) {
    const mt_model_config* c = v->cfg;
    const int Hv = c->vae.hidden, N = c->nfft, hop = c->hop, pad = (N - hop) / 2;
    const float* prev = n >= 1 ? v->h + (size_t)((n - 1) % 3) * Hv : NULL;
    const float* cur = v->h + (size_t)(n % 3) * Hv;
    const float* next = has_next ? v->h + (size_t)((n + 1) % 3) * Hv : NULL;
    or_upsample4(prev, cur, next, Hv, v->frames);
    qwen_forward(&v->stack, v->frames, 4, 4, v->hidden, NULL, NULL);
    if (hidden_out) memcpy(hidden_out, v->hidden, sizeof(float) * 4 * Hv);
    or_linear(v->hidden, Hv, 4, v->w->vae_head_w, NULL, v->w->vae_head_b, N + 2, Hv, v->spec, N + 2, MT_LINEAR_BIAS);
    or_istft_frames(v->spec, N + 2, 4, N, v->w->vae_window, v->ring, 4 * n, 8);
    const int frame_count = 4 * (n + 1);
    const int final_end = has_next ? frame_count * hop - pad : frame_count * hop;
    const int count = final_end - v->emitted;
    or_istft_emit(v->ring, v->w->vae_window, N, hop, v->emitted, count, frame_count - 1, 8, v->pcm);
    v->emitted = final_end;
    v->decoded = n + 1;
    return count;
}

int or_generate(const mt_model_config* cfg, const mt_model_weights* w, or_generate_io* io) {
    const int H = cfg->llm.hidden, L = cfg->latent_dim, Df = cfg->flow.hidden, Da = cfg->agg.hidden;
    const int T = io->prompt_rows;
    if (T < 1 || T >= cfg->llm_capacity) return 1;
    int steps = io->steps;
    if (steps > cfg->llm_capacity - T) steps = cfg->llm_capacity - T;
    const int FS = cfg->flow_steps;

    qwen_state llm;
    qwen_init(&llm, &w->llm, cfg->llm_capacity, T);
    dit_state flow, agg;
    dit_init(&flow, &w->flow, 6);
    dit_init(&agg, &w->agg, 2);
    vae_state vae;
    memset(&vae, 0, sizeof(vae));
    vae.cfg = cfg;
    vae.w = w;
    qwen_init(&vae.stack, &w->vae, 4 * (steps + 1) + 8, 4);
    const int Hv = cfg->vae.hidden;
    vae.h = ALLOC(3 * Hv);
    vae.frames = ALLOC(4 * Hv);
    vae.hidden = ALLOC(4 * Hv);
    vae.spec = ALLOC(4 * (cfg->nfft + 2));
    vae.ring = ALLOC(8 * cfg->nfft);
    vae.pcm = ALLOC(4 * cfg->hop + (cfg->nfft - cfg->hop) / 2);

    /* Time embeddings (Engine.swift:187-198). */
    float* ts = ALLOC(FS + 1);
    or_flow_timesteps(FS, ts);
    float* sinus = ALLOC((size_t)FS * cfg->time_dim);
    for (int k = 0; k < FS; k++) or_sinusoid(ts[k], sinus + (size_t)k * cfg->time_dim);
    float* tmid = ALLOC((size_t)FS * Df);
    float* temb = ALLOC((size_t)FS * Df);
    or_linear(sinus, cfg->time_dim, FS, w->flow_t1_w, NULL, w->flow_t1_b, Df, cfg->time_dim, tmid, Df,
              MT_LINEAR_BIAS | MT_LINEAR_SILU);
    or_linear(tmid, Df, FS, w->flow_t2_w, NULL, w->flow_t2_b, Df, Df, temb, Df, MT_LINEAR_BIAS);

    float* x = ALLOC((size_t)T * H);
    memcpy(x, io->embeds, sizeof(float) * (size_t)T * H);
    float* z = ALLOC(H);
    float* cemb = ALLOC(Df);
    float* y = ALLOC(L);
    float* history = ALLOC(L);
    if (io->initial_history) memcpy(history, io->initial_history, sizeof(float) * L);
    float* ditX = ALLOC(6 * Df);
    float* ditOut = ALLOC(6 * L);
    float* aggX = ALLOC(2 * Da);
    float* xllm = ALLOC(H);
    float* vel = ALLOC(2 * L);

    /* Prefill (Engine.swift:323-333). */
    qwen_forward(&llm, x, T, 1, z, io->layer0_prefill, io->layer_last_prefill);

    long pcm_count = 0;
    int chunks = 0;
    int n = 0;
    io->stopped = 0;
    for (n = 0; n < steps; n++) {
        /* Stage "llm" (Engine.swift:381-385): token n > 0, VAE frames of latent n-2, stop head. */
        if (n > 0) qwen_forward(&llm, xllm, 1, 1, z, NULL, NULL);
        int chunk = -1;
        if (vae.decoded + 1 < vae.latents) {
            chunk = vae_decode(&vae, vae.decoded, 1, io->vae_hidden ? io->vae_hidden + (size_t)vae.decoded * 4 * Hv : NULL);
        }
        float logits[2];
        or_linear(z, H, 1, w->stop_w, NULL, w->stop_b, 2, H, logits, 2, MT_LINEAR_BIAS);
        /* Stage "flow" (Engine.swift:387-403). */
        or_linear(z, H, 1, w->flow_c_w, NULL, w->flow_c_b, Df, H, cemb, Df, MT_LINEAR_BIAS);
        if (n > 0) memcpy(history, y, sizeof(float) * L);
        memcpy(y, io->noise + (size_t)n * L, sizeof(float) * L);
        for (int k = 0; k < FS; k++) {
            or_flow_assemble(y, history, cemb, w->flow_c_b, temb + (size_t)k * Df, w->flow_x_w, w->flow_x_b, Df, L, ditX);
            dit_forward(&flow, ditX, 2, 3, 6, ditOut);
            or_flow_euler(y, ditOut, L, 2, 5, L, io->cfg, ts[k + 1] - ts[k], vel);
            if (n == 0 && io->velocity0) memcpy(io->velocity0 + (size_t)k * 2 * L, vel, sizeof(float) * 2 * L);
        }
        if (io->latents) memcpy(io->latents + (size_t)n * L, y, sizeof(float) * L);
        /* Stage "agg" (Engine.swift:406-410). */
        memcpy(aggX, w->agg_cls, sizeof(float) * Da);
        or_linear(y, L, 1, w->agg_x_w, NULL, w->agg_x_b, Da, L, aggX + Da, Da, MT_LINEAR_BIAS);
        dit_forward(&agg, aggX, 1, 2, 1, xllm);
        /* Stage "vae" (Engine.swift:412-413). */
        vae_fc1(&vae, y);

        if (io->stop_logits) {
            io->stop_logits[2 * n] = logits[0];
            io->stop_logits[2 * n + 1] = logits[1];
        }
        if (io->llm_hidden) memcpy(io->llm_hidden + (size_t)n * H, z, sizeof(float) * H);
        if (io->agg_out) memcpy(io->agg_out + (size_t)n * H, xllm, sizeof(float) * H);
        if (chunk >= 0) {
            if (io->chunk_counts) io->chunk_counts[chunks] = chunk;
            chunks++;
            if (io->pcm && pcm_count + chunk <= io->pcm_cap) memcpy(io->pcm + pcm_count, vae.pcm, sizeof(float) * chunk);
            pcm_count += chunk;
        }
        if (io->step_seconds) {
            struct timespec ts_now;
            clock_gettime(CLOCK_MONOTONIC, &ts_now);
            io->step_seconds[n] = (double)ts_now.tv_sec + 1e-9 * (double)ts_now.tv_nsec;
        }
        const float stop_prob = 1.0f / (1.0f + expf(logits[0] - logits[1]));
        if (io->obey_stop && stop_prob > 0.5f && n > 3) {
            io->stopped = 1;
            n++;
            break;
        }
    }
    io->steps_run = n;
    /* Flush (Engine.swift:360-367). */
    while (vae.decoded < vae.latents) {
        const int d = vae.decoded;
        const int chunk = vae_decode(&vae, d, d + 1 < vae.latents, io->vae_hidden ? io->vae_hidden + (size_t)d * 4 * Hv : NULL);
        if (io->chunk_counts) io->chunk_counts[chunks] = chunk;
        chunks++;
        if (io->pcm && pcm_count + chunk <= io->pcm_cap) memcpy(io->pcm + pcm_count, vae.pcm, sizeof(float) * chunk);
        pcm_count += chunk;
    }
    io->pcm_count = pcm_count;
    io->chunks = chunks;

    qwen_free(&llm);
    qwen_free(&vae.stack);
    dit_free(&flow);
    dit_free(&agg);
    free(vae.h); free(vae.frames); free(vae.hidden); free(vae.spec); free(vae.ring); free(vae.pcm);
    free(ts); free(sinus); free(tmid); free(temb);
    free(x); free(z); free(cemb); free(y); free(history); free(ditX); free(ditOut); free(aggX); free(xllm); free(vel);
    return 0;
}

/* One pass of the Qwen stack over `rows` new rows at positions length.. of a caller-owned cache
 * ([layers][2][kv][cap][64], first `length` positions already filled); z_out gets the final norm of
 * every row. The LLM decode step of the reference is rows = 1. */
int or_llm_decode(const mt_qwen_weights* w, float* cache, int cap, int length, const float* x_in, int rows,
                  float* z_out) {
    qwen_state s;
    const mt_qwen_config* c = &w->cfg;
    s.w = w;
    s.cap = cap;
    s.length = length;
    s.cache = cache;
    for (int i = 0; i < 32; i++) s.inv_freq[i] = 1.0f / powf(c->rope_theta, (float)(2 * i) / 64.0f);
    const int qkvw = (c->heads + 2 * c->kv_heads) * 64;
    s.normed = ALLOC((size_t)rows * c->hidden);
    s.qkv = ALLOC((size_t)rows * qkvw);
    s.attn = ALLOC((size_t)rows * c->heads * 64);
    s.mlp = ALLOC((size_t)rows * c->intermediate);
    float* x = ALLOC((size_t)rows * c->hidden);
    memcpy(x, x_in, sizeof(float) * (size_t)rows * c->hidden);
    qwen_forward(&s, x, rows, rows, z_out, NULL, NULL);
    free(x);
    free(s.normed);
    free(s.qkv);
    free(s.attn);
    free(s.mlp);
    return 0;
}

/* One flow-matching patch (the "flow" stage of MingEngine.encodeStep, Engine.swift:387-403): c_emb of
 * the LLM output z, then flow_steps Euler steps of the CFG DiT from noise with the given history;
 * the latent goes to y_out [latent]. */
int or_flow_patch(const mt_model_config* cfg, const mt_model_weights* w, const float* z, const float* history,
                  const float* noise, float cfg_scale, float* y_out) {
    const int L = cfg->latent_dim, Df = cfg->flow.hidden, FS = cfg->flow_steps;
    float* ts = ALLOC(FS + 1);
    or_flow_timesteps(FS, ts);
    float* sinus = ALLOC((size_t)FS * cfg->time_dim);
    for (int k = 0; k < FS; k++) or_sinusoid(ts[k], sinus + (size_t)k * cfg->time_dim);
    float* tmid = ALLOC((size_t)FS * Df);
    float* temb = ALLOC((size_t)FS * Df);
    or_linear(sinus, cfg->time_dim, FS, w->flow_t1_w, NULL, w->flow_t1_b, Df, cfg->time_dim, tmid, Df,
              MT_LINEAR_BIAS | MT_LINEAR_SILU);
    or_linear(tmid, Df, FS, w->flow_t2_w, NULL, w->flow_t2_b, Df, Df, temb, Df, MT_LINEAR_BIAS);
    float* cemb = ALLOC(Df);
    float* ditX = ALLOC(6 * Df);
    float* ditOut = ALLOC(6 * L);
    float* vel = ALLOC(2 * L);
    dit_state flow;
    dit_init(&flow, &w->flow, 6);
    or_linear(z, cfg->llm.hidden, 1, w->flow_c_w, NULL, w->flow_c_b, Df, cfg->llm.hidden, cemb, Df, MT_LINEAR_BIAS);
    memcpy(y_out, noise, sizeof(float) * L);
    for (int k = 0; k < FS; k++) {
        or_flow_assemble(y_out, history, cemb, w->flow_c_b, temb + (size_t)k * Df, w->flow_x_w, w->flow_x_b, Df, L, ditX);
        dit_forward(&flow, ditX, 2, 3, 6, ditOut);
        or_flow_euler(y_out, ditOut, L, 2, 5, L, cfg_scale, ts[k + 1] - ts[k], vel);
    }
    dit_free(&flow);
    free(ts); free(sinus); free(tmid); free(temb); free(cemb); free(ditX); free(ditOut); free(vel);
    return 0;
}

/* The streaming VAE decoder over `count` latents [count, latent] (VAEDecoder.swift:64-107): fc1 of
 * every latent, then each latent's frames decoded and emitted as the generation loop and its flush
 * do (latent d once latent d + 1 exists, the last one without a look-ahead). pcm receives up to
 * pcm_cap samples; returns the sample count. */
long or_vae_decode_clip(const mt_model_config* cfg, const mt_model_weights* w, const float* latents, int count,
                        float* pcm, long pcm_cap) {
    const int Hv = cfg->vae.hidden;
    vae_state vae;
    memset(&vae, 0, sizeof(vae));
    vae.cfg = cfg;
    vae.w = w;
    qwen_init(&vae.stack, &w->vae, 4 * (count + 1) + 8, 4);
    vae.h = ALLOC(3 * Hv);
    vae.frames = ALLOC(4 * Hv);
    vae.hidden = ALLOC(4 * Hv);
    vae.spec = ALLOC(4 * (cfg->nfft + 2));
    vae.ring = ALLOC(8 * cfg->nfft);
    vae.pcm = ALLOC(4 * cfg->hop + (cfg->nfft - cfg->hop) / 2);
    long total = 0;
    for (int n = 0; n <= count; n++) {
        if (n < count) vae_fc1(&vae, latents + (size_t)n * cfg->latent_dim);
        while (vae.decoded + 1 < vae.latents || (n == count && vae.decoded < vae.latents)) {
            const int d = vae.decoded;
            const int c = vae_decode(&vae, d, d + 1 < vae.latents, NULL);
            if (pcm && total + c <= pcm_cap) memcpy(pcm + total, vae.pcm, sizeof(float) * c);
            total += c;
        }
    }
    qwen_free(&vae.stack);
    free(vae.h); free(vae.frames); free(vae.hidden); free(vae.spec); free(vae.ring); free(vae.pcm);
    return total;
}

/* bf16Rounded (VAEEncoder.swift:110-114). */
static float bf16_rounded(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

int or_vae_encode(const mt_model_config* cfg, const mt_encoder_weights* w, const float* samples, long count,
                  float* mean, float* std_out) {
    const int frame = w->frame, patch = w->patch, pf = w->padded_frame, H = w->stack.cfg.hidden;
    const int L = cfg->latent_dim;
    if (count <= 0 || count % ((long)frame * patch) != 0) return -1;
    const int frames = (int)(count / frame), latents = frames / patch, prow = latents * (patch + 1);
    float* fr = ALLOC((size_t)frames * pf);
    float* proj = ALLOC((size_t)frames * H);
    float* x = ALLOC((size_t)frames * H);
    float* normed = ALLOC((size_t)frames * H);
    float* patches = ALLOC((size_t)prow * H);
    float* pnormed = ALLOC((size_t)prow * H);
    float* cls_rows = ALLOC((size_t)latents * H);
    float* post = ALLOC((size_t)latents * 2 * L);
    for (int f = 0; f < frames; f++)
        for (int i = 0; i < frame; i++) fr[(size_t)f * pf + i] = bf16_rounded(samples[(size_t)f * frame + i]);
    or_linear(fr, pf, frames, w->fc1_w, NULL, NULL, H, pf, proj, H, 0);
    or_linear(proj, H, frames, w->fc2_w, NULL, w->fc2_b, H, H, x, H, MT_LINEAR_BIAS);
    qwen_state st;
    qwen_init(&st, &w->stack, frames, frames);
    qwen_forward(&st, x, frames, frames, normed, NULL, NULL);
    qwen_free(&st);
    for (int p = 0; p < latents; p++) {  /* [patch frame rows | cls] (VAEEncoder.swift:88-92) */
        memcpy(patches + (size_t)p * (patch + 1) * H, normed + (size_t)p * patch * H, sizeof(float) * (size_t)patch * H);
        memcpy(patches + ((size_t)p * (patch + 1) + patch) * H, w->cls, sizeof(float) * (size_t)H);
    }
    qwen_state ag;
    qwen_init(&ag, &w->aggregator, prow, prow);
    qwen_forward(&ag, patches, prow, prow, pnormed, NULL, NULL);
    qwen_free(&ag);
    for (int p = 0; p < latents; p++)
        memcpy(cls_rows + (size_t)p * H, pnormed + ((size_t)p * (patch + 1) + patch) * H, sizeof(float) * (size_t)H);
    or_linear(cls_rows, H, latents, w->fc3_w, NULL, w->fc3_b, 2 * L, H, post, 2 * L, MT_LINEAR_BIAS);
    for (int p = 0; p < latents; p++)
        for (int i = 0; i < L; i++) {
            const float s = post[(size_t)p * 2 * L + L + i];
            mean[(size_t)p * L + i] = post[(size_t)p * 2 * L + i];
            std_out[(size_t)p * L + i] = (s > 20.0f ? s : log1pf(expf(s))) + 1e-4f;  /* softplus + 1e-4 */
        }
    free(fr); free(proj); free(x); free(normed); free(patches); free(pnormed); free(cls_rows); free(post);
    return 0;
}

int or_aggregate_latents(const mt_model_config* cfg, const mt_model_weights* w, const float* latents, int count,
                         float* rows) {
    const int h = cfg->agg.hidden, L = cfg->latent_dim, od = cfg->agg.out_dim;
    float* x = ALLOC((size_t)2 * count * h);
    float* out = ALLOC((size_t)2 * count * od);
    for (int p = 0; p < count; p++) memcpy(x + (size_t)2 * p * h, w->agg_cls, sizeof(float) * (size_t)h);
    or_linear(latents, L, count, w->agg_x_w, NULL, w->agg_x_b, h, L, x + h, 2 * h, MT_LINEAR_BIAS);
    dit_state ds;
    dit_init(&ds, &w->agg, 2 * count);
    dit_forward(&ds, x, count, 2, 2 * count, out);
    dit_free(&ds);
    for (int p = 0; p < count; p++) memcpy(rows + (size_t)p * od, out + (size_t)2 * p * od, sizeof(float) * (size_t)od);
    free(x);
    free(out);
    return 0;
}
