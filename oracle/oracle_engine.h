/*
 * oracle_engine.h -- CPU restatement of one generation (TEST INFRASTRUCTURE ONLY; see oracle.h).
 */
#ifndef MING_ORACLE_ENGINE_H
#define MING_ORACLE_ENGINE_H

#include "../include/mingcuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    /* inputs */
    int prompt_rows;              /* T */
    const float* embeds;          /* [T, llm.hidden] */
    int steps;                    /* generation steps to run (clamped to the cache) */
    float cfg;                    /* CFG scale (2.0) */
    int obey_stop;                /* 1: stop when p > 0.5 and n > 3 (Engine.swift:352-355) */
    const float* noise;           /* [steps, latent] */
    const float* initial_history; /* [latent] or NULL (zeros) */
    /* outputs (any may be NULL) */
    float* stop_logits;           /* [steps, 2] */
    float* llm_hidden;            /* [steps, llm.hidden] z of each step */
    float* latents;               /* [steps, latent] */
    float* agg_out;               /* [steps, llm.hidden] */
    float* velocity0;             /* [flow_steps, 2, latent] step 0 cond/uncond predictions */
    float* vae_hidden;            /* [steps, 4, vae.hidden] decoder final-norm rows per latent */
    float* layer0_prefill;        /* [T, llm.hidden] residual after layer 0 of the prefill */
    float* layer_last_prefill;    /* [T, llm.hidden] residual after the last layer */
    float* pcm;                   /* all emitted samples in order */
    long pcm_cap;
    int* chunk_counts;            /* [steps + 2] samples per emission */
    double* step_seconds;         /* [steps] monotonic seconds at the end of each step (CPU timing) */
    /* results */
    int steps_run;
    int stopped;
    long pcm_count;
    int chunks;
} or_generate_io;

int or_generate(const mt_model_config* cfg, const mt_model_weights* w, or_generate_io* io);
int or_llm_decode(const mt_qwen_weights* w, float* cache, int cap, int length, const float* x_in, int rows,
                  float* z_out);
/* The flow stage of one step (Engine.swift:387-403): 10 CFG Euler steps from noise -> y_out [latent]. */
int or_flow_patch(const mt_model_config* cfg, const mt_model_weights* w, const float* z, const float* history,
                  const float* noise, float cfg_scale, float* y_out);
/* VAEDecoder.swift:64-107 over count latents, flush included; returns the samples emitted. */
long or_vae_decode_clip(const mt_model_config* cfg, const mt_model_weights* w, const float* latents, int count,
                        float* pcm, long pcm_cap);
/* VAEEncoder.encode (VAEEncoder.swift:56-107): count samples (a multiple of frame * patch) ->
 * mean/std [count / (frame * patch), latent]. Returns 0, or -1 on a bad count. */
int or_vae_encode(const mt_model_config* cfg, const mt_encoder_weights* w, const float* samples, long count,
                  float* mean, float* std_out);
/* MingEngine.aggregate (Engine.swift:236-256): count latents [count, latent] -> rows [count, llm.hidden]. */
int or_aggregate_latents(const mt_model_config* cfg, const mt_model_weights* w, const float* latents, int count,
                         float* rows);

#ifdef __cplusplus
}
#endif
#endif
