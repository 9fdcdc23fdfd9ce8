// engine_kernels.cuh -- batched kernels of the generation loop (internal).
#pragma once

#include "common.cuh"

namespace mt {

// Device step state: a flat int array [ST_HEADER + 5 * R]. The header holds the step index n, the
// latent d the VAE decodes this step (-1: none) and whether d has a lookahead latent; then, per
// request, the LLM position of this step's token, the VAE position of the first decoded frame
// (4d), and the emission start, count and last frame.
enum { ST_N = 0, ST_D = 1, ST_HAS_NEXT = 2, ST_HEADER = 4 };
constexpr int VAE_H_RING = 4;  // fc1 outputs kept per request (latents d-1, d, d+1 and the new one)

inline int st_llm_pos(int R) { (void)R; return ST_HEADER; }
inline int st_vae_pos(int R) { return ST_HEADER + R; }
inline int st_emit_s0(int R) { return ST_HEADER + 2 * R; }
inline int st_emit_count(int R) { return ST_HEADER + 3 * R; }
inline int st_emit_last(int R) { return ST_HEADER + 4 * R; }
inline int st_size(int R) { return ST_HEADER + 5 * R; }

struct FlowFinalArgs {
    const float* X; int hidden;
    const uint16_t* norm_w; float eps;
    const uint16_t* final_w; const uint16_t* final_b; int latent;
    float* y; float cfg; float dt;
    float* vel0; int flow_steps; int k;
    float* latents; int steps_cap;
    const int* state;
};

void launch_embed_gather(const int32_t* ids, int rows, const uint16_t* table, int hidden, int vocab, float* x,
                         unsigned int* status, cudaStream_t s);
void launch_flow_begin(float* y, float* hist, const float* noise, int latent, int steps_cap, const int* state,
                       int requests, cudaStream_t s);
void launch_flow_assemble_batched(const float* y, const float* hist, const float* cemb, const uint16_t* cbias,
                                  const float* temb, const uint16_t* xw, const uint16_t* xb, int hidden, int latent,
                                  float* X, int requests, cudaStream_t s);
void launch_flow_final(const FlowFinalArgs& a, int requests, cudaStream_t s);
void launch_agg_assemble(const float* y, const float* cls, const uint16_t* xw, const uint16_t* xb, int hidden,
                         int latent, float* X, int requests, cudaStream_t s);
void launch_vae_fc1(const float* y, const uint16_t* w, const uint16_t* b, int hidden, int latent, float* h,
                    const int* state, int requests, cudaStream_t s);
void launch_vae_upsample(const float* h, int hidden, const int* state, float* frames, int requests, cudaStream_t s);

}  // namespace mt
