/*
 * oracle.h -- CPU restatement of the Ming-TTS hot path (TEST INFRASTRUCTURE ONLY).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load this code, and only
 * as the checker or the timed CPU baseline. The product (libmingcuda.so) never links or calls it.
 *
 * Each function restates one reference kernel or stage (Swift + Metal, maralski/ming-tts) and cites
 * the file:line it follows. Dot products accumulate in double (the "fp64 host check" of the parity
 * bar); element-wise epilogues use fp32 in the reference's operation order.
 *
 * Pinning: the reference ships no golden tensors for kernels (its goldens are unpublished and its
 * KernelTests compare GPU vs scalar CPU loops). The restatement is pinned against independent
 * implementations of the same published algorithms (numpy/torch: irfft, linear interpolation,
 * softmax attention) and against the reference's own CPU reference loops
 * (Tests/MingTTSTests/KernelTests.swift), via fixtures under tests/golden/.
 */
#ifndef MING_ORACLE_H
#define MING_ORACLE_H

#include <stddef.h>
#include <stdint.h>
#include "../include/mingcuda.h"

#ifdef __cplusplus
extern "C" {
#endif

uint16_t or_bf16_bits(float x);
float or_bf16_to_f32(uint16_t v);
float or_gelu_tanh(float x);
float or_silu(float x);

/* KernelTests.swift:21-28 LCG: state = state*6364136223846793005 + 1442695040888963407,
 * value = (state >> 40) / 2^24 * 2 - 1, times scale. Advances *state. */
void or_lcg_floats(uint64_t* state, float* out, size_t n, float scale);
/* Engine.swift:433-453 gaussianNoise. */
void or_gaussian_noise(float* out, size_t count, uint64_t seed);
/* std * gaussianNoise stream rounded to bf16 (the synthetic weight generator). */
void or_randn_bf16(uint16_t* out, size_t count, uint64_t seed, float std);

void or_linear(const float* x, int ldx, int m, const uint16_t* w, const uint16_t* w2,
               const uint16_t* bias, int n, int k, float* y, int ldy, uint32_t flags);
void or_rmsnorm(const float* x, int ldx, int rows, int width, const uint16_t* w, float* y, int ldy,
                float eps);
void or_rope_cache(float* qkv, int ldq, int m, int hq, int hkv, int pos0, float* kc, float* vc,
                   int cap, const float* inv_freq);
void or_attention(const float* q, int ldq, int m, int hq, int hkv, int pos0, int window,
                  const float* kc, const float* vc, int cap, float* out, int ldo);
void or_dit_attention(const float* qkv, int ld, int batch, int seq, int heads,
                      const float* inv_freq, float* out, int ldo);
void or_flow_assemble(const float* y, const float* history, const float* cemb,
                      const uint16_t* cbias, const float* temb, const uint16_t* xw,
                      const uint16_t* xb, int hidden, int latent, float* x);
void or_flow_euler(float* y, const float* pred, int ldp, int pred_row, int null_row, int latent,
                   float cfg, float dt, float* capture);
void or_upsample4(const float* prev, const float* cur, const float* next, int hidden, float* frames);
void or_istft_frames(const float* spec, int ld_spec, int count, int nfft, const float* window,
                     float* frames, int frame0, int ring);
void or_istft_emit(const float* frames, const float* window, int nfft, int hop, int s0, int count,
                   int last_frame, int ring, float* out);

/* FlowSchedule.timesteps (DiT.swift:56-65): steps+1 values. */
void or_flow_timesteps(int steps, float* out);
/* FlowSchedule.sinusoid (DiT.swift:68-79): 256 values. */
void or_sinusoid(float t, float* out256);

#ifdef __cplusplus
}
#endif
#endif
