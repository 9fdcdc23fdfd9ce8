/*
 * oracle.c -- CPU restatement of the reference kernels (TEST INFRASTRUCTURE ONLY; see oracle.h).
 *
 * Reference: maralski/ming-tts, Sources/MingTTS/Engine/Shaders.swift (Metal kernels) and the CPU
 * reference loops of Tests/MingTTSTests/KernelTests.swift. Dot products accumulate in double.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float bf(uint16_t v) {
    uint32_t u = (uint32_t)v << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* KernelTests.swift:30-34: round to nearest even through +0x7FFF + lsb. */
uint16_t or_bf16_bits(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    uint32_t r = u + 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(r >> 16);
}

float or_bf16_to_f32(uint16_t v) { return bf(v); }

/* Shaders.swift:23-27: u clamped to +-15 before tanh. */
float or_gelu_tanh(float x) {
    const float k = 0.7978845608028654f;
    float u = k * (x + 0.044715f * x * x * x);
    if (u > 15.0f) u = 15.0f;
    if (u < -15.0f) u = -15.0f;
    return 0.5f * x * (1.0f + tanhf(u));
}

/* Shaders.swift:29. */
float or_silu(float x) { return x / (1.0f + expf(-x)); }

void or_lcg_floats(uint64_t* state, float* out, size_t n, float scale) {
    uint64_t s = *state;
    for (size_t i = 0; i < n; i++) {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        out[i] = ((float)(s >> 40) / (float)(1 << 24) * 2.0f - 1.0f) * scale;
    }
    *state = s;
}

/* SplitMix64 draw j (1-based) of Engine.swift:434-442: the state starts at seed + golden and is
 * advanced by golden before each mix, so draw j mixes seed + (j + 1) * golden. */
static inline double sm64_draw(uint64_t seed, uint64_t j) {
    const uint64_t g = 0x9E3779B97F4A7C15ull;
    uint64_t z = seed + (j + 1) * g;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (double)(z >> 11) / (double)(1ull << 53);
}

/* Engine.swift:443-452: pair p takes draws 2p+1 (u1, floored at 1e-300) and 2p+2 (u2). */
static inline void gauss_pair(uint64_t seed, uint64_t p, float* a, float* b) {
    double u1 = sm64_draw(seed, 2 * p + 1), u2 = sm64_draw(seed, 2 * p + 2);
    if (u1 < 1e-300) u1 = 1e-300;
    double r = sqrt(-2.0 * log(u1));
    *a = (float)(r * cos(2.0 * M_PI * u2));
    *b = (float)(r * sin(2.0 * M_PI * u2));
}

void or_gaussian_noise(float* out, size_t count, uint64_t seed) {
    for (size_t i = 0; i < count; i += 2) {
        float a, b;
        gauss_pair(seed, i / 2, &a, &b);
        out[i] = a;
        if (i + 1 < count) out[i + 1] = b;
    }
}

void or_randn_bf16(uint16_t* out, size_t count, uint64_t seed, float std) {
    size_t pairs = (count + 1) / 2;
#pragma omp parallel for schedule(static)
    for (size_t p = 0; p < pairs; p++) {
        float a, b;
        gauss_pair(seed, p, &a, &b);
        out[2 * p] = or_bf16_bits(a * std);
        if (2 * p + 1 < count) out[2 * p + 1] = or_bf16_bits(b * std);
    }
}

/* Linear with the gemv epilogue (Shaders.swift:92-103; CPU loop KernelTests.swift:86-101). */
void or_linear(const float* x, int ldx, int m, const uint16_t* w, const uint16_t* w2,
               const uint16_t* bias, int n, int k, float* y, int ldy, uint32_t flags) {
    const int gated = (flags & MT_LINEAR_SILU_GATE) != 0;
#pragma omp parallel for schedule(static) if ((long)n * k * m > (1 << 18))
    for (int c = 0; c < n; c++) {
        const uint16_t* wr = w + (size_t)c * k;
        const uint16_t* w2r = gated ? w2 + (size_t)c * k : NULL;
        float* wf = (float*)malloc(sizeof(float) * (size_t)k * (gated ? 2 : 1));
        for (int i = 0; i < k; i++) wf[i] = bf(wr[i]);
        if (gated)
            for (int i = 0; i < k; i++) wf[k + i] = bf(w2r[i]);
        const float bval = (flags & MT_LINEAR_BIAS) ? bf(bias[c]) : 0.0f;
        for (int r = 0; r < m; r++) {
            const float* xr = x + (size_t)r * ldx;
            double acc = 0.0, acc2 = 0.0;
            for (int i = 0; i < k; i++) acc += (double)xr[i] * (double)wf[i];
            if (gated)
                for (int i = 0; i < k; i++) acc2 += (double)xr[i] * (double)wf[k + i];
            float v = (float)acc + bval;
            if (gated) v = or_silu(v) * (float)acc2;
            if (flags & MT_LINEAR_GELU) v = or_gelu_tanh(v);
            if (flags & MT_LINEAR_SILU) v = or_silu(v);
            float* yp = y + (size_t)r * ldy + c;
            if (flags & MT_LINEAR_ACCUM) v += *yp;
            *yp = v;
        }
        free(wf);
    }
}

/* Shaders.swift:418-441; KernelTests.swift:195-201. */
void or_rmsnorm(const float* x, int ldx, int rows, int width, const uint16_t* w, float* y, int ldy,
                float eps) {
    for (int r = 0; r < rows; r++) {
        const float* xr = x + (size_t)r * ldx;
        double ss = 0.0;
        for (int i = 0; i < width; i++) ss += (double)xr[i] * xr[i];
        const float scale = (float)(1.0 / sqrt(ss / width + (double)eps));
        float* yr = y + (size_t)r * ldy;
        for (int i = 0; i < width; i++) yr[i] = xr[i] * scale * bf(w[i]);
    }
}

/* Shaders.swift:456-486 (NeoX pairs i, i+32; KernelTests.swift:207-216). */
void or_rope_cache(float* qkv, int ldq, int m, int hq, int hkv, int pos0, float* kc, float* vc,
                   int cap, const float* inv_freq) {
    for (int r = 0; r < m; r++) {
        const int pos = pos0 + r;
        float* row = qkv + (size_t)r * ldq;
        for (int slot = 0; slot < hq + 2 * hkv; slot++) {
            float* h = row + slot * 64;
            if (slot >= hq + hkv) {
                float* dst = vc + ((size_t)(slot - hq - hkv) * cap + pos) * 64;
                memcpy(dst, h, 64 * sizeof(float));
                continue;
            }
            float out[64];
            for (int i = 0; i < 32; i++) {
                const float angle = (float)pos * inv_freq[i];
                const double c = cos((double)angle), s = sin((double)angle);
                const double x0 = h[i], x1 = h[i + 32];
                out[i] = (float)(x0 * c - x1 * s);
                out[i + 32] = (float)(x1 * c + x0 * s);
            }
            if (slot < hq) {
                memcpy(h, out, sizeof(out));
            } else {
                float* dst = kc + ((size_t)(slot - hq) * cap + pos) * 64;
                memcpy(dst, out, sizeof(out));
            }
        }
    }
}

/* Shaders.swift:500-591 (causal GQA, window, scale 1/8; KernelTests.swift:246-266). */
void or_attention(const float* q, int ldq, int m, int hq, int hkv, int pos0, int window,
                  const float* kc, const float* vc, int cap, float* out, int ldo) {
    double* sc = (double*)malloc(sizeof(double) * (size_t)(pos0 + m + 1));
    for (int r = 0; r < m; r++) {
        const int qpos = pos0 + r, jEnd = qpos + 1;
        const int jStart = (window > 0 && jEnd > window) ? jEnd - window : 0;
        for (int h = 0; h < hq; h++) {
            const int kvh = h / (hq / hkv);
            const float* qh = q + (size_t)r * ldq + h * 64;
            double mx = -INFINITY;
            for (int j = jStart; j < jEnd; j++) {
                const float* kr = kc + ((size_t)kvh * cap + j) * 64;
                double s = 0.0;
                for (int d = 0; d < 64; d++) s += (double)qh[d] * kr[d];
                s *= 0.125;
                sc[j - jStart] = s;
                if (s > mx) mx = s;
            }
            double sum = 0.0;
            for (int j = jStart; j < jEnd; j++) {
                sc[j - jStart] = exp(sc[j - jStart] - mx);
                sum += sc[j - jStart];
            }
            float* o = out + (size_t)r * ldo + h * 64;
            for (int d = 0; d < 64; d++) {
                double acc = 0.0;
                for (int j = jStart; j < jEnd; j++) acc += sc[j - jStart] * vc[((size_t)kvh * cap + j) * 64 + d];
                o[d] = (float)(acc / sum);
            }
        }
    }
    free(sc);
}

/* Shaders.swift:605-648 (interleaved pairs 2l, 2l+1, angle = row * inv_freq[l];
 * KernelTests.swift:291-321). */
void or_dit_attention(const float* qkv, int ld, int batch, int seq, int heads,
                      const float* inv_freq, float* out, int ldo) {
    const int D = heads * 64;
    for (int b = 0; b < batch; b++)
        for (int h = 0; h < heads; h++) {
            double q[8][64], k[8][64];
            for (int i = 0; i < seq; i++) {
                const float* row = qkv + (size_t)(b * seq + i) * ld + h * 64;
                for (int l = 0; l < 32; l++) {
                    const float angle = (float)i * inv_freq[l];
                    const double c = cos((double)angle), s = sin((double)angle);
                    const double q0 = row[2 * l], q1 = row[2 * l + 1];
                    const double k0 = row[D + 2 * l], k1 = row[D + 2 * l + 1];
                    q[i][2 * l] = q0 * c - q1 * s;
                    q[i][2 * l + 1] = q1 * c + q0 * s;
                    k[i][2 * l] = k0 * c - k1 * s;
                    k[i][2 * l + 1] = k1 * c + k0 * s;
                }
            }
            for (int i = 0; i < seq; i++) {
                double sc[8], mx = -INFINITY, sum = 0.0;
                for (int j = 0; j < seq; j++) {
                    double s = 0.0;
                    for (int d = 0; d < 64; d++) s += q[i][d] * k[j][d];
                    sc[j] = s * 0.125;
                    if (sc[j] > mx) mx = sc[j];
                }
                for (int j = 0; j < seq; j++) {
                    sc[j] = exp(sc[j] - mx);
                    sum += sc[j];
                }
                float* o = out + (size_t)(b * seq + i) * ldo + h * 64;
                for (int d = 0; d < 64; d++) {
                    double acc = 0.0;
                    for (int j = 0; j < seq; j++) acc += sc[j] * qkv[(size_t)(b * seq + j) * ld + 2 * D + h * 64 + d];
                    o[d] = (float)(acc / sum);
                }
            }
        }
}

/* Shaders.swift:654-677. */
void or_flow_assemble(const float* y, const float* history, const float* cemb,
                      const uint16_t* cbias, const float* temb, const uint16_t* xw,
                      const uint16_t* xb, int hidden, int latent, float* x) {
    for (int r = 0; r < 6; r++) {
        const int s = r % 3;
        for (int c = 0; c < hidden; c++) {
            float v;
            if (s == 0) {
                v = temb[c] + (r < 3 ? cemb[c] : bf(cbias[c]));
            } else {
                const float* src = (s == 1) ? history : y;
                double acc = 0.0;
                for (int d = 0; d < latent; d++) acc += (double)bf(xw[(size_t)c * latent + d]) * src[d];
                v = bf(xb[c]) + (float)acc;
            }
            x[(size_t)r * hidden + c] = v;
        }
    }
}

/* Shaders.swift:682-693. */
void or_flow_euler(float* y, const float* pred, int ldp, int pred_row, int null_row, int latent,
                   float cfg, float dt, float* capture) {
    for (int d = 0; d < latent; d++) {
        const float c = pred[(size_t)pred_row * ldp + d];
        const float u = pred[(size_t)null_row * ldp + d];
        if (capture) {
            capture[d] = c;
            capture[latent + d] = u;
        }
        y[d] += (c + (c - u) * cfg) * dt;
    }
}

/* Shaders.swift:704-719; the torch Upsample(linear, x4, align_corners=False) weights
 * (KernelTests.swift:395-401). */
void or_upsample4(const float* prev, const float* cur, const float* next, int hidden, float* frames) {
    for (int r = 0; r < 4; r++)
        for (int c = 0; c < hidden; c++) {
            const float v0 = cur[c];
            float v;
            if (r == 0) v = prev ? 0.625f * v0 + 0.375f * prev[c] : v0;
            else if (r == 1) v = prev ? 0.875f * v0 + 0.125f * prev[c] : v0;
            else if (r == 2) v = next ? 0.875f * v0 + 0.125f * next[c] : v0;
            else v = next ? 0.625f * v0 + 0.375f * next[c] : v0;
            frames[(size_t)r * hidden + c] = v;
        }
}

/* Shaders.swift:726-764: mag = min(exp(logmag), 100), irfft with 1/N, times the window;
 * computed in double as KernelTests.swift:357-372. */
void or_istft_frames(const float* spec, int ld_spec, int count, int nfft, const float* window,
                     float* frames, int frame0, int ring) {
    const int N = nfft, bins = N / 2 + 1;
    double* ct = (double*)malloc(sizeof(double) * N);
    double* st = (double*)malloc(sizeof(double) * N);
    for (int j = 0; j < N; j++) {
        ct[j] = cos(2.0 * M_PI * j / N);
        st[j] = sin(2.0 * M_PI * j / N);
    }
    double* re = (double*)malloc(sizeof(double) * bins);
    double* im = (double*)malloc(sizeof(double) * bins);
    for (int f = 0; f < count; f++) {
        const float* row = spec + (size_t)f * ld_spec;
        for (int k = 0; k < bins; k++) {
            double mag = exp((double)row[k]);
            if (mag > 100.0) mag = 100.0;
            const double ph = row[bins + k];
            re[k] = mag * cos(ph);
            im[k] = mag * sin(ph);
        }
        const int slot = (frame0 + f) % ring;
#pragma omp parallel for schedule(static)
        for (int t = 0; t < N; t++) {
            double acc = re[0] + ((t & 1) ? -re[N / 2] : re[N / 2]);
            double sum = 0.0;
            long idx = 0;
            for (int k = 1; k < N / 2; k++) {
                idx += t;
                if (idx >= N) idx -= N;
                sum += re[k] * ct[idx] - im[k] * st[idx];
            }
            acc += 2.0 * sum;
            frames[(size_t)slot * N + t] = (float)(acc / N * (double)window[t]);
        }
    }
    free(ct);
    free(st);
    free(re);
    free(im);
}

/* Shaders.swift:770-788. */
void or_istft_emit(const float* frames, const float* window, int nfft, int hop, int s0, int count,
                   int last_frame, int ring, float* out) {
    const int pad = (nfft - hop) / 2;
    for (int i = 0; i < count; i++) {
        const int s = s0 + i + pad;
        int fHi = s / hop;
        if (fHi > last_frame) fHi = last_frame;
        const int fLo = (s >= nfft) ? (s - nfft) / hop + 1 : 0;
        double acc = 0.0, env = 0.0;
        for (int f = fLo; f <= fHi; f++) {
            const int t = s - f * hop;
            if (t < 0 || t >= nfft) continue;
            const double w = window[t];
            acc += frames[(size_t)(f % ring) * nfft + t];
            env += w * w;
        }
        out[i] = (float)(acc / env);
    }
}

/* DiT.swift:56-65, evaluated in fp32 as the Swift Float code does. */
void or_flow_timesteps(int steps, float* out) {
    static const int e5[] = {0, 2, 4, 8, 16, 32}, e6[] = {0, 2, 4, 6, 8, 16, 32},
                     e7[] = {0, 2, 4, 6, 8, 16, 24, 32},
                     e10[] = {0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32},
                     e12[] = {0, 2, 4, 6, 8, 10, 12, 14, 16, 20, 24, 28, 32},
                     e16[] = {0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 12, 14, 16, 20, 24, 28, 32};
    const int* tab = steps == 5 ? e5 : steps == 6 ? e6 : steps == 7 ? e7 : steps == 10 ? e10
                   : steps == 12 ? e12 : steps == 16 ? e16 : NULL;
    const float half_pi = 3.14159274101257324f / 2.0f;
    for (int i = 0; i <= steps; i++) {
        const float t = tab ? (float)tab[i] / 32.0f : (float)i / (float)steps;
        out[i] = t - (cosf(half_pi * t) - 1.0f + t);
    }
}

/* DiT.swift:68-79. */
void or_sinusoid(float t, float* out256) {
    const int half = 128;
    const float step = (float)(log(10000.0) / (double)(half - 1));
    for (int i = 0; i < half; i++) {
        const float freq = expf((float)i * -step);
        const float arg = (1000.0f * t) * freq;
        out256[i] = (float)sin((double)arg);
        out256[half + i] = (float)cos((double)arg);
    }
}
