// stack.cu -- persistent small-batch transformer stack: one launch runs every layer of a Qwen
// decode pass (or every block of a DiT pass) for at most 8 activation rows.
//
// Reference: QwenForward.dispatches (Sources/MingTTS/Engine/Qwen.swift:72-97) and DiTForward.encode
// (Sources/MingTTS/Engine/DiT.swift:35-48); the kernels they dispatch are restated here as phases:
// RMSNorm (Shaders.swift:418-441) folded into the linear that consumes it, the linear with its
// epilogue (Shaders.swift:47-108: +bias -> SiLU gate -> GELU-tanh -> +=), NeoX RoPE + KV append +
// causal/windowed GQA attention (Shaders.swift:456-591), interleaved-RoPE DiT attention
// (Shaders.swift:613-648), and the final norm.
//
// Why: with a few rows every linear is a weight stream (a few MB) and the stack is a chain of
// ~170 dependent launches whose fixed costs (launch, ramp-up, drain) exceed the streaming time.
// Here one cooperative launch holds one CTA per SM for the whole pass:
//   * a producer warp copies this CTA's contiguous slice of every phase's weight rows into a
//     shared-memory ring with bulk copies (cp.async.bulk, all 32 lanes issuing pieces), running
//     ahead of the computation by as many phases as the ring holds -- weights never depend on
//     activations, so HBM keeps streaming across the phase boundaries;
//   * eight compute warps run the phases in order; phase q starts once every CTA has finished
//     phase q - 1 (a per-phase device counter, bounded acquire-waits), stages its input rows in
//     shared memory (normalising them when the phase folds an RMSNorm), multiplies them against the
//     weight slice and applies the epilogue to its own output columns.
// Activations written by other CTAs are read through L2 only (ld.global.cg): L1 is not coherent
// between SMs within one launch. Every wait is bounded by the status word's wait limit; one that
// gives up records DEV_TIMEOUT, raises the launch's abort flag, and the producer waits for its own
// copies in flight before the CTA exits.
#include <stdio.h>

#include "common.cuh"
#include "kernels.cuh"

namespace mt {

namespace {

constexpr int PS_CWARPS = 8;                    // compute warps (threads 0..255)
constexpr int PS_CT = PS_CWARPS * 32;
constexpr int PS_THREADS = PS_CT + 32;          // + the producer warp (warp 8)
constexpr int PS_SLOTS = 8;                     // weight slices in flight
constexpr uint32_t PS_RING = 160 * 1024;        // weight ring
constexpr uint32_t PS_ACT = 40 * 1024;          // staged input rows / attention scratch
constexpr uint32_t PS_RED = 8 * 1024;           // cross-warp partial sums
constexpr size_t PS_SMEM = PS_RING + PS_ACT + PS_RED + 128;
// Weight rows per register block: 4 (2 when gated or with 8 activation rows, whose x registers
// already take 64 of the 168 a thread has at one 288-thread block per SM).

constexpr int PS_XOWN = 16;                     // residual columns one CTA owns, at most
constexpr int PS_MAX_CHUNKS = 16;               // CTAs per attention unit, at most

enum PsType : int { PT_LIN = 0, PT_ATTN_QWEN = 1, PT_ATTN_DIT = 2, PT_FINAL = 3 };

struct PsLin {
    const uint16_t *w, *w2, *bias, *gain;
    int n, k;
    const float* in;
    int ld_in;
    float* out;
    int ld_out;
    uint32_t flags;
};

__device__ __forceinline__ int ps_phases(const StackParams& p) {
    return p.layers * 5 + (p.kind == STACK_QWEN && p.z ? 1 : 0);
}

__device__ __forceinline__ int ps_type(const StackParams& p, int q) {
    if (q >= p.layers * 5) return PT_FINAL;
    const int sub = q % 5;
    if (sub == 1) return p.kind == STACK_QWEN ? PT_ATTN_QWEN : PT_ATTN_DIT;
    return PT_LIN;
}

// The linear of phase q (sub 0, 2, 3 or 4 of its layer).
__device__ __forceinline__ PsLin ps_lin(const StackParams& p, int q) {
    const int l = q / 5, sub = q % 5;
    const uint16_t* const* W = p.L[l].p;
    const int H = p.hidden;
    PsLin r{};
    if (p.kind == STACK_QWEN) {
        const int qkvw = (p.heads + 2 * p.kv_heads) * 64, A = p.heads * 64;
        // norm1, qkv_w, qkv_b, o_w, norm2, gate_w, up_w, down_w
        if (sub == 0) r = PsLin{W[1], nullptr, W[2], W[0], qkvw, H, p.x, H, p.qkv, qkvw, MT_LINEAR_BIAS};
        else if (sub == 2) r = PsLin{W[3], nullptr, nullptr, nullptr, H, A, p.attn, A, p.x, H, MT_LINEAR_ACCUM};
        else if (sub == 3) r = PsLin{W[5], W[6], nullptr, W[4], p.inter, H, p.x, H, p.mlp, p.inter, MT_LINEAR_SILU_GATE};
        else r = PsLin{W[7], nullptr, nullptr, nullptr, H, p.inter, p.mlp, p.inter, p.x, H, MT_LINEAR_ACCUM};
    } else {
        // norm1, qkv_w, qkv_b, out_w, out_b, norm2, ff1_w, ff1_b, ff2_w, ff2_b
        if (sub == 0) r = PsLin{W[1], nullptr, W[2], W[0], 3 * H, H, p.x, H, p.qkv, 3 * H, MT_LINEAR_BIAS};
        else if (sub == 2) r = PsLin{W[3], nullptr, W[4], nullptr, H, H, p.attn, H, p.x, H, MT_LINEAR_BIAS | MT_LINEAR_ACCUM};
        else if (sub == 3) r = PsLin{W[6], nullptr, W[7], W[5], p.inter, H, p.x, H, p.mlp, p.inter, MT_LINEAR_BIAS | MT_LINEAR_GELU};
        else r = PsLin{W[8], nullptr, W[9], nullptr, H, p.inter, p.mlp, p.inter, p.x, H, MT_LINEAR_BIAS | MT_LINEAR_ACCUM};
    }
    return r;
}

__device__ __forceinline__ void ps_rows(int n, int cta, int ctas, int& n0, int& n1) {
    n0 = (int)(((long long)n * cta) / ctas);
    n1 = (int)(((long long)n * (cta + 1)) / ctas);
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void named_sync() { asm volatile("bar.sync 1, %0;" ::"n"(PS_CT) : "memory"); }

__device__ __forceinline__ float dot8(const float4& a, const float4& b, const uint4& w) {
    return a.x * bf16_lo(w.x) + a.y * bf16_hi(w.x) + a.z * bf16_lo(w.y) + a.w * bf16_hi(w.y) + b.x * bf16_lo(w.z) +
           b.y * bf16_hi(w.z) + b.z * bf16_lo(w.w) + b.w * bf16_hi(w.w);
}

// Shared state of the CTA.
struct PsShared {
    uint64_t bar[PS_SLOTS];
    uint32_t slot_off[PS_SLOTS];
    volatile unsigned long long free_pos;  // ring bytes released by the compute warps (monotonic)
    volatile int consumed;                 // linear phases fully consumed
    volatile int abort;
    float rscale[8];
    float rot_c[4][32], rot_s[4][32];
    float m_run[32], l_run[32];
    volatile int last;
    float xown[8][PS_XOWN];
};

// Attention chunks per unit: as many CTAs as the grid spares, at most PS_MAX_CHUNKS.
__device__ __host__ __forceinline__ int ps_chunks(int units, int ctas) {
    const int c = units > 0 ? ctas / units : 1;
    return c < 1 ? 1 : c > PS_MAX_CHUNKS ? PS_MAX_CHUNKS : c;
}

// Bounded wait for phase q of every CTA (compute thread 0), then broadcast. False on abort.
__device__ bool ps_wait_phase(const StackParams& p, PsShared& s, int q, int ctas) {
    if (threadIdx.x == 0) {
        const unsigned int* cnt = p.sync + q;
        const unsigned int* ab = p.sync + ps_phases(p);
        uint64_t t0 = 0, limit = 0;
        unsigned ns = 32;
        for (uint32_t it = 0;; it++) {
            if (ld_acquire(cnt) >= (unsigned)ctas) break;
            if (*reinterpret_cast<const volatile unsigned int*>(ab)) {
                s.abort = 1;
                break;
            }
            if ((it & 15u) == 15u) {
                const uint64_t now = global_ns();
                if (t0 == 0) {
                    t0 = now;
                    limit = wait_limit_ns(p.status);
                } else if (now - t0 > limit) {
                    report_status(p.status, DEV_TIMEOUT, 40, (unsigned)q);
                    atomicExch(const_cast<unsigned int*>(ab), 1u);
                    s.abort = 1;
                    break;
                }
            }
            __nanosleep(ns);
            if (ns < 256) ns <<= 1;
        }
        __threadfence();
    }
    named_sync();
    return !s.abort;
}

__device__ __forceinline__ void ps_signal(const StackParams& p, int q) {
    if (threadIdx.x == 0) {
        __threadfence();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.sync + q) : "memory");
    }
}

// Raises the abort flag of the launch (any thread).
__device__ __forceinline__ void ps_abort(const StackParams& p, PsShared& s, unsigned site, unsigned detail) {
    report_status(p.status, DEV_TIMEOUT, site, detail);
    atomicExch(p.sync + ps_phases(p), 1u);
    s.abort = 1;
}

// ---------------------------------------------------------------------------------------------
// Producer warp: walks the phases in order and copies this CTA's weight slice of every linear
// phase into the ring. Lane 0 allocates ring space (contiguous; the ring's tail is skipped when a
// slice does not fit before the end), waits for it to be released and arms the slot barrier; then
// all 32 lanes issue 16-byte-aligned pieces of the slice.
// ---------------------------------------------------------------------------------------------
__device__ __noinline__ void ps_producer(const StackParams& p, PsShared& s, uint8_t* ring, int cta, int ctas) {
    const int lane = threadIdx.x & 31;
    const int P = ps_phases(p);
    unsigned long long alloc = 0;
    int j = 0;
    int last_use[PS_SLOTS];
#pragma unroll
    for (int i = 0; i < PS_SLOTS; i++) last_use[i] = -1;
    for (int q = 0; q < P && !s.abort; q++) {
        if (ps_type(p, q) != PT_LIN) continue;
        const PsLin L = ps_lin(p, q);
        int n0, n1;
        ps_rows(L.n, cta, ctas, n0, n1);
        if (n1 <= n0) continue;
        const uint32_t one = (uint32_t)(n1 - n0) * (uint32_t)L.k * 2u;
        const uint32_t bytes = L.w2 ? 2 * one : one;
        const int slot = j % PS_SLOTS;
        uint32_t off = 0;
        int armed = 0;
        if (lane == 0) {
            // Live slices occupy [free_pos, live_end) of the monotonic cursor. A slice that would
            // straddle the ring's end starts at the next lap instead (the tail is left unused), and
            // may be placed once it does not overlap the live bytes: either nothing is live, or
            // the live bytes end before its image one lap back.
            const unsigned long long live_end = alloc;
            off = (uint32_t)(alloc % PS_RING);
            if (off + bytes > PS_RING) {
                alloc += PS_RING - off;
                off = 0;
            }
            uint64_t t0 = 0, limit = 0;
            for (uint32_t it = 0;; it++) {
                const unsigned long long fp = s.free_pos;
                if ((fp >= live_end || alloc + bytes - fp <= PS_RING) && j - s.consumed < PS_SLOTS) break;
                if (s.abort) break;
                if ((it & 63u) == 63u) {
                    const uint64_t now = global_ns();
                    if (t0 == 0) {
                        t0 = now;
                        limit = wait_limit_ns(p.status);
                    } else if (now - t0 > limit) {
                        ps_abort(p, s, 41, (unsigned)q);
                        break;
                    }
                }
                __nanosleep(64);
            }
            if (!s.abort) {
                s.slot_off[slot] = off;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect_tx(&s.bar[slot], bytes);
                armed = 1;
            }
        }
        // Lane 0's decision for the whole warp: once the barrier is armed every piece is issued.
        if (!__shfl_sync(0xffffffffu, armed, 0)) break;
        off = __shfl_sync(0xffffffffu, off, 0);
        // 32 pieces of each matrix's slice, 16-byte units.
        const uint32_t units = one / 16;
        const uint32_t u0 = units * lane / 32, u1 = units * (lane + 1) / 32;
        if (u1 > u0) {
            const uint8_t* src = reinterpret_cast<const uint8_t*>(L.w + (size_t)n0 * L.k);
            bulk_load(ring + off + u0 * 16, src + (size_t)u0 * 16, (u1 - u0) * 16, &s.bar[slot]);
            if (L.w2) {
                const uint8_t* src2 = reinterpret_cast<const uint8_t*>(L.w2 + (size_t)n0 * L.k);
                bulk_load(ring + off + one + u0 * 16, src2 + (size_t)u0 * 16, (u1 - u0) * 16, &s.bar[slot]);
            }
        }
        last_use[slot] = j;
        alloc += bytes;
        j++;
    }
    // Copies in flight land before the CTA may exit (normally the compute warps already waited).
    if (lane == 0) {
        int dummy = 0;
        volatile int* ab = &dummy;
        for (int sl = 0; sl < PS_SLOTS; sl++)
            if (last_use[sl] >= 0) mbar_wait(&s.bar[sl], (uint32_t)((last_use[sl] / PS_SLOTS) & 1), p.status, 42, ab);
    }
}

// ---------------------------------------------------------------------------------------------
// Linear phase (compute warps).
// ---------------------------------------------------------------------------------------------
template <int MR>
__device__ bool ps_linear(const StackParams& p, PsShared& s, const PsLin& L, const uint8_t* wslice, float* act,
                          float* red, int rows, int n0) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = p.M, K = L.k, nch = K >> 3;
    const bool gated = L.w2 != nullptr;
    const uint32_t one = (uint32_t)rows * K * 2u;
    // Input rows: staged in shared memory (normalised when the phase folds an RMSNorm) when they
    // fit, else read from L2 directly.
    const bool staged = (size_t)M * K * 4 <= PS_ACT;
    const float* xin = staged ? act : L.in;
    const int ldx = staged ? K : L.ld_in;
    if (staged) {
        // One pass of independent L2 loads into shared memory (eight in flight per thread).
        const int per = K >> 2, total = M * per;
        for (int e0 = tid; e0 < total; e0 += 8 * PS_CT) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int e = e0 + u * PS_CT;
                if (e < total) v[u] = ldcg4(L.in + (size_t)(e / per) * L.ld_in + 4 * (e % per));
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int e = e0 + u * PS_CT;
                if (e < total) *reinterpret_cast<float4*>(act + (size_t)(e / per) * K + 4 * (e % per)) = v[u];
            }
        }
        named_sync();
        if (L.gain) {
            // r[m] = rsqrt(mean(x[m]^2) + eps), one warp per row, then x * r * g in place.
            for (int m = warp; m < M; m += PS_CWARPS) {
                const float* xr = act + (size_t)m * K;
                float ss = 0.f;
                for (int c = lane; c < per; c += 32) {
                    const float4 v = *reinterpret_cast<const float4*>(xr + 4 * c);
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
                ss = warp_sum(ss);
                if (lane == 0) s.rscale[m] = rsqrtf(ss / (float)K + p.eps);
            }
            named_sync();
            for (int e = tid; e < total; e += PS_CT) {
                const int m = e / per, c = e % per;
                float4* ap = reinterpret_cast<float4*>(act + (size_t)m * K + 4 * c);
                float4 v = *ap;
                const float r = s.rscale[m];
                const uint2 g = *reinterpret_cast<const uint2*>(L.gain + 4 * c);
                v.x = v.x * r * bf16_lo(g.x);
                v.y = v.y * r * bf16_hi(g.x);
                v.z = v.z * r * bf16_lo(g.y);
                v.w = v.w * r * bf16_hi(g.y);
                *ap = v;
            }
            named_sync();
        }
    }
    // Warps: WK split the K chunks, WR = 8 / WK walk row blocks.
    const int WK = nch >= 512 ? 8 : nch >= 256 ? 4 : nch >= 128 ? 2 : 1;
    const int WR = PS_CWARPS / WK;
    const int wk = warp % WK, wr = warp / WK;
    const int c_lo = nch * wk / WK, c_hi = nch * (wk + 1) / WK;
    constexpr int RB = MR >= 8 ? 2 : 4;
    const int rbk = gated ? 2 : RB;
    const int blocks = (rows + rbk - 1) / rbk;
    const int nv = gated ? 2 : 1;
    for (int b = wr; b < blocks; b += WR) {
        const int r0 = b * rbk;
        float acc[RB][MR], acc2[2][MR];
#pragma unroll
        for (int r = 0; r < RB; r++)
#pragma unroll
            for (int m = 0; m < MR; m++) acc[r][m] = 0.f;
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
            for (int m = 0; m < MR; m++) acc2[r][m] = 0.f;
        for (int c = c_lo + lane; c < c_hi; c += 32) {
            float4 xa[MR], xb[MR];
#pragma unroll
            for (int m = 0; m < MR; m++) {
                if (m < M) {
                    const float* xp = xin + (size_t)m * ldx + 8 * c;
                    if (staged) {
                        xa[m] = *reinterpret_cast<const float4*>(xp);
                        xb[m] = *reinterpret_cast<const float4*>(xp + 4);
                    } else {
                        xa[m] = ldcg4(xp);
                        xb[m] = ldcg4(xp + 4);
                    }
                }
            }
            if (!gated) {
#pragma unroll
                for (int r = 0; r < RB; r++) {
                    if (r0 + r < rows) {
                        const uint4 wv = *reinterpret_cast<const uint4*>(wslice + ((size_t)(r0 + r) * K + 8 * c) * 2);
#pragma unroll
                        for (int m = 0; m < MR; m++)
                            if (m < M) acc[r][m] += dot8(xa[m], xb[m], wv);
                    }
                }
            } else {
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    if (r0 + r < rows) {
                        const size_t o = ((size_t)(r0 + r) * K + 8 * c) * 2;
                        const uint4 wv = *reinterpret_cast<const uint4*>(wslice + o);
                        const uint4 wv2 = *reinterpret_cast<const uint4*>(wslice + one + o);
#pragma unroll
                        for (int m = 0; m < MR; m++) {
                            if (m < M) {
                                acc[r][m] += dot8(xa[m], xb[m], wv);
                                acc2[r][m] += dot8(xa[m], xb[m], wv2);
                            }
                        }
                    }
                }
            }
        }
        // Warp sums, then the lane owning (row, m) stores its partial for the cross-warp sum.
#pragma unroll
        for (int r = 0; r < RB; r++) {
#pragma unroll
            for (int m = 0; m < MR; m++) {
                if (!gated || r < 2) {
                    float v = warp_sum(acc[r][m]);
                    float v2 = gated ? warp_sum(acc2[r < 2 ? r : 0][m]) : 0.f;
                    if (lane == r * MR + m && r0 + r < rows && m < M) {
                        red[((size_t)wk * rows + r0 + r) * MR + m] = v;
                        if (gated) red[((size_t)(WK + wk) * rows + r0 + r) * MR + m] = v2;
                    }
                }
            }
        }
    }
    (void)nv;
    named_sync();
    // Epilogue (reference order): + bias, SiLU gate, GELU, += y. Consecutive threads take
    // consecutive output columns of one row.
    for (int e = tid; e < rows * M; e += PS_CT) {
        const int m = e / rows, r = e % rows;
        float v = 0.f, v2 = 0.f;
        for (int w = 0; w < WK; w++) {
            v += red[((size_t)w * rows + r) * MR + m];
            if (gated) v2 += red[((size_t)(WK + w) * rows + r) * MR + m];
        }
        const int n = n0 + r;
        if (L.flags & MT_LINEAR_BIAS) v += bf16f(L.bias[n]);
        if (gated) v = silu(v) * v2;
        if (L.flags & MT_LINEAR_GELU) v = gelu_tanh(v);
        float* yp = L.out + (size_t)m * L.ld_out + n;
        const bool own = L.out == p.x;  // the residual: this CTA owns column n in every phase that writes it
        if (L.flags & MT_LINEAR_ACCUM) v += own ? s.xown[m][r] : __ldcg(yp);
        if (own) s.xown[m][r] = v;
        *yp = v;
    }
    return true;
}

// ---------------------------------------------------------------------------------------------
// Qwen decode attention of one (sequence, kv head) unit, split by keys over C CTAs: NeoX RoPE of the
// new rows' q heads and key, KV append at positions pos .. pos + S - 1 (slot = position % cap, by
// chunk 0), and causal / windowed softmax attention (scale 1/8) of chunk c's keys, kept as a partial
// (row maximum m, weight sum l, unnormalised output o) in attn_part. The CTA that finishes the
// unit's last chunk (a per-unit counter) merges the C partials, o = sum_c e^(m_c - M) o_c /
// sum_c e^(m_c - M) l_c with M = max_c m_c, into the attention rows. No CTA waits for another.
// ---------------------------------------------------------------------------------------------
constexpr int PS_PART = 68;  // floats per (chunk, query row) partial: m, l, pad, o[64]

__device__ __noinline__ void ps_attn_qwen(const StackParams& p, PsShared& s, int layer, int unit, int c, int C, float* act) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hkv = p.kv_heads, G = p.heads / hkv, S = p.seq_rows, nq = S * G;
    const int r = unit / hkv, h = unit % hkv;
    const int qkvw = (p.heads + 2 * hkv) * 64, A = p.heads * 64;
    const int base = p.pos[r];
    const int W = p.window;
    const int jS = W > 0 ? max(0, base + 1 - W) : 0;
    const int nk = base + S - jS;
    const int k0 = (int)((long long)nk * c / C), k1 = (int)((long long)nk * (c + 1) / C), nkc = k1 - k0;
    const size_t tensor = (size_t)hkv * p.cap * 64;
    float* kc = p.kv + (size_t)r * p.kv_stride + (size_t)(2 * layer) * tensor + (size_t)h * p.cap * 64;
    float* vc = kc + tensor;
    float* qs = act;                     // [nq][64]
    float* nw = qs + (size_t)nq * 64;    // [S][k | v][64]
    float* sc = nw + (size_t)S * 128;    // [nq][nkc]
    // Positions come from device memory: a key range that would not fit the scratch (or a causal
    // cache overrun) is recorded as a bad argument and the unit writes nothing.
    const int nk_fit = (int)((PS_ACT / 4 - (uint32_t)nq * 64 - (uint32_t)S * 128) / (uint32_t)nq);
    if (nkc > nk_fit || base < 0 || (W == 0 && base + S > p.cap)) {
        if (tid == 0) report_status(p.status, DEV_BAD_ARG, 44, (unsigned)base);
        return;
    }
    if (tid < S * 32) {
        const int i = tid >> 5, l = tid & 31;
        float sn, cs;
        sincosf((float)(base + i) * p.inv_freq[l], &sn, &cs);
        s.rot_c[i][l] = cs;
        s.rot_s[i][l] = sn;
    }
    named_sync();
    // New rows: (row i, slot g < G query head | G key | G + 1 value, pair l).
    for (int it = tid; it < S * (G + 2) * 32; it += PS_CT) {
        const int l = it & 31, slot = (it >> 5) % (G + 2), i = (it >> 5) / (G + 2);
        const float* row = p.qkv + (size_t)(r * S + i) * qkvw;
        const int col = slot < G ? (h * G + slot) * 64 : slot == G ? (p.heads + h) * 64 : (p.heads + hkv + h) * 64;
        float v0 = __ldcg(row + col + l), v1 = __ldcg(row + col + l + 32);
        if (slot <= G) {
            const float cs = s.rot_c[i][l], sn = s.rot_s[i][l];
            const float r0 = v0 * cs - v1 * sn, r1 = v1 * cs + v0 * sn;
            v0 = r0;
            v1 = r1;
        }
        if (slot < G) {
            qs[(i * G + slot) * 64 + l] = v0;
            qs[(i * G + slot) * 64 + l + 32] = v1;
        } else {
            if (c == 0) {
                float* dst = (slot == G ? kc : vc) + (size_t)((base + i) % p.cap) * 64;
                dst[l] = v0;
                dst[l + 32] = v1;
            }
            float* st = nw + (i * 2 + (slot - G)) * 64;
            st[l] = v0;
            st[l + 32] = v1;
        }
    }
    named_sync();
    // Scores of this chunk: item (key jj, row i) against the G heads of row i.
    for (int it = tid; it < nkc * S; it += PS_CT) {
        const int jj = it % nkc, i = it / nkc;
        const int j = jS + k0 + jj, pos = base + i;
        const bool valid = j <= pos && (W == 0 || j > pos - W);
        float sg[8];
#pragma unroll
        for (int g = 0; g < 8; g++) sg[g] = 0.f;
        if (valid) {
            const float* kr = j < base ? kc + (size_t)(j % p.cap) * 64 : nw + (size_t)(j - base) * 128;
#pragma unroll
            for (int half = 0; half < 2; half++) {
                float4 k4[8];  // half a key row in flight at once
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    const float* kp = kr + 32 * half + 4 * t;
                    k4[t] = j < base ? ldcg4(kp) : *reinterpret_cast<const float4*>(kp);
                }
#pragma unroll
                for (int t = 0; t < 8; t++) {
#pragma unroll
                    for (int g = 0; g < 8; g++) {
                        if (g < G) {
                            const float4 q4 = *reinterpret_cast<const float4*>(qs + (i * G + g) * 64 + 32 * half + 4 * t);
                            sg[g] += q4.x * k4[t].x + q4.y * k4[t].y + q4.z * k4[t].z + q4.w * k4[t].w;
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < 8; g++)
            if (g < G) sc[(size_t)(i * G + g) * nkc + jj] = valid ? sg[g] * 0.125f : -INFINITY;
    }
    named_sync();
    // Chunk softmax statistics per query row (warp per row): weights relative to the chunk maximum.
    for (int qi = warp; qi < nq; qi += PS_CWARPS) {
        float* srow = sc + (size_t)qi * nkc;
        float mx = -INFINITY;
        for (int jj = lane; jj < nkc; jj += 32) mx = fmaxf(mx, srow[jj]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int jj = lane; jj < nkc; jj += 32) {
            const float e = mx == -INFINITY ? 0.f : expf(srow[jj] - mx);
            srow[jj] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0) {
            s.m_run[qi] = mx;
            s.l_run[qi] = sum;
        }
    }
    named_sync();
    // Chunk P.V: thread (4 dims d4, row i, part) holds the G heads of row i; PP parts split the keys.
    const int d4 = tid & 15, grp = tid >> 4;
    const int PP = (PS_CT / 16) / S;
    const int pv_i = grp % S, pv_part = grp / S;
    const bool pv_live = pv_part < PP;
    float4 acc[8];
#pragma unroll
    for (int g = 0; g < 8; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (pv_live) {
        for (int jj0 = pv_part; jj0 < nkc; jj0 += 4 * PP) {
            float4 v4[4];  // four value rows in flight, then their products
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int jj = jj0 + u * PP, j = jS + k0 + jj;
                v4[u] = jj >= nkc ? make_float4(0.f, 0.f, 0.f, 0.f)
                      : j < base ? ldcg4(vc + (size_t)(j % p.cap) * 64 + 4 * d4)
                                 : *reinterpret_cast<const float4*>(nw + (size_t)(j - base) * 128 + 64 + 4 * d4);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int jj = jj0 + u * PP;
                if (jj >= nkc) break;
#pragma unroll
                for (int g = 0; g < 8; g++) {
                    if (g < G) {
                        const float pj = sc[(size_t)(pv_i * G + g) * nkc + jj];
                        acc[g].x += pj * v4[u].x;
                        acc[g].y += pj * v4[u].y;
                        acc[g].z += pj * v4[u].z;
                        acc[g].w += pj * v4[u].w;
                    }
                }
            }
        }
    }
    named_sync();  // scores are consumed: the part sums overlay the scratch
    float4* part4 = reinterpret_cast<float4*>(act);  // [PP][S][G][16]
    if (pv_live) {
#pragma unroll
        for (int g = 0; g < 8; g++)
            if (g < G) part4[((pv_part * S + pv_i) * G + g) * 16 + d4] = acc[g];
    }
    named_sync();
    float* part = p.attn_part + (size_t)unit * C * nq * PS_PART;  // [C][nq][PS_PART] of this unit
    for (int t = tid; t < nq * 16; t += PS_CT) {
        const int dd = t & 15, qi = t >> 4, i = qi / G, g = qi % G;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int pp = 0; pp < PP; pp++) {
            const float4 v = part4[((pp * S + i) * G + g) * 16 + dd];
            o.x += v.x; o.y += v.y; o.z += v.z; o.w += v.w;
        }
        if (C == 1) {  // the whole key range: normalise and write the attention row directly
            const float inv = 1.0f / s.l_run[qi];
            *reinterpret_cast<float4*>(p.attn + (size_t)(r * S + i) * A + (h * G + g) * 64 + dd * 4) =
                make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
        } else {
            float* rec = part + ((size_t)c * nq + qi) * PS_PART;
            *reinterpret_cast<float4*>(rec + 4 + dd * 4) = o;
            if (dd == 0) {
                rec[0] = s.m_run[qi];
                rec[1] = s.l_run[qi];
            }
        }
    }
    if (C == 1) return;
    // The unit's last chunk to finish merges the partials (threadfence-reduction pattern).
    named_sync();
    if (tid == 0) {
        __threadfence();
        unsigned int* cnt = p.sync + ps_phases(p) + 1 + layer * STACK_MAX_UNITS + unit;
        const unsigned int done = atomicAdd(cnt, 1u);
        s.last = done == (unsigned)(C - 1);
        if (s.last) __threadfence();
    }
    named_sync();
    if (!s.last) return;
    for (int t = tid; t < nq * 16; t += PS_CT) {
        const int dd = t & 15, qi = t >> 4, i = qi / G, g = qi % G;
        float mx = -INFINITY;
        for (int cc = 0; cc < C; cc++) mx = fmaxf(mx, __ldcg(part + ((size_t)cc * nq + qi) * PS_PART));
        float l = 0.f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int cc = 0; cc < C; cc++) {
            const float* rec = part + ((size_t)cc * nq + qi) * PS_PART;
            const float mc = __ldcg(rec);
            if (mc == -INFINITY) continue;  // a chunk without a valid key for this row
            const float sc_ = expf(mc - mx);
            const float4 v = ldcg4(rec + 4 + dd * 4);
            l += __ldcg(rec + 1) * sc_;
            o.x += v.x * sc_; o.y += v.y * sc_; o.z += v.z * sc_; o.w += v.w * sc_;
        }
        const float inv = 1.0f / l;
        *reinterpret_cast<float4*>(p.attn + (size_t)(r * S + i) * A + (h * G + g) * 64 + dd * 4) =
            make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    }
}

// DiT attention of one (sequence, head) unit by one warp: interleaved RoPE (pairs 2l, 2l + 1, angle
// = row * inv_freq[l]), full softmax attention over the sequence's rows, scale 1/8.
template <int S>
__device__ __noinline__ void ps_attn_dit_s(const StackParams& p, int unit) {
    const int lane = threadIdx.x & 31;
    const int heads = p.heads, D = heads * 64;
    const int h = unit % heads, b = unit / heads;
    const float freq = p.inv_freq[lane];
    const float* rows = p.qkv + (size_t)b * S * 3 * D + h * 64 + 2 * lane;
    float2 q[S], k[S], v[S];
#pragma unroll
    for (int j = 0; j < S; j++) {
        q[j] = __ldcg(reinterpret_cast<const float2*>(rows + (size_t)j * 3 * D));
            k[j] = __ldcg(reinterpret_cast<const float2*>(rows + (size_t)j * 3 * D + D));
            v[j] = __ldcg(reinterpret_cast<const float2*>(rows + (size_t)j * 3 * D + 2 * D));
            float sj, cj;
            sincosf((float)j * freq, &sj, &cj);
            q[j] = make_float2(q[j].x * cj - q[j].y * sj, q[j].y * cj + q[j].x * sj);
            k[j] = make_float2(k[j].x * cj - k[j].y * sj, k[j].y * cj + k[j].x * sj);
    }
#pragma unroll
    for (int i = 0; i < S; i++) {
        float sc[S];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < S; j++) {
            sc[j] = warp_sum(q[i].x * k[j].x + q[i].y * k[j].y) * 0.125f;
            mx = fmaxf(mx, sc[j]);
        }
        float sum = 0.f, a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int j = 0; j < S; j++) {
            const float e = expf(sc[j] - mx);
            sum += e;
            a0 += e * v[j].x;
            a1 += e * v[j].y;
        }
        *reinterpret_cast<float2*>(p.attn + (size_t)(b * S + i) * D + h * 64 + 2 * lane) = make_float2(a0 / sum, a1 / sum);
    }
}

// DiT attention unit with the sequence length (1..8) as a compile-time constant: the flow's 3 rows
// and the aggregator's 2 hold only their own q, k, v registers.
__device__ __forceinline__ void ps_attn_dit(const StackParams& p, int unit) {
    switch (p.seq_rows) {
        case 1: ps_attn_dit_s<1>(p, unit); break;
        case 2: ps_attn_dit_s<2>(p, unit); break;
        case 3: ps_attn_dit_s<3>(p, unit); break;
        case 4: ps_attn_dit_s<4>(p, unit); break;
        case 5: ps_attn_dit_s<5>(p, unit); break;
        case 6: ps_attn_dit_s<6>(p, unit); break;
        case 7: ps_attn_dit_s<7>(p, unit); break;
        default: ps_attn_dit_s<8>(p, unit); break;
    }
}

template <int MR>
__global__ void __launch_bounds__(PS_THREADS, 1) stack_kernel(const __grid_constant__ StackParams p) {
    extern __shared__ __align__(128) uint8_t ps_smem[];
    __shared__ PsShared s;
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ps_smem) + 127) & ~uintptr_t(127));
    float* act = reinterpret_cast<float*>(ring + PS_RING);
    float* red = reinterpret_cast<float*>(ring + PS_RING + PS_ACT);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int cta = blockIdx.x, ctas = gridDim.x;
    if (tid == 0) {
        for (int i = 0; i < PS_SLOTS; i++) mbar_init(&s.bar[i], 1);
        s.free_pos = 0;
        s.consumed = 0;
        s.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == PS_CWARPS) {
        ps_producer(p, s, ring, cta, ctas);
        return;
    }
    // This CTA's columns of the residual rows: every phase that adds into x writes the same columns
    // (its share of hidden), so their running values stay in shared memory.
    {
        int xn0, xn1;
        ps_rows(p.hidden, cta, ctas, xn0, xn1);
        const int w = xn1 - xn0;
        for (int e = tid; e < p.M * w; e += PS_CT) s.xown[e / w][e % w] = __ldcg(p.x + (size_t)(e / w) * p.hidden + xn0 + e % w);
        named_sync();
    }
    const int P = ps_phases(p);
    unsigned long long pos_track = 0;  // the ring cursor as the producer computes it
    int j = 0;
    volatile int* abort = &s.abort;
    for (int q = 0; q < P; q++) {
        if (q > 0 && !ps_wait_phase(p, s, q - 1, ctas)) return;
        const int type = ps_type(p, q);
        if (type == PT_LIN) {
            const PsLin L = ps_lin(p, q);
            int n0, n1;
            ps_rows(L.n, cta, ctas, n0, n1);
            if (n1 > n0) {
                const uint32_t one = (uint32_t)(n1 - n0) * (uint32_t)L.k * 2u;
                const uint32_t bytes = L.w2 ? 2 * one : one;
                if (pos_track % PS_RING + bytes > PS_RING) pos_track += PS_RING - pos_track % PS_RING;
                const int slot = j % PS_SLOTS;
                // Every compute thread waits; they agree on the outcome before anyone leaves, so no
                // thread is left at a named barrier that a departed thread would never reach.
                if (!mbar_wait(&s.bar[slot], (uint32_t)((j / PS_SLOTS) & 1), p.status, 43, abort)) ps_abort(p, s, 43, (unsigned)q);
                named_sync();
                if (s.abort) return;
                ps_linear<MR>(p, s, L, ring + s.slot_off[slot], act, red, n1 - n0, n0);
                pos_track += bytes;
                j++;
                named_sync();
                if (tid == 0) {
                    s.free_pos = pos_track;
                    s.consumed = j;
                }
            }
        } else if (type == PT_ATTN_QWEN) {
            // Units (sequence, kv head) split by keys over C CTAs each.
            const int U = p.seqs * p.kv_heads, C = ps_chunks(U, ctas);
            for (int b = cta; b < U * C; b += ctas) {
                ps_attn_qwen(p, s, q / 5, b / C, b % C, C, act);
                named_sync();
            }
        } else if (type == PT_ATTN_DIT) {
            for (int u = cta * PS_CWARPS + warp; u < p.seqs * p.heads; u += ctas * PS_CWARPS) ps_attn_dit(p, u);
        } else {  // final norm of every row (Qwen), one row per CTA
            for (int m = cta; m < p.M; m += ctas) {
                const float* xr = p.x + (size_t)m * p.hidden;
                float ss = 0.f;
                for (int c = tid; c < (p.hidden >> 2); c += PS_CT) {
                    const float4 v = ldcg4(xr + 4 * c);
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
                ss = warp_sum(ss);
                float* part = act;
                if ((tid & 31) == 0) part[warp] = ss;
                named_sync();
                float tot = 0.f;
                for (int w = 0; w < PS_CWARPS; w++) tot += part[w];
                const float r = rsqrtf(tot / (float)p.hidden + p.eps);
                for (int c = tid; c < (p.hidden >> 2); c += PS_CT) {
                    const float4 v = ldcg4(xr + 4 * c);
                    const uint2 g = *reinterpret_cast<const uint2*>(p.final_norm + 4 * c);
                    *reinterpret_cast<float4*>(p.z + (size_t)m * p.hidden + 4 * c) =
                        make_float4(v.x * r * bf16_lo(g.x), v.y * r * bf16_hi(g.x), v.z * r * bf16_lo(g.y),
                                    v.w * r * bf16_hi(g.y));
                }
                named_sync();
            }
        }
        named_sync();  // thread 0's release in ps_signal covers the CTA's writes (it follows the barrier)
        ps_signal(p, q);
    }
}

// Shared-memory opt-in of one instantiation and its blocks per SM (0: the launch cannot be made).
char g_resident_why[256];

template <int MR>
int set_stack_attr() {
    const cudaError_t e1 = cudaFuncSetAttribute(stack_kernel<MR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PS_SMEM);
    int blocks = 0;
    const cudaError_t e2 = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, stack_kernel<MR>, PS_THREADS, PS_SMEM);
    if (e2 != cudaSuccess) blocks = 0;
    if (blocks < 1) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, stack_kernel<MR>);
        snprintf(g_resident_why, sizeof(g_resident_why),
                 "MR %d: set attr %s, occupancy %s, regs %d, static smem %zu, max dyn smem %d, max threads %d, dyn %zu",
                 MR, cudaGetErrorString(e1), cudaGetErrorString(e2), fa.numRegs, fa.sharedSizeBytes,
                 fa.maxDynamicSharedSizeBytes, fa.maxThreadsPerBlock, PS_SMEM);
    }
    cudaGetLastError();
    return blocks;
}

// Per device: every instantiation fits one block per SM (set once, on the first query).
int g_resident[kMaxDevices];
PerDeviceOnce g_attr_once;

bool stack_resident() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    g_attr_once([dev] {
        const int b = min(min(set_stack_attr<1>(), set_stack_attr<2>()), min(set_stack_attr<4>(), set_stack_attr<8>()));
        g_resident[dev] = b;
    });
    return g_resident[dev] >= 1;
}

}  // namespace

const char* stack_resident_why() { return g_resident_why; }

int stack_resident_blocks() {
    int dev = 0;
    if (!stack_resident() && (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)) return 0;
    return g_resident[dev];
}

// Whether a pass fits the persistent kernel: rows, weight slices against the ring, attention
// scratch, cross-warp partial sums.
bool stack_supported(const StackParams& p, int ctas) {
    if (p.M < 1 || p.M > 8 || p.layers < 1 || p.layers > STACK_MAX_LAYERS || ctas < 1) return false;
    if (!stack_resident()) return false;
    if (p.hidden % 8 || p.inter % 8 || (size_t)p.M * p.hidden * 4 > PS_ACT) return false;
    if ((p.hidden + ctas - 1) / ctas > PS_XOWN) return false;
    if (p.kind == STACK_QWEN) {
        const int hkv = p.kv_heads;
        if (hkv < 1 || p.heads % hkv || p.heads / hkv > 8 || p.seq_rows < 1 || p.seq_rows > 4) return false;
        if ((p.heads * 64) % 8 || (size_t)p.M * p.heads * 64 * 4 > PS_ACT) return false;
        const int G = p.heads / hkv, nq = p.seq_rows * G;
        const int U = p.seqs * hkv;
        if (U > STACK_MAX_UNITS || !p.attn_part) return false;
        const int nk = p.window > 0 ? p.window + p.seq_rows - 1 : p.cap;
        const int C = ps_chunks(U, ctas), nkc = (nk + C - 1) / C + 1;
        const size_t att = (size_t)nq * 64 * 4 + (size_t)p.seq_rows * 128 * 4 + (size_t)nq * nkc * 4;
        if (att > PS_ACT || (size_t)16 * 8 * 64 * 4 > PS_ACT) return false;
        if (p.window > 0 && p.window + p.seq_rows - 1 > p.cap) return false;
    } else {
        if (p.seq_rows < 1 || p.seq_rows > 8 || p.hidden != p.heads * 64) return false;
    }
    // Largest weight slice and partial-sum block of any linear.
    const int qkvw = p.kind == STACK_QWEN ? (p.heads + 2 * p.kv_heads) * 64 : 3 * p.hidden;
    const int ns[4] = {qkvw, p.hidden, p.inter, p.hidden};
    const int ks[4] = {p.hidden, p.kind == STACK_QWEN ? p.heads * 64 : p.hidden, p.hidden, p.inter};
    const bool gate[4] = {false, false, p.kind == STACK_QWEN, false};
    for (int i = 0; i < 4; i++) {
        const int rows = (ns[i] + ctas - 1) / ctas;
        const size_t bytes = (size_t)rows * ks[i] * 2 * (gate[i] ? 2 : 1);
        if (bytes > PS_RING) return false;
        const int nch = ks[i] / 8;
        const int WK = nch >= 512 ? 8 : nch >= 256 ? 4 : nch >= 128 ? 2 : 1;
        if ((size_t)rows * WK * 8 * (gate[i] ? 2 : 1) * 4 > PS_RED) return false;
    }
    return true;
}

// Phases of a pass (the sync words needed are this + 1).
int stack_phases(const StackParams& p) { return p.layers * 5 + (p.kind == STACK_QWEN && p.z ? 1 : 0); }

int stack_sync_words(const StackParams& p) { return stack_phases(p) + 1 + p.layers * STACK_MAX_UNITS; }

size_t stack_part_floats(int ctas) { return (size_t)ctas * 32 * PS_PART; }

void launch_stack(const StackParams& p, int ctas, cudaStream_t s) {
    cudaMemsetAsync(p.sync, 0, sizeof(unsigned int) * (size_t)stack_sync_words(p), s);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(PS_THREADS);
    cfg.dynamicSmemBytes = PS_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (they wait on each other)
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.M <= 1) cudaLaunchKernelEx(&cfg, stack_kernel<1>, p);
    else if (p.M <= 2) cudaLaunchKernelEx(&cfg, stack_kernel<2>, p);
    else if (p.M <= 4) cudaLaunchKernelEx(&cfg, stack_kernel<4>, p);
    else cudaLaunchKernelEx(&cfg, stack_kernel<8>, p);
}

}  // namespace mt
