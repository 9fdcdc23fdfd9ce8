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
// Why: with a few rows every linear is a weight stream of a few MB, and the stack is a chain of
// ~120 dependent steps whose fixed costs (launch, ramp-up, drain) exceed the streaming time. Here
// one cooperative launch holds one CTA per SM for the whole pass:
//   * this CTA's slice of every phase's weight rows streams into a shared-memory ring with bulk
//     copies (cp.async.bulk), in pieces of at most half the ring, as far ahead of the computation
//     as the ring holds -- weights never depend on activations, so HBM keeps streaming across the
//     phase boundaries. Warp 0 issues the copies at the start and whenever a consumed piece frees
//     ring space (the only moments space appears), so no warp waits on the ring and all eight
//     warps compute with the full register file;
//   * the eight warps run the phases in order. Every activation a phase writes for other CTAs
//     goes to a mailbox as 8-byte words {fp32 value, tag}, one store each, where the tag names the
//     launch (an epoch counter kept in device memory) and the phase. A consumer polls the words it
//     needs until every tag matches: the data is its own completion flag, so there is no grid
//     barrier, no fence and no second round trip between phases. A word is rewritten only after
//     every reader of its previous value has finished (each phase's inputs depend on all CTAs'
//     previous outputs), so a tag never goes stale under a reader.
//   * each CTA keeps its own columns of the residual rows in shared memory; the caller's x is read
//     at the start and written once at the end.
// Qwen attention: one (sequence, kv head) unit is split by keys over up to `chunks` CTAs; each
// prefetches its cached keys and values (cp.async) before polling the new q/k/v rows, and writes an
// online-softmax partial (max, sum, unnormalised output). The out-projection phase merges the
// partials while staging its input.
// Every wait is bounded by the status word's wait limit; one that gives up records DEV_TIMEOUT and
// raises the launch's abort flag, which every other wait watches; warp 0 waits for the CTA's
// copies in flight before it exits.
#include <stdio.h>

#include "common.cuh"
#include "kernels.cuh"

namespace mt {

namespace {

typedef unsigned long long u64;

constexpr int PS_CWARPS = 8;                    // warps (two per SM sub-partition: up to 255 registers each)
constexpr int PS_CT = PS_CWARPS * 32;
constexpr int PS_THREADS = PS_CT;
constexpr int PS_SLOTS = 12;                    // weight pieces in flight
// Dynamic shared memory: the weight ring, the staged input rows (and attention scratch), the
// cross-warp partial sums. A ring piece is whole weight rows, at most half the ring. A Qwen pass's
// ring holds a whole gate/up slice (33 row pairs of 896 at 148 CTAs); a DiT pass stages up to 96 KB
// of input (6 rows of its 4096-wide MLP).
struct PsLayout {
    uint32_t ring, piece, act;
};
__device__ __host__ __forceinline__ PsLayout ps_layout(int kind) {
    return kind == STACK_QWEN ? PsLayout{132 * 1024, 66 * 1024, 80 * 1024} : PsLayout{116 * 1024, 58 * 1024, 96 * 1024};
}
constexpr uint32_t PS_RED = 4 * 1024;           // cross-warp partial sums
constexpr size_t PS_SMEM = 216 * 1024 + 128;    // ring + act + PS_RED (both kinds) + alignment
constexpr int PS_XOWN = 16;                     // residual columns one CTA owns, at most
constexpr int PS_BIAS = 64;                     // bias rows of one CTA's slice, at most
constexpr int PS_CH = 64;                       // keys of one attention chunk, at most
constexpr int PS_REC = 66;                      // words of one attention partial: max, sum, o[64]
constexpr int PS_KROW = 68;                     // floats per staged key / value row (padded)
constexpr int PS_MAXC = 8;                      // attention chunks per unit, at most

enum PsType : int { PT_LIN = 0, PT_ATTN_QWEN = 1, PT_ATTN_DIT = 2, PT_FINAL = 3 };
enum PsIn : int { IN_PLAIN = 0, IN_X = 1, IN_MERGE = 2, IN_ATT = 3, IN_MLP = 4 };
enum PsOut : int { OUT_QKV = 0, OUT_X = 1, OUT_MLP = 2 };

struct PsLin {
    const uint16_t *w, *w2, *bias, *gain;
    int n, k;
    int in, in_phase;  // input kind and the phase that wrote it
    int out;
    uint32_t flags;
};

__device__ __forceinline__ int ps_phases(const StackParams& p) {
    return p.layers * 5 + (p.kind == STACK_QWEN && p.z ? 1 : 0);
}

__device__ __forceinline__ int ps_type(const StackParams& p, int q) {
    if (q >= p.layers * 5) return PT_FINAL;
    if (q % 5 == 1) return p.kind == STACK_QWEN ? PT_ATTN_QWEN : PT_ATTN_DIT;
    return PT_LIN;
}

// Tag of the words phase q writes in launch `epoch` (never 0: the mailbox starts zeroed).
__device__ __forceinline__ uint32_t ps_tag(uint32_t epoch, int q) { return (epoch << 8) + (uint32_t)q + 1u; }

// The linear of phase q (sub 0, 2, 3 or 4 of its layer).
__device__ __forceinline__ PsLin ps_lin(const StackParams& p, const StackLayer* layers, int q) {
    const int l = q / 5, sub = q % 5;
    const uint16_t* const* W = layers[l].p;
    const int H = p.hidden;
    const int x_in = l == 0 ? IN_PLAIN : IN_X, x_phase = 5 * l - 1;
    PsLin r{};
    if (p.kind == STACK_QWEN) {
        const int qkvw = (p.heads + 2 * p.kv_heads) * 64, A = p.heads * 64;
        // norm1, qkv_w, qkv_b, o_w, norm2, gate_w, up_w, down_w
        if (sub == 0) r = PsLin{W[1], nullptr, W[2], W[0], qkvw, H, x_in, x_phase, OUT_QKV, MT_LINEAR_BIAS};
        else if (sub == 2) r = PsLin{W[3], nullptr, nullptr, nullptr, H, A, IN_MERGE, q - 1, OUT_X, MT_LINEAR_ACCUM};
        else if (sub == 3) r = PsLin{W[5], W[6], nullptr, W[4], p.inter, H, IN_X, q - 1, OUT_MLP, MT_LINEAR_SILU_GATE};
        else r = PsLin{W[7], nullptr, nullptr, nullptr, H, p.inter, IN_MLP, q - 1, OUT_X, MT_LINEAR_ACCUM};
    } else {
        // norm1, qkv_w, qkv_b, out_w, out_b, norm2, ff1_w, ff1_b, ff2_w, ff2_b
        if (sub == 0) r = PsLin{W[1], nullptr, W[2], W[0], 3 * H, H, x_in, x_phase, OUT_QKV, MT_LINEAR_BIAS};
        else if (sub == 2) r = PsLin{W[3], nullptr, W[4], nullptr, H, H, IN_ATT, q - 1, OUT_X, MT_LINEAR_BIAS | MT_LINEAR_ACCUM};
        else if (sub == 3) r = PsLin{W[6], nullptr, W[7], W[5], p.inter, H, IN_X, q - 1, OUT_MLP, MT_LINEAR_BIAS | MT_LINEAR_GELU};
        else r = PsLin{W[8], nullptr, W[9], nullptr, H, p.inter, IN_MLP, q - 1, OUT_X, MT_LINEAR_BIAS | MT_LINEAR_ACCUM};
    }
    return r;
}

__device__ __host__ __forceinline__ void ps_rows(int n, int cta, int ctas, int& n0, int& n1) {
    n0 = (int)(((long long)n * cta) / ctas);
    n1 = (int)(((long long)n * (cta + 1)) / ctas);
}

// Weight rows per ring piece of a linear (its gate and up rows together when gated).
__device__ __host__ __forceinline__ int ps_piece_rows(uint32_t piece, int k, bool gated) {
    const uint32_t row = (uint32_t)k * 2u * (gated ? 2u : 1u);
    const int r = (int)(piece / row);
    return r < 1 ? 1 : r;
}

// ---- mailbox words -------------------------------------------------------------------------------
__device__ __forceinline__ void st_tag(u64* p, float v, uint32_t tag) {
    const u64 w = ((u64)tag << 32) | (u64)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void st_tag2(u64* p, float v0, float v1, uint32_t tag) {
    const u64 a = ((u64)tag << 32) | (u64)__float_as_uint(v0), b = ((u64)tag << 32) | (u64)__float_as_uint(v1);
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_tag2(const u64* p, u64& a, u64& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ u64 ld_tag(const u64* p) {
    u64 a;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
    return a;
}
__device__ __forceinline__ float tag_val(u64 w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ bool tag_ok(u64 w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }

__device__ __forceinline__ void named_sync() { asm volatile("bar.sync 1, %0;" ::"n"(PS_CT) : "memory"); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ float dot8(const float4& a, const float4& b, const uint4& w) {
    return a.x * bf16_lo(w.x) + a.y * bf16_hi(w.x) + a.z * bf16_lo(w.y) + a.w * bf16_hi(w.y) + b.x * bf16_lo(w.z) +
           b.y * bf16_hi(w.z) + b.z * bf16_lo(w.w) + b.w * bf16_hi(w.w);
}

// Shared state of the CTA.
struct PsShared {
    uint64_t bar[PS_SLOTS];
    uint32_t slot_off[PS_SLOTS];
    unsigned long long slot_end[PS_SLOTS];  // ring cursor after each piece (what consuming it frees)
    unsigned long long free_pos;            // ring bytes released by consumed pieces (monotonic)
    int consumed;                           // pieces fully consumed
    // weight stream (warp 0): next phase and row to copy, pieces issued, ring cursor
    int prod_q, prod_r0, prod_j;
    unsigned long long prod_alloc;
    volatile int abort;
    uint32_t epoch;
    float ssw[PS_CWARPS][8];                // per-warp sums of squares of the staged rows
    float m_run[32], l_run[32];
    float bias[PS_BIAS];
    float xown[8][PS_XOWN];
    StackLayer layer[STACK_MAX_LAYERS];     // the pass's weight pointers (read once from the parameters)
};

__device__ __forceinline__ bool ps_global_abort(const StackParams& p) {
    return *reinterpret_cast<const volatile unsigned int*>(p.sync + 2) != 0u;
}

// Raises the abort flag of the launch after a wait gave up (any thread).
__device__ __forceinline__ void ps_timeout(const StackParams& p, PsShared& s, unsigned site, unsigned detail) {
    report_status(p.status, DEV_TIMEOUT, site, detail);
    atomicExch(p.sync + 2, 1u);
    s.abort = 1;
}

// Bookkeeping of one polling loop (a batch of mailbox loads retried until every tag matches):
// every 16 rounds it checks the launch's abort flag and the wait limit. False: give up (a timeout
// raises the abort flag). One copy per polling site keeps the kernel's code small.
__device__ __forceinline__ bool ps_keep_waiting(const StackParams& p, PsShared& s, uint64_t& t0, uint32_t& it,
                                                unsigned site) {
    if ((++it & 15u) != 0u) return true;
    if (s.abort || ps_global_abort(p)) {
        s.abort = 1;
        return false;
    }
    const uint64_t now = global_ns();
    if (t0 == 0) {
        t0 = now;
        return true;
    }
    if (now - t0 > wait_limit_ns(p.status)) {
        ps_timeout(p, s, site, it);
        return false;
    }
    return true;
}

// Qwen attention: chunks of unit row r's keys (1 for an invalid position, which is reported).
__device__ __forceinline__ int ps_unit_keys(const StackParams& p, int r, int& base, int& jS) {
    base = p.pos[r];
    const int W = p.window, S = p.seq_rows;
    jS = W > 0 ? max(0, base + 1 - W) : 0;
    if (base < 0 || (W == 0 && base + S > p.cap)) return -1;
    return base + S - jS;
}
__device__ __forceinline__ int ps_unit_chunks(int nk, int chunks) {
    if (nk <= 0) return 1;
    const int c = (nk + PS_CH - 1) / PS_CH;
    return c > chunks ? chunks : c;
}

// ---------------------------------------------------------------------------------------------
// Weight stream (warp 0): walks the phases in order and copies this CTA's weight slice of every
// linear phase into the ring, one piece (whole rows, gate and up rows together when gated) per
// slot, while the ring and the slots have room. Lane 0 places the piece (contiguous; the ring's
// tail is skipped when a piece does not fit before the end) and arms the slot barrier; then all 32
// lanes issue 16-byte-aligned parts of the piece.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void ps_refill(const StackParams& p, PsShared& s, uint8_t* ring, int cta, int ctas) {
    const int lane = threadIdx.x & 31;
    const int P = ps_phases(p);
    for (;;) {
        int q = s.prod_q, r0 = s.prod_r0;
        PsLin L{};
        int n0 = 0, n1 = 0;
        bool found = false;
        for (; q < P; q++, r0 = -1) {
            if (ps_type(p, q) != PT_LIN) continue;
            L = ps_lin(p, s.layer, q);
            ps_rows(L.n, cta, ctas, n0, n1);
            if (r0 < n0) r0 = n0;
            if (r0 < n1) {
                found = true;
                break;
            }
        }
        __syncwarp();
        if (!found) {
            if (lane == 0) s.prod_q = P;
            __syncwarp();
            return;
        }
        const PsLayout lay = ps_layout(p.kind);
        const bool gated = L.w2 != nullptr;
        const int rows = min(ps_piece_rows(lay.piece, L.k, gated), n1 - r0);
        const uint32_t one = (uint32_t)rows * (uint32_t)L.k * 2u;
        const uint32_t bytes = gated ? 2 * one : one;
        unsigned long long alloc = s.prod_alloc;
        uint32_t off = (uint32_t)(alloc % lay.ring);
        if (off + bytes > lay.ring) {  // the tail counts as allocated
            alloc += lay.ring - off;
            off = 0;
        }
        const int j = s.prod_j;
        if (alloc + bytes - s.free_pos > lay.ring || j - s.consumed >= PS_SLOTS) {
            if (lane == 0) {
                s.prod_q = q;
                s.prod_r0 = r0;
            }
            __syncwarp();
            return;
        }
        const int slot = j % PS_SLOTS;
        if (lane == 0) {
            s.slot_off[slot] = off;
            s.slot_end[slot] = alloc + bytes;
            mbar_expect_tx(&s.bar[slot], bytes);
        }
        __syncwarp();
        // The ring bytes were last read by generic loads (ordered before this by the barrier that
        // released them); order those before the async-proxy writes.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const uint32_t units = one / 16;
        const uint32_t u0 = units * lane / 32, u1 = units * (lane + 1) / 32;
        if (u1 > u0) {
            const uint8_t* src = reinterpret_cast<const uint8_t*>(L.w + (size_t)r0 * L.k);
            bulk_load(ring + off + u0 * 16, src + (size_t)u0 * 16, (u1 - u0) * 16, &s.bar[slot]);
            if (gated) {
                const uint8_t* src2 = reinterpret_cast<const uint8_t*>(L.w2 + (size_t)r0 * L.k);
                bulk_load(ring + off + one + u0 * 16, src2 + (size_t)u0 * 16, (u1 - u0) * 16, &s.bar[slot]);
            }
        }
        __syncwarp();
        if (lane == 0) {
            s.prod_q = q;
            s.prod_r0 = r0 + rows;
            s.prod_j = j + 1;
            s.prod_alloc = alloc + bytes;
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------------------------
// Input staging of a linear phase (compute warps): M rows of K values into act[M][K], multiplied by
// the RMSNorm gain when the phase folds one (the per-row scale is applied in the epilogue), with
// per-warp sums of squares of the raw values in s.ssw.
// ---------------------------------------------------------------------------------------------
template <int MR>
__device__ bool ps_stage_rows(const StackParams& p, PsShared& s, const u64* src, const float* plain, int ld, int M, int K,
                              uint32_t tag, const uint16_t* gain, float* act) {
    constexpr int NB = 8;  // value pairs in flight per thread
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int per = K >> 1;  // value pairs per row
    const int total = M * per;
    float ss[MR];
#pragma unroll
    for (int m = 0; m < MR; m++) ss[m] = 0.f;
    bool ok = true;
    if (plain) {  // the pass's input rows (the caller's fp32 layout)
        for (int e = tid; e < total; e += PS_CT) {
            const int m = e / per, c = e - m * per;
            const float2 v = __ldcg(reinterpret_cast<const float2*>(plain + (size_t)m * ld + 2 * c));
            const uint32_t g = gain ? __ldg(reinterpret_cast<const uint32_t*>(gain) + c) : 0x3F803F80u;
#pragma unroll
            for (int mm = 0; mm < MR; mm++)
                if (mm == m) ss[mm] += v.x * v.x + v.y * v.y;
            *reinterpret_cast<float2*>(act + (size_t)m * K + 2 * c) = make_float2(v.x * bf16_lo(g), v.y * bf16_hi(g));
        }
    } else {
        for (int e0 = tid; e0 < total && ok; e0 += NB * PS_CT) {
            // element e0 + u * PS_CT is pair cu[u] of row mu[u]
            int mu[NB], cu[NB];
            {
                int m = e0 / per, c = e0 - m * per;
#pragma unroll
                for (int u = 0; u < NB; u++) {
                    mu[u] = m;
                    cu[u] = c;
                    c += PS_CT;
                    while (c >= per) {
                        c -= per;
                        m++;
                    }
                }
            }
            u64 a[NB], b[NB];
            uint32_t g[NB];
#pragma unroll
            for (int u = 0; u < NB; u++)
                g[u] = (gain && mu[u] < M) ? __ldg(reinterpret_cast<const uint32_t*>(gain) + cu[u]) : 0x3F803F80u;
            uint64_t t0 = 0;
            uint32_t it = 0;
            for (;;) {
                bool all = true;
#pragma unroll
                for (int u = 0; u < NB; u++) {
                    a[u] = b[u] = ((u64)tag << 32);
                    if (mu[u] < M) ld_tag2(src + (size_t)mu[u] * ld + 2 * cu[u], a[u], b[u]);
                }
#pragma unroll
                for (int u = 0; u < NB; u++) all = all && tag_ok(a[u], tag) && tag_ok(b[u], tag);
                if (all) break;
                if (!ps_keep_waiting(p, s, t0, it, 45)) {
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
#pragma unroll
            for (int u = 0; u < NB; u++) {
                if (mu[u] < M) {
                    const float x0 = tag_val(a[u]), x1 = tag_val(b[u]);
#pragma unroll
                    for (int mm = 0; mm < MR; mm++)
                        if (mm == mu[u]) ss[mm] += x0 * x0 + x1 * x1;
                    *reinterpret_cast<float2*>(act + (size_t)mu[u] * K + 2 * cu[u]) =
                        make_float2(x0 * bf16_lo(g[u]), x1 * bf16_hi(g[u]));
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MR; m++) {
        const float v = warp_sum(ss[m]);
        if (lane == 0) s.ssw[warp][m] = v;
    }
    return ok;
}

// The out-projection's input for Qwen: the attention rows [M][heads * 64], merged from the chunk
// partials (online softmax: o = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c, M = max_c m_c). Warp
// per (unit, query row), lane per pair of output dimensions.
__device__ bool ps_stage_merge(const StackParams& p, PsShared& s, uint32_t tag, float* act) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hkv = p.kv_heads, G = p.heads / hkv, S = p.seq_rows, nq = S * G, A = p.heads * 64;
    const int U = p.seqs * hkv;
    for (int t = warp; t < U * nq; t += PS_CWARPS) {
        const int u = t / nq, qi = t - u * nq, r = u / hkv, h = u - r * hkv, i = qi / G, g = qi - i * G;
        int base, jS;
        const int Cu = ps_unit_chunks(ps_unit_keys(p, r, base, jS), p.chunks);
        const u64* rec0 = p.mb_att + ((size_t)u * p.chunks * nq + qi) * PS_REC;
        float Mx = -INFINITY, Ls = 0.f, o0 = 0.f, o1 = 0.f;
        u64 ml[PS_MAXC][2], ov[PS_MAXC][2];
        bool ok = true;
        uint64_t t0 = 0;
        uint32_t it = 0;
        for (;;) {
            bool all = true;
#pragma unroll
            for (int cc = 0; cc < PS_MAXC; cc++) {
                ml[cc][0] = ml[cc][1] = ov[cc][0] = ov[cc][1] = (u64)tag << 32;
                if (cc < Cu) {
                    const u64* rec = rec0 + (size_t)cc * nq * PS_REC;
                    ld_tag2(rec, ml[cc][0], ml[cc][1]);
                    ld_tag2(rec + 2 + 2 * lane, ov[cc][0], ov[cc][1]);
                }
            }
#pragma unroll
            for (int cc = 0; cc < PS_MAXC; cc++)
                all = all && tag_ok(ml[cc][0], tag) && tag_ok(ml[cc][1], tag) && tag_ok(ov[cc][0], tag) && tag_ok(ov[cc][1], tag);
            if (all) break;
            if (!ps_keep_waiting(p, s, t0, it, 46)) {
                ok = false;
                break;
            }
        }
#pragma unroll
        for (int cc = 0; cc < PS_MAXC; cc++) {
            const float mc = tag_val(ml[cc][0]);
            if (cc >= Cu || !ok || mc == -INFINITY) continue;  // (a chunk without a valid key for this row)
            const float nm = fmaxf(Mx, mc);
            const float so = Mx == -INFINITY ? 0.f : expf(Mx - nm), sc = expf(mc - nm);
            Ls = Ls * so + tag_val(ml[cc][1]) * sc;
            o0 = o0 * so + tag_val(ov[cc][0]) * sc;
            o1 = o1 * so + tag_val(ov[cc][1]) * sc;
            Mx = nm;
        }
        if (!ok) return false;
        const float inv = Ls > 0.f ? 1.0f / Ls : 0.f;
        *reinterpret_cast<float2*>(act + (size_t)(r * S + i) * A + (h * G + g) * 64 + 2 * lane) = make_float2(o0 * inv, o1 * inv);
    }
    return true;
}

// ---------------------------------------------------------------------------------------------
// Linear phase (compute warps): stage the input, then for every ring piece of this CTA's slice
// multiply the staged rows against the piece's weight rows and apply the epilogue.
// ---------------------------------------------------------------------------------------------
template <int MR>
__device__ bool ps_linear(const StackParams& p, PsShared& s, int q, const PsLin& L, uint8_t* ring, float* act,
                          float* red, int& j, int cta, int ctas) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int n0, n1;
    ps_rows(L.n, cta, ctas, n0, n1);
    if (n1 <= n0) return true;
    const int M = p.M, K = L.k, nch = K >> 3;
    const bool gated = L.w2 != nullptr;
    if (L.bias && tid < n1 - n0) s.bias[tid] = bf16f(L.bias[n0 + tid]);
    // Stage the input rows.
    const uint32_t tag_in = ps_tag(s.epoch, L.in_phase);
    bool ok;
    if (L.in == IN_MERGE) {
        ok = ps_stage_merge(p, s, tag_in, act);
    } else {
        const u64* src = L.in == IN_X ? p.mb_x : L.in == IN_ATT ? p.mb_att : p.mb_mlp;
        const int ld = L.in == IN_MLP ? p.inter : p.hidden;
        ok = ps_stage_rows<MR>(p, s, src, L.in == IN_PLAIN ? p.x : nullptr, ld, M, K, tag_in, L.gain, act);
    }
    if (!ok) s.abort = 1;
    named_sync();
    if (s.abort) return false;
    const uint32_t tag_out = ps_tag(s.epoch, q);
    const int rp = ps_piece_rows(ps_layout(p.kind).piece, K, gated);
    for (int r0 = n0; r0 < n1; r0 += rp) {
        const int rows = min(rp, n1 - r0);
        const uint32_t one = (uint32_t)rows * (uint32_t)K * 2u;
        const int slot = j % PS_SLOTS;
        volatile int* abort = &s.abort;
        if (!mbar_wait(&s.bar[slot], (uint32_t)((j / PS_SLOTS) & 1), p.status, 43, abort)) ps_timeout(p, s, 43, (unsigned)q);
        named_sync();
        if (s.abort) return false;
        const uint8_t* wslice = ring + s.slot_off[slot];
        // Warps: WR row groups of rbk-row blocks, WK warps splitting the K chunks of each block.
        constexpr int RB = MR >= 8 ? 2 : 4;
        const int rbk = gated ? 2 : RB;
        const int blocks = (rows + rbk - 1) / rbk;
        const int WR = blocks >= 8 ? 8 : blocks >= 4 ? 4 : blocks >= 2 ? 2 : 1;
        const int WK = PS_CWARPS / WR;
        const int wk = warp % WK, wr = warp / WK;
        const int c_lo = nch * wk / WK, c_hi = nch * (wk + 1) / WK;
        for (int b = wr; b < blocks; b += WR) {
            const int rb0 = b * rbk;
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
                        const float* xp = act + (size_t)m * K + 8 * c;
                        xa[m] = *reinterpret_cast<const float4*>(xp);
                        xb[m] = *reinterpret_cast<const float4*>(xp + 4);
                    }
                }
                if (!gated) {
#pragma unroll
                    for (int r = 0; r < RB; r++) {
                        if (rb0 + r < rows) {
                            const uint4 wv = *reinterpret_cast<const uint4*>(wslice + ((size_t)(rb0 + r) * K + 8 * c) * 2);
#pragma unroll
                            for (int m = 0; m < MR; m++)
                                if (m < M) acc[r][m] += dot8(xa[m], xb[m], wv);
                        }
                    }
                } else {
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        if (rb0 + r < rows) {
                            const size_t o = ((size_t)(rb0 + r) * K + 8 * c) * 2;
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
            // Warp sums; the lane owning (row, m) stores its partial for the cross-warp sum.
#pragma unroll
            for (int r = 0; r < RB; r++) {
#pragma unroll
                for (int m = 0; m < MR; m++) {
                    if (!gated || r < 2) {
                        const float v = warp_sum(acc[r][m]);
                        const float v2 = gated ? warp_sum(acc2[r < 2 ? r : 0][m]) : 0.f;
                        if (lane == r * MR + m && rb0 + r < rows && m < M) {
                            red[((size_t)wk * rows + rb0 + r) * MR + m] = v;
                            if (gated) red[((size_t)(WK + wk) * rows + rb0 + r) * MR + m] = v2;
                        }
                    }
                }
            }
        }
        named_sync();
        // Epilogue (reference order): RMS scale of the folded norm, + bias, SiLU gate, GELU, += y;
        // consecutive threads take consecutive output columns of one row.
        for (int e = tid; e < rows * M; e += PS_CT) {
            const int m = e / rows, r = e - m * rows;
            float v = 0.f, v2 = 0.f;
            for (int w = 0; w < WK; w++) {
                v += red[((size_t)w * rows + r) * MR + m];
                if (gated) v2 += red[((size_t)(WK + w) * rows + r) * MR + m];
            }
            if (L.gain) {
                float ssq = 0.f;
#pragma unroll
                for (int w = 0; w < PS_CWARPS; w++) ssq += s.ssw[w][m];
                const float rs = rsqrtf(ssq / (float)K + p.eps);
                v *= rs;
                v2 *= rs;
            }
            const int n = r0 + r;
            if (L.flags & MT_LINEAR_BIAS) v += s.bias[n - n0];
            if (gated) v = silu(v) * v2;
            if (L.flags & MT_LINEAR_GELU) v = gelu_tanh(v);
            if (L.out == OUT_X) {
                v += s.xown[m][n - n0];  // the residual: this CTA owns column n in every phase that writes it
                s.xown[m][n - n0] = v;
                st_tag(p.mb_x + (size_t)m * p.hidden + n, v, tag_out);
            } else if (L.out == OUT_QKV) {
                st_tag(p.mb_qkv + (size_t)m * (p.kind == STACK_QWEN ? (p.heads + 2 * p.kv_heads) * 64 : 3 * p.hidden) + n, v, tag_out);
            } else {
                st_tag(p.mb_mlp + (size_t)m * p.inter + n, v, tag_out);
            }
        }
        named_sync();
        if (warp == 0) {
            if (lane == 0) {
                s.free_pos = s.slot_end[slot];
                s.consumed = j + 1;
            }
            __syncwarp();
            ps_refill(p, s, ring, cta, ctas);
        }
        j++;
    }
    return true;
}

// ---------------------------------------------------------------------------------------------
// Qwen decode attention of one (sequence, kv head) unit, chunk c of its keys: NeoX RoPE of the new
// rows' q heads and key, KV append at positions pos .. pos + S - 1 (slot = position % cap, by
// chunk 0), and causal / windowed softmax attention (scale 1/8) over the chunk's keys, written as
// an online-softmax partial per query row (max m, weight sum l, unnormalised output o).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ bool ps_attn_qwen(const StackParams& p, PsShared& s, int layer, int u, int c, uint32_t tag_in,
                                          uint32_t tag_out, float* act) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hkv = p.kv_heads, G = p.heads / hkv, S = p.seq_rows, nq = S * G;
    const int r = u / hkv, h = u - r * hkv;
    const int qkvw = (p.heads + 2 * hkv) * 64;
    const int W = p.window;
    int base, jS;
    const int nk = ps_unit_keys(p, r, base, jS);
    const int Cu = ps_unit_chunks(nk, p.chunks);
    if (c >= Cu) return true;
    u64* rec0 = p.mb_att + ((size_t)u * p.chunks * nq) * PS_REC + (size_t)c * nq * PS_REC;
    if (nk < 0) {
        // Positions come from device memory: a bad one is recorded and the unit's partials carry no
        // keys, so the pass completes (its rows come out zero).
        if (tid == 0) report_status(p.status, DEV_BAD_ARG, 44, (unsigned)base);
        for (int t = tid; t < nq * PS_REC / 2; t += PS_CT) {
            const int qi = t / (PS_REC / 2), w = t - qi * (PS_REC / 2);
            st_tag2(rec0 + (size_t)qi * PS_REC + 2 * w, w == 0 ? -INFINITY : 0.f, 0.f, tag_out);
        }
        return true;
    }
    const int k0 = (int)((long long)nk * c / Cu), k1 = (int)((long long)nk * (c + 1) / Cu), nkc = k1 - k0;
    const size_t tensor = (size_t)hkv * p.cap * 64;
    float* kc = p.kv + (size_t)r * p.kv_stride + (size_t)(2 * layer) * tensor + (size_t)h * p.cap * 64;
    float* vc = kc + tensor;
    float* kbuf = act;                             // [PS_CH][PS_KROW] cached keys of the chunk
    float* vbuf = kbuf + PS_CH * PS_KROW;          // [PS_CH][PS_KROW] cached values
    float* qs = vbuf + PS_CH * PS_KROW;            // [nq][64] roped queries
    float* nw = qs + 32 * 64;                      // [S][k | v][64] the new rows (roped key)
    float* sc = nw + 4 * 128;                      // [nq][PS_CH] scores, then weights
    // 1. Cached keys and values of the chunk (positions before base): asynchronous copies.
    const int jc0 = jS + k0, jc1 = min(jS + k1, base);
    const int nold = max(0, jc1 - jc0);
    for (int t = tid; t < nold * 32; t += PS_CT) {
        const int jj = t >> 5, part = t & 31, half = part >> 4, piece = part & 15;
        const int slot = (jc0 + jj) % p.cap;
        cp_async16((half ? vbuf : kbuf) + jj * PS_KROW + 4 * piece, (half ? vc : kc) + (size_t)slot * 64 + 4 * piece);
    }
    // 2. The new rows: (row i, slot g < G query head | G key | G + 1 value, dims l and l + 32).
    bool ok = true;
    for (int it = tid; it < S * (G + 2) * 32 && ok; it += PS_CT) {
        const int l = it & 31, slot = (it >> 5) % (G + 2), i = (it >> 5) / (G + 2);
        const u64* row = p.mb_qkv + (size_t)(r * S + i) * qkvw;
        const int col = slot < G ? (h * G + slot) * 64 : slot == G ? (p.heads + h) * 64 : (p.heads + hkv + h) * 64;
        u64 a, b;
        uint64_t t0 = 0;
        uint32_t wit = 0;
        for (;;) {
            a = ld_tag(row + col + l);
            b = ld_tag(row + col + l + 32);
            if (tag_ok(a, tag_in) && tag_ok(b, tag_in)) break;
            if (!ps_keep_waiting(p, s, t0, wit, 47)) {
                ok = false;
                break;
            }
        }
        if (!ok) break;
        float v0 = tag_val(a), v1 = tag_val(b);
        if (slot <= G) {
            float sn, cs;
            sincosf((float)(base + i) * p.inv_freq[l], &sn, &cs);
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
    if (!ok) s.abort = 1;
    cp_async_wait_all();
    named_sync();
    if (s.abort) return false;
    // 3. Scores: item (key jj, row i) against the G heads of row i.
    for (int it = tid; it < nkc * S; it += PS_CT) {
        const int jj = it % nkc, i = it / nkc;
        const int j = jc0 + jj, pos = base + i;
        const bool valid = j <= pos && (W == 0 || j > pos - W);
        float sg[8];
#pragma unroll
        for (int g = 0; g < 8; g++) sg[g] = 0.f;
        if (valid) {
            const float* kr = j < base ? kbuf + jj * PS_KROW : nw + (size_t)(j - base) * 128;
#pragma unroll
            for (int t = 0; t < 16; t++) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * t);
#pragma unroll
                for (int g = 0; g < 8; g++) {
                    if (g < G) {
                        const float4 q4 = *reinterpret_cast<const float4*>(qs + (i * G + g) * 64 + 4 * t);
                        sg[g] += q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w;
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < 8; g++)
            if (g < G) sc[(i * G + g) * PS_CH + jj] = valid ? sg[g] * 0.125f : -INFINITY;
    }
    named_sync();
    // 4. Chunk softmax statistics per query row (warp per row): weights relative to the chunk maximum.
    for (int qi = warp; qi < nq; qi += PS_CWARPS) {
        float* srow = sc + qi * PS_CH;
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
    // 5. P.V: thread (4 dims d4, row i, part) holds the G heads of row i; PP parts split the keys.
    const int d4 = tid & 15, grp = tid >> 4;
    const int PP = (PS_CT / 16) / S;
    const int pv_i = grp % S, pv_part = grp / S;
    const bool pv_live = pv_part < PP;
    float4 acc[8];
#pragma unroll
    for (int g = 0; g < 8; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (pv_live) {
        for (int jj = pv_part; jj < nkc; jj += PP) {
            const int j = jc0 + jj;
            const float4 v4 = j < base ? *reinterpret_cast<const float4*>(vbuf + jj * PS_KROW + 4 * d4)
                                       : *reinterpret_cast<const float4*>(nw + (size_t)(j - base) * 128 + 64 + 4 * d4);
#pragma unroll
            for (int g = 0; g < 8; g++) {
                if (g < G) {
                    const float pj = sc[(pv_i * G + g) * PS_CH + jj];
                    acc[g].x += pj * v4.x;
                    acc[g].y += pj * v4.y;
                    acc[g].z += pj * v4.z;
                    acc[g].w += pj * v4.w;
                }
            }
        }
    }
    named_sync();  // scores and staged keys are consumed: the part sums overlay them
    float4* part4 = reinterpret_cast<float4*>(act);  // [PP][S][G][16]
    if (pv_live) {
#pragma unroll
        for (int g = 0; g < 8; g++)
            if (g < G) part4[((pv_part * S + pv_i) * G + g) * 16 + d4] = acc[g];
    }
    named_sync();
    // 6. The partial records: m, l, then o[64] (two words per store).
    for (int t = tid; t < nq * 33; t += PS_CT) {
        const int qi = t / 33, w = t - qi * 33, i = qi / G, g = qi - i * G;
        u64* rec = rec0 + (size_t)qi * PS_REC;
        if (w == 0) {
            st_tag2(rec, s.m_run[qi], s.l_run[qi], tag_out);
        } else {
            const int d = 2 * (w - 1);  // dims d, d + 1 of part float4 d / 4
            float o0 = 0.f, o1 = 0.f;
            for (int pp = 0; pp < PP; pp++) {
                const float* v = reinterpret_cast<const float*>(part4 + ((pp * S + i) * G + g) * 16) + d;
                o0 += v[0];
                o1 += v[1];
            }
            st_tag2(rec + 2 + d, o0, o1, tag_out);
        }
    }
    return true;
}

// DiT attention of one (sequence, head) unit by one warp: interleaved RoPE (pairs 2l, 2l + 1, angle
// = row * inv_freq[l]), full softmax attention over the sequence's rows, scale 1/8.
__device__ __forceinline__ bool ps_attn_dit(const StackParams& p, PsShared& s, int unit, uint32_t tag_in, uint32_t tag_out) {
    constexpr int SM = 4;  // rows of a sequence, at most
    const int S = p.seq_rows;
    const int lane = threadIdx.x & 31;
    const int heads = p.heads, D = heads * 64;
    const int h = unit % heads, b = unit / heads;
    const float freq = p.inv_freq[lane];
    const u64* rows = p.mb_qkv + (size_t)b * S * 3 * D + h * 64 + 2 * lane;
    u64 w[SM][3][2];
    bool ok = true;
    uint64_t t0 = 0;
    uint32_t it = 0;
    for (;;) {
        bool all = true;
#pragma unroll
        for (int j = 0; j < SM; j++)
#pragma unroll
            for (int t = 0; t < 3; t++) {
                w[j][t][0] = w[j][t][1] = (u64)tag_in << 32;
                if (j < S) ld_tag2(rows + (size_t)j * 3 * D + t * D, w[j][t][0], w[j][t][1]);
                all = all && tag_ok(w[j][t][0], tag_in) && tag_ok(w[j][t][1], tag_in);
            }
        if (all) break;
        if (!ps_keep_waiting(p, s, t0, it, 48)) {
            ok = false;
            break;
        }
    }
    if (!__all_sync(0xffffffffu, ok)) return false;  // the warp agrees before its shuffles
    // Rotation of row j by angle j * freq: (cos, sin) of freq once, then composed (row 0 is the
    // identity), which keeps a single sincos in the kernel's code.
    float s1, c1;
    sincosf(freq, &s1, &c1);
    float2 q[SM], k[SM], v[SM];
    float cj = 1.f, sj = 0.f;
#pragma unroll
    for (int j = 0; j < SM; j++) {
        q[j] = make_float2(tag_val(w[j][0][0]), tag_val(w[j][0][1]));
        k[j] = make_float2(tag_val(w[j][1][0]), tag_val(w[j][1][1]));
        v[j] = make_float2(tag_val(w[j][2][0]), tag_val(w[j][2][1]));
        if (j == 1) {
            cj = c1;
            sj = s1;
        } else if (j > 1) {
            const float cn = cj * c1 - sj * s1, sn = sj * c1 + cj * s1;
            cj = cn;
            sj = sn;
        }
        q[j] = make_float2(q[j].x * cj - q[j].y * sj, q[j].y * cj + q[j].x * sj);
        k[j] = make_float2(k[j].x * cj - k[j].y * sj, k[j].y * cj + k[j].x * sj);
    }
#pragma unroll
    for (int i = 0; i < SM; i++) {
        if (i >= S) break;
        float sc[SM];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < SM; j++) {
            sc[j] = j < S ? warp_sum(q[i].x * k[j].x + q[i].y * k[j].y) * 0.125f : -INFINITY;
            mx = fmaxf(mx, sc[j]);
        }
        float sum = 0.f, a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int j = 0; j < SM; j++) {
            if (j >= S) break;
            const float e = expf(sc[j] - mx);
            sum += e;
            a0 += e * v[j].x;
            a1 += e * v[j].y;
        }
        st_tag2(p.mb_att + (size_t)(b * S + i) * D + h * 64 + 2 * lane, a0 / sum, a1 / sum, tag_out);
    }
    return true;
}

// Final norm of every row (Qwen), one row per CTA: z = x * rsqrt(mean(x^2) + eps) * g.
__device__ bool ps_final(const StackParams& p, PsShared& s, uint32_t tag_in, float* act, int cta, int ctas) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.hidden;
    for (int m = cta; m < p.M; m += ctas) {
        const u64* row = p.mb_x + (size_t)m * H;
        float ss = 0.f;
        bool ok = true;
        for (int c = tid; c < (H >> 1); c += PS_CT) {
            u64 a, b;
            uint64_t t0 = 0;
            uint32_t it = 0;
            for (;;) {
                ld_tag2(row + 2 * c, a, b);
                if (tag_ok(a, tag_in) && tag_ok(b, tag_in)) break;
                if (!ps_keep_waiting(p, s, t0, it, 49)) {
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
            const float x0 = tag_val(a), x1 = tag_val(b);
            act[2 * c] = x0;
            act[2 * c + 1] = x1;
            ss += x0 * x0 + x1 * x1;
        }
        if (!ok) s.abort = 1;
        ss = warp_sum(ss);
        if (lane == 0) s.ssw[warp][0] = ss;
        named_sync();
        if (s.abort) return false;
        float tot = 0.f;
        for (int w = 0; w < PS_CWARPS; w++) tot += s.ssw[w][0];
        const float rs = rsqrtf(tot / (float)H + p.eps);
        for (int c = tid; c < (H >> 1); c += PS_CT) {
            const uint32_t g = *reinterpret_cast<const uint32_t*>(p.final_norm + 2 * c);
            *reinterpret_cast<float2*>(p.z + (size_t)m * H + 2 * c) =
                make_float2(act[2 * c] * rs * bf16_lo(g), act[2 * c + 1] * rs * bf16_hi(g));
        }
        named_sync();
    }
    return true;
}

template <int MR>
__global__ void __launch_bounds__(PS_THREADS, 1) stack_kernel(const __grid_constant__ StackParams p) {
    extern __shared__ __align__(128) uint8_t ps_smem[];
    __shared__ PsShared s;
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ps_smem) + 127) & ~uintptr_t(127));
    const PsLayout lay = ps_layout(p.kind);
    float* act = reinterpret_cast<float*>(ring + lay.ring);
    float* red = reinterpret_cast<float*>(ring + lay.ring + lay.act);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int cta = blockIdx.x, ctas = gridDim.x;
    if (tid == 0) {
        for (int i = 0; i < PS_SLOTS; i++) mbar_init(&s.bar[i], 1);
        s.free_pos = 0;
        s.consumed = 0;
        s.prod_q = 0;
        s.prod_r0 = -1;
        s.prod_j = 0;
        s.prod_alloc = 0;
        s.abort = 0;
        s.epoch = *reinterpret_cast<const volatile unsigned int*>(p.sync);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = tid; i < p.layers * 10; i += PS_CT) s.layer[i / 10].p[i % 10] = p.L[i / 10].p[i % 10];
    __syncthreads();
    if (warp == 0) ps_refill(p, s, ring, cta, ctas);  // fill the ring
    int xn0, xn1;  // this CTA's columns of the residual rows (every phase that adds into x writes these)
    ps_rows(p.hidden, cta, ctas, xn0, xn1);
    const int xw = xn1 - xn0;
    for (int e = tid; e < p.M * xw; e += PS_CT) s.xown[e / xw][e % xw] = __ldcg(p.x + (size_t)(e / xw) * p.hidden + xn0 + e % xw);
    named_sync();
    const int P = ps_phases(p);
    int j = 0;  // ring pieces consumed
    for (int q = 0; q < P; q++) {
        const int type = ps_type(p, q);
        bool ok = true;
        if (type == PT_LIN) {
            ok = ps_linear<MR>(p, s, q, ps_lin(p, s.layer, q), ring, act, red, j, cta, ctas);
        } else if (type == PT_ATTN_QWEN) {
            const int U = p.seqs * p.kv_heads;
            for (int b = cta; b < U * p.chunks && ok; b += ctas) {
                ok = ps_attn_qwen(p, s, q / 5, b / p.chunks, b % p.chunks, ps_tag(s.epoch, q - 1), ps_tag(s.epoch, q), act);
                named_sync();
            }
        } else if (type == PT_ATTN_DIT) {
            for (int u = cta + warp * ctas; u < p.seqs * p.heads && ok; u += ctas * PS_CWARPS)
                ok = ps_attn_dit(p, s, u, ps_tag(s.epoch, q - 1), ps_tag(s.epoch, q));
        } else {
            ok = ps_final(p, s, ps_tag(s.epoch, q - 1), act, cta, ctas);
        }
        if (!ok) s.abort = 1;
        named_sync();
        if (s.abort) break;
    }
    // The residual rows leave in the caller's layout.
    if (!s.abort)
        for (int e = tid; e < p.M * xw; e += PS_CT) p.x[(size_t)(e / xw) * p.hidden + xn0 + e % xw] = s.xown[e / xw][e % xw];
    // Copies still in flight (after an abort) land before the CTA exits.
    if (tid == 0) {
        int dummy = 0;
        volatile int* ab = &dummy;
        for (int jj = s.consumed; jj < s.prod_j; jj++)
            mbar_wait(&s.bar[jj % PS_SLOTS], (uint32_t)((jj / PS_SLOTS) & 1), p.status, 42, ab);
    }
    __syncthreads();
    // The last CTA to leave closes the launch: the next launch's tags use the next epoch.
    if (tid == 0) {
        __threadfence();
        const unsigned int done = atomicAdd(p.sync + 1, 1u);
        if (done == (unsigned)ctas - 1u) {
            p.sync[1] = 0u;
            p.sync[2] = 0u;
            p.sync[0] = s.epoch + 1u;
            __threadfence();
        }
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

size_t up16(size_t words) { return (words + 15) & ~size_t(15); }  // 128-byte aligned pieces

// Attention chunks per unit for the longest key range a pass can have.
int qwen_chunks(const StackParams& p) {
    const int nk = p.window > 0 ? p.window + p.seq_rows - 1 : p.cap;
    return (nk + PS_CH - 1) / PS_CH;
}

}  // namespace

const char* stack_resident_why() { return g_resident_why; }

int stack_resident_blocks() {
    int dev = 0;
    if (!stack_resident() && (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)) return 0;
    return g_resident[dev];
}

// Stack area of a pass: 16 sync words ([0] epoch, [1] exit count, [2] abort), then the mailbox rows
// x [M][hidden], qkv [M][qkv width], attention (Qwen partials [units][chunks][rows x G][66] or DiT
// rows [M][hidden]) and MLP [M][inter], as 8-byte words.
size_t stack_area_bytes(const StackParams& p) {
    const size_t M = (size_t)p.M;
    const bool qwen = p.kind == STACK_QWEN;
    const size_t qkvw = qwen ? (size_t)(p.heads + 2 * p.kv_heads) * 64 : 3 * (size_t)p.hidden;
    size_t att = M * p.hidden;
    if (qwen && p.kv_heads > 0) {
        const size_t units = (size_t)p.seqs * p.kv_heads, nq = (size_t)p.seq_rows * (p.heads / p.kv_heads);
        att = units * (size_t)qwen_chunks(p) * nq * PS_REC;
    }
    return (16 + up16(M * p.hidden) + up16(M * qkvw) + up16(att) + up16(M * p.inter)) * sizeof(u64);
}

void stack_bind(StackParams& p, void* area) {
    const size_t M = (size_t)p.M;
    const bool qwen = p.kind == STACK_QWEN;
    const size_t qkvw = qwen ? (size_t)(p.heads + 2 * p.kv_heads) * 64 : 3 * (size_t)p.hidden;
    size_t att = M * p.hidden;
    p.chunks = 1;
    if (qwen && p.kv_heads > 0) {
        p.chunks = qwen_chunks(p);
        const size_t units = (size_t)p.seqs * p.kv_heads, nq = (size_t)p.seq_rows * (p.heads / p.kv_heads);
        att = units * (size_t)p.chunks * nq * PS_REC;
    }
    u64* w = static_cast<u64*>(area);
    p.sync = reinterpret_cast<unsigned int*>(w);
    p.mb_x = w + 16;
    p.mb_qkv = p.mb_x + up16(M * p.hidden);
    p.mb_att = p.mb_qkv + up16(M * qkvw);
    p.mb_mlp = p.mb_att + up16(att);
}

mt_status stack_area_alloc(size_t bytes, void** out) {
    *out = nullptr;
    if (cudaMalloc(out, bytes) != cudaSuccess) {
        *out = nullptr;
        return MT_ERR_NOMEM;
    }
    if (cudaMemset(*out, 0, bytes) != cudaSuccess) {  // epoch 0, and no word carries a valid tag
        cudaFree(*out);
        *out = nullptr;
        return MT_ERR_CUDA;
    }
    return MT_OK;
}

// Whether a pass fits the persistent kernel: rows, staged inputs, ring pieces, attention scratch,
// cross-warp partial sums, residual columns and bias rows per CTA.
bool stack_supported(const StackParams& p, int ctas) {
    if (p.M < 1 || p.M > 8 || p.layers < 1 || p.layers > STACK_MAX_LAYERS || ctas < 1) return false;
    if (!stack_resident()) return false;
    if (p.hidden % 8 || p.inter % 8 || p.seqs * p.seq_rows != p.M) return false;
    if ((p.hidden + ctas - 1) / ctas > PS_XOWN) return false;
    const bool qwen = p.kind == STACK_QWEN;
    const int qkvw = qwen ? (p.heads + 2 * p.kv_heads) * 64 : 3 * p.hidden;
    const int A = qwen ? p.heads * 64 : p.hidden;
    if (qwen) {
        const int hkv = p.kv_heads;
        if (hkv < 1 || p.heads % hkv || p.heads / hkv > 8 || p.seq_rows < 1 || p.seq_rows > 4) return false;
        if (p.heads * p.seq_rows > 32 * hkv) return false;  // query rows of a unit: at most 32
        if (p.window > 0 && p.window + p.seq_rows - 1 > p.cap) return false;
        if (qwen_chunks(p) > PS_MAXC) return false;
        const size_t att = ((size_t)2 * PS_CH * PS_KROW + 32 * 64 + 4 * 128 + (size_t)32 * PS_CH) * 4;
        if (att > ps_layout(p.kind).act || (size_t)(PS_CT / 16) * 8 * 16 * 16 > ps_layout(p.kind).act) return false;
    } else {
        if (p.seq_rows < 1 || p.seq_rows > 4 || p.hidden != p.heads * 64) return false;
    }
    // Staged inputs, ring pieces, partial sums and bias rows of every linear.
    const int ns[4] = {qkvw, p.hidden, p.inter, p.hidden};
    const int ks[4] = {p.hidden, A, p.hidden, p.inter};
    const bool gate[4] = {false, false, qwen, false};
    for (int i = 0; i < 4; i++) {
        const PsLayout lay = ps_layout(p.kind);
        if ((size_t)p.M * ks[i] * 4 > lay.act || ks[i] % 8) return false;
        const int rows = (ns[i] + ctas - 1) / ctas;
        if (rows > PS_BIAS) return false;
        const uint32_t rowbytes = (uint32_t)ks[i] * 2u * (gate[i] ? 2u : 1u);
        if (rowbytes > lay.piece) return false;
        const int rp = min(rows, ps_piece_rows(lay.piece, ks[i], gate[i]));
        const int MR = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
        const int rbk = gate[i] ? 2 : (MR >= 8 ? 2 : 4);
        const int blocks = (rp + rbk - 1) / rbk;
        const int WR = blocks >= 8 ? 8 : blocks >= 4 ? 4 : blocks >= 2 ? 2 : 1;
        const int WK = PS_CWARPS / WR;
        if ((size_t)WK * rp * MR * (gate[i] ? 2 : 1) * 4 > PS_RED) return false;
    }
    return true;
}

// Phases of a pass.
int stack_phases(const StackParams& p) { return p.layers * 5 + (p.kind == STACK_QWEN && p.z ? 1 : 0); }

void launch_stack(const StackParams& p, int ctas, cudaStream_t s) {
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
