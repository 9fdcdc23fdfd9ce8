// linear.cu -- Y[m, n] = epi(X[m, :k] . W[n, :k]^T) for small m on CUDA cores, and the mt_linear
// dispatcher (CUDA-core GEMV for m <= 8, tcgen05 tensor-core GEMM above).
//
// Reference semantics: gemv_kernel / gemm8_kernel / gemm_kernel (Shaders.swift:47-108, 191-277,
// 304-408), routing Encoder.linear (Kernels.swift:132-161). fp32 X, bf16 W, fp32 accumulate,
// epilogue order +bias -> silu gate -> gelu -> silu -> accumulate.
//
// GEMV design: the weight matrix is streamed exactly once with 16-byte non-caching loads; a group
// of G threads (8..128, a power of two) owns one output column for all MR rows, G sized so each
// thread has at most eight 16-byte loads, all issued together before the programmatic-launch
// dependency wait; partial sums meet through warp shuffles (and shared memory when G spans warps).
// For 2..8 rows a second kernel (gemv_quad_kernel) gives each warp 4 columns and stages x in shared
// memory once per block, so x is no longer re-read per column group.
#include "common.cuh"
#include "kernels.cuh"

namespace mt {

constexpr int GEMV_THREADS = 256;

// acc[r] (+ acc2[r] for the gated up projection) += x[r, k0:k0+8] . w[k0:k0+8] for the rows present;
// with NORM, x is first scaled by the gain chunk g and ss[r] collects the raw x^2 (the row's RMS).
template <int MR, bool GATED, bool NORM>
__device__ __forceinline__ void gemv_chunk(float (&acc)[MR], float (&acc2)[MR], float (&ss)[MR], const uint4& w,
                                           const uint4& w2, const uint4& g, const float* x, int ldx, int rows, int k0) {
#pragma unroll
    for (int r = 0; r < MR; r++) {
        if (r < rows) {
            float4 x0 = *reinterpret_cast<const float4*>(x + (size_t)r * ldx + k0);
            float4 x1 = *reinterpret_cast<const float4*>(x + (size_t)r * ldx + k0 + 4);
            if (NORM) {
                ss[r] += x0.x * x0.x + x0.y * x0.y + x0.z * x0.z + x0.w * x0.w + x1.x * x1.x + x1.y * x1.y +
                         x1.z * x1.z + x1.w * x1.w;
                x0 = make_float4(x0.x * bf16_lo(g.x), x0.y * bf16_hi(g.x), x0.z * bf16_lo(g.y), x0.w * bf16_hi(g.y));
                x1 = make_float4(x1.x * bf16_lo(g.z), x1.y * bf16_hi(g.z), x1.z * bf16_lo(g.w), x1.w * bf16_hi(g.w));
            }
            acc[r] += x0.x * bf16_lo(w.x) + x0.y * bf16_hi(w.x) + x0.z * bf16_lo(w.y) + x0.w * bf16_hi(w.y) +
                      x1.x * bf16_lo(w.z) + x1.y * bf16_hi(w.z) + x1.z * bf16_lo(w.w) + x1.w * bf16_hi(w.w);
            if (GATED)
                acc2[r] += x0.x * bf16_lo(w2.x) + x0.y * bf16_hi(w2.x) + x0.z * bf16_lo(w2.y) + x0.w * bf16_hi(w2.y) +
                           x1.x * bf16_lo(w2.z) + x1.y * bf16_hi(w2.z) + x1.z * bf16_lo(w2.w) + x1.w * bf16_hi(w2.w);
        }
    }
}

template <int MR, int G, bool GATED, bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_stream_kernel(LinearArgs a) {
    constexpr int C = GEMV_THREADS / G;  // columns per block
    constexpr int U = G >= 128 ? 8 : 4;  // chunks per thread loaded ahead of the dependency wait
    constexpr int NR = 1 + (GATED ? 1 : 0) + (NORM ? 1 : 0);  // partial sums per row: dot, gated dot, x^2
    __shared__ float red[NR][GEMV_THREADS / 32][MR];
    const int tid = threadIdx.x;
    const int group = tid / G, gl = tid % G;
    const int n = blockIdx.x * C + group;
    const int row0 = blockIdx.y * MR;
    const bool live = n < a.n;
    const int chunks = a.k >> 3;
    const uint16_t* wrow = a.w + (size_t)(live ? n : 0) * a.k;
    const uint16_t* w2row = GATED ? a.w2 + (size_t)(live ? n : 0) * a.k : nullptr;

    // The weights (and norm gains) do not depend on the previous kernel: all of this thread's first
    // U 16-byte loads (every load when k <= 8 U G, which the group size ensures up to k = 8192) are
    // issued before the dependency wait, so they stream while the previous kernel drains.
    uint4 wv[U], wv2[U], gv[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
        const int c = gl + u * G;
        wv[u] = wv2[u] = gv[u] = make_uint4(0, 0, 0, 0);
        if (live && c < chunks) {
            wv[u] = ld_stream_u4(wrow + (size_t)c * 8);
            if (GATED) wv2[u] = ld_stream_u4(w2row + (size_t)c * 8);
            if (NORM) gv[u] = __ldg(reinterpret_cast<const uint4*>(a.norm_w + (size_t)c * 8));
        }
    }
    pdl_wait();
    pdl_launch();
    const int rows = min(MR, a.m - row0);

    float acc[MR], acc2[MR], ss[MR];
#pragma unroll
    for (int r = 0; r < MR; r++) { acc[r] = 0.f; acc2[r] = 0.f; ss[r] = 0.f; }

    if (live) {
        const float* x = a.x + (size_t)row0 * a.ldx;
        // Chunks in ascending order (gl, gl + G, ...), one add per chunk into the row's sum.
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = gl + u * G;
            if (c < chunks) gemv_chunk<MR, GATED, NORM>(acc, acc2, ss, wv[u], wv2[u], gv[u], x, a.ldx, rows, c * 8);
        }
        for (int c = gl + U * G; c < chunks; c += G) {
            const uint4 w = ld_stream_u4(wrow + (size_t)c * 8);
            const uint4 w2 = GATED ? ld_stream_u4(w2row + (size_t)c * 8) : make_uint4(0, 0, 0, 0);
            const uint4 g = NORM ? __ldg(reinterpret_cast<const uint4*>(a.norm_w + (size_t)c * 8)) : make_uint4(0, 0, 0, 0);
            gemv_chunk<MR, GATED, NORM>(acc, acc2, ss, w, w2, g, x, a.ldx, rows, c * 8);
        }
    }

    // Reduce over the G threads of the column group.
    constexpr int WG = G < 32 ? G : 32;
#pragma unroll
    for (int r = 0; r < MR; r++) {
#pragma unroll
        for (int o = WG / 2; o > 0; o >>= 1) {
            acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
            if (GATED) acc2[r] += __shfl_xor_sync(0xffffffffu, acc2[r], o);
            if (NORM) ss[r] += __shfl_xor_sync(0xffffffffu, ss[r], o);
        }
    }
    if (G > 32) {
        const int warp = tid >> 5, lane = tid & 31;
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < MR; r++) {
                red[0][warp][r] = acc[r];
                if (GATED) red[1][warp][r] = acc2[r];
                if (NORM) red[NR - 1][warp][r] = ss[r];
            }
        }
        __syncthreads();
        if (gl != 0) return;
        const int w0 = group * (G / 32);
#pragma unroll
        for (int r = 0; r < MR; r++) {
            float s = 0.f, s2 = 0.f, s3 = 0.f;
            for (int w = 0; w < G / 32; w++) {
                s += red[0][w0 + w][r];
                if (GATED) s2 += red[GATED ? 1 : 0][w0 + w][r];
                if (NORM) s3 += red[NR - 1][w0 + w][r];
            }
            acc[r] = s;
            acc2[r] = s2;
            ss[r] = s3;
        }
    } else if (gl != 0) {
        return;
    }
    if (!live) return;

    const float bval = (a.flags & MT_LINEAR_BIAS) ? bf16f(a.bias[n]) : 0.f;
#pragma unroll
    for (int r = 0; r < MR; r++) {
        if (r < rows) {
            float v = acc[r], v2 = acc2[r];
            if (NORM) {
                const float rs = rsqrtf(ss[r] / (float)a.k + a.norm_eps);
                v *= rs;
                v2 *= rs;
            }
            v += bval;
            if (GATED) v = silu(v) * v2;
            if (a.flags & MT_LINEAR_GELU) v = gelu_tanh(v);
            if (a.flags & MT_LINEAR_SILU) v = silu(v);
            if (a.y) {
                float* yp = a.y + (size_t)(row0 + r) * a.ldy + n;
                if (a.flags & MT_LINEAR_ACCUM) v += *yp;
                *yp = v;
            }
            if (a.y_hi) {  // bf16 hi/lo planes for a tensor-core consumer
                uint16_t h, l;
                split_bf16(v, h, l);
                a.y_hi[(size_t)(row0 + r) * a.ld_ysplit + n] = h;
                a.y_lo[(size_t)(row0 + r) * a.ld_ysplit + n] = l;
            }
        }
    }
}

template <int MR, bool GATED, bool NORM>
static void launch_gemv_g(const LinearArgs& a, int G, cudaStream_t s) {
    const int C = GEMV_THREADS / G;
    dim3 grid((a.n + C - 1) / C, (a.m + MR - 1) / MR);
    switch (G) {
        case 8: launch_k(gemv_stream_kernel<MR, 8, GATED, NORM>, grid, GEMV_THREADS, 0, s, a); break;
        case 16: launch_k(gemv_stream_kernel<MR, 16, GATED, NORM>, grid, GEMV_THREADS, 0, s, a); break;
        case 32: launch_k(gemv_stream_kernel<MR, 32, GATED, NORM>, grid, GEMV_THREADS, 0, s, a); break;
        case 64: launch_k(gemv_stream_kernel<MR, 64, GATED, NORM>, grid, GEMV_THREADS, 0, s, a); break;
        default: launch_k(gemv_stream_kernel<MR, 128, GATED, NORM>, grid, GEMV_THREADS, 0, s, a); break;
    }
}

template <int MR>
static void launch_gemv_mr(const LinearArgs& a, int G, bool gated, cudaStream_t s) {
    if (a.norm_w) {
        if (gated) launch_gemv_g<MR, true, true>(a, G, s);
        else launch_gemv_g<MR, false, true>(a, G, s);
    } else {
        if (gated) launch_gemv_g<MR, true, false>(a, G, s);
        else launch_gemv_g<MR, false, false>(a, G, s);
    }
}

// Threads per column: about four 16-byte chunks per thread, 8..128 (up to eight at 128, k <= 8192).
// Measured in graph replay over a weight pool larger than L2: W[4864x896] streams fastest with 32
// threads per column (608 blocks), W[896x4864] with 128 (448 blocks) rather than 256 (896 blocks).
static int gemv_group(int k) {
    const int chunks = k / 8;
    int g = 8;
    while (g < 128 && g * 4 < chunks) g *= 2;
    return g;
}

// GEMV for 2..8 rows. A warp owns 4 output columns; the 8 lanes of a column read 8 consecutive
// 16-byte pieces of its weight row (one 128-byte line per column per load: full coalescing), and
// each lane's 8 K values of x serve all 4 columns. The column-group GEMV above re-reads every row
// of x once per column group (16 bytes of x per weight byte at 8 rows, which bounds it by L1 at
// these row counts); one column per lane instead made each load touch 32 lines. The block's x
// range (and norm gains) is staged in shared memory once, in a lane-interleaved order so that the
// 8 lanes of a load read one contiguous 128 bytes. Warps split a block's columns (WC = 8 / KW
// groups of 4) and its K range (KW parts, met in shared memory); blockIdx.y splits K across blocks
// for plain accumulating linears (partial sums added to y atomically).
constexpr int GQ_WARPS = 8;
constexpr int GQ_MAX_KLEN = 1024;  // K elements staged per block

template <int MR, bool GATED, bool NORM>
__global__ void __launch_bounds__(GQ_WARPS * 32) gemv_quad_kernel(LinearArgs a, int KW, int ks_steps) {
    constexpr int U = GATED ? 8 : 16;  // 64-wide K steps per lane loaded together
    constexpr int NR = GATED ? 2 : 1;
    __shared__ float red[GQ_WARPS][NR][MR][4];
    __shared__ float ssm[MR];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int col = lane >> 3, kl = lane & 7;
    const int WC = GQ_WARPS / KW, wc = warp % WC, wk = warp / WC;
    const int cpb = 4 * WC;
    const int n = blockIdx.x * cpb + wc * 4 + col;
    const bool live = n < a.n;
    const int steps_all = a.k >> 6;
    const int b0 = blockIdx.y * ks_steps, b1 = min(steps_all, b0 + ks_steps);
    const int per = (b1 - b0 + KW - 1) / KW;
    const int s0 = b0 + wk * per, s1 = min(b1, s0 + per);  // this warp's steps (possibly none)
    const uint16_t* wrow = a.w + (size_t)(live ? n : 0) * a.k + kl * 8;
    const uint16_t* w2row = GATED ? a.w2 + (size_t)(live ? n : 0) * a.k + kl * 8 : nullptr;

    uint4 wv[U], wv2[U];
    auto load = [&](int sb) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int st = sb + u;
            wv[u] = wv2[u] = make_uint4(0, 0, 0, 0);
            if (live && st < s1) {
                wv[u] = ld_stream_u4(wrow + (size_t)st * 64);
                if (GATED) wv2[u] = ld_stream_u4(w2row + (size_t)st * 64);
            }
        }
    };
    load(s0);  // weights never depend on the previous kernel
    pdl_wait();
    pdl_launch();
    const int rows = min(MR, a.m);

    // Stage x (and the gains): float4 f of a 64-wide step (lane f / 2, half f % 2) goes to slot
    // 8 (f % 2) + f / 2, so lane l's halves sit at slots l and 8 + l.
    extern __shared__ __align__(16) float xs[];  // [rows][klen], then the gains [klen]
    const int k0 = b0 * 64, klen = (b1 - b0) * 64, q4 = klen >> 2;
    float4* xs4 = reinterpret_cast<float4*>(xs);
    float4* gs4 = xs4 + (size_t)MR * q4;
    constexpr int SV = MR;  // float4s per thread in flight: all of them for klen <= GQ_MAX_KLEN
    for (int i0 = threadIdx.x; i0 < rows * q4; i0 += GQ_WARPS * 32 * SV) {
        float4 v[SV];
#pragma unroll
        for (int u = 0; u < SV; u++) {
            const int i = i0 + u * GQ_WARPS * 32;
            if (i < rows * q4) {
                const int rr = i / q4, f = i - rr * q4;
                v[u] = *reinterpret_cast<const float4*>(a.x + (size_t)rr * a.ldx + k0 + 4 * f);
            }
        }
#pragma unroll
        for (int u = 0; u < SV; u++) {
            const int i = i0 + u * GQ_WARPS * 32;
            if (i < rows * q4) {
                const int rr = i / q4, f = i - rr * q4;
                xs4[rr * q4 + (f & ~15) + 8 * (f & 1) + ((f & 15) >> 1)] = v[u];
            }
        }
    }
    if (NORM) {
        for (int i = threadIdx.x; i < (klen >> 3); i += GQ_WARPS * 32) {
            const uint4 g = *reinterpret_cast<const uint4*>(a.norm_w + k0 + 8 * i);
            const int f = 2 * i;  // float4s f and f + 1: lane (f % 16) / 2, halves 0 and 1
            const int slot = (f & ~15) + ((f & 15) >> 1);
            gs4[slot] = make_float4(bf16_lo(g.x), bf16_hi(g.x), bf16_lo(g.y), bf16_hi(g.y));
            gs4[slot + 8] = make_float4(bf16_lo(g.z), bf16_hi(g.z), bf16_lo(g.w), bf16_hi(g.w));
        }
    }
    __syncthreads();
    if (NORM && warp < rows) {  // sum of squares of each row over the block's range (= all of K)
        float q = 0.f;
        for (int i = lane; i < q4; i += 32) {
            const float4 v = xs4[warp * q4 + i];
            q += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        q = warp_sum(q);
        if (lane == 0) ssm[warp] = q;
    }

    float acc[MR], acc2[MR];
#pragma unroll
    for (int r = 0; r < MR; r++) { acc[r] = 0.f; acc2[r] = 0.f; }
    for (int sb = s0; sb < s1; sb += U) {
        if (sb != s0) load(sb);
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int st = sb + u;
            if (st >= s1) break;  // warp-uniform
            float wf[8], wf2[8];
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wv[u]);
            const uint32_t* wp2 = reinterpret_cast<const uint32_t*>(&wv2[u]);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                wf[2 * j] = bf16_lo(wp[j]);
                wf[2 * j + 1] = bf16_hi(wp[j]);
                if (GATED) {
                    wf2[2 * j] = bf16_lo(wp2[j]);
                    wf2[2 * j + 1] = bf16_hi(wp2[j]);
                }
            }
            const int base = (st - b0) * 16 + kl;
            if (NORM) {
                const float4 g0 = gs4[base], g1 = gs4[base + 8];
                const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    wf[j] *= g[j];
                    if (GATED) wf2[j] *= g[j];
                }
            }
#pragma unroll
            for (int r = 0; r < MR; r++) {
                if (r < rows) {
                    const float4 x0 = xs4[r * q4 + base], x1 = xs4[r * q4 + base + 8];
                    acc[r] += x0.x * wf[0] + x0.y * wf[1] + x0.z * wf[2] + x0.w * wf[3] + x1.x * wf[4] + x1.y * wf[5] +
                              x1.z * wf[6] + x1.w * wf[7];
                    if (GATED)
                        acc2[r] += x0.x * wf2[0] + x0.y * wf2[1] + x0.z * wf2[2] + x0.w * wf2[3] + x1.x * wf2[4] +
                                   x1.y * wf2[5] + x1.z * wf2[6] + x1.w * wf2[7];
                }
            }
        }
    }
    // Sum over the 8 lanes of each column; lane kl then serves row kl.
#pragma unroll
    for (int r = 0; r < MR; r++) {
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
            if (GATED) acc2[r] += __shfl_xor_sync(0xffffffffu, acc2[r], o);
        }
    }
    float v = 0.f, v2 = 0.f;
#pragma unroll
    for (int r = 0; r < MR; r++)
        if (kl == r) { v = acc[r]; v2 = acc2[r]; }
    int r = kl, nn = n;
    if (KW > 1) {  // the KW warps of a column group meet in shared memory
        if (kl < MR) {
            red[warp][0][kl][col] = v;
            if (GATED) red[warp][GATED ? 1 : 0][kl][col] = v2;
        }
        __syncthreads();
        const int t = threadIdx.x;  // task (row r, block column cb)
        if (t >= MR * cpb) return;
        r = t / cpb;
        const int cb = t - r * cpb, cw = cb >> 2, cc = cb & 3;
        v = v2 = 0.f;
        for (int q = 0; q < KW; q++) {
            v += red[q * WC + cw][0][r][cc];
            if (GATED) v2 += red[q * WC + cw][GATED ? 1 : 0][r][cc];
        }
        nn = blockIdx.x * cpb + cb;
    } else if (NORM) {
        __syncthreads();  // ssm
    }
    if (r >= rows || nn >= a.n) return;
    if (NORM) {
        const float rs = rsqrtf(ssm[r] / (float)a.k + a.norm_eps);
        v *= rs;
        v2 *= rs;
    }
    if ((a.flags & MT_LINEAR_BIAS) && blockIdx.y == 0) v += bf16f(a.bias[nn]);
    if (GATED) v = silu(v) * v2;
    if (a.flags & MT_LINEAR_GELU) v = gelu_tanh(v);
    if (a.flags & MT_LINEAR_SILU) v = silu(v);
    if (a.y) {
        float* yp = a.y + (size_t)r * a.ldy + nn;
        if (gridDim.y > 1) {
            atomicAdd(yp, v);  // K split across blocks: plain accumulating epilogue only
        } else {
            if (a.flags & MT_LINEAR_ACCUM) v += *yp;
            *yp = v;
        }
    }
    if (a.y_hi) {
        uint16_t h, l;
        split_bf16(v, h, l);
        a.y_hi[(size_t)r * a.ld_ysplit + nn] = h;
        a.y_lo[(size_t)r * a.ld_ysplit + nn] = l;
    }
}

// Launch shape of the 2..8-row GEMV: K steps per block (split across blocks only for plain
// accumulating epilogues, so that a block stages at most GQ_MAX_KLEN values of each x row) and KW,
// the warps per column group: the smallest that gives about a wave of blocks.
struct GemvQuadShape { int ks_steps, ks, kw; };
static GemvQuadShape gemv_quad_shape(const LinearArgs& a, bool gated) {
    const int steps = a.k / 64;
    const bool plain_accum = (a.flags & MT_LINEAR_ACCUM) && !(a.flags & (MT_LINEAR_GELU | MT_LINEAR_SILU)) && !gated &&
                             !a.norm_w && !a.y_hi;
    GemvQuadShape sh;
    int ks = plain_accum ? (steps * 64 + GQ_MAX_KLEN - 1) / GQ_MAX_KLEN : 1;
    sh.ks_steps = (steps + ks - 1) / ks;
    sh.ks = (steps + sh.ks_steps - 1) / sh.ks_steps;
    sh.kw = 1;
    while (sh.kw < GQ_WARPS && sh.kw < sh.ks_steps &&
           (long long)((a.n + 4 * (GQ_WARPS / sh.kw) - 1) / (4 * (GQ_WARPS / sh.kw))) * sh.ks < 148)
        sh.kw *= 2;
    if (sh.kw > sh.ks_steps) sh.kw = 1;
    return sh;
}

static size_t gemv_quad_smem(const LinearArgs& a, int mr, int ks_steps) {
    return (size_t)ks_steps * 64 * sizeof(float) * (mr + (a.norm_w ? 1 : 0));
}

template <int MR, bool GATED, bool NORM>
static void launch_gemv_quad_g(const LinearArgs& a, cudaStream_t s) {
    const GemvQuadShape sh = gemv_quad_shape(a, GATED);
    const int cpb = 4 * (GQ_WARPS / sh.kw);
    launch_k(gemv_quad_kernel<MR, GATED, NORM>, dim3((a.n + cpb - 1) / cpb, sh.ks), GQ_WARPS * 32,
             gemv_quad_smem(a, MR, sh.ks_steps), s, a, sh.kw, sh.ks_steps);
}

template <int MR>
static void launch_gemv_quad(const LinearArgs& a, bool gated, cudaStream_t s) {
    if (a.norm_w) {
        if (gated) launch_gemv_quad_g<MR, true, true>(a, s);
        else launch_gemv_quad_g<MR, false, true>(a, s);
    } else {
        if (gated) launch_gemv_quad_g<MR, true, false>(a, s);
        else launch_gemv_quad_g<MR, false, false>(a, s);
    }
}

static bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// The 2..8-row kernel takes K a multiple of 64, 16-byte aligned rows, and a staged x range within
// the default 48 KB of dynamic shared memory.
static bool gemv_quad_fits(const LinearArgs& a, bool gated) {
    if (!(a.m >= 2 && a.m <= 8 && a.k % 64 == 0 && a.ldx % 4 == 0 && al16(a.x) && al16(a.w) &&
          (!gated || al16(a.w2)) && (!a.norm_w || al16(a.norm_w))))
        return false;
    const int mr = a.m <= 2 ? 2 : a.m <= 4 ? 4 : 8;
    return gemv_quad_smem(a, mr, gemv_quad_shape(a, gated).ks_steps) <= 48 * 1024;
}

// Few outputs (n <= 4, e.g. the 2-logit stop head): one warp per row of x; lane l covers k
// columns 4l + 128t and every output's dot product, so x is read once and all loads of a warp are
// in flight together. Weights are read before the dependency wait.
constexpr int NARROW_MAX_N = 4;
constexpr int NARROW_MAX_T = 8;  // k <= 1024 held in registers; longer k loops

__global__ void __launch_bounds__(256) gemv_narrow_kernel(LinearArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    const int T = a.k / 128;  // k % 128 == 0
    uint2 w[NARROW_MAX_N][NARROW_MAX_T];
    const bool fits = T <= NARROW_MAX_T;
    if (fits) {
#pragma unroll
        for (int j = 0; j < NARROW_MAX_N; j++)
#pragma unroll
            for (int t = 0; t < NARROW_MAX_T; t++)
                if (j < a.n && t < T) w[j][t] = *reinterpret_cast<const uint2*>(a.w + (size_t)j * a.k + 4 * lane + 128 * t);
    }
    pdl_wait();
    pdl_launch();
    if (row >= a.m) return;
    const float* x = a.x + (size_t)row * a.ldx;
    float acc[NARROW_MAX_N] = {0.f, 0.f, 0.f, 0.f};
    for (int t0 = 0; t0 < T; t0 += NARROW_MAX_T) {
        float4 xv[NARROW_MAX_T];
#pragma unroll
        for (int t = 0; t < NARROW_MAX_T; t++)
            if (t0 + t < T) xv[t] = *reinterpret_cast<const float4*>(x + 4 * lane + 128 * (t0 + t));
#pragma unroll
        for (int j = 0; j < NARROW_MAX_N; j++) {
            if (j >= a.n) break;
#pragma unroll
            for (int t = 0; t < NARROW_MAX_T; t++) {
                if (t0 + t < T) {
                    const uint2 wv = fits ? w[j][t]
                                          : *reinterpret_cast<const uint2*>(a.w + (size_t)j * a.k + 4 * lane + 128 * (t0 + t));
                    acc[j] += xv[t].x * bf16_lo(wv.x) + xv[t].y * bf16_hi(wv.x) + xv[t].z * bf16_lo(wv.y) +
                              xv[t].w * bf16_hi(wv.y);
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < NARROW_MAX_N; j++) acc[j] = warp_sum(acc[j]);
    if (lane >= a.n) return;
    float v = acc[0];
#pragma unroll
    for (int j = 1; j < NARROW_MAX_N; j++) if (lane == j) v = acc[j];
    if (a.flags & MT_LINEAR_BIAS) v += bf16f(a.bias[lane]);
    if (a.flags & MT_LINEAR_GELU) v = gelu_tanh(v);
    if (a.flags & MT_LINEAR_SILU) v = silu(v);
    float* yp = a.y + (size_t)row * a.ldy + lane;
    if (a.flags & MT_LINEAR_ACCUM) v += *yp;
    *yp = v;
}

void launch_gemv(const LinearArgs& a, cudaStream_t s) {
    if (a.n <= NARROW_MAX_N && a.k % 128 == 0 && !(a.flags & MT_LINEAR_SILU_GATE) && a.ldx % 4 == 0 && !a.norm_w && !a.y_hi) {
        launch_k(gemv_narrow_kernel, (a.m + 7) / 8, 256, 0, s, a);
        return;
    }
    const int G = gemv_group(a.k);
    const bool gated = (a.flags & MT_LINEAR_SILU_GATE) != 0;
    const int mr = a.m <= 1 ? 1 : a.m <= 2 ? 2 : a.m <= 4 ? 4 : 8;
    // Two plain rows stay on the column-group kernel (graph replay, weights from DRAM: W[4864x896]
    // 5.28 vs 5.83 us, W[896x4864] 5.52 vs 7.93 us); with a folded norm or an accumulating
    // epilogue the 2..8-row kernel wins at two rows too (config-2 pass at M = 2: 704 vs 765 us).
    const bool quad = mr > 2 || a.norm_w || (a.flags & MT_LINEAR_ACCUM);
    if (mr > 1 && quad && gemv_quad_fits(a, gated)) {
        switch (mr) {
            case 2: launch_gemv_quad<2>(a, gated, s); break;
            case 4: launch_gemv_quad<4>(a, gated, s); break;
            default: launch_gemv_quad<8>(a, gated, s); break;
        }
        return;
    }
    switch (mr) {
        case 1: launch_gemv_mr<1>(a, G, gated, s); break;
        case 2: launch_gemv_mr<2>(a, G, gated, s); break;
        case 4: launch_gemv_mr<4>(a, G, gated, s); break;
        default: launch_gemv_mr<8>(a, G, gated, s); break;
    }
}

}  // namespace mt

using namespace mt;

// Rows up to this many stay on CUDA cores: at these row counts the weight stream, not the
// multiply-adds, bounds the op, and the tensor-core route would pad the rows to its tile.
static const int kGemvMaxRows = 8;

extern "C" {

int mt_linear_route(int m, int n, int k) {
    (void)n;
    (void)k;
    return m <= kGemvMaxRows ? 0 : 1;
}

mt_status mt_linear(mt_ctx* ctx, void* stream, const float* x, int ldx, int m, const mt_bf16* w,
                    const mt_bf16* w2, const mt_bf16* bias, int n, int k, float* y, int ldy, uint32_t flags) {
    MT_REQUIRE(ctx, ctx && x && w && y, MT_ERR_ARG, "mt_linear: null argument");
    MT_REQUIRE(ctx, (flags & ~31u) == 0, MT_ERR_ARG, "mt_linear: unknown flag bits 0x%x", flags);
    MT_REQUIRE(ctx, !(flags & MT_LINEAR_SILU_GATE) || w2, MT_ERR_ARG, "mt_linear: SILU_GATE needs w2");
    MT_REQUIRE(ctx, !(flags & MT_LINEAR_BIAS) || bias, MT_ERR_ARG, "mt_linear: BIAS needs bias");
    MT_REQUIRE(ctx, m >= 0 && n > 0 && k > 0 && k % 8 == 0 && ldx >= k && ldy >= n && ldx % 4 == 0, MT_ERR_SHAPE,
               "mt_linear: m %d n %d k %d ldx %d ldy %d (need k %% 8 == 0, ldx %% 4 == 0)", m, n, k, ldx, ldy);
    MT_REQUIRE(ctx, ((uintptr_t)x & 15u) == 0 && ((uintptr_t)w & 15u) == 0 && (!w2 || ((uintptr_t)w2 & 15u) == 0),
               MT_ERR_ARG, "mt_linear: x, w, w2 need 16-byte alignment");
    if (m == 0) return MT_OK;
    cudaStream_t s = as_stream(stream);
    LinearArgs a{};
    a.x = x; a.ldx = ldx; a.m = m; a.n = n; a.k = k; a.w = w; a.w2 = w2; a.bias = bias;
    a.y = y; a.ldy = ldy; a.flags = flags; a.split_k = 1;
    if (mt_linear_route(m, n, k) == 0) {
        launch_gemv(a, s);
        return check_launch(ctx, "mt_linear (gemv)");
    }
    // Tensor-core route: split X into bf16 hi/lo planes in the context scratch, then the GEMM.
    void* buf = nullptr;
    const size_t plane = (size_t)m * k;
    mt_status st = mt::scratch(ctx, s, plane * 2 * sizeof(uint16_t), &buf);
    if (st != MT_OK) return st;
    uint16_t* hi = static_cast<uint16_t*>(buf);
    uint16_t* lo = hi + plane;
    launch_split(x, ldx, m, k, hi, lo, k, ctx->sm_count, s);
    st = check_launch(ctx, "mt_linear (split)");
    if (st != MT_OK) return st;
    a.x_hi = hi; a.x_lo = lo; a.ld_split = k;
    return launch_gemm_tc(ctx, a, s);
}

mt_status mt_linear_split(mt_ctx* ctx, void* stream, const mt_bf16* x_hi, const mt_bf16* x_lo, int ld_x, int m,
                          const mt_bf16* w, const mt_bf16* w2, const mt_bf16* bias, int n, int k, float* y, int ldy,
                          mt_bf16* y_hi, mt_bf16* y_lo, int ld_ysplit, uint32_t flags) {
    MT_REQUIRE(ctx, ctx && x_hi && x_lo && w && (y || (y_hi && y_lo)), MT_ERR_ARG, "mt_linear_split: null argument");
    MT_REQUIRE(ctx, (flags & ~31u) == 0, MT_ERR_ARG, "mt_linear_split: unknown flag bits 0x%x", flags);
    MT_REQUIRE(ctx, !(flags & MT_LINEAR_SILU_GATE) || w2, MT_ERR_ARG, "mt_linear_split: SILU_GATE needs w2");
    MT_REQUIRE(ctx, m >= 0 && n > 0 && k > 0 && k % 8 == 0 && ld_x >= k && (!y || ldy >= n) &&
                        (!y_hi || ld_ysplit >= n),
               MT_ERR_SHAPE, "mt_linear_split: m %d n %d k %d ld_x %d", m, n, k, ld_x);
    if (m == 0) return MT_OK;
    LinearArgs a{};
    a.x_hi = x_hi; a.x_lo = x_lo; a.ld_split = ld_x; a.m = m; a.n = n; a.k = k; a.w = w; a.w2 = w2; a.bias = bias;
    a.y = y; a.ldy = ldy; a.y_hi = y_hi; a.y_lo = y_lo; a.ld_ysplit = ld_ysplit; a.flags = flags; a.split_k = 1;
    return launch_gemm_tc(ctx, a, as_stream(stream));
}

}  // extern "C"
