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
