// convdec.cu -- the 1-D convolutional waveform decoder of mingcuda.h (mt_convdec_*): latents ->
// 44.1 kHz mono through conv_in, four (SiLU -> transposed conv -> residual block) stages and a
// SiLU -> conv -> tanh head. It has no counterpart in the reference (whose decoder is the windowed
// Qwen stack + ISTFT of VAEDecoder.swift); the layer definitions are in the header.
//
// Every convolution but the last is an implicit GEMM on the tcgen05 tensor-core route
// (gemm_tc.cu): activations are time-major, channels-last rows with `kHalo` zero rows at both ends;
// output channels are the GEMM's weight rows, K = taps x input channels, and K column
// tap * C_in + c of time row t reads activation row t + tap - (taps - 1) / 2, channel c. A 64-wide
// K block lies inside one tap, so each stage of the GEMM pipeline is one TMA box of the activation
// planes at a shifted row. The residual stream is kept in fp32; each GEMM's epilogue also writes
// silu(its output) as the bf16 hi/lo planes the next convolution reads.
//
// A transposed convolution (stride s, kernel 2 s, padding s / 2) is one polyphase GEMM: output
// sample j s + r (phase r) is a sum over input frames j - 1, j, j + 1 with per-phase taps, so with
// weight rows (r, c_out) and a 3-frame window (K = 3 C_in; the one tap a phase does not use is zero)
// the GEMM's output row j holds samples j s .. j s + s - 1 -- exactly the upsampled channels-last
// layout of the next stage.
#include <math.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace mt {

namespace {

constexpr int kHalo = 4;  // zero rows before and after every activation buffer (>= the 3 of a 7-wide
                          // kernel, and a multiple of the frame groups below)

// Conv1d weight [co][ci][k] -> GEMM rows for G output frames per row: row g * co_n + co, column
// w * ci_n + ci over a window of G + k_n - 1 input frames, = weight[co][ci][w - g] (0 outside the
// kernel). G = 1 is the plain [co][k * ci_n + ci] layout.
__global__ void repack_conv_kernel(const uint16_t* __restrict__ w, int co_n, int ci_n, int k_n, int G,
                                   uint16_t* __restrict__ out) {
    const int win = G + k_n - 1;
    const long long total = (long long)G * co_n * win * ci_n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / ((long long)win * ci_n));
        const int col = (int)(i - (long long)row * win * ci_n);
        const int g = row / co_n, co = row - g * co_n;
        const int wi = col / ci_n, ci = col - wi * ci_n;
        const int k = wi - g;
        out[i] = (k >= 0 && k < k_n) ? w[((size_t)co * ci_n + ci) * k_n + k] : (uint16_t)0;
    }
}

// Output frames per GEMM row for a residual-block convolution of C channels: enough to fill the
// MMA's 128 weight rows when C is narrower.
int conv_group(int C) { return (C < 128 && 128 % C == 0 && kHalo % (128 / C) == 0) ? 128 / C : 1; }

// ConvTranspose1d weight [ci][co][2 s] (stride s, padding s / 2) -> polyphase GEMM rows
// [r * co_n + co][tap * ci_n + ci], tap 0/1/2 = input frame j - 1 / j / j + 1 of output sample
// j s + r: with q = r + s / 2, frame j uses kernel tap q, frame j - 1 tap q + s (when q < s) and
// frame j + 1 tap q - s (when q >= s); the bias of row (r, co) is b[co].
__global__ void repack_upconv_kernel(const uint16_t* __restrict__ w, const uint16_t* __restrict__ b, int ci_n, int co_n,
                                     int s, uint16_t* __restrict__ out, uint16_t* __restrict__ bias_out) {
    const long long total = (long long)s * co_n * 3 * ci_n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / (3LL * ci_n));
        const int col = (int)(i - (long long)row * 3 * ci_n);
        const int r = row / co_n, co = row - r * co_n;
        const int tap = col / ci_n, ci = col - tap * ci_n;
        const int q = r + s / 2;
        int k = -1;
        if (tap == 1) k = q;
        else if (tap == 0 && q < s) k = q + s;
        else if (tap == 2 && q >= s) k = q - s;
        out[i] = k >= 0 ? w[((size_t)ci * co_n + co) * (2 * s) + k] : (uint16_t)0;
        if (col == 0) bias_out[row] = b[co];
    }
}

// pcm[t] = tanh(b + sum_k d_k[t + k - (K - 1) / 2]) with d_k[r] = sum_c w[c][k] silu(x[r][c]) over
// channels-last fp32 x (rows outside [0, frames) read as zero, the convolution's padding; silu(0) =
// 0). A block gives each of its rows (its samples plus the kernel's reach) one thread that reads the
// row once (through L1) and forms all K tap sums, then one thread per sample adds K of them.
// (Staging the rows in shared memory with coalesced loads first measured slower: 106 vs 67 us.)
constexpr int kOutTile = 256;
constexpr int kOutMaxK = 7;
__global__ void __launch_bounds__(256) conv_out_tanh_kernel(const float* __restrict__ x_pad, int frames, int C, int K,
                                                            const uint16_t* __restrict__ w, const uint16_t* __restrict__ b,
                                                            float* __restrict__ pcm) {
    extern __shared__ float sm[];
    float* ws = sm;                               // [C][K]
    float* d = sm + (size_t)C * K;                // [kOutTile + K - 1][kOutMaxK]
    pdl_wait();
    const int t0 = blockIdx.x * kOutTile, half = (K - 1) / 2;
    const int rows = kOutTile + K - 1;
    for (int i = threadIdx.x; i < K * C; i += blockDim.x) ws[i] = bf16f(w[i]);  // [1][C][K] as [c][k]
    __syncthreads();
    for (int rr = threadIdx.x; rr < rows; rr += blockDim.x) {
        const int t = t0 + rr - half;  // time index of the row
        float acc[kOutMaxK];
#pragma unroll
        for (int k = 0; k < kOutMaxK; k++) acc[k] = 0.f;
        if (t >= 0 && t < frames) {
            const float4* xr = reinterpret_cast<const float4*>(x_pad + (size_t)(t + kHalo) * C);
            for (int c4 = 0; c4 < C / 4; c4++) {
                const float4 v = __ldg(xr + c4);
                const float sv[4] = {silu(v.x), silu(v.y), silu(v.z), silu(v.w)};
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const float* wr = ws + (size_t)(4 * c4 + u) * K;
#pragma unroll
                    for (int k = 0; k < kOutMaxK; k++)
                        if (k < K) acc[k] = fmaf(wr[k], sv[u], acc[k]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kOutMaxK; k++) d[(size_t)rr * kOutMaxK + k] = acc[k];
    }
    __syncthreads();
    pdl_launch();
    const int t = t0 + threadIdx.x;
    if (t >= frames) return;
    float out = bf16f(b[0]);
    for (int k = 0; k < K; k++) out += d[(size_t)(threadIdx.x + k) * kOutMaxK + k];
    pcm[t] = tanhf(out);
}

}  // namespace

}  // namespace mt

// One activation level: time-major rows of C channels after kHalo zero rows. A call with fewer rows
// than the buffer holds leaves older rows behind its last row; the GEMMs' tensor maps end at the
// last valid row (TMA reads zeros past it), so those rows act as zero padding all the same. `f` is the
// fp32 residual stream, (hi, lo) the bf16 planes of silu(f), (h_hi, h_lo) the planes of the
// residual block's inner activation.
struct ConvLevel {
    int C = 0, frames = 0;  // frames: the rows of the largest call (max_frames x upsampling so far)
    float* f = nullptr;
    uint16_t *hi = nullptr, *lo = nullptr, *h_hi = nullptr, *h_lo = nullptr;
};

struct mt_convdec {
    mt_ctx* ctx = nullptr;
    mt_convdec_config cfg{};
    int max_frames = 0;
    std::vector<void*> allocs;
    // GEMM-layout weights
    uint16_t *in_w = nullptr, *in_b = nullptr;
    uint16_t *up_w[4] = {}, *up_b[4] = {}, *a_w[4] = {}, *a_b[4] = {}, *b_w[4] = {}, *b_b[4] = {};
    int group[4] = {1, 1, 1, 1};  // output frames per GEMM row of stage i's residual-block convolutions
    uint16_t *out_w = nullptr, *out_b = nullptr;
    uint16_t *lat_hi = nullptr, *lat_lo = nullptr;  // latent planes [max_frames + 2 halo][latent_dim]
    ConvLevel lv[5];
    // plans of the last call's frame count
    int plan_frames = -1;
    mt::GemmPlan in_plan, up_plan[4], a_plan[4], b_plan[4];
};

using namespace mt;

namespace {

template <typename T>
mt_status cd_alloc(mt_convdec* d, T** p, size_t count) {
    *p = nullptr;
    if (count == 0) count = 1;
    if (cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)) != cudaSuccess) {
        *p = nullptr;
        return fail(d->ctx, MT_ERR_NOMEM, "mt_convdec: cudaMalloc of %zu bytes", count * sizeof(T));
    }
    d->allocs.push_back(*p);
    if (cudaMemset(*p, 0, count * sizeof(T)) != cudaSuccess)  // halo rows stay zero for good
        return fail(d->ctx, MT_ERR_CUDA, "mt_convdec: cudaMemset");
    return MT_OK;
}

#define CD_TRY(x)                     \
    do {                              \
        const mt_status st_ = (x);    \
        if (st_ != MT_OK) return st_; \
    } while (0)

bool config_ok(const mt_convdec_config& c) {
    if (c.latent_dim <= 0 || c.latent_dim % 64) return false;
    for (int i = 0; i < 5; i++)
        if (c.channels[i] <= 0 || c.channels[i] % 64) return false;
    for (int i = 0; i < 4; i++)
        if (c.strides[i] < 2 || c.strides[i] > 32 || c.strides[i] % 2) return false;
    return c.kernel >= 1 && c.kernel % 2 == 1 && c.kernel <= kOutMaxK && (c.kernel - 1) / 2 <= kHalo;
}

long long level_frames(const mt_convdec_config& c, int frames, int level) {
    long long t = frames;
    for (int i = 0; i < level; i++) t *= c.strides[i];
    return t;
}

void repack_conv(const uint16_t* w, int co, int ci, int k, int G, uint16_t* out) {
    const long long total = (long long)G * co * (G + k - 1) * ci;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148 * 16);
    repack_conv_kernel<<<blocks, 256>>>(w, co, ci, k, G, out);
}

// One implicit-GEMM convolution: `taps` frames of x (planes of C_in channels, rows = H + frames)
// centred on each output frame, into n output channels; G output frames per GEMM row (the planes
// viewed as rows of G frames: frames and kHalo are multiples of G).
LinearArgs conv_args(const uint16_t* x_hi, const uint16_t* x_lo, int c_in, int taps, int frames, int n,
                     const uint16_t* w, const uint16_t* bias, int G = 1) {
    LinearArgs a{};
    a.x_hi = x_hi;
    a.x_lo = x_lo;
    a.ld_split = G * c_in;
    a.conv_cin = c_in;
    a.conv_row0 = kHalo - (taps - 1) / 2;
    a.conv_group = G;
    a.x_rows = (kHalo + frames) / G;
    a.m = frames / G;
    a.n = G * n;
    a.k = (G + taps - 1) * c_in;
    a.w = w;
    a.bias = bias;
    a.flags = MT_LINEAR_BIAS;
    a.split_silu = 1;
    a.split_k = 1;
    return a;
}

mt_status build_plans(mt_convdec* d, int frames) {
    const mt_convdec_config& c = d->cfg;
    const int K = c.kernel, H = kHalo;
    {
        const int C0 = c.channels[0];
        LinearArgs a = conv_args(d->lat_hi, d->lat_lo, c.latent_dim, K, frames, C0, d->in_w, d->in_b);
        a.y = d->lv[0].f + (size_t)H * C0;
        a.ldy = C0;
        a.y_hi = d->lv[0].hi + (size_t)H * C0;
        a.y_lo = d->lv[0].lo + (size_t)H * C0;
        a.ld_ysplit = C0;
        CD_TRY(make_gemm_plan(d->ctx, a, &d->in_plan));
    }
    for (int i = 0; i < 4; i++) {
        const int ci = c.channels[i], co = c.channels[i + 1], s = c.strides[i];
        const int t_in = (int)level_frames(c, frames, i), t_out = (int)level_frames(c, frames, i + 1);
        ConvLevel& src = d->lv[i];
        ConvLevel& dst = d->lv[i + 1];
        // transposed convolution: rows j of the output hold samples j s .. j s + s - 1 of dst
        LinearArgs u = conv_args(src.hi, src.lo, ci, 3, t_in, s * co, d->up_w[i], d->up_b[i]);
        u.y = dst.f + (size_t)H * co;
        u.ldy = s * co;
        u.y_hi = dst.hi + (size_t)H * co;
        u.y_lo = dst.lo + (size_t)H * co;
        u.ld_ysplit = s * co;
        CD_TRY(make_gemm_plan(d->ctx, u, &d->up_plan[i]));
        // residual block: h = conv_a(silu(u)) (its planes hold silu(h)), u += conv_b(silu(h)); G
        // frames per GEMM row
        const int G = d->group[i];
        LinearArgs a = conv_args(dst.hi, dst.lo, co, K, t_out, co, d->a_w[i], d->a_b[i], G);
        a.y_hi = dst.h_hi + (size_t)H * co;
        a.y_lo = dst.h_lo + (size_t)H * co;
        a.ld_ysplit = G * co;
        CD_TRY(make_gemm_plan(d->ctx, a, &d->a_plan[i]));
        LinearArgs b = conv_args(dst.h_hi, dst.h_lo, co, K, t_out, co, d->b_w[i], d->b_b[i], G);
        b.flags |= MT_LINEAR_ACCUM;
        b.y = dst.f + (size_t)H * co;
        b.ldy = G * co;
        if (i < 3) {  // the next stage's transposed convolution reads silu(x); the head reads x itself
            b.y_hi = dst.hi + (size_t)H * co;
            b.y_lo = dst.lo + (size_t)H * co;
            b.ld_ysplit = G * co;
        } else {
            b.split_silu = 0;
        }
        CD_TRY(make_gemm_plan(d->ctx, b, &d->b_plan[i]));
    }
    d->plan_frames = frames;
    return MT_OK;
}

size_t out_smem(const mt_convdec_config& c) {
    return ((size_t)c.channels[4] * c.kernel + (size_t)(kOutTile + c.kernel - 1) * kOutMaxK) * sizeof(float);
}

}  // namespace

extern "C" long long mt_convdec_samples(const mt_convdec_config* cfg, int frames) {
    if (!cfg || frames < 0) return -1;
    return level_frames(*cfg, frames, 4);
}

extern "C" mt_status mt_convdec_create(mt_ctx* ctx, const mt_convdec_config* cfg, const mt_convdec_weights* w,
                                       int max_frames, mt_convdec** out) {
    MT_REQUIRE(ctx, ctx && cfg && w && out, MT_ERR_ARG, "mt_convdec_create: null argument");
    *out = nullptr;
    MT_REQUIRE(ctx, config_ok(*cfg), MT_ERR_SHAPE,
               "mt_convdec_create: latent_dim and channels must be multiples of 64, strides even (2..32), kernel odd "
               "(<= %d)", kOutMaxK);
    MT_REQUIRE(ctx, max_frames >= 1 && level_frames(*cfg, max_frames, 4) + 2 * kHalo < (1LL << 31), MT_ERR_CAPACITY,
               "mt_convdec_create: max_frames %d", max_frames);
    bool have = w->in_w && w->in_b && w->out_w && w->out_b;
    for (int i = 0; i < 4; i++) have = have && w->up_w[i] && w->up_b[i] && w->a_w[i] && w->a_b[i] && w->b_w[i] && w->b_b[i];
    MT_REQUIRE(ctx, have, MT_ERR_ARG, "mt_convdec_create: missing weight tensor");
    mt_convdec* d = new mt_convdec();
    d->ctx = ctx;
    d->cfg = *cfg;
    d->max_frames = max_frames;
    const mt_convdec_config& c = *cfg;
    const int K = c.kernel;
    auto cleanup = [&](mt_status st) {
        mt_convdec_destroy(d);
        return st;
    };
#define CD_ETRY(x)                              \
    do {                                        \
        const mt_status st_ = (x);              \
        if (st_ != MT_OK) return cleanup(st_);  \
    } while (0)
    // weights in GEMM layouts
    CD_ETRY(cd_alloc(d, &d->in_w, (size_t)c.channels[0] * K * c.latent_dim));
    CD_ETRY(cd_alloc(d, &d->in_b, (size_t)c.channels[0]));
    repack_conv(w->in_w, c.channels[0], c.latent_dim, K, 1, d->in_w);
    cudaMemcpy(d->in_b, w->in_b, sizeof(uint16_t) * c.channels[0], cudaMemcpyDefault);
    for (int i = 0; i < 4; i++) {
        const int ci = c.channels[i], co = c.channels[i + 1], s = c.strides[i];
        CD_ETRY(cd_alloc(d, &d->up_w[i], (size_t)s * co * 3 * ci));
        CD_ETRY(cd_alloc(d, &d->up_b[i], (size_t)s * co));
        const long long total = (long long)s * co * 3 * ci;
        repack_upconv_kernel<<<(int)std::min<long long>((total + 255) / 256, 148 * 16), 256>>>(w->up_w[i], w->up_b[i], ci,
                                                                                               co, s, d->up_w[i],
                                                                                               d->up_b[i]);
        // frame groups where every call's row count at this level divides (a product of strides)
        const int G = level_frames(c, 1, i + 1) % conv_group(co) == 0 ? conv_group(co) : 1;
        d->group[i] = G;
        CD_ETRY(cd_alloc(d, &d->a_w[i], (size_t)G * co * (G + K - 1) * co));
        CD_ETRY(cd_alloc(d, &d->a_b[i], (size_t)G * co));
        CD_ETRY(cd_alloc(d, &d->b_w[i], (size_t)G * co * (G + K - 1) * co));
        CD_ETRY(cd_alloc(d, &d->b_b[i], (size_t)G * co));
        repack_conv(w->a_w[i], co, co, K, G, d->a_w[i]);
        repack_conv(w->b_w[i], co, co, K, G, d->b_w[i]);
        for (int g = 0; g < G; g++) {  // the bias of output frame g of a row
            cudaMemcpy(d->a_b[i] + (size_t)g * co, w->a_b[i], sizeof(uint16_t) * co, cudaMemcpyDefault);
            cudaMemcpy(d->b_b[i] + (size_t)g * co, w->b_b[i], sizeof(uint16_t) * co, cudaMemcpyDefault);
        }
    }
    CD_ETRY(cd_alloc(d, &d->out_w, (size_t)c.channels[4] * K));
    CD_ETRY(cd_alloc(d, &d->out_b, 1));
    cudaMemcpy(d->out_w, w->out_w, sizeof(uint16_t) * c.channels[4] * K, cudaMemcpyDefault);  // [1][C4][K] as is
    cudaMemcpy(d->out_b, w->out_b, sizeof(uint16_t), cudaMemcpyDefault);
    // activation levels
    const size_t lat_rows = (size_t)max_frames + 2 * kHalo;
    CD_ETRY(cd_alloc(d, &d->lat_hi, lat_rows * c.latent_dim));
    CD_ETRY(cd_alloc(d, &d->lat_lo, lat_rows * c.latent_dim));
    for (int l = 0; l < 5; l++) {
        ConvLevel& L = d->lv[l];
        L.C = c.channels[l];
        L.frames = (int)level_frames(c, max_frames, l);
        const size_t n = ((size_t)L.frames + 2 * kHalo) * L.C;
        CD_ETRY(cd_alloc(d, &L.f, n));
        CD_ETRY(cd_alloc(d, &L.hi, n));
        CD_ETRY(cd_alloc(d, &L.lo, n));
        if (l > 0) {
            CD_ETRY(cd_alloc(d, &L.h_hi, n));
            CD_ETRY(cd_alloc(d, &L.h_lo, n));
        }
    }
    const cudaError_t sync = cudaDeviceSynchronize();
    if (sync != cudaSuccess) return cleanup(fail(ctx, MT_ERR_CUDA, "mt_convdec_create: %s", cudaGetErrorString(sync)));
    static PerDeviceOnce attr_once;
    attr_once([] {
        cudaFuncSetAttribute(conv_out_tanh_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    });
    MT_REQUIRE(ctx, out_smem(c) <= 200 * 1024, MT_ERR_SHAPE, "mt_convdec_create: C4 %d too wide for the head", c.channels[4]);
#undef CD_ETRY
    *out = d;
    return MT_OK;
}

extern "C" mt_status mt_convdec_decode(mt_convdec* d, void* stream, const float* latents, int frames, float* pcm) {
    if (!d) return MT_ERR_ARG;
    mt_ctx* ctx = d->ctx;
    MT_REQUIRE(ctx, latents && pcm, MT_ERR_ARG, "mt_convdec_decode: null argument");
    MT_REQUIRE(ctx, frames >= 1 && frames <= d->max_frames, MT_ERR_CAPACITY, "mt_convdec_decode: frames %d (1..%d)",
               frames, d->max_frames);
    MT_REQUIRE(ctx, ((uintptr_t)latents & 15u) == 0, MT_ERR_ARG, "mt_convdec_decode: latents need 16-byte alignment");
    const mt_convdec_config& c = d->cfg;
    cudaStream_t s = as_stream(stream);
    if (d->plan_frames != frames) CD_TRY(build_plans(d, frames));
    const int H = kHalo, L = c.latent_dim;
    launch_split(latents, L, frames, L, d->lat_hi + (size_t)H * L, d->lat_lo + (size_t)H * L, L, ctx->sm_count, s);
    run_gemm_plan(d->in_plan, s);
    for (int i = 0; i < 4; i++) {
        run_gemm_plan(d->up_plan[i], s);
        run_gemm_plan(d->a_plan[i], s);
        run_gemm_plan(d->b_plan[i], s);
    }
    const long long n = level_frames(c, frames, 4);
    launch_k(conv_out_tanh_kernel, dim3((unsigned)((n + kOutTile - 1) / kOutTile)), dim3(256), out_smem(c), s,
             d->lv[4].f, (int)n, c.channels[4], c.kernel, d->out_w, d->out_b, pcm);
    return check_launch(ctx, "mt_convdec_decode");
}

extern "C" void mt_convdec_destroy(mt_convdec* d) {
    if (!d) return;
    for (void* p : d->allocs) cudaFree(p);
    delete d;
}
