// istft.cu -- ISTFT frame synthesis and overlap-add emission of the streaming VAE decoder.
//
// Reference semantics: istft_frames / istft_emit (Shaders.swift:726-788), dispatch
// Encoder.istftFrames / istftEmit (Kernels.swift:260-281), counts VAEDecoder.decodeDispatches
// (VAEDecoder.swift:86-107). Spectrum rows hold [log-magnitude (N/2+1) | phase (N/2+1)];
// mag = min(exp(logmag), 100); frame = irfft(mag e^{i phase}) / N * window; output sample s is the
// overlap-add of the frames covering s + pad divided by the window^2 envelope, pad = (N - hop) / 2.
#include "common.cuh"
#include "kernels.cuh"

namespace mt {

constexpr int ISTFT_THREADS = 256;

// Direct path, for lengths whose half has a prime factor above 7. Block (tile of 256 output
// samples, frame f). The spectrum of the frame and a cosine table of N entries (cos(2 pi j / N),
// computed with cospif) sit in shared memory; each thread evaluates one output sample as the
// direct real inverse DFT, walking the table with index k*t mod N.
__global__ void __launch_bounds__(ISTFT_THREADS) istft_frames_kernel(IstftArgs a) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float sm[];
    const int N = a.nfft, bins = N / 2 + 1;
    float* re = sm;
    float* im = re + bins;
    float* ct = im + bins;
    const int f = blockIdx.y;
    const int req = f / a.frames_per_req;
    const float* row = a.spec + (size_t)f * a.ld_spec;
    for (int k = threadIdx.x; k < bins; k += blockDim.x) {
        const float mag = fminf(expf(row[k]), 100.0f);
        float s, c;
        sincosf(row[bins + k], &s, &c);
        re[k] = mag * c;
        im[k] = mag * s;
    }
    for (int j = threadIdx.x; j < N; j += blockDim.x) ct[j] = cospif(2.0f * (float)j / (float)N);
    __syncthreads();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= N) return;
    const int quarter3 = 3 * (N / 4);
    float acc = re[0] + ((t & 1) ? -re[N / 2] : re[N / 2]);
    float sum0 = 0.f, sum1 = 0.f;
    int idx = 0;
    int k = 1;
    for (; k + 1 < N / 2; k += 2) {
        idx += t;
        if (idx >= N) idx -= N;
        int sidx = idx + quarter3;
        if (sidx >= N) sidx -= N;
        sum0 += re[k] * ct[idx] - im[k] * ct[sidx];
        idx += t;
        if (idx >= N) idx -= N;
        sidx = idx + quarter3;
        if (sidx >= N) sidx -= N;
        sum1 += re[k + 1] * ct[idx] - im[k + 1] * ct[sidx];
    }
    for (; k < N / 2; k++) {
        idx += t;
        if (idx >= N) idx -= N;
        int sidx = idx + quarter3;
        if (sidx >= N) sidx -= N;
        sum0 += re[k] * ct[idx] - im[k] * ct[sidx];
    }
    acc += 2.0f * (sum0 + sum1);
    const int frame_index = a.frame0 + (a.frame0_dev ? a.frame0_dev[req] : 0) + f % a.frames_per_req;
    const int slot = frame_index % a.ring;
    a.frames[(size_t)req * a.req_stride + (size_t)slot * N + t] = acc / (float)N * a.window[t];
}

size_t istft_frames_smem(int nfft) { return sizeof(float) * ((size_t)(nfft / 2 + 1) * 2 + nfft); }

// ------------------------------------------------------------------------------------------------
// FFT path. The real inverse DFT of length N = 2M is one complex inverse DFT of length M:
//   Z[k] = E[k] + i O[k],  E = X[k] + conj(X[M-k]),  O = (X[k] - conj(X[M-k])) e^{i pi k / M},
//   z = sum_k Z[k] e^{2 pi i k n / M},  x[2n] = Re z[n] / N,  x[2n+1] = Im z[n] / N
// (X[0] and X[M] taken as real, as the direct sum does). The length-M transform is a Stockham
// autosort FFT in shared memory with radices 2, 3, 4, 5, 7 (M = 1764 = 4 * 3 * 3 * 7 * 7):
// stage with radix R and span Ns reads src[j + r M/R], twiddles by e^{2 pi i r (j % Ns) / (Ns R)},
// does an R-point DFT and writes dst[(j / Ns) Ns R + j % Ns + q Ns]. One block per frame.
// ------------------------------------------------------------------------------------------------
struct FftPlan {
    int M;
    int stages;
    int radix[16];
};

template <int R>
__device__ __forceinline__ void fft_stage(const float2* __restrict__ src, float2* __restrict__ dst, int M, int Ns,
                                          const float2* __restrict__ tw) {
    const int count = M / R, step = M / R;
    float2 wr[R];
#pragma unroll
    for (int q = 0; q < R; q++) wr[q] = tw[(q * (M / R)) % M];  // e^{2 pi i q / R}
    for (int j = threadIdx.x; j < count; j += blockDim.x) {
        const int k = j % Ns;
        const int tstride = M / (Ns * R);
        float2 v[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            float2 x = src[j + r * step];
            if (r > 0) {
                const float2 w = tw[(r * k * tstride) % M];
                x = make_float2(x.x * w.x - x.y * w.y, x.x * w.y + x.y * w.x);
            }
            v[r] = x;
        }
        const int base = (j / Ns) * Ns * R + k;
#pragma unroll
        for (int q = 0; q < R; q++) {
            float2 acc = v[0];
#pragma unroll
            for (int r = 1; r < R; r++) {
                const float2 w = wr[(r * q) % R];
                acc.x += v[r].x * w.x - v[r].y * w.y;
                acc.y += v[r].x * w.y + v[r].y * w.x;
            }
            dst[base + q * Ns] = acc;
        }
    }
}

__global__ void __launch_bounds__(ISTFT_THREADS) istft_fft_kernel(IstftArgs a, FftPlan p) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float2 sm2[];
    const int M = p.M, N = 2 * M;
    float2* xs = sm2;            // X[0..M]
    float2* b0 = xs + (M + 1);   // ping
    float2* b1 = b0 + M;         // pong
    float2* tw = b1 + M;         // e^{2 pi i j / M}
    const int f = blockIdx.x;
    const int req = f / a.frames_per_req;
    const float* row = a.spec + (size_t)f * a.ld_spec;
    for (int k = threadIdx.x; k <= M; k += blockDim.x) {
        const float mag = fminf(expf(row[k]), 100.0f);
        float s, c;
        sincosf(row[M + 1 + k], &s, &c);
        xs[k] = (k == 0 || k == M) ? make_float2(mag * c, 0.f) : make_float2(mag * c, mag * s);
    }
    for (int j = threadIdx.x; j < M; j += blockDim.x) {
        float s, c;
        sincospif(2.0f * (float)j / (float)M, &s, &c);
        tw[j] = make_float2(c, s);
    }
    __syncthreads();
    for (int k = threadIdx.x; k < M; k += blockDim.x) {
        const float2 x = xs[k], y = xs[M - k];
        const float2 e = make_float2(x.x + y.x, x.y - y.y);       // X[k] + conj(X[M-k])
        const float2 d = make_float2(x.x - y.x, x.y + y.y);       // X[k] - conj(X[M-k])
        float s, c;
        sincospif((float)k / (float)M, &s, &c);                   // e^{i pi k / M}
        const float2 o = make_float2(d.x * c - d.y * s, d.x * s + d.y * c);
        b0[k] = make_float2(e.x - o.y, e.y + o.x);                // E + i O
    }
    __syncthreads();
    float2* src = b0;
    float2* dst = b1;
    int Ns = 1;
    for (int st = 0; st < p.stages; st++) {
        const int R = p.radix[st];
        if (R == 4) fft_stage<4>(src, dst, M, Ns, tw);
        else if (R == 2) fft_stage<2>(src, dst, M, Ns, tw);
        else if (R == 3) fft_stage<3>(src, dst, M, Ns, tw);
        else if (R == 5) fft_stage<5>(src, dst, M, Ns, tw);
        else fft_stage<7>(src, dst, M, Ns, tw);
        __syncthreads();
        float2* t = src;
        src = dst;
        dst = t;
        Ns *= R;
    }
    const int frame_index = a.frame0 + (a.frame0_dev ? a.frame0_dev[req] : 0) + f % a.frames_per_req;
    const int slot = frame_index % a.ring;
    float* out = a.frames + (size_t)req * a.req_stride + (size_t)slot * N;
    const float inv = 1.0f / (float)N;
    for (int n = threadIdx.x; n < M; n += blockDim.x) {
        const float2 z = src[n];
        out[2 * n] = z.x * inv * a.window[2 * n];
        out[2 * n + 1] = z.y * inv * a.window[2 * n + 1];
    }
}

// Radices of M from {4, 2, 3, 5, 7} (largest power-of-two part as 4s); false if another prime divides M.
static bool fft_plan(int M, FftPlan* p) {
    p->M = M;
    p->stages = 0;
    int m = M;
    while (m % 4 == 0 && p->stages < 16) { p->radix[p->stages++] = 4; m /= 4; }
    for (int r : {2, 3, 5, 7})
        while (m % r == 0 && p->stages < 16) { p->radix[p->stages++] = r; m /= r; }
    return m == 1;
}

static size_t istft_fft_smem(int M) { return sizeof(float2) * ((size_t)(M + 1) + 3 * (size_t)M); }

void launch_istft_frames(const IstftArgs& a, cudaStream_t s) {
    FftPlan p;
    const int M = a.nfft / 2;
    const size_t fsmem = istft_fft_smem(M);
    if (fft_plan(M, &p) && fsmem <= 200 * 1024) {
        if (fsmem > 48 * 1024)
            cudaFuncSetAttribute(istft_fft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem);
        launch_k(istft_fft_kernel, a.count, ISTFT_THREADS, fsmem, s, a, p);
        return;
    }
    const size_t smem = istft_frames_smem(a.nfft);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(istft_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_k(istft_frames_kernel, dim3((a.nfft + ISTFT_THREADS - 1) / ISTFT_THREADS, a.count), ISTFT_THREADS, smem, s, a);
}

// One thread per output sample; request r = blockIdx.y emits count samples starting at its s0.
__global__ void istft_emit_kernel(EmitArgs a) {
    pdl_wait();
    pdl_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int req = blockIdx.y;
    const int count = a.count_dev ? a.count_dev[req] : a.count;
    if (i >= count) return;
    const int s0 = a.s0 + (a.s0_dev ? a.s0_dev[req] : 0);
    const int last = a.last_frame + (a.last_dev ? a.last_dev[req] : 0);
    const int pad = (a.nfft - a.hop) / 2;
    const int s = s0 + i + pad;
    const int fHi = min(s / a.hop, last);
    const int fLo = (s >= a.nfft) ? (s - a.nfft) / a.hop + 1 : 0;
    const float* frames = a.frames + (size_t)req * a.req_stride;
    float acc = 0.f, env = 0.f;
    for (int f = fLo; f <= fHi; f++) {
        const int t = s - f * a.hop;
        if (t >= a.nfft) continue;
        const float w = a.window[t];
        acc += frames[(size_t)(f % a.ring) * a.nfft + t];
        env += w * w;
    }
    a.out[(size_t)req * a.ld_out + i] = acc / env;
}

void launch_istft_emit(const EmitArgs& a, int max_count, int requests, cudaStream_t s) {
    if (max_count <= 0 || requests <= 0) return;
    launch_k(istft_emit_kernel, dim3((max_count + 255) / 256, requests), 256, 0, s, a);
}

}  // namespace mt

using namespace mt;

extern "C" {

mt_status mt_istft_frames(mt_ctx* ctx, void* stream, const float* spec, int ld_spec, int count, int nfft,
                          const float* cos_table, const float* window, float* frames, int frame0, int ring) {
    (void)cos_table;
    MT_REQUIRE(ctx, ctx && spec && window && frames, MT_ERR_ARG, "mt_istft_frames: null argument");
    MT_REQUIRE(ctx, nfft > 0 && nfft % 4 == 0 && ld_spec >= nfft + 2 && count >= 0 && ring > 0 && frame0 >= 0,
               MT_ERR_SHAPE, "mt_istft_frames: nfft %d ld_spec %d count %d ring %d", nfft, ld_spec, count, ring);
    MT_REQUIRE(ctx, istft_frames_smem(nfft) <= 200 * 1024, MT_ERR_SHAPE, "mt_istft_frames: nfft %d too large", nfft);
    if (count == 0) return MT_OK;
    IstftArgs a{};
    a.spec = spec; a.ld_spec = ld_spec; a.count = count; a.nfft = nfft; a.window = window; a.frames = frames;
    a.frame0 = frame0; a.ring = ring; a.frames_per_req = count; a.req_stride = 0;
    launch_istft_frames(a, as_stream(stream));
    return check_launch(ctx, "mt_istft_frames");
}

mt_status mt_istft_emit(mt_ctx* ctx, void* stream, const float* frames, const float* window, int nfft, int hop,
                        int s0, int count, int last_frame, int ring, float* out) {
    MT_REQUIRE(ctx, ctx && frames && window && out, MT_ERR_ARG, "mt_istft_emit: null argument");
    MT_REQUIRE(ctx, nfft > 0 && hop > 0 && hop <= nfft && (nfft - hop) % 2 == 0 && s0 >= 0 && count >= 0 &&
                        last_frame >= 0 && ring > 0,
               MT_ERR_SHAPE, "mt_istft_emit: nfft %d hop %d s0 %d count %d", nfft, hop, s0, count);
    if (count == 0) return MT_OK;
    EmitArgs a{};
    a.frames = frames; a.window = window; a.nfft = nfft; a.hop = hop; a.s0 = s0; a.count = count;
    a.last_frame = last_frame; a.ring = ring; a.out = out; a.ld_out = count; a.req_stride = 0;
    launch_istft_emit(a, count, 1, as_stream(stream));
    return check_launch(ctx, "mt_istft_emit");
}

}  // extern "C"
