// ops.cu -- element-wise, normalisation and attention kernels, and their C-ABI entry points.
//
// Reference kernels restated (semantics, not code): rmsnorm / copy_rows (Shaders.swift:418-447),
// rope_cache (Shaders.swift:456-486), attention_cache (Shaders.swift:500-591), dit_attention
// (Shaders.swift:613-648), flow_assemble / flow_euler (Shaders.swift:654-693), upsample4
// (Shaders.swift:704-719).
#include "common.cuh"
#include "kernels.cuh"

namespace mt {

// ------------------------------------------------------------------------------------------------
// RMSNorm: one block per row; each thread keeps its float4s of the row in registers, so the row
// is read once; optional fp32 and/or bf16 hi/lo outputs.
// ------------------------------------------------------------------------------------------------
constexpr int RMS_THREADS = 128;
constexpr int RMS_MAXV = 8;  // float4 per thread: width <= 4096

__global__ void __launch_bounds__(RMS_THREADS) rmsnorm_kernel(RmsArgs a) {
    pdl_wait();
    pdl_launch();
    __shared__ float part[RMS_THREADS / 32];
    const int row = blockIdx.x;
    const int n4 = a.width >> 2;
    const float4* x = reinterpret_cast<const float4*>(a.x + (size_t)row * a.ldx);
    float4 v[RMS_MAXV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < RMS_MAXV; i++) {
        const int c = threadIdx.x + i * RMS_THREADS;
        v[i] = c < n4 ? x[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < RMS_THREADS / 32; w++) tot += part[w];
    const float scale = rsqrtf(tot / (float)a.width + a.eps);
    const uint2* w = reinterpret_cast<const uint2*>(a.w);
#pragma unroll
    for (int i = 0; i < RMS_MAXV; i++) {
        const int c = threadIdx.x + i * RMS_THREADS;
        if (c >= n4) break;
        const uint2 wv = w[c];
        float4 o;
        o.x = v[i].x * scale * bf16_lo(wv.x);
        o.y = v[i].y * scale * bf16_hi(wv.x);
        o.z = v[i].z * scale * bf16_lo(wv.y);
        o.w = v[i].w * scale * bf16_hi(wv.y);
        if (a.y) reinterpret_cast<float4*>(a.y + (size_t)row * a.ldy)[c] = o;
        if (a.y_hi) {
            uint16_t h[4], l[4];
            split_bf16(o.x, h[0], l[0]);
            split_bf16(o.y, h[1], l[1]);
            split_bf16(o.z, h[2], l[2]);
            split_bf16(o.w, h[3], l[3]);
            reinterpret_cast<uint2*>(a.y_hi + (size_t)row * a.ld_split)[c] =
                make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
            reinterpret_cast<uint2*>(a.y_lo + (size_t)row * a.ld_split)[c] =
                make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
        }
    }
}

void launch_rmsnorm(const RmsArgs& a, cudaStream_t s) { launch_k(rmsnorm_kernel, a.rows, RMS_THREADS, 0, s, a); }

// fp32 [rows, cols] (row stride ldx) -> bf16 hi/lo planes [rows, cols] (row stride ld_split).
__global__ void split_kernel(const float* __restrict__ x, int ldx, int rows, int cols,
                             uint16_t* __restrict__ hi, uint16_t* __restrict__ lo, int ld_split) {
    pdl_wait();
    pdl_launch();
    const int c4 = cols >> 2;
    const long long total = (long long)rows * c4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / c4), c = (int)(i % c4);
        const float4 v = reinterpret_cast<const float4*>(x + (size_t)r * ldx)[c];
        uint16_t h[4], l[4];
        split_bf16(v.x, h[0], l[0]);
        split_bf16(v.y, h[1], l[1]);
        split_bf16(v.z, h[2], l[2]);
        split_bf16(v.w, h[3], l[3]);
        reinterpret_cast<uint2*>(hi + (size_t)r * ld_split)[c] =
            make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
        reinterpret_cast<uint2*>(lo + (size_t)r * ld_split)[c] =
            make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
    }
}

void launch_split(const float* x, int ldx, int rows, int cols, uint16_t* hi, uint16_t* lo,
                  int ld_split, int sm_count, cudaStream_t s) {
    long long total = (long long)rows * (cols / 4);
    long long blocks = (total + 255) / 256;
    if (blocks > sm_count * 8LL) blocks = sm_count * 8LL;
    if (blocks < 1) blocks = 1;
    launch_k(split_kernel, (unsigned)blocks, 256, 0, s, x, ldx, rows, cols, hi, lo, ld_split);
}

__global__ void copy_kernel(const float* __restrict__ x, int count, float* __restrict__ y) {
    pdl_wait();
    pdl_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) y[i] = x[i];
}

// ------------------------------------------------------------------------------------------------
// NeoX RoPE + KV append. Block = one query row, thread (slot, i): slot over q, k, v heads,
// i over the 32 rotation pairs. Requests: row m belongs to request m / rows_per_req, whose caches
// start at kc/vc + request * req_stride and whose first position is pos0 (+ pos_dev[request]).
// ------------------------------------------------------------------------------------------------
__global__ void rope_cache_kernel(RopeArgs a) {
    pdl_wait();
    pdl_launch();
    const int m = blockIdx.x;
    const int slot = threadIdx.x >> 5, i = threadIdx.x & 31;
    if (slot >= a.hq + 2 * a.hkv) return;
    const int req = m / a.rows_per_req;
    const int pos = a.pos0 + (a.pos_dev ? a.pos_dev[req] : 0) + (m % a.rows_per_req);
    const int cslot = pos % a.cap;
    float* row = a.qkv + (size_t)m * a.ldq + slot * 64;
    float* kc = a.kc + (size_t)req * a.req_stride;
    float* vc = a.vc + (size_t)req * a.req_stride;
    if (slot >= a.hq + a.hkv) {
        float* dst = vc + ((size_t)(slot - a.hq - a.hkv) * a.cap + cslot) * 64;
        dst[i] = row[i];
        dst[i + 32] = row[i + 32];
        return;
    }
    const float angle = (float)pos * a.inv_freq[i];
    float s, c;
    sincosf(angle, &s, &c);
    const float x0 = row[i], x1 = row[i + 32];
    const float r0 = x0 * c - x1 * s;
    const float r1 = x1 * c + x0 * s;
    if (slot < a.hq) {
        row[i] = r0;
        row[i + 32] = r1;
    } else {
        float* dst = kc + ((size_t)(slot - a.hq) * a.cap + cslot) * 64;
        dst[i] = r0;
        dst[i + 32] = r1;
    }
}

void launch_rope_cache(const RopeArgs& a, cudaStream_t s) {
    launch_k(rope_cache_kernel, a.rows, (a.hq + 2 * a.hkv) * 32, 0, s, a);
}

// ------------------------------------------------------------------------------------------------
// Causal GQA attention over the fp32 cache. One block per (query row, kv head): the G = hq / hkv
// query heads of the group share every K and V load. Keys are staged through shared memory in
// chunks of 64; scores for all keys live in shared memory (two-pass softmax), then P.V.
// ------------------------------------------------------------------------------------------------
constexpr int ATT_THREADS = 256;
constexpr int ATT_CHUNK = 64;

__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(AttnArgs a) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float smem[];
    const int m = blockIdx.x, kvh = blockIdx.y;
    const int G = a.hq / a.hkv;
    const int req = m / a.rows_per_req;
    const int qpos = a.pos0 + (a.pos_dev ? a.pos_dev[req] : 0) + (m % a.rows_per_req);
    const int jEnd = qpos + 1;
    const int jStart = (a.window > 0 && jEnd > a.window) ? jEnd - a.window : 0;
    const int nKeys = jEnd - jStart;
    const float* kc = a.kc + (size_t)req * a.req_stride + (size_t)kvh * a.cap * 64;
    const float* vc = a.vc + (size_t)req * a.req_stride + (size_t)kvh * a.cap * 64;

    float* qs = smem;                       // [G][64]
    float* ks = qs + G * 64;                // [ATT_CHUNK][65]  K chunk, then V chunk [ATT_CHUNK][64]
    float* sc = ks + ATT_CHUNK * 65;        // [G][max_keys]
    float* red = sc + (size_t)G * a.max_keys;  // [G]
    const int tid = threadIdx.x;
    for (int i = tid; i < G * 64; i += ATT_THREADS)
        qs[i] = a.q[(size_t)m * a.ldq + (kvh * G + i / 64) * 64 + (i % 64)];

    // Scores, 64 keys at a time: K rows staged coalesced, one (key, head) dot per thread.
    for (int c0 = 0; c0 < nKeys; c0 += ATT_CHUNK) {
        const int cn = min(ATT_CHUNK, nKeys - c0);
        __syncthreads();
        for (int i = tid; i < cn * 16; i += ATT_THREADS) {
            const int kk = i >> 4, d4 = i & 15;
            const int slot = (jStart + c0 + kk) % a.cap;
            const float4 v = reinterpret_cast<const float4*>(kc + (size_t)slot * 64)[d4];
            float* dst = ks + kk * 65 + d4 * 4;
            dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
        }
        __syncthreads();
        for (int i = tid; i < cn * G; i += ATT_THREADS) {
            const int kk = i % cn, g = i / cn;
            const float* qg = qs + g * 64;
            const float* kr = ks + kk * 65;
            float s = 0.f;
#pragma unroll 16
            for (int d = 0; d < 64; d++) s += qg[d] * kr[d];
            sc[(size_t)g * a.max_keys + c0 + kk] = s * 0.125f;
        }
    }
    __syncthreads();
    // Softmax per head: warp g handles head g (G <= 8 warps); scores become unnormalised weights.
    const int warp = tid >> 5, lane = tid & 31;
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
        float* sg = sc + (size_t)g * a.max_keys;
        float mx = -INFINITY;
        for (int j = lane; j < nKeys; j += 32) mx = fmaxf(mx, sg[j]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int j = lane; j < nKeys; j += 32) {
            const float e = expf(sg[j] - mx);
            sg[j] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0) red[g] = 1.0f / sum;
    }
    // P.V, 64 keys at a time: V rows staged coalesced in shared memory; thread (g, d) keeps its
    // output(s) in registers across chunks.
    const int outs = G * 64;
    float acc0 = 0.f, acc1 = 0.f;
    const int o0 = tid, o1 = tid + ATT_THREADS;
    for (int c0 = 0; c0 < nKeys; c0 += ATT_CHUNK) {
        const int cn = min(ATT_CHUNK, nKeys - c0);
        __syncthreads();
        for (int i = tid; i < cn * 16; i += ATT_THREADS) {
            const int kk = i >> 4, d4 = i & 15;
            const int slot = (jStart + c0 + kk) % a.cap;
            reinterpret_cast<float4*>(ks + kk * 64)[d4] = reinterpret_cast<const float4*>(vc + (size_t)slot * 64)[d4];
        }
        __syncthreads();
        if (o0 < outs) {
            const float* sg = sc + (size_t)(o0 / 64) * a.max_keys + c0;
            const int d = o0 % 64;
            for (int kk = 0; kk < cn; kk++) acc0 += sg[kk] * ks[kk * 64 + d];
        }
        if (o1 < outs) {
            const float* sg = sc + (size_t)(o1 / 64) * a.max_keys + c0;
            const int d = o1 % 64;
            for (int kk = 0; kk < cn; kk++) acc1 += sg[kk] * ks[kk * 64 + d];
        }
    }
    for (int t = 0; t < 2; t++) {
        const int o = t == 0 ? o0 : o1;
        if (o >= outs) continue;
        const int g = o / 64, d = o % 64;
        const float val = (t == 0 ? acc0 : acc1) * red[g];
        const size_t off = (size_t)m * a.ldo + (kvh * G + g) * 64 + d;
        if (a.out) a.out[off] = val;
        if (a.out_hi) {
            uint16_t h, l;
            split_bf16(val, h, l);
            const size_t so = (size_t)m * a.ld_split + (kvh * G + g) * 64 + d;
            a.out_hi[so] = h;
            a.out_lo[so] = l;
        }
    }
}

size_t attention_smem(int G, int max_keys) {
    return sizeof(float) * ((size_t)G * 64 + ATT_CHUNK * 65 + (size_t)G * max_keys + (size_t)G);
}

void launch_attention(const AttnArgs& a, cudaStream_t s) {
    const int G = a.hq / a.hkv;
    const size_t smem = attention_smem(G, a.max_keys);
    static bool configured = false;  // set once, before any graph capture (the first call is eager)
    if (!configured) {
        cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        configured = true;
    }
    launch_k(attention_kernel, dim3(a.rows, a.hkv), ATT_THREADS, smem, s, a);
}

// ------------------------------------------------------------------------------------------------
// DiT attention: one warp per (sequence, head) computes every row of the sequence (seq <= 8);
// lane l owns dims 2l, 2l+1 = one interleaved RoPE pair. All q/k/v loads of the warp are issued
// before any use, and each position's rotation is computed once.
// ------------------------------------------------------------------------------------------------
constexpr int DIT_MAX_SEQ = 8;

__global__ void dit_attention_kernel(DitAttnArgs a) {
    pdl_wait();
    pdl_launch();
    const int work = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (work >= a.batch * a.heads) return;
    const int h = work % a.heads, b = work / a.heads;
    const int D = a.heads * 64, S = a.seq;
    const float freq = a.inv_freq[lane];
    const float* rows = a.qkv + (size_t)b * S * a.ld + h * 64 + 2 * lane;
    float2 q[DIT_MAX_SEQ], k[DIT_MAX_SEQ], v[DIT_MAX_SEQ];
#pragma unroll
    for (int j = 0; j < DIT_MAX_SEQ; j++) {
        if (j < S) {
            q[j] = *reinterpret_cast<const float2*>(rows + (size_t)j * a.ld);
            k[j] = *reinterpret_cast<const float2*>(rows + (size_t)j * a.ld + D);
            v[j] = *reinterpret_cast<const float2*>(rows + (size_t)j * a.ld + 2 * D);
        }
    }
#pragma unroll
    for (int j = 0; j < DIT_MAX_SEQ; j++) {  // rotate q and k of position j
        if (j < S) {
            float sj, cj;
            sincosf((float)j * freq, &sj, &cj);
            q[j] = make_float2(q[j].x * cj - q[j].y * sj, q[j].y * cj + q[j].x * sj);
            k[j] = make_float2(k[j].x * cj - k[j].y * sj, k[j].y * cj + k[j].x * sj);
        }
    }
#pragma unroll
    for (int i = 0; i < DIT_MAX_SEQ; i++) {
        if (i >= S) break;
        float sc[DIT_MAX_SEQ];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < DIT_MAX_SEQ; j++) {
            if (j < S) {
                sc[j] = warp_sum(q[i].x * k[j].x + q[i].y * k[j].y) * 0.125f;
                mx = fmaxf(mx, sc[j]);
            }
        }
        float sum = 0.f, acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int j = 0; j < DIT_MAX_SEQ; j++) {
            if (j < S) {
                const float e = expf(sc[j] - mx);
                sum += e;
                acc0 += e * v[j].x;
                acc1 += e * v[j].y;
            }
        }
        const float o0 = acc0 / sum, o1 = acc1 / sum;
        const size_t row = (size_t)(b * S + i);
        if (a.out) *reinterpret_cast<float2*>(a.out + row * a.ldo + h * 64 + 2 * lane) = make_float2(o0, o1);
        if (a.out_hi) {
            uint16_t h0, l0, h1, l1;
            split_bf16(o0, h0, l0);
            split_bf16(o1, h1, l1);
            const size_t so = row * a.ld_split + h * 64 + 2 * lane;
            *reinterpret_cast<uint32_t*>(a.out_hi + so) = h0 | ((uint32_t)h1 << 16);
            *reinterpret_cast<uint32_t*>(a.out_lo + so) = l0 | ((uint32_t)l1 << 16);
        }
    }
}

void launch_dit_attention(const DitAttnArgs& a, cudaStream_t s) {
    const int work = a.batch * a.heads;
    launch_k(dit_attention_kernel, (work + 7) / 8, 256, 0, s, a);
}

// ------------------------------------------------------------------------------------------------
// Flow pieces.
// ------------------------------------------------------------------------------------------------
__global__ void flow_assemble_kernel(const float* __restrict__ y, const float* __restrict__ history,
                                     const float* __restrict__ cemb, const uint16_t* __restrict__ cbias,
                                     const float* __restrict__ temb, const uint16_t* __restrict__ xw,
                                     const uint16_t* __restrict__ xb, int hidden, int latent,
                                     float* __restrict__ x) {
    pdl_wait();
    pdl_launch();
    const int c = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
    if (c >= hidden) return;
    const int s = r % 3;
    float v;
    if (s == 0) {
        v = temb[c] + (r < 3 ? cemb[c] : bf16f(cbias[c]));
    } else {
        const float* src = (s == 1) ? history : y;
        const uint16_t* w = xw + (size_t)c * latent;
        float acc = 0.f;
        for (int d = 0; d < latent; d++) acc += bf16f(w[d]) * src[d];
        v = bf16f(xb[c]) + acc;
    }
    x[(size_t)r * hidden + c] = v;
}

__global__ void flow_euler_kernel(float* __restrict__ y, const float* __restrict__ pred, int ldp,
                                  int pred_row, int null_row, int latent, float cfg, float dt,
                                  float* __restrict__ capture) {
    pdl_wait();
    pdl_launch();
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= latent) return;
    const float c = pred[(size_t)pred_row * ldp + d];
    const float u = pred[(size_t)null_row * ldp + d];
    if (capture) {
        capture[d] = c;
        capture[latent + d] = u;
    }
    y[d] += (c + (c - u) * cfg) * dt;
}

__global__ void upsample4_kernel(const float* __restrict__ prev, const float* __restrict__ cur,
                                 const float* __restrict__ next, int hidden, float* __restrict__ frames) {
    pdl_wait();
    pdl_launch();
    const int c = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
    if (c >= hidden) return;
    const float v0 = cur[c];
    float v;
    if (r == 0) v = prev ? 0.625f * v0 + 0.375f * prev[c] : v0;
    else if (r == 1) v = prev ? 0.875f * v0 + 0.125f * prev[c] : v0;
    else if (r == 2) v = next ? 0.875f * v0 + 0.125f * next[c] : v0;
    else v = next ? 0.625f * v0 + 0.375f * next[c] : v0;
    frames[(size_t)r * hidden + c] = v;
}

}  // namespace mt

// ------------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------------
using namespace mt;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" {

mt_status mt_rmsnorm(mt_ctx* ctx, void* stream, const float* x, int ldx, int rows, int width,
                     const mt_bf16* w, float* y, int ldy, float eps) {
    MT_REQUIRE(ctx, ctx && x && w && y, MT_ERR_ARG, "mt_rmsnorm: null argument");
    MT_REQUIRE(ctx, rows >= 0 && width > 0 && width % 4 == 0 && width <= 4096 && ldx % 4 == 0 && ldy % 4 == 0 &&
                        ldx >= width && ldy >= width,
               MT_ERR_SHAPE, "mt_rmsnorm: width %d ldx %d ldy %d (need width %% 4 == 0, width <= 4096, ld >= width, ld %% 4 == 0)",
               width, ldx, ldy);
    MT_REQUIRE(ctx, aligned16(x) && aligned16(y) && ((uintptr_t)w & 7u) == 0, MT_ERR_ARG,
               "mt_rmsnorm: x/y need 16-byte, w 8-byte alignment");
    if (rows == 0) return MT_OK;
    RmsArgs a{};
    a.x = x; a.ldx = ldx; a.rows = rows; a.width = width; a.w = w; a.y = y; a.ldy = ldy; a.eps = eps;
    launch_rmsnorm(a, as_stream(stream));
    return check_launch(ctx, "mt_rmsnorm");
}

mt_status mt_copy(mt_ctx* ctx, void* stream, const float* x, int count, float* y) {
    MT_REQUIRE(ctx, ctx && x && y, MT_ERR_ARG, "mt_copy: null argument");
    MT_REQUIRE(ctx, count >= 0, MT_ERR_SHAPE, "mt_copy: count %d", count);
    if (count == 0) return MT_OK;
    int blocks = (count + 255) / 256;
    if (blocks > 1024) blocks = 1024;
    launch_k(copy_kernel, blocks, 256, 0, as_stream(stream), x, count, y);
    return check_launch(ctx, "mt_copy");
}

mt_status mt_rope_cache(mt_ctx* ctx, void* stream, float* qkv, int ldq, int m, int hq, int hkv,
                        int pos0, float* k_cache, float* v_cache, int capacity, const float* inv_freq) {
    MT_REQUIRE(ctx, ctx && qkv && k_cache && v_cache && inv_freq, MT_ERR_ARG, "mt_rope_cache: null argument");
    MT_REQUIRE(ctx, m >= 0 && hq > 0 && hkv > 0 && hq % hkv == 0 && hq + 2 * hkv <= 32 && ldq >= (hq + 2 * hkv) * 64,
               MT_ERR_SHAPE, "mt_rope_cache: hq %d hkv %d ldq %d", hq, hkv, ldq);
    MT_REQUIRE(ctx, pos0 >= 0 && capacity > 0 && pos0 + m <= capacity, MT_ERR_CAPACITY,
               "mt_rope_cache: positions %d..%d exceed capacity %d", pos0, pos0 + m, capacity);
    if (m == 0) return MT_OK;
    RopeArgs a{};
    a.qkv = qkv; a.ldq = ldq; a.rows = m; a.rows_per_req = m; a.hq = hq; a.hkv = hkv; a.pos0 = pos0;
    a.kc = k_cache; a.vc = v_cache; a.cap = capacity; a.inv_freq = inv_freq;
    launch_rope_cache(a, as_stream(stream));
    return check_launch(ctx, "mt_rope_cache");
}

mt_status mt_attention(mt_ctx* ctx, void* stream, const float* q, int ldq, int m, int hq, int hkv,
                       int pos0, int window, const float* k_cache, const float* v_cache, int capacity,
                       float* out, int ldo) {
    MT_REQUIRE(ctx, ctx && q && k_cache && v_cache && out, MT_ERR_ARG, "mt_attention: null argument");
    MT_REQUIRE(ctx, m >= 0 && hq > 0 && hkv > 0 && hq % hkv == 0 && hq / hkv <= 8 && ldq >= hq * 64 && ldo >= hq * 64 &&
                        window >= 0 && ldq % 4 == 0,
               MT_ERR_SHAPE, "mt_attention: hq %d hkv %d ldq %d ldo %d window %d", hq, hkv, ldq, ldo, window);
    MT_REQUIRE(ctx, pos0 >= 0 && capacity > 0 && pos0 + m <= capacity, MT_ERR_CAPACITY,
               "mt_attention: positions %d..%d exceed capacity %d", pos0, pos0 + m, capacity);
    if (m == 0) return MT_OK;
    const int max_keys = window > 0 ? (window < pos0 + m ? window : pos0 + m) : pos0 + m;
    MT_REQUIRE(ctx, attention_smem(hq / hkv, max_keys) <= 200 * 1024, MT_ERR_SHAPE,
               "mt_attention: %d keys exceed the shared-memory score buffer", max_keys);
    MT_REQUIRE(ctx, aligned16(k_cache) && aligned16(v_cache), MT_ERR_ARG, "mt_attention: caches need 16-byte alignment");
    AttnArgs a{};
    a.q = q; a.ldq = ldq; a.rows = m; a.rows_per_req = m; a.hq = hq; a.hkv = hkv; a.pos0 = pos0;
    a.window = window; a.kc = k_cache; a.vc = v_cache; a.cap = capacity; a.out = out; a.ldo = ldo;
    a.max_keys = max_keys;
    launch_attention(a, as_stream(stream));
    return check_launch(ctx, "mt_attention");
}

mt_status mt_dit_attention(mt_ctx* ctx, void* stream, const float* qkv, int ld, int batch, int seq,
                           int heads, const float* inv_freq, float* out, int ldo) {
    MT_REQUIRE(ctx, ctx && qkv && inv_freq && out, MT_ERR_ARG, "mt_dit_attention: null argument");
    MT_REQUIRE(ctx, seq >= 1 && seq <= 8, MT_ERR_SHAPE, "mt_dit_attention: seq %d (1..8)", seq);
    MT_REQUIRE(ctx, batch >= 0 && heads > 0 && ld >= 3 * heads * 64 && ldo >= heads * 64 && ld % 2 == 0 && ldo % 2 == 0,
               MT_ERR_SHAPE, "mt_dit_attention: heads %d ld %d ldo %d", heads, ld, ldo);
    if (batch == 0) return MT_OK;
    DitAttnArgs a{};
    a.qkv = qkv; a.ld = ld; a.batch = batch; a.seq = seq; a.heads = heads; a.inv_freq = inv_freq;
    a.out = out; a.ldo = ldo;
    launch_dit_attention(a, as_stream(stream));
    return check_launch(ctx, "mt_dit_attention");
}

mt_status mt_flow_assemble(mt_ctx* ctx, void* stream, const float* y, const float* history, const float* cemb,
                           const mt_bf16* cond_bias, const float* temb, const mt_bf16* x_w, const mt_bf16* x_b,
                           int hidden, int latent_dim, float* x) {
    MT_REQUIRE(ctx, ctx && y && history && cemb && cond_bias && temb && x_w && x_b && x, MT_ERR_ARG,
               "mt_flow_assemble: null argument");
    MT_REQUIRE(ctx, hidden > 0 && latent_dim > 0, MT_ERR_SHAPE, "mt_flow_assemble: hidden %d latent %d", hidden, latent_dim);
    launch_k(flow_assemble_kernel, dim3((hidden + 255) / 256, 6), 256, 0, as_stream(stream), 
        y, history, cemb, cond_bias, temb, x_w, x_b, hidden, latent_dim, x);
    return check_launch(ctx, "mt_flow_assemble");
}

mt_status mt_flow_euler(mt_ctx* ctx, void* stream, float* y, const float* pred, int ldp, int pred_row,
                        int null_row, int latent_dim, float cfg, float dt, float* capture) {
    MT_REQUIRE(ctx, ctx && y && pred, MT_ERR_ARG, "mt_flow_euler: null argument");
    MT_REQUIRE(ctx, latent_dim > 0 && pred_row >= 0 && null_row >= 0 && ldp >= latent_dim, MT_ERR_SHAPE,
               "mt_flow_euler: latent %d ldp %d", latent_dim, ldp);
    launch_k(flow_euler_kernel, (latent_dim + 255) / 256, 256, 0, as_stream(stream), y, pred, ldp, pred_row, null_row,
                                                                           latent_dim, cfg, dt, capture);
    return check_launch(ctx, "mt_flow_euler");
}

mt_status mt_upsample4(mt_ctx* ctx, void* stream, const float* prev, const float* cur, const float* next,
                       int hidden, float* frames) {
    MT_REQUIRE(ctx, ctx && cur && frames, MT_ERR_ARG, "mt_upsample4: null argument");
    MT_REQUIRE(ctx, hidden > 0, MT_ERR_SHAPE, "mt_upsample4: hidden %d", hidden);
    launch_k(upsample4_kernel, dim3((hidden + 255) / 256, 4), 256, 0, as_stream(stream), prev, cur, next, hidden, frames);
    return check_launch(ctx, "mt_upsample4");
}

}  // extern "C"
