// ops.cu -- element-wise, normalisation and attention kernels, and their C-ABI entry points.
//
// Reference kernels restated (semantics, not code): rmsnorm / copy_rows (Shaders.swift:418-447),
// rope_cache (Shaders.swift:456-486), attention_cache (Shaders.swift:500-591), dit_attention
// (Shaders.swift:613-648), flow_assemble / flow_euler (Shaders.swift:654-693), upsample4
// (Shaders.swift:704-719).
#include "common.cuh"
#include "kernels.cuh"

#include <cooperative_groups.h>
namespace cg = cooperative_groups;

namespace mt {

// ------------------------------------------------------------------------------------------------
// RMSNorm: one block per row; each thread keeps its float4s of the row in registers, so the row
// is read once; optional fp32 and/or bf16 hi/lo outputs.
// ------------------------------------------------------------------------------------------------
constexpr int RMS_THREADS = 128;
constexpr int RMS_MAXV = 8;  // float4 per thread: width <= 4096

__global__ void __launch_bounds__(RMS_THREADS) rmsnorm_kernel(RmsArgs a) {
    __shared__ float part[RMS_THREADS / 32];
    const int row = blockIdx.x;
    const int n4 = a.width >> 2;
    // The gains are weights (never written by a kernel): fetched while the previous kernel drains.
    const uint2* w = reinterpret_cast<const uint2*>(a.w);
    uint2 wv[RMS_MAXV];
#pragma unroll
    for (int i = 0; i < RMS_MAXV; i++) {
        const int c = threadIdx.x + i * RMS_THREADS;
        wv[i] = c < n4 ? w[c] : make_uint2(0u, 0u);
    }
    pdl_wait();
    pdl_launch();
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
#pragma unroll
    for (int i = 0; i < RMS_MAXV; i++) {
        const int c = threadIdx.x + i * RMS_THREADS;
        if (c >= n4) break;
        float4 o;
        o.x = v[i].x * scale * bf16_lo(wv[i].x);
        o.y = v[i].y * scale * bf16_hi(wv[i].x);
        o.z = v[i].z * scale * bf16_lo(wv[i].y);
        o.w = v[i].w * scale * bf16_hi(wv[i].y);
        if (a.y) reinterpret_cast<float4*>(a.y + (size_t)row * a.ldy)[c] = o;
        if (a.y_hi) {
            uint32_t h01, l01, h23, l23;
            split_bf16x2(o.x, o.y, h01, l01);
            split_bf16x2(o.z, o.w, h23, l23);
            reinterpret_cast<uint2*>(a.y_hi + (size_t)row * a.ld_split)[c] = make_uint2(h01, h23);
            reinterpret_cast<uint2*>(a.y_lo + (size_t)row * a.ld_split)[c] = make_uint2(l01, l23);
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
        uint32_t h01, l01, h23, l23;
        split_bf16x2(v.x, v.y, h01, l01);
        split_bf16x2(v.z, v.w, h23, l23);
        reinterpret_cast<uint2*>(hi + (size_t)r * ld_split)[c] = make_uint2(h01, h23);
        reinterpret_cast<uint2*>(lo + (size_t)r * ld_split)[c] = make_uint2(l01, l23);
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
    static PerDeviceOnce once;  // per device, on the first (eager) call, before any graph capture
    once([] { cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); });
    launch_k(attention_kernel, dim3(a.rows, a.hkv), ATT_THREADS, smem, s, a);
}

// ------------------------------------------------------------------------------------------------
// Fused decode attention (see AttnDecodeArgs). Block (request, kv head), 256 threads. The union of
// the request rows' key ranges is processed in chunks of SC keys: old keys arrive by bulk copy
// (cp.async.bulk, at most two segments per chunk when the cache ring wraps) on bounded mbarrier
// waits, new keys come from the block's own rotation. Scores use a skewed float4 walk over the
// 64 dims so the 32 keys a warp touches fall in distinct bank groups; softmax is online across
// chunks; thread groups of P own (row-head, 4 dims) accumulators for P.V.
// With few (request, kv head) units the key range is split over gridDim.z blocks that form one
// thread-block cluster: each split keeps its own online-softmax state, and cluster rank 0 merges
// the partials through distributed shared memory between two cluster barriers (the flash-decoding
// split: O = sum_z e^(m_z - M) O_z / sum_z e^(m_z - M) l_z, M = max_z m_z). Only split 0 appends
// the new keys and values to the cache; every split stashes them for its own chunks.
// ------------------------------------------------------------------------------------------------
constexpr int AD_THREADS = 256;
constexpr int AD_MAX_RG = ATTN_DECODE_MAX_ROWS * 8;  // rows x query heads per kv head
constexpr int AD_MAX_SPLITS = 8;                     // key splits per unit: one portable cluster

static size_t ad_dyn_bytes(int SC, int nrows, int nrg) {
    return sizeof(float) * ((size_t)SC * 64 * 2 + (size_t)nrg * 64 + (size_t)nrows * 128 + (size_t)nrg * SC);
}

__global__ void __launch_bounds__(AD_THREADS) attention_decode_kernel(AttnDecodeArgs a, int SC) {
    extern __shared__ __align__(128) float sm[];
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ float m_run[AD_MAX_RG], l_run[AD_MAX_RG], alpha[AD_MAX_RG];
    __shared__ float rot_c[ATTN_DECODE_MAX_ROWS][32], rot_s[ATTN_DECODE_MAX_ROWS][32];
    __shared__ int abort_flag, split_ok;
    const int r = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = gridDim.z, z = blockIdx.z;  // key splits of this unit; this block's split
    const int G = a.hq / a.hkv, nrows = a.rows_per_req, nrg = nrows * G;
    float* Ks = sm;
    float* Vs = Ks + (size_t)SC * 64;
    float* qs = Vs + (size_t)SC * 64;
    float* nw = qs + (size_t)nrg * 64;  // [nrows][k | v][64]
    float* sc = nw + (size_t)nrows * 128;
    volatile int* abort = &abort_flag;

    // Everything up to pdl_wait reads only what earlier kernels and the host finished long ago:
    // positions (host-uploaded step state), rotation frequencies, and the cached keys and values
    // of earlier positions (this launch writes only the new positions' slots).
    const int base = a.pos0 + (a.pos_dev ? a.pos_dev[r] : 0);
    const int p_first = base, p_end = base + nrows;  // new keys [p_first, p_end)
    const int W = a.window;
    const int jS = W > 0 ? max(0, p_first + 1 - W) : 0;
    int s0 = jS, s1 = p_end;  // this split's keys [s0, s1)
    if (S > 1) {
        const int per = ((p_end - jS + S - 1) / S + 15) & ~15;
        s0 = min(p_end, jS + z * per);
        s1 = min(p_end, s0 + per);
    }
    const int chunks = (s1 - s0 + SC - 1) / SC;
    float* kc = a.kc + (size_t)r * a.req_stride + (size_t)h * a.cap * 64;
    float* vc = a.vc + (size_t)r * a.req_stride + (size_t)h * a.cap * 64;
    // Old keys of chunk c: [c0, min(c1, p_first)). Thread 0 arms both barriers for the chunk's
    // bytes (arm), then lane 0 of every warp copies one slice of the keys and values (issue): one
    // thread's bulk copies stream one after another at a few bytes per clock from DRAM, so the
    // slices of eight warps keep eight times as many bytes in flight.
    auto old_keys = [&](int c) {
        const int c0 = s0 + c * SC, c1 = min(c0 + SC, s1);
        return max(0, min(c1, p_first) - c0);
    };
    auto arm = [&](int c) {
        const uint32_t bytes = (uint32_t)old_keys(c) * 256u;
        mbar_expect_tx(&bar[0], bytes);
        mbar_expect_tx(&bar[1], bytes);
    };
    auto issue = [&](int c) {  // lane 0 of warp `warp`
        const int nold = old_keys(c);
        const int per = (nold + AD_THREADS / 32 - 1) / (AD_THREADS / 32);
        const int k0 = warp * per, k1 = min(nold, k0 + per);
        if (k0 >= k1) return;
        const int slot = (s0 + c * SC + k0) % a.cap;  // ring slot of this slice's first key
        const int len1 = min(k1 - k0, a.cap - slot);
        bulk_load(Ks + (size_t)k0 * 64, kc + (size_t)slot * 64, (uint32_t)len1 * 256u, &bar[0]);
        bulk_load(Vs + (size_t)k0 * 64, vc + (size_t)slot * 64, (uint32_t)len1 * 256u, &bar[1]);
        if (k0 + len1 < k1) {  // the slice wraps around the ring
            const uint32_t rest = (uint32_t)(k1 - k0 - len1) * 256u;
            bulk_load(Ks + (size_t)(k0 + len1) * 64, kc, rest, &bar[0]);
            bulk_load(Vs + (size_t)(k0 + len1) * 64, vc, rest, &bar[1]);
        }
    };
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        arm(0);
    }
    if (tid < nrg) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.f;
    }
    if (tid < nrows * 32) {  // NeoX rotation of position base + i, pair (l, l + 32)
        const int i = tid >> 5, l = tid & 31;
        float sn, cs;
        sincosf((float)(base + i) * a.inv_freq[l], &sn, &cs);
        rot_c[i][l] = cs;
        rot_s[i][l] = sn;
    }
    __syncthreads();
    if (lane == 0) issue(0);
    pdl_wait();
    pdl_launch();

    // New rows: item (row i, slot, pair l), slot < G a query head of this kv group, G the key, G + 1
    // the value. All loads first, then rotate, append k and v to the cache and stash them.
    constexpr int NR_MAX = (ATTN_DECODE_MAX_ROWS * 10 * 32 + AD_THREADS - 1) / AD_THREADS;
    const int items = nrows * (G + 2) * 32;
    float x0[NR_MAX], x1[NR_MAX];
#pragma unroll
    for (int u = 0; u < NR_MAX; u++) {
        const int it = tid + u * AD_THREADS;
        if (it < items) {
            const int l = it & 31, slot = (it >> 5) % (G + 2), i = (it >> 5) / (G + 2);
            const float* row = a.qkv + (size_t)(r * nrows + i) * a.ldq;
            const int col = slot < G ? (h * G + slot) * 64 : slot == G ? (a.hq + h) * 64 : (a.hq + a.hkv + h) * 64;
            x0[u] = row[col + l];
            x1[u] = row[col + l + 32];
        }
    }
#pragma unroll
    for (int u = 0; u < NR_MAX; u++) {
        const int it = tid + u * AD_THREADS;
        if (it < items) {
            const int l = it & 31, slot = (it >> 5) % (G + 2), i = (it >> 5) / (G + 2);
            float v0 = x0[u], v1 = x1[u];
            if (slot <= G) {
                const float cs = rot_c[i][l], sn = rot_s[i][l];
                const float r0 = v0 * cs - v1 * sn, r1 = v1 * cs + v0 * sn;
                v0 = r0;
                v1 = r1;
            }
            if (slot < G) {
                qs[(i * G + slot) * 64 + l] = v0;
                qs[(i * G + slot) * 64 + l + 32] = v1;
            } else {
                if (z == 0) {
                    float* dst = (slot == G ? kc : vc) + (size_t)((base + i) % a.cap) * 64;
                    dst[l] = v0;
                    dst[l + 32] = v1;
                }
                float* st = nw + (i * 2 + (slot - G)) * 64;
                st[l] = v0;
                st[l + 32] = v1;
            }
        }
    }

    // P.V ownership: thread (4 dims d4 = tid % 16, row i, part) holds the G heads of row i; the
    // PP parts split the keys, so the 16 lanes of a part read one V row (256 contiguous bytes).
    const int d4 = tid & 15, grp = tid >> 4;  // 16 groups of 16 lanes
    const int PP = (AD_THREADS / 16) / nrows;  // parts per row
    const int pv_i = grp % nrows, pv_part = grp / nrows;
    const bool pv_live = pv_part < PP;
    float4 acc[8];
#pragma unroll
    for (int g = 0; g < 8; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);

    bool ok = true;
    for (int c = 0; c < chunks && ok; c++) {
        const int c0 = s0 + c * SC, c1 = min(c0 + SC, s1), cn = c1 - c0;
        const int old_end = min(c1, p_first);
        const int nold = max(0, old_end - c0);
        __syncthreads();  // the previous chunk's readers are done with Ks, Vs and sc
        if (c > 0 && tid == 0) arm(c);
        // New keys of this chunk from the stash.
        for (int e = tid; e < (cn - nold) * 64; e += AD_THREADS) {
            const int jj = nold + e / 64, d = e % 64;
            const int i = c0 + jj - p_first;
            Ks[(size_t)jj * 64 + d] = nw[(i * 2) * 64 + d];
            Vs[(size_t)jj * 64 + d] = nw[(i * 2 + 1) * 64 + d];
        }
        __syncthreads();  // chunk c armed (thread 0) and the previous chunk's reads done
        if (c > 0 && lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(c);
        }
        if (!mbar_wait(&bar[0], c & 1, a.status, 20, abort)) { ok = false; break; }
        // Scores: item (key pair p, row-head rg) scores keys k0 and k0 + 8 (same 16-byte skew
        // s = p & 7, so the eight lanes of a shared-memory phase read eight distinct bank groups of
        // K and one q chunk serves both keys). One head per item keeps every warp busy when a
        // block holds few keys (a split's 32-64): items per head would leave one warp doing all
        // G heads while the others wait at the barrier.
        const float4* K4 = reinterpret_cast<const float4*>(Ks);
        const float4* Q4 = reinterpret_cast<const float4*>(qs);
        const int npairs = ((cn + 15) / 16) * 8;
        for (int it = tid; it < npairs * nrg; it += AD_THREADS) {
            const int pr = it % npairs, rg = it / npairs, i = rg / G;
            const int k0 = (pr >> 3) * 16 + (pr & 7), k1 = k0 + 8;
            const int sk = pr & 7;
            const bool l0 = k0 < cn, l1 = k1 < cn;
            const float4* q = Q4 + rg * 16;
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int t = 0; t < 16; t++) {
                const int ch = (t + sk) & 15;
                const float4 q4 = q[ch];
                const float4 ka = l0 ? K4[k0 * 16 + ch] : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 kb = l1 ? K4[k1 * 16 + ch] : make_float4(0.f, 0.f, 0.f, 0.f);
                s0 += q4.x * ka.x + q4.y * ka.y + q4.z * ka.z + q4.w * ka.w;
                s1 += q4.x * kb.x + q4.y * kb.y + q4.z * kb.z + q4.w * kb.w;
            }
            const int pos = base + i;
            const int j0 = c0 + k0, j1 = c0 + k1;
            const bool v0 = j0 <= pos && (W == 0 || j0 > pos - W);
            const bool v1 = j1 <= pos && (W == 0 || j1 > pos - W);
            if (l0) sc[(size_t)rg * SC + k0] = v0 ? s0 * 0.125f : -INFINITY;
            if (l1) sc[(size_t)rg * SC + k1] = v1 ? s1 * 0.125f : -INFINITY;
        }
        __syncthreads();
        // Online softmax statistics; scores become weights relative to the running maximum.
        for (int rg = warp; rg < nrg; rg += AD_THREADS / 32) {
            float* srow = sc + (size_t)rg * SC;
            float mx = -INFINITY;
            for (int jj = lane; jj < cn; jj += 32) mx = fmaxf(mx, srow[jj]);
            mx = warp_max(mx);
            const float m_old = m_run[rg];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.f;
            for (int jj = lane; jj < cn; jj += 32) {
                const float e = m_new == -INFINITY ? 0.f : expf(srow[jj] - m_new);
                srow[jj] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float al = m_new == -INFINITY ? 1.f : expf(m_old - m_new);
                alpha[rg] = al;
                l_run[rg] = l_run[rg] * al + sum;
                m_run[rg] = m_new;
            }
        }
        __syncthreads();
        if (!mbar_wait(&bar[1], c & 1, a.status, 21, abort)) { ok = false; break; }
        if (pv_live) {
            const float4* V4 = reinterpret_cast<const float4*>(Vs);
#pragma unroll
            for (int g = 0; g < 8; g++) {
                if (g < G) {
                    const float al = alpha[pv_i * G + g];
                    acc[g].x *= al; acc[g].y *= al; acc[g].z *= al; acc[g].w *= al;
                }
            }
            for (int jj = pv_part; jj < cn; jj += PP) {
                const float4 v4 = V4[jj * 16 + d4];
#pragma unroll
                for (int g = 0; g < 8; g++) {
                    if (g < G) {
                        const float pj = sc[(size_t)(pv_i * G + g) * SC + jj];
                        acc[g].x += pj * v4.x; acc[g].y += pj * v4.y; acc[g].z += pj * v4.z; acc[g].w += pj * v4.w;
                    }
                }
            }
        }
    }
    // Reduce the PP partial sums through shared memory (the K/V chunk area is free now); output
    // task t = (row-head rg, 4 dims dd).
    __syncthreads();
    float4* part4 = reinterpret_cast<float4*>(Ks);  // [PP][nrows][G][16]
    if (ok && pv_live) {
#pragma unroll
        for (int g = 0; g < 8; g++)
            if (g < G) part4[((pv_part * nrows + pv_i) * G + g) * 16 + d4] = acc[g];
    }
    __syncthreads();
    auto write_out = [&](int t, float4 o, float inv) {
        const int dd = t & 15, rg = t >> 4, i = rg / G, g = rg % G;
        const float o0 = o.x * inv, o1 = o.y * inv, o2 = o.z * inv, o3 = o.w * inv;
        const size_t row = (size_t)(r * nrows + i);
        const int head = h * G + g;
        if (a.out) *reinterpret_cast<float4*>(a.out + row * a.ldo + head * 64 + dd * 4) = make_float4(o0, o1, o2, o3);
        if (a.out_hi) {
            uint32_t h01, l01, h23, l23;
            split_bf16x2(o0, o1, h01, l01);
            split_bf16x2(o2, o3, h23, l23);
            const size_t so = row * a.ld_split + head * 64 + dd * 4;
            *reinterpret_cast<uint2*>(a.out_hi + so) = make_uint2(h01, h23);
            *reinterpret_cast<uint2*>(a.out_lo + so) = make_uint2(l01, l23);
        }
    };
    auto part_sum = [&](int t) {
        const int dd = t & 15, rg = t >> 4, i = rg / G, g = rg % G;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < PP; q++) {
            const float4 v = part4[((q * nrows + i) * G + g) * 16 + dd];
            o.x += v.x; o.y += v.y; o.z += v.z; o.w += v.w;
        }
        return o;
    };
    if (S == 1) {
        if (!ok) return;
        for (int t = tid; t < nrg * 16; t += AD_THREADS) write_out(t, part_sum(t), 1.0f / l_run[t >> 4]);
        return;
    }
    // Split: this block's unnormalised sums go to the q area ([nrg][16] float4, free after the
    // key loop); every block of the cluster passes both barriers, failed or not.
    float4* fin4 = reinterpret_cast<float4*>(qs);
    if (ok)
        for (int t = tid; t < nrg * 16; t += AD_THREADS) fin4[t] = part_sum(t);
    if (tid == 0) split_ok = ok ? 1 : 0;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0) {
        // Every remote load of a task is issued before any is used (S <= AD_MAX_SPLITS).
        int n_ok = 0;
#pragma unroll
        for (int q = 0; q < AD_MAX_SPLITS; q++)
            if (q < S) n_ok += *cluster.map_shared_rank(&split_ok, q);
        if (n_ok == S) {
            for (int t = tid; t < nrg * 16; t += AD_THREADS) {
                const int rg = t >> 4;
                float mq[AD_MAX_SPLITS], lq[AD_MAX_SPLITS];
                float4 vq[AD_MAX_SPLITS];
#pragma unroll
                for (int q = 0; q < AD_MAX_SPLITS; q++) {
                    if (q < S) {
                        mq[q] = cluster.map_shared_rank(m_run, q)[rg];
                        lq[q] = cluster.map_shared_rank(l_run, q)[rg];
                        vq[q] = cluster.map_shared_rank(fin4, q)[t];
                    }
                }
                float M = -INFINITY;
#pragma unroll
                for (int q = 0; q < AD_MAX_SPLITS; q++)
                    if (q < S) M = fmaxf(M, mq[q]);
                float L = 0.f;
                float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int q = 0; q < AD_MAX_SPLITS; q++) {
                    if (q < S && mq[q] != -INFINITY) {  // a split that holds no key of this row adds nothing
                        const float wq = expf(mq[q] - M);
                        L += lq[q] * wq;
                        o.x += vq[q].x * wq; o.y += vq[q].y * wq; o.z += vq[q].z * wq; o.w += vq[q].w * wq;
                    }
                }
                write_out(t, o, 1.0f / L);
            }
        }
    }
    cluster.sync();  // no block leaves while rank 0 reads its shared memory
}

bool attention_decode_supported(int rows_per_req, int hq, int hkv) {
    return rows_per_req >= 1 && rows_per_req <= ATTN_DECODE_MAX_ROWS && hkv > 0 && hq % hkv == 0 && hq / hkv <= 8;
}

void launch_attention_decode(const AttnDecodeArgs& a, cudaStream_t s) {
    const int G = a.hq / a.hkv, nrg = a.rows_per_req * G;
    const int nk_max = a.window > 0 ? min(a.window + a.rows_per_req - 1, a.cap) : a.max_keys;
    constexpr size_t kBudget = 223 * 1024;  // dynamic shared memory: 227 KB per block less the static part
    // Key splits: with fewer units than a quarter of the SMs, up to 8 splits of at least 32 keys,
    // as one cluster per unit.
    const int units = a.requests * a.hkv;
    int S = 1;
    if (units * 4 <= 148) S = max(1, min(min(AD_MAX_SPLITS, 148 / units), (nk_max + 31) / 32));
    const int per_max = ((nk_max + S - 1) / S + 15) & ~15;
    int SC = per_max;
    if (a.chunk_keys > 0 && a.chunk_keys < SC) SC = (a.chunk_keys + 15) & ~15;
    if (SC < 8 * G) SC = 8 * G;  // the final reduction reuses the K/V area: 16 x G x 256 bytes
    while (SC > 16 && ad_dyn_bytes(SC, a.rows_per_req, nrg) > kBudget) SC -= 16;
    static PerDeviceOnce once;  // per device, on the first (eager) call, before any graph capture
    once([] { cudaFuncSetAttribute(attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBudget); });
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.requests, a.hkv, S);
    cfg.blockDim = dim3(AD_THREADS);
    cfg.dynamicSmemBytes = ad_dyn_bytes(SC, a.rows_per_req, nrg);
    cfg.stream = s;
    cudaLaunchAttribute attr[3];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na++].val.programmaticStreamSerializationAllowed = 1;
    if (S > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na++].val.clusterDim.z = S;
    }
    if (launch_priority() != 0) {
        attr[na].id = cudaLaunchAttributePriority;
        attr[na++].val.priority = launch_priority();
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    cudaLaunchKernelEx(&cfg, attention_decode_kernel, a, SC);
}

// ------------------------------------------------------------------------------------------------
// DiT attention: one warp per (sequence, head) computes every row of the sequence (seq <= 8);
// lane l owns dims 2l, 2l+1 = one interleaved RoPE pair. All q/k/v loads of the warp are issued
// before any use, and each position's rotation is computed once. The sequence length is a
// template parameter: with a runtime length the unrolled (row, key) loops ran all 8 x 8 pairs
// predicated (measured 3x slower for the 3-row flow sequences).
// ------------------------------------------------------------------------------------------------
template <int DIT_MAX_SEQ>
__global__ void dit_attention_kernel(DitAttnArgs a) {
    pdl_wait();
    pdl_launch();
    const int work = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (work >= a.batch * a.heads) return;
    const int h = work % a.heads, b = work / a.heads;
    const int D = a.heads * 64;
    constexpr int S = DIT_MAX_SEQ;
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
            uint32_t h01, l01;
            split_bf16x2(o0, o1, h01, l01);
            const size_t so = row * a.ld_split + h * 64 + 2 * lane;
            *reinterpret_cast<uint32_t*>(a.out_hi + so) = h01;
            *reinterpret_cast<uint32_t*>(a.out_lo + so) = l01;
        }
    }
}

void launch_dit_attention(const DitAttnArgs& a, cudaStream_t s) {
    const unsigned blocks = (unsigned)((a.batch * a.heads + 7) / 8);
    switch (a.seq) {  // seq in 1..8, checked by the callers
        case 1: launch_k(dit_attention_kernel<1>, blocks, 256, 0, s, a); break;
        case 2: launch_k(dit_attention_kernel<2>, blocks, 256, 0, s, a); break;
        case 3: launch_k(dit_attention_kernel<3>, blocks, 256, 0, s, a); break;
        case 4: launch_k(dit_attention_kernel<4>, blocks, 256, 0, s, a); break;
        case 5: launch_k(dit_attention_kernel<5>, blocks, 256, 0, s, a); break;
        case 6: launch_k(dit_attention_kernel<6>, blocks, 256, 0, s, a); break;
        case 7: launch_k(dit_attention_kernel<7>, blocks, 256, 0, s, a); break;
        default: launch_k(dit_attention_kernel<8>, blocks, 256, 0, s, a); break;
    }
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

mt_status mt_rope_attention(mt_ctx* ctx, void* stream, const float* qkv, int ldq, int m, int hq, int hkv, int pos0,
                            int window, float* k_cache, float* v_cache, int capacity, const float* inv_freq,
                            float* out, int ldo, int chunk_keys) {
    MT_REQUIRE(ctx, ctx && qkv && k_cache && v_cache && inv_freq && out, MT_ERR_ARG, "mt_rope_attention: null argument");
    MT_REQUIRE(ctx, m >= 0 && m <= ATTN_DECODE_MAX_ROWS && attention_decode_supported(m > 0 ? m : 1, hq, hkv) &&
                        ldq >= (hq + 2 * hkv) * 64 && ldo >= hq * 64 && ldo % 4 == 0 && window >= 0 && chunk_keys >= 0,
               MT_ERR_SHAPE, "mt_rope_attention: m %d (<= %d) hq %d hkv %d ldq %d ldo %d window %d", m,
               ATTN_DECODE_MAX_ROWS, hq, hkv, ldq, ldo, window);
    MT_REQUIRE(ctx, pos0 >= 0 && capacity > 0 &&
                        (pos0 + m <= capacity || (window > 0 && window + m - 1 <= capacity)),
               MT_ERR_CAPACITY, "mt_rope_attention: positions %d..%d do not fit capacity %d (window %d)", pos0, pos0 + m,
               capacity, window);
    MT_REQUIRE(ctx, aligned16(k_cache) && aligned16(v_cache) && aligned16(out), MT_ERR_ARG,
               "mt_rope_attention: caches and output need 16-byte alignment");
    if (m == 0) return MT_OK;
    AttnDecodeArgs a{};
    a.qkv = qkv; a.ldq = ldq; a.requests = 1; a.rows_per_req = m; a.hq = hq; a.hkv = hkv; a.pos0 = pos0;
    a.window = window; a.kc = k_cache; a.vc = v_cache; a.req_stride = 0; a.cap = capacity; a.inv_freq = inv_freq;
    a.out = out; a.ldo = ldo; a.max_keys = window > 0 ? window + m - 1 : pos0 + m; a.chunk_keys = chunk_keys;
    a.status = ctx->d_status;
    launch_attention_decode(a, as_stream(stream));
    return check_launch(ctx, "mt_rope_attention");
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
