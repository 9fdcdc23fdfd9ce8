// gemm_tc.cu -- tcgen05 / TMEM tensor-core GEMM for sm_100a:
//     Y[m, n] = epi( sum_k X[m, k] * W[n, k] )  with X fp32 carried as two bf16 planes (hi + lo).
//
// Reference semantics: the tiled GEMM and gemm8 kernels (Shaders.swift:191-277, 304-408) -- fp32
// activations times bf16 weights with fp32 accumulation and the linear epilogue. Tensor cores
// take bf16 operands, so the activations enter as x = hi + lo (both bf16, |x - hi - lo| <= 2^-17|x|);
// the two planes sit next to each other in shared memory, so one MMA of N = 2 bn computes W.hi and
// W.lo side by side in TMEM and the epilogue adds them. The weights are exact in bf16. The result
// matches fp32 FMA accumulation to ~1e-5 relative.
//
// Layout ("swap AB"): the MMA's M side is 128 weight rows (output columns n), its N side is
// 2 x bn activation rows (m), so small row counts still use full 128-lane MMAs. The accumulator is
// D[n_local][m_local] in TMEM (lane = weight row, column = activation row).
//
// Persistent schedule: one CTA per SM walks its share of the (n tile, m tile, k split) space.
// Warp 0 lane 0 issues TMA loads (128B swizzle, no multicast) into a ring of stages shared by all
// of the CTA's tiles; warp 1 lane 0 issues tcgen05.mma into one of two TMEM accumulators and frees
// stages with tcgen05.commit; warps 2-9 (two per TMEM lane quadrant) drain the other accumulator
// through the epilogue, so the epilogue of tile t overlaps the loads and MMAs of tile t + 1.
// Every mbarrier wait is bounded: a wait that gives up writes the context status word, raises the
// CTA's abort flag (all other waits then return at once) and the CTA stops issuing work.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"

namespace mt {

constexpr int TC_THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue (warp 2 owns TMEM)
constexpr int TC_EPI_WARPS = 8;
constexpr int TC_BM = 128;  // weight rows per tile (MMA M)
constexpr int TC_BK = 64;   // bf16 K per atom = one 128-byte swizzle span
constexpr int TC_KA_MAX = 2;  // K atoms per pipeline stage (TcEpi::ka): one barrier round trip and commit per stage



__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle canonical layout
// (8-row x 128-byte atoms, 1024 bytes apart), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: bf16 A and B, fp32 accumulator, both K-major.
__device__ __forceinline__ uint32_t idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 16 consecutive accumulator columns of this thread's TMEM lane; pair with tmem_wait() before use.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Tile t of the plan: k split z = t / (tiles_m * tiles_n); inside a split, consecutive tiles walk
// the m tiles of one n tile (CTAs running together share weight tiles in L2).
struct TileCoord { int n0, m0, kb_begin, kb_end; };
__device__ __forceinline__ TileCoord tile_coord(const TcEpi& e, int t) {
    const int per_split = e.tiles_m * e.tiles_n;
    const int z = t / per_split, r = t % per_split;
    TileCoord c;
    c.m0 = (r % e.tiles_m) * e.bn;
    c.n0 = (r / e.tiles_m) * TC_BM;
    const int kb_total = (e.k + TC_BK - 1) / TC_BK;
    c.kb_begin = z * e.kb_per_split;
    c.kb_end = min(kb_total, c.kb_begin + e.kb_per_split);
    return c;
}

// Bias of this thread's output column in the tile at column n0 (0 where nothing is added: no BIAS
// flag, a column past N, or a split-K partial other than the first). Biases are weights, never
// written by a kernel, so this may run before the wait on the previous kernel.
__device__ __forceinline__ float tile_bias(const TcEpi& e, int n0, int quad, int lane, bool first_split) {
    const int n = n0 + quad * 32 + lane;
    const bool add = (e.flags & MT_LINEAR_BIAS) && n < e.n && (e.mode != 1 || first_split);
    return add ? bf16f(e.bias[n]) : 0.f;
}

// Epilogue of one tile for one warp: 16-column chunks `part`, `part + 2`, ... of TMEM lane quadrant
// `quad` (weight rows n0 + 32 quad + lane).
template <bool GATED>
__device__ __forceinline__ void epilogue_tile(const TcEpi& e, const TileCoord& tc, uint32_t acc, int quad, int part,
                                              int lane, bool first_split) {
    const int n = tc.n0 + quad * 32 + lane;
    const bool live_n = n < e.n;
    const bool add_bias = (e.flags & MT_LINEAR_BIAS) && live_n && (e.mode == 0 || (e.mode == 1 && first_split));
    const float bval = add_bias ? bf16f(e.bias[n]) : 0.f;
    const uint32_t lane_base = acc + ((uint32_t)(quad * 32) << 16);
    for (int c0 = part * 16; c0 < e.bn; c0 += 32) {
        uint32_t rh[16], rl[16], r2h[16], r2l[16];
        tmem_ld16(lane_base + c0, rh);
        tmem_ld16(lane_base + e.bn + c0, rl);
        if (GATED) {
            tmem_ld16(lane_base + 2 * e.bn + c0, r2h);
            tmem_ld16(lane_base + 3 * e.bn + c0, r2l);
        }
        tmem_wait();
        if (!live_n) continue;
        const int valid = min(16, e.m - (tc.m0 + c0));  // activation rows of this chunk inside M
        if (valid <= 0) continue;
        float val[16], val2[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            val[j] = __uint_as_float(rh[j]) + __uint_as_float(rl[j]);
            val2[j] = GATED ? __uint_as_float(r2h[j]) + __uint_as_float(r2l[j]) : 0.f;
        }
        const size_t row0 = (size_t)(tc.m0 + c0);
        if (e.mode == 1) {  // split-K, linear epilogue: reduce into y (zeroed or the residual)
            float* __restrict__ yp = e.y + row0 * e.ldy + n;
#pragma unroll
            for (int j = 0; j < 16; j++)
                if (j < valid) atomicAdd(yp + (size_t)j * e.ldy, val[j] + bval);
            continue;
        }
        if (e.mode == 2) {  // split-K, nonlinear epilogue: raw sums into the workspace
            float* __restrict__ wp = e.ws + row0 * e.ldws + n;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                if (j < valid) {
                    atomicAdd(wp + (size_t)j * e.ldws, val[j]);
                    if (GATED) atomicAdd(wp + (size_t)j * e.ldws + e.n, val2[j]);
                }
            }
            continue;
        }
        const bool accum = (e.flags & MT_LINEAR_ACCUM) && e.y;
        float old[16];
        if (accum) {
            const float* __restrict__ yp = e.y + row0 * e.ldy + n;
#pragma unroll
            for (int j = 0; j < 16; j++) old[j] = j < valid ? yp[(size_t)j * e.ldy] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
            float v = val[j] + bval;
            if (GATED) v = silu(v) * val2[j];
            if (e.flags & MT_LINEAR_GELU) v = gelu_tanh(v);
            if (e.flags & MT_LINEAR_SILU) v = silu(v);
            if (accum) v += old[j];
            val[j] = v;
        }
        if (e.y) {
            float* __restrict__ yp = e.y + row0 * e.ldy + n;
#pragma unroll
            for (int j = 0; j < 16; j++)
                if (j < valid) yp[(size_t)j * e.ldy] = val[j];
        }
        if (e.y_hi) {
            uint16_t* __restrict__ hp = e.y_hi + row0 * e.ld_ysplit + n;
            uint16_t* __restrict__ lp = e.y_lo + row0 * e.ld_ysplit + n;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                uint16_t h, l;
                split_bf16(e.split_silu ? silu(val[j]) : val[j], h, l);
                if (j < valid) {
                    hp[(size_t)j * e.ld_ysplit] = h;
                    lp[(size_t)j * e.ld_ysplit] = l;
                }
            }
        }
    }
}

// The same epilogue for one EpiKind, with every flag decision made at compile time: the chunk body
// is straight-line code (measured ~3x faster per chunk than the runtime-flag path, whose per-value
// flag tests and predicated stores stall the epilogue warps).
template <int KIND, bool GATED>
__device__ __forceinline__ void epilogue_fast(const TcEpi& e, const TileCoord& tc, uint32_t acc, int quad, int part,
                                              int lane, float bval) {
    const int nq = tc.n0 + quad * 32;
    const int n = nq + lane;
    const bool live_n = n < e.n;
    const bool all_live = nq + 32 <= e.n;  // warp-uniform: every lane's output column exists
    const uint32_t lane_base = acc + ((uint32_t)(quad * 32) << 16);
    const size_t ldy = (size_t)e.ldy, lds = (size_t)e.ld_ysplit;
    for (int c0 = part * 16; c0 < e.bn; c0 += 32) {
        const int valid = min(16, e.m - (tc.m0 + c0));  // warp-uniform; chunks only grow in row index
        if (valid <= 0) break;
        uint32_t rh[16], rl[16], r2h[16], r2l[16];
        tmem_ld16(lane_base + c0, rh);
        tmem_ld16(lane_base + e.bn + c0, rl);
        if (GATED) {
            tmem_ld16(lane_base + 2 * e.bn + c0, r2h);
            tmem_ld16(lane_base + 3 * e.bn + c0, r2l);
        }
        tmem_wait();
        const size_t row0 = (size_t)(tc.m0 + c0);
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            float t = __uint_as_float(rh[j]) + __uint_as_float(rl[j]) + bval;
            if (GATED) t = silu(t) * (__uint_as_float(r2h[j]) + __uint_as_float(r2l[j]));
            if (KIND == EPI_SPLIT_GELU) t = gelu_tanh(t);
            if (KIND == EPI_F32_SILU) t = silu(t);
            v[j] = t;
        }
        const bool full = valid == 16 && all_live;
        if (KIND == EPI_F32_SSILU || KIND == EPI_ACC_SSILU || KIND == EPI_SSILU) {
            // fp32 stream (optionally accumulated) and the bf16 hi/lo planes of its silu
            if (KIND != EPI_SSILU) {
                float* __restrict__ yp = e.y + row0 * ldy + n;
                if (KIND == EPI_ACC_SSILU) {
                    float old[16];
#pragma unroll
                    for (int j = 0; j < 16; j++) old[j] = (full || (live_n && j < valid)) ? yp[j * ldy] : 0.f;
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] += old[j];
                }
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (full || (live_n && j < valid)) yp[j * ldy] = v[j];
            }
            uint16_t* __restrict__ hp = e.y_hi + row0 * lds + n;
            uint16_t* __restrict__ lp = e.y_lo + row0 * lds + n;
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
                uint32_t h2, l2;
                split_bf16x2(silu(v[j]), silu(v[j + 1]), h2, l2);
                if (full || (live_n && j < valid)) {
                    hp[j * lds] = (uint16_t)h2;
                    lp[j * lds] = (uint16_t)l2;
                }
                if (full || (live_n && j + 1 < valid)) {
                    hp[(j + 1) * lds] = (uint16_t)(h2 >> 16);
                    lp[(j + 1) * lds] = (uint16_t)(l2 >> 16);
                }
            }
        } else if (KIND == EPI_F32 || KIND == EPI_F32_ACCUM || KIND == EPI_F32_SILU || KIND == EPI_RED) {
            float* __restrict__ yp = e.y + row0 * ldy + n;
            if (full) {
                if (KIND == EPI_F32_ACCUM) {
                    float old[16];
#pragma unroll
                    for (int j = 0; j < 16; j++) old[j] = yp[j * ldy];
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] += old[j];
                }
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (KIND == EPI_RED) atomicAdd(yp + j * ldy, v[j]);
                    else yp[j * ldy] = v[j];
                }
            } else if (live_n) {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (j < valid) {
                        if (KIND == EPI_RED) atomicAdd(yp + j * ldy, v[j]);
                        else if (KIND == EPI_F32_ACCUM) yp[j * ldy] += v[j];
                        else yp[j * ldy] = v[j];
                    }
                }
            }
        } else {  // EPI_SPLIT, EPI_SPLIT_GELU, EPI_SPLIT_GATE
            uint16_t* __restrict__ hp = e.y_hi + row0 * lds + n;
            uint16_t* __restrict__ lp = e.y_lo + row0 * lds + n;
            uint16_t h[16], l[16];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
                uint32_t h2, l2;
                split_bf16x2(v[j], v[j + 1], h2, l2);
                h[j] = (uint16_t)h2, h[j + 1] = (uint16_t)(h2 >> 16);
                l[j] = (uint16_t)l2, l[j + 1] = (uint16_t)(l2 >> 16);
            }
            if (full) {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    hp[j * lds] = h[j];
                    lp[j * lds] = l[j];
                }
            } else if (live_n) {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (j < valid) {
                        hp[j * lds] = h[j];
                        lp[j * lds] = l[j];
                    }
                }
            }
        }
    }
}

template <bool GATED>
__device__ __forceinline__ void epilogue_dispatch(const TcEpi& e, const TileCoord& tc, uint32_t acc, int quad,
                                                  int part, int lane, bool first_split) {
    const float bval = tile_bias(e, tc.n0, quad, lane, first_split);
    if constexpr (GATED) {
        if (e.kind == EPI_SPLIT_GATE) epilogue_fast<EPI_SPLIT_GATE, true>(e, tc, acc, quad, part, lane, bval);
        else epilogue_tile<true>(e, tc, acc, quad, part, lane, first_split);
    } else {
        switch (e.kind) {
            case EPI_F32: epilogue_fast<EPI_F32, false>(e, tc, acc, quad, part, lane, bval); break;
            case EPI_F32_ACCUM: epilogue_fast<EPI_F32_ACCUM, false>(e, tc, acc, quad, part, lane, bval); break;
            case EPI_SPLIT: epilogue_fast<EPI_SPLIT, false>(e, tc, acc, quad, part, lane, bval); break;
            case EPI_SPLIT_GELU: epilogue_fast<EPI_SPLIT_GELU, false>(e, tc, acc, quad, part, lane, bval); break;
            case EPI_F32_SILU: epilogue_fast<EPI_F32_SILU, false>(e, tc, acc, quad, part, lane, bval); break;
            case EPI_RED: epilogue_fast<EPI_RED, false>(e, tc, acc, quad, part, lane, bval); break;
            default: epilogue_tile<false>(e, tc, acc, quad, part, lane, first_split); break;
        }
    }
}

// One kernel per (gated, epilogue kind, K atoms per stage): a launch carries only its own
// epilogue's code (measured: the runtime switch over all epilogues cost ~0.4 us of instruction
// fetch per launch), and the MMA thread's per-stage loop has no runtime trip counts (the loop runs
// at a few hundred cycles per stage; a runtime atom count alone slowed it by 5-10%).
template <bool GATED, int KIND, int KA>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                   const __grid_constant__ CUtensorMap tm_xhi, const __grid_constant__ CUtensorMap tm_xlo, TcEpi e) {
    extern __shared__ __align__(1024) uint8_t dsmem[];
    __shared__ uint64_t full_bar[8], empty_bar[8], acc_full[2], acc_empty[2];
    __shared__ uint32_t tmem_holder;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = e.stages;
    const int tiles_total = e.tiles_m * e.tiles_n * e.split;

    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
    const uint32_t w_bytes = TC_BM * 128, x_bytes = (uint32_t)e.bn * 128;
    // A stage holds KA K atoms, each [weights (both matrices when gated) | x planes]; one full
    // barrier, one empty barrier and one MMA commit per stage.
    const uint32_t atom_bytes = w_bytes * (GATED ? 2 : 1) + 2 * x_bytes;
    const uint32_t stage_bytes = KA * atom_bytes;
    // One accumulator = [W.x_hi | W.x_lo] per weight matrix (2 bn columns each); two of them.
    const uint32_t acc_cols = (uint32_t)e.bn * (GATED ? 4 : 2);
    uint32_t ncols = 32;
    while (ncols < 2 * acc_cols) ncols <<= 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], TC_EPI_WARPS);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_holder)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_holder;
    volatile int* abort = &abort_flag;
    // Barrier init and TMEM allocation above overlap the previous kernel's tail. The previous kernel
    // may still be writing this kernel's activations and outputs, so every access to those waits
    // for it (pdl_wait); the weights are never written by a kernel and are fetched before the wait.
    pdl_launch();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer: one ring of stages across all of this CTA's tiles
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
            if (GATED) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w2)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_xhi)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_xlo)) : "memory");
            // Weight tiles of the first S stages (fresh stages: no empty-slot wait needed).
            int pre = 0;
            for (int t = blockIdx.x; t < tiles_total && pre < S; t += gridDim.x) {
                const TileCoord tc = tile_coord(e, t);
                for (int kb = tc.kb_begin; kb < tc.kb_end && pre < S; kb += KA, pre++) {
                    const int na = KA == 1 ? 1 : min(KA, tc.kb_end - kb);
                    uint8_t* st = base + (size_t)pre * stage_bytes;
                    mbar_expect_tx(&full_bar[pre], na * atom_bytes);
                    for (int a = 0; a < na; a++) {
                        tma_load_2d(st + a * atom_bytes, &tm_w, &full_bar[pre], (kb + a) * TC_BK, tc.n0);
                        if (GATED) tma_load_2d(st + a * atom_bytes + w_bytes, &tm_w2, &full_bar[pre], (kb + a) * TC_BK, tc.n0);
                    }
                }
            }
            pdl_wait();
            // Stage s and the parity of its current use advance incrementally: a division by the
            // runtime stage count on every k block cost more than the MMAs of a k block.
            int g = 0, s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < tiles_total && !*abort; t += gridDim.x) {
                const TileCoord tc = tile_coord(e, t);
                for (int kb = tc.kb_begin; kb < tc.kb_end; kb += KA, g++, s = s + 1 == S ? 0 : s + 1, ph ^= s == 0) {
                    const int na = KA == 1 ? 1 : min(KA, tc.kb_end - kb);
                    uint8_t* st = base + (size_t)s * stage_bytes;
                    if (g >= pre) {
                        if (!mbar_wait(&empty_bar[s], ph ^ 1, e.status, 1, abort)) break;
                        mbar_expect_tx(&full_bar[s], na * atom_bytes);
                        for (int a = 0; a < na; a++) {
                            tma_load_2d(st + a * atom_bytes, &tm_w, &full_bar[s], (kb + a) * TC_BK, tc.n0);
                            if (GATED)
                                tma_load_2d(st + a * atom_bytes + w_bytes, &tm_w2, &full_bar[s], (kb + a) * TC_BK, tc.n0);
                        }
                    }
                    for (int a = 0; a < na; a++) {
                        uint8_t* xs = st + a * atom_bytes + w_bytes * (GATED ? 2 : 1);
                        int kc = (kb + a) * TC_BK, row = tc.m0;
                        if (e.conv_cin) {  // convolution: a K atom lies inside one tap (conv_cin % 64 == 0)
                            const int tap = kc / e.conv_cin, q = tap + e.conv_row0;
                            const int g = q / e.conv_group;
                            kc += (q - g * e.conv_group - tap) * e.conv_cin;
                            row += g;
                        }
                        if (e.x_planes) {  // both planes, one copy (their order is free: the epilogue sums them)
                            tma_load_3d(xs, &tm_xhi, &full_bar[s], kc, row, 0);
                        } else {
                            tma_load_2d(xs, &tm_xhi, &full_bar[s], kc, row);
                            tma_load_2d(xs + x_bytes, &tm_xlo, &full_bar[s], kc, row);
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer: one MMA of N = 2 bn per 16-wide K step per weight matrix
            const uint32_t idesc = idesc_bf16(TC_BM, 2 * e.bn);
            const uint64_t a_desc0 = sw128_desc(smem_u32(base));
            const uint64_t b_desc0 = sw128_desc(smem_u32(base) + w_bytes * (GATED ? 2 : 1));
            int s = 0, tl = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x; t < tiles_total && !*abort; t += gridDim.x, tl++) {
                const TileCoord tc = tile_coord(e, t);
                const int b = tl & 1;
                if (!mbar_wait(&acc_empty[b], ((tl >> 1) & 1) ^ 1, e.status, 2, abort)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + b * acc_cols;
                bool ok = true;
                for (int kb = tc.kb_begin, i = 0; kb < tc.kb_end; kb += KA, i++, s = s + 1 == S ? 0 : s + 1, ph ^= s == 0) {
                    const int na = KA == 1 ? 1 : min(KA, tc.kb_end - kb);
                    if (!mbar_wait(&full_bar[s], ph, e.status, 3, abort)) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    // Descriptors advance by offsets in their 16-byte address field (shared memory
                    // < 256 KB, so the field never carries into the other bits).
                    const uint64_t sd = (uint64_t)(((uint32_t)s * stage_bytes) >> 4);
#pragma unroll
                    for (int a = 0; a < KA; a++) {
                        if (KA > 1 && a >= na) break;
                        const uint64_t ad = a_desc0 + sd + (uint64_t)((a * atom_bytes) >> 4);
                        const uint64_t bd = b_desc0 + sd + (uint64_t)((a * atom_bytes) >> 4);
#pragma unroll
                        for (int kk = 0; kk < TC_BK / 16; kk++) {  // 16 bf16 along K = 32 bytes = 2 units
                            const uint32_t accum = (i > 0 || a > 0 || kk > 0) ? 1u : 0u;
                            mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc, accum);
                            if (GATED) mma_bf16(acc + 2 * e.bn, ad + (w_bytes >> 4) + 2 * kk, bd + 2 * kk, idesc, accum);
                        }
                    }
                    mma_commit(&empty_bar[s]);
                }
                if (!ok) break;
                mma_commit(&acc_full[b]);
            }
        }
    } else {  // epilogue warps 2..9: quadrant = warp % 4, the two warps of a quadrant alternate chunks
        const int quad = warp & 3, part = (warp - 2) >> 2;
        // Pull the epilogue's parameters and the first tile's bias into registers while the
        // previous kernel drains; a later tile's bias loads while its accumulator fills.
        asm volatile("" ::"r"(e.flags), "r"(e.m), "r"(e.n), "r"(e.bn), "l"(e.y), "l"(e.y_hi), "l"(e.bias));
        const int per_split = e.tiles_m * e.tiles_n;
        int t = blockIdx.x;
        float bval = t < tiles_total ? tile_bias(e, tile_coord(e, t).n0, quad, lane, t < per_split) : 0.f;
        pdl_wait();
        for (int tl = 0; t < tiles_total; t += gridDim.x, tl++) {
            const int b = tl & 1;
            if (!mbar_wait(&acc_full[b], (tl >> 1) & 1, e.status, 4, abort)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const TileCoord tc = tile_coord(e, t);
            if constexpr (KIND == EPI_GENERIC)
                epilogue_tile<GATED>(e, tc, tmem + b * acc_cols, quad, part, lane, t < per_split);
            else
                epilogue_fast<KIND, GATED>(e, tc, tmem + b * acc_cols, quad, part, lane, bval);
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
            const int tn = t + gridDim.x;
            if (KIND != EPI_GENERIC && tn < tiles_total) bval = tile_bias(e, tile_coord(e, tn).n0, quad, lane, tn < per_split);
        }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 2) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes a 256-weight-row tile with one
// tcgen05.mma.cta_group::2 (M = 256) per K step. The A operand (weights) is split by rows: CTA
// rank r holds weight rows n0 + 128 r; the B operand is split by columns: rank 0 holds the x_hi
// rows, rank 1 the x_lo rows of the same activation rows, so each CTA's shared memory carries one
// of the two activation planes and the per-CTA bytes per K block drop from W + 2X to W + X. Each
// CTA's TMEM holds its 128 weight rows x [hi | lo] columns, so the epilogue is the one above.
// Protocol: both producers' TMA loads complete on the leader's (rank 0) full barrier, whose
// expected bytes the leader arms for both; the leader's MMA commits arrive on the empty and
// accumulator-full barriers of both CTAs (commit multicast); both CTAs' epilogue warps arrive on
// the leader's accumulator-empty barrier. TMA loads never multicast. Every wait is bounded.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared::cluster address of `local` (a shared::cta variable) in the CTA of rank `rank`.
__device__ __forceinline__ uint32_t map_to_rank(const void* local, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
    return out;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA tile load into this CTA's shared memory, completing on the leader's barrier (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t leader_bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on the barrier at this offset in both CTAs of the pair when the leader's prior MMAs complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ TileCoord tile_coord_pair(const TcEpi& e, int t, int rank) {
    const int per_split = e.tiles_m * e.tiles_n;  // tiles_n counts 256-row pair tiles
    const int z = t / per_split, r = t % per_split;
    TileCoord c;
    c.m0 = (r % e.tiles_m) * e.bn;
    c.n0 = (r / e.tiles_m) * (2 * TC_BM) + rank * TC_BM;
    const int kb_total = (e.k + TC_BK - 1) / TC_BK;
    c.kb_begin = z * e.kb_per_split;
    c.kb_end = min(kb_total, c.kb_begin + e.kb_per_split);
    return c;
}

template <bool GATED>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                        const __grid_constant__ CUtensorMap tm_xhi, const __grid_constant__ CUtensorMap tm_xlo,
                        TcEpi e) {
    extern __shared__ __align__(1024) uint8_t dsmem[];
    __shared__ uint64_t full_bar[8], empty_bar[8], acc_full[2], acc_empty[2];
    __shared__ uint32_t tmem_holder;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const int S = e.stages;
    const int units = e.tiles_m * e.tiles_n * e.split;

    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
    const uint32_t w_bytes = TC_BM * 128, x_bytes = (uint32_t)e.bn * 128;
    const uint32_t stage_bytes = w_bytes * (GATED ? 2 : 1) + x_bytes;  // this CTA's share of a stage
    const uint32_t acc_cols = (uint32_t)e.bn * (GATED ? 4 : 2);
    uint32_t ncols = 32;
    while (ncols < 2 * acc_cols) ncols <<= 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * TC_EPI_WARPS);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_holder)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    cluster_sync_all();  // both CTAs' barriers exist before any remote arrive or load completes on them
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_holder;
    volatile int* abort = &abort_flag;
    pdl_launch();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer (both CTAs)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
            if (GATED) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w2)) : "memory");
            const CUtensorMap* tm_x = rank == 0 ? &tm_xhi : &tm_xlo;
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm_x)) : "memory");
            int pre = 0;
            for (int t = cluster; t < units && pre < S; t += nclusters) {
                const TileCoord tc = tile_coord_pair(e, t, rank);
                for (int kb = tc.kb_begin; kb < tc.kb_end && pre < S; kb++, pre++) {
                    uint8_t* st = base + (size_t)pre * stage_bytes;
                    if (rank == 0) mbar_expect_tx(&full_bar[pre], 2 * stage_bytes);
                    const uint32_t lb = map_to_rank(&full_bar[pre], 0);
                    tma_load_2d_pair(st, &tm_w, lb, kb * TC_BK, tc.n0);
                    if (GATED) tma_load_2d_pair(st + w_bytes, &tm_w2, lb, kb * TC_BK, tc.n0);
                }
            }
            pdl_wait();
            int g = 0;
            for (int t = cluster; t < units && !*abort; t += nclusters) {
                const TileCoord tc = tile_coord_pair(e, t, rank);
                for (int kb = tc.kb_begin; kb < tc.kb_end; kb++, g++) {
                    const int s = g % S;
                    uint8_t* st = base + (size_t)s * stage_bytes;
                    const int kc = kb * TC_BK;
                    const uint32_t lb = map_to_rank(&full_bar[s], 0);
                    if (g >= pre) {
                        if (!mbar_wait(&empty_bar[s], ((g / S) & 1) ^ 1, e.status, 11, abort)) break;
                        if (rank == 0) mbar_expect_tx(&full_bar[s], 2 * stage_bytes);
                        tma_load_2d_pair(st, &tm_w, lb, kc, tc.n0);
                        if (GATED) tma_load_2d_pair(st + w_bytes, &tm_w2, lb, kc, tc.n0);
                    }
                    tma_load_2d_pair(st + w_bytes * (GATED ? 2 : 1), tm_x, lb, kc, tc.m0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {  // MMA issuer: the leader only
            const uint32_t idesc = idesc_bf16(2 * TC_BM, 2 * e.bn);
            int g = 0, tl = 0;
            for (int t = cluster; t < units && !*abort; t += nclusters, tl++) {
                const TileCoord tc = tile_coord_pair(e, t, 0);
                const int b = tl & 1;
                if (!mbar_wait(&acc_empty[b], ((tl >> 1) & 1) ^ 1, e.status, 12, abort)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + b * acc_cols;
                bool ok = true;
                for (int kb = tc.kb_begin, i = 0; kb < tc.kb_end; kb++, i++, g++) {
                    const int s = g % S;
                    if (!mbar_wait(&full_bar[s], (g / S) & 1, e.status, 13, abort)) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t wa = smem_u32(base + (size_t)s * stage_bytes);
                    const uint32_t xa = wa + w_bytes * (GATED ? 2 : 1);
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; kk++) {
                        const uint32_t off = kk * 32;
                        const uint64_t bx = sw128_desc(xa + off);
                        const uint32_t accum = (i > 0 || kk > 0) ? 1u : 0u;
                        mma_bf16_pair(acc, sw128_desc(wa + off), bx, idesc, accum);
                        if (GATED) mma_bf16_pair(acc + 2 * e.bn, sw128_desc(wa + w_bytes + off), bx, idesc, accum);
                    }
                    mma_commit_pair(&empty_bar[s]);
                }
                if (!ok) break;
                mma_commit_pair(&acc_full[b]);
            }
        }
    } else {  // epilogue warps 2..9 of both CTAs, each on its own TMEM rows
        const int quad = warp & 3, part = (warp - 2) >> 2;
        asm volatile("" ::"r"(e.kind), "r"(e.flags), "r"(e.m), "r"(e.n), "r"(e.bn), "l"(e.y), "l"(e.y_hi),
                     "l"(e.bias));
        pdl_wait();
        int tl = 0;
        for (int t = cluster; t < units; t += nclusters, tl++) {
            const int b = tl & 1;
            if (!mbar_wait(&acc_full[b], (tl >> 1) & 1, e.status, 14, abort)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const TileCoord tc = tile_coord_pair(e, t, rank);
            epilogue_dispatch<GATED>(e, tc, tmem + b * acc_cols, quad, part, lane, t < e.tiles_m * e.tiles_n);
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(map_to_rank(&acc_empty[b], 0));
        }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    cluster_sync_all();  // neither CTA leaves while the pair's MMAs or remote arrives may touch it
    if (warp == 2) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

// Finishes a split-K GEMM whose epilogue is nonlinear: y = epi(ws (+ bias)) from the fp32 sums.
__global__ void split_epilogue_kernel(TcEpi e) {
    pdl_wait();
    pdl_launch();
    const long long total = (long long)e.m * e.n;
    const bool gated = (e.flags & MT_LINEAR_SILU_GATE) != 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / e.n), n = (int)(i % e.n);
        float val = e.ws[(size_t)m * e.ldws + n];
        if (e.flags & MT_LINEAR_BIAS) val += bf16f(e.bias[n]);
        if (gated) val = silu(val) * e.ws[(size_t)m * e.ldws + e.n + n];
        if (e.flags & MT_LINEAR_GELU) val = gelu_tanh(val);
        if (e.flags & MT_LINEAR_SILU) val = silu(val);
        if (e.y) {
            float* yp = e.y + (size_t)m * e.ldy + n;
            if (e.flags & MT_LINEAR_ACCUM) val += *yp;
            *yp = val;
        }
        if (e.y_hi) {
            uint16_t h, l;
            split_bf16(val, h, l);
            e.y_hi[(size_t)m * e.ld_ysplit + n] = h;
            e.y_lo[(size_t)m * e.ld_ysplit + n] = l;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// Host side: tensor maps and launch configuration.
// ------------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D bf16 map over a [rows, cols] matrix with row stride ld elements; box = 64 cols x box_rows.
static bool make_map(CUtensorMap* map, const void* ptr, int rows, int cols, int ld, int box_rows) {
    auto enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 3-D map over both activation planes: [plane][rows][cols] with the planes |x_lo - x_hi| bytes
// apart, based at the lower one; box = 64 cols x box_rows x 2 planes, so one TMA copy fills a
// stage's [plane 0 rows | plane 1 rows] (an SM's TMA takes a few hundred cycles per copy, so a
// stage's copies, not its bytes, set the pace of small GEMMs). False where TMA cannot address it.
static bool make_planes_map(CUtensorMap* map, const void* hi, const void* lo, int rows, int cols, int ld, int box_rows) {
    const uintptr_t a = (uintptr_t)hi, b = (uintptr_t)lo;
    const uintptr_t base = a < b ? a : b, gap = a < b ? b - a : a - b;
    if (gap == 0 || (gap & 15u) || gap >= ((uintptr_t)1 << 40)) return false;
    auto enc = get_encode();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, 2};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)gap};
    cuuint32_t box[3] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows, 2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, reinterpret_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

static int round16(int v) { return (v + 15) & ~15; }

// The compile-time epilogue for this plan's flags and outputs, or EPI_GENERIC.
static int epi_kind(const TcEpi& e, bool gated) {
    const uint32_t act = e.flags & (MT_LINEAR_GELU | MT_LINEAR_SILU);
    const bool accum = (e.flags & MT_LINEAR_ACCUM) != 0;
    const bool f32 = e.y != nullptr, split = e.y_hi != nullptr;
    if (e.mode == 1) return EPI_RED;  // split-K of a linear epilogue into fp32 y
    if (e.mode != 0) return EPI_GENERIC;
    if (e.split_silu) {
        if (gated || act || !split) return EPI_GENERIC;
        if (!f32) return accum ? EPI_GENERIC : EPI_SSILU;
        return accum ? EPI_ACC_SSILU : EPI_F32_SSILU;
    }
    if (gated) return (!act && !accum && split && !f32) ? EPI_SPLIT_GATE : EPI_GENERIC;
    if (f32 && !split) {
        if (!act) return accum ? EPI_F32_ACCUM : EPI_F32;
        if (act == MT_LINEAR_SILU && !accum) return EPI_F32_SILU;
        return EPI_GENERIC;
    }
    if (split && !f32 && !accum) {
        if (!act) return EPI_SPLIT;
        if (act == MT_LINEAR_GELU) return EPI_SPLIT_GELU;
    }
    return EPI_GENERIC;
}

using GemmKernel = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, TcEpi);

template <int KA>
static GemmKernel gemm_kernel_ka(bool gated, int kind) {
    if (gated)
        return kind == EPI_SPLIT_GATE ? gemm_tc_kernel<true, EPI_SPLIT_GATE, KA> : gemm_tc_kernel<true, EPI_GENERIC, KA>;
    switch (kind) {
        case EPI_F32: return gemm_tc_kernel<false, EPI_F32, KA>;
        case EPI_F32_ACCUM: return gemm_tc_kernel<false, EPI_F32_ACCUM, KA>;
        case EPI_SPLIT: return gemm_tc_kernel<false, EPI_SPLIT, KA>;
        case EPI_SPLIT_GELU: return gemm_tc_kernel<false, EPI_SPLIT_GELU, KA>;
        case EPI_F32_SILU: return gemm_tc_kernel<false, EPI_F32_SILU, KA>;
        case EPI_RED: return gemm_tc_kernel<false, EPI_RED, KA>;
        case EPI_F32_SSILU: return gemm_tc_kernel<false, EPI_F32_SSILU, KA>;
        case EPI_ACC_SSILU: return gemm_tc_kernel<false, EPI_ACC_SSILU, KA>;
        case EPI_SSILU: return gemm_tc_kernel<false, EPI_SSILU, KA>;
        default: return gemm_tc_kernel<false, EPI_GENERIC, KA>;
    }
}

// The kernel instantiation for a plan: gated plans have the gate epilogue or the generic one.
static GemmKernel gemm_kernel_for(bool gated, int kind, int ka) {
    return ka == 2 ? gemm_kernel_ka<2>(gated, kind) : gemm_kernel_ka<1>(gated, kind);
}

// Shared-memory opt-in for every instantiation, once per device (the attribute belongs to the
// function in the current device's context).
static void set_gemm_attributes() {
    static PerDeviceOnce once;
    once([] {
        const int kinds[] = {EPI_GENERIC, EPI_F32,   EPI_F32_ACCUM, EPI_SPLIT,     EPI_SPLIT_GELU, EPI_SPLIT_GATE,
                             EPI_F32_SILU, EPI_RED, EPI_F32_SSILU, EPI_ACC_SSILU, EPI_SSILU};
        for (int kd : kinds) {
            for (int ka = 1; ka <= TC_KA_MAX; ka++) {
                cudaFuncSetAttribute(gemm_kernel_for(false, kd, ka), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     201 * 1024);
                cudaFuncSetAttribute(gemm_kernel_for(true, kd, ka), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     201 * 1024);
            }
        }
        cudaFuncSetAttribute(gemm_tc_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 201 * 1024);
        cudaFuncSetAttribute(gemm_tc_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 201 * 1024);
    });
}

mt_status make_gemm_plan(mt_ctx* ctx, const LinearArgs& a, GemmPlan* plan) {
    const bool gated = (a.flags & MT_LINEAR_SILU_GATE) != 0;
    MT_REQUIRE(ctx, a.m > 0 && a.n > 0 && a.k > 0, MT_ERR_SHAPE, "gemm_tc: empty shape m %d n %d k %d", a.m, a.n, a.k);
    MT_REQUIRE(ctx, a.k % 8 == 0 && a.ld_split % 8 == 0 && (a.ld_split >= a.k || a.conv_cin > 0), MT_ERR_SHAPE,
               "gemm_tc: k %d ld %d need multiples of 8", a.k, a.ld_split);
    MT_REQUIRE(ctx, ((uintptr_t)a.w & 15u) == 0 && ((uintptr_t)a.x_hi & 15u) == 0 && ((uintptr_t)a.x_lo & 15u) == 0 &&
                        (!gated || ((uintptr_t)a.w2 & 15u) == 0),
               MT_ERR_ARG, "gemm_tc: operands need 16-byte alignment");
    MT_REQUIRE(ctx, a.y || a.y_hi, MT_ERR_ARG, "gemm_tc: no output");
    MT_REQUIRE(ctx, !(a.flags & MT_LINEAR_BIAS) || a.bias, MT_ERR_ARG, "gemm_tc: BIAS needs bias");
    MT_REQUIRE(ctx, !(a.flags & MT_LINEAR_ACCUM) || a.y, MT_ERR_ARG, "gemm_tc: ACCUM needs fp32 y");
    const bool conv = a.conv_cin > 0;
    MT_REQUIRE(ctx, !conv || (a.conv_cin % TC_BK == 0 && a.k % a.conv_cin == 0 && a.conv_row0 >= 0 && a.x_rows > 0 &&
                              a.ld_split >= a.conv_cin && !gated),
               MT_ERR_SHAPE, "gemm_tc: convolution channels %d (multiple of 64 dividing k %d), row offset %d, rows %d",
               a.conv_cin, a.k, a.conv_row0, a.x_rows);
    TcEpi& e = plan->e;
    e = TcEpi{};
    e.m = a.m; e.n = a.n; e.k = a.k;
    e.conv_cin = conv ? a.conv_cin : 0;
    e.conv_row0 = conv ? a.conv_row0 : 0;
    e.conv_group = conv && a.conv_group > 1 ? a.conv_group : 1;
    e.split_silu = a.split_silu ? 1 : 0;
    const bool linear = !(a.flags & (MT_LINEAR_GELU | MT_LINEAR_SILU | MT_LINEAR_SILU_GATE)) && a.y && !a.y_hi;
    // Split-K by default only where partial sums can be reduced into y without zeroing it first
    // (ACCUM: y holds the residual). Tile rows measured on the engine's shapes: narrow tiles for few
    // rows (more CTAs), 128 rows once M is large (fewer weight re-reads through L2).
    const bool splittable = linear && (a.flags & MT_LINEAR_ACCUM) && !conv && !a.split_silu;
    const int kb_total = (a.k + TC_BK - 1) / TC_BK;
    const int sms = ctx->sm_count > 0 ? ctx->sm_count : 148;
    const int n_tiles128 = (a.n + TC_BM - 1) / TC_BM;
    if (a.bn_override > 0) e.bn = a.bn_override;
    else if (a.m <= 32) e.bn = round16(a.m);
    else if (splittable) e.bn = a.m <= 64 ? 32 : a.m <= 128 ? 64 : (a.m > 256 && kb_total <= 16) ? 64 : 128;
    else e.bn = a.m <= 128 ? 32 : a.m <= 256 ? 64 : a.m <= 384 ? 96 : 128;
    // 257-384 rows: 64-row tiles (two K atoms per stage) where they still fit one wave; measured
    // against 96-row tiles at the flow-DiT qkv shape, 7.9 vs 9.3 us.
    if (a.bn_override <= 0 && !splittable && a.m > 256 && a.m <= 384 && !(a.flags & MT_LINEAR_SILU_GATE) &&
        n_tiles128 * ((a.m + 63) / 64) <= sms)
        e.bn = 64;
    if (e.bn < 16) e.bn = 16;
    if (gated && e.bn > 64 && a.bn_override <= 0) e.bn = 64;  // two gated accumulators x 2 buffers fit 512 columns
    MT_REQUIRE(ctx, e.bn % 16 == 0 && e.bn <= (gated ? 64 : 128), MT_ERR_SHAPE, "gemm_tc: tile rows %d (16..%d)", e.bn,
               gated ? 64 : 128);
    // CTA pairs (256 weight rows per tile, one activation plane per CTA): on request only for now.
    const bool pair = ctx->gemm_pairs == 1 && !conv;
    const int tile_rows = pair ? 2 * TC_BM : TC_BM;
    const int tiles_n = (a.n + tile_rows - 1) / tile_rows;
    const int slots = pair ? sms / 2 : sms;  // concurrent work units
    // Two K atoms per stage where three such stages still fit (the MMA thread's fixed cost per stage
    // is then spread over twice the MMAs), one otherwise (fewer bytes in flight lost more than the
    // round trips saved at the 96- and 128-row tiles of the flow DiT).
    const uint32_t atom_bytes = TC_BM * 128 * (gated ? 2 : 1) + 2u * e.bn * 128;
    e.ka = !pair && 3 * TC_KA_MAX * atom_bytes <= 200 * 1024 ? TC_KA_MAX : 1;
    const uint32_t stage_bytes = pair ? TC_BM * 128 * (gated ? 2 : 1) + e.bn * 128 : e.ka * atom_bytes;
    const int tiles = tiles_n * ((a.m + e.bn - 1) / e.bn);
    e.stages = (int)((200 * 1024) / stage_bytes);
    if (e.stages > 8) e.stages = 8;
    if (e.stages < 2) e.stages = 2;
    MT_REQUIRE(ctx, (size_t)e.stages * stage_bytes + 1024 <= 201 * 1024, MT_ERR_SHAPE, "gemm_tc: tile too large");
    int split = a.split_k;
    if (split <= 0) {  // automatic: one wave (work units <= SMs), at least two k blocks each, at most 8 splits
        split = splittable ? slots / tiles : 1;
        if (split > 8) split = 8;
        if (split > kb_total / 2) split = kb_total / 2;
    }
    if (split < 1) split = 1;
    if (split > kb_total) split = kb_total;
    e.kb_per_split = (kb_total + split - 1) / split;
    split = (kb_total + e.kb_per_split - 1) / e.kb_per_split;
    MT_REQUIRE(ctx, split == 1 || linear || a.ws, MT_ERR_ARG,
               "gemm_tc: split-K with a nonlinear epilogue needs a workspace");
    e.split = split;
    e.mode = split == 1 ? 0 : (linear ? 1 : 2);
    e.tiles_n = tiles_n;
    e.tiles_m = (a.m + e.bn - 1) / e.bn;
    e.bias = a.bias; e.y = a.y; e.ldy = a.ldy; e.y_hi = a.y_hi; e.y_lo = a.y_lo; e.ld_ysplit = a.ld_ysplit;
    e.ws = a.ws; e.ldws = gated ? 2 * a.n : a.n;
    e.flags = a.flags; e.status = ctx->d_status;
    e.kind = epi_kind(e, gated);

    bool ok = make_map(&plan->tw, a.w, a.n, a.k, a.k, TC_BM);
    ok = ok && make_map(&plan->tw2, gated ? a.w2 : a.w, a.n, a.k, a.k, TC_BM);
    const int x_rows = conv ? a.x_rows : a.m, x_cols = conv ? a.conv_cin * e.conv_group : a.k;
    MT_REQUIRE(ctx, !conv || a.ld_split >= x_cols, MT_ERR_SHAPE, "gemm_tc: convolution row stride %d < %d",
               a.ld_split, x_cols);
    ok = ok && make_map(&plan->tl, a.x_lo, x_rows, x_cols, a.ld_split, e.bn);
    e.x_planes = !pair && make_planes_map(&plan->th, a.x_hi, a.x_lo, x_rows, x_cols, a.ld_split, e.bn) ? 1 : 0;
    if (!e.x_planes) ok = ok && make_map(&plan->th, a.x_hi, x_rows, x_cols, a.ld_split, e.bn);
    MT_REQUIRE(ctx, ok, MT_ERR_CUDA, "gemm_tc: cuTensorMapEncodeTiled failed (m %d n %d k %d)", a.m, a.n, a.k);
    plan->gated = gated;
    plan->pair = pair;
    plan->smem = (size_t)e.stages * stage_bytes + 1024;
    const int work = e.tiles_n * e.tiles_m * split;
    plan->grid = dim3((pair ? 2 : 1) * (work < slots ? work : slots), 1, 1);
    set_gemm_attributes();
    return MT_OK;
}

// Plan for callers without a context (mt_linear_static): no split-K, no error strings; returns
// MT_ERR_CUDA only if a tensor map cannot be encoded. Inputs are validated by the caller, which
// also sets e.status (the plan leaves it null: a wait that gives up then records nothing).
mt_status make_gemm_plan_bare(int sm_count, const LinearArgs& a, GemmPlan* plan) {
    const bool gated = (a.flags & MT_LINEAR_SILU_GATE) != 0;
    TcEpi& e = plan->e;
    e = TcEpi{};
    e.m = a.m; e.n = a.n; e.k = a.k;
    const int sms = sm_count > 0 ? sm_count : 148;
    e.tiles_n = (a.n + TC_BM - 1) / TC_BM;
    e.bn = a.m <= 32 ? round16(a.m) : a.m <= 128 ? 32 : a.m <= 256 ? 64 : 128;
    if (e.bn < 16) e.bn = 16;
    if (gated && e.bn > 64) e.bn = 64;
    e.tiles_m = (a.m + e.bn - 1) / e.bn;
    e.ka = 1;
    const uint32_t stage_bytes = TC_BM * 128 * (gated ? 2 : 1) + 2u * e.bn * 128;
    e.stages = (int)((200 * 1024) / stage_bytes);
    if (e.stages > 8) e.stages = 8;
    const int kb_total = (a.k + TC_BK - 1) / TC_BK;
    e.kb_per_split = kb_total;
    e.split = 1;
    e.mode = 0;
    e.bias = a.bias; e.y = a.y; e.ldy = a.ldy; e.y_hi = a.y_hi; e.y_lo = a.y_lo; e.ld_ysplit = a.ld_ysplit;
    e.flags = a.flags;
    e.status = nullptr;
    e.kind = epi_kind(e, gated);
    bool ok = make_map(&plan->tw, a.w, a.n, a.k, a.k, TC_BM);
    ok = ok && make_map(&plan->tw2, gated ? a.w2 : a.w, a.n, a.k, a.k, TC_BM);
    ok = ok && make_map(&plan->th, a.x_hi, a.m, a.k, a.ld_split, e.bn);
    ok = ok && make_map(&plan->tl, a.x_lo, a.m, a.k, a.ld_split, e.bn);
    if (!ok) return MT_ERR_CUDA;
    plan->gated = gated;
    plan->pair = false;
    plan->smem = (size_t)e.stages * stage_bytes + 1024;
    const int work = e.tiles_n * e.tiles_m;
    plan->grid = dim3(work < sms ? work : sms, 1, 1);
    set_gemm_attributes();
    return MT_OK;
}

void run_gemm_plan(const GemmPlan& p, cudaStream_t s) {
    const TcEpi& e = p.e;
    if (e.mode == 1 && !(e.flags & MT_LINEAR_ACCUM))
        cudaMemset2DAsync(e.y, (size_t)e.ldy * sizeof(float), 0, (size_t)e.n * sizeof(float), e.m, s);
    if (e.mode == 2) cudaMemsetAsync(e.ws, 0, (size_t)e.m * e.ldws * sizeof(float), s);
    if (p.pair) {
        if (p.gated)
            launch_k_pair(gemm_tc_pair_kernel<true>, p.grid, TC_THREADS, p.smem, s, p.tw, p.tw2, p.th, p.tl, p.e);
        else
            launch_k_pair(gemm_tc_pair_kernel<false>, p.grid, TC_THREADS, p.smem, s, p.tw, p.tw2, p.th, p.tl, p.e);
    } else {
        launch_k(gemm_kernel_for(p.gated, e.kind, e.ka), p.grid, TC_THREADS, p.smem, s, p.tw, p.tw2, p.th, p.tl, p.e);
    }
    if (e.mode == 2) {
        const long long total = (long long)e.m * e.n;
        long long blocks = (total + 255) / 256;
        if (blocks > 148 * 8) blocks = 148 * 8;
        launch_k(split_epilogue_kernel, (unsigned)blocks, 256, 0, s, e);
    }
}

mt_status launch_gemm_tc(mt_ctx* ctx, const LinearArgs& a, cudaStream_t s) {
    GemmPlan plan;
    mt_status st = make_gemm_plan(ctx, a, &plan);
    if (st != MT_OK) return st;
    run_gemm_plan(plan, s);
    return check_launch(ctx, "gemm_tc");
}

}  // namespace mt
