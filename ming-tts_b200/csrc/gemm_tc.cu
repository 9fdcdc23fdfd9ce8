// gemm_tc.cu -- tcgen05 / TMEM tensor-core GEMM for sm_100a:
//     Y[m, n] = epi( sum_k X[m, k] * W[n, k] )  with X fp32 carried as two bf16 planes (hi + lo).
//
// Reference semantics: the tiled GEMM and gemm8 kernels (Shaders.swift:191-277, 304-408) -- fp32
// activations times bf16 weights with fp32 accumulation and the linear epilogue. Tensor cores
// take bf16 operands, so the activations enter as x = hi + lo (both bf16, |x - hi - lo| <= 2^-17|x|)
// and every K step issues two MMAs (W.hi, W.lo) into the same fp32 TMEM accumulator; the
// weights are exact in bf16. The result matches fp32 FMA accumulation to ~1e-5 relative.
//
// Layout ("swap AB"): the MMA's M side is 128 weight rows (output columns n), its N side is up to
// 256 activation rows (m), so small row counts still use full 128-lane MMAs. The accumulator is
// D[n_local][m_local] in TMEM (lane = weight row, column = activation row); the epilogue warp w
// owns TMEM lanes 32w..32w+31 and writes Y rows coalesced along n.
//
// Pipeline: warp 0 lane 0 issues TMA loads (128B swizzle, no multicast) into a ring of stages;
// warp 1 lane 0 issues tcgen05.mma and frees each stage with tcgen05.commit; all four warps run the
// epilogue once the final commit lands. Every mbarrier wait is bounded: a wait that gives up
// writes the context status word and the block skips the rest of its work.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"

namespace mt {

constexpr int TC_THREADS = 128;
constexpr int TC_BM = 128;  // weight rows per tile (MMA M)
constexpr int TC_BK = 64;   // bf16 K per stage = one 128-byte swizzle span
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s per wait



__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on the phase with the given parity: gives up after WAIT_NS of wall time (checked
// every 256 polls), records the site in the status word and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* status, unsigned site) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t i = 0;; i++) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(addr), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 255u) == 0) {
            const uint64_t now = global_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > WAIT_NS) break;
        }
    }
    report_status(status, DEV_TIMEOUT, site, blockIdx.x | (blockIdx.y << 16));
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

template <bool GATED>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                   const __grid_constant__ CUtensorMap tm_xhi, const __grid_constant__ CUtensorMap tm_xlo, TcEpi e) {
    extern __shared__ __align__(1024) uint8_t dsmem[];
    __shared__ uint64_t full_bar[8], empty_bar[8], done_bar;
    __shared__ uint32_t tmem_holder;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * TC_BM, m0 = blockIdx.y * e.bn;
    const int kb_total = (e.k + TC_BK - 1) / TC_BK;
    const int kb_begin = blockIdx.z * e.kb_per_split;
    const int kb_end = min(kb_total, kb_begin + e.kb_per_split);
    const int S = e.stages;

    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
    const uint32_t w_bytes = TC_BM * 128, x_bytes = (uint32_t)e.bn * 128;
    const uint32_t stage_bytes = w_bytes * (GATED ? 2 : 1) + 2 * x_bytes;
    const uint32_t ncols_acc = (uint32_t)e.bn * (GATED ? 2 : 1);
    uint32_t ncols = 32;
    while (ncols < ncols_acc) ncols <<= 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&done_bar, 1);
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

    if (warp == 0 && lane == 0) {
        // TMA producer.
        for (int kb = kb_begin, i = 0; kb < kb_end; kb++, i++) {
            const int s = i % S;
            if (!mbar_wait(&empty_bar[s], ((i / S) & 1) ^ 1, e.status, 1)) { abort_flag = 1; break; }
            if (*(volatile int*)&abort_flag) break;
            uint8_t* st = base + (size_t)s * stage_bytes;
            mbar_expect_tx(&full_bar[s], stage_bytes);
            const int kc = kb * TC_BK;
            tma_load_2d(st, &tm_w, &full_bar[s], kc, n0);
            if (GATED) tma_load_2d(st + w_bytes, &tm_w2, &full_bar[s], kc, n0);
            uint8_t* xs = st + w_bytes * (GATED ? 2 : 1);
            tma_load_2d(xs, &tm_xhi, &full_bar[s], kc, m0);
            tma_load_2d(xs + x_bytes, &tm_xlo, &full_bar[s], kc, m0);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer.
        const uint32_t idesc = idesc_bf16(TC_BM, e.bn);
        bool ok = true;
        for (int kb = kb_begin, i = 0; kb < kb_end; kb++, i++) {
            const int s = i % S;
            if (!mbar_wait(&full_bar[s], (i / S) & 1, e.status, 2)) { ok = false; abort_flag = 1; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint8_t* st = base + (size_t)s * stage_bytes;
            const uint32_t wa = smem_u32(st);
            const uint32_t w2a = wa + w_bytes;
            const uint32_t xa = wa + w_bytes * (GATED ? 2 : 1);
            const uint32_t xla = xa + x_bytes;
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; kk++) {
                const uint32_t off = kk * 32;  // 16 bf16 along K inside the swizzle span
                const uint64_t ad = sw128_desc(wa + off);
                const uint64_t bh = sw128_desc(xa + off), bl = sw128_desc(xla + off);
                const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                mma_bf16(tmem, ad, bh, idesc, acc);
                mma_bf16(tmem, ad, bl, idesc, 1u);
                if (GATED) {
                    const uint64_t ad2 = sw128_desc(w2a + off);
                    mma_bf16(tmem + e.bn, ad2, bh, idesc, acc);
                    mma_bf16(tmem + e.bn, ad2, bl, idesc, 1u);
                }
            }
            mma_commit(&empty_bar[s]);
        }
        if (ok) mma_commit(&done_bar);
    }
    __syncwarp();

    // Epilogue: all four warps; warp w owns accumulator lanes (weight rows) 32w..32w+31.
    const bool have = mbar_wait(&done_bar, 0, e.status, 3);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (have) {
        const int n = n0 + warp * 32 + lane;
        const bool live_n = n < e.n;
        const bool first_split = blockIdx.z == 0;
        const float bval = ((e.flags & MT_LINEAR_BIAS) && live_n && first_split) ? bf16f(e.bias[n]) : 0.f;
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        for (int c0 = 0; c0 < e.bn; c0 += 16) {
            float v[16], v2[16];
            tmem_ld16(lane_base + c0, v);
            if (GATED) tmem_ld16(lane_base + e.bn + c0, v2);
            if (!live_n) continue;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int m = m0 + c0 + j;
                if (m >= e.m) break;
                float val = v[j] + bval;
                if (e.split > 1) {
                    atomicAdd(e.y + (size_t)m * e.ldy + n, val);
                    continue;
                }
                if (GATED) val = silu(val) * v2[j];
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
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 2) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
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

static int round16(int v) { return (v + 15) & ~15; }

mt_status make_gemm_plan(mt_ctx* ctx, const LinearArgs& a, GemmPlan* plan) {
    const bool gated = (a.flags & MT_LINEAR_SILU_GATE) != 0;
    MT_REQUIRE(ctx, a.m > 0 && a.n > 0 && a.k > 0, MT_ERR_SHAPE, "gemm_tc: empty shape m %d n %d k %d", a.m, a.n, a.k);
    MT_REQUIRE(ctx, a.k % 8 == 0 && a.ld_split % 8 == 0 && a.ld_split >= a.k, MT_ERR_SHAPE,
               "gemm_tc: k %d ld %d need multiples of 8", a.k, a.ld_split);
    MT_REQUIRE(ctx, ((uintptr_t)a.w & 15u) == 0 && ((uintptr_t)a.x_hi & 15u) == 0 && ((uintptr_t)a.x_lo & 15u) == 0 &&
                        (!gated || ((uintptr_t)a.w2 & 15u) == 0),
               MT_ERR_ARG, "gemm_tc: operands need 16-byte alignment");
    MT_REQUIRE(ctx, a.y || a.y_hi, MT_ERR_ARG, "gemm_tc: no output");
    MT_REQUIRE(ctx, !(a.flags & MT_LINEAR_BIAS) || a.bias, MT_ERR_ARG, "gemm_tc: BIAS needs bias");
    MT_REQUIRE(ctx, !(a.flags & MT_LINEAR_ACCUM) || a.y, MT_ERR_ARG, "gemm_tc: ACCUM needs fp32 y");
    TcEpi& e = plan->e;
    e = TcEpi{};
    e.m = a.m; e.n = a.n; e.k = a.k;
    e.bn = a.bn_override > 0 ? a.bn_override : (a.m <= 256 ? round16(a.m) : 128);
    if (e.bn < 16) e.bn = 16;
    MT_REQUIRE(ctx, e.bn % 16 == 0 && e.bn <= 256, MT_ERR_SHAPE, "gemm_tc: tile rows %d", e.bn);
    const uint32_t stage_bytes = TC_BM * 128 * (gated ? 2 : 1) + 2u * e.bn * 128;
    const uint32_t budget = 200 * 1024;
    e.stages = (int)(budget / stage_bytes);
    if (e.stages > 8) e.stages = 8;
    MT_REQUIRE(ctx, e.stages >= 2, MT_ERR_SHAPE, "gemm_tc: tile too large");
    const int kb_total = (a.k + TC_BK - 1) / TC_BK;
    int split = a.split_k < 1 ? 1 : a.split_k;
    if (split > kb_total) split = kb_total;
    e.kb_per_split = (kb_total + split - 1) / split;
    split = (kb_total + e.kb_per_split - 1) / e.kb_per_split;
    MT_REQUIRE(ctx, split == 1 || (!gated && !(a.flags & (MT_LINEAR_GELU | MT_LINEAR_SILU)) && a.y && !a.y_hi),
               MT_ERR_ARG, "gemm_tc: split-K needs a linear epilogue into fp32 y");
    e.split = split;
    e.bias = a.bias; e.y = a.y; e.ldy = a.ldy; e.y_hi = a.y_hi; e.y_lo = a.y_lo; e.ld_ysplit = a.ld_ysplit;
    e.flags = a.flags; e.status = ctx->d_status;

    bool ok = make_map(&plan->tw, a.w, a.n, a.k, a.k, TC_BM);
    ok = ok && make_map(&plan->tw2, gated ? a.w2 : a.w, a.n, a.k, a.k, TC_BM);
    ok = ok && make_map(&plan->th, a.x_hi, a.m, a.k, a.ld_split, e.bn);
    ok = ok && make_map(&plan->tl, a.x_lo, a.m, a.k, a.ld_split, e.bn);
    MT_REQUIRE(ctx, ok, MT_ERR_CUDA, "gemm_tc: cuTensorMapEncodeTiled failed (m %d n %d k %d)", a.m, a.n, a.k);
    plan->gated = gated;
    plan->smem = (size_t)e.stages * stage_bytes + 1024;
    plan->grid = dim3((a.n + TC_BM - 1) / TC_BM, (a.m + e.bn - 1) / e.bn, split);
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(gemm_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 201 * 1024);
        cudaFuncSetAttribute(gemm_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 201 * 1024);
        attr_set = true;
    }
    return MT_OK;
}

void run_gemm_plan(const GemmPlan& p, cudaStream_t s) {
    if (p.gated)
        gemm_tc_kernel<true><<<p.grid, TC_THREADS, p.smem, s>>>(p.tw, p.tw2, p.th, p.tl, p.e);
    else
        gemm_tc_kernel<false><<<p.grid, TC_THREADS, p.smem, s>>>(p.tw, p.tw2, p.th, p.tl, p.e);
}

mt_status launch_gemm_tc(mt_ctx* ctx, const LinearArgs& a, cudaStream_t s) {
    GemmPlan plan;
    mt_status st = make_gemm_plan(ctx, a, &plan);
    if (st != MT_OK) return st;
    run_gemm_plan(plan, s);
    return check_launch(ctx, "gemm_tc");
}

}  // namespace mt
