// decode.cu -- mt_qwen_decode: one decode pass of a Qwen stack for a few rows (<= 8 in all).
//
// Reference: QwenForward.dispatches (Sources/MingTTS/Engine/Qwen.swift:72-97) as the LLM decode
// token runs it (one row, Engine.swift:381-385) and as the VAE decoder runs its four frame rows
// (VAEDecoder.swift:86-107), over caller-owned fp32 KV caches in the reference's layout
// (Qwen.swift:7-26). Per layer: RMSNorm -> q/k/v GEMV (+bias) -> RoPE + KV append + attention ->
// o GEMV (+=) -> RMSNorm -> gate/up GEMV (SiLU gate) -> down GEMV (+=); then the final norm of every
// row. Each RMSNorm is folded into the CUDA-core linear that consumes it (gains 16-byte aligned).
// From 3 rows the residual linears (o, down) run on the tensor cores with split K, and from 5 rows
// the gate/up linear too (behind a norm launch that writes its bf16 planes): the routes the engine
// measured for these shapes. Passes that fit run as one launch of the persistent stack kernel
// (stack.cu) when the context asks for it; the others as one launch per kernel above.
#include "common.cuh"
#include "kernels.cuh"

namespace mt {

namespace {

constexpr int kDecodeMaxRows = 8;  // rows of all requests together: the CUDA-core GEMV route

// Scratch of one call, carved from the context's scratch area (fp32): normed rows, q/k/v rows,
// attention rows and the gated MLP rows.
struct Planes {  // bf16 hi/lo planes of M rows (the tensor-core route's input or output)
    uint16_t *hi, *lo;
    int ld;
};
struct DecodeScratch {
    float *normed, *qkv, *attn, *mlp;
    Planes p_norm, p_attn, p_mlp;
};

// Rows from which the residual linears (o, down) and the gate/up linear take the tensor cores.
// Config 2 in graph replay: 8 rows 1164 -> 857 us with both; from 2 rows the residual route was
// 717 against 703 us, so two rows stay on the GEMV.
constexpr int kTcResidualRows = 3;
constexpr int kTcGateUpRows = 5;

size_t decode_scratch_floats(const mt_qwen_config& c, int M) {
    const size_t qkvw = (size_t)(c.heads + 2 * c.kv_heads) * 64;
    auto up = [](size_t n) { return (n + 63) & ~size_t(63); };  // 256-byte aligned pieces
    // fp32 rows, then the plane pairs (two bf16 planes of M x ld take M x ld floats)
    return 2 * (up((size_t)M * c.hidden) + up((size_t)M * c.heads * 64) + up((size_t)M * c.intermediate)) +
           up((size_t)M * qkvw);
}

bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

// The persistent stack kernel's view of the call (without its area), or false when it does not
// apply (shape limits, unaligned weights, or the context's choice).
bool stack_params(mt_ctx* ctx, const mt_qwen_weights* w, int requests, int rows, float* x, float* kv, long long kv_stride,
                  int capacity, const int32_t* positions, float* z, const float* inv_freq, StackParams* out) {
    const mt_qwen_config& c = w->cfg;
    if (ctx->persistent == 0 || c.layers > STACK_MAX_LAYERS) return false;
    StackParams& p = *out;
    p = StackParams{};
    p.kind = STACK_QWEN; p.layers = c.layers; p.M = requests * rows; p.seq_rows = rows; p.seqs = requests;
    p.hidden = c.hidden; p.heads = c.heads; p.kv_heads = c.kv_heads; p.inter = c.intermediate; p.eps = c.eps;
    p.window = c.window; p.cap = capacity; p.kv_stride = kv_stride; p.pos = positions; p.kv = kv; p.inv_freq = inv_freq;
    p.x = x; p.z = z; p.final_norm = w->final_norm; p.status = ctx->d_status;
    if (!aligned(w->final_norm, 8)) return false;
    for (int l = 0; l < c.layers; l++) {
        const mt_qwen_layer& L = w->layers[l];
        const uint16_t* ptrs[8] = {L.norm1, L.qkv_w, L.qkv_b, L.o_w, L.norm2, L.gate_w, L.up_w, L.down_w};
        for (int i = 0; i < 8; i++) p.L[l].p[i] = ptrs[i];
        if (!aligned(L.norm1, 8) || !aligned(L.norm2, 8) || !aligned(L.qkv_w, 16) || !aligned(L.o_w, 16) ||
            !aligned(L.gate_w, 16) || !aligned(L.up_w, 16) || !aligned(L.down_w, 16))
            return false;
    }
    return stack_supported(p, ctx->sm_count);
}

// The context's stack area, grown (after the device drains: earlier launches may still use it)
// to at least `bytes`; a new area starts zeroed.
mt_status ctx_stack_area(mt_ctx* ctx, size_t bytes, void** out) {
    if (bytes > ctx->stack_area_bytes) {
        if (ctx->stack_area) {
            const cudaError_t e = cudaDeviceSynchronize();
            if (e != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "stack area grow sync: %s", cudaGetErrorString(e));
            cudaFree(ctx->stack_area);
            ctx->stack_area = nullptr;
            ctx->stack_area_bytes = 0;
        }
        const size_t want = bytes < ((size_t)1 << 20) ? ((size_t)1 << 20) : bytes;
        const mt_status st = stack_area_alloc(want, &ctx->stack_area);
        if (st != MT_OK) return fail(ctx, st, "persistent-stack area of %zu bytes", want);
        ctx->stack_area_bytes = want;
    }
    *out = ctx->stack_area;
    return MT_OK;
}

DecodeScratch carve(float* base, const mt_qwen_config& c, int M) {
    const size_t qkvw = (size_t)(c.heads + 2 * c.kv_heads) * 64;
    auto up = [](size_t n) { return (n + 63) & ~size_t(63); };
    auto planes = [&](float* at, int ld) {
        Planes p;
        p.hi = reinterpret_cast<uint16_t*>(at);
        p.lo = p.hi + (size_t)M * ld;  // M * ld * 2 bytes: a multiple of 16 (ld % 8 == 0)
        p.ld = ld;
        return p;
    };
    DecodeScratch s;
    s.normed = base;
    s.qkv = s.normed + up((size_t)M * c.hidden);
    s.attn = s.qkv + up((size_t)M * qkvw);
    s.mlp = s.attn + up((size_t)M * c.heads * 64);
    float* pl = s.mlp + up((size_t)M * c.intermediate);
    s.p_norm = planes(pl, c.hidden);
    pl += up((size_t)M * c.hidden);
    s.p_attn = planes(pl, c.heads * 64);
    pl += up((size_t)M * c.heads * 64);
    s.p_mlp = planes(pl, c.intermediate);
    return s;
}

// One tensor-core linear over bf16 planes: fp32 y (accumulated with MT_LINEAR_ACCUM, split K
// chosen by the planner) or bf16 planes out.
mt_status tc_linear(mt_ctx* ctx, const Planes& x, int m, const uint16_t* w, const uint16_t* w2, int n, int k, float* y,
                    int ldy, const Planes* yp, uint32_t flags, cudaStream_t s) {
    LinearArgs a{};
    a.x_hi = x.hi; a.x_lo = x.lo; a.ld_split = x.ld;
    a.m = m; a.n = n; a.k = k; a.w = w; a.w2 = w2;
    a.y = y; a.ldy = ldy;
    if (yp) { a.y_hi = yp->hi; a.y_lo = yp->lo; a.ld_ysplit = yp->ld; }
    a.flags = flags; a.split_k = 0;
    return launch_gemm_tc(ctx, a, s);
}

// One CUDA-core linear; with norm_w it reads RMSNorm(x) * norm_w (the norm folded in: no launch).
// With yp the output goes to bf16 planes (for a tensor-core consumer) instead of y.
void gemv(const float* x, int ldx, int m, const uint16_t* w, const uint16_t* w2, const uint16_t* bias, int n, int k,
          float* y, int ldy, uint32_t flags, cudaStream_t s, const uint16_t* norm_w = nullptr, float eps = 0.f,
          const Planes* yp = nullptr) {
    LinearArgs a{};
    a.x = x; a.ldx = ldx; a.m = m; a.n = n; a.k = k; a.w = w; a.w2 = w2; a.bias = bias;
    a.y = yp ? nullptr : y; a.ldy = ldy; a.flags = flags; a.split_k = 1;
    if (yp) { a.y_hi = yp->hi; a.y_lo = yp->lo; a.ld_ysplit = yp->ld; }
    a.norm_w = norm_w; a.norm_eps = eps;
    launch_gemv(a, s);
}

void norm(const float* x, int ld, int rows, int width, const uint16_t* g, float eps, float* y, cudaStream_t s) {
    RmsArgs a{};
    a.x = x; a.ldx = ld; a.rows = rows; a.width = width; a.w = g; a.eps = eps; a.y = y; a.ldy = ld;
    launch_rmsnorm(a, s);
}

void norm_planes(const float* x, int ld, int rows, int width, const uint16_t* g, float eps, const Planes& y,
                 cudaStream_t s) {
    RmsArgs a{};
    a.x = x; a.ldx = ld; a.rows = rows; a.width = width; a.w = g; a.eps = eps;
    a.y_hi = y.hi; a.y_lo = y.lo; a.ld_split = y.ld;
    launch_rmsnorm(a, s);
}

// RMSNorm(x) * g, then the linear: folded into the GEMV (every row count it takes) when the gain
// is 16-byte aligned (it loads as 16-byte vectors), else the norm's own launch into `normed` first.
void norm_gemv(const float* x, int H, int m, const uint16_t* g, float eps, float* normed, const uint16_t* w,
               const uint16_t* w2, const uint16_t* bias, int n, float* y, int ldy, uint32_t flags, cudaStream_t s,
               const Planes* yp = nullptr) {
    if (m <= 8 && ((uintptr_t)g & 15u) == 0) {
        gemv(x, H, m, w, w2, bias, n, H, y, ldy, flags, s, g, eps, yp);
    } else {
        norm(x, H, m, H, g, eps, normed, s);
        gemv(normed, H, m, w, w2, bias, n, H, y, ldy, flags, s, nullptr, 0.f, yp);
    }
}

}  // namespace

}  // namespace mt

using namespace mt;

extern "C" mt_status mt_qwen_decode(mt_ctx* ctx, void* stream, const mt_qwen_weights* w, int requests, int rows,
                                    float* x, float* kv, long long kv_stride, int capacity, const int32_t* positions,
                                    float* z) {
    MT_REQUIRE(ctx, ctx && w && x && kv && positions && z && w->layers && w->final_norm, MT_ERR_ARG,
               "mt_qwen_decode: null argument");
    const mt_qwen_config& c = w->cfg;
    const int M = requests * rows;
    MT_REQUIRE(ctx, requests >= 1 && rows >= 1 && M <= kDecodeMaxRows && attention_decode_supported(rows, c.heads, c.kv_heads),
               MT_ERR_SHAPE, "mt_qwen_decode: %d requests x %d rows (rows <= %d, at most %d rows in all; heads %d/%d)",
               requests, rows, ATTN_DECODE_MAX_ROWS, kDecodeMaxRows, c.heads, c.kv_heads);
    MT_REQUIRE(ctx, c.layers >= 1 && c.hidden % 8 == 0 && c.intermediate % 8 == 0 && c.heads * 64 % 8 == 0 && c.window >= 0,
               MT_ERR_SHAPE, "mt_qwen_decode: hidden %d intermediate %d", c.hidden, c.intermediate);
    const long long cache_floats = (long long)c.layers * 2 * c.kv_heads * capacity * 64;
    MT_REQUIRE(ctx, capacity > 0 && kv_stride >= cache_floats && kv_stride % 4 == 0 &&
                        (c.window == 0 || c.window + rows - 1 <= capacity),
               MT_ERR_CAPACITY, "mt_qwen_decode: capacity %d, request stride %lld floats (needs %lld), window %d",
               capacity, kv_stride, cache_floats, c.window);
    MT_REQUIRE(ctx, ((uintptr_t)x & 15u) == 0 && ((uintptr_t)kv & 15u) == 0 && ((uintptr_t)z & 15u) == 0, MT_ERR_ARG,
               "mt_qwen_decode: x, kv and z need 16-byte alignment");
    cudaStream_t s = as_stream(stream);
    const float* inv_freq = nullptr;
    mt_status st = rope_table(ctx, c.rope_theta, &inv_freq);
    if (st != MT_OK) return st;
    StackParams sp;
    if (stack_params(ctx, w, requests, rows, x, kv, kv_stride, capacity, positions, z, inv_freq, &sp)) {
        void* area = nullptr;
        st = ctx_stack_area(ctx, stack_area_bytes(sp), &area);
        if (st != MT_OK) return st;
        stack_bind(sp, area);
        launch_stack(sp, ctx->sm_count, s);
        return check_launch(ctx, "mt_qwen_decode (persistent)");
    }
    MT_REQUIRE(ctx, ctx->persistent != 2, MT_ERR_SHAPE,
               "mt_qwen_decode: the persistent stack kernel cannot run this pass (%d requests x %d rows, window %d, "
               "capacity %d; %s %s)", requests, rows, c.window, capacity,
               stack_resident_blocks() < 1 ? "it does not fit one block per SM:" : "shapes", stack_resident_why());
    void* buf = nullptr;
    st = mt::scratch(ctx, s, decode_scratch_floats(c, M) * sizeof(float), &buf);
    if (st != MT_OK) return st;
    DecodeScratch sc = carve(static_cast<float*>(buf), c, M);

    const int H = c.hidden, qkvw = (c.heads + 2 * c.kv_heads) * 64, A = c.heads * 64;
    const size_t tensor = (size_t)c.kv_heads * capacity * 64;
    const bool tc_res = M >= kTcResidualRows, tc_gu = M >= kTcGateUpRows;
    for (int l = 0; l < c.layers; l++) {
        const mt_qwen_layer& L = w->layers[l];
        float* kc = kv + (size_t)(2 * l) * tensor;
        norm_gemv(x, H, M, L.norm1, c.eps, sc.normed, L.qkv_w, nullptr, L.qkv_b, qkvw, sc.qkv, qkvw, MT_LINEAR_BIAS, s);
        AttnDecodeArgs da{};
        da.qkv = sc.qkv; da.ldq = qkvw; da.requests = requests; da.rows_per_req = rows; da.hq = c.heads;
        da.hkv = c.kv_heads; da.pos0 = 0; da.pos_dev = positions; da.window = c.window; da.kc = kc; da.vc = kc + tensor;
        da.req_stride = kv_stride; da.cap = capacity; da.inv_freq = inv_freq; da.out = sc.attn; da.ldo = A;
        da.max_keys = c.window > 0 ? c.window : capacity; da.status = ctx->d_status;
        if (tc_res) { da.out = nullptr; da.out_hi = sc.p_attn.hi; da.out_lo = sc.p_attn.lo; da.ld_split = A; }
        launch_attention_decode(da, s);
        if (tc_res) {
            st = tc_linear(ctx, sc.p_attn, M, L.o_w, nullptr, H, A, x, H, nullptr, MT_LINEAR_ACCUM, s);
            if (st != MT_OK) return st;
        } else {
            gemv(sc.attn, A, M, L.o_w, nullptr, nullptr, H, A, x, H, MT_LINEAR_ACCUM, s);
        }
        if (tc_gu) {
            norm_planes(x, H, M, H, L.norm2, c.eps, sc.p_norm, s);
            st = tc_linear(ctx, sc.p_norm, M, L.gate_w, L.up_w, c.intermediate, H, nullptr, 0, &sc.p_mlp,
                           MT_LINEAR_SILU_GATE, s);
            if (st != MT_OK) return st;
        } else {
            norm_gemv(x, H, M, L.norm2, c.eps, sc.normed, L.gate_w, L.up_w, nullptr, c.intermediate, sc.mlp,
                      c.intermediate, MT_LINEAR_SILU_GATE, s, tc_res ? &sc.p_mlp : nullptr);
        }
        if (tc_res) {
            st = tc_linear(ctx, sc.p_mlp, M, L.down_w, nullptr, H, c.intermediate, x, H, nullptr, MT_LINEAR_ACCUM, s);
            if (st != MT_OK) return st;
        } else {
            gemv(sc.mlp, c.intermediate, M, L.down_w, nullptr, nullptr, H, c.intermediate, x, H, MT_LINEAR_ACCUM, s);
        }
    }
    norm(x, H, M, H, w->final_norm, c.eps, z, s);
    return check_launch(ctx, "mt_qwen_decode");
}
