// engine.cu -- the generation loop of Ming-3.0-tts-0.5B for R concurrent requests on one GPU.
//
// Restates MingEngine.generate / encodeStep (Sources/MingTTS/Engine/Engine.swift:302-415),
// QwenForward.dispatches (Qwen.swift:72-97), DiTForward.encode (DiT.swift:35-52), the streaming
// VAEDecoder (VAEDecoder.swift:64-107) and the temb precompute (Engine.swift:187-198).
//
// B200 layout: every request's rows are stacked, so each projection is one GEMM over all requests
// (LLM R rows, flow DiT 6R, aggregator 2R, VAE 4R, prefill R*T). Row counts <= 8 use the
// CUDA-core GEMV on fp32 activations; larger ones the tcgen05 GEMM on bf16 hi/lo planes, which
// the producing kernels (RMSNorm, attention, the gated/GELU epilogues) write directly.
// Stream A runs LLM token n -> stop head -> flow head -> aggregator -> VAE fc1; stream B decodes
// the VAE frames of latent n-2 concurrently (the reference pairs the same two stacks on one
// concurrent encoder, Qwen.swift:103-114). Step-dependent values live in a device step state
// filled from pinned memory, so steady-state steps replay one captured CUDA graph.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "engine_kernels.cuh"
#include "kernels.cuh"

namespace mt {

static const int kGemvMax = 8;  // rows at or below which linears use the CUDA-core GEMV
static thread_local int g_kernels = 0;  // kernels enqueued by the current engine call
static const int kPcmRing = 4;  // pinned PCM slots mt_engine_generate cycles through

struct Act {  // activation matrix with fp32 and bf16 hi/lo representations
    float* f = nullptr;
    uint16_t* hi = nullptr;
    uint16_t* lo = nullptr;
    int ld = 0;
};

struct Lin {
    bool tc = false;
    LinearArgs g{};
    GemmPlan p{};
};

struct QwenLayerPlans { Lin qkv, o, gu, down; };
struct DitBlockPlans { Lin qkv, out, ff1, ff2; };

struct DitBufs {
    float* x = nullptr;  // residual [rows, hidden]
    Act norm, attn, ff;
    float* qkv = nullptr;
};

struct QwenBufs {
    float* x = nullptr;  // residual
    Act norm, attn, mlp;
    float* qkv = nullptr;
    float* kv = nullptr;  // [R][layers][2][kv][cap][64]
    int cap = 0;
    float* inv_freq = nullptr;  // [32]
};

constexpr int kMaxGroups = 4;

// A contiguous range of requests whose LLM token, flow head, aggregator and VAE fc1 run as one
// chain on the group's own stream. Requests never interact, so the groups of a step are
// independent chains the GPU may run concurrently. The buffers are views into the engine's
// request-major buffers.
struct Group {
    int r0 = 0, R = 0;
    cudaStream_t s = nullptr;     // group 0 runs on the engine's step stream
    cudaEvent_t done = nullptr;
    QwenBufs llm;
    Act z, agg_norm;
    float *stop = nullptr, *cemb = nullptr, *y = nullptr, *hist = nullptr, *noise = nullptr, *latents = nullptr,
          *vel0 = nullptr, *vae_h = nullptr;
    DitBufs flow, agg;
    const int* llm_pos = nullptr;  // device: this group's per-request LLM positions
    std::vector<QwenLayerPlans> llm_dec;
    std::vector<DitBlockPlans> flow_blocks, agg_blocks;
    Lin cond, agg_final, stop_lin;
    // Few rows: the LLM token, flow DiT pass and aggregator as persistent stack launches.
    bool llm_ps = false, flow_ps = false, agg_ps = false;
    StackParams llm_sp{}, flow_sp{}, agg_sp{};
    void* stack_area = nullptr;  // area of this group's stack launches (its stream runs them in turn)
};

}  // namespace mt

using namespace mt;

struct mt_engine {
    mt_ctx* ctx = nullptr;
    const mt_model* model = nullptr;
    mt_model_config cfg{};
    mt_model_weights w{};
    mt_engine_options opt{};
    std::vector<void*> allocs;
    std::vector<float> timesteps;
    int prio_hi = 0;  // launch priority of the step's critical path (the device's highest)

    // Buffers.
    QwenBufs llm, vae;
    Act z;
    float* stop = nullptr;
    float* temb = nullptr;
    float* cemb = nullptr;
    float *y = nullptr, *hist = nullptr, *noise = nullptr, *latents = nullptr, *vel0 = nullptr;
    DitBufs flow, agg;
    Act agg_norm;
    float* vae_h = nullptr;
    Act vae_hidden;
    float* spec = nullptr;
    float* fring = nullptr;
    float* pcm = nullptr;
    int max_chunk = 0;
    int* state_dev = nullptr;
    int* state_host = nullptr;  // pinned step state being filled: one of state_slots
    int* state_slots[2] = {};   // pinned; step n fills slot n & 1 while step n - 1 may still run
    cudaEvent_t state_ev[2] = {};  // recorded after the step that read the slot
    bool state_ev_live[2] = {};
    float* ws_a = nullptr;      // split-K workspace of the main stream (LLM, flow, aggregator)
    float* ws_b = nullptr;      // split-K workspace of the VAE stream
    size_t ws_a_floats = 0, ws_b_floats = 0;

    // Current generation.
    int R = 0, T = 0, steps = 0;
    float cfg_scale = 2.0f;
    int n = 0;          // steps enqueued
    int latents_fed = 0, decoded = 0, emitted = 0;
    bool begun = false, prefilled = false;

    // Plans for the current (R, T).
    int plan_R = -1, plan_T = -1, plan_persistent = -1;
    std::vector<QwenLayerPlans> llm_pre, vae_layers;
    Lin vae_head;
    bool vae_ps = false;        // VAE decode stack as one persistent launch (4R <= 8 rows)
    StackParams vae_sp{};
    void* vae_area = nullptr;   // area of the VAE decode's stack launches
    Group groups[kMaxGroups];
    int G = 1;  // groups of the current generation

    cudaStream_t sa = nullptr;  // step stream (owned, capturable; joined to the caller's stream)
    cudaStream_t sb = nullptr;  // VAE stream
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr, ev_in = nullptr, ev_out = nullptr;
    int step_kernels = 0;       // kernels of the last step
    bool time_stages = false;   // record per-stage events (eager steps only)
    bool stop_rule = false;     // generate/generate_stream end once every request met the stop rule
    cudaEvent_t stage_ev[6] = {};  // A: start, after llm, after flow, after agg; B: decode start, end
    bool stage_valid = false;
    int graph_kernels = 0;      // kernels in the captured step graph
    cudaGraph_t graph[2] = {};  // steady-state step, one per state slot (the upload source differs)
    cudaGraphExec_t graph_exec[2] = {};

    // Host-API staging of mt_engine_generate, allocated once with the engine.
    int32_t* ids_stage = nullptr;  // device copy of the prompt token ids
    float* ring_host = nullptr;    // pinned [kPcmRing][R * max_chunk] PCM slots
    float* stop_host = nullptr;    // pinned [max_steps][R][2] stop logits
    cudaEvent_t ring_ev[kPcmRing] = {};
};

namespace {

template <typename T>
mt_status dalloc(mt_engine* e, T** p, size_t count) {
    *p = nullptr;
    if (count == 0) count = 1;
    cudaError_t err = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
    if (err != cudaSuccess) return fail(e->ctx, MT_ERR_NOMEM, "engine: cudaMalloc of %zu bytes: %s", count * sizeof(T),
                                        cudaGetErrorString(err));
    cudaMemset(*p, 0, count * sizeof(T));
    e->allocs.push_back(*p);
    return MT_OK;
}

mt_status act_alloc(mt_engine* e, Act* a, size_t rows, int cols) {
    a->ld = cols;
    mt_status st = dalloc(e, &a->f, rows * cols);
    if (st == MT_OK) st = dalloc(e, &a->hi, rows * cols);
    if (st == MT_OK) st = dalloc(e, &a->lo, rows * cols);
    return st;
}

#define TRY(expr)                            \
    do {                                     \
        mt_status _st = (expr);              \
        if (_st != MT_OK) return _st;        \
    } while (0)

mt_status qwen_alloc(mt_engine* e, QwenBufs* q, const mt_qwen_config& c, size_t rows, int requests, int cap) {
    const int qkvw = (c.heads + 2 * c.kv_heads) * 64;
    TRY(dalloc(e, &q->x, rows * c.hidden));
    TRY(act_alloc(e, &q->norm, rows, c.hidden));
    TRY(act_alloc(e, &q->attn, rows, c.heads * 64));
    TRY(act_alloc(e, &q->mlp, rows, c.intermediate));
    TRY(dalloc(e, &q->qkv, rows * qkvw));
    q->cap = cap;
    TRY(dalloc(e, &q->kv, (size_t)requests * c.layers * 2 * c.kv_heads * cap * 64));
    TRY(dalloc(e, &q->inv_freq, 32));
    float inv[32];
    for (int i = 0; i < 32; i++) inv[i] = 1.0f / powf(c.rope_theta, (float)(2 * i) / 64.0f);  // Qwen.swift:60
    cudaMemcpy(q->inv_freq, inv, sizeof(inv), cudaMemcpyHostToDevice);
    return MT_OK;
}

mt_status dit_alloc(mt_engine* e, DitBufs* d, const mt_dit_config& c, size_t rows) {
    TRY(dalloc(e, &d->x, rows * c.hidden));
    TRY(act_alloc(e, &d->norm, rows, c.hidden));
    TRY(act_alloc(e, &d->attn, rows, c.hidden));
    TRY(act_alloc(e, &d->ff, rows, c.ff));
    TRY(dalloc(e, &d->qkv, rows * 3 * c.hidden));
    return MT_OK;
}

// A linear over m rows of x: CUDA-core GEMV (fp32 x.f) for m <= 8, else a tcgen05 plan (x.hi/lo).
// Route of a linear over m <= kGemvMax rows, measured with isolated graph-replayed launches whose
// weights stream from DRAM. The GEMV grows about 1 us per row (2 / 4 / 6 / 8 rows: W[3072x1024]
// 5.0 / 7.3 / 8.3 / 9.8 us, gated W[2 x 4864x896] 8.4 / 10.2 / 14.3 / 16.7 us); the tensor-core GEMM
// is flat (5.7 and 9.0 us) but needs its input as bf16 planes, i.e. the RMSNorm in front as its own
// launch (~2.6 us), which the GEMV folds in. Isolated, that puts the crossovers at 5 rows (gated)
// and 7 rows (W[3072x1024]); in the engine step the GEMV's blocks (two per SM, every register)
// also delay the concurrent stream's kernels, and the single-request step measured faster with
// the tensor cores from the thresholds below. n_eff counts both matrices of a gated linear.
// An accumulating linear (the residual projections) splits K on the tensor-core route and wins from
// 2 rows (W[1024x4096] 5.2 / 7.5 / 10.0 us on the GEMV at 2 / 4 / 8 rows against 4.3-4.4 us).
bool small_rows_tc(int m, long long n_eff, int k, bool accum = false) {
    if (m > kGemvMax) return true;
    if (accum) return m >= 2;
    if (k > 2048) return false;
    const long long nk = n_eff * k;
    if (nk >= 8000000) return m >= 2;
    if (nk >= 3000000) return m >= 4;
    if (nk >= 1000000) return m >= 6;
    return false;
}

// `y` receives fp32 output; `ys` (optional) receives the activation for a following linear in the
// representation that linear's route reads (ys_tc: bf16 hi/lo planes, else fp32; either route can
// write either).
// route: 1 tensor cores, 0 CUDA-core GEMV, -1 by the row count alone (tensor cores above kGemvMax).
// Tensor-core linears split K automatically to fill the SMs; a nonlinear epilogue then reduces
// through the stream's fp32 workspace (ws, ws_floats) when it is large enough.
mt_status make_lin(mt_engine* e, Lin* L, const Act& x, int m, const mt_bf16* w, const mt_bf16* w2,
                   const mt_bf16* bias, int n, int k, float* y, int ldy, const Act* ys, uint32_t flags,
                   float* ws = nullptr, size_t ws_floats = 0, int route = -1, int ys_tc = -1) {
    LinearArgs a{};
    a.m = m; a.n = n; a.k = k; a.w = w; a.w2 = w2; a.bias = bias; a.flags = flags | (bias ? MT_LINEAR_BIAS : 0);
    a.split_k = 1;
    L->tc = route >= 0 ? route == 1 : m > kGemvMax;
    const bool planes_out = ys && (ys_tc >= 0 ? ys_tc == 1 : m > kGemvMax);
    if (!L->tc) {
        a.x = x.f; a.ldx = x.ld;
        if (planes_out) {  // the GEMV epilogue writes the planes a tensor-core consumer reads
            a.y_hi = ys->hi; a.y_lo = ys->lo; a.ld_ysplit = ys->ld;
        } else {
            a.y = ys ? ys->f : y;
            a.ldy = ys ? ys->ld : ldy;
        }
        L->g = a;
        return MT_OK;
    }
    a.x_hi = x.hi; a.x_lo = x.lo; a.ld_split = x.ld;
    if (planes_out) {
        a.y_hi = ys->hi; a.y_lo = ys->lo; a.ld_ysplit = ys->ld;
    } else if (ys) {
        a.y = ys->f; a.ldy = ys->ld;
    } else {
        a.y = y; a.ldy = ldy;
    }
    a.split_k = 0;
    a.ws = ws && (size_t)m * 2 * n <= ws_floats ? ws : nullptr;
    return make_gemm_plan(e->ctx, a, &L->p);
}

inline void run(const Lin& L, cudaStream_t s) {
    g_kernels++;
    if (L.tc) run_gemm_plan(L.p, s);
    else launch_gemv(L.g, s);
}

// RMSNorm of `rows` rows into the representation the consumer route reads (consumer_tc: bf16
// hi/lo planes, else fp32); fp32 also when keep_f32.
void norm_to(const float* x, int ldx, int rows, int width, const mt_bf16* w, float eps, const Act& out,
             bool consumer_tc, bool keep_f32, cudaStream_t s) {
    RmsArgs a{};
    a.x = x; a.ldx = ldx; a.rows = rows; a.width = width; a.w = w; a.eps = eps;
    if (!consumer_tc || keep_f32) { a.y = out.f; a.ldy = out.ld; }
    if (consumer_tc) { a.y_hi = out.hi; a.y_lo = out.lo; a.ld_split = out.ld; }
    launch_rmsnorm(a, s);
    g_kernels++;
}

// The same for a consumer routed by its row count alone.
void norm(const float* x, int ldx, int rows, int width, const mt_bf16* w, float eps, const Act& out, int rows_consumer,
          bool keep_f32, cudaStream_t s) {
    norm_to(x, ldx, rows, width, w, eps, out, rows_consumer > kGemvMax, keep_f32, s);
}

// The norm before a linear: folded into a CUDA-core linear (nothing to launch), else in the
// representation its route reads.
void norm_for(const Lin& L, const float* x, int ld, int rows, const mt_bf16* g, float eps, const Act& out,
              cudaStream_t s) {
    if (!L.tc && L.g.norm_w) return;
    norm_to(x, ld, rows, ld, g, eps, out, L.tc, false, s);
}

// Rows up to which a CUDA-core linear folds the RMSNorm before it: every row count of the GEMV
// route (the 2..8-row GEMV stages x once per block, so the gain and x^2 work is small; the fold
// saves the norm's launch, about 2.6 us in a graph).
constexpr int kFoldNormMax = 8;

// A linear after an RMSNorm, on the CUDA-core route with few rows: it reads the residual rows and
// folds the norm in (gain as x loads, 1/rms on the dot product), so the norm has no launch.
bool folds_norm(int rows) { return rows <= kFoldNormMax; }
void fold_norm(Lin* L, const float* x, int ld, const mt_bf16* g, float eps) {
    if (L->tc || !folds_norm(L->g.m)) return;
    L->g.x = x;
    L->g.ldx = ld;
    L->g.norm_w = g;
    L->g.norm_eps = eps;
}

mt_status plan_qwen(mt_engine* e, std::vector<QwenLayerPlans>& plans, const mt_qwen_weights& W, QwenBufs& b, int rows,
                    float* ws, size_t ws_floats) {
    const mt_qwen_config& c = W.cfg;
    const int qkvw = (c.heads + 2 * c.kv_heads) * 64;
    plans.resize(c.layers);
    const int A = c.heads * 64;
    const int r_qkv = small_rows_tc(rows, qkvw, c.hidden), r_o = small_rows_tc(rows, c.hidden, A, true);
    const int r_gu = small_rows_tc(rows, 2LL * c.intermediate, c.hidden);
    const int r_down = small_rows_tc(rows, c.hidden, c.intermediate, true);
    for (int l = 0; l < c.layers; l++) {
        const mt_qwen_layer& L = W.layers[l];
        TRY(make_lin(e, &plans[l].qkv, b.norm, rows, L.qkv_w, nullptr, L.qkv_b, qkvw, c.hidden, b.qkv, qkvw, nullptr, 0,
                     nullptr, 0, r_qkv));
        TRY(make_lin(e, &plans[l].o, b.attn, rows, L.o_w, nullptr, nullptr, c.hidden, A, b.x, c.hidden,
                     nullptr, MT_LINEAR_ACCUM, nullptr, 0, r_o));
        TRY(make_lin(e, &plans[l].gu, b.norm, rows, L.gate_w, L.up_w, nullptr, c.intermediate, c.hidden, nullptr, 0,
                     &b.mlp, MT_LINEAR_SILU_GATE, ws, ws_floats, r_gu, r_down));
        TRY(make_lin(e, &plans[l].down, b.mlp, rows, L.down_w, nullptr, nullptr, c.hidden, c.intermediate, b.x,
                     c.hidden, nullptr, MT_LINEAR_ACCUM, nullptr, 0, r_down));
        fold_norm(&plans[l].qkv, b.x, c.hidden, L.norm1, c.eps);
        fold_norm(&plans[l].gu, b.x, c.hidden, L.norm2, c.eps);
    }
    return MT_OK;
}

mt_status plan_dit(mt_engine* e, std::vector<DitBlockPlans>& plans, const mt_dit_weights& W, DitBufs& b, int rows,
                   float* ws, size_t ws_floats) {
    const mt_dit_config& c = W.cfg;
    plans.resize(c.depth);
    const int r_qkv = small_rows_tc(rows, 3LL * c.hidden, c.hidden);
    const int r_out = small_rows_tc(rows, c.hidden, c.hidden, true);
    const int r_ff1 = small_rows_tc(rows, c.ff, c.hidden), r_ff2 = small_rows_tc(rows, c.hidden, c.ff, true);
    for (int i = 0; i < c.depth; i++) {
        const mt_dit_block& B = W.blocks[i];
        TRY(make_lin(e, &plans[i].qkv, b.norm, rows, B.qkv_w, nullptr, B.qkv_b, 3 * c.hidden, c.hidden, b.qkv,
                     3 * c.hidden, nullptr, 0, nullptr, 0, r_qkv));
        TRY(make_lin(e, &plans[i].out, b.attn, rows, B.out_w, nullptr, B.out_b, c.hidden, c.hidden, b.x, c.hidden,
                     nullptr, MT_LINEAR_ACCUM, nullptr, 0, r_out));
        TRY(make_lin(e, &plans[i].ff1, b.norm, rows, B.ff1_w, nullptr, B.ff1_b, c.ff, c.hidden, nullptr, 0, &b.ff,
                     MT_LINEAR_GELU, ws, ws_floats, r_ff1, r_ff2));
        TRY(make_lin(e, &plans[i].ff2, b.ff, rows, B.ff2_w, nullptr, B.ff2_b, c.hidden, c.ff, b.x, c.hidden, nullptr,
                     MT_LINEAR_ACCUM, nullptr, 0, r_ff2));
        fold_norm(&plans[i].qkv, b.x, c.hidden, B.norm1, c.eps);
        fold_norm(&plans[i].ff1, b.x, c.hidden, B.norm2, c.eps);
    }
    return MT_OK;
}

// A Qwen pass over `rows` rows (rows_per_req per request, positions pos_dev) as one persistent stack
// launch; false where the context disables it or the shapes do not fit (then one launch per op).
bool qwen_stack(mt_engine* e, const mt_qwen_weights& W, const QwenBufs& b, int rows, int rows_per_req,
                const int* pos_dev, float* z, void* area, StackParams* out) {
    const mt_qwen_config& c = W.cfg;
    if (e->ctx->persistent == 0 || rows > kGemvMax || c.layers > STACK_MAX_LAYERS) return false;
    StackParams& p = *out;
    p = StackParams{};
    p.kind = STACK_QWEN; p.layers = c.layers; p.M = rows; p.seq_rows = rows_per_req; p.seqs = rows / rows_per_req;
    p.hidden = c.hidden; p.heads = c.heads; p.kv_heads = c.kv_heads; p.inter = c.intermediate; p.eps = c.eps;
    p.window = c.window; p.cap = b.cap; p.kv_stride = (long long)c.layers * 2 * c.kv_heads * b.cap * 64;
    p.pos = pos_dev; p.kv = b.kv; p.inv_freq = b.inv_freq;
    p.x = b.x; p.z = z; p.final_norm = W.final_norm; p.status = e->ctx->d_status;
    for (int l = 0; l < c.layers; l++) {
        const mt_qwen_layer& L = W.layers[l];
        const mt_bf16* ptrs[8] = {L.norm1, L.qkv_w, L.qkv_b, L.o_w, L.norm2, L.gate_w, L.up_w, L.down_w};
        for (int i = 0; i < 8; i++) p.L[l].p[i] = ptrs[i];
    }
    stack_bind(p, area);
    return stack_supported(p, e->ctx->sm_count);
}

// The blocks of a DiT pass over `batch` sequences of `seq` rows as one persistent stack launch.
bool dit_stack(mt_engine* e, const mt_dit_weights& W, const DitBufs& b, int batch, int seq, void* area, StackParams* out) {
    const mt_dit_config& c = W.cfg;
    if (e->ctx->persistent == 0 || batch * seq > kGemvMax || c.depth > STACK_MAX_LAYERS) return false;
    StackParams& p = *out;
    p = StackParams{};
    p.kind = STACK_DIT; p.layers = c.depth; p.M = batch * seq; p.seq_rows = seq; p.seqs = batch;
    p.hidden = c.hidden; p.heads = c.heads; p.kv_heads = c.heads; p.inter = c.ff; p.eps = c.eps;
    p.inv_freq = W.inv_freq;
    p.x = b.x; p.status = e->ctx->d_status;
    for (int i = 0; i < c.depth; i++) {
        const mt_dit_block& B = W.blocks[i];
        const mt_bf16* ptrs[10] = {B.norm1, B.qkv_w, B.qkv_b, B.out_w, B.out_b, B.norm2, B.ff1_w, B.ff1_b, B.ff2_w, B.ff2_b};
        for (int k = 0; k < 10; k++) p.L[i].p[k] = ptrs[k];
    }
    stack_bind(p, area);
    return stack_supported(p, e->ctx->sm_count);
}

// Stack-area bytes of the largest pass (8 rows) of each kind: a Qwen stack with rows_per_req rows
// per request over a cap-position cache, or a DiT stack.
size_t qwen_area_bound(const mt_qwen_config& c, int rows_per_req, int cap) {
    StackParams p{};
    p.kind = STACK_QWEN; p.M = 8; p.seq_rows = rows_per_req; p.seqs = 8 / rows_per_req;
    p.hidden = c.hidden; p.heads = c.heads; p.kv_heads = c.kv_heads; p.inter = c.intermediate;
    p.window = c.window; p.cap = cap;
    return stack_area_bytes(p);
}
size_t dit_area_bound(const mt_dit_config& c) {
    StackParams p{};
    p.kind = STACK_DIT; p.M = 8; p.seq_rows = 1; p.seqs = 8;
    p.hidden = c.hidden; p.heads = c.heads; p.kv_heads = c.heads; p.inter = c.ff;
    return stack_area_bytes(p);
}

Act act_rows(const Act& a, size_t row) {
    Act v = a;
    const size_t off = row * (size_t)a.ld;
    v.f = a.f ? a.f + off : nullptr;
    v.hi = a.hi ? a.hi + off : nullptr;
    v.lo = a.lo ? a.lo + off : nullptr;
    return v;
}

DitBufs dit_rows(const DitBufs& d, size_t row, int hidden) {
    DitBufs v;
    v.x = d.x + row * hidden;
    v.norm = act_rows(d.norm, row);
    v.attn = act_rows(d.attn, row);
    v.ff = act_rows(d.ff, row);
    v.qkv = d.qkv + row * 3 * hidden;
    return v;
}

// Groups for R requests: the option (default 1); at most kMaxGroups and at most R. Measured on
// B200 at 64 requests: 1 group 642, 2 groups 560, 4 groups 447 audio-s/s -- concurrent chains
// contend for whole SMs (a tensor-core GEMM CTA holds 200 KB of shared memory) and CTAs launched
// early by programmatic dependent launch park on SMs the other chain needs.
int group_count(const mt_engine* e, int R) {
    int G = e->opt.groups > 0 ? e->opt.groups : 1;
    if (G > kMaxGroups) G = kMaxGroups;
    if (G > R) G = R;
    return G < 1 ? 1 : G;
}

// Views and decode-time plans of group g over requests [r0, r0 + Rg).
mt_status plan_group(mt_engine* e, Group& g, int r0, int Rg) {
    const mt_model_config& c = e->cfg;
    const int H = c.llm.hidden, L = c.latent_dim, qkvw = (c.llm.heads + 2 * c.llm.kv_heads) * 64;
    const size_t req_stride = (size_t)c.llm.layers * 2 * c.llm.kv_heads * e->llm.cap * 64;
    g.r0 = r0;
    g.R = Rg;
    g.llm = e->llm;
    g.llm.x = e->llm.x + (size_t)r0 * H;
    g.llm.norm = act_rows(e->llm.norm, r0);
    g.llm.attn = act_rows(e->llm.attn, r0);
    g.llm.mlp = act_rows(e->llm.mlp, r0);
    g.llm.qkv = e->llm.qkv + (size_t)r0 * qkvw;
    g.llm.kv = e->llm.kv + (size_t)r0 * req_stride;
    g.z = act_rows(e->z, r0);
    g.agg_norm = act_rows(e->agg_norm, r0);
    g.stop = e->stop + (size_t)r0 * 2;
    g.cemb = e->cemb + (size_t)r0 * c.flow.hidden;
    g.y = e->y + (size_t)r0 * L;
    g.hist = e->hist + (size_t)r0 * L;
    g.noise = e->noise + (size_t)r0 * e->opt.max_steps * L;
    g.latents = e->latents + (size_t)r0 * e->opt.max_steps * L;
    g.vel0 = e->vel0 + (size_t)r0 * c.flow_steps * 2 * L;
    g.vae_h = e->vae_h + (size_t)r0 * VAE_H_RING * c.vae.hidden;
    g.flow = dit_rows(e->flow, (size_t)6 * r0, c.flow.hidden);
    g.agg = dit_rows(e->agg, (size_t)2 * r0, c.agg.hidden);
    g.llm_pos = e->state_dev + st_llm_pos(e->R) + r0;
    // Split-K workspaces are per stream and the groups run concurrently: group plans use none.
    TRY(plan_qwen(e, g.llm_dec, e->w.llm, g.llm, Rg, nullptr, 0));
    TRY(make_lin(e, &g.cond, g.z, Rg, e->w.flow_c_w, nullptr, e->w.flow_c_b, c.flow.hidden, H, g.cemb, c.flow.hidden,
                 nullptr, 0));
    {
        // The stop head has two outputs: always the GEMV (rows processed in chunks of 8).
        LinearArgs a{};
        a.x = g.z.f; a.ldx = g.z.ld; a.m = Rg; a.n = 2; a.k = H; a.w = e->w.stop_w; a.bias = e->w.stop_b;
        a.flags = MT_LINEAR_BIAS; a.y = g.stop; a.ldy = 2;
        g.stop_lin.tc = false;
        g.stop_lin.g = a;
    }
    TRY(plan_dit(e, g.flow_blocks, e->w.flow, g.flow, 6 * Rg, nullptr, 0));
    TRY(plan_dit(e, g.agg_blocks, e->w.agg, g.agg, 2 * Rg, nullptr, 0));
    TRY(make_lin(e, &g.agg_final, g.agg_norm, Rg, e->w.agg.final_w, nullptr, e->w.agg.final_b, c.agg.out_dim,
                 c.agg.hidden, g.llm.x, H, nullptr, 0));
    // Stack launches take every SM: only where one chain runs at a time (a single request group).
    const bool solo = group_count(e, e->R) == 1;
    g.llm_ps = solo && qwen_stack(e, e->w.llm, g.llm, Rg, 1, g.llm_pos, g.z.f, g.stack_area, &g.llm_sp);
    g.flow_ps = solo && dit_stack(e, e->w.flow, g.flow, 2 * Rg, 3, g.stack_area, &g.flow_sp);
    g.agg_ps = solo && dit_stack(e, e->w.agg, g.agg, Rg, 2, g.stack_area, &g.agg_sp);
    return MT_OK;
}

mt_status build_plans(mt_engine* e) {
    if (e->plan_R == e->R && e->plan_T == e->T && e->plan_persistent == e->ctx->persistent) return MT_OK;
    e->plan_persistent = e->ctx->persistent;
    const int R = e->R, T = e->T;
    const mt_model_config& c = e->cfg;
    TRY(plan_qwen(e, e->llm_pre, e->w.llm, e->llm, R * T, e->ws_a, e->ws_a_floats));
    e->G = group_count(e, R);
    for (int i = 0, r0 = 0; i < e->G; i++) {
        const int Rg = R / e->G + (i < R % e->G ? 1 : 0);
        TRY(plan_group(e, e->groups[i], r0, Rg));
        r0 += Rg;
    }
    TRY(plan_qwen(e, e->vae_layers, e->w.vae, e->vae, 4 * R, e->ws_b, e->ws_b_floats));
    TRY(make_lin(e, &e->vae_head, e->vae_hidden, 4 * R, e->w.vae_head_w, nullptr, e->w.vae_head_b, c.nfft + 2,
                 c.vae.hidden, e->spec, c.nfft + 2, nullptr, 0));
    e->vae_ps = e->G == 1 && qwen_stack(e, e->w.vae, e->vae, 4 * R, 4, e->state_dev + st_vae_pos(R), e->vae_hidden.f,
                                        e->vae_area, &e->vae_sp);
    e->plan_R = R;
    e->plan_T = T;
    return MT_OK;
}

// One pass of a Qwen stack (QwenForward.dispatches, Qwen.swift:72-97) over `rows` rows grouped by
// request (rows_per_req each); positions pos0 + pos_dev[request] + row % rows_per_req.
void qwen_forward(mt_engine* e, const mt_qwen_weights& W, QwenBufs& b, std::vector<QwenLayerPlans>& plans, int rows,
                  int rows_per_req, int pos0, const int* pos_dev, int max_keys, cudaStream_t s) {
    const mt_qwen_config& c = W.cfg;
    const int qkvw = (c.heads + 2 * c.kv_heads) * 64;
    const size_t tensor = (size_t)c.kv_heads * b.cap * 64;
    const long long req_stride = (long long)c.layers * 2 * tensor;
    for (int l = 0; l < c.layers; l++) {
        const mt_qwen_layer& L = W.layers[l];
        float* kc = b.kv + (size_t)(2 * l) * tensor;
        float* vc = kc + tensor;
        const bool tc = plans[l].o.tc;  // the attention rows' consumer
        norm_for(plans[l].qkv, b.x, c.hidden, rows, L.norm1, c.eps, b.norm, s);
        run(plans[l].qkv, s);
        if (attention_decode_supported(rows_per_req, c.heads, c.kv_heads)) {
            // Decode: every row of a request in one block, RoPE and the KV append fused in.
            AttnDecodeArgs da{};
            da.qkv = b.qkv; da.ldq = qkvw; da.requests = rows / rows_per_req; da.rows_per_req = rows_per_req;
            da.hq = c.heads; da.hkv = c.kv_heads; da.pos0 = pos0; da.pos_dev = pos_dev; da.window = c.window;
            da.kc = kc; da.vc = vc; da.req_stride = req_stride; da.cap = b.cap; da.inv_freq = b.inv_freq;
            if (tc) { da.out_hi = b.attn.hi; da.out_lo = b.attn.lo; da.ld_split = b.attn.ld; }
            else { da.out = b.attn.f; da.ldo = b.attn.ld; }
            da.max_keys = max_keys; da.status = e->ctx->d_status;
            launch_attention_decode(da, s); g_kernels++;
            run(plans[l].o, s);
            norm_for(plans[l].gu, b.x, c.hidden, rows, L.norm2, c.eps, b.norm, s);
            run(plans[l].gu, s);
            run(plans[l].down, s);
            continue;
        }
        RopeArgs ra{};
        ra.qkv = b.qkv; ra.ldq = qkvw; ra.rows = rows; ra.rows_per_req = rows_per_req; ra.hq = c.heads;
        ra.hkv = c.kv_heads; ra.pos0 = pos0; ra.pos_dev = pos_dev; ra.kc = kc; ra.vc = vc; ra.req_stride = req_stride;
        ra.cap = b.cap; ra.inv_freq = b.inv_freq;
        launch_rope_cache(ra, s); g_kernels++;
        AttnArgs aa{};
        aa.q = b.qkv; aa.ldq = qkvw; aa.rows = rows; aa.rows_per_req = rows_per_req; aa.hq = c.heads; aa.hkv = c.kv_heads;
        aa.pos0 = pos0; aa.pos_dev = pos_dev; aa.window = c.window; aa.kc = kc; aa.vc = vc; aa.req_stride = req_stride;
        aa.cap = b.cap; aa.max_keys = max_keys;
        if (tc) { aa.out_hi = b.attn.hi; aa.out_lo = b.attn.lo; aa.ld_split = b.attn.ld; }
        else { aa.out = b.attn.f; aa.ldo = b.attn.ld; }
        launch_attention(aa, s); g_kernels++;
        run(plans[l].o, s);
        norm_for(plans[l].gu, b.x, c.hidden, rows, L.norm2, c.eps, b.norm, s);
        run(plans[l].gu, s);
        run(plans[l].down, s);
    }
}

// DiTForward.encode blocks (DiT.swift:35-48) over batch sequences of seq rows; the final layer is
// done by the caller.
void dit_blocks(mt_engine* e, const mt_dit_weights& W, DitBufs& b, std::vector<DitBlockPlans>& plans, int batch,
                int seq, cudaStream_t s) {
    const mt_dit_config& c = W.cfg;
    const int rows = batch * seq;
    for (int i = 0; i < c.depth; i++) {
        const mt_dit_block& B = W.blocks[i];
        const bool tc = plans[i].out.tc;  // the attention rows' consumer
        norm_for(plans[i].qkv, b.x, c.hidden, rows, B.norm1, c.eps, b.norm, s);
        run(plans[i].qkv, s);
        DitAttnArgs da{};
        da.qkv = b.qkv; da.ld = 3 * c.hidden; da.batch = batch; da.seq = seq; da.heads = c.heads;
        da.inv_freq = W.inv_freq;
        if (tc) { da.out_hi = b.attn.hi; da.out_lo = b.attn.lo; da.ld_split = b.attn.ld; }
        else { da.out = b.attn.f; da.ldo = b.attn.ld; }
        launch_dit_attention(da, s); g_kernels++;
        run(plans[i].out, s);
        norm_for(plans[i].ff1, b.x, c.hidden, rows, B.norm2, c.eps, b.norm, s);
        run(plans[i].ff1, s);
        run(plans[i].ff2, s);
    }
}

// DiT.swift:56-65 schedule and :68-79 sinusoid, in fp32 as the Swift Float code.
void flow_timesteps(int steps, float* out) {
    static const int e10[] = {0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32}, e5[] = {0, 2, 4, 8, 16, 32},
                     e6[] = {0, 2, 4, 6, 8, 16, 32}, e7[] = {0, 2, 4, 6, 8, 16, 24, 32},
                     e12[] = {0, 2, 4, 6, 8, 10, 12, 14, 16, 20, 24, 28, 32},
                     e16[] = {0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 12, 14, 16, 20, 24, 28, 32};
    const int* tab = steps == 10 ? e10 : steps == 5 ? e5 : steps == 6 ? e6 : steps == 7 ? e7 : steps == 12 ? e12
                   : steps == 16 ? e16 : nullptr;
    const float half_pi = 3.14159274101257324f / 2.0f;
    for (int i = 0; i <= steps; i++) {
        const float t = tab ? (float)tab[i] / 32.0f : (float)i / (float)steps;
        out[i] = t - (cosf(half_pi * t) - 1.0f + t);
    }
}

void sinusoid(float t, int dim, float* out) {
    const int half = dim / 2;
    const float step = (float)(log(10000.0) / (double)(half - 1));
    for (int i = 0; i < half; i++) {
        const float freq = expf((float)i * -step);
        const float arg = (1000.0f * t) * freq;
        out[i] = (float)sin((double)arg);
        out[half + i] = (float)cos((double)arg);
    }
}

mt_status precompute_temb(mt_engine* e) {
    const mt_model_config& c = e->cfg;
    const int FS = c.flow_steps, Df = c.flow.hidden;
    e->timesteps.resize(FS + 1);
    flow_timesteps(FS, e->timesteps.data());
    std::vector<float> sin_host((size_t)FS * c.time_dim);
    for (int k = 0; k < FS; k++) sinusoid(e->timesteps[k], c.time_dim, sin_host.data() + (size_t)k * c.time_dim);
    float *sinus = nullptr, *mid = nullptr;
    TRY(dalloc(e, &sinus, sin_host.size()));
    TRY(dalloc(e, &mid, (size_t)FS * Df));
    cudaMemcpy(sinus, sin_host.data(), sin_host.size() * sizeof(float), cudaMemcpyHostToDevice);
    TRY(mt_linear(e->ctx, nullptr, sinus, c.time_dim, FS, e->w.flow_t1_w, nullptr, e->w.flow_t1_b, Df, c.time_dim, mid,
                  Df, MT_LINEAR_BIAS | MT_LINEAR_SILU));
    TRY(mt_linear(e->ctx, nullptr, mid, Df, FS, e->w.flow_t2_w, nullptr, e->w.flow_t2_b, Df, Df, e->temb, Df,
                  MT_LINEAR_BIAS));
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return fail(e->ctx, MT_ERR_CUDA, "temb precompute: %s", cudaGetErrorString(err));
    return MT_OK;
}

// ---- step pieces ---------------------------------------------------------------------------------

void llm_token(mt_engine* e, Group& g, cudaStream_t s) {
    const mt_qwen_config& c = e->cfg.llm;
    if (g.llm_ps) {  // every layer and the final norm in one launch
        launch_stack(g.llm_sp, e->ctx->sm_count, s);
        g_kernels++;
        return;
    }
    qwen_forward(e, e->w.llm, g.llm, g.llm_dec, g.R, 1, 0, g.llm_pos, g.llm.cap, s);
    norm(g.llm.x, c.hidden, g.R, c.hidden, e->w.llm.final_norm, c.eps, g.z, g.R, true, s);
}

void flow_stage(mt_engine* e, Group& g, cudaStream_t s) {
    const mt_model_config& c = e->cfg;
    const int R = g.R, L = c.latent_dim, Df = c.flow.hidden;
    run(g.stop_lin, s);
    run(g.cond, s);
    launch_flow_begin(g.y, g.hist, g.noise, L, e->opt.max_steps, e->state_dev, R, s); g_kernels++;
    for (int k = 0; k < c.flow_steps; k++) {
        launch_flow_assemble_batched(g.y, g.hist, g.cemb, e->w.flow_c_b, e->temb + (size_t)k * Df, e->w.flow_x_w,
                                     e->w.flow_x_b, Df, L, g.flow.x, R, s);
        g_kernels++;
        if (g.flow_ps) {
            launch_stack(g.flow_sp, e->ctx->sm_count, s);
            g_kernels++;
        } else {
            dit_blocks(e, e->w.flow, g.flow, g.flow_blocks, 2 * R, 3, s);
        }
        FlowFinalArgs fa{};
        fa.X = g.flow.x; fa.hidden = Df; fa.norm_w = e->w.flow.final_norm; fa.eps = c.flow.eps;
        fa.final_w = e->w.flow.final_w; fa.final_b = e->w.flow.final_b; fa.latent = L; fa.y = g.y;
        fa.cfg = e->cfg_scale; fa.dt = e->timesteps[k + 1] - e->timesteps[k]; fa.vel0 = g.vel0;
        fa.flow_steps = c.flow_steps; fa.k = k; fa.latents = g.latents; fa.steps_cap = e->opt.max_steps;
        fa.state = e->state_dev;
        launch_flow_final(fa, R, s); g_kernels++;
    }
}

// Aggregator (Engine.swift:406-410): [cls, x_emb(latent)] -> DiT -> final layer of row 0 -> LLM input.
void agg_stage(mt_engine* e, Group& g, cudaStream_t s) {
    const mt_model_config& c = e->cfg;
    const int R = g.R, L = c.latent_dim;
    const int Da = c.agg.hidden;
    launch_agg_assemble(g.y, e->w.agg_cls, e->w.agg_x_w, e->w.agg_x_b, Da, L, g.agg.x, R, s); g_kernels++;
    if (g.agg_ps) {
        launch_stack(g.agg_sp, e->ctx->sm_count, s);
        g_kernels++;
    } else {
        dit_blocks(e, e->w.agg, g.agg, g.agg_blocks, R, 2, s);
    }
    norm(g.agg.x, 2 * Da, R, Da, e->w.agg.final_norm, c.agg.eps, g.agg_norm, R, false, s);
    run(g.agg_final, s);
}

void vae_fc1(mt_engine* e, Group& g, cudaStream_t s) {
    const mt_model_config& c = e->cfg;
    launch_vae_fc1(g.y, e->w.vae_fc1_w, e->w.vae_fc1_b, c.vae.hidden, c.latent_dim, g.vae_h, e->state_dev, g.R, s);
    g_kernels++;
}

// VAEDecoder.decodeDispatches (VAEDecoder.swift:86-107) for latent d of every request.
void vae_decode(mt_engine* e, cudaStream_t s) {
    const mt_model_config& c = e->cfg;
    const int R = e->R, Hv = c.vae.hidden;
    launch_vae_upsample(e->vae_h, Hv, e->state_dev, e->vae.x, R, s); g_kernels++;
    const int max_keys = c.vae.window > 0 ? c.vae.window : e->vae.cap;
    if (e->vae_ps) {  // every layer and the final norm in one launch
        launch_stack(e->vae_sp, e->ctx->sm_count, s);
        g_kernels++;
    } else {
        qwen_forward(e, e->w.vae, e->vae, e->vae_layers, 4 * R, 4, 0, e->state_dev + st_vae_pos(R), max_keys, s);
        norm(e->vae.x, Hv, 4 * R, Hv, e->w.vae.final_norm, c.vae.eps, e->vae_hidden, 4 * R, true, s);
    }
    run(e->vae_head, s);
    IstftArgs ia{};
    ia.spec = e->spec; ia.ld_spec = c.nfft + 2; ia.count = 4 * R; ia.nfft = c.nfft; ia.window = e->w.vae_window;
    ia.frames = e->fring; ia.req_stride = 8LL * c.nfft; ia.frames_per_req = 4; ia.frame0 = 0;
    ia.frame0_dev = e->state_dev + st_vae_pos(R); ia.ring = 8;
    launch_istft_frames(ia, s); g_kernels++;
    EmitArgs ea{};
    ea.frames = e->fring; ea.req_stride = 8LL * c.nfft; ea.window = e->w.vae_window; ea.nfft = c.nfft; ea.hop = c.hop;
    ea.s0 = 0; ea.s0_dev = e->state_dev + st_emit_s0(R); ea.count = 0; ea.count_dev = e->state_dev + st_emit_count(R);
    ea.last_frame = 0; ea.last_dev = e->state_dev + st_emit_last(R); ea.ring = 8; ea.out = e->pcm; ea.ld_out = e->max_chunk;
    launch_istft_emit(ea, e->max_chunk, R, s); g_kernels++;
}

// Host-side bookkeeping of one VAE decode (VAEDecoder.swift:96-106); fills the state header and
// per-request emission fields, returns the sample count.
int plan_decode(mt_engine* e, int d, bool has_next) {
    const int hop = e->cfg.hop, pad = (e->cfg.nfft - hop) / 2, R = e->R;
    const int frame_count = 4 * (d + 1);
    const int final_end = has_next ? frame_count * hop - pad : frame_count * hop;
    const int count = final_end - e->emitted;
    int* st = e->state_host;
    st[ST_D] = d;
    st[ST_HAS_NEXT] = has_next ? 1 : 0;
    for (int r = 0; r < R; r++) {
        st[st_vae_pos(R) + r] = 4 * d;
        st[st_emit_s0(R) + r] = e->emitted;
        st[st_emit_count(R) + r] = count;
        st[st_emit_last(R) + r] = frame_count - 1;
    }
    e->emitted = final_end;
    e->decoded = d + 1;
    return count;
}

void upload_state(mt_engine* e, cudaStream_t s) {
    cudaMemcpyAsync(e->state_dev, e->state_host, st_size(e->opt.max_requests) * sizeof(int), cudaMemcpyHostToDevice, s);
}

// Enqueues the device work of a step whose state is already uploaded. with_llm: n > 0;
// with_decode: a VAE decode is due.
// Forks the VAE decode (stream B) and every group's chain from s, and joins them back into s.
// Stage events (timed) are recorded on group 0's chain.
void enqueue_step(mt_engine* e, cudaStream_t s, bool with_llm, bool with_decode, bool timed) {
    cudaEvent_t* ev = e->stage_ev;
    if (timed) cudaEventRecord(ev[0], s);
    // A VAE decode that runs as a persistent stack launch takes every SM for its duration, as the
    // LLM token's does: it runs on the step stream before the groups instead of concurrently.
    const bool serial_decode = with_decode && e->vae_ps;
    if (serial_decode) {
        if (timed) cudaEventRecord(ev[4], s);
        vae_decode(e, s);
        if (timed) {
            cudaEventRecord(ev[5], s);
            cudaEventRecord(ev[0], s);
        }
    }
    cudaEventRecord(e->ev_fork, s);
    if (with_decode && !serial_decode) {
        cudaStreamWaitEvent(e->sb, e->ev_fork, 0);
        if (timed) cudaEventRecord(ev[4], e->sb);
        vae_decode(e, e->sb);
        if (timed) cudaEventRecord(ev[5], e->sb);
        cudaEventRecord(e->ev_join, e->sb);
    }
    // The groups' chain (LLM token -> flow -> aggregator) is the step's critical path; its kernels
    // go first when the concurrent VAE decode's blocks compete for SMs.
    const int prio_saved = launch_priority();
    launch_priority() = e->prio_hi;
    for (int i = 0; i < e->G; i++) {
        Group& g = e->groups[i];
        cudaStream_t gs = i == 0 ? s : g.s;
        if (i > 0) cudaStreamWaitEvent(gs, e->ev_fork, 0);
        if (with_llm) llm_token(e, g, gs);
        if (timed && i == 0) cudaEventRecord(ev[1], gs);
        flow_stage(e, g, gs);
        if (timed && i == 0) cudaEventRecord(ev[2], gs);
        agg_stage(e, g, gs);
        if (timed && i == 0) cudaEventRecord(ev[3], gs);
        vae_fc1(e, g, gs);
        if (i > 0) cudaEventRecord(g.done, gs);
    }
    launch_priority() = prio_saved;
    for (int i = 1; i < e->G; i++) cudaStreamWaitEvent(s, e->groups[i].done, 0);
    if (with_decode && !serial_decode) cudaStreamWaitEvent(s, e->ev_join, 0);
}

}  // namespace

extern "C" {

mt_status mt_engine_create(mt_ctx* ctx, const mt_model* model, const mt_engine_options* opt, mt_engine** out) {
    MT_REQUIRE(ctx, ctx && model && opt && out, MT_ERR_ARG, "mt_engine_create: null argument");
    *out = nullptr;
    const mt_model_config* cfgp = mt_model_get_config(model);
    const mt_model_config& c = *cfgp;
    MT_REQUIRE(ctx, opt->max_requests >= 1 && opt->max_prompt >= 1 && opt->max_steps >= 1 &&
                        opt->max_prompt + opt->max_steps <= c.llm_capacity,
               MT_ERR_CAPACITY, "mt_engine_create: requests %d prompt %d steps %d (prompt + steps <= %d)",
               opt->max_requests, opt->max_prompt, opt->max_steps, c.llm_capacity);
    const int ring = opt->vae_ring > 0 ? opt->vae_ring : 128;
    MT_REQUIRE(ctx, c.vae.window > 0 && ring >= c.vae.window + 3, MT_ERR_CAPACITY,
               "mt_engine_create: VAE ring %d must hold window %d + 3 positions", ring, c.vae.window);
    mt_engine* e = new mt_engine();
    e->ctx = ctx;
    e->model = model;
    e->cfg = c;
    e->w = *mt_model_get_weights(model);
    e->opt = *opt;
    e->opt.vae_ring = ring;
    const int R = opt->max_requests, T = opt->max_prompt, S = opt->max_steps;
    auto cleanup = [&](mt_status st) {
        mt_engine_destroy(e);
        return st;
    };
#define ETRY(expr)                                    \
    do {                                              \
        mt_status _s = (expr);                        \
        if (_s != MT_OK) return cleanup(_s);          \
    } while (0)
    ETRY(qwen_alloc(e, &e->llm, c.llm, (size_t)R * T, R, c.llm_capacity));
    ETRY(act_alloc(e, &e->z, R, c.llm.hidden));
    ETRY(dalloc(e, &e->stop, (size_t)R * 2));
    ETRY(dalloc(e, &e->temb, (size_t)c.flow_steps * c.flow.hidden));
    ETRY(dalloc(e, &e->cemb, (size_t)R * c.flow.hidden));
    ETRY(dalloc(e, &e->y, (size_t)R * c.latent_dim));
    ETRY(dalloc(e, &e->hist, (size_t)R * c.latent_dim));
    ETRY(dalloc(e, &e->noise, (size_t)R * S * c.latent_dim));
    ETRY(dalloc(e, &e->latents, (size_t)R * S * c.latent_dim));
    ETRY(dalloc(e, &e->vel0, (size_t)R * c.flow_steps * 2 * c.latent_dim));
    ETRY(dit_alloc(e, &e->flow, c.flow, (size_t)6 * R));
    ETRY(dit_alloc(e, &e->agg, c.agg, (size_t)2 * R));
    ETRY(act_alloc(e, &e->agg_norm, R, c.agg.hidden));
    ETRY(dalloc(e, &e->vae_h, (size_t)R * VAE_H_RING * c.vae.hidden));
    ETRY(qwen_alloc(e, &e->vae, c.vae, (size_t)4 * R, R, ring));
    ETRY(act_alloc(e, &e->vae_hidden, (size_t)4 * R, c.vae.hidden));
    ETRY(dalloc(e, &e->spec, (size_t)4 * R * (c.nfft + 2)));
    ETRY(dalloc(e, &e->fring, (size_t)R * 8 * c.nfft));
    e->max_chunk = 4 * c.hop + (c.nfft - c.hop) / 2;
    ETRY(dalloc(e, &e->pcm, (size_t)R * e->max_chunk));
    ETRY(dalloc(e, &e->state_dev, (size_t)st_size(R)));
    e->ws_a_floats = std::max({(size_t)R * 2 * c.llm.intermediate, (size_t)6 * R * 2 * c.flow.ff,
                               (size_t)2 * R * 2 * c.agg.ff});
    e->ws_b_floats = (size_t)4 * R * 2 * c.vae.intermediate;
    ETRY(dalloc(e, &e->ws_a, e->ws_a_floats));
    ETRY(dalloc(e, &e->ws_b, e->ws_b_floats));
    ETRY(dalloc(e, &e->ids_stage, (size_t)R * T));
    {
        // Persistent-stack areas (zeroed here, once): one per request group, one for the VAE decode.
        const size_t group_area = std::max(qwen_area_bound(c.llm, 1, c.llm_capacity),
                                           std::max(dit_area_bound(c.flow), dit_area_bound(c.agg)));
        uint8_t* a = nullptr;
        ETRY(dalloc(e, &a, qwen_area_bound(c.vae, 4, ring)));
        e->vae_area = a;
        for (int i = 0; i < kMaxGroups; i++) {
            ETRY(dalloc(e, &a, group_area));
            e->groups[i].stack_area = a;
        }
    }
    if (cudaMallocHost(&e->state_slots[0], st_size(R) * sizeof(int)) != cudaSuccess ||
        cudaMallocHost(&e->state_slots[1], st_size(R) * sizeof(int)) != cudaSuccess ||
        cudaMallocHost(&e->ring_host, (size_t)kPcmRing * R * e->max_chunk * sizeof(float)) != cudaSuccess ||
        cudaMallocHost(&e->stop_host, (size_t)S * R * 2 * sizeof(float)) != cudaSuccess)
        return cleanup(fail(ctx, MT_ERR_NOMEM, "engine: pinned host staging"));
    for (int i = 0; i < kPcmRing; i++)
        if (cudaEventCreateWithFlags(&e->ring_ev[i], cudaEventDisableTiming) != cudaSuccess)
            return cleanup(fail(ctx, MT_ERR_CUDA, "engine: events"));
    memset(e->state_slots[0], 0, st_size(R) * sizeof(int));
    memset(e->state_slots[1], 0, st_size(R) * sizeof(int));
    e->state_host = e->state_slots[0];
    for (int i = 0; i < 2; i++)
        if (cudaEventCreateWithFlags(&e->state_ev[i], cudaEventDisableTiming) != cudaSuccess)
            return cleanup(fail(ctx, MT_ERR_CUDA, "engine: events"));
    for (int i = 0; i < 6; i++)
        if (cudaEventCreate(&e->stage_ev[i]) != cudaSuccess) return cleanup(fail(ctx, MT_ERR_CUDA, "engine: events"));
    // One priority for every stream (a lower-priority VAE stream was measured to slow the VAE
    // decode, 1.8 -> 2.5 ms, without shortening the LLM stage it overlaps); the groups' kernels
    // carry the device's highest priority as a launch attribute instead (enqueue_step).
    {
        int least = 0, greatest = 0;
        cudaDeviceGetStreamPriorityRange(&least, &greatest);
        e->prio_hi = greatest;
    }
    if (cudaStreamCreateWithFlags(&e->sa, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&e->sb, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_join, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_in, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_out, cudaEventDisableTiming) != cudaSuccess)
        return cleanup(fail(ctx, MT_ERR_CUDA, "engine: stream/event creation"));
    for (int i = 1; i < group_count(e, R); i++)
        if (cudaStreamCreateWithFlags(&e->groups[i].s, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&e->groups[i].done, cudaEventDisableTiming) != cudaSuccess)
            return cleanup(fail(ctx, MT_ERR_CUDA, "engine: group stream/event creation"));
    ETRY(precompute_temb(e));
#undef ETRY
    *out = e;
    return MT_OK;
}

void mt_engine_destroy(mt_engine* e) {
    if (!e) return;
    for (int i = 0; i < 2; i++) {
        if (e->graph_exec[i]) cudaGraphExecDestroy(e->graph_exec[i]);
        if (e->graph[i]) cudaGraphDestroy(e->graph[i]);
        if (e->state_ev[i]) cudaEventDestroy(e->state_ev[i]);
        if (e->state_slots[i]) cudaFreeHost(e->state_slots[i]);
    }
    if (e->sa) cudaStreamDestroy(e->sa);
    if (e->sb) cudaStreamDestroy(e->sb);
    for (int i = 0; i < kMaxGroups; i++) {
        if (e->groups[i].s) cudaStreamDestroy(e->groups[i].s);
        if (e->groups[i].done) cudaEventDestroy(e->groups[i].done);
    }
    if (e->ev_fork) cudaEventDestroy(e->ev_fork);
    if (e->ev_join) cudaEventDestroy(e->ev_join);
    if (e->ev_in) cudaEventDestroy(e->ev_in);
    for (int i = 0; i < 6; i++)
        if (e->stage_ev[i]) cudaEventDestroy(e->stage_ev[i]);
    if (e->ev_out) cudaEventDestroy(e->ev_out);
    if (e->ring_host) cudaFreeHost(e->ring_host);
    if (e->stop_host) cudaFreeHost(e->stop_host);
    for (int i = 0; i < kPcmRing; i++)
        if (e->ring_ev[i]) cudaEventDestroy(e->ring_ev[i]);
    for (void* p : e->allocs) cudaFree(p);
    delete e;
}

mt_status mt_engine_begin(mt_engine* e, void* stream, int requests, int prompt_rows, const float* embeds,
                          const int32_t* token_ids, const float* noise, const float* initial_history, int steps,
                          float cfg) {
    if (!e) return MT_ERR_ARG;
    mt_ctx* ctx = e->ctx;
    const mt_model_config& c = e->cfg;
    MT_REQUIRE(ctx, (embeds || token_ids) && noise, MT_ERR_ARG, "mt_engine_begin: need embeds or token ids, and noise");
    MT_REQUIRE(ctx, !token_ids || e->w.embed_tokens, MT_ERR_ARG, "mt_engine_begin: model has no embedding table");
    MT_REQUIRE(ctx, requests >= 1 && requests <= e->opt.max_requests && prompt_rows >= 1 &&
                        prompt_rows <= e->opt.max_prompt && steps >= 1 && steps <= e->opt.max_steps &&
                        prompt_rows + steps <= c.llm_capacity,
               MT_ERR_CAPACITY, "mt_engine_begin: requests %d prompt %d steps %d exceed the engine's capacity",
               requests, prompt_rows, steps);
    cudaStream_t s = as_stream(stream);
    e->R = requests;
    e->T = prompt_rows;
    e->steps = steps;
    e->cfg_scale = cfg;
    e->n = 0;
    e->latents_fed = e->decoded = e->emitted = 0;
    e->prefilled = false;
    if (e->plan_R != requests || e->plan_persistent != ctx->persistent) {
        for (int i = 0; i < 2; i++) {
            if (e->graph_exec[i]) cudaGraphExecDestroy(e->graph_exec[i]);
            if (e->graph[i]) cudaGraphDestroy(e->graph[i]);
            e->graph_exec[i] = nullptr;
            e->graph[i] = nullptr;
        }
    }
    TRY(build_plans(e));
    const int H = c.llm.hidden, L = c.latent_dim, S = e->opt.max_steps;
    if (embeds) {
        cudaMemcpyAsync(e->llm.x, embeds, sizeof(float) * (size_t)requests * prompt_rows * H, cudaMemcpyDefault, s);
    } else {
        launch_embed_gather(token_ids, requests * prompt_rows, e->w.embed_tokens, H, c.vocab, e->llm.x, ctx->d_status, s);
    }
    cudaMemcpy2DAsync(e->noise, (size_t)S * L * sizeof(float), noise, (size_t)steps * L * sizeof(float),
                      (size_t)steps * L * sizeof(float), requests, cudaMemcpyDefault, s);
    if (initial_history)
        cudaMemcpyAsync(e->hist, initial_history, sizeof(float) * (size_t)requests * L, cudaMemcpyDefault, s);
    else
        cudaMemsetAsync(e->hist, 0, sizeof(float) * (size_t)requests * L, s);
    cudaMemsetAsync(e->y, 0, sizeof(float) * (size_t)requests * L, s);
    // KV caches need no reset: every position is written before it is read.
    e->begun = true;
    return check_launch(ctx, "mt_engine_begin");
}

mt_status mt_engine_prefill(mt_engine* e, void* stream) {
    if (!e) return MT_ERR_ARG;
    MT_REQUIRE(e->ctx, e->begun && !e->prefilled, MT_ERR_STATE, "mt_engine_prefill: call after mt_engine_begin, once");
    cudaStream_t s = as_stream(stream);
    const mt_qwen_config& c = e->cfg.llm;
    const int R = e->R, T = e->T;
    qwen_forward(e, e->w.llm, e->llm, e->llm_pre, R * T, T, 0, nullptr, T, s);
    // Final norm of each request's last row -> z (normRows 1, Engine.swift:329).
    norm(e->llm.x + (size_t)(T - 1) * c.hidden, T * c.hidden, R, c.hidden, e->w.llm.final_norm, c.eps, e->z, R, true, s);
    e->prefilled = true;
    return check_launch(e->ctx, "mt_engine_prefill");
}

mt_status mt_engine_step(mt_engine* e, void* stream, int* pcm_count) {
    if (!e) return MT_ERR_ARG;
    mt_ctx* ctx = e->ctx;
    MT_REQUIRE(ctx, e->prefilled, MT_ERR_STATE, "mt_engine_step: prefill first");
    MT_REQUIRE(ctx, e->n < e->steps, MT_ERR_STATE, "mt_engine_step: all %d steps done", e->steps);
    cudaStream_t caller = as_stream(stream);
    cudaStream_t s = e->sa;
    const int R = e->R, n = e->n;
    // Step n fills state slot n & 1; the step that last read that slot (n - 2) must be done with it.
    const int slot = n & 1;
    if (e->state_ev_live[slot]) {
        cudaError_t err = cudaEventSynchronize(e->state_ev[slot]);
        if (err != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "mt_engine_step: %s", cudaGetErrorString(err));
    }
    e->state_host = e->state_slots[slot];
    int* st = e->state_host;
    st[ST_N] = n;
    for (int r = 0; r < R; r++) st[st_llm_pos(R) + r] = e->T + n - 1;
    // Deferred decode (VAEDecoder.deferredDecode, :73-76): latent n-2 once latent n-1 exists.
    const bool with_decode = e->decoded + 1 < e->latents_fed;
    int count = 0;
    if (with_decode) count = plan_decode(e, e->decoded, true);
    else st[ST_D] = -1;
    const bool with_llm = n > 0;
    const bool steady = with_llm && with_decode;
    // The step runs on the engine's own stream, ordered after the caller's work and joined back.
    cudaEventRecord(e->ev_in, caller);
    cudaStreamWaitEvent(s, e->ev_in, 0);
    e->stage_valid = false;
    if (steady && e->opt.use_graphs && !e->time_stages) {
        if (!e->graph_exec[slot]) {
            cudaError_t err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
            if (err != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "step graph capture: %s", cudaGetErrorString(err));
            upload_state(e, s);
            g_kernels = 0;
            enqueue_step(e, s, true, true, false);
            e->graph_kernels = g_kernels;
            err = cudaStreamEndCapture(s, &e->graph[slot]);
            if (err != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "step graph capture: %s", cudaGetErrorString(err));
            err = cudaGraphInstantiate(&e->graph_exec[slot], e->graph[slot], cudaGraphInstantiateFlagUseNodePriority);
            if (err != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "step graph instantiate: %s", cudaGetErrorString(err));
        }
        cudaGraphLaunch(e->graph_exec[slot], s);
        e->step_kernels = e->graph_kernels;
    } else {
        upload_state(e, s);
        g_kernels = 0;
        const bool timed = e->time_stages && with_llm && with_decode;
        enqueue_step(e, s, with_llm, with_decode, timed);
        e->stage_valid = timed;
        e->step_kernels = g_kernels;
    }
    cudaEventRecord(e->ev_out, s);
    cudaStreamWaitEvent(caller, e->ev_out, 0);
    cudaEventRecord(e->state_ev[slot], s);
    e->state_ev_live[slot] = true;
    e->latents_fed++;
    e->n++;
    if (pcm_count) *pcm_count = count;
    return check_launch(ctx, "mt_engine_step");
}

mt_status mt_engine_flush(mt_engine* e, void* stream, int* pcm_count) {
    if (!e) return MT_ERR_ARG;
    MT_REQUIRE(e->ctx, e->prefilled, MT_ERR_STATE, "mt_engine_flush: nothing generated");
    cudaStream_t s = as_stream(stream);
    if (pcm_count) *pcm_count = 0;
    if (e->decoded >= e->latents_fed) return MT_OK;
    cudaStreamSynchronize(s);
    for (int i = 0; i < 2; i++)
        if (e->state_ev_live[i]) cudaEventSynchronize(e->state_ev[i]);
    e->state_host = e->state_slots[0];
    const int d = e->decoded;
    const int count = plan_decode(e, d, d + 1 < e->latents_fed);
    upload_state(e, s);
    vae_decode(e, s);
    if (pcm_count) *pcm_count = count;
    return check_launch(e->ctx, "mt_engine_flush");
}

mt_status mt_engine_buffer(const mt_engine* e, int which, const float** ptr, long long* stride) {
    if (!e || !ptr || !stride) return MT_ERR_ARG;
    const mt_model_config& c = e->cfg;
    switch (which) {
        case MT_BUF_Z: *ptr = e->z.f; *stride = c.llm.hidden; break;
        case MT_BUF_STOP_LOGITS: *ptr = e->stop; *stride = 2; break;
        case MT_BUF_LATENTS: *ptr = e->latents; *stride = (long long)e->opt.max_steps * c.latent_dim; break;
        case MT_BUF_AGG_OUT: *ptr = e->llm.x; *stride = c.llm.hidden; break;
        case MT_BUF_VELOCITY0: *ptr = e->vel0; *stride = (long long)c.flow_steps * 2 * c.latent_dim; break;
        case MT_BUF_VAE_HIDDEN: *ptr = e->vae_hidden.f; *stride = 4LL * c.vae.hidden; break;
        case MT_BUF_PCM: *ptr = e->pcm; *stride = e->max_chunk; break;
        default: return MT_ERR_ARG;
    }
    return MT_OK;
}

int mt_engine_steps_done(const mt_engine* e) { return e ? e->n : -1; }

int mt_engine_step_kernels(const mt_engine* e) { return e ? e->step_kernels : -1; }

mt_status mt_engine_set_stage_timing(mt_engine* e, int on) {
    if (!e) return MT_ERR_ARG;
    e->time_stages = on != 0;
    return MT_OK;
}

mt_status mt_engine_set_stop_rule(mt_engine* e, int on) {
    if (!e) return MT_ERR_ARG;
    e->stop_rule = on != 0;
    return MT_OK;
}

mt_status mt_engine_stage_ms(mt_engine* e, float* ms4) {
    if (!e || !ms4) return MT_ERR_ARG;
    MT_REQUIRE(e->ctx, e->stage_valid, MT_ERR_STATE, "mt_engine_stage_ms: last step was not timed");
    cudaEvent_t* ev = e->stage_ev;
    cudaEventSynchronize(ev[3]);
    cudaEventSynchronize(ev[5]);
    cudaEventElapsedTime(&ms4[0], ev[0], ev[1]);
    cudaEventElapsedTime(&ms4[1], ev[1], ev[2]);
    cudaEventElapsedTime(&ms4[2], ev[2], ev[3]);
    cudaEventElapsedTime(&ms4[3], ev[4], ev[5]);
    return MT_OK;
}

}  // extern "C"

namespace {

// The generation loop shared by mt_engine_generate and mt_engine_generate_stream: prompt and noise
// in, prefill, `steps` steps, flush. Each PCM emission ([R][max_chunk] on the device) is copied into
// the next pinned ring slot behind an event; `sink(i, count, slot, request_stride)` receives emission
// i in order as soon as its copy has landed (polled after every enqueue, waited for only when the
// ring is full or at the end), so the host handles chunk i while the GPU runs later steps. A
// non-zero sink return cancels: no further work is enqueued and MT_ERR_STATE is returned.
template <typename Sink>
mt_status generate_loop(mt_engine* e, void* stream, int requests, int prompt_rows, const float* embeds_host,
                        const int32_t* ids_host, const float* noise_host, int steps, float cfg, long long pcm_limit,
                        float* stop_prob_host, long long* pcm_count, const char* who, Sink&& sink) {
    mt_ctx* ctx = e->ctx;
    const mt_model_config& c = e->cfg;
    MT_REQUIRE(ctx, requests >= 1 && requests <= e->opt.max_requests && prompt_rows >= 1 &&
                        prompt_rows <= e->opt.max_prompt && steps >= 1 && steps <= e->opt.max_steps,
               MT_ERR_CAPACITY, "%s: requests %d prompt %d steps %d exceed the engine", who, requests, prompt_rows,
               steps);
    (void)c;
    cudaStream_t s = as_stream(stream);
    // Prompt and noise go straight from the caller's buffers into the engine (begin copies embeds and
    // noise from host or device memory); token ids go through a device stage for the gather kernel.
    mt_status st = MT_OK;
    const int32_t* ids_dev = nullptr;
    if (!embeds_host) {
        cudaError_t err = cudaMemcpyAsync(e->ids_stage, ids_host, (size_t)requests * prompt_rows * sizeof(int32_t),
                                          cudaMemcpyHostToDevice, s);
        if (err != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "%s: %s", who, cudaGetErrorString(err));
        ids_dev = e->ids_stage;
    }
    st = mt_engine_begin(e, stream, requests, prompt_rows, embeds_host, ids_dev, noise_host, nullptr, steps, cfg);
    if (st == MT_OK) st = mt_engine_prefill(e, stream);

    const size_t chunk_floats = (size_t)requests * e->max_chunk;
    std::vector<int> counts;
    size_t delivered = 0;
    long long total = 0;
    bool cancelled = false;
    auto deliver = [&](size_t i) -> bool {
        const float* src = e->ring_host + (i % kPcmRing) * chunk_floats;
        if (sink(i, counts[i], src, (long long)e->max_chunk) != 0) cancelled = true;
        return !cancelled;
    };
    // Hands over every emission whose copy has landed; with wait, also waits for emission `upto - 1`.
    auto drain = [&](size_t upto, bool wait) -> mt_status {
        while (delivered < upto && !cancelled) {
            cudaEvent_t ev = e->ring_ev[delivered % kPcmRing];
            cudaError_t q = cudaEventQuery(ev);
            if (q == cudaErrorNotReady) {
                if (!wait) break;
                q = cudaEventSynchronize(ev);
            }
            if (q != cudaSuccess) return fail(ctx, MT_ERR_CUDA, "%s: %s", who, cudaGetErrorString(q));
            deliver(delivered++);
        }
        return MT_OK;
    };
    auto emit = [&](int count) -> mt_status {
        MT_REQUIRE(ctx, total + count <= pcm_limit, MT_ERR_CAPACITY, "%s: %lld samples exceed %lld", who,
                   total + count, pcm_limit);
        const size_t i = counts.size();
        if (i >= (size_t)kPcmRing) {  // the slot's previous emission must be handed over first
            mt_status d = drain(i - kPcmRing + 1, true);
            if (d != MT_OK) return d;
        }
        const int slot = (int)(i % kPcmRing);
        cudaMemcpyAsync(e->ring_host + slot * chunk_floats, e->pcm, chunk_floats * sizeof(float),
                        cudaMemcpyDeviceToHost, s);
        cudaEventRecord(e->ring_ev[slot], s);
        counts.push_back(count);
        total += count;
        return drain(counts.size(), false);
    };
    // With the stop rule (MingEngine.generate, Engine.swift:347-355) the host reads each step's stop
    // logits before enqueuing the next step, as the reference does; the batch ends after the step
    // at which the last request has met p > 0.5 with n > 3 (a request keeps its first such step).
    std::vector<char> met(e->stop_rule ? requests : 0, 0);
    int n = 0;
    for (; st == MT_OK && !cancelled && n < steps; n++) {
        int count = 0;
        st = mt_engine_step(e, stream, &count);
        if (st != MT_OK) break;
        cudaMemcpyAsync(e->stop_host + (size_t)n * requests * 2, e->stop, (size_t)requests * 2 * sizeof(float),
                        cudaMemcpyDeviceToHost, s);
        if (count > 0) st = emit(count);
        if (st != MT_OK || !e->stop_rule) continue;
        cudaError_t err = cudaStreamSynchronize(s);
        if (err != cudaSuccess) {
            st = fail(ctx, MT_ERR_CUDA, "%s: %s", who, cudaGetErrorString(err));
            break;
        }
        int remaining = 0;
        for (int r = 0; r < requests; r++) {
            const float* l = e->stop_host + ((size_t)n * requests + r) * 2;
            if (1.0f / (1.0f + expf(l[0] - l[1])) > 0.5f && n > 3) met[r] = 1;
            remaining += !met[r];
        }
        if (remaining == 0) {
            n++;
            break;
        }
    }
    const int ran = n;
    while (st == MT_OK && !cancelled) {
        int count = 0;
        st = mt_engine_flush(e, stream, &count);
        if (st != MT_OK || count == 0) break;
        st = emit(count);
    }
    cudaError_t err = cudaStreamSynchronize(s);
    if (st == MT_OK && err != cudaSuccess) st = fail(ctx, MT_ERR_CUDA, "%s: %s", who, cudaGetErrorString(err));
    if (st == MT_OK && !cancelled) st = drain(counts.size(), true);
    if (st == MT_OK && cancelled)
        st = fail(ctx, MT_ERR_STATE, "%s: cancelled by the chunk callback after chunk %zu", who, delivered - 1);
    if (st == MT_OK) {
        if (pcm_count) *pcm_count = total;
        if (stop_prob_host)
            for (int k = 0; k < steps; k++)
                for (int r = 0; r < requests; r++) {
                    const float* l = e->stop_host + ((size_t)k * requests + r) * 2;
                    stop_prob_host[(size_t)r * steps + k] =
                        k < ran ? 1.0f / (1.0f + expf(l[0] - l[1])) : 0.0f;  // Engine.swift:349
                }
    }
    return st;
}

}  // namespace

extern "C" {

mt_status mt_engine_generate(mt_engine* e, void* stream, int requests, int prompt_rows, const float* embeds_host,
                             const int32_t* ids_host, const float* noise_host, int steps, float cfg, float* pcm_host,
                             long long pcm_stride, long long* pcm_count, float* stop_prob_host) {
    if (!e) return MT_ERR_ARG;
    mt_ctx* ctx = e->ctx;
    MT_REQUIRE(ctx, (embeds_host || ids_host) && noise_host && pcm_host && pcm_count, MT_ERR_ARG,
               "mt_engine_generate: null argument");
    MT_REQUIRE(ctx, pcm_stride >= 4LL * e->cfg.hop * steps, MT_ERR_CAPACITY,
               "mt_engine_generate: pcm_stride %lld < %lld samples", pcm_stride, 4LL * e->cfg.hop * steps);
    long long offset = 0;
    return generate_loop(e, stream, requests, prompt_rows, embeds_host, ids_host, noise_host, steps, cfg, pcm_stride,
                         stop_prob_host, pcm_count, "mt_engine_generate",
                         [&](size_t, int count, const float* src, long long src_stride) {
                             for (int r = 0; r < requests; r++)
                                 memcpy(pcm_host + r * pcm_stride + offset, src + r * src_stride, count * sizeof(float));
                             offset += count;
                             return 0;
                         });
}

mt_status mt_engine_generate_stream(mt_engine* e, void* stream, int requests, int prompt_rows,
                                    const float* embeds_host, const int32_t* ids_host, const float* noise_host,
                                    int steps, float cfg, mt_pcm_chunk_fn on_chunk, void* user,
                                    long long* pcm_count, float* stop_prob_host) {
    if (!e) return MT_ERR_ARG;
    mt_ctx* ctx = e->ctx;
    MT_REQUIRE(ctx, (embeds_host || ids_host) && noise_host && on_chunk, MT_ERR_ARG,
               "mt_engine_generate_stream: null argument");
    return generate_loop(e, stream, requests, prompt_rows, embeds_host, ids_host, noise_host, steps, cfg,
                         1LL << 62, stop_prob_host, pcm_count, "mt_engine_generate_stream",
                         [&](size_t i, int count, const float* src, long long src_stride) {
                             return on_chunk(user, (int)i, requests, count, src, src_stride);
                         });
}

}  // extern "C"
