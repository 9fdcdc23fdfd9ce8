/*
 * mingcuda.h -- C ABI of libmingcuda.so, the B200 (sm_100a) kernels and host engine for the
 * per-step inference loop of Ming-3.0-tts-0.5B.
 *
 * The operator entry points mirror the reference's `Encoder` methods one for one
 * (Sources/MingTTS/Engine/Kernels.swift:89-283): same argument meaning, same row-stride views,
 * same epilogue flag bits. Each appends device work to the caller's stream and returns a status;
 * nothing synchronises and nothing allocates. All device pointers are caller-owned.
 * The engine entry points mirror `MingEngine.generate` / `encodeStep`
 * (Sources/MingTTS/Engine/Engine.swift:302-415) for R concurrent requests.
 *
 * Types: weights are bf16 (mt_bf16 = raw uint16 bits), activations, KV caches and outputs fp32.
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * Errors never cross the ABI as exceptions: every function returns an mt_status; the message of
 * the last failure on a context is mt_last_error(ctx).
 */
#ifndef MINGCUDA_H
#define MINGCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t mt_bf16;
typedef struct mt_ctx mt_ctx;
typedef struct mt_model mt_model;
typedef struct mt_engine mt_engine;

/* Status codes. Replaces the Swift `MingTTSError` enum (Sources/MingTTS/Engine/MetalContext.swift:6-26)
 * and the `precondition` crashes on shape misuse (Kernels.swift:105, 217). */
typedef enum {
    MT_OK = 0,
    MT_ERR_ARG = 1,       /* null pointer, bad stride or flag combination */
    MT_ERR_SHAPE = 2,     /* a shape the kernel does not support */
    MT_ERR_CAPACITY = 3,  /* KV cache or workspace would overflow */
    MT_ERR_CUDA = 4,      /* a CUDA runtime error (message has the CUDA string) */
    MT_ERR_TIMEOUT = 5,   /* a bounded device wait gave up (status word set by a kernel) */
    MT_ERR_NOMEM = 6,     /* a library allocation failed (engine/model creation only) */
    MT_ERR_STATE = 7,     /* call out of order (engine not begun, already flushed, ...) */
    MT_ERR_CHECKPOINT = 8 /* unreadable or malformed checkpoint, missing tensor, wrong dtype or size */
} mt_status;

/* Epilogue flags of a linear, same bits as GemvFlags (Kernels.swift:21-27, Shaders.swift:40-44).
 * Applied in this order: +bias, silu(v)*(x.W2^T), gelu_tanh, silu, +=y. */
enum {
    MT_LINEAR_BIAS = 1,
    MT_LINEAR_ACCUM = 2,
    MT_LINEAR_GELU = 4,
    MT_LINEAR_SILU_GATE = 8,
    MT_LINEAR_SILU = 16
};

/* ---------------------------------------------------------------------------------------------
 * Model description (plain structs of caller-owned pointers)
 * ------------------------------------------------------------------------------------------- */

/* QwenConfig (Sources/MingTTS/Engine/Weights.swift:81-92). Head dim is fixed at 64. */
typedef struct {
    int hidden;        /* 896 */
    int heads;         /* 14 query heads */
    int kv_heads;      /* 2 */
    int intermediate;  /* 4864 */
    int layers;        /* 24 */
    int window;        /* 0 = full causal; 65 for the VAE decoder stack (Weights.swift:216-217) */
    float rope_theta;  /* 1e6 */
    float eps;         /* 1e-6 */
} mt_qwen_config;

/* One Qwen2 layer (QwenLayerWeights, Weights.swift:94-102, 116-131). */
typedef struct {
    const mt_bf16* norm1;   /* input_layernorm [hidden] */
    const mt_bf16* qkv_w;   /* q_proj, k_proj, v_proj rows concatenated [(heads+2*kv)*64, hidden] */
    const mt_bf16* qkv_b;   /* [(heads+2*kv)*64] */
    const mt_bf16* o_w;     /* [hidden, heads*64] */
    const mt_bf16* norm2;   /* post_attention_layernorm [hidden] */
    const mt_bf16* gate_w;  /* [intermediate, hidden] */
    const mt_bf16* up_w;    /* [intermediate, hidden] */
    const mt_bf16* down_w;  /* [hidden, intermediate] */
} mt_qwen_layer;

typedef struct {
    mt_qwen_config cfg;
    const mt_qwen_layer* layers;  /* host array of cfg.layers entries */
    const mt_bf16* final_norm;    /* [hidden] */
} mt_qwen_weights;

/* DiT stack (DiTWeights, Weights.swift:145-172); head dim 64, hidden = heads * 64. */
typedef struct {
    int hidden;   /* 1024 */
    int heads;    /* 16 */
    int depth;    /* 8 */
    int ff;       /* 4096, GELU-tanh MLP */
    int out_dim;  /* 64 for the flow head, 896 for the aggregator */
    float eps;    /* 1e-6 */
} mt_dit_config;

typedef struct {
    const mt_bf16 *norm1, *qkv_w, *qkv_b;  /* qkv: to_q,to_k,to_v concatenated [3*hidden, hidden] */
    const mt_bf16 *out_w, *out_b;          /* attn.to_out.0 [hidden, hidden] */
    const mt_bf16 *norm2;
    const mt_bf16 *ff1_w, *ff1_b;          /* mlp.ff.0.0 [ff, hidden] */
    const mt_bf16 *ff2_w, *ff2_b;          /* mlp.ff.2 [hidden, ff] */
} mt_dit_block;

typedef struct {
    mt_dit_config cfg;
    const mt_dit_block* blocks;                    /* host array of cfg.depth entries */
    const mt_bf16 *final_norm, *final_w, *final_b; /* final_layer.norm_final, final_layer.linear [out_dim, hidden] */
    const float* inv_freq;                         /* rotary_embed.inv_freq [32] */
} mt_dit_weights;

/* Every dimension of the per-step loop. mt_model_config_default gives Ming-3.0-tts-0.5B. */
typedef struct {
    mt_qwen_config llm;   /* LLM stack */
    mt_qwen_config vae;   /* VAE decoder stack (window 65) */
    mt_dit_config flow;   /* flow-matching head DiT (out_dim = latent_dim) */
    mt_dit_config agg;    /* aggregator DiT (out_dim = llm.hidden) */
    int latent_dim;       /* 64 */
    int time_dim;         /* 256: sinusoidal timestep embedding width */
    int vocab;            /* 151936 */
    int nfft;             /* 3528 */
    int hop;              /* 882 */
    int flow_steps;       /* 10 Euler steps */
    int llm_capacity;     /* 512 positions */
} mt_model_config;

/* All weights of the per-step loop, as device (engine) or host (oracle) pointers. Names follow the
 * checkpoint tensors listed in Weights.swift:174-263. */
typedef struct {
    mt_qwen_weights llm;
    const mt_bf16 *stop_w, *stop_b;          /* stop_head [2, llm.hidden] */
    const mt_bf16 *flow_x_w, *flow_x_b;      /* flowloss.cfm.model.x_embedder [flow.hidden, latent] */
    const mt_bf16 *flow_c_w, *flow_c_b;      /* c_embedder.cond_embedder [flow.hidden, llm.hidden] */
    const mt_bf16 *flow_t1_w, *flow_t1_b;    /* t_embedder.time_mlp.0 [flow.hidden, time_dim] */
    const mt_bf16 *flow_t2_w, *flow_t2_b;    /* t_embedder.time_mlp.2 [flow.hidden, flow.hidden] */
    mt_dit_weights flow;
    const mt_bf16 *agg_x_w, *agg_x_b;        /* linear_proj_audio.x_embedder [agg.hidden, latent] */
    const float* agg_cls;                    /* linear_proj_audio.word_embedder.weight [agg.hidden] */
    mt_dit_weights agg;
    const mt_bf16 *vae_fc1_w, *vae_fc1_b;    /* audio.decoder.fc1 [vae.hidden, latent] */
    mt_qwen_weights vae;
    const mt_bf16 *vae_head_w, *vae_head_b;  /* audio.decoder.head.out [nfft+2, vae.hidden] */
    const float* vae_window;                 /* audio.decoder.head.istft.window [nfft] */
    const mt_bf16* embed_tokens;             /* model.model.embed_tokens [vocab, llm.hidden] */
} mt_model_weights;

/* ---------------------------------------------------------------------------------------------
 * Context
 * ------------------------------------------------------------------------------------------- */

/* Binds to CUDA device `device` (makes it current on the calling thread) and allocates the
 * context's device status word. Replaces MetalContext (Sources/MingTTS/Engine/MetalContext.swift:28-111). */
mt_status mt_ctx_create(int device, mt_ctx** out);
void mt_ctx_destroy(mt_ctx* ctx);
/* Message of the last failing call on ctx ("" if none). Valid until the next call on ctx. */
const char* mt_last_error(const mt_ctx* ctx);
/* Library version string, e.g. "mingcuda 0.1.0 sm_100a". */
const char* mt_version(void);
/* Synchronises `stream`, then reads and clears the device status word that bounded waits set.
 * Returns MT_ERR_TIMEOUT if a kernel gave up a wait, MT_ERR_CUDA on a CUDA error.
 * Replaces the command-buffer error check of StepRecorder.finish (Engine.swift:70-85). */
mt_status mt_ctx_check(mt_ctx* ctx, void* stream);
/* Wall-time limit of every bounded device wait of kernels launched with ctx (mbarrier waits on
 * asynchronous copies and tensor-core commits): `microseconds`, or 0 for the default of 2 s. A wait
 * that runs out records MT_ERR_TIMEOUT for mt_ctx_check and ends its kernel early (its outputs are
 * then incomplete). Synchronous; applies to kernels launched after it returns. No counterpart in the
 * reference, whose command-buffer errors surface at StepRecorder.finish (Engine.swift:70-85). */
mt_status mt_ctx_set_wait_limit(mt_ctx* ctx, unsigned int microseconds);
/* Failure-detection check: enqueues a one-thread kernel whose bounded wait nothing completes (a
 * shared-memory barrier that no one arrives on, no copy in flight). It gives up after the wait limit
 * and records a timeout, so the next mt_ctx_check returns MT_ERR_TIMEOUT and clears it; the context
 * then works as before. No counterpart in the reference. */
mt_status mt_ctx_wait_probe(mt_ctx* ctx, void* stream);
/* Small-batch stacks (at most 8 activation rows: mt_qwen_decode, and the engine's decode passes
 * at few requests made on ctx from now on): 1 runs every layer of a pass in one launch of
 * the persistent stack kernel where the shapes fit it, 0 (default) launches one kernel per operation
 * as the reference dispatches them, 2 requires the persistent kernel (mt_qwen_decode then returns
 * MT_ERR_SHAPE for a pass it cannot take). Results agree to rounding; the choice only changes
 * speed. No counterpart in the reference. */
mt_status mt_ctx_set_persistent(mt_ctx* ctx, int mode);
/* Tensor-core GEMM tiling for plans made on ctx from now on: -1 automatic (default), 0 single-CTA
 * tiles of 128 weight rows, 1 CTA pairs (clusters of two SMs sharing 256-weight-row tiles through
 * tcgen05 cta_group::2). Results agree to rounding; the choice only changes speed. No counterpart
 * in the reference (its GEMM has one tiling). */
mt_status mt_ctx_set_gemm_pairs(mt_ctx* ctx, int mode);

/* Which kernel family mt_linear routes a shape to: 0 = CUDA-core GEMV (rows in registers),
 * 1 = tcgen05 tensor-core GEMM. Mirrors Kernels.usesGemm (Kernels.swift:81-86). */
int mt_linear_route(int m, int n, int k);

/* ---------------------------------------------------------------------------------------------
 * Operators (one per Encoder method, Kernels.swift:89-283)
 *
 * Every kernel is launched with programmatic dependent launch: it may start while the previous
 * kernel on the stream drains, and waits for that kernel before it reads activations or writes
 * outputs. mt_linear reads its weights (w, w2) before that wait on every route, so the weights must
 * not be written by the kernel directly before it on the same stream if that kernel triggers
 * programmatic completion early (kernels of other libraries normally do not; model creation in
 * this library synchronises).
 * ------------------------------------------------------------------------------------------- */

/* y[m, n] = epi(x[m, :k] . w[n, :k]^T), x row stride ldx floats, y row stride ldy floats.
 * w2 is the up projection for MT_LINEAR_SILU_GATE (else ignored, may be NULL); bias is read only
 * with MT_LINEAR_BIAS. Rows of x past m are never read.
 * Replaces Encoder.linear (Kernels.swift:132-161) and the gemv/gemm8/gemm kernels
 * (Shaders.swift:47-108, 191-277, 304-408). Requires k % 8 == 0, 16-byte aligned x/w/w2 rows. */
mt_status mt_linear(mt_ctx* ctx, void* stream, const float* x, int ldx, int m,
                    const mt_bf16* w, const mt_bf16* w2, const mt_bf16* bias, int n, int k,
                    float* y, int ldy, uint32_t flags);

/* The tensor-core form of mt_linear with the activations already split into bf16 planes,
 * x ~= x_hi + x_lo (row stride ld_x elements): the form the engine's producers write. Outputs: fp32 y
 * (row stride ldy) and/or bf16 hi/lo planes (row stride ld_ysplit; NULL to skip). Same flags and
 * epilogue as mt_linear; any m >= 1, k % 8 == 0. Replaces the tiled GEMM (Shaders.swift:304-408). */
mt_status mt_linear_split(mt_ctx* ctx, void* stream, const mt_bf16* x_hi, const mt_bf16* x_lo, int ld_x, int m,
                          const mt_bf16* w, const mt_bf16* w2, const mt_bf16* bias, int n, int k, float* y, int ldy,
                          mt_bf16* y_hi, mt_bf16* y_lo, int ld_ysplit, uint32_t flags);

/* mt_linear_static computes what mt_linear computes, always on the tensor-core route, for callers that
 * cannot allocate device memory: a host framework that owns every device allocation through its own
 * pool, or a real-time audio thread that must not block on an allocation. It takes no context and
 * allocates nothing: the scratch for splitting x into bf16 hi/lo planes is a 4 MiB array compiled
 * into the library, held on every GPU that loads the library until the process exits. Nothing in it
 * needs to start at zero (each call writes the planes it then reads). Limit: m * k <= 1,048,576
 * (larger calls return MT_ERR_CAPACITY). The first call on a device looks up the array's device
 * address with that device current; make that first call before any stream capture. Every call on
 * a device uses the same array, so calls that can overlap on the GPU (streams not ordered with each
 * other) race and corrupt each other's results: order them. Argument and launch errors are reported
 * by the returned status only (there is no context for a message); a bounded device wait that gives
 * up while the call runs on the GPU is recorded in a status word of the library's own on that device
 * and reported by mt_linear_static_status. Has no counterpart in the reference. */
mt_status mt_linear_static(void* stream, const float* x, int ldx, int m, const mt_bf16* w, const mt_bf16* w2,
                           const mt_bf16* bias, int n, int k, float* y, int ldy, uint32_t flags);
/* Synchronises `stream`, then reads and clears the device-side status of mt_linear_static on the
 * current device: MT_ERR_TIMEOUT if one of its kernels gave up a bounded wait since the last query
 * (that call's y is incomplete), MT_OK otherwise, MT_ERR_CUDA on a CUDA error. Allocates nothing. */
mt_status mt_linear_static_status(void* stream);

/* y = x * rsqrt(mean(x^2) + eps) * w per row. Replaces Encoder.rmsnorm (Kernels.swift:163-171),
 * kernel rmsnorm (Shaders.swift:418-441). width % 4 == 0. */
mt_status mt_rmsnorm(mt_ctx* ctx, void* stream, const float* x, int ldx, int rows, int width,
                     const mt_bf16* w, float* y, int ldy, float eps);

/* y[i] = x[i], i < count. Replaces Encoder.copy (Kernels.swift:173-178), copy_rows (Shaders.swift:443-447). */
mt_status mt_copy(mt_ctx* ctx, void* stream, const float* x, int count, float* y);

/* NeoX RoPE (pairs i, i+32) on the q heads of qkv in place; rotated k and raw v appended to the
 * fp32 caches [hkv, capacity, 64] at positions pos0..pos0+m-1 (slot = position % capacity).
 * Replaces Encoder.ropeCache (Kernels.swift:182-191), rope_cache (Shaders.swift:456-486). */
mt_status mt_rope_cache(mt_ctx* ctx, void* stream, float* qkv, int ldq, int m, int hq, int hkv,
                        int pos0, float* k_cache, float* v_cache, int capacity, const float* inv_freq);

/* Causal GQA attention of the m query rows at positions pos0.. over the cache, scale 1/8,
 * window = 0 for full causal else keys (pos - window, pos]. out[m, hq*64] row stride ldo.
 * Replaces Encoder.attention (Kernels.swift:195-206), attention_cache (Shaders.swift:500-591). */
mt_status mt_attention(mt_ctx* ctx, void* stream, const float* q, int ldq, int m, int hq, int hkv,
                       int pos0, int window, const float* k_cache, const float* v_cache,
                       int capacity, float* out, int ldo);

/* mt_rope_cache followed by mt_attention in one kernel, for decode steps of m <= 4 rows of one
 * request (the LLM token, the VAE decode's four frames): rotates the q heads and k, appends k and v
 * at positions pos0..pos0+m-1 (slot = position % capacity; the cache may be a ring when window > 0
 * and window + m - 1 <= capacity), attends as mt_attention does, and writes out[m, hq*64]. qkv is
 * not modified. chunk_keys (0 = automatic) bounds the keys staged in shared memory at once.
 * Replaces Encoder.ropeCache + Encoder.attention (Kernels.swift:182-206) on the decode path. */
mt_status mt_rope_attention(mt_ctx* ctx, void* stream, const float* qkv, int ldq, int m, int hq, int hkv, int pos0,
                            int window, float* k_cache, float* v_cache, int capacity, const float* inv_freq,
                            float* out, int ldo, int chunk_keys);

/* One decode pass of a Qwen stack (QwenForward.dispatches, Qwen.swift:72-97) for `requests`
 * independent sequences of `rows` new rows each (rows <= 4, requests * rows <= 8): the reference's LLM
 * decode token (one row, Engine.swift:381-385) and VAE frame decode (four rows, VAEDecoder.swift:86-107).
 * x [requests * rows, hidden] fp32: the new rows' residual stream (the input embeddings), updated in
 * place to the stream after the last layer; z [requests * rows, hidden]: the final norm of every row
 * (normRows = rows). Request r's cache starts at kv + r * kv_stride floats, laid out
 * [layers][K|V][kv_heads][capacity][64] fp32 (KVCache, Qwen.swift:7-26), slot = position % capacity;
 * positions (device int32 [requests]) = tokens already cached per request; the new rows take
 * positions[r] .. positions[r] + rows - 1 and are appended. With w->cfg.window == 0 the caller keeps
 * positions[r] + rows <= capacity; with a window the cache may be a ring (window + rows - 1 <= capacity).
 * Replaces the decode use of QwenForward.dispatches; scratch comes from the context (the first call
 * with a given shape and rope theta sets it up synchronously, so make it before any stream capture).
 * On the persistent path (mt_ctx_set_persistent) the context also keeps a zeroed stack area, grown
 * (after a device synchronisation) when a larger pass needs it; persistent calls on one context must
 * not overlap on the GPU (each takes every SM). */
mt_status mt_qwen_decode(mt_ctx* ctx, void* stream, const mt_qwen_weights* w, int requests, int rows, float* x,
                         float* kv, long long kv_stride, int capacity, const int32_t* positions, float* z);

/* Full attention over `batch` sequences of `seq` <= 8 rows with interleaved RoPE (pairs 2l, 2l+1,
 * angle = row * inv_freq[l]). qkv rows are [q | k | v] of heads*64 each, row stride ld.
 * Replaces Encoder.ditAttention (Kernels.swift:210-220), dit_attention (Shaders.swift:613-648). */
mt_status mt_dit_attention(mt_ctx* ctx, void* stream, const float* qkv, int ld, int batch, int seq,
                           int heads, const float* inv_freq, float* out, int ldo);

/* The 6 flow DiT input rows: r%3==0 -> temb + (r<3 ? cemb : cond_bias), r%3==1 -> x_emb(history),
 * r%3==2 -> x_emb(y), x_emb(v) = x_w . v + x_b. x is [6, hidden] dense.
 * Replaces Encoder.flowAssemble (Kernels.swift:222-235), flow_assemble (Shaders.swift:654-677). */
mt_status mt_flow_assemble(mt_ctx* ctx, void* stream, const float* y, const float* history,
                           const float* cemb, const mt_bf16* cond_bias, const float* temb,
                           const mt_bf16* x_w, const mt_bf16* x_b, int hidden, int latent_dim,
                           float* x);

/* y += (c + (c - u) * cfg) * dt with c = pred[pred_row], u = pred[null_row]; capture = [c, u].
 * Replaces Encoder.flowEuler (Kernels.swift:237-245), flow_euler (Shaders.swift:682-693). */
mt_status mt_flow_euler(mt_ctx* ctx, void* stream, float* y, const float* pred, int ldp,
                        int pred_row, int null_row, int latent_dim, float cfg, float dt,
                        float* capture);

/* Four frames [4, hidden] of linear x4 upsampling (align_corners=False) from h[n-1], h[n], h[n+1];
 * prev/next may be NULL (clamped to cur). Replaces Encoder.upsample4 (Kernels.swift:247-257),
 * upsample4 (Shaders.swift:704-719). */
mt_status mt_upsample4(mt_ctx* ctx, void* stream, const float* prev, const float* cur,
                       const float* next, int hidden, float* frames);

/* `count` windowed ISTFT frames from spectrum rows [logmag (nfft/2+1) | phase (nfft/2+1)] into
 * ring slots (frame0 + f) % ring of `frames` [ring, nfft]. cos_table is unused by this
 * implementation (kept for signature parity, may be NULL). nfft % 4 == 0.
 * Replaces Encoder.istftFrames (Kernels.swift:260-269), istft_frames (Shaders.swift:726-764). */
mt_status mt_istft_frames(mt_ctx* ctx, void* stream, const float* spec, int ld_spec, int count,
                          int nfft, const float* cos_table, const float* window, float* frames,
                          int frame0, int ring);

/* Overlap-add of stream samples s0..s0+count from the ring, divided by the window^2 envelope,
 * pad = (nfft - hop) / 2. Replaces Encoder.istftEmit (Kernels.swift:272-281), istft_emit
 * (Shaders.swift:770-788). count == 0 is a no-op. */
mt_status mt_istft_emit(mt_ctx* ctx, void* stream, const float* frames, const float* window,
                        int nfft, int hop, int s0, int count, int last_frame, int ring, float* out);

/* ---------------------------------------------------------------------------------------------
 * Model: one device arena holding every weight, described by a tensor table
 * (replaces WeightArena + the *Weights structs, Sources/MingTTS/Engine/Weights.swift:8-263)
 * ------------------------------------------------------------------------------------------- */

enum { MT_DTYPE_BF16 = 0, MT_DTYPE_F32 = 1 };
enum { MT_INIT_NORMAL = 0, MT_INIT_ONES = 1, MT_INIT_INV_FREQ = 2, MT_INIT_HANN = 3 };

typedef struct {
    char name[96];     /* checkpoint tensor name; q/k/v are one tensor "...qkv_proj" / "...to_qkv" */
    size_t offset;     /* bytes from the arena base, 256-byte aligned */
    size_t numel;
    int dtype;         /* MT_DTYPE_* */
    int init;          /* MT_INIT_* used by mt_model_create_random */
    float std;         /* MT_INIT_NORMAL: standard deviation (0.02) */
    uint64_t seed;     /* MT_INIT_NORMAL: stream seed of mt_randn_bf16 */
} mt_tensor_info;

/* Ming-3.0-tts-0.5B dimensions (Weights.swift:81-95, 145-148, 174-225; Engine.swift:91-92). */
void mt_model_config_default(mt_model_config* cfg);
/* Fills up to `cap` entries of the tensor table (if out != NULL); returns the tensor count. */
int mt_model_tensors(const mt_model_config* cfg, uint64_t seed, int with_embeddings, mt_tensor_info* out, int cap);
size_t mt_model_arena_bytes(const mt_model_config* cfg, int with_embeddings);
/* Allocates the arena and fills it: bf16 N(0, 0.02) from per-tensor seeds, norm gains 1.0,
 * DiT rotary inv_freq 1/10000^(2i/64), periodic Hann ISTFT window. */
mt_status mt_model_create_random(mt_ctx* ctx, const mt_model_config* cfg, uint64_t seed, int with_embeddings,
                                 mt_model** out);
/* Wraps a caller-owned device arena laid out as mt_model_tensors describes (e.g. a loaded checkpoint). */
mt_status mt_model_create_from_arena(mt_ctx* ctx, const mt_model_config* cfg, void* device_arena,
                                     int with_embeddings, mt_model** out);
/* ---------------------------------------------------------------------------------------------
 * Checkpoint: a safetensors file (replaces SafeTensors.swift:7-87, WeightArena.tensor/linear
 * Weights.swift:32-62 and the tensor names of the *Weights initialisers, Weights.swift:116-263).
 * Every table tensor is found by its checkpoint name: bf16 tensors are copied as stored, the q/k/v
 * projections (weights and biases) concatenated along their first axis into the table's
 * "...qkv_proj" / "...to_qkv" tensor, fp32 table entries (rotary inv_freq, ISTFT window, the
 * aggregator cls row) decoded from BF16 or F32. Failures return MT_ERR_CHECKPOINT with the
 * reference's messages ("bad checkpoint: ...", "missing tensor NAME").
 * ------------------------------------------------------------------------------------------- */
/* Fills a host buffer of arena_bytes (>= mt_model_arena_bytes) laid out as mt_model_tensors
 * describes; padding bytes are zero. Host-only: needs no context and no GPU. The message of a
 * failure goes to err (err_len bytes, may be NULL). */
mt_status mt_checkpoint_fill_arena(const char* path, const mt_model_config* cfg, int with_embeddings,
                                   void* host_arena, size_t arena_bytes, char* err, size_t err_len);
/* Loads the checkpoint into a new model whose device arena the model owns. */
mt_status mt_model_load_safetensors(mt_ctx* ctx, const mt_model_config* cfg, const char* path,
                                    int with_embeddings, mt_model** out);
const mt_model_weights* mt_model_get_weights(const mt_model* model);
const mt_model_config* mt_model_get_config(const mt_model* model);
mt_status mt_model_arena(const mt_model* model, void** ptr, size_t* bytes);
void mt_model_destroy(mt_model* model);

/* ---------------------------------------------------------------------------------------------
 * Engine: the generation loop for R concurrent requests on one GPU
 * (MingEngine.generate / encodeStep, Engine.swift:302-415; VAEDecoder, VAEDecoder.swift:64-107)
 * ------------------------------------------------------------------------------------------- */

typedef struct {
    int max_requests;  /* R capacity */
    int max_prompt;    /* prompt rows per request (all requests of a generation share it) */
    int max_steps;     /* generation steps; prompt + steps <= llm_capacity */
    int vae_ring;      /* VAE KV-cache ring positions (0 = 128); must be >= window + 3 */
    int use_graphs;    /* 1: replay steady-state steps from a captured CUDA graph */
    int groups;        /* request groups stepped concurrently on their own streams (0 = 1; at most
                          4 and at most the requests); one group measured fastest on B200 */
} mt_engine_options;

/* Buffers readable after a step (device pointers, request-major). */
enum {
    MT_BUF_Z = 0,          /* [R, llm.hidden]    LLM final-norm output of the last step */
    MT_BUF_STOP_LOGITS,    /* [R, 2]             stop-head logits of the last step */
    MT_BUF_LATENTS,        /* [R, max_steps, latent] every latent so far */
    MT_BUF_AGG_OUT,        /* [R, llm.hidden]    aggregator output = next LLM input */
    MT_BUF_VELOCITY0,      /* [R, flow_steps, 2, latent] step-0 cond/uncond DiT outputs */
    MT_BUF_VAE_HIDDEN,     /* [R, 4, vae.hidden] decoder final-norm rows of the last decoded latent */
    MT_BUF_PCM             /* [R, max_chunk]     samples of the last emission */
};

mt_status mt_engine_create(mt_ctx* ctx, const mt_model* model, const mt_engine_options* opt, mt_engine** out);
void mt_engine_destroy(mt_engine* engine);
/* Starts a generation of `requests` requests with `prompt_rows` prompt rows each. Inputs: embeds
 * [R, T, llm.hidden] fp32, or token_ids [R, T] (int32, gathered from embed_tokens) when embeds is
 * NULL; noise [R, steps, latent]; initial_history [R, latent] or NULL (zeros). token_ids must be in
 * device memory; embeds, noise and initial_history may be in host or device memory (copied on the
 * stream; pageable host memory makes the copy synchronous).
 * Resets the KV caches and VAE counters (Engine.swift:312-317). */
mt_status mt_engine_begin(mt_engine* engine, void* stream, int requests, int prompt_rows, const float* embeds,
                          const int32_t* token_ids, const float* noise, const float* initial_history, int steps,
                          float cfg);
/* Prompt prefill (Engine.swift:323-333). */
mt_status mt_engine_prefill(mt_engine* engine, void* stream);
/* Enqueues generation step n (the next one): LLM token (n > 0), stop head, flow head, aggregator,
 * VAE fc1, and the VAE frames of latent n-2 on a second stream. *pcm_count = samples per request
 * this step emits into MT_BUF_PCM (0 before step 2). Returns after enqueueing (no host sync). */
mt_status mt_engine_step(mt_engine* engine, void* stream, int* pcm_count);
/* After the last step: decodes one remaining latent per call (Engine.swift:360-367);
 * *pcm_count = 0 once everything is decoded. */
mt_status mt_engine_flush(mt_engine* engine, void* stream, int* pcm_count);
mt_status mt_engine_buffer(const mt_engine* engine, int which, const float** ptr, long long* request_stride);
/* Steps enqueued so far in this generation. */
int mt_engine_steps_done(const mt_engine* engine);
/* Kernels the last mt_engine_step enqueued (all streams). */
int mt_engine_step_kernels(const mt_engine* engine);
/* Per-stage GPU timing, as the reference's split StepRecorder (Engine.swift:31-86): when on, steps
 * with both an LLM token and a VAE decode run eagerly (no graph replay) with events around each
 * stage, and mt_engine_stage_ms returns [llm, flow, agg, vae] milliseconds of the last such step
 * (the VAE decode runs concurrently on its own stream). */
mt_status mt_engine_set_stage_timing(mt_engine* engine, int on);
mt_status mt_engine_stage_ms(mt_engine* engine, float* ms4);
/* The reference's stop rule for mt_engine_generate / mt_engine_generate_stream (MingEngine.generate,
 * Engine.swift:347-355): when on, the host reads step n's stop logits before enqueuing step n + 1,
 * a request meets the rule at its first step with p = 1/(1+exp(l0-l1)) > 0.5 and n > 3, and the
 * generation ends after the step at which every request has met it, then flushes. For one request
 * this is the reference's loop exactly; in a batch, requests that met the rule earlier keep
 * generating until the last one does (their first such step is visible in stop_prob_host).
 * mt_engine_steps_done gives the steps run. Off by default (the serving benchmark runs a fixed
 * number of steps); the per-step host read costs one stream synchronisation per step. */
mt_status mt_engine_set_stop_rule(mt_engine* engine, int on);
/* End to end from host memory: copies embeds (or ids) and noise in, runs prefill, `steps` steps
 * and the flush, and copies every PCM chunk and stop probability out. pcm_host is [R, pcm_stride];
 * pcm_count receives the samples written per request (the same for all). The stop head is
 * evaluated every step; generation runs all `steps` unless mt_engine_set_stop_rule turned the
 * stop rule on (then stop_prob_host is 0 past the steps run). Uses staging the engine allocated at
 * creation (no allocation per call); returns when the last sample is in pcm_host. */
mt_status mt_engine_generate(mt_engine* engine, void* stream, int requests, int prompt_rows, const float* embeds_host,
                             const int32_t* ids_host, const float* noise_host, int steps, float cfg, float* pcm_host,
                             long long pcm_stride, long long* pcm_count, float* stop_prob_host);
/* Streaming delivery (replaces MingTTSModel.stream / synthesize(onChunk:), MingTTS.swift:46-61):
 * the same generation as mt_engine_generate, but each PCM chunk is handed to on_chunk on the calling
 * thread as soon as its copy has reached pinned host memory, in order: chunk index, requests, count
 * samples per request, pcm[r * request_stride + j]. The pointer is valid only during the call.
 * A non-zero return cancels: nothing further is enqueued and the call returns MT_ERR_STATE (the
 * reference's Task cancellation ends the stream with an error the same way). pcm_count receives the
 * samples delivered per request; stop_prob_host may be NULL. */
typedef int (*mt_pcm_chunk_fn)(void* user, int chunk, int requests, int count, const float* pcm,
                               long long request_stride);
mt_status mt_engine_generate_stream(mt_engine* engine, void* stream, int requests, int prompt_rows,
                                    const float* embeds_host, const int32_t* ids_host, const float* noise_host,
                                    int steps, float cfg, mt_pcm_chunk_fn on_chunk, void* user,
                                    long long* pcm_count, float* stop_prob_host);
/* Mono IEEE-float WAV file (RIFF, 16-byte fmt chunk, format 3, 32 bits), as writeWav
 * (main.swift:134-144). Host only. MT_ERR_ARG if the file cannot be written. */
mt_status mt_write_wav_f32(const char* path, const float* samples, long long count, int sample_rate);

/* ---------------------------------------------------------------------------------------------
 * Clone path: the audio VAE encoder (VAEEncoder.swift:56-107) and the aggregator over reference
 * latents (MingEngine.aggregate, Engine.swift:236-256). Not on the per-step path; built from the
 * operator entry points above with per-call device buffers.
 * ------------------------------------------------------------------------------------------- */
typedef struct mt_encoder mt_encoder;

/* VAEEncoderWeights (Weights.swift:229-262). The encoder stack has the VAE decoder's dimensions
 * (window 65); the patch aggregator the same with 4 layers. */
typedef struct {
    int frame;           /* samples per frame = hop (882) */
    int padded_frame;    /* frame rounded up to 64 columns (896): fc1's stored K */
    int patch;           /* frames per latent (4) */
    int max_frames;      /* longest clip mt_vae_encode takes (1600 frames = 32 s) */
    const mt_bf16* fc1_w;               /* [hidden, padded_frame], zero past frame; no bias */
    const mt_bf16 *fc2_w, *fc2_b;       /* [hidden, hidden] */
    mt_qwen_weights stack;              /* audio.encoder.encoder */
    mt_qwen_weights aggregator;         /* audio.encoder.aggregator */
    const float* cls;                   /* audio.encoder.cls_embed [hidden] */
    const mt_bf16 *fc3_w, *fc3_b;       /* posterior head [2 * latent_dim, hidden] */
} mt_encoder_weights;

int mt_encoder_tensors(const mt_model_config* cfg, uint64_t seed, mt_tensor_info* out, int cap);
size_t mt_encoder_arena_bytes(const mt_model_config* cfg);
/* bf16 N(0, 0.02) weights (fc1 zero past frame), norm gains 1.0, fp32 cls N(0, 0.02). */
mt_status mt_encoder_create_random(mt_ctx* ctx, const mt_model_config* cfg, uint64_t seed, mt_encoder** out);
mt_status mt_encoder_create_from_arena(mt_ctx* ctx, const mt_model_config* cfg, void* device_arena,
                                       mt_encoder** out);
/* The encoder tensors of a safetensors checkpoint ("audio.encoder.*", fc1 stored [hidden, frame]
 * and padded with zero columns as WeightArena.paddedLinear does, Weights.swift:64-77). */
mt_status mt_checkpoint_fill_encoder_arena(const char* path, const mt_model_config* cfg, void* host_arena,
                                           size_t arena_bytes, char* err, size_t err_len);
mt_status mt_encoder_load_safetensors(mt_ctx* ctx, const mt_model_config* cfg, const char* path,
                                      mt_encoder** out);
const mt_encoder_weights* mt_encoder_get_weights(const mt_encoder* enc);
mt_status mt_encoder_arena(const mt_encoder* enc, void** ptr, size_t* bytes);
void mt_encoder_destroy(mt_encoder* enc);

/* VAEEncoder.encode: count samples (host, a non-zero multiple of frame * patch, at most max_frames
 * frames) rounded to bf16, then fc1 -> fc2 -> encoder stack -> [4 frame rows | cls] per latent ->
 * aggregator -> fc3 on the cls rows; mean_host and std_host receive [count / (frame * patch),
 * latent_dim]: mean, and softplus(scale) + 1e-4. Synchronises `stream`. */
mt_status mt_vae_encode(mt_encoder* enc, void* stream, const float* samples_host, long long count,
                        float* mean_host, float* std_host);
/* MingEngine.aggregate: the aggregator DiT over count reference latents at once (batch count,
 * sequence [cls, x_embedder(latent)]), row 0 of each sequence; latents_host [count, latent_dim]
 * -> rows_host [count, llm.hidden] (the reference voice's LLM input rows). count <=
 * llm_capacity. Synchronises `stream`. */
mt_status mt_aggregate_latents(mt_ctx* ctx, const mt_model* model, void* stream, const float* latents_host,
                               int count, float* rows_host);

/* ---------------------------------------------------------------------------------------------
 * Synthetic data (seeded random-init weights and noise)
 * ------------------------------------------------------------------------------------------- */

/* Standard normal samples from a SplitMix64 stream with Box-Muller in double, as
 * MingEngine.gaussianNoise (Engine.swift:433-453): out[i] = N(0,1) as fp32. Host. */
void mt_gaussian_noise_host(float* out, size_t count, uint64_t seed);
/* std * N(0,1) from the same stream, rounded to bf16 (round-to-nearest-even). Host (OpenMP)
 * and device versions produce identical bits. */
void mt_randn_bf16_host(mt_bf16* out, size_t count, uint64_t seed, float std);
mt_status mt_randn_bf16(mt_ctx* ctx, void* stream, mt_bf16* out, size_t count, uint64_t seed,
                        float std);

/* ---------------------------------------------------------------------------------------------
 * 1-D convolutional waveform decoder (latents -> 44.1 kHz mono)
 *
 * No counterpart in the reference: its VAE decoder is the windowed Qwen stack + ISTFT above
 * (VAEDecoder.swift:1-108). This is the convolution stack that BASELINE config 4 describes,
 * defined here (parity is against this library's own fp64 host restatement, not the reference):
 *   x   = conv_in(latents)                                  kernel k, latent_dim -> C0
 *   for stage i = 0..3 (stride s_i, C_i -> C_{i+1}):
 *     u = conv_transpose(silu(x))                           kernel 2 s_i, stride s_i, padding s_i / 2
 *     x = u + conv_b(silu(conv_a(silu(u))))                 kernels k, C_{i+1} -> C_{i+1}
 *   pcm = tanh(conv_out(silu(x)))                           kernel k, C_4 -> 1
 * Convolutions pad (k - 1) / 2 zeros at both ends (lengths are kept); every layer has a bias.
 * Layouts follow PyTorch: Conv1d weight [out][in][k], ConvTranspose1d weight [in][out][2 s].
 * Each convolution runs as an implicit GEMM on the tcgen05 tensor cores (time rows x output
 * channels, K = taps x input channels), the transposed ones as one polyphase GEMM each.
 * ------------------------------------------------------------------------------------------- */
typedef struct mt_convdec_config {
    int latent_dim;   /* 64 (a multiple of 64) */
    int channels[5];  /* C0..C4: 512, 256, 128, 64, 64 (multiples of 64) */
    int strides[4];   /* 8, 8, 4, 8 (even) */
    int kernel;       /* 7 (odd, <= 7) */
} mt_convdec_config;

/* Device bf16 weights in PyTorch layouts (see above). */
typedef struct mt_convdec_weights {
    const mt_bf16 *in_w, *in_b;          /* [C0][latent_dim][k], [C0] */
    const mt_bf16 *up_w[4], *up_b[4];    /* [C_i][C_{i+1}][2 s_i], [C_{i+1}] */
    const mt_bf16 *a_w[4], *a_b[4];      /* [C_{i+1}][C_{i+1}][k], [C_{i+1}] */
    const mt_bf16 *b_w[4], *b_b[4];      /* [C_{i+1}][C_{i+1}][k], [C_{i+1}] */
    const mt_bf16 *out_w, *out_b;        /* [1][C4][k], [1] */
} mt_convdec_weights;

typedef struct mt_convdec mt_convdec;

/* Samples out of `frames` latent frames: frames x s_0 x s_1 x s_2 x s_3. */
long long mt_convdec_samples(const mt_convdec_config* cfg, int frames);
/* Repacks the weights into GEMM layouts (the caller's buffers may be freed afterwards) and
 * allocates the activation buffers for up to max_frames frames (zero halo rows included).
 * Synchronous. */
mt_status mt_convdec_create(mt_ctx* ctx, const mt_convdec_config* cfg, const mt_convdec_weights* w, int max_frames,
                            mt_convdec** out);
/* latents: device fp32 [frames][latent_dim]; pcm: device fp32 [mt_convdec_samples(frames)].
 * Enqueued on `stream`; tensor maps are encoded on the host when `frames` differs from the
 * previous call. */
mt_status mt_convdec_decode(mt_convdec* dec, void* stream, const float* latents, int frames, float* pcm);
void mt_convdec_destroy(mt_convdec* dec);

#ifdef __cplusplus
}
#endif
#endif /* MINGCUDA_H */
