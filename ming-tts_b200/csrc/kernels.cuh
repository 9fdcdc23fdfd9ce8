// kernels.cuh -- argument blocks and launchers of the device kernels (internal to libmingcuda.so).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace mt {

struct RmsArgs {
    const float* x; int ldx; int rows; int width;
    const uint16_t* w;
    float* y; int ldy;                 // optional fp32 output
    uint16_t* y_hi; uint16_t* y_lo;    // optional bf16 hi/lo planes
    int ld_split;
    float eps;
};
void launch_rmsnorm(const RmsArgs& a, cudaStream_t s);
void launch_split(const float* x, int ldx, int rows, int cols, uint16_t* hi, uint16_t* lo, int ld_split,
                  int sm_count, cudaStream_t s);

// Rows are grouped by request: row m belongs to request m / rows_per_req and sits at position
// pos0 + pos_dev[request] (pos_dev optional) + m % rows_per_req. Request r's caches start at
// kc/vc + r * req_stride floats; cache slot = position % cap.
struct RopeArgs {
    float* qkv; int ldq; int rows; int rows_per_req; int hq; int hkv;
    int pos0; const int* pos_dev;
    float* kc; float* vc; long long req_stride; int cap;
    const float* inv_freq;
};
void launch_rope_cache(const RopeArgs& a, cudaStream_t s);

struct AttnArgs {
    const float* q; int ldq; int rows; int rows_per_req; int hq; int hkv;
    int pos0; const int* pos_dev; int window;
    const float* kc; const float* vc; long long req_stride; int cap;
    float* out; int ldo;                      // optional fp32 output
    uint16_t* out_hi; uint16_t* out_lo; int ld_split;  // optional bf16 hi/lo output
    int max_keys;                             // upper bound of keys any row attends to
};
size_t attention_smem(int G, int max_keys);
void launch_attention(const AttnArgs& a, cudaStream_t s);

// Decode attention with RoPE and the KV append fused in, for steps where every row of a request
// is in one block (rows_per_req <= 4: the LLM token, the VAE decode): block (request, kv head)
// rotates its rows' q heads and the new k, appends k and v to the cache, and attends over the
// request's cached keys (bulk-copied into shared memory) plus the new ones.
struct AttnDecodeArgs {
    const float* qkv; int ldq; int requests; int rows_per_req; int hq; int hkv;
    int pos0; const int* pos_dev; int window;
    float* kc; float* vc; long long req_stride; int cap;
    const float* inv_freq;                    // [32] NeoX rotation frequencies
    float* out; int ldo;                      // optional fp32 output
    uint16_t* out_hi; uint16_t* out_lo; int ld_split;  // optional bf16 hi/lo output
    int max_keys;                             // keys any row attends to, at most (cache capacity if unbounded)
    int chunk_keys;                           // keys staged per chunk (0: as many as shared memory holds)
    unsigned int* status;                     // bounded-wait failures
};
constexpr int ATTN_DECODE_MAX_ROWS = 4;
bool attention_decode_supported(int rows_per_req, int hq, int hkv);
void launch_attention_decode(const AttnDecodeArgs& a, cudaStream_t s);

struct DitAttnArgs {
    const float* qkv; int ld; int batch; int seq; int heads;
    const float* inv_freq;
    float* out; int ldo;
    uint16_t* out_hi; uint16_t* out_lo; int ld_split;
};
void launch_dit_attention(const DitAttnArgs& a, cudaStream_t s);

// ISTFT frames: spectrum row f belongs to request f / frames_per_req and lands in that request's
// ring (frames + request * req_stride) at slot (frame0 + frame0_dev[request] + f % frames_per_req) % ring.
struct IstftArgs {
    const float* spec; int ld_spec; int count; int nfft;
    const float* window;
    float* frames; long long req_stride; int frames_per_req;
    int frame0; const int* frame0_dev; int ring;
};
size_t istft_frames_smem(int nfft);
void launch_istft_frames(const IstftArgs& a, cudaStream_t s);

// Emission: request r (grid y) writes count (or count_dev[r]) samples of its stream starting at
// s0 (+ s0_dev[r]) to out + r * ld_out, from its ring frames + r * req_stride.
struct EmitArgs {
    const float* frames; long long req_stride;
    const float* window; int nfft; int hop;
    int s0; const int* s0_dev; int count; const int* count_dev;
    int last_frame; const int* last_dev; int ring;
    float* out; long long ld_out;
};
void launch_istft_emit(const EmitArgs& a, int max_count, int requests, cudaStream_t s);

// Linear Y[m, n] = epi(X[m, :k] . W[n, :k]^T) -- see linear.cu / gemm_tc.cu.
struct LinearArgs {
    const float* x; int ldx;                   // fp32 activations (GEMV route)
    const uint16_t* x_hi; const uint16_t* x_lo; int ld_split;  // bf16 planes (tensor-core route)
    int m, n, k;
    const uint16_t* w; const uint16_t* w2; const uint16_t* bias;
    float* y; int ldy;                         // fp32 output (optional on the tensor-core route)
    uint16_t* y_hi; uint16_t* y_lo; int ld_ysplit;  // bf16 hi/lo output planes (optional)
    uint32_t flags;
    int split_k;                               // tensor-core route: K splits (1 = none, 0 = automatic)
    int bn_override;                           // tensor-core route: activation rows per tile (0 = auto)
    float* ws;                                 // tensor-core route: fp32 [m, 2n] workspace for split-K
                                               //   with a nonlinear epilogue (optional)
    // Tensor-core route, implicit-GEMM convolution over time-major rows (0 = a plain GEMM): K is
    // taps x conv_cin; with q = tap + conv_row0, K column tap * conv_cin + c of GEMM row m reads plane
    // row m + q / conv_group, column (q % conv_group) * conv_cin + c (rows outside [0, x_rows) read
    // zeros). conv_group G > 1 views the activations as rows of G frames (ld_split >= G conv_cin).
    int conv_cin, conv_row0, x_rows, conv_group;
    int split_silu;                            // tensor-core route: the hi/lo output planes hold silu(y)
    // CUDA-core route: x is the raw residual stream and the linear reads RMSNorm(x) * norm_w
    // (Shaders.swift:418-441) -- the gain scales x as it loads, the 1/rms of each row the dot
    // product -- so no separate norm launch precedes it (NULL: x is used as is).
    const uint16_t* norm_w;
    float norm_eps;
};
void launch_gemv(const LinearArgs& a, cudaStream_t s);
mt_status launch_gemm_tc(mt_ctx* ctx, const LinearArgs& a, cudaStream_t s);

// Epilogue specialisations of the tensor-core GEMM: the flag combinations the engine runs are
// compiled as straight-line code; any other combination takes the runtime-flag path.
enum EpiKind : int {
    EPI_GENERIC = 0,
    EPI_F32 = 1,         // y = acc (+ bias)
    EPI_F32_ACCUM = 2,   // y += acc (+ bias)
    EPI_SPLIT = 3,       // hi/lo = split(acc (+ bias))
    EPI_SPLIT_GELU = 4,  // hi/lo = split(gelu(acc (+ bias)))
    EPI_SPLIT_GATE = 5,  // hi/lo = split(silu(acc1 (+ bias)) * acc2)
    EPI_F32_SILU = 6,    // y = silu(acc (+ bias))
    EPI_RED = 7,         // split-K partial: y += acc (+ bias on the first split), fp32 reductions
    EPI_F32_SSILU = 8,   // y = acc (+ bias); hi/lo = split(silu(y))          (convolution decoder)
    EPI_ACC_SSILU = 9,   // y += acc (+ bias); hi/lo = split(silu(y))
    EPI_SSILU = 10,      // hi/lo = split(silu(acc (+ bias)))
};

// Epilogue/launch parameters of the tensor-core GEMM (gemm_tc.cu).
struct TcEpi {
    int m, n, k;
    int bn;            // activation rows per tile (MMA N), multiple of 16, <= 256
    int stages;
    int kb_per_split;  // k blocks per blockIdx.z
    const uint16_t* bias;
    float* y; int ldy;
    uint16_t* y_hi; uint16_t* y_lo; int ld_ysplit;
    uint32_t flags;
    int split;         // K splits
    int tiles_m, tiles_n;  // activation-row tiles (bn rows) and weight-row tiles (128 rows)
    int mode;          // 0: epilogue in the kernel; 1: split-K reduced into y; 2: split-K sums into ws
    int kind;          // EPI_* epilogue specialisation chosen by the planner (EPI_GENERIC: runtime flags)
    int x_planes;      // 1: the x_hi map is 3-D and one copy loads both activation planes of a stage
    int ka;            // K atoms (64-wide K blocks) per pipeline stage, 1 or 2
    int conv_cin, conv_row0, conv_group;  // implicit-GEMM convolution (LinearArgs): conv_cin 0 = plain GEMM
    int split_silu;    // the hi/lo planes take silu of the output value
    float* ws; int ldws;
    unsigned int* status;
};

// A tensor-core GEMM with its tensor maps encoded once; run_gemm_plan only launches.
struct GemmPlan {
    CUtensorMap tw, tw2, th, tl;
    TcEpi e;
    dim3 grid;
    size_t smem;
    bool gated;
    bool pair;  // CTA-pair kernel (cluster of two, tcgen05 cta_group::2)
};
mt_status make_gemm_plan(mt_ctx* ctx, const LinearArgs& a, GemmPlan* plan);
mt_status make_gemm_plan_bare(int sm_count, const LinearArgs& a, GemmPlan* plan);
void run_gemm_plan(const GemmPlan& p, cudaStream_t s);

// Persistent small-batch stack (stack.cu): every layer of a Qwen decode pass, or every block of a
// DiT pass, in one cooperative launch over at most 8 activation rows.
constexpr int STACK_MAX_LAYERS = 32;
enum : int { STACK_QWEN = 0, STACK_DIT = 1 };
struct StackLayer { const uint16_t* p[10]; };  // Qwen: norm1 qkv_w qkv_b o_w norm2 gate_w up_w down_w;
                                                // DiT: norm1 qkv_w qkv_b out_w out_b norm2 ff1_w ff1_b ff2_w ff2_b
struct StackParams {
    int kind, layers;
    int M, seq_rows, seqs;           // M = seqs * seq_rows rows; Qwen: rows per request; DiT: sequence length
    int hidden, heads, kv_heads, inter;
    float eps;
    int window, cap;                 // Qwen KV cache: window (0 = causal), capacity (slot = position % cap)
    long long kv_stride;             // floats between requests' caches ([layers][K|V][kv][cap][64] each)
    const int* pos;                  // device [seqs]: cached positions per request (Qwen)
    float* kv;
    const float* inv_freq;           // [32]: NeoX frequencies (Qwen) or the DiT's rotary inv_freq
    float* x;                        // residual rows [M, hidden]: read at the start, written at the end
    float* z;                        // Qwen: final norm of every row [M, hidden] (NULL: none)
    const uint16_t* final_norm;
    // Stack area (stack_bind): sync words and the mailbox rows that carry activations between CTAs.
    unsigned int* sync;
    unsigned long long *mb_x, *mb_qkv, *mb_att, *mb_mlp;
    int chunks;                      // Qwen: attention chunks per unit, at most
    unsigned int* status;            // context status word (bounded waits)
    StackLayer L[STACK_MAX_LAYERS];
};
bool stack_supported(const StackParams& p, int ctas);
int stack_resident_blocks();  // blocks of the stack kernel one SM of the current device holds (>= 1 to launch)
const char* stack_resident_why();  // what kept it below one block, when it is
int stack_phases(const StackParams& p);
// Bytes of the stack area a pass needs (shape fields set). An area belongs to one launch sequence:
// it is zeroed once (stack_area_alloc) and every launch that uses it runs after the previous one on
// the GPU; passes of different shapes may share it.
size_t stack_area_bytes(const StackParams& p);
void stack_bind(StackParams& p, void* area);
mt_status stack_area_alloc(size_t bytes, void** out);
void launch_stack(const StackParams& p, int ctas, cudaStream_t s);

}  // namespace mt
