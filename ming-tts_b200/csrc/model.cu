// model.cu -- model description: default dimensions, the canonical tensor table, a device arena
// holding every weight (random-init or caller-provided) and the mt_model_weights pointer struct.
//
// Reference: the weight layout of Sources/MingTTS/Engine/Weights.swift -- WeightArena packs each
// module's bf16 tensors 256-byte aligned (:8-79); q/k/v rows (and their biases) are concatenated
// (:121-125, :158-159); QwenConfig / DiTWeights / FlowHeadWeights / AggregatorWeights /
// VAEDecoderWeights / LLMWeights give names and shapes (:81-263). Here every module lives in one
// arena, in the order of the table below, so a checkpoint loader can fill it by name.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

#include "common.cuh"

namespace mt {

namespace {

struct Builder {
    std::vector<mt_tensor_info> list;
    size_t cursor = 0;
    uint64_t seed;
    explicit Builder(uint64_t s) : seed(s) {}
    void add(const std::string& name, size_t numel, int dtype, int init, float std = 0.02f) {
        mt_tensor_info t{};
        snprintf(t.name, sizeof(t.name), "%s", name.c_str());
        t.offset = cursor;
        t.numel = numel;
        t.dtype = dtype;
        t.init = init;
        t.std = init == MT_INIT_NORMAL ? std : 0.0f;
        // Each tensor draws its own stream: seed * 1000003 + table index.
        t.seed = seed * 1000003ull + (uint64_t)list.size();
        const size_t bytes = numel * (dtype == MT_DTYPE_BF16 ? 2 : 4);
        cursor += (bytes + 255) & ~size_t(255);
        list.push_back(t);
    }
    void bf(const std::string& name, size_t numel) { add(name, numel, MT_DTYPE_BF16, MT_INIT_NORMAL); }
    void ones(const std::string& name, size_t numel) { add(name, numel, MT_DTYPE_BF16, MT_INIT_ONES); }
};

void add_qwen(Builder& b, const std::string& prefix, const mt_qwen_config& c) {
    const size_t h = c.hidden, qkv = (size_t)(c.heads + 2 * c.kv_heads) * 64, inter = c.intermediate;
    for (int l = 0; l < c.layers; l++) {
        const std::string p = prefix + ".layers." + std::to_string(l);
        b.ones(p + ".input_layernorm.weight", h);
        b.bf(p + ".self_attn.qkv_proj.weight", qkv * h);
        b.bf(p + ".self_attn.qkv_proj.bias", qkv);
        b.bf(p + ".self_attn.o_proj.weight", h * (size_t)c.heads * 64);
        b.ones(p + ".post_attention_layernorm.weight", h);
        b.bf(p + ".mlp.gate_proj.weight", inter * h);
        b.bf(p + ".mlp.up_proj.weight", inter * h);
        b.bf(p + ".mlp.down_proj.weight", h * inter);
    }
    b.ones(prefix + ".norm.weight", h);
}

void add_dit(Builder& b, const std::string& prefix, const mt_dit_config& c) {
    const size_t h = c.hidden, ff = c.ff;
    for (int i = 0; i < c.depth; i++) {
        const std::string p = prefix + ".blocks." + std::to_string(i);
        b.ones(p + ".norm1.weight", h);
        b.bf(p + ".attn.to_qkv.weight", 3 * h * h);
        b.bf(p + ".attn.to_qkv.bias", 3 * h);
        b.bf(p + ".attn.to_out.0.weight", h * h);
        b.bf(p + ".attn.to_out.0.bias", h);
        b.ones(p + ".norm2.weight", h);
        b.bf(p + ".mlp.ff.0.0.weight", ff * h);
        b.bf(p + ".mlp.ff.0.0.bias", ff);
        b.bf(p + ".mlp.ff.2.weight", h * ff);
        b.bf(p + ".mlp.ff.2.bias", h);
    }
    b.ones(prefix + ".final_layer.norm_final.weight", h);
    b.bf(prefix + ".final_layer.linear.weight", (size_t)c.out_dim * h);
    b.bf(prefix + ".final_layer.linear.bias", (size_t)c.out_dim);
    b.add(prefix + ".rotary_embed.inv_freq", 32, MT_DTYPE_F32, MT_INIT_INV_FREQ);
}

std::vector<mt_tensor_info> table(const mt_model_config& c, uint64_t seed, bool embeddings) {
    Builder b(seed);
    add_qwen(b, "model.model", c.llm);
    b.bf("stop_head.weight", 2 * (size_t)c.llm.hidden);
    b.bf("stop_head.bias", 2);
    const std::string f = "flowloss.cfm.model";
    b.bf(f + ".x_embedder.weight", (size_t)c.flow.hidden * c.latent_dim);
    b.bf(f + ".x_embedder.bias", c.flow.hidden);
    b.bf(f + ".c_embedder.cond_embedder.weight", (size_t)c.flow.hidden * c.llm.hidden);
    b.bf(f + ".c_embedder.cond_embedder.bias", c.flow.hidden);
    b.bf(f + ".t_embedder.time_mlp.0.weight", (size_t)c.flow.hidden * c.time_dim);
    b.bf(f + ".t_embedder.time_mlp.0.bias", c.flow.hidden);
    b.bf(f + ".t_embedder.time_mlp.2.weight", (size_t)c.flow.hidden * c.flow.hidden);
    b.bf(f + ".t_embedder.time_mlp.2.bias", c.flow.hidden);
    add_dit(b, f, c.flow);
    const std::string a = "linear_proj_audio";
    b.bf(a + ".x_embedder.weight", (size_t)c.agg.hidden * c.latent_dim);
    b.bf(a + ".x_embedder.bias", c.agg.hidden);
    b.add(a + ".word_embedder.weight", c.agg.hidden, MT_DTYPE_F32, MT_INIT_NORMAL);
    add_dit(b, a, c.agg);
    const std::string v = "audio.decoder";
    b.bf(v + ".fc1.weight", (size_t)c.vae.hidden * c.latent_dim);
    b.bf(v + ".fc1.bias", c.vae.hidden);
    add_qwen(b, v + ".decoder", c.vae);
    b.bf(v + ".head.out.weight", (size_t)(c.nfft + 2) * c.vae.hidden);
    b.bf(v + ".head.out.bias", (size_t)(c.nfft + 2));
    b.add(v + ".head.istft.window", c.nfft, MT_DTYPE_F32, MT_INIT_HANN);
    if (embeddings) b.bf("model.model.embed_tokens.weight", (size_t)c.vocab * c.llm.hidden);
    return b.list;
}

// VAEEncoderWeights (Weights.swift:229-262): frame projections, the encoder stack (the decoder's
// dimensions), the 4-layer patch aggregator with its cls row, and the posterior head.
constexpr int kEncoderAggLayers = 4, kEncoderPatch = 4, kEncoderMaxFrames = 1600;
int encoder_padded_frame(const mt_model_config& c) { return (c.hop + 63) & ~63; }
mt_qwen_config encoder_agg_config(const mt_model_config& c) {
    mt_qwen_config a = c.vae;
    a.layers = kEncoderAggLayers;
    return a;
}

std::vector<mt_tensor_info> encoder_table(const mt_model_config& c, uint64_t seed) {
    Builder b(seed);
    const std::string e = "audio.encoder";
    const size_t h = c.vae.hidden;
    b.bf(e + ".fc1.weight", h * (size_t)encoder_padded_frame(c));
    b.bf(e + ".fc2.weight", h * h);
    b.bf(e + ".fc2.bias", h);
    add_qwen(b, e + ".encoder", c.vae);
    add_qwen(b, e + ".aggregator", encoder_agg_config(c));
    b.add(e + ".cls_embed", h, MT_DTYPE_F32, MT_INIT_NORMAL);
    b.bf(e + ".fc3.weight", 2 * (size_t)c.latent_dim * h);
    b.bf(e + ".fc3.bias", 2 * (size_t)c.latent_dim);
    return b.list;
}

size_t table_bytes(const std::vector<mt_tensor_info>& t) {
    if (t.empty()) return 0;
    const auto& last = t.back();
    const size_t bytes = last.numel * (last.dtype == MT_DTYPE_BF16 ? 2 : 4);
    return last.offset + ((bytes + 255) & ~size_t(255));
}

// Fills fp32 tensors of the table on the device: inv_freq, Hann window, N(0, std) fp32 values
// (bf16-representable, same stream as the bf16 tensors).
__global__ void fill_f32_kernel(float* out, size_t n, int init, uint64_t seed, float std) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = 0.f;
        if (init == MT_INIT_INV_FREQ) v = (float)(1.0 / pow(10000.0, (double)(2 * i) / 64.0));
        else if (init == MT_INIT_HANN) v = (float)(0.5 - 0.5 * cos(2.0 * 3.14159265358979323846 * (double)i / (double)n));
        else if (init == MT_INIT_ONES) v = 1.0f;
        out[i] = v;
    }
}

__global__ void fill_bf16_ones_kernel(uint16_t* out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = 0x3F80;  // 1.0
}

__global__ void bf16_to_f32_kernel(const uint16_t* in, float* out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = bf16f(in[i]);
}

}  // namespace

const mt_tensor_info* find(const std::vector<mt_tensor_info>& t, const std::string& name) {
    for (const auto& i : t)
        if (name == i.name) return &i;
    return nullptr;
}

}  // namespace mt

using namespace mt;

struct mt_model {
    mt_ctx* ctx = nullptr;
    mt_model_config cfg{};
    std::vector<mt_tensor_info> tensors;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    bool owns_arena = false;
    std::vector<mt_qwen_layer> llm_layers, vae_layers;
    std::vector<mt_dit_block> flow_blocks, agg_blocks;
    mt_model_weights w{};
};

struct mt_encoder {
    mt_ctx* ctx = nullptr;
    mt_model_config cfg{};
    std::vector<mt_tensor_info> tensors;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    bool owns_arena = false;
    std::vector<mt_qwen_layer> stack_layers, agg_layers;
    mt_encoder_weights w{};
};

namespace mt {
void model_own_arena(mt_model* m) {
    if (m) m->owns_arena = true;
}
void encoder_own_arena(mt_encoder* e) {
    if (e) e->owns_arena = true;
}
mt_ctx* encoder_ctx(const mt_encoder* e) { return e ? e->ctx : nullptr; }
int encoder_latent_dim(const mt_encoder* e) { return e ? e->cfg.latent_dim : 0; }
}  // namespace mt

namespace {

template <typename T>
const T* at(mt_encoder* m, const std::string& name) {
    const mt_tensor_info* i = find(m->tensors, name);
    return i ? reinterpret_cast<const T*>(m->arena + i->offset) : nullptr;
}

template <typename T>
const T* at(mt_model* m, const std::string& name) {
    const mt_tensor_info* i = find(m->tensors, name);
    return i ? reinterpret_cast<const T*>(m->arena + i->offset) : nullptr;
}

template <typename M>
void bind_qwen(M* m, const std::string& prefix, const mt_qwen_config& c, std::vector<mt_qwen_layer>& layers,
               mt_qwen_weights& w) {
    layers.resize(c.layers);
    for (int l = 0; l < c.layers; l++) {
        const std::string p = prefix + ".layers." + std::to_string(l);
        mt_qwen_layer& L = layers[l];
        L.norm1 = at<mt_bf16>(m, p + ".input_layernorm.weight");
        L.qkv_w = at<mt_bf16>(m, p + ".self_attn.qkv_proj.weight");
        L.qkv_b = at<mt_bf16>(m, p + ".self_attn.qkv_proj.bias");
        L.o_w = at<mt_bf16>(m, p + ".self_attn.o_proj.weight");
        L.norm2 = at<mt_bf16>(m, p + ".post_attention_layernorm.weight");
        L.gate_w = at<mt_bf16>(m, p + ".mlp.gate_proj.weight");
        L.up_w = at<mt_bf16>(m, p + ".mlp.up_proj.weight");
        L.down_w = at<mt_bf16>(m, p + ".mlp.down_proj.weight");
    }
    w.cfg = c;
    w.layers = layers.data();
    w.final_norm = at<mt_bf16>(m, prefix + ".norm.weight");
}

void bind_dit(mt_model* m, const std::string& prefix, const mt_dit_config& c, std::vector<mt_dit_block>& blocks,
              mt_dit_weights& w) {
    blocks.resize(c.depth);
    for (int i = 0; i < c.depth; i++) {
        const std::string p = prefix + ".blocks." + std::to_string(i);
        mt_dit_block& B = blocks[i];
        B.norm1 = at<mt_bf16>(m, p + ".norm1.weight");
        B.qkv_w = at<mt_bf16>(m, p + ".attn.to_qkv.weight");
        B.qkv_b = at<mt_bf16>(m, p + ".attn.to_qkv.bias");
        B.out_w = at<mt_bf16>(m, p + ".attn.to_out.0.weight");
        B.out_b = at<mt_bf16>(m, p + ".attn.to_out.0.bias");
        B.norm2 = at<mt_bf16>(m, p + ".norm2.weight");
        B.ff1_w = at<mt_bf16>(m, p + ".mlp.ff.0.0.weight");
        B.ff1_b = at<mt_bf16>(m, p + ".mlp.ff.0.0.bias");
        B.ff2_w = at<mt_bf16>(m, p + ".mlp.ff.2.weight");
        B.ff2_b = at<mt_bf16>(m, p + ".mlp.ff.2.bias");
    }
    w.cfg = c;
    w.blocks = blocks.data();
    w.final_norm = at<mt_bf16>(m, prefix + ".final_layer.norm_final.weight");
    w.final_w = at<mt_bf16>(m, prefix + ".final_layer.linear.weight");
    w.final_b = at<mt_bf16>(m, prefix + ".final_layer.linear.bias");
    w.inv_freq = at<float>(m, prefix + ".rotary_embed.inv_freq");
}

void bind(mt_model* m) {
    bind_qwen(m, "model.model", m->cfg.llm, m->llm_layers, m->w.llm);
    m->w.stop_w = at<mt_bf16>(m, "stop_head.weight");
    m->w.stop_b = at<mt_bf16>(m, "stop_head.bias");
    const std::string f = "flowloss.cfm.model";
    m->w.flow_x_w = at<mt_bf16>(m, f + ".x_embedder.weight");
    m->w.flow_x_b = at<mt_bf16>(m, f + ".x_embedder.bias");
    m->w.flow_c_w = at<mt_bf16>(m, f + ".c_embedder.cond_embedder.weight");
    m->w.flow_c_b = at<mt_bf16>(m, f + ".c_embedder.cond_embedder.bias");
    m->w.flow_t1_w = at<mt_bf16>(m, f + ".t_embedder.time_mlp.0.weight");
    m->w.flow_t1_b = at<mt_bf16>(m, f + ".t_embedder.time_mlp.0.bias");
    m->w.flow_t2_w = at<mt_bf16>(m, f + ".t_embedder.time_mlp.2.weight");
    m->w.flow_t2_b = at<mt_bf16>(m, f + ".t_embedder.time_mlp.2.bias");
    bind_dit(m, f, m->cfg.flow, m->flow_blocks, m->w.flow);
    const std::string a = "linear_proj_audio";
    m->w.agg_x_w = at<mt_bf16>(m, a + ".x_embedder.weight");
    m->w.agg_x_b = at<mt_bf16>(m, a + ".x_embedder.bias");
    m->w.agg_cls = at<float>(m, a + ".word_embedder.weight");
    bind_dit(m, a, m->cfg.agg, m->agg_blocks, m->w.agg);
    const std::string v = "audio.decoder";
    m->w.vae_fc1_w = at<mt_bf16>(m, v + ".fc1.weight");
    m->w.vae_fc1_b = at<mt_bf16>(m, v + ".fc1.bias");
    bind_qwen(m, v + ".decoder", m->cfg.vae, m->vae_layers, m->w.vae);
    m->w.vae_head_w = at<mt_bf16>(m, v + ".head.out.weight");
    m->w.vae_head_b = at<mt_bf16>(m, v + ".head.out.bias");
    m->w.vae_window = at<float>(m, v + ".head.istft.window");
    m->w.embed_tokens = at<mt_bf16>(m, "model.model.embed_tokens.weight");
}

void bind_encoder(mt_encoder* e) {
    const mt_model_config& c = e->cfg;
    const std::string p = "audio.encoder";
    e->w.frame = c.hop;
    e->w.padded_frame = encoder_padded_frame(c);
    e->w.patch = kEncoderPatch;
    e->w.max_frames = kEncoderMaxFrames;
    e->w.fc1_w = at<mt_bf16>(e, p + ".fc1.weight");
    e->w.fc2_w = at<mt_bf16>(e, p + ".fc2.weight");
    e->w.fc2_b = at<mt_bf16>(e, p + ".fc2.bias");
    bind_qwen(e, p + ".encoder", c.vae, e->stack_layers, e->w.stack);
    bind_qwen(e, p + ".aggregator", encoder_agg_config(c), e->agg_layers, e->w.aggregator);
    e->w.cls = at<float>(e, p + ".cls_embed");
    e->w.fc3_w = at<mt_bf16>(e, p + ".fc3.weight");
    e->w.fc3_b = at<mt_bf16>(e, p + ".fc3.bias");
}

// Random fill of a table's tensors in `arena` (see mt_model_create_random).
cudaError_t fill_random(mt_ctx* ctx, const std::vector<mt_tensor_info>& tensors, uint8_t* arena) {
    for (const auto& t : tensors) {
        void* p = arena + t.offset;
        const unsigned blocks = (unsigned)std::min<size_t>((t.numel + 255) / 256, (size_t)ctx->sm_count * 8);
        if (t.dtype == MT_DTYPE_BF16) {
            if (t.init == MT_INIT_ONES) fill_bf16_ones_kernel<<<blocks, 256>>>(static_cast<uint16_t*>(p), t.numel);
            else mt_randn_bf16(ctx, nullptr, static_cast<mt_bf16*>(p), t.numel, t.seed, t.std);
        } else if (t.init == MT_INIT_NORMAL) {
            // bf16-representable fp32 values: draw as bf16 into a temporary, widen into the slot.
            uint16_t* tmp = nullptr;
            cudaMalloc(&tmp, t.numel * 2);
            mt_randn_bf16(ctx, nullptr, tmp, t.numel, t.seed, t.std);
            bf16_to_f32_kernel<<<blocks, 256>>>(tmp, static_cast<float*>(p), t.numel);
            cudaDeviceSynchronize();
            cudaFree(tmp);
        } else {
            fill_f32_kernel<<<blocks, 256>>>(static_cast<float*>(p), t.numel, t.init, t.seed, t.std);
        }
    }
    return cudaDeviceSynchronize();
}

mt_status check_config(mt_ctx* ctx, const mt_model_config& c) {
    auto ok_qwen = [](const mt_qwen_config& q) {
        return q.hidden > 0 && q.hidden % 64 == 0 && q.heads > 0 && q.kv_heads > 0 && q.heads % q.kv_heads == 0 &&
               q.heads / q.kv_heads <= 8 && q.heads + 2 * q.kv_heads <= 32 && q.intermediate % 64 == 0 && q.layers > 0;
    };
    auto ok_dit = [](const mt_dit_config& d) {
        return d.hidden == d.heads * 64 && d.depth > 0 && d.ff % 64 == 0 && d.out_dim > 0;
    };
    MT_REQUIRE(ctx, ok_qwen(c.llm) && ok_qwen(c.vae) && ok_dit(c.flow) && ok_dit(c.agg), MT_ERR_SHAPE,
               "model config: unsupported stack dimensions (head dim 64, hidden %% 64, heads/kv <= 8)");
    MT_REQUIRE(ctx, c.flow.out_dim == c.latent_dim && c.agg.out_dim == c.llm.hidden && c.latent_dim % 8 == 0 &&
                        c.latent_dim <= 64 && c.flow.hidden % 128 == 0 && c.flow.hidden <= 1024 &&
                        c.time_dim % 8 == 0 && c.nfft % 4 == 0 && c.hop > 0 && (c.nfft - c.hop) % 2 == 0 &&
                        c.flow_steps > 0 && c.llm_capacity > 1,
               MT_ERR_SHAPE, "model config: inconsistent dimensions");
    return MT_OK;
}

}  // namespace

extern "C" {

void mt_model_config_default(mt_model_config* c) {
    if (!c) return;
    memset(c, 0, sizeof(*c));
    c->llm = mt_qwen_config{896, 14, 2, 4864, 24, 0, 1e6f, 1e-6f};
    c->vae = c->llm;
    c->vae.window = 65;
    c->flow = mt_dit_config{1024, 16, 8, 4096, 64, 1e-6f};
    c->agg = mt_dit_config{1024, 16, 8, 4096, 896, 1e-6f};
    c->latent_dim = 64;
    c->time_dim = 256;
    c->vocab = 151936;
    c->nfft = 3528;
    c->hop = 882;
    c->flow_steps = 10;
    c->llm_capacity = 512;
}

int mt_model_tensors(const mt_model_config* cfg, uint64_t seed, int with_embeddings, mt_tensor_info* out, int cap) {
    if (!cfg) return -1;
    auto t = table(*cfg, seed, with_embeddings != 0);
    if (out)
        for (int i = 0; i < (int)t.size() && i < cap; i++) out[i] = t[i];
    return (int)t.size();
}

size_t mt_model_arena_bytes(const mt_model_config* cfg, int with_embeddings) {
    if (!cfg) return 0;
    auto t = table(*cfg, 0, with_embeddings != 0);
    if (t.empty()) return 0;
    const auto& last = t.back();
    const size_t bytes = last.numel * (last.dtype == MT_DTYPE_BF16 ? 2 : 4);
    return last.offset + ((bytes + 255) & ~size_t(255));
}

mt_status mt_model_create_random(mt_ctx* ctx, const mt_model_config* cfg, uint64_t seed, int with_embeddings,
                                 mt_model** out) {
    MT_REQUIRE(ctx, ctx && cfg && out, MT_ERR_ARG, "mt_model_create_random: null argument");
    *out = nullptr;
    mt_status st = check_config(ctx, *cfg);
    if (st != MT_OK) return st;
    mt_model* m = new mt_model();
    m->ctx = ctx;
    m->cfg = *cfg;
    m->tensors = table(*cfg, seed, with_embeddings != 0);
    m->arena_bytes = mt_model_arena_bytes(cfg, with_embeddings);
    cudaError_t e = cudaMalloc(&m->arena, m->arena_bytes);
    if (e != cudaSuccess) {
        delete m;
        return fail(ctx, MT_ERR_NOMEM, "model arena of %zu bytes: %s", m->arena_bytes, cudaGetErrorString(e));
    }
    m->owns_arena = true;
    e = fill_random(ctx, m->tensors, m->arena);
    if (e != cudaSuccess) {
        cudaFree(m->arena);
        delete m;
        return fail(ctx, MT_ERR_CUDA, "model init: %s", cudaGetErrorString(e));
    }
    bind(m);
    *out = m;
    return MT_OK;
}

mt_status mt_model_create_from_arena(mt_ctx* ctx, const mt_model_config* cfg, void* device_arena, int with_embeddings,
                                     mt_model** out) {
    MT_REQUIRE(ctx, ctx && cfg && device_arena && out, MT_ERR_ARG, "mt_model_create_from_arena: null argument");
    MT_REQUIRE(ctx, ((uintptr_t)device_arena & 255u) == 0, MT_ERR_ARG, "mt_model_create_from_arena: arena needs 256-byte alignment");
    *out = nullptr;
    mt_status st = check_config(ctx, *cfg);
    if (st != MT_OK) return st;
    mt_model* m = new mt_model();
    m->ctx = ctx;
    m->cfg = *cfg;
    m->tensors = table(*cfg, 0, with_embeddings != 0);
    m->arena_bytes = mt_model_arena_bytes(cfg, with_embeddings);
    m->arena = static_cast<uint8_t*>(device_arena);
    m->owns_arena = false;
    bind(m);
    *out = m;
    return MT_OK;
}

const mt_model_weights* mt_model_get_weights(const mt_model* m) { return m ? &m->w : nullptr; }

const mt_model_config* mt_model_get_config(const mt_model* m) { return m ? &m->cfg : nullptr; }

mt_status mt_model_arena(const mt_model* m, void** ptr, size_t* bytes) {
    if (!m || !ptr || !bytes) return MT_ERR_ARG;
    *ptr = m->arena;
    *bytes = m->arena_bytes;
    return MT_OK;
}

void mt_model_destroy(mt_model* m) {
    if (!m) return;
    if (m->owns_arena && m->arena) cudaFree(m->arena);
    delete m;
}

int mt_encoder_tensors(const mt_model_config* cfg, uint64_t seed, mt_tensor_info* out, int cap) {
    if (!cfg) return -1;
    auto t = encoder_table(*cfg, seed);
    if (out)
        for (int i = 0; i < (int)t.size() && i < cap; i++) out[i] = t[i];
    return (int)t.size();
}

size_t mt_encoder_arena_bytes(const mt_model_config* cfg) { return cfg ? table_bytes(encoder_table(*cfg, 0)) : 0; }

mt_status mt_encoder_create_random(mt_ctx* ctx, const mt_model_config* cfg, uint64_t seed, mt_encoder** out) {
    MT_REQUIRE(ctx, ctx && cfg && out, MT_ERR_ARG, "mt_encoder_create_random: null argument");
    *out = nullptr;
    mt_status st = check_config(ctx, *cfg);
    if (st != MT_OK) return st;
    mt_encoder* e = new mt_encoder();
    e->ctx = ctx;
    e->cfg = *cfg;
    e->tensors = encoder_table(*cfg, seed);
    e->arena_bytes = table_bytes(e->tensors);
    cudaError_t err = cudaMalloc(&e->arena, e->arena_bytes);
    if (err != cudaSuccess) {
        delete e;
        return fail(ctx, MT_ERR_NOMEM, "encoder arena of %zu bytes: %s", e->arena_bytes, cudaGetErrorString(err));
    }
    e->owns_arena = true;
    err = fill_random(ctx, e->tensors, e->arena);
    if (err == cudaSuccess) {  // fc1 columns past the frame are zero, as WeightArena.paddedLinear stores them
        const int pf = encoder_padded_frame(*cfg), f = cfg->hop;
        if (pf > f)
            err = cudaMemset2D(e->arena + e->tensors[0].offset + (size_t)f * 2, (size_t)pf * 2, 0, (size_t)(pf - f) * 2,
                               (size_t)cfg->vae.hidden);
        if (err == cudaSuccess) err = cudaDeviceSynchronize();
    }
    if (err != cudaSuccess) {
        cudaFree(e->arena);
        delete e;
        return fail(ctx, MT_ERR_CUDA, "encoder init: %s", cudaGetErrorString(err));
    }
    bind_encoder(e);
    *out = e;
    return MT_OK;
}

mt_status mt_encoder_create_from_arena(mt_ctx* ctx, const mt_model_config* cfg, void* device_arena, mt_encoder** out) {
    MT_REQUIRE(ctx, ctx && cfg && device_arena && out, MT_ERR_ARG, "mt_encoder_create_from_arena: null argument");
    MT_REQUIRE(ctx, ((uintptr_t)device_arena & 255u) == 0, MT_ERR_ARG,
               "mt_encoder_create_from_arena: arena needs 256-byte alignment");
    *out = nullptr;
    mt_status st = check_config(ctx, *cfg);
    if (st != MT_OK) return st;
    mt_encoder* e = new mt_encoder();
    e->ctx = ctx;
    e->cfg = *cfg;
    e->tensors = encoder_table(*cfg, 0);
    e->arena_bytes = table_bytes(e->tensors);
    e->arena = static_cast<uint8_t*>(device_arena);
    e->owns_arena = false;
    bind_encoder(e);
    *out = e;
    return MT_OK;
}

const mt_encoder_weights* mt_encoder_get_weights(const mt_encoder* e) { return e ? &e->w : nullptr; }

mt_status mt_encoder_arena(const mt_encoder* e, void** ptr, size_t* bytes) {
    if (!e || !ptr || !bytes) return MT_ERR_ARG;
    *ptr = e->arena;
    *bytes = e->arena_bytes;
    return MT_OK;
}

void mt_encoder_destroy(mt_encoder* e) {
    if (!e) return;
    if (e->owns_arena && e->arena) cudaFree(e->arena);
    delete e;
}

}  // extern "C"
