// checkpoint.cu -- safetensors checkpoint loading into the model arena (host code only).
//
// Reference: SafeTensors.swift:7-87 (a memory-mapped file: u64 little-endian header length, a JSON
// header {name: {dtype, shape, data_offsets}} with an optional "__metadata__" entry, then the raw
// tensor bytes) and WeightArena.tensor / linear (Weights.swift:32-62: bf16 tensors copied into one
// 256-byte-aligned buffer, several names concatenated along their first axis for q/k/v, element
// counts checked), with the tensor names of the *Weights initialisers (Weights.swift:116-263).
// fp32 table entries (rotary inv_freq, the ISTFT window, the aggregator cls row) are decoded from
// BF16 or F32 as SafeTensors.floats does (:66-78).
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <utility>
#include <vector>

#include "common.cuh"

namespace mt {

namespace {

// ---- a small JSON reader: objects, arrays, strings, integers/reals, true/false/null ---------------
struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    bool is_int = false;
    long long i = 0;
    double d = 0;
    std::string s;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const char* key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char* p;
    const char* end;
    int depth = 0;
    bool ok = true;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool lit(const char* w) {
        const size_t n = strlen(w);
        if ((size_t)(end - p) < n || memcmp(p, w, n) != 0) return false;
        p += n;
        return true;
    }
    static void utf8(std::string& out, unsigned cp) {
        if (cp < 0x80) out += (char)cp;
        else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
        else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F));
        } else {
            out += (char)(0xF0 | (cp >> 18)); out += (char)(0x80 | ((cp >> 12) & 0x3F));
            out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(unsigned& v) {
        if (end - p < 4) return false;
        v = 0;
        for (int k = 0; k < 4; k++) {
            const char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool str(std::string& out) {
        if (p >= end || *p != '"') return false;
        p++;
        while (p < end && *p != '"') {
            if (*p != '\\') { out += *p++; continue; }
            if (++p >= end) return false;
            const char c = *p++;
            switch (c) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    unsigned cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
                        unsigned lo;
                        if (end - p < 6 || p[0] != '\\' || p[1] != 'u') return false;
                        p += 2;
                        if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: return false;
            }
        }
        if (p >= end) return false;
        p++;
        return true;
    }
    bool num(JVal& v) {
        const char* s = p;
        if (p < end && *p == '-') p++;
        if (p >= end || *p < '0' || *p > '9') return false;
        while (p < end && *p >= '0' && *p <= '9') p++;
        bool real = false;
        if (p < end && *p == '.') {
            real = true;
            p++;
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        if (p < end && (*p == 'e' || *p == 'E')) {
            real = true;
            p++;
            if (p < end && (*p == '+' || *p == '-')) p++;
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        const std::string text(s, p);
        v.kind = JVal::NUM;
        v.d = strtod(text.c_str(), nullptr);
        v.is_int = !real && text.size() < 19;
        if (v.is_int) v.i = strtoll(text.c_str(), nullptr, 10);
        return true;
    }
    bool value(JVal& v) {
        if (++depth > 64) return false;
        ws();
        if (p >= end) return false;
        bool r = true;
        if (*p == '{') {
            v.kind = JVal::OBJ;
            p++;
            ws();
            if (p < end && *p == '}') { p++; }
            else {
                for (;;) {
                    std::string key;
                    ws();
                    if (!str(key)) { r = false; break; }
                    ws();
                    if (p >= end || *p != ':') { r = false; break; }
                    p++;
                    v.obj.emplace_back(std::move(key), JVal());
                    if (!value(v.obj.back().second)) { r = false; break; }
                    ws();
                    if (p < end && *p == ',') { p++; continue; }
                    if (p < end && *p == '}') { p++; break; }
                    r = false;
                    break;
                }
            }
        } else if (*p == '[') {
            v.kind = JVal::ARR;
            p++;
            ws();
            if (p < end && *p == ']') { p++; }
            else {
                for (;;) {
                    v.arr.emplace_back();
                    if (!value(v.arr.back())) { r = false; break; }
                    ws();
                    if (p < end && *p == ',') { p++; continue; }
                    if (p < end && *p == ']') { p++; break; }
                    r = false;
                    break;
                }
            }
        } else if (*p == '"') {
            v.kind = JVal::STR;
            r = str(v.s);
        } else if (lit("true")) { v.kind = JVal::BOOL; v.b = true; }
        else if (lit("false")) { v.kind = JVal::BOOL; v.b = false; }
        else if (lit("null")) { v.kind = JVal::NUL; }
        else r = num(v);
        depth--;
        return r;
    }
};

// ---- the file -------------------------------------------------------------------------------------
struct Entry {
    std::string name, dtype;
    std::vector<long long> shape;
    long long begin = 0, end = 0;  // byte range inside the data section
    long long count() const {
        long long n = 1;
        for (long long d : shape) n *= d;
        return n;
    }
};

struct SafeTensorsFile {
    int fd = -1;
    const uint8_t* map = nullptr;
    size_t size = 0;
    size_t data_start = 0;
    std::vector<Entry> entries;
    std::string err;

    ~SafeTensorsFile() {
        if (map) munmap(const_cast<uint8_t*>(map), size);
        if (fd >= 0) close(fd);
    }
    bool fail(const char* fmt, ...) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        err = buf;
        return false;
    }
    bool open_file(const char* path) {
        fd = ::open(path, O_RDONLY);
        if (fd < 0) return fail("bad checkpoint: cannot open %s", path);
        struct stat sb;
        if (fstat(fd, &sb) != 0) return fail("bad checkpoint: cannot stat %s", path);
        size = (size_t)sb.st_size;
        if (size < 8) return fail("bad checkpoint: file too small");
        void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (m == MAP_FAILED) return fail("bad checkpoint: cannot map %s", path);
        map = static_cast<const uint8_t*>(m);
        uint64_t hlen;
        memcpy(&hlen, map, 8);
        if (hlen == 0 || hlen > size - 8) return fail("bad checkpoint: header length %llu exceeds file", (unsigned long long)hlen);
        data_start = 8 + (size_t)hlen;
        JParser jp{reinterpret_cast<const char*>(map) + 8, reinterpret_cast<const char*>(map) + data_start};
        JVal root;
        if (!jp.value(root) || root.kind != JVal::OBJ) return fail("bad checkpoint: header is not a JSON object");
        long long last = 0;
        for (const auto& kv : root.obj) {
            if (kv.first == "__metadata__") continue;
            const JVal& v = kv.second;
            const JVal* dt = v.kind == JVal::OBJ ? v.get("dtype") : nullptr;
            const JVal* sh = v.kind == JVal::OBJ ? v.get("shape") : nullptr;
            const JVal* off = v.kind == JVal::OBJ ? v.get("data_offsets") : nullptr;
            bool good = dt && dt->kind == JVal::STR && sh && sh->kind == JVal::ARR && off && off->kind == JVal::ARR &&
                        off->arr.size() == 2;
            Entry e;
            if (good) {
                e.name = kv.first;
                e.dtype = dt->s;
                for (const JVal& d : sh->arr) {
                    if (d.kind != JVal::NUM || !d.is_int || d.i < 0) good = false;
                    e.shape.push_back(d.i);
                }
                for (const JVal& o : off->arr)
                    if (o.kind != JVal::NUM || !o.is_int || o.i < 0) good = false;
                if (good) {
                    e.begin = off->arr[0].i;
                    e.end = off->arr[1].i;
                    good = e.begin <= e.end;
                }
            }
            if (!good) return fail("bad checkpoint: malformed entry %s", kv.first.c_str());
            if (e.end > last) last = e.end;
            entries.push_back(std::move(e));
        }
        if ((unsigned long long)last > size - data_start)
            return fail("bad checkpoint: file holds %zu bytes, header needs %llu; download incomplete?", size,
                        (unsigned long long)(data_start + last));
        return true;
    }
    const Entry* find(const std::string& name) const {
        for (const auto& e : entries)
            if (e.name == name) return &e;
        return nullptr;
    }
    const uint8_t* bytes(const Entry& e) const { return map + data_start + e.begin; }
};

// The checkpoint tensors a table entry is gathered from: q/k/v projections are one table tensor
// (Weights.swift:121-122 for the Qwen stacks, :158-159 for the DiT blocks).
std::vector<std::string> sources(const std::string& name) {
    auto replace = [&](const char* from, const char* const* parts) {
        const size_t at = name.find(from);
        std::vector<std::string> out;
        for (int i = 0; i < 3; i++) {
            std::string s = name;
            s.replace(at, strlen(from), parts[i]);
            out.push_back(s);
        }
        return out;
    };
    static const char* const qwen[3] = {".self_attn.q_proj.", ".self_attn.k_proj.", ".self_attn.v_proj."};
    static const char* const dit[3] = {".attn.to_q.", ".attn.to_k.", ".attn.to_v."};
    if (name.find(".self_attn.qkv_proj.") != std::string::npos) return replace(".self_attn.qkv_proj.", qwen);
    if (name.find(".attn.to_qkv.") != std::string::npos) return replace(".attn.to_qkv.", dit);
    return {name};
}

// A bf16 [rows, stored] checkpoint tensor laid out as [rows, padded] with zero columns past
// `stored` (WeightArena.paddedLinear, Weights.swift:64-77: the encoder's fc1 frames of 882 samples).
struct Padded {
    std::string name;
    long long rows = 0, stored = 0, padded = 0;
};

// Fills `arena` (arena_bytes, laid out as `table`) from the file; err gets the message.
bool fill_table(const SafeTensorsFile& f, const std::vector<mt_tensor_info>& table, size_t table_bytes,
                const std::vector<Padded>& padded, uint8_t* arena, size_t arena_bytes, std::string& err) {
    if (table_bytes > arena_bytes) {
        err = "checkpoint: arena buffer smaller than the table's arena";
        return false;
    }
    memset(arena, 0, arena_bytes);
    char buf[512];
    for (const mt_tensor_info& t : table) {
        const std::vector<std::string> src = sources(t.name);
        uint8_t* dst = arena + t.offset;
        const Padded* pad = nullptr;
        for (const Padded& p : padded)
            if (p.name == t.name) pad = &p;
        if (pad) {
            const Entry* e = f.find(pad->name);
            if (!e) { err = "missing tensor " + pad->name; return false; }
            if (e->dtype != "BF16" || e->shape.size() != 2 || e->shape[0] != pad->rows || e->shape[1] != pad->stored ||
                e->end - e->begin != e->count() * 2) {
                snprintf(buf, sizeof(buf), "bad checkpoint: %s is %s [%lld, %lld], expected BF16 [%lld, %lld]",
                         pad->name.c_str(), e->dtype.c_str(), e->shape.size() > 0 ? e->shape[0] : -1LL,
                         e->shape.size() > 1 ? e->shape[1] : -1LL, pad->rows, pad->stored);
                err = buf;
                return false;
            }
            for (long long r = 0; r < pad->rows; r++)
                memcpy(dst + (size_t)r * pad->padded * 2, f.bytes(*e) + (size_t)r * pad->stored * 2, (size_t)pad->stored * 2);
            continue;
        }
        if (t.dtype == MT_DTYPE_BF16) {
            long long total = 0;
            for (const std::string& s : src) {
                const Entry* e = f.find(s);
                if (!e) { err = "missing tensor " + s; return false; }
                if (e->dtype != "BF16") {
                    snprintf(buf, sizeof(buf), "bad checkpoint: %s is %s, expected BF16", s.c_str(), e->dtype.c_str());
                    err = buf;
                    return false;
                }
                if (e->end - e->begin != e->count() * 2) {
                    snprintf(buf, sizeof(buf), "bad checkpoint: %s holds %lld bytes for %lld elements", s.c_str(),
                             e->end - e->begin, e->count());
                    err = buf;
                    return false;
                }
                total += e->count();
            }
            if (total != (long long)t.numel) {
                snprintf(buf, sizeof(buf), "bad checkpoint: %s has %lld elements, expected %zu", t.name, total, t.numel);
                err = buf;
                return false;
            }
            for (const std::string& s : src) {
                const Entry* e = f.find(s);
                memcpy(dst, f.bytes(*e), (size_t)(e->end - e->begin));
                dst += e->end - e->begin;
            }
        } else {  // fp32 table entry, decoded from BF16 or F32
            const Entry* e = f.find(src[0]);
            if (!e) { err = "missing tensor " + src[0]; return false; }
            const bool bf = e->dtype == "BF16", f32 = e->dtype == "F32";
            if (!bf && !f32) {
                snprintf(buf, sizeof(buf), "bad checkpoint: %s has dtype %s", src[0].c_str(), e->dtype.c_str());
                err = buf;
                return false;
            }
            if (e->count() != (long long)t.numel || e->end - e->begin != e->count() * (bf ? 2 : 4)) {
                snprintf(buf, sizeof(buf), "bad checkpoint: %s has %lld elements, expected %zu", src[0].c_str(),
                         e->count(), t.numel);
                err = buf;
                return false;
            }
            float* out = reinterpret_cast<float*>(dst);
            const uint8_t* in = f.bytes(*e);
            for (size_t i = 0; i < t.numel; i++) {
                if (bf) {
                    uint16_t h;
                    memcpy(&h, in + 2 * i, 2);
                    const uint32_t u = (uint32_t)h << 16;
                    memcpy(&out[i], &u, 4);
                } else {
                    memcpy(&out[i], in + 4 * i, 4);
                }
            }
        }
    }
    return true;
}

bool fill_arena(const SafeTensorsFile& f, const mt_model_config& cfg, bool embeddings, uint8_t* arena,
                size_t arena_bytes, std::string& err) {
    const int n = mt_model_tensors(&cfg, 0, embeddings ? 1 : 0, nullptr, 0);
    std::vector<mt_tensor_info> table((size_t)n);
    mt_model_tensors(&cfg, 0, embeddings ? 1 : 0, table.data(), n);
    return fill_table(f, table, mt_model_arena_bytes(&cfg, embeddings ? 1 : 0), {}, arena, arena_bytes, err);
}

bool fill_encoder_arena(const SafeTensorsFile& f, const mt_model_config& cfg, uint8_t* arena, size_t arena_bytes,
                        std::string& err) {
    const int n = mt_encoder_tensors(&cfg, 0, nullptr, 0);
    std::vector<mt_tensor_info> table((size_t)n);
    mt_encoder_tensors(&cfg, 0, table.data(), n);
    Padded fc1;
    fc1.name = "audio.encoder.fc1.weight";
    fc1.rows = cfg.vae.hidden;
    fc1.stored = cfg.hop;
    fc1.padded = (cfg.hop + 63) & ~63;
    return fill_table(f, table, mt_encoder_arena_bytes(&cfg), {fc1}, arena, arena_bytes, err);
}

}  // namespace

}  // namespace mt

extern "C" {

mt_status mt_checkpoint_fill_arena(const char* path, const mt_model_config* cfg, int with_embeddings, void* host_arena,
                                   size_t arena_bytes, char* err, size_t err_len) {
    if (err && err_len) err[0] = 0;
    auto report = [&](mt_status st, const std::string& msg) {
        if (err && err_len) snprintf(err, err_len, "%s", msg.c_str());
        return st;
    };
    if (!path || !cfg || !host_arena) return report(MT_ERR_ARG, "mt_checkpoint_fill_arena: null argument");
    mt::SafeTensorsFile f;
    if (!f.open_file(path)) return report(MT_ERR_CHECKPOINT, f.err);
    std::string msg;
    if (!mt::fill_arena(f, *cfg, with_embeddings != 0, static_cast<uint8_t*>(host_arena), arena_bytes, msg))
        return report(MT_ERR_CHECKPOINT, msg);
    return MT_OK;
}

mt_status mt_checkpoint_fill_encoder_arena(const char* path, const mt_model_config* cfg, void* host_arena,
                                           size_t arena_bytes, char* err, size_t err_len) {
    if (err && err_len) err[0] = 0;
    auto report = [&](mt_status st, const std::string& msg) {
        if (err && err_len) snprintf(err, err_len, "%s", msg.c_str());
        return st;
    };
    if (!path || !cfg || !host_arena) return report(MT_ERR_ARG, "mt_checkpoint_fill_encoder_arena: null argument");
    mt::SafeTensorsFile f;
    if (!f.open_file(path)) return report(MT_ERR_CHECKPOINT, f.err);
    std::string msg;
    if (!mt::fill_encoder_arena(f, *cfg, static_cast<uint8_t*>(host_arena), arena_bytes, msg))
        return report(MT_ERR_CHECKPOINT, msg);
    return MT_OK;
}

mt_status mt_encoder_load_safetensors(mt_ctx* ctx, const mt_model_config* cfg, const char* path, mt_encoder** out) {
    if (!ctx) return MT_ERR_ARG;
    MT_REQUIRE(ctx, cfg && path && out, MT_ERR_ARG, "mt_encoder_load_safetensors: null argument");
    *out = nullptr;
    const size_t bytes = mt_encoder_arena_bytes(cfg);
    void* host = nullptr;
    if (cudaMallocHost(&host, bytes) != cudaSuccess) {
        cudaGetLastError();
        return mt::fail(ctx, MT_ERR_NOMEM, "mt_encoder_load_safetensors: %zu bytes of pinned host memory", bytes);
    }
    std::vector<char> msg(512);
    mt_status st = mt_checkpoint_fill_encoder_arena(path, cfg, host, bytes, msg.data(), msg.size());
    if (st != MT_OK) {
        cudaFreeHost(host);
        return mt::fail(ctx, st, "%s", msg.data());
    }
    void* dev = nullptr;
    if (cudaMalloc(&dev, bytes) != cudaSuccess) {
        cudaGetLastError();
        cudaFreeHost(host);
        return mt::fail(ctx, MT_ERR_NOMEM, "mt_encoder_load_safetensors: %zu bytes of device memory", bytes);
    }
    const cudaError_t ce = cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice);
    cudaFreeHost(host);
    if (ce != cudaSuccess) {
        cudaFree(dev);
        return mt::fail(ctx, MT_ERR_CUDA, "mt_encoder_load_safetensors: copy to the device: %s", cudaGetErrorString(ce));
    }
    st = mt_encoder_create_from_arena(ctx, cfg, dev, out);
    if (st != MT_OK) {
        cudaFree(dev);
        return st;
    }
    mt::encoder_own_arena(*out);
    return MT_OK;
}

mt_status mt_model_load_safetensors(mt_ctx* ctx, const mt_model_config* cfg, const char* path, int with_embeddings,
                                    mt_model** out) {
    if (!ctx) return MT_ERR_ARG;
    MT_REQUIRE(ctx, cfg && path && out, MT_ERR_ARG, "mt_model_load_safetensors: null argument");
    *out = nullptr;
    const size_t bytes = mt_model_arena_bytes(cfg, with_embeddings);
    void* host = nullptr;
    if (cudaMallocHost(&host, bytes) != cudaSuccess) {
        cudaGetLastError();
        return mt::fail(ctx, MT_ERR_NOMEM, "mt_model_load_safetensors: %zu bytes of pinned host memory", bytes);
    }
    std::vector<char> msg(512);
    mt_status st = mt_checkpoint_fill_arena(path, cfg, with_embeddings, host, bytes, msg.data(), msg.size());
    if (st != MT_OK) {
        cudaFreeHost(host);
        return mt::fail(ctx, st, "%s", msg.data());
    }
    void* dev = nullptr;
    if (cudaMalloc(&dev, bytes) != cudaSuccess) {
        cudaGetLastError();
        cudaFreeHost(host);
        return mt::fail(ctx, MT_ERR_NOMEM, "mt_model_load_safetensors: %zu bytes of device memory", bytes);
    }
    const cudaError_t ce = cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice);
    cudaFreeHost(host);
    if (ce != cudaSuccess) {
        cudaFree(dev);
        return mt::fail(ctx, MT_ERR_CUDA, "mt_model_load_safetensors: copy to the device: %s", cudaGetErrorString(ce));
    }
    st = mt_model_create_from_arena(ctx, cfg, dev, with_embeddings, out);
    if (st != MT_OK) {
        cudaFree(dev);
        return st;
    }
    mt::model_own_arena(*out);
    return MT_OK;
}

}  // extern "C"
