// gguf_loader.cpp -- native GGUF reader and TransformerConfig resolution.
//
// The header parse follows GgufReader (src/Llmdot.Core/Loading/GgufReader.cs:8-126): magic,
// version >= 2, tensor and metadata counts, typed metadata, tensor infos whose dims the
// reference narrows to uint, data section aligned to general.alignment (default 32).
// Config resolution follows ArchitectureResolver.Resolve (ArchitectureResolver.cs:14-112);
// tensors that run past the end of the file are skipped like LoadedModel.LoadTensors does
// (src/Llmdot.Core/Inference/LoadedModel.cs:77-107).  The file is memory-mapped, so tensor
// bytes stream from the page cache straight into the device upload.
#include "gguf_loader.h"

#include <fcntl.h>
#include <math.h>
#include <string.h>
#include <strings.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>

#include "common.cuh"

namespace llmdot {

namespace {

enum { V_U8 = 0, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64 };

struct Value {
    uint32_t type = 0;
    double num = 0;
    std::string str;
    uint32_t arr_type = 0;
    uint64_t arr_n = 0;
    std::vector<double> arr_num;
};

struct Reader {
    const uint8_t *p, *end;
    bool err = false;
    uint64_t n(int k)
    {
        if (p + k > end) { err = true; return 0; }
        uint64_t v = 0;
        for (int i = 0; i < k; i++) v |= (uint64_t)p[i] << (8 * i);
        p += k;
        return v;
    }
    std::string str()
    {
        uint64_t len = n(8);
        if (err || (uint64_t)(end - p) < len) { err = true; return std::string(); }
        std::string s((const char *)p, (size_t)len);
        p += len;
        return s;
    }
    // a nested array's contents (ReadGgufArray reads them recursively; nothing on this path uses
    // them), depth-limited so that a crafted file cannot exhaust the stack
    void skip_array(int depth)
    {
        if (depth > 64) { err = true; return; }
        const uint32_t t = (uint32_t)n(4);
        const uint64_t cnt = n(8);
        for (uint64_t j = 0; j < cnt && !err; j++) {
            if (t == V_STR) str();
            else if (t == V_ARR) skip_array(depth + 1);
            else scalar(t);
        }
    }
    double scalar(uint32_t t)
    {
        switch (t) {
        case V_U8: return (double)(uint8_t)n(1);
        case V_I8: return (double)(int8_t)n(1);
        case V_U16: return (double)(uint16_t)n(2);
        case V_I16: return (double)(int16_t)n(2);
        case V_U32: return (double)(uint32_t)n(4);
        case V_I32: return (double)(int32_t)n(4);
        case V_F32: { uint32_t b = (uint32_t)n(4); float f; memcpy(&f, &b, 4); return (double)f; }
        case V_BOOL: return n(1) ? 1.0 : 0.0;
        case V_U64: return (double)n(8);
        case V_I64: return (double)(int64_t)n(8);
        case V_F64: { uint64_t b = n(8); double d; memcpy(&d, &b, 8); return d; }
        default: err = true; return 0;
        }
    }
};

struct Meta {
    std::map<std::string, Value> kv;
    std::string arch;
    const Value *get(const std::string &k) const
    {
        auto it = kv.find(k);
        return it == kv.end() ? nullptr : &it->second;
    }
    const Value *arch_get(const std::string &k) const { return get(arch + "." + k); }
    static bool numeric(const Value *v) { return v && v->type != V_STR && v->type != V_ARR; }
    int geti(const std::string &k, int def) const
    {
        const Value *v = arch_get(k);
        return numeric(v) ? (int)nearbyint(v->num) : def;  // Convert.ToInt32 rounds half to even
    }
    float getf(const std::string &k, float def, bool *present = nullptr) const
    {
        const Value *v = arch_get(k);
        if (present) *present = numeric(v);
        return numeric(v) ? (float)v->num : def;
    }
};

}  // namespace

int gguf_open(const char *path, GgufModelFile *out)
{
    int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(LLMDOT_E_INVALID, std::string("cannot open ") + path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 4) {
        close(fd);
        return fail(LLMDOT_E_FORMAT, "Invalid GGUF magic. Expected 'GGUF'.");
    }
    void *map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return fail(LLMDOT_E_INVALID, "mmap failed");
    out->map = map;
    out->size = (size_t)st.st_size;
    const uint8_t *base = (const uint8_t *)map;
    auto bad = [&](const std::string &msg) {
        gguf_close(out);
        return fail(LLMDOT_E_FORMAT, msg);
    };
    if (memcmp(base, "GGUF", 4) != 0) return bad("Invalid GGUF magic. Expected 'GGUF'.");
    Reader r{base + 4, base + out->size};
    uint32_t version = (uint32_t)r.n(4);
    if (version < 2) return bad("Unsupported GGUF version: " + std::to_string(version));
    uint64_t nt = r.n(8), nkv = r.n(8);
    Meta meta;
    for (uint64_t i = 0; i < nkv && !r.err; i++) {
        std::string key = r.str();
        Value v;
        v.type = (uint32_t)r.n(4);
        if (v.type == V_STR) v.str = r.str();
        else if (v.type == V_ARR) {
            v.arr_type = (uint32_t)r.n(4);
            v.arr_n = r.n(8);
            for (uint64_t j = 0; j < v.arr_n && !r.err; j++) {
                if (v.arr_type == V_STR) r.str();
                else if (v.arr_type == V_ARR) r.skip_array(1);
                else v.arr_num.push_back(r.scalar(v.arr_type));
            }
        } else v.num = r.scalar(v.type);
        meta.kv[key] = std::move(v);
    }
    for (uint64_t i = 0; i < nt && !r.err; i++) {
        GgufTensor t;
        t.name = r.str();
        t.n_dims = (uint32_t)r.n(4);
        if (t.n_dims > 4) { r.err = true; break; }
        uint32_t ne = 1;  // the reference multiplies uint dims in 32-bit arithmetic
        for (uint32_t d = 0; d < t.n_dims; d++) {
            t.dims[d] = (uint32_t)r.n(8);
            ne *= (uint32_t)t.dims[d];
        }
        t.n_elems = t.n_dims ? ne : 0;
        t.type = (uint32_t)r.n(4);
        t.offset = r.n(8);
        out->tensors.push_back(std::move(t));
    }
    if (r.err) return bad("truncated GGUF header");
    const Value *al = meta.get("general.alignment");
    uint64_t alignment = Meta::numeric(al) ? (uint64_t)al->num : 32;
    if (alignment == 0) return bad("bad general.alignment");
    uint64_t data_off = (uint64_t)(r.p - base);
    data_off += (alignment - data_off % alignment) % alignment;
    for (auto &t : out->tensors) {
        if (block_elems(t.type) == 0) return bad("Unsupported GGML type: " + std::to_string(t.type));
        t.n_bytes = row_bytes(t.type, t.n_elems);
        // overflow-safe form of data_off + offset + n_bytes > file size: a crafted offset must not
        // wrap around and point the tensor outside the mapping
        const uint64_t size = out->size;
        if (t.n_bytes == 0 || data_off > size || t.offset > size - data_off || t.n_bytes > size - data_off - t.offset)
            continue;
        t.data = base + data_off + t.offset;
    }

    // ---- ArchitectureResolver.Resolve
    const Value *a = meta.get("general.architecture");
    if (!a || a->type != V_STR || a->str.empty()) return bad("GGUF model missing 'general.architecture' metadata key.");
    meta.arch = a->str;
    static const char *sup[] = {"llama", "phi3", "qwen2", "phi2", "gptneox", "gemma", "gemma2", "stablelm", "lfm2", "lfm2_moe"};
    bool ok = false;
    for (const char *s : sup) ok |= strcasecmp(s, meta.arch.c_str()) == 0;
    if (!ok) return bad("Unsupported GGUF architecture: '" + meta.arch + "'");
    llmdot_config &c = out->cfg;
    memset(&c, 0, sizeof c);
    const char *A = meta.arch.c_str();
    if (!strcasecmp(A, "phi2") || !strcasecmp(A, "gptneox")) c.template_id = 1;
    else if (!strcasecmp(A, "gemma") || !strcasecmp(A, "gemma2")) c.template_id = 2;
    else if (!strcasecmp(A, "lfm2") || !strcasecmp(A, "lfm2_moe")) c.template_id = 3;
    else c.template_id = 0;
    c.hidden = meta.geti("embedding_length", 0);
    c.layers = meta.geti("block_count", 0);
    c.context = meta.geti("context_length", 0);
    c.ffn = meta.geti("feed_forward_length", 0);
    c.heads = meta.geti("attention.head_count", 0);
    const Value *hkv = meta.arch_get("attention.head_count_kv");
    if (hkv && hkv->type == V_ARR && !hkv->arr_num.empty()) {
        int mx = 0;
        for (double d : hkv->arr_num) mx = std::max(mx, (int)nearbyint(d));
        c.heads_kv = mx;
    } else c.heads_kv = meta.geti("attention.head_count_kv", c.heads);
    c.head_dim = meta.geti("attention.key_length", c.hidden / std::max(c.heads, 1));
    const Value *toks = meta.get("tokenizer.ggml.tokens");
    c.vocab = (toks && toks->type == V_ARR) ? (int)toks->arr_n : 0;
    bool present = false;
    c.eps = meta.getf("attention.layer_norm_rms_epsilon", 0, &present);
    if (present) c.norm_is_rms = 1;
    else {
        c.eps = meta.getf("attention.layer_norm_epsilon", 0, &present);
        if (!present) return bad("No norm epsilon found for architecture '" + meta.arch + "'.");
    }
    c.rope_base = meta.getf("rope.freq_base", 10000.0f);
    c.rope_dim = meta.geti("rope.dimension_count", c.head_dim);
    const Value *rs = meta.arch_get("rope.scaling.type");
    c.rope_scaling = 0;
    if (rs && rs->type == V_STR) {
        if (!strcasecmp(rs->str.c_str(), "linear")) c.rope_scaling = 1;
        else if (!strcasecmp(rs->str.c_str(), "yarn")) c.rope_scaling = 2;
        else if (!strcasecmp(rs->str.c_str(), "longrope")) c.rope_scaling = 3;
    }
    c.rope_factor = meta.getf("rope.scaling.factor", 1.0f);
    bool fused = false, gate = false, post = false, outw = false;
    for (auto &t : out->tensors) {
        fused |= t.name.find("attn_qkv") != std::string::npos;
        gate |= t.name.find("ffn_gate") != std::string::npos;
        post |= t.name.find("post_attention_norm") != std::string::npos || t.name.find("post_ffw_norm") != std::string::npos;
        outw |= t.name == "output.weight";
    }
    c.qkv_fused = fused;
    c.ffn_type = gate ? (c.template_id == 2 ? 2 : 1) : 0;
    const Value *pr = meta.arch_get("use_parallel_residual");
    c.parallel_residual = Meta::numeric(pr) ? (pr->num != 0) : (c.template_id == 1);
    c.tied = !outw;
    bool es = false;
    float esv = meta.getf("embedding_scale", 0, &es);
    c.emb_scale = es ? esv : (c.template_id == 2 ? sqrtf((float)c.hidden) : 1.0f);
    c.has_post_norm = post;
    c.sliding_window = meta.geti("attention.sliding_window", 0);
    c.attn_cap = meta.getf("attn_logit_softcapping", 0, &present);
    c.has_attn_cap = present;
    c.final_cap = meta.getf("final_logit_softcapping", 0, &present);
    c.has_final_cap = present;
    c.expert_count = meta.geti("expert_count", 0);
    const Value *b = meta.get("tokenizer.ggml.bos_token_id"), *e = meta.get("tokenizer.ggml.eos_token_id");
    c.bos = Meta::numeric(b) ? (int)nearbyint(b->num) : 1;
    c.eos = Meta::numeric(e) ? (int)nearbyint(e->num) : 2;
    return LLMDOT_OK;
}

void gguf_descs(const GgufModelFile &f, std::vector<llmdot_tensor_desc> *out)
{
    out->clear();
    for (auto &t : f.tensors) {
        if (!t.data) continue;
        llmdot_tensor_desc d;
        memset(&d, 0, sizeof d);
        d.name = t.name.c_str();
        d.type = t.type;
        d.n_dims = t.n_dims;
        for (int i = 0; i < 4; i++) d.dims[i] = t.dims[i];
        d.data = t.data;
        d.n_bytes = t.n_bytes;
        out->push_back(d);
    }
}

void gguf_close(GgufModelFile *f)
{
    if (f->map) munmap(f->map, f->size);
    f->map = nullptr;
    f->size = 0;
    f->tensors.clear();
}

}  // namespace llmdot
