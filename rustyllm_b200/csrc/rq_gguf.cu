// rq_gguf.cu -- GGUF files straight to the device: the per-layer shard
// reader of the reference (GgufLayer, src/streaming_quantized.rs:42-91,
// which slurps a file and slices tensors out of the buffer) and the shard
// directory layout its loader walks (StreamingLlamaQuantized::
// from_pretrained, src/streaming_quantized.rs:451-501: model.layers.N.gguf,
// model.embed_tokens.gguf, model.norm.gguf, lm_head.gguf; tensor names of
// QBlock::load / QAttn::load / QMlp::load, :170-178, :266-273, :291-294).
//
// GGUF (the format the reference's writer emits through candle's
// gguf_file::write, src/quantize.rs:146-150): little-endian "GGUF", version
// (2 or 3), tensor count and metadata count (u64), metadata key/value pairs,
// tensor infos (name, dims innermost first, ggml type, offset), then the data
// section at the next multiple of general.alignment (default 32).  Every
// read is bounds-checked: a short or malformed file is RQ_ERR_INVALID with a
// message, never a crash.  Host code only.

#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "rq_internal.cuh"

struct rq_gguf {
    struct Tensor {
        std::string name;
        int type;
        int n_dims;
        int64_t dims[4];
        uint64_t offset;  // in the file
        uint64_t nbytes;  // 0 for a type without a known size
    };
    std::vector<uint8_t> buf;
    std::vector<Tensor> tensors;
    uint32_t version = 0, alignment = 32;
};

namespace rq {
namespace {

// (elements, bytes) per block of a ggml type; {0, 0} if unknown
struct TypeSize {
    int elems, bytes;
};
TypeSize ggml_type_size(int t) {
    switch (t) {
        case 0: return {1, 4};      // F32
        case 1: return {1, 2};      // F16
        case 2: return {32, 18};    // Q4_0
        case 3: return {32, 20};    // Q4_1
        case 6: return {32, 22};    // Q5_0
        case 7: return {32, 24};    // Q5_1
        case 8: return {32, 34};    // Q8_0
        case 9: return {32, 36};    // Q8_1
        case 10: return {256, 84};  // Q2_K
        case 11: return {256, 110}; // Q3_K
        case 12: return {256, 144}; // Q4_K
        case 13: return {256, 176}; // Q5_K
        case 14: return {256, 210}; // Q6_K
        case 15: return {256, 292}; // Q8_K
        case 24: return {1, 1};     // I8
        case 25: return {1, 2};     // I16
        case 26: return {1, 4};     // I32
        case 27: return {1, 8};     // I64
        case 28: return {1, 8};     // F64
        case 30: return {1, 2};     // BF16
        default: return {0, 0};
    }
}

struct Cursor {
    const uint8_t* p;
    size_t n, pos = 0;
    bool ok = true;
    bool take(void* dst, size_t k) {
        if (!ok || k > n - pos) {
            ok = false;
            return false;
        }
        memcpy(dst, p + pos, k);
        pos += k;
        return true;
    }
    bool skip(uint64_t k) {
        if (!ok || k > n - pos) {
            ok = false;
            return false;
        }
        pos += (size_t)k;
        return true;
    }
    template <typename T>
    T get() {
        T v{};
        take(&v, sizeof v);
        return v;
    }
    bool str(std::string* s) {
        const uint64_t len = get<uint64_t>();
        if (!ok || len > n - pos) {
            ok = false;
            return false;
        }
        if (s) s->assign(reinterpret_cast<const char*>(p + pos), (size_t)len);
        pos += (size_t)len;
        return true;
    }
};

size_t kv_scalar_bytes(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;  // u8, i8, bool
        case 2: case 3: return 2;          // u16, i16
        case 4: case 5: case 6: return 4;  // u32, i32, f32
        case 10: case 11: case 12: return 8;  // u64, i64, f64
        default: return 0;
    }
}

// Skips one metadata value of type t; reads general.alignment on the way.
bool skip_value(Cursor& c, uint32_t t, int depth) {
    if (depth > 4) return false;
    if (t == 8) return c.str(nullptr);
    if (t == 9) {
        const uint32_t et = c.get<uint32_t>();
        const uint64_t count = c.get<uint64_t>();
        if (!c.ok) return false;
        const size_t sb = kv_scalar_bytes(et);
        if (sb) return count <= (c.n - c.pos) / sb && c.skip(count * sb);
        for (uint64_t i = 0; i < count && c.ok; i++) skip_value(c, et, depth + 1);
        return c.ok;
    }
    const size_t sb = kv_scalar_bytes(t);
    return sb ? c.skip(sb) : (c.ok = false);
}

int parse(rq_gguf* f) {
    Cursor c{f->buf.data(), f->buf.size()};
    const uint32_t magic = c.get<uint32_t>();
    f->version = c.get<uint32_t>();
    if (!c.ok || magic != 0x46554747u) return set_error(RQ_ERR_INVALID, "gguf: not a GGUF file (magic)");
    if (f->version != 2 && f->version != 3)
        return set_error(RQ_ERR_UNSUPPORTED, "gguf: version %u (2 and 3 are supported)", f->version);
    const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
    if (!c.ok || nt > (1u << 24) || nkv > (1u << 24)) return set_error(RQ_ERR_INVALID, "gguf: bad header counts");
    for (uint64_t i = 0; i < nkv; i++) {
        std::string key;
        c.str(&key);
        const uint32_t t = c.get<uint32_t>();
        if (!c.ok) break;
        if (key == "general.alignment" && t == 4) {
            f->alignment = c.get<uint32_t>();
            if (f->alignment == 0 || (f->alignment & (f->alignment - 1)))
                return set_error(RQ_ERR_INVALID, "gguf: general.alignment %u is not a power of two", f->alignment);
        } else if (!skip_value(c, t, 0)) {
            break;
        }
    }
    if (!c.ok) return set_error(RQ_ERR_INVALID, "gguf: truncated or malformed metadata");
    f->tensors.resize((size_t)nt);
    for (auto& t : f->tensors) {
        c.str(&t.name);
        t.n_dims = (int)c.get<uint32_t>();
        if (!c.ok || t.n_dims < 1 || t.n_dims > 4)
            return set_error(RQ_ERR_INVALID, "gguf: tensor '%s': %d dimensions", t.name.c_str(), t.n_dims);
        for (int d = 0; d < 4; d++) t.dims[d] = 1;
        for (int d = 0; d < t.n_dims; d++) {
            const uint64_t v = c.get<uint64_t>();
            if (v == 0 || v > (1ull << 40)) c.ok = false;
            t.dims[d] = (int64_t)v;
        }
        t.type = (int)c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        if (!c.ok) return set_error(RQ_ERR_INVALID, "gguf: truncated or malformed tensor infos");
    }
    const uint64_t data0 = ((uint64_t)c.pos + f->alignment - 1) / f->alignment * f->alignment;
    for (auto& t : f->tensors) {
        const TypeSize ts = ggml_type_size(t.type);
        t.nbytes = 0;
        uint64_t ne = 1;
        for (int d = 0; d < 4; d++) {
            if ((uint64_t)t.dims[d] > (1ull << 62) / ne)
                return set_error(RQ_ERR_INVALID, "gguf: tensor '%s': too many elements", t.name.c_str());
            ne *= (uint64_t)t.dims[d];
        }
        if (t.offset > f->buf.size())
            return set_error(RQ_ERR_INVALID, "gguf: tensor '%s' lies past the end of the file", t.name.c_str());
        if (ts.elems > 0) {
            if (t.dims[0] % ts.elems)
                return set_error(RQ_ERR_INVALID, "gguf: tensor '%s': row of %lld is not whole blocks of %d",
                                 t.name.c_str(), (long long)t.dims[0], ts.elems);
            t.nbytes = ne / (uint64_t)ts.elems * (uint64_t)ts.bytes;
        }
        t.offset += data0;
        if (t.offset > f->buf.size() || t.nbytes > f->buf.size() - t.offset)
            return set_error(RQ_ERR_INVALID, "gguf: tensor '%s' lies past the end of the file", t.name.c_str());
    }
    return RQ_OK;
}

const rq_gguf::Tensor* find(const rq_gguf* f, const char* name) {
    for (const auto& t : f->tensors)
        if (t.name == name) return &t;
    return nullptr;
}

float f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else {  // subnormal: normalise
            int ee = -1;
            uint32_t mm = m;
            do {
                mm <<= 1;
                ee++;
            } while (!(mm & 1024u));
            bits = s | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 1023u) << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7F800000u | (m << 13);
    } else {
        bits = s | ((e + 112u) << 23) | (m << 13);
    }
    float v;
    memcpy(&v, &bits, 4);
    return v;
}

// f32 -> f16 bits, round to nearest even (the conversion numpy's astype uses)
uint16_t f32_to_f16(float v) {
    uint32_t x;
    memcpy(&x, &v, 4);
    const uint32_t s = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(s | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(s | 0x7C00u);  // rounds to infinity
    if (ax < 0x38800000u) {                                  // f16 subnormal or zero
        if (ax < 0x33000000u) return (uint16_t)s;
        const uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126u - e;  // 14 + (113 - e) - 1
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(s | r);
    }
    uint32_t r = ((ax - 0x38000000u) >> 13);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(s | r);
}

int read_f32(const rq_gguf* f, const rq_gguf::Tensor& t, int64_t first, int64_t count, float* out) {
    const uint8_t* p = f->buf.data() + t.offset;
    const int64_t ne = t.dims[0] * t.dims[1] * t.dims[2] * t.dims[3];
    if (first < 0 || count < 0 || first + count > ne)
        return set_error(RQ_ERR_INVALID, "gguf: elements [%lld, %lld) of '%s' (%lld)", (long long)first,
                         (long long)(first + count), t.name.c_str(), (long long)ne);
    for (int64_t i = 0; i < count; i++) {
        const int64_t k = first + i;
        if (t.type == 0) {
            memcpy(out + i, p + 4 * k, 4);
        } else if (t.type == 1) {
            uint16_t h;
            memcpy(&h, p + 2 * k, 2);
            out[i] = f16_to_f32(h);
        } else if (t.type == 30) {
            uint16_t h;
            memcpy(&h, p + 2 * k, 2);
            const uint32_t bits = (uint32_t)h << 16;
            memcpy(out + i, &bits, 4);
        } else {
            return set_error(RQ_ERR_UNSUPPORTED, "gguf: '%s' has ggml type %d, not F32/F16/BF16", t.name.c_str(),
                             t.type);
        }
    }
    return RQ_OK;
}

int read_f16(const rq_gguf* f, const rq_gguf::Tensor& t, int64_t first, int64_t count, uint16_t* out) {
    if (t.type == 1) {
        const int64_t ne = t.dims[0] * t.dims[1] * t.dims[2] * t.dims[3];
        if (first < 0 || count < 0 || first + count > ne)
            return set_error(RQ_ERR_INVALID, "gguf: elements [%lld, %lld) of '%s'", (long long)first,
                             (long long)(first + count), t.name.c_str());
        memcpy(out, f->buf.data() + t.offset + 2 * first, (size_t)count * 2);
        return RQ_OK;
    }
    std::vector<float> tmp((size_t)count);
    int rc = read_f32(f, t, first, count, tmp.data());
    for (int64_t i = 0; i < count && !rc; i++) out[i] = f32_to_f16(tmp[(size_t)i]);
    return rc;
}

// Blocks of rows [row0, row0 + rows) x columns [col0, col0 + cols) of a 2-D
// block-quantized tensor, gathered into one [rows][cols / block] buffer.
int gather_blocks(const rq_gguf* f, const rq_gguf::Tensor& t, int64_t row0, int64_t rows, int64_t col0, int64_t cols,
                  std::vector<uint8_t>& out) {
    const TypeSize ts = ggml_type_size(t.type);
    const int64_t in = t.dims[0], nout = t.dims[1];
    if (t.n_dims != 2 || ts.elems <= 1)
        return set_error(RQ_ERR_INVALID, "gguf: '%s' is not a 2-D block-quantized matrix", t.name.c_str());
    if (row0 < 0 || rows <= 0 || row0 + rows > nout || col0 < 0 || cols <= 0 || col0 + cols > in ||
        col0 % ts.elems || cols % ts.elems)
        return set_error(RQ_ERR_INVALID, "gguf: '%s' [%lld x %lld]: slice rows %lld+%lld, cols %lld+%lld", t.name.c_str(),
                         (long long)nout, (long long)in, (long long)row0, (long long)rows, (long long)col0,
                         (long long)cols);
    const size_t rowb = (size_t)(in / ts.elems) * ts.bytes, segb = (size_t)(cols / ts.elems) * ts.bytes;
    const size_t off = (size_t)(col0 / ts.elems) * ts.bytes;
    out.resize(segb * (size_t)rows);
    const uint8_t* p = f->buf.data() + t.offset;
    for (int64_t r = 0; r < rows; r++) memcpy(out.data() + segb * (size_t)r, p + rowb * (size_t)(row0 + r) + off, segb);
    return RQ_OK;
}

int open_file(const char* path, rq_gguf** out) {
    FILE* fp = fopen(path, "rb");
    if (!fp) return set_error(RQ_ERR_INVALID, "gguf: cannot open '%s'", path);
    rq_gguf* f = new rq_gguf();
    fseek(fp, 0, SEEK_END);
    const long len = ftell(fp);
    fseek(fp, 0, SEEK_SET);
    int rc = RQ_OK;
    if (len < 0) {
        rc = set_error(RQ_ERR_INVALID, "gguf: cannot size '%s'", path);
    } else {
        // one sequential read of the whole file, as GgufLayer::open does
        f->buf.resize((size_t)len);
        if (len > 0 && fread(f->buf.data(), 1, (size_t)len, fp) != (size_t)len)
            rc = set_error(RQ_ERR_INVALID, "gguf: short read of '%s'", path);
    }
    fclose(fp);
    if (!rc) rc = parse(f);
    if (rc) {
        delete f;
        return rc;
    }
    *out = f;
    return RQ_OK;
}

}  // namespace

// Loads the reference's shard directory into m (this rank's shards under
// tensor parallelism); the weights it uploads belong to m.
int llama_load_gguf_dir(rq_ctx* ctx, rq_llama* m, const char* dir, int64_t n_layers, int64_t vocab, int64_t hidden,
                        int world, int rank, const int64_t* dims7_out, const int64_t* dims7_in,
                        std::vector<rq_weight*>& owned) {
    static const char* kNames[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                    "mlp.gate_proj",    "mlp.up_proj",      "mlp.down_proj"};
    static const bool kRowParallel[7] = {false, false, false, true, false, false, true};
    const std::string d(dir);
    for (int64_t l = 0; l < n_layers; l++) {
        const std::string path = d + "/model.layers." + std::to_string(l) + ".gguf";
        rq_gguf* f = nullptr;
        int rc = open_file(path.c_str(), &f);
        if (rc) return rc;
        rq_weight* w7[7] = {};
        std::vector<float> r1((size_t)hidden), r2((size_t)hidden);
        const std::string p = "model.layers." + std::to_string(l) + ".";
        for (int k = 0; k < 7 && !rc; k++) {
            const std::string name = p + kNames[k] + ".weight";
            const rq_gguf::Tensor* t = find(f, name.c_str());
            if (!t) {
                rc = set_error(RQ_ERR_INVALID, "gguf: '%s' has no tensor '%s'", path.c_str(), name.c_str());
                break;
            }
            // full [out, in] of the model; this rank keeps rows (column-
            // parallel) or columns (row-parallel) of it
            const int64_t out_full = dims7_out[k] * (kRowParallel[k] ? 1 : world);
            const int64_t in_full = dims7_in[k] * (kRowParallel[k] ? world : 1);
            if (t->n_dims != 2 || t->dims[0] != in_full || t->dims[1] != out_full) {
                rc = set_error(RQ_ERR_INVALID, "gguf: '%s' is [%lld, %lld], the config needs [%lld, %lld]", name.c_str(),
                               (long long)t->dims[1], (long long)t->dims[0], (long long)out_full, (long long)in_full);
                break;
            }
            const int64_t o = dims7_out[k], i = dims7_in[k];
            std::vector<uint8_t> blocks;
            rc = kRowParallel[k] ? gather_blocks(f, *t, 0, o, (int64_t)rank * i, i, blocks)
                                 : gather_blocks(f, *t, (int64_t)rank * o, o, 0, i, blocks);
            if (!rc) rc = rq_weight_upload(ctx, t->type, blocks.data(), blocks.size(), o, i, &w7[k]);
            if (!rc) owned.push_back(w7[k]);
        }
        for (int k = 0; k < 2 && !rc; k++) {
            const std::string name = p + (k == 0 ? "input_layernorm.weight" : "post_attention_layernorm.weight");
            const rq_gguf::Tensor* t = find(f, name.c_str());
            if (!t || t->dims[0] * t->dims[1] * t->dims[2] * t->dims[3] != hidden)
                rc = set_error(RQ_ERR_INVALID, "gguf: '%s': missing or not %lld elements", name.c_str(), (long long)hidden);
            else
                rc = read_f32(f, *t, 0, hidden, k == 0 ? r1.data() : r2.data());
        }
        delete f;
        if (!rc) rc = rq_llama_set_layer(m, l, w7, r1.data(), r2.data());
        if (rc) return rc;
    }
    // embedding (full vocab), final norm, lm_head (this rank's vocab rows);
    // without lm_head.gguf the head is the embedding (tied)
    std::vector<uint16_t> emb((size_t)(vocab * hidden));
    {
        rq_gguf* f = nullptr;
        int rc = open_file((d + "/model.embed_tokens.gguf").c_str(), &f);
        if (rc) return rc;
        const rq_gguf::Tensor* t = find(f, "model.embed_tokens.weight");
        if (!t || t->dims[0] != hidden || t->dims[1] != vocab)
            rc = set_error(RQ_ERR_INVALID, "gguf: model.embed_tokens.weight missing or not [%lld, %lld]",
                           (long long)vocab, (long long)hidden);
        if (!rc) rc = read_f16(f, *t, 0, vocab * hidden, emb.data());
        delete f;
        if (!rc) rc = rq_llama_set_embedding(m, emb.data());
        if (rc) return rc;
    }
    std::vector<float> lnf((size_t)hidden);
    {
        rq_gguf* f = nullptr;
        int rc = open_file((d + "/model.norm.gguf").c_str(), &f);
        if (rc) return rc;
        const rq_gguf::Tensor* t = find(f, "model.norm.weight");
        if (!t || t->dims[0] * t->dims[1] * t->dims[2] * t->dims[3] != hidden)
            rc = set_error(RQ_ERR_INVALID, "gguf: model.norm.weight missing or not %lld elements", (long long)hidden);
        if (!rc) rc = read_f32(f, *t, 0, hidden, lnf.data());
        delete f;
        if (rc) return rc;
    }
    const int64_t vl = vocab / world;
    std::vector<uint16_t> head((size_t)(vl * hidden));
    const std::string hp = d + "/lm_head.gguf";
    FILE* probe = fopen(hp.c_str(), "rb");
    if (probe) {
        fclose(probe);
        rq_gguf* f = nullptr;
        int rc = open_file(hp.c_str(), &f);
        if (rc) return rc;
        const rq_gguf::Tensor* t = find(f, "lm_head.weight");
        if (!t || t->dims[0] != hidden || t->dims[1] != vocab)
            rc = set_error(RQ_ERR_INVALID, "gguf: lm_head.weight missing or not [%lld, %lld]", (long long)vocab,
                           (long long)hidden);
        if (!rc) rc = read_f16(f, *t, (int64_t)rank * vl * hidden, vl * hidden, head.data());
        delete f;
        if (rc) return rc;
    } else {
        memcpy(head.data(), emb.data() + (size_t)rank * vl * hidden, head.size() * 2);
    }
    return rq_llama_set_head(m, lnf.data(), head.data());
}

}  // namespace rq

using namespace rq;

extern "C" {

int rq_gguf_open(const char* path, rq_gguf** out) {
    if (!path || !out) return set_error(RQ_ERR_INVALID, "rq_gguf_open: NULL argument");
    *out = nullptr;
    return open_file(path, out);
}

int rq_gguf_open_memory(const void* data, size_t nbytes, rq_gguf** out) {
    if (!data || !out) return set_error(RQ_ERR_INVALID, "rq_gguf_open_memory: NULL argument");
    *out = nullptr;
    rq_gguf* f = new rq_gguf();
    f->buf.assign((const uint8_t*)data, (const uint8_t*)data + nbytes);
    int rc = parse(f);
    if (rc) {
        delete f;
        return rc;
    }
    *out = f;
    return RQ_OK;
}

int rq_gguf_free(rq_gguf* f) {
    delete f;
    return RQ_OK;
}

int rq_gguf_tensor_count(const rq_gguf* f, int64_t* count) {
    if (!f || !count) return set_error(RQ_ERR_INVALID, "rq_gguf_tensor_count: NULL argument");
    *count = (int64_t)f->tensors.size();
    return RQ_OK;
}

int rq_gguf_find(const rq_gguf* f, const char* name, int64_t* index) {
    if (!f || !name || !index) return set_error(RQ_ERR_INVALID, "rq_gguf_find: NULL argument");
    for (size_t i = 0; i < f->tensors.size(); i++)
        if (f->tensors[i].name == name) {
            *index = (int64_t)i;
            return RQ_OK;
        }
    *index = -1;
    return set_error(RQ_ERR_INVALID, "gguf: no tensor '%s'", name);
}

int rq_gguf_tensor_info(const rq_gguf* f, int64_t index, char* name, size_t name_cap, int* ggml_type, int* n_dims,
                        int64_t* dims, uint64_t* file_offset, uint64_t* nbytes) {
    if (!f) return set_error(RQ_ERR_INVALID, "rq_gguf_tensor_info: NULL file");
    if (index < 0 || index >= (int64_t)f->tensors.size())
        return set_error(RQ_ERR_INVALID, "rq_gguf_tensor_info: index %lld of %zu", (long long)index, f->tensors.size());
    const rq_gguf::Tensor& t = f->tensors[(size_t)index];
    if (name && name_cap) {
        const size_t k = std::min(name_cap - 1, t.name.size());
        memcpy(name, t.name.data(), k);
        name[k] = 0;
    }
    if (ggml_type) *ggml_type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (dims)
        for (int d = 0; d < 4; d++) dims[d] = t.dims[d];
    if (file_offset) *file_offset = t.offset;
    if (nbytes) *nbytes = t.nbytes;
    return RQ_OK;
}

int rq_gguf_tensor_data(const rq_gguf* f, int64_t index, const void** data, uint64_t* nbytes) {
    if (!f || !data) return set_error(RQ_ERR_INVALID, "rq_gguf_tensor_data: NULL argument");
    if (index < 0 || index >= (int64_t)f->tensors.size())
        return set_error(RQ_ERR_INVALID, "rq_gguf_tensor_data: index %lld of %zu", (long long)index, f->tensors.size());
    const rq_gguf::Tensor& t = f->tensors[(size_t)index];
    if (!t.nbytes) return set_error(RQ_ERR_UNSUPPORTED, "gguf: '%s': unknown ggml type %d", t.name.c_str(), t.type);
    *data = f->buf.data() + t.offset;
    if (nbytes) *nbytes = t.nbytes;
    return RQ_OK;
}

int rq_gguf_read_f32(const rq_gguf* f, const char* name, float* out, int64_t count) {
    if (!f || !name || !out) return set_error(RQ_ERR_INVALID, "rq_gguf_read_f32: NULL argument");
    const rq_gguf::Tensor* t = find(f, name);
    if (!t) return set_error(RQ_ERR_INVALID, "gguf: no tensor '%s'", name);
    return read_f32(f, *t, 0, count, out);
}

int rq_weight_upload_gguf(rq_ctx* ctx, const rq_gguf* f, const char* name, int64_t row0, int64_t rows, int64_t col0,
                          int64_t cols, rq_weight** out) {
    if (!ctx || !f || !name || !out) return set_error(RQ_ERR_INVALID, "rq_weight_upload_gguf: NULL argument");
    const rq_gguf::Tensor* t = find(f, name);
    if (!t) return set_error(RQ_ERR_INVALID, "gguf: no tensor '%s'", name);
    if (t->n_dims == 2) {
        if (rows < 0) rows = t->dims[1] - row0;
        if (cols < 0) cols = t->dims[0] - col0;
    }
    std::vector<uint8_t> blocks;
    int rc = gather_blocks(f, *t, row0, rows, col0, cols, blocks);
    if (!rc) rc = rq_weight_upload(ctx, t->type, blocks.data(), blocks.size(), rows, cols, out);
    return rc;
}

}  // extern "C"
