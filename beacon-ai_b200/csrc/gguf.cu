// gguf.cu -- GGUF v3 files: parse, and load a decoder's weights to the device.
//
// The parser follows crates/beacon-format/src/gguf: the 24-byte header
// (header.rs: magic "GGUF", version 3, tensor and metadata counts), the typed
// metadata key-value pairs (metadata.rs, types.rs), the tensor infos with
// their dims reversed to row-major (tensor_info.rs:40-48) and their data
// offsets resolved against the data section, which starts at the next
// multiple of general.alignment (default 32) after the infos
// (tensor_info.rs:80-125). The file is memory-mapped and tensor bytes are
// read in place, as GgufFile::tensor_data does (mod.rs:79-84).
//
// Loading maps the GGUF tensor names of a Llama-style decoder
// (crates/beacon-core/src/weights.rs:116-166: token_embd, output_norm,
// output, blk.N.attn_norm / attn_q / attn_k / attn_v / attn_output /
// ffn_norm / ffn_gate / ffn_up / ffn_down) to the model's weight slots.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "internal.h"
#include "kernels.h"

namespace {

using bc::fail;
using bc::invalid;

// GGUF tensor type ids (types.rs:8-29) -> BeaconDtype tags; -1: not loadable.
int32_t dtype_of_gguf_type(uint32_t t) {
    switch (t) {
        case 0: return BEACON_CUDA_DTYPE_F32;
        case 1: return BEACON_CUDA_DTYPE_F16;
        case 2: return BEACON_CUDA_DTYPE_Q4_0;
        case 3: return BEACON_CUDA_DTYPE_Q4_1;
        case 6: return BEACON_CUDA_DTYPE_Q5_0;
        case 7: return BEACON_CUDA_DTYPE_Q5_1;
        case 8: return BEACON_CUDA_DTYPE_Q8_0;
        case 10: return BEACON_CUDA_DTYPE_Q2_K;
        case 11: return BEACON_CUDA_DTYPE_Q3_K;
        case 12: return BEACON_CUDA_DTYPE_Q4_K;
        case 13: return BEACON_CUDA_DTYPE_Q5_K;
        case 14: return BEACON_CUDA_DTYPE_Q6_K;
        case 15: return BEACON_CUDA_DTYPE_Q8_K;
        case 24: return BEACON_CUDA_DTYPE_I8;
        case 26: return BEACON_CUDA_DTYPE_I32;
        case 30: return BEACON_CUDA_DTYPE_BF16;
        default: return -1;  // Q8_1, I16, I64, F64 have no BeaconDtype (types.rs:59-79)
    }
}

// (block size, bytes per block) of a GGUF tensor type (types.rs:82-121).
bool gguf_type_geometry(uint32_t t, uint64_t& bs, uint64_t& bb) {
    switch (t) {
        case 0: bs = 1; bb = 4; return true;
        case 1: case 30: case 25: bs = 1; bb = 2; return true;
        case 24: bs = 1; bb = 1; return true;
        case 26: bs = 1; bb = 4; return true;
        case 27: case 28: bs = 1; bb = 8; return true;
        case 2: bs = 32; bb = 18; return true;
        case 3: bs = 32; bb = 20; return true;
        case 6: bs = 32; bb = 22; return true;
        case 7: bs = 32; bb = 24; return true;
        case 8: bs = 32; bb = 34; return true;
        case 9: bs = 32; bb = 40; return true;
        case 10: bs = 256; bb = 84; return true;
        case 11: bs = 256; bb = 110; return true;
        case 12: bs = 256; bb = 144; return true;
        case 13: bs = 256; bb = 176; return true;
        case 14: bs = 256; bb = 210; return true;
        case 15: bs = 256; bb = 292; return true;
        default: return false;
    }
}

struct Value {
    uint32_t type = 0;      // GgufMetaType (types.rs:124-158)
    int64_t i = 0;          // integers and bools
    double f = 0.0;         // floats
    std::string s;          // strings
    uint32_t elem_type = 0; // arrays
    uint64_t count = 0;
    std::vector<int64_t> ints;  // integer arrays
};

struct Tensor {
    std::string name;
    uint32_t gguf_type = 0;
    int32_t dtype = -1;
    std::vector<int64_t> shape;  // row-major (reversed GGUF dims)
    uint64_t offset = 0;         // absolute
    uint64_t length = 0;
};

struct Reader {
    const uint8_t* p;
    size_t n, pos;
    void need(size_t k) {
        if (pos + k > n || pos + k < pos)
            bc::shape_err("gguf: truncated file (needed " + std::to_string(k) + " bytes at offset " +
                          std::to_string(pos) + " of " + std::to_string(n) + ")");
    }
    template <typename T>
    T rd() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p + pos, sizeof(T));
        pos += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t len = rd<uint64_t>();
        need((size_t)len);
        std::string s(reinterpret_cast<const char*>(p + pos), (size_t)len);
        pos += (size_t)len;
        return s;
    }
};

// metadata.rs:95-130 (read_value)
void read_value(Reader& r, uint32_t type, Value& v, int depth) {
    v.type = type;
    switch (type) {
        case 0: v.i = r.rd<uint8_t>(); break;
        case 1: v.i = r.rd<int8_t>(); break;
        case 2: v.i = r.rd<uint16_t>(); break;
        case 3: v.i = r.rd<int16_t>(); break;
        case 4: v.i = r.rd<uint32_t>(); break;
        case 5: v.i = r.rd<int32_t>(); break;
        case 6: v.f = r.rd<float>(); break;
        case 7: v.i = r.rd<uint8_t>() != 0; break;
        case 8: v.s = r.str(); break;
        case 9: {
            if (depth > 4) invalid("gguf: arrays nested too deeply");
            v.elem_type = r.rd<uint32_t>();
            if (v.elem_type > 12) invalid("gguf: unknown array element type " + std::to_string(v.elem_type));
            v.count = r.rd<uint64_t>();
            for (uint64_t k = 0; k < v.count; ++k) {
                Value e;
                read_value(r, v.elem_type, e, depth + 1);
                if (e.type <= 5 || e.type == 7 || e.type == 10 || e.type == 11) v.ints.push_back(e.i);
            }
            break;
        }
        case 10: {
            const uint64_t u = r.rd<uint64_t>();
            v.i = (int64_t)u;
            break;
        }
        case 11: v.i = r.rd<int64_t>(); break;
        case 12: v.f = r.rd<double>(); break;
        default: invalid("gguf: unknown metadata value type " + std::to_string(type));
    }
}

}  // namespace

struct BeaconCudaGguf {
    int fd = -1;
    void* map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    std::map<std::string, Value> meta;
    std::vector<Tensor> tensors;
    ~BeaconCudaGguf() {
        if (map && map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) close(fd);
    }
    const Value* get(const char* key) const {
        auto it = meta.find(key);
        return it == meta.end() ? nullptr : &it->second;
    }
};

namespace {

bool as_int(const Value* v, int64_t& out) {
    if (!v) return false;
    if (v->type <= 5 || v->type == 7 || v->type == 10 || v->type == 11) {
        out = v->i;
        return true;
    }
    return false;
}

bool as_float(const Value* v, double& out) {
    if (!v) return false;
    if (v->type == 6 || v->type == 12) {
        out = v->f;
        return true;
    }
    return false;
}

void parse(BeaconCudaGguf& f) {
    Reader r{static_cast<const uint8_t*>(f.map), f.size, 0};
    // header.rs:17-47
    r.need(24);
    if (std::memcmp(r.p, "GGUF", 4) != 0) invalid("gguf: invalid magic (not a GGUF file)");
    r.pos = 4;
    f.version = r.rd<uint32_t>();
    if (f.version != 3)
        bc::fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "gguf: unsupported version " + std::to_string(f.version));
    const uint64_t tensor_count = r.rd<uint64_t>();
    const uint64_t kv_count = r.rd<uint64_t>();
    // metadata.rs:133-151
    for (uint64_t k = 0; k < kv_count; ++k) {
        std::string key = r.str();
        const uint32_t vt = r.rd<uint32_t>();
        if (vt > 12) invalid("gguf: unknown metadata value type " + std::to_string(vt) + " for key " + key);
        Value v;
        read_value(r, vt, v, 0);
        f.meta[key] = std::move(v);
    }
    // tensor_info.rs:13-77
    if (tensor_count > (1u << 24)) invalid("gguf: implausible tensor count");
    for (uint64_t k = 0; k < tensor_count; ++k) {
        Tensor t;
        t.name = r.str();
        const uint32_t ndim = r.rd<uint32_t>();
        if (ndim > 8) invalid("gguf: tensor " + t.name + " has too many dimensions");
        std::vector<uint64_t> dims(ndim);
        for (uint32_t d = 0; d < ndim; ++d) dims[d] = r.rd<uint64_t>();
        for (uint32_t d = ndim; d-- > 0;) t.shape.push_back((int64_t)dims[d]);  // reversed: row-major
        t.gguf_type = r.rd<uint32_t>();
        uint64_t bs = 0, bb = 0;
        if (!gguf_type_geometry(t.gguf_type, bs, bb))
            bc::fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE,
                     "gguf: tensor " + t.name + " has unsupported GGUF type " + std::to_string(t.gguf_type));
        t.dtype = dtype_of_gguf_type(t.gguf_type);
        t.offset = r.rd<uint64_t>();
        uint64_t elems = 1;
        for (int64_t d : t.shape) elems *= (uint64_t)d;
        t.length = (elems + bs - 1) / bs * bb;  // data_byte_length (types.rs:116-121)
        f.tensors.push_back(std::move(t));
    }
    // tensor_info.rs:80-125: data section at the next alignment boundary
    int64_t align = 32;
    as_int(f.get("general.alignment"), align);
    if (align <= 0) invalid("gguf: bad general.alignment");
    const uint64_t data_start = ((uint64_t)r.pos + (uint64_t)align - 1) / (uint64_t)align * (uint64_t)align;
    for (Tensor& t : f.tensors) {
        t.offset += data_start;
        if (t.offset > f.size || t.length > f.size - t.offset)
            bc::shape_err("gguf: tensor " + t.name + " data lies beyond the end of the file");
    }
}

const Tensor* find(const BeaconCudaGguf& f, const std::string& name) {
    for (const Tensor& t : f.tensors)
        if (t.name == name) return &t;
    return nullptr;
}

}  // namespace

using namespace bc;

extern "C" {

int32_t beacon_cuda_gguf_open(const char* path, BeaconCudaGguf** out) {
    return guard([&]() -> int32_t {
        require(path && out, "gguf_open: null argument");
        auto f = std::make_unique<BeaconCudaGguf>();
        f->fd = open(path, O_RDONLY);
        if (f->fd < 0) invalid(std::string("gguf_open: cannot open ") + path);
        struct stat st;
        if (fstat(f->fd, &st) != 0) invalid(std::string("gguf_open: cannot stat ") + path);
        f->size = (size_t)st.st_size;
        if (f->size < 24) shape_err("gguf: truncated file (needed 24 bytes at offset 0)");
        f->map = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
        if (f->map == MAP_FAILED) {
            f->map = nullptr;
            invalid(std::string("gguf_open: cannot map ") + path);
        }
        parse(*f);
        *out = f.release();
        return BEACON_CUDA_OK;
    });
}

void beacon_cuda_gguf_close(BeaconCudaGguf* f) { delete f; }

int32_t beacon_cuda_gguf_version(const BeaconCudaGguf* f, uint32_t* out) {
    return guard([&]() -> int32_t {
        require(f && out, "gguf_version: null argument");
        *out = f->version;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_gguf_tensor_count(const BeaconCudaGguf* f, int64_t* out) {
    return guard([&]() -> int32_t {
        require(f && out, "gguf_tensor_count: null argument");
        *out = (int64_t)f->tensors.size();
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_gguf_tensor_info(const BeaconCudaGguf* f, int64_t index, const char** out_name,
                                     int32_t* out_dtype, int64_t* out_shape, size_t* inout_ndim,
                                     const void** out_data, uint64_t* out_nbytes) {
    return guard([&]() -> int32_t {
        require(f && inout_ndim, "gguf_tensor_info: null argument");
        if (index < 0 || index >= (int64_t)f->tensors.size()) shape_err("gguf_tensor_info: no such tensor");
        const Tensor& t = f->tensors[(size_t)index];
        const size_t cap = *inout_ndim;
        *inout_ndim = t.shape.size();
        if (cap < t.shape.size()) invalid("gguf_tensor_info: shape capacity too small");
        if (out_shape)
            for (size_t d = 0; d < t.shape.size(); ++d) out_shape[d] = t.shape[d];
        if (out_name) *out_name = t.name.c_str();
        if (out_dtype) *out_dtype = t.dtype;
        if (out_data) *out_data = static_cast<const uint8_t*>(f->map) + t.offset;
        if (out_nbytes) *out_nbytes = t.length;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_gguf_find_tensor(const BeaconCudaGguf* f, const char* name, int64_t* out_index) {
    return guard([&]() -> int32_t {
        require(f && name && out_index, "gguf_find_tensor: null argument");
        for (size_t i = 0; i < f->tensors.size(); ++i)
            if (f->tensors[i].name == name) {
                *out_index = (int64_t)i;
                return BEACON_CUDA_OK;
            }
        invalid(std::string("gguf: no tensor named ") + name);
    });
}

int32_t beacon_cuda_gguf_get_int(const BeaconCudaGguf* f, const char* key, int64_t* out) {
    return guard([&]() -> int32_t {
        require(f && key && out, "gguf_get_int: null argument");
        if (!as_int(f->get(key), *out)) invalid(std::string("gguf: no integer metadata ") + key);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_gguf_get_float(const BeaconCudaGguf* f, const char* key, double* out) {
    return guard([&]() -> int32_t {
        require(f && key && out, "gguf_get_float: null argument");
        if (!as_float(f->get(key), *out)) invalid(std::string("gguf: no float metadata ") + key);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_gguf_get_string(const BeaconCudaGguf* f, const char* key, const char** out) {
    return guard([&]() -> int32_t {
        require(f && key && out, "gguf_get_string: null argument");
        const Value* v = f->get(key);
        if (!v || v->type != 8) invalid(std::string("gguf: no string metadata ") + key);
        *out = v->s.c_str();
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_gguf_get_array_len(const BeaconCudaGguf* f, const char* key, uint64_t* out) {
    return guard([&]() -> int32_t {
        require(f && key && out, "gguf_get_array_len: null argument");
        const Value* v = f->get(key);
        if (!v || v->type != 9) invalid(std::string("gguf: no array metadata ") + key);
        *out = v->count;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_gguf_model_config(const BeaconCudaGguf* f, BeaconCudaModelConfig* cfg) {
    return guard([&]() -> int32_t {
        require(f && cfg, "gguf_model_config: null argument");
        // config_map.rs:14-100
        const Value* arch = f->get("general.architecture");
        if (!arch || arch->type != 8) invalid("gguf: missing metadata general.architecture");
        const std::string a = arch->s;
        if (a != "llama" && a != "qwen2" && a != "qwen" && a != "phi3" && a != "phi" && a.rfind("gemma", 0) != 0)
            fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "gguf: unsupported architecture " + a);
        auto key = [&](const char* k) { return a + "." + k; };
        auto need = [&](const char* k) {
            int64_t v = 0;
            if (!as_int(f->get(key(k).c_str()), v)) invalid("gguf: missing metadata " + key(k));
            return v;
        };
        auto opt_int = [&](const char* k, int64_t dflt) {
            int64_t v = dflt;
            as_int(f->get(key(k).c_str()), v);
            return v;
        };
        auto opt_f = [&](const char* k, double dflt) {
            double v = dflt;
            as_float(f->get(key(k).c_str()), v);
            return v;
        };
        const int64_t hidden = need("embedding_length"), layers = need("block_count"),
                      heads = need("attention.head_count"), ffn = need("feed_forward_length");
        if (heads <= 0) invalid("gguf: attention.head_count must be positive");
        int64_t vocab = 0;
        if (!as_int(f->get(key("vocab_size").c_str()), vocab)) {
            const Value* toks = f->get("tokenizer.ggml.tokens");
            vocab = toks && toks->type == 9 ? (int64_t)toks->count : 0;
        }
        cfg->vocab_size = (int32_t)vocab;
        cfg->hidden_size = (int32_t)hidden;
        cfg->num_layers = (int32_t)layers;
        cfg->num_heads = (int32_t)heads;
        cfg->num_kv_heads = (int32_t)opt_int("attention.head_count_kv", heads);
        cfg->head_dim = (int32_t)opt_int("attention.key_length", hidden / heads);
        cfg->intermediate_size = (int32_t)ffn;
        if (cfg->max_context <= 0) cfg->max_context = (int32_t)opt_int("context_length", 4096);
        cfg->rope_theta = (float)opt_f("rope.freq_base", 10000.0);
        cfg->rms_norm_eps = (float)opt_f("attention.layer_norm_rms_epsilon", 1e-5);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_load_gguf(BeaconCudaModel* m, const BeaconCudaGguf* f) {
    return guard([&]() -> int32_t {
        require(m && f, "model_load_gguf: null argument");
        const BeaconCudaModelConfig& c = model_config_of(m);
        BeaconCudaContext* ctx = model_context_of(m);
        const int64_t H = c.hidden_size, QD = (int64_t)c.num_heads * c.head_dim,
                      KD = (int64_t)c.num_kv_heads * c.head_dim, F = c.intermediate_size, V = c.vocab_size;
        for (const Tensor& t : f->tensors)
            if (t.name.size() > 5 && t.name.compare(t.name.size() - 5, 5, ".bias") == 0)
                fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE,
                     "model_load_gguf: bias tensor " + t.name + " (the Llama op order has none)");
        auto tensor = [&](const std::string& name, std::vector<int64_t> shape) -> const Tensor& {
            const Tensor* t = find(*f, name);
            if (!t) invalid("model_load_gguf: weight not found: " + name);  // EngineError::WeightNotFound
            if (t->shape != shape) shape_err("model_load_gguf: " + name + " has an unexpected shape");
            if (t->dtype < 0)
                fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "model_load_gguf: " + name + " has no BeaconDtype");
            return *t;
        };
        auto data = [&](const Tensor& t) { return static_cast<const uint8_t*>(f->map) + t.offset; };
        auto set = [&](int32_t layer, int32_t slot, const Tensor& t) {
            // Q4_0 nibbles in GGUF files are in the split order (byte i -> elements i, i + 16)
            const int32_t nib = BEACON_CUDA_NIBBLE_GGUF_SPLIT;
            const int32_t st = beacon_cuda_model_set_weight(m, layer, slot, data(t), t.dtype, nib, 0);
            if (st != BEACON_CUDA_OK) fail(st, std::string(get_error()) + " (" + t.name + ")");
        };
        // embeddings: F16 / F32 as they are; quantized ones dequantised on the
        // device to the f16 values dequantize_to_f16 gives (dequant.rs:33-60)
        const Tensor& emb = tensor("token_embd.weight", {V, H});
        if (is_quantized(emb.dtype)) {
            BeaconCudaTensor* q = nullptr;
            BeaconCudaTensor* h = nullptr;
            BeaconCudaStream* s = nullptr;
            int32_t st = beacon_cuda_stream_create(ctx, &s);
            const int64_t shp[2] = {V, H};
            if (st == BEACON_CUDA_OK)
                st = beacon_cuda_tensor_upload(ctx, data(emb), shp, 2, emb.dtype, BEACON_CUDA_NIBBLE_GGUF_SPLIT, &q);
            if (st == BEACON_CUDA_OK) st = beacon_cuda_op_dequantize_to_f16(ctx, s, q, &h);
            if (st == BEACON_CUDA_OK) st = beacon_cuda_stream_synchronize(s);
            if (st == BEACON_CUDA_OK)
                st = beacon_cuda_model_set_weight(m, -1, BEACON_CUDA_W_EMBED, h->data(), BEACON_CUDA_DTYPE_F16, 0, 1);
            const std::string msg = st == BEACON_CUDA_OK ? "" : get_error();
            beacon_cuda_tensor_destroy(h);
            beacon_cuda_tensor_destroy(q);
            beacon_cuda_stream_destroy(s);
            if (st != BEACON_CUDA_OK) fail(st, msg + " (token_embd.weight)");
        } else {
            set(-1, BEACON_CUDA_W_EMBED, emb);
        }
        set(-1, BEACON_CUDA_W_FINAL_NORM, tensor("output_norm.weight", {H}));
        // output.weight, or the tied embedding when the file has none
        set(-1, BEACON_CUDA_W_LM_HEAD, find(*f, "output.weight") ? tensor("output.weight", {V, H}) : emb);
        for (int32_t li = 0; li < c.num_layers; ++li) {
            const std::string p = "blk." + std::to_string(li) + ".";
            set(li, BEACON_CUDA_W_ATTN_NORM, tensor(p + "attn_norm.weight", {H}));
            set(li, BEACON_CUDA_W_Q, tensor(p + "attn_q.weight", {QD, H}));
            set(li, BEACON_CUDA_W_K, tensor(p + "attn_k.weight", {KD, H}));
            set(li, BEACON_CUDA_W_V, tensor(p + "attn_v.weight", {KD, H}));
            set(li, BEACON_CUDA_W_O, tensor(p + "attn_output.weight", {H, QD}));
            set(li, BEACON_CUDA_W_FFN_NORM, tensor(p + "ffn_norm.weight", {H}));
            set(li, BEACON_CUDA_W_GATE, tensor(p + "ffn_gate.weight", {F, H}));
            set(li, BEACON_CUDA_W_UP, tensor(p + "ffn_up.weight", {F, H}));
            set(li, BEACON_CUDA_W_DOWN, tensor(p + "ffn_down.weight", {H, F}));
        }
        return BEACON_CUDA_OK;
    });
}

}  // extern "C"
