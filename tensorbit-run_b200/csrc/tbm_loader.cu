// tbm_loader.cu -- a .tbm model container read straight into device memory.
//
// The reference maps a .tbm file read-only and hands out zero-copy host
// views of every tensor (tb_model_load_tbm, src/model.c:482-580; the views,
// src/model.c:681-739).  Its engine then runs on those host bytes.  Here the
// same container is parsed the same way -- the 4-byte little-endian index
// length at the end of the file, the JSON index before it (architecture,
// config, tensors), a 4096-byte .tb header at each tensor's offset -- and
// every tensor's bytes are streamed into one device allocation:
//   weights at offset + header.weights_offset, (INT4: ceil(n/2) bytes, INT8:
//     n bytes, else n * element size),
//   mask bytes at offset + header.masks_offset,
//   f32 scales right after quantized weights (src/model.c:718-739).
// Quantized tensors stay quantized on the device (the fused GEMV of the
// device runner expands them in registers); tb_b200_tbm_runner_desc fills a
// runner description from the tensors with the reference runner's own name
// lookup (include/tensorbit/run/ops.hpp:61-72, 84-116, 259-276) and its
// config normalisation (ops.hpp:291-323).
//
// Streaming: the file is mapped read-only; chunks of at most kChunk bytes
// are copied into one of two page-locked staging buffers and from there to
// the device on the caller's stream, so the host copy of one chunk overlaps
// the DMA of the previous one.
//
// Where the reference reads without checking, the loader checks: a tensor
// whose bytes run past the end of the file is TB_ERR_TRUNCATED (the
// reference would read out of bounds), and a tensor whose .tb header has a
// bad magic is kept, with no device bytes, and reported by
// tb_b200_tbm_tensor as TB_ERR_BAD_MAGIC (the reference logs a warning at
// load and fails the same tensor's view).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "tb_internal.h"

namespace {

constexpr size_t kHeader = 4096;
constexpr uint32_t kMagic = 0x31304254u;  // "TB01"
constexpr int kMaxTensors = 512;          // the reference's index limit (src/model.c:513)
constexpr size_t kChunk = 32u << 20;      // staging buffer size

// ----------------------------------------------------------------- JSON
// A small JSON reader for the index: objects, arrays, strings (with
// escapes), numbers, true/false/null.
struct JVal {
    enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
    double num = 0.0;
    int64_t inum = 0;
    bool is_int = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
};

struct JParser {
    const char* p;
    const char* end;
    int depth = 0;
    void ws() {
        while (p < end && isspace((unsigned char)*p)) ++p;
    }
    bool eat(char c) {
        ws();
        if (p < end && *p == c) {
            ++p;
            return true;
        }
        return false;
    }
    bool string(std::string& out) {
        ws();
        if (p >= end || *p != '"') return false;
        ++p;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return false;
                const char e = *p++;
                switch (e) {
                    case 'n': c = '\n'; break;
                    case 't': c = '\t'; break;
                    case 'r': c = '\r'; break;
                    case 'b': c = '\b'; break;
                    case 'f': c = '\f'; break;
                    case 'u': {  // keep \uXXXX as '?' (names are ASCII in practice)
                        if (end - p < 4) return false;
                        p += 4;
                        c = '?';
                        break;
                    }
                    default: c = e;
                }
            }
            out.push_back(c);
        }
        if (p >= end) return false;
        ++p;
        return true;
    }
    bool value(JVal& v) {
        ws();
        if (p >= end || ++depth > 64) return false;
        bool r = true;
        const char c = *p;
        if (c == '{') {
            ++p;
            v.kind = JVal::kObj;
            if (!eat('}')) {
                do {
                    std::string k;
                    JVal x;
                    if (!string(k) || !eat(':') || !value(x)) {
                        r = false;
                        break;
                    }
                    v.obj.emplace_back(std::move(k), std::move(x));
                } while (eat(','));
                r = r && eat('}');
            }
        } else if (c == '[') {
            ++p;
            v.kind = JVal::kArr;
            if (!eat(']')) {
                do {
                    JVal x;
                    if (!value(x)) {
                        r = false;
                        break;
                    }
                    v.arr.push_back(std::move(x));
                } while (eat(','));
                r = r && eat(']');
            }
        } else if (c == '"') {
            v.kind = JVal::kStr;
            r = string(v.str);
        } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
            v.kind = JVal::kBool;
            v.num = 1;
            p += 4;
        } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
            v.kind = JVal::kBool;
            p += 5;
        } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
            p += 4;
        } else {
            // a number: copy it out (the buffer is not NUL-terminated)
            const char* q = p;
            while (q < end && (isdigit((unsigned char)*q) || strchr("+-.eE", *q))) ++q;
            if (q == p || q - p > 63) return false;
            char buf[64];
            memcpy(buf, p, (size_t)(q - p));
            buf[q - p] = 0;
            char* e1 = nullptr;
            v.kind = JVal::kNum;
            v.num = strtod(buf, &e1);
            if (*e1) return false;
            v.is_int = !strpbrk(buf, ".eE");
            if (v.is_int) v.inum = strtoll(buf, nullptr, 10);
            p = q;
        }
        --depth;
        return r;
    }
};

int64_t jint(const JVal* v, int64_t dflt = 0) {
    if (!v || v->kind != JVal::kNum) return dflt;
    return v->is_int ? v->inum : (int64_t)v->num;
}
double jnum(const JVal* v, double dflt) {
    return v && v->kind == JVal::kNum ? v->num : dflt;
}

// ---------------------------------------------------------------- model
struct Rec {
    TbB200TbmTensor t;  // device pointers filled after the upload
    bool magic_ok = true;
    uint64_t w_off = 0, m_off = 0, s_off = 0;  // file offsets
    uint64_t w_bytes = 0, m_bytes = 0, s_bytes = 0;
    uint64_t dw = 0, dm = 0, ds = 0;  // device offsets
};

struct TbmModel {
    TbB200TbmConfig cfg;
    std::vector<Rec> recs;
    void* dev = nullptr;
    int device = -1;
};

uint64_t align256(uint64_t v) { return (v + 255) / 256 * 256; }

struct Mapping {
    int fd = -1;
    void* data = MAP_FAILED;
    size_t size = 0;
    ~Mapping() {
        if (data != MAP_FAILED) munmap(data, size);
        if (fd >= 0) close(fd);
    }
};

// The JSON index into `m` (config and tensor descriptors), read as the
// reference reads it (src/model.c:280-475): the top-level keys in file
// order, a repeated key read again; "config" first clears the whole config
// -- the architecture read before it included -- then sets norm_eps 1e-6
// and rope_theta 10000, reads its fields, and makes num_kv_heads =
// num_heads when 0 and head_dim = hidden_size / num_heads.  Without a
// "config" key every field stays 0.  Within a tensor the last of a
// repeated field wins; at most kMaxTensors tensors are read.
int parse_index(const JVal& root, TbmModel& m) {
    if (root.kind != JVal::kObj) return TB_ERR_JSON_PARSE;
    TbB200TbmConfig& c = m.cfg;
    memset(&c, 0, sizeof c);
    for (const auto& kv : root.obj) {
        const std::string& key = kv.first;
        const JVal& v = kv.second;
        if (key == "architecture") {
            if (v.kind != JVal::kStr) return TB_ERR_JSON_PARSE;
            memset(c.architecture, 0, sizeof c.architecture);
            strncpy(c.architecture, v.str.c_str(), sizeof c.architecture - 1);
        } else if (key == "config") {
            if (v.kind != JVal::kObj) return TB_ERR_JSON_PARSE;
            memset(&c, 0, sizeof c);
            c.norm_eps = 1e-6f;
            c.rope_theta = 10000.0f;
            for (const auto& f : v.obj) {
                const JVal* x = &f.second;
                if (f.first == "hidden_size") c.hidden_size = (int)jint(x);
                else if (f.first == "num_heads") c.num_heads = (int)jint(x);
                else if (f.first == "num_kv_heads") c.num_kv_heads = (int)jint(x);
                else if (f.first == "intermediate_size") c.intermediate_size = (int)jint(x);
                else if (f.first == "vocab_size") c.vocab_size = (int)jint(x);
                else if (f.first == "num_layers") c.num_layers = (int)jint(x);
                else if (f.first == "max_seq_len") c.max_seq_len = (int)jint(x);
                else if (f.first == "norm_eps") c.norm_eps = (float)jnum(x, 0.0);
                else if (f.first == "rope_theta") c.rope_theta = (float)jnum(x, 0.0);
            }
            if (c.num_kv_heads == 0) c.num_kv_heads = c.num_heads;
            c.head_dim = c.num_heads > 0 ? c.hidden_size / c.num_heads : 0;
        } else if (key == "tensors") {
            if (v.kind != JVal::kArr) return TB_ERR_JSON_PARSE;
            m.recs.clear();
            for (const JVal& tv : v.arr) {
                if ((int)m.recs.size() >= kMaxTensors) break;
                if (tv.kind != JVal::kObj) return TB_ERR_JSON_PARSE;
                Rec r;
                memset(&r.t, 0, sizeof r.t);
                r.t.dtype = TB_DTYPE_F32;  // the zeroed descriptor's dtype
                for (const auto& f : tv.obj) {
                    const JVal* x = &f.second;
                    if (f.first == "name") {
                        memset(r.t.name, 0, sizeof r.t.name);
                        if (x->kind == JVal::kStr)
                            strncpy(r.t.name, x->str.c_str(), sizeof r.t.name - 1);
                    } else if (f.first == "offset") {
                        r.w_off = (uint64_t)jint(x);
                    } else if (f.first == "shape") {
                        if (x->kind != JVal::kArr) return TB_ERR_JSON_PARSE;
                        for (size_t i = 0; i < x->arr.size() && i < 2; ++i)
                            r.t.shape[i] = jint(&x->arr[i]);
                    } else if (f.first == "nm_n") {
                        r.t.nm_n = (uint32_t)jint(x);
                    } else if (f.first == "nm_m") {
                        r.t.nm_m = (uint32_t)jint(x);
                    } else if (f.first == "dtype") {
                        const std::string& d = x->str;
                        if (d == "fp32") r.t.dtype = TB_DTYPE_F32;
                        else if (d == "fp16") r.t.dtype = TB_DTYPE_F16;
                        else if (d == "bf16") r.t.dtype = TB_DTYPE_BF16;
                        else if (d == "fp64") r.t.dtype = TB_DTYPE_F64;
                        else if (d == "int8") r.t.dtype = TB_DTYPE_INT8;
                        else if (d == "int4") r.t.dtype = TB_DTYPE_INT4;
                    } else if (f.first == "num_weights") {
                        r.t.num_weights = jint(x);
                    } else if (f.first == "num_mask_bytes") {
                        r.t.num_mask_bytes = jint(x);
                    } else if (f.first == "scale_count") {
                        r.t.scale_count = jint(x);
                    } else if (f.first == "group_size") {
                        r.t.group_size = (uint32_t)jint(x);
                    }
                }
                if (r.t.num_weights < 0 || r.t.num_mask_bytes < 0 || r.t.scale_count < 0)
                    return TB_ERR_JSON_PARSE;
                m.recs.push_back(r);
            }
        }
    }
    if (c.num_layers == 0 && !m.recs.empty()) c.num_layers = 1;
    return TB_OK;
}

uint64_t weight_bytes(const TbB200TbmTensor& t) {
    const uint64_t n = (uint64_t)t.num_weights;
    switch (t.dtype) {
        case TB_DTYPE_INT4: return (n + 1) / 2;
        case TB_DTYPE_INT8: return n;
        case TB_DTYPE_F16:
        case TB_DTYPE_BF16: return 2 * n;
        case TB_DTYPE_F64: return 8 * n;
        default: return 4 * n;
    }
}

// Copy `bytes` at host address src to device address dst through the two
// staging buffers.
struct Stager {
    void* host[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int k = 0;
    cudaStream_t s;
    ~Stager() {
        for (int i = 0; i < 2; ++i) {
            if (done[i]) {
                cudaEventSynchronize(done[i]);
                cudaEventDestroy(done[i]);
            }
            if (host[i]) cudaFreeHost(host[i]);
        }
    }
    int init(cudaStream_t st) {
        s = st;
        for (int i = 0; i < 2; ++i) {
            TB_CUDA_TRY(cudaMallocHost(&host[i], kChunk));
            TB_CUDA_TRY(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
        }
        return TB_OK;
    }
    int copy(char* dst, const char* src, uint64_t bytes) {
        while (bytes) {
            const size_t n = bytes < kChunk ? (size_t)bytes : kChunk;
            TB_CUDA_TRY(cudaEventSynchronize(done[k]));  // its previous DMA is over
            memcpy(host[k], src, n);
            TB_CUDA_TRY(cudaMemcpyAsync(dst, host[k], n, cudaMemcpyHostToDevice, s));
            TB_CUDA_TRY(cudaEventRecord(done[k], s));
            k ^= 1;
            dst += n;
            src += n;
            bytes -= n;
        }
        return TB_OK;
    }
};

TbmModel* as_model(const void* h) { return static_cast<TbmModel*>(const_cast<void*>(h)); }

// The reference runner's lookups (ops.hpp:61-72): llama, then gpt-j, then
// a bare component name.
int find(const TbmModel& m, const std::string& name) {
    for (size_t i = 0; i < m.recs.size(); ++i)
        if (name == m.recs[i].t.name) return (int)i;
    return -1;
}
int find_weight(const TbmModel& m, int layer, const char* component) {
    const std::string l = std::to_string(layer);
    int i = find(m, "model.layers." + l + "." + component + ".weight");
    if (i < 0) i = find(m, "transformer.h." + l + "." + component + ".weight");
    if (i < 0) i = find(m, std::string(component) + ".weight");
    return i;
}
int find_first(const TbmModel& m, std::initializer_list<const char*> names) {
    for (const char* n : names) {
        const int i = find(m, n);
        if (i >= 0) return i;
    }
    return -1;
}

TbB200Weight weight_of(const TbmModel& m, int i) {
    TbB200Weight w;
    memset(&w, 0, sizeof w);
    if (i < 0 || !m.recs[i].magic_ok) return w;
    const TbB200TbmTensor& t = m.recs[i].t;
    w.data = t.weights;
    w.dtype = t.dtype;
    w.rows = t.shape[0];
    w.cols = t.shape[1];
    // The reference passes every projection's mask bytes (Model::get_mask,
    // model.hpp:163) whether or not the layer is N:M; only a layer stored
    // with mask bytes has any to give the device.
    w.mask = t.num_mask_bytes > 0 ? t.mask : nullptr;
    if (t.scale_count > 0) {
        w.scales = t.scales;
        w.n_scales = t.scale_count;
        w.group_size = t.group_size;
    }
    return w;
}

}  // namespace

extern "C" {

int tb_b200_tbm_load(const char* path, void* stream, void** model) {
    if (!path || !model) return TB_ERR_INVALID_ARG;
    *model = nullptr;
    Mapping fm;
    fm.fd = open(path, O_RDONLY);
    if (fm.fd < 0) return TB_ERR_FILE_OPEN;
    struct stat st;
    if (fstat(fm.fd, &st) != 0) return TB_ERR_FILE_READ;
    fm.size = (size_t)st.st_size;
    if (fm.size < 4 + 16) return TB_ERR_TRUNCATED;  // src/model.c:489
    fm.data = mmap(nullptr, fm.size, PROT_READ, MAP_PRIVATE, fm.fd, 0);
    if (fm.data == MAP_FAILED) return TB_ERR_FILE_READ;
    madvise(fm.data, fm.size, MADV_SEQUENTIAL);
    const char* base = static_cast<const char*>(fm.data);
    uint32_t index_len;
    memcpy(&index_len, base + fm.size - 4, 4);
    if (index_len == 0 || (size_t)index_len > fm.size - 4) return TB_ERR_TRUNCATED;
    const char* json = base + fm.size - 4 - index_len;

    std::unique_ptr<TbmModel> m(new TbmModel());
    {
        JParser jp{json, json + index_len};
        JVal root;
        if (!jp.value(root)) return TB_ERR_JSON_PARSE;
        const int rc = parse_index(root, *m);
        if (rc) return rc;
    }
    // Headers and extents, all inside the file.
    uint64_t total = 0;
    for (Rec& r : m->recs) {
        const uint64_t off = r.w_off;
        if (off + kHeader > fm.size || off + kHeader < off) return TB_ERR_TRUNCATED;
        uint32_t magic;
        uint64_t woff, moff;
        memcpy(&magic, base + off, 4);
        memcpy(&woff, base + off + 32, 8);
        memcpy(&moff, base + off + 40, 8);
        r.magic_ok = magic == kMagic;  // a bad version only warns in the reference
        if (!r.magic_ok) continue;
        r.w_bytes = weight_bytes(r.t);
        r.m_bytes = (uint64_t)r.t.num_mask_bytes;
        r.s_bytes = 4 * (uint64_t)r.t.scale_count;
        r.w_off = off + woff;
        r.m_off = off + moff;
        r.s_off = r.w_off + r.w_bytes;  // scales follow quantized weights
        if (r.t.scale_count > 0 && r.t.dtype != TB_DTYPE_INT4 && r.t.dtype != TB_DTYPE_INT8)
            r.s_bytes = 0;  // only quantized tensors have scales (src/model.c:718-739)
        auto inside = [&](uint64_t o, uint64_t n) { return o <= fm.size && n <= fm.size - o; };
        if (!inside(r.w_off, r.w_bytes) || (r.m_bytes && !inside(r.m_off, r.m_bytes)) ||
            (r.s_bytes && !inside(r.s_off, r.s_bytes)))
            return TB_ERR_TRUNCATED;
        r.dw = total;
        total += align256(r.w_bytes);
        r.dm = total;
        total += align256(r.m_bytes);
        r.ds = total;
        total += align256(r.s_bytes);
    }
    // One device allocation; every tensor streamed in through the stagers.
    TB_CUDA_TRY(cudaGetDevice(&m->device));
    if (total) TB_CUDA_TRY(cudaMalloc(&m->dev, total));
    cudaStream_t s = tbh::stream_of(stream);
    int rc = TB_OK;
    {
        Stager sg;
        rc = sg.init(s);
        for (size_t i = 0; rc == TB_OK && i < m->recs.size(); ++i) {
            Rec& r = m->recs[i];
            if (!r.magic_ok) continue;
            char* d = static_cast<char*>(m->dev);
            if (r.w_bytes) rc = sg.copy(d + r.dw, base + r.w_off, r.w_bytes);
            if (rc == TB_OK && r.m_bytes) rc = sg.copy(d + r.dm, base + r.m_off, r.m_bytes);
            if (rc == TB_OK && r.s_bytes) rc = sg.copy(d + r.ds, base + r.s_off, r.s_bytes);
            r.t.weights = d + r.dw;
            r.t.mask = r.m_bytes ? reinterpret_cast<const uint8_t*>(d + r.dm) : nullptr;
            r.t.scales = r.s_bytes ? reinterpret_cast<const float*>(d + r.ds) : nullptr;
            r.t.weight_bytes = (int64_t)r.w_bytes;
        }
        if (rc == TB_OK) {
            const cudaError_t e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) {
                tbh::set_error("tb_b200_tbm_load", e);
                rc = TB_ERR_DEVICE;
            }
        }
    }  // the stagers wait for their copies before the mapping goes
    if (rc != TB_OK) {
        if (m->dev) cudaFree(m->dev);
        return rc;
    }
    *model = m.release();
    return TB_OK;
}

int tb_b200_tbm_config(const void* model, TbB200TbmConfig* cfg) {
    if (!model || !cfg) return TB_ERR_INVALID_ARG;
    *cfg = as_model(model)->cfg;
    return TB_OK;
}

int tb_b200_tbm_count(const void* model, int* count) {
    if (!model || !count) return TB_ERR_INVALID_ARG;
    *count = (int)as_model(model)->recs.size();
    return TB_OK;
}

int tb_b200_tbm_find(const void* model, const char* name, int* index) {
    if (!model || !name || !index) return TB_ERR_INVALID_ARG;
    *index = find(*as_model(model), name);
    return *index >= 0 ? TB_OK : TB_ERR_LAYER_NOT_FOUND;
}

int tb_b200_tbm_tensor(const void* model, int index, TbB200TbmTensor* out) {
    if (!model || !out) return TB_ERR_INVALID_ARG;
    const TbmModel& m = *as_model(model);
    if (index < 0 || index >= (int)m.recs.size()) return TB_ERR_LAYER_NOT_FOUND;
    *out = m.recs[index].t;
    return m.recs[index].magic_ok ? TB_OK : TB_ERR_BAD_MAGIC;
}

int tb_b200_tbm_runner_desc(const void* model, int attention, int use_graph,
                            TbB200RunnerDesc* desc, TbB200RunnerLayer* layers, int max_layers) {
    if (!model || !desc || (max_layers > 0 && !layers)) return TB_ERR_INVALID_ARG;
    const TbmModel& m = *as_model(model);
    const TbB200TbmConfig& c = m.cfg;
    // TransformerRunner's normalised config (ops.hpp:304-323): values the
    // index leaves at 0 take Mistral-7B defaults.
    TbB200RunnerDesc d;
    memset(&d, 0, sizeof d);
    d.hidden = c.hidden_size > 0 ? c.hidden_size : 4096;
    d.n_heads = c.num_heads > 0 ? c.num_heads : 32;
    d.n_kv_heads = c.num_kv_heads > 0 ? c.num_kv_heads : 8;
    d.head_dim = c.head_dim > 0 ? c.head_dim : 128;
    d.intermediate = c.intermediate_size > 0 ? c.intermediate_size : 14336;
    d.vocab = c.vocab_size > 0 ? c.vocab_size : 32000;
    d.max_seq = c.max_seq_len > 0 ? c.max_seq_len : 2048;
    d.layers = c.num_layers > 0 ? c.num_layers : 32;
    d.norm_eps = c.norm_eps > 0.0f ? c.norm_eps : 1e-5f;
    d.rope_theta = c.rope_theta > 0.0f ? c.rope_theta : 10000.0f;
    if (d.layers > max_layers) return TB_ERR_INVALID_SHAPE;
    d.attention = attention;
    d.use_graph = use_graph;
    const int emb = find_first(m, {"model.embed_tokens.weight", "transformer.wte.weight",
                                   "transformer.embd.wte.weight"});
    if (emb < 0) return TB_ERR_LAYER_NOT_FOUND;  // ops.hpp:89: no embedding, no forward
    d.embed = weight_of(m, emb);
    const int fn = find_first(m, {"model.norm.weight", "transformer.ln_f.weight",
                                  "transformer.norm.weight"});
    d.final_norm = fn >= 0 && m.recs[fn].magic_ok ? static_cast<const float*>(m.recs[fn].t.weights)
                                                  : nullptr;
    // The lm head (ops.hpp:271-276): lm_head, else the embedding table.
    const int lm = find_first(m, {"lm_head.weight", "model.embed_tokens.weight",
                                  "transformer.wte.weight"});
    d.lm_head = lm >= 0 && lm != emb ? weight_of(m, lm) : TbB200Weight{};
    auto f32_or_absent = [&](int i) { return i < 0 || m.recs[i].t.dtype == TB_DTYPE_F32; };
    if (!f32_or_absent(fn)) return TB_ERR_UNSUPPORTED_DTYPE;
    for (int l = 0; l < d.layers; ++l) {
        TbB200RunnerLayer& L = layers[l];
        memset(&L, 0, sizeof L);
        L.q = weight_of(m, find_weight(m, l, "self_attn.q_proj"));
        L.k = weight_of(m, find_weight(m, l, "self_attn.k_proj"));
        L.v = weight_of(m, find_weight(m, l, "self_attn.v_proj"));
        L.o = weight_of(m, find_weight(m, l, "self_attn.o_proj"));
        L.gate = weight_of(m, find_weight(m, l, "mlp.gate_proj"));
        L.up = weight_of(m, find_weight(m, l, "mlp.up_proj"));
        L.down = weight_of(m, find_weight(m, l, "mlp.down_proj"));
        const int in = find_weight(m, l, "input_layernorm");
        const int pn = find_weight(m, l, "post_attention_layernorm");
        if (!f32_or_absent(in) || !f32_or_absent(pn)) return TB_ERR_UNSUPPORTED_DTYPE;
        L.input_norm = in >= 0 && m.recs[in].magic_ok ? static_cast<const float*>(m.recs[in].t.weights)
                                                      : nullptr;
        L.post_norm = pn >= 0 && m.recs[pn].magic_ok ? static_cast<const float*>(m.recs[pn].t.weights)
                                                     : nullptr;
    }
    d.layer = layers;
    *desc = d;
    return TB_OK;
}

int tb_b200_tbm_free(void* model) {
    if (!model) return TB_OK;
    TbmModel* m = static_cast<TbmModel*>(model);
    if (m->dev) {
        int cur = -1;
        cudaGetDevice(&cur);
        if (m->device >= 0 && cur != m->device) cudaSetDevice(m->device);
        const cudaError_t e = cudaFree(m->dev);
        if (cur >= 0 && cur != m->device) cudaSetDevice(cur);
        delete m;
        if (e != cudaSuccess) {
            tbh::set_error("tb_b200_tbm_free", e);
            return TB_ERR_DEVICE;
        }
        return TB_OK;
    }
    delete m;
    return TB_OK;
}

}  // extern "C"
