// ingest.cu — decoder weights from a safetensors checkpoint, straight to HBM.
//
// The reference memory-maps the checkpoint (ds_safetensors.c: a single
// model.safetensors, else every model-*.safetensors of the directory in
// name order) and points its decoder at the mapped BF16 tensors by name
// (ds_ocr.c:608-690); it then copies every expert's gate and up matrices
// into one host block per layer (ds_ocr.c:696-757). Here the same files
// and names feed the device directly: each tensor is copied from the
// mapping into HBM once, the expert block and the stacked down matrices are
// assembled in HBM (no multi-GB host copy), norms are widened to F32 as the
// reference's loader does, and the token embeddings are a table of their
// own (the reference's tok_embeddings_bf16), not the LM head.
//
// Safetensors layout: an 8-byte little-endian header length N, N bytes of
// JSON {name: {"dtype", "shape", "data_offsets": [begin, end]}, ...,
// "__metadata__": {...}}, then the data; offsets are relative to the data.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <cuda_fp16.h>

#include "ctx.h"
#include "kernels_decode.cuh"

namespace ds {

// dtype codes as the reference's safetensor_dtype_t (ds_safetensors.h)
enum { ST_F32 = 0, ST_F16 = 1, ST_BF16 = 2, ST_I32 = 3, ST_I64 = 4, ST_BOOL = 5, ST_UNKNOWN = -1 };

static int st_dtype(const std::string &s) {
    if (s == "F32") return ST_F32;
    if (s == "F16") return ST_F16;
    if (s == "BF16") return ST_BF16;
    if (s == "I32") return ST_I32;
    if (s == "I64") return ST_I64;
    if (s == "BOOL") return ST_BOOL;
    return ST_UNKNOWN;
}
static size_t st_elem(int dt) {
    switch (dt) {
        case ST_F32: case ST_I32: return 4;
        case ST_F16: case ST_BF16: return 2;
        case ST_I64: return 8;
        case ST_BOOL: return 1;
        default: return 0;
    }
}

struct StTensor {
    int dtype = ST_UNKNOWN;
    std::vector<int64_t> shape;
    size_t begin = 0, end = 0;  // relative to the data section
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t d : shape) n *= d;
        return n;
    }
};

struct StFile {
    std::string path;
    void *map = nullptr;
    size_t size = 0, data0 = 0;
    std::map<std::string, StTensor> tensors;
    ~StFile() {
        if (map) munmap(map, size);
    }
    const uint8_t *data(const StTensor &t) const { return (const uint8_t *)map + data0 + t.begin; }
};

// A small JSON reader for the header: objects, arrays, strings (with
// escapes), numbers, true/false/null; tensor entries keep what they need.
struct Json {
    const char *p, *e;
    std::string err;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool lit(char c) {
        ws();
        if (p < e && *p == c) {
            p++;
            return true;
        }
        return false;
    }
    bool str(std::string &out) {
        ws();
        if (p >= e || *p != '"') return fail("expected a string");
        p++;
        out.clear();
        while (p < e && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= e) return fail("bad escape");
                char x = *p++;
                switch (x) {
                    case 'n': c = '\n'; break;
                    case 't': c = '\t'; break;
                    case 'r': c = '\r'; break;
                    case 'b': c = '\b'; break;
                    case 'f': c = '\f'; break;
                    case 'u': {  // \uXXXX: kept only for ASCII code points
                        if (e - p < 4) return fail("bad \\u escape");
                        unsigned v = 0;
                        for (int i = 0; i < 4; i++) {
                            char h = *p++;
                            v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : (h | 32) - 'a' + 10);
                        }
                        c = v < 128 ? (char)v : '?';
                        break;
                    }
                    default: c = x;
                }
            }
            out.push_back(c);
        }
        if (p >= e) return fail("unterminated string");
        p++;
        return true;
    }
    bool integer(int64_t &v) {
        ws();
        const char *s = p;
        bool neg = p < e && *p == '-';
        if (neg) p++;
        if (p >= e || *p < '0' || *p > '9') return fail("expected an integer");
        v = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            if (v > (INT64_MAX - 9) / 10) return fail("integer overflow");
            v = v * 10 + (*p++ - '0');
        }
        if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) {
            p = s;
            return fail("expected an integer");
        }
        if (neg) v = -v;
        return true;
    }
    bool skip() {  // any value
        ws();
        if (p >= e) return fail("unexpected end");
        if (*p == '"') {
            std::string t;
            return str(t);
        }
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            p++;
            if (lit(close)) return true;
            do {
                if (obj) {
                    std::string k;
                    if (!str(k) || !lit(':')) return fail("bad object");
                }
                if (!skip()) return false;
            } while (lit(','));
            return lit(close) || fail("unterminated container");
        }
        while (p < e && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') p++;
        return true;
    }
    bool fail(const char *m) {
        if (err.empty()) err = m;
        return false;
    }
};

static bool st_parse_entry(Json &j, StTensor &t) {
    if (!j.lit('{')) return j.fail("tensor entry is not an object");
    bool have_offsets = false;
    if (j.lit('}')) return j.fail("empty tensor entry");
    do {
        std::string k;
        if (!j.str(k) || !j.lit(':')) return j.fail("bad tensor entry");
        if (k == "dtype") {
            std::string d;
            if (!j.str(d)) return false;
            t.dtype = st_dtype(d);
        } else if (k == "shape") {
            if (!j.lit('[')) return j.fail("shape is not an array");
            if (!j.lit(']')) {
                do {
                    int64_t v;
                    if (!j.integer(v) || v < 0) return j.fail("bad shape");
                    t.shape.push_back(v);
                } while (j.lit(','));
                if (!j.lit(']')) return j.fail("bad shape");
            }
        } else if (k == "data_offsets") {
            int64_t b, e;
            if (!j.lit('[') || !j.integer(b) || !j.lit(',') || !j.integer(e) || !j.lit(']') || b < 0 || e < b)
                return j.fail("bad data_offsets");
            t.begin = (size_t)b;
            t.end = (size_t)e;
            have_offsets = true;
        } else if (!j.skip()) {
            return false;
        }
    } while (j.lit(','));
    if (!j.lit('}')) return j.fail("unterminated tensor entry");
    return have_offsets || j.fail("tensor entry without data_offsets");
}

// Opens and validates one file; false with a message on any inconsistency.
static bool st_open(const std::string &path, StFile &f, std::string &err) {
    f.path = path;
    int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "cannot open " + path;
        return false;
    }
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
        close(fd);
        err = path + ": not a safetensors file";
        return false;
    }
    f.size = (size_t)sb.st_size;
    f.map = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (f.map == MAP_FAILED) {
        f.map = nullptr;
        err = "cannot map " + path;
        return false;
    }
    uint64_t n = 0;
    memcpy(&n, f.map, 8);  // little-endian hosts only (x86-64, aarch64)
    if (n > f.size - 8) {
        err = path + ": header length beyond the file";
        return false;
    }
    f.data0 = 8 + (size_t)n;
    Json j{(const char *)f.map + 8, (const char *)f.map + 8 + n, {}};
    bool ok = j.lit('{');
    if (ok && !j.lit('}')) {
        do {
            std::string name;
            if (!j.str(name) || !j.lit(':')) {
                ok = false;
                break;
            }
            if (name == "__metadata__") {
                if (!j.skip()) {
                    ok = false;
                    break;
                }
                continue;
            }
            StTensor t;
            if (!st_parse_entry(j, t)) {
                ok = false;
                break;
            }
            const size_t es = st_elem(t.dtype);
            if (t.end > f.size - f.data0 || (es && (size_t)t.numel() * es != t.end - t.begin)) {
                err = path + ": tensor " + name + " has inconsistent size or offsets";
                return false;
            }
            f.tensors[name] = t;
        } while (j.lit(','));
        ok = ok && j.lit('}');
    }
    if (!ok) {
        err = path + ": bad header (" + (j.err.empty() ? "syntax" : j.err) + ")";
        return false;
    }
    return true;
}

// The checkpoint of a model directory: model.safetensors, else every
// model-*.safetensors in name order (ds_safetensors.c:309-371), or a single
// file path.
struct StModel {
    std::vector<StFile *> files;
    ~StModel() {
        for (StFile *f : files) delete f;
    }
    bool open(const std::string &dir, std::string &err) {
        struct stat sb;
        if (stat(dir.c_str(), &sb) == 0 && S_ISREG(sb.st_mode)) return add(dir, err);
        const std::string single = dir + "/model.safetensors";
        if (stat(single.c_str(), &sb) == 0) return add(single, err);
        DIR *d = opendir(dir.c_str());
        if (!d) {
            err = "cannot open directory " + dir;
            return false;
        }
        std::vector<std::string> names;
        while (struct dirent *ent = readdir(d)) {
            const std::string n = ent->d_name;
            if (n.compare(0, 6, "model-") == 0 && n.find(".safetensors") != std::string::npos) names.push_back(n);
        }
        closedir(d);
        if (names.empty()) {
            err = "no safetensors files in " + dir;
            return false;
        }
        std::sort(names.begin(), names.end());
        for (const auto &n : names)
            if (!add(dir + "/" + n, err)) return false;
        return true;
    }
    bool add(const std::string &path, std::string &err) {
        StFile *f = new StFile();
        if (!st_open(path, *f, err)) {
            delete f;
            return false;
        }
        files.push_back(f);
        return true;
    }
    // the first shard holding the name (the reference's lookup order)
    const StTensor *find(const std::string &name, const StFile **in) const {
        for (const StFile *f : files) {
            auto it = f->tensors.find(name);
            if (it != f->tensors.end()) {
                if (in) *in = f;
                return &it->second;
            }
        }
        return nullptr;
    }
    size_t count() const {
        size_t n = 0;
        for (const StFile *f : files) n += f->tensors.size();
        return n;
    }
};

}  // namespace ds

using namespace ds;

static thread_local std::string g_st_err;

// Host-only probes of a checkpoint (no device needed).
extern "C" const char *ds_cuda_safetensors_error(void) { return g_st_err.c_str(); }

extern "C" int ds_cuda_safetensors_count(const char *path) {
    if (!path) return DS_CUDA_EINVAL;
    StModel m;
    if (!m.open(path, g_st_err)) return DS_CUDA_EINVAL;
    return (int)m.count();
}

extern "C" int ds_cuda_safetensors_find(const char *path, const char *name, int *dtype, int *ndim, int64_t *shape8,
                                        size_t *data_offset, size_t *data_size) {
    if (!path || !name) return DS_CUDA_EINVAL;
    StModel m;
    if (!m.open(path, g_st_err)) return DS_CUDA_EINVAL;
    const StTensor *t = m.find(name, nullptr);
    if (!t) return 0;
    if (dtype) *dtype = t->dtype;
    if (ndim) *ndim = (int)t->shape.size();
    if (shape8)
        for (size_t i = 0; i < t->shape.size() && i < 8; i++) shape8[i] = t->shape[i];
    if (data_offset) *data_offset = t->begin;
    if (data_size) *data_size = t->end - t->begin;
    return 1;
}

namespace {

struct Loader {
    ds_cuda_ctx *c;
    StModel st;
    std::string err;

    int fail(const std::string &m) { return ctx_fail(c, DS_CUDA_EINVAL, "decoder_create_from_safetensors: %s", m.c_str()); }

    // the tensor `name`, of `dtype` (or any of BF16/F16/F32 when float_any)
    // with exactly the dims given
    const StTensor *get(const std::string &name, std::initializer_list<int64_t> dims, const StFile **f,
                        bool float_any = false) {
        const StTensor *t = st.find(name, f);
        if (!t) {
            err = "tensor " + name + " not found";
            return nullptr;
        }
        if (float_any ? (t->dtype != ST_BF16 && t->dtype != ST_F32 && t->dtype != ST_F16) : t->dtype != ST_BF16) {
            err = "tensor " + name + " has an unsupported dtype";
            return nullptr;
        }
        if (t->shape.size() != dims.size() || !std::equal(dims.begin(), dims.end(), t->shape.begin())) {
            err = "tensor " + name + " has an unexpected shape";
            return nullptr;
        }
        return t;
    }
    // copy a mapped BF16 tensor into dev (bytes already checked)
    bool copy(void *dev, const std::string &name, std::initializer_list<int64_t> dims) {
        const StFile *f;
        const StTensor *t = get(name, dims, &f);
        if (!t) return false;
        cudaError_t e = cudaMemcpy(dev, f->data(*t), t->end - t->begin, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            err = std::string("copy of ") + name + ": " + cudaGetErrorString(e);
            return false;
        }
        return true;
    }
    void *alloc(size_t bytes) {
        void *d = nullptr;
        if (cudaMalloc(&d, bytes) != cudaSuccess) {
            cudaGetLastError();
            err = "device allocation of " + std::to_string(bytes) + " bytes failed";
            return nullptr;
        }
        return d;
    }
    // device memory handed to the context under a reserved host key
    template <typename T>
    const T *adopt(void *dev, size_t bytes) {
        void *k = ctx_adopt(c, dev, bytes);
        if (!k) {
            cudaFree(dev);
            err = "cannot reserve a host key range";
        }
        return (const T *)k;
    }
    const uint16_t *bf16(const std::string &name, int64_t rows, int64_t cols) {
        const size_t bytes = (size_t)rows * cols * 2;
        void *d = alloc(bytes);
        if (!d) return nullptr;
        if (!copy(d, name, {rows, cols})) {
            cudaFree(d);
            return nullptr;
        }
        return adopt<uint16_t>(d, bytes);
    }
    // a norm vector widened to F32 (the reference loads these with
    // safetensors_get_f32, ds_safetensors.c:255-278)
    const float *f32(const std::string &name, int64_t n) {
        const StFile *f;
        const StTensor *t = get(name, {n}, &f, true);
        if (!t) return nullptr;
        std::vector<float> h((size_t)n);
        const uint8_t *src = f->data(*t);
        for (int64_t i = 0; i < n; i++) {
            if (t->dtype == ST_F32) {
                memcpy(&h[i], src + 4 * i, 4);
            } else {
                uint16_t u;
                memcpy(&u, src + 2 * i, 2);
                if (t->dtype == ST_BF16) {
                    const uint32_t b = (uint32_t)u << 16;
                    memcpy(&h[i], &b, 4);
                } else {
                    h[i] = __half2float(*reinterpret_cast<const __half *>(&u));
                }
            }
        }
        void *d = alloc((size_t)n * 4);
        if (!d) return nullptr;
        if (cudaMemcpy(d, h.data(), (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaFree(d);
            err = "copy of " + name;
            return nullptr;
        }
        return adopt<float>(d, (size_t)n * 4);
    }
    // INT8 copy of device BF16 rows [rows x cols] (the reference quantises
    // the same matrices with ds_int4_quantize_bf16, ds_ocr.c:781-841)
    bool int8(const uint16_t *src_key, int64_t rows, int64_t cols, const int8_t **q, const float **s,
              const float **o) {
        const void *src = ctx_lookup(c, src_key, (size_t)rows * cols * 2, false);
        void *dq = alloc((size_t)rows * cols), *ds_ = alloc((size_t)rows * 4), *dof = alloc((size_t)rows * 4);
        if (!src || !dq || !ds_ || !dof) return false;
        if (launch_quantize_int8((const uint16_t *)src, (int)rows, (int)cols, (int8_t *)dq, (float *)ds_,
                                 (float *)dof, c->stream) != cudaSuccess ||
            cudaStreamSynchronize(c->stream) != cudaSuccess) {
            err = "int8 quantisation launch failed";
            return false;
        }
        *q = adopt<int8_t>(dq, (size_t)rows * cols);
        *s = adopt<float>(ds_, (size_t)rows * 4);
        *o = adopt<float>(dof, (size_t)rows * 4);
        return *q && *s && *o;
    }
};

}  // namespace

extern "C" int ds_cuda_decoder_create_from_safetensors(ds_cuda_ctx_t *c, const char *model_dir,
                                                       const ds_cuda_decoder_config_t *cfg) {
    if (!c || !model_dir || !cfg) return ctx_fail(c, DS_CUDA_EINVAL, "decoder_create_from_safetensors: null argument");
    const auto &g = *cfg;
    if (g.n_layers <= 0 || g.hidden <= 0 || g.n_heads <= 0 || g.head_dim <= 0 || g.vocab <= 0 || g.n_experts <= 0 ||
        g.first_dense < 0 || g.first_dense > g.n_layers)
        return ctx_fail(c, DS_CUDA_EINVAL, "decoder_create_from_safetensors: bad configuration");
    cudaSetDevice(c->device);
    Loader L{c, {}, {}};
    if (!L.st.open(model_dir, L.err)) return L.fail(L.err);
    const int64_t H = g.hidden, QD = (int64_t)g.n_heads * g.head_dim, I = g.moe_inter, E = g.n_experts,
                  S = (int64_t)g.n_shared * g.moe_inter, D = g.dense_inter, V = g.vocab;
    std::vector<ds_cuda_layer_weights_t> lw((size_t)g.n_layers);
    char name[256];
    auto nm = [&](int l, const char *suffix) {
        snprintf(name, sizeof name, "model.layers.%d.%s", l, suffix);
        return std::string(name);
    };
#define NEED(x)                          \
    do {                                 \
        if (!(x)) return L.fail(L.err);  \
    } while (0)
    for (int l = 0; l < g.n_layers; l++) {
        ds_cuda_layer_weights_t &w = lw[(size_t)l];
        memset(&w, 0, sizeof w);
        NEED(w.wq = L.bf16(nm(l, "self_attn.q_proj.weight"), QD, H));
        NEED(w.wk = L.bf16(nm(l, "self_attn.k_proj.weight"), QD, H));
        NEED(w.wv = L.bf16(nm(l, "self_attn.v_proj.weight"), QD, H));
        NEED(w.wo = L.bf16(nm(l, "self_attn.o_proj.weight"), H, QD));
        NEED(w.input_norm = L.f32(nm(l, "input_layernorm.weight"), H));
        NEED(w.post_attn_norm = L.f32(nm(l, "post_attention_layernorm.weight"), H));
        if (l < g.first_dense) {
            NEED(w.dense_gate = L.bf16(nm(l, "mlp.gate_proj.weight"), D, H));
            NEED(w.dense_up = L.bf16(nm(l, "mlp.up_proj.weight"), D, H));
            NEED(w.dense_down = L.bf16(nm(l, "mlp.down_proj.weight"), H, D));
            continue;
        }
        NEED(w.router = L.bf16(nm(l, "mlp.gate.weight"), E, H));
        // [E x (gate I x H ; up I x H)] then the shared [gate S x H ; up S x H]
        // (ds_ocr.c:716-757), assembled in HBM
        const size_t fused = (size_t)2 * I * H;
        const size_t block_bytes = ((size_t)E * fused + (size_t)2 * S * H) * 2;
        uint16_t *blk = (uint16_t *)L.alloc(block_bytes);
        NEED(blk);
        bool ok = true;
        for (int e = 0; e < E && ok; e++) {
            char en[128];
            snprintf(en, sizeof en, "mlp.experts.%d.gate_proj.weight", e);
            ok = L.copy(blk + e * fused, nm(l, en), {I, H});
            snprintf(en, sizeof en, "mlp.experts.%d.up_proj.weight", e);
            ok = ok && L.copy(blk + e * fused + (size_t)I * H, nm(l, en), {I, H});
        }
        if (ok && S > 0) {
            ok = L.copy(blk + E * fused, nm(l, "mlp.shared_experts.gate_proj.weight"), {S, H}) &&
                 L.copy(blk + E * fused + (size_t)S * H, nm(l, "mlp.shared_experts.up_proj.weight"), {S, H});
        }
        if (!ok) {
            cudaFree(blk);
            return L.fail(L.err);
        }
        NEED(w.expert_block = L.adopt<uint16_t>(blk, block_bytes));
        const size_t down_bytes = (size_t)E * H * I * 2;
        uint16_t *dn = (uint16_t *)L.alloc(down_bytes);
        NEED(dn);
        for (int e = 0; e < E && ok; e++) {
            char en[128];
            snprintf(en, sizeof en, "mlp.experts.%d.down_proj.weight", e);
            ok = L.copy(dn + (size_t)e * H * I, nm(l, en), {H, I});
        }
        if (!ok) {
            cudaFree(dn);
            return L.fail(L.err);
        }
        NEED(w.down = L.adopt<uint16_t>(dn, down_bytes));
        if (S > 0) NEED(w.shared_down = L.bf16(nm(l, "mlp.shared_experts.down_proj.weight"), H, S));
        if (g.use_int8) {
            NEED(L.int8(w.expert_block, E * 2 * I, H, &w.gu_q, &w.gu_scale, &w.gu_off));
            NEED(L.int8(w.down, E * H, I, &w.dn_q, &w.dn_scale, &w.dn_off));
            if (S > 0) {
                NEED(L.int8(w.expert_block + E * fused, 2 * S, H, &w.sgu_q, &w.sgu_scale, &w.sgu_off));
                NEED(L.int8(w.shared_down, H, S, &w.sdn_q, &w.sdn_scale, &w.sdn_off));
            }
        }
    }
    const float *final_norm;
    NEED(final_norm = L.f32("model.norm.weight", H));
    const uint16_t *embed;
    NEED(embed = L.bf16("model.embed_tokens.weight", V, H));
    // an absent lm_head means tied embeddings (ds_moe_decoder.c:1023)
    const uint16_t *lm_head = embed;
    if (L.st.find("lm_head.weight", nullptr)) NEED(lm_head = L.bf16("lm_head.weight", V, H));
#undef NEED
    const int id = ds_cuda_decoder_create(c, cfg, lw.data(), final_norm, lm_head);
    if (id <= 0) return id;
    const int rc = ds_cuda_decoder_set_embeddings(c, id, embed);
    if (rc < 0) {
        ds_cuda_decoder_destroy(c, id);
        return rc;
    }
    return id;
}
