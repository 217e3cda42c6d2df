// The reference's model hooks (fn_load, fn_forward, fn_reset, fn_free, fn_debug_layers, fn_use_graphs, fn_n_past,
// fn_last_ms, fn_dev_gb, fn_split; engine/faie2fn.cu:2466-2743) on B200: a GGUF v3 model file (one or two shards)
// with the qwen3next tensor names is read through a memory map, checked, uploaded into the engine's resident handles
// and run by the decode step of fn_decoder.cu, one CUDA graph replay per token.
//
// File layout (little-endian, the format's public specification; the reference parses the same layout in gguf_open,
// engine/faie2fn.cu:197-260): magic "GGUF", uint32 version, uint64 tensor count, uint64 metadata count; metadata
// entries (string key, uint32 value type, value); tensor infos (string name, uint32 dimension count, uint64 dims
// innermost first, uint32 ggml type, uint64 offset); padding to "general.alignment" (default 32); the data section.
// A string is a uint64 length and UTF-8 bytes; an array is a uint32 element type, a uint64 count and the elements.
//
// Tensors (the names the reference's loader reads for this architecture, engine/faie2fn.cu:2617-2657): token_embd,
// output, output_norm; per layer attn_norm, post_attention_norm; a gated-DeltaNet layer's attn_qkv, attn_gate,
// ssm_alpha, ssm_beta, ssm_out, ssm_conv1d, ssm_dt.bias, ssm_a, ssm_norm; a gated-attention layer's attn_q (query and
// gate rows interleaved per head), attn_k, attn_v, attn_output, attn_q_norm, attn_k_norm; the MoE's ffn_gate_inp with
// ffn_gate_inp_shexp (stacked under the router, as the reference's load_qw_cat does, :2651), ffn_gate_exps,
// ffn_up_exps, ffn_down_exps, ffn_gate_shexp, ffn_up_shexp, ffn_down_shexp. The layer kind follows from the tensors
// a layer has and the sizes from their shapes; the experts per token from <arch>.expert_used_count, eps and the RoPE
// base from <arch>.attention.layer_norm_rms_epsilon and <arch>.rope.freq_base. Files carrying the reference model's
// hyper-connection, PLE or indexer tensors are refused by name (no kernels here).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "faie2fn.h"
#include "fn_engine.h"

namespace fn {
namespace gguf {

struct Error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

enum { U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 };
constexpr uint32_t GGML_F32 = 0, GGML_F16 = 1;

struct Meta {
    bool is_num = false, is_str = false;
    double num = 0;
    std::string str;
};

struct Tensor {
    std::string name;
    uint32_t type = 0;
    std::vector<uint64_t> dims;
    const uint8_t *data = nullptr;
    uint64_t nbytes = 0;
    int64_t cols() const { return (int64_t)dims[0]; }
    int64_t rows() const {
        int64_t r = 1;
        for (size_t i = 1; i < dims.size(); ++i) r *= (int64_t)dims[i];
        return r;
    }
    std::string shape() const {
        std::string s = "[";
        for (size_t i = 0; i < dims.size(); ++i) s += (i ? ", " : "") + std::to_string(dims[i]);
        return s + "]";
    }
};

// a read-only memory map of one file
struct Map {
    void *p = nullptr;
    size_t n = 0;
    ~Map() {
        if (p && p != MAP_FAILED) munmap(p, n);
    }
};

static bool block_of(uint32_t t, int &qk, int &bytes) {
    if (t == GGML_F32) return qk = 1, bytes = 4, true;
    if (t == GGML_F16) return qk = 1, bytes = 2, true;
    return type_info(t, qk, bytes);
}

// well-formed UTF-8 (no overlong two-byte forms, continuation bytes where expected)
static bool utf8_ok(const uint8_t *s, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint8_t c = s[i];
        const int k = c < 0x80 ? 0 : (c >> 5) == 6 ? 1 : (c >> 4) == 14 ? 2 : (c >> 3) == 30 ? 3 : -1;
        if (k < 0 || (k == 1 && c < 0xC2) || i + (size_t)k >= n + (k == 0 ? 1 : 0)) return false;
        for (int j = 1; j <= k; ++j)
            if ((s[i + j] & 0xC0) != 0x80) return false;
        i += (size_t)k + 1;
    }
    return true;
}

class Cursor {
  public:
    Cursor(const uint8_t *b, size_t n, const std::string &path) : b_(b), n_(n), path_(path) {}
    size_t pos() const { return o_; }
    const uint8_t *take(size_t k) {
        if (k > n_ - o_) throw Error(path_ + ": truncated at byte " + std::to_string(o_));
        const uint8_t *p = b_ + o_;
        o_ += k;
        return p;
    }
    template <typename T> T scalar() {
        T v;
        std::memcpy(&v, take(sizeof(T)), sizeof(T));
        return v;
    }
    std::string string() {
        const uint64_t k = scalar<uint64_t>();
        const uint8_t *p = take(k);
        if (!utf8_ok(p, k)) throw Error(path_ + ": a string that is not UTF-8 at byte " + std::to_string(o_ - k));
        return std::string((const char *)p, k);
    }
    Meta value(uint32_t t) {
        Meta m;
        switch (t) {
            case U8: m.num = scalar<uint8_t>(); break;
            case I8: m.num = scalar<int8_t>(); break;
            case U16: m.num = scalar<uint16_t>(); break;
            case I16: m.num = scalar<int16_t>(); break;
            case U32: m.num = scalar<uint32_t>(); break;
            case I32: m.num = scalar<int32_t>(); break;
            case F32: m.num = scalar<float>(); break;
            case BOOL: m.num = scalar<uint8_t>(); break;
            case U64: m.num = (double)scalar<uint64_t>(); break;
            case I64: m.num = (double)scalar<int64_t>(); break;
            case F64: m.num = scalar<double>(); break;
            case STR:
                m.str = string();
                m.is_str = true;
                return m;
            case ARR: {
                const uint32_t et = scalar<uint32_t>();
                const uint64_t cnt = scalar<uint64_t>();
                if (et > F64) throw Error(path_ + ": bad array element type " + std::to_string(et));
                for (uint64_t i = 0; i < cnt; ++i) value(et);
                return m;
            }
            default: throw Error(path_ + ": bad metadata value type " + std::to_string(t));
        }
        m.is_num = true;
        return m;
    }

  private:
    const uint8_t *b_;
    size_t n_, o_ = 0;
    const std::string &path_;
};

// The tensors of one or two shards by name, with the checks the loader names a tensor in.
class Model {
  public:
    std::map<std::string, Meta> meta;
    std::map<std::string, Tensor> t;
    std::set<std::string> used;

    void read(const std::string &path) {
        const int fd = open(path.c_str(), O_RDONLY);
        if (fd < 0) throw std::runtime_error(path + ": " + std::strerror(errno));
        struct stat st;
        if (fstat(fd, &st) != 0) {
            close(fd);
            throw std::runtime_error(path + ": " + std::strerror(errno));
        }
        auto m = std::make_unique<Map>();
        m->n = (size_t)st.st_size;
        if (m->n < 24) {
            close(fd);
            throw Error(path + ": truncated at byte 0");
        }
        m->p = mmap(nullptr, m->n, PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (m->p == MAP_FAILED) throw std::runtime_error(path + ": cannot map the file");
        const uint8_t *b = (const uint8_t *)m->p;
        Cursor c(b, m->n, path);
        if (std::memcmp(c.take(4), "GGUF", 4) != 0) throw Error(path + ": not a GGUF file");
        const uint32_t ver = c.scalar<uint32_t>();
        if (ver != 2 && ver != 3) throw Error(path + ": GGUF version " + std::to_string(ver) + " not supported");
        const uint64_t n_t = c.scalar<uint64_t>(), n_kv = c.scalar<uint64_t>();
        std::map<std::string, Meta> fmeta;
        for (uint64_t i = 0; i < n_kv; ++i) {
            std::string k = c.string();
            fmeta[k] = c.value(c.scalar<uint32_t>());
        }
        struct Info {
            std::string name;
            std::vector<uint64_t> dims;
            uint32_t type;
            uint64_t off;
        };
        std::vector<Info> infos;
        for (uint64_t i = 0; i < n_t; ++i) {
            Info in;
            in.name = c.string();
            const uint32_t nd = c.scalar<uint32_t>();
            if (nd < 1 || nd > 4) throw Error(path + ": " + in.name + ": " + std::to_string(nd) + " dimensions");
            for (uint32_t d = 0; d < nd; ++d) in.dims.push_back(c.scalar<uint64_t>());
            in.type = c.scalar<uint32_t>();
            in.off = c.scalar<uint64_t>();
            infos.push_back(std::move(in));
        }
        uint64_t align = 32;
        if (fmeta.count("general.alignment")) {
            const double a = fmeta["general.alignment"].num;
            if (!(a > 0) || a > 1e9 || ((uint64_t)a & ((uint64_t)a - 1))) throw Error(path + ": bad alignment");
            align = (uint64_t)a;
        }
        const uint64_t base = (c.pos() + align - 1) / align * align;
        std::map<std::string, Tensor> ft;
        for (const Info &in : infos) {
            int qk, bytes;
            if (!block_of(in.type, qk, bytes)) throw Error("unsupported ggml type " + std::to_string(in.type));
            if (in.dims[0] % (uint64_t)qk)
                throw Error("row length " + std::to_string(in.dims[0]) + " is not a multiple of the block size of ggml type " +
                            std::to_string(in.type));
            uint64_t rows = 1;
            for (size_t d = 1; d < in.dims.size(); ++d) rows *= in.dims[d];
            const uint64_t n = rows * (in.dims[0] / qk) * bytes;
            if (in.off % align || base + in.off + n > m->n || base + in.off + n < base)
                throw Error(path + ": " + in.name + ": data out of range");
            if (ft.count(in.name)) throw Error(path + ": duplicate tensor " + in.name);
            Tensor x;
            x.name = in.name;
            x.type = in.type;
            x.dims = in.dims;
            x.data = b + base + in.off;
            x.nbytes = n;
            ft[in.name] = x;
        }
        for (auto &kv : fmeta) meta.emplace(kv.first, kv.second);  // the first shard's value wins
        for (auto &kv : ft) {
            if (t.count(kv.first)) throw Error("tensor " + kv.first + " in more than one shard");
            t[kv.first] = kv.second;
        }
        maps.push_back(std::move(m));
    }

    bool has(const std::string &name) const { return t.count(name) != 0; }

    // cols / rows < 0: any
    const Tensor &get(const std::string &name, int64_t cols = -1, int64_t rows = -1, bool quant = true) {
        auto it = t.find(name);
        if (it == t.end()) throw Error("missing tensor " + name);
        const Tensor &x = it->second;
        used.insert(name);
        if ((cols >= 0 && x.cols() != cols) || (rows >= 0 && x.rows() != rows))
            throw Error(name + ": shape " + x.shape() + ", expected " + (cols >= 0 ? std::to_string(cols) : "None") +
                        " columns x " + (rows >= 0 ? std::to_string(rows) : "None") + " rows");
        int qk, bytes;
        if (quant && (x.type == GGML_F32 || x.type == GGML_F16 || !type_info(x.type, qk, bytes)))
            throw Error(name + ": ggml type " + std::to_string(x.type) + " has no GEMV kernel");
        return x;
    }

    // an F32 / F16 tensor as float32 (n values per row, `rows` rows when given)
    std::vector<float> vec(const std::string &name, int64_t n, int64_t rows = -1) {
        const Tensor &x = get(name, n, rows, false);
        const size_t cnt = (size_t)x.rows() * (size_t)x.cols();
        std::vector<float> v(cnt);
        if (x.type == GGML_F32) {
            std::memcpy(v.data(), x.data, cnt * 4);
        } else if (x.type == GGML_F16) {
            for (size_t i = 0; i < cnt; ++i) {
                uint16_t h;
                std::memcpy(&h, x.data + 2 * i, 2);
                v[i] = half_to_float(h);
            }
        } else {
            throw Error(name + ": expected F32 or F16, got ggml type " + std::to_string(x.type));
        }
        return v;
    }

    double num(const std::string &key, double def) const {
        auto it = meta.find(key);
        return it != meta.end() && it->second.is_num ? it->second.num : def;
    }

  private:
    std::vector<std::unique_ptr<Map>> maps;

    static float half_to_float(uint16_t h) {  // IEEE binary16 -> binary32, exact
        const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
        uint32_t r;
        if (e == 0) {
            if (m == 0) {
                r = s;
            } else {  // subnormal: normalise
                int ee = -1;
                uint32_t mm = m;
                do {
                    ++ee;
                    mm <<= 1;
                } while (!(mm & 1024));
                r = s | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 1023) << 13);
            }
        } else if (e == 31) {
            r = s | 0x7F800000u | (m << 13);
        } else {
            r = s | ((e - 15 + 127) << 23) | (m << 13);
        }
        float f;
        std::memcpy(&f, &r, 4);
        return f;
    }
};

}  // namespace gguf

// ---------------------------------------------------------------------------------------------------------------
// the loaded model

constexpr int RUN_DS = 128, RUN_HD = 256, RUN_MAXT = 8;  // head sizes; tokens per forward call (engine/faie2fn.cu:67)
static const char *kUnsupported[] = {"hc_", "ple_", "indexer.", "per_layer_token_embd", "output_hc_"};

struct Runner {
    int dev = 0;
    int D = 0, V = 0, layers = 0, nkh = 0, nvh = 0, nh = 0, nkv = 0, ne = 0, k = 0, ffe = 0;
    float eps = 1e-6f;
    double rope_base = 1e7;
    std::string pattern;
    uint32_t embed_type = 0;
    std::vector<int> w, moe, gdn;  // handles to free
    int head = 0, dec = 0;
    std::vector<void *> bufs;  // device allocations to free
    float *hidden = nullptr, *logits = nullptr;
    int *tokens = nullptr, *pos = nullptr, *next = nullptr, *plen = nullptr;
    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool use_graphs = true;
    float *dbg = nullptr;
    int max_ctx = 0, n_past = 0, split = 0;
    double last_ms = -1.0, bytes = 0;
    int *am_h = nullptr;     // pinned [8]
    float *lg_h = nullptr;   // pinned [8][vocab]
    int *tok_h = nullptr;    // pinned [8 + 1]: the call's token ids, then the prompt length

    void *alloc(size_t n) {
        void *p = nullptr;
        if (cudaMalloc(&p, n) != cudaSuccess) throw std::runtime_error("device allocation failed");
        bufs.push_back(p);
        if (cudaMemset(p, 0, n) != cudaSuccess) throw std::runtime_error("device memset failed");
        return p;
    }
    template <typename T> T *upload(const T *src, size_t n) {
        T *p = (T *)alloc(n * sizeof(T));
        if (cudaMemcpy(p, src, n * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess)
            throw std::runtime_error("upload failed");
        return p;
    }
    int wcreate(uint32_t type, const uint8_t *raw, int rows, int cols) {
        const int h = fn_w_create(type, raw, rows, cols);
        if (h < 0) throw std::runtime_error(err());
        w.push_back(h);
        return h;
    }
    void drop_graph() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        exec = nullptr;
        graph = nullptr;
    }
    ~Runner() {
        if (stream) cudaStreamSynchronize(stream);
        drop_graph();
        if (dec) fn_decoder_free(dec);
        for (int h : w) fn_w_free(h);
        for (int h : moe) fn_moe_free(h);
        for (int h : gdn) fn_gdn_free(h);
        for (void *p : bufs) cudaFree(p);
        if (am_h) cudaFreeHost(am_h);
        if (lg_h) cudaFreeHost(lg_h);
        if (tok_h) cudaFreeHost(tok_h);
        if (stream) cudaStreamDestroy(stream);
    }
};
static Runner *g_run = nullptr;

static std::vector<uint8_t> cat_rows(const gguf::Tensor &a, const gguf::Tensor &b) {
    std::vector<uint8_t> v(a.nbytes + b.nbytes);
    std::memcpy(v.data(), a.data, a.nbytes);
    std::memcpy(v.data() + a.nbytes, b.data, b.nbytes);
    return v;
}
static std::vector<uint8_t> cat_rows3(const gguf::Tensor &a, const gguf::Tensor &b, const gguf::Tensor &c) {
    std::vector<uint8_t> v(a.nbytes + b.nbytes + c.nbytes);
    std::memcpy(v.data(), a.data, a.nbytes);
    std::memcpy(v.data() + a.nbytes, b.data, b.nbytes);
    std::memcpy(v.data() + a.nbytes + b.nbytes, c.data, c.nbytes);
    return v;
}

// reset the sequence: tokens, position and prompt length zeroed, every DeltaNet state and conv history zeroed
static int runner_reset(Runner &r) {
    FN_CK(cudaMemsetAsync(r.tokens, 0, (size_t)r.max_ctx * 4, r.stream));
    FN_CK(cudaMemsetAsync(r.pos, 0, 4, r.stream));
    FN_CK(cudaMemsetAsync(r.plen, 0, 4, r.stream));
    for (int g : r.gdn)
        if (fn_gdn_reset(g, r.stream)) return -1;
    if (fn_sync(r.stream)) return -1;
    r.n_past = 0;
    return 0;
}

// the step captured as a CUDA graph; eager_first (at load): one eager step first, which sets the kernels' attributes
// outside a capture, then the sequence reset (a capture alone executes nothing, so a later one keeps the sequence)
static int runner_capture(Runner &r, bool eager_first) {
    r.drop_graph();
    if (eager_first) {
        FN_CK(cudaMemsetAsync(r.pos, 0, 4, r.stream));
        if (fn_decoder_step(r.dec, r.stream, nullptr, 0) || fn_sync(r.stream)) return -1;
    }
    FN_CK(cudaStreamBeginCapture(r.stream, cudaStreamCaptureModeThreadLocal));
    const int rc = fn_decoder_step(r.dec, r.stream, nullptr, 0);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(r.stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return -1;
    }
    FN_CK(e);
    r.graph = g;
    FN_CK(cudaGraphInstantiate(&r.exec, g, 0));
    return eager_first ? runner_reset(r) : 0;
}

static void runner_build(Runner &r, gguf::Model &M, int max_ctx) {
    using gguf::Error;
    std::vector<std::string> bad;
    for (auto &kv : M.t)
        for (const char *u : kUnsupported)
            if (kv.first.rfind(u, 0) == 0 || kv.first.find(std::string(".") + u) != std::string::npos) {
                bad.push_back(kv.first);
                break;
            }
    if (!bad.empty()) {
        std::string s = "tensors this runner has no kernels for: ";
        for (size_t i = 0; i < bad.size() && i < 4; ++i) s += (i ? ", " : "") + bad[i];
        throw Error(s + (bad.size() > 4 ? " ..." : ""));
    }
    auto am = M.meta.find("general.architecture");
    const std::string arch = am != M.meta.end() && am->second.is_str ? am->second.str : "qwen3next";
    const gguf::Tensor &emb = M.get("token_embd.weight");
    const int D = (int)emb.cols(), V = (int)emb.rows();
    const gguf::Tensor &head = M.get("output.weight", D, V);
    std::set<int> idx;
    for (auto &kv : M.t) {
        const std::string &n = kv.first;
        if (n.rfind("blk.", 0) != 0) continue;
        size_t j = 4;
        while (j < n.size() && isdigit((unsigned char)n[j])) ++j;
        if (j > 4 && j < n.size() && n[j] == '.') idx.insert(std::stoi(n.substr(4, j - 4)));
    }
    if (idx.empty() || *idx.rbegin() != (int)idx.size() - 1) throw Error("layers blk.0 .. blk.N-1 expected");
    if (!M.meta.count(arch + ".expert_used_count")) throw Error("missing metadata " + arch + ".expert_used_count");
    const int k = (int)M.num(arch + ".expert_used_count", 0);

    struct LayerSpec {
        char kind;
        const gguf::Tensor *qkv = nullptr, *z = nullptr, *al = nullptr, *be = nullptr, *out = nullptr;
        const gguf::Tensor *q = nullptr, *kk = nullptr, *v = nullptr, *o = nullptr;
        const gguf::Tensor *r = nullptr, *rs = nullptr, *ge = nullptr, *ue = nullptr, *de = nullptr, *gs = nullptr,
                           *us = nullptr, *ds = nullptr;
        std::vector<float> norm1, norm2, conv_w, dt_bias, ssm_a, gnorm, q_norm, k_norm;
    };
    std::vector<LayerSpec> Ls;
    int nkh = -1, nvh = -1, nh = -1, nkv = -1, ne = -1, ffe = -1;
    for (int l = 0; l < (int)idx.size(); ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        LayerSpec L;
        L.norm1 = M.vec(p + "attn_norm.weight", D);
        L.norm2 = M.vec(p + "post_attention_norm.weight", D);
        if (M.has(p + "attn_q.weight")) {
            L.kind = 'A';
            L.q = &M.get(p + "attn_q.weight", D);
            L.kk = &M.get(p + "attn_k.weight", D);
            if (L.q->rows() % (2 * RUN_HD) || L.kk->rows() % RUN_HD)
                throw Error(p + "attn_q / attn_k: head size " + std::to_string(RUN_HD) + " expected");
            nh = (int)(L.q->rows() / (2 * RUN_HD));
            nkv = (int)(L.kk->rows() / RUN_HD);
            L.v = &M.get(p + "attn_v.weight", D, (int64_t)nkv * RUN_HD);
            L.o = &M.get(p + "attn_output.weight", (int64_t)nh * RUN_HD, D);
            L.q_norm = M.vec(p + "attn_q_norm.weight", RUN_HD);
            L.k_norm = M.vec(p + "attn_k_norm.weight", RUN_HD);
        } else {
            L.kind = 'G';
            const gguf::Tensor &a = M.get(p + "ssm_a", -1, -1, false);
            nvh = (int)a.cols();
            L.qkv = &M.get(p + "attn_qkv.weight", D);
            const int64_t qr = L.qkv->rows();
            if ((qr - (int64_t)nvh * RUN_DS) % (2 * RUN_DS) || qr <= (int64_t)nvh * RUN_DS)
                throw Error(p + "attn_qkv: " + std::to_string(qr) + " rows do not fit " + std::to_string(nvh) +
                            " value heads of " + std::to_string(RUN_DS));
            nkh = (int)((qr - (int64_t)nvh * RUN_DS) / (2 * RUN_DS));
            L.z = &M.get(p + "attn_gate.weight", D, (int64_t)nvh * RUN_DS);
            L.al = &M.get(p + "ssm_alpha.weight", D, nvh);
            L.be = &M.get(p + "ssm_beta.weight", D, nvh);
            L.out = &M.get(p + "ssm_out.weight", (int64_t)nvh * RUN_DS, D);
            if (L.qkv->type != L.z->type || L.al->type != L.be->type)
                throw Error(p + "attn_qkv / attn_gate (or ssm_alpha / ssm_beta) in different formats");
            L.conv_w = M.vec(p + "ssm_conv1d.weight", 4, qr);
            L.dt_bias = M.vec(p + "ssm_dt.bias", nvh);
            L.ssm_a = M.vec(p + "ssm_a", nvh);
            L.gnorm = M.vec(p + "ssm_norm.weight", RUN_DS);
        }
        L.r = &M.get(p + "ffn_gate_inp.weight", D);
        const int lne = (int)L.r->rows();
        L.rs = &M.get(p + "ffn_gate_inp_shexp.weight", D, 1);
        L.ge = &M.get(p + "ffn_gate_exps.weight", D);
        if (L.ge->rows() % lne)
            throw Error(p + "ffn_gate_exps: " + std::to_string(L.ge->rows()) + " rows for " + std::to_string(lne) + " experts");
        const int lffe = (int)(L.ge->rows() / lne);
        L.ue = &M.get(p + "ffn_up_exps.weight", D, (int64_t)lne * lffe);
        L.de = &M.get(p + "ffn_down_exps.weight", lffe, (int64_t)lne * D);
        L.gs = &M.get(p + "ffn_gate_shexp.weight", D, lffe);
        L.us = &M.get(p + "ffn_up_shexp.weight", D, lffe);
        L.ds = &M.get(p + "ffn_down_shexp.weight", lffe, D);
        if (L.r->type != L.rs->type) throw Error(p + "ffn_gate_inp / ffn_gate_inp_shexp in different formats");
        if (L.ge->type != L.ue->type || L.ge->type != L.gs->type || L.ge->type != L.us->type || L.de->type != L.ds->type)
            throw Error(p + "expert gate / up (or down) tensors in different formats");
        if (ne < 0) {
            ne = lne;
            ffe = lffe;
        } else if (ne != lne || ffe != lffe) {
            throw Error(p + ": expert count or size differs between layers");
        }
        Ls.push_back(std::move(L));
    }
    if (nkh < 0 || nh < 0) throw Error("a model with both gated-DeltaNet and attention layers expected");
    std::vector<float> final_norm = M.vec("output_norm.weight", D);
    std::vector<std::string> unused;
    for (auto &kv : M.t)
        if (!M.used.count(kv.first)) unused.push_back(kv.first);
    if (!unused.empty()) {
        std::string s = "tensors this runner does not use: ";
        for (size_t i = 0; i < unused.size() && i < 4; ++i) s += (i ? ", " : "") + unused[i];
        throw Error(s);
    }
    if (k < 1 || k > std::min(ne, 16)) throw Error(arch + ".expert_used_count " + std::to_string(k) + " out of range");

    // ---- device work from here on
    r.D = D;
    r.V = V;
    r.layers = (int)Ls.size();
    r.nkh = nkh;
    r.nvh = nvh;
    r.nh = nh;
    r.nkv = nkv;
    r.ne = ne;
    r.k = k;
    r.ffe = ffe;
    r.eps = (float)M.num(arch + ".attention.layer_norm_rms_epsilon", 1e-6);
    r.rope_base = M.num(arch + ".rope.freq_base", 1e7);
    r.max_ctx = max_ctx;
    r.split = r.layers;
    r.embed_type = emb.type;
    for (auto &kv : M.t) r.bytes += (double)kv.second.nbytes;
    if (cudaGetDevice(&r.dev) != cudaSuccess) throw std::runtime_error("no CUDA device");
    if (cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking) != cudaSuccess)
        throw std::runtime_error("stream creation failed");

    // a decode step is a chain of dependent GEMVs at batch 1: 16 warps per CTA (more loads in flight per SM)
    struct Tune {
        Tune() { fn_gemv_tune(16, 0, 0, 0); }
        ~Tune() { fn_gemv_tune(0, 0, 0, 0); }
    } tune;
    const uint8_t *E = r.upload(emb.data, (size_t)emb.nbytes);
    r.head = r.wcreate(head.type, head.data, V, D);
    std::vector<fn_layer_t> layers(Ls.size());
    const int convch = 2 * nkh * RUN_DS + nvh * RUN_DS;
    int proj_rows = 0;
    for (size_t l = 0; l < Ls.size(); ++l) {
        LayerSpec &L = Ls[l];
        fn_layer_t &o = layers[l];
        std::memset(&o, 0, sizeof(o));
        o.norm1 = r.upload(L.norm1.data(), L.norm1.size());
        o.norm2 = r.upload(L.norm2.data(), L.norm2.size());
        if (L.kind == 'G') {
            o.kind = 0;
            const int rin = convch + nvh * RUN_DS;
            const std::vector<uint8_t> in = cat_rows(*L.qkv, *L.z);
            if (L.qkv->type == L.al->type) {  // [q k v z | alpha beta] as one GEMV
                std::vector<uint8_t> all = in;
                const std::vector<uint8_t> ab = cat_rows(*L.al, *L.be);
                all.insert(all.end(), ab.begin(), ab.end());
                o.w_in[0] = r.wcreate(L.qkv->type, all.data(), rin + 2 * nvh, D);
                o.w_in_rows[0] = rin + 2 * nvh;
            } else {
                o.w_in[0] = r.wcreate(L.qkv->type, in.data(), rin, D);
                o.w_in_rows[0] = rin;
                const std::vector<uint8_t> ab = cat_rows(*L.al, *L.be);
                o.w_in[1] = r.wcreate(L.al->type, ab.data(), 2 * nvh, D);
                o.w_in_rows[1] = 2 * nvh;
            }
            proj_rows = std::max(proj_rows, rin + 2 * nvh);
            o.w_out = r.wcreate(L.out->type, L.out->data, D, nvh * RUN_DS);
            const std::vector<float> S0((size_t)nvh * RUN_DS * RUN_DS, 0.f), c0((size_t)3 * convch, 0.f);
            const int g = fn_gdn_create(nkh, nvh, RUN_DS, L.conv_w.data(), L.dt_bias.data(), L.ssm_a.data(),
                                        L.gnorm.data(), S0.data(), c0.data());
            if (g < 0) throw std::runtime_error(err());
            r.gdn.push_back(g);
            o.gdn = g;
        } else {
            o.kind = 1;
            const int rq = nh * 2 * RUN_HD, rk = nkv * RUN_HD;
            if (L.q->type == L.kk->type && L.q->type == L.v->type) {  // [q gate | k | v] as one GEMV
                const std::vector<uint8_t> all = cat_rows3(*L.q, *L.kk, *L.v);
                o.w_in[0] = r.wcreate(L.q->type, all.data(), rq + 2 * rk, D);
                o.w_in_rows[0] = rq + 2 * rk;
            } else {
                o.w_in[0] = r.wcreate(L.q->type, L.q->data, rq, D);
                o.w_in[1] = r.wcreate(L.kk->type, L.kk->data, rk, D);
                o.w_in[2] = r.wcreate(L.v->type, L.v->data, rk, D);
                o.w_in_rows[0] = rq;
                o.w_in_rows[1] = o.w_in_rows[2] = rk;
            }
            proj_rows = std::max(proj_rows, rq + 2 * rk);
            o.w_out = r.wcreate(L.o->type, L.o->data, D, nh * RUN_HD);
            o.q_norm = r.upload(L.q_norm.data(), L.q_norm.size());
            o.k_norm = r.upload(L.k_norm.data(), L.k_norm.size());
            o.Kc = (float *)r.alloc((size_t)max_ctx * nkv * RUN_HD * 4);
            o.Vc = (float *)r.alloc((size_t)max_ctx * nkv * RUN_HD * 4);
        }
        const std::vector<uint8_t> rt = cat_rows(*L.r, *L.rs);
        o.router = r.wcreate(L.r->type, rt.data(), ne + 1, D);
        const int m = fn_moe_create(L.ge->type, L.de->type, ne, k, ffe, D, L.ge->data, L.ue->data, L.de->data, L.gs->data,
                                    L.us->data, L.ds->data);
        if (m < 0) throw std::runtime_error(err());
        r.moe.push_back(m);
        o.moe = m;
    }
    std::vector<float> inv(32);
    for (int i = 0; i < 32; ++i) inv[i] = (float)(1.0 / std::pow(r.rope_base, 2.0 * i / 64.0));
    fn_model_t mm;
    std::memset(&mm, 0, sizeof(mm));
    mm.D = D;
    mm.nkh = nkh;
    mm.nvh = nvh;
    mm.nh = nh;
    mm.nkv = nkv;
    mm.ne = ne;
    mm.vocab = V;
    mm.max_ctx = max_ctx;
    mm.eps = r.eps;
    mm.embed_type = emb.type;
    mm.embed = E;
    mm.head = r.head;
    mm.final_norm = r.upload(final_norm.data(), final_norm.size());
    mm.inv_freq = r.upload(inv.data(), inv.size());
    mm.fuse_norm = 1;
    mm.prefetch = 1;
    mm.hidden = r.hidden = (float *)r.alloc((size_t)D * 4);
    mm.proj = (float *)r.alloc((size_t)proj_rows * 4);
    mm.core = (float *)r.alloc((size_t)nvh * RUN_DS * 4);
    mm.Q = (float *)r.alloc((size_t)nh * RUN_HD * 4);
    mm.att = (float *)r.alloc((size_t)nh * RUN_HD * 4);
    mm.router_out = (float *)r.alloc((size_t)(ne + 1) * 4);
    mm.logits = r.logits = (float *)r.alloc((size_t)V * 4);
    mm.tokens = r.tokens = (int *)r.alloc((size_t)max_ctx * 4);
    mm.pos = r.pos = (int *)r.alloc(4);
    mm.next = r.next = (int *)r.alloc(4);
    mm.prompt_len = r.plen = (int *)r.alloc(4);
    r.dec = fn_decoder_create(&mm, layers.data(), (int)layers.size());
    if (r.dec < 0) {
        r.dec = 0;
        throw std::runtime_error(err());
    }
    if (cudaMallocHost(&r.am_h, RUN_MAXT * 4) != cudaSuccess ||
        cudaMallocHost(&r.lg_h, (size_t)RUN_MAXT * V * 4) != cudaSuccess ||
        cudaMallocHost(&r.tok_h, (RUN_MAXT + 1) * 4) != cudaSuccess)
        throw std::runtime_error("pinned host allocation failed");
    if (runner_capture(r, true)) throw std::runtime_error(err());
}

static int runner_forward(Runner &r, const int *tokens, int nt, float *logits, int *argmax) {
    if (nt < 1 || nt > RUN_MAXT) return fail("nt out of range");
    if (!tokens) return fail("no tokens");
    if (r.n_past + nt > r.max_ctx) return fail("context full");
    for (int i = 0; i < nt; ++i)
        if (tokens[i] < 0 || tokens[i] >= r.V) return fail("token id out of range");
    const auto t0 = std::chrono::steady_clock::now();
    if (cudaSetDevice(r.dev) != cudaSuccess) return fail("fn_forward: no CUDA device");
    const bool graphs = r.use_graphs && !r.dbg;
    if (graphs && !r.exec && runner_capture(r, false)) return -1;  // dropped by fn_use_graphs: capture again
    std::memcpy(r.tok_h, tokens, (size_t)nt * 4);
    r.tok_h[RUN_MAXT] = r.n_past + nt;  // the step keeps these ids: it writes its argmax only past the prompt
    FN_CK(cudaMemcpyAsync(r.tokens + r.n_past, r.tok_h, (size_t)nt * 4, cudaMemcpyHostToDevice, r.stream));
    FN_CK(cudaMemcpyAsync(r.plen, r.tok_h + RUN_MAXT, 4, cudaMemcpyHostToDevice, r.stream));
    for (int i = 0; i < nt; ++i) {
        if (graphs) {
            FN_CK(cudaGraphLaunch(r.exec, r.stream));
        } else if (fn_decoder_step(r.dec, r.stream, r.dbg ? r.dbg + (size_t)i * r.D : nullptr, (int64_t)nt * r.D)) {
            return -1;
        }
        FN_CK(cudaMemcpyAsync(r.am_h + i, r.next, 4, cudaMemcpyDeviceToHost, r.stream));
        if (logits) FN_CK(cudaMemcpyAsync(r.lg_h + (size_t)i * r.V, r.logits, (size_t)r.V * 4, cudaMemcpyDeviceToHost, r.stream));
    }
    if (fn_sync(r.stream)) return -1;
    if (argmax) std::memcpy(argmax, r.am_h, (size_t)nt * 4);
    if (logits) std::memcpy(logits, r.lg_h, (size_t)nt * r.V * 4);
    r.n_past += nt;
    r.last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return 0;
}

}  // namespace fn

using namespace fn;

FN_API void fn_free() {
    delete g_run;
    g_run = nullptr;
}

FN_API int fn_load(const char *shard1, const char *shard2, int max_ctx, int split) {
    (void)split;  // every layer stays on the current GPU (one B200 holds the model); fn_split reads the layer count
    fn_free();
    if (!shard1 || !*shard1) return fail("no model file");
    if (max_ctx < 1) return fail("max_ctx out of range");
    try {
        gguf::Model M;
        M.read(shard1);
        if (shard2 && *shard2) M.read(shard2);
        Runner *r = new Runner();
        try {
            runner_build(*r, M, max_ctx);
        } catch (...) {
            delete r;
            throw;
        }
        g_run = r;
        return 0;
    } catch (const std::exception &e) {
        return fail(e.what());
    }
}

FN_API int fn_forward(const int *tokens, int nt, float *logits, int *argmax) {
    if (!g_run) return fail("not loaded");
    return runner_forward(*g_run, tokens, nt, logits, argmax);
}

FN_API int fn_reset() {
    if (!g_run) return fail("not loaded");
    if (cudaSetDevice(g_run->dev) != cudaSuccess) return fail("fn_reset: no CUDA device");
    return runner_reset(*g_run);
}

// the residual after every layer of the following forwards into out[layers][nt][D] (host); NULL turns it off
FN_API int fn_debug_layers(float *out) {
    if (!g_run) return fail("not loaded");
    g_run->dbg = out;
    return 0;
}

// graphs on / off; the captured graph is dropped either way and captured again (from a reset sequence) at the next
// forward that uses it, so settings changed since (fn_pdl, fn_moe_var, ...) apply
FN_API int fn_use_graphs(int on) {
    if (!g_run) return fail("not loaded");
    if (cudaSetDevice(g_run->dev) != cudaSuccess) return fail("fn_use_graphs: no CUDA device");
    cudaStreamSynchronize(g_run->stream);
    g_run->drop_graph();
    g_run->use_graphs = on != 0;
    return 0;
}

// Sizes of the loaded model: out[4] = {vocab, hidden size D, layers, max_ctx} (the reference's fn.py keeps them as
// module constants, VOCAB / HCD / NL, flashnext/fn.py:11-13; no counterpart symbol).
FN_API int fn_model_dims(int *out) {
    if (!g_run) return fail("not loaded");
    out[0] = g_run->V;
    out[1] = g_run->D;
    out[2] = g_run->layers;
    out[3] = g_run->max_ctx;
    return 0;
}

FN_API int fn_n_past() { return g_run ? g_run->n_past : -1; }
FN_API double fn_last_ms() { return g_run ? g_run->last_ms : -1.0; }
FN_API double fn_dev_gb(int dv) { return g_run ? (dv == 0 ? g_run->bytes / 1e9 : 0.0) : -1.0; }
FN_API int fn_split() { return g_run ? g_run->split : -1; }
