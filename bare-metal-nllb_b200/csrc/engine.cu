// engine.cu -- sentence-batched translation on one GPU (include/nllb_translate.h).
//
// Host side: safetensors loading, the forward passes as kernel sequences and
// the beam search bookkeeping, restating the reference engine's control flow
// (main.c:294-528, encoder.c:250-287, decoder.c:156-233) for many sentences
// in lockstep.  Device side: engine_kernels.cu plus the attention kernels.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <string>
#include <vector>

#include <cuda_fp16.h>

#include "attn_internal.h"
#include "engine_kernels.h"
#include "planes.cuh"
#include "nllb_translate.h"

using namespace nllb;

namespace nllb {
int set_error(int status, const std::string& msg);  // nllb_attn.cu
}

namespace {

constexpr int D = 1024, H = 16, FFN = 4096, LAYERS = 12, VOCAB = 256206, NB = 4;
constexpr int VOCAB_LD = (VOCAB + 3) & ~3;  // row stride of the logits: rows start 16-byte aligned
constexpr int LANG_START = 256000;

#define ENG_CK(call)                                                                              \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess)                                                                    \
            return nllb::set_error(NLLB_ATTN_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)
#define ENG_RC(call)                 \
    do {                             \
        int r_ = (call);             \
        if (r_ != NLLB_ATTN_OK) return r_; \
    } while (0)

// ---- safetensors header: {"name": {"dtype": .., "shape": [..], "data_offsets": [a, b]}, ...}
struct TensorInfo {
    std::string dtype;
    std::vector<long long> shape;
    long long begin = 0, end = 0;
};

class HeaderParser {
  public:
    explicit HeaderParser(const std::string& s) : s_(s) {}
    bool parse(std::map<std::string, TensorInfo>* out) {
        skip();
        if (!eat('{')) return false;
        skip();
        if (peek() == '}') return true;
        for (;;) {
            std::string name;
            if (!str(&name)) return false;
            skip();
            if (!eat(':')) return false;
            TensorInfo ti;
            bool is_tensor = false;
            if (!object(&ti, &is_tensor)) return false;
            if (is_tensor) (*out)[name] = ti;
            skip();
            if (eat(',')) {
                skip();
                continue;
            }
            return eat('}');
        }
    }

  private:
    const std::string& s_;
    size_t i_ = 0;
    char peek() const { return i_ < s_.size() ? s_[i_] : '\0'; }
    void skip() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\t' || s_[i_] == '\r')) ++i_;
    }
    bool eat(char c) {
        skip();
        if (peek() != c) return false;
        ++i_;
        return true;
    }
    bool str(std::string* o) {
        skip();
        if (!eat('"')) return false;
        while (i_ < s_.size() && s_[i_] != '"') {
            if (s_[i_] == '\\' && i_ + 1 < s_.size()) ++i_;
            o->push_back(s_[i_++]);
        }
        return eat('"');
    }
    bool number(long long* v) {
        skip();
        size_t j = i_;
        if (peek() == '-') ++i_;
        while (i_ < s_.size() && (isdigit((unsigned char)s_[i_]) || s_[i_] == '.' || s_[i_] == 'e' ||
                                  s_[i_] == 'E' || s_[i_] == '+' || s_[i_] == '-'))
            ++i_;
        if (j == i_) return false;
        *v = std::stoll(s_.substr(j, i_ - j));
        return true;
    }
    bool int_list(std::vector<long long>* o) {
        if (!eat('[')) return false;
        skip();
        if (eat(']')) return true;
        for (;;) {
            long long v;
            if (!number(&v)) return false;
            o->push_back(v);
            if (eat(',')) continue;
            return eat(']');
        }
    }
    bool skip_value() {  // strings, numbers, flat objects/arrays of those
        skip();
        const char c = peek();
        if (c == '"') {
            std::string t;
            return str(&t);
        }
        if (c == '{' || c == '[') {
            const char close = (c == '{') ? '}' : ']';
            ++i_;
            int depth = 1;
            bool in_str = false;
            while (i_ < s_.size() && depth > 0) {
                const char d = s_[i_++];
                if (in_str) {
                    if (d == '\\') ++i_;
                    else if (d == '"') in_str = false;
                } else if (d == '"') {
                    in_str = true;
                } else if (d == '{' || d == '[') {
                    ++depth;
                } else if (d == '}' || d == ']') {
                    --depth;
                }
            }
            (void)close;
            return depth == 0;
        }
        long long v;
        return number(&v);
    }
    bool object(TensorInfo* ti, bool* is_tensor) {
        skip();
        if (peek() != '{') return skip_value();
        ++i_;
        skip();
        if (eat('}')) return true;
        for (;;) {
            std::string key;
            if (!str(&key)) return false;
            if (!eat(':')) return false;
            if (key == "dtype") {
                if (!str(&ti->dtype)) return false;
            } else if (key == "shape") {
                if (!int_list(&ti->shape)) return false;
            } else if (key == "data_offsets") {
                std::vector<long long> o;
                if (!int_list(&o) || o.size() != 2) return false;
                ti->begin = o[0];
                ti->end = o[1];
                *is_tensor = true;
            } else if (!skip_value()) {
                return false;
            }
            if (eat(',')) continue;
            return eat('}');
        }
    }
};

struct Lin {
    int8_t* w = nullptr;
    float* scale = nullptr;  // CT2 weight_scale (weight = int8 / scale)
    float* b = nullptr;
    int out = 0, in = 0;
    void* wb = nullptr;  // fp16 copy of w (exact), operand of the TMA-fed tensor-core kernel
    CUtensorMap tm{};    // tensor map of wb: [out][in], box 64 x 128, 128-byte swizzle
    CUtensorMap tm256{}; // the same, box 32 x 256, 64-byte swizzle (persistent kernel)
    CUtensorMap tm_pair{};  // the same, box 32 x 128, 64-byte swizzle (persistent kernel on CTA pairs)
};

}  // namespace

struct nllb_model {
    int device = 0;
    int max_sentences = 0, max_src = 0, max_gen = 0;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
    int8_t* emb = nullptr;
    float* emb_scale = nullptr;  // per-row weight_scale of the shared embedding
    float* emb_inv = nullptr;    // 1 / emb_scale, for the embedding lookup (tensor.c:37-40)
    struct Enc {
        Lin qkv, out, fc1, fc2;
        float *ln1g, *ln1b, *ln2g, *ln2b;
    } enc[LAYERS];
    struct Dec {
        Lin qkv, out, xq, xkv, xout, fc1, fc2;
        float *ln1g, *ln1b, *ln2g, *ln2b, *ln3g, *ln3b;
    } dec[LAYERS];
    float *enc_lng = nullptr, *enc_lnb = nullptr, *dec_lng = nullptr, *dec_lnb = nullptr;
    float* pos_table = nullptr;  // row p: sinusoid of actual position p (encoder.c:27-36)
    int pos_rows = 0;
    nllb_attn_ctx* attn = nullptr;
    LinearWorkspace lws;  // split-K workspace of the tensor-core linear kernel
    Lin vocab;            // tied output projection: the shared embedding (decoder.c:319-354)
    // activations split into fp16 planes for the TMA-fed linear kernel ([2][M][K]),
    // grow-only, with its tensor maps per (M, K)
    // (two buffers: a GEMM that writes planes for the next one reads the other)
    void* planes = nullptr;
    void* planes2 = nullptr;
    size_t planes_elems = 0;
    // tensor maps of the plane buffers, key (buffer, M, K, persistent kernel)
    std::map<std::tuple<const void*, int, int, bool>, CUtensorMap> plane_maps;
    int* live_h = nullptr;          // pinned [max_gen]: running sentences after each step
    cudaEvent_t step_ev[4] = {};    // recorded after each step's count copy
    // buffers of translate calls, kept between calls (grow-only, taken in call order)
    std::vector<std::pair<void*, size_t>> work_pool;
    int num_sms = 148;
    // decision margins of the last translate call, [sentence][step]
    std::vector<std::vector<float>> margins;
    // per-kernel-class profile (nllb_translate_profile): CUDA events around
    // each launch of a class on the engine's stream, resolved after each call
    struct ProfRec {
        int cat;
        cudaEvent_t a, b;
        double flops, bytes;
    };
    bool prof_on = false;
    std::vector<cudaEvent_t> prof_events;  // pool, reused call after call
    size_t prof_next = 0;
    std::vector<ProfRec> prof_recs;
    nllb_kernel_profile prof_agg[NLLB_PROF_CLASSES] = {};
};

namespace {

template <typename T>
int dev_alloc(nllb_model* m, T** p, size_t count) {
    void* v = nullptr;
    ENG_CK(cudaMalloc(&v, std::max<size_t>(count, 1) * sizeof(T)));
    m->allocs.push_back(v);
    *p = static_cast<T*>(v);
    return NLLB_ATTN_OK;
}

const char* const kProfNames[NLLB_PROF_CLASSES] = {
    "gemm_persistent", "gemm_cluster_splitk", "linear_simt_or_tc", "decode_self", "cross",
    "prefill",         "logsoftmax_topk",     "penalties",         "beam_select", "reorder",
    "layernorm",       "embed_pos",           "split_planes",      "set_memory"};

// Times the launches made in its scope as one record of class `cat` (a no-op
// unless profiling is on).  The events order the stream around the scope, so
// a profiled call runs without dependent-launch overlap at those points.
struct ProfScope {
    nllb_model* m;
    int cat;
    double flops, bytes;
    cudaEvent_t b = nullptr;
    ProfScope(nllb_model* m_, int cat_, double flops_ = 0, double bytes_ = 0)
        : m(m_), cat(cat_), flops(flops_), bytes(bytes_) {
        if (!m->prof_on) return;
        cudaEvent_t a = next_event();
        b = next_event();
        if (a && b && cudaEventRecord(a, m->stream) == cudaSuccess)
            m->prof_recs.push_back({cat, a, b, flops, bytes});
        else
            b = nullptr;
    }
    ~ProfScope() {
        if (b) cudaEventRecord(b, m->stream);
    }
    cudaEvent_t next_event() {
        if (m->prof_next == m->prof_events.size()) {
            cudaEvent_t e = nullptr;
            if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
            m->prof_events.push_back(e);
        }
        return m->prof_events[m->prof_next++];
    }
};

// Fold the records of the last call into the totals (after the stream has drained).
void prof_resolve(nllb_model* m) {
    for (const auto& r : m->prof_recs) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) continue;
        nllb_kernel_profile& g = m->prof_agg[r.cat];
        g.launches += 1;
        g.ms += ms;
        g.flops += r.flops;
        g.bytes += r.bytes;
    }
    m->prof_recs.clear();
    m->prof_next = 0;
}

struct Loader {
    nllb_model* m;
    const uint8_t* data;
    std::map<std::string, TensorInfo> tensors;

    int find(const std::string& name, const char* dtype, long long elems, const TensorInfo** out) {
        auto it = tensors.find(name);
        if (it == tensors.end()) return nllb::set_error(NLLB_ATTN_EINVAL, "tensor missing: " + name);
        long long n = 1;
        for (long long s : it->second.shape) n *= s;
        if (it->second.dtype != dtype || n != elems)
            return nllb::set_error(NLLB_ATTN_EINVAL, "unexpected dtype/shape: " + name);
        *out = &it->second;
        return NLLB_ATTN_OK;
    }
    template <typename T>
    int upload(const std::string& name, const char* dtype, long long elems, T** dst) {
        const TensorInfo* ti;
        ENG_RC(find(name, dtype, elems, &ti));
        ENG_RC(dev_alloc(m, dst, (size_t)elems));
        ENG_CK(cudaMemcpy(*dst, data + ti->begin, (size_t)elems * sizeof(T), cudaMemcpyHostToDevice));
        return NLLB_ATTN_OK;
    }
    // weight, weight_scale (dequantised as int8 * (1/scale), tensor.c:75) and bias
    int linear(const std::string& prefix, int out_f, int in_f, Lin* L) {
        L->out = out_f;
        L->in = in_f;
        ENG_RC(upload(prefix + "/weight", "I8", (long long)out_f * in_f, &L->w));
        ENG_RC(upload(prefix + "/weight_scale", "F32", out_f, &L->scale));
        if (tensors.count(prefix + "/bias")) ENG_RC(upload(prefix + "/bias", "F32", out_f, &L->b));
        return half_copy(L);
    }
    // fp16 copy of the int8 weight (every int8 is exact in fp16) and its tensor map
    int half_copy(Lin* L) {
        if (L->in % 64) return NLLB_ATTN_OK;  // the TMA kernel takes K % 64 == 0 only
        plane_t* wb = nullptr;
        ENG_RC(dev_alloc(m, &wb, (size_t)L->out * L->in));
        ENG_CK(launch_int8_to_f16(L->w, wb, (size_t)L->out * L->in, m->stream));
        ENG_CK(encode_half_map(&L->tm, wb, L->in, L->out, 1));
        ENG_CK(encode_half_maps_persistent(nullptr, nullptr, L->in, 0, &L->tm256, wb, L->out));
        ENG_CK(encode_half_map_pair(&L->tm_pair, wb, L->in, L->out));
        L->wb = wb;
        return NLLB_ATTN_OK;
    }
    int norm(const std::string& prefix, float** g, float** b) {
        *g = *b = nullptr;
        if (tensors.count(prefix + "/gamma")) ENG_RC(upload(prefix + "/gamma", "F32", D, g));
        if (tensors.count(prefix + "/beta")) ENG_RC(upload(prefix + "/beta", "F32", D, b));
        return NLLB_ATTN_OK;
    }
};

// Sinusoidal table with the reference's float expressions (encoder.c:27-36).
std::vector<float> position_table(int rows) {
    std::vector<float> t((size_t)rows * D);
    const int half = D / 2;
    for (int p = 0; p < rows; ++p) {
        for (int i = 0; i < half; ++i) {
            const float freq = expf(-(float)i * logf(10000.0f) / (float)(half - 1));
            const float angle = (float)p * freq;
            t[(size_t)p * D + i] = sinf(angle);
            t[(size_t)p * D + i + half] = cosf(angle);
        }
    }
    return t;
}

struct Beam {
    std::vector<int> tokens;
    int n = 0;
    float score = 0.f, eos_score = 0.f;
    bool finished = false;
};
struct Cand {
    int beam, token;
    float score;
};

}  // namespace

extern "C" {

void nllb_model_free(nllb_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->attn) nllb_attn_destroy(m->attn);
    for (void* p : m->allocs) cudaFree(p);
    if (m->planes) cudaFree(m->planes);
    if (m->planes2) cudaFree(m->planes2);
    for (auto& b : m->work_pool)
        if (b.first) cudaFree(b.first);
    for (auto& e : m->step_ev)
        if (e) cudaEventDestroy(e);
    for (auto& e : m->prof_events) cudaEventDestroy(e);
    if (m->live_h) cudaFreeHost(m->live_h);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int nllb_model_load(const char* path, int device, int max_sentences, int max_src, int max_gen, nllb_model** out) {
    if (!path || !out) return nllb::set_error(NLLB_ATTN_EINVAL, "path and out are required");
    *out = nullptr;
    if (max_sentences < 1 || max_src < 2 || max_gen < 6)
        return nllb::set_error(NLLB_ATTN_EINVAL, "max_sentences >= 1, max_src >= 2, max_gen >= 6 required");
    nllb_attn_dims dims{LAYERS, H, 64, max_sentences, NB, max_gen, max_src};
    nllb_attn_ctx* attn = nullptr;
    int rc = nllb_attn_create(device, &dims, &attn);
    if (rc) return rc;
    nllb_model* m = new nllb_model();
    m->device = device;
    m->attn = attn;
    m->max_sentences = max_sentences;
    m->max_src = max_src;
    m->max_gen = max_gen;
    auto fail = [&](int r) {
        nllb_model_free(m);
        return r;
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return fail(nllb::set_error(NLLB_ATTN_ECUDA, "cudaStreamCreate failed"));
    if (configure_linear_tc() != cudaSuccess || configure_linear_tma() != cudaSuccess)
        return fail(nllb::set_error(NLLB_ATTN_ECUDA, "cannot configure the tensor-core linear kernels"));
    m->num_sms = attn->num_sms;
    // split-K: at most 2*SMs*8 partial 128x128 tiles, one counter per tile of the largest output
    m->lws.ws_floats = (size_t)2 * m->num_sms * 8 * 128 * 128;
    m->lws.n_counters = (size_t)((VOCAB + 127) / 128) * ((std::max(max_sentences * NB, max_sentences * max_src) + 127) / 128);
    if (dev_alloc(m, &m->lws.ws, m->lws.ws_floats) || dev_alloc(m, &m->lws.tile_count, m->lws.n_counters) ||
        cudaMemset(m->lws.tile_count, 0, m->lws.n_counters * sizeof(int)) != cudaSuccess)
        return fail(nllb::set_error(NLLB_ATTN_ECUDA, "cannot allocate the linear-layer workspace"));
    nllb_attn_set_stream(attn, m->stream);
    if (cudaHostAlloc(reinterpret_cast<void**>(&m->live_h), (size_t)max_gen * sizeof(int), cudaHostAllocDefault) !=
        cudaSuccess)
        return fail(nllb::set_error(NLLB_ATTN_ECUDA, "cannot allocate pinned host memory"));
    for (auto& e : m->step_ev)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
            return fail(nllb::set_error(NLLB_ATTN_ECUDA, "cannot create events"));

    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(nllb::set_error(NLLB_ATTN_EINVAL, std::string("cannot open ") + path));
    struct stat st;
    fstat(fd, &st);
    const size_t size = (size_t)st.st_size;
    void* map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return fail(nllb::set_error(NLLB_ATTN_EINVAL, "mmap failed"));
    const uint8_t* base = static_cast<const uint8_t*>(map);
    uint64_t hlen = 0;
    memcpy(&hlen, base, 8);
    Loader L{m, base + 8 + hlen, {}};
    int r = NLLB_ATTN_OK;
    if (8 + hlen > size) r = nllb::set_error(NLLB_ATTN_EINVAL, "truncated safetensors header");
    if (!r) {
        std::string header(reinterpret_cast<const char*>(base + 8), (size_t)hlen);
        HeaderParser hp(header);
        if (!hp.parse(&L.tensors)) r = nllb::set_error(NLLB_ATTN_EINVAL, "cannot parse safetensors header");
    }
    auto load_all = [&]() -> int {
        // shared embedding (loader.c:327-335): one device copy serves both stacks
        ENG_RC(L.upload("decoder/embeddings/weight", "I8", (long long)VOCAB * D, &m->emb));
        ENG_RC(L.upload("decoder/embeddings/weight_scale", "F32", VOCAB, &m->emb_scale));
        ENG_RC(dev_alloc(m, &m->emb_inv, VOCAB));
        ENG_CK(launch_reciprocal(m->emb_inv, m->emb_scale, VOCAB, m->stream));
        m->vocab.w = m->emb;
        m->vocab.scale = m->emb_scale;
        m->vocab.out = VOCAB;
        m->vocab.in = D;
        ENG_RC(L.half_copy(&m->vocab));
        for (int i = 0; i < LAYERS; ++i) {
            const std::string p = "encoder/layer_" + std::to_string(i);
            auto& E = m->enc[i];
            ENG_RC(L.linear(p + "/self_attention/linear_0", 3 * D, D, &E.qkv));
            ENG_RC(L.linear(p + "/self_attention/linear_1", D, D, &E.out));
            ENG_RC(L.linear(p + "/ffn/linear_0", FFN, D, &E.fc1));
            ENG_RC(L.linear(p + "/ffn/linear_1", D, FFN, &E.fc2));
            ENG_RC(L.norm(p + "/self_attention/layer_norm", &E.ln1g, &E.ln1b));
            ENG_RC(L.norm(p + "/ffn/layer_norm", &E.ln2g, &E.ln2b));
        }
        ENG_RC(L.norm("encoder/layer_norm", &m->enc_lng, &m->enc_lnb));
        for (int i = 0; i < LAYERS; ++i) {
            const std::string p = "decoder/layer_" + std::to_string(i);
            auto& Dl = m->dec[i];
            ENG_RC(L.linear(p + "/self_attention/linear_0", 3 * D, D, &Dl.qkv));
            ENG_RC(L.linear(p + "/self_attention/linear_1", D, D, &Dl.out));
            ENG_RC(L.linear(p + "/attention/linear_0", D, D, &Dl.xq));
            ENG_RC(L.linear(p + "/attention/linear_1", 2 * D, D, &Dl.xkv));
            ENG_RC(L.linear(p + "/attention/linear_2", D, D, &Dl.xout));
            ENG_RC(L.linear(p + "/ffn/linear_0", FFN, D, &Dl.fc1));
            ENG_RC(L.linear(p + "/ffn/linear_1", D, FFN, &Dl.fc2));
            ENG_RC(L.norm(p + "/self_attention/layer_norm", &Dl.ln1g, &Dl.ln1b));
            ENG_RC(L.norm(p + "/attention/layer_norm", &Dl.ln2g, &Dl.ln2b));
            ENG_RC(L.norm(p + "/ffn/layer_norm", &Dl.ln3g, &Dl.ln3b));
        }
        ENG_RC(L.norm("decoder/layer_norm", &m->dec_lng, &m->dec_lnb));
        m->pos_rows = std::max(max_src, max_gen) + 4;
        const std::vector<float> pt = position_table(m->pos_rows);
        ENG_RC(dev_alloc(m, &m->pos_table, pt.size()));
        ENG_CK(cudaMemcpy(m->pos_table, pt.data(), pt.size() * sizeof(float), cudaMemcpyHostToDevice));
        ENG_CK(cudaStreamSynchronize(m->stream));
        return NLLB_ATTN_OK;
    };
    if (!r) r = load_all();
    munmap(map, size);
    if (r) return fail(r);
    *out = m;
    return NLLB_ATTN_OK;
}

}  // extern "C"

namespace {

// The TMA-fed tensor-core kernels take more than 4 rows, and the vocabulary
// projection at any row count; up to 4 rows of the other layers go to the
// weight-streaming kernel over the int8 matrix.  Measured on B200: 16 rows x
// 1024 -> 1024 in 26 us on the weight-streaming kernel against about 9 us on
// the split-K tensor-core kernel; 4 rows x 1024 -> 256206 in 220 us against
// a persistent kernel over one row tile.
bool tma_path(const nllb_model* m, const Lin& L, int M) {
    return M >= 1 && (M > 4 || L.out >= 65536) && L.wb && (size_t)M * L.in * kPlanes <= m->planes_elems;
}

// out = x W^T / scale + bias (+ relu, + residual).  On the tensor-core path
// the activations are read as fp16 planes: in_planes when the producer wrote
// them already (LayerNorm, the previous GEMM), else x is split into
// m->planes first; with out_planes the result is written as planes for the
// next GEMM instead of to out.
int run_linear(nllb_model* m, const Lin& L, const float* x, int M, float* out, const float* residual, int relu,
               int cblock, int mask_from = -1, const void* in_planes = nullptr, void* out_planes = nullptr) {
    LinearArgs a;
    a.x = x;
    a.ldx = L.in;
    a.w = L.w;
    a.scale = L.scale;
    a.bias = L.b;
    a.out = out;
    a.residual = residual;
    a.M = M;
    a.N = L.out;
    a.K = L.in;
    a.cblock = cblock;
    a.relu = relu;
    a.mask_from = mask_from;
    a.static_weights = 1;  // the model's own weights, written at load
    a.out_planes = out_planes;
    if (tma_path(m, L, M)) {
        if (out_planes && (cblock != L.out || residual))
            return nllb::set_error(NLLB_ATTN_EINVAL, "plane output needs a plain row-major result");
        if (!in_planes) {
            ProfScope ps(m, 12, 0, (double)M * L.in * 10);
            ENG_CK(launch_split_planes(x, L.in, M, L.in, m->planes, m->stream));
            in_planes = m->planes;
        }
        const bool pers = linear_tma_use_persistent(M, L.out, L.in, m->num_sms);
        const auto key = std::make_tuple(in_planes, M, L.in, pers);
        auto it = m->plane_maps.find(key);
        if (it == m->plane_maps.end()) {
            CUtensorMap tx;
            if (pers)
                ENG_CK(encode_half_maps_persistent(&tx, in_planes, L.in, M, nullptr, nullptr, 0));
            else
                ENG_CK(encode_half_map(&tx, in_planes, L.in, M, kPlanes));
            it = m->plane_maps.emplace(key, tx).first;
        }
        const double flops = 2.0 * M * L.out * L.in;
        if (pers) {
            ProfScope ps(m, 0, flops, (double)L.out * L.in * 2);
            ENG_CK(launch_linear_tma_persistent(a, &it->second, &L.tm256, &L.tm_pair, m->num_sms, m->attn->err,
                                                m->stream));
        } else {
            ProfScope ps(m, 1, flops, (double)L.out * L.in * 2);
            ENG_CK(launch_linear_tma(a, &it->second, &L.tm, linear_tma_splits(M, L.out, L.in, m->num_sms),
                                     m->attn->err, m->stream));
        }
        return NLLB_ATTN_OK;
    }
    if (in_planes || out_planes) return nllb::set_error(NLLB_ATTN_EINVAL, "planes need the tensor-core path");
    ProfScope ps(m, 2, 2.0 * M * L.out * L.in, (double)L.out * L.in);
    ENG_CK(launch_linear(a, &m->lws, m->num_sms, m->attn->err, m->stream));
    return NLLB_ATTN_OK;
}

// Grow the activation-plane buffer to `elems` fp16 values.
int ensure_planes(nllb_model* m, size_t elems) {
    if (elems <= m->planes_elems) return NLLB_ATTN_OK;
    ENG_CK(cudaStreamSynchronize(m->stream));
    if (m->planes) cudaFree(m->planes);
    if (m->planes2) cudaFree(m->planes2);
    m->planes = m->planes2 = nullptr;
    m->planes_elems = 0;
    m->plane_maps.clear();
    ENG_CK(cudaMalloc(&m->planes, elems * sizeof(plane_t)));
    ENG_CK(cudaMalloc(&m->planes2, elems * sizeof(plane_t)));
    m->planes_elems = elems;
    return NLLB_ATTN_OK;
}

// Buffers of one translate call.
struct Work {
    int n_sent = 0, S = 0, rows_enc = 0, rows = 0;
    float *ex = nullptr, *eh = nullptr, *eqkv = nullptr, *eattn = nullptr, *effn = nullptr, *ekv = nullptr;
    int *etok = nullptr, *epos = nullptr, *evalid = nullptr;
    int* erow0 = nullptr;  // first encoder row of each sentence (rows packed, no padding)
    float *x = nullptr, *h = nullptr, *qkv = nullptr, *qx = nullptr, *attn = nullptr, *ffn = nullptr;
    float* logits = nullptr;
    int *tok = nullptr, *hist = nullptr, *ntok = nullptr, *parent = nullptr, *top_tok = nullptr;
    float* top_lp = nullptr;
    float* topk_ws = nullptr;  // partials of the vocabulary log-softmax / top-k
    unsigned char* active = nullptr;
    bool h_planes = false;  // the last decoder step left h as fp16 planes in m->planes (else fp32 in h)
    const int* n_src_h = nullptr;  // host: source lengths in the call's internal order (profile bytes)
    // buffers come from the model's pool in call order: a call no larger than
    // an earlier one allocates nothing (the previous call has finished: it
    // returned its results to the host)
    nllb_model* m = nullptr;
    size_t next = 0;
    template <typename T>
    int alloc(T** p, size_t n) {
        const size_t bytes = std::max<size_t>(n, 1) * sizeof(T);
        if (next == m->work_pool.size()) m->work_pool.push_back({nullptr, 0});
        auto& slot = m->work_pool[next++];
        if (slot.second < bytes) {
            if (slot.first) cudaFree(slot.first);
            slot = {nullptr, 0};
            ENG_CK(cudaMalloc(&slot.first, bytes));
            slot.second = bytes;
        }
        *p = static_cast<T*>(slot.first);
        return NLLB_ATTN_OK;
    }
};

int encode(nllb_model* m, Work& w, const std::vector<int>& n_src) {
    const int R = w.rows_enc;
    {
        ProfScope ps(m, 11, 0, (double)R * D * 5);
        ENG_CK(launch_embed_pos(w.ex, w.etok, w.epos, 0, m->emb, m->emb_inv, m->pos_table, 32.0f, R, VOCAB,
                                m->stream));
    }
    // LayerNorm writes the fp16 planes of the next GEMM's input directly when
    // that GEMM runs on the tensor cores, fc1 writes fc2's input planes
    const bool tp = tma_path(m, m->enc[0].qkv, R);
    void* P1 = tp ? m->planes : nullptr;
    void* P2 = tp ? m->planes2 : nullptr;
    float* lnout = tp ? nullptr : w.eh;
    for (int l = 0; l < LAYERS; ++l) {
        auto& E = m->enc[l];
        {
            ProfScope ps(m, 10, 0, (double)R * D * 10);
            ENG_CK(launch_layernorm(lnout, w.ex, nullptr, E.ln1g, E.ln1b, R, P1, m->stream));
        }
        ENG_RC(run_linear(m, E.qkv, w.eh, R, w.eqkv, nullptr, 0, D, -1, P1));
        nllb_attn_prefill_args a{};
        a.q = w.eqkv;
        a.k = w.eqkv + (size_t)R * D;
        a.v = w.eqkv + (size_t)2 * R * D;
        a.out = w.eattn;
        a.batch = w.n_sent;
        a.n_heads = H;
        a.seq_len = w.S;
        a.head_dim = 64;
        a.stride_batch = 0;  // rows packed: sentence s starts at row erow0[s]
        a.stride_head = 64;
        a.stride_row = D;
        a.valid_len = w.evalid;
        a.scale = 1.0f / sqrtf(64.0f);
        {
            double fl = 0;  // dense flops of the valid rows: 4 * S_s^2 * 64 per head
            for (int s = 0; s < w.n_sent; ++s) fl += 4.0 * H * w.n_src_h[s] * w.n_src_h[s] * 64;
            ProfScope ps(m, 5, fl, (double)R * D * 16);
            ENG_RC(nllb::attn_prefill_packed(m->attn, &a, w.erow0, w.rows_enc));
        }
        ENG_RC(run_linear(m, E.out, w.eattn, R, w.ex, w.ex, 0, D));
        {
            ProfScope ps(m, 10, 0, (double)R * D * 10);
            ENG_CK(launch_layernorm(lnout, w.ex, nullptr, E.ln2g, E.ln2b, R, P1, m->stream));
        }
        ENG_RC(run_linear(m, E.fc1, w.eh, R, w.effn, nullptr, 1, FFN, -1, P1, P2));
        ENG_RC(run_linear(m, E.fc2, w.effn, R, w.ex, w.ex, 0, D, -1, P2));
    }
    ENG_CK(launch_layernorm(lnout, w.ex, nullptr, m->enc_lng, m->enc_lnb, R, P1, m->stream));  // encoder_out
    // cross-attention memory of every layer (decoder.c:118-125, projected once)
    nllb_attn_ctx* c = m->attn;
    const size_t layer_floats = (size_t)c->d.max_sentences * H * (size_t)c->d.max_src * 64;
    for (int l = 0; l < LAYERS; ++l) {
        ENG_RC(run_linear(m, m->dec[l].xkv, w.eh, R, w.ekv, nullptr, 0, D, -1, P1));
        ProfScope ps(m, 13, 0, (double)R * D * 16);
        ENG_CK(launch_set_memory_batched(c->km + l * layer_floats, c->vm + l * layer_floats,
                                         c->n_src_dev + (size_t)l * c->d.max_sentences, c->d.max_src, H, w.ekv,
                                         w.ekv + (size_t)R * D, 0, w.erow0, w.evalid, w.n_sent, w.S,
                                         m->stream));
        for (int s = 0; s < w.n_sent; ++s) c->n_src_host[(size_t)l * c->d.max_sentences + s] = n_src[s];
    }
    return NLLB_ATTN_OK;
}

// One decoder step for every row (decoder.c:199-233): token w.tok[row] at
// position `step`; leaves the final-LayerNorm output in w.h.
int decode_step(nllb_model* m, Work& w, int step) {
    const int R = w.rows;
    {
        ProfScope ps(m, 11, 0, (double)R * D * 5);
        ENG_CK(launch_embed_pos(w.x, w.tok, nullptr, step + 2, m->emb, m->emb_inv, m->pos_table, 32.0f, R, VOCAB,
                                m->stream));
    }
    // algorithmic bytes of the attention launches of this step: self-attention
    // K/V of positions 0..step, q/out, new k/v, history (per sentence), and
    // cross-attention memory rows plus q/out
    const double L = step + 1;
    const double self_bytes = (double)w.n_sent * (2.0 * NB * H * L * 256 + 4.0 * NB * H * 256 + 4.0 * NB * L);
    double xrows = 0;
    for (int s = 0; s < w.n_sent; ++s) xrows += w.n_src_h[s];
    const double cross_bytes = 2.0 * H * xrows * 256 + (double)w.n_sent * 2.0 * NB * H * 256;
    const bool tp = tma_path(m, m->dec[0].qkv, R);
    void* P1 = tp ? m->planes : nullptr;
    void* P2 = tp ? m->planes2 : nullptr;
    float* lnout = tp ? nullptr : w.h;
    w.h_planes = tp;  // the final LayerNorm below leaves h as planes (tp) or as fp32
    for (int l = 0; l < LAYERS; ++l) {
        auto& Dl = m->dec[l];
        {
            ProfScope ps(m, 10, 0, (double)R * D * 10);
            ENG_CK(launch_layernorm(lnout, w.x, nullptr, Dl.ln1g, Dl.ln1b, R, P1, m->stream));
        }
        ENG_RC(run_linear(m, Dl.qkv, w.h, R, w.qkv, nullptr, 0, D, -1, P1));
        // on the tensor-core path the attention kernels write the output
        // projection's fp16 planes themselves (no fp32 output, no split pass)
        if (tp && tma_path(m, Dl.out, R)) {
            {
                ProfScope ps(m, 3, 0, self_bytes);
                ENG_RC(nllb::attn_decode_self_planes(m->attn, l, step, w.n_sent, w.qkv, w.qkv + (size_t)R * D,
                                                     w.qkv + (size_t)2 * R * D, m->planes));
            }
            ENG_RC(run_linear(m, Dl.out, w.attn, R, w.x, w.x, 0, D, -1, m->planes));
        } else {
            {
                ProfScope ps(m, 3, 0, self_bytes);
                ENG_RC(nllb_attn_decode_self(m->attn, l, step, w.n_sent, w.qkv, w.qkv + (size_t)R * D,
                                             w.qkv + (size_t)2 * R * D, w.attn));
            }
            ENG_RC(run_linear(m, Dl.out, w.attn, R, w.x, w.x, 0, D));
        }
        {
            ProfScope ps(m, 10, 0, (double)R * D * 10);
            ENG_CK(launch_layernorm(lnout, w.x, nullptr, Dl.ln2g, Dl.ln2b, R, P1, m->stream));
        }
        ENG_RC(run_linear(m, Dl.xq, w.h, R, w.qx, nullptr, 0, D, -1, P1));
        if (tp && tma_path(m, Dl.xout, R)) {
            {
                ProfScope ps(m, 4, 0, cross_bytes);
                ENG_RC(nllb::attn_cross_planes(m->attn, l, w.n_sent, w.qx, m->planes));
            }
            ENG_RC(run_linear(m, Dl.xout, w.attn, R, w.x, w.x, 0, D, -1, m->planes));
        } else {
            {
                ProfScope ps(m, 4, 0, cross_bytes);
                ENG_RC(nllb_attn_cross(m->attn, l, w.n_sent, w.qx, w.attn));
            }
            ENG_RC(run_linear(m, Dl.xout, w.attn, R, w.x, w.x, 0, D));
        }
        {
            ProfScope ps(m, 10, 0, (double)R * D * 10);
            ENG_CK(launch_layernorm(lnout, w.x, nullptr, Dl.ln3g, Dl.ln3b, R, P1, m->stream));
        }
        ENG_RC(run_linear(m, Dl.fc1, w.h, R, w.ffn, nullptr, 1, FFN, -1, P1, P2));
        ENG_RC(run_linear(m, Dl.fc2, w.ffn, R, w.x, w.x, 0, D, -1, P2));
    }
    {
        ProfScope ps(m, 10, 0, (double)R * D * 10);
        ENG_CK(launch_layernorm(lnout, w.x, nullptr, m->dec_lng, m->dec_lnb, R, P1, m->stream));
    }
    return NLLB_ATTN_OK;
}

// Tied vocabulary projection with language rows masked (decoder.c:319-354),
// penalties (main.c:186-213) and log-softmax + top-k (main.c:154-182).
int vocab_topk(nllb_model* m, Work& w, int k, bool penalties, const nllb_translate_opts& o,
               const int* hist = nullptr) {
    ENG_RC(run_linear(m, m->vocab, w.h, w.rows, w.logits, nullptr, 0, VOCAB_LD, LANG_START,
                      w.h_planes ? m->planes : nullptr));
    if (penalties) {
        ProfScope ps(m, 7, 0, (double)w.rows * m->max_gen * 4);
        ENG_CK(launch_penalties(w.logits, VOCAB_LD, hist ? hist : w.hist, m->max_gen, w.ntok, w.active, w.rows,
                                o.repetition_penalty, o.no_repeat_ngram, m->stream));
    }
    ProfScope ps(m, 6, 0, (double)w.rows * VOCAB * 4);
    ENG_CK(launch_logsoftmax_topk(w.logits, VOCAB_LD, VOCAB, w.rows, w.active, k, w.top_tok, w.top_lp, w.topk_ws,
                                  m->stream));
    return NLLB_ATTN_OK;
}

double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

extern "C" int nllb_translate(nllb_model* m, int n_sent, const int* src_tokens, const int* src_offsets,
                              int tgt_lang, const nllb_translate_opts* opts, int* out_tokens, int* out_len,
                              float* out_score, nllb_translate_stats* stats) {
    if (!m || !src_tokens || !src_offsets) return nllb::set_error(NLLB_ATTN_EINVAL, "model and sources required");
    if (n_sent < 1 || n_sent > m->max_sentences)
        return nllb::set_error(NLLB_ATTN_ECAPACITY, "n_sentences outside [1, max_sentences]");
    if (tgt_lang < 0 || tgt_lang >= VOCAB) return nllb::set_error(NLLB_ATTN_EINVAL, "tgt_lang out of range");
    nllb_translate_opts o{m->max_gen, 1.2f, 2};
    if (opts) o = *opts;
    if (o.max_gen < 6 || o.max_gen > m->max_gen)
        return nllb::set_error(NLLB_ATTN_ECAPACITY, "opts.max_gen outside [6, model max_gen]");
    if (!(o.no_repeat_ngram == 0 || o.no_repeat_ngram == 2))
        return nllb::set_error(NLLB_ATTN_EINVAL, "no_repeat_ngram must be 0 or 2");
    ENG_CK(cudaSetDevice(m->device));
    const auto t_start = std::chrono::steady_clock::now();

    Work w;
    w.m = m;
    w.n_sent = n_sent;
    std::vector<int> n_src(n_sent), max_out(n_sent);
    int S = 0;
    for (int s = 0; s < n_sent; ++s) {
        n_src[s] = src_offsets[s + 1] - src_offsets[s];
        if (n_src[s] < 1 || n_src[s] > m->max_src)
            return nllb::set_error(NLLB_ATTN_ECAPACITY, "a source length is outside [1, max_src]");
        for (int i = src_offsets[s]; i < src_offsets[s + 1]; ++i)
            if (src_tokens[i] < 0 || src_tokens[i] >= VOCAB)
                return nllb::set_error(NLLB_ATTN_EINVAL, "source token id out of range");
        S = std::max(S, n_src[s]);
        max_out[s] = std::min(3 * n_src[s] + 10, o.max_gen - 4);  // main.c:315-316
    }
    // Internal order: sentences by decreasing max_out (stable), so that the
    // sentences still running at any step are a prefix of the batch and a
    // step processes only that prefix (perm: internal index -> caller's).
    // Equal max_out: the longer source first, so the per-sentence attention
    // CTAs (dispatched sentence by sentence) start with the longest memories
    // and the last wave holds the short ones.
    std::vector<int> perm(n_sent);
    for (int s = 0; s < n_sent; ++s) perm[s] = s;
    std::stable_sort(perm.begin(), perm.end(), [&](int a, int b) {
        return max_out[a] != max_out[b] ? max_out[a] > max_out[b] : n_src[a] > n_src[b];
    });
    {
        std::vector<int> ns(n_sent), mo(n_sent);
        for (int s = 0; s < n_sent; ++s) ns[s] = n_src[perm[s]], mo[s] = max_out[perm[s]];
        n_src.swap(ns);
        max_out.swap(mo);
    }
    w.S = S;
    w.n_src_h = n_src.data();
    std::vector<int> row0(n_sent);  // encoder rows are packed: sentence s at rows row0[s] ..
    int rows_enc = 0;
    for (int s = 0; s < n_sent; ++s) row0[s] = rows_enc, rows_enc += n_src[s];
    w.rows_enc = rows_enc;
    w.rows = n_sent * NB;
    const size_t RE = (size_t)w.rows_enc, R = (size_t)w.rows;
    ENG_RC(ensure_planes(m, std::max(RE, R) * FFN * kPlanes));
    ENG_RC(w.alloc(&w.ex, RE * D));
    ENG_RC(w.alloc(&w.eh, RE * D));
    ENG_RC(w.alloc(&w.eqkv, RE * 3 * D));
    ENG_RC(w.alloc(&w.eattn, RE * D));
    ENG_RC(w.alloc(&w.effn, RE * FFN));
    ENG_RC(w.alloc(&w.ekv, RE * 2 * D));
    ENG_RC(w.alloc(&w.etok, RE));
    ENG_RC(w.alloc(&w.epos, RE));
    ENG_RC(w.alloc(&w.evalid, n_sent));
    ENG_RC(w.alloc(&w.erow0, n_sent));
    ENG_RC(w.alloc(&w.x, R * D));
    ENG_RC(w.alloc(&w.h, R * D));
    ENG_RC(w.alloc(&w.qkv, R * 3 * D));
    ENG_RC(w.alloc(&w.qx, R * D));
    ENG_RC(w.alloc(&w.attn, R * D));
    ENG_RC(w.alloc(&w.ffn, R * FFN));
    ENG_RC(w.alloc(&w.logits, R * VOCAB_LD));
    ENG_RC(w.alloc(&w.tok, R));
    ENG_RC(w.alloc(&w.hist, R * m->max_gen));
    ENG_RC(w.alloc(&w.ntok, R));
    ENG_RC(w.alloc(&w.parent, R));
    ENG_RC(w.alloc(&w.top_tok, R * 8));
    ENG_RC(w.alloc(&w.topk_ws, vocab_topk_ws_floats(VOCAB, w.rows, 8)));
    ENG_RC(w.alloc(&w.top_lp, R * 8));
    ENG_RC(w.alloc(&w.active, R));

    // ---- encoder: the sentences' rows back to back (no padding rows in the
    // GEMMs); each sentence's attention over its own rows only
    {
        std::vector<int> tok(RE), pos(RE);
        for (int s = 0; s < n_sent; ++s)
            for (int t = 0; t < n_src[s]; ++t) {
                tok[(size_t)row0[s] + t] = src_tokens[src_offsets[perm[s]] + t];
                pos[(size_t)row0[s] + t] = t + 2;  // NLLB position offset (encoder.c:29)
            }
        ENG_CK(cudaMemcpyAsync(w.etok, tok.data(), RE * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(w.epos, pos.data(), RE * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(w.evalid, n_src.data(), n_sent * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(w.erow0, row0.data(), n_sent * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        ENG_RC(nllb_attn_reset(m->attn));
        ENG_RC(encode(m, w, n_src));
        ENG_CK(cudaStreamSynchronize(m->stream));
        ENG_RC(nllb_attn_sync(m->attn));
    }
    const double t_enc = ms_since(t_start);
    const auto t_dec0 = std::chrono::steady_clock::now();

    // ---- beam state (main.c:317-330)
    const int G = o.max_gen;
    std::vector<Beam> beams((size_t)n_sent * NB);
    std::vector<std::vector<Beam>> completed(n_sent);
    std::vector<char> done(n_sent, 0);
    for (auto& b : beams) {
        b.tokens.assign(G, 0);
        b.tokens[0] = 2;  // NLLB decoder start token (main.c:324)
        b.n = 1;
    }
    m->margins.assign(n_sent, {});
    std::vector<int> tok_h(R), parent_h(R), ntok_h(R), hist_h(R * (size_t)m->max_gen, 0);
    std::vector<unsigned char> active_h(R);
    std::vector<int> top_tok_h(R * 8);
    std::vector<float> top_lp_h(R * 8);

    auto upload_tokens = [&]() -> int {
        ENG_CK(cudaMemcpyAsync(w.tok, tok_h.data(), R * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        return NLLB_ATTN_OK;
    };

    // step 0: decoder start token on every beam (main.c:331-333; all beams start equal)
    std::fill(tok_h.begin(), tok_h.end(), 2);
    ENG_RC(upload_tokens());
    ENG_RC(decode_step(m, w, 0));
    // step 1: target language token, top-4 of beam 0 seeds the beams (main.c:343-392)
    std::fill(tok_h.begin(), tok_h.end(), tgt_lang);
    ENG_RC(upload_tokens());
    ENG_RC(decode_step(m, w, 1));
    for (size_t r = 0; r < R; ++r) active_h[r] = (r % NB) == 0;
    ENG_CK(cudaMemcpyAsync(w.active, active_h.data(), R, cudaMemcpyHostToDevice, m->stream));
    ENG_RC(vocab_topk(m, w, NB, false, o));
    ENG_CK(cudaMemcpyAsync(top_tok_h.data(), w.top_tok, R * NB * sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    ENG_CK(cudaMemcpyAsync(top_lp_h.data(), w.top_lp, R * NB * sizeof(float), cudaMemcpyDeviceToHost, m->stream));
    ENG_CK(cudaStreamSynchronize(m->stream));
    for (int s = 0; s < n_sent; ++s)
        for (int b = 0; b < NB; ++b) {
            Beam& bm = beams[(size_t)s * NB + b];
            const size_t r0 = (size_t)s * NB;  // beam 0's row
            bm.tokens[1] = tgt_lang;
            bm.tokens[2] = top_tok_h[r0 * NB + b];
            bm.n = 3;
            bm.score = top_lp_h[r0 * NB + b];
            bm.eos_score = 0.f;
            bm.finished = bm.tokens[2] == 2;
        }
    int steps_run = 2;

    // ---- steps 2 .. max_out+1 (main.c:411-511): selection on the device (beam.cu),
    // the host only reads a running-sentence count, at most two steps behind
    const int GD = m->max_gen;  // row length of the device histories
    BeamState B{};
    B.G = GD;
    B.n_sent = n_sent;
    B.bt0 = w.hist;
    B.bn = w.ntok;
    B.tok = w.tok;
    B.active = w.active;
    B.parent = w.parent;
    int* maxo_d = nullptr;
    ENG_RC(w.alloc(&B.bt1, R * (size_t)GD));
    ENG_RC(w.alloc(&B.bsc, R));
    ENG_RC(w.alloc(&B.beos, R));
    ENG_RC(w.alloc(&B.bfin, R));
    ENG_RC(w.alloc(&B.done, (size_t)n_sent));
    ENG_RC(w.alloc(&maxo_d, (size_t)n_sent));
    B.maxo = maxo_d;
    ENG_RC(w.alloc(&B.ctok, (size_t)n_sent * 8 * GD));
    ENG_RC(w.alloc(&B.cn, (size_t)n_sent * 8));
    ENG_RC(w.alloc(&B.csc, (size_t)n_sent * 8));
    ENG_RC(w.alloc(&B.ceos, (size_t)n_sent * 8));
    ENG_RC(w.alloc(&B.ccnt, (size_t)n_sent));
    ENG_RC(w.alloc(&B.margins, (size_t)n_sent * GD));
    ENG_RC(w.alloc(&B.mcnt, (size_t)n_sent));
    ENG_RC(w.alloc(&B.live, (size_t)GD));
    {
        std::vector<float> bsc(R), beos(R, 0.f);
        std::vector<unsigned char> bfin(R), done_h(n_sent);
        int live0 = 0;
        for (int s = 0; s < n_sent; ++s) {
            int n_active = 0;
            for (int b = 0; b < NB; ++b) {
                const size_t r = (size_t)s * NB + b;
                const Beam& bm = beams[r];
                std::copy(bm.tokens.begin(), bm.tokens.begin() + bm.n, hist_h.begin() + r * GD);
                ntok_h[r] = bm.n;
                tok_h[r] = bm.tokens[bm.n - 1];
                bsc[r] = bm.score;
                bfin[r] = bm.finished ? 1 : 0;
                n_active += !bm.finished;
            }
            done_h[s] = (2 >= max_out[s] + 2 || n_active == 0) ? 1 : 0;  // main.c:411-412 at step 2
            live0 += !done_h[s];
            for (int b = 0; b < NB; ++b) {
                const size_t r = (size_t)s * NB + b;
                active_h[r] = (!done_h[s] && !beams[r].finished) ? 1 : 0;
            }
        }
        ENG_CK(cudaMemcpyAsync(B.bt0, hist_h.data(), R * (size_t)GD * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(B.bn, ntok_h.data(), R * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(B.tok, tok_h.data(), R * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(B.bsc, bsc.data(), R * sizeof(float), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(B.beos, beos.data(), R * sizeof(float), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(B.bfin, bfin.data(), R, cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(B.active, active_h.data(), R, cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(B.done, done_h.data(), n_sent, cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemcpyAsync(maxo_d, max_out.data(), n_sent * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        ENG_CK(cudaMemsetAsync(B.ccnt, 0, n_sent * sizeof(int), m->stream));
        ENG_CK(cudaMemsetAsync(B.mcnt, 0, n_sent * sizeof(int), m->stream));
        ENG_CK(cudaMemsetAsync(B.live, 0, GD * sizeof(int), m->stream));
        ENG_CK(cudaStreamSynchronize(m->stream));  // host vectors above go out of scope
        steps_run += live0 > 0;
        if (live0 == 0) max_out.assign(n_sent, 0);  // nothing to run
    }
    int last_step = 1;
    for (int s = 0; s < n_sent; ++s) last_step = std::max(last_step, max_out[s] + 1);
    if (last_step >= m->max_gen) return nllb::set_error(NLLB_ATTN_ECAPACITY, "decode would run past max_gen");
    int cur = 0, launched_to = 1;
    int n_live = n_sent;  // sentences processed at this step: a sentence runs at step t while t < max_out + 2
    for (int step = 2; step <= last_step; ++step) {
        if (step >= 4) {  // two steps of lookahead: the count of step - 2 decides whether to go on
            ENG_CK(cudaEventSynchronize(m->step_ev[(step - 2) & 3]));
            if (m->live_h[step - 2] == 0) break;
        }
        while (n_live > 0 && step >= max_out[n_live - 1] + 2) --n_live;
        if (n_live == 0) break;
        w.n_sent = n_live;
        w.rows = n_live * NB;
        B.n_sent = n_live;
        ENG_RC(decode_step(m, w, step));
        ENG_RC(vocab_topk(m, w, 8, true, o, cur ? B.bt1 : B.bt0));
        {
            ProfScope ps(m, 8);
            ENG_CK(launch_beam_select(B, cur, w.top_tok, w.top_lp, step, m->stream));
        }
        ENG_CK(cudaMemcpyAsync(m->live_h + step, B.live + step, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
        ENG_CK(cudaEventRecord(m->step_ev[step & 3], m->stream));
        {
            ProfScope ps(m, 9, 0, (double)n_live * (step + 1) * 8);
            ENG_RC(nllb_attn_reorder(m->attn, n_live, w.parent));
        }
        cur ^= 1;
        launched_to = step;
    }
    w.n_sent = n_sent;
    w.rows = (int)R;
    B.n_sent = n_sent;
    ENG_RC(nllb_attn_sync(m->attn));
    if (m->prof_on) prof_resolve(m);
    for (int t = 3; t <= launched_to; ++t) steps_run += m->live_h[t - 1] > 0;

    // ---- device beam state back to the host structures of the final choice
    {
        std::vector<int> bt(R * (size_t)GD), bt_other(R * (size_t)GD), bn(R), cn((size_t)n_sent * 8), ccnt(n_sent),
            mcnt(n_sent);
        std::vector<int> ct((size_t)n_sent * 8 * GD);
        std::vector<float> bsc(R), beos(R), csc((size_t)n_sent * 8), ceos((size_t)n_sent * 8);
        std::vector<float> marg((size_t)n_sent * GD);
        std::vector<unsigned char> bfin(R);
        // the history written by a sentence's last processed step: the selection
        // of step t writes bt1 for even t and bt0 for odd t (bt0 before step 2)
        ENG_CK(cudaMemcpy(bt.data(), B.bt0, bt.size() * sizeof(int), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(bt_other.data(), B.bt1, bt_other.size() * sizeof(int), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(bn.data(), B.bn, R * sizeof(int), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(bsc.data(), B.bsc, R * sizeof(float), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(beos.data(), B.beos, R * sizeof(float), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(bfin.data(), B.bfin, R, cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(ct.data(), B.ctok, ct.size() * sizeof(int), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(cn.data(), B.cn, cn.size() * sizeof(int), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(csc.data(), B.csc, csc.size() * sizeof(float), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(ceos.data(), B.ceos, ceos.size() * sizeof(float), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(ccnt.data(), B.ccnt, n_sent * sizeof(int), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(marg.data(), B.margins, marg.size() * sizeof(float), cudaMemcpyDeviceToHost));
        ENG_CK(cudaMemcpy(mcnt.data(), B.mcnt, n_sent * sizeof(int), cudaMemcpyDeviceToHost));
        for (int s = 0; s < n_sent; ++s) {
            const int last = std::min(max_out[s] + 1, launched_to);  // last step that selected for s
            const std::vector<int>& hs = (last >= 2 && (last & 1) == 0) ? bt_other : bt;
            for (int b = 0; b < NB; ++b) {
                const size_t r = (size_t)s * NB + b;
                Beam& bm = beams[r];
                bm.n = bn[r];
                std::copy(hs.begin() + r * GD, hs.begin() + r * GD + bm.n, bm.tokens.begin());
                bm.score = bsc[r];
                bm.eos_score = beos[r];
                bm.finished = bfin[r] != 0;
            }
            for (int c = 0; c < ccnt[s]; ++c) {
                const size_t k = (size_t)s * 8 + c;
                Beam hb;
                hb.n = cn[k];
                hb.tokens.assign(ct.begin() + k * GD, ct.begin() + k * GD + GD);
                hb.score = csc[k];
                hb.eos_score = ceos[k];
                hb.finished = true;
                completed[s].push_back(hb);
            }
            m->margins[perm[s]].assign(marg.begin() + (size_t)s * GD, marg.begin() + (size_t)s * GD + mcnt[s]);
        }
    }
    const double t_dec = ms_since(t_dec0);

    // ---- final choice (main.c:511-546)
    long long total_out = 0;
    for (int s = 0; s < n_sent; ++s) {
        std::vector<Beam>& cp = completed[s];
        for (int b = 0; b < NB; ++b) {
            const Beam& bm = beams[(size_t)s * NB + b];
            if (bm.finished && cp.size() < (size_t)(2 * NB)) cp.push_back(bm);
        }
        if (cp.empty()) cp.push_back(beams[(size_t)s * NB]);
        int bi = 0;
        float bn = -1e30f;
        for (int c = 0; c < (int)cp.size(); ++c) {
            const int cl = cp[c].n - 2;
            const float ns = (cp[c].score - cp[c].eos_score) / (float)(cl + 1);
            if (ns > bn) {
                bn = ns;
                bi = c;
            }
        }
        const Beam& best = cp[bi];
        const size_t so = (size_t)perm[s];  // the caller's index
        int n_out = 0;
        for (int i = 2; i < best.n; ++i) {
            if (best.tokens[i] == 2) break;
            if (out_tokens) out_tokens[so * G + n_out] = best.tokens[i];
            ++n_out;
        }
        if (out_tokens)
            for (int i = n_out; i < G; ++i) out_tokens[so * G + i] = -1;
        if (out_len) out_len[so] = n_out;
        if (out_score) out_score[so] = bn;
        total_out += n_out;
    }
    if (stats) {
        stats->encode_ms = t_enc;
        stats->decode_ms = t_dec;
        stats->steps = steps_run;
        stats->tokens_out = total_out;
    }
    return NLLB_ATTN_OK;
}

extern "C" int nllb_translate_margins(const nllb_model* m, int sentence, float* out, int max_steps) {
    if (!m || sentence < 0 || sentence >= (int)m->margins.size() || !out) return 0;
    const auto& v = m->margins[sentence];
    const int n = std::min<int>((int)v.size(), max_steps);
    for (int i = 0; i < n; ++i) out[i] = v[i];
    return n;
}

// Error word of nllb_linear_int8 on device `dev` (allocated on the first call
// there): set by a bounded wait that gave up, read and cleared only by
// nllb_linear_int8_status.
static int linear_err_word(int dev, int** out) {
    static std::mutex mu;
    static int* words[64] = {nullptr};
    std::lock_guard<std::mutex> lock(mu);
    if (!words[dev]) {
        ENG_CK(cudaMalloc(&words[dev], sizeof(int)));
        ENG_CK(cudaMemset(words[dev], 0, sizeof(int)));
    }
    *out = words[dev];
    return NLLB_ATTN_OK;
}

extern "C" int nllb_linear_int8_status(void) {
    int dev = 0;
    ENG_CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return nllb::set_error(NLLB_ATTN_ENODEV, "device ordinal beyond 63");
    int* w = nullptr;
    const int rc = linear_err_word(dev, &w);
    if (rc) return rc;
    int h = 0;
    ENG_CK(cudaDeviceSynchronize());
    ENG_CK(cudaMemcpy(&h, w, sizeof(int), cudaMemcpyDeviceToHost));
    ENG_CK(cudaMemset(w, 0, sizeof(int)));
    if (h) return nllb::set_error(NLLB_ATTN_ETIMEOUT, "a bounded device wait of the linear kernel gave up");
    return NLLB_ATTN_OK;
}

extern "C" int nllb_translate_profile(nllb_model* m, int enable) {
    if (!m) return nllb::set_error(NLLB_ATTN_EINVAL, "model required");
    m->prof_on = enable != 0;
    for (int c = 0; c < NLLB_PROF_CLASSES; ++c) {
        m->prof_agg[c] = nllb_kernel_profile{};
        std::snprintf(m->prof_agg[c].name, sizeof(m->prof_agg[c].name), "%s", kProfNames[c]);
    }
    m->prof_recs.clear();
    m->prof_next = 0;
    return NLLB_ATTN_OK;
}

extern "C" int nllb_translate_profile_read(const nllb_model* m, nllb_kernel_profile* out, int max_classes) {
    if (!m || !out) return 0;
    const int n = std::min(max_classes, (int)NLLB_PROF_CLASSES);
    for (int c = 0; c < n; ++c) out[c] = m->prof_agg[c];
    return n;
}

extern "C" int nllb_linear_int8(const float* x, int M, int K, const int8_t* w, const float* weight_scale,
                                const float* bias, int N, float* out, const float* residual, int flags,
                                void* stream) {
    if (!x || !w || !weight_scale || !out) return nllb::set_error(NLLB_ATTN_EINVAL, "x, w, weight_scale, out required");
    if (M < 0 || K < 4 || N < 1 || (K & 3)) return nllb::set_error(NLLB_ATTN_EINVAL, "M >= 0, N >= 1, K a multiple of 4");
    if (M > 0 && M > 16 && K % 32) return nllb::set_error(NLLB_ATTN_EINVAL, "K must be a multiple of 32 beyond 16 rows");
    LinearArgs a;
    a.x = x;
    a.ldx = K;
    a.w = w;
    a.scale = weight_scale;
    a.bias = bias;
    a.out = out;
    a.residual = residual;
    a.M = M;
    a.N = N;
    a.K = K;
    a.cblock = N;
    a.relu = (flags & NLLB_LINEAR_RELU) ? 1 : 0;
    a.mask_from = -1;
    a.static_weights = 0;
    a.out_planes = nullptr;
    // bounded-wait error word of the current device for callers without a context
    int dev = 0;
    ENG_CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return nllb::set_error(NLLB_ATTN_ENODEV, "device ordinal beyond 63");
    int* err_word = nullptr;
    {
        const int rc = linear_err_word(dev, &err_word);
        if (rc) return rc;
    }
    // split-K workspace of the current device, grown on demand
    static LinearWorkspace wss[64];
    LinearWorkspace& W = wss[dev];
    int nsm = 148;
    ENG_CK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    if (M > 16 && linear_tc_supports(a)) {
        const int splits = linear_tc_splits(a, nsm);
        const size_t need = linear_tc_workspace_floats(a, splits), tiles = linear_tc_tiles(a);
        if (need > W.ws_floats) {
            if (W.ws) cudaFree(W.ws);
            W.ws = nullptr;
            W.ws_floats = 0;
            ENG_CK(cudaMalloc(&W.ws, need * sizeof(float)));
            W.ws_floats = need;
        }
        if (tiles > W.n_counters) {
            if (W.tile_count) cudaFree(W.tile_count);
            W.tile_count = nullptr;
            W.n_counters = 0;
            ENG_CK(cudaMalloc(&W.tile_count, tiles * sizeof(int)));
            ENG_CK(cudaMemset(W.tile_count, 0, tiles * sizeof(int)));
            W.n_counters = tiles;
        }
    }
    if (configure_linear_tc() != cudaSuccess) return nllb::set_error(NLLB_ATTN_ECUDA, "configure failed");
    ENG_CK(launch_linear(a, &W, nsm, err_word, static_cast<cudaStream_t>(stream)));
    return NLLB_ATTN_OK;
}
