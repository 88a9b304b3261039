// nllb_attn.cu -- the C ABI of include/nllb_attn.h: context, argument checks,
// split selection, host-buffer staging and the single-head drop-ins.
#include "nllb_attn.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "attn_internal.h"
#include "device_common.cuh"
#include "kernels.h"

using namespace nllb;

namespace {

thread_local std::string t_last_error;
thread_local int t_last_status = NLLB_ATTN_OK;

int fail(int status, const std::string& msg) {
    t_last_error = msg;
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return NLLB_ATTN_ECUDA;
}

#define NLLB_CK(call)                                          \
    do {                                                       \
        cudaError_t e_ = (call);                               \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);    \
    } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace nllb {
// Status + message for the engine translation unit (engine.cu).
int set_error(int status, const std::string& msg) { return fail(status, msg); }
}  // namespace nllb



namespace {

size_t cache_floats(const nllb_attn_dims& d) {
    return (size_t)d.n_layers * d.max_sentences * d.n_heads * (size_t)d.max_tgt * d.n_beams * 64;
}
size_t mem_floats(const nllb_attn_dims& d) {
    return (size_t)d.n_layers * d.max_sentences * d.n_heads * (size_t)d.max_src * 64;
}
int hist_rows(const nllb_attn_dims& d) { return ((d.max_tgt + 1) & ~1) + 2; }

int check_dims(const nllb_attn_dims* d) {
    if (!d) return fail(NLLB_ATTN_EINVAL, "dims is NULL");
    if (d->head_dim != 64) return fail(NLLB_ATTN_EINVAL, "head_dim must be 64");
    if (d->n_heads < 1 || d->n_heads > 1024) return fail(NLLB_ATTN_EINVAL, "n_heads out of range");
    if (!(d->n_beams == 1 || d->n_beams == 2 || d->n_beams == 4 || d->n_beams == 8))
        return fail(NLLB_ATTN_EINVAL, "n_beams must be 1, 2, 4 or 8");
    if (d->max_sentences < 0 || d->n_layers < 0 || d->max_tgt < 0 || d->max_src < 0)
        return fail(NLLB_ATTN_EINVAL, "negative capacity");
    if (d->max_sentences > 0 && (d->n_layers < 1 || d->max_tgt < 1 || d->max_src < 1))
        return fail(NLLB_ATTN_EINVAL, "a context with sentences needs n_layers, max_tgt, max_src >= 1");
    return NLLB_ATTN_OK;
}

size_t device_bytes(const nllb_attn_dims& d) {
    size_t b = 0;
    b += 2 * cache_floats(d) * sizeof(float);
    b += 2 * mem_floats(d) * sizeof(float);
    b += 2 * (size_t)d.max_sentences * hist_rows(d) * 8;  // current and other beam history
    b += (size_t)d.n_layers * d.max_sentences * sizeof(int);
    b += sizeof(int);
    return b;
}

int set_device(nllb_attn_ctx* c) {
    NLLB_CK(cudaSetDevice(c->device));
    return NLLB_ATTN_OK;
}

int ensure_stage(nllb_attn_ctx* c, int slot, size_t bytes) {
    if (c->stg_bytes[slot] >= bytes) return NLLB_ATTN_OK;
    if (c->stg[slot]) cudaFree(c->stg[slot]);
    c->stg[slot] = nullptr;
    c->stg_bytes[slot] = 0;
    NLLB_CK(cudaMalloc(&c->stg[slot], bytes));
    c->stg_bytes[slot] = bytes;
    return NLLB_ATTN_OK;
}

// Reads and clears the device error word (stream must be idle).
int check_device_error(nllb_attn_ctx* c) {
    int e = 0;
    NLLB_CK(cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e == 0) return NLLB_ATTN_OK;
    NLLB_CK(cudaMemset(c->err, 0, sizeof(int)));
    if (e & NLLB_DEV_ERR_TIMEOUT)
        return fail(NLLB_ATTN_ETIMEOUT, "a kernel's bounded wait for a bulk copy gave up");
    return fail(NLLB_ATTN_EINVAL, "reorder: parent index outside [0, n_beams)");
}

// Copy streams, events and pinned words of the pipelined host-buffer calls.
int ensure_host_pipeline(nllb_attn_ctx* c) {
    if (c->copy_in) return NLLB_ATTN_OK;
    NLLB_CK(cudaStreamCreateWithFlags(&c->copy_in, cudaStreamNonBlocking));
    NLLB_CK(cudaStreamCreateWithFlags(&c->copy_out, cudaStreamNonBlocking));
    for (int i = 0; i < nllb_attn_ctx::kHostChunks; ++i) {
        NLLB_CK(cudaEventCreateWithFlags(&c->ev_in[i], cudaEventDisableTiming));
        NLLB_CK(cudaEventCreateWithFlags(&c->ev_k[i], cudaEventDisableTiming));
    }
    NLLB_CK(cudaEventCreateWithFlags(&c->ev_parent, cudaEventDisableTiming));
    NLLB_CK(cudaHostAlloc(reinterpret_cast<void**>(&c->err_h), sizeof(int), cudaHostAllocDefault));
    *c->err_h = 0;
    return NLLB_ATTN_OK;
}

int finish_host_call(nllb_attn_ctx* c) {
    NLLB_CK(cudaStreamSynchronize(c->stream));
    return check_device_error(c);
}

// Apply a pending reorder with the reorder kernel (in place on the current
// history) and forget it.
int flush_reorder(nllb_attn_ctx* c) {
    if (!c->pending_parent) return NLLB_ATTN_OK;
    const int* par = c->pending_parent;
    const int n = c->pending_n;
    c->pending_parent = nullptr;
    c->pending_n = 0;
    NLLB_CK(launch_reorder(c->hist, c->Tp, par, n, c->d.n_beams, c->err, c->stream));
    return NLLB_ATTN_OK;
}

// Split count for a (sentence, head) grid of `units` over `len` rows in
// chunks of `chunk` rows: enough CTAs to cover the SMs twice, each split at
// least one chunk, at most one cluster (kMaxSplit CTAs) per (sentence, head).
void choose_split(const nllb_attn_ctx* c, int units, int len, int chunk, int* n_split, int* pps) {
    int ns = 1;
    if (len > 0 && units < 2 * c->num_sms) {
        ns = (2 * c->num_sms + units - 1) / units;
        ns = std::min(ns, (len + chunk - 1) / chunk);
        ns = std::min(ns, kMaxSplit);
        ns = std::max(ns, 1);
    }
    int per = len > 0 ? (len + ns - 1) / ns : chunk;
    per = ((per + chunk - 1) / chunk) * chunk;
    if (len > 0) ns = (len + per - 1) / per;
    *n_split = ns;
    *pps = per;
}

}  // namespace

extern "C" {

const char* nllb_attn_strerror(int status) {
    switch (status) {
        case NLLB_ATTN_OK: return "ok";
        case NLLB_ATTN_EINVAL: return "invalid argument";
        case NLLB_ATTN_ECAPACITY: return "capacity exceeded";
        case NLLB_ATTN_ECUDA: return "CUDA error";
        case NLLB_ATTN_ETIMEOUT: return "device wait timed out";
        case NLLB_ATTN_ENODEV: return "no usable sm_100 device";
        case NLLB_ATTN_ESTATE: return "invalid call order";
        default: return "unknown status";
    }
}

const char* nllb_attn_last_error(void) { return t_last_error.c_str(); }

size_t nllb_attn_device_bytes(const nllb_attn_dims* dims) {
    if (check_dims(dims) != NLLB_ATTN_OK) return 0;
    return device_bytes(*dims);
}

void nllb_attn_destroy(nllb_attn_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (void* p : {(void*)c->kc, (void*)c->vc, (void*)c->hist, (void*)c->hist_alt, (void*)c->km, (void*)c->vm,
                    (void*)c->n_src_dev, (void*)c->err})
        if (p) cudaFree(p);
    for (void* p : c->stg)
        if (p) cudaFree(p);
    if (c->copy_in) cudaStreamSynchronize(c->copy_in);
    if (c->copy_out) cudaStreamSynchronize(c->copy_out);
    for (int i = 0; i < nllb_attn_ctx::kHostChunks; ++i) {
        if (c->ev_in[i]) cudaEventDestroy(c->ev_in[i]);
        if (c->ev_k[i]) cudaEventDestroy(c->ev_k[i]);
    }
    if (c->ev_parent) {
        cudaEventSynchronize(c->ev_parent);
        cudaEventDestroy(c->ev_parent);
    }
    if (c->copy_in) cudaStreamDestroy(c->copy_in);
    if (c->copy_out) cudaStreamDestroy(c->copy_out);
    if (c->err_h) cudaFreeHost(c->err_h);
    if (c->par_h) cudaFreeHost(c->par_h);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
}

int nllb_attn_create(int device, const nllb_attn_dims* dims, nllb_attn_ctx** out_ctx) {
    if (!out_ctx) return fail(NLLB_ATTN_EINVAL, "out_ctx is NULL");
    *out_ctx = nullptr;
    int rc = check_dims(dims);
    if (rc) return rc;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(NLLB_ATTN_ENODEV, std::string("no CUDA device: ") + cudaGetErrorString(e));
    }
    if (device < 0 || device >= count) return fail(NLLB_ATTN_ENODEV, "device ordinal out of range");
    cudaDeviceProp prop;
    NLLB_CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(NLLB_ATTN_ENODEV, "the kernels are built for sm_100a (compute capability 10.x)");

    nllb_attn_ctx* c = new nllb_attn_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    c->d = *dims;
    c->Tp = hist_rows(*dims);
    auto bail = [&](int r) {
        nllb_attn_destroy(c);
        return r;
    };
#define NLLB_CKC(call)                                              \
    do {                                                            \
        cudaError_t e_ = (call);                                    \
        if (e_ != cudaSuccess) return bail(cuda_fail(e_, #call));   \
    } while (0)
    NLLB_CKC(cudaSetDevice(device));
    NLLB_CKC(configure_decode_kernels());
    NLLB_CKC(configure_prefill_kernels());
    NLLB_CKC(cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking));
    c->stream = c->own_stream;
    const nllb_attn_dims& d = c->d;
    if (d.max_sentences > 0) {
        const size_t cf = cache_floats(d), mf = mem_floats(d);
        NLLB_CKC(cudaMalloc(&c->kc, cf * sizeof(float)));
        NLLB_CKC(cudaMalloc(&c->vc, cf * sizeof(float)));
        NLLB_CKC(cudaMalloc(&c->km, mf * sizeof(float)));
        NLLB_CKC(cudaMalloc(&c->vm, mf * sizeof(float)));
        NLLB_CKC(cudaMalloc(&c->hist, (size_t)d.max_sentences * c->Tp * 8));
        NLLB_CKC(cudaMalloc(&c->hist_alt, (size_t)d.max_sentences * c->Tp * 8));
        NLLB_CKC(cudaMalloc(&c->n_src_dev, (size_t)d.n_layers * d.max_sentences * sizeof(int)));
        NLLB_CKC(cudaMemsetAsync(c->kc, 0, cf * sizeof(float), c->stream));
        NLLB_CKC(cudaMemsetAsync(c->vc, 0, cf * sizeof(float), c->stream));
        NLLB_CKC(cudaMemsetAsync(c->km, 0, mf * sizeof(float), c->stream));
        NLLB_CKC(cudaMemsetAsync(c->vm, 0, mf * sizeof(float), c->stream));
        NLLB_CKC(cudaMemsetAsync(c->n_src_dev, 0, (size_t)d.n_layers * d.max_sentences * sizeof(int),
                                 c->stream));
        NLLB_CKC(launch_hist_init(c->hist, c->Tp, d.max_sentences, c->stream));
        NLLB_CKC(launch_hist_init(c->hist_alt, c->Tp, d.max_sentences, c->stream));
        c->n_src_host.assign((size_t)d.n_layers * d.max_sentences, 0);
    }
    NLLB_CKC(cudaMalloc(&c->err, sizeof(int)));
    NLLB_CKC(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream));
    NLLB_CKC(cudaStreamSynchronize(c->stream));
#undef NLLB_CKC
    *out_ctx = c;
    return NLLB_ATTN_OK;
}

int nllb_attn_set_stream(nllb_attn_ctx* c, void* stream) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
    return NLLB_ATTN_OK;
}

void* nllb_attn_get_stream(nllb_attn_ctx* c) { return c ? (void*)c->stream : nullptr; }

int nllb_attn_sync(nllb_attn_ctx* c) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = flush_reorder(c))) return rc;  // the caller's parent buffer is free afterwards
    return finish_host_call(c);
}

int nllb_attn_reset(nllb_attn_ctx* c) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    int rc = set_device(c);
    if (rc) return rc;
    c->pending_parent = nullptr;
    c->pending_n = 0;
    if (c->d.max_sentences > 0) {
        NLLB_CK(launch_hist_init(c->hist, c->Tp, c->d.max_sentences, c->stream));
        NLLB_CK(cudaMemsetAsync(c->n_src_dev, 0,
                                (size_t)c->d.n_layers * c->d.max_sentences * sizeof(int), c->stream));
        std::fill(c->n_src_host.begin(), c->n_src_host.end(), 0);
    }
    return NLLB_ATTN_OK;
}

// ---------------------------------------------------------------------------
// prefill
// ---------------------------------------------------------------------------
static int check_prefill(const nllb_attn_prefill_args* a) {
    if (!a) return fail(NLLB_ATTN_EINVAL, "args is NULL");
    if (!a->q || !a->k || !a->v || !a->out) return fail(NLLB_ATTN_EINVAL, "q, k, v and out are required");
    if (a->head_dim != 64) return fail(NLLB_ATTN_EINVAL, "head_dim must be 64");
    if (a->batch < 1 || a->n_heads < 1 || a->seq_len < 1)
        return fail(NLLB_ATTN_EINVAL, "batch, n_heads and seq_len must be >= 1");
    if (a->batch > 65535 || a->n_heads > 65535) return fail(NLLB_ATTN_EINVAL, "batch or n_heads too large");
    if (a->stride_batch < 0 || a->stride_head < 0 || a->stride_row < 64)
        return fail(NLLB_ATTN_EINVAL, "strides must be non-negative and stride_row >= 64");
    if ((a->stride_batch | a->stride_head | a->stride_row) & 3)
        return fail(NLLB_ATTN_EINVAL, "strides must be multiples of 4 elements (16-byte rows)");
    if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out))
        return fail(NLLB_ATTN_EINVAL, "q, k, v, out must be 16-byte aligned");
    if (a->mask && (a->mask_stride_batch < 0 || a->mask_stride_head < 0))
        return fail(NLLB_ATTN_EINVAL, "mask strides must be non-negative");
    if (!(a->scale > 0.0f) || !std::isfinite(a->scale)) return fail(NLLB_ATTN_EINVAL, "scale must be positive");
    return NLLB_ATTN_OK;
}

static PrefillParams prefill_params(const nllb_attn_prefill_args* a, int* err) {
    PrefillParams p;
    p.err = err;
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    p.out = a->out;
    p.B = a->batch;
    p.H = a->n_heads;
    p.S = a->seq_len;
    p.sb = a->stride_batch;
    p.sh = a->stride_head;
    p.sr = a->stride_row;
    p.valid_len = a->valid_len;
    p.mask = a->mask;
    p.msb = a->mask_stride_batch;
    p.msh = a->mask_stride_head;
    p.scale_log2 = a->scale * kLog2e;
    p.row_start = nullptr;
    p.rows_total = 0;
    p.map_pos_row = p.map_pos_head = p.map_pos_seq = 0;
    return p;
}

}  // extern "C"

namespace nllb {

int attn_prefill_packed(nllb_attn_ctx* c, const nllb_attn_prefill_args* a, const int* row_start, int rows_total) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    int rc = check_prefill(a);
    if (rc) return rc;
    if (!row_start || !a->valid_len || a->mask)
        return fail(NLLB_ATTN_EINVAL, "packed prefill needs row starts and lengths, and no mask");
    if ((rc = set_device(c))) return rc;
    if (rows_total < 1) return fail(NLLB_ATTN_EINVAL, "packed prefill needs the buffers' row count");
    PrefillParams p = prefill_params(a, c->err);
    p.row_start = row_start;
    p.rows_total = rows_total;
    NLLB_CK(launch_prefill(p, c->stream));
    return NLLB_ATTN_OK;
}

}  // namespace nllb

extern "C" {

int nllb_attn_prefill(nllb_attn_ctx* c, const nllb_attn_prefill_args* a) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    int rc = check_prefill(a);
    if (rc) return rc;
    if ((rc = set_device(c))) return rc;
    NLLB_CK(launch_prefill(prefill_params(a, c->err), c->stream));
    return NLLB_ATTN_OK;
}

int nllb_attn_prefill_host(nllb_attn_ctx* c, const nllb_attn_prefill_args* a) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    int rc = check_prefill(a);
    if (rc) return rc;
    if ((rc = set_device(c))) return rc;
    const long long B = a->batch, H = a->n_heads, S = a->seq_len;
    const size_t extent = (size_t)((B - 1) * a->stride_batch + (H - 1) * a->stride_head +
                                   (S - 1) * a->stride_row + 64);
    const size_t bytes = extent * sizeof(float);
    const bool dense = extent == (size_t)(B * H * S * 64);
    if (a->valid_len) {
        for (int b = 0; b < a->batch; ++b)
            if (a->valid_len[b] < 0 || a->valid_len[b] > a->seq_len)
                return fail(NLLB_ATTN_EINVAL, "valid_len entries must be in [0, seq_len]");
    }
    size_t mask_extent = 0;
    if (a->mask)
        mask_extent = (size_t)((B - 1) * a->mask_stride_batch + (H - 1) * a->mask_stride_head + S * S);
    if ((rc = ensure_stage(c, 0, bytes)) || (rc = ensure_stage(c, 1, bytes)) ||
        (rc = ensure_stage(c, 2, bytes)) || (rc = ensure_stage(c, 3, bytes)))
        return rc;
    if (a->valid_len && (rc = ensure_stage(c, 4, (size_t)a->batch * sizeof(int)))) return rc;
    if (a->mask && (rc = ensure_stage(c, 5, mask_extent * sizeof(float)))) return rc;
    float* dq = static_cast<float*>(c->stg[0]);
    float* dk = static_cast<float*>(c->stg[1]);
    float* dv = static_cast<float*>(c->stg[2]);
    float* dout = static_cast<float*>(c->stg[3]);
    NLLB_CK(cudaMemcpyAsync(dq, a->q, bytes, cudaMemcpyHostToDevice, c->stream));
    NLLB_CK(cudaMemcpyAsync(dk, a->k, bytes, cudaMemcpyHostToDevice, c->stream));
    NLLB_CK(cudaMemcpyAsync(dv, a->v, bytes, cudaMemcpyHostToDevice, c->stream));
    if (!dense) NLLB_CK(cudaMemcpyAsync(dout, a->out, bytes, cudaMemcpyHostToDevice, c->stream));
    nllb_attn_prefill_args d = *a;
    d.q = dq;
    d.k = dk;
    d.v = dv;
    d.out = dout;
    if (a->valid_len) {
        NLLB_CK(cudaMemcpyAsync(c->stg[4], a->valid_len, (size_t)a->batch * sizeof(int),
                                cudaMemcpyHostToDevice, c->stream));
        d.valid_len = static_cast<int*>(c->stg[4]);
    }
    if (a->mask) {
        NLLB_CK(cudaMemcpyAsync(c->stg[5], a->mask, mask_extent * sizeof(float), cudaMemcpyHostToDevice,
                                c->stream));
        d.mask = static_cast<float*>(c->stg[5]);
    }
    NLLB_CK(launch_prefill(prefill_params(&d, c->err), c->stream));
    NLLB_CK(cudaMemcpyAsync(a->out, dout, bytes, cudaMemcpyDeviceToHost, c->stream));
    return finish_host_call(c);
}

// ---------------------------------------------------------------------------
// decoder self-attention
// ---------------------------------------------------------------------------
static int check_beam_call(nllb_attn_ctx* c, int layer, int n_sent) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    if (c->d.max_sentences == 0) return fail(NLLB_ATTN_ESTATE, "context was created without sentence slots");
    if (layer < 0 || layer >= c->d.n_layers) return fail(NLLB_ATTN_EINVAL, "layer out of range");
    if (n_sent < 1) return fail(NLLB_ATTN_EINVAL, "n_sentences must be >= 1");
    if (n_sent > c->d.max_sentences) return fail(NLLB_ATTN_ECAPACITY, "n_sentences > max_sentences");
    if (n_sent > 65535) return fail(NLLB_ATTN_EINVAL, "n_sentences too large for one launch");
    return NLLB_ATTN_OK;
}

// Sentences s0 .. s0 + n_sent - 1; q, k_new, v_new, out point at sentence s0.
// planes: `out` is the base of the output planes of these n_sent sentences
// mode reorder: the pending reorder's parents for these sentences are applied
// on the way and the composed history goes to c->hist_alt (the caller swaps
// the buffers once every sentence has been launched).
static int decode_self_dev(nllb_attn_ctx* c, int layer, int step, int s0, int n_sent, const float* q,
                           const float* k_new, const float* v_new, float* out, bool planes = false,
                           SelfMode mode = SelfMode::plain) {
    const nllb_attn_dims& d = c->d;
    const size_t layer_floats = (size_t)d.max_sentences * d.n_heads * (size_t)d.max_tgt * d.n_beams * 64;
    const size_t sent_floats = (size_t)d.n_heads * d.max_tgt * d.n_beams * 64;
    SelfParams p;
    p.kc = c->kc + (size_t)layer * layer_floats + (size_t)s0 * sent_floats;
    p.vc = c->vc + (size_t)layer * layer_floats + (size_t)s0 * sent_floats;
    p.kc_w = c->kc + (size_t)layer * layer_floats + (size_t)s0 * sent_floats;
    p.vc_w = c->vc + (size_t)layer * layer_floats + (size_t)s0 * sent_floats;
    p.hist = c->hist + (size_t)s0 * c->Tp * 8;
    p.hist_w = (mode == SelfMode::reorder ? c->hist_alt : c->hist) + (size_t)s0 * c->Tp * 8;
    p.q = q;
    p.k_new = k_new;
    p.v_new = v_new;
    p.out = out;
    p.H = d.n_heads;
    p.T = d.max_tgt;
    p.Tp = c->Tp;
    p.step = step;
    choose_split(c, n_sent * d.n_heads, step, self_chunk_positions(d.n_beams), &p.n_split,
                 &p.pos_per_split);
    p.scale_log2 = (1.0f / std::sqrt(64.0f)) * kLog2e;
    p.err = c->err;
    const int* parent = mode == SelfMode::reorder ? c->pending_parent + (size_t)s0 * d.n_beams : nullptr;
    NLLB_CK(launch_decode_self(p, n_sent, d.n_beams, c->stream, planes, mode, parent));
    return NLLB_ATTN_OK;
}

// Before a self-attention call over sentences [0, n_sent): the form of its
// launches.  A pending reorder is applied on the way when it covers exactly
// the call's sentences and those are all of the context's (the other buffer
// then holds every sentence's history after the call); otherwise the reorder
// kernel applies it first.  The bounded-wait test form is taken once.
static int self_mode(nllb_attn_ctx* c, int n_sent, SelfMode* mode) {
    *mode = SelfMode::plain;
    if (c->expire_next_wait) {
        c->expire_next_wait = false;
        if (c->d.n_beams != 4) return fail(NLLB_ATTN_EINVAL, "the bounded-wait test takes 4 beams");
        *mode = SelfMode::expire_wait;
        return flush_reorder(c);
    }
    if (!c->pending_parent) return NLLB_ATTN_OK;
    if (c->pending_n == n_sent && n_sent == c->d.max_sentences) {
        *mode = SelfMode::reorder;
        return NLLB_ATTN_OK;
    }
    return flush_reorder(c);
}

// After the launches of a call made in the reorder form.
static void self_done(nllb_attn_ctx* c, SelfMode mode) {
    if (mode != SelfMode::reorder) return;
    std::swap(c->hist, c->hist_alt);
    c->pending_parent = nullptr;
    c->pending_n = 0;
}

int nllb_attn_decode_self(nllb_attn_ctx* c, int layer, int step, int n_sent, const float* q,
                          const float* k_new, const float* v_new, float* out) {
    int rc = check_beam_call(c, layer, n_sent);
    if (rc) return rc;
    if (step < 0) return fail(NLLB_ATTN_EINVAL, "step must be >= 0");
    if (step >= c->d.max_tgt) return fail(NLLB_ATTN_ECAPACITY, "step >= max_tgt");
    if (!q || !k_new || !v_new || !out) return fail(NLLB_ATTN_EINVAL, "q, k_new, v_new, out are required");
    if (!aligned16(q) || !aligned16(k_new) || !aligned16(v_new) || !aligned16(out))
        return fail(NLLB_ATTN_EINVAL, "q, k_new, v_new, out must be 16-byte aligned");
    if ((rc = set_device(c))) return rc;
    SelfMode mode;
    if ((rc = self_mode(c, n_sent, &mode))) return rc;
    rc = decode_self_dev(c, layer, step, 0, n_sent, q, k_new, v_new, out, false, mode);
    if (rc == NLLB_ATTN_OK) self_done(c, mode);
    return rc;
}

int nllb_attn_decode_self_host(nllb_attn_ctx* c, int layer, int step, int n_sent, const float* q,
                               const float* k_new, const float* v_new, float* out) {
    int rc = check_beam_call(c, layer, n_sent);
    if (rc) return rc;
    if (step < 0) return fail(NLLB_ATTN_EINVAL, "step must be >= 0");
    if (step >= c->d.max_tgt) return fail(NLLB_ATTN_ECAPACITY, "step >= max_tgt");
    if (!q || !k_new || !v_new || !out) return fail(NLLB_ATTN_EINVAL, "q, k_new, v_new, out are required");
    if ((rc = set_device(c))) return rc;
    const size_t sent_floats = (size_t)c->d.n_beams * c->d.n_heads * 64;
    const size_t bytes = (size_t)n_sent * sent_floats * sizeof(float);
    for (int i = 0; i < 4; ++i)
        if ((rc = ensure_stage(c, i, bytes))) return rc;
    if ((rc = ensure_host_pipeline(c))) return rc;
    float* dq = static_cast<float*>(c->stg[0]);
    float* dk = static_cast<float*>(c->stg[1]);
    float* dv = static_cast<float*>(c->stg[2]);
    float* dout = static_cast<float*>(c->stg[3]);
    SelfMode mode;
    if ((rc = self_mode(c, n_sent, &mode))) return rc;
    // chunks of sentences: the input copy of chunk j + 1 and the output copy of
    // chunk j - 1 run while chunk j's kernel runs (separate copy streams)
    const int C = std::min(nllb_attn_ctx::kHostChunks, n_sent);
    for (int j = 0; j < C; ++j) {
        const int s0 = (int)((long long)j * n_sent / C), s1 = (int)((long long)(j + 1) * n_sent / C);
        const size_t off = (size_t)s0 * sent_floats, cb = (size_t)(s1 - s0) * sent_floats * sizeof(float);
        NLLB_CK(cudaMemcpyAsync(dq + off, q + off, cb, cudaMemcpyHostToDevice, c->copy_in));
        NLLB_CK(cudaMemcpyAsync(dk + off, k_new + off, cb, cudaMemcpyHostToDevice, c->copy_in));
        NLLB_CK(cudaMemcpyAsync(dv + off, v_new + off, cb, cudaMemcpyHostToDevice, c->copy_in));
        NLLB_CK(cudaEventRecord(c->ev_in[j], c->copy_in));
        NLLB_CK(cudaStreamWaitEvent(c->stream, c->ev_in[j], 0));
        if ((rc = decode_self_dev(c, layer, step, s0, s1 - s0, dq + off, dk + off, dv + off, dout + off, false,
                                  mode)))
            return rc;
        NLLB_CK(cudaEventRecord(c->ev_k[j], c->stream));
        NLLB_CK(cudaStreamWaitEvent(c->copy_out, c->ev_k[j], 0));
        NLLB_CK(cudaMemcpyAsync(out + off, dout + off, cb, cudaMemcpyDeviceToHost, c->copy_out));
    }
    self_done(c, mode);
    // the error word after the last kernel, with the outputs
    NLLB_CK(cudaMemcpyAsync(c->err_h, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->copy_out));
    NLLB_CK(cudaStreamSynchronize(c->copy_out));
    if (*c->err_h == 0) return NLLB_ATTN_OK;
    return check_device_error(c);  // reads, reports and clears the word
}

int nllb_attn_test_expire_next_wait(nllb_attn_ctx* c) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    if (c->d.n_beams != 4) return fail(NLLB_ATTN_EINVAL, "the bounded-wait test takes 4 beams");
    c->expire_next_wait = true;
    return NLLB_ATTN_OK;
}

int nllb_attn_test_expire_next_cross_wait(nllb_attn_ctx* c) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    if (c->d.n_beams != 4) return fail(NLLB_ATTN_EINVAL, "the bounded-wait test takes 4 beams");
    c->expire_next_cross = true;
    return NLLB_ATTN_OK;
}

int nllb_attn_reorder(nllb_attn_ctx* c, int n_sent, const int* parent) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    if (c->d.max_sentences == 0) return fail(NLLB_ATTN_ESTATE, "context was created without sentence slots");
    if (n_sent < 1) return fail(NLLB_ATTN_EINVAL, "n_sentences must be >= 1");
    if (n_sent > c->d.max_sentences) return fail(NLLB_ATTN_ECAPACITY, "n_sentences > max_sentences");
    if (!parent) return fail(NLLB_ATTN_EINVAL, "parent is NULL");
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = flush_reorder(c))) return rc;  // two reorders in a row: the first one now
    c->pending_parent = parent;
    c->pending_n = n_sent;
    return NLLB_ATTN_OK;
}

int nllb_attn_reorder_host(nllb_attn_ctx* c, int n_sent, const int* parent) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    if (c->d.max_sentences == 0) return fail(NLLB_ATTN_ESTATE, "context was created without sentence slots");
    if (n_sent < 1) return fail(NLLB_ATTN_EINVAL, "n_sentences must be >= 1");
    if (n_sent > c->d.max_sentences) return fail(NLLB_ATTN_ECAPACITY, "n_sentences > max_sentences");
    if (!parent) return fail(NLLB_ATTN_EINVAL, "parent is NULL");
    for (int i = 0; i < n_sent * c->d.n_beams; ++i)
        if (parent[i] < 0 || parent[i] >= c->d.n_beams)
            return fail(NLLB_ATTN_EINVAL, "parent index outside [0, n_beams)");
    int rc = set_device(c);
    if (rc) return rc;
    if ((rc = flush_reorder(c))) return rc;  // it may read the staging buffer refilled below
    const size_t n = (size_t)n_sent * c->d.n_beams;
    if ((rc = ensure_stage(c, 6, n * sizeof(int)))) return rc;
    if ((rc = ensure_host_pipeline(c))) return rc;
    // The parents (checked above) go through a pinned copy, so the call returns
    // once the reorder is enqueued and the caller's buffer is free at once;
    // later calls on the context are ordered after it.
    NLLB_CK(cudaEventSynchronize(c->ev_parent));  // the previous copy has left par_h
    if (c->par_h_ints < n) {
        if (c->par_h) cudaFreeHost(c->par_h);
        c->par_h = nullptr;
        c->par_h_ints = 0;
        NLLB_CK(cudaHostAlloc(reinterpret_cast<void**>(&c->par_h), n * sizeof(int), cudaHostAllocDefault));
        c->par_h_ints = n;
    }
    std::memcpy(c->par_h, parent, n * sizeof(int));
    NLLB_CK(cudaMemcpyAsync(c->stg[6], c->par_h, n * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    NLLB_CK(cudaEventRecord(c->ev_parent, c->stream));
    c->pending_parent = static_cast<int*>(c->stg[6]);
    c->pending_n = n_sent;
    return NLLB_ATTN_OK;
}

// ---------------------------------------------------------------------------
// cross-attention
// ---------------------------------------------------------------------------
static int check_memory_args(nllb_attn_ctx* c, int layer, int sentence, int n_src, const float* k,
                             const float* v, int64_t stride_head, int64_t stride_row) {
    if (!c) return fail(NLLB_ATTN_EINVAL, "ctx is NULL");
    if (c->d.max_sentences == 0) return fail(NLLB_ATTN_ESTATE, "context was created without sentence slots");
    if (layer < 0 || layer >= c->d.n_layers) return fail(NLLB_ATTN_EINVAL, "layer out of range");
    if (sentence < 0 || sentence >= c->d.max_sentences) return fail(NLLB_ATTN_ECAPACITY, "sentence slot out of range");
    if (n_src < 1) return fail(NLLB_ATTN_EINVAL, "n_src must be >= 1");
    if (n_src > c->d.max_src) return fail(NLLB_ATTN_ECAPACITY, "n_src > max_src");
    if (!k || !v) return fail(NLLB_ATTN_EINVAL, "k and v are required");
    if (stride_head < 0 || stride_row < 0 || ((stride_head | stride_row) & 3))
        return fail(NLLB_ATTN_EINVAL, "strides must be non-negative multiples of 4 elements");
    return NLLB_ATTN_OK;
}

static int set_memory_dev(nllb_attn_ctx* c, int layer, int sentence, int n_src, const float* k,
                          const float* v, int64_t stride_head, int64_t stride_row) {
    const nllb_attn_dims& d = c->d;
    const size_t off = (((size_t)layer * d.max_sentences + sentence) * d.n_heads) * (size_t)d.max_src * 64;
    const size_t idx = (size_t)layer * d.max_sentences + sentence;
    NLLB_CK(launch_set_memory(c->km + off, c->vm + off, d.max_src, d.n_heads, k, v, stride_head, stride_row,
                              n_src, c->n_src_dev + idx, c->stream));
    c->n_src_host[idx] = n_src;
    return NLLB_ATTN_OK;
}

int nllb_attn_set_memory(nllb_attn_ctx* c, int layer, int sentence, int n_src, const float* k,
                         const float* v, int64_t stride_head, int64_t stride_row) {
    int rc = check_memory_args(c, layer, sentence, n_src, k, v, stride_head, stride_row);
    if (rc) return rc;
    if (!aligned16(k) || !aligned16(v)) return fail(NLLB_ATTN_EINVAL, "k and v must be 16-byte aligned");
    if ((rc = set_device(c))) return rc;
    return set_memory_dev(c, layer, sentence, n_src, k, v, stride_head, stride_row);
}

int nllb_attn_set_memory_host(nllb_attn_ctx* c, int layer, int sentence, int n_src, const float* k,
                              const float* v, int64_t stride_head, int64_t stride_row) {
    int rc = check_memory_args(c, layer, sentence, n_src, k, v, stride_head, stride_row);
    if (rc) return rc;
    if ((rc = set_device(c))) return rc;
    const size_t extent =
        (size_t)((int64_t)(n_src - 1) * stride_row + (int64_t)(c->d.n_heads - 1) * stride_head + 64);
    const size_t bytes = extent * sizeof(float);
    if ((rc = ensure_stage(c, 0, bytes)) || (rc = ensure_stage(c, 1, bytes))) return rc;
    NLLB_CK(cudaMemcpyAsync(c->stg[0], k, bytes, cudaMemcpyHostToDevice, c->stream));
    NLLB_CK(cudaMemcpyAsync(c->stg[1], v, bytes, cudaMemcpyHostToDevice, c->stream));
    if ((rc = set_memory_dev(c, layer, sentence, n_src, static_cast<float*>(c->stg[0]),
                             static_cast<float*>(c->stg[1]), stride_head, stride_row)))
        return rc;
    return finish_host_call(c);
}

static int cross_dev(nllb_attn_ctx* c, int layer, int n_sent, const float* q, float* out, bool planes = false) {
    const nllb_attn_dims& d = c->d;
    int max_len = 0;
    for (int s = 0; s < n_sent; ++s) {
        const int n = c->n_src_host[(size_t)layer * d.max_sentences + s];
        if (n < 1) return fail(NLLB_ATTN_ESTATE, "cross-attention on a sentence whose memory was not set");
        max_len = std::max(max_len, n);
    }
    const size_t layer_floats = (size_t)d.max_sentences * d.n_heads * (size_t)d.max_src * 64;
    CrossParams p;
    p.km = c->km + (size_t)layer * layer_floats;
    p.vm = c->vm + (size_t)layer * layer_floats;
    p.n_src = c->n_src_dev + (size_t)layer * d.max_sentences;
    p.q = q;
    p.out = out;
    p.H = d.n_heads;
    p.max_src = d.max_src;
    int chunk_rows = cross_chunk_rows(max_len);
    choose_split(c, n_sent * d.n_heads, max_len, chunk_rows, &p.n_split, &p.pos_per_split);
    if (chunk_rows == kCrossLongRows && p.n_split > 1 && p.pos_per_split <= kCrossSplitRows) {
        chunk_rows = kCrossSplitRows;  // one chunk per split CTA
        choose_split(c, n_sent * d.n_heads, max_len, chunk_rows, &p.n_split, &p.pos_per_split);
    }
    p.scale_log2 = (1.0f / std::sqrt(64.0f)) * kLog2e;
    p.err = c->err;
    if (c->expire_next_cross) {  // the bounded-wait test form, taken once
        c->expire_next_cross = false;
        if (d.n_beams != 4 || planes) return fail(NLLB_ATTN_EINVAL, "the bounded-wait test takes 4 beams, fp32 output");
        chunk_rows = kCrossShortRows;
        choose_split(c, n_sent * d.n_heads, max_len, chunk_rows, &p.n_split, &p.pos_per_split);
        NLLB_CK(launch_cross(p, n_sent, d.n_beams, chunk_rows, c->stream, false, true));
        return NLLB_ATTN_OK;
    }
    NLLB_CK(launch_cross(p, n_sent, d.n_beams, chunk_rows, c->stream, planes));
    return NLLB_ATTN_OK;
}

int nllb_attn_cross(nllb_attn_ctx* c, int layer, int n_sent, const float* q, float* out) {
    int rc = check_beam_call(c, layer, n_sent);
    if (rc) return rc;
    if (!q || !out) return fail(NLLB_ATTN_EINVAL, "q and out are required");
    if (!aligned16(q) || !aligned16(out)) return fail(NLLB_ATTN_EINVAL, "q and out must be 16-byte aligned");
    if ((rc = set_device(c))) return rc;
    return cross_dev(c, layer, n_sent, q, out);
}

}  // extern "C"

namespace nllb {

int attn_decode_self_planes(nllb_attn_ctx* c, int layer, int step, int n_sent, const float* q, const float* k_new,
                            const float* v_new, void* planes) {
    int rc = check_beam_call(c, layer, n_sent);
    if (rc) return rc;
    if (step < 0 || step >= c->d.max_tgt) return fail(NLLB_ATTN_EINVAL, "step out of range");
    if (!q || !k_new || !v_new || !planes) return fail(NLLB_ATTN_EINVAL, "q, k_new, v_new, planes are required");
    if ((rc = set_device(c))) return rc;
    SelfMode mode;
    if ((rc = self_mode(c, n_sent, &mode))) return rc;
    rc = decode_self_dev(c, layer, step, 0, n_sent, q, k_new, v_new, static_cast<float*>(planes), true, mode);
    if (rc == NLLB_ATTN_OK) self_done(c, mode);
    return rc;
}

int attn_cross_planes(nllb_attn_ctx* c, int layer, int n_sent, const float* q, void* planes) {
    int rc = check_beam_call(c, layer, n_sent);
    if (rc) return rc;
    if (!q || !planes) return fail(NLLB_ATTN_EINVAL, "q and planes are required");
    if ((rc = set_device(c))) return rc;
    return cross_dev(c, layer, n_sent, q, static_cast<float*>(planes), true);
}

}  // namespace nllb

extern "C" {

int nllb_attn_cross_host(nllb_attn_ctx* c, int layer, int n_sent, const float* q, float* out) {
    int rc = check_beam_call(c, layer, n_sent);
    if (rc) return rc;
    if (!q || !out) return fail(NLLB_ATTN_EINVAL, "q and out are required");
    if ((rc = set_device(c))) return rc;
    const size_t bytes = (size_t)n_sent * c->d.n_beams * c->d.n_heads * 64 * sizeof(float);
    if ((rc = ensure_stage(c, 0, bytes)) || (rc = ensure_stage(c, 3, bytes))) return rc;
    NLLB_CK(cudaMemcpyAsync(c->stg[0], q, bytes, cudaMemcpyHostToDevice, c->stream));
    if ((rc = cross_dev(c, layer, n_sent, static_cast<float*>(c->stg[0]), static_cast<float*>(c->stg[3]))))
        return rc;
    NLLB_CK(cudaMemcpyAsync(out, c->stg[3], bytes, cudaMemcpyDeviceToHost, c->stream));
    return finish_host_call(c);
}

// ---------------------------------------------------------------------------
// drop-ins for attention_head / attention_head_flash (pico.h:85-92)
// ---------------------------------------------------------------------------
}  // extern "C"

namespace {
struct ThreadCtx {
    nllb_attn_ctx* ctx = nullptr;
    ~ThreadCtx() {
        if (ctx) nllb_attn_destroy(ctx);
    }
};
thread_local ThreadCtx t_ctx;

int dropin_ctx(nllb_attn_ctx** out) {
    if (!t_ctx.ctx) {
        int dev = 0;
        if (const char* s = std::getenv("NLLB_ATTN_DEVICE")) dev = std::atoi(s);
        nllb_attn_dims d{};
        d.n_layers = 0;
        d.n_heads = 1;
        d.head_dim = 64;
        d.max_sentences = 0;
        d.n_beams = 1;
        int rc = nllb_attn_create(dev, &d, &t_ctx.ctx);
        if (rc) return rc;
    }
    *out = t_ctx.ctx;
    return NLLB_ATTN_OK;
}

// attention_head / attention_head_flash on the calling thread's context;
// with scores_buf (attention_head) the softmaxed score matrix is written
// there too, from the Q, K and mask the prefill call just staged on the
// device (staging slots 0, 1 and 5) into slot 3 (its output, already copied).
void single_head(const char* name, const float* Q, const float* K, const float* V, const float* mask,
                 float* out, int seq_len, int head_dim, float* scores_buf = nullptr) {
    nllb_attn_ctx* c = nullptr;
    int rc = dropin_ctx(&c);
    if (rc == NLLB_ATTN_OK) {
        nllb_attn_prefill_args a{};
        a.q = Q;
        a.k = K;
        a.v = V;
        a.out = out;
        a.batch = 1;
        a.n_heads = 1;
        a.seq_len = seq_len;
        a.head_dim = head_dim;
        a.stride_batch = (int64_t)seq_len * head_dim;
        a.stride_head = (int64_t)seq_len * head_dim;
        a.stride_row = head_dim;
        a.mask = mask;
        a.mask_stride_batch = (int64_t)seq_len * seq_len;
        a.mask_stride_head = 0;
        a.scale = 1.0f / sqrtf((float)head_dim);  // tensor.c:258, 289
        rc = nllb_attn_prefill_host(c, &a);
        if (rc == NLLB_ATTN_OK && scores_buf) {
            const size_t bytes = (size_t)seq_len * seq_len * sizeof(float);
            rc = ensure_stage(c, 3, bytes);
            if (rc == NLLB_ATTN_OK) {
                cudaError_t e = launch_head_scores(static_cast<const float*>(c->stg[0]),
                                                   static_cast<const float*>(c->stg[1]),
                                                   mask ? static_cast<const float*>(c->stg[5]) : nullptr,
                                                   static_cast<float*>(c->stg[3]), seq_len, a.scale, c->stream);
                if (e == cudaSuccess)
                    e = cudaMemcpyAsync(scores_buf, c->stg[3], bytes, cudaMemcpyDeviceToHost, c->stream);
                if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
                if (e != cudaSuccess) rc = fail(NLLB_ATTN_ECUDA, std::string("scores: ") + cudaGetErrorString(e));
            }
        }
    }
    t_last_status = rc;
    if (rc) std::fprintf(stderr, "%s: %s (%s)\n", name, nllb_attn_strerror(rc), t_last_error.c_str());
}
}  // namespace

extern "C" {

void nllb_attention_head(const float* Q, const float* K, const float* V, const float* mask, float* out,
                         float* scores_buf, int seq_len, int head_dim) {
    single_head("nllb_attention_head", Q, K, V, mask, out, seq_len, head_dim, scores_buf);
}

void nllb_attention_head_flash(const float* Q, const float* K, const float* V, const float* mask,
                               float* out, int seq_len, int head_dim) {
    single_head("nllb_attention_head_flash", Q, K, V, mask, out, seq_len, head_dim);
}

int nllb_attn_last_status(void) { return t_last_status; }

}  // extern "C"
