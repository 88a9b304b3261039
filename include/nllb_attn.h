/*  nllb_attn.h -- C ABI of the B200 attention path for the MetalNLLB engine.
 *
 *  libnllb_attn.so replaces the three attention loops of the reference's C11
 *  engine with sm_100a kernels:
 *
 *    encoder self-attention prefill     encoder.c:166-205 (multi_head_self_attn_flash),
 *                                       and the declared single-head API
 *                                       attention_head / attention_head_flash
 *                                       (pico.h:85-92, tensor.c:255-332)
 *    decoder self-attention, KV cache   decoder.c:48-99   (decoder_self_attn_cached)
 *    cross-attention, encoder memory    decoder.c:103-152 (decoder_cross_attn_cached)
 *
 *  plus the beam reorder of the per-beam KV caches (main.c:462-488), which is
 *  an index permutation here instead of a copy of every cache.
 *
 *  Conventions
 *  - Every int-returning call returns an NLLB_ATTN_* status (0 = success).
 *  - Plain calls take DEVICE pointers (cudaMalloc'd) and only enqueue work on
 *    the context's stream; they return before the GPU finishes.  Call
 *    nllb_attn_sync() (or synchronise the stream) before reading outputs.
 *  - *_host calls take HOST pointers (pageable or pinned), copy inputs in,
 *    run, copy outputs back and return once the outputs are written, the way
 *    the reference's call sites use their stack and heap buffers.
 *  - fp32 in, fp32 out.  head_dim must be 64 (NLLB-200: 16 heads x 64).
 *  - Rows of q/k/v/out hold all heads, head h at columns [64h, 64h+64), as the
 *    reference's projections produce them (decoder.c:57-59, encoder.c:159-163).
 *  - One context belongs to one device and is used by one host thread at a
 *    time.  The reference calls decoder attention from one thread per beam
 *    (main.c:124-150); here one call covers all beams of all sentences.
 *  - No call falls back to a CPU implementation.  Without a usable sm_100
 *    device nllb_attn_create() fails with NLLB_ATTN_ENODEV.
 */
#ifndef NLLB_ATTN_H
#define NLLB_ATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NLLB_ATTN_API __attribute__((visibility("default")))
#else
#define NLLB_ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define NLLB_ATTN_OK        0
#define NLLB_ATTN_EINVAL    1  /* bad argument: NULL pointer, size < 1, head_dim != 64, misaligned */
#define NLLB_ATTN_ECAPACITY 2  /* size beyond the capacity the context was created with */
#define NLLB_ATTN_ECUDA     3  /* a CUDA runtime call failed (see nllb_attn_last_error) */
#define NLLB_ATTN_ETIMEOUT  4  /* a bounded device-side wait gave up; the call's outputs are invalid */
#define NLLB_ATTN_ENODEV    5  /* no CUDA device, or the device is not compute capability 10.x */
#define NLLB_ATTN_ESTATE    6  /* call order violated (e.g. cross-attention before its memory is set) */

typedef struct nllb_attn_ctx nllb_attn_ctx;

/* Capacities fixed at creation; device buffers are sized from them.
 * The reference fixes the same quantities at compile time (pico.h:11-22). */
typedef struct {
    int n_layers;       /* decoder layers with a KV cache and a memory (12) */
    int n_heads;        /* attention heads (16) */
    int head_dim;       /* must be 64 */
    int max_sentences;  /* sentence slots resident on the device (0: prefill only) */
    int n_beams;        /* beams per sentence: 1, 2, 4 or 8 (BEAM_SIZE, pico.h:97) */
    int max_tgt;        /* KV-cache positions per beam (MAX_GEN_LEN, pico.h:19) */
    int max_src;        /* encoder-memory rows per sentence (MAX_SEQ_LEN, pico.h:18) */
} nllb_attn_dims;

/* Create a context on `device` (CUDA ordinal).  Allocates the KV caches
 * [n_layers][max_sentences][n_heads][max_tgt][n_beams][64] (K and V), the
 * encoder memory [n_layers][max_sentences][n_heads][max_src][64] (K and V),
 * the beam history and a small split-K workspace, all zeroed.
 * Replaces the calloc of per-beam caches in main.c:297-302. */
NLLB_ATTN_API int  nllb_attn_create(int device, const nllb_attn_dims* dims, nllb_attn_ctx** out_ctx);
NLLB_ATTN_API void nllb_attn_destroy(nllb_attn_ctx* ctx);

/* Device bytes nllb_attn_create would allocate for `dims`. */
NLLB_ATTN_API size_t nllb_attn_device_bytes(const nllb_attn_dims* dims);

/* Use `stream` (a cudaStream_t) for all later work; NULL restores the
 * context's own stream. */
NLLB_ATTN_API int   nllb_attn_set_stream(nllb_attn_ctx* ctx, void* stream);
NLLB_ATTN_API void* nllb_attn_get_stream(nllb_attn_ctx* ctx);

/* Wait for all enqueued work, then read and clear the device error word
 * (set by a kernel whose bounded wait gave up).  Returns NLLB_ATTN_ETIMEOUT
 * in that case. */
NLLB_ATTN_API int nllb_attn_sync(nllb_attn_ctx* ctx);

/* Forget all sentences: beam histories reset to the identity. */
NLLB_ATTN_API int nllb_attn_reset(nllb_attn_ctx* ctx);

NLLB_ATTN_API const char* nllb_attn_strerror(int status);
/* Text of the last failure seen on the calling thread ("" if none). */
NLLB_ATTN_API const char* nllb_attn_last_error(void);

/* ---- encoder self-attention prefill -------------------------------------
 * Replaces encoder.c:166-205 and attention_head_flash (tensor.c:286-332):
 * for every (batch b, head h, query row i)
 *    s_j  = (q_i . k_j) * scale + mask_ij        (j < seq_len)
 *    out_i = sum_j softmax(s)_j v_j
 * Element (b,h,row,d) of q/k/v/out is at b*stride_batch + h*stride_head +
 * row*stride_row + d (elements).  Both the engine's head-interleaved rows
 * (stride_head = 64, stride_row = n_heads*64) and [B,H,S,64] tensors fit.
 * Keys j >= valid_len[b] are excluded (the reference expresses the same
 * padding as an additive -1e9 mask, tensor.c:309); valid_len may be NULL,
 * entries lie in [0, seq_len], and 0 gives the plain mean of V over all
 * seq_len keys, which is what the -1e9 mask yields when every key is
 * masked.  mask (may be NULL) is an additive
 * fp32 mask, row i of (b,h) at mask + b*mask_stride_batch +
 * h*mask_stride_head + i*seq_len.  Pointers and strides must keep every row
 * 16-byte aligned. */
typedef struct {
    const float* q;
    const float* k;
    const float* v;
    float*       out;
    int batch, n_heads, seq_len, head_dim;
    int64_t stride_batch, stride_head, stride_row;
    const int*   valid_len;
    const float* mask;
    int64_t mask_stride_batch, mask_stride_head;
    float scale;            /* the reference uses 1/sqrt(head_dim) = 0.125 */
} nllb_attn_prefill_args;

NLLB_ATTN_API int nllb_attn_prefill(nllb_attn_ctx* ctx, const nllb_attn_prefill_args* args);
/* Same, with every pointer in args a host pointer. */
NLLB_ATTN_API int nllb_attn_prefill_host(nllb_attn_ctx* ctx, const nllb_attn_prefill_args* args);

/* ---- decoder self-attention over the per-beam KV cache ------------------
 * Replaces decoder.c:64-96 for every beam of sentences [0, n_sentences):
 * writes k_new/v_new at position `step` of each beam's cache (decoder.c:64-69)
 * and attends q over positions 0..step of that beam's history
 * (decoder.c:71-96: scores * 1/sqrt(64), softmax, P.V).
 * q, k_new, v_new, out: [n_sentences][n_beams][n_heads*64].
 * step must be < max_tgt; all sentences advance together. */
NLLB_ATTN_API int nllb_attn_decode_self(nllb_attn_ctx* ctx, int layer, int step, int n_sentences,
                          const float* q, const float* k_new, const float* v_new,
                          float* out);
NLLB_ATTN_API int nllb_attn_decode_self_host(nllb_attn_ctx* ctx, int layer, int step, int n_sentences,
                               const float* q, const float* k_new, const float* v_new,
                               float* out);

/* Beam reorder, replacing the cache copies of main.c:462-488 (and the
 * bootstrap copies main.c:335-340, 384-392): new beam b of sentence s
 * continues the history of old beam parent[s*n_beams + b], for every layer.
 * Applies to positions already written; costs O(n_sentences*max_tgt) bytes,
 * independent of the cache size.  parent: [n_sentences][n_beams] int32.
 * The reorder takes effect for every later call on the context.  It is
 * applied lazily: when the next nllb_attn_decode_self covers exactly these
 * n_sentences and they are all of the context's max_sentences, that launch
 * reads each beam's rows through its parent and writes the composed history
 * itself (one launch per step instead of two); otherwise a reorder kernel
 * runs first.  So nllb_attn_reorder's device buffer `parent` must stay valid
 * and unchanged until the next nllb_attn_decode_self, nllb_attn_reorder,
 * nllb_attn_sync or nllb_attn_reset call on the context.
 * nllb_attn_reorder_host checks the parents on the host and returns once
 * they are copied (the caller may reuse its buffer at once). */
NLLB_ATTN_API int nllb_attn_reorder(nllb_attn_ctx* ctx, int n_sentences, const int* parent);
NLLB_ATTN_API int nllb_attn_reorder_host(nllb_attn_ctx* ctx, int n_sentences, const int* parent);

/* Test of the bounded device waits: the next self-attention launch on this
 * context (nllb_attn_decode_self or _host, 4 beams) waits for a cache chunk
 * that it never requests, with a budget of about 1 ms, so that the wait runs
 * out.  That launch writes no output and sets the device error word, which
 * the call (_host) or the next nllb_attn_sync reports as NLLB_ATTN_ETIMEOUT;
 * the context stays usable.  No counterpart in the reference. */
NLLB_ATTN_API int nllb_attn_test_expire_next_wait(nllb_attn_ctx* ctx);
/* The same for the next cross-attention launch (nllb_attn_cross or _host,
 * 4 beams): it waits ~1 ms for a memory chunk that it never requests, writes
 * no output, and the error is reported as above. */
NLLB_ATTN_API int nllb_attn_test_expire_next_cross_wait(nllb_attn_ctx* ctx);

/* ---- cross-attention over the shared encoder memory ---------------------
 * Stores one sentence's projected encoder keys/values for one layer
 * (what decoder.c:118-125 writes into the shared cache at step 0).
 * Row r, head h of k/v is at k + r*stride_row + h*stride_head (elements):
 * stride_head 64 / stride_row n_heads*64 for the engine's rows,
 * stride_head n_src*64 / stride_row 64 for [H][n_src][64] tensors. */
NLLB_ATTN_API int nllb_attn_set_memory(nllb_attn_ctx* ctx, int layer, int sentence, int n_src,
                         const float* k, const float* v,
                         int64_t stride_head, int64_t stride_row);
NLLB_ATTN_API int nllb_attn_set_memory_host(nllb_attn_ctx* ctx, int layer, int sentence, int n_src,
                              const float* k, const float* v,
                              int64_t stride_head, int64_t stride_row);

/* decoder.c:128-149 for every beam of sentences [0, n_sentences): each
 * beam's query attends all n_src memory rows of its sentence.  The memory
 * is read once per call for all beams.  q, out: [n_sentences][n_beams][n_heads*64]. */
NLLB_ATTN_API int nllb_attn_cross(nllb_attn_ctx* ctx, int layer, int n_sentences,
                    const float* q, float* out);
NLLB_ATTN_API int nllb_attn_cross_host(nllb_attn_ctx* ctx, int layer, int n_sentences,
                         const float* q, float* out);

/* ---- drop-ins for the declared single-head API (pico.h:85-92) -----------
 * Same signatures and meaning as the reference's attention_head
 * (tensor.c:255-282) and attention_head_flash (tensor.c:286-332): host
 * pointers, Q/K/V/out [seq_len][head_dim], optional additive mask
 * [seq_len][seq_len].  They run on the calling thread's own context (device
 * from $NLLB_ATTN_DEVICE, default 0), created on first use.  head_dim must be
 * 64.  attention_head also leaves the softmaxed score matrix [seq_len][seq_len]
 * in scores_buf, as the reference does (tensor.c:258-277).
 * They return void like the originals; a failure is printed to stderr and
 * reported by nllb_attn_last_status(). */
NLLB_ATTN_API void nllb_attention_head(const float* Q, const float* K, const float* V,
                         const float* mask, float* out, float* scores_buf,
                         int seq_len, int head_dim);
NLLB_ATTN_API void nllb_attention_head_flash(const float* Q, const float* K, const float* V,
                               const float* mask, float* out,
                               int seq_len, int head_dim);
NLLB_ATTN_API int  nllb_attn_last_status(void);

#ifdef __cplusplus
}
#endif
#endif /* NLLB_ATTN_H */
