/*  nllb_translate.h -- sentence-batched NLLB translation on one B200.
 *
 *  The engine around the attention path: it runs the reference engine's
 *  whole forward pass and beam search on the GPU for many sentences at once.
 *
 *    weights      loader.c:287-372 (CTranslate2-named INT8 safetensors file)
 *    encoder      pico_encode, encoder.c:250-287
 *    decoder      pico_decode_forward / decoder_layer_step, decoder.c:156-233
 *    vocabulary   pico_vocab_project, decoder.c:319-354 (language rows masked)
 *    beam search  main.c:294-528: steps 0 and 1 seed the beams, then per step
 *                 repetition penalty 1.2, no-repeat bigram, log-softmax, top-8
 *                 per beam, candidate sort, EOS bookkeeping, final choice by
 *                 length-normalised score; max_out = min(3*n_src+10, max_gen-4)
 *
 *  The attention runs through libnllb_attn's kernels; the rest (INT8 linear
 *  layers, LayerNorm, embeddings, vocabulary projection, penalties, top-k and
 *  the candidate selection of each step) are this library's kernels too: the
 *  decode loop runs on the device and the host only polls how many sentences
 *  are still running.
 *
 *  Returns NLLB_ATTN_* status codes (nllb_attn.h).
 */
#ifndef NLLB_TRANSLATE_H
#define NLLB_TRANSLATE_H

#include "nllb_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct nllb_model nllb_model;

typedef struct {
    int max_gen;                /* MAX_GEN_LEN (pico.h:19): caps the target at max_gen - 4 tokens */
    float repetition_penalty;   /* REPETITION_PENALTY (pico.h:100), 1.2 */
    int no_repeat_ngram;        /* NO_REPEAT_NGRAM_SIZE (pico.h:101): 2, or 0 to disable */
} nllb_translate_opts;

typedef struct {
    double encode_ms;           /* encoder + cross-attention memory, all sentences */
    double decode_ms;           /* decoder steps and beam search */
    int steps;                  /* decoder steps run (including the two seeding steps) */
    long long tokens_out;       /* emitted target tokens, EOS excluded (main.c:534-546) */
} nllb_translate_stats;

/* Upload the model in `path` to `device`.  max_sentences / max_src bound the
 * batch a later nllb_translate may pass. */
NLLB_ATTN_API int nllb_model_load(const char* path, int device, int max_sentences, int max_src,
                                  int max_gen, nllb_model** out);
NLLB_ATTN_API void nllb_model_free(nllb_model* m);

/* Translate n_sentences sources.  Sentence i is src_tokens[src_offsets[i] ..
 * src_offsets[i+1]) and must already be [src_lang] ... [2] as main.c:274-290
 * builds it.  out_tokens: [n_sentences][max_gen] (the best hypothesis's
 * tokens, EOS excluded, then -1), out_len: [n_sentences], out_score:
 * [n_sentences] length-normalised score (main.c:519-528).  Any output pointer
 * may be NULL.  Host pointers. */
NLLB_ATTN_API int nllb_translate(nllb_model* m, int n_sentences, const int* src_tokens,
                                 const int* src_offsets, int tgt_lang, const nllb_translate_opts* opts,
                                 int* out_tokens, int* out_len, float* out_score,
                                 nllb_translate_stats* stats);

/* Decision margins of the last nllb_translate call for sentence `sentence`:
 * out[t] = smallest gap between consecutive candidate scores among the best
 * n_beams+1 after the sort of step t+2 (main.c:455-460), i.e. how close the
 * beam choice of that step came to a tie.  Returns the number of steps
 * written (at most max_steps). */
NLLB_ATTN_API int nllb_translate_margins(const nllb_model* m, int sentence, float* out, int max_steps);

/* Kernel time by class.  nllb_translate_profile(m, 1) clears the totals and
 * makes the following nllb_translate calls time every launch of each kernel
 * class with a pair of CUDA events on the engine's stream (which orders the
 * stream at those points: a profiled call runs somewhat slower, without the
 * overlap of dependent launches there); 0 turns it off and clears.
 * nllb_translate_profile_read copies the totals of up to max_classes classes
 * and returns how many it wrote: per class its name, launches, summed
 * milliseconds, and algorithmic work -- dense FLOPs (2*M*N*K for a linear
 * layer, 4*S^2*64 per head for the encoder attention) and bytes (the
 * attention kernels: K/V rows, q/out, new k/v and beam history for
 * self-attention; memory rows and q/out for cross-attention). */
#define NLLB_PROF_CLASSES 14
typedef struct {
    char name[32];
    long long launches;
    double ms;
    double flops;
    double bytes;
} nllb_kernel_profile;
NLLB_ATTN_API int nllb_translate_profile(nllb_model* m, int enable);
NLLB_ATTN_API int nllb_translate_profile_read(const nllb_model* m, nllb_kernel_profile* out, int max_classes);

/* ---- INT8-weight linear layer -------------------------------------------
 * out[m][n] = sum_k x[m][k] * (w[n][k] * (1.0f / weight_scale[n])) + bias[n]
 * for M rows at once: mat_vec_int8 (tensor.c:144-196) batched, with the
 * CTranslate2 scale convention (the int8 value is DIVIDED by weight_scale).
 * With NLLB_LINEAR_RELU the result is clamped at 0 (relu, tensor.c:242-245);
 * a non-NULL residual (same layout as out) is added last (residual_add,
 * tensor.c:249-251).  Device pointers, row-major x [M][K], w [N][K],
 * out [M][N]; asynchronous on `stream` (a cudaStream_t, NULL = default).
 * More than 16 rows run on the tensor cores (int8 weights exact in bf16,
 * activations split into three bf16 parts, fp32 accumulation); there K must
 * be a multiple of 32.  A bounded device wait that gives up leaves the
 * outputs invalid and sets a per-device error word that stays set until
 * nllb_linear_int8_status reads it. */
#define NLLB_LINEAR_RELU 1
NLLB_ATTN_API int nllb_linear_int8(const float* x, int M, int K, const int8_t* w, const float* weight_scale,
                                   const float* bias, int N, float* out, const float* residual, int flags,
                                   void* stream);
/* Synchronises the current device, then reads and clears nllb_linear_int8's
 * error word there: NLLB_ATTN_ETIMEOUT if a call since the last query had a
 * bounded device wait give up (its outputs are invalid), else NLLB_ATTN_OK. */
NLLB_ATTN_API int nllb_linear_int8_status(void);

/* Same computation as nllb_linear_int8, for callers that cannot have a
 * library allocate device memory while they run -- a serving process that
 * hands out all device memory from its own pool reserved at start-up, or a
 * loop with a fixed memory plan that must not pay cudaMalloc's implicit
 * device synchronisation.  No counterpart in the reference (its mat-vec
 * needs no scratch).  Allocates nothing: the split-K scratch is a fixed
 * 8 MB array inside the library that every GPU loading the library holds
 * until exit.  The first call on a device looks that array up (device
 * current); make it before any stream capture.  Calls share the array:
 * calls whose kernels overlap on the GPU race.  At most
 * NLLB_LINEAR_NOALLOC_MAX_ROWS rows, _MAX_OUT outputs, _MAX_IN inputs;
 * larger shapes return NLLB_ATTN_ECAPACITY.  Beyond 16 rows K must be a
 * multiple of 32, as for nllb_linear_int8.  The device address and the SM
 * count are looked up once per device ordinal: a device reset after the
 * first call is not supported.  A bounded device wait that gives up sets an
 * error word in the same array, which no later call clears:
 * nllb_linear_int8_noalloc_status waits for `stream`, reads and clears it
 * (NLLB_ATTN_ETIMEOUT if set), and allocates nothing either. */
#define NLLB_LINEAR_NOALLOC_MAX_ROWS 256
#define NLLB_LINEAR_NOALLOC_MAX_OUT 4096
#define NLLB_LINEAR_NOALLOC_MAX_IN 4096
NLLB_ATTN_API int nllb_linear_int8_noalloc(const float* x, int M, int K, const int8_t* w,
                                           const float* weight_scale, const float* bias, int N, float* out,
                                           const float* residual, int flags, void* stream);
NLLB_ATTN_API int nllb_linear_int8_noalloc_status(void* stream);

/* ---- INT8 linear layer with weights prepared once --------------------------
 * A LinearInt8 (pico.h:26-32) made resident on the current GPU: the layer
 * keeps the caller's device pointers w [N][K], weight_scale [N] and bias [N]
 * (NULL: none) -- they must stay valid until nllb_linear_free -- plus its own
 * fp16 copy of w (exact) with TMA tensor maps.  nllb_linear_run computes
 * what nllb_linear_int8 computes for those weights: more than 16 rows run on
 * the TMA-fed tcgen05 kernels over the fp16 copy, fewer on the SIMT kernel
 * over the int8 matrix.  K must be a positive multiple of 64.  The reference
 * dequantises inside every mat_vec_int8 (tensor.c:144-196) and has no
 * prepared form; this is the form the translation engine keeps its layers in.
 * A layer owns a grow-only activation buffer: runs of one layer whose kernels
 * overlap on the GPU (different streams, no ordering) race on it.  The first
 * run with more rows than before allocates (and synchronises `stream`).
 * nllb_linear_status synchronises the device and reports a bounded device
 * wait that gave up (NLLB_ATTN_ETIMEOUT). */
typedef struct nllb_linear nllb_linear;
NLLB_ATTN_API int nllb_linear_prepare(const int8_t* w, const float* weight_scale, const float* bias, int N, int K,
                                      void* stream, nllb_linear** out);
NLLB_ATTN_API int nllb_linear_run(nllb_linear* layer, const float* x, int M, float* out, const float* residual,
                                  int flags, void* stream);
NLLB_ATTN_API int nllb_linear_status(nllb_linear* layer);
/* Test of the bounded device waits: if the next nllb_linear_run of this layer
 * takes the split-K tensor-core kernel (more than 16 rows, fewer output tiles
 * than the persistent kernel needs), its MMA thread first waits about 1 ms on
 * a barrier nothing arrives on; the launch then takes its timeout path,
 * writes no output and sets the layer's error word, which the next
 * nllb_linear_status reports as NLLB_ATTN_ETIMEOUT (and clears).  The layer
 * stays usable.  No counterpart in the reference. */
NLLB_ATTN_API int nllb_linear_test_expire_next_wait(nllb_linear* layer);
NLLB_ATTN_API void nllb_linear_free(nllb_linear* layer);

/* ---- per-step vocabulary operations of the beam search --------------------
 * nllb_apply_penalties: for each of `rows` rows of logits (row r at
 * logits + r*ld) and its token history (tokens + r*tokens_ld, n_tokens[r]
 * entries): apply_repetition_penalty (main.c:186-194) -- every occurrence of
 * a token at positions 2..n-1 other than 2 divides a positive logit by
 * `penalty` or multiplies a non-positive one, once per occurrence -- then,
 * with no_repeat_ngram 2, apply_no_repeat_ngram (main.c:196-213): every token
 * that followed an earlier occurrence of the last token gets -1e30 (token 2
 * excepted).  no_repeat_ngram: 0 (off) or 2.  Token ids outside [0, ld) in a
 * history are skipped (the reference would index past the row), and a length
 * above tokens_ld is cut to tokens_ld.
 * nllb_logsoftmax_topk: for each row, the k best entries of the row's
 * log-softmax -- log_softmax_inplace + find_topk (main.c:154-182) -- as
 * out_tok[r*k + j] / out_logp[r*k + j], best first, the lower index first
 * among equal logits; the logits are not modified.  Logits a few ulps apart
 * whose log-probabilities round to the same fp32 value keep their logit order
 * here, where find_topk puts the lower index first.  k: 4 or 8; at most 65535
 * rows.  ws: device scratch of nllb_logsoftmax_topk_ws_bytes(vocab, rows, k)
 * bytes, 16-byte aligned.
 * Device pointers; asynchronous on `stream` (a cudaStream_t, NULL = default). */
NLLB_ATTN_API int nllb_apply_penalties(float* logits, long long ld, int rows, const int* tokens, int tokens_ld,
                                       const int* n_tokens, float penalty, int no_repeat_ngram, void* stream);
NLLB_ATTN_API size_t nllb_logsoftmax_topk_ws_bytes(int vocab, int rows, int k);
NLLB_ATTN_API int nllb_logsoftmax_topk(const float* logits, long long ld, int vocab, int rows, int k,
                                       int* out_tok, float* out_logp, void* ws, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* NLLB_TRANSLATE_H */
