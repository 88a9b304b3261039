// search_api.cu -- the beam search's per-step vocabulary operations as entry
// points of their own: the repetition penalty and no-repeat-ngram ban
// (main.c:186-213) and log-softmax + top-k (main.c:154-182), on many rows of
// device-resident logits at once.  The translation engine launches the same
// kernels (engine_kernels.cu) inside its decode loop.
#include <string>

#include "engine_kernels.h"
#include "nllb_translate.h"

namespace nllb {
int set_error(int status, const std::string& msg);  // nllb_attn.cu
}

using namespace nllb;

#define SA_CK(call)                                                                                   \
    do {                                                                                              \
        const cudaError_t e_ = (call);                                                                \
        if (e_ != cudaSuccess) return nllb::set_error(NLLB_ATTN_ECUDA, std::string(#call ": ") + cudaGetErrorString(e_)); \
    } while (0)

extern "C" {

size_t nllb_logsoftmax_topk_ws_bytes(int vocab, int rows, int k) {
    if (vocab < 1 || rows < 1 || (k != 4 && k != 8)) return 0;
    return vocab_topk_ws_floats(vocab, rows, k) * sizeof(float);
}

int nllb_logsoftmax_topk(const float* logits, long long ld, int vocab, int rows, int k, int* out_tok,
                         float* out_logp, void* ws, void* stream) {
    if (rows < 0 || vocab < 1) return set_error(NLLB_ATTN_EINVAL, "rows >= 0 and vocab >= 1 required");
    if (k != 4 && k != 8) return set_error(NLLB_ATTN_EINVAL, "k must be 4 or 8");
    if (vocab < k) return set_error(NLLB_ATTN_EINVAL, "vocab must be at least k");
    if (rows > 65535) return set_error(NLLB_ATTN_ECAPACITY, "at most 65535 rows per call");
    if (rows == 0) return NLLB_ATTN_OK;
    if (!logits || !out_tok || !out_logp || !ws) return set_error(NLLB_ATTN_EINVAL, "null pointer");
    if (ld < vocab) return set_error(NLLB_ATTN_EINVAL, "ld must be at least vocab");
    if (reinterpret_cast<uintptr_t>(ws) & 15u) return set_error(NLLB_ATTN_EINVAL, "ws must be 16-byte aligned");
    SA_CK(launch_logsoftmax_topk(logits, (size_t)ld, vocab, rows, nullptr, k, out_tok, out_logp,
                                 static_cast<float*>(ws), static_cast<cudaStream_t>(stream)));
    return NLLB_ATTN_OK;
}

int nllb_apply_penalties(float* logits, long long ld, int rows, const int* tokens, int tokens_ld,
                         const int* n_tokens, float penalty, int no_repeat_ngram, void* stream) {
    if (rows < 0) return set_error(NLLB_ATTN_EINVAL, "rows >= 0 required");
    if (no_repeat_ngram != 0 && no_repeat_ngram != 2)
        return set_error(NLLB_ATTN_EINVAL, "no_repeat_ngram must be 0 or 2");
    if (!(penalty > 0.f)) return set_error(NLLB_ATTN_EINVAL, "penalty must be positive");
    if (rows == 0) return NLLB_ATTN_OK;
    if (!logits || !tokens || !n_tokens) return set_error(NLLB_ATTN_EINVAL, "null pointer");
    if (ld < 1 || tokens_ld < 1) return set_error(NLLB_ATTN_EINVAL, "ld and tokens_ld must be positive");
    SA_CK(launch_penalties(logits, (size_t)ld, tokens, tokens_ld, n_tokens, nullptr, rows, penalty, no_repeat_ngram,
                           static_cast<cudaStream_t>(stream)));
    return NLLB_ATTN_OK;
}

}  // extern "C"
