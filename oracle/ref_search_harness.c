/*  ref_search_harness.c -- exposes the reference's per-step vocabulary
 *  operations of the beam search.
 *
 *  TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/ from
 *  the reference sources where they lie: main.c is #included below with its
 *  main() renamed, and linked with the reference's other sources under the
 *  reference program's own flags, so the static functions called here are the
 *  ones the reference program runs:
 *    log_softmax_inplace       main.c:154-161
 *    find_topk                 main.c:165-182
 *    apply_repetition_penalty  main.c:186-194
 *    apply_no_repeat_ngram     main.c:196-213
 *  Used by tests/ to pin the numpy restatements in oracle/pyoracle.py.  Never
 *  linked by the product.
 */
#define main nllb_ref_program_main
#include "main.c"
#undef main

/* rows x n logits (row stride ld); in place, as the reference does per beam */
void ref_apply_penalties(float* logits, long ld, int rows, const int* tokens, int tokens_ld,
                         const int* n_tokens, float penalty, int ngram) {
    for (int r = 0; r < rows; r++) {
        float* lg = logits + (long)r * ld;
        const int* tk = tokens + (long)r * tokens_ld;
        apply_repetition_penalty(lg, tk, n_tokens[r], penalty);
        if (ngram > 0) apply_no_repeat_ngram(lg, tk, n_tokens[r], ngram);
    }
}

/* log-softmax of each row in place (n entries), then its k best */
void ref_log_softmax_topk(float* logits, long ld, int n, int rows, int k, int* out_tok, float* out_sc) {
    for (int r = 0; r < rows; r++) {
        float* lg = logits + (long)r * ld;
        log_softmax_inplace(lg, n);
        find_topk(lg, n, k, out_tok + (long)r * k, out_sc + (long)r * k);
    }
}
