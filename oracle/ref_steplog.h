/*  ref_steplog.h -- per-step log of the reference beam search's sorted
 *  candidate scores.  TEST INFRASTRUCTURE ONLY: force-included (after
 *  ref_pico.h) into the reference's main.c for the _steplog programs that
 *  tests/golden/make_e2e_golden.py runs; nothing in the product links it.
 *
 *  The reference sorts each step's candidates by descending score
 *  (main.c:455-460), keeps the first BEAM_SIZE (main.c:466-484) and then
 *  prints its progress line followed by the only fflush() call in main.c
 *  (main.c:491-492), inside the step loop where `step`, `cands` and `nc` are
 *  in scope.  The macro below turns that call into "log the sorted scores,
 *  then fflush", so the program's arithmetic and output are unchanged; the
 *  scores go to stderr as one line per step:
 *
 *      [ref-step] <step> <nc> <score 0> <score 1> ... <score nc-1>
 *
 *  with %.9g, which round-trips an fp32 value exactly.  From these lines the
 *  golden generator computes the reference's own decision margins (the
 *  smallest gap between consecutive sorted scores among the first
 *  BEAM_SIZE + 1), which decide where a token id difference is exempt.
 */
#ifndef NLLB_REF_STEPLOG_H
#define NLLB_REF_STEPLOG_H
#include <stdio.h>
#include <stddef.h>

static void ref_steplog_emit(int step, const float* first_score, size_t stride_bytes, int nc) {
    const char* p = (const char*)first_score;
    fprintf(stderr, "[ref-step] %d %d", step, nc);
    for (int i = 0; i < nc; i++) fprintf(stderr, " %.9g", (double)*(const float*)(p + (size_t)i * stride_bytes));
    fputc('\n', stderr);
}

#define fflush(f) (ref_steplog_emit(step, &cands[0].score, sizeof cands[0], nc), fflush(f))
#endif
