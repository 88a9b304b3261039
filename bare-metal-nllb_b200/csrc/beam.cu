// beam.cu -- beam-search bookkeeping of one decoder step on the device.
//
// Restates main.c:411-511 (the per-step part of the reference's beam search)
// for many sentences at once, one warp per sentence, so the decode loop never
// waits for the host between steps:
//   * candidates: every finished beam carries itself with token 2 and its
//     score, then every unfinished beam offers its 8 best tokens with
//     score + log-probability, in beam order (main.c:413-450);
//   * the reference's exchange sort, descending (main.c:456-460), run for its
//     first NBEAM + 1 outer iterations only: iteration i writes positions >= i,
//     so positions 0..NBEAM (all that is read afterwards) are final by then;
//   * the best 4 candidates become the new beams: tokens of the parent plus
//     the new token, finished when the token is 2, the score of the step that
//     emitted token 2 kept as eos_score (main.c:462-488);
//   * a finished new beam is also recorded among at most 8 completed
//     hypotheses of the sentence (main.c:489-500);
//   * the sentence stops when the next step would reach max_out + 2 or no
//     beam is unfinished (main.c:411-412, 503-509).
// Lane 0 does the scalar work in the reference's order (its float compares
// and adds are the reference's); the lanes load the beams' top-k lists and
// copy token histories.
#include "device_common.cuh"
#include "engine_kernels.h"

namespace nllb {

namespace {

constexpr int NBEAM = 4, TOPK = 8, MAXC = NBEAM * TOPK + NBEAM, MAX_DONE = 8;
constexpr int SENT_PER_CTA = 4;

__global__ void __launch_bounds__(32 * SENT_PER_CTA) beam_select_kernel(const BeamState B, int cur, const int* top_tok,
                                                                         const float* top_lp, int step) {
    __shared__ int c_beam[SENT_PER_CTA][MAXC], c_tok[SENT_PER_CTA][MAXC];
    __shared__ float c_score[SENT_PER_CTA][MAXC];
    __shared__ int n_par[SENT_PER_CTA][NBEAM], n_tok[SENT_PER_CTA][NBEAM], n_len[SENT_PER_CTA][NBEAM];
    __shared__ int n_slot[SENT_PER_CTA][NBEAM];
    __shared__ int s_done[SENT_PER_CTA];
    __shared__ int s_tok[SENT_PER_CTA][NBEAM * TOPK];
    __shared__ float s_lp[SENT_PER_CTA][NBEAM * TOPK];
    static_assert(NBEAM * TOPK == 32, "one top-k entry per lane");
    pdl_launch_dependents();
    pdl_wait_primary();  // the top-k lists come from the previous kernel
    const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int s = blockIdx.x * SENT_PER_CTA + wi;
    if (s >= B.n_sent) return;  // uniform per warp
    const int G = B.G;
    const int* btc = cur ? B.bt1 : B.bt0;
    int* btn = cur ? B.bt0 : B.bt1;
    const int r0 = s * NBEAM;

    if (lane == 0) s_done[wi] = B.done[s];
    s_tok[wi][lane] = top_tok[(size_t)r0 * TOPK + lane];  // the 4 beams' lists are contiguous
    s_lp[wi][lane] = top_lp[(size_t)r0 * TOPK + lane];
    __syncwarp();
    if (s_done[wi]) {
        // finished sentence: beams unchanged (carried into the other buffer), parents identity
        for (int b = 0; b < NBEAM; ++b) {
            const int n = B.bn[r0 + b];
            for (int p = lane; p < n; p += 32) btn[(size_t)(r0 + b) * G + p] = btc[(size_t)(r0 + b) * G + p];
        }
        if (lane < NBEAM) B.parent[r0 + lane] = lane;
        return;
    }

    if (lane == 0) {
        int* cb = c_beam[wi];
        int* ct = c_tok[wi];
        float* cs = c_score[wi];
        int nc = 0;
        for (int b = 0; b < NBEAM; ++b)
            if (B.bfin[r0 + b]) cb[nc] = b, ct[nc] = 2, cs[nc] = B.bsc[r0 + b], ++nc;
        for (int b = 0; b < NBEAM; ++b) {
            if (B.bfin[r0 + b]) continue;
            const float base = B.bsc[r0 + b];
            for (int k = 0; k < TOPK; ++k) {
                cb[nc] = b;
                ct[nc] = s_tok[wi][b * TOPK + k];
                cs[nc] = base + s_lp[wi][b * TOPK + k];
                ++nc;
            }
        }
        const int n_outer = nc - 1 < NBEAM + 1 ? nc - 1 : NBEAM + 1;
        for (int i = 0; i < n_outer; ++i)
            for (int j = i + 1; j < nc; ++j)
                if (cs[j] > cs[i]) {
                    const int tb = cb[i], tt = ct[i];
                    const float tsc = cs[i];
                    cb[i] = cb[j], ct[i] = ct[j], cs[i] = cs[j];
                    cb[j] = tb, ct[j] = tt, cs[j] = tsc;
                }
        float gap = INFINITY;
        const int lim = nc < NBEAM + 1 ? nc : NBEAM + 1;
        for (int i = 0; i + 1 < lim; ++i) gap = fminf(gap, cs[i] - cs[i + 1]);
        B.margins[(size_t)s * G + B.mcnt[s]] = gap;
        B.mcnt[s] += 1;
        int n_active = 0;
        float nsc[NBEAM], neos[NBEAM];
        int nfin[NBEAM];
        for (int i = 0; i < NBEAM; ++i) {
            const int par = cb[i];
            n_par[wi][i] = par;
            n_tok[wi][i] = ct[i];
            n_len[wi][i] = B.bn[r0 + par] + 1;
            nsc[i] = cs[i];
            nfin[i] = ct[i] == 2;
            neos[i] = nfin[i] ? cs[i] - B.bsc[r0 + par] : B.beos[r0 + par];
            n_slot[wi][i] = -1;
            if (nfin[i] && B.ccnt[s] < MAX_DONE) n_slot[wi][i] = B.ccnt[s]++;
            n_active += !nfin[i];
        }
        const int done = (step + 1 >= B.maxo[s] + 2) || n_active == 0;
        B.done[s] = (unsigned char)done;
        for (int i = 0; i < NBEAM; ++i) {
            const int r = r0 + i;
            B.bn[r] = n_len[wi][i];
            B.bsc[r] = nsc[i];
            B.beos[r] = neos[i];
            B.bfin[r] = (unsigned char)nfin[i];
            B.parent[r] = n_par[wi][i];
            B.tok[r] = n_tok[wi][i];
            B.active[r] = (unsigned char)(!done && !nfin[i]);
            const int c = n_slot[wi][i];
            if (c >= 0) {
                B.cn[s * MAX_DONE + c] = n_len[wi][i];
                B.csc[s * MAX_DONE + c] = nsc[i];
                B.ceos[s * MAX_DONE + c] = neos[i];
            }
        }
        if (!done) atomicAdd(&B.live[step], 1);
    }
    __syncwarp();
    // new token histories: the parent's tokens, then the new token
    for (int i = 0; i < NBEAM; ++i) {
        const int par = n_par[wi][i], n_old = n_len[wi][i] - 1;
        const int* src = btc + (size_t)(r0 + par) * G;
        int* dst = btn + (size_t)(r0 + i) * G;
        for (int p = lane; p < n_old; p += 32) dst[p] = src[p];
        if (lane == 0) dst[n_old] = n_tok[wi][i];
        const int c = n_slot[wi][i];
        if (c >= 0) {
            int* cd = B.ctok + ((size_t)s * MAX_DONE + c) * G;
            for (int p = lane; p < n_old; p += 32) cd[p] = src[p];
            if (lane == 0) cd[n_old] = n_tok[wi][i];
        }
    }
}

}  // namespace

cudaError_t launch_beam_select(const BeamState& b, int cur, const int* top_tok, const float* top_lp, int step,
                               cudaStream_t st) {
    if (b.n_sent <= 0) return cudaSuccess;
    return launch_pdl(beam_select_kernel, dim3((b.n_sent + SENT_PER_CTA - 1) / SENT_PER_CTA),
                      dim3(32 * SENT_PER_CTA), 0, st, b, cur, top_tok, top_lp, step);
}

}  // namespace nllb
