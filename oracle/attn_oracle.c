/*  attn_oracle.c -- CPU restatement of the MetalNLLB attention path.
 *
 *  TEST INFRASTRUCTURE ONLY.  This is the checker the CUDA kernels are
 *  compared against; the product never links, loads or calls it.  Only
 *  tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 *
 *  Each function restates the arithmetic of the reference routine it names,
 *  in the same order of operations (fp32 throughout, max-subtracted softmax,
 *  scale applied after the dot product).  The restatement is pinned against
 *  the reference itself (compiled from its own sources by oracle/Makefile
 *  into oracle/_ref/) through the fixtures in tests/golden/.
 *
 *  Built without -ffast-math so its sums run in source order; the reference
 *  builds with -O3 -ffast-math (Makefile:20), so the two agree to rounding
 *  (a few ulp), not bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* softmax in place: max, expf(x-max), sum, divide.  tensor.c:227-238 */
void oracle_softmax(float* x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* Single head, two passes per query row: scores (+additive mask) and their
 * max, then exp-weighted V accumulation and one multiply by 1/sum.
 * tensor.c:286-332 (attention_head_flash); encoder.c:170-204 is the same
 * loop on head-interleaved rows. */
void oracle_attention_head_flash(const float* Q, const float* K, const float* V,
                                 const float* mask, float* out,
                                 int seq_len, int head_dim) {
    float scale = 1.0f / sqrtf((float)head_dim);
    float* scores = (float*)malloc(sizeof(float) * (size_t)(seq_len > 0 ? seq_len : 1));
    for (int i = 0; i < seq_len; i++) {
        const float* qi = Q + (size_t)i * head_dim;
        float* oi = out + (size_t)i * head_dim;
        float mx = -1e30f;
        for (int j = 0; j < seq_len; j++) {
            const float* kj = K + (size_t)j * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; d++) dot += qi[d] * kj[d];
            scores[j] = dot * scale;
            if (mask) scores[j] += mask[(size_t)i * seq_len + j];
            if (scores[j] > mx) mx = scores[j];
        }
        float sum = 0.0f;
        for (int d = 0; d < head_dim; d++) oi[d] = 0.0f;
        for (int j = 0; j < seq_len; j++) {
            float e = expf(scores[j] - mx);
            sum += e;
            const float* vj = V + (size_t)j * head_dim;
            for (int d = 0; d < head_dim; d++) oi[d] += e * vj[d];
        }
        float inv = 1.0f / sum;
        for (int d = 0; d < head_dim; d++) oi[d] *= inv;
    }
    free(scores);
}

/* Single head with a full [seq][seq] score buffer, softmax per row, then a
 * separate P.V pass.  tensor.c:255-282 (attention_head). */
void oracle_attention_head(const float* Q, const float* K, const float* V,
                           const float* mask, float* out, float* scores_buf,
                           int seq_len, int head_dim) {
    float scale = 1.0f / sqrtf((float)head_dim);
    for (int i = 0; i < seq_len; i++) {
        for (int j = 0; j < seq_len; j++) {
            const float* qi = Q + (size_t)i * head_dim;
            const float* kj = K + (size_t)j * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; d++) dot += qi[d] * kj[d];
            scores_buf[(size_t)i * seq_len + j] = dot * scale;
            if (mask) scores_buf[(size_t)i * seq_len + j] += mask[(size_t)i * seq_len + j];
        }
        oracle_softmax(scores_buf + (size_t)i * seq_len, seq_len);
    }
    for (int i = 0; i < seq_len; i++) {
        float* oi = out + (size_t)i * head_dim;
        for (int d = 0; d < head_dim; d++) oi[d] = 0.0f;
        for (int j = 0; j < seq_len; j++) {
            float a = scores_buf[(size_t)i * seq_len + j];
            const float* vj = V + (size_t)j * head_dim;
            for (int d = 0; d < head_dim; d++) oi[d] += a * vj[d];
        }
    }
}

/* Batched, strided prefill with the semantics of attention_head_flash per
 * (batch, head): element (b,h,s,d) of q/k/v/out sits at
 * b*sb + h*sh + s*sr + d.  Key padding (valid_len[b], may be NULL) is the
 * additive -1e9 mask the reference API takes (tensor.c:309) on keys
 * j >= valid_len[b]; `mask` (may be NULL) is a further additive mask whose
 * row i of (b,h) starts at mask + b*msb + h*msh + i*seq_len.  `scale`
 * replaces the reference's 1/sqrt(head_dim) (tensor.c:289). */
void oracle_prefill(const float* q, const float* k, const float* v, float* out,
                    int B, int H, int S, int D,
                    long long sb, long long sh, long long sr,
                    const int* valid_len, const float* mask,
                    long long msb, long long msh, float scale) {
    float* scores = (float*)malloc(sizeof(float) * (size_t)(S > 0 ? S : 1));
    for (int b = 0; b < B; b++) {
        for (int h = 0; h < H; h++) {
            const float* Qh = q + b * sb + h * sh;
            const float* Kh = k + b * sb + h * sh;
            const float* Vh = v + b * sb + h * sh;
            float* Oh = out + b * sb + h * sh;
            const float* Mh = mask ? mask + b * msb + h * msh : NULL;
            for (int i = 0; i < S; i++) {
                const float* qi = Qh + i * sr;
                float* oi = Oh + i * sr;
                float mx = -1e30f;
                for (int j = 0; j < S; j++) {
                    const float* kj = Kh + j * sr;
                    float dot = 0.0f;
                    for (int d = 0; d < D; d++) dot += qi[d] * kj[d];
                    float sc = dot * scale;
                    if (valid_len && j >= valid_len[b]) sc += -1e9f;
                    if (Mh) sc += Mh[(size_t)i * S + j];
                    scores[j] = sc;
                    if (sc > mx) mx = sc;
                }
                float sum = 0.0f;
                for (int d = 0; d < D; d++) oi[d] = 0.0f;
                for (int j = 0; j < S; j++) {
                    float e = expf(scores[j] - mx);
                    sum += e;
                    const float* vj = Vh + j * sr;
                    for (int d = 0; d < D; d++) oi[d] += e * vj[d];
                }
                float inv = 1.0f / sum;
                for (int d = 0; d < D; d++) oi[d] *= inv;
            }
        }
    }
    free(scores);
}

/* One beam, one layer, one decode step over a per-beam cache laid out as the
 * reference lays out one layer of it (decoder.c:24-30):
 *   cache[kv][head][max_gen][head_dim], kv 0 = K, 1 = V.
 * Writes k,v (head h at cols h*head_dim of the [n_heads*head_dim] vectors)
 * at position `step` (decoder.c:64-69), then per head: scores over the
 * step+1 cached keys times 1/sqrt(head_dim), softmax, P.V
 * (decoder.c:71-96).  out is [n_heads*head_dim]. */
void oracle_decode_self_beam(float* cache, int n_heads, int head_dim, int max_gen,
                             int step, const float* q, const float* k,
                             const float* v, float* out) {
    size_t head_stride = (size_t)max_gen * head_dim;
    float* Kc = cache;
    float* Vc = cache + (size_t)n_heads * head_stride;
    for (int h = 0; h < n_heads; h++) {
        memcpy(Kc + h * head_stride + (size_t)step * head_dim, k + h * head_dim,
               sizeof(float) * head_dim);
        memcpy(Vc + h * head_stride + (size_t)step * head_dim, v + h * head_dim,
               sizeof(float) * head_dim);
    }
    int ctx_len = step + 1;
    float scale = 1.0f / sqrtf((float)head_dim);
    float* scores = (float*)malloc(sizeof(float) * (size_t)ctx_len);
    for (int h = 0; h < n_heads; h++) {
        const float* qh = q + h * head_dim;
        const float* Kh = Kc + h * head_stride;
        const float* Vh = Vc + h * head_stride;
        for (int j = 0; j < ctx_len; j++) {
            const float* kj = Kh + (size_t)j * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; d++) dot += qh[d] * kj[d];
            scores[j] = dot * scale;
        }
        oracle_softmax(scores, ctx_len);
        float* oh = out + h * head_dim;
        for (int d = 0; d < head_dim; d++) oh[d] = 0.0f;
        for (int j = 0; j < ctx_len; j++) {
            const float* vj = Vh + (size_t)j * head_dim;
            for (int d = 0; d < head_dim; d++) oh[d] += scores[j] * vj[d];
        }
    }
    free(scores);
}

/* One beam, one layer, one step of cross-attention over n_src encoder rows
 * (decoder.c:128-149).  K and V rows hold all heads (head h at cols
 * h*head_dim), consecutive rows `row_stride` floats apart, as in the shared
 * cache (decoder.c:32-34, rows D_MODEL apart). */
void oracle_cross_beam(const float* K, const float* V, long long row_stride,
                       int n_src, int n_heads, int head_dim,
                       const float* q, float* out) {
    float scale = 1.0f / sqrtf((float)head_dim);
    float* scores = (float*)malloc(sizeof(float) * (size_t)(n_src > 0 ? n_src : 1));
    for (int h = 0; h < n_heads; h++) {
        const float* qh = q + h * head_dim;
        for (int s = 0; s < n_src; s++) {
            const float* ks = K + s * row_stride + h * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; d++) dot += qh[d] * ks[d];
            scores[s] = dot * scale;
        }
        oracle_softmax(scores, n_src);
        float* oh = out + h * head_dim;
        for (int d = 0; d < head_dim; d++) oh[d] = 0.0f;
        for (int s = 0; s < n_src; s++) {
            const float* vs = V + s * row_stride + h * head_dim;
            for (int d = 0; d < head_dim; d++) oh[d] += scores[s] * vs[d];
        }
    }
    free(scores);
}

/* Whole decode sweep of one sentence the way the reference's host loop runs
 * it: before step t, beams are reordered by copying the parent's cache into
 * the child's (main.c:462-488, with double-buffered pools main.c:298-301);
 * then each beam runs one decode step.  parents is [n_steps][n_beams],
 * q/k/v/out are [n_steps][n_beams][n_heads*head_dim].  caches must hold
 * 2*n_beams per-beam layer caches of 2*n_heads*max_gen*head_dim floats
 * (pool 0 then pool 1), zero-initialised by the caller. */
void oracle_decode_sweep(float* caches, int n_beams, int n_heads, int head_dim,
                         int max_gen, int n_steps, const int* parents,
                         const float* q, const float* k, const float* v,
                         float* out) {
    size_t per = (size_t)2 * n_heads * max_gen * head_dim;
    size_t dm = (size_t)n_heads * head_dim;
    int cur = 0;
    for (int t = 0; t < n_steps; t++) {
        if (parents) {
            float* src = caches + (size_t)cur * n_beams * per;
            float* dst = caches + (size_t)(1 - cur) * n_beams * per;
            for (int b = 0; b < n_beams; b++)
                memcpy(dst + b * per, src + (size_t)parents[t * n_beams + b] * per,
                       per * sizeof(float));
            cur = 1 - cur;
        }
        float* pool = caches + (size_t)cur * n_beams * per;
        for (int b = 0; b < n_beams; b++) {
            size_t o = ((size_t)t * n_beams + b) * dm;
            oracle_decode_self_beam(pool + b * per, n_heads, head_dim, max_gen, t,
                                    q + o, k + o, v + o, out + o);
        }
    }
}
