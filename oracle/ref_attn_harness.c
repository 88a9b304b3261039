/*  ref_attn_harness.c -- drives the MetalNLLB reference's own attention code.
 *
 *  TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/ from
 *  the reference sources where they lie (tensor.c and decoder.c are #included
 *  below, after ref_pico.h raises the capacity constants).  Used to generate
 *  the golden fixtures under tests/golden/ and, in bench.py's reference arm,
 *  to time the reference's CPU attention.  Never linked by the product.
 *
 *  The live attention of the reference is inlined in static functions:
 *    decoder_self_attn_cached   decoder.c:48-99   (per-beam KV cache)
 *    decoder_cross_attn_cached  decoder.c:103-152 (shared encoder memory)
 *  and the declared single-head API is attention_head / attention_head_flash
 *  (tensor.c:255-332).  The statics are reached by including decoder.c.
 *
 *  Injection ("bias trick"): the q/k/v projections are given in_features = 0,
 *  so mat_vec_int8 (tensor.c:144-196) returns exactly their bias vector, which
 *  carries the desired q, k or v.  The output projection is either the exact
 *  identity (int8 weight 1 on the diagonal, scale NULL -> 1.0f, no bias), which
 *  returns the attention output bit-for-bit, or (for timing) in_features = 0 so
 *  that only the attention loops themselves cost time.
 */
#include "ref_pico.h"
#include "tensor.c"
#include "decoder.c"

#include <pthread.h>
#include <time.h>

/* ---- layout queries (decoder.c:24-45) ----------------------------------- */

long ref_kv_cache_floats(void)    { return (long)KV_CACHE_TOTAL_FLOATS; }
long ref_kv_layer_floats(void)    { return (long)KV_CACHE_LAYER_STRIDE; }
long ref_xattn_cache_floats(void) { return (long)XATTN_CACHE_TOTAL_FLOATS; }
int  ref_max_gen_len(void)        { return MAX_GEN_LEN; }
int  ref_max_seq_len(void)        { return MAX_SEQ_LEN; }

/* float offset of (layer, K=0|V=1, head, pos) in a per-beam cache, decoder.c:26-28 */
long ref_sa_offset(int layer, int kv, int head, int pos) {
    long base = kv ? (long)SA_V_OFFSET(layer) : (long)SA_K_OFFSET(layer);
    return base + (long)head * SA_HEAD_STRIDE + (long)pos * HEAD_DIM;
}

/* float offset of (layer, K=0|V=1, src row) in the shared cross cache, decoder.c:32-34 */
long ref_xa_offset(int layer, int kv, int src) {
    long base = kv ? (long)XA_V_OFFSET(layer) : (long)XA_K_OFFSET(layer);
    return base + (long)src * D_MODEL;
}

/* ---- projection stand-ins ------------------------------------------------ */

static int8_t g_identity[D_MODEL * D_MODEL];
static pthread_once_t g_identity_once = PTHREAD_ONCE_INIT;
static void init_identity(void) {
    memset(g_identity, 0, sizeof(g_identity));
    for (int i = 0; i < D_MODEL; i++) g_identity[(size_t)i * D_MODEL + i] = 1;
}
static const int8_t g_dummy_w[16];

static void bias_linear(LinearInt8* l, const float* bias) {
    l->weight = g_dummy_w;
    l->scale = NULL;
    l->bias = bias;
    l->out_features = D_MODEL;
    l->in_features = 0;
}

static void make_attn(Attention* a, const float* q, const float* k,
                      const float* v, int exact_out) {
    pthread_once(&g_identity_once, init_identity);
    bias_linear(&a->q_proj, q);
    bias_linear(&a->k_proj, k);
    bias_linear(&a->v_proj, v);
    a->out_proj.weight = g_identity;
    a->out_proj.scale = NULL;
    a->out_proj.bias = NULL;
    a->out_proj.out_features = D_MODEL;
    a->out_proj.in_features = exact_out ? D_MODEL : 0;
}

/* One beam, one layer, one decode step of decoder_self_attn_cached:
 * writes k,v at position `step` of `kv_cache` and returns the attention
 * output over positions 0..step in `out` [D_MODEL] (head h at cols 64h). */
void ref_decode_self_beam(float* kv_cache, int layer, int step,
                          const float* q, const float* k, const float* v,
                          float* out, int exact_out) {
    Attention a;
    float x[D_MODEL];
    memset(x, 0, sizeof(x));
    make_attn(&a, q, k, v, exact_out);
    decoder_self_attn_cached(&a, x, out, kv_cache, layer, step, NULL);
}

/* One beam, one layer, one step (step > 0, memory already in the cache) of
 * decoder_cross_attn_cached over `n_src` encoder rows. */
void ref_cross_beam(float* xattn_cache, int layer, int n_src,
                    const float* q, float* out, int exact_out) {
    Attention a;
    float x[D_MODEL];
    memset(x, 0, sizeof(x));
    make_attn(&a, q, NULL, NULL, exact_out);
    decoder_cross_attn_cached(&a, x, NULL, n_src, out, xattn_cache, layer, 1, NULL);
}

/* Batched prefill through attention_head_flash (tensor.c:286), one call per
 * (batch, head) on contiguous [seq][64] slices of [B,H,S,64] tensors, with
 * the key-padding mask expressed as the additive [S][S] mask the API takes:
 * -1e9 on keys j >= valid_len[b] (finite, since the reference builds with
 * -ffast-math).  valid_len may be NULL (no mask). */
void ref_prefill_flash(const float* Q, const float* K, const float* V,
                       const int* valid_len, float* out,
                       int B, int H, int S) {
    float* mask = NULL;
    if (valid_len) mask = (float*)malloc((size_t)S * S * sizeof(float));
    for (int b = 0; b < B; b++) {
        if (mask) {
            for (int i = 0; i < S; i++)
                for (int j = 0; j < S; j++)
                    mask[(size_t)i * S + j] = (j >= valid_len[b]) ? -1e9f : 0.0f;
        }
        for (int h = 0; h < H; h++) {
            size_t off = ((size_t)b * H + h) * (size_t)S * HEAD_DIM;
            attention_head_flash(Q + off, K + off, V + off, mask, out + off, S, HEAD_DIM);
        }
    }
    free(mask);
}

/* The reference's INT8 linear layer, mat_vec_int8 (tensor.c:144-196), on M
 * input rows one after the other: out[m] = dequant(w) x[m] + bias, with the
 * CTranslate2 convention w / scale (tensor.c:75).  w [N][K] int8, scale [N],
 * bias [N] or NULL, x [M][K], out [M][N]. */
void ref_mat_vec_int8_rows(const int8_t* w, const float* scale, const float* bias, int N, int K,
                           const float* x, int M, float* out) {
    LinearInt8 l = {w, scale, bias, N, K};
    for (int m = 0; m < M; m++) mat_vec_int8(&l, x + (size_t)m * K, out + (size_t)m * N);
}

/* ---- timing of the reference attention on all host threads -------------- */

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + (double)ts.tv_nsec * 1e-9;
}

static uint64_t splitmix(uint64_t* s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static float urand_sym(uint64_t* s) {  /* U(-1.7,1.7): variance ~1 */
    return ((float)(splitmix(s) >> 40) / (float)(1ull << 24) - 0.5f) * 3.4641f;
}

typedef struct {
    int kind;            /* 0 decode sweep, 1 cross, 2 prefill */
    int n_items;         /* work items per phase */
    int n_threads;
    int n_beams;
    int phase_step;      /* decode: current step */
    float** cache_cur;   /* decode: [n_items] per-beam layer-0 caches */
    float** cache_nxt;
    const float* vec;    /* pool of random vectors */
    int vec_count;
    float* xattn;        /* cross: per-sentence caches */
    int n_src;
    const float* pq; const float* pk; const float* pv; float* po; int S; int H;
    const float* mask;
    pthread_barrier_t bar;
    volatile int stop;
} TimingJob;

typedef struct { TimingJob* job; int tid; } TimingArg;

static void run_items(TimingJob* j, int tid) {
    float out[D_MODEL];
    for (int it = tid; it < j->n_items; it += j->n_threads) {
        if (j->kind == 0) {
            int st = j->phase_step;
            const float* base = j->vec + (size_t)((it * 7 + st * 13) % j->vec_count) * 3 * D_MODEL;
            Attention a;
            float x[D_MODEL];
            memset(x, 0, sizeof(x));
            make_attn(&a, base, base + D_MODEL, base + 2 * D_MODEL, 0);
            decoder_self_attn_cached(&a, x, out, j->cache_cur[it], 0, st, NULL);
        } else if (j->kind == 1) {
            const float* q = j->vec + (size_t)(it % j->vec_count) * 3 * D_MODEL;
            int sent = it / j->n_beams;
            ref_cross_beam(j->xattn + (size_t)sent * (2 * MAX_SEQ_LEN * D_MODEL), 0,
                           j->n_src, q, out, 0);
        } else {
            size_t off = (size_t)it * (size_t)j->S * HEAD_DIM;
            float* o = j->po + off;
            attention_head_flash(j->pq + off, j->pk + off, j->pv + off,
                                 j->mask ? j->mask + (size_t)(it / j->H) * j->S * j->S : NULL,
                                 o, j->S, HEAD_DIM);
        }
    }
}

static void* timing_worker(void* p) {
    TimingArg* a = (TimingArg*)p;
    for (;;) {
        pthread_barrier_wait(&a->job->bar);
        if (a->job->stop) break;
        run_items(a->job, a->tid);
        pthread_barrier_wait(&a->job->bar);
    }
    return NULL;
}

static void run_phase(TimingJob* j, pthread_t* th, TimingArg* args, int start) {
    (void)th;
    if (start) { pthread_barrier_wait(&j->bar); }
    run_items(j, 0);
    pthread_barrier_wait(&j->bar);
    (void)args;
}

static void start_pool(TimingJob* j, pthread_t* th, TimingArg* args) {
    pthread_barrier_init(&j->bar, NULL, (unsigned)j->n_threads);
    j->stop = 0;
    for (int t = 1; t < j->n_threads; t++) {
        args[t].job = j;
        args[t].tid = t;
        pthread_create(&th[t], NULL, timing_worker, &args[t]);
    }
}

static void stop_pool(TimingJob* j, pthread_t* th) {
    j->stop = 1;
    pthread_barrier_wait(&j->bar);
    for (int t = 1; t < j->n_threads; t++) pthread_join(th[t], NULL);
    pthread_barrier_destroy(&j->bar);
}

/* Decoder self-attention decode sweep, the way main.c runs it: for each step
 * t in [0, n_steps), every sentence reorders its beams (a random permutation;
 * the child copies the parent's cache as main.c:481-482 does, restricted to
 * the one layer being run) and then every (sentence, beam) runs
 * decoder_self_attn_cached at step t.  (sentence, beam) items are spread over
 * n_threads threads (main.c:124-150 runs one beam per thread).  Returns the
 * wall time in seconds of the whole sweep. */
double ref_time_decode_sweep(int n_sent, int n_beams, int n_steps, int n_threads,
                             unsigned long long seed) {
    if (n_steps > MAX_GEN_LEN || n_threads < 1 || n_beams < 1) return -1.0;
    int n_items = n_sent * n_beams;
    size_t layer_floats = (size_t)KV_CACHE_LAYER_STRIDE;
    float** cur = (float**)malloc(sizeof(float*) * n_items);
    float** nxt = (float**)malloc(sizeof(float*) * n_items);
    for (int i = 0; i < n_items; i++) {
        cur[i] = (float*)calloc(layer_floats, sizeof(float));
        nxt[i] = (float*)calloc(layer_floats, sizeof(float));
    }
    int vec_count = 64;
    float* vec = (float*)malloc(sizeof(float) * (size_t)vec_count * 3 * D_MODEL);
    uint64_t s = seed;
    for (size_t i = 0; i < (size_t)vec_count * 3 * D_MODEL; i++) vec[i] = urand_sym(&s);

    TimingJob j;
    memset(&j, 0, sizeof(j));
    j.kind = 0; j.n_items = n_items; j.n_threads = n_threads; j.n_beams = n_beams;
    j.cache_cur = cur; j.cache_nxt = nxt; j.vec = vec; j.vec_count = vec_count;
    pthread_t* th = (pthread_t*)calloc((size_t)n_threads, sizeof(pthread_t));
    TimingArg* args = (TimingArg*)calloc((size_t)n_threads, sizeof(TimingArg));
    start_pool(&j, th, args);
    int* perm = (int*)malloc(sizeof(int) * n_beams);

    double t0 = now_s();
    for (int st = 0; st < n_steps; st++) {
        /* beam reorder by full copy into the other pool (main.c:462-488) */
        for (int sn = 0; sn < n_sent; sn++) {
            for (int b = 0; b < n_beams; b++) perm[b] = b;
            for (int b = n_beams - 1; b > 0; b--) {
                int r = (int)(splitmix(&s) % (uint64_t)(b + 1));
                int t = perm[b]; perm[b] = perm[r]; perm[r] = t;
            }
            for (int b = 0; b < n_beams; b++)
                memcpy(nxt[sn * n_beams + b], cur[sn * n_beams + perm[b]],
                       layer_floats * sizeof(float));
        }
        float** tmp = cur; cur = nxt; nxt = tmp;
        j.cache_cur = cur; j.cache_nxt = nxt;
        j.phase_step = st;
        run_phase(&j, th, args, 1);
    }
    double dt = now_s() - t0;

    stop_pool(&j, th);
    for (int i = 0; i < n_items; i++) { free(cur[i]); free(nxt[i]); }
    free(cur); free(nxt); free(vec); free(th); free(args); free(perm);
    return dt;
}

/* Cross-attention: n_steps steps of decoder_cross_attn_cached for every
 * (sentence, beam) over n_src rows of one layer's shared memory.  Returns
 * wall seconds. */
double ref_time_cross(int n_sent, int n_beams, int n_src, int n_steps, int n_threads,
                      unsigned long long seed) {
    if (n_src > MAX_SEQ_LEN || n_threads < 1) return -1.0;
    size_t per_sent = (size_t)2 * MAX_SEQ_LEN * D_MODEL;   /* layer 0 of XATTN layout */
    float* xattn = (float*)malloc(per_sent * (size_t)n_sent * sizeof(float));
    uint64_t s = seed;
    for (size_t i = 0; i < per_sent * (size_t)n_sent; i++) xattn[i] = urand_sym(&s);
    int vec_count = 64;
    float* vec = (float*)malloc(sizeof(float) * (size_t)vec_count * 3 * D_MODEL);
    for (size_t i = 0; i < (size_t)vec_count * 3 * D_MODEL; i++) vec[i] = urand_sym(&s);

    TimingJob j;
    memset(&j, 0, sizeof(j));
    j.kind = 1; j.n_items = n_sent * n_beams; j.n_threads = n_threads; j.n_beams = n_beams;
    j.vec = vec; j.vec_count = vec_count; j.xattn = xattn; j.n_src = n_src;
    pthread_t* th = (pthread_t*)calloc((size_t)n_threads, sizeof(pthread_t));
    TimingArg* args = (TimingArg*)calloc((size_t)n_threads, sizeof(TimingArg));
    start_pool(&j, th, args);
    double t0 = now_s();
    for (int st = 0; st < n_steps; st++) run_phase(&j, th, args, 1);
    double dt = now_s() - t0;
    stop_pool(&j, th);
    free(xattn); free(vec); free(th); free(args);
    return dt;
}

/* Prefill: attention_head_flash for every (batch, head) of [B,H,S,64] inputs
 * with the additive key-padding mask (-1e9 beyond valid_len[b]); (b,h) pairs
 * spread over n_threads.  Returns wall seconds for n_reps repetitions. */
double ref_time_prefill(int B, int H, int S, const int* valid_len, int n_reps,
                        int n_threads, unsigned long long seed) {
    if (S > MAX_SEQ_LEN || n_threads < 1) return -1.0;
    size_t n = (size_t)B * H * S * HEAD_DIM;
    float* q = (float*)malloc(n * sizeof(float));
    float* k = (float*)malloc(n * sizeof(float));
    float* v = (float*)malloc(n * sizeof(float));
    float* o = (float*)malloc(n * sizeof(float));
    uint64_t s = seed;
    for (size_t i = 0; i < n; i++) { q[i] = urand_sym(&s); k[i] = urand_sym(&s); v[i] = urand_sym(&s); }
    float* mask = NULL;
    if (valid_len) {
        mask = (float*)malloc((size_t)B * S * S * sizeof(float));
        for (int b = 0; b < B; b++)
            for (int i = 0; i < S; i++)
                for (int jj = 0; jj < S; jj++)
                    mask[((size_t)b * S + i) * S + jj] = (jj >= valid_len[b]) ? -1e9f : 0.0f;
    }
    TimingJob j;
    memset(&j, 0, sizeof(j));
    j.kind = 2; j.n_items = B * H; j.n_threads = n_threads;
    j.pq = q; j.pk = k; j.pv = v; j.po = o; j.S = S; j.H = H; j.mask = mask;
    pthread_t* th = (pthread_t*)calloc((size_t)n_threads, sizeof(pthread_t));
    TimingArg* args = (TimingArg*)calloc((size_t)n_threads, sizeof(TimingArg));
    start_pool(&j, th, args);
    double t0 = now_s();
    for (int r = 0; r < n_reps; r++) run_phase(&j, th, args, 1);
    double dt = now_s() - t0;
    stop_pool(&j, th);
    free(q); free(k); free(v); free(o); free(mask); free(th); free(args);
    return dt;
}
