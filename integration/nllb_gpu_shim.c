/*  nllb_gpu_shim.c -- see nllb_gpu_shim.h.  C11 + pthreads, built with the
 *  reference's own flags and capacity constants; links libnllb_attn.so.
 */
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "nllb_attn.h"
#include "nllb_gpu_shim.h"

static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t g_cv = PTHREAD_COND_INITIALIZER;
static nllb_attn_ctx* g_ctx;

/* the reference's per-beam cache pointers (main.c:298-301) as handles */
static const float* g_handle[2][BEAM_SIZE];

/* one slot per beam for the q/k/v the beam threads leave at a meeting */
static float g_q[BEAM_SIZE][D_MODEL], g_k[BEAM_SIZE][D_MODEL], g_v[BEAM_SIZE][D_MODEL];
static float g_o[BEAM_SIZE][D_MODEL];
static int g_arrived;
static unsigned long g_generation;
static int g_expect_step = -1, g_expect_n = 1;
static _Thread_local int t_beam;  /* the beam this thread decodes (from its cache pointer) */

/* parents staged by the step's cache copies, applied before the next call */
static int g_parent[BEAM_SIZE];
static int g_pending;

static void die(const char* what, int rc) {
    fprintf(stderr, "[nllb-gpu] %s: %s (%s)\n", what, nllb_attn_strerror(rc), nllb_attn_last_error());
    exit(1);
}

static void destroy_ctx(void) {
    if (g_ctx) nllb_attn_destroy(g_ctx);
    g_ctx = NULL;
}

/* The device context, created on first use with the program's capacities
 * (pico.h:11-22, BEAM_SIZE pico.h:97): one sentence, BEAM_SIZE beams.
 * Device: $NLLB_ATTN_DEVICE, default 0.  Called with g_mu held. */
static nllb_attn_ctx* ctx(void) {
    if (!g_ctx) {
        nllb_attn_dims d = {DECODER_LAYERS, N_HEADS, HEAD_DIM, 1, BEAM_SIZE, MAX_GEN_LEN, MAX_SEQ_LEN};
        const char* dev = getenv("NLLB_ATTN_DEVICE");
        const int rc = nllb_attn_create(dev ? atoi(dev) : 0, &d, &g_ctx);
        if (rc) die("nllb_attn_create", rc);
        atexit(destroy_ctx);
    }
    return g_ctx;
}

static int beam_of(const float* cache) {
    for (int p = 0; p < 2; p++)
        for (int b = 0; b < BEAM_SIZE; b++)
            if (g_handle[p][b] == cache) return b;
    fprintf(stderr, "[nllb-gpu] unknown KV-cache pointer\n");
    exit(1);
}

float* nllb_gpu_beam_cache(int pool, int beam) {
    float* h = (float*)calloc(16, sizeof(float));  /* freed by main.c's cleanup */
    if (!h || pool < 0 || pool > 1 || beam < 0 || beam >= BEAM_SIZE) {
        fprintf(stderr, "[nllb-gpu] bad KV-cache slot\n");
        exit(1);
    }
    pthread_mutex_lock(&g_mu);
    g_handle[pool][beam] = h;
    pthread_mutex_unlock(&g_mu);
    return h;
}

void nllb_gpu_copy_beam(const float* dst_cache, const float* src_cache) {
    pthread_mutex_lock(&g_mu);
    int parent[BEAM_SIZE];
    for (int b = 0; b < BEAM_SIZE; b++) parent[b] = b;
    parent[beam_of(dst_cache)] = beam_of(src_cache);
    const int rc = nllb_attn_reorder_host(ctx(), 1, parent);
    pthread_mutex_unlock(&g_mu);
    if (rc) die("nllb_attn_reorder_host", rc);
}

void nllb_gpu_stage_copy(const float* dst_cache, const float* src_cache) {
    pthread_mutex_lock(&g_mu);
    if (!g_pending) {
        for (int b = 0; b < BEAM_SIZE; b++) g_parent[b] = b;
        g_pending = 1;
    }
    g_parent[beam_of(dst_cache)] = beam_of(src_cache);
    pthread_mutex_unlock(&g_mu);
}

void nllb_gpu_expect_beams(int step, int n_beams) {
    pthread_mutex_lock(&g_mu);
    g_expect_step = step;
    g_expect_n = n_beams > 0 ? n_beams : 1;
    pthread_mutex_unlock(&g_mu);
}

/* Called with g_mu held by a beam thread that has left its inputs: returns 1
 * in the thread that completes the meeting (it makes the call), 0 in the
 * others once that call is done. */
static int arrive(int step) {
    const int expect = (step == g_expect_step) ? g_expect_n : 1;
    if (++g_arrived == expect) return 1;
    const unsigned long gen = g_generation;
    while (gen == g_generation) pthread_cond_wait(&g_cv, &g_mu);
    return 0;
}

static void release(void) {
    g_arrived = 0;
    g_generation++;
    pthread_cond_broadcast(&g_cv);
}

void nllb_gpu_encoder_attention(const float* Q, const float* K, const float* V, float* head_out, int seq_len) {
    nllb_attn_prefill_args a;
    memset(&a, 0, sizeof(a));
    a.q = Q;
    a.k = K;
    a.v = V;
    a.out = head_out;
    a.batch = 1;
    a.n_heads = N_HEADS;
    a.seq_len = seq_len;
    a.head_dim = HEAD_DIM;
    a.stride_batch = (int64_t)seq_len * D_MODEL;  /* one sequence */
    a.stride_head = HEAD_DIM;                     /* head h at columns 64h (encoder.c:171) */
    a.stride_row = D_MODEL;                       /* token rows */
    a.scale = 1.0f / sqrtf((float)HEAD_DIM);      /* encoder.c:167 */
    pthread_mutex_lock(&g_mu);
    const int rc = nllb_attn_prefill_host(ctx(), &a);
    pthread_mutex_unlock(&g_mu);
    if (rc) die("nllb_attn_prefill_host", rc);
}

void nllb_gpu_self_attention(const float* kv_cache, int layer, int step, const float* q, const float* k,
                             const float* v, float* out) {
    pthread_mutex_lock(&g_mu);
    const int b = beam_of(kv_cache);
    t_beam = b;
    memcpy(g_q[b], q, sizeof(g_q[b]));
    memcpy(g_k[b], k, sizeof(g_k[b]));
    memcpy(g_v[b], v, sizeof(g_v[b]));
    int rc = 0;
    if (arrive(step)) {
        if (g_pending) {  /* the previous step's parents (main.c:481-482) */
            rc = nllb_attn_reorder_host(ctx(), 1, g_parent);
            g_pending = 0;
        }
        if (!rc) rc = nllb_attn_decode_self_host(ctx(), layer, step, 1, &g_q[0][0], &g_k[0][0], &g_v[0][0],
                                                 &g_o[0][0]);
        release();
    }
    memcpy(out, g_o[b], sizeof(g_o[b]));
    pthread_mutex_unlock(&g_mu);
    if (rc) die("decoder self-attention", rc);
}

void nllb_gpu_cross_attention(int layer, int step, int n_src, const float* K, const float* V, const float* q,
                              float* out) {
    pthread_mutex_lock(&g_mu);
    const int b = t_beam;  /* set by this thread's self-attention call of the same layer */
    memcpy(g_q[b], q, sizeof(g_q[b]));
    int rc = 0;
    if (arrive(step)) {
        /* step 0: the memory rows the reference just projected into its shared
         * cache (decoder.c:118-125), [n_src][D_MODEL], head h at columns 64h */
        if (step == 0) rc = nllb_attn_set_memory_host(ctx(), layer, 0, n_src, K, V, HEAD_DIM, D_MODEL);
        if (!rc) rc = nllb_attn_cross_host(ctx(), layer, 1, &g_q[0][0], &g_o[0][0]);
        release();
    }
    memcpy(out, g_o[b], sizeof(g_o[b]));
    pthread_mutex_unlock(&g_mu);
    if (rc) die("decoder cross-attention", rc);
}
