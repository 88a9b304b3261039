// engine_kernels.cu -- the non-attention kernels of the GPU translation engine
// (sm_100a): embedding + positions, LayerNorm, INT8-weight linear layers,
// vocabulary penalties, log-softmax with top-k, and the batched store of the
// cross-attention memory.  Each restates the arithmetic of the reference
// routine named in its comment; fp32 throughout.
#include <cfloat>
#include <cstdint>

#include "device_common.cuh"
#include "engine_kernels.h"
#include "planes.cuh"

namespace nllb {

namespace {

// ---------------------------------------------------------------------------
// embedding * sqrt(d_model) + sinusoidal position
// encoder.c:262-270 / decoder.c:208-223, tensor.c:29-53, encoder.c:27-36
// ---------------------------------------------------------------------------
__global__ void embed_pos_kernel(float* x, const int* tokens, const int* positions, int pos_const,
                                 const int8_t* emb, const float* emb_inv_scale, const float* pos_table,
                                 float embed_scale, int rows, int vocab) {
    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int tok = min(max(tokens[r], 0), vocab - 1);
    const int pos = positions ? positions[r] : pos_const;  // table row = position + 2 offset applied on host
    const float inv = emb_inv_scale[tok];
    const int8_t* w = emb + (size_t)tok * 1024;
    const float* pe = pos_table + (size_t)pos * 1024;
    for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
        const float e = __fmul_rn(__fmul_rn((float)w[i], inv), embed_scale);
        x[(size_t)r * 1024 + i] = __fadd_rn(e, pe[i]);
    }
}

// ---------------------------------------------------------------------------
// LayerNorm over 1024 (layernorm, tensor.c:200-223), optionally adding a residual first:
// x = x + res (residual_add, tensor.c:249-251), out = LN(x).  One CTA per row.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_sum_256(float v, float* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = (l < (int)(blockDim.x >> 5)) ? sh[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

__global__ void __launch_bounds__(256) layernorm_kernel(float* out, float* x, const float* res,
                                                         const float* gamma, const float* beta, int rows,
                                                         plane_t* planes) {
    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    __shared__ float sh[8];
    const int r = blockIdx.x;
    if (r >= rows) return;
    float4* xr = reinterpret_cast<float4*>(x + (size_t)r * 1024);
    float4 v = xr[threadIdx.x];
    if (res) {
        const float4 a = reinterpret_cast<const float4*>(res + (size_t)r * 1024)[threadIdx.x];
        v = make_float4(v.x + a.x, v.y + a.y, v.z + a.z, v.w + a.w);
        xr[threadIdx.x] = v;
    }
    const float mean = block_sum_256(v.x + v.y + v.z + v.w, sh) / 1024.0f;
    const float4 d = make_float4(v.x - mean, v.y - mean, v.z - mean, v.w - mean);
    const float var = block_sum_256(d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w, sh) / 1024.0f;
    const float inv_std = 1.0f / sqrtf(var + 1e-5f);
    const float4 g = gamma ? reinterpret_cast<const float4*>(gamma)[threadIdx.x] : make_float4(1.f, 1.f, 1.f, 1.f);
    const float4 b = beta ? reinterpret_cast<const float4*>(beta)[threadIdx.x] : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 y = make_float4(d.x * inv_std * g.x + b.x, d.y * inv_std * g.y + b.y, d.z * inv_std * g.z + b.z,
                                 d.w * inv_std * g.w + b.w);
    if (out) reinterpret_cast<float4*>(out + (size_t)r * 1024)[threadIdx.x] = y;
    if (planes) store_planes_x4(planes, (size_t)rows * 1024, (size_t)r * 1024 + 4 * threadIdx.x, y);
}

// ---------------------------------------------------------------------------
// INT8-weight linear layer: out[m][n] = (sum_k x[m][k] * w[n][k]) / scale[n]
// + bias[n], then ReLU and/or + residual (mat_vec_int8, tensor.c:70-138 per
// row of x; relu tensor.c:242-245; residual_add tensor.c:249-251).  Output
// column n of row m goes to out + (n / cblock) * (M * cblock) + m * cblock +
// n % cblock: cblock = N is plain row-major, cblock = 1024 stores a fused
// [q|k|v] projection as three stacked [M][1024] matrices.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void linear_store(const LinearArgs& a, int m, int n, float acc) {
    float y = acc * (1.0f / a.scale[n]);
    if (a.bias) y += a.bias[n];
    if (a.relu) y = fmaxf(y, 0.f);
    if (a.mask_from >= 0 && n >= a.mask_from) y = -1e30f;
    const size_t o = (size_t)(n / a.cblock) * ((size_t)a.M * a.cblock) + (size_t)m * a.cblock + (n % a.cblock);
    if (a.residual) y += a.residual[o];
    a.out[o] = y;
}

// Skinny shape (M <= MT rows): a warp owns RPW output rows; lane l reads 4
// consecutive weights of a row at k = 128 j + 4 l (a warp reads 128 B of a
// row per load); the rows' activations for the current 512-wide K chunk sit
// in shared memory and are read once per 4 weights for all RPW rows.
template <int MT, int RPW>
__global__ void __launch_bounds__(256) linear_skinny_kernel(const LinearArgs a) {
    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    constexpr int KC = 512;
    __shared__ __align__(16) float xs[MT][KC];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = (blockIdx.x * 8 + warp) * RPW;
    float acc[RPW][MT];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;
    for (int k0 = 0; k0 < a.K; k0 += KC) {
        const int kc = min(KC, a.K - k0);
        __syncthreads();
        for (int i = threadIdx.x; i < MT * (KC / 4); i += 256) {
            const int m = i / (KC / 4), c4 = i % (KC / 4);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < a.M && c4 * 4 < kc) v = *reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx + k0 + c4 * 4);
            reinterpret_cast<float4*>(xs[m])[c4] = v;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < KC / 128; ++j) {
            const int k = j * 128 + lane * 4;
            if (k >= kc) break;
            char4 w[RPW];
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                const int n = n0 + r;
                w[r] = (n < a.N) ? *reinterpret_cast<const char4*>(a.w + (size_t)n * a.K + k0 + k)
                                 : make_char4(0, 0, 0, 0);
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= a.M) break;
                const float4 xv = reinterpret_cast<const float4*>(xs[m])[k >> 2];
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    acc[r][m] = fmaf((float)w[r].x, xv.x, acc[r][m]);
                    acc[r][m] = fmaf((float)w[r].y, xv.y, acc[r][m]);
                    acc[r][m] = fmaf((float)w[r].z, xv.z, acc[r][m]);
                    acc[r][m] = fmaf((float)w[r].w, xv.w, acc[r][m]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float v = acc[r][m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && m < a.M && n0 + r < a.N) linear_store(a, m, n0 + r, v);
        }
    }
}

// Weight-streaming shape (M <= MT rows, K % 1024 == 0): lane l of every warp
// owns output column n = 32 blockIdx.x + l.  The 8 warps of a CTA take K / 8
// each, in blocks of 128 weights: a lane issues eight independent 16-byte
// loads of its row (the block in flight at once), the next block's loads go
// out before the current block is multiplied with x[m][k..k+127] (the same
// address for every lane: broadcast loads).  The weights, scale and bias are
// constants, so the first block and the column's factors are fetched before
// waiting for the predecessor kernel.  Partial dots are summed through shared
// memory.
template <int MT>
__global__ void __launch_bounds__(256) linear_gemv_kernel(const LinearArgs a) {
    __shared__ float red[8][MT][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 32 + lane;
    const int kw = a.K >> 3, k0 = warp * kw;
    const int nc = min(n, a.N - 1);  // columns past N: repeat a row, not stored
    const int8_t* wrow = a.w + (size_t)nc * a.K;
    if (!a.static_weights) pdl_wait_primary();  // the caller may have written the weights just before
    int4 w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = __ldg(reinterpret_cast<const int4*>(wrow + k0) + i);
    float inv = 0.f, bias = 0.f;
    if (warp == 0) {
        inv = 1.0f / a.scale[nc];  // 1/scale as tensor.c:75
        if (a.bias) bias = a.bias[nc];
    }
    pdl_launch_dependents();
    pdl_wait_primary();  // x comes from the previous kernel
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    for (int kb = k0; kb < k0 + kw; kb += 128) {
        const bool more = kb + 128 < k0 + kw;
        int4 wn[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            wn[i] = more ? __ldg(reinterpret_cast<const int4*>(wrow + kb + 128) + i) : make_int4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int words[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
            float wf[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) wf[q] = (float)(int8_t)(words[q >> 2] >> (8 * (q & 3)));
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= a.M) break;
                const float4* xp = reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx + kb + 16 * i);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float4 xv = __ldg(xp + c);
                    acc[m] = fmaf(wf[4 * c], xv.x, acc[m]);
                    acc[m] = fmaf(wf[4 * c + 1], xv.y, acc[m]);
                    acc[m] = fmaf(wf[4 * c + 2], xv.z, acc[m]);
                    acc[m] = fmaf(wf[4 * c + 3], xv.w, acc[m]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = wn[i];
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) red[warp][m][lane] = acc[m];
    __syncthreads();
    if (warp == 0 && n < a.N) {
        const size_t col = (size_t)(n / a.cblock) * ((size_t)a.M * a.cblock) + (n % a.cblock);
        // the residual may be the output itself: every row's value is loaded
        // before the first store, so the loads overlap
        float res[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) res[m] = (a.residual && m < a.M) ? a.residual[col + (size_t)m * a.cblock] : 0.f;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m >= a.M) break;
            float v = red[0][m][lane];
#pragma unroll
            for (int w8 = 1; w8 < 8; ++w8) v += red[w8][m][lane];
            float y = v * inv;
            if (a.bias) y += bias;
            if (a.relu) y = fmaxf(y, 0.f);
            if (a.mask_from >= 0 && n >= a.mask_from) y = -1e30f;
            if (a.residual) y += res[m];
            a.out[col + (size_t)m * a.cblock] = y;
        }
    }
}

// General shape: 64 x 64 output tile per CTA, 256 threads with 4 x 4
// outputs each, K in steps of 32 through shared memory (x transposed to
// k-major, weights converted to fp32).
__global__ void __launch_bounds__(256) linear_tiled_kernel(const LinearArgs a) {
    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    constexpr int BM = 64, BN = 64, BK = 32;
    __shared__ __align__(16) float xs[BK][BM + 4];
    __shared__ __align__(16) float ws[BK][BN + 4];
    const int tid = threadIdx.x, tm = tid >> 4, tn = tid & 15;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int k0 = 0; k0 < a.K; k0 += BK) {
        __syncthreads();
        // x tile: 64 rows x 32 k = 512 float4, 2 per thread
#pragma unroll
        for (int it = 0; it < 2; ++it) {
            const int i = it * 256 + tid, r = i >> 3, c4 = i & 7;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m0 + r < a.M) v = *reinterpret_cast<const float4*>(a.x + (size_t)(m0 + r) * a.ldx + k0 + c4 * 4);
            xs[c4 * 4 + 0][r] = v.x;
            xs[c4 * 4 + 1][r] = v.y;
            xs[c4 * 4 + 2][r] = v.z;
            xs[c4 * 4 + 3][r] = v.w;
        }
        // weight tile: 64 rows x 32 k int8 = 128 x 16 B
        if (tid < 128) {
            const int r = tid >> 1, h = tid & 1;
            int4 raw = make_int4(0, 0, 0, 0);
            if (n0 + r < a.N) raw = *reinterpret_cast<const int4*>(a.w + (size_t)(n0 + r) * a.K + k0 + h * 16);
            const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
            for (int e = 0; e < 16; ++e) ws[h * 16 + e][r] = (float)b[e];
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < BK; ++k) {
            const float4 xv = *reinterpret_cast<const float4*>(&xs[k][tm * 4]);
            const float4 wv = *reinterpret_cast<const float4*>(&ws[k][tn * 4]);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + tm * 4 + i, n = n0 + tn * 4 + j;
            if (m < a.M && n < a.N) linear_store(a, m, n, acc[i][j]);
        }
}

// ---------------------------------------------------------------------------
// Penalties on one beam's logits (main.c:186-213): repetition penalty over
// tokens[2..n) (skipping EOS 2), compounding for repeated tokens, then the
// no-repeat-bigram ban.  One thread per row: the updates are sequential.
// ---------------------------------------------------------------------------
// One warp per row.  Repetition penalty (main.c:186-194): every occurrence of
// a token at positions 2..n-1 (token 2 skipped) scales its logit once, in
// sequence; the lane holding the first occurrence of a token applies all of
// its occurrences, so the float operations are the reference's.  A positive
// logit is multiplied by the fp32 reciprocal of the penalty: every release
// build of the reference (Makefile:15,19,33) compiles `logits[t] /= penalty`
// under -ffast-math, which turns the division by the constant into that
// multiplication.  Then the no-repeat-bigram ban (main.c:196-213) sets the
// banned logits to -1e30.
// A lane owns positions g0 + lane + 32q (q < 4) of a 128-position group; one
// branch-free pass over the history (the same address for all lanes) finds for
// each whether an earlier position holds its token and how many later ones
// do, then the logits of first occurrences are loaded together and written.
__global__ void penalties_kernel(float* logits, size_t ld, const int* hist, int hist_ld, const int* n_tokens,
                                 const unsigned char* active, int rows, float penalty, int ngram) {
    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows || (active && !active[r])) return;  // uniform per warp
    float* lg = logits + (size_t)r * ld;
    const int* tk = hist + (size_t)r * hist_ld;
    const int n = min(n_tokens[r], hist_ld);  // a history longer than its row is cut to the row
    const float inv_penalty = 1.0f / penalty;
    for (int g0 = 2; g0 < n; g0 += 128) {
        int t[4], cnt[4];    // t = -1: no position, or token 2 (never penalised, never matches)
        unsigned seen = 0;   // bit q: an earlier position holds t[q]
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int g = g0 + 32 * q + lane;
            t[q] = g < n ? __ldg(tk + g) : -1;
            if (t[q] == 2 || (size_t)t[q] >= ld) t[q] = -1;  // token 2, or an id outside the row: skipped
            cnt[q] = t[q] >= 0 ? 1 : 0;
        }
#pragma unroll 4
        for (int j = 2; j < n; ++j) {
            const int u = __ldg(tk + j);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int g = g0 + 32 * q + lane;
                const bool eq = u == t[q];
                seen |= (eq && j < g) ? (1u << q) : 0u;
                cnt[q] += (eq && j > g) ? 1 : 0;
            }
        }
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (t[q] >= 0 && cnt[q] > 0 && !((seen >> q) & 1u)) v[q] = lg[t[q]];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (t[q] >= 0 && cnt[q] > 0 && !((seen >> q) & 1u)) {
                float x = v[q];
                for (int c = 0; c < cnt[q]; ++c) x = (x > 0.f) ? x * inv_penalty : x * penalty;
                lg[t[q]] = x;
            }
    }
    __syncwarp();
    if (ngram == 2 && n >= 2) {
        const int cur = tk[n - 1];
        for (int i = lane; i <= n - 2; i += 32) {
            const int nx = tk[i + 1];
            if (tk[i] == cur && nx != 2 && (size_t)nx < ld) lg[nx] = -1e30f;
        }
    }
}

// ---------------------------------------------------------------------------
// log-softmax over the vocabulary and the K best entries (main.c:154-182):
// each row split into C column chunks (vocab_topk_chunks); one
// streaming pass per chunk keeps an online max and sum of exp and a per-thread
// top-K (greater value first, lower index first among equals, as find_topk's
// strict comparison does); a warp per row then merges the C partials.
// ---------------------------------------------------------------------------
struct Cand {
    float v;
    int i;
};
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
    return va > vb || (va == vb && ia < ib);
}

// (max, sum of exp relative to max) of two parts
__device__ __forceinline__ void lse_combine(float& m, float& s, float mo, float so) {
    const float mn = fmaxf(m, mo);
    s = s * expf(m - mn) + so * expf(mo - mn);
    m = mn;
}

// Warp-wide merge of the lanes' sorted K-lists into the K best (every lane
// gets the result in rv/ri; lanes that hold nothing pass -FLT_MAX lists).
template <int K>
__device__ __forceinline__ void warp_merge_topk(float (&tv)[K], int (&ti)[K], float (&rv)[K], int (&ri)[K]) {
#pragma unroll
    for (int q = 0; q < K; ++q) {
        float bv = tv[0];
        int bi = ti[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
        }
        rv[q] = bv;
        ri[q] = bi;
        if (ti[0] == bi && tv[0] == bv) {  // the owner of the head advances (indices are unique)
#pragma unroll
            for (int j = 0; j < K - 1; ++j) tv[j] = tv[j + 1], ti[j] = ti[j + 1];
            tv[K - 1] = -FLT_MAX;
            ti[K - 1] = 0x7fffffff;
        }
    }
}

// A warp's running top-K, spread over lanes 0..K-1 (lane 0 best), with the
// K-th entry (the admission threshold) in every lane.
template <int K>
struct WarpTopK {
    float v = -FLT_MAX, tv = -FLT_MAX;  // own entry, threshold value
    int i = 0x7fffffff, ti = 0x7fffffff;

    // Insert a warp-uniform candidate that beats the threshold.
    __device__ __forceinline__ void insert(float cv, int ci, int lane) {
        const bool ahead = lane < K && better(v, i, cv, ci);
        const int pos = __popc(__ballot_sync(0xffffffffu, ahead));  // entries ahead form a prefix
        const float uv = __shfl_up_sync(0xffffffffu, v, 1);
        const int ui = __shfl_up_sync(0xffffffffu, i, 1);
        if (lane > pos && lane < K) v = uv, i = ui;
        if (lane == pos) v = cv, i = ci;
        tv = __shfl_sync(0xffffffffu, v, K - 1);
        ti = __shfl_sync(0xffffffffu, i, K - 1);
    }
    // Offer each lane's (x, ix) (valid lanes only); warp-uniform call.
    __device__ __forceinline__ void offer(float x, int ix, bool valid, int lane) {
        unsigned mask = __ballot_sync(0xffffffffu, valid && better(x, ix, tv, ti));
        while (mask) {
            const int src = __ffs(mask) - 1;
            mask &= mask - 1;
            const float cv = __shfl_sync(0xffffffffu, x, src);
            const int ci = __shfl_sync(0xffffffffu, ix, src);
            if (better(cv, ci, tv, ti)) insert(cv, ci, lane);
        }
    }
};

// Online (max, sum of exp relative to max) with e^d computed as 2^(d log2 e).
__device__ __forceinline__ void lse_add4(float& m, float& s, float4 v, float m4) {
    if (m4 > m) {  // rare after the first elements; m = -FLT_MAX at the start
        s *= exp2f((m - m4) * kLog2e);
        m = m4;
    }
    s += exp2f((v.x - m) * kLog2e) + exp2f((v.y - m) * kLog2e) + exp2f((v.z - m) * kLog2e) +
         exp2f((v.w - m) * kLog2e);
}

// Partial over columns [c*chunk, (c+1)*chunk) of row r (grid: chunks x rows):
// online max and sum of exp per thread, a top-K per warp (one ballot per
// float4 against the warp's threshold; insertions are rare after the first
// few elements), then a block merge.  Written to ws[r][c] = {m, s, v[K], i[K]}.
template <int K>
__global__ void __launch_bounds__(256) vocab_partial_kernel(const float* logits, size_t ld, int V, int chunk,
                                                            const unsigned char* active, float* ws) {
    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    __shared__ float sh_m[8], sh_s[8], sh_v[8 * K];
    __shared__ int sh_i[8 * K];
    const int r = blockIdx.y, c = blockIdx.x, C = gridDim.x;
    if (active && !active[r]) return;  // uniform per CTA
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* lg = logits + (size_t)r * ld;
    const int lo = c * chunk, hi = min(V, lo + chunk);
    float m = -FLT_MAX, s = 0.f;
    WarpTopK<K> top;
    // scalar head up to a 16-byte boundary and scalar tail: warp 0, one element per lane
    const int head = min(hi - lo, (int)(((16u - (uint32_t)(reinterpret_cast<uintptr_t>(lg + lo) & 15u)) & 15u) >> 2));
    const int b0 = lo + head, nb4 = (hi - b0) >> 2, t0 = b0 + 4 * nb4;
    if (warp == 0) {
        for (int e = 0; e < 2; ++e) {
            const int idx = e == 0 ? lo + lane : t0 + lane;
            const bool valid = e == 0 ? lane < head : idx < hi;
            const float x = valid ? lg[idx] : -INFINITY;
            lse_add4(m, s, make_float4(x, -INFINITY, -INFINITY, -INFINITY), x);
            top.offer(x, idx, valid, lane);
        }
    }
    // float4 body in batches of kBatch float4 per thread (element j0 + 256 u +
    // thread, u < kBatch), the next batch in flight while this one is used:
    // 2 kBatch loads of 16 B outstanding per thread keep enough bytes in
    // flight to stream at HBM speed.  The loop bound is uniform per CTA.
    constexpr int kBatch = 4;
    const float4* body = reinterpret_cast<const float4*>(lg + b0);
    const float4 none = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    const int jt = warp * 32 + lane;
    float4 cur[kBatch], nxt[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) cur[u] = jt + 256 * u < nb4 ? __ldcs(body + jt + 256 * u) : none;
    for (int j0 = 0; j0 < nb4; j0 += 256 * kBatch) {
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int jn = j0 + 256 * (kBatch + u) + jt;
            nxt[u] = jn < nb4 ? __ldcs(body + jn) : none;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int j = j0 + 256 * u + jt;
            const bool valid = j < nb4;
            const float4 v = cur[u];
            const float m4 = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
            lse_add4(m, s, v, m4);
            const int i0 = b0 + 4 * j;
            unsigned mask = __ballot_sync(0xffffffffu, valid && m4 >= top.tv);
            while (mask) {
                const int src = __ffs(mask) - 1;
                mask &= mask - 1;
                const float c0 = __shfl_sync(0xffffffffu, v.x, src), c1 = __shfl_sync(0xffffffffu, v.y, src);
                const float c2 = __shfl_sync(0xffffffffu, v.z, src), c3 = __shfl_sync(0xffffffffu, v.w, src);
                const int ci = __shfl_sync(0xffffffffu, i0, src);
                if (better(c0, ci, top.tv, top.ti)) top.insert(c0, ci, lane);
                if (better(c1, ci + 1, top.tv, top.ti)) top.insert(c1, ci + 1, lane);
                if (better(c2, ci + 2, top.tv, top.ti)) top.insert(c2, ci + 2, lane);
                if (better(c3, ci + 3, top.tv, top.ti)) top.insert(c3, ci + 3, lane);
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) cur[u] = nxt[u];
    }
    // warp, then block
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, o), so = __shfl_xor_sync(0xffffffffu, s, o);
        lse_combine(m, s, mo, so);
    }
    if (lane == 0) sh_m[warp] = m, sh_s[warp] = s;
    if (lane < K) sh_v[warp * K + lane] = top.v, sh_i[warp * K + lane] = top.i;
    __syncthreads();
    if (warp == 0) {
        m = lane < 8 ? sh_m[lane] : -FLT_MAX;
        s = lane < 8 ? sh_s[lane] : 0.f;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
            const float mo = __shfl_xor_sync(0xffffffffu, m, o), so = __shfl_xor_sync(0xffffffffu, s, o);
            lse_combine(m, s, mo, so);
        }
        float tv[K], rv[K];
        int ti[K], ri[K];
#pragma unroll
        for (int q = 0; q < K; ++q) {
            tv[q] = lane < 8 ? sh_v[lane * K + q] : -FLT_MAX;
            ti[q] = lane < 8 ? sh_i[lane * K + q] : 0x7fffffff;
        }
        warp_merge_topk<K>(tv, ti, rv, ri);
        float* out = ws + ((size_t)r * C + c) * (2 + 2 * K);
        if (lane == 0) out[0] = m, out[1] = s;
#pragma unroll
        for (int q = 0; q < K; ++q)
            if (lane == q) out[2 + q] = rv[q], out[2 + K + q] = __int_as_float(ri[q]);
    }
}

// One warp per row: combine the C partials, write the K best as
// (token, log-probability = logit - (max + log(sum of exp))).
template <int K>
__global__ void __launch_bounds__(256) vocab_merge_kernel(const float* ws, int C, int rows,
                                                          const unsigned char* active, int* out_tok,
                                                          float* out_logp) {
    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows || (active && !active[r])) return;  // uniform per warp
    const float* p = ws + (size_t)r * C * (2 + 2 * K);
    float m = -FLT_MAX, s = 0.f;
    float tv[K];
    int ti[K];
#pragma unroll
    for (int q = 0; q < K; ++q) tv[q] = -FLT_MAX, ti[q] = 0x7fffffff;
    if (lane < C) {
        const float* e = p + (size_t)lane * (2 + 2 * K);
        m = e[0];
        s = e[1];
#pragma unroll
        for (int q = 0; q < K; ++q) tv[q] = e[2 + q], ti[q] = __float_as_int(e[2 + K + q]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, o), so = __shfl_xor_sync(0xffffffffu, s, o);
        lse_combine(m, s, mo, so);
    }
    float rv[K];
    int ri[K];
    warp_merge_topk<K>(tv, ti, rv, ri);
    const float ln = m + logf(s);
#pragma unroll
    for (int q = 0; q < K; ++q)
        if (lane == q) {
            out_tok[(size_t)r * K + q] = ri[q];
            out_logp[(size_t)r * K + q] = rv[q] - ln;
        }
}

// ---------------------------------------------------------------------------
// cross-attention memory of many sentences for one layer: rows of sentence s
// at kv + s * row_stride_sent (K) and + v_off (V), [n][1024] head-interleaved,
// into the context's head-major [sentence][head][max_src][64]
// ---------------------------------------------------------------------------
__global__ void set_memory_batched_kernel(float* km, float* vm, int* n_src_slots, int max_src, int H,
                                          const float* k, const float* v, long long sent_stride,
                                          const int* row_start, const int* n_src, int n_sent) {
    // No early pdl_launch_dependents: the cross-attention kernel reads the
    // memory before its own wait on the previous kernel, which is safe only
    // because no kernel after this one starts before it completes.
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    const int s = blockIdx.y;
    const int n = n_src[s];
    if (blockIdx.x == 0 && threadIdx.x == 0) n_src_slots[s] = n;
    const size_t total = (size_t)H * n * 16;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int q4 = (int)(i & 15);
        const size_t hr = i >> 4;
        const int r = (int)(hr % n), h = (int)(hr / n);
        const size_t s0 = row_start ? (size_t)row_start[s] * (H * 64) : (size_t)s * sent_stride;
        const size_t src = s0 + (size_t)r * (H * 64) + (size_t)h * 64;
        const size_t dst = (((size_t)s * H + h) * max_src + r) * 64;
        reinterpret_cast<float4*>(km + dst)[q4] = reinterpret_cast<const float4*>(k + src)[q4];
        reinterpret_cast<float4*>(vm + dst)[q4] = reinterpret_cast<const float4*>(v + src)[q4];
    }
}

__global__ void reciprocal_kernel(float* out, const float* in, size_t n) {
    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels; outputs may still be read by them
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = 1.0f / in[i];
}

}  // namespace

cudaError_t launch_embed_pos(float* x, const int* tokens, const int* positions, int pos_const, const int8_t* emb,
                             const float* emb_inv_scale, const float* pos_table, float embed_scale, int rows,
                             int vocab, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    return launch_pdl(embed_pos_kernel, dim3(rows), dim3(256), 0, st, x, tokens, positions, pos_const, emb,
                      emb_inv_scale, pos_table, embed_scale, rows, vocab);
}

cudaError_t launch_layernorm(float* out, float* x, const float* res, const float* gamma, const float* beta,
                             int rows, void* planes, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    return launch_pdl(layernorm_kernel, dim3(rows), dim3(256), 0, st, out, x, res, gamma, beta, rows,
                      static_cast<plane_t*>(planes));
}

cudaError_t launch_linear(const LinearArgs& a, const LinearWorkspace* wsp, int num_sms, int* err, cudaStream_t st) {
    if (a.M <= 0) return cudaSuccess;
    if ((a.K & 3) || (a.ldx & 3)) return cudaErrorInvalidValue;
    const bool gemv = (a.K % 1024 == 0) && (a.ldx % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.w) & 15) == 0) &&
                      ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
    if (gemv && a.M <= 4) {
        return launch_pdl(linear_gemv_kernel<4>, dim3((a.N + 31) / 32), dim3(256), 0, st, a);
    } else if (gemv && a.M <= 16) {
        return launch_pdl(linear_gemv_kernel<16>, dim3((a.N + 31) / 32), dim3(256), 0, st, a);
    } else if (a.M <= 4) {
        return launch_pdl(linear_skinny_kernel<4, 2>, dim3((a.N + 15) / 16), dim3(256), 0, st, a);
    } else if (a.M <= 16) {
        return launch_pdl(linear_skinny_kernel<16, 2>, dim3((a.N + 15) / 16), dim3(256), 0, st, a);
    } else if (linear_tc_supports(a)) {
        int splits = linear_tc_splits(a, num_sms);
        if (!wsp || linear_tc_workspace_floats(a, splits) > wsp->ws_floats || linear_tc_tiles(a) > wsp->n_counters)
            splits = 1;
        return launch_linear_tc(a, splits, wsp ? wsp->ws : nullptr, wsp ? wsp->tile_count : nullptr, err, st);
    } else {
        if (a.K % 32) return cudaErrorInvalidValue;
        dim3 grid((a.N + 63) / 64, (a.M + 63) / 64);
        return launch_pdl(linear_tiled_kernel, grid, dim3(256), 0, st, a);
    }
    return cudaGetLastError();
}

cudaError_t launch_penalties(float* logits, size_t ld, const int* hist, int hist_ld, const int* n_tokens,
                             const unsigned char* active, int rows, float penalty, int ngram, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    return launch_pdl(penalties_kernel, dim3((rows + 3) / 4), dim3(128), 0, st, logits, ld, hist, hist_ld,
                      n_tokens, active, rows, penalty, ngram);
}

// Chunks for about 2 CTAs per SM in all, i.e. one CTA per row from 296 rows
// up.  Measured on B200 (256206 logits per row, vocab_partial + merge): 512
// rows 121 us with 2, 133 with 4, 154 with 8, 196 with 16; 4096 rows 740 us
// for all of them (one chunk per row).
#ifndef NLLB_TOPK_CTAS_PER_SM
#define NLLB_TOPK_CTAS_PER_SM 2
#endif
int vocab_topk_chunks(int V, int rows) {
    int C = (148 * NLLB_TOPK_CTAS_PER_SM + rows - 1) / rows;
    C = C < 1 ? 1 : (C > 32 ? 32 : C);
    while (C > 1 && V / C < 4096) --C;
    return C;
}

size_t vocab_topk_ws_floats(int V, int rows, int k) {
    return (size_t)rows * vocab_topk_chunks(V, rows) * (2 + 2 * (size_t)k);
}

cudaError_t launch_logsoftmax_topk(const float* logits, size_t ld, int V, int rows, const unsigned char* active,
                                   int k, int* out_tok, float* out_logp, float* ws, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    const int C = vocab_topk_chunks(V, rows);
    const int chunk = (((V + C - 1) / C) + 3) & ~3;
    const dim3 g1(C, rows), g2((rows + 7) / 8);
    if (k == 8) {
        cudaError_t e = launch_pdl(vocab_partial_kernel<8>, g1, dim3(256), 0, st, logits, ld, V, chunk, active, ws);
        if (e != cudaSuccess) return e;
        return launch_pdl(vocab_merge_kernel<8>, g2, dim3(256), 0, st, ws, C, rows, active, out_tok, out_logp);
    } else if (k == 4) {
        cudaError_t e = launch_pdl(vocab_partial_kernel<4>, g1, dim3(256), 0, st, logits, ld, V, chunk, active, ws);
        if (e != cudaSuccess) return e;
        return launch_pdl(vocab_merge_kernel<4>, g2, dim3(256), 0, st, ws, C, rows, active, out_tok, out_logp);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_set_memory_batched(float* km, float* vm, int* n_src_slots, int max_src, int H, const float* k,
                                      const float* v, long long sent_stride, const int* row_start,
                                      const int* n_src, int n_sent, int max_n, cudaStream_t st) {
    if (n_sent <= 0) return cudaSuccess;
    const int bx = (int)(((size_t)H * max_n * 16 + 255) / 256);
    return launch_pdl(set_memory_batched_kernel, dim3(bx < 64 ? bx : 64, n_sent), dim3(256), 0, st, km, vm,
                      n_src_slots, max_src, H, k, v, sent_stride, row_start, n_src, n_sent);
}

cudaError_t launch_reciprocal(float* out, const float* in, size_t n, cudaStream_t st) {
    reciprocal_kernel<<<256, 256, 0, st>>>(out, in, n);
    return cudaGetLastError();
}

}  // namespace nllb
