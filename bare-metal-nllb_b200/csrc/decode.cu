// decode.cu -- decoder self-attention over the per-beam KV cache and
// cross-attention over the shared encoder memory (sm_100a).
//
// Both kernels are HBM-bound streams: every (sentence, head) reads its K/V
// rows once per call and does 2 FMA per fp32 loaded per beam.  Design:
//   * grid (split, head, sentence), 128 threads = 8 half-warps;
//   * K/V arrive in 64-row chunks (16 KB each for K and V) by cp.async.bulk
//     into a 3-stage shared-memory ring completing on mbarriers, so 2 chunks
//     (64 KB) are in flight per CTA while the third is consumed;
//   * a half-warp owns 64-float rows: 16 lanes x float4, dot product by four
//     xor-shuffles; online softmax in base 2 per half-warp;
//   * split-KV when (sentences x heads) cannot fill the 148 SMs: each split
//     writes (max, sum, acc) to a workspace and the last CTA of a
//     (sentence, head) to finish - found with one atomic, no waiting - merges
//     them (flash-decoding combine).
//
// Self-attention cache row (p, slot) of a (sentence, head) is at
// ((p * n_beams) + slot) * 64: all beams' rows of one position are adjacent,
// so a chunk of positions is one contiguous block whatever the beam history.
// hist[s][p][b] names the slot that holds position p of logical beam b; a
// beam reorder permutes these bytes (reorder_kernel) instead of copying
// caches (the reference copies each parent cache, main.c:481-482).
#include "device_common.cuh"
#include "kernels.h"

namespace nllb {

namespace {

constexpr int kThreads = 128;
constexpr int kStages = 3;

// ---------------------------------------------------------------------------
// Split record helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_part(float* rec, int q4, float m, float l, float4 acc) {
    if (q4 == 0) {
        rec[0] = m;
        rec[1] = l;
    }
    reinterpret_cast<float4*>(rec + 4)[q4] = acc;
}

// Merge the n_split records of one (sentence, head, beam) and write out.
__device__ __forceinline__ void merge_parts(const float* part0, int n_split, int rec_stride,
                                            int q4, float* dst) {
    float M = -INFINITY;
    for (int i = 0; i < n_split; ++i) M = fmaxf(M, __ldcg(part0 + (size_t)i * rec_stride));
    float L = 0.f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < n_split; ++i) {
        const float* rec = part0 + (size_t)i * rec_stride;
        const float w = safe_exp2_diff(__ldcg(rec), M);
        L = fmaf(w, __ldcg(rec + 1), L);
        A = f4_fma(w, __ldcg(reinterpret_cast<const float4*>(rec + 4) + q4), A);
    }
    reinterpret_cast<float4*>(dst)[q4] = f4_scale(A, 1.0f / L);
}

// ---------------------------------------------------------------------------
// Decoder self-attention
// ---------------------------------------------------------------------------
template <int NB>
__global__ void __launch_bounds__(kThreads) decode_self_kernel(const SelfParams p) {
    constexpr int CP = 64 / NB;       // positions per chunk
    constexpr int NSUB = 8 / NB;      // half-warps per beam
    constexpr int RPH = CP / NSUB;    // positions per half-warp per chunk (= 8)
    constexpr int KV_FLOATS = CP * NB * 64;
    constexpr int H_BYTES = CP * 8;

    extern __shared__ __align__(128) unsigned char smem[];
    float* sK = reinterpret_cast<float*>(smem);
    float* sV = sK + kStages * KV_FLOATS;
    unsigned char* sH = reinterpret_cast<unsigned char*>(sV + kStages * KV_FLOATS);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sH + kStages * H_BYTES);
    __shared__ int s_abort;
    __shared__ int s_last;

    const int split = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x, hw = tid >> 4, l16 = tid & 15;
    const int b = hw % NB, sub = hw / NB;

    const int len = p.step;
    const int p0 = split * p.pos_per_split;
    const int p1 = min(len, p0 + p.pos_per_split);
    const int nchunk = (p1 > p0) ? (p1 - p0 + CP - 1) / CP : 0;
    const bool owns_new = (split == p.n_split - 1);

    const size_t head_pos0 = ((size_t)s * p.H + h) * (size_t)p.T;
    const float* gK = p.kc + head_pos0 * NB * 64;
    const float* gV = p.vc + head_pos0 * NB * 64;
    const unsigned char* gH = p.hist + (size_t)s * p.Tp * 8;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&bar[i], 1);
        fence_barrier_init();
        s_abort = 0;
    }
    __syncthreads();

    auto issue = [&](int c) {
        const int st = c % kStages;
        const int pc0 = p0 + c * CP;
        const int np = min(CP, p1 - pc0);
        const uint32_t kvb = (uint32_t)np * NB * 256u;
        const uint32_t hb = (uint32_t)((np * 8 + 15) & ~15);
        mbar_arrive_expect_tx(&bar[st], 2u * kvb + hb);
        bulk_g2s(sK + st * KV_FLOATS, gK + (size_t)pc0 * NB * 64, kvb, &bar[st]);
        bulk_g2s(sV + st * KV_FLOATS, gV + (size_t)pc0 * NB * 64, kvb, &bar[st]);
        bulk_g2s(sH + st * H_BYTES, gH + (size_t)pc0 * 8, hb, &bar[st]);
    };
    if (tid == 0) {
        for (int c = 0; c < kStages - 1 && c < nchunk; ++c) issue(c);
    }

    const size_t qrow = ((size_t)s * NB + b) * (size_t)p.H * 64 + (size_t)h * 64;
    const float4 qv = __ldg(reinterpret_cast<const float4*>(p.q + qrow) + l16);

    float m = -INFINITY, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int consumed = 0;

    for (int c = 0; c < nchunk; ++c) {
        const int st = c % kStages;
        const uint32_t par = (uint32_t)((c / kStages) & 1);
        if (!mbar_wait_bounded(&bar[st], par)) s_abort = 1;
        __syncthreads();  // stage (c-1) fully consumed; abort flag visible
        if (s_abort) break;
        consumed = c + 1;
        if (tid == 0 && c + kStages - 1 < nchunk) issue(c + kStages - 1);

        const int np = min(CP, p1 - (p0 + c * CP));
        const float* K = sK + st * KV_FLOATS;
        const float* V = sV + st * KV_FLOATS;
        const unsigned char* Hs = sH + st * H_BYTES;

        float sc[RPH];
        int slot[RPH];
#pragma unroll
        for (int i = 0; i < RPH; ++i) {
            const int pl = sub + i * NSUB;
            const bool ok = pl < np;
            slot[i] = ok ? Hs[pl * 8 + b] : 0;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok) kv = reinterpret_cast<const float4*>(K + (pl * NB + slot[i]) * 64)[l16];
            const float d = halfwarp_sum(f4_dot(qv, kv));
            sc[i] = ok ? d * p.scale_log2 : -INFINITY;
        }
        float mc = sc[0];
#pragma unroll
        for (int i = 1; i < RPH; ++i) mc = fmaxf(mc, sc[i]);
        const float mn = fmaxf(m, mc);
        if (mn != -INFINITY) {
            const float corr = safe_exp2_diff(m, mn);
            l *= corr;
            acc = f4_scale(acc, corr);
#pragma unroll
            for (int i = 0; i < RPH; ++i) {
                const int pl = sub + i * NSUB;
                if (pl < np) {
                    const float e = exp2f(sc[i] - mn);
                    l += e;
                    const float4 vv = reinterpret_cast<const float4*>(V + (pl * NB + slot[i]) * 64)[l16];
                    acc = f4_fma(e, vv, acc);
                }
            }
            m = mn;
        }
    }

    if (s_abort) {
        // drain copies still in flight into this CTA's shared memory, then leave
        if (tid == 0) {
            atomicOr(p.err, NLLB_DEV_ERR_TIMEOUT);
            const int issued = min(nchunk, consumed + kStages - 1);
            for (int c = consumed; c < issued; ++c)
                (void)mbar_wait_bounded(&bar[c % kStages], (uint32_t)((c / kStages) & 1));
        }
        return;
    }

    // The new token at position `step`: every beam attends to its own k_new.
    if (owns_new) {
        const float4 kn = __ldg(reinterpret_cast<const float4*>(p.k_new + qrow) + l16);
        const float4 vn = __ldg(reinterpret_cast<const float4*>(p.v_new + qrow) + l16);
        const float d = halfwarp_sum(f4_dot(qv, kn)) * p.scale_log2;
        if (sub == 0) {
            const float mn = fmaxf(m, d);
            const float corr = safe_exp2_diff(m, mn);
            const float e = exp2f(d - mn);
            l = fmaf(l, corr, e);
            acc = f4_fma(e, vn, f4_scale(acc, corr));
            m = mn;
            // append to the cache: position `step`, physical slot b
            const size_t row = (head_pos0 + (size_t)p.step) * NB + b;
            reinterpret_cast<float4*>(p.kc_w + row * 64)[l16] = kn;
            reinterpret_cast<float4*>(p.vc_w + row * 64)[l16] = vn;
            if (h == 0 && l16 == 0) p.hist_w[((size_t)s * p.Tp + p.step) * 8 + b] = (unsigned char)b;
        }
    }

    // Merge the NSUB half-warp states of each beam (stage buffers are free now).
    __syncthreads();
    float* red = sK;  // [8 hw][68]
    {
        float* rec = red + hw * kPartFloats;
        if (l16 == 0) {
            rec[0] = m;
            rec[1] = l;
        }
        reinterpret_cast<float4*>(rec + 4)[l16] = acc;
    }
    __syncthreads();

    const size_t unit = (size_t)s * p.H + h;
    for (int idx = tid; idx < NB * 16; idx += kThreads) {
        const int bb = idx >> 4, q4 = idx & 15;
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < NSUB; ++j) M = fmaxf(M, red[(bb + NB * j) * kPartFloats]);
        float L = 0.f;
        float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < NSUB; ++j) {
            const float* rec = red + (bb + NB * j) * kPartFloats;
            const float w = safe_exp2_diff(rec[0], M);
            L = fmaf(w, rec[1], L);
            A = f4_fma(w, reinterpret_cast<const float4*>(rec + 4)[q4], A);
        }
        if (p.n_split == 1) {
            float* dst = p.out + ((size_t)s * NB + bb) * (size_t)p.H * 64 + (size_t)h * 64;
            reinterpret_cast<float4*>(dst)[q4] = f4_scale(A, 1.0f / L);
        } else {
            float* rec = p.part + ((unit * p.n_split + split) * NB + bb) * kPartFloats;
            store_part(rec, q4, M, L, A);
        }
    }
    if (p.n_split == 1) return;

    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&p.counters[unit], 1) == p.n_split - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int idx = tid; idx < NB * 16; idx += kThreads) {
        const int bb = idx >> 4, q4 = idx & 15;
        const float* part0 = p.part + (unit * p.n_split * NB + bb) * kPartFloats;
        float* dst = p.out + ((size_t)s * NB + bb) * (size_t)p.H * 64 + (size_t)h * 64;
        merge_parts(part0, p.n_split, NB * kPartFloats, q4, dst);
    }
    if (tid == 0) p.counters[unit] = 0;
}

// ---------------------------------------------------------------------------
// Cross-attention: all beams of a sentence share each memory row.
// ---------------------------------------------------------------------------
template <int NB>
__global__ void __launch_bounds__(kThreads) cross_kernel(const CrossParams p) {
    constexpr int CP = kCrossChunkRows;
    constexpr int RPH = CP / 8;  // rows per half-warp per chunk
    constexpr int KV_FLOATS = CP * 64;

    extern __shared__ __align__(128) unsigned char smem[];
    float* sK = reinterpret_cast<float*>(smem);
    float* sV = sK + kStages * KV_FLOATS;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sV + kStages * KV_FLOATS);
    __shared__ int s_abort;
    __shared__ int s_last;

    const int split = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x, hw = tid >> 4, l16 = tid & 15;

    const int len = __ldg(p.n_src + s);
    const int p0 = split * p.pos_per_split;
    const int p1 = min(len, p0 + p.pos_per_split);
    const int nchunk = (p1 > p0) ? (p1 - p0 + CP - 1) / CP : 0;

    const size_t head_row0 = ((size_t)s * p.H + h) * (size_t)p.max_src;
    const float* gK = p.km + head_row0 * 64;
    const float* gV = p.vm + head_row0 * 64;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&bar[i], 1);
        fence_barrier_init();
        s_abort = 0;
    }
    __syncthreads();

    auto issue = [&](int c) {
        const int st = c % kStages;
        const int pc0 = p0 + c * CP;
        const int np = min(CP, p1 - pc0);
        const uint32_t kvb = (uint32_t)np * 256u;
        mbar_arrive_expect_tx(&bar[st], 2u * kvb);
        bulk_g2s(sK + st * KV_FLOATS, gK + (size_t)pc0 * 64, kvb, &bar[st]);
        bulk_g2s(sV + st * KV_FLOATS, gV + (size_t)pc0 * 64, kvb, &bar[st]);
    };
    if (tid == 0) {
        for (int c = 0; c < kStages - 1 && c < nchunk; ++c) issue(c);
    }

    float4 qv[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const size_t qrow = ((size_t)s * NB + b) * (size_t)p.H * 64 + (size_t)h * 64;
        qv[b] = __ldg(reinterpret_cast<const float4*>(p.q + qrow) + l16);
    }
    float m[NB], l[NB];
    float4 acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        m[b] = -INFINITY;
        l[b] = 0.f;
        acc[b] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    int consumed = 0;

    for (int c = 0; c < nchunk; ++c) {
        const int st = c % kStages;
        const uint32_t par = (uint32_t)((c / kStages) & 1);
        if (!mbar_wait_bounded(&bar[st], par)) s_abort = 1;
        __syncthreads();
        if (s_abort) break;
        consumed = c + 1;
        if (tid == 0 && c + kStages - 1 < nchunk) issue(c + kStages - 1);

        const int np = min(CP, p1 - (p0 + c * CP));
        const float* K = sK + st * KV_FLOATS;
        const float* V = sV + st * KV_FLOATS;

        float sc[NB][RPH];
#pragma unroll
        for (int i = 0; i < RPH; ++i) {
            const int r = hw + 8 * i;
            const bool ok = r < np;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok) kv = reinterpret_cast<const float4*>(K + r * 64)[l16];
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const float d = halfwarp_sum(f4_dot(qv[b], kv));
                sc[b][i] = ok ? d * p.scale_log2 : -INFINITY;
            }
        }
        float mn[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            float mc = sc[b][0];
#pragma unroll
            for (int i = 1; i < RPH; ++i) mc = fmaxf(mc, sc[b][i]);
            mn[b] = fmaxf(m[b], mc);
            const float corr = safe_exp2_diff(m[b], mn[b]);
            l[b] *= corr;
            acc[b] = f4_scale(acc[b], corr);
            m[b] = mn[b];
        }
#pragma unroll
        for (int i = 0; i < RPH; ++i) {
            const int r = hw + 8 * i;
            if (r < np) {
                const float4 vv = reinterpret_cast<const float4*>(V + r * 64)[l16];
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const float e = exp2f(sc[b][i] - mn[b]);
                    l[b] += e;
                    acc[b] = f4_fma(e, vv, acc[b]);
                }
            }
        }
    }

    if (s_abort) {
        if (tid == 0) {
            atomicOr(p.err, NLLB_DEV_ERR_TIMEOUT);
            const int issued = min(nchunk, consumed + kStages - 1);
            for (int c = consumed; c < issued; ++c)
                (void)mbar_wait_bounded(&bar[c % kStages], (uint32_t)((c / kStages) & 1));
        }
        return;
    }

    __syncthreads();
    float* red = sK;  // [8 hw][NB][68]
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float* rec = red + (hw * NB + b) * kPartFloats;
        if (l16 == 0) {
            rec[0] = m[b];
            rec[1] = l[b];
        }
        reinterpret_cast<float4*>(rec + 4)[l16] = acc[b];
    }
    __syncthreads();

    const size_t unit = (size_t)s * p.H + h;
    for (int idx = tid; idx < NB * 16; idx += kThreads) {
        const int bb = idx >> 4, q4 = idx & 15;
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) M = fmaxf(M, red[(j * NB + bb) * kPartFloats]);
        float L = 0.f;
        float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float* rec = red + (j * NB + bb) * kPartFloats;
            const float w = safe_exp2_diff(rec[0], M);
            L = fmaf(w, rec[1], L);
            A = f4_fma(w, reinterpret_cast<const float4*>(rec + 4)[q4], A);
        }
        if (p.n_split == 1) {
            float* dst = p.out + ((size_t)s * NB + bb) * (size_t)p.H * 64 + (size_t)h * 64;
            reinterpret_cast<float4*>(dst)[q4] = f4_scale(A, 1.0f / L);
        } else {
            float* rec = p.part + ((unit * p.n_split + split) * NB + bb) * kPartFloats;
            store_part(rec, q4, M, L, A);
        }
    }
    if (p.n_split == 1) return;

    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&p.counters[unit], 1) == p.n_split - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int idx = tid; idx < NB * 16; idx += kThreads) {
        const int bb = idx >> 4, q4 = idx & 15;
        const float* part0 = p.part + (unit * p.n_split * NB + bb) * kPartFloats;
        float* dst = p.out + ((size_t)s * NB + bb) * (size_t)p.H * 64 + (size_t)h * 64;
        merge_parts(part0, p.n_split, NB * kPartFloats, q4, dst);
    }
    if (tid == 0) p.counters[unit] = 0;
}

// ---------------------------------------------------------------------------
// Beam history maintenance
// ---------------------------------------------------------------------------
// new slot of (p, b) = old slot of (p, parent[b]), in place, one CTA per sentence.
__global__ void reorder_kernel(unsigned char* hist, int Tp, const int* parent, int n_beams,
                               int* err) {
    const int s = blockIdx.x;
    __shared__ int par[8];
    __shared__ int bad;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    if (threadIdx.x < n_beams) {
        int v = parent[s * n_beams + threadIdx.x];
        if (v < 0 || v >= n_beams) {
            bad = 1;
            v = threadIdx.x;
        }
        par[threadIdx.x] = v;
    }
    __syncthreads();
    if (bad) {
        if (threadIdx.x == 0) atomicOr(err, NLLB_DEV_ERR_BAD_PARENT);
        return;
    }
    uint2* rows = reinterpret_cast<uint2*>(hist + (size_t)s * Tp * 8);
    for (int pos = threadIdx.x; pos < Tp; pos += blockDim.x) {
        uint2 v = rows[pos];
        unsigned char old[8], nw[8];
        memcpy(old, &v, 8);
#pragma unroll
        for (int b = 0; b < 8; ++b) nw[b] = (b < n_beams) ? old[par[b]] : old[b];
        memcpy(&v, nw, 8);
        rows[pos] = v;
    }
}

__global__ void hist_init_kernel(unsigned char* hist, size_t n_rows) {
    const uint2 ident = make_uint2(0x03020100u, 0x07060504u);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_rows;
         i += (size_t)gridDim.x * blockDim.x)
        reinterpret_cast<uint2*>(hist)[i] = ident;
}

// k[r*stride_row + h*stride_head + d] -> km[h][r][d] (one layer, one sentence)
__global__ void set_memory_kernel(float* km, float* vm, int max_src, int H, const float* k,
                                  const float* v, long long stride_head, long long stride_row,
                                  int n_src) {
    const size_t total = (size_t)H * n_src * 16;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int q4 = (int)(i & 15);
        const size_t hr = i >> 4;
        const int r = (int)(hr % n_src);
        const int h = (int)(hr / n_src);
        const size_t src = (size_t)r * stride_row + (size_t)h * stride_head;
        const size_t dst = ((size_t)h * max_src + r) * 64;
        reinterpret_cast<float4*>(km + dst)[q4] = __ldg(reinterpret_cast<const float4*>(k + src) + q4);
        reinterpret_cast<float4*>(vm + dst)[q4] = __ldg(reinterpret_cast<const float4*>(v + src) + q4);
    }
}

template <int NB>
size_t self_smem_bytes() {
    constexpr int CP = 64 / NB;
    return (size_t)kStages * (2 * CP * NB * 64 * sizeof(float) + CP * 8) + kStages * sizeof(uint64_t);
}

size_t cross_smem_bytes() {
    return (size_t)kStages * 2 * kCrossChunkRows * 64 * sizeof(float) + kStages * sizeof(uint64_t);
}

template <int NB>
cudaError_t configure_nb() {
    cudaError_t e = cudaFuncSetAttribute(decode_self_kernel<NB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)self_smem_bytes<NB>());
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(cross_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)cross_smem_bytes());
}

template <int NB>
cudaError_t launch_self_nb(const SelfParams& p, int n_sent, cudaStream_t st) {
    dim3 grid(p.n_split, p.H, n_sent);
    decode_self_kernel<NB><<<grid, kThreads, self_smem_bytes<NB>(), st>>>(p);
    return cudaGetLastError();
}

template <int NB>
cudaError_t launch_cross_nb(const CrossParams& p, int n_sent, cudaStream_t st) {
    dim3 grid(p.n_split, p.H, n_sent);
    cross_kernel<NB><<<grid, kThreads, cross_smem_bytes(), st>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t configure_decode_kernels() {
    cudaError_t e;
    if ((e = configure_nb<1>()) != cudaSuccess) return e;
    if ((e = configure_nb<2>()) != cudaSuccess) return e;
    if ((e = configure_nb<4>()) != cudaSuccess) return e;
    return configure_nb<8>();
}

cudaError_t launch_decode_self(const SelfParams& p, int n_sent, int n_beams, cudaStream_t st) {
    switch (n_beams) {
        case 1: return launch_self_nb<1>(p, n_sent, st);
        case 2: return launch_self_nb<2>(p, n_sent, st);
        case 4: return launch_self_nb<4>(p, n_sent, st);
        case 8: return launch_self_nb<8>(p, n_sent, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_cross(const CrossParams& p, int n_sent, int n_beams, cudaStream_t st) {
    switch (n_beams) {
        case 1: return launch_cross_nb<1>(p, n_sent, st);
        case 2: return launch_cross_nb<2>(p, n_sent, st);
        case 4: return launch_cross_nb<4>(p, n_sent, st);
        case 8: return launch_cross_nb<8>(p, n_sent, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_reorder(uint8_t* hist, int Tp, const int* parent, int n_sent, int n_beams,
                           int* err, cudaStream_t st) {
    reorder_kernel<<<n_sent, 128, 0, st>>>(hist, Tp, parent, n_beams, err);
    return cudaGetLastError();
}

cudaError_t launch_hist_init(uint8_t* hist, int Tp, int n_sent, cudaStream_t st) {
    const size_t rows = (size_t)Tp * n_sent;
    if (rows == 0) return cudaSuccess;
    const int blocks = (int)((rows + 255) / 256 < 4096 ? (rows + 255) / 256 : 4096);
    hist_init_kernel<<<blocks, 256, 0, st>>>(hist, rows);
    return cudaGetLastError();
}

cudaError_t launch_set_memory(float* km, float* vm, int max_src, int H, const float* k,
                              const float* v, long long stride_head, long long stride_row,
                              int n_src, cudaStream_t st) {
    const size_t total = (size_t)H * n_src * 16;
    const int blocks = (int)((total + 255) / 256 < 2048 ? (total + 255) / 256 : 2048);
    set_memory_kernel<<<blocks, 256, 0, st>>>(km, vm, max_src, H, k, v, stride_head, stride_row,
                                              n_src);
    return cudaGetLastError();
}

}  // namespace nllb
