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
//   * split-KV when (sentences x heads) cannot fill the 148 SMs: the splits
//     of one (sentence, head) form a thread-block cluster; each leaves its
//     (max, sum, acc) record in its own shared memory and cluster rank 0
//     merges them over distributed shared memory (flash-decoding combine
//     without a global workspace, atomics or a second launch);
//   * programmatic dependent launch: a kernel lets the next one in the stream
//     start its prologue early and waits (griddepcontrol.wait) before it
//     touches anything a predecessor writes.
//
// Self-attention cache row (p, slot) of a (sentence, head) is at
// ((p * n_beams) + slot) * 64: all beams' rows of one position are adjacent,
// so a chunk of positions is one contiguous block whatever the beam history.
// hist[s][p][b] names the slot that holds position p of logical beam b; a
// beam reorder permutes these bytes (reorder_kernel) instead of copying
// caches (the reference copies each parent cache, main.c:481-482).
#include "device_common.cuh"
#include "kernels.h"
#include "planes.cuh"

namespace nllb {

namespace {

constexpr int kThreads = 128;
constexpr int kBarBytes = 128;  // mbarriers at the start of dynamic shared memory

// ---------------------------------------------------------------------------
// Split merge over the cluster
// ---------------------------------------------------------------------------
// rec: this CTA's per-beam records [NB][68] (m, l, -, -, acc[64]) in shared
// memory; abort_flag: this CTA's abort word.  Rank 0 merges the n_split
// records of each beam and writes out[bb*row_stride + 0..63].  Every thread of
// every CTA of the cluster calls this (the barriers are cluster-wide), so
// no CTA leaves while its records may still be read.
// Where a CTA's output rows go: fp32 rows, or (PLANES) the same element
// offsets in the two fp16 planes.  A template parameter, so that the fp32 form
// compiles exactly as a kernel without the option.
template <bool PLANES>
struct OutRows;
template <>
struct OutRows<false> {
    float* out;  // row 0, column 0 of this (sentence, head)
    size_t row_stride;
    __device__ __forceinline__ void put(int bb, int q4, float4 v) const {
        reinterpret_cast<float4*>(out + bb * row_stride)[q4] = v;
    }
};
template <>
struct OutRows<true> {
    plane_t* planes;  // the same offset in plane 0
    size_t row_stride, plane_stride;
    __device__ __forceinline__ void put(int bb, int q4, float4 v) const {
        store_planes_x4(planes, plane_stride, (size_t)bb * row_stride + 4 * q4, v);
    }
};
// PLANES: p.out is the base of the fp16 planes covering the launch's rows
// (gridDim.z sentences x NB beams x H heads x 64), one plane after the other.
template <bool PLANES, int NB, typename Params>
__device__ __forceinline__ OutRows<PLANES> out_rows(const Params& p, size_t off) {
    if constexpr (PLANES)
        return OutRows<true>{reinterpret_cast<plane_t*>(p.out) + off, (size_t)p.H * 64,
                             (size_t)gridDim.z * NB * p.H * 64};
    else
        return OutRows<false>{p.out + off, (size_t)p.H * 64};
}

template <int NB, typename Dst>
__device__ __forceinline__ void cluster_merge(const float* rec, const int* abort_flag, int n_split,
                                              const Dst& dst) {
    cluster_sync_all();
    if (cluster_ctarank() == 0) {
        bool any_abort = false;
        for (int r = 0; r < n_split; ++r) any_abort |= ld_cluster_s32(map_rank(abort_flag, r)) != 0;
        if (!any_abort) {
            for (int idx = threadIdx.x; idx < NB * 16; idx += blockDim.x) {
                const int bb = idx >> 4, q4 = idx & 15;
                const float* mine = rec + bb * kPartFloats;
                float M = -INFINITY;
                for (int r = 0; r < n_split; ++r) M = fmaxf(M, ld_cluster_f32(map_rank(mine, r)));
                float L = 0.f;
                float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int r = 0; r < n_split; ++r) {
                    const uint32_t base = map_rank(mine, r);
                    const float w = safe_exp2_diff(ld_cluster_f32(base), M);
                    L = fmaf(w, ld_cluster_f32(base + 4), L);
                    A = f4_fma(w, ld_cluster_f4(base + 16 + 16 * q4), A);
                }
                dst.put(bb, q4, f4_scale(A, 1.0f / L));
            }
        }
    }
    cluster_sync_all();
}

// Merge `nsrc` (m, l, acc) records of one beam held in shared memory
// (record j at recs + j*stride) into (M, L, A quad q4).
__device__ __forceinline__ void merge_local(const float* recs, int nsrc, int stride, int q4, float& M,
                                            float& L, float4& A) {
    M = -INFINITY;
    for (int j = 0; j < nsrc; ++j) M = fmaxf(M, recs[j * stride]);
    L = 0.f;
    A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < nsrc; ++j) {
        const float* rc = recs + j * stride;
        const float w = safe_exp2_diff(rc[0], M);
        L = fmaf(w, rc[1], L);
        A = f4_fma(w, reinterpret_cast<const float4*>(rc + 4)[q4], A);
    }
}

// ---------------------------------------------------------------------------
// Decoder self-attention
// ---------------------------------------------------------------------------
// MODE 0: the history as it is.  MODE 1 (P = SelfParamsR): a pending beam
// reorder is applied on the way -- logical beam b reads the slot of its
// parent, hist[p][parent[b]], from the current history p.hist, and the
// head-0 CTAs write the composed rows of their positions, plus the new
// position, to the other history buffer p.hist_w; no reorder launch.
// MODE 2: the bounded-wait test -- chunk 0 is never requested and the main
// loop waits for it with a ~1 ms budget, so the wait runs out; the kernel
// takes its timeout path (error bit, drain of the copies it did issue, no
// output).
template <int NB, bool PLANES, int MODE, typename P>
__global__ void __launch_bounds__(kThreads) decode_self_kernel(const P p) {
    constexpr int CP = kSelfChunkRows / NB;  // positions per chunk
    constexpr int NSUB = 8 / NB;         // half-warps per beam
    constexpr int RPH = CP / NSUB;       // positions per half-warp per chunk
    constexpr int KV_FLOATS = CP * NB * 64;
    constexpr int H_BYTES = CP * 8;

    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    float* sK = reinterpret_cast<float*>(smem + kBarBytes);
    float* sV = sK + kSelfStages * KV_FLOATS;
    unsigned char* sH = reinterpret_cast<unsigned char*>(sV + kSelfStages * KV_FLOATS);
    __shared__ int s_abort;
    __shared__ int s_par[8];  // MODE 1: parent of each logical beam

    pdl_launch_dependents();

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
    const size_t qrow = ((size_t)s * NB + b) * (size_t)p.H * 64 + (size_t)h * 64;

    if (tid == 0) {
        for (int i = 0; i < kSelfStages; ++i) mbar_init(&bar[i], 1);
        fence_barrier_init();
        s_abort = 0;
    }
    __syncthreads();
    pdl_wait_primary();  // cache, history and q come from earlier kernels

    auto issue = [&](int c) {
        const int st = c % kSelfStages;
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
        for (int c = 0; c < kSelfStages - 1 && c < nchunk; ++c)
            if (MODE != 2 || c != 0) issue(c);
    }
    if constexpr (MODE == 1) {
        // parents come from an earlier kernel (after the wait above); seen by
        // all threads after the first chunk's barrier
        if (tid < NB) {
            int v = p.parent[(size_t)s * NB + tid];
            if (v < 0 || v >= NB) {
                if (split == 0 && h == 0) atomicOr(p.err, NLLB_DEV_ERR_BAD_PARENT);
                v = tid;  // stays in bounds; the call reports the error
            }
            s_par[tid] = v;
        }
    }

    const float4 qv = __ldg(reinterpret_cast<const float4*>(p.q + qrow) + l16);
    // the new token's k/v, loaded now so their latency hides behind the stream
    float4 kn = make_float4(0.f, 0.f, 0.f, 0.f), vn = kn;
    if (owns_new) {
        kn = __ldg(reinterpret_cast<const float4*>(p.k_new + qrow) + l16);
        vn = __ldg(reinterpret_cast<const float4*>(p.v_new + qrow) + l16);
    }

    float m = -INFINITY, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int consumed = 0;

    for (int c = 0; c < nchunk; ++c) {
        const int st = c % kSelfStages;
        const uint32_t par = (uint32_t)((c / kSelfStages) & 1);
        if (!mbar_wait_bounded(&bar[st], par, MODE == 2 ? kTestWaitBudgetCycles : kWaitBudgetCycles)) s_abort = 1;
        __syncthreads();  // stage (c-1) fully consumed; abort flag visible
        if (s_abort) break;
        consumed = c + 1;
        if (tid == 0 && c + kSelfStages - 1 < nchunk) issue(c + kSelfStages - 1);

        const int np = min(CP, p1 - (p0 + c * CP));
        const float* K = sK + st * KV_FLOATS;
        const float* V = sV + st * KV_FLOATS;
        const unsigned char* Hs = sH + st * H_BYTES;
        int hb = b;  // the byte of a history row naming this beam's slot
        if constexpr (MODE == 1) {
            hb = s_par[b];
            if (h == 0 && tid < np) {  // composed row of position p0 + c*CP + tid
                const unsigned char* src = Hs + tid * 8;
                unsigned char row[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) row[j] = (j < NB) ? src[s_par[j]] : src[j];
                uint2 v;
                memcpy(&v, row, 8);
                *reinterpret_cast<uint2*>(p.hist_w + ((size_t)s * p.Tp + (p0 + c * CP + tid)) * 8) = v;
            }
        }

        float sc[RPH];
        int slot[RPH];
#pragma unroll
        for (int i = 0; i < RPH; ++i) {
            const int pl = sub + i * NSUB;
            const bool ok = pl < np;
            slot[i] = ok ? Hs[pl * 8 + hb] : 0;
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

    float* red = sK;                    // [8 half-warps][68], overlays the ring (free after the loop)
    float* rec = sK + 8 * kPartFloats;  // [NB][68] this CTA's merged records
    const size_t out_off = (size_t)s * NB * p.H * 64 + (size_t)h * 64;
    const auto dst = out_rows<PLANES, NB>(p, out_off);

    if (s_abort) {
        // let copies still in flight into this CTA's shared memory land, then stop
        if (tid == 0) {
            atomicOr(p.err, NLLB_DEV_ERR_TIMEOUT);
            const int issued = min(nchunk, consumed + kSelfStages - 1);
            for (int c = consumed; c < issued; ++c)
                if (MODE != 2 || c != 0)  // the test mode never requested chunk 0
                    (void)mbar_wait_bounded(&bar[c % kSelfStages], (uint32_t)((c / kSelfStages) & 1));
        }
    } else {
        // The new token at position `step`: every beam attends to its own k_new.
        if (owns_new) {
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
                if (h == 0 && l16 == 0)
                    p.hist_w[((size_t)s * p.Tp + p.step) * 8 + b] = (unsigned char)b;
            }
        }
        __syncthreads();
        {
            float* r = red + hw * kPartFloats;
            if (l16 == 0) {
                r[0] = m;
                r[1] = l;
            }
            reinterpret_cast<float4*>(r + 4)[l16] = acc;
        }
        __syncthreads();
        for (int idx = tid; idx < NB * 16; idx += kThreads) {
            const int bb = idx >> 4, q4 = idx & 15;
            float M, L;
            float4 A;
            merge_local(red + bb * kPartFloats, NSUB, NB * kPartFloats, q4, M, L, A);
            if (p.n_split == 1) {
                dst.put(bb, q4, f4_scale(A, 1.0f / L));
            } else {
                float* r = rec + bb * kPartFloats;
                if (q4 == 0) {
                    r[0] = M;
                    r[1] = L;
                }
                reinterpret_cast<float4*>(r + 4)[q4] = A;
            }
        }
    }
    if (p.n_split > 1) cluster_merge<NB>(rec, &s_abort, p.n_split, dst);
}

// ---------------------------------------------------------------------------
// Cross-attention: all beams of a sentence share each memory row.
// ---------------------------------------------------------------------------
// EXPIRE: the bounded-wait test -- chunk 0 is never requested and the main
// loop waits for it with a ~1 ms budget, so the wait runs out and the kernel
// takes its timeout path (error bit, drain of the copies it did issue, no output).
template <int NB, int CP, int kCrossStages, bool PLANES, bool EXPIRE = false>
__global__ void __launch_bounds__(kThreads) cross_kernel(const CrossParams p) {
    constexpr int RPH = CP / 8;  // rows per half-warp per chunk
    constexpr int KV_FLOATS = CP * 64;

    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    float* sK = reinterpret_cast<float*>(smem + kBarBytes);
    float* sV = sK + kCrossStages * KV_FLOATS;
    __shared__ int s_abort;

    pdl_launch_dependents();

    const int split = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x, hw = tid >> 4, l16 = tid & 15;

    if (tid == 0) {
        for (int i = 0; i < kCrossStages; ++i) mbar_init(&bar[i], 1);
        fence_barrier_init();
        s_abort = 0;
    }
    __syncthreads();
    // The memory rows and lengths are read before the wait on the previous
    // kernel: their writers (set_memory_kernel, set_memory_batched_kernel)
    // let no dependent start before they complete, so every kernel after
    // them in the stream starts after the memory is written.  The first
    // chunks' copies thus overlap the previous kernel's tail; q comes after
    // the wait.
    const int len = __ldg(p.n_src + s);
    const int p0 = split * p.pos_per_split;
    const int p1 = min(len, p0 + p.pos_per_split);
    const int nchunk = (p1 > p0) ? (p1 - p0 + CP - 1) / CP : 0;

    const size_t head_row0 = ((size_t)s * p.H + h) * (size_t)p.max_src;
    const float* gK = p.km + head_row0 * 64;
    const float* gV = p.vm + head_row0 * 64;

    auto issue = [&](int c) {
        const int st = c % kCrossStages;
        const int pc0 = p0 + c * CP;
        const int np = min(CP, p1 - pc0);
        const uint32_t kvb = (uint32_t)np * 256u;
        mbar_arrive_expect_tx(&bar[st], 2u * kvb);
        bulk_g2s(sK + st * KV_FLOATS, gK + (size_t)pc0 * 64, kvb, &bar[st]);
        bulk_g2s(sV + st * KV_FLOATS, gV + (size_t)pc0 * 64, kvb, &bar[st]);
    };
    if (tid == 0) {
        for (int c = 0; c < kCrossStages - 1 && c < nchunk; ++c)
            if (!EXPIRE || c != 0) issue(c);
    }
    pdl_wait_primary();  // q comes from the previous kernel; the output may still be read by it

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
        const int st = c % kCrossStages;
        const uint32_t par = (uint32_t)((c / kCrossStages) & 1);
        if (!mbar_wait_bounded(&bar[st], par, EXPIRE ? kTestWaitBudgetCycles : kWaitBudgetCycles)) s_abort = 1;
        __syncthreads();
        if (s_abort) break;
        consumed = c + 1;
        if (tid == 0 && c + kCrossStages - 1 < nchunk) issue(c + kCrossStages - 1);

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
            if constexpr (NB == 4) {
                float pd[4], d[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) pd[b] = f4_dot(qv[b], kv);
                halfwarp_sum4(pd, d);
#pragma unroll
                for (int b = 0; b < 4; ++b) sc[b][i] = ok ? d[b] * p.scale_log2 : -INFINITY;
            } else {
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const float d = halfwarp_sum(f4_dot(qv[b], kv));
                    sc[b][i] = ok ? d * p.scale_log2 : -INFINITY;
                }
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

    float* red = sK;                         // [8 half-warps][NB][68], overlays the ring
    float* rec = sK + 8 * NB * kPartFloats;  // [NB][68]
    const size_t out_off = (size_t)s * NB * p.H * 64 + (size_t)h * 64;
    const auto dst = out_rows<PLANES, NB>(p, out_off);

    if (s_abort) {
        if (tid == 0) {
            atomicOr(p.err, NLLB_DEV_ERR_TIMEOUT);
            const int issued = min(nchunk, consumed + kCrossStages - 1);
            for (int c = consumed; c < issued; ++c)
                if (!EXPIRE || c != 0)  // the test form never requested chunk 0
                    (void)mbar_wait_bounded(&bar[c % kCrossStages], (uint32_t)((c / kCrossStages) & 1));
        }
    } else {
        __syncthreads();
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            float* r = red + (hw * NB + b) * kPartFloats;
            if (l16 == 0) {
                r[0] = m[b];
                r[1] = l[b];
            }
            reinterpret_cast<float4*>(r + 4)[l16] = acc[b];
        }
        __syncthreads();
        for (int idx = tid; idx < NB * 16; idx += kThreads) {
            const int bb = idx >> 4, q4 = idx & 15;
            float M, L;
            float4 A;
            merge_local(red + bb * kPartFloats, 8, NB * kPartFloats, q4, M, L, A);
            if (p.n_split == 1) {
                dst.put(bb, q4, f4_scale(A, 1.0f / L));
            } else {
                float* r = rec + bb * kPartFloats;
                if (q4 == 0) {
                    r[0] = M;
                    r[1] = L;
                }
                reinterpret_cast<float4*>(r + 4)[q4] = A;
            }
        }
    }
    if (p.n_split > 1) cluster_merge<NB>(rec, &s_abort, p.n_split, dst);
}

// ---------------------------------------------------------------------------
// Beam history maintenance
// ---------------------------------------------------------------------------
// new slot of (p, b) = old slot of (p, parent[b]), in place, one CTA per sentence.
__global__ void reorder_kernel(unsigned char* hist, int Tp, const int* parent, int n_beams,
                               int* err) {
    pdl_launch_dependents();
    pdl_wait_primary();  // earlier kernels may still read the history / write parent
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

// k[r*stride_row + h*stride_head + d] -> km[h][r][d] (one layer, one sentence);
// thread 0 of block 0 also records the row count.  Launched without
// programmatic dependent launch and never triggering its dependents early
// (cross_kernel reads the memory before its wait on the previous kernel).
__global__ void set_memory_kernel(float* km, float* vm, int max_src, int H, const float* k,
                                  const float* v, long long stride_head, long long stride_row,
                                  int n_src, int* n_src_slot) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *n_src_slot = n_src;
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

// Ring (K, V and history stages) or, after the loop, the merge records
// overlaid on it, whichever is larger, after the barrier block.
template <int NB>
size_t self_smem_bytes() {
    constexpr int CP = kSelfChunkRows / NB;
    const size_t ring = (size_t)kSelfStages * (2 * CP * NB * 64 * sizeof(float) + CP * 8);
    const size_t merge = (size_t)(8 + NB) * kPartFloats * sizeof(float);
    return kBarBytes + (ring > merge ? ring : merge);
}

template <int NB, int CP, int kCrossStages>
size_t cross_smem_bytes() {
    const size_t ring = (size_t)kCrossStages * 2 * CP * 64 * sizeof(float);
    const size_t merge = (size_t)(8 * NB + NB) * kPartFloats * sizeof(float);
    return kBarBytes + (ring > merge ? ring : merge);
}

// Launch with programmatic stream serialisation and, for split-KV, a cluster
// of n_split CTAs along x.
template <typename Params>
cudaError_t launch_ex(void (*kernel)(Params), dim3 grid, size_t smem, int cluster_x,
                      cudaStream_t st, const Params& p) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    int n = 0;
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = kPdlLaunch;
    ++n;
    if (cluster_x > 1) {
        attrs[n].id = cudaLaunchAttributeClusterDimension;
        attrs[n].val.clusterDim.x = (unsigned)cluster_x;
        attrs[n].val.clusterDim.y = 1;
        attrs[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int NB, bool PLANES>
cudaError_t configure_nb_out() {
    cudaError_t e = cudaFuncSetAttribute(decode_self_kernel<NB, PLANES, 0, SelfParams>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)self_smem_bytes<NB>());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(decode_self_kernel<NB, PLANES, 1, SelfParamsR>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)self_smem_bytes<NB>());
    if (e != cudaSuccess) return e;
    if constexpr (NB == 4 && !PLANES) {
        e = cudaFuncSetAttribute(decode_self_kernel<4, false, 2, SelfParams>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)self_smem_bytes<4>());
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(cross_kernel<4, kCrossShortRows, 3, false, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)cross_smem_bytes<4, kCrossShortRows, 3>());
        if (e != cudaSuccess) return e;
    }
    e = cudaFuncSetAttribute(cross_kernel<NB, kCrossShortRows, 3, PLANES>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)cross_smem_bytes<NB, kCrossShortRows, 3>());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(cross_kernel<NB, kCrossLongRows, 3, PLANES>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)cross_smem_bytes<NB, kCrossLongRows, 3>());
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(cross_kernel<NB, kCrossSplitRows, 2, PLANES>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)cross_smem_bytes<NB, kCrossSplitRows, 2>());
}

template <int NB>
cudaError_t configure_nb() {
    cudaError_t e = configure_nb_out<NB, false>();
    if (e != cudaSuccess) return e;
    return configure_nb_out<NB, true>();
}

template <int NB, bool PLANES>
cudaError_t launch_self_out(const SelfParams& p, int n_sent, cudaStream_t st, SelfMode mode, const int* parent) {
    const dim3 grid(p.n_split, p.H, n_sent);
    if (mode == SelfMode::reorder) {
        SelfParamsR r;
        static_cast<SelfParams&>(r) = p;
        r.parent = parent;
        return launch_ex(decode_self_kernel<NB, PLANES, 1, SelfParamsR>, grid, self_smem_bytes<NB>(), p.n_split,
                         st, r);
    }
    if (mode == SelfMode::expire_wait) {
        if constexpr (NB == 4 && !PLANES)
            return launch_ex(decode_self_kernel<4, false, 2, SelfParams>, grid, self_smem_bytes<4>(), p.n_split,
                             st, p);
        else
            return cudaErrorInvalidValue;
    }
    return launch_ex(decode_self_kernel<NB, PLANES, 0, SelfParams>, grid, self_smem_bytes<NB>(), p.n_split, st, p);
}

template <int NB>
cudaError_t launch_self_nb(const SelfParams& p, int n_sent, cudaStream_t st, bool planes, SelfMode mode,
                           const int* parent) {
    return planes ? launch_self_out<NB, true>(p, n_sent, st, mode, parent)
                  : launch_self_out<NB, false>(p, n_sent, st, mode, parent);
}

template <int NB, bool PLANES>
cudaError_t launch_cross_out(const CrossParams& p, int n_sent, int chunk_rows, cudaStream_t st) {
    if (chunk_rows == kCrossSplitRows)
        return launch_ex(cross_kernel<NB, kCrossSplitRows, 2, PLANES>, dim3(p.n_split, p.H, n_sent),
                         cross_smem_bytes<NB, kCrossSplitRows, 2>(), p.n_split, st, p);
    if (chunk_rows == kCrossLongRows)
        return launch_ex(cross_kernel<NB, kCrossLongRows, 3, PLANES>, dim3(p.n_split, p.H, n_sent),
                         cross_smem_bytes<NB, kCrossLongRows, 3>(), p.n_split, st, p);
    return launch_ex(cross_kernel<NB, kCrossShortRows, 3, PLANES>, dim3(p.n_split, p.H, n_sent),
                     cross_smem_bytes<NB, kCrossShortRows, 3>(), p.n_split, st, p);
}

template <int NB>
cudaError_t launch_cross_nb(const CrossParams& p, int n_sent, int chunk_rows, cudaStream_t st, bool planes) {
    return planes ? launch_cross_out<NB, true>(p, n_sent, chunk_rows, st)
                  : launch_cross_out<NB, false>(p, n_sent, chunk_rows, st);
}

}  // namespace

cudaError_t configure_decode_kernels() {
    cudaError_t e;
    if ((e = configure_nb<1>()) != cudaSuccess) return e;
    if ((e = configure_nb<2>()) != cudaSuccess) return e;
    if ((e = configure_nb<4>()) != cudaSuccess) return e;
    return configure_nb<8>();
}

cudaError_t launch_decode_self(const SelfParams& p, int n_sent, int n_beams, cudaStream_t st, bool planes,
                               SelfMode mode, const int* parent) {
    switch (n_beams) {
        case 1: return launch_self_nb<1>(p, n_sent, st, planes, mode, parent);
        case 2: return launch_self_nb<2>(p, n_sent, st, planes, mode, parent);
        case 4: return launch_self_nb<4>(p, n_sent, st, planes, mode, parent);
        case 8: return launch_self_nb<8>(p, n_sent, st, planes, mode, parent);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_cross(const CrossParams& p, int n_sent, int n_beams, int chunk_rows, cudaStream_t st,
                         bool planes, bool expire_wait) {
    if (expire_wait) {
        if (n_beams != 4 || planes || chunk_rows != kCrossShortRows) return cudaErrorInvalidValue;
        return launch_ex(cross_kernel<4, kCrossShortRows, 3, false, true>, dim3(p.n_split, p.H, n_sent),
                         cross_smem_bytes<4, kCrossShortRows, 3>(), p.n_split, st, p);
    }
    switch (n_beams) {
        case 1: return launch_cross_nb<1>(p, n_sent, chunk_rows, st, planes);
        case 2: return launch_cross_nb<2>(p, n_sent, chunk_rows, st, planes);
        case 4: return launch_cross_nb<4>(p, n_sent, chunk_rows, st, planes);
        case 8: return launch_cross_nb<8>(p, n_sent, chunk_rows, st, planes);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_reorder(uint8_t* hist, int Tp, const int* parent, int n_sent, int n_beams,
                           int* err, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_sent, 1, 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = kPdlLaunch;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, reorder_kernel, hist, Tp, parent, n_beams, err);
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
                              int n_src, int* n_src_slot, cudaStream_t st) {
    const size_t total = (size_t)H * n_src * 16;
    const int blocks = (int)((total + 255) / 256 < 2048 ? (total + 255) / 256 : 2048);
    set_memory_kernel<<<blocks, 256, 0, st>>>(km, vm, max_src, H, k, v, stride_head, stride_row,
                                              n_src, n_src_slot);
    return cudaGetLastError();
}

}  // namespace nllb
