// prefill.cu -- encoder self-attention prefill, fp32 (sm_100a).
//
// Two kernels compute attention_head_flash (tensor.c:286-332) /
// encoder.c:166-205 for every (sequence, head, query row):
//
// prefill_tc_kernel (seq_len 33..256): 5th-generation tensor cores.  One CTA
//   per (128-query tile, head, sequence) with 8 warps: query row r is TMEM
//   lane r, owned by two threads (warps w and w+4 reach the same lane quarter)
//   that take alternate 32-key halves of every 64-key chunk.  Inputs are split while they are staged into
//   128-byte-swizzled shared memory: hi = x with the low 13 mantissa bits
//   cleared (exact in tf32), lo = x - hi.  Each product is taken as
//   hi*hi' + hi*lo' + lo*hi' (3xTF32 on tcgen05.mma kind::tf32, fp32
//   accumulation in TMEM), which keeps fp32 accuracy.  The softmax is the
//   reference's two-pass form: all scores of a row sit in TMEM (256 columns),
//   pass 1 takes the row max, pass 2 forms P = exp(s - max) 64 keys at a time,
//   stages P (split) and V^T (split) in shared memory and accumulates
//   O += P.V in TMEM; the row sum is divided out at the end.  Q.K^T runs in
//   groups of 128 keys (one N=128 MMA group for seq_len <= 128).  The loads of
//   Q and the first K group are all issued before any is stored, and the V
//   chunks travel in registers while the score MMAs and softmax run, so a CTA
//   pays about two DRAM latencies, not one per tile.
// prefill_ffma_kernel (other lengths): SIMT fp32 flash attention with an
//   online softmax over 64-key tiles.
#include <algorithm>

#include "device_common.cuh"
#include "kernels.h"

namespace nllb {

namespace {

constexpr int BQ = 64;     // queries per CTA
constexpr int BK = 64;     // keys per tile
constexpr int LDS = 68;    // padded smem row stride (floats), keeps float4 alignment
constexpr int kThreads = 128;

__global__ void __launch_bounds__(kThreads) prefill_ffma_kernel(const PrefillParams p) {
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;               // [BQ][LDS]
    float* Ks = Qs + BQ * LDS;    // [BK][LDS]
    float* Vs = Ks + BK * LDS;    // [BK][LDS]
    float* Ps = Vs + BK * LDS;    // [BQ][LDS]

    pdl_launch_dependents();
    pdl_wait_primary();  // inputs come from earlier kernels

    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int S = p.S;
    const int q0 = qt * BQ;
    const long long base = (p.row_start ? (long long)__ldg(p.row_start + b) * p.sr : (long long)b * p.sb) +
                           (long long)h * p.sh;
    // valid_len[b] <= 0 leaves no unmasked key; the reference's additive -1e9
    // mask then makes every score equal, i.e. the plain mean of V: do that.
    int kv_len = S;
    bool uniform = false;
    if (p.valid_len) {
        const int vl = __ldg(p.valid_len + b);
        if (vl <= 0) uniform = true;
        else kv_len = min(vl, S);
    }
    // query rows read and written: packed rows end at the sequence's length
    const int q_lim = p.row_start ? (uniform ? 0 : kv_len) : S;
    if (q0 >= q_lim) return;  // packed rows: this query tile lies past the sequence (uniform per CTA)
    const float* mrow0 =
        p.mask ? p.mask + (long long)b * p.msb + (long long)h * p.msh : nullptr;

    // Q tile (rows beyond S read as zero)
    for (int i = tid; i < BQ * 16; i += kThreads) {
        const int r = i >> 4, c4 = i & 15;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + r < q_lim) v = __ldg(reinterpret_cast<const float4*>(p.q + base + (long long)(q0 + r) * p.sr) + c4);
        reinterpret_cast<float4*>(Qs + r * LDS)[c4] = v;
    }

    float m[8], lsum[8];
    float4 o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        m[i] = -INFINITY;
        lsum[i] = 0.f;
        o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    const int n_kt = (kv_len + BK - 1) / BK;
    for (int kt = 0; kt < n_kt; ++kt) {
        const int k0 = kt * BK;
        __syncthreads();  // previous tile's K/V/P no longer read
        for (int i = tid; i < BK * 16; i += kThreads) {
            const int r = i >> 4, c4 = i & 15;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (k0 + r < kv_len) {
                const long long off = base + (long long)(k0 + r) * p.sr;
                kv = __ldg(reinterpret_cast<const float4*>(p.k + off) + c4);
                vv = __ldg(reinterpret_cast<const float4*>(p.v + off) + c4);
            }
            reinterpret_cast<float4*>(Ks + r * LDS)[c4] = kv;
            reinterpret_cast<float4*>(Vs + r * LDS)[c4] = vv;
        }
        __syncthreads();

        // scores: s[i][j] for rows ty+8i, keys tx+16j
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
        for (int k4 = 0; k4 < 16; ++k4) {
            float4 kf[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) kf[j] = reinterpret_cast<const float4*>(Ks + (tx + 16 * j) * LDS)[k4];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 qf = reinterpret_cast<const float4*>(Qs + (ty + 8 * i) * LDS)[k4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    s[i][j] = fmaf(qf.x, kf[j].x, s[i][j]);
                    s[i][j] = fmaf(qf.y, kf[j].y, s[i][j]);
                    s[i][j] = fmaf(qf.z, kf[j].z, s[i][j]);
                    s[i][j] = fmaf(qf.w, kf[j].w, s[i][j]);
                }
            }
        }

        // scale, masks, online softmax
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int qr = q0 + ty + 8 * i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kc = k0 + tx + 16 * j;
                float v = uniform ? 0.f : s[i][j] * p.scale_log2;
                if (mrow0 && !uniform && qr < S && kc < kv_len)
                    v = fmaf(__ldg(mrow0 + (long long)qr * S + kc), kLog2e, v);
                if (kc >= kv_len) v = -INFINITY;
                s[i][j] = v;
                mx = fmaxf(mx, v);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            const float mn = fmaxf(m[i], mx);
            const float corr = safe_exp2_diff(m[i], mn);
            float rs = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float e = (s[i][j] == -INFINITY) ? 0.f : exp2f(s[i][j] - mn);
                Ps[(ty + 8 * i) * LDS + tx + 16 * j] = e;
                rs += e;
            }
            lsum[i] = fmaf(lsum[i], corr, rs);
            o[i] = f4_scale(o[i], corr);
            m[i] = mn;
        }
        __syncthreads();

        // o[i] += P[row][:] . V[:, 4tx..4tx+3]
#pragma unroll 2
        for (int c4 = 0; c4 < 16; ++c4) {
            float4 vf[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) vf[j] = reinterpret_cast<const float4*>(Vs + (4 * c4 + j) * LDS)[tx];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 pf = reinterpret_cast<const float4*>(Ps + (ty + 8 * i) * LDS)[c4];
                o[i] = f4_fma(pf.x, vf[0], o[i]);
                o[i] = f4_fma(pf.y, vf[1], o[i]);
                o[i] = f4_fma(pf.z, vf[2], o[i]);
                o[i] = f4_fma(pf.w, vf[3], o[i]);
            }
        }
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float l = lsum[i];
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        const int qr = q0 + ty + 8 * i;
        if (qr < q_lim) {
            float* dst = p.out + base + (long long)qr * p.sr;
            reinterpret_cast<float4*>(dst)[tx] = f4_scale(o[i], 1.0f / l);
        }
    }
}


// ---------------------------------------------------------------------------
// tcgen05 kernel
// ---------------------------------------------------------------------------
constexpr int TC_THREADS = 256;  // two threads per query row / TMEM lane
constexpr int TC_THREADS_SPLIT = TC_THREADS;
constexpr int TC_Q = 128;      // queries per CTA (MMA M)
constexpr int TC_KG = 128;     // keys per score group (MMA N of Q.K^T)
constexpr int TC_K = 64;       // keys per P.V chunk (MMA K of P.V)
constexpr int TC_MAX_S = 256;  // score columns held in TMEM
constexpr uint32_t TC_TMEM_COLS = 512;
// shared-memory plan (bytes from a 1024-byte aligned base); every operand is
// K-major, 128-byte swizzled, in 32-column k-blocks of rows*128 bytes -- the
// layout a TMA box of [rows][32 fp32] lands in with the 128-byte swizzle
constexpr uint32_t SQH = 0, SQL = 32768;        // Q hi/lo [2][128 rows][128 B]; P hi/lo after the scores
constexpr uint32_t SKH = 65536, SKL = 98304;    // K hi/lo [2][128 keys][128 B]
constexpr uint32_t SVH = 131072, SVL = 147456;  // V^T hi/lo [2][64 dims][128 B]
constexpr uint32_t SVR = 163840;                // V as loaded: [2][128 keys][128 B] (two P.V chunks)
constexpr uint32_t SBAR = 196608;
constexpr uint32_t TC_SMEM = SBAR + 64 + 1024;  // + alignment slack
constexpr uint32_t TC_BOX_BYTES = 128 * 128;    // one [128 rows][32 fp32] box

// byte offset of (row, col) in a K-major SWIZZLE_128B operand of `nrows`
// rows x 64 fp32 columns: 32-column k-blocks of nrows*128 B, 128-B rows,
// 16-B chunks XOR-ed with row % 8.
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int nrows) {
    return (uint32_t)((col >> 5) * nrows * 128 + row * 128 + ((((col & 31) >> 2) ^ (row & 7)) << 4) +
                      ((col & 3) << 2));
}

// D[128 x N] (+)= A[128 x 64] . B[N x 64]^T with both operands split:
// Ah.Bh + Ah.Bl + Al.Bh over 8 k-steps of 8 (A has 128 rows, B has N rows).
template <int N>
__device__ __forceinline__ void mma_3xtf32(uint32_t d, uint32_t ah, uint32_t al, uint32_t bh, uint32_t bl,
                                           bool accumulate_first) {
    constexpr uint32_t idesc = umma_idesc_tf32(128, N);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        const uint32_t ao = (ks >> 2) * (128 * 128) + (ks & 3) * 32;
        const uint32_t bo = (ks >> 2) * (N * 128) + (ks & 3) * 32;
        const uint64_t dah = umma_desc_k_sw128(ah + ao), dal = umma_desc_k_sw128(al + ao);
        const uint64_t dbh = umma_desc_k_sw128(bh + bo), dbl = umma_desc_k_sw128(bl + bo);
        tc_mma_tf32(d, dah, dbh, idesc, (accumulate_first || ks > 0) ? 1u : 0u);
        tc_mma_tf32(d, dah, dbl, idesc, 1u);
        tc_mma_tf32(d, dal, dbh, idesc, 1u);
    }
}

// TMA: a box of the 4-D fp32 tensor map (d, then the row/head/sequence axes
// in the order of their strides) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// The two 32-column boxes of rows [r0, r0 + 128) of (sequence b, head h):
// coordinates (column, then the three outer axes in map order).
__device__ __forceinline__ void tma_rows128(uint32_t dst, const CUtensorMap* map, const PrefillParams& p, int r0,
                                            int h, int b, uint64_t* bar) {
    auto at = [&](int i) { return p.map_pos_row == i ? r0 : (p.map_pos_head == i ? h : b); };
    const int c0 = at(0), c1 = at(1), c2 = at(2);
    tma_load_4d(dst, map, 0, c0, c1, c2, bar);
    tma_load_4d(dst + TC_BOX_BYTES, map, 32, c0, c1, c2, bar);
}

// In place over `bytes` of loaded fp32 at hi: hi = x with the low 13 mantissa
// bits cleared (exact in tf32), lo (same offset at lo) = x - hi.
__device__ __forceinline__ void split_in_place(unsigned char* hi, unsigned char* lo, uint32_t bytes, int tid) {
    for (uint32_t off = (uint32_t)tid * 16; off < bytes; off += TC_THREADS_SPLIT * 16) {
        const float4 x = *reinterpret_cast<const float4*>(hi + off);
        const float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
        *reinterpret_cast<float4*>(hi + off) = h;
        *reinterpret_cast<float4*>(lo + off) = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    }
}

__device__ __forceinline__ void split_store4(unsigned char* hi_base, unsigned char* lo_base, uint32_t off,
                                             float4 x) {
    float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
    float4 l = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    *reinterpret_cast<float4*>(hi_base + off) = h;
    *reinterpret_cast<float4*>(lo_base + off) = l;
}

__device__ __forceinline__ float ex2_approx(float x) {  // 2^x, -inf -> +0
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// One CTA per (128-query tile, head, sequence), 8 warps.  Q, K and V tiles
// arrive by TMA (one thread issues the boxes after the wait on the previous
// kernel; V for the first 128 keys travels while the scores are computed)
// in the 128-byte-swizzled K-major layout the MMAs read; the threads then
// split Q and K in place (hi, lo) and transpose-split V chunk by chunk.
__global__ void __launch_bounds__(TC_THREADS, 1) prefill_tc_kernel(const PrefillParams p,
                                                                   const __grid_constant__ CUtensorMap map_q,
                                                                   const __grid_constant__ CUtensorMap map_k,
                                                                   const __grid_constant__ CUtensorMap map_v) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
    unsigned char* base = smem_raw + (base_addr - raw_addr);
    uint64_t* mma_bar = reinterpret_cast<uint64_t*>(base + SBAR);
    uint64_t* qk_bar = reinterpret_cast<uint64_t*>(base + SBAR + 8);  // Q and K group loads
    uint64_t* v_bar = reinterpret_cast<uint64_t*>(base + SBAR + 16);  // V loads
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + SBAR + 24);
    volatile int* s_abort = reinterpret_cast<volatile int*>(base + SBAR + 32);
    __shared__ float s_red[TC_THREADS];

    pdl_launch_dependents();

    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;  // TMEM lane quarter, column half
    const int S = p.S;
    const int q0 = qt * TC_Q;

    if (warp == 0) tmem_alloc(tmem_slot, TC_TMEM_COLS);
    if (tid == 0) {
        mbar_init(mma_bar, 1);
        mbar_init(qk_bar, 1);
        mbar_init(v_bar, 1);
        fence_barrier_init();
        *s_abort = 0;
        prefetch_map(&map_q);
        prefetch_map(&map_k);
        prefetch_map(&map_v);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off;             // scores: columns [0, 256)
    const uint32_t tO = tmem + lane_off + TC_MAX_S;  // output: columns [256, 320)

    pdl_wait_primary();  // q, k, v, lengths, row starts and mask come from earlier kernels

    // row coordinate of the sequence's row 0 in the tensor maps (packed rows:
    // its first row in the buffer; the sequence axis is then unused)
    const int row0 = p.row_start ? __ldg(p.row_start + b) : 0;
    const int bq = p.row_start ? 0 : b;
    const long long hbase = (p.row_start ? (long long)row0 * p.sr : (long long)b * p.sb) + (long long)h * p.sh;
    int kv_len = S;
    bool uniform = false;  // valid_len 0: equal weights over all keys (see prefill_ffma_kernel)
    if (p.valid_len) {
        const int vl = __ldg(p.valid_len + b);
        if (vl <= 0) uniform = true;
        else kv_len = min(vl, S);
    }
    // query rows read and written: packed rows end at the sequence's length
    const int q_lim = p.row_start ? (uniform ? 0 : kv_len) : S;
    if (q0 >= q_lim) {  // packed rows: this query tile lies past the sequence (uniform per CTA)
        tc_fence_before();
        __syncthreads();
        if (warp == 0) {
            tc_fence_after();
            tmem_dealloc(tmem, TC_TMEM_COLS);
        }
        return;
    }
    const int n_kg = (kv_len + TC_KG - 1) / TC_KG;  // score groups of 128 keys
    const int n_kc = (kv_len + TC_K - 1) / TC_K;    // P.V chunks of 64 keys
    const int rloc = quarter * 32 + lane;           // query row within the tile = TMEM lane
    const int row = q0 + rloc;
    const float* mrow = (p.mask && row < S)
                            ? p.mask + (long long)b * p.msb + (long long)h * p.msh + (long long)row * S
                            : nullptr;
    const float sl2 = p.scale_log2;

    // Q, K group 0 and V keys 0..127: every box issued at once.  A box counts
    // its full bytes toward the barrier, rows outside the tensor included
    // (they arrive as zeros).
    if (tid == 0) {
        mbar_arrive_expect_tx(qk_bar, 4 * TC_BOX_BYTES);
        tma_rows128(base_addr + SQH, &map_q, p, row0 + q0, h, bq, qk_bar);
        tma_rows128(base_addr + SKH, &map_k, p, row0, h, bq, qk_bar);
        mbar_arrive_expect_tx(v_bar, 2 * TC_BOX_BYTES);
        tma_rows128(base_addr + SVR, &map_v, p, row0, h, bq, v_bar);
    }

    uint32_t phase = 0, qk_phase = 0, v_phase = 0;         // waits completed per barrier
    uint32_t mma_issued = 0, qk_issued = 1, v_issued = 1;  // (thread 0) phases armed per barrier
    auto wait_bar = [&](uint64_t* bar, uint32_t& ph) -> bool {
        if (!mbar_wait_bounded(bar, ph & 1u)) *s_abort = 1;
        ++ph;
        __syncthreads();
        return *s_abort == 0;
    };
    // 32 scores (base-2 logits) of this thread's row, keys j0..j0+31
    auto scores32 = [&](int j0, float* v) {
        tmem_ld32(tS + (uint32_t)j0, v);
        if (uniform) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = (j0 + i < kv_len) ? 0.f : -INFINITY;
        } else if (mrow) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                v[i] = (j0 + i < kv_len) ? fmaf(__ldg(mrow + j0 + i), kLog2e, v[i] * sl2) : -INFINITY;
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = (j0 + i < kv_len) ? v[i] * sl2 : -INFINITY;
        }
    };

    bool ok = wait_bar(qk_bar, qk_phase);  // Q and K group 0 have landed
    if (ok) split_in_place(base + SQH, base + SQL, 2 * TC_BOX_BYTES, tid);
    for (int g = 0; g < n_kg && ok; ++g) {
        if (g > 0) {
            if (!(ok = wait_bar(mma_bar, phase))) break;  // group g-1's MMAs have read KH/KL
            if (tid == 0) {
                mbar_arrive_expect_tx(qk_bar, 2 * TC_BOX_BYTES);
                tma_rows128(base_addr + SKH, &map_k, p, row0 + g * TC_KG, h, bq, qk_bar);
                ++qk_issued;
            }
            if (!(ok = wait_bar(qk_bar, qk_phase))) break;
        }
        split_in_place(base + SKH, base + SKL, 2 * TC_BOX_BYTES, tid);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            mma_3xtf32<TC_KG>(tmem + (uint32_t)(g * TC_KG), base_addr + SQH, base_addr + SQL, base_addr + SKH,
                              base_addr + SKL, false);
            tc_commit(mma_bar);
            ++mma_issued;
        }
    }
    if (ok) ok = wait_bar(mma_bar, phase);  // scores in TMEM; Q's buffers are free (P goes there)
    tc_fence_after();

    // pass 1: row max (this thread: columns half*32 + 64c .. +31 of every chunk)
    float mx = -INFINITY;
    if (ok) {
        for (int kc = 0; kc < n_kc; ++kc) {
            float v[32];
            scores32(kc * TC_K + half * 32, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) mx = fmaxf(mx, v[i]);
        }
        s_red[tid] = mx;
    }
    __syncthreads();
    if (ok) mx = fmaxf(mx, s_red[tid ^ 128]);

    // pass 2: P chunk by chunk, O += P . V_chunk
    float sum = 0.f;
    for (int kc = 0; kc < n_kc && ok; ++kc) {
        if (kc > 0 && !(ok = wait_bar(mma_bar, phase))) break;  // previous chunk's MMAs have read P and V^T
        if ((kc & 1) == 0) {  // V keys 128*(kc/2) .. +127 have landed in SVR
            if (kc > 0 && tid == 0) {
                mbar_arrive_expect_tx(v_bar, 2 * TC_BOX_BYTES);
                tma_rows128(base_addr + SVR, &map_v, p, row0 + kc * TC_K, h, bq, v_bar);
                ++v_issued;
            }
            if (!(ok = wait_bar(v_bar, v_phase))) break;
        }
        {
            float v[32];
            scores32(kc * TC_K + half * 32, v);
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
                float e[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    e[i] = ex2_approx(v[c4 * 4 + i] - mx);
                    sum += e[i];
                }
                split_store4(base + SQH, base + SQL, sw128_off(rloc, half * 32 + c4 * 4, TC_Q),
                             make_float4(e[0], e[1], e[2], e[3]));
            }
        }
        // V chunk kc, transposed (row = head dim, column = key) and split;
        // keys past the sequence's length as zeros
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int jj = tid & 63, d4 = (tid >> 6) + 4 * it;  // key within the chunk, head-dim quad
            const int jr = (kc & 1) * TC_K + jj;                 // key row within SVR
            float4 x = *reinterpret_cast<const float4*>(base + SVR + sw128_off(jr, d4 * 4, 128));
            if (kc * TC_K + jj >= kv_len) x = make_float4(0.f, 0.f, 0.f, 0.f);
            const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t off = sw128_off(d4 * 4 + i, jj, 64);
                const float hv = tf32_hi(xs[i]);
                *reinterpret_cast<float*>(base + SVH + off) = hv;
                *reinterpret_cast<float*>(base + SVL + off) = xs[i] - hv;
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();  // also: every thread is done reading SVR for this chunk
        if (tid == 0) {
            tc_fence_after();
            mma_3xtf32<TC_K>(tmem + TC_MAX_S, base_addr + SQH, base_addr + SQL, base_addr + SVH, base_addr + SVL,
                             kc > 0);
            tc_commit(mma_bar);
            ++mma_issued;
        }
    }
    if (ok) ok = wait_bar(mma_bar, phase);
    tc_fence_after();

    if (ok) {
        s_red[tid] = sum;  // wait_bar ended with a barrier, pass-1 values are consumed
        __syncthreads();
        sum += s_red[tid ^ 128];
        float o[32];
        tmem_ld32(tO + (uint32_t)(half * 32), o);
        if (row < q_lim) {
            const float inv = 1.0f / sum;
            float4* dst = reinterpret_cast<float4*>(p.out + hbase + (long long)row * p.sr) + half * 8;
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4)
                dst[c4] = make_float4(o[4 * c4] * inv, o[4 * c4 + 1] * inv, o[4 * c4 + 2] * inv, o[4 * c4 + 3] * inv);
        }
    } else if (tid == 0) {
        atomicOr(p.err, NLLB_DEV_ERR_TIMEOUT);
        // let what is still in flight land (MMAs, TMA boxes): each barrier's
        // armed phases not waited for yet, oldest first
        for (; phase < mma_issued; ++phase) (void)mbar_wait_bounded(mma_bar, phase & 1u);
        for (; qk_phase < qk_issued; ++qk_phase) (void)mbar_wait_bounded(qk_bar, qk_phase & 1u);
        for (; v_phase < v_issued; ++v_phase) (void)mbar_wait_bounded(v_bar, v_phase & 1u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TC_TMEM_COLS);
    }
}

// The score matrix of attention_head (tensor.c:258-277): row i holds
// softmax_j((q_i . k_j) * scale + mask[i][j]) over j < S, the max subtracted
// before the exponentials (softmax, tensor.c:227-238).  One CTA per row;
// q, k: [S][64], mask [S][S] or null, p: [S][S].
__global__ void __launch_bounds__(256) head_scores_kernel(const float* q, const float* k, const float* mask,
                                                          float* p, int S, float scale) {
    __shared__ float qs[64];
    __shared__ float red[8];
    const int i = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < 64) qs[tid] = q[(size_t)i * 64 + tid];
    __syncthreads();
    float* row = p + (size_t)i * S;
    float mx = -INFINITY;
    for (int j = tid; j < S; j += blockDim.x) {
        const float4* kj = reinterpret_cast<const float4*>(k + (size_t)j * 64);
        float dot = 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            const float4 kv = kj[c];
            dot = fmaf(qs[4 * c], kv.x, dot);
            dot = fmaf(qs[4 * c + 1], kv.y, dot);
            dot = fmaf(qs[4 * c + 2], kv.z, dot);
            dot = fmaf(qs[4 * c + 3], kv.w, dot);
        }
        float sc = dot * scale;
        if (mask) sc += mask[(size_t)i * S + j];
        row[j] = sc;
        mx = fmaxf(mx, sc);
    }
    auto block_reduce = [&](float v, bool is_max) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? fmaxf(v, w) : v + w;
        }
        __syncthreads();
        if (lane == 0) red[warp] = v;
        __syncthreads();
        float t = red[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = is_max ? fmaxf(t, red[w]) : t + red[w];
        return t;
    };
    mx = block_reduce(mx, true);
    float sum = 0.f;
    for (int j = tid; j < S; j += blockDim.x) {
        const float e = expf(row[j] - mx);
        row[j] = e;
        sum += e;
    }
    sum = block_reduce(sum, false);
    const float inv = 1.0f / sum;
    for (int j = tid; j < S; j += blockDim.x) row[j] *= inv;
}

}  // namespace

cudaError_t launch_head_scores(const float* q, const float* k, const float* mask, float* p, int S, float scale,
                               cudaStream_t st) {
    if (S <= 0) return cudaSuccess;
    head_scores_kernel<<<S, 256, 0, st>>>(q, k, mask, p, S, scale);
    return cudaGetLastError();
}

// The fp32 tensor map of q, k or v for the tensor-core kernel: 4-D, column
// (64, contiguous) first, then the row, head and sequence axes in the order
// of their strides, box [32 columns][128 rows], 128-byte swizzle.  Rows
// outside the tensor read as zeros.  False where the layout does not fit a
// tensor map (overlapping or zero strides): the SIMT kernel runs instead.
bool prefill_map(const PrefillParams& p, const float* base, CUtensorMap* map, int pos[3]) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return false;
    struct Axis {
        long long stride, extent;
        int which;  // 0 row, 1 head, 2 sequence
    } ax[3] = {{p.sr, p.row_start ? (long long)p.rows_total : (long long)p.S, 0},
               {p.sh, p.H, 1},
               {p.sb, p.row_start ? 1LL : (long long)p.B, 2}};
    // axes of extent 1 go last, with a stride that keeps the strides ordered
    std::sort(ax, ax + 3, [](const Axis& x, const Axis& y) {
        if ((x.extent == 1) != (y.extent == 1)) return y.extent == 1;
        return x.stride < y.stride;
    });
    long long span = 64;  // elements covered by the axes so far
    cuuint64_t dims[4] = {64, 1, 1, 1}, strides[3];
    cuuint32_t box[4] = {32, 1, 1, 1}, estr[4] = {1, 1, 1, 1};
    for (int i = 0; i < 3; ++i) {
        long long st = ax[i].stride;
        if (ax[i].extent == 1) st = std::max(st, span);
        if (ax[i].extent < 1 || st < span || st % 4) return false;
        dims[i + 1] = (cuuint64_t)ax[i].extent;
        strides[i] = (cuuint64_t)st * 4;
        span = st * ax[i].extent;
        pos[ax[i].which] = i;
        if (ax[i].which == 0) box[i + 1] = 128;
    }
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t configure_prefill_kernels() {
    const int smem = 4 * BQ * LDS * (int)sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(prefill_ffma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
}

bool prefill_uses_tensor_cores(int seq_len) { return seq_len > 32 && seq_len <= TC_MAX_S; }

cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = kPdlLaunch;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cfg.stream = st;
    cfg.blockDim = dim3(128, 1, 1);
    if (prefill_uses_tensor_cores(p.S)) {
        PrefillParams q = p;
        CUtensorMap mq, mk, mv;
        int pos[3], pos_k[3], pos_v[3];
        if (prefill_map(p, p.q, &mq, pos) && prefill_map(p, p.k, &mk, pos_k) && prefill_map(p, p.v, &mv, pos_v)) {
            q.map_pos_row = pos[0] + 0;
            q.map_pos_head = pos[1];
            q.map_pos_seq = pos[2];
            cfg.blockDim = dim3(TC_THREADS, 1, 1);
            cfg.gridDim = dim3((p.S + TC_Q - 1) / TC_Q, p.H, p.B);
            cfg.dynamicSmemBytes = TC_SMEM;
            return cudaLaunchKernelEx(&cfg, prefill_tc_kernel, q, mq, mk, mv);
        }
    }
    cfg.gridDim = dim3((p.S + BQ - 1) / BQ, p.H, p.B);
    cfg.dynamicSmemBytes = 4 * BQ * LDS * sizeof(float);
    return cudaLaunchKernelEx(&cfg, prefill_ffma_kernel, p);
}

}  // namespace nllb
