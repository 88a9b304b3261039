// prefill.cu -- encoder self-attention prefill, fp32 (sm_100a).
//
// Two kernels compute attention_head_flash (tensor.c:286-332) /
// encoder.c:166-205 for every (sequence, head, query row):
//
// prefill_tc_kernel (seq_len 33..256): 5th-generation tensor cores.  One CTA
//   per (128-query tile, head, sequence) with 8 warps: query row r is TMEM
//   lane r, owned by two threads (warps w and w+4 reach the same lane quarter)
//   that take alternate 32-key halves of every 64 keys.  Q, K and V arrive by
//   TMA as fp32 and are split into two fp16 parts each (x = hi + lo, hi
//   rounded to 11 significant bits, lo the rest); every product is taken as hi*hi' + hi*lo' +
//   lo*hi' on tcgen05.mma kind::f16 with fp32 accumulation in TMEM, which keeps
//   fp32 accuracy for |q|, |k|, |v| < 65504.  The softmax is the reference's
//   two-pass form: all scores of a row sit in TMEM (256 columns), pass 1
//   takes the row max, pass 2 forms P = exp(s - max) per 128-key group
//   (scaled by 2^15 before its split), stages its parts in shared memory and
//   accumulates O += P.V in TMEM with V read as an MN-major operand (no
//   transpose); the row sum is divided out at the end.
// prefill_ffma_kernel (other lengths): SIMT fp32 flash attention with an
//   online softmax over 64-key tiles.
#include <algorithm>

#include "device_common.cuh"
#include "kernels.h"
#include "planes.cuh"

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
constexpr int TC_Q = 128;        // queries per CTA (MMA M)
constexpr int TC_KG = 128;       // keys per group: N of the score MMAs, K of a group's P.V MMAs
constexpr int TC_MAX_S = 256;    // score columns held in TMEM
constexpr uint32_t TC_TMEM_COLS = 512;
// P is scaled by 2^15 before its split so that weights down to ~2e-9 keep
// both fp16 parts normal; the output is scaled back exactly.
constexpr float kPScale = 32768.0f, kPUnscale = 1.0f / 32768.0f;
// Shared-memory plan (bytes from a 1024-byte aligned base).  TMA lands fp32
// tiles as [rows][32 fp32] boxes (128-byte swizzle); the threads split them
// into the fp16 MMA operands, K-major with the 128-byte swizzle: rows of 64
// fp16 (128 B), 8-row atoms 1024 B apart.
constexpr uint32_t SQF = 0, SKF = 32768;        // Q, K group fp32 staging, 2 boxes each
constexpr uint32_t SPP = 0;                     // P parts [2][2 k-blocks][128 rows][128 B] over SQF/SKF
constexpr uint32_t SVF = 65536;                 // V group fp32 staging, 2 boxes
constexpr uint32_t SQP = 98304;                 // Q parts [2][128 rows][128 B]
constexpr uint32_t SKP = 131072;                // K group parts [2][128 keys][128 B]
constexpr uint32_t SVP = 163840;                // V group parts [2][128 keys][128 B] (MN-major B)
constexpr uint32_t SBAR = 196608;
constexpr uint32_t TC_SMEM = SBAR + 64 + 1024;  // + alignment slack
constexpr uint32_t TC_BOX_BYTES = 128 * 128;    // one [128 rows][32 fp32] box
constexpr uint32_t PART16 = 16384;              // one fp16 part of a [128][64] operand
constexpr uint32_t P_PART = 32768;              // one fp16 part of P ([128 queries][128 keys])

// byte offset of (row, col) in an fp32 [nrows][64] tile as TMA lands it:
// 32-column boxes of nrows*128 B, 128-B rows, 16-B chunks XOR-ed with row % 8.
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int nrows) {
    return (uint32_t)((col >> 5) * nrows * 128 + row * 128 + ((((col & 31) >> 2) ^ (row & 7)) << 4) +
                      ((col & 3) << 2));
}

// byte offset of the 16-byte chunk holding fp16 elements k .. k+7 (k % 8 == 0)
// of row `row` in a K-major 128-byte-swizzled fp16 operand of `nrows` rows:
// 64-element k-blocks of nrows*128 B.
__device__ __forceinline__ uint32_t sw128_f16_chunk(int row, int k, int nrows) {
    return (uint32_t)((k >> 6) * nrows * 128 + row * 128 + ((((k & 63) >> 3) ^ (row & 7)) << 4));
}

// fp32 -> two fp16 parts x = hi + lo, packed in pairs: hi = x rounded to 11
// significant bits in fp32 (exact in fp16), lo = x - hi (exact in fp32, then
// rounded to fp16: |x - hi - lo| <= 2^-23 |x| for |x| in fp16's normal
// range).  Two packed conversions per pair of values instead of six scalar
// ones: the conversion pipe, not the math, bounds these splits.
__device__ __forceinline__ float round11(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ void split8(const float (&x)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = round11(x[2 * i]), b = round11(x[2 * i + 1]);
        const __half2 hh = __floats2half2_rn(a, b);  // .x (low half) = element 2i
        const __half2 ll = __floats2half2_rn(x[2 * i] - a, x[2 * i + 1] - b);
        h[i] = *reinterpret_cast<const uint32_t*>(&hh);
        l[i] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// A [128 rows][64 fp32] tile staged by TMA at src -> its two fp16 parts at
// dst and dst + PART16 ([128 rows][64], 128-byte swizzle: K-major for Q and
// K, MN-major for V).  Rows >= valid are zero.
__device__ __forceinline__ void split_rows64(const unsigned char* src, unsigned char* dst, int valid, int tid) {
#pragma unroll
    for (int it = 0; it < (128 * 8) / TC_THREADS; ++it) {
        const int item = tid + it * TC_THREADS;
        const int row = item >> 3, k = (item & 7) * 8;
        float x[8];
        const float4 a = *reinterpret_cast<const float4*>(src + sw128_off(row, k, 128));
        const float4 b = *reinterpret_cast<const float4*>(src + sw128_off(row, k + 4, 128));
        x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
        if (row >= valid) {
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = 0.f;
        }
        uint4 hi, lo;
        split8(x, hi, lo);
        const uint32_t o = sw128_f16_chunk(row, k, 128);
        *reinterpret_cast<uint4*>(dst + o) = hi;
        *reinterpret_cast<uint4*>(dst + PART16 + o) = lo;
    }
}

// D[128 x N] (+)= (A0 + A1)[128 x K] . (B0 + B1)^T as A0.B0 + A0.B1 + A1.B0
// over K / 16 k-steps (fp16 parts, fp32 accumulation; A1.B1 is below the
// fp32 rounding of the sum).  A is K-major with the 128-byte swizzle: a0
// addresses the first 64-element k-block of part 0, a_part the distance to
// part 1, a_kb between k-blocks.  B is either K-major like A ([N rows][K],
// b_kb between k-blocks) or, with B_MN, MN-major: [K rows][N = 64 elements],
// one 128-byte swizzled row per k, so a k-step of 16 is 2048 bytes.
template <int N, int K, bool B_MN>
__device__ __forceinline__ void mma_2part(uint32_t d, uint32_t a0, uint32_t a_part, uint32_t a_kb, uint32_t b0,
                                          uint32_t b_part, uint32_t b_kb, bool accumulate_first) {
    static_assert(!B_MN || N == 64, "an MN-major B operand here is one 64-element row per k");
    constexpr uint32_t idesc = umma_idesc_f16(128, N) | (B_MN ? (1u << 16) : 0u);  // bit 16: B is MN-major
#pragma unroll
    for (int ks = 0; ks < K / 16; ++ks) {
        const uint32_t ao = (ks >> 2) * a_kb + (ks & 3) * 32;
        const uint32_t bo = B_MN ? (uint32_t)ks * 2048u : (ks >> 2) * b_kb + (ks & 3) * 32;
        const uint64_t da0 = umma_desc_k_sw128(a0 + ao), da1 = umma_desc_k_sw128(a0 + a_part + ao);
        const uint64_t db0 = umma_desc_k_sw128(b0 + bo), db1 = umma_desc_k_sw128(b0 + b_part + bo);
        tc_mma_f16(d, da0, db0, idesc, (accumulate_first || ks > 0) ? 1u : 0u);
        tc_mma_f16(d, da0, db1, idesc, 1u);
        tc_mma_f16(d, da1, db0, idesc, 1u);
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

__device__ __forceinline__ float ex2_approx(float x) {  // 2^x, -inf -> +0
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// One CTA per (128-query tile, head, sequence), 8 warps.  Q, K and V tiles
// arrive by TMA as fp32 (one thread issues the boxes after the wait on the
// previous kernel); the threads split them into two fp16 parts each, and
// every product runs as three kind::f16 MMAs with fp32 accumulation in TMEM.
// Scores go to TMEM in groups of 128 keys (the next group's K loads while a
// group is split); V's parts are made while the score MMAs run; the softmax
// is the two-pass form (row max, then P = exp(s - max) per 128-key group,
// split into parts and accumulated as O += P.V with V an MN-major operand).
__global__ void __launch_bounds__(TC_THREADS, 1) prefill_tc_kernel(const PrefillParams p,
                                                                   const __grid_constant__ CUtensorMap map_q,
                                                                   const __grid_constant__ CUtensorMap map_k,
                                                                   const __grid_constant__ CUtensorMap map_v) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
    unsigned char* base = smem_raw + (base_addr - raw_addr);
    uint64_t* mma_bar = reinterpret_cast<uint64_t*>(base + SBAR);
    uint64_t* k_bar = reinterpret_cast<uint64_t*>(base + SBAR + 8);   // K group loads
    uint64_t* v_bar = reinterpret_cast<uint64_t*>(base + SBAR + 16);  // V group loads
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + SBAR + 24);
    volatile int* s_abort = reinterpret_cast<volatile int*>(base + SBAR + 32);
    uint64_t* q_bar = reinterpret_cast<uint64_t*>(base + SBAR + 40);  // the Q load
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
        mbar_init(q_bar, 1);
        mbar_init(k_bar, 1);
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
    const int n_kg = (kv_len + TC_KG - 1) / TC_KG;  // key groups of 128 (at most 2)
    const int rloc = quarter * 32 + lane;           // query row within the tile = TMEM lane
    const int row = q0 + rloc;
    const float* mrow = (p.mask && row < S)
                            ? p.mask + (long long)b * p.msb + (long long)h * p.msh + (long long)row * S
                            : nullptr;
    const float sl2 = p.scale_log2;

    // Q, K group 0 and V group 0: every box issued at once, Q on its own
    // barrier so that its split overlaps K's arrival.  A box counts its full
    // bytes toward the barrier, rows outside the tensor included (they arrive
    // as zeros).
    if (tid == 0) {
        mbar_arrive_expect_tx(q_bar, 2 * TC_BOX_BYTES);
        tma_rows128(base_addr + SQF, &map_q, p, row0 + q0, h, bq, q_bar);
        mbar_arrive_expect_tx(k_bar, 2 * TC_BOX_BYTES);
        tma_rows128(base_addr + SKF, &map_k, p, row0, h, bq, k_bar);
        mbar_arrive_expect_tx(v_bar, 2 * TC_BOX_BYTES);
        tma_rows128(base_addr + SVF, &map_v, p, row0, h, bq, v_bar);
    }

    uint32_t phase = 0, q_phase = 0, k_phase = 0, v_phase = 0;  // waits completed per barrier
    uint32_t mma_issued = 0, k_issued = 1, v_issued = 1;        // (thread 0) phases armed per barrier
    auto wait_bar = [&](uint64_t* bar, uint32_t& ph) -> bool {
        if (!mbar_wait_bounded(bar, ph & 1u)) *s_abort = 1;
        ++ph;
        __syncthreads();
        return *s_abort == 0;
    };
    // 32 scores (base-2 logits) of this thread's row, keys j0..j0+31
    // 32 scores (base-2 logits) of this thread's row at keys j0..j0+31 and at
    // j1..j1+31, both TMEM loads under one wait; keys at or past the length
    // (and columns no MMA wrote) become -inf
    auto scores32x2 = [&](int j0, int j1, float* v0, float* v1) {
        tmem_ld32x2(tS + (uint32_t)j0, tS + (uint32_t)j1, v0, v1);
        auto fix = [&](int jb, float* v) {
            if (uniform) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = (jb + i < kv_len) ? 0.f : -INFINITY;
            } else if (mrow) {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    v[i] = (jb + i < kv_len) ? fmaf(__ldg(mrow + jb + i), kLog2e, v[i] * sl2) : -INFINITY;
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = (jb + i < kv_len) ? v[i] * sl2 : -INFINITY;
            }
        };
        fix(j0, v0);
        fix(j1, v1);
    };

    // ---- scores S = Q.K^T, group g in TMEM columns [128 g, 128 g + 128)
    bool ok = wait_bar(q_bar, q_phase);  // Q has landed
    if (ok) split_rows64(base + SQF, base + SQP, TC_Q, tid);
    for (int g = 0; g < n_kg && ok; ++g) {
        if (g > 0 && !(ok = wait_bar(mma_bar, phase))) break;  // group g-1's MMAs have read the K parts
        if (!(ok = wait_bar(k_bar, k_phase))) break;           // K group g has landed
        split_rows64(base + SKF, base + SKP, TC_KG, tid);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();  // the parts are visible to the tensor core, the K staging is free
        if (tid == 0) {
            if (g + 1 < n_kg) {
                mbar_arrive_expect_tx(k_bar, 2 * TC_BOX_BYTES);
                tma_rows128(base_addr + SKF, &map_k, p, row0 + (g + 1) * TC_KG, h, bq, k_bar);
                ++k_issued;
            }
            tc_fence_after();
            mma_2part<TC_KG, 64, false>(tmem + (uint32_t)(g * TC_KG), base_addr + SQP, PART16, 0, base_addr + SKP,
                                        PART16, 0, false);
            tc_commit(mma_bar);
            ++mma_issued;
        }
    }
    // ---- V group 0's parts while the score MMAs run; the staging then takes group 1
    if (ok && (ok = wait_bar(v_bar, v_phase))) {
        split_rows64(base + SVF, base + SVP, kv_len, tid);
        __syncthreads();  // every thread is done reading the V staging
        if (tid == 0 && n_kg > 1) {
            mbar_arrive_expect_tx(v_bar, 2 * TC_BOX_BYTES);
            tma_rows128(base_addr + SVF, &map_v, p, row0 + TC_KG, h, bq, v_bar);
            ++v_issued;
        }
    }
    if (ok) ok = wait_bar(mma_bar, phase);  // scores in TMEM; the Q and K staging is free (P goes there)
    tc_fence_after();

    // pass 1: row max (this thread: columns half*32 + 64c .. +31 of every 64-key chunk)
    float mx = -INFINITY;
    if (ok) {
        const int n_kc = (kv_len + 63) / 64;  // 64-key chunks, two per load (TMEM columns < 256)
        for (int kc = 0; kc < n_kc; kc += 2) {
            float v0[32], v1[32];
            scores32x2(kc * 64 + half * 32, kc * 64 + 64 + half * 32, v0, v1);
#pragma unroll
            for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fmaxf(v0[i], v1[i]));
        }
        s_red[tid] = mx;
    }
    __syncthreads();
    if (ok) mx = fmaxf(mx, s_red[tid ^ 128]);

    // pass 2, per key group: P = exp(s - max) (keys past the length give 0),
    // scaled and split into parts, then O += P.V
    float sum = 0.f;
    for (int g = 0; g < n_kg && ok; ++g) {
        if (g > 0) {
            if (!(ok = wait_bar(mma_bar, phase))) break;  // group g-1's P.V MMAs have read P and V's parts
            if (!(ok = wait_bar(v_bar, v_phase))) break;  // V group g has landed
            split_rows64(base + SVF, base + SVP, kv_len - g * TC_KG, tid);
        }
        float vv[2][32];
        scores32x2(g * TC_KG + half * 32, g * TC_KG + 64 + half * 32, vv[0], vv[1]);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int jl = c * 64 + half * 32;  // first key of this thread's 32 within the group
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float x[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float e = ex2_approx(vv[c][q * 8 + i] - mx);
                    sum += e;
                    x[i] = e * kPScale;
                }
                uint4 hi, lo;
                split8(x, hi, lo);
                const uint32_t o = sw128_f16_chunk(rloc, jl + q * 8, TC_Q);
                *reinterpret_cast<uint4*>(base + SPP + o) = hi;
                *reinterpret_cast<uint4*>(base + SPP + P_PART + o) = lo;
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            mma_2part<64, TC_KG, true>(tmem + TC_MAX_S, base_addr + SPP, P_PART, TC_Q * 128, base_addr + SVP, PART16,
                                       0, g > 0);
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
            const float inv = kPUnscale / sum;  // P was scaled by 2^15
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
        for (; q_phase < 1; ++q_phase) (void)mbar_wait_bounded(q_bar, 0u);
        for (; k_phase < k_issued; ++k_phase) (void)mbar_wait_bounded(k_bar, k_phase & 1u);
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
