// linear_tma.cu -- INT8-weight linear layer for the translation engine on
// tcgen05 tensor cores, fed by TMA (sm_100a).
//
// int8 weights are exact in fp16 and fp32 activations are taken as two fp16
// parts x = x1 + x2 (planes.cuh, 22 significant bits): two MMAs per k-step
// (kind::f16), fp32 accumulation in TMEM.  The engine keeps an fp16 copy of
// every weight matrix (converted once at load) and the producers of the
// activations write them as planes (LayerNorm, the attention kernels, the
// previous GEMM's epilogue; split_planes_kernel otherwise), so the GEMM's
// operands are plain fp16 matrices that TMA tensor maps load straight into
// swizzled shared memory.
//
// CTA: warps 0-7 epilogue, warp 8 lane 0 TMA producer, warp 9 lane 0 MMA
// issuer; 128 x 128 output tile; K in stages of 64 (2 X planes + W = 48 KB
// per stage, 3 stages).  Split-K over a thread-block cluster along x: the S
// CTAs of a tile each leave their 128 x 128 partial sum in shared memory and
// cluster rank z reduces rows [z*128/S, (z+1)*128/S) over all S partials in
// rank order (distributed shared memory; deterministic; no workspace).
// Grid x = (row tile, split) fastest, so the row tiles that share a weight
// tile run together and the weight tile is read from DRAM once.
//
// Larger outputs take a persistent kernel over 128 x 256 tiles (one CTA per
// SM), or, from 129 rows and two rounds of such tiles per SM, its pair form:
// 256 x 256 tiles on two-CTA clusters with tcgen05.mma.cta_group::2, each CTA
// loading half of the weight tile.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "device_common.cuh"
#include "engine_kernels.h"
#include "planes.cuh"

namespace nllb {

namespace {

#ifndef NLLB_SPLIT_STAGES
#define NLLB_SPLIT_STAGES 3
#endif
constexpr int TM = 128, TN = 128, TK = 64, STAGES = NLLB_SPLIT_STAGES;
constexpr int EPI_WARPS = 8, THREADS = (EPI_WARPS + 2) * 32;
constexpr uint32_t PLANE = TM * TK * 2;                 // 16 KB
constexpr uint32_t W_OFF = kPlanes * PLANE;             // the weight tile follows the X planes
constexpr uint32_t STAGE_BYTES = (kPlanes + 1) * PLANE;  // x1, x2, w
constexpr uint32_t SMEM_BAR = STAGES * STAGE_BYTES;
constexpr uint32_t SMEM_TOTAL = SMEM_BAR + 128 + 1024;
constexpr uint32_t TMEM_COLS = 128;
constexpr int PART_STRIDE = TN + 4;  // floats per row of the partial tile in shared memory
// the partial tile and, behind it, the rows the other ranks send (fewer than TM)
static_assert(2 * TM * PART_STRIDE * 4 <= SMEM_BAR, "the partial tile and the received rows overlay the stage ring");
// dynamic shared memory a launch may take: the 227 KB of a CTA less the static per-column factors
constexpr uint32_t kSplitSmemMax = 232448 - 2 * TN * 4;
static_assert(SMEM_TOTAL <= kSplitSmemMax, "fits the 227 KB of shared memory a CTA may use");


__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// 16-byte asynchronous copy global -> shared (no registers), and its completion
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ uint32_t dynamic_smem_bytes() {
    uint32_t r;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
    return r;
}

// Bulk copy from this CTA's shared memory into another CTA's of the cluster
// (dst and bar: shared::cluster addresses there), completing on that CTA's
// barrier.  16-byte aligned addresses, bytes a multiple of 16.
__device__ __forceinline__ void bulk_s2s_cluster(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "r"(smem_u32(src)), "r"(bytes), "r"(bar)
        : "memory");
}

// y = accumulator / scale[n] (the per-column dequantisation factor of tensor.c:75)
__device__ __forceinline__ void epilogue_store(const LinearArgs& a, int m, int n, float y) {
    if (a.bias) y += a.bias[n];
    if (a.relu) y = fmaxf(y, 0.f);
    if (a.mask_from >= 0 && n >= a.mask_from) y = -1e30f;
    const size_t o = (size_t)(n / a.cblock) * ((size_t)a.M * a.cblock) + (size_t)m * a.cblock + (n % a.cblock);
    if (a.residual) y += a.residual[o];
    if (a.out_planes)
        store_planes_x1(static_cast<plane_t*>(a.out_planes), (size_t)a.M * a.N, o, y);
    else
        a.out[o] = y;
}

__global__ void __launch_bounds__(THREADS, 1)
    linear_tma_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
                      const LinearArgs a, int splits, int* err) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base_addr = (raw + 1023u) & ~1023u;
    unsigned char* base = smem_raw + (base_addr - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + SMEM_BAR);
    uint64_t* empty = full + STAGES;
    uint64_t* done = empty + STAGES;
    uint64_t* never = done + 1;  // test_expire: a barrier nothing arrives on
    uint64_t* recv = never + 1;  // split-K: the other ranks' rows of this rank's share have landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv + 1);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);
    __shared__ __align__(16) float s_inv[TN];
    __shared__ __align__(16) float s_bias[TN];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = splits, z = blockIdx.x % S, mt = blockIdx.x / S;
    const int m0 = mt * TM, n0 = blockIdx.y * TN;
    const int nk_all = a.K / TK;
    const int kc0 = (int)((long long)z * nk_all / S), kc1 = (int)((long long)(z + 1) * nk_all / S);
    const int nk = kc1 - kc0;

    if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        mbar_init(never, 1);
        mbar_init(recv, 1);
        fence_barrier_init();
        *s_abort = 0;
    }
    pdl_launch_dependents();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool producer = warp == EPI_WARPS && lane == 0;
    // rows [z*R, (z+1)*R) of the tile are finished by this rank
    const int R = TM / S, r_begin = z * R;
    const bool vec = (a.cblock % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(a.residual) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(a.bias) & 15) == 0);
    // The residual rows of this rank's share are copied into shared memory
    // (behind the stage ring, when the launch gave the room) by the epilogue
    // warps while the MMAs run, instead of being loaded after them.
    float* res_s = reinterpret_cast<float*>(base + SMEM_BAR + 128);
    const bool res_pre = a.residual && vec && a.cblock % TN == 0 && n0 + TN <= a.N &&
                         (base_addr - raw) + SMEM_BAR + 128 + (uint32_t)R * TN * 4 <= dynamic_smem_bytes();
    if (!producer) {
        pdl_wait_primary();  // the output may still be read by earlier kernels
        if (res_pre && warp < EPI_WARPS) {
            const size_t tb = (size_t)(n0 / a.cblock) * ((size_t)a.M * a.cblock) + (n0 % a.cblock);
            for (int i = tid; i < R * (TN / 4); i += EPI_WARPS * 32) {
                const int rr = i / (TN / 4), q = i % (TN / 4), m = m0 + r_begin + rr;
                if (m < a.M) cp_async16(res_s + rr * TN + q * 4, a.residual + tb + (size_t)m * a.cblock + q * 4);
            }
        }
        if (tid < TN) s_inv[tid] = (n0 + tid < a.N) ? 1.0f / a.scale[n0 + tid] : 0.f;  // 1/scale as tensor.c:75
        else if (tid < 2 * TN)
            s_bias[tid - TN] = (a.bias && n0 + tid - TN < a.N) ? a.bias[n0 + tid - TN] : 0.f;
    }

    if (producer) {
        // ---- TMA producer.  The model's weights do not depend on earlier
        // kernels: the first stages' weight tiles go out before waiting for
        // the previous kernel, whose output (the planes) is loaded after.
        prefetch_tensormap(&tx);
        prefetch_tensormap(&tw);
        const int pre = nk < STAGES ? nk : STAGES;
        if (a.static_weights)
            for (int c = 0; c < pre; ++c) {
                mbar_arrive_expect_tx(&full[c], STAGE_BYTES);
                tma_load_2d(base + c * STAGE_BYTES + W_OFF, &tw, (kc0 + c) * TK, n0, &full[c]);
            }
        pdl_wait_primary();
        for (int c = 0; c < pre; ++c) {
            unsigned char* st = base + c * STAGE_BYTES;
            if (!a.static_weights) {
                mbar_arrive_expect_tx(&full[c], STAGE_BYTES);
                tma_load_2d(st + W_OFF, &tw, (kc0 + c) * TK, n0, &full[c]);
            }
            tma_load_3d(st, &tx, (kc0 + c) * TK, m0, 0, &full[c]);  // box 64 x 128 x 2: the planes
        }
        for (int c = pre; c < nk; ++c) {
            const int s = c % STAGES;
            if (c >= STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)((c / STAGES - 1) & 1))) {
                atomicExch(s_abort, 1);
                break;
            }
            unsigned char* st = base + s * STAGE_BYTES;
            const int k = (kc0 + c) * TK;
            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            tma_load_3d(st, &tx, k, m0, 0, &full[s]);  // box 64 x 128 x 2: the planes
            tma_load_2d(st + W_OFF, &tw, k, n0, &full[s]);
        }
    } else if (warp == EPI_WARPS + 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = umma_idesc_f16(TM, TN);
        // test of the bounded waits: this one runs out after ~1 ms, no MMA is
        // issued and `done` never fires, so the producer's and the epilogue's
        // waits run out in turn and the launch writes nothing
        const bool expired = a.test_expire && !mbar_wait_bounded(never, 0u, kTestWaitBudgetCycles);
        if (expired) atomicExch(s_abort, 1);
        for (int c = 0; c < nk && !expired; ++c) {
            const int s = c % STAGES;
            if (!mbar_wait_bounded(&full[s], (uint32_t)((c / STAGES) & 1))) {
                atomicExch(s_abort, 1);
                break;
            }
            tc_fence_after();
            const uint32_t st = base_addr + s * STAGE_BYTES;
#pragma unroll
            for (int ks = 0; ks < TK / 16; ++ks) {
                const uint64_t bw = umma_desc_k_sw128(st + W_OFF + ks * 32);
                tc_mma_f16(tmem, umma_desc_k_sw128(st + 0 * PLANE + ks * 32), bw, idesc, (c > 0 || ks > 0) ? 1u : 0u);
                tc_mma_f16(tmem, umma_desc_k_sw128(st + 1 * PLANE + ks * 32), bw, idesc, 1u);
            }
            tc_commit(&empty[s]);
        }
        tc_commit(done);
    }

    // ---- accumulator -> shared memory (two threads per row, 64 columns each)
    float* part = reinterpret_cast<float*>(base);  // the stage ring is idle once `done` has fired
    if (warp < EPI_WARPS) {
        const int quarter = warp & 3, half = (warp >> 2) & 1;
        const int rloc = quarter * 32 + lane;
        const bool ok = mbar_wait_bounded(done, 0u);
        tc_fence_after();
        if (!ok) {
            atomicExch(s_abort, 1);
        } else {
            float v[64];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * 64), v);
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * 64 + 32), v + 32);
            float4* row = reinterpret_cast<float4*>(part + rloc * PART_STRIDE + half * 64);
#pragma unroll
            for (int j = 0; j < 16; ++j) row[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        if (res_pre) cp_async_wait_all();  // this thread's residual copies (the barrier below shares them)
    }
    // ---- split-K: every rank sends the rows of its partial tile that rank d
    // finishes to rank d (one bulk shared-to-shared copy per pair, into the
    // idle stage ring behind the partial tile); the first sent row's padding
    // column carries the sender's abort flag
    const uint32_t slot_bytes = (uint32_t)R * PART_STRIDE * 4;
    float* recv_buf = part + TM * PART_STRIDE;  // [S-1][R][PART_STRIDE]: from ranks 0..S-1 without z
    if (S == 1) {
        __syncthreads();
    } else {
        fence_async_smem();  // the partial tile's generic writes, seen by the copies
        if (tid == 0) mbar_arrive_expect_tx(recv, (uint32_t)(S - 1) * slot_bytes);
        cluster_sync_all();  // every rank's partial tile written and its receive barrier armed
        if (tid == 0) {
            const int my_abort = *(volatile int*)s_abort;  // final: the producer and MMA threads are done
            for (int d = 0; d < S; ++d) {
                if (d == (int)z) continue;
                float* rows = part + d * R * PART_STRIDE;
                rows[TN] = __int_as_float(my_abort);
                fence_async_smem();
                const int slot = z < d ? z : z - 1;  // this rank's slot at rank d
                bulk_s2s_cluster(map_rank(recv_buf + (size_t)slot * R * PART_STRIDE, d), rows, slot_bytes,
                                 map_rank(recv, d));
            }
        }
        if (!mbar_wait_bounded(recv, 0u)) atomicExch(s_abort, 1);
    }

    // ---- rank z finishes rows [z*R, (z+1)*R) of the tile: sum of the S partials
    // in rank order, epilogue, coalesced stores (one warp per 128-column row)
    int aborted = *(volatile int*)s_abort;
    for (int r = 0; r < S - 1; ++r) aborted |= __float_as_int(recv_buf[(size_t)r * R * PART_STRIDE + TN]);
    // the partial of rank r for row rr of this rank's share
    auto part_row = [&](int r, int rr) -> const float* {
        return r == (int)z ? part + (z * R + rr) * PART_STRIDE
                           : recv_buf + ((size_t)(r < (int)z ? r : r - 1) * R + rr) * PART_STRIDE;
    };
    if (aborted) {
        if (tid == 0) atomicOr(err, NLLB_DEV_ERR_TIMEOUT);
    } else {
        if (vec && a.cblock % TN == 0) {
            // A warp stores one 128-column row as float4s.  THREADS is a
            // multiple of the 32 float4 of a row, so a thread keeps one column
            // quad (its factors, bias and mask loaded once) and walks rows
            // THREADS / 32 apart, kU rows per pass with every load of the pass
            // issued before its first store.  The tile lies in one column
            // block, whose offset is found once.
            static_assert(THREADS % (TN / 4) == 0, "a thread keeps one column quad");
            constexpr int kU = 4, kRowStep = THREADS / (TN / 4);
            const int c4 = tid % (TN / 4), nl = c4 * 4, n = n0 + nl;
            const size_t tile_off = (size_t)(n0 / a.cblock) * ((size_t)a.M * a.cblock) + (n0 % a.cblock) + nl;
            const float4 inv = *reinterpret_cast<const float4*>(s_inv + nl);
            const float4 bias = a.bias ? *reinterpret_cast<const float4*>(s_bias + nl) : make_float4(0.f, 0.f, 0.f, 0.f);
            const bool full4 = n + 3 < a.N;
            bool masked[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) masked[j] = a.mask_from >= 0 && n + j >= a.mask_from;
            for (int r0 = tid / (TN / 4); r0 < R; r0 += kRowStep * kU) {
                float4 acc[kU], res[kU];
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int rr = r0 + u * kRowStep;  // row within this rank's share
                    const int m = m0 + z * R + rr;
                    const bool live = rr < R && m < a.M;
                    const int rl = live ? rr : 0;
                    acc[u] = *reinterpret_cast<const float4*>(part_row(0, rl) + nl);
                    for (int r = 1; r < S; ++r) {  // rank order: the sum is the same on every run
                        const float4 q = *reinterpret_cast<const float4*>(part_row(r, rl) + nl);
                        acc[u].x += q.x, acc[u].y += q.y, acc[u].z += q.z, acc[u].w += q.w;
                    }
                    res[u] = (a.residual && live && full4)
                                 ? (res_pre ? *reinterpret_cast<const float4*>(res_s + rr * TN + nl)
                                            : *reinterpret_cast<const float4*>(a.residual + tile_off +
                                                                               (size_t)m * a.cblock))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int rr = r0 + u * kRowStep;
                    const int m = m0 + z * R + rr;
                    if (rr >= R || m >= a.M) continue;
                    float y[4] = {acc[u].x * inv.x, acc[u].y * inv.y, acc[u].z * inv.z, acc[u].w * inv.w};
                    if (full4) {
                        if (a.bias) y[0] += bias.x, y[1] += bias.y, y[2] += bias.z, y[3] += bias.w;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            if (a.relu) y[j] = fmaxf(y[j], 0.f);
                            if (masked[j]) y[j] = -1e30f;
                        }
                        if (a.residual) y[0] += res[u].x, y[1] += res[u].y, y[2] += res[u].z, y[3] += res[u].w;
                        const size_t o = tile_off + (size_t)m * a.cblock;
                        const float4 yv = make_float4(y[0], y[1], y[2], y[3]);
                        if (a.out_planes) {
                            store_planes_x4(static_cast<plane_t*>(a.out_planes), (size_t)a.M * a.N, o, yv);
                        } else {
                            *reinterpret_cast<float4*>(a.out + o) = yv;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (n + j < a.N) epilogue_store(a, m, n + j, y[j]);
                    }
                }
            }
        } else {
            // a warp stores 32 consecutive columns of one row per instruction
            for (int item = tid; item < R * TN; item += THREADS) {
                const int rl = item / TN, nl = item % TN;
                const int m = m0 + z * R + rl, n = n0 + nl;
                if (m >= a.M) break;
                if (n >= a.N) continue;
                float acc = part_row(0, rl)[nl];
                for (int r = 1; r < S; ++r) acc += part_row(r, rl)[nl];  // rank order
                epilogue_store(a, m, n, acc * s_inv[nl]);
            }
        }
    }
    if (S > 1) cluster_sync_all();  // partners keep their partials until every rank is done reading
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Persistent form for outputs with at least one 128 x 256 tile per SM: one CTA
// per SM walks tiles t = blockIdx.x, + gridDim.x, ... (row tile fastest, so
// CTAs running at the same time share a weight tile in L2).  Warp 0 lane 0
// streams 32-wide K chunks (2 planes 8 KB + weight 16 KB, 64-byte swizzle)
// through a 5-stage ring, warp 1 lane 0 issues 128 x 256 x 16 MMAs into one
// of two TMEM accumulators (2 x 256 columns), and warps 2-9 drain the other
// accumulator meanwhile: TMEM -> registers -> a per-warp transpose buffer ->
// stores of 32 consecutive columns per row.
// ---------------------------------------------------------------------------
namespace pers {
constexpr int TM = 128, TN = 256, TK = 32, STAGES = 5;
constexpr int EPI_WARPS = 8, THREADS = (EPI_WARPS + 2) * 32;
constexpr uint32_t A_PLANE = TM * TK * 2;                // 8 KB
constexpr uint32_t B_BYTES = TN * TK * 2;                // 16 KB
constexpr uint32_t W_OFF = kPlanes * A_PLANE;                 // weight tile after the X planes
constexpr uint32_t STAGE_BYTES = kPlanes * A_PLANE + B_BYTES;  // 32 KB
constexpr int BUF_LD = 33;                               // transpose buffer row stride (floats)
constexpr uint32_t SMEM_EPI = STAGES * STAGE_BYTES;
constexpr uint32_t SMEM_BAR = SMEM_EPI + EPI_WARPS * 32 * BUF_LD * 4;
constexpr uint32_t SMEM_TOTAL = SMEM_BAR + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;
}  // namespace pers

// K-major operand in the 64-byte swizzled layout: rows of 64 B (32 fp16),
// 8-row atoms 512 B apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_k_sw64(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(512u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)4u << 61);
}

// Bounded wait whose outcome every lane of the warp shares (the tcgen05 loads
// that follow are warp-collective).
__device__ __forceinline__ bool warp_wait_bounded(uint64_t* bar, uint32_t parity) {
    const bool ok = mbar_wait_bounded(bar, parity);
    return __all_sync(0xffffffffu, ok);
}

// Epilogue of one 128 x 256 accumulator by one warp: TMEM lanes of rows
// mrow..mrow+31 (taddr: the warp's lane quarter and the accumulator's first
// column), columns n0 + half*128 .. +127, 32 at a time: TMEM -> registers ->
// the warp's transpose buffer (32 x BUF_LD floats) -> stores of 32
// consecutive columns per row, with the per-column factors loaded once.
__device__ __forceinline__ void drain_tile_256(const LinearArgs& a, uint32_t taddr, float* buf, int lane, int half,
                                               int mrow, int n0) {
    constexpr int BUF_LD = pers::BUF_LD;
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
        const int col0 = half * 128 + ch * 32;
        float v[32];
        tmem_ld32(taddr + (uint32_t)col0, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) buf[lane * BUF_LD + j] = v[j];
        __syncwarp();
        // lane = column: per-column factors once, then one row per store
        const int n = n0 + col0 + lane;
        const bool nok = n < a.N;
        const float inv = nok ? 1.0f / a.scale[n] : 0.f;  // 1/scale as tensor.c:75
        const float bias = (nok && a.bias) ? a.bias[n] : 0.f;
        const bool masked = a.mask_from >= 0 && n >= a.mask_from;
        const size_t colbase = nok ? (size_t)(n / a.cblock) * ((size_t)a.M * a.cblock) + (size_t)(n % a.cblock) : 0;
        const int rows = min(32, a.M - mrow);
        if (nok) {
            // The residual may be the output itself (in-place x += f(x)): its
            // 32 rows are all loaded before the first store, so the loads are
            // in flight together instead of one per store.  Each element is
            // still read before it is written.
            float res[32];
            if (a.residual) {
#pragma unroll
                for (int r = 0; r < 32; ++r)
                    res[r] = r < rows ? a.residual[colbase + (size_t)(mrow + r) * a.cblock] : 0.f;
            }
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                if (r >= rows) break;
                float y = buf[r * BUF_LD + lane] * inv;
                if (a.bias) y += bias;
                if (a.relu) y = fmaxf(y, 0.f);
                if (masked) y = -1e30f;
                const size_t o = colbase + (size_t)(mrow + r) * a.cblock;
                if (a.residual) y += res[r];
                if (a.out_planes)
                    store_planes_x1(static_cast<plane_t*>(a.out_planes), (size_t)a.M * a.N, o, y);
                else
                    a.out[o] = y;
            }
        }
        __syncwarp();
    }
}

__global__ void __launch_bounds__(pers::THREADS, 1)
    linear_tma_persistent_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
                                 const LinearArgs a, int* err) {
    constexpr int TM = pers::TM, TN = pers::TN, TK = pers::TK, STAGES = pers::STAGES, EPI_WARPS = pers::EPI_WARPS;
    constexpr int BUF_LD = pers::BUF_LD;
    constexpr uint32_t A_PLANE = pers::A_PLANE, STAGE_BYTES = pers::STAGE_BYTES, SMEM_EPI = pers::SMEM_EPI;
    constexpr uint32_t W_OFF = pers::W_OFF;
    constexpr uint32_t SMEM_BAR = pers::SMEM_BAR, TMEM_COLS = pers::TMEM_COLS;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base_addr = (raw + 1023u) & ~1023u;
    unsigned char* base = smem_raw + (base_addr - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + SMEM_BAR);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int MT = (a.M + TM - 1) / TM, NT = (a.N + TN - 1) / TN;
    const int tiles = MT * NT, nk = a.K / TK;

    if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
    if (tid == 32) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], EPI_WARPS);
        }
        *s_abort = 0;
        fence_barrier_init();
    }
    pdl_launch_dependents();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (!(warp == 0 && lane == 0)) pdl_wait_primary();  // the output may still be read by earlier kernels

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            // the model's weights do not depend on earlier kernels: the first
            // tile's first weight tiles go out before waiting for the planes
            prefetch_tensormap(&tx);
            prefetch_tensormap(&tw);
            const int pre = (int)blockIdx.x < tiles ? (nk < STAGES ? nk : STAGES) : 0;
            if (a.static_weights)
                for (int c = 0; c < pre; ++c) {
                    mbar_arrive_expect_tx(&full[c], STAGE_BYTES);
                    tma_load_2d(base + c * STAGE_BYTES + W_OFF, &tw, c * TK, ((int)blockIdx.x / MT) * TN,
                                &full[c]);
                }
            pdl_wait_primary();
            uint32_t g = 0;
            for (int t = blockIdx.x; t < tiles && !*s_abort; t += gridDim.x) {
                const int m0 = (t % MT) * TM, n0 = (t / MT) * TN;
                for (int c = 0; c < nk; ++c, ++g) {
                    const uint32_t s = g % STAGES, use = g / STAGES;
                    if ((int)g < pre) {  // fresh stage of the first tile
                        unsigned char* st = base + s * STAGE_BYTES;
                        if (!a.static_weights) {
                            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                            tma_load_2d(st + W_OFF, &tw, c * TK, n0, &full[s]);
                        }
                        tma_load_3d(st, &tx, c * TK, m0, 0, &full[s]);  // box 32 x 128 x 2: the planes
                        continue;
                    }
                    if (!mbar_wait_bounded(&empty[s], (use & 1u) ^ 1u)) {
                        *s_abort = 1;
                        break;
                    }
                    unsigned char* st = base + s * STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                    tma_load_3d(st, &tx, c * TK, m0, 0, &full[s]);  // box 32 x 128 x 2: the planes
                    tma_load_2d(st + W_OFF, &tw, c * TK, n0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            constexpr uint32_t idesc = umma_idesc_f16(TM, TN);
            uint32_t g = 0, i = 0;
            for (int t = blockIdx.x; t < tiles && !*s_abort; t += gridDim.x, ++i) {
                const uint32_t acc = i & 1u;
                if (!mbar_wait_bounded(&tempty[acc], ((i >> 1) & 1u) ^ 1u)) {
                    *s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc * TN;
                bool ok = true;
                for (int c = 0; c < nk; ++c, ++g) {
                    const uint32_t s = g % STAGES, use = g / STAGES;
                    if (!mbar_wait_bounded(&full[s], use & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = base_addr + s * STAGE_BYTES;
#pragma unroll
                    for (int ks = 0; ks < TK / 16; ++ks) {
                        const uint64_t bw = umma_desc_k_sw64(sa + W_OFF + ks * 32);
                        tc_mma_f16(d, umma_desc_k_sw64(sa + 0 * A_PLANE + ks * 32), bw, idesc, (c > 0 || ks > 0) ? 1u : 0u);
                        tc_mma_f16(d, umma_desc_k_sw64(sa + 1 * A_PLANE + ks * 32), bw, idesc, 1u);
                    }
                    tc_commit(&empty[s]);
                }
                if (!ok) {
                    *s_abort = 1;
                    break;
                }
                tc_commit(&tfull[acc]);
            }
        }
    } else {  // ---- epilogue warps 2-9: lane quarter warp % 4, column half (warp - 2) / 4
        const int quarter = warp & 3, half = (warp - 2) >> 2;
        float* buf = reinterpret_cast<float*>(base + SMEM_EPI) + (warp - 2) * 32 * BUF_LD;
        uint32_t i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
            const uint32_t acc = i & 1u;
            const bool go = __all_sync(0xffffffffu, *s_abort == 0);  // warp-uniform
            if (!go || !warp_wait_bounded(&tfull[acc], (i >> 1) & 1u)) {
                *s_abort = 1;
                break;
            }
            tc_fence_after();
            drain_tile_256(a, tmem + ((uint32_t)(quarter * 32) << 16) + acc * TN, buf, lane, half,
                           (t % MT) * TM + quarter * 32, (t / MT) * TN);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
    if (tid == 0 && *s_abort) atomicOr(err, NLLB_DEV_ERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// Pair form of the persistent kernel: 256 x 256 output tiles, each run by a
// cluster of two CTAs on two SMs with tcgen05.mma.cta_group::2.  CTA r of the
// pair loads rows [128r, 128r + 128) of the tile's activation planes and
// weight rows (output columns) [128r, 128r + 128) of its 256, 24 KB per
// 32-wide K chunk instead of the 32 KB of the one-CTA form, where both row
// halves of a 256-column weight tile read all of it; each CTA's TMEM holds
// its 128 output rows x 256 columns.  CTA 0 issues the MMAs of both: every
// TMA load of the pair completes on CTA 0's `full` barrier (loads in the
// cta_group::2 form, each into its own CTA's shared memory), every MMA batch
// commits to the `empty` and accumulator-ready barriers of both CTAs, and the
// epilogue warps of both arrive on CTA 0's accumulator-free barrier.  The
// roles, stage ring and double-buffered accumulators are the one-CTA form's.
// ---------------------------------------------------------------------------
namespace pair {
constexpr int TM = 128, TN = 256, TK = 32, STAGES = 7;  // TM: rows per CTA, 256 per pair
constexpr int EPI_WARPS = 8, THREADS = (EPI_WARPS + 2) * 32;
constexpr uint32_t A_PLANE = TM * TK * 2;                      // 8 KB
constexpr uint32_t B_HALF = (TN / 2) * TK * 2;                 // 8 KB: this CTA's half of the weight tile
constexpr uint32_t W_OFF = kPlanes * A_PLANE;
constexpr uint32_t STAGE_BYTES = kPlanes * A_PLANE + B_HALF;   // 24 KB per CTA
constexpr uint32_t SMEM_EPI = STAGES * STAGE_BYTES;
constexpr uint32_t SMEM_BAR = SMEM_EPI + EPI_WARPS * 32 * pers::BUF_LD * 4;
constexpr uint32_t SMEM_TOTAL = SMEM_BAR + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;
static_assert(SMEM_TOTAL <= 232448, "fits the 227 KB of shared memory a CTA may use");
}  // namespace pair

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// One arrival on `bar` in each CTA of the pair once the MMAs issued so far are done.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}
// TMA loads into this CTA's shared memory that complete on the barrier at
// cluster address `bar` (CTA 0's).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::THREADS, 1)
    linear_tma_pair_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
                           const LinearArgs a, int* err) {
    constexpr int TM = pair::TM, TN = pair::TN, TK = pair::TK, STAGES = pair::STAGES, EPI_WARPS = pair::EPI_WARPS;
    constexpr int BUF_LD = pers::BUF_LD;
    constexpr uint32_t A_PLANE = pair::A_PLANE, STAGE_BYTES = pair::STAGE_BYTES, SMEM_EPI = pair::SMEM_EPI;
    constexpr uint32_t W_OFF = pair::W_OFF;
    constexpr uint32_t SMEM_BAR = pair::SMEM_BAR, TMEM_COLS = pair::TMEM_COLS;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base_addr = (raw + 1023u) & ~1023u;  // the same offset in both CTAs (same kernel, same layout)
    unsigned char* base = smem_raw + (base_addr - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + SMEM_BAR);  // used in CTA 0
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;  // used in CTA 0
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_ctarank();
    const int MT = (a.M + 2 * TM - 1) / (2 * TM), NT = (a.N + TN - 1) / TN;
    const int tiles = MT * NT, nk = a.K / TK;
    const int pair_id = (int)blockIdx.x >> 1, npairs = (int)gridDim.x >> 1;

    if (warp == 0) tmem_alloc_pair(tmem_slot, TMEM_COLS);
    if (tid == 32) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * EPI_WARPS);
        }
        *s_abort = 0;
        fence_barrier_init();
    }
    pdl_launch_dependents();
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers exist before the first load or arrival from the partner
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (!(warp == 0 && lane == 0)) pdl_wait_primary();  // the output may still be read by earlier kernels

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer (both CTAs)
            prefetch_tensormap(&tx);
            prefetch_tensormap(&tw);
            const uint32_t full0 = map_rank(full, 0);  // CTA 0's full[s] at full0 + 8 s
            const int pre = pair_id < tiles ? (nk < STAGES ? nk : STAGES) : 0;
            if (a.static_weights) {
                const int wrow = (pair_id / MT) * TN + (int)rank * (TN / 2);
                for (int c = 0; c < pre; ++c) {
                    if (rank == 0) mbar_arrive_expect_tx(&full[c], 2 * STAGE_BYTES);
                    tma_load_2d_pair(base + c * STAGE_BYTES + W_OFF, &tw, c * TK, wrow, full0 + 8u * c);
                }
            }
            pdl_wait_primary();
            uint32_t g = 0;
            for (int t = pair_id; t < tiles && !*s_abort; t += npairs) {
                const int m0 = (t % MT) * (2 * TM) + (int)rank * TM, n0 = (t / MT) * TN + (int)rank * (TN / 2);
                for (int c = 0; c < nk; ++c, ++g) {
                    const uint32_t s = g % STAGES, use = g / STAGES;
                    unsigned char* st = base + s * STAGE_BYTES;
                    if ((int)g < pre) {  // fresh stage of the first tile
                        if (!a.static_weights) {
                            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
                            tma_load_2d_pair(st + W_OFF, &tw, c * TK, n0, full0 + 8u * s);
                        }
                        tma_load_3d_pair(st, &tx, c * TK, m0, 0, full0 + 8u * s);  // box 32 x 128 x 2
                        continue;
                    }
                    if (!mbar_wait_bounded(&empty[s], (use & 1u) ^ 1u)) {
                        *s_abort = 1;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
                    tma_load_3d_pair(st, &tx, c * TK, m0, 0, full0 + 8u * s);
                    tma_load_2d_pair(st + W_OFF, &tw, c * TK, n0, full0 + 8u * s);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {  // ---- MMA issuer for the pair (CTA 0)
            constexpr uint32_t idesc = umma_idesc_f16(2 * TM, TN);
            uint32_t g = 0, i = 0;
            for (int t = pair_id; t < tiles && !*s_abort; t += npairs, ++i) {
                const uint32_t acc = i & 1u;
                if (!mbar_wait_bounded(&tempty[acc], ((i >> 1) & 1u) ^ 1u)) {
                    *s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc * TN;
                bool ok = true;
                for (int c = 0; c < nk; ++c, ++g) {
                    const uint32_t s = g % STAGES, use = g / STAGES;
                    if (!mbar_wait_bounded(&full[s], use & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = base_addr + s * STAGE_BYTES;
#pragma unroll
                    for (int ks = 0; ks < TK / 16; ++ks) {
                        const uint64_t bw = umma_desc_k_sw64(sa + W_OFF + ks * 32);
                        mma_f16_pair(d, umma_desc_k_sw64(sa + 0 * A_PLANE + ks * 32), bw, idesc,
                                     (c > 0 || ks > 0) ? 1u : 0u);
                        mma_f16_pair(d, umma_desc_k_sw64(sa + 1 * A_PLANE + ks * 32), bw, idesc, 1u);
                    }
                    tc_commit_pair(&empty[s]);
                }
                if (!ok) {
                    *s_abort = 1;
                    break;
                }
                tc_commit_pair(&tfull[acc]);
            }
        }
    } else {  // ---- epilogue warps 2-9 (both CTAs): lane quarter warp % 4, column half (warp - 2) / 4
        const int quarter = warp & 3, half = (warp - 2) >> 2;
        float* buf = reinterpret_cast<float*>(base + SMEM_EPI) + (warp - 2) * 32 * BUF_LD;
        const uint32_t tempty0 = map_rank(tempty, 0);
        uint32_t i = 0;
        for (int t = pair_id; t < tiles; t += npairs, ++i) {
            const uint32_t acc = i & 1u;
            const bool go = __all_sync(0xffffffffu, *s_abort == 0);  // warp-uniform
            if (!go || !warp_wait_bounded(&tfull[acc], (i >> 1) & 1u)) {
                *s_abort = 1;
                break;
            }
            tc_fence_after();
            drain_tile_256(a, tmem + ((uint32_t)(quarter * 32) << 16) + acc * TN, buf, lane, half,
                           (t % MT) * (2 * TM) + (int)rank * TM + quarter * 32, (t / MT) * TN);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tempty0 + 8u * acc);
        }
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync_all();  // neither CTA leaves while its partner may still use its barriers or TMEM
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, TMEM_COLS);
    }
    if (tid == 0 && *s_abort) atomicOr(err, NLLB_DEV_ERR_TIMEOUT);
}

// x [M][ldx] fp32 -> planes [2][M][K] fp16 with x = p0 + p1 (planes.cuh)
__global__ void split_planes_kernel(const float* x, int ldx, int M, int K, plane_t* planes) {
    pdl_launch_dependents();
    pdl_wait_primary();  // x comes from the previous kernel; the planes may still be read by the previous GEMM
    const size_t n4 = (size_t)M * (K / 4);
    const size_t plane = (size_t)M * K;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / (K / 4)), k = (int)(i % (K / 4)) * 4;
        const float4 v = *reinterpret_cast<const float4*>(x + (size_t)m * ldx + k);
        store_planes_x4(planes, plane, (size_t)m * K + k, v);
    }
}

__global__ void int8_to_f16_kernel(const int8_t* w, plane_t* out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn((float)w[i]);  // exact: |w| <= 127
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

}  // namespace

cudaError_t configure_linear_tma() {
    cudaError_t e =
        cudaFuncSetAttribute(linear_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSplitSmemMax);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(linear_tma_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)pers::SMEM_TOTAL);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(linear_tma_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)pair::SMEM_TOTAL);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(linear_tma_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    std::call_once(g_encode_once, [] {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode;
}

// Tensor map of a row-major fp16 matrix stack: `planes` matrices of
// [rows][cols] (K-major), box box_cols x box_rows (x planes), with the
// 128-byte swizzle (box_cols 64) or the 64-byte swizzle (box_cols 32).
cudaError_t encode_half_map_box(CUtensorMap* map, const void* base, int cols, int rows, int planes, int box_cols,
                                int box_rows) {
    if (!tensor_map_encoder()) return cudaErrorNotSupported;
    if (box_cols != 64 && box_cols != 32) return cudaErrorInvalidValue;
    const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)planes};
    const cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)cols * rows * 2};
    const cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, (cuuint32_t)planes};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r =
        g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, planes > 1 ? 3 : 2, const_cast<void*>(base), dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encode_half_map(CUtensorMap* map, const void* base, int cols, int rows, int planes) {
    return encode_half_map_box(map, base, cols, rows, planes, TK, TM);
}

cudaError_t encode_half_maps_persistent(CUtensorMap* x_map, const void* planes, int K, int M, CUtensorMap* w_map,
                                        const void* wb, int N) {
    cudaError_t e = cudaSuccess;
    if (x_map) e = encode_half_map_box(x_map, planes, K, M, kPlanes, pers::TK, pers::TM);
    if (e == cudaSuccess && w_map) e = encode_half_map_box(w_map, wb, K, N, 1, pers::TK, pers::TN);
    return e;
}

// The persistent kernel runs each 128 x 256 tile's whole K loop in one CTA;
// the split-K kernel spreads a 128 x 128 tile's K over a cluster of up to 8
// CTAs.  Measured on B200 over M 256..4096, N 1024..4096, K 1024 / 4096
// (split depth as linear_tma_splits picks it): the persistent kernel wins from
// about 96 tiles of 128 x 256 up (1024 x 1024 -> 3072: 28 us against 36) and
// loses below 64 (512 x 1024 -> 3072: 27 us against 20), whatever K.
bool linear_tma_use_persistent(int M, int N, int K, int num_sms) {
    (void)K;
    const long long tiles = (long long)((M + pers::TM - 1) / pers::TM) * ((N + pers::TN - 1) / pers::TN);
    return tiles * 148 >= 80LL * num_sms;
}

// CTA pairs of the pair kernel that can be resident at once on the current
// device (both CTAs of a cluster sit in one GPC), queried once per device;
// 0 if the query fails.
int pair_capacity() {
    static std::mutex mu;
    static int cap[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (cap[dev] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2, 1, 1);
        cfg.blockDim = dim3(pair::THREADS, 1, 1);
        cfg.dynamicSmemBytes = pair::SMEM_TOTAL;  // cluster shape: the kernel's own __cluster_dims__
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, linear_tma_pair_kernel, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();  // clear
            n = -1;
        }
        cap[dev] = n;
    }
    return cap[dev] > 0 ? cap[dev] : 0;
}

// The pair kernel takes the persistent kernel's shapes from NLLB_PAIR_MIN_ROWS
// rows up (below that a 256-row pair tile would be mostly rows past M) when the
// output has at least two rounds of 128 x 256 tiles per SM.  Measured on B200
// (prepared linear, 4096 rows): 1024 -> 256206 in 3131 us on pairs against
// 3385 on single CTAs, 1024 -> 3072 and -> 4096 equal, 1024 -> 1024 26.6
// against 24.8 us and 4096 -> 1024 75.3 against 72.3 (one round of tiles:
// the pairs' co-scheduling costs more than the operand bytes they save).
#ifndef NLLB_PAIR_MIN_ROWS
#define NLLB_PAIR_MIN_ROWS 129
#endif
bool linear_tma_use_pair(int M, int N, int num_sms) {
    const long long tiles = (long long)((M + pers::TM - 1) / pers::TM) * ((N + pers::TN - 1) / pers::TN);
    return M >= NLLB_PAIR_MIN_ROWS && tiles >= 2LL * num_sms && pair_capacity() > 0;
}

cudaError_t launch_linear_tma_persistent(const LinearArgs& a, const CUtensorMap* tx, const CUtensorMap* tw,
                                         const CUtensorMap* tw_pair, int num_sms, int* err, cudaStream_t st) {
    if (tw_pair && linear_tma_use_pair(a.M, a.N, num_sms)) {
        const int tiles = ((a.M + 2 * pair::TM - 1) / (2 * pair::TM)) * ((a.N + pair::TN - 1) / pair::TN);
        const int cap = pair_capacity();
        const int pairs = tiles < cap ? tiles : cap;
        if (pairs < 1) return cudaSuccess;
        return launch_pdl(linear_tma_pair_kernel, dim3(2 * pairs), dim3(pair::THREADS), pair::SMEM_TOTAL, st, *tx,
                          *tw_pair, a, err);
    }
    const int tiles = ((a.M + pers::TM - 1) / pers::TM) * ((a.N + pers::TN - 1) / pers::TN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    if (grid < 1) return cudaSuccess;
    return launch_pdl(linear_tma_persistent_kernel, dim3(grid), dim3(pers::THREADS), pers::SMEM_TOTAL, st, *tx, *tw, a,
                      err);
}

cudaError_t encode_half_map_pair(CUtensorMap* map, const void* wb, int K, int N) {
    return encode_half_map_box(map, wb, K, N, 1, pair::TK, pair::TN / 2);
}

// Clusters of S CTAs of the split-K kernel that can be resident at once on the
// current device (thread-block clusters must fit inside one GPC, so this is
// below num_sms / S for large S).  Queried once per device and S.
int cluster_capacity(int S) {
    static std::mutex mu;
    static int cap[64][4] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    const int idx = S == 2 ? 1 : S == 4 ? 2 : S == 8 ? 3 : 0;
    std::lock_guard<std::mutex> lock(mu);
    if (cap[dev][idx] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S, 1, 1);
        cfg.blockDim = dim3(THREADS, 1, 1);
        cfg.dynamicSmemBytes = SMEM_TOTAL;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = (unsigned)S;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, linear_tma_kernel, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();  // clear
            n = -1;
        }
        cap[dev][idx] = n;
    }
    return cap[dev][idx];
}

// Split-K depth: the largest of 1, 2, 4, 8 whose clusters all fit on the GPU
// at once (one wave) with every CTA keeping at least two K chunks.  Measured
// on B200: 16 tiles run 17 us as 16 clusters of 8 (more than one wave) and
// 11 us as 16 clusters of 4; 8 tiles run fastest as 8 clusters of 8.
int linear_tma_splits(int M, int N, int K, int num_sms) {
    const int tiles = ((N + TN - 1) / TN) * ((M + TM - 1) / TM);
    const int nk = K / TK;
    int S = 1;
    while (S < 8 && tiles * 2 * S <= num_sms && nk / (2 * S) >= 2 && tiles <= cluster_capacity(2 * S)) S *= 2;
    return S;
}

cudaError_t launch_split_planes(const float* x, int ldx, int M, int K, void* planes, cudaStream_t st) {
    const size_t n4 = (size_t)M * (K / 4);
    int blocks = (int)((n4 + 255) / 256);
    blocks = blocks < 4096 ? blocks : 4096;
    if (blocks < 1) return cudaSuccess;
    return launch_pdl(split_planes_kernel, dim3(blocks), dim3(256), 0, st, x, ldx, M, K,
                      static_cast<plane_t*>(planes));
}

cudaError_t launch_int8_to_f16(const int8_t* w, void* out, size_t n, cudaStream_t st) {
    int blocks = (int)((n + 255) / 256);
    blocks = blocks < 8192 ? blocks : 8192;
    int8_to_f16_kernel<<<blocks, 256, 0, st>>>(w, static_cast<plane_t*>(out), n);
    return cudaGetLastError();
}

cudaError_t launch_linear_tma(const LinearArgs& a, const CUtensorMap* tx, const CUtensorMap* tw, int splits, int* err,
                              cudaStream_t st) {
    const int mt = (a.M + TM - 1) / TM, nt = (a.N + TN - 1) / TN;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(mt * splits, nt, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    // with a residual: room for this rank's residual rows behind the stage ring, where it fits
    const uint32_t res_bytes = a.residual ? (uint32_t)(TM / splits) * TN * 4 : 0;
    cfg.dynamicSmemBytes = SMEM_TOTAL + res_bytes <= kSplitSmemMax ? SMEM_TOTAL + res_bytes : SMEM_TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel waits after its prologue
    attr[1].val.programmaticStreamSerializationAllowed = kPdlLaunch;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, linear_tma_kernel, *tx, *tw, a, splits, err);
}

}  // namespace nllb
