// linear_tc.cu -- INT8-weight linear layer on 5th-generation tensor cores (sm_100a).
//
// out[m][n] = (sum_k x[m][k] * w[n][k]) / scale[n] + bias[n] (+ReLU, +residual),
// the arithmetic of mat_vec_int8 (tensor.c:70-138) for many rows at once.
//
// Exactness: int8 weights are exact in bf16.  Each fp32 activation is split
// into three bf16 parts x = x1 + x2 + x3 (x1 = bf16(x), x2 = bf16(x - x1),
// x3 = bf16(x - x1 - x2)), which carry 24 significant bits, and every k-step
// issues three tcgen05.mma kind::f16 (bf16 x bf16 -> fp32 in TMEM).  Products
// of bf16 values are exact in fp32, so the result matches an fp32 dot product
// to accumulation rounding.
//
// Tile: 128 rows x 128 outputs per CTA, K in stages of 64.  Warps 0-7 load x
// (fp32) and w (int8) from global memory, convert, and store into 128-byte
// swizzled K-major shared memory (3-stage ring, full/empty mbarriers); warp 8
// issues the MMAs and commits each stage back to its producers; after the
// last stage warps 0-7 read the accumulator from TMEM (two threads per row)
// and apply the epilogue.
#include <cuda_bf16.h>

#include "device_common.cuh"
#include "engine_kernels.h"

namespace nllb {

namespace {

constexpr int TM = 128, TN = 128, TK = 64, STAGES = 3;
constexpr int PRODUCERS = 256, THREADS = PRODUCERS + 32;
constexpr uint32_t PLANE = TM * TK * 2;  // 16 KB: one bf16 operand tile, 128 rows x 128 B
constexpr uint32_t STAGE_BYTES = 4 * PLANE;  // x1, x2, x3, w
constexpr uint32_t SMEM_BAR = STAGES * STAGE_BYTES;
constexpr uint32_t SMEM_TOTAL = SMEM_BAR + 128 + 1024;  // barriers + alignment slack
constexpr uint32_t TMEM_COLS = 128;

__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// byte offset of the 16-B chunk holding k-column c (bf16) of `row` in a
// 128 B-row swizzled tile
__device__ __forceinline__ uint32_t chunk_off(int row, int c) {
    return (uint32_t)(row * 128 + ((((c >> 3) ^ (row & 7))) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat16 ha = __float2bfloat16_rn(a), hb = __float2bfloat16_rn(b);
    return (uint32_t)__bfloat16_as_ushort(ha) | ((uint32_t)__bfloat16_as_ushort(hb) << 16);
}

// Split-K: CTA z of a tile covers k-stages [z*nk/S, (z+1)*nk/S).  With S > 1
// each CTA writes its raw tile to ws[(tile * S + z)][128][128]; the last CTA
// of the tile to finish (one atomic on tile_count[tile], no waiting) adds the
// S partial tiles in split order and applies the epilogue, so the result does
// not depend on which CTA finishes last.
__global__ void __launch_bounds__(THREADS, 1) linear_tc_kernel(const LinearArgs a, int* err, float* ws,
                                                               int* tile_count) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base_addr = (raw + 1023u) & ~1023u;
    unsigned char* base = smem_raw + (base_addr - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + SMEM_BAR);
    uint64_t* empty = full + STAGES;
    uint64_t* done = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    const int S = gridDim.z, z = blockIdx.z;
    const int nk_all = a.K / TK;
    const int kc0 = (int)((long long)z * nk_all / S), kc1 = (int)((long long)(z + 1) * nk_all / S);
    const int nk = kc1 - kc0;
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    __shared__ int s_last;

    if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], PRODUCERS);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        *s_abort = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 8) {
        // ---- producers: global -> registers (one stage ahead) -> convert -> swizzled shared memory
        float4 xr[8];
        int4 wr[2];
        auto load_stage = [&](int c) {
            const int k0 = (kc0 + c) * TK;
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int i = it * PRODUCERS + tid, r = i >> 4, q = i & 15;
                xr[it] = (m0 + r < a.M) ? *reinterpret_cast<const float4*>(a.x + (size_t)(m0 + r) * a.ldx + k0 + q * 4)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                const int i = it * PRODUCERS + tid, r = i >> 2, q = i & 3;
                wr[it] = (n0 + r < a.N) ? *reinterpret_cast<const int4*>(a.w + (size_t)(n0 + r) * a.K + k0 + q * 16)
                                        : make_int4(0, 0, 0, 0);
            }
        };
        if (nk > 0) load_stage(0);
        for (int c = 0; c < nk; ++c) {
            const int s = c % STAGES;
            if (c >= STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)((c / STAGES - 1) & 1))) {
                *s_abort = 1;
                break;
            }
            unsigned char* st = base + s * STAGE_BYTES;
            // x: 128 rows x 64 fp32 = 2048 float4, 8 per thread, split into 3 bf16 parts
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int i = it * PRODUCERS + tid, r = i >> 4, q = i & 15;
                const float f[4] = {xr[it].x, xr[it].y, xr[it].z, xr[it].w};
                float p1[4], p2[4], p3[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    p1[e] = __bfloat162float(__float2bfloat16_rn(f[e]));
                    const float r1 = f[e] - p1[e];
                    p2[e] = __bfloat162float(__float2bfloat16_rn(r1));
                    p3[e] = r1 - p2[e];
                }
                const uint32_t off = chunk_off(r, q * 4) + (uint32_t)((q & 1) * 8);
                *reinterpret_cast<uint2*>(st + 0 * PLANE + off) = make_uint2(pack_bf16(p1[0], p1[1]), pack_bf16(p1[2], p1[3]));
                *reinterpret_cast<uint2*>(st + 1 * PLANE + off) = make_uint2(pack_bf16(p2[0], p2[1]), pack_bf16(p2[2], p2[3]));
                *reinterpret_cast<uint2*>(st + 2 * PLANE + off) = make_uint2(pack_bf16(p3[0], p3[1]), pack_bf16(p3[2], p3[3]));
            }
            // w: 128 rows x 64 int8 = 512 x 16 B, 2 per thread, exact in bf16
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                const int i = it * PRODUCERS + tid, r = i >> 2, q = i & 3;  // q: 16-k group
                const int8_t* b = reinterpret_cast<const int8_t*>(&wr[it]);
                uint4 lo, hi;
                lo.x = pack_bf16((float)b[0], (float)b[1]);
                lo.y = pack_bf16((float)b[2], (float)b[3]);
                lo.z = pack_bf16((float)b[4], (float)b[5]);
                lo.w = pack_bf16((float)b[6], (float)b[7]);
                hi.x = pack_bf16((float)b[8], (float)b[9]);
                hi.y = pack_bf16((float)b[10], (float)b[11]);
                hi.z = pack_bf16((float)b[12], (float)b[13]);
                hi.w = pack_bf16((float)b[14], (float)b[15]);
                *reinterpret_cast<uint4*>(st + 3 * PLANE + chunk_off(r, q * 16)) = lo;
                *reinterpret_cast<uint4*>(st + 3 * PLANE + chunk_off(r, q * 16 + 8)) = hi;
            }
            if (c + 1 < nk) load_stage(c + 1);  // next stage's loads fly while this one is consumed
            fence_async_smem();
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&full[s])) : "memory");
        }
    } else if (lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = idesc_bf16(TM, TN);
        bool ok = true;
        for (int c = 0; c < nk; ++c) {
            const int s = c % STAGES;
            if (!mbar_wait_bounded(&full[s], (uint32_t)((c / STAGES) & 1))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t st = base_addr + s * STAGE_BYTES;
#pragma unroll
            for (int ks = 0; ks < TK / 16; ++ks) {
                const uint64_t bw = umma_desc_k_sw128(st + 3 * PLANE + ks * 32);
                const uint32_t first = (c > 0 || ks > 0) ? 1u : 0u;
                mma_bf16(tmem, umma_desc_k_sw128(st + 0 * PLANE + ks * 32), bw, idesc, first);
                mma_bf16(tmem, umma_desc_k_sw128(st + 1 * PLANE + ks * 32), bw, idesc, 1u);
                mma_bf16(tmem, umma_desc_k_sw128(st + 2 * PLANE + ks * 32), bw, idesc, 1u);
            }
            tc_commit(&empty[s]);
        }
        if (!ok) *s_abort = 1;
        tc_commit(done);  // arrives once everything issued so far is complete
    }

    // ---- epilogue (warps 0-7): accumulator rows from TMEM
    // The residual may be the output itself: callers load the residual
    // values of a run of outputs before storing any of them (the loads
    // overlap; each element is still read before it is written).
    auto out_index = [&](int m, int n) -> size_t {
        return (size_t)(n / a.cblock) * ((size_t)a.M * a.cblock) + (size_t)m * a.cblock + (n % a.cblock);
    };
    auto store_out = [&](int m, int n, float acc, float res) {
        float y = acc * (1.0f / a.scale[n]);
        if (a.bias) y += a.bias[n];
        if (a.relu) y = fmaxf(y, 0.f);
        if (a.mask_from >= 0 && n >= a.mask_from) y = -1e30f;
        if (a.residual) y += res;
        a.out[out_index(m, n)] = y;
    };
    bool ok = true;
    const int quarter = warp & 3, half = warp >> 2;
    const int rloc = quarter * 32 + lane;
    if (warp < 8) {
        ok = mbar_wait_bounded(done, 0u) && !*s_abort;
        tc_fence_after();
        float v[32];
#pragma unroll
        for (int part = 0; part < 2; ++part) {
            const int col0 = half * 64 + part * 32;
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0, v);
            if (!ok) continue;
            if (S == 1) {
                const int m = m0 + rloc;
                if (m < a.M) {
                    float res[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        res[j] = (a.residual && n0 + col0 + j < a.N) ? a.residual[out_index(m, n0 + col0 + j)] : 0.f;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (n0 + col0 + j < a.N) store_out(m, n0 + col0 + j, v[j], res[j]);
                }
            } else {
                float4* dst = reinterpret_cast<float4*>(ws + ((size_t)tile * S + z) * (TM * TN) + rloc * TN + col0);
#pragma unroll
                for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
        }
        if (!ok && tid == 0) atomicOr(err, NLLB_DEV_ERR_TIMEOUT);
    }
    if (S > 1) {
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = (atomicAdd(&tile_count[tile], 1) == S - 1);
        __syncthreads();
        if (s_last && warp < 8) {
            __threadfence();
            const int m = m0 + rloc;
            for (int col0 = half * 64; col0 < half * 64 + 64; col0 += 4) {
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int zz = 0; zz < S; ++zz) {
                    const float4 p = __ldcg(reinterpret_cast<const float4*>(
                        ws + ((size_t)tile * S + zz) * (TM * TN) + rloc * TN + col0));
                    acc.x += p.x;
                    acc.y += p.y;
                    acc.z += p.z;
                    acc.w += p.w;
                }
                if (m < a.M) {
                    const float av[4] = {acc.x, acc.y, acc.z, acc.w};
                    float res[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        res[j] = (a.residual && n0 + col0 + j < a.N) ? a.residual[out_index(m, n0 + col0 + j)] : 0.f;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (n0 + col0 + j < a.N) store_out(m, n0 + col0 + j, av[j], res[j]);
                }
            }
            if (tid == 0) tile_count[tile] = 0;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

cudaError_t configure_linear_tc() {
    return cudaFuncSetAttribute(linear_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TOTAL);
}

bool linear_tc_supports(const LinearArgs& a) { return a.K % TK == 0 && a.ldx % 4 == 0; }

int linear_tc_splits(const LinearArgs& a, int num_sms) {
    const int tiles = ((a.N + TN - 1) / TN) * ((a.M + TM - 1) / TM);
    const int nk = a.K / TK;
    int S = (2 * num_sms + tiles - 1) / tiles;
    S = S < 8 ? S : 8;
    S = S < nk / 2 ? S : nk / 2;
    return S > 1 ? S : 1;
}

size_t linear_tc_workspace_floats(const LinearArgs& a, int splits) {
    if (splits <= 1) return 0;
    const size_t tiles = (size_t)((a.N + TN - 1) / TN) * ((a.M + TM - 1) / TM);
    return tiles * splits * TM * TN;
}

size_t linear_tc_tiles(const LinearArgs& a) { return (size_t)((a.N + TN - 1) / TN) * ((a.M + TM - 1) / TM); }

cudaError_t launch_linear_tc(const LinearArgs& a, int splits, float* ws, int* tile_count, int* err,
                             cudaStream_t st) {
    dim3 grid((a.N + TN - 1) / TN, (a.M + TM - 1) / TM, splits > 1 ? splits : 1);
    linear_tc_kernel<<<grid, THREADS, SMEM_TOTAL, st>>>(a, err, ws, tile_count);
    return cudaGetLastError();
}

}  // namespace nllb
