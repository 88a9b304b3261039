// device_common.cuh -- PTX helpers shared by the attention kernels (sm_100a).
//
// Bulk copies (cp.async.bulk, the 1-D form of TMA) move contiguous K/V
// blocks from HBM into shared memory and complete on an mbarrier.  Every copy
// targets the issuing CTA's own shared memory only (no cluster-wide copies),
// and no kernel reads another GPU's memory.  Every wait on an mbarrier is bounded by a clock64() budget;
// on expiry the kernel records NLLB_DEV_ERR_TIMEOUT in the context's device
// error word and leaves without writing outputs.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include <utility>

namespace nllb {

constexpr int kHeadDim = 64;
constexpr float kLog2e = 1.4426950408889634f;

// device error word bits (read and cleared by nllb_attn_sync)
constexpr int NLLB_DEV_ERR_TIMEOUT = 1;
constexpr int NLLB_DEV_ERR_BAD_PARENT = 2;

// ~1 s at 2 GHz: far above any legitimate wait for a copy of a few KB.
constexpr long long kWaitBudgetCycles = 2000000000LL;
// ~1 ms: the budget of the one wait the bounded-wait test makes run out.
constexpr long long kTestWaitBudgetCycles = 2000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Make barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// global -> shared bulk copy; dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; false if the budget (clock64
// cycles) ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long budget = kWaitBudgetCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > budget) return false;
    }
    return true;
}

__device__ __forceinline__ float4 f4_scale(float4 a, float s) {
    return make_float4(a.x * s, a.y * s, a.z * s, a.w * s);
}
__device__ __forceinline__ float4 f4_fma(float s, float4 v, float4 acc) {
    return make_float4(fmaf(s, v.x, acc.x), fmaf(s, v.y, acc.y), fmaf(s, v.z, acc.z),
                       fmaf(s, v.w, acc.w));
}
__device__ __forceinline__ float f4_dot(float4 a, float4 b) {
    return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)));
}

// Sum over the 16 lanes of a half-warp (both halves reduce independently).
// Must be reached by all 32 lanes.
__device__ __forceinline__ float halfwarp_sum(float x) {
    x += __shfl_xor_sync(0xffffffffu, x, 8);
    x += __shfl_xor_sync(0xffffffffu, x, 4);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    return x;
}

// Four half-warp sums at once (four beams' partial dots of one row), each
// bit for bit halfwarp_sum(v[b]): partners swap the beams they do not keep
// (xor 8: two, xor 4: one), so every addition is one that halfwarp_sum makes
// for that beam; two more tree steps and a broadcast follow.  9 shuffles and
// 5 adds instead of 16 and 16.
__device__ __forceinline__ void halfwarp_sum4(const float (&v)[4], float (&out)[4]) {
    const int lane = threadIdx.x & 31;
    const bool hi8 = (lane & 8) != 0, hi4 = (lane & 4) != 0;
    const float r0 = __shfl_xor_sync(0xffffffffu, hi8 ? v[0] : v[2], 8);
    const float r1 = __shfl_xor_sync(0xffffffffu, hi8 ? v[1] : v[3], 8);
    const float a0 = (hi8 ? v[2] : v[0]) + r0;  // beam 2*hi8
    const float a1 = (hi8 ? v[3] : v[1]) + r1;  // beam 2*hi8 + 1
    const float r = __shfl_xor_sync(0xffffffffu, hi4 ? a0 : a1, 4);
    float t = (hi4 ? a1 : a0) + r;  // beam 2*hi8 + hi4
    t += __shfl_xor_sync(0xffffffffu, t, 2);
    t += __shfl_xor_sync(0xffffffffu, t, 1);
    const int base = lane & 16;
    out[0] = __shfl_sync(0xffffffffu, t, base);
    out[1] = __shfl_sync(0xffffffffu, t, base + 4);
    out[2] = __shfl_sync(0xffffffffu, t, base + 8);
    out[3] = __shfl_sync(0xffffffffu, t, base + 12);
}

// exp2 of a difference that may be -inf - -inf (empty state): weight 0.
__device__ __forceinline__ float safe_exp2_diff(float a, float m) {
    return (a == -INFINITY) ? 0.0f : exp2f(a - m);
}

}  // namespace nllb

namespace nllb {

// ---- thread-block clusters (distributed shared memory) --------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// All threads of every CTA of the cluster; release/acquire orders the shared
// memory writes before it with the remote reads after it.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ int ld_cluster_s32(uint32_t addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// ---- programmatic dependent launch -----------------------------------------
// Let the next kernel in the stream start its prologue on SMs this grid frees.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Wait until the previous kernel in the stream has completed and its memory
// is visible; everything that reads a predecessor's output comes after this.
__device__ __forceinline__ void pdl_wait_primary() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Programmatic dependent launch for every kernel of the library (builds for
// per-kernel timing set NLLB_NO_PDL: each kernel then waits for the full
// completion of its predecessor, so profiler durations do not overlap).
#ifdef NLLB_NO_PDL
constexpr int kPdlLaunch = 0;
#else
constexpr int kPdlLaunch = 1;
#endif

// Launch with programmatic stream serialisation: the kernel may be scheduled
// while its predecessor in the stream finishes (once every predecessor CTA has
// started or triggered); it must execute pdl_wait_primary() before reading the
// predecessor's outputs or writing global memory.  Waiting also covers every
// earlier kernel of the stream, since each of them waited on its own
// predecessor before finishing.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = kPdlLaunch;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace nllb

namespace nllb {

// ---- tcgen05 (5th-generation tensor cores, tensor memory) ------------------
// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzled
// canonical layout: rows of 128 B (32 tf32 values), 8-row atoms 1024 B apart
// (stride byte offset), leading byte offset 16 B, descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor: kind::tf32, fp32 accumulate, A and B K-major.
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor: kind::f16, fp32 accumulate, A and B fp16, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes become visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Warp-wide: allocate `ncols` TMEM columns, base address written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp-wide).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 32-column loads of this thread's TMEM lane (warp-wide) under one wait.
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, uint32_t tb, float* va, float* vb) {
    uint32_t r[64];
#define NLLB_TMEM_LD32(T, R)                                                                                  \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "                                                    \
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "                    \
                 "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"    \
                 : "=r"(R[0]), "=r"(R[1]), "=r"(R[2]), "=r"(R[3]), "=r"(R[4]), "=r"(R[5]), "=r"(R[6]),        \
                   "=r"(R[7]), "=r"(R[8]), "=r"(R[9]), "=r"(R[10]), "=r"(R[11]), "=r"(R[12]), "=r"(R[13]),    \
                   "=r"(R[14]), "=r"(R[15]), "=r"(R[16]), "=r"(R[17]), "=r"(R[18]), "=r"(R[19]), "=r"(R[20]), \
                   "=r"(R[21]), "=r"(R[22]), "=r"(R[23]), "=r"(R[24]), "=r"(R[25]), "=r"(R[26]), "=r"(R[27]), \
                   "=r"(R[28]), "=r"(R[29]), "=r"(R[30]), "=r"(R[31])                                         \
                 : "r"(T))
    NLLB_TMEM_LD32(ta, r);
    NLLB_TMEM_LD32(tb, (r + 32));
#undef NLLB_TMEM_LD32
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        va[i] = __uint_as_float(r[i]);
        vb[i] = __uint_as_float(r[32 + i]);
    }
}

// fp32 -> (hi, lo) with hi exactly representable in tf32 (low 13 mantissa
// bits cleared) and lo = x - hi exact; hi*hi' + hi*lo' + lo*hi' reproduces an
// fp32 product to ~2^-21 relative.
__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

}  // namespace nllb
