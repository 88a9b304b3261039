// prefill.cu -- encoder self-attention prefill, fp32 (sm_100a).
//
// Flash-attention form of attention_head_flash (tensor.c:286-332) /
// encoder.c:166-205: one CTA per (64-query tile, head, sequence) streams
// 64-key tiles of K and V through shared memory with an online softmax in
// base 2, so nothing of size seq x seq is ever stored.  FFMA with fp32
// accumulation: every product is an exact fp32 product, matching the
// reference's arithmetic to rounding.
//
// Thread tile: 128 threads as 8 (ty) x 16 (tx).  A thread owns query rows
// ty + 8i (i < 8); for scores it owns key columns tx + 16j (j < 4), for the
// output it owns dims 4tx..4tx+3.  Row statistics reduce over the 16 tx
// lanes of a half-warp with xor-shuffles.
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

    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int S = p.S;
    const int q0 = qt * BQ;
    const long long base = (long long)b * p.sb + (long long)h * p.sh;
    // valid_len[b] <= 0 leaves no unmasked key; the reference's additive -1e9
    // mask then makes every score equal, i.e. the plain mean of V: do that.
    int kv_len = S;
    bool uniform = false;
    if (p.valid_len) {
        const int vl = __ldg(p.valid_len + b);
        if (vl <= 0) uniform = true;
        else kv_len = min(vl, S);
    }
    const float* mrow0 =
        p.mask ? p.mask + (long long)b * p.msb + (long long)h * p.msh : nullptr;

    // Q tile (rows beyond S read as zero)
    for (int i = tid; i < BQ * 16; i += kThreads) {
        const int r = i >> 4, c4 = i & 15;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + r < S) v = __ldg(reinterpret_cast<const float4*>(p.q + base + (long long)(q0 + r) * p.sr) + c4);
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
        if (qr < S) {
            float* dst = p.out + base + (long long)qr * p.sr;
            reinterpret_cast<float4*>(dst)[tx] = f4_scale(o[i], 1.0f / l);
        }
    }
}

}  // namespace

cudaError_t configure_prefill_kernels() {
    const int smem = 4 * BQ * LDS * (int)sizeof(float);
    return cudaFuncSetAttribute(prefill_ffma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t st) {
    const int smem = 4 * BQ * LDS * (int)sizeof(float);
    dim3 grid((p.S + BQ - 1) / BQ, p.H, p.B);
    prefill_ffma_kernel<<<grid, kThreads, smem, st>>>(p);
    return cudaGetLastError();
}

}  // namespace nllb
