// planes.cuh -- fp32 -> three bf16 planes, x = p0 + p1 + p2 to 24 bits.
//
// Every int8 weight is exact in bf16, so x * w is three bf16 MMAs with fp32
// accumulation.  The split is the same wherever it is made (split3_kernel,
// LayerNorm, GEMM epilogues), so a value gives the same planes on every path.
#pragma once
#include <cuda_bf16.h>

namespace nllb {

__device__ __forceinline__ void split3_value(float x, __nv_bfloat16& p0, __nv_bfloat16& p1, __nv_bfloat16& p2) {
    p0 = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(p0);
    p1 = __float2bfloat16_rn(r1);
    p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
}

// Four consecutive values -> 8 bytes in each plane (plane stride in elements).
__device__ __forceinline__ void store_split3_x4(__nv_bfloat16* planes, size_t plane_stride, size_t o, float4 v) {
    __nv_bfloat16 p[3][4];
    split3_value(v.x, p[0][0], p[1][0], p[2][0]);
    split3_value(v.y, p[0][1], p[1][1], p[2][1]);
    split3_value(v.z, p[0][2], p[1][2], p[2][2]);
    split3_value(v.w, p[0][3], p[1][3], p[2][3]);
#pragma unroll
    for (int q = 0; q < 3; ++q)
        *reinterpret_cast<uint2*>(planes + q * plane_stride + o) = *reinterpret_cast<const uint2*>(p[q]);
}

__device__ __forceinline__ void store_split3_x1(__nv_bfloat16* planes, size_t plane_stride, size_t o, float v) {
    __nv_bfloat16 p0, p1, p2;
    split3_value(v, p0, p1, p2);
    planes[o] = p0;
    planes[plane_stride + o] = p1;
    planes[2 * plane_stride + o] = p2;
}

}  // namespace nllb
