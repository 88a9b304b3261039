// planes.cuh -- fp32 -> two fp16 planes, x = p0 + p1 to 22 bits.
//
// Every int8 weight is exact in fp16, so x * w is two fp16 MMAs (kind::f16)
// with fp32 accumulation, each product exact in fp32.  p0 = fp16(x) keeps 11
// significant bits, p1 = fp16(x - p0) the next 11: |x - p0 - p1| <= 2^-22 |x|
// while |x - p0| >= 2^-14 (below that p1 is subnormal and the error is at most
// 2^-25 in absolute terms).  Valid for |x| < 65504, the fp16 range; the
// engine's activations (LayerNorm outputs, attention outputs, the FFN's
// hidden layer) stay far inside it.  The split is the same wherever it is
// made (split kernel, LayerNorm, attention kernels, GEMM epilogues), so a
// value gives the same planes on every path.
#pragma once
#include <cuda_fp16.h>

namespace nllb {

using plane_t = __half;
constexpr int kPlanes = 2;

__device__ __forceinline__ void split_value(float x, plane_t& p0, plane_t& p1) {
    p0 = __float2half_rn(x);
    p1 = __float2half_rn(x - __half2float(p0));
}

// Four consecutive values -> 8 bytes in each plane (plane stride in elements).
__device__ __forceinline__ void store_planes_x4(plane_t* planes, size_t plane_stride, size_t o, float4 v) {
    plane_t p[kPlanes][4];
    split_value(v.x, p[0][0], p[1][0]);
    split_value(v.y, p[0][1], p[1][1]);
    split_value(v.z, p[0][2], p[1][2]);
    split_value(v.w, p[0][3], p[1][3]);
#pragma unroll
    for (int q = 0; q < kPlanes; ++q)
        *reinterpret_cast<uint2*>(planes + q * plane_stride + o) = *reinterpret_cast<const uint2*>(p[q]);
}

__device__ __forceinline__ void store_planes_x1(plane_t* planes, size_t plane_stride, size_t o, float v) {
    plane_t p0, p1;
    split_value(v, p0, p1);
    planes[o] = p0;
    planes[plane_stride + o] = p1;
}

}  // namespace nllb
