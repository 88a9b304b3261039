// linear_prepared.cu -- INT8 linear layer with weights prepared once.
//
// The reference holds each layer as a LinearInt8 (pico.h:26-32) pointing into
// the mmap'd model and dequantises inside every mat-vec (tensor.c:144-196).
// nllb_linear_prepare is the resident form of one LinearInt8: it keeps an fp16
// copy of the int8 matrix (every int8 value is exact in fp16) with its TMA
// tensor map, so nllb_linear_run feeds the tcgen05 GEMM straight from DRAM
// through TMA (linear_tma.cu).  Up to 16 rows run on the SIMT kernel over the
// int8 matrix, which moves half the bytes.
#include <cuda_fp16.h>

#include <string>

#include "engine_kernels.h"
#include "planes.cuh"
#include "nllb_translate.h"

namespace nllb {
int set_error(int status, const std::string& msg);  // nllb_attn.cu
}

using namespace nllb;

struct nllb_linear {
    int device = 0;
    const int8_t* w = nullptr;
    const float* scale = nullptr;
    const float* bias = nullptr;
    int N = 0, K = 0;
    int num_sms = 148;
    void* wb = nullptr;       // [N][K] fp16
    CUtensorMap tm{};         // of wb, box 64 x 128 (split-K kernel)
    CUtensorMap tm256{};      // of wb, box 32 x 256 (persistent kernel)
    CUtensorMap tm_pair{};    // of wb, box 32 x 128 (persistent kernel on CTA pairs)
    void* planes = nullptr;   // [2][M][K] fp16, grow-only
    size_t planes_elems = 0;
    int map_rows = -1;        // rows the plane maps were encoded for
    CUtensorMap tx{}, tx_pers{};
    int* err = nullptr;       // bounded-wait error word
    bool expire_next = false; // nllb_linear_test_expire_next_wait: the next split-K launch times out
};

#define LP_CK(call)                                                                                   \
    do {                                                                                              \
        const cudaError_t e_ = (call);                                                                \
        if (e_ != cudaSuccess) return nllb::set_error(NLLB_ATTN_ECUDA, std::string(#call ": ") + cudaGetErrorString(e_)); \
    } while (0)

extern "C" {

void nllb_linear_free(nllb_linear* L) {
    if (!L) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(L->device);
    cudaDeviceSynchronize();
    if (L->wb) cudaFree(L->wb);
    if (L->planes) cudaFree(L->planes);
    if (L->err) cudaFree(L->err);
    cudaSetDevice(cur);
    delete L;
}

int nllb_linear_prepare(const int8_t* w, const float* weight_scale, const float* bias, int N, int K, void* stream,
                        nllb_linear** out) {
    if (!out) return nllb::set_error(NLLB_ATTN_EINVAL, "out required");
    *out = nullptr;
    if (!w || !weight_scale) return nllb::set_error(NLLB_ATTN_EINVAL, "w and weight_scale required");
    if (N < 1 || K < 64 || K % 64) return nllb::set_error(NLLB_ATTN_EINVAL, "N >= 1 and K a positive multiple of 64");
    if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(weight_scale) & 3))
        return nllb::set_error(NLLB_ATTN_EINVAL, "w must be 16-byte aligned, weight_scale 4-byte aligned");
    int dev = 0;
    LP_CK(cudaGetDevice(&dev));
    int major = 0;
    LP_CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10) return nllb::set_error(NLLB_ATTN_ENODEV, "the tensor-core linear kernel needs an sm_100 device");
    if (configure_linear_tma() != cudaSuccess)
        return nllb::set_error(NLLB_ATTN_ECUDA, "cannot configure the TMA linear kernel");
    nllb_linear* L = new nllb_linear();
    L->device = dev;
    L->w = w;
    L->scale = weight_scale;
    L->bias = bias;
    L->N = N;
    L->K = K;
    cudaDeviceGetAttribute(&L->num_sms, cudaDevAttrMultiProcessorCount, dev);
    auto fail = [&](int rc) {
        nllb_linear_free(L);
        return rc;
    };
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMalloc(&L->wb, (size_t)N * K * sizeof(plane_t)) != cudaSuccess ||
        cudaMalloc(&L->err, sizeof(int)) != cudaSuccess || cudaMemsetAsync(L->err, 0, sizeof(int), st) != cudaSuccess)
        return fail(nllb::set_error(NLLB_ATTN_ECUDA, "cannot allocate the fp16 weight copy"));
    if (launch_int8_to_f16(w, L->wb, (size_t)N * K, st) != cudaSuccess)
        return fail(nllb::set_error(NLLB_ATTN_ECUDA, "weight conversion launch failed"));
    if (encode_half_map(&L->tm, L->wb, K, N, 1) != cudaSuccess ||
        encode_half_maps_persistent(nullptr, nullptr, K, 0, &L->tm256, L->wb, N) != cudaSuccess ||
        encode_half_map_pair(&L->tm_pair, L->wb, K, N) != cudaSuccess)
        return fail(nllb::set_error(NLLB_ATTN_ECUDA, "cuTensorMapEncodeTiled failed for the weight"));
    *out = L;
    return NLLB_ATTN_OK;
}

int nllb_linear_run(nllb_linear* L, const float* x, int M, float* out, const float* residual, int flags,
                    void* stream) {
    if (!L || !out || (M > 0 && !x)) return nllb::set_error(NLLB_ATTN_EINVAL, "layer, x and out required");
    if (M < 0) return nllb::set_error(NLLB_ATTN_EINVAL, "M >= 0");
    if (M == 0) return NLLB_ATTN_OK;
    if (reinterpret_cast<uintptr_t>(x) & 15) return nllb::set_error(NLLB_ATTN_EINVAL, "x must be 16-byte aligned");
    int dev = -1;
    LP_CK(cudaGetDevice(&dev));
    if (dev != L->device) return nllb::set_error(NLLB_ATTN_EINVAL, "the layer was prepared on another device");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    LinearArgs a;
    a.x = x;
    a.ldx = L->K;
    a.w = L->w;
    a.scale = L->scale;
    a.bias = L->bias;
    a.out = out;
    a.residual = residual;
    a.M = M;
    a.N = L->N;
    a.K = L->K;
    a.cblock = L->N;
    a.test_expire = L->expire_next ? 1 : 0;  // read by the split-K kernel only
    L->expire_next = false;
    a.relu = (flags & NLLB_LINEAR_RELU) ? 1 : 0;
    a.mask_from = -1;
    a.static_weights = 0;
    a.out_planes = nullptr;
    if (M <= 16) {
        LP_CK(launch_linear(a, nullptr, L->num_sms, L->err, st));
        return NLLB_ATTN_OK;
    }
    const size_t need = (size_t)M * L->K * kPlanes;
    if (need > L->planes_elems) {
        LP_CK(cudaStreamSynchronize(st));  // the previous planes may still be read
        if (L->planes) cudaFree(L->planes);
        L->planes = nullptr;
        L->planes_elems = 0;
        L->map_rows = -1;
        LP_CK(cudaMalloc(&L->planes, need * sizeof(plane_t)));
        L->planes_elems = need;
    }
    if (L->map_rows != M) {
        LP_CK(encode_half_map(&L->tx, L->planes, L->K, M, kPlanes));
        LP_CK(encode_half_maps_persistent(&L->tx_pers, L->planes, L->K, M, nullptr, nullptr, 0));
        L->map_rows = M;
    }
    LP_CK(launch_split_planes(x, L->K, M, L->K, L->planes, st));
    if (linear_tma_use_persistent(M, L->N, L->K, L->num_sms))
        LP_CK(launch_linear_tma_persistent(a, &L->tx_pers, &L->tm256, &L->tm_pair, L->num_sms, L->err, st));
    else
        LP_CK(launch_linear_tma(a, &L->tx, &L->tm, linear_tma_splits(M, L->N, L->K, L->num_sms), L->err, st));
    return NLLB_ATTN_OK;
}

int nllb_linear_test_expire_next_wait(nllb_linear* L) {
    if (!L) return nllb::set_error(NLLB_ATTN_EINVAL, "layer required");
    L->expire_next = true;
    return NLLB_ATTN_OK;
}

int nllb_linear_status(nllb_linear* L) {
    if (!L) return nllb::set_error(NLLB_ATTN_EINVAL, "layer required");
    int cur = 0, h = 0;
    LP_CK(cudaGetDevice(&cur));
    LP_CK(cudaSetDevice(L->device));
    LP_CK(cudaDeviceSynchronize());
    LP_CK(cudaMemcpy(&h, L->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) LP_CK(cudaMemset(L->err, 0, sizeof(int)));  // reported once; the layer stays usable
    cudaSetDevice(cur);
    if (h) return nllb::set_error(NLLB_ATTN_ETIMEOUT, "a bounded device wait of the linear kernel gave up");
    return NLLB_ATTN_OK;
}

}  // extern "C"
