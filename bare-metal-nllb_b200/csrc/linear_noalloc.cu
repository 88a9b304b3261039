// linear_noalloc.cu -- the INT8-weight linear layer with no device allocation.
//
// nllb_linear_int8 grows a per-device split-K workspace with cudaMalloc the
// first time a shape needs it.  Some callers cannot let a library allocate in
// the middle of their work: a serving process that carves all device memory
// into its own pool at start-up (a run-time cudaMalloc then fails, or takes
// memory the pool's accounting does not know about), or a decode loop with a
// fixed memory plan where cudaMalloc's implicit device synchronisation would
// stall the other streams.  nllb_linear_int8_noalloc serves them: its split-K
// workspace, tile counters and error word live in one fixed-size
// __device__ array of this file, which every GPU that loads the library holds
// until the process exits (8 MB + 1 KB).
//
// Properties a caller relies on:
//   * no cudaMalloc, cudaFree or allocating library call, ever;
//   * the first call on a device looks the array's device address up with
//     cudaGetSymbolAddress (that device current) and remembers it; make that
//     first call before any stream capture;
//   * all calls share the array, which keeps the last call's contents: each
//     call clears the tile counters on its stream first, and two calls whose
//     kernels overlap on the GPU (different streams, no ordering between
//     them) race on the workspace and give wrong results;
//   * the error word is sticky: a bounded wait that gave up sets it and no
//     later call clears it; nllb_linear_int8_noalloc_status reads and clears
//     it (also without allocating);
//   * the device address and the SM count are kept per device ordinal for the
//     life of the process: a device reset (cudaDeviceReset) after the first
//     call is not supported;
//   * shapes beyond NLLB_LINEAR_NOALLOC_MAX_ROWS x _MAX_OUT x _MAX_IN are
//     rejected with NLLB_ATTN_ECAPACITY.
#include <mutex>
#include <string>

#include "engine_kernels.h"
#include "nllb_translate.h"

namespace nllb {
int set_error(int status, const std::string& msg);  // nllb_attn.cu
}

using namespace nllb;

namespace {

// Workspace for 128 partial 128x128 tiles, then 256 tile counters and the
// error word (as ints).
constexpr size_t kWsFloats = (size_t)128 * 128 * 128;
constexpr int kCounters = 256;
constexpr size_t kScratchFloats = kWsFloats + kCounters + 64;
constexpr int kMaxPartialTiles = 128;

static __device__ __align__(256) float g_linear_scratch[kScratchFloats];

std::mutex g_mu;
float* g_scratch_dev[64] = {nullptr};  // device address of g_linear_scratch, per device
int g_num_sms[64] = {0};               // multiprocessor count, per device

int scratch_address(int dev, float** out, int* num_sms) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_dev[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_linear_scratch);
        if (e != cudaSuccess)
            return nllb::set_error(NLLB_ATTN_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        int nsm = 0;
        e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || nsm < 1)
            return nllb::set_error(NLLB_ATTN_ECUDA, "cannot read the multiprocessor count");
        if (configure_linear_tc() != cudaSuccess)
            return nllb::set_error(NLLB_ATTN_ECUDA, "cannot configure the tensor-core linear kernel");
        g_num_sms[dev] = nsm;
        g_scratch_dev[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_dev[dev];
    *num_sms = g_num_sms[dev];
    return NLLB_ATTN_OK;
}

int current_device(int* dev) {
    if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= 64)
        return nllb::set_error(NLLB_ATTN_ENODEV, "no current CUDA device (ordinal 0..63)");
    return NLLB_ATTN_OK;
}

}  // namespace

extern "C" int nllb_linear_int8_noalloc(const float* x, int M, int K, const int8_t* w, const float* weight_scale,
                                        const float* bias, int N, float* out, const float* residual, int flags,
                                        void* stream) {
    if (!x || !w || !weight_scale || !out) return nllb::set_error(NLLB_ATTN_EINVAL, "x, w, weight_scale, out required");
    if (M < 0 || K < 4 || N < 1 || (K & 3)) return nllb::set_error(NLLB_ATTN_EINVAL, "M >= 0, N >= 1, K a multiple of 4");
    if (M > NLLB_LINEAR_NOALLOC_MAX_ROWS || N > NLLB_LINEAR_NOALLOC_MAX_OUT || K > NLLB_LINEAR_NOALLOC_MAX_IN)
        return nllb::set_error(NLLB_ATTN_ECAPACITY,
                               "nllb_linear_int8_noalloc takes at most 256 rows, 4096 outputs and 4096 inputs "
                               "(fixed 8 MB scratch)");
    if (M > 16 && K % 32) return nllb::set_error(NLLB_ATTN_EINVAL, "K must be a multiple of 32 beyond 16 rows");
    int dev = 0, nsm = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    float* scratch = nullptr;
    rc = scratch_address(dev, &scratch, &nsm);
    if (rc) return rc;
    float* ws = scratch;
    int* counters = reinterpret_cast<int*>(scratch + kWsFloats);
    int* err = counters + kCounters;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (M == 0) return NLLB_ATTN_OK;

    LinearArgs a;
    a.x = x;
    a.ldx = K;
    a.w = w;
    a.scale = weight_scale;
    a.bias = bias;
    a.out = out;
    a.residual = residual;
    a.M = M;
    a.N = N;
    a.K = K;
    a.cblock = N;
    a.relu = (flags & NLLB_LINEAR_RELU) ? 1 : 0;
    a.mask_from = -1;
    a.static_weights = 0;
    a.out_planes = nullptr;

    cudaError_t e = cudaMemsetAsync(counters, 0, kCounters * sizeof(int), st);
    if (e != cudaSuccess) return nllb::set_error(NLLB_ATTN_ECUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    if (M <= 16 || !linear_tc_supports(a)) {
        // SIMT paths (at most 16 rows; K not a multiple of 64: the tiled kernel): no scratch
        e = launch_linear(a, nullptr, nsm, err, st);
    } else {
        const int tiles = (int)linear_tc_tiles(a);
        int splits = linear_tc_splits(a, nsm);
        if (splits * tiles > kMaxPartialTiles) splits = kMaxPartialTiles / tiles;
        if (splits < 1) splits = 1;
        e = launch_linear_tc(a, splits, ws, counters, err, st);
    }
    if (e != cudaSuccess) return nllb::set_error(NLLB_ATTN_ECUDA, std::string("launch: ") + cudaGetErrorString(e));
    return NLLB_ATTN_OK;
}

extern "C" int nllb_linear_int8_noalloc_status(void* stream) {
    int dev = 0, nsm = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    float* scratch = nullptr;
    rc = scratch_address(dev, &scratch, &nsm);
    if (rc) return rc;
    int* err = reinterpret_cast<int*>(scratch + kWsFloats) + kCounters;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(err, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return nllb::set_error(NLLB_ATTN_ECUDA, std::string("status: ") + cudaGetErrorString(e));
    if (h) return nllb::set_error(NLLB_ATTN_ETIMEOUT, "a bounded device wait of the linear kernel gave up");
    return NLLB_ATTN_OK;
}
