// engine_kernels.h -- launchers of the translation engine's non-attention kernels.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace nllb {

// out = epilogue(x[M][K] . (w[N][K] / scale[N])^T + bias), see engine_kernels.cu
struct LinearArgs {
    const float* x;
    int ldx;                 // row stride of x (elements)
    const int8_t* w;         // [N][K] int8
    const float* scale;      // [N] CT2 weight_scale: weight = int8 * (1.0f / scale)
    const float* bias;       // [N] or null
    float* out;
    const float* residual;   // same addressing as out, or null
    int M, N, K;
    int cblock;              // output column block (N for row-major)
    int relu;
    int mask_from;           // columns >= mask_from are set to -1e30 (-1: none)
    int static_weights;      // 1: w, scale, bias are not written by earlier kernels of the stream
                             // (a kernel may fetch them before waiting for its predecessor)
    void* out_planes;        // TMA kernels only: write fp16 planes [2][M][N] (planes.cuh split of the result)
                             // instead of out; requires cblock == N and no residual
    int test_expire = 0;     // split-K TMA kernel only: the MMA issuer first waits ~1 ms on a barrier nothing
                             // arrives on, so that the launch takes its timeout path (tests of the bounded waits)
};

cudaError_t launch_embed_pos(float* x, const int* tokens, const int* positions, int pos_const, const int8_t* emb,
                             const float* emb_inv_scale, const float* pos_table, float embed_scale, int rows,
                             int vocab, cudaStream_t st);
// out (fp32, may be null) and/or planes (fp16 [2][rows][1024], may be null)
cudaError_t launch_layernorm(float* out, float* x, const float* res, const float* gamma, const float* beta,
                             int rows, void* planes, cudaStream_t st);
// Split-K workspace of the tensor-core linear kernel: partial tiles and one
// arrival counter per output tile (zero between calls).
struct LinearWorkspace {
    float* ws = nullptr;
    size_t ws_floats = 0;
    int* tile_count = nullptr;
    size_t n_counters = 0;
};

// Dispatch: <= 16 rows skinny SIMT kernel, else the tcgen05 kernel (K % 64 == 0;
// split-K when the output has fewer tiles than twice the SMs and the workspace
// is large enough) or the tiled SIMT kernel.  err: device error word.
cudaError_t launch_linear(const LinearArgs& a, const LinearWorkspace* wsp, int num_sms, int* err, cudaStream_t st);
cudaError_t configure_linear_tc();
bool linear_tc_supports(const LinearArgs& a);
int linear_tc_splits(const LinearArgs& a, int num_sms);
size_t linear_tc_workspace_floats(const LinearArgs& a, int splits);
size_t linear_tc_tiles(const LinearArgs& a);
cudaError_t launch_linear_tc(const LinearArgs& a, int splits, float* ws, int* tile_count, int* err,
                             cudaStream_t st);
// TMA-fed tcgen05 linear layer over fp16 operands (linear_tma.cu): weights
// kept as an fp16 copy of the int8 matrix, activations split into two fp16
// planes [2][M][K] by launch_split_planes.  K % 64 == 0, K >= 64.
cudaError_t configure_linear_tma();
cudaError_t encode_half_map(CUtensorMap* map, const void* base, int cols, int rows, int planes);
int linear_tma_splits(int M, int N, int K, int num_sms);
// Persistent 128 x 256-tile form (K % 32 == 0), used when the output has
// enough tiles for its K (linear_tma_use_persistent); its tensor maps: planes box 32 x 128 x 2,
// weight box 32 x 256 (64-byte swizzle).  Either map pointer may be null.
bool linear_tma_use_persistent(int M, int N, int K, int num_sms);
cudaError_t encode_half_maps_persistent(CUtensorMap* x_map, const void* planes, int K, int M, CUtensorMap* w_map,
                                        const void* wb, int N);
// From 129 rows and 2 * num_sms tiles of 128 x 256 the launch runs 256 x 256
// tiles on CTA pairs (cta_group::2) when tw_pair is given: the weight's map
// with box 32 x 128 (64-byte swizzle, encode_half_map_pair); the planes map is
// the same.
bool linear_tma_use_pair(int M, int N, int num_sms);
cudaError_t encode_half_map_pair(CUtensorMap* map, const void* wb, int K, int N);
cudaError_t launch_linear_tma_persistent(const LinearArgs& a, const CUtensorMap* tx, const CUtensorMap* tw,
                                         const CUtensorMap* tw_pair, int num_sms, int* err, cudaStream_t st);
cudaError_t launch_split_planes(const float* x, int ldx, int M, int K, void* planes, cudaStream_t st);
cudaError_t launch_int8_to_f16(const int8_t* w, void* out, size_t n, cudaStream_t st);
cudaError_t launch_linear_tma(const LinearArgs& a, const CUtensorMap* tx, const CUtensorMap* tw, int splits, int* err,
                              cudaStream_t st);
cudaError_t launch_penalties(float* logits, size_t ld, const int* hist, int hist_ld, const int* n_tokens,
                             const unsigned char* active, int rows, float penalty, int ngram, cudaStream_t st);
// ws: vocab_topk_ws_floats(V, rows, k) floats of scratch
size_t vocab_topk_ws_floats(int V, int rows, int k);
cudaError_t launch_logsoftmax_topk(const float* logits, size_t ld, int V, int rows, const unsigned char* active,
                                   int k, int* out_tok, float* out_logp, float* ws, cudaStream_t st);
// row_start (optional): sentence s's rows start at row_start[s] (packed), else at s * sent_stride
cudaError_t launch_set_memory_batched(float* km, float* vm, int* n_src_slots, int max_src, int H, const float* k,
                                      const float* v, long long sent_stride, const int* row_start,
                                      const int* n_src, int n_sent, int max_n, cudaStream_t st);
cudaError_t launch_reciprocal(float* out, const float* in, size_t n, cudaStream_t st);

// Beam-search state of a translate call on the device (4 beams per sentence,
// G = positions per beam), updated by launch_beam_select after every step.
struct BeamState {
    int* bt0;                // [rows][G] token histories, two buffers: step parity `cur` reads
    int* bt1;                //   bt0 (cur 0) or bt1 (cur 1) and writes the other
    int* bn;                 // [rows] tokens per beam
    float* bsc;              // [rows] beam score
    float* beos;             // [rows] score at the step that emitted token 2
    unsigned char* bfin;     // [rows] finished
    unsigned char* done;     // [sentences] no further step
    const int* maxo;         // [sentences] max_out (main.c:315-316)
    int* ctok;               // [sentences][8][G] completed hypotheses
    int* cn;                 // [sentences][8]
    float* csc;              // [sentences][8]
    float* ceos;             // [sentences][8]
    int* ccnt;               // [sentences]
    float* margins;          // [sentences][G] smallest gap among the best 5 candidates, per step
    int* mcnt;               // [sentences]
    int* tok;                // [rows] last token (next step's input)
    unsigned char* active;   // [rows] unfinished beam of a running sentence
    int* parent;             // [rows] parent beam of each new beam
    int* live;               // [G] running sentences after each step (zeroed before the loop)
    int G, n_sent;
};
cudaError_t launch_beam_select(const BeamState& b, int cur, const int* top_tok, const float* top_lp, int step,
                               cudaStream_t st);

}  // namespace nllb
