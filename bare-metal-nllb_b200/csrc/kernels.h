// kernels.h -- launch parameters and launchers of the attention kernels.
// Host-side only types; shared by the C ABI (nllb_attn.cu) and the kernel
// translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace nllb {

// Cache rows (of 64 fp32 = 256 B) per bulk-copy chunk, and chunks in flight
// per CTA (ring depth), for the self-attention and the cross-attention
// kernels.  A self-attention chunk holds kSelfChunkRows / n_beams positions
// (all beams of each position), a cross-attention chunk 16 or 32 memory rows
// (cross_chunk_rows).  Measured on B200: 32 x 3 (4 CTAs per SM) for the
// self-attention stream; for cross-attention 16 x 3 when every memory of the
// call has at most 160 rows (1024 sentences of 18..130 rows: 127 us against
// 189 us for 64 x 2), 32 x 3 for longer memories (16 x 512 rows: 16.6 us
// against 24 us), and 64 x 2 when split-KV leaves each CTA at most 64 rows
// (one sentence of 512 rows: one chunk per split CTA, 6.2 us against 7.4).
#ifndef NLLB_SELF_CHUNK_ROWS
#define NLLB_SELF_CHUNK_ROWS 32
#endif
#ifndef NLLB_SELF_STAGES
#define NLLB_SELF_STAGES 3
#endif
constexpr int kSelfChunkRows = NLLB_SELF_CHUNK_ROWS;
constexpr int kSelfStages = NLLB_SELF_STAGES;
constexpr int kCrossShortRows = 16, kCrossLongRows = 32, kCrossSplitRows = 64, kCrossLongFrom = 160;
// Chunk rows for the longest memory of a call (the split plan may then move
// to kCrossSplitRows, see the cross-attention entry point).
inline int cross_chunk_rows(int max_len) { return max_len <= kCrossLongFrom ? kCrossShortRows : kCrossLongRows; }
static_assert(kSelfChunkRows % 16 == 0 && kSelfChunkRows >= 16, "chunk rows: multiple of 16");
static_assert(kSelfStages >= 1 && kSelfStages <= 16,
              "ring depth: 1..16 (the barrier block holds 16)");
inline int self_chunk_positions(int n_beams) { return kSelfChunkRows / n_beams; }
constexpr int kPartFloats = 68;  // split record per beam: m, l, pad, pad, acc[64]
// Split-KV CTAs of one (sentence, head) form one thread-block cluster.
constexpr int kMaxSplit = 8;

// ---- decoder self-attention (decode.cu) ----------------------------------
// Cache layout of one layer: [sentence][head][T][n_beams][64] fp32 for K and
// V; beam history hist[sentence][Tp][8] uint8: physical beam slot that holds
// position p of logical beam b.
struct SelfParams {
    const float* kc;      // layer base, K
    const float* vc;      // layer base, V
    float* kc_w;          // same as kc (written at `step`)
    float* vc_w;
    const uint8_t* hist;  // [S][Tp][8]
    uint8_t* hist_w;      // same buffer, written at `step` (head 0 only); the other
                          // history buffer in the reorder form (SelfParamsR)
    const float* q;       // [n_sent][n_beams][H*64]
    const float* k_new;
    const float* v_new;
    // fp32 output, or (launch_decode_self with planes) the two fp16 planes
    // of the output (x = p0 + p1, planes.cuh) at the same element
    // offsets, one plane per n_sent * n_beams * H * 64 elements: the A operand
    // of the output projection
    float* out;
    int H, T, Tp;
    int step;             // position of the new token; cache holds 0..step-1
    int n_split, pos_per_split;
    float scale_log2;     // scale * log2(e)
    int* err;
};

// (Adding fields to SelfParams changed the register allocation of the
// self-attention kernel -- 48 to 40 registers -- and cost 4 % of its stream
// rate on B200; the plane output therefore reuses `out`, and the reorder
// form below is a separate type that only its own instantiation takes.)

// A launch that applies a pending beam reorder on the way: logical beam b of
// sentence s reads position p from slot hist[p][parent[s*n_beams + b]] of the
// current history (hist) and the composed rows go to the other history
// buffer (hist_w), which becomes the current one.
struct SelfParamsR : SelfParams {
    const int* parent;  // [n_sent][n_beams], device
};

// Which form of the self-attention kernel a launch uses.
enum class SelfMode { plain = 0, reorder = 1, expire_wait = 2 };

// ---- cross-attention (decode.cu) ------------------------------------------
// Memory layout of one layer: [sentence][head][max_src][64] fp32, K and V.
struct CrossParams {
    const float* km;
    const float* vm;
    const int* n_src;     // [S] rows per sentence for this layer
    const float* q;       // [n_sent][n_beams][H*64]
    float* out;           // as in SelfParams
    int H, max_src;
    int n_split, pos_per_split;
    float scale_log2;
    int* err;
};

// ---- prefill (prefill.cu) -------------------------------------------------
struct PrefillParams {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    int B, H, S;
    long long sb, sh, sr;
    const int* valid_len;
    const float* mask;
    long long msb, msh;
    float scale_log2;
    int* err;
    // packed rows (optional): sequence b's row r is at row_start[b] + r (its
    // base is row_start[b] * sr + h * sh, sb unused); only its valid_len[b]
    // rows are read and written, so sequences may lie back to back
    const int* row_start;
    int rows_total;  // packed rows: rows in the q/k/v buffers (the tensor maps' extent)
    // (set by the launcher) positions 0..2 of the row, head and sequence axes
    // among the outer axes of the tensor-core kernel's tensor maps
    int map_pos_row, map_pos_head, map_pos_seq;
};

// cuTensorMapEncodeTiled from the driver (nullptr if unavailable); linear_tma.cu.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Per-device kernel attributes (dynamic shared memory); call once per device.
cudaError_t configure_decode_kernels();
cudaError_t configure_prefill_kernels();

// planes: p.out is the base of the output planes (see SelfParams::out).
// mode reorder: `parent` is the pending reorder (SelfParamsR::parent) and
// p.hist_w the other history buffer.  mode expire_wait: the bounded-wait
// test (4 beams, fp32 output only).
cudaError_t launch_decode_self(const SelfParams& p, int n_sent, int n_beams, cudaStream_t st, bool planes = false,
                               SelfMode mode = SelfMode::plain, const int* parent = nullptr);
// chunk_rows: cross_chunk_rows(longest memory of the call)
// expire_wait: the bounded-wait test form (4 beams, fp32 output, 16-row chunks)
cudaError_t launch_cross(const CrossParams& p, int n_sent, int n_beams, int chunk_rows, cudaStream_t st,
                         bool planes = false, bool expire_wait = false);
cudaError_t launch_reorder(uint8_t* hist, int Tp, const int* parent, int n_sent, int n_beams,
                           int* err, cudaStream_t st);
cudaError_t launch_hist_init(uint8_t* hist, int Tp, int n_sent, cudaStream_t st);
cudaError_t launch_set_memory(float* km, float* vm, int max_src, int H, const float* k,
                              const float* v, long long stride_head, long long stride_row,
                              int n_src, int* n_src_slot, cudaStream_t st);
cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t st);
// attention_head's softmaxed score matrix (tensor.c:258-277): p [S][S] from
// q, k [S][64] and an additive mask [S][S] (may be null).
cudaError_t launch_head_scores(const float* q, const float* k, const float* mask, float* p, int S, float scale,
                               cudaStream_t st);
// seq_len range served by the tcgen05 kernel (others: FFMA kernel)
bool prefill_uses_tensor_cores(int seq_len);

}  // namespace nllb
