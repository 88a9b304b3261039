// kernels.h -- launch parameters and launchers of the attention kernels.
// Host-side only types; shared by the C ABI (nllb_attn.cu) and the kernel
// translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace nllb {

// Positions per bulk-copy chunk of the self-attention cache:
// 64 cache rows (of 64 fp32) per chunk whatever the beam count.
inline int self_chunk_positions(int n_beams) { return 64 / n_beams; }
constexpr int kCrossChunkRows = 64;
constexpr int kPartFloats = 68;  // split record per beam: m, l, pad, pad, acc[64]

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
    uint8_t* hist_w;      // same buffer, written at `step` (head 0 only)
    const float* q;       // [n_sent][n_beams][H*64]
    const float* k_new;
    const float* v_new;
    float* out;
    int H, T, Tp;
    int step;             // position of the new token; cache holds 0..step-1
    int n_split, pos_per_split;
    float scale_log2;     // scale * log2(e)
    float* part;          // split records [n_sent*H][n_split][n_beams][68]
    int* counters;        // [n_sent*H]
    int* err;
};

// ---- cross-attention (decode.cu) ------------------------------------------
// Memory layout of one layer: [sentence][head][max_src][64] fp32, K and V.
struct CrossParams {
    const float* km;
    const float* vm;
    const int* n_src;     // [S] rows per sentence for this layer
    const float* q;       // [n_sent][n_beams][H*64]
    float* out;
    int H, max_src;
    int n_split, pos_per_split;
    float scale_log2;
    float* part;
    int* counters;
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
};

// Per-device kernel attributes (dynamic shared memory); call once per device.
cudaError_t configure_decode_kernels();
cudaError_t configure_prefill_kernels();

cudaError_t launch_decode_self(const SelfParams& p, int n_sent, int n_beams, cudaStream_t st);
cudaError_t launch_cross(const CrossParams& p, int n_sent, int n_beams, cudaStream_t st);
cudaError_t launch_reorder(uint8_t* hist, int Tp, const int* parent, int n_sent, int n_beams,
                           int* err, cudaStream_t st);
cudaError_t launch_hist_init(uint8_t* hist, int Tp, int n_sent, cudaStream_t st);
cudaError_t launch_set_memory(float* km, float* vm, int max_src, int H, const float* k,
                              const float* v, long long stride_head, long long stride_row,
                              int n_src, cudaStream_t st);
cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t st);

}  // namespace nllb
