// attn_internal.h -- the attention context, shared by the C ABI (nllb_attn.cu)
// and the translation engine (engine.cu), which writes the encoder memory of
// many sentences in one launch.
#pragma once
#include <cstddef>
#include <vector>

#include <cuda_runtime.h>

#include "nllb_attn.h"

struct nllb_attn_ctx {
    int device = 0;
    int num_sms = 148;
    nllb_attn_dims d{};
    int Tp = 0;  // beam-history rows per sentence (max_tgt rounded up, +2 for 16-B copies)
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    float* kc = nullptr;  // [L][S][H][T][NB][64]
    float* vc = nullptr;
    unsigned char* hist = nullptr;      // [S][Tp][8], the current beam history
    unsigned char* hist_alt = nullptr;  // the other history buffer (a fused reorder writes it)
    // a reorder not applied yet: the next self-attention launch over all
    // max_sentences sentences applies it on the way (then the buffers swap);
    // anything else applies it with the reorder kernel first
    const int* pending_parent = nullptr;  // device [pending_n][n_beams]
    int pending_n = 0;
    bool expire_next_wait = false;  // test: the next self-attention launch's wait runs out
    bool expire_next_cross = false;  // test: the next cross-attention launch's wait runs out
    float* km = nullptr;  // [L][S][H][max_src][64]
    float* vm = nullptr;
    int* n_src_dev = nullptr;  // [L][S]
    std::vector<int> n_src_host;
    int* err = nullptr;
    // staging for *_host calls, grown on demand
    // (slot 6: reorder_host's parents, which a pending reorder may still read)
    void* stg[7] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    size_t stg_bytes[7] = {0, 0, 0, 0, 0, 0, 0};
    // pipelined host-buffer decode: input copies on copy_in, kernels on stream,
    // output copies on copy_out, chunk by chunk of sentences (created on first use)
// Measured on B200 (128 sentences x 4 beams, pinned buffers): 1 chunk 288 us
// per step, 2 chunks 254 us, 4 chunks 275 us, 8 chunks 314 us.
#ifndef NLLB_HOST_CHUNKS
#define NLLB_HOST_CHUNKS 2
#endif
    static constexpr int kHostChunks = NLLB_HOST_CHUNKS;
    cudaStream_t copy_in = nullptr, copy_out = nullptr;
    cudaEvent_t ev_in[kHostChunks] = {}, ev_k[kHostChunks] = {};
    cudaEvent_t ev_parent = nullptr;  // the last host parent copy has left par_h
    int* err_h = nullptr;             // pinned: device error word read with the outputs
    int* par_h = nullptr;             // pinned staging of reorder_host's parents
    size_t par_h_ints = 0;
};

namespace nllb {
// The engine's forms of nllb_attn_decode_self / nllb_attn_cross (device
// buffers): the output goes out as the two fp16 planes of the output
// projection's input (planes.cuh) at the fp32 output's element offsets, one
// plane per n_sent * n_beams * H * 64 elements.  Not exported.
int attn_decode_self_planes(nllb_attn_ctx* c, int layer, int step, int n_sent, const float* q, const float* k_new,
                            const float* v_new, void* planes);
int attn_cross_planes(nllb_attn_ctx* c, int layer, int n_sent, const float* q, void* planes);
// nllb_attn_prefill over packed rows: sequence b's row r at row_start[b] + r
// (device array; stride_batch unused); only its valid_len[b] >= 1 rows are
// read and written; the q/k/v buffers hold rows_total rows.  Not exported.
int attn_prefill_packed(nllb_attn_ctx* c, const nllb_attn_prefill_args* a, const int* row_start, int rows_total);
}  // namespace nllb
