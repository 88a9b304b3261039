/*  nllb_gpu_shim.h -- the thin layer between the reference's C host
 *  (main.c beam search, encoder.c, decoder.c; MetalNLLB) and libnllb_attn.
 *
 *  The reference program, rebuilt by integration/Makefile with its three
 *  attention loops and its KV-cache copies replaced by these calls, keeps
 *  everything else: its loader, its INT8 mat-vecs, LayerNorm, vocabulary
 *  projection, penalties, top-k, its per-beam thread pool and its beam
 *  search.  Force-included (-include) into every edited source.
 *
 *  Replaced call sites (reference file:line) and their replacement:
 *    encoder.c:165-205  attention loop of multi_head_self_attn_flash
 *                       -> nllb_gpu_encoder_attention (nllb_attn_prefill_host)
 *    decoder.c:61-96    cache append + attention of decoder_self_attn_cached
 *                       -> nllb_gpu_self_attention (nllb_attn_decode_self_host)
 *    decoder.c:127-149  attention of decoder_cross_attn_cached; the step-0
 *                       K/V projection into the shared cache (:115-125) stays
 *                       -> nllb_gpu_cross_attention (set_memory_host at step 0,
 *                          nllb_attn_cross_host)
 *    main.c:301         calloc of each per-beam KV cache -> nllb_gpu_beam_cache
 *                       (a small handle: the caches live on the GPU)
 *    main.c:338-339, 390-391  bootstrap cache copies -> nllb_gpu_copy_beam
 *    main.c:444         dispatch of the beam threads, preceded by
 *                       nllb_gpu_expect_beams (how many beams run this step)
 *    main.c:481-482     parent-cache copy per child -> nllb_gpu_stage_copy
 *                       (one nllb_attn_reorder_host before the next step)
 *
 *  The reference runs one thread per live beam (main.c:124-150) and each
 *  calls the decoder on its own cache.  The GPU calls take all beams at
 *  once, so the beam threads meet at each attention call: each leaves its
 *  q/k/v in its beam's slot, the last to arrive makes the call for all
 *  beams, and each takes its own output back.  Beams that do not run at a
 *  step (finished, or beams 1..3 at steps 0 and 1) compute on stale inputs
 *  in the same call; their outputs are not read and their cache rows are
 *  never reached by a live beam's history.
 *
 *  Any failure of the GPU path prints the library's message and exits the
 *  program (the reference's own error convention, encoder.c:78-81); there
 *  is no CPU fallback.
 */
#ifndef NLLB_GPU_SHIM_H
#define NLLB_GPU_SHIM_H

float* nllb_gpu_beam_cache(int pool, int beam);
void   nllb_gpu_copy_beam(const float* dst_cache, const float* src_cache);
void   nllb_gpu_stage_copy(const float* dst_cache, const float* src_cache);
void   nllb_gpu_expect_beams(int step, int n_beams);

void nllb_gpu_encoder_attention(const float* Q, const float* K, const float* V, float* head_out, int seq_len);
void nllb_gpu_self_attention(const float* kv_cache, int layer, int step, const float* q, const float* k,
                             const float* v, float* out);
void nllb_gpu_cross_attention(int layer, int step, int n_src, const float* K, const float* V, const float* q,
                              float* out);

#endif
