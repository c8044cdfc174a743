/*
 * fpx — B200-native (sm_100a) block-sparse prefill attention with block-mean K/V correction.
 *
 * The C ABI of libfpx.so. Every entry point takes raw device pointers, sizes and
 * element strides, launches on the given CUDA stream, never allocates device
 * memory, never synchronises, and returns an fpx_status (0 = ok, negative =
 * error; fpx_status_string() names it). Where a reference op mutates nothing
 * and returns fresh tensors, the caller passes the output buffers.
 *
 * Layouts follow the reference's public entry points (exp3 attention.py:211-213
 * makes them contiguous): q [B, L, H, d], k / v [B, L, Hkv, d] bf16 with the
 * last dimension contiguous and the other three strides given in elements;
 * block scores [B, nb, nb, H] fp32 (query block, key block, head); block index
 * lists [B, nb, nb, H] int64 ascending with sentinel nb; counts [B, nb, H] int32;
 * masks [B, nb, nb, H] uint8 (0/1, torch.bool storage). nb = ceil(L / block).
 * Only block = 128 and head dim d in {128, 256} are compiled; other values
 * return FPX_ERR_UNSUPPORTED.
 *
 * Reference file:line citations are to the exp3 tree; "upstream" means
 * upstream/flashprefill_native_forward.py.
 */
#ifndef FPX_H_
#define FPX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *fpx_stream_t; /* a cudaStream_t; NULL = legacy default stream */

enum fpx_status {
  FPX_OK = 0,
  FPX_ERR_INVALID = -1,     /* bad argument (null pointer, non-positive size, unknown enum) */
  FPX_ERR_SHAPE = -2,       /* inconsistent shapes (H not a multiple of Hkv, ranges out of bounds) */
  FPX_ERR_UNSUPPORTED = -3, /* head_dim / block size / method not compiled */
  FPX_ERR_CUDA = -4,        /* a CUDA launch failed; cudaGetLastError() has the cause */
  FPX_ERR_WORKSPACE = -5,   /* workspace too small or misaligned (256 B) */
  FPX_ERR_TIMEOUT = -6      /* a bounded device-side wait gave up (see fpx_device_error) */
};

/* attention.py:15-24 METHODS, in order. */
enum fpx_method {
  FPX_METHOD_DENSE = 0,
  FPX_METHOD_FP_V1 = 1,
  FPX_METHOD_MEAN_NATIVE = 2,
  FPX_METHOD_MEAN_BALANCED = 3,
  FPX_METHOD_CGF_MEAN = 4,
  FPX_METHOD_DISPERSION_MEAN = 5,
  FPX_METHOD_FP_V1_RESCUE = 6,   /* V1 routing + exact + rescue-token tail (kernels.py:233-309) */
  FPX_METHOD_FP_V1_RESCUE_V2 = 7 /* the same, plus the remainder means (remainder=True) */
};

/* Stage bits for fpx_prefill_attention (the profile stages of attention.py:66-75). */
enum fpx_stage {
  FPX_STAGE_ROUTE = 1, /* "descriptor" + "selector" + "indices" */
  FPX_STAGE_EXACT = 2, /* "exact" */
  FPX_STAGE_MEAN = 4,  /* "mean" + "merge" (fused) */
  FPX_STAGE_ALL = 7
};

const char *fpx_status_string(int status);
int fpx_version(void);

/* Process-wide options (no reference counterpart). Key 1 selects the exact-attention kernel of
 * fpx_prefill_attention and fpx_exact_attention at head dim 128: 0 = tcgen05/TMEM/TMA, two
 * query tiles per CTA (default), 1 = mma.sync (cross-check), 2 = tcgen05, one query tile per
 * CTA with double-buffered S (the kernel head dim 256 always uses). Key 2 sets how many of
 * every 8 exp2 pairs the tcgen05 kernel evaluates with an FMA-pipe polynomial instead of the
 * special-function unit: 0 (default), 2 or 3. Key 3 selects the V1 routing kernel
 * (fpx_prefill_attention and fpx_v1_scores): 0 = tcgen05, transposed block-mean x Q products
 * in TMEM (default), 1 = mma.sync (cross-check). Key 4 selects the tail kernels of
 * fpx_prefill_attention: 0 = tcgen05 (default; block means as bf16 high + low halves, rescue
 * rows gathered into swizzled tiles), 1 = fp32 CUDA cores (cross-check). Key 5 selects the
 * routing kernel of the new selectors in fpx_prefill_attention: 0 = tcgen05, descriptors as
 * bf16 high + low halves, two passes (default), 1 = fp32 CUDA cores (cross-check). */
int fpx_set_option(int key, int value);

/* Reads (and with reset != 0 clears) the device error word set when a bounded wait inside a
 * kernel gave up (1 = wait timeout); synchronous. No reference counterpart. */
int fpx_device_error(int *code, int reset);

/* ---- routing ------------------------------------------------------------------------ */
/* Head dim d = 128 or 256 (the Qwen3.5 shape) for every attention entry point: routing,
 * descriptors, selectors, exact attention, the tails, the merge, prefill_attention with every
 * method, and decode. (At 256 the selector routing and the tails run on fp32 kernels.) */

/* upstream:420-442 block_mean_k (compute_mean_vector upstream:27-69): bf16 mean of the
 * valid K rows of each (block, KV head) -> mean_k bf16 [B, nb, Hkv, d] contiguous.
 * Sum order: fp32, rows in sequence; fp32 division by the row count; RNE to bf16. */
int fpx_block_mean_k(const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                     int B, int L, int Hkv, int d, int block, void *mean_k, fpx_stream_t stream);

/* kernels.py:22-46 block_descriptors: fp32 mean_k, mean_v, var_k [B, nb, Hkv, d],
 * sigma_v [B, nb, Hkv], counts [nb] int32. */
int fpx_block_descriptors(const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                          const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                          int B, int L, int Hkv, int d, int block,
                          float *mean_k, float *mean_v, float *var_k, float *sigma_v,
                          int32_t *counts, fpx_stream_t stream);

/* upstream:445-475 v1_scores (compute_block_score upstream:89-175 + normalize_scores
 * upstream:410-417): normalised V1 proxy scores [B, nb, nb, H] fp32 from bf16 mean_k. */
int fpx_v1_scores(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                  const void *mean_k, int B, int L, int H, int Hkv, int d, int block,
                  double scale, float *scores, fpx_stream_t stream);

/* upstream:357-407 deal_output_score: keep = score >= alpha * max (or the min_budget
 * top-k rule, upstream:368-371; ties broken towards the lower block id), OR the
 * sink / window / last-blocks protection, AND causal -> ascending int64 indices with
 * sentinel nb and int32 counts. */
int fpx_deal_output_score(const float *scores, int B, int nb, int H, int sink, int window,
                          double alpha, int last_full, int min_budget,
                          int64_t *indices, int32_t *counts, fpx_stream_t stream);

/* kernels.py:49-126 selector_scores for selector = FPX_METHOD_MEAN_BALANCED,
 * FPX_METHOD_CGF_MEAN or FPX_METHOD_DISPERSION_MEAN -> [B, nb, nb, H] fp32. */
int fpx_selector_scores(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                        const float *mean_k, const float *var_k, const float *sigma_v,
                        const int32_t *counts, int B, int L, int H, int Hkv, int d, int block,
                        int selector, double scale, float *scores, fpx_stream_t stream);

/* kernels.py:129-151 protected_selection -> mask [B, nb, nb, H] uint8. */
int fpx_protected_selection(const float *scores, int B, int nb, int H, double alpha, int sink,
                            int window, int last_full, uint8_t *selected, fpx_stream_t stream);

/* kernels.py:154-160 indices_from_mask and kernels.py:163-176 mask_from_indices. */
int fpx_indices_from_mask(const uint8_t *selected, int B, int nb, int H,
                          int64_t *indices, int32_t *counts, fpx_stream_t stream);
int fpx_mask_from_indices(const int64_t *indices, const int32_t *counts, int B, int nb, int H,
                          uint8_t *selected, fpx_stream_t stream);

/* kernels.py:328-407 selection_accounting, device part: counters[0] = exact token pairs,
 * counters[1] = selected block entries, counters[2] = mean proxy entries (int64). */
int fpx_selection_accounting(const uint8_t *selected, int B, int nb, int H, int L, int block,
                             int64_t *counters, fpx_stream_t stream);

/* ---- exact path, mean tail, merge ---------------------------------------------------- */

/* upstream:478-521 exact_attention (_flash_forward upstream:215-354): block-sparse causal
 * attention over the listed blocks -> out bf16 [B, L, H, d] contiguous, lse fp32 [B, L, H]
 * natural log. */
int fpx_exact_attention(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                        const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                        const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                        const int64_t *indices, const int32_t *counts,
                        int B, int L, int H, int Hkv, int d, int block, double scale,
                        void *out, float *lse, fpx_stream_t stream);

/* kernels.py:179-230 mean_tail: unselected strictly-earlier blocks through fp32 block
 * means (+ log count) -> out fp32 [B, L, H, d], lse fp32 [B, L, H] (-inf without tail). */
int fpx_mean_tail(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                  const float *mean_k, const float *mean_v, const int32_t *counts,
                  const uint8_t *selected, int B, int L, int H, int Hkv, int d, int block,
                  double scale, float *out, float *lse, fpx_stream_t stream);

/* kernels.py:233-309 rescue_tail: for every unselected full-history block of each (query tile,
 * head), exact attention to its rescue token (the key maximising the tile's mean query . k,
 * ties to the first), and with remainder != 0 also to the block's other 127 tokens through
 * their mean with weight ln 127 -> out fp32 [B, L, H, d], lse fp32 [B, L, H] (-inf without
 * tail). selected is the [B, nb, nb, H] bool mask. The workspace (fpx_rescue_tail_workspace_bytes,
 * 256-byte aligned) holds the choices and the block means; reused across calls. */
size_t fpx_rescue_tail_workspace_bytes(int B, int L, int H, int Hkv, int d, int block);
int fpx_rescue_tail(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh, const void *k, int64_t k_sb,
                    int64_t k_sl, int64_t k_sh, const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                    const uint8_t *selected, int B, int L, int H, int Hkv, int d, int block, double scale,
                    int remainder, float *out, float *lse, void *workspace, size_t workspace_bytes,
                    fpx_stream_t stream);

/* kernels.py:312-325 merge_exact_mean over rows = B * L * H rows of d: out (bf16, the
 * exact output's dtype) and lse fp32. */
int fpx_merge_exact_mean(const void *exact_out, const float *exact_lse, const float *mean_out,
                         const float *mean_lse, int64_t rows, int d, void *out, float *lse,
                         fpx_stream_t stream);

/* ---- one-shot all-reduce over NVLink peer memory (no reference counterpart) -------- */
/* For the tensor-parallel decode step's small all-reduces. Each rank creates one buffer of
 * fpx_ar_buffer_bytes(max_elems) (fpx_ar_create: cudaMalloc'd and zeroed, with its CUDA IPC
 * handle, 64 bytes), the ranks exchange handles and map their peers' buffers (fpx_ar_open), and
 * every rank then calls fpx_allreduce_bf16 with the world's buffer bases in rank order (its own
 * at index rank; at most 8 ranks). A call stores the rank's input and a flag into every rank's
 * buffer, polls the flags of its own buffer and sums its own slots. The sum is taken in rank
 * order in fp32, so all ranks get the same bits; the call counter lives in the buffer, so calls
 * can be captured in a CUDA graph. Waits for peers
 * are bounded; a wait that gives up sets the buffer's error word (fpx_ar_error) and later calls
 * return at once. Set-up allocates; the calls do not. */
size_t fpx_ar_buffer_bytes(int max_elems);
int fpx_ar_create(size_t bytes, void **base, void *ipc_handle);
int fpx_ar_open(const void *ipc_handle, void **peer_base);
int fpx_ar_close(void *peer_base);
int fpx_ar_destroy(void *base);
int fpx_ar_error(const void *base, int *code);
int fpx_allreduce_bf16(void *inout, int64_t n, void *const *bases, int rank, int world, int max_elems,
                       fpx_stream_t stream);

/* ---- the fused prefill path (attention.py:210-333) ---------------------------------- */

/* Device bytes of workspace fpx_prefill_attention needs (256-byte aligned). */
size_t fpx_prefill_workspace_bytes(int method, int B, int L, int H, int Hkv, int d, int block);

/* The prefill branch of AttentionBackend.forward (attention.py:210-333) for the KV heads
 * [kv_begin, kv_end) and query tiles [tile_begin, tile_end) (pass 0, Hkv, 0, nb for all):
 * route -> exact -> mean + merge. out bf16 with element strides (o_sb, o_sl, o_sh);
 * lse fp32 [B, L, H] or NULL. `stages` (fpx_stage bits) runs a subset of the stages on
 * the same workspace, so each can be timed; a later stage needs the earlier ones' output
 * in the workspace. */
int fpx_prefill_attention(int method, double alpha, int sink, int window, int last_full,
                          const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                          const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                          const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                          int B, int L, int H, int Hkv, int d, int block, double scale,
                          int kv_begin, int kv_end, int tile_begin, int tile_end,
                          void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh, float *lse,
                          void *workspace, size_t workspace_bytes, int stages,
                          fpx_stream_t stream);

/* Copies the routing result of the last fpx_prefill_attention on this workspace (run over
 * all KV heads and tiles) out in the reference's layouts: selected mask uint8
 * [B, nb, nb, H] and, if non-NULL, ascending int64 indices [B, nb, nb, H] with sentinel nb
 * and int32 counts [B, nb, H]. */
int fpx_prefill_export_routing(int method, int B, int L, int H, int Hkv, int d, int block,
                               const void *workspace, size_t workspace_bytes,
                               uint8_t *selected, int64_t *indices, int32_t *counts,
                               fpx_stream_t stream);

/* ---- the Qwen2 decoder layer around attention (the model exp3 drives) ------------------ */

/* Residual add + RMSNorm over rows of `hidden` bf16 (HF Qwen2RMSNorm rounding): with residual
 * non-NULL, s = residual + x (bf16) is written to residual_out (may alias residual) and
 * normalised; out = weight * bf16(s * rsqrt(mean(s^2) + eps)). */
int fpx_rmsnorm(const void *x, const void *residual, const void *weight, double eps, int64_t rows, int hidden,
                void *out, void *residual_out, fpx_stream_t stream);

/* NeoX rotary embedding in place on a strided [B, L, heads, 128] bf16 view, positions
 * pos0 .. pos0 + L - 1, inv_freq = theta^(-2i/128) (HF apply_rotary_pos_emb rounding). */
int fpx_rope_neox(void *x, int64_t x_sb, int64_t x_sl, int64_t x_sh, int B, int L, int heads, int d, int pos0,
                  double theta, fpx_stream_t stream);
/* fpx_rope_neox with the position of row 0 read from device memory (no reference counterpart;
 * for captured decode steps). */
int fpx_rope_neox_at(void *x, int64_t x_sb, int64_t x_sl, int64_t x_sh, int B, int L, int heads, int d,
                     const int32_t *pos0, double theta, fpx_stream_t stream);

/* SwiGLU: out[r, j] = silu(gate_up[r, j]) * gate_up[r, inter + j] (bf16, HF Qwen2MLP rounding). */
int fpx_silu_mul(const void *gate_up, int64_t rows, int inter, void *out, fpx_stream_t stream);

/* ---- dense decode (attention.py:178-189) --------------------------------------------- */
/* Head dim d = 128 or 256 (the Qwen3.5 shape); at most 16 query heads per KV head. */

/* Device bytes of workspace fpx_decode_attention needs. */
size_t fpx_decode_workspace_bytes(int B, int Lq, int H, int Hkv, int S, int d);

/* The decode branch of AttentionBackend.forward (attention.py:178-189: q_len != k_len, so
 * F.scaled_dot_product_attention(is_causal=False, enable_gqa=True)): every query row of
 * q [B, Lq, H, d] attends to all S keys of k / v [B, S, Hkv, d] (strided views of HF's
 * [B, Hkv, S, d] cache are fine) -> out bf16 with element strides, lse fp32 [B, Lq, H] or
 * NULL. Split-K over the cache; H / Hkv <= 16. */
int fpx_decode_attention(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                         const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                         const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                         int B, int Lq, int S, int H, int Hkv, int d, double scale,
                         void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh, float *lse,
                         void *workspace, size_t workspace_bytes, fpx_stream_t stream);

/* fpx_decode_attention with the key count read from device memory (*S_keys <= S_max, no
 * reference counterpart): the launches do not change between decode steps, so a step can be
 * captured once in a CUDA graph and replayed. The workspace is sized for S_max. */
int fpx_decode_attention_at(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh, const void *k, int64_t k_sb,
                            int64_t k_sl, int64_t k_sh, const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                            int B, int Lq, int S_max, const int32_t *S_keys, int H, int Hkv, int d, double scale,
                            void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh, float *lse, void *workspace,
                            size_t workspace_bytes, fpx_stream_t stream);

/* Decode that allocates nothing and takes no workspace. No counterpart in the reference: it
 * exists for callers that cannot allocate device memory where they decode (an engine that
 * only hands out memory from its own fixed pool, a plug-in called inside another runtime's
 * step, a C caller without an allocator). Same arguments and result as fpx_decode_attention
 * minus the workspace; the split-K partials live in a fixed array of
 * FPX_DECODE_NOALLOC_SCRATCH_BYTES compiled into the library, held on every GPU that loads
 * it until the process exits. Problems whose partials
 * (fpx_decode_workspace_bytes(B, Lq, H, Hkv, S, d)) exceed that size return
 * FPX_ERR_WORKSPACE before anything runs. The first call on a device looks the array's
 * address up (cudaGetSymbolAddress), so make it before any stream capture; the address is
 * kept for the life of the process, so do not use the library across a cudaDeviceReset. All
 * calls share the array: calls that overlap on the GPU race; nothing in it needs to start at
 * zero. */
#define FPX_DECODE_NOALLOC_SCRATCH_BYTES (2u << 20)
int fpx_decode_attention_noalloc(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                 const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                 const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                                 int B, int Lq, int S, int H, int Hkv, int d, double scale,
                                 void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh, float *lse,
                                 fpx_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FPX_H_ */
