/*
 * q3vl.h -- C ABI of the B200 (sm_100a) Qwen3-VL tensor-parallel decoder path.
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer to
 * densely packed row-major data unless a stride argument says otherwise.
 * Every call is asynchronous on the given stream (a cudaStream_t passed as
 * void*; NULL means the legacy default stream), never throws, and returns an
 * int status (Q3_OK on success).  q3_last_error() gives the reason for the
 * last non-zero status on the calling host thread.
 *
 * The reference implements this path in Python (PyTorch eager + NKI); each
 * declaration names the reference function it replaces as file:line within
 * the yahavb/qwen3-vl project.  Weights follow the reference convention of
 * the public Python API ([in, out], x @ W) at the module level; at this ABI
 * level they are stored [out, in] (K-major) so the tensor-core loads read
 * contiguous K.
 */
#ifndef Q3VL_H_
#define Q3VL_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define Q3_API __attribute__((visibility("default")))
#else
#define Q3_API
#endif

typedef void* q3_stream_t; /* cudaStream_t */

enum q3_status {
  Q3_OK = 0,
  Q3_ERR_INVALID = 1,     /* bad shape, pointer alignment or argument     */
  Q3_ERR_UNSUPPORTED = 2, /* valid request this build does not implement  */
  Q3_ERR_CUDA = 3,        /* CUDA runtime/driver error                    */
  Q3_ERR_TIMEOUT = 4,     /* a bounded in-kernel wait gave up             */
  Q3_ERR_COMM = 5,        /* peer setup / exchange failure                */
  Q3_ERR_NO_MEMORY = 6    /* a pool (KV pages) has too few free entries   */
};

enum q3_dtype { Q3_F32 = 0, Q3_BF16 = 1 };

enum q3_epilogue {
  Q3_EPI_NONE = 0,     /* C = A W^T                                          */
  Q3_EPI_RESIDUAL = 1, /* C = bf16(R + bf16(A W^T)); R = aux [M,N]           */
  Q3_EPI_SWIGLU = 2,   /* W rows interleaved gate/up in blocks of 8 (rows
                          16j..16j+7 = gate 8j..8j+7, 16j+8..16j+15 = up);
                          C[M, N/2] = silu(gate) * up                          */
  /* q3_gemm_bias only (nn.Linear with bias; v = bf16(A W^T + b)):           */
  Q3_EPI_BIAS = 3,           /* C = v                                        */
  Q3_EPI_BIAS_GELU_TANH = 4, /* C = bf16(gelu_tanh(v))                       */
  Q3_EPI_BIAS_GELU = 5,      /* C = bf16(gelu_erf(v))                        */
  Q3_EPI_BIAS_RESIDUAL = 6   /* C = bf16(R + v); R = aux [M, N]              */
};

/* ---- library ---------------------------------------------------------- */
Q3_API int q3_version(void);
Q3_API const char* q3_last_error(void);
/* Reads (and with clear!=0 resets) the device error word that kernels set
 * when a bounded wait times out; 0 means no error was recorded. */
Q3_API int q3_device_error(int clear);
/* Kernels this library has launched in this process (every entry point
 * counts the launches it makes, including the split-K merge of decode
 * attention when it runs as a separate kernel); for launch accounting. */
Q3_API uint64_t q3_launch_count(void);

/* ---- a1: RMSNorm -------------------------------------------------------
 * Replaces RMSNorm.forward (model_fused.py:37-40; model.py:44-47) and the
 * inlined norms of AttentionBlock (model_fused.py:97-100) and MLPBlock
 * (model_fused.py:159-162).  y = bf16(bf16(h * rsqrt(mean(h^2)+eps)) * w).
 * If `add` is non-NULL, h = bf16(x + add) (the residual add of
 * model_fused.py:269/275) and h is written to `h_out` when that is non-NULL;
 * otherwise h = x.  x, add, h_out, y: bf16 [rows, hidden]; w: bf16 [hidden]. */
Q3_API int q3_rmsnorm(const void* x, const void* add, void* h_out, const void* w, void* y, int64_t rows,
               int64_t hidden, float eps, q3_stream_t stream);

/* ---- a9: standalone RoPE -----------------------------------------------
 * Replaces qwen3_rope (kernels/rope.py:24-96).  x bf16 [seq, heads, head_dim];
 * cos_sin f32 [seq, head_dim] (cos in [0, D/2), sin in [D/2, D));
 * out = x*cat(cos,cos) + rotate_half(x)*cat(sin,sin), fp32 math, bf16 out. */
Q3_API int q3_rope(const void* x, const float* cos_sin, void* out, int64_t seq, int heads, int head_dim,
            q3_stream_t stream);

/* ---- a4: interleaved M-RoPE angle tables --------------------------------
 * Replaces Qwen3VLTextRotaryEmbedding.forward + apply_interleaved_mrope
 * (transformers 5.5.0 modeling_qwen3_vl.py:352-386).  pos int64 [3, n_tok]
 * (t, h, w rows); inv_freq f32 [head_dim/2]; frequency j takes axis h when
 * j%3==1 and j<3*sec_h, axis w when j%3==2 and j<3*sec_w, else t.
 * cos_out/sin_out f32 [n_tok, head_dim/2]. */
Q3_API int q3_mrope_cos_sin(const int64_t* pos, const float* inv_freq, int64_t n_tok, int head_dim,
                     int sec_h, int sec_w, float* cos_out, float* sin_out, q3_stream_t stream);

/* ---- paged KV cache: page allocator (host only) ---------------------------
 * Replaces the per-request contiguous cache of init_kv_cache
 * (model_fused.py:224-232) with pages shared by every sequence.  The caller
 * owns the device storage, [num_pages, Hkv, page_tokens, D] per layer for K
 * and for V; the allocator hands out page indices.  A slot (a sequence) owns
 * pages in position order: position p lives in page row[p / page_tokens] at
 * offset p % page_tokens.  page_tokens is a multiple of 64.  A reservation
 * grows the slot to the smallest bucket (ascending token capacities, each a
 * multiple of page_tokens) that covers `tokens`, or with no buckets to whole
 * pages; it is all-or-nothing and returns Q3_ERR_NO_MEMORY when the pool is
 * short.  Pages come from a LIFO free list that starts in ascending order,
 * so ranks issuing the same calls hold identical tables.  Thread-safe. */
Q3_API int q3_kv_pages_create(int num_pages, int page_tokens, int max_seqs, int max_pages_per_seq,
                       const int64_t* buckets, int n_buckets, void** pool_out);
Q3_API int q3_kv_pages_destroy(void* pool);
/* Grow `slot` to cover `tokens` positions; capacity_out (may be NULL) gets the
 * slot's capacity in tokens after the call. */
Q3_API int q3_kv_pages_reserve(void* pool, int slot, int64_t tokens, int64_t* capacity_out);
/* Return every page of `slot` to the pool. */
Q3_API int q3_kv_pages_release(void* pool, int slot);
/* Block-table rows of n slots into host int32 [n, width]; entries past a
 * slot's pages are -1. */
Q3_API int q3_kv_pages_table(const void* pool, const int32_t* slots, int n, int width,
                      int32_t* table_out);
/* Free pages of the pool and, if slot_pages is non-NULL, pages held by `slot`. */
Q3_API int q3_kv_pages_stats(const void* pool, int slot, int64_t* free_pages, int64_t* slot_pages);
/* Device side: copy new K/V rows bf16 [B, Hkv, S, 128] (as q3_qkv_norm_rope
 * writes k_out / v_out) into the page pools at positions pos .. pos+S-1 of
 * each sequence, pos = *pos_dev if non-NULL else start_pos; block_table int32
 * [B, table_stride] on the device (q3_kv_pages_table rows).  A position past
 * the table or a page outside [0, num_pages) is skipped and recorded in the
 * device error word (q3_device_error). */
Q3_API int q3_kv_pages_write(const void* k_src, const void* v_src, void* k_pages, void* v_pages, int B,
                      int Hkv, int S, int head_dim, const int32_t* block_table,
                      int64_t table_stride, int page_tokens, int num_pages, int64_t start_pos,
                      const int32_t* pos_dev, q3_stream_t stream);
/* Decode attention over paged K/V (q3_attn_decode semantics, bf16): k_pages,
 * v_pages [num_pages, Hkv, page_tokens, 128]; position t of sequence b is read
 * from page block_table[b * table_stride + t / page_tokens].  page_tokens is a
 * multiple of 64; workspace as q3_attn_decode_workspace_bytes(B, Hq, Hkv, 128,
 * kv_len).  A table entry outside the pool is recorded in the device error
 * word and page 0 read in its place. */
Q3_API int q3_attn_decode_paged(const void* q, const void* k_pages, const void* v_pages, void* out,
                         int B, int Hq, int Hkv, int head_dim, int64_t kv_len,
                         const int32_t* kv_len_dev, const int32_t* block_table,
                         int64_t table_stride, int page_tokens, int num_pages, float scale,
                         void* workspace, size_t workspace_bytes, q3_stream_t stream);

/* ---- vision tower (transformers 5.5.0 Qwen3VLVisionModel, which the
 * reference runs at vision.py:51-53, :74-76) --------------------------------
 * Tokens are patches in merge-block order.  The image table `imgs` is int32
 * [n_img][4] = {t, h, w, first token} in device memory, with the same table in
 * host memory as `imgs_host` (checked before launch: h, w multiples of merge,
 * first tokens the running sums of t*h*w, n_tok tokens in all). */

/* LayerNorm over the last dim: y = bf16((x - mean) * rstd * w + b), fp32
 * statistics (nn.LayerNorm of Qwen3VLVisionBlock :268-269 and the mergers
 * :113).  x, y bf16 [rows, cols]; w, b bf16 [cols]; cols % 8 == 0. */
Q3_API int q3_layernorm(const void* x, const void* w, const void* b, void* y, int64_t rows, int64_t cols,
                 float eps, q3_stream_t stream);
/* Bilinear position embeddings, fast_pos_embed_interpolate :702-763: table
 * bf16 [side*side, hidden]; out bf16 [n_tok, hidden] in merge-block order. */
Q3_API int q3_vision_pos_embed(const void* table, int side, int hidden, const int32_t* imgs,
                        const int32_t* imgs_host, int n_img, int merge, int64_t n_tok, void* out,
                        q3_stream_t stream);
/* 2-D vision RoPE in place on q and k of the packed qkv bf16 [n_tok, 3*heads*72]
 * (rot_pos_emb :662-700, apply_rotary_pos_emb_vision :131-142); inv_freq f32
 * [18] (head_dim/4 frequencies; the first 18 angles use the patch row, the
 * next 18 the column). */
Q3_API int q3_vision_rope(void* qkv, int heads, int head_dim, const float* inv_freq,
                   const int32_t* imgs, const int32_t* imgs_host, int n_img, int merge,
                   int64_t n_tok, q3_stream_t stream);
/* Non-causal attention inside each frame (Qwen3VLVisionAttention.forward
 * :196-262): qkv bf16 [n_tok, 3*heads*72] after the RoPE; out bf16 [n_tok,
 * heads*72].  blocks int32 [n_blocks][3] = {frame first token, frame length,
 * first query row (a multiple of 128)}: one entry per 128-row query block of
 * every frame, device and host copies. */
Q3_API int q3_vision_attention(const void* qkv, void* out, int heads, int head_dim,
                        const int32_t* blocks, const int32_t* blocks_host, int n_blocks,
                        int64_t n_tok, q3_stream_t stream);

/* ---- a4: multimodal 3-axis position ids ----------------------------------
 * Replaces Qwen3VLModel.get_rope_index (transformers 5.5.0
 * modeling_qwen3_vl.py:1031-1122, with get_vision_position_ids :975-1029).
 * types int32 [B, S] (0 text, 1 image, 2 video); mask int32 [B, S] or NULL
 * (nonzero = kept); image_thw int64 [n_image, 3]; video_thw int64 [n_video, 3]
 * (each video is t frames of grid (1, h, w); n_video <= 4096); merge = the
 * vision spatial merge size.  Grids are consumed in batch order.
 * pos_out int64 [3, B, S] (masked tokens 0); delta_out int64 [B] = max
 * position + 1 - kept tokens.  status_out int32 [B]: 0, or per sequence
 * 1 more vision runs than grids, 2 a run length differs from its grid's
 * token count, 3 a type outside {0, 1, 2}, 4 no kept token (the cases the
 * reference rejects); outputs of a sequence with a nonzero status are
 * unspecified.  workspace: q3_rope_index_workspace_bytes(B) bytes of device
 * memory.  Asynchronous on `stream`. */
Q3_API size_t q3_rope_index_workspace_bytes(int B);
Q3_API int q3_rope_index(const int32_t* types, const int32_t* mask, int B, int64_t S,
                  const int64_t* image_thw, int n_image, const int64_t* video_thw, int n_video,
                  int merge, int64_t* pos_out, int64_t* delta_out, int32_t* status_out,
                  void* workspace, size_t workspace_bytes, q3_stream_t stream);

/* ---- a3 epilogue + a5: per-head QK-RMSNorm, RoPE, KV-cache write ---------
 * Replaces AttentionBlock.forward after the QKV matmul (model_fused.py:107-129)
 * and the cache slice assignment (model_fused.py:244-246).
 * qkv bf16 [B*S, (Hq+2*Hkv)*D] laid out [q | k | v] per token.
 * RoPE row for token (b, s): cs + (cs_use_pos*pos + cs_offset + b*cs_stride_b
 * + s) * D/2, where pos = *pos_dev if pos_dev != NULL else start_pos (the
 * cache position); cs dtype = cs_dtype (bf16 tables as RotaryEmbedding builds
 * them, or f32 M-RoPE rows).  cs_offset shifts text positions after an image
 * (the M-RoPE rope delta) without moving the cache position.
 * Outputs (each may be NULL): q_out bf16 [B, Hq, S, D]; k_out, v_out bf16
 * [B, Hkv, S, D]; k_cache, v_cache bf16 [B, Hkv, max_seq, D] written at
 * positions pos..pos+S-1. */
Q3_API int q3_qkv_norm_rope(const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos,
                     const void* sin, int cs_dtype, int cs_use_pos, int64_t cs_offset,
                     int64_t cs_stride_b, void* q_out, void* k_out, void* v_out, void* k_cache, void* v_cache, int B,
                     int S, int Hq, int Hkv, int head_dim, int64_t start_pos,
                     const int32_t* pos_dev, int64_t max_seq, float eps, q3_stream_t stream);

/* The same with the K/V rows written into page pools [num_pages, Hkv,
 * page_tokens, 128] through block_table (int32 [B, table_stride] on the
 * device): row (b, s) at position pos + s lives in page
 * block_table[b * table_stride + (pos + s) / page_tokens].  q_out may be
 * NULL.  A position the table does not map into the pool is recorded in the
 * device error word and that row not written. */
Q3_API int q3_qkv_norm_rope_paged(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                           const void* cos, const void* sin, int cs_dtype, int cs_use_pos,
                           int64_t cs_offset, int64_t cs_stride_b, void* q_out, void* k_pages,
                           void* v_pages, int B, int S, int Hq, int Hkv, int head_dim,
                           int64_t start_pos, const int32_t* pos_dev, const int32_t* block_table,
                           int64_t table_stride, int page_tokens, int num_pages, float eps,
                           q3_stream_t stream);

/* ---- a6/a8: GQA decode attention (one query token) -----------------------
 * Replaces the S=1 case of the eager attention in forward_layer
 * (model_fused.py:248-262) and the unfinished decode_attention_simple
 * (kernels/decode_attention.py:56-134).  q [B, Hq, D]; caches [B, Hkv,
 * max_seq, D]; out [B, Hq, D]; all of dtype `dtype` (Q3_F32 or Q3_BF16).
 * Attends to cache positions [0, kv_len) where kv_len = *kv_len_dev if that
 * is non-NULL, else kv_len; head h reads KV head h / (Hq/Hkv).  Split-K over
 * SMs: workspace must hold q3_attn_decode_workspace_bytes(...) bytes.
 * With kv_len_dev, kv_len is the upper bound the grid is planned for and the
 * splits share the positions actually present.  Ordering: q and cache row
 * kv_len-1 may come from the kernel just before this call on the stream (as
 * q3_qkv_norm_rope writes them); *kv_len_dev and the cache rows below
 * kv_len-1 must be complete before that kernel is launched, because the bf16
 * kernel starts streaming them while its predecessor finishes.
 * Cache rows from kv_len up to the next multiple of 64 are read and given
 * probability 0, as the reference's masked softmax gives the rows past the
 * prompt (model_fused.py:259-262): they must hold finite values, which
 * zero-filled caches (init_kv_cache, :224-232) and rows written earlier do. */
Q3_API size_t q3_attn_decode_workspace_bytes(int B, int Hq, int Hkv, int head_dim, int64_t max_kv_len);
Q3_API int q3_attn_decode(const void* q, const void* k_cache, const void* v_cache, void* out, int B,
                   int Hq, int Hkv, int head_dim, int64_t kv_len, const int32_t* kv_len_dev,
                   int64_t max_seq, float scale, int dtype, void* workspace,
                   size_t workspace_bytes, q3_stream_t stream);

/* Decode attention with the head norms, RoPE and the KV-cache write folded in:
 * replaces q3_qkv_norm_rope (its decode use) followed by q3_attn_decode, for
 * bf16 caches and bf16 RoPE tables.  qkv bf16 [B, (Hq+2*Hkv)*128] is the raw
 * QKV projection of the new tokens ([q | k | v] per token); the new token sits
 * at cache position kv_len-1 (kv_len = *kv_len_dev when that is non-NULL) and
 * uses RoPE row kv_len-1 + cs_offset.  Each (sequence, KV head) normalises and
 * rotates its query heads itself; the split that holds the new position
 * writes the new k (normed, rotated) and v rows to the caches and adds them to
 * its softmax, and the other rows [0, kv_len-1) stream from the caches without
 * waiting for the preceding kernel.  Workspace as for q3_attn_decode. */
Q3_API int q3_attn_decode_qkv(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                              const void* cos, const void* sin, int64_t cs_offset, void* k_cache,
                              void* v_cache, void* out, int B, int Hq, int Hkv, int head_dim,
                              int64_t kv_len, const int32_t* kv_len_dev, int64_t max_seq,
                              float scale, float eps, void* workspace, size_t workspace_bytes,
                              q3_stream_t stream);
/* q3_attn_decode_qkv over a page pool, as q3_attn_decode_paged reads one:
 * k_pages / v_pages bf16 [num_pages, Hkv, page_tokens, 128], block_table int32
 * [B, table_stride] on the device.  The new token's k and v rows go to page
 * block_table[b, (kv_len-1) / page_tokens] (the caller has grown the table to
 * hold it; a table entry outside [0, num_pages) skips the write and sets the
 * device error word to 0x402).  Replaces q3_qkv_norm_rope_paged followed by
 * q3_attn_decode_paged at decode time (model_fused.py:244-262). */
Q3_API int q3_attn_decode_qkv_paged(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                    const void* cos, const void* sin, int64_t cs_offset,
                                    void* k_pages, void* v_pages, void* out, int B, int Hq,
                                    int Hkv, int head_dim, int64_t kv_len,
                                    const int32_t* kv_len_dev, const int32_t* block_table,
                                    int64_t table_stride, int page_tokens, int num_pages,
                                    float scale, float eps, void* workspace,
                                    size_t workspace_bytes, q3_stream_t stream);

/* Same computation as q3_attn_decode, for callers that cannot allocate device
 * memory at call time (a runtime whose free HBM is already committed to its
 * own pools, or a binding that owns only these buffers).  No counterpart in
 * the reference.  Needs no workspace: split-K partials go to a 4 MiB array
 * built into the library (held by every GPU that loads it until exit);
 * requests needing more are rejected with Q3_ERR_INVALID.  All calls on a
 * device share that array, so calls that overlap on the GPU race; order them
 * on one stream.  The first call on a device looks up the array's address:
 * make it before any stream capture.  That address is kept for the life of
 * the process, so after a device reset (cudaDeviceReset) the library must be
 * reloaded before this entry point is called again.  The split plan launches
 * at most about two CTAs per SM, so on a 148-SM B200 the partials of any
 * supported head ratio (1, 2, 4, 8) need at most about 2.5 MB: the 4 MiB limit
 * binds only on GPUs with more SMs, or for shapes the kernels do not support.
 * Allocates nothing. */
Q3_API int q3_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                  void* out, int B, int Hq, int Hkv, int head_dim,
                                  int64_t kv_len, const int32_t* kv_len_dev, int64_t max_seq,
                                  float scale, int dtype, q3_stream_t stream);

/* ---- a6/a7: causal GQA prefill attention ---------------------------------
 * Replaces the S>1 eager attention of forward_layer (model_fused.py:248-262)
 * and prefill_gqa_flash_attention (kernels/prefill_attention.py:28-149).
 * bf16 throughout; head_dim 128.  Element (b, h, s, d) of q/k/v/out lives at
 * base + b*stride_b + h*stride_h + s*stride_s + d.  Query row s has absolute
 * position start_pos + s and (when causal) attends to keys 0..start_pos+s;
 * keys 0..start_pos+S-1 must be present in k/v. */
Q3_API int q3_attn_prefill(const void* q, const void* k, const void* v, void* out, int B, int Hq,
                    int Hkv, int S, int head_dim, int64_t start_pos, int causal, float scale,
                    const int64_t* q_strides, const int64_t* kv_strides, const int64_t* o_strides,
                    q3_stream_t stream);
/* The same on the tcgen05 tensor cores (S accumulates in TMEM, softmax in fp32).
 * q contiguous [B, Hq, S, 128]; k/v [B, Hkv, kv_rows_per_head, 128] (a cache
 * with kv_rows_per_head >= start_pos + S rows per head); out strides o_strides
 * (b, h, s) in elements, multiples of 8.  variant 0: V is transposed in shared
 * memory so every MMA operand is K-major, and each tile's P V is folded into
 * fp32 registers; variant 1: V feeds the MMA as an MN-major operand and O
 * accumulates in TMEM, rescaled only when a row's maximum grows by more than
 * 2^8; variant 2: one CTA holds the same 128 query rows of two heads of one KV
 * head (Hq / Hkv even), 128-key tiles, P kept in TMEM and read by the MMA from
 * there, the two tiles' softmax and MMAs overlapped; any other variant is
 * rejected.  Cache rows past start_pos + S up to the next
 * multiple of 64 are read with probability 0 and must hold finite values
 * (variant 0 zeroes them). */
Q3_API int q3_attn_prefill_tc(const void* q, const void* k, const void* v, void* out, int B, int Hq,
                       int Hkv, int S, int head_dim, int64_t start_pos, int causal, float scale,
                       int64_t kv_rows_per_head, const int64_t* o_strides, int variant,
                       q3_stream_t stream);
/* q3_attn_prefill_tc variant 2 over paged K/V: k_pages, v_pages [num_pages,
 * Hkv, page_tokens, 128] (page_tokens a multiple of 128); key position t of
 * sequence b is read from page block_table[b * table_stride + t / page_tokens]
 * (entries outside [0, num_pages) are recorded in the device error word and
 * page 0 is read).  q contiguous [B, Hq, S, 128], Hq / Hkv even; out strides as
 * for q3_attn_prefill_tc.  Key rows past start_pos + S in the last page are
 * read with probability 0 and must hold finite values. */
Q3_API int q3_attn_prefill_tc_paged(const void* q, const void* k_pages, const void* v_pages,
                                    void* out, int B, int Hq, int Hkv, int S, int head_dim,
                                    int64_t start_pos, int causal, float scale,
                                    const int64_t* o_strides, const int32_t* block_table,
                                    int64_t table_stride, int page_tokens, int num_pages,
                                    q3_stream_t stream);
/* The same over paged K/V: k_pages, v_pages [num_pages, Hkv, page_tokens, 128];
 * key position t of sequence b is read from page block_table[b * table_stride
 * + t / page_tokens] (page_tokens a multiple of 64).  Keys 0..start_pos+S-1
 * must already be in the pages.  A table entry outside the pool is recorded
 * in the device error word and page 0 read in its place. */
Q3_API int q3_attn_prefill_paged(const void* q, const void* k_pages, const void* v_pages, void* out,
                          int B, int Hq, int Hkv, int S, int head_dim, int64_t start_pos,
                          int causal, float scale, const int64_t* q_strides,
                          const int64_t* o_strides, const int32_t* block_table,
                          int64_t table_stride, int page_tokens, int num_pages,
                          q3_stream_t stream);

/* ---- a3/a10/a11: bf16 GEMM with fused epilogues ---------------------------
 * Replaces the projections h @ Wqkv (model_fused.py:103), x @ Wo (:141),
 * h @ Wgate_up + SiLU*up (:165-169), h @ Wdown (:172) and lm_head (:183).
 * A bf16 [M, K]; W bf16 [N, K] (K-major); C bf16 [M, N] (or [M, N/2] for
 * Q3_EPI_SWIGLU); aux = residual R [M, N] for Q3_EPI_RESIDUAL.  M <= 16 runs
 * the HBM-streaming decode kernel, larger M the tcgen05/TMEM kernel. */
Q3_API int q3_gemm(const void* A, const void* W, void* C, int64_t M, int64_t N, int64_t K, int epilogue,
            const void* aux, q3_stream_t stream);

/* MLPBlock's gate/up projection with SwiGLU (model_fused.py:160-169):
 * C[M, inter] = silu(h Wgate) * (h Wup) with h = rmsnorm(A; norm_w, eps)
 * (model_fused.py:37-40) when norm_w != NULL, else h = A.  A bf16 [M, K];
 * W_gate_up bf16 [2*inter, K] K-major with gate and up rows interleaved in
 * blocks of 8 (Q3_EPI_SWIGLU); inter % 8 == 0.  The fused norm is for decode
 * shapes (M <= 16); larger M takes the normalised rows (q3_rmsnorm) and runs
 * the tcgen05 kernel.  The down projection follows through q3_gemm or
 * q3_gemm_ar. */
Q3_API int q3_gate_up_swiglu(const void* A, const void* W_gate_up, void* C, int64_t M,
                             int64_t inter, int64_t K, const void* norm_w, float eps,
                             q3_stream_t stream);

/* ---- vision tower linears: nn.Linear with bias (tcgen05 GEMM) -------------
 * Replaces the vision tower's linears (transformers 5.5.0 modeling_qwen3_vl.py:
 * attn.qkv / attn.proj :189-190, mlp.linear_fc1/fc2 :64-65, merger fc1/fc2
 * :114-116, the patch-embed Conv3d :72-89 as a GEMM) with the epilogues that
 * follow them: Q3_EPI_BIAS, Q3_EPI_BIAS_GELU_TANH (MLP), Q3_EPI_BIAS_GELU
 * (mergers), Q3_EPI_BIAS_RESIDUAL (block residual adds :288-295, and the
 * position-embedding add after the patch embed :783).  A bf16 [M, K]; W bf16
 * [N, K] (nn.Linear's own layout); bias bf16 [N]; C bf16 [M, N]; aux = R
 * [M, N].  K % 8 == 0 and N % 8 == 0; K and N need not fill the tiles. */
Q3_API int q3_gemm_bias(const void* A, const void* W, const void* bias, void* C, int64_t M, int64_t N,
                 int64_t K, int epilogue, const void* aux, q3_stream_t stream);

/* Prefill QKV projection with its epilogue fused (tcgen05 GEMM): h @ Wqkv
 * (model_fused.py:103) followed by the per-head QK-RMSNorm, rotate-half RoPE
 * and KV-cache write of AttentionBlock.forward (:107-129) and forward_layer
 * (:244-246), without materialising qkv.  A bf16 [B*S, hidden] (the normed
 * input rows, B*S > 16); W bf16 [(Hq+2*Hkv)*128, hidden] K-major, rows
 * [q | k | v]; RoPE rows, tables and outputs as for q3_qkv_norm_rope (token
 * (b, s) sits at cache position start_pos + s; the tables must hold every
 * row the tokens use).  q_out bf16 [B, Hq, S, 128]; k_cache/v_cache bf16
 * [B, Hkv, max_seq, 128] written at start_pos .. start_pos + S - 1. */
Q3_API int q3_gemm_qkv_rope(const void* A, const void* W, int64_t hidden, const void* q_norm_w,
                            const void* k_norm_w, const void* cos, const void* sin, int cs_dtype,
                            int cs_use_pos, int64_t cs_offset, int64_t cs_stride_b, void* q_out,
                            void* k_cache, void* v_cache, int B, int S, int Hq, int Hkv,
                            int head_dim, int64_t start_pos, int64_t max_seq, float eps,
                            q3_stream_t stream);
/* The same with k/v written into page pools [num_pages, Hkv, page_tokens, 128]
 * through block_table (int32 [B, table_stride] on the device; position t of
 * sequence b in page block_table[b * table_stride + t / page_tokens]).  A
 * table entry outside the pool is recorded in the device error word and that
 * row not written. */
Q3_API int q3_gemm_qkv_rope_paged(const void* A, const void* W, int64_t hidden,
                                  const void* q_norm_w, const void* k_norm_w, const void* cos,
                                  const void* sin, int cs_dtype, int cs_use_pos,
                                  int64_t cs_offset, int64_t cs_stride_b, void* q_out,
                                  void* k_pages, void* v_pages, int B, int S, int Hq, int Hkv,
                                  int head_dim, int64_t start_pos, const int32_t* block_table,
                                  int64_t table_stride, int page_tokens, int num_pages,
                                  float eps, q3_stream_t stream);

/* Decode projection with the preceding RMSNorm fused in: C = epilogue(
 * rmsnorm(A; norm_w, eps) W^T) for 1 <= M <= 16, where rmsnorm is
 * model_fused.py:37-40 over the full row of A (the input norm of
 * AttentionBlock, :97-100, before h @ Wqkv; the post-attention norm of
 * MLPBlock, :159-162, before h @ Wgate_up).  Saves the separate norm kernel
 * and its activation round trip on every decode layer. */
Q3_API int q3_gemm_norm(const void* A, const void* norm_w, float eps, const void* W, void* C,
                        int64_t M, int64_t N, int64_t K, int epilogue, const void* aux,
                        q3_stream_t stream);

/* General decode projection (1 <= M <= 16) with the fusions of one decoder
 * layer: C = epilogue(norm(A) W^T) where norm is the RMSNorm above when
 * norm_w != NULL (else identity).  The norm's per-token sum of squares is
 * either recomputed from A or, when ss_in != NULL, summed (in a fixed order)
 * from ss_tiles partials ss_in[ss_tiles][16].  With the residual epilogue,
 * ss_out != NULL receives those partials for the stored outputs,
 * ss_out[ceil(N/64)][16], so the next projection can normalise C without
 * re-reading it.  (The o_proj residual output feeds the post-attention norm
 * of gate/up; the down residual output feeds the next layer's input norm.) */
Q3_API int q3_gemm_decode(const void* A, const void* W, void* C, int64_t M, int64_t N, int64_t K,
                          int epilogue, const void* aux, const void* norm_w, float eps,
                          const float* ss_in, int ss_tiles, float* ss_out, q3_stream_t stream);

/* ---- a10/a11 + 8(e): row-parallel projection fused with the TP all-reduce --
 * Replaces `x @ W` followed by dist.all_reduce(SUM) and the residual add of
 * forward_layer (model_fused.py:265-269 for o_proj, :272-275 for down_proj).
 * A communicator holds one device buffer per rank, opened by every peer
 * through CUDA IPC:
 *   q3_comm_create   allocates this rank's buffer (sized for outputs of up to
 *                    max_cols columns) and writes its IPC handle
 *                    (q3_comm_handle_bytes() bytes) to ipc_handle_out;
 *   q3_comm_open_peers takes the world's handles concatenated in rank order
 *                    (an all-gather done by the caller) and maps the peers;
 *   q3_comm_destroy  unmaps and frees (after a device synchronize).
 * q3_gemm_ar: C = residual + sum over ranks of (A W^T), for decode shapes
 * (1 <= M <= 16, N % 64 == 0); every rank must make the same sequence of calls
 * (like the reference's collectives).  Each output tile's partial is pushed
 * to the peers from inside the kernel over NVLink, in 8-byte words that carry
 * the call number as their arrival flag, and reduced in rank order, so all
 * ranks hold identical results.  residual may be NULL.  ss_out, when not NULL,
 * receives per-64-column-tile sums of squares of C, ss_out[N/64][16], for the
 * RMSNorm fused into the next projection (q3_gemm_decode's ss_in). */
Q3_API int q3_comm_handle_bytes(void);
Q3_API int q3_comm_create(int rank, int world, int64_t max_cols, void** comm_out,
                          void* ipc_handle_out);
Q3_API int q3_comm_open_peers(void* comm, const void* all_handles);
Q3_API int q3_comm_destroy(void* comm);
/* q3_init_comm(rank, world, peer IPC handles): the set-up step in one call
 * for a communicator made by q3_comm_create: checks that comm was created for
 * this rank and world size, then maps every peer's buffer as
 * q3_comm_open_peers does (all_handles: every rank's handle in rank order). */
Q3_API int q3_init_comm(void* comm, int rank, int world, const void* all_handles);
/* Peers reached without IPC (no counterpart in the reference, whose
 * collectives go through torch.distributed): q3_comm_buffer returns this
 * rank's exchange buffer and its size; q3_comm_attach_peer gives the
 * communicator a device pointer to peer_rank's buffer that the caller mapped
 * itself (one process driving several GPUs with peer access enabled, or
 * memory shared by other means).  Once every peer has a buffer the
 * communicator is open.  Attached buffers are not unmapped by
 * q3_comm_destroy.
 * q3_comm_set_wait_limit bounds every in-kernel wait on a peer's words
 * (default 2 s, accepted range 1 ms .. 60 s); when it runs out the kernel
 * records 0x501 in the device error word, stops waiting and completes, so a
 * peer that never arrives surfaces on the host as Q3_ERR_TIMEOUT instead of
 * a hang.  The partial results of such a call are undefined, and the
 * communicator's call numbers are then out of step with its peers: destroy
 * it and create a new one. */
Q3_API int q3_comm_buffer(const void* comm, void** buffer_out, size_t* bytes_out);
Q3_API int q3_comm_attach_peer(void* comm, int peer_rank, void* peer_buffer);
Q3_API int q3_comm_set_wait_limit(void* comm, uint64_t wait_ns);
Q3_API int q3_gemm_ar(const void* A, const void* W, void* C, int64_t M, int64_t N, int64_t K,
                      const void* residual, float* ss_out, void* comm, q3_stream_t stream);

/* ---- a10/a11 + 8(e), prefill shapes: projection + two-shot all-reduce -----
 * Replaces `x @ W`, dist.all_reduce(SUM) and the residual add of forward_layer
 * (model_fused.py:265-269, :272-275) for calls of many tokens.  The output
 * rows are split into one stripe of 128-row tiles per rank; the tcgen05 GEMM's
 * epilogue writes each bf16 partial tile into the owning rank's receive
 * stripe over NVLink (reduce-scatter, overlapped with the MMAs of later
 * tiles); each rank then sums its stripe in rank order (fp32, rounded to
 * bf16), adds the residual, and pulls the other stripes from their owners
 * (all-gather).  C = residual + sum over ranks of (A W^T), identical bits on
 * every rank.  Every rank must make the same calls in the same order.
 *   q3_prefill_comm_create  allocates this rank's exchange buffer, sized for
 *                           calls of up to max_rows x max_cols outputs
 *                           (max_cols a multiple of 32), and writes its IPC
 *                           handle (q3_comm_handle_bytes() bytes);
 *   q3_prefill_comm_open    maps every peer's buffer (the world's handles
 *                           concatenated in rank order);
 *   q3_gemm_allreduce       A bf16 [M, K], W bf16 [N, K] K-major (this rank's
 *                           row shard), C / residual bf16 [M, N]; 16 < M <=
 *                           max_rows, N % 32 == 0, K % 32 == 0; residual may
 *                           be NULL.  A peer that never delivers ends the wait
 *                           after a bounded time with Q3_ERR_TIMEOUT codes
 *                           0x701 / 0x702 in the device error word. */
Q3_API int q3_prefill_comm_create(int rank, int world, int64_t max_rows, int64_t max_cols,
                                  void** comm_out, void* ipc_handle_out);
Q3_API int q3_prefill_comm_open(void* comm, const void* all_handles);
Q3_API int q3_prefill_comm_destroy(void* comm);
/* As q3_comm_buffer / q3_comm_attach_peer / q3_comm_set_wait_limit, for the
 * prefill exchange (its waits record 0x701 / 0x702 when they run out). */
Q3_API int q3_prefill_comm_buffer(const void* comm, void** buffer_out, size_t* bytes_out);
Q3_API int q3_prefill_comm_attach_peer(void* comm, int peer_rank, void* peer_buffer);
Q3_API int q3_prefill_comm_set_wait_limit(void* comm, uint64_t wait_ns);
Q3_API int q3_gemm_allreduce(const void* A, const void* W, void* C, int64_t M, int64_t N,
                             int64_t K, const void* residual, void* comm, q3_stream_t stream);

/* ---- a12/a13: the whole decode step of every layer in one launch ----------
 * Replaces forward_layer (model_fused.py:234-277) at S = 1 for all layers of
 * decode_step (model_fused.py:295-300): input RMSNorm, QKV projection,
 * per-head QK-RMSNorm + RoPE, KV-cache write at the new position, GQA
 * attention, o_proj + residual, post-attention RMSNorm, gate/up + SwiGLU, down
 * + residual.  One persistent kernel, one CTA per SM: weights and old cache
 * rows stream by TMA without waiting for other CTAs, activations wait on
 * grid-wide phase counters (bounded waits).  Tensor parallelism 1 (the
 * projections are this rank's shards; no all-reduce is done), 4 query heads
 * per KV head, head_dim 128, 1..16 sequences (one new token each).
 * q3_step_layer: per-layer device pointers, weights K-major as for q3_gemm
 * (gate/up interleaved in blocks of 8 rows); caches [batch, kv_heads,
 * max_seq, 128].  rope_cos/rope_sin: bf16 [rope_rows, 64] tables
 * (RotaryEmbedding, model_fused.py:43-58).
 * q3_decode_step: x bf16 [batch, hidden] holds the embedded new tokens and
 * receives the last layer's output; ss float [hidden/128][16] receives its
 * per-128-column sums of squares (for the final norm fused into the lm_head,
 * q3_gemm_decode with ss_tiles = hidden/128).  *kv_len_dev = new position + 1,
 * set before the launch; RoPE row = position + rope_delta.  A plan holds
 * workspaces for one step at a time: order its steps on one stream.  After a
 * Q3_ERR_TIMEOUT in the device error word, destroy and recreate the plan. */
typedef struct q3_step_layer {
  const void* w_qkv;      /* [(q_heads + 2*kv_heads)*128, hidden] */
  const void* w_o;        /* [hidden, q_heads*128] */
  const void* w_gate_up;  /* [2*inter, hidden], gate/up interleaved */
  const void* w_down;     /* [hidden, inter] */
  const void* input_norm; /* [hidden] */
  const void* post_norm;  /* [hidden] */
  const void* q_norm;     /* [128] */
  const void* k_norm;     /* [128] */
  void* k_cache;          /* [batch, kv_heads, max_seq, 128] */
  void* v_cache;
} q3_step_layer;
Q3_API int q3_decode_step_create(const q3_step_layer* layers, int n_layers, int batch, int hidden,
                                 int q_heads, int kv_heads, int inter, int64_t max_seq, float eps,
                                 const void* rope_cos, const void* rope_sin, int64_t rope_rows,
                                 void** plan_out);
Q3_API int q3_decode_step(void* plan, void* x, float* ss, const int32_t* kv_len_dev,
                          int64_t rope_delta, q3_stream_t stream);
Q3_API int q3_decode_step_destroy(void* plan);

/* ---- a12/a13 + 8(e): the decode step at tensor parallelism in one launch ---
 * Replaces forward_layer (model_fused.py:234-277) at S = 1 for every layer,
 * with its two dist.all_reduce calls per layer (:267, :274), on one rank of a
 * tensor-parallel group (layers: this rank's shards, as q3_step_layer gives
 * them, except w_gate_up: its rows come in granules of 8, the 4 gate rows of
 * 4 consecutive features then their 4 up rows, so every granule holds whole
 * features (ops.gate_up_granules4 builds it from q3_gemm's 8-row interleave);
 * q_heads, kv_heads and inter per rank).  One persistent kernel per GPU
 * (one CTA per SM, cooperative launch) runs every phase of every layer,
 * separated by grid-wide barriers; weight tiles stream through a TMA ring
 * across phase boundaries; o_proj and down reduce over the ranks inside the
 * kernel through the communicator's peer buffers (8-byte words that carry
 * their call number; ranks summed in rank order, so every rank holds the same
 * bits).  `comm` is a q3_comm_create communicator of this rank's group with
 * max_cols >= hidden, opened, and used by this plan only (its buffer holds
 * this kernel's words).  batch 1..8; every projection's rows must fit 16
 * granules of 8 rows per SM (the 8B shape needs TP >= 2); the reduction
 * lengths (hidden, q_heads * 128, inter) must leave room in shared memory
 * (up to 6144).
 * q3_decode_tp: x bf16 [batch, hidden]: the embedded new tokens in, the last
 * layer's output (before the final norm) out.  *kv_len_dev = new position +
 * 1 (the same for every sequence); RoPE row = position + rope_delta.  Every
 * rank of the group must run the same steps in the same order.  A plan holds
 * workspaces for one step at a time: order its steps on one stream.  After a
 * Q3_ERR_TIMEOUT in the device error word (0x501: a peer never delivered;
 * 0x801-0x808: a barrier, ring, attention-pair or staging wait ran out;
 * 0x80a: *kv_len_dev outside 1..max_seq, nothing ran), destroy and recreate the
 * plan and the communicator. */
Q3_API int q3_decode_tp_create(const q3_step_layer* layers, int n_layers, int batch, int hidden,
                               int q_heads, int kv_heads, int inter, int64_t max_seq, float eps,
                               const void* rope_cos, const void* rope_sin, int64_t rope_rows,
                               void* comm, void** plan_out);
/* q3_decode_tp_create_paged: the same step over a paged KV cache (the
 * bucketed cache of model_fused.py:224-232, :244-246 kept in pages): every
 * layer's k_cache / v_cache is a page pool [num_pages, kv_heads, page_tokens,
 * 128] with page_tokens a multiple of 64, and sequence b's position t lives in
 * page block_table[b * table_stride + t / page_tokens] (device int32 [batch,
 * table_stride], read at every launch, so its entries may change between
 * steps; table_stride * page_tokens >= max_seq).  A table entry outside the
 * pool records 0x809 and abandons the step. */
Q3_API int q3_decode_tp_create_paged(const q3_step_layer* layers, int n_layers, int batch,
                                     int hidden, int q_heads, int kv_heads, int inter,
                                     int64_t max_seq, float eps, const void* rope_cos,
                                     const void* rope_sin, int64_t rope_rows, void* comm,
                                     const int32_t* block_table, int table_stride,
                                     int page_tokens, int64_t num_pages, void** plan_out);
Q3_API int q3_decode_tp(void* plan, void* x, const int32_t* kv_len_dev, int64_t rope_delta,
                        q3_stream_t stream);
Q3_API int q3_decode_tp_destroy(void* plan);

/* ---- a13: embedding gather and greedy argmax -----------------------------
 * Replaces embed_tokens(input_ids) (model_fused.py:281) and
 * logits.argmax(-1) (model_fused.py:310,320).  ids int64 [n]; table bf16
 * [vocab, hidden]; out bf16 [n, hidden].  Out-of-range ids are an error
 * recorded in the device error word and produce zero rows. */
Q3_API int q3_embed(const int64_t* ids, const void* table, void* out, int64_t n, int64_t hidden,
             int64_t vocab, q3_stream_t stream);
/* out = bf16(a + b) elementwise over n bf16 values (n % 8 == 0): the residual
 * add `residual + mlp_out` of forward_layer (model_fused.py:275). */
Q3_API int q3_add(const void* a, const void* b, void* out, int64_t n, q3_stream_t stream);
/* Row-wise argmax of bf16 logits [rows, V] (first index on ties), int64 out. */
Q3_API int q3_argmax(const void* logits, int64_t rows, int64_t V, int64_t* out_idx, q3_stream_t stream);
/* Distributed greedy argmax at TP > 1: replaces the all_gather of every rank's
 * logits followed by argmax (model_fused.py:289-292,310,320).  Each rank
 * writes, per row of its slice [rows, V] whose first column is vocabulary
 * index col_offset, an int64 key that orders by value and then by lower
 * global index; a MAX all-reduce (any library) of the ranks' keys followed by
 * q3_argmax_key_index gives torch.argmax of the gathered logits, first index
 * on ties.  col_offset + V < 2^32. */
Q3_API int q3_argmax_key(const void* logits, int64_t rows, int64_t V, int64_t col_offset,
                  int64_t* out_key, q3_stream_t stream);
Q3_API int q3_argmax_key_index(const int64_t* keys, int64_t rows, int64_t* out_idx,
                        q3_stream_t stream);
/* Brings [ptr, ptr + bytes) into L2 with bulk prefetches and writes nothing:
 * launched before a kernel that leaves HBM bandwidth idle (decode attention
 * reads only the cache rows of a few sequences), it loads the weights of the
 * projection that follows (o_proj, model_fused.py:141) so that projection
 * reads them from L2.  The kernel lets the next kernel start at once and
 * completes after the kernel before it, so stream order is kept.  ptr 16-byte
 * aligned, bytes a multiple of 16. */
Q3_API int q3_l2_prefetch(const void* ptr, int64_t bytes, q3_stream_t stream);

/* The greedy next token of each row in one call: the final RMSNorm
 * (model_fused.py:286; skipped when norm_w is NULL and hidden is already
 * normalised), the lm_head projection (:289) and the argmax (:310,320).
 * hidden bf16 [rows, K]; norm_w bf16 [K] needs rows <= 16 (decode shapes);
 * W_lm bf16 [V, K] K-major, this rank's vocabulary slice whose first row is
 * vocabulary index col_offset; logits_ws bf16 [rows, V] receives the slice's
 * logits.  keys == 0: out[rows] = argmax index over the slice (col_offset must
 * be 0: the slice is the whole vocabulary); keys != 0: out[rows] = the
 * q3_argmax_key keys, for a MAX all-reduce across ranks and then
 * q3_argmax_key_index. */
Q3_API int q3_lm_head_argmax(const void* hidden, const void* norm_w, float eps, const void* W_lm,
                             int64_t rows, int64_t V, int64_t K, int64_t col_offset,
                             void* logits_ws, int keys, int64_t* out, q3_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* Q3VL_H_ */
