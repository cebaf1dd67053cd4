/*
 * sdl_b200.h -- C ABI of the B200 paged-KV speculative-decoding kernels.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches stream-ordered work and returns an sdl_status.
 * The library never allocates device memory: the caller owns the KV pools,
 * the metadata arrays, the split-K workspace and every output buffer.
 *
 * Errors found by a kernel (exhausted free list, block-table overflow, an
 * out-of-range block id or slot, a pipeline wait that ran out) are OR-ed
 * into a caller-owned device int32 "error word" (SDL_DEVERR_* bits).  The
 * host reads that word at its per-round sync and raises.
 *
 * The host-side drop-in (Python package engine/, specdec/) binds these
 * symbols with ctypes (engine/_lib.py).
 *
 * Reference interfaces each entry point replaces are cited as
 * <file>:<line> inside sup-zzj/speculative-decoding-lab.
 */
#ifndef SDL_B200_H
#define SDL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
typedef enum sdl_status {
    SDL_OK = 0,
    SDL_ERR_INVALID = 1,      /* bad pointer, shape or stride            */
    SDL_ERR_UNSUPPORTED = 2,  /* dtype / head_dim / block_size not built */
    SDL_ERR_CUDA = 3,         /* a CUDA runtime call failed              */
    SDL_ERR_WORKSPACE = 4     /* workspace too small for the split plan  */
} sdl_status;

/* Bits OR-ed into the device error word. */
#define SDL_DEVERR_EXHAUSTED      1   /* free list empty (BlockExhaustedError) */
#define SDL_DEVERR_TABLE_OVERFLOW 2   /* sequence needs more than `width` blocks */
#define SDL_DEVERR_BAD_INDEX      4   /* row / block id outside the pool       */
#define SDL_DEVERR_TIMEOUT        8   /* a bounded pipeline wait gave up       */
#define SDL_DEVERR_BAD_SLOT       16  /* slot outside capacity*block_size      */
#define SDL_DEVERR_BAD_SAMPLE     32  /* all-zero sampling weights             */
#define SDL_DEVERR_UNIFORMS       64  /* uniform stream read past its end      */

typedef enum sdl_dtype { SDL_F32 = 0, SDL_BF16 = 1, SDL_F16 = 2 } sdl_dtype;

/* Device-resident paged-KV metadata (all arrays caller-owned, int32).
 * Rows of block_table are indexed by sequence id (the reference keys
 * block_tables / seq_lengths by seq_id, engine/kv.py:103-105).          */
typedef struct sdl_kv_meta {
    int32_t* block_table;   /* [max_rows, width] physical block ids        */
    int32_t* num_blocks;    /* [max_rows] length of each row's table       */
    int32_t* seq_lens;      /* [max_rows] valid logical positions          */
    int32_t* free_stack;    /* [capacity] LIFO free list (top = end)       */
    int32_t* free_top;      /* [1] number of entries in free_stack         */
    uint8_t* is_free;       /* [capacity] 1 while a block is on the stack  */
    int32_t* err;           /* [1] device error word                       */
    int32_t capacity;       /* physical blocks in the pool                 */
    int32_t width;          /* max blocks per sequence                     */
    int32_t max_rows;       /* rows allocated in block_table               */
    int32_t block_size;     /* tokens per block                            */
} sdl_kv_meta;

/* Flags for sdl_kv_release (per sequence). */
#define SDL_REL_TRUNCATE        1  /* rewind to new_len, free the tail in reverse */
#define SDL_REL_ONLY_IF_LONGER  2  /* ... only when seq_len > new_len             */
#define SDL_REL_CLEAR           4  /* then free the rest forward, len = 0        */

/* ------------------------------------------------------------ library info */
const char* sdl_version(void);
/* Last host-side error message of the calling thread ("" when none). */
const char* sdl_last_error(void);

/* ----------------------------------------------------- allocator / KV meta */

/* Initialise a free list to the reference's virgin state: the stack holds
 * [0, 1, ..., capacity-1] so the first pop returns capacity-1
 * (replaces BlockAllocator.__init__, engine/kv.py:48-56). */
int sdl_block_init(int32_t* free_stack, int32_t* free_top, uint8_t* is_free,
                   int32_t capacity, void* stream);

/* Pop n blocks (replaces BlockAllocator.alloc, engine/kv.py:61-70).  On an
 * empty stack nothing is popped and SDL_DEVERR_EXHAUSTED is set. */
int sdl_block_alloc(int32_t* free_stack, int32_t* free_top, uint8_t* is_free,
                    int32_t capacity, int32_t n, int32_t* out_blocks,
                    int32_t* err, void* stream);

/* Push blocks in order, skipping ids already free (idempotent double free,
 * engine/kv.py:72-76). */
int sdl_block_free(int32_t* free_stack, int32_t* free_top, uint8_t* is_free,
                   int32_t capacity, int32_t n, const int32_t* blocks,
                   int32_t* err, void* stream);

/* Grow each listed sequence so positions [start, start+count) are backed by
 * blocks, popping new blocks sequence-major / block-minor exactly as the
 * reference's per-token write loop does (engine/kv.py:119-123, 125-147;
 * call order engine/model.py:143-145,184-187), extend seq_lens, and write the
 * slot (phys*block_size + offset) of every position to `slots`
 * (sequence-major, Σcount entries).  Aborts without side effects (slots = -1)
 * on exhaustion or table overflow. */
int sdl_kv_reserve(const sdl_kv_meta* meta, int32_t n, const int32_t* rows,
                   const int32_t* starts, const int32_t* counts,
                   int32_t* slots, void* stream);

/* Scatter T token rows of K and V into layer `layer` of the pools
 * (K[layer, phys, off] = k; engine/kv.py:141-144).  Pools are
 * [num_layers, capacity, block_size, row_elems] with row_elems = Hkv*d.
 * Slots < 0 are skipped. */
int sdl_kv_append(void* k_pool, void* v_pool, int32_t dtype, int32_t num_layers,
                  int32_t capacity, int32_t block_size, int32_t row_elems,
                  int32_t layer, int32_t num_tokens, const int32_t* slots,
                  const void* k_src, const void* v_src, int64_t src_row_stride,
                  int32_t* err, void* stream);

/* Per-sequence rewind / drop, processed in list order so free-list pushes
 * keep the reference's order: truncate frees the tail in reverse
 * (engine/kv.py:150-162), clear frees forward (engine/kv.py:164-171). */
int sdl_kv_release(const sdl_kv_meta* meta, int32_t n, const int32_t* rows,
                   const int32_t* new_lens, const int32_t* flags, void* stream);

/* Alias of sdl_kv_release with SDL_REL_TRUNCATE for every row (the name the
 * reference-side binding expects for PagedKVCache.truncate). */
int sdl_kv_truncate(const sdl_kv_meta* meta, int32_t n, const int32_t* rows,
                    const int32_t* new_lens, void* stream);

/* Device-side commit of one speculative round (replaces the per-sequence
 * commit loop engine/spec_scheduler.py:270-322): k = min(n_out, remaining),
 * EOS cut, keep = start + k, rewind the target cache, align the draft cache
 * (truncate when longer, reserve the one catch-up position when shorter),
 * clear finished sequences.  Sequences are processed in list order so both
 * free lists see the reference's push/pop order.
 *   k_out[b]       committed tokens this round
 *   flags_out[b]   bit0 finished, bit1 eos hit
 *   catchup_slot[b] draft slot for the catch-up token, -1 when none (or when
 *                  the sequence finished, whose K/V the reference discards)
 * draft may be NULL (plain scheduler: clears finished rows only). */
int sdl_spec_commit(const sdl_kv_meta* target, const sdl_kv_meta* draft,
                    int32_t n, const int32_t* rows, const int32_t* n_out,
                    const int32_t* tokens, int32_t tok_stride,
                    const int32_t* remaining, int32_t eos,
                    const int32_t* starts, int32_t* k_out, int32_t* flags_out,
                    int32_t* catchup_slot, void* stream);

/* sdl_spec_commit for a batch padded to n rows (a captured round): only
 * the first *n_valid rows (device int32, read when the kernel runs) are
 * committed; the rest are left alone.  No counterpart in the reference. */
int sdl_spec_commit_n(const sdl_kv_meta* target, const sdl_kv_meta* draft,
                      int32_t n, const int32_t* rows, const int32_t* n_out,
                      const int32_t* tokens, int32_t tok_stride,
                      const int32_t* remaining, int32_t eos,
                      const int32_t* starts, int32_t* k_out, int32_t* flags_out,
                      int32_t* catchup_slot, const int32_t* n_valid,
                      void* stream);

/* ------------------------------------------------------------- attention */

/* Encode the TMA descriptor (128-byte CUtensorMap) the tensor-core attention
 * path uses for a pool [num_tokens_total, Hkv, head_dim] of bf16/f16.
 * num_tokens_total = num_layers*capacity*block_size for a paged pool, or
 * B*chunk for a dense K/V tensor.  Requires head_dim in {64,128}. */
int sdl_make_kv_tensor_map(void* out_map128, const void* base, int32_t dtype,
                           int64_t num_tokens_total, int32_t num_kv_heads,
                           int32_t head_dim);

/* Query-side description shared by the attention entry points.
 * Row j (0 <= j < chunk) of batch entry b sits at absolute position
 * starts[b] + j and attends positions [0, starts[b] + j] (inclusive):
 *   decode  (engine/attention.py:96-118):  chunk = 1, starts = len - 1
 *   extend  (engine/attention.py:170-215): starts = start_positions
 *   prefill (engine/attention.py:121-167): starts = 0, valid_rows = lengths
 * Rows j >= valid_rows[b] are not written (caller zero-fills).
 * GQA: q head h reads kv head h / (Hq/Hkv) (engine/attention.py:32-38).   */
typedef struct sdl_attn_args {
    const void* q;            /* [B, chunk, Hq, d] with the strides below  */
    int64_t q_sb, q_sj, q_sh; /* element strides                           */
    void* out;                /* [B, chunk, Hq, d]                         */
    int64_t o_sb, o_sj, o_sh;
    int32_t out_dtype;        /* sdl_dtype of out (may differ from q)      */
    int32_t dtype;            /* sdl_dtype of q and of the K/V pool        */
    /* paged K/V (k_pool != NULL) */
    const void* k_pool;       /* [L, cap, bs, Hkv, d]                      */
    const void* v_pool;
    const void* tmap_k;       /* 128-byte CUtensorMap, or NULL             */
    const void* tmap_v;
    const int32_t* block_table; int32_t width; int32_t capacity;
    int32_t num_layers; int32_t layer; int32_t block_size;
    const int32_t* rows;      /* [B] block-table row (= seq id)            */
    /* dense K/V (k_pool == NULL): [B, kv_len, Hkv, d] contiguous          */
    const void* k_dense; const void* v_dense; int32_t kv_len;
    const int32_t* starts;    /* [B]                                       */
    const int32_t* valid_rows;/* [B] or NULL (= chunk)                     */
    int32_t B, chunk, Hq, Hkv, head_dim;
    int32_t max_limit;        /* host upper bound of starts[b]+chunk       */
    float scale;              /* softmax scale (1/sqrt(d) in the reference)*/
    float* workspace;         /* split-K partials, fp32                    */
    size_t workspace_bytes;
    int32_t pages_per_split;  /* 0 = choose automatically                  */
    int32_t force_generic;    /* 1 = CUDA-core path even when TC applies   */
    int32_t kv_heads_per_cta; /* 0 = automatic; caps kv heads per CTA      */
    int32_t use_umma;         /* 1 = the tcgen05 kernel where it applies
                                 (up to 64 query rows per kv head);
                                 -1 = the mma.sync kernel; 0 = automatic:
                                 tcgen05 for blocks of at least 48 query
                                 rows per kv head over a mean span of at
                                 least 4096 keys (key_count / B, or
                                 max_limit without a key count)           */
    int32_t cluster_merge;    /* mma.sync kernel with split rows: 0 = fp32
                                 partials in the workspace and a separate
                                 merge launch (default); 1 = the splits of
                                 a row run as one thread-block cluster and
                                 merge their partials in distributed shared
                                 memory, no workspace, when the split count
                                 allows (<= 16).  Slower on ragged batches:
                                 a cluster holds its idle splits' slots    */
    int64_t key_count;        /* 0, or the host's count of keys the call
                                 attends, sum over b of starts[b] + chunk:
                                 the mma.sync plan then sizes its split-K
                                 grid to one wave of resident CTAs; or < 0:
                                 ragged rows of unknown lengths (a plan a
                                 CUDA graph captures and replays over other
                                 batches), split into CTAs of
                                 max(n/16, max_limit/256) pages for decode
                                 and max(n/16, max_limit/512) for blocks,
                                 8..64 (n = unsplit CTAs, one per sequence
                                 and kv-head group), with
                                 rows on M for head_dim-128 blocks of
                                 24+ rows, register-direct loads for
                                 head_dim-64 decode of at most 128
                                 sequences (splits of max(n/8,
                                 max_limit/256) pages) and no automatic
                                 tcgen05 kernel.  Only the launch shape
                                 depends on it, never the result (the
                                 grid still covers max_limit)              */
    int32_t mma_layout;       /* mma.sync kernels: 0 = automatic (query rows
                                 on the MMA M dimension for blocks of at
                                 least 48 query rows per kv head, 16 at
                                 head_dim 64, 24 at head_dim 128 when
                                 key_count gives a mean span below 1024
                                 keys; keys on M below that, with
                                 register-direct loads (3) for head_dim-64
                                 decode when key_count gives a mean span
                                 of at most 1280 keys), 1 =
                                 keys on M (query columns on N: the decode
                                 layout), 2 = query rows on M
                                 (FlashAttention-2 register layout), 3 =
                                 keys on M with K/V loaded from the pool
                                 straight into the MMA fragments (blocks
                                 of at most 8 query columns per kv head
                                 over 16-byte aligned K/V; others keep
                                 the automatic choice)                    */
    /* Fused K/V append (paged pools only): when k_new != NULL the rows
     * k_new/v_new [B*chunk][Hkv*head_dim] (row stride new_row_stride
     * elements, the pool's dtype) are stored at positions starts[b] + j
     * (j below the valid rows) before attending -- the write-then-attend of
     * engine/model.py:143-149 in one call.  The positions' blocks must be
     * reserved already.  The mma.sync kernel writes them itself (16-byte
     * aligned rows); other paths launch a small append kernel first. */
    const void* k_new;
    const void* v_new;
    int64_t new_row_stride;
    int32_t* err;
    /* RoPE inside the launch (engine/model.py:50-56 apply_rotary, called on
     * q and k at engine/qwen.py:157-164 before the cache write): when
     * rope_cos != NULL the call attends x' = T(T(x*c) + T(rotate_half(x)*s))
     * of q and stores that of k_new, c / s being row b*chunk + j of rope_cos
     * / rope_sin (q's dtype, rope_stride elements apart, head_dim wide) --
     * the framework chain's roundings, so the result equals rotating q and k
     * first.  q and k_new are only read.  Only plans whose kernel stores the
     * new rows itself take it (sdl_attention_fuses_rope); others refuse it
     * with SDL_ERR_UNSUPPORTED. */
    const void* rope_cos;
    const void* rope_sin;
    int64_t rope_stride;
    /* 1: the caller launches attention over distinct layers back to back on
     * the stream (a decode step of an attention stack), so no kernel still
     * running when this one starts writes this layer's older pool pages.
     * The mma.sync kernels then let the next launch become resident at once
     * and, with the fused append, stream their first pages of older keys
     * before waiting on the preceding kernel, so a layer's ramp overlaps
     * the previous layer's tail and split merge.  0 (default): dependents
     * start after the main loop and every pool read follows the wait. */
    int32_t overlap_layers;
} sdl_attn_args;

/* Bytes of workspace sdl_paged_attention needs for `args` (0 when one
 * split per row suffices or the splits merge on chip). */
size_t sdl_attention_workspace_bytes(const sdl_attn_args* args);

/* Kernel launches sdl_paged_attention makes for `args` with a workspace of
 * sdl_attention_workspace_bytes(args): the attention kernel, the split-K
 * merge when the plan splits, and the positional append when k_new is set on
 * a path that does not write inside the attention kernel.  -1 when `args`
 * is invalid.  No counterpart in the reference. */
int sdl_attention_launches(const sdl_attn_args* args);

/* 1 when sdl_paged_attention applies RoPE (rope_cos / rope_sin) inside the
 * launch for `args` -- the mma.sync kernels with keys or query rows on M
 * (TMA-fed or register-direct), writing the new K/V rows themselves -- else
 * 0; -1 when `args` is invalid.
 * No counterpart in the reference. */
int sdl_attention_fuses_rope(const sdl_attn_args* args);

/* Kernel sdl_paged_attention runs for `args`: 0 = CUDA-core (generic),
 * 1 = mma.sync split-K with keys on M, 2 = tcgen05 persistent, 3 = mma.sync
 * split-K with query rows on M, 4 = mma.sync split-K with keys on M and K/V
 * loaded straight into the MMA fragments; -1 when `args` is invalid.
 * No counterpart in the reference. */
int sdl_attention_kernel(const sdl_attn_args* args);

/* Paged / dense attention for decode, verify (extend) and prefill rows. */
int sdl_paged_attention(const sdl_attn_args* args, void* stream);

/* Allocation-free variant of sdl_paged_attention (no counterpart in the
 * reference).  For callers that cannot allocate device memory when they call
 * in: a runtime whose pool allocator owns all HBM, or an FFI host that only
 * owns its input/output buffers.  args->workspace is ignored; split-K
 * partials go to a static 8 MiB device array (sdl_noalloc_scratch_bytes())
 * that every GPU loading the library keeps until exit.  The automatic split
 * size grows until the partials fit the array; calls whose plan still needs
 * more (an explicit pages_per_split, the tcgen05 kernel) return
 * SDL_ERR_WORKSPACE without launching.  The first
 * call on a device looks up the array's address (cudaGetSymbolAddress), so
 * make that first call before any stream capture.  All calls share the one
 * array: calls that overlap on the GPU (other streams, other threads) race. */
int sdl_paged_attention_noalloc(const sdl_attn_args* args, void* stream);
size_t sdl_noalloc_scratch_bytes(void);

/* Named aliases a reference-side binding would call:
 *   sdl_paged_decode  -> paged_attention_decode  (engine/attention.py:96)
 *   sdl_paged_verify  -> paged_attention_extend  (engine/attention.py:170)
 *   sdl_prefill_chunk -> paged_attention_prefill_chunk (engine/attention.py:121) */
int sdl_paged_decode(const sdl_attn_args* args, void* stream);
int sdl_paged_verify(const sdl_attn_args* args, void* stream);
int sdl_prefill_chunk(const sdl_attn_args* args, void* stream);

/* -------------------------------------------------------------- sampling */

/* logits_to_probs (specdec/sampler.py:19-36) for temperature > 0 without
 * top-k/top-p: p = softmax(logits / max(T, eps)) in fp32, one row per row.
 * With greedy != 0 writes a one-hot row at the first argmax instead. */
int sdl_logits_to_probs(const void* logits, int32_t dtype, int64_t row_stride,
                        int32_t rows, int32_t vocab, float temperature,
                        float eps, int32_t greedy, float* probs,
                        int64_t probs_stride, void* stream);

/* First-index argmax per row (logits.argmax(-1), specdec/sampler.py:29;
 * engine/scheduler.py:227-233). */
int sdl_argmax_rows(const void* logits, int32_t dtype, int64_t row_stride,
                    int32_t rows, int32_t vocab, int32_t* out, void* stream);

/* Draw one index per row with the defined inverse-CDF rule over fp32
 * weights w (replaces sample_token, specdec/sampler.py:59-69):
 *   W_i = floor(w_i * 2^62), S = sum W_i, U = floor(u * 2^64),
 *   token = min{ i : W_0 + ... + W_i > floor(U * S / 2^64) }.
 * Row r uses uniforms[*u_base + u_offset + r] (u_base may be NULL = 0). */
int sdl_sample_rows(const float* weights, int64_t row_stride, int32_t rows,
                    int32_t vocab, const float* uniforms, int64_t num_uniforms,
                    const int64_t* u_base, int64_t u_offset, int32_t* out,
                    int32_t* err, void* stream);

/* Advance a device uniform-stream counter by `delta`. */
int sdl_counter_add(int64_t* counter, int64_t delta, void* stream);

/* Fused rejection sampling for a batch of draft blocks (replaces
 * batch_accept, engine/spec_scheduler.py:46-88, with acceptance_probability
 * specdec/sampler.py:86-92 and residual_distribution :72-83).
 * Uniform stream semantics: sequences in list order; for each, one uniform
 * per accept test until the first rejection, then one uniform for the
 * residual (or bonus) draw -- the order the reference draws them.
 *   p: target probs [B][gamma+1][V] (row strides p_sb, p_sj)
 *   q: draft probs  [B][gamma][V]   (strides q_sb, q_sj)
 * In greedy mode p_arg [B][gamma+1] (argmax of each target row) replaces p
 * and q (draft proposals are then the draft argmax); uniforms are still
 * consumed in the same pattern.
 * The accept phase starts at uniform index *u_base + u_skip (u_skip = the
 * B*gamma uniforms the draft proposals consumed this round).
 * Outputs tokens [B][gamma+1] (accepted proposals then the resampled or bonus
 * token) and n_out[B] = accepted + 1; sets *u_base past the last uniform used.
 * Residual draws use the rule of sdl_sample_rows on clamp(p - q, 0) without
 * normalisation (the rule is scale-free); when that residual's total is
 * <= 1e-12 the draw uses p instead (specdec/sampler.py:80-82). */
int sdl_spec_sample(const float* p, int64_t p_sb, int64_t p_sj,
                    const float* q, int64_t q_sb, int64_t q_sj,
                    const int32_t* p_arg, const int32_t* proposals,
                    int32_t B, int32_t gamma, int32_t vocab, int32_t greedy,
                    const float* uniforms, int64_t num_uniforms, int64_t* u_base,
                    int64_t u_skip, int32_t* tokens, int32_t* n_out,
                    int32_t* scratch_i32, int32_t* err, void* stream);

/* Bytes of int32 scratch sdl_spec_sample needs (2*B entries). */
size_t sdl_spec_sample_scratch_bytes(int32_t B);

/* ------------------------------------------------------ logits-in sampling
 * The temperature softmax p = softmax(logits / max(T, eps)) is defined with
 * a fixed reduction order (chunks of 8192 elements, see
 * csrc/sampler_logits.cu), so every entry point below derives bit-identical
 * p_i from the same logits; sdl_logits_to_probs (temperature mode) writes
 * exactly those values.  Draws use the integer rule of sdl_sample_rows.
 * Workspaces must be 256-byte aligned and at least
 * sdl_sampler_workspace_bytes(rows, vocab) bytes, rows = logit rows read;
 * their first 64 KB are a control block of the one-launch speculative
 * sampler that must be zero before a workspace's first use (the library
 * keeps it consistent afterwards; after a call that set an error bit, zero
 * it again). */
size_t sdl_sampler_workspace_bytes(int32_t rows, int32_t vocab);

/* sample_token (specdec/sampler.py:59-69) applied to logits_to_probs
 * (specdec/sampler.py:19-36) of every row, without writing p: equal to
 * sdl_logits_to_probs followed by sdl_sample_rows.  Row r uses uniform
 * *u_base + u_offset + r. */
int sdl_sample_logits_rows(const void* logits, int32_t dtype, int64_t row_stride,
                           int32_t rows, int32_t vocab, float temperature,
                           float eps, const float* uniforms,
                           int64_t num_uniforms, const int64_t* u_base,
                           int64_t u_offset, int32_t* out, void* workspace,
                           size_t workspace_bytes, int32_t* err, void* stream);

/* batch_accept (engine/spec_scheduler.py:46-88) from target logits
 * [B][gamma+1][V] and draft logits [B][gamma][V] (same dtype) without
 * materialising probability rows: equal to sdl_logits_to_probs on both
 * blocks followed by sdl_spec_sample (sampling mode), including the uniform
 * consumption and *u_base update.  Five launches by default (statistics,
 * merge, accept walk, per-slice draw sums, draw); with
 * sdl_set_spec_sampler_mode(1), one launch (a thread-block cluster per
 * sequence: row statistics, the fp64 accept tests in the reference's
 * uniform order, the (p-q)+ residual or bonus draw) wherever the batch's
 * clusters can all be resident at once and vocab <= 1048576.  Both give
 * the same bits. */
int sdl_spec_sample_logits(const void* p_logits, int64_t p_sb, int64_t p_sj,
                           const void* q_logits, int64_t q_sb, int64_t q_sj,
                           int32_t dtype, float temperature, float eps,
                           const int32_t* proposals, int32_t B, int32_t gamma,
                           int32_t vocab, const float* uniforms,
                           int64_t num_uniforms, int64_t* u_base, int64_t u_skip,
                           int32_t* tokens, int32_t* n_out, void* workspace,
                           size_t workspace_bytes, int32_t* err, void* stream);

/* sdl_spec_sample_logits for a batch padded to B sequences (a captured
 * round): the accept walk consumes uniforms for the first *n_valid
 * sequences only (device int32) and the counter advances by theirs; the
 * padding sequences' outputs are bonus draws to be ignored.  Always the
 * five-launch chain.  No counterpart in the reference. */
int sdl_spec_sample_logits_n(const void* p_logits, int64_t p_sb, int64_t p_sj,
                             const void* q_logits, int64_t q_sb, int64_t q_sj,
                             int32_t dtype, float temperature, float eps,
                             const int32_t* proposals, int32_t B, int32_t gamma,
                             int32_t vocab, const float* uniforms,
                             int64_t num_uniforms, int64_t* u_base, int64_t u_skip,
                             int32_t* tokens, int32_t* n_out, void* workspace,
                             size_t workspace_bytes, int32_t* err,
                             const int32_t* n_valid, void* stream);

/* 0 (default): sdl_spec_sample_logits runs its five-launch chain; 1: its
 * one-launch kernel wherever that applies.  Process-wide.  No counterpart in
 * the reference. */
int sdl_set_spec_sampler_mode(int32_t mode);

/* Copy the device error word to *out (stream-ordered D2H; *out is valid
 * after the stream synchronises) and optionally clear it. */
int sdl_get_error(int32_t* err_word, int32_t* out_host, int32_t clear,
                  void* stream);

/* ---------------------------------------------------------------------
 * Fused elementwise ops of a decoder layer (16-bit models; no counterpart
 * as a function in the reference, which chains framework ops:
 * engine/model.py:41-72 RMSNorm / rotate_half / apply_rotary,
 * engine/qwen.py:43-75 SwiGLU).  Each rounds to the model dtype where the
 * reference's chain rounds.
 * ------------------------------------------------------------------- */

/* out = T((xf / sqrt(mean(xf^2) + eps)) * w) per row, xf = x as fp32.  With
 * delta != NULL the residual add comes first: x_out = T(x + delta) and the
 * norm is taken of x_out.  Strides are in elements, rows of `dim`. */
int sdl_rmsnorm(const void* x, int64_t x_stride, const void* delta, int64_t delta_stride,
                void* x_out, int64_t x_out_stride, const void* weight, void* out,
                int64_t out_stride, int32_t rows, int32_t dim, float eps,
                int32_t dtype, void* stream);

/* In-place rotate-half RoPE of `rows` rows of `heads` x `head_dim`:
 * x' = T(T(x * cos) + T(rotate_half(x) * sin)), one cos / sin row of
 * head_dim per x row (engine/model.py:50-56). */
int sdl_rope(void* x, int64_t x_row_stride, int32_t rows, int32_t heads,
             int32_t head_dim, const void* cos, int64_t cos_row_stride,
             const void* sin, int64_t sin_row_stride, int32_t dtype, void* stream);

/* out = T(T(silu(gate)) * up), silu(g) = g / (1 + exp(-g)) (engine/qwen.py:49-50). */
int sdl_silu_mul(const void* gate, const void* up, void* out, int64_t n,
                 int32_t dtype, void* stream);

/* The same gate on the output of one GEMM over the concatenated gate and up
 * weights: row r of x holds gate[r][0..inter) then up[r][0..inter) (row
 * stride x_row_stride elements); out[r][i] = T(T(silu(gate)) * up)
 * (engine/qwen.py:49-50 with the two projections fused). */
int sdl_swiglu(const void* x, int64_t x_row_stride, void* out, int64_t out_row_stride,
               int32_t rows, int32_t inter, int32_t dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SDL_B200_H */
