/*
 * b2_decode_attn.h - C ABI of the B200 LFM2.5 decode-attention library
 * (libb2attn.so).
 *
 * The library implements one hot path of the LFM2.5-230M decoder: for each
 * sequence of a batch and one attention layer,
 *   1. per-head RMSNorm of the raw q/k projections, rotate-half RoPE, and the
 *      append of the new (k, v) into a paged BF16 KV cache      (b2_append_rope)
 *   2. grouped-query attention of the one new query over every cached token,
 *      split along the token axis into partial softmax states (b2_decode_attn)
 *   3. the log-sum-exp merge of those partial states              (b2_combine)
 *
 * Shapes are fixed by the model: 16 query heads, 8 KV heads, head_dim 64,
 * query head h reads KV head h / 2, KV blocks of 64 tokens.
 *
 * Memory layout (all buffers are owned by the caller; nothing is allocated here):
 *   qkv          bf16 [batch][row_stride]; a row starts with
 *                q[16][64] | k[8][64] | v[8][64]  (the reference's qkv vector,
 *                experiments/kernels/lfm25_attention_append_cache.cc:20-21)
 *   k_pool/v_pool bf16 [num_blocks][8 kv heads][64 tokens][64 dims]: one
 *                (block, head) tile is 8 KiB contiguous
 *   block_tables int32 [batch][max_blocks_per_seq]: logical block -> pool block
 *                (max_blocks_per_seq <= 2^25 - 1, so that every length in
 *                tokens fits an int32; wider tables are refused)
 *   past_lens    int32 [batch]: tokens cached before this step (the slot the
 *                new token is written to, and its RoPE position)
 *   seq_lens     int32 [batch]: tokens attended (cached + the new one)
 *   part_ml      fp32 [batch][num_splits][16][2]: partial (max, sum) per head,
 *                max in log2 units (scores are pre-multiplied by scale*log2 e)
 *   part_o       fp32 [batch][num_splits][16][64]: unnormalised partial output
 *
 * bf16 values are passed as their raw 16-bit patterns (uint16_t).  `stream`
 * is a cudaStream_t.  Every call is stream-ordered and asynchronous.  Return
 * value: B2_OK, or a negative B2_ERR_* code; b2_last_error() gives the
 * message (thread-local).  Faults the host cannot see (a block id outside the
 * pool, a length beyond the block table, a bounded wait that ran out) are
 * OR-ed into the caller's device word `dev_err` as B2_DEV_* bits; the kernel
 * skips the bad access instead of performing it.
 */
#ifndef B2_DECODE_ATTN_H
#define B2_DECODE_ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  B2_OK = 0,
  B2_ERR_ARG = -1,    /* bad pointer, shape, alignment or mode */
  B2_ERR_CUDA = -2,   /* the CUDA runtime refused a launch */
  B2_ERR_NOSYM = -3   /* the driver lacks cuTensorMapEncodeTiled */
};

enum {
  B2_DEV_BAD_BLOCK = 1,     /* block table entry outside [0, num_blocks) */
  B2_DEV_BAD_LENGTH = 2,    /* length/position outside the block table */
  B2_DEV_BAD_POSITION = 4,  /* RoPE position outside the cos/sin table */
  B2_DEV_TIMEOUT = 8        /* an mbarrier wait gave up (no hang) */
};

/* b2_append_rope mode bits */
enum {
  B2_NORM_QK = 1,   /* per-head RMSNorm of q and k, times gamma */
  B2_ROPE_QK = 2,   /* rotate-half RoPE of q and k at position past_lens[b] */
  B2_STORE_KV = 4,  /* write k and v into slot past_lens[b] of the pool */
  /* b2_decode_step only, for tests of the failure path: one consumer warp of
   * the first CTA waits on a barrier that nothing completes, gives up after
   * the wait limit (b2_set_wait_limits), reports B2_DEV_TIMEOUT and leaves;
   * the rest of the CTA then times out and unwinds the same way.  The step's
   * results are invalid; the counters must be zeroed before the next step. */
  B2_TEST_STALL = 0x100
};

/* Library ABI version (major * 100 + minor). */
int b2_version(void);

/* Copy the calling thread's last error message into buf (NUL-terminated,
 * truncated to len).  Returns the message length. */
int b2_last_error(char *buf, int len);

/*
 * Limits of the kernels' bounded waits, for every launch of this process
 * after the call (a per-process setting read at launch):
 *   wait_ns  a wait of one warp on another warp of its CTA (mbarrier phases
 *            of the TMA rings, epilogue barrier, merger queue); default 2 s.
 *            It must exceed the longest legitimate wait, about one work
 *            item's streaming time (microseconds at the benchmark sizes).
 *   poll_ns  the multi-GPU exchange's poll for the other ranks' state words
 *            (b2_exchange_merge, b2_decode_step_exchange); default 5 s.
 * A value <= 0 restores the default; values above 60 s are refused.  A wait
 * of a CTA for its own copies or tensor-core products keeps a fixed 2 s.
 * On expiry the kernel ORs B2_DEV_TIMEOUT into dev_err and returns.
 *
 * The reference's analogue is the watchdog around an NPU run and the raise
 * on a run that did not complete (scripts/run_npu_timeout.ps1:1-19,
 * experiments/npu_direct.py:110-114).
 */
int b2_set_wait_limits(int64_t wait_ns, int64_t poll_ns);

/* The limits in force (nanoseconds); either pointer may be NULL. */
int b2_get_wait_limits(int64_t *wait_ns, int64_t *poll_ns);

/*
 * Fused q/k RMSNorm + RoPE + KV append for one decode token per sequence.
 *
 * Replaces, for the whole batch in one launch:
 *   append_attention_cache(qkv, prior_cache, next_cache)
 *     experiments/lfm25_attention_append_cache_kernel.py:20-73 with its core
 *     kernel lfm25_attention_append_cache{,_dynamic}
 *     (experiments/kernels/lfm25_attention_append_cache.cc:5-39), and
 *   lfm25_attention_norm_rope(qkv, aux)
 *     (experiments/kernels/lfm25_attention_norm_rope.cc:17-54; the x8
 *     engine's norm_rope, experiments/kernels/x8/x8_math.h:150-177).
 * Unlike the reference, the old cache is not copied: only the new token's
 * 128-byte k and v rows are written, in place, into the paged pool.
 *
 * qkv          bf16 rows of row_stride elements (row_stride >= 2048, multiple
 *              of 8), 16-byte aligned.
 * gamma_q/k    bf16 [64] RMSNorm weights (required when B2_NORM_QK).
 * eps          RMSNorm epsilon (LFM2: 1e-5).
 * rope_cos/sin bf16 [rope_rows][64] tables (required when B2_ROPE_QK).
 * q_out        bf16 [batch][16][64] normalised + rotated query, or NULL.
 * k/v_pool     required when B2_STORE_KV.
 */
int b2_append_rope(const uint16_t *qkv, int64_t row_stride,
                   const uint16_t *gamma_q, const uint16_t *gamma_k, float eps,
                   const uint16_t *rope_cos, const uint16_t *rope_sin,
                   int32_t rope_rows,
                   const int32_t *past_lens,
                   const int32_t *block_tables, int32_t max_blocks_per_seq,
                   uint16_t *k_pool, uint16_t *v_pool, int32_t num_blocks,
                   uint16_t *q_out, int32_t batch, int32_t mode,
                   int32_t *dev_err, void *stream);

/*
 * Split-KV flash-decode over the paged pool: one CTA per
 * (split, kv head, sequence); split s covers logical blocks
 * [s * blocks_per_split, (s + 1) * blocks_per_split) of its sequence.  K/V
 * tiles stream HBM -> shared memory through TMA (128-byte swizzle) in a
 * 4-stage mbarrier pipeline; both query heads of the GQA pair share each tile.
 *
 * Replaces the context computation of
 *   attention_context(qkv, past_cache, context)
 *     experiments/lfm25_attention_context_kernel.py:20-72,
 *     experiments/kernels/lfm25_attention_context_head.cc:19-82
 *   attention_context_cache / _fixed64 / _chunked
 *     experiments/lfm25_attention_context_cache_kernel.py:16-106,
 *     experiments/lfm25_attention_fixed64_cache_kernel.py:30-136,
 *     experiments/lfm25_attention_chunked_cache_kernel.py:21-89 and the
 *     online softmax of experiments/kernels/lfm25_attention_chunked_head.cc:49-88
 *   the x8 engine's attn_prep/attn_block/attn_final + attn_positions
 *     experiments/kernels/x8/x8_core.cc:89-121, x8/x8_math.h:185-254
 *
 * q            bf16 [batch][16][64] (output of b2_append_rope).
 * num_splits   >= ceil(max_blocks_per_seq / blocks_per_split).
 * scale        softmax scale (head_dim^-0.5 = 0.125).
 * Pool pointers must be 16-byte aligned; num_blocks * 512 < 2^31.
 */
int b2_decode_attn(const uint16_t *q,
                   const uint16_t *k_pool, const uint16_t *v_pool,
                   int32_t num_blocks,
                   const int32_t *block_tables, int32_t max_blocks_per_seq,
                   const int32_t *seq_lens, int32_t batch,
                   int32_t blocks_per_split, int32_t num_splits, float scale,
                   float *part_ml, float *part_o,
                   int32_t *dev_err, void *stream);

/*
 * Log-sum-exp merge of partial states [batch][num_parts][16] into either the
 * bf16 context out[batch][16][64] (head-major, the reference's context layout,
 * experiments/kernels/lfm25_attention_context_head.cc:75) and/or one merged
 * fp32 state (state_ml [batch][16][2], state_o [batch][16][64]) for a further
 * merge across GPUs.  With seq_lens != NULL only the parts that cover tokens
 * of each sequence are read (ceil(ceil(len/64)/blocks_per_split)); with NULL
 * all num_parts are read.  Replaces the final acc/l step of
 * experiments/kernels/lfm25_attention_chunked_head.cc:84-88 and attn_final
 * (experiments/kernels/x8/x8_core.cc:113-121).
 */
int b2_combine(const float *part_ml, const float *part_o, int32_t num_parts,
               const int32_t *seq_lens, int32_t blocks_per_split,
               int32_t batch, uint16_t *out, float *state_ml, float *state_o,
               void *stream);

/*
 * One fused decode step in a single persistent launch: q/k RMSNorm + RoPE,
 * append of the new k/v into slot past_lens[b] of the pool, split-KV
 * attention over past_lens[b] + 1 tokens and the merge of the splits, for
 * the whole batch.  Same results as b2_append_rope + b2_decode_attn +
 * b2_combine (the same device arithmetic); replaces, together, the
 * reference's per-layer chain norm_rope -> append -> context
 * (experiments/kernels/x8/x8_core.cc:89-121 attn_prep/attn_block/attn_final,
 * experiments/lfm25_attention_context_cache_kernel.py:54-71).
 *
 * A persistent grid (3 CTAs per SM, or max_ctas if smaller and > 0) takes
 * work items (sequence, split, kv head) from a counter; a sequence that fits
 * one split is written to out directly, the others leave partial states in
 * part_ml/part_o and the last split of a (sequence, kv head) to finish
 * merges them (a dedicated warp per CTA counts the arrivals and merges, off
 * the path of the warps that stream the cache; one split per lane of that
 * warp, so all splits' loads are in flight together).  With more than 16
 * splits per sequence the merge is left to the parallel combine kernel,
 * which this call launches after the decode kernel as a programmatic
 * dependent.
 *
 * seq_lens     NULL: attend over past_lens[b] + 1 tokens (the usual decode
 *              step).  Otherwise tokens attended per sequence; with
 *              B2_STORE_KV it must equal past_lens[b] + 1, without it
 *              past_lens[b] is only the RoPE position (a GPU that holds a
 *              slice of a long sequence's tokens, see b2_combine).
 * out          bf16 [batch][16][64] context, or NULL when state_ml/state_o
 *              (fp32 [batch][16][2] / [batch][16][64], as b2_combine) are
 *              given: the merged state of the attended tokens, for a
 *              further merge across GPUs.
 * counters     int32 [b2_decode_step_counters(batch)] (= 2 + 8 * batch); must be zero
 *              before the first call; every call that completes leaves it
 *              zero again (after a device error, zero it again).
 * part_ml/o    as b2_decode_attn with num_splits = ceil(max_blocks / bps);
 *              16-byte aligned (as are state_ml / state_o).
 * blocks_per_split  1 .. 64.
 * q_out        optional bf16 [batch][16][64] normalised + rotated q.
 * Calls sharing `counters` must not overlap on the GPU.
 */
int b2_decode_step_counters(int32_t batch);
int b2_decode_step(const uint16_t *qkv, int64_t row_stride,
                   const uint16_t *gamma_q, const uint16_t *gamma_k, float eps,
                   const uint16_t *rope_cos, const uint16_t *rope_sin,
                   int32_t rope_rows, const int32_t *past_lens,
                   const int32_t *seq_lens,
                   const int32_t *block_tables, int32_t max_blocks_per_seq,
                   uint16_t *k_pool, uint16_t *v_pool, int32_t num_blocks,
                   int32_t batch, int32_t blocks_per_split, float scale,
                   int32_t mode, uint16_t *out, uint16_t *q_out,
                   float *state_ml, float *state_o,
                   float *part_ml, float *part_o, int32_t *counters,
                   int32_t max_ctas, int32_t *dev_err, void *stream);

/*
 * The fused decode step for 1 to 4 new tokens per sequence (a prompt chunk,
 * or the reference's x8p engine's 4-token batches,
 * experiments/kernels/x8/x8p_core.cc:137-226 attn_prep/attn_block4): q/k
 * RMSNorm + RoPE of every new token t at position past_lens[b] + t, the
 * append of its k/v into that slot, and attention of token t over the
 * cached tokens and the new tokens up to itself (causal), in one launch at
 * the decode kernel's streaming rate (its tensor-core tile has 8 query
 * columns: tokens x the GQA pair).  tokens == 1 is b2_decode_step.
 *
 * qkv          row b * tokens + t (stride row_stride) = the raw [q | k | v]
 *              projections of token t of sequence b.
 * chunk_lens   NULL: every sequence has `tokens` new tokens; else int32
 *              [batch], 1 .. tokens of them valid (the rest of the rows
 *              are ignored and their contexts left unwritten).  Unused
 *              with tokens == 1.
 * out, q_out   bf16 [batch][tokens][16][64] (q_out optional).
 * part_ml/o    fp32 [batch][tokens][num_splits][16][2 / 64] with num_splits
 *              = ceil(max_blocks_per_seq / blocks_per_split), which must be
 *              at most 16 for tokens > 1 (the kernel merges the splits).
 * counters, blocks_per_split, mode, max_ctas as b2_decode_step; 2 CTAs per SM
 * for tokens > 1.
 */
int b2_decode_step_tokens(const uint16_t *qkv, int64_t row_stride, int32_t tokens, const int32_t *chunk_lens,
                          const uint16_t *gamma_q, const uint16_t *gamma_k, float eps, const uint16_t *rope_cos,
                          const uint16_t *rope_sin, int32_t rope_rows, const int32_t *past_lens,
                          const int32_t *block_tables, int32_t max_blocks_per_seq, uint16_t *k_pool,
                          uint16_t *v_pool, int32_t num_blocks, int32_t batch, int32_t blocks_per_split,
                          float scale, int32_t mode, uint16_t *out, uint16_t *q_out, float *part_ml,
                          float *part_o, int32_t *counters, int32_t max_ctas, int32_t *dev_err, void *stream);

/*
 * One decode step fed from host memory, in one call and stream order: copy
 * the qkv rows (batch x 2048 bf16, packed) and past lengths from pinned host
 * memory into the caller's device staging buffers, run b2_decode_step
 * (norm + RoPE + append + attention, B2_NORM_QK | B2_ROPE_QK | B2_STORE_KV),
 * copy the context (batch x 16 x 64 bf16) back into out_host.  For hosts that
 * drive the decode loop from the CPU (the reference's X8Model.step submits one
 * program per token, experiments/lfm25_x8_model.py:133-148).  Asynchronous:
 * out_host is valid after the stream is synchronised.
 */
int b2_decode_step_host(const uint16_t *qkv_host, const int32_t *past_host,
                        uint16_t *out_host, uint16_t *qkv_dev, int32_t *past_dev,
                        uint16_t *out_dev, const uint16_t *gamma_q,
                        const uint16_t *gamma_k, float eps,
                        const uint16_t *rope_cos, const uint16_t *rope_sin,
                        int32_t rope_rows, const int32_t *block_tables,
                        int32_t max_blocks_per_seq, uint16_t *k_pool,
                        uint16_t *v_pool, int32_t num_blocks, int32_t batch,
                        int32_t blocks_per_split, float scale, float *part_ml,
                        float *part_o, int32_t *counters, int32_t *dev_err,
                        void *stream);

/*
 * Double-buffered form of b2_decode_step_host for a host loop that keeps the
 * GPU busy: the caller alternates slot 0 and 1 and provides two staging slots
 * (qkv_dev2 [2][batch][2048], past_dev2 [2][batch], out_dev2 [2][batch][16][64]).
 * Uploads run on a library-owned stream, ahead of the kernel of the previous
 * step; the kernel runs on `stream`; downloads on a second library-owned
 * stream, overlapping the next kernel.  The streams and events are created on
 * the first call on a device (no device memory is allocated).
 * b2_decode_step_host_join(stream) makes `stream` wait for every download
 * issued so far (then synchronising `stream` makes all out_host valid).
 */
int b2_decode_step_host2(const uint16_t *qkv_host, const int32_t *past_host,
                         uint16_t *out_host, uint16_t *qkv_dev2, int32_t *past_dev2,
                         uint16_t *out_dev2, int32_t slot,
                         const uint16_t *gamma_q, const uint16_t *gamma_k, float eps,
                         const uint16_t *rope_cos, const uint16_t *rope_sin,
                         int32_t rope_rows, const int32_t *block_tables,
                         int32_t max_blocks_per_seq, uint16_t *k_pool,
                         uint16_t *v_pool, int32_t num_blocks, int32_t batch,
                         int32_t blocks_per_split, float scale, float *part_ml,
                         float *part_o, int32_t *counters, int32_t *dev_err,
                         void *stream);
int b2_decode_step_host_join(void *stream);

/*
 * Merge states gathered from several GPUs (config C4: one sequence split
 * along the token axis).  `states` holds num_parts blocks of
 * batch * 16 * 66 fp32, each laid out [state_ml batch*16*2 | state_o
 * batch*16*64] - what b2_decode_step / b2_combine write when state_o =
 * state_ml + batch * 32, i.e. the buffer one all-gather collects.  Output as
 * b2_combine (bf16 context and/or a merged state).
 */
int b2_merge_states(const float *states, int32_t num_parts, int32_t batch,
                    uint16_t *out, float *state_ml, float *state_o,
                    void *stream);

/*
 * Multi-GPU merge without a collective library (config C4 over NVLink).
 * Replaces the all-gather + b2_merge_states pair that the split-KV long
 * context needs (the reference itself has no multi-device code: its long
 * contexts stream 64-token blocks through one NPU core,
 * experiments/lfm25_attention_chunked_cache_kernel.py:21-89, and merge with
 * the chunked kernel's online-softmax state, kernels/lfm25_attention_chunked_head.cc:73-88).
 *
 * Every rank owns an exchange area of b2_exchange_bytes(world, batch) bytes
 * in its own device memory, zeroed before first use, and maps the other
 * ranks' areas with b2_ipc_handle (export: a 64-byte handle and the offset of
 * `ptr` in its allocation) / b2_ipc_open (import on another process) /
 * b2_ipc_close.  b2_exchange_merge(state_ml [batch][16][2], state_o
 * [batch][16][64], areas[world] = every rank's area as mapped on this GPU,
 * areas[rank] = this rank's own) writes this rank's state into every area
 * (each value with a step tag in one 8-byte store), waits until the other
 * ranks' values of this step are in its own area and merges the world's
 * states into out (bf16 [batch][16][64]).  All ranks must
 * call it the same number of times, each on its own GPU (it waits for the
 * others; two ranks on one GPU are not supported).  A wait gives up after
 * 5 s and sets B2_DEV_TIMEOUT in dev_err, leaving out unwritten; the areas
 * must then be zeroed again on every rank before the next call.
 * Launched as a programmatic dependent of the previous kernel in the stream.
 */
#define B2_XCHG_MAX_WORLD 8
/*
 * b2_decode_step with the exchange fused into its merge: the splits of every
 * (sequence, query head) are merged by the combine kernel, which then runs
 * the exchange of b2_exchange_merge itself (this rank's merged state into
 * every rank's area, the world's states merged) and writes the context into
 * out.  One call, two launches (the step kernel and the combine kernel as its
 * programmatic dependent); the same rules for the areas as b2_exchange_merge.
 */
int b2_decode_step_exchange(const uint16_t *qkv, int64_t row_stride,
                            const uint16_t *gamma_q, const uint16_t *gamma_k, float eps,
                            const uint16_t *rope_cos, const uint16_t *rope_sin,
                            int32_t rope_rows, const int32_t *past_lens,
                            const int32_t *seq_lens, const int32_t *block_tables,
                            int32_t max_blocks_per_seq, uint16_t *k_pool, uint16_t *v_pool,
                            int32_t num_blocks, int32_t batch, int32_t blocks_per_split,
                            float scale, int32_t mode, uint16_t *out, uint16_t *q_out,
                            float *part_ml, float *part_o, int32_t *counters,
                            int32_t max_ctas, void *const *areas, int32_t world,
                            int32_t rank, int32_t *dev_err, void *stream);
int64_t b2_exchange_bytes(int32_t world, int32_t batch);
int b2_ipc_handle(const void *ptr, void *handle64, int64_t *offset);
int b2_ipc_open(const void *handle64, int64_t offset, void **peer_ptr);
int b2_ipc_close(void *peer_ptr, int64_t offset);
int b2_exchange_merge(const float *state_ml, const float *state_o, int32_t batch,
                      void *const *areas, int32_t world, int32_t rank,
                      uint16_t *out, int32_t *dev_err, void *stream);

/*
 * Batched-prompt (prefill) attention: a chunk of `tokens` new tokens per
 * sequence, rows qkv[b * tokens + t] (chunk_lens[b] <= tokens valid, NULL:
 * all), token t at position past_lens[b] + t.
 *
 * b2_prefill_append: q/k RMSNorm + RoPE and the append of every chunk token's
 * k/v (the decode append, one CTA per token); q_out [batch][tokens][16][64].
 * b2_prefill_attn: each chunk token attends to the cached tokens and
 * causally to the chunk (query t sees positions <= past_lens[b] + t), on the
 * tcgen05 tensor cores: one CTA per (64-token query tile, kv head, sequence)
 * computes S = Q.K^T and P.V as 128 x 64 x 64 MMAs with the accumulators in
 * tensor memory.  out [batch][tokens][16][64] bf16.
 *
 * Replaces the reference's batched prompt attention: the x8p engine's
 * attn_prep / attn_block4 (4 tokens x 2 heads per KV head, cached part then
 * causal in-batch part, experiments/kernels/x8/x8p_core.cc:137-226) and the
 * prefill pair operator (experiments/lfm25_prefill_pair_attention_context_kernel.py:21-85).
 */
int b2_prefill_append(const uint16_t *qkv, int64_t row_stride,
                      const uint16_t *gamma_q, const uint16_t *gamma_k, float eps,
                      const uint16_t *rope_cos, const uint16_t *rope_sin,
                      int32_t rope_rows, const int32_t *past_lens,
                      const int32_t *chunk_lens, int32_t tokens,
                      const int32_t *block_tables, int32_t max_blocks_per_seq,
                      uint16_t *k_pool, uint16_t *v_pool, int32_t num_blocks,
                      uint16_t *q_out, int32_t batch, int32_t mode,
                      int32_t *dev_err, void *stream);
int b2_prefill_attn(const uint16_t *q, const uint16_t *k_pool,
                    const uint16_t *v_pool, int32_t num_blocks,
                    const int32_t *block_tables, int32_t max_blocks_per_seq,
                    const int32_t *past_lens, const int32_t *chunk_lens,
                    int32_t tokens, int32_t batch, float scale,
                    uint16_t *out, int32_t *dev_err, void *stream);

/*
 * b2_prefill_attn with the keys of every query tile split in ranges of
 * blocks_per_split 64-token blocks over more CTAs (for short chunks the
 * longest sequence otherwise bounds the launch): each CTA writes the partial
 * softmax state of its rows into part_ml [nsplit][batch][tokens][16][2] and
 * part_o [nsplit][batch][tokens][16][64] (fp32, nsplit = ceil(max_blocks_per_seq
 * / blocks_per_split)), and the combine kernel merges them into out (rows past
 * a sequence's chunk become 0).  batch * nsplit <= 65535.
 */
int b2_prefill_attn_split(const uint16_t *q, const uint16_t *k_pool,
                          const uint16_t *v_pool, int32_t num_blocks,
                          const int32_t *block_tables, int32_t max_blocks_per_seq,
                          const int32_t *past_lens, const int32_t *chunk_lens,
                          int32_t tokens, int32_t batch, float scale,
                          int32_t blocks_per_split, float *part_ml, float *part_o,
                          uint16_t *out, int32_t *dev_err, void *stream);

/*
 * Allocation-free decode: b2_decode_attn followed by b2_combine, with the
 * partial softmax states kept in a static device array inside this library
 * instead of caller-provided part_ml / part_o buffers.  It has no counterpart
 * in the reference.
 *
 * It is meant for callers that hold device pointers but cannot allocate
 * device memory of their own: a host written in another language that binds
 * only this C ABI and has no CUDA allocator, or an embedder whose device
 * memory is already committed to another framework's pool.
 *
 * Limit: batch * ceil(max_blocks_per_seq / blocks_per_split) must not exceed
 * B2_NOALLOC_MAX_PARTS; larger calls return B2_ERR_ARG without launching.
 * The array (B2_NOALLOC_MAX_PARTS x 16 heads x 66 floats = 4.125 MiB) is held
 * on every GPU that loads the library until the process exits.  The first
 * call on a device looks up that device's copy of the array
 * (cudaGetSymbolAddress) with the device current; make that first call before
 * any stream capture.  All calls on a device share the one array and it keeps
 * the previous call's contents (every entry this call reads is written by
 * this call first): calls that can overlap on the GPU, e.g. on two streams
 * without ordering between them, race on it and must be serialised by the
 * caller.  Nothing is allocated or freed, by this library or any other.
 */
#define B2_NOALLOC_MAX_PARTS 1024
int b2_decode_attn_noalloc(const uint16_t *q,
                           const uint16_t *k_pool, const uint16_t *v_pool,
                           int32_t num_blocks,
                           const int32_t *block_tables, int32_t max_blocks_per_seq,
                           const int32_t *seq_lens, int32_t batch,
                           int32_t blocks_per_split, float scale,
                           uint16_t *out, int32_t *dev_err, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B2_DECODE_ATTN_H */
