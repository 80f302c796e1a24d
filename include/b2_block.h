/*
 * C ABI of the LFM2.5 layer kernels around the attention hot path
 * (libb2attn.so), used by the whole-token decode runner: the layer's
 * projection GEMMs on the tensor cores (with the SwiGLU gate fused into the
 * stacked w1 / w3 product), the residual add fused with the RMSNorm that
 * follows it, the SwiGLU gate on its own, one decode step of the gated short
 * convolution, and the greedy argmax.
 *
 * Conventions as in b2_decode_attn.h: bf16 values as uint16_t bit patterns,
 * row-major, device pointers owned by the caller, a cudaStream_t as void *,
 * 0 or a negative B2_ERR_* status with a message from b2_last_error().
 * Numerics follow the model definition the reference's CPU path runs
 * (transformers modeling_lfm2.py: Lfm2RMSNorm.forward 59-64, Lfm2MLP.forward
 * 135-152, Lfm2ShortConv.slow_forward 356-387, Lfm2DecoderLayer.forward
 * 413-442; the conv-state roll of cache_utils.py 771-786), rounding to bf16
 * where those tensors are bf16.
 */
#ifndef B2_BLOCK_H
#define B2_BLOCK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* b2_gemm epilogues */
enum {
  B2_GEMM_PLAIN = 0,  /* d = bf16(a . w^T) */
  B2_GEMM_SWIGLU = 1  /* w = [w1; w3] (2n rows): d = bf16(bf16(silu(bf16(a . w1^T))) * bf16(a . w3^T)) */
};

/*
 * d[m, n] = a[m, k] . w[n, k]^T (torch's Linear: y = x W^T) with bf16
 * operands, fp32 accumulation on the tensor cores (tcgen05, TMEM
 * accumulators) and a bf16 result rounded to nearest even; with
 * B2_GEMM_SWIGLU, w holds the w1 rows and then the w3 rows (2n rows) and d
 * receives the SwiGLU gate of the two products at the rounding points of
 * b2_swiglu.  Row-major operands with row strides lda, ldw, ldd (elements):
 * k % 64 == 0, lda and ldw >= k, ldd >= n, all three multiples of 8, the
 * pointers 16-byte aligned.  tile_n (output columns per CTA: a multiple of
 * 16 dividing n, <= 128, <= 64 with SwiGLU) and splits (K split over a
 * cluster of that many CTAs: 1, 2, 4 or 8, dividing k / 64) are chosen by
 * b2_gemm_plan when passed as 0.  Split-K partials are summed in a fixed
 * order, so results are deterministic.  The kernel is launched with
 * programmatic stream serialization: it starts fetching w before the
 * previous kernel in the stream has finished and reads a only after it.
 * A wait that gives up (b2_set_wait_limits) ORs B2_DEV_TIMEOUT into dev_err.
 * Replaces the reference's bf16 GEMV (experiments/lfm25_bf16_gemv_kernel.py:19-60:
 * fp32 accumulation, bf16 output; experiments/kernels/x8/x8_core.cc:166-177)
 * for a batch of rows.
 */
int b2_gemm(const uint16_t *a, int64_t lda, const uint16_t *w, int64_t ldw, uint16_t *d, int64_t ldd,
            int32_t m, int32_t n, int32_t k, int32_t mode, int32_t tile_n, int32_t splits, int32_t *dev_err,
            void *stream);

/*
 * The tiling b2_gemm would use for an m x n x k product: tile_n and splits
 * in/out (0 = choose), ctas (may be NULL) the launch's CTA count.
 */
int b2_gemm_plan(int32_t m, int32_t n, int32_t k, int32_t mode, int32_t *tile_n, int32_t *splits, int32_t *ctas);

/*
 * sum = bf16(x + residual) (skipped when residual is NULL: sum = x), then
 * norm_out = bf16(gamma * bf16(sum * rsqrt(mean(sum^2) + eps))), per row of
 * `width` values (width % 8 == 0, width <= 4096).  sum_out (may alias
 * residual or x) receives sum when not NULL.  For width % 32 == 0 the result
 * is bit-identical to the reference's CPU path (torch's Lfm2RMSNorm): the
 * squares are summed in torch's CPU reduction order and rsqrt is 1 / sqrt
 * with IEEE-rounded sqrt and divide.  Replaces the reference's
 * RMSNorm kernels (experiments/kernels/lfm25_rms_norm.cc:21-40,
 * experiments/kernels/x8/x8_math.h:126-148) and the residual adds between
 * them.
 */
int b2_add_rmsnorm(const uint16_t *x, const uint16_t *residual, const uint16_t *gamma,
                   float eps, uint16_t *sum_out, uint16_t *norm_out, int32_t rows,
                   int32_t width, void *stream);

/*
 * out[r][i] = bf16(bf16(silu(gu[r][i])) * gu[r][ffn + i]) for gu = [w1 x | w3 x]
 * (one GEMM with the two weights stacked), ffn % 8 == 0.  Replaces the x8
 * engine's silu_gate (experiments/kernels/x8/x8_core.cc:37-57).
 */
int b2_swiglu(const uint16_t *gu, uint16_t *out, int32_t rows, int32_t ffn, void *stream);

/*
 * One decode step of the gated short convolution (kernel 3), per row and
 * channel c of `hidden`: from bcx = [B | C | x] (in_proj output, 3 * hidden
 * per row), Bx = bf16(B * x); the state [rows][hidden][3] rolls by one
 * (s0, s1, s2) -> (s1, s2, Bx); conv = bf16(sum_i bf16(state_i * w[c][i]))
 * with the sum in fp32; out = bf16(C * conv).  Replaces the x8 engine's
 * conv_gate (experiments/kernels/x8/x8_core.cc:61-85).
 */
int b2_shortconv_step(const uint16_t *bcx, uint16_t *conv_state, const uint16_t *conv_w,
                      uint16_t *out, int32_t rows, int32_t hidden, void *stream);

/*
 * out[r] = index of the largest of the `cols` bf16 values of row r (the
 * first one on ties; NaN counts as the largest), as torch.argmax returns it,
 * for the greedy token choice after the vocabulary head (the reference's
 * X8Model.step select, experiments/lfm25_x8_model.py:133-148).
 */
int b2_argmax_rows(const uint16_t *logits, int32_t rows, int32_t cols, int64_t *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B2_BLOCK_H */
