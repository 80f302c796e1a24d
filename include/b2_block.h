/*
 * C ABI of the LFM2.5 layer kernels around the attention hot path
 * (libb2attn.so), used by the whole-token decode runner: the residual add
 * fused with the RMSNorm that follows it, the SwiGLU gate of the feed-forward
 * block, and one decode step of the gated short convolution.  The GEMMs of
 * the layer stay library GEMMs (cuBLAS through the caller).
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
