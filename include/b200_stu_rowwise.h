/* C ABI of the row-wise STU-layer kernels that sit either side of the attention operator:
 * the weighted layer norm (optionally SiLU-gated) in front of the u/v/q/k projection, and the
 * layer-norm * gate stage (with optional concatenation and row-wise fp8 quantisation) behind it.
 *
 * Reference semantics (CPU, ATen): recir/ops/kjt_split_per_feature.cpp
 *   weightedLayerNorm          :197-244  schema generative_recommenders::triton_weighted_layer_norm_fwd (:724-727)
 *   layerNormMulQuantized      :558-600  schema ..._triton_layer_norm_mul_dropout_quantization_fwd_impl (:744-747)
 *   quantizeFp8Rowwise         :492-501
 * The reference ignores dropout_ratio / training / seed on this path; so does this library.
 *
 * Same conventions as b200_hstu.h: plain pointers and sizes, caller-owned buffers, nothing is
 * allocated or synchronised, launches go to the given stream, results are negative on error
 * (B200_HSTU_E* codes of b200_hstu.h).
 */
#ifndef B200_STU_ROWWISE_H
#define B200_STU_ROWWISE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_ROWWISE_FLAG_SWISH 0x1u        /* layer norm: y = sigmoid(ln(x)) * x            (is_swish) */
#define B200_ROWWISE_FLAG_STATS_IN 0x2u     /* layer norm: use mean_in / rstd_in instead of computing them */
#define B200_ROWWISE_FLAG_SILU_U 0x4u       /* mul: the concatenated copy of u is silu(u)     (silu_u) */
#define B200_ROWWISE_FLAG_CONCAT_U 0x8u     /* mul: output row = [u' | ...]                   (concat_u) */
#define B200_ROWWISE_FLAG_CONCAT_X 0x10u    /* mul: output row = [... | x | ...]              (concat_x) */
#define B200_ROWWISE_FLAG_ACT_SILU 0x20u    /* mul: gate = silu(u)      (mul_u_activation_type == "silu") */
#define B200_ROWWISE_FLAG_ACT_SIGMOID 0x40u /* mul: gate = sigmoid(u)   (mul_u_activation_type == "sigmoid") */

typedef struct B200RowwiseParams {
  uint32_t struct_size; /* sizeof(B200RowwiseParams) */
  uint32_t flags;
  int32_t dtype;        /* B200_HSTU_F32 / _BF16 / _F16: element type of x, u, weight, bias, y */
  float eps;
  int64_t rows, cols;   /* x is [rows, cols]; cols a multiple of 8, at most 2048 */
  int64_t x_row_stride, u_row_stride, y_row_stride, q8_row_stride; /* in elements */
  const void* x;        /* [rows, cols] */
  const void* u;        /* [rows, cols] (mul only) */
  const void* weight;   /* [cols] or NULL (then bias must be NULL too; layer norm only) */
  const void* bias;     /* [cols] or NULL */
  const float* mean_in; /* [rows] with FLAG_STATS_IN */
  const float* rstd_in;
  void* y;              /* layer norm: [rows, cols]; mul: [rows, parts*cols] or NULL (save_y == false) */
  float* mean;          /* [rows] */
  float* rstd;          /* [rows] */
  float* scale;         /* [rows] row scale of the fp8 copy, or NULL (no fp8 copy) */
  void* q8;             /* float8 e4m3 copy of y (1 byte each): [rows, cols] (layer norm) / [rows, parts*cols] (mul), or NULL */
} B200RowwiseParams;

/* y = ln(x) * weight + bias (or plain ln(x)), optionally sigmoid(y) * x; writes mean and rstd, and
 * optionally the row-wise fp8 copy of y (weightedLayerNormQuantized, :504-531). */
int b200_stu_layer_norm_fwd(const B200RowwiseParams* p, void* stream);
/* out row = [u' | x | ln(x) * gate(u)] (the first two parts are optional); optionally also its
 * row-wise fp8 copy: scale = max(|row|, 1e-12) / 448, q8 = clamp(row / scale, +-448) as e4m3. */
int b200_stu_layer_norm_mul_fwd(const B200RowwiseParams* p, void* stream);
/* Number of column blocks of the mul output: 1 + concat_u + concat_x. */
int b200_stu_layer_norm_mul_parts(uint32_t flags);

/* Backward of b200_stu_layer_norm_fwd (statistics computed from x, i.e. without FLAG_STATS_IN).  The
 * reference has no backward operator for weightedLayerNorm (:197-244): it differentiates the ATen
 * composite by autograd; this entry point computes the closed form of that derivative,
 *   dn = dy (is_swish: dy * x * s * (1 - s), s = sigmoid(ln(x) * w + b)),  dweight = sum_rows dn * xh,
 *   dbias = sum_rows dn,  dx = rstd * (dn * w - mean_cols(dn * w) - xh * mean_cols(dn * w * xh)) (+ dy * s),
 * in float32 with one rounding per gradient, and deterministically (no atomics: per-CTA partial column sums
 * go to the caller's workspace and are added in a fixed order).  cols a multiple of 8, at most 1024. */
typedef struct B200LayerNormBwdParams {
  uint32_t struct_size; /* sizeof(B200LayerNormBwdParams) */
  uint32_t flags;       /* B200_ROWWISE_FLAG_SWISH */
  int32_t dtype;        /* element type of dy, x, weight, bias, dx, dweight, dbias */
  int32_t reserved;
  int64_t rows, cols;
  int64_t dy_row_stride, x_row_stride, dx_row_stride; /* in elements */
  const void* dy;       /* [rows, cols] gradient of the layer norm's output */
  const void* x;        /* [rows, cols] the forward input */
  const void* weight;   /* [cols] or NULL (then bias, dweight, dbias are NULL too) */
  const void* bias;
  const float* mean;    /* [rows] as returned by the forward */
  const float* rstd;
  void* dx;             /* [rows, cols] */
  void* dweight;        /* [cols] */
  void* dbias;          /* [cols] */
  float* workspace;     /* b200_stu_layer_norm_bwd_workspace_bytes(rows, cols) bytes, 16-byte aligned (with weight) */
  uint64_t workspace_bytes;
} B200LayerNormBwdParams;

size_t b200_stu_layer_norm_bwd_workspace_bytes(int64_t rows, int64_t cols);
int b200_stu_layer_norm_bwd(const B200LayerNormBwdParams* p, void* stream);

/* Backward of the gate stage (layerNormMulQuantized, recir/ops/kjt_split_per_feature.cpp:558-600), which the
 * reference differentiates by autograd through the composite: gradients of its saved output
 * combined = [ (silu(u) or u) | x | layer_norm(x) * act(u) ] (the first two parts as the CONCAT flags say) with
 * respect to x, u, weight and bias; the fp8 copy and its scale carry no gradient.  With n the layer norm of x,
 * m = act(u) and d_u | d_x | d_mult the parts of dout:
 *   dn = d_mult * m,  du = d_mult * n * act'(u) (+ d_u * (silu'(u) or 1)),  dweight / dbias / dx from dn as in
 *   b200_stu_layer_norm_bwd (+ d_x),
 * in float32 with one rounding per gradient, deterministically.  flags: B200_ROWWISE_FLAG_SILU_U, _CONCAT_U,
 * _CONCAT_X, _ACT_SILU, _ACT_SIGMOID as in the forward.  cols a multiple of 8, at most 1024. */
typedef struct B200LayerNormMulBwdParams {
  uint32_t struct_size; /* sizeof(B200LayerNormMulBwdParams) */
  uint32_t flags;
  int32_t dtype;        /* element type of dout, x, u, weight, bias and of every gradient */
  int32_t reserved;
  int64_t rows, cols;   /* of x and u; dout has parts * cols columns */
  int64_t dout_row_stride, x_row_stride, u_row_stride, dx_row_stride, du_row_stride; /* in elements */
  const void* dout;     /* [rows, parts * cols] gradient of the forward's saved output */
  const void* x;        /* [rows, cols] */
  const void* u;        /* [rows, cols] */
  const void* weight;   /* [cols] */
  const void* bias;     /* [cols] */
  const float* mean;    /* [rows] as returned by the forward */
  const float* rstd;
  void* dx;             /* [rows, cols] */
  void* du;             /* [rows, cols] */
  void* dweight;        /* [cols] */
  void* dbias;          /* [cols] */
  float* workspace;     /* b200_stu_layer_norm_bwd_workspace_bytes(rows, cols) bytes, 16-byte aligned */
  uint64_t workspace_bytes;
} B200LayerNormMulBwdParams;

int b200_stu_layer_norm_mul_bwd(const B200LayerNormMulBwdParams* p, void* stream);

#ifdef __cplusplus
}
#endif
#endif
