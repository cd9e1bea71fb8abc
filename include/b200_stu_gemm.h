/* C ABI of the STU-layer projections on the tensor cores: out = bias + A W with A = x or the weighted
 * layer norm of x computed inside the same kernel.
 *
 * Reference semantics (CPU, ATen), recir/ops/kjt_split_per_feature.cpp:
 *   tritonAddMm        :246-262  at::addmm(bias, x, w); schema generative_recommenders::triton_addmm_fwd
 *   weightedLayerNorm  :197-244  (the stage in front of the u/v/q/k projection of an STU layer)
 * The fused form computes addmm(bias, weightedLayerNorm(x, ln_weight, ln_bias, eps, is_swish)[0], w) and also
 * returns the row statistics the layer norm returns.  As in the reference the normalised rows are rounded to
 * the element type before the product; sums run in float32; the result is rounded once, after the bias.
 * The output may be consumed in place as column slices (u | v | q | k with row stride N): the attention entry
 * points of b200_hstu.h take row-strided inputs.
 *
 * Served shapes: bfloat16 / float16, K a multiple of 64 and at most 512 (a CTA keeps its 128 x K operand in
 * shared memory), N a multiple of 8, 16-byte aligned bases and row strides.  b200_stu_addmm_supported tells.
 *
 * Conventions of b200_hstu.h: plain pointers and sizes, caller-owned buffers, nothing allocated or
 * synchronised, launches go to the given stream, negative B200_HSTU_E* codes on error; status (optional,
 * device int32[4], zeroed by the caller) receives in status[1] the code of a pipeline wait that gave up
 * (111 producer, 112 MMA issuer, 113 epilogue; 114: shared memory not 1024-byte aligned, nothing ran).
 */
#ifndef B200_STU_GEMM_H
#define B200_STU_GEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_GEMM_FLAG_LAYER_NORM 0x1u /* A = layer norm of x (else A = x) */
#define B200_GEMM_FLAG_SWISH 0x2u      /* with LAYER_NORM and ln_weight: A = sigmoid(ln(x)) * x   (is_swish) */

typedef struct B200GemmParams {
  uint32_t struct_size; /* sizeof(B200GemmParams) */
  uint32_t flags;
  int32_t dtype;        /* B200_HSTU_BF16 / _F16: element type of x, w, bias, ln_weight, ln_bias, out */
  float eps;            /* layer norm */
  int64_t M, K, N;      /* x [M, K], w [K, N], out [M, N] */
  int64_t x_row_stride, w_row_stride, out_row_stride; /* in elements */
  int64_t bias_row_stride; /* 0: one bias row [N] for every output row; else bias is [M, N] with this stride */
  const void* x;
  const void* w;
  const void* bias;
  const void* ln_weight; /* [K] or NULL (then ln_bias must be NULL too) */
  const void* ln_bias;
  void* out;
  float* mean;           /* [M], written with LAYER_NORM */
  float* rstd;           /* [M] */
  int32_t* status;       /* optional */
} B200GemmParams;

/* 1 if b200_stu_addmm serves this dtype and these sizes, else 0. */
int b200_stu_addmm_supported(const B200GemmParams* p);
int b200_stu_addmm(const B200GemmParams* p, void* stream);

/* Per-sequence projection of jagged rows: out[rows of b] = bias_b + x[rows of b] * w[b], where sequence b owns
 * rows [seq_offsets[b], seq_offsets[b + 1]) of x and w is a stack of num_seqs matrices [K, N].
 * Reference: jaggedDenseBmmAdd, recir/ops/kjt_split_per_feature.cpp:262-305 (a loop of at::addmm over the
 * sequences; schema generative_recommenders::triton_jagged_dense_bmm_add_fwd).  p describes x [M, K], out
 * [M, N] and the sizes as for b200_stu_addmm, with p->flags == 0, p->w = the first matrix and
 * w_seq_stride = K * w_row_stride (densely stacked matrices); the bias is one row per sequence
 * (per_row_bias == 0: bias [num_seqs, N], bias_row_stride its row stride) or one row per output row
 * (per_row_bias != 0: bias [M, N]).  The same tcgen05 kernel as b200_stu_addmm runs over a list of
 * (sequence, 128-row block) items that a small kernel builds on the device from the offsets (no host read);
 * workspace: b200_stu_jagged_bmm_workspace_bytes(M, num_seqs) bytes, 16-byte aligned, caller-owned.  Rows at
 * or past seq_offsets[num_seqs] are written as zeros.  Malformed offsets are clamped into [0, M] and flagged in
 * status[0] bit 0 like in b200_hstu.h. */
size_t b200_stu_jagged_bmm_workspace_bytes(int64_t rows, int64_t num_seqs);
int b200_stu_jagged_dense_bmm_add(const B200GemmParams* p, const void* seq_offsets, int offsets_i64, int64_t num_seqs,
                                  int64_t w_seq_stride, int per_row_bias, void* workspace, uint64_t workspace_bytes,
                                  void* stream);

/* Row-wise scaled fp8 projection: out = (a * a_scale[:, None]) (b * b_scale[:, None])^T (+ bias), with a [M, K] and
 * b [N, K] in float8 e4m3 (b is the weight, K-major as the reference takes it) and float32 scales per row of each.
 * Reference: fp8RowwiseAddMm, recir/ops/kjt_split_per_feature.cpp:533-556 (dequantise, at::mm in float32, add the
 * bias, cast; schema generative_recommenders::_triton_fp8_rowwise_addmm_fwd_impl).  Here the 8-bit products are
 * summed in float32 on the tensor cores (tcgen05.mma kind::f8f6f4, the same CTA-pair kernel as b200_stu_addmm)
 * and each sum is multiplied by its row's and its column's scale before the bias is added and the result
 * rounded once to bfloat16.  Served: K a multiple of 128 up to 1024, N a multiple of 8, bfloat16 bias [N] (or
 * NULL) and output, 16-byte aligned bases and row strides (strides in elements). */
typedef struct B200Fp8GemmParams {
  uint32_t struct_size; /* sizeof(B200Fp8GemmParams) */
  uint32_t flags;       /* 0 */
  int32_t out_dtype;    /* B200_HSTU_BF16 */
  int32_t reserved;
  int64_t M, K, N;
  int64_t a_row_stride, b_row_stride, out_row_stride;
  const void* a;        /* [M, K] float8 e4m3 */
  const void* b;        /* [N, K] float8 e4m3 */
  const float* a_scale; /* [M] */
  const float* b_scale; /* [N] */
  const void* bias;     /* [N] bfloat16 or NULL */
  void* out;            /* [M, N] bfloat16 */
  int32_t* status;      /* optional, as above */
} B200Fp8GemmParams;

int b200_stu_fp8_rowwise_addmm_supported(const B200Fp8GemmParams* p);
int b200_stu_fp8_rowwise_addmm(const B200Fp8GemmParams* p, void* stream);

#ifdef __cplusplus
}
#endif
#endif
