/* C ABI of the jagged <-> dense marshalling and jagged concat / split kernels of an STU layer
 * (pure row copies driven by sequence offsets; bit-exact, HBM-bound).
 *
 * Reference semantics (Python, pure torch): recir/ops/jagged_ops.py
 *   _jagged_to_padded_dense_impl   :29-66     op recir::jagged_to_padded_dense (:118)
 *   _dense_to_jagged_forward_impl  :69-109    op recir::dense_to_jagged        (:115)
 *   _concat_2d_jagged_cpu          :218-250   op recir::concat_2d_jagged       (:123)
 *   _split_2d_jagged_cpu           :253-277   op recir::split_2d_jagged        (:128)
 * Every quirk of those index formulas is kept (clamped source rows, a sequence longer than the
 * padded width reading on into the next dense row), because parity is judged against them.
 *
 * Conventions of b200_hstu.h: plain pointers and sizes, caller-owned buffers, nothing allocated
 * or synchronised, launches go to the given stream, negative B200_HSTU_E* codes on error.
 */
#ifndef B200_STU_JAGGED_H
#define B200_STU_JAGGED_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  B200_JAGGED_TO_PADDED_DENSE = 0, /* dst [B*N rows] <- src0 [L rows] by offsets0, padding elsewhere */
  B200_DENSE_TO_JAGGED = 1,        /* dst [total_L rows] <- src0 [B*N rows] by offsets0, zeros where invalid */
  B200_JAGGED_CONCAT = 2,          /* dst [La+Lb rows] <- per sequence: rows of src0 then rows of src1 */
  B200_JAGGED_SPLIT_LEFT = 3,      /* dst [seq_len_a rows] <- src0 (the concatenated rows), left parts */
  B200_JAGGED_SPLIT_RIGHT = 4      /* dst [seq_len_b rows] <- src0, right parts */
};

#define B200_JAGGED_FLAG_OFFSETS_I64 0x1u /* offsets are int64 (else int32) */

typedef struct B200JaggedParams {
  uint32_t struct_size; /* sizeof(B200JaggedParams) */
  uint32_t flags;
  int32_t mode;
  int32_t reserved;
  int64_t num_seqs;     /* B: offsets arrays hold B + 1 entries */
  int64_t padded_len;   /* N (modes 0 and 1) */
  int64_t dst_rows;     /* rows to write */
  int64_t src0_rows, src1_rows;
  int64_t row_bytes;    /* bytes per row (same for sources and destination), a multiple of 2 */
  int64_t dst_row_stride, src0_row_stride, src1_row_stride; /* in bytes */
  const void* src0;
  const void* src1;     /* mode 2 only */
  void* dst;
  const void* offsets0; /* modes 0, 1: the sequence offsets; modes 2-4: offsets of the left parts */
  const void* offsets1; /* modes 2-4: offsets of the right parts */
  unsigned char pad[16]; /* mode 0: one padding element repeated to fill 16 bytes */
} B200JaggedParams;

int b200_stu_jagged_copy(const B200JaggedParams* p, void* stream);

#ifdef __cplusplus
}
#endif
#endif
