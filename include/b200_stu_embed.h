/* C ABI of the position + timestamp embedding add in front of the STU stack.
 *
 * Reference semantics (CPU, ATen): addTimestampPositionEmbeddings,
 * recir/ops/kjt_split_per_feature.cpp:307-428, schema hammer::add_ts_pos_emb_fwd_op (:776-779).
 * For token i of sequence b (L = sequence length, t = num_targets, C = max_contextual_seq_len,
 * P = rows of the position table):
 *   high = L - t * (interleave_targets ? 2 : 1)
 *   pos  = i < C ? i : min(high - min(i, high) + C, P - 1)
 *   dt   = max(float(ts[b, L-1] - ts[b, i]), 1e-6) / 60
 *   tsb  = clamp(int64(log(dt)) or int64(sqrt(dt)), 0, 2048)
 *   out[i] = x[i] + cast(pos_table[pos] + ts_table[tsb])
 * The kernel writes out, pos and tsb per token; sorting the two index arrays (the reference
 * returns them sorted together with the sort permutations) is left to the caller.  Rows at or past
 * seq_offsets[B] belong to no sequence: their out rows are zeros and their indices 0.
 *
 * Conventions of b200_hstu.h: plain pointers and sizes, caller-owned buffers, nothing allocated
 * or synchronised, launches go to the given stream, negative B200_HSTU_E* codes on error.
 */
#ifndef B200_STU_EMBED_H
#define B200_STU_EMBED_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_EMBED_FLAG_OFFSETS_I64 0x1u      /* seq_offsets int64 (else int32) */
#define B200_EMBED_FLAG_LENGTHS_I64 0x2u      /* seq_lengths and num_targets int64 (else int32) */
#define B200_EMBED_FLAG_INTERLEAVE 0x4u       /* interleave_targets */
#define B200_EMBED_FLAG_SQRT 0x8u             /* time_bucket_fn == "sqrt" (else "log") */
#define B200_EMBED_FLAG_TABLES_F32 0x10u      /* embedding tables are float32 although x is 16-bit */

typedef struct B200EmbedParams {
  uint32_t struct_size; /* sizeof(B200EmbedParams) */
  uint32_t flags;
  int32_t dtype;        /* B200_HSTU_F32 / _BF16 / _F16: element type of x and out */
  int32_t reserved;
  int64_t rows, cols;   /* x is [rows, cols]; cols a multiple of 8 */
  int64_t num_seqs;     /* B */
  int64_t pos_rows;     /* P */
  int64_t ts_cols;      /* second dimension of timestamps */
  int64_t max_contextual_seq_len;
  int64_t x_row_stride, out_row_stride, pos_row_stride, ts_table_row_stride; /* in elements */
  const void* x;
  const void* pos_table;   /* [P, cols] */
  const void* ts_table;    /* [>= 2049, cols] */
  const int64_t* timestamps; /* [B, ts_cols], row-major */
  const void* seq_offsets; /* [B + 1] */
  const void* seq_lengths; /* [B] */
  const void* num_targets; /* [B] or NULL */
  void* out;               /* [rows, cols] */
  int32_t* pos_index;      /* [rows] */
  int32_t* ts_index;       /* [rows] */
  int32_t* status;         /* optional device int32[>= 1], zeroed by the caller: bit 0 of status[0] is set when
                              a position or timestamp index fell outside its table and was clamped into it
                              (sequence length 0 or beyond ts_cols, more contextual rows than table rows);
                              the reference refuses such inputs on the host (:363-373) */
} B200EmbedParams;

int b200_stu_add_ts_pos_emb(const B200EmbedParams* p, void* stream);

#ifdef __cplusplus
}
#endif
#endif
