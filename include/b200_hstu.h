/*
 * b200_hstu.h -- C ABI of the B200 (sm_100a) HSTU jagged attention library.
 *
 * The library implements one operator, forward and backward: the HSTU jagged
 * causal pointwise (SiLU, not softmax) attention that the reference exposes as
 *
 *   hammer::triton_ragged_attention_fwd(int N, float alpha, Tensor q, Tensor k,
 *       Tensor v, Tensor seq_offsets, str invalid_attn_mask_type,
 *       Tensor? num_targets, Tensor? attn_scale, int max_attn_len,
 *       int contextual_seq_len, int full_attn_size, int num_softmax_heads=0)
 *       -> (Tensor, Tensor)
 *
 * (reference: recir/ops/kjt_split_per_feature.cpp:602-693, schema :780-783),
 * and whose backward argument list the reference fixes in
 * recir/ops/helion/jagged_hstu_attention.py:875-887.
 *
 * Conventions
 *  - Every pointer in B200HstuParams is a DEVICE pointer owned by the caller.
 *    The entry points below never allocate or free device memory, never
 *    synchronise, and launch only on the stream they are given.
 *  - q, k: [T, H, Dqk]; v, o, d_o: [T, H, Dv]; gradients have the shape of the
 *    tensor they belong to.  Heads are dense inside a token row; the distance
 *    between token rows is given per tensor in ELEMENTS (>= H*D), the innermost
 *    dimension is contiguous.
 *  - Rows at or past seq_offsets[B] of every output are written as zeros.
 *  - Return value: 0 on success, a negative B200_HSTU_E* code otherwise.
 *    Argument errors are detected on the host before anything is launched.
 *  - Thread safety: the entry points keep no mutable global state besides
 *    one-time function-attribute set-up and, for b200_hstu_fwd_static_scratch, a
 *    mutex-guarded per-device cache of its scratch array's address; they may be
 *    called concurrently from several host threads on different streams (calls of
 *    b200_hstu_fwd_static_scratch on ONE device share its array and must not
 *    overlap on the GPU, see there).
 *  - Device-side diagnostics: kernels cannot return codes, so conditions found
 *    on the device are reported through params->status (optional, device
 *    int32[4], zeroed by the caller; the kernels only ever set bits / codes):
 *      status[0] bit 0  seq_offsets were malformed (negative, decreasing, past T,
 *                       or describing more 128-row blocks than T/128 + B): the
 *                       offending values were clamped and the call still ran
 *                       inside its buffers, but its results are not meaningful;
 *      status[1]        0, or the code of the first pipeline wait that gave up
 *                       after its time limit (101 TMA producer, 102 MMA issuer,
 *                       103 epilogue, 104 work-item scheduler): the kernel drained
 *                       and returned, outputs are incomplete.
 *    C callers should pass a status word and read it at a synchronisation point
 *    they already have.
 */
#ifndef B200_HSTU_H_
#define B200_HSTU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_HSTU_ABI_VERSION 1

/* B200HstuParams.dtype */
#define B200_HSTU_F32 0
#define B200_HSTU_BF16 1
#define B200_HSTU_F16 2

/* B200HstuParams.flags */
#define B200_HSTU_FLAG_CAUSAL 0x1u          /* invalid_attn_mask_type == "lower_triangular" */
#define B200_HSTU_FLAG_OFFSETS_I64 0x2u     /* seq_offsets is int64 (else int32) */
#define B200_HSTU_FLAG_TARGETS_I64 0x4u     /* num_targets is int64 (else int32) */
#define B200_HSTU_FLAG_SCALE_PER_TOKEN 0x8u /* attn_scale has T values (else 1) */
#define B200_HSTU_FLAG_FORCE_SIMT 0x10u     /* use the plain CUDA-core kernels (cross-check path) */
#define B200_HSTU_FLAG_BWD_SKIP_DQ 0x20u    /* backward: run only the dK/dV pass (dq is left untouched) */
#define B200_HSTU_FLAG_BWD_SKIP_DKV 0x40u   /* backward: run only the dQ pass (dk, dv are left untouched) */
#define B200_HSTU_FLAG_BWD_RECOMPUTE_DQ 0x100u /* backward: the dQ pass recomputes S and dP (small workspace) instead of
                                                 reading the dS tiles the dK/dV pass stored (see b200_hstu_workspace_bytes) */
#define B200_HSTU_FLAG_TRACE 0x80u /* instrumented builds (-DB200_HSTU_PROFILING) only: status is then a buffer of
                                         16 + 8192 ints and CTA 0 records an event trace behind the four status words */

/* error codes */
#define B200_HSTU_OK 0
#define B200_HSTU_EINVAL (-1)      /* null/ill-formed argument */
#define B200_HSTU_EUNSUPPORTED (-2) /* dtype / head dim outside what the kernels cover */
#define B200_HSTU_EALIGN (-3)      /* pointer or stride alignment */
#define B200_HSTU_EWORKSPACE (-4)  /* workspace missing or too small */
#define B200_HSTU_ELAUNCH (-5)     /* CUDA launch / driver error */
#define B200_HSTU_EVERSION (-6)    /* struct_size does not match this library */
#define B200_HSTU_ESCRATCH (-7)    /* problem needs more scratch than the built-in array holds */

typedef struct B200HstuParams {
  uint32_t struct_size; /* sizeof(B200HstuParams) as compiled by the caller */
  uint32_t flags;
  const void* q;
  const void* k;
  const void* v;
  void* o;         /* forward output (forward only) */
  const void* d_o; /* upstream gradient (backward only) */
  void* dq;        /* backward outputs */
  void* dk;
  void* dv;
  const void* seq_offsets; /* [B+1], monotone, last value <= T */
  const void* num_targets; /* [B] or NULL */
  const float* attn_scale; /* NULL => 1/max_seq_len; else 1 or T fp32 values */
  void* workspace;         /* >= b200_hstu_workspace_bytes(), 256-byte aligned */
  uint64_t workspace_bytes;
  int32_t* status; /* optional device int32[4]: device-side diagnostics, see the header comment */
  int64_t T;       /* token rows in q/k/v */
  int64_t q_row_stride, k_row_stride, v_row_stride, o_row_stride;
  int64_t do_row_stride, dq_row_stride, dk_row_stride, dv_row_stride;
  int32_t B, H, Dqk, Dv;
  int32_t dtype;
  int32_t max_seq_len; /* N: the default scale is 1/N; also sizes the locality chunks of the work list */
  int32_t max_attn_len;
  int32_t contextual_seq_len;
  int32_t full_attn_size;
  float alpha;
} B200HstuParams;

/* Forward: o = ((silu(alpha q k^T) * scale) .* keep) v.
 * Replaces raggedAttention, recir/ops/kjt_split_per_feature.cpp:602-693. */
int b200_hstu_fwd(const B200HstuParams* params, void* cuda_stream);

/* Backward: dq, dk, dv from d_o (two passes: a dK/dV-major pass and a dQ pass, no atomics
 * on the gradients).  Replaces autograd through raggedAttention / the backward op of
 * recir/ops/helion/jagged_hstu_attention.py:875-920. */
int b200_hstu_bwd(const B200HstuParams* params, void* cuda_stream);

/* Scratch bytes the call needs in params->workspace.  pass: 0 = forward, 1 = backward.
 * Depends only on B, H, T, Dqk, Dv, dtype, max_seq_len, contextual_seq_len and flags.
 * The forward needs a few hundred KB (the device-built work list).  The tensor-core backward by default also
 * keeps every 128 x 128 dS tile the dK/dV pass computes (32 KB each) for the dQ pass, which then has one
 * GEMM per tile left instead of three and no transcendental: room for H * (T / 128 + B) * (ceil(max_seq_len /
 * 128) + 1) / 2 tiles (twice that with a contextual prefix), of which only the tiles the mask keeps are
 * touched.  Above B200_HSTU_DS_WORKSPACE_LIMIT bytes, or with B200_HSTU_FLAG_BWD_RECOMPUTE_DQ, the dQ pass
 * recomputes S and dP instead and the workspace is as small as the forward's. */
#define B200_HSTU_DS_WORKSPACE_LIMIT (48ull << 30)
size_t b200_hstu_workspace_bytes(const B200HstuParams* params, int pass);

/* 1 if the tensor-core (tcgen05/TMA) kernels will serve this problem, 0 if the CUDA-core
 * kernels will, negative error code if the arguments are invalid.  pass as above. */
int b200_hstu_uses_tensor_cores(const B200HstuParams* params, int pass);

/* Number of kernels one call of the given pass launches (for launch accounting). */
int b200_hstu_launch_count(const B200HstuParams* params, int pass);

/* Forward for callers that cannot provide scratch memory.  (No counterpart in the reference;
 * added for this library's own callers.)
 *
 * b200_hstu_fwd needs a small work list in params->workspace, which normally comes from the
 * caller's allocator.  Some callers have no allocator to ask at the point of the call: a
 * host thread that must not block on cudaMalloc's implicit device synchronisation, a plugin
 * loaded into a runtime that owns all device memory and hands out none, or a replay loop
 * whose memory plan is frozen.  This entry point computes exactly what b200_hstu_fwd
 * computes but keeps the work list in an array built into the library
 * (B200_HSTU_STATIC_SCRATCH_BYTES of device memory, reserved on every GPU that loads the
 * library, until the process exits).  params->workspace and workspace_bytes are ignored.
 *
 *  - It never calls cudaMalloc/cudaFree or any allocating routine.
 *  - Problems whose work list does not fit (b200_hstu_workspace_bytes(params, 0) greater than
 *    B200_HSTU_STATIC_SCRATCH_BYTES) are rejected with B200_HSTU_ESCRATCH before anything
 *    is launched.
 *  - The first call on each device looks up the array's device address; make that first
 *    call before starting any stream capture on that device.
 *  - All calls on one device share the one array (it keeps the previous call's contents;
 *    every call rebuilds what it reads).  Two calls that overlap on the GPU, e.g. on two
 *    streams, race on it: serialise them. */
#define B200_HSTU_STATIC_SCRATCH_BYTES (4u << 20)
int b200_hstu_fwd_static_scratch(const B200HstuParams* params, void* cuda_stream);

const char* b200_hstu_strerror(int code);
/* Name and text of the CUDA runtime error behind the calling thread's most recent
 * B200_HSTU_ELAUNCH result ("" if there was none).  The pointer stays valid until the thread's
 * next failing call.  No counterpart in the reference. */
const char* b200_hstu_last_cuda_error(void);
/* Self-test of the bounded waits inside the tensor-core kernels: launches a one-warp kernel that waits
 * (limit_ns, at most 1e8) on a barrier nothing completes; the wait gives up, stores `code` in
 * status[1] (device int32[4], zeroed by the caller) and counts in status[2]; the kernel then ends
 * normally and the context stays usable.  No counterpart in the reference. */
int b200_hstu_debug_bounded_wait(int32_t* status, int code, uint64_t limit_ns, void* stream);
int b200_hstu_version(void);
/* sizeof(B200HstuParams) as this library was compiled (for foreign-language bindings). */
size_t b200_hstu_params_size(void);

/* ---- host-only diagnostics (no GPU needed) ---------------------------------------------
 * They evaluate, on the host, the very same inline functions the kernels compile for the
 * device, so a CPU test can check the mask rule and the tile-skipping logic against the
 * reference rule (recir/ops/kjt_split_per_feature.cpp:639-674).
 * A sequence is described by len, has_targets/num_targets; the mask by causal,
 * max_attn_len, contextual_seq_len and full_attn_size. */
typedef struct B200HstuMaskQuery {
  int32_t len, has_targets, num_targets;
  int32_t causal, max_attn_len, contextual_seq_len, full_attn_size;
} B200HstuMaskQuery;

/* keep(m, n): 1 if query m attends to key n (0 <= m, n < len). */
int b200_hstu_debug_keep(const B200HstuMaskQuery* mq, int m, int n);
/* Class of the 128x128 tile at (m0, n0): 0 = skipped, 1 = partial, 2 = fully kept.
 * rows_dont_care != 0: query rows past the sequence end may be treated as kept. */
int b200_hstu_debug_classify_tile(const B200HstuMaskQuery* mq, int m0, int n0, int rows_dont_care);
/* Interval form of the rule the tensor-core kernels evaluate per element:
 * row:  keep(m, n) <=> out[0] <= n < out[1] || n == out[2] || n == out[3]
 * col:  keep(m, n) <=> m == out[3] || out[0] <= m < out[1] || out[2] <= m < len */
void b200_hstu_debug_row_mask(const B200HstuMaskQuery* mq, int m, int32_t out[4]);
void b200_hstu_debug_col_mask(const B200HstuMaskQuery* mq, int n, int32_t out[4]);
/* Key blocks visited for the query block starting at m0: out = {lo, hi, extra_block0}. */
void b200_hstu_debug_key_blocks(const B200HstuMaskQuery* mq, int m0, int32_t out[3]);
/* Query blocks visited for the key block starting at n0: out = {lo, hi, 0}. */
void b200_hstu_debug_query_blocks(const B200HstuMaskQuery* mq, int n0, int32_t out[3]);

#ifdef __cplusplus
}
#endif
#endif /* B200_HSTU_H_ */
