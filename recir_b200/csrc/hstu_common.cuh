// Shared host/device definitions for the HSTU jagged attention kernels:
// the per-sequence descriptor, the keep-mask predicate and small math helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_hstu.h"

#if defined(__CUDACC__)
#define HSTU_HD __host__ __device__ __forceinline__
#else
#define HSTU_HD inline
#endif

namespace hstu {

// Mask options shared by a whole call.
struct MaskOpts {
  int causal;  // 1 = "lower_triangular"
  int window;  // max_attn_len (0 = unlimited)
  int ctx;     // contextual_seq_len > 0
  int full;    // full_attn_size
};

// One sequence of the jagged batch.
struct SeqInfo {
  long long start;  // first token row
  int len;          // L
  int hist;         // L - num_targets when targets are given (may be <= 0), else L
  int has_targets;
  int boundary;     // L - num_targets - full_attn_size
  long long tile_base;  // backward with stored dS tiles: index of the sequence's first tile (else unused)
};

// keep(m, n) for 0 <= m, n < len.  Same rule as the reference builds with tensors in
// recir/ops/kjt_split_per_feature.cpp:639-674 (ids clamped at the first target, diagonal
// always kept, causal/window on clamped-id distance, optional full-attention tail on
// ids zeroed below a boundary, contextual flag makes clamped id 0 visible to everyone).
HSTU_HD bool keep(int m, int n, const SeqInfo& s, const MaskOpts& o) {
  if (m == n) return true;
  const int im = s.has_targets ? (m < s.hist ? m : s.hist) : m;
  const int in = s.has_targets ? (n < s.hist ? n : s.hist) : n;
  int d = im - in;
  if (!o.causal) d = d < 0 ? -d : d;
  bool k = false;
  if (o.window > 0) {
    k = o.causal ? (d > 0 && d <= o.window) : (d <= o.window);
    if (o.full > 0) {
      const int gm = im < s.boundary ? 0 : im;
      const int gn = in < s.boundary ? 0 : in;
      k = k || (gm - gn > 0);
    }
  } else if (o.causal) {
    k = d > 0;
  }
  if (o.ctx) k = k || (in == 0);
  return k;
}

// True when no key with index > m can be kept for any query m (upper triangle empty),
// which lets causal kernels stop the key loop at the diagonal.
HSTU_HD bool upper_triangle_empty(const SeqInfo& s, const MaskOpts& o) {
  if (!o.causal) return false;
  // contextual flag with clamped id 0 on every token (hist == 0) keeps the whole square
  if (o.ctx && s.has_targets && s.hist == 0) return false;
  return true;
}

struct KernelArgs {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  const void* d_o;
  void* dq;
  void* dk;
  void* dv;
  const void* seq_offsets;
  const void* num_targets;
  const float* attn_scale;
  int* status;
  int* trace_buf;  // instrumented builds only: event trace of CTA 0 (B200_HSTU_FLAG_TRACE), else null
  long long T;
  long long q_rs, k_rs, v_rs, o_rs, do_rs, dq_rs, dk_rs, dv_rs;
  int B, H, Dqk, Dv;
  int offsets_i64, targets_i64, scale_mode;  // scale_mode: 0 = 1/N, 1 = scalar, 2 = per token
  int skip_dq, skip_dkv;                     // backward: leave one of the two passes out (timing aid)
  int max_seq_len;                           // the caller's bound on sequence lengths (sizes locality chunks)
  int recompute_dq;                          // backward: the dQ pass recomputes S and dP instead of reading stored dS tiles
  // Backward with stored dS tiles (set by the tensor-core launch code from the workspace, null otherwise):
  // the dK/dV pass writes every 128 x 128 dS^T tile it computes (keys x queries, 16-bit, 32 KB), the dQ
  // pass reads them back as the A operand of dQ += dS K.
  unsigned char* ds_tiles;                   // first tile
  const long long* ds_tile_base;             // [B] first tile index of every sequence (per head)
  long long ds_tile_cap;                     // tiles the region holds (indices are clamped to it)
  int ds_square;                             // tiles of a sequence indexed as a square (else as a triangle)
  float alpha;
  float inv_n;
  MaskOpts mask;
};

#if defined(__CUDACC__)
__device__ __forceinline__ long long load_index(const void* p, int i64, long long idx) {
  return i64 ? reinterpret_cast<const long long*>(p)[idx]
             : static_cast<long long>(reinterpret_cast<const int*>(p)[idx]);
}

// Reads sequence b, clamping malformed offsets into [0, T] (and flagging them in status[0]).
__device__ __forceinline__ SeqInfo load_seq(const KernelArgs& a, int b) {
  long long s = load_index(a.seq_offsets, a.offsets_i64, b);
  long long e = load_index(a.seq_offsets, a.offsets_i64, b + 1);
  bool bad = false;
  if (s < 0) { s = 0; bad = true; }
  if (s > a.T) { s = a.T; bad = true; }
  if (e < s) { e = s; bad = true; }
  if (e > a.T) { e = a.T; bad = true; }
  if (e - s > 0x3fffffffLL) { e = s + 0x3fffffffLL; bad = true; }
  if (bad && a.status) atomicOr(a.status, 1);
  SeqInfo r;
  r.start = s;
  r.len = static_cast<int>(e - s);
  long long t = 0;
  r.has_targets = a.num_targets != nullptr;
  if (r.has_targets) {
    t = load_index(a.num_targets, a.targets_i64, b);
    if (t < -0x3fffffffLL) t = -0x3fffffffLL;
    if (t > 0x3fffffffLL) t = 0x3fffffffLL;
  }
  r.hist = r.has_targets ? static_cast<int>(r.len - t) : r.len;
  r.boundary = static_cast<int>(r.len - t) - a.mask.full;
  r.tile_base = 0;
  return r;
}

// Same without the diagnostics: no branch depends on the loaded values, so the loads can stay
// in flight while other work proceeds (used to fetch the next work item early).
__device__ __forceinline__ SeqInfo load_seq_quiet(const KernelArgs& a, int b) {
  long long s = load_index(a.seq_offsets, a.offsets_i64, b);
  long long e = load_index(a.seq_offsets, a.offsets_i64, b + 1);
  s = s < 0 ? 0 : (s > a.T ? a.T : s);
  e = e < s ? s : (e > a.T ? a.T : e);
  e = (e - s > 0x3fffffffLL) ? s + 0x3fffffffLL : e;
  SeqInfo r;
  r.start = s;
  r.len = static_cast<int>(e - s);
  long long t = 0;
  r.has_targets = a.num_targets != nullptr;
  if (r.has_targets) {
    t = load_index(a.num_targets, a.targets_i64, b);
    t = t < -0x3fffffffLL ? -0x3fffffffLL : (t > 0x3fffffffLL ? 0x3fffffffLL : t);
  }
  r.hist = r.has_targets ? static_cast<int>(r.len - t) : r.len;
  r.boundary = static_cast<int>(r.len - t) - a.mask.full;
  r.tile_base = 0;
  return r;
}

// Two-step variant for software-pipelined fetches: `load_seq_raw` only issues the loads (no
// instruction consumes them), `finish_seq` turns them into a SeqInfo later.
struct SeqRaw {
  long long s, e, t;
};
__device__ __forceinline__ SeqRaw load_seq_raw(const KernelArgs& a, int b) {
  SeqRaw r;
  r.s = load_index(a.seq_offsets, a.offsets_i64, b);
  r.e = load_index(a.seq_offsets, a.offsets_i64, b + 1);
  r.t = a.num_targets != nullptr ? load_index(a.num_targets, a.targets_i64, b) : 0;
  return r;
}
__device__ __forceinline__ SeqInfo finish_seq(const KernelArgs& a, const SeqRaw& raw) {
  long long s = raw.s, e = raw.e, t = raw.t;
  s = s < 0 ? 0 : (s > a.T ? a.T : s);
  e = e < s ? s : (e > a.T ? a.T : e);
  e = (e - s > 0x3fffffffLL) ? s + 0x3fffffffLL : e;
  t = t < -0x3fffffffLL ? -0x3fffffffLL : (t > 0x3fffffffLL ? 0x3fffffffLL : t);
  SeqInfo r;
  r.start = s;
  r.len = static_cast<int>(e - s);
  r.has_targets = a.num_targets != nullptr;
  r.hist = r.has_targets ? static_cast<int>(r.len - t) : r.len;
  r.boundary = static_cast<int>(r.len - t) - a.mask.full;
  r.tile_base = 0;
  return r;
}

__device__ __forceinline__ float row_scale(const KernelArgs& a, long long token) {
  if (a.scale_mode == 0) return a.inv_n;
  if (a.scale_mode == 1) return __ldg(a.attn_scale);
  return __ldg(a.attn_scale + token);
}

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
#endif

}  // namespace hstu
