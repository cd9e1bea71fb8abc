// Position + timestamp embedding add (HBM-bound gather-add).
// Reference: addTimestampPositionEmbeddings, recir/ops/kjt_split_per_feature.cpp:307-428.
// Persistent CTAs; a warp takes 32 tokens at a time: each lane finds one token's sequence (binary search
// over the offsets, cached in shared memory when they fit) and computes its position index and time
// bucket, then the warp adds the two table rows to each token's row in turn.  The bucket arithmetic follows the
// reference step by step in float32 (int64 difference -> float, max with 1e-6, division by 60,
// log or sqrt, truncation, clamp to [0, 2048]); the sum of the two table rows is rounded to the
// tables' dtype and then to x's dtype before it is added, as the reference's tensor ops do.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_hstu.h"
#include "../../include/b200_stu_embed.h"
#include "hstu_launch.h"

namespace hstu {
namespace embed {
namespace {

constexpr int WARPS_PER_BLOCK = 8;

struct Args {
  const void* x; const void* pos; const void* ts; const long long* stamps;
  const void* off; const void* len; const void* tgt;
  void* out; int* pos_idx; int* ts_idx; int* status;
  long long rows, B, P, S, C, x_rs, out_rs, pos_rs, ts_rs;
  int cols, off64, len64, interleave, use_sqrt;
};

__device__ __forceinline__ long long at_i(const void* p, int i64, long long i) {
  return i64 ? reinterpret_cast<const long long*>(p)[i] : static_cast<long long>(reinterpret_cast<const int*>(p)[i]);
}

template <typename T> __device__ __forceinline__ void load8(const T* p, float (&f)[8]);
template <> __device__ __forceinline__ void load8<float>(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
template <> __device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) { f[2 * i] = __uint_as_float(w[i] << 16); f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u); }
}
template <> __device__ __forceinline__ void load8<__half>(const __half* p, float (&f)[8]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) { const float2 x = __half22float2(h[i]); f[2 * i] = x.x; f[2 * i + 1] = x.y; }
}
template <typename T> __device__ __forceinline__ float round_to(float x);
template <> __device__ __forceinline__ float round_to<float>(float x) { return x; }
template <> __device__ __forceinline__ float round_to<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <> __device__ __forceinline__ float round_to<__half>(float x) { return __half2float(__float2half_rn(x)); }
template <typename T> __device__ __forceinline__ void store8(T* p, const float (&f)[8]);
template <> __device__ __forceinline__ void store8<float>(float* p, const float (&f)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}
template <> __device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 v; uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) { const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]); w[i] = *reinterpret_cast<const uint32_t*>(&h); }
  *reinterpret_cast<uint4*>(p) = v;
}
template <> __device__ __forceinline__ void store8<__half>(__half* p, const float (&f)[8]) {
  uint4 v; uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) { const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]); w[i] = *reinterpret_cast<const uint32_t*>(&h); }
  *reinterpret_cast<uint4*>(p) = v;
}

// X = element type of x / out, TAB = element type of the tables (X or float)
template <typename X, typename TAB, bool SMEM>
__global__ void __launch_bounds__(WARPS_PER_BLOCK * 32) add_ts_pos_emb_kernel(Args a) {
  extern __shared__ long long sm_off[];
  if (SMEM) {
    for (long long i = threadIdx.x; i <= a.B; i += blockDim.x) sm_off[i] = at_i(a.off, a.off64, i);
    __syncthreads();
  }
  auto off = [&](long long i) { return SMEM ? sm_off[i] : at_i(a.off, a.off64, i); };
  const int lane = threadIdx.x & 31;
  const int nv = a.cols >> 3;
  const long long warps = static_cast<long long>(gridDim.x) * WARPS_PER_BLOCK;
  // A warp takes 32 consecutive tokens at a time: every lane resolves one token's sequence, position
  // index and time bucket (in parallel), then the warp processes the 32 rows one by one.
  for (long long r0 = (static_cast<long long>(blockIdx.x) * WARPS_PER_BLOCK + (threadIdx.x >> 5)) * 32; r0 < a.rows;
       r0 += warps * 32) {
    int my_pos = 0, my_tsb = 0, my_owned = 0;
    const long long r = r0 + lane;
    if (r < a.rows) {
      // sequence of packed row r: the last b with offsets[b] <= r (empty sequences are skipped)
      long long lo = 0, hi = a.B;
      while (lo < hi) {
        const long long mid = (lo + hi) >> 1;
        if (off(mid + 1) <= r) lo = mid + 1; else hi = mid;
      }
      if (lo < a.B && off(lo) <= r) {
        my_owned = 1;
        const long long b = lo, i = r - off(b);
        const long long L = at_i(a.len, a.len64, b);
        long long high = L;
        if (a.tgt) high -= at_i(a.tgt, a.len64, b) * (a.interleave ? 2 : 1);
        long long p = high - (i < high ? i : high) + a.C;  // kjt_split_per_feature.cpp:376-377
        if (p > a.P - 1) p = a.P - 1;
        if (i < a.C) p = i;
        // The reference rejects these inputs on the host (:363-373) and its index ops throw; a kernel
        // cannot throw, so out-of-range indices are clamped into the tables and flagged in status[0].
        bool clamped = false;
        if (p < 0) { p = 0; clamped = true; }
        if (p > a.P - 1) { p = a.P - 1; clamped = true; }
        my_pos = static_cast<int>(p);
        const long long* row = a.stamps + b * a.S;
        long long c_last = L - 1, c_i = i;
        if (c_last < 0) { c_last = 0; clamped = true; }
        if (c_last > a.S - 1) { c_last = a.S - 1; clamped = true; }
        if (c_i > a.S - 1) { c_i = a.S - 1; clamped = true; }
        if (clamped && a.status) atomicOr(a.status, 1);
        float d = static_cast<float>(row[c_last] - row[c_i]);  // :385-389
        d = fmaxf(d, 1e-6f) / 60.0f;
        d = a.use_sqrt ? sqrtf(d) : logf(d);
        long long q = static_cast<long long>(d);  // truncation toward zero
        my_tsb = static_cast<int>(q < 0 ? 0 : (q > 2048 ? 2048 : q));
      }
      a.pos_idx[r] = my_pos;  // coalesced: one index per lane; rows no sequence owns get index 0
      a.ts_idx[r] = my_tsb;
    }
    const int count = a.rows - r0 < 32 ? static_cast<int>(a.rows - r0) : 32;
    for (int k = 0; k < count; ++k) {
      const int pos = __shfl_sync(0xffffffffu, my_pos, k), tsb = __shfl_sync(0xffffffffu, my_tsb, k);
      const X* xr = reinterpret_cast<const X*>(a.x) + (r0 + k) * a.x_rs;
      X* orow = reinterpret_cast<X*>(a.out) + (r0 + k) * a.out_rs;
      if (!__shfl_sync(0xffffffffu, my_owned, k)) {
        // rows past the last offset belong to no sequence: defined output (zeros), never stale memory
        const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int v = lane; v < nv; v += 32) store8<X>(orow + 8 * v, z);
        continue;
      }
      const TAB* pr = reinterpret_cast<const TAB*>(a.pos) + static_cast<long long>(pos) * a.pos_rs;
      const TAB* tr = reinterpret_cast<const TAB*>(a.ts) + static_cast<long long>(tsb) * a.ts_rs;
      for (int v = lane; v < nv; v += 32) {
        float xv[8], pv[8], tv[8], o[8];
        load8<X>(xr + 8 * v, xv);
        load8<TAB>(pr + 8 * v, pv);
        load8<TAB>(tr + 8 * v, tv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = xv[i] + round_to<X>(round_to<TAB>(pv[i] + tv[i]));
        store8<X>(orow + 8 * v, o);
      }
    }
  }
}

}  // namespace
}  // namespace embed
}  // namespace hstu

extern "C" int b200_stu_add_ts_pos_emb(const B200EmbedParams* p, void* stream) {
  using namespace hstu::embed;
  if (p == nullptr) return B200_HSTU_EINVAL;
  if (p->struct_size != sizeof(B200EmbedParams)) return B200_HSTU_EVERSION;
  if (p->dtype != B200_HSTU_F32 && p->dtype != B200_HSTU_BF16 && p->dtype != B200_HSTU_F16) return B200_HSTU_EUNSUPPORTED;
  if (p->rows < 0 || p->cols <= 0 || p->num_seqs < 0) return B200_HSTU_EINVAL;
  if (p->cols % 8 != 0) return B200_HSTU_EUNSUPPORTED;
  if (p->rows == 0) return B200_HSTU_OK;
  if (!p->x || !p->out || !p->pos_table || !p->ts_table || !p->timestamps || !p->seq_offsets || !p->seq_lengths ||
      !p->pos_index || !p->ts_index || p->num_seqs == 0 || p->pos_rows <= 0 || p->ts_cols <= 0)
    return B200_HSTU_EINVAL;
  if (p->x_row_stride < p->cols || p->out_row_stride < p->cols || p->pos_row_stride < p->cols || p->ts_table_row_stride < p->cols)
    return B200_HSTU_EINVAL;
  auto bad = [](const void* q, long long stride) { return reinterpret_cast<uintptr_t>(q) % 16 != 0 || stride % 8 != 0; };
  if (bad(p->x, p->x_row_stride) || bad(p->out, p->out_row_stride) || bad(p->pos_table, p->pos_row_stride) ||
      bad(p->ts_table, p->ts_table_row_stride) || reinterpret_cast<uintptr_t>(p->timestamps) % 8 != 0)
    return B200_HSTU_EALIGN;
  Args a;
  a.x = p->x; a.pos = p->pos_table; a.ts = p->ts_table; a.stamps = reinterpret_cast<const long long*>(p->timestamps);
  a.off = p->seq_offsets; a.len = p->seq_lengths; a.tgt = p->num_targets;
  a.out = p->out; a.pos_idx = p->pos_index; a.ts_idx = p->ts_index; a.status = p->status;
  a.rows = p->rows; a.B = p->num_seqs; a.P = p->pos_rows; a.S = p->ts_cols; a.C = p->max_contextual_seq_len;
  a.x_rs = p->x_row_stride; a.out_rs = p->out_row_stride; a.pos_rs = p->pos_row_stride; a.ts_rs = p->ts_table_row_stride;
  a.cols = static_cast<int>(p->cols);
  a.off64 = (p->flags & B200_EMBED_FLAG_OFFSETS_I64) ? 1 : 0;
  a.len64 = (p->flags & B200_EMBED_FLAG_LENGTHS_I64) ? 1 : 0;
  a.interleave = (p->flags & B200_EMBED_FLAG_INTERLEAVE) ? 1 : 0;
  a.use_sqrt = (p->flags & B200_EMBED_FLAG_SQRT) ? 1 : 0;
  const bool tab32 = p->dtype == B200_HSTU_F32 || (p->flags & B200_EMBED_FLAG_TABLES_F32);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long per_block = static_cast<long long>(WARPS_PER_BLOCK) * 32;  // tokens one CTA takes per round
  const long long want = (a.rows + per_block - 1) / per_block, cap = static_cast<long long>(sms) * 8;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  const size_t smem = static_cast<size_t>(a.B + 1) * sizeof(long long);
  const bool use_smem = smem <= 40 * 1024 && a.rows >= 16 * (a.B + 1);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  hstu::set_error_stage("position/timestamp embedding kernel");
#define B200_EMBED_LAUNCH(X, TAB)                                                                   \
  if (use_smem) add_ts_pos_emb_kernel<X, TAB, true><<<grid, WARPS_PER_BLOCK * 32, smem, st>>>(a);    \
  else add_ts_pos_emb_kernel<X, TAB, false><<<grid, WARPS_PER_BLOCK * 32, 0, st>>>(a)
  if (p->dtype == B200_HSTU_F32) { B200_EMBED_LAUNCH(float, float); }
  else if (p->dtype == B200_HSTU_BF16) { if (tab32) { B200_EMBED_LAUNCH(__nv_bfloat16, float); } else { B200_EMBED_LAUNCH(__nv_bfloat16, __nv_bfloat16); } }
  else { if (tab32) { B200_EMBED_LAUNCH(__half, float); } else { B200_EMBED_LAUNCH(__half, __half); } }
#undef B200_EMBED_LAUNCH
  return cudaGetLastError() == cudaSuccess ? B200_HSTU_OK : B200_HSTU_ELAUNCH;
}
