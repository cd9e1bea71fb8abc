// Jagged <-> dense marshalling and jagged concat / split: one row-gather kernel, five index rules.
// Reference: recir/ops/jagged_ops.py:29-66 (jagged_to_padded_dense), :69-109 (dense_to_jagged),
// :218-250 (concat_2d_jagged), :253-277 (split_2d_jagged).  Byte copies, so any element type.
//
// Persistent CTAs; a warp takes 32 consecutive destination rows at a time: each lane finds the source
// of one row (a binary search over the B + 1 offsets where the rule needs the sequence of a packed
// position), then the warp copies the rows one by one in 16-byte pieces (2-byte pieces for rows or
// pointers that are not 16-byte aligned).  When they fit, the offsets are copied to shared memory
// once per CTA so that the searches do not wait on global memory.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_hstu.h"
#include "../../include/b200_stu_jagged.h"
#include "hstu_launch.h"

namespace hstu {
namespace jagged {
namespace {

constexpr int WARPS_PER_BLOCK = 8;

struct Args {
  const unsigned char* src0; const unsigned char* src1; unsigned char* dst;
  const void* off0; const void* off1;
  long long B, N, dst_rows, src0_rows, src1_rows, row_bytes, dst_rs, src0_rs, src1_rs;
  int mode, i64;
  uint4 pad;
};

__device__ __forceinline__ long long off_at(const void* p, int i64, long long i) {
  return i64 ? reinterpret_cast<const long long*>(p)[i] : static_cast<long long>(reinterpret_cast<const int*>(p)[i]);
}
__device__ __forceinline__ long long clampll(long long v, long long lo, long long hi) { return v < lo ? lo : (v > hi ? hi : v); }

// number of entries among f(first .. first + count - 1) that are <= x, for a non-decreasing f
// (torch.searchsorted(seq, x, right=True))
template <typename F>
__device__ __forceinline__ long long upper_bound(F f, long long first, long long count, long long x) {
  long long lo = 0, hi = count;
  while (lo < hi) {
    const long long mid = (lo + hi) >> 1;
    if (f(first + mid) <= x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Source of destination row r: which = 0 (src0), 1 (src1), 2 (padding pattern), 3 (zeros).
template <bool SMEM>
__device__ __forceinline__ void locate(const Args& a, const long long* sm0, const long long* sm1, long long r, int& which,
                                       long long& src) {
  auto o0 = [&](long long i) { return SMEM ? sm0[i] : off_at(a.off0, a.i64, i); };
  auto o1 = [&](long long i) { return SMEM ? sm1[i] : off_at(a.off1, a.i64, i); };
  which = 0;
  src = 0;
  switch (a.mode) {
    case B200_JAGGED_TO_PADDED_DENSE: {  // jagged_ops.py:46-63
      const long long b = r / a.N, n = r - b * a.N;
      const long long start = o0(b), len = o0(b + 1) - start;
      if (n < len) src = clampll(start + n, 0, a.src0_rows > 0 ? a.src0_rows - 1 : 0);
      else which = 2;
      if (a.src0_rows == 0) which = 2;
      break;
    }
    case B200_DENSE_TO_JAGGED: {  // jagged_ops.py:91-108
      // segment id = number of interior boundaries offsets[1 .. B-1] that are <= r (and < total_L), at most B - 1
      long long seg = upper_bound(o0, 1, a.B - 1, r);
      seg = clampll(seg, 0, a.B - 1);
      const long long intra = r - o0(seg), len = o0(seg + 1) - o0(seg);
      const bool valid = r < o0(a.B) && intra >= 0 && intra < len;
      src = clampll(seg * a.N + intra, 0, a.B * a.N > 0 ? a.B * a.N - 1 : 0);
      if (!valid) which = 3;
      break;
    }
    case B200_JAGGED_CONCAT: {  // jagged_ops.py:235-250
      auto comb = [&](long long i) { return o0(i) + o1(i); };
      const long long b = clampll(upper_bound(comb, 1, a.B, r), 0, a.B - 1);
      const long long intra = r - comb(b), la = o0(b + 1) - o0(b);
      if (intra < la) {
        src = clampll(o0(b) + intra, 0, a.src0_rows - 1);
      } else {
        which = 1;
        src = clampll(o1(b) + intra - la, 0, a.src1_rows - 1);
      }
      break;
    }
    case B200_JAGGED_SPLIT_LEFT: {  // jagged_ops.py:266-270
      const long long b = clampll(upper_bound(o0, 1, a.B, r), 0, a.B - 1);
      src = clampll(r + o1(b), 0, a.src0_rows - 1);
      break;
    }
    default: {  // B200_JAGGED_SPLIT_RIGHT, jagged_ops.py:271-276
      const long long b = clampll(upper_bound(o1, 1, a.B, r), 0, a.B - 1);
      src = clampll(r + o0(b + 1), 0, a.src0_rows - 1);
      break;
    }
  }
}

template <bool VEC16, bool SMEM>
__global__ void __launch_bounds__(WARPS_PER_BLOCK * 32) jagged_copy_kernel(Args a) {
  extern __shared__ long long sm_off[];
  const long long* sm0 = sm_off;
  const long long* sm1 = sm_off + (a.B + 1);
  if (SMEM) {
    for (long long i = threadIdx.x; i <= a.B; i += blockDim.x) {
      sm_off[i] = off_at(a.off0, a.i64, i);
      if (a.off1) sm_off[a.B + 1 + i] = off_at(a.off1, a.i64, i);
    }
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * WARPS_PER_BLOCK;
  // A warp takes 32 consecutive destination rows at a time: every lane resolves the source of one
  // row (the searches run in parallel instead of one after the other), then the warp copies the
  // rows one by one.
  for (long long r0 = (static_cast<long long>(blockIdx.x) * WARPS_PER_BLOCK + (threadIdx.x >> 5)) * 32; r0 < a.dst_rows;
       r0 += warps * 32) {
    int my_which = 3;
    long long my_src = 0;
    if (r0 + lane < a.dst_rows) locate<SMEM>(a, sm0, sm1, r0 + lane, my_which, my_src);
    const int count = a.dst_rows - r0 < 32 ? static_cast<int>(a.dst_rows - r0) : 32;
    for (int k = 0; k < count; ++k) {
      const int which = __shfl_sync(0xffffffffu, my_which, k);
      const long long src = __shfl_sync(0xffffffffu, my_src, k);
      unsigned char* d = a.dst + (r0 + k) * a.dst_rs;
      const unsigned char* s = which == 0 ? a.src0 + src * a.src0_rs : (which == 1 ? a.src1 + src * a.src1_rs : nullptr);
      if (VEC16) {
        const long long nv = a.row_bytes >> 4;
        const uint4 fill = which == 2 ? a.pad : make_uint4(0u, 0u, 0u, 0u);
        for (long long v = lane; v < nv; v += 32)
          reinterpret_cast<uint4*>(d)[v] = s ? __ldg(reinterpret_cast<const uint4*>(s) + v) : fill;
      } else {
        const long long nv = a.row_bytes >> 1;
        for (long long v = lane; v < nv; v += 32) {
          unsigned short x = 0;
          if (s) x = reinterpret_cast<const unsigned short*>(s)[v];
          else if (which == 2) x = reinterpret_cast<const unsigned short*>(&a.pad)[v & 7];  // 2-byte pieces of the pattern
          reinterpret_cast<unsigned short*>(d)[v] = x;
        }
      }
    }
  }
}

}  // namespace
}  // namespace jagged
}  // namespace hstu

extern "C" int b200_stu_jagged_copy(const B200JaggedParams* p, void* stream) {
  using namespace hstu::jagged;
  if (p == nullptr) return B200_HSTU_EINVAL;
  if (p->struct_size != sizeof(B200JaggedParams)) return B200_HSTU_EVERSION;
  if (p->mode < B200_JAGGED_TO_PADDED_DENSE || p->mode > B200_JAGGED_SPLIT_RIGHT) return B200_HSTU_EINVAL;
  if (p->dst_rows < 0 || p->row_bytes <= 0 || p->row_bytes % 2 != 0 || p->num_seqs < 0) return B200_HSTU_EINVAL;
  if (p->dst_rows == 0) return B200_HSTU_OK;
  if (p->num_seqs == 0 || !p->dst || !p->offsets0) return B200_HSTU_EINVAL;
  const bool two_offsets = p->mode >= B200_JAGGED_CONCAT;
  if (two_offsets && !p->offsets1) return B200_HSTU_EINVAL;
  if (p->mode == B200_JAGGED_CONCAT && (!p->src0 || !p->src1 || p->src0_rows <= 0 || p->src1_rows <= 0)) return B200_HSTU_EINVAL;
  if (p->mode != B200_JAGGED_TO_PADDED_DENSE && p->mode != B200_JAGGED_CONCAT && (!p->src0 || p->src0_rows <= 0)) return B200_HSTU_EINVAL;
  if (p->mode == B200_JAGGED_TO_PADDED_DENSE && p->src0_rows > 0 && !p->src0) return B200_HSTU_EINVAL;
  if ((p->mode <= B200_DENSE_TO_JAGGED) && p->padded_len <= 0) return B200_HSTU_EINVAL;
  const int osz = (p->flags & B200_JAGGED_FLAG_OFFSETS_I64) ? 8 : 4;
  if (reinterpret_cast<uintptr_t>(p->offsets0) % osz != 0 || (two_offsets && reinterpret_cast<uintptr_t>(p->offsets1) % osz != 0))
    return B200_HSTU_EALIGN;
  if (p->dst_row_stride < p->row_bytes || (p->src0 && p->src0_row_stride < p->row_bytes) ||
      (p->src1 && p->src1_row_stride < p->row_bytes))
    return B200_HSTU_EINVAL;
  auto a16 = [](const void* q, long long stride) { return reinterpret_cast<uintptr_t>(q) % 16 == 0 && stride % 16 == 0; };
  auto a2 = [](const void* q, long long stride) { return reinterpret_cast<uintptr_t>(q) % 2 == 0 && stride % 2 == 0; };
  if (!a2(p->dst, p->dst_row_stride) || (p->src0 && !a2(p->src0, p->src0_row_stride)) || (p->src1 && !a2(p->src1, p->src1_row_stride)))
    return B200_HSTU_EALIGN;
  const bool vec = p->row_bytes % 16 == 0 && a16(p->dst, p->dst_row_stride) && (!p->src0 || a16(p->src0, p->src0_row_stride)) &&
                   (!p->src1 || a16(p->src1, p->src1_row_stride));
  Args a;
  a.src0 = static_cast<const unsigned char*>(p->src0); a.src1 = static_cast<const unsigned char*>(p->src1);
  a.dst = static_cast<unsigned char*>(p->dst); a.off0 = p->offsets0; a.off1 = p->offsets1;
  a.B = p->num_seqs; a.N = p->padded_len; a.dst_rows = p->dst_rows; a.src0_rows = p->src0_rows; a.src1_rows = p->src1_rows;
  a.row_bytes = p->row_bytes; a.dst_rs = p->dst_row_stride; a.src0_rs = p->src0_row_stride; a.src1_rs = p->src1_row_stride;
  a.mode = p->mode; a.i64 = (p->flags & B200_JAGGED_FLAG_OFFSETS_I64) ? 1 : 0;
  a.pad = *reinterpret_cast<const uint4*>(p->pad);
  hstu::set_error_stage("jagged row copy kernel");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long per_block = static_cast<long long>(WARPS_PER_BLOCK) * 32;  // rows one CTA takes per round
  const long long want = (a.dst_rows + per_block - 1) / per_block, cap = static_cast<long long>(sms) * 8;
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  const size_t smem = static_cast<size_t>(a.B + 1) * sizeof(long long) * (two_offsets ? 2 : 1);
  const bool use_smem = smem <= 40 * 1024 && a.dst_rows >= 16 * (a.B + 1);  // worth it only when a CTA handles many rows
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_smem) {
    if (vec) jagged_copy_kernel<true, true><<<grid, WARPS_PER_BLOCK * 32, smem, st>>>(a);
    else jagged_copy_kernel<false, true><<<grid, WARPS_PER_BLOCK * 32, smem, st>>>(a);
  } else {
    if (vec) jagged_copy_kernel<true, false><<<grid, WARPS_PER_BLOCK * 32, 0, st>>>(a);
    else jagged_copy_kernel<false, false><<<grid, WARPS_PER_BLOCK * 32, 0, st>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? B200_HSTU_OK : B200_HSTU_ELAUNCH;
}
