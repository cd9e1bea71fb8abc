// CUDA-core (SIMT) HSTU jagged attention kernels: forward, dQ pass, dK/dV pass.
//
// These cover every dtype, head dimension (<= 256) and mask option of the operator and
// serve (a) the shapes the tensor-core kernels do not take (fp32, Dqk != Dv, head dims
// other than 128, non-causal masks) and (b) an independent
// on-device cross-check of the tensor-core path.  All arithmetic is fp32 with an exact
// sigmoid; results are rounded once on store.
//
// Tiling: one CTA of 256 threads owns a 32-row tile of queries (forward, dQ) or of keys
// (dK/dV) of one (sequence, head) and streams 32-row tiles of the other side through
// shared memory.  Thread (ty, tx) = (warp, lane) computes scores for rows ty*4..ty*4+3,
// column tx, then accumulates output rows ty*4..+3, columns tx + 32*j.
#include "hstu_common.cuh"
#include "hstu_launch.h"

namespace hstu {
namespace {

constexpr int TILE = 32;
constexpr int THREADS = 256;
constexpr int MAXJ = 8;  // head dim <= 256

template <typename T>
__device__ __forceinline__ void load_tile(float* dst, int ld, const T* src, long long row_stride,
                                          long long first_row, int rows_valid, int head_off, int D) {
  // dst[r][d] = src[(first_row + r) * row_stride + head_off + d], zero for r >= rows_valid
  for (int idx = threadIdx.x; idx < TILE * D; idx += THREADS) {
    const int r = idx / D, d = idx - r * D;
    float x = 0.f;
    if (r < rows_valid) x = to_f32<T>(src[(first_row + r) * row_stride + head_off + d]);
    dst[r * ld + d] = x;
  }
}

__device__ __forceinline__ float dot_rows(const float* a, const float* b, int D) {
  float s = 0.f;
#pragma unroll 8
  for (int d = 0; d < D; ++d) s = fmaf(a[d], b[d], s);
  return s;
}

__device__ __forceinline__ float sigmoidf_exact(float x) { return 1.f / (1.f + expf(-x)); }

// ---------------------------------------------------------------------------------
// forward (MODE 0) and dQ (MODE 1): query-tile-major
// ---------------------------------------------------------------------------------
template <typename T, int MODE>
__global__ void __launch_bounds__(THREADS) simt_q_major(KernelArgs a) {
  extern __shared__ float smem[];
  const int Dq = a.Dqk, Dv = a.Dv;
  const int ldq = Dq + 1, ldv = Dv + 1;
  float* Qs = smem;                    // [32][ldq]
  float* Ks = Qs + TILE * ldq;         // [32][ldq]
  float* Vs = Ks + TILE * ldq;         // [32][ldv]
  float* Ps = Vs + TILE * ldv;         // [32][33]
  float* dOs = Ps + TILE * (TILE + 1); // [32][ldv]  (dQ only)

  const int b = blockIdx.z, head = blockIdx.y;
  const SeqInfo s = load_seq(a, b);
  const int L = s.len;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const bool tri = upper_triangle_empty(s, a.mask);
  const int DJ = (MODE == 0 ? Dv : Dq);  // width of the accumulated output

  for (int m0 = blockIdx.x * TILE; m0 < L; m0 += gridDim.x * TILE) {
    const int mrows = min(TILE, L - m0);
    __syncthreads();
    load_tile<T>(Qs, ldq, reinterpret_cast<const T*>(a.q), a.q_rs, s.start + m0, mrows, head * Dq, Dq);
    if (MODE == 1)
      load_tile<T>(dOs, ldv, reinterpret_cast<const T*>(a.d_o), a.do_rs, s.start + m0, mrows, head * Dv, Dv);
    float acc[4][MAXJ];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < MAXJ; ++j) acc[i][j] = 0.f;

    const int n_end = tri ? min(L, m0 + TILE) : L;
    for (int n0 = 0; n0 < n_end; n0 += TILE) {
      const int nrows = min(TILE, L - n0);
      __syncthreads();
      load_tile<T>(Ks, ldq, reinterpret_cast<const T*>(a.k), a.k_rs, s.start + n0, nrows, head * Dq, Dq);
      load_tile<T>(Vs, ldv, reinterpret_cast<const T*>(a.v), a.v_rs, s.start + n0, nrows, head * Dv, Dv);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty * 4 + i;
        const int m = m0 + r, n = n0 + tx;
        float val = 0.f;
        if (m < L && n < L && keep(m, n, s, a.mask)) {
          const float x = a.alpha * dot_rows(Qs + r * ldq, Ks + tx * ldq, Dq);
          const float sg = sigmoidf_exact(x);
          if (MODE == 0) {
            val = x * sg;
          } else {
            const float dp = dot_rows(dOs + r * ldv, Vs + tx * ldv, Dv);
            val = dp * sg * (1.f + x * (1.f - sg));
          }
        }
        Ps[r * (TILE + 1) + tx] = val;
      }
      __syncthreads();
      const float* Bs = (MODE == 0) ? Vs : Ks;
      const int ldb = (MODE == 0) ? ldv : ldq;
      for (int n = 0; n < TILE; ++n) {
        float p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = Ps[(ty * 4 + i) * (TILE + 1) + n];
#pragma unroll
        for (int j = 0; j < MAXJ; ++j) {
          const int c = tx + 32 * j;
          if (c < DJ) {
            const float bv = Bs[n * ldb + c];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i][j] = fmaf(p[i], bv, acc[i][j]);
          }
        }
      }
    }
    // epilogue: per-row scale (and alpha for dQ), one rounding on store
    T* outp = reinterpret_cast<T*>(MODE == 0 ? a.o : a.dq);
    const long long ors = (MODE == 0 ? a.o_rs : a.dq_rs);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + ty * 4 + i;
      if (m < L) {
        float sc = row_scale(a, s.start + m);
        if (MODE == 1) sc *= a.alpha;
#pragma unroll
        for (int j = 0; j < MAXJ; ++j) {
          const int c = tx + 32 * j;
          if (c < DJ) outp[(s.start + m) * ors + head * DJ + c] = from_f32<T>(acc[i][j] * sc);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// dK/dV: key-tile-major
// ---------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(THREADS) simt_kv_major(KernelArgs a) {
  extern __shared__ float smem[];
  const int Dq = a.Dqk, Dv = a.Dv;
  const int ldq = Dq + 1, ldv = Dv + 1;
  float* Qs = smem;                     // [32][ldq]
  float* Ks = Qs + TILE * ldq;          // [32][ldq]
  float* Vs = Ks + TILE * ldq;          // [32][ldv]
  float* dOs = Vs + TILE * ldv;         // [32][ldv]
  float* Pt = dOs + TILE * ldv;         // [n][m] 32 x 33
  float* dSt = Pt + TILE * (TILE + 1);  // [n][m] 32 x 33

  const int b = blockIdx.z, head = blockIdx.y;
  const SeqInfo s = load_seq(a, b);
  const int L = s.len;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const bool tri = upper_triangle_empty(s, a.mask);

  for (int n0 = blockIdx.x * TILE; n0 < L; n0 += gridDim.x * TILE) {
    const int nrows = min(TILE, L - n0);
    __syncthreads();
    load_tile<T>(Ks, ldq, reinterpret_cast<const T*>(a.k), a.k_rs, s.start + n0, nrows, head * Dq, Dq);
    load_tile<T>(Vs, ldv, reinterpret_cast<const T*>(a.v), a.v_rs, s.start + n0, nrows, head * Dv, Dv);
    float acck[4][MAXJ], accv[4][MAXJ];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < MAXJ; ++j) { acck[i][j] = 0.f; accv[i][j] = 0.f; }

    for (int m0 = tri ? n0 : 0; m0 < L; m0 += TILE) {
      const int mrows = min(TILE, L - m0);
      __syncthreads();
      load_tile<T>(Qs, ldq, reinterpret_cast<const T*>(a.q), a.q_rs, s.start + m0, mrows, head * Dq, Dq);
      load_tile<T>(dOs, ldv, reinterpret_cast<const T*>(a.d_o), a.do_rs, s.start + m0, mrows, head * Dv, Dv);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty * 4 + i;  // query row inside the tile
        const int m = m0 + r, n = n0 + tx;
        float pv = 0.f, dsv = 0.f;
        if (m < L && n < L && keep(m, n, s, a.mask)) {
          const float x = a.alpha * dot_rows(Qs + r * ldq, Ks + tx * ldq, Dq);
          const float sg = sigmoidf_exact(x);
          const float sc = row_scale(a, s.start + m);
          const float dp = dot_rows(dOs + r * ldv, Vs + tx * ldv, Dv);
          pv = x * sg * sc;
          dsv = dp * sc * sg * (1.f + x * (1.f - sg));
        }
        Pt[tx * (TILE + 1) + r] = pv;
        dSt[tx * (TILE + 1) + r] = dsv;
      }
      __syncthreads();
      for (int m = 0; m < TILE; ++m) {
        float p[4], ds[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          p[i] = Pt[(ty * 4 + i) * (TILE + 1) + m];
          ds[i] = dSt[(ty * 4 + i) * (TILE + 1) + m];
        }
#pragma unroll
        for (int j = 0; j < MAXJ; ++j) {
          const int c = tx + 32 * j;
          if (c < Dv) {
            const float x = dOs[m * ldv + c];
#pragma unroll
            for (int i = 0; i < 4; ++i) accv[i][j] = fmaf(p[i], x, accv[i][j]);
          }
          if (c < Dq) {
            const float x = Qs[m * ldq + c];
#pragma unroll
            for (int i = 0; i < 4; ++i) acck[i][j] = fmaf(ds[i], x, acck[i][j]);
          }
        }
      }
    }
    T* dkp = reinterpret_cast<T*>(a.dk);
    T* dvp = reinterpret_cast<T*>(a.dv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = n0 + ty * 4 + i;
      if (n < L) {
#pragma unroll
        for (int j = 0; j < MAXJ; ++j) {
          const int c = tx + 32 * j;
          if (c < Dq) dkp[(s.start + n) * a.dk_rs + head * Dq + c] = from_f32<T>(acck[i][j] * a.alpha);
          if (c < Dv) dvp[(s.start + n) * a.dv_rs + head * Dv + c] = from_f32<T>(accv[i][j]);
        }
      }
    }
  }
}

// Zero rows [seq_offsets[B], T) of up to three outputs (rows no sequence owns).
template <typename T>
__global__ void zero_tail_rows(KernelArgs a, T* o0, long long rs0, int w0, T* o1, long long rs1, int w1,
                               T* o2, long long rs2, int w2) {
  long long first = load_index(a.seq_offsets, a.offsets_i64, a.B);
  if (first < 0) first = 0;
  if (first > a.T) first = a.T;
  const long long rows = a.T - first;
  const int wmax = max(w0, max(w1, w2));
  const long long total = rows * wmax;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = first + i / wmax;
    const int c = static_cast<int>(i % wmax);
    if (o0 && c < w0) o0[r * rs0 + c] = from_f32<T>(0.f);
    if (o1 && c < w1) o1[r * rs1 + c] = from_f32<T>(0.f);
    if (o2 && c < w2) o2[r * rs2 + c] = from_f32<T>(0.f);
  }
}

size_t smem_q_major(const KernelArgs& a, int mode) {
  const int ldq = a.Dqk + 1, ldv = a.Dv + 1;
  size_t f = 2 * TILE * ldq + TILE * ldv + TILE * (TILE + 1);
  if (mode == 1) f += TILE * ldv;
  return f * sizeof(float);
}
size_t smem_kv_major(const KernelArgs& a) {
  const int ldq = a.Dqk + 1, ldv = a.Dv + 1;
  return (size_t)(2 * TILE * ldq + 2 * TILE * ldv + 2 * TILE * (TILE + 1)) * sizeof(float);
}

int grid_x(const KernelArgs& a, int max_seq_len) {
  // one CTA per 32-row tile of the longest sequence the caller announces; CTAs stride
  // over the remaining tiles, so sequences longer than max_seq_len are still covered
  long long est = max_seq_len > 0 ? max_seq_len : 1;
  if (est > a.T) est = a.T;
  long long gx = (est + TILE - 1) / TILE;
  if (gx < 1) gx = 1;
  if (gx > 4096) gx = 4096;
  return static_cast<int>(gx);
}

template <typename T>
cudaError_t launch_fwd_t(const KernelArgs& a, int max_seq_len, cudaStream_t st) {
  zero_tail_rows<T><<<64, 256, 0, st>>>(a, reinterpret_cast<T*>(a.o), a.o_rs, a.H * a.Dv, (T*)nullptr, 0, 0,
                                        (T*)nullptr, 0, 0);
  if (a.B <= 0 || a.T <= 0) return cudaGetLastError();
  const size_t sm = smem_q_major(a, 0);
  cudaError_t e = cudaFuncSetAttribute(simt_q_major<T, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  dim3 grid(grid_x(a, max_seq_len), a.H, a.B);
  simt_q_major<T, 0><<<grid, THREADS, sm, st>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_bwd_t(const KernelArgs& a, int max_seq_len, cudaStream_t st) {
  zero_tail_rows<T><<<64, 256, 0, st>>>(a, reinterpret_cast<T*>(a.dq), a.dq_rs, a.H * a.Dqk,
                                        reinterpret_cast<T*>(a.dk), a.dk_rs, a.H * a.Dqk,
                                        reinterpret_cast<T*>(a.dv), a.dv_rs, a.H * a.Dv);
  if (a.B <= 0 || a.T <= 0) return cudaGetLastError();
  const size_t sm1 = smem_q_major(a, 1), sm2 = smem_kv_major(a);
  cudaError_t e = cudaFuncSetAttribute(simt_q_major<T, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(simt_kv_major<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2);
  if (e != cudaSuccess) return e;
  dim3 grid(grid_x(a, max_seq_len), a.H, a.B);
  if (!a.skip_dkv) simt_kv_major<T><<<grid, THREADS, sm2, st>>>(a);
  if (!a.skip_dq) simt_q_major<T, 1><<<grid, THREADS, sm1, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t simt_forward(const KernelArgs& a, int dtype, int max_seq_len, cudaStream_t st) {
  switch (dtype) {
    case B200_HSTU_F32: return launch_fwd_t<float>(a, max_seq_len, st);
    case B200_HSTU_BF16: return launch_fwd_t<__nv_bfloat16>(a, max_seq_len, st);
    default: return launch_fwd_t<__half>(a, max_seq_len, st);
  }
}

cudaError_t simt_backward(const KernelArgs& a, int dtype, int max_seq_len, cudaStream_t st) {
  switch (dtype) {
    case B200_HSTU_F32: return launch_bwd_t<float>(a, max_seq_len, st);
    case B200_HSTU_BF16: return launch_bwd_t<__nv_bfloat16>(a, max_seq_len, st);
    default: return launch_bwd_t<__half>(a, max_seq_len, st);
  }
}

cudaError_t zero_tail(const KernelArgs& a, int dtype, bool backward, cudaStream_t st) {
  if (dtype == B200_HSTU_F32) {
    using T = float;
    if (!backward)
      zero_tail_rows<T><<<64, 256, 0, st>>>(a, (T*)a.o, a.o_rs, a.H * a.Dv, (T*)0, 0, 0, (T*)0, 0, 0);
    else
      zero_tail_rows<T><<<64, 256, 0, st>>>(a, (T*)a.dq, a.dq_rs, a.H * a.Dqk, (T*)a.dk, a.dk_rs, a.H * a.Dqk,
                                            (T*)a.dv, a.dv_rs, a.H * a.Dv);
  } else {
    using T = __half;  // bf16 and fp16 share the all-zero bit pattern
    if (!backward)
      zero_tail_rows<T><<<64, 256, 0, st>>>(a, (T*)a.o, a.o_rs, a.H * a.Dv, (T*)0, 0, 0, (T*)0, 0, 0);
    else
      zero_tail_rows<T><<<64, 256, 0, st>>>(a, (T*)a.dq, a.dq_rs, a.H * a.Dqk, (T*)a.dk, a.dk_rs, a.H * a.Dqk,
                                            (T*)a.dv, a.dv_rs, a.H * a.Dv);
  }
  return cudaGetLastError();
}

}  // namespace hstu
