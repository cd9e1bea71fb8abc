// Backward of the weighted layer norm of the STU layer (HBM-bound).
// Reference: weightedLayerNorm, recir/ops/kjt_split_per_feature.cpp:197-244, which the reference
// differentiates by autograd through the ATen composite; the closed form of that derivative is, with
// xh = (x - mean) * rstd, n = xh * w + b and y = n (or sigmoid(n) * x for is_swish):
//   dn  = dy                          (or dy * x * s * (1 - s), s = sigmoid(n))
//   dw  = sum over rows of dn * xh,   db = sum over rows of dn
//   dxh = dn * w
//   dx  = rstd * (dxh - mean_cols(dxh) - xh * mean_cols(dxh * xh))      (+ dy * s for is_swish)
// All arithmetic is float32 and every gradient is rounded once, as the composite does.
//
// The gate stage (layerNormMulQuantized, :558-600: combined = [ silu(u) or u | x | n * act(u) ], the first two
// parts optional; its fp8 copy carries no gradient) is differentiated the same way, by a second kernel of the
// same shape: with m = act(u) and d_u | d_x | d_mult the parts of the incoming gradient,
//   dn = d_mult * m,   du = d_mult * n * act'(u) (+ d_u * (silu'(u) or 1)),   dx as above from dn (+ d_x).
//
// One warp owns one row at a time (x and dy stay in registers between the two row reductions and the
// output, so each crosses HBM once) and walks rows with a grid stride, adding its rows' dn * xh and dn into
// per-lane column accumulators.  At the end the eight warps of a CTA add theirs up in shared memory and
// the CTA writes ONE partial row per gradient to the caller's workspace; a second small kernel adds the
// partial rows in a fixed order.  No atomics: the column sums are deterministic.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_hstu.h"
#include "../../include/b200_stu_rowwise.h"
#include "hstu_launch.h"
#include "stu_vec.cuh"

namespace hstu {
namespace rowwise_bwd {
namespace {

using namespace vec;
constexpr int WARPS = 8;
constexpr int MAX_COLS = 1024;

struct Args {
  const void* dy; const void* x; const void* weight; const void* bias;
  const float* mean; const float* rstd;
  void* dx; void* dw; void* db; float* partial;
  long long rows, dy_rs, x_rs, dx_rs;
  int cols, swish, affine, grid;
  // gate stage only: dy is the d_mult part of the incoming gradient; dy_u / dy_x its optional other parts
  const void* u; const void* dy_u; const void* dy_x; void* du;
  long long u_rs, du_rs;
  int act, silu_u;  // act: 0 none, 1 silu, 2 sigmoid
};

template <typename T, int VPL>
__global__ void __launch_bounds__(WARPS * 32) layer_norm_bwd_kernel(Args a) {
  __shared__ float red[WARPS][MAX_COLS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nv = a.cols >> 3;
  const float inv_cols = 1.f / static_cast<float>(a.cols);
  float dwacc[VPL][8], dbacc[VPL][8];
#pragma unroll
  for (int j = 0; j < VPL; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) { dwacc[j][i] = 0.f; dbacc[j][i] = 0.f; }
  const long long stride = static_cast<long long>(gridDim.x) * WARPS;
  for (long long row = static_cast<long long>(blockIdx.x) * WARPS + warp; row < a.rows; row += stride) {
    const T* xr = reinterpret_cast<const T*>(a.x) + row * a.x_rs;
    const T* gr = reinterpret_cast<const T*>(a.dy) + row * a.dy_rs;
    float xv[VPL][8], gv[VPL][8];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nv) {
        load8<T>(xr + 8 * v, xv[j]);
        load8<T>(gr + 8 * v, gv[j]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) { xv[j][i] = 0.f; gv[j][i] = 0.f; }
      }
    }
    const float mean = a.mean[row], rstd = a.rstd[row];
    float s1 = 0.f, s2 = 0.f;
    // after this loop: xv = xh, gv = dxh; the gated form's direct term dy * s is kept in `direct`
    float direct[VPL][8];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      float w[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) { w[i] = 1.f; b[i] = 0.f; }
      if (a.affine && v < nv) {
        load8<T>(reinterpret_cast<const T*>(a.weight) + 8 * v, w);
        load8<T>(reinterpret_cast<const T*>(a.bias) + 8 * v, b);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float x = xv[j][i], xh = (x - mean) * rstd;
        float dn = gv[j][i];
        direct[j][i] = 0.f;
        if (a.swish) {
          const float s = sigmoid_t<T>(xh * w[i] + b[i]);
          direct[j][i] = dn * s;
          dn = dn * x * s * (1.f - s);
        }
        if (v < nv) {
          dwacc[j][i] += dn * xh;
          dbacc[j][i] += dn;
        }
        const float dxh = v < nv ? dn * w[i] : 0.f;
        s1 += dxh;
        s2 += dxh * xh;
        xv[j][i] = xh;
        gv[j][i] = dxh;
      }
    }
    const float c1 = warp_sum(s1) * inv_cols, c2 = warp_sum(s2) * inv_cols;
    T* dxr = reinterpret_cast<T*>(a.dx) + row * a.dx_rs;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v >= nv) continue;
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = rstd * (gv[j][i] - c1 - xv[j][i] * c2) + direct[j][i];
      store8<T>(dxr + 8 * v, o);
    }
  }
  if (!a.affine) return;
  // column sums of this CTA: dw first, then db, through the same shared buffer
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nv) {
#pragma unroll
        for (int i = 0; i < 8; ++i) red[warp][8 * v + i] = pass == 0 ? dwacc[j][i] : dbacc[j][i];
      }
    }
    __syncthreads();
    for (int c = threadIdx.x; c < a.cols; c += WARPS * 32) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) s += red[w][c];
      a.partial[(static_cast<long long>(blockIdx.x) * 2 + pass) * a.cols + c] = s;
    }
    __syncthreads();
  }
}

// Gate stage: out = [ (silu(u) or u) | x | layer_norm(x) * act(u) ].  Same structure as the kernel above; x, u
// and the incoming gradient cross HBM once, dx and du are written once.
template <typename T, int VPL>
__global__ void __launch_bounds__(WARPS * 32) layer_norm_mul_bwd_kernel(Args a) {
  __shared__ float red[WARPS][MAX_COLS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nv = a.cols >> 3;
  const float inv_cols = 1.f / static_cast<float>(a.cols);
  float dwacc[VPL][8], dbacc[VPL][8];
#pragma unroll
  for (int j = 0; j < VPL; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) { dwacc[j][i] = 0.f; dbacc[j][i] = 0.f; }
  const long long stride = static_cast<long long>(gridDim.x) * WARPS;
  for (long long row = static_cast<long long>(blockIdx.x) * WARPS + warp; row < a.rows; row += stride) {
    const T* xr = reinterpret_cast<const T*>(a.x) + row * a.x_rs;
    const T* ur = reinterpret_cast<const T*>(a.u) + row * a.u_rs;
    const T* gr = reinterpret_cast<const T*>(a.dy) + row * a.dy_rs;
    const T* gur = a.dy_u ? reinterpret_cast<const T*>(a.dy_u) + row * a.dy_rs : nullptr;
    const T* gxr = a.dy_x ? reinterpret_cast<const T*>(a.dy_x) + row * a.dy_rs : nullptr;
    T* dur = reinterpret_cast<T*>(a.du) + row * a.du_rs;
    const float mean = a.mean[row], rstd = a.rstd[row];
    float s1 = 0.f, s2 = 0.f;
    float xh[VPL][8], dxh[VPL][8];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
#pragma unroll
      for (int i = 0; i < 8; ++i) { xh[j][i] = 0.f; dxh[j][i] = 0.f; }
      if (v >= nv) continue;
      float x[8], u[8], g[8], gu[8], w[8], b[8], du[8];
      load8<T>(xr + 8 * v, x);
      load8<T>(ur + 8 * v, u);
      load8<T>(gr + 8 * v, g);
      load8<T>(reinterpret_cast<const T*>(a.weight) + 8 * v, w);
      load8<T>(reinterpret_cast<const T*>(a.bias) + 8 * v, b);
      if (gur) {
        load8<T>(gur + 8 * v, gu);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) gu[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float h = (x[i] - mean) * rstd, n = h * w[i] + b[i];
        const float s = sigmoid_t<T>(u[i]);
        const float silu_grad = s * (1.f + u[i] * (1.f - s));
        float m = u[i], dm = 1.f;
        if (a.act == 1) { m = u[i] * s; dm = silu_grad; }
        else if (a.act == 2) { m = s; dm = s * (1.f - s); }
        const float dn = g[i] * m;
        du[i] = g[i] * n * dm + gu[i] * (a.silu_u ? silu_grad : 1.f);
        dwacc[j][i] += dn * h;
        dbacc[j][i] += dn;
        const float d = dn * w[i];
        s1 += d;
        s2 += d * h;
        xh[j][i] = h;
        dxh[j][i] = d;
      }
      store8<T>(dur + 8 * v, du);
    }
    const float c1 = warp_sum(s1) * inv_cols, c2 = warp_sum(s2) * inv_cols;
    T* dxr = reinterpret_cast<T*>(a.dx) + row * a.dx_rs;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v >= nv) continue;
      float o[8], gx[8];
      if (gxr) {
        load8<T>(gxr + 8 * v, gx);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) gx[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = rstd * (dxh[j][i] - c1 - xh[j][i] * c2) + gx[i];
      store8<T>(dxr + 8 * v, o);
    }
  }
  // column sums of this CTA: dw first, then db, through the same shared buffer
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < nv) {
#pragma unroll
        for (int i = 0; i < 8; ++i) red[warp][8 * v + i] = pass == 0 ? dwacc[j][i] : dbacc[j][i];
      }
    }
    __syncthreads();
    for (int c = threadIdx.x; c < a.cols; c += WARPS * 32) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) s += red[w][c];
      a.partial[(static_cast<long long>(blockIdx.x) * 2 + pass) * a.cols + c] = s;
    }
    __syncthreads();
  }
}

// dw[c] = sum over CTAs of partial[cta][0][c] (db: [1]).  A CTA owns 32 columns; its eight warps add up
// every eighth partial row each (four independent running sums per thread, so that the loads overlap), then
// the eight per-warp sums are added in warp order: a fixed order, hence bitwise repeatable.
template <typename T>
__global__ void __launch_bounds__(256) layer_norm_bwd_reduce(Args a) {
  __shared__ float red[2][8][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float sw[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
  if (c < a.cols) {
    int g = warp;
    for (; g + 24 < a.grid; g += 32) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        sw[u] += a.partial[(static_cast<long long>(g + 8 * u) * 2 + 0) * a.cols + c];
        sb[u] += a.partial[(static_cast<long long>(g + 8 * u) * 2 + 1) * a.cols + c];
      }
    }
    for (; g < a.grid; g += 8) {
      sw[0] += a.partial[(static_cast<long long>(g) * 2 + 0) * a.cols + c];
      sb[0] += a.partial[(static_cast<long long>(g) * 2 + 1) * a.cols + c];
    }
  }
  red[0][warp][lane] = (sw[0] + sw[1]) + (sw[2] + sw[3]);
  red[1][warp][lane] = (sb[0] + sb[1]) + (sb[2] + sb[3]);
  __syncthreads();
  if (warp == 0 && c < a.cols) {
    float tw = 0.f, tb = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) { tw += red[0][w][lane]; tb += red[1][w][lane]; }
    reinterpret_cast<T*>(a.dw)[c] = from_float<T>(tw);
    reinterpret_cast<T*>(a.db)[c] = from_float<T>(tb);
  }
}

int grid_for(long long rows) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (rows + WARPS - 1) / WARPS, cap = static_cast<long long>(sms) * 4;
  return static_cast<int>(want < cap ? (want < 1 ? 1 : want) : cap);
}

template <typename T>
cudaError_t launch_t(const Args& a, cudaStream_t st) {
  const int vpl = (a.cols / 8 + 31) / 32;
  if (vpl <= 1) layer_norm_bwd_kernel<T, 1><<<a.grid, WARPS * 32, 0, st>>>(a);
  else if (vpl <= 2) layer_norm_bwd_kernel<T, 2><<<a.grid, WARPS * 32, 0, st>>>(a);
  else layer_norm_bwd_kernel<T, 4><<<a.grid, WARPS * 32, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !a.affine) return e;
  layer_norm_bwd_reduce<T><<<(a.cols + 31) / 32, 256, 0, st>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_mul_t(const Args& a, cudaStream_t st) {
  const int vpl = (a.cols / 8 + 31) / 32;
  if (vpl <= 1) layer_norm_mul_bwd_kernel<T, 1><<<a.grid, WARPS * 32, 0, st>>>(a);
  else if (vpl <= 2) layer_norm_mul_bwd_kernel<T, 2><<<a.grid, WARPS * 32, 0, st>>>(a);
  else layer_norm_mul_bwd_kernel<T, 4><<<a.grid, WARPS * 32, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  layer_norm_bwd_reduce<T><<<(a.cols + 31) / 32, 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace
}  // namespace rowwise_bwd
}  // namespace hstu

extern "C" {

size_t b200_stu_layer_norm_bwd_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return static_cast<size_t>(hstu::rowwise_bwd::grid_for(rows)) * 2 * static_cast<size_t>(cols) * sizeof(float);
}

int b200_stu_layer_norm_bwd(const B200LayerNormBwdParams* p, void* stream) {
  using namespace hstu::rowwise_bwd;
  if (p == nullptr) return B200_HSTU_EINVAL;
  if (p->struct_size != sizeof(B200LayerNormBwdParams)) return B200_HSTU_EVERSION;
  if (p->dtype != B200_HSTU_F32 && p->dtype != B200_HSTU_BF16 && p->dtype != B200_HSTU_F16) return B200_HSTU_EUNSUPPORTED;
  if (p->rows < 0 || p->cols <= 0) return B200_HSTU_EINVAL;
  if (p->cols % 8 != 0 || p->cols > MAX_COLS) return B200_HSTU_EUNSUPPORTED;
  const bool affine = p->weight != nullptr;
  if ((p->weight == nullptr) != (p->bias == nullptr)) return B200_HSTU_EINVAL;
  if ((p->flags & B200_ROWWISE_FLAG_SWISH) && !affine) return B200_HSTU_EINVAL;
  if (affine && (!p->dweight || !p->dbias)) return B200_HSTU_EINVAL;
  if (p->rows == 0) {
    if (affine) {  // empty sums
      const size_t bytes = static_cast<size_t>(p->cols) * (p->dtype == B200_HSTU_F32 ? 4 : 2);
      cudaMemsetAsync(p->dweight, 0, bytes, static_cast<cudaStream_t>(stream));
      cudaMemsetAsync(p->dbias, 0, bytes, static_cast<cudaStream_t>(stream));
    }
    return B200_HSTU_OK;
  }
  if (!p->dy || !p->x || !p->mean || !p->rstd || !p->dx) return B200_HSTU_EINVAL;
  if (p->dy_row_stride < p->cols || p->x_row_stride < p->cols || p->dx_row_stride < p->cols) return B200_HSTU_EINVAL;
  auto bad = [](const void* q, long long stride) { return reinterpret_cast<uintptr_t>(q) % 16 != 0 || stride % 8 != 0; };
  if (bad(p->dy, p->dy_row_stride) || bad(p->x, p->x_row_stride) || bad(p->dx, p->dx_row_stride) ||
      (affine && (bad(p->weight, 0) || bad(p->bias, 0))))
    return B200_HSTU_EALIGN;
  Args a;
  a.dy = p->dy; a.x = p->x; a.weight = p->weight; a.bias = p->bias; a.mean = p->mean; a.rstd = p->rstd;
  a.dx = p->dx; a.dw = p->dweight; a.db = p->dbias; a.partial = p->workspace;
  a.rows = p->rows; a.dy_rs = p->dy_row_stride; a.x_rs = p->x_row_stride; a.dx_rs = p->dx_row_stride;
  a.cols = static_cast<int>(p->cols); a.swish = (p->flags & B200_ROWWISE_FLAG_SWISH) ? 1 : 0; a.affine = affine ? 1 : 0;
  a.grid = grid_for(p->rows);
  a.u = a.dy_u = a.dy_x = nullptr; a.du = nullptr; a.u_rs = a.du_rs = 0; a.act = a.silu_u = 0;
  if (affine) {
    const size_t need = b200_stu_layer_norm_bwd_workspace_bytes(p->rows, p->cols);
    if (p->workspace == nullptr || p->workspace_bytes < need || reinterpret_cast<uintptr_t>(p->workspace) % 16 != 0)
      return B200_HSTU_EWORKSPACE;
  }
  hstu::set_error_stage("layer norm backward kernels");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = p->dtype == B200_HSTU_F32    ? launch_t<float>(a, st)
                        : p->dtype == B200_HSTU_BF16 ? launch_t<__nv_bfloat16>(a, st)
                                                     : launch_t<__half>(a, st);
  return e == cudaSuccess ? B200_HSTU_OK : B200_HSTU_ELAUNCH;
}

int b200_stu_layer_norm_mul_bwd(const B200LayerNormMulBwdParams* p, void* stream) {
  using namespace hstu::rowwise_bwd;
  if (p == nullptr) return B200_HSTU_EINVAL;
  if (p->struct_size != sizeof(B200LayerNormMulBwdParams)) return B200_HSTU_EVERSION;
  if (p->dtype != B200_HSTU_F32 && p->dtype != B200_HSTU_BF16 && p->dtype != B200_HSTU_F16) return B200_HSTU_EUNSUPPORTED;
  if (p->rows < 0 || p->cols <= 0) return B200_HSTU_EINVAL;
  if (p->cols % 8 != 0 || p->cols > MAX_COLS) return B200_HSTU_EUNSUPPORTED;
  if (!p->weight || !p->bias || !p->dweight || !p->dbias) return B200_HSTU_EINVAL;
  if ((p->flags & B200_ROWWISE_FLAG_ACT_SILU) && (p->flags & B200_ROWWISE_FLAG_ACT_SIGMOID)) return B200_HSTU_EINVAL;
  const size_t esize = p->dtype == B200_HSTU_F32 ? 4 : 2;
  if (p->rows == 0) {  // empty sums
    cudaMemsetAsync(p->dweight, 0, static_cast<size_t>(p->cols) * esize, static_cast<cudaStream_t>(stream));
    cudaMemsetAsync(p->dbias, 0, static_cast<size_t>(p->cols) * esize, static_cast<cudaStream_t>(stream));
    return B200_HSTU_OK;
  }
  if (!p->dout || !p->x || !p->u || !p->mean || !p->rstd || !p->dx || !p->du) return B200_HSTU_EINVAL;
  const int parts = 1 + ((p->flags & B200_ROWWISE_FLAG_CONCAT_U) ? 1 : 0) + ((p->flags & B200_ROWWISE_FLAG_CONCAT_X) ? 1 : 0);
  if (p->dout_row_stride < parts * p->cols || p->x_row_stride < p->cols || p->u_row_stride < p->cols ||
      p->dx_row_stride < p->cols || p->du_row_stride < p->cols)
    return B200_HSTU_EINVAL;
  auto bad = [](const void* q, long long stride) { return reinterpret_cast<uintptr_t>(q) % 16 != 0 || stride % 8 != 0; };
  if (bad(p->dout, p->dout_row_stride) || bad(p->x, p->x_row_stride) || bad(p->u, p->u_row_stride) ||
      bad(p->dx, p->dx_row_stride) || bad(p->du, p->du_row_stride) || bad(p->weight, 0) || bad(p->bias, 0))
    return B200_HSTU_EALIGN;
  const size_t need = b200_stu_layer_norm_bwd_workspace_bytes(p->rows, p->cols);
  if (p->workspace == nullptr || p->workspace_bytes < need || reinterpret_cast<uintptr_t>(p->workspace) % 16 != 0)
    return B200_HSTU_EWORKSPACE;
  Args a;
  a.x = p->x; a.weight = p->weight; a.bias = p->bias; a.mean = p->mean; a.rstd = p->rstd;
  a.dx = p->dx; a.dw = p->dweight; a.db = p->dbias; a.partial = p->workspace;
  a.rows = p->rows; a.dy_rs = p->dout_row_stride; a.x_rs = p->x_row_stride; a.dx_rs = p->dx_row_stride;
  a.cols = static_cast<int>(p->cols); a.swish = 0; a.affine = 1;
  a.grid = grid_for(p->rows);
  // the parts of an incoming-gradient row, in the order the forward concatenates them
  const char* part = static_cast<const char*>(p->dout);
  a.dy_u = a.dy_x = nullptr;
  if (p->flags & B200_ROWWISE_FLAG_CONCAT_U) { a.dy_u = part; part += static_cast<size_t>(p->cols) * esize; }
  if (p->flags & B200_ROWWISE_FLAG_CONCAT_X) { a.dy_x = part; part += static_cast<size_t>(p->cols) * esize; }
  a.dy = part;
  a.u = p->u; a.du = p->du; a.u_rs = p->u_row_stride; a.du_rs = p->du_row_stride;
  a.act = (p->flags & B200_ROWWISE_FLAG_ACT_SILU) ? 1 : ((p->flags & B200_ROWWISE_FLAG_ACT_SIGMOID) ? 2 : 0);
  a.silu_u = (p->flags & B200_ROWWISE_FLAG_SILU_U) ? 1 : 0;
  hstu::set_error_stage("gate stage backward kernels");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = p->dtype == B200_HSTU_F32    ? launch_mul_t<float>(a, st)
                        : p->dtype == B200_HSTU_BF16 ? launch_mul_t<__nv_bfloat16>(a, st)
                                                     : launch_mul_t<__half>(a, st);
  return e == cudaSuccess ? B200_HSTU_OK : B200_HSTU_ELAUNCH;
}

}  // extern "C"
