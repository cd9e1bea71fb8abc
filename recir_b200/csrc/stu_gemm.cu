// Projections of the STU layer on the tensor cores (sm_100a): out = bias + A W, where A is either x
// itself or the weighted layer norm of x, computed inside the kernel as the prologue of the A operand.
//
// Reference semantics: tritonAddMm (recir/ops/kjt_split_per_feature.cpp:246-262: at::addmm(bias, x, w))
// and weightedLayerNorm (:197-244) in front of it, i.e. the "layer norm -> u/v/q/k projection" pair of an
// STU layer.  The reference materialises the normalised rows in the input dtype before the product; so
// does this kernel (they are rounded to the 16-bit A operand), the sums run in fp32 and the result is
// rounded once after the bias has been added.  Fusing the two saves one write and one read of the
// activations (2 * rows * K * 2 bytes) and one launch.
//
// Tiling.  A CTA owns a block of 128 rows and keeps its whole A operand (K <= 512: eight 64-column boxes,
// 128 KB, 128-byte swizzle) in shared memory; W streams through a 4-stage ring of [32 k-rows x 256
// n-columns] tiles (TMA, four 64-column boxes, used as the N-major B operand).  One tcgen05.mma
// M128 N256 K16 per k-step accumulates into one of two 256-column TMEM accumulators, so the epilogue of
// an output tile (bias, rounding, staged bulk tensor stores) overlaps the MMAs of the next one.  W (K x N x 2 bytes, at most
// a few MB) stays in L2; per 128 rows a CTA ingests it once, which is what bounds the kernel (shared
// memory ingest per SM), not the tensor pipe.
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = MMA issuer (one elected lane), warps 2-9 =
// layer-norm prologue (16 rows per warp, four at a time in registers) and epilogue (TMEM lane quadrant
// warp % 4, column half (warp - 2) / 4).  Every wait is bounded (see sm100_ptx.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <type_traits>

#include "../../include/b200_hstu.h"
#include "../../include/b200_stu_gemm.h"
#include "hstu_launch.h"
#include "hstu_tc_host.h"
#include "sm100_ptx.cuh"
#include "stu_vec.cuh"

namespace hstu {
namespace gemm {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 32;   // BK: k-rows of W per pipeline stage (two k-steps of 16)
constexpr int MAX_K = 512;
constexpr int B_STAGES = 4;
constexpr int A_BOX_BYTES = BM * 128;        // 128 rows x 64 k-columns of 16-bit elements
constexpr int B_BOX_BYTES = BK * 128;        // 32 k-rows x 64 n-columns
constexpr int B_STAGE_BYTES = 4 * B_BOX_BYTES;
constexpr int OUT_BOX_BYTES = BM * 128;      // staging of 128 rows x 64 output columns, one per epilogue group
constexpr int THREADS = 320;  // 10 warps: 200 registers each without any reallocation
constexpr int TMEM_COLS = 512;
enum { WAIT_GEMM_PRODUCER = 111, WAIT_GEMM_MMA = 112, WAIT_GEMM_EPILOGUE = 113 };

struct Shared {
  unsigned char a[MAX_K / 64][A_BOX_BYTES];
  unsigned char b[B_STAGES][B_STAGE_BYTES];
  unsigned char out[2][OUT_BOX_BYTES];
  unsigned long long a_full, a_empty;
  unsigned long long b_full[B_STAGES], b_empty[B_STAGES];
  unsigned long long acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct Maps {
  CUtensorMap x;  // [M, K], box 64 columns x 128 rows (unused with the layer-norm prologue)
  CUtensorMap w;  // [K, N], box 64 columns x 32 rows
  CUtensorMap o;  // [M, N], box 64 columns x 128 rows (bulk stores; rows past M and columns past N are clipped)
};

struct Args {
  const void* x; const void* ln_w; const void* ln_b; const void* bias; void* out;
  float* mean; float* rstd; int* status;
  long long M, x_rs, out_rs, bias_rs;
  int K, N, fuse_ln, swish, affine;
  float eps;
  int dbg;  // instrumented builds only (B200_GEMM_DBG): 1 no W loads / waits, 2 no output staging, 4 no MMAs, 8 N=128 MMAs
};

using vec::load8;
using vec::warp_sum;
template <bool BF16> __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}
template <bool BF16>
__global__ void __launch_bounds__(THREADS, 1) stu_addmm_tc(const __grid_constant__ Maps maps, Args a) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ unsigned char smem_raw[];
  Shared& sh = *reinterpret_cast<Shared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &sh.abort_flag;
  const int kboxes = a.K / 64;   // 64-column boxes of the A operand
  const int kstages = a.K / BK;  // pipeline stages of W per output tile
  const int n_tiles = (a.N + BN - 1) / BN;
  const long long n_blocks = (a.M + BM - 1) / BM;

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    mbar_init(smem_u32(&sh.a_full), a.fuse_ln ? 256 : 1);
    mbar_init(smem_u32(&sh.a_empty), 1);
    for (int i = 0; i < B_STAGES; ++i) { mbar_init(smem_u32(&sh.b_full[i]), 1); mbar_init(smem_u32(&sh.b_empty[i]), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(smem_u32(&sh.acc_full[i]), 1); mbar_init(smem_u32(&sh.acc_empty[i]), 256); }
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&sh.tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) { prefetch_tensormap(&maps.w); if (!a.fuse_ln) prefetch_tensormap(&maps.x); }
    uint32_t it = 0, st = 0, ph = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_GEMM_PRODUCER));
    };
    for (long long blk = blockIdx.x; blk < n_blocks && ok; blk += gridDim.x, ++it) {
      if (!a.fuse_ln) {
        ok = wait_all(&sh.a_empty, (it & 1) ^ 1);
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(smem_u32(&sh.a_full), static_cast<uint32_t>(kboxes) * A_BOX_BYTES);
          for (int kb = 0; kb < kboxes; ++kb)
            tma_load_2d(smem_u32(sh.a[kb]), &maps.x, smem_u32(&sh.a_full), kb * 64, static_cast<int>(blk * BM));
        }
        __syncwarp();
      }
      for (int nt = 0; nt < n_tiles && ok; ++nt) {
        for (int kb = 0; kb < kstages; ++kb) {
#ifdef B200_HSTU_PROFILING
          if (a.dbg & 1) continue;
#endif
          ok = wait_all(&sh.b_empty[st], ph ^ 1);
          if (!ok) break;
          if (elect_one()) {
            mbar_arrive_expect_tx(smem_u32(&sh.b_full[st]), B_STAGE_BYTES);
#pragma unroll
            for (int j = 0; j < 4; ++j)  // columns past N are filled with zeros
              tma_load_2d(smem_u32(sh.b[st]) + j * B_BOX_BYTES, &maps.w, smem_u32(&sh.b_full[st]), nt * BN + j * 64, kb * BK);
          }
          __syncwarp();
          if (++st == B_STAGES) { st = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC = idesc_f16(BF16 ? 1 : 0, BM, BN, 0, 1);  // A K-major (shared memory), B N-major
    constexpr uint32_t HI = desc_hi_sw128(1024);
    const uint32_t a_lo0 = desc_lo_sw128(smem_u32(sh.a[0]), 16);
    const uint32_t b_lo0 = desc_lo_sw128(smem_u32(sh.b[0]), B_BOX_BYTES);  // 64-column groups are one box apart
    uint32_t it = 0, st = 0, ph = 0, g = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_GEMM_MMA));
    };
    for (long long blk = blockIdx.x; blk < n_blocks && ok; blk += gridDim.x, ++it) {
      ok = wait_all(&sh.a_full, it & 1);
      if (!ok) break;
      tc_fence_after();
      for (int nt = 0; nt < n_tiles && ok; ++nt, ++g) {
        const uint32_t buf = g & 1;
        ok = wait_all(&sh.acc_empty[buf], ((g >> 1) & 1) ^ 1);
        if (!ok) break;
        tc_fence_after();
        for (int kb = 0; kb < kstages; ++kb) {
#ifdef B200_HSTU_PROFILING
          if (a.dbg & 1) {
            if (elect_one() && !(a.dbg & 4)) {
              for (int kk = 0; kk < BK / 16; ++kk)
                mma_ss(tmem + buf * BN, desc_join(a_lo0 + (kb >> 1) * (A_BOX_BYTES >> 4) + (((kb & 1) << 1) + kk) * 2, HI),
                       desc_join(b_lo0 + (kb & 3) * (B_STAGE_BYTES >> 4) + kk * (2048 >> 4), HI), IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            __syncwarp();
            continue;
          }
#endif
          ok = wait_all(&sh.b_full[st], ph);
          if (!ok) break;
          tc_fence_after();
#ifdef B200_HSTU_PROFILING
          if (a.dbg & (4 | 8)) {
            if (elect_one()) {
              if (a.dbg & 8) {
                constexpr uint32_t IDESC_H = idesc_f16(BF16 ? 1 : 0, BM, 128, 0, 1);
                for (int kk = 0; kk < BK / 16; ++kk)
                  for (int hh = 0; hh < 2; ++hh)
                    mma_ss(tmem + buf * BN + hh * 128,
                           desc_join(a_lo0 + (kb >> 1) * (A_BOX_BYTES >> 4) + (((kb & 1) << 1) + kk) * 2, HI),
                           desc_join(b_lo0 + st * (B_STAGE_BYTES >> 4) + hh * (2 * B_BOX_BYTES >> 4) + kk * (2048 >> 4), HI),
                           IDESC_H, (kb > 0 || kk > 0) ? 1u : 0u);
              }
              tc_commit(smem_u32(&sh.b_empty[st]));
            }
            __syncwarp();
            if (++st == B_STAGES) { st = 0; ph ^= 1; }
            continue;
          }
#endif
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              // A: box kb / 2, k-step ((kb % 2) * 2 + kk) of its four (32 bytes each); B: k-step kk of the stage
              mma_ss(tmem + buf * BN, desc_join(a_lo0 + (kb >> 1) * (A_BOX_BYTES >> 4) + (((kb & 1) << 1) + kk) * 2, HI),
                     desc_join(b_lo0 + st * (B_STAGE_BYTES >> 4) + kk * (2048 >> 4), HI), IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
            tc_commit(smem_u32(&sh.b_empty[st]));
          }
          __syncwarp();
          if (++st == B_STAGES) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        if (elect_one()) tc_commit(smem_u32(&sh.acc_full[buf]));
        __syncwarp();
      }
      if (!ok) break;
      if (elect_one()) tc_commit(smem_u32(&sh.a_empty));  // every MMA that reads this block's A has been issued
      __syncwarp();
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ prologue + epilogue warps (2..9)
    const int ew = warp - 2;                  // 0..7
    const int wg = ew >> 2;                   // column half of the output tile
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const int row_in_blk = ((warp & 3) << 5) | lane;
    const int nv = a.K >> 3;  // 16-byte vectors per row (at most 64: two per lane)
    uint32_t it = 0, g = 0;
    bool ok = true;
    // layer-norm weight and bias of this lane's columns, packed (16 registers) for the whole kernel: loaded per
    // use they would come from L2 each time (no L1 to speak of beside 224 KB of shared memory)
    uint4 lnw[2], lnb[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int v = lane + 32 * j;
      lnw[j] = lnb[j] = make_uint4(0u, 0u, 0u, 0u);
      if (a.fuse_ln && a.affine && v < nv) {
        lnw[j] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.ln_w) + 8 * v));
        lnb[j] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.ln_b) + 8 * v));
      }
    }
    for (long long blk = blockIdx.x; blk < n_blocks && ok; blk += gridDim.x, ++it) {
      if (a.fuse_ln) {
        // ---- layer norm of 16 rows per warp, four rows at a time, into the swizzled A operand
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.a_empty), (it & 1) ^ 1, abort_flag, a.status, WAIT_GEMM_EPILOGUE));
        if (!ok) break;
        for (int r0 = 0; r0 < 16; r0 += 4) {
          float xv[4][2][8];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const long long row = blk * BM + ew * 16 + r0 + r;
            const T* xr = reinterpret_cast<const T*>(a.x) + (row < a.M ? row : a.M - 1) * a.x_rs;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int v = lane + 32 * j;
              if (v < nv) {
                load8<T>(xr + 8 * v, xv[r][j]);
              } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) xv[r][j][i] = 0.f;
              }
            }
          }
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int rb = ew * 16 + r0 + r;  // row inside the block
            const long long row = blk * BM + rb;
            // mean first, then the mean of squared deviations (kjt_split_per_feature.cpp:223-226)
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < 2; ++j)
              if (lane + 32 * j < nv) {
#pragma unroll
                for (int i = 0; i < 8; ++i) s += xv[r][j][i];
              }
            const float mean = warp_sum(s) / static_cast<float>(a.K);
            float q = 0.f;
#pragma unroll
            for (int j = 0; j < 2; ++j)
              if (lane + 32 * j < nv) {
#pragma unroll
                for (int i = 0; i < 8; ++i) { const float d = xv[r][j][i] - mean; q += d * d; }
              }
            const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(a.K) + a.eps);
            if (lane == 0 && row < a.M) { a.mean[row] = mean; a.rstd[row] = rstd; }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int v = lane + 32 * j;
              if (v >= nv) continue;
              uint4 pk = make_uint4(0u, 0u, 0u, 0u);  // rows past M enter the product as zeros
              if (row < a.M) {
                float n[8], wv[8], bv[8];
                vec::unpack8<T>(lnw[j], wv);
                vec::unpack8<T>(lnb[j], bv);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  float y = (xv[r][j][i] - mean) * rstd;
                  if (a.affine) y = y * wv[i] + bv[i];
                  if (a.swish) y = __fdividef(1.f, 1.f + __expf(-y)) * xv[r][j][i];
                  n[i] = y;
                }
                pk.x = pack2<BF16>(n[0], n[1]); pk.y = pack2<BF16>(n[2], n[3]);
                pk.z = pack2<BF16>(n[4], n[5]); pk.w = pack2<BF16>(n[6], n[7]);
              }
              // vector v = 8 columns: box v / 8, 16-byte chunk v % 8 of the 128-byte box row, swizzled
              unsigned char* dst = sh.a[v >> 3] + rb * 128 + (((v & 7) ^ (rb & 7)) << 4);
              *reinterpret_cast<uint4*>(dst) = pk;
            }
          }
        }
        fence_proxy_async();
        mbar_arrive(smem_u32(&sh.a_full));
      }
      if (a.fuse_ln) {
        // pull the rows of this CTA's NEXT block towards L2 while the tensor cores work on this one, so that
        // the next prologue's loads (four dependent batches of four rows per warp) pay L2 instead of HBM latency
        const long long nblk = blk + gridDim.x;
        if (nblk < n_blocks) {
          const int tid = threadIdx.x - 64;  // 0..255: two threads per row, alternating 128-byte lines
          const long long prow = nblk * BM + (tid >> 1);
          if (prow < a.M) {
            const char* base = reinterpret_cast<const char*>(a.x) + prow * a.x_rs * static_cast<long long>(sizeof(T));
            for (int off = (tid & 1) * 128; off < a.K * static_cast<int>(sizeof(T)); off += 256)
              asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
          }
        }
      }
      // ---- epilogue of every output tile of the block: bias, rounding, staged bulk stores.
      // Group wg owns output columns [128 wg, 128 wg + 128) of the tile and sends them out as two boxes of
      // 64 columns through its own staging buffer (128-byte-swizzled rows, as the bulk tensor store expects);
      // a thread-per-row store straight to global memory would be 32 separate 16-byte transactions per
      // instruction, which costs more than the MMAs of the tile.
      const long long row = blk * BM + row_in_blk;
      const long long brow_idx = row < a.M ? row : a.M - 1;
      unsigned char* stage = sh.out[wg];
      for (int nt = 0; nt < n_tiles && ok; ++nt, ++g) {
        const uint32_t buf = g & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.acc_full[buf]), (g >> 1) & 1, abort_flag, a.status, WAIT_GEMM_EPILOGUE));
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + lane_addr + buf * BN + wg * 128;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col0 = nt * BN + wg * 128 + h * 64;
          // The bias of this box first (eight 16-byte loads in flight together, raw): with nearly all of the
          // SM's L1 carved out as shared memory they come from L2, and one dependent load per use costs more
          // than the rest of the box.
          uint4 braw[8];
          {
            const T* brow = reinterpret_cast<const T*>(a.bias) + brow_idx * a.bias_rs + col0;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              braw[j] = (col0 + 8 * j < a.N) ? __ldg(reinterpret_cast<const uint4*>(brow + 8 * j)) : make_uint4(0u, 0u, 0u, 0u);
          }
          uint32_t v0[32], v1[32];
          tmem_ld32(acc + h * 64, v0);
          tmem_ld32(acc + h * 64 + 32, v1);
          tmem_wait_ld(v0);
          tmem_wait_ld(v1);
          if (h == 1) {
            tc_fence_before();
            mbar_arrive(smem_u32(&sh.acc_empty[buf]));  // the accumulator is in registers: the MMAs may reuse it
          }
          if (col0 >= a.N) continue;  // uniform for the group
#ifdef B200_HSTU_PROFILING
          if (a.dbg & 2) continue;
#endif
#ifdef B200_HSTU_PROFILING
          long long tq0 = 0, tq1 = 0, tq2 = 0, tq3 = 0, tq4 = 0;
          const bool tr = (a.dbg & 32) && blockIdx.x == 0 && threadIdx.x == 64 && g < 12;
          if (tr) tq0 = clock64();
#endif
          if (row_in_blk == 0) bulk_wait_read_all();  // the group's previous box has left the staging buffer
          asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");
#ifdef B200_HSTU_PROFILING
          if (tr) tq1 = clock64();
#endif
          unsigned char* my_row = stage + row_in_blk * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* v = j < 4 ? v0 : v1;
            const int jj = j & 3;
            float bf[8];
            vec::unpack8<T>(braw[j], bf);
            uint4 o;
            o.x = pack2<BF16>(__uint_as_float(v[8 * jj + 0]) + bf[0], __uint_as_float(v[8 * jj + 1]) + bf[1]);
            o.y = pack2<BF16>(__uint_as_float(v[8 * jj + 2]) + bf[2], __uint_as_float(v[8 * jj + 3]) + bf[3]);
            o.z = pack2<BF16>(__uint_as_float(v[8 * jj + 4]) + bf[4], __uint_as_float(v[8 * jj + 5]) + bf[5]);
            o.w = pack2<BF16>(__uint_as_float(v[8 * jj + 6]) + bf[6], __uint_as_float(v[8 * jj + 7]) + bf[7]);
            *reinterpret_cast<uint4*>(my_row + ((j ^ (row_in_blk & 7)) << 4)) = o;
          }
#ifdef B200_HSTU_PROFILING
          if (tr) tq2 = clock64();
#endif
          fence_proxy_async();
#ifdef B200_HSTU_PROFILING
          if (tr) tq3 = clock64();
#endif
          asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");  // the box is staged
          if (row_in_blk == 0) {
            tma_store_2d(&maps.o, smem_u32(stage), col0, static_cast<int>(blk * BM));
            bulk_commit();
          }
#ifdef B200_HSTU_PROFILING
          if (tr) {
            tq4 = clock64();
            printf("box g=%u h=%d: wait_read+bar %lld, bias+math+st.shared %lld, fence %lld, bar+tma %lld | t=%lld\n", g, h,
                   tq1 - tq0, tq2 - tq1, tq3 - tq2, tq4 - tq3, tq4);
          }
#endif
        }
      }
    }
    if (row_in_blk == 0) bulk_wait_all();  // shared memory must outlive the stores that read it
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    if (*abort_flag) {  // a wait gave up: let copies and MMAs in flight finish before the TMEM is released
      const unsigned long long t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
    }
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace
}  // namespace gemm
}  // namespace hstu

extern "C" int b200_stu_addmm_supported(const B200GemmParams* p) {
  if (p == nullptr || p->struct_size != sizeof(B200GemmParams)) return 0;
  if (p->dtype != B200_HSTU_BF16 && p->dtype != B200_HSTU_F16) return 0;
  if (p->M <= 0 || p->K <= 0 || p->N <= 0) return 0;
  if (p->K % 64 != 0 || p->K > hstu::gemm::MAX_K || p->N % 8 != 0) return 0;
  if (p->M >= (1LL << 31) - 256 || p->N >= (1LL << 30)) return 0;
  return 1;
}

extern "C" int b200_stu_addmm(const B200GemmParams* p, void* stream) {
  using namespace hstu::gemm;
  if (p == nullptr) return B200_HSTU_EINVAL;
  if (p->struct_size != sizeof(B200GemmParams)) return B200_HSTU_EVERSION;
  if (p->M < 0 || p->K <= 0 || p->N <= 0) return B200_HSTU_EINVAL;
  if (p->M == 0) return B200_HSTU_OK;
  if (!b200_stu_addmm_supported(p)) return B200_HSTU_EUNSUPPORTED;
  const bool fuse = (p->flags & B200_GEMM_FLAG_LAYER_NORM) != 0;
  if (!p->x || !p->w || !p->bias || !p->out) return B200_HSTU_EINVAL;
  if (fuse && (!p->mean || !p->rstd)) return B200_HSTU_EINVAL;
  if ((p->ln_weight == nullptr) != (p->ln_bias == nullptr)) return B200_HSTU_EINVAL;
  if ((p->flags & B200_GEMM_FLAG_SWISH) && (!fuse || !p->ln_weight)) return B200_HSTU_EINVAL;
  if (p->x_row_stride < p->K || p->w_row_stride < p->N || p->out_row_stride < p->N) return B200_HSTU_EINVAL;
  if (p->bias_row_stride != 0 && p->bias_row_stride < p->N) return B200_HSTU_EINVAL;
  auto bad = [](const void* q, long long stride) { return reinterpret_cast<uintptr_t>(q) % 16 != 0 || stride % 8 != 0; };
  if (bad(p->x, p->x_row_stride) || bad(p->w, p->w_row_stride) || bad(p->out, p->out_row_stride) ||
      bad(p->bias, p->bias_row_stride) || (p->ln_weight && (bad(p->ln_weight, 0) || bad(p->ln_bias, 0))))
    return B200_HSTU_EALIGN;
  const bool bf16 = p->dtype == B200_HSTU_BF16;
  hstu::set_error_stage("addmm: tensor maps");
  if (!hstu::tc::ensure_current_context(p->x)) return B200_HSTU_ELAUNCH;
  Maps maps;
  if (!hstu::tc::make_map_box(&maps.w, p->w, p->K, p->N, p->w_row_stride, BK, bf16)) return B200_HSTU_ELAUNCH;
  if (!hstu::tc::make_map_box(&maps.o, p->out, p->M, p->N, p->out_row_stride, BM, bf16)) return B200_HSTU_ELAUNCH;
  if (fuse) maps.x = maps.w;  // not used by the kernel
  else if (!hstu::tc::make_map_box(&maps.x, p->x, p->M, p->K, p->x_row_stride, 128, bf16)) return B200_HSTU_ELAUNCH;
  Args a;
  a.x = p->x; a.ln_w = p->ln_weight; a.ln_b = p->ln_bias; a.bias = p->bias; a.out = p->out;
  a.mean = p->mean; a.rstd = p->rstd; a.status = p->status;
  a.M = p->M; a.x_rs = p->x_row_stride; a.out_rs = p->out_row_stride; a.bias_rs = p->bias_row_stride;
  a.K = static_cast<int>(p->K); a.N = static_cast<int>(p->N);
  a.fuse_ln = fuse ? 1 : 0; a.swish = (p->flags & B200_GEMM_FLAG_SWISH) ? 1 : 0; a.affine = p->ln_weight ? 1 : 0;
  a.eps = p->eps;
  a.dbg = 0;
#ifdef B200_HSTU_PROFILING
  if (const char* e = getenv("B200_GEMM_DBG")) a.dbg = atoi(e);
#endif
  const long long n_blocks = (p->M + BM - 1) / BM;
  const int sms = hstu::tc::sm_count();
  const unsigned grid = static_cast<unsigned>(n_blocks < sms ? n_blocks : sms);
  const size_t smem = sizeof(Shared) + 1024;
  auto kern = bf16 ? stu_addmm_tc<true> : stu_addmm_tc<false>;
  hstu::set_error_stage("addmm: kernel");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return B200_HSTU_ELAUNCH;
  kern<<<grid, THREADS, smem, static_cast<cudaStream_t>(stream)>>>(maps, a);
  return cudaGetLastError() == cudaSuccess ? B200_HSTU_OK : B200_HSTU_ELAUNCH;
}
