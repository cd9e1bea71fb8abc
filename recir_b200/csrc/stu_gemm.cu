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
// Tiling.  A CTA owns a block of 128 rows and keeps its whole A operand (K <= 512) in tensor memory:
// 16 k-values of a row are 8 TMEM columns, so K = 512 takes 256 of the 512 columns; the other 256 are two
// 128-column fp32 accumulators.  The rows reach TMEM 64 at a time through a 64 KB staging buffer in the
// 128-byte-swizzled box layout: written by TMA (plain and jagged mode) or by the layer-norm prologue, then
// copied row-per-thread with tcgen05.st by the warps whose TMEM lane quadrant holds those rows.  W streams
// through an 8-stage ring of [64 k-rows x 128 n-columns] tiles (TMA, two 64-column boxes, N-major B
// operand); four tcgen05.mma M128 N128 K16 (A from TMEM) per stage.  The epilogue of an output tile (bias,
// rounding, staged bulk tensor stores) overlaps the MMAs of the next one.  With A out of shared memory the
// MMAs read only W from it, half of what the SS form reads, and the ring is deep enough (128 KB) to ride
// out the L2 latency of W, which stays L2-resident (K x N x 2 bytes, a few MB at most).
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = MMA issuer (one elected lane), warps 2-9 =
// layer-norm prologue (8 rows per warp and round, four at a time in registers), staging-to-TMEM copy and
// epilogue (TMEM lane quadrant warp % 4, column half (warp - 2) / 4).  Every wait is bounded (see
// sm100_ptx.cuh).
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

constexpr int BM = 128, BN = 128, BK = 64;  // BK: k-rows of W per pipeline stage (four k-steps of 16)
constexpr int MAX_K = 512;
constexpr int W_STAGES = 8;
constexpr int W_BOX_BYTES = BK * 128;        // 64 k-rows x 64 n-columns of 16-bit elements
constexpr int W_STAGE_BYTES = 2 * W_BOX_BYTES;
constexpr int X_ROWS = 64;                   // rows of x staged at a time on their way into TMEM
constexpr int X_BOX_BYTES = X_ROWS * 128;    // 64 rows x 64 k-columns
constexpr int OUT_BOX_BYTES = BM * 128;      // 128 rows x 64 output columns, one box per epilogue group
constexpr int THREADS = 320;                 // 10 warps: 200 registers each without any reallocation
constexpr int TMEM_COLS = 512;
constexpr int TMEM_A = 0, TMEM_ACC0 = 256;   // A operand: K / 2 columns (two 16-bit values each); 2 x 128 accumulator columns
enum { WAIT_GEMM_PRODUCER = 111, WAIT_GEMM_MMA = 112, WAIT_GEMM_EPILOGUE = 113 };

struct Shared {
  unsigned char w[W_STAGES][W_STAGE_BYTES];       // 128 KB weight ring
  unsigned char x[MAX_K / 64][X_BOX_BYTES];       // 64 KB: 64 rows of the A operand in the swizzled box layout
  unsigned char out[2][OUT_BOX_BYTES];            // 32 KB output staging
  unsigned long long x_full, x_free;              // plain mode: TMA landed a 64-row round / the round was copied to TMEM
  unsigned long long a_ready, a_free;             // the block's A operand is in TMEM / every MMA reading it has run
  unsigned long long w_full[W_STAGES], w_empty[W_STAGES];
  unsigned long long acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct Maps {
  CUtensorMap x;  // [M, K], box 64 columns x 64 rows (unused with the layer-norm prologue)
  CUtensorMap w;  // [K, N] (jagged mode: [B * K, N]), box 64 columns x 64 rows
  CUtensorMap o;  // [M, N], box 64 columns x 128 rows (bulk stores; rows past M and columns past N are clipped)
};

struct Args {
  const void* x; const void* ln_w; const void* ln_b; const void* bias; void* out;
  float* mean; float* rstd; int* status;
  long long M, x_rs, out_rs, bias_rs;
  int K, N, fuse_ln, swish, affine;
  float eps;
  // jagged mode (per-sequence weight matrices): the row blocks come from a device-built list
  const int4* items;     // (sequence, first row, valid rows, 0) per 128-row block; null = plain row blocks of x
  const int* n_items;    // number of list entries
  const void* offsets;   // jagged mode: seq_offsets (to find the first row no sequence owns)
  int off64, num_seqs;
  int per_seq_bias;      // bias row = sequence index (else: output row index, or the single row when bias_rs == 0)
  int dbg;  // instrumented builds only (B200_GEMM_DBG): 1 no W loads / waits, 2 no output staging, 4 no MMAs
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
  const int kboxes = a.K / 64;   // 64-column boxes of the A operand = pipeline stages of W per output tile
  const int n_tiles = (a.N + BN - 1) / BN;
  const long long n_blocks = a.items ? static_cast<long long>(*a.n_items) : (a.M + BM - 1) / BM;
  // block -> (sequence, first row, valid rows); plain mode: one "sequence" holding every row
  auto block_of = [&](long long blk) -> int4 {
    if (a.items) return a.items[blk];
    const long long row0 = blk * BM, left = a.M - row0;
    return make_int4(0, static_cast<int>(row0), static_cast<int>(left < BM ? left : BM), 0);
  };

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    mbar_init(smem_u32(&sh.x_full), 1);
    mbar_init(smem_u32(&sh.x_free), 128);  // the 128 threads that copy a 64-row round
    mbar_init(smem_u32(&sh.a_ready), 256);
    mbar_init(smem_u32(&sh.a_free), 1);
    for (int i = 0; i < W_STAGES; ++i) { mbar_init(smem_u32(&sh.w_full[i]), 1); mbar_init(smem_u32(&sh.w_empty[i]), 1); }
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
    uint32_t round = 0, st = 0, ph = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_GEMM_PRODUCER));
    };
    // x of a block arrives in two rounds of 64 rows through the staging buffer (plain and jagged mode)
    auto load_x_round = [&](const int4& bi, int r) -> bool {
      if (!wait_all(&sh.x_free, (round & 1) ^ 1)) return false;
      if (elect_one()) {
        mbar_arrive_expect_tx(smem_u32(&sh.x_full), static_cast<uint32_t>(kboxes) * X_BOX_BYTES);
        for (int kb = 0; kb < kboxes; ++kb)
          tma_load_2d(smem_u32(sh.x[kb]), &maps.x, smem_u32(&sh.x_full), kb * 64, bi.y + r * X_ROWS);
      }
      __syncwarp();
      ++round;
      return true;
    };
    long long blk = blockIdx.x;
    if (!a.fuse_ln && blk < n_blocks) ok = load_x_round(block_of(blk), 0);
    for (; blk < n_blocks && ok; blk += gridDim.x) {
      const int4 bi = block_of(blk);
      const int w_row0 = bi.x * a.K;  // first row of this sequence's matrix in the stacked [B * K, N] weights
      for (int nt = 0; nt < n_tiles && ok; ++nt) {
        for (int kb = 0; kb < kboxes; ++kb) {
#ifdef B200_HSTU_PROFILING
          if (a.dbg & 1) continue;
#endif
          ok = wait_all(&sh.w_empty[st], ph ^ 1);
          if (!ok) break;
          if (elect_one()) {
            mbar_arrive_expect_tx(smem_u32(&sh.w_full[st]), W_STAGE_BYTES);
#pragma unroll
            for (int j = 0; j < 2; ++j)  // columns past N are filled with zeros
              tma_load_2d(smem_u32(sh.w[st]) + j * W_BOX_BYTES, &maps.w, smem_u32(&sh.w_full[st]), nt * BN + j * 64,
                          w_row0 + kb * BK);
          }
          __syncwarp();
          if (++st == W_STAGES) { st = 0; ph ^= 1; }
        }
        if (a.fuse_ln || !ok) continue;
        // Behind the first output tile's weights (they only wait for the previous block's MMAs): the second
        // 64 rows of this block, as soon as the first 64 have been copied into TMEM.  Behind the second
        // tile's weights: the next block's first 64 rows, which then land while this block computes.
        if (nt == 0) ok = load_x_round(bi, 1);
        if (ok && nt == (n_tiles > 1 ? 1 : 0) && blk + gridDim.x < n_blocks) ok = load_x_round(block_of(blk + gridDim.x), 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC = idesc_f16(BF16 ? 1 : 0, BM, BN, 0, 1);  // A from TMEM, B N-major in shared memory
    constexpr uint32_t HI = desc_hi_sw128(1024);
    const uint32_t w_lo0 = desc_lo_sw128(smem_u32(sh.w[0]), W_BOX_BYTES);  // 64-column groups are one box apart
    uint32_t it = 0, st = 0, ph = 0, g = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_GEMM_MMA));
    };
    for (long long blk = blockIdx.x; blk < n_blocks && ok; blk += gridDim.x, ++it) {
      ok = wait_all(&sh.a_ready, it & 1);
      if (!ok) break;
      tc_fence_after();
      for (int nt = 0; nt < n_tiles && ok; ++nt, ++g) {
        const uint32_t buf = g & 1;
        ok = wait_all(&sh.acc_empty[buf], ((g >> 1) & 1) ^ 1);
        if (!ok) break;
        tc_fence_after();
        for (int kb = 0; kb < kboxes; ++kb) {
#ifdef B200_HSTU_PROFILING
          if (a.dbg & 1) {
            if (elect_one() && !(a.dbg & 4)) {
              for (int kk = 0; kk < BK / 16; ++kk)
                mma_ts(tmem + TMEM_ACC0 + buf * BN, tmem + TMEM_A + (kb * 4 + kk) * 8,
                       desc_join(w_lo0 + (kb & 7) * (W_STAGE_BYTES >> 4) + kk * (2048 >> 4), HI), IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            __syncwarp();
            continue;
          }
#endif
          ok = wait_all(&sh.w_full[st], ph);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
#ifdef B200_HSTU_PROFILING
            if (!(a.dbg & 4))
#endif
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              // A: 16 k-values = 8 TMEM columns; B: k-step kk of the stage (16 rows of 128 bytes per box)
              mma_ts(tmem + TMEM_ACC0 + buf * BN, tmem + TMEM_A + (kb * 4 + kk) * 8,
                     desc_join(w_lo0 + st * (W_STAGE_BYTES >> 4) + kk * (2048 >> 4), HI), IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
            tc_commit(smem_u32(&sh.w_empty[st]));
          }
          __syncwarp();
          if (++st == W_STAGES) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        if (elect_one()) tc_commit(smem_u32(&sh.acc_full[buf]));
        __syncwarp();
      }
      if (!ok) break;
      if (elect_one()) tc_commit(smem_u32(&sh.a_free));  // every MMA that reads this block's A operand has been issued
      __syncwarp();
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ prologue + epilogue warps (2..9)
    const int ew = warp - 2;                  // 0..7
    const int wg = ew >> 2;                   // column half of the output tile / k half of the A operand
    const int quad = warp & 3;                // TMEM lane quadrant this warp may touch
    const uint32_t lane_addr = static_cast<uint32_t>(quad << 5) << 16;
    const int row_in_blk = (quad << 5) | lane;
    const int nv = a.K >> 3;  // 16-byte vectors per row (at most 64: two per lane)
    uint32_t it = 0, g = 0, round = 0;
    bool ok = true;
    if (a.items) {
      // rows at or past the last offset belong to no sequence: defined output (zeros), never stale memory
      long long first = a.off64 ? reinterpret_cast<const long long*>(a.offsets)[a.num_seqs]
                                : static_cast<long long>(reinterpret_cast<const int*>(a.offsets)[a.num_seqs]);
      first = first < 0 ? 0 : (first > a.M ? a.M : first);
      const long long chunks_per_row = a.N >> 3, total = (a.M - first) * chunks_per_row;
      for (long long c = static_cast<long long>(blockIdx.x) * 256 + (threadIdx.x - 64); c < total; c += static_cast<long long>(gridDim.x) * 256) {
        const long long r = first + c / chunks_per_row, col = (c % chunks_per_row) * 8;
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + r * a.out_rs + col) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
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
    // Copies this thread's row of the staged 64-row round into the A operand in TMEM: warps of lane quadrants
    // 2 r and 2 r + 1 own the rows of round r; group wg copies k-columns [K/2 wg, K/2 wg + K/2).
    auto copy_round_to_tmem = [&](int r) {
      if ((quad >> 1) != r) return;
      const int rl = row_in_blk - r * X_ROWS;  // row inside the staging buffer
      const int boxes_half = kboxes >> 1, b0 = wg * boxes_half, b1 = (wg == 0) ? boxes_half : kboxes;
      for (int b = b0; b < b1; ++b) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 2 x 32 elements = 2 x 16 TMEM columns per 64-column box
          uint32_t rr[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int chunk = h * 4 + j;
            const uint4 xq = *reinterpret_cast<const uint4*>(sh.x[b] + rl * 128 + ((chunk ^ (rl & 7)) << 4));
            rr[4 * j + 0] = xq.x; rr[4 * j + 1] = xq.y; rr[4 * j + 2] = xq.z; rr[4 * j + 3] = xq.w;
          }
          tmem_st16(tmem + lane_addr + TMEM_A + b * 32 + h * 16, rr);
        }
      }
    };
    for (long long blk = blockIdx.x; blk < n_blocks && ok; blk += gridDim.x, ++it) {
      const int4 bi = block_of(blk);
      // ---- A operand of the block into TMEM, 64 rows at a time through the staging buffer
      for (int r = 0; r < 2 && ok; ++r, ++round) {
        if (a.fuse_ln) {
          // layer norm of 8 rows per warp (four at a time in registers) into the swizzled staging boxes
          for (int r0 = 0; r0 < 8; r0 += 4) {
            float xv[4][2][8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const long long row = static_cast<long long>(bi.y) + r * X_ROWS + ew * 8 + r0 + q;
              const T* xr = reinterpret_cast<const T*>(a.x) + (row < a.M ? row : a.M - 1) * a.x_rs;
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int v = lane + 32 * j;
                if (v < nv) {
                  load8<T>(xr + 8 * v, xv[q][j]);
                } else {
#pragma unroll
                  for (int i = 0; i < 8; ++i) xv[q][j][i] = 0.f;
                }
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int rl = ew * 8 + r0 + q;  // row inside the staging buffer
              const long long row = static_cast<long long>(bi.y) + r * X_ROWS + rl;
              // mean first, then the mean of squared deviations (kjt_split_per_feature.cpp:223-226)
              float s = 0.f;
#pragma unroll
              for (int j = 0; j < 2; ++j)
                if (lane + 32 * j < nv) {
#pragma unroll
                  for (int i = 0; i < 8; ++i) s += xv[q][j][i];
                }
              const float mean = warp_sum(s) / static_cast<float>(a.K);
              float sq = 0.f;
#pragma unroll
              for (int j = 0; j < 2; ++j)
                if (lane + 32 * j < nv) {
#pragma unroll
                  for (int i = 0; i < 8; ++i) { const float d = xv[q][j][i] - mean; sq += d * d; }
                }
              const float rstd = rsqrtf(warp_sum(sq) / static_cast<float>(a.K) + a.eps);
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
                    float y = (xv[q][j][i] - mean) * rstd;
                    if (a.affine) y = y * wv[i] + bv[i];
                    if (a.swish) y = __fdividef(1.f, 1.f + __expf(-y)) * xv[q][j][i];
                    n[i] = y;
                  }
                  pk.x = pack2<BF16>(n[0], n[1]); pk.y = pack2<BF16>(n[2], n[3]);
                  pk.z = pack2<BF16>(n[4], n[5]); pk.w = pack2<BF16>(n[6], n[7]);
                }
                // vector v = 8 columns: box v / 8, 16-byte chunk v % 8 of the 128-byte box row, swizzled
                *reinterpret_cast<uint4*>(sh.x[v >> 3] + rl * 128 + (((v & 7) ^ (rl & 7)) << 4)) = pk;
              }
            }
          }
          asm volatile("bar.sync 3, 256;" ::: "memory");  // the 64 rows are staged
        } else {
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.x_full), round & 1, abort_flag, a.status, WAIT_GEMM_EPILOGUE));
          if (!ok) break;
        }
        if (r == 0) {  // the previous block's MMAs must have finished reading the A operand before it is overwritten
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.a_free), (it & 1) ^ 1, abort_flag, a.status, WAIT_GEMM_EPILOGUE));
          if (!ok) break;
          tc_fence_after();
        }
        copy_round_to_tmem(r);
        if (a.fuse_ln) {
          asm volatile("bar.sync 3, 256;" ::: "memory");  // the staging buffer may be overwritten
        } else if ((quad >> 1) == r) {
          mbar_arrive(smem_u32(&sh.x_free));  // the round has been read: the next one may land
        }
      }
      if (!ok) break;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&sh.a_ready));
      // ---- epilogue of every output tile of the block: bias, rounding, staged bulk stores.
      // Group wg owns output columns [64 wg, 64 wg + 64) of the tile and sends them out as one box through
      // its own staging buffer (128-byte-swizzled rows, as the bulk tensor store expects).
      const long long row = static_cast<long long>(bi.y) + row_in_blk;
      const long long brow_idx = a.per_seq_bias ? bi.x : (row < a.M ? row : a.M - 1);
      unsigned char* stage = sh.out[wg];
      for (int nt = 0; nt < n_tiles && ok; ++nt, ++g) {
        const uint32_t buf = g & 1;
        const int col0 = nt * BN + wg * 64;
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
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.acc_full[buf]), (g >> 1) & 1, abort_flag, a.status, WAIT_GEMM_EPILOGUE));
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + lane_addr + TMEM_ACC0 + buf * BN + wg * 64;
        uint32_t v0[32], v1[32];
        tmem_ld32(acc, v0);
        tmem_ld32(acc + 32, v1);
        tmem_wait_ld(v0);
        tmem_wait_ld(v1);
        tc_fence_before();
        mbar_arrive(smem_u32(&sh.acc_empty[buf]));  // the accumulator is in registers: the MMAs may reuse it
        if (col0 >= a.N) continue;  // uniform for the group
#ifdef B200_HSTU_PROFILING
        if (a.dbg & 2) continue;
#endif
        if (row_in_blk == 0) bulk_wait_read_all();  // the group's previous box has left the staging buffer
        asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");
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
        fence_proxy_async();
        asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");  // the box is staged
        if (bi.z >= BM || !a.items) {
          // whole block (in plain mode the tensor map clips rows past M): one bulk tensor store
          if (row_in_blk == 0) {
            tma_store_2d(&maps.o, smem_u32(stage), col0, bi.y);
            bulk_commit();
          }
        } else {
          // ragged last block of a sequence: the rows behind it belong to the next sequence, so the valid
          // rows are copied out by the threads (8 lanes per 128-byte row segment)
          const int chunk = row_in_blk & 7;
          if (col0 + chunk * 8 < a.N) {
            T* obase = reinterpret_cast<T*>(a.out) + static_cast<long long>(bi.y) * a.out_rs + col0 + chunk * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = i * 16 + (row_in_blk >> 3);
              if (r < bi.z)
                *reinterpret_cast<uint4*>(obase + static_cast<long long>(r) * a.out_rs) =
                    *reinterpret_cast<const uint4*>(stage + r * 128 + ((chunk ^ (r & 7)) << 4));
            }
          }
        }  // (the barrier at the top of the next box orders these reads before its writes)
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

// Row blocks of a jagged batch: entry i = (sequence, first row, valid rows) for every 128-row block of
// every sequence, in sequence order; ws[0] = number of entries.  One CTA; offsets are clamped into [0, T]
// like everywhere else in this library, and the list is cut at its capacity (T / 128 + B entries cover
// every batch whose sequences do not overlap).
__global__ void __launch_bounds__(1024) build_gemm_items(const void* offsets, int off64, int B, long long T, int* ws,
                                                         long long max_items, int* status) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  int4* items = reinterpret_cast<int4*>(ws + 4);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  auto off = [&](int i) -> long long {
    long long v = off64 ? reinterpret_cast<const long long*>(offsets)[i] : static_cast<long long>(reinterpret_cast<const int*>(offsets)[i]);
    return v < 0 ? 0 : (v > T ? T : v);
  };
  for (int base = 0; base < B; base += 1024) {
    const int b = base + tid;
    long long s = 0, e = 0;
    if (b < B) { s = off(b); e = off(b + 1); if (e < s) e = s; }
    const int nb = static_cast<int>((e - s + BM - 1) / BM);
    int incl = nb;  // inclusive scan over the CTA
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) { const int t = __shfl_up_sync(0xffffffffu, incl, o); if (lane >= o) incl += t; }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      int t = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) { const int u = __shfl_up_sync(0xffffffffu, t, o); if (lane >= o) t += u; }
      warp_tot[lane] = t;
    }
    __syncthreads();
    const int first = carry + (wid > 0 ? warp_tot[wid - 1] : 0) + incl - nb;
    for (int i = 0; i < nb; ++i) {
      const long long slot = static_cast<long long>(first) + i;
      if (slot >= max_items) { if (status) atomicOr(status, 1); break; }
      const long long row0 = s + static_cast<long long>(i) * BM, left = e - row0;
      items[slot] = make_int4(b, static_cast<int>(row0), static_cast<int>(left < BM ? left : BM), 0);
    }
    __syncthreads();
    if (tid == 0) carry += warp_tot[31];
    __syncthreads();
  }
  if (tid == 0) ws[0] = static_cast<int>(carry < max_items ? carry : max_items);
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

namespace {
// Shared launch path of the two entry points.
int launch_gemm(const B200GemmParams* p, const void* w_base, long long w_rows, const int4* items, const int* n_items,
                long long max_blocks, int per_seq_bias, const void* offsets, int off64, int num_seqs, void* stream) {
  using namespace hstu::gemm;
  const bool fuse = (p->flags & B200_GEMM_FLAG_LAYER_NORM) != 0;
  const bool bf16 = p->dtype == B200_HSTU_BF16;
  hstu::set_error_stage("addmm: tensor maps");
  if (!hstu::tc::ensure_current_context(p->x)) return B200_HSTU_ELAUNCH;
  Maps maps;
  if (!hstu::tc::make_map_box(&maps.w, w_base, w_rows, p->N, p->w_row_stride, BK, bf16)) return B200_HSTU_ELAUNCH;
  if (!hstu::tc::make_map_box(&maps.o, p->out, p->M, p->N, p->out_row_stride, BM, bf16)) return B200_HSTU_ELAUNCH;
  if (fuse) maps.x = maps.w;  // not used by the kernel
  else if (!hstu::tc::make_map_box(&maps.x, p->x, p->M, p->K, p->x_row_stride, X_ROWS, bf16)) return B200_HSTU_ELAUNCH;
  Args a;
  a.x = p->x; a.ln_w = p->ln_weight; a.ln_b = p->ln_bias; a.bias = p->bias; a.out = p->out;
  a.mean = p->mean; a.rstd = p->rstd; a.status = p->status;
  a.M = p->M; a.x_rs = p->x_row_stride; a.out_rs = p->out_row_stride; a.bias_rs = p->bias_row_stride;
  a.K = static_cast<int>(p->K); a.N = static_cast<int>(p->N);
  a.fuse_ln = fuse ? 1 : 0; a.swish = (p->flags & B200_GEMM_FLAG_SWISH) ? 1 : 0; a.affine = p->ln_weight ? 1 : 0;
  a.eps = p->eps;
  a.items = items; a.n_items = n_items; a.per_seq_bias = per_seq_bias;
  a.offsets = offsets; a.off64 = off64; a.num_seqs = num_seqs;
  a.dbg = 0;
#ifdef B200_HSTU_PROFILING
  if (const char* e = getenv("B200_GEMM_DBG")) a.dbg = atoi(e);
#endif
  const int sms = hstu::tc::sm_count();
  const unsigned grid = static_cast<unsigned>(max_blocks < sms ? (max_blocks < 1 ? 1 : max_blocks) : sms);
  const size_t smem = sizeof(Shared) + 1024;
  auto kern = bf16 ? stu_addmm_tc<true> : stu_addmm_tc<false>;
  hstu::set_error_stage("addmm: kernel");
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return B200_HSTU_ELAUNCH;
  kern<<<grid, THREADS, smem, static_cast<cudaStream_t>(stream)>>>(maps, a);
  return cudaGetLastError() == cudaSuccess ? B200_HSTU_OK : B200_HSTU_ELAUNCH;
}

int check_common(const B200GemmParams* p) {
  if (p == nullptr) return B200_HSTU_EINVAL;
  if (p->struct_size != sizeof(B200GemmParams)) return B200_HSTU_EVERSION;
  if (p->M < 0 || p->K <= 0 || p->N <= 0) return B200_HSTU_EINVAL;
  if (p->M == 0) return B200_HSTU_OK;
  if (!b200_stu_addmm_supported(p)) return B200_HSTU_EUNSUPPORTED;
  if (!p->x || !p->w || !p->bias || !p->out) return B200_HSTU_EINVAL;
  if (p->x_row_stride < p->K || p->w_row_stride < p->N || p->out_row_stride < p->N) return B200_HSTU_EINVAL;
  if (p->bias_row_stride != 0 && p->bias_row_stride < p->N) return B200_HSTU_EINVAL;
  auto bad = [](const void* q, long long stride) { return reinterpret_cast<uintptr_t>(q) % 16 != 0 || stride % 8 != 0; };
  if (bad(p->x, p->x_row_stride) || bad(p->w, p->w_row_stride) || bad(p->out, p->out_row_stride) ||
      bad(p->bias, p->bias_row_stride))
    return B200_HSTU_EALIGN;
  return 1;  // go on
}
}  // namespace

extern "C" int b200_stu_addmm(const B200GemmParams* p, void* stream) {
  const int rc = check_common(p);
  if (rc != 1) return rc;
  const bool fuse = (p->flags & B200_GEMM_FLAG_LAYER_NORM) != 0;
  if (fuse && (!p->mean || !p->rstd)) return B200_HSTU_EINVAL;
  if ((p->ln_weight == nullptr) != (p->ln_bias == nullptr)) return B200_HSTU_EINVAL;
  if ((p->flags & B200_GEMM_FLAG_SWISH) && (!fuse || !p->ln_weight)) return B200_HSTU_EINVAL;
  if (p->ln_weight && (reinterpret_cast<uintptr_t>(p->ln_weight) % 16 != 0 || reinterpret_cast<uintptr_t>(p->ln_bias) % 16 != 0))
    return B200_HSTU_EALIGN;
  return launch_gemm(p, p->w, p->K, nullptr, nullptr, (p->M + hstu::gemm::BM - 1) / hstu::gemm::BM, 0, nullptr, 0, 0, stream);
}

extern "C" size_t b200_stu_jagged_bmm_workspace_bytes(int64_t rows, int64_t num_seqs) {
  if (rows < 0 || num_seqs < 0) return 0;
  const long long max_items = rows / hstu::gemm::BM + num_seqs;
  return static_cast<size_t>(16 + 16 * max_items + 255) & ~static_cast<size_t>(255);
}

extern "C" int b200_stu_jagged_dense_bmm_add(const B200GemmParams* p, const void* seq_offsets, int offsets_i64,
                                             int64_t num_seqs, int64_t w_seq_stride, int per_row_bias, void* workspace,
                                             uint64_t workspace_bytes, void* stream) {
  using namespace hstu::gemm;
  const int rc = check_common(p);
  if (rc != 1) return rc;
  if (p->flags != 0 || seq_offsets == nullptr || num_seqs <= 0) return B200_HSTU_EINVAL;
  if (w_seq_stride != p->K * p->w_row_stride) return B200_HSTU_EUNSUPPORTED;  // the matrices must be stacked densely
  if (num_seqs * p->K >= (1LL << 31)) return B200_HSTU_EUNSUPPORTED;
  if (per_row_bias ? p->bias_row_stride < p->N : (p->bias_row_stride != 0 && p->bias_row_stride < p->N)) return B200_HSTU_EINVAL;
  const size_t need = b200_stu_jagged_bmm_workspace_bytes(p->M, num_seqs);
  if (workspace == nullptr || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
    return B200_HSTU_EWORKSPACE;
  const long long max_items = p->M / BM + num_seqs;
  int* ws = reinterpret_cast<int*>(workspace);
  hstu::set_error_stage("jagged bmm: row-block list");
  build_gemm_items<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(seq_offsets, offsets_i64 ? 1 : 0, static_cast<int>(num_seqs),
                                                                      p->M, ws, max_items, p->status);
  if (cudaGetLastError() != cudaSuccess) return B200_HSTU_ELAUNCH;
  return launch_gemm(p, p->w, num_seqs * p->K, reinterpret_cast<const int4*>(ws + 4), ws, max_items, per_row_bias ? 0 : 1,
                     seq_offsets, offsets_i64 ? 1 : 0, static_cast<int>(num_seqs), stream);
}
