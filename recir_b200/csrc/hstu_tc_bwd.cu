// Tensor-core backward of the HSTU jagged attention for sm_100a: a dK/dV pass that is
// key-block-major and a dQ pass that is query-block-major.  Every gradient row is owned by
// exactly one work item, so no atomics touch the gradients and results are deterministic.
//
// Both kernels recompute S = alpha Q K^T and dP = dO V^T tile by tile (nothing but q, k, v
// was saved by the forward), form P and dS on the TMEM accumulators and feed them back to
// the tensor cores as 16-bit TMEM operands:
//   dQ pass   (rows = queries): dQ += dS K              Q and dO sit in TMEM as A operands
//   dK/dV pass (rows = keys)  : dV += P^T dO, dK += dS^T Q   with S^T = K Q^T, dP^T = V dO^T
// Score tiles are processed as 64-column halves of a 128-row shared-memory tile so that two
// halves can be in flight (one in the tensor cores, one in the epilogue warps) inside the
// 512 TMEM columns.  silu'(x) = sigma (1 + x (1 - sigma)); with t = tanh(x / 2) this is
// 0.5 (1 + t)(1 + (x/2)(1 - t)); the 0.5, alpha and a scalar attn_scale are applied once per
// output row when the accumulator leaves TMEM.
#include <cuda.h>
#include <cuda_runtime.h>

#include "hstu_launch.h"
#include "hstu_tc_common.cuh"
#include "hstu_tc_host.h"

namespace hstu {
namespace tc {
namespace {

using namespace sm100;

constexpr int BWD_THREADS = 384;
constexpr int TMEM_COLS = 512;

struct MapsBwd {
  CUtensorMap q, k, v, d_o;
};

// 16 feature columns (one MMA k-step) inside a K-major tile: 32 bytes inside a 64-column box,
// boxes 16 KB apart.
__device__ __forceinline__ uint32_t kstep_offset(int kk) { return (kk >> 2) * HALF_TILE_BYTES + (kk & 3) * 32; }

// u = alpha/2 * s, t = tanh(u):  p = x sigma(x) = u t + u,  2 silu'(x) = (1 + t)(1 + u (1 - t))
__device__ __forceinline__ void silu_terms(float s, float c1, float& p, float& dsilu2) {
  const float u = c1 * s;
  const float t = tanh_approx(u);
  p = fmaf(u, t, u);
  dsilu2 = (1.f + t) * (fmaf(-u, t, u) + 1.f);
}

// ------------------------------------------------------------------------------------
// dQ pass
// ------------------------------------------------------------------------------------
constexpr int DQ_STAGES = 3;
constexpr int DQ_QA = 0, DQ_DOA = 64, DQ_S0 = 128, DQ_DP0 = 256, DQ_ACC = 384;  // S1 = S0 + 64, DP1 = DP0 + 64

struct DqShared {
  unsigned char k[DQ_STAGES][TILE_BYTES];
  unsigned char v[DQ_STAGES][TILE_BYTES];
  unsigned long long k_full[DQ_STAGES], k_empty[DQ_STAGES];
  unsigned long long v_full[DQ_STAGES], v_empty[DQ_STAGES];
  unsigned long long a_ready, s_full[2], ds_ready[2], acc_full, acc_empty;
  uint32_t tmem_base;
  int abort_flag;
};

template <bool IS_BF16>
__global__ void __launch_bounds__(BWD_THREADS, 1)
hstu_bwd_dq_tc(const __grid_constant__ MapsBwd maps, KernelArgs a, const int* __restrict__ ws, long long off_items) {
  extern __shared__ unsigned char smem_raw[];
  DqShared& sh = *reinterpret_cast<DqShared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = ws[0];
  if (static_cast<int>(blockIdx.x) >= total_items) return;
  const int2* items = reinterpret_cast<const int2*>(ws + off_items);
  volatile int* abort_flag = &sh.abort_flag;

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    for (int i = 0; i < DQ_STAGES; ++i) {
      mbar_init(smem_u32(&sh.k_full[i]), 1); mbar_init(smem_u32(&sh.k_empty[i]), 1);
      mbar_init(smem_u32(&sh.v_full[i]), 1); mbar_init(smem_u32(&sh.v_empty[i]), 1);
    }
    mbar_init(smem_u32(&sh.a_ready), 256);
    for (int i = 0; i < 2; ++i) { mbar_init(smem_u32(&sh.s_full[i]), 1); mbar_init(smem_u32(&sh.ds_ready[i]), 128); }
    mbar_init(smem_u32(&sh.acc_full), 1);
    mbar_init(smem_u32(&sh.acc_empty), 256);
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
    if (lane == 0) {
      prefetch_tensormap(&maps.k);
      prefetch_tensormap(&maps.v);
      uint32_t gt = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const int2 w = items[item];
        if (w.x < 0) continue;
        const int b = w.x & 0xffff, head = w.x >> 16, qblk = w.y;
        const SeqInfo s = load_seq(a, b);
        const int m0 = qblk * BLK, col0 = head * HEAD_DIM;
        const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
        for (int idx = 0; idx < kr.count() && ok; ++idx) {
          const int nb = kr.at(idx);
          if (classify_tile(m0, nb * BLK, s, a.mask) == TILE_SKIP) continue;
          const int krow = static_cast<int>(s.start) + nb * BLK;
          const uint32_t st = gt % DQ_STAGES, ph = (gt / DQ_STAGES) & 1;
          ok = mbar_wait(smem_u32(&sh.k_empty[st]), ph ^ 1, abort_flag, a.status, WAIT_PRODUCER);
          if (!ok) break;
          mbar_arrive_expect_tx(smem_u32(&sh.k_full[st]), TILE_BYTES);
          tma_load_2d(smem_u32(sh.k[st]), &maps.k, smem_u32(&sh.k_full[st]), col0, krow);
          tma_load_2d(smem_u32(sh.k[st]) + HALF_TILE_BYTES, &maps.k, smem_u32(&sh.k_full[st]), col0 + 64, krow);
          ok = mbar_wait(smem_u32(&sh.v_empty[st]), ph ^ 1, abort_flag, a.status, WAIT_PRODUCER);
          if (!ok) break;
          mbar_arrive_expect_tx(smem_u32(&sh.v_full[st]), TILE_BYTES);
          tma_load_2d(smem_u32(sh.v[st]), &maps.v, smem_u32(&sh.v_full[st]), col0, krow);
          tma_load_2d(smem_u32(sh.v[st]) + HALF_TILE_BYTES, &maps.v, smem_u32(&sh.v_full[st]), col0 + 64, krow);
          ++gt;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_f16(IS_BF16 ? 1 : 0, BLK, 64, 0, 0);          // A (TMEM) x K/V half (K-major)
      constexpr uint32_t IDESC_ACC = idesc_f16(IS_BF16 ? 1 : 0, BLK, HEAD_DIM, 0, 1);  // dS (TMEM) x K half (N-major)
      uint32_t gt = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const int2 w = items[item];
        if (w.x < 0) continue;
        const int b = w.x & 0xffff, qblk = w.y;
        const SeqInfo s = load_seq(a, b);
        const int m0 = qblk * BLK;
        ok = mbar_wait(smem_u32(&sh.a_ready), it & 1, abort_flag, a.status, WAIT_MMA);
        if (!ok) break;
        tc_fence_after();
        bool have_prev = false;
        uint32_t prev_gt = 0, prev_sub = 0, n_acc = 0;
        auto issue_acc = [&](uint32_t pgt, uint32_t psub) -> bool {
          if (!mbar_wait(smem_u32(&sh.ds_ready[psub]), pgt & 1, abort_flag, a.status, WAIT_MMA)) return false;
          if (n_acc == 0 && !mbar_wait(smem_u32(&sh.acc_empty), (it & 1) ^ 1, abort_flag, a.status, WAIT_MMA))
            return false;
          tc_fence_after();
          const uint32_t st = pgt % DQ_STAGES;
          const uint32_t kbase = smem_u32(sh.k[st]) + psub * SUBTILE_BYTES;
          const uint32_t ds_tmem = tmem + DQ_DP0 + psub * 64;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bd = smem_desc_sw128(kbase + kk * 2048, HALF_TILE_BYTES, 1024);
            mma_ts(tmem + DQ_ACC, ds_tmem + kk * 8, bd, IDESC_ACC, (n_acc > 0 || kk > 0) ? 1u : 0u);
          }
          if (psub == 1) tc_commit(smem_u32(&sh.k_empty[st]));
          ++n_acc;
          return true;
        };
        const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
        for (int idx = 0; idx < kr.count() && ok; ++idx) {
          const int nb = kr.at(idx);
          if (classify_tile(m0, nb * BLK, s, a.mask) == TILE_SKIP) continue;
          const uint32_t st = gt % DQ_STAGES, ph = (gt / DQ_STAGES) & 1;
          ok = mbar_wait(smem_u32(&sh.k_full[st]), ph, abort_flag, a.status, WAIT_MMA);
          if (!ok) break;
          ok = mbar_wait(smem_u32(&sh.v_full[st]), ph, abort_flag, a.status, WAIT_MMA);
          if (!ok) break;
          tc_fence_after();
          for (uint32_t sub = 0; sub < 2 && ok; ++sub) {
            const uint32_t kbase = smem_u32(sh.k[st]) + sub * SUBTILE_BYTES;
            const uint32_t vbase = smem_u32(sh.v[st]) + sub * SUBTILE_BYTES;
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
              mma_ts(tmem + DQ_S0 + sub * 64, tmem + DQ_QA + kk * 8,
                     smem_desc_sw128(kbase + kstep_offset(kk), 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
              mma_ts(tmem + DQ_DP0 + sub * 64, tmem + DQ_DOA + kk * 8,
                     smem_desc_sw128(vbase + kstep_offset(kk), 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
            tc_commit(smem_u32(&sh.s_full[sub]));
            if (have_prev) ok = issue_acc(prev_gt, prev_sub);
            prev_gt = gt; prev_sub = sub; have_prev = true;
          }
          if (!ok) break;
          tc_commit(smem_u32(&sh.v_empty[st]));
          ++gt;
        }
        if (!ok) break;
        if (have_prev) ok = issue_acc(prev_gt, prev_sub);
        if (!ok) break;
        tc_commit(smem_u32(&sh.acc_full));
        ++it;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue groups
    const int wg = (warp - 4) >> 2;
    const int tid_wg = (threadIdx.x - 128) & 127;
    const int row = ((warp & 3) << 5) | lane;
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const float c1 = 0.5f * a.alpha;
    uint32_t gt = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
      const int2 w = items[item];
      if (w.x < 0) continue;
      const int b = w.x & 0xffff, head = w.x >> 16, qblk = w.y;
      const SeqInfo s = load_seq(a, b);
      const int m0 = qblk * BLK, m = m0 + row;
      // ---- A operands straight from global memory into TMEM: group 0 loads Q, group 1 loads dO.
      // (the previous item's MMAs are complete: both groups waited for its accumulator)
      {
        const unsigned short* src = wg == 0
            ? reinterpret_cast<const unsigned short*>(a.q) + (s.start + m) * a.q_rs + head * HEAD_DIM
            : reinterpret_cast<const unsigned short*>(a.d_o) + (s.start + m) * a.do_rs + head * HEAD_DIM;
        const uint32_t dst = tmem + lane_addr + (wg == 0 ? DQ_QA : DQ_DOA);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if (m < s.len) x = __ldg(reinterpret_cast<const uint4*>(src) + c * 4 + j);
            r[4 * j + 0] = x.x; r[4 * j + 1] = x.y; r[4 * j + 2] = x.z; r[4 * j + 3] = x.w;
          }
          tmem_st16(dst + c * 16, r);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&sh.a_ready));
      }
      const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
      for (int idx = 0; idx < kr.count() && ok; ++idx) {
        const int nb = kr.at(idx);
        const int cls = classify_tile(m0, nb * BLK, s, a.mask);
        if (cls == TILE_SKIP) continue;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.s_full[wg]), gt & 1, abort_flag, a.status, WAIT_EPILOGUE));
        if (!ok) break;
        tc_fence_after();
        const uint32_t s_addr = tmem + lane_addr + DQ_S0 + wg * 64;
        const uint32_t dp_addr = tmem + lane_addr + DQ_DP0 + wg * 64;
        const int nbase = nb * BLK + wg * 64;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t sv[32], dpv[32], pk[16];
          tmem_ld32(s_addr + half * 32, sv);
          tmem_ld32(dp_addr + half * 32, dpv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float p0, g0, p1, g1;
            silu_terms(__uint_as_float(sv[2 * i]), c1, p0, g0);
            silu_terms(__uint_as_float(sv[2 * i + 1]), c1, p1, g1);
            float d0 = __uint_as_float(dpv[2 * i]) * g0;
            float d1 = __uint_as_float(dpv[2 * i + 1]) * g1;
            if (cls == TILE_PARTIAL) {
              const int n = nbase + half * 32 + 2 * i;
              if (!(m < s.len && n < s.len && keep(m, n, s, a.mask))) d0 = 0.f;
              if (!(m < s.len && n + 1 < s.len && keep(m, n + 1, s, a.mask))) d1 = 0.f;
            }
            pk[i] = pack2<IS_BF16>(d0, d1);
          }
          tmem_st16(dp_addr + half * 16, pk);
        }
        if (nb * BLK + BLK > s.len) {
          // key rows past the sequence end feed the dQ MMA as B rows: clear them (0 * NaN = NaN)
          zero_tile_half_row(sh.k[gt % DQ_STAGES], s.len - nb * BLK, wg * 64 + (tid_wg & 63), tid_wg >> 6);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&sh.ds_ready[wg]));
        ++gt;
      }
      if (!ok) break;
      // ---- dQ leaves TMEM: group wg converts columns [64*wg, 64*wg+64) of its row
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.acc_full), it & 1, abort_flag, a.status, WAIT_EPILOGUE));
      if (!ok) break;
      tc_fence_after();
      uint32_t ov0[32], ov1[32];
      tmem_ld32(tmem + lane_addr + DQ_ACC + wg * 64, ov0);
      tmem_ld32(tmem + lane_addr + DQ_ACC + wg * 64 + 32, ov1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(smem_u32(&sh.acc_empty));
      if (m < s.len) {
        const float sc = 0.5f * a.alpha * row_scale(a, s.start + m);
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<unsigned short*>(a.dq) + (s.start + m) * a.dq_rs +
                                              head * HEAD_DIM + wg * 64);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 x;
          x.x = pack2<IS_BF16>(__uint_as_float(ov0[8 * j + 0]) * sc, __uint_as_float(ov0[8 * j + 1]) * sc);
          x.y = pack2<IS_BF16>(__uint_as_float(ov0[8 * j + 2]) * sc, __uint_as_float(ov0[8 * j + 3]) * sc);
          x.z = pack2<IS_BF16>(__uint_as_float(ov0[8 * j + 4]) * sc, __uint_as_float(ov0[8 * j + 5]) * sc);
          x.w = pack2<IS_BF16>(__uint_as_float(ov0[8 * j + 6]) * sc, __uint_as_float(ov0[8 * j + 7]) * sc);
          dst[j] = x;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 x;
          x.x = pack2<IS_BF16>(__uint_as_float(ov1[8 * j + 0]) * sc, __uint_as_float(ov1[8 * j + 1]) * sc);
          x.y = pack2<IS_BF16>(__uint_as_float(ov1[8 * j + 2]) * sc, __uint_as_float(ov1[8 * j + 3]) * sc);
          x.z = pack2<IS_BF16>(__uint_as_float(ov1[8 * j + 4]) * sc, __uint_as_float(ov1[8 * j + 5]) * sc);
          x.w = pack2<IS_BF16>(__uint_as_float(ov1[8 * j + 6]) * sc, __uint_as_float(ov1[8 * j + 7]) * sc);
          dst[4 + j] = x;
        }
      }
      ++it;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    if (*abort_flag) {
      const unsigned long long t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
    }
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------
// dK/dV pass
// ------------------------------------------------------------------------------------
constexpr int KV_STAGES = 2;
constexpr int KV_ST0 = 0, KV_DPT0 = 128, KV_DK = 256, KV_DV = 384;  // ST1 = ST0 + 64, DPT1 = DPT0 + 64

struct DkvShared {
  unsigned char k[TILE_BYTES];
  unsigned char v[TILE_BYTES];
  unsigned char q[KV_STAGES][TILE_BYTES];
  unsigned char d_o[KV_STAGES][TILE_BYTES];
  unsigned long long kv_full, kv_empty;
  unsigned long long qd_full[KV_STAGES], qd_empty[KV_STAGES];
  unsigned long long s_full[2], p_ready[2], acc_full, acc_empty;
  uint32_t tmem_base;
  int abort_flag;
};

template <bool IS_BF16>
__global__ void __launch_bounds__(BWD_THREADS, 1)
hstu_bwd_dkv_tc(const __grid_constant__ MapsBwd maps, KernelArgs a, const int* __restrict__ ws, long long off_items) {
  extern __shared__ unsigned char smem_raw[];
  DkvShared& sh = *reinterpret_cast<DkvShared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = ws[0];
  if (static_cast<int>(blockIdx.x) >= total_items) return;
  const int2* items = reinterpret_cast<const int2*>(ws + off_items);
  volatile int* abort_flag = &sh.abort_flag;

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    mbar_init(smem_u32(&sh.kv_full), 1);
    mbar_init(smem_u32(&sh.kv_empty), 1);
    for (int i = 0; i < KV_STAGES; ++i) { mbar_init(smem_u32(&sh.qd_full[i]), 1); mbar_init(smem_u32(&sh.qd_empty[i]), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(smem_u32(&sh.s_full[i]), 1); mbar_init(smem_u32(&sh.p_ready[i]), 128); }
    mbar_init(smem_u32(&sh.acc_full), 1);
    mbar_init(smem_u32(&sh.acc_empty), 256);
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
    if (lane == 0) {
      prefetch_tensormap(&maps.q);
      prefetch_tensormap(&maps.k);
      prefetch_tensormap(&maps.v);
      prefetch_tensormap(&maps.d_o);
      uint32_t gt = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const int2 w = items[item];
        if (w.x < 0) continue;
        const int b = w.x & 0xffff, head = w.x >> 16;
        const SeqInfo s = load_seq(a, b);
        const int kvblk = (s.len + BLK - 1) / BLK - 1 - w.y;
        const int n0 = kvblk * BLK, col0 = head * HEAD_DIM;
        const int krow = static_cast<int>(s.start) + n0;
        ok = mbar_wait(smem_u32(&sh.kv_empty), (it & 1) ^ 1, abort_flag, a.status, WAIT_PRODUCER);
        if (!ok) break;
        mbar_arrive_expect_tx(smem_u32(&sh.kv_full), 2 * TILE_BYTES);
        tma_load_2d(smem_u32(sh.k), &maps.k, smem_u32(&sh.kv_full), col0, krow);
        tma_load_2d(smem_u32(sh.k) + HALF_TILE_BYTES, &maps.k, smem_u32(&sh.kv_full), col0 + 64, krow);
        tma_load_2d(smem_u32(sh.v), &maps.v, smem_u32(&sh.kv_full), col0, krow);
        tma_load_2d(smem_u32(sh.v) + HALF_TILE_BYTES, &maps.v, smem_u32(&sh.kv_full), col0 + 64, krow);
        const BlockRange qr = query_blocks_for_key_block(n0, s, a.mask);
        for (int idx = 0; idx < qr.count() && ok; ++idx) {
          const int qb = qr.at(idx);
          if (classify_tile(qb * BLK, n0, s, a.mask) == TILE_SKIP) continue;
          const int qrow = static_cast<int>(s.start) + qb * BLK;
          const uint32_t st = gt % KV_STAGES, ph = (gt / KV_STAGES) & 1;
          ok = mbar_wait(smem_u32(&sh.qd_empty[st]), ph ^ 1, abort_flag, a.status, WAIT_PRODUCER);
          if (!ok) break;
          mbar_arrive_expect_tx(smem_u32(&sh.qd_full[st]), 2 * TILE_BYTES);
          tma_load_2d(smem_u32(sh.q[st]), &maps.q, smem_u32(&sh.qd_full[st]), col0, qrow);
          tma_load_2d(smem_u32(sh.q[st]) + HALF_TILE_BYTES, &maps.q, smem_u32(&sh.qd_full[st]), col0 + 64, qrow);
          tma_load_2d(smem_u32(sh.d_o[st]), &maps.d_o, smem_u32(&sh.qd_full[st]), col0, qrow);
          tma_load_2d(smem_u32(sh.d_o[st]) + HALF_TILE_BYTES, &maps.d_o, smem_u32(&sh.qd_full[st]), col0 + 64, qrow);
          ++gt;
        }
        ++it;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_f16(IS_BF16 ? 1 : 0, BLK, 64, 0, 0);          // K/V (K-major) x Q/dO half (K-major)
      constexpr uint32_t IDESC_ACC = idesc_f16(IS_BF16 ? 1 : 0, BLK, HEAD_DIM, 0, 1);  // P^T/dS^T (TMEM) x dO/Q half (N-major)
      uint32_t gt = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const int2 w = items[item];
        if (w.x < 0) continue;
        const int b = w.x & 0xffff;
        const SeqInfo s = load_seq(a, b);
        const int kvblk = (s.len + BLK - 1) / BLK - 1 - w.y;
        const int n0 = kvblk * BLK;
        ok = mbar_wait(smem_u32(&sh.kv_full), it & 1, abort_flag, a.status, WAIT_MMA);
        if (!ok) break;
        tc_fence_after();
        bool have_prev = false;
        uint32_t prev_gt = 0, prev_sub = 0, n_acc = 0;
        auto issue_acc = [&](uint32_t pgt, uint32_t psub) -> bool {
          if (!mbar_wait(smem_u32(&sh.p_ready[psub]), pgt & 1, abort_flag, a.status, WAIT_MMA)) return false;
          if (n_acc == 0 && !mbar_wait(smem_u32(&sh.acc_empty), (it & 1) ^ 1, abort_flag, a.status, WAIT_MMA))
            return false;
          tc_fence_after();
          const uint32_t st = pgt % KV_STAGES;
          const uint32_t dobase = smem_u32(sh.d_o[st]) + psub * SUBTILE_BYTES;
          const uint32_t qbase = smem_u32(sh.q[st]) + psub * SUBTILE_BYTES;
          const uint32_t acc = (n_acc > 0) ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + KV_DV, tmem + KV_ST0 + psub * 64 + kk * 8,
                   smem_desc_sw128(dobase + kk * 2048, HALF_TILE_BYTES, 1024), IDESC_ACC, (acc || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + KV_DK, tmem + KV_DPT0 + psub * 64 + kk * 8,
                   smem_desc_sw128(qbase + kk * 2048, HALF_TILE_BYTES, 1024), IDESC_ACC, (acc || kk > 0) ? 1u : 0u);
          if (psub == 1) tc_commit(smem_u32(&sh.qd_empty[st]));
          ++n_acc;
          return true;
        };
        const BlockRange qr = query_blocks_for_key_block(n0, s, a.mask);
        const uint32_t kb = smem_u32(sh.k), vb = smem_u32(sh.v);
        for (int idx = 0; idx < qr.count() && ok; ++idx) {
          const int qb = qr.at(idx);
          if (classify_tile(qb * BLK, n0, s, a.mask) == TILE_SKIP) continue;
          const uint32_t st = gt % KV_STAGES, ph = (gt / KV_STAGES) & 1;
          ok = mbar_wait(smem_u32(&sh.qd_full[st]), ph, abort_flag, a.status, WAIT_MMA);
          if (!ok) break;
          tc_fence_after();
          for (uint32_t sub = 0; sub < 2 && ok; ++sub) {
            const uint32_t qbase = smem_u32(sh.q[st]) + sub * SUBTILE_BYTES;
            const uint32_t dobase = smem_u32(sh.d_o[st]) + sub * SUBTILE_BYTES;
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
              mma_ss(tmem + KV_ST0 + sub * 64, smem_desc_sw128(kb + kstep_offset(kk), 16, 1024),
                     smem_desc_sw128(qbase + kstep_offset(kk), 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
              mma_ss(tmem + KV_DPT0 + sub * 64, smem_desc_sw128(vb + kstep_offset(kk), 16, 1024),
                     smem_desc_sw128(dobase + kstep_offset(kk), 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
            tc_commit(smem_u32(&sh.s_full[sub]));
            if (have_prev) ok = issue_acc(prev_gt, prev_sub);
            prev_gt = gt; prev_sub = sub; have_prev = true;
          }
          if (!ok) break;
          ++gt;
        }
        if (!ok) break;
        tc_commit(smem_u32(&sh.kv_empty));  // every score MMA of this item has been issued
        if (have_prev) ok = issue_acc(prev_gt, prev_sub);
        if (!ok) break;
        tc_commit(smem_u32(&sh.acc_full));
        ++it;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue groups
    const int wg = (warp - 4) >> 2;
    const int tid_wg = (threadIdx.x - 128) & 127;
    const int row = ((warp & 3) << 5) | lane;  // key row inside the block
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const float c1 = 0.5f * a.alpha;
    const bool per_token = a.scale_mode == 2;
    uint32_t gt = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
      const int2 w = items[item];
      if (w.x < 0) continue;
      const int b = w.x & 0xffff, head = w.x >> 16;
      const SeqInfo s = load_seq(a, b);
      const int kvblk = (s.len + BLK - 1) / BLK - 1 - w.y;
      const int n0 = kvblk * BLK, n = n0 + row;
      const BlockRange qr = query_blocks_for_key_block(n0, s, a.mask);
      for (int idx = 0; idx < qr.count() && ok; ++idx) {
        const int qb = qr.at(idx);
        const int cls = classify_tile(qb * BLK, n0, s, a.mask);
        if (cls == TILE_SKIP) continue;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.s_full[wg]), gt & 1, abort_flag, a.status, WAIT_EPILOGUE));
        if (!ok) break;
        tc_fence_after();
        const uint32_t st_addr = tmem + lane_addr + KV_ST0 + wg * 64;
        const uint32_t dp_addr = tmem + lane_addr + KV_DPT0 + wg * 64;
        const int mbase = qb * BLK + wg * 64;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t sv[32], dpv[32], pp[16], pd[16];
          tmem_ld32(st_addr + half * 32, sv);
          tmem_ld32(dp_addr + half * 32, dpv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float p0, g0, p1, g1;
            silu_terms(__uint_as_float(sv[2 * i]), c1, p0, g0);
            silu_terms(__uint_as_float(sv[2 * i + 1]), c1, p1, g1);
            float d0 = __uint_as_float(dpv[2 * i]) * g0;
            float d1 = __uint_as_float(dpv[2 * i + 1]) * g1;
            const int mm = mbase + half * 32 + 2 * i;
            if (per_token) {  // one scale per query token = per column here
              const float s0 = mm < s.len ? __ldg(a.attn_scale + s.start + mm) : 0.f;
              const float s1 = mm + 1 < s.len ? __ldg(a.attn_scale + s.start + mm + 1) : 0.f;
              p0 *= s0; d0 *= s0; p1 *= s1; d1 *= s1;
            }
            if (cls == TILE_PARTIAL) {
              const bool k0 = n < s.len && mm < s.len && keep(mm, n, s, a.mask);
              const bool k1 = n < s.len && mm + 1 < s.len && keep(mm + 1, n, s, a.mask);
              if (!k0) { p0 = 0.f; d0 = 0.f; }
              if (!k1) { p1 = 0.f; d1 = 0.f; }
            }
            pp[i] = pack2<IS_BF16>(p0, p1);
            pd[i] = pack2<IS_BF16>(d0, d1);
          }
          tmem_st16(st_addr + half * 16, pp);
          tmem_st16(dp_addr + half * 16, pd);
        }
        if (qb * BLK + BLK > s.len) {
          // query rows past the sequence end are B rows of the dV / dK MMAs: clear them
          const int r = wg * 64 + (tid_wg & 63);
          zero_tile_half_row(sh.q[gt % KV_STAGES], s.len - qb * BLK, r, tid_wg >> 6);
          zero_tile_half_row(sh.d_o[gt % KV_STAGES], s.len - qb * BLK, r, tid_wg >> 6);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&sh.p_ready[wg]));
        ++gt;
      }
      if (!ok) break;
      // ---- accumulators leave TMEM: group 0 writes dK, group 1 writes dV (128 columns each)
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.acc_full), it & 1, abort_flag, a.status, WAIT_EPILOGUE));
      if (!ok) break;
      tc_fence_after();
      const float scal = per_token ? 1.f : row_scale(a, 0);
      const float sc = wg == 0 ? 0.5f * a.alpha * scal : scal;
      unsigned short* outp = wg == 0 ? reinterpret_cast<unsigned short*>(a.dk) + (s.start + n) * a.dk_rs
                                     : reinterpret_cast<unsigned short*>(a.dv) + (s.start + n) * a.dv_rs;
      uint4* dst = reinterpret_cast<uint4*>(outp + head * HEAD_DIM);
      const uint32_t acc_addr = tmem + lane_addr + (wg == 0 ? KV_DK : KV_DV);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ov[32];
        tmem_ld32(acc_addr + c * 32, ov);
        tmem_wait_ld();
        if (c == 3) {
          tc_fence_before();
          mbar_arrive(smem_u32(&sh.acc_empty));
        }
        if (n < s.len) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 x;
            x.x = pack2<IS_BF16>(__uint_as_float(ov[8 * j + 0]) * sc, __uint_as_float(ov[8 * j + 1]) * sc);
            x.y = pack2<IS_BF16>(__uint_as_float(ov[8 * j + 2]) * sc, __uint_as_float(ov[8 * j + 3]) * sc);
            x.z = pack2<IS_BF16>(__uint_as_float(ov[8 * j + 4]) * sc, __uint_as_float(ov[8 * j + 5]) * sc);
            x.w = pack2<IS_BF16>(__uint_as_float(ov[8 * j + 6]) * sc, __uint_as_float(ov[8 * j + 7]) * sc);
            dst[c * 4 + j] = x;
          }
        }
      }
      ++it;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    if (*abort_flag) {
      const unsigned long long t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
    }
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace
}  // namespace tc

cudaError_t tc_backward(const KernelArgs& a, int dtype, void* workspace, cudaStream_t st) {
  using namespace tc;
  const bool bf16 = dtype == B200_HSTU_BF16;
  const WorkspaceLayout w = workspace_layout(a.T, a.B, a.H);
  int* ws = reinterpret_cast<int*>(workspace);
  MapsBwd maps;
  const long long width = (long long)a.H * HEAD_DIM;
  if (!make_map(&maps.q, a.q, a.T, width, a.q_rs, bf16) || !make_map(&maps.k, a.k, a.T, width, a.k_rs, bf16) ||
      !make_map(&maps.v, a.v, a.T, width, a.v_rs, bf16) || !make_map(&maps.d_o, a.d_o, a.T, width, a.do_rs, bf16))
    return cudaErrorInvalidValue;
  cudaError_t e = launch_prep(a, bf16, ws, w, true, st);
  if (e != cudaSuccess) return e;
  long long grid = w.max_items < sm_count() ? w.max_items : sm_count();
  if (grid < 1) grid = 1;
  {
    const size_t smem = sizeof(DkvShared) + 1024;
    auto kern = bf16 ? hstu_bwd_dkv_tc<true> : hstu_bwd_dkv_tc<false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(grid), BWD_THREADS, smem, st>>>(maps, a, ws, w.off_items);
  }
  {
    const size_t smem = sizeof(DqShared) + 1024;
    auto kern = bf16 ? hstu_bwd_dq_tc<true> : hstu_bwd_dq_tc<false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(grid), BWD_THREADS, smem, st>>>(maps, a, ws, w.off_items);
  }
  return cudaGetLastError();
}

}  // namespace hstu
