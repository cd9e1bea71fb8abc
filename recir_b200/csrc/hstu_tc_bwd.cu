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
// 512 TMEM columns; epilogue group w owns half w of every tile.
// With u = (alpha/2) s and t = tanh(u):  x sigma(x) = u t + u  and
// silu'(x) = 0.5 (1 + t)(1 + u (1 - t)); the 0.5, alpha and a scalar attn_scale are applied
// once per output row when the accumulator leaves TMEM.
//
// Warp roles (384 threads): warp 0 = TMA producer and tile scheduler, warp 1 = MMA issuer
// (both walk their loops warp-uniformly, one elected lane issues), warps 4-11 = two epilogue
// groups.  Registers are moved from warps 0-3 to the epilogue warps (setmaxnreg).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdlib.h>

#include "hstu_launch.h"
#include "hstu_tc_common.cuh"
#include "hstu_tc_host.h"

namespace hstu {
namespace tc {
namespace {

using namespace sm100;

constexpr int BWD_THREADS = 384;
constexpr int TMEM_COLS = 512;
constexpr int META_RING = 16;

// Optional cycle accounting (PROF): per-role wait/busy cycles, summed over CTAs into workspace ints 2..15.
enum { PB_MMA_TOTAL = 0, PB_MMA_WAIT_LOAD, PB_MMA_WAIT_P, PB_MMA_WAIT_ACC, PB_MMA_WAIT_ITEM, PB_EPI_TOTAL,
       PB_EPI_WAIT_S, PB_EPI_WAIT_ACC, PB_EPI_TILE, PB_EPI_DRAIN, PB_EPI_LD, PB_EPI_ST, PB_PROD_WAIT, PB_PROD_TOTAL };
constexpr int TRACE_SLOTS = 8192;
template <bool PROF>
__device__ __forceinline__ void trace_event(int* status, int slot_base, int idx, int ev, int n_ev) {
  if (PROF && status != nullptr && blockIdx.x == 0) {
    const int slot = slot_base + idx * n_ev + ev;
    if (slot < TRACE_SLOTS) status[16 + slot] = static_cast<int>(clock64());
  }
}

template <bool PROF>
struct Stopwatch {
  long long t;
  __device__ __forceinline__ void start() { if (PROF) t = clock64(); }
  __device__ __forceinline__ void stop(long long& acc) { if (PROF) acc += clock64() - t; }
};

struct MapsBwd {
  CUtensorMap q, k, v, d_o;
  CUtensorMap dq, dk, dv;  // outputs (bulk stores of whole 128-row blocks)
  CUtensorMap ds;          // stored dS^T tiles as one [tiles * 128, 128] matrix (dQ pass from stored tiles only)
};

// low-word offset (16-byte units) of k-step kk inside a K-major tile: 32 bytes inside a
// 64-column box, boxes 16 KB apart
__device__ __forceinline__ constexpr uint32_t kstep_lo(int kk) { return (kk >> 2) * (HALF_TILE_BYTES >> 4) + (kk & 3) * 2; }

// P and dS for two scores with packed 16-bit math (one MUFU operation for the pair).
//   u = (alpha/2) s, t = tanh(u);  p = u t + u;  2 silu'(x) = (1 + t)(1 + u (1 - t));  ds = dp * 2 silu'
template <bool IS_BF16, bool WANT_P>
__device__ __forceinline__ void bwd_pair(uint32_t s0, uint32_t s1, uint32_t dp0, uint32_t dp1, uint64_t c1, uint32_t& p2,
                                         uint32_t& ds2) {
  float u0, u1;
  mul_f32x2(s0, s1, c1, u0, u1);
  const uint32_t u2 = pack2<IS_BF16>(u0, u1);
  const uint32_t t2 = tanh2<IS_BF16>(u2);
  if (WANT_P) p2 = fma2<IS_BF16>(u2, t2, u2);
  const uint32_t w1 = add2<IS_BF16>(t2, one2<IS_BF16>());
  const uint32_t w2 = add2<IS_BF16>(fma2<IS_BF16>(neg2<IS_BF16>(u2), t2, u2), one2<IS_BF16>());
  const uint32_t d2 = pack2<IS_BF16>(__uint_as_float(dp0), __uint_as_float(dp1));
  ds2 = mul2<IS_BF16>(d2, mul2<IS_BF16>(w1, w2));
}

// 32 score columns -> 16 packed pairs of dS (and P).  Branch-free inside: the mask and the
// per-token scale are compile-time variants, so the 16 pairs interleave freely.
template <bool IS_BF16, bool WANT_P, bool MASKED>
__device__ __forceinline__ void bwd_chunk(const uint32_t (&sv)[32], const uint32_t (&dpv)[32], uint32_t (&pp)[16],
                                          uint32_t (&pd)[16], uint64_t c1, uint32_t bits) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t p2 = 0u, d2;
    bwd_pair<IS_BF16, WANT_P>(sv[2 * i], sv[2 * i + 1], dpv[2 * i], dpv[2 * i + 1], c1, p2, d2);
    if (MASKED) {
      const uint32_t pm = pair_mask(bits, 2 * i);
      if (WANT_P) p2 &= pm;
      d2 &= pm;
    }
    if (WANT_P) pp[i] = p2;
    pd[i] = d2;
  }
}

// Multiplies 16 packed pairs by one fp32 scale per column (scales of columns col0 .. col0 + 31).
template <bool IS_BF16>
__device__ __forceinline__ void scale_chunk(uint32_t (&x)[16], const float* scales, long long first, int col0, int len) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = col0 + 2 * i;
    const float s0 = c < len ? __ldg(scales + first + c) : 0.f;
    const float s1 = c + 1 < len ? __ldg(scales + first + c + 1) : 0.f;
    x[i] = mul2<IS_BF16>(x[i], pack2<IS_BF16>(s0, s1));
  }
}

// Bitmap of the kept rows among the 64 query rows [mbase, mbase + 64) for a column mask.
__device__ __forceinline__ unsigned long long col_mask_bits64(const ColMask& cm, int len, int mbase) {
  auto range = [&](int lo, int hi) -> unsigned long long {
    lo -= mbase; hi -= mbase;
    lo = lo < 0 ? 0 : (lo > 64 ? 64 : lo);
    hi = hi < 0 ? 0 : (hi > 64 ? 64 : hi);
    if (hi <= lo) return 0ull;
    const unsigned long long below_hi = hi >= 64 ? ~0ull : ((1ull << hi) - 1ull);
    const unsigned long long below_lo = (1ull << lo) - 1ull;  // lo < 64 here
    return below_hi & ~below_lo;
  };
  unsigned long long bits = range(cm.a_lo, cm.a_hi) | range(cm.b_lo, len);
  const int d = cm.diag - mbase;
  if (cm.diag >= 0 && d >= 0 && d < 64) bits |= 1ull << d;
  return bits;
}

// Writes this thread's 64 accumulator columns (two 32-column register blocks, scaled) as one
// 128-byte row of a staging half tile; chunk index XOR (row & 7) spreads the banks.
template <bool IS_BF16>
__device__ __forceinline__ void stage_row64(unsigned char* half_tile, int row, const uint32_t (&v0)[32],
                                            const uint32_t (&v1)[32], float sc) {
  unsigned char* my_row = half_tile + row * 128;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 x;
    x.x = pack2<IS_BF16>(__uint_as_float(v0[8 * j + 0]) * sc, __uint_as_float(v0[8 * j + 1]) * sc);
    x.y = pack2<IS_BF16>(__uint_as_float(v0[8 * j + 2]) * sc, __uint_as_float(v0[8 * j + 3]) * sc);
    x.z = pack2<IS_BF16>(__uint_as_float(v0[8 * j + 4]) * sc, __uint_as_float(v0[8 * j + 5]) * sc);
    x.w = pack2<IS_BF16>(__uint_as_float(v0[8 * j + 6]) * sc, __uint_as_float(v0[8 * j + 7]) * sc);
    *reinterpret_cast<uint4*>(my_row + ((j ^ (row & 7)) << 4)) = x;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 x;
    x.x = pack2<IS_BF16>(__uint_as_float(v1[8 * j + 0]) * sc, __uint_as_float(v1[8 * j + 1]) * sc);
    x.y = pack2<IS_BF16>(__uint_as_float(v1[8 * j + 2]) * sc, __uint_as_float(v1[8 * j + 3]) * sc);
    x.z = pack2<IS_BF16>(__uint_as_float(v1[8 * j + 4]) * sc, __uint_as_float(v1[8 * j + 5]) * sc);
    x.w = pack2<IS_BF16>(__uint_as_float(v1[8 * j + 6]) * sc, __uint_as_float(v1[8 * j + 7]) * sc);
    *reinterpret_cast<uint4*>(my_row + (((4 + j) ^ (row & 7)) << 4)) = x;
  }
}

// Copies a staged half tile (128 rows x 64 columns) to global memory: 8 lanes write one
// 128-byte row segment, a warp writes 4 rows per instruction.  dst points at (row 0, column 0).
__device__ __forceinline__ void store_staged64(const unsigned char* half_tile, unsigned short* dst, long long row_stride,
                                               int rows_valid, int tid_wg) {
  const int chunk = tid_wg & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 16 + (tid_wg >> 3);
    if (r < rows_valid) {
      const uint4 x = *reinterpret_cast<const uint4*>(half_tile + r * 128 + ((chunk ^ (r & 7)) << 4));
      *reinterpret_cast<uint4*>(dst + static_cast<long long>(r) * row_stride + chunk * 8) = x;
    }
  }
}

__device__ __forceinline__ void group_barrier(int wg) { asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory"); }

// ------------------------------------------------------------------------------------
// dQ pass
// ------------------------------------------------------------------------------------
constexpr int DQ_STAGES = 2;
constexpr int DQ_QA = 0, DQ_DOA = 64, DQ_S0 = 128, DQ_DP0 = 256, DQ_ACC = 384;  // S1 = S0 + 64, DP1 = DP0 + 64

struct DqShared {
  unsigned char k[DQ_STAGES][TILE_BYTES];
  unsigned char v[DQ_STAGES][TILE_BYTES];
  unsigned char q[TILE_BYTES];    // Q and dO tiles of the NEXT work item (TMA), copied row by row into
  unsigned char d_o[TILE_BYTES];  // TMEM when that item starts
  unsigned char stage[TILE_BYTES];
  unsigned long long qd_full, qd_empty;
  unsigned long long k_full[DQ_STAGES], k_empty[DQ_STAGES];
  unsigned long long v_full[DQ_STAGES], v_empty[DQ_STAGES];
  unsigned long long a_ready, s_full[2], ds_ready[2], acc_full, acc_empty;
  int meta[META_RING];
  ItemRing ring;
  uint32_t tmem_base;
  int abort_flag;
};

template <bool IS_BF16, bool PROF>
__global__ void __launch_bounds__(BWD_THREADS, 1)
hstu_bwd_dq_tc(const __grid_constant__ MapsBwd maps, KernelArgs a, int* __restrict__ ws, long long off_items) {
  extern __shared__ unsigned char smem_raw[];
  DqShared& sh = *reinterpret_cast<DqShared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = ws[0];
  if (static_cast<int>(blockIdx.x) >= total_items) {
    grid_dependency_wait();  // see the end of the kernel
    return;
  }
  const int2* items = reinterpret_cast<const int2*>(ws + off_items);
  volatile int* abort_flag = &sh.abort_flag;

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    item_ring_init(sh.ring);
    for (int i = 0; i < DQ_STAGES; ++i) {
      mbar_init(smem_u32(&sh.k_full[i]), 1); mbar_init(smem_u32(&sh.k_empty[i]), 1);
      mbar_init(smem_u32(&sh.v_full[i]), 1); mbar_init(smem_u32(&sh.v_empty[i]), 1);
    }
    mbar_init(smem_u32(&sh.a_ready), 256);
    mbar_init(smem_u32(&sh.qd_full), 1);
    mbar_init(smem_u32(&sh.qd_empty), 256);
    for (int i = 0; i < 2; ++i) { mbar_init(smem_u32(&sh.s_full[i]), 1); mbar_init(smem_u32(&sh.ds_ready[i]), 256); }
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
  if (warp < 4) setmaxnreg_dec<120>(); else setmaxnreg_inc<184>();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer / tile scheduler
    if (lane == 0) {
      prefetch_tensormap(&maps.k); prefetch_tensormap(&maps.v);
      prefetch_tensormap(&maps.q); prefetch_tensormap(&maps.d_o);
    }
    uint32_t gt = 0, st = 0, ph = 0, pit = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_PRODUCER));
    };
    int2 w;
    SeqInfo s;
    uint32_t todo0 = 0u, full0 = 0u;
    for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w, s, todo0, full0, ok, abort_flag, a.status, WAIT_PRODUCER); ++n_item) {
      const int head = w.x >> 16, qblk = w.y;
      const int m0 = qblk * BLK, col0 = head * HEAD_DIM;
      {
        // Q and dO rows of this item: the buffer is free as soon as the previous item's rows have
        // been copied into TMEM, i.e. early in the previous item, so this load is a prefetch
        const int qrow = static_cast<int>(s.start) + m0;
        ok = wait_all(&sh.qd_empty, (pit & 1) ^ 1);
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(smem_u32(&sh.qd_full), 2 * TILE_BYTES);
          tma_load_2d(smem_u32(sh.q), &maps.q, smem_u32(&sh.qd_full), col0, qrow);
          tma_load_2d(smem_u32(sh.q) + HALF_TILE_BYTES, &maps.q, smem_u32(&sh.qd_full), col0 + 64, qrow);
          tma_load_2d(smem_u32(sh.d_o), &maps.d_o, smem_u32(&sh.qd_full), col0, qrow);
          tma_load_2d(smem_u32(sh.d_o) + HALF_TILE_BYTES, &maps.d_o, smem_u32(&sh.qd_full), col0 + 64, qrow);
        }
        __syncwarp();
        ++pit;
      }
      const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
      const int cnt = kr.count();
      // the last candidate (diagonal block, or last block of the sequence) is never skipped
      for (int base = 0; base < cnt && ok; base += 32) {
        uint32_t todo = todo0;  // the scheduler warp classified the first 32 candidates
        if (base > 0) {
          int my_cls = TILE_SKIP;
          if (base + lane < cnt) my_cls = classify_tile(m0, kr.at(base + lane) * BLK, s, a.mask, true);
          todo = __ballot_sync(0xffffffffu, my_cls != TILE_SKIP);
        }
        while (todo != 0u && ok) {
          const int bit = __ffs(todo) - 1;
          todo &= todo - 1;
          const int idx = base + bit;
          const int krow = static_cast<int>(s.start) + kr.at(idx) * BLK;
          // V first: its stage is released when the tile's last dP MMA has run, half a tile before the
          // K stage (which the dQ MMAs still read), so its copy is already under way when K's can start
          ok = wait_all(&sh.v_empty[st], ph ^ 1);
          if (!ok) break;
          if (elect_one()) {
            mbar_arrive_expect_tx(smem_u32(&sh.v_full[st]), TILE_BYTES);
            tma_load_2d(smem_u32(sh.v[st]), &maps.v, smem_u32(&sh.v_full[st]), col0, krow);
            tma_load_2d(smem_u32(sh.v[st]) + HALF_TILE_BYTES, &maps.v, smem_u32(&sh.v_full[st]), col0 + 64, krow);
          }
          __syncwarp();
          ok = wait_all(&sh.k_empty[st], ph ^ 1);
          if (!ok) break;
          if (elect_one()) {
            sh.meta[gt & (META_RING - 1)] = (idx == cnt - 1) ? 1 : 0;
            mbar_arrive_expect_tx(smem_u32(&sh.k_full[st]), TILE_BYTES);
            tma_load_2d(smem_u32(sh.k[st]), &maps.k, smem_u32(&sh.k_full[st]), col0, krow);
            tma_load_2d(smem_u32(sh.k[st]) + HALF_TILE_BYTES, &maps.k, smem_u32(&sh.k_full[st]), col0 + 64, krow);
          }
          __syncwarp();
          ++gt;
          if (++st == DQ_STAGES) { st = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC_S = idesc_f16(IS_BF16 ? 1 : 0, BLK, 64, 0, 0);          // A (TMEM) x K/V half (K-major)
    constexpr uint32_t IDESC_ACC = idesc_f16(IS_BF16 ? 1 : 0, BLK, HEAD_DIM, 0, 1);  // dS (TMEM) x K half (N-major)
    constexpr uint32_t HI = desc_hi_sw128(1024);
    const uint32_t k_lo0 = desc_lo_sw128(smem_u32(sh.k[0]), 16);
    const uint32_t v_lo0 = desc_lo_sw128(smem_u32(sh.v[0]), 16);
    const uint32_t kn_lo0 = desc_lo_sw128(smem_u32(sh.k[0]), HALF_TILE_BYTES);  // K as N-major operand
    uint32_t gt = 0, it = 0, st = 0, ph = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_MMA));
    };
    int2 w_unused;
    SeqInfo s_unused;
    uint32_t t_unused = 0u, f_unused = 0u;
    for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w_unused, s_unused, t_unused, f_unused, ok, abort_flag, a.status, WAIT_MMA); ++n_item) {
      ok = wait_all(&sh.a_ready, it & 1);
      if (!ok) break;
      tc_fence_after();
      bool have_prev = false;
      uint32_t prev_gt = 0, prev_sub = 0, prev_st = 0, n_acc = 0;
      auto issue_acc = [&](uint32_t pgt, uint32_t psub, uint32_t pst) -> bool {
        if (!wait_all(&sh.ds_ready[psub], pgt & 1)) return false;
        if (n_acc == 0 && !wait_all(&sh.acc_empty, (it & 1) ^ 1)) return false;
        if (lane == 0) trace_event<PROF>(a.trace_buf, 0, 2 * pgt + psub, 2, 4);
        tc_fence_after();
        const uint32_t kn_lo = kn_lo0 + pst * (TILE_BYTES >> 4) + psub * (SUBTILE_BYTES >> 4);
        const uint32_t ds_tmem = tmem + DQ_DP0 + psub * 64;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            // dS of keys 0..31 of the half tile sits at columns 0..15, keys 32..63 at columns 32..47
            mma_ts(tmem + DQ_ACC, ds_tmem + (kk >> 1) * 32 + (kk & 1) * 8, desc_join(kn_lo + kk * (2048 >> 4), HI), IDESC_ACC,
                   (n_acc > 0 || kk > 0) ? 1u : 0u);
          if (psub == 1) tc_commit(smem_u32(&sh.k_empty[pst]));
        }
        __syncwarp();
        if (lane == 0) trace_event<PROF>(a.trace_buf, 0, 2 * pgt + psub, 3, 4);
        ++n_acc;
        return true;
      };
      bool last = false;
      while (!last && ok) {
        ok = wait_all(&sh.k_full[st], ph);
        if (ok) ok = wait_all(&sh.v_full[st], ph);
        if (!ok) break;
        last = sh.meta[gt & (META_RING - 1)] & 1;
        if (lane == 0) trace_event<PROF>(a.trace_buf, 0, 2 * gt, 0, 4);
        tc_fence_after();
        for (uint32_t sub = 0; sub < 2 && ok; ++sub) {
          const uint32_t k_lo = k_lo0 + st * (TILE_BYTES >> 4) + sub * (SUBTILE_BYTES >> 4);
          const uint32_t v_lo = v_lo0 + st * (TILE_BYTES >> 4) + sub * (SUBTILE_BYTES >> 4);
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
              mma_ts(tmem + DQ_S0 + sub * 64, tmem + DQ_QA + kk * 8, desc_join(k_lo + kstep_lo(kk), HI), IDESC_S,
                     kk > 0 ? 1u : 0u);
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
              mma_ts(tmem + DQ_DP0 + sub * 64, tmem + DQ_DOA + kk * 8, desc_join(v_lo + kstep_lo(kk), HI), IDESC_S,
                     kk > 0 ? 1u : 0u);
            tc_commit(smem_u32(&sh.s_full[sub]));
            if (sub == 1) tc_commit(smem_u32(&sh.v_empty[st]));
          }
          __syncwarp();
          if (lane == 0) trace_event<PROF>(a.trace_buf, 0, 2 * gt + sub, 1, 4);
          if (have_prev) ok = issue_acc(prev_gt, prev_sub, prev_st);
          prev_gt = gt; prev_sub = sub; prev_st = st; have_prev = true;
        }
        ++gt;
        if (++st == DQ_STAGES) { st = 0; ph ^= 1; }
      }
      if (!ok) break;
      if (have_prev) ok = issue_acc(prev_gt, prev_sub, prev_st);
      if (!ok) break;
      if (elect_one()) tc_commit(smem_u32(&sh.acc_full));
      __syncwarp();
      ++it;
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ work-item scheduler
    run_item_scheduler<false>(sh.ring, a, items, total_items, ws + WS_CURSOR1, abort_flag);
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue groups
    const int wg = (warp - 4) >> 2;
    const int row = ((warp & 3) << 5) | lane;  // query row inside the block = thread index in the group
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const uint64_t c1 = dup_f32x2(0.5f * a.alpha);
    unsigned char* stage = sh.stage + wg * HALF_TILE_BYTES;
    uint32_t gt = 0, it = 0;
    bool ok = true;
    int2 w;
    SeqInfo s;
    uint32_t todo0 = 0u, full0 = 0u;
    // A operands of an item: its Q and dO tiles were prefetched into shared memory by TMA; group 0
    // copies its Q row, group 1 its dO row into TMEM (rows past the sequence end as zeros).  The copy
    // for item n + 1 is made at the END of item n, right after its last half tile: by then every score
    // MMA of item n has completed (the epilogue waited for each of them), so nothing reads the operand
    // columns any more, while the last dQ MMAs and the accumulator drain are still to come.  The MMA
    // warp can therefore issue the next item's first score MMAs while this item's dQ leaves TMEM.
    auto copy_a_operands = [&](uint32_t item, int m_row, int len) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.qd_full), item & 1, abort_flag, a.status, WAIT_EPILOGUE)))
        return false;
      const unsigned char* tile = wg == 0 ? sh.q : sh.d_o;
      const uint32_t dst = tmem + lane_addr + (wg == 0 ? DQ_QA : DQ_DOA);
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 4 x 16 TMEM columns = 4 x 32 elements; box = c / 2, chunks (c % 2) * 4 ..
        uint32_t r[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int chunk = (c & 1) * 4 + j;  // 16-byte chunk inside the 128-byte box row
          uint4 x = *reinterpret_cast<const uint4*>(tile + (c >> 1) * HALF_TILE_BYTES + row * 128 +
                                                    ((chunk ^ (row & 7)) << 4));
          if (m_row >= len) x = make_uint4(0u, 0u, 0u, 0u);
          r[4 * j + 0] = x.x; r[4 * j + 1] = x.y; r[4 * j + 2] = x.z; r[4 * j + 3] = x.w;
        }
        tmem_st16(dst + c * 16, r);
      }
      mbar_arrive(smem_u32(&sh.qd_empty));  // the tile has been read: the item after may land
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&sh.a_ready));
      return true;
    };
    bool have = next_item(sh.ring, 0, w, s, todo0, full0, ok, abort_flag, a.status, WAIT_EPILOGUE);
    if (have) ok = copy_a_operands(0, w.y * BLK + row, s.len);
    for (uint32_t n_item = 0; ok && have; ++n_item) {
      const int head = w.x >> 16, qblk = w.y;
      const int m0 = qblk * BLK, m = m0 + row;
      const RowMask rm = row_mask(m, s, a.mask);
      const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
      const int cnt = kr.count();
      for (int base = 0; base < cnt && ok; base += 32) {
        uint32_t todo = todo0, full_bits = full0;  // the scheduler warp classified the first 32 candidates
        if (base > 0) {
          int my_cls = TILE_SKIP;
          if (base + lane < cnt) my_cls = classify_tile(m0, kr.at(base + lane) * BLK, s, a.mask, true);
          todo = __ballot_sync(0xffffffffu, my_cls != TILE_SKIP);
          full_bits = __ballot_sync(0xffffffffu, my_cls == TILE_FULL);
        }
        while (todo != 0u && ok) {
          const int bit = __ffs(todo) - 1;
          todo &= todo - 1;
          const int n0 = kr.at(base + bit) * BLK;
          const bool full = (full_bits >> bit) & 1u;
          // both groups work on every 64-column half tile: group wg owns its columns [32 wg, 32 wg + 32)
          for (int sub = 0; sub < 2 && ok; ++sub) {
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 0, 6);
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.s_full[sub]), gt & 1, abort_flag, a.status, WAIT_EPILOGUE));
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 1, 6);
            if (!ok) break;
            tc_fence_after();
            const uint32_t s_addr = tmem + lane_addr + DQ_S0 + sub * 64 + wg * 32;
            const uint32_t dp_addr = tmem + lane_addr + DQ_DP0 + sub * 64 + wg * 32;
            uint32_t sv[32], dpv[32], pk[16], unused[16];
            tmem_ld32(s_addr, sv);
            tmem_ld32(dp_addr, dpv);
            tmem_wait_ld(sv);
            tmem_wait_ld(dpv);
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 2, 6);
            // on partial tiles most 32-column chunks are all-kept or all-dropped for a whole warp
            // (32 consecutive rows): vote, mask per element only where the boundary crosses
            const uint32_t hb = full ? 0xffffffffu
                                     : static_cast<uint32_t>(row_mask_bits64(rm, n0 + sub * 64) >> (32 * wg));
            if (__all_sync(0xffffffffu, hb == 0xffffffffu)) {
              bwd_chunk<IS_BF16, false, false>(sv, dpv, unused, pk, c1, 0u);
            } else if (__all_sync(0xffffffffu, hb == 0u)) {
#pragma unroll
              for (int i = 0; i < 16; ++i) pk[i] = 0u;
            } else {
              bwd_chunk<IS_BF16, false, true>(sv, dpv, unused, pk, c1, hb);
            }
            tmem_st16(dp_addr, pk);  // dS (16 columns) over the group's own dP columns
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 3, 6);
            if (n0 + BLK > s.len && wg == 0) {
              // key rows past the sequence end feed the dQ MMA as B rows: clear them (0 * NaN = NaN)
              const int first_bad = s.len - n0, lo = first_bad > sub * 64 ? first_bad : sub * 64;
              zero_box_rows(sh.k[gt % DQ_STAGES] + (row >> 6) * HALF_TILE_BYTES, lo, sub * 64 + 64, row & 63, 64);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(smem_u32(&sh.ds_ready[sub]));
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 4, 6);
          }
          ++gt;
        }
      }
      if (!ok) break;
      // ---- next item: take it from the ring and put its A operands in place (see copy_a_operands)
      int2 w_next;
      SeqInfo s_next;
      uint32_t todo_next = 0u, full_next = 0u;
      const bool have_next = next_item(sh.ring, n_item + 1, w_next, s_next, todo_next, full_next, ok, abort_flag, a.status,
                                       WAIT_EPILOGUE);
      if (!ok) break;
      if (have_next) {
        ok = copy_a_operands(it + 1, w_next.y * BLK + row, s_next.len);
        if (!ok) break;
      }
      // ---- dQ leaves TMEM: group wg converts columns [64 wg, 64 wg + 64) of its row
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.acc_full), it & 1, abort_flag, a.status, WAIT_EPILOGUE));
      if (!ok) break;
      tc_fence_after();
      uint32_t ov0[32], ov1[32];
      tmem_ld32(tmem + lane_addr + DQ_ACC + wg * 64, ov0);
      tmem_ld32(tmem + lane_addr + DQ_ACC + wg * 64 + 32, ov1);
      tmem_wait_ld(ov0);
      tmem_wait_ld(ov1);
      tc_fence_before();
      mbar_arrive(smem_u32(&sh.acc_empty));
      const float sc = m < s.len ? 0.5f * a.alpha * row_scale(a, s.start + m) : 0.f;
      // A whole 128-row block leaves as one bulk tensor store per group (the staging layout is the
      // 128-byte-swizzled box layout), which runs in the background; the ragged last block of a
      // sequence is copied out by the threads, row by row.
      if (row == 0) bulk_wait_read_all();  // the previous item's store has read the staging buffer
      group_barrier(wg);
      stage_row64<IS_BF16>(stage, row, ov0, ov1, sc);
      if (m0 + BLK <= s.len) {
        fence_proxy_async();
        group_barrier(wg);
        if (row == 0) {
          tma_store_2d(&maps.dq, smem_u32(stage), head * HEAD_DIM + wg * 64, static_cast<int>(s.start) + m0);
          bulk_commit();
        }
      } else {
        group_barrier(wg);
        store_staged64(stage, reinterpret_cast<unsigned short*>(a.dq) + (s.start + m0) * a.dq_rs + head * HEAD_DIM + wg * 64,
                       a.dq_rs, s.len - m0, row);
      }
      if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt, 5, 6);
      ++it;
      w = w_next; s = s_next; todo0 = todo_next; full0 = full_next; have = have_next;
    }
    if (row == 0) bulk_wait_all();  // shared memory must outlive the stores that read it
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
  // This kernel may have been started before the dK/dV kernel ahead of it in the stream finished
  // (programmatic dependent launch): it must not complete first, or work queued behind it could see
  // unfinished dK / dV.
  grid_dependency_wait();
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
  unsigned char stage[TILE_BYTES];
  unsigned long long kv_full, kv_empty;
  unsigned long long qd_full[KV_STAGES], qd_empty[KV_STAGES];
  unsigned long long s_full[2], p_ready[2], acc_full, acc_empty;
  int meta[META_RING];
  ItemRing ring;
  uint32_t tmem_base;
  int abort_flag;
};

template <bool IS_BF16, bool PROF>
__global__ void __launch_bounds__(BWD_THREADS, 1)
hstu_bwd_dkv_tc(const __grid_constant__ MapsBwd maps, KernelArgs a, int* __restrict__ ws, long long off_items) {
  extern __shared__ unsigned char smem_raw[];
  DkvShared& sh = *reinterpret_cast<DkvShared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Launched as a dependent of the work-list kernel, which lets its dependents become resident as soon as it
  // starts: nothing of the workspace is read before this wait, after which the work list is complete.
  grid_dependency_wait();
  const int total_items = ws[0];
  // Let the CTAs of the dQ kernel that follows in the stream become resident on the SMs that this kernel's
  // CTAs leave, instead of after the last of them has finished.  The recomputing dQ kernel reads nothing this
  // kernel writes and starts working at once; the one that reads the stored dS tiles waits at its top until
  // this whole grid has completed and its writes are visible.  (After the wait above, so that neither can
  // start before the work list is complete.)
  grid_launch_dependents();
  if (static_cast<int>(blockIdx.x) >= total_items) return;
  const int2* items = reinterpret_cast<const int2*>(ws + off_items);
  volatile int* abort_flag = &sh.abort_flag;
  int* prof = ws + 2;

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    item_ring_init(sh.ring);
    mbar_init(smem_u32(&sh.kv_full), 1);
    mbar_init(smem_u32(&sh.kv_empty), 1);
    for (int i = 0; i < KV_STAGES; ++i) { mbar_init(smem_u32(&sh.qd_full[i]), 1); mbar_init(smem_u32(&sh.qd_empty[i]), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(smem_u32(&sh.s_full[i]), 1); mbar_init(smem_u32(&sh.p_ready[i]), 256); }
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
  if (warp < 4) setmaxnreg_dec<136>(); else setmaxnreg_inc<176>();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer / tile scheduler
    if (lane == 0) {
      prefetch_tensormap(&maps.q); prefetch_tensormap(&maps.k);
      prefetch_tensormap(&maps.v); prefetch_tensormap(&maps.d_o);
    }
    uint32_t gt = 0, it = 0, st = 0, ph = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_PRODUCER));
    };
    int2 w;
    SeqInfo s;
    uint32_t todo0 = 0u, full0 = 0u;
    for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w, s, todo0, full0, ok, abort_flag, a.status, WAIT_PRODUCER); ++n_item) {
      const int head = w.x >> 16;
      const int kvblk = (s.len + BLK - 1) / BLK - 1 - w.y;
      const int n0 = kvblk * BLK, col0 = head * HEAD_DIM;
      const int krow = static_cast<int>(s.start) + n0;
      ok = wait_all(&sh.kv_empty, (it & 1) ^ 1);
      if (!ok) break;
      if (elect_one()) {
        mbar_arrive_expect_tx(smem_u32(&sh.kv_full), 2 * TILE_BYTES);
        tma_load_2d(smem_u32(sh.k), &maps.k, smem_u32(&sh.kv_full), col0, krow);
        tma_load_2d(smem_u32(sh.k) + HALF_TILE_BYTES, &maps.k, smem_u32(&sh.kv_full), col0 + 64, krow);
        tma_load_2d(smem_u32(sh.v), &maps.v, smem_u32(&sh.kv_full), col0, krow);
        tma_load_2d(smem_u32(sh.v) + HALF_TILE_BYTES, &maps.v, smem_u32(&sh.kv_full), col0 + 64, krow);
      }
      __syncwarp();
      const BlockRange qr = query_blocks_for_key_block(n0, s, a.mask);
      const int cnt = qr.count();
      // first pass: how many query blocks are kept (to flag the last one for the MMA warp)
      int n_tiles = __popc(todo0);  // the scheduler warp classified the first 32 candidates
      for (int base = 32; base < cnt; base += 32) {
        int my_cls = TILE_SKIP;
        if (base + lane < cnt) my_cls = classify_tile(qr.at(base + lane) * BLK, n0, s, a.mask);
        n_tiles += __popc(__ballot_sync(0xffffffffu, my_cls != TILE_SKIP));
      }
      int emitted = 0;
      for (int base = 0; base < cnt && ok; base += 32) {
        uint32_t todo = todo0;
        if (base > 0) {
          int my_cls = TILE_SKIP;
          if (base + lane < cnt) my_cls = classify_tile(qr.at(base + lane) * BLK, n0, s, a.mask);
          todo = __ballot_sync(0xffffffffu, my_cls != TILE_SKIP);
        }
        while (todo != 0u && ok) {
          const int bit = __ffs(todo) - 1;
          todo &= todo - 1;
          const int qrow = static_cast<int>(s.start) + qr.at(base + bit) * BLK;
          ok = wait_all(&sh.qd_empty[st], ph ^ 1);
          if (!ok) break;
          ++emitted;
          if (elect_one()) {
            sh.meta[gt & (META_RING - 1)] = (emitted == n_tiles) ? 1 : 0;
            mbar_arrive_expect_tx(smem_u32(&sh.qd_full[st]), 2 * TILE_BYTES);
            tma_load_2d(smem_u32(sh.q[st]), &maps.q, smem_u32(&sh.qd_full[st]), col0, qrow);
            tma_load_2d(smem_u32(sh.q[st]) + HALF_TILE_BYTES, &maps.q, smem_u32(&sh.qd_full[st]), col0 + 64, qrow);
            tma_load_2d(smem_u32(sh.d_o[st]), &maps.d_o, smem_u32(&sh.qd_full[st]), col0, qrow);
            tma_load_2d(smem_u32(sh.d_o[st]) + HALF_TILE_BYTES, &maps.d_o, smem_u32(&sh.qd_full[st]), col0 + 64, qrow);
          }
          __syncwarp();
          ++gt;
          if (++st == KV_STAGES) { st = 0; ph ^= 1; }
        }
      }
      ++it;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC_S = idesc_f16(IS_BF16 ? 1 : 0, BLK, 64, 0, 0);          // K/V (K-major) x Q/dO half (K-major)
    constexpr uint32_t IDESC_ACC = idesc_f16(IS_BF16 ? 1 : 0, BLK, HEAD_DIM, 0, 1);  // P^T/dS^T (TMEM) x dO/Q half (N-major)
    constexpr uint32_t HI = desc_hi_sw128(1024);
    const uint32_t k_lo = desc_lo_sw128(smem_u32(sh.k), 16);
    const uint32_t v_lo = desc_lo_sw128(smem_u32(sh.v), 16);
    const uint32_t q_lo0 = desc_lo_sw128(smem_u32(sh.q[0]), 16);
    const uint32_t do_lo0 = desc_lo_sw128(smem_u32(sh.d_o[0]), 16);
    const uint32_t qn_lo0 = desc_lo_sw128(smem_u32(sh.q[0]), HALF_TILE_BYTES);     // Q as N-major operand
    const uint32_t don_lo0 = desc_lo_sw128(smem_u32(sh.d_o[0]), HALF_TILE_BYTES);  // dO as N-major operand
    uint32_t gt = 0, it = 0, st = 0, ph = 0;
    bool ok = true;
    long long pf[5] = {0, 0, 0, 0, 0};
    Stopwatch<PROF> sw_total, sw;
    sw_total.start();
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_MMA));
    };
    int2 w_unused;
    SeqInfo s_unused;
    uint32_t t_unused = 0u, f_unused = 0u;
    for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w_unused, s_unused, t_unused, f_unused, ok, abort_flag, a.status, WAIT_MMA); ++n_item) {
      sw.start();
      ok = wait_all(&sh.kv_full, it & 1);
      sw.stop(pf[PB_MMA_WAIT_ITEM]);
      if (!ok) break;
      tc_fence_after();
      bool have_prev = false;
      uint32_t prev_gt = 0, prev_sub = 0, prev_st = 0, n_acc = 0;
      auto issue_acc = [&](uint32_t pgt, uint32_t psub, uint32_t pst) -> bool {
        sw.start();
        const bool g1 = wait_all(&sh.p_ready[psub], pgt & 1);
        sw.stop(pf[PB_MMA_WAIT_P]);
        if (!g1) return false;
        sw.start();
        const bool g2 = n_acc != 0 || wait_all(&sh.acc_empty, (it & 1) ^ 1);
        sw.stop(pf[PB_MMA_WAIT_ACC]);
        if (!g2) return false;
        if (lane == 0) trace_event<PROF>(a.trace_buf, 0, 2 * pgt + psub, 1, 4);
        tc_fence_after();
        const uint32_t don_lo = don_lo0 + pst * (TILE_BYTES >> 4) + psub * (SUBTILE_BYTES >> 4);
        const uint32_t qn_lo = qn_lo0 + pst * (TILE_BYTES >> 4) + psub * (SUBTILE_BYTES >> 4);
        const uint32_t acc = (n_acc > 0) ? 1u : 0u;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + KV_DV, tmem + KV_ST0 + psub * 64 + (kk >> 1) * 32 + (kk & 1) * 8, desc_join(don_lo + kk * (2048 >> 4), HI), IDESC_ACC,
                   (acc || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + KV_DK, tmem + KV_DPT0 + psub * 64 + (kk >> 1) * 32 + (kk & 1) * 8, desc_join(qn_lo + kk * (2048 >> 4), HI), IDESC_ACC,
                   (acc || kk > 0) ? 1u : 0u);
          if (psub == 1) tc_commit(smem_u32(&sh.qd_empty[pst]));
        }
        __syncwarp();
        if (lane == 0) trace_event<PROF>(a.trace_buf, 0, 2 * pgt + psub, 2, 4);
        ++n_acc;
        return true;
      };
      bool last = false;
      if (lane == 0) trace_event<PROF>(a.trace_buf, 0, 2 * gt, 3, 4);  // item start (kv tiles landed)
      while (!last && ok) {
        sw.start();
        ok = wait_all(&sh.qd_full[st], ph);
        sw.stop(pf[PB_MMA_WAIT_LOAD]);
        if (!ok) break;
        last = sh.meta[gt & (META_RING - 1)] & 1;
        tc_fence_after();
        for (uint32_t sub = 0; sub < 2 && ok; ++sub) {
          const uint32_t q_lo = q_lo0 + st * (TILE_BYTES >> 4) + sub * (SUBTILE_BYTES >> 4);
          const uint32_t do_lo = do_lo0 + st * (TILE_BYTES >> 4) + sub * (SUBTILE_BYTES >> 4);
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
              mma_ss(tmem + KV_ST0 + sub * 64, desc_join(k_lo + kstep_lo(kk), HI), desc_join(q_lo + kstep_lo(kk), HI),
                     IDESC_S, kk > 0 ? 1u : 0u);
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
              mma_ss(tmem + KV_DPT0 + sub * 64, desc_join(v_lo + kstep_lo(kk), HI), desc_join(do_lo + kstep_lo(kk), HI),
                     IDESC_S, kk > 0 ? 1u : 0u);
            tc_commit(smem_u32(&sh.s_full[sub]));
          }
          __syncwarp();
          if (lane == 0) trace_event<PROF>(a.trace_buf, 0, 2 * gt + sub, 0, 4);
          if (have_prev) ok = issue_acc(prev_gt, prev_sub, prev_st);
          prev_gt = gt; prev_sub = sub; prev_st = st; have_prev = true;
        }
        ++gt;
        if (++st == KV_STAGES) { st = 0; ph ^= 1; }
      }
      if (!ok) break;
      if (elect_one()) tc_commit(smem_u32(&sh.kv_empty));  // every score MMA of this item has been issued
      __syncwarp();
      if (have_prev) ok = issue_acc(prev_gt, prev_sub, prev_st);
      if (!ok) break;
      if (elect_one()) tc_commit(smem_u32(&sh.acc_full));
      __syncwarp();
      ++it;
    }
    sw_total.stop(pf[PB_MMA_TOTAL]);
    if (PROF && lane == 0)
      for (int i = 0; i < 5; ++i) atomicAdd(prof + i, (int)(pf[i] >> 6));
  } else if (warp == 2) {
    // ------------------------------------------------------------------ work-item scheduler
    run_item_scheduler<true>(sh.ring, a, items, total_items, ws + WS_CURSOR0, abort_flag);
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue groups
    const int wg = (warp - 4) >> 2;
    const int row = ((warp & 3) << 5) | lane;  // key row inside the block = thread index in the group
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const uint64_t c1 = dup_f32x2(0.5f * a.alpha);
    const bool per_token = a.scale_mode == 2;
    unsigned char* stage = sh.stage + wg * HALF_TILE_BYTES;
    uint32_t gt = 0, it = 0;
    bool ok = true;
    long long pe_total = 0, pe_ws = 0, pe_wacc = 0, pe_tile = 0, pe_drain = 0, pe_ld = 0, pe_st = 0;
    Stopwatch<PROF> sw_total, sw, sw2;
    sw_total.start();
    int2 w;
    SeqInfo s;
    uint32_t todo0 = 0u, full0 = 0u;
    for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w, s, todo0, full0, ok, abort_flag, a.status, WAIT_EPILOGUE); ++n_item) {
      const int head = w.x >> 16;
      const int kvblk = (s.len + BLK - 1) / BLK - 1 - w.y;
      const int n0 = kvblk * BLK, n = n0 + row;
      const ColMask cm = col_mask(n, s, a.mask);
      const BlockRange qr = query_blocks_for_key_block(n0, s, a.mask);
      const int cnt = qr.count();
      for (int base = 0; base < cnt && ok; base += 32) {
        uint32_t todo = todo0, full_bits = full0;  // the scheduler warp classified the first 32 candidates
        if (base > 0) {
          int my_cls = TILE_SKIP;
          if (base + lane < cnt) my_cls = classify_tile(qr.at(base + lane) * BLK, n0, s, a.mask);
          todo = __ballot_sync(0xffffffffu, my_cls != TILE_SKIP);
          full_bits = __ballot_sync(0xffffffffu, my_cls == TILE_FULL);
        }
        while (todo != 0u && ok) {
          const int bit = __ffs(todo) - 1;
          todo &= todo - 1;
          const int q0 = qr.at(base + bit) * BLK;
          const bool full = (full_bits >> bit) & 1u;
          // both groups work on every 64-column half tile: group wg owns its columns [32 wg, 32 wg + 32)
          for (int sub = 0; sub < 2 && ok; ++sub) {
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 0, 6);
            sw.start();
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.s_full[sub]), gt & 1, abort_flag, a.status, WAIT_EPILOGUE));
            sw.stop(pe_ws);
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 1, 6);
            if (!ok) break;
            tc_fence_after();
            sw.start();
            const uint32_t st_addr = tmem + lane_addr + KV_ST0 + sub * 64 + wg * 32;
            const uint32_t dp_addr = tmem + lane_addr + KV_DPT0 + sub * 64 + wg * 32;
            const int mbase = q0 + sub * 64;
            uint32_t sv[32], dpv[32], pp[16], pd[16];
            sw2.start();
            tmem_ld32(st_addr, sv);
            tmem_ld32(dp_addr, dpv);
            tmem_wait_ld(sv);
            tmem_wait_ld(dpv);
            sw2.stop(pe_ld);
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 2, 6);
            const uint32_t hb = full ? 0xffffffffu
                                     : static_cast<uint32_t>(col_mask_bits64(cm, s.len, mbase) >> (32 * wg));
            if (__all_sync(0xffffffffu, hb == 0xffffffffu)) {
              bwd_chunk<IS_BF16, true, false>(sv, dpv, pp, pd, c1, 0u);
            } else if (__all_sync(0xffffffffu, hb == 0u)) {
#pragma unroll
              for (int i = 0; i < 16; ++i) { pp[i] = 0u; pd[i] = 0u; }
            } else {
              bwd_chunk<IS_BF16, true, true>(sv, dpv, pp, pd, c1, hb);
            }
            if (per_token) {  // one scale per query token = per column here (masked entries stay zero)
              scale_chunk<IS_BF16>(pp, a.attn_scale, s.start, mbase + wg * 32, s.len);
              scale_chunk<IS_BF16>(pd, a.attn_scale, s.start, mbase + wg * 32, s.len);
            }
            tmem_st16(st_addr, pp);  // P^T and dS^T (16 columns each) over the group's own score columns
            tmem_st16(dp_addr, pd);
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 3, 6);
            if (q0 + BLK > s.len && wg == 0) {
              // query rows past the sequence end are B rows of the dV / dK MMAs: clear them
              const int first_bad = s.len - q0, lo = first_bad > sub * 64 ? first_bad : sub * 64;
              zero_box_rows(sh.q[gt % KV_STAGES] + (row >> 6) * HALF_TILE_BYTES, lo, sub * 64 + 64, row & 63, 64);
              zero_box_rows(sh.d_o[gt % KV_STAGES] + (row >> 6) * HALF_TILE_BYTES, lo, sub * 64 + 64, row & 63, 64);
            }
            sw2.start();
            tmem_wait_st();
            sw2.stop(pe_st);
            tc_fence_before();
            mbar_arrive(smem_u32(&sh.p_ready[sub]));
            if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt + sub, 4, 6);
            // (behind the hand-over, so that the dV / dK MMAs of this half tile run meanwhile)
            if (a.ds_tiles != nullptr) {
              // The dQ pass reads this dS^T tile back (keys x queries) instead of recomputing it.  The group
              // stages its 2 x 32 query columns of the tile as ONE 64-column box (row = this thread's key row,
              // 128-byte-swizzled as the bulk store expects) and sends the box out once per tile: the stored
              // tile therefore holds the query columns in the order [group][half][32], i.e. with bits 5 and 6
              // of the column index swapped, which the dQ pass undoes when it drains its accumulator.
              if (sub == 0) {
                if (row == 0) bulk_wait_read_all();  // the group's previous box (or drain) has left the buffer
                group_barrier(wg);
              }
              unsigned char* my = stage + row * 128;
#pragma unroll
              for (int i = 0; i < 4; ++i)
                *reinterpret_cast<uint4*>(my + (((sub * 4 + i) ^ (row & 7)) << 4)) =
                    make_uint4(pd[4 * i], pd[4 * i + 1], pd[4 * i + 2], pd[4 * i + 3]);
              if (sub == 1) {
                fence_proxy_async();
                group_barrier(wg);
                if (row == 0) {
                  long long t = s.tile_base + ds_tile_index(q0 / BLK, kvblk, (s.len + BLK - 1) / BLK, a.ds_square);
                  t = t * a.H + head;
                  if (t >= a.ds_tile_cap) {  // a sequence longer than the caller's bound: stay inside the region
                    t = a.ds_tile_cap - 1;
                    if (a.status) atomicOr(a.status, 1);
                  }
                  tma_store_2d(&maps.ds, smem_u32(stage), wg * 64, static_cast<int>(t * BLK));
                  bulk_commit();
                }
              }
            }
            sw.stop(pe_tile);
          }
          ++gt;
        }
      }
      if (!ok) break;
      // ---- accumulators leave TMEM: group 0 writes dK, group 1 writes dV, 64 columns at a time
      sw.start();
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.acc_full), it & 1, abort_flag, a.status, WAIT_EPILOGUE));
      sw.stop(pe_wacc);
      if (!ok) break;
      tc_fence_after();
      sw.start();
      const float scal = per_token ? 1.f : row_scale(a, 0);
      const float sc = n < s.len ? (wg == 0 ? 0.5f * a.alpha * scal : scal) : 0.f;
      const long long out_rs = wg == 0 ? a.dk_rs : a.dv_rs;
      unsigned short* out0 = (wg == 0 ? reinterpret_cast<unsigned short*>(a.dk) : reinterpret_cast<unsigned short*>(a.dv)) +
                             (s.start + n0) * out_rs + head * HEAD_DIM;
      const uint32_t acc_addr = tmem + lane_addr + (wg == 0 ? KV_DK : KV_DV);
      {
        // Round 0 is staged first; the second half of the accumulator is pulled into registers
        // (which frees TMEM for the next item's MMAs) before any global store is issued.
        uint32_t ov0[32], ov1[32];
        tmem_ld32(acc_addr, ov0);
        tmem_ld32(acc_addr + 32, ov1);
        tmem_wait_ld(ov0);
        tmem_wait_ld(ov1);
        if (row == 0) bulk_wait_read_all();  // the previous item's stores have read the staging buffer
        group_barrier(wg);
        stage_row64<IS_BF16>(stage, row, ov0, ov1, sc);
        tmem_ld32(acc_addr + 64, ov0);
        tmem_ld32(acc_addr + 96, ov1);
        tmem_wait_ld(ov0);
        tmem_wait_ld(ov1);
        tc_fence_before();
        mbar_arrive(smem_u32(&sh.acc_empty));
        if (n0 + BLK <= s.len) {
          // whole 128-row block: two bulk tensor stores per group (64 columns each) run in the
          // background; the second waits until the first has read the staging buffer
          const CUtensorMap* omap = wg == 0 ? &maps.dk : &maps.dv;
          const int orow = static_cast<int>(s.start) + n0, ocol = head * HEAD_DIM;
          fence_proxy_async();
          group_barrier(wg);
          if (row == 0) {
            tma_store_2d(omap, smem_u32(stage), ocol, orow);
            bulk_commit();
            bulk_wait_read_all();
          }
          group_barrier(wg);
          stage_row64<IS_BF16>(stage, row, ov0, ov1, sc);
          fence_proxy_async();
          group_barrier(wg);
          if (row == 0) {
            tma_store_2d(omap, smem_u32(stage), ocol + 64, orow);
            bulk_commit();
          }
        } else {
          group_barrier(wg);
          store_staged64(stage, out0, out_rs, s.len - n0, row);
          group_barrier(wg);
          stage_row64<IS_BF16>(stage, row, ov0, ov1, sc);
          group_barrier(wg);
          store_staged64(stage, out0 + 64, out_rs, s.len - n0, row);
        }
      }
      sw.stop(pe_drain);
      if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, 2 * gt, 5, 6);  // drain finished (before half tile 2*gt)
      ++it;
    }
    if (row == 0) bulk_wait_all();  // shared memory must outlive the stores that read it
    sw_total.stop(pe_total);
    if (PROF && (threadIdx.x == 128 || threadIdx.x == 256)) {
      atomicAdd(prof + PB_EPI_TOTAL, (int)(pe_total >> 6)); atomicAdd(prof + PB_EPI_WAIT_S, (int)(pe_ws >> 6));
      atomicAdd(prof + PB_EPI_WAIT_ACC, (int)(pe_wacc >> 6)); atomicAdd(prof + PB_EPI_TILE, (int)(pe_tile >> 6));
      atomicAdd(prof + PB_EPI_DRAIN, (int)(pe_drain >> 6)); atomicAdd(prof + PB_EPI_LD, (int)(pe_ld >> 6));
      atomicAdd(prof + PB_EPI_ST, (int)(pe_st >> 6));
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
// dQ pass from stored dS tiles
// ------------------------------------------------------------------------------------
// The dK/dV pass has written every dS^T tile it computed (keys x queries, 16-bit, masked entries zero, the
// per-token scale folded in).  What is left of the dQ pass is dQ[query block] = sum over its key blocks of
// dS K: per tile ONE GEMM (M128 N128 K128, both operands from shared memory: dS^T as the M-major A operand, K
// as the N-major B operand) instead of three, no transcendental, no mask, no operand copies into TMEM.  The
// pass is bound by bringing in 64 KB per tile (the dS tile from HBM, the K tile mostly from L2).
// Two accumulators: the MMAs of the next query block run while the previous one leaves TMEM.
constexpr int DQS_STAGES = 3;
constexpr int DQS_ACC0 = 0;  // accumulator b at columns 128 b

struct DqsShared {
  unsigned char ds[DQS_STAGES][TILE_BYTES];
  unsigned char k[DQS_STAGES][TILE_BYTES];
  unsigned char stage[TILE_BYTES];
  unsigned long long full[DQS_STAGES], empty[DQS_STAGES];
  unsigned long long acc_full[2], acc_empty[2];
  int meta[META_RING];  // per tile: bit 0 = last tile of its item, bits 8.. = key rows of the tile inside the sequence
  ItemRing ring;
  uint32_t tmem_base;
  int abort_flag;
};

template <bool IS_BF16>
__global__ void __launch_bounds__(BWD_THREADS, 1)
hstu_bwd_dq_stored_tc(const __grid_constant__ MapsBwd maps, KernelArgs a, int* __restrict__ ws, long long off_items) {
  extern __shared__ unsigned char smem_raw[];
  DqsShared& sh = *reinterpret_cast<DqsShared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Every dS tile this kernel reads was written by the dK/dV kernel before it in the stream, which may still be
  // running when this CTA becomes resident (programmatic dependent launch).  The producer warp therefore waits
  // for that kernel to have completed, with its writes visible, before its first load (a no-op for an ordinary
  // launch); barrier set-up, the TMEM allocation and the first claims from the work list, which was complete
  // before the dK/dV kernel started, do not wait.  A CTA without work waits too, so that this kernel never
  // completes before the one ahead of it.
  const int total_items = ws[0];
  if (static_cast<int>(blockIdx.x) >= total_items) {
    grid_dependency_wait();
    return;
  }
  const int2* items = reinterpret_cast<const int2*>(ws + off_items);
  volatile int* abort_flag = &sh.abort_flag;

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    item_ring_init(sh.ring);
    for (int i = 0; i < DQS_STAGES; ++i) { mbar_init(smem_u32(&sh.full[i]), 1); mbar_init(smem_u32(&sh.empty[i]), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(smem_u32(&sh.acc_full[i]), 1); mbar_init(smem_u32(&sh.acc_empty[i]), 256); }
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&sh.tmem_base), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer / tile scheduler
    if (lane == 0) { prefetch_tensormap(&maps.k); prefetch_tensormap(&maps.ds); }
    grid_dependency_wait();  // the dS tiles are complete and visible from here on
    uint32_t gt = 0, st = 0, ph = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_PRODUCER));
    };
    int2 w;
    SeqInfo s;
    uint32_t todo0 = 0u, full0 = 0u;
    for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w, s, todo0, full0, ok, abort_flag, a.status, WAIT_PRODUCER); ++n_item) {
      const int head = w.x >> 16, qblk = w.y;
      const int m0 = qblk * BLK, col0 = head * HEAD_DIM;
      const long long nb = (s.len + BLK - 1) / BLK;
      const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
      const int cnt = kr.count();
      // The tiles of this query block are the ones the dK/dV pass did not skip (the same classification;
      // whether a tile is skipped does not depend on which pass asks).
      int n_tiles = __popc(todo0);  // the scheduler warp classified the first 32 candidates
      for (int base = 32; base < cnt; base += 32) {
        int my_cls = TILE_SKIP;
        if (base + lane < cnt) my_cls = classify_tile(m0, kr.at(base + lane) * BLK, s, a.mask);
        n_tiles += __popc(__ballot_sync(0xffffffffu, my_cls != TILE_SKIP));
      }
      int emitted = 0;
      for (int base = 0; base < cnt && ok; base += 32) {
        uint32_t todo = todo0;
        if (base > 0) {
          int my_cls = TILE_SKIP;
          if (base + lane < cnt) my_cls = classify_tile(m0, kr.at(base + lane) * BLK, s, a.mask);
          todo = __ballot_sync(0xffffffffu, my_cls != TILE_SKIP);
        }
        while (todo != 0u && ok) {
          const int bit = __ffs(todo) - 1;
          todo &= todo - 1;
          const int kblk = kr.at(base + bit);
          ok = wait_all(&sh.empty[st], ph ^ 1);
          if (!ok) break;
          ++emitted;
          if (elect_one()) {
            long long t = (s.tile_base + ds_tile_index(qblk, kblk, nb, a.ds_square)) * a.H + head;
            if (t >= a.ds_tile_cap) t = a.ds_tile_cap - 1;  // (flagged by the pass that wrote the tiles)
            const int trow = static_cast<int>(t * BLK), krow = static_cast<int>(s.start) + kblk * BLK;
            const int rows_in = s.len - kblk * BLK;  // key rows of the tile that belong to the sequence
            sh.meta[gt & (META_RING - 1)] = ((emitted == n_tiles) ? 1 : 0) | ((rows_in < BLK ? rows_in : BLK) << 8);
            mbar_arrive_expect_tx(smem_u32(&sh.full[st]), 2 * TILE_BYTES);
            tma_load_2d(smem_u32(sh.ds[st]), &maps.ds, smem_u32(&sh.full[st]), 0, trow);
            tma_load_2d(smem_u32(sh.ds[st]) + HALF_TILE_BYTES, &maps.ds, smem_u32(&sh.full[st]), 64, trow);
            tma_load_2d(smem_u32(sh.k[st]), &maps.k, smem_u32(&sh.full[st]), col0, krow);
            tma_load_2d(smem_u32(sh.k[st]) + HALF_TILE_BYTES, &maps.k, smem_u32(&sh.full[st]), col0 + 64, krow);
          }
          __syncwarp();
          ++gt;
          if (++st == DQS_STAGES) { st = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC = idesc_f16(IS_BF16 ? 1 : 0, BLK, HEAD_DIM, 1, 1);  // dS^T (M-major A) x K (N-major B)
    constexpr uint32_t HI = desc_hi_sw128(1024);
    const uint32_t ds_lo0 = desc_lo_sw128(smem_u32(sh.ds[0]), HALF_TILE_BYTES);  // 64-query groups one box apart
    const uint32_t k_lo0 = desc_lo_sw128(smem_u32(sh.k[0]), HALF_TILE_BYTES);    // 64-column groups one box apart
    uint32_t gt = 0, it = 0, st = 0, ph = 0;
    bool ok = true;
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_MMA));
    };
    int2 w_unused;
    SeqInfo s_unused;
    uint32_t t_unused = 0u, f_unused = 0u;
    for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w_unused, s_unused, t_unused, f_unused, ok, abort_flag, a.status, WAIT_MMA); ++n_item, ++it) {
      const uint32_t ab = it & 1;
      ok = wait_all(&sh.acc_empty[ab], ((it >> 1) & 1) ^ 1);
      if (!ok) break;
      tc_fence_after();
      bool last = false;
      uint32_t n_acc = 0;
      while (!last && ok) {
        ok = wait_all(&sh.full[st], ph);
        if (!ok) break;
        const int meta = sh.meta[gt & (META_RING - 1)];
        last = meta & 1;
        const int rows_in = meta >> 8;
        if (rows_in < BLK) {
          // Key rows past the sequence end belong to the next sequence (or are zero fill): their dS entries
          // are zero, but 0 * NaN would not be, so the rows are cleared before they feed the MMA.
          zero_box_rows(sh.k[st], rows_in, BLK, lane, 32);
          zero_box_rows(sh.k[st] + HALF_TILE_BYTES, rows_in, BLK, lane, 32);
          __syncwarp();
        }
        tc_fence_after();
        if (elect_one()) {
          const uint32_t a_lo = ds_lo0 + st * (TILE_BYTES >> 4), b_lo = k_lo0 + st * (TILE_BYTES >> 4);
#pragma unroll
          for (int kk = 0; kk < BLK / 16; ++kk)  // 16 keys per step: 16 rows of 128 bytes in each box
            mma_ss(tmem + DQS_ACC0 + ab * HEAD_DIM, desc_join(a_lo + kk * (2048 >> 4), HI), desc_join(b_lo + kk * (2048 >> 4), HI),
                   IDESC, (n_acc > 0 || kk > 0) ? 1u : 0u);
          tc_commit(smem_u32(&sh.empty[st]));
          if (last) tc_commit(smem_u32(&sh.acc_full[ab]));
        }
        __syncwarp();
        ++n_acc;
        ++gt;
        if (++st == DQS_STAGES) { st = 0; ph ^= 1; }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ work-item scheduler
    run_item_scheduler<false>(sh.ring, a, items, total_items, ws + WS_CURSOR1, abort_flag);
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ accumulator drain (two groups, 64 columns each)
    const int wg = (warp - 4) >> 2;
    const int row = ((warp & 3) << 5) | lane;  // query row inside the block = thread index in the group
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) << 5) << 16;
    unsigned char* stage = sh.stage + wg * HALF_TILE_BYTES;
    const bool per_token = a.scale_mode == 2;
    uint32_t it = 0;
    bool ok = true;
    int2 w;
    SeqInfo s;
    uint32_t todo0 = 0u, full0 = 0u;
    for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w, s, todo0, full0, ok, abort_flag, a.status, WAIT_EPILOGUE); ++n_item, ++it) {
      // accumulator row r holds the query whose index inside the block is r with bits 5 and 6 swapped (the
      // column order of the stored tiles)
      const int qrow = (row & 31) | (((row >> 6) & 1) << 5) | (((row >> 5) & 1) << 6);
      const int head = w.x >> 16, m0 = w.y * BLK, m = m0 + qrow;
      const uint32_t ab = it & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.acc_full[ab]), (it >> 1) & 1, abort_flag, a.status, WAIT_EPILOGUE));
      if (!ok) break;
      tc_fence_after();
      uint32_t ov0[32], ov1[32];
      const uint32_t acc = tmem + lane_addr + DQS_ACC0 + ab * HEAD_DIM + wg * 64;
      tmem_ld32(acc, ov0);
      tmem_ld32(acc + 32, ov1);
      tmem_wait_ld(ov0);
      tmem_wait_ld(ov1);
      tc_fence_before();
      mbar_arrive(smem_u32(&sh.acc_empty[ab]));
      // 1/2 and alpha once per output row; the stored tiles carry a per-token scale already, a scalar one not
      const float sc = m < s.len ? 0.5f * a.alpha * (per_token ? 1.f : row_scale(a, 0)) : 0.f;
      if (row == 0) bulk_wait_read_all();  // the previous item's store has read the staging buffer
      group_barrier(wg);
      stage_row64<IS_BF16>(stage, qrow, ov0, ov1, sc);
      if (m0 + BLK <= s.len) {
        fence_proxy_async();
        group_barrier(wg);
        if (row == 0) {
          tma_store_2d(&maps.dq, smem_u32(stage), head * HEAD_DIM + wg * 64, static_cast<int>(s.start) + m0);
          bulk_commit();
        }
      } else {
        group_barrier(wg);
        store_staged64(stage, reinterpret_cast<unsigned short*>(a.dq) + (s.start + m0) * a.dq_rs + head * HEAD_DIM + wg * 64,
                       a.dq_rs, s.len - m0, row);
      }
    }
    if (row == 0) bulk_wait_all();  // shared memory must outlive the stores that read it
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    if (*abort_flag) {
      const unsigned long long t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
    }
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace
}  // namespace tc

cudaError_t tc_backward(const KernelArgs& a_in, int dtype, void* workspace, cudaStream_t st) {
  using namespace tc;
  const bool bf16 = dtype == B200_HSTU_BF16;
  const WorkspaceLayout w = backward_layout(a_in);
  int* ws = reinterpret_cast<int*>(workspace);
  KernelArgs a = a_in;
  const bool stored_ds = w.ds_tile_cap > 0;
  if (stored_ds) {
    unsigned char* base = reinterpret_cast<unsigned char*>(workspace);
    a.ds_tiles = base + w.off_ds_tiles;
    a.ds_tile_base = reinterpret_cast<const long long*>(base + w.off_tile_base);
    a.ds_tile_cap = w.ds_tile_cap;
    a.ds_square = w.ds_square;
  }
  MapsBwd maps;
  const long long width = (long long)a.H * HEAD_DIM;
  set_error_stage("backward: tensor maps");
  if (!ensure_current_context(a.q)) return cudaErrorInvalidValue;
  if (!make_map(&maps.q, a.q, a.T, width, a.q_rs, bf16) || !make_map(&maps.k, a.k, a.T, width, a.k_rs, bf16) ||
      !make_map(&maps.v, a.v, a.T, width, a.v_rs, bf16) || !make_map(&maps.d_o, a.d_o, a.T, width, a.do_rs, bf16) ||
      !make_map(&maps.dq, a.dq, a.T, width, a.dq_rs, bf16) || !make_map(&maps.dk, a.dk, a.T, width, a.dk_rs, bf16) ||
      !make_map(&maps.dv, a.dv, a.T, width, a.dv_rs, bf16))
    return cudaErrorInvalidValue;
  if (stored_ds) {
    if (!make_map(&maps.ds, a.ds_tiles, w.ds_tile_cap * BLK, BLK, BLK, bf16)) return cudaErrorInvalidValue;
  } else {
    maps.ds = maps.q;  // not used
  }
  set_error_stage("backward: work-list kernels");
  cudaError_t e = launch_prep(a, bf16, ws, w, true, st);
  if (e != cudaSuccess) return e;
  const int grid = main_grid(w);
  if (!a.skip_dkv) {
    set_error_stage("backward: dK/dV kernel");
    const size_t smem = sizeof(DkvShared) + 1024;
#ifdef B200_HSTU_PROFILING
    static const bool profile = getenv("B200_HSTU_PROFILE") != nullptr;
    auto kern = profile ? (bf16 ? hstu_bwd_dkv_tc<true, true> : hstu_bwd_dkv_tc<false, true>)
                        : (bf16 ? hstu_bwd_dkv_tc<true, false> : hstu_bwd_dkv_tc<false, false>);
#else
    auto kern = bf16 ? hstu_bwd_dkv_tc<true, false> : hstu_bwd_dkv_tc<false, false>;
#endif
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    e = launch_dependent(kern, static_cast<unsigned>(grid), BWD_THREADS, smem, st, true, maps, a, ws, w.off_items);
    if (e != cudaSuccess) return e;
  }
  if (!a.skip_dq && stored_ds) {
    set_error_stage("backward: dQ kernel (stored dS tiles)");
    const size_t smem = sizeof(DqsShared) + 1024;
    auto kern = bf16 ? hstu_bwd_dq_stored_tc<true> : hstu_bwd_dq_stored_tc<false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    // behind the dK/dV kernel as a dependent launch: its CTAs become resident early, and wait at their top
    // until that kernel has completed
    e = launch_dependent(kern, static_cast<unsigned>(grid), BWD_THREADS, smem, st, !a.skip_dkv, maps, a, ws, w.off_items);
    if (e != cudaSuccess) return e;
  } else if (!a.skip_dq) {
    set_error_stage("backward: dQ kernel");
    const size_t smem = sizeof(DqShared) + 1024;
#ifdef B200_HSTU_PROFILING
    static const bool profile = getenv("B200_HSTU_PROFILE_DQ") != nullptr;
    auto kern = profile ? (bf16 ? hstu_bwd_dq_tc<true, true> : hstu_bwd_dq_tc<false, true>)
                        : (bf16 ? hstu_bwd_dq_tc<true, false> : hstu_bwd_dq_tc<false, false>);
#else
    auto kern = bf16 ? hstu_bwd_dq_tc<true, false> : hstu_bwd_dq_tc<false, false>;
#endif
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    // a dependent launch only behind the dK/dV kernel, whose output this kernel does not read; alone, it
    // is an ordinary launch behind build_work_items
    e = launch_dependent(kern, static_cast<unsigned>(grid), BWD_THREADS, smem, st, !a.skip_dkv, maps, a, ws, w.off_items);
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

}  // namespace hstu
