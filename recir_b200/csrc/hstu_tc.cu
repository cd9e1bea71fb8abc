// Tensor-core HSTU jagged attention for sm_100a: TMA tile loads, tcgen05 MMAs with TMEM
// accumulators, the scale/SiLU/mask epilogue fused on the accumulator.
//
// Shapes served: bf16 or fp16, Dqk == Dv == 128, causal mask (with every option of the
// mask rule).  Anything else is served by the CUDA-core kernels.
//
// Work decomposition.  A small device-side pass builds a work list of (sequence, head,
// 128-row block) items sorted so that the most expensive items come first; persistent CTAs
// (one per SM) walk the list with a fixed stride.  The forward kernel is warp-specialised:
//   warp 0      TMA producer: Q tile of the item, then K and V tiles of every kept key block
//   warp 1      MMA issuer (one elected lane): S = Q K^T into TMEM, O += P V from TMEM
//   warps 4-7   epilogue group 0   } alternate over key blocks: read S from TMEM, apply
//   warps 8-11  epilogue group 1   } alpha / SiLU / mask, write P (16-bit) back over S
// The output scale (1/N or attn_scale) is a per-query-row factor, so it is applied once
// when O leaves TMEM, not per score.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "hstu_launch.h"
#include "hstu_tc_common.cuh"
#include "hstu_tc_host.h"

namespace hstu {
namespace tc {
namespace {

using namespace sm100;

// ------------------------------------------------------------------------------------
// Work-list construction (device side, no host synchronisation)
// ------------------------------------------------------------------------------------

__device__ __forceinline__ int blocks_of(const KernelArgs& a, int b) {
  const SeqInfo s = load_seq(a, b);
  return (s.len + BLK - 1) / BLK;
}

// out[j] = sum_{i > j} in[i] for j in [0, n): exclusive suffix sum, one CTA of 1024 threads.
__device__ void suffix_sum_exclusive(const int* in, int* out, long long n, int* sh /*1024*/) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const long long chunk = (n + nt - 1) / nt;
  const long long beg = (long long)tid * chunk;
  long long end = beg + chunk;
  if (end > n) end = n;
  int local = 0;
  for (long long i = beg; i < end; ++i) local += in[i];
  sh[tid] = local;
  __syncthreads();
  // inclusive suffix scan over the per-thread totals (Hillis-Steele)
  for (int off = 1; off < nt; off <<= 1) {
    int v = (tid + off < nt) ? sh[tid + off] : 0;
    __syncthreads();
    sh[tid] += v;
    __syncthreads();
  }
  int run = (tid + 1 < nt) ? sh[tid + 1] : 0;  // sum of everything owned by later threads
  __syncthreads();
  for (long long i = end - 1; i >= beg; --i) {
    const int v = in[i];
    out[i] = run;
    run += v;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(1024) build_block_index(KernelArgs a, int* ws, WorkspaceLayout w) {
  __shared__ int sh[1024];
  int* sorted = ws + w.off_sorted;
  int* hist = ws + w.off_hist;
  int* cnt = ws + w.off_cnt;
  int* start = ws + w.off_start;
  const int tid = threadIdx.x;
  for (long long i = tid; i < w.nbins; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int b = tid; b < a.B; b += blockDim.x) {
    long long nb = blocks_of(a, b);
    if (nb > w.nbins - 1) nb = w.nbins - 1;  // cannot happen for offsets within [0, T]
    atomicAdd(&hist[nb], 1);
  }
  __syncthreads();
  suffix_sum_exclusive(hist, cnt, w.nbins, sh);  // cnt[j] = #sequences with more than j blocks
  for (long long i = tid; i < w.nbins; i += blockDim.x) hist[i] = 0;  // reuse as fill counters
  __syncthreads();
  for (int b = tid; b < a.B; b += blockDim.x) {
    long long nb = blocks_of(a, b);
    if (nb > w.nbins - 1) nb = w.nbins - 1;
    if (nb > 0) sorted[cnt[nb] + atomicAdd(&hist[nb], 1)] = b;
  }
  __syncthreads();
  // start[j] = H * sum_{j' > j} cnt[j'] : items of the highest block index come first
  suffix_sum_exclusive(cnt, start, w.nbins, sh);
  for (long long i = tid; i < w.nbins; i += blockDim.x) start[i] *= a.H;
  __syncthreads();
  if (tid == 0) {
    ws[0] = start[0] + cnt[0] * a.H;
    ws[1] = cnt[0];
  }
}

// One thread per work item: find its block index by bisection over start[], then decode.
// Also zeroes the output rows no sequence owns (rows at or past the last offset).
template <typename T>
__global__ void __launch_bounds__(256) build_work_items(KernelArgs a, int* ws, WorkspaceLayout w, T* z0,
                                                        long long rs0, int w0, T* z1, long long rs1, int w1,
                                                        T* z2, long long rs2, int w2) {
  const int* sorted = ws + w.off_sorted;
  const int* cnt = ws + w.off_cnt;
  const int* start = ws + w.off_start;
  int2* items = reinterpret_cast<int2*>(ws + w.off_items);
  const int total = ws[0];
  const long long gtid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long gsz = (long long)gridDim.x * blockDim.x;
  for (long long p = gtid; p < total; p += gsz) {
    // start[] is non-increasing in j; find the largest... smallest j with start[j] <= p
    long long lo = 0, hi = w.nbins - 1;
    while (lo < hi) {
      const long long mid = (lo + hi) >> 1;
      if (start[mid] <= p) hi = mid; else lo = mid + 1;
    }
    const int j = static_cast<int>(lo);
    const int r = static_cast<int>(p - start[j]);
    const int i = r / a.H, head = r - i * a.H;
    int2 it;
    it.x = (i < cnt[j]) ? (sorted[i] | (head << 16)) : -1;
    it.y = j;
    items[p] = it;
  }
  // tail rows
  long long first = load_index(a.seq_offsets, a.offsets_i64, a.B);
  if (first < 0) first = 0;
  if (first > a.T) first = a.T;
  const long long rows = a.T - first;
  const int wmax = max(w0, max(w1, w2));
  const long long tot = rows * wmax;
  for (long long i = gtid; i < tot; i += gsz) {
    const long long r = first + i / wmax;
    const int c = static_cast<int>(i % wmax);
    if (z0 && c < w0) z0[r * rs0 + c] = from_f32<T>(0.f);
    if (z1 && c < w1) z1[r * rs1 + c] = from_f32<T>(0.f);
    if (z2 && c < w2) z2[r * rs2 + c] = from_f32<T>(0.f);
  }
}

// ------------------------------------------------------------------------------------
// Forward kernel
// ------------------------------------------------------------------------------------

constexpr int NUM_K_STAGES = 3;
constexpr int NUM_V_STAGES = 3;
constexpr int FWD_THREADS = 384;
constexpr int TMEM_COLS = 512;
constexpr int TMEM_S0 = 0, TMEM_S1 = 128, TMEM_O0 = 256, TMEM_O1 = 384;

struct FwdShared {
  // tiles first: every tile base must be 1024-byte aligned for the 128-byte swizzle
  unsigned char q[TILE_BYTES];
  unsigned char k[NUM_K_STAGES][TILE_BYTES];
  unsigned char v[NUM_V_STAGES][TILE_BYTES];
  unsigned long long q_full, q_empty;
  unsigned long long k_full[NUM_K_STAGES], k_empty[NUM_K_STAGES];
  unsigned long long v_full[NUM_V_STAGES], v_empty[NUM_V_STAGES];
  unsigned long long s_full[2], p_ready[2];
  unsigned long long o_full[2], o_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct TensorMaps {
  CUtensorMap q, k, v;
};

template <bool IS_BF16>
__global__ void __launch_bounds__(FWD_THREADS, 1)
hstu_fwd_tc(const __grid_constant__ TensorMaps maps, KernelArgs a, const int* __restrict__ ws, long long off_items) {
  extern __shared__ unsigned char smem_raw[];
  // dynamic shared memory is only guaranteed 16-byte aligned: round up to 1024
  FwdShared& sh = *reinterpret_cast<FwdShared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_items = ws[0];
  if (static_cast<int>(blockIdx.x) >= total_items) return;  // uniform per CTA
  const int2* items = reinterpret_cast<const int2*>(ws + off_items);
  volatile int* abort_flag = &sh.abort_flag;

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    mbar_init(smem_u32(&sh.q_full), 1);
    mbar_init(smem_u32(&sh.q_empty), 1);
    for (int i = 0; i < NUM_K_STAGES; ++i) { mbar_init(smem_u32(&sh.k_full[i]), 1); mbar_init(smem_u32(&sh.k_empty[i]), 1); }
    for (int i = 0; i < NUM_V_STAGES; ++i) { mbar_init(smem_u32(&sh.v_full[i]), 1); mbar_init(smem_u32(&sh.v_empty[i]), 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&sh.s_full[i]), 1);
      mbar_init(smem_u32(&sh.p_ready[i]), 128);
      mbar_init(smem_u32(&sh.o_full[i]), 1);
      mbar_init(smem_u32(&sh.o_empty[i]), 256);
    }
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
      uint32_t g = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const int2 w = items[item];
        if (w.x < 0) continue;
        const int b = w.x & 0xffff, head = w.x >> 16, qblk = w.y;
        const SeqInfo s = load_seq(a, b);
        const int m0 = qblk * BLK;
        const int row0 = static_cast<int>(s.start) + m0;
        const int col0 = head * HEAD_DIM;
        // Q: wait until the previous item's score MMAs have drained the buffer
        ok = mbar_wait(smem_u32(&sh.q_empty), (it & 1) ^ 1, abort_flag, a.status, WAIT_PRODUCER);
        if (!ok) break;
        mbar_arrive_expect_tx(smem_u32(&sh.q_full), TILE_BYTES);
        tma_load_2d(smem_u32(sh.q), &maps.q, smem_u32(&sh.q_full), col0, row0);
        tma_load_2d(smem_u32(sh.q) + HALF_TILE_BYTES, &maps.q, smem_u32(&sh.q_full), col0 + 64, row0);
        const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
        for (int idx = 0; idx < kr.count() && ok; ++idx) {
          const int nb = kr.at(idx);
          if (classify_tile(m0, nb * BLK, s, a.mask) == TILE_SKIP) continue;
          const int krow = static_cast<int>(s.start) + nb * BLK;
          const uint32_t ks = g % NUM_K_STAGES, kph = (g / NUM_K_STAGES) & 1;
          ok = mbar_wait(smem_u32(&sh.k_empty[ks]), kph ^ 1, abort_flag, a.status, WAIT_PRODUCER);
          if (!ok) break;
          mbar_arrive_expect_tx(smem_u32(&sh.k_full[ks]), TILE_BYTES);
          tma_load_2d(smem_u32(sh.k[ks]), &maps.k, smem_u32(&sh.k_full[ks]), col0, krow);
          tma_load_2d(smem_u32(sh.k[ks]) + HALF_TILE_BYTES, &maps.k, smem_u32(&sh.k_full[ks]), col0 + 64, krow);
          const uint32_t vs = g % NUM_V_STAGES, vph = (g / NUM_V_STAGES) & 1;
          ok = mbar_wait(smem_u32(&sh.v_empty[vs]), vph ^ 1, abort_flag, a.status, WAIT_PRODUCER);
          if (!ok) break;
          mbar_arrive_expect_tx(smem_u32(&sh.v_full[vs]), TILE_BYTES);
          tma_load_2d(smem_u32(sh.v[vs]), &maps.v, smem_u32(&sh.v_full[vs]), col0, krow);
          tma_load_2d(smem_u32(sh.v[vs]) + HALF_TILE_BYTES, &maps.v, smem_u32(&sh.v_full[vs]), col0 + 64, krow);
          ++g;
        }
        ++it;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_f16(IS_BF16 ? 1 : 0, BLK, BLK, 0, 0);       // Q (K-major) x K (K-major)
      constexpr uint32_t IDESC_O = idesc_f16(IS_BF16 ? 1 : 0, BLK, HEAD_DIM, 0, 1);  // P (TMEM) x V (N-major)
      uint32_t g = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
        const int2 w = items[item];
        if (w.x < 0) continue;
        const int b = w.x & 0xffff, qblk = w.y;
        const SeqInfo s = load_seq(a, b);
        const int m0 = qblk * BLK;
        const uint32_t ob = it & 1;
        const uint32_t o_tmem = tmem + (ob ? TMEM_O1 : TMEM_O0);
        ok = mbar_wait(smem_u32(&sh.q_full), it & 1, abort_flag, a.status, WAIT_MMA);
        if (!ok) break;
        ok = mbar_wait(smem_u32(&sh.o_empty[ob]), ((it >> 1) & 1) ^ 1, abort_flag, a.status, WAIT_MMA);
        if (!ok) break;
        tc_fence_after();
        const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
        bool have_prev = false;
        uint32_t prev_g = 0, n_pv = 0;
        // issues O += P V for the key block whose scores were issued as tile `pg`
        auto issue_pv = [&](uint32_t pg) -> bool {
          const uint32_t sb = pg & 1, ph = (pg >> 1) & 1;
          if (!mbar_wait(smem_u32(&sh.p_ready[sb]), ph, abort_flag, a.status, WAIT_MMA)) return false;
          const uint32_t vs = pg % NUM_V_STAGES, vph = (pg / NUM_V_STAGES) & 1;
          if (!mbar_wait(smem_u32(&sh.v_full[vs]), vph, abort_flag, a.status, WAIT_MMA)) return false;
          tc_fence_after();
          const uint32_t p_tmem = tmem + (sb ? TMEM_S1 : TMEM_S0);
          const uint32_t vbase = smem_u32(sh.v[vs]);
#pragma unroll
          for (int kk = 0; kk < BLK / 16; ++kk) {
            // A: 16 key columns of P = 8 TMEM columns; B: 16 key rows of V (N-major, two 64-wide halves)
            const uint64_t bd = smem_desc_sw128(vbase + kk * 2048, HALF_TILE_BYTES, 1024);
            mma_ts(o_tmem, p_tmem + kk * 8, bd, IDESC_O, (n_pv > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(smem_u32(&sh.v_empty[vs]));
          ++n_pv;
          return true;
        };
        for (int idx = 0; idx < kr.count() && ok; ++idx) {
          const int nb = kr.at(idx);
          if (classify_tile(m0, nb * BLK, s, a.mask) == TILE_SKIP) continue;
          const uint32_t ks = g % NUM_K_STAGES, kph = (g / NUM_K_STAGES) & 1;
          ok = mbar_wait(smem_u32(&sh.k_full[ks]), kph, abort_flag, a.status, WAIT_MMA);
          if (!ok) break;
          tc_fence_after();
          const uint32_t s_tmem = tmem + ((g & 1) ? TMEM_S1 : TMEM_S0);
          const uint32_t qbase = smem_u32(sh.q), kbase = smem_u32(sh.k[ks]);
#pragma unroll
          for (int kk = 0; kk < HEAD_DIM / 16; ++kk) {
            // 16 feature columns = 32 bytes inside a 64-column (128-byte) box; boxes are 16 KB apart
            const uint32_t off = (kk >> 2) * HALF_TILE_BYTES + (kk & 3) * 32;
            const uint64_t ad = smem_desc_sw128(qbase + off, 16, 1024);
            const uint64_t bd = smem_desc_sw128(kbase + off, 16, 1024);
            mma_ss(s_tmem, ad, bd, IDESC_S, kk > 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&sh.k_empty[ks]));
          tc_commit(smem_u32(&sh.s_full[g & 1]));
          if (have_prev) ok = issue_pv(prev_g);
          prev_g = g;
          have_prev = true;
          ++g;
        }
        if (!ok) break;
        tc_commit(smem_u32(&sh.q_empty));  // every score MMA of this item has been issued
        if (have_prev) ok = issue_pv(prev_g);
        if (!ok) break;
        tc_commit(smem_u32(&sh.o_full[ob]));
        ++it;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue groups
    const int wg = (warp - 4) >> 2;                 // 0 or 1
    const int row = ((warp & 3) << 5) | lane;       // TMEM lane = query row inside the block
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const float c1 = 0.5f * a.alpha;
    uint32_t g = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total_items && ok; item += gridDim.x) {
      const int2 w = items[item];
      if (w.x < 0) continue;
      const int b = w.x & 0xffff, head = w.x >> 16, qblk = w.y;
      const SeqInfo s = load_seq(a, b);
      const int m0 = qblk * BLK;
      const int m = m0 + row;
      const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
      for (int idx = 0; idx < kr.count() && ok; ++idx) {
        const int nb = kr.at(idx);
        const int cls = classify_tile(m0, nb * BLK, s, a.mask);
        if (cls == TILE_SKIP) continue;
        if ((g & 1) == static_cast<uint32_t>(wg)) {
          const uint32_t sb = g & 1, ph = (g >> 1) & 1;
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.s_full[sb]), ph, abort_flag, a.status, WAIT_EPILOGUE));
          if (!ok) break;
          tc_fence_after();
          const uint32_t s_addr = tmem + lane_addr + (sb ? TMEM_S1 : TMEM_S0);
          const int n0 = nb * BLK;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t sv[32];
            tmem_ld32(s_addr + c * 32, sv);
            tmem_wait_ld();
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float u0 = c1 * __uint_as_float(sv[2 * i]);
              const float u1 = c1 * __uint_as_float(sv[2 * i + 1]);
              float p0 = fmaf(u0, tanh_approx(u0), u0);
              float p1 = fmaf(u1, tanh_approx(u1), u1);
              if (cls == TILE_PARTIAL) {
                const int n = n0 + c * 32 + 2 * i;
                if (!(m < s.len && n < s.len && keep(m, n, s, a.mask))) p0 = 0.f;
                if (!(m < s.len && n + 1 < s.len && keep(m, n + 1, s, a.mask))) p1 = 0.f;
              }
              pk[i] = pack2<IS_BF16>(p0, p1);
            }
            tmem_st16(s_addr + c * 16, pk);
          }
          if (n0 + BLK > s.len) {
            // Key rows past the end of the sequence belong to someone else (or to nobody) and may
            // hold anything, NaN included; their P columns are exact zeros, but 0 * NaN is NaN,
            // so the V rows themselves are cleared before the MMA reads the tile.
            const uint32_t vs = g % NUM_V_STAGES, vph = (g / NUM_V_STAGES) & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.v_full[vs]), vph, abort_flag, a.status, WAIT_EPILOGUE));
            if (!ok) break;
            zero_tile_rows(sh.v[vs], s.len - n0, row);
          }
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(smem_u32(&sh.p_ready[sb]));
        }
        ++g;
      }
      if (!ok) break;
      // ---- O leaves TMEM: group wg converts columns [64*wg, 64*wg+64) of its row
      const uint32_t ob = it & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.o_full[ob]), (it >> 1) & 1, abort_flag, a.status, WAIT_EPILOGUE));
      if (!ok) break;
      tc_fence_after();
      const uint32_t o_addr = tmem + lane_addr + (ob ? TMEM_O1 : TMEM_O0) + wg * 64;
      uint32_t ov0[32], ov1[32];
      tmem_ld32(o_addr, ov0);
      tmem_ld32(o_addr + 32, ov1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(smem_u32(&sh.o_empty[ob]));
      if (m < s.len) {
        const float sc = row_scale(a, s.start + m);
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<unsigned short*>(a.o) +
                                              (s.start + m) * a.o_rs + head * HEAD_DIM + wg * 64);
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

  // ---------------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    if (*abort_flag) {
      // a wait gave up: let copies and MMAs in flight finish before the TMEM is released
      const unsigned long long t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
    }
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------

}  // namespace

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [rows, H*128] 16-bit matrix, box = 64 columns x 128 rows, 128-byte swizzle, zero fill out of range.
bool make_map(CUtensorMap* m, const void* base, long long rows, long long width, long long row_stride, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
  cuuint32_t box[2] = {64, BLK};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  });
  return n;
}

template <typename T>
static cudaError_t launch_prep_t(const KernelArgs& a, int* ws, const WorkspaceLayout& w, bool backward, cudaStream_t st) {
  build_block_index<<<1, 1024, 0, st>>>(a, ws, w);
  const int blocks = sm_count() * 2;
  if (!backward)
    build_work_items<T><<<blocks, 256, 0, st>>>(a, ws, w, reinterpret_cast<T*>(a.o), a.o_rs, a.H * a.Dv,
                                                (T*)nullptr, 0, 0, (T*)nullptr, 0, 0);
  else
    build_work_items<T><<<blocks, 256, 0, st>>>(a, ws, w, reinterpret_cast<T*>(a.dq), a.dq_rs, a.H * a.Dqk,
                                                reinterpret_cast<T*>(a.dk), a.dk_rs, a.H * a.Dqk,
                                                reinterpret_cast<T*>(a.dv), a.dv_rs, a.H * a.Dv);
  return cudaGetLastError();
}

cudaError_t launch_prep(const KernelArgs& a, bool bf16, int* ws, const WorkspaceLayout& w, bool backward,
                        cudaStream_t st) {
  return bf16 ? launch_prep_t<__nv_bfloat16>(a, ws, w, backward, st) : launch_prep_t<__half>(a, ws, w, backward, st);
}

}  // namespace tc

bool tc_supported(const B200HstuParams& p, const KernelArgs& a, int pass) {
  if (p.flags & B200_HSTU_FLAG_FORCE_SIMT) return false;
  if (p.dtype != B200_HSTU_BF16 && p.dtype != B200_HSTU_F16) return false;
  if (a.Dqk != tc::HEAD_DIM || a.Dv != tc::HEAD_DIM) return false;
  if (!a.mask.causal) return false;
  if (a.T <= 0 || a.B <= 0) return false;
  if (a.T >= (1LL << 31) - 256 || a.H >= 32768) return false;
  // TMA: 16-byte aligned bases and row strides; vector stores: 16-byte aligned output rows
  auto ok16 = [](const void* ptr, long long row_stride) {
    return (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) && (row_stride % 8 == 0);
  };
  if (!ok16(a.q, a.q_rs) || !ok16(a.k, a.k_rs) || !ok16(a.v, a.v_rs)) return false;
  if (pass == 0 && !ok16(a.o, a.o_rs)) return false;
  if (pass == 1 && (!ok16(a.d_o, a.do_rs) || !ok16(a.dq, a.dq_rs) || !ok16(a.dk, a.dk_rs) || !ok16(a.dv, a.dv_rs)))
    return false;
  return true;
}

size_t tc_workspace_bytes(const KernelArgs& a, int pass) {
  (void)pass;
  const tc::WorkspaceLayout w = tc::workspace_layout(a.T, a.B, a.H);
  return (static_cast<size_t>(w.total_ints) * sizeof(int) + 255) & ~static_cast<size_t>(255);
}

int tc_launch_count(const KernelArgs& a, int pass) {
  (void)a;
  return pass == 0 ? 3 : 4;
}

cudaError_t tc_forward(const KernelArgs& a, int dtype, void* workspace, cudaStream_t st) {
  using namespace tc;
  const bool bf16 = dtype == B200_HSTU_BF16;
  const WorkspaceLayout w = workspace_layout(a.T, a.B, a.H);
  int* ws = reinterpret_cast<int*>(workspace);
  TensorMaps maps;
  const long long width = (long long)a.H * HEAD_DIM;
  if (!make_map(&maps.q, a.q, a.T, width, a.q_rs, bf16) || !make_map(&maps.k, a.k, a.T, width, a.k_rs, bf16) ||
      !make_map(&maps.v, a.v, a.T, width, a.v_rs, bf16))
    return cudaErrorInvalidValue;
  cudaError_t e = launch_prep(a, bf16, ws, w, false, st);
  if (e != cudaSuccess) return e;
  const size_t smem = sizeof(FwdShared) + 1024;
  auto kern = bf16 ? hstu_fwd_tc<true> : hstu_fwd_tc<false>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  long long grid = w.max_items < sm_count() ? w.max_items : sm_count();
  if (grid < 1) grid = 1;
  kern<<<static_cast<unsigned>(grid), FWD_THREADS, smem, st>>>(maps, a, ws, w.off_items);
  return cudaGetLastError();
}


}  // namespace hstu
