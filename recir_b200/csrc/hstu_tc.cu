// Tensor-core HSTU jagged attention for sm_100a: TMA tile loads, tcgen05 MMAs with TMEM
// accumulators, the scale/SiLU/mask epilogue fused on the accumulator.
//
// Shapes served: bf16 or fp16, Dqk == Dv == 128, causal mask (with every option of the
// mask rule).  Anything else is served by the CUDA-core kernels.
//
// Work decomposition.  A small device-side pass builds a work list of (sequence, head,
// 128-row block) items ordered so that expensive items come first and items that read the same
// K/V rows sit close together; persistent CTAs (one per SM) claim entries of the list dynamically
// (an atomic cursor, read by one scheduler warp per CTA).  The forward kernel is warp-specialised:
//   warp 0      TMA producer: Q tile of the item, then K and V tiles of every kept key block
//   warp 1      MMA issuer (one elected lane): S = Q K^T into TMEM, O += P V from TMEM
//   warp 2      work-item scheduler (claims items, classifies their tiles, feeds the item ring)
//   warps 4-7   epilogue group 0   } both groups work on EVERY key tile, group g on score columns
//   warps 8-11  epilogue group 1   } [64 g, 64 g + 64): read S from TMEM, apply alpha / SiLU / mask,
//                                    write P (16-bit) back over S
// The output scale (1/N or attn_scale) is a per-query-row factor, so it is applied once
// when O leaves TMEM, not per score.
#define SM100_OUTLINE_WAIT_SLOW_PATH  // one shared copy of the wait loop: see sm100_ptx.cuh
#include <cuda.h>
#include <cuda_runtime.h>

#include <stdio.h>
#include <stdlib.h>

#include <mutex>

#include "hstu_launch.h"
#include "hstu_tc_common.cuh"
#include "hstu_tc_host.h"
#include "sm100_pair.cuh"

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

// out[j] = sum_{i > j} in[i] for j in [0, n): exclusive suffix sum, one CTA of up to 1024 threads (whole
// warps).  Every thread sums a contiguous chunk; the per-thread totals are scanned with warp shuffles
// (two block barriers instead of the twenty of a shared-memory scan).
__device__ void suffix_sum_exclusive(const int* in, int* out, long long n, int* sh /*>= 64 ints*/) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nwarps = nt >> 5;
  const long long chunk = (n + nt - 1) / nt;
  const long long beg = (long long)tid * chunk;
  long long end = beg + chunk;
  if (end > n) end = n;
  int local = 0;
  for (long long i = beg; i < end; ++i) local += in[i];
  // v = sum over the lanes >= this one of the warp
  int v = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int t = __shfl_down_sync(0xffffffffu, v, off);
    if (lane + off < 32) v += t;
  }
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nwarps ? sh[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_down_sync(0xffffffffu, t, off);
      if (lane + off < 32) t += u;
    }
    sh[32 + lane] = t;  // sum of the totals of warps >= lane
  }
  __syncthreads();
  int run = (v - local) + (warp + 1 < nwarps ? sh[32 + warp + 1] : 0);  // everything owned by later threads
  for (long long i = end - 1; i >= beg; --i) {
    const int x = in[i];
    out[i] = run;
    run += x;
  }
  __syncthreads();
}

// The three per-block-count tables (histogram, suffix counts, starts) live in shared memory when they
// fit (tables_in_smem; 3 * nbins ints of dynamic shared memory), so that the dozen dependent phases of
// this single-CTA kernel pay shared-memory instead of global-memory latency; the suffix counts are
// copied to the workspace at the end for build_work_items.
__device__ __forceinline__ void block_index_body(const KernelArgs& a, int* ws, const WorkspaceLayout& w, int tables_in_smem,
                                                 int* sh /* 1024 ints */, int* tab) {
  int* sorted = ws + w.off_sorted;
  int* hist = tables_in_smem ? tab : ws + w.off_hist;
  int* cnt = tables_in_smem ? tab + w.nbins : ws + w.off_cnt;
  int* start = tables_in_smem ? tab + 2 * w.nbins : ws + w.off_start;
  const int tid = threadIdx.x;
  for (long long i = tid; i < w.nbins; i += blockDim.x) hist[i] = 0;
  // block count of the first sequence of this thread stays in a register for the second pass
  long long nb_first = 0;
  if (tid < a.B) {
    nb_first = blocks_of(a, tid);
    if (nb_first > w.nbins - 1) nb_first = w.nbins - 1;  // cannot happen for offsets within [0, T]
  }
  __syncthreads();
  for (int b = tid; b < a.B; b += blockDim.x) {
    long long nb = nb_first;
    if (b != tid) {
      nb = blocks_of(a, b);
      if (nb > w.nbins - 1) nb = w.nbins - 1;
    }
    atomicAdd(&hist[nb], 1);
  }
  __syncthreads();
  suffix_sum_exclusive(hist, cnt, w.nbins, sh);  // cnt[j] = #sequences with more than j blocks
  for (long long i = tid; i < w.nbins; i += blockDim.x) hist[i] = 0;  // reuse as fill counters
  __syncthreads();
  for (int b = tid; b < a.B; b += blockDim.x) {
    long long nb = nb_first;
    if (b != tid) {
      nb = blocks_of(a, b);
      if (nb > w.nbins - 1) nb = w.nbins - 1;
    }
    if (nb > 0) sorted[cnt[nb] + atomicAdd(&hist[nb], 1)] = b;
  }
  __syncthreads();
  // start[j] = H * sum_{j' > j} cnt[j'] : items of the highest block index come first
  suffix_sum_exclusive(cnt, start, w.nbins, sh);
  for (long long i = tid; i < w.nbins; i += blockDim.x) start[i] *= a.H;
  __syncthreads();
  if (tid == 0) {
    // The item array holds max_items = H * (T / 128 + B) entries, which covers every batch whose
    // sequences do not overlap.  Offsets that go backwards are clamped one sequence at a time
    // (load_seq), so a malformed array such as [0, T, 0, T, ...] can describe more blocks than that:
    // the list is cut at the capacity (the extra items are dropped) and the call is flagged.
    long long total = static_cast<long long>(start[0]) + static_cast<long long>(cnt[0]) * a.H;
    if (total < 0 || total > w.max_items) {
      total = w.max_items;
      if (a.status) atomicOr(a.status, 1);
    }
    ws[0] = static_cast<int>(total);
    ws[1] = cnt[0];
  }
  // chunk_base[c] = items owned by the first c * chunk_seqs sequences of the sorted order:
  // sequence i has more than j blocks iff i < cnt[j], so its block count is #{j : cnt[j] > i}
  int* chunk_base = ws + w.off_chunk;
  const int n_seq = cnt[0];
  const int n_chunks = (n_seq + w.chunk_seqs - 1) / w.chunk_seqs;
  for (int c = tid; c <= n_chunks; c += blockDim.x) {
    const long long lim = min((long long)c * w.chunk_seqs, (long long)n_seq);
    long long sum = 0;
    for (long long j = 0; j < w.nbins; ++j) {
      const int v = cnt[j];
      if (v == 0) break;
      sum += v < lim ? v : lim;
    }
    chunk_base[c] = static_cast<int>(sum * a.H);
  }
  if (tables_in_smem) {
    int* g_cnt = ws + w.off_cnt;
    int* g_start = ws + w.off_start;
    for (long long i = tid; i < w.nbins; i += blockDim.x) {
      g_cnt[i] = cnt[i];
      g_start[i] = start[i];
    }
  }
  if (a.ds_tile_base != nullptr) {
    // Backward with stored dS tiles: first tile of every sequence = exclusive prefix sum of the sequences'
    // tile counts (per head).  Every thread sums a contiguous run of sequences; the per-thread totals are
    // scanned with warp shuffles.
    long long* tile_base = const_cast<long long*>(a.ds_tile_base);
    const int nt = blockDim.x, lane = tid & 31, wid = tid >> 5;
    const long long chunk = (a.B + nt - 1) / nt;
    long long b0 = static_cast<long long>(tid) * chunk, b1 = b0 + chunk;
    if (b0 > a.B) b0 = a.B;
    if (b1 > a.B) b1 = a.B;
    long long local = 0;
    for (long long b = b0; b < b1; ++b) local += ds_tiles_of(blocks_of(a, static_cast<int>(b)), a.ds_square);
    long long incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    long long* wtot = reinterpret_cast<long long*>(sh);  // one entry per warp
    __syncthreads();
    if (lane == 31) wtot[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      long long v = lane < (nt >> 5) ? wtot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      wtot[lane] = v;
    }
    __syncthreads();
    long long base = (wid > 0 ? wtot[wid - 1] : 0) + incl - local;
    for (long long b = b0; b < b1; ++b) {
      tile_base[b] = base;
      base += ds_tiles_of(blocks_of(a, static_cast<int>(b)), a.ds_square);
    }
  }
}

__global__ void __launch_bounds__(1024) build_block_index(KernelArgs a, int* ws, WorkspaceLayout w, int tables_in_smem) {
  __shared__ int sh[1024];
  extern __shared__ int tab[];
  grid_launch_dependents();  // build_work_items may be made resident now; it waits for this kernel to finish
  block_index_body(a, ws, w, tables_in_smem, sh, tab);
}

// One thread per work-list entry: decode its rank into (sequence, head, block index).
// `stride` is the grid of the main kernels: CTA c starts with entry c and claims further entries
// from a cursor, so the list only has to be in a good ORDER (expensive items early, items that
// share K/V or Q/dO rows close together); no static deal is needed.
// Also zeroes the output rows no sequence owns (rows at or past the last offset).
template <typename T>
__device__ __forceinline__ void work_items_body(const KernelArgs& a, int* ws, const WorkspaceLayout& w, int stride,
                                                int tables_in_smem, int* tab, long long gtid, long long gsz, T* z0,
                                                long long rs0, int w0, T* z1, long long rs1, int w1, T* z2,
                                                long long rs2, int w2) {
  const int* sorted = ws + w.off_sorted;
  const int* cnt = ws + w.off_cnt;
  const int* chunk_base = ws + w.off_chunk;
  int2* items = reinterpret_cast<int2*>(ws + w.off_items);
  const int total = ws[0];
  // the two tables every thread searches are copied to shared memory first when they fit
  // (tables_in_smem: nbins + n_chunks + 1 ints of dynamic shared memory)
    if (tables_in_smem) {
    const int n_chunks1 = (ws[1] + w.chunk_seqs - 1) / w.chunk_seqs + 1;
    int* s_cnt = tab;
    int* s_chunk = tab + w.nbins;
    for (long long i = threadIdx.x; i < w.nbins; i += blockDim.x) s_cnt[i] = cnt[i];
    for (int i = threadIdx.x; i < n_chunks1; i += blockDim.x) s_chunk[i] = chunk_base[i];
    __syncthreads();
    cnt = s_cnt;
    chunk_base = s_chunk;
  }
  for (long long slot = gtid; slot < total; slot += gsz) {
    const long long p = slot;  // rank in the list order
    // Rank p -> item.  The sorted sequences are cut into chunks of chunk_seqs; the list is
    // chunk-major, and inside a chunk block-index-major (highest block index = most expensive
    // first), then sequence, then head.  All items that read the same K/V (or Q/dO) rows are
    // therefore close together in the list and run at about the same time, which is what
    // keeps those rows in L2 between their readers.
    const int n_seq = ws[1];
    const int n_chunks = (n_seq + w.chunk_seqs - 1) / w.chunk_seqs;
    int lo = 0, hi = n_chunks - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (chunk_base[mid] <= p) lo = mid; else hi = mid - 1;
    }
    const int first = lo * w.chunk_seqs;
    const int n_c = min(w.chunk_seqs, n_seq - first);
    long long r = p - chunk_base[lo];
    // highest block index present in the chunk: largest j with cnt[j] > first
    long long jl = 0, jh = w.nbins - 1;
    while (jl < jh) {
      const long long mid = (jl + jh + 1) >> 1;
      if (cnt[mid] > first) jl = mid; else jh = mid - 1;
    }
    int j = static_cast<int>(jl);
    for (; j > 0; --j) {
      const long long nj = (long long)min(cnt[j] - first, n_c) * a.H;
      if (r < nj) break;
      r -= nj;
    }
    const int i = static_cast<int>(r / a.H), head = static_cast<int>(r - (long long)i * a.H);
    int2 it;
    it.x = (first + i < n_seq) ? (sorted[first + i] | (head << 16)) : -1;
    it.y = j;
    items[slot] = it;
  }
  if (gtid == 0) {
    // CTA c starts with entry c; the rest of the list is claimed dynamically from these cursors
    ws[WS_CURSOR0] = stride;
    ws[WS_CURSOR1] = stride;
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

template <typename T>
__global__ void __launch_bounds__(256) build_work_items(KernelArgs a, int* ws, WorkspaceLayout w, int stride,
                                                        int tables_in_smem, T* z0,
                                                        long long rs0, int w0, T* z1, long long rs1, int w1,
                                                        T* z2, long long rs2, int w2) {
  extern __shared__ int tab[];
  grid_dependency_wait();    // build_block_index has finished and its tables are visible
  grid_launch_dependents();  // the main kernel may be made resident; it waits for this kernel to finish
  work_items_body<T>(a, ws, w, stride, tables_in_smem, tab, blockIdx.x * (long long)blockDim.x + threadIdx.x,
                     (long long)gridDim.x * blockDim.x, z0, rs0, w0, z1, rs1, w1, z2, rs2, w2);
}

// Both steps in one launch: a cluster of WORK_LIST_CLUSTER CTAs.  The CTA of rank 0 builds the tables (one
// CTA's work: a dozen dependent phases over the sequences), the cluster barrier publishes them, and all CTAs
// decode the entries.  One launch and no dependency between two grids: about a third less time in front of
// every main kernel than the two kernels above, which remain for tables too large for shared memory.
constexpr int WORK_LIST_CLUSTER = 8;
template <typename T>
__global__ void __launch_bounds__(1024) build_work_list(KernelArgs a, int* ws, WorkspaceLayout w, int stride, T* z0,
                                                       long long rs0, int w0, T* z1, long long rs1, int w1, T* z2,
                                                       long long rs2, int w2) {
  __shared__ int sh[1024];
  extern __shared__ int tab[];
  grid_launch_dependents();  // the main kernel may be made resident; it waits for this kernel to finish
  const uint32_t rank = cluster_cta_rank();
  if (rank == 0) block_index_body(a, ws, w, 1, sh, tab);
  __threadfence();
  cluster_sync_all();  // the tables in the workspace are complete and visible to the whole cluster
  work_items_body<T>(a, ws, w, stride, 1, tab, rank * (long long)blockDim.x + threadIdx.x,
                     (long long)WORK_LIST_CLUSTER * blockDim.x, z0, rs0, w0, z1, rs1, w1, z2, rs2, w2);
}

// ------------------------------------------------------------------------------------
// Forward kernel
// ------------------------------------------------------------------------------------

constexpr int NUM_K_STAGES = 2;
constexpr int NUM_V_STAGES = 3;
constexpr int FWD_THREADS = 384;
constexpr int TMEM_COLS = 512;
constexpr int TMEM_S0 = 0, TMEM_S1 = 128, TMEM_O0 = 256, TMEM_O1 = 384;
constexpr int META_RING = 16;

struct FwdShared {
  // tiles first: every tile base must be 1024-byte aligned for the 128-byte swizzle
  unsigned char q[TILE_BYTES];
  unsigned char k[NUM_K_STAGES][TILE_BYTES];
  unsigned char v[NUM_V_STAGES][TILE_BYTES];
  unsigned char o_stage[TILE_BYTES];  // O tile on its way to global memory (row-major, chunk-swizzled)
  unsigned long long q_full, q_empty;
  unsigned long long k_full[NUM_K_STAGES], k_empty[NUM_K_STAGES];
  unsigned long long v_full[NUM_V_STAGES], v_empty[NUM_V_STAGES];
  unsigned long long s_full[2], p_ready[2];
  unsigned long long o_full[2], o_empty[2];
  int meta[META_RING];  // per key tile, written by the producer: bit 0 = last tile of its item
  ItemRing ring;
  uint32_t tmem_base;
  int abort_flag;
};

struct TensorMaps {
  CUtensorMap q, k, v;
  CUtensorMap o;  // output (bulk stores of whole 128-row blocks)
};

// Optional cycle accounting (PROF): per-role wait/busy cycles, summed over CTAs into 14 ints.
enum { PF_MMA_TOTAL = 0, PF_MMA_KFULL, PF_MMA_PREADY, PF_MMA_VFULL, PF_MMA_ITEM, PF_EPI_TOTAL, PF_EPI_SFULL,
       PF_EPI_OFULL, PF_EPI_PARTIAL, PF_EPI_FULL, PF_N_PARTIAL, PF_N_FULL, PF_PROD_WAIT, PF_PROD_TOTAL };

// Event trace (PROF only): CTA 0 records 32-bit clock samples into status[16 + slot]; the
// profiling caller passes a status buffer large enough (16 + TRACE_SLOTS ints).
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

// Tile class for candidates past the first 32 of an item (sequences longer than 32 blocks only; the
// scheduler warp classifies the first 32): kept out of line so that this rarely executed code does not
// sit in the middle of the per-item paths.
static __device__ __noinline__ int classify_tile_cold(int m0, int n0, SeqInfo s, MaskOpts o) {
  return classify_tile(m0, n0, s, o, true);
}

// One 32-column chunk of scores -> 16 packed 16-bit pairs of P; `bits` = kept columns of the chunk.
template <bool IS_BF16, bool MASKED>
__device__ __forceinline__ void silu_chunk(const uint32_t (&sv)[32], uint32_t (&pk)[16], uint64_t c1, uint32_t bits) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t p2 = silu_pair<IS_BF16>(sv[2 * i], sv[2 * i + 1], c1);
    if (MASKED) p2 &= pair_mask(bits, 2 * i);
    pk[i] = p2;
  }
}

template <bool IS_BF16, bool PROF>
__global__ void __launch_bounds__(FWD_THREADS, 1)
hstu_fwd_tc(const __grid_constant__ TensorMaps maps, KernelArgs a, int* __restrict__ ws, long long off_items) {
  extern __shared__ unsigned char smem_raw[];
  // dynamic shared memory is only guaranteed 16-byte aligned: round up to 1024
  FwdShared& sh = *reinterpret_cast<FwdShared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  grid_dependency_wait();  // launched as a dependent of build_work_items: the work list is complete from here on
  const int total_items = ws[0];
  if (static_cast<int>(blockIdx.x) >= total_items) return;  // uniform per CTA
  const int2* items = reinterpret_cast<const int2*>(ws + off_items);
  volatile int* abort_flag = &sh.abort_flag;
  int* prof = ws + 2;

  if (threadIdx.x == 0) {
    sh.abort_flag = 0;
    item_ring_init(sh.ring);
    mbar_init(smem_u32(&sh.q_full), 1);
    mbar_init(smem_u32(&sh.q_empty), 1);
    for (int i = 0; i < NUM_K_STAGES; ++i) { mbar_init(smem_u32(&sh.k_full[i]), 1); mbar_init(smem_u32(&sh.k_empty[i]), 1); }
    for (int i = 0; i < NUM_V_STAGES; ++i) { mbar_init(smem_u32(&sh.v_full[i]), 1); mbar_init(smem_u32(&sh.v_empty[i]), 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&sh.s_full[i]), 1);
      mbar_init(smem_u32(&sh.p_ready[i]), 256);
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

  // warps 0-3 (producer, MMA issuer, two idle) give registers to the eight epilogue warps
  if (warp < 4) setmaxnreg_dec<152>(); else setmaxnreg_inc<168>();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer / tile scheduler
    // Whole warp on one control path; one elected lane issues the copies.
    {
      if (lane == 0) {
        prefetch_tensormap(&maps.q);
        prefetch_tensormap(&maps.k);
        prefetch_tensormap(&maps.v);
      }
      long long pf_wait = 0, pf_total = 0;
      Stopwatch<PROF> sw_total, sw;
      sw_total.start();
      uint32_t g = 0, it = 0, ks = 0, kph = 0, vs = 0, vph = 0;
      bool ok = true;
      auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
        sw.start();
        const bool r = __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_PRODUCER));
        sw.stop(pf_wait);
        return r;
      };
      int2 w;
      SeqInfo s;
      uint32_t todo0 = 0u, full0 = 0u;
      for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w, s, todo0, full0, ok, abort_flag, a.status, WAIT_PRODUCER); ++n_item) {
        const int head = w.x >> 16, qblk = w.y;
        const int m0 = qblk * BLK;
        const int row0 = static_cast<int>(s.start) + m0;
        const int col0 = head * HEAD_DIM;
        // Q: wait until the previous item's score MMAs have drained the buffer
        ok = wait_all(&sh.q_empty, (it & 1) ^ 1);
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(smem_u32(&sh.q_full), TILE_BYTES);
          tma_load_2d(smem_u32(sh.q), &maps.q, smem_u32(&sh.q_full), col0, row0);
          tma_load_2d(smem_u32(sh.q) + HALF_TILE_BYTES, &maps.q, smem_u32(&sh.q_full), col0 + 64, row0);
        }
        __syncwarp();
        const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
        const int cnt = kr.count();
        // 32 candidate key blocks are classified at a time, one per lane; the last candidate of an
        // item (the diagonal block, or the last block of the sequence) is never skipped
        for (int base = 0; base < cnt && ok; base += 32) {
          uint32_t todo = todo0;  // the scheduler warp classified the first 32 candidates
          if (base > 0) {
            int my_cls = TILE_SKIP;
            if (base + lane < cnt) my_cls = classify_tile_cold(m0, kr.at(base + lane) * BLK, s, a.mask);
            todo = __ballot_sync(0xffffffffu, my_cls != TILE_SKIP);
          }
          while (todo != 0u && ok) {
            const int bit = __ffs(todo) - 1;
            todo &= todo - 1;
            const int idx = base + bit;
            const int krow = static_cast<int>(s.start) + kr.at(idx) * BLK;
            ok = wait_all(&sh.k_empty[ks], kph ^ 1);
            if (!ok) break;
            if (elect_one()) {
              sh.meta[g & (META_RING - 1)] = (idx == cnt - 1) ? 1 : 0;
              mbar_arrive_expect_tx(smem_u32(&sh.k_full[ks]), TILE_BYTES);
              tma_load_2d(smem_u32(sh.k[ks]), &maps.k, smem_u32(&sh.k_full[ks]), col0, krow);
              tma_load_2d(smem_u32(sh.k[ks]) + HALF_TILE_BYTES, &maps.k, smem_u32(&sh.k_full[ks]), col0 + 64, krow);
            }
            __syncwarp();
            ok = wait_all(&sh.v_empty[vs], vph ^ 1);
            if (!ok) break;
            if (elect_one()) {
              mbar_arrive_expect_tx(smem_u32(&sh.v_full[vs]), TILE_BYTES);
              tma_load_2d(smem_u32(sh.v[vs]), &maps.v, smem_u32(&sh.v_full[vs]), col0, krow);
              tma_load_2d(smem_u32(sh.v[vs]) + HALF_TILE_BYTES, &maps.v, smem_u32(&sh.v_full[vs]), col0 + 64, krow);
            }
            __syncwarp();
            ++g;
            if (++ks == NUM_K_STAGES) { ks = 0; kph ^= 1; }
            if (++vs == NUM_V_STAGES) { vs = 0; vph ^= 1; }
          }
        }
        ++it;
      }
      sw_total.stop(pf_total);
      if (PROF && lane == 0) { atomicAdd(prof + PF_PROD_WAIT, (int)(pf_wait >> 6)); atomicAdd(prof + PF_PROD_TOTAL, (int)(pf_total >> 6)); }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp walks the loop (uniform control flow, uniform descriptor arithmetic);
    // one elected lane issues the tcgen05 instructions.
    {
      constexpr uint32_t IDESC_S = idesc_f16(IS_BF16 ? 1 : 0, BLK, BLK, 0, 0);       // Q (K-major) x K (K-major)
      constexpr uint32_t IDESC_O = idesc_f16(IS_BF16 ? 1 : 0, BLK, HEAD_DIM, 0, 1);  // P (TMEM) x V (N-major)
      constexpr uint32_t HI = desc_hi_sw128(1024);
      const uint32_t q_lo = desc_lo_sw128(smem_u32(sh.q), 16);
      const uint32_t k_lo0 = desc_lo_sw128(smem_u32(sh.k[0]), 16);
      const uint32_t v_lo0 = desc_lo_sw128(smem_u32(sh.v[0]), HALF_TILE_BYTES);
      long long pf[5] = {0, 0, 0, 0, 0};
      Stopwatch<PROF> sw_total, sw;
      sw_total.start();
      uint32_t g = 0, it = 0, ks = 0, kph = 0, vs_cur = 0, vph_cur = 0;
      bool ok = true;
      auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_MMA));
      };
      int2 w_unused;
      SeqInfo s_unused;
      uint32_t t_unused = 0u, f_unused = 0u;
      for (uint32_t n_item = 0; ok && next_item(sh.ring, n_item, w_unused, s_unused, t_unused, f_unused, ok, abort_flag, a.status, WAIT_MMA); ++n_item) {
        const uint32_t ob = it & 1;
        const uint32_t o_tmem = tmem + (ob ? TMEM_O1 : TMEM_O0);
        sw.start();
        ok = wait_all(&sh.q_full, it & 1);
        if (ok) ok = wait_all(&sh.o_empty[ob], ((it >> 1) & 1) ^ 1);
        sw.stop(pf[PF_MMA_ITEM]);
        if (!ok) break;
        bool have_prev = false;
        uint32_t prev_g = 0, prev_vs = 0, prev_vph = 0, n_pv = 0;
        // issues O += P V for the key tile whose scores were issued as tile `pg`
        auto issue_pv = [&](uint32_t pg, uint32_t vs, uint32_t vph) -> bool {
          const uint32_t sb = pg & 1, ph = (pg >> 1) & 1;
          sw.start();
          bool good = wait_all(&sh.p_ready[sb], ph);
          sw.stop(pf[PF_MMA_PREADY]);
          if (!good) return false;
          sw.start();
          good = wait_all(&sh.v_full[vs], vph);
          sw.stop(pf[PF_MMA_VFULL]);
          if (!good) return false;
          if (lane == 0) trace_event<PROF>(a.trace_buf, 0, pg, 2, 4);
          tc_fence_after();
          const uint32_t p_tmem = tmem + (sb ? TMEM_S1 : TMEM_S0);
          const uint32_t v_lo = v_lo0 + vs * (TILE_BYTES >> 4);
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < BLK / 16; ++kk) {
              // A: 16 key columns of P = 8 TMEM columns (keys 0..63 at columns 0..31, keys 64..127 at
              // columns 64..95: each epilogue group stores P over its own score columns);
              // B: 16 key rows of V (N-major, two 64-wide halves)
              mma_ts(o_tmem, p_tmem + (kk >> 2) * 64 + (kk & 3) * 8, desc_join(v_lo + kk * (2048 >> 4), HI), IDESC_O,
                     (n_pv > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(smem_u32(&sh.v_empty[vs]));
          }
          __syncwarp();
          if (lane == 0) trace_event<PROF>(a.trace_buf, 0, pg, 3, 4);
          ++n_pv;
          return true;
        };
        bool last = false;
        while (!last && ok) {
          sw.start();
          ok = wait_all(&sh.k_full[ks], kph);
          sw.stop(pf[PF_MMA_KFULL]);
          if (!ok) break;
          last = sh.meta[g & (META_RING - 1)] & 1;
          if (lane == 0) trace_event<PROF>(a.trace_buf, 0, g, 0, 4);
          tc_fence_after();
          const uint32_t s_tmem = tmem + ((g & 1) ? TMEM_S1 : TMEM_S0);
          const uint32_t k_lo = k_lo0 + ks * (TILE_BYTES >> 4);
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk) {
              // 16 feature columns = 32 bytes inside a 64-column (128-byte) box; boxes are 16 KB apart
              const uint32_t off = ((kk >> 2) * HALF_TILE_BYTES + (kk & 3) * 32) >> 4;
              mma_ss(s_tmem, desc_join(q_lo + off, HI), desc_join(k_lo + off, HI), IDESC_S, kk > 0 ? 1u : 0u);
            }
            tc_commit(smem_u32(&sh.k_empty[ks]));
            tc_commit(smem_u32(&sh.s_full[g & 1]));
          }
          __syncwarp();
          if (lane == 0) trace_event<PROF>(a.trace_buf, 0, g, 1, 4);
          if (have_prev) ok = issue_pv(prev_g, prev_vs, prev_vph);
          prev_g = g; prev_vs = vs_cur; prev_vph = vph_cur;
          have_prev = true;
          ++g;
          if (++ks == NUM_K_STAGES) { ks = 0; kph ^= 1; }
          if (++vs_cur == NUM_V_STAGES) { vs_cur = 0; vph_cur ^= 1; }
        }
        if (!ok) break;
        if (elect_one()) tc_commit(smem_u32(&sh.q_empty));  // every score MMA of this item has been issued
        __syncwarp();
        if (have_prev) ok = issue_pv(prev_g, prev_vs, prev_vph);
        if (!ok) break;
        if (elect_one()) tc_commit(smem_u32(&sh.o_full[ob]));
        __syncwarp();
        ++it;
      }
      sw_total.stop(pf[PF_MMA_TOTAL]);
      if (PROF && lane == 0)
        for (int i = 0; i < 5; ++i) atomicAdd(prof + i, (int)(pf[i] >> 6));
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ work-item scheduler
    run_item_scheduler<false>(sh.ring, a, items, total_items, ws + WS_CURSOR0, abort_flag);
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue groups
    const int wg = (warp - 4) >> 2;                 // 0 or 1
    const int row = ((warp & 3) << 5) | lane;       // TMEM lane = query row inside the block
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const uint64_t c1 = dup_f32x2(0.5f * a.alpha);
    const bool prof_thread = PROF && (threadIdx.x == 128 || threadIdx.x == 256);
    long long pf_total = 0, pf_sfull = 0, pf_ofull = 0, pf_part = 0, pf_fullt = 0, pf_fence = 0, pf_drain = 0;
    int n_part = 0, n_fullt = 0;
    Stopwatch<PROF> sw_total, sw;
    sw_total.start();
    uint32_t g = 0, it = 0;
    bool ok = true;
    // O of a finished item leaves TMEM: group wg converts columns [64 wg, 64 wg + 64) of its row.
    // It runs one key tile into the next item, so that the tensor cores already have new work
    // while the epilogue warps drain the previous accumulator.
    long long d_start = 0;
    int d_len = 0, d_m0 = 0, d_head = 0;
    uint32_t d_it = 0;
    bool drain_pending = false;
    auto drain_o = [&]() -> bool {
      // ---- O leaves TMEM: group wg converts columns [64*wg, 64*wg+64) of its row
      const uint32_t ob = d_it & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.o_full[ob]), (d_it >> 1) & 1, abort_flag, a.status, WAIT_EPILOGUE));
      if (!ok) return false;
      tc_fence_after();
      const uint32_t o_addr = tmem + lane_addr + (ob ? TMEM_O1 : TMEM_O0) + wg * 64;
      // Rows are handed to global memory through shared memory.  Each group stages its own 64
      // columns as a 128-row half tile in the 128-byte-swizzled box layout (16-byte chunk index
      // XOR (row & 7)).  A whole block then leaves as one bulk tensor store per group, which runs
      // in the background; the ragged last block of a sequence is copied out by the threads
      // (8 lanes write one 128-byte row segment, a warp 4 rows per instruction).
      {
        const float sc = d_m0 + row < d_len ? row_scale(a, d_start + d_m0 + row) : 0.f;
        const int tid_wg = row;  // 0..127 inside the group
        unsigned char* half = sh.o_stage + wg * HALF_TILE_BYTES;
        if (tid_wg == 0) bulk_wait_read_all();  // the previous item's store has read the staging buffer
        asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");
        unsigned char* my_row = half + row * 128;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t ov[32];
          tmem_ld32(o_addr + h * 32, ov);
          tmem_wait_ld(ov);
          if (h == 1) {
            tc_fence_before();
            mbar_arrive(smem_u32(&sh.o_empty[ob]));
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 x;
            x.x = pack2<IS_BF16>(__uint_as_float(ov[8 * j + 0]) * sc, __uint_as_float(ov[8 * j + 1]) * sc);
            x.y = pack2<IS_BF16>(__uint_as_float(ov[8 * j + 2]) * sc, __uint_as_float(ov[8 * j + 3]) * sc);
            x.z = pack2<IS_BF16>(__uint_as_float(ov[8 * j + 4]) * sc, __uint_as_float(ov[8 * j + 5]) * sc);
            x.w = pack2<IS_BF16>(__uint_as_float(ov[8 * j + 6]) * sc, __uint_as_float(ov[8 * j + 7]) * sc);
            *reinterpret_cast<uint4*>(my_row + (((h * 4 + j) ^ (row & 7)) << 4)) = x;
          }
        }
        const int rows_valid = d_len - d_m0;
        if (rows_valid >= BLK) {
          fence_proxy_async();
          asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");  // the group's half tile is staged
          if (tid_wg == 0) {
            tma_store_2d(&maps.o, smem_u32(half), d_head * HEAD_DIM + wg * 64, static_cast<int>(d_start) + d_m0);
            bulk_commit();
          }
        } else {
          asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");  // the group's half tile is staged
          const int chunk = tid_wg & 7;
          unsigned short* obase = reinterpret_cast<unsigned short*>(a.o) + (d_start + d_m0) * a.o_rs + d_head * HEAD_DIM +
                                  wg * 64 + chunk * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 16 + (tid_wg >> 3);
            if (r < rows_valid) {
              const uint4 x = *reinterpret_cast<const uint4*>(half + r * 128 + ((chunk ^ (r & 7)) << 4));
              *reinterpret_cast<uint4*>(obase + static_cast<long long>(r) * a.o_rs) = x;
            }
          }
        }
      }
      drain_pending = false;
      return true;
    };
    int2 w;
    SeqInfo s;
    uint32_t todo0 = 0u, full0 = 0u;
    // The loop runs once more after the last item (have_item == false, no tiles) so that the final
    // accumulator is drained by the same copy of the drain code as all the others.
    for (uint32_t n_item = 0; ok; ++n_item) {
      const bool have_item = next_item(sh.ring, n_item, w, s, todo0, full0, ok, abort_flag, a.status, WAIT_EPILOGUE);
      if (!ok) break;
      const int head = w.x >> 16, qblk = w.y;
      const int m0 = qblk * BLK;
      const int m = m0 + row;
      const RowMask rm = row_mask(m, s, a.mask);
      const BlockRange kr = key_blocks_for_query_block(m0, s, a.mask);
      const int cnt = kr.count();
      // Kept key blocks of this item, in order; 32 candidates are classified at a time (one per lane).
      int base_next = 0, cur_base = 0;
      uint32_t todo = 0u, full_bits = 0u;
      auto next_tile = [&](int& n0_out, bool& full_out) -> bool {
        while (todo == 0u) {
          if (base_next >= cnt) return false;
          cur_base = base_next;
          base_next += 32;
          if (cur_base == 0) {  // classified by the scheduler warp
            todo = todo0;
            full_bits = full0;
          } else {
            int my_cls = TILE_SKIP;
            if (cur_base + lane < cnt) my_cls = classify_tile_cold(m0, kr.at(cur_base + lane) * BLK, s, a.mask);
            todo = __ballot_sync(0xffffffffu, my_cls != TILE_SKIP);
            full_bits = __ballot_sync(0xffffffffu, my_cls == TILE_FULL);
          }
        }
        const int bit = __ffs(todo) - 1;
        todo &= todo - 1;
        n0_out = kr.at(cur_base + bit) * BLK;
        full_out = (full_bits >> bit) & 1u;
        return true;
      };
      auto s_addr_of = [&](uint32_t tile) -> uint32_t {
        return tmem + lane_addr + ((tile & 1) ? TMEM_S1 : TMEM_S0) + wg * 64;
      };
      auto wait_scores = [&](uint32_t tile) -> bool {
        sw.start();
        const bool r = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.s_full[tile & 1]), (tile >> 1) & 1, abort_flag,
                                                         a.status, WAIT_EPILOGUE));
        sw.stop(pf_sfull);
        if (r) tc_fence_after();
        return r;
      };
      // Both groups work on every key tile: group wg owns score columns [64 wg, 64 wg + 64), handled
      // as two 32-column chunks.  The chunk loads run ahead of the math: the second chunk is
      // fetched while the first is processed, and the first chunk of the NEXT tile is fetched
      // before this tile's P is handed to the MMA warp.
      uint32_t sa[32], sb2[32], pk[16];
      int n0 = 0, n0_next = 0;
      bool full = false, full_next = false;
      bool have = have_item && next_tile(n0, full);
      if (have) {
        if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, g, 0, 6);
        ok = wait_scores(g);
        if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, g, 1, 6);
        if (ok) tmem_ld32(s_addr_of(g), sa);
      }
      while ((have || (!have_item && drain_pending)) && ok) {
        bool have_next = false;
        if (have) {
          have_next = next_tile(n0_next, full_next);
          const uint32_t s_addr = s_addr_of(g);
          const uint32_t sb = g & 1;
          sw.start();
          tmem_wait_ld(sa);
          tmem_ld32(s_addr + 32, sb2);
          if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, g, 2, 6);
          if (full) {
            silu_chunk<IS_BF16, false>(sa, pk, c1, 0u);
            tmem_st16(s_addr, pk);  // P (16 columns per chunk) goes over the group's own score columns
            tmem_wait_ld(sb2);
            silu_chunk<IS_BF16, false>(sb2, pk, c1, 0u);
            tmem_st16(s_addr + 16, pk);
          } else {
            // A warp covers 32 consecutive rows, so on a diagonal tile most 32-column chunks are
            // entirely kept or entirely dropped for the whole warp: vote, and only the chunks that
            // straddle the mask boundary pay for per-element masking; dropped chunks skip the math.
            const unsigned long long bits = row_mask_bits64(rm, n0 + wg * 64);
            const uint32_t b0 = static_cast<uint32_t>(bits), b1 = static_cast<uint32_t>(bits >> 32);
            if (__all_sync(0xffffffffu, b0 == 0xffffffffu)) {
              silu_chunk<IS_BF16, false>(sa, pk, c1, 0u);
            } else if (__all_sync(0xffffffffu, b0 == 0u)) {
  #pragma unroll
              for (int i = 0; i < 16; ++i) pk[i] = 0u;
            } else {
              silu_chunk<IS_BF16, true>(sa, pk, c1, b0);
            }
            tmem_st16(s_addr, pk);
            tmem_wait_ld(sb2);
            if (__all_sync(0xffffffffu, b1 == 0xffffffffu)) {
              silu_chunk<IS_BF16, false>(sb2, pk, c1, 0u);
            } else if (__all_sync(0xffffffffu, b1 == 0u)) {
  #pragma unroll
              for (int i = 0; i < 16; ++i) pk[i] = 0u;
            } else {
              silu_chunk<IS_BF16, true>(sb2, pk, c1, b1);
            }
            tmem_st16(s_addr + 16, pk);
          }
          if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, g, 3, 6);
          if (n0 + BLK > s.len) {
            // Key rows past the end of the sequence belong to someone else (or to nobody) and may
            // hold anything, NaN included; their P columns are exact zeros, but 0 * NaN is NaN,
            // so the V rows themselves are cleared before the MMA reads the tile.
            const uint32_t vs = g % NUM_V_STAGES, vph = (g / NUM_V_STAGES) & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sh.v_full[vs]), vph, abort_flag, a.status, WAIT_EPILOGUE));
            if (!ok) break;
            zero_box_rows(sh.v[vs] + wg * HALF_TILE_BYTES, s.len - n0, BLK, row, 128);
          }
          if (have_next) {
            // scores of the next tile were issued before the MMA warp started waiting for this P
            ok = wait_scores(g + 1);
            if (!ok) break;
            tmem_ld32(s_addr_of(g + 1), sa);
          }
          tmem_wait_st();
          if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, g, 4, 6);
          tc_fence_before();
          mbar_arrive(smem_u32(&sh.p_ready[sb]));
          if (threadIdx.x == 128) trace_event<PROF>(a.trace_buf, 4096, g, 5, 6);
          if (full) { sw.stop(pf_fullt); ++n_fullt; } else { sw.stop(pf_part); ++n_part; }
          ++g;
        }
        if (drain_pending) { sw.start(); ok = drain_o(); sw.stop(pf_drain); }
        n0 = n0_next; full = full_next; have = have_next;
      }
      if (!ok || !have_item) break;
      // hand the accumulator over: it is drained after the first key tile of the next item
      d_start = s.start; d_len = s.len; d_m0 = m0; d_head = head; d_it = it;
      drain_pending = true;
      ++it;
    }
    if (row == 0) bulk_wait_all();  // shared memory must outlive the stores that read it
    sw_total.stop(pf_total);
    if (prof_thread) {
      atomicAdd(prof + PF_EPI_TOTAL, (int)(pf_total >> 6)); atomicAdd(prof + PF_EPI_SFULL, (int)(pf_sfull >> 6));
      atomicAdd(prof + PF_EPI_OFULL, (int)(pf_ofull >> 6)); atomicAdd(prof + PF_EPI_PARTIAL, (int)(pf_part >> 6));
      atomicAdd(prof + PF_EPI_FULL, (int)(pf_fullt >> 6)); atomicAdd(prof + PF_N_PARTIAL, (int)(pf_fence >> 6));
      atomicAdd(prof + PF_N_FULL, (int)(pf_drain >> 6));
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

// Tensor-map encoding is a driver call and fails with CUDA_ERROR_INVALID_CONTEXT on a thread that
// has no current context yet (a fresh worker thread, e.g. an autograd thread whose first CUDA work
// is this library).  If none is current, the primary context of the device that owns `device_ptr`
// is made current (cudaSetDevice initialises and binds it).
bool ensure_current_context(const void* device_ptr) {
  typedef CUresult (*GetCurrentFn)(CUcontext*);
  static GetCurrentFn get_current = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
  });
  CUcontext ctx = nullptr;
  if (get_current && get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr) return true;
  cudaPointerAttributes at;
  int dev = 0;
  if (cudaPointerGetAttributes(&at, device_ptr) == cudaSuccess && at.type == cudaMemoryTypeDevice) dev = at.device;
  return cudaSetDevice(dev) == cudaSuccess;
}

// [rows, H*128] 16-bit matrix, box = 64 columns x 128 rows, 128-byte swizzle, zero fill out of range.
bool make_map(CUtensorMap* m, const void* base, long long rows, long long width, long long row_stride, bool bf16) {
  return make_map_box(m, base, rows, width, row_stride, BLK, bf16);
}

// Encoded tensor maps are kept per (base, shape, stride, box, element type): a training step calls the same
// operators on the same buffers again and again, and each encoding is a driver call on the launch path.  The
// map holds nothing but those values, so a hit is exact; 64 entries, replaced round robin.
namespace {
struct MapKey {
  const void* base; long long rows, width, row_stride; int box_rows, kind;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && width == o.width && row_stride == o.row_stride && box_rows == o.box_rows &&
           kind == o.kind;
  }
};
struct MapCache {
  static constexpr int N = 64;
  std::mutex mu;
  MapKey key[N];
  CUtensorMap map[N];
  bool used[N] = {};
  int next = 0;
  bool find(const MapKey& k, CUtensorMap* out) {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < N; ++i)
      if (used[i] && key[i] == k) { *out = map[i]; return true; }
    return false;
  }
  void put(const MapKey& k, const CUtensorMap& m) {
    std::lock_guard<std::mutex> lock(mu);
    key[next] = k; map[next] = m; used[next] = true;
    next = (next + 1) % N;
  }
};
MapCache& map_cache() { static MapCache c; return c; }
}  // namespace

// Same with a box of 64 columns x `box_rows` rows (at most 256).
bool make_map_box(CUtensorMap* m, const void* base, long long rows, long long width, long long row_stride, int box_rows,
                  bool bf16) {
  const MapKey k{base, rows, width, row_stride, box_rows, bf16 ? 1 : 0};
  if (map_cache().find(k, m)) return true;
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error_stage("tensor map: cuTensorMapEncodeTiled entry point not found");
    return false;
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    static thread_local char why[160];
    snprintf(why, sizeof(why), "tensor map: CUresult %d for base %p rows %lld width %lld row stride %lld", (int)r, base, rows,
             width, row_stride);
    set_error_stage(why);
  } else {
    map_cache().put(k, *m);
  }
  return r == CUDA_SUCCESS;
}

// [rows, width] matrix of bytes (8-bit elements), box = 128 columns x `box_rows` rows, 128-byte swizzle, zero fill.
bool make_map_bytes(CUtensorMap* m, const void* base, long long rows, long long width, long long row_stride, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error_stage("tensor map: cuTensorMapEncodeTiled entry point not found");
    return false;
  }
  const MapKey k{base, rows, width, row_stride, box_rows, 2};
  if (map_cache().find(k, m)) return true;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride)};
  cuuint32_t box[2] = {128, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) set_error_stage("tensor map: encoding a byte matrix failed");
  else map_cache().put(k, *m);
  return r == CUDA_SUCCESS;
}

// Grid of the persistent kernels: one CTA per SM, fewer if there cannot be that many items.
int main_grid(const WorkspaceLayout& w) {
  long long grid = w.max_items < sm_count() ? w.max_items : sm_count();
  return grid < 1 ? 1 : static_cast<int>(grid);
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

// Sequences per locality chunk of the work list: the K/V (or Q/dO) rows of one chunk should stay in
// L2 while its items run, about 16 k tokens of 4 heads x 128 columns; chunks start with the longest
// sequences, so the caller's length bound sizes them.  Measured: 4 is best for sequences up to 4224
// tokens (1 % over 8), 6-12 are level for 2112-token sequences, 4 and 8 are level for 8 heads x 8 k.
static int chunk_seqs_for(const KernelArgs& a) {
  const long long budget = 16384LL * 4 / (a.H > 0 ? a.H : 1);
  const long long n = a.max_seq_len > 0 ? a.max_seq_len : 1;
  const long long c = (budget + n / 2) / n;
  int chunk = static_cast<int>(c < 4 ? 4 : (c > 16 ? 16 : c));
#ifdef B200_HSTU_PROFILING
  if (const char* e = getenv("B200_HSTU_CHUNK")) chunk = atoi(e) > 0 ? atoi(e) : chunk;
#endif
  return chunk;
}

// Ints of dynamic shared memory of the table step and of the entry step of the work-list construction; the
// tables live in shared memory when they fit under the default 48 KB (next to 4 KB of static shared memory).
constexpr long long WORK_LIST_SMEM_INTS = 10240;
static long long index_table_ints(const WorkspaceLayout& w) { return 3 * w.nbins; }
static long long item_table_ints(const KernelArgs& a, const WorkspaceLayout& w) {
  return w.nbins + (a.B + w.chunk_seqs - 1) / w.chunk_seqs + 1;
}

template <typename T>
static cudaError_t launch_prep_t(const KernelArgs& a, int* ws, const WorkspaceLayout& w_in, bool backward, cudaStream_t st) {
  WorkspaceLayout w = w_in;
  w.chunk_seqs = chunk_seqs_for(a);
  const long long index_ints = index_table_ints(w);
  const int index_smem = index_ints <= WORK_LIST_SMEM_INTS ? 1 : 0;
  const int stride = main_grid(w);
  const long long item_ints = item_table_ints(a, w);
  const int item_smem = item_ints <= WORK_LIST_SMEM_INTS ? 1 : 0;
  const size_t item_bytes = item_smem ? item_ints * sizeof(int) : 0;
  T *z0 = reinterpret_cast<T*>(a.o), *z1 = nullptr, *z2 = nullptr;
  long long rs0 = a.o_rs, rs1 = 0, rs2 = 0;
  int w0 = a.H * a.Dv, w1 = 0, w2 = 0;
  if (backward) {
    z0 = reinterpret_cast<T*>(a.dq); rs0 = a.dq_rs; w0 = a.H * a.Dqk;
    z1 = reinterpret_cast<T*>(a.dk); rs1 = a.dk_rs; w1 = a.H * a.Dqk;
    z2 = reinterpret_cast<T*>(a.dv); rs2 = a.dv_rs; w2 = a.H * a.Dv;
  }
  if (index_smem && item_smem) {
    // one launch: a cluster whose first CTA builds the tables and whose CTAs all decode the entries
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(WORK_LIST_CLUSTER);
    cfg.blockDim = dim3(1024);
    cfg.dynamicSmemBytes = static_cast<size_t>(index_ints > item_ints ? index_ints : item_ints) * sizeof(int);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = WORK_LIST_CLUSTER;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, build_work_list<T>, a, ws, w, stride, z0, rs0, w0, z1, rs1, w1, z2, rs2, w2) ==
        cudaSuccess)
      return cudaSuccess;
    (void)cudaGetLastError();  // a device that cannot place the cluster: the two kernels below do the same work
  }
  build_block_index<<<1, 1024, index_smem ? index_ints * sizeof(int) : 0, st>>>(a, ws, w, index_smem);
  const int blocks = sm_count() * 2;
  return launch_dependent(build_work_items<T>, blocks, 256, item_bytes, st, true, a, ws, w, stride, item_smem, z0, rs0,
                          w0, z1, rs1, w1, z2, rs2, w2);
}

// Workspace of a backward call: the work list, and (unless the caller asked for the recomputing dQ pass, or
// one of the two passes is left out, or the region would exceed B200_HSTU_DS_WORKSPACE_LIMIT) the dS tiles.
WorkspaceLayout backward_layout(const KernelArgs& a) {
  WorkspaceLayout w = workspace_layout(a.T, a.B, a.H);
  if (!a.recompute_dq) add_ds_region(w, a.T, a.B, a.H, a.max_seq_len, a.mask.ctx ? 1 : 0, B200_HSTU_DS_WORKSPACE_LIMIT);
  return w;
}

cudaError_t launch_prep(const KernelArgs& a, bool bf16, int* ws, const WorkspaceLayout& w, bool backward,
                        cudaStream_t st) {
  return bf16 ? launch_prep_t<__nv_bfloat16>(a, ws, w, backward, st) : launch_prep_t<__half>(a, ws, w, backward, st);
}

// Exercises the bounded wait that every pipeline wait of the tensor-core kernels goes through: one warp
// waits on a barrier that nothing will ever complete, with a limit of `limit_ns`; the wait must give up,
// record `code` in status[1] and let the kernel finish normally.
__global__ void bounded_wait_probe(int* status, int code, unsigned long long limit_ns) {
  __shared__ unsigned long long bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    sm100::mbar_init(sm100::smem_u32(&bar), 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  const bool ok = sm100::mbar_wait(sm100::smem_u32(&bar), 0u, &abort_flag, status, code, limit_ns);
  if (!ok && threadIdx.x == 0) atomicAdd(status + 2, 1);  // how many probes saw the wait give up
}

cudaError_t launch_bounded_wait_probe(int* status, int code, unsigned long long limit_ns, cudaStream_t st) {
  bounded_wait_probe<<<1, 32, 0, st>>>(status, code, limit_ns);
  return cudaGetLastError();
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
  const tc::WorkspaceLayout w = pass == 1 ? tc::backward_layout(a) : tc::workspace_layout(a.T, a.B, a.H);
  return static_cast<size_t>(w.total_bytes);
}

int tc_launch_count(const KernelArgs& a, int pass) {
  // the work list (one launch when its tables fit shared memory, else two), then the main kernel(s)
  tc::WorkspaceLayout w = tc::workspace_layout(a.T, a.B, a.H);
  w.chunk_seqs = tc::chunk_seqs_for(a);
  const bool one = tc::index_table_ints(w) <= tc::WORK_LIST_SMEM_INTS && tc::item_table_ints(a, w) <= tc::WORK_LIST_SMEM_INTS;
  return (one ? 1 : 2) + (pass == 0 ? 1 : 2);
}

cudaError_t tc_forward(const KernelArgs& a, int dtype, void* workspace, cudaStream_t st) {
  using namespace tc;
  const bool bf16 = dtype == B200_HSTU_BF16;
  const WorkspaceLayout w = workspace_layout(a.T, a.B, a.H);
  int* ws = reinterpret_cast<int*>(workspace);
  TensorMaps maps;
  const long long width = (long long)a.H * HEAD_DIM;
  set_error_stage("forward: tensor maps");
  if (!ensure_current_context(a.q)) return cudaErrorInvalidValue;
  if (!make_map(&maps.q, a.q, a.T, width, a.q_rs, bf16) || !make_map(&maps.k, a.k, a.T, width, a.k_rs, bf16) ||
      !make_map(&maps.v, a.v, a.T, width, a.v_rs, bf16) || !make_map(&maps.o, a.o, a.T, width, a.o_rs, bf16))
    return cudaErrorInvalidValue;
  set_error_stage("forward: work-list kernels");
  cudaError_t e = launch_prep(a, bf16, ws, w, false, st);
  if (e != cudaSuccess) return e;
  set_error_stage("forward: main kernel");
  const size_t smem = sizeof(FwdShared) + 1024;
  // The kernels carry optional cycle accounting and event traces (template parameter PROF).  Those
  // variants are only instantiated in a build with -DB200_HSTU_PROFILING, which also honours the
  // tuning environment variables; the shipped library has one instantiation per kernel and dtype.
#ifdef B200_HSTU_PROFILING
  static const bool profile = getenv("B200_HSTU_PROFILE") != nullptr;  // cycle accounting into workspace ints 2..15
  auto kern = profile ? (bf16 ? hstu_fwd_tc<true, true> : hstu_fwd_tc<false, true>)
                      : (bf16 ? hstu_fwd_tc<true, false> : hstu_fwd_tc<false, false>);
#else
  auto kern = bf16 ? hstu_fwd_tc<true, false> : hstu_fwd_tc<false, false>;
#endif
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  e = launch_dependent(kern, static_cast<unsigned>(main_grid(w)), FWD_THREADS, smem, st, true, maps, a, ws, w.off_items);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}


}  // namespace hstu
