// Shared pieces of the tensor-core kernels: the work list built on the device, tile
// classification against the keep mask, and tensor-map helpers.
#pragma once
#include <cuda.h>

#include "hstu_common.cuh"
#include "sm100_ptx.cuh"

namespace hstu {
namespace tc {

constexpr int BLK = 128;  // rows per query block and per key block
constexpr int HEAD_DIM = 128;

// ---- workspace layout (ints) ------------------------------------------------
// [0]            number of work items
// [1]            number of non-empty sequences
// [2 .. 15]      reserved
// [16 .. )       sorted[B]   : sequence ids, longest first
//                hist[nbins] : sequences per block count, then reused as fill counters
//                cnt[nbins]  : cnt[j] = sequences with more than j blocks
//                start[nbins]: first work item of block index j
//                items[2 * max_items] : (seq | head << 16, block index) per work item
struct WorkspaceLayout {
  long long nbins, max_items;
  long long off_sorted, off_hist, off_cnt, off_start, off_chunk, off_items, total_ints;
  int chunk_seqs;  // sequences per locality chunk of the work list
  // backward with stored dS tiles (ds_tile_cap == 0: not used), behind the ints above:
  long long off_tile_base;   // byte offset of the per-sequence first-tile indices ([B] long long)
  long long off_ds_tiles;    // byte offset of the tile region (1024-byte aligned)
  long long ds_tile_cap;     // tiles it holds
  long long total_bytes;     // whole workspace
  int ds_square;             // tiles of a sequence indexed as a square (contextual prefix) or a triangle
};

HSTU_HD WorkspaceLayout workspace_layout(long long T, int B, int H) {
  WorkspaceLayout w;
  w.nbins = (T + BLK - 1) / BLK + 2;
  w.max_items = (long long)H * (T / BLK + B);
  w.off_sorted = 32;  // ints 0..31: totals, profiling counters, work-list cursors (WS_CURSOR0/1)
  w.off_hist = w.off_sorted + B;
  w.off_cnt = w.off_hist + w.nbins;
  w.off_start = w.off_cnt + w.nbins;
  w.off_chunk = w.off_start + w.nbins;
  w.off_items = (w.off_chunk + B + 2 + 1) & ~1LL;  // int2 alignment
  w.chunk_seqs = 8;
  w.total_ints = w.off_items + 2 * w.max_items;
  w.off_tile_base = w.off_ds_tiles = w.ds_tile_cap = 0;
  w.ds_square = 0;
  w.total_bytes = (w.total_ints * 4 + 255) & ~255LL;
  return w;
}

constexpr int DS_TILE_BYTES = BLK * BLK * 2;  // one 128 x 128 16-bit dS^T tile

// Tiles of one (sequence, head) with nb 128-row blocks, and the index of tile (query block i, key block j)
// among them.  Causal masks keep j <= i (a triangle); with a contextual prefix a sequence whose tokens are all
// targets keeps the whole square.
HSTU_HD long long ds_tiles_of(long long nb, int square) { return square ? nb * nb : nb * (nb + 1) / 2; }
HSTU_HD long long ds_tile_index(int i, int j, long long nb, int square) {
  return square ? i * nb + j : static_cast<long long>(i) * (i + 1) / 2 + j;
}

// Adds the stored-dS region to a backward workspace: room for every tile any batch of T tokens in B
// sequences of at most max_seq_len tokens can have.  limit_bytes: leave the region out above this size.
HSTU_HD void add_ds_region(WorkspaceLayout& w, long long T, int B, int H, long long max_seq_len, int square,
                           unsigned long long limit_bytes) {
  if (max_seq_len <= 0) return;
  const long long nbmax = (max_seq_len + BLK - 1) / BLK, blocks = T / BLK + B;
  // sum over sequences of tiles(nb_b) <= (sum of nb_b) * max over nb <= nbmax of tiles(nb) / nb
  const long long per_block_2 = square ? 2 * nbmax : nbmax + 1;  // twice the bound per block
  const long long cap = (blocks * per_block_2 + 1) / 2 * H;
  if (cap <= 0 || static_cast<unsigned long long>(cap) > limit_bytes / DS_TILE_BYTES) return;
  w.off_tile_base = (w.total_ints * 4 + 255) & ~255LL;
  w.off_ds_tiles = (w.off_tile_base + 8LL * (B + 1) + 1023) & ~1023LL;
  w.ds_tile_cap = cap;
  w.ds_square = square;
  w.total_bytes = w.off_ds_tiles + cap * DS_TILE_BYTES;
}

// Workspace header slots: next unclaimed work-list entry, one cursor per main kernel of a call.
constexpr int WS_CURSOR0 = 16, WS_CURSOR1 = 17;

enum TileClass { TILE_SKIP = 0, TILE_PARTIAL = 1, TILE_FULL = 2 };

// Classifies the 128x128 tile with query rows [m0, m0+128) and key rows [n0, n0+128) of one
// sequence under a causal ("lower_triangular") mask:
//   SKIP    no pair of the tile is kept (safe to never compute),
//   FULL    every pair is kept and every row/column lies inside the sequence,
//   PARTIAL anything else (the exact predicate is evaluated per element).
//
// rows_dont_care: the caller never uses query rows at or past the sequence end (query-major
// passes: such rows are not stored and cannot influence other rows), so a tile may be FULL
// even if it hangs over the end of the sequence in the row direction.
HSTU_HD int classify_tile(int m0, int n0, const SeqInfo& s, const MaskOpts& o, bool rows_dont_care = false) {
  const int L = s.len;
  if (m0 >= L || n0 >= L) return TILE_SKIP;
  const int m1 = m0 + BLK - 1, n1 = n0 + BLK - 1;
  const int m1e = m1 < L ? m1 : L - 1, n1e = n1 < L ? n1 : L - 1;
  if (o.ctx && s.has_targets && s.hist == 0) return TILE_PARTIAL;  // whole square kept
  if (n0 > m1e) return TILE_SKIP;                                  // strictly above the diagonal
  const int hist = s.has_targets ? s.hist : L;
  const bool diag = (n0 <= m1e) && (m0 <= n1e);
  if (hist < 0) return diag ? TILE_PARTIAL : TILE_SKIP;  // every id equal: diagonal only
  const int idm0 = m0 < hist ? m0 : hist, idm1 = m1e < hist ? m1e : hist;
  const int idn0 = n0 < hist ? n0 : hist, idn1 = n1e < hist ? n1e : hist;
  const int maxd = idm1 - idn0, mind = idm0 - idn1;
  bool any = diag;
  any = any || (maxd > 0 && (o.window <= 0 || mind <= o.window));
  any = any || (o.ctx && n0 == 0);
  if (o.window > 0 && o.full > 0) {
    const int gm = idm1 < s.boundary ? 0 : idm1;
    const int gn = idn0 < s.boundary ? 0 : idn0;
    any = any || (gm - gn > 0);
  }
  if (!any) return TILE_SKIP;
  if ((m1 >= L && !rows_dont_care) || n1 >= L) return TILE_PARTIAL;
  if (mind > 0 && (o.window <= 0 || maxd <= o.window)) return TILE_FULL;
  return TILE_PARTIAL;
}

// Key blocks a query block [m0, m0+128) can touch: optionally block 0, then lo..hi.
struct BlockRange {
  int lo, hi, extra0;
  HSTU_HD int count() const { return hi - lo + 1 + extra0; }
  HSTU_HD int at(int idx) const { return extra0 ? (idx == 0 ? 0 : lo + idx - 1) : lo + idx; }
};

HSTU_HD BlockRange key_blocks_for_query_block(int m0, const SeqInfo& s, const MaskOpts& o) {
  BlockRange r;
  const int L = s.len;
  const bool whole = o.ctx && s.has_targets && s.hist == 0;
  const int m1e = (m0 + BLK - 1 < L ? m0 + BLK - 1 : L - 1);
  r.hi = (whole ? L - 1 : m1e) / BLK;
  r.lo = 0;
  r.extra0 = 0;
  if (o.window > 0 && o.full <= 0 && !whole) {
    const int hist = s.has_targets ? s.hist : L;
    if (hist >= 0) {
      const int idm0 = m0 < hist ? m0 : hist;
      int nlo = idm0 - o.window;
      if (nlo < 0) nlo = 0;
      r.lo = nlo / BLK;
      if (r.lo > r.hi) r.lo = r.hi;
      r.extra0 = (o.ctx && r.lo > 0) ? 1 : 0;
    }
  }
  return r;
}

// Query blocks a key block [n0, n0+128) can be touched by: lo..hi (hi = last block).
// With a sliding window the far rows are dropped unless a full-attention tail, the
// contextual column or the target rows need them; classification skips the rest.
HSTU_HD BlockRange query_blocks_for_key_block(int n0, const SeqInfo& s, const MaskOpts& o) {
  BlockRange r;
  const int L = s.len;
  const bool whole = o.ctx && s.has_targets && s.hist == 0;
  r.lo = whole ? 0 : n0 / BLK;
  r.hi = (L - 1) / BLK;
  r.extra0 = 0;
  return r;
}

// Exact per-row form of the causal keep rule: for a fixed query m,
//   keep(m, n)  <=>  lo <= n < hi  ||  n == diag  ||  n == extra      (diag / extra = -1: unused)
// Rows at or past the sequence end keep nothing.
struct RowMask {
  int lo, hi, diag, extra;
};

HSTU_HD RowMask row_mask(int m, const SeqInfo& s, const MaskOpts& o) {
  RowMask r;
  r.lo = 0; r.hi = 0; r.diag = -1; r.extra = -1;
  const int L = s.len;
  if (m >= L || m < 0) return r;
  r.diag = m;
  if (o.ctx && s.has_targets && s.hist == 0) { r.hi = L; return r; }  // every id is 0: whole square
  const int hist = s.has_targets ? s.hist : L;
  if (hist <= 0) return r;  // all ids equal: diagonal only
  const int idm = m < hist ? m : hist;
  r.hi = idm;  // keys n < min(m, hist) have a smaller id
  if (o.window > 0) {
    r.lo = idm - o.window > 0 ? idm - o.window : 0;
    if (o.full > 0 && idm >= s.boundary && idm > 0) r.lo = 0;  // full-attention tail row
  }
  if (o.ctx) r.extra = 0;  // key 0 carries id 0 (hist > 0 here)
  return r;
}

// Exact per-column form: for a fixed key n,
//   keep(m, n)  <=>  m == diag  ||  a_lo <= m < a_hi  ||  b_lo <= m < len
struct ColMask {
  int a_lo, a_hi, b_lo, diag;
};

HSTU_HD ColMask col_mask(int n, const SeqInfo& s, const MaskOpts& o) {
  ColMask c;
  const int L = s.len;
  c.a_lo = 0; c.a_hi = 0; c.b_lo = L; c.diag = -1;
  if (n >= L || n < 0) return c;
  c.diag = n;
  if (o.ctx && s.has_targets && s.hist == 0) { c.a_hi = L; return c; }
  const int hist = s.has_targets ? s.hist : L;
  if (hist <= 0 || n >= hist) return c;  // target column (or all ids equal): diagonal only
  if (o.ctx && n == 0) { c.a_hi = L; return c; }  // id 0: visible to every query
  c.a_lo = n + 1;
  if (o.window <= 0) { c.a_hi = L; return c; }
  c.a_hi = n + o.window + 1 < hist ? n + o.window + 1 : hist;  // history rows inside the window
  if (hist - n <= o.window) c.a_hi = L;                        // target rows carry id hist
  if (o.full > 0) {
    int bl = s.boundary > n + 1 ? s.boundary : n + 1;
    if (bl < 1) bl = 1;
    c.b_lo = bl < L ? bl : L;
  }
  return c;
}

constexpr int TILE_BYTES = BLK * HEAD_DIM * 2;  // 32 KB: one 128x128 16-bit tile (two 64-column boxes)
constexpr int HALF_TILE_BYTES = TILE_BYTES / 2;
constexpr int SUBTILE_BYTES = 64 * 128;  // 64 rows of one box: rows [64, 128) of a tile start here

// codes written to status[1] by a wait that gave up
enum { WAIT_PRODUCER = 101, WAIT_MMA = 102, WAIT_EPILOGUE = 103 };

#if defined(__CUDACC__)
template <bool IS_BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return IS_BF16 ? sm100::pack_bf16x2(lo, hi) : sm100::pack_f16x2(lo, hi);
}

// Bitmap of the kept columns among the 64 columns [cbase, cbase + 64) for a row mask.
__device__ __forceinline__ unsigned long long row_mask_bits64(const RowMask& rm, int cbase) {
  int lo = rm.lo - cbase, hi = rm.hi - cbase;
  lo = lo < 0 ? 0 : (lo > 64 ? 64 : lo);
  hi = hi < 0 ? 0 : (hi > 64 ? 64 : hi);
  const unsigned long long below_hi = hi >= 64 ? ~0ull : ((1ull << hi) - 1ull);
  const unsigned long long below_lo = lo >= 64 ? ~0ull : ((1ull << lo) - 1ull);
  unsigned long long bits = hi > lo ? (below_hi & ~below_lo) : 0ull;
  const int d = rm.diag - cbase, e = rm.extra - cbase;
  if (rm.diag >= 0 && d >= 0 && d < 64) bits |= 1ull << d;
  if (rm.extra >= 0 && e >= 0 && e < 64) bits |= 1ull << e;
  return bits;
}

// x sigma(x) for two scores with packed 16-bit math: u = (alpha/2) s in fp32, then
// t = tanh(u) (one MUFU operation for the pair) and p = u t + u in 16-bit FMA.
template <bool IS_BF16>
__device__ __forceinline__ uint32_t silu_pair(uint32_t s0, uint32_t s1, uint64_t c1x2) {
  float u0, u1;
  sm100::mul_f32x2(s0, s1, c1x2, u0, u1);
  const uint32_t u2 = pack2<IS_BF16>(u0, u1);
  return sm100::fma2<IS_BF16>(u2, sm100::tanh2<IS_BF16>(u2), u2);
}

// Clears rows [row_lo, row_hi) of one 64-column box of a tile (128 bytes per box row, rows
// contiguous in shared memory) and makes the write visible to the async proxy (TMA / MMA).
// `nthreads` threads with ids `tid` write consecutive 16-byte chunks, so a warp store covers 512
// contiguous bytes (no bank conflicts; a thread-per-row version was 32-way conflicted and cost
// thousands of cycles per ragged tile).  The 128-byte swizzle only permutes chunks inside a row,
// so whole rows can be cleared without knowing it.
__device__ __forceinline__ void zero_box_rows(unsigned char* box, int row_lo, int row_hi, int tid, int nthreads) {
  if (row_lo < 0) row_lo = 0;
  if (row_lo >= row_hi) return;
  uint4* p = reinterpret_cast<uint4*>(box);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int c = row_lo * 8 + tid; c < row_hi * 8; c += nthreads) p[c] = z;
  sm100::fence_proxy_async();
}

// ------------------------------------------------------------------ work-item ring
// Work items are handed out dynamically: one otherwise idle warp of every CTA (the scheduler)
// claims the next entry of the work list with an atomic add on a cursor in the workspace,
// reads the entry and the sequence it belongs to, and publishes both through a two-slot ring in
// shared memory.  The producer warp, the MMA warp and the eight epilogue warps each take every
// item from the ring (copying the slot into registers and releasing it at once), so none of
// them touches global memory to find out what to do next, and a CTA that finishes early simply
// claims more.  The first item of a CTA is entry blockIdx.x; the cursor starts at gridDim.x.
struct ItemSlot {
  int2 w;     // (sequence | head << 16, block index); w.x < 0: the list is exhausted
  SeqInfo s;
  uint32_t todo, full;  // classes of the item's first 32 candidate tiles: bit i = not skipped / fully kept
};
constexpr int ITEM_RING = 2;
constexpr int ITEM_CONSUMERS = 10;  // producer warp, MMA warp, eight epilogue warps
enum { WAIT_SCHEDULER = 104 };
struct ItemRing {
  ItemSlot slot[ITEM_RING];
  unsigned long long full[ITEM_RING], empty[ITEM_RING];
};

__device__ __forceinline__ void item_ring_init(ItemRing& r) {
  for (int i = 0; i < ITEM_RING; ++i) {
    sm100::mbar_init(sm100::smem_u32(&r.full[i]), 1);
    sm100::mbar_init(sm100::smem_u32(&r.empty[i]), ITEM_CONSUMERS);
  }
}

// Class of candidate tile i of an item.  KEY_MAJOR = false: the item is a query block and the
// candidates are its key blocks (forward, dQ pass; query rows past the sequence end do not
// matter); true: the item is a key block and the candidates are its query blocks (dK/dV pass).
template <bool KEY_MAJOR>
__device__ __forceinline__ int item_tile_class(const int2& w, const SeqInfo& s, const MaskOpts& o, int i, int* count) {
  if (!KEY_MAJOR) {
    const int m0 = w.y * BLK;
    const BlockRange kr = key_blocks_for_query_block(m0, s, o);
    *count = kr.count();
    return i < kr.count() ? classify_tile(m0, kr.at(i) * BLK, s, o, true) : TILE_SKIP;
  }
  const int n0 = ((s.len + BLK - 1) / BLK - 1 - w.y) * BLK;
  const BlockRange qr = query_blocks_for_key_block(n0, s, o);
  *count = qr.count();
  return i < qr.count() ? classify_tile(qr.at(i) * BLK, n0, s, o) : TILE_SKIP;
}

// Body of the scheduler warp (all 32 lanes call it): lane 0 claims and reads the item, every
// lane classifies one of its first 32 candidate tiles, so that the other warps do not repeat it.
template <bool KEY_MAJOR>
__device__ __forceinline__ void run_item_scheduler(ItemRing& r, const KernelArgs& a, const int2* items, int total,
                                                   int* cursor, volatile int* abort_flag) {
  const int lane = threadIdx.x & 31;
  int idx = blockIdx.x;
  for (uint32_t n = 0;; ++n) {
    const uint32_t sl = n % ITEM_RING, par = ((n / ITEM_RING) & 1) ^ 1;
    if (!__all_sync(0xffffffffu, sm100::mbar_wait(sm100::smem_u32(&r.empty[sl]), par, abort_flag, a.status, WAIT_SCHEDULER)))
      return;
    const bool have = idx < total;
    ItemSlot it;
    it.w = make_int2(-1, 0);
    it.s.start = 0; it.s.len = 0; it.s.hist = 0; it.s.has_targets = 0; it.s.boundary = 0; it.s.tile_base = 0;
    it.todo = 0u; it.full = 0u;
    if (have) {
      if (lane == 0) {
        it.w = items[idx];
        it.s = load_seq(a, it.w.x & 0xffff);
        if (a.ds_tile_base != nullptr) it.s.tile_base = a.ds_tile_base[it.w.x & 0xffff];
      }
      it.w.x = __shfl_sync(0xffffffffu, it.w.x, 0);
      it.w.y = __shfl_sync(0xffffffffu, it.w.y, 0);
      it.s.start = __shfl_sync(0xffffffffu, it.s.start, 0);
      it.s.len = __shfl_sync(0xffffffffu, it.s.len, 0);
      it.s.hist = __shfl_sync(0xffffffffu, it.s.hist, 0);
      it.s.has_targets = __shfl_sync(0xffffffffu, it.s.has_targets, 0);
      it.s.boundary = __shfl_sync(0xffffffffu, it.s.boundary, 0);
      it.s.tile_base = __shfl_sync(0xffffffffu, it.s.tile_base, 0);
      int count = 0;
      const int cls = item_tile_class<KEY_MAJOR>(it.w, it.s, a.mask, lane, &count);
      it.todo = __ballot_sync(0xffffffffu, cls != TILE_SKIP);
      it.full = __ballot_sync(0xffffffffu, cls == TILE_FULL);
    }
    if (lane == 0) {
      r.slot[sl] = it;
      sm100::mbar_arrive(sm100::smem_u32(&r.full[sl]));  // release: the slot is written before the arrival
    }
    __syncwarp();
    if (!have) return;
    if (lane == 0) idx = atomicAdd(cursor, 1);
    idx = __shfl_sync(0xffffffffu, idx, 0);
  }
}

// Takes item n from the ring (whole warp).  Returns false when the list is exhausted or a wait
// gave up (then `ok` is cleared as well).
__device__ __forceinline__ bool next_item(ItemRing& r, uint32_t n, int2& w, SeqInfo& s, uint32_t& todo0,
                                          uint32_t& full0, bool& ok, volatile int* abort_flag, int* status, int code) {
  const uint32_t sl = n % ITEM_RING, par = (n / ITEM_RING) & 1;
  if (!__all_sync(0xffffffffu, sm100::mbar_wait(sm100::smem_u32(&r.full[sl]), par, abort_flag, status, code))) {
    ok = false;
    return false;
  }
  w = r.slot[sl].w;
  s = r.slot[sl].s;
  todo0 = r.slot[sl].todo;
  full0 = r.slot[sl].full;
  __syncwarp();
  if ((threadIdx.x & 31) == 0) sm100::mbar_arrive(sm100::smem_u32(&r.empty[sl]));
  return w.x >= 0;
}
#endif

}  // namespace tc
}  // namespace hstu
