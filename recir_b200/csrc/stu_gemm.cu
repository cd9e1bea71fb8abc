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
// 128-column fp32 accumulators.  The rows of the NEXT block are parked in shared memory while the current
// one computes (128 x K, 128-byte-swizzled boxes of 64 columns): landed there by TMA, and with the
// layer-norm prologue normalised there in place by two dedicated warps; when the last accumulator of the
// current block is complete they are copied row-per-thread into TMEM (tcgen05.st, by the warps whose TMEM
// lane quadrant holds those rows) BEFORE that accumulator is drained, so the MMAs of the next block start
// under the drain.  W streams through a ring of [64 k-rows x 128 n-columns] tiles (TMA, N-major B operand)
// in whatever shared memory is left (64 KB at K = 512); four tcgen05.mma K16 (A from TMEM) per stage.  The
// epilogue of an output tile (bias, rounding, staged bulk tensor stores) overlaps the MMAs of the next one.
//
// CTA pairs.  Outside the jagged mode two CTAs (a cluster on the two SMs of a TPC) work on 256 consecutive
// rows with ONE tcgen05.mma.cta_group::2 M256 N128 K16 per k-step, issued by the CTA of rank 0; each CTA
// then loads only its half of every W tile (64 of the 128 columns).  W is L2-resident (K x N x 2 bytes, a
// few MB at most) but every 128-row block reads all of it, and that L2 -> SM stream is what bounds a
// single-CTA kernel of this shape; the pair halves it.  Nothing is broadcast: each CTA's TMA loads land in
// its own shared memory and only mbarrier arrivals / byte counts cross to the peer.
//
// Warp roles (384 threads): warp 0 = TMA producer, warp 1 = MMA issuer (one elected lane; in a pair only
// rank 0 issues), warps 2-9 = A-operand install and epilogue (TMEM lane quadrant warp % 4, column half
// (warp - 2) / 4), warps 10-11 = layer norm (idle without it).  Every wait is bounded (see sm100_ptx.cuh);
// the waits off the critical path sleep between polls.
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
#include "sm100_pair.cuh"
#include "sm100_ptx.cuh"
#include "stu_vec.cuh"

namespace hstu {
namespace gemm {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 128, BK = 64;  // BK: k-rows of W per pipeline stage (four k-steps of 16)
constexpr int MAX_K = 512;
constexpr int MAX_W_STAGES = 16;
constexpr int W_BOX_BYTES = BK * 128;        // 64 k-rows x 64 n-columns of 16-bit elements
constexpr int PARK_BOX_BYTES = BM * 128;     // 128 rows x 64 k-columns
constexpr int OUT_BOX_BYTES = BM * 128;      // 128 rows x 64 output columns, one box per epilogue group
constexpr int CONTROL_BYTES = 1024;
constexpr int DATA_BYTES = 224 * 1024;       // output staging + parked A operand + weight ring
constexpr int THREADS = 384;                 // 12 warps, 168 registers each
constexpr int TMEM_COLS = 512;
constexpr int TMEM_A = 0, TMEM_ACC0 = 256;   // A operand: K / 2 columns (two 16-bit values each); 2 x 128 accumulator columns
constexpr int LN_WARPS = 2;                  // warps 10 and 11 normalise the next block's rows (layer-norm prologue)
constexpr int LN_BATCH = 2;                  // rows a layer-norm warp takes through every stage together
enum { WAIT_GEMM_PRODUCER = 111, WAIT_GEMM_MMA = 112, WAIT_GEMM_EPILOGUE = 113, WAIT_GEMM_LAYOUT = 114 };

// Barriers and the like, in the first KB of the (1024-byte aligned) shared memory; behind it the data:
// output staging (2 x 16 KB), the parked A operand of the next block (K / 64 boxes of 16 KB), and the weight
// ring in whatever is left of 224 KB.
struct Control {
  unsigned long long x_full, x_free;  // a block's rows are in the park (landed by TMA, or normalised) / they were copied to TMEM
  unsigned long long x_raw;           // layer-norm prologue: TMA landed the raw rows in the park (x_full: they are normalised)
  unsigned long long a_ready;         // the block's A operand is in TMEM (in a pair: of both CTAs)
  unsigned long long w_full[MAX_W_STAGES], w_empty[MAX_W_STAGES];
  unsigned long long acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Control) <= CONTROL_BYTES, "control block");

struct Maps {
  CUtensorMap x;  // [M, K], box 64 columns x 128 rows
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
  const float* a_scale;  // fp8: [M] scale of every row of A
  const float* b_scale;  // fp8: [N] scale of every row of W, i.e. of every output column
  int dbg;  // instrumented builds only (B200_GEMM_DBG): 1 no W loads / waits, 2 no output staging, 4 no MMAs
};

using vec::warp_sum;
// Instrumented builds: cycles spent per phase by one lane of each role, printed by CTAs 0 and 1
// (B200_GEMM_DBG bit 32).
#ifdef B200_HSTU_PROFILING
#define GEMM_T0() const long long t0_ = clock64()
#define GEMM_T1(acc) (acc) += clock64() - t0_
#define GEMM_MARK(acc) do { const long long now_ = clock64(); (acc) += now_ - mark_; mark_ = now_; } while (0)
#define GEMM_REPORT(role) \
  do { if ((a.dbg & 32) && blockIdx.x < 2 && lane == 0) \
    printf("cta %d warp %d %s: %lld %lld %lld %lld %lld %lld [%lld %lld] | total %lld\n", blockIdx.x, warp, role, tw[0], tw[1], tw[2], tw[3], \
           tw[4], tw[5], tw[6], tw[7], clock64() - t_start_); } while (0)
#else
#define GEMM_T0() do {} while (0)
#define GEMM_T1(acc) do {} while (0)
#define GEMM_MARK(acc) do {} while (0)
#define GEMM_REPORT(role) do {} while (0)
#endif
// Bounded wait for the roles that are not on the critical path (everything but the MMA issuer): between
// polls the warp sleeps, so that a dozen polling warps do not draw power, and issue slots, that the part
// would rather give to the tensor pipe (the kernel runs at the power limit).
__device__ __forceinline__ bool mbar_wait_idle(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = 0;
  for (uint32_t i = 1;; ++i) {
    __nanosleep(96);
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (*abort_flag) return false;
      const unsigned long long now = globaltimer_ns();
      if (t0 == 0) t0 = now;
      if (now - t0 > 2000000000ull) {
        *abort_flag = 1;
        if (status) atomicCAS(status + 1, 0, code);
        return false;
      }
    }
  }
}
template <bool BF16> __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

// PAIR: two CTAs (a cluster on the two SMs of a TPC) work on 256 consecutive rows, 128 each, with ONE
// tcgen05.mma.cta_group::2 M256 N128 K16 per k-step issued by the CTA of rank 0.  Each CTA then holds only
// its half of the B operand (64 of the tile's 128 columns), so each SM pulls half as much of W out of L2 -
// and L2 bandwidth for W is what bounds the single-CTA form.  The jagged mode (a weight matrix per
// sequence, so two neighbouring row blocks may need different B operands) runs unpaired.
// ET: 0 float16, 1 bfloat16, 2 float8 e4m3 operands with bfloat16 bias and output (row-wise scaled product:
// A is [M, K] with a scale per row, W is given K-major as [N, K] with a scale per row, i.e. per output column;
// pairs only, no layer norm).  In bytes everything is the same: 128-byte box rows, 32 bytes of K per MMA.
template <int ET, bool PAIR, bool FUSE>
__global__ void __launch_bounds__(THREADS, 1) stu_addmm_tc(const __grid_constant__ Maps maps, Args a) {
  constexpr bool FP8 = ET == 2, BF16 = ET != 0;
  static_assert(!FP8 || (PAIR && !FUSE), "the fp8 form runs on pairs, without the layer-norm prologue");
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;  // element type of bias and out
  extern __shared__ __align__(1024) unsigned char smem[];  // the swizzled boxes need 1024-byte alignment (checked below)
  Control& c = *reinterpret_cast<Control*>(smem);
  if ((smem_u32(smem) & 1023u) != 0u) {  // (the same in every CTA: nobody is left waiting)
    if (threadIdx.x == 0 && a.status) atomicCAS(a.status + 1, 0, WAIT_GEMM_LAYOUT);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &c.abort_flag;
  const int kboxes = FP8 ? a.K / 128 : a.K / 64;  // 128-byte boxes of a row of the A operand = stages of W per tile
  unsigned char* const out_stage = smem + CONTROL_BYTES;
  unsigned char* const park = out_stage + 2 * OUT_BOX_BYTES;
  unsigned char* const wring = park + kboxes * PARK_BOX_BYTES;
  constexpr int STAGE_BYTES = PAIR ? W_BOX_BYTES : 2 * W_BOX_BYTES;  // this CTA's part of a [64 x 128] tile of W
  int w_stages = (DATA_BYTES - 2 * OUT_BOX_BYTES - kboxes * PARK_BOX_BYTES) / STAGE_BYTES;
  if (w_stages > MAX_W_STAGES) w_stages = MAX_W_STAGES;
  const int n_tiles = (a.N + BN - 1) / BN;
  const long long n_blocks = a.items ? static_cast<long long>(*a.n_items) : (a.M + BM - 1) / BM;
  // work units: a row block, or in a pair the two blocks 2 u and 2 u + 1 (the second may lie past the end)
  const uint32_t rank = PAIR ? cluster_cta_rank() : 0u;
  const long long n_units = PAIR ? (n_blocks + 1) / 2 : n_blocks;
  const long long u0 = PAIR ? (blockIdx.x >> 1) : blockIdx.x, ustride = PAIR ? (gridDim.x >> 1) : gridDim.x;
  // Every CTA walks the output tiles of its blocks in the same cyclic order but starts at a different
  // tile: CTAs that run in step would otherwise all ask L2 for the same few lines of W at the same time.
  const int tile_rot = static_cast<int>(u0 % n_tiles);
  auto tile_of = [&](int nt) -> int { const int t = nt + tile_rot; return t >= n_tiles ? t - n_tiles : t; };
  auto blk_of = [&](long long u) -> long long { return PAIR ? 2 * u + rank : u; };
  // block -> (sequence, first row, valid rows); plain mode: one "sequence" holding every row
  auto block_of = [&](long long blk) -> int4 {
    if (a.items) return a.items[blk];
    const long long row0 = blk * BM, left = a.M - row0;
    return make_int4(0, static_cast<int>(row0), static_cast<int>(left < 0 ? 0 : (left < BM ? left : BM)), 0);
  };
  // One arrival per warp on a barrier of the CTA that issues the MMAs, once every lane has got here.  What
  // the arrival hands over lives in TMEM and is complete by then (the tcgen05.wait before it is warp-wide),
  // so in a pair it is a RELAXED arrival: a release at cluster scope would first wait for every memory
  // operation the lane has in flight - the bias piece it has just requested from L2 among them.
  auto arrive_at_issuer = [&](unsigned long long* bar) {
    __syncwarp();
    if (lane == 0) {
      if constexpr (PAIR) mbar_arrive_cluster_relaxed(map_to_cta(smem_u32(bar), 0));
      else mbar_arrive(smem_u32(bar));
    }
  };

  if (threadIdx.x == 0) {
    c.abort_flag = 0;
    mbar_init(smem_u32(&c.x_full), FUSE ? LN_WARPS : 1);
    mbar_init(smem_u32(&c.x_raw), 1);
    mbar_init(smem_u32(&c.x_free), 256);
    mbar_init(smem_u32(&c.a_ready), PAIR ? 16 : 8);  // one arrival per epilogue warp
    for (int i = 0; i < MAX_W_STAGES; ++i) { mbar_init(smem_u32(&c.w_full[i]), 1); mbar_init(smem_u32(&c.w_empty[i]), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(smem_u32(&c.acc_full[i]), 1); mbar_init(smem_u32(&c.acc_empty[i]), PAIR ? 16 : 8); }
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0) {
    if constexpr (PAIR) { tmem_alloc_pair(smem_u32(&c.tmem_base), TMEM_COLS); tmem_relinquish_pair(); }
    else { tmem_alloc(smem_u32(&c.tmem_base), TMEM_COLS); tmem_relinquish(); }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // the peer's barriers exist before anything is sent to them
  tc_fence_after();
  const uint32_t tmem = c.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) { prefetch_tensormap(&maps.w); prefetch_tensormap(&maps.x); }
    uint32_t xr = 0, st = 0, ph = 0;
    bool ok = true;
    [[maybe_unused]] long long tw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    [[maybe_unused]] const long long t_start_ = clock64();
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait_idle(smem_u32(bar), parity, abort_flag, a.status, WAIT_GEMM_PRODUCER));
    };
    // the 128 rows of a block into the park; rows past the end arrive as zeros.  With the layer-norm prologue
    // they are raw rows, announced to the layer-norm warps; otherwise they are the A operand as it is.
    const uint32_t x_landed = smem_u32(FUSE ? &c.x_raw : &c.x_full);
    auto load_x = [&](long long blk) -> bool {
      { GEMM_T0(); const bool w = wait_all(&c.x_free, (xr & 1) ^ 1); GEMM_T1(tw[1]); if (!w) return false; }
      if (elect_one()) {
        const int4 bi = block_of(blk);
        mbar_arrive_expect_tx(x_landed, static_cast<uint32_t>(kboxes) * PARK_BOX_BYTES);
        for (int kb = 0; kb < kboxes; ++kb)
          tma_load_2d(smem_u32(park + kb * PARK_BOX_BYTES), &maps.x, x_landed, kb * (FP8 ? 128 : 64), bi.y);
      }
      __syncwarp();
      ++xr;
      return true;
    };
    const uint32_t w_full_issuer = PAIR ? map_to_cta(smem_u32(&c.w_full[0]), 0) : 0u;
    long long u = u0;
    if (u < n_units) ok = load_x(blk_of(u));
    for (; u < n_units && ok; u += ustride) {
      // first row of this sequence's matrix in the stacked [B * K, N] weights (0 outside the jagged mode)
      const int w_row0 = a.items ? block_of(blk_of(u)).x * a.K : 0;
      for (int nt = 0; nt < n_tiles && ok; ++nt) {
        for (int kb = 0; kb < kboxes; ++kb) {
#ifdef B200_HSTU_PROFILING
          if (a.dbg & 1) continue;
#endif
          { GEMM_T0(); ok = wait_all(&c.w_empty[st], ph ^ 1); GEMM_T1(tw[0]); }
          if (!ok) break;
          if (elect_one()) {
            const uint32_t dst = smem_u32(wring + st * STAGE_BYTES);
            if constexpr (PAIR) {
              // both halves of the stage are credited to the issuing CTA's barrier; columns past N arrive as zeros
              if (rank == 0) mbar_arrive_expect_tx(smem_u32(&c.w_full[st]), 2 * W_BOX_BYTES);
              if constexpr (FP8)  // W is [N, K]: this CTA's 64 output columns are 64 rows of it, 128 bytes of K each
                tma_load_2d_pair(dst, &maps.w, w_full_issuer + st * 8, kb * 128, tile_of(nt) * BN + static_cast<int>(rank) * 64);
              else
                tma_load_2d_pair(dst, &maps.w, w_full_issuer + st * 8, tile_of(nt) * BN + static_cast<int>(rank) * 64, w_row0 + kb * BK);
            } else {
              mbar_arrive_expect_tx(smem_u32(&c.w_full[st]), STAGE_BYTES);
#pragma unroll
              for (int j = 0; j < 2; ++j)
                tma_load_2d(dst + j * W_BOX_BYTES, &maps.w, smem_u32(&c.w_full[st]), tile_of(nt) * BN + j * 64, w_row0 + kb * BK);
            }
          }
          __syncwarp();
          if (++st == static_cast<uint32_t>(w_stages)) { st = 0; ph ^= 1; }
        }
        // behind the first tile's weights: the next block's rows, which land while this block computes
        if (nt == 0 && ok && u + ustride < n_units) ok = load_x(blk_of(u + ustride));
      }
    }
    GEMM_REPORT("producer (w_empty, x_free)");
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (in a pair: rank 0 only)
    // A from TMEM; B from shared memory, N-major (16-bit: W is [K, N]) or K-major (fp8: W is [N, K])
    constexpr uint32_t IDESC = FP8 ? idesc_f8_e4m3(PAIR ? 2 * BM : BM, BN) : idesc_f16(BF16 ? 1 : 0, PAIR ? 2 * BM : BM, BN, 0, 1);
    constexpr uint32_t KSTEP = FP8 ? (32 >> 4) : (2048 >> 4);  // descriptor units per k-step: 32 bytes along a row / 16 rows
    constexpr uint32_t HI = desc_hi_sw128(1024);
    const uint32_t w_lo0 = desc_lo_sw128(smem_u32(wring), W_BOX_BYTES);  // 64-column groups are one box apart
    const uint32_t w_empty_peer = PAIR ? map_to_cta(smem_u32(&c.w_empty[0]), 1) : 0u;
    const uint32_t w_empty_own = PAIR ? map_to_cta(smem_u32(&c.w_empty[0]), 0) : 0u;
    const uint32_t acc_full_peer = PAIR ? map_to_cta(smem_u32(&c.acc_full[0]), 1) : 0u;
    const uint32_t acc_full_own = PAIR ? map_to_cta(smem_u32(&c.acc_full[0]), 0) : 0u;
    uint32_t it = 0, st = 0, ph = 0, g = 0;
    bool ok = rank == 0;
    [[maybe_unused]] long long tw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    [[maybe_unused]] const long long t_start_ = clock64();
    auto wait_all = [&](unsigned long long* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity, abort_flag, a.status, WAIT_GEMM_MMA));
    };
    for (long long u = u0; u < n_units && ok; u += ustride, ++it) {
      { GEMM_T0(); ok = wait_all(&c.a_ready, it & 1); GEMM_T1(tw[0]); }
      if (!ok) break;
      tc_fence_after();
      for (int nt = 0; nt < n_tiles && ok; ++nt, ++g) {
        const uint32_t buf = g & 1;
        { GEMM_T0(); ok = wait_all(&c.acc_empty[buf], ((g >> 1) & 1) ^ 1); GEMM_T1(tw[1]); }
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + TMEM_ACC0 + buf * BN;
        for (int kb = 0; kb < kboxes; ++kb) {
#ifdef B200_HSTU_PROFILING
          if (a.dbg & 1) {
            if (elect_one() && !(a.dbg & 4)) {
              for (int kk = 0; kk < BK / 16; ++kk) {
                const uint64_t bd = desc_join(w_lo0 + (kb % w_stages) * (STAGE_BYTES >> 4) + kk * KSTEP, HI);
                if constexpr (FP8) mma_ts_pair_f8(d_tmem, tmem + TMEM_A + (kb * 4 + kk) * 8, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                else if constexpr (PAIR) mma_ts_pair(d_tmem, tmem + TMEM_A + (kb * 4 + kk) * 8, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                else mma_ts(d_tmem, tmem + TMEM_A + (kb * 4 + kk) * 8, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
              }
            }
            __syncwarp();
            continue;
          }
#endif
          { GEMM_T0(); ok = wait_all(&c.w_full[st], ph); GEMM_T1(tw[2]); }
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
#ifdef B200_HSTU_PROFILING
            if (!(a.dbg & 4))
#endif
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              // A: 16 k-values = 8 TMEM columns; B: k-step kk of the stage (16 rows of 128 bytes per box)
              const uint64_t bd = desc_join(w_lo0 + st * (STAGE_BYTES >> 4) + kk * KSTEP, HI);
              if constexpr (FP8) mma_ts_pair_f8(d_tmem, tmem + TMEM_A + (kb * 4 + kk) * 8, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
              else if constexpr (PAIR) mma_ts_pair(d_tmem, tmem + TMEM_A + (kb * 4 + kk) * 8, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
              else mma_ts(d_tmem, tmem + TMEM_A + (kb * 4 + kk) * 8, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            if constexpr (PAIR) { tc_commit_pair(w_empty_own + st * 8); tc_commit_pair(w_empty_peer + st * 8); }
            else tc_commit(smem_u32(&c.w_empty[st]));
          }
          __syncwarp();
          if (++st == static_cast<uint32_t>(w_stages)) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        if (elect_one()) {
          if constexpr (PAIR) { tc_commit_pair(acc_full_own + buf * 8); tc_commit_pair(acc_full_peer + buf * 8); }
          else tc_commit(smem_u32(&c.acc_full[buf]));
        }
        __syncwarp();
      }
    }
    GEMM_REPORT("mma (a_ready, acc_empty, w_full)");
  } else if (warp < 10) {
    // ------------------------------------------------------------------ A-operand install + epilogue warps (2..9)
    const int ew = warp - 2;                  // 0..7
    const int wg = ew >> 2;                   // column half of the output tile / k half of the A operand
    const int quad = warp & 3;                // TMEM lane quadrant this warp may touch
    const uint32_t lane_addr = static_cast<uint32_t>(quad << 5) << 16;
    const int row_in_blk = (quad << 5) | lane;
    uint32_t g = 0, xr = 0;
    bool ok = true;
    const bool bias_shared = a.bias_rs == 0 || a.per_seq_bias;
    uint4 bnext = make_uint4(0u, 0u, 0u, 0u);
    [[maybe_unused]] float4 snext = make_float4(0.f, 0.f, 0.f, 0.f);
    [[maybe_unused]] long long tw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    [[maybe_unused]] const long long t_start_ = clock64();
    [[maybe_unused]] long long mark_ = 0;
    if (a.items) {
      // rows at or past the last offset belong to no sequence: defined output (zeros), never stale memory
      long long first = a.off64 ? reinterpret_cast<const long long*>(a.offsets)[a.num_seqs]
                                : static_cast<long long>(reinterpret_cast<const int*>(a.offsets)[a.num_seqs]);
      first = first < 0 ? 0 : (first > a.M ? a.M : first);
      const long long chunks_per_row = a.N >> 3, total = (a.M - first) * chunks_per_row;
      for (long long i = static_cast<long long>(blockIdx.x) * 256 + (threadIdx.x - 64); i < total; i += static_cast<long long>(gridDim.x) * 256) {
        const long long r = first + i / chunks_per_row, col = (i % chunks_per_row) * 8;
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + r * a.out_rs + col) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    // Copies this thread's row of the parked block into the A operand in TMEM (the warp's lane quadrant
    // holds its 32 rows); group wg copies the k-columns of its half of the boxes.
    auto copy_park_to_tmem = [&]() {
      const int half = kboxes >> 1, b0 = wg == 0 ? 0 : half, b1 = wg == 0 ? half : kboxes;
      for (int b = b0; b < b1; ++b) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 2 x 32 elements = 2 x 16 TMEM columns per 64-column box
          uint32_t rr[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int chunk = h * 4 + j;
            const uint4 xq = *reinterpret_cast<const uint4*>(park + b * PARK_BOX_BYTES + row_in_blk * 128 + ((chunk ^ (row_in_blk & 7)) << 4));
            rr[4 * j + 0] = xq.x; rr[4 * j + 1] = xq.y; rr[4 * j + 2] = xq.z; rr[4 * j + 3] = xq.w;
          }
          tmem_st16(tmem + lane_addr + TMEM_A + b * 32 + h * 16, rr);
        }
      }
    };
    // The parked block (rows landed by TMA, or normalised by the layer-norm warps) becomes the A operand.  The caller
    // has made sure that no MMA still reads the previous one.
    auto install_a = [&]() -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait_idle(smem_u32(&c.x_full), xr & 1, abort_flag, a.status, WAIT_GEMM_EPILOGUE))) return false;
      ++xr;
      copy_park_to_tmem();
      tmem_wait_st();
      tc_fence_before();
      arrive_at_issuer(&c.a_ready);
      mbar_arrive(smem_u32(&c.x_free));  // the park may be overwritten
      return true;
    };

    long long u = u0;
    if (u < n_units) {  // the first block's A operand up front
      ok = install_a();
    }
    for (; u < n_units && ok; u += ustride) {
      const int4 bi = block_of(blk_of(u));
      const bool has_next = u + ustride < n_units;
      // ---- epilogue of every output tile of the block: bias, rounding, staged bulk stores.
      // Group wg owns output columns [64 wg, 64 wg + 64) of the tile and sends them out as one box through
      // its own staging buffer (128-byte-swizzled rows, as the bulk tensor store expects).
      const long long row = static_cast<long long>(bi.y) + row_in_blk;
      // Bias.  One row for the whole block (a vector, or the sequence's row in jagged mode): lane l keeps the
      // 16-byte piece l % 8 of the box's 64 columns, fetched one tile AHEAD (with nearly all of the SM's L1
      // carved out as shared memory it comes from L2, a latency no tile should wait for), and the pieces
      // reach the other lanes by shuffles.  A row of its own per output row: loaded where it is used.
      const T* bias_blk = reinterpret_cast<const T*>(a.bias) + (a.per_seq_bias ? bi.x * a.bias_rs : 0);
      const T* bias_row = reinterpret_cast<const T*>(a.bias) + (row < a.M ? row : a.M - 1) * a.bias_rs;
      auto bias_piece = [&](int tile) -> uint4 {
        const int col = tile * BN + wg * 64 + 8 * (lane & 7);
        return (a.bias != nullptr && col < a.N) ? __ldg(reinterpret_cast<const uint4*>(bias_blk + col)) : make_uint4(0u, 0u, 0u, 0u);
      };
      if (bias_shared && (a.per_seq_bias || u == u0)) bnext = bias_piece(tile_of(0));
      // fp8: the scale of this thread's row of A, and the scales of the box's 64 columns of W the way the bias
      // travels (lane l keeps the four of piece l % 16, a tile ahead)
      float row_scale = 1.f;
      auto scale_piece = [&](int tile) -> float4 {
        const int col = tile * BN + wg * 64 + 4 * (lane & 15);
        return col < a.N ? __ldg(reinterpret_cast<const float4*>(a.b_scale + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
      };
      if constexpr (FP8) {
        row_scale = a.a_scale[row < a.M ? row : a.M - 1];
        if (u == u0) snext = scale_piece(tile_of(0));
      }
      unsigned char* stage = out_stage + wg * OUT_BOX_BYTES;
      for (int nt = 0; nt < n_tiles && ok; ++nt, ++g) {
        const uint32_t buf = g & 1;
        const int col0 = tile_of(nt) * BN + wg * 64;
        const uint4 bcur = bnext;
        if (bias_shared) bnext = bias_piece(tile_of(nt + 1 < n_tiles ? nt + 1 : 0));
        [[maybe_unused]] const float4 scur = snext;
        if constexpr (FP8) snext = scale_piece(tile_of(nt + 1 < n_tiles ? nt + 1 : 0));
        { GEMM_T0(); ok = __all_sync(0xffffffffu, mbar_wait_idle(smem_u32(&c.acc_full[buf]), (g >> 1) & 1, abort_flag, a.status, WAIT_GEMM_EPILOGUE)); GEMM_T1(tw[0]); }
        if (!ok) break;
        tc_fence_after();
#ifdef B200_HSTU_PROFILING
        mark_ = clock64();
#endif
        if (nt + 1 == n_tiles && has_next) {
          // The last tile's accumulator is complete, so every MMA of this block has run: the next block's A
          // operand goes into TMEM BEFORE this accumulator is drained, and the MMAs of the next block's
          // first tile (other accumulator) run under the drain.
          ok = install_a();
          if (!ok) break;
        }
        GEMM_MARK(tw[1]);
        const uint32_t acc = tmem + lane_addr + TMEM_ACC0 + buf * BN + wg * 64;
        bool store = bi.z > 0 && col0 < a.N;  // uniform for the group
#ifdef B200_HSTU_PROFILING
        if (a.dbg & 2) store = false;
#endif
        if (store) {
          if (row_in_blk == 0) bulk_wait_read_all();  // the group's previous box has left the staging buffer
          asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");
        }
        GEMM_MARK(tw[5]);
        unsigned char* my_row = stage + row_in_blk * 128;
        uint32_t v0[32], v1[32];  // the box's 64 columns of this thread's row
        tmem_ld32(acc, v0);
        tmem_ld32(acc + 32, v1);
        tmem_wait_ld(v0);
        tmem_wait_ld(v1);
        tc_fence_before();
        arrive_at_issuer(&c.acc_empty[buf]);  // the accumulator is in registers: the MMAs may reuse it
        if (store) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* v = j < 4 ? v0 : v1;
            const int jj = j & 3;
            uint4 bj;
            if (bias_shared) {
              bj.x = __shfl_sync(0xffffffffu, bcur.x, j); bj.y = __shfl_sync(0xffffffffu, bcur.y, j);
              bj.z = __shfl_sync(0xffffffffu, bcur.z, j); bj.w = __shfl_sync(0xffffffffu, bcur.w, j);
            } else {
              const int col = col0 + 8 * j;
              bj = col < a.N ? __ldg(reinterpret_cast<const uint4*>(bias_row + col)) : make_uint4(0u, 0u, 0u, 0u);
            }
            float bf[8];
            vec::unpack8<T>(bj, bf);
            float acc8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc8[e] = __uint_as_float(v[8 * jj + e]);
            if constexpr (FP8) {  // out = (sum of products) * scale of the row of A * scale of the column of W + bias
              float sc[8];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                sc[4 * h + 0] = __shfl_sync(0xffffffffu, scur.x, 2 * j + h); sc[4 * h + 1] = __shfl_sync(0xffffffffu, scur.y, 2 * j + h);
                sc[4 * h + 2] = __shfl_sync(0xffffffffu, scur.z, 2 * j + h); sc[4 * h + 3] = __shfl_sync(0xffffffffu, scur.w, 2 * j + h);
              }
#pragma unroll
              for (int e = 0; e < 8; ++e) acc8[e] *= row_scale * sc[e];
            }
            uint4 o;
            o.x = pack2<BF16>(acc8[0] + bf[0], acc8[1] + bf[1]);
            o.y = pack2<BF16>(acc8[2] + bf[2], acc8[3] + bf[3]);
            o.z = pack2<BF16>(acc8[4] + bf[4], acc8[5] + bf[5]);
            o.w = pack2<BF16>(acc8[6] + bf[6], acc8[7] + bf[7]);
            *reinterpret_cast<uint4*>(my_row + ((j ^ (row_in_blk & 7)) << 4)) = o;
          }
        }
        GEMM_MARK(tw[2]);
        if (store) {
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
        GEMM_MARK(tw[3]);
      }
    }
    if (warp == 2 || warp == 6) GEMM_REPORT("epilogue (acc_full, install, drain, stage+store, -, staging free)");
    if (row_in_blk == 0) bulk_wait_all();  // shared memory must outlive the stores that read it
  } else if (FUSE) {
    // ------------------------------------------------------------------ layer-norm warps (10, 11)
    // The raw rows of the NEXT block land in the park by TMA while the current block computes; each of
    // these warps normalises 64 of the 128 rows IN PLACE (a row at a time across the warp, two 16-byte
    // vectors per lane, each lane writing back exactly what it read), LN_BATCH rows through every stage
    // together.  Nothing here waits for global memory: loads in flight in registers would stall the
    // shuffles and stores of the rows being normalised.
    const int lw = warp - 10;
    const int nv = a.K >> 3;  // 16-byte vectors per row (at most 64: two per lane)
    constexpr int ROWS = BM / LN_WARPS, BATCHES = ROWS / LN_BATCH;
    bool ok = true;
    uint32_t xr = 0;
    [[maybe_unused]] long long tw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    [[maybe_unused]] const long long t_start_ = clock64();
    // layer-norm weight and bias of this lane's columns, as fp32 in registers for the whole kernel
    float wv[2][8], bv[2][8];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int v = lane + 32 * j;
#pragma unroll
      for (int i = 0; i < 8; ++i) { wv[j][i] = 1.f; bv[j][i] = 0.f; }
      if (a.affine && v < nv) {
        vec::unpack8<T>(__ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.ln_w) + 8 * v)), wv[j]);
        vec::unpack8<T>(__ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.ln_b) + 8 * v)), bv[j]);
      }
    }
    // where vector v (8 columns) of row rl lives: box v / 8, 16-byte chunk v % 8 of the 128-byte box row, swizzled
    auto park_at = [&](int v, int rl) -> uint4* {
      return reinterpret_cast<uint4*>(park + (v >> 3) * PARK_BOX_BYTES + rl * 128 + (((v & 7) ^ (rl & 7)) << 4));
    };
    // rows rl0 .. rl0 + 3 of the block whose first row is row0
    auto norm_batch = [&](long long row0, int rl0) {
      float xv[LN_BATCH][2][8], mean[LN_BATCH], rstd[LN_BATCH];
#pragma unroll
      for (int q = 0; q < LN_BATCH; ++q) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int v = lane + 32 * j;
          const uint4 raw = v < nv ? *park_at(v, rl0 + q) : make_uint4(0u, 0u, 0u, 0u);
          vec::unpack8<T>(raw, xv[q][j]);
        }
      }
      // mean first, then the mean of squared deviations (kjt_split_per_feature.cpp:223-226)
#pragma unroll
      for (int q = 0; q < LN_BATCH; ++q) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 2; ++j)
          if (lane + 32 * j < nv) {
#pragma unroll
            for (int i = 0; i < 8; ++i) s += xv[q][j][i];
          }
        mean[q] = s;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int q = 0; q < LN_BATCH; ++q) mean[q] += __shfl_xor_sync(0xffffffffu, mean[q], o);
      }
#pragma unroll
      for (int q = 0; q < LN_BATCH; ++q) {
        mean[q] /= static_cast<float>(a.K);
        float sq = 0.f;
#pragma unroll
        for (int j = 0; j < 2; ++j)
          if (lane + 32 * j < nv) {
#pragma unroll
            for (int i = 0; i < 8; ++i) { const float d = xv[q][j][i] - mean[q]; sq += d * d; if (!a.swish) xv[q][j][i] = d; }
          }
        rstd[q] = sq;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int q = 0; q < LN_BATCH; ++q) rstd[q] += __shfl_xor_sync(0xffffffffu, rstd[q], o);
      }
#pragma unroll
      for (int q = 0; q < LN_BATCH; ++q) {
        rstd[q] = rsqrtf(rstd[q] / static_cast<float>(a.K) + a.eps);
        const long long row = row0 + rl0 + q;
        if (lane == 0 && row < a.M) { a.mean[row] = mean[q]; a.rstd[row] = rstd[q]; }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int v = lane + 32 * j;
          if (v >= nv) continue;
          uint4 pk = make_uint4(0u, 0u, 0u, 0u);  // rows past M enter the product as zeros
          if (row < a.M) {
            float n[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              // (without the swish gate xv already holds x - mean; with it x itself is needed once more)
              float y = (a.swish ? xv[q][j][i] - mean[q] : xv[q][j][i]) * rstd[q];
              y = y * wv[j][i] + bv[j][i];  // (weight 1 and bias 0 without the affine part: exact)
              if (a.swish) y = __fdividef(1.f, 1.f + __expf(-y)) * xv[q][j][i];
              n[i] = y;
            }
            pk.x = pack2<BF16>(n[0], n[1]); pk.y = pack2<BF16>(n[2], n[3]);
            pk.z = pack2<BF16>(n[4], n[5]); pk.w = pack2<BF16>(n[6], n[7]);
          }
          *park_at(v, rl0 + q) = pk;
        }
      }
    };
    for (long long u = u0; u < n_units && ok; u += ustride, ++xr) {
      { GEMM_T0(); ok = __all_sync(0xffffffffu, mbar_wait_idle(smem_u32(&c.x_raw), xr & 1, abort_flag, a.status, WAIT_GEMM_PRODUCER)); GEMM_T1(tw[0]); }
      if (!ok) break;
      const long long row0 = block_of(blk_of(u)).y;
      for (int b = 0; b < BATCHES; ++b) norm_batch(row0, lw * ROWS + b * LN_BATCH);
      fence_proxy_async();  // (the next block's rows will be written over these by TMA)
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&c.x_full));  // a release: the normalised rows are in the park
    }
    GEMM_REPORT("layer norm (raw rows landed)");
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // neither CTA leaves while the other may still signal it
  if (warp == 0) {
    if (*abort_flag) {  // a wait gave up: let copies and MMAs in flight finish before the TMEM is released
      const unsigned long long t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
    }
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, TMEM_COLS);
    else tmem_dealloc(tmem, TMEM_COLS);
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
// One persistent CTA (or CTA pair) per SM (pair of SMs), fewer if there are not that many row blocks.
template <typename Kern>
int launch_kernel(Kern kern, bool pair, long long max_blocks, const hstu::gemm::Maps& maps, const hstu::gemm::Args& a, void* stream) {
  using namespace hstu::gemm;
  const int sms = hstu::tc::sm_count();
  const long long units = pair ? (max_blocks + 1) / 2 : max_blocks;
  const long long ctas = pair ? sms / 2 : sms;
  const unsigned grid = static_cast<unsigned>((units < ctas ? (units < 1 ? 1 : units) : ctas) * (pair ? 2 : 1));
  const size_t smem = CONTROL_BYTES + DATA_BYTES;  // 227 KB: all a CTA can have
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return B200_HSTU_ELAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pair ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kern, maps, a);
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? B200_HSTU_OK : B200_HSTU_ELAUNCH;
}

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
  if (!hstu::tc::make_map_box(&maps.x, p->x, p->M, p->K, p->x_row_stride, BM, bf16)) return B200_HSTU_ELAUNCH;
  Args a;
  a.x = p->x; a.ln_w = p->ln_weight; a.ln_b = p->ln_bias; a.bias = p->bias; a.out = p->out;
  a.mean = p->mean; a.rstd = p->rstd; a.status = p->status;
  a.M = p->M; a.x_rs = p->x_row_stride; a.out_rs = p->out_row_stride; a.bias_rs = p->bias_row_stride;
  a.K = static_cast<int>(p->K); a.N = static_cast<int>(p->N);
  a.fuse_ln = fuse ? 1 : 0; a.swish = (p->flags & B200_GEMM_FLAG_SWISH) ? 1 : 0; a.affine = p->ln_weight ? 1 : 0;
  a.eps = p->eps;
  a.items = items; a.n_items = n_items; a.per_seq_bias = per_seq_bias;
  a.offsets = offsets; a.off64 = off64; a.num_seqs = num_seqs;
  a.a_scale = a.b_scale = nullptr;
  a.dbg = 0;
#ifdef B200_HSTU_PROFILING
  if (const char* e = getenv("B200_GEMM_DBG")) a.dbg = atoi(e);
#endif
  const int sms = hstu::tc::sm_count();
  const bool pair = items == nullptr && sms >= 2;  // per-sequence weights cannot share a B operand across two row blocks
  if (fuse && !pair) return B200_HSTU_EUNSUPPORTED;  // (the jagged mode has no layer-norm prologue)
  auto kern = fuse   ? (bf16 ? stu_addmm_tc<1, true, true> : stu_addmm_tc<0, true, true>)
              : pair ? (bf16 ? stu_addmm_tc<1, true, false> : stu_addmm_tc<0, true, false>)
                     : (bf16 ? stu_addmm_tc<1, false, false> : stu_addmm_tc<0, false, false>);
  hstu::set_error_stage("addmm: kernel");
  return launch_kernel(kern, pair, max_blocks, maps, a, stream);
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

extern "C" int b200_stu_fp8_rowwise_addmm_supported(const B200Fp8GemmParams* p) {
  if (p == nullptr || p->struct_size != sizeof(B200Fp8GemmParams)) return 0;
  if (p->out_dtype != B200_HSTU_BF16) return 0;
  if (p->M <= 0 || p->K <= 0 || p->N <= 0) return 0;
  if (p->K % 128 != 0 || p->K > 2 * hstu::gemm::MAX_K || p->N % 8 != 0) return 0;
  if (p->M >= (1LL << 31) - 256 || p->N >= (1LL << 30)) return 0;
  return hstu::tc::sm_count() >= 2 ? 1 : 0;
}

extern "C" int b200_stu_fp8_rowwise_addmm(const B200Fp8GemmParams* p, void* stream) {
  using namespace hstu::gemm;
  if (p == nullptr) return B200_HSTU_EINVAL;
  if (p->struct_size != sizeof(B200Fp8GemmParams)) return B200_HSTU_EVERSION;
  if (p->M < 0 || p->K <= 0 || p->N <= 0) return B200_HSTU_EINVAL;
  if (p->M == 0) return B200_HSTU_OK;
  if (!b200_stu_fp8_rowwise_addmm_supported(p)) return B200_HSTU_EUNSUPPORTED;
  if (!p->a || !p->b || !p->a_scale || !p->b_scale || !p->out) return B200_HSTU_EINVAL;
  if (p->a_row_stride < p->K || p->b_row_stride < p->K || p->out_row_stride < p->N) return B200_HSTU_EINVAL;
  auto bad = [](const void* q, long long stride, int unit) { return reinterpret_cast<uintptr_t>(q) % 16 != 0 || stride % unit != 0; };
  if (bad(p->a, p->a_row_stride, 16) || bad(p->b, p->b_row_stride, 16) || bad(p->out, p->out_row_stride, 8) ||
      bad(p->b_scale, 0, 1) || (p->bias && bad(p->bias, 0, 1)))
    return B200_HSTU_EALIGN;
  hstu::set_error_stage("fp8 addmm: tensor maps");
  if (!hstu::tc::ensure_current_context(p->a)) return B200_HSTU_ELAUNCH;
  Maps maps;
  if (!hstu::tc::make_map_bytes(&maps.x, p->a, p->M, p->K, p->a_row_stride, BM)) return B200_HSTU_ELAUNCH;
  if (!hstu::tc::make_map_bytes(&maps.w, p->b, p->N, p->K, p->b_row_stride, 64)) return B200_HSTU_ELAUNCH;
  if (!hstu::tc::make_map_box(&maps.o, p->out, p->M, p->N, p->out_row_stride, BM, true)) return B200_HSTU_ELAUNCH;
  Args a;
  a.x = p->a; a.ln_w = nullptr; a.ln_b = nullptr; a.bias = p->bias; a.out = p->out;
  a.mean = nullptr; a.rstd = nullptr; a.status = p->status;
  a.M = p->M; a.x_rs = p->a_row_stride; a.out_rs = p->out_row_stride; a.bias_rs = 0;
  a.K = static_cast<int>(p->K); a.N = static_cast<int>(p->N);
  a.fuse_ln = 0; a.swish = 0; a.affine = 0; a.eps = 0.f;
  a.items = nullptr; a.n_items = nullptr; a.per_seq_bias = 0;
  a.offsets = nullptr; a.off64 = 0; a.num_seqs = 0;
  a.a_scale = p->a_scale; a.b_scale = p->b_scale;
  a.dbg = 0;
  hstu::set_error_stage("fp8 addmm: kernel");
  return launch_kernel(stu_addmm_tc<2, true, false>, true, (p->M + BM - 1) / BM, maps, a, stream);
}
