// C ABI of the library (declared in include/b200_hstu.h): argument validation, kernel
// selection and launch.  No device allocation, no synchronisation, caller's stream only.
#include <cuda_runtime.h>
#include <string.h>

#include <stdio.h>

#include <mutex>

#include "hstu_common.cuh"
#include "hstu_launch.h"
#include "hstu_tc_common.cuh"
#include "hstu_tc_host.h"

using hstu::KernelArgs;

namespace {

int elem_size(int dtype) { return dtype == B200_HSTU_F32 ? 4 : 2; }

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Validates the arguments one pass needs and fills the kernel argument block.
int validate(const B200HstuParams* p, int pass, KernelArgs* a) {
  if (p == nullptr) return B200_HSTU_EINVAL;
  if (p->struct_size != sizeof(B200HstuParams)) return B200_HSTU_EVERSION;
  if (p->dtype != B200_HSTU_F32 && p->dtype != B200_HSTU_BF16 && p->dtype != B200_HSTU_F16)
    return B200_HSTU_EUNSUPPORTED;
  if (p->T < 0 || p->B < 0 || p->H <= 0 || p->Dqk <= 0 || p->Dv <= 0) return B200_HSTU_EINVAL;
  if (p->B > 65535 || p->H > 65535) return B200_HSTU_EUNSUPPORTED;
  if (p->Dqk > 256 || p->Dv > 256) return B200_HSTU_EUNSUPPORTED;
  if (p->max_seq_len <= 0 || p->max_attn_len < 0 || p->contextual_seq_len < 0 || p->full_attn_size < 0)
    return B200_HSTU_EINVAL;
  if (p->seq_offsets == nullptr) return B200_HSTU_EINVAL;
  if (p->T > 0 && (p->q == nullptr || p->k == nullptr || p->v == nullptr)) return B200_HSTU_EINVAL;
  const long long wq = (long long)p->H * p->Dqk, wv = (long long)p->H * p->Dv;
  if (p->q_row_stride < wq || p->k_row_stride < wq || p->v_row_stride < wv) return B200_HSTU_EINVAL;
  if (pass == 0) {
    if (p->T > 0 && p->o == nullptr) return B200_HSTU_EINVAL;
    if (p->o_row_stride < wv) return B200_HSTU_EINVAL;
  } else {
    if (p->T > 0 && (p->d_o == nullptr || p->dq == nullptr || p->dk == nullptr || p->dv == nullptr))
      return B200_HSTU_EINVAL;
    if (p->do_row_stride < wv || p->dq_row_stride < wq || p->dk_row_stride < wq || p->dv_row_stride < wv)
      return B200_HSTU_EINVAL;
  }
  const size_t es = elem_size(p->dtype);
  const void* ptrs[] = {p->q, p->k, p->v, p->o, p->d_o, p->dq, p->dk, p->dv};
  for (const void* x : ptrs)
    if (!aligned(x, es)) return B200_HSTU_EALIGN;
  if (!aligned(p->seq_offsets, (p->flags & B200_HSTU_FLAG_OFFSETS_I64) ? 8 : 4)) return B200_HSTU_EALIGN;
  if (p->num_targets && !aligned(p->num_targets, (p->flags & B200_HSTU_FLAG_TARGETS_I64) ? 8 : 4))
    return B200_HSTU_EALIGN;
  if (p->attn_scale && !aligned(p->attn_scale, 4)) return B200_HSTU_EALIGN;

  memset(a, 0, sizeof(*a));
  a->q = p->q; a->k = p->k; a->v = p->v; a->o = p->o; a->d_o = p->d_o;
  a->dq = p->dq; a->dk = p->dk; a->dv = p->dv;
  a->seq_offsets = p->seq_offsets; a->num_targets = p->num_targets; a->attn_scale = p->attn_scale;
  a->status = p->status;
  a->trace_buf = (p->flags & B200_HSTU_FLAG_TRACE) ? p->status : nullptr;
  a->T = p->T;
  a->q_rs = p->q_row_stride; a->k_rs = p->k_row_stride; a->v_rs = p->v_row_stride; a->o_rs = p->o_row_stride;
  a->do_rs = p->do_row_stride; a->dq_rs = p->dq_row_stride; a->dk_rs = p->dk_row_stride; a->dv_rs = p->dv_row_stride;
  a->B = p->B; a->H = p->H; a->Dqk = p->Dqk; a->Dv = p->Dv;
  a->offsets_i64 = (p->flags & B200_HSTU_FLAG_OFFSETS_I64) ? 1 : 0;
  a->targets_i64 = (p->flags & B200_HSTU_FLAG_TARGETS_I64) ? 1 : 0;
  a->scale_mode = p->attn_scale == nullptr ? 0 : ((p->flags & B200_HSTU_FLAG_SCALE_PER_TOKEN) ? 2 : 1);
  a->skip_dq = (p->flags & B200_HSTU_FLAG_BWD_SKIP_DQ) ? 1 : 0;
  a->skip_dkv = (p->flags & B200_HSTU_FLAG_BWD_SKIP_DKV) ? 1 : 0;
  a->max_seq_len = static_cast<int>(p->max_seq_len > 0x3fffffff ? 0x3fffffff : p->max_seq_len);
  a->recompute_dq = (p->flags & B200_HSTU_FLAG_BWD_RECOMPUTE_DQ) ? 1 : 0;
  a->ds_tiles = nullptr; a->ds_tile_base = nullptr; a->ds_tile_cap = 0; a->ds_square = 0;
  a->alpha = p->alpha;
  a->inv_n = 1.0f / static_cast<float>(p->max_seq_len);
  a->mask.causal = (p->flags & B200_HSTU_FLAG_CAUSAL) ? 1 : 0;
  a->mask.window = p->max_attn_len;
  a->mask.ctx = p->contextual_seq_len > 0 ? 1 : 0;
  a->mask.full = p->full_attn_size;
  return B200_HSTU_OK;
}

}  // namespace

static thread_local char g_last_cuda_error[192] = "";
static thread_local const char* g_error_stage = "";

namespace hstu {
void set_error_stage(const char* what) { g_error_stage = what; }
}  // namespace hstu

extern "C" {

int b200_hstu_version(void) { return B200_HSTU_ABI_VERSION; }

size_t b200_hstu_params_size(void) { return sizeof(B200HstuParams); }

const char* b200_hstu_strerror(int code) {
  switch (code) {
    case B200_HSTU_OK: return "ok";
    case B200_HSTU_EINVAL: return "invalid argument (null pointer, negative size or row stride smaller than H*D)";
    case B200_HSTU_EUNSUPPORTED: return "unsupported dtype, head dimension (> 256) or batch/head count (> 65535)";
    case B200_HSTU_EALIGN: return "pointer or stride not aligned as required";
    case B200_HSTU_EWORKSPACE: return "workspace missing, misaligned or smaller than b200_hstu_workspace_bytes()";
    case B200_HSTU_ELAUNCH: return "CUDA launch or driver call failed";
    case B200_HSTU_EVERSION: return "struct_size does not match this library's B200HstuParams";
    case B200_HSTU_ESCRATCH: return "work list larger than the built-in scratch array (B200_HSTU_STATIC_SCRATCH_BYTES)";
    default: return "unknown b200_hstu error code";
  }
}

int b200_hstu_uses_tensor_cores(const B200HstuParams* p, int pass) {
  KernelArgs a;
  const int rc = validate(p, pass, &a);
  if (rc != B200_HSTU_OK) return rc;
  return hstu::tc_supported(*p, a, pass) ? 1 : 0;
}

size_t b200_hstu_workspace_bytes(const B200HstuParams* p, int pass) {
  KernelArgs a;
  if (validate(p, pass, &a) != B200_HSTU_OK) return 0;
  if (!hstu::tc_supported(*p, a, pass)) return 0;
  return hstu::tc_workspace_bytes(a, pass);
}

int b200_hstu_launch_count(const B200HstuParams* p, int pass) {
  KernelArgs a;
  const int rc = validate(p, pass, &a);
  if (rc != B200_HSTU_OK) return rc;
  if (hstu::tc_supported(*p, a, pass)) return hstu::tc_launch_count(a, pass);
  if (a.B <= 0 || a.T <= 0) return 1;
  return pass == 0 ? 2 : 3;
}


static int launch_result(cudaError_t e) {
  if (e == cudaSuccess) return B200_HSTU_OK;
  snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s [%s]", cudaGetErrorName(e), cudaGetErrorString(e),
           g_error_stage);
  return B200_HSTU_ELAUNCH;
}

const char* b200_hstu_last_cuda_error(void) { return g_last_cuda_error; }


static int run(const B200HstuParams* p, int pass, void* stream) {
  KernelArgs a;
  const int rc = validate(p, pass, &a);
  if (rc != B200_HSTU_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (hstu::tc_supported(*p, a, pass)) {
    const size_t need = hstu::tc_workspace_bytes(a, pass);
    if (need > 0 && (p->workspace == nullptr || p->workspace_bytes < need || !aligned(p->workspace, 256)))
      return B200_HSTU_EWORKSPACE;
    e = pass == 0 ? hstu::tc_forward(a, p->dtype, p->workspace, st)
                  : hstu::tc_backward(a, p->dtype, p->workspace, st);
  } else {
    e = pass == 0 ? hstu::simt_forward(a, p->dtype, p->max_seq_len, st)
                  : hstu::simt_backward(a, p->dtype, p->max_seq_len, st);
  }
  return launch_result(e);
}

static void mask_query(const B200HstuMaskQuery* mq, hstu::SeqInfo* s, hstu::MaskOpts* o) {
  s->start = 0;
  s->len = mq->len;
  s->has_targets = mq->has_targets ? 1 : 0;
  const int t = mq->has_targets ? mq->num_targets : 0;
  s->hist = mq->has_targets ? mq->len - t : mq->len;
  s->boundary = mq->len - t - mq->full_attn_size;
  o->causal = mq->causal ? 1 : 0;
  o->window = mq->max_attn_len;
  o->ctx = mq->contextual_seq_len > 0 ? 1 : 0;
  o->full = mq->full_attn_size;
}

int b200_hstu_debug_keep(const B200HstuMaskQuery* mq, int m, int n) {
  hstu::SeqInfo s; hstu::MaskOpts o;
  mask_query(mq, &s, &o);
  return hstu::keep(m, n, s, o) ? 1 : 0;
}

int b200_hstu_debug_classify_tile(const B200HstuMaskQuery* mq, int m0, int n0, int rows_dont_care) {
  hstu::SeqInfo s; hstu::MaskOpts o;
  mask_query(mq, &s, &o);
  return hstu::tc::classify_tile(m0, n0, s, o, rows_dont_care != 0);
}

void b200_hstu_debug_row_mask(const B200HstuMaskQuery* mq, int m, int32_t out[4]) {
  hstu::SeqInfo s; hstu::MaskOpts o;
  mask_query(mq, &s, &o);
  const hstu::tc::RowMask r = hstu::tc::row_mask(m, s, o);
  out[0] = r.lo; out[1] = r.hi; out[2] = r.diag; out[3] = r.extra;
}

void b200_hstu_debug_col_mask(const B200HstuMaskQuery* mq, int n, int32_t out[4]) {
  hstu::SeqInfo s; hstu::MaskOpts o;
  mask_query(mq, &s, &o);
  const hstu::tc::ColMask c = hstu::tc::col_mask(n, s, o);
  out[0] = c.a_lo; out[1] = c.a_hi; out[2] = c.b_lo; out[3] = c.diag;
}

void b200_hstu_debug_key_blocks(const B200HstuMaskQuery* mq, int m0, int32_t out[3]) {
  hstu::SeqInfo s; hstu::MaskOpts o;
  mask_query(mq, &s, &o);
  const hstu::tc::BlockRange r = hstu::tc::key_blocks_for_query_block(m0, s, o);
  out[0] = r.lo; out[1] = r.hi; out[2] = r.extra0;
}

void b200_hstu_debug_query_blocks(const B200HstuMaskQuery* mq, int n0, int32_t out[3]) {
  hstu::SeqInfo s; hstu::MaskOpts o;
  mask_query(mq, &s, &o);
  const hstu::tc::BlockRange r = hstu::tc::query_blocks_for_key_block(n0, s, o);
  out[0] = r.lo; out[1] = r.hi; out[2] = r.extra0;
}

int b200_hstu_fwd(const B200HstuParams* p, void* stream) { return run(p, 0, stream); }

}  // extern "C"

// ---- forward with built-in scratch -------------------------------------------------------
// The work list of the tensor-core forward lives in this array instead of caller memory.
// In host code the name below is only a handle for the runtime: the device address has to be
// looked up per device with cudaGetSymbolAddress and that pointer is what the kernels get.
static __device__ __align__(256) unsigned char g_static_scratch[B200_HSTU_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the device that owns `device_ptr` (looked up once per device).
// That device is made current for the lookup: on a host thread that has no context yet, or whose
// current device is another one, the symbol would otherwise resolve to the wrong GPU's copy.
int static_scratch_address(const void* device_ptr, void** out) {
  int dev = -1;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, device_ptr) == cudaSuccess && at.type == cudaMemoryTypeDevice) dev = at.device;
  else if (cudaGetDevice(&dev) != cudaSuccess) return B200_HSTU_ELAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return B200_HSTU_ELAUNCH;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != dev) {
    if (cudaSetDevice(dev) != cudaSuccess) return B200_HSTU_ELAUNCH;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_static_scratch) != cudaSuccess || ptr == nullptr) return B200_HSTU_ELAUNCH;
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return B200_HSTU_OK;
}
}  // namespace

extern "C" {

int b200_hstu_fwd_static_scratch(const B200HstuParams* p, void* stream) {
  KernelArgs a;
  const int rc = validate(p, 0, &a);
  if (rc != B200_HSTU_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (hstu::tc_supported(*p, a, 0)) {
    if (hstu::tc_workspace_bytes(a, 0) > B200_HSTU_STATIC_SCRATCH_BYTES) return B200_HSTU_ESCRATCH;
    void* scratch = nullptr;
    const int src = static_scratch_address(p->q, &scratch);
    if (src != B200_HSTU_OK) return src;
    e = hstu::tc_forward(a, p->dtype, scratch, st);
  } else {
    e = hstu::simt_forward(a, p->dtype, p->max_seq_len, st);  // needs no scratch at all
  }
  return launch_result(e);
}
int b200_hstu_bwd(const B200HstuParams* p, void* stream) { return run(p, 1, stream); }

int b200_hstu_debug_bounded_wait(int32_t* status, int code, uint64_t limit_ns, void* stream) {
  if (status == nullptr || limit_ns == 0 || limit_ns > 100000000ull) return B200_HSTU_EINVAL;  // at most 0.1 s
  hstu::set_error_stage("bounded-wait probe");
  return launch_result(hstu::tc::launch_bounded_wait_probe(status, code, limit_ns, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
