// Host-side helpers shared by the tensor-core translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "hstu_tc_common.cuh"

namespace hstu {
namespace tc {

// Tensor map over a [rows, width] 16-bit matrix with the given row stride (elements):
// box = 64 columns x 128 rows, 128-byte swizzle, zero fill outside the matrix.
// Makes sure the calling thread has a current CUDA context (needed by the tensor-map encoder).
bool ensure_current_context(const void* device_ptr);
bool make_map(CUtensorMap* m, const void* base, long long rows, long long width, long long row_stride, bool bf16);
bool make_map_box(CUtensorMap* m, const void* base, long long rows, long long width, long long row_stride, int box_rows,
                  bool bf16);
// The same over a [rows, width] matrix of bytes: box = 128 columns x box_rows rows.
bool make_map_bytes(CUtensorMap* m, const void* base, long long rows, long long width, long long row_stride, int box_rows);
int sm_count();
// Grid of the persistent kernels (also the stride with which CTAs walk the work list).
int main_grid(const WorkspaceLayout& w);
// Workspace layout of a backward call (work list, and the stored dS tiles when they are used).
WorkspaceLayout backward_layout(const KernelArgs& a);
// Builds the work list in the workspace and zeroes the output rows no sequence owns.
cudaError_t launch_prep(const KernelArgs& a, bool bf16, int* ws, const WorkspaceLayout& w, bool backward,
                        cudaStream_t st);

// Launches `kern` so that it may be scheduled while the kernel before it in the stream still runs
// (programmatic dependent launch): the kernel before must execute grid_launch_dependents(), and `kern`
// must execute grid_dependency_wait() before it reads anything that kernel wrote.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                                    bool dependent, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dependent ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Launches the bounded-wait self-test kernel (see b200_hstu_debug_bounded_wait).
cudaError_t launch_bounded_wait_probe(int* status, int code, unsigned long long limit_ns, cudaStream_t st);

}  // namespace tc
}  // namespace hstu
