// Internal launch interface between the C ABI and the kernel translation units.
#pragma once
#include <cuda_runtime.h>

#include "hstu_common.cuh"

namespace hstu {

// Names the step a launch function is in; a failing call reports it through
// b200_hstu_last_cuda_error().  `what` must be a string literal.
void set_error_stage(const char* what);

// CUDA-core kernels (hstu_simt.cu): zero the unowned tail rows, then run the pass.
cudaError_t simt_forward(const KernelArgs& a, int dtype, int max_seq_len, cudaStream_t st);
cudaError_t simt_backward(const KernelArgs& a, int dtype, int max_seq_len, cudaStream_t st);
cudaError_t zero_tail(const KernelArgs& a, int dtype, bool backward, cudaStream_t st);

}  // namespace hstu

namespace hstu {

// Tensor-core (TMA + tcgen05/TMEM) kernels (hstu_tc.cu).
bool tc_supported(const B200HstuParams& p, const KernelArgs& a, int pass);
size_t tc_workspace_bytes(const KernelArgs& a, int pass);
int tc_launch_count(const KernelArgs& a, int pass);
cudaError_t tc_forward(const KernelArgs& a, int dtype, void* workspace, cudaStream_t st);
cudaError_t tc_backward(const KernelArgs& a, int dtype, void* workspace, cudaStream_t st);

}  // namespace hstu
