// Launch entry points of the sequential-chain kernels, shared by the
// operators that own their weights (ternary.cu, dense.cu) and the host-to-HBM
// sweep (sweep.cu), which points them at a ring slot instead.
#pragma once
#include <cuda_runtime.h>

#include "dense_kernel.cuh"
#include "qblock_kernel.cuh"
#include "ternary_kernel.cuh"

namespace spm {

// Both return cudaErrorInvalidConfiguration when rows x chains need more
// than 2^31 - 1 blocks.
cudaError_t launch_ternary_gemv(const TernaryArgs& a, int sms, cudaStream_t stream);
cudaError_t launch_dense_streamed(const DenseArgs& a, bool bf16, int sms, cudaStream_t stream);
// encoding: the .spm code of a block profile (SPM_ENC_Q8_0, _Q6K, _Q5K).
cudaError_t launch_qblock_chain(const QBlockArgs& a, uint8_t encoding, int sms, cudaStream_t stream);

}  // namespace spm
