// Streaming GEMV instantiations for one block type (see gemv_impl.cuh).
#include "gemv_impl.cuh"

namespace spm {
namespace gemv {
template cudaError_t launch_enc<SPM_Q5_K>(const GemvLaunch&, bool, int, int, size_t, cudaStream_t, bool);
template int occupancy_enc<SPM_Q5_K>(const GemvLaunch&, bool, int, size_t);
}  // namespace gemv
}  // namespace spm
