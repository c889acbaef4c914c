// tcgen05 chunk path (bf16/fp16, K = V = 128).  Placeholder until the
// tensor-core kernels land: the generic path serves every shape.
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
bool tc_path_applies(const gdn_chunk_args&) { return false; }
size_t tc_workspace_bytes(const gdn_chunk_args&) { return 0; }
cudaError_t launch_chunk_tc(const gdn_chunk_args&, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace gdn
