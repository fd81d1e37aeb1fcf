// kda_chunk_tc.cu -- tcgen05 tensor-core chunkwise KDA (sm_100a).
#include "kda_internal.cuh"

namespace kda {

bool chunk_tc_supported(const ChunkParams&) { return false; }
size_t chunk_tc_workspace_bytes(const ChunkParams&) { return 0; }
cudaError_t launch_chunk_tc(const ChunkParams&, void*, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace kda
