// kda_internal.cuh -- parameter blocks shared by the C-ABI layer and kernels.
#pragma once

#include <cuda.h>   // CUtensorMap and its enums (header only)
#include <cuda_runtime.h>

#include <utility>

#include "kda_common.cuh"

namespace kda {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda);
// nullptr when the driver does not provide it
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled encode_tiled();

// Launch with programmatic stream serialization: the grid may start while the
// previous kernel on the stream is still running (once all of that kernel's
// CTAs have executed griddepcontrol.launch_dependents, or exited); it must
// execute griddepcontrol.wait before touching anything that kernel writes.
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*k)(Params...), dim3 grid, int threads, size_t smem,
                             cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

namespace mla {
int read_device_error(bool clear);   // the MLA kernels' error word (mla_decode.cu)
}

constexpr int kRecMaxK = 256;    // recurrent kernel: K <= 256, any V
constexpr int kSimtMaxK = 256;   // SIMT chunkwise kernel: K <= 256, any V

// Device-side view of KdaArgs (strides in elements, innermost stride == 1).
struct RecParams {
  int B, T, H, K, V;
  int io_dtype, state_in_dtype, state_out_dtype;
  float scale;
  const void* q; int64_t q_s[4];
  const void* k; int64_t k_s[4];
  const void* v; int64_t v_s[4];
  const float* g; int64_t g_s[4];
  const float* beta; int64_t b_s[3];
  const void* state_in; int64_t si_s[4];
  void* o; int64_t o_s[4];
  void* state_out; int64_t so_s[4];
  // 16-byte vector access is legal for 4 consecutive columns
  bool state_vec, state_out_vec, o_vec;
  // 16-byte access is legal for 8 consecutive 16-bit v / o elements
  bool v_vec16, o_vec16;
  // 2-element access is legal (g: 8 bytes; q, k and v: 4 bytes)
  bool g_vec2, qk_vec2, v_vec2;
  // run the CUDA-core chunkwise kernel even where the tensor-core one applies
  bool force_simt;
};

using ChunkParams = RecParams;

// Device-side view of KdaPrologueArgs (strides in elements).
struct PrologueParams {
  int B, T, H, K, V, conv_size;
  int io_dtype, gate_dtype;
  float eps;
  const void *q_in, *k_in, *v_in;
  int64_t in_s[3][2];                  // (batch, time) strides of q_in, k_in, v_in
  const float *w_q, *w_k, *w_v;        // [D, conv_size]
  const float *b_q, *b_k, *b_v;        // [D] or null
  const void *hist_q, *hist_k, *hist_v;
  int64_t hist_bs[3];                  // batch strides of the histories
  void *new_q, *new_k, *new_v;         // [B, conv_size - 1, D] contiguous, or null
  const void* gk; int64_t gk_s[2];
  const void* beta_logit; int64_t bl_s[2];
  const float *A_log, *dt_bias;        // [H, K]
  void *q, *k, *v;
  int64_t out_s[3][4];
  float* g; int64_t g_s[4];
  float* beta; int64_t beta_s[3];
};

// Device-side view of KdaEpilogueArgs.
struct EpilogueParams {
  int B, T, H, V, io_dtype;
  float eps;
  const void* o; int64_t o_s[4];
  const void* og; int64_t og_s[2];
  const float* weight;
  void* y; int64_t y_s[2];
};

// Device-side view of KdaBackwardArgs.
struct BwdParams {
  int B, T, H, K, V, io_dtype, state_in_dtype;
  float scale;
  const void* q; int64_t q_s[4];
  const void* k; int64_t k_s[4];
  const void* v; int64_t v_s[4];
  const float* g; int64_t g_s[4];
  const float* beta; int64_t b_s[3];
  const void* state_in; int64_t si_s[4];
  const void* dout; int64_t do_s[4];
  const float* dstate_out; int64_t dso_s[4];
  float *dq_part, *dk_part, *dg_part, *dbeta_part;
  float* dv; int64_t dv_s[4];
  float* dstate_in; int64_t dsi_s[4];
  float* ckpt;
  // optional final sums of the partials (dq == nullptr: partials only)
  void* dq; int64_t dq_s[4];
  void* dk; int64_t dk_s[4];
  float* dg; int64_t dg_s[4];
  float* dbeta; int64_t dbeta_s[3];
};

size_t backward_ckpt_floats(int B, int H, int T, int K, int V);
cudaError_t launch_backward(const BwdParams& p, cudaStream_t s);
// dq, dk, dg, dbeta = sums of the V/16 partials (after launch_backward)
cudaError_t launch_backward_reduce(const BwdParams& p, cudaStream_t s);
// chunkwise backward (kda_backward_chunk.cu): writes dq, dk, dv, dg, dbeta and
// dstate_in directly (no partials); needs dq set, V <= 128 and a workspace of
// backward_chunk_ws_floats() floats in ckpt
bool backward_chunk_supported(const BwdParams& p);
size_t backward_chunk_ws_floats(int B, int H, int T, int K, int V);
cudaError_t launch_backward_chunk(const BwdParams& p, cudaStream_t s);

cudaError_t launch_prologue(const PrologueParams& p, cudaStream_t s);
cudaError_t launch_epilogue(const EpilogueParams& p, cudaStream_t s);

cudaError_t launch_recurrent(const RecParams& p, cudaStream_t s);
cudaError_t launch_chunk_simt(const ChunkParams& p, cudaStream_t s);
bool chunk_tc_supported(const ChunkParams& p);
size_t chunk_tc_workspace_bytes(const ChunkParams& p);
cudaError_t launch_chunk_tc(const ChunkParams& p, void* workspace, cudaStream_t s);
// error word set by kernels whose bounded waits gave up (0 = none)
int read_device_error(bool clear);

}  // namespace kda
