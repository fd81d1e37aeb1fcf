// kda_capi.cu -- extern "C" entry points declared in include/kda_b200.h.
//
// Validates a KdaArgs block (shapes, dtypes, strides, alignment, device
// architecture), converts it to the kernels' parameter block and launches on
// the caller's stream.  Nothing here synchronises, allocates or reads device
// memory, so both entry points can be captured in a CUDA graph.
#include <cstring>
#include <mutex>

#include "kda_internal.cuh"

namespace kda {

EncodeTiled encode_tiled() {
  static EncodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
    tried = true;
  }
  return fn;
}

}  // namespace kda

namespace kda {


namespace {

constexpr int kMaxDevices = 64;
int g_arch_ok[kMaxDevices];   // 0 = unknown, 1 = sm_100, -1 = other
std::mutex g_arch_mu;

int elt_size(int dt) { return dt == KDA_DTYPE_F32 ? 4 : 2; }
bool dtype_ok(int dt) { return dt == KDA_DTYPE_F32 || dt == KDA_DTYPE_F16 || dt == KDA_DTYPE_BF16; }

// 1 when the current device is compute capability 10.0 (B200 family).
int check_arch() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KDA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return KDA_ERR_ARCH;
  int known = __atomic_load_n(&g_arch_ok[dev], __ATOMIC_ACQUIRE);
  if (known == 0) {
    std::lock_guard<std::mutex> lk(g_arch_mu);
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return KDA_ERR_CUDA;
    known = (major == 10 && minor == 0) ? 1 : -1;
    __atomic_store_n(&g_arch_ok[dev], known, __ATOMIC_RELEASE);
  }
  return known == 1 ? KDA_OK : KDA_ERR_ARCH;
}

// 4 consecutive innermost elements at any row start are 4-element aligned.
bool vec4_ok(const void* ptr, const int64_t* stride, int ndim_outer, int dt) {
  const uintptr_t align = (uintptr_t)(4 * elt_size(dt));
  if ((reinterpret_cast<uintptr_t>(ptr) % align) != 0) return false;
  for (int d = 0; d < ndim_outer; ++d)
    if (stride[d] % 4 != 0) return false;
  return true;
}

// 8 consecutive 16-bit innermost elements at any row start are 16-byte aligned.
bool vec8_ok(const void* ptr, const int64_t* stride) {
  if ((reinterpret_cast<uintptr_t>(ptr) % 16) != 0) return false;
  for (int d = 0; d < 3; ++d)
    if (stride[d] % 8 != 0) return false;
  return true;
}

// 2 consecutive innermost elements at any row start are 2-element aligned.
bool vec2_ok(const void* ptr, const int64_t* stride, int esize) {
  if ((reinterpret_cast<uintptr_t>(ptr) % (uintptr_t)(2 * esize)) != 0) return false;
  for (int d = 0; d < 3; ++d)
    if (stride[d] % 2 != 0) return false;
  return true;
}

int validate(const KdaArgs* a, bool chunkwise) {
  if (a == nullptr) return KDA_ERR_NULL_POINTER;
  if (a->abi_version != KDA_B200_ABI_VERSION) return KDA_ERR_SHAPE;
  if (a->B < 0 || a->T < 0 || a->H < 0 || a->K < 1 || a->V < 1) return KDA_ERR_SHAPE;
  if (a->K > kRecMaxK || a->K > kSimtMaxK) return KDA_ERR_SHAPE;
  if (a->B > 65535 || a->H > 65535) return KDA_ERR_SHAPE;
  if (!dtype_ok(a->io_dtype) || !dtype_ok(a->state_out_dtype)) return KDA_ERR_DTYPE;
  if (a->state_in != nullptr && !dtype_ok(a->state_in_dtype)) return KDA_ERR_DTYPE;
  if (chunkwise) {
    if (a->chunk_size < 1) return KDA_ERR_CHUNK;
    if (a->T % a->chunk_size != 0) return KDA_ERR_CHUNK;
  }
  if (a->B == 0 || a->H == 0) return KDA_OK;   // nothing to compute
  if (a->state_out == nullptr) return KDA_ERR_NULL_POINTER;
  if (a->T > 0 &&
      (a->q == nullptr || a->k == nullptr || a->v == nullptr || a->g == nullptr ||
       a->beta == nullptr || a->o == nullptr))
    return KDA_ERR_NULL_POINTER;
  if (a->q_stride[3] != 1 || a->k_stride[3] != 1 || a->v_stride[3] != 1 ||
      a->g_stride[3] != 1 || a->o_stride[3] != 1 || a->state_out_stride[3] != 1)
    return KDA_ERR_STRIDE;
  if (a->state_in != nullptr && a->state_in_stride[3] != 1) return KDA_ERR_STRIDE;
  // natural alignment of every element pointer
  const uintptr_t e = (uintptr_t)elt_size(a->io_dtype);
  if ((reinterpret_cast<uintptr_t>(a->q) % e) || (reinterpret_cast<uintptr_t>(a->k) % e) ||
      (reinterpret_cast<uintptr_t>(a->v) % e) || (reinterpret_cast<uintptr_t>(a->o) % e) ||
      (reinterpret_cast<uintptr_t>(a->g) % 4) || (reinterpret_cast<uintptr_t>(a->beta) % 4))
    return KDA_ERR_ALIGNMENT;
  if (reinterpret_cast<uintptr_t>(a->state_out) % (uintptr_t)elt_size(a->state_out_dtype))
    return KDA_ERR_ALIGNMENT;
  if (a->state_in != nullptr &&
      reinterpret_cast<uintptr_t>(a->state_in) % (uintptr_t)elt_size(a->state_in_dtype))
    return KDA_ERR_ALIGNMENT;
  // an output state that aliases the input (in-place update) must be exactly
  // the same view: every kernel reads the state tile it owns before writing it
  if (a->state_in != nullptr && a->state_in == a->state_out) {
    if (a->state_in_dtype != a->state_out_dtype) return KDA_ERR_DTYPE;
    for (int d = 0; d < 4; ++d)
      if (a->state_in_stride[d] != a->state_out_stride[d]) return KDA_ERR_STRIDE;
  }
  return KDA_OK;
}

RecParams to_params(const KdaArgs* a) {
  RecParams p;
  std::memset(&p, 0, sizeof(p));
  p.B = a->B; p.T = a->T; p.H = a->H; p.K = a->K; p.V = a->V;
  p.io_dtype = a->io_dtype;
  p.state_in_dtype = a->state_in != nullptr ? a->state_in_dtype : KDA_DTYPE_F32;
  p.state_out_dtype = a->state_out_dtype;
  p.scale = a->scale;
  p.q = a->q; p.k = a->k; p.v = a->v; p.g = a->g; p.beta = a->beta;
  p.state_in = a->state_in; p.o = a->o; p.state_out = a->state_out;
  for (int d = 0; d < 4; ++d) {
    p.q_s[d] = a->q_stride[d]; p.k_s[d] = a->k_stride[d]; p.v_s[d] = a->v_stride[d];
    p.g_s[d] = a->g_stride[d]; p.o_s[d] = a->o_stride[d];
    p.si_s[d] = a->state_in_stride[d]; p.so_s[d] = a->state_out_stride[d];
  }
  for (int d = 0; d < 3; ++d) p.b_s[d] = a->beta_stride[d];
  p.state_vec = a->state_in != nullptr && vec4_ok(a->state_in, a->state_in_stride, 3,
                                                  a->state_in_dtype);
  p.state_out_vec = vec4_ok(a->state_out, a->state_out_stride, 3, a->state_out_dtype);
  p.o_vec = vec4_ok(a->o, a->o_stride, 3, a->io_dtype);
  p.v_vec16 = a->io_dtype != KDA_DTYPE_F32 && vec8_ok(a->v, a->v_stride);
  p.o_vec16 = a->io_dtype != KDA_DTYPE_F32 && vec8_ok(a->o, a->o_stride);
  p.force_simt = (a->flags & KDA_FLAG_FORCE_SIMT) != 0;
  p.g_vec2 = vec2_ok(a->g, a->g_stride, 4);
  p.qk_vec2 = vec2_ok(a->q, a->q_stride, elt_size(a->io_dtype)) &&
              vec2_ok(a->k, a->k_stride, elt_size(a->io_dtype));
  p.v_vec2 = vec2_ok(a->v, a->v_stride, elt_size(a->io_dtype));
  return p;
}

int launch_status(cudaError_t e) {
  if (e == cudaSuccess) return KDA_OK;
  return (e == cudaErrorInvalidConfiguration || e == cudaErrorLaunchFailure ||
          e == cudaErrorInvalidValue || e == cudaErrorLaunchOutOfResources)
             ? KDA_ERR_LAUNCH
             : KDA_ERR_CUDA;
}

int validate_prologue(const KdaPrologueArgs* a) {
  if (a == nullptr) return KDA_ERR_NULL_POINTER;
  if (a->abi_version != KDA_B200_ABI_VERSION) return KDA_ERR_SHAPE;
  if (a->B < 0 || a->T < 0 || a->H < 0) return KDA_ERR_SHAPE;
  if (a->K != a->V || (a->K != 32 && a->K != 64 && a->K != 128)) return KDA_ERR_SHAPE;
  if (a->conv_size < 1 || a->conv_size > 4) return KDA_ERR_SHAPE;
  if (!dtype_ok(a->io_dtype) || !dtype_ok(a->gate_dtype)) return KDA_ERR_DTYPE;
  if (!(a->l2norm_eps > 0.f)) return KDA_ERR_SHAPE;
  if (!a->q_in || !a->k_in || !a->v_in || !a->gk || !a->beta_logit || !a->A_log ||
      !a->dt_bias || !a->q || !a->k || !a->v || !a->g || !a->beta)
    return KDA_ERR_NULL_POINTER;
  for (int i = 0; i < 3; ++i)
    if (!a->conv_w[i]) return KDA_ERR_NULL_POINTER;
  if (a->q_stride[3] != 1 || a->k_stride[3] != 1 || a->v_stride[3] != 1 || a->g_stride[3] != 1 ||
      a->beta_stride[2] != 1)
    return KDA_ERR_STRIDE;
  return KDA_OK;
}

PrologueParams to_prologue(const KdaPrologueArgs* a) {
  PrologueParams p{};
  p.B = a->B; p.T = a->T; p.H = a->H; p.K = a->K; p.V = a->V;
  p.conv_size = a->conv_size;
  p.io_dtype = a->io_dtype; p.gate_dtype = a->gate_dtype;
  p.eps = a->l2norm_eps;
  p.q_in = a->q_in; p.k_in = a->k_in; p.v_in = a->v_in;
  for (int d = 0; d < 2; ++d) {
    p.in_s[0][d] = a->q_in_stride[d];
    p.in_s[1][d] = a->k_in_stride[d];
    p.in_s[2][d] = a->v_in_stride[d];
    p.gk_s[d] = a->gk_stride[d];
    p.bl_s[d] = a->beta_logit_stride[d];
  }
  p.w_q = a->conv_w[0]; p.w_k = a->conv_w[1]; p.w_v = a->conv_w[2];
  p.b_q = a->conv_b[0]; p.b_k = a->conv_b[1]; p.b_v = a->conv_b[2];
  p.hist_q = a->hist[0]; p.hist_k = a->hist[1]; p.hist_v = a->hist[2];
  for (int i = 0; i < 3; ++i) p.hist_bs[i] = a->hist_batch_stride[i];
  p.new_q = a->new_hist[0]; p.new_k = a->new_hist[1]; p.new_v = a->new_hist[2];
  p.gk = a->gk; p.beta_logit = a->beta_logit;
  p.A_log = a->A_log; p.dt_bias = a->dt_bias;
  p.q = a->q; p.k = a->k; p.v = a->v;
  std::memcpy(p.out_s[0], a->q_stride, sizeof(p.out_s[0]));
  std::memcpy(p.out_s[1], a->k_stride, sizeof(p.out_s[1]));
  std::memcpy(p.out_s[2], a->v_stride, sizeof(p.out_s[2]));
  p.g = a->g; std::memcpy(p.g_s, a->g_stride, sizeof(p.g_s));
  p.beta = a->beta; std::memcpy(p.beta_s, a->beta_stride, sizeof(p.beta_s));
  return p;
}

int validate_epilogue(const KdaEpilogueArgs* a) {
  if (a == nullptr) return KDA_ERR_NULL_POINTER;
  if (a->abi_version != KDA_B200_ABI_VERSION) return KDA_ERR_SHAPE;
  if (a->B < 0 || a->T < 0 || a->H < 0) return KDA_ERR_SHAPE;
  if (a->V < 32 || a->V > 128 || a->V % 32 != 0) return KDA_ERR_SHAPE;
  if (!dtype_ok(a->io_dtype)) return KDA_ERR_DTYPE;
  if (!(a->eps >= 0.f)) return KDA_ERR_SHAPE;
  if (!a->o || !a->og || !a->weight || !a->y) return KDA_ERR_NULL_POINTER;
  if (a->o_stride[3] != 1) return KDA_ERR_STRIDE;
  return KDA_OK;
}

EpilogueParams to_epilogue(const KdaEpilogueArgs* a) {
  EpilogueParams p{};
  p.B = a->B; p.T = a->T; p.H = a->H; p.V = a->V; p.io_dtype = a->io_dtype; p.eps = a->eps;
  p.o = a->o; std::memcpy(p.o_s, a->o_stride, sizeof(p.o_s));
  p.og = a->og; std::memcpy(p.og_s, a->og_stride, sizeof(p.og_s));
  p.weight = a->weight;
  p.y = a->y; std::memcpy(p.y_s, a->y_stride, sizeof(p.y_s));
  return p;
}

int validate_backward(const KdaBackwardArgs* a) {
  if (a == nullptr) return KDA_ERR_NULL_POINTER;
  if (a->abi_version != KDA_B200_ABI_VERSION) return KDA_ERR_SHAPE;
  if (a->B < 0 || a->T < 0 || a->H < 0) return KDA_ERR_SHAPE;
  if (a->K != 32 && a->K != 64 && a->K != 128) return KDA_ERR_SHAPE;
  if (a->V < 16 || a->V % 16 != 0) return KDA_ERR_SHAPE;
  if (a->B > 65535 || a->H > 65535) return KDA_ERR_SHAPE;
  if (!dtype_ok(a->io_dtype)) return KDA_ERR_DTYPE;
  if (a->state_in != nullptr && !dtype_ok(a->state_in_dtype)) return KDA_ERR_DTYPE;
  if (a->B == 0 || a->H == 0 || a->T == 0) return KDA_OK;
  if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->dout || !a->dv || !a->ckpt)
    return KDA_ERR_NULL_POINTER;
  // the partial sums are needed unless the chunkwise path (dq set, V <= 128)
  // writes the final gradients itself
  const bool chunkwise = a->dq != nullptr && a->V <= 128;
  if (!chunkwise && (!a->dq_part || !a->dk_part || !a->dg_part || !a->dbeta_part))
    return KDA_ERR_NULL_POINTER;
  if (a->q_stride[3] != 1 || a->k_stride[3] != 1 || a->v_stride[3] != 1 || a->g_stride[3] != 1 ||
      a->dout_stride[3] != 1 || a->dv_stride[3] != 1)
    return KDA_ERR_STRIDE;
  if (a->state_in != nullptr && a->state_in_stride[3] != 1) return KDA_ERR_STRIDE;
  if (a->dstate_out != nullptr && a->dstate_out_stride[3] != 1) return KDA_ERR_STRIDE;
  if (a->dstate_in != nullptr && a->dstate_in_stride[3] != 1) return KDA_ERR_STRIDE;
  if (a->ckpt_floats < backward_ckpt_floats(a->B, a->H, a->T, a->K, a->V)) return KDA_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(a->ckpt) % 16) return KDA_ERR_ALIGNMENT;
  if (a->dq != nullptr) {
    if (!a->dk || !a->dg || !a->dbeta) return KDA_ERR_NULL_POINTER;
    if (a->dq_stride[3] != 1 || a->dk_stride[3] != 1 || a->dg_stride[3] != 1)
      return KDA_ERR_STRIDE;
  }
  return KDA_OK;
}

BwdParams to_backward(const KdaBackwardArgs* a) {
  BwdParams p{};
  p.B = a->B; p.T = a->T; p.H = a->H; p.K = a->K; p.V = a->V;
  p.io_dtype = a->io_dtype;
  p.state_in_dtype = a->state_in ? a->state_in_dtype : KDA_DTYPE_F32;
  p.scale = a->scale;
  p.q = a->q; std::memcpy(p.q_s, a->q_stride, sizeof(p.q_s));
  p.k = a->k; std::memcpy(p.k_s, a->k_stride, sizeof(p.k_s));
  p.v = a->v; std::memcpy(p.v_s, a->v_stride, sizeof(p.v_s));
  p.g = a->g; std::memcpy(p.g_s, a->g_stride, sizeof(p.g_s));
  p.beta = a->beta; std::memcpy(p.b_s, a->beta_stride, sizeof(p.b_s));
  p.state_in = a->state_in; std::memcpy(p.si_s, a->state_in_stride, sizeof(p.si_s));
  p.dout = a->dout; std::memcpy(p.do_s, a->dout_stride, sizeof(p.do_s));
  p.dstate_out = a->dstate_out; std::memcpy(p.dso_s, a->dstate_out_stride, sizeof(p.dso_s));
  p.dq_part = a->dq_part; p.dk_part = a->dk_part; p.dg_part = a->dg_part;
  p.dbeta_part = a->dbeta_part;
  p.dv = a->dv; std::memcpy(p.dv_s, a->dv_stride, sizeof(p.dv_s));
  p.dstate_in = a->dstate_in; std::memcpy(p.dsi_s, a->dstate_in_stride, sizeof(p.dsi_s));
  p.ckpt = a->ckpt;
  p.dq = a->dq; std::memcpy(p.dq_s, a->dq_stride, sizeof(p.dq_s));
  p.dk = a->dk; std::memcpy(p.dk_s, a->dk_stride, sizeof(p.dk_s));
  p.dg = a->dg; std::memcpy(p.dg_s, a->dg_stride, sizeof(p.dg_s));
  p.dbeta = a->dbeta; std::memcpy(p.dbeta_s, a->dbeta_stride, sizeof(p.dbeta_s));
  return p;
}

}  // namespace
}  // namespace kda

using namespace kda;

extern "C" {

int kda_recurrent_fwd(const KdaArgs* args, void* stream) {
  int st = validate(args, /*chunkwise=*/false);
  if (st != KDA_OK) return st;
  if (args->B == 0 || args->H == 0) return KDA_OK;
  st = check_arch();
  if (st != KDA_OK) return st;
  const RecParams p = to_params(args);
  return launch_status(launch_recurrent(p, static_cast<cudaStream_t>(stream)));
}

int kda_chunkwise_path(const KdaArgs* args) {
  int st = validate(args, /*chunkwise=*/true);
  if (st != KDA_OK) return -st;
  const RecParams p = to_params(args);
  return chunk_tc_supported(p) ? 1 : 0;
}

size_t kda_chunkwise_workspace_bytes(const KdaArgs* args) {
  if (validate(args, /*chunkwise=*/true) != KDA_OK) return 0;
  const RecParams p = to_params(args);
  return chunk_tc_supported(p) ? chunk_tc_workspace_bytes(p) : 0;
}

int kda_chunkwise_fwd(const KdaArgs* args, void* stream) {
  int st = validate(args, /*chunkwise=*/true);
  if (st != KDA_OK) return st;
  if (args->B == 0 || args->H == 0) return KDA_OK;
  st = check_arch();
  if (st != KDA_OK) return st;
  const RecParams p = to_params(args);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (chunk_tc_supported(p)) {
    const size_t need = chunk_tc_workspace_bytes(p);
    if (need > 0 && (args->workspace == nullptr || args->workspace_bytes < need))
      return KDA_ERR_WORKSPACE;
    if (need > 0 && (reinterpret_cast<uintptr_t>(args->workspace) % 256) != 0)
      return KDA_ERR_ALIGNMENT;
    return launch_status(launch_chunk_tc(p, args->workspace, s));
  }
  return launch_status(launch_chunk_simt(p, s));
}

const char* kda_status_string(int status) {
  switch (status) {
    case KDA_OK: return "ok";
    case KDA_ERR_NULL_POINTER: return "a required pointer is NULL";
    case KDA_ERR_SHAPE: return "unsupported shape (need K <= 256, B and H <= 65535) or ABI mismatch";
    case KDA_ERR_DTYPE: return "unsupported dtype (f32, f16 or bf16)";
    case KDA_ERR_STRIDE: return "innermost stride must be 1";
    case KDA_ERR_ALIGNMENT: return "pointer is not aligned to its element size";
    case KDA_ERR_ARCH: return "device is not an sm_100 (B200) GPU";
    case KDA_ERR_LAUNCH: return "kernel launch failed";
    case KDA_ERR_CHUNK: return "T is not a multiple of chunk_size";
    case KDA_ERR_WORKSPACE: return "workspace missing or too small";
    case KDA_ERR_CUDA: return "CUDA runtime error";
    default: return "unknown status";
  }
}

int kda_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return -1;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess)
    return -1;
  return (major == 10 && minor == 0) ? 1 : 0;
}

int kda_device_error(int clear) {
  const int a = read_device_error(clear != 0);
  const int b = kda::mla::read_device_error(clear != 0);
  if (a < 0 || b < 0) return -1;
  return a ? a : b;
}

int kda_prologue_fwd(const KdaPrologueArgs* args, void* stream) {
  int st = validate_prologue(args);
  if (st != KDA_OK) return st;
  if (args->B == 0 || args->T == 0 || args->H == 0) return KDA_OK;
  st = check_arch();
  if (st != KDA_OK) return st;
  return launch_status(launch_prologue(to_prologue(args), static_cast<cudaStream_t>(stream)));
}

int kda_epilogue_fwd(const KdaEpilogueArgs* args, void* stream) {
  int st = validate_epilogue(args);
  if (st != KDA_OK) return st;
  if (args->B == 0 || args->T == 0 || args->H == 0) return KDA_OK;
  st = check_arch();
  if (st != KDA_OK) return st;
  return launch_status(launch_epilogue(to_epilogue(args), static_cast<cudaStream_t>(stream)));
}

int kda_backward(const KdaBackwardArgs* args, void* stream) {
  int st = validate_backward(args);
  if (st != KDA_OK) return st;
  if (args->B == 0 || args->H == 0 || args->T == 0) return KDA_OK;
  st = check_arch();
  if (st != KDA_OK) return st;
  const BwdParams p = to_backward(args);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (backward_chunk_supported(p)) {
    e = launch_backward_chunk(p, s);
  } else {
    e = launch_backward(p, s);
    if (e == cudaSuccess && p.dq != nullptr) e = launch_backward_reduce(p, s);
  }
  return launch_status(e);
}

size_t kda_backward_ckpt_floats(int B, int H, int T, int K, int V) {
  if (B < 0 || H < 0 || T < 0 || K < 0 || V < 0) return 0;
  return backward_ckpt_floats(B, H, T, K, V);
}

size_t kda_backward_args_size(void) { return sizeof(KdaBackwardArgs); }

size_t kda_prologue_args_size(void) { return sizeof(KdaPrologueArgs); }

size_t kda_epilogue_args_size(void) { return sizeof(KdaEpilogueArgs); }

size_t kda_args_size(void) { return sizeof(KdaArgs); }

int kda_abi_version(void) { return KDA_B200_ABI_VERSION; }

}  // extern "C"
