/*
 * kda_b200.h -- C ABI of the B200 (sm_100a) Kimi Delta Attention core.
 *
 * Drop-in boundary for the two kernels of Lazy-Hakimi/-kimi-linear-:
 *
 *   kda_chunkwise_fwd  replaces kimi_linear/kda.py:58-185 (kda_chunkwise)
 *   kda_recurrent_fwd  replaces kimi_linear/kda.py:188-219 (kda_recurrent)
 *
 * and, around it, the fused prologue / epilogue of the KDA block
 * (kda_prologue_fwd, kda_epilogue_fwd), the gradient of the core
 * (kda_backward) and the static-buffer MLA decode step of the full-attention
 * layers (mla_decode_fwd, kimi_linear/mla.py:117-181).
 *
 * Plain pointers, sizes and element strides only.  The Python host layer
 * (-kimi-linear-_b200/ops.py) keeps the reference's Python signatures and
 * calls these entry points through ctypes; any other FFI can bind them the
 * same way.
 *
 * Tensor conventions (identical to the reference):
 *   q, k, g : [B, T, H, K]     v, o : [B, T, H, V]     beta : [B, T, H]
 *   state   : [B, H, K, V]
 * Strides are in ELEMENTS; the innermost (last) stride of every tensor must
 * be 1.  g and beta are fp32 (the reference promotes them with .float(),
 * kda.py:119-120,202-203).  q is multiplied by `scale` inside the kernel (the
 * reference uses K^-0.5, kda.py:132,199).  Inputs are never written.
 *
 * state_out may be exactly state_in (same pointer, dtype and strides) for an
 * in-place state update: every kernel reads the state tile it owns before
 * writing it.  Any other overlap between outputs and inputs is not allowed.
 *
 * Every call is asynchronous on `stream` (a cudaStream_t, NULL = legacy
 * default stream), performs no host<->device synchronisation, no allocation
 * and no host read of device data, so it can be captured in a CUDA graph.
 */
#ifndef KDA_B200_H
#define KDA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KDA_B200_ABI_VERSION 2

/* Element types. */
typedef enum {
  KDA_DTYPE_F32 = 0,
  KDA_DTYPE_F16 = 1,
  KDA_DTYPE_BF16 = 2
} kda_dtype_t;

/* Status codes: 0 = success; the Python layer maps the rest to exceptions. */
typedef enum {
  KDA_OK = 0,
  KDA_ERR_NULL_POINTER = 1, /* a required pointer is NULL                    */
  KDA_ERR_SHAPE = 2,        /* a size is out of the supported range          */
  KDA_ERR_DTYPE = 3,        /* unsupported dtype combination                 */
  KDA_ERR_STRIDE = 4,       /* innermost stride != 1                          */
  KDA_ERR_ALIGNMENT = 5,    /* pointer / stride alignment not met             */
  KDA_ERR_ARCH = 6,         /* device is not sm_100 (B200 family)             */
  KDA_ERR_LAUNCH = 7,       /* kernel launch failed (cudaGetLastError)        */
  KDA_ERR_CHUNK = 8,        /* T is not a multiple of chunk_size (kda.py:124) */
  KDA_ERR_WORKSPACE = 9,    /* workspace missing or too small                 */
  KDA_ERR_CUDA = 10         /* another CUDA runtime error                     */
} kda_status_t;

/* KdaArgs.flags bits. */
#define KDA_FLAG_FORCE_SIMT 1  /* chunkwise: use the CUDA-core kernel even where the
                                  tensor-core kernel applies (cross-checking) */

/* Arguments shared by both entry points. */
typedef struct KdaArgs {
  int32_t abi_version;      /* must be KDA_B200_ABI_VERSION */
  int32_t B, T, H, K, V;
  int32_t chunk_size;       /* reference chunk_size; chunkwise only */
  int32_t io_dtype;         /* dtype of q, k, v and o (kda_dtype_t) */
  int32_t state_in_dtype;   /* dtype of state_in (ignored when NULL) */
  int32_t state_out_dtype;  /* dtype of state_out */
  float scale;              /* multiplier applied to q (K^-0.5 in the reference) */
  int32_t flags;            /* KDA_FLAG_* bits, 0 by default */
  const void* q;     int64_t q_stride[4];
  const void* k;     int64_t k_stride[4];
  const void* v;     int64_t v_stride[4];
  const float* g;    int64_t g_stride[4];
  const float* beta; int64_t beta_stride[3];
  const void* state_in;  int64_t state_in_stride[4];  /* NULL = zero state */
  void* o;           int64_t o_stride[4];
  void* state_out;   int64_t state_out_stride[4];
  void* workspace;          /* device scratch, >= kda_chunkwise_workspace_bytes() */
  size_t workspace_bytes;
} KdaArgs;

/*
 * Chunkwise KDA forward (paper Eq. 6-9).
 * Reference: kimi_linear/kda.py:58-185, kda_chunkwise(q, k, v, g, beta,
 * initial_state, chunk_size, tile_size, state_dtype) -> (o, S).
 * state_in  = initial_state (kda.py:134-137); state_out = returned S
 * (kda.py:185).  Returns KDA_ERR_CHUNK when T % chunk_size != 0, where the
 * reference's reshape fails (kda.py:124).
 */
int kda_chunkwise_fwd(const KdaArgs* args, void* stream);

/*
 * Recurrent KDA forward (paper Eq. 1), any T >= 1.
 * Reference: kimi_linear/kda.py:188-219, kda_recurrent(q, k, v, g, beta,
 * state, state_dtype) -> (o, S).  fp16 outputs are clamped to +-60000
 * (kda.py:217-218, FP16_MAX_SAFE of kimi_linear/fp16.py:97).
 */
int kda_recurrent_fwd(const KdaArgs* args, void* stream);

/*
 * kda_chunkwise_fwd without any device allocation by anyone: the tensor-core
 * path's scratch is a fixed 32 MiB array inside this library instead of a
 * caller-allocated workspace (args->workspace is ignored).  For callers that
 * cannot call cudaMalloc on their hot path -- a host that reserves all device
 * memory up front, an engine plugin whose enqueue may not allocate, or a plain
 * C caller without a device allocator.  The caller still provides o and
 * state_out.  Returns KDA_ERR_WORKSPACE when kda_chunkwise_workspace_bytes()
 * exceeds 32 MiB (B * H * ceil(T / 64) > 407 on the tensor-core path).  The
 * first call on a device looks up the array's address (cudaGetSymbolAddress),
 * so make it before any CUDA-graph capture; the address is cached per device
 * for the primary context (the runtime's and PyTorch's).  Every GPU that
 * loads the library holds the array until exit.  All calls share the array: calls whose kernels
 * overlap on the GPU race.  No counterpart in the reference.
 */
int kda_chunkwise_fwd_noalloc(const KdaArgs* args, void* stream);

/*
 * Device scratch bytes kda_chunkwise_fwd needs for `args` (0 = none).
 * No reference counterpart: the reference allocates its transients inside
 * torch (kda.py:131-138,148-149).
 */
size_t kda_chunkwise_workspace_bytes(const KdaArgs* args);

/*
 * Which implementation kda_chunkwise_fwd selects for `args`:
 * 0 = CUDA-core (SIMT) kernel, 1 = tcgen05 tensor-core kernel, <0 = status
 * error.  No reference counterpart (diagnostic).
 */
int kda_chunkwise_path(const KdaArgs* args);

/* Human-readable text for a status code.  No reference counterpart. */
const char* kda_status_string(int status);

/* 1 when `device` is an sm_100 GPU these kernels run on, 0 otherwise,
 * <0 on a CUDA error.  No reference counterpart. */
int kda_device_supported(int device);

/*
 * Error word written by a kernel that abandoned its work after a bounded wait
 * on the GPU ran out, or (MLA decode) found pos outside the buffer (0 = none);
 * clear != 0 resets it.  Synchronises with the device.  <0 on a CUDA error.
 * No reference counterpart (diagnostic).
 */
int kda_device_error(int clear);

/*
 * Prologue of the KDA block after its projection GEMMs: causal depthwise
 * ShortConv (conv_size <= 4, optional bias, optional conv history) and SiLU of
 * q_in / k_in / v_in, per-head L2 normalisation of q and k (fp32 reduction,
 * rsqrt clamped at 1 / l2norm_eps), the log decay
 * g = -exp(A_log) * softplus(gk + dt_bias) and beta = sigmoid(beta_logit).
 * Reference: the elementwise part of KimiDeltaAttention._projections,
 * kimi_linear/kda.py:399-461 (ShortConv kda.py:282-310, l2norm kda.py:313-325),
 * for both its batch path and its single-token decode path (conv history =
 * the module's conv cache).  One pass over HBM instead of the reference's
 * separate elementwise passes.
 *
 * Layouts (strides in elements, innermost stride 1):
 *   q_in, k_in : [B, T, H*K]   v_in : [B, T, H*V]   gk : [B, T, H*K]
 *   beta_logit : [B, T, H]     (stride pairs are (batch, time))
 *   conv_w[i]  : [D, conv_size] fp32 contiguous (nn.Conv1d weight [D, 1, cs])
 *   conv_b[i]  : [D] fp32 or NULL;  A_log, dt_bias : [H, K] fp32 contiguous
 *   hist[i]    : conv history [B, conv_size-1, D] (time stride D, batch
 *                stride hist_batch_stride[i]) or NULL for zeros
 *   new_hist[i]: [B, conv_size-1, D] contiguous output, or NULL
 *   q, k : [B, T, H, K]  v : [B, T, H, V]  (io_dtype);  g : [B, T, H, K] fp32;
 *   beta : [B, T, H] fp32.   Index i: 0 = q, 1 = k, 2 = v.
 * Requires K == V in {32, 64, 128}.
 */
typedef struct KdaPrologueArgs {
  int32_t abi_version;
  int32_t B, T, H, K, V;
  int32_t conv_size;                 /* 1..4 */
  int32_t io_dtype;                  /* q_in/k_in/v_in, histories, q/k/v */
  int32_t gate_dtype;                /* gk and beta_logit */
  float l2norm_eps;
  const void* q_in; int64_t q_in_stride[2];
  const void* k_in; int64_t k_in_stride[2];
  const void* v_in; int64_t v_in_stride[2];
  const float* conv_w[3];
  const float* conv_b[3];
  const void* hist[3];
  int64_t hist_batch_stride[3];
  void* new_hist[3];
  const void* gk; int64_t gk_stride[2];
  const void* beta_logit; int64_t beta_logit_stride[2];
  const float* A_log;
  const float* dt_bias;
  void* q; int64_t q_stride[4];
  void* k; int64_t k_stride[4];
  void* v; int64_t v_stride[4];
  float* g; int64_t g_stride[4];
  float* beta; int64_t beta_stride[3];
} KdaPrologueArgs;

int kda_prologue_fwd(const KdaPrologueArgs* args, void* stream);

/*
 * Epilogue of the KDA block before o_proj: head-wise RMSNorm of o (fp32,
 * per-head weight [H, V]) rounded to io_dtype, times sigmoid(og) in fp32,
 * rounded to io_dtype.  Reference: KimiDeltaAttention._output without its
 * o_proj GEMM, kimi_linear/kda.py:464-470, and HeadwiseRMSNorm
 * kimi_linear/kda.py:258-279.
 *   o : [B, T, H, V] (strides in elements)   og, y : [B, T, H*V] (batch, time)
 * Requires V in {32, 64, 96, 128}.
 */
typedef struct KdaEpilogueArgs {
  int32_t abi_version;
  int32_t B, T, H, V;
  int32_t io_dtype;
  float eps;
  const void* o; int64_t o_stride[4];
  const void* og; int64_t og_stride[2];
  const float* weight;               /* [H, V] fp32 contiguous */
  void* y; int64_t y_stride[2];
} KdaEpilogueArgs;

int kda_epilogue_fwd(const KdaEpilogueArgs* args, void* stream);

/*
 * Gradient of the KDA forward (kda_chunkwise or kda_recurrent: the same
 * function) with respect to q, k, v, g, beta and the initial state, given the
 * gradients of o and of the returned state.  The reference obtains it from
 * torch autograd through kimi_linear/kda.py:58-219; this is the exact
 * reverse-mode gradient of the token recurrence (kda.py:207-216).
 *
 *   dout       : [B, T, H, V] in io_dtype (gradient of o)
 *   dstate_out : [B, H, K, V] fp32 (gradient of the returned state) or NULL
 *   dv         : [B, T, H, V] fp32 output
 *   dstate_in  : [B, H, K, V] fp32 output, or NULL
 *   dq_part, dk_part, dg_part : [V/16, B, T, H, K] fp32 partial sums over
 *                16-column tiles of V (dq, dk, dg = their sums over axis 0)
 *   dbeta_part : [V/16, B, T, H] fp32 partial sums
 *   ckpt       : workspace of kda_backward_ckpt_floats() fp32 values
 *   dq, dk     : [B, T, H, K] in io_dtype, or NULL; when dq is set, the call
 *                also writes dq, dk, dg ([B, T, H, K] fp32) and dbeta
 *                ([B, T, H] fp32) on the same stream
 * With dq set and V <= 128 the call runs the chunkwise backward (64-token
 * chunks in parallel, the chunk-boundary states and their gradients by two
 * chains), writes the final gradients directly and ignores the partial-sum
 * pointers, which may be NULL.  Otherwise it runs the token-serial reverse
 * sweep into the partials (and sums them when dq is set).
 * Requires K in {32, 64, 128} and V % 16 == 0.
 */
typedef struct KdaBackwardArgs {
  int32_t abi_version;
  int32_t B, T, H, K, V;
  int32_t io_dtype;
  int32_t state_in_dtype;
  float scale;
  const void* q;     int64_t q_stride[4];
  const void* k;     int64_t k_stride[4];
  const void* v;     int64_t v_stride[4];
  const float* g;    int64_t g_stride[4];
  const float* beta; int64_t beta_stride[3];
  const void* state_in;  int64_t state_in_stride[4];   /* NULL = zero state */
  const void* dout;      int64_t dout_stride[4];
  const float* dstate_out; int64_t dstate_out_stride[4];
  float* dq_part;
  float* dk_part;
  float* dg_part;
  float* dbeta_part;
  float* dv;         int64_t dv_stride[4];
  float* dstate_in;  int64_t dstate_in_stride[4];
  float* ckpt;
  size_t ckpt_floats;
  void* dq;          int64_t dq_stride[4];      /* NULL: partial sums only */
  void* dk;          int64_t dk_stride[4];
  float* dg;         int64_t dg_stride[4];
  float* dbeta;      int64_t dbeta_stride[3];
} KdaBackwardArgs;

int kda_backward(const KdaBackwardArgs* args, void* stream);

/* fp32 values of the backward workspace: for V <= 128 the chunkwise records,
 * B * H * ceil(T/64) * (4*64*64 + 5*64*K + K + 2*K*V); for wider V the
 * token-serial checkpoints, B * H * ceil(T/64) * K * V. */
size_t kda_backward_ckpt_floats(int B, int H, int T, int K, int V);

/* sizeof(KdaBackwardArgs) as compiled. */
size_t kda_backward_args_size(void);

/* sizeof(KdaPrologueArgs) / sizeof(KdaEpilogueArgs) as compiled. */
size_t kda_prologue_args_size(void);
size_t kda_epilogue_args_size(void);

/*
 * Single-token MLA decode over a static latent buffer: the attention core of
 * MLA._decode_step_static (kimi_linear/mla.py:117-181) for NoPE layers
 * (qk_rope_head_dim == 0), everything between the projections and o_proj:
 *   kv_buf[b, pos] = c_kv[b]; q_lat = q_nope W_nope (fp32);
 *   p = softmax(scale q_lat kv_buf[b, :pos+1]^T) (fp32, positions > pos masked);
 *   mixed = p kv_buf (kv_buf's dtype); out = mixed W_v^T (fp32 -> io dtype);
 *   pos += 1.
 * pos is read and advanced in device memory (capturable in a CUDA graph).
 *   q_nope : [B, H, DN]      c_kv : [B, KVL]        (io dtype, any strides)
 *   kv_buf : [B, L, KVL]     io dtype, unit channel stride, 16-byte rows
 *   pos    : int64[1] device memory
 *   w      : kv_b_proj.weight [H*(DN+DV), KVL]       (io dtype)
 *   out    : [B, H, DV]      io dtype
 * Requires io dtype f16 or bf16, H <= 16, KVL in {64, 128, 256, 512}.
 */
typedef struct MlaDecodeArgs {
  int32_t abi_version;
  int32_t B, L, H, KVL, DN, DV;
  int32_t io_dtype;
  float scale;                 /* (DN + qk_rope_head_dim)^-0.5 in the reference */
  const void* q_nope; int64_t q_nope_stride[3];
  const void* c_kv;   int64_t c_kv_stride[2];
  void* kv_buf;       int64_t kv_buf_stride[3];
  int64_t* pos;
  const void* w;      int64_t w_stride[2];
  void* out;          int64_t out_stride[3];
  void* workspace;    size_t workspace_bytes;   /* mla_decode_workspace_bytes(), 256-byte aligned */
} MlaDecodeArgs;

int mla_decode_fwd(const MlaDecodeArgs* args, void* stream);

/* device workspace of mla_decode_fwd for these B, L, KVL (0 for invalid sizes). */
size_t mla_decode_workspace_bytes(const MlaDecodeArgs* args);

/* sizeof(MlaDecodeArgs) as compiled. */
size_t mla_decode_args_size(void);

/* sizeof(KdaArgs) as compiled, for FFI layout checks. */
size_t kda_args_size(void);

/* KDA_B200_ABI_VERSION as compiled. */
int kda_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KDA_B200_H */
