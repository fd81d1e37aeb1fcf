// kda_io.cu -- fused prologue and epilogue of the KDA block for sm_100a.
//
// Prologue (replaces the elementwise part of KimiDeltaAttention._projections,
// kimi_linear/kda.py:399-461, after the projection GEMMs):
//   q, k, v = l2norm(silu(ShortConv(q_in))), l2norm(silu(ShortConv(k_in))),
//             silu(ShortConv(v_in))                      (kda.py:282-325,446-450)
//   g       = -exp(A_log) * softplus(gk + dt_bias)       (kda.py:455-460)
//   beta    = sigmoid(beta_logit)                        (kda.py:452)
//   plus the new conv cache (the last conv_size - 1 inputs, kda.py:427-440).
// The reference runs ~10 separate passes over HBM for this; here one CTA per
// (b, head, 64-token tile, tensor) reads each input once and writes each
// output once.  The causal conv of a channel is a sliding window in
// registers (thread = channel); the per-token L2 norm is a warp reduction
// over the head dimension staged in shared memory.
//
// Epilogue (KimiDeltaAttention._output before o_proj, kda.py:464-470, with
// HeadwiseRMSNorm kda.py:258-279):
//   o = (rmsnorm_head(o_core) * w).to(dtype);  o = (o * sigmoid(og)).to(dtype)
// one warp per (b, t, h) row.
//
// Rounding follows the reference's fp16/bf16 path: the conv output, the SiLU
// output and the RMSNorm output are rounded to the I/O dtype where the
// reference materialises them in that dtype; reductions are fp32.
#include <type_traits>

#include "kda_internal.cuh"
#include "tc_ptx.cuh"

namespace kda {
namespace io {

constexpr int TT = 64;   // tokens per prologue CTA

// x rounded to T and back (identity for fp32)
template <typename T> __device__ __forceinline__ float rnd(float x);
template <> __device__ __forceinline__ float rnd<float>(float x) { return x; }
template <> __device__ __forceinline__ float rnd<__half>(float x) {
  return __half2float(__float2half_rn(x));
}
template <> __device__ __forceinline__ float rnd<__nv_bfloat16>(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }
// torch.nn.functional.softplus with beta = 1, threshold = 20
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float sigmoidf(float x) { return 1.f / (1.f + expf(-x)); }

// blockIdx.x: token tile, blockIdx.y: tensor * H + head (tensor 0 q, 1 k, 2 v,
// 3 gates), blockIdx.z: batch.  blockDim.x = head dim (32, 64 or 128).
template <typename TIO, typename TG>
__global__ void __launch_bounds__(128)
prologue_kernel(const PrologueParams p) {
  // launched as a programmatic dependent: nothing is touched before the
  // previous kernel on the stream completed; the next one may start launching
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  __shared__ float ys[TT][128 + 1];
  __shared__ float rstd[TT];
  const int c = threadIdx.x;                       // channel within the head
  const int HD = blockDim.x;
  const int tensor = blockIdx.y / p.H, h = blockIdx.y - tensor * p.H;
  const int b = blockIdx.z;
  const int t0 = blockIdx.x * TT;
  const int nt = min(TT, p.T - t0);
  const int lane = c & 31, warp = c >> 5, nw = HD >> 5;

  if (tensor == 3) {                               // decay and beta gates
    const int ch = h * p.K + c;
    if (c < p.K) {
      const float a = -expf(p.A_log[ch]);
      const float dtb = p.dt_bias[ch];
      const TG* gk = static_cast<const TG*>(p.gk) + b * p.gk_s[0] + ch;
      float* g = p.g + b * p.g_s[0] + h * p.g_s[2] + c;
      for (int i = 0; i < nt; ++i) {
        const int t = t0 + i;
        g[(int64_t)t * p.g_s[1]] = a * softplus(ld(gk + (int64_t)t * p.gk_s[1]) + dtb);
      }
    }
    for (int i = c; i < nt; i += blockDim.x) {         // beta: every token of the tile
      const int t = t0 + i;
      const TG* bl = static_cast<const TG*>(p.beta_logit) + b * p.bl_s[0] + (int64_t)t * p.bl_s[1] + h;
      p.beta[b * p.beta_s[0] + (int64_t)t * p.beta_s[1] + h] = sigmoidf(ld(bl));
    }
    return;
  }

  const int D = tensor == 2 ? p.H * p.V : p.H * p.K;
  const int ch = h * HD + c;                       // channel in [0, D)
  const TIO* x = static_cast<const TIO*>(tensor == 0 ? p.q_in : tensor == 1 ? p.k_in : p.v_in) +
                 b * p.in_s[tensor][0] + ch;
  const int64_t xs = p.in_s[tensor][1];
  const TIO* hist = static_cast<const TIO*>(tensor == 0 ? p.hist_q : tensor == 1 ? p.hist_k : p.hist_v);
  const float* w = (tensor == 0 ? p.w_q : tensor == 1 ? p.w_k : p.w_v) + (int64_t)ch * p.conv_size;
  const float* bias = tensor == 0 ? p.b_q : tensor == 1 ? p.b_k : p.b_v;
  const int cs = p.conv_size, keep = cs - 1;

  // input at time t (t < 0 reads the conv history, or zero without one)
  auto xin = [&](int t) -> float {
    if (t >= 0) return ld(x + (int64_t)t * xs);
    if (hist == nullptr) return 0.f;
    return ld(hist + b * p.hist_bs[tensor] + (int64_t)(keep + t) * D + ch);
  };
  // a fixed four-tap window: after the shift of step i, win[j] = x(t0+i-3+j);
  // the conv_size taps sit at its right end and the rest are never used
  // (static register indexing).  Before the first shift slots 1-3 hold
  // x(t0-3 .. t0-1).
  float wr[4], win[4];
  const float bv = bias ? bias[ch] : 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    wr[j] = (j >= 4 - cs) ? w[j - (4 - cs)] : 0.f;
    win[j] = (j >= 1 && j - 1 >= 4 - cs) ? xin(t0 - 4 + j) : 0.f;
  }
  for (int i = 0; i < nt; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) win[j] = win[j + 1];
    win[3] = xin(t0 + i);
    float acc = bv;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j >= 4 - cs) acc = fmaf(win[j], wr[j], acc);
    // conv output in the I/O dtype, SiLU of it, again in the I/O dtype
    ys[i][c] = rnd<TIO>(silu(rnd<TIO>(acc)));
  }
  // new conv cache: the last keep inputs of cat(history, x)
  if (p.new_q != nullptr && t0 + nt == p.T && keep > 0) {
    TIO* nc = static_cast<TIO*>(tensor == 0 ? p.new_q : tensor == 1 ? p.new_k : p.new_v) +
              b * (int64_t)keep * D + ch;
    for (int j = 0; j < keep; ++j) st(nc + (int64_t)j * D, xin(p.T - keep + j));
  }
  __syncthreads();

  const bool norm = tensor < 2;
  if (norm) {                                      // per-token L2 norm over the head
    for (int i = warp; i < nt; i += nw) {
      float ss = 0.f;
      for (int cc = lane; cc < HD; cc += 32) ss = fmaf(ys[i][cc], ys[i][cc], ss);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) rstd[i] = fminf(rsqrtf(ss), 1.f / p.eps);
    }
    __syncthreads();
  }
  TIO* out = static_cast<TIO*>(tensor == 0 ? p.q : tensor == 1 ? p.k : p.v) +
             b * p.out_s[tensor][0] + h * p.out_s[tensor][2] + c;
  const int64_t os = p.out_s[tensor][1];
  for (int i = 0; i < nt; ++i) {
    const float y = norm ? ys[i][c] * rstd[i] : ys[i][c];
    st(out + (int64_t)(t0 + i) * os, y);
  }
}

// 8 consecutive values from a 16-byte-aligned address as fp32 / 8 fp32 values
// stored as T (round to nearest) at a 16-byte-aligned address
template <typename T>
__device__ __forceinline__ void ld8v(const T* ptr, float (&x)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = *reinterpret_cast<const float4*>(ptr);
    const float4 c = *reinterpret_cast<const float4*>(ptr + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(ptr);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f;
      if constexpr (std::is_same<T, __half>::value)
        f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      else
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
}
template <typename T>
__device__ __forceinline__ void st8v(T* ptr, const float (&x)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __half>::value) {
      const __half2 hv = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&hv);
    } else {
      const __nv_bfloat162 hv = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&hv);
    }
  }
  *reinterpret_cast<uint4*>(ptr) = make_uint4(w[0], w[1], w[2], w[3]);
}

// The same prologue for 16-bit I/O with 16-byte-aligned rows (what the module
// passes), head dim HD in {32, 64, 128}: a CTA walks NTL tiles of one tensor
// and head; a tile's input rows (and the three before it, the conv window)
// arrive in one of two shared-memory buffers by 16-byte cp.async copies issued
// while the previous tile computes, and a thread owns 4 adjacent channels of a
// run of TPT tokens (8-byte shared loads and global stores; a token's HD / 4
// channel groups are consecutive lanes, so its L2 norm is a shuffle reduction).
// The thread-per-channel kernel above issues 2-byte accesses, 64 bytes per
// warp request, and the SM's limit on outstanding requests caps it near
// 0.6 TB/s.  Tiles of TTV = 32 tokens; 4 channels a thread keep the conv taps
// in 16 registers (80 a thread, six CTAs an SM).  The grid's y index
// interleaves the four tensors (q, k, v, gates) head by head, so the cheaper
// gate CTAs do not all land in the last wave.  A thread's channels are
// computed in pairs with the two-lane fp32 instructions of sm_100 (FFMA2 /
// FADD2 / FMUL2, each lane rounded like the scalar instruction): the kernel
// is issue-bound.  Same rounding points; SiLU,
// sigmoid and softplus use the fast exponential, logarithm and divide, whose
// ~1e-6 relative error vanishes in the rounding of SiLU's output to the
// 16-bit I/O type and is far below the fp32 gates' tolerance.
constexpr int TTV = 32;   // tokens per tile of the vectorised prologue
constexpr int NTL = 3;    // tiles per CTA: the next tile's copies fly while this one computes

__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
// softplus (threshold 20): log1p(u), u = e^x, by its series to u^7 below
// u = 1/8 (truncation < u^8 / 8, relative 2^-24) and by log(1 + u) above it
// (rounding of 1 + u and the fast logarithm: ~1e-6 relative)
__device__ __forceinline__ float softplus_fast(float x) {
  const float u = __expf(x);
  const float ser = u * (1.f - u * (0.5f - u * (1.f / 3 - u * (0.25f - u * (0.2f - u * (1.f / 6 - u * (1.f / 7)))))));
  const float lg = __logf(1.f + u);
  return x > 20.f ? x : (u < 0.125f ? ser : lg);
}

// Two lanes of fp32 arithmetic per instruction (sm_100 FFMA2 / FADD2 / FMUL2,
// each lane rounded to nearest like the scalar instruction)
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
// a pair rounded to T and back (identity for fp32)
template <typename T>
__device__ __forceinline__ float2 rnd2(float2 x) {
  if constexpr (std::is_same<T, __half>::value) {
    return __half22float2(__floats2half2_rn(x.x, x.y));
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __bfloat1622float2(__floats2bfloat162_rn(x.x, x.y));
  } else {
    return x;
  }
}
// softplus_fast of a pair: the series and the final scaling two lanes at a time
__device__ __forceinline__ float2 softplus2_fast(float2 x) {
  const float2 u = f2(__expf(x.x), __expf(x.y));
  const float2 nu = f2(-u.x, -u.y);
  float2 ser = __ffma2_rn(nu, f2(1.f / 7, 1.f / 7), f2(1.f / 6, 1.f / 6));
  ser = __ffma2_rn(nu, ser, f2(0.2f, 0.2f));
  ser = __ffma2_rn(nu, ser, f2(0.25f, 0.25f));
  ser = __ffma2_rn(nu, ser, f2(1.f / 3, 1.f / 3));
  ser = __ffma2_rn(nu, ser, f2(0.5f, 0.5f));
  ser = __ffma2_rn(nu, ser, f2(1.f, 1.f));
  ser = __fmul2_rn(u, ser);
  const float2 w = __fadd2_rn(f2(1.f, 1.f), u);
  const float lx = __logf(w.x), ly = __logf(w.y);
  return f2(x.x > 20.f ? x.x : (u.x < 0.125f ? ser.x : lx),
            x.y > 20.f ? x.y : (u.y < 0.125f ? ser.y : ly));
}

// 16-byte asynchronous copy global -> shared (L2 only); src_bytes = 0 fills zeros
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// every committed group of this thread except the newest one has landed
__device__ __forceinline__ void cp_async_wait_prev() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}


// N in {4, 8} consecutive values (16-byte or, for N = 4 and 16-bit T, 8-byte
// aligned) as fp32, and back
template <int N, typename T>
__device__ __forceinline__ void ldv(const T* ptr, float (&x)[N]) {
  if constexpr (N == 8) {
    ld8v(ptr, x);
  } else if constexpr (std::is_same<T, float>::value) {
    const float4 a = *reinterpret_cast<const float4*>(ptr);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(ptr);
    const uint32_t w[2] = {u.x, u.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float2 f;
      if constexpr (std::is_same<T, __half>::value)
        f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      else
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
}
template <int N, typename T>
__device__ __forceinline__ void stv(T* ptr, const float (&x)[N]) {
  if constexpr (std::is_same<T, float>::value) {
#pragma unroll
    for (int i = 0; i < N; i += 4)
      *reinterpret_cast<float4*>(ptr + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
  } else if constexpr (N == 8) {
    st8v(ptr, x);
  } else {
    uint32_t w[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if constexpr (std::is_same<T, __half>::value) {
        const __half2 hv = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&hv);
      } else {
        const __nv_bfloat162 hv = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&hv);
      }
    }
    *reinterpret_cast<uint2*>(ptr) = make_uint2(w[0], w[1]);
  }
}

template <typename TIO, typename TG, int HD>
__global__ void __launch_bounds__(128)
prologue_vec_kernel(const PrologueParams p) {
  // launched as a programmatic dependent: nothing is touched before the
  // previous kernel on the stream completed; the next one may start launching
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  constexpr int CPT = 4, C8 = HD / 8, CG = HD / CPT, TGRP = 128 / CG, TPT = TTV / TGRP;
  static_assert(TPT >= 1 && TPT * TGRP == TTV, "tile split");
  __shared__ __align__(16) TIO xst[2][TTV + 3][HD];   // input rows t0 - 3 .. t0 + TTV - 1
  const int tid = threadIdx.x, cg = tid % CG, tg = tid / CG;
  const int tensor = blockIdx.y & 3, h = blockIdx.y >> 2;   // y = 4 h + tensor
  const int b = blockIdx.z;
  const int tile0 = blockIdx.x * NTL;
  const int ntl = min(NTL, (p.T + TTV - 1) / TTV - tile0);
  const int i0 = tg * TPT;                         // first token of this thread in a tile

  if (tensor == 3) {                               // decay and beta gates
    const int ch0 = h * p.K + CPT * cg;
    float a[CPT], dtb[CPT];
#pragma unroll
    for (int e = 0; e < CPT; ++e) {
      a[e] = -expf(p.A_log[ch0 + e]);
      dtb[e] = p.dt_bias[ch0 + e];
    }
    const TG* gk = static_cast<const TG*>(p.gk) + b * p.gk_s[0] + ch0;
    float* g = p.g + b * p.g_s[0] + h * p.g_s[2] + CPT * cg;
    for (int k = 0; k < ntl; ++k) {
    const int t0 = (tile0 + k) * TTV;
    const int nt = min(TTV, p.T - t0);
    float gv[TPT][CPT];
    const TG* grow = gk + (int64_t)(t0 + i0) * p.gk_s[1];   // input row of token i0 + i
    float* orow = g + (int64_t)(t0 + i0) * p.g_s[1];        // output row of token i0 + i
#pragma unroll
    for (int i = 0; i < TPT; ++i)
      if (i0 + i < nt) ldv<CPT>(grow + i * p.gk_s[1], gv[i]);
#pragma unroll
    for (int i = 0; i < TPT; ++i) {
      if (i0 + i >= nt) break;
      float y[CPT];
#pragma unroll
      for (int e = 0; e < CPT; e += 2) {
        const float2 sp = softplus2_fast(__fadd2_rn(f2(gv[i][e], gv[i][e + 1]), f2(dtb[e], dtb[e + 1])));
        const float2 r = __fmul2_rn(f2(a[e], a[e + 1]), sp);
        y[e] = r.x;
        y[e + 1] = r.y;
      }
      stv<CPT>(orow, y);
      orow += p.g_s[1];
    }
    for (int i = tid; i < nt; i += blockDim.x) {       // beta: every token of the tile
      const int t = t0 + i;
      const TG* bl = static_cast<const TG*>(p.beta_logit) + b * p.bl_s[0] + (int64_t)t * p.bl_s[1] + h;
      p.beta[b * p.beta_s[0] + (int64_t)t * p.beta_s[1] + h] = sigmoid_fast(ld(bl));
    }
    }  // tiles
    return;
  }

  const int D = tensor == 2 ? p.H * p.V : p.H * p.K;
  const int ch0 = h * HD + CPT * cg;
  const TIO* x = static_cast<const TIO*>(tensor == 0 ? p.q_in : tensor == 1 ? p.k_in : p.v_in) +
                 b * p.in_s[tensor][0] + ch0;
  const int64_t xs = p.in_s[tensor][1];
  const TIO* hist = static_cast<const TIO*>(tensor == 0 ? p.hist_q : tensor == 1 ? p.hist_k : p.hist_v);
  const TIO* hb = hist ? hist + b * p.hist_bs[tensor] + ch0 : nullptr;
  const float* w = (tensor == 0 ? p.w_q : tensor == 1 ? p.w_k : p.w_v) + (int64_t)ch0 * p.conv_size;
  const float* bias = tensor == 0 ? p.b_q : tensor == 1 ? p.b_k : p.b_v;
  const int cs = p.conv_size, keep = cs - 1;

  // tile k's rows t0 - 3 .. t0 + TTV - 1 of this head into staging buffer
  // k % 2 by 16-byte asynchronous copies (no registers held while they fly;
  // rows outside the input and the history are zero-filled)
  const TIO* xh = x - CPT * cg;                      // channel 0 of this head
  const TIO* hh = hb ? hb - CPT * cg : nullptr;
  // A thread copies the same 16-byte column c8 of every (128 / C8)-th row, so
  // its source and destination advance by constant strides.
  auto stage = [&](int k) {
    constexpr int RS = 128 / C8;                   // rows per pass of the CTA
    static_assert(RS * C8 == 128, "whole rows per pass");
    const int t0 = (tile0 + k) * TTV, nt = min(TTV, p.T - t0);
    const int c8 = tid % C8;
    int row = tid / C8;
    int64_t off = (int64_t)(t0 + row - 3) * xs + 8 * c8;   // element offset of row's input
    const int64_t step = (int64_t)RS * xs;
    TIO* dst = &xst[k & 1][row][8 * c8];
    for (; row < TTV + 3; row += RS, off += step, dst += RS * HD) {
      const int i = row - 3, t = t0 + i;
      const TIO* src = xh;
      uint32_t bytes = 0;
      if (i < nt && t >= 0) {
        src = xh + off;
        bytes = 16;
      } else if (i < nt && hh != nullptr && t >= -keep) {
        src = hh + (int64_t)(keep + t) * D + 8 * c8;
        bytes = 16;
      }
      cp_async16(dst, src, bytes);
    }
  };
  stage(0);
  cp_async_commit();
  // taps at the right end of a four-wide window, as in the kernel above
  float wv[CPT][4], bv[CPT];
#pragma unroll
  for (int e = 0; e < CPT; ++e) {
    bv[e] = bias ? bias[ch0 + e] : 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) wv[e][j] = (j >= 4 - cs) ? w[e * cs + j - (4 - cs)] : 0.f;
  }
  const bool norm = tensor < 2;
  TIO* out = static_cast<TIO*>(tensor == 0 ? p.q : tensor == 1 ? p.k : p.v) +
             b * p.out_s[tensor][0] + h * p.out_s[tensor][2] + CPT * cg;
  const int64_t os = p.out_s[tensor][1];
  for (int k = 0; k < ntl; ++k) {
  const int t0 = (tile0 + k) * TTV;
  const int nt = min(TTV, p.T - t0);
  if (k + 1 < ntl) stage(k + 1);                   // into the buffer tile k - 1 used
  cp_async_commit();                               // (empty on the last tile)
  cp_async_wait_prev();                            // tile k's copies have landed
  __syncthreads();
  // the thread's TPT tokens need window rows i0 .. i0 + TPT + 2: each row is
  // read from shared memory once and slides through the four-row window.  The
  // CG channel groups of a token are CG consecutive lanes, so the per-token L2
  // norm is a shuffle reduction, done for NB tokens at a time: a reduce-scatter
  // over lane bits 0 .. log2(NB) - 1 (at each step a lane keeps half of its
  // tokens' partial sums and adds its partner's partial of the same tokens),
  // then a plain butterfly over the remaining bits.  The lanes pair up exactly
  // as in a butterfly of each token alone (xor 1, 2, 4, ...), so every sum is
  // bit-identical to it; the norm costs ~7 instead of ~13 instructions per token.
  // Rows past nt are zeros and are not stored.
  {
    constexpr int NB = TPT < 4 ? TPT : 4;          // tokens per reduction (8 measured slower)
    constexpr int LNB = NB == 4 ? 2 : NB == 2 ? 1 : 0;
    const int gbase = (tid & 31) - cg;             // first lane of this token group
    const TIO* xb = &xst[k & 1][i0][CPT * cg];
    TIO* orow = out + (int64_t)(t0 + i0) * os;       // output row of token i0 + i
    float xw[4][CPT];
#pragma unroll
    for (int j = 0; j < 3; ++j) ldv<CPT>(xb + j * HD, xw[j + 1]);
#pragma unroll
    for (int ib = 0; ib < TPT; ib += NB) {
      float y[NB][CPT], ss[NB];
#pragma unroll
      for (int u = 0; u < NB; ++u) {
#pragma unroll
        for (int j = 0; j < 3; ++j)
#pragma unroll
          for (int e = 0; e < CPT; ++e) xw[j][e] = xw[j + 1][e];
        ldv<CPT>(xb + (ib + u + 3) * HD, xw[3]);
        // two channels per instruction: conv, the SiLU denominator, the squares
        float2 ss2 = f2(0.f, 0.f);
#pragma unroll
        for (int e = 0; e < CPT; e += 2) {
          float2 acc = f2(bv[e], bv[e + 1]);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j >= 4 - cs)
              acc = __ffma2_rn(f2(xw[j][e], xw[j][e + 1]), f2(wv[e][j], wv[e + 1][j]), acc);
          const float2 c = rnd2<TIO>(acc);
          const float2 den = __fadd2_rn(f2(1.f, 1.f), f2(__expf(-c.x), __expf(-c.y)));
          const float2 sv = rnd2<TIO>(f2(__fdividef(c.x, den.x), __fdividef(c.y, den.y)));
          ss2 = __ffma2_rn(sv, sv, ss2);
          y[u][e] = sv.x;
          y[u][e + 1] = sv.y;
        }
        ss[u] = ss2.x + ss2.y;
      }
      if (norm) {
#pragma unroll
        for (int bit = 0; bit < LNB; ++bit) {
          const int half = NB >> (bit + 1);
          const bool hi = (cg >> bit) & 1;
#pragma unroll
          for (int j = 0; j < half; ++j) {
            const float send = hi ? ss[j] : ss[j + half];
            const float keep = hi ? ss[j + half] : ss[j];
            ss[j] = keep + __shfl_xor_sync(0xffffffffu, send, 1 << bit);
          }
        }
        // this lane now sums token sum_b hi_b * NB / 2^(b + 1) of the batch
        float tot = ss[0];
#pragma unroll
        for (int off = NB; off < CG; off <<= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
        const float r = fminf(rsqrtf(tot), 1.f / p.eps);
#pragma unroll
        for (int u = 0; u < NB; ++u) {
          int src = 0;                             // a lane holding token u: bits of u reversed
#pragma unroll
          for (int bit = 0; bit < LNB; ++bit) src |= ((u >> (LNB - 1 - bit)) & 1) << bit;
          const float ru = __shfl_sync(0xffffffffu, r, gbase + src);
#pragma unroll
          for (int e = 0; e < CPT; e += 2) {
            const float2 sc = __fmul2_rn(f2(y[u][e], y[u][e + 1]), f2(ru, ru));
            y[u][e] = sc.x;
            y[u][e + 1] = sc.y;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < NB; ++u) {
        if (i0 + ib + u < nt) stv<CPT>(orow, y[u]);
        orow += os;
      }
    }
  }
  // new conv cache: the last keep inputs of cat(history, x)
  if (p.new_q != nullptr && t0 + nt == p.T && keep > 0 && tg == 0) {
    TIO* nc = static_cast<TIO*>(tensor == 0 ? p.new_q : tensor == 1 ? p.new_k : p.new_v) +
              b * (int64_t)keep * D + ch0;
    for (int j = 0; j < keep; ++j) {
      const int t = p.T - keep + j;
#pragma unroll
      for (int e = 0; e < CPT; ++e) {
        const float v = t >= 0 ? ld(x + (int64_t)t * xs + e)
                               : (hb != nullptr ? ld(hb + (int64_t)(keep + t) * D + e) : 0.f);
        st(nc + (int64_t)j * D + e, v);
      }
    }
  }
  __syncthreads();                                 // this staging buffer free
  }  // tiles
}

// one warp per (b, t, h) row of V channels (V <= 128, multiple of 32)
template <typename TIO>
__global__ void __launch_bounds__(256)
epilogue_kernel(const EpilogueParams p) {
  // launched as a programmatic dependent: nothing is touched before the
  // previous kernel on the stream completed; the next one may start launching
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const long rows = (long)p.B * p.T * p.H;
  if (warp >= rows) return;
  const int h = warp % p.H;
  const long bt = warp / p.H;
  const int t = (int)(bt % p.T), b = (int)(bt / p.T);
  const TIO* o = static_cast<const TIO*>(p.o) + b * p.o_s[0] + (int64_t)t * p.o_s[1] + h * p.o_s[2];
  const TIO* og = static_cast<const TIO*>(p.og) + b * p.og_s[0] + (int64_t)t * p.og_s[1] + h * p.V;
  TIO* y = static_cast<TIO*>(p.y) + b * p.y_s[0] + (int64_t)t * p.y_s[1] + h * p.V;
  const float* w = p.weight + h * p.V;
  float xv[4] = {0.f, 0.f, 0.f, 0.f};
  float ss = 0.f;
  const int n = p.V >> 5;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j < n) xv[j] = ld(o + lane + 32 * j);
    ss = fmaf(xv[j], xv[j], ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float r = rsqrtf(ss / p.V + p.eps);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j >= n) break;
    const int cc = lane + 32 * j;
    const float nrm = rnd<TIO>(xv[j] * r * w[cc]);                 // g_norm output dtype
    st(y + cc, nrm * sigmoidf(ld(og + cc)));                       // gate in fp32, round once
  }
}

// every address the vectorised prologue touches with 16-byte accesses is
// 16-byte aligned (pointers and strides; inner strides are 1 by contract)
static bool vec_ok(const PrologueParams& p, size_t gate_size) {
  auto al = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; };
  if (!(p.K == p.V && (p.K == 32 || p.K == 64 || p.K == 128))) return false;
  const void* in[3] = {p.q_in, p.k_in, p.v_in};
  const void* out[3] = {p.q, p.k, p.v};
  const void* hist[3] = {p.hist_q, p.hist_k, p.hist_v};
  for (int t = 0; t < 3; ++t) {
    if (!al(in[t]) || p.in_s[t][0] % 8 || p.in_s[t][1] % 8) return false;
    if (!al(out[t]) || p.out_s[t][0] % 8 || p.out_s[t][1] % 8 || p.out_s[t][2] % 8 ||
        p.out_s[t][3] != 1)
      return false;
    if (hist[t] != nullptr && (!al(hist[t]) || p.hist_bs[t] % 8)) return false;
  }
  const int64_t gper = 16 / (int64_t)gate_size;
  if (!al(p.gk) || p.gk_s[0] % gper || p.gk_s[1] % gper) return false;
  if (!al(p.g) || p.g_s[0] % 4 || p.g_s[1] % 4 || p.g_s[2] % 4 || p.g_s[3] != 1) return false;
  return true;
}

template <typename TIO, typename TG>
static cudaError_t launch_pro_g(const PrologueParams& p, cudaStream_t s) {
  dim3 grid((p.T + TT - 1) / TT, 4 * p.H, p.B);
  if constexpr (!std::is_same<TIO, float>::value) {
    if (vec_ok(p, sizeof(TG))) {
      const dim3 vgrid((p.T + TTV * NTL - 1) / (TTV * NTL), 4 * p.H, p.B);
      switch (p.K) {
        case 32: return launch_dependent(prologue_vec_kernel<TIO, TG, 32>, vgrid, 128, 0, s, p);
        case 64: return launch_dependent(prologue_vec_kernel<TIO, TG, 64>, vgrid, 128, 0, s, p);
        default: return launch_dependent(prologue_vec_kernel<TIO, TG, 128>, vgrid, 128, 0, s, p);
      }
    }
  }
  const int threads = p.K;   // K == V enforced by the caller
  return launch_dependent(prologue_kernel<TIO, TG>, grid, threads, 0, s, p);
}

// The epilogue for 16-bit I/O with V = 128 and 16-byte-aligned rows: a half
// warp owns one (b, t, h) row, lane l of it channels 8l .. 8l + 7 (one 16-byte
// access per tensor and row), and a warp walks EPI_ROWS rows whose loads are
// all issued before the first row computes, so each thread keeps
// EPI_ROWS / 2 x 32 bytes in flight (the scalar kernel above makes 2-byte
// accesses, one row per warp).  Same rounding points; the gate's sigmoid uses
// the fast exponential and divide (~1e-6 relative, below the output's 16-bit
// rounding).
constexpr int EPI_ROWS = 4;   // rows per warp of the vectorised epilogue

template <typename TIO>
__global__ void __launch_bounds__(256)
epilogue_vec_kernel(const EpilogueParams p) {
  // launched as a programmatic dependent: nothing is touched before the
  // previous kernel on the stream completed; the next one may start launching
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  constexpr int NI = EPI_ROWS / 2;
  const long warp = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, half = lane >> 4, c = lane & 15;
  const long rows = (long)p.B * p.T * p.H;
  const long r0 = warp * EPI_ROWS + half;
  if (warp * EPI_ROWS >= rows) return;
  // (b, t, h) of row r0; the row two further on is h + 2 with carries into t, b
  const int h0 = (int)(r0 % p.H);
  const long bt0 = r0 / p.H;
  const int t0 = (int)(bt0 % p.T), b0 = (int)(bt0 / p.T);
  auto next = [&](int& b, int& t, int& h) {
    for (h += 2; h >= p.H; h -= p.H)
      if (++t == p.T) { t = 0; ++b; }
  };
  uint4 xo[NI], xg[NI];
  {
    int b = b0, t = t0, h = h0;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      if (i > 0) next(b, t, h);
      xo[i] = make_uint4(0u, 0u, 0u, 0u);
      xg[i] = xo[i];
      if (r0 + 2 * i < rows) {
        xo[i] = *reinterpret_cast<const uint4*>(static_cast<const TIO*>(p.o) + b * p.o_s[0] +
                                                (int64_t)t * p.o_s[1] + h * p.o_s[2] + 8 * c);
        xg[i] = *reinterpret_cast<const uint4*>(static_cast<const TIO*>(p.og) + b * p.og_s[0] +
                                                (int64_t)t * p.og_s[1] + h * 128 + 8 * c);
      }
    }
  }
  int b = b0, t = t0, h = h0;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    if (i > 0) next(b, t, h);
    float xv[8], gv[8];
    ld8v(reinterpret_cast<const TIO*>(&xo[i]), xv);
    ld8v(reinterpret_cast<const TIO*>(&xg[i]), gv);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(xv[j], xv[j], ss);
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (r0 + 2 * i >= rows) continue;
    const float rs = rsqrtf(ss / 128.f + p.eps);
    const float* w = p.weight + h * 128 + 8 * c;
    const float4 w0 = *reinterpret_cast<const float4*>(w);
    const float4 w1 = *reinterpret_cast<const float4*>(w + 4);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = rnd<TIO>(xv[j] * rs * wv[j]) * sigmoid_fast(gv[j]);
    st8v(static_cast<TIO*>(p.y) + b * p.y_s[0] + (int64_t)t * p.y_s[1] + h * 128 + 8 * c, out);
  }
}

template <typename TIO>
static cudaError_t launch_pro_t(const PrologueParams& p, cudaStream_t s) {
  if (p.gate_dtype == KDA_DTYPE_F32) return launch_pro_g<TIO, float>(p, s);
  if (p.gate_dtype == KDA_DTYPE_F16) return launch_pro_g<TIO, __half>(p, s);
  return launch_pro_g<TIO, __nv_bfloat16>(p, s);
}

}  // namespace io

cudaError_t launch_prologue(const PrologueParams& p, cudaStream_t s) {
  switch (p.io_dtype) {
    case KDA_DTYPE_F32: return io::launch_pro_t<float>(p, s);
    case KDA_DTYPE_F16: return io::launch_pro_t<__half>(p, s);
    default: return io::launch_pro_t<__nv_bfloat16>(p, s);
  }
}

cudaError_t launch_epilogue(const EpilogueParams& p, cudaStream_t s) {
  const long rows = (long)p.B * p.T * p.H;
  const int threads = 256;
  const long blocks = (rows * 32 + threads - 1) / threads;
  auto al16 = [](const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; };
  const bool vec = p.io_dtype != KDA_DTYPE_F32 && p.V == 128 && al16(p.o) && al16(p.og) &&
                   al16(p.y) && al16(p.weight) && p.o_s[0] % 8 == 0 && p.o_s[1] % 8 == 0 &&
                   p.o_s[2] % 8 == 0 && p.og_s[0] % 8 == 0 && p.og_s[1] % 8 == 0 &&
                   p.y_s[0] % 8 == 0 && p.y_s[1] % 8 == 0;
  const long vblocks = (rows + io::EPI_ROWS * (threads / 32) - 1) / (io::EPI_ROWS * (threads / 32));
  switch (p.io_dtype) {
    case KDA_DTYPE_F32:
      return launch_dependent(io::epilogue_kernel<float>, dim3(blocks), threads, 0, s, p);
    case KDA_DTYPE_F16:
      return vec ? launch_dependent(io::epilogue_vec_kernel<__half>, dim3(vblocks), threads, 0, s, p)
                 : launch_dependent(io::epilogue_kernel<__half>, dim3(blocks), threads, 0, s, p);
    default:
      return vec ? launch_dependent(io::epilogue_vec_kernel<__nv_bfloat16>, dim3(vblocks), threads, 0, s, p)
                 : launch_dependent(io::epilogue_kernel<__nv_bfloat16>, dim3(blocks), threads, 0, s, p);
  }
}

}  // namespace kda
