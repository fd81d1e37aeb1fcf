// kda_backward.cu -- gradient of the KDA recurrence for sm_100a.
//
// The reference gets gradients from torch autograd through kda_chunkwise /
// kda_recurrent (kimi_linear/kda.py:58-219).  Both compute the same function,
// the token recurrence (paper Eq. 1), per (b, h):
//   St = Diag(alpha_t) S_{t-1},  a_t = k_t^T St,  u_t = beta_t (v_t - a_t),
//   S_t = St + k_t u_t^T,        o_t = S_t^T q'_t      (q' = scale q, alpha = exp g)
// whose exact reverse-mode gradient, per step from t = T-1 down to 0, is
//   dS   += q'_t dO_t^T              dq'_t  = S_t dO_t
//   du    = dS^T k_t                 dv_t   = beta_t du
//   dbeta_t = du . (v_t - a_t)       da     = -beta_t du
//   dk_t  = dS u_t + St da           dSt    = dS + k_t da^T
//   dg_t  = rowsum(dSt (.) St)       dS_{t-1} = Diag(alpha_t) dSt
// (dg = alpha (.) dalpha with dalpha = rowsum(dSt (.) S_{t-1})).
//
// Two kernels, one CTA per (b, h, 16-column tile of V); a thread owns 4
// adjacent columns of K/32 rows:
//  * checkpoint_kernel runs the recurrence forward and stores the state tile
//    before every 64-step chunk (fp32);
//  * backward_kernel walks the chunks backwards: it reruns a chunk from its
//    checkpoint keeping every 8th state, then per 8-step block reruns the
//    block keeping each step's S_{t-1}, u_t and v_t - a_t, and applies the
//    reverse steps above.  All per-step state copies are thread-private
//    (each thread stores and reloads only its own elements), so only the two
//    reductions over K (a_t in the rerun, du in the reverse step) need a
//    barrier.  dq, dk, dg and dbeta sum over the V columns: each tile writes
//    its partial sums, added up afterwards over the V/16 tiles.
#include "kda_internal.cuh"

namespace kda {
namespace bwd {

constexpr int NTH = 128;
constexpr int CT = 4;              // column groups of 4 -> 16 columns per tile
constexpr int VT = 4 * CT;
constexpr int RG = NTH / CT;       // 32 row groups
constexpr int CK = 64;             // checkpoint interval (steps)
constexpr int SB = 8;              // sub-checkpoint interval inside a chunk

// per-step vectors of step t for this thread: q', k, alpha of its rows, v of
// its columns and beta
template <typename TIO, int R>
struct StepIn {
  float q[R], k[R], al[R], v[4], beta;
};

template <typename TIO, int R>
__device__ __forceinline__ void load_step(const BwdParams& p, int b, int h, int t, int rg,
                                          int col0, StepIn<TIO, R>& s) {
  const TIO* qb = static_cast<const TIO*>(p.q) + b * p.q_s[0] + (int64_t)t * p.q_s[1] + h * p.q_s[2];
  const TIO* kb = static_cast<const TIO*>(p.k) + b * p.k_s[0] + (int64_t)t * p.k_s[1] + h * p.k_s[2];
  const TIO* vb = static_cast<const TIO*>(p.v) + b * p.v_s[0] + (int64_t)t * p.v_s[1] + h * p.v_s[2];
  const float* gb = p.g + b * p.g_s[0] + (int64_t)t * p.g_s[1] + h * p.g_s[2];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = rg + RG * r;
    s.q[r] = ld(qb + i) * p.scale;
    s.k[r] = ld(kb + i);
    s.al[r] = expf(gb[i]);
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) s.v[c] = ld(vb + col0 + c);
  s.beta = p.beta[b * p.b_s[0] + (int64_t)t * p.b_s[1] + h * p.b_s[2]];
}

// sum over the K rows of per-column values x[4]: 8 row groups per warp by
// shuffles, 4 warps through shared memory; every thread gets the totals of
// its 4 columns
__device__ __forceinline__ void row_reduce(float (&x)[4], float (*red)[VT], int lane, int warp,
                                           int ct) {
#pragma unroll
  for (int off = CT; off < 32; off <<= 1)
#pragma unroll
    for (int c = 0; c < 4; ++c) x[c] += __shfl_xor_sync(0xffffffffu, x[c], off);
  if (lane < CT) {
#pragma unroll
    for (int c = 0; c < 4; ++c) red[warp][4 * ct + c] = x[c];
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < 4; ++c)
    x[c] = red[0][4 * ct + c] + red[1][4 * ct + c] + red[2][4 * ct + c] + red[3][4 * ct + c];
  __syncthreads();
}

// sum over the 4 column groups (lanes with the same row group)
__device__ __forceinline__ float col_reduce(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

// one forward step on the state tile; returns u (own columns) and v - a
template <typename TIO, int R>
__device__ __forceinline__ void fwd_step(float (&S)[R][4], const StepIn<TIO, R>& s,
                                         float (&u)[4], float (&vma)[4], float (*red)[VT],
                                         int lane, int warp, int ct) {
  float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      S[r][c] *= s.al[r];
      a[c] = fmaf(s.k[r], S[r][c], a[c]);
    }
  row_reduce(a, red, lane, warp, ct);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    vma[c] = s.v[c] - a[c];
    u[c] = s.beta * vma[c];
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) S[r][c] = fmaf(s.k[r], u[c], S[r][c]);
}

template <typename TIO, typename TSI, int R>
__global__ void __launch_bounds__(NTH, 1)
checkpoint_kernel(const BwdParams p) {
  __shared__ float red[4][VT];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ct = tid % CT, rg = tid / CT;
  const int b = blockIdx.z, h = blockIdx.y;
  const int col0 = blockIdx.x * VT + 4 * ct;
  const int NC = (p.T + CK - 1) / CK;
  float S[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = rg + RG * r;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      S[r][c] = p.state_in ? ld(static_cast<const TSI*>(p.state_in) + b * p.si_s[0] +
                                h * p.si_s[1] + (int64_t)i * p.si_s[2] + col0 + c)
                           : 0.f;
  }
  float* ck = p.ckpt + ((size_t)(b * p.H + h) * NC) * p.K * p.V;
  for (int t = 0; t < p.T; ++t) {
    if (t % CK == 0) {
      float* dst = ck + (size_t)(t / CK) * p.K * p.V;
#pragma unroll
      for (int r = 0; r < R; ++r)
        *reinterpret_cast<float4*>(dst + (size_t)(rg + RG * r) * p.V + col0) =
            make_float4(S[r][0], S[r][1], S[r][2], S[r][3]);
    }
    StepIn<TIO, R> s;
    load_step<TIO, R>(p, b, h, t, rg, col0, s);
    float u[4], vma[4];
    fwd_step<TIO, R>(S, s, u, vma, red, lane, warp, ct);
  }
}

template <typename TIO, typename TSO, int R>
__global__ void __launch_bounds__(NTH, 1)
backward_kernel(const BwdParams p) {
  extern __shared__ __align__(16) float smem[];
  // thread-private slots, element e of thread tid at [e * NTH + tid]
  float* subck = smem;                                   // SB sub-checkpoints x R*4
  float* sprev = subck + (size_t)SB * R * 4 * NTH;       // SB steps of S_{t-1}  x R*4
  float* su = sprev + (size_t)SB * R * 4 * NTH;          // SB steps of u       x 4
  float* svma = su + (size_t)SB * 4 * NTH;               // SB steps of v - a   x 4
  __shared__ float red[4][VT];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ct = tid % CT, rg = tid / CT;
  const int b = blockIdx.z, h = blockIdx.y, vt = blockIdx.x;
  const int col0 = vt * VT + 4 * ct;
  const int T = p.T, K = p.K, V = p.V;
  const int NC = (T + CK - 1) / CK;
  const float* ck = p.ckpt + ((size_t)(b * p.H + h) * NC) * K * V;

  // dS starts as the gradient of the returned state (zero when unused)
  float dS[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = rg + RG * r;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      dS[r][c] = p.dstate_out ? p.dstate_out[b * p.dso_s[0] + h * p.dso_s[1] +
                                             (int64_t)i * p.dso_s[2] + col0 + c]
                              : 0.f;
  }
  // partial-sum outputs of this column tile: [vt][b][t][h][k] and [vt][b][t][h]
  const size_t pk = (size_t)p.B * T * p.H * K;
  float* dq_p = p.dq_part + vt * pk;
  float* dk_p = p.dk_part + vt * pk;
  float* dg_p = p.dg_part + vt * pk;
  float* db_p = p.dbeta_part + (size_t)vt * p.B * T * p.H;
  auto kidx = [&](int t, int i) { return (((size_t)b * T + t) * p.H + h) * K + i; };

  for (int n = NC - 1; n >= 0; --n) {
    const int t0 = n * CK, t1 = min(T, t0 + CK);
    // rerun the chunk from its checkpoint, keeping every SB-th state
    float S[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float4 x = *reinterpret_cast<const float4*>(ck + (size_t)n * K * V +
                                                        (size_t)(rg + RG * r) * V + col0);
      S[r][0] = x.x; S[r][1] = x.y; S[r][2] = x.z; S[r][3] = x.w;
    }
    for (int t = t0; t < t1; ++t) {
      if ((t - t0) % SB == 0) {
        float* d = subck + (size_t)((t - t0) / SB) * R * 4 * NTH;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) d[(r * 4 + c) * NTH + tid] = S[r][c];
      }
      if (t + 1 < t1) {     // the chunk's last state is not needed
        StepIn<TIO, R> s;
        load_step<TIO, R>(p, b, h, t, rg, col0, s);
        float u[4], vma[4];
        fwd_step<TIO, R>(S, s, u, vma, red, lane, warp, ct);
      }
    }
    // the SB-step blocks, last first
    const int nsb = (t1 - t0 + SB - 1) / SB;
    for (int sb = nsb - 1; sb >= 0; --sb) {
      const int ts = t0 + sb * SB, te = min(t1, ts + SB);
      {
        const float* d = subck + (size_t)sb * R * 4 * NTH;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) S[r][c] = d[(r * 4 + c) * NTH + tid];
      }
      for (int t = ts; t < te; ++t) {   // rerun: keep S_{t-1}, u_t, v_t - a_t
        float* d = sprev + (size_t)(t - ts) * R * 4 * NTH;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) d[(r * 4 + c) * NTH + tid] = S[r][c];
        StepIn<TIO, R> s;
        load_step<TIO, R>(p, b, h, t, rg, col0, s);
        float u[4], vma[4];
        fwd_step<TIO, R>(S, s, u, vma, red, lane, warp, ct);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          su[((t - ts) * 4 + c) * NTH + tid] = u[c];
          svma[((t - ts) * 4 + c) * NTH + tid] = vma[c];
        }
      }
      for (int t = te - 1; t >= ts; --t) {   // reverse steps
        StepIn<TIO, R> s;
        load_step<TIO, R>(p, b, h, t, rg, col0, s);
        const TIO* dob = static_cast<const TIO*>(p.dout) + b * p.do_s[0] +
                         (int64_t)t * p.do_s[1] + h * p.do_s[2];
        float dO[4], u[4], vma[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          dO[c] = ld(dob + col0 + c);
          u[c] = su[((t - ts) * 4 + c) * NTH + tid];
          vma[c] = svma[((t - ts) * 4 + c) * NTH + tid];
        }
        const float* d = sprev + (size_t)(t - ts) * R * 4 * NTH;
        float St[R][4];                       // alpha (.) S_{t-1}
        float dqp[R], du[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float acc = 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            St[r][c] = s.al[r] * d[(r * 4 + c) * NTH + tid];
            const float Snew = fmaf(s.k[r], u[c], St[r][c]);   // S_t
            acc = fmaf(Snew, dO[c], acc);
            dS[r][c] = fmaf(s.q[r], dO[c], dS[r][c]);
            du[c] = fmaf(dS[r][c], s.k[r], du[c]);
          }
          dqp[r] = acc;
        }
        row_reduce(du, red, lane, warp, ct);
        float dbp = 0.f, da[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          dbp = fmaf(du[c], vma[c], dbp);
          da[c] = -s.beta * du[c];
        }
        if (rg == 0) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            p.dv[b * p.dv_s[0] + (int64_t)t * p.dv_s[1] + h * p.dv_s[2] + col0 + c] =
                s.beta * du[c];
        }
        dbp = col_reduce(dbp);
        if (tid == 0) db_p[((size_t)b * T + t) * p.H + h] = dbp;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float dkp = 0.f, dgp = 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            dkp = fmaf(dS[r][c], u[c], dkp);
            dkp = fmaf(St[r][c], da[c], dkp);
            const float dSt = fmaf(s.k[r], da[c], dS[r][c]);
            dgp = fmaf(dSt, St[r][c], dgp);
            dS[r][c] = s.al[r] * dSt;
          }
          const float q1 = col_reduce(dqp[r]), k1 = col_reduce(dkp), g1 = col_reduce(dgp);
          if (ct == 0) {
            const size_t at = kidx(t, rg + RG * r);
            dq_p[at] = q1 * p.scale;
            dk_p[at] = k1;
            dg_p[at] = g1;
          }
        }
      }
    }
  }
  // gradient of the initial state
  if (p.dstate_in != nullptr) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float* dst = p.dstate_in + b * p.dsi_s[0] + h * p.dsi_s[1] +
                   (int64_t)(rg + RG * r) * p.dsi_s[2] + col0;
#pragma unroll
      for (int c = 0; c < 4; ++c) dst[c] = dS[r][c];
    }
  }
}

template <typename TIO, typename TSI, int R>
static cudaError_t launch_r(const BwdParams& p, cudaStream_t s) {
  dim3 grid(p.V / VT, p.H, p.B);
  checkpoint_kernel<TIO, TSI, R><<<grid, NTH, 0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t smem = ((size_t)2 * SB * R * 4 + 2 * SB * 4) * NTH * sizeof(float);
  e = cudaFuncSetAttribute(backward_kernel<TIO, float, R>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  backward_kernel<TIO, float, R><<<grid, NTH, smem, s>>>(p);
  return cudaGetLastError();
}

template <typename TIO, typename TSI>
static cudaError_t launch_k(const BwdParams& p, cudaStream_t s) {
  switch (p.K) {
    case 32: return launch_r<TIO, TSI, 1>(p, s);
    case 64: return launch_r<TIO, TSI, 2>(p, s);
    default: return launch_r<TIO, TSI, 4>(p, s);
  }
}

template <typename TIO>
static cudaError_t launch_si(const BwdParams& p, cudaStream_t s) {
  switch (p.state_in_dtype) {
    case KDA_DTYPE_F32: return launch_k<TIO, float>(p, s);
    case KDA_DTYPE_F16: return launch_k<TIO, __half>(p, s);
    default: return launch_k<TIO, __nv_bfloat16>(p, s);
  }
}

}  // namespace bwd

size_t backward_ckpt_floats(int B, int H, int T, int K, int V) {
  return (size_t)B * H * ((T + bwd::CK - 1) / bwd::CK) * K * V;
}

cudaError_t launch_backward(const BwdParams& p, cudaStream_t s) {
  switch (p.io_dtype) {
    case KDA_DTYPE_F32: return bwd::launch_si<float>(p, s);
    case KDA_DTYPE_F16: return bwd::launch_si<__half>(p, s);
    default: return bwd::launch_si<__nv_bfloat16>(p, s);
  }
}

}  // namespace kda
