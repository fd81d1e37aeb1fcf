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
// Two kernels, one CTA of four warps per (b, h, 16-column tile of V).  A warp
// owns 4 adjacent value columns and all K rows (lane i: rows i, i+32, ...), so
// the two reductions over K on the chain (a_t in a forward step, du in a
// reverse step) are warp shuffles: the sequential steps never wait at a block
// barrier.
//  * checkpoint_kernel runs the recurrence forward and stores the state tile
//    before every 64-step chunk (fp32);
//  * backward_kernel walks the chunks backwards: it reruns a chunk from its
//    checkpoint keeping every 8th state, then per 8-step block reruns the
//    block keeping each step's S_{t-1}, u_t and v_t - a_t, and applies the
//    reverse steps above.  State copies are lane-private (each lane stores and
//    reloads only its own elements); u and v - a are per warp.
// dq, dk, dg and dbeta sum over the V columns: the four warps' per-row sums of
// a block of steps meet in shared memory once per block (one barrier pair per
// 8 steps, off the chain), and each column tile writes its partial sums,
// added up afterwards over the V/16 tiles.
#include "kda_internal.cuh"

namespace kda {
namespace bwd {

constexpr int NW = 4;              // warps per CTA, 4 value columns each
constexpr int NTH = 32 * NW;
constexpr int VT = 4 * NW;         // 16 columns per tile
constexpr int CK = 64;             // checkpoint interval (steps)
constexpr int SB = 8;              // sub-checkpoint interval inside a chunk

// per-step vectors of step t for this lane: q', k, alpha of its rows, v and
// dO of its warp's columns and beta.  Every sequential loop below issues the
// loads of step t+1 (or t-1) as raw values (StepRaw: no arithmetic on them,
// so nothing waits for them) while it computes step t, and converts them
// (cook) when that step comes.
template <typename TIO, int R>
struct StepIn {
  float q[R], k[R], al[R], v[4], dO[4], beta;
};
template <typename TIO, int R>
struct StepRaw {
  TIO q[R], k[R], v[4], dO[4];
  float g[R], beta;
};

template <typename TIO, int R>
__device__ __forceinline__ void load_step(const BwdParams& p, int b, int h, int t, int lane,
                                          int col0, StepRaw<TIO, R>& s, bool with_dout = false) {
  const TIO* qb = static_cast<const TIO*>(p.q) + b * p.q_s[0] + (int64_t)t * p.q_s[1] + h * p.q_s[2];
  const TIO* kb = static_cast<const TIO*>(p.k) + b * p.k_s[0] + (int64_t)t * p.k_s[1] + h * p.k_s[2];
  const TIO* vb = static_cast<const TIO*>(p.v) + b * p.v_s[0] + (int64_t)t * p.v_s[1] + h * p.v_s[2];
  const float* gb = p.g + b * p.g_s[0] + (int64_t)t * p.g_s[1] + h * p.g_s[2];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane + 32 * r;
    s.q[r] = qb[i];
    s.k[r] = kb[i];
    s.g[r] = gb[i];
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) s.v[c] = vb[col0 + c];
  s.beta = p.beta[b * p.b_s[0] + (int64_t)t * p.b_s[1] + h * p.b_s[2]];
  if (with_dout) {
    const TIO* dob = static_cast<const TIO*>(p.dout) + b * p.do_s[0] + (int64_t)t * p.do_s[1] +
                     h * p.do_s[2];
#pragma unroll
    for (int c = 0; c < 4; ++c) s.dO[c] = dob[col0 + c];
  }
}

template <typename TIO, int R>
__device__ __forceinline__ StepIn<TIO, R> cook(const StepRaw<TIO, R>& r, float scale,
                                               bool with_dout = false) {
  StepIn<TIO, R> s;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    s.q[i] = ld(&r.q[i]) * scale;
    s.k[i] = ld(&r.k[i]);
    s.al[i] = expf(r.g[i]);
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    s.v[c] = ld(&r.v[c]);
    s.dO[c] = with_dout ? ld(&r.dO[c]) : 0.f;
  }
  s.beta = r.beta;
  return s;
}

// sum over the K rows (the 32 lanes) of per-column values x[4]; every lane
// gets the totals
__device__ __forceinline__ void warp_sum4(float (&x)[4]) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int c = 0; c < 4; ++c) x[c] += __shfl_xor_sync(0xffffffffu, x[c], off);
}

// one forward step on the state tile; returns u and v - a (warp-uniform)
template <typename TIO, int R>
__device__ __forceinline__ void fwd_step(float (&S)[R][4], const StepIn<TIO, R>& s,
                                         float (&u)[4], float (&vma)[4]) {
  float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      S[r][c] *= s.al[r];
      a[c] = fmaf(s.k[r], S[r][c], a[c]);
    }
  warp_sum4(a);
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
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.z, h = blockIdx.y;
  const int col0 = blockIdx.x * VT + 4 * warp;
  const int NC = (p.T + CK - 1) / CK;
  float S[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane + 32 * r;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      S[r][c] = p.state_in ? ld(static_cast<const TSI*>(p.state_in) + b * p.si_s[0] +
                                h * p.si_s[1] + (int64_t)i * p.si_s[2] + col0 + c)
                           : 0.f;
  }
  float* ck = p.ckpt + ((size_t)(b * p.H + h) * NC) * p.K * p.V;
  StepRaw<TIO, R> cur, nxt;
  load_step<TIO, R>(p, b, h, 0, lane, col0, cur);
  for (int t = 0; t < p.T; ++t) {
    load_step<TIO, R>(p, b, h, min(t + 1, p.T - 1), lane, col0, nxt);
    if (t % CK == 0) {
      float* dst = ck + (size_t)(t / CK) * p.K * p.V;
#pragma unroll
      for (int r = 0; r < R; ++r)
        *reinterpret_cast<float4*>(dst + (size_t)(lane + 32 * r) * p.V + col0) =
            make_float4(S[r][0], S[r][1], S[r][2], S[r][3]);
    }
    float u[4], vma[4];
    fwd_step<TIO, R>(S, cook(cur, p.scale), u, vma);
    cur = nxt;
  }
}

// dynamic shared memory of backward_kernel (floats)
template <int R>
struct BwdSmem {
  static constexpr int SUBCK = SB * R * 4 * NTH;     // lane-private sub-checkpoints
  static constexpr int SPREV = SB * R * 4 * NTH;     // lane-private S_{t-1} of a block
  static constexpr int UV = SB * NW * 4;             // u (and v - a) per step and warp
  static constexpr int OUT = SB * 3 * NW * 32 * R;   // per-warp row sums of dq', dk, dg
  static constexpr int OUTB = SB * NW;               // per-warp dbeta
  static constexpr int FLOATS = SUBCK + SPREV + 2 * UV + OUT + OUTB;
  static constexpr size_t BYTES = (size_t)FLOATS * sizeof(float);
};

template <typename TIO, int R>
__global__ void __launch_bounds__(NTH, 1)
backward_kernel(const BwdParams p) {
  using L = BwdSmem<R>;
  extern __shared__ __align__(16) float smem[];
  float* subck = smem;                 // [SB][R*4][NTH], element e of thread tid at e*NTH + tid
  float* sprev = subck + L::SUBCK;     // [SB][R*4][NTH]
  float* su = sprev + L::SPREV;        // [SB][NW][4]
  float* svma = su + L::UV;            // [SB][NW][4]
  float* sout = svma + L::UV;          // [SB][3][NW][32 R]: dq', dk, dg row sums per warp
  float* soutb = sout + L::OUT;        // [SB][NW]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.z, h = blockIdx.y, vt = blockIdx.x;
  const int col0 = vt * VT + 4 * warp;
  const int T = p.T, K = p.K, V = p.V;
  const int NC = (T + CK - 1) / CK;
  const float* ck = p.ckpt + ((size_t)(b * p.H + h) * NC) * K * V;

  // dS starts as the gradient of the returned state (zero when unused)
  float dS[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane + 32 * r;
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

  for (int n = NC - 1; n >= 0; --n) {
    const int t0 = n * CK, t1 = min(T, t0 + CK);
    // rerun the chunk from its checkpoint, keeping every SB-th state
    float S[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float4 x = *reinterpret_cast<const float4*>(ck + (size_t)n * K * V +
                                                        (size_t)(lane + 32 * r) * V + col0);
      S[r][0] = x.x; S[r][1] = x.y; S[r][2] = x.z; S[r][3] = x.w;
    }
    {
      StepRaw<TIO, R> cur, nxt;
      load_step<TIO, R>(p, b, h, t0, lane, col0, cur);
      for (int t = t0; t < t1; ++t) {
        if ((t - t0) % SB == 0) {
          float* d = subck + (size_t)((t - t0) / SB) * R * 4 * NTH;
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) d[(r * 4 + c) * NTH + tid] = S[r][c];
        }
        if (t + 1 < t1) {     // the chunk's last state is not needed
          load_step<TIO, R>(p, b, h, t + 1, lane, col0, nxt);
          float u[4], vma[4];
          fwd_step<TIO, R>(S, cook(cur, p.scale), u, vma);
          cur = nxt;
        }
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
      StepRaw<TIO, R> cur, nxt;
      load_step<TIO, R>(p, b, h, ts, lane, col0, cur);
      for (int t = ts; t < te; ++t) {   // rerun: keep S_{t-1}, u_t, v_t - a_t
        load_step<TIO, R>(p, b, h, min(t + 1, te - 1), lane, col0, nxt);
        float* d = sprev + (size_t)(t - ts) * R * 4 * NTH;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) d[(r * 4 + c) * NTH + tid] = S[r][c];
        float u[4], vma[4];
        fwd_step<TIO, R>(S, cook(cur, p.scale), u, vma);
        if (lane == 0) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            su[((t - ts) * NW + warp) * 4 + c] = u[c];
            svma[((t - ts) * NW + warp) * 4 + c] = vma[c];
          }
        }
        cur = nxt;
      }
      __syncwarp();
      load_step<TIO, R>(p, b, h, te - 1, lane, col0, cur, true);
      for (int t = te - 1; t >= ts; --t) {   // reverse steps
        load_step<TIO, R>(p, b, h, max(t - 1, ts), lane, col0, nxt, true);
        const StepIn<TIO, R> s = cook(cur, p.scale, true);
        const int j = t - ts;
        float u[4], vma[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          u[c] = su[(j * NW + warp) * 4 + c];
          vma[c] = svma[(j * NW + warp) * 4 + c];
        }
        const float* d = sprev + (size_t)j * R * 4 * NTH;
        float St[R][4];                       // alpha (.) S_{t-1}
        float dqp[R], du[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float acc = 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            St[r][c] = s.al[r] * d[(r * 4 + c) * NTH + tid];
            const float Snew = fmaf(s.k[r], u[c], St[r][c]);   // S_t
            acc = fmaf(Snew, s.dO[c], acc);
            dS[r][c] = fmaf(s.q[r], s.dO[c], dS[r][c]);
            du[c] = fmaf(dS[r][c], s.k[r], du[c]);
          }
          dqp[r] = acc;
        }
        warp_sum4(du);
        float dbp = 0.f, da[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          dbp = fmaf(du[c], vma[c], dbp);
          da[c] = -s.beta * du[c];
        }
        if (lane < 4) {
          const float duc = lane == 0 ? du[0] : lane == 1 ? du[1] : lane == 2 ? du[2] : du[3];
          p.dv[b * p.dv_s[0] + (int64_t)t * p.dv_s[1] + h * p.dv_s[2] + col0 + lane] =
              s.beta * duc;
        }
        if (lane == 0) soutb[j * NW + warp] = dbp;
        float* so = sout + (size_t)j * 3 * NW * 32 * R;
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
          const int row = lane + 32 * r;
          so[(0 * NW + warp) * 32 * R + row] = dqp[r];
          so[(1 * NW + warp) * 32 * R + row] = dkp;
          so[(2 * NW + warp) * 32 * R + row] = dgp;
        }
        cur = nxt;
      }
      // the block's row sums over the four warps (16 columns) -> partial outputs
      __syncthreads();
      for (int idx = tid; idx < (te - ts) * K; idx += NTH) {
        const int j = idx / K, row = idx - j * K;
        const float* so = sout + (size_t)j * 3 * NW * 32 * R;
        float q1 = 0.f, k1 = 0.f, g1 = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          q1 += so[(0 * NW + w) * 32 * R + row];
          k1 += so[(1 * NW + w) * 32 * R + row];
          g1 += so[(2 * NW + w) * 32 * R + row];
        }
        const size_t at = (((size_t)b * T + ts + j) * p.H + h) * K + row;
        dq_p[at] = q1 * p.scale;
        dk_p[at] = k1;
        dg_p[at] = g1;
      }
      if (tid < te - ts) {
        float s1 = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) s1 += soutb[tid * NW + w];
        db_p[((size_t)b * T + ts + tid) * p.H + h] = s1;
      }
      __syncthreads();
    }
  }
  // gradient of the initial state
  if (p.dstate_in != nullptr) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float* dst = p.dstate_in + b * p.dsi_s[0] + h * p.dsi_s[1] +
                   (int64_t)(lane + 32 * r) * p.dsi_s[2] + col0;
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
  const size_t smem = BwdSmem<R>::BYTES;
  e = cudaFuncSetAttribute(backward_kernel<TIO, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
  if (e != cudaSuccess) return e;
  backward_kernel<TIO, R><<<grid, NTH, smem, s>>>(p);
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

// the token-serial kernels need one state per 64-step chunk; the chunkwise
// path (V <= 128) needs its per-chunk records, which include those states
size_t backward_ckpt_floats(int B, int H, int T, int K, int V) {
  const size_t serial = (size_t)B * H * ((T + bwd::CK - 1) / bwd::CK) * K * V;
  const size_t chunk = V <= 128 ? backward_chunk_ws_floats(B, H, T, K, V) : 0;
  return serial > chunk ? serial : chunk;
}

namespace bwd {
// dq, dk (io dtype), dg, dbeta (fp32) = sums over the V/16 column tiles of the
// partials [vt][b][t][h][k] and [vt][b][t][h]; a thread sums four consecutive
// k of one (b, t, h) in tile order (deterministic), and (k4 == 0) its dbeta
template <typename TIO>
__global__ void __launch_bounds__(256)
reduce_kernel(const BwdParams p) {
  const int K4 = p.K >> 2, nvt = p.V >> 4;
  const size_t rows = (size_t)p.B * p.T * p.H;
  const size_t n = rows * p.K;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * K4;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / K4;
    const int k = (int)(i - row * K4) * 4;
    const int h = (int)(row % p.H);
    const size_t bt = row / p.H;
    const int t = (int)(bt % p.T), b = (int)(bt / p.T);
    float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f), k4 = q4, g4 = q4;
    float db = 0.f;
    for (int vt = 0; vt < nvt; ++vt) {
      const size_t o = vt * n + row * p.K + k;
      const float4 a = *reinterpret_cast<const float4*>(p.dq_part + o);
      const float4 c = *reinterpret_cast<const float4*>(p.dk_part + o);
      const float4 e = *reinterpret_cast<const float4*>(p.dg_part + o);
      q4.x += a.x; q4.y += a.y; q4.z += a.z; q4.w += a.w;
      k4.x += c.x; k4.y += c.y; k4.z += c.z; k4.w += c.w;
      g4.x += e.x; g4.y += e.y; g4.z += e.z; g4.w += e.w;
      if (k == 0) db += p.dbeta_part[vt * rows + row];
    }
    const float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
    TIO* dq = static_cast<TIO*>(p.dq) + b * p.dq_s[0] + (int64_t)t * p.dq_s[1] + h * p.dq_s[2] + k;
    TIO* dk = static_cast<TIO*>(p.dk) + b * p.dk_s[0] + (int64_t)t * p.dk_s[1] + h * p.dk_s[2] + k;
    float* dg = p.dg + b * p.dg_s[0] + (int64_t)t * p.dg_s[1] + h * p.dg_s[2] + k;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      st(dq + j, qv[j]);
      st(dk + j, kv[j]);
    }
    dg[0] = g4.x; dg[1] = g4.y; dg[2] = g4.z; dg[3] = g4.w;
    if (k == 0) p.dbeta[b * p.dbeta_s[0] + (int64_t)t * p.dbeta_s[1] + h * p.dbeta_s[2]] = db;
  }
}

template <typename TIO>
cudaError_t launch_reduce(const BwdParams& p, cudaStream_t s) {
  const size_t work = (size_t)p.B * p.T * p.H * (p.K >> 2);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t want = (work + 255) / 256, cap = (size_t)sms * 8;
  reduce_kernel<TIO><<<(unsigned)(want < cap ? want : cap), 256, 0, s>>>(p);
  return cudaGetLastError();
}
}  // namespace bwd

cudaError_t launch_backward_reduce(const BwdParams& p, cudaStream_t s) {
  switch (p.io_dtype) {
    case KDA_DTYPE_F32: return bwd::launch_reduce<float>(p, s);
    case KDA_DTYPE_F16: return bwd::launch_reduce<__half>(p, s);
    default: return bwd::launch_reduce<__nv_bfloat16>(p, s);
  }
}

cudaError_t launch_backward(const BwdParams& p, cudaStream_t s) {
  switch (p.io_dtype) {
    case KDA_DTYPE_F32: return bwd::launch_si<float>(p, s);
    case KDA_DTYPE_F16: return bwd::launch_si<__half>(p, s);
    default: return bwd::launch_si<__nv_bfloat16>(p, s);
  }
}

}  // namespace kda
