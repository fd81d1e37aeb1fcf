// kda_recurrent.cu -- token-recurrent KDA (paper Eq. 1) for sm_100a.
//
// Replaces kimi_linear/kda.py:188-219 (kda_recurrent).  Per token t of one
// (batch b, head h) the reference computes, all in fp32:
//     S <- Diag(exp g_t) S                       (kda.py:208-209)
//     S <- S - beta_t k_t (k_t^T S)              (kda.py:212-213)
//     S <- S + beta_t k_t v_t^T                  (kda.py:214)
//     o_t = S^T (q_t * K^-0.5)                   (kda.py:199,216)
// which is S' = A S + k u^T with A = Diag(alpha), u = beta (v - k^T A S) and
// o = (A S)^T q + (q.k) u.  Both projections k^T(AS) and q^T(AS) are reduced in
// ONE pass over the state, so each step needs a single cross-thread reduction.
//
// Layout: the state [K, V] of a head is split into column tiles of VT = 4*CT
// columns (one CTA each).  A thread owns 4 adjacent columns (one 16-byte fp32
// vector per row) of R rows (rows rg, rg + RG, ...).  The tile stays in
// registers across all T steps: HBM sees the state read once and written once
// per launch, which is the whole cost of a decode step (T = 1).
#include "kda_internal.cuh"
#include "tc_ptx.cuh"

namespace kda {

// FULL: the launch guarantees K == RG * R, V % VT == 0, a state_in, and
// 16-byte-aligned state rows in and out, so every row / column guard and the
// scalar fallbacks drop out (the configuration of every model head, K = V = 128).
template <int NTH, int CT, int R, bool FULL, typename TIO, typename TSI, typename TSO>
__global__ void __launch_bounds__(NTH, FULL ? 1024 / NTH : 1)
recurrent_kernel(const RecParams p) {
  constexpr int RG = NTH / CT;   // row groups
  constexpr int VT = 4 * CT;     // columns per CTA
  constexpr int NW = NTH / 32;
  static_assert(RG * CT == NTH, "CT must divide 128");
  static_assert(CT <= 32 && (32 % CT) == 0, "a warp holds whole row groups");

  const int tid = threadIdx.x;
  const int ct = tid % CT;
  const int rg = tid / CT;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int b = blockIdx.z, h = blockIdx.y;
  const int K = p.K, V = p.V;
  const int col0 = blockIdx.x * VT + 4 * ct;        // first of my 4 columns

  // double-buffered per-step vectors: scaled q, k, alpha = exp(g)
  __shared__ float sq[2][kRecMaxK], sk[2][kRecMaxK], sa[2][kRecMaxK];
  __shared__ float sbeta[2];
  // cross-warp partials: [warp][k^T AS (VT) | q^T AS (VT) | q.k, pad]; rows
  // padded to 16 bytes so the final sums read one float4 per warp and vector
  __shared__ __align__(16) float red[NW][2 * VT + 4];

  // Launched as a programmatic dependent.  The state tile is only prefetched
  // into L2 before the previous kernel on the stream completed (a prefetch
  // never returns data, and L2 is where that kernel's writes land, so it is
  // safe even if that kernel writes the state); every load and store waits.
  if (FULL) {
#pragma unroll
    for (int r = 0; r < R; ++r)
      ptx::prefetch_l2(static_cast<const TSI*>(p.state_in) + b * p.si_s[0] + h * p.si_s[1] +
                       (int64_t)(rg + RG * r) * p.si_s[2] + col0);
  }
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();
  float S[R][4];
  // ---- load the state tile (zeros when no initial state) -------------------
  const bool vec_s = p.state_vec;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = rg + RG * r;
#pragma unroll
    for (int c = 0; c < 4; ++c) S[r][c] = 0.f;
    if (FULL || (p.state_in != nullptr && i < K)) {
      const TSI* src = static_cast<const TSI*>(p.state_in) + b * p.si_s[0] + h * p.si_s[1] +
                       (int64_t)i * p.si_s[2];
      if (FULL || (vec_s && col0 + 3 < V)) {
        ld4(src + col0, S[r]);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (col0 + c < V) S[r][c] = ld(src + col0 + c);
      }
    }
  }

  const TIO* qb = static_cast<const TIO*>(p.q) + b * p.q_s[0] + h * p.q_s[2];
  const TIO* kb = static_cast<const TIO*>(p.k) + b * p.k_s[0] + h * p.k_s[2];
  const TIO* vb = static_cast<const TIO*>(p.v) + b * p.v_s[0] + h * p.v_s[2];
  const float* gb = p.g + b * p.g_s[0] + h * p.g_s[2];
  const float* bb = p.beta + b * p.b_s[0] + h * p.b_s[2];
  TIO* ob = static_cast<TIO*>(p.o) + b * p.o_s[0] + h * p.o_s[2];

  for (int t = 0; t < p.T; ++t) {
    const int buf = t & 1;
    // ---- stage 1: per-step vectors into shared memory ----------------------
    for (int i = tid; i < K; i += NTH) {
      sq[buf][i] = ld(qb + (int64_t)t * p.q_s[1] + i) * p.scale;
      sk[buf][i] = ld(kb + (int64_t)t * p.k_s[1] + i);
      sa[buf][i] = expf(gb[(int64_t)t * p.g_s[1] + i]);
    }
    if (tid == 0) sbeta[buf] = bb[(int64_t)t * p.b_s[1]];
    float vv[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      vv[c] = (FULL || col0 + c < V) ? ld(vb + (int64_t)t * p.v_s[1] + col0 + c) : 0.f;
    __syncthreads();

    // ---- stage 2: decay and the two projections over my rows ---------------
    float a[4] = {0.f, 0.f, 0.f, 0.f}, bq[4] = {0.f, 0.f, 0.f, 0.f}, qk = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = rg + RG * r;
      if (FULL || i < K) {
        const float al = sa[buf][i], kk = sk[buf][i], qq = sq[buf][i];
        qk = fmaf(qq, kk, qk);
        // column pairs as two-lane fp32 instructions (each lane rounded like
        // the scalar instruction, so the values are those of the scalar code)
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
          const float2 s2 = __fmul2_rn(make_float2(S[r][c], S[r][c + 1]), make_float2(al, al));
          const float2 a2 = __ffma2_rn(make_float2(kk, kk), s2, make_float2(a[c], a[c + 1]));
          const float2 b2 = __ffma2_rn(make_float2(qq, qq), s2, make_float2(bq[c], bq[c + 1]));
          S[r][c] = s2.x;
          S[r][c + 1] = s2.y;
          a[c] = a2.x;
          a[c + 1] = a2.y;
          bq[c] = b2.x;
          bq[c + 1] = b2.y;
        }
      }
    }
    // reduce across the row groups inside the warp ...
#pragma unroll
    for (int off = CT; off < 32; off <<= 1) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        a[c] += __shfl_xor_sync(0xffffffffu, a[c], off);
        bq[c] += __shfl_xor_sync(0xffffffffu, bq[c], off);
      }
      qk += __shfl_xor_sync(0xffffffffu, qk, off);
    }
    // ... then across warps
    if (lane < CT) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        red[warp][4 * ct + c] = a[c];
        red[warp][VT + 4 * ct + c] = bq[c];
      }
      if (ct == 0) red[warp][2 * VT] = qk;
    }
    __syncthreads();
    float at[4] = {0.f, 0.f, 0.f, 0.f}, bt[4] = {0.f, 0.f, 0.f, 0.f}, qkt = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float4 ra4 = *reinterpret_cast<const float4*>(&red[w][4 * ct]);
      const float4 rb4 = *reinterpret_cast<const float4*>(&red[w][VT + 4 * ct]);
      at[0] += ra4.x; at[1] += ra4.y; at[2] += ra4.z; at[3] += ra4.w;
      bt[0] += rb4.x; bt[1] += rb4.y; bt[2] += rb4.z; bt[3] += rb4.w;
      qkt += red[w][2 * VT];
    }
    const float beta = sbeta[buf];
    float u[4], o[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      u[c] = beta * (vv[c] - at[c]);
      o[c] = clamp_out<TIO>(fmaf(qkt, u[c], bt[c]));
    }
    // ---- stage 3: rank-1 update S += k u^T ---------------------------------
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = rg + RG * r;
      if (FULL || i < K) {
        const float kk = sk[buf][i];
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
          const float2 s2 = __ffma2_rn(make_float2(kk, kk), make_float2(u[c], u[c + 1]),
                                       make_float2(S[r][c], S[r][c + 1]));
          S[r][c] = s2.x;
          S[r][c + 1] = s2.y;
        }
      }
    }
    if (rg == 0) {
      TIO* dst = ob + (int64_t)t * p.o_s[1];
      if (p.o_vec && (FULL || col0 + 3 < V)) {
        st4(dst + col0, o);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (col0 + c < V) st(dst + col0 + c, o[c]);
      }
    }
  }

  // ---- write the final state ------------------------------------------------
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = rg + RG * r;
    if (FULL || i < K) {
      TSO* dst = static_cast<TSO*>(p.state_out) + b * p.so_s[0] + h * p.so_s[1] +
                 (int64_t)i * p.so_s[2];
      if (FULL || (p.state_out_vec && col0 + 3 < V)) {
        st4(dst + col0, S[r]);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (col0 + c < V) st(dst + col0 + c, S[r][c]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// dispatch
// ---------------------------------------------------------------------------
template <int NTH, int CT, int R, bool FULL, typename TIO, typename TSI, typename TSO>
static cudaError_t launch_rec(const RecParams& p, cudaStream_t s) {
  constexpr int VT = 4 * CT;
  dim3 grid((p.V + VT - 1) / VT, p.H, p.B);
  return launch_dependent(recurrent_kernel<NTH, CT, R, FULL, TIO, TSI, TSO>, grid, NTH, 0, s, p);
}

#ifndef KDA_REC_FULL_NTH
#define KDA_REC_FULL_NTH 256
#endif

template <typename TIO, typename TSI, typename TSO>
static cudaError_t launch_rec_k(const RecParams& p, cudaStream_t s) {
  // K = 128 with whole 64-column tiles and vector-aligned states: the guard-free
  // kernel; NTH / 16 row groups of R rows cover the 128 rows exactly.
  if (p.K == 128 && p.V % 64 == 0 && p.state_in != nullptr && p.state_vec &&
      p.state_out_vec) {
    constexpr int NTH = KDA_REC_FULL_NTH;
    return launch_rec<NTH, 16, 128 * 16 / NTH, true, TIO, TSI, TSO>(p, s);
  }
  // (CT, R): RG = 128 / CT row groups of R rows cover K <= RG * R.
  if (p.K <= 32) return launch_rec<128, 8, 2, false, TIO, TSI, TSO>(p, s);
  if (p.K <= 64) return launch_rec<128, 16, 8, false, TIO, TSI, TSO>(p, s);
  if (p.K <= 128) return launch_rec<128, 16, 16, false, TIO, TSI, TSO>(p, s);
  return launch_rec<128, 16, 32, false, TIO, TSI, TSO>(p, s);
}

template <typename TIO, typename TSI>
static cudaError_t launch_rec_so(const RecParams& p, cudaStream_t s) {
  switch (p.state_out_dtype) {
    case KDA_DTYPE_F32: return launch_rec_k<TIO, TSI, float>(p, s);
    case KDA_DTYPE_F16: return launch_rec_k<TIO, TSI, __half>(p, s);
    default: return launch_rec_k<TIO, TSI, __nv_bfloat16>(p, s);
  }
}

template <typename TIO>
static cudaError_t launch_rec_si(const RecParams& p, cudaStream_t s) {
  switch (p.state_in_dtype) {
    case KDA_DTYPE_F32: return launch_rec_so<TIO, float>(p, s);
    case KDA_DTYPE_F16: return launch_rec_so<TIO, __half>(p, s);
    default: return launch_rec_so<TIO, __nv_bfloat16>(p, s);
  }
}

cudaError_t launch_recurrent(const RecParams& p, cudaStream_t s) {
  switch (p.io_dtype) {
    case KDA_DTYPE_F32: return launch_rec_si<float>(p, s);
    case KDA_DTYPE_F16: return launch_rec_si<__half>(p, s);
    default: return launch_rec_si<__nv_bfloat16>(p, s);
  }
}

}  // namespace kda
