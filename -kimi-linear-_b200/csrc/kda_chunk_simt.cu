// kda_chunk_simt.cu -- chunkwise KDA on CUDA cores (fp32 arithmetic).
//
// Replaces kimi_linear/kda.py:58-185 (kda_chunkwise) for every shape and dtype
// the tensor-core kernel does not take: fp32 inputs (parity 1e-5, which TF32 or
// bf16 operands cannot meet), K or V outside the tensor-core tile, and small
// problems.  All arithmetic is fp32.
//
// One CTA owns (batch b, head h, a tile of VT value columns) and walks the
// sequence in chunks of CC rows.  The algorithm is the reference's, per chunk
// (gc = within-chunk cumulative log decay, kda.py:129):
//   L[c,i]    = beta_c sum_k k_ck k_ik exp(gc_ck - gc_ik)   i < c  (kda.py:159-165)
//   Aout[c,i] = sum_k qs_ck k_ik exp(gc_ck - gc_ik)          i <= c (kda.py:166-168)
//   M = (I + L)^-1 Diag(beta)                                      (kda.py:170-171)
//   W = M (exp(gc) * K),  U = M V                                  (kda.py:172-173)
//   P = U - W S                                                    (kda.py:177)
//   O = (qs * exp(gc)) S + Aout P                                  (kda.py:178)
//   S = exp(gc_last) * S + (exp(gc_last - gc) * K)^T P             (kda.py:179-182)
// The chunk length CC is internal: the chunkwise recurrence is exact for any
// partition of the sequence, so results equal the reference's to fp32
// rounding whatever chunk_size it was called with.  Rows past T are padded
// with k = q = v = g = beta = 0, which leaves the state unchanged.
#include <type_traits>

#include "kda_internal.cuh"

namespace kda {

constexpr int kSimtCC = 32;    // rows per internal chunk (= warp width)
constexpr int kSimtVT = 32;    // value columns per CTA
constexpr int kSimtThreads = 256;

struct SimtSmem {
  int KP, CP, VP;
  size_t oQ, oK, oG, oW, oL, oM, oA, oV, oU, oS, oBeta, oDC, total;
  __host__ __device__ SimtSmem(int K) {
    KP = K + 1; CP = kSimtCC + 1; VP = kSimtVT + 1;
    size_t o = 0;
    oQ = o; o += (size_t)kSimtCC * KP;
    oK = o; o += (size_t)kSimtCC * KP;
    oG = o; o += (size_t)kSimtCC * KP;
    oW = o; o += (size_t)kSimtCC * KP;
    oL = o; o += (size_t)kSimtCC * CP;
    oM = o; o += (size_t)kSimtCC * CP;
    oA = o; o += (size_t)kSimtCC * CP;
    oV = o; o += (size_t)kSimtCC * VP;
    oU = o; o += (size_t)kSimtCC * VP;
    oS = o; o += (size_t)K * VP;
    oBeta = o; o += kSimtCC;
    oDC = o; o += K;
    total = o * sizeof(float);
  }
};

template <typename TIO, typename TSI, typename TSO, bool PRECISE>
__global__ void __launch_bounds__(kSimtThreads)
chunk_simt_kernel(const ChunkParams p) {
  constexpr int CC = kSimtCC, VT = kSimtVT, NTH = kSimtThreads;
  extern __shared__ float smem[];
  const int K = p.K, V = p.V, T = p.T;
  const SimtSmem L(K);
  const int KP = L.KP, CP = L.CP, VP = L.VP;
  float* sQ = smem + L.oQ;  float* sK = smem + L.oK;  float* sG = smem + L.oG;
  float* sW = smem + L.oW;  float* sL = smem + L.oL;  float* sM = smem + L.oM;
  float* sA = smem + L.oA;  float* sV = smem + L.oV;  float* sU = smem + L.oU;
  float* sS = smem + L.oS;  float* sBeta = smem + L.oBeta;  float* sDC = smem + L.oDC;

  const int tid = threadIdx.x;
  const int b = blockIdx.z, h = blockIdx.y;
  const int v0 = blockIdx.x * VT;

  const TIO* qb = static_cast<const TIO*>(p.q) + b * p.q_s[0] + h * p.q_s[2];
  const TIO* kb = static_cast<const TIO*>(p.k) + b * p.k_s[0] + h * p.k_s[2];
  const TIO* vb = static_cast<const TIO*>(p.v) + b * p.v_s[0] + h * p.v_s[2];
  const float* gb = p.g + b * p.g_s[0] + h * p.g_s[2];
  const float* bb = p.beta + b * p.b_s[0] + h * p.b_s[2];
  TIO* ob = static_cast<TIO*>(p.o) + b * p.o_s[0] + h * p.o_s[2];

  // ---- initial state tile ---------------------------------------------------
  for (int idx = tid; idx < K * VT; idx += NTH) {
    const int i = idx / VT, j = idx % VT;
    float s = 0.f;
    if (p.state_in != nullptr && v0 + j < V)
      s = ld(static_cast<const TSI*>(p.state_in) + b * p.si_s[0] + h * p.si_s[1] +
             (int64_t)i * p.si_s[2] + v0 + j);
    sS[i * VP + j] = s;
  }

  const int nchunks = (T + CC - 1) / CC;
  for (int n = 0; n < nchunks; ++n) {
    const int t0 = n * CC;
    // ---- 1. load the chunk (zero padding past T) ----------------------------
    for (int idx = tid; idx < CC * K; idx += NTH) {
      const int c = idx / K, kk = idx % K;
      const int t = t0 + c;
      float qv = 0.f, kv = 0.f, gv = 0.f;
      if (t < T) {
        qv = ld(qb + (int64_t)t * p.q_s[1] + kk) * p.scale;
        kv = ld(kb + (int64_t)t * p.k_s[1] + kk);
        gv = gb[(int64_t)t * p.g_s[1] + kk];
      }
      sQ[c * KP + kk] = qv; sK[c * KP + kk] = kv; sG[c * KP + kk] = gv;
    }
    for (int idx = tid; idx < CC * VT; idx += NTH) {
      const int c = idx / VT, j = idx % VT;
      const int t = t0 + c;
      sV[c * VP + j] = (t < T && v0 + j < V) ? ld(vb + (int64_t)t * p.v_s[1] + v0 + j) : 0.f;
    }
    if (tid < CC) sBeta[tid] = (t0 + tid < T) ? bb[(int64_t)(t0 + tid) * p.b_s[1]] : 0.f;
    __syncthreads();

    // ---- 2. within-chunk cumulative decay gc (kda.py:129) -------------------
    for (int kk = tid; kk < K; kk += NTH) {
      float run = 0.f;
      for (int c = 0; c < CC; ++c) {
        run += sG[c * KP + kk];
        sG[c * KP + kk] = run;
      }
      sDC[kk] = dexp<PRECISE>(run);
    }
    __syncthreads();

    // ---- 3. decay-weighted Gram L and Aout, per pair (kda.py:159-168) -------
    {
      const int i = tid % CC;
      for (int c = tid / CC; c < CC; c += NTH / CC) {
        float kk_sum = 0.f, qk_sum = 0.f;
        if (i <= c) {
          const float* kc = sK + c * KP; const float* qc = sQ + c * KP;
          const float* gc = sG + c * KP; const float* ki = sK + i * KP;
          const float* gi = sG + i * KP;
          for (int kk = 0; kk < K; ++kk) {
            const float d = dexp<PRECISE>(gc[kk] - gi[kk]) * ki[kk];
            kk_sum = fmaf(kc[kk], d, kk_sum);
            qk_sum = fmaf(qc[kk], d, qk_sum);
          }
        }
        sL[c * CP + i] = (i < c) ? sBeta[c] * kk_sum : 0.f;
        sA[c * CP + i] = (i <= c) ? qk_sum : 0.f;
      }
    }
    __syncthreads();

    // ---- 4. decayed operands: Qbar, Ktilde (in sG), Kbar (in sK) -----------
    for (int idx = tid; idx < CC * K; idx += NTH) {
      const int c = idx / K, kk = idx % K;
      const float gam = sG[c * KP + kk];
      const float gl = sG[(CC - 1) * KP + kk];
      const float e = dexp<PRECISE>(gam);
      const float kv = sK[c * KP + kk];
      sQ[c * KP + kk] *= e;                              // (q * scale) exp(gc)
      sK[c * KP + kk] = kv * dexp<PRECISE>(gl - gam);    // exp(gc_last - gc) k
      // Ktilde goes to sW (free until W is formed): gc of the last row must
      // stay readable by every thread during this pass
      sW[c * KP + kk] = kv * e;                          // exp(gc) k
    }
    // ---- 5. M = (I + L)^-1 Diag(beta) by forward substitution (warp 0) ----
    if (tid < 32) {
      const int j = tid;                 // this lane's column of (I + L)^-1
      float x[CC];
#pragma unroll
      for (int c = 0; c < CC; ++c) {
        float acc = (c == j) ? 1.f : 0.f;
#pragma unroll
        for (int i = 0; i < c; ++i) acc = fmaf(-sL[c * CP + i], x[i], acc);
        x[c] = acc;
      }
      const float bj = sBeta[j];
#pragma unroll
      for (int c = 0; c < CC; ++c) sM[c * CP + j] = x[c] * bj;
    }
    __syncthreads();

    // ---- 6. W = M Ktilde (into sG: gc is dead), U = M V (kda.py:172-173) ----
    for (int idx = tid; idx < CC * K; idx += NTH) {
      const int c = idx / K, kk = idx % K;
      float acc = 0.f;
      for (int i = 0; i <= c; ++i) acc = fmaf(sM[c * CP + i], sW[i * KP + kk], acc);
      sG[c * KP + kk] = acc;
    }
    for (int idx = tid; idx < CC * VT; idx += NTH) {
      const int c = idx / VT, j = idx % VT;
      float acc = 0.f;
      for (int i = 0; i <= c; ++i) acc = fmaf(sM[c * CP + i], sV[i * VP + j], acc);
      sU[c * VP + j] = acc;
    }
    __syncthreads();

    // ---- 7. P = U - W S  (stored over V) (kda.py:177) ----------------------
    for (int idx = tid; idx < CC * VT; idx += NTH) {
      const int c = idx / VT, j = idx % VT;
      float acc = sU[c * VP + j];
      for (int kk = 0; kk < K; ++kk) acc = fmaf(-sG[c * KP + kk], sS[kk * VP + j], acc);
      sV[c * VP + j] = acc;
    }
    __syncthreads();

    // ---- 8. O = Qbar S + Aout P (kda.py:178) --------------------------------
    for (int idx = tid; idx < CC * VT; idx += NTH) {
      const int c = idx / VT, j = idx % VT;
      float acc = 0.f;
      for (int kk = 0; kk < K; ++kk) acc = fmaf(sQ[c * KP + kk], sS[kk * VP + j], acc);
      for (int i = 0; i <= c; ++i) acc = fmaf(sA[c * CP + i], sV[i * VP + j], acc);
      const int t = t0 + c;
      if (t < T && v0 + j < V) st(ob + (int64_t)t * p.o_s[1] + v0 + j, acc);
    }
    __syncthreads();

    // ---- 9. S = exp(gc_last) S + Kbar^T P (kda.py:179-182) ------------------
    for (int idx = tid; idx < K * VT; idx += NTH) {
      const int kk = idx / VT, j = idx % VT;
      float acc = sDC[kk] * sS[kk * VP + j];
      for (int c = 0; c < CC; ++c) acc = fmaf(sK[c * KP + kk], sV[c * VP + j], acc);
      sS[kk * VP + j] = acc;
    }
    __syncthreads();
  }

  // ---- final state ------------------------------------------------------------
  for (int idx = tid; idx < K * VT; idx += NTH) {
    const int i = idx / VT, j = idx % VT;
    if (v0 + j < V)
      st(static_cast<TSO*>(p.state_out) + b * p.so_s[0] + h * p.so_s[1] +
             (int64_t)i * p.so_s[2] + v0 + j,
         sS[i * VP + j]);
  }
}

// ---------------------------------------------------------------------------
template <typename TIO, typename TSI, typename TSO>
static cudaError_t launch_simt3(const ChunkParams& p, cudaStream_t s) {
  const SimtSmem L(p.K);
  constexpr bool PRECISE = std::is_same<TIO, float>::value;
  auto kern = chunk_simt_kernel<TIO, TSI, TSO, PRECISE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)L.total);
  if (e != cudaSuccess) return e;
  dim3 grid((p.V + kSimtVT - 1) / kSimtVT, p.H, p.B);
  kern<<<grid, kSimtThreads, L.total, s>>>(p);
  return cudaGetLastError();
}

template <typename TIO, typename TSI>
static cudaError_t launch_simt2(const ChunkParams& p, cudaStream_t s) {
  switch (p.state_out_dtype) {
    case KDA_DTYPE_F32: return launch_simt3<TIO, TSI, float>(p, s);
    case KDA_DTYPE_F16: return launch_simt3<TIO, TSI, __half>(p, s);
    default: return launch_simt3<TIO, TSI, __nv_bfloat16>(p, s);
  }
}

template <typename TIO>
static cudaError_t launch_simt1(const ChunkParams& p, cudaStream_t s) {
  switch (p.state_in_dtype) {
    case KDA_DTYPE_F32: return launch_simt2<TIO, float>(p, s);
    case KDA_DTYPE_F16: return launch_simt2<TIO, __half>(p, s);
    default: return launch_simt2<TIO, __nv_bfloat16>(p, s);
  }
}

size_t chunk_simt_smem_bytes(int K) { return SimtSmem(K).total; }

cudaError_t launch_chunk_simt(const ChunkParams& p, cudaStream_t s) {
  switch (p.io_dtype) {
    case KDA_DTYPE_F32: return launch_simt1<float>(p, s);
    case KDA_DTYPE_F16: return launch_simt1<__half>(p, s);
    default: return launch_simt1<__nv_bfloat16>(p, s);
  }
}

}  // namespace kda
