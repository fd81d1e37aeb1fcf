// kda_backward_chunk.cu -- chunkwise gradient of the KDA recurrence (sm_100a).
//
// The same gradient as kda_backward.cu (the exact reverse-mode gradient of the
// token recurrence, kimi_linear/kda.py:207-216, which kda_chunkwise,
// kda.py:58-185, computes chunk by chunk), organised by 64-token chunks so
// that all but two short chains run in parallel over (b, h, chunk).
//
// Per chunk (C tokens, per-channel cumulative log decay G_i = sum_{s<=i} g_s,
// Gam_i = exp G_i, GamC = Gam_{C-1}, q' = K^-1/2 q, chunk-start state S):
//   Lraw_ij = sum_c k_ic k_jc exp(G_ic - G_jc)   (j < i)
//   Mq_ij   = sum_c q'_ic k_jc exp(G_ic - G_jc)  (j <= i)
//   Tinv    = (I + Diag(beta) Lraw)^-1           (unit lower triangular)
//   KG = k (.) Gam,  Kbar = k (.) GamC / Gam,  EQ = q' (.) Gam
//   X = KG S,  Z = V - X,  P = Tinv Diag(beta) Z          (pseudo-values)
//   O = EQ S + Mq P,       S_next = Diag(GamC) S + Kbar^T P
// (the WY form of kda.py:170-182).  Reverse mode, given dO and dS_next:
//   dP = Mq^T dO + Kbar dS_next,  dR = Tinv^T dP,  dZ = Diag(beta) dR
//   dS = EQ^T dO + Diag(GamC) dS_next - KG^T dZ
//   dv = dZ,  dbeta_i = dR_i . Z_i + sum_j dL_ij Lraw_ij,  dL = -(dR P^T) (j < i)
//   dMq = dO P^T (j <= i),  dEQ = dO S^T,  dKG = -dZ S^T,  dKbar = P dS_next^T
// and the pair terms of dL, dMq through exp(G_ic - G_jc) give dq', dk and dG
// channel by channel; dg is the reverse cumulative sum of dG within the chunk.
// Tokens past T are zero rows (q = k = v = g = beta = 0 leave the state and
// every gradient unchanged).
//
// Three kernels, fp32 data; every GEMM runs on the tensor cores as 3xTF32
// (x = hi + lo, both exact in tf32; hi*hi + hi*lo + lo*hi, ~fp32 accuracy):
//  * prep_kernel  (b, h, chunk): the pair sums Lraw and Mq as anchored 16-row
//    block GEMMs (exp(G_ic - G_jc) = exp(G_ic - G_ac) exp(G_ac - G_jc) with the
//    anchor a at the start of i's block, each factor within e^-80 .. e^80;
//    channels for which a block is steeper add their exact pair terms
//    separately), Tinv by forward substitution, KG, Kbar, EQ, GamC -- written
//    to the per-chunk record;
//  * chains_kernel, two kinds of CTA in one launch:
//    - forward chain (b, h, 32 state columns): S chunk by chunk (X = KG S,
//      P = Tinv R, S_next = GamC S + Kbar^T P), storing every chunk-start
//      state and the chunk's P and Z;
//    - reverse chain (b, h, 32 columns): dS from the end backwards, storing
//      the gradient of every chunk-end state and dR, writing dv; it needs no
//      S, so it runs at the same time as the forward chain;
//  * grad_kernel  (b, h, chunk): dL, dMq, dEQ, dKG, dKbar from the stored
//    P, dR, states and dO, the pair terms (the same anchored block GEMMs), and
//    dq, dk, dg, dbeta (final sums, no partials over V).
// The GEMMs are warp tiles of mma.sync m16n8k8 over operands in shared memory
// read through (row, k) strides, so no operand needs a transposed copy; row
// strides are padded so that the fragment loads are free of bank conflicts.
#include "kda_internal.cuh"
#include "tc_ptx.cuh"

namespace kda {
namespace bwdc {

constexpr int C = 64;        // chunk length
constexpr int NTH = 256;     // threads of every kernel here
constexpr int NW = NTH / 32;
constexpr int VT = 32;       // state columns per chain CTA

// per-(b, h, chunk) record in the workspace, offsets in floats, every array
// row-major: TINV [C][C], KG, KBAR, EQ [C][K], MQ, LRAW [C][C], GCV [K],
// SN, DSN [K][V], PP, ZZ, DRR [C][V]
struct Rec {
  int K, V;
  __host__ __device__ size_t tinv() const { return 0; }
  __host__ __device__ size_t kg() const { return (size_t)C * C; }
  __host__ __device__ size_t kbar() const { return kg() + (size_t)C * K; }
  __host__ __device__ size_t eq() const { return kbar() + (size_t)C * K; }
  __host__ __device__ size_t mq() const { return eq() + (size_t)C * K; }
  __host__ __device__ size_t lraw() const { return mq() + (size_t)C * C; }
  __host__ __device__ size_t gcv() const { return lraw() + (size_t)C * C; }
  __host__ __device__ size_t sn() const { return gcv() + K; }
  __host__ __device__ size_t dsn() const { return sn() + (size_t)K * V; }
  __host__ __device__ size_t pp() const { return dsn() + (size_t)K * V; }
  __host__ __device__ size_t zz() const { return pp() + (size_t)C * V; }
  __host__ __device__ size_t drr() const { return zz() + (size_t)C * V; }
  __host__ __device__ size_t size() const { return drr() + (size_t)C * V; }
};

__host__ __device__ inline int num_chunks(int T) { return (T + C - 1) / C; }

// 16-byte asynchronous copy global -> shared (L2 only)
__device__ __forceinline__ void cpa16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// n floats (a multiple of 4, 16-byte aligned at both ends) by the whole CTA
__device__ __forceinline__ void cpa_floats(float* dst, const float* src, int n) {
  for (int i = 4 * threadIdx.x; i < n; i += 4 * NTH) cpa16(dst + i, src + i);
}
// rows x cols floats from a row-major global array (row stride gs floats) into
// shared memory with row stride ss; cols a multiple of 4
__device__ __forceinline__ void cpa_rows(float* dst, int ss, const float* src, size_t gs, int rows,
                                         int cols) {
  const int c4 = cols >> 2;
  for (int i = threadIdx.x; i < rows * c4; i += NTH) {
    const int r = i / c4, c = (i - r * c4) * 4;
    cpa16(dst + r * ss + c, src + r * gs + c);
  }
}

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// x ~= hi + lo, both exact in tf32
__device__ __forceinline__ void split3(float x, uint32_t& hi, uint32_t& lo) {
  hi = ptx::f32_to_tf32(x);
  lo = ptx::f32_to_tf32(x - __uint_as_float(hi));
}

// Warp tile acc[mt][nt] (rows m0 + 16 mt, columns n0 + 8 nt) += A B over
// k in [k0, k1) (multiples of 8), 3xTF32.  A(m, k) = A[m * am + k * ak],
// B(k, n) = B[k * bk + n * bn].  Fragment layout of mma.sync m16n8k8 tf32:
// a0..a3 = A(g, t), A(g + 8, t), A(g, t + 4), A(g + 8, t + 4); b0, b1 =
// B(t, g), B(t + 4, g); c0..c3 = C(g, 2t), C(g, 2t + 1), C(g + 8, 2t),
// C(g + 8, 2t + 1), with g = lane / 4, t = lane % 4.
template <int MT, int NT>
__device__ __forceinline__ void wgemm3(float (&acc)[MT][NT][4], const float* A, int am, int ak,
                                       int m0, const float* B, int bk, int bn, int n0, int k0,
                                       int k1, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll 2
  for (int k = k0; k < k1; k += 8) {
    uint32_t ah[MT][4], al[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const float* a = A + (m0 + 16 * mt + g) * am + (k + t) * ak;
      split3(a[0], ah[mt][0], al[mt][0]);
      split3(a[8 * am], ah[mt][1], al[mt][1]);
      split3(a[4 * ak], ah[mt][2], al[mt][2]);
      split3(a[8 * am + 4 * ak], ah[mt][3], al[mt][3]);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float* bp = B + (k + t) * bk + (n0 + 8 * nt + g) * bn;
      uint32_t bh[2], bl[2];
      split3(bp[0], bh[0], bl[0]);
      split3(bp[4 * bk], bh[1], bl[1]);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        ptx::mma_tf32_16x8x8(acc[mt][nt], al[mt], bh);
        ptx::mma_tf32_16x8x8(acc[mt][nt], ah[mt], bl);
        ptx::mma_tf32_16x8x8(acc[mt][nt], ah[mt], bh);
      }
    }
  }
}
// (row, column) of element e of a thread's accumulator tile at (m0, n0 + 8 nt)
__device__ __forceinline__ int acc_row(int m0, int lane, int e) { return m0 + (lane >> 2) + 8 * (e >> 1); }
__device__ __forceinline__ int acc_col(int n0, int nt, int lane, int e) {
  return n0 + 8 * nt + 2 * (lane & 3) + (e & 1);
}
template <int MT, int NT>
__device__ __forceinline__ void zero(float (&acc)[MT][NT][4]) {
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
}


// ---------------------------------------------------------------------------
// prep_kernel: one CTA per (chunk, h, b)
// ---------------------------------------------------------------------------
template <int KD>
struct PrepSmem {
  static constexpr int LD = C + 4;                  // row stride of the [c][i] arrays
  static constexpr int QT = 0;                      // q' transposed [KD][LD]
  static constexpr int KT = QT + KD * LD;           // k transposed
  static constexpr int GT = KT + KD * LD;           // G (natural log) transposed
  // once the pair sums are done the [c][i] arrays are dead: Diag(beta) Lraw
  // and Tinv ([C][C + 1] each) reuse their space (two CTAs fit an SM)
  static constexpr int LS = 0;
  static constexpr int TS = LS + C * (C + 1);
  static constexpr int END = GT + KD * LD > TS + C * (C + 1) ? GT + KD * LD : TS + C * (C + 1);
  static constexpr int BS = END;                    // beta [C]
  static constexpr int STP = BS + C;                // steep-block bits of each channel [KD]
  static constexpr int FLOATS = STP + KD;
  static constexpr size_t BYTES = (size_t)FLOATS * sizeof(float);
};

template <typename TIO, int KD>
__global__ void __launch_bounds__(NTH, 2)
prep_kernel(const BwdParams p, float* __restrict__ ws) {
  using L = PrepSmem<KD>;
  extern __shared__ __align__(16) float sm[];
  float* qT = sm + L::QT;
  float* kT = sm + L::KT;
  float* gT = sm + L::GT;
  float* Ls = sm + L::LS;
  float* Ts = sm + L::TS;
  float* bs = sm + L::BS;
  unsigned* STP = reinterpret_cast<unsigned*>(sm + L::STP);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int NC = num_chunks(p.T);
  const Rec R{KD, p.V};
  float* rec = ws + ((size_t)(b * p.H + h) * NC + n) * R.size();
  const TIO* q = static_cast<const TIO*>(p.q) + b * p.q_s[0] + h * p.q_s[2];
  const TIO* k = static_cast<const TIO*>(p.k) + b * p.k_s[0] + h * p.k_s[2];
  const float* g = p.g + b * p.g_s[0] + h * p.g_s[2];

  // inputs of the chunk, transposed to [channel][row]; rows past T are zero
#pragma unroll 4
  for (int e = tid; e < C * KD; e += NTH) {
    const int i = e / KD, c = e - i * KD;
    const int t = n * C + i;
    const bool ok = t < p.T;
    qT[c * L::LD + i] = ok ? ld(q + (int64_t)t * p.q_s[1] + c) * p.scale : 0.f;
    kT[c * L::LD + i] = ok ? ld(k + (int64_t)t * p.k_s[1] + c) : 0.f;
    gT[c * L::LD + i] = ok ? g[(int64_t)t * p.g_s[1] + c] : 0.f;
  }
  if (tid < C) {
    const int t = n * C + tid;
    bs[tid] = t < p.T ? p.beta[b * p.b_s[0] + (int64_t)t * p.b_s[1] + h * p.b_s[2]] : 0.f;
  }
  __syncthreads();
  if (tid < KD) {                                   // cumulative log decay, fp32
    // and the channel's steep blocks: block I (anchor a = 16 I) is steep when a
    // factor exp(G_i - G_a) (i in I) or exp(G_a - G_j) (j < a + 16) leaves
    // e^-80 .. e^80
    float G = 0.f, runmin = 0.f, ga = 0.f, bmin = 0.f, bmax = 0.f;
    unsigned bits = 0u;
    for (int i = 0; i < C; ++i) {
      G += gT[tid * L::LD + i];
      gT[tid * L::LD + i] = G;
      if ((i & 15) == 0) {
        ga = G;
        bmin = bmax = G;
      }
      bmin = fminf(bmin, G);
      bmax = fmaxf(bmax, G);
      runmin = i == 0 ? G : fminf(runmin, G);
      if ((i & 15) == 15 && (bmin - ga < -80.f || bmax - ga > 80.f || ga - runmin > 80.f))
        bits |= 1u << (i >> 4);
    }
    STP[tid] = bits;
  }
  __syncthreads();

  // KG = k Gam, Kbar = k GamC / Gam, EQ = q' Gam, GamC
#pragma unroll 4
  for (int e = tid; e < C * KD; e += NTH) {
    const int i = e / KD, c = e - i * KD;           // row-major: c fastest
    const float G = gT[c * L::LD + i], Gl = gT[c * L::LD + C - 1];
    const float kv = kT[c * L::LD + i];
    const float gam = expf(G);
    rec[R.kg() + e] = kv * gam;
    rec[R.kbar() + e] = kv * expf(Gl - G);
    rec[R.eq() + e] = qT[c * L::LD + i] * gam;
  }
  if (tid < KD) rec[R.gcv() + tid] = expf(gT[tid * L::LD + C - 1]);

  // pair sums by anchored 16-row blocks (3xTF32 mma.sync): for rows i of
  // block I (anchor a = 16 I), exp(G_ic - G_jc) = exp(G_ic - G_ac) exp(G_ac - G_jc).
  // The 20 tiles (block I, 8 columns) of the lower block triangle go round the
  // warps; A(i, c) = k_ic exp(G_ic - G_ac) (Lraw) and q'_ic exp(G_ic - G_ac)
  // (Mq), B(c, j) = k_jc exp(G_ac - G_jc).  Channels for which block I is steep
  // are left out and added exactly below.
  float* lraw = rec + R.lraw();
  float* mqg = rec + R.mq();
  {
    const int g = lane >> 2, tq = lane & 3;
    for (int q = w; q < 20; q += NW) {
      const int I = q < 2 ? 0 : q < 6 ? 1 : q < 12 ? 2 : 3;
      const int j0 = 8 * (q - (I == 0 ? 0 : I == 1 ? 2 : I == 2 ? 6 : 12));
      const int a = 16 * I;
      float al[4] = {0.f, 0.f, 0.f, 0.f}, am[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
      for (int kc = 0; kc < KD; kc += 8) {
        uint32_t kh[4], kl[4], qh[4], ql[4], bh[2], bl[2];
#pragma unroll
        for (int e = 0; e < 4; ++e) {                // A(i, c): rows a + g (+8), channels kc + tq (+4)
          const int i = a + g + 8 * (e & 1), c = kc + tq + 4 * (e >> 1);
          const bool st = (STP[c] >> I) & 1u;
          const float wa = st ? 0.f : __expf(gT[c * L::LD + i] - gT[c * L::LD + a]);
          split3(kT[c * L::LD + i] * wa, kh[e], kl[e]);
          split3(qT[c * L::LD + i] * wa, qh[e], ql[e]);
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {                // B(c, j): channels kc + tq (+4), column j0 + g
          const int c = kc + tq + 4 * e, j = j0 + g;
          const bool st = (STP[c] >> I) & 1u;
          const float wb = st ? 0.f : __expf(gT[c * L::LD + a] - gT[c * L::LD + j]);
          split3(kT[c * L::LD + j] * wb, bh[e], bl[e]);
        }
        ptx::mma_tf32_16x8x8(al, kl, bh);
        ptx::mma_tf32_16x8x8(al, kh, bl);
        ptx::mma_tf32_16x8x8(al, kh, bh);
        ptx::mma_tf32_16x8x8(am, ql, bh);
        ptx::mma_tf32_16x8x8(am, qh, bl);
        ptx::mma_tf32_16x8x8(am, qh, bh);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(a, lane, e), j = acc_col(j0, 0, lane, e);
        lraw[i * C + j] = j < i ? al[e] : 0.f;
        mqg[i * C + j] = j <= i ? am[e] : 0.f;
      }
    }
    // the rest of each row block (columns past the block) is zero
    for (int e = tid; e < C * C; e += NTH) {
      const int i = e / C, j = e - i * C;
      if (j >= 16 * ((i >> 4) + 1)) {
        lraw[e] = 0.f;
        mqg[e] = 0.f;
      }
    }
  }
  __syncthreads();
  // steep blocks: exact pair terms of the left-out channels (rare)
  for (int x = tid; x < 2 * KD; x += NTH) {
    const int c = x % KD, half = x / KD;
    const unsigned bits = STP[c];
    if (bits == 0u) continue;
    for (int I = 0; I < 4; ++I) {
      if (!((bits >> I) & 1u)) continue;
      for (int i = 16 * I + half; i < 16 * I + 16; i += 2) {
        const float Gi = gT[c * L::LD + i], ki = kT[c * L::LD + i], qi = qT[c * L::LD + i];
        for (int j = 0; j <= i; ++j) {
          const float t = kT[c * L::LD + j] * __expf(Gi - gT[c * L::LD + j]);
          if (j < i) atomicAdd(&lraw[i * C + j], ki * t);
          atomicAdd(&mqg[i * C + j], qi * t);
        }
      }
    }
  }
  __syncthreads();                                  // the [c][i] arrays are dead from here
  for (int e = tid; e < C * (C + 1); e += NTH) Ts[e] = 0.f;
  for (int e = tid; e < C * C; e += NTH) {
    const int i = e / C, j = e - i * C;
    Ls[i * (C + 1) + j] = bs[i] * lraw[e];
  }
  __syncthreads();

  // Tinv = (I + Ls)^-1 by forward substitution, column j by the four lanes
  // 4j .. 4j + 3 (each sums every fourth l), rows in order; a column's rows
  // are written and read only by its own warp
  {
    const int j = tid >> 2, qq = tid & 3;
    for (int i = 0; i < C; ++i) {
      float acc = 0.f;
      for (int l = qq; l < i; l += 4) acc = fmaf(Ls[i * (C + 1) + l], Ts[l * (C + 1) + j], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (qq == 0 && i >= j) Ts[i * (C + 1) + j] = (i == j ? 1.f : 0.f) - acc;
      __syncwarp();
    }
  }
  __syncthreads();
  for (int e = tid; e < C * C; e += NTH) {
    const int i = e / C, j = e - i * C;
    rec[R.tinv() + e] = Ts[i * (C + 1) + j];
  }
}

// ---------------------------------------------------------------------------
// chain kernels: one CTA per (32 state columns, h, b).  Warp tiles: the C x 32
// chunk tiles (X, P, dP, dR) as m-tile w % 4 and n-tiles 2 (w / 4) .. + 1;
// the KD x 32 state tiles as KD / 32 n-tiles of m-tile w / (4 / (KD / 32)).
// ---------------------------------------------------------------------------
constexpr int LDV = VT + 8;                        // [rows][VT] tiles read as B(k, col)

template <int KD>
struct StateTile {
  static constexpr int NT = KD / 32;
  static constexpr int WPM = 4 / NT;               // warps per 16-row m-tile
};


template <int KD>
struct FchainSmem {
  static constexpr int LTI = C + 4;                 // Tinv, read as A(i, l)
  static constexpr int LKG = KD + 4;                // KG, read as A(i, c)
  static constexpr int LKB = KD + 8;                // Kbar, read as A(c, i)
  static constexpr int SS = 0;                      // S tile [KD][LDV]
  static constexpr int RS = SS + KD * LDV;          // R = beta Z [C][LDV]
  static constexpr int PS = RS + C * LDV;           // P [C][LDV]
  static constexpr int ASZ = C * LTI + C * LKG;     // Tinv | KG
  static constexpr int ABUF = PS + C * LDV;         // two of them
  static constexpr int BSZ = C * LKB;               // Kbar
  static constexpr int BBUF = ABUF + 2 * ASZ;       // two of them
  static constexpr int FLOATS = BBUF + 2 * BSZ;
  static constexpr size_t BYTES = (size_t)FLOATS * sizeof(float);
};

template <typename TIO, typename TSI, int KD>
__device__ __forceinline__ void fchain_cta(const BwdParams& p, float* __restrict__ ws, int xt) {
  using L = FchainSmem<KD>;
  using ST = StateTile<KD>;
  extern __shared__ __align__(16) float sm[];
  float* Ss = sm + L::SS;
  float* Rs = sm + L::RS;
  float* Ps = sm + L::PS;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int h = blockIdx.y, b = blockIdx.z;
  const int col0 = xt * VT;
  const int V = p.V;
  const int NC = num_chunks(p.T);
  const Rec R{KD, V};
  float* recs = ws + (size_t)(b * p.H + h) * NC * R.size();
  const TIO* v = static_cast<const TIO*>(p.v) + b * p.v_s[0] + h * p.v_s[2] + col0;
  const float* beta = p.beta + b * p.b_s[0] + h * p.b_s[2];
  const int mX = 16 * (w & 3), nX = 16 * (w >> 2);              // C x 32 tiles
  const int mS = 16 * (w / ST::WPM), nS = 8 * ST::NT * (w % ST::WPM);   // KD x 32

  auto issue = [&](int m) {                         // chunk m's operands into buffer m & 1
    if (m < NC) {
      const float* rec = recs + (size_t)m * R.size();
      float* A = sm + L::ABUF + (m & 1) * L::ASZ;
      cpa_rows(A, L::LTI, rec + R.tinv(), C, C, C);
      cpa_rows(A + C * L::LTI, L::LKG, rec + R.kg(), KD, C, KD);
      cpa_commit();
      cpa_rows(sm + L::BBUF + (m & 1) * L::BSZ, L::LKB, rec + R.kbar(), KD, C, KD);
      cpa_commit();
    } else {
      cpa_commit();
      cpa_commit();
    }
  };
  issue(0);
  issue(1);

  // initial state tile, also chunk 0's start state; columns past V stay zero
  for (int e = tid; e < KD * VT; e += NTH) {
    const int c = e / VT, col = e - c * VT;
    float x = 0.f;
    if (col0 + col < V) {
      if (p.state_in != nullptr)
        x = ld(static_cast<const TSI*>(p.state_in) + b * p.si_s[0] + h * p.si_s[1] +
               (int64_t)c * p.si_s[2] + col0 + col);
      recs[R.sn() + (size_t)c * V + col0 + col] = x;
    }
    Ss[c * LDV + col] = x;
  }

  // per-chunk scalars of this thread, loaded one chunk ahead: v at its X tile
  // positions, beta of its two X rows, GamC of its two state rows
  struct Pre {
    float v[2][4], bt[2], gc[2];
  };
  auto fetch = [&](int m, Pre& f) {
    if (m >= NC) return;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int t = m * C + acc_row(mX, lane, 2 * hh);
      f.bt[hh] = t < p.T ? beta[(int64_t)t * p.b_s[1]] : 0.f;
      f.gc[hh] = recs[(size_t)m * R.size() + R.gcv() + acc_row(mS, lane, 2 * hh)];
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = m * C + acc_row(mX, lane, e), col = acc_col(nX, nt, lane, e);
        f.v[nt][e] = (t < p.T && col0 + col < V) ? ld(v + (int64_t)t * p.v_s[1] + col) : 0.f;
      }
  };
  Pre cur, nxt;
  fetch(0, cur);

  for (int n = 0; n < NC; ++n) {
    float* rec = recs + (size_t)n * R.size();
    const float* Ti = sm + L::ABUF + (n & 1) * L::ASZ;
    const float* Kg = Ti + C * L::LTI;
    const float* Kb = sm + L::BBUF + (n & 1) * L::BSZ;
    fetch(n + 1, nxt);
    cpa_wait<3>();
    __syncthreads();
    float acc[1][2][4];
    // X = KG S; Z = v - X; R = beta Z
    zero(acc);
    wgemm3<1, 2>(acc, Kg, L::LKG, 1, mX, Ss, LDV, 1, nX, 0, KD, lane);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(mX, lane, e), col = acc_col(nX, nt, lane, e);
        const bool cok = col0 + col < V;
        const float z = cok ? cur.v[nt][e] - acc[0][nt][e] : 0.f;
        Rs[i * LDV + col] = cur.bt[e >> 1] * z;
        if (cok) rec[R.zz() + (size_t)i * V + col0 + col] = z;
      }
    __syncthreads();
    // P = Tinv R (Tinv lower triangular: l < mX + 16)
    zero(acc);
    wgemm3<1, 2>(acc, Ti, L::LTI, 1, mX, Rs, LDV, 1, nX, 0, mX + 16, lane);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(mX, lane, e), col = acc_col(nX, nt, lane, e);
        Ps[i * LDV + col] = acc[0][nt][e];
        if (col0 + col < V) rec[R.pp() + (size_t)i * V + col0 + col] = acc[0][nt][e];
      }
    cpa_wait<2>();
    __syncthreads();
    // S_next = Diag(GamC) S + Kbar^T P
    {
      float sa[1][ST::NT][4];
#pragma unroll
      for (int nt = 0; nt < ST::NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = acc_row(mS, lane, e), col = acc_col(nS, nt, lane, e);
          sa[0][nt][e] = cur.gc[e >> 1] * Ss[c * LDV + col];
        }
      wgemm3<1, ST::NT>(sa, Kb, 1, L::LKB, mS, Ps, LDV, 1, nS, 0, C, lane);
#pragma unroll
      for (int nt = 0; nt < ST::NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = acc_row(mS, lane, e), col = acc_col(nS, nt, lane, e);
          Ss[c * LDV + col] = sa[0][nt][e];
          if (n + 1 < NC && col0 + col < V)
            recs[(size_t)(n + 1) * R.size() + R.sn() + (size_t)c * V + col0 + col] = sa[0][nt][e];
        }
    }
    __syncthreads();
    issue(n + 2);
    cur = nxt;
  }
}

template <int KD>
struct BchainSmem {
  static constexpr int LMQ = C + 8;                 // Mq, read as A(i, l) = Mq[l][i]
  static constexpr int LKB = KD + 4;                // Kbar, read as A(i, c)
  static constexpr int LTI = C + 8;                 // Tinv, read as A(i, l) = Tinv[l][i]
  static constexpr int LEQ = KD + 8;                // EQ and KG, read as A(c, i)
  static constexpr int DSS = 0;                     // dS tile [KD][LDV]
  static constexpr int DOS = DSS + KD * LDV;        // dO [C][LDV]
  static constexpr int DPS = DOS + C * LDV;         // dP [C][LDV]
  static constexpr int DZS = DPS + C * LDV;         // -beta dR [C][LDV]
  static constexpr int ABUF = DZS + C * LDV;        // Mq | Kbar | Tinv
  static constexpr int ASZ = C * LMQ + C * LKB + C * LTI;
  static constexpr int BBUF = ABUF + ASZ;           // EQ | KG
  static constexpr int BSZ = 2 * C * LEQ;
  static constexpr int FLOATS = BBUF + BSZ;
  static constexpr size_t BYTES = (size_t)FLOATS * sizeof(float);
};

template <typename TIO, int KD>
__device__ __forceinline__ void bchain_cta(const BwdParams& p, float* __restrict__ ws, int xt) {
  using L = BchainSmem<KD>;
  using ST = StateTile<KD>;
  extern __shared__ __align__(16) float sm[];
  float* dSs = sm + L::DSS;
  float* dOs = sm + L::DOS;
  float* dPs = sm + L::DPS;
  float* dZs = sm + L::DZS;
  const float* Mq = sm + L::ABUF;
  const float* Kb = Mq + C * L::LMQ;
  const float* Ti = Kb + C * L::LKB;
  const float* Eq = sm + L::BBUF;
  const float* Kg = Eq + C * L::LEQ;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int h = blockIdx.y, b = blockIdx.z;
  const int col0 = xt * VT;
  const int V = p.V;
  const int NC = num_chunks(p.T);
  const Rec R{KD, V};
  float* recs = ws + (size_t)(b * p.H + h) * NC * R.size();
  const TIO* dout = static_cast<const TIO*>(p.dout) + b * p.do_s[0] + h * p.do_s[2] + col0;
  float* dv = p.dv + b * p.dv_s[0] + h * p.dv_s[2] + col0;
  const float* beta = p.beta + b * p.b_s[0] + h * p.b_s[2];
  const int mX = 16 * (w & 3), nX = 16 * (w >> 2);
  const int mS = 16 * (w / ST::WPM), nS = 8 * ST::NT * (w % ST::WPM);

  auto issueA = [&](int m) {
    if (m >= 0) {
      const float* rec = recs + (size_t)m * R.size();
      float* A = sm + L::ABUF;
      cpa_rows(A, L::LMQ, rec + R.mq(), C, C, C);
      cpa_rows(A + C * L::LMQ, L::LKB, rec + R.kbar(), KD, C, KD);
      cpa_rows(A + C * L::LMQ + C * L::LKB, L::LTI, rec + R.tinv(), C, C, C);
    }
    cpa_commit();
  };
  auto issueB = [&](int m) {
    if (m >= 0) {
      const float* rec = recs + (size_t)m * R.size();
      cpa_rows(sm + L::BBUF, L::LEQ, rec + R.eq(), KD, C, KD);
      cpa_rows(sm + L::BBUF + C * L::LEQ, L::LEQ, rec + R.kg(), KD, C, KD);
    }
    cpa_commit();
  };
  issueA(NC - 1);
  issueB(NC - 1);

  float ds[1][ST::NT][4];                           // dS at this warp's state tile
#pragma unroll
  for (int nt = 0; nt < ST::NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = acc_row(mS, lane, e), col = acc_col(nS, nt, lane, e);
      ds[0][nt][e] = (p.dstate_out != nullptr && col0 + col < V)
                         ? p.dstate_out[b * p.dso_s[0] + h * p.dso_s[1] +
                                        (int64_t)c * p.dso_s[2] + col0 + col]
                         : 0.f;
      dSs[c * LDV + col] = ds[0][nt][e];
    }

  // per-chunk inputs of this thread, loaded one chunk ahead: its share of the
  // dO tile, beta of its two dP rows, GamC of its two state rows
  constexpr int NDO = C * VT / NTH;
  struct Pre {
    float dO[NDO], bt[2], gc[2];
  };
  auto fetch = [&](int m, Pre& f) {
    if (m < 0) return;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int t = m * C + acc_row(mX, lane, 2 * hh);
      f.bt[hh] = t < p.T ? beta[(int64_t)t * p.b_s[1]] : 0.f;
      f.gc[hh] = recs[(size_t)m * R.size() + R.gcv() + acc_row(mS, lane, 2 * hh)];
    }
#pragma unroll
    for (int q = 0; q < NDO; ++q) {
      const int e = tid + q * NTH, i = e / VT, col = e - i * VT;
      const int t = m * C + i;
      f.dO[q] = (t < p.T && col0 + col < V) ? ld(dout + (int64_t)t * p.do_s[1] + col) : 0.f;
    }
  };
  Pre cur, nxt;
  fetch(NC - 1, cur);

  for (int n = NC - 1; n >= 0; --n) {
    float* rec = recs + (size_t)n * R.size();
    fetch(n - 1, nxt);
#pragma unroll
    for (int nt = 0; nt < ST::NT; ++nt)             // gradient of chunk n's end state
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = acc_row(mS, lane, e), col = acc_col(nS, nt, lane, e);
        if (col0 + col < V) rec[R.dsn() + (size_t)c * V + col0 + col] = ds[0][nt][e];
      }
#pragma unroll
    for (int q = 0; q < NDO; ++q) {
      const int e = tid + q * NTH, i = e / VT, col = e - i * VT;
      dOs[i * LDV + col] = cur.dO[q];
    }
    cpa_wait<1>();
    __syncthreads();
    float acc[1][2][4];
    // dP = Mq^T dO + Kbar dS  (Mq[l][i] = 0 for l < i)
    zero(acc);
    wgemm3<1, 2>(acc, Mq, 1, L::LMQ, mX, dOs, LDV, 1, nX, mX, C, lane);
    wgemm3<1, 2>(acc, Kb, L::LKB, 1, mX, dSs, LDV, 1, nX, 0, KD, lane);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        dPs[acc_row(mX, lane, e) * LDV + acc_col(nX, nt, lane, e)] = acc[0][nt][e];
    __syncthreads();
    // dR = Tinv^T dP (Tinv[l][i] = 0 for l < i); dv = beta dR
    zero(acc);
    wgemm3<1, 2>(acc, Ti, 1, L::LTI, mX, dPs, LDV, 1, nX, mX, C, lane);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(mX, lane, e), col = acc_col(nX, nt, lane, e);
        const int t = n * C + i;
        const bool cok = col0 + col < V;
        const float bt = cur.bt[e >> 1];
        dZs[i * LDV + col] = -bt * acc[0][nt][e];
        if (cok) rec[R.drr() + (size_t)i * V + col0 + col] = acc[0][nt][e];
        if (cok && t < p.T) dv[(int64_t)t * p.dv_s[1] + col] = bt * acc[0][nt][e];
      }
    __syncthreads();
    issueA(n - 1);
    cpa_wait<1>();
    __syncthreads();
    // dS_prev = Diag(GamC) dS + EQ^T dO - KG^T (beta dR)
    {
#pragma unroll
      for (int nt = 0; nt < ST::NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) ds[0][nt][e] *= cur.gc[e >> 1];
      wgemm3<1, ST::NT>(ds, Eq, 1, L::LEQ, mS, dOs, LDV, 1, nS, 0, C, lane);
      wgemm3<1, ST::NT>(ds, Kg, 1, L::LEQ, mS, dZs, LDV, 1, nS, 0, C, lane);
#pragma unroll
      for (int nt = 0; nt < ST::NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          dSs[acc_row(mS, lane, e) * LDV + acc_col(nS, nt, lane, e)] = ds[0][nt][e];
    }
    __syncthreads();
    issueB(n - 1);
    cur = nxt;
  }
  if (p.dstate_in != nullptr) {
#pragma unroll
    for (int nt = 0; nt < ST::NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = acc_row(mS, lane, e), col = acc_col(nS, nt, lane, e);
        if (col0 + col < V)
          p.dstate_in[b * p.dsi_s[0] + h * p.dsi_s[1] + (int64_t)c * p.dsi_s[2] + col0 + col] =
              ds[0][nt][e];
      }
  }
}

// fchain CTAs (blockIdx.x < ceil(V / VT)) and bchain CTAs (the rest) in one
// launch: the two chains are independent and run side by side
template <typename TIO, typename TSI, int KD>
__global__ void __launch_bounds__(NTH, 1)
chains_kernel(const BwdParams p, float* __restrict__ ws) {
  const int nvt = (p.V + VT - 1) / VT;
  if ((int)blockIdx.x < nvt)
    fchain_cta<TIO, TSI, KD>(p, ws, blockIdx.x);
  else
    bchain_cta<TIO, KD>(p, ws, blockIdx.x - nvt);
}

// ---------------------------------------------------------------------------
// grad_kernel: one CTA per (chunk, h, b); V <= VMAX
// ---------------------------------------------------------------------------
constexpr int VMAX = 128;
constexpr int VS = VMAX + 4;                       // row stride of the [*][v] arrays (k = v)
constexpr int LDK = 33;                            // row stride of the [i][c] channel slices
constexpr int LDL = C + 4;                         // row stride of beta dL and dMq

struct GradSmem {
  static constexpr int DRS = 0;                    // dR [C][VS]
  static constexpr int PS = DRS + C * VS;          // P [C][VS]
  static constexpr int DOS = PS + C * VS;          // dO [C][VS]
  static constexpr int SS = DOS + C * VS;          // S rows of a 32-channel slice [32][VS]
  static constexpr int DSS = SS + 32 * VS;         // dS_next rows [32][VS]
  static constexpr int LR = DSS + 32 * VS;         // beta dL (j < i) [C][LDL]
  static constexpr int MQD = LR + C * LDL;         // dMq (j <= i) [C][LDL]
  static constexpr int QS = MQD + C * LDL;         // q' [C][LDK]
  static constexpr int KS = QS + C * LDK;          // k
  static constexpr int GS = KS + C * LDK;          // G
  static constexpr int E8 = GS + C * LDK;          // dEQ, then dG
  static constexpr int KG8 = E8 + C * LDK;         // dR S^T (dKG = -beta dR S^T)
  static constexpr int KB8 = KG8 + C * LDK;        // dKbar
  static constexpr int RED = KB8 + C * LDK;        // [2][NW][32] column partial sums
  static constexpr int DB = RED + 2 * NW * 32;     // dbeta [3][C]
  static constexpr int STP = DB + 3 * C;           // steep-block bits of each channel [32]
  static constexpr int FLOATS = STP + 32;
  static constexpr size_t BYTES = (size_t)FLOATS * sizeof(float);
};
static_assert(GradSmem::BYTES <= 227 * 1024, "grad_kernel shared memory");
static_assert(4 * C * LDK <= 2 * 32 * VS, "pair sums alias the state slices");

template <typename TIO, int KD>
__global__ void __launch_bounds__(NTH, 1)
grad_kernel(const BwdParams p, const float* __restrict__ ws) {
  using L = GradSmem;
  extern __shared__ __align__(16) float sm[];
  float* DRs = sm + L::DRS;
  float* Ps = sm + L::PS;
  float* DOs = sm + L::DOS;
  float* SSs = sm + L::SS;
  float* DSSs = sm + L::DSS;
  float* LR = sm + L::LR;
  float* MQD = sm + L::MQD;
  float* QS = sm + L::QS;
  float* KS = sm + L::KS;
  float* GS = sm + L::GS;
  float* E8 = sm + L::E8;
  float* KG8 = sm + L::KG8;
  float* KB8 = sm + L::KB8;
  float* RED = sm + L::RED;
  float* DB = sm + L::DB;
  unsigned* STP = reinterpret_cast<unsigned*>(sm + L::STP);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int NC = num_chunks(p.T);
  const int V = p.V, VP = 32 * ((V + 31) >> 5);
  const Rec R{KD, V};
  const float* rec = ws + ((size_t)(b * p.H + h) * NC + n) * R.size();
  const float* beta = p.beta + b * p.b_s[0] + h * p.b_s[2];

  // dR, P (chunk record) and dO into shared memory; columns V .. VP are zero
  cpa_rows(DRs, VS, rec + R.drr(), V, C, V);
  cpa_rows(Ps, VS, rec + R.pp(), V, C, V);
  cpa_commit();
  for (int e = tid; e < C * (VP - V); e += NTH) {
    const int i = e / (VP - V), col = V + e % (VP - V);
    DRs[i * VS + col] = 0.f;
    Ps[i * VS + col] = 0.f;
  }
  for (int e = tid; e < 32 * (VP - V); e += NTH) {
    const int c = e / (VP - V), col = V + e % (VP - V);
    SSs[c * VS + col] = 0.f;
    DSSs[c * VS + col] = 0.f;
  }
  {
    const TIO* db = static_cast<const TIO*>(p.dout) + b * p.do_s[0] + h * p.do_s[2];
#pragma unroll 8
    for (int e = tid; e < C * VP; e += NTH) {
      const int i = e / VP, col = e - i * VP;
      const int t = n * C + i;
      DOs[i * VS + col] = (t < p.T && col < V) ? ld(db + (int64_t)t * p.do_s[1] + col) : 0.f;
    }
  }
  // dbeta_i = dR_i . Z_i (+ the dL term below): warp w, rows 8w .. 8w + 7
  {
    float part[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int i = 8 * w + r;
      part[r] = 0.f;
#pragma unroll
      for (int j = 0; j < VMAX / 32; ++j) {
        const int col = lane + 32 * j;
        if (col < V)
          part[r] = fmaf(rec[R.drr() + (size_t)i * V + col], rec[R.zz() + (size_t)i * V + col],
                         part[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part[r] += __shfl_xor_sync(0xffffffffu, part[r], off);
      if (lane == 0) DB[8 * w + r] = part[r];
    }
  }
  cpa_wait<0>();
  __syncthreads();

  // dL = -(dR P^T) (j < i), dMq = dO P^T (j <= i); warp tile rows 16 (w % 4),
  // columns 32 (w / 4) .. + 31
  {
    const int m0 = 16 * (w & 3), n0 = 32 * (w >> 2);
    float al[1][4][4], am[1][4][4];
    zero(al);
    zero(am);
    wgemm3<1, 4>(al, DRs, VS, 1, m0, Ps, 1, VS, n0, 0, VP, lane);
    wgemm3<1, 4>(am, DOs, VS, 1, m0, Ps, 1, VS, n0, 0, VP, lane);
    const float* lraw = rec + R.lraw();
    float part[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = acc_row(m0, lane, e), j = acc_col(n0, nt, lane, e);
        const int t = n * C + i;
        const float bt = t < p.T ? beta[(int64_t)t * p.b_s[1]] : 0.f;
        const float dl = j < i ? -al[0][nt][e] : 0.f;
        part[e >> 1] = fmaf(dl, lraw[i * C + j], part[e >> 1]);
        LR[i * LDL + j] = bt * dl;
        MQD[i * LDL + j] = j <= i ? am[0][nt][e] : 0.f;
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      part[hh] += __shfl_xor_sync(0xffffffffu, part[hh], 1);
      part[hh] += __shfl_xor_sync(0xffffffffu, part[hh], 2);
    }
    if ((lane & 3) == 0) {
      DB[C * (1 + (w >> 2)) + acc_row(m0, lane, 0)] = part[0];
      DB[C * (1 + (w >> 2)) + acc_row(m0, lane, 2)] = part[1];
    }
  }
  __syncthreads();
  if (tid < C) {
    const int t = n * C + tid;
    if (t < p.T)
      p.dbeta[b * p.dbeta_s[0] + (int64_t)t * p.dbeta_s[1] + h * p.dbeta_s[2]] =
          DB[tid] + DB[C + tid] + DB[2 * C + tid];
  }

  // the K side, 32 channels at a time
  const TIO* qb = static_cast<const TIO*>(p.q) + b * p.q_s[0] + h * p.q_s[2];
  const TIO* kb = static_cast<const TIO*>(p.k) + b * p.k_s[0] + h * p.k_s[2];
  const float* gb = p.g + b * p.g_s[0] + h * p.g_s[2];
  TIO* dqb = static_cast<TIO*>(p.dq) + b * p.dq_s[0] + h * p.dq_s[2];
  TIO* dkb = static_cast<TIO*>(p.dk) + b * p.dk_s[0] + h * p.dk_s[2];
  float* dgb = p.dg + b * p.dg_s[0] + h * p.dg_s[2];
  const int i0 = 8 * w;                             // pair-term rows of this warp
  float bet[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int t = n * C + i0 + r;
    bet[r] = t < p.T ? beta[(int64_t)t * p.b_s[1]] : 0.f;
  }
  for (int s = 0; s < KD / 32; ++s) {
    const int c0 = 32 * s;
    __syncthreads();                                // previous slice consumed
    cpa_rows(SSs, VS, rec + R.sn() + (size_t)c0 * V, V, 32, V);
    cpa_rows(DSSs, VS, rec + R.dsn() + (size_t)c0 * V, V, 32, V);
    cpa_commit();
#pragma unroll 8
    for (int e = tid; e < C * 32; e += NTH) {       // q', k, g of the slice
      const int i = e >> 5, c = e & 31;
      const int t = n * C + i;
      const bool ok = t < p.T;
      QS[i * LDK + c] = ok ? ld(qb + (int64_t)t * p.q_s[1] + c0 + c) * p.scale : 0.f;
      KS[i * LDK + c] = ok ? ld(kb + (int64_t)t * p.k_s[1] + c0 + c) : 0.f;
      GS[i * LDK + c] = ok ? gb[(int64_t)t * p.g_s[1] + c0 + c] : 0.f;
    }
    cpa_wait<0>();
    __syncthreads();
    if (w == 0) {                                   // cumulative log decay of channel lane
      // and its steep blocks: block I (anchor a = 16 I) is steep when a factor
      // exp(G_i - G_a) (i in I) or exp(G_a - G_j) (j < a + 16) leaves e^-80 .. e^80
      float G = 0.f, runmin = 0.f, ga = 0.f, bmin = 0.f, bmax = 0.f;
      unsigned bits = 0u;
      for (int i = 0; i < C; ++i) {
        G += GS[i * LDK + lane];
        GS[i * LDK + lane] = G;
        if ((i & 15) == 0) {
          ga = G;
          bmin = bmax = G;
        }
        bmin = fminf(bmin, G);
        bmax = fmaxf(bmax, G);
        runmin = i == 0 ? G : fminf(runmin, G);
        if ((i & 15) == 15 && (bmin - ga < -80.f || bmax - ga > 80.f || ga - runmin > 80.f))
          bits |= 1u << (i >> 4);
      }
      STP[lane] = bits;
    }
    // dEQ = dO S^T, dR S^T, dKbar = P dS_next^T: rows 16 (w % 4), channels 16 (w / 4) .. + 15
    {
      const int m0 = 16 * (w & 3), n0 = 16 * (w >> 2);
      float ae[1][2][4], ak[1][2][4], ab[1][2][4];
      zero(ae);
      zero(ak);
      zero(ab);
      wgemm3<1, 2>(ae, DOs, VS, 1, m0, SSs, 1, VS, n0, 0, VP, lane);
      wgemm3<1, 2>(ak, DRs, VS, 1, m0, SSs, 1, VS, n0, 0, VP, lane);
      wgemm3<1, 2>(ab, Ps, VS, 1, m0, DSSs, 1, VS, n0, 0, VP, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = acc_row(m0, lane, e), c = acc_col(n0, nt, lane, e);
          E8[i * LDK + c] = ae[0][nt][e];
          KG8[i * LDK + c] = ak[0][nt][e];
          KB8[i * LDK + c] = ab[0][nt][e];
        }
    }
    {                                               // dGamC partials: sum_v dS_next S
      float gcp = 0.f;
      for (int col = w; col < V; col += NW) gcp = fmaf(DSSs[lane * VS + col], SSs[lane * VS + col], gcp);
      RED[w * 32 + lane] = gcp;
    }
    __syncthreads();
    // pair terms of dLraw and dMq by anchored 16-row blocks: for i in block I
    // (anchor a = 16 I), exp(G_ic - G_jc) = exp(G_ic - G_ac) exp(G_ac - G_jc),
    // both factors within e^-80 .. e^80 unless the block is steep for channel
    // c (those pairs are left out here and added exactly below).  Warp w:
    // block R = w % 4, channels cb .. cb + 15 (cb = 16 (w / 4)).
    //   rowA_i = exp(G_i - G_aR) sum_j LR_ij k_j exp(G_aR - G_j),  rowB: MQD
    //   colA_j = sum_{I >= R} exp(G_aI - G_j) sum_{i in I} LR_ij k_i exp(G_i - G_aI),
    //   colB_j: MQD and q'
    float* RA = SSs;                                // the state slices are dead here
    float* RB = RA + C * LDK;
    float* CA = RB + C * LDK;
    float* CB = CA + C * LDK;
    {
      const int R = w & 3, cb = 16 * (w >> 2);
      const int g = lane >> 2, tq = lane & 3;
      float ra[1][2][4], rb[1][2][4];
      zero(ra);
      zero(rb);
      for (int k = 0; k < 16 * (R + 1); k += 8) {
        uint32_t lh[4], ll[4], mh[4], ml[4];
        const float* la = LR + (16 * R + g) * LDL + k + tq;
        const float* ma = MQD + (16 * R + g) * LDL + k + tq;
        split3(la[0], lh[0], ll[0]);
        split3(la[8 * LDL], lh[1], ll[1]);
        split3(la[4], lh[2], ll[2]);
        split3(la[8 * LDL + 4], lh[3], ll[3]);
        split3(ma[0], mh[0], ml[0]);
        split3(ma[8 * LDL], mh[1], ml[1]);
        split3(ma[4], mh[2], ml[2]);
        split3(ma[8 * LDL + 4], mh[3], ml[3]);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int c = cb + 8 * nt + g;
          const bool st = (STP[c] >> R) & 1u;
          const float gaR = GS[16 * R * LDK + c];
          const int j0 = k + tq, j1 = j0 + 4;
          const float b0 = st ? 0.f : KS[j0 * LDK + c] * __expf(gaR - GS[j0 * LDK + c]);
          const float b1 = st ? 0.f : KS[j1 * LDK + c] * __expf(gaR - GS[j1 * LDK + c]);
          uint32_t bh[2], bl[2];
          split3(b0, bh[0], bl[0]);
          split3(b1, bh[1], bl[1]);
          ptx::mma_tf32_16x8x8(ra[0][nt], ll, bh);
          ptx::mma_tf32_16x8x8(ra[0][nt], lh, bl);
          ptx::mma_tf32_16x8x8(ra[0][nt], lh, bh);
          ptx::mma_tf32_16x8x8(rb[0][nt], ml, bh);
          ptx::mma_tf32_16x8x8(rb[0][nt], mh, bl);
          ptx::mma_tf32_16x8x8(rb[0][nt], mh, bh);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = acc_row(16 * R, lane, e), c = acc_col(cb, nt, lane, e);
          const bool st = (STP[c] >> R) & 1u;
          const float sc = st ? 0.f : __expf(GS[i * LDK + c] - GS[16 * R * LDK + c]);
          RA[i * LDK + c] = ra[0][nt][e] * sc;
          RB[i * LDK + c] = rb[0][nt][e] * sc;
        }
      float ca[1][2][4], cq[1][2][4];
      zero(ca);
      zero(cq);
      for (int I = R; I < 4; ++I) {
        float ta[1][2][4], tb[1][2][4];
        zero(ta);
        zero(tb);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int k = 16 * I + 8 * kk;
          uint32_t lh[4], ll[4], mh[4], ml[4];      // A(j, i) = LR[i][j], rows j of block R
          const float* la = LR + (k + tq) * LDL + 16 * R + g;
          const float* ma = MQD + (k + tq) * LDL + 16 * R + g;
          split3(la[0], lh[0], ll[0]);
          split3(la[8], lh[1], ll[1]);
          split3(la[4 * LDL], lh[2], ll[2]);
          split3(la[4 * LDL + 8], lh[3], ll[3]);
          split3(ma[0], mh[0], ml[0]);
          split3(ma[8], mh[1], ml[1]);
          split3(ma[4 * LDL], mh[2], ml[2]);
          split3(ma[4 * LDL + 8], mh[3], ml[3]);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int c = cb + 8 * nt + g;
            const bool st = (STP[c] >> I) & 1u;
            const float gaI = GS[16 * I * LDK + c];
            const int i0_ = k + tq, i1_ = i0_ + 4;
            const float w0 = st ? 0.f : __expf(GS[i0_ * LDK + c] - gaI);
            const float w1 = st ? 0.f : __expf(GS[i1_ * LDK + c] - gaI);
            uint32_t bh[2], bl[2], qh[2], ql[2];
            split3(KS[i0_ * LDK + c] * w0, bh[0], bl[0]);
            split3(KS[i1_ * LDK + c] * w1, bh[1], bl[1]);
            split3(QS[i0_ * LDK + c] * w0, qh[0], ql[0]);
            split3(QS[i1_ * LDK + c] * w1, qh[1], ql[1]);
            ptx::mma_tf32_16x8x8(ta[0][nt], ll, bh);
            ptx::mma_tf32_16x8x8(ta[0][nt], lh, bl);
            ptx::mma_tf32_16x8x8(ta[0][nt], lh, bh);
            ptx::mma_tf32_16x8x8(tb[0][nt], ml, qh);
            ptx::mma_tf32_16x8x8(tb[0][nt], mh, ql);
            ptx::mma_tf32_16x8x8(tb[0][nt], mh, qh);
          }
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = acc_row(16 * R, lane, e), c = acc_col(cb, nt, lane, e);
            const bool st = (STP[c] >> I) & 1u;
            const float sc = st ? 0.f : __expf(GS[16 * I * LDK + c] - GS[j * LDK + c]);
            ca[0][nt][e] = fmaf(ta[0][nt][e], sc, ca[0][nt][e]);
            cq[0][nt][e] = fmaf(tb[0][nt][e], sc, cq[0][nt][e]);
          }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = acc_row(16 * R, lane, e), c = acc_col(cb, nt, lane, e);
          CA[j * LDK + c] = ca[0][nt][e];
          CB[j * LDK + c] = cq[0][nt][e];
        }
    }
    __syncthreads();
    {                                               // steep blocks: exact pair terms
      const unsigned stc = STP[lane];
      for (int I = 0; I < 4 && stc != 0u; ++I) {
        if (!((stc >> I) & 1u)) continue;
#pragma unroll 1
        for (int ii = 0; ii < 2; ++ii) {
          const int i = 16 * I + 2 * w + ii;
          const float Gi = GS[i * LDK + lane], ki = KS[i * LDK + lane], qi = QS[i * LDK + lane];
          float sa = 0.f, sb = 0.f;
          for (int j = 0; j <= i; ++j) {
            const float D = __expf(Gi - GS[j * LDK + lane]);
            const float l = LR[i * LDL + j] * D, m = MQD[i * LDL + j] * D;
            const float kj = KS[j * LDK + lane];
            sa = fmaf(l, kj, sa);
            sb = fmaf(m, kj, sb);
            atomicAdd(&CA[j * LDK + lane], l * ki);
            atomicAdd(&CB[j * LDK + lane], m * qi);
          }
          RA[i * LDK + lane] += sa;
          RB[i * LDK + lane] += sb;
        }
      }
    }
    __syncthreads();
    float Gi[8], ki[8], qi[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      Gi[r] = GS[(i0 + r) * LDK + lane];
      ki[r] = KS[(i0 + r) * LDK + lane];
      qi[r] = QS[(i0 + r) * LDK + lane];
    }
    // combine; dG replaces dEQ in E8, Kbar-column partial sums into RED[1]
    const float Gl = GS[(C - 1) * LDK + lane];
    float kbs = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int i = i0 + r, t = n * C + i;
      const float gam = expf(Gi[r]), eb = expf(Gl - Gi[r]);
      const float kbar = ki[r] * eb;
      const float e8 = E8[i * LDK + lane], kb8 = KB8[i * LDK + lane];
      const float dkg = -bet[r] * KG8[i * LDK + lane];
      const float rA = RA[i * LDK + lane], rB = RB[i * LDK + lane];
      const float cA = CA[i * LDK + lane], cB = CB[i * LDK + lane];
      const float dq = rB + e8 * gam;
      const float dk = rA + cA + cB + dkg * gam + kb8 * eb;
      const float dG = ki[r] * (rA - cA) + qi[r] * rB - ki[r] * cB + e8 * qi[r] * gam +
                       dkg * ki[r] * gam - kb8 * kbar;
      kbs = fmaf(kb8, kbar, kbs);
      E8[i * LDK + lane] = dG;
      if (t < p.T) {
        st(dqb + (int64_t)t * p.dq_s[1] + c0 + lane, dq * p.scale);
        st(dkb + (int64_t)t * p.dk_s[1] + c0 + lane, dk);
      }
    }
    RED[NW * 32 + w * 32 + lane] = kbs;
    __syncthreads();
    if (w == 0) {                                   // chunk-end terms, reverse cumsum
      float gc = 0.f, ks = 0.f;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) {
        gc += RED[ww * 32 + lane];
        ks += RED[NW * 32 + ww * 32 + lane];
      }
      float acc2 = ks + gc * expf(Gl);
      for (int i = C - 1; i >= 0; --i) {
        acc2 += E8[i * LDK + lane];
        const int t = n * C + i;
        if (t < p.T) dgb[(int64_t)t * p.dg_s[1] + c0 + lane] = acc2;
      }
    }
  }
}

template <typename TIO, typename TSI, int KD>
static cudaError_t launch_kd(const BwdParams& p, cudaStream_t s) {
  const int NC = num_chunks(p.T);
  const int nvt = (p.V + VT - 1) / VT;
  const dim3 cgrid(NC, p.H, p.B), vgrid(2 * nvt, p.H, p.B);
  const size_t s0 = PrepSmem<KD>::BYTES, s3 = GradSmem::BYTES;
  const size_t s1 = FchainSmem<KD>::BYTES > BchainSmem<KD>::BYTES ? FchainSmem<KD>::BYTES
                                                                    : BchainSmem<KD>::BYTES;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(prep_kernel<TIO, KD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)s0)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(chains_kernel<TIO, TSI, KD>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s1)) !=
          cudaSuccess ||
      (e = cudaFuncSetAttribute(grad_kernel<TIO, KD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)s3)) != cudaSuccess)
    return e;
  prep_kernel<TIO, KD><<<cgrid, NTH, s0, s>>>(p, p.ckpt);
  chains_kernel<TIO, TSI, KD><<<vgrid, NTH, s1, s>>>(p, p.ckpt);
  grad_kernel<TIO, KD><<<cgrid, NTH, s3, s>>>(p, p.ckpt);
  return cudaGetLastError();
}

template <typename TIO, typename TSI>
static cudaError_t launch_k(const BwdParams& p, cudaStream_t s) {
  switch (p.K) {
    case 32: return launch_kd<TIO, TSI, 32>(p, s);
    case 64: return launch_kd<TIO, TSI, 64>(p, s);
    default: return launch_kd<TIO, TSI, 128>(p, s);
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

}  // namespace bwdc

bool backward_chunk_supported(const BwdParams& p) {
  return p.dq != nullptr && (p.K == 32 || p.K == 64 || p.K == 128) && p.V >= 16 &&
         p.V % 16 == 0 && p.V <= bwdc::VMAX;
}

size_t backward_chunk_ws_floats(int B, int H, int T, int K, int V) {
  return (size_t)B * H * bwdc::num_chunks(T) * bwdc::Rec{K, V}.size();
}

cudaError_t launch_backward_chunk(const BwdParams& p, cudaStream_t s) {
  switch (p.io_dtype) {
    case KDA_DTYPE_F32: return bwdc::launch_si<float>(p, s);
    case KDA_DTYPE_F16: return bwdc::launch_si<__half>(p, s);
    default: return bwdc::launch_si<__nv_bfloat16>(p, s);
  }
}

}  // namespace kda
