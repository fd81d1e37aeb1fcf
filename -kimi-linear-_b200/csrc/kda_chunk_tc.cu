// kda_chunk_tc.cu -- tensor-core chunkwise KDA for sm_100a (fp16 / bf16 q,k,v; K = 128).
//
// Replaces kimi_linear/kda.py:58-185 (kda_chunkwise) for the shapes of the
// 1.5B model and the benchmark configurations.  Two kernels on one stream:
//
// 1. prep_kernel  -- one CTA per (b, h, chunk of 64 rows), fully parallel.
//    Everything of a chunk that does not depend on the carried state:
//      gc = cumsum(g)                                        (kda.py:129)
//      L[c,i]    = beta_c sum_k k_ck k_ik exp(gc_ck - gc_ik), i < c  (kda.py:159-165)
//      Aout[c,i] = sum_k s q_ck k_ik exp(gc_ck - gc_ik),      i <= c (kda.py:166-168)
//      M = (I + L)^-1 Diag(beta)                             (kda.py:170-171)
//      W = M (exp(gc) * K)                                   (kda.py:172)
//      Qbar = s q exp(gc),  Kbar = exp(gc_last - gc) k,  d = exp(gc_last)
//    and writes them as ONE 66,048-byte image per chunk whose byte layout is
//    exactly the tcgen05 shared-memory operand layout the second kernel uses,
//    so that kernel moves it with a single bulk (TMA-engine) copy.
//
//    The decay products exp(gc_c - gc_i) are never formed pair by pair.  The
//    chunk is split into four 16-row blocks; with the per-step decays
//    alpha = exp(g), each row gets ra_c = exp(gc_c - gc_blockstart) (prefix
//    product) and nb_c = exp(gc_nextblockstart - gc_c) (suffix product), both
//    in (0, 1].  For a pair in different blocks the decay is
//    ra_c * nb_i * (product of the whole-block decays in between): a dense
//    16x16x128 tensor-core GEMM on pre-scaled operands (tf32 mma.sync), with
//    no overflow possible.  Inside a diagonal block the decay is
//    ra_c * nb_i * exp(-Z_r) with Z_r the block's total decay; that factor is
//    at most e^80 when the block is not "steep" (Z_r >= -80), which tf32 holds
//    exactly.  Channels of a steep block are removed from that GEMM and their
//    exact pair terms exp(gc_c - gc_i) are added separately (rare).
//    (I + L)^-1 is a blocked forward substitution in fp32: 16x16 diagonal
//    blocks by substitution, off-diagonal blocks M_rj = -D_r sum_t L_rt M_tj.
//
// 2. state_kernel -- one CTA per (b, h, slice of VS value columns), walking the
//    chunks in order with the fp32 state S[128, VS] resident in TMEM.  Per
//    chunk (kda.py:176-182):
//      R2 = [M; Aout] V            R1 = [-W; Qbar] S          (tcgen05)
//      P  = R2[0:64] + R1[0:64]  (= U - W S)                  (registers -> smem f16)
//      R1 += [M; Aout] P  -> rows 64..127 = Qbar S + Aout P = O  (tcgen05)
//      R3  = d * S,  R3 += Kbar^T P  -> next S                  (tcgen05)
//    Operands are f16 (bf16 inputs are exactly representable in f16 at these
//    magnitudes); every product accumulates in fp32 TMEM, and the carried
//    state never leaves fp32 (the reference rounds S to the transient dtype
//    for its two state GEMMs, kda.py:176, as the f16 copy here does).
//    The images are double-buffered in shared memory and fetched two chunks
//    ahead with cp.async.bulk; every mbarrier wait is bounded in time and
//    aborts the CTA cleanly (error word, TMEM freed) instead of hanging.
#include <type_traits>

#include "kda_internal.cuh"
#include "tc_ptx.cuh"

namespace kda {

__device__ int g_kda_device_error = 0;

namespace tc {

constexpr int CH = 64;        // rows per chunk
constexpr int KD = 128;       // head dim K of this path
// chunk image (bytes); all operands f16, no-swizzle K-major core-matrix layout
constexpr int IMG_A1 = 0;         // [-W; Qbar]  128 x 128, LBO 128, SBO 2048
constexpr int IMG_A2 = 32768;     // [M; Aout]   128 x 64,  LBO 128, SBO 1024
constexpr int IMG_A3 = 49152;     // Kbar^T      128 x 64,  LBO 128, SBO 1024
constexpr int IMG_D = 65536;      // d = exp(gc_last), fp32[128]
constexpr int IMG_BYTES = 66048;
constexpr int IMG_PAD = 66560;    // 65 KiB, keeps the next buffer 1 KiB aligned

constexpr float kSteep = 80.f;                  // block decay beyond which exp(-Z) is unsafe
constexpr uint64_t kWaitNs = 2000000000ull;     // bound on every mbarrier wait (2 s)

__device__ __forceinline__ int a1_off(int m, int k) {
  return (m >> 3) * 2048 + (k >> 3) * 128 + (m & 7) * 16 + (k & 7) * 2;
}
__device__ __forceinline__ int a2_off(int m, int k) {
  return (m >> 3) * 1024 + (k >> 3) * 128 + (m & 7) * 16 + (k & 7) * 2;
}

// ---------------------------------------------------------------------------
// prep kernel
// ---------------------------------------------------------------------------
constexpr int AXP = 132;   // fp32 pitch of the Gram operand arrays (bank spread)
constexpr int LMP = 68;    // fp32 pitch of L and M
constexpr int P_IMG = 0;
constexpr int P_AXK = IMG_PAD;                         // k * ra          fp32 [64][132]
constexpr int P_AXQ = P_AXK + CH * AXP * 4;            // s q * ra        fp32 [64][132]
constexpr int P_YB = P_AXQ + CH * AXP * 4;             // k * nb          fp32 [64][132]
constexpr int P_LM = P_YB + CH * AXP * 4;              // L               fp32 [64][68]
constexpr int P_FAC = P_LM + CH * LMP * 4;             // P02,P03,P13,E[4] fp32 [7][128]
constexpr int P_BETA = P_FAC + 7 * KD * 4;             // beta            fp32 [64]
constexpr int P_STEEP = P_BETA + CH * 4;               // steep bits      u32 [4][4]
constexpr int PREP_SMEM = P_STEEP + 16 * 4;
static_assert(PREP_SMEM <= 227 * 1024, "prep shared memory");
// M (fp32, pitch LMP) reuses the k*ra array and the inversion scratch the
// q*ra array once the Gram is done
constexpr int PREP_THREADS = 256;

template <typename TIO>
__global__ void __launch_bounds__(PREP_THREADS, 1)
prep_kernel(const ChunkParams p, uint8_t* __restrict__ ws) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* img = sm + P_IMG;
  float* Axk = reinterpret_cast<float*>(sm + P_AXK);
  float* Axq = reinterpret_cast<float*>(sm + P_AXQ);
  float* Yb = reinterpret_cast<float*>(sm + P_YB);
  float* Lm = reinterpret_cast<float*>(sm + P_LM);
  float* P02 = reinterpret_cast<float*>(sm + P_FAC);
  float* P03 = P02 + KD;
  float* P13 = P03 + KD;
  float* Ef = P13 + KD;                                   // [4][128]
  float* sbeta = reinterpret_cast<float*>(sm + P_BETA);
  uint32_t* steep = reinterpret_cast<uint32_t*>(sm + P_STEEP);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int NT = gridDim.x;
  const int t0 = n * CH;
  const int nvalid = min(CH, p.T - t0);
  const float s = p.scale;
  const TIO* qb = static_cast<const TIO*>(p.q) + b * p.q_s[0] + h * p.q_s[2];
  const TIO* kb = static_cast<const TIO*>(p.k) + b * p.k_s[0] + h * p.k_s[2];
  const float* gb = p.g + b * p.g_s[0] + h * p.g_s[2];
  const float* bb = p.beta + b * p.b_s[0] + h * p.b_s[2];

  // ---- 0. zero L, the Aout half of [M; Aout], the steep mask; beta ---------
  for (int i = tid; i < CH * LMP; i += PREP_THREADS) Lm[i] = 0.f;
  for (int i = tid; i < 8192 / 16; i += PREP_THREADS)
    reinterpret_cast<int4*>(img + IMG_A2 + 8192)[i] = make_int4(0, 0, 0, 0);
  if (tid < 16) steep[tid] = 0u;
  if (tid < CH) sbeta[tid] = (tid < nvalid) ? bb[(int64_t)(t0 + tid) * p.b_s[1]] : 0.f;
  __syncthreads();

  // ---- 1. per channel: decays, factors, decayed operands -------------------
  {
    const int k = tid & (KD - 1), half = tid >> 7;
    float gv[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c)
      gv[c] = (c < nvalid) ? gb[(int64_t)(t0 + c) * p.g_s[1] + k] : 0.f;
    float Zp[4], eZ[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int hi = (r < 3) ? 16 * (r + 1) : CH - 1;
      float z = 0.f;
#pragma unroll
      for (int t = 16 * r + 1; t <= hi; ++t) z += gv[t];
      Zp[r] = z;
      eZ[r] = expf(z);
    }
    const float a0 = expf(gv[0]);
    float Bf[4], Af[4];
    Bf[0] = a0;
    Bf[1] = Bf[0] * eZ[0];
    Bf[2] = Bf[1] * eZ[1];
    Bf[3] = Bf[2] * eZ[2];
    Af[3] = 1.f;
    Af[2] = eZ[3];
    Af[1] = eZ[2] * eZ[3];
    Af[0] = eZ[1] * Af[1];
    if (half == 0) {
      P02[k] = eZ[1];
      P03[k] = eZ[1] * eZ[2];
      P13[k] = eZ[2];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const bool st = Zp[r] < -kSteep;
        Ef[r * KD + k] = st ? 0.f : expf(-Zp[r]);
        if (st) atomicOr(&steep[r * 4 + (k >> 5)], 1u << (k & 31));
      }
      reinterpret_cast<float*>(img + IMG_D)[k] = Bf[3] * eZ[3];   // exp(gc_last)
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if ((r >> 1) != half) continue;
      const int hi = (r < 3) ? 16 * (r + 1) : CH - 1;
      float al[17];
#pragma unroll
      for (int i = 1; i <= 16; ++i) al[i] = (16 * r + i <= hi) ? expf(gv[16 * r + i]) : 1.f;
      float ra[16], nb[16];
      ra[0] = 1.f;
#pragma unroll
      for (int i = 1; i < 16; ++i) ra[i] = ra[i - 1] * al[i];
      nb[15] = al[16];
#pragma unroll
      for (int i = 14; i >= 0; --i) nb[i] = nb[i + 1] * al[i + 1];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int c = 16 * r + i;
        float qv = 0.f, kv = 0.f;
        if (c < nvalid) {
          qv = ld(qb + (int64_t)(t0 + c) * p.q_s[1] + k);
          kv = ld(kb + (int64_t)(t0 + c) * p.k_s[1] + k);
        }
        const float qs = qv * s;
        const float eg = Bf[r] * ra[i];                   // exp(gc_c)
        *reinterpret_cast<__half*>(img + IMG_A1 + a1_off(64 + c, k)) = __float2half_rn(qs * eg);
        *reinterpret_cast<__half*>(img + IMG_A1 + a1_off(c, k)) = __float2half_rn(kv * eg);
        *reinterpret_cast<__half*>(img + IMG_A3 + a2_off(k, c)) =
            __float2half_rn(kv * nb[i] * Af[r]);            // exp(gc_last - gc_c) k
        Axk[c * AXP + k] = kv * ra[i];
        Axq[c * AXP + k] = qs * ra[i];
        Yb[c * AXP + k] = kv * nb[i];
      }
    }
  }
  __syncthreads();

  // ---- 2. Gram blocks L and Aout (tf32 mma.sync, fp32 accumulate) ----------
  {
    const int gid = lane >> 2, tig = lane & 3;
    for (int task = warp; task < 20; task += PREP_THREADS / 32) {
      const int type = task / 10;                     // 0: L (x = k), 1: Aout (x = s q)
      int j = task % 10, r = 0;
      while (j > r) { j -= r + 1; ++r; }
      const float* Ax = type ? Axq : Axk;
      const float* f = nullptr;                       // per-channel factor on the B side
      if (j == r) f = Ef + r * KD;
      else if (r - j == 2) f = (j == 0) ? P02 : P13;
      else if (r - j == 3) f = P03;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const float* ar0 = Ax + (16 * r + gid) * AXP;
      const float* ar1 = ar0 + 8 * AXP;
      const float* br0 = Yb + (16 * j + gid) * AXP;
      const float* br1 = br0 + 8 * AXP;
#pragma unroll 4
      for (int k0 = 0; k0 < KD; k0 += 8) {
        const uint32_t a[4] = {ptx::f32_to_tf32(ar0[k0 + tig]), ptx::f32_to_tf32(ar1[k0 + tig]),
                               ptx::f32_to_tf32(ar0[k0 + tig + 4]),
                               ptx::f32_to_tf32(ar1[k0 + tig + 4])};
        const float f0 = f ? f[k0 + tig] : 1.f, f1 = f ? f[k0 + tig + 4] : 1.f;
        const uint32_t b0[2] = {ptx::f32_to_tf32(br0[k0 + tig] * f0),
                                ptx::f32_to_tf32(br0[k0 + tig + 4] * f1)};
        const uint32_t b1[2] = {ptx::f32_to_tf32(br1[k0 + tig] * f0),
                                ptx::f32_to_tf32(br1[k0 + tig + 4] * f1)};
        ptx::mma_tf32_16x8x8(acc[0], a, b0);
        ptx::mma_tf32_16x8x8(acc[1], a, b1);
      }
      if (j == r) {
        // exact pair terms of the steep channels of this diagonal block
#pragma unroll 1
        for (int w4 = 0; w4 < 4; ++w4) {
          uint32_t m = steep[r * 4 + w4];
          while (m) {
            const int kk = w4 * 32 + __ffs(m) - 1;
            m &= m - 1;
            float pre[16];
            pre[0] = 0.f;
#pragma unroll
            for (int i = 1; i < 16; ++i) {
              const int c = 16 * r + i;
              pre[i] = pre[i - 1] + ((c < nvalid) ? gb[(int64_t)(t0 + c) * p.g_s[1] + kk] : 0.f);
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int rl = gid + 8 * (e >> 1), cl = 8 * nt + 2 * tig + (e & 1);
                const int c = 16 * r + rl, i = 16 * r + cl;
                if (cl <= rl && c < nvalid) {
                  const float xr = type ? s * ld(qb + (int64_t)(t0 + c) * p.q_s[1] + kk)
                                        : ld(kb + (int64_t)(t0 + c) * p.k_s[1] + kk);
                  const float ki = ld(kb + (int64_t)(t0 + i) * p.k_s[1] + kk);
                  acc[nt][e] = fmaf(xr * ki, expf(pre[rl] - pre[cl]), acc[nt][e]);
                }
              }
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = 16 * r + gid + 8 * (e >> 1);
          const int col = 16 * j + 8 * nt + 2 * tig + (e & 1);
          const float v = acc[nt][e];
          if (type == 0) {
            if (col < row) Lm[row * LMP + col] = sbeta[row] * v;
          } else if (col <= row) {
            *reinterpret_cast<__half*>(img + IMG_A2 + a2_off(64 + row, col)) = __float2half_rn(v);
          }
        }
    }
  }
  __syncthreads();

  // ---- 3. M = (I + L)^-1 Diag(beta), blocked forward substitution (fp32) ---
  float* Mm = Axk;                     // pitch LMP
  float* Ts = Axq;                     // per-warp 16x17 scratch
  if (warp < 4) {
    const int r = warp;
    if (lane < 16) {
      const int j = lane;
      float x[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float acc = (c == j) ? 1.f : 0.f;
#pragma unroll
        for (int i = 0; i < c; ++i) acc = fmaf(-Lm[(16 * r + c) * LMP + 16 * r + i], x[i], acc);
        x[c] = acc;
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) Mm[(16 * r + c) * LMP + 16 * r + j] = x[c];
    }
  } else {
    for (int idx = tid - 128; idx < CH * CH; idx += 128) {
      const int row = idx >> 6, col = idx & 63;
      if ((col >> 4) > (row >> 4)) Mm[row * LMP + col] = 0.f;
    }
  }
  __syncthreads();
  for (int dist = 1; dist <= 3; ++dist) {
    if (warp < 4 - dist) {
      const int j = warp, r = warp + dist;
      float* T = Ts + warp * (16 * 17);
      for (int o = lane; o < 256; o += 32) {
        const int row = o >> 4, col = o & 15;
        float acc = 0.f;
        for (int cp = 16 * j; cp < 16 * r; ++cp)
          acc = fmaf(Lm[(16 * r + row) * LMP + cp], Mm[cp * LMP + 16 * j + col], acc);
        T[row * 17 + col] = acc;
      }
      __syncwarp();
      for (int o = lane; o < 256; o += 32) {
        const int row = o >> 4, col = o & 15;
        float acc = 0.f;
        for (int i = 0; i <= row; ++i)
          acc = fmaf(Mm[(16 * r + row) * LMP + 16 * r + i], T[i * 17 + col], acc);
        Mm[(16 * r + row) * LMP + 16 * j + col] = -acc;
      }
    }
    __syncthreads();
  }
  for (int idx = tid; idx < CH * CH; idx += PREP_THREADS) {
    const int row = idx >> 6, col = idx & 63;
    *reinterpret_cast<__half*>(img + IMG_A2 + a2_off(row, col)) =
        __float2half_rn(Mm[row * LMP + col] * sbeta[col]);
  }
  __syncthreads();

  // ---- 4. W = M Ktilde (f16 mma.sync); store -W over Ktilde ----------------
  {
    const int gid = lane >> 2, tig = lane & 3;
    const int rb = warp & 3, ch = warp >> 2;
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    const int mi = lane >> 3;
    for (int ks = 0; ks <= rb; ++ks) {
      uint32_t a[4];
      ptx::ldmatrix_x4(a, img + IMG_A2 + a2_off(16 * rb + (lane & 7) + ((mi & 1) ? 8 : 0),
                                                16 * ks + ((mi & 2) ? 8 : 0)));
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t bq[4];
        ptx::ldmatrix_x4_trans(bq, img + IMG_A1 + a1_off(16 * ks + (lane & 7) + ((mi & 1) ? 8 : 0),
                                                         64 * ch + 8 * nt + ((mi & 2) ? 8 : 0)));
        ptx::mma_f16_16x8x16(acc[nt], a, bq);
        ptx::mma_f16_16x8x16(acc[nt + 1], a, bq + 2);
      }
    }
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int row = 16 * rb + gid + 8 * hr;
        const int col = 64 * ch + 8 * nt + 2 * tig;
        *reinterpret_cast<__half2*>(img + IMG_A1 + a1_off(row, col)) =
            __floats2half2_rn(-acc[nt][2 * hr], -acc[nt][2 * hr + 1]);
      }
  }
  __syncthreads();

  // ---- 5. image -> workspace ----------------------------------------------
  int4* dst = reinterpret_cast<int4*>(ws + ((size_t)(b * p.H + h) * NT + n) * IMG_BYTES);
  const int4* src = reinterpret_cast<const int4*>(img);
  for (int i = tid; i < IMG_BYTES / 16; i += PREP_THREADS) dst[i] = src[i];
}

// ---------------------------------------------------------------------------
// state kernel
// ---------------------------------------------------------------------------
template <int VS>
struct StateCfg {
  static constexpr int NCOL = VS <= 16 ? 64 : (VS <= 32 ? 128 : (VS <= 64 ? 256 : 512));
  static constexpr int R1 = 0, R2 = VS, R3 = 2 * VS;
  static constexpr int VT_BYTES = CH * VS * 2;                 // V tile, K = 64 rows
  static constexpr int STAGE = IMG_PAD + ((VT_BYTES + 1023) / 1024) * 1024;
  static constexpr int SB_OFF = 2 * STAGE;                     // S  (K = 128) f16
  static constexpr int PB_OFF = SB_OFF + KD * VS * 2;          // P  (K = 64)  f16
  static constexpr int BAR_OFF = PB_OFF + CH * VS * 2;
  static constexpr int SMEM = BAR_OFF + 64;
  static_assert(SMEM <= 227 * 1024, "state shared memory");
};

// 8 fp32 -> 8 f16 packed in 16 bytes
__device__ __forceinline__ int4 pack8_f16(const float* x) {
  __half2 h0 = __floats2half2_rn(x[0], x[1]), h1 = __floats2half2_rn(x[2], x[3]);
  __half2 h2 = __floats2half2_rn(x[4], x[5]), h3 = __floats2half2_rn(x[6], x[7]);
  int4 r;
  r.x = *reinterpret_cast<int*>(&h0);
  r.y = *reinterpret_cast<int*>(&h1);
  r.z = *reinterpret_cast<int*>(&h2);
  r.w = *reinterpret_cast<int*>(&h3);
  return r;
}

// V tile of chunk n (rows t = 64n + c, columns v0 .. v0+VS) as the f16
// MN-major B operand: offset(c, v) = (v/8)*1024 + (c/8)*128 + (c%8)*16 + (v%8)*2
template <int VS, typename TIO>
__device__ __forceinline__ void load_vtile(uint8_t* vt, const ChunkParams& p, int b, int h,
                                           int v0, int n) {
  constexpr int GPR = VS / 8;
  for (int piece = threadIdx.x; piece < CH * GPR; piece += 128) {
    const int c = piece / GPR, gv = piece % GPR;
    const int t = n * CH + c;
    float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (t < p.T) {
      const TIO* src = static_cast<const TIO*>(p.v) + b * p.v_s[0] + (int64_t)t * p.v_s[1] +
                       h * p.v_s[2] + v0 + 8 * gv;
      if (p.v_vec16) {
        ld4(src, *reinterpret_cast<float(*)[4]>(x));
        ld4(src + 4, *reinterpret_cast<float(*)[4]>(x + 4));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = ld(src + e);
      }
    }
    *reinterpret_cast<int4*>(vt + gv * 1024 + (c >> 3) * 128 + (c & 7) * 16) = pack8_f16(x);
  }
}

template <int VS, typename TIO, typename TSI, typename TSO>
__global__ void __launch_bounds__(128, 1)
state_kernel(const ChunkParams p, const uint8_t* __restrict__ ws) {
  using Cfg = StateCfg<VS>;
  constexpr int CW = VS < 32 ? VS : 32;   // TMEM columns per register piece
  constexpr int NP = VS / CW;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* Sb = sm + Cfg::SB_OFF;
  uint8_t* Pb = sm + Cfg::PB_OFF;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Cfg::BAR_OFF);   // [2]
  uint64_t* mbar = full + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = blockIdx.z, h = blockIdx.y, v0 = blockIdx.x * VS;
  const int T = p.T;
  const int NT = (T + CH - 1) / CH;
  const uint8_t* wsh = ws + (size_t)(b * p.H + h) * NT * IMG_BYTES;
  constexpr uint32_t IDESC = ptx::idesc_f16_f32(128, VS, false, true);

  if (warp == 0) {
    ptx::tmem_alloc(tslot, Cfg::NCOL);
    ptx::tmem_relinquish();
  }
  if (tid == 0) {
    ptx::mbar_init(&full[0], 1);
    ptx::mbar_init(&full[1], 1);
    ptx::mbar_init(mbar, 1);
    ptx::fence_mbar_init();
    *abort_flag = 0;
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tlane = tbase + (static_cast<uint32_t>(warp * 32) << 16);

  // thread 0: stages with a bulk copy in flight and the parity of its phase
  uint32_t pending = 0, pend_par = 0;
  if (tid == 0) {
    for (int sg = 0; sg < 2 && sg < NT; ++sg) {
      ptx::mbar_arrive_expect_tx(&full[sg], IMG_BYTES);
      ptx::bulk_g2s(sm + sg * Cfg::STAGE, wsh + (size_t)sg * IMG_BYTES, IMG_BYTES, &full[sg]);
      pending |= 1u << sg;
    }
  }
#pragma unroll 1
  for (int pc = 0; pc < NP; ++pc) {                        // initial state -> R3
    float srow[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) srow[j] = 0.f;
    if (p.state_in != nullptr) {
      const TSI* src = static_cast<const TSI*>(p.state_in) + b * p.si_s[0] + h * p.si_s[1] +
                       (int64_t)tid * p.si_s[2] + v0 + pc * CW;
#pragma unroll
      for (int j = 0; j < CW; ++j) srow[j] = ld(src + j);
    }
    ptx::tmem_st<CW>(tlane + Cfg::R3 + pc * CW, srow);
  }
  ptx::tmem_wait_st();
  load_vtile<VS, TIO>(sm + IMG_PAD, p, b, h, v0, 0);

  bool aborted = false;
  for (int n = 0; n < NT; ++n) {
    const int sg = n & 1;
    uint8_t* stg = sm + sg * Cfg::STAGE;
    uint8_t* vt = stg + IMG_PAD;
    if (tid == 0) {
      if (ptx::mbar_wait(&full[sg], (n >> 1) & 1, kWaitNs)) pending &= ~(1u << sg);
      else *abort_flag = 1;
    }
    __syncthreads();                                       // (1) image n in smem
    if (*abort_flag) { aborted = true; break; }
    {
      // S -> f16 B operand (MN-major, K = 128): offset(k, v) = (v/8)*2048 + (k/8)*128 + (k%8)*16
      // and R3 <- d * S, in pieces of CW columns (register budget)
      const float dk = reinterpret_cast<const float*>(stg + IMG_D)[tid];
#pragma unroll 1
      for (int pc = 0; pc < NP; ++pc) {
        float srow[CW];
        ptx::tmem_ld<CW>(tlane + Cfg::R3 + pc * CW, srow);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int g8 = 0; g8 < CW / 8; ++g8)
          *reinterpret_cast<int4*>(Sb + (pc * (CW / 8) + g8) * 2048 + (tid >> 3) * 128 +
                                   (tid & 7) * 16) = pack8_f16(srow + 8 * g8);
#pragma unroll
        for (int j = 0; j < CW; ++j) srow[j] *= dk;
        ptx::tmem_st<CW>(tlane + Cfg::R3 + pc * CW, srow);
      }
      ptx::tmem_wait_st();
    }
    ptx::fence_proxy_async_smem();
    ptx::tc_fence_before();
    __syncthreads();                                       // (2) Sb, V tile, d*S ready
    if (tid == 0) {
      ptx::tc_fence_after();
      const uint32_t a2 = ptx::smem_u32(stg + IMG_A2), a1 = ptx::smem_u32(stg + IMG_A1);
      const uint32_t vb = ptx::smem_u32(vt), sb = ptx::smem_u32(Sb);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)                       // R2 = [M; Aout] V
        ptx::mma_f16_ss(tbase + Cfg::R2, ptx::sdesc(a2 + 256 * ks, 128, 1024),
                        ptx::sdesc(vb + 256 * ks, 128, 1024), IDESC, ks > 0);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)                       // R1 = [-W; Qbar] S
        ptx::mma_f16_ss(tbase + Cfg::R1, ptx::sdesc(a1 + 256 * ks, 128, 2048),
                        ptx::sdesc(sb + 256 * ks, 128, 2048), IDESC, ks > 0);
      ptx::tc_commit(mbar);
    }
    if (n + 1 < NT) load_vtile<VS, TIO>(sm + (sg ^ 1) * Cfg::STAGE + IMG_PAD, p, b, h, v0, n + 1);
    if (tid == 0 && !ptx::mbar_wait(mbar, 0, kWaitNs)) *abort_flag = 1;
    __syncthreads();                                       // (3) R1, R2 ready
    if (*abort_flag) { aborted = true; break; }
    ptx::tc_fence_after();
    if (warp < 2) {                                        // P = U - W S, rows c = tid
#pragma unroll 1
      for (int pc = 0; pc < NP; ++pc) {
        float u[CW], w[CW];
        ptx::tmem_ld<CW>(tlane + Cfg::R2 + pc * CW, u);
        ptx::tmem_ld<CW>(tlane + Cfg::R1 + pc * CW, w);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < CW; ++j) u[j] += w[j];
#pragma unroll
        for (int g8 = 0; g8 < CW / 8; ++g8)
          *reinterpret_cast<int4*>(Pb + (pc * (CW / 8) + g8) * 1024 + (tid >> 3) * 128 +
                                   (tid & 7) * 16) = pack8_f16(u + 8 * g8);
      }
    }
    ptx::fence_proxy_async_smem();
    ptx::tc_fence_before();
    __syncthreads();                                       // (4) P ready
    if (tid == 0) {
      ptx::tc_fence_after();
      const uint32_t a2 = ptx::smem_u32(stg + IMG_A2), a3 = ptx::smem_u32(stg + IMG_A3);
      const uint32_t pb = ptx::smem_u32(Pb);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)                       // R1 += [M; Aout] P
        ptx::mma_f16_ss(tbase + Cfg::R1, ptx::sdesc(a2 + 256 * ks, 128, 1024),
                        ptx::sdesc(pb + 256 * ks, 128, 1024), IDESC, 1u);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)                       // R3 += Kbar^T P
        ptx::mma_f16_ss(tbase + Cfg::R3, ptx::sdesc(a3 + 256 * ks, 128, 1024),
                        ptx::sdesc(pb + 256 * ks, 128, 1024), IDESC, 1u);
      ptx::tc_commit(mbar);
      if (!ptx::mbar_wait(mbar, 1, kWaitNs)) {
        *abort_flag = 1;
      } else if (n + 2 < NT) {                             // stage free: fetch chunk n+2
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive_expect_tx(&full[sg], IMG_BYTES);
        ptx::bulk_g2s(stg, wsh + (size_t)(n + 2) * IMG_BYTES, IMG_BYTES, &full[sg]);
        pending |= 1u << sg;
        pend_par = (pend_par & ~(1u << sg)) | ((((n + 2) >> 1) & 1u) << sg);
      }
    }
    __syncthreads();                                       // (5) O and next S ready
    if (*abort_flag) { aborted = true; break; }
    ptx::tc_fence_after();
    if (warp >= 2) {                                       // O rows c = tid - 64
      const int t = n * CH + (tid - 64);
      TIO* dst = static_cast<TIO*>(p.o) + b * p.o_s[0] + (int64_t)t * p.o_s[1] +
                 h * p.o_s[2] + v0;
#pragma unroll 1
      for (int pc = 0; pc < NP; ++pc) {
        float o[CW];
        ptx::tmem_ld<CW>(tlane + Cfg::R1 + pc * CW, o);
        ptx::tmem_wait_ld();
        if (t < T) {
          if (p.o_vec16) {
#pragma unroll
            for (int j = 0; j < CW; j += 4)
              st4(dst + pc * CW + j, *reinterpret_cast<float(*)[4]>(o + j));
          } else {
#pragma unroll
            for (int j = 0; j < CW; ++j) st(dst + pc * CW + j, o[j]);
          }
        }
      }
    }
    ptx::tc_fence_before();
  }

  __syncthreads();
  if (!aborted) {
    ptx::tc_fence_after();
    TSO* dst = static_cast<TSO*>(p.state_out) + b * p.so_s[0] + h * p.so_s[1] +
               (int64_t)tid * p.so_s[2] + v0;
#pragma unroll 1
    for (int pc = 0; pc < NP; ++pc) {
      float srow[CW];
      ptx::tmem_ld<CW>(tlane + Cfg::R3 + pc * CW, srow);
      ptx::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < CW; ++j) st(dst + pc * CW + j, srow[j]);
    }
  } else if (tid == 0) {
    atomicExch(&g_kda_device_error, 1);
    // let bulk copies still in flight land before this CTA's smem is released
    for (int sg = 0; sg < 2; ++sg)
      if (pending & (1u << sg)) ptx::mbar_wait(&full[sg], (pend_par >> sg) & 1u, kWaitNs / 2);
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, Cfg::NCOL);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int pick_vs(const ChunkParams& p) {
  const long heads = (long)p.B * p.H;
  int vs = 128;
  while (vs > 16 && (p.V % vs != 0 || heads * (p.V / vs) < 120)) vs /= 2;
  return (p.V % vs == 0) ? vs : 0;
}

template <typename TIO, typename TSI, typename TSO, int VS>
cudaError_t launch_state(const ChunkParams& p, const uint8_t* ws, cudaStream_t s) {
  auto kern = state_kernel<VS, TIO, TSI, TSO>;
  static bool attr_set = false;   // one attribute call per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         StateCfg<VS>::SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  dim3 grid(p.V / VS, p.H, p.B);
  kern<<<grid, 128, StateCfg<VS>::SMEM, s>>>(p, ws);
  return cudaGetLastError();
}

template <typename TIO, typename TSI, typename TSO>
cudaError_t launch_tc3(const ChunkParams& p, uint8_t* ws, cudaStream_t s) {
  auto prep = prep_kernel<TIO>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PREP_SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int NT = (p.T + CH - 1) / CH;
  dim3 pgrid(NT, p.H, p.B);
  prep<<<pgrid, PREP_THREADS, PREP_SMEM, s>>>(p, ws);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  switch (pick_vs(p)) {
    case 16: return launch_state<TIO, TSI, TSO, 16>(p, ws, s);
    case 32: return launch_state<TIO, TSI, TSO, 32>(p, ws, s);
    case 64: return launch_state<TIO, TSI, TSO, 64>(p, ws, s);
    case 128: return launch_state<TIO, TSI, TSO, 128>(p, ws, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename TIO, typename TSI>
cudaError_t launch_tc2(const ChunkParams& p, uint8_t* ws, cudaStream_t s) {
  switch (p.state_out_dtype) {
    case KDA_DTYPE_F32: return launch_tc3<TIO, TSI, float>(p, ws, s);
    case KDA_DTYPE_F16: return launch_tc3<TIO, TSI, __half>(p, ws, s);
    default: return launch_tc3<TIO, TSI, __nv_bfloat16>(p, ws, s);
  }
}

template <typename TIO>
cudaError_t launch_tc1(const ChunkParams& p, uint8_t* ws, cudaStream_t s) {
  switch (p.state_in_dtype) {
    case KDA_DTYPE_F32: return launch_tc2<TIO, float>(p, ws, s);
    case KDA_DTYPE_F16: return launch_tc2<TIO, __half>(p, ws, s);
    default: return launch_tc2<TIO, __nv_bfloat16>(p, ws, s);
  }
}

}  // namespace tc

bool chunk_tc_supported(const ChunkParams& p) {
  if (p.force_simt) return false;
  if (p.io_dtype != KDA_DTYPE_F16 && p.io_dtype != KDA_DTYPE_BF16) return false;
  if (p.K != tc::KD || p.T < 1 || p.V % 16 != 0) return false;
  return tc::pick_vs(p) != 0;
}

size_t chunk_tc_workspace_bytes(const ChunkParams& p) {
  const size_t NT = (size_t)(p.T + tc::CH - 1) / tc::CH;
  return (size_t)p.B * p.H * NT * tc::IMG_BYTES;
}

cudaError_t launch_chunk_tc(const ChunkParams& p, void* workspace, cudaStream_t s) {
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (p.io_dtype == KDA_DTYPE_F16) return tc::launch_tc1<__half>(p, ws, s);
  return tc::launch_tc1<__nv_bfloat16>(p, ws, s);
}

int read_device_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kda_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_kda_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

}  // namespace kda
