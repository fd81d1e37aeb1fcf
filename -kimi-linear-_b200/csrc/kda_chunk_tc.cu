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
//    and writes them, with V converted to f16, as ONE 82,432-byte image per
//    chunk whose byte layout is exactly the tcgen05 shared-memory operand
//    layout the second kernel uses, so that kernel moves a chunk with two bulk
//    (TMA-engine) copies: the shared operands and its own slice of V.
//
//    The decay products exp(gc_c - gc_i) are never formed pair by pair.  The
//    chunk is split into four 16-row blocks; with the per-step decays
//    alpha = exp(g), each row gets ra_c = exp(gc_c - gc_blockstart) (prefix
//    product) and nb_c = exp(gc_nextblockstart - gc_c) (suffix product), both
//    in (0, 1].  For a pair in different blocks the decay is
//    ra_c * nb_i * (product of the whole-block decays in between): a dense
//    16x16x128 tensor-core GEMM on pre-scaled operands (tf32 mma.sync, the A
//    fragments of a row block held in registers), with no overflow possible.  Inside a diagonal block the decay is
//    ra_c * nb_i * exp(-Z_r) with Z_r the block's total decay; that factor is
//    at most e^80 when the block is not "steep" (Z_r >= -80), which tf32 holds
//    exactly.  Channels of a steep block are removed from that GEMM and their
//    exact pair terms exp(gc_c - gc_i) are added separately (rare).
//    (I + L)^-1 is a blocked forward substitution: 16x16 diagonal blocks by
//    fp32 substitution, off-diagonal blocks M_rj = -D_r sum_t L_rt M_tj as
//    3xTF32 tensor-core products (fp32-level accuracy).
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
// chunk image (bytes); all operands f16 in the no-swizzle core-matrix layout
// (8 rows x 16 bytes per core matrix; LBO = stride along K, SBO = along M/N)
constexpr int IMG_A1 = 0;         // [-W; Qbar]  128 x 128 K-major, LBO 128, SBO 2048
constexpr int IMG_A2 = 32768;     // [M; Aout]   128 x 64  K-major, LBO 128, SBO 1024
constexpr int IMG_A3 = 49152;     // Kbar^T      128 x 64  K-major, LBO 128, SBO 1024
constexpr int IMG_D = 65536;      // d = exp(gc_last), fp32[128]
constexpr int IMG_SHARED = 66048; // bytes every value slice needs
constexpr int IMG_V = 66048;      // V 64 x 128 MN-major, LBO 128, SBO 1024 (slice v0: +v0*128)
constexpr int IMG_BYTES = 82432;
constexpr int IMG_PAD = 66560;    // shared part rounded up to 1 KiB (stage layout)

constexpr float kSteep = 80.f;                  // block decay beyond which exp(-Z) is unsafe
constexpr uint64_t kWaitNs = 2000000000ull;     // bound on every mbarrier wait (2 s)

__device__ __forceinline__ int a1_off(int m, int k) {
  return (m >> 3) * 2048 + (k >> 3) * 128 + (m & 7) * 16 + (k & 7) * 2;
}
__device__ __forceinline__ int a2_off(int m, int k) {
  return (m >> 3) * 1024 + (k >> 3) * 128 + (m & 7) * 16 + (k & 7) * 2;
}
// MN-major B operand with K = 64 rows: offset(c, v)
__device__ __forceinline__ int vb_off(int c, int v) {
  return (v >> 3) * 1024 + (c >> 3) * 128 + (c & 7) * 16 + (v & 7) * 2;
}

// two consecutive innermost elements as fp32 (vector load when `vec`)
template <typename T>
__device__ __forceinline__ float2 ld2(const T* p, bool vec) {
  if (vec) {
    if constexpr (std::is_same<T, float>::value) return *reinterpret_cast<const float2*>(p);
    if constexpr (std::is_same<T, __half>::value)
      return __half22float2(*reinterpret_cast<const __half2*>(p));
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
      return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  return make_float2(ld(p), ld(p + 1));
}
__device__ __forceinline__ void st_h2(uint8_t* base, int off, float a, float b) {
  *reinterpret_cast<__half2*>(base + off) = __floats2half2_rn(a, b);
}

// ---------------------------------------------------------------------------
// prep kernel
// ---------------------------------------------------------------------------
constexpr int AXP = 144;   // fp32 pitch of the Gram operands: float4 fragment loads conflict-free
constexpr int LMP = 68;    // fp32 pitch of L and M
constexpr int TSP = 24;    // fp32 pitch of the per-warp 16x16 scratch (conflict-free B loads)
constexpr int P_IMG = 0;
constexpr int P_AXK = 82944;                           // k * ra          fp32 [64][144]
constexpr int P_AXQ = P_AXK + CH * AXP * 4;            // s q * ra        fp32 [64][144]
constexpr int P_YB = P_AXQ + CH * AXP * 4;             // k * nb          fp32 [64][144]
constexpr int P_LM = P_YB + CH * AXP * 4;              // L               fp32 [64][68]
constexpr int P_FAC = P_LM + CH * LMP * 4;             // P02,P03,P13,E[4],Z[4],a0  [12][128]
constexpr int P_BETA = P_FAC + 12 * KD * 4;            // beta            fp32 [64]
constexpr int P_STEEP = P_BETA + CH * 4;               // steep bits      u32 [4][4]
constexpr int PREP_SMEM = P_STEEP + 16 * 4;
static_assert(P_AXK >= IMG_BYTES, "image staging");
static_assert(PREP_SMEM <= 227 * 1024, "prep shared memory");
// M (fp32, pitch LMP) reuses the k*ra array once the Gram is done, and the
// inversion scratch the q*ra array
constexpr int PREP_THREADS = 256;

// 3xTF32 split: x ~= hi + lo with both parts exact in tf32
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = ptx::f32_to_tf32(x);
  lo = ptx::f32_to_tf32(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma3_tf32(float* acc, const uint32_t* ah, const uint32_t* al,
                                          const uint32_t* bh, const uint32_t* bl) {
  ptx::mma_tf32_16x8x8(acc, al, bh);
  ptx::mma_tf32_16x8x8(acc, ah, bl);
  ptx::mma_tf32_16x8x8(acc, ah, bh);
}

// C[16x16] = A[16 x 8*ksteps] * B[8*ksteps x 16] in ~fp32 precision (3xTF32);
// A(row, k) = Ab[row*lda + k], B(k, col) = Bb[k*ldb + col]; result in acc[2][4]
// (n-tile nt: rows gid / gid+8, cols 8nt + 2tig (+1))
__device__ __forceinline__ void gemm16_3xtf32(float (*acc)[4], const float* Ab, int lda,
                                              const float* Bb, int ldb, int ksteps, int lane) {
  const int gid = lane >> 2, tig = lane & 3;
  for (int ks = 0; ks < ksteps; ++ks) {
    const int k0 = 8 * ks;
    uint32_t ah[4], al[4];
    split_tf32(Ab[gid * lda + k0 + tig], ah[0], al[0]);
    split_tf32(Ab[(gid + 8) * lda + k0 + tig], ah[1], al[1]);
    split_tf32(Ab[gid * lda + k0 + tig + 4], ah[2], al[2]);
    split_tf32(Ab[(gid + 8) * lda + k0 + tig + 4], ah[3], al[3]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      uint32_t bh[2], bl[2];
      split_tf32(Bb[(k0 + tig) * ldb + 8 * nt + gid], bh[0], bl[0]);
      split_tf32(Bb[(k0 + tig + 4) * ldb + 8 * nt + gid], bh[1], bl[1]);
      mma3_tf32(acc[nt], ah, al, bh, bl);
    }
  }
}

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
  float* Ef = P13 + KD;            // [4][128]  exp(-Z_r), 0 for steep channels
  float* Zs = Ef + 4 * KD;         // [4][128]  block decays Z_r
  float* A0 = Zs + 4 * KD;         // [128]     exp(g of row 0)
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
  const TIO* vb = static_cast<const TIO*>(p.v) + b * p.v_s[0] + h * p.v_s[2];
  const float* gb = p.g + b * p.g_s[0] + h * p.g_s[2];
  const float* bb = p.beta + b * p.b_s[0] + h * p.b_s[2];

  // ---- 0. zero L, the Aout half of [M; Aout], the steep mask; beta ---------
  for (int i = tid; i < CH * LMP; i += PREP_THREADS) Lm[i] = 0.f;
  for (int i = tid; i < 8192 / 16; i += PREP_THREADS)
    reinterpret_cast<int4*>(img + IMG_A2 + 8192)[i] = make_int4(0, 0, 0, 0);
  if (tid < 16) steep[tid] = 0u;
  if (tid < CH) sbeta[tid] = (tid < nvalid) ? bb[(int64_t)(t0 + tid) * p.b_s[1]] : 0.f;

  // ---- 1. per (16-row block r, channel pair): decays and decayed operands --
  const int r = tid >> 6, k0 = 2 * (tid & 63);
  float2 al[17];                    // al[i] = exp(g) of row 16r + i (i >= 1)
  float2 zr;
  {
    float2 gr[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) {
      const int c = 16 * r + i;
      gr[i] = (c < nvalid) ? ld2(gb + (int64_t)(t0 + c) * p.g_s[1] + k0, p.g_vec2)
                           : make_float2(0.f, 0.f);
    }
    // Z_r = sum of g over rows 16r+1 .. 16r+16 (..63 for the last block)
    zr = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 1; i < 17; ++i) {
      if (i == 16 && r == 3) break;
      zr.x += gr[i].x;
      zr.y += gr[i].y;
    }
#pragma unroll
    for (int i = 1; i < 17; ++i) al[i] = make_float2(__expf(gr[i].x), __expf(gr[i].y));
    if (r == 3) al[16] = make_float2(1.f, 1.f);
    Zs[r * KD + k0] = zr.x;
    Zs[r * KD + k0 + 1] = zr.y;
    if (r == 0) {
      A0[k0] = expf(gr[0].x);
      A0[k0 + 1] = expf(gr[0].y);
    }
  }
  __syncthreads();
  {
    float eZx[4], eZy[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      eZx[j] = expf(Zs[j * KD + k0]);
      eZy[j] = expf(Zs[j * KD + k0 + 1]);
    }
    float bfx = A0[k0], bfy = A0[k0 + 1];        // exp(gc at the block start)
    float afx = 1.f, afy = 1.f;                  // exp(gc_last - gc at the next block start)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j < r) { bfx *= eZx[j]; bfy *= eZy[j]; }
      if (j > r) { afx *= eZx[j]; afy *= eZy[j]; }
    }
    if (r == 0) {
      P02[k0] = eZx[1];                P02[k0 + 1] = eZy[1];
      P03[k0] = eZx[1] * eZx[2];       P03[k0 + 1] = eZy[1] * eZy[2];
      P13[k0] = eZx[2];                P13[k0 + 1] = eZy[2];
      float* dimg = reinterpret_cast<float*>(img + IMG_D);
      dimg[k0] = A0[k0] * eZx[0] * eZx[1] * eZx[2] * eZx[3];
      dimg[k0 + 1] = A0[k0 + 1] * eZy[0] * eZy[1] * eZy[2] * eZy[3];
    }
    {
      const bool stx = zr.x < -kSteep, sty = zr.y < -kSteep;
      Ef[r * KD + k0] = stx ? 0.f : expf(-zr.x);
      Ef[r * KD + k0 + 1] = sty ? 0.f : expf(-zr.y);
      const uint32_t bits = (stx ? 1u : 0u) | (sty ? 2u : 0u);
      if (bits) atomicOr(&steep[r * 4 + (k0 >> 5)], bits << (k0 & 31));
    }
    // ra: prefix products from the block start; nb: suffix products to the next block start
    float2 ra[16], nb[16];
    ra[0] = make_float2(1.f, 1.f);
#pragma unroll
    for (int i = 1; i < 16; ++i) ra[i] = make_float2(ra[i - 1].x * al[i].x, ra[i - 1].y * al[i].y);
    nb[15] = al[16];
#pragma unroll
    for (int i = 14; i >= 0; --i)
      nb[i] = make_float2(nb[i + 1].x * al[i + 1].x, nb[i + 1].y * al[i + 1].y);
    float kbx[16], kby[16];         // Kbar for the transposed store
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int c = 16 * r + i;
      float2 qv = make_float2(0.f, 0.f), kv = qv, vv = qv;
      if (c < nvalid) {
        qv = ld2(qb + (int64_t)(t0 + c) * p.q_s[1] + k0, p.qk_vec2);
        kv = ld2(kb + (int64_t)(t0 + c) * p.k_s[1] + k0, p.qk_vec2);
        vv = ld2(vb + (int64_t)(t0 + c) * p.v_s[1] + k0, p.v_vec2);
      }
      const float qsx = qv.x * s, qsy = qv.y * s;
      const float egx = bfx * ra[i].x, egy = bfy * ra[i].y;     // exp(gc_c)
      st_h2(img, IMG_A1 + a1_off(64 + c, k0), qsx * egx, qsy * egy);   // Qbar
      st_h2(img, IMG_A1 + a1_off(c, k0), kv.x * egx, kv.y * egy);      // Ktilde
      st_h2(img, IMG_V + vb_off(c, k0), vv.x, vv.y);                   // V (f16)
      kbx[i] = kv.x * nb[i].x * afx;                                   // Kbar
      kby[i] = kv.y * nb[i].y * afy;
      *reinterpret_cast<float2*>(Axk + c * AXP + k0) = make_float2(kv.x * ra[i].x, kv.y * ra[i].y);
      *reinterpret_cast<float2*>(Axq + c * AXP + k0) = make_float2(qsx * ra[i].x, qsy * ra[i].y);
      *reinterpret_cast<float2*>(Yb + c * AXP + k0) = make_float2(kv.x * nb[i].x, kv.y * nb[i].y);
    }
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      st_h2(img, IMG_A3 + a2_off(k0, 16 * r + i), kbx[i], kbx[i + 1]);
      st_h2(img, IMG_A3 + a2_off(k0 + 1, 16 * r + i), kby[i], kby[i + 1]);
    }
  }
  __syncthreads();

  // ---- 2. Gram blocks: warp = (row block rr, type); A fragments in registers.
  // The K order inside each 16-channel group is permuted (sums are order-free)
  // so every fragment element pair comes from one float4 load.
  {
    const int gid = lane >> 2, tig = lane & 3;
    const int rr = warp & 3, type = warp >> 2;          // type 0: L (x = k), 1: Aout (x = s q)
    const float* Ax = type ? Axq : Axk;
    uint32_t af[8][2][4];                               // [16-channel group][k-step][frag]
    float4 arow0[8], arow1[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      arow0[g] = *reinterpret_cast<const float4*>(Ax + (16 * rr + gid) * AXP + 16 * g + 4 * tig);
      arow1[g] = *reinterpret_cast<const float4*>(Ax + (16 * rr + gid + 8) * AXP + 16 * g + 4 * tig);
    }
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      af[g][0][0] = ptx::f32_to_tf32(arow0[g].x);
      af[g][0][1] = ptx::f32_to_tf32(arow1[g].x);
      af[g][0][2] = ptx::f32_to_tf32(arow0[g].y);
      af[g][0][3] = ptx::f32_to_tf32(arow1[g].y);
      af[g][1][0] = ptx::f32_to_tf32(arow0[g].z);
      af[g][1][1] = ptx::f32_to_tf32(arow1[g].z);
      af[g][1][2] = ptx::f32_to_tf32(arow0[g].w);
      af[g][1][3] = ptx::f32_to_tf32(arow1[g].w);
    }
    for (int j = 0; j <= rr; ++j) {
      const float* f = nullptr;                         // per-channel factor on the B side
      if (j == rr) f = Ef + rr * KD;
      else if (rr - j == 2) f = (j == 0) ? P02 : P13;
      else if (rr - j == 3) f = P03;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const int kc = 16 * g + 4 * tig;
        const float4 fv = f ? *reinterpret_cast<const float4*>(f + kc) : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float4 y = *reinterpret_cast<const float4*>(Yb + (16 * j + 8 * nt + gid) * AXP + kc);
          const uint32_t b0[2] = {ptx::f32_to_tf32(y.x * fv.x), ptx::f32_to_tf32(y.y * fv.y)};
          const uint32_t b1[2] = {ptx::f32_to_tf32(y.z * fv.z), ptx::f32_to_tf32(y.w * fv.w)};
          ptx::mma_tf32_16x8x8(acc[nt], af[g][0], b0);
          ptx::mma_tf32_16x8x8(acc[nt], af[g][1], b1);
        }
      }
      if (j == rr) {
        // exact pair terms of the steep channels of this diagonal block (rare)
#pragma unroll 1
        for (int w4 = 0; w4 < 4; ++w4) {
          uint32_t m = steep[rr * 4 + w4];
          while (m) {
            const int kk = w4 * 32 + __ffs(m) - 1;
            m &= m - 1;
            float pre[16];
            pre[0] = 0.f;
#pragma unroll
            for (int i = 1; i < 16; ++i) {
              const int c = 16 * rr + i;
              pre[i] = pre[i - 1] + ((c < nvalid) ? gb[(int64_t)(t0 + c) * p.g_s[1] + kk] : 0.f);
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int rl = gid + 8 * (e >> 1), cl = 8 * nt + 2 * tig + (e & 1);
                const int c = 16 * rr + rl, i = 16 * rr + cl;
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
          const int row = 16 * rr + gid + 8 * (e >> 1);
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

  // ---- 3. M = (I + L)^-1 Diag(beta): blocked forward substitution ----------
  float* Mm = Axk;                     // pitch LMP
  float* Ts = Axq;                     // per-warp 16 x TSP scratch
  if (warp < 4) {                      // diagonal blocks by substitution (fp32)
    const int rb = warp;
    if (lane < 16) {
      const int j = lane;
      float x[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float acc = (c == j) ? 1.f : 0.f;
#pragma unroll
        for (int i = 0; i < c; ++i) acc = fmaf(-Lm[(16 * rb + c) * LMP + 16 * rb + i], x[i], acc);
        x[c] = acc;
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) Mm[(16 * rb + c) * LMP + 16 * rb + j] = x[c];
    }
  } else {
    for (int idx = tid - 128; idx < CH * CH; idx += 128) {
      const int row = idx >> 6, col = idx & 63;
      if ((col >> 4) > (row >> 4)) Mm[row * LMP + col] = 0.f;
    }
  }
  __syncthreads();
  // off-diagonal blocks M_rj = -D_r sum_{t=j}^{r-1} L_rt M_tj, by distance r - j
  for (int dist = 1; dist <= 3; ++dist) {
    if (warp < 4 - dist) {
      const int j = warp, rb = warp + dist;
      const int gid = lane >> 2, tig = lane & 3;
      float tacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      gemm16_3xtf32(tacc, Lm + (16 * rb) * LMP + 16 * j, LMP, Mm + (16 * j) * LMP + 16 * j, LMP,
                    2 * dist, lane);
      float* T = Ts + warp * (16 * TSP);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          T[(gid + 8 * (e >> 1)) * TSP + 8 * nt + 2 * tig + (e & 1)] = tacc[nt][e];
      __syncwarp();
      float macc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      gemm16_3xtf32(macc, Mm + (16 * rb) * LMP + 16 * rb, LMP, T, TSP, 2, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          Mm[(16 * rb + gid + 8 * (e >> 1)) * LMP + 16 * j + 8 * nt + 2 * tig + (e & 1)] =
              -macc[nt][e];
    }
    __syncthreads();
  }
  for (int idx = tid; idx < CH * CH / 2; idx += PREP_THREADS) {
    const int row = idx >> 5, col = 2 * (idx & 31);
    st_h2(img, IMG_A2 + a2_off(row, col), Mm[row * LMP + col] * sbeta[col],
          Mm[row * LMP + col + 1] * sbeta[col + 1]);
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
        st_h2(img, IMG_A1 + a1_off(row, col), -acc[nt][2 * hr], -acc[nt][2 * hr + 1]);
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
  static constexpr int VT_BYTES = CH * VS * 2;                 // V slice, K = 64 rows
  static constexpr int STAGE = IMG_PAD + ((VT_BYTES + 1023) / 1024) * 1024;
  static constexpr int SB_OFF = 2 * STAGE;                     // S  (K = 128) f16
  static constexpr int PB_OFF = SB_OFF + KD * VS * 2;          // P  (K = 64)  f16
  static constexpr int BAR_OFF = PB_OFF + CH * VS * 2;
  static constexpr int SMEM = BAR_OFF + 64;
  static constexpr uint32_t TX = IMG_SHARED + VT_BYTES;        // bytes per chunk
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

__device__ __forceinline__ void named_barrier_64() {
  asm volatile("bar.sync 1, 64;" ::: "memory");
}

template <int VS>
__device__ __forceinline__ void fetch_chunk(uint8_t* stg, const uint8_t* img_g, int v0,
                                            uint64_t* bar) {
  ptx::mbar_arrive_expect_tx(bar, StateCfg<VS>::TX);
  ptx::bulk_g2s(stg, img_g, IMG_SHARED, bar);
  ptx::bulk_g2s(stg + IMG_PAD, img_g + IMG_V + v0 * 128, StateCfg<VS>::VT_BYTES, bar);
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
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Cfg::BAR_OFF);   // [2] chunk images
  uint64_t* mbarA = full + 2;      // first MMA batch of a chunk done (one phase per chunk)
  uint64_t* mbarB = full + 3;      // second MMA batch of a chunk done (one phase per chunk)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(full + 4);
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
    ptx::mbar_init(mbarA, 1);
    ptx::mbar_init(mbarB, 1);
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
      fetch_chunk<VS>(sm + sg * Cfg::STAGE, wsh + (size_t)sg * IMG_BYTES, v0, &full[sg]);
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

  bool aborted = false;
  for (int n = 0; n < NT; ++n) {
    const int sg = n & 1;
    uint8_t* stg = sm + sg * Cfg::STAGE;
    uint8_t* vt = stg + IMG_PAD;
    // every thread waits for image n itself (bounded)
    if (ptx::mbar_wait(&full[sg], (n >> 1) & 1, kWaitNs)) {
      if (tid == 0) pending &= ~(1u << sg);
    } else {
      *abort_flag = 1;
    }
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
    __syncthreads();                                       // Sb and d*S ready
    if (*abort_flag) { aborted = true; break; }
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
      ptx::tc_commit(mbarA);
    }
    // Warps 0-1 consume the first MMA batch; warps 2-3 only need the second.
    // Each batch has its own barrier completing once per chunk, so the phase a
    // thread waits for has parity n & 1 and can never be lapped: the next
    // phase of either barrier needs the next chunk's CTA barrier.
    const uint32_t par = static_cast<uint32_t>(n & 1);
    if (warp < 2) {                                        // P = U - W S, rows c = tid
      if (!ptx::mbar_wait(mbarA, par, kWaitNs)) *abort_flag = 1;
      ptx::tc_fence_after();
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
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      named_barrier_64();                                  // P ready (warps 0-1)
      if (tid == 0) {
        ptx::tc_fence_after();
        const uint32_t a2 = ptx::smem_u32(stg + IMG_A2), a3 = ptx::smem_u32(stg + IMG_A3);
        const uint32_t pb = ptx::smem_u32(Pb);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)                     // R3 += Kbar^T P (next state first)
          ptx::mma_f16_ss(tbase + Cfg::R3, ptx::sdesc(a3 + 256 * ks, 128, 1024),
                          ptx::sdesc(pb + 256 * ks, 128, 1024), IDESC, 1u);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)                     // R1 += [M; Aout] P
          ptx::mma_f16_ss(tbase + Cfg::R1, ptx::sdesc(a2 + 256 * ks, 128, 1024),
                          ptx::sdesc(pb + 256 * ks, 128, 1024), IDESC, 1u);
        ptx::tc_commit(mbarB);
      }
    }
    if (!ptx::mbar_wait(mbarB, par, kWaitNs)) *abort_flag = 1;
    ptx::tc_fence_after();
    if (tid == 0 && n + 2 < NT && !*abort_flag) {          // stage free: fetch chunk n+2
      ptx::fence_proxy_async_smem();
      fetch_chunk<VS>(stg, wsh + (size_t)(n + 2) * IMG_BYTES, v0, &full[sg]);
      pending |= 1u << sg;
      pend_par = (pend_par & ~(1u << sg)) | ((((n + 2) >> 1) & 1u) << sg);
    }
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
  if (!aborted && !*abort_flag) {
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
  if (p.K != tc::KD || p.V != tc::KD || p.T < 1) return false;
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
