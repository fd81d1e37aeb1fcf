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
//      W = M (exp(gc) * K),  U = M V                         (kda.py:172-173)
//      Qbar = s q exp(gc),  Kbar = exp(gc_last - gc) k,  d = exp(gc_last)
//      E = Qbar - Aout W,   F = Aout U
//    (kda.py:177-178 give O = Qbar S + Aout (U - W S) = E S + F, so the state
//    pass needs no Aout product of its own) and writes them as ONE
//    82,432-byte image per chunk whose byte layout is exactly the shared-memory
//    layout the second kernel uses, so that kernel moves a chunk with three
//    bulk (TMA-engine) copies: the shared operands and its slices of U and F.
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
//    chunk (kda.py:176-182), 12 tcgen05 MMAs in two dependent batches:
//      R1  = [-W; E] S                                        (8 MMAs, K = 128)
//      P   = U + R1[0:64]  (= U - W S)   -> smem f16          (warps 0-1)
//      O   = R1[64:128] + F  (= Qbar S + Aout P)  -> global   (warps 2-3)
//      R3  = d * S,  R3 += Kbar^T P  -> next S                (4 MMAs, K = 64)
//    Operands are f16 (bf16 inputs are exactly representable in f16 at these
//    magnitudes); every product accumulates in fp32 TMEM, and the carried
//    state never leaves fp32 (the reference rounds S to the transient dtype
//    for its two state GEMMs, kda.py:176, as the f16 copy here does).
//    The images are double-buffered in shared memory and fetched two chunks
//    ahead with cp.async.bulk; every mbarrier wait is bounded in time and
//    aborts the CTA cleanly (error word, TMEM freed) instead of hanging.
#include <cuda.h>            // CUtensorMap (header only; the encoder comes from the runtime)
#include <type_traits>

#include "kda_internal.cuh"
#include "tc_ptx.cuh"

namespace kda {

__device__ int g_kda_device_error = 0;

namespace tc {

constexpr int CH = 64;        // rows per chunk
constexpr int KD = 128;       // head dim K (= V) of this path
// Chunk image (bytes).  A1 and A3 are tcgen05 A operands in the no-swizzle
// K-major core-matrix layout (8 rows x 16 bytes per core matrix; LBO = stride
// along K, SBO = along M).  U and F are read by threads; their layout
// (v/8)*1024 + c*16 + (v%8)*2 keeps a slice of value columns v0..v0+VS one
// contiguous byte range (v0*128 .. (v0+VS)*128).
constexpr int IMG_A1 = 0;         // [-W; E]   128 x 128 f16, LBO 128, SBO 2048  (E = Qbar - Aout W)
constexpr int IMG_A3 = 32768;     // Kbar^T    128 x 64  f16, LBO 128, SBO 1024
constexpr int IMG_D = 49152;      // d = exp(gc_last), fp32[128]
constexpr int IMG_SHARED = 49664; // bytes every value slice needs
constexpr int IMG_U = 49664;      // U = M V        64 x 128 f16
constexpr int IMG_F = 66048;      // F = Aout U     64 x 128 f16
constexpr int IMG_BYTES = 82432;

constexpr float kSteep = 80.f;                  // block decay beyond which exp(-Z) is unsafe
constexpr uint64_t kWaitNs = 2000000000ull;     // bound on every mbarrier wait (2 s)

__device__ __forceinline__ int a1_off(int m, int k) {
  return (m >> 3) * 2048 + (k >> 3) * 128 + (m & 7) * 16 + (k & 7) * 2;
}
__device__ __forceinline__ int a2_off(int m, int k) {
  return (m >> 3) * 1024 + (k >> 3) * 128 + (m & 7) * 16 + (k & 7) * 2;
}
// 64 x 128 layout of V, U and F: offset(c, v).  Each block of 8 value columns
// is 1 KiB (64 rows x 16 bytes).  For V this is the MN-major no-swizzle
// operand layout of the phase-5 GEMM (core-matrix stride 128 bytes along the
// chunk rows, 1 KiB along the value columns); U and F are read by threads.
__device__ __forceinline__ int vb_off(int c, int v) {
  return (v >> 3) * 1024 + c * 16 + (v & 7) * 2;
}
// pack two fp32 as f16x2
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// 4x4 transpose of 32-bit values across the four lanes of a quad:
// in: x[i] = value of this lane for item i; out: x[i] = value of lane i for
// item (lane & 3)
__device__ __forceinline__ void quad_transpose(uint32_t (&x)[4], int tig) {
  {
    const bool hi = tig & 2;
    const uint32_t r0 = __shfl_xor_sync(0xffffffffu, hi ? x[0] : x[2], 2);
    const uint32_t r1 = __shfl_xor_sync(0xffffffffu, hi ? x[1] : x[3], 2);
    if (hi) { x[0] = r0; x[1] = r1; } else { x[2] = r0; x[3] = r1; }
  }
  {
    const bool od = tig & 1;
    const uint32_t r0 = __shfl_xor_sync(0xffffffffu, od ? x[0] : x[1], 1);
    const uint32_t r1 = __shfl_xor_sync(0xffffffffu, od ? x[2] : x[3], 1);
    if (od) { x[0] = r0; x[2] = r1; } else { x[1] = r0; x[3] = r1; }
  }
}

// two consecutive innermost elements as fp32 through the read-only path
template <bool VEC, typename T>
__device__ __forceinline__ float2 ldg2(const T* p) {
  if constexpr (VEC) {
    if constexpr (std::is_same<T, float>::value) {
      return __ldg(reinterpret_cast<const float2*>(p));
    } else {
      const unsigned int u = __ldg(reinterpret_cast<const unsigned int*>(p));
      if constexpr (std::is_same<T, __half>::value)
        return __half22float2(*reinterpret_cast<const __half2*>(&u));
      else
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
    }
  } else {
    return make_float2(ld(p), ld(p + 1));
  }
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
constexpr int P_IMG = 0;                               // output image staging
constexpr int P_A2 = 82944;                            // [M; Aout] f16, K-major LBO 128 SBO 1024
constexpr int P_AXK = P_A2 + 16384;                    // k * ra          fp32 [64][144]
constexpr int P_AXQ = P_AXK + CH * AXP * 4;            // s q * ra        fp32 [64][144]
constexpr int P_YB = P_AXQ + CH * AXP * 4;             // k * nb          fp32 [64][144]
constexpr int P_LM = P_YB + CH * AXP * 4;              // L               fp32 [64][68]
constexpr int P_FAC = P_LM + CH * LMP * 4;             // P02,P03,P13,E[4]  fp32 [7][128]
constexpr int P_BETA = P_FAC + 7 * KD * 4;             // beta            fp32 [64]
constexpr int P_STEEP = P_BETA + CH * 4;               // steep bits      u32 [4][4]
constexpr int P_MBAR = P_STEEP + 16 * 4;               // tcgen05 commit barrier (u64)
constexpr int P_TBAR = P_MBAR + 8;                     // input tensor copies (u64)
constexpr int P_TSLOT = P_TBAR + 8;                    // TMEM base address (u32)
// LOAD == 3: the chunk's raw q, k, v (64 x 128, I/O dtype) and g (64 x 128
// fp32) rows land by tensor copies here, in the Gram-operand region that
// phase 1 writes only after every thread has read its inputs
constexpr int P_STG = P_AXK;
constexpr int STG_BYTES_G = CH * KD * 4;
constexpr int PREP_SMEM = P_TSLOT + 8;
constexpr int kPrepTmemCols = 256;                     // D[128 x 256] fp32 of phase 5
static_assert(P_A2 >= IMG_BYTES, "image staging");
static_assert(PREP_SMEM <= 227 * 1024, "prep shared memory");
// Aliases once their owners are dead: half-block decays Z[8][128] and exp(g_0)[128]
// live in the L array during phase 1 (L is written only in phase 2, and only
// where it is read later); M (fp32, pitch LMP) reuses the k*ra array and the
// inversion scratch the q*ra array once the Gram is done.
constexpr int PREP_THREADS = 512;

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

// C[16x16] += A[16 x 8*KSTEPS] * B[8*KSTEPS x 16] at ~fp32 accuracy (3xTF32);
// A(row, k) = Ab[row*lda + k], B(k, col) = Bb[k*ldb + col]; acc[nt] holds
// rows gid / gid+8, cols 8nt + 2tig (+1)
template <int KSTEPS>
__device__ __forceinline__ void gemm16_3xtf32(float (*acc)[4], const float* Ab, int lda,
                                              const float* Bb, int ldb, int lane) {
  const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
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

// C[16x8] += A[16 x 8*KSTEPS] * B[8*KSTEPS x 8] at ~fp32 accuracy (3xTF32),
// one n-tile of gemm16_3xtf32: B(k, col) = Bb[k*ldb + col], col < 8
template <int KSTEPS>
__device__ __forceinline__ void gemm16x8_3xtf32(float* acc, const float* Ab, int lda,
                                                const float* Bb, int ldb, int lane) {
  const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    const int k0 = 8 * ks;
    uint32_t ah[4], al[4], bh[2], bl[2];
    split_tf32(Ab[gid * lda + k0 + tig], ah[0], al[0]);
    split_tf32(Ab[(gid + 8) * lda + k0 + tig], ah[1], al[1]);
    split_tf32(Ab[gid * lda + k0 + tig + 4], ah[2], al[2]);
    split_tf32(Ab[(gid + 8) * lda + k0 + tig + 4], ah[3], al[3]);
    split_tf32(Bb[(k0 + tig) * ldb + gid], bh[0], bl[0]);
    split_tf32(Bb[(k0 + tig + 4) * ldb + gid], bh[1], bl[1]);
    mma3_tf32(acc, ah, al, bh, bl);
  }
}

// tensor maps of q, k, v ([B, T, H, K], I/O dtype) and g (fp32) for LOAD == 3:
// box = one (b, h) and 64 rows x 128 channels
struct alignas(64) PrepMaps {
  CUtensorMap q, k, v, g;
};

// two consecutive elements of a shared-memory row as fp32
template <typename T>
__device__ __forceinline__ float2 lds2(const T* p) {
  if constexpr (std::is_same<T, float>::value) {
    return *reinterpret_cast<const float2*>(p);
  } else if constexpr (std::is_same<T, __half>::value) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
  } else {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
}

// LOAD: how phase 1 reads its inputs -- 0 scalar loads, 1 two-element vector
// loads, 2 vector loads and, every input row being a 16-byte-aligned range,
// the next wave's L2 prefetch issued as one bulk (TMA-engine) prefetch per
// row; 3 as 2 but the chunk's inputs arrive by four tensor copies (TMA)
// instead of per-thread loads, which the SM's limit on outstanding loads caps
// at ~10 bytes per cycle.
template <typename TIO, int LOAD>
__global__ void __launch_bounds__(PREP_THREADS, 1)
prep_kernel(const ChunkParams p, uint8_t* __restrict__ ws, const __grid_constant__ PrepMaps tm) {
  constexpr bool VEC = LOAD >= 1;
  ptx::grid_dep_launch();          // the state pass may start launching (it waits for this grid)
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* img = sm + P_IMG;
  uint8_t* A2 = sm + P_A2;
  float* Axk = reinterpret_cast<float*>(sm + P_AXK);
  float* Axq = reinterpret_cast<float*>(sm + P_AXQ);
  float* Yb = reinterpret_cast<float*>(sm + P_YB);
  float* Lm = reinterpret_cast<float*>(sm + P_LM);
  float* Zs = Lm;                  // [4][2][128] half-block decay sums (phase 1 only)
  float* A0 = Lm + 8 * KD;         // [128]       exp(g of row 0)        (phase 1 only)
  float* P02 = reinterpret_cast<float*>(sm + P_FAC);
  float* P03 = P02 + KD;
  float* P13 = P03 + KD;
  float* Ef = P13 + KD;            // [4][128]  exp(-Z_r), 0 for steep channels
  float* sbeta = reinterpret_cast<float*>(sm + P_BETA);
  uint32_t* steep = reinterpret_cast<uint32_t*>(sm + P_STEEP);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + P_MBAR);
  uint64_t* tbar = reinterpret_cast<uint64_t*>(sm + P_TBAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + P_TSLOT);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const float s = p.scale;
  // chunk images in linear order n + NT (h + H b) (the workspace order).  The
  // TMA-input instantiation is persistent (one CTA per SM walks every
  // stride-th chunk); the others run one chunk per CTA over an (NT, H, B) grid.
  const int NT = (p.T + CH - 1) / CH;
  const int total = NT * p.H * p.B;                   // < 2^31 (checked on the host)
  const int stride = gridDim.x * gridDim.y * gridDim.z;
  int chunk = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  // the four input boxes of chunk c into the staging region (thread 32; rows
  // past T arrive as zeros)
  auto issue_inputs = [&](int c) {
    const int n2 = c % NT, h2 = (c / NT) % p.H, b2 = c / (NT * p.H);
    uint8_t* stg = sm + P_STG;
    ptx::mbar_arrive_expect_tx(tbar, 3 * CH * KD * sizeof(TIO) + STG_BYTES_G);
    ptx::tma_load_4d(stg, &tm.q, 0, h2, n2 * CH, b2, tbar);
    ptx::tma_load_4d(stg + CH * KD * sizeof(TIO), &tm.k, 0, h2, n2 * CH, b2, tbar);
    ptx::tma_load_4d(stg + 2 * CH * KD * sizeof(TIO), &tm.v, 0, h2, n2 * CH, b2, tbar);
    ptx::tma_load_4d(stg + 3 * CH * KD * sizeof(TIO), &tm.g, 0, h2, n2 * CH, b2, tbar);
  };

  // the first chunk's input copies go first
  if (tid == 32) {
    ptx::mbar_init(mbar, 1);
    if constexpr (LOAD == 3) ptx::mbar_init(tbar, 1);
    ptx::fence_mbar_init();
    if constexpr (LOAD == 3) {
      if (chunk < total) issue_inputs(chunk);
    }
  }
  if (warp == 0) {                  // TMEM for phase 5 (one CTA per SM: never contended)
    ptx::tmem_alloc(tslot, kPrepTmemCols);
    ptx::tmem_relinquish();
    ptx::tc_fence_before();
  }

#pragma unroll 1
  for (uint32_t it = 0; chunk < total; chunk += stride, ++it) {
  const int n = chunk % NT, h = (chunk / NT) % p.H, b = chunk / (NT * p.H);
  const int t0 = n * CH;
  const int nvalid = min(CH, p.T - t0);
  const TIO* qb = static_cast<const TIO*>(p.q) + b * p.q_s[0] + h * p.q_s[2];
  const TIO* kb = static_cast<const TIO*>(p.k) + b * p.k_s[0] + h * p.k_s[2];
  const TIO* vb = static_cast<const TIO*>(p.v) + b * p.v_s[0] + h * p.v_s[2];
  const float* gb = p.g + b * p.g_s[0] + h * p.g_s[2];
  const float* bb = p.beta + b * p.b_s[0] + h * p.b_s[2];

  // beta waits in a register until the inputs landed (its load latency then
  // overlaps theirs) and reaches shared memory with the phase-1 barrier
  if (tid < 16) steep[tid] = 0u;
  const float beta_c = (tid < nvalid) ? bb[(int64_t)(t0 + min(tid, CH - 1)) * p.b_s[1]] : 0.f;

  // L2 prefetch of inputs a chunk period ahead: the next chunk of this CTA
  // (persistent; its copies are issued after phase 3 and then hit L2), or the
  // chunk one SM-count further in launch order (the CTA that starts on this
  // SM when this one retires).
  {
    const long tgt = LOAD == 3 ? (long)chunk + stride : (long)chunk + ptx::num_sms();
    if (tgt < total) {
      const int n2 = (int)(tgt % NT), h2 = (int)((tgt / NT) % p.H), b2 = (int)(tgt / ((long)NT * p.H));
      if constexpr (LOAD == 3) {                   // four box prefetches
        if (tid == 32) {
          ptx::tma_prefetch_4d(&tm.q, 0, h2, n2 * CH, b2);
          ptx::tma_prefetch_4d(&tm.k, 0, h2, n2 * CH, b2);
          ptx::tma_prefetch_4d(&tm.v, 0, h2, n2 * CH, b2);
          ptx::tma_prefetch_4d(&tm.g, 0, h2, n2 * CH, b2);
        }
      } else if constexpr (LOAD == 2) {            // one TMA-engine prefetch per row
        const int c = tid >> 2, part = tid & 3;
        const int64_t t = (int64_t)n2 * CH + c;
        if (c < CH && t < p.T) {
          if (part == 0)
            ptx::bulk_prefetch_l2(static_cast<const TIO*>(p.q) + b2 * p.q_s[0] + t * p.q_s[1] + h2 * p.q_s[2], KD * sizeof(TIO));
          else if (part == 1)
            ptx::bulk_prefetch_l2(static_cast<const TIO*>(p.k) + b2 * p.k_s[0] + t * p.k_s[1] + h2 * p.k_s[2], KD * sizeof(TIO));
          else if (part == 2)
            ptx::bulk_prefetch_l2(static_cast<const TIO*>(p.v) + b2 * p.v_s[0] + t * p.v_s[1] + h2 * p.v_s[2], KD * sizeof(TIO));
          else
            ptx::bulk_prefetch_l2(p.g + b2 * p.g_s[0] + t * p.g_s[1] + h2 * p.g_s[2], KD * 4);
        }
      } else
      for (int idx = tid; idx < CH * 10; idx += PREP_THREADS) {
        const int c = idx / 10, part = idx - 10 * (idx / 10);
        const int t = n2 * CH + c;
        if (t >= p.T) continue;
        const uint8_t* a;
        if (part < 2)
          a = reinterpret_cast<const uint8_t*>(static_cast<const TIO*>(p.q) + b2 * p.q_s[0] +
                                               (int64_t)t * p.q_s[1] + h2 * p.q_s[2]) + 128 * part;
        else if (part < 4)
          a = reinterpret_cast<const uint8_t*>(static_cast<const TIO*>(p.k) + b2 * p.k_s[0] +
                                               (int64_t)t * p.k_s[1] + h2 * p.k_s[2]) + 128 * (part - 2);
        else if (part < 6)
          a = reinterpret_cast<const uint8_t*>(static_cast<const TIO*>(p.v) + b2 * p.v_s[0] +
                                               (int64_t)t * p.v_s[1] + h2 * p.v_s[2]) + 128 * (part - 4);
        else
          a = reinterpret_cast<const uint8_t*>(p.g + b2 * p.g_s[0] + (int64_t)t * p.g_s[1] +
                                               h2 * p.g_s[2]) + 128 * (part - 6);
        ptx::prefetch_l2(a);
      }
    }
  }

  // ---- 1. per (16-row block r, 8-row half hf, channel pair): decays and
  // decayed operands.  Warp w: r = w / 4, hf = (w / 2) % 2, channels
  // 64 (w % 2) .. +63 (a channel pair per lane).  The two halves of a block
  // meet through shared memory (their partial decay sums).
  const int r = warp >> 2, hf = (warp >> 1) & 1;
  const int k0 = 64 * (warp & 1) + 2 * lane;
  const int rb0 = 16 * r + 8 * hf;                 // first row of this thread
  // every input row of this thread, loaded unconditionally (rows past T are
  // clamped to the last valid row and zeroed below) so the loads overlap;
  // gr[8] is the row after the half (next half or next block)
  float2 gr[9], qr[8], kr[8], vr[8];
  if constexpr (LOAD == 3) {
    __syncthreads();                                 // tbar initialised, steep reset
    const bool in_ok = ptx::mbar_wait(tbar, it & 1u, kWaitNs);
    if (__syncthreads_or(!in_ok)) {                  // the copies never landed: give up
      if (tid == 32) {
        atomicExch(&g_kda_device_error, 3);
        ptx::mbar_wait(tbar, it & 1u, kWaitNs / 2);  // let them land before smem is released
      }
      __syncthreads();
      if (warp == 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(*tslot, kPrepTmemCols);
      }
      return;
    }
    const TIO* sq = reinterpret_cast<const TIO*>(sm + P_STG);
    const TIO* sk = sq + CH * KD;
    const TIO* sv = sk + CH * KD;
    const float* sgp = reinterpret_cast<const float*>(sv + CH * KD);
#pragma unroll
    for (int i = 0; i < 9; ++i)      // row 64 (last half, i = 8) is not needed: clamp, zeroed below
      gr[i] = *reinterpret_cast<const float2*>(sgp + min(rb0 + i, CH - 1) * KD + k0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      qr[i] = lds2(sq + (rb0 + i) * KD + k0);
      kr[i] = lds2(sk + (rb0 + i) * KD + k0);
      vr[i] = lds2(sv + (rb0 + i) * KD + k0);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 9; ++i) {
      const int c = min(rb0 + i, nvalid - 1);
      gr[i] = ldg2<VEC>(gb + (int64_t)(t0 + c) * p.g_s[1] + k0);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = min(rb0 + i, nvalid - 1);
      qr[i] = ldg2<VEC>(qb + (int64_t)(t0 + c) * p.q_s[1] + k0);
      kr[i] = ldg2<VEC>(kb + (int64_t)(t0 + c) * p.k_s[1] + k0);
      vr[i] = ldg2<VEC>(vb + (int64_t)(t0 + c) * p.v_s[1] + k0);
    }
  }
  float2 al[9];                     // al[i] = exp(g) of row rb0 + i (i >= 1)
  float2 zh = make_float2(0.f, 0.f);  // sum of g over rows rb0+1 .. rb0+8 (this half's share of Z_r)
#pragma unroll
  for (int i = 0; i < 9; ++i) {
    const bool ok = (rb0 + i < nvalid) && !(i == 8 && hf == 1 && r == 3);
    if (!ok) gr[i] = make_float2(0.f, 0.f);
    if (i >= 1) {
      zh.x += gr[i].x;
      zh.y += gr[i].y;
      al[i] = make_float2(__expf(gr[i].x), __expf(gr[i].y));
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (rb0 + i >= nvalid) qr[i] = kr[i] = vr[i] = make_float2(0.f, 0.f);
  Zs[(2 * r + hf) * KD + k0] = zh.x;                // [4 blocks][2 halves][128]
  Zs[(2 * r + hf) * KD + k0 + 1] = zh.y;
  if (r == 0 && hf == 0) {
    A0[k0] = expf(gr[0].x);
    A0[k0 + 1] = expf(gr[0].y);
  }
  if (tid < CH) sbeta[tid] = beta_c;
  __syncthreads();
  {
    float Zx[4], Zy[4], eZx[4], eZy[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      Zx[j] = Zs[(2 * j) * KD + k0] + Zs[(2 * j + 1) * KD + k0];
      Zy[j] = Zs[(2 * j) * KD + k0 + 1] + Zs[(2 * j + 1) * KD + k0 + 1];
      eZx[j] = expf(Zx[j]);
      eZy[j] = expf(Zy[j]);
    }
    // the other half's share of the block decay
    const float ox = Zs[(2 * r + (hf ^ 1)) * KD + k0], oy = Zs[(2 * r + (hf ^ 1)) * KD + k0 + 1];
    float bfx = A0[k0], bfy = A0[k0 + 1];        // exp(gc at the block start)
    float afx = 1.f, afy = 1.f;                  // exp(gc_last - gc at the next block start)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j < r) { bfx *= eZx[j]; bfy *= eZy[j]; }
      if (j > r) { afx *= eZx[j]; afy *= eZy[j]; }
    }
    if (r == 0 && hf == 0) {
      P02[k0] = eZx[1];                P02[k0 + 1] = eZy[1];
      P03[k0] = eZx[1] * eZx[2];       P03[k0 + 1] = eZy[1] * eZy[2];
      P13[k0] = eZx[2];                P13[k0 + 1] = eZy[2];
      float* dimg = reinterpret_cast<float*>(img + IMG_D);
      dimg[k0] = A0[k0] * eZx[0] * eZx[1] * eZx[2] * eZx[3];
      dimg[k0 + 1] = A0[k0 + 1] * eZy[0] * eZy[1] * eZy[2] * eZy[3];
    }
    if (hf == 0) {
      const float zx = Zx[r], zy = Zy[r];
      const bool stx = zx < -kSteep, sty = zy < -kSteep;
      Ef[r * KD + k0] = stx ? 0.f : expf(-zx);
      Ef[r * KD + k0 + 1] = sty ? 0.f : expf(-zy);
      const uint32_t bits = (stx ? 1u : 0u) | (sty ? 2u : 0u);
      if (bits) atomicOr(&steep[r * 4 + (k0 >> 5)], bits << (k0 & 31));
    }
    // ra: prefix products from the block start (the second half starts from
    // the first half's total); nb: suffix products to the next block start
    // (the first half ends with the second half's total)
    float2 ra[8], nb[8];
    if (hf == 1 && r == 3) al[8] = make_float2(1.f, 1.f);
    ra[0] = hf ? make_float2(__expf(ox), __expf(oy)) : make_float2(1.f, 1.f);
#pragma unroll
    for (int i = 1; i < 8; ++i) ra[i] = make_float2(ra[i - 1].x * al[i].x, ra[i - 1].y * al[i].y);
    nb[7] = hf ? al[8] : make_float2(al[8].x * __expf(ox), al[8].y * __expf(oy));
#pragma unroll
    for (int i = 6; i >= 0; --i)
      nb[i] = make_float2(nb[i + 1].x * al[i + 1].x, nb[i + 1].y * al[i + 1].y);
    // Qbar, Ktilde and V go out as 16-byte core-matrix rows: the four lanes of
    // a quad hold the four channel pairs of one 8-channel group, so after a
    // quad transpose of four rows each lane owns one whole row of the group.
#pragma unroll
    for (int i4 = 0; i4 < 8; i4 += 4) {
      uint32_t qh[4], kh[4], vh[4];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const int i = i4 + ii, c = rb0 + i;
        const float2 qv = qr[i], kv = kr[i], vv = vr[i];
        const float qsx = qv.x * s, qsy = qv.y * s;
        const float egx = bfx * ra[i].x, egy = bfy * ra[i].y;   // exp(gc_c)
        qh[ii] = pack_h2(qsx * egx, qsy * egy);                  // Qbar (-> E later)
        kh[ii] = pack_h2(kv.x * egx, kv.y * egy);                // Ktilde (-> -W later)
        vh[ii] = pack_h2(vv.x, vv.y);                            // V (-> U later)
        *reinterpret_cast<float2*>(Axk + c * AXP + k0) = make_float2(kv.x * ra[i].x, kv.y * ra[i].y);
        *reinterpret_cast<float2*>(Axq + c * AXP + k0) = make_float2(qsx * ra[i].x, qsy * ra[i].y);
        *reinterpret_cast<float2*>(Yb + c * AXP + k0) = make_float2(kv.x * nb[i].x, kv.y * nb[i].y);
      }
      quad_transpose(qh, tig);
      quad_transpose(kh, tig);
      quad_transpose(vh, tig);
      const int c = rb0 + i4 + tig;
      *reinterpret_cast<uint4*>(img + IMG_U + vb_off(c, k0 & ~7)) = make_uint4(vh[0], vh[1], vh[2], vh[3]);
      *reinterpret_cast<uint4*>(img + IMG_A1 + a1_off(64 + c, k0 & ~7)) = make_uint4(qh[0], qh[1], qh[2], qh[3]);
      *reinterpret_cast<uint4*>(img + IMG_A1 + a1_off(c, k0 & ~7)) = make_uint4(kh[0], kh[1], kh[2], kh[3]);
    }
    // Kbar^T (k rows, c cols): this thread's eight rows of one channel = 16 bytes
    {
      uint32_t ex[4], ey[4];
#pragma unroll
      for (int ii = 0; ii < 8; ii += 2) {
        ex[ii / 2] = pack_h2(kr[ii].x * nb[ii].x * afx, kr[ii + 1].x * nb[ii + 1].x * afx);
        ey[ii / 2] = pack_h2(kr[ii].y * nb[ii].y * afy, kr[ii + 1].y * nb[ii + 1].y * afy);
      }
      *reinterpret_cast<uint4*>(img + IMG_A3 + a2_off(k0, rb0)) = make_uint4(ex[0], ex[1], ex[2], ex[3]);
      *reinterpret_cast<uint4*>(img + IMG_A3 + a2_off(k0 + 1, rb0)) = make_uint4(ey[0], ey[1], ey[2], ey[3]);
    }
  }
  ptx::fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {              // Kbar^T and d are final: [IMG_A3, IMG_SHARED) leaves now
    ptx::bulk_s2g(ws + (size_t)chunk * IMG_BYTES + IMG_A3, img + IMG_A3, IMG_SHARED - IMG_A3);
    ptx::bulk_commit();
  }

  // ---- 2. Gram blocks: 8 warps per type (L: x = k, Aout: x = s q); A
  // fragments in registers.  The K order inside each 16-channel group is
  // permuted (sums are order-free) so every fragment element pair comes from
  // one float4 load.  The 10 block pairs (rr, j <= rr) of a type go one or
  // two per warp: (3,0) (3,1) (3,2) (3,3) (2,0-1) (2,2) (1,0-1) (0,0).
  {
    const int type = warp >> 3, slot = warp & 7;
    const float* Ax = type ? Axq : Axk;
    const int rr = slot < 4 ? 3 : (slot < 6 ? 2 : (slot == 6 ? 1 : 0));
    const int jlo = slot < 4 ? slot : (slot == 5 ? 2 : 0);
    const int jhi = slot < 4 ? slot : (slot == 4 ? 1 : (slot == 5 ? 2 : (slot == 6 ? 1 : 0)));
    {
    uint32_t af[8][2][4];                               // [16-channel group][k-step][frag]
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const float4 a0 = *reinterpret_cast<const float4*>(Ax + (16 * rr + gid) * AXP + 16 * g + 4 * tig);
      const float4 a1 = *reinterpret_cast<const float4*>(Ax + (16 * rr + gid + 8) * AXP + 16 * g + 4 * tig);
      af[g][0][0] = ptx::f32_to_tf32(a0.x);
      af[g][0][1] = ptx::f32_to_tf32(a1.x);
      af[g][0][2] = ptx::f32_to_tf32(a0.y);
      af[g][0][3] = ptx::f32_to_tf32(a1.y);
      af[g][1][0] = ptx::f32_to_tf32(a0.z);
      af[g][1][1] = ptx::f32_to_tf32(a1.z);
      af[g][1][2] = ptx::f32_to_tf32(a0.w);
      af[g][1][3] = ptx::f32_to_tf32(a1.w);
    }
#pragma unroll 1
    for (int j = jlo; j <= jhi; ++j) {
      const float* f = nullptr;                         // per-channel factor on the B side
      if (j == rr) f = Ef + rr * KD;
      else if (rr - j == 2) f = (j == 0) ? P02 : P13;
      else if (rr - j == 3) f = P03;
      // two partial sums per n-tile (even / odd channel groups): four
      // independent MMA chains instead of two
      float acc2[2][2][4] = {};
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const int kc = 16 * g + 4 * tig;
        const float4 fv = f ? *reinterpret_cast<const float4*>(f + kc) : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float4 y = *reinterpret_cast<const float4*>(Yb + (16 * j + 8 * nt + gid) * AXP + kc);
          const uint32_t b0[2] = {ptx::f32_to_tf32(y.x * fv.x), ptx::f32_to_tf32(y.y * fv.y)};
          const uint32_t b1[2] = {ptx::f32_to_tf32(y.z * fv.z), ptx::f32_to_tf32(y.w * fv.w)};
          ptx::mma_tf32_16x8x8(acc2[g & 1][nt], af[g][0], b0);
          ptx::mma_tf32_16x8x8(acc2[g & 1][nt], af[g][1], b1);
        }
      }
      float acc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = acc2[0][nt][e] + acc2[1][nt][e];
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
                  float prl = 0.f, pcl = 0.f;              // static indexing of pre[]
#pragma unroll
                  for (int u = 0; u < 16; ++u) {
                    prl = (u == rl) ? pre[u] : prl;
                    pcl = (u == cl) ? pre[u] : pcl;
                  }
                  acc[nt][e] = fmaf(xr * ki, expf(prl - pcl), acc[nt][e]);
                }
              }
          }
        }
      }
      // L (type 0) where the inversion reads it: strictly below the diagonal.
      // Aout (type 1) as the f16 A operand of phase 5: the full lower blocks
      // plus zeros above the diagonal inside the diagonal block.
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = 16 * rr + gid + 8 * (e >> 1);
          const int col = 16 * j + 8 * nt + 2 * tig + (e & 1);
          const float v = acc[nt][e];
          if (type == 0) {
            if (col < row) Lm[row * LMP + col] = sbeta[row] * v;
          } else {
            *reinterpret_cast<__half*>(A2 + a2_off(64 + row, col)) =
                __float2half_rn(col <= row ? v : 0.f);
          }
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
      // column j of (I + L_rb)^-1, right-looking: once x[i] is final it is
      // eliminated from every later row, so each step is one dependent FMA
      const int j = lane;
      const float* lb = Lm + (16 * rb) * LMP + 16 * rb;
      float x[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) x[c] = (c == j) ? 1.f : 0.f;
#pragma unroll
      for (int i = 0; i < 15; ++i)
#pragma unroll
        for (int c = i + 1; c < 16; ++c) x[c] = fmaf(-lb[c * LMP + i], x[i], x[c]);
#pragma unroll
      for (int c = 0; c < 16; ++c) Mm[(16 * rb + c) * LMP + 16 * rb + j] = x[c];
    }
  } else {
    for (int idx = tid - 128; idx < CH * CH; idx += PREP_THREADS - 128) {
      const int row = idx >> 6, col = idx & 63;
      if ((col >> 4) > (row >> 4)) Mm[row * LMP + col] = 0.f;
    }
  }
  __syncthreads();
  // off-diagonal blocks M_rj = -D_r sum_{t=j}^{r-1} L_rt M_tj, by distance r - j;
  // a warp pair per block, one 8-column n-tile each (the products are
  // column-separable)
  for (int dist = 1; dist <= 3; ++dist) {
    if (warp < 2 * (4 - dist)) {
      const int j = warp >> 1, nt = warp & 1, rb = j + dist;
      float tacc[4] = {0.f, 0.f, 0.f, 0.f};
      const float* La = Lm + (16 * rb) * LMP + 16 * j;
      const float* Mb = Mm + (16 * j) * LMP + 16 * j + 8 * nt;
      if (dist == 1) gemm16x8_3xtf32<2>(tacc, La, LMP, Mb, LMP, lane);
      else if (dist == 2) gemm16x8_3xtf32<4>(tacc, La, LMP, Mb, LMP, lane);
      else gemm16x8_3xtf32<6>(tacc, La, LMP, Mb, LMP, lane);
      float* Tw = Ts + warp * (16 * TSP);
#pragma unroll
      for (int e = 0; e < 4; ++e) Tw[(gid + 8 * (e >> 1)) * TSP + 2 * tig + (e & 1)] = tacc[e];
      __syncwarp();
      float macc[4] = {0.f, 0.f, 0.f, 0.f};
      gemm16x8_3xtf32<2>(macc, Mm + (16 * rb) * LMP + 16 * rb, LMP, Tw, TSP, lane);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        Mm[(16 * rb + gid + 8 * (e >> 1)) * LMP + 16 * j + 8 * nt + 2 * tig + (e & 1)] = -macc[e];
    }
    __syncthreads();
  }
  for (int idx = tid; idx < CH * CH / 2; idx += PREP_THREADS) {
    const int row = idx >> 5, col = 2 * (idx & 31);
    st_h2(A2, a2_off(row, col), Mm[row * LMP + col] * sbeta[col],
          Mm[row * LMP + col + 1] * sbeta[col + 1]);
  }
  // the staging region (inputs, then the phase-1..3 operands) is dead from
  // here on: the next chunk's copies land in it while phases 4-5 run
  if constexpr (LOAD == 3) ptx::fence_proxy_async_smem();
  __syncthreads();
  if constexpr (LOAD == 3) {
    if (tid == 32 && chunk + stride < total) issue_inputs(chunk + stride);
  }

  // ---- 4. AM = Aout M over Aout (rows 64-127 of A2) -------------------------
  // Aout M is block lower triangular like M: with it, one GEMM gives W, U,
  // Aout W = AM Ktilde and F = Aout U = AM V.
  {
    const int rb = warp & 3, q4 = warp >> 2;             // row block, 16-column quarter
    const int mi = lane >> 3;
    float acc[2][4] = {};
    for (int ks = 0; ks <= rb; ++ks) {
      uint32_t a[4], bq[4];
      ptx::ldmatrix_x4(a, A2 + a2_off(64 + 16 * rb + (lane & 7) + ((mi & 1) ? 8 : 0),
                                      16 * ks + ((mi & 2) ? 8 : 0)));
      ptx::ldmatrix_x4_trans(bq, A2 + a2_off(16 * ks + (lane & 7) + ((mi & 1) ? 8 : 0),
                                             16 * q4 + ((mi & 2) ? 8 : 0)));
      ptx::mma_f16_16x8x16(acc[0], a, bq);
      ptx::mma_f16_16x8x16(acc[1], a, bq + 2);
    }
    __syncthreads();                                     // every warp is done reading Aout
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr)
        st_h2(A2, a2_off(64 + 16 * rb + gid + 8 * hr, 16 * q4 + 8 * nt + 2 * tig),
              acc[nt][2 * hr], acc[nt][2 * hr + 1]);
  }
  ptx::fence_proxy_async_smem();                         // A2, Ktilde, V -> tensor core
  ptx::tc_fence_before();
  __syncthreads();

  // ---- 5. D[128 x 256] = [M; AM] [Ktilde | V] on tcgen05 (fp32 in TMEM) -----
  //   rows 0-63:   [W | U]            rows 64-127: [Aout W | F]
  ptx::tc_fence_after();
  const uint32_t tbase = *tslot;
  if (warp == 0) {
    if (ptx::elect_one()) {
      const uint64_t dA = ptx::sdesc(ptx::smem_u32(A2), 128, 1024);            // K-major
      const uint64_t dK = ptx::sdesc(ptx::smem_u32(img + IMG_A1), 2048, 128);  // MN-major
      const uint64_t dV = ptx::sdesc(ptx::smem_u32(img + IMG_U), 128, 1024);   // MN-major
      constexpr uint32_t ID = ptx::idesc_f16_f32(128, 128, false, true);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {                   // K = 64 chunk rows, 16 per MMA
        ptx::mma_f16_ss(tbase, dA + 16 * ks, dK + 256 * ks, ID, ks > 0);
        ptx::mma_f16_ss(tbase + 128, dA + 16 * ks, dV + 16 * ks, ID, ks > 0);
      }
      ptx::tc_commit(mbar);
    }
    __syncwarp();
  }
  const bool mma_ok = ptx::mbar_wait(mbar, it & 1u, kWaitNs);
  ptx::tc_fence_after();
  if (__syncthreads_or(!mma_ok)) {                       // the GEMM never finished: give up
    if (tid == 0) {
      atomicExch(&g_kda_device_error, 2);
      ptx::mbar_wait(mbar, it & 1u, kWaitNs / 2);
      ptx::bulk_wait_read();
    }
    if (LOAD == 3 && tid == 32 && chunk + stride < total)   // the next chunk's copies in flight
      ptx::mbar_wait(tbar, (it + 1u) & 1u, kWaitNs / 2);
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
      ptx::tc_fence_after();
      ptx::tmem_dealloc(tbase, kPrepTmemCols);
    }
    return;
  }
  {
    // TMEM lane quarter of this warp = D rows 32 lq .. 32 lq + 31 (one per lane);
    // warp group qd = warp / 4 reads D columns 64 qd .. 64 qd + 63
    const int lq = warp & 3, row = 32 * lq + lane, qd = warp >> 2, half = qd >> 1;
    const uint32_t taddr = tbase + (static_cast<uint32_t>(32 * lq) << 16) + 64 * qd;
#pragma unroll 1
    for (int pc = 0; pc < 2; ++pc) {
      float v[32];
      ptx::tmem_ld<32>(taddr + 32 * pc, v);
      ptx::tmem_wait_ld();
#pragma unroll
      // ---- 6. straight from registers to the workspace image: a warp's 32
      // rows of one 8-column group are four (A1) or one (U, F) whole 128-byte
      // lines, so these 16-byte stores coalesce without staging
      for (int o = 0; o < 4; ++o) {
        const int col = 64 * (qd & 1) + 32 * pc + 8 * o;    // within the 128-column half
        float* x = v + 8 * o;
        int off;
        if (half == 0) {
          off = IMG_A1 + a1_off(row, col);
          if (row < 64) {                                  // -W
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = -x[e];
          } else {                                         // E = Qbar - Aout W
            const uint4 qv = *reinterpret_cast<const uint4*>(img + off);
            const __half2* qh = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(qh[e]);
              x[2 * e] = f.x - x[2 * e];
              x[2 * e + 1] = f.y - x[2 * e + 1];
            }
          }
        } else {                                           // U, F
          off = row < 64 ? IMG_U + vb_off(row, col) : IMG_F + vb_off(row - 64, col);
        }
        *reinterpret_cast<uint4*>(ws + (size_t)chunk * IMG_BYTES + off) =
            make_uint4(pack_h2(x[0], x[1]), pack_h2(x[2], x[3]), pack_h2(x[4], x[5]),
                       pack_h2(x[6], x[7]));
      }
    }
  }
  // end of the chunk: TMEM read out, and the Kbar^T / d store must have read
  // shared memory before the next chunk's phase 1 rewrites the image region
  ptx::tc_fence_before();
  __syncthreads();
  if (tid == 0) ptx::bulk_wait_read();
  __syncthreads();
  ptx::tc_fence_after();
  }  // chunk loop

  if (warp == 0) {
    ptx::tmem_dealloc(*tslot, kPrepTmemCols);
  }
}

// ---------------------------------------------------------------------------
// state kernel
// ---------------------------------------------------------------------------
template <int VS>
struct StateCfg {
  static constexpr int NCOL = VS <= 16 ? 64 : (VS <= 32 ? 128 : (VS <= 64 ? 256 : 512));
  static constexpr int R1 = 0, R3 = 2 * VS;                    // TMEM columns
  static constexpr int SLICE = CH * VS * 2;                    // U or F slice bytes
  static constexpr int ST_U = 50176;                           // shared part, 1 KiB padded
  static constexpr int ST_F = ST_U + SLICE;
  static constexpr int STAGE = ((ST_F + SLICE + 1023) / 1024) * 1024;
  // chunk images in flight: three where they fit (the refill of a stage is
  // issued when its chunk is done, so with three it has two chunk periods to land)
  static constexpr int NST = 3 * STAGE + (KD + CH) * VS * 2 + 64 <= 227 * 1024 ? 3 : 2;
  static constexpr int SB_OFF = NST * STAGE;                   // S  (K = 128) f16
  static constexpr int PB_OFF = SB_OFF + KD * VS * 2;          // P  (K = 64)  f16
  static constexpr int BAR_OFF = PB_OFF + CH * VS * 2;
  static constexpr int SMEM = BAR_OFF + 64;
  static constexpr uint32_t TX = IMG_SHARED + 2 * SLICE;       // bytes per chunk
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
// 8 f16 (16 bytes) added into 8 fp32
__device__ __forceinline__ void add8_f16(float* x, int4 v) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    x[2 * i] += f.x;
    x[2 * i + 1] += f.y;
  }
}

__device__ __forceinline__ void named_barrier_64() {
  asm volatile("bar.sync 1, 64;" ::: "memory");
}

template <int VS>
__device__ __forceinline__ void fetch_chunk(uint8_t* stg, const uint8_t* img_g, int v0,
                                            uint64_t* bar) {
  using Cfg = StateCfg<VS>;
  ptx::mbar_arrive_expect_tx(bar, Cfg::TX);
  ptx::bulk_g2s(stg, img_g, IMG_SHARED, bar);
  ptx::bulk_g2s(stg + Cfg::ST_U, img_g + IMG_U + v0 * 128, Cfg::SLICE, bar);
  ptx::bulk_g2s(stg + Cfg::ST_F, img_g + IMG_F + v0 * 128, Cfg::SLICE, bar);
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
  constexpr int NST = Cfg::NST;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Cfg::BAR_OFF);   // [NST] chunk images
  uint64_t* mbarA = full + NST;        // R1 = [-W; E] S done           (one phase per chunk)
  uint64_t* mbarB = full + NST + 1;    // R3 += Kbar^T P done           (one phase per chunk)
  uint64_t* fcons = full + NST + 2;    // warps 2-3 finished reading F  (one phase per chunk)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(full + NST + 3);
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
    for (int sg = 0; sg < NST; ++sg) ptx::mbar_init(&full[sg], 1);
    ptx::mbar_init(mbarA, 1);
    ptx::mbar_init(mbarB, 1);
    ptx::mbar_init(fcons, 64);
    ptx::fence_mbar_init();
    *abort_flag = 0;
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tlane = tbase + (static_cast<uint32_t>(warp * 32) << 16);

  // thread 64 (the copy issuer): stages with a bulk copy in flight and their phase parity
  uint32_t pending = 0, pend_par = 0;
  ptx::grid_dep_wait();               // the prep grid's chunk images are complete
  if (tid == 64) {
    for (int sg = 0; sg < NST && sg < NT; ++sg) {
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

  // shared-memory descriptors of the fixed operands (built once); all
  // descriptors advance by 256 bytes (16 in the >>4 address field) per k-step
  const uint32_t st0 = ptx::smem_u32(sm);
  const uint64_t dSb = ptx::sdesc(ptx::smem_u32(Sb), 128, 2048);
  const uint64_t dPb = ptx::sdesc(ptx::smem_u32(Pb), 128, 1024);

  bool aborted = false;
  for (int n = 0; n < NT; ++n) {
    const int sg = n % NST;
    uint8_t* stg = sm + sg * Cfg::STAGE;
    const uint32_t par = static_cast<uint32_t>(n & 1);
    // every thread waits for image n itself (bounded)
    if (ptx::mbar_wait(&full[sg], (n / NST) & 1, kWaitNs)) {
      if (tid == 64) pending &= ~(1u << sg);
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
    if (warp == 0) {                                       // warp-uniform issue, one lane
      ptx::tc_fence_after();
      const uint64_t dA1 = ptx::sdesc(st0 + sg * Cfg::STAGE + IMG_A1, 128, 2048);
      if (ptx::elect_one()) {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)                     // R1 = [-W; E] S
          ptx::mma_f16_ss(tbase + Cfg::R1, dA1 + 16 * ks, dSb + 16 * ks, IDESC, ks > 0);
        ptx::tc_commit(mbarA);
      }
      __syncwarp();
    }
    // every warp needs the first batch (P rows 0-63, O rows 64-127); the
    // barriers complete once per chunk, so parity n & 1 can never be lapped
    if (!ptx::mbar_wait(mbarA, par, kWaitNs)) *abort_flag = 1;
    ptx::tc_fence_after();
    if (warp < 2) {                                        // P = U - W S, rows c = tid
      const uint8_t* ub = stg + Cfg::ST_U;
#pragma unroll 1
      for (int pc = 0; pc < NP; ++pc) {
        float u[CW];
        ptx::tmem_ld<CW>(tlane + Cfg::R1 + pc * CW, u);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int g8 = 0; g8 < CW / 8; ++g8) {
          const int gg = pc * (CW / 8) + g8;
          add8_f16(u + 8 * g8, *reinterpret_cast<const int4*>(ub + gg * 1024 + tid * 16));
          *reinterpret_cast<int4*>(Pb + gg * 1024 + (tid >> 3) * 128 + (tid & 7) * 16) =
              pack8_f16(u + 8 * g8);
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      named_barrier_64();                                  // P ready (warps 0-1)
      if (warp == 0) {
        ptx::tc_fence_after();
        const uint64_t dA3 = ptx::sdesc(st0 + sg * Cfg::STAGE + IMG_A3, 128, 1024);
        if (ptx::elect_one()) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)                   // R3 += Kbar^T P
            ptx::mma_f16_ss(tbase + Cfg::R3, dA3 + 16 * ks, dPb + 16 * ks, IDESC, 1u);
          ptx::tc_commit(mbarB);
        }
        __syncwarp();
      }
    } else {                                               // O = E S + F, rows c = tid - 64
      const int c = tid - 64;
      const int t = n * CH + c;
      const uint8_t* fb = stg + Cfg::ST_F;
      TIO* dst = static_cast<TIO*>(p.o) + b * p.o_s[0] + (int64_t)t * p.o_s[1] +
                 h * p.o_s[2] + v0;
      int4 fr[VS / 8];                                     // F row first: frees the stage early
#pragma unroll
      for (int gg = 0; gg < VS / 8; ++gg)
        fr[gg] = *reinterpret_cast<const int4*>(fb + gg * 1024 + c * 16);
      ptx::mbar_arrive(fcons);                             // F of this stage consumed
#pragma unroll
      for (int pc = 0; pc < NP; ++pc) {
        float o[CW];
        ptx::tmem_ld<CW>(tlane + Cfg::R1 + pc * CW, o);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int g8 = 0; g8 < CW / 8; ++g8) add8_f16(o + 8 * g8, fr[pc * (CW / 8) + g8]);
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
    if (!ptx::mbar_wait(mbarB, par, kWaitNs)) *abort_flag = 1;
    ptx::tc_fence_after();
    // thread 64 refills the stage (off the chain that warp 0 runs): after the
    // second batch the MMAs and warps 0-1 are done with it, after fcons warps 2-3
    if (tid == 64 && n + NST < NT && !*abort_flag) {       // stage free: fetch chunk n+NST
      if (ptx::mbar_wait(fcons, par, kWaitNs)) {
        ptx::fence_proxy_async_smem();
        fetch_chunk<VS>(stg, wsh + (size_t)(n + NST) * IMG_BYTES, v0, &full[sg]);
        pending |= 1u << sg;
        pend_par = (pend_par & ~(1u << sg)) | ((((n + NST) / NST) & 1u) << sg);
      } else {
        *abort_flag = 1;
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
  } else if (tid == 64) {
    atomicExch(&g_kda_device_error, 1);
    // let bulk copies still in flight land before this CTA's smem is released
    for (int sg = 0; sg < NST; ++sg)
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
// state kernel, register-resident variant
// ---------------------------------------------------------------------------
// The same chain as state_kernel, S' = d (.) S + Kbar^T (U - W S) and
// O = E S + F per chunk, with the fp32 master state held in mma.sync
// accumulator registers: S' accumulates Kbar^T P straight onto d (.) S, and the
// only hand-offs per chunk are the f16 copies of S and P through shared memory.
// The chain is latency-bound (M = 128, N = VS, one chunk after another), so it
// gets warps of its own:
//  * chain warps 0-3: S -> f16 copy, P rows 16w.. (split-K accumulators) ->
//    f16 copy, S <- d (.) S + Kbar^T P for key rows 32w..;
//  * output warps 4-7: O rows 16(w-4).. = E S + F from the f16 copy of S
//    (double-buffered, so the chain can write the next one meanwhile).
// Per chunk one block barrier (copy of S and image ready; the previous chunk
// fully consumed) and one 128-thread barrier among the chain warps (P ready).
template <int VS>
struct MmaStateCfg {
  static constexpr int SLICE = CH * VS * 2;
  static constexpr int ST_U = 50176;
  static constexpr int ST_F = ST_U + SLICE;
  static constexpr int STAGE = ((ST_F + SLICE + 1023) / 1024) * 1024;
  static constexpr int PS = VS * 2 + 16;   // row pitch of the f16 S and P copies (conflict-free)
  static constexpr int NST = 3 * STAGE + (2 * KD + CH) * PS + 64 <= 227 * 1024 ? 3 : 2;
  static constexpr int SX_OFF = NST * STAGE;             // [2][128][PS]
  static constexpr int PX_OFF = SX_OFF + 2 * KD * PS;    // [64][PS]
  static constexpr int BAR_OFF = PX_OFF + CH * PS;
  static constexpr int SMEM = BAR_OFF + 64;
  static constexpr uint32_t TX = IMG_SHARED + 2 * SLICE;
  static_assert(SMEM <= 227 * 1024, "state shared memory");
};
constexpr int MMA_STATE_WARPS = 8;

template <typename T> struct Pair;
template <> struct Pair<float> {
  static __device__ __forceinline__ void store(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
  }
};
template <> struct Pair<__half> {
  static __device__ __forceinline__ void store(__half* p, float a, float b) {
    *reinterpret_cast<__half2*>(p) = __floats2half2_rn(a, b);
  }
};
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
  }
};

template <int VS>
__device__ __forceinline__ void fetch_chunk_mma(uint8_t* stg, const uint8_t* img_g, int v0,
                                                uint64_t* bar) {
  using Cfg = MmaStateCfg<VS>;
  ptx::mbar_arrive_expect_tx(bar, Cfg::TX);
  ptx::bulk_g2s(stg, img_g, IMG_SHARED, bar);
  ptx::bulk_g2s(stg + Cfg::ST_U, img_g + IMG_U + v0 * 128, Cfg::SLICE, bar);
  ptx::bulk_g2s(stg + Cfg::ST_F, img_g + IMG_F + v0 * 128, Cfg::SLICE, bar);
}

__device__ __forceinline__ void chain_barrier() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

template <int VS, typename TIO, typename TSI, typename TSO>
__global__ void __launch_bounds__(MMA_STATE_WARPS * 32, 1)
state_mma_kernel(const ChunkParams p, const uint8_t* __restrict__ ws) {
  using Cfg = MmaStateCfg<VS>;
  constexpr int NST = Cfg::NST, PS = Cfg::PS;
  constexpr int NTL = VS / 8;         // 8-column tiles
  static_assert(NTL % 2 == 0, "VS must be a multiple of 16");
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* Px = sm + Cfg::PX_OFF;     // P  f16 [64 rows][VS], pitch PS
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Cfg::BAR_OFF);   // [NST] chunk images
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + NST);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const bool chain = warp < 4;
  const int b = blockIdx.z, h = blockIdx.y, v0 = blockIdx.x * VS;
  const int T = p.T;
  const int NT = (T + CH - 1) / CH;
  const int KR = 32 * (warp & 3);     // chain warps: first key row
  const int CR = 16 * (warp & 3);     // first P row (chain) or O row (output) of this warp
  const uint8_t* wsh = ws + (size_t)(b * p.H + h) * NT * IMG_BYTES;
  // ldmatrix row addresses: matrix j = lane / 8 supplies its row lane % 8
  const int lm_row = (lane & 7) + 8 * ((lane >> 3) & 1);   // A: rows, B (trans): k rows
  const int lm_col = 8 * (lane >> 4);                      // A: k offset, B: column offset

  if (tid == 0) {
    for (int sg = 0; sg < NST; ++sg) ptx::mbar_init(&full[sg], 1);
    ptx::fence_mbar_init();
    *abort_flag = 0;
  }
  __syncthreads();
  // the copy issuer is lane 0 of the last output warp; it tracks the stages
  // with a copy in flight and their phase parity
  const bool issuer = tid == MMA_STATE_WARPS * 32 - 32;
  uint32_t pending = 0, pend_par = 0;

  // chain warps: master state, accumulator layout S[mt][nt] rows
  // KR + 16 mt + gid (+8), columns 8 nt + 2 tig (+1)
  float S[2][NTL][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = 0.f;
        if (chain && p.state_in != nullptr) {
          const int row = KR + 16 * mt + gid + 8 * (e >> 1);
          const int col = v0 + 8 * nt + 2 * tig + (e & 1);
          x = ld(static_cast<const TSI*>(p.state_in) + b * p.si_s[0] + h * p.si_s[1] +
                 (int64_t)row * p.si_s[2] + col);
        }
        S[mt][nt][e] = x;
      }
  ptx::grid_dep_wait();               // the prep grid's chunk images are complete
  if (issuer) {
    for (int sg = 0; sg < NST && sg < NT; ++sg) {
      fetch_chunk_mma<VS>(sm + sg * Cfg::STAGE, wsh + (size_t)sg * IMG_BYTES, v0, &full[sg]);
      pending |= 1u << sg;
    }
  }

  bool aborted = false;
#pragma unroll 1
  for (int n = 0; n < NT; ++n) {
    const int sg = n % NST;
    const uint8_t* stg = sm + sg * Cfg::STAGE;
    uint8_t* Sx = sm + Cfg::SX_OFF + (n & 1) * KD * PS;   // f16 copy of S_n [128][PS]
    if (chain) {                      // S -> f16 copy (rows = key, columns = value)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NTL; ++nt) {
          const int row = KR + 16 * mt + gid, col = 8 * nt + 2 * tig;
          st_h2(Sx, row * PS + col * 2, S[mt][nt][0], S[mt][nt][1]);
          st_h2(Sx, (row + 8) * PS + col * 2, S[mt][nt][2], S[mt][nt][3]);
        }
    }
    if (ptx::mbar_wait(&full[sg], (n / NST) & 1, kWaitNs)) {
      if (issuer) pending &= ~(1u << sg);
    } else {
      *abort_flag = 1;
    }
    __syncthreads();                  // copy of S_n and image n ready; chunk n-1 consumed
    if (*abort_flag) { aborted = true; break; }
    if (issuer && n >= 1 && n - 1 + NST < NT) {          // refill the stage of chunk n-1
      const int s1 = (n - 1) % NST;
      ptx::fence_proxy_async_smem();
      fetch_chunk_mma<VS>(sm + s1 * Cfg::STAGE, wsh + (size_t)(n - 1 + NST) * IMG_BYTES, v0,
                          &full[s1]);
      pending |= 1u << s1;
      pend_par = (pend_par & ~(1u << s1)) | ((((n - 1 + NST) / NST) & 1u) << s1);
    }
    // rows 16(w%4).. of [-W; E] S: P rows for the chain warps, O rows (64 +)
    // for the output warps; two accumulators (even / odd k-steps)
    float ra[2][NTL][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) ra[i][nt][e] = 0.f;
    {
      const int arow = (chain ? 0 : CH) + CR + lm_row;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t bf[NTL / 2][4], af[4];
#pragma unroll
        for (int jp = 0; jp < NTL / 2; ++jp)
          ptx::ldmatrix_x4_trans(bf[jp], Sx + (16 * ks + lm_row) * PS + (16 * jp + lm_col) * 2);
        ptx::ldmatrix_x4(af, stg + IMG_A1 + a1_off(arow, 16 * ks + lm_col));
#pragma unroll
        for (int nt = 0; nt < NTL; ++nt)
          ptx::mma_f16_16x8x16(ra[ks & 1][nt], af, &bf[nt >> 1][2 * (nt & 1)]);
      }
    }
    if (chain) {
      // P = U - W S -> f16 copy
      const uint8_t* ub = stg + Cfg::ST_U;
#pragma unroll
      for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int c = CR + gid + 8 * hf, col = 8 * nt + 2 * tig;
          const float2 u = __half22float2(*reinterpret_cast<const __half2*>(ub + vb_off(c, col)));
          st_h2(Px, c * PS + col * 2, ra[0][nt][2 * hf] + ra[1][nt][2 * hf] + u.x,
                ra[0][nt][2 * hf + 1] + ra[1][nt][2 * hf + 1] + u.y);
        }
      chain_barrier();                // P complete
      // S <- d (.) S + Kbar^T P for key rows KR..
      const float* dv = reinterpret_cast<const float*>(stg + IMG_D);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const float dlo = dv[KR + 16 * mt + gid], dhi = dv[KR + 16 * mt + gid + 8];
#pragma unroll
        for (int nt = 0; nt < NTL; ++nt) {
          S[mt][nt][0] *= dlo; S[mt][nt][1] *= dlo;
          S[mt][nt][2] *= dhi; S[mt][nt][3] *= dhi;
        }
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t bf[NTL / 2][4];
#pragma unroll
        for (int jp = 0; jp < NTL / 2; ++jp)
          ptx::ldmatrix_x4_trans(bf[jp], Px + (16 * ks + lm_row) * PS + (16 * jp + lm_col) * 2);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t af[4];
          ptx::ldmatrix_x4(af, stg + IMG_A3 + a2_off(KR + 16 * mt + lm_row, 16 * ks + lm_col));
#pragma unroll
          for (int nt = 0; nt < NTL; ++nt)
            ptx::mma_f16_16x8x16(S[mt][nt], af, &bf[nt >> 1][2 * (nt & 1)]);
        }
      }
    } else {
      // O = E S + F for chunk rows CR..
      const uint8_t* fb = stg + Cfg::ST_F;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int c = CR + gid + 8 * hf;
        const int t = n * CH + c;
        if (t >= T) continue;
        TIO* dst = static_cast<TIO*>(p.o) + b * p.o_s[0] + (int64_t)t * p.o_s[1] +
                   h * p.o_s[2] + v0;
#pragma unroll
        for (int nt = 0; nt < NTL; ++nt) {
          const int col = 8 * nt + 2 * tig;
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(fb + vb_off(c, col)));
          const float o0 = ra[0][nt][2 * hf] + ra[1][nt][2 * hf] + f.x;
          const float o1 = ra[0][nt][2 * hf + 1] + ra[1][nt][2 * hf + 1] + f.y;
          if (p.o_vec16) {
            Pair<TIO>::store(dst + col, o0, o1);
          } else {
            st(dst + col, o0);
            st(dst + col + 1, o1);
          }
        }
      }
    }
  }

  if (!aborted) {
    if (chain) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = KR + 16 * mt + gid + 8 * (e >> 1);
            const int col = v0 + 8 * nt + 2 * tig + (e & 1);
            st(static_cast<TSO*>(p.state_out) + b * p.so_s[0] + h * p.so_s[1] +
                   (int64_t)row * p.so_s[2] + col,
               S[mt][nt][e]);
          }
    }
  } else if (issuer) {
    atomicExch(&g_kda_device_error, 1);
    // let bulk copies still in flight land before this CTA's smem is released
    for (int sg = 0; sg < NST; ++sg)
      if (pending & (1u << sg)) ptx::mbar_wait(&full[sg], (pend_par >> sg) & 1u, kWaitNs / 2);
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
  // per call: the attribute belongs to the current device's context
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       StateCfg<VS>::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.V / VS, p.H, p.B);
  // programmatic dependent of the prep grid: set-up and S0 loads overlap its tail
  return launch_dependent(kern, grid, 128, StateCfg<VS>::SMEM, s, p, ws);
}

template <typename TIO, typename TSI, typename TSO, int VS>
cudaError_t launch_state_mma(const ChunkParams& p, const uint8_t* ws, cudaStream_t s) {
  auto kern = state_mma_kernel<VS, TIO, TSI, TSO>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       MmaStateCfg<VS>::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(p.V / VS, p.H, p.B);
  // programmatic dependent of the prep grid: set-up and S0 loads overlap its tail
  return launch_dependent(kern, grid, MMA_STATE_WARPS * 32, MmaStateCfg<VS>::SMEM, s, p, ws);
}

// which state pass runs: the register-resident one (true) or the TMEM one
bool state_in_registers(int vs) { return vs <= 32; }

template <typename TIO, int LOAD>
cudaError_t launch_prep(const ChunkParams& p, uint8_t* ws, cudaStream_t s,
                        const PrepMaps& maps = PrepMaps{}) {
  auto prep = prep_kernel<TIO, LOAD>;
  // per call: the attribute belongs to the current device's context
  cudaError_t e = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       PREP_SMEM);
  if (e != cudaSuccess) return e;
  const int NT = (p.T + CH - 1) / CH;
  if ((long long)NT * p.H * p.B > 0x7fffffffLL) return cudaErrorInvalidValue;   // int chunk index
  dim3 pgrid(NT, p.H, p.B);
  if constexpr (LOAD == 3) {        // persistent: one CTA per SM walks the chunks
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long total = (long)NT * p.H * p.B;
    pgrid = dim3((unsigned)(total < sms ? total : sms), 1, 1);
  }
  prep<<<pgrid, PREP_THREADS, PREP_SMEM, s>>>(p, ws, maps);
  return cudaGetLastError();
}

// every q/k/v/g row a 16-byte-aligned contiguous range (bulk-copy rules)
template <typename TIO>
bool bulk_rows_ok(const ChunkParams& p) {
  auto al = [](const void* ptr, const int64_t* st, size_t esz) {
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return false;
    for (int d = 0; d < 3; ++d)
      if ((st[d] * (int64_t)esz) % 16) return false;
    return st[3] == 1;
  };
  return al(p.q, p.q_s, sizeof(TIO)) && al(p.k, p.k_s, sizeof(TIO)) &&
         al(p.v, p.v_s, sizeof(TIO)) && al(p.g, p.g_s, 4);
}

// map of a [B, T, H, K = 128] tensor (element strides st) with a box of one
// (b, h) and 64 rows x 128 channels; false when the driver rejects it
bool encode_rows(CUtensorMap* m, CUtensorMapDataType dt, size_t esz, const void* ptr,
                 const int64_t* st, const ChunkParams& p) {
  EncodeTiled enc = encode_tiled();
  if (enc == nullptr) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)KD, (cuuint64_t)p.H, (cuuint64_t)p.T, (cuuint64_t)p.B};
  const cuuint64_t strides[3] = {(cuuint64_t)(st[2] * esz), (cuuint64_t)(st[1] * esz),
                                 (cuuint64_t)(st[0] * esz)};
  const cuuint32_t box[4] = {(cuuint32_t)KD, 1u, (cuuint32_t)CH, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  for (int d = 0; d < 3; ++d)
    if (st[d] <= 0) return false;
  return enc(m, dt, 4, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename TIO>
bool make_prep_maps(const ChunkParams& p, PrepMaps* m) {
  const CUtensorMapDataType dt = std::is_same<TIO, __half>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return encode_rows(&m->q, dt, sizeof(TIO), p.q, p.q_s, p) &&
         encode_rows(&m->k, dt, sizeof(TIO), p.k, p.k_s, p) &&
         encode_rows(&m->v, dt, sizeof(TIO), p.v, p.v_s, p) &&
         encode_rows(&m->g, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.g, p.g_s, p);
}

template <typename TIO, typename TSI, typename TSO>
cudaError_t launch_tc3(const ChunkParams& p, uint8_t* ws, cudaStream_t s) {
  const bool vec = p.g_vec2 && p.qk_vec2 && p.v_vec2;
  cudaError_t e;
  PrepMaps maps;
  if (bulk_rows_ok<TIO>(p) && make_prep_maps<TIO>(p, &maps))
    e = launch_prep<TIO, 3>(p, ws, s, maps);
  else
    e = bulk_rows_ok<TIO>(p) ? launch_prep<TIO, 2>(p, ws, s)
        : vec                ? launch_prep<TIO, 1>(p, ws, s)
                             : launch_prep<TIO, 0>(p, ws, s);
  if (e != cudaSuccess) return e;
  const int vs = pick_vs(p);
  if (state_in_registers(vs)) {
    switch (vs) {
      case 16: return launch_state_mma<TIO, TSI, TSO, 16>(p, ws, s);
      case 32: return launch_state_mma<TIO, TSI, TSO, 32>(p, ws, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (vs) {
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
