// kda_chunk_tc.cu -- tensor-core chunkwise KDA for sm_100a (fp16 / bf16 q,k,v; K = V = 128).
//
// Replaces kimi_linear/kda.py:58-185 (kda_chunkwise) for the shapes of the
// 1.5B model and the benchmark configurations.  Two kernels on one stream,
// which run at the same time when the heads are few:
//
// 1. prep_kernel  -- persistent (one CTA per SM it is given) over the chunks of
//    64 rows, taken chunk index first (every head's chunk n before any head's
//    chunk n + 1).  Everything of a chunk that does not depend on the carried
//    state:
//      gc = cumsum(g)                                        (kda.py:129)
//      L[c,i]    = beta_c sum_k k_ck k_ik exp(gc_ck - gc_ik), i < c  (kda.py:159-165)
//      Aout[c,i] = sum_k s q_ck k_ik exp(gc_ck - gc_ik),      i <= c (kda.py:166-168)
//      M = (I + L)^-1 Diag(beta)                             (kda.py:170-171)
//      W = M (exp(gc) * K),  U = M V                         (kda.py:172-173)
//      Qbar = s q exp(gc),  Kbar = exp(gc_last - gc) k,  d = exp(gc_last)
//      E = Qbar - Aout W,   F = Aout U
//    (kda.py:177-178 give O = Qbar S + Aout (U - W S) = E S + F, so the state
//    pass needs no Aout product of its own), written as ONE 82,432-byte image
//    per chunk whose byte layout is the shared-memory layout the state pass
//    uses (it moves an image with one bulk copy), then a ready flag per image.
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
// 2. state_kernel -- one CTA per (b, h), walking that head's chunks in order
//    as their ready flags appear, with the fp32 master state in registers and
//    every GEMM transposed (value columns = TMEM lanes, A operands in TMEM);
//    see the comment above the kernel.
#include <cuda.h>            // CUtensorMap (header only; the encoder comes from the runtime)
#include <type_traits>

#include "kda_internal.cuh"
#include "tc_ptx.cuh"

namespace kda {

__device__ int g_kda_device_error = 0;

namespace tc {

constexpr int CH = 64;        // rows per chunk
constexpr int KD = 128;       // head dim K (= V) of this path
// Chunk image (bytes).  A1 and A3 are tcgen05 operands in the no-swizzle
// K-major core-matrix layout (8 rows x 16 bytes per core matrix; LBO = stride
// along K, SBO = along M / N).  U^T and F^T are read by threads, one 128-byte
// row per value column v with 16-byte chunk j at ((j ^ (v % 8)) * 16).
constexpr int IMG_A1 = 0;         // [-W; E]   128 x 128 f16, LBO 128, SBO 2048  (E = Qbar - Aout W)
constexpr int IMG_A3 = 32768;     // Kbar^T    128 x 64  f16, LBO 128, SBO 1024
constexpr int IMG_D = 49152;      // d = exp(gc_last), fp32[128]
constexpr int IMG_SHARED = 49664; // end of the operands written right after phase 1
constexpr int IMG_U = 49664;      // U^T = (M V)^T      128 x 64 f16 (V staging in prep)
constexpr int IMG_F = 66048;      // F^T = (Aout U)^T   128 x 64 f16
constexpr int IMG_BYTES = 82432;

constexpr float kSteep = 80.f;                  // block decay beyond which exp(-Z) is unsafe
constexpr uint64_t kWaitNs = 2000000000ull;     // bound on every mbarrier wait (2 s)

__device__ __forceinline__ int a1_off(int m, int k) {
  return (m >> 3) * 2048 + (k >> 3) * 128 + (m & 7) * 16 + (k & 7) * 2;
}
__device__ __forceinline__ int a2_off(int m, int k) {
  return (m >> 3) * 1024 + (k >> 3) * 128 + (m & 7) * 16 + (k & 7) * 2;
}
// 64 x 128 layout of the V staging in prep: offset(c, v).  Each block of 8
// value columns is 1 KiB (64 rows x 16 bytes): the MN-major no-swizzle layout
// of V^T as the A operand of the phase-5 GEMM (core-matrix stride 128 bytes
// along the chunk rows, 1 KiB along the value columns).
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
// the prep thread that issues the bulk stores of the chunk images and
// publishes them (warp 14: idle in the phase during which it publishes)
constexpr int PUB = 448;

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
prep_kernel(const ChunkParams p, uint8_t* __restrict__ ws, unsigned int* __restrict__ flags,
            const __grid_constant__ PrepMaps tm) {
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
  // Chunks are taken in the order c = n * (B H) + (b H + h): every head's chunk
  // n is prepared before any head's chunk n + 1, so the state pass (which may
  // run concurrently and consumes each head's chunks in order) is never left
  // waiting for a late head.  The image of chunk c lives at (b H + h) NT + n.
  // The TMA-input instantiation is persistent (a CTA walks every stride-th
  // chunk); the others run one chunk per CTA over a 1-D grid.
  const int NT = (p.T + CH - 1) / CH;
  const int BH = p.B * p.H;
  const int total = NT * BH;                          // < 2^31 (checked on the host)
  const int stride = gridDim.x;
  int chunk = blockIdx.x;
  // image whose ready flag thread PUB still owes (set once its bulk stores
  // completed; with `newest` the most recently committed store may still run).
  // PUB issued those stores, so it alone can wait for them; the async-proxy
  // fence orders them before the release, and the release (gpu scope) orders
  // every other thread's stores of the image, which precede it through a CTA
  // barrier.
  long pend = -1;
  auto publish = [&](bool newest) {
    if (pend >= 0) {
      if (newest) ptx::bulk_wait_le<1>();
      else ptx::bulk_wait_all();
      ptx::fence_proxy_async_global();
      ptx::st_release_gpu(flags + pend, 1u);
      pend = -1;
    }
  };
  // the four input boxes of chunk c into the staging region (thread 32; rows
  // past T arrive as zeros)
  auto issue_inputs = [&](int c) {
    const int n2 = c / BH, bh2 = c - n2 * BH, h2 = bh2 % p.H, b2 = bh2 / p.H;
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
  const int n = chunk / BH, bh = chunk - n * BH, h = bh % p.H, b = bh / p.H;
  const size_t img_off = ((size_t)bh * NT + n) * IMG_BYTES;   // this chunk's image
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
      const int n2 = (int)(tgt / BH), bh2 = (int)(tgt - (long)n2 * BH);
      const int h2 = bh2 % p.H, b2 = bh2 / p.H;
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
  // the image staging region is written from here on: the previous chunk's
  // bulk stores must have read it
  if (tid == PUB) ptx::bulk_wait_read();
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
    // channel pairs as two-lane fp32 multiplies (each lane rounded like a
    // scalar multiply, so the values are those of the scalar code)
#pragma unroll
    for (int i = 1; i < 8; ++i) ra[i] = __fmul2_rn(ra[i - 1], al[i]);
    nb[7] = hf ? al[8] : __fmul2_rn(al[8], make_float2(__expf(ox), __expf(oy)));
#pragma unroll
    for (int i = 6; i >= 0; --i) nb[i] = __fmul2_rn(nb[i + 1], al[i + 1]);
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
        const float2 qs = __fmul2_rn(qv, make_float2(s, s));
        const float2 eg = __fmul2_rn(make_float2(bfx, bfy), ra[i]);   // exp(gc_c)
        const float2 qb2 = __fmul2_rn(qs, eg), kt2 = __fmul2_rn(kv, eg);
        qh[ii] = pack_h2(qb2.x, qb2.y);                          // Qbar (-> E later)
        kh[ii] = pack_h2(kt2.x, kt2.y);                          // Ktilde (-> -W later)
        vh[ii] = pack_h2(vv.x, vv.y);                            // V (-> U later)
        *reinterpret_cast<float2*>(Axk + c * AXP + k0) = __fmul2_rn(kv, ra[i]);
        *reinterpret_cast<float2*>(Axq + c * AXP + k0) = __fmul2_rn(qs, ra[i]);
        *reinterpret_cast<float2*>(Yb + c * AXP + k0) = __fmul2_rn(kv, nb[i]);
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
  if (tid == PUB) {            // Kbar^T and d are final: [IMG_A3, IMG_SHARED) leaves now
    ptx::bulk_s2g(ws + img_off + IMG_A3, img + IMG_A3, IMG_SHARED - IMG_A3);
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
          const float2 yf0 = __fmul2_rn(make_float2(y.x, y.y), make_float2(fv.x, fv.y));
          const float2 yf1 = __fmul2_rn(make_float2(y.z, y.w), make_float2(fv.z, fv.w));
          const uint32_t b0[2] = {ptx::f32_to_tf32(yf0.x), ptx::f32_to_tf32(yf0.y)};
          const uint32_t b1[2] = {ptx::f32_to_tf32(yf1.x), ptx::f32_to_tf32(yf1.y)};
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
  // the previous chunk's image is complete once its bulk stores are: PUB
  // publishes it while warps 0-11 run the first doubling level (its release
  // waits for the stores; this chunk's Kbar^T / d store, the newest, may run on)
  if (tid == PUB) publish(true);
  // off-diagonal blocks by recursive doubling, D_r = M_rr: the 32 x 32 halves
  // first (M10 = -D1 L10 D0, M32 = -D3 L32 D2), then the lower-left quarter
  // X = -[D2 0; M32 D3] [L20 L21; L30 L31] [D0 0; M10 D1].  Two levels instead
  // of three (by distance r - j), the products that need only the diagonal
  // blocks in the first.  A warp owns one 8-column n-tile of a block (the
  // products are column-separable); T / Y tiles go through shared memory.
  {
    float* Tw = Ts + warp * (16 * TSP);            // per-warp 16 x 16 scratch
    float* Ys = Ts + 16 * (16 * TSP);              // Y[r - 2][j], 16 x TSP each
    auto blk = [&](int r, int j) { return Mm + (16 * r) * LMP + 16 * j; };
    auto lblk = [&](int r, int j) { return Lm + (16 * r) * LMP + 16 * j; };
    auto yblk = [&](int r, int j) { return Ys + ((r - 2) * 2 + j) * (16 * TSP); };
    // fragment <-> 16 x 8 tile at column offset c0 of a pitch-TSP array
    auto st_frag = [&](float* dst, int c0, const float* acc) {
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[(gid + 8 * (e >> 1)) * TSP + c0 + 2 * tig + (e & 1)] = acc[e];
    };
    auto ld_frag = [&](const float* src, int c0, float* acc) {
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] = src[(gid + 8 * (e >> 1)) * TSP + c0 + 2 * tig + (e & 1)];
    };
    auto st_m = [&](int r, int j, int nt, const float* acc) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        Mm[(16 * r + gid + 8 * (e >> 1)) * LMP + 16 * j + 8 * nt + 2 * tig + (e & 1)] = -acc[e];
    };
    if (warp < 12) {                               // level 1
      const int nt = warp & 1;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (warp < 4) {                              // M10 (warps 0-1), M32 (warps 2-3)
        const int r = warp < 2 ? 1 : 3, j = r - 1;
        gemm16x8_3xtf32<2>(acc, lblk(r, j), LMP, blk(j, j) + 8 * nt, LMP, lane);
        st_frag(Tw, 0, acc);
        __syncwarp();
        float macc[4] = {0.f, 0.f, 0.f, 0.f};
        gemm16x8_3xtf32<2>(macc, blk(r, r), LMP, Tw, TSP, lane);
        st_m(r, j, nt, macc);
      } else {                                     // Y21, Y31 = L_r1 D1; Y20', Y30' = L_r0 D0
        const int j = warp < 8 ? 1 : 0, r = 2 + ((warp >> 1) & 1);
        gemm16x8_3xtf32<2>(acc, lblk(r, j), LMP, blk(j, j) + 8 * nt, LMP, lane);
        st_frag(yblk(r, j), 8 * nt, acc);
      }
    }
    __syncthreads();
    if (warp < 8) {                                // level 2: blocks (r, j), r in {2, 3}
      const int r = 2 + (warp >> 2), j = (warp >> 1) & 1, nt = warp & 1;
      float macc[4] = {0.f, 0.f, 0.f, 0.f};
      if (j == 0) {                                // Y20 = Y20' + L21 M10 (and Y30 for r = 3)
        float y[4];
        ld_frag(yblk(2, 0), 8 * nt, y);
        gemm16x8_3xtf32<2>(y, lblk(2, 1), LMP, blk(1, 0) + 8 * nt, LMP, lane);
        st_frag(Tw, 0, y);
        if (r == 3) {
          ld_frag(yblk(3, 0), 8 * nt, y);
          gemm16x8_3xtf32<2>(y, lblk(3, 1), LMP, blk(1, 0) + 8 * nt, LMP, lane);
          st_frag(Tw, 8, y);
        }
        __syncwarp();
        if (r == 2) {                              // M20 = -D2 Y20
          gemm16x8_3xtf32<2>(macc, blk(2, 2), LMP, Tw, TSP, lane);
        } else {                                   // M30 = -(M32 Y20 + D3 Y30)
          gemm16x8_3xtf32<2>(macc, blk(3, 2), LMP, Tw, TSP, lane);
          gemm16x8_3xtf32<2>(macc, blk(3, 3), LMP, Tw + 8, TSP, lane);
        }
      } else if (r == 2) {                         // M21 = -D2 Y21
        gemm16x8_3xtf32<2>(macc, blk(2, 2), LMP, yblk(2, 1) + 8 * nt, TSP, lane);
      } else {                                     // M31 = -(M32 Y21 + D3 Y31)
        gemm16x8_3xtf32<2>(macc, blk(3, 2), LMP, yblk(2, 1) + 8 * nt, TSP, lane);
        gemm16x8_3xtf32<2>(macc, blk(3, 3), LMP, yblk(3, 1) + 8 * nt, TSP, lane);
      }
      st_m(r, j, nt, macc);
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

  // ---- 5. two tcgen05 GEMMs, fp32 in TMEM -----------------------------------
  //   columns 0-127:   [M; AM] Ktilde  = rows 0-63 W, rows 64-127 Aout W
  //   columns 128-255: V^T [M; AM]^T   = row v: [U^T | F^T] (the state pass
  //                    consumes U and F per value column)
  ptx::tc_fence_after();
  const uint32_t tbase = *tslot;
  if (warp == 0) {
    if (ptx::elect_one()) {
      const uint64_t dA = ptx::sdesc(ptx::smem_u32(A2), 128, 1024);            // K-major
      const uint64_t dK = ptx::sdesc(ptx::smem_u32(img + IMG_A1), 2048, 128);  // MN-major
      const uint64_t dV = ptx::sdesc(ptx::smem_u32(img + IMG_U), 128, 1024);   // MN-major
      constexpr uint32_t ID = ptx::idesc_f16_f32(128, 128, false, true);
      constexpr uint32_t IDT = ptx::idesc_f16_f32(128, 128, true, false);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {                   // K = 64 chunk rows, 16 per MMA
        ptx::mma_f16_ss(tbase, dA + 16 * ks, dK + 256 * ks, ID, ks > 0);
        ptx::mma_f16_ss(tbase + 128, dV + 16 * ks, dA + 16 * ks, IDT, ks > 0);
      }
      ptx::tc_commit(mbar);
    }
    __syncwarp();
  }
  const bool mma_ok = ptx::mbar_wait(mbar, it & 1u, kWaitNs);
  ptx::tc_fence_after();
  if (__syncthreads_or(!mma_ok)) {                       // the GEMM never finished: give up
    if (tid == PUB) {
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
    // U^T / F^T rows are staged in shared memory (the V staging is dead once the
    // GEMMs completed) and leave as one bulk store: 16-byte chunk j of row v at
    // ((j ^ (v % 8)) * 16), so the state pass reads them without bank conflicts
    uint8_t* trow = img + (qd == 2 ? IMG_U : IMG_F) + row * 128;
    const uint32_t taddr = tbase + (static_cast<uint32_t>(32 * lq) << 16) + 64 * qd;
#pragma unroll 1
    for (int pc = 0; pc < 2; ++pc) {
      float v[32];
      ptx::tmem_ld<32>(taddr + 32 * pc, v);
      ptx::tmem_wait_ld();
#pragma unroll
      // ---- 6. [-W; E] straight from registers to the workspace image: a
      // warp's 32 rows of one 8-column group are four whole 128-byte lines, so
      // these 16-byte stores coalesce without staging
      for (int o = 0; o < 4; ++o) {
        const int col = 64 * (qd & 1) + 32 * pc + 8 * o;    // within the 128-column half
        float* x = v + 8 * o;
        if (half == 1) {                                   // U^T (qd 2) / F^T (qd 3), row = v
          const int j = 4 * pc + o;
          *reinterpret_cast<uint4*>(trow + ((j ^ (row & 7)) << 4)) =
              make_uint4(pack_h2(x[0], x[1]), pack_h2(x[2], x[3]), pack_h2(x[4], x[5]),
                         pack_h2(x[6], x[7]));
          continue;
        }
        const int off = IMG_A1 + a1_off(row, col);
        if (row < 64) {                                    // -W
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = -x[e];
        } else {                                           // E = Qbar - Aout W
          const uint4 qv = *reinterpret_cast<const uint4*>(img + off);
          const __half2* qh = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(qh[e]);
            x[2 * e] = f.x - x[2 * e];
            x[2 * e + 1] = f.y - x[2 * e + 1];
          }
        }
        *reinterpret_cast<uint4*>(ws + img_off + off) =
            make_uint4(pack_h2(x[0], x[1]), pack_h2(x[2], x[3]), pack_h2(x[4], x[5]),
                       pack_h2(x[6], x[7]));
      }
    }
  }
  // end of the chunk: TMEM read out, U^T / F^T staged; they leave with one bulk
  // store, and the image is published (ready flag) once all its stores are
  // complete -- by thread PUB during the next chunk, or right after the loop
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  if (tid == PUB) {
    ptx::bulk_s2g(ws + img_off + IMG_U, img + IMG_U, IMG_BYTES - IMG_U);
    ptx::bulk_commit();
    pend = (long)(img_off / IMG_BYTES);
    // a CTA's first chunk is published right away: the state pass starts on
    // it (later chunks are published during the next chunk, off its path)
    if (it == 0) publish(false);
  }
  ptx::tc_fence_after();
  }  // chunk loop

  if (tid == PUB) publish(false);
  if (warp == 0) {
    ptx::tmem_dealloc(*tslot, kPrepTmemCols);
  }
}

// ---------------------------------------------------------------------------
// 8 f16 (16 bytes) added into 8 fp32
__device__ __forceinline__ void add8_f16(float* x, int4 v) {
  const __half2* hv = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(hv[i]);
    x[2 * i] += f.x;
    x[2 * i + 1] += f.y;
  }
}

// ---------------------------------------------------------------------------
// state pass
// ---------------------------------------------------------------------------
// One CTA per (b, h) walks that head's chunk images in order.  Every product
// is transposed so that its rows are the 128 value columns v (TMEM lanes);
// the carried state is S^T[v, k] (kda.py:176-182):
//   D1 = S16^T (-W)^T     [128 x 64]  = P^T - U^T       (P = U - W S)
//   P16^T = f16(U^T + D1)             -> TMEM, A operand of D3
//   D3 = P16^T Kbar       [128 x 128] = (Kbar^T P)^T
//   S^T <- S^T Diag(d) + D3           fp32 master state, in registers
//   O^T = S16^T E^T + F^T [128 x 64]                    (O = E S + F)
// S16^T is the f16 copy of S both GEMMs use, as the reference rounds S to its
// transient dtype for them (kda.py:176).  A operands come from TMEM (no shared
// memory round trip of S or P); B operands are the chunk image in shared memory.
// Warp roles:
//  * chain warps 0-7: warp w owns TMEM lanes 32 (w % 4) .. +31 (value columns
//    v = 32 (w % 4) + lane) and half w / 4 of every product's columns; thread
//    (v, half) keeps S^T[v, 64 half .. 64 half + 63] in registers.  Per chunk:
//    P hand-off after D1, then the state update after D3, which writes the
//    next chunk's f16 copy of S into the other TMEM buffer.
//  * output warps 8-11: O = F + D2 of each chunk (O double-buffered in TMEM),
//    transposed through a shared-memory tile into 16-byte global stores.
//  * MMA warp 12: one thread issues every GEMM: D1 as soon as S16 is in
//    TMEM, D3 as soon as P16 is, then the chunk's output GEMM, which the
//    tensor pipe runs while the chain warps update the state.
//  * producer warp 13: waits for each image's ready flag (set by the prep grid,
//    which may still be running) and copies the parts the chain needs
//    (-W, Kbar^T, d, U^T: three stages) and the parts the output GEMM and its
//    warps need (E, F^T: two stages) into shared memory.
// Every wait is bounded; on expiry the CTA sets the device error word, lets its
// copies and MMAs in flight finish, frees TMEM and returns.
constexpr int ST_CHAIN_WARPS = 8, ST_OUT_WARPS = 4;
constexpr int ST_MMA_WARP = ST_CHAIN_WARPS + ST_OUT_WARPS;
constexpr int ST_PROD_WARP = ST_MMA_WARP + 1;
constexpr int ST_WARPS = ST_PROD_WARP + 1;
// chain stage: -W [64 x 128] | Kbar^T [128 x 64] | d | U^T
constexpr int CS_W = 0, CS_A3 = 16384, CS_D = 32768, CS_U = 33280, CS_BYTES = 49664;
// output stage: E [64 x 128] | F^T
constexpr int OS_E = 0, OS_F = 16384, OS_BYTES = 32768;
constexpr int ST_NCS = 3, ST_NOS = 2;             // stages per ring
constexpr int ST_OS0 = ST_NCS * CS_BYTES;
constexpr int ST_OT = ST_OS0 + ST_NOS * OS_BYTES;  // output tile O [64][128] (I/O dtype)
constexpr int ST_BAR = ST_OT + CH * KD * 2;
constexpr int ST_SMEM = ST_BAR + 192;
static_assert(ST_SMEM <= 227 * 1024, "state shared memory");
static_assert(CS_D - CS_A3 == IMG_D - IMG_A3 && CS_U - CS_A3 == IMG_U - IMG_A3 &&
                  CS_BYTES - CS_A3 == IMG_F - IMG_A3, "chain stage layout");
// prep (231 KB) and state CTAs can never share an SM, so TMEM allocations of
// the two grids never contend
static_assert(ST_SMEM + PREP_SMEM > 228 * 1024, "prep and state CTAs must not share an SM");
// TMEM columns: D1 fp32 [128 x 64]; D3 fp32 [128 x 128]; O fp32 [128 x 64]
// twice (by chunk parity); two f16 copies of S^T (A operands, 128 keys = 64
// columns each, by chunk parity); P16^T (64 chunk rows = 32 columns)
constexpr uint32_t TC_D1 = 0, TC_D3 = 64, TC_O = 192, TC_S = 320, TC_P = 448;
constexpr uint32_t ST_TMEM_COLS = 512;

// bounded mbarrier wait that also gives up as soon as the CTA is aborting
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity,
                                                   volatile int* abort_flag) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort_flag || ptx::globaltimer_ns() - t0 > kWaitNs) return false;
  }
}
// bounded wait for a chunk image's ready flag (acquire)
__device__ __forceinline__ bool wait_ready(const unsigned int* f, volatile int* abort_flag) {
  if (ptx::ld_acquire_gpu(f)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  for (;;) {
    __nanosleep(32);
    if (ptx::ld_acquire_gpu(f)) return true;
    if (*abort_flag || ptx::globaltimer_ns() - t0 > kWaitNs) return false;
  }
}
// 16-byte chunk j of the 128-byte U^T / F^T row v (swizzled by the prep kernel)
__device__ __forceinline__ const int4* trow_chunk(const uint8_t* rowp, int j, int v) {
  return reinterpret_cast<const int4*>(rowp + ((j ^ (v & 7)) << 4));
}
__device__ __forceinline__ void bar_named(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <typename TIO, typename TSI, typename TSO>
__global__ void __launch_bounds__(ST_WARPS * 32, 1)
state_kernel(const ChunkParams p, const uint8_t* __restrict__ ws,
             const unsigned int* __restrict__ flags) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + ST_BAR);
  uint64_t* cfull = bars;          // [3] chain part landed (producer, bytes)
  uint64_t* cempty = bars + 3;     // [3] chain part consumed (8 chain warps)
  uint64_t* ofull = bars + 6;      // [2] output part landed
  uint64_t* oempty = bars + 8;     // [2] output part consumed (4 output warps)
  uint64_t* odone = bars + 10;     // [2] output GEMM complete (MMA commit)
  uint64_t* ofree = bars + 12;     // [2] O buffer read out (4 output warps)
  uint64_t* d1full = bars + 14;    // D1 complete
  uint64_t* d3full = bars + 15;    // D3 complete
  uint64_t* sready = bars + 16;    // S16 written to TMEM (8 chain warps)
  uint64_t* pready = bars + 17;    // P16 written to TMEM (8 chain warps)
  uint64_t* mfin = bars + 18;      // every MMA issued has completed (teardown)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int T = p.T;
  const int NT = (T + CH - 1) / CH;
  const uint8_t* wsh = ws + (size_t)bh * NT * IMG_BYTES;
  const unsigned int* fl = flags + (size_t)bh * NT;

  if (warp == 0) {
    ptx::tmem_alloc(tslot, ST_TMEM_COLS);
    ptx::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < ST_NCS; ++s) {
      ptx::mbar_init(&cfull[s], 1);
      ptx::mbar_init(&cempty[s], ST_CHAIN_WARPS);
    }
    for (int s = 0; s < ST_NOS; ++s) {
      ptx::mbar_init(&ofull[s], 1);
      ptx::mbar_init(&oempty[s], ST_OUT_WARPS);
      ptx::mbar_init(&odone[s], 1);
      ptx::mbar_init(&ofree[s], ST_OUT_WARPS);
    }
    ptx::mbar_init(d1full, 1);
    ptx::mbar_init(d3full, 1);
    ptx::mbar_init(sready, ST_CHAIN_WARPS);
    ptx::mbar_init(pready, ST_CHAIN_WARPS);
    ptx::mbar_init(mfin, 1);
    ptx::fence_mbar_init();
    *abort_flag = 0;
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == ST_PROD_WARP) {
    // ---- producer: ready flag -> bulk copies of the chain and output parts --
    if (lane == 0) {
      int clast[ST_NCS] = {-1, -1, -1}, olast[ST_NOS] = {-1, -1};
      bool ok = true;
      for (int n = 0; n < NT && ok; ++n) {
        const int cs = n % ST_NCS, os = n & 1;
        const uint8_t* img = wsh + (size_t)n * IMG_BYTES;
        if (n >= ST_NCS) ok = mbar_wait_or_abort(&cempty[cs], (n / ST_NCS - 1) & 1, abort_flag);
        if (ok) ok = wait_ready(fl + n, abort_flag);
        if (!ok) break;
        ptx::fence_proxy_async_global();     // the image was published by the generic proxy
        uint8_t* cst = sm + cs * CS_BYTES;
        ptx::mbar_arrive_expect_tx(&cfull[cs], CS_BYTES);
        ptx::bulk_g2s(cst + CS_W, img + IMG_A1, 16384, &cfull[cs]);
        ptx::bulk_g2s(cst + CS_A3, img + IMG_A3, CS_BYTES - CS_A3, &cfull[cs]);
        clast[cs] = n;
        if (n >= ST_NOS) ok = mbar_wait_or_abort(&oempty[os], ((n >> 1) - 1) & 1, abort_flag);
        if (!ok) break;
        uint8_t* ost = sm + ST_OS0 + os * OS_BYTES;
        ptx::mbar_arrive_expect_tx(&ofull[os], OS_BYTES);
        ptx::bulk_g2s(ost + OS_E, img + IMG_A1 + 16384, 16384, &ofull[os]);
        ptx::bulk_g2s(ost + OS_F, img + IMG_F, 16384, &ofull[os]);
        olast[os] = n;
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(&g_kda_device_error, 1);
      }
      // no copy may still be landing when the CTA's shared memory is released
      for (int s = 0; s < ST_NCS; ++s)
        if (clast[s] >= 0) ptx::mbar_wait(&cfull[s], (clast[s] / ST_NCS) & 1, kWaitNs / 2);
      for (int s = 0; s < ST_NOS; ++s)
        if (olast[s] >= 0) ptx::mbar_wait(&ofull[s], (olast[s] >> 1) & 1, kWaitNs / 2);
    }
  } else if (warp == ST_MMA_WARP) {
    // ---- MMA issue (one thread) ---------------------------------------------
    if (lane == 0) {
      const uint32_t sm0 = ptx::smem_u32(sm);
      constexpr uint32_t ID64 = ptx::idesc_f16_f32(128, 64, false, false);
      constexpr uint32_t ID128 = ptx::idesc_f16_f32(128, 128, false, false);
      bool ok = true;
      for (int n = 0; n < NT && ok; ++n) {
        const int cs = n % ST_NCS, os = n & 1;
        const uint32_t as = tbase + TC_S + 64 * (n & 1);
        // D1 = S16^T (-W)^T: S16(n) in TMEM, image n's chain part landed
        ok = mbar_wait_or_abort(sready, n & 1, abort_flag) &&
             mbar_wait_or_abort(&cfull[cs], (n / ST_NCS) & 1, abort_flag);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint64_t bw = ptx::sdesc(sm0 + cs * CS_BYTES + CS_W, 128, 2048);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          ptx::mma_f16_ts(tbase + TC_D1, as + 8 * ks, bw + 16 * ks, ID64, ks > 0);
        ptx::tc_commit(d1full);
        // D3 = P16^T Kbar once the chain warps wrote P16(n)
        ok = mbar_wait_or_abort(pready, n & 1, abort_flag);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint64_t bk = ptx::sdesc(sm0 + cs * CS_BYTES + CS_A3, 128, 1024);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          ptx::mma_f16_ts(tbase + TC_D3, tbase + TC_P + 8 * ks, bk + 16 * ks, ID128, ks > 0);
        ptx::tc_commit(d3full);
        // O(n) = S16^T(n) E^T into O buffer n & 1 (the output warps read O(n - 2)
        // out of it); the tensor pipe runs it during the state update
        ok = mbar_wait_or_abort(&ofull[os], (n >> 1) & 1, abort_flag);
        if (ok && n >= ST_NOS) ok = mbar_wait_or_abort(&ofree[os], ((n >> 1) - 1) & 1, abort_flag);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint64_t be = ptx::sdesc(sm0 + ST_OS0 + os * OS_BYTES + OS_E, 128, 2048);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          ptx::mma_f16_ts(tbase + TC_O + 64 * os, as + 8 * ks, be + 16 * ks, ID64, ks > 0);
        ptx::tc_commit(&odone[os]);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(&g_kda_device_error, 1);
      }
      // nothing may still run on TMEM when it is released
      ptx::tc_commit(mfin);
      ptx::mbar_wait(mfin, 0, kWaitNs / 2);
    }
    __syncwarp();
  } else if (warp >= ST_CHAIN_WARPS) {
    // ---- output warps: O = F + D2, one value column per thread -------------
    const int v = 32 * (warp - ST_CHAIN_WARPS) + lane;
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * (warp - ST_CHAIN_WARPS)) << 16);
    TIO* obase = static_cast<TIO*>(p.o) + b * p.o_s[0] + h * p.o_s[2];
    // o rows as 16-byte vectors (every row a 16-byte-aligned 256-byte range)
    const bool ovec = (reinterpret_cast<uintptr_t>(p.o) % 16) == 0 && p.o_s[0] % 8 == 0 &&
                      p.o_s[1] % 8 == 0 && p.o_s[2] % 8 == 0;
    TIO* otile = reinterpret_cast<TIO*>(sm + ST_OT);
    const int ot = tid - ST_CHAIN_WARPS * 32;      // 0 .. 127
#pragma unroll 1
    for (int m = 0; m < NT; ++m) {
      const int os = m & 1;
      // the four warps agree, so none is left alone at the tile barriers below
      const bool ok = mbar_wait_or_abort(&odone[os], (m >> 1) & 1, abort_flag) &&
                      mbar_wait_or_abort(&ofull[os], (m >> 1) & 1, abort_flag);
      if (ptx::bar_red_or(2, ST_OUT_WARPS * 32, !ok)) break;
      ptx::tc_fence_after();
      float o[64];
      ptx::tmem_ld<32>(tl + TC_O + 64 * os, o);
      ptx::tmem_ld<32>(tl + TC_O + 64 * os + 32, o + 32);
      ptx::tmem_wait_ld();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&ofree[os]);       // O buffer may be rewritten
      const uint8_t* frow = sm + ST_OS0 + os * OS_BYTES + OS_F + v * 128;
#pragma unroll
      for (int i = 0; i < 8; ++i) add8_f16(o + 8 * i, *trow_chunk(frow, i, v));
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&oempty[os]);      // E (read by O(m)) and F consumed
      bar_named(2, ST_OUT_WARPS * 32);                    // previous tile stored
#pragma unroll
      for (int c = 0; c < CH; ++c) st(otile + c * KD + v, o[c]);
      bar_named(2, ST_OUT_WARPS * 32);                    // tile complete
      // 64 rows x 256 bytes = 1024 vectors of 16 bytes over 128 threads
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = ot + 128 * i, r = idx >> 4, c8 = (idx & 15) * 8;
        const int t = m * CH + r;
        if (t >= T) continue;
        TIO* dst = obase + (int64_t)t * p.o_s[1] + c8;
        const TIO* src = otile + r * KD + c8;
        if (ovec) {
          *reinterpret_cast<int4*>(dst) = *reinterpret_cast<const int4*>(src);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) dst[e] = src[e];
        }
      }
    }
  } else {
    // ---- chain warps --------------------------------------------------------
    const int wq = warp & 3, hh = warp >> 2;
    const int v = 32 * wq + lane;                  // value column = TMEM lane
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * wq) << 16);

    float S[64];                                   // S^T[v, 64 hh + j]
    if (p.state_in != nullptr) {
      const TSI* src = static_cast<const TSI*>(p.state_in) + b * p.si_s[0] + h * p.si_s[1] + v;
#pragma unroll
      for (int j = 0; j < 64; ++j) S[j] = ld(src + (int64_t)(64 * hh + j) * p.si_s[2]);
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j) S[j] = 0.f;
    }
    // f16 copy of S^T (A operand of D1 and the output GEMM) into TMEM buffer
    // `col`, 16 keys at a time
    auto store_s16 = [&](uint32_t col, int q) {
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pk[i] = pack_h2(S[16 * q + 2 * i], S[16 * q + 2 * i + 1]);
      asm volatile(
          "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
              tl + col + 32 * hh + 8 * q),
          "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3]), "r"(pk[4]), "r"(pk[5]), "r"(pk[6]),
          "r"(pk[7])
          : "memory");
    };
    // every arrival of a warp comes after its TMEM stores completed
    auto signal = [&](uint64_t* bar) {
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar);
    };
#pragma unroll
    for (int q = 0; q < 4; ++q) store_s16(TC_S, q);
    signal(sready);
    bool ok = true;
#pragma unroll 1
    for (int n = 0; n < NT; ++n) {
      const int cs = n % ST_NCS;
      const uint8_t* cst = sm + cs * CS_BYTES;
      // (a) P^T = U^T + D1 -> f16 -> TMEM; U^T is read while D1 runs
      ok = mbar_wait_or_abort(&cfull[cs], (n / ST_NCS) & 1, abort_flag);
      if (!ok) break;
      int4 ur[4];
      {
        const uint8_t* urow = cst + CS_U + v * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) ur[i] = *trow_chunk(urow, 4 * hh + i, v);
      }
      ok = mbar_wait_or_abort(d1full, n & 1, abort_flag);
      if (!ok) break;
      ptx::tc_fence_after();
      {
        float x[32];
        ptx::tmem_ld<32>(tl + TC_D1 + 32 * hh, x);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i) add8_f16(x + 8 * i, ur[i]);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_h2(x[2 * i], x[2 * i + 1]);
        ptx::tmem_st<16>(tl + TC_P + 16 * hh, reinterpret_cast<const float*>(pk));
      }
      signal(pready);
      // (b) S^T <- S^T Diag(d) + D3, and its f16 copy for chunk n + 1 into the
      // other TMEM buffer (last read by D1(n - 1) and O(n - 1), which completed
      // before D1(n))
      ok = mbar_wait_or_abort(d3full, n & 1, abort_flag);
      if (!ok) break;
      ptx::tc_fence_after();
      const float* dk = reinterpret_cast<const float*>(cst + CS_D) + 64 * hh;
      const uint32_t snext = TC_S + 64 * ((n + 1) & 1);
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        float x[32];
        ptx::tmem_ld<32>(tl + TC_D3 + 64 * hh + 32 * h2, x);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = reinterpret_cast<const float4*>(dk + 32 * h2)[i];
          float* sp = S + 32 * h2 + 4 * i;
          sp[0] = fmaf(sp[0], t.x, x[4 * i]);
          sp[1] = fmaf(sp[1], t.y, x[4 * i + 1]);
          sp[2] = fmaf(sp[2], t.z, x[4 * i + 2]);
          sp[3] = fmaf(sp[3], t.w, x[4 * i + 3]);
        }
        store_s16(snext, 2 * h2);
        store_s16(snext, 2 * h2 + 1);
      }
      signal(sready);
      if (lane == 0) ptx::mbar_arrive(&cempty[cs]);
    }
    if (!ok) {
      *abort_flag = 1;
      if (lane == 0) atomicExch(&g_kda_device_error, 1);
    } else {
      TSO* dst = static_cast<TSO*>(p.state_out) + b * p.so_s[0] + h * p.so_s[1] + v;
#pragma unroll
      for (int j = 0; j < 64; ++j) st(dst + (int64_t)(64 * hh + j) * p.so_s[2], S[j]);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, ST_TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <typename TIO, typename TSI, typename TSO>
cudaError_t launch_state(const ChunkParams& p, const uint8_t* ws, const unsigned int* flags,
                         cudaStream_t s) {
  auto kern = state_kernel<TIO, TSI, TSO>;
  // per call: the attribute belongs to the current device's context
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       ST_SMEM);
  if (e != cudaSuccess) return e;
  // programmatic dependent of the prep grid: it starts as soon as SMs are free
  // and follows the prep grid chunk by chunk through the ready flags
  return launch_dependent(kern, dim3(p.B * p.H), ST_WARPS * 32, ST_SMEM, s, p, ws, flags);
}

template <typename TIO, int LOAD>
cudaError_t launch_prep(const ChunkParams& p, uint8_t* ws, unsigned int* flags, int ctas,
                        cudaStream_t s, const PrepMaps& maps = PrepMaps{}) {
  auto prep = prep_kernel<TIO, LOAD>;
  // per call: the attribute belongs to the current device's context
  cudaError_t e = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       PREP_SMEM);
  if (e != cudaSuccess) return e;
  prep<<<dim3((unsigned)ctas), PREP_THREADS, PREP_SMEM, s>>>(p, ws, flags, maps);
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

// Persistent prep CTAs for a call.  The state pass needs one SM per (b, h)
// for the whole call; when the heads are few it runs beside the prep grid on
// SMs the prep grid leaves free, so the call costs the prep time on fewer SMs
// plus one chunk of the chain, instead of the full prep time plus the whole
// chain.  Measured costs on B200: ~12.7 us per chunk and prep
// CTA, ~0.7 us per chunk of the state chain.
int prep_ctas_for(long total, int NT, int BH, int sms) {
  constexpr double kPrepUs = 12.7, kChainUs = 0.7;
  auto rounds = [&](long ctas) { return (double)((total + ctas - 1) / ctas); };
  const double sequential = rounds(sms) * kPrepUs + NT * kChainUs;
  const double beside = BH < sms ? rounds(sms - BH) * kPrepUs + kChainUs : 1e300;
  const int ctas = beside < sequential ? sms - BH : sms;
  return (int)(total < ctas ? total : ctas);
}

template <typename TIO, typename TSI, typename TSO>
cudaError_t launch_tc3(const ChunkParams& p, uint8_t* ws, cudaStream_t s) {
  const int NT = (p.T + CH - 1) / CH;
  const long total = (long)NT * p.B * p.H;
  if (total > 0x7fffffffL) return cudaErrorInvalidValue;       // int chunk index
  unsigned int* flags = reinterpret_cast<unsigned int*>(ws + (size_t)total * IMG_BYTES);
  cudaError_t e = cudaMemsetAsync(flags, 0, (size_t)total * sizeof(unsigned int), s);
  if (e != cudaSuccess) return e;
  PrepMaps maps;
  if (bulk_rows_ok<TIO>(p) && make_prep_maps<TIO>(p, &maps)) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = launch_prep<TIO, 3>(p, ws, flags, prep_ctas_for(total, NT, p.B * p.H, sms), s, maps);
  } else {
    const bool vec = p.g_vec2 && p.qk_vec2 && p.v_vec2;
    const int ctas = (int)total;                               // one chunk per CTA
    e = bulk_rows_ok<TIO>(p) ? launch_prep<TIO, 2>(p, ws, flags, ctas, s)
        : vec                ? launch_prep<TIO, 1>(p, ws, flags, ctas, s)
                             : launch_prep<TIO, 0>(p, ws, flags, ctas, s);
  }
  if (e != cudaSuccess) return e;
  return launch_state<TIO, TSI, TSO>(p, ws, flags, s);
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
  return p.K == tc::KD && p.V == tc::KD && p.T >= 1;
}

// chunk images, then one ready flag per image
size_t chunk_tc_workspace_bytes(const ChunkParams& p) {
  const size_t NT = (size_t)(p.T + tc::CH - 1) / tc::CH;
  const size_t n = (size_t)p.B * p.H * NT;
  return n * tc::IMG_BYTES + ((n * sizeof(unsigned int) + 255) & ~(size_t)255);
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
