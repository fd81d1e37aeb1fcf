// mla_decode.cu -- single-token MLA decode over a static latent buffer (sm_100a).
//
// Drop-in for the attention core of MLA._decode_step_static
// (kimi_linear/mla.py:117-181), NoPE (qk_rope_head_dim = 0): with
// W = kv_b_proj.weight viewed [H, DN + DV, KVL] (W_nope = rows < DN, W_v the rest)
//   kv_buf[b, pos] = c_kv[b]                                      (index_copy_)
//   q_lat[b, h]    = q_nope[b, h] W_nope[h]                       (fp32)
//   score[b, h, s] = scale * q_lat[b, h] . kv_buf[b, s],  s <= pos, else -inf
//   p              = softmax_s(score)                             (fp32)
//   mixed[b, h]    = sum_s p kv_buf[b, s]      (p and the result in kv_buf's dtype)
//   out[b, h]      = mixed[b, h] W_v[h]^T                         (fp32, then I/O dtype)
//   pos           += 1
// Three kernels on the caller's stream, reading `pos` from device memory
// (graph-capturable).  All three are launched as programmatic dependents of
// the kernel before them (launch, barrier set-up, the tile loads that do not
// need the previous kernel's output and the W_v loads overlap its tail; the
// first waits before any read, since its inputs come from whatever precedes it):
//  * mla_qlat_kernel: q_lat in fp32 (one CTA per (h, 64-channel slab)); the
//    CTAs of head h also write batch row h's new latent row at pos;
//  * mla_attn_kernel: flash decoding.  One CTA per (split, b) walks 64-position
//    tiles of kv_buf[b] (tiles past pos are not loaded), three TMA stages with a
//    128-byte swizzle, the first tile requested ahead of the others.  Scores: f16/bf16 mma.sync with q_lat split into hi + lo
//    parts (fp32-level scores against exact buffer values), K split over the
//    four warps and summed in shared memory; online softmax in fp32; mixing
//    P . tile with N split over the warps.  Writes (max, sum, acc) partials;
//  * mla_mixout_kernel: per (128-channel slab, h, b) merges the partials,
//    rounds mixed to the buffer dtype as the reference does and projects the
//    slab with W_v in fp32; the last slab CTA of (b, h) writes out[b, h].
//    Advances pos.
#include <cuda.h>
#include <cstring>
#include <type_traits>
#include <utility>

#include "kda_internal.cuh"
#include "tc_ptx.cuh"

namespace kda {
namespace mla {

// this file's device error word (device variables are per translation unit
// without relocatable device code); kda_device_error() reports it too
__device__ int g_mla_device_error = 0;

constexpr int TS = 64;            // positions per tile
constexpr int NW = 4;             // warps per attention CTA
constexpr int HM = 16;            // heads per CTA (MMA M); H <= 16
constexpr int PP = TS * 2 + 16;   // pitch of P [16][64] in bytes (conflict-free ldmatrix)
constexpr int RP = TS + 8;        // pitch of the score partials [16][64] in floats: the
                                  // eight fragment rows of a warp's stores hit distinct banks
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kMaxSplits = 256;   // splits of the position range per batch row

template <typename T> struct MmaT;
template <> struct MmaT<__half> {
  static __device__ __forceinline__ void mma(float* d, const uint32_t* a, const uint32_t* b) {
    ptx::mma_f16_16x8x16(d, a, b);
  }
  static __device__ __forceinline__ uint32_t pack(float x, float y) {
    const __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
  }
};
template <> struct MmaT<__nv_bfloat16> {
  static __device__ __forceinline__ void mma(float* d, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  static __device__ __forceinline__ uint32_t pack(float x, float y) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
  }
};

// x = hi + lo with hi, lo in T (pairs packed): hi carries the leading bits,
// lo the residual, so hi . b + lo . b is the fp32 product to ~2^-17 relative
template <typename T>
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
  hi = MmaT<T>::pack(x, y);
  const float2 h = MmaT<T>::unpack(hi);
  lo = MmaT<T>::pack(x - h.x, y - h.y);
}

// byte offset of (row s, 16-byte chunk j) of a tile of 64-channel boxes
// (TMA SWIZZLE_128B: 128-byte rows, chunk index xor row % 8)
__device__ __forceinline__ int swz(int group, int s, int j) {
  return group * (TS * 128) + s * 128 + ((j ^ (s & 7)) << 4);
}

struct MlaParams {
  int B, L, H, KVL, DN, DV;
  float scale;
  const void* q_nope; int64_t q_s[3];
  const void* c_kv; int64_t c_s[2];
  void* kv_buf; int64_t kv_s[3];
  int64_t* pos;
  const void* w; int64_t w_s[2];
  void* out; int64_t o_s[3];
  float* qlat;      // [B][16][KVL] fp32 (heads >= H zero)
  float* part;      // [B][nsplit][16][KVL + 2]: acc, then max and sum
  float* opart;     // [B][16][nslab][DV] fp32 slab partials of out
  int* count;       // [B][16] slab partials written (zeroed by the q_lat kernel)
  int nsplit, tiles_per_cta, nslab;
  bool w_vec;       // kv_b_proj.weight rows are 16-byte-aligned unit-stride ranges
};

// w[row, c .. c + 7] as fp32 (one 16-byte load when p.w_vec)
template <typename T>
__device__ __forceinline__ void ld8(const MlaParams& p, const T* w, int64_t row, int c,
                                    float (&x)[8]) {
  const T* r = w + row * p.w_s[0];
  if (p.w_vec) {
    const uint4 u = *reinterpret_cast<const uint4*>(r + c);
    const uint32_t v[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = MmaT<T>::unpack(v[i]);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = ld(r + (int64_t)(c + i) * p.w_s[1]);
  }
}

// ---------------------------------------------------------------------------
// One CTA per (head, 64-channel slab): reads its slab of W_nope once for all
// batch rows.  Thread t: 8-channel chunk t % 8 of the slab, rows d = t / 8,
// t / 8 + 32, ...; the 32 row-partials meet in shared memory.  All loads of a
// pass (weights, q_nope, the new latent row) are issued before their first use.
// CTA (h, y) also copies c_kv[b] into kv_buf[b, pos] for b = h, h + 16, ...
// over its channel slab.
constexpr int QL_COLS = 64;       // channels per CTA
constexpr int QL_RG = 32;         // row groups per CTA
constexpr int QL_BB = 4;          // batch rows per pass

template <typename T>
__global__ void __launch_bounds__(256)
mla_qlat_kernel(const MlaParams p) {
  extern __shared__ float part[];  // [QL_RG][QL_BB][QL_COLS] row partials
  const int h = blockIdx.x, c0 = blockIdx.y * QL_COLS, tid = threadIdx.x;
  const int chunk = tid & 7, dsub = tid >> 3;
  const int ncols = min(QL_COLS, p.KVL - c0);         // KVL = 64: half a slab
  // launched as a programmatic dependent of whatever precedes it on the stream
  // (q_nope and c_kv come from it, pos from the previous step's merge grid):
  // nothing is read before the wait
  ptx::grid_dep_wait();
  ptx::grid_dep_launch();                             // the attention grid may start launching
  if (blockIdx.y == 0)                                // slab-partial counters of this call
    for (int b = tid; b < p.B; b += blockDim.x) p.count[b * HM + h] = 0;
  // kv_buf[b, pos] = c_kv[b]: loads here, stores after the weight loads
  const int64_t pos = *p.pos;
  const bool pos_ok = pos >= 0 && pos < p.L;
  const bool lat = tid < ncols && h < p.B;
  T lat_v{};
  if (lat) lat_v = static_cast<const T*>(p.c_kv)[h * p.c_s[0] + (int64_t)(c0 + tid) * p.c_s[1]];
  auto write_latent = [&]() {
    if (!pos_ok) {
      if (h == 0 && blockIdx.y == 0 && tid == 0)
        atomicExch(&g_mla_device_error, 4);           // position outside the buffer
      return;
    }
    T* row = static_cast<T*>(p.kv_buf) + pos * p.kv_s[1] + c0;   // unit channel stride
    if (lat) row[h * p.kv_s[0] + tid] = lat_v;
    for (int b = h + HM; b < p.B; b += HM)            // more than 16 batch rows
      for (int c = tid; c < ncols; c += blockDim.x)
        row[b * p.kv_s[0] + c] =
            static_cast<const T*>(p.c_kv)[b * p.c_s[0] + (int64_t)(c0 + c) * p.c_s[1]];
  };
  if (h >= p.H) {                                     // padded head rows: zero
    for (int b = 0; b < p.B; ++b)
      for (int c = tid; c < ncols; c += blockDim.x)
        p.qlat[((size_t)b * HM + h) * p.KVL + c0 + c] = 0.f;
    write_latent();
    return;
  }
  const T* wb = static_cast<const T*>(p.w) + (int64_t)h * (p.DN + p.DV) * p.w_s[0];
  const T* qn = static_cast<const T*>(p.q_nope) + h * p.q_s[1];
  for (int b0 = 0; b0 < p.B; b0 += QL_BB) {
    const int nb = min(QL_BB, p.B - b0);
    float acc[QL_BB][8];
#pragma unroll
    for (int bb = 0; bb < QL_BB; ++bb)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[bb][e] = 0.f;
    if (8 * chunk < ncols) {
      // rows d = dsub + 32 k, four at a time: their weight and q_nope loads overlap
      for (int d0 = dsub; d0 < p.DN; d0 += 4 * QL_RG) {
        float x[4][8], qv[4][QL_BB];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (d0 + QL_RG * u < p.DN) ld8(p, wb, d0 + QL_RG * u, c0 + 8 * chunk, x[u]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int bb = 0; bb < QL_BB; ++bb)
            qv[u][bb] = (d0 + QL_RG * u < p.DN && bb < nb)
                            ? ld(qn + (b0 + bb) * p.q_s[0] + (int64_t)(d0 + QL_RG * u) * p.q_s[2])
                            : 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (d0 + QL_RG * u >= p.DN) break;
#pragma unroll
          for (int bb = 0; bb < QL_BB; ++bb)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[bb][e] = fmaf(qv[u][bb], x[u][e], acc[bb][e]);
        }
      }
    }
    __syncthreads();                                  // part free
#pragma unroll
    for (int bb = 0; bb < QL_BB; ++bb) {
      float4* dst = reinterpret_cast<float4*>(part + (dsub * QL_BB + bb) * QL_COLS + 8 * chunk);
      dst[0] = make_float4(acc[bb][0], acc[bb][1], acc[bb][2], acc[bb][3]);
      dst[1] = make_float4(acc[bb][4], acc[bb][5], acc[bb][6], acc[bb][7]);
    }
    __syncthreads();
    for (int i = tid; i < nb * QL_COLS; i += blockDim.x) {
      const int bb = i / QL_COLS, c = i - bb * QL_COLS;
      if (c >= ncols) continue;
      float x = 0.f;
#pragma unroll
      for (int ds = 0; ds < QL_RG; ++ds) x += part[(ds * QL_BB + bb) * QL_COLS + c];
      p.qlat[((size_t)(b0 + bb) * HM + h) * p.KVL + c0 + c] = x;
    }
  }
  write_latent();
}

// ---------------------------------------------------------------------------
template <typename T, int KVL>
struct AttnCfg {
  static constexpr int GROUPS = KVL / 64;             // 64-channel TMA boxes per tile
  static constexpr int TILE = TS * KVL * 2;           // bytes per stage
  static constexpr int KW = KVL / NW;                 // score channels per warp
  static constexpr int KSTEPS = KW / 16;
  static constexpr int NTW = KVL / NW / 8;            // mixing n-tiles per warp
  // tile stages in flight: three where they fit
  static constexpr int NST = 3 * TILE + HM * PP + NW * HM * RP * 4 + 128 <= 227 * 1024 ? 3 : 2;
  static constexpr int OFF_P = NST * TILE;            // P [16][64] in T, pitch PP
  static constexpr int OFF_RED = OFF_P + HM * PP;     // [NW][16][RP] fp32 score partials
  static constexpr int OFF_ALPHA = OFF_RED + NW * HM * RP * 4;   // [16] rescale factors
  static constexpr int OFF_BAR = OFF_ALPHA + HM * 4;
  static constexpr int SMEM = OFF_BAR + 64;
  static_assert(SMEM <= 227 * 1024, "mla shared memory");
};

template <typename T, int KVL>
__global__ void __launch_bounds__(NW * 32, 1)
mla_attn_kernel(const MlaParams p, const __grid_constant__ CUtensorMap tm) {
  using C = AttnCfg<T, KVL>;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* Ps = sm + C::OFF_P;
  float* red = reinterpret_cast<float*>(sm + C::OFF_RED);
  float* alpha_s = reinterpret_cast<float*>(sm + C::OFF_ALPHA);
  constexpr int NST = C::NST;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);   // [NST]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + NST);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int sp = blockIdx.x, b = blockIdx.y;
  const int ntiles = (p.L + TS - 1) / TS;
  const int64_t pos = *p.pos;                         // valid positions: 0 .. pos
  const int last = (int)(pos < (int64_t)p.L - 1 ? pos : (int64_t)p.L - 1);
  const int t_beg = sp * p.tiles_per_cta;
  const int t_end = min(min(ntiles, t_beg + p.tiles_per_cta), last / TS + 1);
  const int lm_row = (lane & 7) + 8 * ((lane >> 3) & 1);
  const int lm_hi = lane >> 4;

  if (tid == 0) {
    for (int st = 0; st < NST; ++st) ptx::mbar_init(&full[st], 1);
    ptx::fence_mbar_init();
    *abort_flag = 0;
  }
  ptx::grid_dep_launch();                             // the merge grid may start launching
  __syncthreads();
  auto fetch = [&](int t, int stage) {                // thread 0 only
    ptx::mbar_arrive_expect_tx(&full[stage], C::TILE);
    for (int g = 0; g < C::GROUPS; ++g)
      ptx::tma_load_3d(sm + stage * C::TILE + g * TS * 128, &tm, 64 * g, t * TS, b, &full[stage]);
  };
  // The first tile is requested alone and the other first-stage tiles once it
  // has landed: with every CTA asking for all of its stages at once, the
  // first tiles share HBM with the later ones and compute starts late.  Only
  // the tile holding pos is written by the q_lat grid (the new latent row), so
  // unless it is that tile the first one loads while that grid still runs.
  uint32_t pending = 0, pend_par = 0;
  const int pos_tile = last / TS;
  if (tid == 0 && t_beg < t_end && t_beg != pos_tile) {
    fetch(t_beg, 0);
    pending |= 1u;
  }
  ptx::grid_dep_wait();                               // q_lat and kv_buf[., pos] visible
  if (tid == 0 && t_beg < t_end && t_beg == pos_tile) {
    ptx::fence_proxy_async_global();
    fetch(t_beg, 0);
    pending |= 1u;
  }

  // q_lat of this warp's channel range as hi / lo A fragments
  uint32_t ahi[C::KSTEPS][4], alo[C::KSTEPS][4];
  {
    const float* ql = p.qlat + (size_t)b * HM * KVL;
#pragma unroll
    for (int ks = 0; ks < C::KSTEPS; ++ks) {
      const int c = warp * C::KW + 16 * ks + 2 * tig;
      const float2 r0 = *reinterpret_cast<const float2*>(ql + gid * KVL + c);
      const float2 r1 = *reinterpret_cast<const float2*>(ql + (gid + 8) * KVL + c);
      const float2 r2 = *reinterpret_cast<const float2*>(ql + gid * KVL + c + 8);
      const float2 r3 = *reinterpret_cast<const float2*>(ql + (gid + 8) * KVL + c + 8);
      split2<T>(r0.x, r0.y, ahi[ks][0], alo[ks][0]);
      split2<T>(r1.x, r1.y, ahi[ks][1], alo[ks][1]);
      split2<T>(r2.x, r2.y, ahi[ks][2], alo[ks][2]);
      split2<T>(r3.x, r3.y, ahi[ks][3], alo[ks][3]);
    }
  }
  // running softmax state (threads: head tid / 8, 8 positions each) and the
  // output accumulator (warp: channels 128 w .., rows gid and gid + 8)
  float m_run = -INFINITY, l_run = 0.f;
  float acc[C::NTW][4];
#pragma unroll
  for (int nt = 0; nt < C::NTW; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  int k = 0;
  for (int t = t_beg; t < t_end; ++t, ++k) {
    const int stage = k % NST;
    const uint8_t* tile = sm + stage * C::TILE;
    const bool landed = ptx::mbar_wait(&full[stage], (k / NST) & 1, kWaitNs);
    if (landed) {
      if (tid == 0) pending &= ~(1u << stage);
    } else {
      *abort_flag = 1;
    }
    if (k == 0 && tid == 0 && landed) {               // the rest of the first stages
      ptx::fence_proxy_async_global();
      for (int i = 1; i < NST && t_beg + i < t_end; ++i) {
        fetch(t_beg + i, i);
        pending |= 1u << i;
      }
    }
    // ---- scores: this warp's KW channels, all 64 positions
    float sc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < C::KSTEPS; ++ks) {
      const int c0 = warp * C::KW + 16 * ks;          // multiple of 16
      const int g = c0 >> 6, j0 = (c0 & 63) >> 3;
#pragma unroll
      for (int np = 0; np < 4; ++np) {                // pairs of 8-position n-tiles
        // matrices: (rows 16np.., chunk j0), (.., j0 + 1), (rows 16np + 8.., j0), (.., j0 + 1)
        const int s = 16 * np + (lane & 7) + 8 * lm_hi;
        const int j = j0 + ((lane >> 3) & 1);
        uint32_t bf[4];
        ptx::ldmatrix_x4(bf, tile + swz(g, s, j));
        MmaT<T>::mma(sc[2 * np], ahi[ks], bf);
        MmaT<T>::mma(sc[2 * np], alo[ks], bf);
        MmaT<T>::mma(sc[2 * np + 1], ahi[ks], bf + 2);
        MmaT<T>::mma(sc[2 * np + 1], alo[ks], bf + 2);
      }
    }
    {
      float* rw = red + warp * HM * RP;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int s = 8 * nt + 2 * tig;
        *reinterpret_cast<float2*>(rw + gid * RP + s) = make_float2(sc[nt][0], sc[nt][1]);
        *reinterpret_cast<float2*>(rw + (gid + 8) * RP + s) = make_float2(sc[nt][2], sc[nt][3]);
      }
    }
    __syncthreads();
    if (*abort_flag) break;
    // ---- online softmax: thread -> head hh, positions 4 q .. 4 q + 3 and
    // 32 + 4 q .. 32 + 4 q + 3 (16-byte reads: the eight threads of a head
    // cover 128 contiguous bytes per read)
    {
      const int hh = tid >> 3, q = tid & 7;
      float v[8];
      float mt = -INFINITY;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int s0 = 32 * half + 4 * q;
        float4 x = *reinterpret_cast<const float4*>(red + hh * RP + s0);
#pragma unroll
        for (int w = 1; w < NW; ++w) {
          const float4 y = *reinterpret_cast<const float4*>(red + w * HM * RP + hh * RP + s0);
          x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
        }
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float xv = xs[i] * p.scale;
          if ((int64_t)t * TS + s0 + i > last || hh >= p.H) xv = -INFINITY;
          v[4 * half + i] = xv;
          mt = fmaxf(mt, xv);
        }
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m_run, mt);
      // __expf (ex2.approx based, ~1e-6 relative here): p is rounded to the
      // buffer dtype right after, which dominates the error by far
      const float a = (m_new == -INFINITY) ? 1.f : __expf(m_run - m_new);
      float ls = 0.f;
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const float e0 = (v[i] == -INFINITY) ? 0.f : __expf(v[i] - m_new);
        const float e1 = (v[i + 1] == -INFINITY) ? 0.f : __expf(v[i + 1] - m_new);
        ls += e0 + e1;
        pk[i / 2] = MmaT<T>::pack(e0, e1);
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
      l_run = l_run * a + ls;
      m_run = m_new;
      *reinterpret_cast<uint2*>(Ps + hh * PP + 8 * q) = make_uint2(pk[0], pk[1]);
      *reinterpret_cast<uint2*>(Ps + hh * PP + 64 + 8 * q) = make_uint2(pk[2], pk[3]);
      if (q == 0) alpha_s[hh] = a;
    }
    __syncthreads();
    // ---- acc = alpha acc + P . tile for this warp's channels
    {
      const float a0 = alpha_s[gid], a1 = alpha_s[gid + 8];
#pragma unroll
      for (int nt = 0; nt < C::NTW; ++nt) {
        acc[nt][0] *= a0; acc[nt][1] *= a0;
        acc[nt][2] *= a1; acc[nt][3] *= a1;
      }
#pragma unroll
      for (int ks = 0; ks < TS / 16; ++ks) {
        uint32_t af[4];
        ptx::ldmatrix_x4(af, Ps + lm_row * PP + (16 * ks + 8 * lm_hi) * 2);
#pragma unroll
        for (int np = 0; np < C::NTW / 2; ++np) {
          // B[k = s][n = c]: rows s, transposed; matrices (s 16ks.., c 16np'..),
          // (s 16ks + 8.., same c), (s 16ks.., c + 8), (s 16ks + 8.., c + 8)
          const int c0 = warp * (KVL / NW) + 16 * np;
          const int g = c0 >> 6, j = ((c0 & 63) >> 3) + lm_hi;
          const int s = 16 * ks + (lane & 7) + 8 * ((lane >> 3) & 1);
          uint32_t bf[4];
          ptx::ldmatrix_x4_trans(bf, tile + swz(g, s, j));
          MmaT<T>::mma(acc[2 * np], af, bf);
          MmaT<T>::mma(acc[2 * np + 1], af, bf + 2);
        }
      }
    }
    __syncthreads();                                  // stage, P and red free
    if (tid == 0 && t + NST < t_end) {
      ptx::fence_proxy_async_smem();
      fetch(t + NST, stage);
      pending |= 1u << stage;
      pend_par = (pend_par & ~(1u << stage)) | ((((k + NST) / NST) & 1u) << stage);
    }
  }

  if (*abort_flag) {
    if (tid == 0) {
      atomicExch(&g_mla_device_error, 5);
      for (int st = 0; st < NST; ++st)
        if (pending & (1u << st)) ptx::mbar_wait(&full[st], (pend_par >> st) & 1u, kWaitNs / 2);
    }
    return;
  }
  // partials: acc rows (heads) gid, gid + 8; then max and sum per head
  float* pb = p.part + (((size_t)b * p.nsplit + sp) * HM) * (KVL + 2);
#pragma unroll
  for (int nt = 0; nt < C::NTW; ++nt) {
    const int c = warp * (KVL / NW) + 8 * nt + 2 * tig;
    *reinterpret_cast<float2*>(pb + gid * (KVL + 2) + c) = make_float2(acc[nt][0], acc[nt][1]);
    *reinterpret_cast<float2*>(pb + (gid + 8) * (KVL + 2) + c) = make_float2(acc[nt][2], acc[nt][3]);
  }
  if ((tid & 7) == 0) {
    const int hh = tid >> 3;
    pb[hh * (KVL + 2) + KVL] = m_run;
    pb[hh * (KVL + 2) + KVL + 1] = l_run;
  }
}

// ---------------------------------------------------------------------------
// mla_mixout_kernel: one CTA per (128-channel slab, head, batch row), a thread
// per channel: merges the splits' partials into mixed = sum p kv_buf / sum p,
// rounded to the buffer dtype (the reference's p.to(buf.dtype) @ buf returns
// that dtype), then projects the slab with its columns of W_v (thread d: out
// row d) in fp32 into a slab partial.  The last CTA of (b, h) to finish sums
// the slab partials in slab order and writes out[b, h] in the I/O dtype.
// CTA (0, 0, 0) advances pos.
constexpr int MX_COLS = 128;
constexpr int MX_PF = 48;         // splits loaded before the merge weights are known

template <typename T>
__global__ void __launch_bounds__(MX_COLS)
mla_mixout_kernel(const MlaParams p) {
  __shared__ float wsc[kMaxSplits];
  __shared__ float red[MX_COLS / 32];
  __shared__ __align__(16) float mixed[MX_COLS];
  __shared__ float max_s, tot_s;
  __shared__ int last_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int slab = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int KVL = p.KVL, ns = p.nsplit, c0 = slab * MX_COLS, c = c0 + tid;
  const int ncols = min(MX_COLS, KVL - c0);
  // W_v[h, d = tid, slab]: no earlier grid of this call writes it, so its
  // loads are issued before waiting for the attention grid
  const T* wv = static_cast<const T*>(p.w) + ((int64_t)h * (p.DN + p.DV) + p.DN) * p.w_s[0];
  const bool wpre = p.w_vec && tid < p.DV;
  uint4 wr[MX_COLS / 8];
#pragma unroll
  for (int j = 0; j < MX_COLS / 8; ++j)
    if (wpre && 8 * j < ncols)
      wr[j] = *reinterpret_cast<const uint4*>(wv + (int64_t)tid * p.w_s[0] + c0 + 8 * j);
  ptx::grid_dep_wait();                               // the attention partials are visible
  ptx::grid_dep_launch();                             // a following dependent grid may launch
  if (slab == 0 && h == 0 && b == 0 && tid == 0) *p.pos += 1;   // its readers have finished

  const float* pb = p.part + ((size_t)b * ns * HM + h) * (KVL + 2);
  const size_t sstride = (size_t)HM * (KVL + 2);
  // this channel's values of the first MX_PF splits: in flight during the weights
  float v[MX_PF];
#pragma unroll
  for (int u = 0; u < MX_PF; ++u) v[u] = (u < ns && tid < ncols) ? pb[u * sstride + c] : 0.f;
  // (max, sum) of split tid (kMaxSplits <= 2 * MX_COLS: at most two per thread)
  static_assert(kMaxSplits <= 2 * MX_COLS, "two splits per merge thread");
  float2 ml0 = make_float2(-INFINITY, 0.f), ml1 = make_float2(-INFINITY, 0.f);
  if (tid < ns) ml0 = *reinterpret_cast<const float2*>(pb + tid * sstride + KVL);
  if (tid + MX_COLS < ns) ml1 = *reinterpret_cast<const float2*>(pb + (tid + MX_COLS) * sstride + KVL);
  float M = fmaxf(ml0.x, ml1.x);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  if (tid == 0) {
    float m = red[0];
    for (int w = 1; w < MX_COLS / 32; ++w) m = fmaxf(m, red[w]);
    max_s = m;
  }
  __syncthreads();
  M = max_s;
  float lw = 0.f;
  if (tid < ns) {
    const float wi = ml0.x == -INFINITY ? 0.f : expf(ml0.x - M);
    wsc[tid] = wi;
    lw = wi * ml0.y;
  }
  if (tid + MX_COLS < ns) {
    const float wi = ml1.x == -INFINITY ? 0.f : expf(ml1.x - M);
    wsc[tid + MX_COLS] = wi;
    lw = fmaf(wi, ml1.y, lw);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
  __syncthreads();                                    // every thread has read red[] (max)
  if (lane == 0) red[warp] = lw;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < MX_COLS / 32; ++w) t += red[w];
    tot_s = t;
  }
  __syncthreads();
  const float inv = tot_s > 0.f ? 1.f / tot_s : 0.f;
  // sixteen independent partial sums (split i into sum i % 16)
  float xs[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) xs[u] = 0.f;
#pragma unroll
  for (int u = 0; u < MX_PF; ++u) xs[u % 16] = fmaf(u < ns ? wsc[u] : 0.f, v[u], xs[u % 16]);
  for (int i = MX_PF; i < ns; i += 16) {
    float w16[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) w16[u] = (i + u < ns && tid < ncols) ? pb[(i + u) * sstride + c] : 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u) xs[u] = fmaf(i + u < ns ? wsc[i + u] : 0.f, w16[u], xs[u]);
  }
  float x = 0.f;
#pragma unroll
  for (int u = 0; u < 16; ++u) x += xs[u];
  if (tid < ncols) mixed[tid] = static_cast<float>(static_cast<T>(x * inv));
  __syncthreads();

  // slab partial of out[b, h, d], d = tid, tid + 128, ...
  float* op = p.opart + (((size_t)b * HM + h) * p.nslab + slab) * p.DV;
  for (int d = tid; d < p.DV; d += MX_COLS) {
    float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};   // independent chains
#pragma unroll
    for (int j = 0; j < MX_COLS / 8; ++j) {
      if (8 * j >= ncols) break;
      float w8[8];
      if (wpre && d == tid) {
        const uint32_t u4[4] = {wr[j].x, wr[j].y, wr[j].z, wr[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = MmaT<T>::unpack(u4[i]);
          w8[2 * i] = f.x;
          w8[2 * i + 1] = f.y;
        }
      } else {
        ld8(p, wv, d, c0 + 8 * j, w8);
      }
      const float4 m0 = *reinterpret_cast<const float4*>(mixed + 8 * j);
      const float4 m1 = *reinterpret_cast<const float4*>(mixed + 8 * j + 4);
      acc8[0] = fmaf(m0.x, w8[0], acc8[0]); acc8[1] = fmaf(m0.y, w8[1], acc8[1]);
      acc8[2] = fmaf(m0.z, w8[2], acc8[2]); acc8[3] = fmaf(m0.w, w8[3], acc8[3]);
      acc8[4] = fmaf(m1.x, w8[4], acc8[4]); acc8[5] = fmaf(m1.y, w8[5], acc8[5]);
      acc8[6] = fmaf(m1.z, w8[6], acc8[6]); acc8[7] = fmaf(m1.w, w8[7], acc8[7]);
    }
    op[d] = ((acc8[0] + acc8[1]) + (acc8[2] + acc8[3])) + ((acc8[4] + acc8[5]) + (acc8[6] + acc8[7]));
  }
  // the barrier orders every thread's slab-partial stores before thread 0's
  // release; its acquire orders the last CTA's reads after the other CTAs' stores
  __syncthreads();
  if (tid == 0) last_s = ptx::atom_add_acq_rel_gpu(p.count + b * HM + h, 1) == p.nslab - 1;
  __syncthreads();
  if (!last_s) return;
  const float* ob_part = p.opart + ((size_t)b * HM + h) * p.nslab * p.DV;
  T* ob = static_cast<T*>(p.out) + b * p.o_s[0] + h * p.o_s[1];
  for (int d = tid; d < p.DV; d += MX_COLS) {
    float y = 0.f;
    for (int k = 0; k < p.nslab; ++k) y += __ldcg(ob_part + (size_t)k * p.DV + d);
    st(ob + (int64_t)d * p.o_s[2], y);
  }
}

}  // namespace mla
}  // namespace kda

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace kda {
namespace mla {
namespace {

// positions split over CTAs: about one CTA per SM over all batch rows
void plan(int B, int L, int num_sms, int* nsplit, int* tpc) {
  const int ntiles = (L + TS - 1) / TS;
  int t = (int)(((long)ntiles * B + num_sms - 1) / num_sms);
  t = max(t, 1);
  int n = (ntiles + t - 1) / t;
  if (n > kMaxSplits) {
    t = (ntiles + kMaxSplits - 1) / kMaxSplits;
    n = (ntiles + t - 1) / t;
  }
  *nsplit = n;
  *tpc = t;
}

int device_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int num_slabs(int KVL) { return (KVL + MX_COLS - 1) / MX_COLS; }

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// workspace: q_lat | split partials | out slab partials | counters
size_t ws_bytes(int B, int L, int KVL, int DV) {
  int ns, tpc;
  plan(B, L, device_sms(), &ns, &tpc);
  const size_t qlat = (size_t)B * HM * KVL * 4;
  const size_t part = (size_t)B * ns * HM * (KVL + 2) * 4;
  const size_t opart = (size_t)B * HM * num_slabs(KVL) * DV * 4;
  const size_t count = (size_t)B * HM * 4;
  return align256(qlat) + align256(part) + align256(opart) + count;
}

bool kvl_ok(int kvl) { return kvl == 64 || kvl == 128 || kvl == 256 || kvl == 512; }

int validate(const MlaDecodeArgs* a) {
  if (a == nullptr) return KDA_ERR_NULL_POINTER;
  if (a->abi_version != KDA_B200_ABI_VERSION) return KDA_ERR_SHAPE;
  if (a->B < 1 || a->L < 1 || a->H < 1 || a->H > HM || !kvl_ok(a->KVL) || a->DN < 1 ||
      a->DV < 1 || a->B > 65535)
    return KDA_ERR_SHAPE;
  if (a->io_dtype != KDA_DTYPE_F16 && a->io_dtype != KDA_DTYPE_BF16) return KDA_ERR_DTYPE;
  if (!a->q_nope || !a->c_kv || !a->kv_buf || !a->pos || !a->w || !a->out || !a->workspace)
    return KDA_ERR_NULL_POINTER;
  // kv_buf goes through a tensor map: unit channel stride, 16-byte rows
  if (a->kv_buf_stride[2] != 1) return KDA_ERR_STRIDE;
  if (reinterpret_cast<uintptr_t>(a->kv_buf) % 16 || (a->kv_buf_stride[0] * 2) % 16 ||
      (a->kv_buf_stride[1] * 2) % 16 || a->kv_buf_stride[0] <= 0 || a->kv_buf_stride[1] <= 0)
    return KDA_ERR_ALIGNMENT;
  if (reinterpret_cast<uintptr_t>(a->workspace) % 256 ||
      reinterpret_cast<uintptr_t>(a->pos) % 8)
    return KDA_ERR_ALIGNMENT;
  if (a->workspace_bytes < ws_bytes(a->B, a->L, a->KVL, a->DV)) return KDA_ERR_WORKSPACE;
  return KDA_OK;
}

template <typename T, int KVL>
cudaError_t launch_attn(const MlaParams& p, const CUtensorMap& tm, cudaStream_t s) {
  auto k = mla_attn_kernel<T, KVL>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       AttnCfg<T, KVL>::SMEM);
  if (e != cudaSuccess) return e;
  return launch_dependent(k, dim3(p.nsplit, p.B), NW * 32, AttnCfg<T, KVL>::SMEM, s, p, tm);
}

template <typename T>
cudaError_t launch_all(const MlaParams& p, const CUtensorMap& tm, cudaStream_t s) {
  // programmatic dependent too: it waits for the preceding kernel before its
  // first read, and its launch overlaps that kernel's tail when the kernel
  // triggers early (the previous step's merge grid does)
  const size_t qsm = (size_t)QL_RG * QL_BB * QL_COLS * sizeof(float);
  cudaError_t e = launch_dependent(mla_qlat_kernel<T>, dim3(HM, (p.KVL + QL_COLS - 1) / QL_COLS),
                                   256, qsm, s, p);
  if (e != cudaSuccess) return e;
  switch (p.KVL) {
    case 64: e = launch_attn<T, 64>(p, tm, s); break;
    case 128: e = launch_attn<T, 128>(p, tm, s); break;
    case 256: e = launch_attn<T, 256>(p, tm, s); break;
    default: e = launch_attn<T, 512>(p, tm, s); break;
  }
  if (e != cudaSuccess) return e;
  return launch_dependent(mla_mixout_kernel<T>, dim3(p.nslab, p.H, p.B), MX_COLS, 0, s, p);
}

}  // namespace

int read_device_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_mla_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_mla_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

}  // namespace mla
}  // namespace kda

extern "C" {

size_t mla_decode_workspace_bytes(const MlaDecodeArgs* a) {
  if (a == nullptr || a->B < 1 || a->L < 1 || a->DV < 1 || !kda::mla::kvl_ok(a->KVL)) return 0;
  return kda::mla::ws_bytes(a->B, a->L, a->KVL, a->DV);
}

size_t mla_decode_args_size(void) { return sizeof(MlaDecodeArgs); }

int mla_decode_fwd(const MlaDecodeArgs* a, void* stream) {
  using namespace kda;
  using namespace kda::mla;
  int st = validate(a);
  if (st != KDA_OK) return st;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return KDA_ERR_LAUNCH;
  if (major != 10) return KDA_ERR_ARCH;
  MlaParams p{};
  p.B = a->B; p.L = a->L; p.H = a->H; p.KVL = a->KVL; p.DN = a->DN; p.DV = a->DV;
  p.scale = a->scale;
  p.q_nope = a->q_nope; std::memcpy(p.q_s, a->q_nope_stride, sizeof(p.q_s));
  p.c_kv = a->c_kv; std::memcpy(p.c_s, a->c_kv_stride, sizeof(p.c_s));
  p.kv_buf = a->kv_buf; std::memcpy(p.kv_s, a->kv_buf_stride, sizeof(p.kv_s));
  p.pos = a->pos;
  p.w = a->w; std::memcpy(p.w_s, a->w_stride, sizeof(p.w_s));
  p.out = a->out; std::memcpy(p.o_s, a->out_stride, sizeof(p.o_s));
  p.w_vec = a->w_stride[1] == 1 && reinterpret_cast<uintptr_t>(a->w) % 16 == 0 &&
            (a->w_stride[0] * 2) % 16 == 0;
  plan(p.B, p.L, device_sms(), &p.nsplit, &p.tiles_per_cta);
  p.nslab = num_slabs(p.KVL);
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  p.qlat = reinterpret_cast<float*>(ws);
  ws += align256((size_t)p.B * HM * p.KVL * 4);
  p.part = reinterpret_cast<float*>(ws);
  ws += align256((size_t)p.B * p.nsplit * HM * (p.KVL + 2) * 4);
  p.opart = reinterpret_cast<float*>(ws);
  ws += align256((size_t)p.B * HM * p.nslab * p.DV * 4);
  p.count = reinterpret_cast<int*>(ws);
  // kv_buf [B, L, KVL] as a 3-D tensor map: boxes of 64 channels x 64 positions
  EncodeTiled enc = encode_tiled();
  if (enc == nullptr) return KDA_ERR_LAUNCH;
  CUtensorMap tm;
  const cuuint64_t dims[3] = {(cuuint64_t)p.KVL, (cuuint64_t)p.L, (cuuint64_t)p.B};
  const cuuint64_t strides[2] = {(cuuint64_t)(p.kv_s[1] * 2), (cuuint64_t)(p.kv_s[0] * 2)};
  const cuuint32_t box[3] = {64u, (cuuint32_t)TS, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt = a->io_dtype == KDA_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (enc(&tm, dt, 3, a->kv_buf, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return KDA_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = a->io_dtype == KDA_DTYPE_F16 ? launch_all<__half>(p, tm, s)
                                               : launch_all<__nv_bfloat16>(p, tm, s);
  return e == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}

}  // extern "C"
