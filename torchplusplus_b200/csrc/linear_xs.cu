// Decode-shaped linear layers, x-stationary form:
//   y[M, N] = epilogue(x[M, K] . W[N, K]^T)      for M <= 32, N <= 64 x SMs.
//
// At decode the weights are read once per step and M is a handful of tokens.
// Two measured B200 facts shape this kernel:
//  * Back-to-back tcgen05.mma instructions never cost less than ~52 SM clocks
//    each for N <= 64 (a single one's latency is ~390), so with 32 tokens on
//    one side the 5th-generation path sustains ~1250 FMA/clock/SM, about
//    what warp-level mma.sync m16n8k16 gives (~1000 FMA/clock/SM from four
//    warps) without TMEM traffic or a single issuing thread.  (Large GEMMs
//    stay on tcgen05 in linear_tc.cu.)
//  * A CTA's TMA throughput is set by its number of requests (~0.2 us each)
//    more than by their size, so operands arrive in few large chunks.
// Design:
//  * Every CTA owns NR complete output rows (NR = N / SMs rounded up to 8,
//    <= 64): no split-K, no cross-CTA reduction.  The tokens are the MMA's M
//    side (16 or 32), the CTA's weight rows its N side.
//  * One producer warp streams chunks of KC 64-wide k-blocks: the weight part
//    as one 3-D TMA box {64, NR, KC} (or one bulk copy from a packed image),
//    the x part as one box {64, T, KC} (or a bulk copy of packed x), into a
//    ring of full/empty mbarriers.  The weight parts of the first `stages`
//    chunks are requested before the programmatic-dependent-launch wait.
//  * Four compute warps: warp w takes k16 step w of every k-block (ldmatrix
//    from the 128-byte-swizzled tiles, conflict-free), accumulating all
//    tokens x rows in registers; a shared-memory reduction over the warps
//    precedes the epilogue.
//  * SwiGLU: the weight part of each k-block holds G gate rows then the G
//    matching up rows (a 4-D box over W viewed as [2][N][K]).
//  * Fused RMSNorm (norm weight folded into W): each token's sum of squares
//    comes from the A fragments the MMAs already load.
//  * Epilogue: bias, activation / SwiGLU, residual (prefetched into shared
//    memory while the weights stream), 16-byte stores, optionally a second
//    packed copy of y for the next decode linear.
// Reference: csrc/blas/hgemv/hgemv_kernels.cuh:19-85 (one warp per row, fp16
// accumulation, never built) and the CUTLASS Sm80 fused linear of
// csrc/activation/fused_gemm.cuh:143-170.  Accumulation here is fp32.
#include <cuda_fp8.h>
#include <stdlib.h>
#include "tc_common.cuh"
#include "mma_common.cuh"

namespace tpp {
namespace {

// Compute warps per CTA (plus one producer warp).  Kept a function of the
// register tile: 12 or 16 warps for the wide slices measured no faster (16
// spill at the 544-thread register cap).
__host__ __device__ constexpr int xs_warps(int) { return 8; }
__host__ __device__ constexpr int xs_threads(int ntm) { return (xs_warps(ntm) + 1) * 32; }
constexpr int kMaxNT = 8;                      // 8-row n-tiles per CTA (NR <= 64)
// Register tiles are sized for NTM n-tiles (2, 4 or 8).  Up to 4 the kernel
// fits two CTAs per SM, so the next kernel's CTA can be resident (and
// prefetch its weights) while this one finishes.
constexpr int kMaxStages = 4;
constexpr size_t kBudget = 110 * 1024;  // two CTAs (of two kernels) per SM
constexpr size_t kBudget16 = 72 * 1024; // 16-token tiles: three CTAs per SM
constexpr size_t kBudget1 = 227 * 1024; // one CTA per SM

bool tsplit_enabled();
bool wide_enabled();
int xs_trigger_at();
}  // namespace
int xs_outputs_per_cta(int64_t N, int act);
int xs_token_tile(int64_t M);
namespace {

struct XsArgs {
  const void* bias;
  const void* residual;
  void* y;
  int64_t ldy;
  int M, N, K;
  int act;
  int nr;      // weight rows per CTA (SwiGLU: gate rows + up rows)
  int kc;      // k-blocks per chunk
  int nch;     // chunks
  int stages;  // ring depth
  int vec_ok;
  float eps;   // fused RMSNorm (NORM variant)
  int* err;
  // Packed operands (optional): W as per-CTA images [cta][kb][NR][128 B] and
  // x / y as [kb][T][128 B], both in the 128-byte-swizzled order the kernel
  // stages, so every chunk is one contiguous bulk copy.
  const uint8_t* wpk;
  const uint8_t* xpk;
  uint8_t* ypk;
  // fp8 weights (W8 variant): per-row dequantisation scales [N] (SwiGLU: [2N])
  const float* wscale;
  int trigger_at;  // dependents released: 0 at the wait, 1 once x has landed, 2 after the MMAs
#ifdef TPP_DEBUG_STAMPS
  unsigned dbg_id;
#endif
};

#ifdef TPP_DEBUG_STAMPS
// [launch % 64][cta < 256][16] globaltimer stamps
__device__ unsigned long long g_xs_stamps[64 * 256 * 16];
unsigned g_xs_launch = 0;
#define XS_TS(i) do { if (blockIdx.x < 256) { unsigned long long _t; \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(_t)); \
    g_xs_stamps[((p.dbg_id % 64) * 256 + blockIdx.x) * 16 + (i)] = _t; } } while (0)
#else
#define XS_TS(i) do {} while (0)
#endif

// Shared-memory plan; W8: fp8 weights, 64 bytes per row and k-block.
template <int BN, int KW, bool W8 = false>
struct XsPlan {
  static constexpr uint32_t kWRow = W8 ? 64 : 128;  // weight bytes per row and k-block
  // weight part of a stage, padded so the x part after it keeps the
  // 1024-byte alignment of a 128-byte-swizzled TMA destination
  __host__ __device__ static uint32_t wpart(int nr, int kc) {
    return ((uint32_t)nr * kWRow * kc + 1023) & ~1023u;
  }
  __host__ __device__ static uint32_t stage(int nr, int kc) {
    return wpart(nr, kc) + (uint32_t)BN * 128 * kc;
  }
  __host__ __device__ static uint32_t red(int nr) { return (uint32_t)KW * BN * (nr + 4) * 4; }
  static uint32_t rsd(int nro) { return ((uint32_t)BN * nro * 2 + 15) & ~15u; }
  __host__ __device__ static size_t ring(int nr, int kc, int stages) {
    const size_t r = (size_t)stages * stage(nr, kc);
    return r > red(nr) ? r : red(nr);
  }
  static size_t smem(int nr, int nro, int kc, int stages) {
    return 1024 + ring(nr, kc, stages) + 4096 + rsd(nro);
  }
};

template <typename T>
__device__ __forceinline__ float sq2(uint32_t v) {
  float2 f;
  if constexpr (IsBf16<T>::value) f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
  else f = __half22float2(*reinterpret_cast<__half2*>(&v));
  return f.x * f.x + f.y * f.y;
}

// fp16 / bf16 pair from two e4m3 bytes (low byte -> low half); exact
template <typename T>
__device__ __forceinline__ uint32_t e4m3x2_to(uint32_t v16) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)v16));
  if constexpr (IsBf16<T>::value) {
    const float2 f = __half22float2(*reinterpret_cast<__half2*>(&h));
    __nv_bfloat162 b = __float22bfloat162_rn(f);
    return *reinterpret_cast<uint32_t*>(&b);
  } else {
    return h;
  }
}

// Global loads issued where they are written (asm volatile keeps them ahead
// of the MMA loop instead of being sunk next to their use).
__device__ __forceinline__ float ldg_early_f32(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ldg_early_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// NTC > 0: the slice's n-tile count as a compile-time constant.  The MMA
// loop's per-n-tile guards then fold away; with a runtime count they split
// each k-block's MMAs with branches and the loop runs ~2x slower (measured
// on the gate/up slice: 3334 vs 1618 SM clocks per pass).
template <typename T, int BN, int NTM, bool SWIGLU, bool NORM, bool W8, int NTC = 0>
__global__ void __launch_bounds__(xs_threads(NTM), NTM > 4 ? 1 : (BN == 16 ? 3 : 2))
    linear_xs_kernel(const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_x, XsArgs p) {
  constexpr int MT = BN / 16;  // m-tiles (16 tokens)
  constexpr int KW = xs_warps(NTM);  // compute warps
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  const int NR = p.nr, KC = p.kc, S = p.stages, NCH = p.nch;
  const int NRO = SWIGLU ? NR / 2 : NR;  // outputs per CTA
  const int NT = NTC > 0 ? NTC : NR / 8;  // n-tiles
  const int RST = NR + 4;                // row stride of the reduction buffer
  constexpr uint32_t WROW = XsPlan<BN, KW, W8>::kWRow;
  const uint32_t wbytes = (uint32_t)NR * KC * WROW;  // weight bytes a stage receives
  const uint32_t xoff = XsPlan<BN, KW, W8>::wpart(NR, KC);  // x part of a stage
  const uint32_t xbytes = (uint32_t)BN * KC * 128;
  const uint32_t sbytes = xoff + xbytes;
  uint8_t* misc = smem + XsPlan<BN, KW, W8>::ring(NR, KC, S);
  uint64_t* full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* empty = full + kMaxStages;
  float* ssw = reinterpret_cast<float*>(misc + 128);  // [KW][BN] sums of squares (<= 2 KB)
  T* rsd = reinterpret_cast<T*>(misc + 4096);         // [BN][NRO] residual slice
  float* red = reinterpret_cast<float*>(smem);        // [KW][BN][RST], after the ring

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * NRO;  // first output (and weight row) of this CTA
  const int t0 = blockIdx.y * BN;     // first token of this CTA (token-split grids)
  const int nkb = (p.K + 63) / 64;
  const int mt = p.M - t0 < BN ? p.M - t0 : BN;

#ifdef TPP_DEBUG_STAMPS
  const unsigned long long clk0 = clock64();
#endif
  if (threadIdx.x == 0) {
    XS_TS(0);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], KW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == KW) {
    // ---------------- TMA / bulk producer ----------------
    if (lane != 0) return;
    bool ok = true;
    auto kbc = [&](int c) { return nkb - c * KC < KC ? nkb - c * KC : KC; };
    auto tx_bytes = [&](int c) {
      return (p.wpk ? (uint32_t)kbc(c) * NR * 128 : wbytes) +
             (p.xpk ? (uint32_t)kbc(c) * BN * 128 : xbytes);
    };
    auto load_w = [&](int c) {
      uint8_t* dst = smem + (c % S) * sbytes;
      if (W8) {
        tma_load_4d(dst, &tm_w, &full[c % S], 0, row0 % 32, c * KC, row0 / 32);
        if (SWIGLU) {
          const int u = p.N + row0;
          tma_load_4d(dst + (uint32_t)KC * NRO * 64, &tm_w, &full[c % S], 0, u % 32, c * KC,
                      u / 32);
        }
      } else if (p.wpk)
        bulk_load(dst, p.wpk + ((size_t)blockIdx.x * nkb + (size_t)c * KC) * NR * 128,
                  (uint32_t)kbc(c) * NR * 128, &full[c % S]);
      else if (SWIGLU)
        tma_load_4d(dst, &tm_w, &full[c % S], 0, row0, 0, c * KC);
      else
        tma_load_3d(dst, &tm_w, &full[c % S], 0, row0, c * KC);
    };
    auto load_x = [&](int c) {
      uint8_t* dst = smem + (c % S) * sbytes + xoff;
      if (p.xpk)
        bulk_load(dst, p.xpk + (size_t)c * KC * BN * 128, (uint32_t)kbc(c) * BN * 128,
                  &full[c % S]);
      else
        tma_load_3d(dst, &tm_x, &full[c % S], 0, t0, c * KC);
    };
    XS_TS(4);
    if (!p.wpk) prefetch_tmap(&tm_w);
    if (!p.xpk) prefetch_tmap(&tm_x);
    XS_TS(5);
    const int pre = NCH < S ? NCH : S;
    for (int c = 0; c < pre; ++c) {
      mbar_arrive_expect_tx(&full[c], tx_bytes(c));
      load_w(c);  // weights: independent of the previous kernel
    }
    XS_TS(12);
    pdl_wait();
    XS_TS(13);
    if (p.trigger_at == 0) pdl_trigger();
    for (int c = 0; c < pre; ++c) load_x(c);
    for (int c = pre; c < NCH && ok; ++c) {
      const int s = c % S;
      ok = mbar_wait(&empty[s], ((c / S) & 1) ^ 1, p.err, 21);
      if (!ok) break;
      mbar_arrive_expect_tx(&full[s], tx_bytes(c));
      load_w(c);
      load_x(c);
    }
    return;
  }

  // ---------------- compute warps ----------------
  pdl_wait();
  if (threadIdx.x == 0) XS_TS(1);
  const int tid = threadIdx.x;  // 0 .. 127
  if (p.residual && p.vec_ok) {
    const T* res = static_cast<const T*>(p.residual);
    const int chunks = NRO / 8;
    for (int e = tid; e < mt * chunks; e += KW * 32) {
      const int t = e / chunks, ch = e % chunks;
      const int n0 = row0 + ch * 8;
      if (n0 + 8 <= p.N)
        *reinterpret_cast<uint4*>(rsd + t * NRO + ch * 8) =
            *reinterpret_cast<const uint4*>(res + (int64_t)(t0 + t) * p.ldy + n0);
    }
  }
  float acc[MT][NTM][4];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int ni = 0; ni < NTM; ++ni)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[mi][ni][q] = 0.f;
  float ssl[MT][2] = {};
  bool ok = true;
  if constexpr (W8) {
    // fp8 weights: warp w takes whole k-blocks w, w + KW, ... of each chunk.
    // Within a k-block a weight row holds 64 bytes in the order the MMA
    // fragments want them: bytes 16c + 4s + (0..3) are the k indices
    // 16s + {2c, 2c+1, 2c+8, 2c+9} -- B fragment (b0, b1) of k16 step s for
    // the lane with c = lane % 4 -- so one 16-byte load per n-tile gives a
    // lane all four steps' fragments, dequantised once and used for every
    // token tile.
    uint32_t offa[4][MT];
#pragma unroll
    for (int st = 0; st < 4; ++st)
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        const int row = mi * 16 + (lane & 15);
        const int ch = st * 2 + (lane >> 4);
        offa[st][mi] = (uint32_t)(row * 128 + ((ch ^ (row & 7)) << 4));
      }
    const uint32_t offw = (uint32_t)((lane >> 2) * 64 + (lane & 3) * 16);
    // stage layout [half][k-block][NRO rows][64 B] (half: SwiGLU gate / up)
    const int hn = SWIGLU ? NT / 2 : NT;            // n-tiles per half
    const uint32_t xstride = BN * 128, wstride = (uint32_t)NRO * 64;
    const uint32_t hstride = (uint32_t)KC * NRO * 64;
    for (int c = 0; c < NCH && ok; ++c) {
      const int s = c % S;
      ok = mbar_wait(&full[s], (c / S) & 1, p.err, 22);
      if (!ok) break;
      const uint32_t ws = smem_u32(smem + s * sbytes);
      const uint32_t xs = ws + xoff;
      const int nj = nkb - c * KC < KC ? nkb - c * KC : KC;
      for (int j = warp; j < nj; j += KW) {
        const uint32_t xj = xs + j * xstride, wj = ws + j * wstride;
        uint32_t a[4][MT][4];
#pragma unroll
        for (int st = 0; st < 4; ++st)
#pragma unroll
          for (int mi = 0; mi < MT; ++mi) ldsm_x4(xj + offa[st][mi], a[st][mi]);
        if (NORM) {
#pragma unroll
          for (int st = 0; st < 4; ++st)
#pragma unroll
            for (int mi = 0; mi < MT; ++mi) {
              ssl[mi][0] += sq2<T>(a[st][mi][0]) + sq2<T>(a[st][mi][2]);
              ssl[mi][1] += sq2<T>(a[st][mi][1]) + sq2<T>(a[st][mi][3]);
            }
        }
#pragma unroll
        for (int ni = 0; ni < NTM; ++ni) {
          if (ni >= NT) break;
          const int hf = ni >= hn ? 1 : 0;
          const uint4 wv = lds128(wj + hf * hstride + (ni - hf * hn) * 8 * 64 + offw);
          const uint32_t wq[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int st = 0; st < 4; ++st) {
            const uint32_t b0 = e4m3x2_to<T>(wq[st] & 0xFFFFu);
            const uint32_t b1 = e4m3x2_to<T>(wq[st] >> 16);
#pragma unroll
            for (int mi = 0; mi < MT; ++mi) mma<T>(acc[mi][ni], a[st][mi], b0, b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  } else {
    // Warp w takes k16 step (w % 4) of every (KW / 4)-th k-block of each
    // chunk.
    constexpr int kJStep = KW / 4;  // k-block stride of one warp
    const int kk = warp & 3, jpar = warp >> 2;
    // Per-thread ldmatrix offsets inside a k-block tile (constant: this warp
    // always reads the same k16 step); 128-byte swizzle: 16-byte chunk q of
    // row r sits at position q ^ (r % 8).
    uint32_t offa[MT], offb[NTM / 2];
  #pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
      const int row = mi * 16 + (lane & 15);
      const int ch = kk * 2 + (lane >> 4);
      offa[mi] = (uint32_t)(row * 128 + ((ch ^ (row & 7)) << 4));
    }
  #pragma unroll
    for (int np = 0; np < NTM / 2; ++np) {
      // n-tiles 2np and 2np+1 (the second clamped to the first when NT is odd)
      const int nt = (2 * np + 1 < NT) ? 2 * np + ((lane >> 4) & 1) : 2 * np;
      const int n = nt * 8 + (lane & 7);
      const int ch = kk * 2 + ((lane >> 3) & 1);
      offb[np] = (uint32_t)(n * 128 + ((ch ^ (n & 7)) << 4));
    }
    const uint32_t xstride = BN * 128, wstride = (uint32_t)NR * 128;  // bytes per k-block tile
    auto load_frags = [&](uint32_t ws, uint32_t xs, int j, uint32_t (&a)[MT][4],
                          uint32_t (&b)[NTM / 2][4]) {
      const uint32_t xj = xs + j * xstride, wj = ws + j * wstride;
  #pragma unroll
      for (int mi = 0; mi < MT; ++mi) ldsm_x4(xj + offa[mi], a[mi]);
  #pragma unroll
      for (int np = 0; np < NTM / 2; ++np) {
        if (2 * np >= NT) break;
        ldsm_x4(wj + offb[np], b[np]);
      }
    };
    for (int c = 0; c < NCH && ok; ++c) {
      const int s = c % S;
      ok = mbar_wait(&full[s], (c / S) & 1, p.err, 22);
      if (!ok) break;
      if (threadIdx.x == 0 && c < 2) XS_TS(2 + c);
      if (threadIdx.x == 0 && c == 0 && p.trigger_at == 1) pdl_trigger();
      const uint32_t ws = smem_u32(smem + s * sbytes);
      const uint32_t xs = ws + xoff;
      const int nj = nkb - c * KC < KC ? nkb - c * KC : KC;
      auto mmas = [&](const uint32_t (&a)[MT][4], const uint32_t (&b)[NTM / 2][4]) {
  #pragma unroll
        for (int mi = 0; mi < MT; ++mi) {
          if (NORM) {
            ssl[mi][0] += sq2<T>(a[mi][0]) + sq2<T>(a[mi][2]);
            ssl[mi][1] += sq2<T>(a[mi][1]) + sq2<T>(a[mi][3]);
          }
  #pragma unroll
          for (int np = 0; np < NTM / 2; ++np) {
            if (2 * np >= NT) break;
            mma<T>(acc[mi][2 * np], a[mi], b[np][0], b[np][1]);
            if (2 * np + 1 < NT) mma<T>(acc[mi][2 * np + 1], a[mi], b[np][2], b[np][3]);
          }
        }
      };
      // A plain load-then-MMA loop: on B200 it schedules better than a
      // hand-written two-buffer pipeline (measured ~20% faster).
      for (int j = jpar; j < nj; j += kJStep) {
        uint32_t a0[MT][4], b0[NTM / 2][4];
        load_frags(ws, xs, j, a0, b0);
        mmas(a0, b0);
      }
      __syncwarp();
      if (threadIdx.x == 0 && c == 0) XS_TS(14);
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }

  // ---------------- cross-warp reduction ----------------
  if (threadIdx.x == 0) XS_TS(8);
  if (threadIdx.x == 0 && p.trigger_at == 2) pdl_trigger();
  asm volatile("bar.sync 1, %0;" ::"n"(KW * 32) : "memory");  // ring no longer read
  if (threadIdx.x == 0) XS_TS(9);
  {
    const int g = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
#pragma unroll
      for (int ni = 0; ni < NTM; ++ni) {
        if (ni >= NT) break;
        const int n = ni * 8 + cq * 2;
        float* r0 = red + (warp * BN + mi * 16 + g) * RST + n;
        float* r1 = r0 + 8 * RST;
        r0[0] = acc[mi][ni][0]; r0[1] = acc[mi][ni][1];
        r1[0] = acc[mi][ni][2]; r1[1] = acc[mi][ni][3];
      }
      if (NORM) {
        float lo = ssl[mi][0], hi = ssl[mi][1];
        lo += __shfl_xor_sync(0xffffffffu, lo, 1);
        lo += __shfl_xor_sync(0xffffffffu, lo, 2);
        hi += __shfl_xor_sync(0xffffffffu, hi, 1);
        hi += __shfl_xor_sync(0xffffffffu, hi, 2);
        if (cq == 0) {
          ssw[warp * BN + mi * 16 + g] = lo;
          ssw[warp * BN + mi * 16 + g + 8] = hi;
        }
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(KW * 32) : "memory");
  if (threadIdx.x == 0) XS_TS(10);

  // ---------------- epilogue ----------------
  const T* bias = static_cast<const T*>(p.bias);
  const T* res = static_cast<const T*>(p.residual);
  T* Y = static_cast<T*>(p.y);
  const int groups = NRO / 8;
  const float inv_k = 1.0f / (float)p.K;
  for (int e = tid; e < mt * groups; e += KW * 32) {
    const int t = e / groups, c0 = (e % groups) * 8;
    const int n0 = row0 + c0;
    if (n0 >= p.N) continue;
    float rs = 1.f;
    if (NORM) {
      float ss = 0.f;
#pragma unroll
      for (int w = 0; w < KW; ++w) ss += ssw[w * BN + t];
      rs = rsqrtf(ss * inv_k + p.eps);
    }
    if (threadIdx.x == 0) XS_TS(6);
    float g8[8], u8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { g8[i] = 0.f; u8[i] = 0.f; }
#pragma unroll
    for (int w = 0; w < KW; ++w) {
      const float* rr = red + (w * BN + t) * RST + c0;
      const float4 p0 = *reinterpret_cast<const float4*>(rr);
      const float4 p1 = *reinterpret_cast<const float4*>(rr + 4);
      g8[0] += p0.x; g8[1] += p0.y; g8[2] += p0.z; g8[3] += p0.w;
      g8[4] += p1.x; g8[5] += p1.y; g8[6] += p1.z; g8[7] += p1.w;
      if (SWIGLU) {
        const float4 q0 = *reinterpret_cast<const float4*>(rr + NRO);
        const float4 q1 = *reinterpret_cast<const float4*>(rr + NRO + 4);
        u8[0] += q0.x; u8[1] += q0.y; u8[2] += q0.z; u8[3] += q0.w;
        u8[4] += q1.x; u8[5] += q1.y; u8[6] += q1.z; u8[7] += q1.w;
      }
    }
    if (threadIdx.x == 0) XS_TS(7);
    if constexpr (W8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const bool in = n0 + i < p.N;
        g8[i] *= in ? p.wscale[n0 + i] : 0.f;
        if (SWIGLU) u8[i] *= in ? p.wscale[p.N + n0 + i] : 0.f;
      }
    }
    float o[8];
    const bool vec = p.vec_ok && n0 + 8 <= p.N;
    if (bias && vec) {
      float bg[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(bias + n0), bg);
#pragma unroll
      for (int i = 0; i < 8; ++i) g8[i] = g8[i] * rs + bg[i];
      if (SWIGLU) {
        unpack8<T>(*reinterpret_cast<const uint4*>(bias + p.N + n0), bg);
#pragma unroll
        for (int i = 0; i < 8; ++i) u8[i] = u8[i] * rs + bg[i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const bool in = bias && n0 + i < p.N;
        g8[i] = g8[i] * rs + (in ? to_f32(bias[n0 + i]) : 0.f);
        if (SWIGLU) u8[i] = u8[i] * rs + (in ? to_f32(bias[p.N + n0 + i]) : 0.f);
      }
    }
    if (SWIGLU) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = act_silu(g8[i]) * u8[i];
    } else if (p.act == TPP_ACT_SILU) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = act_silu(g8[i]);
    } else if (p.act == TPP_ACT_GELU) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = act_gelu_tanh(g8[i]);
    } else if (p.act == TPP_ACT_RELU) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = act_relu(g8[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = g8[i];
    }
    T* yr = Y + (int64_t)(t0 + t) * p.ldy;
    if (vec) {
      if (res) {
        float rf[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(rsd + t * NRO + c0), rf);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += rf[i];
      }
      const uint4 pk = pack8<T>(o);
      *reinterpret_cast<uint4*>(yr + n0) = pk;
      if (p.ypk)  // packed copy for the next decode linear: [kb][T][128 B], swizzled
        *reinterpret_cast<uint4*>(p.ypk + ((size_t)(n0 >> 6) * BN + t) * 128 +
                                  ((((n0 >> 3) & 7) ^ (t & 7)) << 4)) = pk;
    } else {
      const T* rr = res ? res + (int64_t)(t0 + t) * p.ldy : nullptr;
      for (int i = 0; i < 8 && n0 + i < p.N; ++i) {
        float v = o[i];
        if (rr) v += to_f32(rr[n0 + i]);
        yr[n0 + i] = from_f32<T>(v);
      }
    }
  }
  if (threadIdx.x == 0) XS_TS(11);
#ifdef TPP_DEBUG_STAMPS
  if (threadIdx.x == 0 && blockIdx.x < 256)
    g_xs_stamps[((p.dbg_id % 64) * 256 + blockIdx.x) * 16 + 15] = clock64() - clk0;
#endif
}

// ---------------------------------------------------------------------------
// Wide fp8 layers (the LM head, N >> 64 x SMs): a persistent form.  One CTA
// per SM keeps the whole x tile (BN tokens x K) in shared memory, loaded
// once, while the producer warp streams 32-row weight groups (all of K per
// group) through a ring.  Without this form every 32-row CTA of a many-wave
// grid reloads x, which costs more shared-memory traffic than the weights.
//  * x is converted once, in place, to fp16 with a per-token power-of-two
//    prescale (largest |x| below 2^14: exact, no overflow), so each pair of
//    e4m3 weights becomes an MMA operand with one cvt.rn.f16x2.e4m3x2; the
//    epilogue undoes the prescale.
//  * The twelve compute warps form three teams of four that take turns on
//    groups (the CTA's groups blockIdx.x, blockIdx.x + gridDim.x, ...): warp
//    w of a team multiplies k-blocks w, w + 4, ...; the team's partial sums
//    meet in its own shared-memory buffer; the epilogue (per-row scale,
//    norm factor, bias, activation, residual; scales and bias loaded when
//    the group starts) runs while the other teams multiply.
// ---------------------------------------------------------------------------
constexpr int kWideKW = 12;      // compute warps (three teams of four)
constexpr int kWideTW = 4;       // warps per team
constexpr int kWideNR = 32;      // weight rows per group
constexpr int kWideStages = 3;   // weight ring depth

template <int BN>
struct WidePlan {
  __host__ __device__ static size_t xbytes(int nkb) { return (size_t)BN * nkb * 128; }
  __host__ __device__ static size_t wstage(int nkb) { return (size_t)kWideNR * nkb * 64; }
  __host__ __device__ static size_t red() { return (size_t)kWideKW * BN * (kWideNR + 4) * 4; }
  static size_t smem(int nkb) {
    return 1024 + xbytes(nkb) + kWideStages * wstage(nkb) + red() + 1024;
  }
};

template <typename T, int BN, bool NORM>
__global__ void __launch_bounds__((kWideKW + 1) * 32, 1)
    linear_xs8_wide_kernel(const __grid_constant__ CUtensorMap tm_x, XsArgs p) {
  constexpr int MT = BN / 16, NT = kWideNR / 8, KW = kWideKW, TW = kWideTW, S = kWideStages;
  constexpr int RST = kWideNR + 4;
  constexpr int ITEMS = BN * (kWideNR / 8);  // epilogue items (8 outputs) per group
  static_assert(ITEMS <= TW * 32, "one epilogue item per team thread");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  const int nkb = p.K / 64;
  const uint32_t xbytes = (uint32_t)WidePlan<BN>::xbytes(nkb);
  const uint32_t wstage = (uint32_t)WidePlan<BN>::wstage(nkb);
  uint8_t* xsm = smem;
  uint8_t* ring = smem + xbytes;
  float* red = reinterpret_cast<float*>(ring + S * wstage);     // [KW][BN][RST]
  uint8_t* misc = reinterpret_cast<uint8_t*>(red + KW * BN * RST);
  uint64_t* full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* empty = full + S;
  uint64_t* xbar = empty + S;
  float* tokf = reinterpret_cast<float*>(misc + 128);           // [BN] per-token factor

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (p.N + kWideNR - 1) / kWideNR;
  const int mt = p.M < BN ? p.M : BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], TW);
    }
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == KW) {
    // ---------------- producer ----------------
    if (lane != 0) return;
    prefetch_tmap(&tm_x);
    int it = 0;
    int g = blockIdx.x;
    // weights of the first S groups: independent of the previous kernel.
    // A group is one contiguous block of the grouped fp8 layout.
    for (; g < groups && it < S; g += gridDim.x, ++it) {
      mbar_arrive_expect_tx(&full[it], wstage);
      bulk_load(ring + it * wstage, p.wpk + (size_t)g * wstage, wstage, &full[it]);
    }
    pdl_wait();
    pdl_trigger();
    mbar_arrive_expect_tx(xbar, xbytes);
    tma_load_3d(xsm, &tm_x, xbar, 0, 0, 0);
    for (; g < groups; g += gridDim.x, ++it) {
      const int s = it % S;
      if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, p.err, 21)) return;
      mbar_arrive_expect_tx(&full[s], wstage);
      bulk_load(ring + s * wstage, p.wpk + (size_t)g * wstage, wstage, &full[s]);
    }
    return;
  }

  // ---------------- compute warps ----------------
  pdl_wait();
  bool ok = mbar_wait(xbar, 0, p.err, 22);
  // x -> fp16 in place, token t scaled by 2^e(t); tokf[t] = 2^-e(t) (times
  // the RMSNorm factor for NORM)
  for (int t = warp; t < BN; t += KW) {
    float ss = 0.f, amax = 0.f;
    for (int ch = lane; ch < nkb * 8 && ok; ch += 32) {
      const int kb = ch >> 3, q = ch & 7;
      float f[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(xsm + (size_t)kb * BN * 128 + t * 128 +
                                                 ((q ^ (t & 7)) << 4)), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) { ss += f[i] * f[i]; amax = fmaxf(amax, fabsf(f[i])); }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    }
    int ex = 0;
    if (amax > 0.f) {
      frexpf(amax, &ex);          // amax < 2^ex
      ex = 14 - ex;               // amax * 2^ex < 2^14
      ex = ex > 100 ? 100 : (ex < -100 ? -100 : ex);
    }
    const float up = ldexpf(1.f, ex);
    for (int ch = lane; ch < nkb * 8 && ok; ch += 32) {
      const int kb = ch >> 3, q = ch & 7;
      uint4* ptr = reinterpret_cast<uint4*>(xsm + (size_t)kb * BN * 128 + t * 128 +
                                            ((q ^ (t & 7)) << 4));
      float f[8];
      unpack8<T>(*ptr, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] *= up;
      *ptr = pack8<__half>(f);
    }
    if (lane == 0)
      tokf[t] = ldexpf(1.f, -ex) * (NORM ? rsqrtf(ss / (float)p.K + p.eps) : 1.f);
  }
  asm volatile("bar.sync 8, %0;" ::"n"(KW * 32) : "memory");

  constexpr int TEAMS = KW / TW;
  const int team = warp / TW, wt = warp % TW, ttid = threadIdx.x % (TW * 32);
  uint32_t offa[4][MT];
#pragma unroll
  for (int st = 0; st < 4; ++st)
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
      const int row = mi * 16 + (lane & 15);
      const int ch = st * 2 + (lane >> 4);
      offa[st][mi] = (uint32_t)(row * 128 + ((ch ^ (row & 7)) << 4));
    }
  const uint32_t offw = (uint32_t)((lane >> 2) * 64 + (lane & 3) * 16);
  const uint32_t xs = smem_u32(xsm);
  float* tred = red + team * TW * BN * RST;   // this team's partials [TW][BN][RST]
  const T* bias = static_cast<const T*>(p.bias);
  const T* res = static_cast<const T*>(p.residual);
  T* Y = static_cast<T*>(p.y);
  // this thread's epilogue item of every group
  const bool has_item = ttid < ITEMS && ttid / (kWideNR / 8) < mt;
  const int et = ttid / (kWideNR / 8), ec0 = (ttid % (kWideNR / 8)) * 8;
  const float etf = has_item ? tokf[et] : 0.f;

  int it = team;
  for (int g = blockIdx.x + team * gridDim.x; g < groups; g += TEAMS * gridDim.x, it += TEAMS) {
    const int s = it % S;
    const int n0 = g * kWideNR + ec0;
    float sc[8], bs[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const bool in = has_item && n0 + i < p.N;
      sc[i] = in ? ldg_early_f32(p.wscale + n0 + i) : 0.f;
      if (in && bias) {
        const uint16_t h = ldg_early_u16(bias + n0 + i);
        bs[i] = to_f32(*reinterpret_cast<const T*>(&h));
      } else {
        bs[i] = 0.f;
      }
    }
    float acc[MT][NT][4];
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int ni = 0; ni < NT; ++ni)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[mi][ni][q] = 0.f;
    if (ok) ok = mbar_wait(&full[s], (it / S) & 1, p.err, 22);
    if (ok) {
      const uint32_t ws = smem_u32(ring + s * wstage);
      for (int j = wt; j < nkb; j += TW) {
        const uint32_t xj = xs + j * BN * 128, wj = ws + j * kWideNR * 64;
        uint32_t a[4][MT][4];
#pragma unroll
        for (int st = 0; st < 4; ++st)
#pragma unroll
          for (int mi = 0; mi < MT; ++mi) ldsm_x4(xj + offa[st][mi], a[st][mi]);
#pragma unroll
        for (int ni = 0; ni < NT; ++ni) {
          const uint4 wv = lds128(wj + ni * 8 * 64 + offw);
          const uint32_t wq[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int st = 0; st < 4; ++st) {
            const uint32_t b0 = e4m3x2_to<__half>(wq[st] & 0xFFFFu);
            const uint32_t b1 = e4m3x2_to<__half>(wq[st] >> 16);
#pragma unroll
            for (int mi = 0; mi < MT; ++mi) mma<__half>(acc[mi][ni], a[st][mi], b0, b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // the team's previous epilogue has finished reading its partials
    asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "n"(TW * 32) : "memory");
    {
      const int gq = lane >> 2, cq = lane & 3;
#pragma unroll
      for (int mi = 0; mi < MT; ++mi)
#pragma unroll
        for (int ni = 0; ni < NT; ++ni) {
          float* r0 = tred + (wt * BN + mi * 16 + gq) * RST + ni * 8 + cq * 2;
          *reinterpret_cast<float2*>(r0) = make_float2(acc[mi][ni][0], acc[mi][ni][1]);
          *reinterpret_cast<float2*>(r0 + 8 * RST) = make_float2(acc[mi][ni][2], acc[mi][ni][3]);
        }
    }
    asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "n"(TW * 32) : "memory");
    if (!ok || !has_item || n0 >= p.N) continue;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.f;
#pragma unroll
    for (int w = 0; w < TW; ++w) {
      const float* rr = tred + (w * BN + et) * RST + ec0;
      const float4 p0 = *reinterpret_cast<const float4*>(rr);
      const float4 p1 = *reinterpret_cast<const float4*>(rr + 4);
      o[0] += p0.x; o[1] += p0.y; o[2] += p0.z; o[3] += p0.w;
      o[4] += p1.x; o[5] += p1.y; o[6] += p1.z; o[7] += p1.w;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = apply_act(p.act, o[i] * sc[i] * etf + bs[i]);
    T* yr = Y + (int64_t)et * p.ldy;
    const T* rr = res ? res + (int64_t)et * p.ldy : nullptr;
    if (p.vec_ok && n0 + 8 <= p.N) {
      if (rr) {
        float rf[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(rr + n0), rf);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += rf[i];
      }
      *reinterpret_cast<uint4*>(yr + n0) = pack8<T>(o);
    } else {
      for (int i = 0; i < 8 && n0 + i < p.N; ++i) {
        float v = o[i];
        if (rr) v += to_f32(rr[n0 + i]);
        yr[n0 + i] = from_f32<T>(v);
      }
    }
  }
}

template <typename T, int BN, bool NORM>
int launch_xs8_wide(const void* x, int64_t ldx, const void* q, XsArgs& a, cudaStream_t st) {
  const int nkb = a.K / 64;
  CUtensorMap tx;
  a.wpk = static_cast<const uint8_t*>(q);  // grouped fp8 weight (bulk copies)
  {
    const int dtype = IsBf16<T>::value ? TPP_BF16 : TPP_F16;
    const uint64_t dims[3] = {64, (uint64_t)a.M, (uint64_t)nkb};
    const uint64_t strides[2] = {(uint64_t)ldx * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)BN, (uint32_t)nkb};
    const int rc = make_tmap(&tx, x, dtype, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  }
  auto kern = linear_xs8_wide_kernel<T, BN, NORM>;
  const size_t smem = WidePlan<BN>::smem(nkb);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess) {
    set_error("linear_xs8_wide_kernel: cannot reserve shared memory");
    return TPP_ERR_LAUNCH;
  }
  const int groups = (a.N + kWideNR - 1) / kWideNR;
  const int grid = groups < sm_budget() ? groups : sm_budget();
  return launch("linear_xs8_wide_kernel", kern, dim3((unsigned)grid), dim3((kWideKW + 1) * 32),
                smem, st, 1u, tx, a);
}

// Launch geometry chosen on the host (plan_xs).
struct XsLaunch {
  int nro;     // outputs per CTA
  int bn;      // token tile (16 or 32)
  int tsplit;  // token tiles (grid y)
  int kc, nch, stages;
};

template <typename T, int BN, int NTM, bool SW, bool NORM, bool W8, int NTC = 0>
int launch_xs(const void* x, int64_t ldx, const void* w, XsArgs& a, int dtype, cudaStream_t st,
              const XsLaunch& L) {
  using Plan = XsPlan<BN, xs_warps(NTM), W8>;
  const int nro = L.nro, tsplit = L.tsplit, kc = L.kc, nch = L.nch, stages = L.stages;
  const int nr = SW ? 2 * nro : nro;
  const int nkb = (a.K + 63) / 64;
  a.nr = nr; a.kc = kc; a.nch = nch; a.stages = stages;
#ifdef TPP_DEBUG_STAMPS
  a.dbg_id = g_xs_launch++;
#endif

  CUtensorMap tw, tx;
  if (W8) {
    // fp8 W in 32-row groups [G][k-block][32][64 B] (fp8_weight_offset) as
    // {byte, row in group, k-block, group}; a box is nro rows of one group
    // (nro divides 32), no swizzle (the kernel's 16-byte row reads are
    // conflict-free as laid out).  SwiGLU: one box for the gate rows, one
    // for the up rows.
    const int rows = SW ? 2 * a.N : a.N;
    const uint64_t dims[4] = {64, 32, (uint64_t)nkb, (uint64_t)((rows + 31) / 32)};
    const uint64_t strides[3] = {64, 2048, (uint64_t)nkb * 2048};
    const uint32_t box[4] = {64, (uint32_t)nro, (uint32_t)kc, 1};
    const int rc = make_tmap(&tw, w, kTmapU8, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TPP_OK) return rc;
  } else if (a.wpk) {
    // unused by the kernel (bulk copies), but a valid map keeps the launch uniform
    const uint64_t dims[2] = {64, 8};
    const uint64_t strides[1] = {128};
    const uint32_t box[2] = {64, 8};
    const int rc = make_tmap(&tw, a.wpk, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  } else if (SW) {
    // W [2N][K] as {k in block, row, half, k-block}
    const uint64_t dims[4] = {64, (uint64_t)a.N, 2, (uint64_t)nkb};
    const uint64_t strides[3] = {(uint64_t)a.K * 2, (uint64_t)a.N * a.K * 2, 128};
    const uint32_t box[4] = {64, (uint32_t)nro, 2, (uint32_t)kc};
    const int rc = make_tmap(&tw, w, dtype, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  } else {
    const uint64_t dims[3] = {64, (uint64_t)a.N, (uint64_t)nkb};
    const uint64_t strides[2] = {(uint64_t)a.K * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)nr, (uint32_t)kc};
    const int rc = make_tmap(&tw, w, dtype, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  }
  if (a.xpk) {
    const uint64_t dims[2] = {64, 8};
    const uint64_t strides[1] = {128};
    const uint32_t box[2] = {64, 8};
    const int rc = make_tmap(&tx, a.xpk, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  } else {
    const uint64_t dims[3] = {64, (uint64_t)a.M, (uint64_t)nkb};
    const uint64_t strides[2] = {(uint64_t)ldx * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)BN, (uint32_t)kc};
    const int rc = make_tmap(&tx, x, dtype, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  }
  const int ctas = (a.N + nro - 1) / nro;
  auto kern = linear_xs_kernel<T, BN, NTM, SW, NORM, W8, NTC>;
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kBudget1) != cudaSuccess) {
      set_error("linear_xs_kernel: cannot reserve shared memory");
      return TPP_ERR_LAUNCH;
    }
    configured |= bit;
  }
  return launch("linear_xs_kernel", kern, dim3((unsigned)ctas, (unsigned)tsplit), dim3(xs_threads(NTM)),
                Plan::smem(nr, nro, kc, stages), st, 1u, tw, tx, a);
}

// Persistent wide fp8 form on unless TPP_XS8_WIDE=0 (A/B measurements).
bool wide_enabled() {
  static const bool on = [] {
    const char* e = getenv("TPP_XS8_WIDE");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Where dependents are released (TPP_XS_TRIGGER_AT, A/B measurements).
int xs_trigger_at() {
  static const int v = [] {
    const char* e = getenv("TPP_XS_TRIGGER_AT");
    return e ? atoi(e) : 0;
  }();
  return v;
}

// Token split on unless TPP_XS_TSPLIT=0 (A/B measurements).
bool tsplit_enabled() {
  static const bool on = [] {
    const char* e = getenv("TPP_XS_TSPLIT");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Shared memory of a plan (XsPlan<BN>::smem with a runtime token tile).
size_t xs_smem(int bn, int nr, int nro, int kc, int stages, bool w8 = false) {
  const int ntm = nr <= 16 ? 2 : (nr <= 32 ? 4 : 8);
  const size_t wpart = ((size_t)nr * (w8 ? 64 : 128) * kc + 1023) & ~(size_t)1023;
  const size_t ring = (size_t)stages * (wpart + (size_t)bn * 128 * kc);
  const size_t red = (size_t)xs_warps(ntm) * bn * (nr + 4) * 4;
  return 1024 + (ring > red ? ring : red) + 4096 + (((size_t)bn * nro * 2 + 15) & ~(size_t)15);
}

// Chunking for a given slice: one chunk (one request per operand, one memory
// round trip) when the CTA's whole weight slice and x fit `limit`; else
// chunks of up to 8 k-blocks (x part <= 32 KB) in a ring of >= 2 stages.
bool xs_chunks(int bn, int nr, int nro, int nkb, size_t limit, size_t ring_limit, XsLaunch& L,
               bool w8 = false) {
  if (nkb <= 256 && xs_smem(bn, nr, nro, nkb, 1, w8) <= limit) {
    L.kc = nkb; L.nch = 1; L.stages = 1;
    return true;
  }
  int kc = nkb < 8 ? nkb : 8;
  while (kc > 1 && (bn * kc * 128 > 32768 || xs_smem(bn, nr, nro, kc, 2, w8) > ring_limit)) --kc;
  if (xs_smem(bn, nr, nro, kc, nkb > kc ? 2 : 1, w8) > ring_limit) return false;
  L.kc = kc;
  L.nch = (nkb + kc - 1) / kc;
  L.stages = L.nch < kMaxStages ? L.nch : kMaxStages;
  while (L.stages > 1 && xs_smem(bn, nr, nro, kc, L.stages, w8) > ring_limit) --L.stages;
  return true;
}

// Host plan for the unpacked path: among slice widths of 8..64 weight rows
// (token-split into 16-token tiles where the register tile allows), keep
// those whose grid fits one wave (two CTAs per SM within 110 KB of shared
// memory, or one per SM within 227 KB) and take a single-chunk plan with
// the fewest operand bytes per CTA; otherwise the multi-chunk fallback.
bool plan_xs(int64_t M, int64_t N, int64_t K, int act, XsLaunch& out, bool w8 = false) {
  const int sms = sm_budget();
  const int per_row = act == TPP_ACT_SWIGLU ? 2 : 1;
  const int nkb = (int)(K / 64);
  size_t best = ~(size_t)0;
  for (int nro = 8; nro * per_row <= 8 * kMaxNT; nro += 8) {
    const int nr = nro * per_row;
    // fp8 slices are boxes inside one 32-row group (and, for SwiGLU, the up
    // rows start on a slice boundary)
    if (w8 && (32 % nro != 0 || (per_row == 2 && N % nro != 0))) continue;
    const int ntm = nr <= 16 ? 2 : (nr <= 32 ? 4 : 8);
    const int tsplit = (M > 16 && ntm <= 4 && tsplit_enabled()) ? (int)((M + 15) / 16) : 1;
    const int bn = (M <= 16 || tsplit > 1) ? 16 : 32;
    const int64_t grid = (N + nro - 1) / nro * tsplit;
    if (grid > 2 * (int64_t)sms) continue;
    const size_t limit = grid <= sms ? kBudget1 : kBudget;
    if (nkb > 256 || xs_smem(bn, nr, nro, nkb, 1, w8) > limit) continue;
    const size_t bytes = ((size_t)nr * (w8 ? 64 : 128) + bn * 128) * nkb;
    if (bytes < best) {
      best = bytes;
      out.nro = nro; out.bn = bn; out.tsplit = tsplit;
      out.kc = nkb; out.nch = 1; out.stages = 1;
    }
  }
  if (best != ~(size_t)0) return true;
  if (w8) {
    // wide fp8 layers (the LM head): several waves of narrow slices, two or
    // three CTAs per SM, so one CTA's weights stream while another computes
    int nro = 32 / per_row;
    while (per_row == 2 && nro >= 8 && N % nro != 0) nro /= 2;
    if (nro < 8) return false;
    const int rows = nro * per_row;
    out.nro = nro;
    out.tsplit = 1;
    out.bn = M <= 16 ? 16 : 32;
    return xs_chunks(out.bn, rows, out.nro, nkb, kBudget, kBudget, out, true);
  }
  const int nro = xs_outputs_per_cta(N, act);
  if (nro == 0) return false;
  const int nr = nro * per_row;
  const int ntm = nr <= 16 ? 2 : (nr <= 32 ? 4 : 8);
  if (ntm > 4) return false;  // wide slices: the weight-streaming kernel does better
  out.nro = nro;
  out.tsplit = (M > 16 && tsplit_enabled()) ? (int)((M + 15) / 16) : 1;
  out.bn = (M <= 16 || out.tsplit > 1) ? 16 : 32;
  const int64_t grid = (N + nro - 1) / nro * out.tsplit;
  return xs_chunks(out.bn, nr, nro, nkb, grid <= 2 * (int64_t)sms ? kBudget : 0,
                   out.tsplit > 1 ? kBudget16 : kBudget, out);
}

// Packed operands: the slice width is fixed by the packed weight image
// (xs_outputs_per_cta) and the token tile by the packed activation.
bool plan_packed(int64_t M, int64_t N, int64_t K, int act, XsLaunch& out) {
  const int nro = xs_outputs_per_cta(N, act);
  if (nro == 0) return false;
  const int nr = act == TPP_ACT_SWIGLU ? 2 * nro : nro;
  out.nro = nro;
  out.tsplit = 1;
  out.bn = xs_token_tile(M);
  const int64_t grid = (N + nro - 1) / nro;
  return xs_chunks(out.bn, nr, nro, (int)(K / 64), grid <= 2 * (int64_t)num_sms() ? kBudget : 0,
                   kBudget, out);
}

template <typename T, int NTM, bool NORM, bool W8, int NTC = 0>
int xs_dispatch_nt(const void* x, int64_t ldx, const void* w, XsArgs& a, int dtype,
                   cudaStream_t st, const XsLaunch& L) {
  const bool sw = a.act == TPP_ACT_SWIGLU;
  if (L.bn == 16)
    return sw ? launch_xs<T, 16, NTM, true, NORM, W8, NTC>(x, ldx, w, a, dtype, st, L)
              : launch_xs<T, 16, NTM, false, NORM, W8, NTC>(x, ldx, w, a, dtype, st, L);
  return sw ? launch_xs<T, 32, NTM, true, NORM, W8, NTC>(x, ldx, w, a, dtype, st, L)
            : launch_xs<T, 32, NTM, false, NORM, W8, NTC>(x, ldx, w, a, dtype, st, L);
}

// The exact n-tile count as a template constant (see linear_xs_kernel).
template <typename T, int NTM, bool NORM, bool W8>
int xs_dispatch_exact(const void* x, int64_t ldx, const void* w, XsArgs& a, int dtype,
                      cudaStream_t st, const XsLaunch& L, int nt) {
  {
    if constexpr (NTM == 2) {
      return nt == 1 ? xs_dispatch_nt<T, 2, NORM, W8, 1>(x, ldx, w, a, dtype, st, L)
                     : xs_dispatch_nt<T, 2, NORM, W8, 2>(x, ldx, w, a, dtype, st, L);
    } else if constexpr (NTM == 4) {
      return nt == 3 ? xs_dispatch_nt<T, 4, NORM, W8, 3>(x, ldx, w, a, dtype, st, L)
                     : xs_dispatch_nt<T, 4, NORM, W8, 4>(x, ldx, w, a, dtype, st, L);
    } else {
      switch (nt) {
        case 5: return xs_dispatch_nt<T, 8, NORM, W8, 5>(x, ldx, w, a, dtype, st, L);
        case 6: return xs_dispatch_nt<T, 8, NORM, W8, 6>(x, ldx, w, a, dtype, st, L);
        case 7: return xs_dispatch_nt<T, 8, NORM, W8, 7>(x, ldx, w, a, dtype, st, L);
        default: return xs_dispatch_nt<T, 8, NORM, W8, 8>(x, ldx, w, a, dtype, st, L);
      }
    }
  }
}

template <typename T, bool NORM, bool W8 = false>
int xs_dispatch(const void* x, int64_t ldx, const void* w, XsArgs& a, int dtype, cudaStream_t st,
                const XsLaunch& L) {
  const int nt = (a.act == TPP_ACT_SWIGLU ? 2 * L.nro : L.nro) / 8;
  if (nt <= 2) return xs_dispatch_exact<T, 2, NORM, W8>(x, ldx, w, a, dtype, st, L, nt);
  if (nt <= 4) return xs_dispatch_exact<T, 4, NORM, W8>(x, ldx, w, a, dtype, st, L, nt);
  return xs_dispatch_exact<T, 8, NORM, W8>(x, ldx, w, a, dtype, st, L, nt);
}

}  // namespace


// Decode linear in x-stationary form.  Returns -1 (nothing launched) when the
// shape is better served by the weight-streaming kernel (very wide N, or a
// slice that does not fit the shared-memory budget); otherwise a TPP status.
#ifdef TPP_DEBUG_STAMPS
extern "C" void tpp_debug_xs_stamps(unsigned long long* host) {
  cudaMemcpyFromSymbol(host, g_xs_stamps, sizeof(unsigned long long) * 64 * 256 * 16);
}
extern "C" unsigned tpp_debug_xs_launches() { return g_xs_launch; }
#endif

// Outputs per CTA (SwiGLU CTAs hold that many gate rows plus as many up
// rows) for an N-wide layer on this device, or 0 when N is too wide.
int xs_outputs_per_cta(int64_t N, int act) {
  const int sms = num_sms();  // fixed per device: packed weight images depend on it
  const int per_row = act == TPP_ACT_SWIGLU ? 2 : 1;  // weight rows per output
  int64_t nro = (N + sms - 1) / sms;
  nro = (nro + 7) / 8 * 8;
  // Prefer slices of <= 32 weight rows (4 n-tiles: two CTAs fit an SM) as
  // long as the grid still fits two CTAs per SM.
  const int64_t small = 32 / per_row;
  if (nro * per_row > 32 && (N + small - 1) / small <= 2 * (int64_t)sms) nro = small;
#ifdef TPP_DEBUG_STAMPS
  if (const char* e = getenv("TPP_XS_ROWS")) {  // tuning experiments only
    const int64_t f = atoi(e) / per_row;
    if (f >= 8 && f % 8 == 0) nro = f;
  }
#endif
  return nro * per_row > 8 * kMaxNT ? 0 : (int)nro;
}
int xs_token_tile(int64_t M) { return M <= 16 ? 16 : 32; }

int linear_xs_impl(const void* x, int64_t ldx, const void* w, const void* bias,
                   const void* residual, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                   int act, int dtype, cudaStream_t st, float norm_eps, const void* wpk,
                   const void* xpk, void* ypk) {
  // The 3-D views address k-block kb of a row at +128 * kb bytes: rows must
  // be whole k-blocks, or the last one would run into the next row.
  if (K % 64 != 0 || M > 32) return -1;
  XsLaunch L;
  const bool packed = wpk || xpk || ypk;
  if (!(packed ? plan_packed(M, N, K, act, L) : plan_xs(M, N, K, act, L))) return -1;
  XsArgs a;
  a.bias = bias; a.residual = residual; a.y = y; a.ldy = ldy;
  a.M = (int)M; a.N = (int)N; a.K = (int)K; a.act = act;
  a.vec_ok = (N % 8 == 0) && (ldy % 8 == 0) && aligned16(y) &&
             (!residual || aligned16(residual)) && (!bias || aligned16(bias));
  a.eps = norm_eps;
  a.err = device_error_flag();
  a.wpk = static_cast<const uint8_t*>(wpk);
  a.xpk = static_cast<const uint8_t*>(xpk);
  a.ypk = static_cast<uint8_t*>(ypk);
  a.wscale = nullptr;
  a.trigger_at = xs_trigger_at();
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return norm_eps >= 0.f ? xs_dispatch<T, true>(x, ldx, w, a, dtype, st, L)
                           : xs_dispatch<T, false>(x, ldx, w, a, dtype, st, L);
  });
}

}  // namespace tpp

namespace tpp {

int linear_xs(const void* x, int64_t ldx, const void* w, const void* bias, const void* residual,
              void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act, int dtype,
              cudaStream_t st, float norm_eps) {
  return linear_xs_impl(x, ldx, w, bias, residual, y, ldy, M, N, K, act, dtype, st, norm_eps,
                        nullptr, nullptr, nullptr);
}

// Decode linear on fp8 (e4m3) weights with per-row scales: y = act(eps-norm
// * scale[n] * (x . Q[n]) + bias) + residual.  Q in the kernel's k order
// (quantize_fp8_kernel).  Returns -1 (nothing launched) without a plan.
int linear_xs_fp8(const void* x, int64_t ldx, const void* q, const float* scale,
                  const void* bias, const void* residual, void* y, int64_t ldy, int64_t M,
                  int64_t N, int64_t K, int act, int dtype, cudaStream_t st, float norm_eps) {
  if (K % 64 != 0 || M > 32) return -1;
  XsLaunch L;
  XsLaunch one_wave;
  // wide layers that no one-wave slice plan covers: the persistent form when
  // x and a 3-deep weight ring fit one CTA's shared memory
  const int bnw = M <= 16 ? 16 : 32;
  const bool wide = !plan_xs(M, N, K, act, one_wave, false) && act != TPP_ACT_SWIGLU &&
                    (bnw == 16 ? WidePlan<16>::smem((int)(K / 64))
                               : WidePlan<32>::smem((int)(K / 64))) <= kBudget1 &&
                    wide_enabled();
  if (!wide && !plan_xs(M, N, K, act, L, true)) return -1;
  XsArgs a;
  a.bias = bias; a.residual = residual; a.y = y; a.ldy = ldy;
  a.M = (int)M; a.N = (int)N; a.K = (int)K; a.act = act;
  a.vec_ok = (N % 8 == 0) && (ldy % 8 == 0) && aligned16(y) &&
             (!residual || aligned16(residual)) && (!bias || aligned16(bias));
  a.eps = norm_eps;
  a.err = device_error_flag();
  a.wpk = nullptr; a.xpk = nullptr; a.ypk = nullptr;
  a.wscale = scale;
  a.trigger_at = xs_trigger_at();
  if (wide)
    return TPP_DISPATCH_HALF(dtype, T, [&] {
      if (bnw == 16)
        return norm_eps >= 0.f ? launch_xs8_wide<T, 16, true>(x, ldx, q, a, st)
                               : launch_xs8_wide<T, 16, false>(x, ldx, q, a, st);
      return norm_eps >= 0.f ? launch_xs8_wide<T, 32, true>(x, ldx, q, a, st)
                             : launch_xs8_wide<T, 32, false>(x, ldx, q, a, st);
    });
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return norm_eps >= 0.f ? xs_dispatch<T, true, true>(x, ldx, q, a, dtype, st, L)
                           : xs_dispatch<T, false, true>(x, ldx, q, a, dtype, st, L);
  });
}

namespace {
// Logical k index held by byte `pos` (0..63) of a k-block in the fp8 weight
// layout: bytes 16c + 4s + j hold k = 16s + {2c, 2c+1, 2c+8, 2c+9}[j].
__host__ __device__ __forceinline__ int fp8_k_of(int pos) {
  const int c = pos >> 4, s = (pos >> 2) & 3, j = pos & 3;
  return 16 * s + 2 * c + (j & 1) + (j >> 1) * 8;
}
// Byte offset of (row, k-block) in the grouped fp8 layout
// [row / 32][k-block][row % 32][64 B]: a 32-row group is contiguous.
__host__ __device__ __forceinline__ int64_t fp8_row_block(int64_t row, int kb, int nkb) {
  return ((row >> 5) * nkb + kb) * 2048 + (row & 31) * 64;
}

// One CTA per weight row: scale = amax / 448 (1 for an all-zero row), bytes
// = e4m3(w / scale) with round-to-nearest-even and saturation, in the
// kernel's k order.
template <typename T>
__global__ void __launch_bounds__(256) quantize_fp8_kernel(const T* __restrict__ w, int64_t rows,
                                                           int K, uint8_t* __restrict__ q,
                                                           float* __restrict__ scale) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  const int nkb = K / 64;
  if (blockIdx.x >= rows) {  // padding rows of the last group: zero bytes
    for (int grp = threadIdx.x; grp < K / 16; grp += 256)
      *reinterpret_cast<uint4*>(q + fp8_row_block(blockIdx.x, grp >> 2, nkb) + (grp & 3) * 16) =
          make_uint4(0, 0, 0, 0);
    return;
  }
  const T* wr = w + (int64_t)blockIdx.x * K;
  float amax = 0.f;
  for (int i = threadIdx.x * 8; i < K; i += 256 * 8) {
    float f[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(wr + i), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, red[i]);
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  if (threadIdx.x == 0) scale[blockIdx.x] = sc;
  for (int grp = threadIdx.x; grp < K / 16; grp += 256) {
    const int kb = grp >> 2;
    uint32_t v[4];
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
      v[wd] = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pos = (grp & 3) * 16 + wd * 4 + j;
        const float x = to_f32(wr[kb * 64 + fp8_k_of(pos)]) / sc;
        const uint32_t b = (uint32_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
        v[wd] |= b << (8 * j);
      }
    }
    *reinterpret_cast<uint4*>(q + fp8_row_block(blockIdx.x, kb, nkb) + (grp & 3) * 16) =
        make_uint4(v[0], v[1], v[2], v[3]);
  }
}

// Inverse: w[n, k] = T(e4m3 value * scale[n]) in natural k order.
template <typename T>
__global__ void __launch_bounds__(256) dequantize_fp8_kernel(const uint8_t* __restrict__ q,
                                                             const float* __restrict__ scale,
                                                             int K, int64_t total,
                                                             T* __restrict__ w) {
  pdl_wait();
  pdl_trigger();
  const int nkb = K / 64;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / K;
    const int kk = (int)(i % K);  // stored position within the row
    const int k = (kk & ~63) + fp8_k_of(kk & 63);
    const uint8_t b = q[fp8_row_block(row, kk >> 6, nkb) + (kk & 63)];
    const __half h = __nv_cvt_fp8_to_halfraw(b, __NV_E4M3);
    w[row * K + k] = from_f32<T>(__half2float(h) * scale[row]);
  }
}
}  // namespace

int quantize_weight_fp8(const void* w, int64_t rows, int64_t K, int dtype, void* q, float* scale,
                        cudaStream_t st) {
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return launch("quantize_fp8_kernel", quantize_fp8_kernel<T>,
                  dim3((unsigned)((rows + 31) / 32 * 32)), dim3(256), 0, st, 0u,
                  static_cast<const T*>(w), rows, (int)K, static_cast<uint8_t*>(q), scale);
  });
}

int dequantize_weight_fp8(const void* q, const float* scale, int64_t rows, int64_t K, int dtype,
                          void* w, cudaStream_t st) {
  const int64_t total = rows * K;
  const int blocks = (int)((total + 255) / 256 < 8192 ? (total + 255) / 256 : 8192);
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return launch("dequantize_fp8_kernel", dequantize_fp8_kernel<T>, dim3(blocks), dim3(256), 0,
                  st, 0u, static_cast<const uint8_t*>(q), scale, (int)K, total,
                  static_cast<T*>(w));
  });
}

namespace {
// W [N or 2N][K] -> per-CTA images [cta][kb][NR][128 B]; 16-byte chunk j of
// image row rr is stored at position j ^ (rr % 8) (128-byte swizzle).  Rows
// past N are zero.
__global__ void pack_weight_kernel(const uint8_t* __restrict__ w, int N, int K, int nro, int nr,
                                   int swiglu, int64_t total, uint8_t* __restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  const int nkb = K / 64;
  for (int64_t id = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; id < total;
       id += (int64_t)gridDim.x * blockDim.x) {
    const int pos = (int)(id & 7);
    const int64_t q = id >> 3;
    const int rr = (int)(q % nr);
    const int64_t q2 = q / nr;
    const int kb = (int)(q2 % nkb);
    const int64_t cta = q2 / nkb;
    const int j = pos ^ (rr & 7);
    int64_t grow;
    bool valid;
    if (swiglu) {
      const int g = nr / 2;
      const int64_t r = cta * g + rr % g;
      valid = r < N;
      grow = (rr / g) * (int64_t)N + r;
    } else {
      grow = cta * nro + rr;
      valid = grow < N;
    }
    uint4 v = make_uint4(0, 0, 0, 0);
    if (valid) v = *reinterpret_cast<const uint4*>(w + (grow * K + kb * 64 + j * 8) * 2);
    *reinterpret_cast<uint4*>(dst + id * 16) = v;
  }
}
// x [M][K] -> [kb][BN][128 B], swizzled like the weights; rows >= M are zero.
__global__ void pack_activation_kernel(const uint8_t* __restrict__ x, int64_t ldx, int M, int K,
                                       int bn, int64_t total, uint8_t* __restrict__ dst) {
  pdl_wait();
  pdl_trigger();
  for (int64_t id = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; id < total;
       id += (int64_t)gridDim.x * blockDim.x) {
    const int pos = (int)(id & 7);
    const int t = (int)((id >> 3) % bn);
    const int kb = (int)((id >> 3) / bn);
    const int j = pos ^ (t & 7);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < M) v = *reinterpret_cast<const uint4*>(x + (t * ldx + kb * 64 + j * 8) * 2);
    *reinterpret_cast<uint4*>(dst + id * 16) = v;
  }
}
}  // namespace

int64_t xs_packed_weight_bytes(int64_t N, int64_t K, int act) {
  if (K % 64 != 0) return 0;
  const int nro = xs_outputs_per_cta(N, act);
  if (nro == 0) return 0;
  const int64_t nr = act == TPP_ACT_SWIGLU ? 2 * nro : nro;
  return (N + nro - 1) / nro * (K / 64) * nr * 128;
}
int64_t xs_packed_activation_bytes(int64_t M, int64_t K) {
  return K % 64 != 0 ? 0 : (K / 64) * xs_token_tile(M) * 128;
}
int xs_pack_weight(const void* w, int64_t N, int64_t K, int act, void* dst, cudaStream_t st) {
  const int nro = xs_outputs_per_cta(N, act);
  const int nr = act == TPP_ACT_SWIGLU ? 2 * nro : nro;
  const int64_t total = xs_packed_weight_bytes(N, K, act) / 16;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  return launch("pack_weight_kernel", pack_weight_kernel, dim3(blocks), dim3(256), 0, st, 1u,
                static_cast<const uint8_t*>(w), (int)N, (int)K, nro, nr,
                act == TPP_ACT_SWIGLU ? 1 : 0, total, static_cast<uint8_t*>(dst));
}
int xs_pack_activation(const void* x, int64_t ldx, int64_t M, int64_t K, void* dst,
                       cudaStream_t st) {
  const int64_t total = xs_packed_activation_bytes(M, K) / 16;
  const int blocks = (int)((total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024);
  return launch("pack_activation_kernel", pack_activation_kernel, dim3(blocks), dim3(256), 0,
                st, 1u, static_cast<const uint8_t*>(x), ldx, (int)M, (int)K, xs_token_tile(M),
                total, static_cast<uint8_t*>(dst));
}

}  // namespace tpp
