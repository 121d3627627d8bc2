// Decode attention on tensor cores: one query token per sequence, the G query
// heads of a KV group stacked as the rows of m16n8k16 MMA tiles, K/V streamed
// by TMA through a shared-memory ring, split-KV partials merged inside a
// thread-block cluster over distributed shared memory.
//
// Semantics as decode_attn_kernel (attn_decode.cu): keys [p - window_left, p]
// of a BHSD cache, p = seqlen - 1; query head h reads kv head h / G (the
// repeat_interleave of torchpp/attention/gqa.py:120-121, not materialised).
//
// Design (HBM-bound on the cache):
//  * grid (split, kv_head x head_pass, batch), cluster (splits, 1, 1) when
//    there are at most 8 splits.  A CTA streams one slice of one kv head's
//    key range once for all (up to 16) query heads of the group.
//  * Thread 0 issues 4-D TMA loads (128-byte swizzle, per-CTA loads) of
//    64-key K and V tiles into a kStages ring (full/empty mbarriers, bounded
//    waits).  Each of the 4 warps takes 16 keys of every tile:
//    S = Q.K^T (D/16 x 2 MMAs), fp32 online softmax in the exp2 domain,
//    O += P.V (D/8 MMAs); fragments come from ldmatrix on the swizzled tiles.
//  * The 4 warps merge in shared memory; the splits then merge at cluster
//    rank 0 (peers push (o, lse) with 16-byte remote stores), or -- beyond 8
//    splits -- write (o, lse) partials to the caller's workspace for
//    decode_combine_kernel.
#include <math.h>
#include <type_traits>
#include <cooperative_groups.h>
#include "mma_common.cuh"
#include "tc_common.cuh"
#include "attn_decode.cuh"

namespace cg = cooperative_groups;

namespace tpp {



namespace {

#ifdef TPP_DEBUG_STAMPS
// [launch % 32][cta < 512][16] globaltimer stamps (thread 0)
__device__ unsigned long long g_dec_stamps[32 * 512 * 16];
unsigned g_dec_launch = 0;
#define DEC_TS(i) do { const unsigned _c = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z); \
    if (threadIdx.x == 0 && _c < 512) { unsigned long long _t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(_t)); \
    g_dec_stamps[((p.dbg_id % 32) * 512 + _c) * 16 + (i)] = _t; } } while (0)
#else
#define DEC_TS(i) do {} while (0)
#endif

constexpr int kThreads = 128;
constexpr int KT = 64;      // keys per tile
constexpr int kStages = 3;
constexpr int QR = 16;      // query-head rows per CTA (MMA M)

// Address of 16-byte chunk `chunk` of row r in a TMA 128B-swizzled tile made of
// 64-element-wide boxes stacked along the row (box b holds chunks 8b..8b+7).
__device__ __forceinline__ uint32_t sw_addr(uint32_t base, int box_rows, int r, int chunk) {
  return base + (uint32_t)((chunk >> 3) * box_rows * 128 + r * 128 + (((chunk & 7) ^ (r & 7)) << 4));
}

template <int D>
struct DecSmem {
  static constexpr uint32_t kTile = KT * D * 2;                 // one K or V tile
  static constexpr uint32_t kRing = kStages * 2 * kTile;
  static constexpr uint32_t kWc = 4 * QR * (D + 4) * 4;         // per-warp (m, l, -, -, o)
  static constexpr uint32_t kRecv = 8 * QR * (D + 4) * 4;       // per-split (o, lse)
  static constexpr uint32_t kWork = (kRing > kWc + kRecv) ? kRing : (kWc + kRecv);
  static constexpr uint32_t kQ = QR * D * 2;
  // + barriers (64 B), then the fused mode's new k and v rows (fp32) and the
  // new key's score per query row
  static constexpr uint32_t kNew = 2 * D * 4 + QR * 4;
  static constexpr size_t kBytes = 1024 + kWork + kQ + 64 + kNew;
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) decode_mma_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
    DecMmaArgs p) {
  using SM = DecSmem<D>;
  constexpr int NCH = D / 8;  // 16-byte chunks per row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* ring = smem;
  uint8_t* sq = smem + SM::kWork;
  uint64_t* full = reinterpret_cast<uint64_t*>(sq + SM::kQ);
  uint64_t* empty = full + kStages;
  float* knew = reinterpret_cast<float*>(sq + SM::kQ + 64);   // fused mode: new k row
  float* vnew = knew + D;                                     //             new v row
  float* snew = vnew + D;                                     //             q.k_new per row
  float* wc = reinterpret_cast<float*>(smem);                 // after the loop
  float* recv = reinterpret_cast<float*>(smem + SM::kWc);     // after the loop

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.passes;
  const int pass = blockIdx.y % p.passes;
  const int b = blockIdx.z;
  const int h0 = kvh * p.G + pass * QR;
  const int nh = min(QR, p.G - pass * QR);
  DEC_TS(0);

  if (tid == 0) {
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // Unfused mode: q and this step's cache row come from the previous kernel.
  // Fused mode: the streamed keys exclude this step's row, and the lengths
  // and earlier rows were written by kernels of earlier steps, which had
  // completed before this one could start (every kernel of the library calls
  // launch_dependents only after its own wait) -- so the K/V stream starts
  // before the wait, under the QKV projection's tail; only the raw qkv row
  // waits for it.
  const bool fused = p.qkv != nullptr;
  if (!fused) {
    pdl_wait();
    pdl_trigger();
  }

  const int64_t L = p.seqlens ? (int64_t)p.seqlens[b] : p.max_seqlen;
  int64_t lo = 0;
  if (p.window_left >= 0) lo = max((int64_t)0, L - 1 - p.window_left);
  // Paged caches: a tile is one 64-key block, so the split ranges start on a
  // block boundary and keys below lo are masked.
  const bool paged = p.table != nullptr;
  const int64_t lo_t = paged ? lo / KT * KT : lo;
  const int64_t n = L > lo_t ? L - lo_t : 0;
  int64_t per = (n + p.splits - 1) / p.splits;
  per = (per + KT - 1) / KT * KT;
  const int64_t k0 = lo_t + (int64_t)split * per;
  const int64_t k1c = min(L, k0 + per);
  // Fused mode: the CTA whose key range holds the new token's position takes
  // that key from registers (normalised, rotated) rather than from the cache
  // row it writes, so it streams only the keys before it.
  const int64_t pos = fused ? (int64_t)p.positions[b] : 0;
  const bool has_new = fused && pos >= k0 && pos < k1c;
  const int64_t k1 = has_new ? pos : k1c;
  const int ntiles = k1 > k0 ? (int)((k1 - k0 + KT - 1) / KT) : 0;

  auto issue = [&](int i) {
    const int s = i % kStages;
    uint8_t* kd = ring + s * 2 * SM::kTile;
    uint8_t* vd = kd + SM::kTile;
    const int64_t key = k0 + (int64_t)i * KT;
    mbar_arrive_expect_tx(&full[s], 2 * SM::kTile);
    // one request per operand: the D/64 column boxes of the tile come from a
    // 5-D view {64, key, D/64, kv head, batch} (paged: {64, row in block,
    // D/64, kv head, block})
    if (paged) {
      const int blk = p.table[b * p.tbl_stride + key / KT];
      tma_load_5d(kd, &tm_k, &full[s], 0, 0, 0, kvh, blk);
      tma_load_5d(vd, &tm_v, &full[s], 0, 0, 0, kvh, blk);
    } else {
      tma_load_5d(kd, &tm_k, &full[s], 0, (int)key, 0, kvh, b);
      tma_load_5d(vd, &tm_v, &full[s], 0, (int)key, 0, kvh, b);
    }
  };
  if (tid == 0) {
    for (int i = 0; i < ntiles && i < kStages; ++i) issue(i);
  }
  // fused mode: the static RoPE tables and norm weights load before the wait
  constexpr int EPL = D / 32;
  float cv[EPL], sv[EPL], wq[EPL], wk[EPL];
  if (fused) {
    const __half* cs = static_cast<const __half*>(p.cosp) + pos * p.cs_stride + lane * EPL;
    const __half* sn = static_cast<const __half*>(p.sinp) + pos * p.cs_stride + lane * EPL;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      cv[j] = __half2float(cs[j]);
      sv[j] = __half2float(sn[j]);
      wq[j] = p.qn_w ? to_f32(static_cast<const T*>(p.qn_w)[lane * EPL + j]) : 1.f;
      wk[j] = p.kn_w ? to_f32(static_cast<const T*>(p.kn_w)[lane * EPL + j]) : 1.f;
    }
    pdl_wait();
    pdl_trigger();
  }
  DEC_TS(1);

  // ---- Q rows (heads h0 .. h0+nh-1, zero padding) -> swizzled smem -> A fragments ----
  const uint32_t sq_a = smem_u32(sq);
  if (fused) {
    // q/k RMSNorm + RoPE as qk_norm_rope_cache_kernel (rope.cu) computes them:
    // fp32 math on the raw projection, one rounding to T at the end.  Each
    // warp owns 4 q rows plus the new k row (every warp recomputes it, so the
    // dot products need no block barrier); lane l holds elements
    // [EPL*l, EPL*l + EPL), its rotate-half partner is lane l ^ 16.  All rows
    // go through each phase together (one load round trip, interleaved
    // shuffles).
    constexpr int RPW = QR / 4;  // q rows per warp
    constexpr int NRW = RPW + 1;  // + the new k row
    using VT = typename std::conditional<EPL == 4, uint2, uint32_t>::type;
    const T* row = static_cast<const T*>(p.qkv) + b * p.qkv_sb;
    VT raw[NRW], rawv = VT{};
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int r = warp + 4 * i;
      raw[i] = r < nh ? *reinterpret_cast<const VT*>(row + (int64_t)(h0 + r) * D + lane * EPL)
                      : VT{};
    }
    raw[RPW] = has_new ? *reinterpret_cast<const VT*>(row + (int64_t)(p.Hq + kvh) * D + lane * EPL)
                       : VT{};
    if (has_new && warp == 0)
      rawv = *reinterpret_cast<const VT*>(row + (int64_t)(p.Hq + p.Hkv + kvh) * D + lane * EPL);
    float x[NRW][EPL];
#pragma unroll
    for (int i = 0; i < NRW; ++i) {
      const T* e = reinterpret_cast<const T*>(&raw[i]);
#pragma unroll
      for (int j = 0; j < EPL; ++j) x[i][j] = to_f32(e[j]);
    }
    // RMSNorm (rows without a weight are left as they are)
    float ss[NRW];
#pragma unroll
    for (int i = 0; i < NRW; ++i) {
      ss[i] = 0.f;
#pragma unroll
      for (int j = 0; j < EPL; ++j) ss[i] += x[i][j] * x[i][j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < NRW; ++i) ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], o);
#pragma unroll
    for (int i = 0; i < NRW; ++i) {
      const bool has_w = i < RPW ? p.qn_w != nullptr : p.kn_w != nullptr;
      if (!has_w) continue;
      const float inv = rsqrtf(ss[i] / (float)D + p.eps);
      const float* w = i < RPW ? wq : wk;
#pragma unroll
      for (int j = 0; j < EPL; ++j) x[i][j] *= inv * w[j];
    }
    // RoPE (rotate-half partner in lane ^ 16), then the one rounding to T
    float pr[NRW][EPL];
#pragma unroll
    for (int j = 0; j < EPL; ++j)
#pragma unroll
      for (int i = 0; i < NRW; ++i) pr[i][j] = __shfl_xor_sync(0xffffffffu, x[i][j], 16);
#pragma unroll
    for (int i = 0; i < NRW; ++i)
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const float v = lane < 16 ? x[i][j] * cv[j] - pr[i][j] * sv[j]
                                  : x[i][j] * cv[j] + pr[i][j] * sv[j];
        x[i][j] = to_f32(from_f32<T>(v));
      }
    // q rows -> swizzled smem; q . k_new per row
    float dot[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int r = warp + 4 * i;
      VT packed;
      T* pe = reinterpret_cast<T*>(&packed);
      dot[i] = 0.f;
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const float v = r < nh ? x[i][j] : 0.f;
        pe[j] = from_f32<T>(v);
        dot[i] += v * x[RPW][j];
      }
      *reinterpret_cast<VT*>(sq + (sw_addr(sq_a, QR, r, (lane * EPL) >> 3) - sq_a) +
                             ((lane * EPL) & 7) * 2) = packed;
    }
    if (has_new) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < RPW; ++i) dot[i] += __shfl_xor_sync(0xffffffffu, dot[i], o);
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
          const int r = warp + 4 * i;
          snew[r] = r < nh ? dot[i] * p.scale_log2 : -INFINITY;
        }
      }
      if (warp == 0) {
        // the step's cache rows (k normed + rotated, v as projected) and the
        // v row the fold below reads
        VT pk, pv;
        T* ek = reinterpret_cast<T*>(&pk);
        T* ev = reinterpret_cast<T*>(&pv);
        const T* rv = reinterpret_cast<const T*>(&rawv);
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
          ek[j] = from_f32<T>(x[RPW][j]);
          ev[j] = rv[j];
          vnew[lane * EPL + j] = to_f32(rv[j]);
        }
        if (pass == 0) {
          const int64_t off =
              (paged ? ((int64_t)p.table[b * p.tbl_stride + pos / KT] * p.Hkv + kvh) * (KT * D) +
                           (pos % KT) * D
                     : b * p.c_sb + kvh * p.c_sh + pos * p.c_ss) +
              lane * EPL;
          *reinterpret_cast<VT*>(static_cast<T*>(p.kc) + off) = pk;
          *reinterpret_cast<VT*>(static_cast<T*>(p.vc) + off) = pv;
        }
      }
    }
  } else {
    const T* Q = static_cast<const T*>(p.q) + b * p.q_sb;
    for (int e = tid; e < QR * NCH; e += kThreads) {
      const int r = e / NCH, ch = e % NCH;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < nh) v = __ldg(reinterpret_cast<const uint4*>(Q + (int64_t)(h0 + r) * p.q_sh) + ch);
      *reinterpret_cast<uint4*>(sq + (sw_addr(sq_a, QR, r, ch) - sq_a)) = v;
    }
  }
  __syncthreads();
  DEC_TS(2);
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
    ldsm_x4(sw_addr(sq_a, QR, r, ks * 2 + (lane >> 4)), qf[ks]);
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  bool ok = true;

  const int kr0 = warp * 16;  // this warp's 16 keys of every tile
  // S = Q.K^T for this warp's 16 keys of tile i; even and odd k-steps
  // accumulate in separate registers (4 independent MMA chains instead of 2)
  auto compute_s = [&](int i, float (&sc)[2][4]) {
    const uint32_t kb = smem_u32(ring + (i % kStages) * 2 * SM::kTile);
    float sd[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[j][e] = sd[j][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t bf[4];
      const int r = kr0 + (lane & 7) + (lane >> 4) * 8;
      ldsm_x4(sw_addr(kb, KT, r, ks * 2 + ((lane >> 3) & 1)), bf);
      float (&acc)[2][4] = (ks & 1) ? sd : sc;
      mma<T>(acc[0], qf[ks], bf[0], bf[1]);
      mma<T>(acc[1], qf[ks], bf[2], bf[3]);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[j][e] += sd[j][e];
  };
  // Software pipeline: the S MMAs of tile i+1 are issued before the PV MMAs
  // of tile i (they are independent), so the two latency chains overlap.
  float sc[2][4];
  if (ntiles > 0) {
    if (mbar_wait(&full[0], 0, p.err, 22)) compute_s(0, sc);
    else ok = false;
  }
  for (int i = 0; i < ntiles && ok; ++i) {
    const int s = i % kStages;
    // refill the stage released one iteration ago
    if (tid == 0 && i >= 1 && i - 1 + kStages < ntiles) {
      const int sp = (i - 1) % kStages;
      ok = mbar_wait(&empty[sp], ((i - 1) / kStages) & 1, p.err, 21) && ok;
      if (ok) issue(i - 1 + kStages);
    }
    if (i < 10) DEC_TS(3 + i);
    const uint32_t vb = smem_u32(ring + s * 2 * SM::kTile) + SM::kTile;
    const int64_t kbase = k0 + (int64_t)i * KT + kr0;
    if (kbase >= lo && kbase + 16 <= k1) {  // this warp's 16 keys all in range
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[j][e] *= p.scale_log2;
    } else {
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t key = kbase + j * 8 + 2 * c + (e & 1);
          sc[j][e] = (key < k1 && key >= lo) ? sc[j][e] * p.scale_log2 : -INFINITY;
        }
    }
    // Lazy rescale: the exponent base m_r moves (and o, l are rescaled) only
    // when a row's maximum grows by more than 2^8 (log2 units); otherwise the
    // probabilities are taken against the old base (at most 2^8 in fp32).
    float corr[2];
    bool grow = false;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = fmaxf(fmaxf(sc[0][2 * hr], sc[0][2 * hr + 1]),
                       fmaxf(sc[1][2 * hr], sc[1][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      corr[hr] = 1.f;
      if (mx > m_r[hr] + 8.f) {
        corr[hr] = ex2_ftz(m_r[hr] - mx);  // 0 when no key was seen yet
        m_r[hr] = mx;
        grow = true;
      }
      mx = m_r[hr];
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = sc[j][2 * hr + e];
          const float pv = (v == -INFINITY) ? 0.f : ex2_ftz(v - mx);
          sc[j][2 * hr + e] = pv;
          sum += pv;
        }
      l_r[hr] = l_r[hr] * corr[hr] + sum;
    }
    if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
      for (int d = 0; d < D / 8; ++d) {
        o[d][0] *= corr[0]; o[d][1] *= corr[0];
        o[d][2] *= corr[1]; o[d][3] *= corr[1];
      }
    }
    uint32_t pa[4];
    pa[0] = pack2<T>(sc[0][0], sc[0][1]);
    pa[1] = pack2<T>(sc[0][2], sc[0][3]);
    pa[2] = pack2<T>(sc[1][0], sc[1][1]);
    pa[3] = pack2<T>(sc[1][2], sc[1][3]);
    const bool more = i + 1 < ntiles;
    if (more) {
      if (mbar_wait(&full[(i + 1) % kStages], ((i + 1) / kStages) & 1, p.err, 22))
        compute_s(i + 1, sc);  // sc is free again: P went to registers above
      else
        ok = false;
    }
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t bf[4];
      const int r = kr0 + (lane & 7) + ((lane >> 3) & 1) * 8;
      ldsm_x4_t(sw_addr(vb, KT, r, dp * 2 + (lane >> 4)), bf);
      mma<T>(o[2 * dp], pa, bf[0], bf[1]);
      mma<T>(o[2 * dp + 1], pa, bf[2], bf[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  DEC_TS(13);
  // ---- fused mode: fold the new key into warp 0's online-softmax state ----
  if (has_new && warp == 0) {
    __syncwarp();
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const float sk = snew[g + hr * 8];
      if (sk == -INFINITY) continue;  // padding row
      const float mx = fmaxf(m_r[hr], sk);
      const float corr = ex2_ftz(m_r[hr] - mx);  // 0 when no key was seen yet
      const float pn = ex2_ftz(sk - mx);
      l_r[hr] = l_r[hr] * corr + (c == 0 ? pn : 0.f);  // l is summed over the quad
#pragma unroll
      for (int d = 0; d < D / 8; ++d) {
        o[d][2 * hr] = o[d][2 * hr] * corr + pn * vnew[d * 8 + 2 * c];
        o[d][2 * hr + 1] = o[d][2 * hr + 1] * corr + pn * vnew[d * 8 + 2 * c + 1];
      }
      m_r[hr] = mx;
    }
  }

  // ---- merge the 4 warps (rows g, g+8 of each; l is quad-partial) ----
  if (p.cluster && p.splits > 1)
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  __syncthreads();  // every warp is done with the ring
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = l_r[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int r = g + hr * 8;
    float* base = wc + (warp * QR + r) * (D + 4);
    if (c == 0) { base[0] = m_r[hr]; base[1] = l; }
#pragma unroll
    for (int d = 0; d < D / 8; ++d)
      *reinterpret_cast<float2*>(base + 4 + d * 8 + 2 * c) = make_float2(o[d][2 * hr], o[d][2 * hr + 1]);
  }
  __syncthreads();
  if (p.splits == 1) {
    // One split: each thread finishes 8 consecutive outputs of a row straight
    // from the four warps' partials (weights exp2(m_w - M) / L recomputed per
    // item) and stores them with one 16-byte write.
    DEC_TS(14);
    T* out = static_cast<T*>(p.o) + b * p.o_sb;
    const bool vec = ((reinterpret_cast<uintptr_t>(p.o) & 15) == 0) && (p.o_sh % 8 == 0) &&
                     (p.o_sb % 8 == 0);
    for (int e = tid; e < nh * (D / 8); e += kThreads) {
      const int r = e / (D / 8), d0 = (e % (D / 8)) * 8;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) M = fmaxf(M, wc[(w * QR + r) * (D + 4)]);
      float ew[4], Ls = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float* bw = wc + (w * QR + r) * (D + 4);
        ew[w] = (M == -INFINITY || bw[0] == -INFINITY) ? 0.f : exp2f(bw[0] - M);
        Ls += bw[1] * ew[w];
      }
      const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
      float acc[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float* ow = wc + (w * QR + r) * (D + 4) + 4 + d0;
        const float4 a0 = *reinterpret_cast<const float4*>(ow);
        const float4 a1 = *reinterpret_cast<const float4*>(ow + 4);
        const float f = ew[w] * inv;
        acc[0] += a0.x * f; acc[1] += a0.y * f; acc[2] += a0.z * f; acc[3] += a0.w * f;
        acc[4] += a1.x * f; acc[5] += a1.y * f; acc[6] += a1.z * f; acc[7] += a1.w * f;
      }
      T* dst = out + (int64_t)(h0 + r) * p.o_sh + d0;
      if (vec) {
        *reinterpret_cast<uint4*>(dst) = pack8<T>(acc);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = from_f32<T>(acc[q]);
      }
    }
    DEC_TS(15);
    return;
  }
  // CTA partial for row r: normalised o (fp32) and lse (log2 domain) in the
  // receive slot of this split (cluster mode: slots 0..7 = cluster ranks;
  // otherwise slot 0)
  const int slot = (p.cluster && p.splits > 1) ? split : 0;
  // per row: the weight of each warp's partial (exp2(m_w - M) / L) and lse,
  // computed once (into the spent new-key area), then applied per element
  float* fac = knew;           // [QR][4]
  float* rlse = knew + 4 * QR; // [QR]
  if (tid < nh) {
    const int r = tid;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wc[(w * QR + r) * (D + 4)]);
    float e[4], Ls = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* bw = wc + (w * QR + r) * (D + 4);
      e[w] = (M == -INFINITY || bw[0] == -INFINITY) ? 0.f : exp2f(bw[0] - M);
      Ls += bw[1] * e[w];
    }
    const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) fac[r * 4 + w] = e[w] * inv;
    rlse[r] = Ls > 0.f ? M + log2f(Ls) : -INFINITY;
  }
  __syncthreads();
  for (int e = tid; e < nh * D; e += kThreads) {
    const int r = e / D, d = e % D;
    float on = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) on += wc[(w * QR + r) * (D + 4) + 4 + d] * fac[r * 4 + w];
    recv[(slot * QR + r) * (D + 4) + 4 + d] = on;
    if (d == 0) recv[(slot * QR + r) * (D + 4)] = rlse[r];
  }
  __syncthreads();


  if (!p.cluster) {
    for (int e = tid; e < nh * D; e += kThreads) {
      const int r = e / D, d = e % D;
      const int64_t wslot = ((int64_t)b * p.Hq + h0 + r) * p.splits + split;
      p.ws_o[wslot * D + d] = recv[r * (D + 4) + 4 + d];
      if (d == 0) p.ws_lse[wslot] = recv[r * (D + 4)];
    }
    return;
  }
  // ---- cluster merge at rank 0 ----
  cg::cluster_group cluster = cg::this_cluster();
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (split != 0) {
    const uint32_t base = smem_u32(recv) + (uint32_t)((split * QR) * (D + 4) * 4);
    uint32_t rbase;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbase) : "r"(base), "r"(0));
    for (int e = tid; e < nh * (D + 4) / 4; e += kThreads) {
      const float4 v = *reinterpret_cast<const float4*>(recv + (split * QR) * (D + 4) + e * 4);
      asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(rbase + 16 * e),
                   "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                   : "memory");
    }
  }
  cluster.sync();
  if (split != 0) return;
  T* out = static_cast<T*>(p.o) + b * p.o_sb;
  for (int e = tid; e < nh * D; e += kThreads) {
    const int r = e / D, d = e % D;
    float M = -INFINITY;
    for (int sp = 0; sp < p.splits; ++sp) M = fmaxf(M, recv[(sp * QR + r) * (D + 4)]);
    float W = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int sp = 0; sp < p.splits; ++sp) {
        const float* bs = recv + (sp * QR + r) * (D + 4);
        const float w = bs[0] == -INFINITY ? 0.f : exp2f(bs[0] - M);
        W += w;
        O += w * bs[4 + d];
      }
    }
    out[(int64_t)(h0 + r) * p.o_sh + d] = from_f32<T>(W > 0.f ? O / W : 0.f);
  }
  (void)ok;
}

}  // namespace

// Split count of the tensor-core decode path: as many splits as keep the
// grid within one wave of resident CTAs (two per SM) -- a partial second wave
// costs a whole extra CTA lifetime.
int decode_mma_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t range) {
  const int64_t G = Hq / Hkv;
  const int64_t ctas = B * Hkv * ((G + QR - 1) / QR);
  int64_t s = (2LL * sm_budget()) / (ctas > 0 ? ctas : 1);
  int64_t maxs = (range + KT - 1) / KT;
  if (maxs < 1) maxs = 1;
  if (s > maxs) s = maxs;
  if (s > 64) s = 64;
  return (int)(s < 1 ? 1 : s);
}

#ifdef TPP_DEBUG_STAMPS
extern "C" void tpp_debug_dec_stamps(unsigned long long* host) {
  cudaMemcpyFromSymbol(host, g_dec_stamps, sizeof(unsigned long long) * 32 * 512 * 16);
}
extern "C" unsigned tpp_debug_dec_launches() { return g_dec_launch; }
#endif

int decode_mma_launch(DecMmaArgs& a, const void* k_cache, const void* v_cache, int64_t c_sb,
                      int64_t c_sh, int64_t c_ss, int64_t B, int64_t D, int dtype,
                      cudaStream_t st) {
#ifdef TPP_DEBUG_STAMPS
  a.dbg_id = g_dec_launch++;
#endif
  CUtensorMap tk, tv;
  const uint64_t smax = (uint64_t)(a.max_seqlen > 0 ? a.max_seqlen : 1);
  // {64 columns, key, column box (D/64), kv head, batch}: the tile's column
  // boxes land one after another ([box][key][128 B]), as the kernel reads
  // them.  Paged pools [block][Hkv][64][D]: {64, row, D/64, kv head, block}.
  const bool paged = a.table != nullptr;
  const uint64_t dims[5] = {64, paged ? (uint64_t)KT : smax, (uint64_t)(D / 64), (uint64_t)a.Hkv,
                            paged ? (uint64_t)a.num_blocks : (uint64_t)B};
  const uint64_t strides[4] = {
      (uint64_t)D * 2, 128, paged ? (uint64_t)KT * D * 2 : (uint64_t)c_sh * 2,
      paged ? (uint64_t)a.Hkv * KT * D * 2 : (uint64_t)c_sb * 2};
  const uint32_t box[5] = {64, KT, (uint32_t)(D / 64), 1, 1};
  int rc = make_tmap(&tk, k_cache, dtype, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != TPP_OK) return rc;
  rc = make_tmap(&tv, v_cache, dtype, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != TPP_OK) return rc;
  a.passes = (a.G + QR - 1) / QR;
  a.cluster = a.splits <= 8 ? 1 : 0;
  const dim3 grid((unsigned)a.splits, (unsigned)(a.Hkv * a.passes), (unsigned)B);
  auto go = [&](auto kern, size_t smem) -> int {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
      set_error("decode_mma_kernel: cannot reserve shared memory");
      return TPP_ERR_LAUNCH;
    }
    return launch("decode_mma_kernel", kern, grid, dim3(kThreads), smem, st,
                  0u, tk, tv, a);
  };
  // the cluster spans the split dimension (x); launch() clusters along y, so
  // build the launch here when needed
  if (a.cluster && a.splits > 1) {
    auto launch_x = [&](auto kern, size_t smem) -> int {
      // (set on every call: one cache per lambda would be shared by the
      // fp16 and bf16 kernels, whose pointers have the same type)
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess) {
        set_error("decode_mma_kernel: cannot reserve shared memory");
        return TPP_ERR_LAUNCH;
      }
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = grid;
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[2];
      unsigned na = 0;
      if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
      }
      attr[na].id = cudaLaunchAttributeClusterDimension;
      attr[na].val.clusterDim.x = (unsigned)a.splits;
      attr[na].val.clusterDim.y = 1;
      attr[na].val.clusterDim.z = 1;
      ++na;
      cfg.attrs = attr;
      cfg.numAttrs = na;
      const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tk, tv, a);
      if (e != cudaSuccess) {
        set_error(std::string("decode_mma_kernel: ") + cudaGetErrorString(e));
        return TPP_ERR_LAUNCH;
      }
      return check_launch("decode_mma_kernel");
    };
    return TPP_DISPATCH_HALF(dtype, T, [&] {
      return D == 64 ? launch_x(decode_mma_kernel<T, 64>, DecSmem<64>::kBytes)
                     : launch_x(decode_mma_kernel<T, 128>, DecSmem<128>::kBytes);
    });
  }
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return D == 64 ? go(decode_mma_kernel<T, 64>, DecSmem<64>::kBytes)
                   : go(decode_mma_kernel<T, 128>, DecSmem<128>::kBytes);
  });
}

}  // namespace tpp
