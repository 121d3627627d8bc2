// Flash attention forward on the 5th-generation tensor cores (head dim 128).
//
// Same semantics as prefill_attn_kernel (attn_prefill.cu): flash_attn_func
// (q, k, v, causal, window_size=(w-1, 0)) as torchpp calls it
// (torchpp/attention/gqa.py:128, swa.py:85-89), GQA by head mapping instead
// of the repeat_interleave of gqa.py:120-121, bottom-right causal alignment.
//
// One CTA = one (batch, query head, 128-query block).  384 threads:
//   warp 0 / lane 0 : TMA producer: Q once, then K and V tiles of 128 keys
//                     into separate rings (3 K, 2 V stages; 128-byte swizzle,
//                     per-CTA loads), K running ahead of V.
//   warp 1 / lane 0 : MMA issuer:  S_j = Q . K_j^T   (tcgen05, M=N=128, K=128)
//                                  O  += P_j . V_j   (A = P_j read from TMEM,
//                                                     B = V_j MN-major in smem)
//   warps 4..11     : softmax, two warpgroups, one query row per lane (TMEM
//                     lane) and one half of the keys per warpgroup: row max
//                     (exchanged once per tile through shared memory) and sum
//                     without shuffles, P_j written back to TMEM as
//                     bf16/fp16 over S_j, O rescaled in TMEM only when the
//                     running max grows by more than 2^8 (otherwise the stale
//                     max stays the reference: exact, since the final
//                     normalisation uses the same reference).
// TMEM: O in columns [0,128), S/P in three buffers [128,256), [256,384),
// [384,512), so S_{j+1}, S_{j+2} are computed while the softmax of tile j
// runs and P.V_j never has to finish before the next S is issued.  The output is
// normalised, staged in shared memory (the Q buffer) and written by TMA.
#include <math.h>
#include "tc_common.cuh"
#include "mma_common.cuh"

namespace tpp {

struct TcAttnArgs {
  int Sq, Sk, Hq, Hkv;
  int causal;
  int64_t window_left;
  float scale_log2;
  int* err;
};

namespace {

#ifdef TPP_DEBUG_STAMPS
__device__ unsigned long long g_fa_stamps[4 * 64];
__device__ __forceinline__ void fa_ts(int kind, int j) {
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && j < 64) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_fa_stamps[kind * 64 + j] = t;
  }
}
#define FA_TS(k, j) fa_ts(k, j)
#else
#define FA_TS(k, j)
#endif

constexpr int D = 128;
constexpr int BQ = 128;   // queries per CTA
constexpr int BKV = 128;  // keys per tile
constexpr int kKSt = 3;       // K tiles in flight (freed when S_j completes)
constexpr int kVSt = 2;       // V tiles in flight (freed when P.V_j completes)
constexpr int kSP = 3;        // S/P buffers in TMEM
constexpr int kThreads = 384;  // 4 control warps + 8 softmax warps
constexpr int kSoftWarp0 = 4;
constexpr uint32_t kQBytes = BQ * D * 2;     // 32 KB (2 boxes of [128][64])
constexpr uint32_t kTile = BKV * D * 2;      // 32 KB per K or V tile
constexpr size_t kSmem = 1024 + kQBytes + (kKSt + kVSt) * kTile + 256 + 6 * BQ * 4;
constexpr float kRescaleThreshold = 8.0f;    // log2 units

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v,
                           const __grid_constant__ CUtensorMap tm_o, TcAttnArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kQBytes;            // kKSt K tiles
  uint8_t* sV = sK + kKSt * kTile;          // kVSt V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kVSt * kTile);
  uint64_t* q_full = bars;                  // 1
  uint64_t* k_full = bars + 1;              // kKSt
  uint64_t* k_empty = k_full + kKSt;        // kKSt
  uint64_t* v_full = k_empty + kKSt;        // kVSt
  uint64_t* v_empty = v_full + kVSt;        // kVSt
  uint64_t* s_full = v_empty + kVSt;        // kSP: S_j in TMEM buffer j % kSP
  uint64_t* p_full = s_full + kSP;         // kSP: P_j written (8 softmax warps)
  uint64_t* pv_done = p_full + kSP;        // kSP: P.V_j complete (buffer j % kSP free)
  uint64_t* o_final = pv_done + kSP;       // 1 (after the last P.V)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);
  float* xmax = reinterpret_cast<float*>(bars + 32);  // [2 parity][2 half][BQ] row maxima, then sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heavy (late, causal) query blocks first
  const int nqb = gridDim.x;
  const int qb = nqb - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qb * BQ;
  const int off = p.Sk - p.Sq;
  const int qp_lo = q0 + off, qp_hi = min(q0 + BQ, p.Sq) - 1 + off;
  int k_end = p.Sk;
  if (p.causal) k_end = min(k_end, qp_hi + 1);
  int k_beg = 0;
  if (p.window_left >= 0) k_beg = (int)max((int64_t)0, (int64_t)qp_lo - p.window_left);
  k_beg = (k_beg / BKV) * BKV;
  const int nt = k_end > k_beg ? (k_end - k_beg + BKV - 1) / BKV : 0;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_o);
    mbar_init(q_full, 1);
    for (int s = 0; s < kKSt; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVSt; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < kSP; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_final, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    // Two rings: K tile j may load once S_{j-kKSt} is done, V tile j once
    // P.V_{j-kVSt} is done; K runs ahead of V.
    mbar_arrive_expect_tx(q_full, kQBytes);
    for (int bx = 0; bx < 2; ++bx)
      tma_load_4d(sQ + bx * (BQ * 128), &tm_q, q_full, bx * 64, q0, h, b);
    int nkl = 0, nvl = 0;
    uint32_t idle = 0;
    while (ok && nvl < nt) {
      bool progressed = false;
      if (nkl < nt && (nkl < kKSt || mbar_try_wait(&k_empty[nkl % kKSt],
                                                   ((nkl / kKSt) & 1) ^ 1))) {
        const int s = nkl % kKSt;
        mbar_arrive_expect_tx(&k_full[s], kTile);
        for (int bx = 0; bx < 2; ++bx)
          tma_load_4d(sK + s * kTile + bx * (BKV * 128), &tm_k, &k_full[s], bx * 64,
                      k_beg + nkl * BKV, kvh, b);
        ++nkl;
        progressed = true;
      }
      if (nvl < nkl && (nvl < kVSt || mbar_try_wait(&v_empty[nvl % kVSt],
                                                    ((nvl / kVSt) & 1) ^ 1))) {
        const int s = nvl % kVSt;
        mbar_arrive_expect_tx(&v_full[s], kTile);
        for (int bx = 0; bx < 2; ++bx)
          tma_load_4d(sV + s * kTile + bx * (BKV * 128), &tm_v, &v_full[s], bx * 64,
                      k_beg + nvl * BKV, kvh, b);
        ++nvl;
        progressed = true;
      }
      if (progressed) {
        idle = 0;
      } else if (++idle > (kWaitLimit << 2)) {
        if (p.err) atomicExch(p.err, 31);
        ok = false;
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    // Event loop: issue S_ns as soon as its K tile is resident and its TMEM
    // buffer is free (P.V_{ns-3} complete), and P.V_npv as soon as P_npv is
    // written -- never blocking on one while the other is ready.
    constexpr uint32_t idesc_s = make_idesc_f16(BQ, BKV, IsBf16<T>::value, 0, 0);
    constexpr uint32_t idesc_o = make_idesc_f16(BQ, D, IsBf16<T>::value, 0, 1);
    const uint32_t tO = tmem, tS0 = tmem + 128;
    ok = mbar_wait(q_full, 0, p.err, 33);
    tc_fence_after();
    const uint32_t qa = smem_u32(sQ);
    int ns = 0, npv = 0;
    uint32_t idle = 0;
    while (ok && npv < nt) {
      bool progressed = false;
      if (ns < nt && ns < npv + kSP) {
        const int b = ns % kSP;
        // buffer b last held P_{ns-kSP}: its P.V must be complete (the use
        // before that was awaited before issuing S_{ns-kSP}, so this parity
        // test cannot alias)
        const bool buf_free = ns < kSP || mbar_try_wait(&pv_done[b], ((ns - kSP) / kSP) & 1);
        const int s = ns % kKSt;
        if (buf_free && mbar_try_wait(&k_full[s], (ns / kKSt) & 1)) {
          tc_fence_after();
          const uint32_t ka = smem_u32(sK + s * kTile);
          const uint32_t dst = tS0 + (uint32_t)(b * 128);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t o = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;
            tc_mma_f16(dst, make_sdesc(qa + o, 16, 1024, 2), make_sdesc(ka + o, 16, 1024, 2),
                       idesc_s, kk != 0);
          }
          tc_commit(&s_full[b]);
          tc_commit(&k_empty[s]);
          FA_TS(0, ns);
          ++ns;
          progressed = true;
        }
      }
      if (npv < ns && mbar_try_wait(&p_full[npv % kSP], (npv / kSP) & 1) &&
          mbar_try_wait(&v_full[npv % kVSt], (npv / kVSt) & 1)) {
        tc_fence_after();
        const int s = npv % kVSt;
        const uint32_t va = smem_u32(sV + s * kTile);
        const uint32_t pa = tS0 + (uint32_t)((npv % kSP) * 128);  // P: 64 packed columns
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          // B = V tile, MN-major 128B swizzle: 64-dim boxes LBO = 16 KB apart,
          // 8-key groups SBO = 1 KB apart; a K step of 16 keys = 2 KB.
          tc_mma_f16_ts(tO, pa + kk * 8, make_sdesc(va + kk * 2048, BKV * 128, 1024, 2),
                        idesc_o, (npv | kk) != 0);
        }
        tc_commit(&pv_done[npv % kSP]);
        tc_commit(&v_empty[s]);
        FA_TS(3, npv);
        ++npv;
        progressed = true;
      }
      if (progressed) {
        idle = 0;
      } else if (++idle > (kWaitLimit << 2)) {
        if (p.err) atomicExch(p.err, 34);
        ok = false;
      }
    }
    // every tcgen05 op of this thread (the last P.V included) is complete
    tc_commit(o_final);
  } else if (warp >= kSoftWarp0) {
    // ---------------- softmax ----------------
    // Two warpgroups: warp w handles TMEM lanes 32*(w%4).. (query rows) and
    // half hf of the 128 key columns of every tile; the two threads of a row
    // exchange their partial max through shared memory once per tile.
    constexpr int HK = BKV / 2;  // keys per thread per tile
    const int quarter = warp & 3, hf = (warp - kSoftWarp0) >> 2;
    const int rl = quarter * 32 + lane;
    const int qpos = q0 + rl + off;  // absolute key position of this query
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_off + (uint32_t)(hf * (D / 2));  // this half of O
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < nt && ok; ++j) {
      ok = mbar_wait(&s_full[j % kSP], (j / kSP) & 1, p.err, 36);
      if (!ok) break;
      tc_fence_after();
      if (threadIdx.x == 128) FA_TS(1, j);
      const uint32_t tSb = tmem + 128 + (uint32_t)((j % kSP) * 128) + lane_off;
      const int key0 = k_beg + j * BKV + hf * HK;
      const bool need_mask = (key0 + HK > p.Sk) || (p.causal && key0 + HK - 1 > qp_lo) ||
                             (p.window_left >= 0 && key0 < (int64_t)qp_hi - p.window_left);
      float sv[HK];
      {
        uint32_t r[HK];
        tmem_ld32(tSb + hf * HK, r);
        tmem_ld32(tSb + hf * HK + 32, r + 32);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < HK; ++i) sv[i] = __uint_as_float(r[i]);
      }
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < HK; ++i) {
          const int key = key0 + i;
          bool valid = key < p.Sk;
          if (p.causal) valid = valid && key <= qpos;
          if (p.window_left >= 0) valid = valid && (int64_t)key >= (int64_t)qpos - p.window_left;
          if (!valid) sv[i] = -INFINITY;
        }
      }
      // row max: 8 independent chains of three-input max over the 64 keys
      float pm[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pm[u] = fmaxf(sv[u], sv[8 + u]);
#pragma unroll
      for (int i = 16; i < HK; i += 16)
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = fmax3(pm[u], sv[i + u], sv[i + 8 + u]);
      float mx = fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]),
                       fmaxf(pm[6], pm[7]));
      // exchange with the other half of the row (slot by tile parity); also
      // orders every S load of this tile before any P store below (P of the
      // whole tile overwrites the first 64 S columns)
      xmax[((j & 1) * 2 + hf) * BQ + rl] = mx;
      asm volatile("bar.sync 2, 256;" ::: "memory");
      mx = fmaxf(mx, xmax[((j & 1) * 2 + (hf ^ 1)) * BQ + rl]) * p.scale_log2;
      // New reference max for this row?  The O rescale below runs tcgen05.ld/st,
      // which are warp-collective (.sync.aligned): the decision is made per
      // warp (both halves of a row reach the same decision), lanes that keep
      // their reference use the factor 1.
      const bool need = mx > m_ref + kRescaleThreshold;  // also true for the first finite max
      const float corr = need ? ((m_ref == -INFINITY) ? 0.f : exp2f(m_ref - mx)) : 1.f;
      if (need) {
        l *= corr;
        m_ref = mx;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // P.V_{j-1} (and with it every earlier P.V) must be done.  Its
        // barrier's previous use, P.V_{j-1-kSP}, completed before S_{j-1}
        // was issued, so the parity wait is unambiguous.
        ok = mbar_wait(&pv_done[(j - 1) % kSP], ((j - 1) / kSP) & 1, p.err, 37) && ok;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 2; c += 32) {
          uint32_t r[32];
          tmem_ld32(tO + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st32(tO + c, r);
        }
        tmem_wait_st();
      }
      // p = exp2(s * scale - m_ref); masked entries are -inf -> 0
      // pairs of keys on the two-lane fp32 pipe: scale and shift, then the
      // two exponentials, then the running sums (4 pair accumulators)
      uint64_t ps[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t pk[HK / 2];
      const float nm = (m_ref == -INFINITY) ? 0.f : -m_ref;
      const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nm2 = f2_pack(nm, nm);
#pragma unroll
      for (int i = 0; i < HK; i += 2) {
        float a0, a1;
        f2_unpack(f2_fma(f2_pack(sv[i], sv[i + 1]), sc2, nm2), a0, a1);
        const float p0 = ex2_ftz(a0), p1 = ex2_ftz(a1);
        const uint64_t pp = f2_pack(p0, p1);
        ps[(i >> 1) & 3] = f2_add(ps[(i >> 1) & 3], pp);
        pk[i / 2] = pack2<T>(p0, p1);
      }
      {
        const uint64_t t2 = f2_add(f2_add(ps[0], ps[1]), f2_add(ps[2], ps[3]));
        float t0, t1;
        f2_unpack(t2, t0, t1);
        l += t0 + t1;
      }
      tmem_st32(tSb + hf * (HK / 2), pk);  // P columns of this half's keys
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j % kSP]);
      if (threadIdx.x == 128) FA_TS(2, j);
    }
    // ---------------- epilogue: O / l -> smem (Q buffer) -> TMA store ----------------
    float* xl = xmax + 4 * BQ;  // [2 half][BQ] row sums (separate from the max slots)
    xl[hf * BQ + rl] = l;
    if (nt > 0 && ok) {
      ok = mbar_wait(o_final, 0, p.err, 38);
      tc_fence_after();
    }
    asm volatile("bar.sync 2, 256;" ::: "memory");
    const float lt = l + xl[(hf ^ 1) * BQ + rl];
    const float inv = (lt > 0.f && nt > 0) ? 1.f / lt : 0.f;
#pragma unroll
    for (int c = 0; c < D / 2; c += 32) {
      uint32_t r[32];
      tmem_ld32(tO + c, r);
      tmem_wait_ld();
      if (nt == 0) {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      uint8_t* box = sQ + hf * (BQ * 128);  // box hf = dims [64 hf, 64 hf + 64)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(r[q * 8 + i]) * inv;
        const int chunk = (c >> 3) + q;
        *reinterpret_cast<uint4*>(box + rl * 128 + ((chunk ^ (rl & 7)) << 4)) = pack8<T>(f);
      }
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 2, 256;" ::: "memory");
    if (warp == kSoftWarp0 && lane == 0) {
      for (int bx = 0; bx < 2; ++bx) tma_store_4d(&tm_o, sQ + bx * (BQ * 128), bx * 64, q0, h, b);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

int make_bshd_map(CUtensorMap* m, const void* base, int dtype, int64_t S, int64_t H, int64_t B,
                  int64_t sb, int64_t ss, int64_t sh, uint32_t rows) {
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)(S > 0 ? S : 1), (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)ss * 2, (uint64_t)sh * 2, (uint64_t)sb * 2};
  const uint32_t box[4] = {64, rows, 1, 1};
  return make_tmap(m, base, dtype, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

#ifdef TPP_DEBUG_STAMPS
extern "C" void tpp_debug_stamps_fa(unsigned long long* host, int n) {
  cudaMemcpyFromSymbol(host, g_fa_stamps, sizeof(unsigned long long) * n);
}
#endif

// Launches the tensor-core prefill kernel; returns TPP_ERR_UNSUPPORTED when
// the shape is outside it (the caller then uses the register-tile kernel).
int attn_prefill_tc(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, const void* k,
                    int64_t k_sb, int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb,
                    int64_t v_ss, int64_t v_sh, void* o, int64_t o_sb, int64_t o_ss,
                    int64_t o_sh, int64_t B, int64_t Sq, int64_t Sk, int64_t Hq, int64_t Hkv,
                    int64_t Dh, int causal, int64_t window_left, float scale, int dtype,
                    cudaStream_t st) {
  if (Dh != D || !aligned16(o) || o_sb % 8 || o_ss % 8 || o_sh % 8 || B > 65535 || Hq > 65535)
    return TPP_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv, to;
  int rc = make_bshd_map(&tq, q, dtype, Sq, Hq, B, q_sb, q_ss, q_sh, BQ);
  if (rc == TPP_OK) rc = make_bshd_map(&tk, k, dtype, Sk, Hkv, B, k_sb, k_ss, k_sh, BKV);
  if (rc == TPP_OK) rc = make_bshd_map(&tv, v, dtype, Sk, Hkv, B, v_sb, v_ss, v_sh, BKV);
  if (rc == TPP_OK) rc = make_bshd_map(&to, o, dtype, Sq, Hq, B, o_sb, o_ss, o_sh, BQ);
  if (rc != TPP_OK) return rc;
  TcAttnArgs a;
  a.Sq = (int)Sq; a.Sk = (int)Sk; a.Hq = (int)Hq; a.Hkv = (int)Hkv;
  a.causal = causal; a.window_left = window_left;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = device_error_flag();
  const dim3 grid((unsigned)((Sq + BQ - 1) / BQ), (unsigned)Hq, (unsigned)B);
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    auto kern = attn_prefill_tc_kernel<T>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) !=
        cudaSuccess) {
      set_error("attn_prefill_tc_kernel: cannot reserve shared memory");
      return (int)TPP_ERR_LAUNCH;
    }
    return launch("attn_prefill_tc_kernel", kern, grid, dim3(kThreads), kSmem, st, 0u, tq, tk,
                  tv, to, a);
  });
}

}  // namespace tpp
