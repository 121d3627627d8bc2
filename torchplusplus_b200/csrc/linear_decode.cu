// Decode-shaped linear layers: y[M,N] = epilogue(x[M,K] . W[N,K]^T) for M <= 64.
//
// At decode the weight matrix is read exactly once per step and the token
// count is tiny, so the kernel is bound by HBM bandwidth on W.  Design
// ("swap-AB" on the 5th-generation tensor cores):
//  * The MMA's M side is 128 weight rows, its N side the (padded) tokens
//    (BN = 16/32/64): D[128 x BN] += W_tile[128 x 64] . x_tile[BN x 64]^T with
//    tcgen05.mma kind::f16, fp32 accumulator in TMEM (BN columns).
//  * W and x tiles arrive by TMA (128-byte swizzle, per-CTA loads) in a
//    kStages-deep shared-memory ring guarded by full/empty mbarriers: up to
//    kStages x 16 KB of weights in flight per CTA, independent of registers.
//  * The first kStages weight tiles are requested BEFORE the programmatic-
//    dependent-launch wait: weights never depend on the previous kernel, so
//    they stream while that kernel drains.  x tiles follow after the wait.
//  * Short-and-wide matrices split K over the CTAs of a thread-block cluster
//    (1, 2, 4 or 8).  The tile's outputs are divided among the ranks; every
//    rank pushes its TMEM partial rows to their owners with remote shared-
//    memory stores, and after one cluster barrier each owner sums its slice
//    and runs the fused epilogue (bias, activation, SwiGLU gate*up, residual
//    add).  No global scratch.
//  * Epilogue stores are staged through shared memory as [token][output] so
//    y is written with coalesced 16-byte stores.
//  * SwiGLU: the 128-row A tile holds 64 gate rows then the 64 matching up
//    rows (two TMA boxes), so one tile yields 64 outputs silu(g)*u.
// Roles in the 128-thread CTA: warp 0 / lane 0 issues TMA, warp 1 / lane 0
// issues MMAs, all 4 warps run the epilogue (warp w owns TMEM lanes
// 32w..32w+31 = tile rows).
// Reference: the unbuilt hgemv kernels csrc/blas/hgemv/hgemv_kernels.cuh:19-85
// (one warp per row, fp16 accumulation) and the CUTLASS Sm80 fused linear of
// csrc/activation/fused_gemm.cuh:143-170 (128x128 tiles over M, which waste
// >= 75% of the MMA at M <= 32).  Accumulation here is fp32.
#include <cooperative_groups.h>
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace tpp {
namespace {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // 128 bytes: one swizzle row
constexpr int kMaxStages = 8;
constexpr int kThreads = 128;
constexpr uint32_t kStageA = BM * BK * 2;  // 16 KB

template <int BN>
constexpr uint32_t stage_b() { return BN * BK * 2; }

// Shared-memory plan (offsets from the 1024-aligned base):
//   [0, ring)                 W and x stages (runtime depth p.stages); once the
//                             CTA's MMAs are done the ring is reused for the
//                             epilogue staging
//   [ring, ring + 1024)       mbarriers, TMEM slot, RMSNorm statistics
//   [ring + 1024, ...)        split-K only: receive buffer for the partial
//                             rows other ranks push here, their RMSNorm sums,
//                             and the prefetched residual slice.  These never
//                             alias the ring, so a rank may push as soon as
//                             its own MMAs are done.
template <int BN>
struct SkinnyPlan {
  static constexpr int RSV = BN + 4;                      // receive row stride (16-byte rows)
  static constexpr uint32_t recv_bytes = BM * RSV * 4;    // 128 rows over all source ranks
  static constexpr uint32_t ssr_bytes = 8 * 64 * 4;       // [source rank][token] sums of squares
  static constexpr uint32_t rsd_bytes = BN * 64 * 2;      // residual [token][<= 64 outputs]
  static constexpr uint32_t split_bytes = recv_bytes + ssr_bytes + rsd_bytes;
  __host__ __device__ static uint32_t ring(int stages) { return (uint32_t)stages * (kStageA + stage_b<BN>()); }
  static size_t smem(int stages, bool split) {
    return 1024 + ring(stages) + 1024 + (split ? split_bytes : 0);
  }
};

struct SkinnyArgs {
  const void* bias;
  const void* residual;
  void* y;
  int64_t ldy;
  int M, N, K;
  int act;
  int kb_per_split;
  int stages;
  int vec_ok;
  float eps;  // fused RMSNorm of x (NORM variant)
  int* err;
#ifdef TPP_DEBUG_STAMPS
  unsigned dbg_id;
#endif
};

#ifdef TPP_DEBUG_STAMPS
// [launch % 64][cta < 512][10] globaltimer stamps of thread 0
__device__ unsigned long long g_dbg_stamps[64 * 512 * 10];
unsigned g_dbg_launch = 0;
#endif

template <int BN>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, float* v) {
  uint32_t r[32];
  if constexpr (BN == 16) {
    tmem_ld16(taddr, r);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
  } else {
#pragma unroll
    for (int h = 0; h < BN / 32; ++h) {
      tmem_ld32(taddr + h * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) v[h * 32 + j] = __uint_as_float(r[j]);
    }
  }
}

// Remote shared-memory stores that report their bytes to the destination
// CTA's mbarrier (complete_tx), so the receiver needs no cluster barrier.
__device__ __forceinline__ uint32_t map_rank(uint32_t local, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_async_v4(uint32_t addr, float a, float b, float c, float d,
                                            uint32_t bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, "
      "[%5];" ::"r"(addr),
      "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void st_async_f32(uint32_t addr, float a, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(
                   addr),
               "f"(a), "r"(bar)
               : "memory");
}
// Bounded wait with cluster-scope acquire (the bytes were written by other
// CTAs of the cluster).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err,
                                                  int code) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  if (err) atomicExch(err, code);
  return false;
}

template <typename T, int BN, bool SWIGLU, bool NORM>
__global__ void __launch_bounds__(kThreads, 1)
    linear_skinny_kernel(const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_x, SkinnyArgs p) {
  using Plan = SkinnyPlan<BN>;
  constexpr uint32_t kStageB = stage_b<BN>();
  constexpr int TCOLS = BN < 32 ? 32 : BN;  // TMEM allocation (power of 2 >= 32)
  constexpr int NOUT = SWIGLU ? BM / 2 : BM;
  constexpr int RS = BN + 1;   // padded row stride for the SwiGLU hand-over (odd: no conflicts)
  constexpr int RSV = Plan::RSV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  const int S = p.stages;
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kStageA;
  uint8_t* misc = smem + Plan::ring(S);
  uint64_t* full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* empty = full + kMaxStages;
  uint64_t* accum = empty + kMaxStages;
  uint64_t* rbar = accum + 1;  // split-K: all pushed partials for my slice have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 1);
  // RMSNorm statistics (fused-norm variant): own partial sum of squares per
  // token, final 1/rms per token.
  float* ss_part = reinterpret_cast<float*>(misc + 256);
  float* rtok = ss_part + 64;
  float* recv = reinterpret_cast<float*>(misc + 1024);              // [src][rows][RSV]
  float* ss_recv = reinterpret_cast<float*>(misc + 1024 + Plan::recv_bytes);  // [8][64]
  T* rsd = reinterpret_cast<T*>(misc + 1024 + Plan::recv_bytes + Plan::ssr_bytes);
  // Ring reuse after the MMAs: SwiGLU hand-over (no split) and output staging.
  float* hand = reinterpret_cast<float*>(smem);

#ifdef TPP_DEBUG_STAMPS
  unsigned long long stamps[10] = {};
  auto ts = [&](int i) { asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(stamps[i])); };
  ts(0);
#define TPP_TS(i) ts(i)
#else
#define TPP_TS(i)
#endif
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int out0 = blockIdx.x * NOUT;  // first output feature of this tile
  const int nkb = (p.K + BK - 1) / BK;
  const int kb0 = crank * p.kb_per_split;
  const int kb1 = min(nkb, kb0 + p.kb_per_split);
  const int nk = kb1 > kb0 ? kb1 - kb0 : 0;
  const int per = NOUT / csize;  // csize divides NOUT (host picks 1, 2, 4 or 8)
  const int o0 = crank * per;    // my slice of the tile's outputs
  const int rows_per = SWIGLU ? 2 * per : per;
  const int mt = p.M < BN ? p.M : BN;
  float* stage = csize > 1 ? hand : hand + (SWIGLU ? (BM / 2) * RS : 0);  // [BN][per + 1]

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NORM ? 3 : 1);  // MMA commit (+ the two norm warps)
    }
    mbar_init(accum, 1);
    mbar_init(rbar, 1);
    if (csize > 1)  // every rank pushes rows_per rows (+ its per-token sums) to me
      mbar_arrive_expect_tx(rbar, (uint32_t)(csize * rows_per * BN * 4 + (NORM ? csize * BN * 4 : 0)));
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TCOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Publish the initialised barriers to the cluster; the matching wait sits
  // just before the first remote store, long after every rank got here.
  if (csize > 1) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  TPP_TS(1);

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    auto load_w = [&](int i) {
      const int s = i % S;
      const int kc = (kb0 + i) * BK;
      mbar_arrive_expect_tx(&full[s], kStageA + kStageB);
      if (SWIGLU) {
        tma_load_2d(sA + s * kStageA, &tm_w, &full[s], kc, out0);
        tma_load_2d(sA + s * kStageA + kStageA / 2, &tm_w, &full[s], kc, p.N + out0);
      } else {
        tma_load_2d(sA + s * kStageA, &tm_w, &full[s], kc, out0);
      }
    };
    const int pre = nk < S ? nk : S;
    for (int i = 0; i < pre; ++i) load_w(i);  // weights: independent of the previous kernel
    pdl_wait();
    TPP_TS(8);
    pdl_trigger();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(sB + (i % S) * kStageB, &tm_x, &full[i % S], (kb0 + i) * BK, 0);
    for (int i = pre; i < nk && ok; ++i) {
      const int s = i % S;
      ok = mbar_wait(&empty[s], ((i / S) & 1) ^ 1, p.err, 11);
      if (!ok) break;
      load_w(i);
      tma_load_2d(sB + s * kStageB, &tm_x, &full[s], (kb0 + i) * BK, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    pdl_wait();
    constexpr uint32_t idesc = make_idesc_f16(BM, BN, IsBf16<T>::value, 0, 0);
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % S;
      ok = mbar_wait(&full[s], (i / S) & 1, p.err, 12);
      if (!ok) break;
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + s * kStageA);
      const uint32_t b0 = smem_u32(sB + s * kStageB);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {
        const uint64_t ad = make_sdesc(a0 + k * 32, 16, 1024, 2);
        const uint64_t bd = make_sdesc(b0 + k * 32, 16, 1024, 2);
        tc_mma_f16(tmem, ad, bd, idesc, (i | k) != 0);
      }
      tc_commit(&empty[s]);
    }
    tc_commit(accum);
  } else {
    pdl_wait();
    if (warp >= 2) {
      const int tid2 = threadIdx.x - 64;
      // ---------------- residual prefetch (split-K) ----------------
      // The owner of each output slice reads its residual now, while the
      // weights stream, instead of after the reduction.
      if (csize > 1 && p.residual && p.vec_ok) {
        const T* res = static_cast<const T*>(p.residual);
        const int chunks = per / 8;
        for (int e = tid2; e < mt * chunks; e += 64) {
          const int t = e / chunks, ch = e % chunks;
          const int n0 = out0 + o0 + ch * 8;
          if (n0 + 8 <= p.N)
            *reinterpret_cast<uint4*>(rsd + t * per + ch * 8) =
                *reinterpret_cast<const uint4*>(res + (int64_t)t * p.ldy + n0);
        }
      }
      if (NORM) {
        // ---------------- RMSNorm statistics from the staged x tiles ----------------
        constexpr int TPR = 64 / BN;   // threads per token row
        constexpr int CPT = 8 / TPR;   // 16-byte chunks per thread (a row is 128 B)
        const int t = tid2 / TPR, part = tid2 % TPR;
        float ss = 0.f;
        for (int i = 0; i < nk && ok; ++i) {
          const int s = i % S;
          ok = mbar_wait(&full[s], (i / S) & 1, p.err, 14);
          if (!ok) break;
          const uint8_t* xr = sB + s * kStageB + t * 128 + part * CPT * 16;
#pragma unroll
          for (int q = 0; q < CPT; ++q) {
            float f[8];
            unpack8<T>(*reinterpret_cast<const uint4*>(xr + q * 16), f);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
#pragma unroll
        for (int o = TPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (part == 0) ss_part[t] = ss;
      }
    }
  }
  __syncwarp();

  // ---------------- accumulator -> registers ----------------
  const bool got = mbar_wait(accum, 0, p.err, 13);
  tc_fence_after();
  TPP_TS(2);
  const int row = warp * 32 + lane;  // tile row = TMEM lane
  const T* bias = static_cast<const T*>(p.bias);
  float v[BN];
  tmem_ld_row<BN>(tmem + ((uint32_t)(warp * 32) << 16), v);
  if (!got || nk == 0) {
#pragma unroll
    for (int j = 0; j < BN; ++j) v[j] = 0.f;
  }
  TPP_TS(3);
  if (NORM) __syncthreads();  // ss_part complete
  if (NORM && csize == 1) {
    if (threadIdx.x < BN) rtok[threadIdx.x] = rsqrtf(ss_part[threadIdx.x] / (float)p.K + p.eps);
    __syncthreads();
  }
  if (csize > 1) {
    // ---------------- split-K reduce-scatter over DSMEM ----------------
    // Rank r owns outputs [o0, o0 + per) of the tile.  Every rank pushes its
    // partial rows for them (gate rows then the matching up rows for SwiGLU)
    // into the owner's receive buffer recv[src][rowl][RSV] with st.async;
    // each store reports its bytes to the owner's rbar, so the owner only
    // waits for its own barrier.
    const int orow = SWIGLU ? (row % (BM / 2)) : row;  // output index of my row
    const int owner = orow / per;
    const int rowl = (orow % per) + ((SWIGLU && row >= BM / 2) ? per : 0);
    const uint32_t rdst =
        map_rank(smem_u32(recv) + (uint32_t)(((crank * rows_per + rowl) * RSV) * 4), owner);
    const uint32_t rb = map_rank(smem_u32(rbar), owner);
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    TPP_TS(5);
    if (NORM && threadIdx.x < BN) {
      // every rank needs every rank's sum of squares for token threadIdx.x
      const uint32_t sdst = smem_u32(ss_recv + crank * 64 + threadIdx.x);
      const float mine = ss_part[threadIdx.x];
      for (int r = 0; r < csize; ++r)
        st_async_f32(map_rank(sdst, r), mine, map_rank(smem_u32(rbar), r));
    }
#pragma unroll
    for (int j = 0; j < BN; j += 4) st_async_v4(rdst + 4 * j, v[j], v[j + 1], v[j + 2], v[j + 3], rb);
    const bool arrived = mbar_wait_cluster(rbar, 0, p.err, 15);
    TPP_TS(4);
    if (NORM) {
      if (threadIdx.x < BN) {
        float ss = 0.f;
        for (int r = 0; r < csize; ++r) ss += ss_recv[r * 64 + threadIdx.x];
        rtok[threadIdx.x] = rsqrtf(ss / (float)p.K + p.eps);
      }
      __syncthreads();
    }
    // token-fastest mapping: conflict-free reads of recv rows and (per + 1 is
    // odd) conflict-free writes of stage columns
    for (int e = threadIdx.x; e < per * BN; e += kThreads) {
      const int t = e % BN, ol = e / BN;
      float g = 0.f, u = 0.f;
      if (arrived) {
        float gs[8], us[8];  // independent loads: one shared-memory latency, not csize
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          gs[r] = r < csize ? recv[(r * rows_per + ol) * RSV + t] : 0.f;
          us[r] = (SWIGLU && r < csize) ? recv[(r * rows_per + per + ol) * RSV + t] : 0.f;
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) { g += gs[r]; u += us[r]; }
      }
      if (NORM) { g *= rtok[t]; u *= rtok[t]; }
      const int n = out0 + o0 + ol;
      float out = 0.f;
      if (n < p.N) {
        if (SWIGLU) {
          if (bias) { g += to_f32(bias[n]); u += to_f32(bias[p.N + n]); }
          out = act_silu(g) * u;
        } else {
          if (bias) g += to_f32(bias[n]);
          out = apply_act(p.act, g);
        }
      }
      stage[t * (per + 1) + ol] = out;
    }
  } else {
    TPP_TS(4);
    if (NORM) {
#pragma unroll
      for (int j = 0; j < BN; ++j) v[j] *= rtok[j];
    }
    if (SWIGLU) {
      // up rows (warps 2, 3) hand their values to the gate rows via smem
      if (row >= BM / 2) {
#pragma unroll
        for (int j = 0; j < BN; ++j) hand[(row - BM / 2) * RS + j] = v[j];
      }
      __syncthreads();
      if (row < BM / 2) {
        const int n = out0 + row;
        const float bg = (bias && n < p.N) ? to_f32(bias[n]) : 0.f;
        const float bu = (bias && n < p.N) ? to_f32(bias[p.N + n]) : 0.f;
#pragma unroll
        for (int j = 0; j < BN; ++j)
          stage[j * (per + 1) + row] = act_silu(v[j] + bg) * (hand[row * RS + j] + bu);
      }
    } else {
      const int n = out0 + row;
      const float bb = (bias && n < p.N) ? to_f32(bias[n]) : 0.f;
      const int act = p.act;
#pragma unroll
      for (int j = 0; j < BN; ++j) stage[j * (per + 1) + row] = apply_act(act, v[j] + bb);
    }
  }
  __syncthreads();
  TPP_TS(6);

  // ---------------- coalesced store (+ residual) ----------------
  {
    const T* res = static_cast<const T*>(p.residual);
    const bool res_smem = csize > 1 && p.vec_ok;  // prefetched above
    T* Y = static_cast<T*>(p.y);
    const int chunks = per / 8;  // 8 outputs = 16 bytes per store
    for (int e = threadIdx.x; e < mt * chunks; e += kThreads) {
      const int t = e / chunks, ch = e % chunks;
      const int n0 = out0 + o0 + ch * 8;
      if (n0 >= p.N) continue;
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = stage[t * (per + 1) + ch * 8 + j];
      T* yr = Y + (int64_t)t * p.ldy;
      const T* rr = res ? res + (int64_t)t * p.ldy : nullptr;
      if (p.vec_ok && n0 + 8 <= p.N) {
        if (rr) {
          float rf[8];
          unpack8<T>(res_smem ? *reinterpret_cast<const uint4*>(rsd + t * per + ch * 8)
                              : *reinterpret_cast<const uint4*>(rr + n0),
                     rf);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += rf[j];
        }
        *reinterpret_cast<uint4*>(yr + n0) = pack8<T>(o);
      } else {
        for (int j = 0; j < 8 && n0 + j < p.N; ++j) {
          float a = o[j];
          if (rr) a += to_f32(rr[n0 + j]);
          yr[n0 + j] = from_f32<T>(a);
        }
      }
    }
  }
#ifdef TPP_DEBUG_STAMPS
  TPP_TS(7);
  if (threadIdx.x == 0) {
    const int id = blockIdx.y * gridDim.x + blockIdx.x;
    if (id < 512)
      for (int i = 0; i < 10; ++i) g_dbg_stamps[((p.dbg_id % 64) * 512 + id) * 10 + i] = stamps[i];
  }
#endif
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TCOLS);
}

template <typename T, int BN, bool SW, bool NORM>
int launch_skinny(const void* x, int64_t ldx, const void* w, SkinnyArgs& a, int dtype,
                  cudaStream_t st) {
  using Plan = SkinnyPlan<BN>;
  constexpr int NOUT = SW ? BM / 2 : BM;
  CUtensorMap tw, tx;
  {
    const uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)(SW ? 2 * (int64_t)a.N : a.N)};
    const uint64_t strides[1] = {(uint64_t)a.K * 2};
    const uint32_t box[2] = {BK, (uint32_t)(SW ? BM / 2 : BM)};
    const int rc = make_tmap(&tw, w, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)a.M};
    const uint64_t strides[1] = {(uint64_t)ldx * 2};
    const uint32_t box[2] = {BK, (uint32_t)BN};
    const int rc = make_tmap(&tx, x, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  }
  const int sms = sm_budget();
  const int tiles = (a.N + NOUT - 1) / NOUT;
  const int nkb = (a.K + BK - 1) / BK;
  // Enough CTAs for two per SM; every split keeps >= 2 k-blocks.
  int ks = (2 * sms + tiles - 1) / tiles;
  int maxks = nkb / 2 > 0 ? nkb / 2 : 1;
  if (maxks > 8) maxks = 8;
  ks = ks < 1 ? 1 : (ks > maxks ? maxks : ks);
  // cluster size 1, 2, 4 or 8 (it must divide the tile's outputs for the
  // reduce-scatter); a split may end up with fewer k-blocks than others
  ks = ks >= 8 ? 8 : (ks >= 4 ? 4 : (ks >= 2 ? 2 : 1));
#ifdef TPP_DEBUG_STAMPS
  if (const char* e = getenv("TPP_SKINNY_KS")) {
    const int f = atoi(e);
    if (f >= 1 && f <= 8 && (f & (f - 1)) == 0 && f <= nkb) ks = f;
  }
#endif
  a.kb_per_split = (nkb + ks - 1) / ks;
  // Ring depth: every k-block of a split in flight at once when it fits (all
  // weights requested before the previous kernel ends), within half of the
  // SM's shared memory: two CTAs per SM, and room for this kernel's CTAs to
  // start (and prefetch) while the previous kernel's CTAs still run.
  const bool split = ks > 1;
  const size_t budget = 113 * 1024;
  int stages = a.kb_per_split < kMaxStages ? a.kb_per_split : kMaxStages;
  while (stages > 2 && Plan::smem(stages, split) > budget) --stages;
  // the ring also holds the epilogue staging once the MMAs are done
  const size_t alias_need =
      split ? (size_t)BN * (NOUT / ks + 1) * 4
            : (size_t)BN * (NOUT + 1) * 4 + (SW ? (size_t)(BM / 2) * (BN + 1) * 4 : 0);
  while (Plan::ring(stages) < alias_need) ++stages;
  if (stages < 2) stages = 2;
  a.stages = stages;
  const size_t smem = Plan::smem(stages, split);
  auto kern = linear_skinny_kernel<T, BN, SW, NORM>;
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess) {
      set_error("linear_skinny_kernel: cannot reserve shared memory");
      return TPP_ERR_LAUNCH;
    }
    configured |= bit;
  }
  return launch("linear_skinny_kernel", kern, dim3((unsigned)tiles, (unsigned)ks, 1),
                dim3(kThreads), smem, st, (unsigned)ks, tw, tx, a);
}

template <typename T, bool NORM>
int skinny_dispatch(const void* x, int64_t ldx, const void* w, SkinnyArgs& a, int dtype,
                    cudaStream_t st) {
  const bool sw = a.act == TPP_ACT_SWIGLU;
  if (a.M <= 16)
    return sw ? launch_skinny<T, 16, true, NORM>(x, ldx, w, a, dtype, st)
              : launch_skinny<T, 16, false, NORM>(x, ldx, w, a, dtype, st);
  if (a.M <= 32)
    return sw ? launch_skinny<T, 32, true, NORM>(x, ldx, w, a, dtype, st)
              : launch_skinny<T, 32, false, NORM>(x, ldx, w, a, dtype, st);
  return sw ? launch_skinny<T, 64, true, NORM>(x, ldx, w, a, dtype, st)
            : launch_skinny<T, 64, false, NORM>(x, ldx, w, a, dtype, st);
}

}  // namespace

#ifdef TPP_DEBUG_STAMPS
extern "C" void tpp_debug_stamps(unsigned long long* host, int n) {
  cudaMemcpyFromSymbol(host, g_dbg_stamps, sizeof(unsigned long long) * n);
}
extern "C" unsigned tpp_debug_launches() { return g_dbg_launch; }
#endif

// Entry used by tpp_linear (linear.cu) for M <= 64.
// norm_eps >= 0: x is RMS-normalised on the fly (the caller has folded the
// norm weight into W); norm_eps < 0: plain linear.
int linear_xs(const void* x, int64_t ldx, const void* w, const void* bias, const void* residual,
              void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act, int dtype,
              cudaStream_t st, float norm_eps);

// x-stationary kernel (linear_xs.cu) unless TPP_LINEAR_XS=0 (A/B measurements).
static bool xs_enabled() {
  static const bool on = [] {
    const char* e = getenv("TPP_LINEAR_XS");
    return !(e && e[0] == '0');
  }();
  return on;
}

int linear_decode(const void* x, int64_t ldx, const void* w, const void* bias,
                  const void* residual, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                  int act, int dtype, cudaStream_t st, float norm_eps) {
  if (xs_enabled()) {
    const int rc = linear_xs(x, ldx, w, bias, residual, y, ldy, M, N, K, act, dtype, st, norm_eps);
    if (rc != -1) return rc;
  }
  SkinnyArgs a;
  a.bias = bias; a.residual = residual; a.y = y; a.ldy = ldy;
  a.M = (int)M; a.N = (int)N; a.K = (int)K; a.act = act; a.kb_per_split = 0;
  a.vec_ok = (N % 8 == 0) && (ldy % 8 == 0) && aligned16(y) && (!residual || aligned16(residual));
  a.err = device_error_flag();
  a.eps = norm_eps;
#ifdef TPP_DEBUG_STAMPS
  a.dbg_id = g_dbg_launch++;
#endif
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return norm_eps >= 0.f ? skinny_dispatch<T, true>(x, ldx, w, a, dtype, st)
                           : skinny_dispatch<T, false>(x, ldx, w, a, dtype, st);
  });
}

}  // namespace tpp
