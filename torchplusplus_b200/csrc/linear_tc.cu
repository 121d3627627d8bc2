// Prefill-shaped linear layers on the 5th-generation tensor cores:
//   y[M,N] = epilogue(x[M,K] . W[N,K]^T), M > 64.
//
// Persistent, warp-specialised kernel: one CTA per SM walks output tiles of
// 128 x NOUT (NOUT = 192, or 128 SwiGLU outputs from a 256-wide gate|up
// tile).  Two fp32 accumulators live in TMEM so the epilogue of one tile
// overlaps the MMAs of the next.  384 threads:
//   warp 0 / lane 0 : TMA producer.  Streams 64-wide K slices of x and W
//                     through a shared-memory ring (128-byte swizzle,
//                     per-CTA loads), full/empty mbarrier per stage, continuous
//                     across tiles.
//   warp 1 / lane 0 : MMA issuer.  tcgen05.mma kind::f16 (M=128, N=BN, K=16)
//                     x4 per stage into accumulator j%2; tcgen05.commit frees
//                     the stage and, after the tile's last slice, hands the
//                     accumulator to the epilogue.
//   warps 4..11     : epilogue.  Warp w reads TMEM lanes 32*(w%4).. (tile
//                     rows) for one half of the columns, applies bias /
//                     activation / SwiGLU / residual in fp32, stages the tile
//                     as 128-byte-swizzled [128 x 64] boxes and one thread
//                     writes it with TMA bulk tensor stores.
// SwiGLU: the B stage holds 128 gate rows then 128 up rows (two TMA boxes), so
// accumulator columns [0,128) are gate and [128,256) up for the same outputs.
// Reference: the CUTLASS 2.x Sm80 fused linear of
// csrc/activation/fused_gemm.cuh:143-170 (mma.sync 16x8x16, 128x128x32 tiles,
// activation epilogue at fused_gemm.cuh:79-105 whose accumulator conversion is
// missing); parity here is against the PyTorch formula act(x W^T + b).
#include <stdlib.h>
#include "tc_common.cuh"

namespace tpp {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 128 bytes of fp16/bf16: one swizzle row
constexpr int kThreads = 384;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiThreads = 256;
#ifndef TPP_TC_BN2
#define TPP_TC_BN2 192
#endif
constexpr uint32_t kSubA = BM * BK * 2;  // one 64-wide k-block of x: 16 KB

// KS k-blocks per ring stage.  A stage's operands arrive as ONE TMA request
// each (a 3-D / 4-D box spanning KS k-blocks): a CTA's TMA issue rate, not
// the bytes, bounds the feed at these tile sizes, so KS = 2 halves the
// requests per tile (KS = 1 serves K not a multiple of 64, with 2-D maps).
template <bool SWIGLU, int KS>
struct TcCfg {
  static constexpr int BN = SWIGLU ? 256 : (KS == 2 ? TPP_TC_BN2 : 192);  // MMA N
  static constexpr int NOUT = SWIGLU ? BN / 2 : BN;   // output columns per tile
  static constexpr int kStages = KS == 2 ? (SWIGLU || BN > 128 ? 2 : 3) : (SWIGLU ? 3 : 4);
  static constexpr uint32_t kSubB = BN * BK * 2;      // one k-block of W
  static constexpr uint32_t kStageA = KS * kSubA;
  static constexpr uint32_t kStageB = KS * kSubB;
  static constexpr uint32_t kOut = BM * NOUT * 2;     // staged output tile
  static constexpr size_t kSmem =
      (size_t)kStages * (kStageA + kStageB) + kOut + 1024 /*align*/ + 256 /*bars*/;
  static_assert(kSmem <= 227 * 1024, "shared memory plan exceeds 227 KB");
};

struct TcArgs {
  const void* bias;
  const void* residual;
  void* y;
  int64_t ldy;
  int M, N, K;
  int act;
  int vec_ok;  // y/residual rows allow TMA stores / 16-byte loads
  int* err;
};

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
}

template <typename T, bool SWIGLU, int KS>
__global__ void __launch_bounds__(kThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_y, TcArgs p) {
  using C = TcCfg<SWIGLU, KS>;
  constexpr int BN = C::BN, NOUT = C::NOUT, S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment: the 128B-swizzle pattern repeats every 8 rows of 128 B.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::kStageA;
  uint8_t* sout = sB + S * C::kStageB;
  uint64_t* full = reinterpret_cast<uint64_t*>(sout + C::kOut);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntm = (p.M + BM - 1) / BM;
  const int ntiles = ntm * ((p.N + NOUT - 1) / NOUT);
  const int nk = (p.K + BK * KS - 1) / (BK * KS);  // ring stages per tile

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_y);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiThreads / 32);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);  // two BN-column accumulators
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Barrier init, TMEM allocation and descriptor prefetch above overlap the
  // previous kernel; everything below reads its outputs.
  pdl_wait();
  pdl_trigger();

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int it = 0;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int m0 = (t % ntm) * BM, n0 = (t / ntm) * NOUT;
      for (int kb = 0; kb < nk && ok; ++kb, ++it) {
        const int s = it % S;
        if (it >= S) ok = mbar_wait(&empty[s], ((it / S) & 1) ^ 1, p.err, 1);
        if (!ok) break;
        mbar_arrive_expect_tx(&full[s], C::kStageA + C::kStageB);
        if constexpr (KS == 1) {
          tma_load_2d(sA + s * C::kStageA, &tm_x, &full[s], kb * BK, m0);
          if (SWIGLU) {
            tma_load_2d(sB + s * C::kStageB, &tm_w, &full[s], kb * BK, n0);
            tma_load_2d(sB + s * C::kStageB + C::kStageB / 2, &tm_w, &full[s], kb * BK,
                        p.N + n0);
          } else {
            tma_load_2d(sB + s * C::kStageB, &tm_w, &full[s], kb * BK, n0);
          }
        } else {
          // {64, row, k-block} boxes: smem [k-block][row][128 B]; SwiGLU W as
          // {64, row, half, k-block}: [k-block][gate rows | up rows][128 B]
          tma_load_3d(sA + s * C::kStageA, &tm_x, &full[s], 0, m0, kb * KS);
          if (SWIGLU)
            tma_load_4d(sB + s * C::kStageB, &tm_w, &full[s], 0, n0, 0, kb * KS);
          else
            tma_load_3d(sB + s * C::kStageB, &tm_w, &full[s], 0, n0, kb * KS);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = make_idesc_f16(BM, BN, IsBf16<T>::value, 0, 0);
    int it = 0, j = 0;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++j) {
      const int buf = j & 1;
      if (j >= 2) ok = mbar_wait(&tempty[buf], ((j >> 1) & 1) ^ 1, p.err, 4);
      if (!ok) break;
      tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)(buf * BN);
      for (int kb = 0; kb < nk && ok; ++kb, ++it) {
        const int s = it % S;
        ok = mbar_wait(&full[s], (it / S) & 1, p.err, 2);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * C::kStageA);
        const uint32_t b0 = smem_u32(sB + s * C::kStageB);
#pragma unroll
        for (int k = 0; k < KS * BK / 16; ++k) {
          // K-major, 128B swizzle: 8-row groups 1024 B apart; a K step of 16
          // elements advances the start address by 32 bytes inside the row;
          // k-block j of the stage starts j sub-tiles further.
          const uint32_t j = k >> 2, kk = k & 3;
          const uint64_t ad = make_sdesc(a0 + j * kSubA + kk * 32, 16, 1024, 2);
          const uint64_t bd = make_sdesc(b0 + j * C::kSubB + kk * 32, 16, 1024, 2);
          tc_mma_f16(acc, ad, bd, idesc, (kb | k) != 0);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(&tfull[buf]);
    }
  } else if (warp >= kEpiWarp0) {
    // ---------------- epilogue ----------------
    constexpr int HALF = NOUT / 2;  // columns per warp half
    const int ew = warp - kEpiWarp0;
    const int quarter = warp & 3, hc = ew >> 2;
    const int rl = quarter * 32 + lane;  // tile row = TMEM lane
    const T* bias = static_cast<const T*>(p.bias);
    const T* res = static_cast<const T*>(p.residual);
    T* Y = static_cast<T*>(p.y);
    const bool use_tma = p.vec_ok != 0;
    const bool leader = (ew == 0 && lane == 0);
    int j = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++j) {
      const int m0 = (t % ntm) * BM, n_out0 = (t / ntm) * NOUT;
      const int buf = j & 1;
      const bool got = mbar_wait(&tfull[buf], (j >> 1) & 1, p.err, 3);
      tc_fence_after();
      const uint32_t trow = tmem + (uint32_t)(buf * BN) + ((uint32_t)(quarter * 32) << 16);
      const int row = m0 + rl;
      // the staging buffer is free once the previous tile's TMA store has read it
      if (use_tma) {
        if (leader) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        epi_bar();
      }
#pragma unroll 1
      for (int cc = 0; cc < HALF; cc += 32) {
        const int c = hc * HALF + cc;  // first column of this chunk within the tile
        uint32_t r[32], r2[32];
        tmem_ld32(trow + c, r);
        if (SWIGLU) tmem_ld32(trow + BN / 2 + c, r2);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int n = n_out0 + c + jj;
          float a = __uint_as_float(r[jj]);
          if (SWIGLU) {
            float u = __uint_as_float(r2[jj]);
            if (bias && n < p.N) { a += to_f32(bias[n]); u += to_f32(bias[p.N + n]); }
            a = act_silu(a) * u;
          } else {
            if (bias && n < p.N) a += to_f32(bias[n]);
            a = apply_act(p.act, a);
          }
          v[jj] = a;
        }
        const int n0 = n_out0 + c;
        const T* rr = (res && row < p.M) ? res + (int64_t)row * p.ldy : nullptr;
        if (use_tma) {
          uint8_t* box = sout + (c >> 6) * (BM * 128);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (rr && n0 + q * 8 + 8 <= p.N) {
              float rf[8];
              unpack8<T>(*reinterpret_cast<const uint4*>(rr + n0 + q * 8), rf);
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) v[q * 8 + jj] += rf[jj];
            } else if (rr) {
              for (int jj = 0; jj < 8 && n0 + q * 8 + jj < p.N; ++jj)
                v[q * 8 + jj] += to_f32(rr[n0 + q * 8 + jj]);
            }
            const int chunk = ((c & 63) >> 3) + q;  // 16-byte chunk within the 128-byte row
            *reinterpret_cast<uint4*>(box + rl * 128 + ((chunk ^ (rl & 7)) << 4)) =
                pack8<T>(v + q * 8);
          }
        } else if (got && row < p.M) {
          T* yr = Y + (int64_t)row * p.ldy;
          for (int jj = 0; jj < 32; ++jj) {
            const int n = n0 + jj;
            if (n >= p.N) break;
            float a = v[jj];
            if (rr) a += to_f32(rr[n]);
            yr[n] = from_f32<T>(a);
          }
        }
      }
      // accumulator `buf` may be overwritten by the MMAs of tile j + 2
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      if (use_tma) {
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the TMA engine
        epi_bar();
        if (leader && got) {
#pragma unroll
          for (int b = 0; b < NOUT / 64; ++b) {
            asm volatile(
                "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                    reinterpret_cast<uint64_t>(&tm_y)),
                "r"(n_out0 + b * 64), "r"(m0), "r"(smem_u32(sout + b * (BM * 128)))
                : "memory");
          }
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
    }
    if (leader) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace

int linear_tc(const void* x, int64_t ldx, const void* w, const void* bias, const void* residual,
              void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act, int dtype,
              cudaStream_t st) {
  TPP_REQUIRE(ldx % 8 == 0 && K % 8 == 0 && aligned16(x) && aligned16(w), TPP_ERR_ALIGN,
              "tensor-core path needs 16-byte aligned x/W rows (K and ldx multiples of 8)");
  const bool sw = act == TPP_ACT_SWIGLU;
  const int64_t wrows = sw ? 2 * N : N;
  // k-blocks per stage: 2 (one 3-D / 4-D box per operand and stage) when the
  // rows are whole 64-element k-blocks, else 1 (2-D boxes, ragged K zero-filled)
  static const bool ks2_on = [] {  // TPP_TC_KS=1 forces one k-block per stage (A/B)
    const char* e = getenv("TPP_TC_KS");
    return !(e && e[0] == '1');
  }();
  const int ks = (K % 64 == 0 && ks2_on) ? 2 : 1;
  CUtensorMap tx, tw;
  if (ks == 1) {
    {
      uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
      uint64_t strides[1] = {(uint64_t)ldx * 2};
      uint32_t box[2] = {BK, BM};
      int rc = make_tmap(&tx, x, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != TPP_OK) return rc;
    }
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)wrows};
    uint64_t strides[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {BK, (uint32_t)(sw ? TcCfg<true, 1>::BN / 2 : TcCfg<false, 1>::BN)};
    int rc = make_tmap(&tw, w, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  } else {
    const uint64_t nkb = (uint64_t)(K / 64);
    {
      uint64_t dims[3] = {64, (uint64_t)M, nkb};
      uint64_t strides[2] = {(uint64_t)ldx * 2, 128};
      uint32_t box[3] = {64, BM, 2};
      int rc = make_tmap(&tx, x, dtype, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != TPP_OK) return rc;
    }
    int rc;
    if (sw) {
      uint64_t dims[4] = {64, (uint64_t)N, 2, nkb};
      uint64_t strides[3] = {(uint64_t)K * 2, (uint64_t)N * K * 2, 128};
      uint32_t box[4] = {64, (uint32_t)(TcCfg<true, 2>::BN / 2), 2, 2};
      rc = make_tmap(&tw, w, dtype, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
      uint64_t dims[3] = {64, (uint64_t)N, nkb};
      uint64_t strides[2] = {(uint64_t)K * 2, 128};
      uint32_t box[3] = {64, (uint32_t)TcCfg<false, 2>::BN, 2};
      rc = make_tmap(&tw, w, dtype, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc != TPP_OK) return rc;
  }
  CUtensorMap ty;
  const bool y_tma = (N % 8 == 0) && (ldy % 8 == 0) && aligned16(y);
  if (y_tma) {
    uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    uint64_t strides[1] = {(uint64_t)ldy * 2};
    uint32_t box[2] = {64, BM};
    int rc = make_tmap(&ty, y, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  } else {
    ty = tx;  // unused
  }
  TcArgs a;
  a.bias = bias; a.residual = residual; a.y = y; a.ldy = ldy;
  a.M = (int)M; a.N = (int)N; a.K = (int)K; a.act = act;
  a.vec_ok = y_tma && (!residual || aligned16(residual));
  a.err = device_error_flag();
  const int nout = ks == 2 ? (sw ? TcCfg<true, 2>::NOUT : TcCfg<false, 2>::NOUT)
                           : (sw ? TcCfg<true, 1>::NOUT : TcCfg<false, 1>::NOUT);
  const int64_t tiles = ((N + nout - 1) / nout) * ((M + BM - 1) / BM);
  const int grid = (int)(tiles < num_sms() ? tiles : num_sms());  // persistent
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    auto go = [&](auto kern, size_t smem) -> int {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess) {
        set_error("linear_tc_kernel: cannot reserve shared memory");
        return (int)TPP_ERR_LAUNCH;
      }
      return launch("linear_tc_kernel", kern, dim3((unsigned)grid), dim3(kThreads), smem, st, 0,
                    tx, tw, ty, a);
    };
    if (ks == 2)
      return sw ? go(linear_tc_kernel<T, true, 2>, TcCfg<true, 2>::kSmem)
                : go(linear_tc_kernel<T, false, 2>, TcCfg<false, 2>::kSmem);
    return sw ? go(linear_tc_kernel<T, true, 1>, TcCfg<true, 1>::kSmem)
              : go(linear_tc_kernel<T, false, 1>, TcCfg<false, 1>::kSmem);
  });
}

}  // namespace tpp
