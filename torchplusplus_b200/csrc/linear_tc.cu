// Prefill-shaped linear layers on the 5th-generation tensor cores:
//   y[M,N] = epilogue(x[M,K] . W[N,K]^T), M > 64.
//
// One CTA computes a 128 x BN output tile (BN = 256) with the fp32
// accumulator in TMEM (BN columns).  128 threads, warp-specialised:
//   warp 0 / lane 0 : TMA producer.  Streams 64-wide K slices of x and W into
//                     a kStages-deep ring of shared-memory stages (128-byte
//                     swizzle, no multicast), each guarded by a full/empty
//                     mbarrier pair.
//   warp 1 / lane 0 : MMA issuer.  tcgen05.mma kind::f16 (M=128, N=BN, K=16)
//                     x4 per stage; tcgen05.commit releases the stage back to
//                     the producer and, after the last slice, signals the
//                     epilogue.
//   warps 0..3      : epilogue.  Each warp owns TMEM lanes 32w..32w+31 (= tile
//                     rows), reads 32 fp32 columns at a time with tcgen05.ld,
//                     applies bias / activation / SwiGLU / residual in fp32
//                     and stores 16-byte vectors.
// SwiGLU: the B stage holds 128 gate rows then 128 up rows (two TMA boxes), so
// accumulator columns [0,128) are gate and [128,256) up for the same outputs.
// Reference: the CUTLASS 2.x Sm80 fused linear of
// csrc/activation/fused_gemm.cuh:143-170 (mma.sync 16x8x16, 128x128x32 tiles,
// activation epilogue at fused_gemm.cuh:79-105 whose accumulator conversion is
// missing); parity here is against the PyTorch formula act(x W^T + b).
#include "tc_common.cuh"

namespace tpp {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // 128 bytes of fp16/bf16: one swizzle row
constexpr int kStages = 4;
constexpr int kThreads = 256;
constexpr uint32_t kStageA = BM * BK * 2;  // 16 KB
constexpr uint32_t kStageB = BN * BK * 2;  // 32 KB
constexpr size_t kSmem = (size_t)kStages * (kStageA + kStageB) + 1024 /*align*/ + 256 /*bars*/;

struct TcArgs {
  const void* bias;
  const void* residual;
  void* y;
  int64_t ldy;
  int M, N, K;
  int act;
  int vec_ok;  // y/residual rows allow 16-byte stores
  int* err;
};

#ifdef TPP_DEBUG_STAMPS
__device__ unsigned long long g_tc_stamps[8 * 1024];
#define TC_TS(i) do { asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(st_[i])); } while (0)
#else
#define TC_TS(i) do {} while (0)
#endif

template <typename T, bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_y, TcArgs p) {
#ifdef TPP_DEBUG_STAMPS
  unsigned long long st_[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#endif
  TC_TS(0);
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment: the 128B-swizzle pattern repeats every 8 rows of 128 B.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kStages * kStageB);
  uint64_t* empty = full + kStages;
  uint64_t* accum = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_out0 = blockIdx.x * (SWIGLU ? BN / 2 : BN);  // first output column
  const int m0 = blockIdx.y * BM;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_y);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, BN);
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
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % kStages;
      const uint32_t ph = (kb / kStages) & 1;
      if (kb >= kStages) ok = mbar_wait(&empty[s], ph ^ 1, p.err, 1);
      if (!ok) break;
      mbar_arrive_expect_tx(&full[s], kStageA + kStageB);
      tma_load_2d(sA + s * kStageA, &tm_x, &full[s], kb * BK, m0);
      if (SWIGLU) {
        tma_load_2d(sB + s * kStageB, &tm_w, &full[s], kb * BK, n_out0);
        tma_load_2d(sB + s * kStageB + kStageB / 2, &tm_w, &full[s], kb * BK, p.N + n_out0);
      } else {
        tma_load_2d(sB + s * kStageB, &tm_w, &full[s], kb * BK, n_out0);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = make_idesc_f16(BM, BN, IsBf16<T>::value, 0, 0);
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % kStages;
      const uint32_t ph = (kb / kStages) & 1;
      ok = mbar_wait(&full[s], ph, p.err, 2);
      if (!ok) break;
      if (kb == 0) TC_TS(1);
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + s * kStageA);
      const uint32_t b0 = smem_u32(sB + s * kStageB);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) {
        // K-major, 128B swizzle: 8-row groups 1024 B apart; a K step of 16
        // elements advances the start address by 32 bytes inside the row.
        const uint64_t ad = make_sdesc(a0 + k * 32, 16, 1024, 2);
        const uint64_t bd = make_sdesc(b0 + k * 32, 16, 1024, 2);
        tc_mma_f16(tmem, ad, bd, idesc, (kb | k) != 0);
      }
      tc_commit(&empty[s]);
    }
    tc_commit(accum);
    TC_TS(2);
  }
  __syncwarp();

  // ---------------- epilogue (all 8 warps) ----------------
  // Warp w reads TMEM lanes 32*(w%4).. (tile rows) and one half of the
  // output columns; results (bias, activation, SwiGLU, residual applied in
  // fp32) are staged in shared memory as 128-byte-swizzled [128 x 64] boxes
  // and written by TMA bulk tensor stores (full-line, coalesced writes).
  const bool got = mbar_wait(accum, 0, p.err, 3);
  tc_fence_after();
  TC_TS(3);
  constexpr int NOUT = SWIGLU ? BN / 2 : BN;
  constexpr int HALF = NOUT / 2;  // columns per warp half
  const int quarter = warp & 3, hc = warp >> 2;
  const int rl = quarter * 32 + lane;  // tile row
  const int row = m0 + rl;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
  const T* bias = static_cast<const T*>(p.bias);
  const T* res = static_cast<const T*>(p.residual);
  T* Y = static_cast<T*>(p.y);
  const bool use_tma = p.vec_ok != 0;
  uint8_t* sout = smem;  // the operand ring is idle now: NOUT/64 boxes of 16 KB
#pragma unroll 1
  for (int cc = 0; cc < HALF; cc += 32) {
    const int c = hc * HALF + cc;  // first column of this chunk within the tile
    uint32_t r[32], r2[32];
    tmem_ld32(trow + c, r);
    if (SWIGLU) tmem_ld32(trow + BN / 2 + c, r2);
    tmem_wait_ld();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n_out0 + c + j;
      float a = __uint_as_float(r[j]);
      if (SWIGLU) {
        float u = __uint_as_float(r2[j]);
        if (bias && n < p.N) { a += to_f32(bias[n]); u += to_f32(bias[p.N + n]); }
        a = act_silu(a) * u;
      } else {
        if (bias && n < p.N) a += to_f32(bias[n]);
        a = apply_act(p.act, a);
      }
      v[j] = a;
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
          for (int j = 0; j < 8; ++j) v[q * 8 + j] += rf[j];
        } else if (rr) {
          for (int j = 0; j < 8 && n0 + q * 8 + j < p.N; ++j) v[q * 8 + j] += to_f32(rr[n0 + q * 8 + j]);
        }
        const int chunk = ((c & 63) >> 3) + q;  // 16-byte chunk within the 128-byte row
        *reinterpret_cast<uint4*>(box + rl * 128 + ((chunk ^ (rl & 7)) << 4)) =
            pack8<T>(v + q * 8);
      }
    } else if (got && row < p.M) {
      T* yr = Y + (int64_t)row * p.ldy;
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + j;
        if (n >= p.N) break;
        float a = v[j];
        if (rr) a += to_f32(rr[n]);
        yr[n] = from_f32<T>(a);
      }
    }
  }
  if (use_tma) {
    fence_proxy_async_smem();  // generic-proxy writes -> visible to the TMA engine
    __syncthreads();
    if (threadIdx.x == 0 && got) {
#pragma unroll
      for (int b = 0; b < NOUT / 64; ++b) {
        asm volatile(
            "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                reinterpret_cast<uint64_t>(&tm_y)),
            "r"(n_out0 + b * 64), "r"(m0), "r"(smem_u32(sout + b * (BM * 128)))
            : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
  }
  TC_TS(4);
#ifdef TPP_DEBUG_STAMPS
  if (threadIdx.x == 32) {  // MMA lane: has 1, 2
    const int id = blockIdx.y * gridDim.x + blockIdx.x;
    g_tc_stamps[8 * id + 1] = st_[1]; g_tc_stamps[8 * id + 2] = st_[2];
  }
  if (threadIdx.x == 0) {
    const int id = blockIdx.y * gridDim.x + blockIdx.x;
    g_tc_stamps[8 * id] = st_[0]; g_tc_stamps[8 * id + 3] = st_[3]; g_tc_stamps[8 * id + 4] = st_[4];
  }
#endif
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, BN);
}

}  // namespace

#ifdef TPP_DEBUG_STAMPS
extern "C" void tpp_debug_stamps_tc(unsigned long long* host, int n) {
  cudaMemcpyFromSymbol(host, g_tc_stamps, sizeof(unsigned long long) * n);
}
#endif

int linear_tc(const void* x, int64_t ldx, const void* w, const void* bias, const void* residual,
              void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act, int dtype,
              cudaStream_t st) {
  TPP_REQUIRE(ldx % 8 == 0 && K % 8 == 0 && aligned16(x) && aligned16(w), TPP_ERR_ALIGN,
              "tensor-core path needs 16-byte aligned x/W rows (K and ldx multiples of 8)");
  const bool sw = act == TPP_ACT_SWIGLU;
  const int64_t wrows = sw ? 2 * N : N;
  CUtensorMap tx, tw;
  {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    uint64_t strides[1] = {(uint64_t)ldx * 2};
    uint32_t box[2] = {BK, BM};
    int rc = make_tmap(&tx, x, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != TPP_OK) return rc;
  }
  {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)wrows};
    uint64_t strides[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {BK, (uint32_t)(sw ? BN / 2 : BN)};
    int rc = make_tmap(&tw, w, dtype, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
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
  const int nout = sw ? BN / 2 : BN;
  dim3 grid((unsigned)((N + nout - 1) / nout), (unsigned)((M + BM - 1) / BM), 1);
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    auto kern = sw ? linear_tc_kernel<T, true> : linear_tc_kernel<T, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) !=
        cudaSuccess) {
      set_error("linear_tc_kernel: cannot reserve shared memory");
      return (int)TPP_ERR_LAUNCH;
    }
    return launch("linear_tc_kernel", kern, dim3(grid), dim3(kThreads), kSmem, st, 0, tx, tw, ty, a);
  });
}

}  // namespace tpp
