// Decode-shaped linear layers: y[M,N] = epilogue(x[M,K] . W[N,K]^T) for M <= 64.
//
// At decode the weight matrix is read exactly once per step and the token
// count is tiny, so the kernel is bound by HBM bandwidth on W.  Design:
//  * A warp owns 16 weight rows (the M side of an m16n8k16 tensor-core MMA;
//    tokens are the N side, 8 per MMA tile).  W is streamed straight from HBM
//    into registers with 16-byte evict-first loads; no shared-memory staging.
//  * K is processed in 64-element chunks.  Lane (g, c) of the warp loads
//    elements [16c, 16c+16) of the chunk for rows g and g+8, i.e. a whole
//    128-byte line per row per chunk.  Those 16 physical k are assigned to the
//    MMA's logical k slots by a fixed permutation that depends on c only, and
//    the activation fragment (x) is loaded with the same permutation, so the
//    dot product is unchanged (a sum over k is order independent).
//  * K is split across the 8 warps of a CTA and, for short-and-wide matrices,
//    across the CTAs of a thread-block cluster (up to 8).  Partial tiles are
//    reduced in shared memory and then over distributed shared memory into
//    the cluster's rank-0 CTA, which runs the fused epilogue (bias,
//    activation, SwiGLU gate*up, residual add).  No global scratch.
// Reference: the unbuilt hgemv kernels csrc/blas/hgemv/hgemv_kernels.cuh:19-85
// (one warp per row, fp16 accumulation) and the CUTLASS fused linear of
// csrc/activation/fused_gemm.cuh:143-170 (128x128 tiles, which waste >= 75% of
// the MMA at M <= 32).  Accumulation here is fp32.
#include <cooperative_groups.h>
#include "common.cuh"

namespace cg = cooperative_groups;

namespace tpp {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

template <typename T>
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float* d, const uint32_t* a, uint32_t b0,
                                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* d, const uint32_t* a, uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pick(const uint4& lo, const uint4& hi, int i) {
  switch (i) {
    case 0: return lo.x; case 1: return lo.y; case 2: return lo.z; case 3: return lo.w;
    case 4: return hi.x; case 5: return hi.y; case 6: return hi.z; default: return hi.w;
  }
}

struct LinearArgs {
  const void* x; int64_t ldx;
  const void* w;
  const void* bias;
  const void* residual;
  void* y; int64_t ldy;
  int M, N, K;
  int act;
  int chunks_per_split;  // 64-element K chunks per (warp, cluster-rank) split
};

// NRG: row sets per CTA (1, or 2 for SwiGLU gate+up). MT: 8-token MMA tiles.
template <typename T, int NRG, int MT, bool V8>
__global__ void __launch_bounds__(kThreads) linear_decode_kernel(LinearArgs p) {
  constexpr int WK = kWarps / NRG;  // warps along K per row set
  constexpr int TOK = MT * 8;
  extern __shared__ float smem[];
  float* part = smem;                              // [kWarps][16][TOK]
  float* red = smem + kWarps * 16 * TOK;           // [NRG][16][TOK]

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rs = warp / WK;       // row set (0 = plain/gate, 1 = up)
  const int wk = warp % WK;
  const int row_base = blockIdx.x * 16 + (rs ? p.N : 0);
  const int rows_total = NRG == 2 ? 2 * p.N : p.N;
  const int ra = blockIdx.x * 16 + g;  // row within the set
  const int rowA = row_base + g, rowB = row_base + g + 8;
  const bool okA = ra < p.N, okB = ra + 8 < p.N;
  (void)rows_total;

  const T* W = static_cast<const T*>(p.w);
  const T* X = static_cast<const T*>(p.x);
  const int nchunks = (p.K + 63) >> 6;
  const int split = crank * WK + wk;
  const int c0 = split * p.chunks_per_split;
  const int c1 = min(nchunks, c0 + p.chunks_per_split);

  float acc[MT][4];
#pragma unroll
  for (int t = 0; t < MT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

  const T* wA = W + (int64_t)rowA * p.K;
  const T* wB = W + (int64_t)rowB * p.K;
  const uint4 z = make_uint4(0, 0, 0, 0);

  constexpr int U = 2;  // chunks in flight per iteration
  for (int j0 = c0; j0 < c1; j0 += U) {
    uint4 a[U][4];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u;
      const int k = j * 64 + c * 16;
      const bool in = j < c1;
      const bool k0 = in && k < p.K, k1 = in && k + 8 < p.K;
      if (V8 && k1) {
        // whole 32-byte run in range: one 256-bit load per row
        if (okA) ldg_stream_v8(wA + k, a[u][0], a[u][1]); else { a[u][0] = z; a[u][1] = z; }
        if (okB) ldg_stream_v8(wB + k, a[u][2], a[u][3]); else { a[u][2] = z; a[u][3] = z; }
      } else {
        a[u][0] = (okA && k0) ? ldg_nc_v4(wA + k) : z;
        a[u][1] = (okA && k1) ? ldg_nc_v4(wA + k + 8) : z;
        a[u][2] = (okB && k0) ? ldg_nc_v4(wB + k) : z;
        a[u][3] = (okB && k1) ? ldg_nc_v4(wB + k + 8) : z;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u;
      if (j >= c1) break;
      const int k = j * 64 + c * 16;
      const bool k0 = k < p.K, k1 = k + 8 < p.K;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int tok = t * 8 + g;
        uint4 blo = z, bhi = z;
        if (tok < p.M) {
          const T* xr = X + (int64_t)tok * p.ldx + k;
          if (k0) blo = __ldg(reinterpret_cast<const uint4*>(xr));
          if (k1) bhi = __ldg(reinterpret_cast<const uint4*>(xr + 8));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t af[4];
          af[0] = pick(a[u][0], a[u][1], 2 * q);
          af[1] = pick(a[u][2], a[u][3], 2 * q);
          af[2] = pick(a[u][0], a[u][1], 2 * q + 1);
          af[3] = pick(a[u][2], a[u][3], 2 * q + 1);
          mma16816<T>(acc[t], af, pick(blo, bhi, 2 * q), pick(blo, bhi, 2 * q + 1));
        }
      }
    }
  }

  // ---- reduction: warps -> CTA -> cluster rank 0 ----
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    float* pw = part + warp * 16 * TOK;
    pw[g * TOK + t * 8 + 2 * c] = acc[t][0];
    pw[g * TOK + t * 8 + 2 * c + 1] = acc[t][1];
    pw[(g + 8) * TOK + t * 8 + 2 * c] = acc[t][2];
    pw[(g + 8) * TOK + t * 8 + 2 * c + 1] = acc[t][3];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < NRG * 16 * TOK; e += kThreads) {
    const int s = e / (16 * TOK);
    const int off = e % (16 * TOK);
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < WK; ++w) v += part[(s * WK + w) * 16 * TOK + off];
    red[e] = v;
  }
  if (csize > 1) {
    cluster.sync();
    if (crank == 0) {
      for (int r = 1; r < csize; ++r) {
        const float* peer = cluster.map_shared_rank(red, r);
        for (int e = threadIdx.x; e < NRG * 16 * TOK; e += kThreads) red[e] += peer[e];
      }
    }
    cluster.sync();  // peers keep their shared memory alive until rank 0 has read it
    if (crank != 0) return;
  } else {
    __syncthreads();
  }

  // ---- epilogue (rank 0): token-major so 16 consecutive rows are contiguous ----
  const T* bias = static_cast<const T*>(p.bias);
  const T* res = static_cast<const T*>(p.residual);
  T* Y = static_cast<T*>(p.y);
  for (int e = threadIdx.x; e < 16 * TOK; e += kThreads) {
    const int tok = e / 16, r = e % 16;
    const int n = blockIdx.x * 16 + r;
    if (tok >= p.M || n >= p.N) continue;
    float v = red[r * TOK + tok];
    if (NRG == 2) {
      float u = red[16 * TOK + r * TOK + tok];
      if (bias) { v += to_f32(bias[n]); u += to_f32(bias[p.N + n]); }
      v = act_silu(v) * u;
    } else {
      if (bias) v += to_f32(bias[n]);
      v = apply_act(p.act, v);
    }
    if (res) v += to_f32(res[(int64_t)tok * p.ldy + n]);
    Y[(int64_t)tok * p.ldy + n] = from_f32<T>(v);
  }
}

template <typename T, int NRG, int MT>
int launch_linear_decode(const LinearArgs& a0, cudaStream_t st) {
  LinearArgs a = a0;
  const int nrb = (a.N + 15) / 16;
  const int nchunks = (a.K + 63) / 64;
  constexpr int WK = kWarps / NRG;
  // Enough CTAs to keep every SM streaming, but each split gets >= 1 chunk.
  const int target = 2 * num_sms();
  int ck = (target + nrb - 1) / nrb;
  ck = ck < 1 ? 1 : (ck > 8 ? 8 : ck);
  while (ck > 1 && ck * WK > nchunks) --ck;
  const int splits = ck * WK;
  a.chunks_per_split = (nchunks + splits - 1) / splits;
  const size_t smem = (size_t)(kWarps * 16 * MT * 8 + NRG * 16 * MT * 8) * sizeof(float);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nrb, (unsigned)ck, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)ck;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // 256-bit weight loads need 32-byte aligned rows.
  const bool v8 = (a.K % 16 == 0) && ((reinterpret_cast<uintptr_t>(a.w) & 31u) == 0);
  cudaError_t e = v8 ? cudaLaunchKernelEx(&cfg, linear_decode_kernel<T, NRG, MT, true>, a)
                     : cudaLaunchKernelEx(&cfg, linear_decode_kernel<T, NRG, MT, false>, a);
  if (e != cudaSuccess) {
    set_error(std::string("linear_decode_kernel: ") + cudaGetErrorString(e));
    return TPP_ERR_LAUNCH;
  }
  return check_launch("linear_decode_kernel");
}

template <typename T>
int linear_decode_dispatch(const LinearArgs& a, cudaStream_t st) {
  const bool sw = a.act == TPP_ACT_SWIGLU;
  auto go = [&](auto mt) -> int {
    constexpr int MT = decltype(mt)::value;
    return sw ? launch_linear_decode<T, 2, MT>(a, st) : launch_linear_decode<T, 1, MT>(a, st);
  };
  if (a.M <= 8) return go(std::integral_constant<int, 1>{});
  if (a.M <= 16) return go(std::integral_constant<int, 2>{});
  if (a.M <= 32) return go(std::integral_constant<int, 4>{});
  return go(std::integral_constant<int, 8>{});
}

}  // namespace

// Entry used by tpp_linear (linear.cu) for M <= 64.
int linear_decode(const void* x, int64_t ldx, const void* w, const void* bias,
                  const void* residual, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                  int act, int dtype, cudaStream_t st) {
  LinearArgs a;
  a.x = x; a.ldx = ldx; a.w = w; a.bias = bias; a.residual = residual; a.y = y; a.ldy = ldy;
  a.M = (int)M; a.N = (int)N; a.K = (int)K; a.act = act; a.chunks_per_split = 0;
  return TPP_DISPATCH_HALF(dtype, T, [&] { return linear_decode_dispatch<T>(a, st); });
}

}  // namespace tpp
