// RMSNorm / fused add+RMSNorm / LayerNorm for fp16 and bf16 rows.
//
// Reference semantics: csrc/dlops/rmsnorm/rmsnorm_fp16.cuh:43-115 (fp32 sum of
// squares, x * rsqrt(mean + eps) * gamma, fp32 until the final store) and
// csrc/dlops/layernorm/layernorm_fp16.cuh:46-144 (mean/var normalisation with
// gamma, no beta).  Design here: a row is held in registers by a group of G
// lanes (G <= 32) using 16-byte loads; statistics are reduced with warp
// shuffles only (no shared memory, no __syncthreads).  The LayerNorm variance
// is computed two-pass from the register copy (sum (x-mean)^2) instead of the
// reference's E[x^2]-mean^2, which cancels badly for large means.  Rows whose
// width is not a multiple of 8 elements or whose pointers are not 16-byte
// aligned take a generic block-per-row path.
#include "common.cuh"

namespace tpp {
namespace {

template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// MODE 0: rmsnorm, 1: add+rmsnorm (res in/out), 2: layernorm
template <typename T, int G, int NV, int MODE>
__global__ void __launch_bounds__(256) norm_rows_kernel(
    const T* __restrict__ x, int64_t ldx, T* res, const T* __restrict__ w,
    const T* __restrict__ b, T* __restrict__ y, int64_t ldy, int64_t rows, int cols,
    float eps) {
  const int groups = blockDim.x / G;
  const int64_t row = (int64_t)blockIdx.x * groups + threadIdx.x / G;
  const int lane = threadIdx.x % G;
  const bool valid_row = row < rows;
  const int nvec = cols >> 3;
  // gamma (and beta) do not depend on the previous kernel: requested before
  // the dependency wait, so they are not a round trip after the reduction
  uint4 gw[NV], bw[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * G;
    const bool in = valid_row && c < nvec;
    gw[i] = in ? __ldg(reinterpret_cast<const uint4*>(w) + c) : make_uint4(0, 0, 0, 0);
    bw[i] = in && MODE == 2 && b != nullptr ? __ldg(reinterpret_cast<const uint4*>(b) + c)
                                            : make_uint4(0, 0, 0, 0);
  }
  pdl_wait();
  pdl_trigger();

  float v[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * G;
    if (valid_row && c < nvec) {
      uint4 u;
      if (MODE == 1 && x == nullptr) {
        u = make_uint4(0, 0, 0, 0);
      } else {
        u = ldg_nc_v4(x + row * ldx + (int64_t)c * 8);
      }
      unpack8<T>(u, v[i]);
      if (MODE == 1) {
        float r[8];
        T* rp = res + row * ldx + (int64_t)c * 8;
        unpack8<T>(*reinterpret_cast<const uint4*>(rp), r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        // The residual stream keeps the dtype-rounded sum; normalise that.
        uint4 packed = pack8<T>(v[i]);
        *reinterpret_cast<uint4*>(rp) = packed;
        unpack8<T>(packed, v[i]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    }
  }

  float mean = 0.f;
  if (MODE == 2) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[i][j];
    mean = group_sum<G>(s) / (float)cols;
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * G;
    if (c < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[i][j] - mean;
        ss += d * d;
      }
    }
  }
  ss = group_sum<G>(ss);
  const float inv = rsqrtf(ss / (float)cols + eps);
  if (!valid_row) return;

#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * G;
    if (c < nvec) {
      float g[8], o[8], bb[8];
      unpack8<T>(gw[i], g);
      unpack8<T>(bw[i], bb);  // zeros without a beta
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (v[i][j] - mean) * inv * g[j] + bb[j];
      *reinterpret_cast<uint4*>(y + row * ldy + (int64_t)c * 8) = pack8<T>(o);
    }
  }
}

// Generic path: one 256-thread block per row, scalar accesses, any width.
template <typename T, int MODE>
__global__ void __launch_bounds__(256) norm_rows_generic_kernel(
    const T* __restrict__ x, int64_t ldx, T* res, const T* __restrict__ w,
    const T* __restrict__ b, T* __restrict__ y, int64_t ldy, int64_t rows, int cols,
    float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  auto block_sum = [&](float v) -> float {
    v = warp_sum(v);
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = v;
    __syncthreads();
    float t = (tid < (int)(blockDim.x >> 5)) ? red[tid] : 0.f;
    if (tid < 32) t = warp_sum(t);
    if (tid == 0) red[0] = t;
    __syncthreads();
    return red[0];
  };
  if (MODE == 1) {
    for (int c = tid; c < cols; c += blockDim.x) {
      float s = to_f32(res[row * ldx + c]) + (x ? to_f32(x[row * ldx + c]) : 0.f);
      res[row * ldx + c] = from_f32<T>(s);
    }
    __syncthreads();
  }
  const T* src = (MODE == 1) ? res : x;
  float mean = 0.f;
  if (MODE == 2) {
    float s = 0.f;
    for (int c = tid; c < cols; c += blockDim.x) s += to_f32(src[row * ldx + c]);
    mean = block_sum(s) / (float)cols;
  }
  float ss = 0.f;
  for (int c = tid; c < cols; c += blockDim.x) {
    const float d = to_f32(src[row * ldx + c]) - mean;
    ss += d * d;
  }
  const float inv = rsqrtf(block_sum(ss) / (float)cols + eps);
  for (int c = tid; c < cols; c += blockDim.x) {
    float o = (to_f32(src[row * ldx + c]) - mean) * inv * to_f32(w[c]);
    if (MODE == 2 && b != nullptr) o += to_f32(b[c]);
    y[row * ldy + c] = from_f32<T>(o);
  }
}

template <typename T, int G, int NV, int MODE>
int launch_rows(const T* x, int64_t ldx, T* res, const T* w, const T* b, T* y, int64_t ldy,
                int64_t rows, int cols, float eps, cudaStream_t st) {
  const int threads = 256;
  const int groups = threads / G;
  const int64_t grid = (rows + groups - 1) / groups;
  return launch("norm_rows_kernel", norm_rows_kernel<T, G, NV, MODE>, dim3((unsigned)grid), dim3(threads), 0, st, 0, x, ldx, res, w, b, y, ldy,
                                                                       rows, cols, eps);
}

template <typename T, int MODE>
int norm_dispatch(const void* xv, int64_t ldx, void* resv, const void* wv, const void* bv,
                  void* yv, int64_t ldy, int64_t rows, int64_t cols, float eps,
                  cudaStream_t st) {
  const T* x = static_cast<const T*>(xv);
  T* res = static_cast<T*>(resv);
  const T* w = static_cast<const T*>(wv);
  const T* b = static_cast<const T*>(bv);
  T* y = static_cast<T*>(yv);
  if (rows == 0) return TPP_OK;
  const bool vec_ok = (cols % 8 == 0) && (ldx % 8 == 0) && (ldy % 8 == 0) &&
                      (x == nullptr || aligned16(x)) && (res == nullptr || aligned16(res)) &&
                      aligned16(w) && (b == nullptr || aligned16(b)) && aligned16(y);
  const int nvec = (int)(cols / 8);
  if (vec_ok && cols <= 4096) {
    if (nvec <= 4) return launch_rows<T, 4, 1, MODE>(x, ldx, res, w, b, y, ldy, rows, (int)cols, eps, st);
    if (nvec <= 8) return launch_rows<T, 8, 1, MODE>(x, ldx, res, w, b, y, ldy, rows, (int)cols, eps, st);
    if (nvec <= 16) return launch_rows<T, 16, 1, MODE>(x, ldx, res, w, b, y, ldy, rows, (int)cols, eps, st);
    if (nvec <= 32) return launch_rows<T, 32, 1, MODE>(x, ldx, res, w, b, y, ldy, rows, (int)cols, eps, st);
    if (nvec <= 64) return launch_rows<T, 32, 2, MODE>(x, ldx, res, w, b, y, ldy, rows, (int)cols, eps, st);
    if (nvec <= 128) return launch_rows<T, 32, 4, MODE>(x, ldx, res, w, b, y, ldy, rows, (int)cols, eps, st);
    if (nvec <= 256) return launch_rows<T, 32, 8, MODE>(x, ldx, res, w, b, y, ldy, rows, (int)cols, eps, st);
    return launch_rows<T, 32, 16, MODE>(x, ldx, res, w, b, y, ldy, rows, (int)cols, eps, st);
  }
  TPP_REQUIRE(rows <= 0x7fffffffLL, TPP_ERR_SHAPE, "too many rows for the generic path");
  return launch("norm_rows_generic_kernel", norm_rows_generic_kernel<T, MODE>, dim3((unsigned)rows), dim3(256), 0, st, 0, x, ldx, res, w, b, y, ldy, rows,
                                                                    (int)cols, eps);
}

}  // namespace
}  // namespace tpp

using namespace tpp;

extern "C" int tpp_rmsnorm(const void* x, int64_t x_row_stride, const void* w, void* y,
                           int64_t y_row_stride, int64_t rows, int64_t cols, float eps,
                           int dtype, void* stream) {
  if (rows == 0) return TPP_OK;
  TPP_REQUIRE(x && w && y, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(rows >= 0 && cols > 0 && cols <= 0x7fffffff, TPP_ERR_SHAPE, "bad rows/cols");
  TPP_REQUIRE(x_row_stride >= cols && y_row_stride >= cols, TPP_ERR_SHAPE, "row stride < cols");
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return norm_dispatch<T, 0>(x, x_row_stride, nullptr, w, nullptr, y, y_row_stride, rows, cols,
                               eps, as_stream(stream));
  });
}

extern "C" int tpp_add_rmsnorm(const void* x, void* res, const void* w, void* y, int64_t rows,
                               int64_t cols, float eps, int dtype, void* stream) {
  if (rows == 0) return TPP_OK;
  TPP_REQUIRE(res && w && y, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(rows >= 0 && cols > 0 && cols <= 0x7fffffff, TPP_ERR_SHAPE, "bad rows/cols");
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return norm_dispatch<T, 1>(x, cols, res, w, nullptr, y, cols, rows, cols, eps,
                               as_stream(stream));
  });
}

extern "C" int tpp_layernorm(const void* x, const void* w, const void* b, void* y, int64_t rows,
                             int64_t cols, float eps, int dtype, void* stream) {
  if (rows == 0) return TPP_OK;
  TPP_REQUIRE(x && w && y, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(rows >= 0 && cols > 0 && cols <= 0x7fffffff, TPP_ERR_SHAPE, "bad rows/cols");
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return norm_dispatch<T, 2>(x, cols, nullptr, w, b, y, cols, rows, cols, eps,
                               as_stream(stream));
  });
}
