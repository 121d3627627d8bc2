// C-ABI entry points for linear layers: shape checks and the dispatch between
// the decode-shaped streaming kernel (M <= 64, linear_decode.cu) and the
// tcgen05 tensor-core GEMM (linear_tc.cu).
#include "common.cuh"

namespace tpp {
int linear_decode(const void* x, int64_t ldx, const void* w, const void* bias,
                  const void* residual, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                  int act, int dtype, cudaStream_t st, float norm_eps);
int linear_tc(const void* x, int64_t ldx, const void* w, const void* bias, const void* residual,
              void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act, int dtype,
              cudaStream_t st);
int64_t xs_packed_weight_bytes(int64_t N, int64_t K, int act);
int64_t xs_packed_activation_bytes(int64_t M, int64_t K);
int xs_pack_weight(const void* w, int64_t N, int64_t K, int act, void* dst, cudaStream_t st);
int xs_pack_activation(const void* x, int64_t ldx, int64_t M, int64_t K, void* dst,
                       cudaStream_t st);
int linear_xs_impl(const void* x, int64_t ldx, const void* w, const void* bias,
                   const void* residual, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                   int act, int dtype, cudaStream_t st, float norm_eps, const void* wpk,
                   const void* xpk, void* ypk);
int linear_xs_fp8(const void* x, int64_t ldx, const void* q, const float* scale,
                  const void* bias, const void* residual, void* y, int64_t ldy, int64_t M,
                  int64_t N, int64_t K, int act, int dtype, cudaStream_t st, float norm_eps);
int quantize_weight_fp8(const void* w, int64_t rows, int64_t K, int dtype, void* q, float* scale,
                        cudaStream_t st);
int dequantize_weight_fp8(const void* q, const float* scale, int64_t rows, int64_t K, int dtype,
                          void* w, cudaStream_t st);
constexpr int64_t kDecodeMaxM = 64;
}  // namespace tpp

using namespace tpp;

extern "C" int tpp_linear(const void* x, int64_t ldx, const void* w, const void* bias,
                          const void* residual, void* y, int64_t ldy, int64_t M, int64_t N,
                          int64_t K, int act, int dtype, void* stream) {
  if (M == 0) return TPP_OK;
  TPP_REQUIRE(x && w && y, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(M >= 0 && N > 0 && K > 0, TPP_ERR_SHAPE, "need M >= 0, N > 0, K > 0");
  TPP_REQUIRE(M <= 0x7fffffff && N <= 0x3fffffff && K <= 0x7fffffff, TPP_ERR_SHAPE,
              "sizes exceed 32-bit kernel indexing");
  TPP_REQUIRE(ldx >= K && ldy >= N, TPP_ERR_SHAPE, "row stride smaller than the row");
  TPP_REQUIRE(act >= TPP_ACT_NONE && act <= TPP_ACT_SWIGLU, TPP_ERR_UNSUPPORTED, "unknown activation");
  TPP_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && aligned16(x) && aligned16(w), TPP_ERR_ALIGN,
              "x and W rows must be 16-byte aligned (K and ldx multiples of 8)");
  if (M == 0) return TPP_OK;
  cudaStream_t st = as_stream(stream);
  if (M <= kDecodeMaxM)
    return linear_decode(x, ldx, w, bias, residual, y, ldy, M, N, K, act, dtype, st, -1.f);
  return linear_tc(x, ldx, w, bias, residual, y, ldy, M, N, K, act, dtype, st);
}

extern "C" int tpp_hgemv(const void* W, const void* x, void* y, int64_t N, int64_t K, int dtype,
                         void* stream) {
  return tpp_linear(x, K, W, nullptr, nullptr, y, N, 1, N, K, TPP_ACT_NONE, dtype, stream);
}

extern "C" int tpp_rmsnorm_linear(const void* x, int64_t ldx, const void* w_folded,
                                  const void* bias, const void* residual, void* y, int64_t ldy,
                                  int64_t M, int64_t N, int64_t K, float eps, int act, int dtype,
                                  void* stream) {
  if (M == 0) return TPP_OK;
  TPP_REQUIRE(x && w_folded && y, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(M > 0 && N > 0 && K > 0 && N <= 0x3fffffff && K <= 0x7fffffff, TPP_ERR_SHAPE,
              "bad sizes");
  TPP_REQUIRE(M <= kDecodeMaxM, TPP_ERR_UNSUPPORTED,
              "the fused norm+linear serves decode shapes (M <= 64); use tpp_rmsnorm + tpp_linear");
  TPP_REQUIRE(ldx >= K && ldy >= N && eps >= 0.f, TPP_ERR_SHAPE, "bad strides or eps");
  TPP_REQUIRE(act >= TPP_ACT_NONE && act <= TPP_ACT_SWIGLU, TPP_ERR_UNSUPPORTED, "unknown activation");
  TPP_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && aligned16(x) && aligned16(w_folded), TPP_ERR_ALIGN,
              "x and W rows must be 16-byte aligned (K and ldx multiples of 8)");
  return linear_decode(x, ldx, w_folded, bias, residual, y, ldy, M, N, K, act, dtype,
                       as_stream(stream), eps);
}

extern "C" int64_t tpp_packed_weight_bytes(int64_t N, int64_t K, int act) {
  if (N <= 0 || K <= 0 || N > 0x3fffffff || K > 0x7fffffff) return 0;
  return xs_packed_weight_bytes(N, K, act);
}

extern "C" int64_t tpp_packed_activation_bytes(int64_t M, int64_t K) {
  if (M <= 0 || M > 32 || K <= 0 || K > 0x7fffffff) return 0;
  return xs_packed_activation_bytes(M, K);
}

extern "C" int tpp_pack_weight(const void* w, int64_t N, int64_t K, int act, int dtype,
                               void* w_packed, void* stream) {
  TPP_REQUIRE(w && w_packed, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(dtype == TPP_F16 || dtype == TPP_BF16, TPP_ERR_DTYPE, "dtype must be f16 or bf16");
  TPP_REQUIRE(act >= TPP_ACT_NONE && act <= TPP_ACT_SWIGLU, TPP_ERR_UNSUPPORTED, "unknown activation");
  TPP_REQUIRE(tpp_packed_weight_bytes(N, K, act) > 0, TPP_ERR_UNSUPPORTED,
              "layer too wide for the packed form, or K not a multiple of 64");
  TPP_REQUIRE(aligned16(w) && aligned16(w_packed), TPP_ERR_ALIGN, "16-byte alignment required");
  return xs_pack_weight(w, N, K, act, w_packed, as_stream(stream));
}

extern "C" int tpp_pack_activation(const void* x, int64_t ldx, int64_t M, int64_t K, int dtype,
                                   void* x_packed, void* stream) {
  TPP_REQUIRE(x && x_packed, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(dtype == TPP_F16 || dtype == TPP_BF16, TPP_ERR_DTYPE, "dtype must be f16 or bf16");
  TPP_REQUIRE(tpp_packed_activation_bytes(M, K) > 0 && ldx >= K, TPP_ERR_SHAPE,
              "need 0 < M <= 32, K a multiple of 64, ldx >= K");
  TPP_REQUIRE(ldx % 8 == 0 && aligned16(x) && aligned16(x_packed), TPP_ERR_ALIGN,
              "16-byte alignment required");
  return xs_pack_activation(x, ldx, M, K, x_packed, as_stream(stream));
}

extern "C" int tpp_linear_packed(const void* x_packed, const void* w_packed, const void* bias,
                                 const void* residual, void* y, int64_t ldy, void* y_packed,
                                 int64_t M, int64_t N, int64_t K, float eps, int act, int dtype,
                                 void* stream) {
  TPP_REQUIRE(x_packed && w_packed && y, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(M > 0 && M <= 32 && ldy >= N, TPP_ERR_SHAPE, "need 0 < M <= 32, ldy >= N");
  TPP_REQUIRE(act >= TPP_ACT_NONE && act <= TPP_ACT_SWIGLU, TPP_ERR_UNSUPPORTED, "unknown activation");
  TPP_REQUIRE(tpp_packed_weight_bytes(N, K, act) > 0, TPP_ERR_UNSUPPORTED,
              "layer too wide for the packed form, or K not a multiple of 64");
  TPP_REQUIRE(aligned16(x_packed) && aligned16(w_packed), TPP_ERR_ALIGN, "16-byte alignment required");
  TPP_REQUIRE(!y_packed || (N % 64 == 0 && ldy % 8 == 0 && aligned16(y) && aligned16(y_packed) &&
                            (!residual || aligned16(residual))),
              TPP_ERR_ALIGN, "a packed output needs N % 64 == 0 and 16-byte aligned rows");
  return linear_xs_impl(nullptr, K, nullptr, bias, residual, y, ldy, M, N, K, act, dtype,
                        as_stream(stream), eps, w_packed, x_packed, y_packed);
}

extern "C" int tpp_quantize_weight_fp8(const void* w, int64_t rows, int64_t K, int dtype, void* q,
                                       float* scale, void* stream) {
  if (rows == 0) return TPP_OK;
  TPP_REQUIRE(w && q && scale, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(rows > 0 && rows <= 0x7fffffff && K > 0 && K <= 0x3fffffff && K % 64 == 0,
              TPP_ERR_SHAPE, "need rows > 0 and K a positive multiple of 64");
  TPP_REQUIRE(aligned16(w) && aligned16(q), TPP_ERR_ALIGN, "16-byte alignment required");
  return quantize_weight_fp8(w, rows, K, dtype, q, scale, as_stream(stream));
}

extern "C" int64_t tpp_fp8_weight_bytes(int64_t rows, int64_t K) {
  if (rows <= 0 || K <= 0 || K % 64 != 0 || rows > 0x7fffffff) return 0;
  return (rows + 31) / 32 * 32 * K;
}

extern "C" int tpp_dequantize_weight_fp8(const void* q, const float* scale, int64_t rows,
                                         int64_t K, int dtype, void* w, void* stream) {
  if (rows == 0) return TPP_OK;
  TPP_REQUIRE(w && q && scale, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(rows > 0 && K > 0 && K % 64 == 0 && rows * K < ((int64_t)1 << 46), TPP_ERR_SHAPE,
              "need rows > 0 and K a positive multiple of 64");
  return dequantize_weight_fp8(q, scale, rows, K, dtype, w, as_stream(stream));
}

extern "C" int tpp_linear_fp8(const void* x, int64_t ldx, const void* q, const float* scale,
                              const void* bias, const void* residual, void* y, int64_t ldy,
                              int64_t M, int64_t N, int64_t K, float eps, int act, int dtype,
                              void* stream) {
  if (M == 0) return TPP_OK;
  TPP_REQUIRE(x && q && scale && y, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(M > 0 && M <= 32, TPP_ERR_UNSUPPORTED,
              "fp8 decode linear serves 1..32 tokens (larger M: dequantize + tpp_linear)");
  TPP_REQUIRE(N > 0 && N <= 0x3fffffff && K > 0 && K <= 0x3fffffff && K % 64 == 0,
              TPP_ERR_SHAPE, "need N > 0 and K a positive multiple of 64");
  TPP_REQUIRE(ldx >= K && ldy >= N, TPP_ERR_SHAPE, "row stride smaller than the row");
  TPP_REQUIRE(act >= TPP_ACT_NONE && act <= TPP_ACT_SWIGLU, TPP_ERR_UNSUPPORTED, "unknown activation");
  TPP_REQUIRE(ldx % 8 == 0 && aligned16(x) && aligned16(q), TPP_ERR_ALIGN,
              "x rows and the fp8 weight must be 16-byte aligned");
  const int rc = linear_xs_fp8(x, ldx, q, scale, bias, residual, y, ldy, M, N, K, act, dtype,
                               as_stream(stream), eps);
  if (rc == -1) {
    set_error("tpp_linear_fp8: no launch plan for this shape");
    return TPP_ERR_UNSUPPORTED;
  }
  return rc;
}
