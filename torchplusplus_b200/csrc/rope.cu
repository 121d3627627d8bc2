// Rotary position embedding (NeoX rotate-half form), its Q+K variant, the
// fused decode-step q/k-norm + RoPE + KV-cache append, and the plain KV append.
//
// Reference semantics: csrc/dlops/rope/apply_rope.cuh:4-47 computes
// out = x*cos + rotate_half(x)*sin with rotate_half(x) = cat(-x[D/2:], x[:D/2]),
// cos/sin tables [S,D] from torchpp/dlops/rope.py:43-54.  The reference does the
// arithmetic in fp16 (__hmul/__hadd); here it is fp32 with one rounding at the
// store.  One thread owns 8 elements of the first half and the matching 8 of
// the second half, so every load/store is a 16-byte vector.
#include "common.cuh"

namespace tpp {
namespace {

template <typename CS>
__device__ __forceinline__ void load_cs8(const CS* p, float* f);
template <>
__device__ __forceinline__ void load_cs8<__half>(const __half* p, float* f) {
  unpack8<__half>(__ldg(reinterpret_cast<const uint4*>(p)), f);
}
template <>
__device__ __forceinline__ void load_cs8<__nv_bfloat16>(const __nv_bfloat16* p, float* f) {
  unpack8<__nv_bfloat16>(__ldg(reinterpret_cast<const uint4*>(p)), f);
}
template <>
__device__ __forceinline__ void load_cs8<float>(const float* p, float* f) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p));
  float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Rotates the 8-element chunk pair (lo at d0, hi at d0 + D/2) in place.
template <typename CS>
__device__ __forceinline__ void rotate8(float* lo, float* hi, const CS* cos_row,
                                        const CS* sin_row, int d0, int half) {
  float cl[8], sl[8], ch[8], sh[8];
  load_cs8<CS>(cos_row + d0, cl);
  load_cs8<CS>(sin_row + d0, sl);
  load_cs8<CS>(cos_row + d0 + half, ch);
  load_cs8<CS>(sin_row + d0 + half, sh);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float a = lo[j], b = hi[j];
    lo[j] = a * cl[j] - b * sl[j];
    hi[j] = b * ch[j] + a * sh[j];
  }
}

// x: [B,H,S,D] strided (D contiguous); out contiguous [B,H,S,D].
template <typename T, typename CS>
__global__ void __launch_bounds__(256) rope_vec_kernel(
    const T* __restrict__ x, int64_t sb, int64_t sh, int64_t ss, const CS* __restrict__ cosp,
    const CS* __restrict__ sinp, int64_t cs_stride, T* __restrict__ out, int64_t H, int64_t S,
    int D, int64_t pos_offset, int64_t total) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int chunks = D >> 4;  // 8-element chunks per half
  const int c = (int)(idx % chunks);
  const int64_t row = idx / chunks;  // (b, h, s)
  const int64_t s = row % S;
  const int64_t bh = row / S;
  const int64_t h = bh % H;
  const int64_t b = bh / H;
  const int half = D >> 1;
  const int d0 = c * 8;
  const T* xr = x + b * sb + h * sh + s * ss;
  float lo[8], hi[8];
  unpack8<T>(ldg_nc_v4(xr + d0), lo);
  unpack8<T>(ldg_nc_v4(xr + d0 + half), hi);
  const int64_t crow = (s + pos_offset) * cs_stride;
  rotate8<CS>(lo, hi, cosp + crow, sinp + crow, d0, half);
  T* orow = out + row * D;
  *reinterpret_cast<uint4*>(orow + d0) = pack8<T>(lo);
  *reinterpret_cast<uint4*>(orow + d0 + half) = pack8<T>(hi);
}

// Scalar fallback for odd head dims / unaligned pointers.
template <typename T, typename CS>
__global__ void __launch_bounds__(256) rope_scalar_kernel(
    const T* __restrict__ x, int64_t sb, int64_t sh, int64_t ss, const CS* __restrict__ cosp,
    const CS* __restrict__ sinp, int64_t cs_stride, T* __restrict__ out, int64_t H, int64_t S,
    int D, int64_t pos_offset, int64_t total) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int half = D >> 1;
  const int d = (int)(idx % half);
  const int64_t row = idx / half;
  const int64_t s = row % S;
  const int64_t bh = row / S;
  const int64_t h = bh % H;
  const int64_t b = bh / H;
  const T* xr = x + b * sb + h * sh + s * ss;
  const float a = to_f32(xr[d]), bb = to_f32(xr[d + half]);
  const int64_t crow = (s + pos_offset) * cs_stride;
  const float lo = a * to_f32(cosp[crow + d]) - bb * to_f32(sinp[crow + d]);
  const float hi = bb * to_f32(cosp[crow + d + half]) + a * to_f32(sinp[crow + d + half]);
  out[row * D + d] = from_f32<T>(lo);
  out[row * D + d + half] = from_f32<T>(hi);
}

template <typename T, typename CS>
int rope_launch(const T* x, int64_t sb, int64_t sh, int64_t ss, const CS* c, const CS* s,
                int64_t cs_stride, T* out, int64_t B, int64_t H, int64_t S, int64_t D,
                int64_t pos_offset, cudaStream_t st) {
  const bool vec = (D % 16 == 0) && sb % 8 == 0 && sh % 8 == 0 && ss % 8 == 0 &&
                   cs_stride % 8 == 0 && aligned16(x) && aligned16(out) && aligned16(c) &&
                   aligned16(s);
  const int64_t rows = B * H * S;
  if (rows == 0) return TPP_OK;
  if (vec) {
    const int64_t total = rows * (D / 16);
    const int64_t grid = (total + 255) / 256;
    return launch("rope_vec_kernel", rope_vec_kernel<T, CS>, dim3((unsigned)grid), dim3(256), 0, st, 0, x, sb, sh, ss, c, s, cs_stride, out, H,
                                                          S, (int)D, pos_offset, total);
  }
  const int64_t total = rows * (D / 2);
  const int64_t grid = (total + 255) / 256;
  return launch("rope_scalar_kernel", rope_scalar_kernel<T, CS>, dim3((unsigned)grid), dim3(256), 0, st, 0, x, sb, sh, ss, c, s, cs_stride, out,
                                                           H, S, (int)D, pos_offset, total);
}

template <typename T>
int rope_cs_dispatch(int cs_dtype, const void* x, int64_t sb, int64_t sh, int64_t ss,
                     const void* c, const void* s, int64_t cs_stride, void* out, int64_t B,
                     int64_t H, int64_t S, int64_t D, int64_t pos_offset, cudaStream_t st) {
  const T* xt = static_cast<const T*>(x);
  T* ot = static_cast<T*>(out);
  switch (cs_dtype) {
    case TPP_F16:
      return rope_launch<T, __half>(xt, sb, sh, ss, (const __half*)c, (const __half*)s, cs_stride,
                                    ot, B, H, S, D, pos_offset, st);
    case TPP_BF16:
      return rope_launch<T, __nv_bfloat16>(xt, sb, sh, ss, (const __nv_bfloat16*)c,
                                           (const __nv_bfloat16*)s, cs_stride, ot, B, H, S, D,
                                           pos_offset, st);
    case TPP_F32:
      return rope_launch<T, float>(xt, sb, sh, ss, (const float*)c, (const float*)s, cs_stride, ot,
                                   B, H, S, D, pos_offset, st);
    default:
      set_error("tpp_rope: cos/sin dtype must be f16, bf16 or f32");
      return TPP_ERR_DTYPE;
  }
}

// ---------------------------------------------------------------------------
// Fused q/k RMSNorm + RoPE + KV append.  A group of G = D/8 lanes owns one
// (token, head) row; lane l holds elements [8l, 8l+8).  The rotate-half
// partner chunk lives in lane l ^ (G/2) and is fetched with shuffles.
// ---------------------------------------------------------------------------
template <typename T, typename CS, int G>
__global__ void __launch_bounds__(256) qk_norm_rope_cache_kernel(
    const T* __restrict__ qkv, int64_t ld_qkv, const T* __restrict__ qn_w,
    const T* __restrict__ kn_w, float eps, const CS* __restrict__ cosp,
    const CS* __restrict__ sinp, int64_t cs_stride, const int32_t* __restrict__ positions,
    T* __restrict__ q_out, T* __restrict__ k_cache, T* __restrict__ v_cache, int64_t c_sb,
    int64_t c_sh, int64_t c_ss, int64_t B, int64_t S, int Hq, int Hkv, int D) {
  pdl_wait();
  pdl_trigger();
  const int groups_per_block = blockDim.x / G;
  const int heads = Hq + 2 * Hkv;
  const int64_t item = (int64_t)blockIdx.x * groups_per_block + threadIdx.x / G;
  const int lane = threadIdx.x % G;
  const int64_t total = B * S * heads;
  const bool valid = item < total;
  const int64_t it = valid ? item : 0;
  const int h = (int)(it % heads);
  const int64_t tok = it / heads;  // b * S + s
  const int64_t s = tok % S;
  const int64_t b = tok / S;
  const T* src = qkv + tok * ld_qkv + (int64_t)h * D + lane * 8;
  float v[8];
  unpack8<T>(ldg_nc_v4(src), v);
  const bool is_q = h < Hq;
  const bool is_k = !is_q && h < Hq + Hkv;
  const int64_t pos = (int64_t)positions[b] + s;
  // Every lane takes part in the shuffles below (a warp can hold groups of
  // different head kinds), only the arithmetic is predicated.
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const T* nw = is_q ? qn_w : (is_k ? kn_w : nullptr);
  if (nw != nullptr) {
    const float inv = rsqrtf(ss / (float)D + eps);
    float g[8];
    unpack8<T>(__ldg(reinterpret_cast<const uint4*>(nw) + lane), g);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = v[j] * inv * g[j];
  }
  float p[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) p[j] = __shfl_xor_sync(0xffffffffu, v[j], G / 2);
  if (is_q || is_k) {
    const bool first_half = lane < G / 2;
    const int d0 = lane * 8;
    float c8[8], s8[8];
    load_cs8<CS>(cosp + pos * cs_stride + d0, c8);
    load_cs8<CS>(sinp + pos * cs_stride + d0, s8);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // first half: x1*cos - x2*sin ; second half: x2*cos + x1*sin
      v[j] = first_half ? (v[j] * c8[j] - p[j] * s8[j]) : (v[j] * c8[j] + p[j] * s8[j]);
    }
  }
  if (!valid) return;
  const uint4 packed = pack8<T>(v);
  if (is_q) {
    T* dst = q_out + (tok * Hq + h) * (int64_t)D + lane * 8;
    *reinterpret_cast<uint4*>(dst) = packed;
  } else if (is_k) {
    T* dst = k_cache + b * c_sb + (int64_t)(h - Hq) * c_sh + pos * c_ss + lane * 8;
    *reinterpret_cast<uint4*>(dst) = packed;
  } else {
    T* dst = v_cache + b * c_sb + (int64_t)(h - Hq - Hkv) * c_sh + pos * c_ss + lane * 8;
    *reinterpret_cast<uint4*>(dst) = packed;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) kv_append_kernel(
    const T* __restrict__ k, int64_t k_sb, int64_t k_sh, int64_t k_ss, const T* __restrict__ v,
    int64_t v_sb, int64_t v_sh, int64_t v_ss, T* __restrict__ kc, T* __restrict__ vc,
    int64_t c_sb, int64_t c_sh, int64_t c_ss, int64_t Hkv, int64_t S, int D, int64_t start_pos,
    const int32_t* __restrict__ positions, int64_t total, bool vec) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int per_row = vec ? D / 8 : D;
  const int c = (int)(idx % per_row);
  const int64_t row = idx / per_row;
  const int64_t s = row % S;
  const int64_t bh = row / S;
  const int64_t h = bh % Hkv;
  const int64_t b = bh / Hkv;
  const int64_t pos = (positions ? (int64_t)positions[b] : start_pos) + s;
  const int64_t ko = b * k_sb + h * k_sh + s * k_ss;
  const int64_t vo = b * v_sb + h * v_sh + s * v_ss;
  const int64_t co = b * c_sb + h * c_sh + pos * c_ss;
  if (vec) {
    reinterpret_cast<uint4*>(kc + co)[c] = reinterpret_cast<const uint4*>(k + ko)[c];
    reinterpret_cast<uint4*>(vc + co)[c] = reinterpret_cast<const uint4*>(v + vo)[c];
  } else {
    kc[co + c] = k[ko + c];
    vc[co + c] = v[vo + c];
  }
}

}  // namespace
}  // namespace tpp

using namespace tpp;

extern "C" int tpp_rope(const void* x, int64_t sb, int64_t sh, int64_t ss, const void* cos,
                        const void* sin, int64_t cs_stride, int cs_dtype, void* out, int64_t B,
                        int64_t H, int64_t S, int64_t D, int64_t pos_offset, int dtype,
                        void* stream) {
  if (B * H * S == 0) return TPP_OK;
  TPP_REQUIRE(x && cos && sin && out, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(B >= 0 && H >= 0 && S >= 0 && D > 0 && D % 2 == 0, TPP_ERR_SHAPE,
              "head dim must be even and sizes non-negative");
  TPP_REQUIRE(pos_offset >= 0 && cs_stride >= D, TPP_ERR_SHAPE, "bad cos/sin table stride/offset");
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return rope_cs_dispatch<T>(cs_dtype, x, sb, sh, ss, cos, sin, cs_stride, out, B, H, S, D,
                               pos_offset, as_stream(stream));
  });
}

extern "C" int tpp_qkrope(const void* q, const void* k, const void* cos, const void* sin,
                          int64_t cs_stride, int cs_dtype, void* q_out, void* k_out, int64_t B,
                          int64_t Hq, int64_t Hk, int64_t S, int64_t D, int64_t pos_offset,
                          int dtype, void* stream) {
  if (B * S == 0) return TPP_OK;
  TPP_REQUIRE(q && k && cos && sin && q_out && k_out, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(B >= 0 && Hq >= 0 && Hk >= 0 && S >= 0 && D > 0 && D % 2 == 0, TPP_ERR_SHAPE,
              "head dim must be even and sizes non-negative");
  TPP_REQUIRE(pos_offset >= 0 && cs_stride >= D, TPP_ERR_SHAPE, "bad cos/sin table stride/offset");
  // Two launches on the same stream: Q rows then K rows.  (One fused launch
  // would save a few microseconds; Q and K are independent and each launch
  // already fills the GPU at prefill sizes.)
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    int st = rope_cs_dispatch<T>(cs_dtype, q, Hq * S * D, S * D, D, cos, sin, cs_stride, q_out, B,
                                 Hq, S, D, pos_offset, as_stream(stream));
    if (st != TPP_OK) return st;
    return rope_cs_dispatch<T>(cs_dtype, k, Hk * S * D, S * D, D, cos, sin, cs_stride, k_out, B,
                               Hk, S, D, pos_offset, as_stream(stream));
  });
}

template <typename T, typename CS>
static int qnrc_launch(const void* qkv, int64_t ld, const void* qn, const void* kn, float eps,
                       const void* c, const void* s, int64_t cs_stride, const int32_t* pos,
                       void* q_out, void* kc, void* vc, int64_t c_sb, int64_t c_sh, int64_t c_ss,
                       int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D,
                       cudaStream_t st) {
  const int64_t total = B * S * (Hq + 2 * Hkv);
  if (total == 0) return TPP_OK;
  auto go = [&](auto g_tag) -> int {
    constexpr int G = decltype(g_tag)::value;
    const int per_block = 256 / G;
    const int64_t grid = (total + per_block - 1) / per_block;
    return launch("qk_norm_rope_cache_kernel", qk_norm_rope_cache_kernel<T, CS, G>, dim3((unsigned)grid), dim3(256), 0, st, 0, 
        (const T*)qkv, ld, (const T*)qn, (const T*)kn, eps, (const CS*)c, (const CS*)s, cs_stride,
        pos, (T*)q_out, (T*)kc, (T*)vc, c_sb, c_sh, c_ss, B, S, (int)Hq, (int)Hkv, (int)D);
  };
  switch (D) {
    case 16: return go(std::integral_constant<int, 2>{});
    case 32: return go(std::integral_constant<int, 4>{});
    case 64: return go(std::integral_constant<int, 8>{});
    case 128: return go(std::integral_constant<int, 16>{});
    case 256: return go(std::integral_constant<int, 32>{});
    default:
      set_error("tpp_qk_norm_rope_cache: head dim must be 16, 32, 64, 128 or 256");
      return TPP_ERR_UNSUPPORTED;
  }
}

namespace tpp {
namespace {
// K/V rows [B, Hkv, S, D] (strided) -> paged pools [num_blocks][Hkv][64][D]
// at positions (positions[b] or start_pos) + s, block table lookup per row.
template <typename T>
__global__ void __launch_bounds__(256) kv_append_paged_kernel(
    const T* __restrict__ k, int64_t k_sb, int64_t k_sh, int64_t k_ss, const T* __restrict__ v,
    int64_t v_sb, int64_t v_sh, int64_t v_ss, T* __restrict__ kp, T* __restrict__ vp,
    const int32_t* __restrict__ table, int64_t tbl_stride, int64_t Hkv, int64_t S, int D,
    int64_t start_pos, const int32_t* __restrict__ positions, int64_t total) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int per_row = D / 8;
  const int c = (int)(idx % per_row);
  const int64_t row = idx / per_row;
  const int64_t s = row % S;
  const int64_t bh = row / S;
  const int64_t h = bh % Hkv;
  const int64_t b = bh / Hkv;
  const int64_t pos = (positions ? (int64_t)positions[b] : start_pos) + s;
  const int64_t blk = table[b * tbl_stride + pos / 64];
  const int64_t dst = ((blk * Hkv + h) * 64 + pos % 64) * D + c * 8;
  *reinterpret_cast<uint4*>(kp + dst) =
      *reinterpret_cast<const uint4*>(k + b * k_sb + h * k_sh + s * k_ss + c * 8);
  *reinterpret_cast<uint4*>(vp + dst) =
      *reinterpret_cast<const uint4*>(v + b * v_sb + h * v_sh + s * v_ss + c * 8);
}
}  // namespace
}  // namespace tpp

extern "C" int tpp_kv_append_paged(const void* k, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                                   const void* v, int64_t v_sb, int64_t v_sh, int64_t v_ss,
                                   void* k_pool, void* v_pool, int64_t num_blocks,
                                   const int32_t* block_table, int64_t table_stride,
                                   const int32_t* positions, int64_t start_pos, int64_t B,
                                   int64_t Hkv, int64_t S, int64_t D, int dtype, void* stream) {
  if (B * S == 0) return TPP_OK;
  TPP_REQUIRE(k && v && k_pool && v_pool && block_table, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(B > 0 && Hkv > 0 && S > 0 && D > 0 && D % 8 == 0 && num_blocks > 0, TPP_ERR_SHAPE,
              "bad sizes (D must be a multiple of 8)");
  TPP_REQUIRE(k_sb % 8 == 0 && k_sh % 8 == 0 && k_ss % 8 == 0 && v_sb % 8 == 0 &&
                  v_sh % 8 == 0 && v_ss % 8 == 0 && aligned16(k) && aligned16(v) &&
                  aligned16(k_pool) && aligned16(v_pool),
              TPP_ERR_ALIGN, "rows must be 16-byte aligned");
  const int64_t total = B * Hkv * S * (D / 8);
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return launch("kv_append_paged_kernel", kv_append_paged_kernel<T>,
                  dim3((unsigned)((total + 255) / 256)), dim3(256), 0, as_stream(stream), 0u,
                  (const T*)k, k_sb, k_sh, k_ss, (const T*)v, v_sb, v_sh, v_ss, (T*)k_pool,
                  (T*)v_pool, block_table, table_stride, Hkv, S, (int)D, start_pos, positions,
                  total);
  });
}

extern "C" int tpp_qk_norm_rope_cache(const void* qkv, int64_t ld_qkv, const void* qn_w,
                                      const void* kn_w, float eps, const void* cos,
                                      const void* sin, int64_t cs_stride, int cs_dtype,
                                      const int32_t* positions, void* q_out, void* k_cache,
                                      void* v_cache, int64_t c_sb, int64_t c_sh, int64_t c_ss,
                                      int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D,
                                      int dtype, void* stream) {
  if (B * S == 0) return TPP_OK;
  TPP_REQUIRE(qkv && cos && sin && positions && q_out && k_cache && v_cache, TPP_ERR_SHAPE,
              "null pointer");
  TPP_REQUIRE(B >= 0 && S >= 0 && Hq > 0 && Hkv > 0 && D > 0, TPP_ERR_SHAPE, "bad sizes");
  TPP_REQUIRE(ld_qkv >= (Hq + 2 * Hkv) * D && ld_qkv % 8 == 0, TPP_ERR_SHAPE,
              "qkv row stride must cover (Hq+2Hkv)*D and be a multiple of 8");
  TPP_REQUIRE(c_ss % 8 == 0 && c_sh % 8 == 0 && c_sb % 8 == 0 && cs_stride % 8 == 0,
              TPP_ERR_ALIGN, "cache/table strides must be multiples of 8 elements");
  TPP_REQUIRE(aligned16(qkv) && aligned16(q_out) && aligned16(k_cache) && aligned16(v_cache) &&
                  aligned16(cos) && aligned16(sin) && (!qn_w || aligned16(qn_w)) &&
                  (!kn_w || aligned16(kn_w)),
              TPP_ERR_ALIGN, "pointers must be 16-byte aligned");
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    switch (cs_dtype) {
      case TPP_F16:
        return qnrc_launch<T, __half>(qkv, ld_qkv, qn_w, kn_w, eps, cos, sin, cs_stride, positions,
                                      q_out, k_cache, v_cache, c_sb, c_sh, c_ss, B, S, Hq, Hkv, D,
                                      as_stream(stream));
      case TPP_BF16:
        return qnrc_launch<T, __nv_bfloat16>(qkv, ld_qkv, qn_w, kn_w, eps, cos, sin, cs_stride,
                                             positions, q_out, k_cache, v_cache, c_sb, c_sh, c_ss,
                                             B, S, Hq, Hkv, D, as_stream(stream));
      case TPP_F32:
        return qnrc_launch<T, float>(qkv, ld_qkv, qn_w, kn_w, eps, cos, sin, cs_stride, positions,
                                     q_out, k_cache, v_cache, c_sb, c_sh, c_ss, B, S, Hq, Hkv, D,
                                     as_stream(stream));
      default:
        set_error("tpp_qk_norm_rope_cache: cos/sin dtype must be f16, bf16 or f32");
        return (int)TPP_ERR_DTYPE;
    }
  });
}

extern "C" int tpp_kv_append(const void* k, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                             const void* v, int64_t v_sb, int64_t v_sh, int64_t v_ss,
                             void* k_cache, void* v_cache, int64_t c_sb, int64_t c_sh,
                             int64_t c_ss, int64_t B, int64_t Hkv, int64_t S, int64_t D,
                             int64_t start_pos, const int32_t* positions, int dtype,
                             void* stream) {
  if (B * Hkv * S == 0) return TPP_OK;
  TPP_REQUIRE(k && v && k_cache && v_cache, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(B >= 0 && Hkv >= 0 && S >= 0 && D > 0 && start_pos >= 0, TPP_ERR_SHAPE, "bad sizes");
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    const bool vec = D % 8 == 0 && k_sb % 8 == 0 && k_sh % 8 == 0 && k_ss % 8 == 0 &&
                     v_sb % 8 == 0 && v_sh % 8 == 0 && v_ss % 8 == 0 && c_sb % 8 == 0 &&
                     c_sh % 8 == 0 && c_ss % 8 == 0 && aligned16(k) && aligned16(v) &&
                     aligned16(k_cache) && aligned16(v_cache);
    const int64_t total = B * Hkv * S * (vec ? D / 8 : D);
    if (total == 0) return (int)TPP_OK;
    const int64_t grid = (total + 255) / 256;
    return launch("kv_append_kernel", kv_append_kernel<T>, dim3((unsigned)grid), dim3(256), 0, as_stream(stream), 0, 
        (const T*)k, k_sb, k_sh, k_ss, (const T*)v, v_sb, v_sh, v_ss, (T*)k_cache, (T*)v_cache,
        c_sb, c_sh, c_ss, Hkv, S, (int)D, start_pos, positions, total, vec);
  });
}
