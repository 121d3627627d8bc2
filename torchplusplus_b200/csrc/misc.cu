// Decode-step helpers: greedy argmax over the vocabulary and the token
// embedding gather, so a whole decode step stays on the device (and inside one
// CUDA graph) instead of syncing to the host per token as
// torchpp/llmops/llm.py:205-222 does with token.item().
#include <math.h>
#include "common.cuh"

namespace tpp {
namespace {

// One CTA per row.  Ties resolve to the smallest index, like torch.argmax.
// NaN compares greater than everything (torch.argmax treats NaN as the max).
template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ x, int64_t ld,
                                                      int64_t V, int64_t* __restrict__ out,
                                                      bool vec) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const T* row = x + (int64_t)blockIdx.x * ld;
  float best = -INFINITY;
  int64_t bi = V;  // sentinel larger than any index
  auto take = [&](float v, int64_t i) {
    const bool vn = isnan(v), bn = isnan(best);
    if ((vn && !bn) || (!bn && v > best) || ((v == best || (vn && bn)) && i < bi)) {
      best = v;
      bi = i;
    }
  };
  if (vec) {
    const int64_t nv = V / 8;
    const int64_t step = blockDim.x;
    int64_t c = threadIdx.x;
    // four independent 16-byte loads in flight per thread (the logits were
    // just written: each round trip is an L2 latency); order does not matter,
    // ties are resolved by index
    for (; c + 3 * step < nv; c += 4 * step) {
      uint4 u[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) u[q] = ldg_nc_v4(row + (c + q * step) * 8);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float f[8];
        unpack8<T>(u[q], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) take(f[j], (c + q * step) * 8 + j);
      }
    }
    for (; c < nv; c += step) {
      float f[8];
      unpack8<T>(ldg_nc_v4(row + c * 8), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) take(f[j], c * 8 + j);
    }
    for (int64_t i = nv * 8 + threadIdx.x; i < V; i += blockDim.x) take(to_f32(row[i]), i);
  } else {
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) take(to_f32(row[i]), i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    take(ov, oi);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : V;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      take(ov, oi);
    }
    if (lane == 0) out[blockIdx.x] = bi < V ? bi : 0;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) embedding_kernel(const int64_t* __restrict__ ids, int64_t T_,
                                                        const T* __restrict__ table, int64_t V,
                                                        int64_t D, T* __restrict__ out, bool vec) {
  pdl_wait();
  pdl_trigger();
  const int64_t per_row = vec ? D / 8 : D;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T_ * per_row) return;
  const int64_t t = idx / per_row, c = idx % per_row;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < V;
  if (vec) {
    uint4 v = ok ? __ldg(reinterpret_cast<const uint4*>(table + id * D) + c) : make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(out + t * D)[c] = v;
  } else {
    out[t * D + c] = ok ? table[id * D + c] : from_f32<T>(0.f);
  }
}

__global__ void decode_advance_kernel(const int64_t* __restrict__ next, int64_t* __restrict__ out_ids,
                                      int64_t ld_out, int32_t* __restrict__ positions,
                                      int32_t* __restrict__ seqlens, int64_t B, int64_t cap) {
  pdl_wait();
  pdl_trigger();
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int32_t p = positions[b] + 1;
  if (out_ids != nullptr && p < cap) out_ids[b * ld_out + p] = next[b];
  positions[b] = p;
  if (seqlens != nullptr) seqlens[b] = p + 1;
}

}  // namespace
}  // namespace tpp

using namespace tpp;

extern "C" int tpp_decode_advance(const int64_t* next_tokens, int64_t* out_ids, int64_t ld_out,
                                  int64_t out_cap, int32_t* positions, int32_t* seqlens,
                                  int64_t B, void* stream) {
  TPP_REQUIRE(next_tokens && positions, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(B >= 0 && (out_ids == nullptr || (ld_out >= out_cap && out_cap >= 0)),
              TPP_ERR_SHAPE, "bad sizes");
  if (B == 0) return TPP_OK;
  return launch("decode_advance_kernel", decode_advance_kernel, dim3((unsigned)((B + 127) / 128)), dim3(128), 0, as_stream(stream), 0, 
      next_tokens, out_ids, ld_out, positions, seqlens, B, out_cap);
}

extern "C" int tpp_argmax(const void* logits, int64_t ld, int64_t B, int64_t V, int64_t* out,
                          int dtype, void* stream) {
  if (B == 0) return TPP_OK;
  TPP_REQUIRE(logits && out, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(B >= 0 && V > 0 && ld >= V, TPP_ERR_SHAPE, "bad sizes");
  if (B == 0) return TPP_OK;
  auto go = [&](auto tag) -> int {
    using T = decltype(tag);
    const bool vec = (ld % 8 == 0) && aligned16(logits) && sizeof(T) == 2;
    return launch("argmax_kernel", argmax_kernel<T>, dim3((unsigned)B), dim3(1024), 0, as_stream(stream), 0, (const T*)logits, ld, V, out,
                                                                  vec);
  };
  if (dtype == TPP_F16) return go(__half());
  if (dtype == TPP_BF16) return go(__nv_bfloat16());
  if (dtype == TPP_F32) {
    return launch("argmax_kernel", argmax_kernel<float>, dim3((unsigned)B), dim3(1024), 0, as_stream(stream), 0, (const float*)logits, ld, V,
                                                                      out, false);
  }
  set_error("tpp_argmax: dtype must be f16, bf16 or f32");
  return TPP_ERR_DTYPE;
}

extern "C" int tpp_embedding(const int64_t* ids, int64_t T_, const void* table, int64_t V,
                             int64_t D, void* out, int dtype, void* stream) {
  if (T_ == 0) return TPP_OK;
  TPP_REQUIRE(ids && table && out, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(T_ >= 0 && V > 0 && D > 0, TPP_ERR_SHAPE, "bad sizes");
  if (T_ == 0) return TPP_OK;
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    const bool vec = D % 8 == 0 && aligned16(table) && aligned16(out);
    const int64_t total = T_ * (vec ? D / 8 : D);
    return launch("embedding_kernel", embedding_kernel<T>, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, as_stream(stream), 0, 
        ids, T_, (const T*)table, V, D, (T*)out, vec);
  });
}

// ---------------------------------------------------------------------------
// L2 warm-up: bulk prefetch of [ptr, ptr + bytes) into L2 (no data is moved
// to the SMs).  A decode engine launches it on a parallel graph branch so the
// next layers' weights are L2 hits when their kernels load them.
// ---------------------------------------------------------------------------
namespace tpp {
namespace {
__global__ void l2_prefetch_kernel(const uint8_t* __restrict__ p, int64_t bytes) {
  constexpr int64_t kPiece = 64 * 1024;
  const int64_t n = (bytes + kPiece - 1) / kPiece;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t off = i * kPiece;
    const int64_t len = bytes - off < kPiece ? bytes - off : kPiece;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"((uint32_t)len)
                 : "memory");
  }
}
}  // namespace
}  // namespace tpp

extern "C" int tpp_l2_prefetch(const void* ptr, int64_t bytes, void* stream) {
  if (bytes <= 0) return TPP_OK;
  TPP_REQUIRE(ptr, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(aligned16(ptr) && bytes % 16 == 0, TPP_ERR_ALIGN,
              "prefetch range must be 16-byte aligned and a multiple of 16 bytes");
  const int64_t pieces = (bytes + 65535) / 65536;
  const int threads = 32;
  const int blocks = (int)((pieces + threads - 1) / threads < 64 ? (pieces + threads - 1) / threads : 64);
  l2_prefetch_kernel<<<blocks, threads, 0, as_stream(stream)>>>(static_cast<const uint8_t*>(ptr),
                                                                bytes);
  return check_launch("l2_prefetch_kernel");
}
