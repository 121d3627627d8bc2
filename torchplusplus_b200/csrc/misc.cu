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

// ---------------------------------------------------------------------------
// On-device sampling: temperature + top-k + top-p (nucleus) + one draw per
// row, the semantics of LLMInference.sample_top_k / sample_top_p
// (torchpp/llmops/llm.py:114-203): softmax(logits / T) restricted to the k
// largest logits and/or to the smallest descending prefix whose cumulative
// probability exceeds p (the crossing token included).
//
// One CTA per row.  Thresholds come from an exact radix selection on the
// 16-bit orderable keys of the logits (two passes of 256-bin histograms:
// counts for top-k, probability mass for top-p), so tokens tied with the
// threshold are all kept (torch's sort/topk keep an arbitrary subset of
// such ties).  The draw is an inverse-CDF walk over the kept tokens in the
// kernel's fixed visiting order with u from SplitMix64 (Steele, Lea & Flood,
// OOPSLA 2014) of (seed, row, counter[row]) -- a different random stream
// than torch.multinomial, the same distribution.
// ---------------------------------------------------------------------------
namespace tpp {
namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

template <typename T>
__device__ __forceinline__ uint32_t order_key(T v) {
  const uint16_t h = *reinterpret_cast<const uint16_t*>(&v);
  return (h & 0x8000u) ? (uint32_t)(~h & 0xFFFFu) : (uint32_t)(h | 0x8000u);
}

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(
    const T* __restrict__ x, int64_t ld, int64_t V, float inv_temp_log2, int64_t top_k,
    float top_p, uint64_t seed, const int32_t* __restrict__ counters, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t sm_raw[];
  uint32_t* hc = reinterpret_cast<uint32_t*>(sm_raw);                     // [warps][256]
  float* hm = reinterpret_cast<float*>(hc + kSampleWarps * 256);         // [warps][256]
  float* red = hm + kSampleWarps * 256;                                   // [warps]
  __shared__ uint32_t s_key;
  __shared__ float s_f[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x;
  const T* row = x + (int64_t)b * ld;
  const int64_t nv = V / 8;  // V % 8 == 0 (host)

  auto block_max = [&](float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
      v = lane < kSampleWarps ? red[lane] : -INFINITY;
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) s_f[0] = v;
    }
    __syncthreads();
    const float r = s_f[0];
    __syncthreads();
    return r;
  };
  auto for_row = [&](auto&& f) {  // f(key, value, index) over the whole row
    for (int64_t c = tid; c < nv; c += kSampleThreads) {
      const uint4 u = ldg_nc_v4(row + c * 8);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) f(order_key<T>(e[j]), to_f32(e[j]), c * 8 + j);
    }
  };

  // 1. row max (softmax stabiliser) and its first index (the fallback pick)
  float mx = -INFINITY;
  int64_t mi = V;
  for_row([&](uint32_t, float v, int64_t i) {
    if (v > mx || (v == mx && i < mi)) { mx = v; mi = i; }
  });
  __shared__ long long s_arg;
  if (tid == 0) s_arg = V;
  const float rmx = block_max(mx);
  if (mx == rmx) atomicMin(&s_arg, (long long)mi);
  mx = rmx;
  auto weight = [&](float v) { return exp2f((v - mx) * inv_temp_log2); };

  // radix selection helpers: per-warp histograms, then a descending scan
  auto clear = [&]() {
    for (int i = tid; i < kSampleWarps * 256; i += kSampleThreads) { hc[i] = 0u; hm[i] = 0.f; }
    __syncthreads();
  };
  // descending scan of the (summed) bins: first bin from the top whose
  // cumulative total reaches `target` (counts: >=, mass: >); returns the bin
  // and writes the total above it to s_f[1]
  auto pick_bin = [&](bool mass, float target) -> uint32_t {
    if (tid < 256) {
      float c = 0.f;
      for (int w = 0; w < kSampleWarps; ++w)
        c += mass ? hm[w * 256 + tid] : (float)hc[w * 256 + tid];
      hm[tid] = c;  // warp 0's row now holds the totals
    }
    __syncthreads();
    if (tid == 0) {
      float above = 0.f;
      uint32_t bin = 0;
      for (int i = 255; i >= 0; --i) {
        const float c = hm[i];
        const bool hit = mass ? (above + c > target) : (above + c >= target);
        if (hit) { bin = (uint32_t)i; break; }
        above += c;
      }
      s_key = bin;
      s_f[1] = above;
    }
    __syncthreads();
    return s_key;
  };

  // 2. top-k threshold on the keys
  uint32_t tk = 0;
  if (top_k > 0 && top_k < V) {
    clear();
    for_row([&](uint32_t k, float, int64_t) { atomicAdd(&hc[warp * 256 + (k >> 8)], 1u); });
    __syncthreads();
    const uint32_t hb = pick_bin(false, (float)top_k);
    const float above = s_f[1];
    __syncthreads();
    clear();
    for_row([&](uint32_t k, float, int64_t) {
      if ((k >> 8) == hb) atomicAdd(&hc[warp * 256 + (k & 255u)], 1u);
    });
    __syncthreads();
    const uint32_t lb = pick_bin(false, (float)top_k - above);
    tk = (hb << 8) | lb;
  }
  // 3. top-p threshold among the kept keys, by probability mass
  uint32_t t = tk;
  if (top_p < 1.f) {
    clear();
    for_row([&](uint32_t k, float v, int64_t) {
      if (k >= tk) atomicAdd(&hm[warp * 256 + (k >> 8)], weight(v));
    });
    __syncthreads();
    // total mass Z first (the bins sum to it)
    if (tid < 256) {
      float c = 0.f;
      for (int w = 0; w < kSampleWarps; ++w) c += hm[w * 256 + tid];
      hc[tid] = __float_as_uint(c);
    }
    __syncthreads();
    if (tid == 0) {
      float z = 0.f;
      for (int i = 0; i < 256; ++i) z += __uint_as_float(hc[i]);
      s_f[0] = z;
    }
    __syncthreads();
    const float target = top_p * s_f[0];
    const uint32_t hb = pick_bin(true, target);
    const float above = s_f[1];
    __syncthreads();
    clear();
    for_row([&](uint32_t k, float v, int64_t) {
      if (k >= tk && (k >> 8) == hb) atomicAdd(&hm[warp * 256 + (k & 255u)], weight(v));
    });
    __syncthreads();
    const uint32_t lb = pick_bin(true, target - above);
    const uint32_t tp = (hb << 8) | lb;
    t = tp > tk ? tp : tk;
  }
  // 4. inverse-CDF draw over kept tokens (key >= t), fixed visiting order
  float part = 0.f;
  for_row([&](uint32_t k, float v, int64_t) { if (k >= t) part += weight(v); });
  // inclusive block scan of the per-thread partial sums
  float incl = part;
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    float w = lane < kSampleWarps ? red[lane] : 0.f;
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    if (lane < kSampleWarps) red[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const float before_warp = warp > 0 ? red[warp - 1] : 0.f;
  const float total = red[kSampleWarps - 1];
  const float excl = before_warp + incl - part;
  const uint64_t r = splitmix64(seed ^ ((uint64_t)b * 0xD1B54A32D192ED03ull) ^
                                ((uint64_t)(counters ? counters[b] : 0) << 32));
  const float u = (float)(r >> 40) * (1.0f / 16777216.0f) * total;
  __shared__ long long s_pick;
  if (tid == 0) s_pick = -1;
  __syncthreads();
  // the thread whose range holds u walks its elements again (same order and
  // arithmetic as `part`, so its running sum reproduces excl .. excl + part)
  if (part > 0.f && u >= excl && (u < excl + part || tid == kSampleThreads - 1 ||
                                   excl + part >= total)) {
    float run = excl;
    int64_t last = -1, pick = -1;
    for_row([&](uint32_t k, float v, int64_t i) {
      if (k >= t && pick < 0) {
        run += weight(v);
        last = i;
        if (run > u) pick = i;
      }
    });
    atomicMax(&s_pick, (long long)(pick >= 0 ? pick : last));
  }
  __syncthreads();
  if (tid == 0) {
    // u fell between two threads' ranges through rounding: take the row max
    const long long pk = s_pick >= 0 ? s_pick : s_arg;
    out[b] = pk;
  }
}
}  // namespace
}  // namespace tpp

extern "C" int tpp_sample(const void* logits, int64_t ld, int64_t B, int64_t V, float temperature,
                          int64_t top_k, float top_p, uint64_t seed, const int32_t* counters,
                          int64_t* out, int dtype, void* stream) {
  if (B == 0) return TPP_OK;
  TPP_REQUIRE(logits && out, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(B > 0 && V > 0 && ld >= V && V % 8 == 0 && ld % 8 == 0, TPP_ERR_SHAPE,
              "need V and the row stride multiples of 8");
  TPP_REQUIRE(aligned16(logits), TPP_ERR_ALIGN, "logits must be 16-byte aligned");
  TPP_REQUIRE(temperature > 0.f && top_p > 0.f && top_k >= 0, TPP_ERR_SHAPE,
              "need temperature > 0, top_p > 0, top_k >= 0 (greedy: tpp_argmax)");
  const size_t smem = (size_t)kSampleWarps * 256 * 8 + kSampleWarps * 4;
  const float itl = 1.4426950408889634f / temperature;
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    cudaFuncSetAttribute(sample_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    return launch("sample_kernel", sample_kernel<T>, dim3((unsigned)B), dim3(kSampleThreads),
                  smem, as_stream(stream), 0u, (const T*)logits, ld, V, itl, top_k, top_p,
                  seed, counters, out);
  });
}
