// Decode-step helpers: greedy argmax over the vocabulary and the token
// embedding gather, so a whole decode step stays on the device (and inside one
// CUDA graph) instead of syncing to the host per token as
// torchpp/llmops/llm.py:205-222 does with token.item().
#include <math.h>
#include "common.cuh"

namespace tpp {
namespace {

// Rows are split over a cluster of kRowCtas CTAs (one slice each); the
// slices' partial results meet through distributed shared memory, so a batch
// of 32 rows fills 256 SMs' worth of CTAs instead of 32.
constexpr int kRowCtas = 8;
constexpr int kRowThreads = 512;
constexpr int kRowWarps = kRowThreads / 32;

__device__ __forceinline__ uint32_t cl_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// full cluster barrier: this CTA's shared-memory writes are visible to the
// peers' reads after it
__device__ __forceinline__ void cl_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_peer_f32(const float* p, uint32_t rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(peer_addr(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ long long ld_peer_s64(const long long* p, uint32_t rank) {
  long long v;
  asm volatile("ld.shared::cluster.s64 %0, [%1];" : "=l"(v) : "r"(peer_addr(p, rank)) : "memory");
  return v;
}

// One cluster per row.  Ties resolve to the smallest index, like torch.argmax.
// NaN compares greater than everything (torch.argmax treats NaN as the max).
template <typename T>
__global__ void __launch_bounds__(kRowThreads) argmax_kernel(const T* __restrict__ x, int64_t ld,
                                                             int64_t V, int64_t* __restrict__ out,
                                                             bool vec) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[kRowWarps];
  __shared__ long long si[kRowWarps];
  __shared__ float c_v;
  __shared__ long long c_i;
  const uint32_t cr = cl_rank();
  const T* row = x + (int64_t)blockIdx.x * ld;
  float best = -INFINITY;
  long long bi = V;  // sentinel larger than any index
  auto take = [&](float v, long long i) {
    const bool vn = isnan(v), bn = isnan(best);
    if ((vn && !bn) || (!bn && v > best) || ((v == best || (vn && bn)) && i < bi)) {
      best = v;
      bi = i;
    }
  };
  bool done = false;
  if constexpr (sizeof(T) == 2) {  // 16-byte vectors of 8 elements (16-bit types only)
  if (vec) {
    done = true;
    const int64_t nv = V / 8, per = (nv + kRowCtas - 1) / kRowCtas;
    const int64_t c0 = (int64_t)cr * per, c1 = c0 + per < nv ? c0 + per : nv;
    constexpr int step = kRowThreads;
    int64_t c = c0 + threadIdx.x;
    // up to eight independent 16-byte loads in flight per thread: one
    // memory round trip covers a row slice of up to 8 x 512 x 8 elements
    // (the logits were just written: each round trip is an L2 latency);
    // order does not matter, ties are resolved by index
    for (; c < c1; c += 8 * step) {
      uint4 u[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        u[q] = c + q * step < c1 ? ldg_nc_v4(row + (c + q * step) * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (c + q * step >= c1) break;
        float f[8];
        unpack8<T>(u[q], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) take(f[j], (c + q * step) * 8 + j);
      }
    }
    if (cr == kRowCtas - 1)
      for (int64_t i = nv * 8 + threadIdx.x; i < V; i += kRowThreads) take(to_f32(row[i]), i);
  }
  }
  if (!done) {
    const int64_t per = (V + kRowCtas - 1) / kRowCtas;
    const int64_t i0 = (int64_t)cr * per, i1 = i0 + per < V ? i0 + per : V;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += kRowThreads) take(to_f32(row[i]), i);
  }
  auto warp_take = [&]() {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const long long oi = __shfl_xor_sync(0xffffffffu, bi, o);
      take(ov, oi);
    }
  };
  warp_take();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = lane < kRowWarps ? sv[lane] : -INFINITY;
    bi = lane < kRowWarps ? si[lane] : V;
    warp_take();
    if (lane == 0) { c_v = best; c_i = bi; }
  }
  cl_sync();
  if (cr == 0 && warp == 0) {
    best = lane < kRowCtas ? ld_peer_f32(&c_v, lane) : -INFINITY;
    bi = lane < kRowCtas ? ld_peer_s64(&c_i, lane) : V;
    warp_take();
    if (lane == 0) out[blockIdx.x] = bi < V ? bi : 0;
  }
  cl_sync();  // the peers' shared memory stays live until rank 0 has read it
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
    return launch("argmax_kernel", argmax_kernel<T>, dim3((unsigned)B, kRowCtas),
                  dim3(kRowThreads), 0, as_stream(stream), (unsigned)kRowCtas,
                  (const T*)logits, ld, V, out, vec);
  };
  if (dtype == TPP_F16) return go(__half());
  if (dtype == TPP_BF16) return go(__nv_bfloat16());
  if (dtype == TPP_F32) {
    return launch("argmax_kernel", argmax_kernel<float>, dim3((unsigned)B, kRowCtas),
                  dim3(kRowThreads), 0, as_stream(stream), (unsigned)kRowCtas,
                  (const float*)logits, ld, V, out, false);
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
// One cluster of kRowCtas CTAs per row; each CTA stages its slice of the
// row in shared memory once and every later pass reads it from there.
// Thresholds come from an exact radix selection on the 16-bit orderable keys
// of the logits (two passes of 256-bin histograms: counts for top-k,
// probability mass for top-p), so tokens tied with the threshold are all
// kept (torch's sort/topk keep an arbitrary subset of such ties).  The
// histograms are lane-replicated ([bin][lane]) so the many logits that share
// a high byte do not serialise a warp's shared-memory atomics; the slices'
// bin totals are summed through distributed shared memory, in the same
// order in every CTA, so all CTAs pick the same thresholds.  The draw is an
// inverse-CDF walk over the kept tokens in a fixed visiting order (slices in
// rank order, threads in index order) with u from SplitMix64 (Steele, Lea &
// Flood, OOPSLA 2014) of (seed, row, counter[row]) -- a different random
// stream than torch.multinomial, the same distribution.
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

// dynamic shared memory of the sampling kernel: histogram [256][32] words,
// two merge buffers [2][256], the cluster totals [256], then the staged slice
// (16-byte vectors) when it fits
constexpr int kHistWords = 256 * 32;
constexpr size_t kSampleFixedSmem = (size_t)(kHistWords + 3 * 256) * 4;

template <typename T>
__global__ void __launch_bounds__(kRowThreads) sample_kernel(
    const T* __restrict__ x, int64_t ld, int64_t V, float inv_temp_log2, int64_t top_k,
    float top_p, uint64_t seed, const int32_t* __restrict__ counters, int64_t* __restrict__ out,
    bool staged) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint32_t* hist = reinterpret_cast<uint32_t*>(sm_raw);           // [256][32]
  float* mbuf = reinterpret_cast<float*>(hist + kHistWords);      // [2][256]
  float* gtot = mbuf + 2 * 256;                                    // [256]
  uint4* slice = reinterpret_cast<uint4*>(gtot + 256);
  __shared__ float red[kRowWarps];
  __shared__ long long redi[kRowWarps];
  __shared__ float s_f[2];
  __shared__ uint32_t s_bin;
  __shared__ long long s_arg, s_pick;
  __shared__ int s_owner;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t cr = cl_rank();
  const int b = blockIdx.x;
  const T* row = x + (int64_t)b * ld;
  const int64_t nv = V / 8;  // V % 8 == 0 (host)
  const int64_t per = (nv + kRowCtas - 1) / kRowCtas;
  const int64_t c0 = (int64_t)cr * per;
  const int n = (int)(c0 >= nv ? 0 : (nv - c0 < per ? nv - c0 : per));
  int mb = 0;  // merge buffer in use

  // sums a 256-entry per-CTA array over the cluster into gtot (rank order)
  auto merge = [&](const float* mine) {
    cl_sync();
    if (tid < 256) {
      float t = 0.f;
#pragma unroll
      for (int r = 0; r < kRowCtas; ++r) t += ld_peer_f32(mine + tid, r);
      gtot[tid] = t;
    }
    __syncthreads();
  };
  auto for_slice = [&](auto&& f) {  // f(key, value, index) over this CTA's slice
    for (int c = tid; c < n; c += kRowThreads) {
      const uint4 u = staged ? slice[c] : ldg_nc_v4(row + (c0 + c) * 8);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) f(order_key<T>(e[j]), to_f32(e[j]), (c0 + c) * 8 + j);
    }
  };

  // 1. stage the slice; row max (softmax stabiliser) and its first index
  float mx = -INFINITY;
  long long mi = V;
  auto take = [&](float v, long long i) {
    if (v > mx || (v == mx && i < mi)) { mx = v; mi = i; }
  };
  {
    int c = tid;
    for (; c + 3 * kRowThreads < n; c += 4 * kRowThreads) {
      uint4 u[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) u[q] = ldg_nc_v4(row + (c0 + c + q * kRowThreads) * 8);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (staged) slice[c + q * kRowThreads] = u[q];
        const T* e = reinterpret_cast<const T*>(&u[q]);
#pragma unroll
        for (int j = 0; j < 8; ++j) take(to_f32(e[j]), (c0 + c + q * kRowThreads) * 8 + j);
      }
    }
    for (; c < n; c += kRowThreads) {
      const uint4 u = ldg_nc_v4(row + (c0 + c) * 8);
      if (staged) slice[c] = u;
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) take(to_f32(e[j]), (c0 + c) * 8 + j);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, mx, o);
    const long long oi = __shfl_xor_sync(0xffffffffu, mi, o);
    take(ov, oi);
  }
  if (lane == 0) { red[warp] = mx; redi[warp] = mi; }
  __syncthreads();
  if (warp == 0) {
    mx = lane < kRowWarps ? red[lane] : -INFINITY;
    mi = lane < kRowWarps ? redi[lane] : V;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, mx, o);
      const long long oi = __shfl_xor_sync(0xffffffffu, mi, o);
      take(ov, oi);
    }
    if (lane == 0) {
      mbuf[0] = mx;
      reinterpret_cast<long long*>(mbuf)[1] = mi;  // words 2..3
    }
  }
  cl_sync();
  if (warp == 0) {
    mx = lane < kRowCtas ? ld_peer_f32(mbuf, lane) : -INFINITY;
    mi = lane < kRowCtas ? ld_peer_s64(reinterpret_cast<const long long*>(mbuf) + 1, lane) : V;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, mx, o);
      const long long oi = __shfl_xor_sync(0xffffffffu, mi, o);
      take(ov, oi);
    }
    if (lane == 0) { s_f[0] = mx; s_arg = mi < V ? mi : 0; }
  }
  __syncthreads();
  mx = s_f[0];
  mb = 1;
  auto weight = [&](float v) { return exp2f((v - mx) * inv_temp_log2); };

  // radix selection helpers
  auto clear = [&]() {
    uint4* h4 = reinterpret_cast<uint4*>(hist);
    for (int i = tid; i < kHistWords / 4; i += kRowThreads) h4[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
  };
  // folds the lane copies into this CTA's 256 totals, then sums the cluster
  auto fold_merge = [&](bool mass) {
    __syncthreads();
    float* mine = mbuf + mb * 256;
    if (tid < 256) {
      float t = 0.f;
      for (int l = 0; l < 32; ++l) {
        const uint32_t w = hist[tid * 32 + ((l + tid) & 31)];
        t += mass ? __uint_as_float(w) : (float)w;
      }
      mine[tid] = t;
    }
    merge(mine);
    mb ^= 1;
  };
  // descending scan of gtot: the first bin from the top whose cumulative
  // total reaches `target` (counts: >=, mass: >); target = frac * total when
  // frac >= 0.  Writes the total above that bin to s_f[1]; with no such bin
  // (rounding), bin 0 and the whole total.
  auto pick_bin = [&](bool mass, float target, float frac) -> uint32_t {
    if (warp == 0) {
      float c[8], own = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) { c[j] = gtot[lane * 8 + j]; own += c[j]; }
      float suf = own;  // sum over lanes >= this lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float nb = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += nb;
      }
      const float total = __shfl_sync(0xffffffffu, suf, 0);
      if (frac >= 0.f) target = frac * total;
      float above = suf - own;
      int hit = -1;
      float hit_above = 0.f;
#pragma unroll
      for (int j = 7; j >= 0; --j) {
        const bool h = mass ? (above + c[j] > target) : (above + c[j] >= target);
        if (h && hit < 0) { hit = j; hit_above = above; }
        above += c[j];
      }
      const unsigned bal = __ballot_sync(0xffffffffu, hit >= 0);
      if (bal == 0u) {
        if (lane == 0) { s_bin = 0u; s_f[1] = total; s_f[0] = target; }
      } else {
        const int hl = 31 - __clz(bal);
        if (lane == hl) { s_bin = (uint32_t)(lane * 8 + hit); s_f[1] = hit_above; s_f[0] = target; }
      }
    }
    __syncthreads();
    return s_bin;
  };

  // 2. top-k threshold on the keys
  uint32_t tk = 0;
  if (top_k > 0 && top_k < V) {
    clear();
    for_slice([&](uint32_t k, float, int64_t) { atomicAdd(&hist[(k >> 8) * 32 + lane], 1u); });
    fold_merge(false);
    const uint32_t hb = pick_bin(false, (float)top_k, -1.f);
    const float above = s_f[1];
    clear();
    for_slice([&](uint32_t k, float, int64_t) {
      if ((k >> 8) == hb) atomicAdd(&hist[(k & 255u) * 32 + lane], 1u);
    });
    fold_merge(false);
    const uint32_t lb = pick_bin(false, (float)top_k - above, -1.f);
    tk = (hb << 8) | lb;
  }
  // 3. top-p threshold among the kept keys, by probability mass
  uint32_t t = tk;
  if (top_p < 1.f) {
    float* hm = reinterpret_cast<float*>(hist);
    clear();
    for_slice([&](uint32_t k, float v, int64_t) {
      if (k >= tk) atomicAdd(&hm[(k >> 8) * 32 + lane], weight(v));
    });
    fold_merge(true);
    const uint32_t hb = pick_bin(true, 0.f, top_p);
    const float target = s_f[0], above = s_f[1];
    __syncthreads();
    clear();
    for_slice([&](uint32_t k, float v, int64_t) {
      if (k >= tk && (k >> 8) == hb) atomicAdd(&hm[(k & 255u) * 32 + lane], weight(v));
    });
    fold_merge(true);
    const uint32_t lb = pick_bin(true, target - above, -1.f);
    const uint32_t tp = (hb << 8) | lb;
    t = tp > tk ? tp : tk;
  }
  // 4. inverse-CDF draw over kept tokens (key >= t), fixed visiting order
  float part = 0.f;
  for_slice([&](uint32_t k, float v, int64_t) { if (k >= t) part += weight(v); });
  float incl = part;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float nb = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += nb;
  }
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    float w = lane < kRowWarps ? red[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float nb = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += nb;
    }
    if (lane < kRowWarps) red[lane] = w;  // inclusive warp totals
    if (lane == kRowWarps - 1) mbuf[mb * 256] = w;  // this slice's kept mass
  }
  cl_sync();
  const uint64_t r = splitmix64(seed ^ ((uint64_t)b * 0xD1B54A32D192ED03ull) ^
                                ((uint64_t)(counters ? counters[b] : 0) << 32));
  if (tid == 0) {
    // slice masses in rank order; the owner slice holds u (or, through
    // rounding, the last slice with mass)
    float sl[kRowCtas], total = 0.f;
#pragma unroll
    for (int q = 0; q < kRowCtas; ++q) { sl[q] = ld_peer_f32(mbuf + mb * 256, q); total += sl[q]; }
    const float u = (float)(r >> 40) * (1.0f / 16777216.0f) * total;
    int owner = -1, last = -1;
    float before = 0.f, own_before = 0.f, last_before = 0.f;
    for (int q = 0; q < kRowCtas; ++q) {
      if (sl[q] > 0.f) {
        last = q;
        last_before = before;
        if (owner < 0 && u >= before && u < before + sl[q]) { owner = q; own_before = before; }
      }
      before += sl[q];
    }
    if (owner < 0) { owner = last; own_before = last_before; }
    s_owner = owner;
    s_f[0] = u - own_before;  // u within the owner slice
    s_pick = -1;
  }
  cl_sync();  // peers' shared memory is not read after this point
  if ((int)cr != s_owner) {
    if (s_owner < 0 && cr == 0 && tid == 0) out[b] = s_arg;
    return;
  }
  const float u = s_f[0];
  const float before_warp = warp > 0 ? red[warp - 1] : 0.f;
  const float total = red[kRowWarps - 1];
  const float excl = before_warp + incl - part;
  // the thread whose range holds u walks its elements again (same order and
  // arithmetic as `part`, so its running sum reproduces excl .. excl + part)
  if (part > 0.f && u >= excl && (u < excl + part || tid == kRowThreads - 1 ||
                                   excl + part >= total)) {
    float run = excl;
    long long lastk = -1, pick = -1;
    for_slice([&](uint32_t k, float v, int64_t i) {
      if (k >= t && pick < 0) {
        run += weight(v);
        lastk = i;
        if (run > u) pick = i;
      }
    });
    atomicMax(&s_pick, pick >= 0 ? pick : lastk);
  }
  __syncthreads();
  if (tid == 0) {
    // u fell between two threads' ranges through rounding: take the row max
    out[b] = s_pick >= 0 ? s_pick : s_arg;
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
  const int64_t per = (V / 8 + kRowCtas - 1) / kRowCtas;
  const size_t slice_bytes = (size_t)per * 16;
  const bool staged = kSampleFixedSmem + slice_bytes <= 200 * 1024;
  const size_t smem = kSampleFixedSmem + (staged ? slice_bytes : 0);
  const float itl = 1.4426950408889634f / temperature;
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    cudaFuncSetAttribute(sample_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    return launch("sample_kernel", sample_kernel<T>, dim3((unsigned)B, kRowCtas),
                  dim3(kRowThreads), smem, as_stream(stream), (unsigned)kRowCtas,
                  (const T*)logits, ld, V, itl, top_k, top_p, seed, counters, out, staged);
  });
}
