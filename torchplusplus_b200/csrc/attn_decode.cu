// Decode attention: one query token per sequence against a BHSD KV cache,
// GQA/MQA head sharing and an optional sliding window, split-KV.
//
// Semantics follow flash_attn_func as torchpp calls it at decode
// (torchpp/attention/gqa.py:117-128 with the KV cache, swa.py:85-89 for the
// window): o = softmax(q.K^T * scale) V over keys j in [p - window_left, p],
// p = seqlen-1 the query position; query head h reads kv head h / (Hq/Hkv)
// (the repeat_interleave of gqa.py:120-121, without materialising it).
//
// Design (HBM-bound on the cache):
//  * grid (split, kv_head x head_pass, batch); a CTA streams one slice of the
//    key range of one kv head once and serves all G query heads that share it
//    (up to 8 per pass), so K/V bytes are read once per kv head, not per q head.
//  * 128 threads = 128/LG "streams" of LG = D/8 lanes; a stream takes one key
//    row at a time (LG lanes x 16 bytes = one contiguous row), keeps fp32
//    online-softmax state (m, l, acc[8] per head) in registers, and processes
//    4 keys per step with a single rescale.
//  * streams merge in shared memory; with one split the CTA writes o, else it
//    writes (o, lse) partials to the workspace and decode_combine_kernel
//    merges the splits.
#include <math.h>
#include <mutex>
#include "tc_common.cuh"
#include "attn_decode.cuh"

namespace tpp {

int attn_decode_num_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t range) {
  const int64_t G = Hkv > 0 ? Hq / Hkv : 1;
  const int64_t passes = (G + 7) / 8;
  const int64_t ctas = B * Hkv * passes;
  int64_t target = (8LL * sm_budget() + ctas - 1) / (ctas > 0 ? ctas : 1);
  int64_t maxs = range / 128;
  if (maxs < 1) maxs = 1;
  if (target > maxs) target = maxs;
  if (target > 256) target = 256;
  return (int)(target < 1 ? 1 : target);
}

namespace {

constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeArgs {
  const void* q; int64_t q_sb, q_sh;
  const void* kc; const void* vc; int64_t c_sb, c_sh, c_ss;
  const int32_t* seqlens; int64_t max_seqlen;
  void* o; int64_t o_sb, o_sh;
  int Hq, Hkv, G;  // G = Hq / Hkv
  int64_t window_left;
  float scale_log2;
  int num_splits;
  float* ws_o;    // [B, Hq, splits, D]
  float* ws_lse;  // [B, Hq, splits]
};

template <typename T, int D, int GP>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(DecodeArgs p) {
  pdl_wait();
  pdl_trigger();
  constexpr int LG = D / 8;            // lanes per stream
  constexpr int NS = kThreads / LG;    // streams per CTA
  constexpr int U = 4;                 // keys per step
  __shared__ float sm_m[NS][GP];
  __shared__ float sm_l[NS][GP];
  __shared__ float sm_acc[NS][GP][D];

  const int split = blockIdx.x;
  const int passes = (p.G + GP - 1) / GP;
  const int kvh = blockIdx.y / passes;
  const int pass = blockIdx.y % passes;
  const int b = blockIdx.z;
  const int stream = threadIdx.x / LG;
  const int ln = threadIdx.x % LG;
  const int h0 = kvh * p.G + pass * GP;          // first q head of this pass
  const int nh = min(GP, p.G - pass * GP);        // heads in this pass

  const int64_t L = p.seqlens ? (int64_t)p.seqlens[b] : p.max_seqlen;
  int64_t lo = 0;
  if (p.window_left >= 0) lo = max((int64_t)0, L - 1 - p.window_left);
  const int64_t n = L > lo ? L - lo : 0;
  const int64_t per = (n + p.num_splits - 1) / p.num_splits;
  const int64_t k0 = lo + (int64_t)split * per;
  const int64_t k1 = min(L, k0 + per);

  const T* Q = static_cast<const T*>(p.q);
  float q[GP][8];
#pragma unroll
  for (int g = 0; g < GP; ++g) {
    if (g < nh) {
      unpack8<T>(__ldg(reinterpret_cast<const uint4*>(Q + b * p.q_sb + (int64_t)(h0 + g) * p.q_sh) + ln), q[g]);
#pragma unroll
      for (int j = 0; j < 8; ++j) q[g][j] *= p.scale_log2;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) q[g][j] = 0.f;
    }
  }
  float m[GP], l[GP], acc[GP][8];
#pragma unroll
  for (int g = 0; g < GP; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[g][j] = 0.f;
  }

  const T* Kb = static_cast<const T*>(p.kc) + b * p.c_sb + (int64_t)kvh * p.c_sh + ln * 8;
  const T* Vb = static_cast<const T*>(p.vc) + b * p.c_sb + (int64_t)kvh * p.c_sh + ln * 8;
  const uint4 z = make_uint4(0, 0, 0, 0);

  // The trip count is uniform across the CTA (the shuffles below need whole
  // warps); keys past k1 are masked.
  // Register double buffer: the rows of the next step are requested before
  // the current step's math, so each stream always has 2*U K/V rows in flight.
  uint4 nk[U], nv[U];
  auto fetch = [&](int64_t it) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t key = it + stream + (int64_t)u * NS;
      const bool ok = key < k1;
      nk[u] = ok ? ldg_nc_v4(Kb + key * p.c_ss) : z;
      nv[u] = ok ? ldg_nc_v4(Vb + key * p.c_ss) : z;
    }
  };
  fetch(k0);
  for (int64_t it = k0; it < k1; it += (int64_t)NS * U) {
    const int64_t base = it + stream;
    uint4 kr[U], vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) { kr[u] = nk[u]; vr[u] = nv[u]; }
    fetch(it + (int64_t)NS * U);
    float s[U][GP];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float kf[8];
      unpack8<T>(kr[u], kf);
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        float d = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) d = fmaf(q[g][j], kf[j], d);
#pragma unroll
        for (int o = LG / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        s[u][g] = (base + (int64_t)u * NS < k1) ? d : -INFINITY;
      }
    }
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < U; ++u) mx = fmaxf(mx, s[u][g]);
      const float corr = (mx == -INFINITY) ? 1.f : exp2f(m[g] - mx);
      m[g] = mx;
      l[g] *= corr;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[g][j] *= corr;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float pr = (s[u][g] == -INFINITY) ? 0.f : exp2f(s[u][g] - mx);
        l[g] += pr;
        s[u][g] = pr;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float vf[8];
      unpack8<T>(vr[u], vf);
#pragma unroll
      for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g][j] = fmaf(s[u][g], vf[j], acc[g][j]);
    }
  }

  // ---- merge the NS streams ----
#pragma unroll
  for (int g = 0; g < GP; ++g) {
    if (ln == 0) { sm_m[stream][g] = m[g]; sm_l[stream][g] = l[g]; }
#pragma unroll
    for (int j = 0; j < 8; ++j) sm_acc[stream][g][ln * 8 + j] = acc[g][j];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < GP * D; e += kThreads) {
    const int g = e / D, d = e % D;
    if (g >= nh) continue;
    float M = -INFINITY;
#pragma unroll 4
    for (int s2 = 0; s2 < NS; ++s2) M = fmaxf(M, sm_m[s2][g]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll 4
      for (int s2 = 0; s2 < NS; ++s2) {
        const float w = (sm_m[s2][g] == -INFINITY) ? 0.f : exp2f(sm_m[s2][g] - M);
        Ls += sm_l[s2][g] * w;
        O += sm_acc[s2][g][d] * w;
      }
    }
    const int h = h0 + g;
    if (p.num_splits == 1) {
      T* out = static_cast<T*>(p.o) + b * p.o_sb + (int64_t)h * p.o_sh;
      out[d] = from_f32<T>(Ls > 0.f ? O / Ls : 0.f);
    } else {
      const int64_t slot = ((int64_t)b * p.Hq + h) * p.num_splits + split;
      p.ws_o[slot * D + d] = Ls > 0.f ? O / Ls : 0.f;
      if (d == 0) p.ws_lse[slot] = (Ls > 0.f) ? M + log2f(Ls) : -INFINITY;
    }
  }
}

// One warp per (batch, q head): merges the splits' (o, lse) partials.
template <typename T, int D>
__global__ void __launch_bounds__(256) decode_combine_kernel(DecodeArgs p, int64_t B) {
  pdl_wait();
  pdl_trigger();
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= B * p.Hq) return;
  const int64_t b = wid / p.Hq;
  const int h = (int)(wid % p.Hq);
  const float* lse = p.ws_lse + wid * p.num_splits;
  float M = -INFINITY;
  for (int s = lane; s < p.num_splits; s += 32) M = fmaxf(M, lse[s]);
  M = warp_max(M);
  float wsum = 0.f;
  for (int s = lane; s < p.num_splits; s += 32)
    wsum += (lse[s] == -INFINITY) ? 0.f : exp2f(lse[s] - M);
  wsum = warp_sum(wsum);
  constexpr int PER = D / 32;
  float o[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) o[i] = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < p.num_splits; ++s) {
      const float ls = lse[s];
      if (ls == -INFINITY) continue;
      const float w = exp2f(ls - M) / wsum;
      const float* src = p.ws_o + (wid * p.num_splits + s) * D;
#pragma unroll
      for (int i = 0; i < PER; ++i) o[i] = fmaf(w, src[lane + 32 * i], o[i]);
    }
  }
  T* out = static_cast<T*>(p.o) + b * p.o_sb + (int64_t)h * p.o_sh;
#pragma unroll
  for (int i = 0; i < PER; ++i) out[lane + 32 * i] = from_f32<T>(o[i]);
}

template <typename T, int D>
int decode_launch(DecodeArgs& a, int64_t B, cudaStream_t st) {
  const int gp = a.G >= 8 ? 8 : (a.G >= 4 ? 4 : (a.G >= 2 ? 2 : 1));
  const int passes = (a.G + gp - 1) / gp;
  dim3 grid((unsigned)a.num_splits, (unsigned)(a.Hkv * passes), (unsigned)B);
  int rc = TPP_OK;
  switch (gp) {
    case 1: rc = launch("decode_attn_kernel", decode_attn_kernel<T, D, 1>, dim3(grid), dim3(kThreads), 0, st, 0, a); break;
    case 2: rc = launch("decode_attn_kernel", decode_attn_kernel<T, D, 2>, dim3(grid), dim3(kThreads), 0, st, 0, a); break;
    case 4: rc = launch("decode_attn_kernel", decode_attn_kernel<T, D, 4>, dim3(grid), dim3(kThreads), 0, st, 0, a); break;
    default: rc = launch("decode_attn_kernel", decode_attn_kernel<T, D, 8>, dim3(grid), dim3(kThreads), 0, st, 0, a); break;
  }
  if (rc != TPP_OK || a.num_splits == 1) return rc;
  const int64_t warps = B * a.Hq;
  const int64_t blocks = (warps * 32 + 255) / 256;
  return launch("decode_combine_kernel", decode_combine_kernel<T, D>, dim3((unsigned)blocks),
                dim3(256), 0, st, 0, a, B);
}

}  // namespace

int64_t attn_decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t range, int64_t D) {
  if (D == 64 || D == 128) {
    // tensor-core path: up to 8 splits merge inside a cluster, more go
    // through the workspace
    const int s = decode_mma_splits(B, Hq, Hkv, range);
    if (s <= 8) return 0;
    return B * Hq * (int64_t)s * (D + 1) * (int64_t)sizeof(float) + 256;
  }
  const int s = attn_decode_num_splits(B, Hq, Hkv, range);
  if (s <= 1) return 0;
  return B * Hq * (int64_t)s * (D + 1) * (int64_t)sizeof(float) + 256;
}

// Shared by the public entry point and by any variant that brings its own
// workspace; `ws` must hold attn_decode_workspace_bytes(...) bytes.
// Fused-mode inputs of tpp_attention_decode_qkv (see DecMmaArgs).
struct FusedQkv {
  const void* qkv; int64_t qkv_sb;
  const void* qn_w; const void* kn_w; float eps;
  const void* cosp; const void* sinp; int64_t cs_stride;
  const int32_t* positions;
};

// Paged caches (see DecMmaArgs): block pools [num_blocks][Hkv][64][D].
struct PagedKv {
  const int32_t* table; int64_t tbl_stride; int64_t num_blocks;
};

int attn_decode_run(const void* q, int64_t q_sb, int64_t q_sh, const void* k_cache,
                    const void* v_cache, int64_t c_sb, int64_t c_sh, int64_t c_ss,
                    const int32_t* seqlens, int64_t max_seqlen, void* o, int64_t o_sb,
                    int64_t o_sh, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                    int64_t window_left, float scale, void* ws, int64_t ws_bytes, int dtype,
                    cudaStream_t st, const FusedQkv* fz = nullptr, const PagedKv* pg = nullptr) {
  if (B == 0) return TPP_OK;
  TPP_REQUIRE((q || fz) && k_cache && v_cache && o, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(!fz || D == 64 || D == 128, TPP_ERR_UNSUPPORTED,
              "the fused q/k norm + RoPE decode path needs head dim 64 or 128");
  TPP_REQUIRE(!pg || D == 64 || D == 128, TPP_ERR_UNSUPPORTED,
              "paged decode attention needs head dim 64 or 128");
  if (pg) {  // pool layout is fixed: strides implied
    TPP_REQUIRE(pg->table && pg->num_blocks > 0 && pg->tbl_stride >= (max_seqlen + 63) / 64,
                TPP_ERR_SHAPE, "block table must cover max_seqlen (64-key blocks)");
    c_ss = D; c_sh = 64 * D; c_sb = Hkv * 64 * D;
  }
  TPP_REQUIRE(B >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0, TPP_ERR_SHAPE,
              "Hq must be a positive multiple of Hkv");
  TPP_REQUIRE(D == 64 || D == 128 || D == 256, TPP_ERR_UNSUPPORTED, "head dim must be 64, 128 or 256");
  TPP_REQUIRE(max_seqlen >= 0, TPP_ERR_SHAPE, "max_seqlen < 0");
  TPP_REQUIRE(q_sb % 8 == 0 && q_sh % 8 == 0 && c_sb % 8 == 0 && c_sh % 8 == 0 && c_ss % 8 == 0,
              TPP_ERR_ALIGN, "strides must be multiples of 8 elements");
  TPP_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache), TPP_ERR_ALIGN,
              "q/cache pointers must be 16-byte aligned");
  if (B == 0) return TPP_OK;
  int64_t range = max_seqlen;
  if (window_left >= 0 && window_left + 1 < range) range = window_left + 1;
  if (D == 64 || D == 128) {
    TPP_REQUIRE(c_ss == D, TPP_ERR_ALIGN, "cache rows must be contiguous (seq stride == head dim)");
    DecMmaArgs m = {};
    m.q = q; m.q_sb = q_sb; m.q_sh = q_sh;
    if (fz) {
      m.qkv = fz->qkv; m.qkv_sb = fz->qkv_sb;
      m.qn_w = fz->qn_w; m.kn_w = fz->kn_w; m.eps = fz->eps;
      m.cosp = fz->cosp; m.sinp = fz->sinp; m.cs_stride = fz->cs_stride;
      m.positions = fz->positions;
      m.kc = const_cast<void*>(k_cache); m.vc = const_cast<void*>(v_cache);
      m.c_sb = c_sb; m.c_sh = c_sh; m.c_ss = c_ss;
    }
    if (pg) {
      m.table = pg->table; m.tbl_stride = pg->tbl_stride; m.num_blocks = pg->num_blocks;
    }
    m.o = o; m.o_sb = o_sb; m.o_sh = o_sh;
    m.seqlens = seqlens; m.max_seqlen = max_seqlen;
    m.Hq = (int)Hq; m.Hkv = (int)Hkv; m.G = (int)(Hq / Hkv); m.passes = 1;
    m.window_left = window_left;
    m.scale_log2 = scale * kLog2e;
    m.splits = decode_mma_splits(B, Hq, Hkv, range);
    m.cluster = 1;
    m.ws_o = nullptr; m.ws_lse = nullptr;
    m.err = device_error_flag();
    if (m.splits > 8) {
      const int64_t need = attn_decode_workspace_bytes(B, Hq, Hkv, range, D);
      TPP_REQUIRE(ws != nullptr && ws_bytes >= need, TPP_ERR_WORKSPACE,
                  "workspace too small: need " + std::to_string(need) + " bytes");
      TPP_REQUIRE(aligned16(ws), TPP_ERR_ALIGN, "workspace must be 16-byte aligned");
      m.ws_o = static_cast<float*>(ws);
      m.ws_lse = m.ws_o + B * Hq * (int64_t)m.splits * D;
    }
    int rc = decode_mma_launch(m, k_cache, v_cache, c_sb, c_sh, c_ss, B, D, dtype, st);
    if (rc != TPP_OK || m.splits <= 8) return rc;
    DecodeArgs a;
    a.o = o; a.o_sb = o_sb; a.o_sh = o_sh; a.Hq = (int)Hq; a.num_splits = m.splits;
    a.ws_o = m.ws_o; a.ws_lse = m.ws_lse;
    const int64_t blocks = (B * Hq * 32 + 255) / 256;
    return TPP_DISPATCH_HALF(dtype, T, [&] {
      return D == 64 ? launch("decode_combine_kernel", decode_combine_kernel<T, 64>,
                              dim3((unsigned)blocks), dim3(256), 0, st, 0u, a, B)
                     : launch("decode_combine_kernel", decode_combine_kernel<T, 128>,
                              dim3((unsigned)blocks), dim3(256), 0, st, 0u, a, B);
    });
  }
  DecodeArgs a;
  a.q = q; a.q_sb = q_sb; a.q_sh = q_sh;
  a.kc = k_cache; a.vc = v_cache; a.c_sb = c_sb; a.c_sh = c_sh; a.c_ss = c_ss;
  a.seqlens = seqlens; a.max_seqlen = max_seqlen;
  a.o = o; a.o_sb = o_sb; a.o_sh = o_sh;
  a.Hq = (int)Hq; a.Hkv = (int)Hkv; a.G = (int)(Hq / Hkv);
  a.window_left = window_left;
  a.scale_log2 = scale * kLog2e;
  a.num_splits = attn_decode_num_splits(B, Hq, Hkv, range);
  a.ws_o = nullptr; a.ws_lse = nullptr;
  if (a.num_splits > 1) {
    const int64_t need = attn_decode_workspace_bytes(B, Hq, Hkv, range, D);
    TPP_REQUIRE(ws != nullptr && ws_bytes >= need, TPP_ERR_WORKSPACE,
                "workspace too small: need " + std::to_string(need) + " bytes");
    TPP_REQUIRE(aligned16(ws), TPP_ERR_ALIGN, "workspace must be 16-byte aligned");
    a.ws_o = static_cast<float*>(ws);
    a.ws_lse = a.ws_o + B * Hq * (int64_t)a.num_splits * D;
  }
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    switch (D) {
      case 64: return decode_launch<T, 64>(a, B, st);
      case 128: return decode_launch<T, 128>(a, B, st);
      default: return decode_launch<T, 256>(a, B, st);
    }
  });
}

}  // namespace tpp

using namespace tpp;

extern "C" int64_t tpp_attention_decode_workspace(int64_t B, int64_t Hq, int64_t max_seqlen,
                                                  int64_t D) {
  // Hkv only changes the split count through the CTA count; the bound below
  // uses Hkv = 1 (fewest CTAs, most splits), which covers every Hkv.
  int64_t worst = 0;
  for (int64_t hkv = 1; hkv <= Hq; ++hkv) {
    if (Hq % hkv) continue;
    const int64_t b = attn_decode_workspace_bytes(B, Hq, hkv, max_seqlen, D);
    if (b > worst) worst = b;
  }
  return worst;
}

extern "C" int64_t tpp_attention_decode_workspace_exact(int64_t B, int64_t Hq, int64_t Hkv,
                                                        int64_t max_seqlen, int64_t D,
                                                        int64_t window_left) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || D <= 0 || max_seqlen <= 0) return 0;
  int64_t range = max_seqlen;
  if (window_left >= 0 && window_left + 1 < range) range = window_left + 1;
  return attn_decode_workspace_bytes(B, Hq, Hkv, range, D);
}

extern "C" int tpp_attention_decode(const void* q, int64_t q_sb, int64_t q_sh,
                                    const void* k_cache, const void* v_cache, int64_t c_sb,
                                    int64_t c_sh, int64_t c_ss, const int32_t* seqlens,
                                    int64_t max_seqlen, void* o, int64_t o_sb, int64_t o_sh,
                                    int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                    int64_t window_left, float scale, void* workspace,
                                    int64_t workspace_bytes, int dtype, void* stream) {
  return attn_decode_run(q, q_sb, q_sh, k_cache, v_cache, c_sb, c_sh, c_ss, seqlens, max_seqlen,
                         o, o_sb, o_sh, B, Hq, Hkv, D, window_left, scale, workspace,
                         workspace_bytes, dtype, as_stream(stream));
}

extern "C" int tpp_attention_decode_qkv(
    const void* qkv, int64_t ld_qkv, const void* qn_w, const void* kn_w, float eps,
    const void* cos, const void* sin, int64_t cs_stride, int cs_dtype,
    const int32_t* positions, void* k_cache, void* v_cache, int64_t c_sb, int64_t c_sh,
    int64_t c_ss, const int32_t* seqlens, int64_t max_seqlen, void* o, int64_t o_sb,
    int64_t o_sh, int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t window_left,
    float scale, void* workspace, int64_t workspace_bytes, int dtype, void* stream) {
  if (B == 0) return TPP_OK;
  TPP_REQUIRE(qkv && cos && sin && positions && seqlens, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(cs_dtype == TPP_F16, TPP_ERR_DTYPE, "RoPE tables must be fp16 (compute_rope_params)");
  TPP_REQUIRE(ld_qkv >= (Hq + 2 * Hkv) * D, TPP_ERR_SHAPE, "qkv row shorter than (Hq+2Hkv)*D");
  TPP_REQUIRE(cs_stride >= D, TPP_ERR_SHAPE, "RoPE table row shorter than D");
  FusedQkv fz{qkv, ld_qkv, qn_w, kn_w, eps, cos, sin, cs_stride, positions};
  return attn_decode_run(nullptr, 0, 0, k_cache, v_cache, c_sb, c_sh, c_ss, seqlens, max_seqlen,
                         o, o_sb, o_sh, B, Hq, Hkv, D, window_left, scale, workspace,
                         workspace_bytes, dtype, as_stream(stream), &fz);
}

extern "C" int tpp_attention_decode_paged(
    const void* q, int64_t q_sb, int64_t q_sh, const void* k_pool, const void* v_pool,
    int64_t num_blocks, const int32_t* block_table, int64_t table_stride,
    const int32_t* seqlens, int64_t max_seqlen, void* o, int64_t o_sb, int64_t o_sh, int64_t B,
    int64_t Hq, int64_t Hkv, int64_t D, int64_t window_left, float scale, void* workspace,
    int64_t workspace_bytes, int dtype, void* stream) {
  if (B == 0) return TPP_OK;
  TPP_REQUIRE(seqlens, TPP_ERR_SHAPE, "paged decode needs per-sequence lengths");
  PagedKv pg{block_table, table_stride, num_blocks};
  return attn_decode_run(q, q_sb, q_sh, k_pool, v_pool, 0, 0, 0, seqlens, max_seqlen, o, o_sb,
                         o_sh, B, Hq, Hkv, D, window_left, scale, workspace, workspace_bytes,
                         dtype, as_stream(stream), nullptr, &pg);
}

extern "C" int tpp_attention_decode_qkv_paged(
    const void* qkv, int64_t ld_qkv, const void* qn_w, const void* kn_w, float eps,
    const void* cos, const void* sin, int64_t cs_stride, int cs_dtype,
    const int32_t* positions, void* k_pool, void* v_pool, int64_t num_blocks,
    const int32_t* block_table, int64_t table_stride, const int32_t* seqlens,
    int64_t max_seqlen, void* o, int64_t o_sb, int64_t o_sh, int64_t B, int64_t Hq, int64_t Hkv,
    int64_t D, int64_t window_left, float scale, void* workspace, int64_t workspace_bytes,
    int dtype, void* stream) {
  if (B == 0) return TPP_OK;
  TPP_REQUIRE(qkv && cos && sin && positions && seqlens, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(cs_dtype == TPP_F16, TPP_ERR_DTYPE, "RoPE tables must be fp16 (compute_rope_params)");
  TPP_REQUIRE(ld_qkv >= (Hq + 2 * Hkv) * D, TPP_ERR_SHAPE, "qkv row shorter than (Hq+2Hkv)*D");
  TPP_REQUIRE(cs_stride >= D, TPP_ERR_SHAPE, "RoPE table row shorter than D");
  FusedQkv fz{qkv, ld_qkv, qn_w, kn_w, eps, cos, sin, cs_stride, positions};
  PagedKv pg{block_table, table_stride, num_blocks};
  return attn_decode_run(nullptr, 0, 0, k_pool, v_pool, 0, 0, 0, seqlens, max_seqlen, o, o_sb,
                         o_sh, B, Hq, Hkv, D, window_left, scale, workspace, workspace_bytes,
                         dtype, as_stream(stream), &fz, &pg);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of tpp_attention_decode.
//
// Some callers cannot allocate device memory at the point where they decode:
// code running inside a custom allocator or memory-pool callback, runtimes
// that forbid cudaMalloc after start-up (fixed memory budgets, real-time
// serving loops), and plain-C hosts that have no allocator of their own to
// hand a workspace from.  This entry point keeps the split-KV partial results
// in a fixed scratch array that lives in this library's device image instead
// of a caller workspace.  It never calls cudaMalloc/cudaFree.
//
// Limits and sharing: the array holds kNoAllocScratchBytes (8 MiB) on every
// GPU that loads the library, until the process exits.  Every call on a
// device uses the same array, so calls whose kernels overlap on the GPU (two
// streams at once, or two host threads) race on it; serialise them.  Nothing
// in the array has to start at zero: each call writes every partial it later
// reads.  The first call on each device looks up the array's device address
// (cudaGetSymbolAddress) -- make that first call before any stream capture.
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kNoAllocScratchBytes = 8ll << 20;
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];
constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("tpp_attention_decode_noalloc: no usable current CUDA device");
    return TPP_ERR_LAUNCH;
  }
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error(std::string("tpp_attention_decode_noalloc: cudaGetSymbolAddress failed: ") +
                cudaGetErrorString(e));
      return TPP_ERR_LAUNCH;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TPP_OK;
}
}  // namespace

extern "C" int64_t tpp_attention_decode_noalloc_max_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int tpp_attention_decode_noalloc(const void* q, int64_t q_sb, int64_t q_sh,
                                            const void* k_cache, const void* v_cache,
                                            int64_t c_sb, int64_t c_sh, int64_t c_ss,
                                            const int32_t* seqlens, int64_t max_seqlen, void* o,
                                            int64_t o_sb, int64_t o_sh, int64_t B, int64_t Hq,
                                            int64_t Hkv, int64_t D, int64_t window_left,
                                            float scale, int dtype, void* stream) {
  if (B == 0) return TPP_OK;
  TPP_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && D > 0 && max_seqlen >= 0,
              TPP_ERR_SHAPE, "bad sizes");
  int64_t range = max_seqlen;
  if (window_left >= 0 && window_left + 1 < range) range = window_left + 1;
  const int64_t need = attn_decode_workspace_bytes(B, Hq, Hkv, range, D);
  TPP_REQUIRE(need <= kNoAllocScratchBytes, TPP_ERR_WORKSPACE,
              "this shape needs " + std::to_string(need) + " bytes of split-KV scratch, more "
              "than the fixed " + std::to_string(kNoAllocScratchBytes) +
              " bytes; use tpp_attention_decode with a caller workspace");
  void* ws = nullptr;
  if (need > 0) {
    const int rc = scratch_for_current_device(&ws);
    if (rc != TPP_OK) return rc;
  }
  return attn_decode_run(q, q_sb, q_sh, k_cache, v_cache, c_sb, c_sh, c_ss, seqlens, max_seqlen,
                         o, o_sb, o_sh, B, Hq, Hkv, D, window_left, scale, ws,
                         kNoAllocScratchBytes, dtype, as_stream(stream));
}
