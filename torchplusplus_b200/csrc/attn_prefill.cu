// Flash attention forward for q_len >= 1 (prefill / chunked prefill):
// GQA/MQA by head mapping, bottom-right-aligned causal mask, sliding window,
// arbitrary (batch, seq, head) strides so both the BSHD activations and the
// BHSD KV cache are read in place.
//
// Semantics: flash_attn_func(q, k, v, causal, window_size=(w-1, 0)) as torchpp
// calls it (torchpp/attention/gqa.py:128, swa.py:85-89); GQA replaces the
// repeat_interleave of gqa.py:120-121 (kv head = q head / (Hq/Hkv)).
//
// This is the register-tile tensor-core version (m16n8k16 MMAs, fragments
// fed by ldmatrix from XOR-swizzled shared memory, cp.async double-buffered
// K/V tiles, fp32 online softmax in the exp2 domain).  CTA = 4 warps x 16
// query rows; K/V blocks of 64 keys.
#include <math.h>
#include "mma_common.cuh"

namespace tpp {
namespace {

constexpr int BLOCK_M = 64;
constexpr int BLOCK_N = 64;
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

struct PrefillArgs {
  const void* q; int64_t q_sb, q_ss, q_sh;
  const void* k; int64_t k_sb, k_ss, k_sh;
  const void* v; int64_t v_sb, v_ss, v_sh;
  void* o; int64_t o_sb, o_ss, o_sh;
  int Sq, Sk, Hq, Hkv;
  int causal;
  int64_t window_left;
  float scale_log2;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Tile of R rows x D elements, rows of D*2 bytes, 16-byte chunks XOR-swizzled
// by (row & 7) so that ldmatrix's 8 row addresses hit 8 different bank groups.
template <int D>
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + row * (D * 2) + ((chunk ^ (row & 7)) << 4);
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) prefill_attn_kernel(PrefillArgs p) {
  pdl_wait();
  pdl_trigger();
  constexpr int CH = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const uint32_t sK0 = sQ + BLOCK_M * D * 2;
  const uint32_t sV0 = sK0 + 2 * BLOCK_N * D * 2;
  constexpr uint32_t kTile = BLOCK_N * D * 2;

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;

  const T* Q = static_cast<const T*>(p.q) + b * p.q_sb + (int64_t)h * p.q_sh;
  const T* K = static_cast<const T*>(p.k) + b * p.k_sb + (int64_t)kvh * p.k_sh;
  const T* V = static_cast<const T*>(p.v) + b * p.v_sb + (int64_t)kvh * p.v_sh;
  const int q0 = qb * BLOCK_M;
  const int off = p.Sk - p.Sq;  // absolute position of query i is i + off

  // key range touched by this query block
  const int qp_lo = q0 + off, qp_hi = min(q0 + BLOCK_M, p.Sq) - 1 + off;
  int k_end = p.Sk;
  if (p.causal) k_end = min(k_end, qp_hi + 1);
  int k_beg = 0;
  if (p.window_left >= 0) k_beg = (int)max((int64_t)0, (int64_t)qp_lo - p.window_left);
  k_beg = (k_beg / BLOCK_N) * BLOCK_N;

  // ---- Q tile -> smem -> A fragments ----
  for (int i = tid; i < BLOCK_M * CH; i += kThreads) {
    const int r = i / CH, ch = i % CH;
    const bool ok = q0 + r < p.Sq;
    cp_async16(swz<D>(sQ, r, ch), Q + (int64_t)(ok ? q0 + r : 0) * p.q_ss + ch * 8, ok);
  }
  cp_async_commit();

  auto load_kv = [&](int kb, int stage) {
    const int k0 = kb;
    for (int i = tid; i < BLOCK_N * CH; i += kThreads) {
      const int r = i / CH, ch = i % CH;
      const bool ok = k0 + r < p.Sk;
      const int64_t row = ok ? k0 + r : 0;
      cp_async16(swz<D>(sK0 + stage * kTile, r, ch), K + row * p.k_ss + ch * 8, ok);
      cp_async16(swz<D>(sV0 + stage * kTile, r, ch), V + row * p.v_ss + ch * 8, ok);
    }
    cp_async_commit();
  };

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

  const bool any = k_beg < k_end;
  if (any) load_kv(k_beg, 0);
  cp_async_wait<0>();  // Q (and possibly the first K/V) resident
  __syncthreads();
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int ch = ks * 2 + (lane >> 4);
    ldsm_x4(swz<D>(sQ, r, ch), qf[ks]);
  }

  const int row_a = q0 + warp * 16 + g;  // this thread's two query rows: row_a, row_a + 8
  int stage = 0;
  for (int kb = k_beg; kb < k_end; kb += BLOCK_N, stage ^= 1) {
    if (kb + BLOCK_N < k_end) {
      load_kv(kb + BLOCK_N, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + stage * kTile, sV = sV0 + stage * kTile;

    // S = Q K^T : 16 rows x 64 keys per warp
    float s[BLOCK_N / 8][4];
#pragma unroll
    for (int j = 0; j < BLOCK_N / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int jp = 0; jp < BLOCK_N / 16; ++jp) {
        uint32_t bf[4];
        const int r = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int ch = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(swz<D>(sK, r, ch), bf);
        mma<T>(s[2 * jp], qf[ks], bf[0], bf[1]);
        mma<T>(s[2 * jp + 1], qf[ks], bf[2], bf[3]);
      }
    }
    // scale (log2 domain) + mask
    const bool need_mask = (kb + BLOCK_N > p.Sk) || (p.causal && kb + BLOCK_N - 1 > qp_lo) ||
                           (p.window_left >= 0 && kb < (int64_t)qp_hi - p.window_left);
#pragma unroll
    for (int j = 0; j < BLOCK_N / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * p.scale_log2;
        if (need_mask) {
          const int key = kb + j * 8 + 2 * c + (e & 1);
          const int qp = row_a + ((e >> 1) ? 8 : 0) + off;
          bool ok = key < p.Sk;
          if (p.causal) ok = ok && key <= qp;
          if (p.window_left >= 0) ok = ok && (int64_t)key >= (int64_t)qp - p.window_left;
          if (!ok) v = -INFINITY;
        }
        s[j][e] = v;
      }
    }
    // online softmax (rows g and g+8; the 4 lanes of a quad share a row)
    float corr[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = m_r[hr];
#pragma unroll
      for (int j = 0; j < BLOCK_N / 8; ++j) mx = fmaxf(mx, fmaxf(s[j][2 * hr], s[j][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      corr[hr] = (mx == -INFINITY) ? 1.f : exp2f(m_r[hr] - mx);
      m_r[hr] = mx;
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < BLOCK_N / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = s[j][2 * hr + e];
          const float pv = (v == -INFINITY) ? 0.f : exp2f(v - mx);
          s[j][2 * hr + e] = pv;
          sum += pv;
        }
      }
      l_r[hr] = l_r[hr] * corr[hr] + sum;  // quad-partial; reduced at the end
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= corr[0]; o[i][1] *= corr[0];
      o[i][2] *= corr[1]; o[i][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BLOCK_N / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bf[4];
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = dp * 2 + (lane >> 4);
        ldsm_x4_t(swz<D>(sV, r, ch), bf);
        mma<T>(o[2 * dp], pa, bf[0], bf[1]);
        mma<T>(o[2 * dp + 1], pa, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }

  // ---- normalise and store ----
  float inv[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = l_r[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    inv[hr] = l > 0.f ? 1.f / l : 0.f;
  }
  T* O = static_cast<T*>(p.o) + b * p.o_sb + (int64_t)h * p.o_sh;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = row_a + hr * 8;
    if (row >= p.Sq) continue;
    T* orow = O + (int64_t)row * p.o_ss;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const uint32_t v = pack2<T>(o[i][2 * hr] * inv[hr], o[i][2 * hr + 1] * inv[hr]);
      *reinterpret_cast<uint32_t*>(orow + i * 8 + 2 * c) = v;
    }
  }
}

template <typename T, int D>
int prefill_launch(const PrefillArgs& a, int64_t B, cudaStream_t st) {
  const size_t smem = (size_t)(BLOCK_M + 4 * BLOCK_N) * D * 2;
  auto kern = prefill_attn_kernel<T, D>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess) {
    set_error("prefill_attn_kernel: cannot reserve shared memory");
    return TPP_ERR_LAUNCH;
  }
  dim3 grid((unsigned)((a.Sq + BLOCK_M - 1) / BLOCK_M), (unsigned)a.Hq, (unsigned)B);
  return launch("prefill_attn_kernel", kern, dim3(grid), dim3(kThreads), smem, st, 0, a);
}

}  // namespace
int attn_prefill_tc(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, const void* k,
                    int64_t k_sb, int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb,
                    int64_t v_ss, int64_t v_sh, void* o, int64_t o_sb, int64_t o_ss,
                    int64_t o_sh, int64_t B, int64_t Sq, int64_t Sk, int64_t Hq, int64_t Hkv,
                    int64_t Dh, int causal, int64_t window_left, float scale, int dtype,
                    cudaStream_t st);

}  // namespace tpp

using namespace tpp;

extern "C" int tpp_attention_prefill(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh,
                                     const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                                     const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                                     void* o, int64_t o_sb, int64_t o_ss, int64_t o_sh, int64_t B,
                                     int64_t Sq, int64_t Sk, int64_t Hq, int64_t Hkv, int64_t D,
                                     int causal, int64_t window_left, float scale, int dtype,
                                     void* stream) {
  if (B == 0 || Sq == 0) return TPP_OK;
  TPP_REQUIRE(q && k && v && o, TPP_ERR_SHAPE, "null pointer");
  TPP_REQUIRE(B >= 0 && Sq >= 0 && Sk >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0, TPP_ERR_SHAPE,
              "Hq must be a positive multiple of Hkv");
  TPP_REQUIRE(Sq <= 0x7fffffff && Sk <= 0x7fffffff && B <= 65535 && Hq <= 65535, TPP_ERR_SHAPE,
              "sizes exceed kernel limits");
  TPP_REQUIRE(D == 64 || D == 128, TPP_ERR_UNSUPPORTED, "head dim must be 64 or 128");
  TPP_REQUIRE(q_sb % 8 == 0 && q_ss % 8 == 0 && q_sh % 8 == 0 && k_sb % 8 == 0 && k_ss % 8 == 0 &&
                  k_sh % 8 == 0 && v_sb % 8 == 0 && v_ss % 8 == 0 && v_sh % 8 == 0 &&
                  o_ss % 2 == 0 && o_sh % 2 == 0 && o_sb % 2 == 0,
              TPP_ERR_ALIGN, "q/k/v strides must be multiples of 8 elements");
  TPP_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) &&
                  (reinterpret_cast<uintptr_t>(o) & 3u) == 0,
              TPP_ERR_ALIGN, "q/k/v must be 16-byte aligned");
  if (B == 0 || Sq == 0) return TPP_OK;
  cudaStream_t st = as_stream(stream);
  if (D == 128) {
    const int rc = attn_prefill_tc(q, q_sb, q_ss, q_sh, k, k_sb, k_ss, k_sh, v, v_sb, v_ss, v_sh,
                                   o, o_sb, o_ss, o_sh, B, Sq, Sk, Hq, Hkv, D, causal,
                                   window_left, scale, dtype, st);
    if (rc != TPP_ERR_UNSUPPORTED) return rc;
  }
  PrefillArgs a;
  a.q = q; a.q_sb = q_sb; a.q_ss = q_ss; a.q_sh = q_sh;
  a.k = k; a.k_sb = k_sb; a.k_ss = k_ss; a.k_sh = k_sh;
  a.v = v; a.v_sb = v_sb; a.v_ss = v_ss; a.v_sh = v_sh;
  a.o = o; a.o_sb = o_sb; a.o_ss = o_ss; a.o_sh = o_sh;
  a.Sq = (int)Sq; a.Sk = (int)Sk; a.Hq = (int)Hq; a.Hkv = (int)Hkv;
  a.causal = causal; a.window_left = window_left;
  a.scale_log2 = scale * kLog2e;
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    return D == 64 ? prefill_launch<T, 64>(a, B, st) : prefill_launch<T, 128>(a, B, st);
  });
}
