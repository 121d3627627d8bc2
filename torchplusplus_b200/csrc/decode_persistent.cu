// The whole decode step of one sequence as ONE persistent, cooperative
// kernel (tpp_decode_step_persistent).
//
// At batch 1 the step is a chain of ~140 small dependent phases (five per
// layer); as separate launches every phase pays a kernel boundary and
// re-stages its operands, so the step runs at ~22% of HBM although its work
// is one pass over the weights.  Here one CTA per SM stays resident for the
// whole step:
//  * consumer warps 0..14 run the phases; a grid-wide barrier (an atomic
//    arrival count and a generation word in global memory, bounded waits)
//    separates a phase from the next one that reads its output;
//  * producer warp 15 streams this CTA's weight slice of every phase, in
//    phase order, through two 96 KB shared-memory slots with bulk copies
//    (cp.async.bulk, mbarrier completion).  Weights do not depend on the
//    barriers, so the next phases' slices are in flight (or resident) while
//    the current phase computes and waits;
//  * per layer: QKV (RMSNorm folded into the weights, each CTA a contiguous
//    row range) | attention (kv head x key-range units; q/k RMSNorm + RoPE
//    and the K/V append of the new token in the unit that owns its
//    position; the last unit of a head to finish merges the head's
//    partials) | o-proj + residual | gate/up + SwiGLU | down + residual;
//    then the LM head (row chunks, per-CTA argmax) and the token bookkeeping.
// GEMVs run on CUDA cores (one token: one weight byte is used once), a warp
// per output row, fp32 accumulation; every stored activation is rounded to
// the step's dtype as the launch-per-phase path rounds it.
#include <stdlib.h>
#include "tc_common.cuh"

namespace tpp {
namespace {

constexpr int kThr = 512;                // 15 consumer warps + 1 producer warp
constexpr int kCons = 480;
constexpr int kProdWarp = 15;
constexpr uint32_t kSlot = 96 * 1024;    // one weight slot
constexpr int kMaxG = 4;                 // query heads per kv head (at most)
constexpr int kTK = 256;                 // keys per attention tile
constexpr int kMaxCTAs = 256;
constexpr uint32_t kSpinLimit = 1u << 24;

#ifdef TPP_DEBUG_STAMPS
// [CTA < 256][512] globaltimer stamps of thread 0 (phase boundaries)
__device__ unsigned long long g_dp_stamps[256 * 512];
#define DP_TS(i) do { if (threadIdx.x == 0 && blockIdx.x < 256) { unsigned long long _t; \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(_t)); \
    g_dp_stamps[blockIdx.x * 512 + (i)] = _t; } } while (0)
#else
#define DP_TS(i) do {} while (0)
#endif

// Workspace layout (bytes, from a 256-aligned base): sync words, then the
// activations of the step.
struct Ws {
  uint32_t* count;      // barrier arrivals
  uint32_t* gen;        // barrier generation
  uint32_t* abortf;     // set when any wait gave up: every CTA winds down
  void* x;              // [E] residual stream (dtype)
  void* qkv;            // [(Hq+2Hkv) D]
  float* part;          // [Hq][S][D + 2] attention partials (o, m, l)
  void* o;              // [Hq D] merged attention output
  uint32_t* head_cnt;   // [Hkv] attention units finished (self-resetting)
  void* ff;             // [F] SwiGLU output
  float* amax_v;        // [CTAs] per-CTA best logit
  int* amax_i;          // [CTAs] its index
};

__host__ __device__ inline size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

__host__ __device__ inline size_t ws_layout(char* base, int64_t E, int64_t Hq, int64_t Hkv,
                                            int64_t D, int64_t F, Ws* w) {
  size_t off = 0;
  auto take = [&](size_t bytes) { char* p = base + off; off += al256(bytes); return p; };
  char* sync = take(256 + 4 * 64);
  char* x = take((size_t)E * 2);
  char* qkv = take((size_t)(Hq + 2 * Hkv) * D * 2);
  char* part = take((size_t)Hq * kMaxCTAs * (D + 2) * 4);
  char* o = take((size_t)Hq * D * 2);
  char* ff = take((size_t)F * 2);
  char* av = take((size_t)kMaxCTAs * 4);
  char* ai = take((size_t)kMaxCTAs * 4);
  if (w) {
    w->count = reinterpret_cast<uint32_t*>(sync);
    w->gen = reinterpret_cast<uint32_t*>(sync + 64);
    w->abortf = reinterpret_cast<uint32_t*>(sync + 128);
    w->x = x; w->qkv = qkv; w->o = o;
    w->head_cnt = reinterpret_cast<uint32_t*>(sync + 256); w->part = reinterpret_cast<float*>(part); w->ff = ff;
    w->amax_v = reinterpret_cast<float*>(av); w->amax_i = reinterpret_cast<int*>(ai);
  }
  return off;
}

struct StepArgs {
  const tpp_decode_layer* layers;
  int n_layers;
  const void* emb;
  const void* lm_head;
  const __half* cosp;
  const __half* sinp;
  int64_t cs_stride;
  int64_t* tokens;
  int32_t* positions;
  int32_t* seqlens;
  int64_t* out_ids;
  int64_t out_cap;
  void* logits;
  char* ws;
  int E, Hq, Hkv, D, F, V, Smax;
  float eps, scale_log2;
  int lm_rows_per_job;  // LM-head rows per weight job
  int* err;
};

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void cons_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCons) : "memory");
}

// Grid-wide barrier among the consumer warps of all CTAs: one 64-bit
// arrival counter that only grows (each barrier adds gridDim.x), so a
// barrier is one atomic add plus polling for the next multiple -- no reset
// and no second word.  `target` is this CTA's running target.  Returns false
// (every CTA then winds down) when a wait gave up or another CTA aborted.
__device__ __forceinline__ void grid_arrive(const Ws& w, unsigned long long& target) {
  cons_sync();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    __threadfence();
    atomicAdd(reinterpret_cast<unsigned long long*>(w.count), 1ull);
  }
}
__device__ bool grid_wait(const Ws& w, unsigned long long target, int* flag, int* err,
                          int code) {
  if (threadIdx.x == 0) {
    bool ok = true;
    const unsigned long long* cnt = reinterpret_cast<const unsigned long long*>(w.count);
    uint32_t i = 0;
    for (; i < kSpinLimit; ++i) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(cnt) : "memory");
      if (v >= target) break;
      if ((i & 255) == 255 && ld_acquire(w.abortf) != 0) { ok = false; break; }
    }
    if (i == kSpinLimit) {
      ok = false;
      if (err) atomicExch(err, code);
      atomicExch(w.abortf, 1u);
    }
    *flag = ok ? 1 : 0;
  }
  cons_sync();
  return *flag != 0;
}
__device__ __forceinline__ bool grid_sync(const Ws& w, unsigned long long& target, int* flag,
                                          int* err, int code) {
  grid_arrive(w, target);
  return grid_wait(w, target, flag, err, code);
}

template <typename T>
__device__ __forceinline__ float ldT(const void* p, int64_t i) {
  return to_f32(__ldcg(static_cast<const T*>(p) + i));
}
template <typename T>
__device__ __forceinline__ float rndT(float v) { return to_f32(from_f32<T>(v)); }

// xs[0..n) = src[0..n) (dtype -> fp32), 8 elements (16 bytes) per load
template <typename T>
__device__ __forceinline__ void load_vec(float* xs, const void* src, int n, int ctid) {
  const uint4* p = static_cast<const uint4*>(src);
  for (int i = ctid; i < n / 8; i += kCons) {
    float f[8];
    unpack8<T>(__ldcg(p + i), f);
    *reinterpret_cast<float4*>(xs + 8 * i) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(xs + 8 * i + 4) = make_float4(f[4], f[5], f[6], f[7]);
  }
}

// Row r of a [rows][K] slice in shared memory dotted with xs[K] (fp32),
// by one warp; returns the full sum in every lane.
template <typename T>
__device__ __forceinline__ float row_dot(const uint8_t* slot, int r, int K, const float* xs,
                                         int lane) {
  const T* w = reinterpret_cast<const T*>(slot) + (size_t)r * K;
  float acc = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(w + k);
    float f[8];
    unpack8<T>(v, f);
    const float4 a = *reinterpret_cast<const float4*>(xs + k);
    const float4 b = *reinterpret_cast<const float4*>(xs + k + 4);
    acc = fmaf(f[0], a.x, acc); acc = fmaf(f[1], a.y, acc);
    acc = fmaf(f[2], a.z, acc); acc = fmaf(f[3], a.w, acc);
    acc = fmaf(f[4], b.x, acc); acc = fmaf(f[5], b.y, acc);
    acc = fmaf(f[6], b.z, acc); acc = fmaf(f[7], b.w, acc);
  }
  return warp_sum(acc);
}

// Contiguous share [r0, r1) of `rows` for CTA c of G.
__device__ __forceinline__ void share(int rows, int c, int G, int& r0, int& r1) {
  r0 = (int)((int64_t)rows * c / G);
  r1 = (int)((int64_t)rows * (c + 1) / G);
}


// ---- weight jobs: this CTA's slice of every weighted phase, in order ------
// Job j < 4 L: layer j / 4, phase j % 4 (0 QKV, 1 o-proj, 2 gate/up, 3 down);
// then the LM head in chunks of lm_rows_per_job rows.
struct Job {
  const uint8_t* src0;
  uint32_t bytes0;
  const uint8_t* src1;   // gate/up: the up rows (placed after the gate rows)
  uint32_t bytes1;
};

__device__ __forceinline__ Job job_of(const StepArgs& a, int j, int c, int G) {
  Job jb = {nullptr, 0, nullptr, 0};
  const int esz = 2;
  if (j < 4 * a.n_layers) {
    const tpp_decode_layer& L = a.layers[j / 4];
    int r0, r1;
    switch (j % 4) {
      case 0: {
        share((a.Hq + 2 * a.Hkv) * a.D, c, G, r0, r1);
        jb.src0 = static_cast<const uint8_t*>(L.wqkv) + (size_t)r0 * a.E * esz;
        jb.bytes0 = (uint32_t)((r1 - r0) * a.E * esz);
        break;
      }
      case 1: {
        share(a.E, c, G, r0, r1);
        jb.src0 = static_cast<const uint8_t*>(L.wo) + (size_t)r0 * a.Hq * a.D * esz;
        jb.bytes0 = (uint32_t)((r1 - r0) * a.Hq * a.D * esz);
        break;
      }
      case 2: {
        share(a.F, c, G, r0, r1);
        jb.src0 = static_cast<const uint8_t*>(L.wgu) + (size_t)r0 * a.E * esz;
        jb.bytes0 = (uint32_t)((r1 - r0) * a.E * esz);
        jb.src1 = static_cast<const uint8_t*>(L.wgu) + (size_t)(a.F + r0) * a.E * esz;
        jb.bytes1 = jb.bytes0;
        break;
      }
      default: {
        share(a.E, c, G, r0, r1);
        jb.src0 = static_cast<const uint8_t*>(L.wdown) + (size_t)r0 * a.F * esz;
        jb.bytes0 = (uint32_t)((r1 - r0) * a.F * esz);
        break;
      }
    }
  } else {
    int v0, v1;
    share(a.V, c, G, v0, v1);
    const int q = j - 4 * a.n_layers;
    const int r0 = v0 + q * a.lm_rows_per_job;
    const int r1 = min(v1, r0 + a.lm_rows_per_job);
    jb.src0 = static_cast<const uint8_t*>(a.lm_head) + (size_t)r0 * a.E * esz;
    jb.bytes0 = r1 > r0 ? (uint32_t)((r1 - r0) * a.E * esz) : 0u;
  }
  return jb;
}

__device__ __forceinline__ int n_jobs(const StepArgs& a, int c, int G) {
  int v0, v1;
  share(a.V, c, G, v0, v1);
  return 4 * a.n_layers + (v1 - v0 + a.lm_rows_per_job - 1) / a.lm_rows_per_job;
}


// Shared memory (after the two 1024-aligned weight slots).
struct Smem {
  float xs[3072 + 64];        // the phase's input vector (fp32), >= max(E, Hq D, F)
  float q[kMaxG][128];        // attention: normed + rotated q rows
  float knew[128], vnew[128];
  float sc[kMaxG][kTK];       // scores / probabilities of one key tile
  float oacc[kMaxG][128];     // the unit's P.V sums (warps added)
  float mrun[kMaxG], lrun[kMaxG], corr[kMaxG];
  float red[32];
  float best_v[16];
  int best_i[16];
  uint64_t full[2], empty[2];
  int flag;
  int abort_local;            // consumers gave up: the producer stops
  int issued;                 // jobs the producer issued
};

template <typename T>
__device__ float block_sumsq(Smem& sm, int n, int ctid) {
  float p = 0.f;
  for (int i = ctid; i < n; i += kCons) p += sm.xs[i] * sm.xs[i];
  p = warp_sum(p);
  if ((ctid & 31) == 0) sm.red[ctid >> 5] = p;
  cons_sync();
  if (ctid == 0) {
    float t = 0.f;
    for (int w = 0; w < kCons / 32; ++w) t += sm.red[w];
    sm.red[31] = t;
  }
  cons_sync();
  return sm.red[31];
}

template <typename T, int NG>
__global__ void __launch_bounds__(kThr, 1) decode_step_kernel(const StepArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  uint8_t* slot[2] = {base, base + kSlot};
  Smem& sm = *reinterpret_cast<Smem*>(base + 2 * kSlot);
  Ws w;
  ws_layout(a.ws, a.E, a.Hq, a.Hkv, a.D, a.F, &w);
  const int c = blockIdx.x, G = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int njobs = n_jobs(a, c, G);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    sm.abort_local = 0;
    sm.issued = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kProdWarp) {
    // ---------------- producer: weight slices of every phase, in order ----------------
    if (lane == 0) {
      int j = 0;
      for (; j < njobs; ++j) {
        const int s = j & 1;
        if (j >= 2) {
          bool got = false;
          for (uint32_t i = 0; i < kSpinLimit && !got; ++i) {
            got = mbar_try_wait(&sm.empty[s], ((j >> 1) & 1) ^ 1);
            if (!got && *(volatile int*)&sm.abort_local) break;
          }
          if (!got) break;
        }
        const Job jb = job_of(a, j, c, G);
        mbar_arrive_expect_tx(&sm.full[s], jb.bytes0 + jb.bytes1);
        if (jb.bytes0) bulk_load(slot[s], jb.src0, jb.bytes0, &sm.full[s]);
        if (jb.bytes1) bulk_load(slot[s] + jb.bytes0, jb.src1, jb.bytes1, &sm.full[s]);
      }
      *(volatile int*)&sm.issued = j;
    }
    __syncwarp();
  } else {
    // ---------------- consumers: the phases ----------------
    const int ctid = threadIdx.x;  // 0 .. kCons-1
    bool ok = true;
    int jc = 0;  // next job to consume
    auto acquire = [&]() -> const uint8_t* {
      const int s = jc & 1;
      if (!mbar_wait(&sm.full[s], (jc >> 1) & 1, a.err, 61)) ok = false;
      return slot[s];
    };
    auto release = [&]() {
      cons_sync();
      if (ctid == 0) mbar_arrive(&sm.empty[jc & 1]);
      ++jc;
    };
    DP_TS(0);
    // this launch's barrier base: the counter is a whole multiple of the grid
    // between launches, and cannot pass the next one before this CTA arrives
    unsigned long long bar_target = 0;
    if (ctid == 0) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];"
                   : "=l"(v) : "l"(reinterpret_cast<unsigned long long*>(w.count)) : "memory");
      bar_target = v / gridDim.x * gridDim.x;
    }
    const int64_t tok = a.tokens[0];
    const int pos = a.positions[0];
    const int R = (a.Hq + 2 * a.Hkv) * a.D;
    constexpr int GQ = NG;  // query heads per kv head
    const float inv_e = 1.f / (float)a.E;
    const void* emb_row = static_cast<const T*>(a.emb) + tok * a.E;
    int r0, r1;
    for (int l = 0; l < a.n_layers && ok; ++l) {
      const tpp_decode_layer& L = a.layers[l];
      const void* xsrc = l == 0 ? emb_row : w.x;
      // ---- QKV: qkv[r] = (x . Wqkv_f[r]) * rsqrt(mean(x^2) + eps) ----
      {
        const uint8_t* sl = acquire();
        DP_TS(8 + l * 16 + 0);
        load_vec<T>(sm.xs, xsrc, a.E, ctid);
        cons_sync();
        const float rs = rsqrtf(block_sumsq<T>(sm, a.E, ctid) * inv_e + a.eps);
        share(R, c, G, r0, r1);
        for (int r = r0 + warp; r < r1 && ok; r += kCons / 32) {
          const float v = row_dot<T>(sl, r - r0, a.E, sm.xs, lane);
          if (lane == 0) static_cast<T*>(w.qkv)[r] = from_f32<T>(v * rs);
        }
        DP_TS(8 + l * 16 + 1);
        release();
      }
      if (!ok) break;
      grid_arrive(w, bar_target);
      // ---- the attention unit of this CTA (kv head h, key range sp) is known
      // before the QKV results: its first cached K/V rows and the q/k
      // prologue's constants load under the barrier ----
      constexpr int NW = kCons / 32;
      const int Lk = pos + 1;
      const int S = max(1, min((Lk + 63) / 64, G / a.Hkv));
      const int units = a.Hkv * S;
      const bool in_att = c < units;
      const int h = in_att ? c / S : 0, sp = in_att ? c % S : 0;
      const int per = (Lk + S - 1) / S;
      const int k0 = sp * per, k1 = min(Lk, k0 + per);
      const bool own_new = in_att && pos >= k0 && pos < k1;
      const int kend = own_new ? pos : k1;  // cached keys; the new one comes last
      const int ktot = in_att ? max(0, kend - k0) + (own_new ? 1 : 0) : 0;
      const T* kc = static_cast<const T*>(L.kc) + (int64_t)h * a.Smax * 128;
      const T* vc = static_cast<const T*>(L.vc) + (int64_t)h * a.Smax * 128;
      uint2 kpre[4], vpre[4];
      float nwv[4] = {1.f, 1.f, 1.f, 1.f}, cv4[4] = {0.f, 0.f, 0.f, 0.f}, sv4[4] = {0.f, 0.f, 0.f, 0.f};
      bool has_nw = false;
      if (in_att) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int key = k0 + warp + u * NW;
          kpre[u] = make_uint2(0, 0);
          vpre[u] = make_uint2(0, 0);
          if (key < kend) {
            kpre[u] = *reinterpret_cast<const uint2*>(kc + (int64_t)key * 128 + lane * 4);
            vpre[u] = *reinterpret_cast<const uint2*>(vc + (int64_t)key * 128 + lane * 4);
          }
        }
        if (warp <= GQ) {
          const T* nw = static_cast<const T*>(warp < GQ ? L.qn : L.kn);
          has_nw = nw != nullptr;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (has_nw) nwv[j] = to_f32(nw[lane * 4 + j]);
            cv4[j] = __half2float(a.cosp[(int64_t)pos * a.cs_stride + lane * 4 + j]);
            sv4[j] = __half2float(a.sinp[(int64_t)pos * a.cs_stride + lane * 4 + j]);
          }
        }
      }
      if (!grid_wait(w, bar_target, &sm.flag, a.err, 62)) { ok = false; break; }
      DP_TS(8 + l * 16 + 2);
      // ---- attention ----
      {
        if (in_att) {
          const int D = 128;
          // q rows of the G query heads, the new k row (normed + rotated) and v row
          if (warp <= GQ + 1) {
            const T* qkv = static_cast<const T*>(w.qkv);
            const int row = warp < GQ ? (h * GQ + warp) : (warp == GQ ? a.Hq + h : a.Hq + a.Hkv + h);
            float x[4];
            {
              const uint2 u = __ldcg(reinterpret_cast<const uint2*>(qkv + (int64_t)row * D + lane * 4));
              const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
              for (int j = 0; j < 4; ++j) x[j] = to_f32(e[j]);
            }
            if (warp <= GQ) {
              if (has_nw) {
                float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
                ss = warp_sum(ss);
                const float inv = rsqrtf(ss / (float)D + a.eps);
#pragma unroll
                for (int j = 0; j < 4; ++j) x[j] *= inv * nwv[j];
              }
              float pr[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) pr[j] = __shfl_xor_sync(0xffffffffu, x[j], 16);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                x[j] = rndT<T>(lane < 16 ? x[j] * cv4[j] - pr[j] * sv4[j]
                                         : x[j] * cv4[j] + pr[j] * sv4[j]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (warp < GQ) sm.q[warp][lane * 4 + j] = x[j];
              else if (warp == GQ) sm.knew[lane * 4 + j] = x[j];
              else sm.vnew[lane * 4 + j] = x[j];
            }
            if (own_new && warp >= GQ) {  // the step's cache row
              T* dst = static_cast<T*>(warp == GQ ? L.kc : L.vc) +
                       ((int64_t)h * a.Smax + pos) * D + lane * 4;
#pragma unroll
              for (int j = 0; j < 4; ++j) dst[j] = from_f32<T>(x[j]);
            }
          }
          if (ctid < GQ) { sm.mrun[ctid] = -INFINITY; sm.lrun[ctid] = 0.f; }
          for (int i = ctid; i < kMaxG * 128; i += kCons) (&sm.oacc[0][0])[i] = 0.f;
          cons_sync();
          if (l < 2) DP_TS(470 + l * 10);
          // Warp w takes keys w, w + 15, ... of each tile; lane l holds head
          // dims [4l, 4l + 4) of q, k and v, so a key costs one coalesced
          // 256-byte row read per operand and a shuffle reduction per head.
          float qv[NG][4];
#pragma unroll
          for (int g = 0; g < NG; ++g)
#pragma unroll
            for (int j = 0; j < 4; ++j) qv[g][j] = g < GQ ? sm.q[g][lane * 4 + j] : 0.f;
          float ow[NG][4];
#pragma unroll
          for (int g = 0; g < NG; ++g)
#pragma unroll
            for (int j = 0; j < 4; ++j) ow[g][j] = 0.f;
          auto row4 = [&](const T* base, int key, float* f) {
            if (key < kend) {
              const uint2 u = *reinterpret_cast<const uint2*>(base + (int64_t)key * 128 + lane * 4);
              const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
              for (int j = 0; j < 4; ++j) f[j] = to_f32(e[j]);
            } else {
              const float* src = base == kc ? sm.knew : sm.vnew;
#pragma unroll
              for (int j = 0; j < 4; ++j) f[j] = src[lane * 4 + j];
            }
          };
          for (int t0 = 0; t0 < ktot; t0 += kTK) {
            const int nt = min(kTK, ktot - t0);
            // scores, 4 keys of a warp in flight at a time
            for (int i0 = warp; i0 < nt; i0 += 4 * NW) {
              float kf[4][4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * NW;
                if (i >= nt) continue;
                if (t0 == 0 && i0 == warp && k0 + i < kend) {
                  const T* e = reinterpret_cast<const T*>(&kpre[u]);
#pragma unroll
                  for (int j = 0; j < 4; ++j) kf[u][j] = to_f32(e[j]);
                } else {
                  row4(kc, k0 + t0 + i, kf[u]);
                }
              }
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * NW;
                if (i >= nt) break;
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                  if (g >= GQ) break;
                  float d = qv[g][0] * kf[u][0] + qv[g][1] * kf[u][1] + qv[g][2] * kf[u][2] +
                            qv[g][3] * kf[u][3];
                  d = warp_sum(d);
                  if (lane == 0) sm.sc[g][i] = d * a.scale_log2;
                }
              }
            }
            cons_sync();
            if (l < 2 && t0 == 0) DP_TS(471 + l * 10);
            // tile max, probabilities and running sums per head (warp g)
            if (warp < GQ) {
              float m = -INFINITY;
              for (int i = lane; i < nt; i += 32) m = fmaxf(m, sm.sc[warp][i]);
              m = warp_max(m);
              const float mo = sm.mrun[warp];
              const float mn = fmaxf(mo, m);
              float l = 0.f;
              for (int i = lane; i < nt; i += 32) {
                const float pv = exp2f(sm.sc[warp][i] - mn);
                sm.sc[warp][i] = pv;
                l += pv;
              }
              l = warp_sum(l);
              if (lane == 0) {
                const float cr = mo == -INFINITY ? 0.f : exp2f(mo - mn);
                sm.corr[warp] = cr;
                sm.lrun[warp] = sm.lrun[warp] * cr + l;
                sm.mrun[warp] = mn;
              }
            }
            cons_sync();
            if (l < 2 && t0 == 0) DP_TS(472 + l * 10);
            // o = o * corr + P . V over this warp's keys
#pragma unroll
            for (int g = 0; g < NG; ++g)
#pragma unroll
              for (int j = 0; j < 4; ++j) ow[g][j] *= g < GQ ? sm.corr[g] : 0.f;
            for (int i0 = warp; i0 < nt; i0 += 4 * NW) {
              float vf[4][4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * NW;
                if (i >= nt) continue;
                if (t0 == 0 && i0 == warp && k0 + i < kend) {
                  const T* e = reinterpret_cast<const T*>(&vpre[u]);
#pragma unroll
                  for (int j = 0; j < 4; ++j) vf[u][j] = to_f32(e[j]);
                } else {
                  row4(vc, k0 + t0 + i, vf[u]);
                }
              }
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * NW;
                if (i >= nt) break;
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                  if (g >= GQ) break;
                  const float pg = sm.sc[g][i];
#pragma unroll
                  for (int j = 0; j < 4; ++j) ow[g][j] = fmaf(pg, vf[u][j], ow[g][j]);
                }
              }
            }
            cons_sync();
            if (l < 2 && t0 == 0) DP_TS(473 + l * 10);
          }
          // sum the warps' o accumulators
#pragma unroll
          for (int g = 0; g < NG; ++g) {
            if (g >= GQ) break;
#pragma unroll
            for (int j = 0; j < 4; ++j) atomicAdd(&sm.oacc[g][lane * 4 + j], ow[g][j]);
          }
          cons_sync();
          // partial (o, m, l) of each query head of this unit
          const int npair = GQ * 128;
          for (int pi = ctid; pi < npair; pi += kCons) {
            const int g = pi / 128, d = pi % 128;
            float* dst = w.part + ((int64_t)(h * GQ + g) * S + sp) * (128 + 2);
            dst[d] = sm.oacc[g][d];
            if (d == 0) { dst[128] = sm.mrun[g]; dst[129] = sm.lrun[g]; }
          }
          __threadfence();
          cons_sync();
          if (l < 2) DP_TS(474 + l * 10);
          // the last unit of head h to finish merges its S partials: (m, l)
          // staged once, per-head weights, then one (query head, dim) pair
          // per thread with its S loads in flight
          if (ctid == 0) {
            const uint32_t prev = atomicAdd(&w.head_cnt[h], 1u);
            const bool last = prev == (uint32_t)(S - 1);
            if (last) atomicExch(&w.head_cnt[h], 0u);
            sm.flag = last ? 1 : 0;
          }
          cons_sync();
          if (sm.flag) {
            __threadfence();
            float* st = &sm.sc[0][0];  // [GQ][S] m -> weights, [GQ][S] l, [GQ] 1 / den
            const int GS = GQ * S;
            for (int i = ctid; i < GS; i += kCons) {
              const float* src = w.part + ((int64_t)h * GQ * S + i) * 130;
              st[i] = __ldcg(src + 128);
              st[GS + i] = __ldcg(src + 129);
            }
            cons_sync();
            if (ctid < GQ) {
              float M = -INFINITY;
              for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, st[ctid * S + s2]);
              float den = 0.f;
              for (int s2 = 0; s2 < S; ++s2) {
                const float m2 = st[ctid * S + s2];
                const float e = m2 == -INFINITY ? 0.f : exp2f(m2 - M);
                st[ctid * S + s2] = e;
                den = fmaf(e, st[GS + ctid * S + s2], den);
              }
              st[2 * GS + ctid] = den > 0.f ? 1.f / den : 0.f;
            }
            cons_sync();
            for (int pi = ctid; pi < npair; pi += kCons) {
              const int g = pi / 128, d = pi % 128;
              const float* src = w.part + (int64_t)(h * GQ + g) * S * 130 + d;
              float num = 0.f;
#pragma unroll 8
              for (int s2 = 0; s2 < S; ++s2) num = fmaf(st[g * S + s2], __ldcg(src + s2 * 130), num);
              static_cast<T*>(w.o)[(int64_t)(h * GQ + g) * 128 + d] =
                  from_f32<T>(num * st[2 * GS + g]);
            }
          }
          if (l < 2) DP_TS(475 + l * 10);
        }
      }
      DP_TS(8 + l * 16 + 3);
      if (!grid_sync(w, bar_target, &sm.flag, a.err, 63)) { ok = false; break; }
      DP_TS(8 + l * 16 + 4);
      // ---- o-proj + residual: x[r] = x[r] + o . Wo[r] ----
      {
        const uint8_t* sl = acquire();
        DP_TS(8 + l * 16 + 5);
        const int K = a.Hq * a.D;
        load_vec<T>(sm.xs, w.o, K, ctid);
        cons_sync();
        share(a.E, c, G, r0, r1);
        for (int r = r0 + warp; r < r1; r += kCons / 32) {
          const float v = row_dot<T>(sl, r - r0, K, sm.xs, lane);
          if (lane == 0) static_cast<T*>(w.x)[r] = from_f32<T>(ldT<T>(xsrc, r) + v);
        }
        release();
      }
      DP_TS(8 + l * 16 + 6);
      if (!ok || !grid_sync(w, bar_target, &sm.flag, a.err, 64)) { ok = false; break; }
      DP_TS(8 + l * 16 + 7);
      // ---- gate/up + SwiGLU: ff[f] = silu(g * rs) * (u * rs) ----
      {
        const uint8_t* sl = acquire();
        load_vec<T>(sm.xs, w.x, a.E, ctid);
        cons_sync();
        const float rs = rsqrtf(block_sumsq<T>(sm, a.E, ctid) * inv_e + a.eps);
        share(a.F, c, G, r0, r1);
        const int nf = r1 - r0;
        for (int f = warp; f < nf; f += kCons / 32) {
          const float g = row_dot<T>(sl, f, a.E, sm.xs, lane) * rs;
          const float u = row_dot<T>(sl, nf + f, a.E, sm.xs, lane) * rs;
          if (lane == 0) static_cast<T*>(w.ff)[r0 + f] = from_f32<T>(act_silu(g) * u);
        }
        release();
      }
      DP_TS(8 + l * 16 + 9);
      if (!ok || !grid_sync(w, bar_target, &sm.flag, a.err, 65)) { ok = false; break; }
      DP_TS(8 + l * 16 + 10);
      // ---- down + residual: x[r] = x[r] + ff . Wd[r] ----
      {
        const uint8_t* sl = acquire();
        load_vec<T>(sm.xs, w.ff, a.F, ctid);
        cons_sync();
        share(a.E, c, G, r0, r1);
        for (int r = r0 + warp; r < r1; r += kCons / 32) {
          const float v = row_dot<T>(sl, r - r0, a.F, sm.xs, lane);
          if (lane == 0) static_cast<T*>(w.x)[r] = from_f32<T>(ldT<T>(w.x, r) + v);
        }
        release();
      }
      DP_TS(8 + l * 16 + 12);
      if (!ok || !grid_sync(w, bar_target, &sm.flag, a.err, 66)) { ok = false; break; }
      DP_TS(8 + l * 16 + 13);
    }
    // ---- LM head: logits = (x . Wh_f) * rs, per-CTA argmax ----
    if (ok) {
      load_vec<T>(sm.xs, w.x, a.E, ctid);
      cons_sync();
      const float rs = rsqrtf(block_sumsq<T>(sm, a.E, ctid) * inv_e + a.eps);
      int v0, v1;
      share(a.V, c, G, v0, v1);
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int q = 0; jc < njobs && ok; ++q) {
        const uint8_t* sl = acquire();
        const int rr0 = v0 + q * a.lm_rows_per_job, rr1 = min(v1, rr0 + a.lm_rows_per_job);
        for (int r = rr0 + warp; r < rr1; r += kCons / 32) {
          const float v = rndT<T>(row_dot<T>(sl, r - rr0, a.E, sm.xs, lane) * rs);
          if (lane == 0) {
            static_cast<T*>(a.logits)[r] = from_f32<T>(v);
            if (v > bv || (v == bv && r < bi)) { bv = v; bi = r; }
          }
        }
        release();
      }
      if (lane == 0) { sm.best_v[warp] = bv; sm.best_i[warp] = bi; }
      cons_sync();
      if (ctid == 0) {
        for (int i = 1; i < kCons / 32; ++i)
          if (sm.best_v[i] > bv || (sm.best_v[i] == bv && sm.best_i[i] < bi)) {
            bv = sm.best_v[i];
            bi = sm.best_i[i];
          }
        w.amax_v[c] = bv;
        w.amax_i[c] = bi;
      }
      DP_TS(500);
      ok = grid_sync(w, bar_target, &sm.flag, a.err, 67);
      DP_TS(501);
      if (ok && c == 0 && warp == 0) {
        float v = -INFINITY;
        int idx = 0x7fffffff;
        for (int i = lane; i < G; i += 32) {
          const float vv = __ldcg(w.amax_v + i);
          const int ii = __ldcg(w.amax_i + i);
          if (vv > v || (vv == v && ii < idx)) { v = vv; idx = ii; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
          const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
          if (v2 > v || (v2 == v && i2 < idx)) { v = v2; idx = i2; }
        }
        if (lane == 0) {
          const int p1 = pos + 1;
          a.tokens[0] = idx;
          if (a.out_ids != nullptr && p1 < a.out_cap) a.out_ids[p1] = idx;
          a.positions[0] = p1;
          if (a.seqlens != nullptr) a.seqlens[0] = p1 + 1;
        }
      }
    }
    if (!ok) *(volatile int*)&sm.abort_local = 1;
    // jobs issued but not consumed (an aborted step) land before the CTA exits
    __syncwarp();
    cons_sync();
    if (ctid == 0) sm.red[0] = __int_as_float(jc);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int consumed = __float_as_int(sm.red[0]);
    for (int j = consumed; j < sm.issued; ++j) mbar_wait(&sm.full[j & 1], (j >> 1) & 1, a.err, 68);
  }
}
}  // namespace
}  // namespace tpp

using namespace tpp;

#ifdef TPP_DEBUG_STAMPS
extern "C" void tpp_debug_dp_stamps(unsigned long long* host) {
  cudaMemcpyFromSymbol(host, g_dp_stamps, sizeof(unsigned long long) * 256 * 512);
}
#endif

namespace {
// Whether a model shape fits the persistent plan on this device: head dim
// 128, <= 4 query heads per kv head, activation vectors <= 3072 wide, and
// every phase's per-CTA weight slice within one 96 KB slot.
bool persistent_fits(int64_t E, int64_t Hq, int64_t Hkv, int64_t D, int64_t F) {
  if (E <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || F <= 0) return false;
  const int sms = num_sms();
  const int G = sms < kMaxCTAs ? sms : kMaxCTAs;
  const int64_t GQ = Hq / Hkv;
  const int64_t R = (Hq + 2 * Hkv) * D;
  auto per = [&](int64_t rows) { return (rows + G - 1) / G; };
  return D == 128 && (GQ == 1 || GQ == 2 || GQ == 4) && GQ + 2 <= kCons / 32 && GQ * D <= 2 * kCons && Hkv <= 64 &&
         E % 8 == 0 && F % 8 == 0 && E <= 3072 && Hq * D <= 3072 && F <= 3072 &&
         per(R) * E * 2 <= kSlot && per(E) * Hq * D * 2 <= kSlot && 2 * per(F) * E * 2 <= kSlot &&
         per(E) * F * 2 <= kSlot;
}
}  // namespace

extern "C" int64_t tpp_decode_step_persistent_workspace(int64_t E, int64_t Hq, int64_t Hkv,
                                                        int64_t D, int64_t F, int64_t) {
  if (!persistent_fits(E, Hq, Hkv, D, F)) return 0;
  return (int64_t)ws_layout(nullptr, E, Hq, Hkv, D, F, nullptr) + 256;
}

extern "C" int tpp_decode_step_persistent(
    const tpp_decode_layer* layers, int64_t n_layers, const void* emb, const void* lm_head,
    const void* cos, const void* sin, int64_t cs_stride, int64_t* tokens, int32_t* positions,
    int32_t* seqlens, int64_t* out_ids, int64_t out_cap, void* logits, void* workspace,
    int64_t workspace_bytes, int64_t E, int64_t Hq, int64_t Hkv, int64_t D, int64_t F,
    int64_t V, int64_t Smax, float eps, int dtype, void* stream) {
  TPP_REQUIRE(layers && emb && lm_head && cos && sin && tokens && positions && logits &&
                  workspace,
              TPP_ERR_SHAPE, "null operand");
  TPP_REQUIRE(n_layers > 0 && V > 0 && Smax > 0 && Smax <= (1 << 30), TPP_ERR_SHAPE, "bad sizes");
  if (!persistent_fits(E, Hq, Hkv, D, F)) {
    set_error("tpp_decode_step_persistent: shape outside the persistent plan");
    return TPP_ERR_UNSUPPORTED;
  }
  const int sms = num_sms();
  const int G = sms < kMaxCTAs ? sms : kMaxCTAs;
  TPP_REQUIRE(workspace_bytes >= tpp_decode_step_persistent_workspace(E, Hq, Hkv, D, F, Smax),
              TPP_ERR_WORKSPACE, "workspace too small");
  TPP_REQUIRE(aligned16(emb) && aligned16(lm_head), TPP_ERR_ALIGN,
              "embedding / LM head must be 16-byte aligned");
  StepArgs a;
  a.layers = layers; a.n_layers = (int)n_layers; a.emb = emb; a.lm_head = lm_head;
  a.cosp = static_cast<const __half*>(cos); a.sinp = static_cast<const __half*>(sin);
  a.cs_stride = cs_stride; a.tokens = tokens; a.positions = positions; a.seqlens = seqlens;
  a.out_ids = out_ids; a.out_cap = out_cap; a.logits = logits;
  a.ws = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~(uintptr_t)255);
  a.E = (int)E; a.Hq = (int)Hq; a.Hkv = (int)Hkv; a.D = (int)D; a.F = (int)F; a.V = (int)V;
  a.Smax = (int)Smax; a.eps = eps;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
  a.lm_rows_per_job = (int)(kSlot / (E * 2));
  a.err = device_error_flag();
  const size_t smem = 1024 + 2 * (size_t)kSlot + sizeof(Smem);
  cudaStream_t st = as_stream(stream);
  return TPP_DISPATCH_HALF(dtype, T, [&] {
    const int64_t gq = Hq / Hkv;
    auto kern = gq == 1 ? decode_step_kernel<T, 1>
                        : (gq == 2 ? decode_step_kernel<T, 2> : decode_step_kernel<T, 4>);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
      set_error("decode_step_kernel: cannot reserve shared memory");
      return (int)TPP_ERR_LAUNCH;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThr, smem) != cudaSuccess ||
        per_sm < 1) {
      set_error("decode_step_kernel: one CTA per SM does not fit");
      return (int)TPP_ERR_LAUNCH;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G);
    cfg.blockDim = dim3(kThr);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) {
      set_error(std::string("decode_step_kernel: ") + cudaGetErrorString(e));
      return (int)TPP_ERR_LAUNCH;
    }
    return check_launch("decode_step_kernel");
  });
}
