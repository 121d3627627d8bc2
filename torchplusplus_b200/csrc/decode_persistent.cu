// The whole decode step of one sequence as ONE persistent, cooperative
// kernel (tpp_decode_step_persistent).
//
// At batch 1 the step is a chain of ~140 small dependent phases (five per
// layer); as separate launches every phase pays a kernel boundary and
// re-stages its operands, so the step runs at ~22% of HBM although its work
// is one pass over the weights.  Here one CTA per SM stays resident for the
// whole step:
//  * consumer warps 0..14 run the phases.  A phase's output (QKV rows,
//    attention output, residual stream, SwiGLU output) goes to the
//    workspace as 64-bit words {value, epoch of the writing phase}; the
//    next phase polls the words it reads until all carry that epoch, so the
//    data load is the synchronisation (no separate grid barrier).  Every
//    phase reads the whole output of the previous one, so no CTA can run
//    more than one phase ahead of another and a buffer is never rewritten
//    while it is still read.  The per-CTA argmax picks are tagged words
//    too; CTA 0 polls them and writes the token, the others count
//    themselves in (an atomic arrival count that numbers the steps, and so
//    the epochs) and leave;
//  * producer warp 15 streams this CTA's weight slice of every phase, in
//    phase order, through two 96 KB shared-memory slots with bulk copies
//    (cp.async.bulk, mbarrier completion).  Weights do not depend on the
//    barriers, so the next phases' slices are in flight (or resident) while
//    the current phase computes and waits;
//  * per layer: QKV (RMSNorm folded into the weights, each CTA a contiguous
//    row range) | attention (kv head x key-range units; q/k RMSNorm + RoPE
//    and the K/V append of the new token in the unit that owns its
//    position; unit 0 of a head merges the head's
//    partials) | o-proj + residual | gate/up + SwiGLU | down + residual;
//    then the LM head (row chunks, per-CTA argmax) and the token bookkeeping.
// GEMVs run on CUDA cores (one token: one weight byte is used once), a warp
// per output row, fp32 accumulation; every stored activation is rounded to
// the step's dtype as the launch-per-phase path rounds it.
#include <stdio.h>
#include <stdlib.h>
#include "tc_common.cuh"
#include "mma_common.cuh"

namespace tpp {
namespace {

constexpr int kThr = 512;                // 15 consumer warps + 1 producer warp
constexpr int kCons = 480;
constexpr int kProdWarp = 15;
constexpr uint32_t kSlot = 96 * 1024;    // one weight slot
constexpr int kMaxG = 4;                 // query heads per kv head (at most)
constexpr int kTK = 256;                 // keys per attention tile
constexpr int kMaxCTAs = 256;
constexpr int kPaceMax = 8;
constexpr int kMaxRes = 64;              // residual rows per CTA (at most)
constexpr int kRG = 4;                   // rows of one GEMV work item
constexpr int kKC = 256;                 // K elements of one GEMV work item
constexpr int kPad = TPP_PERSISTENT_ROW_PAD;  // weight row pitch = K + kPad elements
constexpr int kMaxPart = 512;            // GEMV partial sums per phase (chunks x rows)
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
  // Activations exchanged between CTAs are tagged words: the value (fp32 of
  // the dtype-rounded number) in the low half, the epoch of the phase that
  // wrote it in the high half; one 64-bit store / load is single-copy
  // atomic, so a reader that sees the current epoch sees the value too.
  uint64_t* x;          // [E] residual stream
  uint64_t* qkv;        // [(Hq+2Hkv) D]
  uint64_t* part;       // [Hq][S][D + 2] attention partials (o, m, l), tagged
  uint64_t* o;          // [Hq D] merged attention output
  uint64_t* ff;         // [F] SwiGLU output
  uint64_t* amax_v;     // [CTAs] per-CTA best logit (tagged)
  uint64_t* amax_i;     // [CTAs] its index (tagged, bits of the int)
};

__host__ __device__ inline size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

__host__ __device__ inline size_t ws_layout(char* base, int64_t E, int64_t Hq, int64_t Hkv,
                                            int64_t D, int64_t F, Ws* w) {
  size_t off = 0;
  auto take = [&](size_t bytes) { char* p = base + off; off += al256(bytes); return p; };
  char* sync = take(256 + 4 * 64);
  char* x = take((size_t)E * 8);
  char* qkv = take((size_t)(Hq + 2 * Hkv) * D * 8);
  char* part = take((size_t)Hq * kMaxCTAs * (D + 2) * 8);
  char* o = take((size_t)Hq * D * 8);
  char* ff = take((size_t)F * 8);
  char* av = take((size_t)kMaxCTAs * 8);
  char* ai = take((size_t)kMaxCTAs * 8);
  if (w) {
    w->count = reinterpret_cast<uint32_t*>(sync);
    w->gen = reinterpret_cast<uint32_t*>(sync + 64);
    w->abortf = reinterpret_cast<uint32_t*>(sync + 128);
    w->x = reinterpret_cast<uint64_t*>(x); w->qkv = reinterpret_cast<uint64_t*>(qkv);
    w->o = reinterpret_cast<uint64_t*>(o);
    w->part = reinterpret_cast<uint64_t*>(part); w->ff = reinterpret_cast<uint64_t*>(ff);
    w->amax_v = reinterpret_cast<uint64_t*>(av); w->amax_i = reinterpret_cast<uint64_t*>(ai);
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
  int pace_chunk;       // layer weight slices stream in chunks of this many bytes ...
  int pace_depth;       // ... with at most this many in flight per CTA (0: one burst)
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
    // release at gpu scope: covers this CTA's writes ordered before it by
    // the CTA barrier above
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(w.count) : "memory");
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

// ---- tagged activation words ----
__device__ __forceinline__ void st_tag(uint64_t* p, float v, uint32_t ep) {
  const uint64_t wv = ((uint64_t)ep << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(wv) : "memory");
}
__device__ __forceinline__ uint64_t ld_tag(const uint64_t* p) {
  uint64_t wv;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(wv) : "l"(p) : "memory");
  return wv;
}
// Polls n tagged words (n <= kPollMax, all loads of a round in flight at
// once) until every one carries epoch ep; bounded, gives up when another
// CTA aborted.  Returns false on give-up (error code set, abort raised).
constexpr int kPollMax = 8;
template <int N>
__device__ __forceinline__ bool poll_tags(const uint64_t* const (&src)[N], int n, uint32_t ep,
                                          uint64_t (&v)[N], const Ws& w, int* err, int code) {
#pragma unroll
  for (int u = 0; u < N; ++u) v[u] = u < n ? ld_tag(src[u]) : ((uint64_t)ep << 32);
  for (uint32_t it = 0;; ++it) {
    bool all = true;
#pragma unroll
    for (int u = 0; u < N; ++u) all = all && (uint32_t)(v[u] >> 32) == ep;
    if (all) return true;
    if (it >= kSpinLimit) {
      if (err) atomicExch(err, code);
      atomicExch(w.abortf, 1u);
      return false;
    }
    if ((it & 255) == 255 && ld_acquire(w.abortf) != 0) return false;
#pragma unroll
    for (int u = 0; u < N; ++u)
      if (u < n && (uint32_t)(v[u] >> 32) != ep) v[u] = ld_tag(src[u]);
  }
}

template <typename T>
__device__ __forceinline__ float ldT(const void* p, int64_t i) {
  return to_f32(__ldcg(static_cast<const T*>(p) + i));
}
template <typename T>
__device__ __forceinline__ float rndT(float v) { return to_f32(from_f32<T>(v)); }

// xh[0..n) = src[0..n) (the step's dtype, copied as is), 16 bytes per
// load.  With red != nullptr each warp also leaves its share of sum(x^2)
// (fp32) in red[warp] (read back with sumsq_of after the next consumer
// barrier).
template <typename T>
__device__ __forceinline__ void load_vec(uint16_t* xh, const void* src, int n, int ctid,
                                         float* red = nullptr) {
  const uint4* p = static_cast<const uint4*>(src);
  float ss = 0.f;
  for (int i = ctid; i < n / 8; i += kCons) {
    const uint4 u = __ldcg(p + i);
    if (red != nullptr) {
      float f[8];
      unpack8<T>(u, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
    reinterpret_cast<uint4*>(xh)[i] = u;
  }
  if (red != nullptr) {
    ss = warp_sum(ss);
    if ((ctid & 31) == 0) red[ctid >> 5] = ss;
  }
}
// xh[0..n) = the tagged vector src[0..n) once every word carries epoch ep
// (the phase that writes it has finished in every CTA), as load_vec.  On
// give-up sets *fail.
template <typename T>
__device__ __forceinline__ void load_tagged(uint16_t* xh, const uint64_t* src, int n,
                                            uint32_t ep, int ctid, float* red, const Ws& w,
                                            int* err, int code, int* fail) {
  const uint64_t* ptr[kPollMax];
  int m = 0;
#pragma unroll
  for (int u = 0; u < kPollMax; ++u) {
    const int i = ctid + u * kCons;
    ptr[u] = src + (i < n ? i : 0);
    m += i < n ? 1 : 0;
  }
  uint64_t v[kPollMax];
  if (!poll_tags<kPollMax>(ptr, m, ep, v, w, err, code)) *(volatile int*)fail = 1;
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < kPollMax; ++u) {
    const int i = ctid + u * kCons;
    if (i < n) {
      const float f = __uint_as_float((uint32_t)v[u]);
      ss = fmaf(f, f, ss);
      const T t = from_f32<T>(f);
      xh[i] = *reinterpret_cast<const uint16_t*>(&t);
    }
  }
  if (red != nullptr) {
    ss = warp_sum(ss);
    if ((ctid & 31) == 0) red[ctid >> 5] = ss;
  }
}
__device__ __forceinline__ float sumsq_of(const float* red) {
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kCons / 32; ++w) t += red[w];
  return t;
}

// Partial GEMV of this CTA's weight slice on the tensor cores: rows [0, R)
// of a slice in shared memory with row pitch K + kPad elements, times x (the
// step's dtype, shared).  Work item (c, tile): 256-wide K chunk c x 16 rows;
// a consumer warp takes items w, w + 15, ...  Per 32-wide k block a lane
// loads 16 contiguous bytes (k = 8t .. 8t+7, t = lane % 4) of rows g and
// g + 8 (g = lane / 4) and of x, and feeds them to two m16n8k16 MMAs with
// the weights as A (16 rows x 16 k) and x as B (the same x in all 8
// columns): the k order inside a block is permuted the same way for both
// operands (physical 8t + {0,1,2,3} = logical {2t, 2t+1, 2t+8, 2t+9} of the
// first MMA, 8t + {4..7} of the second), so each MMA sees every k of its
// 16 once.  The 64-byte row padding puts rows g and g+1 16 banks apart: the
// 16-byte loads are conflict-free.  Lane 4g holds the fp32 sums of rows g
// (d[0]) and g + 8 (d[2]) and writes part[c * R + row].  Callers sum the
// K/256 chunk partials of a row in chunk order after a consumer barrier.
template <typename T>
__device__ __forceinline__ void slice_dot(uint32_t slot_s, int R, int K, uint32_t xh_s,
                                          float* part, int warp, int lane) {
  const int NC = K / kKC;
  const int NT = (R + 15) / 16;
  const uint32_t pitch = (uint32_t)(K + kPad) * 2u;
  const int g = lane >> 2, t = lane & 3;
  // item it = tile * NC + c, stepped by 15 without a division per item
  int c = warp % NC, tile = warp / NC;
  for (int it = warp; it < NC * NT; it += kCons / 32) {
    if (it != warp) {
      c += kCons / 32;
      while (c >= NC) { c -= NC; ++tile; }
    }
    const int ra = tile * 16 + g, rb = ra + 8;
    // rows past R read a valid row; their sums are dropped
    const uint32_t koff = (uint32_t)(c * kKC + 8 * t) * 2u;
    const uint32_t wa = slot_s + (uint32_t)min(ra, R - 1) * pitch + koff;
    const uint32_t wb = slot_s + (uint32_t)min(rb, R - 1) * pitch + koff;
    const uint32_t xa = xh_s + koff;
    // two accumulators: the two MMAs of a k block do not wait on each other
    float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int kb = 0; kb < kKC / 32; ++kb) {
      uint32_t A0[4], A1[4], X[4];
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(A0[0]), "=r"(A0[1]), "=r"(A0[2]), "=r"(A0[3]) : "r"(wa + kb * 64));
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(A1[0]), "=r"(A1[1]), "=r"(A1[2]), "=r"(A1[3]) : "r"(wb + kb * 64));
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(X[0]), "=r"(X[1]), "=r"(X[2]), "=r"(X[3]) : "r"(xa + kb * 64));
      const uint32_t a0[4] = {A0[0], A1[0], A0[1], A1[1]};
      mma<T>(d, a0, X[0], X[1]);
      const uint32_t a1[4] = {A0[2], A1[2], A0[3], A1[3]};
      mma<T>(e, a1, X[2], X[3]);
    }
    d[0] += e[0];
    d[2] += e[2];
    if (t == 0) {
      if (ra < R) part[c * R + ra] = d[0];
      if (rb < R) part[c * R + rb] = d[2];
    }
  }
}

// Row r's full dot product: its chunk partials summed in chunk order.
__device__ __forceinline__ float row_sum(const float* part, int R, int K, int r) {
  float t = 0.f;
  for (int c = 0; c < K / kKC; ++c) t += part[c * R + r];
  return t;
}

// Contiguous share [r0, r1) of `rows` for CTA c of G (32-bit: rows * G
// stays below 2^32 for every plan this kernel accepts).
__device__ __forceinline__ void share(int rows, int c, int G, int& r0, int& r1) {
  r0 = (int)((uint32_t)rows * (uint32_t)c / (uint32_t)G);
  r1 = (int)((uint32_t)rows * (uint32_t)(c + 1) / (uint32_t)G);
}
// This CTA's row ranges of every phase, computed once per launch (integer
// division is a multi-instruction routine): QKV rows, E rows (o-proj, down,
// residual), F features (gate/up), V rows (LM head).
struct Shares {
  int q0, q1, e0, e1, f0, f1, v0, v1;
};
__device__ __forceinline__ Shares shares_of(int R, int E, int F, int V, int c, int G) {
  Shares h;
  share(R, c, G, h.q0, h.q1);
  share(E, c, G, h.e0, h.e1);
  share(F, c, G, h.f0, h.f1);
  share(V, c, G, h.v0, h.v1);
  return h;
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

__device__ __forceinline__ Job job_of(const StepArgs& a, int j, const Shares& h) {
  Job jb = {nullptr, 0, nullptr, 0};
  const int esz = 2;
  if (j < 4 * a.n_layers) {
    const tpp_decode_layer& L = a.layers[j / 4];
    int r0, r1;
    switch (j % 4) {
      case 0: {
        r0 = h.q0; r1 = h.q1;
        jb.src0 = static_cast<const uint8_t*>(L.wqkv) + (size_t)r0 * (a.E + kPad) * esz;
        jb.bytes0 = (uint32_t)((r1 - r0) * (a.E + kPad) * esz);
        break;
      }
      case 1: {
        r0 = h.e0; r1 = h.e1;
        jb.src0 = static_cast<const uint8_t*>(L.wo) + (size_t)r0 * (a.Hq * a.D + kPad) * esz;
        jb.bytes0 = (uint32_t)((r1 - r0) * (a.Hq * a.D + kPad) * esz);
        break;
      }
      case 2: {
        r0 = h.f0; r1 = h.f1;
        jb.src0 = static_cast<const uint8_t*>(L.wgu) + (size_t)r0 * (a.E + kPad) * esz;
        jb.bytes0 = (uint32_t)((r1 - r0) * (a.E + kPad) * esz);
        jb.src1 = static_cast<const uint8_t*>(L.wgu) + (size_t)(a.F + r0) * (a.E + kPad) * esz;
        jb.bytes1 = jb.bytes0;
        break;
      }
      default: {
        r0 = h.e0; r1 = h.e1;
        jb.src0 = static_cast<const uint8_t*>(L.wdown) + (size_t)r0 * (a.F + kPad) * esz;
        jb.bytes0 = (uint32_t)((r1 - r0) * (a.F + kPad) * esz);
        break;
      }
    }
  } else {
    const int v0 = h.v0, v1 = h.v1;
    const int q = j - 4 * a.n_layers;
    const int r0 = v0 + q * a.lm_rows_per_job;
    const int r1 = min(v1, r0 + a.lm_rows_per_job);
    jb.src0 = static_cast<const uint8_t*>(a.lm_head) + (size_t)r0 * (a.E + kPad) * esz;
    jb.bytes0 = r1 > r0 ? (uint32_t)((r1 - r0) * (a.E + kPad) * esz) : 0u;
  }
  return jb;
}

__device__ __forceinline__ int n_jobs(const StepArgs& a, const Shares& h) {
  return 4 * a.n_layers + (h.v1 - h.v0 + a.lm_rows_per_job - 1) / a.lm_rows_per_job;
}


// The attention unit of CTA c: kv head h, key range [k0, k1) of the Lk = pos
// + 1 keys (S units per head, >= ~64 keys each).  The cached keys are
// [k0, kend); the unit that owns position pos also takes the new key.
struct AttUnit {
  bool in_att, own_new;
  int h, sp, S, k0, kend, ktot;
  int nst;  // cached keys staged in shared memory (after the o-proj weights)
};
__device__ __forceinline__ AttUnit att_unit(const StepArgs& a, int pos, int c, int G,
                                            uint32_t o_bytes) {
  AttUnit u;
  const int Lk = pos + 1;
  u.S = max(1, min((Lk + 63) / 64, G / a.Hkv));
  u.in_att = c < a.Hkv * u.S;
  u.h = u.in_att ? c / u.S : 0;
  u.sp = u.in_att ? c % u.S : 0;
  const int per = (Lk + u.S - 1) / u.S;
  u.k0 = u.sp * per;
  const int k1 = min(Lk, u.k0 + per);
  u.own_new = u.in_att && pos >= u.k0 && pos < k1;
  u.kend = u.own_new ? pos : k1;
  u.ktot = u.in_att ? max(0, u.kend - u.k0) + (u.own_new ? 1 : 0) : 0;
  // K rows, V rows (256 B each) and the two norm weight rows after the
  // o-proj slice in its slot
  const int room = ((int)kSlot - (int)o_bytes - 512) / 512;
  u.nst = u.in_att ? max(0, min(u.kend - u.k0, room)) : 0;
  return u;
}

// Shared memory (after the two 1024-aligned weight slots).
struct Smem {
  union {
    struct {
      uint16_t xh[3072 + 64]; // the phase's input vector (step dtype), >= max(E, Hq D, F)
      float q[kMaxG][128];    // attention: normed + rotated q rows
      float knew[128], vnew[128];
      float sc[kMaxG][kTK];   // scores / probabilities of one key tile
    };
    float wpart[kCons / 32][2][128];  // attention end (<= 2 query heads): each warp's P.V sums
  };
  float oacc[kMaxG][128];     // the unit's P.V sums (warps added)
  float mrun[kMaxG], lrun[kMaxG], corr[kMaxG];
  float red[32];
  float xres[kMaxRes];        // this CTA's rows of the residual stream (o-proj / down rows)
  float gpart[kMaxPart];      // GEMV chunk partials of the current phase
  float best_v[16];
  int best_i[16];
  uint64_t full[2], empty[2];
  uint64_t pace[kPaceMax];
  uint64_t kvbar;             // the layer's staged K/V rows + norm weights landed
  float cs[2][128];           // cos, sin rows of this step's position
  int kv_issued;              // layers whose K/V staging the producer issued
  int kvfail;                 // a staged-K/V wait gave up
  int flag;
  int poll_fail;              // a tagged-vector poll gave up
  uint32_t ep_base;           // this step's epoch base
  int abort_local;            // consumers gave up: the producer stops
  int issued;                 // jobs the producer issued
};


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
  const Shares sh = shares_of((a.Hq + 2 * a.Hkv) * a.D, a.E, a.F, a.V, c, G);
  const int njobs = n_jobs(a, sh);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < kPaceMax; ++i) mbar_init(&sm.pace[i], 1);
    mbar_init(&sm.kvbar, 1);
    sm.kv_issued = 0;
    sm.kvfail = 0;
    sm.abort_local = 0;
    sm.issued = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kProdWarp) {
    // ---------------- producer: weight slices of every phase, in order ----------------
    // A layer's slices are needed one phase at a time, but a slot frees up
    // while latency-bound phases (attention, barriers) run: issued as one
    // burst per CTA, a slice fills the memory queues for microseconds and
    // every dependent load of those phases waits behind it.  So layer slices
    // stream in pace_chunk pieces with at most pace_depth in flight per CTA
    // (their own mbarriers), and the slot's full barrier is arrived on once
    // the slice has landed.  LM-head chunks have nothing behind them and go
    // out as single bursts.
    if (lane == 0) {
      const int depth = a.pace_depth;
      uint32_t q = 0;  // paced chunks issued
      bool alive = true;
      auto pace_wait = [&](uint32_t k, bool stop_on_abort) {  // chunk k has landed
        for (uint32_t i = 0; i < kSpinLimit; ++i) {
          if (mbar_try_wait(&sm.pace[k % depth], (k / depth) & 1)) return true;
          if (stop_on_abort && *(volatile int*)&sm.abort_local) break;
        }
        return false;
      };
      // with an o-proj slice (its slot sits idle through QKV and attention):
      // this CTA's cached K/V rows of the layer's attention unit and the q/k
      // norm weights, after the weights (they depend on nothing in the
      // step), on their own barrier
      const int ppos = a.positions[0];
      const AttUnit pu = att_unit(a, ppos, c, G, job_of(a, 1, sh).bytes0);
      int kv_issued = 0;
      auto stage_kv = [&](int j, uint8_t* dst) {
        if (!pu.in_att || j >= 4 * a.n_layers || (j & 3) != 1) return;
        const tpp_decode_layer& L = a.layers[j >> 2];
        const uint32_t rb = (uint32_t)pu.nst * 256u;
        mbar_arrive_expect_tx(&sm.kvbar, 2 * rb + (L.qn ? 256u : 0u) + (L.kn ? 256u : 0u));
        const int64_t row0 = ((int64_t)pu.h * a.Smax + pu.k0) * 128;
        if (rb) {
          bulk_load(dst, static_cast<const T*>(L.kc) + row0, rb, &sm.kvbar);
          bulk_load(dst + rb, static_cast<const T*>(L.vc) + row0, rb, &sm.kvbar);
        }
        if (L.qn) bulk_load(dst + 2 * rb, L.qn, 256u, &sm.kvbar);
        if (L.kn) bulk_load(dst + 2 * rb + 256, L.kn, 256u, &sm.kvbar);
        *(volatile int*)&sm.kv_issued = ++kv_issued;
      };
      int j = 0;
      for (; j < njobs && alive; ++j) {
        const int s = j & 1;
        if (j >= 2) {
          bool got = false;
          for (uint32_t i = 0; i < kSpinLimit && !got; ++i) {
            got = mbar_try_wait(&sm.empty[s], ((j >> 1) & 1) ^ 1);
            if (!got && *(volatile int*)&sm.abort_local) break;
          }
          if (!got) break;
        }
        const Job jb = job_of(a, j, sh);
        if (depth == 0 || j >= 4 * a.n_layers) {
          mbar_arrive_expect_tx(&sm.full[s], jb.bytes0 + jb.bytes1);
          if (jb.bytes0) bulk_load(slot[s], jb.src0, jb.bytes0, &sm.full[s]);
          if (jb.bytes1) bulk_load(slot[s] + jb.bytes0, jb.src1, jb.bytes1, &sm.full[s]);
          stage_kv(j, slot[s] + jb.bytes0 + jb.bytes1);
          continue;
        }
        for (int part = 0; part < 2 && alive; ++part) {
          const uint8_t* src = part ? jb.src1 : jb.src0;
          const uint32_t bytes = part ? jb.bytes1 : jb.bytes0;
          uint8_t* dst = slot[s] + (part ? jb.bytes0 : 0u);
          for (uint32_t off = 0; off < bytes; off += (uint32_t)a.pace_chunk) {
            if (q >= (uint32_t)depth && !pace_wait(q - depth, true)) { alive = false; break; }
            const uint32_t n = min((uint32_t)a.pace_chunk, bytes - off);
            mbar_arrive_expect_tx(&sm.pace[q % depth], n);
            bulk_load(dst + off, src + off, n, &sm.pace[q % depth]);
            ++q;
          }
        }
        if (alive) stage_kv(j, slot[s] + jb.bytes0 + jb.bytes1);
        // the slice has landed once its last depth chunks have
        for (uint32_t k = q > (uint32_t)depth ? q - depth : 0u; k < q && alive; ++k)
          if (!pace_wait(k, true)) alive = false;
        if (!alive) break;
        mbar_arrive(&sm.full[s]);
      }
      // chunks in flight land before the CTA can exit
      for (uint32_t k = q > (uint32_t)depth ? q - depth : 0u; k < q; ++k) pace_wait(k, false);
      *(volatile int*)&sm.issued = j;  // jobs whose full barrier completes
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
      // one grid barrier per step: v / G steps have run; epochs of this
      // step's phases follow those of every earlier step
      sm.ep_base = (uint32_t)(v / gridDim.x) * (uint32_t)(5 * a.n_layers + 2);
      sm.poll_fail = 0;
    }
    cons_sync();
    const uint32_t ep_base = sm.ep_base;
    // epoch of phase ph (0 QKV, 1 attention, 2 o-proj, 3 gate/up, 4 down) of layer l
    auto ep = [&](int l, int ph) { return ep_base + (uint32_t)(5 * l + ph + 1); };
    auto polled = [&]() { return *(volatile int*)&sm.poll_fail == 0; };
    const int64_t tok = a.tokens[0];
    const int pos = a.positions[0];
    const int R = (a.Hq + 2 * a.Hkv) * a.D;
    constexpr int GQ = NG;  // query heads per kv head
    const float inv_e = 1.f / (float)a.E;
    const uint32_t xs_s = smem_u32(sm.xh);
    const void* emb_row = static_cast<const T*>(a.emb) + tok * a.E;
    const uint32_t o_bytes = job_of(a, 1, sh).bytes0;
    const AttUnit au = att_unit(a, pos, c, G, o_bytes);
    int kv_waited = 0;
    for (int i = ctid; i < 256; i += kCons)
      sm.cs[i >> 7][i & 127] =
          __half2float((i < 128 ? a.cosp : a.sinp)[(int64_t)pos * a.cs_stride + (i & 127)]);
    int r0, r1;
    for (int l = 0; l < a.n_layers && ok; ++l) {
      const tpp_decode_layer& L = a.layers[l];
      // ---- QKV: qkv[r] = (x . Wqkv_f[r]) * rsqrt(mean(x^2) + eps) ----
      {
        const uint8_t* sl = acquire();
        DP_TS(8 + l * 16 + 0);
        if (l == 0)
          load_vec<T>(sm.xh, emb_row, a.E, ctid, sm.red);
        else
          load_tagged<T>(sm.xh, w.x, a.E, ep(l - 1, 4), ctid, sm.red, w, a.err, 62, &sm.poll_fail);
        cons_sync();
        if (!polled()) { release(); ok = false; break; }
        DP_TS(8 + l * 16 + 14);
        {  // this CTA's residual rows, for the o-proj and down phases
          const int e0 = sh.e0, e1 = sh.e1;
          for (int i = ctid; i < e1 - e0; i += kCons)
            sm.xres[i] = to_f32(reinterpret_cast<const T*>(sm.xh)[e0 + i]);
        }
        r0 = sh.q0; r1 = sh.q1;
        slice_dot<T>(smem_u32(sl), r1 - r0, a.E, xs_s, sm.gpart, warp, lane);
        const float rs = rsqrtf(sumsq_of(sm.red) * inv_e + a.eps);
        DP_TS(8 + l * 16 + 1);
        release();
        for (int r = ctid; r < r1 - r0; r += kCons)
          st_tag(w.qkv + r0 + r, rndT<T>(row_sum(sm.gpart, r1 - r0, a.E, r) * rs), ep(l, 0));
      }
      if (!ok) break;
      constexpr int NW = kCons / 32;
      const int S = au.S, h = au.h, sp = au.sp, k0 = au.k0, kend = au.kend, ktot = au.ktot;
      const int nst = au.nst;
      const bool in_att = au.in_att, own_new = au.own_new;
      const T* kc = static_cast<const T*>(L.kc) + (int64_t)h * a.Smax * 128;
      const T* vc = static_cast<const T*>(L.vc) + (int64_t)h * a.Smax * 128;
      // staged rows: K [nst][128], V [nst][128], q-norm, k-norm weights
      const T* kvs = reinterpret_cast<const T*>(slot[(4 * l + 1) & 1] + o_bytes);
      DP_TS(8 + l * 16 + 2);
      // ---- attention ----
      {
        if (in_att) {
          const int D = 128;
          if (!mbar_wait(&sm.kvbar, l & 1, a.err, 69)) sm.kvfail = 1;
          kv_waited = l + 1;
          float nwv[4] = {1.f, 1.f, 1.f, 1.f}, cv4[4], sv4[4];
          bool has_nw = false;
          if (warp <= GQ) {
            has_nw = (warp < GQ ? L.qn : L.kn) != nullptr;
            const T* nw = kvs + 2 * nst * 128 + (warp < GQ ? 0 : 128);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (has_nw) nwv[j] = to_f32(nw[lane * 4 + j]);
              cv4[j] = sm.cs[0][lane * 4 + j];
              sv4[j] = sm.cs[1][lane * 4 + j];
            }
          }
          // q rows of the G query heads, the new k row (normed + rotated) and v row
          if (warp <= GQ + 1) {
            const int row = warp < GQ ? (h * GQ + warp) : (warp == GQ ? a.Hq + h : a.Hq + a.Hkv + h);
            float x[4];
            {
              // the row's four tagged words of this lane, once QKV of this
              // layer has stored them
              const uint64_t* src = w.qkv + (int64_t)row * D + lane * 4;
              const uint64_t* const ptr[4] = {src, src + 1, src + 2, src + 3};
              uint64_t v4[4];
              if (!poll_tags<4>(ptr, 4, ep(l, 0), v4, w, a.err, 70)) sm.kvfail = 1;
#pragma unroll
              for (int j = 0; j < 4; ++j) x[j] = __uint_as_float((uint32_t)v4[j]);
              __syncwarp();
            }
            if (l < 2) DP_TS(476 + l * 10);
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
          if (l < 2) DP_TS(477 + l * 10);
          if (ctid < GQ) { sm.mrun[ctid] = -INFINITY; sm.lrun[ctid] = 0.f; }
          for (int i = ctid; i < kMaxG * 128; i += kCons) (&sm.oacc[0][0])[i] = 0.f;
          cons_sync();
          const bool kv_ok = sm.kvfail == 0;
          if (!kv_ok) {
            ok = false;
            if (ctid == 0) atomicExch(w.abortf, 1u);
          }
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
          // row `key` of K (which 0) or V (1): staged in shared memory, else
          // from the cache, else (the new key) the prologue's row
          auto row4 = [&](int which, int key, float* f) {
            const int kk = key - k0;
            if (kk < nst || key < kend) {
              const uint2 u =
                  kk < nst ? *reinterpret_cast<const uint2*>(kvs + (which * nst + kk) * 128 + lane * 4)
                           : *reinterpret_cast<const uint2*>((which ? vc : kc) + (int64_t)key * 128 +
                                                             lane * 4);
              const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
              for (int j = 0; j < 4; ++j) f[j] = to_f32(e[j]);
            } else {
              const float* src = which ? sm.vnew : sm.knew;
#pragma unroll
              for (int j = 0; j < 4; ++j) f[j] = src[lane * 4 + j];
            }
          };
          for (int t0 = 0; kv_ok && t0 < ktot; t0 += kTK) {
            const int nt = min(kTK, ktot - t0);
            // scores, 4 keys of a warp in flight at a time
            for (int i0 = warp; i0 < nt; i0 += 4 * NW) {
              float kf[4][4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * NW;
                if (i >= nt) continue;
                row4(0, k0 + t0 + i, kf[u]);
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
                const float pv = ex2_ftz(sm.sc[warp][i] - mn);
                sm.sc[warp][i] = pv;
                l += pv;
              }
              l = warp_sum(l);
              if (lane == 0) {
                const float cr = mo == -INFINITY ? 0.f : ex2_ftz(mo - mn);
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
                row4(1, k0 + t0 + i, vf[u]);
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
          // sum the warps' o accumulators: with <= 2 query heads each warp
          // stores its sums (over the now idle vector / score buffers) and a
          // thread per (head, dim) adds the 15; else shared-memory atomics
          const int npair = GQ * 128;
          if constexpr (NG <= 2) {
#pragma unroll
            for (int g = 0; g < NG; ++g)
              *reinterpret_cast<float4*>(&sm.wpart[warp][g][lane * 4]) =
                  make_float4(ow[g][0], ow[g][1], ow[g][2], ow[g][3]);
            cons_sync();
          } else {
#pragma unroll
            for (int g = 0; g < NG; ++g)
#pragma unroll
              for (int j = 0; j < 4; ++j) atomicAdd(&sm.oacc[g][lane * 4 + j], ow[g][j]);
            cons_sync();
          }
          if (kv_ok) {
            // partial (o, m, l) of each query head of this unit
            for (int pi = ctid; pi < npair; pi += kCons) {
              const int g = pi / 128, d = pi % 128;
              float t;
              if constexpr (NG <= 2) {
                t = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < kCons / 32; ++w2) t += sm.wpart[w2][g][d];
              } else {
                t = sm.oacc[g][d];
              }
              uint64_t* dst = w.part + ((int64_t)(h * GQ + g) * S + sp) * (128 + 2);
              st_tag(dst + d, t, ep(l, 1));
              if (d == 0) {
                st_tag(dst + 128, sm.mrun[g], ep(l, 1));
                st_tag(dst + 129, sm.lrun[g], ep(l, 1));
              }
            }
            if (l < 2) DP_TS(474 + l * 10);
            // unit 0 of head h merges the S partials once every one carries
            // this layer's epoch (no hand-shake between the units: the poll
            // of the tagged partials is the wait).  One (query head, dim)
            // pair per thread; the partials' (o, m, l) 8 at a time, every
            // load of a group in flight, folded with a running max.
            if (sp == 0) {
              for (int pi = ctid; pi < npair; pi += kCons) {
                const int g = pi / 128, d = pi % 128;
                const uint64_t* src = w.part + (int64_t)(h * GQ + g) * S * 130;
                float M = -INFINITY, den = 0.f, num = 0.f;
                for (int s0 = 0; s0 < S; s0 += 8) {
                  const int nin = min(8, S - s0);
                  const uint64_t* ptr[24];
#pragma unroll
                  for (int u = 0; u < 8; ++u) {
                    const uint64_t* sp2 = src + (int64_t)(s0 + (u < nin ? u : 0)) * 130;
                    ptr[u] = sp2 + 128;
                    ptr[8 + u] = sp2 + 129;
                    ptr[16 + u] = sp2 + d;
                  }
                  uint64_t tv[24];
                  if (!poll_tags<24>(ptr, 24, ep(l, 1), tv, w, a.err, 71)) {
                    *(volatile int*)&sm.poll_fail = 1;
                    break;
                  }
                  float mv[8], lv[8], ov[8];
#pragma unroll
                  for (int u = 0; u < 8; ++u) {
                    const bool in = u < nin;
                    mv[u] = in ? __uint_as_float((uint32_t)tv[u]) : -INFINITY;
                    lv[u] = in ? __uint_as_float((uint32_t)tv[8 + u]) : 0.f;
                    ov[u] = in ? __uint_as_float((uint32_t)tv[16 + u]) : 0.f;
                  }
                  float mc = M;
#pragma unroll
                  for (int u = 0; u < 8; ++u) mc = fmaxf(mc, mv[u]);
                  if (mc == -INFINITY) continue;
                  const float cr = M == -INFINITY ? 0.f : ex2_ftz(M - mc);
                  den *= cr;
                  num *= cr;
#pragma unroll
                  for (int u = 0; u < 8; ++u) {
                    const float e = mv[u] == -INFINITY ? 0.f : ex2_ftz(mv[u] - mc);
                    den = fmaf(e, lv[u], den);
                    num = fmaf(e, ov[u], num);
                  }
                  M = mc;
                }
                st_tag(w.o + (int64_t)(h * GQ + g) * 128 + d, rndT<T>(den > 0.f ? num / den : 0.f),
                       ep(l, 1));
              }
              cons_sync();
              if (!polled()) ok = false;
            }
          }
          if (l < 2) DP_TS(475 + l * 10);
        }
      }
      DP_TS(8 + l * 16 + 3);
      if (!ok) break;
      DP_TS(8 + l * 16 + 4);
      // ---- o-proj + residual: x[r] = x[r] + o . Wo[r] ----
      {
        const uint8_t* sl = acquire();
        DP_TS(8 + l * 16 + 5);
        const int K = a.Hq * a.D;
        load_tagged<T>(sm.xh, w.o, K, ep(l, 1), ctid, nullptr, w, a.err, 63, &sm.poll_fail);
        cons_sync();
        if (!polled()) { release(); ok = false; break; }
        DP_TS(8 + l * 16 + 15);
        r0 = sh.e0; r1 = sh.e1;
        slice_dot<T>(smem_u32(sl), r1 - r0, K, xs_s, sm.gpart, warp, lane);
        release();
        for (int r = ctid; r < r1 - r0; r += kCons) {
          const T nv = from_f32<T>(sm.xres[r] + row_sum(sm.gpart, r1 - r0, K, r));
          st_tag(w.x + r0 + r, to_f32(nv), ep(l, 2));
          sm.xres[r] = to_f32(nv);
        }
      }
      DP_TS(8 + l * 16 + 6);
      if (!ok) break;
      DP_TS(8 + l * 16 + 7);
      // ---- gate/up + SwiGLU: ff[f] = silu(g * rs) * (u * rs) ----
      {
        const uint8_t* sl = acquire();
        load_tagged<T>(sm.xh, w.x, a.E, ep(l, 2), ctid, sm.red, w, a.err, 64, &sm.poll_fail);
        cons_sync();
        if (!polled()) { release(); ok = false; break; }
        DP_TS(8 + l * 16 + 8);
        r0 = sh.f0; r1 = sh.f1;
        const int nf = r1 - r0;
        // the slice: nf gate rows, then the nf up rows of the same features
        slice_dot<T>(smem_u32(sl), 2 * nf, a.E, xs_s, sm.gpart, warp, lane);
        const float rs = rsqrtf(sumsq_of(sm.red) * inv_e + a.eps);
        release();
        for (int f = ctid; f < nf; f += kCons) {
          const float g = row_sum(sm.gpart, 2 * nf, a.E, f);
          const float u = row_sum(sm.gpart, 2 * nf, a.E, nf + f);
          st_tag(w.ff + r0 + f, rndT<T>(act_silu(g * rs) * (u * rs)), ep(l, 3));
        }
      }
      DP_TS(8 + l * 16 + 9);
      if (!ok) break;
      DP_TS(8 + l * 16 + 10);
      // ---- down + residual: x[r] = x[r] + ff . Wd[r] ----
      {
        const uint8_t* sl = acquire();
        load_tagged<T>(sm.xh, w.ff, a.F, ep(l, 3), ctid, nullptr, w, a.err, 65, &sm.poll_fail);
        cons_sync();
        if (!polled()) { release(); ok = false; break; }
        DP_TS(8 + l * 16 + 11);
        r0 = sh.e0; r1 = sh.e1;
        slice_dot<T>(smem_u32(sl), r1 - r0, a.F, xs_s, sm.gpart, warp, lane);
        release();
        for (int r = ctid; r < r1 - r0; r += kCons) {
          const T nv = from_f32<T>(sm.xres[r] + row_sum(sm.gpart, r1 - r0, a.F, r));
          st_tag(w.x + r0 + r, to_f32(nv), ep(l, 4));
          sm.xres[r] = to_f32(nv);
        }
      }
      DP_TS(8 + l * 16 + 12);
      if (!ok) break;
      DP_TS(8 + l * 16 + 13);
    }
    // ---- LM head: logits = (x . Wh_f) * rs, per-CTA argmax ----
    if (ok) {
      load_tagged<T>(sm.xh, w.x, a.E, ep(a.n_layers - 1, 4), ctid, sm.red, w, a.err, 66,
                     &sm.poll_fail);
      cons_sync();
      ok = polled();
    }
    if (ok) {
      const float rs = rsqrtf(sumsq_of(sm.red) * inv_e + a.eps);
      const int v0 = sh.v0, v1 = sh.v1;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int q = 0; jc < njobs && ok; ++q) {
        const uint8_t* sl = acquire();
        const int rr0 = v0 + q * a.lm_rows_per_job, rr1 = min(v1, rr0 + a.lm_rows_per_job);
        // partials of consecutive jobs alternate halves of gpart, so a job's
        // epilogue can run while the next job's dot products are written
        float* gp = sm.gpart + (q & 1) * (kMaxPart / 2);
        slice_dot<T>(smem_u32(sl), rr1 - rr0, a.E, xs_s, gp, warp, lane);
        release();
        for (int r = ctid; r < rr1 - rr0; r += kCons) {
          const float vi = rndT<T>(row_sum(gp, rr1 - rr0, a.E, r) * rs);
          static_cast<T*>(a.logits)[rr0 + r] = from_f32<T>(vi);
          if (vi > bv || (vi == bv && rr0 + r < bi)) { bv = vi; bi = rr0 + r; }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        if (v2 > bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; }
      }
      if (lane == 0) { sm.best_v[warp] = bv; sm.best_i[warp] = bi; }
      cons_sync();
      if (ctid == 0) {
        for (int i = 1; i < kCons / 32; ++i)
          if (sm.best_v[i] > bv || (sm.best_v[i] == bv && sm.best_i[i] < bi)) {
            bv = sm.best_v[i];
            bi = sm.best_i[i];
          }
        st_tag(w.amax_v + c, bv, ep(a.n_layers, 0));
        st_tag(w.amax_i + c, __int_as_float(bi), ep(a.n_layers, 0));
      }
      DP_TS(500);
      // every CTA counts itself in for this step (the count sets the next
      // step's epochs) and leaves; CTA 0 waits for the others' tagged picks
      grid_arrive(w, bar_target);
      DP_TS(501);
      if (ok && c == 0 && warp == 0) {
        float v = -INFINITY;
        int idx = 0x7fffffff;
        const uint64_t* ptr[16];
        int n = 0;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = lane + 32 * u;
          const int ic = i < G ? i : 0;
          ptr[u] = w.amax_v + ic;
          ptr[8 + u] = w.amax_i + ic;
        }
        for (int u = 0; u < 8; ++u) n += lane + 32 * u < G ? 1 : 0;
        uint64_t tv[16];
        if (!poll_tags<16>(ptr, 16, ep(a.n_layers, 0), tv, w, a.err, 67)) ok = false;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (u >= n) break;
          const float vv = __uint_as_float((uint32_t)tv[u]);
          const int ii = (int)(uint32_t)tv[8 + u];
          if (vv > v || (vv == v && ii < idx)) { v = vv; idx = ii; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
          const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
          if (v2 > v || (v2 == v && i2 < idx)) { v = v2; idx = i2; }
        }
        const bool all_ok = __all_sync(0xffffffffu, ok);
        if (lane == 0 && all_ok) {
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
    if (ctid == 0) { sm.red[0] = __int_as_float(jc); sm.red[1] = __int_as_float(kv_waited); }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int consumed = __float_as_int(sm.red[0]);
    for (int j = consumed; j < sm.issued; ++j) mbar_wait(&sm.full[j & 1], (j >> 1) & 1, a.err, 68);
    for (int k = __float_as_int(sm.red[1]); k < sm.kv_issued; ++k)
      mbar_wait(&sm.kvbar, k & 1, a.err, 68);
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
         per(R) * (E + kPad) * 2 <= kSlot && per(E) * (Hq * D + kPad) * 2 <= kSlot &&
         2 * per(F) * (E + kPad) * 2 <= kSlot && per(E) * (F + kPad) * 2 <= kSlot &&
         per(E) <= kMaxRes &&
         E % kKC == 0 && (Hq * D) % kKC == 0 && F % kKC == 0 &&
         per(R) * (E / kKC) <= kMaxPart && 2 * per(F) * (E / kKC) <= kMaxPart &&
         per(E) * (Hq * D / kKC) <= kMaxPart && per(E) * (F / kKC) <= kMaxPart &&
         2 * (int64_t)(kSlot / (2 * (E + kPad))) * (E / kKC) <= kMaxPart;
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
  a.lm_rows_per_job = (int)(kSlot / ((E + kPad) * 2));
  // TPP_DP_PACE="<chunk KiB>,<chunks in flight>" (",0": one burst per slice)
  a.pace_chunk = 16 * 1024;
  a.pace_depth = 8;
  if (const char* pe = getenv("TPP_DP_PACE")) {
    int kb = 0, d = 0;
    if (sscanf(pe, "%d,%d", &kb, &d) == 2 && kb >= 1 && kb <= 96 && d >= 0 && d <= kPaceMax) {
      a.pace_chunk = kb * 1024;
      a.pace_depth = d;
    }
  }
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
