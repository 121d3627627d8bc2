// Shared device/host helpers for the sm_100a kernels of libtpp_b200.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>
#include <utility>
#include "../../include/tpp_b200.h"

namespace tpp {

// ---------------------------------------------------------------------------
// Host-side error plumbing: thread-local message + status codes.
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
void count_launch(uint64_t n = 1);

#define TPP_REQUIRE(cond, code, msg)                 \
  do {                                               \
    if (!(cond)) {                                   \
      ::tpp::set_error(std::string(__func__) + ": " + (msg)); \
      return (code);                                 \
    }                                                \
  } while (0)

// Checks the launch that was just issued; returns TPP_ERR_LAUNCH on failure.
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// SMs a decode-step launch plans for: all of the device's unless the calling
// host thread set a budget (tpp_set_sm_budget), so that independent
// sub-batches recorded as parallel graph branches each size their grids for
// their share of the GPU and run side by side.
int sm_budget();

// ---------------------------------------------------------------------------
// Element types.
// ---------------------------------------------------------------------------
template <typename T> struct Vec;  // 16-byte vector of 8 elements
template <> struct Vec<__half> { using type = uint4; };
template <> struct Vec<__nv_bfloat16> { using type = uint4; };

__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }

// Unpack 8 packed 16-bit elements (a uint4) into fp32.
// Two packed 16-bit elements (low half first) of a 32-bit word into fp32,
// with register operations only (taking the address of a register vector
// can put it in local memory).
template <typename T> struct Unpack2;
template <> struct Unpack2<__half> {
  static __device__ __forceinline__ void run(uint32_t w, float& lo, float& hi) {
    unsigned short a, b;
    asm("mov.b32 {%0, %1}, %2;" : "=h"(a), "=h"(b) : "r"(w));
    lo = __half2float(__ushort_as_half(a));
    hi = __half2float(__ushort_as_half(b));
  }
};
template <> struct Unpack2<__nv_bfloat16> {
  static __device__ __forceinline__ void run(uint32_t w, float& lo, float& hi) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  }
};
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  Unpack2<T>::run(u.x, f[0], f[1]);
  Unpack2<T>::run(u.y, f[2], f[3]);
  Unpack2<T>::run(u.z, f[4], f[5]);
  Unpack2<T>::run(u.w, f[6], f[7]);
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  T* e = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(f[i]);
  return u;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// 256-bit streaming load of data read exactly once (weights): evict-first in
// L2, no L1 allocation.  p must be 32-byte aligned.
__device__ __forceinline__ void ldg_stream_v8(const void* p, uint4& lo, uint4& hi) {
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y), "=r"(hi.z),
        "=r"(hi.w)
      : "l"(p));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Activations, fp32 in/out, following csrc/activation/activation.cuh:26-67
// of the reference (GeLU-tanh with sqrt(2/pi) and 0.044715; SiLU x/(1+e^-x)).
// 2^x with the hardware's approximate base-2 exponential (PTX ex2.approx,
// flush-to-zero): one special-function instruction.  Relative error about
// 2^-22 (PTX ISA bound); results below 2^-126 become 0, which a softmax
// weight of that size is anyway.  -inf gives 0.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}
// Packed pairs of fp32 (low word first) for the sm_100 two-lane fp32 ops.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// a * b + c and a + b on both lanes of packed fp32 pairs (round to nearest).
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float act_silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float act_gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}
__device__ __forceinline__ float act_relu(float x) { return fmaxf(x, 0.0f); }
__device__ __forceinline__ float apply_act(int act, float x) {
  switch (act) {
    case TPP_ACT_SILU: return act_silu(x);
    case TPP_ACT_GELU: return act_gelu_tanh(x);
    case TPP_ACT_RELU: return act_relu(x);
    default: return x;
  }
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).  Every kernel of this library is
// launched with programmatic stream serialization allowed, calls pdl_wait()
// before it touches memory written by earlier work on the stream (and before
// its first global write), and pdl_trigger() once its dependents may be
// scheduled.  The next kernel can therefore be resident and run its
// independent prologue (e.g. start streaming weights) while this one drains.
// Outside a PDL launch both instructions are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// PDL on unless the environment sets TPP_PDL=0 (for A/B measurements).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
int launch(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
           cudaStream_t st, unsigned cluster_y, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_y > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = cluster_y;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return TPP_ERR_LAUNCH;
  }
  return check_launch(what);
}

// Dispatch a dtype code to a template functor.
#define TPP_DISPATCH_HALF(dtype, T, ...)                         \
  [&]() -> int {                                                 \
    if ((dtype) == TPP_F16) { using T = __half; return __VA_ARGS__(); }          \
    if ((dtype) == TPP_BF16) { using T = __nv_bfloat16; return __VA_ARGS__(); }  \
    ::tpp::set_error(std::string(__func__) + ": dtype must be f16 (0) or bf16 (1)"); \
    return (int)TPP_ERR_DTYPE;                                   \
  }()

}  // namespace tpp
