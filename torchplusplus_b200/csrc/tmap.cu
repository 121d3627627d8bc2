// Host helper: tensor-map creation through cudaGetDriverEntryPoint, plus the
// device error flag shared by kernels with bounded waits.
#include <mutex>
#include "tc_common.cuh"

namespace tpp {

static __device__ int g_device_error = 0;

int* device_error_flag() {
  static int* cached[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

namespace {
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn g_encode = nullptr;
std::once_flag g_once;
}  // namespace

int make_tmap(CUtensorMap* map, const void* base, int dtype, int rank, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  std::call_once(g_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeFn>(fn);
  });
  if (!g_encode) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return TPP_ERR_LAUNCH;
  }
  CUtensorMapDataType dt;
  switch (dtype) {
    case TPP_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case TPP_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case TPP_F32: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    case kTmapU8: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    default: set_error("make_tmap: bad dtype"); return TPP_ERR_DTYPE;
  }
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, dt, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
    return TPP_ERR_ALIGN;
  }
  return TPP_OK;
}

}  // namespace tpp

namespace {
// The expiry path of mbar_wait, exercised on purpose: one thread waits on an
// mbarrier that nothing arrives on and no copy completes on, with a short
// poll limit; the wait gives up, raises the flag and the kernel returns.
__global__ void bounded_wait_expiry_kernel(int* err, uint32_t polls, int code) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  tpp::mbar_init(&bar, 1);
  tpp::fence_mbar_init();
  tpp::mbar_wait(&bar, 0, err, code, polls);
}
}  // namespace

extern "C" int tpp_debug_expire_wait(uint32_t polls, int code, void* stream) {
  TPP_REQUIRE(polls > 0 && polls <= (1u << 16) && code != 0, TPP_ERR_SHAPE,
              "polls must be in [1, 65536] and code nonzero");
  int* err = tpp::device_error_flag();
  TPP_REQUIRE(err != nullptr, TPP_ERR_LAUNCH, "device error flag unavailable");
  bounded_wait_expiry_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(err, polls,
                                                                                   code);
  return tpp::check_launch("bounded_wait_expiry_kernel");
}

// Reads and clears the device-side error flag raised by bounded waits.
extern "C" int tpp_device_error(void* stream) {
  int v = 0, zero = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyFromSymbolAsync(&v, tpp::g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                st) != cudaSuccess ||
      cudaMemcpyToSymbolAsync(tpp::g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                              st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    tpp::set_error(std::string("tpp_device_error: ") + cudaGetErrorString(cudaGetLastError()));
    return -TPP_ERR_LAUNCH;
  }
  return v;
}
