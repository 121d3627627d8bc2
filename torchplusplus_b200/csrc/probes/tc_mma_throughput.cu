// tcgen05.mma throughput probe: back-to-back MMAs into one TMEM accumulator,
// one commit, timed with clock64 by the issuing thread.  Operands: zeroed
// smem tiles (values do not matter), 128B-swizzle K-major descriptors.
#include <cstdio>
#include <cuda_runtime.h>
#include "../tc_common.cuh"
using namespace tpp;

template <int M, int N>
__global__ void __launch_bounds__(128, 1) probe(long long* out, int nmma, int reps) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;                 // M x 64 bf16 = M*128 B
  uint8_t* sB = smem + 128 * 128;     // N x 64
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t slot;
  for (int i = threadIdx.x; i < (128 * 128 + 256 * 128) / 4; i += blockDim.x) ((uint32_t*)smem)[i] = 0;
  if (threadIdx.x == 0) { mbar_init(&bar, 1); fence_mbar_init(); }
  if (threadIdx.x < 32) tmem_alloc(&slot, 256);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot;
  constexpr uint32_t idesc = make_idesc_f16(M, N, 1, 0, 0);
  long long best = 1ll << 62;
  if (threadIdx.x == 0) {
    const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
    for (int r = 0; r < reps; ++r) {
      const long long t0 = clock64();
      for (int i = 0; i < nmma; ++i) {
        const int k = i & 3;
        tc_mma_f16(tmem, make_sdesc(a0 + k * 32, 16, 1024, 2), make_sdesc(b0 + k * 32, 16, 1024, 2), idesc, i != 0);
      }
      tc_commit(&bar);
      mbar_wait(&bar, r & 1, nullptr, 0);
      const long long t1 = clock64();
      if (t1 - t0 < best) best = t1 - t0;
    }
    out[blockIdx.x] = best;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem, 256);
}

template <int M, int N>
void run(long long* d, long long* h, int ctas) {
  const int ns[] = {1, 2, 4, 8, 16, 64, 256};
  cudaFuncSetAttribute(probe<M, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  for (int n : ns) {
    probe<M, N><<<ctas, 128, 64 * 1024>>>(d, n, 5);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { printf("err %s\n", cudaGetErrorString(e)); return; }
    cudaMemcpy(h, d, sizeof(long long) * ctas, cudaMemcpyDeviceToHost);
    long long mx = 0; for (int i = 0; i < ctas; ++i) mx = h[i] > mx ? h[i] : mx;
    const double flop = 2.0 * M * N * 16 * n;
    printf("M%3d N%3d ctas %3d nmma %4d: %7lld clk  %6.1f clk/mma  %7.0f FLOP/clk/SM\n", M, N, ctas, n, mx,
           (double)mx / n, flop / mx);
  }
}

int main() {
  long long *d, h[256];
  cudaMalloc(&d, sizeof(long long) * 256);
  for (int ctas : {1, 148}) {
    run<64, 32>(d, h, ctas);
    run<128, 32>(d, h, ctas);
    run<128, 64>(d, h, ctas);
    run<128, 128>(d, h, ctas);
    run<128, 256>(d, h, ctas);
  }
  return 0;
}
