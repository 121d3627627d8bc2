// DSMEM bulk-copy probe: CTA 0 of a cluster copies S bytes of its shared
// memory into each peer's shared memory with cp.async.bulk.shared::cluster.
// shared::cta (completion on the peer's mbarrier); each peer stamps
// globaltimer when its copy lands; CTA 0 stamps before issuing.
#include <cstdio>
#include <cuda_runtime.h>
#include "../tc_common.cuh"
using namespace tpp;

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t;
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r; asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r)); return r;
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r; asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank)); return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned; barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void probe(unsigned long long* out, int bytes, int npeers) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  const uint32_t rank = cluster_rank();
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  cluster_sync();
  if (threadIdx.x == 0) {
    if (rank != 0) mbar_arrive_expect_tx(&bar, bytes);
  }
  cluster_sync();
  if (threadIdx.x == 0) {
    if (rank == 0) {
      out[blockIdx.x * 2] = gtime();
      for (int p = 1; p <= npeers; ++p) {
        const uint32_t dst = mapa(smem_u32(smem), p), mb = mapa(smem_u32(&bar), p);
        asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     :: "r"(dst), "r"(smem_u32(smem)), "r"(bytes), "r"(mb) : "memory");
      }
    } else {
      mbar_wait(&bar, 0, nullptr, 0);
      out[blockIdx.x * 2 + 1] = gtime();
    }
  }
  cluster_sync();
}

int main() {
  unsigned long long *d, h[2 * 148 * 8];
  cudaMalloc(&d, sizeof(h));
  cudaFuncSetAttribute(probe, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024);
  for (int cl : {2, 4, 8}) {
    for (int bytes : {16384, 32768, 65536, 131072}) {
      const int ctas = 144;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(ctas); cfg.blockDim = dim3(128); cfg.dynamicSmemBytes = 128 * 1024;
      cudaLaunchAttribute a[1];
      a[0].id = cudaLaunchAttributeClusterDimension; a[0].val.clusterDim.x = cl; a[0].val.clusterDim.y = 1; a[0].val.clusterDim.z = 1;
      cfg.attrs = a; cfg.numAttrs = 1;
      double best = 1e30;
      for (int rep = 0; rep < 5; ++rep) {
        cudaMemset(d, 0, sizeof(h));
        cudaError_t e = cudaLaunchKernelEx(&cfg, probe, d, bytes, cl - 1);
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess) { printf("err %s\n", cudaGetErrorString(e)); return 1; }
        cudaMemcpy(h, d, sizeof(unsigned long long) * 2 * ctas, cudaMemcpyDeviceToHost);
        // per cluster: last peer arrival - sender start; report median-ish (max over clusters)
        double mx = 0;
        for (int c = 0; c < ctas / cl; ++c) {
          unsigned long long s = h[2 * (c * cl)], last = 0;
          for (int p = 1; p < cl; ++p) last = h[2 * (c * cl + p) + 1] > last ? h[2 * (c * cl + p) + 1] : last;
          mx = (double)(last - s) > mx ? (double)(last - s) : mx;
        }
        best = mx < best ? mx : best;
      }
      printf("cluster %d bytes %6d x %d peers: %7.0f ns  -> %6.1f GB/s out of the sender SM (all clusters at once)\n",
             cl, bytes, cl - 1, best, (double)bytes * (cl - 1) / best);
    }
  }
  return 0;
}
