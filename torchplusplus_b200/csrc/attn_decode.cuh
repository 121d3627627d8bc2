// Shared declarations of the decode-attention kernels.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

namespace tpp {

// Arguments of the tensor-core decode kernel (attn_decode_mma.cu).
struct DecMmaArgs {
  const void* q; int64_t q_sb, q_sh;
  void* o; int64_t o_sb, o_sh;
  const int32_t* seqlens; int64_t max_seqlen;
  int Hq, Hkv, G, passes;
  int64_t window_left;
  float scale_log2;
  int splits;
  int cluster;     // 1: merge splits in the cluster; 0: write partials to ws
  float* ws_o;     // [B, Hq, splits, D]
  float* ws_lse;   // [B, Hq, splits]
  int* err;
};

// Split count of the tensor-core decode path for B sequences, Hq/Hkv heads
// and `range` keys (about two CTAs per SM).
int decode_mma_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t range);
// Launches the tensor-core decode kernel (and nothing else).
int decode_mma_launch(DecMmaArgs& a, const void* k_cache, const void* v_cache, int64_t c_sb,
                      int64_t c_sh, int64_t c_ss, int64_t B, int64_t D, int dtype,
                      cudaStream_t st);

}  // namespace tpp
