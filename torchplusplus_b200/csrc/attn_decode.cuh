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
  // Fused mode (qkv != nullptr): q and the step's new k/v come raw from the
  // QKV projection row [q (Hq*D) | k (Hkv*D) | v (Hkv*D)]; the kernel applies
  // the q/k RMSNorm (weights may be null) and RoPE at positions[b], writes
  // the new k/v into the cache at that row and uses them directly.  Requires
  // positions[b] == seqlens[b] - 1.
  const void* qkv; int64_t qkv_sb;
  const void* qn_w; const void* kn_w; float eps;
  const void* cosp; const void* sinp; int64_t cs_stride;  // fp16 tables [ctx, D]
  const int32_t* positions;
  void* kc; void* vc; int64_t c_sb, c_sh, c_ss;           // cache (element strides)
  // Paged mode (table != nullptr): the caches are block pools
  // [num_blocks][Hkv][64][D]; key k of sequence b lives in block
  // table[b * tbl_stride + k / 64], row k % 64.
  const int32_t* table; int64_t tbl_stride; int64_t num_blocks;
#ifdef TPP_DEBUG_STAMPS
  unsigned dbg_id;
#endif
};

// Split count of the tensor-core decode path for B sequences, Hq/Hkv heads
// and `range` keys (about two CTAs per SM).
int decode_mma_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t range);
// Launches the tensor-core decode kernel (and nothing else).
int decode_mma_launch(DecMmaArgs& a, const void* k_cache, const void* v_cache, int64_t c_sb,
                      int64_t c_sh, int64_t c_ss, int64_t B, int64_t D, int dtype,
                      cudaStream_t st);

}  // namespace tpp
