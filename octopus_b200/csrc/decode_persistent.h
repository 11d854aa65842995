// Persistent paged decode attention (decode_persistent.cu): parameters and launcher.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace octo {

struct DecodePersistParams {
  const __nv_bfloat16* q;        // [B, Hq * 128], row stride ldq
  const __nv_bfloat16* k_cache;  // [slots, Hkv * 128]
  const __nv_bfloat16* v_cache;
  __nv_bfloat16* o;              // [B, Hq * 128], row stride ldo
  const int32_t* kv_start;       // [B]
  const int32_t* kv_len;         // [B]
  const int32_t* kv_indices;
  float* part_o;                 // [B, Hq, splits, 128] (splits > 1)
  float* part_lse;               // [B, Hq, splits]
  int ldq, ldo;
  int B, Hq, Hkv;
  int num_splits;
  float scale;
};

int decode_persistent_smem_bytes();
void decode_persistent_launch(const DecodePersistParams& p, int grid, int* status, cudaStream_t st);

}  // namespace octo
