// Shared-prefix paged decode attention (decode_shared.cu): parameters and launcher.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace octo {

constexpr int kSegRows = 16;  // rows one segment may serve (table stride)

struct DecodeSharedParams {
  const __nv_bfloat16* q;        // [B, Hq * 128], row stride ldq
  const __nv_bfloat16* k_cache;  // [slots, Hkv * 128]
  const __nv_bfloat16* v_cache;
  __nv_bfloat16* o;              // [B, Hq * 128], row stride ldo
  const int32_t* kv_indices;     // key slot lists
  const int32_t* kv_len;         // [B] current keys of each row (dynamic segments end there)
  const int32_t* seg_rows;       // [nseg, kSegRows] rows served (-1 = none)
  const int32_t* seg_slot;       // [nseg, kSegRows] first partial slot of each row for this segment
  const int32_t* seg_start;      // [nseg] index-list offset of the segment's first key
  const int32_t* seg_len;        // [nseg] keys; -1: dynamic (kv_len[row 0] - seg_off)
  const int32_t* seg_off;        // [nseg] the segment's offset inside its row's key list
  const int32_t* items;          // [n_chunks] seg << 8 | chunk; work item i -> items[i / Hkv], kv head i % Hkv
  const int32_t* n_items;        // device scalars: [0] n_chunks * Hkv, [1] keys per work item (the plan's chunk)
  const int32_t* row_nslot;      // [B] slots a row's partials occupy
  float* part_o;                 // [B, Hq, max_slots, 128]
  float* part_lse;               // [B, Hq, max_slots] (log2 units)
  int ldq, ldo;
  int B, Hq, Hkv;
  int max_slots;
  int chunk;                     // largest keys per work item any plan may use (host checks)
  float scale;
  long long n_slots;             // rows of the K / V caches: slot ids outside [0, n_slots) are reported
                                 // (kErrBadIndex) and read as slot 0 instead; 0 disables the check
  unsigned long long* trace;     // optional event timestamps of CTA 0 (tcgen05 kernel; debugging)
};

int decode_shared_smem_bytes();
void decode_shared_launch(const DecodeSharedParams& p, int grid, int* status, cudaStream_t st);
// merges every row's partial slots into p.o
void decode_shared_combine(const DecodeSharedParams& p, cudaStream_t st);

// tcgen05 variant (decode_shared_tc.cu): TMA maps of the K / V caches [slots, Hkv * 128],
// box 64 columns x 64 rows, 128-byte swizzle.  Segments may serve up to 128 / G rows.
struct DecodeSharedMaps {
  CUtensorMap k, v;
};
int decode_shared_tc_smem_bytes();
// (persistent: the grid is derived from the SM count)
void decode_shared_tc_launch(const DecodeSharedParams& p, const DecodeSharedMaps& maps, int sms, int* status,
                             cudaStream_t st);

}  // namespace octo
