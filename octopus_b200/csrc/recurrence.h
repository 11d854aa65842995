// Linear recurrences (GDN delta rule, simple GLA) and causal conv1d: launch interfaces.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace octo {

struct RecurParams {
  const __nv_bfloat16* q;   // [rows, H * dk] (row strides ldq / ldk / ldv)
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;   // [rows, H * dv], dv == dk
  int ldq, ldk, ldv;
  const float* g;           // [rows, H] log gate (a = exp(g))
  const float* beta;        // [rows, H] delta-rule step (GDN only)
  __nv_bfloat16* o;         // [rows, H * dv]
  int ldo;
  const int32_t* seg_start; // [n_seg] first row of each segment
  const int32_t* seg_len;   // [n_seg] rows of each segment
  int H;
  float scale;
  int delta;                // 1: gated delta rule, 0: simple GLA
  const float* init_state;  // [n_init, H, dv, dk] or null
  const int32_t* init_idx;  // [n_seg] row of init_state per segment (-1: zeros)
  float* final_state;       // [n_seg, H, dv, dk] or null
  float* ckpt;              // [sum chunks, H, dv, dk] states every recur_chunk() tokens (needed by backward)
  const int32_t* ckpt_off;  // [n_seg] first checkpoint of each segment
  float* scratch;           // backward: recur_scratch_floats(n_seg, H, dk)
};

struct RecurGrads {
  const __nv_bfloat16* d_o;
  __nv_bfloat16* dq;  // same strides as q / k / v
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  float* dg;          // [rows, H]
  float* dbeta;       // [rows, H] (GDN)
  const float* d_final;  // [n_seg, H, dv, dk] or null
  float* d_init;         // [n_seg, H, dv, dk] or null (per segment)
};

int recur_chunk();
size_t recur_scratch_floats(int n_seg, int H, int dk);
void recur_fwd(const RecurParams& p, int n_seg, int dk, cudaStream_t st);
void recur_bwd(const RecurParams& p, const RecurGrads& g, int n_seg, int dk, cudaStream_t st);

struct ConvParams {
  const __nv_bfloat16* x;   // [rows, C], row stride ldx
  int ldx;
  const float* w;           // [C, W] depthwise taps
  const float* bias;        // [C] or null
  __nv_bfloat16* y;         // [rows, C], row stride ldy
  int ldy;
  const int32_t* cu;        // [n_seg + 1]
  int C, W;                 // W <= 8
  const float* ctx;         // [n_ctx, W - 1, C] context rows before each segment, or null
  const int32_t* ctx_idx;   // [n_seg] (-1: zeros)
  int silu;
};

void conv_fwd(const ConvParams& p, int n_seg, cudaStream_t st);
void conv_bwd(const ConvParams& p, int n_seg, const void* dy, void* dx, float* dw, float* dbias, float* dctx,
              cudaStream_t st);

}  // namespace octo
