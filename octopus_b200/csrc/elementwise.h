// Launch functions of elementwise.cu (no torch types).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace octo {
void head_combine(const float* part, int M, int T, const int32_t* labels, float* logp, float* ent, float* lse,
                  cudaStream_t st);
void sample_combine(const float* part, int M, int T, uint64_t seed, const int64_t* row_stream, int64_t* tokens,
                    float* logprob, cudaStream_t st);
void rmsnorm_fwd(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, __nv_bfloat16* y, int ldy, float* rstd,
                 int T, int H, float eps, int plus_one, cudaStream_t st);
void rmsnorm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w, const float* rstd,
                 const __nv_bfloat16* dres, __nv_bfloat16* dx, float* dw, int T, int H, int plus_one,
                 cudaStream_t st);
void rope_apply(__nv_bfloat16* qkv, int ld, const int32_t* pos, int T, int Hq, int Hkv, int D, float theta,
                bool inverse, cudaStream_t st);
void swiglu_fwd(const __nv_bfloat16* gu, __nv_bfloat16* out, int T, int F, cudaStream_t st);
void swiglu_bwd(const __nv_bfloat16* gu, const __nv_bfloat16* dout, __nv_bfloat16* dgu, int T, int F,
                cudaStream_t st);
void embed_fwd(const int64_t* ids, const __nv_bfloat16* W, __nv_bfloat16* out, int T, int H, int V, int* status,
               cudaStream_t st);
void embed_bwd(const int64_t* ids, const __nv_bfloat16* dout, float* dW, int T, int H, int V, int* status,
               cudaStream_t st);
void kv_write(const __nv_bfloat16* qkv, int ld, int Hq, int Hkv, int D, const int64_t* slots, __nv_bfloat16* kc,
              __nv_bfloat16* vc, int T, long long n_slots, int* status, cudaStream_t st);
void sqnorm_accum(const float* g, long n, float* out, cudaStream_t st);
// decode_fused.cu: split-K finishes fused with the layer's next element-wise step
void splitk_finish_norm(const float* ws, int splits, int M, int N, const __nv_bfloat16* bias,
                        const __nv_bfloat16* res, int ldr, __nv_bfloat16* x, int ldx, const __nv_bfloat16* w,
                        float eps, bool plus_one, __nv_bfloat16* h, int ldh, cudaStream_t st);
void splitk_finish_qkv(const float* ws, int splits, int M, int Hq, int Hkv, int D, const __nv_bfloat16* bias,
                       const int32_t* pos, float theta, __nv_bfloat16* q, int ldq, const int64_t* slots,
                       __nv_bfloat16* kc, __nv_bfloat16* vc, long long n_slots, int* status, cudaStream_t st);
void adamw_step(float* p, const float* g, float* m, float* v, __nv_bfloat16* p16, long n, float lr, float b1,
                float b2, float eps, float wd, int step, const float* sqnorm, float max_norm, float grad_scale,
                cudaStream_t st);
}  // namespace octo
