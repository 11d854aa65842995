// Host-side helpers: TMA tensor-map encoding through the driver entry point, device
// properties, and the per-device status word the kernels report into.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

namespace octo {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "octopus_b200: cannot resolve cuTensorMapEncodeTiled");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2D bf16 tensor map over a row-major [outer, inner] matrix with row stride
// `row_stride_elems`, tile box {box_inner, box_outer}, 128-byte swizzle.
inline CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                                     uint32_t box_inner, uint32_t box_outer,
                                     CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  TORCH_CHECK(ptr != nullptr && inner > 0 && outer > 0, "TMA map of an empty tensor");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tmap_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", static_cast<int>(r));
  return m;
}

inline int num_sms(int device) {
  static int cached[64] = {0};
  if (cached[device] == 0) {
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, device);
    cached[device] = p.multiProcessorCount;
  }
  return cached[device];
}

// GEMM N-tile width for an M x N problem on `sms` SMs (hint 64/128/256 forces it).
int pick_bn(int M, int N, int sms, int hint);
// Split count of `k_blocks` K blocks into about `want` splits with none empty (the kernel
// gives split s the blocks [s * per, s * per + per) with per = ceil(k_blocks / splits)).
inline int nonempty_splits(int k_blocks, int want) {
  if (want <= 1 || k_blocks <= 1) return 1;
  const int per = (k_blocks + want - 1) / want;
  return (k_blocks + per - 1) / per;
}  // L2 prefetch distance (K-blocks) of B for an M-row GEMM

// Status word: int32[2] per device = {code, where}.  Zero means OK.
int* status_ptr(int device);
torch::Tensor status_tensor(int device);

}  // namespace octo
