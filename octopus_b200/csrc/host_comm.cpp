// Host side of the peer-memory collectives: IPC-capable buffers (cudaMalloc'd, wrapped
// as torch tensors), handle export/import, and the fused kernels' entry points.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <string>

#include "comm.h"
#include "tmap.h"

namespace octo {

// A device buffer from cudaMalloc (so it can be exported with cudaIpcGetMemHandle),
// owned by the returned tensor.
torch::Tensor symm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<int>(device));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, static_cast<size_t>(nbytes)));
  C10_CUDA_CHECK(cudaMemset(p, 0, static_cast<size_t>(nbytes)));
  auto opts = torch::dtype(torch::kUInt8).device(torch::kCUDA, static_cast<int>(device));
  return torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

py::bytes ipc_handle(torch::Tensor t) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, t.data_ptr()));
  return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(py::bytes handle, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<int>(device));
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

static std::vector<int64_t> ptr_list(const std::vector<int64_t>& v) {
  TORCH_CHECK(!v.empty() && v.size() <= 8, "1..8 ranks supported");
  return v;
}

// out[i] = sum_r grads_r[off + i], sq += sum out^2
void rs_sum_sq_t(std::vector<int64_t> grad_ptrs, int64_t off, torch::Tensor out, torch::Tensor sq) {
  c10::cuda::CUDAGuard guard(out.get_device());
  auto p = ptr_list(grad_ptrs);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous(), "rs: fp32 out");
  rs_sum_sq(p.data(), static_cast<int>(p.size()), static_cast<size_t>(off), out.numel(), out.data_ptr<float>(),
            sq.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_bcast_t(torch::Tensor p32, torch::Tensor g, torch::Tensor m, torch::Tensor v,
                   std::vector<int64_t> dst_ptrs, int64_t off, double lr, double b1, double b2, double eps,
                   double wd, int64_t step, torch::Tensor sq, double max_norm, double grad_scale) {
  c10::cuda::CUDAGuard guard(p32.get_device());
  auto d = ptr_list(dst_ptrs);
  TORCH_CHECK(p32.numel() % 8 == 0, "adamw_bcast: shard size must be a multiple of 8");
  adamw_bcast(p32.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), d.data(),
              static_cast<int>(d.size()), static_cast<size_t>(off), p32.numel(), lr, b1, b2, eps, wd,
              static_cast<int>(step), sq.data_ptr<float>(), max_norm, grad_scale,
              at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void bcast_bf16_t(torch::Tensor src, std::vector<int64_t> dst_ptrs, int64_t off) {
  c10::cuda::CUDAGuard guard(src.get_device());
  auto d = ptr_list(dst_ptrs);
  TORCH_CHECK(src.numel() % 8 == 0, "bcast: multiple of 8");
  bcast_bf16(reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), d.data(), static_cast<int>(d.size()),
             static_cast<size_t>(off), src.numel(), at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dst[r * n + j] = rank r's bf16 buffer[off + j] (the FSDP per-layer all-gather)
void peer_gather_bf16_t(std::vector<int64_t> ptrs, int64_t off, int64_t n, torch::Tensor dst) {
  c10::cuda::CUDAGuard guard(dst.get_device());
  TORCH_CHECK(dst.scalar_type() == torch::kBFloat16 && dst.is_contiguous(), "peer_gather: bf16 contiguous dst");
  TORCH_CHECK(n % 8 == 0 && off % 8 == 0 && dst.numel() >= n * static_cast<int64_t>(ptrs.size()),
              "peer_gather: n and off multiples of 8, dst holds world * n");
  auto p = ptr_list(ptrs);
  for (auto& x : p) x += off * 2;
  peer_gather_bf16(p.data(), static_cast<int>(p.size()), static_cast<size_t>(n),
                   reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// acc[j] += sum_r rank r's fp32 buffer[off + j] (the FSDP per-layer reduce-scatter)
void peer_rs_acc_t(std::vector<int64_t> ptrs, int64_t off, torch::Tensor acc) {
  c10::cuda::CUDAGuard guard(acc.get_device());
  TORCH_CHECK(acc.scalar_type() == torch::kFloat32 && acc.is_contiguous(), "peer_rs_acc: fp32 contiguous acc");
  TORCH_CHECK(acc.numel() % 4 == 0 && off % 4 == 0, "peer_rs_acc: sizes multiples of 4");
  auto p = ptr_list(ptrs);
  for (auto& x : p) x += off * 4;
  peer_rs_acc(p.data(), static_cast<int>(p.size()), static_cast<size_t>(acc.numel()), acc.data_ptr<float>(),
              at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_barrier_t(std::vector<int64_t> flag_ptrs, int64_t me, int64_t seq, int64_t device, int64_t budget_us) {
  c10::cuda::CUDAGuard guard(static_cast<int>(device));
  auto f = ptr_list(flag_ptrs);
  peer_barrier(f.data(), static_cast<int>(f.size()), static_cast<int>(me), static_cast<int>(seq),
               status_ptr(static_cast<int>(device)), at::cuda::getCurrentCUDAStream().stream(),
               static_cast<unsigned long long>(budget_us > 0 ? budget_us : 0) * 1000ull);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_comm(py::module& m) {
  m.def("symm_alloc", &symm_alloc);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("rs_sum_sq", &rs_sum_sq_t);
  m.def("adamw_bcast", &adamw_bcast_t);
  m.def("bcast_bf16", &bcast_bf16_t);
  m.def("peer_barrier", &peer_barrier_t, py::arg("flag_ptrs"), py::arg("me"), py::arg("seq"), py::arg("device"),
        py::arg("budget_us") = 0);
  m.def("peer_gather_bf16", &peer_gather_bf16_t);
  m.def("peer_rs_acc", &peer_rs_acc_t);
}

}  // namespace octo
