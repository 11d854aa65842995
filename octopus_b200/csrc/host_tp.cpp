// Host side of the tensor-parallel fused kernels: tensor maps over peer shards, slot
// counters in the IPC sync buffers, launch bookkeeping.  Peer pointers come from
// cudaIpcOpenMemHandle (mapped once per buffer by the Python side).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdlib>
#include <vector>

#include "tmap.h"
#include "tp.h"

namespace octo {

static TpSlot make_slot(int64_t sync_local, const std::vector<int64_t>& sync_ptrs, int64_t me, int64_t slot) {
  TORCH_CHECK(!sync_ptrs.empty() && sync_ptrs.size() <= static_cast<size_t>(kMaxTp), "tp: 1..8 ranks");
  TORCH_CHECK(slot >= 0 && slot < kTpSlots, "tp: slot out of range");
  TORCH_CHECK(me >= 0 && me < static_cast<int64_t>(sync_ptrs.size()), "tp: rank out of range");
  TpSlot s{};
  s.tp = static_cast<int>(sync_ptrs.size());
  s.me = static_cast<int>(me);
  int* base = reinterpret_cast<int*>(sync_local);
  s.flags = base + slot * kMaxTp;
  s.done = base + kTpSlots * kMaxTp + slot;
  for (int r = 0; r < s.tp; ++r) s.peer_flags[r] = reinterpret_cast<int*>(sync_ptrs[r]) + slot * kMaxTp;
  return s;
}

static void check_rows_s(int64_t rows_s) {
  TORCH_CHECK(rows_s > 0 && rows_s % 8 == 0 && (rows_s >= 128 ? rows_s % 128 == 0 : 128 % rows_s == 0),
              "tp: rows per rank must be 8, 16, 32, 64 or a multiple of 128 (got ", rows_s, ")");
}

// GEMM launch for C[M, N] = A[M, K] @ W[N, K]^T where A is described by the caller.
static GemmLaunch base_launch(int M, const torch::Tensor& W, int bn_hint) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == torch::kBFloat16 && W.dim() == 2 && W.stride(1) == 1,
              "tp gemm: W must be a bf16 [N, K] row-major CUDA tensor");
  GemmLaunch g{};
  const int N = W.size(0), K = W.size(1);
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0 && M % 8 == 0, "tp gemm: M, N, K multiples of 8");
  const int dev = W.get_device();
  const int sms = num_sms(dev);
  g.bn = pick_bn(M, N, sms, bn_hint);
  g.s.M = M;
  g.s.N = N;
  g.s.K = K;
  g.s.m_tiles = (M + 127) / 128;
  g.s.n_tiles = (N + g.bn - 1) / g.bn;
  g.s.k_blocks = (K + 63) / 64;
  g.s.num_tiles = g.s.m_tiles * g.s.n_tiles;
  g.tb = make_tmap_bf16_2d(W.data_ptr(), K, N, W.stride(0), 64, g.bn);
  g.status = status_ptr(dev);
  g.grid = std::min(g.s.num_tiles, sms);
  g.stream = at::cuda::getCurrentCUDAStream(dev).stream();
  g.alpha = 1.f;
  g.vocab_limit = N;
  g.s.b_prefetch = 0;
  return g;
}

// stage: local bf16 [tp * rows_s, K] staging buffer; work: local int32 counters
// [1 + m_tiles], zero between calls (the kernel's last CTA resets them).
// Split-K for decode-sized tensor-parallel GEMMs (as decode_shape in host_ops.cpp): BN = 256
// tiles split along K to about one tile per SM; returns 1 for none.  Rebuilds the B map.
static int tp_splits(GemmLaunch& g, const torch::Tensor& W) {
  if (g.s.M > 256 || g.s.N < 256) return 1;
  if (const char* e = std::getenv("OCTO_SPLITK"); e != nullptr && e[0] == '0') return 1;
  const int sms = num_sms(W.get_device());
  const int n_tiles = (g.s.N + 255) / 256;
  const int tiles = g.s.m_tiles * n_tiles;
  if (tiles * 4 >= sms * 3) return 1;
  const int splits = nonempty_splits(g.s.k_blocks, std::min(sms / tiles, g.s.k_blocks / 4));
  if (splits < 2) return 1;
  g.bn = 256;
  g.s.n_tiles = n_tiles;
  g.s.k_splits = splits;
  g.s.num_tiles = tiles * splits;
  g.grid = std::min(g.s.num_tiles, sms);
  g.tb = make_tmap_bf16_2d(W.data_ptr(), g.s.K, g.s.N, W.stride(0), 64, 256);
  return splits;
}

static AgLaunch ag_launch(const std::vector<int64_t>& x_ptrs, int64_t rows_s, int64_t ldx, const torch::Tensor& W,
                          int64_t me, int64_t sync_local, const std::vector<int64_t>& sync_ptrs, int64_t slot,
                          int64_t bn_hint, const torch::Tensor& stage, const torch::Tensor& work) {
  check_rows_s(rows_s);
  TORCH_CHECK(x_ptrs.size() == sync_ptrs.size(), "ag_gemm: one shard pointer per rank");
  AgLaunch L{};
  const int tp = static_cast<int>(x_ptrs.size());
  L.g = base_launch(static_cast<int>(rows_s * tp), W, static_cast<int>(bn_hint));
  L.rows_s = static_cast<int>(rows_s);
  L.box_rows = static_cast<int>(std::min<int64_t>(128, rows_s));
  const int K = W.size(1);
  TORCH_CHECK(K % 8 == 0 && ldx % 8 == 0, "ag_gemm: K and the shard row stride must be multiples of 8");
  TORCH_CHECK(stage.scalar_type() == torch::kBFloat16 && stage.is_contiguous() &&
                  stage.numel() >= static_cast<int64_t>(tp) * rows_s * K,
              "ag_gemm: staging buffer too small");
  TORCH_CHECK(work.scalar_type() == torch::kInt32 && work.is_contiguous() && work.numel() >= 1 + L.g.s.m_tiles,
              "ag_gemm: work counters too small");
  auto* st = reinterpret_cast<__nv_bfloat16*>(stage.data_ptr());
  for (int r = 0; r < tp; ++r) {
    L.peer_x[r] = reinterpret_cast<const void*>(x_ptrs[r]);
    if (r == me)
      L.a[r] = make_tmap_bf16_2d(reinterpret_cast<const void*>(x_ptrs[r]), K, rows_s, ldx, 64, L.box_rows);
    else
      L.a[r] = make_tmap_bf16_2d(st + static_cast<size_t>(r) * rows_s * K, K, rows_s, K, 64, L.box_rows);
  }
  L.ldx = static_cast<int>(ldx);
  L.stage = stage.data_ptr();
  L.work = work.data_ptr<int>();
  if (rows_s >= 128) L.g.s.m_shift = static_cast<int>(me * rows_s / 128);  // own rows first: no copy to wait for
  L.slot = make_slot(sync_local, sync_ptrs, me, slot);
  L.peer_grid = L.g.grid;  // identical shapes on every rank -> identical grids
  return L;
}

// C[tp*rows_s, N] (bf16) = AG(x shards)[tp*rows_s, K] @ W[N, K]^T (+ bias)
void ag_gemm_t(std::vector<int64_t> x_ptrs, int64_t rows_s, int64_t ldx, torch::Tensor W, torch::Tensor C,
               c10::optional<torch::Tensor> bias, int64_t me, int64_t sync_local, std::vector<int64_t> sync_ptrs,
               int64_t slot, int64_t bn_hint, torch::Tensor stage, torch::Tensor work) {
  c10::cuda::CUDAGuard guard(W.get_device());
  AgLaunch L = ag_launch(x_ptrs, rows_s, ldx, W, me, sync_local, sync_ptrs, slot, bn_hint, stage, work);
  TORCH_CHECK(C.is_cuda() && C.scalar_type() == torch::kBFloat16 && C.dim() == 2 && C.size(0) == L.g.s.M &&
                  C.size(1) == L.g.s.N && C.stride(1) == 1 && C.stride(0) % 8 == 0,
              "ag_gemm: C must be bf16 [tp*rows_s, N]");
  const void* bp = nullptr;
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->is_contiguous() && bias->numel() == L.g.s.N,
                "ag_gemm: bias bf16 [N]");
    bp = bias->data_ptr();
  }
  const int splits = tp_splits(L.g, W);
  if (splits > 1) {
    auto ws = torch::empty({splits, L.g.s.M, L.g.s.N}, C.options().dtype(torch::kFloat32));
    L.g.epi = kEpiSplitK;
    L.g.C = ws.data_ptr();
    L.peer_grid = L.g.grid;
    ag_gemm_launch(L);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    splitk_finish(ws.data_ptr<float>(), splits, L.g.s.M, L.g.s.N, bp, nullptr, 0, C.data_ptr(), C.stride(0),
                  L.g.stream);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  L.g.epi = kEpiBF16;
  L.g.C = C.data_ptr();
  L.g.ldc = C.stride(0);
  L.g.bias = bp;
  ag_gemm_launch(L);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Partial A[M, K_loc] @ W[N, K_loc]^T stored into the owners' receive buffers; returns
// the grid (the number of signals the owners' reduce must wait for).
std::vector<int64_t> gemm_rs_t(torch::Tensor A, torch::Tensor W, std::vector<int64_t> recv_ptrs, int64_t recv_elems,
                               int64_t me, int64_t sync_local, std::vector<int64_t> sync_ptrs, int64_t slot,
                               int64_t bn_hint) {
  c10::cuda::CUDAGuard guard(A.get_device());
  TORCH_CHECK(A.is_cuda() && A.scalar_type() == torch::kBFloat16 && A.dim() == 2 && A.stride(1) == 1,
              "gemm_rs: A bf16 [M, K] row-major");
  const int tp = static_cast<int>(recv_ptrs.size());
  TORCH_CHECK(tp == static_cast<int>(sync_ptrs.size()), "gemm_rs: one receive buffer per rank");
  const int M = A.size(0);
  TORCH_CHECK(M % tp == 0, "gemm_rs: rows must split evenly over ranks");
  RsLaunch L{};
  L.g = base_launch(M, W, static_cast<int>(bn_hint));
  TORCH_CHECK(A.size(1) == L.g.s.K, "gemm_rs: K mismatch");
  L.g.ta = make_tmap_bf16_2d(A.data_ptr(), L.g.s.K, M, A.stride(0), 64, 128);
  for (int r = 0; r < tp; ++r) L.recv[r] = reinterpret_cast<void*>(recv_ptrs[r]);
  L.ldc = L.g.s.N;
  L.rows_s = M / tp;
  L.slot = make_slot(sync_local, sync_ptrs, me, slot);
  // no split-K here: every split's partial would cross NVLink (the owner sums splits x tp slices)
  const int splits = 1;
  TORCH_CHECK(static_cast<int64_t>(splits) * M * L.g.s.N <= recv_elems,
              "gemm_rs: receive buffers too small for ", splits, " split partials");
  gemm_rs_launch(L);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {L.g.grid, splits};
}

// h[rows_s, N] += sum_r recv[r]; x = rmsnorm(h) * w (if w given)
void tp_reduce_t(torch::Tensor recv, int64_t splits, torch::Tensor h, c10::optional<torch::Tensor> w,
                 c10::optional<torch::Tensor> x, double eps, bool plus_one, int64_t me, int64_t sync_local,
                 std::vector<int64_t> sync_ptrs, int64_t slot, int64_t peer_grid) {
  c10::cuda::CUDAGuard guard(h.get_device());
  const int tp = static_cast<int>(sync_ptrs.size());
  TORCH_CHECK(h.scalar_type() == torch::kBFloat16 && h.dim() == 2 && h.stride(1) == 1 && h.stride(0) % 8 == 0,
              "tp_reduce: h bf16 [rows, N]");
  const int rows_s = h.size(0), N = h.size(1);
  TORCH_CHECK(N % 8 == 0, "tp_reduce: N % 8 == 0");
  const int parts = static_cast<int>(splits) * tp;
  TORCH_CHECK(recv.scalar_type() == torch::kBFloat16 && recv.is_contiguous() &&
                  recv.numel() >= static_cast<int64_t>(parts) * rows_s * N,
              "tp_reduce: recv bf16 [splits * tp, rows, N]");
  const void* wp = nullptr;
  void* xp = nullptr;
  int ldx = 0;
  if (w.has_value() && w->defined()) {
    TORCH_CHECK(x.has_value() && x->defined(), "tp_reduce: norm output required with a norm weight");
    TORCH_CHECK(w->numel() == N && x->size(0) == rows_s && x->size(1) == N && x->stride(1) == 1 &&
                    x->stride(0) % 8 == 0,
                "tp_reduce: norm shapes");
    wp = w->data_ptr();
    xp = x->data_ptr();
    ldx = x->stride(0);
  }
  TpSlot s = make_slot(sync_local, sync_ptrs, me, slot);
  tp_reduce(recv.data_ptr(), parts, h.data_ptr(), h.stride(0), N, rows_s, wp, xp, ldx, static_cast<float>(eps),
            plus_one ? 1 : 0, s, static_cast<int>(peer_grid), status_ptr(h.get_device()),
            at::cuda::getCurrentCUDAStream(h.get_device()).stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Vocab-parallel sampling head: AG(final-normed shards) @ W_shard^T with the sampling
// epilogue (global columns col_base + j), local combine, exchange, merge.
std::vector<torch::Tensor> tp_sample_head_t(std::vector<int64_t> x_ptrs, int64_t rows_s, int64_t ldx, torch::Tensor W,
                                            double alpha, int64_t seed, torch::Tensor row_stream, int64_t vocab_limit,
                                            int64_t col_base, int64_t me, int64_t sync_local,
                                            std::vector<int64_t> sync_ptrs, int64_t slot_ag, int64_t slot_smp,
                                            std::vector<int64_t> xch_ptrs, torch::Tensor xch_local,
                                            torch::Tensor stage, torch::Tensor work) {
  c10::cuda::CUDAGuard guard(W.get_device());
  AgLaunch L = ag_launch(x_ptrs, rows_s, ldx, W, me, sync_local, sync_ptrs, slot_ag, 0, stage, work);
  const int M = L.g.s.M;
  TORCH_CHECK(row_stream.scalar_type() == torch::kInt64 && row_stream.is_contiguous() && row_stream.numel() == M,
              "tp_sample_head: one stream id per row");
  TORCH_CHECK(xch_ptrs.size() == sync_ptrs.size(), "tp_sample_head: one exchange buffer per rank");
  TORCH_CHECK(xch_local.numel() * xch_local.element_size() >= static_cast<int64_t>(xch_ptrs.size()) * M * 16,
              "tp_sample_head: exchange buffer too small");
  auto f32 = torch::dtype(torch::kFloat32).device(W.device());
  auto part = torch::empty({M, L.g.s.n_tiles, 4}, f32);
  auto tokens = torch::empty({M}, torch::dtype(torch::kInt64).device(W.device()));
  auto logprob = torch::empty({M}, f32);
  L.g.epi = kEpiSample;
  L.g.alpha = static_cast<float>(alpha);
  L.g.partial = part.data_ptr<float>();
  L.g.seed = static_cast<uint64_t>(seed);
  L.g.row_offset = row_stream.data_ptr<int64_t>();
  L.g.vocab_limit = static_cast<int>(vocab_limit);
  L.g.col_base = static_cast<int>(col_base);
  ag_gemm_launch(L);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  TpSlot s = make_slot(sync_local, sync_ptrs, me, slot_smp);
  std::vector<void*> xp(xch_ptrs.size());
  for (size_t r = 0; r < xch_ptrs.size(); ++r) xp[r] = reinterpret_cast<void*>(xch_ptrs[r]);
  const int g1 = tp_sample_local(part.data_ptr<float>(), M, L.g.s.n_tiles, xp.data(), s, L.g.stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  tp_sample_final(xch_local.data_ptr(), M, L.g.seed, row_stream.data_ptr<int64_t>(), tokens.data_ptr<int64_t>(),
                  logprob.data_ptr<float>(), s, g1, L.g.status, L.g.stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {tokens, logprob};
}

void tp_barrier_t(int64_t me, int64_t sync_local, std::vector<int64_t> sync_ptrs, int64_t slot, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<int>(device));
  TpSlot s = make_slot(sync_local, sync_ptrs, me, slot);
  tp_barrier(s, status_ptr(static_cast<int>(device)),
             at::cuda::getCurrentCUDAStream(static_cast<int>(device)).stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// segs: int64 [nseg, 6] = (src, dst, lds, ldd, rows | cols << 32, first) on the device
void reshard_copy_t(torch::Tensor segs, int64_t total_chunks) {
  c10::cuda::CUDAGuard guard(segs.get_device());
  static_assert(sizeof(ReshardSeg) == 48, "ReshardSeg layout");
  TORCH_CHECK(segs.scalar_type() == torch::kInt64 && segs.is_contiguous() && segs.dim() == 2 && segs.size(1) == 6,
              "reshard: segs int64 [n, 6]");
  reshard_copy(reinterpret_cast<const ReshardSeg*>(segs.data_ptr()), segs.size(0), total_chunks,
               at::cuda::getCurrentCUDAStream(segs.get_device()).stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t tp_sync_bytes() { return kTpSyncBytes; }

void register_tp(py::module& m) {
  m.def("ag_gemm", &ag_gemm_t);
  m.def("gemm_rs", &gemm_rs_t);
  m.def("tp_reduce", &tp_reduce_t);
  m.def("tp_sample_head", &tp_sample_head_t);
  m.def("tp_barrier", &tp_barrier_t);
  m.def("reshard_copy", &reshard_copy_t);
  m.def("tp_sync_bytes", &tp_sync_bytes);
}

}  // namespace octo
