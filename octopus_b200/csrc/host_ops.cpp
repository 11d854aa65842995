// Torch-facing host glue of the octopus_b200 extension (compiled by g++, no device code).
// Every entry point checks devices, dtypes, shapes and strides, then calls a plain
// launcher from the CUDA translation units on the current stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>
#include <mutex>
#include <vector>

#include "attention.h"
#include "decode_persistent.h"
#include "decode_shared.h"
#include "elementwise.h"
#include "octo_api.h"
#include "tmap.h"

namespace octo {

static std::mutex g_status_mu;
static std::vector<torch::Tensor> g_status(64);

torch::Tensor status_tensor(int device) {
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_status[device].defined()) {
    g_status[device] = torch::zeros({kStatusWordsHost}, torch::dtype(torch::kInt32).device(torch::kCUDA, device));
  }
  return g_status[device];
}
int* status_ptr(int device) { return status_tensor(device).data_ptr<int>(); }

static cudaStream_t cur_stream(const torch::Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.get_device()).stream();
}

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == torch::kBFloat16, #x " must be bf16")
#define CHECK_F32(x) TORCH_CHECK((x).scalar_type() == torch::kFloat32, #x " must be fp32")
#define CHECK_I32(x) TORCH_CHECK((x).scalar_type() == torch::kInt32, #x " must be int32")
#define CHECK_I64(x) TORCH_CHECK((x).scalar_type() == torch::kInt64, #x " must be int64")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define BF(x) reinterpret_cast<__nv_bfloat16*>((x).data_ptr())
#define CBF(x) reinterpret_cast<const __nv_bfloat16*>((x).data_ptr())

// Shared-prefix decode: segment tables from ops.decode.plan_shared (all int32, device).
void attn_decode_shared_t(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor kv_indices,
                          torch::Tensor kv_len, torch::Tensor seg_rows, torch::Tensor seg_slot, torch::Tensor seg_start,
                          torch::Tensor seg_len, torch::Tensor seg_off, torch::Tensor items, torch::Tensor n_items,
                          torch::Tensor row_nslot, torch::Tensor o, torch::Tensor part_o, torch::Tensor part_lse,
                          int64_t Hq, int64_t Hkv, int64_t max_slots, int64_t chunk, double scale, bool use_tc,
                          c10::optional<torch::Tensor> trace) {
  c10::cuda::CUDAGuard guard(q.get_device());
  for (auto* t : {&kv_indices, &kv_len, &seg_rows, &seg_slot, &seg_start, &seg_len, &seg_off, &items, &n_items,
                  &row_nslot}) {
    TORCH_CHECK(t->scalar_type() == torch::kInt32 && t->is_contiguous() && t->is_cuda(),
                "decode_shared: int32 contiguous CUDA tables");
  }
  CHECK_BF16(q);
  CHECK_BF16(kc);
  CHECK_BF16(vc);
  CHECK_BF16(o);
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= 16, "decode_shared: GQA group must be <= 16");
  TORCH_CHECK(q.stride(1) == 1 && o.stride(1) == 1 && kc.is_contiguous() && vc.is_contiguous(), "decode: layout");
  TORCH_CHECK(kc.size(-1) == Hkv * 128, "decode_shared: head_dim 128 only");
  TORCH_CHECK(chunk % 64 == 0 && chunk > 0, "decode_shared: chunk must be a multiple of 64");
  TORCH_CHECK(n_items.numel() >= 2, "decode_shared: n_items holds [work items, keys per item]");
  DecodeSharedParams p{};
  p.q = CBF(q);
  p.k_cache = CBF(kc);
  p.v_cache = CBF(vc);
  p.o = BF(o);
  p.kv_indices = kv_indices.data_ptr<int32_t>();
  p.kv_len = kv_len.data_ptr<int32_t>();
  p.seg_rows = seg_rows.data_ptr<int32_t>();
  p.seg_slot = seg_slot.data_ptr<int32_t>();
  p.seg_start = seg_start.data_ptr<int32_t>();
  p.seg_len = seg_len.data_ptr<int32_t>();
  p.seg_off = seg_off.data_ptr<int32_t>();
  p.items = items.data_ptr<int32_t>();
  p.n_items = n_items.data_ptr<int32_t>();
  p.row_nslot = row_nslot.data_ptr<int32_t>();
  p.ldq = q.stride(0);
  p.ldo = o.stride(0);
  p.B = q.size(0);
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.max_slots = static_cast<int>(max_slots);
  p.chunk = static_cast<int>(chunk);
  p.scale = static_cast<float>(scale);
  p.n_slots = kc.numel() / (Hkv * 128);
  TORCH_CHECK(row_nslot.numel() >= p.B, "decode_shared: row_nslot too small");
  TORCH_CHECK(part_o.numel() >= static_cast<int64_t>(p.B) * Hq * max_slots * 128 &&
                  part_lse.numel() >= static_cast<int64_t>(p.B) * Hq * max_slots,
              "decode_shared: scratch too small");
  p.part_o = part_o.data_ptr<float>();
  p.part_lse = part_lse.data_ptr<float>();
  p.trace = (trace.has_value() && trace->defined()) ? reinterpret_cast<unsigned long long*>(trace->data_ptr())
                                                      : nullptr;
  if (p.B == 0) return;
  if (use_tc) {
    DecodeSharedMaps maps;
    maps.k = make_tmap_bf16_2d(kc.data_ptr(), Hkv * 128, kc.size(0), Hkv * 128, 64, 64);
    maps.v = make_tmap_bf16_2d(vc.data_ptr(), Hkv * 128, vc.size(0), Hkv * 128, 64, 64);
    decode_shared_tc_launch(p, maps, num_sms(q.get_device()), status_ptr(q.get_device()), cur_stream(q));
  } else {
    decode_shared_launch(p, 2 * num_sms(q.get_device()), status_ptr(q.get_device()), cur_stream(q));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ GEMM
// GEMMs launched while set are programmatic dependents of the preceding kernel (decode
// graphs of the engine): their prologue and weight prefetch overlap its tail.
static bool g_pdl = false;
void set_pdl(bool on) { g_pdl = on; }


int pick_bn(int M, int N, int sms, int hint) {
  if (hint == 64 || hint == 128 || hint == 256) return hint;
  const int mt = (M + 127) / 128;
  auto tiles = [&](int bn) { return mt * ((N + bn - 1) / bn); };
  if (N >= 256 && tiles(256) >= sms) return 256;
  if (N >= 128 && tiles(128) >= (sms * 3) / 4) return 128;
  return 64;
}

static GemmLaunch make_launch(const torch::Tensor& A, bool a_mn, const torch::Tensor& B, bool b_mn, int bn_hint) {
  CHECK_CUDA(A);
  CHECK_CUDA(B);
  CHECK_BF16(A);
  CHECK_BF16(B);
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "gemm: 2D operands");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm: unit inner stride required");
  GemmLaunch g{};
  const int M = a_mn ? A.size(1) : A.size(0);
  const int K = a_mn ? A.size(0) : A.size(1);
  const int N = b_mn ? B.size(1) : B.size(0);
  const int Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "gemm: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0 && M % 8 == 0, "gemm: M, N, K must be multiples of 8 (got ", M, ", ", N,
              ", ", K, ")");
  const int device = A.get_device();
  const int sms = num_sms(device);
  const int BN = pick_bn(M, N, sms, bn_hint);
  g.bn = BN;
  g.mt = 1;
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.s.M = M;
  g.s.N = N;
  g.s.K = K;
  g.s.m_tiles = (M + 127) / 128;
  g.s.n_tiles = (N + BN - 1) / BN;
  g.s.k_blocks = (K + 63) / 64;
  g.s.num_tiles = g.s.m_tiles * g.s.n_tiles;
  g.status = status_ptr(device);
  g.stream = cur_stream(A);
  TORCH_CHECK(K > 0 || M == 0 || N == 0, "gemm: K must be positive");
  if (M == 0 || N == 0) return g;  // empty product: callers return before launching; no tensor maps
  g.ta = a_mn ? make_tmap_bf16_2d(A.data_ptr(), M, K, A.stride(0), 64, 64)
              : make_tmap_bf16_2d(A.data_ptr(), K, M, A.stride(0), 64, 128);
  g.tb = b_mn ? make_tmap_bf16_2d(B.data_ptr(), N, K, B.stride(0), 64, 64)
              : make_tmap_bf16_2d(B.data_ptr(), K, N, B.stride(0), 64, BN);
  g.grid = std::min(g.s.num_tiles, sms);
  g.alpha = 1.f;
  g.vocab_limit = N;
  g.s.pdl = g_pdl ? 1 : 0;
  g.s.b_prefetch = 0;  // L2 prefetch of B only in PDL launches (see gemm_sm100.cuh)
  return g;
}

// Decode-sized forward GEMMs (M <= 256, K-major operands, bf16 out, alpha 1): 256-wide N
// tiles.  When those tiles cannot fill the GPU, K is split until ~one tile per SM (keeping
// >= 4 K blocks per split).  When they can and M > 128, both 128-row M-blocks go to one CTA
// (MT = 2) so each weight tile is loaded once.  Rebuilds the launch's B map for BN = 256 and
// returns the split count (1 for none).  OCTO_SPLITK=0 switches split-K off; OCTO_GEMM_MT=1
// / =2 force one / two M-tiles per CTA.
static int decode_shape(GemmLaunch& g, int64_t bn_hint, int device, const torch::Tensor& B) {
  if (bn_hint != 0 || g.a_mn || g.b_mn || g.alpha != 1.f || g.s.M > 256 || g.s.N < 256) return 1;
  const char* e_sk = std::getenv("OCTO_SPLITK");
  const char* e_mt = std::getenv("OCTO_GEMM_MT");
  const bool allow_split = !(e_sk != nullptr && e_sk[0] == '0');
  const int force_mt = e_mt != nullptr ? std::atoi(e_mt) : 0;
  const int sms = num_sms(device);
  const int n_tiles = (g.s.N + 255) / 256;
  const int m1 = (g.s.M + 127) / 128, m2 = (g.s.M + 255) / 256;
  int mt = 1;
  if (g.s.M > 128 && force_mt != 1 && (force_mt == 2 || m2 * n_tiles * 4 >= sms * 3)) mt = 2;
  const int m_tiles = mt == 2 ? m2 : m1;
  const int tiles = m_tiles * n_tiles;
  int splits = 1;
  if (allow_split && tiles * 4 < sms * 3)
    splits = nonempty_splits(g.s.k_blocks, std::max(1, std::min(sms / tiles, g.s.k_blocks / 4)));
  if (mt == 1 && splits < 2) return 1;  // the default launch
  g.mt = mt;
  g.bn = 256;
  g.s.m_tiles = m_tiles;
  g.s.n_tiles = n_tiles;
  g.s.k_splits = splits > 1 ? splits : 0;
  g.s.num_tiles = tiles * splits;
  g.grid = std::min(g.s.num_tiles, sms);
  g.tb = make_tmap_bf16_2d(B.data_ptr(), g.s.K, g.s.N, B.stride(0), 64, 256);
  return splits;
}

// C[M,N] = alpha * A_log[M,K] @ B_log[N,K]^T (+ bias) (+ residual)   or   C += ... (fp32)
//   a_mn false: A is [M, K];  true: A is [K, M].   b_mn false: B is [N, K];  true: B is [K, N].
void gemm_out(torch::Tensor A, bool a_mn, torch::Tensor B, bool b_mn, torch::Tensor C, double alpha,
              c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> bias, bool accumulate,
              int64_t bn_hint) {
  c10::cuda::CUDAGuard guard(A.get_device());
  GemmLaunch g = make_launch(A, a_mn, B, b_mn, static_cast<int>(bn_hint));
  CHECK_CUDA(C);
  TORCH_CHECK(C.dim() == 2 && C.size(0) == g.s.M && C.size(1) == g.s.N && C.stride(1) == 1, "gemm: bad output");
  if (g.s.M == 0 || g.s.N == 0) return;
  g.alpha = static_cast<float>(alpha);
  g.C = C.data_ptr();
  g.ldc = C.stride(0);
  if (C.scalar_type() == torch::kBFloat16) {
    TORCH_CHECK(!accumulate, "gemm: accumulate requires an fp32 output");
    TORCH_CHECK(C.stride(0) % 8 == 0, "gemm: output row stride must be a multiple of 8");
    const int splits = decode_shape(g, bn_hint, A.get_device(), B);
    if (splits > 1) {
      // decode-sized M: wide N tiles (each CTA re-reads fewer activation bytes) split along K so
      // every SM streams weights; fp32 partials are summed with bias / residual by splitk_finish
      auto ws = torch::empty({splits, g.s.M, g.s.N}, C.options().dtype(torch::kFloat32));
      g.epi = kEpiSplitK;
      g.C = ws.data_ptr();
      gemm_launch(g);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      const void* rp = nullptr;
      int ldr = 0;
      if (residual.has_value() && residual->defined()) {
        CHECK_BF16(*residual);
        TORCH_CHECK(residual->size(0) == g.s.M && residual->size(1) == g.s.N && residual->stride(1) == 1 &&
                        residual->stride(0) % 8 == 0,
                    "gemm: bad residual");
        rp = residual->data_ptr();
        ldr = residual->stride(0);
      }
      const void* bp = nullptr;
      if (bias.has_value() && bias->defined()) {
        CHECK_BF16(*bias);
        TORCH_CHECK(bias->is_contiguous() && bias->numel() == g.s.N, "gemm: bias must have N elements");
        bp = bias->data_ptr();
      }
      splitk_finish(ws.data_ptr<float>(), splits, g.s.M, g.s.N, bp, rp, ldr, C.data_ptr(), C.stride(0), g.stream);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      return;
    }
    g.epi = kEpiBF16;
    if (residual.has_value() && residual->defined()) {
      const auto& R = *residual;
      CHECK_BF16(R);
      TORCH_CHECK(R.dim() == 2 && R.size(0) == g.s.M && R.size(1) == g.s.N && R.stride(1) == 1 &&
                      R.stride(0) % 8 == 0,
                  "gemm: bad residual");
      g.R = R.data_ptr();
      g.ldr = R.stride(0);
    }
    if (bias.has_value() && bias->defined()) {
      const auto& b = *bias;
      CHECK_BF16(b);
      CHECK_CONTIG(b);
      TORCH_CHECK(b.numel() == g.s.N, "gemm: bias must have N elements");
      g.bias = b.data_ptr();
    }
  } else {
    CHECK_F32(C);
    TORCH_CHECK(C.stride(0) % 4 == 0, "gemm: fp32 output row stride must be a multiple of 4");
    TORCH_CHECK(!(residual.has_value() && residual->defined()) && !(bias.has_value() && bias->defined()),
                "gemm: residual/bias only with bf16 output");
    g.epi = kEpiF32;
    g.accumulate = accumulate ? 1 : 0;
  }
  gemm_launch(g);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Decode projection fused with what follows it in the layer (engine decode graphs):
//   (x, h) = (A W^T + bias + residual, RMSNorm(x) * norm_w)
// Split-K launches (every decode-sized o / down projection) finish in one kernel that also
// normalises; other shapes run the GEMM and the norm separately.
// Gated MLP projection fused with its activation: act[M, F] = silu(A W_gate^T) * (A W_up^T),
// W = [W_gate; W_up] ([2F, K], the checkpoint's gate_up layout).  Each tile pairs 128 gate
// rows with the matching 128 up rows (two TMA boxes into one 256-row B stage), so the
// epilogue holds both halves of its 128 output columns; no [M, 2F] intermediate is written.
// F must be a multiple of 128 (callers fall back to GEMM + swiglu otherwise).
torch::Tensor gemm_swiglu_t(torch::Tensor A, torch::Tensor W) {
  c10::cuda::CUDAGuard guard(A.get_device());
  TORCH_CHECK(W.dim() == 2 && W.size(0) % 256 == 0, "gemm_swiglu: W rows must be 2F with F a multiple of 128");
  GemmLaunch g = make_launch(A, false, W, false, 256);
  const int M = g.s.M, F = g.s.N / 2;
  auto out = torch::empty({M, F}, A.options());
  if (M == 0) return out;
  const int sms = num_sms(A.get_device());
  g.bn = 256;
  g.s.N = F;
  g.s.n_tiles = F / 128;
  g.s.b_pair = F;
  g.s.k_splits = 0;
  g.tb = make_tmap_bf16_2d(W.data_ptr(), g.s.K, 2 * static_cast<int64_t>(F), W.stride(0), 64, 128);
  // decode-sized M (129..256 rows): both 128-row M-blocks in one CTA when the tiles fill the GPU
  g.mt = (M > 128 && M <= 256 && g.s.n_tiles * 4 >= sms * 3) ? 2 : 1;
  g.s.m_tiles = g.mt == 2 ? 1 : (M + 127) / 128;
  g.s.num_tiles = g.s.m_tiles * g.s.n_tiles;
  g.grid = std::min(g.s.num_tiles, sms);
  g.epi = kEpiSwiGLU;
  g.C = out.data_ptr();
  g.ldc = F;
  gemm_launch(g);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Training QKV projection with the rotary embedding in the GEMM epilogue:
//   out = rope(A W^T + bias) on the Hq + Hkv q / k heads (v heads unrotated), head dim 64 or 128.
// One N tile per head, so each epilogue thread holds both rotary halves of its row's head.
torch::Tensor gemm_rope_t(torch::Tensor A, torch::Tensor W, c10::optional<torch::Tensor> bias, torch::Tensor pos,
                          double theta, int64_t Hq, int64_t Hkv, int64_t D) {
  c10::cuda::CUDAGuard guard(A.get_device());
  TORCH_CHECK(D == 64 || D == 128, "gemm_rope: head_dim 64 or 128");
  GemmLaunch g = make_launch(A, false, W, false, static_cast<int>(D));
  const int M = g.s.M, N = g.s.N;
  TORCH_CHECK(N == (Hq + 2 * Hkv) * D, "gemm_rope: W rows must be (Hq + 2 Hkv) * D");
  CHECK_I32(pos);
  CHECK_CONTIG(pos);
  TORCH_CHECK(pos.numel() >= M, "gemm_rope: one position per row");
  auto out = torch::empty({M, N}, A.options());
  if (M == 0) return out;
  if (bias.has_value() && bias->defined()) {
    CHECK_BF16(*bias);
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == N, "gemm_rope: bias must have N elements");
    g.bias = bias->data_ptr();
  }
  g.epi = kEpiQKVRope;
  g.C = out.data_ptr();
  g.ldc = N;
  g.pos = pos.data_ptr<int32_t>();
  g.rope_log2_theta = log2f(static_cast<float>(theta));
  g.rope_heads = static_cast<int>(Hq + Hkv);
  gemm_launch(g);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

std::vector<torch::Tensor> gemm_res_norm_t(torch::Tensor A, torch::Tensor W, torch::Tensor residual,
                                           torch::Tensor norm_w, double eps, bool plus_one,
                                           c10::optional<torch::Tensor> bias) {
  c10::cuda::CUDAGuard guard(A.get_device());
  GemmLaunch g = make_launch(A, false, W, false, 0);
  const int M = g.s.M, N = g.s.N;
  CHECK_BF16(residual);
  CHECK_BF16(norm_w);
  CHECK_CONTIG(norm_w);
  TORCH_CHECK(residual.dim() == 2 && residual.size(0) == M && residual.size(1) == N && residual.stride(1) == 1 &&
                  residual.stride(0) % 8 == 0,
              "gemm_res_norm: bad residual");
  TORCH_CHECK(norm_w.numel() == N && N % 8 == 0 && N / 8 <= 1024, "gemm_res_norm: norm width");
  const void* bp = nullptr;
  if (bias.has_value() && bias->defined()) {
    CHECK_BF16(*bias);
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == N, "gemm_res_norm: bias must have N elements");
    bp = bias->data_ptr();
  }
  auto x = torch::empty({M, N}, A.options());
  auto h = torch::empty({M, N}, A.options());
  if (M == 0) return {x, h};
  const int splits = decode_shape(g, 0, A.get_device(), W);
  if (splits > 1) {
    auto ws = torch::empty({splits, M, N}, A.options().dtype(torch::kFloat32));
    g.epi = kEpiSplitK;
    g.C = ws.data_ptr();
    gemm_launch(g);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    splitk_finish_norm(ws.data_ptr<float>(), splits, M, N, static_cast<const __nv_bfloat16*>(bp), CBF(residual),
                       residual.stride(0), BF(x), N, CBF(norm_w), static_cast<float>(eps), plus_one, BF(h), N,
                       g.stream);
  } else {
    gemm_out(A, false, W, false, x, 1.0, residual, bias, false, 0);
    rmsnorm_fwd(CBF(x), N, CBF(norm_w), BF(h), N, nullptr, M, N, static_cast<float>(eps), plus_one ? 1 : 0,
                g.stream);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {x, h};
}

// Decode qkv projection fused with the rotary embedding and the KV-cache write:
//   qkv = A W^T + bias;  rotate the q and k heads at positions pos;  k, v rows -> kc / vc at
//   slots (negative: not written);  returns the q rows [M, Hq * D].
torch::Tensor gemm_qkv_rope_t(torch::Tensor A, torch::Tensor W, c10::optional<torch::Tensor> bias, torch::Tensor pos,
                              double theta, int64_t Hq, int64_t Hkv, int64_t D, torch::Tensor slots, torch::Tensor kc,
                              torch::Tensor vc) {
  c10::cuda::CUDAGuard guard(A.get_device());
  GemmLaunch g = make_launch(A, false, W, false, 0);
  const int M = g.s.M, N = g.s.N;
  TORCH_CHECK(N == (Hq + 2 * Hkv) * D && D % 16 == 0, "gemm_qkv_rope: W rows must be (Hq + 2 Hkv) * D");
  CHECK_I32(pos);
  CHECK_CONTIG(pos);
  CHECK_I64(slots);
  CHECK_CONTIG(slots);
  CHECK_CONTIG(kc);
  CHECK_CONTIG(vc);
  CHECK_BF16(kc);
  CHECK_BF16(vc);
  TORCH_CHECK(pos.numel() >= M && slots.numel() >= M, "gemm_qkv_rope: one position and slot per row");
  TORCH_CHECK(kc.size(-1) == Hkv * D && vc.size(-1) == Hkv * D, "gemm_qkv_rope: cache width");
  const void* bp = nullptr;
  if (bias.has_value() && bias->defined()) {
    CHECK_BF16(*bias);
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == N, "gemm_qkv_rope: bias must have N elements");
    bp = bias->data_ptr();
  }
  if (M == 0) return torch::empty({0, Hq * D}, A.options());
  const int splits = decode_shape(g, 0, A.get_device(), W);
  if (splits > 1) {
    auto ws = torch::empty({splits, M, N}, A.options().dtype(torch::kFloat32));
    g.epi = kEpiSplitK;
    g.C = ws.data_ptr();
    gemm_launch(g);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    auto q = torch::empty({M, Hq * D}, A.options());
    splitk_finish_qkv(ws.data_ptr<float>(), splits, M, Hq, Hkv, D, static_cast<const __nv_bfloat16*>(bp),
                      pos.data_ptr<int32_t>(), static_cast<float>(theta), BF(q), Hq * D, slots.data_ptr<int64_t>(),
                      BF(kc), BF(vc), kc.numel() / (Hkv * D), g.status, g.stream);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return q;
  }
  auto qkv = torch::empty({M, N}, A.options());
  gemm_out(A, false, W, false, qkv, 1.0, c10::nullopt, bias, false, 0);
  rope_apply(BF(qkv), N, pos.data_ptr<int32_t>(), M, Hq, Hkv, D, static_cast<float>(theta), false, g.stream);
  kv_write(CBF(qkv), N, Hq, Hkv, D, slots.data_ptr<int64_t>(), BF(kc), BF(vc), M, kc.numel() / (Hkv * D), g.status, g.stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return qkv.narrow(1, 0, Hq * D);
}

// Chunked logprob head forward: per row (log p(label), entropy, lse) of softmax(alpha * h W^T)
// without materialising logits.  labels < 0 mark unscored rows (logp = 0).
std::vector<torch::Tensor> head_fwd(torch::Tensor h, torch::Tensor W, torch::Tensor labels, double alpha,
                                    int64_t vocab_limit) {
  c10::cuda::CUDAGuard guard(h.get_device());
  CHECK_I32(labels);
  CHECK_CONTIG(labels);
  GemmLaunch g = make_launch(h, false, W, false, 256);
  TORCH_CHECK(labels.numel() == g.s.M, "head_fwd: one label per row");
  auto f32 = torch::dtype(torch::kFloat32).device(h.device());
  auto part = torch::empty({g.s.M, g.s.n_tiles, 4}, f32);
  auto logp = torch::empty({g.s.M}, f32), ent = torch::empty({g.s.M}, f32), lse = torch::empty({g.s.M}, f32);
  if (g.s.M == 0) return {logp, ent, lse};
  g.epi = kEpiHeadLse;
  g.alpha = static_cast<float>(alpha);
  g.labels = labels.data_ptr<int32_t>();
  g.partial = part.data_ptr<float>();
  g.vocab_limit = vocab_limit > 0 ? static_cast<int>(vocab_limit) : g.s.N;
  gemm_launch(g);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  head_combine(part.data_ptr<float>(), g.s.M, g.s.n_tiles, labels.data_ptr<int32_t>(), logp.data_ptr<float>(),
               ent.data_ptr<float>(), lse.data_ptr<float>(), g.stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {logp, ent, lse};
}

// d loss / d logits of the head (bf16 [M, N]) recomputed from (lse, entropy).
void head_grad_logits(torch::Tensor h, torch::Tensor W, torch::Tensor labels, torch::Tensor lse, torch::Tensor ent,
                      torch::Tensor g_lp, torch::Tensor g_ent, torch::Tensor dz, double alpha, int64_t vocab_limit) {
  c10::cuda::CUDAGuard guard(h.get_device());
  GemmLaunch g = make_launch(h, false, W, false, 256);
  for (auto* t : {&lse, &ent, &g_lp, &g_ent}) {
    CHECK_F32(*t);
    CHECK_CONTIG(*t);
    TORCH_CHECK(t->numel() == g.s.M, "head_grad: per-row vectors");
  }
  CHECK_I32(labels);
  CHECK_BF16(dz);
  TORCH_CHECK(dz.size(0) == g.s.M && dz.size(1) == g.s.N && dz.stride(1) == 1 && dz.stride(0) % 8 == 0,
              "head_grad: bad dz");
  if (g.s.M == 0) return;
  g.epi = kEpiHeadGrad;
  g.C = dz.data_ptr();
  g.ldc = dz.stride(0);
  g.labels = labels.data_ptr<int32_t>();
  g.lse = lse.data_ptr<float>();
  g.ent = ent.data_ptr<float>();
  g.g_lp = g_lp.data_ptr<float>();
  g.g_ent = g_ent.data_ptr<float>();
  g.alpha = static_cast<float>(alpha);
  g.vocab_limit = vocab_limit > 0 ? static_cast<int>(vocab_limit) : g.s.N;
  gemm_launch(g);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fused sampling head: token ~ softmax(alpha * h W^T) by Gumbel-max, plus its logprob.
std::vector<torch::Tensor> sample_head(torch::Tensor h, torch::Tensor W, double alpha, int64_t seed,
                                       c10::optional<torch::Tensor> row_stream, int64_t vocab_limit) {
  c10::cuda::CUDAGuard guard(h.get_device());
  GemmLaunch g = make_launch(h, false, W, false, 0);
  auto f32 = torch::dtype(torch::kFloat32).device(h.device());
  auto part = torch::empty({g.s.M, g.s.n_tiles, 4}, f32);
  auto tokens = torch::empty({g.s.M}, torch::dtype(torch::kInt64).device(h.device()));
  auto logprob = torch::empty({g.s.M}, f32);
  if (g.s.M == 0) return {tokens, logprob};
  const int64_t* rs = nullptr;
  if (row_stream.has_value() && row_stream->defined()) {
    CHECK_I64(*row_stream);
    CHECK_CONTIG(*row_stream);
    TORCH_CHECK(row_stream->numel() == g.s.M, "sample_head: one stream id per row");
    rs = row_stream->data_ptr<int64_t>();
  }
  g.epi = kEpiSample;
  g.alpha = static_cast<float>(alpha);
  g.partial = part.data_ptr<float>();
  g.seed = static_cast<uint64_t>(seed);
  g.row_offset = rs;
  g.vocab_limit = vocab_limit > 0 ? static_cast<int>(vocab_limit) : g.s.N;
  gemm_launch(g);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  sample_combine(part.data_ptr<float>(), g.s.M, g.s.n_tiles, g.seed, rs, tokens.data_ptr<int64_t>(),
                 logprob.data_ptr<float>(), g.stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {tokens, logprob};
}

// ------------------------------------------------------------------ elementwise
std::vector<torch::Tensor> rmsnorm_fwd_t(torch::Tensor x, torch::Tensor w, double eps, bool plus_one) {
  c10::cuda::CUDAGuard guard(x.get_device());
  CHECK_BF16(x);
  CHECK_BF16(w);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 8 == 0, "rmsnorm: x [T, H] row-major");
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && w.numel() == H, "rmsnorm: H % 8 == 0 and w [H]");
  auto y = torch::empty({T, H}, x.options());
  auto rstd = torch::empty({T}, x.options().dtype(torch::kFloat32));
  rmsnorm_fwd(CBF(x), x.stride(0), CBF(w), BF(y), H, rstd.data_ptr<float>(), T, H, static_cast<float>(eps),
              plus_one ? 1 : 0, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, rstd};
}

torch::Tensor rmsnorm_bwd_t(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                            c10::optional<torch::Tensor> dres, torch::Tensor dw, bool plus_one) {
  c10::cuda::CUDAGuard guard(x.get_device());
  CHECK_BF16(dy);
  CHECK_CONTIG(dy);
  CHECK_F32(dw);
  const int T = x.size(0), H = x.size(1);
  auto dx = torch::empty({T, H}, x.options());
  const __nv_bfloat16* dr = nullptr;
  if (dres.has_value() && dres->defined()) {
    CHECK_CONTIG(*dres);
    dr = CBF(*dres);
  }
  rmsnorm_bwd(CBF(dy), CBF(x), x.stride(0), CBF(w), rstd.data_ptr<float>(), dr, BF(dx), dw.data_ptr<float>(), T, H,
              plus_one ? 1 : 0, cur_stream(x));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

void rope_t(torch::Tensor qkv, torch::Tensor pos, int64_t Hq, int64_t Hkv, int64_t D, double theta, bool inverse) {
  c10::cuda::CUDAGuard guard(qkv.get_device());
  CHECK_BF16(qkv);
  CHECK_I32(pos);
  CHECK_CONTIG(pos);
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1, "rope: qkv [T, W]");
  rope_apply(BF(qkv), qkv.stride(0), pos.data_ptr<int32_t>(), qkv.size(0), Hq, Hkv, D, static_cast<float>(theta),
             inverse, cur_stream(qkv));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

torch::Tensor swiglu_fwd_t(torch::Tensor gu) {
  c10::cuda::CUDAGuard guard(gu.get_device());
  CHECK_BF16(gu);
  CHECK_CONTIG(gu);
  const int T = gu.size(0), F = gu.size(1) / 2;
  TORCH_CHECK(F % 8 == 0, "swiglu: F % 8 == 0");
  auto out = torch::empty({T, F}, gu.options());
  swiglu_fwd(CBF(gu), BF(out), T, F, cur_stream(gu));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

torch::Tensor swiglu_bwd_t(torch::Tensor gu, torch::Tensor dout) {
  c10::cuda::CUDAGuard guard(gu.get_device());
  CHECK_CONTIG(gu);
  CHECK_CONTIG(dout);
  const int T = gu.size(0), F = gu.size(1) / 2;
  auto dgu = torch::empty_like(gu);
  swiglu_bwd(CBF(gu), CBF(dout), BF(dgu), T, F, cur_stream(gu));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dgu;
}

torch::Tensor embed_fwd_t(torch::Tensor ids, torch::Tensor W) {
  c10::cuda::CUDAGuard guard(W.get_device());
  CHECK_I64(ids);
  CHECK_CONTIG(ids);
  CHECK_CONTIG(W);
  const int T = ids.numel(), V = W.size(0), H = W.size(1);
  auto out = torch::empty({T, H}, W.options());
  embed_fwd(ids.data_ptr<int64_t>(), CBF(W), BF(out), T, H, V, status_ptr(W.get_device()), cur_stream(W));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void embed_bwd_t(torch::Tensor ids, torch::Tensor dout, torch::Tensor dW) {
  c10::cuda::CUDAGuard guard(dW.get_device());
  CHECK_F32(dW);
  CHECK_CONTIG(dout);
  embed_bwd(ids.data_ptr<int64_t>(), CBF(dout), dW.data_ptr<float>(), ids.numel(), dW.size(1), dW.size(0),
            status_ptr(dW.get_device()), cur_stream(dW));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_write_t(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t D, torch::Tensor slots, torch::Tensor kc,
                torch::Tensor vc) {
  c10::cuda::CUDAGuard guard(qkv.get_device());
  CHECK_I64(slots);
  CHECK_CONTIG(slots);
  CHECK_CONTIG(kc);
  CHECK_CONTIG(vc);
  TORCH_CHECK(qkv.stride(1) == 1, "kv_write: qkv rows");
  TORCH_CHECK(kc.numel() == vc.numel() && kc.size(-1) == Hkv * D, "kv_write: k / v cache shapes");
  kv_write(CBF(qkv), qkv.stride(0), Hq, Hkv, D, slots.data_ptr<int64_t>(), BF(kc), BF(vc), slots.numel(),
           kc.numel() / (Hkv * D), status_ptr(qkv.get_device()), cur_stream(qkv));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sqnorm_accum_t(torch::Tensor g, torch::Tensor out) {
  c10::cuda::CUDAGuard guard(g.get_device());
  CHECK_F32(g);
  CHECK_CONTIG(g);
  sqnorm_accum(g.data_ptr<float>(), g.numel(), out.data_ptr<float>(), cur_stream(g));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_t(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p16,
             double lr, double b1, double b2, double eps, double wd, int64_t step,
             c10::optional<torch::Tensor> sqnorm, double max_norm, double grad_scale) {
  c10::cuda::CUDAGuard guard(p.get_device());
  for (auto* t : {&p, &g, &m, &v}) {
    CHECK_F32(*t);
    CHECK_CONTIG(*t);
    TORCH_CHECK(t->numel() == p.numel(), "adamw: size mismatch");
  }
  __nv_bfloat16* w16 = nullptr;
  if (p16.has_value() && p16->defined()) {
    CHECK_BF16(*p16);
    CHECK_CONTIG(*p16);
    TORCH_CHECK(p16->numel() == p.numel(), "adamw: bf16 copy size");
    w16 = BF(*p16);
  }
  const float* sq = (sqnorm.has_value() && sqnorm->defined()) ? sqnorm->data_ptr<float>() : nullptr;
  adamw_step(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), w16, p.numel(),
             lr, b1, b2, eps, wd, static_cast<int>(step), sq, max_norm, grad_scale, cur_stream(p));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ attention
std::vector<torch::Tensor> attn_fwd_t(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor cu_q,
                                      torch::Tensor cu_k, torch::Tensor key_idx, torch::Tensor tiles, int64_t Hq,
                                      int64_t Hkv, int64_t D, double scale, bool causal, bool want_lse,
                                      int64_t use_tc, c10::optional<torch::Tensor> trace) {
  c10::cuda::CUDAGuard guard(q.get_device());
  CHECK_BF16(q);
  CHECK_BF16(k);
  CHECK_BF16(v);
  for (auto* t : {&cu_q, &cu_k, &key_idx, &tiles}) {
    CHECK_I32(*t);
    CHECK_CONTIG(*t);
  }
  TORCH_CHECK(D == 64 || D == 128, "attention: head dim 64 or 128");
  TORCH_CHECK(Hq % Hkv == 0, "attention: Hq % Hkv == 0");
  TORCH_CHECK(q.stride(1) == 1 && k.stride(1) == 1 && v.stride(1) == 1, "attention: rows must be contiguous");
  TORCH_CHECK(k.stride(0) == v.stride(0), "attention: k and v must share a row stride");
  TORCH_CHECK(q.stride(0) % 8 == 0 && k.stride(0) % 8 == 0, "attention: row strides multiple of 8");
  const int Tq = q.size(0);
  auto o = torch::empty({Tq, Hq * D}, q.options());
  auto lse = want_lse ? torch::empty({Hq, Tq}, q.options().dtype(torch::kFloat32)) : torch::Tensor();
  AttnParams p{};
  p.q = CBF(q);
  p.k = CBF(k);
  p.v = CBF(v);
  p.o = BF(o);
  p.lse = want_lse ? lse.data_ptr<float>() : nullptr;
  p.cu_q = cu_q.data_ptr<int32_t>();
  p.cu_k = cu_k.data_ptr<int32_t>();
  p.key_idx = key_idx.data_ptr<int32_t>();
  p.tiles = tiles.data_ptr<int32_t>();
  p.ldq = q.stride(0);
  p.ldk = k.stride(0);
  p.ldo = Hq * D;
  p.Tq = Tq;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = static_cast<float>(scale);
  p.causal = causal ? 1 : 0;
  p.trace = (trace.has_value() && trace->defined()) ? reinterpret_cast<unsigned long long*>(trace->data_ptr())
                                                      : nullptr;
  if (use_tc == 2) {
    // two query tiles per CTA; tiles hold q0 multiples of 256
    TORCH_CHECK(D == 128, "attention: the tcgen05 forward needs head_dim 128");
    AttnMaps maps;
    maps.q = make_tmap_bf16_2d(q.data_ptr(), Hq * D, Tq, q.stride(0), 64, 128);
    maps.k = make_tmap_bf16_2d(k.data_ptr(), Hkv * D, k.size(0), k.stride(0), 64, 64);
    maps.v = make_tmap_bf16_2d(v.data_ptr(), Hkv * D, v.size(0), v.stride(0), 64, 64);
    attn_fwd_pp(p, maps, tiles.numel() / 2, status_ptr(q.get_device()), cur_stream(q));
  } else {
    TORCH_CHECK(use_tc == 0, "attention: kernel mode must be 2 (tcgen05, head_dim 128) or 0 (mma.sync)");
    attn_fwd(p, tiles.numel() / 2, D, cur_stream(q));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, lse};
}

// Returns dq (bf16 [Tq, Hq*D]); dk/dv are accumulated into the fp32 buffers.
torch::Tensor attn_bwd_t(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dO,
                         torch::Tensor lse, torch::Tensor cu_q, torch::Tensor cu_k, torch::Tensor key_idx,
                         torch::Tensor qtiles, torch::Tensor ktiles, torch::Tensor dk_acc, torch::Tensor dv_acc,
                         int64_t Hq, int64_t Hkv, int64_t D, double scale, bool causal, int64_t use_tc) {
  c10::cuda::CUDAGuard guard(q.get_device());
  CHECK_CONTIG(dO);
  CHECK_CONTIG(o);
  CHECK_F32(dk_acc);
  CHECK_F32(dv_acc);
  TORCH_CHECK(dk_acc.stride(0) == dv_acc.stride(0), "attn_bwd: accumulators share a row stride");
  const int Tq = q.size(0);
  auto delta = torch::empty({Hq, Tq}, q.options().dtype(torch::kFloat32));
  attn_bwd_delta(CBF(o), o.stride(0), CBF(dO), dO.stride(0), delta.data_ptr<float>(), Tq, Hq, D, cur_stream(q));
  auto dq = torch::empty({Tq, Hq * D}, q.options());
  AttnBwdParams p{};
  p.q = CBF(q);
  p.k = CBF(k);
  p.v = CBF(v);
  p.dO = CBF(dO);
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq = BF(dq);
  p.dk_acc = dk_acc.data_ptr<float>();
  p.dv_acc = dv_acc.data_ptr<float>();
  p.cu_q = cu_q.data_ptr<int32_t>();
  p.cu_k = cu_k.data_ptr<int32_t>();
  p.key_idx = key_idx.data_ptr<int32_t>();
  p.tiles = qtiles.data_ptr<int32_t>();
  p.ktiles = ktiles.data_ptr<int32_t>();
  p.ldq = q.stride(0);
  p.ldk = k.stride(0);
  p.lddo = dO.stride(0);
  p.lddq = Hq * D;
  p.ld_acc = dk_acc.stride(0);
  p.Tq = Tq;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = static_cast<float>(scale);
  p.causal = causal ? 1 : 0;
  if (use_tc) {
    // tcgen05 kernels: qtiles / ktiles hold 128-row tiles
    TORCH_CHECK(D == 128, "attention: the tcgen05 backward needs head_dim 128");
    TORCH_CHECK(dO.stride(0) % 8 == 0, "attn_bwd: dO row stride multiple of 8");
    AttnBwdMaps maps;
    maps.q = make_tmap_bf16_2d(q.data_ptr(), Hq * D, Tq, q.stride(0), 64, 64);
    maps.dO = make_tmap_bf16_2d(dO.data_ptr(), Hq * D, Tq, dO.stride(0), 64, 64);
    maps.k = make_tmap_bf16_2d(k.data_ptr(), Hkv * D, k.size(0), k.stride(0), 64, 64);
    maps.v = make_tmap_bf16_2d(v.data_ptr(), Hkv * D, v.size(0), v.stride(0), 64, 64);
    attn_bwd_tc(p, maps, qtiles.numel() / 2, ktiles.numel() / 2, status_ptr(q.get_device()), cur_stream(q));
  } else {
    attn_bwd(p, qtiles.numel() / 2, ktiles.numel() / 2, D, cur_stream(q));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dq;
}

void attn_decode_t(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor kv_start,
                   torch::Tensor kv_len, torch::Tensor kv_indices, torch::Tensor o, torch::Tensor part_o, torch::Tensor part_lse,
                   int64_t Hq, int64_t Hkv, int64_t D, int64_t num_splits, double scale) {
  c10::cuda::CUDAGuard guard(q.get_device());
  CHECK_I32(kv_start);
  CHECK_I32(kv_len);
  CHECK_I32(kv_indices);
  TORCH_CHECK(Hq / Hkv <= 16, "decode: GQA group must be <= 16");
  TORCH_CHECK(q.stride(1) == 1 && o.stride(1) == 1, "decode: rows contiguous");
  const int B = q.size(0);
  TORCH_CHECK(kv_start.numel() >= B && kv_len.numel() >= B, "decode: kv_start/kv_len per request");
  DecodeParams p{};
  p.q = CBF(q);
  p.k_cache = CBF(kc);
  p.v_cache = CBF(vc);
  p.o = BF(o);
  p.kv_start = kv_start.data_ptr<int32_t>();
  p.kv_len = kv_len.data_ptr<int32_t>();
  p.kv_indices = kv_indices.data_ptr<int32_t>();
  p.num_splits = static_cast<int>(num_splits);
  if (num_splits > 1) {
    TORCH_CHECK(part_o.numel() >= static_cast<int64_t>(B) * Hq * num_splits * D &&
                    part_lse.numel() >= static_cast<int64_t>(B) * Hq * num_splits,
                "decode: scratch too small");
    p.part_o = part_o.data_ptr<float>();
    p.part_lse = part_lse.data_ptr<float>();
  }
  p.ldq = q.stride(0);
  p.ldk = Hkv * D;
  p.ldo = o.stride(0);
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = static_cast<float>(scale);
  attn_decode(p, B, D, cur_stream(q));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Persistent split-K decode (head_dim 128): grid = min(items, 2 CTAs per SM).
void attn_decode_persistent_t(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor kv_start,
                              torch::Tensor kv_len, torch::Tensor kv_indices, torch::Tensor o, torch::Tensor part_o,
                              torch::Tensor part_lse, int64_t Hq, int64_t Hkv, int64_t num_splits, double scale) {
  c10::cuda::CUDAGuard guard(q.get_device());
  CHECK_I32(kv_start);
  CHECK_I32(kv_len);
  CHECK_I32(kv_indices);
  CHECK_BF16(q);
  CHECK_BF16(kc);
  CHECK_BF16(vc);
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= 16, "decode: GQA group must be <= 16");
  TORCH_CHECK(q.stride(1) == 1 && o.stride(1) == 1 && kc.is_contiguous() && vc.is_contiguous(), "decode: layout");
  TORCH_CHECK(kc.size(-1) == Hkv * 128, "decode_persistent: head_dim 128 only");
  DecodePersistParams p{};
  p.q = CBF(q);
  p.k_cache = CBF(kc);
  p.v_cache = CBF(vc);
  p.o = BF(o);
  p.kv_start = kv_start.data_ptr<int32_t>();
  p.kv_len = kv_len.data_ptr<int32_t>();
  p.kv_indices = kv_indices.data_ptr<int32_t>();
  p.ldq = q.stride(0);
  p.ldo = o.stride(0);
  p.B = q.size(0);
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.num_splits = static_cast<int>(num_splits);
  p.scale = static_cast<float>(scale);
  if (num_splits > 1) {
    TORCH_CHECK(part_o.numel() >= static_cast<int64_t>(p.B) * Hq * num_splits * 128 &&
                    part_lse.numel() >= static_cast<int64_t>(p.B) * Hq * num_splits,
                "decode: scratch too small");
    p.part_o = part_o.data_ptr<float>();
    p.part_lse = part_lse.data_ptr<float>();
  }
  const int items = p.B * p.Hkv * p.num_splits;
  const int grid = std::min(items, 2 * num_sms(q.get_device()));
  if (p.B == 0) return;
  decode_persistent_launch(p, grid, status_ptr(q.get_device()), cur_stream(q));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_comm(py::module& m);
void register_tp(py::module& m);
void register_recur(py::module& m);

}  // namespace octo

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace octo;
  register_comm(m);
  register_tp(m);
  register_recur(m);
  m.doc() = "octopus_b200 sm_100a kernels";
  m.def("status_tensor", [](int64_t d) { return status_tensor(static_cast<int>(d)); });
  m.def("gemm_out", &gemm_out, py::arg("A"), py::arg("a_mn"), py::arg("B"), py::arg("b_mn"), py::arg("C"),
        py::arg("alpha") = 1.0, py::arg("residual") = py::none(), py::arg("bias") = py::none(),
        py::arg("accumulate") = false, py::arg("bn") = 0);
  m.def("head_fwd", &head_fwd);
  m.def("head_grad_logits", &head_grad_logits);
  m.def("sample_head", &sample_head);
  m.def("rmsnorm_fwd", &rmsnorm_fwd_t);
  m.def("rmsnorm_bwd", &rmsnorm_bwd_t);
  m.def("rope", &rope_t);
  m.def("swiglu_fwd", &swiglu_fwd_t);
  m.def("swiglu_bwd", &swiglu_bwd_t);
  m.def("embed_fwd", &embed_fwd_t);
  m.def("embed_bwd", &embed_bwd_t);
  m.def("kv_write", &kv_write_t);
  m.def("gemm_swiglu", &gemm_swiglu_t);
  m.def("gemm_rope", &gemm_rope_t, py::arg("A"), py::arg("W"), py::arg("bias"), py::arg("pos"), py::arg("theta"),
        py::arg("Hq"), py::arg("Hkv"), py::arg("D"));
  m.def("gemm_res_norm", &gemm_res_norm_t, py::arg("A"), py::arg("W"), py::arg("residual"), py::arg("norm_w"),
        py::arg("eps"), py::arg("plus_one"), py::arg("bias") = py::none());
  m.def("gemm_qkv_rope", &gemm_qkv_rope_t, py::arg("A"), py::arg("W"), py::arg("bias"), py::arg("pos"),
        py::arg("theta"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("slots"), py::arg("kc"),
        py::arg("vc"));
  m.def("sqnorm_accum", &sqnorm_accum_t);
  m.def("adamw", &adamw_t);
  m.def("attn_fwd", &attn_fwd_t, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("cu_q"), py::arg("cu_k"),
        py::arg("key_idx"), py::arg("tiles"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("scale"),
        py::arg("causal"), py::arg("want_lse"), py::arg("use_tc") = 0, py::arg("trace") = py::none());
  m.def("attn_bwd", &attn_bwd_t, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("dO"),
        py::arg("lse"), py::arg("cu_q"), py::arg("cu_k"), py::arg("key_idx"), py::arg("qtiles"), py::arg("ktiles"),
        py::arg("dk_acc"), py::arg("dv_acc"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("scale"),
        py::arg("causal"), py::arg("use_tc") = 0);
  m.def("attn_decode", &attn_decode_t);
  m.def("attn_decode_persistent", &attn_decode_persistent_t);
  m.def("attn_decode_shared", &attn_decode_shared_t, py::arg("q"), py::arg("kc"), py::arg("vc"),
        py::arg("kv_indices"), py::arg("kv_len"), py::arg("seg_rows"), py::arg("seg_slot"), py::arg("seg_start"),
        py::arg("seg_len"), py::arg("seg_off"), py::arg("items"), py::arg("n_items"), py::arg("row_nslot"),
        py::arg("o"), py::arg("part_o"), py::arg("part_lse"), py::arg("Hq"), py::arg("Hkv"), py::arg("max_slots"),
        py::arg("chunk"), py::arg("scale"), py::arg("use_tc") = false, py::arg("trace") = py::none());
  m.def("set_pdl", &set_pdl);
}
