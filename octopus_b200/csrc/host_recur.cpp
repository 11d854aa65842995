// Host side of the linear-recurrence and causal-conv kernels (recurrence.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "recurrence.h"

namespace octo {

#define RCHECK(c, m) TORCH_CHECK(c, "recurrence: ", m)

static const __nv_bfloat16* cbf(const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
static __nv_bfloat16* bf(torch::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

static RecurParams make_params(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                               const torch::Tensor& g, const c10::optional<torch::Tensor>& beta,
                               const torch::Tensor& seg, int64_t H, double scale, bool delta,
                               const c10::optional<torch::Tensor>& init_state,
                               const c10::optional<torch::Tensor>& init_idx, const torch::Tensor& ckpt_off) {
  const int64_t dk = q.size(1) / H;
  RCHECK(dk == 64 || dk == 128, "head dim must be 64 or 128");
  RCHECK(k.size(1) == H * dk && v.size(1) == H * dk, "q, k, v widths");
  for (auto* t : {&q, &k, &v}) RCHECK(t->scalar_type() == torch::kBFloat16 && t->stride(1) == 1, "bf16 rows");
  RCHECK(g.scalar_type() == torch::kFloat32 && g.is_contiguous(), "g fp32 [rows, H]");
  RCHECK(seg.scalar_type() == torch::kInt32 && seg.is_contiguous() && seg.dim() == 2 && seg.size(0) == 2 &&
             ckpt_off.scalar_type() == torch::kInt32,
         "seg int32 [2, n_seg] (start; len), int32 checkpoint offsets");
  RecurParams p{};
  p.q = cbf(q);
  p.k = cbf(k);
  p.v = cbf(v);
  p.ldq = q.stride(0);
  p.ldk = k.stride(0);
  p.ldv = v.stride(0);
  p.g = g.data_ptr<float>();
  if (delta) {
    RCHECK(beta.has_value() && beta->scalar_type() == torch::kFloat32 && beta->is_contiguous(), "beta fp32");
    p.beta = beta->data_ptr<float>();
  }
  p.seg_start = seg.data_ptr<int32_t>();
  p.seg_len = seg.data_ptr<int32_t>() + seg.size(1);
  p.H = static_cast<int>(H);
  p.scale = static_cast<float>(scale);
  p.delta = delta ? 1 : 0;
  if (init_state.has_value() && init_state->defined()) {
    RCHECK(init_idx.has_value(), "init_idx with init_state");
    p.init_state = init_state->data_ptr<float>();
    p.init_idx = init_idx->data_ptr<int32_t>();
  }
  p.ckpt_off = ckpt_off.data_ptr<int32_t>();
  return p;
}

// returns (o, final_state [n_seg, H, dv, dk], ckpt)
std::vector<torch::Tensor> recur_fwd_t(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                       c10::optional<torch::Tensor> beta, torch::Tensor seg, int64_t H, double scale,
                                       bool delta, c10::optional<torch::Tensor> init_state,
                                       c10::optional<torch::Tensor> init_idx, torch::Tensor ckpt_off,
                                       int64_t n_ckpt) {
  c10::cuda::CUDAGuard guard(q.get_device());
  RecurParams p = make_params(q, k, v, g, beta, seg, H, scale, delta, init_state, init_idx, ckpt_off);
  const int64_t dk = q.size(1) / H, n_seg = seg.size(1);
  auto o = torch::empty({q.size(0), H * dk}, q.options());
  auto f32 = q.options().dtype(torch::kFloat32);
  auto fin = torch::empty({n_seg, H, dk, dk}, f32);
  auto ck = torch::empty({std::max<int64_t>(1, n_ckpt), H, dk, dk}, f32);
  p.o = bf(o);
  p.ldo = o.stride(0);
  p.final_state = fin.data_ptr<float>();
  p.ckpt = ck.data_ptr<float>();
  recur_fwd(p, static_cast<int>(n_seg), static_cast<int>(dk), at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, fin, ck};
}

// returns (dq, dk, dv, dg, dbeta, d_init)
std::vector<torch::Tensor> recur_bwd_t(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                       c10::optional<torch::Tensor> beta, torch::Tensor seg, int64_t H, double scale,
                                       bool delta, c10::optional<torch::Tensor> init_state,
                                       c10::optional<torch::Tensor> init_idx, torch::Tensor ckpt_off,
                                       torch::Tensor ckpt, torch::Tensor d_o, c10::optional<torch::Tensor> d_final) {
  c10::cuda::CUDAGuard guard(q.get_device());
  RecurParams p = make_params(q, k, v, g, beta, seg, H, scale, delta, init_state, init_idx, ckpt_off);
  const int64_t dk = q.size(1) / H, n_seg = seg.size(1);
  p.ckpt = ckpt.data_ptr<float>();
  p.ldo = d_o.stride(0);
  RCHECK(d_o.scalar_type() == torch::kBFloat16 && d_o.stride(1) == 1, "d_o bf16");
  auto scratch = torch::empty({static_cast<int64_t>(recur_scratch_floats(static_cast<int>(n_seg), static_cast<int>(H),
                                                                          static_cast<int>(dk)))},
                              q.options().dtype(torch::kFloat32));
  p.scratch = scratch.data_ptr<float>();
  auto dq = torch::empty_like(q, at::MemoryFormat::Contiguous);
  auto dkk = torch::empty_like(k, at::MemoryFormat::Contiguous);
  auto dv = torch::empty_like(v, at::MemoryFormat::Contiguous);
  RCHECK(dq.stride(0) == p.ldq && dkk.stride(0) == p.ldk && dv.stride(0) == p.ldv,
         "q, k, v must be contiguous [rows, H * d] (gradients use their strides)");
  auto f32 = q.options().dtype(torch::kFloat32);
  auto dg = torch::empty_like(g);
  auto dbeta = delta ? torch::empty_like(*beta) : torch::empty({0}, f32);
  auto dinit = torch::empty({n_seg, H, dk, dk}, f32);
  RecurGrads gr{};
  gr.d_o = cbf(d_o);
  gr.dq = bf(dq);
  gr.dk = bf(dkk);
  gr.dv = bf(dv);
  gr.dg = dg.data_ptr<float>();
  gr.dbeta = delta ? dbeta.data_ptr<float>() : nullptr;
  if (d_final.has_value() && d_final->defined()) gr.d_final = d_final->data_ptr<float>();
  gr.d_init = dinit.data_ptr<float>();
  recur_bwd(p, gr, static_cast<int>(n_seg), static_cast<int>(dk), at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dq, dkk, dv, dg, dbeta, dinit};
}

static ConvParams make_conv(const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& bias,
                            const torch::Tensor& cu, const c10::optional<torch::Tensor>& ctx,
                            const c10::optional<torch::Tensor>& ctx_idx, bool silu) {
  RCHECK(x.scalar_type() == torch::kBFloat16 && x.stride(1) == 1, "conv x bf16 rows");
  RCHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.dim() == 2 && w.size(0) == x.size(1) &&
             w.size(1) <= 8,
         "conv w fp32 [C, W <= 8]");
  ConvParams p{};
  p.x = cbf(x);
  p.ldx = x.stride(0);
  p.w = w.data_ptr<float>();
  if (bias.has_value() && bias->defined()) p.bias = bias->data_ptr<float>();
  p.cu = cu.data_ptr<int32_t>();
  p.C = x.size(1);
  p.W = w.size(1);
  if (ctx.has_value() && ctx->defined()) {
    RCHECK(ctx->scalar_type() == torch::kFloat32 && ctx->is_contiguous(), "conv ctx fp32 [n, W - 1, C]");
    p.ctx = ctx->data_ptr<float>();
    p.ctx_idx = ctx_idx->data_ptr<int32_t>();
  }
  p.silu = silu ? 1 : 0;
  return p;
}

torch::Tensor conv_fwd_t(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias, torch::Tensor cu,
                         c10::optional<torch::Tensor> ctx, c10::optional<torch::Tensor> ctx_idx, bool silu) {
  c10::cuda::CUDAGuard guard(x.get_device());
  ConvParams p = make_conv(x, w, bias, cu, ctx, ctx_idx, silu);
  auto y = torch::empty({x.size(0), x.size(1)}, x.options());
  p.y = bf(y);
  p.ldy = y.stride(0);
  conv_fwd(p, static_cast<int>(cu.numel() - 1), at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// returns (dx, dw, dbias, dctx [n_seg, W - 1, C])
std::vector<torch::Tensor> conv_bwd_t(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                                      torch::Tensor cu, c10::optional<torch::Tensor> ctx,
                                      c10::optional<torch::Tensor> ctx_idx, bool silu, torch::Tensor dy) {
  c10::cuda::CUDAGuard guard(x.get_device());
  ConvParams p = make_conv(x, w, bias, cu, ctx, ctx_idx, silu);
  RCHECK(dy.scalar_type() == torch::kBFloat16 && dy.is_contiguous() && dy.sizes() == x.sizes(), "conv dy");
  p.ldy = dy.stride(0);
  auto dx = torch::empty({x.size(0), x.size(1)}, x.options());
  RCHECK(dx.stride(0) == p.ldx, "conv: x must be contiguous");
  auto dw = torch::zeros_like(w);
  auto db = torch::zeros({x.size(1)}, w.options());
  const int64_t n_seg = cu.numel() - 1;
  auto dctx = torch::zeros({n_seg, std::max<int64_t>(1, w.size(1) - 1), x.size(1)}, w.options());
  conv_bwd(p, static_cast<int>(n_seg), dy.data_ptr(), dx.data_ptr(), dw.data_ptr<float>(), db.data_ptr<float>(),
           dctx.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dx, dw, db, dctx};
}

int64_t recur_chunk_t() { return recur_chunk(); }

void register_recur(py::module& m) {
  m.def("recur_fwd", &recur_fwd_t);
  m.def("recur_bwd", &recur_bwd_t);
  m.def("conv_fwd", &conv_fwd_t);
  m.def("conv_bwd", &conv_bwd_t);
  m.def("recur_chunk", &recur_chunk_t);
}

}  // namespace octo
