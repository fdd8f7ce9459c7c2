// torch_ext.cpp - thin torch binding of the krsi_b200 C ABI.
//
// Registers the operator names and schemas the reference registers through
// torch.library.triton_op (library/rmsnorm.py:86-103, library/geglu.py:85-101,
// library/relpos_attention.py:175-195), so that torch.compile(fullgraph=True) traces them
// as opaque ops.  The binding owns allocation (outputs and workspaces come from the torch
// caching allocator on the input's device), passes the current CUDA stream, and turns a
// nonzero krsi_status into a Python RuntimeError.  No synchronisation, so the ops can be
// captured in CUDA graphs.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "../../include/krsi_b200.h"

namespace {

int krsi_dtype_of(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return KRSI_F32;
    case at::kBFloat16: return KRSI_BF16;
    case at::kHalf: return KRSI_F16;
    default: TORCH_CHECK(false, "krsi: unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == KRSI_OK, what, " failed: ", krsi_error_string(rc), " (status ", rc, ")");
}

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "krsi: ", name, " must be a CUDA tensor");
}

at::Tensor workspace(const at::Tensor& like, size_t bytes) {
  return at::empty({(int64_t)std::max<size_t>(bytes, 16)}, like.options().dtype(at::kByte));
}

// ---------------------------------------------------------------- RMSNorm
std::tuple<at::Tensor, at::Tensor> rmsnorm_fwd(const at::Tensor& x2d_in, const at::Tensor& w_in, double eps) {
  check_cuda(x2d_in, "x2d");
  check_cuda(w_in, "w");
  TORCH_CHECK(x2d_in.dim() == 2, "rmsnorm: x2d must be 2-D, got ", x2d_in.dim(), "-D");
  TORCH_CHECK(w_in.dim() == 1 && w_in.size(0) == x2d_in.size(1), "rmsnorm: w must be [", x2d_in.size(1), "]");
  c10::cuda::CUDAGuard guard(x2d_in.device());
  auto x2d = x2d_in.contiguous();
  auto w = w_in.contiguous();
  auto y = at::empty_like(x2d);
  auto rstd = at::empty({x2d.size(0)}, x2d.options().dtype(at::kFloat));
  check_rc(krsi_rmsnorm_fwd(x2d.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr<float>(), x2d.size(0),
                            x2d.size(1), (float)eps, krsi_dtype_of(x2d), krsi_dtype_of(w),
                            at::cuda::getCurrentCUDAStream()),
           "krsi_rmsnorm_fwd");
  return {y, rstd};
}

std::tuple<at::Tensor, at::Tensor> rmsnorm_bwd(const at::Tensor& g_in, const at::Tensor& x2d_in,
                                               const at::Tensor& w_in, const at::Tensor& rstd_in) {
  check_cuda(g_in, "g");
  check_cuda(x2d_in, "x2d");
  TORCH_CHECK(x2d_in.dim() == 2 && g_in.sizes() == x2d_in.sizes(), "rmsnorm_bwd: g must match x2d");
  TORCH_CHECK(rstd_in.scalar_type() == at::kFloat && rstd_in.numel() == x2d_in.size(0), "rmsnorm_bwd: bad rstd");
  c10::cuda::CUDAGuard guard(x2d_in.device());
  auto x2d = x2d_in.contiguous();
  auto g = g_in.to(x2d.scalar_type()).contiguous();
  auto w = w_in.contiguous();
  auto rstd = rstd_in.contiguous();
  auto dx = at::empty_like(x2d);
  auto dw = at::empty_like(w);
  size_t ws = 0;
  check_rc(krsi_rmsnorm_bwd_workspace_size(x2d.size(0), x2d.size(1), &ws), "krsi_rmsnorm_bwd_workspace_size");
  auto wsp = workspace(x2d, ws);
  check_rc(krsi_rmsnorm_bwd(g.data_ptr(), x2d.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dx.data_ptr(),
                            dw.data_ptr(), wsp.data_ptr(), (size_t)wsp.numel(), x2d.size(0), x2d.size(1),
                            krsi_dtype_of(x2d), krsi_dtype_of(w), at::cuda::getCurrentCUDAStream()),
           "krsi_rmsnorm_bwd");
  return {dx, dw};
}

std::tuple<at::Tensor, at::Tensor> rmsnorm_bwd_add(const at::Tensor& g_in, const at::Tensor& x2d_in,
                                                   const at::Tensor& w_in, const at::Tensor& rstd_in,
                                                   const at::Tensor& gadd_in) {
  check_cuda(g_in, "g");
  check_cuda(x2d_in, "x2d");
  check_cuda(gadd_in, "gadd");
  TORCH_CHECK(x2d_in.dim() == 2 && g_in.sizes() == x2d_in.sizes() && gadd_in.sizes() == x2d_in.sizes(),
              "rmsnorm_bwd_add: g and gadd must match x2d");
  TORCH_CHECK(rstd_in.scalar_type() == at::kFloat && rstd_in.numel() == x2d_in.size(0), "rmsnorm_bwd_add: bad rstd");
  c10::cuda::CUDAGuard guard(x2d_in.device());
  auto x2d = x2d_in.contiguous();
  auto g = g_in.to(x2d.scalar_type()).contiguous();
  auto gadd = gadd_in.to(x2d.scalar_type()).contiguous();
  auto w = w_in.contiguous();
  auto rstd = rstd_in.contiguous();
  auto dx = at::empty_like(x2d);
  auto dw = at::empty_like(w);
  size_t ws = 0;
  check_rc(krsi_rmsnorm_bwd_workspace_size(x2d.size(0), x2d.size(1), &ws), "krsi_rmsnorm_bwd_workspace_size");
  auto wsp = workspace(x2d, ws);
  check_rc(krsi_rmsnorm_bwd_add(g.data_ptr(), x2d.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), gadd.data_ptr(),
                                dx.data_ptr(), dw.data_ptr(), wsp.data_ptr(), (size_t)wsp.numel(), x2d.size(0),
                                x2d.size(1), krsi_dtype_of(x2d), krsi_dtype_of(w), at::cuda::getCurrentCUDAStream()),
           "krsi_rmsnorm_bwd_add");
  return {dx, dw};
}

// ---------------------------------------------------------------- GEGLU
at::Tensor geglu_fwd(const at::Tensor& u_in) {
  check_cuda(u_in, "u");
  TORCH_CHECK(u_in.dim() == 2 && u_in.size(1) % 2 == 0, "geglu: u must be [rows, 2F]");
  c10::cuda::CUDAGuard guard(u_in.device());
  auto u = u_in.contiguous();
  const int64_t F = u.size(1) / 2;
  auto out = at::empty({u.size(0), F}, u.options());
  check_rc(krsi_geglu_fwd(u.data_ptr(), out.data_ptr(), u.size(0), F, krsi_dtype_of(u),
                          at::cuda::getCurrentCUDAStream()),
           "krsi_geglu_fwd");
  return out;
}

at::Tensor geglu_bwd(const at::Tensor& g_in, const at::Tensor& u_in) {
  check_cuda(g_in, "g");
  check_cuda(u_in, "u");
  TORCH_CHECK(u_in.dim() == 2 && u_in.size(1) % 2 == 0, "geglu_bwd: u must be [rows, 2F]");
  TORCH_CHECK(g_in.dim() == 2 && g_in.size(0) == u_in.size(0) && g_in.size(1) * 2 == u_in.size(1),
              "geglu_bwd: g must be [rows, F]");
  c10::cuda::CUDAGuard guard(u_in.device());
  auto u = u_in.contiguous();
  auto g = g_in.to(u.scalar_type()).contiguous();
  auto du = at::empty_like(u);
  check_rc(krsi_geglu_bwd(g.data_ptr(), u.data_ptr(), du.data_ptr(), u.size(0), u.size(1) / 2, krsi_dtype_of(u),
                          at::cuda::getCurrentCUDAStream()),
           "krsi_geglu_bwd");
  return du;
}

// ---------------------------------------------------------------- projection + GEGLU
std::tuple<at::Tensor, at::Tensor> linear_geglu_fwd(const at::Tensor& x_in, const at::Tensor& w_in) {
  check_cuda(x_in, "x2d");
  check_cuda(w_in, "w");
  TORCH_CHECK(x_in.dim() == 2, "linear_geglu: x2d must be 2-D, got ", x_in.dim(), "-D");
  TORCH_CHECK(w_in.dim() == 2 && w_in.size(1) == x_in.size(1) && w_in.size(0) % 2 == 0,
              "linear_geglu: w must be [2F, ", x_in.size(1), "]");
  TORCH_CHECK(x_in.scalar_type() == w_in.scalar_type(), "linear_geglu: x2d and w must have one dtype");
  c10::cuda::CUDAGuard guard(x_in.device());
  auto x = x_in.contiguous();
  auto w = w_in.contiguous();
  const int64_t F = w.size(0) / 2;
  auto u = at::empty({x.size(0), 2 * F}, x.options());
  auto out = at::empty({x.size(0), F}, x.options());
  check_rc(krsi_linear_geglu_fwd(x.data_ptr(), w.data_ptr(), u.data_ptr(), out.data_ptr(), x.size(0), x.size(1), F,
                                 krsi_dtype_of(x), at::cuda::getCurrentCUDAStream()),
           "krsi_linear_geglu_fwd");
  return {u, out};
}

at::Tensor linear_geglu_bwd(const at::Tensor& dy_in, const at::Tensor& w_in, const at::Tensor& u_in) {
  check_cuda(dy_in, "dy");
  check_cuda(w_in, "w");
  check_cuda(u_in, "u");
  TORCH_CHECK(dy_in.dim() == 2 && w_in.dim() == 2 && u_in.dim() == 2, "linear_geglu_bwd: 2-D tensors expected");
  TORCH_CHECK(w_in.size(0) == dy_in.size(1), "linear_geglu_bwd: w must be [", dy_in.size(1), ", F]");
  TORCH_CHECK(u_in.size(0) == dy_in.size(0) && u_in.size(1) == 2 * w_in.size(1),
              "linear_geglu_bwd: u must be [", dy_in.size(0), ", ", 2 * w_in.size(1), "]");
  TORCH_CHECK(dy_in.scalar_type() == w_in.scalar_type() && u_in.scalar_type() == w_in.scalar_type(),
              "linear_geglu_bwd: dy, w and u must have one dtype");
  c10::cuda::CUDAGuard guard(dy_in.device());
  auto dy = dy_in.contiguous();
  auto w = w_in.contiguous();
  auto u = u_in.contiguous();
  auto du = at::empty_like(u);
  check_rc(krsi_linear_geglu_bwd(dy.data_ptr(), w.data_ptr(), u.data_ptr(), du.data_ptr(), dy.size(0), dy.size(1),
                                 w.size(1), krsi_dtype_of(dy), at::cuda::getCurrentCUDAStream()),
           "krsi_linear_geglu_bwd");
  return du;
}

// ---------------------------------------------------------------- relpos attention
void check_attn_shapes(const at::Tensor& qkv, const at::Tensor& pd, int64_t B, int64_t S, int64_t H, int64_t D) {
  TORCH_CHECK(B >= 0 && S >= 0 && H > 0 && D > 0, "relpos_attention: bad B/S/H/D");
  TORCH_CHECK(qkv.dim() == 2 && qkv.size(0) == B * S && qkv.size(1) == 3 * H * D,
              "relpos_attention: qkv must be [B*S, 3*H*D] = [", B * S, ", ", 3 * H * D, "], got ", qkv.sizes());
  TORCH_CHECK(pd.dim() == 2 && pd.size(0) == H && pd.size(1) == std::max<int64_t>(2 * S - 1, 0),
              "relpos_attention: pd must be [H, 2S-1] = [", H, ", ", 2 * S - 1, "], got ", pd.sizes());
}

// qkv may be a row-strided view (the reference reads it in place with stride(0)); the
// kernels need unit column stride and a row stride that is a multiple of 8 elements.
at::Tensor qkv_view(const at::Tensor& qkv) {
  if (qkv.stride(1) == 1 && qkv.stride(0) % 8 == 0 && qkv.stride(0) >= qkv.size(1) &&
      (reinterpret_cast<uintptr_t>(qkv.data_ptr()) & 15u) == 0)
    return qkv;
  return qkv.contiguous();
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> relpos_attn_fwd(const at::Tensor& qkv_in, const at::Tensor& pd_in,
                                                               int64_t B, int64_t S, int64_t H, int64_t D,
                                                               double scale) {
  check_cuda(qkv_in, "qkv");
  check_cuda(pd_in, "pd");
  check_attn_shapes(qkv_in, pd_in, B, S, H, D);
  c10::cuda::CUDAGuard guard(qkv_in.device());
  auto qkv = qkv_view(qkv_in);
  auto pd = pd_in.to(at::kFloat).contiguous();
  auto out = at::empty({B * S, H * D}, qkv.options().memory_format(at::MemoryFormat::Contiguous));
  auto out32 = at::empty({B * S, H * D}, qkv.options().dtype(at::kFloat));
  auto lse = at::empty({B * H, S}, qkv.options().dtype(at::kFloat));
  check_rc(krsi_relpos_attn_fwd(qkv.data_ptr(), qkv.stride(0), pd.data_ptr<float>(), out.data_ptr(),
                                out32.data_ptr<float>(), lse.data_ptr<float>(), B, S, H, D, (float)scale,
                                krsi_dtype_of(qkv), at::cuda::getCurrentCUDAStream()),
           "krsi_relpos_attn_fwd");
  return {out, out32, lse};
}

std::tuple<at::Tensor, at::Tensor> relpos_attn_bwd(const at::Tensor& dout_in, const at::Tensor& qkv_in,
                                                   const at::Tensor& pd_in, const at::Tensor& out32_in,
                                                   const at::Tensor& lse_in, int64_t B, int64_t S, int64_t H,
                                                   int64_t D, double scale) {
  check_cuda(dout_in, "dout");
  check_cuda(qkv_in, "qkv");
  check_attn_shapes(qkv_in, pd_in, B, S, H, D);
  TORCH_CHECK(dout_in.numel() == B * S * H * D, "relpos_attn_bwd: dout must have B*S*H*D elements");
  TORCH_CHECK(out32_in.scalar_type() == at::kFloat && out32_in.numel() == B * S * H * D, "relpos_attn_bwd: bad out32");
  TORCH_CHECK(lse_in.scalar_type() == at::kFloat && lse_in.numel() == B * H * S, "relpos_attn_bwd: bad lse");
  c10::cuda::CUDAGuard guard(qkv_in.device());
  auto qkv = qkv_view(qkv_in);
  auto dout = dout_in.to(qkv.scalar_type()).contiguous();
  auto pd = pd_in.to(at::kFloat).contiguous();
  auto out32 = out32_in.contiguous();
  auto lse = lse_in.contiguous();
  auto dqkv = at::empty({B * S, 3 * H * D}, qkv.options().memory_format(at::MemoryFormat::Contiguous));
  auto dpd = at::empty({H, std::max<int64_t>(2 * S - 1, 0)}, qkv.options().dtype(at::kFloat));
  size_t ws = 0;
  check_rc(krsi_relpos_attn_bwd_workspace_size(B, S, H, D, &ws), "krsi_relpos_attn_bwd_workspace_size");
  auto wsp = workspace(qkv, ws);
  check_rc(krsi_relpos_attn_bwd(dout.data_ptr(), qkv.data_ptr(), qkv.stride(0), pd.data_ptr<float>(),
                                out32.data_ptr<float>(), lse.data_ptr<float>(), dqkv.data_ptr(), dqkv.stride(0),
                                dpd.data_ptr<float>(), wsp.data_ptr(), (size_t)wsp.numel(), B, S, H, D,
                                (float)scale, krsi_dtype_of(qkv), at::cuda::getCurrentCUDAStream()),
           "krsi_relpos_attn_bwd");
  return {dqkv, dpd};
}

// ---------------------------------------------------------------- T5 bucketed relative position
at::Tensor t5_bias_fwd(const at::Tensor& table_in, int64_t S, int64_t num_buckets, int64_t max_distance,
                       bool bidirectional) {
  check_cuda(table_in, "table");
  TORCH_CHECK(table_in.dim() == 2 && table_in.size(0) == num_buckets, "t5_bias: table must be [num_buckets, H]");
  TORCH_CHECK(S >= 0, "t5_bias: S must be >= 0");
  c10::cuda::CUDAGuard guard(table_in.device());
  auto table = table_in.contiguous();
  auto pd = at::empty({table.size(1), std::max<int64_t>(2 * S - 1, 0)}, table.options().dtype(at::kFloat));
  check_rc(krsi_t5_bias_fwd(table.data_ptr(), pd.data_ptr<float>(), S, table.size(1), (int)num_buckets,
                            (int)max_distance, bidirectional ? 1 : 0, krsi_dtype_of(table),
                            at::cuda::getCurrentCUDAStream()),
           "krsi_t5_bias_fwd");
  return pd;
}

at::Tensor t5_bias_bwd(const at::Tensor& dpd_in, const at::Tensor& table, int64_t S, int64_t num_buckets,
                       int64_t max_distance, bool bidirectional) {
  check_cuda(dpd_in, "dpd");
  TORCH_CHECK(table.dim() == 2 && table.size(0) == num_buckets, "t5_bias_bwd: table must be [num_buckets, H]");
  TORCH_CHECK(dpd_in.dim() == 2 && dpd_in.size(0) == table.size(1) && dpd_in.size(1) == std::max<int64_t>(2 * S - 1, 0),
              "t5_bias_bwd: dpd must be [H, 2S-1]");
  c10::cuda::CUDAGuard guard(dpd_in.device());
  auto dpd = dpd_in.to(at::kFloat).contiguous();
  auto dtable = at::empty(table.sizes(), table.options().memory_format(at::MemoryFormat::Contiguous));
  check_rc(krsi_t5_bias_bwd(dpd.data_ptr<float>(), dtable.data_ptr(), S, table.size(1), (int)num_buckets,
                            (int)max_distance, bidirectional ? 1 : 0, krsi_dtype_of(table),
                            at::cuda::getCurrentCUDAStream()),
           "krsi_t5_bias_bwd");
  return dtable;
}

}  // namespace

TORCH_LIBRARY(krsi, m) {
  m.def("rmsnorm_fwd(Tensor x2d, Tensor w, float eps) -> (Tensor, Tensor)");
  m.def("rmsnorm_bwd(Tensor g, Tensor x2d, Tensor w, Tensor rstd) -> (Tensor, Tensor)");
  m.def("rmsnorm_bwd_add(Tensor g, Tensor x2d, Tensor w, Tensor rstd, Tensor gadd) -> (Tensor, Tensor)");
  m.def("geglu_fwd(Tensor u) -> Tensor");
  m.def("geglu_bwd(Tensor g, Tensor u) -> Tensor");
  m.def("linear_geglu_fwd(Tensor x2d, Tensor w) -> (Tensor, Tensor)");
  m.def("linear_geglu_bwd(Tensor dy, Tensor w, Tensor u) -> Tensor");
  m.def("relpos_attn_fwd(Tensor qkv, Tensor pd, int B, int S, int H, int D, float scale) -> (Tensor, Tensor, Tensor)");
  m.def("relpos_attn_bwd(Tensor dout, Tensor qkv, Tensor pd, Tensor out32, Tensor lse, int B, int S, int H, int D, "
        "float scale) -> (Tensor, Tensor)");
  m.def("t5_bias_fwd(Tensor table, int S, int num_buckets, int max_distance, bool bidirectional) -> Tensor");
  m.def("t5_bias_bwd(Tensor dpd, Tensor table, int S, int num_buckets, int max_distance, bool bidirectional) -> Tensor");
}

TORCH_LIBRARY_IMPL(krsi, CUDA, m) {
  m.impl("rmsnorm_fwd", &rmsnorm_fwd);
  m.impl("rmsnorm_bwd", &rmsnorm_bwd);
  m.impl("rmsnorm_bwd_add", &rmsnorm_bwd_add);
  m.impl("geglu_fwd", &geglu_fwd);
  m.impl("geglu_bwd", &geglu_bwd);
  m.impl("linear_geglu_fwd", &linear_geglu_fwd);
  m.impl("linear_geglu_bwd", &linear_geglu_bwd);
  m.impl("relpos_attn_fwd", &relpos_attn_fwd);
  m.impl("relpos_attn_bwd", &relpos_attn_bwd);
  m.impl("t5_bias_fwd", &t5_bias_fwd);
  m.impl("t5_bias_bwd", &t5_bias_bwd);
}
