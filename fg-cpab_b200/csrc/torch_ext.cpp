// _cpab_ext: the transform_grid autograd node in C++ over the C ABI of
// libcpab_b200 (include/cpab_b200.h).
//
// The Python autograd.Function (cpab/pytorch/transformer.py, _CPABFunction)
// computes the same thing; this one exists because a step's host time is
// otherwise dominated by Python: per forward two ctypes calls with a dozen
// converted arguments each, tensor allocations and checks from Python, and a
// Python backward called back by the autograd engine.  Here the forward is one
// call from Python and the backward never enters Python.  Kernels, launch
// order, streams and results are exactly those of the Python path: both call
// the same C ABI entry points with the same arguments.
//
// Mirrors cpab/pytorch/transformer.py:73-168 of the reference (forward: A =
// B theta, expm, integrate; backward: adjoint moments, dtheta = B^T m).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "cpab_b200.h"

namespace {

using torch::Tensor;
using torch::autograd::AutogradContext;
using torch::autograd::variable_list;

void check(int status) {
  TORCH_CHECK(status == 0, "libcpab_b200: ", cpab_b200_last_error());
}

cpab_stream_t stream_of(const Tensor &t) {
  return reinterpret_cast<cpab_stream_t>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

const float *fptr(const Tensor &t) { return t.defined() ? t.data_ptr<float>() : nullptr; }
float *fptr_mut(Tensor &t) { return t.defined() ? t.data_ptr<float>() : nullptr; }
const int32_t *iptr(const Tensor &t) { return t.defined() ? t.data_ptr<int32_t>() : nullptr; }

int64_t cells(const std::vector<int64_t> &nc) {
  int64_t n = 1;
  for (int64_t c : nc) n *= c;
  return nc.size() == 1 ? n : (nc.size() == 2 ? 4 * n : 5 * n);
}

// The basis on the device, as DeviceBasis of transformer.py holds it.
struct Basis {
  Tensor rowptr, colidx, vals, t_rowptr, t_colidx, t_vals;
  int64_t d;
  bool dense;
};

Basis basis_of(const std::vector<Tensor> &b, int64_t d, bool dense) {
  TORCH_CHECK(b.size() == 6, "basis: expected 6 tensors (B and B^T in CSR)");
  return Basis{b[0], b[1], b[2], b[3], b[4], b[5], d, dense};
}

class TransformFunction : public torch::autograd::Function<TransformFunction> {
 public:
  // points [ndim, nP] or [n, ndim, nP]; theta [n, d]; order [1 or n, nP] or
  // undefined; returns [n, ndim, nP].
  static Tensor forward(AutogradContext *ctx, Tensor points, Tensor theta,
                        std::vector<Tensor> basis, int64_t d, bool dense,
                        std::vector<int64_t> nc, int64_t nstepsolver, bool adaptive,
                        c10::optional<Tensor> order, bool compute_points_grad, bool batched) {
    TORCH_CHECK(points.is_cuda() && theta.is_cuda(), "Only GPU tensors supported");
    TORCH_CHECK(points.device() == theta.device(), "points and theta must be on one device");
    TORCH_CHECK(points.scalar_type() == at::kFloat && theta.scalar_type() == at::kFloat,
                "points and theta must be float32");
    const c10::cuda::CUDAGuard guard(theta.device());
    const Basis B = basis_of(basis, d, dense);
    const int nd = (int)nc.size();
    const int64_t nC = cells(nc);
    const int64_t n = theta.size(0);
    const int64_t nP = points.size(-1);
    Tensor th = theta.contiguous();
    Tensor pts = points.contiguous();
    auto opts = th.options();
    Tensor As = at::empty({n, nC, nd, nd + 1}, opts);
    Tensor trels = nd > 1 ? at::empty_like(As) : Tensor();
    const float dT = nd > 1 ? 1.0f / (float)nstepsolver : 0.0f;
    const cpab_stream_t s = stream_of(th);
    if (B.dense) {
      Tensor th_t = th.t().contiguous();
      check(cpab_b200_build_A_tt(nd, nC, B.d, (int)n, iptr(B.rowptr), iptr(B.colidx),
                                 fptr(B.vals), fptr(th_t), dT, fptr_mut(As), fptr_mut(trels), s));
    } else {
      check(cpab_b200_build_A(nd, nC, B.d, (int)n, iptr(B.rowptr), iptr(B.colidx), fptr(B.vals),
                              fptr(th), dT, fptr_mut(As), fptr_mut(trels), s));
    }
    Tensor ord = order.has_value() ? order->contiguous() : Tensor();
    Tensor out = at::empty({n, nd, nP}, opts);
    std::vector<int32_t> nc32(nc.begin(), nc.end());
    if (nd == 1) {
      check(cpab_b200_forward_1d_closed_form(fptr(pts), nP, batched ? 1 : 0, iptr(ord), fptr(As),
                                             (int)n, nc32[0], fptr_mut(out), s));
    } else {
      check(cpab_b200_forward(nd, nc32.data(), fptr(pts), nP, batched ? 1 : 0, iptr(ord),
                              fptr(trels), fptr(As), (int)n, (int)nstepsolver, adaptive ? 1 : 0,
                              fptr_mut(out), s));
    }
    ctx->save_for_backward({pts, As});
    ctx->saved_data["basis"] = basis;
    ctx->saved_data["d"] = d;
    ctx->saved_data["dense"] = dense;
    ctx->saved_data["nc"] = nc;
    ctx->saved_data["T"] = nstepsolver;
    ctx->saved_data["adaptive"] = adaptive;
    ctx->saved_data["order"] = ord;
    ctx->saved_data["cpg"] = compute_points_grad;
    ctx->saved_data["batched"] = batched;
    return out;
  }

  static variable_list backward(AutogradContext *ctx, variable_list grads) {
    auto saved = ctx->get_saved_variables();
    Tensor pts = saved[0], As = saved[1];
    const c10::cuda::CUDAGuard guard(As.device());
    const Basis B = basis_of(ctx->saved_data["basis"].toTensorVector(),
                             ctx->saved_data["d"].toInt(), ctx->saved_data["dense"].toBool());
    const std::vector<int64_t> nc = ctx->saved_data["nc"].toIntVector();
    const int nd = (int)nc.size();
    const int64_t nC = cells(nc), n = As.size(0), nP = pts.size(-1);
    const bool batched = ctx->saved_data["batched"].toBool();
    Tensor ord = ctx->saved_data["order"].toTensor();
    const bool want_points = ctx->saved_data["cpg"].toBool() && ctx->needs_input_grad(0);
    Tensor grad = grads[0].contiguous();
    auto opts = As.options();
    Tensor moments = at::empty({n, nC, nd * (nd + 1)}, opts);
    Tensor gp = want_points ? at::empty({n, nd, nP}, opts) : Tensor();
    std::vector<int32_t> nc32(nc.begin(), nc.end());
    const cpab_stream_t s = stream_of(As);
    check(cpab_b200_backward(nd, nc32.data(), fptr(pts), nP, batched ? 1 : 0, iptr(ord),
                             fptr(As), (int)n, fptr(grad), (int)ctx->saved_data["T"].toInt(),
                             ctx->saved_data["adaptive"].toBool() ? 1 : 0, fptr_mut(moments),
                             fptr_mut(gp), s));
    if (gp.defined() && pts.dim() == 2) gp = gp.sum(0);
    Tensor gtheta;
    if (ctx->needs_input_grad(1)) {
      gtheta = at::empty({n, B.d}, opts);
      const int64_t D = nC * nd * (nd + 1);
      if (B.dense) {
        Tensor mt = moments.reshape({n, D}).t().contiguous();
        check(cpab_b200_project_tt(B.d, D, (int)n, iptr(B.t_rowptr), iptr(B.t_colidx),
                                   fptr(B.t_vals), fptr(mt), fptr_mut(gtheta), s));
      } else {
        check(cpab_b200_project(B.d, D, (int)n, iptr(B.t_rowptr), iptr(B.t_colidx),
                                fptr(B.t_vals), fptr(moments), fptr_mut(gtheta), s));
      }
    }
    // one gradient per forward input (only points and theta are differentiable)
    return {gp, gtheta, Tensor(), Tensor(), Tensor(), Tensor(), Tensor(), Tensor(), Tensor(),
            Tensor(), Tensor()};
  }
};

// As (and Trels) of n rows of theta [n, d] through the basis B (transposed
// operands for dense bases, as the Python build_A helper).
std::pair<Tensor, Tensor> build_tables(const Basis &B, int nd, int64_t nC, const Tensor &th,
                                       int64_t T, cpab_stream_t s) {
  const int64_t n = th.size(0);
  Tensor As = at::empty({n, nC, nd, nd + 1}, th.options());
  Tensor trels = at::empty_like(As);
  const float dT = 1.0f / (float)T;
  if (B.dense) {
    Tensor th_t = th.t().contiguous();
    check(cpab_b200_build_A_tt(nd, nC, B.d, (int)n, iptr(B.rowptr), iptr(B.colidx),
                               fptr(B.vals), fptr(th_t), dT, fptr_mut(As), fptr_mut(trels), s));
  } else {
    check(cpab_b200_build_A(nd, nC, B.d, (int)n, iptr(B.rowptr), iptr(B.colidx), fptr(B.vals),
                            fptr(th), dT, fptr_mut(As), fptr_mut(trels), s));
  }
  return {As, trels};
}

// dtheta [n, d] = B^T vec(moments[n]).
Tensor project_moments(const Basis &B, const Tensor &moments, cpab_stream_t s) {
  const int64_t n = moments.size(0);
  const int64_t D = moments.numel() / n;
  Tensor g = at::empty({n, B.d}, moments.options());
  if (B.dense) {
    Tensor mt = moments.reshape({n, D}).t().contiguous();
    check(cpab_b200_project_tt(B.d, D, (int)n, iptr(B.t_rowptr), iptr(B.t_colidx),
                               fptr(B.t_vals), fptr(mt), fptr_mut(g), s));
  } else {
    check(cpab_b200_project(B.d, D, (int)n, iptr(B.t_rowptr), iptr(B.t_colidx), fptr(B.t_vals),
                            fptr(moments), fptr_mut(g), s));
  }
  return g;
}

// The fused spatial-transformer warp (cpab/pytorch/warp.py, _Warp): data
// [B or 1, C, *size], thetas K tensors [B, d] (theta_K acts first: the chain
// runs them reversed), pixel axes and their cell order.  Arguments after
// thetas are constants; backward returns one gradient per forward input
// (data, each theta, then the constants).
class WarpFunction : public torch::autograd::Function<WarpFunction> {
 public:
  static constexpr int kConstArgs = 9;  // basis .. padding

  static Tensor forward(AutogradContext *ctx, Tensor data, at::TensorList thetas,
                        std::vector<Tensor> basis, int64_t d, bool dense,
                        std::vector<int64_t> nc, int64_t nstepsolver, bool adaptive, Tensor axes,
                        c10::optional<Tensor> order, int64_t padding) {
    TORCH_CHECK(!thetas.empty(), "at least one theta is needed");
    TORCH_CHECK(data.is_cuda() && data.scalar_type() == at::kFloat, "x must be a float32 CUDA tensor");
    const c10::cuda::CUDAGuard guard(data.device());
    const Basis B = basis_of(basis, d, dense);
    const int nd = (int)nc.size();
    const int64_t nC = cells(nc), K = (int64_t)thetas.size(), n = thetas[0].size(0);
    std::vector<Tensor> stages(thetas.rbegin(), thetas.rend());  // stage 0 = theta_K
    for (const Tensor &t : stages)
      TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.dim() == 2 &&
                      t.size(0) == n && t.size(1) == d && t.device() == data.device(),
                  "each theta must be a float32 tensor [B, ", d, "] on x's device");
    TORCH_CHECK(data.dim() == (int64_t)nc.size() + 2 && (data.size(0) == n || data.size(0) == 1),
                "x must be [B or 1, C, *spatial] with ", nc.size(), " spatial axes");
    const cpab_stream_t s = stream_of(data);
    Tensor th = K == 1 ? stages[0].contiguous() : at::cat(stages, 0);
    auto tabs = build_tables(B, nd, nC, th, nstepsolver, s);
    Tensor data_c = data.contiguous();
    std::vector<int64_t> size(data_c.sizes().begin() + 2, data_c.sizes().end());
    int64_t P = 1;
    for (int64_t v : size) P *= v;
    std::vector<int64_t> out_shape{n, data_c.size(1)};
    out_shape.insert(out_shape.end(), size.begin(), size.end());
    Tensor out = at::empty(out_shape, data_c.options());
    Tensor grid_t = at::empty({n, nd, P}, data_c.options());
    Tensor sp = K > 1 ? at::empty({K - 1, n, nd, P}, data_c.options()) : Tensor();
    Tensor ord = order.has_value() ? order->contiguous() : Tensor();
    std::vector<int32_t> nc32(nc.begin(), nc.end());
    const int batched = data_c.size(0) == n ? 1 : 0;
    check(cpab_b200_warp(nd, nc32.data(), size.data(), fptr(axes), iptr(ord), fptr(tabs.second),
                         fptr(tabs.first), (int)K, (int)n, (int)nstepsolver, adaptive ? 1 : 0,
                         fptr(data_c), batched, (int)data_c.size(1), size.data(), (int)padding,
                         fptr_mut(sp), fptr_mut(grid_t), fptr_mut(out), s));
    ctx->save_for_backward({data_c, tabs.first, grid_t, axes});
    ctx->saved_data["sp"] = sp;
    ctx->saved_data["order"] = ord;
    ctx->saved_data["basis"] = basis;
    ctx->saved_data["d"] = d;
    ctx->saved_data["dense"] = dense;
    ctx->saved_data["nc"] = nc;
    ctx->saved_data["T"] = nstepsolver;
    ctx->saved_data["adaptive"] = adaptive;
    ctx->saved_data["padding"] = padding;
    ctx->saved_data["K"] = K;
    return out;
  }

  static variable_list backward(AutogradContext *ctx, variable_list grads) {
    auto saved = ctx->get_saved_variables();
    Tensor data = saved[0], As = saved[1], grid_t = saved[2], axes = saved[3];
    const c10::cuda::CUDAGuard guard(As.device());
    const int64_t K = ctx->saved_data["K"].toInt();
    bool want_theta = false;
    for (int64_t i = 1; i <= K; ++i) want_theta = want_theta || ctx->needs_input_grad(i);
    const bool want_data = ctx->needs_input_grad(0);
    variable_list res(1 + K + kConstArgs);
    if (!(want_data || want_theta)) return res;
    const Basis B = basis_of(ctx->saved_data["basis"].toTensorVector(),
                             ctx->saved_data["d"].toInt(), ctx->saved_data["dense"].toBool());
    const std::vector<int64_t> nc = ctx->saved_data["nc"].toIntVector();
    const int nd = (int)nc.size();
    const int64_t nC = cells(nc), n = As.size(0) / K;
    Tensor sp = ctx->saved_data["sp"].toTensor();
    Tensor ord = ctx->saved_data["order"].toTensor();
    std::vector<int64_t> size(data.sizes().begin() + 2, data.sizes().end());
    std::vector<int32_t> nc32(nc.begin(), nc.end());
    Tensor grad = grads[0].contiguous();
    Tensor moments = at::empty({K * n, nC, nd * (nd + 1)}, As.options());
    Tensor gd = want_data ? at::empty_like(data) : Tensor();
    const cpab_stream_t s = stream_of(As);
    check(cpab_b200_warp_backward(
        nd, nc32.data(), size.data(), fptr(axes), iptr(ord), fptr(As), (int)K, (int)n,
        (int)ctx->saved_data["T"].toInt(), ctx->saved_data["adaptive"].toBool() ? 1 : 0,
        fptr(data), data.size(0) == n ? 1 : 0, (int)data.size(1), size.data(),
        (int)ctx->saved_data["padding"].toInt(), fptr(sp), fptr(grid_t), fptr(grad),
        fptr_mut(moments), fptr_mut(gd), s));
    res[0] = gd;
    if (want_theta) {
      Tensor g = project_moments(B, moments, s);  // [K * n, d], stage-major
      for (int64_t i = 0; i < K; ++i) res[1 + i] = g.narrow(0, (K - 1 - i) * n, n);
    }
    return res;
  }
};

Tensor warp(Tensor data, std::vector<Tensor> thetas, std::vector<Tensor> basis, int64_t d,
            bool dense, std::vector<int64_t> nc, int64_t nstepsolver, bool adaptive, Tensor axes,
            c10::optional<Tensor> order, int64_t padding) {
  return WarpFunction::apply(data, at::TensorList(thetas), basis, d, dense, nc, nstepsolver,
                             adaptive, axes, order, padding);
}

Tensor transform(Tensor points, Tensor theta, std::vector<Tensor> basis, int64_t d, bool dense,
                 std::vector<int64_t> nc, int64_t nstepsolver, bool adaptive,
                 c10::optional<Tensor> order, bool compute_points_grad, bool batched) {
  return TransformFunction::apply(points, theta, basis, d, dense, nc, nstepsolver, adaptive,
                                  order, compute_points_grad, batched);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "transform_grid autograd node over libcpab_b200 (C++)";
  m.def("transform", &transform,
        "points, theta, basis (6 CSR tensors of B and B^T), d, dense, nc, nstepsolver, "
        "adaptive, order or None, compute_points_grad, batched -> transformed points");
  m.def("warp", &warp,
        "x, thetas (list), basis (6 CSR tensors), d, dense, nc, nstepsolver, adaptive, pixel "
        "axes, order or None, padding mode -> grid_sample of x on the warped pixel grid");
}
