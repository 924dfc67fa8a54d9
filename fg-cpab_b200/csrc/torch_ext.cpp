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
}
