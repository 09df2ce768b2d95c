// PyTorch custom-op registration over the C ABI (include/bfb_b200.h).
//
// torch only allocates outputs and workspaces and supplies the current CUDA
// stream; every kernel runs inside libbfb_b200.so.  There is no CPU kernel:
// CPU tensors are rejected.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <vector>

#include "bfb_b200.h"

namespace {

void check(int status, const char* what) {
  if (status == BFB_OK) return;
  if (status == BFB_ERR_CUDA)
    TORCH_CHECK(false, what, " failed: ", bfb_status_string(status), " (", bfb_last_cuda_error(), ")");
  if (status == BFB_ERR_INVALID_ARG || status == BFB_ERR_TOO_LARGE)
    TORCH_CHECK_VALUE(false, what, " failed: ", bfb_status_string(status));
  if (status == BFB_ERR_UNSUPPORTED_DTYPE) TORCH_CHECK_TYPE(false, what, " failed: ", bfb_status_string(status));
  TORCH_CHECK(false, what, " failed: ", bfb_status_string(status));
}

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return BFB_F32;
    case at::kHalf: return BFB_F16;
    case at::kBFloat16: return BFB_BF16;
    default: TORCH_CHECK_TYPE(false, "unsupported floating dtype ", t.scalar_type());
  }
  return -1;
}

void* stream_of(const at::Tensor& t) {
  return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void require_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor (this library has no CPU path)");
}

// ---------------------------------------------------------------- bev_pool
std::tuple<at::Tensor, at::Tensor> bev_pool_forward(const at::Tensor& feats_in, const at::Tensor& coords_in,
                                                     int64_t B, int64_t D, int64_t H, int64_t W) {
  require_cuda(feats_in, "feats");
  require_cuda(coords_in, "coords");
  TORCH_CHECK(feats_in.device() == coords_in.device(), "feats and coords must be on one device");
  c10::cuda::CUDAGuard guard(feats_in.device());
  auto feats = feats_in.contiguous();
  auto coords = coords_in.contiguous();
  const int64_t n = feats.size(0), c = feats.size(1);
  const int itype = coords.scalar_type() == at::kLong ? BFB_I64 : BFB_I32;
  size_t plan_b = 0, scratch_b = 0;
  check(bfb_bev_pool_workspace_sizes(n, c, B, D, H, W, &plan_b, &scratch_b), "bev_pool workspace query");
  auto opts = feats.options().dtype(at::kByte);
  auto plan = at::empty({(int64_t)plan_b}, opts);
  auto scratch = at::empty({(int64_t)scratch_b}, opts);
  auto out = at::empty({B, c, D, H, W}, feats.options());
  check(bfb_bev_pool_forward(feats.data_ptr(), dtype_code(feats), coords.data_ptr(), itype, n, c, B, D, H, W,
                             out.data_ptr(), plan.data_ptr(), plan_b, scratch.data_ptr(), scratch_b,
                             stream_of(feats)),
        "bev_pool forward");
  return {out, plan};
}

at::Tensor bev_pool_plan(const at::Tensor& coords_in, int64_t B, int64_t D, int64_t H, int64_t W) {
  require_cuda(coords_in, "coords");
  c10::cuda::CUDAGuard guard(coords_in.device());
  auto coords = coords_in.contiguous();
  const int64_t n = coords.size(0);
  const int itype = coords.scalar_type() == at::kLong ? BFB_I64 : BFB_I32;
  size_t plan_b = 0, scratch_b = 0;
  check(bfb_bev_pool_workspace_sizes(n, 1, B, D, H, W, &plan_b, &scratch_b), "bev_pool workspace query");
  auto opts = coords.options().dtype(at::kByte);
  auto plan = at::empty({(int64_t)plan_b}, opts);
  auto scratch = at::empty({(int64_t)scratch_b}, opts);
  check(bfb_bev_pool_plan(coords.data_ptr(), itype, n, B, D, H, W, plan.data_ptr(), plan_b, scratch.data_ptr(),
                          scratch_b, stream_of(coords)),
        "bev_pool plan");
  return plan;
}

at::Tensor bev_pool_forward_planned(const at::Tensor& feats_in, const at::Tensor& plan, int64_t B, int64_t D,
                                    int64_t H, int64_t W) {
  require_cuda(feats_in, "feats");
  c10::cuda::CUDAGuard guard(feats_in.device());
  auto feats = feats_in.contiguous();
  const int64_t n = feats.size(0), c = feats.size(1);
  auto out = at::empty({B, c, D, H, W}, feats.options());
  check(bfb_bev_pool_forward_planned(feats.data_ptr(), dtype_code(feats), n, c, B, D, H, W, plan.data_ptr(),
                                     (size_t)plan.numel(), out.data_ptr(), stream_of(feats)),
        "bev_pool forward");
  return out;
}

at::Tensor bev_pool_backward(const at::Tensor& grad_in, const at::Tensor& plan, int64_t n, int64_t B, int64_t D,
                             int64_t H, int64_t W) {
  require_cuda(grad_in, "grad_out");
  c10::cuda::CUDAGuard guard(grad_in.device());
  auto grad = grad_in.contiguous();
  TORCH_CHECK(grad.dim() == 5 && grad.size(0) == B && grad.size(2) == D && grad.size(3) == H && grad.size(4) == W,
              "grad_out must have shape [B, C, D, H, W]");
  const int64_t c = grad.size(1);
  auto gfeat = at::empty({n, c}, grad.options());
  check(bfb_bev_pool_backward(grad.data_ptr(), dtype_code(grad), n, c, B, D, H, W, plan.data_ptr(),
                              (size_t)plan.numel(), gfeat.data_ptr(), stream_of(grad)),
        "bev_pool backward");
  return gfeat;
}

int64_t bev_pool_invalid_count(const at::Tensor& plan) {
  c10::cuda::CUDAGuard guard(plan.device());
  int64_t v = 0;
  check(bfb_bev_pool_invalid_count(plan.data_ptr(), &v, stream_of(plan)), "bev_pool invalid count");
  return v;
}

}  // namespace

TORCH_LIBRARY(bfb_b200, m) {
  m.def("bev_pool_forward(Tensor feats, Tensor coords, int B, int D, int H, int W) -> (Tensor, Tensor)");
  m.def("bev_pool_plan(Tensor coords, int B, int D, int H, int W) -> Tensor");
  m.def("bev_pool_forward_planned(Tensor feats, Tensor plan, int B, int D, int H, int W) -> Tensor");
  m.def("bev_pool_backward(Tensor grad_out, Tensor plan, int n, int B, int D, int H, int W) -> Tensor");
  m.def("bev_pool_invalid_count(Tensor plan) -> int");
}

TORCH_LIBRARY_IMPL(bfb_b200, CUDA, m) {
  m.impl("bev_pool_forward", &bev_pool_forward);
  m.impl("bev_pool_plan", &bev_pool_plan);
  m.impl("bev_pool_forward_planned", &bev_pool_forward_planned);
  m.impl("bev_pool_backward", &bev_pool_backward);
  m.impl("bev_pool_invalid_count", &bev_pool_invalid_count);
}
