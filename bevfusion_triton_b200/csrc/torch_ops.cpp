// PyTorch custom-op registration over the C ABI (include/bfb_b200.h).
//
// torch only allocates outputs and workspaces and supplies the current CUDA
// stream; every kernel runs inside libbfb_b200.so.  There is no CPU kernel:
// CPU tensors are rejected.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "bfb_b200.h"

namespace {

// An NVTX range around every op (header-only NVTX3; inert unless a profiler
// such as Nsight Systems is attached), named bfb_b200::<op>.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
};

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
// A plan tensor is allocated at exactly the size its geometry needs, so a plan
// handed in with other (n, B, D, H, W) is refused here when its size differs;
// the kernels compare the geometry stamped in the plan as well and write
// nothing on a mismatch.
void check_plan(const at::Tensor& plan, int64_t n, int64_t B, int64_t D, int64_t H, int64_t W) {
  require_cuda(plan, "plan");
  TORCH_CHECK_VALUE(plan.scalar_type() == at::kByte && plan.dim() == 1 && plan.is_contiguous(),
                    "plan must be the uint8 tensor returned by a bev_pool plan call");
  size_t plan_b = 0;
  check(bfb_bev_pool_workspace_sizes(n, 1, B, D, H, W, &plan_b, nullptr), "bev_pool workspace query");
  TORCH_CHECK_VALUE((size_t)plan.numel() == plan_b, "bev_pool plan was built for another geometry: it holds ",
                    plan.numel(), " bytes, (n=", n, ", B=", B, ", D=", D, ", H=", H, ", W=", W, ") needs ", plan_b);
}

std::tuple<at::Tensor, at::Tensor> bev_pool_forward(const at::Tensor& feats_in, const at::Tensor& coords_in,
                                                     int64_t B, int64_t D, int64_t H, int64_t W) {
  NvtxRange nvtx_("bfb_b200::bev_pool_forward");
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
  NvtxRange nvtx_("bfb_b200::bev_pool_plan");
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
  NvtxRange nvtx_("bfb_b200::bev_pool_forward_planned");
  require_cuda(feats_in, "feats");
  c10::cuda::CUDAGuard guard(feats_in.device());
  auto feats = feats_in.contiguous();
  const int64_t n = feats.size(0), c = feats.size(1);
  check_plan(plan, n, B, D, H, W);
  auto out = at::empty({B, c, D, H, W}, feats.options());
  check(bfb_bev_pool_forward_planned(feats.data_ptr(), dtype_code(feats), n, c, B, D, H, W, plan.data_ptr(),
                                     (size_t)plan.numel(), out.data_ptr(), stream_of(feats)),
        "bev_pool forward");
  return out;
}

at::Tensor bev_pool_backward(const at::Tensor& grad_in, const at::Tensor& plan, int64_t n, int64_t B, int64_t D,
                             int64_t H, int64_t W) {
  NvtxRange nvtx_("bfb_b200::bev_pool_backward");
  require_cuda(grad_in, "grad_out");
  c10::cuda::CUDAGuard guard(grad_in.device());
  auto grad = grad_in.contiguous();
  TORCH_CHECK(grad.dim() == 5 && grad.size(0) == B && grad.size(2) == D && grad.size(3) == H && grad.size(4) == W,
              "grad_out must have shape [B, C, D, H, W]");
  const int64_t c = grad.size(1);
  check_plan(plan, n, B, D, H, W);
  auto gfeat = at::empty({n, c}, grad.options());
  // Gather form when its row buffer (one row per grid cell) is no larger than
  // grad_feats itself; the scatter form needs no buffer.
  size_t rows_bytes = 0;
  check(bfb_bev_pool_backward_workspace_size(n, c, B, D, H, W, dtype_code(grad), &rows_bytes),
        "bev_pool backward workspace");
  if (n > 0 && rows_bytes <= (size_t)gfeat.numel() * gfeat.element_size()) {
    auto rows = at::empty({(int64_t)rows_bytes}, grad.options().dtype(at::kByte));
    check(bfb_bev_pool_backward_gather(grad.data_ptr(), dtype_code(grad), n, c, B, D, H, W, plan.data_ptr(),
                                       (size_t)plan.numel(), gfeat.data_ptr(), rows.data_ptr(), rows_bytes,
                                       stream_of(grad)),
          "bev_pool backward");
  } else {
    check(bfb_bev_pool_backward(grad.data_ptr(), dtype_code(grad), n, c, B, D, H, W, plan.data_ptr(),
                                (size_t)plan.numel(), gfeat.data_ptr(), stream_of(grad)),
          "bev_pool backward");
  }
  return gfeat;
}

at::Tensor bev_pool_plan_cells(const at::Tensor& plan, int64_t n, int64_t B, int64_t D, int64_t H, int64_t W) {
  NvtxRange nvtx_("bfb_b200::bev_pool_plan_cells");
  require_cuda(plan, "plan");
  c10::cuda::CUDAGuard guard(plan.device());
  check_plan(plan, n, B, D, H, W);
  auto cells = at::empty({n}, plan.options().dtype(at::kLong));
  check(bfb_bev_pool_plan_cells(plan.data_ptr(), (size_t)plan.numel(), n, B, D, H, W, cells.data_ptr<int64_t>(),
                                stream_of(plan)),
        "bev_pool plan cells");
  return cells;
}

bool bev_pool_plan_check(const at::Tensor& plan, int64_t n, int64_t B, int64_t D, int64_t H, int64_t W) {
  NvtxRange nvtx_("bfb_b200::bev_pool_plan_check");
  require_cuda(plan, "plan");
  c10::cuda::CUDAGuard guard(plan.device());
  const int s = bfb_bev_pool_plan_check(plan.data_ptr(), n, B, D, H, W, stream_of(plan));
  if (s == BFB_ERR_PLAN_MISMATCH) return false;
  check(s, "bev_pool plan check");
  return true;
}

int64_t bev_pool_invalid_count(const at::Tensor& plan) {
  NvtxRange nvtx_("bfb_b200::bev_pool_invalid_count");
  c10::cuda::CUDAGuard guard(plan.device());
  int64_t v = 0;
  check(bfb_bev_pool_invalid_count(plan.data_ptr(), &v, stream_of(plan)), "bev_pool invalid count");
  return v;
}

// ------------------------------------------------- fused depth x context pooling
std::tuple<at::Tensor, at::Tensor> bev_pool_dc_forward(const at::Tensor& depth_in, const at::Tensor& ctx_in,
                                                       const at::Tensor& coords_in, int64_t B, int64_t D, int64_t H,
                                                       int64_t W) {
  NvtxRange nvtx_("bfb_b200::bev_pool_dc_forward");
  require_cuda(depth_in, "depth");
  require_cuda(ctx_in, "context");
  require_cuda(coords_in, "coords");
  c10::cuda::CUDAGuard guard(depth_in.device());
  TORCH_CHECK_TYPE(depth_in.scalar_type() == at::kFloat && ctx_in.scalar_type() == at::kFloat,
                   "depth and context must be float32");
  TORCH_CHECK_VALUE(depth_in.dim() == 4 && ctx_in.dim() == 4, "depth [cams, D, fH, fW] and context [cams, C, fH, fW]");
  auto depth = depth_in.contiguous();
  auto ctx = ctx_in.contiguous();
  auto coords = coords_in.contiguous();
  const int64_t cams = depth.size(0), nd = depth.size(1), fh = depth.size(2), fw = depth.size(3), c = ctx.size(1);
  TORCH_CHECK_VALUE(ctx.size(0) == cams && ctx.size(2) == fh && ctx.size(3) == fw, "context does not match depth");
  TORCH_CHECK_VALUE(coords.dim() == 2 && coords.size(0) == cams * nd * fh * fw && coords.size(1) == 4,
                    "coords must hold one (x, y, z, b) row per frustum point");
  const int itype = coords.scalar_type() == at::kLong ? BFB_I64 : BFB_I32;
  size_t plan_b = 0, scr_b = 0, aux_b = 0, bwd_b = 0;
  check(bfb_bev_pool_dc_workspace_sizes(cams, nd, fh, fw, c, B, D, H, W, &plan_b, &scr_b, &aux_b, &bwd_b),
        "bev_pool_dc workspace query");
  auto opts = depth.options().dtype(at::kByte);
  auto plan = at::empty({(int64_t)plan_b}, opts);
  auto scratch = at::empty({(int64_t)scr_b}, opts);
  auto aux = at::empty({(int64_t)aux_b}, opts);
  auto out = at::empty({B, c, D, H, W}, depth.options());
  check(bfb_bev_pool_dc_forward(depth.data_ptr<float>(), ctx.data_ptr<float>(), coords.data_ptr(), itype, cams, nd, fh,
                                fw, c, B, D, H, W, out.data_ptr<float>(), plan.data_ptr(), plan_b, scratch.data_ptr(),
                                scr_b, aux.data_ptr(), aux_b, stream_of(depth)),
        "bev_pool_dc forward");
  return {out, aux};
}

std::tuple<at::Tensor, at::Tensor> bev_pool_dc_forward_planned(const at::Tensor& depth_in, const at::Tensor& ctx_in,
                                                               const at::Tensor& plan, int64_t B, int64_t D, int64_t H,
                                                               int64_t W) {
  NvtxRange nvtx_("bfb_b200::bev_pool_dc_forward_planned");
  require_cuda(depth_in, "depth");
  require_cuda(ctx_in, "context");
  require_cuda(plan, "plan");
  c10::cuda::CUDAGuard guard(depth_in.device());
  TORCH_CHECK_TYPE(depth_in.scalar_type() == at::kFloat && ctx_in.scalar_type() == at::kFloat,
                   "depth and context must be float32");
  TORCH_CHECK_VALUE(depth_in.dim() == 4 && ctx_in.dim() == 4, "depth [cams, D, fH, fW] and context [cams, C, fH, fW]");
  auto depth = depth_in.contiguous();
  auto ctx = ctx_in.contiguous();
  const int64_t cams = depth.size(0), nd = depth.size(1), fh = depth.size(2), fw = depth.size(3), c = ctx.size(1);
  TORCH_CHECK_VALUE(ctx.size(0) == cams && ctx.size(2) == fh && ctx.size(3) == fw, "context does not match depth");
  check_plan(plan, cams * nd * fh * fw, B, D, H, W);
  size_t plan_b = 0, scr_b = 0, aux_b = 0;
  check(bfb_bev_pool_dc_workspace_sizes(cams, nd, fh, fw, c, B, D, H, W, &plan_b, &scr_b, &aux_b, nullptr),
        "bev_pool_dc workspace query");
  auto opts = depth.options().dtype(at::kByte);
  auto scratch = at::empty({(int64_t)scr_b}, opts);
  auto aux = at::empty({(int64_t)aux_b}, opts);
  auto out = at::empty({B, c, D, H, W}, depth.options());
  check(bfb_bev_pool_dc_forward_planned(depth.data_ptr<float>(), ctx.data_ptr<float>(), cams, nd, fh, fw, c, B, D, H,
                                        W, plan.data_ptr(), (size_t)plan.numel(), out.data_ptr<float>(),
                                        scratch.data_ptr(), scr_b, aux.data_ptr(), aux_b, stream_of(depth)),
        "bev_pool_dc forward");
  return {out, aux};
}

at::Tensor bev_pool_geometry_plan(const at::Tensor& frustum_in, const at::Tensor& post_rots_in,
                                  const at::Tensor& post_trans_in, const at::Tensor& combine_in,
                                  const at::Tensor& trans_in, const std::optional<at::Tensor>& extra_rots_in,
                                  const std::optional<at::Tensor>& extra_trans_in, at::ArrayRef<double> lower,
                                  at::ArrayRef<double> dx, int64_t D, int64_t H, int64_t W) {
  NvtxRange nvtx_("bfb_b200::bev_pool_geometry_plan");
  require_cuda(frustum_in, "frustum");
  c10::cuda::CUDAGuard guard(frustum_in.device());
  auto f32 = [](const at::Tensor& t) { return t.contiguous().to(at::kFloat); };
  auto frustum = f32(frustum_in);
  auto post_rots = f32(post_rots_in), post_trans = f32(post_trans_in);
  auto combine = f32(combine_in), trans = f32(trans_in);
  TORCH_CHECK_VALUE(frustum.dim() == 4 && frustum.size(3) == 3, "frustum must be [D, fH, fW, 3]");
  TORCH_CHECK_VALUE(post_rots.dim() == 4 && post_rots.size(2) == 3 && post_rots.size(3) == 3,
                    "post_rots must be [B, N, 3, 3]");
  const int64_t B = post_rots.size(0), ncam = post_rots.size(1);
  TORCH_CHECK_VALUE(combine.sizes() == post_rots.sizes(), "combine must be [B, N, 3, 3]");
  TORCH_CHECK_VALUE(post_trans.dim() == 3 && post_trans.size(0) == B && post_trans.size(1) == ncam &&
                        post_trans.size(2) == 3 && trans.sizes() == post_trans.sizes(),
                    "post_trans and camera2lidar_trans must be [B, N, 3]");
  TORCH_CHECK_VALUE(lower.size() == 3 && dx.size() == 3, "lower and dx need 3 values");
  at::Tensor er, et;
  if (extra_rots_in.has_value()) {
    er = f32(*extra_rots_in);
    TORCH_CHECK_VALUE(er.dim() == 3 && er.size(0) == B && er.size(1) == 3 && er.size(2) == 3,
                      "extra_rots must be [B, 3, 3]");
  }
  if (extra_trans_in.has_value()) {
    et = f32(*extra_trans_in);
    TORCH_CHECK_VALUE(et.dim() == 2 && et.size(0) == B && et.size(1) == 3, "extra_trans must be [B, 3]");
  }
  const int64_t nd = frustum.size(0), fh = frustum.size(1), fw = frustum.size(2);
  const int64_t n = B * ncam * nd * fh * fw;
  size_t plan_b = 0, scratch_b = 0;
  check(bfb_bev_pool_workspace_sizes(n, 1, B, D, H, W, &plan_b, &scratch_b), "bev_pool workspace query");
  auto opts = frustum.options().dtype(at::kByte);
  auto plan = at::empty({(int64_t)plan_b}, opts);
  auto scratch = at::empty({(int64_t)scratch_b}, opts);
  const float lo[3] = {(float)lower[0], (float)lower[1], (float)lower[2]};
  const float d3[3] = {(float)dx[0], (float)dx[1], (float)dx[2]};
  check(bfb_bev_pool_geometry_plan(frustum.data_ptr<float>(), nd, fh, fw, post_rots.data_ptr<float>(),
                                   post_trans.data_ptr<float>(), combine.data_ptr<float>(), trans.data_ptr<float>(),
                                   er.defined() ? er.data_ptr<float>() : nullptr,
                                   et.defined() ? et.data_ptr<float>() : nullptr, B, ncam, lo, d3, D, H, W,
                                   plan.data_ptr(), plan_b, scratch.data_ptr(), scratch_b, stream_of(frustum)),
        "bev_pool geometry plan");
  return plan;
}

std::tuple<at::Tensor, at::Tensor> bev_pool_dc_backward(const at::Tensor& grad_in, const at::Tensor& depth_in,
                                                        const at::Tensor& coords_in, const at::Tensor& aux,
                                                        int64_t c, int64_t B, int64_t D, int64_t H, int64_t W) {
  NvtxRange nvtx_("bfb_b200::bev_pool_dc_backward");
  require_cuda(grad_in, "grad_out");
  c10::cuda::CUDAGuard guard(grad_in.device());
  auto grad = grad_in.contiguous().to(at::kFloat);
  auto depth = depth_in.contiguous();
  auto coords = coords_in.contiguous();
  const int64_t cams = depth.size(0), nd = depth.size(1), fh = depth.size(2), fw = depth.size(3);
  const int itype = coords.scalar_type() == at::kLong ? BFB_I64 : BFB_I32;
  size_t bwd_b = 0;
  check(bfb_bev_pool_dc_workspace_sizes(cams, nd, fh, fw, c, B, D, H, W, nullptr, nullptr, nullptr, &bwd_b),
        "bev_pool_dc workspace query");
  auto ws = at::empty({(int64_t)bwd_b}, depth.options().dtype(at::kByte));
  auto gdepth = at::empty_like(depth);
  auto gctx = at::empty({cams, c, fh, fw}, depth.options());
  check(bfb_bev_pool_dc_backward(grad.data_ptr<float>(), depth.data_ptr<float>(), coords.data_ptr(), itype, cams, nd,
                                 fh, fw, c, B, D, H, W, aux.data_ptr(), (size_t)aux.numel(), ws.data_ptr(), bwd_b,
                                 gdepth.data_ptr<float>(), gctx.data_ptr<float>(), stream_of(grad)),
        "bev_pool_dc backward");
  return {gdepth, gctx};
}

// ------------------------------------------------------------ voxelisation
std::vector<float> as_floats(const c10::ArrayRef<double>& v, size_t n, const char* what) {
  TORCH_CHECK_VALUE(v.size() == n, what, " must have length ", n);
  std::vector<float> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = (float)v[i];
  return out;
}

// One hash table per (device, stream), initialised once and left clean by
// every successful call; dropped (and re-initialised next time) after a
// failure.
struct TableCache {
  std::mutex mu;
  std::map<std::pair<int, int64_t>, at::Tensor> tables;
};
TableCache& table_cache() {
  static TableCache c;
  return c;
}

at::Tensor table_for(const at::Tensor& like, size_t bytes, void* stream) {
  auto key = std::make_pair((int)like.device().index(), (int64_t)reinterpret_cast<intptr_t>(stream));
  auto& c = table_cache();
  std::lock_guard<std::mutex> g(c.mu);
  auto it = c.tables.find(key);
  if (it != c.tables.end() && (size_t)it->second.numel() >= bytes) return it->second;
  auto t = at::empty({(int64_t)bytes}, like.options().dtype(at::kByte));
  check(bfb_hard_voxelize_table_init(t.data_ptr(), bytes, stream), "voxel table init");
  c.tables[key] = t;
  return t;
}

void drop_table(const at::Tensor& like, void* stream) {
  auto& c = table_cache();
  std::lock_guard<std::mutex> g(c.mu);
  c.tables.erase(std::make_pair((int)like.device().index(), (int64_t)reinterpret_cast<intptr_t>(stream)));
}

void require_contig(const at::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.is_contiguous(), name, " must be contiguous");
}

void dynamic_voxelize(const at::Tensor& points_in, at::Tensor& coors, c10::ArrayRef<double> voxel_size,
                      c10::ArrayRef<double> coors_range) {
  NvtxRange nvtx_("bfb_b200::dynamic_voxelize");
  require_cuda(points_in, "points");
  require_cuda(coors, "coors");
  c10::cuda::CUDAGuard guard(points_in.device());
  auto points = points_in.contiguous();
  TORCH_CHECK_VALUE(points.dim() == 2 && points.size(1) >= 3, "points must have shape [N, >=3]");
  TORCH_CHECK_TYPE(coors.scalar_type() == at::kInt, "coors must be int32");
  TORCH_CHECK_VALUE(coors.dim() == 2 && coors.size(0) == points.size(0) && coors.size(1) == 3,
                    "coors must have shape [N, 3]");
  auto vs = as_floats(voxel_size, 3, "voxel_size");
  auto cr = as_floats(coors_range, 6, "coors_range");
  at::Tensor out = coors.is_contiguous() ? coors : at::empty_like(coors, at::MemoryFormat::Contiguous);
  check(bfb_dynamic_voxelize(points.data_ptr(), dtype_code(points), points.size(0), points.size(1), vs.data(),
                             cr.data(), out.data_ptr<int32_t>(), stream_of(points)),
        "dynamic_voxelize");
  if (!coors.is_contiguous()) coors.copy_(out);
}

void hard_voxelize_batch(const at::Tensor& points_in, c10::ArrayRef<int64_t> offsets, at::Tensor& voxels,
                         at::Tensor& coors, at::Tensor& num_points, at::Tensor& voxel_num,
                         c10::ArrayRef<double> voxel_size, c10::ArrayRef<double> coors_range, int64_t max_points,
                         int64_t max_voxels, bool zero_tail) {
  NvtxRange nvtx_("bfb_b200::hard_voxelize_batch");
  require_cuda(points_in, "points");
  c10::cuda::CUDAGuard guard(points_in.device());
  auto points = points_in.contiguous();
  TORCH_CHECK_VALUE(points.dim() == 2 && points.size(1) >= 3, "points must have shape [N, >=3]");
  for (auto* t : {&voxels, &coors, &num_points, &voxel_num}) {
    require_cuda(*t, "output");
    require_contig(*t, "outputs");
  }
  TORCH_CHECK_TYPE(voxels.scalar_type() == points.scalar_type(), "voxels must have the dtype of points");
  TORCH_CHECK_TYPE(coors.scalar_type() == at::kInt && num_points.scalar_type() == at::kInt &&
                       voxel_num.scalar_type() == at::kInt,
                   "coors, num_points and voxel_num must be int32");
  const int64_t n = points.size(0), f = points.size(1);
  const int64_t batch = (int64_t)offsets.size() - 1;
  TORCH_CHECK_VALUE(batch >= 1, "offsets must hold batch + 1 entries");
  const int64_t P = max_points < 0 ? n : max_points;
  const int64_t MV = max_voxels < 0 ? n : max_voxels;
  TORCH_CHECK_VALUE(voxels.numel() >= batch * MV * P * f && coors.numel() >= batch * MV * 3 &&
                        num_points.numel() >= batch * MV && voxel_num.numel() >= batch,
                    "output buffers are too small for max_voxels / max_points");
  auto vs = as_floats(voxel_size, 3, "voxel_size");
  auto cr = as_floats(coors_range, 6, "coors_range");
  size_t table_b = 0, scratch_b = 0;
  check(bfb_hard_voxelize_workspace_sizes(n, batch, max_points, &table_b, &scratch_b),
        "hard_voxelize workspace query");
  void* st = stream_of(points);
  auto table = table_for(points, table_b, st);
  auto scratch = at::empty({(int64_t)scratch_b}, points.options().dtype(at::kByte));
  const int rc = bfb_hard_voxelize_batch(points.data_ptr(), dtype_code(points), offsets.data(), batch, n, f,
                                         vs.data(), cr.data(), max_points, max_voxels, voxels.data_ptr(),
                                         coors.data_ptr<int32_t>(), num_points.data_ptr<int32_t>(),
                                         voxel_num.data_ptr<int32_t>(), zero_tail ? 1 : 0, table.data_ptr(),
                                         (size_t)table.numel(), scratch.data_ptr(), scratch_b, st);
  if (rc != BFB_OK) drop_table(points, st);
  check(rc, "hard_voxelize");
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> voxelize_mean_epilogue(const at::Tensor& voxels,
                                                                                  const at::Tensor& coors,
                                                                                  const at::Tensor& num_points,
                                                                                  const at::Tensor& voxel_num) {
  NvtxRange nvtx_("bfb_b200::voxelize_mean_epilogue");
  require_cuda(voxels, "voxels");
  c10::cuda::CUDAGuard guard(voxels.device());
  TORCH_CHECK_VALUE(voxels.dim() == 4, "voxels must be [batch, max_voxels, max_points, F]");
  const int64_t B = voxels.size(0), MV = voxels.size(1), P = voxels.size(2), F = voxels.size(3);
  TORCH_CHECK_VALUE(coors.dim() == 3 && coors.size(0) == B && coors.size(1) == MV && coors.size(2) == 3,
                    "coors must be [batch, max_voxels, 3]");
  TORCH_CHECK_VALUE(num_points.dim() == 2 && num_points.size(0) == B && num_points.size(1) == MV,
                    "num_points must be [batch, max_voxels]");
  TORCH_CHECK_VALUE(voxel_num.numel() == B, "voxel_num must hold batch counts");
  for (auto* t : {&voxels, &coors, &num_points, &voxel_num}) require_contig(*t, "epilogue inputs");
  TORCH_CHECK_TYPE(coors.scalar_type() == at::kInt && num_points.scalar_type() == at::kInt &&
                       voxel_num.scalar_type() == at::kInt,
                   "coors, num_points and voxel_num must be int32");
  auto feats = at::empty({B * MV, F}, voxels.options());
  auto coords = at::empty({B * MV, 4}, coors.options());
  auto sizes = at::empty({B * MV}, coors.options());
  auto total = at::empty({1}, coors.options());
  check(bfb_voxelize_mean_epilogue(voxels.data_ptr(), dtype_code(voxels), coors.data_ptr<int32_t>(),
                                   num_points.data_ptr<int32_t>(), voxel_num.data_ptr<int32_t>(), B, MV, P, F,
                                   feats.data_ptr(), coords.data_ptr<int32_t>(), sizes.data_ptr<int32_t>(),
                                   total.data_ptr<int32_t>(), stream_of(voxels)),
        "voxelize mean epilogue");
  return {feats, coords, sizes, total};
}

int64_t hard_voxelize(const at::Tensor& points, at::Tensor& voxels, at::Tensor& coors, at::Tensor& num_points,
                      c10::ArrayRef<double> voxel_size, c10::ArrayRef<double> coors_range, int64_t max_points,
                      int64_t max_voxels, bool zero_tail) {
  NvtxRange nvtx_("bfb_b200::hard_voxelize");
  require_cuda(points, "points");
  c10::cuda::CUDAGuard guard(points.device());
  auto vn = at::empty({1}, points.options().dtype(at::kInt));
  const int64_t offs[2] = {0, points.size(0)};
  hard_voxelize_batch(points, c10::ArrayRef<int64_t>(offs, 2), voxels, coors, num_points, vn, voxel_size,
                      coors_range, max_points, max_voxels, zero_tail);
  return vn.item<int32_t>();  // the reference API returns a Python int
}

// ------------------------------------------------------------ dynamic scatter
int reduce_code(c10::string_view r) {
  if (r == "sum" || r == "none") return 0;
  if (r == "mean") return 1;
  if (r == "max") return 2;
  TORCH_CHECK_VALUE(false, "Unsupported reduce_type: ", r);
  return -1;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> dynamic_scatter_forward(const at::Tensor& feats_in,
                                                                                   const at::Tensor& coors_in,
                                                                                   c10::string_view reduce,
                                                                                   at::OptionalIntArrayRef extents) {
  NvtxRange nvtx_("bfb_b200::dynamic_scatter_forward");
  require_cuda(feats_in, "feats");
  require_cuda(coors_in, "coors");
  c10::cuda::CUDAGuard guard(feats_in.device());
  auto feats = feats_in.contiguous();
  auto coors = coors_in.to(at::kInt).contiguous();
  const int64_t n = feats.size(0), c = feats.size(1), ndim = coors.size(1);
  const int r = reduce_code(reduce);
  size_t wb = 0;
  check(bfb_dynamic_scatter_workspace_size(n, c, ndim, &wb), "dynamic_scatter workspace query");
  auto ws = at::empty({(int64_t)wb}, feats.options().dtype(at::kByte));
  auto out = at::empty({n, c}, feats.options());
  auto oc = at::empty({n, ndim}, coors.options());
  auto map = at::empty({n}, coors.options());
  auto cnt = at::empty({n}, coors.options());
  int64_t m = 0;
  if (extents.has_value())
    TORCH_CHECK_VALUE((int64_t)extents->size() == ndim, "extents must give one value per coordinate column");
  const int64_t* ext = extents.has_value() ? extents->data() : nullptr;
  const int st = bfb_dynamic_scatter_forward(feats.data_ptr(), dtype_code(feats), coors.data_ptr<int32_t>(), n, c, ndim, r,
                                    ext, out.data_ptr(), oc.data_ptr<int32_t>(), map.data_ptr<int32_t>(),
                                    cnt.data_ptr<int32_t>(), &m, ws.data_ptr(), wb, stream_of(feats));
  TORCH_CHECK_VALUE(st != BFB_ERR_DEVICE_STATUS, "dynamic_scatter: a coordinate lies beyond the given extents");
  check(st, "dynamic_scatter forward");
  return {out.narrow(0, 0, m), oc.narrow(0, 0, m), map, cnt.narrow(0, 0, m)};
}

void dynamic_scatter_backward(at::Tensor& grad_feats, const at::Tensor& grad_out_in, const at::Tensor& feats_in,
                              const at::Tensor& reduced_in, const at::Tensor& map_in, const at::Tensor& counts_in,
                              c10::string_view reduce) {
  NvtxRange nvtx_("bfb_b200::dynamic_scatter_backward");
  require_cuda(grad_feats, "grad_feats");
  c10::cuda::CUDAGuard guard(grad_feats.device());
  require_contig(grad_feats, "grad_feats");
  auto gout = grad_out_in.contiguous();
  auto feats = feats_in.contiguous();
  auto reduced = reduced_in.to(feats.scalar_type()).contiguous();
  auto map = map_in.to(at::kInt).contiguous();
  auto counts = counts_in.to(at::kInt).contiguous();
  TORCH_CHECK_TYPE(gout.scalar_type() == grad_feats.scalar_type() && feats.scalar_type() == grad_feats.scalar_type(),
                   "grad_feats, grad_out and feats must share a dtype");
  const int64_t n = feats.size(0), c = feats.size(1), m = reduced.size(0);
  const int r = reduce_code(reduce);
  at::Tensor from;
  if (r == 2) from = at::empty({std::max<int64_t>(m * c, 1)}, map.options());
  check(bfb_dynamic_scatter_backward(grad_feats.data_ptr(), gout.data_ptr(), feats.data_ptr(), reduced.data_ptr(),
                                     map.data_ptr<int32_t>(), counts.data_ptr<int32_t>(), dtype_code(feats), n, m, c, r,
                                     r == 2 ? from.data_ptr<int32_t>() : nullptr,
                                     r == 2 ? sizeof(int32_t) * (size_t)from.numel() : 0, stream_of(feats)),
        "dynamic_scatter backward");
}

}  // namespace

// ------------------------------------------------- sparse-convolution rulebook
std::tuple<at::Tensor, at::Tensor, at::Tensor> get_indice_pairs(const at::Tensor& indices_in, int64_t batch,
                                                                at::IntArrayRef out_shape, at::IntArrayRef ksize,
                                                                at::IntArrayRef stride, at::IntArrayRef padding,
                                                                at::IntArrayRef dilation, bool subm, bool transpose) {
  NvtxRange nvtx_("bfb_b200::get_indice_pairs");
  require_cuda(indices_in, "indices");
  c10::cuda::CUDAGuard guard(indices_in.device());
  auto indices = indices_in.contiguous().to(at::kInt);
  TORCH_CHECK_VALUE(indices.dim() == 2 && indices.size(1) >= 2, "indices must be [N, ndim + 1]");
  const int64_t n = indices.size(0);
  const int ndim = (int)indices.size(1) - 1;
  TORCH_CHECK_VALUE((int64_t)out_shape.size() == ndim && (int64_t)ksize.size() == ndim &&
                        (int64_t)stride.size() == ndim && (int64_t)padding.size() == ndim &&
                        (int64_t)dilation.size() == ndim,
                    "every convolution parameter needs ndim values");
  int64_t K = 1;
  for (auto k : ksize) K *= k;
  size_t ws_b = 0;
  check(bfb_indice_pairs_workspace_size(n, ndim, batch, out_shape.data(), ksize.data(), subm ? 1 : 0, &ws_b),
        "indice pairs workspace query");
  auto opts = indices.options();
  auto ws = at::empty({(int64_t)ws_b}, opts.dtype(at::kByte));
  auto pairs = at::empty({K, 2, n}, opts);
  auto num = at::empty({K}, opts);
  auto nout = at::empty({1}, opts);
  check(bfb_get_indice_pairs(indices.data_ptr<int32_t>(), n, ndim, batch, out_shape.data(), ksize.data(),
                             stride.data(), padding.data(), dilation.data(), subm ? 1 : 0, transpose ? 1 : 0,
                             pairs.data_ptr<int32_t>(), num.data_ptr<int32_t>(), nout.data_ptr<int32_t>(),
                             ws.data_ptr(), ws_b, stream_of(indices)),
        "get_indice_pairs");
  if (subm) return {indices, pairs, num};
  const int64_t u = nout.item<int32_t>();  // one host sync, as the reference's
  auto outids = at::empty({u, ndim + 1}, opts);
  check(bfb_indice_pairs_outids(n, ndim, batch, out_shape.data(), ksize.data(), ws.data_ptr(), ws_b,
                                outids.data_ptr<int32_t>(), stream_of(indices)),
        "get_indice_pairs outids");
  return {outids, pairs, num};
}

// ------------------------------------------------------ sparse convolution
namespace {

struct Rulebook {
  at::Tensor pairs, num;
  int64_t K, cap;
};

Rulebook rulebook_of(const at::Tensor& pairs_in, const at::Tensor& num_in, const at::Tensor& like) {
  require_cuda(pairs_in, "indice_pairs");
  require_cuda(num_in, "indice_pair_num");
  TORCH_CHECK_VALUE(pairs_in.dim() == 3 && pairs_in.size(1) == 2, "indice_pairs must be [K, 2, N]");
  TORCH_CHECK_VALUE(num_in.numel() == pairs_in.size(0), "indice_pair_num must hold K counts");
  TORCH_CHECK(pairs_in.device() == like.device() && num_in.device() == like.device(),
              "features and the rulebook must be on one device");
  return {pairs_in.to(at::kInt).contiguous(), num_in.to(at::kInt).contiguous(), pairs_in.size(0), pairs_in.size(2)};
}

// filters [*ksize, Cin, Cout] viewed [K, Cin, Cout]
at::Tensor filters_of(const at::Tensor& filters, const at::Tensor& feats, int64_t* K, int64_t* cout) {
  require_cuda(filters, "filters");
  TORCH_CHECK_VALUE(filters.dim() >= 2 && filters.size(-2) == feats.size(1),
                    "filters must be [..., Cin, Cout] with Cin = features.size(1)");
  TORCH_CHECK_TYPE(filters.scalar_type() == feats.scalar_type(), "filters must have the dtype of features");
  *cout = filters.size(-1);
  *K = filters.numel() / std::max<int64_t>(1, feats.size(1) * *cout);
  return filters.contiguous();
}

}  // namespace

at::Tensor indice_conv(const at::Tensor& features_in, const at::Tensor& filters_in, const at::Tensor& indice_pairs,
                       const at::Tensor& indice_pair_num, int64_t num_activate_out, bool inverse,
                       const c10::optional<at::Tensor>& bias_in) {
  NvtxRange nvtx_("bfb_b200::indice_conv");
  require_cuda(features_in, "features");
  c10::cuda::CUDAGuard guard(features_in.device());
  TORCH_CHECK_VALUE(features_in.dim() == 2, "features must be [N, Cin]");
  auto feats = features_in.contiguous();
  int64_t K = 0, cout = 0;
  auto filters = filters_of(filters_in, feats, &K, &cout);
  auto rb = rulebook_of(indice_pairs, indice_pair_num, feats);
  TORCH_CHECK_VALUE(rb.K == K, "indice_pairs has ", rb.K, " rules, the filters ", K, " offsets");
  at::Tensor bias;
  if (bias_in.has_value() && bias_in->defined()) {
    bias = bias_in->to(feats.scalar_type()).contiguous();
    require_cuda(bias, "bias");
    TORCH_CHECK_VALUE(bias.numel() == cout, "bias must hold Cout values");
  }
  const int dt = dtype_code(feats);
  size_t ws_b = 0;
  check(bfb_indice_conv_workspace_size(feats.size(0), num_activate_out, K, feats.size(1), cout, rb.cap, dt, 0, &ws_b),
        "indice_conv workspace query");
  auto ws = at::empty({(int64_t)ws_b}, feats.options().dtype(at::kByte));
  auto out = at::empty({num_activate_out, cout}, feats.options());
  check(bfb_indice_conv(feats.data_ptr(), dt, feats.size(0), feats.size(1), filters.data_ptr(), K, cout,
                        rb.pairs.data_ptr<int32_t>(), rb.cap, rb.num.data_ptr<int32_t>(), num_activate_out,
                        inverse ? 1 : 0, bias.defined() ? bias.data_ptr() : nullptr, out.data_ptr(), ws.data_ptr(),
                        ws_b, stream_of(feats)),
        "indice_conv");
  return out;
}

std::tuple<at::Tensor, at::Tensor> indice_conv_backward(const at::Tensor& features_in, const at::Tensor& filters_in,
                                                        const at::Tensor& out_bp_in, const at::Tensor& indice_pairs,
                                                        const at::Tensor& indice_pair_num, bool inverse) {
  NvtxRange nvtx_("bfb_b200::indice_conv_backward");
  require_cuda(features_in, "features");
  require_cuda(out_bp_in, "out_bp");
  c10::cuda::CUDAGuard guard(features_in.device());
  TORCH_CHECK_VALUE(features_in.dim() == 2 && out_bp_in.dim() == 2, "features and out_bp must be 2-D");
  auto feats = features_in.contiguous();
  int64_t K = 0, cout = 0;
  auto filters = filters_of(filters_in, feats, &K, &cout);
  auto gout = out_bp_in.to(feats.scalar_type()).contiguous();
  TORCH_CHECK_VALUE(gout.size(1) == cout, "out_bp must be [num_out, Cout]");
  auto rb = rulebook_of(indice_pairs, indice_pair_num, feats);
  TORCH_CHECK_VALUE(rb.K == K, "indice_pairs has ", rb.K, " rules, the filters ", K, " offsets");
  const int dt = dtype_code(feats);
  size_t ws_b = 0;
  check(bfb_indice_conv_workspace_size(feats.size(0), gout.size(0), K, feats.size(1), cout, rb.cap, dt, 1, &ws_b),
        "indice_conv_backward workspace query");
  auto ws = at::empty({(int64_t)ws_b}, feats.options().dtype(at::kByte));
  auto gin = at::empty_like(feats);
  auto gw = at::empty_like(filters);
  check(bfb_indice_conv_backward(feats.data_ptr(), dt, feats.size(0), feats.size(1), filters.data_ptr(), K, cout,
                                 gout.data_ptr(), gout.size(0), rb.pairs.data_ptr<int32_t>(), rb.cap,
                                 rb.num.data_ptr<int32_t>(), inverse ? 1 : 0, gin.data_ptr(), gw.data_ptr(),
                                 ws.data_ptr(), ws_b, stream_of(feats)),
        "indice_conv_backward");
  return {gin, gw};
}

at::Tensor indice_maxpool(const at::Tensor& features_in, const at::Tensor& indice_pairs,
                          const at::Tensor& indice_pair_num, int64_t num_activate_out) {
  NvtxRange nvtx_("bfb_b200::indice_maxpool");
  require_cuda(features_in, "features");
  c10::cuda::CUDAGuard guard(features_in.device());
  TORCH_CHECK_VALUE(features_in.dim() == 2, "features must be [N, C]");
  auto feats = features_in.contiguous();
  auto rb = rulebook_of(indice_pairs, indice_pair_num, feats);
  size_t ws_b = 0;
  check(bfb_indice_maxpool_workspace_size(feats.size(0), num_activate_out, rb.K, 0, &ws_b),
        "indice_maxpool workspace query");
  auto ws = at::empty({std::max<int64_t>((int64_t)ws_b, 1)}, feats.options().dtype(at::kByte));
  auto out = at::empty({num_activate_out, feats.size(1)}, feats.options());
  check(bfb_indice_maxpool(feats.data_ptr(), dtype_code(feats), feats.size(0), feats.size(1),
                           rb.pairs.data_ptr<int32_t>(), rb.K, rb.cap, rb.num.data_ptr<int32_t>(), num_activate_out,
                           out.data_ptr(), ws.data_ptr(), ws_b, stream_of(feats)),
        "indice_maxpool");
  return out;
}

at::Tensor indice_maxpool_backward(const at::Tensor& features_in, const at::Tensor& out_features_in,
                                   const at::Tensor& out_bp_in, const at::Tensor& indice_pairs,
                                   const at::Tensor& indice_pair_num) {
  NvtxRange nvtx_("bfb_b200::indice_maxpool_backward");
  require_cuda(features_in, "features");
  require_cuda(out_features_in, "out_features");
  require_cuda(out_bp_in, "out_bp");
  c10::cuda::CUDAGuard guard(features_in.device());
  auto feats = features_in.contiguous();
  auto y = out_features_in.to(feats.scalar_type()).contiguous();
  auto gy = out_bp_in.to(feats.scalar_type()).contiguous();
  TORCH_CHECK_VALUE(feats.dim() == 2 && y.dim() == 2 && y.sizes() == gy.sizes() && y.size(1) == feats.size(1),
                    "features [N, C], out_features and out_bp [M, C]");
  auto rb = rulebook_of(indice_pairs, indice_pair_num, feats);
  size_t ws_b = 0;
  check(bfb_indice_maxpool_workspace_size(feats.size(0), y.size(0), rb.K, 1, &ws_b),
        "indice_maxpool_backward workspace query");
  auto ws = at::empty({std::max<int64_t>((int64_t)ws_b, 1)}, feats.options().dtype(at::kByte));
  auto gx = at::empty_like(feats);
  check(bfb_indice_maxpool_backward(feats.data_ptr(), y.data_ptr(), gy.data_ptr(), dtype_code(feats), feats.size(0),
                                    y.size(0), feats.size(1), rb.pairs.data_ptr<int32_t>(), rb.K, rb.cap,
                                    rb.num.data_ptr<int32_t>(), gx.data_ptr(), ws.data_ptr(), ws_b,
                                    stream_of(feats)),
        "indice_maxpool_backward");
  return gx;
}

TORCH_LIBRARY(bfb_b200, m) {
  m.def("bev_pool_forward(Tensor feats, Tensor coords, int B, int D, int H, int W) -> (Tensor, Tensor)");
  m.def("bev_pool_plan(Tensor coords, int B, int D, int H, int W) -> Tensor");
  m.def("bev_pool_forward_planned(Tensor feats, Tensor plan, int B, int D, int H, int W) -> Tensor");
  m.def("bev_pool_backward(Tensor grad_out, Tensor plan, int n, int B, int D, int H, int W) -> Tensor");
  m.def("bev_pool_invalid_count(Tensor plan) -> int");
  m.def("bev_pool_plan_check(Tensor plan, int n, int B, int D, int H, int W) -> bool");
  m.def("bev_pool_plan_cells(Tensor plan, int n, int B, int D, int H, int W) -> Tensor");
  m.def("bev_pool_dc_forward(Tensor depth, Tensor context, Tensor coords, int B, int D, int H, int W) -> (Tensor, Tensor)");
  m.def("bev_pool_dc_forward_planned(Tensor depth, Tensor context, Tensor plan, int B, int D, int H, int W) -> (Tensor, Tensor)");
  m.def(
      "bev_pool_geometry_plan(Tensor frustum, Tensor post_rots, Tensor post_trans, Tensor combine, Tensor trans, "
      "Tensor? extra_rots, Tensor? extra_trans, float[] lower, float[] dx, int D, int H, int W) -> Tensor");
  m.def(
      "bev_pool_dc_backward(Tensor grad_out, Tensor depth, Tensor coords, Tensor aux, int C, int B, int D, int H, "
      "int W) -> (Tensor, Tensor)");
  m.def("dynamic_voxelize(Tensor points, Tensor(a!) coors, float[] voxel_size, float[] coors_range) -> ()");
  m.def(
      "hard_voxelize(Tensor points, Tensor(a!) voxels, Tensor(b!) coors, Tensor(c!) num_points, "
      "float[] voxel_size, float[] coors_range, int max_points, int max_voxels, bool zero_tail) -> int");
  m.def(
      "hard_voxelize_batch(Tensor points, int[] offsets, Tensor(a!) voxels, Tensor(b!) coors, "
      "Tensor(c!) num_points, Tensor(d!) voxel_num, float[] voxel_size, float[] coors_range, int max_points, "
      "int max_voxels, bool zero_tail) -> ()");
  m.def(
      "voxelize_mean_epilogue(Tensor voxels, Tensor coors, Tensor num_points, Tensor voxel_num) -> (Tensor, Tensor, "
      "Tensor, Tensor)");
  m.def(
      "get_indice_pairs(Tensor indices, int batch, int[] out_shape, int[] ksize, int[] stride, int[] padding, "
      "int[] dilation, bool subm, bool transpose) -> (Tensor, Tensor, Tensor)");
  m.def(
      "dynamic_scatter_forward(Tensor feats, Tensor coors, str reduce, int[]? extents=None) -> (Tensor, Tensor, "
      "Tensor, Tensor)");
  m.def(
      "dynamic_scatter_backward(Tensor(a!) grad_feats, Tensor grad_out, Tensor feats, Tensor reduced, Tensor map, "
      "Tensor counts, str reduce) -> ()");
  m.def(
      "indice_conv(Tensor features, Tensor filters, Tensor indice_pairs, Tensor indice_pair_num, "
      "int num_activate_out, bool inverse=False, Tensor? bias=None) -> Tensor");
  m.def(
      "indice_conv_backward(Tensor features, Tensor filters, Tensor out_bp, Tensor indice_pairs, "
      "Tensor indice_pair_num, bool inverse=False) -> (Tensor, Tensor)");
  m.def("indice_maxpool(Tensor features, Tensor indice_pairs, Tensor indice_pair_num, int num_activate_out) -> Tensor");
  m.def(
      "indice_maxpool_backward(Tensor features, Tensor out_features, Tensor out_bp, Tensor indice_pairs, "
      "Tensor indice_pair_num) -> Tensor");
}

TORCH_LIBRARY_IMPL(bfb_b200, CUDA, m) {
  m.impl("bev_pool_forward", &bev_pool_forward);
  m.impl("bev_pool_plan", &bev_pool_plan);
  m.impl("bev_pool_forward_planned", &bev_pool_forward_planned);
  m.impl("bev_pool_backward", &bev_pool_backward);
  m.impl("bev_pool_invalid_count", &bev_pool_invalid_count);
  m.impl("bev_pool_plan_check", &bev_pool_plan_check);
  m.impl("bev_pool_plan_cells", &bev_pool_plan_cells);
  m.impl("bev_pool_dc_forward", &bev_pool_dc_forward);
  m.impl("bev_pool_dc_forward_planned", &bev_pool_dc_forward_planned);
  m.impl("bev_pool_geometry_plan", &bev_pool_geometry_plan);
  m.impl("bev_pool_dc_backward", &bev_pool_dc_backward);
  m.impl("dynamic_voxelize", &dynamic_voxelize);
  m.impl("hard_voxelize", &hard_voxelize);
  m.impl("hard_voxelize_batch", &hard_voxelize_batch);
  m.impl("voxelize_mean_epilogue", &voxelize_mean_epilogue);
  m.impl("dynamic_scatter_forward", &dynamic_scatter_forward);
  m.impl("get_indice_pairs", &get_indice_pairs);
  m.impl("dynamic_scatter_backward", &dynamic_scatter_backward);
  m.impl("indice_conv", &indice_conv);
  m.impl("indice_conv_backward", &indice_conv_backward);
  m.impl("indice_maxpool", &indice_maxpool);
  m.impl("indice_maxpool_backward", &indice_maxpool_backward);
}
