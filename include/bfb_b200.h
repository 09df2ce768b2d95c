/*
 * bfb_b200.h -- C ABI of the B200 (sm_100a) grid scatter-reduce hot path of
 * BEVFusion: LSS camera->BEV pooling (bev_pool, forward + backward), LiDAR
 * hard / dynamic voxelisation and dynamic scatter.
 *
 * Conventions
 *  - Every pointer argument named *_dev is CUDA device memory; nothing here
 *    allocates device memory.  Callers size workspaces with the *_sizes()
 *    queries and pass them in.  Outputs are caller-allocated.
 *  - Every entry point is asynchronous on `stream` (a cudaStream_t passed as
 *    void*, NULL = legacy default stream) unless documented otherwise, and
 *    returns a bfb_status (0 = success).  No C++ exception crosses the ABI and
 *    no kernel traps: device-side problems (out-of-range coordinates, full
 *    hash tables) are counted into status words that the host reads on
 *    request.
 *  - Element types are given as bfb_dtype / bfb_itype codes.
 *
 * Each declaration cites the reference interface it replaces, by path within
 * the ziyangyeh/bevfusion-triton project.
 */
#ifndef BFB_B200_H_
#define BFB_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BFB_ABI_VERSION 2

typedef enum bfb_dtype {
  BFB_F32 = 0,
  BFB_F16 = 1,
  BFB_BF16 = 2,
} bfb_dtype;

typedef enum bfb_itype {
  BFB_I32 = 0,
  BFB_I64 = 1,
} bfb_itype;

typedef enum bfb_status {
  BFB_OK = 0,
  BFB_ERR_INVALID_ARG = -1,       /* bad shape, size, pointer or enum */
  BFB_ERR_UNSUPPORTED_DTYPE = -2, /* dtype code not accepted by this op */
  BFB_ERR_WORKSPACE = -3,         /* workspace NULL or smaller than required */
  BFB_ERR_TOO_LARGE = -4,         /* sizes exceed the 32-bit index space */
  BFB_ERR_CUDA = -5,              /* a CUDA runtime call or launch failed */
  BFB_ERR_DEVICE_STATUS = -6,     /* device-side check failed (see op doc) */
  BFB_ERR_PLAN_MISMATCH = -7,     /* a bev_pool plan used with another geometry */
} bfb_status;

/* Library ABI version (BFB_ABI_VERSION of the build). */
int bfb_abi_version(void);
/* Static description of a status code. */
const char* bfb_status_string(int status);
/* Text of the last CUDA error seen by this thread inside the library. */
const char* bfb_last_cuda_error(void);
/* Number of kernels this library has launched in this process (all threads). */
uint64_t bfb_kernel_launches(void);

/* Debugging aids (no reference counterpart; the reference has no
 * diagnostics on this path).
 *
 * A debug build (`python -m bevfusion_triton_b200._build --debug-checks`,
 * which compiles with -DBFB_DEBUG_CHECKS into bevfusion_triton_b200/debug/)
 * checks indices the kernels take from plans and workspaces (permutation
 * entries, cell ranks, member slots, voxel and pair slots) and counts each
 * violation into a device error word instead of trapping, skipping the
 * access.  bfb_debug_checks_enabled() says which build is loaded;
 * bfb_debug_violations() reads (and optionally clears) the summed error word
 * of the current device, synchronously; bfb_debug_selftest(k) counts k
 * synthetic violations (0 in a release build).
 *
 * bfb_debug_inject_status(status, calls): the next `calls` calls of the main
 * entry points (plans, forwards, backwards, voxelisation, scatter, rulebook)
 * return `status` at once, without touching their arguments -- host-side
 * fault injection for testing error paths; status 0 disarms. */
int bfb_debug_checks_enabled(void);
int bfb_debug_violations(uint64_t* count, int reset);
int bfb_debug_selftest(int k, void* stream);
int bfb_debug_inject_status(int status, int calls);

/* ------------------------------------------------------------------------
 * bev_pool: out[b, c, z, x, y] = sum_{n : coords[n] = (x, y, z, b)} feats[n, c]
 *
 * Replaces ops/bev_pool/src/bev_pool_triton.py:219-227 (`bev_pool`), its
 * autograd pair :153-216, and the legacy extension entry points
 * ops/bev_pool/csrc/bev_pool_cpu.cpp:89-94 (`bev_pool_forward`,
 * `bev_pool_backward`).
 *
 * feats [n, c] row-major (f32 / f16 / bf16), coords [n, 4] row-major int32
 * or int64 with columns (x, y, z, b), 0 <= x < H, 0 <= y < W, 0 <= z < D,
 * 0 <= b < B.  out [B, c, D, H, W] contiguous, same dtype as feats; every
 * element is written (empty cells get 0), so `out` needs no zero-fill.
 * Points whose coordinates fall outside the grid are dropped and counted
 * (bfb_bev_pool_invalid_count); the reference CPU path raises for them.
 *
 * Within a cell, values are summed in fp32 in ascending point order
 * (the order of torch.index_add_ in the reference CPU path), so results are
 * bitwise deterministic run to run.
 *
 * The plan (sorted cell ranks, point permutation and work list) is written by
 * bfb_bev_pool_plan / bfb_bev_pool_forward into `plan_dev` and reused by
 * bfb_bev_pool_forward_planned and bfb_bev_pool_backward, so keep it alive
 * between the forward and the backward.  `scratch_dev` is only used during
 * the call.
 *
 * A plan records the geometry (n, B, D, H, W) it was built for.  Every call
 * that reads a plan compares it with its own arguments on the device: on a
 * mismatch the call's kernels write no output and read nothing past the plan
 * header, and they raise a flag in the header.  bfb_bev_pool_plan_check
 * reads that state (synchronously) and returns BFB_ERR_PLAN_MISMATCH.
 * ---------------------------------------------------------------------- */
int bfb_bev_pool_workspace_sizes(int64_t n, int64_t c, int64_t B, int64_t D, int64_t H,
                                 int64_t W, size_t* plan_bytes, size_t* scratch_bytes);

int bfb_bev_pool_plan(const void* coords_dev, int coords_itype, int64_t n, int64_t B, int64_t D,
                      int64_t H, int64_t W, void* plan_dev, size_t plan_bytes, void* scratch_dev,
                      size_t scratch_bytes, void* stream);

int bfb_bev_pool_forward_planned(const void* feats_dev, int feats_dtype, int64_t n, int64_t c,
                                 int64_t B, int64_t D, int64_t H, int64_t W, const void* plan_dev,
                                 size_t plan_bytes, void* out_dev, void* stream);

int bfb_bev_pool_forward(const void* feats_dev, int feats_dtype, const void* coords_dev,
                         int coords_itype, int64_t n, int64_t c, int64_t B, int64_t D, int64_t H,
                         int64_t W, void* out_dev, void* plan_dev, size_t plan_bytes,
                         void* scratch_dev, size_t scratch_bytes, void* stream);

/* grad_feats[n, :] = grad_out[b, :, z, x, y] for every in-grid point, 0 for
 * dropped points.  grad_out [B, c, D, H, W] contiguous, same dtype as
 * grad_feats. */
int bfb_bev_pool_backward(const void* grad_out_dev, int dtype, int64_t n, int64_t c, int64_t B,
                          int64_t D, int64_t H, int64_t W, const void* plan_dev,
                          size_t plan_bytes, void* grad_feats_dev, void* stream);

/* The same backward in gather form: grad_out rows of the non-empty cells are
 * first copied into `workspace_dev` (one row of c elements per grid cell,
 * B*D*H*W*c*sizeof(dtype) bytes, from bfb_bev_pool_backward_workspace_size),
 * then grad_feats is written in point order as one contiguous stream.  Same
 * result as bfb_bev_pool_backward, bit for bit; faster when the row buffer is
 * small next to grad_feats (dense point clouds such as the LSS frustum). */
int bfb_bev_pool_backward_workspace_size(int64_t n, int64_t c, int64_t B, int64_t D, int64_t H,
                                         int64_t W, int dtype, size_t* bytes);

int bfb_bev_pool_backward_gather(const void* grad_out_dev, int dtype, int64_t n, int64_t c,
                                 int64_t B, int64_t D, int64_t H, int64_t W, const void* plan_dev,
                                 size_t plan_bytes, void* grad_feats_dev, void* workspace_dev,
                                 size_t workspace_bytes, void* stream);

/* Fused camera branch: bev_pool of feats[n, c] = depth[n] * context[cam, c, h, w]
 * without materialising feats.  Replaces models/vtransforms/depth_lss.py:91-94
 * (softmax(depth) (x) context) followed by models/vtransforms/base.py:136-160
 * (flatten, filter, ops.bev_pool).  depth [cams, nd, fh, fw] fp32 (already
 * softmaxed), context [cams, c, fh, fw] fp32, coords [cams*nd*fh*fw, 4] for
 * EVERY frustum point in (cam, d, h, w) order (points outside the grid are
 * dropped, which is the caller's filter), c % 4 == 0 and c <= 128.  The
 * forward equals bfb_bev_pool_forward on the materialised product bit for bit.
 * `aux` (cams*fh*fw*c floats + one cell per frustum point, from *_sizes) is
 * written by the forward and read by the backward; `bwd` is the backward's
 * scratch.  grad_depth has the layout of depth, grad_context that of
 * context. */
int bfb_bev_pool_dc_workspace_sizes(int64_t cams, int64_t nd, int64_t fh, int64_t fw, int64_t c,
                                    int64_t B, int64_t D, int64_t H, int64_t W, size_t* plan_bytes,
                                    size_t* scratch_bytes, size_t* aux_bytes, size_t* bwd_bytes);

int bfb_bev_pool_dc_forward(const float* depth_dev, const float* context_dev,
                            const void* coords_dev, int coords_itype, int64_t cams, int64_t nd,
                            int64_t fh, int64_t fw, int64_t c, int64_t B, int64_t D, int64_t H,
                            int64_t W, float* out_dev, void* plan_dev, size_t plan_bytes,
                            void* scratch_dev, size_t scratch_bytes, void* aux_dev,
                            size_t aux_bytes, void* stream);

/* The fused forward on a plan made beforehand (bfb_bev_pool_plan over the
 * frustum points' coords, or bfb_bev_pool_geometry_plan); bfb_bev_pool_dc_forward
 * is bfb_bev_pool_plan followed by this call. */
int bfb_bev_pool_dc_forward_planned(const float* depth_dev, const float* context_dev, int64_t cams,
                                    int64_t nd, int64_t fh, int64_t fw, int64_t c, int64_t B,
                                    int64_t D, int64_t H, int64_t W, const void* plan_dev,
                                    size_t plan_bytes, float* out_dev, void* scratch_dev,
                                    size_t scratch_bytes, void* aux_dev, size_t aux_bytes,
                                    void* stream);

/* coords_dev / coords_itype are not read (the forward left every point's cell
 * in aux) and may be NULL / 0. */
int bfb_bev_pool_dc_backward(const float* grad_out_dev, const float* depth_dev,
                             const void* coords_dev, int coords_itype, int64_t cams, int64_t nd,
                             int64_t fh, int64_t fw, int64_t c, int64_t B, int64_t D, int64_t H,
                             int64_t W, const void* aux_dev, size_t aux_bytes, void* bwd_dev,
                             size_t bwd_bytes, float* grad_depth_dev, float* grad_context_dev,
                             void* stream);

/* bev_pool plan straight from the camera parameters: the frustum geometry of
 * models/vtransforms/base.py:82-126 (get_geometry) and the quantise + in-grid
 * filter of base.py:131-158 (BaseTransform.bev_pool) for every frustum point,
 * without a coordinate tensor.  The plan covers all B*ncam*nd*fh*fw frustum
 * points in (b, cam, d, h, w) order; points outside the grid are dropped, so
 * bfb_bev_pool_forward_planned takes the UNFILTERED [B*ncam*nd*fh*fw, c]
 * features (no boolean-mask gather) and bfb_bev_pool_dc_forward_planned takes
 * depth / context directly.  frustum [nd, fh, fw, 3] (u, v, depth);
 * post_rots, combine [B*ncam, 3, 3]; post_trans, trans [B*ncam, 3]; combine =
 * camera2lidar_rots @ intrins^-1 as the reference forms it (linalg.solve);
 * extra_rots [B, 3, 3] and extra_trans [B, 3] may be NULL.  lower[3] = bx -
 * dx / 2 and dx[3] are HOST arrays (x, y, z); the grid is D = nz, H = nx,
 * W = ny cells.  Each row of a 3x3 product is fma(a1, p1, a0*p0) + a2*p2,
 * which matches torch's CUDA matmul of these shapes on all but a few values
 * in a million; a point lying within rounding of a cell edge can therefore
 * still quantise into the neighbouring cell.
 * Workspace sizes: bfb_bev_pool_workspace_sizes(B*ncam*nd*fh*fw, c, B, D, H, W). */
/* The cell rank ((b*D + z)*H + x)*W + y the plan gave every point, in input
 * order, or -1 for a dropped point: cells [n] int64. */
int bfb_bev_pool_plan_cells(const void* plan_dev, size_t plan_bytes, int64_t n, int64_t B, int64_t D,
                            int64_t H, int64_t W, int64_t* cells_dev, void* stream);

int bfb_bev_pool_geometry_plan(const float* frustum_dev, int64_t nd, int64_t fh, int64_t fw,
                               const float* post_rots_dev, const float* post_trans_dev,
                               const float* combine_dev, const float* trans_dev,
                               const float* extra_rots_dev, const float* extra_trans_dev,
                               int64_t B, int64_t ncam, const float* lower, const float* dx,
                               int64_t D, int64_t H, int64_t W, void* plan_dev, size_t plan_bytes,
                               void* scratch_dev, size_t scratch_bytes, void* stream);

/* bev_pool forward that allocates nothing and takes no workspace.  It has no
 * counterpart in the reference.  It is for callers that cannot allocate GPU
 * memory at call time -- code in a real-time loop where cudaMalloc would
 * stall, or code that may not own an allocator -- and uses one fixed 64 MiB
 * device array inside this library instead (held on every GPU that loads the
 * library, until exit; bfb_bev_pool_noalloc_capacity() returns its size).
 * Sizes whose plan + scratch exceed it are refused with BFB_ERR_TOO_LARGE
 * (one det sample of 1.77 M points on a 360 x 360 grid fits).  The first call
 * on a device looks up the array's device address, so make it before any
 * stream capture.  All calls share the array: calls that overlap on the GPU
 * (other streams, other threads) race, and the plan is not kept for a
 * backward. */
int bfb_bev_pool_forward_noalloc(const void* feats_dev, int feats_dtype, const void* coords_dev,
                                 int coords_itype, int64_t n, int64_t c, int64_t B, int64_t D,
                                 int64_t H, int64_t W, void* out_dev, void* stream);
size_t bfb_bev_pool_noalloc_capacity(void);

/* Synchronously checks that `plan_dev` was built for (n, B, D, H, W) and that
 * no call has been handed it with another geometry since: BFB_OK, or
 * BFB_ERR_PLAN_MISMATCH.  No reference counterpart (the reference keeps no
 * plan between calls). */
int bfb_bev_pool_plan_check(const void* plan_dev, int64_t n, int64_t B, int64_t D, int64_t H,
                            int64_t W, void* stream);

/* Synchronously reads how many points the plan dropped as out of range. */
int bfb_bev_pool_invalid_count(const void* plan_dev, int64_t* count, void* stream);

/* ------------------------------------------------------------------------
 * Voxelisation.
 *
 * voxel_size[3] = (vx, vy, vz), coors_range[6] = (xmin, ymin, zmin, xmax,
 * ymax, zmax); the grid is round((max - min) / size) per axis, computed in
 * double as the reference does (ops/voxel/src/voxelization_triton.py:23-39).
 * A point's cell is floor((p - min) / size) in IEEE fp32.
 * ---------------------------------------------------------------------- */

/* coors[n, 3] int32 = (cx, cy, cz) per point, or (-1, -1, -1) when the point
 * is outside the grid.  Replaces ops/voxel/voxel_layer.py:33-36 ->
 * ops/voxel/src/voxelization_triton.py:428-463 (`dynamic_voxelize`) and the
 * legacy ops/voxel/csrc/voxelization.h:115-130. */
int bfb_dynamic_voxelize(const void* points_dev, int points_dtype, int64_t n, int64_t f,
                         const float* voxel_size, const float* coors_range, int32_t* coors_dev,
                         void* stream);

/* Hard voxelisation, first-occurrence order.  Replaces
 * ops/voxel/voxel_layer.py:27-30 -> ops/voxel/src/voxelization_triton.py:674-710
 * (`hard_voxelize`) and the legacy ops/voxel/csrc/voxelization.h:86-113.
 *
 * Voxel ids follow the first in-range point of each voxel; at most
 * max_voxels voxels are created (points of later new voxels are dropped) and
 * each voxel keeps its first max_points points in input order
 * (max_points = -1: no per-voxel limit, the voxels buffer then holds n slots
 * per voxel; max_voxels = -1: no voxel limit, the buffers then hold n
 * voxels).  Outputs: voxels [max_voxels, max_points, f] (dtype of points),
 * coors [max_voxels, 3] int32 (x, y, z), num_points [max_voxels] int32,
 * voxel_num [1] int32 (device).  Rows [0, voxel_num) are written in full
 * (unused point slots are 0); rows [voxel_num, max_voxels) are zero-filled
 * only when zero_tail != 0.  The `deterministic` flag of the reference is
 * accepted by the Python layer and always served by this deterministic
 * kernel.
 *
 * Workspaces: `table` is a hash table that must be initialised once with
 * bfb_hard_voxelize_table_init; every successful call leaves it clean, so it
 * can be reused call after call (re-initialise it after a failed call).  Its
 * capacity (from table_bytes) must be at least twice the point count of a
 * call.  `scratch` is only used during the call; its size depends on
 * max_points (1 <= max_points <= 64 selects a four-launch pipeline whose
 * member table keeps each voxel's max_points smallest point indices; other
 * values use a general bucket pipeline). */
int bfb_hard_voxelize_workspace_sizes(int64_t n, int64_t batch, int64_t max_points,
                                      size_t* table_bytes, size_t* scratch_bytes);

int bfb_hard_voxelize_table_init(void* table_dev, size_t table_bytes, void* stream);

int bfb_hard_voxelize(const void* points_dev, int points_dtype, int64_t n, int64_t f,
                      const float* voxel_size, const float* coors_range, int64_t max_points,
                      int64_t max_voxels, void* voxels_dev, int32_t* coors_dev,
                      int32_t* num_points_dev, int32_t* voxel_num_dev, int zero_tail,
                      void* table_dev, size_t table_bytes, void* scratch_dev, size_t scratch_bytes,
                      void* stream);

/* Batched hard voxelisation of `batch` independent samples in one set of
 * launches.  It has no single reference counterpart: it replaces the
 * per-sample loop of models/fusion_models/bevfusion.py:269-296 over
 * `Voxelization.forward`.  Sample s owns points [offsets[s], offsets[s+1])
 * (offsets: int64 [batch + 1], HOST memory, offsets[0] = 0,
 * offsets[batch] = n) and the output slices voxels[s] =
 * [max_voxels, max_points, f], coors[s] = [max_voxels, 3],
 * num_points[s] = [max_voxels]; voxel_num_dev holds [batch] counts. */
int bfb_hard_voxelize_batch(const void* points_dev, int points_dtype, const int64_t* offsets,
                            int64_t batch, int64_t n, int64_t f, const float* voxel_size,
                            const float* coors_range, int64_t max_points, int64_t max_voxels,
                            void* voxels_dev, int32_t* coors_dev, int32_t* num_points_dev,
                            int32_t* voxel_num_dev, int zero_tail, void* table_dev,
                            size_t table_bytes, void* scratch_dev, size_t scratch_bytes,
                            void* stream);

/* Mean epilogue of a batched voxelisation, one launch.  Replaces the loop of
 * models/fusion_models/bevfusion.py:269-296 after the per-sample
 * voxelisation: the rows [0, voxel_num[s]) of every sample s of the outputs
 * of bfb_hard_voxelize_batch (voxels [batch, max_voxels, max_points, f],
 * coors [batch, max_voxels, 3], num_points [batch, max_voxels], voxel_num
 * [batch], all device) are packed sample after sample into out_feats [M, f]
 * (mean over the voxel's point slots: the slots are summed in slot order in
 * fp32, unused slots hold zeros, then divided by the count), out_coords
 * [M, 4] int32 = (sample, x, y, z) and out_sizes [M] int32, with M =
 * sum(voxel_num) <= batch * max_voxels (size the outputs for that); the
 * device int32 *total_dev receives M (may be NULL).  batch <= 4096. */
int bfb_voxelize_mean_epilogue(const void* voxels_dev, int dtype, const int32_t* coors_dev,
                               const int32_t* num_points_dev, const int32_t* voxel_num_dev,
                               int64_t batch, int64_t max_voxels, int64_t max_points, int64_t f,
                               void* out_feats_dev, int32_t* out_coords_dev, int32_t* out_sizes_dev,
                               int32_t* total_dev, void* stream);

/* Synchronously reads the device status of the last call that used this
 * scratch: *table_full = points whose insert found no free table slot
 * (always 0 when the table capacity rule above holds). */
int bfb_hard_voxelize_status(const void* scratch_dev, int64_t n, int64_t batch, int64_t max_points,
                             int64_t* table_full, void* stream);

/* ------------------------------------------------------------------------
 * Dynamic scatter: per-voxel reduce of point features.  Replaces
 * ops/voxel/voxel_layer.py:39-48 -> ops/voxel/src/scatter_points_triton.py:253-424
 * (`dynamic_point_to_voxel_forward` / `_backward`) and the legacy
 * ops/voxel/csrc/voxelization.h:132-140.
 *
 * Rows of coors [n, ndim] int32 with any negative entry are ignored; the
 * unique remaining rows are numbered in ascending lexicographic order.
 * reduce: 0 = sum (also the reference's 'none'), 1 = mean, 2 = max.  Outputs
 * are sized for the worst case (n voxels): out_feats [n, c] (dtype of feats),
 * out_coors [n, ndim], point2voxel [n] (-1 for ignored rows), counts [n];
 * the first *num_voxels rows are valid.  Synchronous: the voxel count is
 * returned on the host.  `extents` (HOST, ndim values, or NULL) bounds each
 * column (0 <= coors[:, d] < extents[d]): with it the row keys are packed
 * without a pass over the coordinates and one host read is saved; a valid
 * row beyond an extent makes the call return BFB_ERR_DEVICE_STATUS.  The
 * packed row key may be up to 62 bits wide (e.g. batched (b, x, y, z) rows
 * on a 1440 x 1440 x 41 grid for any batch up to 2^30).
 * ---------------------------------------------------------------------- */
int bfb_dynamic_scatter_workspace_size(int64_t n, int64_t c, int64_t ndim, size_t* bytes);

int bfb_dynamic_scatter_forward(const void* feats_dev, int dtype, const int32_t* coors_dev, int64_t n,
                                int64_t c, int64_t ndim, int reduce, const int64_t* extents,
                                void* out_feats_dev, int32_t* out_coors_dev, int32_t* point2voxel_dev,
                                int32_t* counts_dev, int64_t* num_voxels, void* ws_dev,
                                size_t ws_bytes, void* stream);

/* grad_feats [n, c] (fully written): sum copies grad_out[map], mean divides
 * it by the voxel's count, max sends each channel's gradient to the lowest
 * point index whose feature equals the reduced value (others 0).  max needs
 * argmax_ws of m * c int32. */
int bfb_dynamic_scatter_backward(void* grad_feats_dev, const void* grad_out_dev,
                                 const void* feats_dev, const void* reduced_dev,
                                 const int32_t* point2voxel_dev, const int32_t* counts_dev,
                                 int dtype, int64_t n, int64_t m, int64_t c, int reduce,
                                 int32_t* argmax_ws_dev, size_t argmax_ws_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Sparse-convolution rulebook.  Replaces get_indice_pairs
 * (ops/spconv/ops.py:53-93 -> ops/spconv/src/spconv_triton.py:792-915).
 *
 * indices [n, ndim + 1] int32 rows (b, c0, .., c{ndim-1}), 1 <= ndim <= 4;
 * out_shape, ksize, stride, padding, dilation: ndim values each (host
 * arrays; out_shape is the caller's output spatial shape, the input shape for
 * submanifold).  K = prod(ksize).  Outputs: indice_pairs [K, 2, n] int32
 * (rule k's pairs in [k, 0/1, 0 .. indice_num[k]) as (input row, output
 * row), the rest -1), indice_num [K] int32, *num_out_dev (device int32) = the
 * number of output rows.  Submanifold: the output rows are the input rows; a
 * regular or transposed rulebook numbers its output sites in ascending
 * (b, c0, .., c{ndim-1}) order (the Triton path's order) and
 * bfb_indice_pairs_outids writes them, [num_out, ndim + 1], from the same
 * workspace once the caller has read the count.  Within a rule, pairs are in
 * ascending input row.  batch * prod(out_shape) must be below 2^32.  The
 * workspace holds one bit per output grid cell for a regular rulebook.
 * ---------------------------------------------------------------------- */
int bfb_indice_pairs_workspace_size(int64_t n, int ndim, int64_t batch, const int64_t* out_shape,
                                    const int64_t* ksize, int subm, size_t* bytes);

int bfb_get_indice_pairs(const int32_t* indices_dev, int64_t n, int ndim, int64_t batch,
                         const int64_t* out_shape, const int64_t* ksize, const int64_t* stride,
                         const int64_t* padding, const int64_t* dilation, int subm, int transpose,
                         int32_t* indice_pairs_dev, int32_t* indice_num_dev, int32_t* num_out_dev,
                         void* workspace_dev, size_t workspace_bytes, void* stream);

int bfb_indice_pairs_outids(int64_t n, int ndim, int64_t batch, const int64_t* out_shape,
                            const int64_t* ksize, const void* workspace_dev, size_t workspace_bytes,
                            int32_t* outids_dev, void* stream);

/* ------------------------------------------------------------------------
 * Sparse convolution and sparse max-pooling over a rulebook.  Replace
 * indice_conv / fused_indice_conv / indice_conv_backward / indice_maxpool /
 * indice_maxpool_backward (ops/spconv/ops.py:95-188 ->
 * ops/spconv/src/spconv_triton.py:981-1111).
 *
 * features [n_in, cin]; filters [K, cin, cout] (the reference's
 * [*ksize, Cin, Cout] viewed flat), same dtype; indice_pairs [K, 2, pair_cap]
 * int32 and indice_num [K] int32 on the device, as bfb_get_indice_pairs
 * writes them: rule k's pair i joins input indice_pairs[k, s, i] to output
 * indice_pairs[k, 1 - s, i], s = inverse ? 1 : 0, for i < indice_num[k].
 * A rulebook holds at most one pair per (output, k) and per (input, k);
 * pairs naming rows outside [0, n_in) x [0, n_out) are ignored.
 *
 * out [n_out, cout] is fully written: out[o] = sum over k ascending of
 * features[in(o, k)] @ filters[k], accumulated in fp32 and rounded once, then
 * + bias (nullable; the reference's fused form rounds the sum and the biased
 * value separately, and so does this).  fp16 / bf16 with cin and cout
 * multiples of 16 (cout <= 256) run on the tensor cores; everything else
 * (fp32 included) on fp32 FMA.  K <= 343 (7x7x7), any channel count.  The workspace
 * (bfb_indice_conv_workspace_size, backward = 0 or 1) holds the neighbour
 * table and the filters in the kernels' layout.
 * ---------------------------------------------------------------------- */
int bfb_indice_conv_workspace_size(int64_t n_in, int64_t n_out, int64_t K, int64_t cin, int64_t cout,
                                   int64_t pair_cap, int dtype, int backward, size_t* bytes);

int bfb_indice_conv(const void* features_dev, int dtype, int64_t n_in, int64_t cin, const void* filters_dev,
                    int64_t K, int64_t cout, const int32_t* indice_pairs_dev, int64_t pair_cap,
                    const int32_t* indice_num_dev, int64_t n_out, int inverse, const void* bias_dev,
                    void* out_dev, void* workspace_dev, size_t workspace_bytes, void* stream);

/* input_grad [n_in, cin] = sum over k ascending of out_bp[out(i, k)] @
 * filters[k]^T (0 rows for inputs in no pair); filters_grad [K, cin, cout] =
 * sum over rule k's pairs of features[in]^T out_bp[out], in fp32, summed over
 * fixed chunks of pairs in a fixed order (deterministic). */
int bfb_indice_conv_backward(const void* features_dev, int dtype, int64_t n_in, int64_t cin,
                             const void* filters_dev, int64_t K, int64_t cout, const void* out_bp_dev,
                             int64_t n_out, const int32_t* indice_pairs_dev, int64_t pair_cap,
                             const int32_t* indice_num_dev, int inverse, void* input_grad_dev,
                             void* filters_grad_dev, void* workspace_dev, size_t workspace_bytes, void* stream);

/* Max-pooling: out [n_out, C] = max(0, max over the output's inputs) (the
 * reference pools into zeros with include_self).  Backward: input_grad
 * [n_in, C] = sum over k ascending of out_bp where features == out_features
 * (every equal maximum receives it), rounded to the dtype after each add.
 * Workspace: one int32 per (row, k) (bfb_indice_maxpool_workspace_size). */
int bfb_indice_maxpool_workspace_size(int64_t n_in, int64_t n_out, int64_t K, int backward, size_t* bytes);

int bfb_indice_maxpool(const void* features_dev, int dtype, int64_t n_in, int64_t C,
                       const int32_t* indice_pairs_dev, int64_t K, int64_t pair_cap,
                       const int32_t* indice_num_dev, int64_t n_out, void* out_dev, void* workspace_dev,
                       size_t workspace_bytes, void* stream);

int bfb_indice_maxpool_backward(const void* features_dev, const void* out_features_dev, const void* out_bp_dev,
                                int dtype, int64_t n_in, int64_t n_out, int64_t C,
                                const int32_t* indice_pairs_dev, int64_t K, int64_t pair_cap,
                                const int32_t* indice_num_dev, void* input_grad_dev, void* workspace_dev,
                                size_t workspace_bytes, void* stream);

/* Number of bounded waits in the tensor-core convolution that gave up (0 in
 * a correct run); reset = 1 clears it.  No reference counterpart. */
int bfb_spconv_timeouts(uint64_t* count, int reset);

#ifdef __cplusplus
}
#endif

#endif /* BFB_B200_H_ */
