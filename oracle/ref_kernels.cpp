// Runs the reference's own Metal kernels on the host CPU.
//
// Test infrastructure only (never linked into the product). Each reference
// kernel source under <reference>/fastgs_core/metal/ is included verbatim from
// the read-only reference tree (the build passes -DFGS_REF_DIR) inside its own
// namespace, on top of the host stand-in for metal_stdlib in ref_shim/. The
// extern "C" runners below play the role of the reference's dispatch code:
//   preprocess forward   fastgs_core/fastgs_preprocess.cpp:113-168
//   duplicate with keys  fastgs_core/fastgs_binning.cpp:62-105
//   tile ranges/buckets  fastgs_core/fastgs_tile_prep.cpp:47-98
//   render forward       fastgs_core/fastgs_rasterize.cpp:90-168
//   render backward      fastgs_core/fastgs_rasterize_backward.cpp:85-166
//   preprocess backward  fastgs_core/fastgs_preprocess_backward.cpp:89-183
// Outputs must be zero-filled by the caller, as the reference's eval_gpu does
// with memset before every dispatch.
#include <metal_stdlib>

#define FGS_STR2(x) #x
#define FGS_STR(x) FGS_STR2(x)

namespace metal {
ShimGroup* g_shim_group = nullptr;
int g_shim_lane = 0;
}  // namespace metal

#include <functional>
#include <memory>

namespace {
// Runs `lane_fn(lane)` for n lanes of one threadgroup as coroutines: every
// round resumes each unfinished lane once, in lane order, until all returned.
struct LaneRunner {
  static constexpr size_t kStack = 256 * 1024;
  static void entry(int lo, int hi) {
    LaneRunner* self = reinterpret_cast<LaneRunner*>((uintptr_t(uint32_t(hi)) << 32) | uint32_t(lo));
    const int lane = metal::g_shim_lane;
    self->fn(lane);
    self->done[lane] = 1;
    swapcontext(&self->grp->lanes[lane], &self->grp->sched);
  }
  std::function<void(int)> fn;
  metal::ShimGroup* grp;
  std::vector<char> done;
  void run(int n, std::function<void(int)> f) {
    fn = std::move(f);
    auto g = std::make_unique<metal::ShimGroup>();
    grp = g.get();
    std::vector<ucontext_t> lanes(n);
    std::vector<int> counts(n, 0);
    std::vector<std::unique_ptr<char[]>> stacks(n);
    g->lanes = lanes.data();
    g->shuffle_count = counts.data();
    g->n = n;
    done.assign(n, 0);
    const uintptr_t me = reinterpret_cast<uintptr_t>(this);
    for (int l = 0; l < n; ++l) {
      stacks[l].reset(new char[kStack]);
      getcontext(&lanes[l]);
      lanes[l].uc_stack.ss_sp = stacks[l].get();
      lanes[l].uc_stack.ss_size = kStack;
      lanes[l].uc_link = nullptr;
      makecontext(&lanes[l], (void (*)())entry, 2, int(uint32_t(me)), int(uint32_t(me >> 32)));
    }
    metal::g_shim_group = grp;
    for (;;) {
      bool any = false;
      for (int l = 0; l < n; ++l) {
        if (done[l]) continue;
        any = true;
        metal::g_shim_lane = l;
        swapcontext(&g->sched, &lanes[l]);
      }
      if (!any) break;
    }
  }
};
}  // namespace

namespace ref_pre {
#include FGS_STR(FGS_REF_DIR/fastgs_preprocess.metal)
}
namespace ref_bin {
#include FGS_STR(FGS_REF_DIR/fastgs_binning.metal)
}
namespace ref_tile {
#include FGS_STR(FGS_REF_DIR/fastgs_tile_prep.metal)
}
namespace ref_fwd {
#include FGS_STR(FGS_REF_DIR/fastgs_rasterize.metal)
}
namespace ref_bwd {
#include FGS_STR(FGS_REF_DIR/fastgs_rasterize_backward.metal)
}
namespace ref_pbwd {
#include FGS_STR(FGS_REF_DIR/fastgs_preprocess_backward.metal)
}

using metal::uint;

extern "C" {

// Mirrors fastgs_preprocess.cpp:113-130 (focal = W / (2 tan_fovx)).
void ref_preprocess_forward(int n, int degree, int max_sh_coeffs, float scale_modifier, float mult,
                            float tan_fovx, float tan_fovy, int image_width, int image_height,
                            int prefiltered, int use_cov3d_precomp, int use_colors_precomp,
                            const float* means3d, const float* dc, const float* shs,
                            const float* colors_precomp, const float* opacities,
                            const float* scales, const float* rotations,
                            const float* cov3d_precomp, const float* viewmatrix,
                            const float* projmatrix, const float* cam_pos,
                            const float* viewspace_in, int* radii, float* xys, float* depths,
                            float* cov3ds, float* rgb, float* conic_opacity,
                            uint32_t* tiles_touched, bool* clamped, float* viewspace_out) {
  ref_pre::PreprocessKernelParams p;
  p.degree = degree;
  p.max_sh_coeffs = max_sh_coeffs;
  p.scale_modifier = scale_modifier;
  p.mult = mult;
  p.tan_fovx = tan_fovx;
  p.tan_fovy = tan_fovy;
  p.focal_x = static_cast<float>(image_width) / (2.0f * tan_fovx);
  p.focal_y = static_cast<float>(image_height) / (2.0f * tan_fovy);
  p.image_width = (uint)image_width;
  p.image_height = (uint)image_height;
  p.tile_bounds_x = (uint)((image_width + 15) / 16);
  p.tile_bounds_y = (uint)((image_height + 15) / 16);
  p.tile_bounds_z = 1;
  p.prefiltered = (uint)prefiltered;
  p.use_cov3d_precomp = (uint)use_cov3d_precomp;
  p.use_colors_precomp = (uint)use_colors_precomp;
  for (int t = 0; t < n; ++t) {
    ref_pre::fastgs_preprocess_forward_kernel(
        n, p, means3d, dc, shs, colors_precomp, opacities, scales, rotations, cov3d_precomp,
        viewmatrix, projmatrix, cam_pos, viewspace_in, radii, xys, depths, cov3ds, rgb,
        conic_opacity, tiles_touched, clamped, viewspace_out, (uint)t);
  }
}

void ref_duplicate_with_keys(int n, float mult, int tile_bounds_x, int tile_bounds_y,
                             float* xys, float* depths, uint32_t* point_offsets,
                             float* conic_opacity, uint32_t* tiles_touched, uint64_t* keys,
                             uint32_t* values) {
  ref_bin::BinningKernelParams p;
  p.mult = mult;
  p.tile_bounds_x = (uint)tile_bounds_x;
  p.tile_bounds_y = (uint)tile_bounds_y;
  p.tile_bounds_z = 1;
  for (int t = 0; t < n; ++t) {
    ref_bin::fastgs_duplicate_with_keys_kernel(n, p, xys, depths, point_offsets, conic_opacity,
                                               tiles_touched, keys, values,
                                               metal::uint3((uint)t, 0, 0));
  }
}

void ref_tile_prep(int num_rendered, int num_tiles, uint64_t* keys, uint32_t* ranges,
                   uint32_t* bucket_count) {
  ref_tile::TilePrepKernelParams p;
  p.num_rendered = (uint)num_rendered;
  p.num_tiles = (uint)num_tiles;
  for (int g = 0; g < num_rendered; ++g)
    ref_tile::fastgs_identify_tile_ranges_kernel(p, keys, ranges, (uint)g);
  for (int g = 0; g < num_tiles; ++g)
    ref_tile::fastgs_per_tile_bucket_count_kernel(p, ranges, bucket_count, (uint)g);
}

// One 16x16 threadgroup per tile: 256 coroutine lanes (see LaneRunner).
void ref_render_forward(int image_width, int image_height, int num_tiles, int bucket_sum,
                        int get_flag, uint32_t* ranges, uint32_t* point_list,
                        uint32_t* bucket_offsets, float* means2d, float* colors,
                        float* conic_opacity, float* background, int* radii, int* metric_map,
                        uint32_t* bucket_to_tile, float* sampled_t, float* sampled_ar,
                        float* final_t, uint32_t* n_contrib, uint32_t* max_contrib,
                        float* pixel_colors, float* out_color, int* metric_count) {
  ref_fwd::RasterizeKernelParams p;
  p.image_width = (uint)image_width;
  p.image_height = (uint)image_height;
  p.block_x = 16;
  p.block_y = 16;
  p.num_channels = 3;
  p.num_tiles = (uint)num_tiles;
  p.bucket_sum = (uint)bucket_sum;
  p.get_flag = (uint)get_flag;
  const uint gx = (uint)((image_width + 15) / 16), gy = (uint)((image_height + 15) / 16);
  for (uint ty = 0; ty < gy; ++ty) {
    for (uint tx = 0; tx < gx; ++tx) {
      LaneRunner r;
      r.run(256, [&](int l) {
        const uint lx = uint(l) % 16, ly = uint(l) / 16;
        ref_fwd::fastgs_render_forward_kernel(
            p, ranges, point_list, bucket_offsets, means2d, colors, conic_opacity, background,
            radii, metric_map, bucket_to_tile, sampled_t, sampled_ar, final_t, n_contrib,
            max_contrib, pixel_colors, out_color, metric_count, metal::uint2(lx, ly),
            metal::uint2(tx * 16 + lx, ty * 16 + ly), metal::uint2(tx, ty));
      });
    }
  }
}

// One 32-lane simdgroup per bucket: 32 coroutine lanes (see LaneRunner).
void ref_render_backward(int image_width, int image_height, int num_tiles, int bucket_sum,
                         const uint32_t* ranges, const uint32_t* point_list,
                         const uint32_t* bucket_offsets, const float* means2d,
                         const float* colors, const float* conic_opacity,
                         const float* background, const float* dL_dout_color,
                         const uint32_t* bucket_to_tile, const float* sampled_t,
                         const float* sampled_ar, const float* final_t,
                         const uint32_t* n_contrib, const uint32_t* max_contrib,
                         const float* pixel_colors, float* dL_dmeans2d, float* dL_dcolors,
                         float* dL_dconic_opacity, float* dL_dviewspace) {
  ref_bwd::RasterizeBackwardKernelParams p;
  p.image_width = (uint)image_width;
  p.image_height = (uint)image_height;
  p.block_x = 16;
  p.block_y = 16;
  p.num_channels = 3;
  p.num_tiles = (uint)(num_tiles > 1 ? num_tiles : 1);
  p.bucket_sum = (uint)bucket_sum;
  p.block_size = 256;
  for (int b = 0; b < bucket_sum; ++b) {
    LaneRunner r;
    r.run(32, [&](int lane) {
      ref_bwd::fastgs_render_backward_kernel(
          p, ranges, point_list, bucket_offsets, means2d, colors, conic_opacity, background,
          dL_dout_color, bucket_to_tile, sampled_t, sampled_ar, final_t, n_contrib, max_contrib,
          pixel_colors, (metal::atomic_float*)dL_dmeans2d, (metal::atomic_float*)dL_dcolors,
          (metal::atomic_float*)dL_dconic_opacity, (metal::atomic_float*)dL_dviewspace,
          uint(lane), uint(lane), metal::uint3((uint)b, 0, 0), 32u);
    });
  }
}

// Mirrors fastgs_preprocess_backward.cpp:133-146 (focal uses max(tan, 1e-6)).
void ref_preprocess_backward(int n, int image_width, int image_height, int use_cov3d_precomp,
                             int use_colors_precomp, float scale_modifier, float tan_fovx,
                             float tan_fovy, int degree, int max_sh_coeffs, const float* means3d,
                             const float* scales, const float* quats, const float* viewmat,
                             const float* projmat, const float* cam_pos, const float* sh,
                             const float* cov3d_precomp, const float* cov3d_fwd,
                             const float* dL_dcov3d, const float* dL_drgb, const float* dL_dxys,
                             const float* dL_ddepths, const float* dL_dconic_opacity,
                             const float* dL_dviewspace_out, const int* radii,
                             const bool* clamped, float* dL_dmeans3d, float* dL_ddc,
                             float* dL_dsh, float* dL_dcolors_precomp, float* dL_dopacities,
                             float* dL_dscales, float* dL_dquats, float* dL_dviewspace_in) {
  ref_pbwd::PreprocessBackwardKernelParams p;
  p.n = (uint)n;
  p.image_width = (uint)image_width;
  p.image_height = (uint)image_height;
  p.use_cov3d_precomp = (uint)use_cov3d_precomp;
  p.use_colors_precomp = (uint)use_colors_precomp;
  p.scale_modifier = scale_modifier;
  p.tan_fovx = tan_fovx;
  p.tan_fovy = tan_fovy;
  p.focal_x = 0.5f * static_cast<float>(image_width) / std::max(tan_fovx, 1e-6f);
  p.focal_y = 0.5f * static_cast<float>(image_height) / std::max(tan_fovy, 1e-6f);
  p.degree = degree;
  p.max_sh_coeffs = max_sh_coeffs;
  for (int t = 0; t < n; ++t) {
    ref_pbwd::fastgs_preprocess_backward_kernel(
        p, means3d, scales, quats, viewmat, projmat, cam_pos, sh, cov3d_precomp, cov3d_fwd,
        dL_dcov3d, dL_drgb, dL_dxys, dL_ddepths, dL_dconic_opacity, dL_dviewspace_out, radii,
        clamped, dL_dmeans3d, dL_ddc, dL_dsh, dL_dcolors_precomp, dL_dopacities, dL_dscales,
        dL_dquats, dL_dviewspace_in, (uint)t);
  }
}

}  // extern "C"
