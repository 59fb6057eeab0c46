// Tile rasterizer forward and backward on sm_100a.
//
// Forward follows fastgs_core/metal/fastgs_rasterize.metal:25-159: one CTA of
// 256 threads per 16x16 tile, one pixel per thread. Unlike the reference
// (every pixel thread gathers every Gaussian record from device memory), the
// CTA stages batches of 256 records (position, conic, opacity, colour; 36 B)
// in shared memory with one cooperative gather, so each record crosses L2
// once per tile and is then read by all 256 pixels as a shared-memory
// broadcast. The CTA leaves the splat loop as soon as every pixel has
// terminated (__syncthreads_count). Bucket samples (T and the accumulated
// colour before every 32nd splat) are written as the reference writes them,
// zeros where a pixel has terminated.
//
// Backward follows fastgs_core/metal/fastgs_rasterize_backward.metal:24-278:
// one warp per bucket of 32 consecutive splats of a tile, one splat per lane;
// the per-pixel blend state enters at lane 0 and moves one lane per step
// (__shfl_up_sync) so that, for every pixel, the 32 splats are undone front
// to back starting from the bucket's sample; per-splat partial gradients stay
// in registers and are added with one atomic per output element per bucket.
#include "../../include/fastgs_b200.h"
#include "fgs_common.cuh"

namespace fgs {

constexpr int kTile = 256;

struct FwdArgs {
  int W, H, gx, num_tiles, get_flag;
  const uint2* ranges;
  const uint32_t* point_list;
  const uint32_t* bucket_offsets;
  const float2* means2d;
  const float* colors;
  const float4* conic;
  const float* bg;
  const int32_t* metric_map;
  uint32_t* bucket_to_tile;
  float* sampled_t;
  float* sampled_ar;
  float* final_t;
  uint32_t* n_contrib;
  uint32_t* max_contrib;
  float* pixel_colors;
  float* out_color;
  int32_t* metric_count;
};

__global__ void __launch_bounds__(kTile) raster_fwd_kernel(FwdArgs a) {
  __shared__ float4 s_r0[kTile];  // x, y, conic.x, conic.y
  __shared__ float4 s_r1[kTile];  // conic.z, opacity, r, g
  __shared__ float s_c2[kTile];   // b
  __shared__ uint32_t s_id[kTile];
  __shared__ uint32_t s_wmax[kTile / 32];

  const int tile = blockIdx.x;
  const int lr = threadIdx.x;
  const int tx = tile % a.gx, ty = tile / a.gx;
  const int px = tx * FGS_BLOCK + (lr & 15), py = ty * FGS_BLOCK + (lr >> 4);
  const bool inside = px < a.W && py < a.H;
  const size_t P = (size_t)a.W * a.H;
  const size_t pix = inside ? (size_t)py * a.W + px : 0;
  const uint2 range = a.ranges[tile];
  const int to_do = (int)(range.y - range.x);
  const int nb = (to_do + 31) / 32;
  const uint32_t bbm0 = (tile == 0) ? 0u : a.bucket_offsets[tile - 1];
  for (int b = lr; b < nb; b += kTile) a.bucket_to_tile[bbm0 + b] = (uint32_t)tile;

  const float pfx = (float)px, pfy = (float)py;
  const bool count_metric = a.get_flag && inside && a.metric_map[pix] == 1;
  float T = 1.0f;
  float C0 = 0.f, C1 = 0.f, C2 = 0.f;
  uint32_t contributor = 0, last = 0;
  bool done = !inside;
  int processed = 0;
  for (int batch = 0; batch < to_do; batch += kTile) {
    if (__syncthreads_count(!done) == 0) break;
    const int j = batch + lr;
    if (j < to_do) {
      const uint32_t g = a.point_list[range.x + j];
      const float2 xy = a.means2d[g];
      const float4 co = a.conic[g];
      s_r0[lr] = make_float4(xy.x, xy.y, co.x, co.y);
      s_r1[lr] = make_float4(co.z, co.w, a.colors[3 * (size_t)g], a.colors[3 * (size_t)g + 1]);
      s_c2[lr] = a.colors[3 * (size_t)g + 2];
      s_id[lr] = g;
    }
    __syncthreads();
    const int cnt = min(kTile, to_do - batch);
    for (int k0 = 0; k0 < cnt; k0 += 32) {
      const size_t b = (size_t)bbm0 + (size_t)((batch + k0) >> 5);
      a.sampled_t[b * kTile + lr] = done ? 0.0f : T;
      float* ar = a.sampled_ar + b * 3 * kTile + lr;
      ar[0] = done ? 0.0f : C0;
      ar[kTile] = done ? 0.0f : C1;
      ar[2 * kTile] = done ? 0.0f : C2;
      if (done) continue;
      const int kend = min(k0 + 32, cnt);
      for (int k = k0; k < kend; ++k) {
        contributor++;
        const float4 r0 = s_r0[k];
        const float4 r1 = s_r1[k];
        const float dx = r0.x - pfx, dy = r0.y - pfy;
        const float power = -0.5f * (r0.z * dx * dx + r1.x * dy * dy) - r0.w * dx * dy;
        if (power > 0.0f) continue;
        const float alpha = fmin_t(0.99f, r1.y * fgs_expf(power));
        if (alpha < 1.0f / 255.0f) continue;
        const float test_t = T * (1.0f - alpha);
        if (test_t < 0.0001f) {
          done = true;
          break;
        }
        C0 += r1.z * alpha * T;
        C1 += r1.w * alpha * T;
        C2 += s_c2[k] * alpha * T;
        if (count_metric) atomicAdd(a.metric_count + s_id[k], 1);
        T = test_t;
        last = contributor;
      }
    }
    processed = batch + cnt;
    __syncthreads();
  }
  // buckets the CTA never reached (every pixel had terminated): zero samples
  for (int bl = (processed + 31) >> 5; bl < nb; ++bl) {
    const size_t b = (size_t)bbm0 + bl;
    a.sampled_t[b * kTile + lr] = 0.0f;
    float* ar = a.sampled_ar + b * 3 * kTile + lr;
    ar[0] = 0.0f;
    ar[kTile] = 0.0f;
    ar[2 * kTile] = 0.0f;
  }
  if (inside) {
    const float bg0 = a.bg[0], bg1 = a.bg[1], bg2 = a.bg[2];
    a.final_t[pix] = T;
    a.n_contrib[pix] = last;
    a.pixel_colors[pix] = C0;
    a.pixel_colors[P + pix] = C1;
    a.pixel_colors[2 * P + pix] = C2;
    a.out_color[pix] = C0 + T * bg0;
    a.out_color[P + pix] = C1 + T * bg1;
    a.out_color[2 * P + pix] = C2 + T * bg2;
  }
  const uint32_t m = __reduce_max_sync(0xffffffffu, inside ? last : 0u);
  if ((lr & 31) == 0) s_wmax[lr >> 5] = m;
  __syncthreads();
  if (lr < 32) {
    const uint32_t v = lr < kTile / 32 ? s_wmax[lr] : 0u;
    const uint32_t mm = __reduce_max_sync(0xffffffffu, v);
    if (lr == 0) a.max_contrib[tile] = mm;
  }
}

__global__ void zero_i32_kernel(int32_t* p, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = 0;
}

// ------------------------------------------------------------------ backward
struct BwdArgs {
  int W, H, gx, num_tiles;
  int64_t bucket_sum;
  const uint2* ranges;
  const uint32_t* point_list;
  const uint32_t* bucket_offsets;
  const float2* means2d;
  const float* colors;
  const float4* conic;
  const float* bg;
  const float* dL_dout;
  const uint32_t* bucket_to_tile;
  const float* sampled_t;
  const float* sampled_ar;
  const float* final_t;
  const uint32_t* n_contrib;
  const uint32_t* max_contrib;
  const float* pixel_colors;
  float* dmeans2d;
  float* dcolors;
  float* dconic;
  float* dviewspace;
};

constexpr int kBwdWarps = 8;

__global__ void __launch_bounds__(kBwdWarps * 32) raster_bwd_kernel(BwdArgs a) {
  // per warp: 32 pixels x {T, ar0, ar1, ar2, T_final, last, dp0, dp1, dp2}
  __shared__ float s_px[kBwdWarps][9][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t bucket = (int64_t)blockIdx.x * kBwdWarps + w;
  if (bucket >= a.bucket_sum) return;
  const uint32_t tile = a.bucket_to_tile[bucket];
  if (tile >= (uint32_t)a.num_tiles) return;
  const uint2 range = a.ranges[tile];
  const int nsplat = (int)(range.y - range.x);
  const uint32_t bbm = (tile == 0u) ? 0u : a.bucket_offsets[tile - 1u];
  const int bidx = (int)((uint32_t)bucket - bbm);
  if (bidx * 32 >= (int)a.max_contrib[tile]) return;
  const int sidx = bidx * 32 + lane;
  const bool valid_splat = sidx < nsplat;
  uint32_t g = 0;
  float2 xy = make_float2(0.f, 0.f);
  float4 co = make_float4(0.f, 0.f, 0.f, 0.f);
  float c0 = 0.f, c1 = 0.f, c2 = 0.f;
  if (valid_splat) {
    g = a.point_list[range.x + sidx];
    xy = a.means2d[g];
    co = a.conic[g];
    c0 = a.colors[3 * (size_t)g];
    c1 = a.colors[3 * (size_t)g + 1];
    c2 = a.colors[3 * (size_t)g + 2];
  }
  float rm_x = 0.f, rm_y = 0.f, rm_z = 0.f, rm_w = 0.f;
  float rc_x = 0.f, rc_y = 0.f, rc_w = 0.f, rop = 0.f;
  float rcol0 = 0.f, rcol1 = 0.f, rcol2 = 0.f;
  const int tx = (int)tile % a.gx, ty = (int)tile / a.gx;
  const int pminx = tx * FGS_BLOCK, pminy = ty * FGS_BLOCK;
  const float ddelx_dx = 0.5f * (float)a.W, ddely_dy = 0.5f * (float)a.H;
  const size_t P = (size_t)a.W * a.H;
  const float* st = a.sampled_t + (size_t)bucket * kTile;
  const float* sar = a.sampled_ar + (size_t)bucket * 3 * kTile;
  const float bg0 = a.bg[0], bg1 = a.bg[1], bg2 = a.bg[2];

  float T = 0.f, T_final = 0.f, last = 0.f, ar0 = 0.f, ar1 = 0.f, ar2 = 0.f;
  float dp0 = 0.f, dp1 = 0.f, dp2 = 0.f;
  for (int i = 0; i < kTile + 31; ++i) {
    if ((i & 31) == 0 && i < kTile) {
      // stage pixels i .. i+31 of the tile: lane l takes pixel i + l
      __syncwarp();
      const int li = i + lane;
      const int ppx = pminx + (li & 15), ppy = pminy + (li >> 4);
      if (ppx < a.W && ppy < a.H) {
        const size_t id = (size_t)ppy * a.W + ppx;
        s_px[w][0][lane] = st[li];
        s_px[w][1][lane] = -a.pixel_colors[id] + sar[li];
        s_px[w][2][lane] = -a.pixel_colors[P + id] + sar[kTile + li];
        s_px[w][3][lane] = -a.pixel_colors[2 * P + id] + sar[2 * kTile + li];
        s_px[w][4][lane] = a.final_t[id];
        s_px[w][5][lane] = (float)a.n_contrib[id];
        s_px[w][6][lane] = a.dL_dout[id];
        s_px[w][7][lane] = a.dL_dout[P + id];
        s_px[w][8][lane] = a.dL_dout[2 * P + id];
      }
      __syncwarp();
    }
    T = __shfl_up_sync(0xffffffffu, T, 1);
    last = __shfl_up_sync(0xffffffffu, last, 1);
    T_final = __shfl_up_sync(0xffffffffu, T_final, 1);
    ar0 = __shfl_up_sync(0xffffffffu, ar0, 1);
    ar1 = __shfl_up_sync(0xffffffffu, ar1, 1);
    ar2 = __shfl_up_sync(0xffffffffu, ar2, 1);
    dp0 = __shfl_up_sync(0xffffffffu, dp0, 1);
    dp1 = __shfl_up_sync(0xffffffffu, dp1, 1);
    dp2 = __shfl_up_sync(0xffffffffu, dp2, 1);
    const int idx = i - lane;
    const int ppx = pminx + (idx & 15), ppy = pminy + (idx >> 4);
    const bool valid_pixel = idx >= 0 && idx < kTile && ppx < a.W && ppy < a.H;
    if (lane == 0 && valid_pixel) {
      const int ii = i & 31;
      T = s_px[w][0][ii];
      ar0 = s_px[w][1][ii];
      ar1 = s_px[w][2][ii];
      ar2 = s_px[w][3][ii];
      T_final = s_px[w][4][ii];
      last = s_px[w][5][ii];
      dp0 = s_px[w][6][ii];
      dp1 = s_px[w][7][ii];
      dp2 = s_px[w][8][ii];
    }
    if (!(valid_splat && valid_pixel)) continue;
    if (sidx >= (int)last) continue;
    const float dx = xy.x - (float)ppx, dy = xy.y - (float)ppy;
    const float power = -0.5f * (co.x * dx * dx + co.z * dy * dy) - co.y * dx * dy;
    if (power > 0.0f) continue;
    const float G = fgs_expf(power);
    const float alpha = fmin_t(0.99f, co.w * G);
    if (alpha < (1.0f / 255.0f)) continue;
    const float dchannel_dcolor = alpha * T;
    const float rec = 1.0f / (1.0f - alpha);
    float dL_dalpha = 0.0f;
    ar0 += dchannel_dcolor * c0;
    rcol0 += dchannel_dcolor * dp0;
    dL_dalpha += (c0 * T + rec * ar0) * dp0;
    ar1 += dchannel_dcolor * c1;
    rcol1 += dchannel_dcolor * dp1;
    dL_dalpha += (c1 * T + rec * ar1) * dp1;
    ar2 += dchannel_dcolor * c2;
    rcol2 += dchannel_dcolor * dp2;
    dL_dalpha += (c2 * T + rec * ar2) * dp2;
    float bg_dot = 0.0f;
    bg_dot += bg0 * dp0;
    bg_dot += bg1 * dp1;
    bg_dot += bg2 * dp2;
    dL_dalpha += (-T_final * rec) * bg_dot;
    T *= (1.0f - alpha);
    const float dL_dG = co.w * dL_dalpha;
    const float gdx = G * dx, gdy = G * dy;
    const float dG_ddelx = -gdx * co.x - gdy * co.y;
    const float dG_ddely = -gdy * co.z - gdx * co.y;
    if (co.w * G > 0.99f) continue;
    const float tmp_x = dL_dG * dG_ddelx * ddelx_dx;
    const float tmp_y = dL_dG * dG_ddely * ddely_dy;
    rm_x += tmp_x;
    rm_y += tmp_y;
    rm_z += fabsf(tmp_x);
    rm_w += fabsf(tmp_y);
    rc_x += -0.5f * gdx * dx * dL_dG;
    rc_y += -0.5f * gdx * dy * dL_dG;
    rc_w += -0.5f * gdy * dy * dL_dG;
    rop += G * dL_dalpha;
  }
  if (valid_splat) {
    atomicAdd(a.dmeans2d + 2 * (size_t)g, rm_x);
    atomicAdd(a.dmeans2d + 2 * (size_t)g + 1, rm_y);
    atomicAdd(a.dviewspace + 4 * (size_t)g, rm_x);
    atomicAdd(a.dviewspace + 4 * (size_t)g + 1, rm_y);
    atomicAdd(a.dviewspace + 4 * (size_t)g + 2, rm_z);
    atomicAdd(a.dviewspace + 4 * (size_t)g + 3, rm_w);
    atomicAdd(a.dconic + 4 * (size_t)g, rc_x);
    atomicAdd(a.dconic + 4 * (size_t)g + 1, rc_y);
    atomicAdd(a.dconic + 4 * (size_t)g + 2, rc_w);
    atomicAdd(a.dconic + 4 * (size_t)g + 3, rop);
    atomicAdd(a.dcolors + 3 * (size_t)g, rcol0);
    atomicAdd(a.dcolors + 3 * (size_t)g + 1, rcol1);
    atomicAdd(a.dcolors + 3 * (size_t)g + 2, rcol2);
  }
}

}  // namespace fgs

using namespace fgs;

extern "C" {

int fgs_rasterize_forward(const fgs_raster_params* p, const uint32_t* ranges,
                          const uint32_t* point_list, const uint32_t* bucket_offsets,
                          const float* means2d, const float* colors, const float* conic_opacity,
                          const float* background, const int32_t* metric_map,
                          uint32_t* bucket_to_tile, float* sampled_t, float* sampled_ar,
                          float* final_t, uint32_t* n_contrib, uint32_t* max_contrib,
                          float* pixel_colors, float* out_color, int32_t* metric_count,
                          void* stream) {
  FGS_CHECK_ARG(p != nullptr, "params is NULL");
  FGS_CHECK_ARG(p->image_width > 0 && p->image_height > 0, "image size must be positive");
  const int gx = (p->image_width + 15) / 16, gy = (p->image_height + 15) / 16;
  FGS_CHECK_ARG(p->num_tiles == gx * gy, "num_tiles (%d) must equal ceil(W/16)*ceil(H/16) (%d)",
                p->num_tiles, gx * gy);
  FGS_CHECK_ARG(p->bucket_sum >= 0, "bucket_sum must be >= 0");
  FGS_CHECK_ARG(ranges && bucket_offsets && final_t && n_contrib && max_contrib && pixel_colors &&
                    out_color && background,
                "missing pointer");
  FGS_CHECK_ARG(p->bucket_sum == 0 || (point_list && means2d && colors && conic_opacity &&
                                       bucket_to_tile && sampled_t && sampled_ar),
                "missing pointer");
  FGS_CHECK_ARG(!p->get_flag || (metric_map && metric_count), "get_flag needs metric_map / metric_count");
  cudaStream_t s = (cudaStream_t)stream;
  FwdArgs a;
  a.W = p->image_width;
  a.H = p->image_height;
  a.gx = gx;
  a.num_tiles = p->num_tiles;
  a.get_flag = p->get_flag;
  a.ranges = (const uint2*)ranges;
  a.point_list = point_list;
  a.bucket_offsets = bucket_offsets;
  a.means2d = (const float2*)means2d;
  a.colors = colors;
  a.conic = (const float4*)conic_opacity;
  a.bg = background;
  a.metric_map = metric_map;
  a.bucket_to_tile = bucket_to_tile;
  a.sampled_t = sampled_t;
  a.sampled_ar = sampled_ar;
  a.final_t = final_t;
  a.n_contrib = n_contrib;
  a.max_contrib = max_contrib;
  a.pixel_colors = pixel_colors;
  a.out_color = out_color;
  a.metric_count = metric_count;
  if (p->get_flag && p->num_gaussians > 0)
    zero_i32_kernel<<<(p->num_gaussians + 255) / 256, 256, 0, s>>>(metric_count, p->num_gaussians);
  raster_fwd_kernel<<<p->num_tiles, kTile, 0, s>>>(a);
  return check_launch("rasterize_forward");
}

int fgs_rasterize_backward(const fgs_raster_params* p, const uint32_t* ranges,
                           const uint32_t* point_list, const uint32_t* bucket_offsets,
                           const float* means2d, const float* colors, const float* conic_opacity,
                           const float* background, const float* dL_dout_color,
                           const uint32_t* bucket_to_tile, const float* sampled_t,
                           const float* sampled_ar, const float* final_t,
                           const uint32_t* n_contrib, const uint32_t* max_contrib,
                           const float* pixel_colors, float* dL_dmeans2d, float* dL_dcolors,
                           float* dL_dconic_opacity, float* dL_dviewspace, void* stream) {
  FGS_CHECK_ARG(p != nullptr, "params is NULL");
  FGS_CHECK_ARG(p->image_width > 0 && p->image_height > 0, "image size must be positive");
  const int gx = (p->image_width + 15) / 16, gy = (p->image_height + 15) / 16;
  FGS_CHECK_ARG(p->num_tiles == gx * gy, "num_tiles must equal ceil(W/16)*ceil(H/16)");
  FGS_CHECK_ARG(p->bucket_sum >= 0, "bucket_sum must be >= 0");
  if (p->bucket_sum == 0) return FGS_OK;
  FGS_CHECK_ARG(ranges && point_list && bucket_offsets && means2d && colors && conic_opacity &&
                    background && dL_dout_color && bucket_to_tile && sampled_t && sampled_ar &&
                    final_t && n_contrib && max_contrib && pixel_colors && dL_dmeans2d &&
                    dL_dcolors && dL_dconic_opacity && dL_dviewspace,
                "missing pointer");
  cudaStream_t s = (cudaStream_t)stream;
  BwdArgs a;
  a.W = p->image_width;
  a.H = p->image_height;
  a.gx = gx;
  a.num_tiles = p->num_tiles;
  a.bucket_sum = p->bucket_sum;
  a.ranges = (const uint2*)ranges;
  a.point_list = point_list;
  a.bucket_offsets = bucket_offsets;
  a.means2d = (const float2*)means2d;
  a.colors = colors;
  a.conic = (const float4*)conic_opacity;
  a.bg = background;
  a.dL_dout = dL_dout_color;
  a.bucket_to_tile = bucket_to_tile;
  a.sampled_t = sampled_t;
  a.sampled_ar = sampled_ar;
  a.final_t = final_t;
  a.n_contrib = n_contrib;
  a.max_contrib = max_contrib;
  a.pixel_colors = pixel_colors;
  a.dmeans2d = dL_dmeans2d;
  a.dcolors = dL_dcolors;
  a.dconic = dL_dconic_opacity;
  a.dviewspace = dL_dviewspace;
  const int64_t blocks = (p->bucket_sum + kBwdWarps - 1) / kBwdWarps;
  raster_bwd_kernel<<<(unsigned)blocks, kBwdWarps * 32, 0, s>>>(a);
  return check_launch("rasterize_backward");
}

}  // extern "C"
