// Tile rasterizer backward on sm_100a (fastgs_core/metal/fastgs_rasterize_backward.metal:24-278).
//
// One warp per bucket (32 consecutive splats of one tile, one splat per
// lane). Pixel i of the tile enters at lane 0 on step i with the bucket's
// sample (transmittance T and the colour accumulated before the bucket) and
// moves one lane per step, so every pixel is undone through the bucket's 32
// splats front to back; each lane keeps its splat's gradient partials in
// registers and adds them with one atomic per output element at the end.
// Only the mutable blend state (T and the three remaining-colour sums) moves
// between lanes; the per-pixel read-only data (dL/dpixel, T_final * bg.dL,
// n_contrib) and the bucket samples are staged once per warp in shared memory.
//
// This file is compiled with multiply-add contraction: gradient arithmetic is
// free to fuse. The per-pair decisions must match the forward pass exactly,
// so the exponent (splat_power), the opacity product and the exponential use
// explicitly rounded operations (see fgs_common.cuh).
#include "../../include/fastgs_b200.h"
#include "fgs_common.cuh"

namespace fgs {

constexpr int kTilePx = 256;
constexpr int kBwdWarps = 8;

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

struct WarpStage {
  float4 state[kTilePx];  // bucket sample: T, ar0, ar1, ar2 (ar = sampled colour - final colour)
  float4 ro[kTilePx];     // dL/dpix r, g, b and T_final * (bg . dL/dpix)
  int last[kTilePx];      // n_contrib (0 outside the image)
};

__global__ void __launch_bounds__(kBwdWarps * 32) raster_bwd_kernel(BwdArgs a) {
  extern __shared__ __align__(16) unsigned char s_raw[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  WarpStage& S = reinterpret_cast<WarpStage*>(s_raw)[w];
  const int64_t bucket = (int64_t)blockIdx.x * kBwdWarps + w;
  if (bucket >= a.bucket_sum) return;
  const uint32_t tile = a.bucket_to_tile[bucket];
  if (tile >= (uint32_t)a.num_tiles) return;
  const uint2 range = a.ranges[tile];
  const int nsplat = (int)(range.y - range.x);
  const uint32_t bbm = (tile == 0u) ? 0u : a.bucket_offsets[tile - 1u];
  const int bidx = (int)((uint32_t)bucket - bbm);
  if (bidx * 32 >= (int)a.max_contrib[tile]) return;

  const int tx = (int)tile % a.gx, ty = (int)tile / a.gx;
  const int pminx = tx * FGS_BLOCK, pminy = ty * FGS_BLOCK;
  const size_t P = (size_t)a.W * a.H;
  const float bg0 = a.bg[0], bg1 = a.bg[1], bg2 = a.bg[2];
  // stage this bucket's pixel data: lane takes pixels lane, lane + 32, ...
  {
    const float* st = a.sampled_t + (size_t)bucket * kTilePx;
    const float* sar = a.sampled_ar + (size_t)bucket * 3 * kTilePx;
    for (int li = lane; li < kTilePx; li += 32) {
      const int ppx = pminx + (li & 15), ppy = pminy + (li >> 4);
      if (ppx < a.W && ppy < a.H) {
        const size_t id = (size_t)ppy * a.W + ppx;
        const float d0 = a.dL_dout[id], d1 = a.dL_dout[P + id], d2 = a.dL_dout[2 * P + id];
        const float bg_dot = bg0 * d0 + bg1 * d1 + bg2 * d2;
        S.state[li] = make_float4(st[li], -a.pixel_colors[id] + sar[li],
                                  -a.pixel_colors[P + id] + sar[kTilePx + li],
                                  -a.pixel_colors[2 * P + id] + sar[2 * kTilePx + li]);
        S.ro[li] = make_float4(d0, d1, d2, a.final_t[id] * bg_dot);
        S.last[li] = (int)a.n_contrib[id];
      } else {
        S.state[li] = make_float4(0.f, 0.f, 0.f, 0.f);
        S.ro[li] = make_float4(0.f, 0.f, 0.f, 0.f);
        S.last[li] = 0;
      }
    }
  }
  __syncwarp();

  const int sidx0 = bidx * 32 + lane;
  const bool valid_splat = sidx0 < nsplat;
  const int sidx = valid_splat ? sidx0 : 0x7fffffff;  // never below n_contrib
  uint32_t g = 0;
  float2 xy = make_float2(0.f, 0.f);
  float4 co = make_float4(0.f, 0.f, 0.f, 0.f);
  float c0 = 0.f, c1 = 0.f, c2 = 0.f;
  if (valid_splat) {
    g = a.point_list[range.x + sidx0];
    xy = a.means2d[g];
    co = a.conic[g];
    c0 = a.colors[3 * (size_t)g];
    c1 = a.colors[3 * (size_t)g + 1];
    c2 = a.colors[3 * (size_t)g + 2];
  }
  const float pcut = power_cut(co.w);
  const float hw = 0.5f * (float)a.W, hh = 0.5f * (float)a.H;
  float rm_x = 0.f, rm_y = 0.f, rm_z = 0.f, rm_w = 0.f;
  float rc_x = 0.f, rc_y = 0.f, rc_w = 0.f, rop = 0.f;
  float rcol0 = 0.f, rcol1 = 0.f, rcol2 = 0.f;

  float T = 0.f, ar0 = 0.f, ar1 = 0.f, ar2 = 0.f;
  for (int i = 0; i < kTilePx + 31; ++i) {
    T = __shfl_up_sync(0xffffffffu, T, 1);
    ar0 = __shfl_up_sync(0xffffffffu, ar0, 1);
    ar1 = __shfl_up_sync(0xffffffffu, ar1, 1);
    ar2 = __shfl_up_sync(0xffffffffu, ar2, 1);
    {
      const float4 inj = S.state[i & (kTilePx - 1)];
      if (lane == 0) {
        T = inj.x;
        ar0 = inj.y;
        ar1 = inj.z;
        ar2 = inj.w;
      }
    }
    const int idx = i - lane;
    if ((unsigned)idx >= (unsigned)kTilePx) continue;
    if (sidx >= S.last[idx]) continue;
    const float dx = xy.x - (float)(pminx + (idx & 15));
    const float dy = xy.y - (float)(pminy + (idx >> 4));
    const float power = splat_power(co.x, co.y, co.z, dx, dy);
    if (power > 0.0f || power <= pcut) continue;
    const float G = fgs_expf_neg(power);
    const float oG = __fmul_rn(co.w, G);
    const float alpha = fmin_t(0.99f, oG);
    if (alpha < 1.0f / 255.0f) continue;
    const float4 ro = S.ro[idx];
    const float wgt = alpha * T;
    const float rec = __fdividef(1.0f, 1.0f - alpha);
    ar0 += wgt * c0;
    ar1 += wgt * c1;
    ar2 += wgt * c2;
    rcol0 += wgt * ro.x;
    rcol1 += wgt * ro.y;
    rcol2 += wgt * ro.z;
    const float cdot = c0 * ro.x + c1 * ro.y + c2 * ro.z;
    const float adot = ar0 * ro.x + ar1 * ro.y + ar2 * ro.z;
    const float dL_dalpha = T * cdot + rec * (adot - ro.w);
    T *= (1.0f - alpha);
    if (oG > 0.99f) continue;
    const float dL_dG = co.w * dL_dalpha;
    const float gdx = G * dx, gdy = G * dy;
    const float tmp_x = dL_dG * (-gdx * co.x - gdy * co.y) * hw;
    const float tmp_y = dL_dG * (-gdy * co.z - gdx * co.y) * hh;
    rm_x += tmp_x;
    rm_y += tmp_y;
    rm_z += fabsf(tmp_x);
    rm_w += fabsf(tmp_y);
    const float q = -0.5f * dL_dG;
    rc_x += q * gdx * dx;
    rc_y += q * gdx * dy;
    rc_w += q * gdy * dy;
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
  const int smem = (int)(kBwdWarps * sizeof(WarpStage));
  static unsigned long long attr_done = 0;
  smem_attr_once(raster_bwd_kernel, smem, &attr_done);
  const int64_t blocks = (p->bucket_sum + kBwdWarps - 1) / kBwdWarps;
  raster_bwd_kernel<<<(unsigned)blocks, kBwdWarps * 32, smem, s>>>(a);
  return check_launch("rasterize_backward");
}

}  // extern "C"
