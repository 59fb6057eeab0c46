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
// Pixels terminate the loop early (T < 1e-4) and whole warps skip splats
// whose opacity-aware extent misses their two pixel rows. The backward pass
// is in raster_bwd.cu.
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
  const uint32_t* tile_order;
  uint32_t* contrib_mask;  // optional [bucket][256]: contributing splats of the bucket per pixel
  int sparse;              // samples of pixels terminated before a bucket are not written
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

// Conservative range of tile-local pixel rows [lo, hi] on which a splat can
// reach alpha >= 1/255: the ellipse 0.5 (a dx^2 + 2 b dx dy + c dy^2) <= ln(255 o)
// spans |dy| <= sqrt(2 ln(255 o) a / (a c - b^2)); widened by 0.1% + 0.01 px.
// Non-positive-definite conics get the whole tile; o <= 1/255 gets no rows.
__device__ __forceinline__ void splat_rows(float y, float a, float b, float c, float o, int pminy,
                                           int& lo, int& hi) {
  lo = 0;
  hi = FGS_BLOCK - 1;
  const float det = a * c - b * b;
  if (!(a > 0.0f && det > 0.0f && o == o)) return;
  if (!(o * 255.0f > 1.0f)) {
    lo = 1;
    hi = 0;
    return;
  }
  const float L = logf(255.0f * o);
  const float dymax = sqrtf(2.0f * L * a / det) * 1.001f + 0.01f;
  if (!(dymax < 1e6f)) return;
  const float yl = y - (float)pminy;
  lo = max(-1, (int)ceilf(yl - dymax));
  hi = min(FGS_BLOCK, (int)floorf(yl + dymax));
}

// PX pixels per thread: a warp covers 2*PX consecutive pixel rows (lane l:
// column l % 16, rows base + l / 16 + 2k), so staged-record reads, the
// warp-level row culling and the loop are shared by PX pixels. The per-pixel
// arithmetic is unchanged (bit-identical results).
template <int PX, bool kMask, bool kMetric>
// six resident CTAs per SM (config 3: 0.646 ms; four: 0.662 ms; seven, at 32
// registers with spills: 0.647 ms)
__global__ void __launch_bounds__(kTile / PX, 6) raster_fwd_kernel(FwdArgs a) {
  constexpr int kThreads = kTile / PX;
  constexpr int kWarpRows = 2 * PX;
  __shared__ float4 s_r0[kTile];  // x, y, conic.x, conic.y
  __shared__ float4 s_r1[kTile];  // conic.z, opacity, r, g
  __shared__ float4 s_r2[kTile];  // b, exponent cut, -, -
  __shared__ uint32_t s_id[kTile];
  __shared__ uint32_t s_wmax[kThreads / 32];
  // per warp and 32-splat block of the batch: which splats can reach the
  // warp's rows (bit j: splat 32 * block + j)
  __shared__ uint32_t s_wmask[kThreads / 32][kTile / 32];

  const int tile = a.tile_order ? (int)a.tile_order[blockIdx.x] : (int)blockIdx.x;
  const int lr = threadIdx.x, lane = lr & 31;
  const int tx = tile % a.gx, ty = tile / a.gx;
  const int wrow = (lr >> 5) * kWarpRows;  // this warp's first tile row
  const size_t P = (size_t)a.W * a.H;
  const uint2 range = a.ranges[tile];
  const int to_do = (int)(range.y - range.x);
  const int nb = (to_do + 31) / 32;
  const uint32_t bbm0 = (tile == 0) ? 0u : a.bucket_offsets[tile - 1];
  for (int b = lr; b < nb; b += kThreads) a.bucket_to_tile[bbm0 + b] = (uint32_t)tile;

  int lpix[PX];
  size_t pix[PX];
  bool inside[PX], done[PX], count_metric[PX];
  float pfx[PX], pfy[PX], T[PX], C0[PX], C1[PX], C2[PX];
  uint32_t last[PX];
#pragma unroll
  for (int k = 0; k < PX; ++k) {
    const int row = wrow + (lane >> 4) + 2 * k;
    lpix[k] = row * FGS_BLOCK + (lane & 15);
    const int px = tx * FGS_BLOCK + (lane & 15), py = ty * FGS_BLOCK + row;
    inside[k] = px < a.W && py < a.H;
    pix[k] = inside[k] ? (size_t)py * a.W + px : 0;
    pfx[k] = (float)px;
    pfy[k] = (float)py;
    count_metric[k] = kMetric && inside[k] && a.metric_map[pix[k]] == 1;
    T[k] = 1.0f;
    C0[k] = C1[k] = C2[k] = 0.f;
    last[k] = 0;
    done[k] = !inside[k];
  }
  int processed = 0;
  for (int batch = 0; batch < to_do; batch += kTile) {
    bool live = false;
#pragma unroll
    for (int k = 0; k < PX; ++k) live |= !done[k];
    if (__syncthreads_count(live) == 0) break;
    for (int q = lr; q < kTile; q += kThreads) {
      const int j = batch + q;
      uint32_t bands = 0u;  // warps whose rows the splat can reach
      if (j < to_do) {
        const uint32_t g = a.point_list[range.x + j];
        const float2 xy = a.means2d[g];
        const float4 co = a.conic[g];
        int rlo, rhi;
        splat_rows(xy.y, co.x, co.y, co.z, co.w, ty * FGS_BLOCK, rlo, rhi);
        s_r0[q] = make_float4(xy.x, xy.y, co.x, co.y);
        s_r1[q] = make_float4(co.z, co.w, a.colors[3 * (size_t)g], a.colors[3 * (size_t)g + 1]);
        s_r2[q] = make_float4(a.colors[3 * (size_t)g + 2], power_cut(co.w), 0.0f, 0.0f);
        s_id[q] = g;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w)
          if (rhi >= w * kWarpRows && rlo <= w * kWarpRows + kWarpRows - 1) bands |= 1u << w;
      }
      // a warp stages one whole 32-splat block per pass (kThreads is a multiple of 32)
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) {
        const uint32_t bm = __ballot_sync(0xffffffffu, (bands >> w) & 1u);
        if (lane == 0) s_wmask[w][q >> 5] = bm;
      }
    }
    __syncthreads();
    const int cnt = min(kTile, to_do - batch);
    for (int k0 = 0; k0 < cnt; k0 += 32) {
      const size_t b = (size_t)bbm0 + (size_t)((batch + k0) >> 5);
      bool any = false;
#pragma unroll
      for (int k = 0; k < PX; ++k) {
        if (!(done[k] && a.sparse)) {
          a.sampled_t[b * kTile + lpix[k]] = done[k] ? 0.0f : T[k];
          float* ar = a.sampled_ar + b * 3 * kTile + lpix[k];
          ar[0] = done[k] ? 0.0f : C0[k];
          ar[kTile] = done[k] ? 0.0f : C1[k];
          ar[2 * kTile] = done[k] ? 0.0f : C2[k];
        }
        any |= !done[k];
      }
      if (!any) {
        if (kMask && !a.sparse) {
#pragma unroll
          for (int k = 0; k < PX; ++k) a.contrib_mask[b * kTile + lpix[k]] = 0u;
        }
        continue;
      }
      uint32_t msk[PX];
#pragma unroll
      for (int k = 0; k < PX; ++k) msk[k] = 0u;
      // walk only the block's splats that can reach this warp's rows, in order
      for (uint32_t wm = s_wmask[lr >> 5][k0 >> 5]; wm != 0u; wm &= wm - 1u) {
        const int j = k0 + __ffs(wm) - 1;
        const float4 r2 = s_r2[j];
        const float4 r0 = s_r0[j];
        const float4 r1 = s_r1[j];
        // the reference counts every splat it steps over (fastgs_rasterize.metal:99)
        const uint32_t contributor = (uint32_t)(batch + j + 1);
#pragma unroll
        for (int k = 0; k < PX; ++k) {
          if (done[k]) continue;
          const float dx = r0.x - pfx[k], dy = r0.y - pfy[k];
          const float power = splat_power(r0.z, r0.w, r1.x, dx, dy);
          if (power > 0.0f) continue;
          if (power <= r2.y) continue;  // alpha < 1/255 for certain
          const float alpha = fmin_t(0.99f, r1.y * fgs_expf_neg(power));
          if (alpha < 1.0f / 255.0f) continue;
          const float test_t = T[k] * (1.0f - alpha);
          if (test_t < 0.0001f) {
            done[k] = true;
            continue;
          }
          // one weight per pair, fused accumulation (the CPU checker's
          // definition: c = fma(col, alpha * T, c))
          const float wgt = alpha * T[k];
          C0[k] = fmaf(r1.z, wgt, C0[k]);
          C1[k] = fmaf(r1.w, wgt, C1[k]);
          C2[k] = fmaf(r2.x, wgt, C2[k]);
          if (kMetric && count_metric[k]) atomicAdd(a.metric_count + s_id[j], 1);
          T[k] = test_t;
          last[k] = contributor;
          if (kMask) msk[k] |= 1u << (j & 31);  // k0 is a multiple of 32
        }
      }
      if (kMask) {
#pragma unroll
        for (int k = 0; k < PX; ++k)
          if (!(a.sparse && msk[k] == 0u && done[k])) a.contrib_mask[b * kTile + lpix[k]] = msk[k];
      }
    }
    processed = batch + cnt;
    __syncthreads();
  }
  // buckets the CTA never reached (every pixel had terminated): zero samples
  // (sparse: left unwritten, the backward pass does not read them)
  for (int bl = a.sparse ? nb : (processed + 31) >> 5; bl < nb; ++bl) {
    const size_t b = (size_t)bbm0 + bl;
#pragma unroll
    for (int k = 0; k < PX; ++k) {
      a.sampled_t[b * kTile + lpix[k]] = 0.0f;
      float* ar = a.sampled_ar + b * 3 * kTile + lpix[k];
      ar[0] = 0.0f;
      ar[kTile] = 0.0f;
      ar[2 * kTile] = 0.0f;
      if (kMask) a.contrib_mask[b * kTile + lpix[k]] = 0u;
    }
  }
  const float bg0 = a.bg[0], bg1 = a.bg[1], bg2 = a.bg[2];
  uint32_t mymax = 0;
#pragma unroll
  for (int k = 0; k < PX; ++k) {
    if (!inside[k]) continue;
    const size_t q = pix[k];
    a.final_t[q] = T[k];
    a.n_contrib[q] = last[k];
    a.pixel_colors[q] = C0[k];
    a.pixel_colors[P + q] = C1[k];
    a.pixel_colors[2 * P + q] = C2[k];
    a.out_color[q] = C0[k] + T[k] * bg0;
    a.out_color[P + q] = C1[k] + T[k] * bg1;
    a.out_color[2 * P + q] = C2[k] + T[k] * bg2;
    mymax = last[k] > mymax ? last[k] : mymax;
  }
  const uint32_t m = __reduce_max_sync(0xffffffffu, mymax);
  if (lane == 0) s_wmax[lr >> 5] = m;
  __syncthreads();
  if (lr < 32) {
    const uint32_t v = lr < kThreads / 32 ? s_wmax[lr] : 0u;
    const uint32_t mm = __reduce_max_sync(0xffffffffu, v);
    if (lr == 0) a.max_contrib[tile] = mm;
  }
}

__global__ void zero_i32_kernel(int32_t* p, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = 0;
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
  FGS_CHECK_ARG(FGS_ALIGNED(ranges, 8) && FGS_ALIGNED(means2d, 8) && FGS_ALIGNED(conic_opacity, 16),
                "ranges and means2d must be 8-byte, conic_opacity 16-byte aligned");
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
  a.tile_order = p->tile_order;
  a.contrib_mask = p->contrib_mask;
  a.sparse = p->sparse_samples != 0;
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
  // one pixel per thread (config 3: 0.805 ms; two per thread measured 0.826 ms)
  const dim3 grid(p->num_tiles), block(kTile);
  if (a.contrib_mask && a.get_flag)
    raster_fwd_kernel<1, true, true><<<grid, block, 0, s>>>(a);
  else if (a.contrib_mask)
    raster_fwd_kernel<1, true, false><<<grid, block, 0, s>>>(a);
  else if (a.get_flag)
    raster_fwd_kernel<1, false, true><<<grid, block, 0, s>>>(a);
  else
    raster_fwd_kernel<1, false, false><<<grid, block, 0, s>>>(a);
  return check_launch("rasterize_forward");
}

}  // extern "C"
