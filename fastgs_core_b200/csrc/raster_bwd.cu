// Tile rasterizer backward on sm_100a (fastgs_core/metal/fastgs_rasterize_backward.metal:24-278).
//
// Same gradients as the reference's per-bucket kernel, organised pixel-
// parallel: one CTA per 16x16 tile, one thread per pixel. The CTA walks the
// tile's buckets (32 consecutive splats); each pixel starts a bucket from its
// forward sample (transmittance T and the colour accumulated before the
// bucket) and undoes the bucket's splats front to back. Per splat, a warp
// (two pixel rows) skips the splat outright when the splat's opacity-aware
// row extent misses its rows, or when no lane's pair passes the alpha test
// (ballot); otherwise the eleven per-pair partials are summed across the warp
// with a four-level transposed butterfly (lane 2k ends with value k) and added
// to the bucket's shared-memory accumulators; after the bucket, one global
// atomic per splat and output element. Compared with one warp per bucket
// (the reference's layout), this evaluates the same pairs but skips whole
// warp-splat blocks that cannot contribute and avoids the 31-step pipeline
// fill of the lane-to-lane state shift.
//
// Compiled with multiply-add contraction: gradient arithmetic may fuse. The
// per-pair decisions must match the forward pass exactly, so the exponent
// (splat_power), the opacity product and the exponential use explicitly
// rounded operations (fgs_common.cuh).
#include "../../include/fastgs_b200.h"
#include "fgs_common.cuh"

namespace fgs {

constexpr int kTilePx = 256;

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

// accumulator slots per splat
enum { kMx, kMy, kMxAbs, kMyAbs, kCx, kCy, kCw, kOp, kR, kG, kB, kSlots };

// Conservative tile-local pixel rows [lo, hi] where a splat can reach alpha >=
// 1/255 (same bound as the forward kernel's row culling).
__device__ __forceinline__ void bwd_splat_rows(float y, float a, float b, float c, float o, int pminy,
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

// Sum p[0..15] across the warp so that lanes 2k and 2k+1 hold sum_k.
__device__ __forceinline__ float warp_transpose_sum16(float (&p)[16], int lane) {
  {
    const bool hi = lane & 16;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float send = hi ? p[k] : p[k + 8];
      const float keep = hi ? p[k + 8] : p[k];
      p[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  {
    const bool hi = lane & 8;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float send = hi ? p[k] : p[k + 4];
      const float keep = hi ? p[k + 4] : p[k];
      p[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  {
    const bool hi = lane & 4;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float send = hi ? p[k] : p[k + 2];
      const float keep = hi ? p[k + 2] : p[k];
      p[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
  }
  {
    const bool hi = lane & 2;
    const float send = hi ? p[0] : p[1];
    const float keep = hi ? p[1] : p[0];
    p[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return p[0] + __shfl_xor_sync(0xffffffffu, p[0], 1);
}

__global__ void __launch_bounds__(kTilePx) raster_bwd_kernel(BwdArgs a) {
  __shared__ float4 s_r0[32];  // x, y, conic.x, conic.y
  __shared__ float4 s_r1[32];  // conic.z, opacity, r, g
  __shared__ float4 s_r2[32];  // b, exponent cut, rows lo / hi (int bits)
  __shared__ uint32_t s_id[32];
  __shared__ float s_acc[32][kSlots + 1];

  const int tile = blockIdx.x;
  const int lr = threadIdx.x, lane = lr & 31;
  const int wrow = (lr >> 5) * 2;
  const uint2 range = a.ranges[tile];
  const int nsplat = (int)(range.y - range.x);
  const int nb = (nsplat + 31) / 32;
  const int nb_active = min(nb, (int)((a.max_contrib[tile] + 31u) / 32u));
  if (nb_active == 0) return;
  const uint32_t bbm0 = (tile == 0) ? 0u : a.bucket_offsets[tile - 1];
  const int tx = tile % a.gx, ty = tile / a.gx;
  const int pminx = tx * FGS_BLOCK, pminy = ty * FGS_BLOCK;
  const int px = pminx + (lr & 15), py = pminy + (lr >> 4);
  const bool inside = px < a.W && py < a.H;
  const size_t P = (size_t)a.W * a.H;
  const size_t pix = inside ? (size_t)py * a.W + px : 0;
  const float pfx = (float)px, pfy = (float)py;
  float d0 = 0.f, d1 = 0.f, d2 = 0.f, tfbg = 0.f, pc0 = 0.f, pc1 = 0.f, pc2 = 0.f;
  int last = 0;
  if (inside) {
    d0 = a.dL_dout[pix];
    d1 = a.dL_dout[P + pix];
    d2 = a.dL_dout[2 * P + pix];
    tfbg = a.final_t[pix] * (a.bg[0] * d0 + a.bg[1] * d1 + a.bg[2] * d2);
    pc0 = a.pixel_colors[pix];
    pc1 = a.pixel_colors[P + pix];
    pc2 = a.pixel_colors[2 * P + pix];
    last = (int)a.n_contrib[pix];
  }
  const float hw = 0.5f * (float)a.W, hh = 0.5f * (float)a.H;

  for (int b = 0; b < nb_active; ++b) {
    const size_t bucket = (size_t)bbm0 + b;
    __syncthreads();  // previous bucket's accumulators flushed, records free
    if (lr < 32) {
      const int s = b * 32 + lr;
      if (s < nsplat) {
        const uint32_t g = a.point_list[range.x + s];
        const float2 xy = a.means2d[g];
        const float4 co = a.conic[g];
        int rlo, rhi;
        bwd_splat_rows(xy.y, co.x, co.y, co.z, co.w, pminy, rlo, rhi);
        s_r0[lr] = make_float4(xy.x, xy.y, co.x, co.y);
        s_r1[lr] = make_float4(co.z, co.w, a.colors[3 * (size_t)g], a.colors[3 * (size_t)g + 1]);
        s_r2[lr] = make_float4(a.colors[3 * (size_t)g + 2], power_cut(co.w), __int_as_float(rlo),
                               __int_as_float(rhi));
        s_id[lr] = g;
      } else {
        s_r2[lr] = make_float4(0.f, 0.f, __int_as_float(1), __int_as_float(0));  // no rows
        s_id[lr] = 0xffffffffu;
      }
    }
    for (int k = lr; k < 32 * (kSlots + 1); k += kTilePx) (&s_acc[0][0])[k] = 0.0f;
    float T = a.sampled_t[bucket * kTilePx + lr];
    const float* sar = a.sampled_ar + bucket * 3 * kTilePx + lr;
    float ar0 = sar[0] - pc0, ar1 = sar[kTilePx] - pc1, ar2 = sar[2 * kTilePx] - pc2;
    __syncthreads();
    const int s0 = b * 32;
    for (int j = 0; j < 32; ++j) {
      const float4 r2 = s_r2[j];
      if (__float_as_int(r2.w) < wrow || __float_as_int(r2.z) > wrow + 1) continue;  // warp-uniform
      const float4 r0 = s_r0[j];
      const float4 r1 = s_r1[j];
      const float dx = r0.x - pfx, dy = r0.y - pfy;
      const float power = splat_power(r0.z, r0.w, r1.x, dx, dy);
      // same decisions as the forward pass (NaN exponents included)
      bool v = (s0 + j < last) && !(power > 0.0f) && !(power <= r2.y);
      float G = 0.f, oG = 0.f, alpha = 0.f;
      if (v) {
        G = fgs_expf_neg(power);
        oG = __fmul_rn(r1.y, G);
        alpha = fmin_t(0.99f, oG);
        v = alpha >= 1.0f / 255.0f;
      }
      if (__ballot_sync(0xffffffffu, v) == 0u) continue;  // warp-uniform
      float p[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) p[k] = 0.0f;
      if (v) {
        const float c0 = r1.z, c1 = r1.w, c2 = r2.x;
        const float wgt = alpha * T;
        const float rec = __fdividef(1.0f, 1.0f - alpha);
        ar0 += wgt * c0;
        ar1 += wgt * c1;
        ar2 += wgt * c2;
        p[kR] = wgt * d0;
        p[kG] = wgt * d1;
        p[kB] = wgt * d2;
        const float cdot = c0 * d0 + c1 * d1 + c2 * d2;
        const float adot = ar0 * d0 + ar1 * d1 + ar2 * d2;
        const float dL_dalpha = T * cdot + rec * (adot - tfbg);
        T *= (1.0f - alpha);
        if (!(oG > 0.99f)) {
          const float dL_dG = r1.y * dL_dalpha;
          const float gdx = G * dx, gdy = G * dy;
          const float tmp_x = dL_dG * (-gdx * r0.z - gdy * r0.w) * hw;
          const float tmp_y = dL_dG * (-gdy * r1.x - gdx * r0.w) * hh;
          p[kMx] = tmp_x;
          p[kMy] = tmp_y;
          p[kMxAbs] = fabsf(tmp_x);
          p[kMyAbs] = fabsf(tmp_y);
          const float q = -0.5f * dL_dG;
          p[kCx] = q * gdx * dx;
          p[kCy] = q * gdx * dy;
          p[kCw] = q * gdy * dy;
          p[kOp] = G * dL_dalpha;
        }
      }
      const float tot = warp_transpose_sum16(p, lane);
      const int slot = lane >> 1;
      if (!(lane & 1) && slot < kSlots) atomicAdd(&s_acc[j][slot], tot);
    }
    __syncthreads();
    for (int k = lr; k < 32 * kSlots; k += kTilePx) {
      const int j = k / kSlots, slot = k % kSlots;
      const uint32_t g = s_id[j];
      if (g == 0xffffffffu) continue;
      const float v = s_acc[j][slot];
      float* dst;
      switch (slot) {
        case kMx: dst = a.dmeans2d + 2 * (size_t)g; break;
        case kMy: dst = a.dmeans2d + 2 * (size_t)g + 1; break;
        case kMxAbs: dst = a.dviewspace + 4 * (size_t)g + 2; break;
        case kMyAbs: dst = a.dviewspace + 4 * (size_t)g + 3; break;
        case kCx: dst = a.dconic + 4 * (size_t)g; break;
        case kCy: dst = a.dconic + 4 * (size_t)g + 1; break;
        case kCw: dst = a.dconic + 4 * (size_t)g + 2; break;
        case kOp: dst = a.dconic + 4 * (size_t)g + 3; break;
        case kR: dst = a.dcolors + 3 * (size_t)g; break;
        case kG: dst = a.dcolors + 3 * (size_t)g + 1; break;
        default: dst = a.dcolors + 3 * (size_t)g + 2; break;
      }
      atomicAdd(dst, v);
      if (slot == kMx) atomicAdd(a.dviewspace + 4 * (size_t)g, v);
      if (slot == kMy) atomicAdd(a.dviewspace + 4 * (size_t)g + 1, v);
    }
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
  raster_bwd_kernel<<<p->num_tiles, kTilePx, 0, s>>>(a);
  return check_launch("rasterize_backward");
}

}  // extern "C"
