// Tile rasterizer backward on sm_100a (fastgs_core/metal/fastgs_rasterize_backward.metal:24-278).
//
// Same gradients as the reference's per-bucket kernel, organised pixel-
// parallel: one CTA per 16x16 tile, one thread per pixel. The CTA stages the
// records of up to 256 splats (8 buckets) at a time; each warp (two pixel
// rows) then walks them front to back on its own, restarting each bucket from
// the pixel's forward sample (transmittance T and the colour accumulated
// before the bucket, kept as its dot product with dL/dpixel, which is all the
// alpha gradient needs). Per splat, a warp skips the splat outright when the
// splat's opacity-aware row extent misses its rows, or when no lane's pair
// passes the alpha test (ballot); otherwise the eleven per-pair partials are
// summed across the warp with a five-level transposed butterfly (lane 2k ends
// with value k) and added to shared-memory accumulators; after the chunk, one
// global atomic per splat and output element. Compared with one warp per bucket
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

constexpr int kChunk = 256;  // splats (8 buckets) staged per CTA pass

__global__ void __launch_bounds__(kTilePx) raster_bwd_kernel(BwdArgs a) {
  // splat records of the current chunk
  __shared__ float4 s_r0[kChunk];  // x, y, conic.a, conic.b
  __shared__ float4 s_r1[kChunk];  // conic.c, opacity, r, g
  __shared__ float4 s_r2[kChunk];  // b, exponent cut, rows lo / hi (int bits)
  __shared__ uint32_t s_id[kChunk];
  __shared__ float s_acc[kChunk][kSlots];

  const int tile = blockIdx.x;
  const int lr = threadIdx.x, lane = lr & 31;
  const int wrow = (lr >> 5) * 2;
  const uint2 range = a.ranges[tile];
  const int nsplat = (int)(range.y - range.x);
  // buckets at or past max_contrib have no contributing pixel (reference:
  // fastgs_rasterize_backward.metal:72-74)
  const int nact = min(nsplat, (int)((a.max_contrib[tile] + 31u) / 32u) * 32);
  if (nact <= 0) return;
  const uint32_t bbm0 = (tile == 0) ? 0u : a.bucket_offsets[tile - 1];
  const int tx = tile % a.gx, ty = tile / a.gx;
  const int pminx = tx * FGS_BLOCK, pminy = ty * FGS_BLOCK;
  const int px = pminx + (lr & 15), py = pminy + (lr >> 4);
  const bool inside = px < a.W && py < a.H;
  const size_t P = (size_t)a.W * a.H;
  const size_t pix = inside ? (size_t)py * a.W + px : 0;
  const float pfx = (float)px, pfy = (float)py;
  float d0 = 0.f, d1 = 0.f, d2 = 0.f, tfbg = 0.f, pcd = 0.f;
  int last = 0;
  if (inside) {
    d0 = a.dL_dout[pix];
    d1 = a.dL_dout[P + pix];
    d2 = a.dL_dout[2 * P + pix];
    tfbg = a.final_t[pix] * (a.bg[0] * d0 + a.bg[1] * d1 + a.bg[2] * d2);
    // final colour . dL/dpix: the per-bucket remaining-colour dot starts from
    // (sampled colour - final colour) . dL/dpix
    pcd = a.pixel_colors[pix] * d0 + a.pixel_colors[P + pix] * d1 + a.pixel_colors[2 * P + pix] * d2;
    last = (int)a.n_contrib[pix];
  }
  const float hw = 0.5f * (float)a.W, hh = 0.5f * (float)a.H;

  for (int c0 = 0; c0 < nact; c0 += kChunk) {
    const int cn = min(kChunk, nact - c0);
    __syncthreads();  // previous chunk flushed
    if (lr < cn) {
      const uint32_t g = a.point_list[range.x + c0 + lr];
      const float2 xy = a.means2d[g];
      const float4 co = a.conic[g];
      int rlo, rhi;
      bwd_splat_rows(xy.y, co.x, co.y, co.z, co.w, pminy, rlo, rhi);
      s_r0[lr] = make_float4(xy.x, xy.y, co.x, co.y);
      s_r1[lr] = make_float4(co.z, co.w, a.colors[3 * (size_t)g], a.colors[3 * (size_t)g + 1]);
      s_r2[lr] = make_float4(a.colors[3 * (size_t)g + 2], power_cut(co.w), __int_as_float(rlo),
                             __int_as_float(rhi));
      s_id[lr] = g;
    }
    for (int k = lr; k < kChunk * kSlots; k += kTilePx) (&s_acc[0][0])[k] = 0.0f;
    __syncthreads();
    float T = 0.f, adot = 0.f;
    for (int j = 0; j < cn; ++j) {
      const int s = c0 + j;
      if ((s & 31) == 0) {
        // bucket start: the forward sample of this pixel
        const size_t bucket = (size_t)bbm0 + (size_t)(s >> 5);
        T = a.sampled_t[bucket * kTilePx + lr];
        const float* sar = a.sampled_ar + bucket * 3 * kTilePx + lr;
        adot = sar[0] * d0 + sar[kTilePx] * d1 + sar[2 * kTilePx] * d2 - pcd;
      }
      const float4 r2 = s_r2[j];
      if (__float_as_int(r2.w) < wrow || __float_as_int(r2.z) > wrow + 1) continue;  // warp-uniform
      const float4 r0 = s_r0[j];
      const float4 r1 = s_r1[j];
      const float dx = r0.x - pfx, dy = r0.y - pfy;
      const float power = splat_power(r0.z, r0.w, r1.x, dx, dy);
      // same decisions as the forward pass (NaN exponents included)
      bool v = (s < last) && !(power > 0.0f) && !(power <= r2.y);
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
        const float c0c = r1.z, c1c = r1.w, c2c = r2.x;
        const float wgt = alpha * T;
        const float rec = __fdividef(1.0f, 1.0f - alpha);
        const float cdot = c0c * d0 + c1c * d1 + c2c * d2;
        adot += wgt * cdot;  // remaining colour after this splat, dotted with dL/dpix
        const float dL_dalpha = T * cdot + rec * (adot - tfbg);
        T *= (1.0f - alpha);
        p[kR] = wgt * d0;
        p[kG] = wgt * d1;
        p[kB] = wgt * d2;
        if (!(oG > 0.99f)) {
          const float u = r1.y * dL_dalpha * G;  // dL/dG * G
          const float tmp_x = -u * (r0.z * dx + r0.w * dy) * hw;
          const float tmp_y = -u * (r1.x * dy + r0.w * dx) * hh;
          p[kMx] = tmp_x;
          p[kMy] = tmp_y;
          p[kMxAbs] = fabsf(tmp_x);
          p[kMyAbs] = fabsf(tmp_y);
          const float q = -0.5f * u;
          const float qdx = q * dx;
          p[kCx] = qdx * dx;
          p[kCy] = qdx * dy;
          p[kCw] = q * dy * dy;
          p[kOp] = G * dL_dalpha;
        }
      }
      const float tot = warp_transpose_sum16(p, lane);
      const int slot = lane >> 1;
      if (!(lane & 1) && slot < kSlots) atomicAdd(&s_acc[j][slot], tot);
    }
    __syncthreads();
    if (lr < cn) {
      const size_t g = s_id[lr];
      const float* v = s_acc[lr];
      atomicAdd(a.dmeans2d + 2 * g, v[kMx]);
      atomicAdd(a.dmeans2d + 2 * g + 1, v[kMy]);
      atomicAdd(a.dviewspace + 4 * g, v[kMx]);
      atomicAdd(a.dviewspace + 4 * g + 1, v[kMy]);
      atomicAdd(a.dviewspace + 4 * g + 2, v[kMxAbs]);
      atomicAdd(a.dviewspace + 4 * g + 3, v[kMyAbs]);
      atomicAdd(a.dconic + 4 * g, v[kCx]);
      atomicAdd(a.dconic + 4 * g + 1, v[kCy]);
      atomicAdd(a.dconic + 4 * g + 2, v[kCw]);
      atomicAdd(a.dconic + 4 * g + 3, v[kOp]);
      atomicAdd(a.dcolors + 3 * g, v[kR]);
      atomicAdd(a.dcolors + 3 * g + 1, v[kG]);
      atomicAdd(a.dcolors + 3 * g + 2, v[kB]);
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
