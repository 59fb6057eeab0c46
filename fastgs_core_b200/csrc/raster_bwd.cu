// Tile rasterizer backward on sm_100a (fastgs_core/metal/fastgs_rasterize_backward.metal:24-278).
//
// Same gradients as the reference's per-bucket kernel, organised pixel-
// parallel with two pixels per thread. Work is split by buckets, not tiles: a
// CTA takes one bucket (32 splats) of the global bucket list, which bounds
// every CTA's work whatever the tile's splat count; a bucket is a valid
// starting point because the forward pass sampled each pixel's transmittance
// and accumulated colour there. Each warp (four pixel rows) walks the staged
// splats front to back on its own, restarting at each bucket from the forward
// sample (the accumulated colour is kept as its dot product with dL/dpixel,
// which is all the alpha gradient needs). Per splat, a warp skips the splat
// outright when the splat's opacity-aware row extent misses its rows, or when
// no lane's pair passes the alpha test (ballot); otherwise the eleven per-pair
// partials are summed across the warp with a transposed butterfly (13
// shuffles) and added to shared-memory accumulators; at the end, one global
// atomic per splat and output element. Compared with one warp per bucket (the
// reference's layout), this evaluates the same pairs but skips whole warp-splat
// blocks that cannot contribute and avoids the 31-step pipeline fill of the
// lane-to-lane state shift.
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
  const uint32_t* contrib_mask;
  int sparse;  // samples of pixels whose last contributor precedes the bucket are not read
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

// Sum p[0..10] across the warp in 13 shuffles (a transposed butterfly: at each
// level a lane pair splits the values it still holds, each half keeping one
// part and adding the partner's copy of it). Returns the full sum of slot
// `slot` (lanes that end with no slot get slot = -1). Level by level the lane
// bits select: bit 4 -> slots 0-5 / 6-10, bit 3 -> positions 0-2 / 3-5,
// bit 2 -> positions 0-1 / 2, bit 1 -> the position within that, bit 0 -> the
// final pairwise sum.
__device__ __forceinline__ float warp_transpose_sum11(const float (&p)[kSlots], int lane, int& slot) {
  float q[6];
  {
    const bool hi = lane & 16;
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const float up = (6 + i < kSlots) ? p[6 + i] : 0.0f;
      const float send = hi ? p[i] : up;
      const float keep = hi ? up : p[i];
      q[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  float r[3];
  {
    const bool hi = lane & 8;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const float send = hi ? q[i] : q[3 + i];
      const float keep = hi ? q[3 + i] : q[i];
      r[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  float t0, t1;
  {
    const bool hi = lane & 4;
    t0 = (hi ? r[2] : r[0]) + __shfl_xor_sync(0xffffffffu, hi ? r[0] : r[2], 4);
    t1 = (hi ? 0.0f : r[1]) + __shfl_xor_sync(0xffffffffu, r[1], 4);
  }
  float w;
  {
    const bool hi = lane & 2;
    w = (hi ? t1 : t0) + __shfl_xor_sync(0xffffffffu, hi ? t0 : t1, 2);
  }
  w += __shfl_xor_sync(0xffffffffu, w, 1);
  const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1, b1 = (lane >> 1) & 1;
  const int pos = 3 * b3 + (b2 ? 2 + b1 : b1);
  slot = ((lane & 1) || (b2 && b1)) ? -1 : 6 * b4 + pos;
  if (slot >= kSlots) slot = -1;
  return w;
}

__device__ __forceinline__ float2 pk2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 bc2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Per-pair partials of one splat for a thread's two pixels, which share a
// column (one dx) and sit two rows apart (dy.x, dy.y), on the contribution-mask
// path: v0 / v1 say whether the pair contributed in the forward pass. Pixel
// state (T, the remaining-colour dot adot, dL/dpixel d0..d2, and -T_final
// (bg . dL/dpixel) in ntfbg) is packed per pixel pair so that the arithmetic
// issues as f32x2 instructions. The exponential is the fast one except close
// to the 0.99 clamp, where the forward pass's exact arithmetic decides on
// which side of the clamp the pair lies (only that side passes a gradient to
// G). Writes the eleven slot sums of the two pixels into p.
__device__ __forceinline__ void mask_pair_partials(float (&p)[kSlots], const float4 r0,
                                                   const float4 r1, const float4 r2, bool v0,
                                                   bool v1, float pfx, float2 npfy, float2& T,
                                                   float2& adot, float2 d0, float2 d1, float2 d2,
                                                   float2 ntfbg) {
  const float dx = r0.x - pfx;
  const float2 dy = __fadd2_rn(bc2(r0.y), npfy);
  // power = -0.5 (a dx^2 + c dy^2) - b dx dy = -0.5 a dx^2 + dy (-0.5 c dy - b dx)
  const float adx = r0.z * dx, bdx = r0.w * dx;
  const float2 t = __ffma2_rn(bc2(-0.5f * r1.x), dy, bc2(-bdx));
  const float2 power = __ffma2_rn(t, dy, bc2(-0.5f * adx * dx));
  const float2 pl = __fmul2_rn(power, bc2(1.44269504f));
  float2 G = pk2(ex2_approx(pl.x), ex2_approx(pl.y));
  float2 oG = __fmul2_rn(bc2(r1.y), G);
  if (v0 && fabsf(oG.x - 0.99f) < 1e-4f) {
    G.x = fgs_expf_neg(splat_power(r0.z, r0.w, r1.x, dx, dy.x));
    oG.x = __fmul_rn(r1.y, G.x);
  }
  if (v1 && fabsf(oG.y - 0.99f) < 1e-4f) {
    G.y = fgs_expf_neg(splat_power(r0.z, r0.w, r1.x, dx, dy.y));
    oG.y = __fmul_rn(r1.y, G.y);
  }
  const bool vg0 = v0 && !(oG.x > 0.99f), vg1 = v1 && !(oG.y > 0.99f);
  const float2 al = pk2(v0 ? fmin_t(0.99f, oG.x) : 0.0f, v1 ? fmin_t(0.99f, oG.y) : 0.0f);
  const float2 wgt = __fmul2_rn(al, T);
  const float2 om = __ffma2_rn(al, bc2(-1.0f), bc2(1.0f));
  const float2 rec = pk2(__fdividef(1.0f, om.x), __fdividef(1.0f, om.y));
  const float2 cdot =
      __ffma2_rn(bc2(r2.x), d2, __ffma2_rn(bc2(r1.w), d1, __fmul2_rn(bc2(r1.z), d0)));
  adot = __ffma2_rn(wgt, cdot, adot);  // remaining colour after this splat, dotted with dL/dpix
  const float2 dla = __ffma2_rn(T, cdot, __fmul2_rn(rec, __fadd2_rn(adot, ntfbg)));
  T = __fmul2_rn(T, om);
  const float2 cr = __fmul2_rn(wgt, d0), cg = __fmul2_rn(wgt, d1), cb = __fmul2_rn(wgt, d2);
  p[kR] = cr.x + cr.y;
  p[kG] = cg.x + cg.y;
  p[kB] = cb.x + cb.y;
  // dL/dG * G; the constant factors (-W/2, -H/2, -1/2) are applied at the flush
  const float2 u = __fmul2_rn(pk2(vg0 ? oG.x : 0.0f, vg1 ? oG.y : 0.0f), dla);
  const float2 tx = __fmul2_rn(u, __ffma2_rn(bc2(r0.w), dy, bc2(adx)));  // u (a dx + b dy)
  const float2 ty = __fmul2_rn(u, __ffma2_rn(bc2(r1.x), dy, bc2(bdx)));  // u (c dy + b dx)
  p[kMx] = tx.x + tx.y;
  p[kMy] = ty.x + ty.y;
  p[kMxAbs] = fabsf(tx.x) + fabsf(tx.y);
  p[kMyAbs] = fabsf(ty.x) + fabsf(ty.y);
  const float2 udy = __fmul2_rn(u, dy);
  const float usum = u.x + u.y;
  p[kCx] = usum * dx * dx;
  p[kCy] = (udy.x + udy.y) * dx;
  p[kCw] = fmaf(udy.x, dy.x, udy.y * dy.y);
  const float2 og = __fmul2_rn(pk2(vg0 ? G.x : 0.0f, vg1 ? G.y : 0.0f), dla);
  p[kOp] = og.x + og.y;
}

// splats staged per CTA: one bucket (config 3, B200: 1.17 ms; 2 buckets 1.19,
// 4 buckets 1.24, 8 buckets 1.26)
constexpr int kChunk = 32;
constexpr int kBwdPixelsPerThread = 2;
// contribution-mask path with packed pixel pairs (config 3: 0.855 ms; four
// pixels per thread 0.967 ms)
constexpr int kBwdMaskPx = 2;

// One CTA per group of kGroupBuckets consecutive buckets of the global bucket
// list (kChunk splats at most), so that every CTA carries the same bounded work
// whatever the per-tile splat counts (tiles of this workload range from a few
// splats to thousands). A group may cover the tail of one tile and the head of
// the next: the warps walk it bucket by bucket, loading a tile's pixel state
// when the tile changes and the forward sample (T, accumulated colour) at every
// bucket start, which is what makes a bucket a valid starting point.
//
// PX pixels per thread: a warp covers 2*PX consecutive pixel rows of the tile
// (lane l: column l % 16, rows base + l / 16 + 2k), so the cross-lane reduction
// of a splat's partials is shared by 32*PX pixels.
constexpr int kGroupBuckets = kChunk / 32;

template <int PX, bool kMask>
// no occupancy cap: 48 registers (capping at 40 / 32 for 12 / 14 CTAs per SM
// spills and measured 10% / 20% slower on config 3)
__global__ void __launch_bounds__(kTilePx / PX) raster_bwd_kernel(BwdArgs a) {
  constexpr int kThreads = kTilePx / PX;
  constexpr int kWarpRows = 2 * PX;
  // splat records of the group
  __shared__ float4 s_r0[kChunk];  // x, y, conic.a, conic.b
  __shared__ float4 s_r1[kChunk];  // conic.c, opacity, r, g
  __shared__ float4 s_r2[kChunk];  // b, exponent cut, -, warp bands (bits)
  __shared__ uint32_t s_id[kChunk];
  __shared__ float s_acc[kChunk][kSlots];
  __shared__ int s_btile[kGroupBuckets];   // tile of each bucket
  __shared__ int s_blocal[kGroupBuckets];  // bucket index within its tile
  __shared__ int s_bcount[kGroupBuckets];  // splats of the bucket to walk (0: skip)
  __shared__ uint32_t s_bfirst[kGroupBuckets];  // key index of the bucket's first splat

  const int lr = threadIdx.x, lane = lr & 31, warp = lr >> 5;
  const int wrow = warp * kWarpRows;
  const int64_t gb0 = (int64_t)blockIdx.x * kGroupBuckets;
  if (lr < kGroupBuckets) {
    const int64_t b = gb0 + lr;
    int tile = -1, local = 0, count = 0;
    uint32_t first = 0;
    if (b < a.bucket_sum) {
      const uint32_t t = a.bucket_to_tile[b];
      if (t < (uint32_t)a.num_tiles) {
        tile = (int)t;
        const uint32_t bbm0 = (t == 0) ? 0u : a.bucket_offsets[t - 1];
        const uint2 range = a.ranges[t];
        const int nsplat = (int)(range.y - range.x);
        // splats at or past max_contrib touch no pixel (reference:
        // fastgs_rasterize_backward.metal:72-74)
        const int nact = min(nsplat, (int)((a.max_contrib[t] + 31u) / 32u) * 32);
        local = (int)((uint32_t)b - bbm0);
        count = max(0, min(32, nact - 32 * local));
        first = range.x + 32u * (uint32_t)local;
      }
    }
    s_btile[lr] = count > 0 ? tile : -1;
    s_blocal[lr] = local;
    s_bcount[lr] = count;
    s_bfirst[lr] = first;
  }
  __syncthreads();
  {
    int total = 0;
#pragma unroll
    for (int i = 0; i < kGroupBuckets; ++i) total += s_bcount[i];
    if (total == 0) return;  // uniform: no barrier follows for this CTA
  }
  for (int q = lr; q < kChunk; q += kThreads) {
    const int bi = q >> 5;
    uint32_t g = 0xffffffffu;
    if ((q & 31) < s_bcount[bi]) {
      const int t = s_btile[bi];
      g = a.point_list[s_bfirst[bi] + (q & 31)];
      const float2 xy = a.means2d[g];
      const float4 co = a.conic[g];
      // warps (bands of kWarpRows tile rows) the splat can reach
      uint32_t bands = (1u << (kThreads / 32)) - 1u;
      if (!kMask) {
        int rlo, rhi;
        bwd_splat_rows(xy.y, co.x, co.y, co.z, co.w, (t / a.gx) * FGS_BLOCK, rlo, rhi);
        bands = 0u;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w)
          if (rhi >= w * kWarpRows && rlo <= w * kWarpRows + kWarpRows - 1) bands |= 1u << w;
      }
      s_r0[q] = make_float4(xy.x, xy.y, co.x, co.y);
      s_r1[q] = make_float4(co.z, co.w, a.colors[3 * (size_t)g], a.colors[3 * (size_t)g + 1]);
      s_r2[q] = make_float4(a.colors[3 * (size_t)g + 2], power_cut(co.w), 0.0f, __uint_as_float(bands));
    }
    s_id[q] = g;
  }
  for (int k = lr; k < kChunk * kSlots; k += kThreads) (&s_acc[0][0])[k] = 0.0f;
  __syncthreads();

  const size_t P = (size_t)a.W * a.H;
  const float hw = 0.5f * (float)a.W, hh = 0.5f * (float)a.H;
  int lpix[PX];  // pixel index within the tile
  float pfx[PX], pfy[PX], d0[PX], d1[PX], d2[PX], tfbg[PX], pcd[PX], T[PX], adot[PX];
  int last[PX];
  uint32_t msk[PX];  // contrib_mask of the current bucket (kMask)
#pragma unroll
  for (int k = 0; k < PX; ++k) msk[k] = 0u;
  int cur_tile = -1;
  for (int bi = 0; bi < kGroupBuckets; ++bi) {
    const int cnt = s_bcount[bi];
    if (cnt == 0) continue;  // uniform
    const int tile = s_btile[bi];
    if (tile != cur_tile) {
      // the pixel state of a new tile
      cur_tile = tile;
      const int pminx = (tile % a.gx) * FGS_BLOCK, pminy = (tile / a.gx) * FGS_BLOCK;
#pragma unroll
      for (int k = 0; k < PX; ++k) {
        const int row = wrow + (lane >> 4) + 2 * k;
        lpix[k] = row * FGS_BLOCK + (lane & 15);
        const int px = pminx + (lane & 15), py = pminy + row;
        pfx[k] = (float)px;
        pfy[k] = (float)py;
        d0[k] = d1[k] = d2[k] = tfbg[k] = pcd[k] = 0.f;
        last[k] = 0;
        if (px < a.W && py < a.H) {
          const size_t pix = (size_t)py * a.W + px;
          d0[k] = a.dL_dout[pix];
          d1[k] = a.dL_dout[P + pix];
          d2[k] = a.dL_dout[2 * P + pix];
          tfbg[k] = a.final_t[pix] * (a.bg[0] * d0[k] + a.bg[1] * d1[k] + a.bg[2] * d2[k]);
          // final colour . dL/dpix: the per-bucket remaining-colour dot starts
          // from (sampled colour - final colour) . dL/dpix
          pcd[k] = a.pixel_colors[pix] * d0[k] + a.pixel_colors[P + pix] * d1[k] +
                   a.pixel_colors[2 * P + pix] * d2[k];
          last[k] = (int)a.n_contrib[pix];
        }
      }
    }
    {
      // bucket start: the forward sample of each pixel
      const size_t bucket = (size_t)(gb0 + bi);
      const int bstart = 32 * s_blocal[bi];
#pragma unroll
      for (int k = 0; k < PX; ++k) {
        if (a.sparse && last[k] <= bstart) {
          // no splat of this bucket contributes to the pixel: its sample was
          // not written, and none of the values below is used
          T[k] = 0.0f;
          adot[k] = 0.0f;
          msk[k] = 0u;
          continue;
        }
        T[k] = a.sampled_t[bucket * kTilePx + lpix[k]];
        const float* sar = a.sampled_ar + bucket * 3 * kTilePx + lpix[k];
        adot[k] = sar[0] * d0[k] + sar[kTilePx] * d1[k] + sar[2 * kTilePx] * d2[k] - pcd[k];
        if (kMask) msk[k] = a.contrib_mask[bucket * kTilePx + lpix[k]];
      }
    }
    uint32_t mor = 0u;  // pairs of this thread that contributed, any pixel
#pragma unroll
    for (int k = 0; k < PX; ++k) mor |= msk[k];
    const int sbase = 32 * s_blocal[bi];
    // the bucket's splats to walk; with the mask, only those that contributed
    // to one of this warp's pixels (warp-uniform)
    uint32_t todo = cnt == 32 ? 0xffffffffu : ((1u << cnt) - 1u);
    if constexpr (kMask) todo &= __reduce_or_sync(0xffffffffu, mor);
    for (; todo != 0u; todo &= todo - 1u) {
      const int jj = __ffs(todo) - 1;
      const int j = 32 * bi + jj;  // staged record
      const int s = sbase + jj;    // splat index within the tile
      bool v[PX], vg[PX];
      float dx[PX], dy[PX], G[PX], oG[PX], alpha[PX];
      float4 r0, r1, r2;
      if constexpr (kMask) {
        // the forward pass recorded which pairs contributed (the walk skips
        // splats none of this warp's pairs took part in); the exponential is
        // the fast intrinsic, except close to the 0.99 clamp, whose side
        // decides whether G receives a gradient and is therefore taken from
        // the forward pass's exact arithmetic
        r0 = s_r0[j];
        r1 = s_r1[j];
        r2 = s_r2[j];
#pragma unroll
        for (int k = 0; k < PX; ++k) {
          v[k] = (msk[k] >> jj) & 1u;
          if constexpr (PX % 2 == 0) continue;  // the packed path below evaluates the pairs
          dx[k] = r0.x - pfx[k];
          dy[k] = r0.y - pfy[k];
          const float power =
              -0.5f * (r0.z * dx[k] * dx[k] + r1.x * dy[k] * dy[k]) - r0.w * dx[k] * dy[k];
          G[k] = __expf(power);
          oG[k] = r1.y * G[k];
          if (v[k] && fabsf(oG[k] - 0.99f) < 1e-4f) {
            G[k] = fgs_expf_neg(splat_power(r0.z, r0.w, r1.x, dx[k], dy[k]));
            oG[k] = __fmul_rn(r1.y, G[k]);
          }
          alpha[k] = fmin_t(0.99f, oG[k]);
          vg[k] = v[k] && !(oG[k] > 0.99f);
        }
      } else {
        r2 = s_r2[j];
        // warp-uniform: the splat cannot reach this warp's rows
        if (!((__float_as_uint(r2.w) >> warp) & 1u)) continue;
        r0 = s_r0[j];
        r1 = s_r1[j];
        // Branch-free per pair: every lane evaluates the exponential (on 0
        // for pairs that fail the exponent test, whose result is discarded),
        // and an invalid pair enters the gradient arithmetic with alpha = 0
        // and G = 0, so it leaves T and the remaining-colour dot unchanged
        // and adds zeros.
        bool any = false;
#pragma unroll
        for (int k = 0; k < PX; ++k) {
          dx[k] = r0.x - pfx[k];
          dy[k] = r0.y - pfy[k];
          const float power = splat_power(r0.z, r0.w, r1.x, dx[k], dy[k]);
          // same decisions as the forward pass (NaN exponents included)
          const bool pre = (s < last[k]) && !(power > 0.0f) && !(power <= r2.y);
          G[k] = fgs_expf_neg(pre ? power : 0.0f);
          oG[k] = __fmul_rn(r1.y, G[k]);
          alpha[k] = fmin_t(0.99f, oG[k]);
          v[k] = pre && alpha[k] >= 1.0f / 255.0f;
          vg[k] = v[k] && !(oG[k] > 0.99f);
          any |= v[k];
        }
        if (__ballot_sync(0xffffffffu, any) == 0u) continue;  // warp-uniform
      }
      float p[kSlots];
      if constexpr (kMask && PX % 2 == 0) {
        // a thread's pixels share a column (dx) and sit two rows apart: their
        // arithmetic runs as packed pairs (one f32x2 instruction per two
        // lanes' worth of work on the issue-bound pipe)
#pragma unroll
        for (int k = 0; k < PX; k += 2) {
          float2 T2 = pk2(T[k], T[k + 1]), ad2 = pk2(adot[k], adot[k + 1]);
          float pk[kSlots];
          mask_pair_partials(k == 0 ? p : pk, r0, r1, r2, v[k], v[k + 1], pfx[0],
                             pk2(-pfy[k], -pfy[k + 1]), T2, ad2, pk2(d0[k], d0[k + 1]),
                             pk2(d1[k], d1[k + 1]), pk2(d2[k], d2[k + 1]),
                             pk2(-tfbg[k], -tfbg[k + 1]));
          if (k > 0) {
#pragma unroll
            for (int q = 0; q < kSlots; ++q) p[q] += pk[q];
          }
          T[k] = T2.x;
          T[k + 1] = T2.y;
          adot[k] = ad2.x;
          adot[k + 1] = ad2.y;
        }
      } else {
#pragma unroll
      for (int q = 0; q < kSlots; ++q) p[q] = 0.0f;
      const float c0c = r1.z, c1c = r1.w, c2c = r2.x;
#pragma unroll
      for (int k = 0; k < PX; ++k) {
        const float al = v[k] ? alpha[k] : 0.0f;
        const float wgt = al * T[k];
        const float rec = __fdividef(1.0f, 1.0f - al);
        const float cdot = c0c * d0[k] + c1c * d1[k] + c2c * d2[k];
        adot[k] += wgt * cdot;  // remaining colour after this splat, dotted with dL/dpix
        const float dL_dalpha = T[k] * cdot + rec * (adot[k] - tfbg[k]);
        T[k] *= (1.0f - al);
        p[kR] += wgt * d0[k];
        p[kG] += wgt * d1[k];
        p[kB] += wgt * d2[k];
        // dL/dG * G; the constant factors (-W/2, -H/2, -1/2) are applied at the flush
        const float u = (vg[k] ? oG[k] : 0.0f) * dL_dalpha;
        const float tmp_x = u * (r0.z * dx[k] + r0.w * dy[k]);
        const float tmp_y = u * (r1.x * dy[k] + r0.w * dx[k]);
        p[kMx] += tmp_x;
        p[kMy] += tmp_y;
        p[kMxAbs] += fabsf(tmp_x);
        p[kMyAbs] += fabsf(tmp_y);
        const float udx = u * dx[k];
        p[kCx] += udx * dx[k];
        p[kCy] += udx * dy[k];
        p[kCw] += u * dy[k] * dy[k];
        p[kOp] += (vg[k] ? G[k] : 0.0f) * dL_dalpha;
      }
      }
      int slot;
      const float tot = warp_transpose_sum11(p, lane, slot);
      if (slot >= 0) atomicAdd(&s_acc[j][slot], tot);
    }
  }
  __syncthreads();
  for (int q = lr; q < kChunk; q += kThreads) {
    const uint32_t gid = s_id[q];
    if (gid == 0xffffffffu) continue;
    const size_t g = gid;
    const float* vv = s_acc[q];
    const float mx = -hw * vv[kMx], my = -hh * vv[kMy];
    atomicAdd(a.dmeans2d + 2 * g, mx);
    atomicAdd(a.dmeans2d + 2 * g + 1, my);
    atomicAdd(a.dviewspace + 4 * g, mx);
    atomicAdd(a.dviewspace + 4 * g + 1, my);
    atomicAdd(a.dviewspace + 4 * g + 2, hw * vv[kMxAbs]);
    atomicAdd(a.dviewspace + 4 * g + 3, hh * vv[kMyAbs]);
    atomicAdd(a.dconic + 4 * g, -0.5f * vv[kCx]);
    atomicAdd(a.dconic + 4 * g + 1, -0.5f * vv[kCy]);
    atomicAdd(a.dconic + 4 * g + 2, -0.5f * vv[kCw]);
    atomicAdd(a.dconic + 4 * g + 3, vv[kOp]);
    atomicAdd(a.dcolors + 3 * g, vv[kR]);
    atomicAdd(a.dcolors + 3 * g + 1, vv[kG]);
    atomicAdd(a.dcolors + 3 * g + 2, vv[kB]);
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
  FGS_CHECK_ARG(FGS_ALIGNED(ranges, 8) && FGS_ALIGNED(means2d, 8) && FGS_ALIGNED(conic_opacity, 16),
                "ranges and means2d must be 8-byte, conic_opacity 16-byte aligned");
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
  // two pixels per thread (measured on config 3: 1.68 ms vs 1.91 ms with one
  // and 1.98 ms with four, where occupancy drops)
  const int64_t groups = (p->bucket_sum + kGroupBuckets - 1) / kGroupBuckets;
  FGS_CHECK_ARG(groups <= 0x7fffffff, "too many buckets");
  a.contrib_mask = p->contrib_mask;
  a.sparse = p->sparse_samples != 0;
  if (a.contrib_mask)
    raster_bwd_kernel<kBwdMaskPx, true><<<(unsigned)groups, kTilePx / kBwdMaskPx, 0, s>>>(a);
  else
    raster_bwd_kernel<kBwdPixelsPerThread, false><<<(unsigned)groups, kTilePx / kBwdPixelsPerThread, 0, s>>>(a);
  return check_launch("rasterize_backward");
}

}  // extern "C"
