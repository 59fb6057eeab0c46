// FastGS exact ellipse / tile-row intersection walk, shared by the preprocess
// (count only) and duplicate-with-keys (emit keys) kernels so both produce the
// same tiles. Follows fastgs_core/metal/fastgs_preprocess.metal:247-382 and
// fastgs_core/metal/fastgs_binning.metal:23-180 operation for operation.
#pragma once
#include "fgs_common.cuh"

namespace fgs {

// intersections of the opacity-aware ellipse with the line u = coord
// (is_y: u is the y axis); returns (low, high) on the other axis
__device__ __forceinline__ void ellipse_line(const float4 co, float disc, float t, float px,
                                             float py, bool is_y, float coord, float& lo,
                                             float& hi) {
  const float p_u = is_y ? py : px;
  const float p_v = is_y ? px : py;
  const float coeff = is_y ? co.x : co.z;
  const float h = coord - p_u;
  const float sq = sqrtf(disc * h * h + t * coeff);
  lo = (-co.y * h - sq) / coeff + p_v;
  hi = (-co.y * h + sq) / coeff + p_v;
}

// Walks the tiles covered by the Gaussian at pixel (px, py) with conic/opacity
// `co`. Emit(tile_id) is called once per covered tile in walk order; returns
// the count (the reference's tiles_touched).
template <typename Emit>
__device__ __forceinline__ uint32_t tile_walk(float px, float py, const float4 co, int gx, int gy,
                                              float mult, Emit&& emit) {
  const float disc = co.y * co.y - co.x * co.z;
  if (co.x <= 0.0f || co.z <= 0.0f || disc >= 0.0f) return 0u;
  float t = 2.0f * fgs_logf(co.w * 255.0f);
  t = mult * t;
  float x_term = sqrtf(-(co.y * co.y * t) / (disc * co.x));
  x_term = (co.y < 0.0f) ? x_term : -x_term;
  float y_term = sqrtf(-(co.y * co.y * t) / (disc * co.z));
  y_term = (co.y < 0.0f) ? y_term : -y_term;
  float am_x = py - y_term, am_y = px - x_term;
  float aM_x = py + y_term, aM_y = px + x_term;
  float lo, hi;
  float bmin_x, bmin_y, bmax_x, bmax_y;
  ellipse_line(co, disc, t, px, py, true, am_x, lo, hi);
  bmin_x = lo;
  ellipse_line(co, disc, t, px, py, false, am_y, lo, hi);
  bmin_y = lo;
  ellipse_line(co, disc, t, px, py, true, aM_x, lo, hi);
  bmax_x = hi;
  ellipse_line(co, disc, t, px, py, false, aM_y, lo, hi);
  bmax_y = hi;
  int rmin_x = imax(0, imin(gx, f2i(bmin_x / 16.0f)));
  int rmin_y = imax(0, imin(gy, f2i(bmin_y / 16.0f)));
  int rmax_x = imax(0, imin(gx, f2i(bmax_x / 16.0f + 1.0f)));
  int rmax_y = imax(0, imin(gy, f2i(bmax_y / 16.0f + 1.0f)));
  const int y_span = rmax_y - rmin_y, x_span = rmax_x - rmin_x;
  if (y_span * x_span == 0) return 0u;
  const bool is_y = y_span < x_span;
  if (is_y) {
    int ti;
    float tf;
    ti = rmin_x; rmin_x = rmin_y; rmin_y = ti;
    ti = rmax_x; rmax_x = rmax_y; rmax_y = ti;
    tf = bmin_x; bmin_x = bmin_y; bmin_y = tf;
    tf = bmax_x; bmax_x = bmax_y; bmax_y = tf;
    tf = am_x; am_x = am_y; am_y = tf;
    tf = aM_x; aM_x = aM_y; aM_y = tf;
  }
  uint32_t count = 0;
  float imin_lo, imin_hi;
  float imax_lo = bmax_y, imax_hi = bmin_y;
  float min_line = (float)rmin_x * 16.0f;
  if (bmin_x <= min_line) {
    ellipse_line(co, disc, t, px, py, is_y, (float)rmin_x * 16.0f, imin_lo, imin_hi);
  } else {
    imin_lo = imax_lo;
    imin_hi = imax_hi;
  }
  for (int u = rmin_x; u < rmax_x; ++u) {
    const float max_line = min_line + 16.0f;
    if (max_line <= bmax_x) ellipse_line(co, disc, t, px, py, is_y, max_line, imax_lo, imax_hi);
    float e_min, e_max;
    if (min_line <= am_y && am_y < max_line)
      e_min = bmin_y;
    else
      e_min = fmin_t(imin_lo, imax_lo);
    if (min_line <= aM_y && aM_y < max_line)
      e_max = bmax_y;
    else
      e_max = fmax_t(imin_hi, imax_hi);
    const int v0 = imax(rmin_y, imin(rmax_y, f2i(e_min / 16.0f)));
    const int v1 = imin(rmax_y, imax(rmin_y, f2i(e_max / 16.0f + 1.0f)));
    for (int v = v0; v < v1; ++v) emit(is_y ? (u * gx + v) : (v * gx + u));
    count += (uint32_t)(v1 - v0);
    imin_lo = imax_lo;
    imin_hi = imax_hi;
    min_line = max_line;
  }
  return count;
}

}  // namespace fgs
