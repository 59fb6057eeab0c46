/*
 * CPU oracle for the FastGS tile rasterizer hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Imported by tests/, by __graft_entry__.smoke() and
 * by bench.py's CPU-baseline / reference arm, always as the checker or the
 * timed CPU baseline, never as part of the product path.
 *
 * A statement-by-statement restatement in C of the reference kernels
 * (paths relative to the reference project):
 *   fastgs_core/metal/fastgs_preprocess.metal           preprocess forward
 *   fastgs_core/metal/fastgs_binning.metal              duplicate-with-keys
 *   fastgs_core/metal/fastgs_tile_prep.metal            tile ranges, bucket counts
 *   fastgs_core/metal/fastgs_rasterize.metal            render forward
 *   fastgs_core/metal/fastgs_rasterize_backward.metal   render backward
 *   fastgs_core/metal/fastgs_preprocess_backward.metal  preprocess backward
 *   fastgs_core/binding/binding.cpp:153-212             cumsum / argsort / take
 * Each function below names the lines it follows.
 *
 * Arithmetic contract (the reference builds with Metal fast-math, so its own
 * rounding is unspecified; this file fixes one reading of it):
 *   - every float operation is a separate IEEE-754 binary32 op, evaluated in
 *     the source order of the reference expression (build: -ffp-contract=off);
 *   - Metal float3x3 is column-major (m[col][row]); products sum left to right;
 *   - min(a,b) = b<a ? b : a, max(a,b) = a<b ? b : a (the reference's template
 *     reading; NaN selects the first operand);
 *   - float->int conversion truncates toward zero, saturates, NaN -> 0;
 *   - exp/log: with FGS_ORACLE_LIBM they are libm expf/logf and every
 *     expression keeps the reference's unfused operations (this build is
 *     pinned bit-for-bit against the reference kernels compiled on this CPU);
 *     otherwise ("gpu" mode) they are fgs_expf/fgs_logf below and the
 *     per-splat colour accumulation is one fused multiply-add, exactly as
 *     the CUDA kernels compute them, so integer outputs (tiles touched, keys,
 *     ranges, n_contrib) and the rendered image are bit-identical between
 *     this oracle and the GPU.
 *
 * Defined behaviour where the reference's is undefined:
 *   - max_contrib is the max of n_contrib over in-image pixels of the tile
 *     (fastgs_rasterize.metal:77-79 returns out-of-image threads before the
 *     barrier at :143, so the reference reads unwritten slots).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BLOCK 16

/* ------------------------------------------------------------------ math */

/* e^x for binary32. Cody-Waite reduction x = k ln2 + r with ln2 split in a
 * 24-bit high part and a low part, |r| <= ln2/2, then the degree-7 Taylor
 * polynomial of e^r (coefficients 1/j!) in Horner form with fused
 * multiply-adds, scaled by 2^k through the exponent field. Inputs below -87
 * return 0 and above 88 return +inf. Max error about 1 ulp. */
static inline float fgs_expf(float x) {
  if (!(x > -87.0f)) return (x != x) ? x : 0.0f;
  if (x > 88.0f) return INFINITY;
  const float k = rintf(x * 1.44269502f);
  float r = fmaf(k, -0.693145752f, x);  /* ln2 high: 0x3f317200 */
  r = fmaf(k, -1.42860677e-06f, r);      /* ln2 - high */
  float p = 1.98412701e-04f;             /* 1/7! */
  p = fmaf(p, r, 1.38888892e-03f);       /* 1/6! */
  p = fmaf(p, r, 8.33333377e-03f);       /* 1/5! */
  p = fmaf(p, r, 4.16666679e-02f);       /* 1/4! */
  p = fmaf(p, r, 1.66666672e-01f);       /* 1/3! */
  p = fmaf(p, r, 5.00000000e-01f);       /* 1/2! */
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ki = (int)k;
  /* 2^k as two factors so that k down to -126 stays normal */
  const int k1 = ki / 2, k2 = ki - k1;
  union { uint32_t u; float f; } s1, s2;
  s1.u = (uint32_t)(k1 + 127) << 23;
  s2.u = (uint32_t)(k2 + 127) << 23;
  return (p * s1.f) * s2.f;
}

/* ln(x) for binary32. x = m 2^e with m in [sqrt(1/2), sqrt(2)),
 * ln(m) = 2 atanh(s), s = (m-1)/(m+1), atanh series to s^11 (|s| <= 0.1716,
 * truncation < 1e-11), ln(x) = e ln2 + ln(m) with ln2 split high/low.
 * x <= 0 gives -inf (x == 0) or NaN; subnormal x is scaled first. */
static inline float fgs_logf(float x) {
  if (x != x || x < 0.0f) return NAN;
  if (x == 0.0f) return -INFINITY;
  if (x == INFINITY) return x;
  union { float f; uint32_t u; } v;
  v.f = x;
  int e = 0;
  if (v.u < 0x00800000u) { /* subnormal */
    v.f = x * 16777216.0f;
    e = -24;
  }
  e += (int)((v.u >> 23) & 0xffu) - 127;
  v.u = (v.u & 0x007fffffu) | 0x3f800000u; /* m in [1, 2) */
  if (v.f > 1.41421354f) {
    v.f = v.f * 0.5f;
    e += 1;
  }
  const float m = v.f;
  const float s = (m - 1.0f) / (m + 1.0f);
  const float s2 = s * s;
  float q = 9.09090936e-02f;       /* 1/11 */
  q = fmaf(q, s2, 1.11111112e-01f); /* 1/9 */
  q = fmaf(q, s2, 1.42857149e-01f); /* 1/7 */
  q = fmaf(q, s2, 2.00000003e-01f); /* 1/5 */
  q = fmaf(q, s2, 3.33333343e-01f); /* 1/3 */
  const float ln_m = fmaf(2.0f * s * s2, q, 2.0f * s);
  const float fe = (float)e;
  return fmaf(fe, 0.693145752f, fmaf(fe, 1.42860677e-06f, ln_m));
}

#ifdef FGS_ORACLE_LIBM
#define O_EXP(x) expf(x)
#define O_LOG(x) logf(x)
/* colour accumulation c += (col * alpha) * T as rounded ops, in the
   reference's order (fastgs_rasterize.metal:122) */
#define O_ACC(c, col, alpha, t) ((c) + ((col) * (alpha)) * (t))
#else
#define O_EXP(x) fgs_expf(x)
#define O_LOG(x) fgs_logf(x)
/* the CUDA kernels weight once per pair and fuse the accumulation:
   w = alpha * T (rounded), c = fma(col, w, c) */
#define O_ACC(c, col, alpha, t) fmaf((col), (alpha) * (t), (c))
#endif

static inline float fmin_t(float a, float b) { return b < a ? b : a; }
static inline float fmax_t(float a, float b) { return a < b ? b : a; }
static inline int imin(int a, int b) { return b < a ? b : a; }
static inline int imax(int a, int b) { return a < b ? b : a; }

/* truncating, saturating float -> int; NaN -> 0 */
static inline int f2i(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return 2147483647;
  if (v <= -2147483648.0f) return (int)0x80000000;
  return (int)v;
}

typedef struct { float x, y, z; } v3;
typedef struct { v3 c[3]; } m3; /* column-major: c[col] */

static inline v3 V3(float x, float y, float z) { v3 r = {x, y, z}; return r; }
static inline float v3_at(v3 v, int i) { return i == 0 ? v.x : (i == 1 ? v.y : v.z); }
static inline m3 M3(float a0, float a1, float a2, float a3, float a4, float a5, float a6,
                    float a7, float a8) {
  m3 m;
  m.c[0] = V3(a0, a1, a2);
  m.c[1] = V3(a3, a4, a5);
  m.c[2] = V3(a6, a7, a8);
  return m;
}
static inline float m3_at(const m3* m, int col, int row) { return v3_at(m->c[col], row); }
static inline v3 m3_mulv(const m3* m, v3 v) {
  return V3(m->c[0].x * v.x + m->c[1].x * v.y + m->c[2].x * v.z,
            m->c[0].y * v.x + m->c[1].y * v.y + m->c[2].y * v.z,
            m->c[0].z * v.x + m->c[1].z * v.y + m->c[2].z * v.z);
}
static inline m3 m3_mul(const m3* a, const m3* b) {
  m3 r;
  for (int j = 0; j < 3; ++j) r.c[j] = m3_mulv(a, b->c[j]);
  return r;
}
static inline m3 m3_tr(const m3* a) {
  return M3(a->c[0].x, a->c[1].x, a->c[2].x, a->c[0].y, a->c[1].y, a->c[2].y, a->c[0].z,
            a->c[1].z, a->c[2].z);
}
static inline m3 m3_scale(float s, const m3* a) {
  m3 r;
  for (int j = 0; j < 3; ++j) r.c[j] = V3(s * a->c[j].x, s * a->c[j].y, s * a->c[j].z);
  return r;
}
static inline float dot3(v3 a, v3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }

static const float SH_C0 = 0.28209479177387814f;
static const float SH_C1 = 0.4886025119029199f;
static const float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                               -1.0925484305920792f, 0.5462742152960396f};
static const float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                               0.3731763325901154f,  -0.4570457994644658f, 1.445305721320277f,
                               -0.5900435899266435f};

/* ------------------------------------------------------- preprocess fwd */

typedef struct {
  int degree, max_sh_coeffs;
  float scale_modifier, mult, tan_fovx, tan_fovy, focal_x, focal_y;
  int image_width, image_height, grid_x, grid_y;
  int use_cov3d_precomp, use_colors_precomp;
} o_pre_params;

/* fastgs_preprocess.metal:46-48 */
static inline float ndc2pix(float v, int s) { return ((v + 1.0f) * (float)s - 1.0f) * 0.5f; }

/* fastgs_preprocess.metal:207-231 */
static void o_cov3d(v3 scale, float mod, const float* rot, float* cov) {
  m3 s = M3(1.f, 0.f, 0.f, 0.f, 1.f, 0.f, 0.f, 0.f, 1.f);
  s.c[0].x = mod * scale.x;
  s.c[1].y = mod * scale.y;
  s.c[2].z = mod * scale.z;
  const float r = rot[0], x = rot[1], y = rot[2], z = rot[3];
  m3 rm = M3(1.f - 2.f * (y * y + z * z), 2.f * (x * y - r * z), 2.f * (x * z + r * y),
             2.f * (x * y + r * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - r * x),
             2.f * (x * z - r * y), 2.f * (y * z + r * x), 1.f - 2.f * (x * x + y * y));
  m3 m = m3_mul(&s, &rm);
  m3 mt = m3_tr(&m);
  m3 sig = m3_mul(&mt, &m);
  cov[0] = sig.c[0].x;
  cov[1] = sig.c[0].y;
  cov[2] = sig.c[0].z;
  cov[3] = sig.c[1].y;
  cov[4] = sig.c[1].z;
  cov[5] = sig.c[2].z;
}

static inline v3 xform43(v3 p, const float* m) {
  return V3(m[0] * p.x + m[4] * p.y + m[8] * p.z + m[12],
            m[1] * p.x + m[5] * p.y + m[9] * p.z + m[13],
            m[2] * p.x + m[6] * p.y + m[10] * p.z + m[14]);
}

/* fastgs_preprocess.metal:171-205 */
static v3 o_cov2d(v3 mean, float fx, float fy, float tanx, float tany, const float* c3,
                  const float* vm) {
  v3 t = xform43(mean, vm);
  const float limx = 1.3f * tanx, limy = 1.3f * tany;
  const float txtz = t.x / t.z, tytz = t.y / t.z;
  t.x = fmin_t(limx, fmax_t(-limx, txtz)) * t.z;
  t.y = fmin_t(limy, fmax_t(-limy, tytz)) * t.z;
  m3 j = M3(fx / t.z, 0.0f, -(fx * t.x) / (t.z * t.z), 0.0f, fy / t.z, -(fy * t.y) / (t.z * t.z),
            0.0f, 0.0f, 0.0f);
  m3 w = M3(vm[0], vm[1], vm[2], vm[4], vm[5], vm[6], vm[8], vm[9], vm[10]);
  m3 tm = m3_mul(&w, &j);
  m3 vrk = M3(c3[0], c3[1], c3[2], c3[1], c3[3], c3[4], c3[2], c3[4], c3[5]);
  m3 tmt = m3_tr(&tm), vrkt = m3_tr(&vrk);
  m3 a = m3_mul(&tmt, &vrkt);
  m3 cov = m3_mul(&a, &tm);
  cov.c[0].x += 0.3f;
  cov.c[1].y += 0.3f;
  return V3(cov.c[0].x, cov.c[0].y, cov.c[1].y);
}

/* fastgs_preprocess.metal:247-260 (is_y selects the walk axis) */
static inline void o_ellipse_x(const float* co, float disc, float t, float px, float py, int is_y,
                               float coord, float* lo, float* hi) {
  const float p_u = is_y ? py : px;
  const float p_v = is_y ? px : py;
  const float coeff = is_y ? co[0] : co[2];
  const float h = coord - p_u;
  const float sq = sqrtf(disc * h * h + t * coeff);
  *lo = (-co[1] * h - sq) / coeff + p_v;
  *hi = (-co[1] * h + sq) / coeff + p_v;
}

/* Shared tile walk of fastgs_preprocess.metal:262-382 and
 * fastgs_binning.metal:39-180. With keys == NULL it only counts; otherwise it
 * writes (tile << 32 | depth bits, idx) at keys/values[off...]. */
static uint32_t o_tile_walk(float px, float py, const float* co, int gx, int gy, float mult,
                            uint32_t idx, float depth, uint64_t* keys, uint32_t* values,
                            uint64_t off) {
  const float disc = co[1] * co[1] - co[0] * co[2];
  if (co[0] <= 0.0f || co[2] <= 0.0f || disc >= 0.0f) return 0u;
  float t = 2.0f * O_LOG(co[3] * 255.0f);
  t = mult * t;
  float x_term = sqrtf(-(co[1] * co[1] * t) / (disc * co[0]));
  x_term = (co[1] < 0.0f) ? x_term : -x_term;
  float y_term = sqrtf(-(co[1] * co[1] * t) / (disc * co[2]));
  y_term = (co[1] < 0.0f) ? y_term : -y_term;
  /* float2 bbox_argmin = (p.y - y_term, p.x - x_term) */
  float am_x = py - y_term, am_y = px - x_term;
  float aM_x = py + y_term, aM_y = px + x_term;
  float lo, hi;
  float bmin_x, bmin_y, bmax_x, bmax_y;
  o_ellipse_x(co, disc, t, px, py, 1, am_x, &lo, &hi);
  bmin_x = lo;
  o_ellipse_x(co, disc, t, px, py, 0, am_y, &lo, &hi);
  bmin_y = lo;
  o_ellipse_x(co, disc, t, px, py, 1, aM_x, &lo, &hi);
  bmax_x = hi;
  o_ellipse_x(co, disc, t, px, py, 0, aM_y, &lo, &hi);
  bmax_y = hi;
  int rmin_x = imax(0, imin(gx, f2i(bmin_x / BLOCK)));
  int rmin_y = imax(0, imin(gy, f2i(bmin_y / BLOCK)));
  int rmax_x = imax(0, imin(gx, f2i(bmax_x / BLOCK + 1)));
  int rmax_y = imax(0, imin(gy, f2i(bmax_y / BLOCK + 1)));
  const int y_span = rmax_y - rmin_y, x_span = rmax_x - rmin_x;
  if (y_span * x_span == 0) return 0u;
  const int is_y = y_span < x_span;
  /* process_tiles: swap to (u, v) = walk axis, other axis */
  const float block_u = 16.0f, block_v = 16.0f;
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
  float imax_lo = bmax_y, imax_hi = bmin_y; /* float2(bbox_max.y, bbox_min.y) */
  float min_line = (float)rmin_x * block_u;
  if (bmin_x <= min_line) {
    o_ellipse_x(co, disc, t, px, py, is_y, (float)rmin_x * block_u, &imin_lo, &imin_hi);
  } else {
    imin_lo = imax_lo;
    imin_hi = imax_hi;
  }
  for (int u = rmin_x; u < rmax_x; ++u) {
    const float max_line = min_line + block_u;
    if (max_line <= bmax_x) o_ellipse_x(co, disc, t, px, py, is_y, max_line, &imax_lo, &imax_hi);
    float e_min, e_max;
    if (min_line <= am_y && am_y < max_line)
      e_min = bmin_y;
    else
      e_min = fmin_t(imin_lo, imax_lo);
    if (min_line <= aM_y && aM_y < max_line)
      e_max = bmax_y;
    else
      e_max = fmax_t(imin_hi, imax_hi);
    const int v0 = imax(rmin_y, imin(rmax_y, f2i(e_min / block_v)));
    const int v1 = imin(rmax_y, imax(rmin_y, f2i(e_max / block_v + 1)));
    if (keys) {
      for (int v = v0; v < v1; ++v) {
        const int tile = is_y ? (u * gx + v) : (v * gx + u);
        uint32_t db;
        memcpy(&db, &depth, 4);
        keys[off] = ((uint64_t)(int64_t)tile << 32) | (uint64_t)db;
        values[off] = idx;
        off++;
      }
    }
    count += (uint32_t)(v1 - v0);
    imin_lo = imax_lo;
    imin_hi = imax_hi;
    min_line = max_line;
  }
  return count;
}

/* fastgs_preprocess.metal:117-169 */
static v3 o_sh_color(int i, int deg, int maxc, const float* means, v3 campos, const float* dc,
                     const float* shs, uint8_t* clamped) {
  const v3 pos = V3(means[3 * i], means[3 * i + 1], means[3 * i + 2]);
  v3 d = V3(pos.x - campos.x, pos.y - campos.y, pos.z - campos.z);
  const float l = sqrtf(dot3(d, d));
  const float x = d.x / l, y = d.y / l, z = d.z / l;
  const float* sh = shs + (size_t)i * (size_t)maxc * 3u;
  float res[3];
  for (int c = 0; c < 3; ++c) res[c] = SH_C0 * dc[3 * i + c];
  if (deg > 0) {
    for (int c = 0; c < 3; ++c) {
      float r = res[c] - SH_C1 * y * sh[0 * 3 + c];
      r = r + SH_C1 * z * sh[1 * 3 + c];
      r = r - SH_C1 * x * sh[2 * 3 + c];
      res[c] = r;
    }
    if (deg > 1) {
      const float xx = x * x, yy = y * y, zz = z * z;
      const float xy = x * y, yz = y * z, xz = x * z;
      for (int c = 0; c < 3; ++c) {
        float s = SH_C2[0] * xy * sh[3 * 3 + c];
        s = s + SH_C2[1] * yz * sh[4 * 3 + c];
        s = s + SH_C2[2] * (2.0f * zz - xx - yy) * sh[5 * 3 + c];
        s = s + SH_C2[3] * xz * sh[6 * 3 + c];
        s = s + SH_C2[4] * (xx - yy) * sh[7 * 3 + c];
        res[c] = res[c] + s;
      }
      if (deg > 2) {
        for (int c = 0; c < 3; ++c) {
          float s = SH_C3[0] * y * (3.0f * xx - yy) * sh[8 * 3 + c];
          s = s + SH_C3[1] * xy * z * sh[9 * 3 + c];
          s = s + SH_C3[2] * y * (4.0f * zz - xx - yy) * sh[10 * 3 + c];
          s = s + SH_C3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy) * sh[11 * 3 + c];
          s = s + SH_C3[4] * x * (4.0f * zz - xx - yy) * sh[12 * 3 + c];
          s = s + SH_C3[5] * z * (xx - yy) * sh[13 * 3 + c];
          s = s + SH_C3[6] * x * (xx - 3.0f * yy) * sh[14 * 3 + c];
          res[c] = res[c] + s;
        }
      }
    }
  }
  v3 out;
  float o[3];
  for (int c = 0; c < 3; ++c) {
    const float r = res[c] + 0.5f;
    clamped[3 * i + c] = r < 0.0f;
    o[c] = fmax_t(r, 0.0f);
  }
  out = V3(o[0], o[1], o[2]);
  return out;
}

/* fastgs_preprocess.metal:384-484 (one Gaussian) */
static void o_preprocess_one(int i, const o_pre_params* p, const float* means3d, const float* dc,
                             const float* shs, const float* colors_precomp,
                             const float* opacities, const float* scales, const float* rotations,
                             const float* cov3d_precomp, const float* vm, const float* pm,
                             const float* cam_pos, const float* vs_in, int* radii, float* xys,
                             float* depths, float* cov3ds, float* rgb, float* conic_opacity,
                             uint32_t* tiles_touched, uint8_t* clamped, float* vs_out) {
  radii[i] = 0;
  tiles_touched[i] = 0u;
  const v3 po = V3(means3d[3 * i], means3d[3 * i + 1], means3d[3 * i + 2]);
  /* in_frustum (:96-115) */
  const v3 pv = xform43(po, vm);
  if (pv.z <= 0.2f) return;
  const float ph_x = pm[0] * po.x + pm[4] * po.y + pm[8] * po.z + pm[12];
  const float ph_y = pm[1] * po.x + pm[5] * po.y + pm[9] * po.z + pm[13];
  const float ph_w = pm[3] * po.x + pm[7] * po.y + pm[11] * po.z + pm[15];
  const float p_w = 1.0f / (ph_w + 1.0e-7f);
  const float pp_x = ph_x * p_w, pp_y = ph_y * p_w;
  float c3[6];
  if (p->use_cov3d_precomp) {
    for (int k = 0; k < 6; ++k) {
      c3[k] = cov3d_precomp[6 * i + k];
      cov3ds[6 * i + k] = c3[k];
    }
  } else {
    o_cov3d(V3(scales[3 * i], scales[3 * i + 1], scales[3 * i + 2]), p->scale_modifier,
            rotations + 4 * i, c3);
    for (int k = 0; k < 6; ++k) cov3ds[6 * i + k] = c3[k];
  }
  const v3 cov = o_cov2d(po, p->focal_x, p->focal_y, p->tan_fovx, p->tan_fovy, c3, vm);
  const float det = cov.x * cov.z - cov.y * cov.y;
  if (det == 0.0f) return;
  const float det_inv = 1.f / det;
  const float con_x = cov.z * det_inv, con_y = -cov.y * det_inv, con_z = cov.x * det_inv;
  const float mid = 0.5f * (cov.x + cov.z);
  const float l1 = mid + sqrtf(fmax_t(0.1f, mid * mid - det));
  const float l2 = mid - sqrtf(fmax_t(0.1f, mid * mid - det));
  const float my_radius = ceilf(3.f * sqrtf(fmax_t(l1, l2)));
  const float img_x = ndc2pix(pp_x, p->image_width);
  const float img_y = ndc2pix(pp_y, p->image_height);
  const float co[4] = {con_x, con_y, con_z, opacities[i]};
  const uint32_t tc =
      o_tile_walk(img_x, img_y, co, p->grid_x, p->grid_y, p->mult, 0, 0.f, NULL, NULL, 0);
  if (tc == 0u) return;
  if (p->use_colors_precomp) {
    for (int c = 0; c < 3; ++c) {
      rgb[3 * i + c] = colors_precomp[3 * i + c];
      clamped[3 * i + c] = 0;
    }
  } else {
    const v3 cp = V3(cam_pos[0], cam_pos[1], cam_pos[2]);
    const v3 col = o_sh_color(i, p->degree, p->max_sh_coeffs, means3d, cp, dc, shs, clamped);
    rgb[3 * i] = col.x;
    rgb[3 * i + 1] = col.y;
    rgb[3 * i + 2] = col.z;
  }
  depths[i] = pv.z;
  radii[i] = f2i(my_radius);
  xys[2 * i] = img_x;
  xys[2 * i + 1] = img_y;
  for (int k = 0; k < 4; ++k) conic_opacity[4 * i + k] = co[k];
  tiles_touched[i] = tc;
  vs_out[4 * i] = pv.x;
  vs_out[4 * i + 1] = pv.y;
  vs_out[4 * i + 2] = pv.z;
  vs_out[4 * i + 3] = vs_in[4 * i + 3];
}

void o_set_threads(int n) {
#ifdef _OPENMP
  omp_set_num_threads(n > 0 ? n : 1);
#else
  (void)n;
#endif
}

/* focal follows fastgs_preprocess.cpp:120-121 (W / (2 tan_fovx)) */
void o_preprocess_forward(int n, int degree, int max_sh_coeffs, float scale_modifier, float mult,
                          float tan_fovx, float tan_fovy, int image_width, int image_height,
                          int use_cov3d_precomp, int use_colors_precomp, const float* means3d,
                          const float* dc, const float* shs, const float* colors_precomp,
                          const float* opacities, const float* scales, const float* rotations,
                          const float* cov3d_precomp, const float* viewmatrix,
                          const float* projmatrix, const float* cam_pos,
                          const float* viewspace_in, int* radii, float* xys, float* depths,
                          float* cov3ds, float* rgb, float* conic_opacity,
                          uint32_t* tiles_touched, uint8_t* clamped, float* viewspace_out) {
  o_pre_params p;
  p.degree = degree;
  p.max_sh_coeffs = max_sh_coeffs;
  p.scale_modifier = scale_modifier;
  p.mult = mult;
  p.tan_fovx = tan_fovx;
  p.tan_fovy = tan_fovy;
  p.focal_x = (float)image_width / (2.0f * tan_fovx);
  p.focal_y = (float)image_height / (2.0f * tan_fovy);
  p.image_width = image_width;
  p.image_height = image_height;
  p.grid_x = (image_width + BLOCK - 1) / BLOCK;
  p.grid_y = (image_height + BLOCK - 1) / BLOCK;
  p.use_cov3d_precomp = use_cov3d_precomp;
  p.use_colors_precomp = use_colors_precomp;
#pragma omp parallel for schedule(dynamic, 1024)
  for (int i = 0; i < n; ++i)
    o_preprocess_one(i, &p, means3d, dc, shs, colors_precomp, opacities, scales, rotations,
                     cov3d_precomp, viewmatrix, projmatrix, cam_pos, viewspace_in, radii, xys,
                     depths, cov3ds, rgb, conic_opacity, tiles_touched, clamped, viewspace_out);
}

/* ---------------------------------------------------------------- binning */

/* binding.cpp:153 (mx::cumsum inclusive) */
void o_inclusive_scan_u32(int n, const uint32_t* in, uint32_t* out) {
  uint32_t acc = 0;
  for (int i = 0; i < n; ++i) {
    acc += in[i];
    out[i] = acc;
  }
}

/* fastgs_binning.metal:182-213; offsets is the inclusive scan of tiles_touched */
void o_duplicate_with_keys(int n, float mult, int grid_x, int grid_y, const float* xys,
                           const float* depths, const uint32_t* point_offsets,
                           const float* conic_opacity, const uint32_t* tiles_touched,
                           uint64_t* keys, uint32_t* values) {
#pragma omp parallel for schedule(dynamic, 1024)
  for (int i = 0; i < n; ++i) {
    if (tiles_touched[i] == 0u) continue;
    const uint64_t off = (i == 0) ? 0u : point_offsets[i - 1];
    o_tile_walk(xys[2 * i], xys[2 * i + 1], conic_opacity + 4 * i, grid_x, grid_y, mult,
                (uint32_t)i, depths[i], keys, values, off);
  }
}

/* binding.cpp:195-197: sort by the 64-bit key, ties kept in input order
 * (stable LSD radix sort over 8-bit digits, only the digits that can be
 * non-zero: 32 depth bits + enough bits for the largest tile id). */
void o_sort_pairs(int64_t k, int key_bits, uint64_t* keys, uint32_t* values, uint64_t* tmp_keys,
                  uint32_t* tmp_values) {
  uint64_t* src_k = keys;
  uint32_t* src_v = values;
  uint64_t* dst_k = tmp_keys;
  uint32_t* dst_v = tmp_values;
  const int passes = (key_bits + 7) / 8;
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = 8 * pass;
    int64_t cnt[257];
    memset(cnt, 0, sizeof(cnt));
    for (int64_t i = 0; i < k; ++i) cnt[((src_k[i] >> shift) & 0xffu) + 1]++;
    for (int d = 0; d < 256; ++d) cnt[d + 1] += cnt[d];
    for (int64_t i = 0; i < k; ++i) {
      const int d = (int)((src_k[i] >> shift) & 0xffu);
      const int64_t o = cnt[d]++;
      dst_k[o] = src_k[i];
      dst_v[o] = src_v[i];
    }
    uint64_t* tk = src_k; src_k = dst_k; dst_k = tk;
    uint32_t* tv = src_v; src_v = dst_v; dst_v = tv;
  }
  if (src_k != keys) {
    memcpy(keys, src_k, (size_t)k * 8u);
    memcpy(values, src_v, (size_t)k * 4u);
  }
}

/* fastgs_tile_prep.metal:10-53; ranges must be zeroed by the caller */
void o_tile_prep(int64_t num_rendered, int num_tiles, const uint64_t* keys, uint32_t* ranges,
                 uint32_t* bucket_count) {
  for (int64_t g = 0; g < num_rendered; ++g) {
    const uint32_t cur = (uint32_t)(keys[g] >> 32);
    const int valid = cur != 0xffffffffu;
    if (g == 0) {
      ranges[2 * (size_t)cur] = 0u;
    } else {
      const uint32_t prev = (uint32_t)(keys[g - 1] >> 32);
      if (cur != prev) {
        ranges[2 * (size_t)prev + 1] = (uint32_t)g;
        if (valid) ranges[2 * (size_t)cur] = (uint32_t)g;
      }
    }
    if (g == num_rendered - 1 && valid) ranges[2 * (size_t)cur + 1] = (uint32_t)num_rendered;
  }
  for (int t = 0; t < num_tiles; ++t) {
    const int ns = (int)(ranges[2 * t + 1] - ranges[2 * t]);
    bucket_count[t] = (uint32_t)((ns + 31) / 32);
  }
}

/* ---------------------------------------------------------- render forward */

/* fastgs_rasterize.metal:25-159. Outputs must be zeroed by the caller. */
void o_render_forward(int W, int H, int get_flag, const uint32_t* ranges,
                      const uint32_t* point_list, const uint32_t* bucket_offsets,
                      const float* means2d, const float* colors, const float* conic_opacity,
                      const float* background, const int* metric_map, uint32_t* bucket_to_tile,
                      float* sampled_t, float* sampled_ar, float* final_t, uint32_t* n_contrib,
                      uint32_t* max_contrib, float* pixel_colors, float* out_color,
                      int* metric_count) {
  const int gx = (W + BLOCK - 1) / BLOCK, gy = (H + BLOCK - 1) / BLOCK;
  const size_t P = (size_t)W * (size_t)H;
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < gx * gy; ++tile) {
    const int tx = tile % gx, ty = tile / gx;
    const uint32_t r0 = ranges[2 * tile], r1 = ranges[2 * tile + 1];
    const int to_do = (int)(r1 - r0);
    const int nb = (to_do + 31) / 32;
    const uint32_t bbm0 = (tile == 0) ? 0u : bucket_offsets[tile - 1];
    for (int b = 0; b < nb; ++b) bucket_to_tile[bbm0 + b] = (uint32_t)tile;
    uint32_t tile_max = 0;
    for (int ly = 0; ly < BLOCK; ++ly) {
      for (int lx = 0; lx < BLOCK; ++lx) {
        const int px = tx * BLOCK + lx, py = ty * BLOCK + ly;
        if (px >= W || py >= H) continue;
        const int lr = ly * BLOCK + lx;
        const size_t pix = (size_t)py * W + px;
        const float pfx = (float)px, pfy = (float)py;
        float T = 1.0f;
        uint32_t contributor = 0, last = 0;
        float C[3] = {0.f, 0.f, 0.f};
        uint32_t bbm = bbm0;
        for (uint32_t idx = r0; idx < r1; ++idx) {
          if (((idx - r0) % 32u) == 0u) {
            sampled_t[(size_t)bbm * 256u + lr] = T;
            for (int ch = 0; ch < 3; ++ch) sampled_ar[(size_t)bbm * 768u + ch * 256u + lr] = C[ch];
            bbm++;
          }
          contributor++;
          const uint32_t g = point_list[idx];
          const float dx = means2d[2 * g] - pfx, dy = means2d[2 * g + 1] - pfy;
          const float* co = conic_opacity + 4 * (size_t)g;
          const float power = -0.5f * (co[0] * dx * dx + co[2] * dy * dy) - co[1] * dx * dy;
          if (power > 0.0f) continue;
          const float alpha = fmin_t(0.99f, co[3] * O_EXP(power));
          if (alpha < 1.0f / 255.0f) continue;
          const float test_t = T * (1.0f - alpha);
          if (test_t < 0.0001f) break;
          for (int ch = 0; ch < 3; ++ch) C[ch] = O_ACC(C[ch], colors[3 * (size_t)g + ch], alpha, T);
          if (get_flag && metric_map[pix] == 1) {
#pragma omp atomic
            metric_count[g] += 1;
          }
          T = test_t;
          last = contributor;
        }
        final_t[pix] = T;
        n_contrib[pix] = last;
        for (int ch = 0; ch < 3; ++ch) {
          pixel_colors[ch * P + pix] = C[ch];
          out_color[ch * P + pix] = C[ch] + T * background[ch];
        }
        if (last > tile_max) tile_max = last;
      }
    }
    max_contrib[tile] = tile_max;
  }
}

/* --------------------------------------------------------- render backward */

/* fastgs_rasterize_backward.metal:24-278. For each bucket the 32 lanes see
 * every pixel of the tile in pixel order, and for each pixel the lanes run in
 * lane order (the simd_shuffle_up wavefront), so the sequential loop below
 * reproduces each lane's register sums exactly; only the order of the final
 * float atomics across buckets differs from the device. Gradient outputs
 * accumulate (the caller zeroes them). */
void o_render_backward(int W, int H, int bucket_sum, const uint32_t* ranges,
                       const uint32_t* point_list, const uint32_t* bucket_offsets,
                       const float* means2d, const float* colors, const float* conic_opacity,
                       const float* background, const float* dL_dout,
                       const uint32_t* bucket_to_tile, const float* sampled_t,
                       const float* sampled_ar, const float* final_t, const uint32_t* n_contrib,
                       const uint32_t* max_contrib, const float* pixel_colors, float* dL_dmeans2d,
                       float* dL_dcolors, float* dL_dconic, float* dL_dviewspace) {
  const int gx = (W + BLOCK - 1) / BLOCK, gy = (H + BLOCK - 1) / BLOCK;
  const int T_tiles = gx * gy;
  const size_t P = (size_t)W * (size_t)H;
  const float ddelx_dx = 0.5f * (float)W, ddely_dy = 0.5f * (float)H;
#pragma omp parallel for schedule(dynamic, 4)
  for (int bucket = 0; bucket < bucket_sum; ++bucket) {
    const uint32_t tile = bucket_to_tile[bucket];
    if ((int)tile >= T_tiles) continue;
    const uint32_t r0 = ranges[2 * tile], r1 = ranges[2 * tile + 1];
    const int nsplat = (int)(r1 - r0);
    const uint32_t bbm = (tile == 0) ? 0u : bucket_offsets[tile - 1];
    const int bidx = (int)((uint32_t)bucket - bbm);
    if (bidx * 32 >= (int)max_contrib[tile]) continue;
    const int tx = (int)tile % gx, ty = (int)tile / gx;
    int valid[32], gidx[32];
    float sx[32], sy[32], co[32][4], col[32][3];
    float acc[32][11];
    memset(acc, 0, sizeof(acc));
    for (int l = 0; l < 32; ++l) {
      const int s = bidx * 32 + l;
      valid[l] = s < nsplat;
      gidx[l] = 0;
      sx[l] = sy[l] = 0.f;
      co[l][0] = co[l][1] = co[l][2] = co[l][3] = 0.f;
      col[l][0] = col[l][1] = col[l][2] = 0.f;
      if (valid[l]) {
        const uint32_t g = point_list[r0 + s];
        gidx[l] = (int)g;
        sx[l] = means2d[2 * g];
        sy[l] = means2d[2 * g + 1];
        for (int k = 0; k < 4; ++k) co[l][k] = conic_opacity[4 * (size_t)g + k];
        for (int k = 0; k < 3; ++k) col[l][k] = colors[3 * (size_t)g + k];
      }
    }
    for (int idx = 0; idx < 256; ++idx) {
      const int px = tx * BLOCK + idx % BLOCK, py = ty * BLOCK + idx / BLOCK;
      if (px >= W || py >= H) continue;
      const size_t pix = (size_t)py * W + px;
      float T = sampled_t[(size_t)bucket * 256u + idx];
      float ar[3];
      for (int ch = 0; ch < 3; ++ch)
        ar[ch] = -pixel_colors[ch * P + pix] + sampled_ar[(size_t)bucket * 768u + ch * 256u + idx];
      const float T_final = final_t[pix];
      const float last = (float)n_contrib[pix];
      float dp[3];
      for (int ch = 0; ch < 3; ++ch) dp[ch] = dL_dout[ch * P + pix];
      const float pfx = (float)px, pfy = (float)py;
      for (int l = 0; l < 32; ++l) {
        if (!valid[l]) continue;
        if (bidx * 32 + l >= (int)last) continue;
        const float dx = sx[l] - pfx, dy = sy[l] - pfy;
        const float* c = co[l];
        const float power = -0.5f * (c[0] * dx * dx + c[2] * dy * dy) - c[1] * dx * dy;
        if (power > 0.0f) continue;
        const float G = O_EXP(power);
        const float alpha = fmin_t(0.99f, c[3] * G);
        if (alpha < (1.0f / 255.0f)) continue;
        const float dchannel_dcolor = alpha * T;
        const float rec = 1.0f / (1.0f - alpha);
        float dL_dalpha = 0.0f;
        for (int ch = 0; ch < 3; ++ch) {
          ar[ch] += dchannel_dcolor * col[l][ch];
          acc[l][8 + ch] += dchannel_dcolor * dp[ch];
          dL_dalpha += (col[l][ch] * T + rec * ar[ch]) * dp[ch];
        }
        float bg_dot = 0.0f;
        for (int ch = 0; ch < 3; ++ch) bg_dot += background[ch] * dp[ch];
        dL_dalpha += (-T_final * rec) * bg_dot;
        T *= (1.0f - alpha);
        const float dL_dG = c[3] * dL_dalpha;
        const float gdx = G * dx, gdy = G * dy;
        const float dG_ddelx = -gdx * c[0] - gdy * c[1];
        const float dG_ddely = -gdy * c[2] - gdx * c[1];
        if (c[3] * G > 0.99f) continue;
        const float tmp_x = dL_dG * dG_ddelx * ddelx_dx;
        const float tmp_y = dL_dG * dG_ddely * ddely_dy;
        acc[l][0] += tmp_x;
        acc[l][1] += tmp_y;
        acc[l][2] += fabsf(tmp_x);
        acc[l][3] += fabsf(tmp_y);
        acc[l][4] += -0.5f * gdx * dx * dL_dG;
        acc[l][5] += -0.5f * gdx * dy * dL_dG;
        acc[l][6] += -0.5f * gdy * dy * dL_dG;
        acc[l][7] += G * dL_dalpha;
      }
    }
    for (int l = 0; l < 32; ++l) {
      if (!valid[l]) continue;
      const size_t g = (size_t)gidx[l];
      float* a = acc[l];
#pragma omp atomic
      dL_dmeans2d[2 * g] += a[0];
#pragma omp atomic
      dL_dmeans2d[2 * g + 1] += a[1];
#pragma omp atomic
      dL_dviewspace[4 * g] += a[0];
#pragma omp atomic
      dL_dviewspace[4 * g + 1] += a[1];
#pragma omp atomic
      dL_dviewspace[4 * g + 2] += a[2];
#pragma omp atomic
      dL_dviewspace[4 * g + 3] += a[3];
#pragma omp atomic
      dL_dconic[4 * g] += a[4];
#pragma omp atomic
      dL_dconic[4 * g + 1] += a[5];
#pragma omp atomic
      dL_dconic[4 * g + 2] += a[6];
#pragma omp atomic
      dL_dconic[4 * g + 3] += a[7];
#pragma omp atomic
      dL_dcolors[3 * g] += a[8];
#pragma omp atomic
      dL_dcolors[3 * g + 1] += a[9];
#pragma omp atomic
      dL_dcolors[3 * g + 2] += a[10];
    }
  }
}

/* ------------------------------------------------------ preprocess backward */

typedef struct {
  float scale_modifier, tan_fovx, tan_fovy, focal_x, focal_y;
  int degree, max_sh_coeffs, use_cov3d_precomp, use_colors_precomp;
} o_pbwd_params;

static inline v3 v3s(float s, v3 a) { return V3(s * a.x, s * a.y, s * a.z); }
static inline v3 v3sr(v3 a, float s) { return V3(a.x * s, a.y * s, a.z * s); }
static inline v3 v3add(v3 a, v3 b) { return V3(a.x + b.x, a.y + b.y, a.z + b.z); }
static inline v3 ldv3(const float* p) { return V3(p[0], p[1], p[2]); }

/* fastgs_preprocess_backward.metal:60-430 (one Gaussian) */
static void o_pbwd_one(int i, const o_pbwd_params* P, const float* means3d, const float* scales,
                       const float* quats, const float* vm, const float* pm, const float* cam_pos,
                       const float* sh, const float* cov3d_precomp, const float* cov3d_fwd,
                       const float* dL_dcov3d, const float* dL_drgb, const float* dL_dxys,
                       const float* dL_dconic, const float* dL_dvs_out, const int* radii,
                       const uint8_t* clamped, float* dL_dmeans3d, float* dL_ddc, float* dL_dsh,
                       float* dL_dcolors_precomp, float* dL_dopacities, float* dL_dscales,
                       float* dL_dquats, float* dL_dvs_in) {
  if (!(radii[i] > 0)) return;
  const v3 p = ldv3(means3d + 3 * i);
  const float ph_w = pm[3] * p.x + pm[7] * p.y + pm[11] * p.z + pm[15];
  const size_t cb = 6u * (size_t)i;
  const float gx = dL_dxys[2 * i], gy = dL_dxys[2 * i + 1];
  const float* cov3D = (P->use_cov3d_precomp ? cov3d_precomp : cov3d_fwd) + cb;
  const float cg_x = dL_dconic[4 * i], cg_y = dL_dconic[4 * i + 1], cg_z = dL_dconic[4 * i + 2];
  float dce[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  v3 dmean_cov;
  {
    v3 t = xform43(p, vm);
    const float limx = 1.3f * P->tan_fovx, limy = 1.3f * P->tan_fovy;
    const float txtz = t.x / t.z, tytz = t.y / t.z;
    t.x = fmin_t(limx, fmax_t(-limx, txtz)) * t.z;
    t.y = fmin_t(limy, fmax_t(-limy, tytz)) * t.z;
    const float x_grad_mul = (txtz < -limx || txtz > limx) ? 0.0f : 1.0f;
    const float y_grad_mul = (tytz < -limy || tytz > limy) ? 0.0f : 1.0f;
    const float fx = P->focal_x, fy = P->focal_y;
    const m3 J = M3(fx / t.z, 0.0f, -(fx * t.x) / (t.z * t.z), 0.0f, fy / t.z,
                    -(fy * t.y) / (t.z * t.z), 0.0f, 0.0f, 0.0f);
    const m3 Wm = M3(vm[0], vm[1], vm[2], vm[4], vm[5], vm[6], vm[8], vm[9], vm[10]);
    const m3 V = M3(cov3D[0], cov3D[1], cov3D[2], cov3D[1], cov3D[3], cov3D[4], cov3D[2],
                    cov3D[4], cov3D[5]);
    const m3 Tm = m3_mul(&Wm, &J);
    const m3 Tt = m3_tr(&Tm), Vt = m3_tr(&V);
    const m3 A = m3_mul(&Tt, &Vt);
    const m3 c2 = m3_mul(&A, &Tm);
    const float a = c2.c[0].x + 0.3f, b = c2.c[0].y, c = c2.c[1].y + 0.3f;
    const float denom = a * c - b * b;
    const float denom2inv = 1.0f / ((denom * denom) + 1e-7f);
    float dL_da = 0.f, dL_db = 0.f, dL_dc = 0.f;
#define T_(i_, j_) m3_at(&Tm, i_, j_)
#define V_(i_, j_) m3_at(&V, i_, j_)
#define W_(i_, j_) m3_at(&Wm, i_, j_)
    if (denom2inv != 0.0f) {
      dL_da = denom2inv * (-c * c * cg_x + 2.0f * b * c * cg_y + (denom - a * c) * cg_z);
      dL_dc = denom2inv * (-a * a * cg_z + 2.0f * a * b * cg_y + (denom - a * c) * cg_x);
      dL_db = denom2inv * 2.0f * (b * c * cg_x - (denom + 2.0f * b * b) * cg_y + a * b * cg_z);
      dce[0] = (T_(0, 0) * T_(0, 0) * dL_da + T_(0, 0) * T_(1, 0) * dL_db +
                T_(1, 0) * T_(1, 0) * dL_dc);
      dce[3] = (T_(0, 1) * T_(0, 1) * dL_da + T_(0, 1) * T_(1, 1) * dL_db +
                T_(1, 1) * T_(1, 1) * dL_dc);
      dce[5] = (T_(0, 2) * T_(0, 2) * dL_da + T_(0, 2) * T_(1, 2) * dL_db +
                T_(1, 2) * T_(1, 2) * dL_dc);
      dce[1] = 2.0f * T_(0, 0) * T_(0, 1) * dL_da +
               (T_(0, 0) * T_(1, 1) + T_(0, 1) * T_(1, 0)) * dL_db +
               2.0f * T_(1, 0) * T_(1, 1) * dL_dc;
      dce[2] = 2.0f * T_(0, 0) * T_(0, 2) * dL_da +
               (T_(0, 0) * T_(1, 2) + T_(0, 2) * T_(1, 0)) * dL_db +
               2.0f * T_(1, 0) * T_(1, 2) * dL_dc;
      dce[4] = 2.0f * T_(0, 2) * T_(0, 1) * dL_da +
               (T_(0, 1) * T_(1, 2) + T_(0, 2) * T_(1, 1)) * dL_db +
               2.0f * T_(1, 1) * T_(1, 2) * dL_dc;
    }
    const float dT00 = 2.0f * (T_(0, 0) * V_(0, 0) + T_(0, 1) * V_(0, 1) + T_(0, 2) * V_(0, 2)) * dL_da +
                       (T_(1, 0) * V_(0, 0) + T_(1, 1) * V_(0, 1) + T_(1, 2) * V_(0, 2)) * dL_db;
    const float dT01 = 2.0f * (T_(0, 0) * V_(1, 0) + T_(0, 1) * V_(1, 1) + T_(0, 2) * V_(1, 2)) * dL_da +
                       (T_(1, 0) * V_(1, 0) + T_(1, 1) * V_(1, 1) + T_(1, 2) * V_(1, 2)) * dL_db;
    const float dT02 = 2.0f * (T_(0, 0) * V_(2, 0) + T_(0, 1) * V_(2, 1) + T_(0, 2) * V_(2, 2)) * dL_da +
                       (T_(1, 0) * V_(2, 0) + T_(1, 1) * V_(2, 1) + T_(1, 2) * V_(2, 2)) * dL_db;
    const float dT10 = 2.0f * (T_(1, 0) * V_(0, 0) + T_(1, 1) * V_(0, 1) + T_(1, 2) * V_(0, 2)) * dL_dc +
                       (T_(0, 0) * V_(0, 0) + T_(0, 1) * V_(0, 1) + T_(0, 2) * V_(0, 2)) * dL_db;
    const float dT11 = 2.0f * (T_(1, 0) * V_(1, 0) + T_(1, 1) * V_(1, 1) + T_(1, 2) * V_(1, 2)) * dL_dc +
                       (T_(0, 0) * V_(1, 0) + T_(0, 1) * V_(1, 1) + T_(0, 2) * V_(1, 2)) * dL_db;
    const float dT12 = 2.0f * (T_(1, 0) * V_(2, 0) + T_(1, 1) * V_(2, 1) + T_(1, 2) * V_(2, 2)) * dL_dc +
                       (T_(0, 0) * V_(2, 0) + T_(0, 1) * V_(2, 1) + T_(0, 2) * V_(2, 2)) * dL_db;
    const float dJ00 = W_(0, 0) * dT00 + W_(0, 1) * dT01 + W_(0, 2) * dT02;
    const float dJ02 = W_(2, 0) * dT00 + W_(2, 1) * dT01 + W_(2, 2) * dT02;
    const float dJ11 = W_(1, 0) * dT10 + W_(1, 1) * dT11 + W_(1, 2) * dT12;
    const float dJ12 = W_(2, 0) * dT10 + W_(2, 1) * dT11 + W_(2, 2) * dT12;
#undef T_
#undef V_
#undef W_
    const float tz = 1.0f / t.z;
    const float tz2 = tz * tz;
    const float tz3 = tz2 * tz;
    const float dtx = x_grad_mul * -fx * tz2 * dJ02;
    const float dty = y_grad_mul * -fy * tz2 * dJ12;
    const float dtz = -fx * tz2 * dJ00 - fy * tz2 * dJ11 + (2.0f * fx * t.x) * tz3 * dJ02 +
                      (2.0f * fy * t.y) * tz3 * dJ12;
    dmean_cov = V3(vm[0] * dtx + vm[1] * dty + vm[2] * dtz, vm[4] * dtx + vm[5] * dty + vm[6] * dtz,
                   vm[8] * dtx + vm[9] * dty + vm[10] * dtz);
  }
  /* :188-205 */
  const float m_w = 1.0f / (ph_w + 1.0e-7f);
  const float mul1 = (pm[0] * p.x + pm[4] * p.y + pm[8] * p.z + pm[12]) * m_w * m_w;
  const float mul2 = (pm[1] * p.x + pm[5] * p.y + pm[9] * p.z + pm[13]) * m_w * m_w;
  const float dmx = (pm[0] * m_w - pm[3] * mul1) * gx + (pm[1] * m_w - pm[3] * mul2) * gy;
  const float dmy = (pm[4] * m_w - pm[7] * mul1) * gx + (pm[5] * m_w - pm[7] * mul2) * gy;
  const float dmz = (pm[8] * m_w - pm[11] * mul1) * gx + (pm[9] * m_w - pm[11] * mul2) * gy;
  float dm0 = dmx + dmean_cov.x, dm1 = dmy + dmean_cov.y, dm2 = dmz + dmean_cov.z;
  dL_dopacities[i] = dL_dconic[4 * i + 3];
  if (P->use_colors_precomp) {
    for (int c = 0; c < 3; ++c) dL_dcolors_precomp[3 * i + c] = dL_drgb[3 * i + c];
  } else {
    const v3 dRGB = V3(clamped[3 * i] ? 0.0f : dL_drgb[3 * i],
                       clamped[3 * i + 1] ? 0.0f : dL_drgb[3 * i + 1],
                       clamped[3 * i + 2] ? 0.0f : dL_drgb[3 * i + 2]);
    dL_ddc[3 * i] = SH_C0 * dRGB.x;
    dL_ddc[3 * i + 1] = SH_C0 * dRGB.y;
    dL_ddc[3 * i + 2] = SH_C0 * dRGB.z;
    for (int c = 0; c < 3; ++c) dL_dcolors_precomp[3 * i + c] = 0.0f;
    if (P->degree > 0 && P->max_sh_coeffs >= 3) {
      const v3 pos = ldv3(means3d + 3 * i);
      const v3 cp = ldv3(cam_pos);
      const v3 dir_orig = V3(pos.x - cp.x, pos.y - cp.y, pos.z - cp.z);
      const float dl = sqrtf(dot3(dir_orig, dir_orig));
      const float x = dir_orig.x / dl, y = dir_orig.y / dl, z = dir_orig.z / dl;
      const size_t base = (size_t)i * (size_t)P->max_sh_coeffs * 3u;
      const float* s = sh + base;
      float* g = dL_dsh + base;
#define SHC(k) ldv3(s + 3 * (k))
#define PUT(k, v) do { v3 v_ = (v); g[3 * (k)] = v_.x; g[3 * (k) + 1] = v_.y; g[3 * (k) + 2] = v_.z; } while (0)
      PUT(0, v3s(-SH_C1 * y, dRGB));
      PUT(1, v3s(SH_C1 * z, dRGB));
      PUT(2, v3s(-SH_C1 * x, dRGB));
      v3 dx_ = v3s(-SH_C1, SHC(2));
      v3 dy_ = v3s(-SH_C1, SHC(0));
      v3 dz_ = v3s(SH_C1, SHC(1));
      if (P->degree > 1 && P->max_sh_coeffs >= 8) {
        const float xx = x * x, yy = y * y, zz = z * z;
        const float xy = x * y, yz = y * z, xz = x * z;
        PUT(3, v3s(SH_C2[0] * xy, dRGB));
        PUT(4, v3s(SH_C2[1] * yz, dRGB));
        PUT(5, v3s(SH_C2[2] * (2.0f * zz - xx - yy), dRGB));
        PUT(6, v3s(SH_C2[3] * xz, dRGB));
        PUT(7, v3s(SH_C2[4] * (xx - yy), dRGB));
        /* dRGBdx += C2[0]*y*sh3 + C2[2]*2*-x*sh5 + C2[3]*z*sh6 + C2[4]*2*x*sh7 */
        {
          v3 s1 = v3s(SH_C2[0] * y, SHC(3));
          s1 = v3add(s1, v3s(SH_C2[2] * 2.f * -x, SHC(5)));
          s1 = v3add(s1, v3s(SH_C2[3] * z, SHC(6)));
          s1 = v3add(s1, v3s(SH_C2[4] * 2.f * x, SHC(7)));
          dx_ = v3add(dx_, s1);
        }
        {
          v3 s1 = v3s(SH_C2[0] * x, SHC(3));
          s1 = v3add(s1, v3s(SH_C2[1] * z, SHC(4)));
          s1 = v3add(s1, v3s(SH_C2[2] * 2.f * -y, SHC(5)));
          s1 = v3add(s1, v3s(SH_C2[4] * 2.f * -y, SHC(7)));
          dy_ = v3add(dy_, s1);
        }
        {
          v3 s1 = v3s(SH_C2[1] * y, SHC(4));
          s1 = v3add(s1, v3s(SH_C2[2] * 4.f * z, SHC(5)));
          s1 = v3add(s1, v3s(SH_C2[3] * x, SHC(6)));
          dz_ = v3add(dz_, s1);
        }
        if (P->degree > 2 && P->max_sh_coeffs >= 15) {
          PUT(8, v3s(SH_C3[0] * y * (3.f * xx - yy), dRGB));
          PUT(9, v3s(SH_C3[1] * xy * z, dRGB));
          PUT(10, v3s(SH_C3[2] * y * (4.f * zz - xx - yy), dRGB));
          PUT(11, v3s(SH_C3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy), dRGB));
          PUT(12, v3s(SH_C3[4] * x * (4.f * zz - xx - yy), dRGB));
          PUT(13, v3s(SH_C3[5] * z * (xx - yy), dRGB));
          PUT(14, v3s(SH_C3[6] * x * (xx - 3.f * yy), dRGB));
          /* (C * sh) * a * b: vector first, then scalars left to right */
          {
            v3 s1 = v3sr(v3sr(v3s(SH_C3[0], SHC(8)), 6.f), xy);
            s1 = v3add(s1, v3sr(v3s(SH_C3[1], SHC(9)), yz));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[2], SHC(10)), -2.f), xy));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[3], SHC(11)), -6.f), xz));
            s1 = v3add(s1, v3sr(v3s(SH_C3[4], SHC(12)), (-3.f * xx + 4.f * zz - yy)));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[5], SHC(13)), 2.f), xz));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[6], SHC(14)), 3.f), (xx - yy)));
            dx_ = v3add(dx_, s1);
          }
          {
            v3 s1 = v3sr(v3sr(v3s(SH_C3[0], SHC(8)), 3.f), (xx - yy));
            s1 = v3add(s1, v3sr(v3s(SH_C3[1], SHC(9)), xz));
            s1 = v3add(s1, v3sr(v3s(SH_C3[2], SHC(10)), (-3.f * yy + 4.f * zz - xx)));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[3], SHC(11)), -6.f), yz));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[4], SHC(12)), -2.f), xy));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[5], SHC(13)), -2.f), yz));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[6], SHC(14)), -6.f), xy));
            dy_ = v3add(dy_, s1);
          }
          {
            v3 s1 = v3sr(v3s(SH_C3[1], SHC(9)), xy);
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[2], SHC(10)), 8.f), yz));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[3], SHC(11)), 3.f), (2.f * zz - xx - yy)));
            s1 = v3add(s1, v3sr(v3sr(v3s(SH_C3[4], SHC(12)), 8.f), xz));
            s1 = v3add(s1, v3sr(v3s(SH_C3[5], SHC(13)), (xx - yy)));
            dz_ = v3add(dz_, s1);
          }
        }
      }
#undef SHC
#undef PUT
      const v3 ddir = V3(dot3(dx_, dRGB), dot3(dy_, dRGB), dot3(dz_, dRGB));
      /* dnormvdv (:54-58) */
      const float len = fmax_t(sqrtf(dot3(dir_orig, dir_orig)), 1e-6f);
      const v3 nn = V3(dir_orig.x / len, dir_orig.y / len, dir_orig.z / len);
      const float nd = dot3(nn, ddir);
      const v3 gm = V3((ddir.x - nn.x * nd) / len, (ddir.y - nn.y * nd) / len,
                       (ddir.z - nn.z * nd) / len);
      dm0 = dm0 + gm.x;
      dm1 = dm1 + gm.y;
      dm2 = dm2 + gm.z;
    }
  }
  dL_dmeans3d[3 * i] = dm0;
  dL_dmeans3d[3 * i + 1] = dm1;
  dL_dmeans3d[3 * i + 2] = dm2;
  if (!P->use_cov3d_precomp) {
    const v3 scale = ldv3(scales + 3 * i);
    const float* q = quats + 4 * i;
    const float r = q[0], x = q[1], y = q[2], z = q[3];
    const m3 R = M3(1.f - 2.f * (y * y + z * z), 2.f * (x * y - r * z), 2.f * (x * z + r * y),
                    2.f * (x * y + r * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - r * x),
                    2.f * (x * z - r * y), 2.f * (y * z + r * x), 1.f - 2.f * (x * x + y * y));
    const v3 s = v3s(P->scale_modifier, scale);
    m3 S = M3(1.f, 0.f, 0.f, 0.f, 1.f, 0.f, 0.f, 0.f, 1.f);
    S.c[0].x = s.x;
    S.c[1].y = s.y;
    S.c[2].z = s.z;
    const m3 M = m3_mul(&S, &R);
    const float c0 = dL_dcov3d[cb + 0] + dce[0];
    const float c1 = dL_dcov3d[cb + 1] + dce[1];
    const float c2 = dL_dcov3d[cb + 2] + dce[2];
    const float c3 = dL_dcov3d[cb + 3] + dce[3];
    const float c4 = dL_dcov3d[cb + 4] + dce[4];
    const float c5 = dL_dcov3d[cb + 5] + dce[5];
    const m3 dSigma = M3(c0, 0.5f * c1, 0.5f * c2, 0.5f * c1, c3, 0.5f * c4, 0.5f * c2, 0.5f * c4,
                         c5);
    const m3 M2 = m3_scale(2.0f, &M);
    const m3 dM = m3_mul(&M2, &dSigma);
    const m3 Rt = m3_tr(&R);
    m3 dMt = m3_tr(&dM);
    dL_dscales[3 * i] = dot3(Rt.c[0], dMt.c[0]);
    dL_dscales[3 * i + 1] = dot3(Rt.c[1], dMt.c[1]);
    dL_dscales[3 * i + 2] = dot3(Rt.c[2], dMt.c[2]);
    dMt.c[0] = v3sr(dMt.c[0], s.x);
    dMt.c[1] = v3sr(dMt.c[1], s.y);
    dMt.c[2] = v3sr(dMt.c[2], s.z);
#define D_(i_, j_) m3_at(&dMt, i_, j_)
    dL_dquats[4 * i] = 2 * z * (D_(0, 1) - D_(1, 0)) + 2 * y * (D_(2, 0) - D_(0, 2)) +
                       2 * x * (D_(1, 2) - D_(2, 1));
    dL_dquats[4 * i + 1] = 2 * y * (D_(1, 0) + D_(0, 1)) + 2 * z * (D_(2, 0) + D_(0, 2)) +
                           2 * r * (D_(1, 2) - D_(2, 1)) - 4 * x * (D_(2, 2) + D_(1, 1));
    dL_dquats[4 * i + 2] = 2 * x * (D_(1, 0) + D_(0, 1)) + 2 * r * (D_(2, 0) - D_(0, 2)) +
                           2 * z * (D_(1, 2) + D_(2, 1)) - 4 * y * (D_(2, 2) + D_(0, 0));
    dL_dquats[4 * i + 3] = 2 * r * (D_(0, 1) - D_(1, 0)) + 2 * x * (D_(2, 0) + D_(0, 2)) +
                           2 * y * (D_(1, 2) + D_(2, 1)) - 4 * z * (D_(1, 1) + D_(0, 0));
#undef D_
  }
  for (int k = 0; k < 4; ++k) dL_dvs_in[4 * i + k] = dL_dvs_out[4 * i + k];
}

/* focal follows fastgs_preprocess_backward.cpp:134-137 */
void o_preprocess_backward(int n, int image_width, int image_height, int use_cov3d_precomp,
                           int use_colors_precomp, float scale_modifier, float tan_fovx,
                           float tan_fovy, int degree, int max_sh_coeffs, const float* means3d,
                           const float* scales, const float* quats, const float* viewmat,
                           const float* projmat, const float* cam_pos, const float* sh,
                           const float* cov3d_precomp, const float* cov3d_fwd,
                           const float* dL_dcov3d, const float* dL_drgb, const float* dL_dxys,
                           const float* dL_dconic_opacity, const float* dL_dviewspace_out,
                           const int* radii, const uint8_t* clamped, float* dL_dmeans3d,
                           float* dL_ddc, float* dL_dsh, float* dL_dcolors_precomp,
                           float* dL_dopacities, float* dL_dscales, float* dL_dquats,
                           float* dL_dviewspace_in) {
  o_pbwd_params P;
  P.scale_modifier = scale_modifier;
  P.tan_fovx = tan_fovx;
  P.tan_fovy = tan_fovy;
  P.focal_x = 0.5f * (float)image_width / fmax_t(tan_fovx, 1e-6f);
  P.focal_y = 0.5f * (float)image_height / fmax_t(tan_fovy, 1e-6f);
  P.degree = degree;
  P.max_sh_coeffs = max_sh_coeffs;
  P.use_cov3d_precomp = use_cov3d_precomp;
  P.use_colors_precomp = use_colors_precomp;
#pragma omp parallel for schedule(dynamic, 1024)
  for (int i = 0; i < n; ++i)
    o_pbwd_one(i, &P, means3d, scales, quats, viewmat, projmat, cam_pos, sh, cov3d_precomp,
               cov3d_fwd, dL_dcov3d, dL_drgb, dL_dxys, dL_dconic_opacity, dL_dviewspace_out,
               radii, clamped, dL_dmeans3d, dL_ddc, dL_dsh, dL_dcolors_precomp, dL_dopacities,
               dL_dscales, dL_dquats, dL_dviewspace_in);
}

/* exported for the tests of the shared exp/log definition */
float o_fgs_expf(float x) { return fgs_expf(x); }
float o_fgs_logf(float x) { return fgs_logf(x); }
