// Preprocess forward / backward and the tiles-touched prefix sum (sm_100a).
//
// Forward follows fastgs_core/metal/fastgs_preprocess.metal:46-484, backward
// fastgs_core/metal/fastgs_preprocess_backward.metal:24-430, statement by
// statement (same operation order; see fgs_common.cuh for the arithmetic
// contract). Layout: one thread per Gaussian; the [n, S, 3] SH block of a CTA
// is staged through shared memory with 16-byte vector loads (the largest
// per-Gaussian read: 180 B at degree 3), everything else is read and written
// directly in the reference's AoS layout. Every output element is written,
// zeros for culled Gaussians, so no separate clearing pass is needed.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/fastgs_b200.h"
#include "fgs_common.cuh"
#include "tile_walk.cuh"

namespace fgs {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return FGS_ERR_CUDA;
  }
  return FGS_OK;
}

constexpr int kPreThreads = 128;

// Activations of the training parameters (the trainers' getters,
// scripts/train_scanner_fixed.py:523-535): opacity = sigmoid(logit), scale =
// exp(log_scale), rotation = q / (|q| + 1e-8). The training variants of the
// preprocess forward and backward kernels both evaluate them from the flat
// raw-parameter buffer with these functions (same file, same rounding), so no
// activated copy is written or read.
__device__ __forceinline__ float act_opacity(float logit) { return 1.0f / (1.0f + expf(-logit)); }
__device__ __forceinline__ float act_scale(float log_scale) { return expf(log_scale); }
__device__ __forceinline__ float4 raw_quat(const float* q4) {
  return make_float4(q4[0], q4[1], q4[2], q4[3]);  // scalar loads: the segment may be unaligned
}
__device__ __forceinline__ float4 act_quat(float4 q) {
  const float inv = 1.0f / (sqrtf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w) + 1e-8f);
  return make_float4(q.x * inv, q.y * inv, q.z * inv, q.w * inv);
}

struct PreArgs {
  fgs_preprocess_params p;
  const float* raw;  // training variant: the flat raw parameters (59 n floats)
  float focal_x, focal_y;
  int gx, gy;
  const float *means3d, *dc, *sh, *colors_precomp, *opacities, *scales, *quats, *cov3d_precomp,
      *viewmatrix, *projmatrix, *cam_pos, *vs_in;
  int32_t* radii;
  float *xys, *depths, *cov3d, *rgb, *conic;
  uint32_t* tiles;
  uint8_t* clamped;
  float* vs_out;
  int skip_color;  // geometry only: rgb and clamped are neither computed nor written
};

// Stage `count` floats starting at g (16-byte aligned chunk boundaries are
// handled with a scalar head/tail) into shared memory.
__device__ __forceinline__ void stage_floats(float* s, const float* g, int64_t count) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(g);
  const int head = (int)(((16u - (addr & 15u)) & 15u) / 4u);
  const int h = (int)((int64_t)head < count ? (int64_t)head : count);
  for (int i = threadIdx.x; i < h; i += blockDim.x) s[i] = __ldg(g + i);
  const int64_t body = (count - h) / 4;
  const float4* g4 = reinterpret_cast<const float4*>(g + h);
  for (int64_t i = threadIdx.x; i < body; i += blockDim.x) {
    const float4 v = __ldg(g4 + i);
    s[h + 4 * i] = v.x;
    s[h + 4 * i + 1] = v.y;
    s[h + 4 * i + 2] = v.z;
    s[h + 4 * i + 3] = v.w;
  }
  for (int64_t i = h + body * 4 + threadIdx.x; i < count; i += blockDim.x) s[i] = __ldg(g + i);
}

// fastgs_preprocess.metal:117-169; `s` points at this Gaussian's S*3 coefficients
__device__ __forceinline__ v3 sh_color(int deg, v3 dir_unnorm, const float* dcp, const float* s,
                                       uint8_t* clamped) {
  const float l = sqrtf(dot3(dir_unnorm, dir_unnorm));
  const float x = dir_unnorm.x / l, y = dir_unnorm.y / l, z = dir_unnorm.z / l;
  float res[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) res[c] = kSH_C0 * dcp[c];
  if (deg > 0) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float r = res[c] - kSH_C1 * y * s[0 * 3 + c];
      r = r + kSH_C1 * z * s[1 * 3 + c];
      r = r - kSH_C1 * x * s[2 * 3 + c];
      res[c] = r;
    }
    if (deg > 1) {
      const float xx = x * x, yy = y * y, zz = z * z;
      const float xy = x * y, yz = y * z, xz = x * z;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        float q = 1.0925484305920792f * xy * s[3 * 3 + c];
        q = q + -1.0925484305920792f * yz * s[4 * 3 + c];
        q = q + 0.31539156525252005f * (2.0f * zz - xx - yy) * s[5 * 3 + c];
        q = q + -1.0925484305920792f * xz * s[6 * 3 + c];
        q = q + 0.5462742152960396f * (xx - yy) * s[7 * 3 + c];
        res[c] = res[c] + q;
      }
      if (deg > 2) {
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          float q = -0.5900435899266435f * y * (3.0f * xx - yy) * s[8 * 3 + c];
          q = q + 2.890611442640554f * xy * z * s[9 * 3 + c];
          q = q + -0.4570457994644658f * y * (4.0f * zz - xx - yy) * s[10 * 3 + c];
          q = q + 0.3731763325901154f * z * (2.0f * zz - 3.0f * xx - 3.0f * yy) * s[11 * 3 + c];
          q = q + -0.4570457994644658f * x * (4.0f * zz - xx - yy) * s[12 * 3 + c];
          q = q + 1.445305721320277f * z * (xx - yy) * s[13 * 3 + c];
          q = q + -0.5900435899266435f * x * (xx - 3.0f * yy) * s[14 * 3 + c];
          res[c] = res[c] + q;
        }
      }
    }
  }
  v3 out;
  float o[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const float r = res[c] + 0.5f;
    clamped[c] = r < 0.0f;
    o[c] = fmax_t(r, 0.0f);
  }
  out = V3(o[0], o[1], o[2]);
  return out;
}

template <bool kRaw>
// eight resident CTAs per SM (config 3: 0.101 ms; four: 0.112 ms)
__global__ void __launch_bounds__(kPreThreads, 8) preprocess_fwd_kernel(PreArgs a) {
  extern __shared__ float s_sh[];
  const fgs_preprocess_params& p = a.p;
  const int base = blockIdx.x * kPreThreads;
  const int i = base + threadIdx.x;
  const int S3 = p.max_sh_coeffs * 3;
  const bool use_sh = !a.skip_color && !p.use_colors_precomp && p.degree > 0 && p.max_sh_coeffs > 0;
  if (use_sh) {
    const int cnt = min(kPreThreads, p.n - base);
    stage_floats(s_sh, a.sh + (int64_t)base * S3, (int64_t)cnt * S3);
    __syncthreads();
  }
  if (i >= p.n) return;

  int32_t radius_out = 0;
  uint32_t tiles_out = 0;
  float2 xy_out = make_float2(0.f, 0.f);
  float depth_out = 0.f;
  float4 conic_out = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 vs_o = make_float4(0.f, 0.f, 0.f, 0.f);
  float rgb_out[3] = {0.f, 0.f, 0.f};
  uint8_t cl[3] = {0, 0, 0};
  float c3[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};

  const v3 po = V3(a.means3d[3 * i], a.means3d[3 * i + 1], a.means3d[3 * i + 2]);
  const float* vm = a.viewmatrix;
  const float* pm = a.projmatrix;
  const v3 pv = xform43(po, vm);
  if (pv.z > 0.2f) {  // in_frustum, fastgs_preprocess.metal:96-115
    const float ph_x = pm[0] * po.x + pm[4] * po.y + pm[8] * po.z + pm[12];
    const float ph_y = pm[1] * po.x + pm[5] * po.y + pm[9] * po.z + pm[13];
    const float ph_w = pm[3] * po.x + pm[7] * po.y + pm[11] * po.z + pm[15];
    const float p_w = 1.0f / (ph_w + 1.0e-7f);
    const float pp_x = ph_x * p_w, pp_y = ph_y * p_w;
    if (p.use_cov3d_precomp) {
#pragma unroll
      for (int k = 0; k < 6; ++k) c3[k] = a.cov3d_precomp[6 * (int64_t)i + k];
    } else {
      // compute_cov3d, fastgs_preprocess.metal:207-231
      const float mod = p.scale_modifier;
      m3 s = M3(1.f, 0.f, 0.f, 0.f, 1.f, 0.f, 0.f, 0.f, 1.f);
      const int64_t n = p.n;
      s.c[0].x = mod * (kRaw ? act_scale(a.raw[52 * n + 3 * i]) : a.scales[3 * i]);
      s.c[1].y = mod * (kRaw ? act_scale(a.raw[52 * n + 3 * i + 1]) : a.scales[3 * i + 1]);
      s.c[2].z = mod * (kRaw ? act_scale(a.raw[52 * n + 3 * i + 2]) : a.scales[3 * i + 2]);
      const float4 q = kRaw ? act_quat(raw_quat(a.raw + 55 * n + 4 * (int64_t)i))
                            : reinterpret_cast<const float4*>(a.quats)[i];
      const float r = q.x, x = q.y, y = q.z, z = q.w;
      const m3 rm = M3(1.f - 2.f * (y * y + z * z), 2.f * (x * y - r * z), 2.f * (x * z + r * y),
                       2.f * (x * y + r * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - r * x),
                       2.f * (x * z - r * y), 2.f * (y * z + r * x), 1.f - 2.f * (x * x + y * y));
      const m3 m = mul(s, rm);
      const m3 sig = mul(tr(m), m);
      c3[0] = sig.c[0].x;
      c3[1] = sig.c[0].y;
      c3[2] = sig.c[0].z;
      c3[3] = sig.c[1].y;
      c3[4] = sig.c[1].z;
      c3[5] = sig.c[2].z;
    }
    // compute_cov2d, fastgs_preprocess.metal:171-205
    v3 t = pv;
    const float limx = 1.3f * p.tan_fovx, limy = 1.3f * p.tan_fovy;
    const float txtz = t.x / t.z, tytz = t.y / t.z;
    t.x = fmin_t(limx, fmax_t(-limx, txtz)) * t.z;
    t.y = fmin_t(limy, fmax_t(-limy, tytz)) * t.z;
    const float fx = a.focal_x, fy = a.focal_y;
    const m3 j = M3(fx / t.z, 0.0f, -(fx * t.x) / (t.z * t.z), 0.0f, fy / t.z,
                    -(fy * t.y) / (t.z * t.z), 0.0f, 0.0f, 0.0f);
    const m3 w = M3(vm[0], vm[1], vm[2], vm[4], vm[5], vm[6], vm[8], vm[9], vm[10]);
    const m3 tm = mul(w, j);
    const m3 vrk = M3(c3[0], c3[1], c3[2], c3[1], c3[3], c3[4], c3[2], c3[4], c3[5]);
    m3 cov = mul(mul(tr(tm), tr(vrk)), tm);
    cov.c[0].x += 0.3f;
    cov.c[1].y += 0.3f;
    const float cx = cov.c[0].x, cy = cov.c[0].y, cz = cov.c[1].y;
    const float det = cx * cz - cy * cy;
    if (det != 0.0f) {
      const float det_inv = 1.f / det;
      const float op = kRaw ? act_opacity(a.raw[51 * (int64_t)p.n + i]) : a.opacities[i];
      const float4 co = make_float4(cz * det_inv, -cy * det_inv, cx * det_inv, op);
      const float mid = 0.5f * (cx + cz);
      const float l1 = mid + sqrtf(fmax_t(0.1f, mid * mid - det));
      const float l2 = mid - sqrtf(fmax_t(0.1f, mid * mid - det));
      const float my_radius = ceilf(3.f * sqrtf(fmax_t(l1, l2)));
      const float img_x = ((pp_x + 1.0f) * (float)p.image_width - 1.0f) * 0.5f;
      const float img_y = ((pp_y + 1.0f) * (float)p.image_height - 1.0f) * 0.5f;
      const uint32_t tc = tile_walk(img_x, img_y, co, a.gx, a.gy, p.mult, [](int) {});
      if (tc != 0u) {
        if (a.skip_color) {
        } else if (p.use_colors_precomp) {
#pragma unroll
          for (int c = 0; c < 3; ++c) rgb_out[c] = a.colors_precomp[3 * (int64_t)i + c];
        } else {
          const v3 d = V3(po.x - a.cam_pos[0], po.y - a.cam_pos[1], po.z - a.cam_pos[2]);
          const float* shp = use_sh ? (s_sh + threadIdx.x * S3) : nullptr;
          const v3 col = sh_color(use_sh ? p.degree : 0, d, a.dc + 3 * (int64_t)i, shp, cl);
          rgb_out[0] = col.x;
          rgb_out[1] = col.y;
          rgb_out[2] = col.z;
        }
        depth_out = pv.z;
        radius_out = f2i(my_radius);
        xy_out = make_float2(img_x, img_y);
        conic_out = co;
        tiles_out = tc;
        vs_o = make_float4(pv.x, pv.y, pv.z, a.vs_in[4 * (int64_t)i + 3]);
      }
    }
  }
  a.radii[i] = radius_out;
  a.tiles[i] = tiles_out;
  reinterpret_cast<float2*>(a.xys)[i] = xy_out;
  a.depths[i] = depth_out;
  reinterpret_cast<float4*>(a.conic)[i] = conic_out;
  reinterpret_cast<float4*>(a.vs_out)[i] = vs_o;
  if (!a.skip_color) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      a.rgb[3 * (int64_t)i + c] = rgb_out[c];
      a.clamped[3 * (int64_t)i + c] = cl[c];
    }
  }
  float2* cv = reinterpret_cast<float2*>(a.cov3d + 6 * (int64_t)i);
  cv[0] = make_float2(c3[0], c3[1]);
  cv[1] = make_float2(c3[2], c3[3]);
  cv[2] = make_float2(c3[4], c3[5]);
}

// Colour step of the training preprocess on its own: the SH colour (degree
// `degree`, 15 rest coefficients per Gaussian staged through shared memory)
// of every Gaussian that touches a tile, zeros and no clamp flags elsewhere;
// the same operations as preprocess_fwd_kernel<true>, so the same bits.
__global__ void __launch_bounds__(kPreThreads) color_train_kernel(int64_t n, int degree,
                                                                 const float* __restrict__ raw,
                                                                 const float* __restrict__ cam_pos,
                                                                 const uint32_t* __restrict__ tiles,
                                                                 float* __restrict__ rgb,
                                                                 uint8_t* __restrict__ clamped) {
  extern __shared__ float s_sh[];
  constexpr int S3 = 45;
  const int64_t base = (int64_t)blockIdx.x * kPreThreads;
  const int64_t i = base + threadIdx.x;
  const bool use_sh = degree > 0;
  if (use_sh) {
    const int cnt = (int)min((int64_t)kPreThreads, n - base);
    stage_floats(s_sh, raw + 6 * n + base * S3, (int64_t)cnt * S3);
    __syncthreads();
  }
  if (i >= n) return;
  float o[3] = {0.f, 0.f, 0.f};
  uint8_t cl[3] = {0, 0, 0};
  if (tiles[i] != 0u) {
    const v3 d = V3(raw[3 * i] - cam_pos[0], raw[3 * i + 1] - cam_pos[1], raw[3 * i + 2] - cam_pos[2]);
    const float* shp = use_sh ? (s_sh + threadIdx.x * S3) : nullptr;
    const v3 col = sh_color(use_sh ? degree : 0, d, raw + 3 * n + 3 * i, shp, cl);
    o[0] = col.x;
    o[1] = col.y;
    o[2] = col.z;
  }
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    rgb[3 * i + c] = o[c];
    clamped[3 * i + c] = cl[c];
  }
}

// ------------------------------------------------------------ prefix sum
constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp,
                                                         uint32_t& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[w] = x;
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    uint32_t s = lane < nw ? s_warp[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) s_warp[lane] = s;
  }
  __syncthreads();
  total = s_warp[(blockDim.x >> 5) - 1];
  const uint32_t r = x - v + (w > 0 ? s_warp[w - 1] : 0u);
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const uint32_t* in, int64_t n,
                                                                   uint64_t* tile_sums) {
  __shared__ uint32_t s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * kScanTile;
  uint32_t s = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t idx = base + (int64_t)k * kScanThreads + threadIdx.x;
    if (idx < n) s += in[idx];
  }
  uint32_t total;
  block_exclusive_scan(s, s_warp, total);
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

// one CTA: exclusive scan of the per-tile sums (64-bit), total into *total
__global__ void __launch_bounds__(1024) scan_tiles_kernel(uint64_t* tile_sums, int64_t ntiles,
                                                          uint64_t* total) {
  __shared__ uint64_t s_w[32];
  __shared__ uint64_t s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int64_t base = 0; base < ntiles; base += 1024) {
    const int64_t idx = base + threadIdx.x;
    const uint64_t v = idx < ntiles ? tile_sums[idx] : 0ull;
    uint64_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_w[w] = x;
    __syncthreads();
    if (w == 0) {
      uint64_t s = s_w[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint64_t y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      s_w[lane] = s;
    }
    __syncthreads();
    const uint64_t excl = s_carry + x - v + (w > 0 ? s_w[w - 1] : 0ull);
    if (idx < ntiles) tile_sums[idx] = excl;
    __syncthreads();
    if (threadIdx.x == 0) s_carry += s_w[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = s_carry;
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const uint32_t* in, int64_t n,
                                                                  const uint64_t* tile_prefix,
                                                                  uint32_t* out) {
  __shared__ uint32_t s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * kScanTile;
  // blocked arrangement: thread t owns items [t*kScanItems, (t+1)*kScanItems)
  uint32_t v[kScanItems];
  uint32_t s = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t idx = base + (int64_t)threadIdx.x * kScanItems + k;
    v[k] = idx < n ? in[idx] : 0u;
    s += v[k];
  }
  uint32_t total;
  uint32_t run = block_exclusive_scan(s, s_warp, total) + (uint32_t)tile_prefix[blockIdx.x];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t idx = base + (int64_t)threadIdx.x * kScanItems + k;
    run += v[k];
    if (idx < n) out[idx] = run;
  }
}

// ------------------------------------------------------- preprocess backward
struct PbwdArgs {
  fgs_preprocess_params p;
  float focal_x, focal_y;
  const float *means3d, *scales, *quats, *vm, *pm, *cam_pos, *sh, *cov3d_precomp, *cov3d_fwd,
      *dcov3d, *drgb, *dxys, *dconic, *dvs_out;
  const int32_t* radii;
  const uint8_t* clamped;
  float *dmeans3d, *ddc, *dsh, *dcolors_precomp, *dopac, *dscales, *dquats, *dvs_in;
  // training mode (kTrain): gradients w.r.t. the raw parameters, accumulated
  // into a flat buffer, plus densification statistics
  const float* raw;  // the flat raw parameters (59 n floats)
  float *g_means, *g_dc, *g_rest, *g_logit, *g_logscale, *g_rot;
  float *st_acc, *st_acc_abs, *st_denom, *st_max_radii;
  int accumulate;
  // Adam fused in (kAdam): the flat raw parameters and moments in the
  // gradient buffer's layout, one learning rate per attribute segment
  float *ap, *am, *av;
  float lr[6];
  float b1, b2, eps, bc1, bc2;
  // push mode (kPush): no Adam; the staged gradients
  // are added into the owning rank's gradient buffer instead (rank r owns flat
  // elements [r shard, (r + 1) shard); peer_g[r] is rank r's buffer base)
  int64_t shard;
  float* peer_g[8];
};

// Shared-memory staging of the register-held gradients in the fused Adam
// pass, per CTA: [segment][kPreThreads * width] at these offsets (units of
// kPreThreads floats); 14 floats per Gaussian in all.
enum { kAdamMeans = 0, kAdamDc = 3, kAdamLogit = 6, kAdamScale = 7, kAdamRot = 10, kAdamStaged = 14 };

// Adam over one attribute segment of the flat layout (means 3, dc 3, sh rest
// 45, opacity logit 1, log-scale 3, rotation 4 floats per Gaussian, each
// segment attribute-major) for this CTA's Gaussians [base, base + cnt): a
// contiguous run of cnt * width floats from seg + base * width, gradients in
// shared memory in the same order.
// float4s per thread per iteration of the Adam pass (config 3: 0.366 ms;
// 1: 0.373 ms, 4: 0.370 ms)
constexpr int kAdamUnroll = 2;
__device__ __forceinline__ void adam_block(const PbwdArgs& a, int64_t seg, int width, int base,
                                           int cnt, const float* sgrad, float lr) {
  float* __restrict__ P = a.ap + seg + (int64_t)base * width;
  float* __restrict__ M = a.am + seg + (int64_t)base * width;
  float* __restrict__ V = a.av + seg + (int64_t)base * width;
  if (lr < 0.0f) return;  // the group does not step this iteration
  const int count = cnt * width;
  // the three buffers share their offsets and 16-byte alignment: scalar head
  // up to the first 16-byte boundary, float4 body (two per thread per
  // iteration: six 16-byte loads in flight), scalar tail (config 3: 0.370 ms
  // for the fused kernel; 0.383 ms with four scalar elements per thread)
  const int head = min(count, (int)(((16u - (reinterpret_cast<uintptr_t>(P) & 15u)) & 15u) / 4u));
  const int body4 = (count - head) / 4;
  const int tail0 = head + 4 * body4;
  const int t = threadIdx.x;
  if (t < head || (t >= 32 && t - 32 < count - tail0)) {
    const int k = t < head ? t : tail0 + (t - 32);
    float pv = P[k], mv = M[k], vv = V[k];
    adam_elem(pv, mv, vv, sgrad[k], lr, a.b1, a.b2, a.eps, a.bc1, a.bc2);
    P[k] = pv;
    M[k] = mv;
    V[k] = vv;
  }
  float4* P4 = reinterpret_cast<float4*>(P + head);
  float4* M4 = reinterpret_cast<float4*>(M + head);
  float4* V4 = reinterpret_cast<float4*>(V + head);
  const float* G = sgrad + head;
  for (int j0 = t; j0 < body4; j0 += kAdamUnroll * kPreThreads) {
    float4 pv[kAdamUnroll], mv[kAdamUnroll], vv[kAdamUnroll];
#pragma unroll
    for (int u = 0; u < kAdamUnroll; ++u) {
      const int j = j0 + u * kPreThreads;
      if (j < body4) {
        pv[u] = P4[j];
        mv[u] = M4[j];
        vv[u] = V4[j];
      }
    }
#pragma unroll
    for (int u = 0; u < kAdamUnroll; ++u) {
      const int j = j0 + u * kPreThreads;
      if (j < body4) {
        adam_elem(pv[u].x, mv[u].x, vv[u].x, G[4 * j], lr, a.b1, a.b2, a.eps, a.bc1, a.bc2);
        adam_elem(pv[u].y, mv[u].y, vv[u].y, G[4 * j + 1], lr, a.b1, a.b2, a.eps, a.bc1, a.bc2);
        adam_elem(pv[u].z, mv[u].z, vv[u].z, G[4 * j + 2], lr, a.b1, a.b2, a.eps, a.bc1, a.bc2);
        adam_elem(pv[u].w, mv[u].w, vv[u].w, G[4 * j + 3], lr, a.b1, a.b2, a.eps, a.bc1, a.bc2);
        P4[j] = pv[u];
        M4[j] = mv[u];
        V4[j] = vv[u];
      }
    }
  }
}

__device__ __forceinline__ void red_add_sys(float* dst, float v) {
  asm volatile("red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(dst), "f"(v) : "memory");
}
__device__ __forceinline__ void red_add_sys4(float* dst, float4 v) {
  asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Push mode: adds the CTA's staged gradients of one attribute segment (the
// contiguous flat run [seg + base * width, + cnt * width)) into the buffer of
// the rank that owns each element, over NVLink for the other ranks' shards:
// 16-byte vector reductions on 4-float boundaries of the flat index (a shard
// is a multiple of 4 floats, so no vector crosses two owners), scalar ones for
// the ragged head and tail.
__device__ __forceinline__ void push_block(const PbwdArgs& a, int64_t seg, int width, int base,
                                           int cnt, const float* sgrad) {
  const int64_t g0 = seg + (int64_t)base * width;
  const int count = cnt * width;
  const int head = min(count, (int)((4 - (g0 & 3)) & 3));
  const int body4 = (count - head) / 4;
  const int tail0 = head + 4 * body4;
  const int t = threadIdx.x;
  if (t < head || (t >= 32 && t - 32 < count - tail0)) {
    const int k = t < head ? t : tail0 + (t - 32);
    const int64_t g = g0 + k;
    red_add_sys(a.peer_g[g / a.shard] + g, sgrad[k]);
  }
  for (int j = t; j < body4; j += kPreThreads) {
    const int k = head + 4 * j;
    const int64_t g = g0 + k;
    red_add_sys4(a.peer_g[g / a.shard] + g,
                 make_float4(sgrad[k], sgrad[k + 1], sgrad[k + 2], sgrad[k + 3]));
  }
}

__device__ __forceinline__ v3 v3s(float s, v3 a) { return V3(s * a.x, s * a.y, s * a.z); }
__device__ __forceinline__ v3 v3sr(v3 a, float s) { return V3(a.x * s, a.y * s, a.z * s); }
__device__ __forceinline__ v3 v3add(v3 a, v3 b) { return V3(a.x + b.x, a.y + b.y, a.z + b.z); }

// kPush (with kAdam's staging): the gradients go to their owning ranks instead
// of an Adam step (fgs_preprocess_backward_push)
template <bool kTrain, bool kAdam, bool kPush = false>
__global__ void __launch_bounds__(kPreThreads) preprocess_bwd_kernel(PbwdArgs a) {
  extern __shared__ float s_buf[];  // [kPreThreads * S3]: staged sh, overwritten by dsh
  const fgs_preprocess_params& P = a.p;
  const int base = blockIdx.x * kPreThreads;
  const int i = base + threadIdx.x;
  const int S3 = P.max_sh_coeffs * 3;
  const int cnt = min(kPreThreads, P.n - base);
  const bool sh_path = !P.use_colors_precomp && S3 > 0;
  float* s_sh = s_buf;
  float* s_dsh = s_buf;  // each thread's gradient row aliases its own sh row
  if (sh_path) {
    stage_floats(s_sh, a.sh + (int64_t)base * S3, (int64_t)cnt * S3);
    __syncthreads();
  }
  int32_t my_radius = 0;
  float4 my_dvs = make_float4(0.f, 0.f, 0.f, 0.f);
  int n_put = 0;  // leading sh coefficients of this thread's row holding gradients
  if (i < P.n) {
    float dm[3] = {0.f, 0.f, 0.f};
    float ddc[3] = {0.f, 0.f, 0.f};
    float dcp[3] = {0.f, 0.f, 0.f};
    float dop = 0.f;
    float dsc[3] = {0.f, 0.f, 0.f};
    float dq[4] = {0.f, 0.f, 0.f, 0.f};
    float4 dvs = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.radii[i] > 0) {
      const float* vm = a.vm;
      const float* pm = a.pm;
      const v3 p = V3(a.means3d[3 * i], a.means3d[3 * i + 1], a.means3d[3 * i + 2]);
      const float ph_w = pm[3] * p.x + pm[7] * p.y + pm[11] * p.z + pm[15];
      const int64_t cb = 6 * (int64_t)i;
      const float gx = a.dxys[2 * (int64_t)i], gy = a.dxys[2 * (int64_t)i + 1];
      const float* cov3D = (P.use_cov3d_precomp ? a.cov3d_precomp : a.cov3d_fwd) + cb;
      const float4 cg = reinterpret_cast<const float4*>(a.dconic)[i];
      float dce[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      v3 dmean_cov;
      {
        v3 t = xform43(p, vm);
        const float limx = 1.3f * P.tan_fovx, limy = 1.3f * P.tan_fovy;
        const float txtz = t.x / t.z, tytz = t.y / t.z;
        t.x = fmin_t(limx, fmax_t(-limx, txtz)) * t.z;
        t.y = fmin_t(limy, fmax_t(-limy, tytz)) * t.z;
        const float x_grad_mul = (txtz < -limx || txtz > limx) ? 0.0f : 1.0f;
        const float y_grad_mul = (tytz < -limy || tytz > limy) ? 0.0f : 1.0f;
        const float fx = a.focal_x, fy = a.focal_y;
        const m3 J = M3(fx / t.z, 0.0f, -(fx * t.x) / (t.z * t.z), 0.0f, fy / t.z,
                        -(fy * t.y) / (t.z * t.z), 0.0f, 0.0f, 0.0f);
        const m3 Wm = M3(vm[0], vm[1], vm[2], vm[4], vm[5], vm[6], vm[8], vm[9], vm[10]);
        const m3 V = M3(cov3D[0], cov3D[1], cov3D[2], cov3D[1], cov3D[3], cov3D[4], cov3D[2],
                        cov3D[4], cov3D[5]);
        const m3 Tm = mul(Wm, J);
        const m3 c2 = mul(mul(tr(Tm), tr(V)), Tm);
        const float aa = c2.c[0].x + 0.3f, b = c2.c[0].y, c = c2.c[1].y + 0.3f;
        const float denom = aa * c - b * b;
        const float denom2inv = 1.0f / ((denom * denom) + 1e-7f);
        float dL_da = 0.f, dL_db = 0.f, dL_dc = 0.f;
#define T_(i_, j_) mat(Tm, i_, j_)
#define V_(i_, j_) mat(V, i_, j_)
#define W_(i_, j_) mat(Wm, i_, j_)
        if (denom2inv != 0.0f) {
          dL_da = denom2inv * (-c * c * cg.x + 2.0f * b * c * cg.y + (denom - aa * c) * cg.z);
          dL_dc = denom2inv * (-aa * aa * cg.z + 2.0f * aa * b * cg.y + (denom - aa * c) * cg.x);
          dL_db = denom2inv * 2.0f * (b * c * cg.x - (denom + 2.0f * b * b) * cg.y + aa * b * cg.z);
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
        dmean_cov = V3(vm[0] * dtx + vm[1] * dty + vm[2] * dtz,
                       vm[4] * dtx + vm[5] * dty + vm[6] * dtz,
                       vm[8] * dtx + vm[9] * dty + vm[10] * dtz);
      }
      const float m_w = 1.0f / (ph_w + 1.0e-7f);
      const float mul1 = (pm[0] * p.x + pm[4] * p.y + pm[8] * p.z + pm[12]) * m_w * m_w;
      const float mul2 = (pm[1] * p.x + pm[5] * p.y + pm[9] * p.z + pm[13]) * m_w * m_w;
      const float dmx = (pm[0] * m_w - pm[3] * mul1) * gx + (pm[1] * m_w - pm[3] * mul2) * gy;
      const float dmy = (pm[4] * m_w - pm[7] * mul1) * gx + (pm[5] * m_w - pm[7] * mul2) * gy;
      const float dmz = (pm[8] * m_w - pm[11] * mul1) * gx + (pm[9] * m_w - pm[11] * mul2) * gy;
      dm[0] = dmx + dmean_cov.x;
      dm[1] = dmy + dmean_cov.y;
      dm[2] = dmz + dmean_cov.z;
      dop = cg.w;
      if (P.use_colors_precomp) {
#pragma unroll
        for (int c = 0; c < 3; ++c) dcp[c] = a.drgb[3 * (int64_t)i + c];
      } else {
        const v3 dRGB = V3(a.clamped[3 * (int64_t)i] ? 0.0f : a.drgb[3 * (int64_t)i],
                           a.clamped[3 * (int64_t)i + 1] ? 0.0f : a.drgb[3 * (int64_t)i + 1],
                           a.clamped[3 * (int64_t)i + 2] ? 0.0f : a.drgb[3 * (int64_t)i + 2]);
        ddc[0] = kSH_C0 * dRGB.x;
        ddc[1] = kSH_C0 * dRGB.y;
        ddc[2] = kSH_C0 * dRGB.z;
        if (P.degree > 0 && P.max_sh_coeffs >= 3) {
          const v3 dir_orig = V3(p.x - a.cam_pos[0], p.y - a.cam_pos[1], p.z - a.cam_pos[2]);
          const float dl = sqrtf(dot3(dir_orig, dir_orig));
          const float x = dir_orig.x / dl, y = dir_orig.y / dl, z = dir_orig.z / dl;
          const float* s = s_sh + threadIdx.x * S3;
          float* g = s_dsh + threadIdx.x * S3;
#define SHC(k) V3(s[3 * (k)], s[3 * (k) + 1], s[3 * (k) + 2])
#define PUT(k, v)            \
  do {                       \
    const v3 v_ = (v);       \
    g[3 * (k)] = v_.x;       \
    g[3 * (k) + 1] = v_.y;   \
    g[3 * (k) + 2] = v_.z;   \
  } while (0)
          const float C1 = kSH_C1;
          const float xx = x * x, yy = y * y, zz = z * z;
          const float xy = x * y, yz = y * z, xz = x * z;
          v3 dx_ = v3s(-C1, SHC(2));
          v3 dy_ = v3s(-C1, SHC(0));
          v3 dz_ = v3s(C1, SHC(1));
          if (P.degree > 1 && P.max_sh_coeffs >= 8) {
            const float C20 = 1.0925484305920792f, C21 = -1.0925484305920792f,
                        C22 = 0.31539156525252005f, C23 = -1.0925484305920792f,
                        C24 = 0.5462742152960396f;
            {
              v3 s1 = v3s(C20 * y, SHC(3));
              s1 = v3add(s1, v3s(C22 * 2.f * -x, SHC(5)));
              s1 = v3add(s1, v3s(C23 * z, SHC(6)));
              s1 = v3add(s1, v3s(C24 * 2.f * x, SHC(7)));
              dx_ = v3add(dx_, s1);
            }
            {
              v3 s1 = v3s(C20 * x, SHC(3));
              s1 = v3add(s1, v3s(C21 * z, SHC(4)));
              s1 = v3add(s1, v3s(C22 * 2.f * -y, SHC(5)));
              s1 = v3add(s1, v3s(C24 * 2.f * -y, SHC(7)));
              dy_ = v3add(dy_, s1);
            }
            {
              v3 s1 = v3s(C21 * y, SHC(4));
              s1 = v3add(s1, v3s(C22 * 4.f * z, SHC(5)));
              s1 = v3add(s1, v3s(C23 * x, SHC(6)));
              dz_ = v3add(dz_, s1);
            }
            if (P.degree > 2 && P.max_sh_coeffs >= 15) {
              const float C30 = -0.5900435899266435f, C31 = 2.890611442640554f,
                          C32 = -0.4570457994644658f, C33 = 0.3731763325901154f,
                          C34 = -0.4570457994644658f, C35 = 1.445305721320277f,
                          C36 = -0.5900435899266435f;
              {
                v3 s1 = v3sr(v3sr(v3s(C30, SHC(8)), 6.f), xy);
                s1 = v3add(s1, v3sr(v3s(C31, SHC(9)), yz));
                s1 = v3add(s1, v3sr(v3sr(v3s(C32, SHC(10)), -2.f), xy));
                s1 = v3add(s1, v3sr(v3sr(v3s(C33, SHC(11)), -6.f), xz));
                s1 = v3add(s1, v3sr(v3s(C34, SHC(12)), (-3.f * xx + 4.f * zz - yy)));
                s1 = v3add(s1, v3sr(v3sr(v3s(C35, SHC(13)), 2.f), xz));
                s1 = v3add(s1, v3sr(v3sr(v3s(C36, SHC(14)), 3.f), (xx - yy)));
                dx_ = v3add(dx_, s1);
              }
              {
                v3 s1 = v3sr(v3sr(v3s(C30, SHC(8)), 3.f), (xx - yy));
                s1 = v3add(s1, v3sr(v3s(C31, SHC(9)), xz));
                s1 = v3add(s1, v3sr(v3s(C32, SHC(10)), (-3.f * yy + 4.f * zz - xx)));
                s1 = v3add(s1, v3sr(v3sr(v3s(C33, SHC(11)), -6.f), yz));
                s1 = v3add(s1, v3sr(v3sr(v3s(C34, SHC(12)), -2.f), xy));
                s1 = v3add(s1, v3sr(v3sr(v3s(C35, SHC(13)), -2.f), yz));
                s1 = v3add(s1, v3sr(v3sr(v3s(C36, SHC(14)), -6.f), xy));
                dy_ = v3add(dy_, s1);
              }
              {
                v3 s1 = v3sr(v3s(C31, SHC(9)), xy);
                s1 = v3add(s1, v3sr(v3sr(v3s(C32, SHC(10)), 8.f), yz));
                s1 = v3add(s1, v3sr(v3sr(v3s(C33, SHC(11)), 3.f), (2.f * zz - xx - yy)));
                s1 = v3add(s1, v3sr(v3sr(v3s(C34, SHC(12)), 8.f), xz));
                s1 = v3add(s1, v3sr(v3s(C35, SHC(13)), (xx - yy)));
                dz_ = v3add(dz_, s1);
              }
            }
          }
          // Every SHC read above precedes the first PUT: the gradient row
          // overwrites this thread's own staged coefficients in place.
          {
            const float C20 = 1.0925484305920792f, C21 = -1.0925484305920792f,
                        C22 = 0.31539156525252005f, C23 = -1.0925484305920792f,
                        C24 = 0.5462742152960396f;
            const float C30 = -0.5900435899266435f, C31 = 2.890611442640554f,
                        C32 = -0.4570457994644658f, C33 = 0.3731763325901154f,
                        C34 = -0.4570457994644658f, C35 = 1.445305721320277f,
                        C36 = -0.5900435899266435f;
            PUT(0, v3s(-C1 * y, dRGB));
            PUT(1, v3s(C1 * z, dRGB));
            PUT(2, v3s(-C1 * x, dRGB));
            n_put = 3;
            if (P.degree > 1 && P.max_sh_coeffs >= 8) {
              PUT(3, v3s(C20 * xy, dRGB));
              PUT(4, v3s(C21 * yz, dRGB));
              PUT(5, v3s(C22 * (2.0f * zz - xx - yy), dRGB));
              PUT(6, v3s(C23 * xz, dRGB));
              PUT(7, v3s(C24 * (xx - yy), dRGB));
              n_put = 8;
              if (P.degree > 2 && P.max_sh_coeffs >= 15) {
                PUT(8, v3s(C30 * y * (3.f * xx - yy), dRGB));
                PUT(9, v3s(C31 * xy * z, dRGB));
                PUT(10, v3s(C32 * y * (4.f * zz - xx - yy), dRGB));
                PUT(11, v3s(C33 * z * (2.f * zz - 3.f * xx - 3.f * yy), dRGB));
                PUT(12, v3s(C34 * x * (4.f * zz - xx - yy), dRGB));
                PUT(13, v3s(C35 * z * (xx - yy), dRGB));
                PUT(14, v3s(C36 * x * (xx - 3.f * yy), dRGB));
                n_put = 15;
              }
            }
          }
#undef SHC
#undef PUT
          const v3 ddir = V3(dot3(dx_, dRGB), dot3(dy_, dRGB), dot3(dz_, dRGB));
          const float len = fmax_t(sqrtf(dot3(dir_orig, dir_orig)), 1e-6f);
          const v3 nn = V3(dir_orig.x / len, dir_orig.y / len, dir_orig.z / len);
          const float nd = dot3(nn, ddir);
          dm[0] = dm[0] + (ddir.x - nn.x * nd) / len;
          dm[1] = dm[1] + (ddir.y - nn.y * nd) / len;
          dm[2] = dm[2] + (ddir.z - nn.z * nd) / len;
        }
      }
      if (!P.use_cov3d_precomp) {
        v3 scale;
        float4 q;
        if constexpr (kTrain) {
          const float* ls = a.raw + 52 * (int64_t)P.n + 3 * (int64_t)i;
          scale = V3(act_scale(ls[0]), act_scale(ls[1]), act_scale(ls[2]));
          q = act_quat(raw_quat(a.raw + 55 * (int64_t)P.n + 4 * (int64_t)i));
        } else {
          scale = V3(a.scales[3 * i], a.scales[3 * i + 1], a.scales[3 * i + 2]);
          q = reinterpret_cast<const float4*>(a.quats)[i];
        }
        const float r = q.x, x = q.y, y = q.z, z = q.w;
        const m3 R = M3(1.f - 2.f * (y * y + z * z), 2.f * (x * y - r * z), 2.f * (x * z + r * y),
                        2.f * (x * y + r * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - r * x),
                        2.f * (x * z - r * y), 2.f * (y * z + r * x), 1.f - 2.f * (x * x + y * y));
        const v3 s = v3s(P.scale_modifier, scale);
        m3 S = M3(1.f, 0.f, 0.f, 0.f, 1.f, 0.f, 0.f, 0.f, 1.f);
        S.c[0].x = s.x;
        S.c[1].y = s.y;
        S.c[2].z = s.z;
        const m3 M = mul(S, R);
        float dc3[6];
#pragma unroll
        for (int k = 0; k < 6; ++k) dc3[k] = (a.dcov3d ? a.dcov3d[cb + k] : 0.0f) + dce[k];
        const m3 dSigma = M3(dc3[0], 0.5f * dc3[1], 0.5f * dc3[2], 0.5f * dc3[1], dc3[3],
                             0.5f * dc3[4], 0.5f * dc3[2], 0.5f * dc3[4], dc3[5]);
        m3 M2;
#pragma unroll
        for (int k = 0; k < 3; ++k) M2.c[k] = v3s(2.0f, M.c[k]);
        const m3 dM = mul(M2, dSigma);
        const m3 Rt = tr(R);
        m3 dMt = tr(dM);
        dsc[0] = dot3(Rt.c[0], dMt.c[0]);
        dsc[1] = dot3(Rt.c[1], dMt.c[1]);
        dsc[2] = dot3(Rt.c[2], dMt.c[2]);
        dMt.c[0] = v3sr(dMt.c[0], s.x);
        dMt.c[1] = v3sr(dMt.c[1], s.y);
        dMt.c[2] = v3sr(dMt.c[2], s.z);
#define D_(i_, j_) mat(dMt, i_, j_)
        dq[0] = 2 * z * (D_(0, 1) - D_(1, 0)) + 2 * y * (D_(2, 0) - D_(0, 2)) +
                2 * x * (D_(1, 2) - D_(2, 1));
        dq[1] = 2 * y * (D_(1, 0) + D_(0, 1)) + 2 * z * (D_(2, 0) + D_(0, 2)) +
                2 * r * (D_(1, 2) - D_(2, 1)) - 4 * x * (D_(2, 2) + D_(1, 1));
        dq[2] = 2 * x * (D_(1, 0) + D_(0, 1)) + 2 * r * (D_(2, 0) - D_(0, 2)) +
                2 * z * (D_(1, 2) + D_(2, 1)) - 4 * y * (D_(2, 2) + D_(0, 0));
        dq[3] = 2 * r * (D_(0, 1) - D_(1, 0)) + 2 * x * (D_(2, 0) + D_(0, 2)) +
                2 * y * (D_(1, 2) + D_(2, 1)) - 4 * z * (D_(1, 1) + D_(0, 0));
#undef D_
      }
      dvs = reinterpret_cast<const float4*>(a.dvs_out)[i];
    }
    if constexpr (!kTrain) {
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        a.dmeans3d[3 * (int64_t)i + c] = dm[c];
        a.ddc[3 * (int64_t)i + c] = ddc[c];
        a.dcolors_precomp[3 * (int64_t)i + c] = dcp[c];
        a.dscales[3 * (int64_t)i + c] = dsc[c];
      }
      a.dopac[i] = dop;
      reinterpret_cast<float4*>(a.dquats)[i] = make_float4(dq[0], dq[1], dq[2], dq[3]);
      reinterpret_cast<float4*>(a.dvs_in)[i] = dvs;
    } else {
      // activation backward: opacity = sigmoid(logit), scale = exp(log_scale),
      // quat = q / (|q| + 1e-8) (the trainers' getters,
      // scripts/train_scanner_fixed.py:523-535)
      const float o = act_opacity(a.raw[51 * (int64_t)P.n + i]);
      const float dlogit = dop * o * (1.0f - o);
      float dls[3];
#pragma unroll
      for (int c = 0; c < 3; ++c)
        dls[c] = dsc[c] * act_scale(a.raw[52 * (int64_t)P.n + 3 * (int64_t)i + c]);
      // scalar accesses to the flat buffers: their rotation segment starts at
      // 55 n floats, 16-byte aligned only when n is a multiple of 4
      const float4 qr = raw_quat(a.raw + 55 * (int64_t)P.n + 4 * (int64_t)i);
      const float qn = sqrtf(qr.x * qr.x + qr.y * qr.y + qr.z * qr.z + qr.w * qr.w);
      const float inv = 1.0f / (qn + 1e-8f);
      const float qdot = qr.x * dq[0] + qr.y * dq[1] + qr.z * dq[2] + qr.w * dq[3];
      const float corr = qn > 0.0f ? qdot * inv * inv / qn : 0.0f;
      const float dr[4] = {dq[0] * inv - qr.x * corr, dq[1] * inv - qr.y * corr,
                           dq[2] * inv - qr.z * corr, dq[3] * inv - qr.w * corr};
      if constexpr (kAdam) {
        // staged for the CTA-wide, coalesced Adam pass at the end
        float* sg = s_buf + kPreThreads * S3;
        const int t = threadIdx.x;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          sg[kAdamMeans * kPreThreads + 3 * t + c] = dm[c];
          sg[kAdamDc * kPreThreads + 3 * t + c] = ddc[c];
          sg[kAdamScale * kPreThreads + 3 * t + c] = dls[c];
        }
        sg[kAdamLogit * kPreThreads + t] = dlogit;
#pragma unroll
        for (int c = 0; c < 4; ++c) sg[kAdamRot * kPreThreads + 4 * t + c] = dr[c];
      } else {
        const bool acc = a.accumulate != 0;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          float* gm = a.g_means + 3 * (int64_t)i + c;
          float* gd = a.g_dc + 3 * (int64_t)i + c;
          float* gs = a.g_logscale + 3 * (int64_t)i + c;
          *gm = acc ? *gm + dm[c] : dm[c];
          *gd = acc ? *gd + ddc[c] : ddc[c];
          *gs = acc ? *gs + dls[c] : dls[c];
        }
        a.g_logit[i] = acc ? a.g_logit[i] + dlogit : dlogit;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float* gr = a.g_rot + 4 * (int64_t)i + c;
          *gr = acc ? *gr + dr[c] : dr[c];
        }
      }
      my_radius = a.radii[i];
      my_dvs = dvs;
      // densification statistics (scripts/train_scanner_fastgs.py:391-405)
      if (my_radius > 0) {
        a.st_acc[i] += sqrtf(my_dvs.x * my_dvs.x + my_dvs.y * my_dvs.y);
        a.st_acc_abs[i] += sqrtf(my_dvs.z * my_dvs.z + my_dvs.w * my_dvs.w);
        a.st_denom[i] += 1.0f;
        a.st_max_radii[i] = fmax_t(a.st_max_radii[i], (float)my_radius);
      }
    }
  }
  float* dsh_dst = kTrain ? a.g_rest : a.dsh;
  if (sh_path) {
    if (threadIdx.x < cnt) {
      float* row = s_dsh + threadIdx.x * S3;
      for (int k = 3 * n_put; k < S3; ++k) row[k] = 0.0f;
    }
    __syncthreads();
    float* gdst = dsh_dst + (int64_t)base * S3;
    if constexpr (kPush) {
      const int64_t n = P.n;
      const float* sg = s_buf + kPreThreads * S3;
      push_block(a, 0, 3, base, cnt, sg + kAdamMeans * kPreThreads);
      push_block(a, 3 * n, 3, base, cnt, sg + kAdamDc * kPreThreads);
      push_block(a, 6 * n, S3, base, cnt, s_dsh);
      push_block(a, 51 * n, 1, base, cnt, sg + kAdamLogit * kPreThreads);
      push_block(a, 52 * n, 3, base, cnt, sg + kAdamScale * kPreThreads);
      push_block(a, 55 * n, 4, base, cnt, sg + kAdamRot * kPreThreads);
      // the reductions reach the other GPUs before the caller's barrier
      asm volatile("fence.acq_rel.sys;" ::: "memory");
    } else if (kAdam) {
      const int64_t n = P.n;
      const float* sg = s_buf + kPreThreads * S3;
      adam_block(a, 0, 3, base, cnt, sg + kAdamMeans * kPreThreads, a.lr[0]);
      adam_block(a, 3 * n, 3, base, cnt, sg + kAdamDc * kPreThreads, a.lr[1]);
      adam_block(a, 6 * n, S3, base, cnt, s_dsh, a.lr[2]);
      adam_block(a, 51 * n, 1, base, cnt, sg + kAdamLogit * kPreThreads, a.lr[3]);
      adam_block(a, 52 * n, 3, base, cnt, sg + kAdamScale * kPreThreads, a.lr[4]);
      adam_block(a, 55 * n, 4, base, cnt, sg + kAdamRot * kPreThreads, a.lr[5]);
    } else if (kTrain && a.accumulate) {
      for (int k = threadIdx.x; k < cnt * S3; k += blockDim.x) gdst[k] += s_dsh[k];
    } else {
      for (int k = threadIdx.x; k < cnt * S3; k += blockDim.x) gdst[k] = s_dsh[k];
    }
  } else if (S3 > 0 && dsh_dst && !(kTrain && a.accumulate)) {
    float* gdst = dsh_dst + (int64_t)base * S3;
    for (int k = threadIdx.x; k < cnt * S3; k += blockDim.x) gdst[k] = 0.0f;
  }
  (void)my_radius;
}

}  // namespace fgs

using namespace fgs;

extern "C" {

const char* fgs_last_error(void) { return fgs::g_err; }
int fgs_version(void) { return 0x000100; }

static int validate_pre(const fgs_preprocess_params* p) {
  FGS_CHECK_ARG(p != nullptr, "params is NULL");
  FGS_CHECK_ARG(p->n >= 0, "n must be >= 0");
  FGS_CHECK_ARG(p->max_sh_coeffs >= 0 && p->max_sh_coeffs <= 15,
                "max_sh_coeffs must be in [0, 15], got %d", p->max_sh_coeffs);
  FGS_CHECK_ARG(p->image_width > 0 && p->image_height > 0, "image size must be positive");
  return FGS_OK;
}

int fgs_preprocess_forward(const fgs_preprocess_params* p, const float* means3d, const float* dc,
                           const float* sh, const float* colors_precomp, const float* opacities,
                           const float* scales, const float* quats, const float* cov3d_precomp,
                           const float* viewmatrix, const float* projmatrix, const float* cam_pos,
                           const float* viewspace_in, int32_t* radii, float* xys, float* depths,
                           float* cov3d, float* rgb, float* conic_opacity, uint32_t* tiles_touched,
                           uint8_t* clamped, float* viewspace_out, void* stream) {
  int st = validate_pre(p);
  if (st) return st;
  if (p->n == 0) return FGS_OK;
  FGS_CHECK_ARG(means3d && opacities && viewmatrix && projmatrix && cam_pos && viewspace_in,
                "missing required input pointer");
  FGS_CHECK_ARG(p->use_colors_precomp ? colors_precomp != nullptr : dc != nullptr,
                "missing colour input");
  FGS_CHECK_ARG(p->use_colors_precomp || p->max_sh_coeffs == 0 || sh != nullptr, "missing sh");
  FGS_CHECK_ARG(p->use_cov3d_precomp ? cov3d_precomp != nullptr : (scales && quats),
                "missing geometry input");
  FGS_CHECK_ARG(radii && xys && depths && cov3d && rgb && conic_opacity && tiles_touched &&
                    clamped && viewspace_out,
                "missing output pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(xys, 8) && FGS_ALIGNED(cov3d, 8) && FGS_ALIGNED(conic_opacity, 16) &&
                    FGS_ALIGNED(viewspace_out, 16) && (p->use_cov3d_precomp || FGS_ALIGNED(quats, 16)),
                "xys and cov3d must be 8-byte, conic_opacity, viewspace_out and rotations "
                "16-byte aligned");
  PreArgs a;
  memset(&a, 0, sizeof(a));
  a.p = *p;
  a.focal_x = (float)p->image_width / (2.0f * p->tan_fovx);
  a.focal_y = (float)p->image_height / (2.0f * p->tan_fovy);
  a.gx = (p->image_width + 15) / 16;
  a.gy = (p->image_height + 15) / 16;
  a.means3d = means3d; a.dc = dc; a.sh = sh; a.colors_precomp = colors_precomp;
  a.opacities = opacities; a.scales = scales; a.quats = quats; a.cov3d_precomp = cov3d_precomp;
  a.viewmatrix = viewmatrix; a.projmatrix = projmatrix; a.cam_pos = cam_pos; a.vs_in = viewspace_in;
  a.radii = radii; a.xys = xys; a.depths = depths; a.cov3d = cov3d; a.rgb = rgb;
  a.conic = conic_opacity; a.tiles = tiles_touched; a.clamped = clamped; a.vs_out = viewspace_out;
  const bool use_sh = !p->use_colors_precomp && p->degree > 0 && p->max_sh_coeffs > 0;
  const size_t smem = use_sh ? (size_t)kPreThreads * p->max_sh_coeffs * 3 * sizeof(float) : 0;
  static unsigned long long attr_done = 0;
  if (smem > 48 * 1024) smem_attr_once(preprocess_fwd_kernel<false>, (int)smem, &attr_done);
  const int blocks = (p->n + kPreThreads - 1) / kPreThreads;
  preprocess_fwd_kernel<false><<<blocks, kPreThreads, smem, (cudaStream_t)stream>>>(a);
  return check_launch("preprocess_forward");
}

static int launch_forward_train(const fgs_preprocess_params* p, const float* params,
                                const float* viewmatrix, const float* projmatrix,
                                const float* cam_pos, const float* viewspace_in, int32_t* radii,
                                float* xys, float* depths, float* cov3d, float* rgb,
                                float* conic_opacity, uint32_t* tiles_touched, uint8_t* clamped,
                                float* viewspace_out, bool color, void* stream) {
  int st = validate_pre(p);
  if (st) return st;
  if (p->n == 0) return FGS_OK;
  FGS_CHECK_ARG(!p->use_cov3d_precomp && !p->use_colors_precomp,
                "training mode needs the scales+quats and dc+sh paths");
  FGS_CHECK_ARG(p->max_sh_coeffs == 15, "training mode stores 15 SH rest coefficients");
  FGS_CHECK_ARG(params && viewmatrix && projmatrix && viewspace_in && (cam_pos || !color),
                "missing input pointer");
  FGS_CHECK_ARG(radii && xys && depths && cov3d && conic_opacity && tiles_touched &&
                    viewspace_out && ((rgb && clamped) || !color),
                "missing output pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(xys, 8) && FGS_ALIGNED(cov3d, 8) && FGS_ALIGNED(conic_opacity, 16) &&
                    FGS_ALIGNED(viewspace_out, 16),
                "xys and cov3d must be 8-byte, conic_opacity and viewspace_out 16-byte aligned");
  const int64_t n = p->n;
  PreArgs a;
  memset(&a, 0, sizeof(a));
  a.p = *p;
  a.focal_x = (float)p->image_width / (2.0f * p->tan_fovx);
  a.focal_y = (float)p->image_height / (2.0f * p->tan_fovy);
  a.gx = (p->image_width + 15) / 16;
  a.gy = (p->image_height + 15) / 16;
  a.raw = params;
  a.means3d = params; a.dc = params + 3 * n; a.sh = params + 6 * n;
  a.viewmatrix = viewmatrix; a.projmatrix = projmatrix; a.cam_pos = cam_pos; a.vs_in = viewspace_in;
  a.radii = radii; a.xys = xys; a.depths = depths; a.cov3d = cov3d; a.rgb = rgb;
  a.conic = conic_opacity; a.tiles = tiles_touched; a.clamped = clamped; a.vs_out = viewspace_out;
  a.skip_color = color ? 0 : 1;
  const bool use_sh = color && p->degree > 0;
  const size_t smem = use_sh ? (size_t)kPreThreads * p->max_sh_coeffs * 3 * sizeof(float) : 0;
  static unsigned long long attr_done = 0;
  if (smem > 48 * 1024) smem_attr_once(preprocess_fwd_kernel<true>, (int)smem, &attr_done);
  const int blocks = (int)((n + kPreThreads - 1) / kPreThreads);
  preprocess_fwd_kernel<true><<<blocks, kPreThreads, smem, (cudaStream_t)stream>>>(a);
  return check_launch(color ? "preprocess_forward_train" : "preprocess_forward_train_geometry");
}

int fgs_preprocess_forward_train(const fgs_preprocess_params* p, const float* params,
                                 const float* viewmatrix, const float* projmatrix,
                                 const float* cam_pos, const float* viewspace_in, int32_t* radii,
                                 float* xys, float* depths, float* cov3d, float* rgb,
                                 float* conic_opacity, uint32_t* tiles_touched, uint8_t* clamped,
                                 float* viewspace_out, void* stream) {
  return launch_forward_train(p, params, viewmatrix, projmatrix, cam_pos, viewspace_in, radii, xys,
                              depths, cov3d, rgb, conic_opacity, tiles_touched, clamped,
                              viewspace_out, true, stream);
}

int fgs_preprocess_forward_train_geometry(const fgs_preprocess_params* p, const float* params,
                                          const float* viewmatrix, const float* projmatrix,
                                          const float* viewspace_in, int32_t* radii, float* xys,
                                          float* depths, float* cov3d, float* conic_opacity,
                                          uint32_t* tiles_touched, float* viewspace_out,
                                          void* stream) {
  return launch_forward_train(p, params, viewmatrix, projmatrix, nullptr, viewspace_in, radii, xys,
                              depths, cov3d, nullptr, conic_opacity, tiles_touched, nullptr,
                              viewspace_out, false, stream);
}

int fgs_preprocess_colors_train(const fgs_preprocess_params* p, const float* params,
                                const float* cam_pos, const uint32_t* tiles_touched, float* rgb,
                                uint8_t* clamped, void* stream) {
  int st = validate_pre(p);
  if (st) return st;
  if (p->n == 0) return FGS_OK;
  FGS_CHECK_ARG(!p->use_colors_precomp && p->max_sh_coeffs == 15,
                "training mode stores dc + 15 SH rest coefficients");
  FGS_CHECK_ARG(p->degree >= 0 && p->degree <= 3, "degree must be in [0, 3]");
  FGS_CHECK_ARG(params && cam_pos && tiles_touched && rgb && clamped, "missing pointer");
  const size_t smem = p->degree > 0 ? (size_t)kPreThreads * 45 * sizeof(float) : 0;
  static unsigned long long attr_done = 0;
  if (smem > 48 * 1024) smem_attr_once(color_train_kernel, (int)smem, &attr_done);
  const int64_t n = p->n;
  const unsigned blocks = (unsigned)((n + kPreThreads - 1) / kPreThreads);
  color_train_kernel<<<blocks, kPreThreads, smem, (cudaStream_t)stream>>>(n, p->degree, params,
                                                                         cam_pos, tiles_touched,
                                                                         rgb, clamped);
  return check_launch("preprocess_colors_train");
}

size_t fgs_scan_scratch_bytes(int64_t n) {
  const int64_t tiles = (n + kScanTile - 1) / kScanTile;
  return (size_t)(tiles > 0 ? tiles : 1) * sizeof(uint64_t);
}

int fgs_inclusive_scan_u32(int64_t n, const uint32_t* in, uint32_t* out, uint64_t* total,
                           void* scratch, void* stream) {
  FGS_CHECK_ARG(n >= 0, "n must be >= 0");
  FGS_CHECK_ARG(total && scratch, "missing total / scratch");
  cudaStream_t s = (cudaStream_t)stream;
  if (n == 0) {
    cudaMemsetAsync(total, 0, sizeof(uint64_t), s);
    return check_launch("inclusive_scan");
  }
  FGS_CHECK_ARG(in && out, "missing in / out");
  const int64_t tiles = (n + kScanTile - 1) / kScanTile;
  uint64_t* ts = (uint64_t*)scratch;
  scan_reduce_kernel<<<(unsigned)tiles, kScanThreads, 0, s>>>(in, n, ts);
  scan_tiles_kernel<<<1, 1024, 0, s>>>(ts, tiles, total);
  scan_apply_kernel<<<(unsigned)tiles, kScanThreads, 0, s>>>(in, n, ts, out);
  return check_launch("inclusive_scan");
}

int fgs_preprocess_backward(const fgs_preprocess_params* p, const float* means3d,
                            const float* scales, const float* quats, const float* viewmatrix,
                            const float* projmatrix, const float* cam_pos, const float* sh,
                            const float* cov3d_precomp, const float* cov3d_fwd,
                            const float* dL_dcov3d, const float* dL_drgb, const float* dL_dxys,
                            const float* dL_dconic_opacity, const float* dL_dviewspace_out,
                            const int32_t* radii, const uint8_t* clamped, float* dL_dmeans3d,
                            float* dL_ddc, float* dL_dsh, float* dL_dcolors_precomp,
                            float* dL_dopacities, float* dL_dscales, float* dL_dquats,
                            float* dL_dviewspace_in, void* stream) {
  int st = validate_pre(p);
  if (st) return st;
  if (p->n == 0) return FGS_OK;
  FGS_CHECK_ARG(means3d && viewmatrix && projmatrix && cam_pos && dL_drgb && dL_dxys &&
                    dL_dconic_opacity && dL_dviewspace_out && radii && clamped,
                "missing input pointer");
  FGS_CHECK_ARG(p->use_cov3d_precomp ? cov3d_precomp != nullptr : (scales && quats && cov3d_fwd),
                "missing geometry input");
  FGS_CHECK_ARG(p->use_colors_precomp || p->max_sh_coeffs == 0 || sh != nullptr, "missing sh");
  FGS_CHECK_ARG(dL_dmeans3d && dL_ddc && dL_dcolors_precomp && dL_dopacities && dL_dscales &&
                    dL_dquats && dL_dviewspace_in && (p->max_sh_coeffs == 0 || dL_dsh),
                "missing output pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(dL_dconic_opacity, 16) && FGS_ALIGNED(dL_dviewspace_out, 16) &&
                    FGS_ALIGNED(dL_dquats, 16) && FGS_ALIGNED(dL_dviewspace_in, 16) &&
                    (p->use_cov3d_precomp || FGS_ALIGNED(quats, 16)),
                "rotations, conic and viewspace gradients must be 16-byte aligned");
  PbwdArgs a;
  memset(&a, 0, sizeof(a));
  a.p = *p;
  a.focal_x = 0.5f * (float)p->image_width / (p->tan_fovx < 1e-6f ? 1e-6f : p->tan_fovx);
  a.focal_y = 0.5f * (float)p->image_height / (p->tan_fovy < 1e-6f ? 1e-6f : p->tan_fovy);
  a.means3d = means3d; a.scales = scales; a.quats = quats; a.vm = viewmatrix; a.pm = projmatrix;
  a.cam_pos = cam_pos; a.sh = sh; a.cov3d_precomp = cov3d_precomp; a.cov3d_fwd = cov3d_fwd;
  a.dcov3d = dL_dcov3d; a.drgb = dL_drgb; a.dxys = dL_dxys; a.dconic = dL_dconic_opacity;
  a.dvs_out = dL_dviewspace_out; a.radii = radii; a.clamped = clamped;
  a.dmeans3d = dL_dmeans3d; a.ddc = dL_ddc; a.dsh = dL_dsh; a.dcolors_precomp = dL_dcolors_precomp;
  a.dopac = dL_dopacities; a.dscales = dL_dscales; a.dquats = dL_dquats; a.dvs_in = dL_dviewspace_in;
  const bool sh_path = !p->use_colors_precomp && p->max_sh_coeffs > 0;
  const size_t smem = sh_path ? (size_t)kPreThreads * p->max_sh_coeffs * 3 * sizeof(float) : 0;
  static unsigned long long attr_done = 0;
  if (smem > 48 * 1024) smem_attr_once(preprocess_bwd_kernel<false, false>, (int)smem, &attr_done);
  const int blocks = (p->n + kPreThreads - 1) / kPreThreads;
  preprocess_bwd_kernel<false, false><<<blocks, kPreThreads, smem, (cudaStream_t)stream>>>(a);
  return check_launch("preprocess_backward");
}

int fgs_preprocess_backward_train(const fgs_preprocess_params* p, const float* params,
                                  const float* viewmatrix, const float* projmatrix,
                                  const float* cam_pos, const float* cov3d_fwd,
                                  const float* dL_drgb, const float* dL_dxys,
                                  const float* dL_dconic_opacity, const float* dL_dviewspace,
                                  const int32_t* radii, const uint8_t* clamped, int32_t accumulate,
                                  float* grad_flat, float* stats, void* stream) {
  int st = validate_pre(p);
  if (st) return st;
  if (p->n == 0) return FGS_OK;
  FGS_CHECK_ARG(!p->use_cov3d_precomp && !p->use_colors_precomp,
                "training mode needs the scales+quats and dc+sh paths");
  FGS_CHECK_ARG(p->max_sh_coeffs == 15, "training mode stores 15 SH rest coefficients");
  FGS_CHECK_ARG(params && viewmatrix && projmatrix && cam_pos && cov3d_fwd && dL_drgb && dL_dxys &&
                    dL_dconic_opacity && dL_dviewspace && radii && clamped && grad_flat && stats,
                "missing pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(dL_dconic_opacity, 16) && FGS_ALIGNED(dL_dviewspace, 16),
                "conic and viewspace gradients must be 16-byte aligned");
  const int64_t n = p->n;
  PbwdArgs a;
  memset(&a, 0, sizeof(a));
  a.p = *p;
  a.focal_x = 0.5f * (float)p->image_width / (p->tan_fovx < 1e-6f ? 1e-6f : p->tan_fovx);
  a.focal_y = 0.5f * (float)p->image_height / (p->tan_fovy < 1e-6f ? 1e-6f : p->tan_fovy);
  a.raw = params;
  a.means3d = params; a.sh = params + 6 * n; a.vm = viewmatrix; a.pm = projmatrix;
  a.cam_pos = cam_pos; a.cov3d_fwd = cov3d_fwd;
  a.drgb = dL_drgb; a.dxys = dL_dxys; a.dconic = dL_dconic_opacity; a.dvs_out = dL_dviewspace;
  a.radii = radii; a.clamped = clamped;
  a.g_means = grad_flat;
  a.g_dc = grad_flat + 3 * n;
  a.g_rest = grad_flat + 6 * n;
  a.g_logit = grad_flat + 51 * n;
  a.g_logscale = grad_flat + 52 * n;
  a.g_rot = grad_flat + 55 * n;
  a.st_acc = stats;
  a.st_acc_abs = stats + n;
  a.st_denom = stats + 2 * n;
  a.st_max_radii = stats + 3 * n;
  a.accumulate = accumulate;
  const size_t smem = (size_t)kPreThreads * p->max_sh_coeffs * 3 * sizeof(float);
  static unsigned long long attr_done = 0;
  if (smem > 48 * 1024) smem_attr_once(preprocess_bwd_kernel<true, false>, (int)smem, &attr_done);
  const int blocks = (int)((n + kPreThreads - 1) / kPreThreads);
  preprocess_bwd_kernel<true, false><<<blocks, kPreThreads, smem, (cudaStream_t)stream>>>(a);
  return check_launch("preprocess_backward_train");
}

int fgs_preprocess_backward_push(const fgs_preprocess_params* p, const float* params,
                                 const float* viewmatrix, const float* projmatrix,
                                 const float* cam_pos, const float* cov3d_fwd,
                                 const float* dL_drgb, const float* dL_dxys,
                                 const float* dL_dconic_opacity, const float* dL_dviewspace,
                                 const int32_t* radii, const uint8_t* clamped, int32_t world,
                                 int64_t shard, float* const* grad_ranks, float* stats,
                                 void* stream) {
  int st = validate_pre(p);
  if (st) return st;
  if (p->n == 0) return FGS_OK;
  FGS_CHECK_ARG(!p->use_cov3d_precomp && !p->use_colors_precomp,
                "training mode needs the scales+quats and dc+sh paths");
  FGS_CHECK_ARG(p->max_sh_coeffs == 15, "training mode stores 15 SH rest coefficients");
  FGS_CHECK_ARG(world >= 1 && world <= 8, "world must be in [1, 8]");
  FGS_CHECK_ARG(shard > 0 && shard % 4 == 0 && shard * world >= 59 * (int64_t)p->n,
                "shard must be a positive multiple of 4 with world * shard >= 59 n");
  FGS_CHECK_ARG(params && viewmatrix && projmatrix && cam_pos && cov3d_fwd && dL_drgb && dL_dxys &&
                    dL_dconic_opacity && dL_dviewspace && radii && clamped && grad_ranks && stats,
                "missing pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(dL_dconic_opacity, 16) && FGS_ALIGNED(dL_dviewspace, 16),
                "conic and viewspace gradients must be 16-byte aligned");
  const int64_t n = p->n;
  PbwdArgs a;
  memset(&a, 0, sizeof(a));
  for (int r = 0; r < world; ++r) {
    FGS_CHECK_ARG(grad_ranks[r] && FGS_ALIGNED(grad_ranks[r], 16),
                  "gradient buffer of rank %d missing or not 16-byte aligned", r);
    a.peer_g[r] = grad_ranks[r];
  }
  a.p = *p;
  a.focal_x = 0.5f * (float)p->image_width / (p->tan_fovx < 1e-6f ? 1e-6f : p->tan_fovx);
  a.focal_y = 0.5f * (float)p->image_height / (p->tan_fovy < 1e-6f ? 1e-6f : p->tan_fovy);
  a.raw = params;
  a.means3d = params; a.sh = params + 6 * n; a.vm = viewmatrix; a.pm = projmatrix;
  a.cam_pos = cam_pos; a.cov3d_fwd = cov3d_fwd;
  a.drgb = dL_drgb; a.dxys = dL_dxys; a.dconic = dL_dconic_opacity; a.dvs_out = dL_dviewspace;
  a.radii = radii; a.clamped = clamped;
  a.st_acc = stats;
  a.st_acc_abs = stats + n;
  a.st_denom = stats + 2 * n;
  a.st_max_radii = stats + 3 * n;
  a.shard = shard;
  const size_t smem = (size_t)kPreThreads * (p->max_sh_coeffs * 3 + kAdamStaged) * sizeof(float);
  static unsigned long long attr_done = 0;
  if (smem > 48 * 1024) smem_attr_once(preprocess_bwd_kernel<true, true, true>, (int)smem, &attr_done);
  const int blocks = (int)((n + kPreThreads - 1) / kPreThreads);
  preprocess_bwd_kernel<true, true, true><<<blocks, kPreThreads, smem, (cudaStream_t)stream>>>(a);
  return check_launch("preprocess_backward_push");
}

int fgs_preprocess_backward_adam(const fgs_preprocess_params* p, const float* viewmatrix,
                                 const float* projmatrix, const float* cam_pos,
                                 const float* cov3d_fwd, const float* dL_drgb, const float* dL_dxys,
                                 const float* dL_dconic_opacity, const float* dL_dviewspace,
                                 const int32_t* radii, const uint8_t* clamped, float* params,
                                 float* exp_avg, float* exp_avg_sq, const float* group_lr,
                                 float beta1, float beta2, float eps, int32_t step,
                                 int32_t bias_correction, float* stats, void* stream) {
  int st = validate_pre(p);
  if (st) return st;
  if (p->n == 0) return FGS_OK;
  FGS_CHECK_ARG(!p->use_cov3d_precomp && !p->use_colors_precomp,
                "training mode needs the scales+quats and dc+sh paths");
  FGS_CHECK_ARG(p->max_sh_coeffs == 15, "training mode stores 15 SH rest coefficients");
  FGS_CHECK_ARG(viewmatrix && projmatrix && cam_pos && cov3d_fwd && dL_drgb && dL_dxys &&
                    dL_dconic_opacity && dL_dviewspace && radii && clamped && params && exp_avg &&
                    exp_avg_sq && group_lr && stats,
                "missing pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(dL_dconic_opacity, 16) && FGS_ALIGNED(dL_dviewspace, 16),
                "conic and viewspace gradients must be 16-byte aligned");
  FGS_CHECK_ARG(!bias_correction || step >= 1, "step must be >= 1 with bias correction");
  const int64_t n = p->n;
  PbwdArgs a;
  memset(&a, 0, sizeof(a));
  a.p = *p;
  a.focal_x = 0.5f * (float)p->image_width / (p->tan_fovx < 1e-6f ? 1e-6f : p->tan_fovx);
  a.focal_y = 0.5f * (float)p->image_height / (p->tan_fovy < 1e-6f ? 1e-6f : p->tan_fovy);
  // the raw parameters are read from the buffer that this launch updates: each
  // Gaussian's values are read before its own update, and the sh rows are
  // staged in shared memory first
  a.raw = params;
  a.means3d = params; a.sh = params + 6 * n; a.vm = viewmatrix; a.pm = projmatrix;
  a.cam_pos = cam_pos; a.cov3d_fwd = cov3d_fwd;
  a.drgb = dL_drgb; a.dxys = dL_dxys; a.dconic = dL_dconic_opacity; a.dvs_out = dL_dviewspace;
  a.radii = radii; a.clamped = clamped;
  a.st_acc = stats;
  a.st_acc_abs = stats + n;
  a.st_denom = stats + 2 * n;
  a.st_max_radii = stats + 3 * n;
  a.ap = params;
  a.am = exp_avg;
  a.av = exp_avg_sq;
  for (int k = 0; k < 6; ++k) a.lr[k] = group_lr[k];
  a.b1 = beta1;
  a.b2 = beta2;
  a.eps = eps;
  a.bc1 = bias_correction ? 1.0f / (1.0f - powf(beta1, (float)step)) : 1.0f;
  a.bc2 = bias_correction ? 1.0f / (1.0f - powf(beta2, (float)step)) : 1.0f;
  const size_t smem = (size_t)kPreThreads * (p->max_sh_coeffs * 3 + kAdamStaged) * sizeof(float);
  static unsigned long long attr_done = 0;
  if (smem > 48 * 1024) smem_attr_once(preprocess_bwd_kernel<true, true>, (int)smem, &attr_done);
  const int blocks = (int)((n + kPreThreads - 1) / kPreThreads);
  preprocess_bwd_kernel<true, true><<<blocks, kPreThreads, smem, (cudaStream_t)stream>>>(a);
  return check_launch("preprocess_backward_adam");
}

}  // extern "C"
