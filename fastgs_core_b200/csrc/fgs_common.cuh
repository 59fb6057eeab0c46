// Shared device-side definitions for the FastGS sm_100a kernels.
//
// Arithmetic contract (kept identical to the CPU checker so that integer
// outputs -- tiles touched, keys, ranges, n_contrib -- and the rendered image
// are bit-identical to it): every float operation is one IEEE binary32 op in
// the source order of the reference expression (the library is compiled with
// -fmad=false; fused ops appear only where written as fmaf), IEEE division and
// square root, min/max with the select semantics below, truncating saturating
// float->int conversion (NaN -> 0), and the exp/log defined here.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define FGS_BLOCK 16
#define FGS_TILE_PIXELS 256

namespace fgs {

// e^x: Cody-Waite reduction x = k ln2 + r (ln2 split 0x3f317200 + low part),
// degree-7 Taylor polynomial of e^r (coefficients 1/j!) in Horner form with
// fused multiply-adds, then 2^k applied as two exact power-of-two factors.
__device__ __forceinline__ float fgs_expf(float x) {
  if (!(x > -87.0f)) return (x != x) ? x : 0.0f;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  const float k = rintf(x * 1.44269502f);
  float r = fmaf(k, -0.693145752f, x);
  r = fmaf(k, -1.42860677e-06f, r);
  float p = 1.98412701e-04f;
  p = fmaf(p, r, 1.38888892e-03f);
  p = fmaf(p, r, 8.33333377e-03f);
  p = fmaf(p, r, 4.16666679e-02f);
  p = fmaf(p, r, 1.66666672e-01f);
  p = fmaf(p, r, 5.00000000e-01f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ki = __float2int_rz(k);
  const int k1 = ki / 2, k2 = ki - k1;
  const float s1 = __int_as_float((k1 + 127) << 23);
  const float s2 = __int_as_float((k2 + 127) << 23);
  return (p * s1) * s2;
}

// ln x: x = m 2^e, m in [sqrt(1/2), sqrt(2)); ln m = 2 atanh(s),
// s = (m-1)/(m+1), series through s^11; e ln2 added with ln2 split high/low.
__device__ __forceinline__ float fgs_logf(float x) {
  if (x != x || x < 0.0f) return __int_as_float(0x7fc00000);
  if (x == 0.0f) return __int_as_float(0xff800000);
  if (x == __int_as_float(0x7f800000)) return x;
  uint32_t u = __float_as_uint(x);
  int e = 0;
  if (u < 0x00800000u) {
    u = __float_as_uint(x * 16777216.0f);
    e = -24;
  }
  e += (int)((u >> 23) & 0xffu) - 127;
  float m = __uint_as_float((u & 0x007fffffu) | 0x3f800000u);
  if (m > 1.41421354f) {
    m = m * 0.5f;
    e += 1;
  }
  const float s = (m - 1.0f) / (m + 1.0f);
  const float s2 = s * s;
  float q = 9.09090936e-02f;
  q = fmaf(q, s2, 1.11111112e-01f);
  q = fmaf(q, s2, 1.42857149e-01f);
  q = fmaf(q, s2, 2.00000003e-01f);
  q = fmaf(q, s2, 3.33333343e-01f);
  const float ln_m = fmaf(2.0f * s * s2, q, 2.0f * s);
  const float fe = (float)e;
  return fmaf(fe, 0.693145752f, fmaf(fe, 1.42860677e-06f, ln_m));
}

// fgs_expf restricted to x in (-87, 0]: same operations and bits (2^k with
// k in [-126, 0] is applied in one exact multiply instead of two), no range
// checks. Callers guarantee the domain.
__device__ __forceinline__ float fgs_expf_neg(float x) {
  const float k = rintf(__fmul_rn(x, 1.44269502f));
  float r = fmaf(k, -0.693145752f, x);
  r = fmaf(k, -1.42860677e-06f, r);
  float p = 1.98412701e-04f;
  p = fmaf(p, r, 1.38888892e-03f);
  p = fmaf(p, r, 8.33333377e-03f);
  p = fmaf(p, r, 4.16666679e-02f);
  p = fmaf(p, r, 1.66666672e-01f);
  p = fmaf(p, r, 5.00000000e-01f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  return __fmul_rn(p, __int_as_float((__float2int_rz(k) + 127) << 23));
}

// Gaussian exponent of a splat at pixel offset (dx, dy), in the reference's
// operation order (fastgs_rasterize.metal:106-107), never contracted:
// -0.5 * (a dx^2 + c dy^2) - b dx dy
__device__ __forceinline__ float splat_power(float a, float b, float c, float dx, float dy) {
  const float q = __fadd_rn(__fmul_rn(__fmul_rn(a, dx), dx), __fmul_rn(__fmul_rn(c, dy), dy));
  return __fsub_rn(__fmul_rn(-0.5f, q), __fmul_rn(__fmul_rn(b, dx), dy));
}

// Lower bound on the exponent below which a splat of opacity o cannot reach
// alpha >= 1/255: for o <= 1, o * e^p < e^-5.55 = 0.003887 < 1/255. Skipping
// those pairs before the exponential gives the same decision as evaluating it.
// Otherwise -87 (the domain limit of fgs_expf_neg; fgs_expf is 0 below it).
__device__ __forceinline__ float power_cut(float o) { return o <= 1.0f ? -5.55f : -87.0f; }

// One Adam element update (torch.optim.Adam, no weight decay, bias corrections
// passed as reciprocals bc1 = 1 / (1 - beta1^t), bc2 = 1 / (1 - beta2^t)), with
// explicitly rounded operations so that every kernel that applies it (the
// plain, the multicast and the one fused into the preprocess backward pass)
// produces the same bits whatever its file's contraction setting.
__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, float g, float lr, float b1,
                                          float b2, float eps, float bc1, float bc2) {
  // a negative learning rate marks a parameter group that does not step this
  // iteration: its value and moments stay as they are
  if (lr < 0.0f) return;
  m = __fmaf_rn(b1, m, __fmul_rn(1.0f - b1, g));
  v = __fmaf_rn(b2, v, __fmul_rn(__fmul_rn(1.0f - b2, g), g));
  p = __fsub_rn(p, __fdiv_rn(__fmul_rn(lr, __fmul_rn(m, bc1)),
                             __fadd_rn(__fsqrt_rn(__fmul_rn(v, bc2)), eps)));
}

__device__ __forceinline__ float fmin_t(float a, float b) { return b < a ? b : a; }
__device__ __forceinline__ float fmax_t(float a, float b) { return a < b ? b : a; }
__device__ __forceinline__ int imin(int a, int b) { return b < a ? b : a; }
__device__ __forceinline__ int imax(int a, int b) { return a < b ? b : a; }
// truncating, saturating, NaN -> 0 (cvt.rzi.s32.f32)
__device__ __forceinline__ int f2i(float v) { return __float2int_rz(v); }

struct v3 {
  float x, y, z;
};
__device__ __forceinline__ v3 V3(float x, float y, float z) { return v3{x, y, z}; }
__device__ __forceinline__ float at(const v3& v, int i) { return i == 0 ? v.x : (i == 1 ? v.y : v.z); }
__device__ __forceinline__ float dot3(v3 a, v3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }

// column-major 3x3: c[col]
struct m3 {
  v3 c[3];
};
__device__ __forceinline__ m3 M3(float a0, float a1, float a2, float a3, float a4, float a5,
                                 float a6, float a7, float a8) {
  m3 m;
  m.c[0] = V3(a0, a1, a2);
  m.c[1] = V3(a3, a4, a5);
  m.c[2] = V3(a6, a7, a8);
  return m;
}
__device__ __forceinline__ v3 mulv(const m3& m, v3 v) {
  return V3(m.c[0].x * v.x + m.c[1].x * v.y + m.c[2].x * v.z,
            m.c[0].y * v.x + m.c[1].y * v.y + m.c[2].y * v.z,
            m.c[0].z * v.x + m.c[1].z * v.y + m.c[2].z * v.z);
}
__device__ __forceinline__ m3 mul(const m3& a, const m3& b) {
  m3 r;
  r.c[0] = mulv(a, b.c[0]);
  r.c[1] = mulv(a, b.c[1]);
  r.c[2] = mulv(a, b.c[2]);
  return r;
}
__device__ __forceinline__ m3 tr(const m3& a) {
  return M3(a.c[0].x, a.c[1].x, a.c[2].x, a.c[0].y, a.c[1].y, a.c[2].y, a.c[0].z, a.c[1].z,
            a.c[2].z);
}
__device__ __forceinline__ float mat(const m3& m, int col, int row) { return at(m.c[col], row); }

// point transform by a column-major 4x4 read from a row-major array
__device__ __forceinline__ v3 xform43(v3 p, const float* m) {
  return V3(m[0] * p.x + m[4] * p.y + m[8] * p.z + m[12],
            m[1] * p.x + m[5] * p.y + m[9] * p.z + m[13],
            m[2] * p.x + m[6] * p.y + m[10] * p.z + m[14]);
}

constexpr float kSH_C0 = 0.28209479177387814f;
constexpr float kSH_C1 = 0.4886025119029199f;

}  // namespace fgs

// ------------------------------------------------------------- host helpers
namespace fgs {
void set_error(const char* fmt, ...);
int check_launch(const char* what);

// Raise a kernel's dynamic shared-memory limit once per device (the
// attribute belongs to the function in each device's context).
template <typename Kernel>
inline void smem_attr_once(Kernel* k, int bytes, unsigned long long* done_mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(*done_mask & bit)) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    *done_mask |= bit;
  }
}
}  // namespace fgs

// pointers the kernels access as float2 / float4 / uint2 vectors
#define FGS_ALIGNED(p, bytes) ((((uintptr_t)(p)) & ((bytes)-1)) == 0)

#define FGS_CHECK_ARG(cond, ...)     \
  do {                               \
    if (!(cond)) {                   \
      fgs::set_error(__VA_ARGS__);   \
      return FGS_ERR_INVALID;        \
    }                                \
  } while (0)
