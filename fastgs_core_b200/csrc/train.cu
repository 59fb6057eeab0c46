// Training-step kernels around the rasterizer (sm_100a): parameter
// activations, the L1 + D-SSIM photometric loss and its gradient, the Adam
// update over the flat parameter buffer, and the FastGS multi-view score
// accumulation (metric map, contribution counts, importance / pruning
// scores).
//
// Flat parameter / gradient layout (59 floats per Gaussian, N Gaussians):
//   [0, 3N) means3d | [3N, 6N) features_dc | [6N, 51N) features_rest (15x3)
//   [51N, 52N) opacity logits | [52N, 55N) log scales | [55N, 59N) rotations
// This is the buffer the data-parallel step all-reduces.
#include <cstdio>
#include <cstring>

#include "../../include/fastgs_b200.h"
#include "fgs_common.cuh"

namespace fgs {

// ------------------------------------------------------------ activations
__global__ void activate_kernel(int64_t n, const float* __restrict__ flat, float* __restrict__ opac,
                                float* __restrict__ scales, float* __restrict__ quats) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float lg = flat[51 * n + i];
  opac[i] = 1.0f / (1.0f + expf(-lg));
#pragma unroll
  for (int c = 0; c < 3; ++c) scales[3 * i + c] = expf(flat[52 * n + 3 * i + c]);
  // scalar loads: the rotation segment starts at 55 n floats, 16-byte aligned
  // only when n is a multiple of 4
  const float* qp = flat + 55 * n + 4 * i;
  const float4 q = make_float4(qp[0], qp[1], qp[2], qp[3]);
  // explicitly rounded (this file may contract multiply-adds): the same bits
  // as the preprocess kernels' in-kernel activation
  const float ss = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(q.x, q.x), __fmul_rn(q.y, q.y)),
                                       __fmul_rn(q.z, q.z)),
                             __fmul_rn(q.w, q.w));
  const float inv = 1.0f / (sqrtf(ss) + 1e-8f);
  reinterpret_cast<float4*>(quats)[i] = make_float4(q.x * inv, q.y * inv, q.z * inv, q.w * inv);
}

// --------------------------------------------------------------- L1 + SSIM
// 11x11 Gaussian window, sigma 1.5 (separable), zero padding, C1 = 0.01^2,
// C2 = 0.03^2; loss = w_l1 * mean|x - y| + w_ssim * (1 - mean SSIM(x, y)) over
// the 3 x H x W image (x = render, y = target, both CHW).
constexpr int kR = 5;
__constant__ float c_win[11];

// Fused L1 + D-SSIM forward and backward: one CTA per 32x32 output tile and
// channel. The CTA loads its 52x52 input window once, forms the five local
// moments by separable 11-tap convolution, evaluates SSIM and its partial
// derivatives (dS/dmu_x, dS/dE[x^2], dS/dE[xy]) on the 42x42 region the
// backward convolution needs (recomputing the 5-pixel halo instead of writing
// and re-reading global maps), convolves them back and writes dL/dimage.
constexpr int kFO = 32;               // output tile
constexpr int kFM = kFO + 2 * kR;     // 42: derivative-map region
constexpr int kFI = kFM + 2 * kR;     // 52: input region
// shared memory: region A holds the input window, then (aliased) the
// derivative maps; region B the horizontal moments, then the second pass
constexpr int kRegionA = 2 * kFI * (kFI + 1);
constexpr int kRegionB = 5 * kFI * kFM;
static_assert(3 * kFM * (kFM + 1) <= kRegionA, "maps must fit the input region");
static_assert(3 * kFM * kFO <= kRegionB, "second pass must fit the moment region");
constexpr int kFusedSmemFloats = kRegionA + kRegionB;

// The image and target of a pixel are packed as one float2 (x, y): the
// moments (mu_x, mu_y) and (E[x^2], E[y^2]) and the derivative pair
// (dS/dmu_x, dS/dE[x^2]) are convolved as f32x2 pairs, E[xy] and dS/dE[xy] as
// single floats, so three of every five (two of every three) window
// multiply-adds issue as one instruction (config 3: 0.192 ms; 0.2025 ms with
// five scalar maps).
__device__ __forceinline__ float2 f2b(float a) { return make_float2(a, a); }

__global__ void __launch_bounds__(256)
    ssim_pair_kernel(int W, int H, const float* __restrict__ x, const float* __restrict__ y,
                     float w_l1_n, float w_ssim_n, float* __restrict__ dx,
                     float* __restrict__ partials) {
  extern __shared__ float sm[];
  float2* sxy = reinterpret_cast<float2*>(sm);                   // [kFI][kFI+1]  (region A)
  float2* smu = reinterpret_cast<float2*>(sm + kRegionA);       // [kFI][kFM]    (region B)
  float2* se2 = smu + kFI * kFM;                                 // [kFI][kFM]
  float* sexy = reinterpret_cast<float*>(se2 + kFI * kFM);       // [kFI][kFM]
  float2* mpp = reinterpret_cast<float2*>(sm);                   // [kFM][kFM+1] over region A
  float* mps = reinterpret_cast<float*>(mpp + kFM * (kFM + 1));  // [kFM][kFM+1]
  float2* h2p = reinterpret_cast<float2*>(sm + kRegionA);       // [kFM][kFO] over region B
  float* h2s = reinterpret_cast<float*>(h2p + kFM * kFO);        // [kFM][kFO]
  static_assert(3 * kFM * (kFM + 1) <= kRegionA, "derivative maps must fit region A");
  static_assert(3 * kFM * kFO <= kRegionB, "second pass must fit region B");
  __shared__ float s_red[2][8];
  const int x0 = blockIdx.x * kFO, y0 = blockIdx.y * kFO, c = blockIdx.z;
  const size_t P = (size_t)W * H;
  const float* xc = x + c * P;
  const float* yc = y + c * P;
  const int t = threadIdx.x;
  for (int k = t; k < kFI * kFI; k += 256) {
    const int r = k / kFI, q = k % kFI;
    const int gy = y0 - 2 * kR + r, gx = x0 - 2 * kR + q;
    const bool in = gx >= 0 && gx < W && gy >= 0 && gy < H;
    const size_t o = (size_t)gy * W + gx;
    sxy[r * (kFI + 1) + q] = in ? make_float2(xc[o], yc[o]) : make_float2(0.0f, 0.0f);
  }
  __syncthreads();
  // horizontal moments: 52 rows x 14 segments of 3 outputs
  constexpr int kSeg = 3;
  constexpr int kHSeg = kFM / kSeg;
  for (int k = t; k < kFI * kHSeg; k += 256) {
    const int r = k / kHSeg, q0 = (k % kHSeg) * kSeg;
    float2 v[kSeg + 10], e[kSeg + 10];
    float cxy[kSeg + 10];
#pragma unroll
    for (int i = 0; i < kSeg + 10; ++i) {
      v[i] = sxy[r * (kFI + 1) + q0 + i];
      e[i] = __fmul2_rn(v[i], v[i]);
      cxy[i] = v[i].x * v[i].y;
    }
#pragma unroll
    for (int o = 0; o < kSeg; ++o) {
      float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
      float a4 = 0.f;
#pragma unroll
      for (int j = 0; j < 11; ++j) {
        const float w = c_win[j];
        a01 = __ffma2_rn(f2b(w), v[o + j], a01);
        a23 = __ffma2_rn(f2b(w), e[o + j], a23);
        a4 = fmaf(w, cxy[o + j], a4);
      }
      smu[r * kFM + q0 + o] = a01;
      se2[r * kFM + q0 + o] = a23;
      sexy[r * kFM + q0 + o] = a4;
    }
  }
  __syncthreads();
  // vertical moments, SSIM and its derivatives on the 42x42 map region: 42
  // columns x 6 segments of 7 rows
  float ssum = 0.f, lsum = 0.f;
  constexpr int kVSeg = 7;
  constexpr int kV1Items = kFM * (kFM / kVSeg);
  static_assert(kV1Items <= 256, "one vertical item per thread");
  float2 dmp[kVSeg];
  float dms[kVSeg];
  const bool v1 = t < kV1Items;
  const int vq = t % kFM, vr0 = (t / kFM) * kVSeg;
  if (v1) {
    float2 m01[kVSeg], m23[kVSeg];
    float m4[kVSeg];
    {
      float2 col[kVSeg + 10];
#pragma unroll
      for (int i = 0; i < kVSeg + 10; ++i) col[i] = smu[(vr0 + i) * kFM + vq];
#pragma unroll
      for (int o = 0; o < kVSeg; ++o) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 11; ++j) acc = __ffma2_rn(f2b(c_win[j]), col[o + j], acc);
        m01[o] = acc;
      }
    }
    {
      float2 col[kVSeg + 10];
#pragma unroll
      for (int i = 0; i < kVSeg + 10; ++i) col[i] = se2[(vr0 + i) * kFM + vq];
#pragma unroll
      for (int o = 0; o < kVSeg; ++o) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 11; ++j) acc = __ffma2_rn(f2b(c_win[j]), col[o + j], acc);
        m23[o] = acc;
      }
    }
    {
      float col[kVSeg + 10];
#pragma unroll
      for (int i = 0; i < kVSeg + 10; ++i) col[i] = sexy[(vr0 + i) * kFM + vq];
#pragma unroll
      for (int o = 0; o < kVSeg; ++o) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 11; ++j) acc = fmaf(c_win[j], col[o + j], acc);
        m4[o] = acc;
      }
    }
#pragma unroll
    for (int o = 0; o < kVSeg; ++o) {
      const int r = vr0 + o;
      const int gy = y0 - kR + r, gx = x0 - kR + vq;
      float d_mu = 0.f, d_exx = 0.f, d_exy = 0.f;
      if (gx >= 0 && gx < W && gy >= 0 && gy < H) {
        const float mu_x = m01[o].x, mu_y = m01[o].y, exx = m23[o].x, eyy = m23[o].y, exy = m4[o];
        const float C1 = 0.0001f, C2 = 0.0009f;
        const float A = 2.f * mu_x * mu_y + C1;
        const float B = 2.f * (exy - mu_x * mu_y) + C2;
        const float Cc = mu_x * mu_x + mu_y * mu_y + C1;
        const float D = (exx - mu_x * mu_x) + (eyy - mu_y * mu_y) + C2;
        const float inv = 1.0f / (Cc * D);
        const float ssim = A * B * inv;
        d_mu = 2.f * mu_y * (B - A) * inv - 2.f * mu_x * ssim * (1.f / Cc - 1.f / D);
        d_exx = -ssim / D;
        d_exy = 2.f * A * inv;
        if (r >= kR && r < kR + kFO && vq >= kR && vq < kR + kFO) ssum += ssim;  // own pixels
      }
      dmp[o] = make_float2(d_mu, d_exx);
      dms[o] = d_exy;
    }
  }
  __syncthreads();  // the input window is dead from here on
  if (v1) {
#pragma unroll
    for (int o = 0; o < kVSeg; ++o) {
      mpp[(vr0 + o) * (kFM + 1) + vq] = dmp[o];
      mps[(vr0 + o) * (kFM + 1) + vq] = dms[o];
    }
  }
  __syncthreads();
  // horizontal convolution of the derivative maps: 42 rows x 4 segments of 8
  constexpr int kSeg2 = 8;
  for (int k = t; k < kFM * (kFO / kSeg2); k += 256) {
    const int r = k / (kFO / kSeg2), q0 = (k % (kFO / kSeg2)) * kSeg2;
    float2 rp[kSeg2 + 10];
    float rs[kSeg2 + 10];
#pragma unroll
    for (int i = 0; i < kSeg2 + 10; ++i) {
      rp[i] = mpp[r * (kFM + 1) + q0 + i];
      rs[i] = mps[r * (kFM + 1) + q0 + i];
    }
#pragma unroll
    for (int o = 0; o < kSeg2; ++o) {
      float2 ap = make_float2(0.f, 0.f);
      float as = 0.f;
#pragma unroll
      for (int j = 0; j < 11; ++j) {
        ap = __ffma2_rn(f2b(c_win[j]), rp[o + j], ap);
        as = fmaf(c_win[j], rs[o + j], as);
      }
      h2p[r * kFO + q0 + o] = ap;
      h2s[r * kFO + q0 + o] = as;
    }
  }
  __syncthreads();
  // vertical convolution and the image gradient: 32 columns x 8 segments of 4 rows
  constexpr int kSeg3 = 4;
  static_assert(kFO * (kFO / kSeg3) == 256, "one final item per thread");
  {
    const int q = t % kFO, r0 = (t / kFO) * kSeg3;
    float2 cp[kSeg3 + 10];
    float cs[kSeg3 + 10];
#pragma unroll
    for (int i = 0; i < kSeg3 + 10; ++i) {
      cp[i] = h2p[(r0 + i) * kFO + q];
      cs[i] = h2s[(r0 + i) * kFO + q];
    }
#pragma unroll
    for (int o = 0; o < kSeg3; ++o) {
      float2 gp = make_float2(0.f, 0.f);
      float gs = 0.f;
#pragma unroll
      for (int j = 0; j < 11; ++j) {
        gp = __ffma2_rn(f2b(c_win[j]), cp[o + j], gp);
        gs = fmaf(c_win[j], cs[o + j], gs);
      }
      const int r = r0 + o;
      const int gy = y0 + r, gx = x0 + q;
      if (gx >= W || gy >= H) continue;
      const size_t pix = c * P + (size_t)gy * W + gx;
      const float xv = x[pix], yv = y[pix];
      lsum += fabsf(xv - yv);
      const float sgn = xv > yv ? 1.f : (xv < yv ? -1.f : 0.f);
      dx[pix] = w_l1_n * sgn - w_ssim_n * (gp.x + 2.f * xv * gp.y + yv * gs);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
  }
  if ((t & 31) == 0) {
    s_red[0][t >> 5] = ssum;
    s_red[1][t >> 5] = lsum;
  }
  __syncthreads();
  if (t == 0) {
    float sa = 0.f, sb = 0.f;
    for (int k = 0; k < 8; ++k) {
      sa += s_red[0][k];
      sb += s_red[1][k];
    }
    const size_t blk = ((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    partials[2 * blk] = sa;
    partials[2 * blk + 1] = sb;
  }
}

__global__ void loss_finalize_kernel(const float* __restrict__ partials, int nblk, float w_l1,
                                     float w_ssim, float inv_n, float* __restrict__ out) {
  __shared__ float s[2][32];
  float a = 0.f, b = 0.f;
  for (int k = threadIdx.x; k < nblk; k += blockDim.x) {
    a += partials[2 * k];
    b += partials[2 * k + 1];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s[0][threadIdx.x >> 5] = a;
    s[1][threadIdx.x >> 5] = b;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sa = 0.f, sb = 0.f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) {
      sa += s[0][k];
      sb += s[1][k];
    }
    const float ssim = sa * inv_n, l1 = sb * inv_n;
    out[0] = w_l1 * l1 + w_ssim * (1.0f - ssim);
    out[1] = l1;
    out[2] = ssim;
  }
}

// Mean squared error and its gradient (the reference trainer's warm-up loss):
// one strided pass, a per-block partial of sum (x - y)^2 in partials[2 blk + 1]
// (partials[2 blk] = 0: the SSIM slot loss_finalize_kernel also reads).
__global__ void __launch_bounds__(256)
    mse_kernel(int64_t n, const float* __restrict__ x, const float* __restrict__ y, float g_scale,
               float* __restrict__ dimg, float* __restrict__ partials) {
  __shared__ float s_w[8];
  float acc = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float d = x[i] - y[i];
    acc = fmaf(d, d, acc);
    dimg[i] = g_scale * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int k = 0; k < 8; ++k) t += s_w[k];
    partials[2 * blockIdx.x] = 0.0f;
    partials[2 * blockIdx.x + 1] = t;
  }
}

// -------------------------------------------------------------------- Adam
struct AdamGroups {
  int64_t end[8];
  float lr[8];
  int count;
};

// learning rate of the group holding flat element idx (the last group past
// every end); a fully unrolled search, so the table stays in registers
__device__ __forceinline__ float adam_lr(const AdamGroups& grp, int64_t idx) {
  float lr = 0.0f;
  bool found = false;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const bool hit = !found && q < grp.count && (idx < grp.end[q] || q == grp.count - 1);
    lr = hit ? grp.lr[q] : lr;
    found = found || hit;
  }
  return lr;
}

__device__ __forceinline__ void adam_update4(float4& pp, const float4 gg, float4& mm, float4& vv,
                                             const AdamGroups& grp, int64_t i, float b1, float b2,
                                             float eps, float bc1, float bc2) {
  float* pa = &pp.x;
  const float* ga = &gg.x;
  float* ma = &mm.x;
  float* va = &vv.x;
  // one group lookup for the four elements unless a group boundary falls inside
  const float lr0 = adam_lr(grp, i);
  const bool same = adam_lr(grp, i + 3) == lr0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float lr = same ? lr0 : adam_lr(grp, i + k);
    adam_elem(pa[k], ma[k], va[k], ga[k], lr, b1, b2, eps, bc1, bc2);
  }
}

// Two float4 per thread per iteration (eight independent 16-byte loads in
// flight), grid-stride over a grid sized to the SMs; every stream is read
// once and written once, so loads and stores are marked streaming.
__global__ void __launch_bounds__(256) adam_kernel(int64_t total, float* __restrict__ p,
                                                   const float* __restrict__ g, float* __restrict__ m,
                                                   float* __restrict__ v, AdamGroups grp, float b1,
                                                   float b2, float eps, float bc1, float bc2) {
  const int64_t n4 = total / 4;
  float4* p4 = reinterpret_cast<float4*>(p);
  const float4* g4 = reinterpret_cast<const float4*>(g);
  float4* m4 = reinterpret_cast<float4*>(m);
  float4* v4 = reinterpret_cast<float4*>(v);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; j + stride < n4; j += 2 * stride) {
    const int64_t j2 = j + stride;
    float4 pa = __ldcs(p4 + j), pb = __ldcs(p4 + j2);
    const float4 ga = __ldcs(g4 + j), gb = __ldcs(g4 + j2);
    float4 ma = __ldcs(m4 + j), mb = __ldcs(m4 + j2);
    float4 va = __ldcs(v4 + j), vb = __ldcs(v4 + j2);
    adam_update4(pa, ga, ma, va, grp, 4 * j, b1, b2, eps, bc1, bc2);
    adam_update4(pb, gb, mb, vb, grp, 4 * j2, b1, b2, eps, bc1, bc2);
    __stcs(p4 + j, pa);
    __stcs(p4 + j2, pb);
    __stcs(m4 + j, ma);
    __stcs(m4 + j2, mb);
    __stcs(v4 + j, va);
    __stcs(v4 + j2, vb);
  }
  if (j < n4) {
    float4 pa = __ldcs(p4 + j);
    const float4 ga = __ldcs(g4 + j);
    float4 ma = __ldcs(m4 + j), va = __ldcs(v4 + j);
    adam_update4(pa, ga, ma, va, grp, 4 * j, b1, b2, eps, bc1, bc2);
    __stcs(p4 + j, pa);
    __stcs(m4 + j, ma);
    __stcs(v4 + j, va);
  }
  // tail elements past the last full float4
  if (blockIdx.x == 0 && threadIdx.x < (unsigned)(total - 4 * n4)) {
    const int64_t idx = 4 * n4 + threadIdx.x;
    const float lr = adam_lr(grp, idx);
    float pv = p[idx], mv = m[idx], vv = v[idx];
    adam_elem(pv, mv, vv, g[idx], lr, b1, b2, eps, bc1, bc2);
    p[idx] = pv;
    m[idx] = mv;
    v[idx] = vv;
  }
}

// ------------------------------------------- Adam fused with the exchange
// Data-parallel update of one rank's parameter shard over NVLink multicast
// (NVLS): the summed gradient of the shard is read with multimem.ld_reduce
// (the NVSwitch adds every rank's copy), Adam runs on it, and the updated
// parameters are written to every rank's copy with one multimem.st. This
// replaces reduce-scatter + Adam + all-gather: the gradient reads use each
// GPU's NVLink egress and the parameter broadcast its ingress, so the two
// halves of the exchange overlap instead of running back to back.
__device__ __forceinline__ float4 mc_ld_reduce_add(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void mc_store(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ void adam4(float4& pp, float4& mm, float4& vv, const float4 gg,
                                      int64_t idx0, const AdamGroups& grp, float b1, float b2,
                                      float eps, float bc1, float bc2) {
  float* pa = &pp.x;
  const float* ga = &gg.x;
  float* ma = &mm.x;
  float* va = &vv.x;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t idx = idx0 + k;
    adam_elem(pa[k], ma[k], va[k], ga[k], adam_lr(grp, idx), b1, b2, eps, bc1, bc2);
  }
}

// ---------------------------------------- Adam fused with a unicast exchange
// Data-parallel update over plain peer loads and stores: the owner of a shard
// sums every rank's gradient for it (ranks in order; its own from local
// memory, the others' over NVLink), applies Adam to its shard and stores the
// new parameters into every rank's copy. Per GPU this moves (world - 1) /
// world of the buffer in each direction twice (gradients in, parameters
// out), which at two ranks is less than the multicast kernel's traffic.
constexpr int kMaxPeers = 8;
struct PeerPtrs {
  float* p[kMaxPeers];
  const float* g[kMaxPeers];
};
constexpr int kPeerUnroll = 2;

__global__ void __launch_bounds__(256)
    adam_peers_kernel(int64_t n4, int world, int rank, int nstore, PeerPtrs pp, float* __restrict__ m,
                      float* __restrict__ v, AdamGroups grp, float b1, float b2, float eps,
                      float bc1, float bc2) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t base = t; base < n4; base += stride * kPeerUnroll) {
    float4 gg[kPeerUnroll];
#pragma unroll
    for (int u = 0; u < kPeerUnroll; ++u) {
      const int64_t i4 = base + u * stride;
      if (i4 >= n4) continue;
      // peers' memory is read past L1 (it changes every step)
      float4 a = __ldcg(reinterpret_cast<const float4*>(pp.g[0]) + i4);
      for (int r = 1; r < world; ++r) {
        const float4 b = __ldcg(reinterpret_cast<const float4*>(pp.g[r]) + i4);
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
      }
      gg[u] = a;
    }
#pragma unroll
    for (int u = 0; u < kPeerUnroll; ++u) {
      const int64_t i4 = base + u * stride;
      if (i4 >= n4) break;
      float4 p4 = reinterpret_cast<const float4*>(pp.p[rank])[i4];
      float4 mm = reinterpret_cast<float4*>(m)[i4];
      float4 vv = reinterpret_cast<float4*>(v)[i4];
      adam4(p4, mm, vv, gg[u], 4 * i4, grp, b1, b2, eps, bc1, bc2);
      reinterpret_cast<float4*>(m)[i4] = mm;
      reinterpret_cast<float4*>(v)[i4] = vv;
      for (int r = 0; r < nstore; ++r) reinterpret_cast<float4*>(pp.p[r])[i4] = p4;
    }
  }
  // make the stores to the peers visible system-wide before the caller's barrier
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// ------------------------------------------- Adam of a pushed gradient shard
// The ranks have already added their gradients into the owner's buffer
// (fgs_preprocess_backward_push): the owner reads its summed shard, clears it
// for the next step, applies Adam and stores the new parameters into every
// rank's copy (peer stores, or one multimem.st when params_mc is given).
__global__ void __launch_bounds__(256)
    adam_owner_kernel(int64_t n4, int world, int rank, PeerPtrs pp, float* p_mc,
                      float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                      AdamGroups grp, float b1, float b2, float eps, float bc1, float bc2) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float4* g4 = reinterpret_cast<float4*>(g);
  for (int64_t base = t; base < n4; base += stride * kPeerUnroll) {
    float4 gg[kPeerUnroll], p4[kPeerUnroll], mm[kPeerUnroll], vv[kPeerUnroll];
#pragma unroll
    for (int u = 0; u < kPeerUnroll; ++u) {
      const int64_t i4 = base + u * stride;
      if (i4 >= n4) continue;
      gg[u] = __ldcg(g4 + i4);
      p4[u] = reinterpret_cast<const float4*>(pp.p[rank])[i4];
      mm[u] = reinterpret_cast<float4*>(m)[i4];
      vv[u] = reinterpret_cast<float4*>(v)[i4];
    }
#pragma unroll
    for (int u = 0; u < kPeerUnroll; ++u) {
      const int64_t i4 = base + u * stride;
      if (i4 >= n4) break;
      g4[i4] = make_float4(0.f, 0.f, 0.f, 0.f);
      adam4(p4[u], mm[u], vv[u], gg[u], 4 * i4, grp, b1, b2, eps, bc1, bc2);
      reinterpret_cast<float4*>(m)[i4] = mm[u];
      reinterpret_cast<float4*>(v)[i4] = vv[u];
      if (p_mc) {
        mc_store(p_mc + 4 * i4, p4[u]);
      } else {
        for (int r = 0; r < world; ++r) reinterpret_cast<float4*>(pp.p[r])[i4] = p4[u];
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

constexpr int kMcUnroll = 4;  // independent multicast loads in flight per thread

__global__ void __launch_bounds__(256)
    adam_nvls_kernel(int64_t total4, const float* __restrict__ p_local, float* p_mc,
                     const float* g_mc, float* __restrict__ m, float* __restrict__ v,
                     AdamGroups grp, float b1, float b2, float eps, float bc1, float bc2) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t base = t; base < total4; base += stride * kMcUnroll) {
    float4 gg[kMcUnroll];
#pragma unroll
    for (int u = 0; u < kMcUnroll; ++u) {
      const int64_t i4 = base + u * stride;
      if (i4 < total4) gg[u] = mc_ld_reduce_add(g_mc + 4 * i4);
    }
#pragma unroll
    for (int u = 0; u < kMcUnroll; ++u) {
      const int64_t i4 = base + u * stride;
      if (i4 >= total4) break;
      float4 pp = reinterpret_cast<const float4*>(p_local)[i4];
      float4 mm = reinterpret_cast<float4*>(m)[i4];
      float4 vv = reinterpret_cast<float4*>(v)[i4];
      adam4(pp, mm, vv, gg[u], 4 * i4, grp, b1, b2, eps, bc1, bc2);
      reinterpret_cast<float4*>(m)[i4] = mm;
      reinterpret_cast<float4*>(v)[i4] = vv;
      mc_store(p_mc + 4 * i4, pp);
    }
  }
  // make the broadcast visible system-wide before the caller's barrier
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// ------------------------------------------------------------ FastGS scores
// scripts/train_scanner_fastgs.py:262-340
__global__ void l1_map_kernel(int64_t P, const float* __restrict__ pred,
                              const float* __restrict__ tgt, float* __restrict__ l1map,
                              unsigned int* __restrict__ minmax, float* __restrict__ l1sum) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float s = 0.f;
  if (i < P) {
    const float a = fabsf(pred[i] - tgt[i]);
    const float b = fabsf(pred[P + i] - tgt[P + i]);
    const float c = fabsf(pred[2 * P + i] - tgt[2 * P + i]);
    s = a + b + c;
    const float mval = s / 3.0f;
    l1map[i] = mval;
    // non-negative floats order like their bit patterns
    atomicMin(minmax, __float_as_uint(mval));
    atomicMax(minmax + 1, __float_as_uint(mval));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(l1sum, s);
}

__global__ void metric_map_kernel(int64_t P, const float* __restrict__ l1map,
                                  const unsigned int* __restrict__ minmax, float thresh,
                                  int32_t* __restrict__ metric_map) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  const float mn = __uint_as_float(minmax[0]), mx = __uint_as_float(minmax[1]);
  const float denom = fmaxf(mx - mn, 1.0e-6f);
  metric_map[i] = ((l1map[i] - mn) / denom) > thresh ? 1 : 0;
}

__global__ void score_accumulate_kernel(int64_t n, const int32_t* __restrict__ counts,
                                        const float* __restrict__ l1sum, float inv_elems,
                                        float* __restrict__ counts_acc, float* __restrict__ score_acc) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float c = (float)counts[i];
  const float photometric = l1sum[0] * inv_elems;
  counts_acc[i] += c;
  score_acc[i] += photometric * c;
}

__global__ void minmax_kernel(int64_t n, const float* __restrict__ x, unsigned int* __restrict__ mm) {
  // order-preserving map of any float to unsigned
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t b = __float_as_uint(x[i]);
  const uint32_t k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  atomicMin(mm, k);
  atomicMax(mm + 1, k);
}

__device__ __forceinline__ float unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__global__ void score_finalize_kernel(int64_t n, const float* __restrict__ counts_acc,
                                      const float* __restrict__ score_acc,
                                      const unsigned int* __restrict__ mm, float inv_views,
                                      float* __restrict__ importance, float* __restrict__ pruning) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float mn = unkey(mm[0]), mx = unkey(mm[1]);
  if (importance) importance[i] = floorf(counts_acc[i] * inv_views);
  pruning[i] = (score_acc[i] - mn) / fmaxf(mx - mn, 1.0e-6f);
}

__global__ void init_pair_kernel(unsigned int* p, unsigned int a, unsigned int b) {
  p[0] = a;
  p[1] = b;
}

// grid budget of the exchange kernels (resident CTAs per SM; 0: their defaults)
static int g_exchange_bps = 0;
static bool g_win_ready[64] = {false};  // per device: c_win lives in each device's constant bank
static int ensure_window() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && g_win_ready[dev]) return FGS_OK;
  float w[11];
  double s = 0.0, e[11];
  for (int i = 0; i < 11; ++i) {
    e[i] = exp(-((i - 5) * (i - 5)) / (2.0 * 1.5 * 1.5));
    s += e[i];
  }
  for (int i = 0; i < 11; ++i) w[i] = (float)(e[i] / s);
  cudaError_t err = cudaMemcpyToSymbol(c_win, w, sizeof(w));
  if (err != cudaSuccess) {
    set_error("ssim window upload: %s", cudaGetErrorString(err));
    return FGS_ERR_CUDA;
  }
  if (dev >= 0 && dev < 64) g_win_ready[dev] = true;
  return FGS_OK;
}

}  // namespace fgs

using namespace fgs;

extern "C" {

int fgs_activate_params(int64_t n, const float* params_flat, float* opacities, float* scales,
                        float* quats, void* stream) {
  FGS_CHECK_ARG(n >= 0, "n must be >= 0");
  if (n == 0) return FGS_OK;
  FGS_CHECK_ARG(params_flat && opacities && scales && quats, "missing pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(quats, 16), "rotations output must be 16-byte aligned");
  activate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      n, params_flat, opacities, scales, quats);
  return check_launch("activate_params");
}

size_t fgs_loss_scratch_bytes(int32_t width, int32_t height) {
  const size_t blocks = (size_t)((width + kFO - 1) / kFO) * ((height + kFO - 1) / kFO) * 3;
  return (2 * blocks + 64) * sizeof(float);
}

int fgs_mse_loss(int32_t width, int32_t height, const float* image, const float* target, float w_mse,
                 float* loss_out, float* dL_dimage, void* scratch, void* stream) {
  FGS_CHECK_ARG(width > 0 && height > 0, "image size must be positive");
  FGS_CHECK_ARG(image && target && loss_out && dL_dimage && scratch, "missing pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t n = 3 * (int64_t)width * height;
  // as many blocks as the fused L1 + D-SSIM pass (the scratch is sized for those)
  const int64_t tiles = (int64_t)((width + kFO - 1) / kFO) * ((height + kFO - 1) / kFO) * 3;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int nblk = (int)(tiles < (int64_t)sms * 8 ? tiles : (int64_t)sms * 8);
  const float inv_n = 1.0f / (float)n;
  mse_kernel<<<nblk, 256, 0, s>>>(n, image, target, 2.0f * w_mse * inv_n, dL_dimage, (float*)scratch);
  // out[0] = w_mse * mse, out[1] = mse, out[2] = 0
  loss_finalize_kernel<<<1, 1024, 0, s>>>((const float*)scratch, nblk, w_mse, 0.0f, inv_n, loss_out);
  return check_launch("mse_loss");
}

int fgs_l1_dssim_loss(int32_t width, int32_t height, const float* image, const float* target,
                      float w_l1, float w_ssim, float* loss_out, float* dL_dimage, void* scratch,
                      void* stream) {
  FGS_CHECK_ARG(width > 0 && height > 0, "image size must be positive");
  FGS_CHECK_ARG(image && target && loss_out && dL_dimage && scratch, "missing pointer");
  int st = ensure_window();
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t P = (size_t)width * height;
  float* partials = (float*)scratch;
  dim3 grid((width + kFO - 1) / kFO, (height + kFO - 1) / kFO, 3);
  const int nblk = (int)(grid.x * grid.y * grid.z);
  const float inv_n = 1.0f / (float)(3 * P);
  const int smem = kFusedSmemFloats * (int)sizeof(float);
  static unsigned long long attr_done = 0;
  smem_attr_once(ssim_pair_kernel, smem, &attr_done);
  ssim_pair_kernel<<<grid, 256, smem, s>>>(width, height, image, target, w_l1 * inv_n,
                                           w_ssim * inv_n, dL_dimage, partials);
  loss_finalize_kernel<<<1, 1024, 0, s>>>(partials, nblk, w_l1, w_ssim, inv_n, loss_out);
  return check_launch("l1_dssim_loss");
}

int fgs_adam_step(int64_t total, float* params, const float* grads, float* exp_avg,
                  float* exp_avg_sq, int32_t num_groups, const int64_t* group_end,
                  const float* group_lr, float beta1, float beta2, float eps, int32_t step,
                  int32_t bias_correction, void* stream) {
  FGS_CHECK_ARG(total >= 0, "total must be >= 0");
  FGS_CHECK_ARG(num_groups >= 1 && num_groups <= 8, "num_groups must be in [1, 8]");
  FGS_CHECK_ARG(group_end && group_lr, "missing group table");
  if (total == 0) return FGS_OK;
  FGS_CHECK_ARG(params && grads && exp_avg && exp_avg_sq, "missing pointer");
  FGS_CHECK_ARG(((uintptr_t)params | (uintptr_t)grads | (uintptr_t)exp_avg | (uintptr_t)exp_avg_sq) % 16 == 0,
                "Adam buffers must be 16-byte aligned");
  AdamGroups g;
  memset(&g, 0, sizeof(g));
  g.count = num_groups;
  for (int k = 0; k < num_groups; ++k) {
    g.end[k] = group_end[k];
    g.lr[k] = group_lr[k];
  }
  float bc1 = 1.f, bc2 = 1.f;
  if (bias_correction) {
    FGS_CHECK_ARG(step >= 1, "step must be >= 1 with bias correction");
    bc1 = 1.0f / (1.0f - powf(beta1, (float)step));
    bc2 = 1.0f / (1.0f - powf(beta2, (float)step));
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n4 = (total + 3) / 4;
  const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, (int64_t)sms * 8);
  adam_kernel<<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, (cudaStream_t)stream>>>(
      total, params, grads, exp_avg, exp_avg_sq, g, beta1, beta2, eps, bc1, bc2);
  return check_launch("adam_step");
}

int fgs_set_exchange_grid(int32_t blocks_per_sm) {
  FGS_CHECK_ARG(blocks_per_sm >= 0 && blocks_per_sm <= 8, "blocks_per_sm must be in [0, 8]");
  g_exchange_bps = blocks_per_sm;
  return FGS_OK;
}

int fgs_adam_step_peers(int64_t shard, int32_t world, int32_t rank, float* const* params_ranks,
                        const float* const* grads_ranks, float* exp_avg, float* exp_avg_sq,
                        int32_t num_groups, const int64_t* group_end, const float* group_lr,
                        float beta1, float beta2, float eps, int32_t step, int32_t bias_correction,
                        void* stream) {
  FGS_CHECK_ARG(shard >= 0 && shard % 4 == 0, "shard length must be a multiple of 4");
  FGS_CHECK_ARG(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world,
                "world must be in [1, %d] and rank in [0, world)", kMaxPeers);
  FGS_CHECK_ARG(num_groups >= 1 && num_groups <= 8, "num_groups must be in [1, 8]");
  FGS_CHECK_ARG(group_end && group_lr && params_ranks && grads_ranks, "missing pointer table");
  if (shard == 0) return FGS_OK;
  FGS_CHECK_ARG(exp_avg && exp_avg_sq, "missing pointer");
  PeerPtrs pp;
  memset(&pp, 0, sizeof(pp));
  uintptr_t align = (uintptr_t)exp_avg | (uintptr_t)exp_avg_sq;
  for (int r = 0; r < world; ++r) {
    FGS_CHECK_ARG(params_ranks[r] && grads_ranks[r], "missing pointer for rank %d", r);
    pp.p[r] = params_ranks[r];
    pp.g[r] = grads_ranks[r];
    align |= (uintptr_t)params_ranks[r] | (uintptr_t)grads_ranks[r];
  }
  FGS_CHECK_ARG(align % 16 == 0, "buffers must be 16-byte aligned");
  AdamGroups g;
  memset(&g, 0, sizeof(g));
  g.count = num_groups;
  for (int k = 0; k < num_groups; ++k) {
    g.end[k] = group_end[k];
    g.lr[k] = group_lr[k];
  }
  float bc1 = 1.f, bc2 = 1.f;
  if (bias_correction) {
    FGS_CHECK_ARG(step >= 1, "step must be >= 1 with bias correction");
    bc1 = 1.0f / (1.0f - powf(beta1, (float)step));
    bc2 = 1.0f / (1.0f - powf(beta2, (float)step));
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n4 = shard / 4;
  const int64_t want = (n4 + 255) / 256;
  const int64_t cap = (int64_t)sms * (g_exchange_bps > 0 ? g_exchange_bps : 8);
  const int blocks = (int)(want < cap ? want : cap);
  adam_peers_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(n4, world, rank, world, pp, exp_avg,
                                                              exp_avg_sq, g, beta1, beta2, eps,
                                                              bc1, bc2);
  return check_launch("adam_step_peers");
}

int fgs_adam_step_gathered(int64_t shard, int32_t world, const float* const* grads,
                           float* params, float* exp_avg, float* exp_avg_sq, int32_t num_groups,
                           const int64_t* group_end, const float* group_lr, float beta1,
                           float beta2, float eps, int32_t step, int32_t bias_correction,
                           void* stream) {
  FGS_CHECK_ARG(shard >= 0 && shard % 4 == 0, "shard length must be a multiple of 4");
  FGS_CHECK_ARG(world >= 1 && world <= kMaxPeers, "world must be in [1, %d]", kMaxPeers);
  FGS_CHECK_ARG(num_groups >= 1 && num_groups <= 8, "num_groups must be in [1, 8]");
  FGS_CHECK_ARG(group_end && group_lr && grads, "missing pointer table");
  if (shard == 0) return FGS_OK;
  FGS_CHECK_ARG(params && exp_avg && exp_avg_sq, "missing pointer");
  PeerPtrs pp;
  memset(&pp, 0, sizeof(pp));
  uintptr_t align = (uintptr_t)params | (uintptr_t)exp_avg | (uintptr_t)exp_avg_sq;
  for (int r = 0; r < world; ++r) {
    FGS_CHECK_ARG(grads[r], "missing gradient pointer %d", r);
    pp.g[r] = grads[r];
    align |= (uintptr_t)grads[r];
  }
  pp.p[0] = params;
  FGS_CHECK_ARG(align % 16 == 0, "buffers must be 16-byte aligned");
  AdamGroups g;
  memset(&g, 0, sizeof(g));
  g.count = num_groups;
  for (int k = 0; k < num_groups; ++k) {
    g.end[k] = group_end[k];
    g.lr[k] = group_lr[k];
  }
  float bc1 = 1.f, bc2 = 1.f;
  if (bias_correction) {
    FGS_CHECK_ARG(step >= 1, "step must be >= 1 with bias correction");
    bc1 = 1.0f / (1.0f - powf(beta1, (float)step));
    bc2 = 1.0f / (1.0f - powf(beta2, (float)step));
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n4 = shard / 4;
  const int64_t want = (n4 + 255) / 256;
  const int64_t cap = (int64_t)sms * (g_exchange_bps > 0 ? g_exchange_bps : 8);
  const int blocks = (int)(want < cap ? want : cap);
  adam_peers_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(n4, world, 0, 1, pp, exp_avg,
                                                              exp_avg_sq, g, beta1, beta2, eps,
                                                              bc1, bc2);
  return check_launch("adam_step_gathered");
}

int fgs_adam_step_owner(int64_t shard, int32_t world, int32_t rank, float* const* params_ranks,
                        float* params_mc, float* grads, float* exp_avg, float* exp_avg_sq,
                        int32_t num_groups, const int64_t* group_end, const float* group_lr,
                        float beta1, float beta2, float eps, int32_t step, int32_t bias_correction,
                        void* stream) {
  FGS_CHECK_ARG(shard >= 0 && shard % 4 == 0, "shard length must be a multiple of 4");
  FGS_CHECK_ARG(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world,
                "world must be in [1, %d] and rank in [0, world)", kMaxPeers);
  FGS_CHECK_ARG(num_groups >= 1 && num_groups <= 8, "num_groups must be in [1, 8]");
  FGS_CHECK_ARG(group_end && group_lr && params_ranks, "missing pointer table");
  if (shard == 0) return FGS_OK;
  FGS_CHECK_ARG(grads && exp_avg && exp_avg_sq, "missing pointer");
  PeerPtrs pp;
  memset(&pp, 0, sizeof(pp));
  uintptr_t align = (uintptr_t)grads | (uintptr_t)exp_avg | (uintptr_t)exp_avg_sq | (uintptr_t)params_mc;
  for (int r = 0; r < world; ++r) {
    FGS_CHECK_ARG(params_ranks[r], "missing parameter pointer for rank %d", r);
    pp.p[r] = params_ranks[r];
    align |= (uintptr_t)params_ranks[r];
  }
  FGS_CHECK_ARG(align % 16 == 0, "buffers must be 16-byte aligned");
  AdamGroups g;
  memset(&g, 0, sizeof(g));
  g.count = num_groups;
  for (int k = 0; k < num_groups; ++k) {
    g.end[k] = group_end[k];
    g.lr[k] = group_lr[k];
  }
  float bc1 = 1.f, bc2 = 1.f;
  if (bias_correction) {
    FGS_CHECK_ARG(step >= 1, "step must be >= 1 with bias correction");
    bc1 = 1.0f / (1.0f - powf(beta1, (float)step));
    bc2 = 1.0f / (1.0f - powf(beta2, (float)step));
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n4 = shard / 4;
  const int64_t want = (n4 + 255) / 256;
  const int64_t cap = (int64_t)sms * (g_exchange_bps > 0 ? g_exchange_bps : 8);
  const int blocks = (int)(want < cap ? want : cap);
  adam_owner_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(n4, world, rank, pp, params_mc, grads,
                                                              exp_avg, exp_avg_sq, g, beta1, beta2,
                                                              eps, bc1, bc2);
  return check_launch("adam_step_owner");
}

int fgs_adam_step_multicast(int64_t shard, const float* params_local, float* params_mc,
                            const float* grads_mc, float* exp_avg, float* exp_avg_sq,
                            int32_t num_groups, const int64_t* group_end, const float* group_lr,
                            float beta1, float beta2, float eps, int32_t step,
                            int32_t bias_correction, void* stream) {
  FGS_CHECK_ARG(shard >= 0 && shard % 4 == 0, "shard length must be a multiple of 4");
  FGS_CHECK_ARG(num_groups >= 1 && num_groups <= 8, "num_groups must be in [1, 8]");
  FGS_CHECK_ARG(group_end && group_lr, "missing group table");
  if (shard == 0) return FGS_OK;
  FGS_CHECK_ARG(params_local && params_mc && grads_mc && exp_avg && exp_avg_sq, "missing pointer");
  FGS_CHECK_ARG(((uintptr_t)params_local | (uintptr_t)params_mc | (uintptr_t)grads_mc |
                 (uintptr_t)exp_avg | (uintptr_t)exp_avg_sq) % 16 == 0,
                "buffers must be 16-byte aligned");
  AdamGroups g;
  memset(&g, 0, sizeof(g));
  g.count = num_groups;
  for (int k = 0; k < num_groups; ++k) {
    g.end[k] = group_end[k];
    g.lr[k] = group_lr[k];
  }
  float bc1 = 1.f, bc2 = 1.f;
  if (bias_correction) {
    FGS_CHECK_ARG(step >= 1, "step must be >= 1 with bias correction");
    bc1 = 1.0f / (1.0f - powf(beta1, (float)step));
    bc2 = 1.0f / (1.0f - powf(beta2, (float)step));
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t n4 = shard / 4;
  const int64_t want = (n4 + 255) / 256;
  const int64_t cap = (int64_t)sms * (g_exchange_bps > 0 ? g_exchange_bps : 4);
  const int blocks = (int)(want < cap ? want : cap);
  adam_nvls_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      n4, params_local, params_mc, grads_mc, exp_avg, exp_avg_sq, g, beta1, beta2, eps, bc1, bc2);
  return check_launch("adam_step_multicast");
}

int fgs_metric_map(int64_t num_pixels, const float* pred, const float* target, float loss_thresh,
                   int32_t* metric_map, float* l1_sum, void* scratch, void* stream) {
  FGS_CHECK_ARG(num_pixels > 0, "num_pixels must be > 0");
  FGS_CHECK_ARG(pred && target && metric_map && l1_sum && scratch, "missing pointer");
  cudaStream_t s = (cudaStream_t)stream;
  float* l1map = (float*)scratch;
  unsigned int* mm = (unsigned int*)(l1map + num_pixels);
  init_pair_kernel<<<1, 1, 0, s>>>(mm, 0x7f800000u, 0u);
  cudaMemsetAsync(l1_sum, 0, sizeof(float), s);
  const unsigned blocks = (unsigned)((num_pixels + 255) / 256);
  l1_map_kernel<<<blocks, 256, 0, s>>>(num_pixels, pred, target, l1map, mm, l1_sum);
  metric_map_kernel<<<blocks, 256, 0, s>>>(num_pixels, l1map, mm, loss_thresh, metric_map);
  return check_launch("metric_map");
}

int fgs_score_accumulate(int64_t n, const int32_t* metric_count, const float* l1_sum,
                         int64_t num_elements, float* counts_acc, float* score_acc, void* stream) {
  FGS_CHECK_ARG(n >= 0 && num_elements > 0, "bad sizes");
  if (n == 0) return FGS_OK;
  FGS_CHECK_ARG(metric_count && l1_sum && counts_acc && score_acc, "missing pointer");
  score_accumulate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      n, metric_count, l1_sum, 1.0f / (float)num_elements, counts_acc, score_acc);
  return check_launch("score_accumulate");
}

int fgs_score_finalize(int64_t n, const float* counts_acc, const float* score_acc, int32_t n_views,
                       float* importance, float* pruning, void* scratch, void* stream) {
  FGS_CHECK_ARG(n >= 0, "n must be >= 0");
  if (n == 0) return FGS_OK;
  FGS_CHECK_ARG(score_acc && pruning && scratch && (importance == nullptr || counts_acc),
                "missing pointer");
  cudaStream_t s = (cudaStream_t)stream;
  unsigned int* mm = (unsigned int*)scratch;
  init_pair_kernel<<<1, 1, 0, s>>>(mm, 0xffffffffu, 0u);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  minmax_kernel<<<blocks, 256, 0, s>>>(n, score_acc, mm);
  score_finalize_kernel<<<blocks, 256, 0, s>>>(n, counts_acc, score_acc, mm,
                                               1.0f / (float)(n_views > 0 ? n_views : 1),
                                               importance, pruning);
  return check_launch("score_finalize");
}

}  // extern "C"
