// FastGS densification on the device (scripts/train_scanner_fastgs.py:470-795):
// the per-Gaussian decision masks, the row gathers that prune, clone and
// split the flat training buffers, the split children's means and scales,
// and the opacity cap. The host makes the random draws (split offsets, the
// weighted prune budget) with the caller's generator, as the reference does.
//
// Flat training layout: segment k of width w_k holds rows [0, n) attribute-
// major at offset (w_0 + ... + w_{k-1}) * n; the parameters use widths
// {3, 3, 45, 1, 3, 4} (means, dc, sh rest, opacity logit, log-scale,
// rotation), the Adam moments the same, the densification statistics {1, 1,
// 1, 1} (acc, acc_abs, denom, max_radii).
#include <cstdint>
#include <cstring>

#include "../../include/fastgs_b200.h"
#include "fgs_common.cuh"

namespace fgs {

constexpr int kMaxSegments = 8;
struct Segments {
  int count;
  int width[kMaxSegments];
  int prefix[kMaxSegments];  // sum of the widths before segment k
  int row;                   // sum of all widths
};

// dst row j of every segment = src row index[j] (index < 0: zeros)
__global__ void gather_rows_kernel(int64_t n_in, int64_t n_out, const int64_t* __restrict__ index,
                                   Segments seg, const float* __restrict__ src,
                                   float* __restrict__ dst) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // element of the output
  if (e >= n_out * seg.row) return;
  // segment of element e: offsets prefix[k] * n_out .. (prefix[k] + width[k]) * n_out
  int k = 0;
#pragma unroll
  for (int q = 1; q < kMaxSegments; ++q)
    if (q < seg.count && e >= (int64_t)seg.prefix[q] * n_out) k = q;
  const int w = seg.width[k];
  const int64_t local = e - (int64_t)seg.prefix[k] * n_out;
  const int64_t row = local / w;
  const int c = (int)(local - row * w);
  const int64_t s = index[row];
  dst[e] = s >= 0 ? src[(int64_t)seg.prefix[k] * n_in + s * w + c] : 0.0f;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  const float m = a > b ? a : b;
  return m > c ? m : c;
}

// bit 0: clone, bit 1: split, bit 2: importance above the threshold
// (densify_and_prune_fastgs, scripts/train_scanner_fastgs.py:671-683)
__global__ void densify_masks_kernel(int64_t n, const float* __restrict__ params,
                                     const float* __restrict__ stats,
                                     const float* __restrict__ importance, float grad_thresh,
                                     float grad_abs_thresh, float dense_extent,
                                     float importance_thresh, uint8_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float denom = fmaxf(stats[2 * n + i], 1.0f);
  const float g = fabsf(stats[i] / denom);
  const float ga = fabsf(stats[n + i] / denom);
  const float* ls = params + 52 * n + 3 * i;
  const float max_scale = max3(expf(ls[0]), expf(ls[1]), expf(ls[2]));
  const bool metric = importance[i] > importance_thresh;
  const bool clone = metric && max_scale <= dense_extent && g >= grad_thresh;
  const bool split = metric && max_scale > dense_extent && ga >= grad_abs_thresh;
  out[i] = (uint8_t)((clone ? 1 : 0) | (split ? 2 : 0) | (metric ? 4 : 0));
}

// bit 0: opacity below min_opacity, bit 1: screen radius above max_screen
// (if > 0), bit 2: largest scale above max_world (if > 0)
// (densify_and_prune_fastgs, scripts/train_scanner_fastgs.py:703-714)
__global__ void prune_masks_kernel(int64_t n, const float* __restrict__ params,
                                   const float* __restrict__ max_radii, float min_opacity,
                                   float max_screen, float max_world, uint8_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float op = 1.0f / (1.0f + expf(-params[51 * n + i]));
  const float* ls = params + 52 * n + 3 * i;
  const bool a = op < min_opacity;
  const bool b = max_screen > 0.0f && max_radii[i] > max_screen;
  const bool c = max_world > 0.0f && max3(expf(ls[0]), expf(ls[1]), expf(ls[2])) > max_world;
  out[i] = (uint8_t)((a ? 1 : 0) | (b ? 2 : 0) | (c ? 4 : 0));
}

// split children rows [row0, row0 + m) already copy their sources: offset the
// mean by R(q) * sample and shrink the scale by 0.8 * split_factor
// (densify_and_split_fastgs, scripts/train_scanner_fastgs.py:582-593)
__global__ void split_fixup_kernel(int64_t n, int64_t row0, int64_t m, const float* __restrict__ samples,
                                   float split_factor, float* __restrict__ params) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= m) return;
  const int64_t i = row0 + t;
  const float* q = params + 55 * n + 4 * i;
  const float nrm = fmaxf(sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]), 1.0e-8f);
  const float w = q[0] / nrm, x = q[1] / nrm, y = q[2] / nrm, z = q[3] / nrm;
  const float s0 = samples[3 * t], s1 = samples[3 * t + 1], s2 = samples[3 * t + 2];
  float* mean = params + 3 * i;
  mean[0] += (1.0f - 2.0f * (y * y + z * z)) * s0 + 2.0f * (x * y - z * w) * s1 + 2.0f * (x * z + y * w) * s2;
  mean[1] += 2.0f * (x * y + z * w) * s0 + (1.0f - 2.0f * (x * x + z * z)) * s1 + 2.0f * (y * z - x * w) * s2;
  mean[2] += 2.0f * (x * z - y * w) * s0 + 2.0f * (y * z + x * w) * s1 + (1.0f - 2.0f * (x * x + y * y)) * s2;
  float* ls = params + 52 * n + 3 * i;
#pragma unroll
  for (int c = 0; c < 3; ++c) ls[c] = logf(expf(ls[c]) / (0.8f * split_factor));
}

// logit(min(sigmoid(l), cap)) with the reference's clip to [1e-6, 1 - 1e-6],
// and the opacity moments restarted at zero (cap_opacity_logits /
// reset_opacity_logits, scripts/train_scanner_fastgs.py:621-658, with
// replace_state_np :140-154)
__global__ void opacity_cap_kernel(int64_t n, float cap, float* __restrict__ params,
                                   float* __restrict__ m, float* __restrict__ v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float* l = params + 51 * n + i;
  const float op = 1.0f / (1.0f + expf(-*l));
  float p = op < cap ? op : cap;
  p = fminf(fmaxf(p, 1.0e-6f), 1.0f - 1.0e-6f);
  *l = logf(p / (1.0f - p));
  if (m) m[51 * n + i] = 0.0f;
  if (v) v[51 * n + i] = 0.0f;
}

static unsigned blocks_for(int64_t count) { return (unsigned)((count + 255) / 256); }

}  // namespace fgs

using namespace fgs;

extern "C" {

int fgs_gather_rows(int64_t n_in, int64_t n_out, const int64_t* index, int32_t num_segments,
                    const int32_t* widths, const float* src, float* dst, void* stream) {
  FGS_CHECK_ARG(n_in >= 0 && n_out >= 0, "sizes must be >= 0");
  FGS_CHECK_ARG(num_segments >= 1 && num_segments <= kMaxSegments, "1 to 8 segments");
  FGS_CHECK_ARG(widths, "missing widths");
  if (n_out == 0) return FGS_OK;
  FGS_CHECK_ARG(index && src && dst, "missing pointer");
  FGS_CHECK_ARG(src != dst, "gather cannot run in place");
  Segments seg;
  memset(&seg, 0, sizeof(seg));
  seg.count = num_segments;
  for (int k = 0; k < num_segments; ++k) {
    FGS_CHECK_ARG(widths[k] >= 1, "segment widths must be >= 1");
    seg.width[k] = widths[k];
    seg.prefix[k] = seg.row;
    seg.row += widths[k];
  }
  gather_rows_kernel<<<blocks_for(n_out * seg.row), 256, 0, (cudaStream_t)stream>>>(n_in, n_out, index, seg,
                                                                                  src, dst);
  return check_launch("gather_rows");
}

int fgs_densify_masks(int64_t n, const float* params, const float* stats, const float* importance,
                      float grad_thresh, float grad_abs_thresh, float dense_extent,
                      float importance_thresh, uint8_t* mask, void* stream) {
  FGS_CHECK_ARG(n >= 0, "n must be >= 0");
  if (n == 0) return FGS_OK;
  FGS_CHECK_ARG(params && stats && importance && mask, "missing pointer");
  densify_masks_kernel<<<blocks_for(n), 256, 0, (cudaStream_t)stream>>>(
      n, params, stats, importance, grad_thresh, grad_abs_thresh, dense_extent, importance_thresh, mask);
  return check_launch("densify_masks");
}

int fgs_prune_masks(int64_t n, const float* params, const float* max_radii, float min_opacity,
                    float max_screen, float max_world, uint8_t* mask, void* stream) {
  FGS_CHECK_ARG(n >= 0, "n must be >= 0");
  if (n == 0) return FGS_OK;
  FGS_CHECK_ARG(params && max_radii && mask, "missing pointer");
  prune_masks_kernel<<<blocks_for(n), 256, 0, (cudaStream_t)stream>>>(n, params, max_radii, min_opacity,
                                                                    max_screen, max_world, mask);
  return check_launch("prune_masks");
}

int fgs_split_fixup(int64_t n, int64_t row0, int64_t m, const float* samples, int32_t split_factor,
                    float* params, void* stream) {
  FGS_CHECK_ARG(n >= 0 && row0 >= 0 && m >= 0 && row0 + m <= n, "rows out of range");
  FGS_CHECK_ARG(split_factor >= 1, "split_factor must be >= 1");
  if (m == 0) return FGS_OK;
  FGS_CHECK_ARG(samples && params, "missing pointer");
  split_fixup_kernel<<<blocks_for(m), 256, 0, (cudaStream_t)stream>>>(n, row0, m, samples,
                                                                    (float)split_factor, params);
  return check_launch("split_fixup");
}

int fgs_opacity_cap(int64_t n, float cap, float* params, float* exp_avg, float* exp_avg_sq,
                    void* stream) {
  FGS_CHECK_ARG(n >= 0, "n must be >= 0");
  if (n == 0) return FGS_OK;
  FGS_CHECK_ARG(params, "missing pointer");
  opacity_cap_kernel<<<blocks_for(n), 256, 0, (cudaStream_t)stream>>>(n, cap, params, exp_avg, exp_avg_sq);
  return check_launch("opacity_cap");
}

}  // extern "C"
