// Binning on sm_100a: duplicate-with-keys, a stable LSD onesweep radix sort of
// the (tile | depth) keys, and tile ranges / bucket counts.
//
// Duplicate follows fastgs_core/metal/fastgs_binning.metal:182-213 (the tile
// walk itself is tile_walk.cuh). The sort replaces mx::argsort + mx::take
// (fastgs_core/binding/binding.cpp:195-197) with a hand-written onesweep LSD
// radix sort over 8-bit digits of the significant bits only: one histogram
// pass over the keys computes every digit histogram, then each digit pass
// reads and writes the pairs once (24 B per key per pass), ranking keys in a
// CTA with warp match/popc multi-split and resolving the CTA's global digit
// offsets by a decoupled look-back over earlier CTAs. Look-back waits are
// bounded: after kSpinLimit polls a CTA flags FGS_ERR_TIMEOUT, stops waiting
// and clamps its stores to the output. Tile ranges follow
// fastgs_core/metal/fastgs_tile_prep.metal:10-53.
#include <cstdio>
#include <mutex>

#include "../../include/fastgs_b200.h"
#include "fgs_common.cuh"
#include "tile_walk.cuh"

namespace fgs {

// ---------------------------------------------------------------- duplicate
constexpr int kDupThreads = 256;

// Thread j emits the keys of Gaussian i = order[j] (order == NULL: i = j) at
// the offsets of the inclusive scan `offsets` taken in that order.
__global__ void __launch_bounds__(kDupThreads)
    duplicate_kernel(int n, float mult, int gx, int gy, const float2* __restrict__ xys,
                     const float* __restrict__ depths, const uint32_t* __restrict__ order,
                     const uint32_t* __restrict__ offsets, const float4* __restrict__ conic,
                     const uint32_t* __restrict__ tiles, int64_t num_rendered,
                     uint64_t* __restrict__ keys, uint32_t* __restrict__ values) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const int i = order ? (int)order[j] : j;
  if ((unsigned)i >= (unsigned)n) return;
  const uint32_t cnt = tiles[i];
  if (cnt == 0u) return;
  const int64_t off0 = (j == 0) ? 0 : (int64_t)offsets[j - 1];
  const uint64_t dbits = (uint64_t)__float_as_uint(depths[i]);
  const float2 p = xys[i];
  int64_t off = off0;
  const int64_t end = off0 + cnt;
  tile_walk(p.x, p.y, conic[i], gx, gy, mult, [&](int tile) {
    if (off < end && off < num_rendered) {
      keys[off] = ((uint64_t)(int64_t)tile << 32) | dbits;
      values[off] = (uint32_t)i;
    }
    ++off;
  });
  // The reference's zero-filled outputs leave any slot the walk did not reach
  // at (key 0, value 0); write that explicitly.
  for (; off < end && off < num_rendered; ++off) {
    keys[off] = 0ull;
    values[off] = 0u;
  }
}

// The depth-first ordering of the training path: (depth bits, index) pairs of
// every Gaussian, then the per-position tile counts in the sorted order.
__global__ void depth_keys_kernel(int n, const float* __restrict__ depths,
                                  uint64_t* __restrict__ keys, uint32_t* __restrict__ vals) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  keys[i] = (uint64_t)__float_as_uint(depths[i]);
  vals[i] = (uint32_t)i;
}

__global__ void gather_u32_kernel(int n, const uint32_t* __restrict__ src,
                                  const uint32_t* __restrict__ index, uint32_t* __restrict__ dst) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const uint32_t i = index[j];
  dst[j] = i < (uint32_t)n ? src[i] : 0u;
}

// --------------------------------------------------------------------- sort
constexpr int kRadix = 256;
constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 15;
constexpr int kPart = kSortThreads * kSortItems;  // keys per partition (3840)
constexpr int kMaxPasses = 8;
constexpr uint32_t kFlagAgg = 1u << 30;
constexpr uint32_t kFlagPrefix = 2u << 30;
constexpr uint32_t kValueMask = (1u << 30) - 1u;
constexpr int kSpinLimit = 1 << 22;
constexpr int kLookWindow = 8;  // predecessors read per look-back round trip
constexpr int kSortDynSmem = kPart * (8 + 4);

__global__ void __launch_bounds__(256)
    sort_histogram_kernel(const uint64_t* __restrict__ keys, int64_t n, int bit0, int passes,
                          uint32_t* __restrict__ hist) {
  __shared__ uint32_t s_h[kMaxPasses][kRadix];
  for (int k = threadIdx.x; k < kMaxPasses * kRadix; k += blockDim.x) (&s_h[0][0])[k] = 0u;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint64_t k = keys[i];
    for (int p = 0; p < passes; ++p) atomicAdd(&s_h[p][(k >> (bit0 + 8 * p)) & 0xffu], 1u);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < passes * kRadix; k += blockDim.x) {
    const uint32_t v = (&s_h[0][0])[k];
    if (v) atomicAdd(hist + k, v);
  }
}

// exclusive scan of each pass's 256 digit counts (one CTA per pass)
__global__ void __launch_bounds__(kRadix) sort_hist_scan_kernel(uint32_t* hist) {
  __shared__ uint32_t s_w[kRadix / 32];
  uint32_t* h = hist + blockIdx.x * kRadix;
  const uint32_t v = h[threadIdx.x];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_w[w] = x;
  __syncthreads();
  uint32_t add = 0;
  for (int k = 0; k < w; ++k) add += s_w[k];
  h[threadIdx.x] = x - v + add;
}

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kSortThreads)
    onesweep_kernel(const uint64_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                    uint64_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, int64_t n,
                    int shift, const uint32_t* __restrict__ digit_offsets,
                    uint32_t* __restrict__ lookback, uint32_t* __restrict__ counter,
                    int* __restrict__ err, int spin_limit, int withhold_first,
                    const uint32_t* __restrict__ vals_orig, uint32_t* __restrict__ done) {
  __shared__ uint32_t s_part;
  __shared__ uint32_t s_whist[kSortWarps][kRadix];  // per-warp digit counts -> warp offsets
  __shared__ uint32_t s_local_start[kRadix];
  __shared__ uint32_t s_global_base[kRadix];
  __shared__ uint32_t s_wsum[kSortWarps];
  extern __shared__ __align__(16) unsigned char s_dyn[];
  uint64_t* s_keys = reinterpret_cast<uint64_t*>(s_dyn);       // [kPart]
  uint32_t* s_vals = reinterpret_cast<uint32_t*>(s_keys + kPart);  // [kPart]

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) s_part = atomicAdd(counter, 1u);
  for (int k = tid; k < kSortWarps * kRadix; k += kSortThreads) (&s_whist[0][0])[k] = 0u;
  __syncthreads();
  const uint32_t part = s_part;
  const int64_t base = (int64_t)part * kPart;
  const int valid = (int)((int64_t)kPart < n - base ? (int64_t)kPart : n - base);

  // warp-striped load: warp w owns [w*32*I, (w+1)*32*I), item i of lane l is +i*32+l
  uint64_t k[kSortItems];
  uint32_t v[kSortItems];
  uint32_t r[kSortItems];
#pragma unroll
  for (int i = 0; i < kSortItems; ++i) {
    const int li = w * 32 * kSortItems + i * 32 + lane;
    if (li < valid) {
      k[i] = keys_in[base + li];
      v[i] = vals_in[base + li];
    } else {
      k[i] = ~0ull;  // pads: digit 255, ranked after every real key of the partition
      v[i] = 0u;
    }
  }
  const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
  for (int i = 0; i < kSortItems; ++i) {
    const uint32_t d = (uint32_t)(k[i] >> shift) & 0xffu;
#ifdef FGS_SORT_MATCH_ANY
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
#else
    // the lanes holding the same digit: one ballot per digit bit
    uint32_t peers = 0xffffffffu;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t bal = __ballot_sync(0xffffffffu, (d >> b) & 1u);
      peers &= ((d >> b) & 1u) ? bal : ~bal;
    }
#endif
    const uint32_t before = s_whist[w][d];
    __syncwarp();
    if (lane == (__ffs(peers) - 1)) s_whist[w][d] = before + __popc(peers);
    __syncwarp();
    r[i] = before + __popc(peers & lt_mask);
  }
  __syncthreads();
  // thread d: warp offsets within the digit and the CTA's digit count
  const uint32_t d = tid;
  uint32_t cnt = 0;
#pragma unroll
  for (int ww = 0; ww < kSortWarps; ++ww) {
    const uint32_t c = s_whist[ww][d];
    s_whist[ww][d] = cnt;
    cnt += c;
  }
  const uint32_t pads = (uint32_t)(kPart - valid);
  const uint32_t real_cnt = (d == kRadix - 1) ? cnt - pads : cnt;
  // publish this partition's aggregate as early as possible
  uint32_t* lb = lookback + (size_t)part * kRadix + d;
  if (part == 0) {
    // (test hook) withhold_first: partition 0 publishes nothing, so its
    // successor's bounded wait runs out and reports FGS_ERR_TIMEOUT
    if (!withhold_first) st_volatile(lb, kFlagPrefix | real_cnt);
  } else {
    st_volatile(lb, kFlagAgg | real_cnt);
  }
  // CTA-local exclusive scan over digits (for the shared-memory sort)
  {
    uint32_t x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_wsum[w] = x;
    __syncthreads();
    uint32_t add = 0;
    for (int ww = 0; ww < w; ++ww) add += s_wsum[ww];
    s_local_start[d] = x - cnt + add;
  }
  // decoupled look-back over earlier partitions for digit d, reading a window
  // of kLookWindow predecessors per round trip: their values are summed from
  // the nearest one down until an inclusive prefix is met; a predecessor that
  // has published nothing yet ends the round, and the next window starts there
  uint32_t excl = 0;
  if (part > 0) {
    int64_t j = (int64_t)part - 1;
    int spins = 0;
    while (j >= 0) {
      uint32_t sv[kLookWindow];
#pragma unroll
      for (int u = 0; u < kLookWindow; ++u)
        sv[u] = (j - u >= 0) ? ld_volatile(lookback + (size_t)(j - u) * kRadix + d) : 0u;
      bool found = false;
      int used = 0;
#pragma unroll
      for (int u = 0; u < kLookWindow; ++u) {
        if (j - u < 0) break;
        const uint32_t flag = sv[u] & ~kValueMask;
        if (flag == 0u) break;
        excl += sv[u] & kValueMask;
        ++used;
        if (flag == kFlagPrefix) {
          found = true;
          break;
        }
      }
      if (found) break;
      j -= used;
      if (used < kLookWindow && j >= 0) {
        // the predecessor at j has published nothing yet: wait and re-read
        if (++spins > spin_limit) {
          atomicExch(err, 1);
          break;
        }
        __nanosleep(32);
      }
    }
    st_volatile(lb, kFlagPrefix | ((excl + real_cnt) & kValueMask));
  }
  s_global_base[d] = digit_offsets[d] + excl;
  __syncthreads();
  // scatter into shared memory in digit order (stable)
#pragma unroll
  for (int i = 0; i < kSortItems; ++i) {
    const uint32_t dd = (uint32_t)(k[i] >> shift) & 0xffu;
    const uint32_t pos = s_local_start[dd] + s_whist[w][dd] + r[i];
    s_keys[pos] = k[i];
    s_vals[pos] = v[i];
  }
  __syncthreads();
  for (int j = tid; j < valid; j += kSortThreads) {
    const uint64_t key = s_keys[j];
    const uint32_t dd = (uint32_t)(key >> shift) & 0xffu;
    const uint64_t dst = (uint64_t)s_global_base[dd] + (uint64_t)(j - (int)s_local_start[dd]);
    if (dst < (uint64_t)n) {
      keys_out[dst] = key;
      vals_out[dst] = s_vals[j];
    }
  }
  // Last pass only (done != NULL): the CTA that finishes last checks the
  // timeout flag of every pass. After a timeout the arrangement is undefined
  // (slots may be unwritten), so it replaces the output with a safe one: every
  // key all ones (an invalid tile id, which tile prep skips: nothing renders)
  // and the caller's values in input order (in range for any consumer that
  // indexes with them).
  if (done != nullptr) {
    __shared__ bool s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_last && ld_volatile(reinterpret_cast<const uint32_t*>(err)) != 0u) {
      __threadfence();
      for (int64_t i = tid; i < n; i += kSortThreads) {
        keys_out[i] = ~0ull;
        vals_out[i] = vals_orig[i];
      }
    }
  }
}

// ---------------------------------------------------------------- tile prep
__global__ void tile_ranges_kernel(const uint64_t* __restrict__ keys, int64_t n, int num_tiles,
                                   uint32_t* __restrict__ ranges) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n) return;
  const uint32_t cur = (uint32_t)(keys[g] >> 32);
  const bool valid = cur != 0xffffffffu;
  if (g == 0) {
    if (cur < (uint32_t)num_tiles) ranges[2 * (size_t)cur] = 0u;
  } else {
    const uint32_t prev = (uint32_t)(keys[g - 1] >> 32);
    if (cur != prev) {
      if (prev < (uint32_t)num_tiles) ranges[2 * (size_t)prev + 1] = (uint32_t)g;
      if (valid && cur < (uint32_t)num_tiles) ranges[2 * (size_t)cur] = (uint32_t)g;
    }
  }
  if (g == n - 1 && valid && cur < (uint32_t)num_tiles) ranges[2 * (size_t)cur + 1] = (uint32_t)n;
}

// one CTA: tiles in descending order of their splat count (counting sort on
// ceil(count / 16), 256 classes, the last class open-ended). Rendering the
// heaviest tiles first keeps a few long tiles from finishing alone at the end
// of a tile-per-CTA launch. The order within a class is unspecified; every
// tile's results are independent of it.
constexpr int kOrderClasses = 256;
__device__ __forceinline__ int tile_order_class(const uint32_t* ranges, int t) {
  const uint32_t ns = ranges[2 * t + 1] - ranges[2 * t];
  return (int)min((ns + 15u) / 16u, (uint32_t)(kOrderClasses - 1));
}

// The counting sort of tile_order_kernel by one whole CTA (all threads call it).
__device__ __forceinline__ void tile_order_cta(const uint32_t* __restrict__ ranges, int num_tiles,
                                               uint32_t* __restrict__ order) {
  __shared__ uint32_t s_hist[kOrderClasses];
  for (int c = threadIdx.x; c < kOrderClasses; c += blockDim.x) s_hist[c] = 0;
  __syncthreads();
  for (int t = threadIdx.x; t < num_tiles; t += blockDim.x) atomicAdd(&s_hist[tile_order_class(ranges, t)], 1u);
  __syncthreads();
  if (threadIdx.x < 32) {
    // exclusive scan from the heaviest class down: lane l owns classes
    // 255 - 8l ... 248 - 8l
    const int lane = threadIdx.x;
    uint32_t v[8], sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      v[k] = s_hist[kOrderClasses - 1 - (8 * lane + k)];
      sum += v[k];
    }
    uint32_t x = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    uint32_t run = x - sum;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      s_hist[kOrderClasses - 1 - (8 * lane + k)] = run;
      run += v[k];
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < num_tiles; t += blockDim.x)
    order[atomicAdd(&s_hist[tile_order_class(ranges, t)], 1u)] = (uint32_t)t;
}

__global__ void __launch_bounds__(1024)
    tile_order_kernel(const uint32_t* __restrict__ ranges, int num_tiles, uint32_t* __restrict__ order) {
  tile_order_cta(ranges, num_tiles, order);
}

// one CTA: bucket counts, their inclusive scan and the total
__global__ void __launch_bounds__(1024)
    bucket_count_kernel(const uint32_t* __restrict__ ranges, int num_tiles,
                        uint32_t* __restrict__ bucket_count, uint32_t* __restrict__ bucket_offsets,
                        uint64_t* __restrict__ bucket_sum, uint32_t* __restrict__ order,
                        uint32_t* __restrict__ bucket_to_tile, int64_t bucket_to_tile_len) {
  __shared__ uint32_t s_w[32];
  __shared__ uint32_t s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int base = 0; base < num_tiles; base += 1024) {
    const int t = base + threadIdx.x;
    uint32_t c = 0;
    if (t < num_tiles) {
      const int ns = (int)(ranges[2 * t + 1] - ranges[2 * t]);
      c = (uint32_t)((ns + 31) / 32);
      bucket_count[t] = c;
    }
    uint32_t x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_w[w] = x;
    __syncthreads();
    if (w == 0) {
      uint32_t s = s_w[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      s_w[lane] = s;
    }
    __syncthreads();
    if (t < num_tiles) bucket_offsets[t] = s_carry + x + (w > 0 ? s_w[w - 1] : 0u);
    __syncthreads();
    if (threadIdx.x == 0) s_carry += s_w[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) *bucket_sum = s_carry;
  // optional: the heaviest-first tile order, and bucket-to-tile entries past
  // the bucket total marked invalid (a caller that sizes the bucket arrays by
  // a bound instead of the total)
  if (order) tile_order_cta(ranges, num_tiles, order);
  if (bucket_to_tile)
    for (int64_t b = (int64_t)s_carry + threadIdx.x; b < bucket_to_tile_len; b += blockDim.x)
      bucket_to_tile[b] = 0xffffffffu;
}

static inline int sort_passes(int key_bits) { return (key_bits + 7) / 8; }

// Test hooks of the look-back wait (fgs_sort_set_test_hooks); the defaults
// are the production values.
static int g_spin_limit = kSpinLimit;
static int g_withhold_first = 0;
static inline int64_t sort_parts(int64_t n) { return (n + kPart - 1) / kPart; }

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace fgs

using namespace fgs;

extern "C" {

int fgs_duplicate_with_keys(int32_t n, float mult, int32_t tile_bounds_x, int32_t tile_bounds_y,
                            const float* xys, const float* depths, const uint32_t* point_offsets,
                            const float* conic_opacity, const uint32_t* tiles_touched,
                            int64_t num_rendered, uint64_t* keys_unsorted,
                            uint32_t* values_unsorted, void* stream) {
  FGS_CHECK_ARG(n >= 0 && num_rendered >= 0, "sizes must be >= 0");
  if (n == 0 || num_rendered == 0) return FGS_OK;
  FGS_CHECK_ARG(xys && depths && point_offsets && conic_opacity && tiles_touched && keys_unsorted &&
                    values_unsorted,
                "missing pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(xys, 8) && FGS_ALIGNED(conic_opacity, 16),
                "xys must be 8-byte, conic_opacity 16-byte aligned");
  FGS_CHECK_ARG(tile_bounds_x > 0 && tile_bounds_y > 0, "tile bounds must be positive");
  duplicate_kernel<<<(n + kDupThreads - 1) / kDupThreads, kDupThreads, 0, (cudaStream_t)stream>>>(
      n, mult, tile_bounds_x, tile_bounds_y, (const float2*)xys, depths, nullptr, point_offsets,
      (const float4*)conic_opacity, tiles_touched, num_rendered, keys_unsorted, values_unsorted);
  return check_launch("duplicate_with_keys");
}

int fgs_duplicate_with_keys_ordered(int32_t n, float mult, int32_t tile_bounds_x,
                                    int32_t tile_bounds_y, const float* xys, const float* depths,
                                    const uint32_t* order, const uint32_t* offsets_in_order,
                                    const float* conic_opacity, const uint32_t* tiles_touched,
                                    int64_t num_rendered, uint64_t* keys, uint32_t* values,
                                    void* stream) {
  FGS_CHECK_ARG(n >= 0 && num_rendered >= 0, "sizes must be >= 0");
  if (n == 0 || num_rendered == 0) return FGS_OK;
  FGS_CHECK_ARG(xys && depths && order && offsets_in_order && conic_opacity && tiles_touched &&
                    keys && values,
                "missing pointer");
  FGS_CHECK_ARG(FGS_ALIGNED(xys, 8) && FGS_ALIGNED(conic_opacity, 16),
                "xys must be 8-byte, conic_opacity 16-byte aligned");
  FGS_CHECK_ARG(tile_bounds_x > 0 && tile_bounds_y > 0, "tile bounds must be positive");
  duplicate_kernel<<<(n + kDupThreads - 1) / kDupThreads, kDupThreads, 0, (cudaStream_t)stream>>>(
      n, mult, tile_bounds_x, tile_bounds_y, (const float2*)xys, depths, order, offsets_in_order,
      (const float4*)conic_opacity, tiles_touched, num_rendered, keys, values);
  return check_launch("duplicate_with_keys_ordered");
}

size_t fgs_sort_workspace_bytes(int64_t num_rendered, int32_t key_bits) {
  const int passes = sort_passes(key_bits);
  const int64_t parts = sort_parts(num_rendered > 0 ? num_rendered : 1);
  size_t b = 0;
  b += align256(4);                                         // timeout flag (offset 0)
  b += align256((size_t)passes * kRadix * 4);               // hist
  b += align256((size_t)passes * parts * kRadix * 4);       // lookback
  b += align256((size_t)(passes + 1) * 4);                  // tickets, done counter
  b += align256((size_t)(num_rendered > 0 ? num_rendered : 1) * 8);  // tmp keys
  b += align256((size_t)(num_rendered > 0 ? num_rendered : 1) * 4);  // tmp vals
  return b;
}

int fgs_sort_pairs(int64_t num_rendered, int32_t key_bits, const uint64_t* keys_in,
                   const uint32_t* values_in, uint64_t* keys_out, uint32_t* values_out,
                   void* workspace, size_t workspace_bytes, void* stream) {
  return fgs_sort_pairs_bits(num_rendered, 0, key_bits, keys_in, values_in, keys_out, values_out,
                             workspace, workspace_bytes, stream);
}

int fgs_sort_pairs_bits(int64_t num_rendered, int32_t bit_begin, int32_t bit_end,
                        const uint64_t* keys_in, const uint32_t* values_in, uint64_t* keys_out,
                        uint32_t* values_out, void* workspace, size_t workspace_bytes,
                        void* stream) {
  FGS_CHECK_ARG(num_rendered >= 0, "num_rendered must be >= 0");
  FGS_CHECK_ARG(bit_begin >= 0 && bit_end > bit_begin && bit_end <= 64,
                "need 0 <= bit_begin < bit_end <= 64");
  const int32_t key_bits = bit_end - bit_begin;
  if (num_rendered == 0) return FGS_OK;
  if (num_rendered > (int64_t)kValueMask) {
    fgs::set_error("sort supports at most %u keys, got %lld", kValueMask, (long long)num_rendered);
    return FGS_ERR_CAPACITY;
  }
  const int passes = sort_passes(key_bits);
  FGS_CHECK_ARG(passes <= kMaxPasses, "too many key bits");
  FGS_CHECK_ARG(keys_in && values_in && keys_out && values_out && workspace, "missing pointer");
  const size_t need = fgs_sort_workspace_bytes(num_rendered, key_bits);
  FGS_CHECK_ARG(workspace_bytes >= need, "sort workspace too small: %zu < %zu", workspace_bytes, need);
  const int64_t parts = sort_parts(num_rendered);
  static unsigned long long attr_done = 0;
  smem_attr_once(onesweep_kernel, kSortDynSmem, &attr_done);
  char* w = (char*)workspace;
  int* err = (int*)w;  // offset 0: fgs_sort_status reads it
  w += align256(4);
  uint32_t* hist = (uint32_t*)w;
  w += align256((size_t)passes * kRadix * 4);
  uint32_t* lookback = (uint32_t*)w;
  w += align256((size_t)passes * parts * kRadix * 4);
  uint32_t* counters = (uint32_t*)w;  // [passes] tickets, then the last pass's done counter
  w += align256((size_t)(passes + 1) * 4);
  uint64_t* tmp_keys = (uint64_t*)w;
  w += align256((size_t)num_rendered * 8);
  uint32_t* tmp_vals = (uint32_t*)w;
  cudaStream_t s = (cudaStream_t)stream;
  // err .. counters are contiguous: clear them in one memset
  cudaMemsetAsync(err, 0, (size_t)((char*)tmp_keys - (char*)err), s);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t hb = (num_rendered + 4095) / 4096;
  const int hblocks = (int)(hb < (int64_t)sms * 4 ? hb : (int64_t)sms * 4);
  sort_histogram_kernel<<<hblocks > 0 ? hblocks : 1, 256, 0, s>>>(keys_in, num_rendered, bit_begin,
                                                                  passes, hist);
  sort_hist_scan_kernel<<<passes, kRadix, 0, s>>>(hist);
  const uint64_t* src_k = keys_in;
  const uint32_t* src_v = values_in;
  for (int p = 0; p < passes; ++p) {
    // the last pass lands in the output buffers
    const bool to_out = ((passes - 1 - p) % 2) == 0;
    uint64_t* dk = to_out ? keys_out : tmp_keys;
    uint32_t* dv = to_out ? values_out : tmp_vals;
    onesweep_kernel<<<(unsigned)parts, kSortThreads, kSortDynSmem, s>>>(
        src_k, src_v, dk, dv, num_rendered, bit_begin + 8 * p, hist + p * kRadix,
        lookback + (size_t)p * parts * kRadix, counters + p, err, g_spin_limit, g_withhold_first,
        values_in, p == passes - 1 ? counters + passes : nullptr);
    src_k = dk;
    src_v = dv;
  }
  return check_launch("sort_pairs");
}

size_t fgs_depth_order_workspace_bytes(int32_t n) {
  const int64_t m = n > 0 ? n : 1;
  return fgs_sort_workspace_bytes(m, 32) + align256((size_t)m * 8) * 2 + align256((size_t)m * 4);
}

int fgs_depth_order(int32_t n, const float* depths, const uint32_t* tiles_touched, uint32_t* order,
                    uint32_t* tiles_in_order, void* workspace, size_t workspace_bytes,
                    void* stream) {
  FGS_CHECK_ARG(n >= 0, "n must be >= 0");
  if (n == 0) return FGS_OK;
  FGS_CHECK_ARG(depths && tiles_touched && order && tiles_in_order && workspace, "missing pointer");
  FGS_CHECK_ARG(workspace_bytes >= fgs_depth_order_workspace_bytes(n), "depth order workspace too small");
  // the sort's workspace comes first, so that its timeout flag sits at
  // offset 0 of this workspace too (fgs_sort_status)
  const size_t sws = fgs_sort_workspace_bytes(n, 32);
  char* sort_ws = (char*)workspace;
  char* w = sort_ws + sws;
  uint64_t* keys = (uint64_t*)w;
  w += align256((size_t)n * 8);
  uint64_t* skeys = (uint64_t*)w;
  w += align256((size_t)n * 8);
  uint32_t* vals = (uint32_t*)w;
  cudaStream_t s = (cudaStream_t)stream;
  depth_keys_kernel<<<(n + 255) / 256, 256, 0, s>>>(n, depths, keys, vals);
  int st = fgs_sort_pairs_bits(n, 0, 32, keys, vals, skeys, order, sort_ws, sws, stream);
  if (st) return st;
  gather_u32_kernel<<<(n + 255) / 256, 256, 0, s>>>(n, tiles_touched, order, tiles_in_order);
  return check_launch("depth_order");
}

int fgs_tile_prep(int64_t num_rendered, int32_t num_tiles, const uint64_t* sorted_keys,
                  uint32_t* ranges, uint32_t* bucket_count, uint32_t* bucket_offsets,
                  uint64_t* bucket_sum, void* stream) {
  FGS_CHECK_ARG(num_rendered >= 0 && num_tiles >= 0, "sizes must be >= 0");
  cudaStream_t s = (cudaStream_t)stream;
  if (num_tiles == 0) {
    if (bucket_sum) cudaMemsetAsync(bucket_sum, 0, 8, s);
    return check_launch("tile_prep");
  }
  FGS_CHECK_ARG(ranges && bucket_count && bucket_offsets && bucket_sum, "missing pointer");
  FGS_CHECK_ARG(num_rendered == 0 || sorted_keys, "missing keys");
  cudaMemsetAsync(ranges, 0, (size_t)num_tiles * 2 * sizeof(uint32_t), s);
  if (num_rendered > 0)
    tile_ranges_kernel<<<(unsigned)((num_rendered + 255) / 256), 256, 0, s>>>(sorted_keys, num_rendered,
                                                                              num_tiles, ranges);
  bucket_count_kernel<<<1, 1024, 0, s>>>(ranges, num_tiles, bucket_count, bucket_offsets, bucket_sum,
                                         nullptr, nullptr, 0);
  return check_launch("tile_prep");
}

int fgs_tile_prep_ordered(int64_t num_rendered, int32_t num_tiles, const uint64_t* sorted_keys,
                          uint32_t* ranges, uint32_t* bucket_count, uint32_t* bucket_offsets,
                          uint64_t* bucket_sum, uint32_t* tile_order, uint32_t* bucket_to_tile,
                          int64_t bucket_to_tile_len, void* stream) {
  FGS_CHECK_ARG(num_rendered >= 0 && num_tiles > 0 && bucket_to_tile_len >= 0, "bad sizes");
  FGS_CHECK_ARG(ranges && bucket_count && bucket_offsets && bucket_sum && tile_order, "missing pointer");
  FGS_CHECK_ARG(num_rendered == 0 || sorted_keys, "missing keys");
  FGS_CHECK_ARG(bucket_to_tile_len == 0 || bucket_to_tile, "missing bucket_to_tile");
  cudaStream_t s = (cudaStream_t)stream;
  cudaMemsetAsync(ranges, 0, (size_t)num_tiles * 2 * sizeof(uint32_t), s);
  if (num_rendered > 0)
    tile_ranges_kernel<<<(unsigned)((num_rendered + 255) / 256), 256, 0, s>>>(sorted_keys, num_rendered,
                                                                              num_tiles, ranges);
  bucket_count_kernel<<<1, 1024, 0, s>>>(ranges, num_tiles, bucket_count, bucket_offsets, bucket_sum,
                                         tile_order, bucket_to_tile, bucket_to_tile_len);
  return check_launch("tile_prep_ordered");
}

int fgs_tile_order(int32_t num_tiles, const uint32_t* ranges, uint32_t* tile_order, void* stream) {
  FGS_CHECK_ARG(num_tiles >= 0, "num_tiles must be >= 0");
  if (num_tiles == 0) return FGS_OK;
  FGS_CHECK_ARG(ranges && tile_order, "missing pointer");
  tile_order_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(ranges, num_tiles, tile_order);
  return check_launch("tile_order");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free sort: fgs_sort_pairs on a fixed scratch area that lives in
// this library's device image instead of caller-provided memory.
//
// Some callers cannot allocate device memory when they sort: host
// applications that load this library as a plug-in under a fixed GPU memory
// budget and forbid allocation after start-up, and callers that must not pay
// for (or risk the implicit device synchronisation of) cudaMalloc/cudaFree in
// the middle of their frame. They pass only their keys and values.
//
// The scratch is a file-scope device array sized for kStaticSortMaxKeys keys
// with up to 64 key bits; every GPU that loads the library holds it (about
// 15 MB) until the process exits. Its address is looked up once per device,
// on the first call made with that device current.
namespace fgs {
constexpr int64_t kStaticSortMaxKeys = FGS_SORT_STATIC_MAX_KEYS;
constexpr int64_t kStaticSortParts = (kStaticSortMaxKeys + kPart - 1) / kPart;
constexpr size_t kStaticSortBytes =
    256 +                                                                      // timeout flag
    ((size_t)kMaxPasses * kRadix * 4 + 255) / 256 * 256 +                     // digit histograms
    ((size_t)kMaxPasses * kStaticSortParts * kRadix * 4 + 255) / 256 * 256 +  // look-back
    ((size_t)(kMaxPasses + 1) * 4 + 255) / 256 * 256 +                        // tickets, done
    ((size_t)kStaticSortMaxKeys * 8 + 255) / 256 * 256 +                      // ping-pong keys
    ((size_t)kStaticSortMaxKeys * 4 + 255) / 256 * 256;                       // ping-pong values

static __device__ __align__(256) unsigned char g_sort_scratch[kStaticSortBytes];

static std::mutex g_sort_scratch_mu;
static void* g_sort_scratch_ptr[64] = {nullptr};

// Device address of g_sort_scratch on the current device (host code may not
// use the symbol itself: on the host it names a stand-in, not device memory).
static int sort_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("sort_pairs_static: cudaGetDevice: %s", cudaGetErrorString(e));
    return FGS_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) {
    set_error("sort_pairs_static: device ordinal %d out of range", dev);
    return FGS_ERR_CAPACITY;
  }
  std::lock_guard<std::mutex> lk(g_sort_scratch_mu);
  if (g_sort_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_sort_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      set_error("sort_pairs_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return FGS_ERR_CUDA;
    }
    g_sort_scratch_ptr[dev] = ptr;
  }
  *out = g_sort_scratch_ptr[dev];
  return FGS_OK;
}
}  // namespace fgs

extern "C" int fgs_sort_pairs_static(int64_t num_rendered, int32_t key_bits,
                                     const uint64_t* keys_in, const uint32_t* values_in,
                                     uint64_t* keys_out, uint32_t* values_out, void* stream) {
  FGS_CHECK_ARG(num_rendered >= 0, "num_rendered must be >= 0");
  if (num_rendered > fgs::kStaticSortMaxKeys) {
    fgs::set_error("sort_pairs_static sorts at most %lld keys (its scratch is fixed); got %lld: "
                   "use fgs_sort_pairs with caller-provided workspace",
                   (long long)fgs::kStaticSortMaxKeys, (long long)num_rendered);
    return FGS_ERR_CAPACITY;
  }
  FGS_CHECK_ARG(key_bits >= 1 && key_bits <= 64, "key_bits must be in [1, 64]");
  if (num_rendered == 0) return FGS_OK;
  void* scratch = nullptr;
  const int st = fgs::sort_scratch_address(&scratch);
  if (st != FGS_OK) return st;
  // fgs_sort_pairs clears the histograms, look-back flags, tickets and the
  // timeout flag at the start of every call, so leftovers of the previous
  // call do not matter; the key/value halves need no clearing.
  return fgs_sort_pairs(num_rendered, key_bits, keys_in, values_in, keys_out, values_out, scratch,
                        fgs::kStaticSortBytes, stream);
}

// ---------------------------------------------------------------------------
// Status of the last sort run in a workspace: its timeout flag is the int at
// offset 0 (for the static sort, of the static scratch on the current device).
extern "C" int fgs_sort_status(const void* workspace, void* stream) {
  const void* flag = workspace;
  if (flag == nullptr) {
    void* scratch = nullptr;
    const int st = fgs::sort_scratch_address(&scratch);
    if (st != FGS_OK) return st;
    flag = scratch;
  }
  cudaStream_t s = (cudaStream_t)stream;
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, flag, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    fgs::set_error("sort_status: %s", cudaGetErrorString(e));
    return FGS_ERR_CUDA;
  }
  if (host != 0) {
    fgs::set_error("sort: a look-back wait gave up after its poll limit; the output holds "
                   "all-ones keys and the input values instead of the sorted pairs");
    return FGS_ERR_TIMEOUT;
  }
  return FGS_OK;
}

extern "C" int fgs_sort_set_test_hooks(int32_t spin_limit, int32_t withhold_first_partition) {
  FGS_CHECK_ARG(spin_limit >= 0, "spin_limit must be >= 0");
  fgs::g_spin_limit = spin_limit > 0 ? spin_limit : fgs::kSpinLimit;
  fgs::g_withhold_first = withhold_first_partition ? 1 : 0;
  return FGS_OK;
}
