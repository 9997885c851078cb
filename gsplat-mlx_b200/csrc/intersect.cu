// Tile intersection: count -> exclusive scan -> encode -> stable 64-bit
// radix sort -> tile offsets.
//
// Reference: gsplat_intersect.cpp:60-112 (tile rect and key encoding),
// :174-307 (staged pipeline), metal/gsplat_intersect.metal:33-136.  The
// reference sorts with MLX argsort+take (:266-286); here a hand-written LSD
// radix sort over only the key bits that can be non-zero
// (32 depth bits + tile bits + image bits) replaces it.  LSD radix sorting is
// stable, so equal keys keep encode order exactly as a stable argsort does.
//
// All integer work; this file is compiled without FMA contraction so that
// the float tile-rect arithmetic (divide, floor, ceil) rounds like the CPU.
#include <algorithm>

#include "common.cuh"

namespace gsb {
namespace {

// ------------------------------------------------------------ count/encode

struct Rect {
  int x0, y0, x1, y1;
};

// gsplat_intersect.cpp:67-99 == metal/gsplat_intersect.metal:43-59
__device__ __forceinline__ Rect tile_rect(float mx, float my, int rx, int ry, int ts, int tw,
                                          int th) {
  Rect r{0, 0, 0, 0};
  if (rx <= 0 || ry <= 0) return r;
  const float fts = (float)ts;
  const float trx = (float)rx / fts, try_ = (float)ry / fts;
  const float tx = mx / fts, ty = my / fts;
  r.x0 = min(max(0, (int)floorf(tx - trx)), tw);
  r.y0 = min(max(0, (int)floorf(ty - try_)), th);
  r.x1 = min(max(0, (int)ceilf(tx + trx)), tw);
  r.y1 = min(max(0, (int)ceilf(ty + try_)), th);
  return r;
}

// With `total`, the counts are also summed into *total (zeroed by the caller).
// Rect clipped to the tile-row window [ty0, ty1) (the whole grid: 0, th).
__device__ __forceinline__ Rect band_rect(float mx, float my, int rx, int ry, int ts, int tw,
                                          int th, int ty0, int ty1) {
  Rect r = tile_rect(mx, my, rx, ry, ts, tw, th);
  r.y0 = max(r.y0, ty0);
  r.y1 = min(r.y1, ty1);
  if (r.y1 < r.y0) r.y1 = r.y0;
  return r;
}

// Bins of the binned encode: blocks of kBinTiles x kBinTiles tiles.
constexpr int kBinTiles = 4;

// Number of bins along one axis that the tile range [a0, a1) touches.
__device__ __forceinline__ int bin_span(int a0, int a1) {
  return a1 > a0 ? (a1 - 1) / kBinTiles - a0 / kBinTiles + 1 : 0;
}

// Bins a rect touches (0 for an empty rect).
__device__ __forceinline__ int rect_bins(const Rect& r) {
  return (r.x1 > r.x0 && r.y1 > r.y0) ? bin_span(r.x0, r.x1) * bin_span(r.y0, r.y1) : 0;
}

// With `totals`, the tile counts are summed into totals[0] and, with
// `bins`, the bin counts into totals[1] (zeroed by the caller).
__global__ void __launch_bounds__(256) count_kernel(int64_t n, const float* __restrict__ means2d,
                                                    const int32_t* __restrict__ radii, int ts,
                                                    int tw, int th, int ty0, int ty1,
                                                    int32_t* __restrict__ tiles_per_gauss,
                                                    unsigned long long* __restrict__ totals,
                                                    int bins) {
  unsigned long long sum = 0, sum_b = 0;
  // kCountUnroll elements per round, their loads all in flight before the
  // rect arithmetic (the kernel is bound by load latency, not bandwidth)
  constexpr int kCountUnroll = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < n;
       i0 += kCountUnroll * stride) {
    int2 rad[kCountUnroll];
    float2 m[kCountUnroll];
#pragma unroll
    for (int u = 0; u < kCountUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      rad[u] = i < n ? __ldg(reinterpret_cast<const int2*>(radii) + i) : make_int2(0, 0);
      m[u] = i < n ? __ldg(reinterpret_cast<const float2*>(means2d) + i) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kCountUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= n) break;
      const Rect r = band_rect(m[u].x, m[u].y, rad[u].x, rad[u].y, ts, tw, th, ty0, ty1);
      const int c = (r.y1 - r.y0) * (r.x1 - r.x0);
      tiles_per_gauss[i] = c;
      sum += (unsigned long long)c;
      if (bins) sum_b += (unsigned long long)rect_bins(r);
    }
  }
  if (totals) {  // one atomic per CTA and total
    __shared__ unsigned long long s_sum[2][8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
      sum_b += __shfl_xor_sync(0xffffffffu, sum_b, o);
    }
    if ((threadIdx.x & 31) == 0) {
      s_sum[0][threadIdx.x >> 5] = sum;
      s_sum[1][threadIdx.x >> 5] = sum_b;
    }
    __syncthreads();
    if (threadIdx.x < 2 && (threadIdx.x == 0 || bins)) {
      unsigned long long t = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_sum[threadIdx.x][w];
      if (t) atomicAdd(totals + threadIdx.x, t);
    }
  }
}

// One warp encodes 32 consecutive Gaussians at a time.  A warp scan of their
// tile counts flattens the 32 runs into one index space j; lane l emits
// entries j = l, l+32, ...: the owner Gaussian of j is the last one whose
// run starts at or before j (found per 32-entry window from a bit mask of
// the run starts), its k-th tile in row-major order of its rect.  Run i
// starts at offsets[i] -- the reference's scan order (adjacent runs, so
// stores are coalesced) or any other order of the runs; every write is
// bounds-checked like the CPU path (gsplat_intersect.cpp:473).  With
// `packed_out`, each intersection is written there as one word (high key
// word << 32 | element id) instead of to isect_ids / flatten_ids.
// With `hist`, the kernel also counts the digits of the key bits above the depth
// word for the radix passes that follow (hist[p][d], 8-bit digits from
// bit 32, sign bit xor hist_flip: the digits the passes see).
constexpr int kEncodeThreads = 256;
constexpr int kEncodeWarps = kEncodeThreads / 32;

__global__ void __launch_bounds__(kEncodeThreads) encode_kernel(
    int64_t n, int n_per_image, const float* __restrict__ means2d,
    const int32_t* __restrict__ radii, const float* __restrict__ depths,
    const int32_t* __restrict__ offsets, int ts, int tw, int th, int ty0, int ty1, int tile_bits,
    int64_t n_isects, int64_t* __restrict__ isect_ids, int32_t* __restrict__ flatten_ids,
    uint64_t* __restrict__ packed_out, uint32_t* __restrict__ hist, int hist_passes,
    uint32_t hist_flip) {
  __shared__ int s_pref[kEncodeWarps][32];
  __shared__ int s_x0[kEncodeWarps][32], s_y0[kEncodeWarps][32], s_w[kEncodeWarps][32];
  __shared__ float s_invw[kEncodeWarps][32];
  __shared__ int s_e[kEncodeWarps][32], s_start[kEncodeWarps][32];
  __shared__ int64_t s_off[kEncodeWarps][32], s_base[kEncodeWarps][32];
  __shared__ uint32_t s_hist[4][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (hist)
    for (int i = threadIdx.x; i < 4 * 256; i += kEncodeThreads) (&s_hist[0][0])[i] = 0;
  __syncthreads();
  const int64_t chunks = (n + 31) / 32;
  for (int64_t ch = (int64_t)blockIdx.x * kEncodeWarps + warp; ch < chunks;
       ch += (int64_t)gridDim.x * kEncodeWarps) {
    const int64_t i = ch * 32 + lane;
    int cnt = 0;
    if (i < n) {
      const int2 rad = __ldg(reinterpret_cast<const int2*>(radii) + i);
      if (rad.x > 0 && rad.y > 0) {
        const float2 m = __ldg(reinterpret_cast<const float2*>(means2d) + i);
        const Rect r = band_rect(m.x, m.y, rad.x, rad.y, ts, tw, th, ty0, ty1);
        const int w = r.x1 - r.x0;
        cnt = (r.y1 - r.y0) * w;
        if (cnt > 0) {
          s_x0[warp][lane] = r.x0;
          s_y0[warp][lane] = r.y0;
          s_w[warp][lane] = w;
          s_invw[warp][lane] = 1.0f / (float)w;
          s_e[warp][lane] = (int)i;
          s_off[warp][lane] = __ldg(offsets + i);
          const int64_t image_id = i / n_per_image;
          s_base[warp][lane] = (image_id << (32 + tile_bits)) |
                               (int64_t)__float_as_uint(__ldg(depths + i));
        }
      }
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const int excl = incl - cnt;
    s_pref[warp][lane] = excl;
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    int carry = 0;  // owner of the last entry of the previous window
    for (int j0 = 0; j0 < total; j0 += 32) {
      // runs starting inside this window: bit (start - j0), owner in s_start
      const bool st = cnt > 0 && excl >= j0 && excl < j0 + 32;
      if (st) s_start[warp][excl - j0] = lane;
      const uint32_t starts = __reduce_or_sync(0xffffffffu, st ? 1u << (excl - j0) : 0u);
      __syncwarp();
      const uint32_t upto = starts & (0xFFFFFFFFu >> (31 - lane));
      const int o = upto ? s_start[warp][31 - __clz(upto)] : carry;
      carry = __shfl_sync(0xffffffffu, o, 31);
      const int j = j0 + lane;
      if (j < total) {
        const int k = j - s_pref[warp][o];
        const int w = s_w[warp][o];
        int dy = (int)(((float)k + 0.5f) * s_invw[warp][o]);  // k / w, then made exact
        if (dy * w > k) --dy;
        if ((dy + 1) * w <= k) ++dy;
        const int y = s_y0[warp][o] + dy;
        const int x = s_x0[warp][o] + (k - dy * w);
        const int64_t pos = s_off[warp][o] + k;
        const int64_t key = s_base[warp][o] | ((int64_t)(y * tw + x) << 32);
        if (pos >= 0 && pos < n_isects) {
          const uint32_t hi = (uint32_t)((uint64_t)key >> 32);
          if (packed_out) {
            packed_out[pos] = ((uint64_t)hi << 32) | (uint32_t)s_e[warp][o];
          } else {
            isect_ids[pos] = key;
            flatten_ids[pos] = s_e[warp][o];
          }
          if (hist) {
            const uint32_t h = hi ^ hist_flip;
            for (int p = 0; p < hist_passes; ++p) atomicAdd(&s_hist[p][(h >> (8 * p)) & 0xFFu], 1u);
          }
        }
      }
      __syncwarp();
    }
  }
  if (hist) {
    __syncthreads();
    for (int i = threadIdx.x; i < hist_passes * 256; i += kEncodeThreads) {
      const uint32_t c = (&s_hist[0][0])[i];
      if (c) atomicAdd(hist + i, c);
    }
  }
}

// ------------------------------------------------------------ scan

constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;
constexpr int kScanChunk = kScanThreads * kScanItems;

// Block-wide exclusive scan of one int64 value per thread; returns the
// exclusive prefix and writes the block total to *total.
template <int THREADS>
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, int64_t* s_warp, int64_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    constexpr int W = THREADS / 32;
    int64_t w = lane < W ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    if (lane < W) s_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const int64_t warp_prefix = warp == 0 ? 0 : s_warp[warp - 1];
  *total = s_warp[THREADS / 32 - 1];
  const int64_t excl = warp_prefix + incl - v;
  __syncthreads();
  return excl;
}

// With `perm`, element i of the scanned sequence is in[perm[i * stride]]
// (stride 2: the low words of packed 64-bit sort words); with `n_dev`, the
// length is *n_dev (the grid covers the host bound n).
__device__ __forceinline__ int32_t scan_value(const int32_t* in, const int32_t* perm, int stride,
                                              int64_t i) {
  return __ldg(in + (perm ? (int64_t)__ldg(perm + i * stride) : i));
}

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(int64_t n,
                                                                    const int32_t* __restrict__ in,
                                                                    const int32_t* __restrict__ perm,
                                                                    int stride,
                                                                    const int64_t* __restrict__ n_dev,
                                                                    int64_t* __restrict__ sums) {
  __shared__ int64_t s_warp[32];
  if (n_dev) n = *n_dev;
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int64_t acc = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    if (i < n) acc += scan_value(in, perm, stride, i);
  }
  int64_t total;
  block_exclusive_scan<kScanThreads>(acc, s_warp, &total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Single CTA: exclusive scan of the block sums in place; total to *total.
__global__ void __launch_bounds__(1024) scan_sums_kernel(int64_t nb, int64_t* __restrict__ sums,
                                                         int64_t* __restrict__ total_out) {
  __shared__ int64_t s_warp[32];
  const int64_t per = (nb + 1023) / 1024;
  const int64_t b0 = (int64_t)threadIdx.x * per;
  int64_t acc = 0;
  for (int64_t k = 0; k < per; ++k)
    if (b0 + k < nb) acc += sums[b0 + k];
  int64_t total;
  int64_t run = block_exclusive_scan<1024>(acc, s_warp, &total);
  for (int64_t k = 0; k < per; ++k)
    if (b0 + k < nb) {
      const int64_t v = sums[b0 + k];
      sums[b0 + k] = run;
      run += v;
    }
  if (threadIdx.x == 0 && total_out) *total_out = total;
}

// Without `perm` it may run in place (in == out): every element is read
// before it is written.  With `perm` the scanned sequence is in[perm[i]] and its prefix of
// position i is stored at out[perm[i]] (scattered back to element order).
__global__ void __launch_bounds__(kScanThreads) scan_down_kernel(int64_t n, const int32_t* in,
                                                                  const int32_t* __restrict__ perm,
                                                                  int stride,
                                                                  const int64_t* __restrict__ n_dev,
                                                                  const int64_t* __restrict__ sums,
                                                                  int32_t* out) {
  __shared__ int64_t s_warp[32];
  if (n_dev) n = *n_dev;
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int32_t v[kScanItems];
  int64_t acc = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    v[k] = i < n ? (perm ? scan_value(in, perm, stride, i) : in[i]) : 0;
    acc += v[k];
  }
  int64_t total;
  int64_t run = block_exclusive_scan<kScanThreads>(acc, s_warp, &total) + sums[blockIdx.x];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    if (i < n) out[perm ? (int64_t)__ldg(perm + i * stride) : i] = (int32_t)run;
    run += v[k];
  }
}

// The whole scan in one CTA of kScanThreads threads, chunk by chunk with a
// running carry (no perm, no device length): for short sequences, where
// the three-launch scan is all latency.
constexpr int64_t kSmallScan = 4 * kScanChunk;

__global__ void __launch_bounds__(kScanThreads) scan_small_kernel(int64_t n,
                                                                   const int32_t* __restrict__ in,
                                                                   int32_t* __restrict__ out,
                                                                   int64_t* __restrict__ total_out) {
  __shared__ int64_t s_warp[32];
  int64_t carry = 0;
  for (int64_t base = 0; base < n; base += kScanChunk) {
    int32_t v[kScanItems];
    int64_t acc = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
      const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
      v[k] = i < n ? __ldg(in + i) : 0;
      acc += v[k];
    }
    int64_t total;
    int64_t run = block_exclusive_scan<kScanThreads>(acc, s_warp, &total) + carry;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
      const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
      if (i < n) out[i] = (int32_t)run;
      run += v[k];
    }
    carry += total;
  }
  if (threadIdx.x == 0 && total_out) *total_out = carry;
}

size_t scan_ws_bytes(int64_t n) {
  const int64_t nb = ceil_div(n < 1 ? 1 : n, kScanChunk);
  return (size_t)((nb * 8 + 255) / 256 * 256);
}

int scan_i32(int64_t n, const int32_t* in, int32_t* out, int64_t* total, void* ws, size_t ws_bytes,
             cudaStream_t s, const int32_t* perm = nullptr, int perm_stride = 1,
             const int64_t* n_dev = nullptr) {
  if (n <= 0) {
    if (total) cudaMemsetAsync(total, 0, sizeof(int64_t), s);
    return launch_status("scan");
  }
  if (!ws || ws_bytes < scan_ws_bytes(n)) {
    set_error("scan: workspace of %zu bytes needed", scan_ws_bytes(n));
    return GS_ERR_WORKSPACE;
  }
  if (n <= kSmallScan && !perm && !n_dev && in != out) {
    scan_small_kernel<<<1, kScanThreads, 0, s>>>(n, in, out, total);
    return launch_status("scan");
  }
  const int64_t nb = ceil_div(n, kScanChunk);
  int64_t* sums = static_cast<int64_t*>(ws);
  scan_reduce_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(n, in, perm, perm_stride, n_dev, sums);
  scan_sums_kernel<<<1, 1024, 0, s>>>(nb, sums, total);
  scan_down_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(n, in, perm, perm_stride, n_dev, sums, out);
  return launch_status("scan");
}

// Visible elements -- both radii positive, a superset of the elements with
// tiles in any tile-row window -- in element order: block counts, then
// (with the scanned counts) packed words (depth bits << 32 | element) at
// their compacted positions, the input of the depth sort.
__device__ __forceinline__ int visible_at(const int32_t* radii, int64_t i) {
  const int2 r = __ldg(reinterpret_cast<const int2*>(radii) + i);
  return (r.x > 0 && r.y > 0) ? 1 : 0;
}

__global__ void __launch_bounds__(kScanThreads) visible_count_kernel(
    int64_t n, const int32_t* __restrict__ radii, int64_t* __restrict__ sums) {
  __shared__ int64_t s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int64_t acc = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    if (i < n) acc += visible_at(radii, i);
  }
  int64_t total;
  block_exclusive_scan<kScanThreads>(acc, s_warp, &total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kScanThreads) visible_depth_keys_kernel(
    int64_t n, const int32_t* __restrict__ radii, const float* __restrict__ depths,
    const int64_t* __restrict__ sums, uint64_t* __restrict__ words) {
  __shared__ int64_t s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int f[kScanItems];
  int64_t acc = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    f[k] = i < n ? visible_at(radii, i) : 0;
    acc += f[k];
  }
  int64_t total;
  int64_t run = block_exclusive_scan<kScanThreads>(acc, s_warp, &total) + sums[blockIdx.x];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    if (f[k]) {
      const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
      words[run] = ((uint64_t)__float_as_uint(__ldg(depths + i)) << 32) | (uint32_t)i;
      ++run;
    }
  }
}

// With the scanned block counts of visible_count_kernel: the visible
// elements' projection outputs as packed rows, in element (image, Gaussian)
// order -- image and Gaussian ids, radii, means2d, depths, conics and, when
// given, compensations.  Rows past `capacity` are dropped.
struct PackArgs {
  int64_t n, capacity;
  int N;
  const int32_t* radii;
  const float *means2d, *depths, *conics, *comps;
  int32_t *image_ids, *gaussian_ids, *p_radii;
  float *p_means2d, *p_depths, *p_conics, *p_comps;
};

__global__ void __launch_bounds__(kScanThreads) pack_rows_kernel(const PackArgs a,
                                                                 const int64_t* __restrict__ sums) {
  __shared__ int64_t s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int f[kScanItems];
  int64_t acc = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    f[k] = i < a.n ? visible_at(a.radii, i) : 0;
    acc += f[k];
  }
  int64_t total;
  int64_t run = block_exclusive_scan<kScanThreads>(acc, s_warp, &total) + sums[blockIdx.x];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    if (!f[k]) continue;
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    if (run < a.capacity) {
      const int64_t r = run;
      a.image_ids[r] = (int32_t)(i / a.N);
      a.gaussian_ids[r] = (int32_t)(i % a.N);
      reinterpret_cast<int2*>(a.p_radii)[r] = __ldg(reinterpret_cast<const int2*>(a.radii) + i);
      reinterpret_cast<float2*>(a.p_means2d)[r] =
          __ldg(reinterpret_cast<const float2*>(a.means2d) + i);
      a.p_depths[r] = __ldg(a.depths + i);
#pragma unroll
      for (int c = 0; c < 3; ++c) a.p_conics[r * 3 + c] = __ldg(a.conics + i * 3 + c);
      if (a.comps) a.p_comps[r] = __ldg(a.comps + i);
    }
    ++run;
  }
}

// ------------------------------------------------------------ radix sort
// LSD radix sort, 8-bit digits, one kernel per digit ("onesweep": Adinets &
// Merrill, 2022).  A histogram kernel counts the digits of every pass in
// one read of the keys.  Each pass kernel then takes tiles of 4096 keys in
// the order its CTAs start (an atomic tile counter), ranks them stably in
// shared memory, publishes its per-digit tile counts, and finds the counts
// of all earlier tiles by decoupled look-back: walking back over the
// published tile states until one carries an inclusive prefix.  Keys are
// read once and written once per pass.
//
// Every look-back wait is bounded: a tile waits only for tiles whose CTAs
// already started, which publish their counts without waiting themselves,
// so the wait ends; should it not within the bound (a bug, not a workload),
// the kernel raises the error word in the workspace, takes the count as 0
// and finishes -- the output is then wrong but no GPU is held.

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 16;                          // keys per thread
constexpr int kSortTile = kSortThreads * kSortItems;    // 4096 keys per CTA
constexpr int kWarpSpan = 32 * kSortItems;              // 512 keys per warp
constexpr int kRadix = 256;
constexpr int kMaxPasses = 8;
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t digit_of(uint64_t k, int shift, uint64_t flip) {
  return (uint32_t)(((k ^ flip) >> shift) & 0xFFu);
}

// hist[p][d] += number of keys whose digit of pass p is d, for passes
// 0..passes-1 starting at bit begin_bit.
__global__ void __launch_bounds__(256) radix_hist_kernel(int64_t n,
                                                         const uint64_t* __restrict__ keys,
                                                         int begin_bit, int passes, uint64_t flip,
                                                         const int64_t* __restrict__ n_dev,
                                                         uint32_t* __restrict__ hist) {
  __shared__ uint32_t s_hist[kMaxPasses][kRadix];
  if (n_dev) n = *n_dev;
  for (int i = threadIdx.x; i < kMaxPasses * kRadix; i += blockDim.x) (&s_hist[0][0])[i] = 0;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 4;
  for (int64_t i0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i0 < n; i0 += stride) {
    uint64_t k[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) k[r] = i0 + r < n ? __ldg(keys + i0 + r) : 0ull;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if (i0 + r >= n) break;
      for (int p = 0; p < passes; ++p)
        atomicAdd(&s_hist[p][digit_of(k[r], begin_bit + 8 * p, flip)], 1u);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRadix; i += blockDim.x) {
    const uint32_t c = (&s_hist[0][0])[i];
    if (c) atomicAdd(hist + i, c);
  }
}

// Key sources and sinks of a pass.
//   kKV     64-bit keys and int32 values in two arrays (the plain key sort);
//   kPacked one 64-bit word per key: (high key word << 32) | 32-bit value;
//   kFinal  sink only: the word's value is an element e; the pass writes the
//           full key (high word | bits of depths[e]) and e.
enum PassIO { kKV = 0, kPacked = 1, kFinal = 2 };

template <bool VALS>
struct PassSmem {
  uint64_t keys[kSortTile];
  int32_t vals[VALS ? kSortTile : 1];
  uint32_t hist[kSortWarps][kRadix];  // warp counts -> warp exclusive offsets
  uint32_t digit_start[kRadix];       // CTA-local exclusive prefix over digits
  uint64_t goff[kRadix];              // global offset of each digit for this tile
  int64_t warp_tot[32];
  int tile;
};

struct PassArgs {
  int64_t n;
  const uint64_t* keys_in;
  const int32_t* vals_in;  // kKV
  uint64_t* keys_out;      // kKV, kPacked; kFinal: the int64 keys
  int32_t* vals_out;       // kKV; kFinal: the element ids
  const float* depths;     // kFinal
  int shift;
  uint64_t flip;
  int pass;
  const uint32_t* pass_hist;
  uint32_t* tile_counter;
  uint64_t* state;
  uint32_t* error_word;
  const int64_t* n_dev;  // when set, the length is *n_dev (the grid covers n)
  uint32_t spin_limit;   // polls of one look-back wait before it gives up
};

__device__ __forceinline__ uint64_t load_state(const uint64_t* p) {
  return *reinterpret_cast<const volatile uint64_t*>(p);
}
__device__ __forceinline__ void store_state(uint64_t* p, uint64_t v) {
  *reinterpret_cast<volatile uint64_t*>(p) = v;
}

// One digit pass.  state[tile][digit] = (tag << 32) | value with tag
// 2*pass+1 (value = this tile's count) or 2*pass+2 (value = inclusive
// prefix over tiles 0..tile); words of other passes or zero mean "not yet".
template <int IN, int OUT>
__global__ void __launch_bounds__(kSortThreads, 3) radix_onesweep_kernel(const PassArgs a) {
  constexpr bool VALS = IN == kKV;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PassSmem<VALS>& sm = *reinterpret_cast<PassSmem<VALS>*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) sm.tile = (int)atomicAdd(a.tile_counter, 1u);
  const uint32_t hist_d = __ldg(a.pass_hist + threadIdx.x);  // this pass's total of digit tid
  for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&sm.hist[0][0])[i] = 0;
  __syncthreads();
  const int tile = sm.tile;
  const int64_t tile_base = (int64_t)tile * kSortTile;
  int64_t n = a.n;
  if (a.n_dev) {
    // the grid covers the host bound; tiles past the device length leave
    // (nothing waits on them: look-back only reads earlier tiles)
    n = *a.n_dev;
    if (tile_base >= n) return;
  }
  const int shift = a.shift;
  const uint64_t flip = a.flip;
  const int64_t base = tile_base + (int64_t)warp * kWarpSpan;
  uint64_t k[kSortItems];
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {  // all loads in flight before ranking
    const int64_t i = base + r * 32 + lane;
    k[r] = i < n ? __ldg(a.keys_in + i) : 0ull;
  }
  // Stable ranks: a warp's keys in index order (round r covers keys
  // r*32..r*32+31 of its span), lanes in lane order; invalid lanes (past
  // n) form their own group and count nowhere.  Two 16-bit ranks per word.
  uint32_t rank[kSortItems / 2];
  const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    const bool valid = base + r * 32 + lane < n;
    const uint32_t d = valid ? digit_of(k[r], shift, flip) : (uint32_t)kRadix;
    // lanes with the same digit: one ballot per digit bit (and one for
    // validity) -- faster than __match_any_sync here
    uint32_t peers = __ballot_sync(0xffffffffu, valid);
    if (!valid) peers = ~peers;
#pragma unroll
    for (int bit = 0; bit < 8; ++bit) {
      const uint32_t bal = __ballot_sync(0xffffffffu, (d >> bit) & 1u);
      peers &= ((d >> bit) & 1u) ? bal : ~bal;
    }
    const uint32_t before = __popc(peers & lt_mask);
    const int leader = __ffs(peers) - 1;
    uint32_t cur = 0;
    if (valid) cur = sm.hist[warp][d];
    __syncwarp();
    if (valid && lane == leader) sm.hist[warp][d] = cur + __popc(peers);
    __syncwarp();
    const uint32_t rk = cur + before;
    if (r & 1) rank[r >> 1] |= rk << 16;
    else rank[r >> 1] = rk;
  }
  __syncthreads();
  const int d = threadIdx.x;  // one thread per digit
  uint32_t cta_count = 0;
#pragma unroll
  for (int w = 0; w < kSortWarps; ++w) {
    const uint32_t c = sm.hist[w][d];
    sm.hist[w][d] = cta_count;
    cta_count += c;
  }
  // Publish this tile's counts before anything else, so that later tiles
  // can sum them while this one stages its keys.
  const uint64_t tag_agg = (uint64_t)(2 * a.pass + 1) << 32;
  const uint64_t tag_inc = (uint64_t)(2 * a.pass + 2) << 32;
  uint64_t* my = a.state + (int64_t)tile * kRadix + d;
  store_state(my, (tile == 0 ? tag_inc : tag_agg) | cta_count);
  int64_t total;
  const int64_t start = block_exclusive_scan<kSortThreads>(cta_count, sm.warp_tot, &total);
  sm.digit_start[d] = (uint32_t)start;
  __syncthreads();
  // Stage the keys at their places in this tile's digit order; the
  // registers that held them serve the look-back below.
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    const int64_t i = base + r * 32 + lane;
    if (i < n) {
      const uint32_t dg = digit_of(k[r], shift, flip);
      const uint32_t rk = (rank[r >> 1] >> ((r & 1) * 16)) & 0xFFFFu;
      const uint32_t p = sm.digit_start[dg] + sm.hist[warp][dg] + rk;
      sm.keys[p] = k[r];
      if constexpr (VALS) sm.vals[p] = __ldg(a.vals_in + i);
    }
  }
  // Look back for the exclusive prefix over earlier tiles, kLookback tile
  // states per round with all their loads in flight: when every tile of a
  // small sort runs at once, the inclusive prefixes advance kLookback tiles
  // per memory round trip.
  uint64_t excl = 0;
  if (tile > 0) {
    constexpr int kLookback = 32;
    bool found = false;
    for (int t0 = tile - 1; t0 >= 0 && !found; t0 -= kLookback) {
      uint64_t w[kLookback];
#pragma unroll
      for (int i = 0; i < kLookback; ++i)
        w[i] = t0 - i >= 0 ? load_state(a.state + (int64_t)(t0 - i) * kRadix + d) : tag_inc;
#pragma unroll
      for (int i = 0; i < kLookback; ++i) {
        if (found) break;
        const uint64_t* q = a.state + (int64_t)(t0 - i) * kRadix + d;
        uint64_t v = w[i];
        uint32_t spins = 0;
        while ((v & ~0xFFFFFFFFull) != tag_agg && (v & ~0xFFFFFFFFull) != tag_inc) {
          if (++spins > a.spin_limit) {
            atomicOr(a.error_word, 1u);
            v = tag_inc;  // give up: count 0, stop walking
            break;
          }
          __nanosleep(32);
          v = load_state(q);
        }
        excl += (uint32_t)v;
        found = (v & ~0xFFFFFFFFull) == tag_inc;
      }
    }
    store_state(my, tag_inc | (uint32_t)(excl + cta_count));
  }
  // Global digit bases: exclusive scan of this pass's digit totals.
  int64_t unused;
  const int64_t dbase = block_exclusive_scan<kSortThreads>(hist_d, sm.warp_tot, &unused);
  sm.goff[d] = (uint64_t)dbase + excl;
  __syncthreads();
  const int64_t tile_n = (n - tile_base) < kSortTile ? (n - tile_base) : kSortTile;
  if constexpr (OUT == kFinal) {
    // all depth gathers of this thread in flight before the stores
    uint32_t dep[kSortItems];
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
      const int i = threadIdx.x + r * kSortThreads;
      dep[r] = i < tile_n ? __float_as_uint(__ldg(a.depths + (uint32_t)sm.keys[i])) : 0u;
    }
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
      const int i = threadIdx.x + r * kSortThreads;
      if (i < tile_n) {
        const uint64_t key = sm.keys[i];
        const uint32_t dg = digit_of(key, shift, flip);
        const int64_t dst = (int64_t)sm.goff[dg] + (i - (int64_t)sm.digit_start[dg]);
        a.keys_out[dst] = (key & 0xFFFFFFFF00000000ull) | (uint64_t)dep[r];
        a.vals_out[dst] = (int32_t)(uint32_t)key;
      }
    }
  } else {
    for (int i = threadIdx.x; i < tile_n; i += kSortThreads) {
      const uint64_t key = sm.keys[i];
      const uint32_t dg = digit_of(key, shift, flip);
      const int64_t dst = (int64_t)sm.goff[dg] + (i - (int64_t)sm.digit_start[dg]);
      a.keys_out[dst] = key;
      if constexpr (OUT == kKV) a.vals_out[dst] = sm.vals[i];
    }
  }
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Workspace of a sort of n keys: the look-back error word (first, so that
// its place does not depend on n; cleared by the public entry points), the
// ping-pong buffers, then one region cleared per sort (digit histograms of
// every pass, tile counters, one tile-state slice shared by the passes).
struct SortLayout {
  size_t err, keys_alt, vals_alt, hist, ctrl, state, total;
};

SortLayout sort_layout(int64_t n) {
  SortLayout L;
  const int64_t n1 = n < 1 ? 1 : n;
  const int64_t tiles = ceil_div(n1, kSortTile);
  L.err = 0;
  L.keys_alt = 256;
  L.vals_alt = L.keys_alt + align256(sizeof(uint64_t) * (size_t)n1);
  L.hist = L.vals_alt + align256(sizeof(int32_t) * (size_t)n1);
  L.ctrl = L.hist + align256(sizeof(uint32_t) * kMaxPasses * kRadix);
  L.state = L.ctrl + 256;
  L.total = L.state + align256(sizeof(uint64_t) * (size_t)tiles * kRadix);
  return L;
}

// Clears the per-call region of sort_layout(n) at `ws` and returns its
// digit histograms, for a producer that counts the digits itself.
uint32_t* radix_reset(int64_t n, char* ws, cudaStream_t s) {
  const SortLayout L = sort_layout(n);
  cudaMemsetAsync(ws + L.hist, 0, L.total - L.hist, s);
  return reinterpret_cast<uint32_t*>(ws + L.hist);
}

template <int IN, int OUT>
void launch_pass(int tiles, const PassArgs& a, cudaStream_t s) {
  const int smem = (int)sizeof(PassSmem<IN == kKV>);
  cudaFuncSetAttribute(radix_onesweep_kernel<IN, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       smem);
  radix_onesweep_kernel<IN, OUT><<<tiles, kSortThreads, smem, s>>>(a);
}

void launch_pass(int in, int out, int tiles, const PassArgs& a, cudaStream_t s) {
  if (in == kKV) launch_pass<kKV, kKV>(tiles, a, s);
  else if (out == kPacked) launch_pass<kPacked, kPacked>(tiles, a, s);
  else launch_pass<kPacked, kFinal>(tiles, a, s);
}

// LSD passes over key bits [begin_bit, end_bit) with the scratch of
// sort_layout(n) at `ws`; the last pass lands in (out_k, out_v) and the
// input is only read.  `in` is the source form (kKV or kPacked), `out` the
// sink form of the last pass (kKV, kPacked or kFinal); the passes between
// move kKV (kKV sorts) or kPacked words through the scratch and out_k.  With end_bit == 64 and signed_keys the
// sign bit is flipped so that the unsigned digit order is the signed int64
// order.
// The digit histograms come from radix_hist_kernel, or from the producer
// of the keys after radix_reset (hist_ready).
void sort_passes(int64_t n, int begin_bit, int end_bit, int in, int out, const uint64_t* in_k,
                 const int32_t* in_v, uint64_t* out_k, int32_t* out_v, char* ws, cudaStream_t s,
                 bool hist_ready = false, const int64_t* n_dev = nullptr,
                 const float* depths = nullptr, bool signed_keys = true) {
  const SortLayout L = sort_layout(n);
  uint64_t* alt_k = reinterpret_cast<uint64_t*>(ws + L.keys_alt);
  int32_t* alt_v = reinterpret_cast<int32_t*>(ws + L.vals_alt);
  uint32_t* hist = reinterpret_cast<uint32_t*>(ws + L.hist);
  const int tiles = (int)ceil_div(n, kSortTile);
  const int passes = (end_bit - begin_bit + 7) / 8;
  const uint64_t flip = signed_keys && end_bit == 64 ? (1ull << 63) : 0ull;
  if (!hist_ready) {  // else radix_reset ran and the producer counted the digits
    cudaMemsetAsync(ws + L.hist, 0, L.total - L.hist, s);
    radix_hist_kernel<<<grid_for(ceil_div(n, 4), 256, 2), 256, 0, s>>>(
        n, in_k, begin_bit, passes, flip, n_dev, hist);
  }
  PassArgs a{};
  a.n = n;
  a.keys_in = in_k;
  a.vals_in = in_v;
  a.depths = depths;
  a.flip = flip;
  a.state = reinterpret_cast<uint64_t*>(ws + L.state);
  a.error_word = reinterpret_cast<uint32_t*>(ws + L.err);
  a.n_dev = n_dev;
  a.spin_limit = kSpinLimit;
  int src = in;
  for (int pass = 0; pass < passes; ++pass) {
    const bool last = pass == passes - 1;
    const bool to_out = ((passes - 1 - pass) % 2) == 0;
    const int dst = last ? out : (in == kKV ? kKV : kPacked);
    a.keys_out = to_out ? out_k : alt_k;
    a.vals_out = to_out ? out_v : alt_v;
    a.shift = begin_bit + pass * 8;
    a.pass = pass;
    a.pass_hist = hist + pass * kRadix;
    a.tile_counter = reinterpret_cast<uint32_t*>(ws + L.ctrl) + pass;
    launch_pass(src, dst, tiles, a, s);
    a.keys_in = a.keys_out;
    a.vals_in = a.vals_out;
    src = dst;
  }
}

void radix_passes(int64_t n, int begin_bit, int end_bit, const uint64_t* in_k, const int32_t* in_v,
                  uint64_t* out_k, int32_t* out_v, char* ws, cudaStream_t s) {
  sort_passes(n, begin_bit, end_bit, kKV, kKV, in_k, in_v, out_k, out_v, ws, s);
}

// Workspace of the depth-first sorted encode (n elements, m intersections).
struct SortedEncodeLayout {
  size_t sort, nvis, ek, pk, offs, scan, dk, total;
};

SortedEncodeLayout sorted_encode_layout(int64_t n, int64_t m) {
  // element arrays first (their places depend on n only, so that a later
  // call with the same elements can reuse the depth order), then the sort
  // scratch and the depth-ordered intersections (sized by m)
  SortedEncodeLayout L;
  const int64_t big = (n > m ? n : m) < 1 ? 1 : (n > m ? n : m);
  const int64_t n1 = n < 1 ? 1 : n, m1 = m < 1 ? 1 : m;
  size_t o = 0;
  L.nvis = o; o += 256;
  L.ek = o; o += align256(8 * (size_t)n1);
  L.pk = o; o += align256(8 * (size_t)n1);
  L.offs = o; o += align256(4 * (size_t)n1);
  L.scan = o; o += scan_ws_bytes(n1);
  L.sort = o; o += sort_layout(big).total;
  L.dk = o; o += align256(8 * (size_t)m1);
  L.total = o;
  return L;
}

// ------------------------------------------------------------ binned encode
// The tile grid is cut into bins of kBinTiles x kBinTiles tiles.  Every
// element lists itself once per bin its tile rect touches, as the entry
// (bin << 32 | depth bits, element) -- bin << 31 when the caller promises
// positive depths, one key bit fewer; a stable sort of those entries groups
// them by bin, in depth-bit order and, for equal depth bits, in element
// order.  One CTA per tile then walks its bin's list and keeps the elements
// whose rect covers the tile: its intersections, already in the order of
// the full 64-bit key sort, written at the tile's offset.  The walk runs
// over work items of at most kItemEntries entries of one bin (so that the
// dense bins do not set the kernel's length), each for all 16 tiles of its
// bin: a count phase, a scan of the tiles' counts into their offsets, and a
// write phase.

// Element rect in 16-bit tile units: x = x0 | x1 << 16, y = y0 | y1 << 16.
__device__ __forceinline__ uint2 pack_rect(const Rect& r) {
  return make_uint2((uint32_t)r.x0 | ((uint32_t)r.x1 << 16), (uint32_t)r.y0 | ((uint32_t)r.y1 << 16));
}

// Tiles of a bin an entry's rect covers: bit 4j+i for tile (bx*4+i, by*4+j).
__device__ __forceinline__ uint32_t cover_mask(uint2 r, int tx0, int ty0_) {
  const int x0 = (int)(r.x & 0xFFFFu) - tx0, x1 = (int)(r.x >> 16) - tx0;
  const int y0 = (int)(r.y & 0xFFFFu) - ty0_, y1 = (int)(r.y >> 16) - ty0_;
  auto span = [](int a0, int a1) -> uint32_t {  // bits [max(a0,0), min(a1,4))
    const int lo = a0 < 0 ? 0 : (a0 > 4 ? 4 : a0), hi = a1 < 0 ? 0 : (a1 > 4 ? 4 : a1);
    return hi > lo ? ((1u << hi) - 1u) & ~((1u << lo) - 1u) : 0u;
  };
  const uint32_t xm = span(x0, x1), ym = span(y0, y1);
  uint32_t m = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if ((ym >> j) & 1u) m |= xm << (4 * j);
  return m;
}

// The tiles of a bin mask (bit 4j+i: tile column i, row j of the bin) that
// a Gaussian may reach with alpha >= 1/255 at some pixel centre; the others
// are dropped.  (mx, my) is the mean relative to the bin's first pixel
// centre; sigma(u, v) = 0.5 (c0 u^2 + c2 v^2) + c1 u v with (u, v) = pixel
// centre - mean, as the rasterizer evaluates it.
//
// A pixel can pass only inside the ellipse sigma <= tau with tau =
// ln(255 o / 0.998) plus 1e-5 (1 + mag), mag bounding the terms of sigma over
// the bin (the rasterizer's fp32 sigma is within a few ulp of mag of the
// exact value, and the 0.998 covers __expf).  Per row of tiles the ellipse's
// u-range over the row's strip of v is exact: the largest u lies at the
// clamp of the ellipse's rightmost point into the strip (u_max(v) is
// concave), the smallest at the clamp of the leftmost; the range is widened
// by 0.4% of the ellipse's half width + 0.01 px, four times the worst fp32
// error of the square roots (the determinant is formed with a compensated
// product; the hardware reciprocal and reciprocal square root, a few ulp,
// are far inside that widening).  A tile stays when its pixel-centre span
// meets the row's range.
// Conics that are not positive definite and NaN opacities keep every tile.
// sqrt(max(x, 0)) from the hardware reciprocal square root (0 at x <= 0).
__device__ __forceinline__ float fast_sqrt(float x) {
  x = fmaxf(x, 0.0f);
  return x * rsqrtf(fmaxf(x, 1.0e-30f));
}

__device__ __forceinline__ uint32_t bin_hit_mask(uint32_t m, float mx, float my, float c0,
                                                 float c1, float c2, float o, int ts) {
  // non-finite opacities reach alpha 0.99 somewhere (NaN, +inf: everywhere;
  // -inf: where the exponential underflows): kept
  if (!(c0 > 0.0f && c2 > 0.0f) || !(fabsf(o) < INFINITY)) return m;
  const float pc = c1 * c1;
  const float det = __fadd_rn(__fmaf_rn(c0, c2, -pc), -__fmaf_rn(c1, c1, -pc));
  if (!(det > 0.0f)) return m;
  const float span = (float)(kBinTiles * ts - 1), fts = (float)ts;
  const float ul = -mx, uh = span - mx, vl = -my, vh = span - my;
  const float U = fmaxf(fabsf(ul), fabsf(uh)), V = fmaxf(fabsf(vl), fabsf(vh));
  const float mag = 0.5f * (c0 * U * U + c2 * V * V) + fabsf(c1) * U * V;
  const float lvl = o * (255.0f / 0.998f);
  if (!(lvl > 0.0f)) return 0u;  // o <= 0: alpha below the threshold everywhere
  const float tau = __logf(lvl) + 1.0e-5f * mag + 1.0e-5f;
  if (!(tau > 0.0f)) return 0u;  // even the centre stays below the threshold
  const float t2 = 2.0f * tau;
  const float inv_det = __fdividef(1.0f, det);
  const float ur = fast_sqrt(t2 * c2 * inv_det);  // half width of the ellipse in u
  const float ve = fast_sqrt(t2 * c0 * inv_det);  // half height in v
  const float inv_c0 = __fdividef(1.0f, c0);
  const float vr = -c1 * ur * __fdividef(1.0f, c2);  // v of the rightmost point
  const float eps_u = 4.0e-3f * ur + 0.01f, ve_w = ve * 1.004f + 0.01f;
  const float t2c0 = t2 * c0;
  uint32_t out = 0u;
#pragma unroll
  for (int j = 0; j < kBinTiles; ++j) {
    const uint32_t row = (m >> (4 * j)) & 0xFu;
    const float v0 = vl + (float)j * fts, v1 = v0 + (fts - 1.0f);
    if (!row || v0 > ve_w || v1 < -ve_w) continue;
    const float lo = fmaxf(v0, -ve), hi = fminf(v1, ve);
    const float va = fminf(fmaxf(vr, lo), hi), vb = fminf(fmaxf(-vr, lo), hi);
    const float umax = (-c1 * va + fast_sqrt(t2c0 - det * va * va)) * inv_c0 + eps_u;
    const float umin = (-c1 * vb - fast_sqrt(t2c0 - det * vb * vb)) * inv_c0 - eps_u;
#pragma unroll
    for (int i = 0; i < kBinTiles; ++i) {
      const float u0 = ul + (float)i * fts, u1 = u0 + (fts - 1.0f);
      if (((row >> i) & 1u) && u1 >= umin && u0 <= umax) out |= 1u << (4 * j + i);
    }
  }
  return out;
}

struct BinArgs {
  int64_t n;  // elements I*N
  int n_per_image, ts, tw, th, ty0, ty1;
  int sw, n_bins_per_image;  // bins per row, bins per image
  int dbits;                 // depth bits in the entry key: 32, or 31 (sign bit clear)
  const float* means2d;
  const int32_t* radii;
  const float* depths;
  const int32_t* image_ids;  // packed rows: each row's image (else i / n_per_image)
};

// Block sums of the per-element bin counts (the scan's first half).
__global__ void __launch_bounds__(kScanThreads) bin_count_kernel(const BinArgs a,
                                                                 int64_t* __restrict__ sums) {
  __shared__ int64_t s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int2 rad[kScanItems];
  float2 mu[kScanItems];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {  // all loads in flight first
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    rad[k] = i < a.n ? __ldg(reinterpret_cast<const int2*>(a.radii) + i) : make_int2(0, 0);
    mu[k] = i < a.n ? __ldg(reinterpret_cast<const float2*>(a.means2d) + i)
                    : make_float2(0.0f, 0.0f);
  }
  int64_t acc = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k)
    acc += rect_bins(band_rect(mu[k].x, mu[k].y, rad[k].x, rad[k].y, a.ts, a.tw, a.th, a.ty0,
                               a.ty1));
  int64_t total;
  block_exclusive_scan<kScanThreads>(acc, s_warp, &total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// With the scanned block sums: each element's entries at its place in
// element order and its packed rect.  A block takes its kScanChunk elements
// in kScanItems rounds of one element per thread; each warp then writes the
// entries of its 32 elements together (entry j of the warp's run: owner
// from a bit mask of run starts, as in the encode), so that the stores are
// coalesced.  Entries past n_entries are dropped.
constexpr int kScanWarps = kScanThreads / 32;

__global__ void __launch_bounds__(kScanThreads) bin_emit_kernel(
    const BinArgs a, const int64_t* __restrict__ sums, int64_t n_entries,
    uint64_t* __restrict__ keys, int32_t* __restrict__ vals, uint2* __restrict__ rects) {
  __shared__ int64_t s_warp[32];
  __shared__ int s_pref[kScanWarps][32], s_start[kScanWarps][32], s_bw[kScanWarps][32];
  __shared__ int64_t s_bin0[kScanWarps][32];
  __shared__ uint32_t s_low[kScanWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int64_t block_run = sums[blockIdx.x];
  // every round's element loads in flight before the first round's work
  int2 rad[kScanItems];
  float2 mu[kScanItems];
#pragma unroll
  for (int round = 0; round < kScanItems; ++round) {
    const int64_t i = base + (int64_t)round * kScanThreads + threadIdx.x;
    rad[round] = i < a.n ? __ldg(reinterpret_cast<const int2*>(a.radii) + i) : make_int2(0, 0);
    mu[round] = i < a.n ? __ldg(reinterpret_cast<const float2*>(a.means2d) + i)
                        : make_float2(0.0f, 0.0f);
  }
#pragma unroll
  for (int round = 0; round < kScanItems; ++round) {
    const int64_t i = base + (int64_t)round * kScanThreads + threadIdx.x;
    int c = 0;
    if (i < a.n) {
      const Rect q = band_rect(mu[round].x, mu[round].y, rad[round].x, rad[round].y, a.ts, a.tw,
                               a.th, a.ty0, a.ty1);
      c = rect_bins(q);
      if (c > 0) {
        const int64_t image = a.image_ids ? (int64_t)__ldg(a.image_ids + i) : i / a.n_per_image;
        rects[i] = pack_rect(q);
        const int bx0 = q.x0 / kBinTiles, by0 = q.y0 / kBinTiles;
        s_bw[warp][lane] = (q.x1 - 1) / kBinTiles - bx0 + 1;
        s_bin0[warp][lane] = image * a.n_bins_per_image + (int64_t)by0 * a.sw + bx0;
        s_low[warp][lane] = __float_as_uint(__ldg(a.depths + i)) & (0xFFFFFFFFu >> (32 - a.dbits));
      }
    }
    int64_t tot;
    const int64_t excl = block_exclusive_scan<kScanThreads>(c, s_warp, &tot);
    const int64_t excl0 = __shfl_sync(0xffffffffu, excl, 0);
    const int wexcl = (int)(excl - excl0);  // within the warp
    const int wtot = __shfl_sync(0xffffffffu, wexcl + c, 31);
    const int64_t wpos = block_run + excl0;
    s_pref[warp][lane] = wexcl;
    __syncwarp();
    int carry = 0;  // owner of the last entry of the previous window
    for (int j0 = 0; j0 < wtot; j0 += 32) {
      const bool st = c > 0 && wexcl >= j0 && wexcl < j0 + 32;
      if (st) s_start[warp][wexcl - j0] = lane;
      const uint32_t starts = __reduce_or_sync(0xffffffffu, st ? 1u << (wexcl - j0) : 0u);
      __syncwarp();
      const uint32_t upto = starts & (0xFFFFFFFFu >> (31 - lane));
      const int o = upto ? s_start[warp][31 - __clz(upto)] : carry;
      carry = __shfl_sync(0xffffffffu, o, 31);
      const int j = j0 + lane;
      if (j < wtot) {
        const int k = j - s_pref[warp][o];
        const int bw = s_bw[warp][o];
        const int dy = k / bw;
        const int64_t bin = s_bin0[warp][o] + (int64_t)dy * a.sw + (k - dy * bw);
        const int64_t pos = wpos + j;
        if (pos >= 0 && pos < n_entries) {
          keys[pos] = ((uint64_t)bin << a.dbits) | s_low[warp][o];
          vals[pos] = (int32_t)(base + (int64_t)round * kScanThreads + warp * 32 + o);
        }
      }
      __syncwarp();
    }
    block_run += tot;
  }
}

// One pass over the sorted entries: bin_start[b] = first entry of bin b
// (bins without entries point at the next one; bin_start[n_bins] =
// n_entries), and next to every entry the mask of its bin's tiles that it
// covers (empty for an element id outside [0, n), which only a wrong entry
// total can leave).  With conics and opacities (the culled encode) a tile
// leaves the mask when tile_may_hit proves that the Gaussian stays below
// alpha 1/255 at every pixel centre of the tile -- the rasterizer would skip
// it at each of them.
struct FinishArgs {
  int64_t n_entries, n, n_bins, per_image;
  int sw, dbits, ts;
  const uint64_t* keys;
  const int32_t* vals;
  const uint2* rects;
  const float* means2d;    // culled encode only
  const float* conics;     // null: no culling
  const float* opacities;
  int32_t opac_n;          // > 0: opacities are [opac_n], element e reads e mod opac_n
  int32_t* bin_start;
  uint32_t* masks;
};

__global__ void __launch_bounds__(256) bin_finish_kernel(const FinishArgs a) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < a.n_entries;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = (int64_t)(__ldg(a.keys + p) >> a.dbits);
    const int64_t bp = p > 0 ? (int64_t)(__ldg(a.keys + p - 1) >> a.dbits) : -1;
    for (int64_t q = bp + 1; q <= b && q <= a.n_bins; ++q) a.bin_start[q] = (int32_t)p;
    if (p == a.n_entries - 1)
      for (int64_t q = b + 1; q <= a.n_bins; ++q) a.bin_start[q] = (int32_t)a.n_entries;
    const int32_t e = __ldg(a.vals + p);
    uint32_t m = 0u;
    if (e >= 0 && e < a.n && b < a.n_bins) {
      const int64_t image = b / a.per_image;
      const int rem = (int)(b - image * a.per_image);
      const int tx0 = (rem % a.sw) * kBinTiles, ty0_ = (rem / a.sw) * kBinTiles;
      m = cover_mask(__ldg(a.rects + e), tx0, ty0_);
      if (a.conics && m) {
        const float2 mu = __ldg(reinterpret_cast<const float2*>(a.means2d) + e);
        const float c0 = __ldg(a.conics + (int64_t)e * 3), c1 = __ldg(a.conics + (int64_t)e * 3 + 1);
        const float c2 = __ldg(a.conics + (int64_t)e * 3 + 2), o = __ldg(a.opacities + (a.opac_n > 0 ? e % a.opac_n : e));
        m = bin_hit_mask(m, mu.x - ((float)(tx0 * a.ts) + 0.5f),
                         mu.y - ((float)(ty0_ * a.ts) + 0.5f), c0, c1, c2, o, a.ts);
      }
    }
    a.masks[p] = m;
  }
}

// Work items of the tile pass: a bin's sorted entries cut into chunks of
// kItemEntries.  Every item handles its bin's 16 tiles at once: per entry a
// 16-bit mask of the covered tiles, per tile counts packed four to a 64-bit
// word (16-bit fields: a CTA holds at most kItemEntries entries).
constexpr int kItemThreads = 256;
constexpr int kItemPer = 8;  // consecutive entries per thread
constexpr int kItemEntries = kItemThreads * kItemPer;

// chunks[b] = items of bin b.
__global__ void __launch_bounds__(256) bin_chunks_kernel(int64_t n_bins,
                                                         const int32_t* __restrict__ bin_start,
                                                         int32_t* __restrict__ chunks) {
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < n_bins;
       b += (int64_t)gridDim.x * blockDim.x) {
    const int len = __ldg(bin_start + b + 1) - __ldg(bin_start + b);
    chunks[b] = (len + kItemEntries - 1) / kItemEntries;
  }
}

// Bit t of a 16-bit mask to 16-bit field t of four words (tiles 4w..4w+3
// in word w).
__device__ __forceinline__ void spread16(uint32_t m, uint64_t f[4]) {
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint64_t x = (m >> (4 * w)) & 0xFu;
    x = (x | (x << 30)) & 0x0000000300000003ull;  // bits 2,3 -> bits 32,33
    x = (x | (x << 15)) & 0x0001000100010001ull;  // bits 1,33 -> bits 16,48
    f[w] = x;
  }
}

struct ItemArgs {
  int64_t n_bins, per_image;
  int sw, tw, ty0, rows, dbits;
  const int32_t* bin_start;
  const int32_t* chunk_prefix;  // exclusive prefix of the bins' item counts
  const int64_t* n_items;       // device total of items
  const uint32_t* masks;  // per sorted entry: the tiles of its bin it lands in
};

// The item of this CTA: its bin and its entries [lo, hi).  False past the
// device's item total.
__device__ __forceinline__ bool item_of(const ItemArgs& a, int64_t item, int64_t& bin, int& lo,
                                        int& hi) {
  if (item >= *a.n_items) return false;
  int64_t l = 0, h = a.n_bins;  // last bin whose prefix is <= item
  while (l < h) {
    const int64_t mid = l + (h - l) / 2;
    if (__ldg(a.chunk_prefix + mid) <= item) l = mid + 1;
    else h = mid;
  }
  bin = l - 1;
  const int chunk = (int)(item - __ldg(a.chunk_prefix + bin));
  const int b0 = __ldg(a.bin_start + bin), b1 = __ldg(a.bin_start + bin + 1);
  lo = b0 + chunk * kItemEntries;
  hi = lo + kItemEntries < b1 ? lo + kItemEntries : b1;
  return true;
}

__device__ __forceinline__ void bin_origin(const ItemArgs& a, int64_t bin, int64_t& image, int& tx0,
                                           int& ty0_) {
  image = bin / a.per_image;
  const int rem = (int)(bin - image * a.per_image);
  tx0 = (rem % a.sw) * kBinTiles;
  ty0_ = (rem / a.sw) * kBinTiles;
}

// Sums four packed words over the CTA: returns this thread's exclusive
// prefix; the CTA totals land in s_tot.
__device__ __forceinline__ void block_scan_packed(uint64_t v[4], uint64_t pre[4],
                                                  uint64_t (*s_w)[4], uint64_t* s_tot) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t inc[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    inc[w] = v[w];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t t = __shfl_up_sync(0xffffffffu, inc[w], o);
      if (lane >= o) inc[w] += t;
    }
    if (lane == 31) s_w[warp][w] = inc[w];
  }
  __syncthreads();
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint64_t before = 0, tot = 0;
#pragma unroll
    for (int k = 0; k < kItemThreads / 32; ++k) {
      const uint64_t x = s_w[k][w];
      before += k < warp ? x : 0;
      tot += x;
    }
    pre[w] = before + inc[w] - v[w];
    if (threadIdx.x == 0) s_tot[w] = tot;
  }
  __syncthreads();
}

// Count phase: item_counts[item][16] = entries of the item covering each
// of its bin's tiles.
__global__ void __launch_bounds__(kItemThreads) item_count_kernel(const ItemArgs a,
                                                                  int32_t* __restrict__ item_counts) {
  __shared__ uint64_t s_w[kItemThreads / 32][4];
  __shared__ uint64_t s_tot[4];
  int64_t bin;
  int lo, hi;
  if (!item_of(a, blockIdx.x, bin, lo, hi)) return;
  const int p0 = lo + threadIdx.x * kItemPer;
  uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
  for (int k = 0; k < kItemPer; ++k) {
    const int p = p0 + k;
    if (p < hi) {
      uint64_t f[4];
      spread16(__ldg(a.masks + p), f);
#pragma unroll
      for (int w = 0; w < 4; ++w) acc[w] += f[w];
    }
  }
  uint64_t pre[4];
  block_scan_packed(acc, pre, s_w, s_tot);
  if (threadIdx.x < 16)
    item_counts[(int64_t)blockIdx.x * 16 + threadIdx.x] =
        (int32_t)((s_tot[threadIdx.x >> 2] >> (16 * (threadIdx.x & 3))) & 0xFFFFu);
}

// Per tile slot: its intersection count, summed over its bin's items.
__global__ void __launch_bounds__(256) slot_count_kernel(const ItemArgs a, int64_t n_slots,
                                                         const int32_t* __restrict__ item_counts,
                                                         int32_t* __restrict__ counts) {
  const int64_t per_image_slots = (int64_t)a.rows * a.tw;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n_slots;
       s += (int64_t)gridDim.x * blockDim.x) {
    const int64_t image = s / per_image_slots;
    const int rem = (int)(s - image * per_image_slots);
    const int y = a.ty0 + rem / a.tw, x = rem % a.tw;
    const int64_t bin = image * a.per_image + (int64_t)(y / kBinTiles) * a.sw + x / kBinTiles;
    const int t = (y % kBinTiles) * kBinTiles + x % kBinTiles;
    const int i0 = __ldg(a.chunk_prefix + bin);
    const int i1 = bin + 1 < a.n_bins ? __ldg(a.chunk_prefix + bin + 1) : (int)*a.n_items;
    int32_t c = 0;
    for (int i = i0; i < i1; ++i) c += __ldg(item_counts + (int64_t)i * 16 + t);
    counts[s] = c;
  }
}

// Write phase: every entry of the item at its place in each tile it covers
// -- the tile's offset, the counts of the bin's earlier items, the covering
// entries before it in this item -- as the full key and the element id.
// Rounds of one entry per thread (consecutive entries on consecutive
// threads) and, within a round, tile by tile: the lanes that cover a tile
// store to consecutive places.  (Staging a round's copies tile-major in
// shared memory and storing them densely was slower: 64 KB per CTA.)
__global__ void __launch_bounds__(kItemThreads) item_write_kernel(
    const ItemArgs a, int tile_bits, const int32_t* __restrict__ item_counts,
    const int32_t* __restrict__ offsets, const uint64_t* __restrict__ keys,
    const int32_t* __restrict__ vals, int64_t n_isects, int64_t* __restrict__ isect_ids,
    int32_t* __restrict__ flatten_ids) {
  __shared__ uint64_t s_w[kItemThreads / 32][4];
  __shared__ uint64_t s_tot[4];
  __shared__ int64_t s_base[16];
  __shared__ uint32_t s_tile[16];  // image << tile_bits | tile id
  int64_t bin;
  int lo, hi;
  if (!item_of(a, blockIdx.x, bin, lo, hi)) return;
  int64_t image;
  int tx0, ty0_;
  bin_origin(a, bin, image, tx0, ty0_);
  if (threadIdx.x < 16) {
    const int t = threadIdx.x;
    const int x = tx0 + (t & 3), y = ty0_ + (t >> 2);
    int64_t base = 0;
    if (x < a.tw && y >= a.ty0 && y < a.ty0 + a.rows) {
      base = __ldg(offsets + image * a.rows * a.tw + (int64_t)(y - a.ty0) * a.tw + x);
      for (int i = __ldg(a.chunk_prefix + bin); i < (int)blockIdx.x; ++i)
        base += __ldg(item_counts + (int64_t)i * 16 + t);
    }
    s_base[t] = base;
    s_tile[t] = (uint32_t)((image << tile_bits) | ((int64_t)y * a.tw + x));
  }
  uint64_t run[4] = {0, 0, 0, 0};  // covering entries of earlier rounds, per tile
  for (int r = 0; r < kItemPer; ++r) {
    const int p = lo + r * kItemThreads + threadIdx.x;
    const uint32_t m = p < hi ? __ldg(a.masks + p) : 0u;
    uint64_t f[4], pre[4];
    spread16(m, f);
    block_scan_packed(f, pre, s_w, s_tot);  // the first also orders s_base / s_tile
    if (m) {
      const uint64_t low = __ldg(keys + p) & ((1ull << a.dbits) - 1ull);
      const int32_t e = __ldg(vals + p);
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        if ((m >> t) & 1u) {
          const int w = t >> 2, sh = 16 * (t & 3);
          const int64_t pos = s_base[t] + (int64_t)(((run[w] + pre[w]) >> sh) & 0xFFFFu);
          if (pos >= 0 && pos < n_isects) {
            isect_ids[pos] = (int64_t)(((uint64_t)s_tile[t] << 32) | low);
            flatten_ids[pos] = e;
          }
        }
      }
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) run[w] += s_tot[w];
    if (lo + (r + 1) * kItemThreads >= hi) break;  // uniform: the item's entries are done
  }
}

// ------------------------------------------------------------ offsets

// tile_offsets[o] = lower bound of key(o) = (image << tb) | tile in
// isect_ids >> 32, for the slots o of tile rows [ty0, ty0 + rows) of every
// image (the whole grid: ty0 = 0, rows = th): one thread per slot, binary
// search over the sorted keys, as the reference does
// (gsplat_intersect.cpp:605-641, metal :110-136).
__global__ void __launch_bounds__(256) offset_kernel(int64_t m, const int64_t* __restrict__ ids,
                                                     int I, int tw, int ty0, int rows, int tb,
                                                     int32_t* __restrict__ offsets) {
  const int64_t per_image = (int64_t)rows * tw;
  const int64_t n_off = (int64_t)I * per_image;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < n_off;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t image = o / per_image;
    const int64_t tile = (int64_t)ty0 * tw + (o - image * per_image);
    const int64_t key = (image << tb) | tile;
    int64_t lo = 0, hi = m;
    while (lo < hi) {
      const int64_t mid = lo + (hi - lo) / 2;
      if ((__ldg(ids + mid) >> 32) < key) lo = mid + 1;
      else hi = mid;
    }
    offsets[o] = (int32_t)lo;
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

// The tile-row window of the call: the whole grid unless tile_y1 > tile_y0.
static void tile_rows(const gs_isect_params* p, int& ty0, int& ty1) {
  ty0 = 0;
  ty1 = p->tile_height;
  if (p->tile_y1 > p->tile_y0) {
    ty0 = p->tile_y0 < 0 ? 0 : (p->tile_y0 > p->tile_height ? p->tile_height : p->tile_y0);
    ty1 = p->tile_y1 > p->tile_height ? p->tile_height : p->tile_y1;
  }
}

static int check_isect(const gs_isect_params* p) {
  if (!p) return invalid("intersect: params missing");
  if (p->I <= 0 || p->N < 0 || (int64_t)p->I * p->N > INT32_MAX)
    return invalid("intersect_tile_count dense path expects depths size to equal I * N.");
  if (p->tile_size <= 0 || p->tile_width <= 0 || p->tile_height <= 0)
    return invalid("intersect expects positive image/tile counts.");
  return GS_OK;
}

extern "C" int gs_isect_tile_count(const gs_isect_params* p, const float* means2d,
                                   const int32_t* radii, int32_t* tiles_per_gauss,
                                   gs_stream_t stream) {
  if (int rc = check_isect(p)) return rc;
  const int64_t n = (int64_t)p->I * p->N;
  if (n == 0) return GS_OK;
  if (!means2d || !radii || !tiles_per_gauss) return invalid("intersect_tile_count: missing buffer");
  int ty0, ty1;
  tile_rows(p, ty0, ty1);
  count_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
      n, means2d, radii, p->tile_size, p->tile_width, p->tile_height, ty0, ty1, tiles_per_gauss,
      nullptr, 0);
  return launch_status("intersect_tile_count");
}

extern "C" int gs_isect_tile_count_total(const gs_isect_params* p, const float* means2d,
                                         const int32_t* radii, int32_t* tiles_per_gauss,
                                         int64_t* total_device, gs_stream_t stream) {
  if (int rc = check_isect(p)) return rc;
  if (!total_device) return invalid("intersect_tile_count_total: missing total");
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(total_device, 0, sizeof(int64_t), s) != cudaSuccess)
    return launch_status("intersect_tile_count_total");
  const int64_t n = (int64_t)p->I * p->N;
  if (n == 0) return GS_OK;
  if (!means2d || !radii || !tiles_per_gauss)
    return invalid("intersect_tile_count_total: missing buffer");
  int ty0, ty1;
  tile_rows(p, ty0, ty1);
  count_kernel<<<grid_for(n, 256), 256, 0, s>>>(n, means2d, radii, p->tile_size, p->tile_width,
                                                  p->tile_height, ty0, ty1, tiles_per_gauss,
                                                  reinterpret_cast<unsigned long long*>(total_device),
                                                  0);
  return launch_status("intersect_tile_count_total");
}

extern "C" size_t gs_isect_scan_workspace_size(int64_t n) { return scan_ws_bytes(n); }

extern "C" int gs_isect_scan(int64_t n, const int32_t* counts, int32_t* offsets,
                             int64_t* total_device, void* workspace, size_t workspace_bytes,
                             gs_stream_t stream) {
  if (n < 0) return invalid("intersect_tile_offsets: negative size");
  if (n > 0 && (!counts || !offsets)) return invalid("intersect_tile_offsets: missing buffer");
  return scan_i32(n, counts, offsets, total_device, workspace, workspace_bytes, as_stream(stream));
}

extern "C" int gs_isect_tile_encode(const gs_isect_params* p, const float* means2d,
                                    const int32_t* radii, const float* depths,
                                    const int32_t* offsets, int64_t n_isects, int64_t* isect_ids,
                                    int32_t* flatten_ids, gs_stream_t stream) {
  if (int rc = check_isect(p)) return rc;
  if (n_isects < 0) return invalid("intersect_tile_encode expects non-negative total_isects.");
  if (n_isects > INT32_MAX) {
    set_error("intersect_tile_encode: %lld intersections exceed the int32 offsets", (long long)n_isects);
    return GS_ERR_OVERFLOW;
  }
  const int n_tiles = p->tile_width * p->tile_height;
  const int tile_bits = gs_floor_log2_plus_one(n_tiles);
  const int image_bits = gs_floor_log2_plus_one(p->I);
  if (image_bits + tile_bits > 32)
    return invalid("intersect_tile_encode image id and tile id require more than 32 bits.");
  const int64_t n = (int64_t)p->I * p->N;
  if (n == 0 || n_isects == 0) return GS_OK;
  if (!means2d || !radii || !depths || !offsets || !isect_ids || !flatten_ids)
    return invalid("intersect_tile_encode: missing buffer");
  int ty0, ty1;
  tile_rows(p, ty0, ty1);
  encode_kernel<<<grid_for((n + 31) / 32, kEncodeWarps), kEncodeThreads, 0, as_stream(stream)>>>(
      n, p->N, means2d, radii, depths, offsets, p->tile_size, p->tile_width,
      p->tile_height, ty0, ty1, tile_bits, n_isects, isect_ids, flatten_ids, nullptr, nullptr, 0, 0u);
  return launch_status("intersect_tile_encode");
}

extern "C" size_t gs_isect_tile_encode_sorted_workspace_size(int64_t n_elements,
                                                            int64_t n_isects) {
  return sorted_encode_layout(n_elements, n_isects).total;
}

// Depth-first sorted encode: the visible elements (i, n) are first put in
// stable order of their depth bits (4 radix passes over them), the
// intersections are then encoded in that order, and a stable sort over the
// key bits above the depth word (tile and image: 2 passes at 1297x840)
// finishes the job.  Within one (image, tile) the order is by depth bits,
// then by element index -- exactly the stable order of the full 64-bit key
// over the reference's encode order, because an element meets each tile at
// most once.
extern "C" int gs_isect_tile_encode_sorted(const gs_isect_params* p, const float* means2d,
                                           const int32_t* radii, const float* depths,
                                           const int32_t* tiles_per_gauss, int64_t n_isects,
                                           int64_t* isect_ids, int32_t* flatten_ids,
                                           void* workspace, size_t workspace_bytes,
                                           gs_stream_t stream) {
  if (int rc = check_isect(p)) return rc;
  if (n_isects < 0) return invalid("intersect_tile_encode expects non-negative total_isects.");
  if (n_isects > INT32_MAX) {
    set_error("intersect_tile_encode: %lld intersections exceed the int32 offsets", (long long)n_isects);
    return GS_ERR_OVERFLOW;
  }
  const int n_tiles = p->tile_width * p->tile_height;
  const int tile_bits = gs_floor_log2_plus_one(n_tiles);
  const int image_bits = gs_floor_log2_plus_one(p->I);
  if (image_bits + tile_bits > 32)
    return invalid("intersect_tile_encode image id and tile id require more than 32 bits.");
  const int64_t n = (int64_t)p->I * p->N;
  if (n == 0 || n_isects == 0) return GS_OK;
  if (!means2d || !radii || !depths || !tiles_per_gauss || !isect_ids || !flatten_ids)
    return invalid("intersect_tile_encode_sorted: missing buffer");
  const SortedEncodeLayout L = sorted_encode_layout(n, n_isects);
  if (!workspace || workspace_bytes < L.total) {
    set_error("intersect_tile_encode_sorted: workspace of %zu bytes needed", L.total);
    return GS_ERR_WORKSPACE;
  }
  cudaStream_t s = as_stream(stream);
  char* ws = static_cast<char*>(workspace);
  cudaMemsetAsync(ws + L.sort + sort_layout(1).err, 0, sizeof(uint32_t), s);
  auto K = [&](size_t off) { return reinterpret_cast<uint64_t*>(ws + off); };
  auto V = [&](size_t off) { return reinterpret_cast<int32_t*>(ws + off); };
  int64_t* n_vis = reinterpret_cast<int64_t*>(ws + L.nvis);
  if (!p->reuse_depth_order) {
    // only the visible elements take part in the depth order; their count
    // stays on the device and bounds the passes and the scan below
    const int64_t nb = ceil_div(n, kScanChunk);
    int64_t* sums = reinterpret_cast<int64_t*>(ws + L.scan);
    visible_count_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(n, radii, sums);
    scan_sums_kernel<<<1, 1024, 0, s>>>(nb, sums, n_vis);
    visible_depth_keys_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(n, radii, depths, sums,
                                                                     K(L.ek));
    // the depth bits are the low key word: unsigned order
    sort_passes(n, 32, 64, kPacked, kPacked, K(L.ek), nullptr, K(L.pk), nullptr, ws + L.sort, s,
                false, n_vis, nullptr, /*signed_keys=*/false);
  }
  // element of each depth-ordered place: the low words of the sorted words
  const int32_t* perm = V(L.pk);
  if (int rc = scan_i32(n, tiles_per_gauss, V(L.offs), nullptr, ws + L.scan, scan_ws_bytes(n), s,
                        perm, 2, n_vis))
    return rc;
  // V(L.offs)[e] is now element e's offset in depth order; encoding in
  // element order keeps the warps' work as balanced as the plain encode
  // (depth order would cluster the large near-camera footprints).
  // The encode also counts the digits of the tile/image passes.
  const int hb = tile_bits + image_bits;
  uint32_t* hist = radix_reset(n_isects, ws + L.sort, s);
  int ty0, ty1;
  tile_rows(p, ty0, ty1);
  encode_kernel<<<grid_for((n + 31) / 32, kEncodeWarps), kEncodeThreads, 0, s>>>(
      n, p->N, means2d, radii, depths, V(L.offs), p->tile_size, p->tile_width,
      p->tile_height, ty0, ty1, tile_bits, n_isects, nullptr, nullptr, K(L.dk), hist, (hb + 7) / 8,
      hb == 32 ? 0x80000000u : 0u);  // keys with the sign bit set sort first
  // the passes move (high word << 32 | element) words; the last one writes
  // the full keys (depth bits gathered) and the element ids
  sort_passes(n_isects, 32, 32 + hb, kPacked, kFinal, K(L.dk), nullptr,
              reinterpret_cast<uint64_t*>(isect_ids), flatten_ids, ws + L.sort, s,
              /*hist_ready=*/true, nullptr, depths);
  return launch_status("intersect_tile_encode_sorted");
}

extern "C" size_t gs_isect_sort_workspace_size(int64_t n_isects) {
  return sort_layout(n_isects).total;
}

extern "C" int gs_isect_sort(int64_t n, int32_t key_bits, const int64_t* isect_ids,
                             const int32_t* flatten_ids, int64_t* sorted_isect_ids,
                             int32_t* sorted_flatten_ids, void* workspace, size_t workspace_bytes,
                             gs_stream_t stream) {
  if (n < 0 || key_bits < 1 || key_bits > 64) return invalid("intersect_tile_sort: bad arguments");
  if (n > INT32_MAX) return invalid("intersect_tile_sort: more than 2^31 intersections");
  if (n == 0) return GS_OK;
  if (!isect_ids || !flatten_ids || !sorted_isect_ids || !sorted_flatten_ids)
    return invalid("intersect_tile_sort: missing buffer");
  const SortLayout L = sort_layout(n);
  if (!workspace || workspace_bytes < L.total) {
    set_error("intersect_tile_sort: workspace of %zu bytes needed", L.total);
    return GS_ERR_WORKSPACE;
  }
  cudaStream_t s = as_stream(stream);
  char* ws = static_cast<char*>(workspace);
  cudaMemsetAsync(ws + L.err, 0, sizeof(uint32_t), s);
  radix_passes(n, 0, key_bits, reinterpret_cast<const uint64_t*>(isect_ids), flatten_ids,
               reinterpret_cast<uint64_t*>(sorted_isect_ids), sorted_flatten_ids,
               ws, s);
  return launch_status("intersect_tile_sort");
}

// The look-back error word of the last sort that used `ws` with n keys:
// waits for `stream`, then GS_OK, or GS_ERR_DEVICE when a bounded wait gave up.
static int read_sort_error(int64_t n, const char* ws, cudaStream_t s) {
  const SortLayout L = sort_layout(n);
  uint32_t word = 0;
  if (cudaMemcpyAsync(&word, ws + L.err, sizeof(word), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return launch_status("intersect sort check");
  if (word) {
    set_error("intersect sort: a look-back wait gave up; the sorted output is invalid");
    return GS_ERR_DEVICE;
  }
  return GS_OK;
}

extern "C" int gs_isect_sort_check(int64_t n_isects, const void* workspace, gs_stream_t stream) {
  if (n_isects <= 0) return GS_OK;
  if (!workspace) return invalid("intersect_tile_sort_check: missing workspace");
  return read_sort_error(n_isects, static_cast<const char*>(workspace), as_stream(stream));
}

extern "C" int gs_isect_tile_encode_sorted_check(int64_t n_elements, int64_t n_isects,
                                                 const void* workspace, gs_stream_t stream) {
  if (n_elements <= 0 || n_isects <= 0) return GS_OK;
  if (!workspace) return invalid("intersect_tile_encode_sorted_check: missing workspace");
  const SortedEncodeLayout L = sorted_encode_layout(n_elements, n_isects);
  // one error word serves the depth passes and the tile passes
  return read_sort_error(n_isects, static_cast<const char*>(workspace) + L.sort,
                         as_stream(stream));
}

// n int64 values from device memory to pinned host memory by one warp's
// stores through the host mapping (no copy engine).
__global__ void store_i64_kernel(const int64_t* __restrict__ src, int64_t* __restrict__ dst, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

// A small device-to-host read that must not queue behind large transfers:
// a cudaMemcpyAsync to host runs on a copy engine, where it can wait for
// another stream's download of hundreds of MB; a kernel storing into the
// pinned buffer's device mapping does not.  Falls back to cudaMemcpyAsync
// when host_dst has no device mapping.
extern "C" int gs_store_to_host_i64(const int64_t* src, int64_t* host_dst, int32_t n,
                                    gs_stream_t stream) {
  if (n < 0 || n > 1024 || (n > 0 && (!src || !host_dst)))
    return invalid("store_to_host_i64: bad arguments");
  if (n == 0) return GS_OK;
  cudaStream_t s = as_stream(stream);
  void* mapped = nullptr;
  if (cudaHostGetDevicePointer(&mapped, host_dst, 0) != cudaSuccess || !mapped) {
    cudaGetLastError();  // clear the lookup's error: not a mapped host buffer
    if (cudaMemcpyAsync(host_dst, src, sizeof(int64_t) * (size_t)n, cudaMemcpyDeviceToHost, s) !=
        cudaSuccess)
      return launch_status("store_to_host_i64");
    return GS_OK;
  }
  store_i64_kernel<<<1, 32, 0, s>>>(src, static_cast<int64_t*>(mapped), n);
  return launch_status("store_to_host_i64");
}

extern "C" int gs_isect_tile_count_totals(const gs_isect_params* p, const float* means2d,
                                          const int32_t* radii, int32_t* tiles_per_gauss,
                                          int64_t* totals_device, gs_stream_t stream) {
  if (int rc = check_isect(p)) return rc;
  if (!totals_device) return invalid("intersect_tile_count_totals: missing totals");
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(totals_device, 0, 2 * sizeof(int64_t), s) != cudaSuccess)
    return launch_status("intersect_tile_count_totals");
  const int64_t n = (int64_t)p->I * p->N;
  if (n == 0) return GS_OK;
  if (!means2d || !radii || !tiles_per_gauss)
    return invalid("intersect_tile_count_totals: missing buffer");
  int ty0, ty1;
  tile_rows(p, ty0, ty1);
  count_kernel<<<grid_for(n, 256), 256, 0, s>>>(n, means2d, radii, p->tile_size, p->tile_width,
                                                  p->tile_height, ty0, ty1, tiles_per_gauss,
                                                  reinterpret_cast<unsigned long long*>(totals_device),
                                                  1);
  return launch_status("intersect_tile_count_totals");
}

// Bins of the binned encode and their key bits.
struct BinGeom {
  int sw, sh;
  int64_t per_image, total;
  int bits;
};

static BinGeom bin_geom(const gs_isect_params* p) {
  BinGeom g;
  g.sw = (int)ceil_div(p->tile_width, kBinTiles);
  g.sh = (int)ceil_div(p->tile_height, kBinTiles);
  g.per_image = (int64_t)g.sw * g.sh;
  g.total = (int64_t)p->I * g.per_image;
  g.bits = g.total > 1 ? 64 - __builtin_clzll((unsigned long long)(g.total - 1)) : 0;
  return g;
}

// Workspace of the binned encode; the sort scratch comes first, so that its
// error word sits at offset 0.
struct BinnedLayout {
  size_t sort, nent, nitems, nkept, keys, vals, skeys, svals, rects, masks, bstart, chunks, cprefix,
      icounts, counts, offs, scan, total;
  int64_t items;  // bound on the work items
};

// packed: the elements are N packed rows (with their own image ids), not
// I * N.
static BinnedLayout binned_layout(const gs_isect_params* p, int64_t n_entries,
                                  bool packed = false) {
  int ty0, ty1;
  tile_rows(p, ty0, ty1);
  const BinGeom g = bin_geom(p);
  const int64_t n = packed ? (int64_t)p->N : (int64_t)p->I * p->N;
  const int64_t slots = (int64_t)p->I * (ty1 - ty0) * p->tile_width;
  const int64_t e1 = n_entries < 1 ? 1 : n_entries, n1 = n < 1 ? 1 : n;
  BinnedLayout L;
  size_t o = 0;
  L.sort = o; o += sort_layout(e1).total;
  L.nent = o; o += 256;
  L.nkept = o; o += 256;
  L.keys = o; o += align256(8 * (size_t)e1);
  L.vals = o; o += align256(4 * (size_t)e1);
  L.skeys = o; o += align256(8 * (size_t)e1);
  L.svals = o; o += align256(4 * (size_t)e1);
  L.rects = o; o += align256(8 * (size_t)n1);
  L.masks = o; o += align256(4 * (size_t)e1);
  L.items = ceil_div(e1, kItemEntries) + g.total;
  L.nitems = o; o += 256;
  L.bstart = o; o += align256(4 * (size_t)(g.total + 1));
  L.chunks = o; o += align256(4 * (size_t)g.total);
  L.cprefix = o; o += align256(4 * (size_t)g.total);
  L.icounts = o; o += align256(64 * (size_t)L.items);
  L.counts = o; o += align256(4 * (size_t)(slots < 1 ? 1 : slots));
  L.offs = o; o += align256(4 * (size_t)(slots < 1 ? 1 : slots));
  L.scan = o;
  o += std::max(std::max(scan_ws_bytes(n1), scan_ws_bytes(slots < 1 ? 1 : slots)),
                scan_ws_bytes(g.total));
  L.total = o;
  return L;
}

extern "C" size_t gs_isect_tile_encode_binned_workspace_size(const gs_isect_params* p,
                                                            int64_t n_bin_entries) {
  if (!p || check_isect(p) != GS_OK) return 0;
  return binned_layout(p, n_bin_entries).total;
}

// offsets[s] += n_isects - kept: the culled lists end at n_isects.
__global__ void __launch_bounds__(256) offsets_gap_kernel(int64_t slots, int64_t n_isects,
                                                          const int64_t* __restrict__ kept,
                                                          int32_t* __restrict__ offsets) {
  const int32_t gap = (int32_t)(n_isects - *kept);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < slots;
       i += (int64_t)gridDim.x * blockDim.x)
    offsets[i] += gap;
}

// Binned sorted encode (see the kernels above): the same isect_ids /
// flatten_ids as the encode followed by the stable 64-bit key sort, plus
// the tile offsets of the call's tile rows when tile_offsets is given.
// n_bin_entries is the second total of gs_isect_tile_count_totals.  With
// conics the tile-culled form (gs_isect_tile_encode_binned_culled).
static int encode_binned(const gs_isect_params* p, const int32_t* image_ids,
                         const float* means2d, const int32_t* radii,
                         const float* depths, const float* conics, const float* opacities,
                         int64_t n_isects, int64_t n_bin_entries, int64_t* isect_ids,
                         int32_t* flatten_ids, int32_t* tile_offsets, int64_t* n_kept,
                         void* workspace, size_t workspace_bytes, gs_stream_t stream) {
  if (int rc = check_isect(p)) return rc;
  if (n_isects < 0 || n_bin_entries < 0 || n_bin_entries > n_isects)
    return invalid("intersect_tile_encode_binned: bad intersection / bin entry totals");
  if (n_isects > INT32_MAX) {
    set_error("intersect_tile_encode: %lld intersections exceed the int32 offsets", (long long)n_isects);
    return GS_ERR_OVERFLOW;
  }
  const int n_tiles = p->tile_width * p->tile_height;
  const int tile_bits = gs_floor_log2_plus_one(n_tiles);
  const int image_bits = gs_floor_log2_plus_one(p->I);
  if (image_bits + tile_bits > 32)
    return invalid("intersect_tile_encode image id and tile id require more than 32 bits.");
  if (p->tile_width > 65535 || p->tile_height > 65535)
    return invalid("intersect_tile_encode_binned: more than 65535 tiles per row or column "
                   "(use gs_isect_tile_encode_sorted)");
  int ty0, ty1;
  tile_rows(p, ty0, ty1);
  const int rows = ty1 - ty0;
  const int64_t slots = (int64_t)p->I * rows * p->tile_width;
  cudaStream_t s = as_stream(stream);
  const int64_t n = image_ids ? (int64_t)p->N : (int64_t)p->I * p->N;
  if (n == 0 || n_isects == 0) {
    if (tile_offsets && slots > 0 &&
        cudaMemsetAsync(tile_offsets, 0, sizeof(int32_t) * (size_t)slots, s) != cudaSuccess)
      return launch_status("intersect_tile_encode_binned");
    if (n_kept && cudaMemsetAsync(n_kept, 0, sizeof(int64_t), s) != cudaSuccess)
      return launch_status("intersect_tile_encode_binned");
    return GS_OK;
  }
  if (!means2d || !radii || !depths || !isect_ids || !flatten_ids)
    return invalid("intersect_tile_encode_binned: missing buffer");
  const BinnedLayout L = binned_layout(p, n_bin_entries, image_ids != nullptr);
  if (!workspace || workspace_bytes < L.total) {
    set_error("intersect_tile_encode_binned: workspace of %zu bytes needed", L.total);
    return GS_ERR_WORKSPACE;
  }
  char* ws = static_cast<char*>(workspace);
  const BinGeom g = bin_geom(p);
  auto K = [&](size_t off) { return reinterpret_cast<uint64_t*>(ws + off); };
  auto V = [&](size_t off) { return reinterpret_cast<int32_t*>(ws + off); };
  auto R = [&](size_t off) { return reinterpret_cast<uint2*>(ws + off); };
  cudaMemsetAsync(ws + L.sort + sort_layout(1).err, 0, sizeof(uint32_t), s);
  // with positive depths the key's depth field drops the (clear) sign bit:
  // 31 + bin bits, one radix pass fewer when that crosses a multiple of 8
  const int dbits = p->positive_depths ? 31 : 32;
  BinArgs a{n, p->N, p->tile_size, p->tile_width, p->tile_height, ty0, ty1,
            g.sw, (int)g.per_image, dbits, means2d, radii, depths, image_ids};
  const int64_t nb = ceil_div(n, kScanChunk);
  const size_t scan_bytes = L.total - L.scan;
  int64_t* sums = reinterpret_cast<int64_t*>(ws + L.scan);
  bin_count_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(a, sums);
  scan_sums_kernel<<<1, 1024, 0, s>>>(nb, sums, reinterpret_cast<int64_t*>(ws + L.nent));
  bin_emit_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(a, sums, n_bin_entries, K(L.keys),
                                                        V(L.vals), R(L.rects));
  if (n_bin_entries > 0) {
    // the depth bits are the low key field and bin ids are unsigned
    sort_passes(n_bin_entries, 0, dbits + g.bits, kKV, kKV, K(L.keys), V(L.vals), K(L.skeys),
                V(L.svals), ws + L.sort, s, false, nullptr, nullptr, /*signed_keys=*/false);
    const FinishArgs fa{n_bin_entries, n, g.total, g.per_image, g.sw, dbits, p->tile_size,
                        K(L.skeys), V(L.svals), R(L.rects), means2d, conics, opacities,
                        p->shared_opacities ? p->N : 0, V(L.bstart),
                        reinterpret_cast<uint32_t*>(ws + L.masks)};
    bin_finish_kernel<<<grid_for(n_bin_entries, 256), 256, 0, s>>>(fa);
  } else {
    cudaMemsetAsync(ws + L.bstart, 0, 4 * (size_t)(g.total + 1), s);
  }
  // work items: bins cut into chunks
  bin_chunks_kernel<<<grid_for(g.total, 256), 256, 0, s>>>(g.total, V(L.bstart), V(L.chunks));
  int64_t* n_items = reinterpret_cast<int64_t*>(ws + L.nitems);
  if (int rc = scan_i32(g.total, V(L.chunks), V(L.cprefix), n_items, ws + L.scan, scan_bytes, s))
    return rc;
  ItemArgs ia{g.total, g.per_image, g.sw, p->tile_width, ty0, rows, dbits,
              V(L.bstart), V(L.cprefix), n_items, reinterpret_cast<const uint32_t*>(ws + L.masks)};
  item_count_kernel<<<(unsigned)L.items, kItemThreads, 0, s>>>(ia, V(L.icounts));
  int32_t* offs = tile_offsets ? tile_offsets : V(L.offs);
  int64_t* kept = n_kept ? n_kept : reinterpret_cast<int64_t*>(ws + L.nkept);
  if (slots > 0) {
    slot_count_kernel<<<grid_for(slots, 256), 256, 0, s>>>(ia, slots, V(L.icounts), V(L.counts));
    if (int rc = scan_i32(slots, V(L.counts), offs, conics ? kept : nullptr, ws + L.scan,
                          scan_bytes, s))
      return rc;
    if (conics)  // the culled lists take the last `kept` places
      offsets_gap_kernel<<<grid_for(slots, 256), 256, 0, s>>>(slots, n_isects, kept, offs);
  } else if (conics && cudaMemsetAsync(kept, 0, sizeof(int64_t), s) != cudaSuccess) {
    return launch_status("intersect_tile_encode_binned");
  }

  item_write_kernel<<<(unsigned)L.items, kItemThreads, 0, s>>>(
      ia, tile_bits, V(L.icounts), offs, K(L.skeys), V(L.svals), n_isects, isect_ids, flatten_ids);
  return launch_status("intersect_tile_encode_binned");
}

extern "C" int gs_isect_tile_encode_binned(const gs_isect_params* p, const float* means2d,
                                           const int32_t* radii, const float* depths,
                                           int64_t n_isects, int64_t n_bin_entries,
                                           int64_t* isect_ids, int32_t* flatten_ids,
                                           int32_t* tile_offsets, void* workspace,
                                           size_t workspace_bytes, gs_stream_t stream) {
  return encode_binned(p, nullptr, means2d, radii, depths, nullptr, nullptr, n_isects,
                       n_bin_entries,
                       isect_ids, flatten_ids, tile_offsets, nullptr, workspace, workspace_bytes,
                       stream);
}

extern "C" int gs_isect_tile_encode_binned_culled(
    const gs_isect_params* p, const float* means2d, const int32_t* radii, const float* depths,
    const float* conics, const float* opacities, int64_t n_isects, int64_t n_bin_entries,
    int64_t* isect_ids, int32_t* flatten_ids, int32_t* tile_offsets, int64_t* n_kept,
    void* workspace, size_t workspace_bytes, gs_stream_t stream) {
  if (!conics || !opacities)
    return invalid("intersect_tile_encode_binned_culled: conics and opacities are required");
  return encode_binned(p, nullptr, means2d, radii, depths, conics, opacities, n_isects,
                       n_bin_entries,
                       isect_ids, flatten_ids, tile_offsets, n_kept, workspace, workspace_bytes,
                       stream);
}

extern "C" size_t gs_isect_tile_encode_binned_packed_workspace_size(const gs_isect_params* p,
                                                                   int64_t n_bin_entries) {
  if (!p || check_isect(p) != GS_OK) return 0;
  return binned_layout(p, n_bin_entries, true).total;
}

extern "C" int gs_isect_tile_encode_binned_packed(
    const gs_isect_params* p, const int32_t* image_ids, const float* means2d,
    const int32_t* radii, const float* depths, int64_t n_isects, int64_t n_bin_entries,
    int64_t* isect_ids, int32_t* flatten_ids, int32_t* tile_offsets, void* workspace,
    size_t workspace_bytes, gs_stream_t stream) {
  if (p && p->N > 0 && !image_ids)
    return invalid("intersect_tile_encode_binned_packed: image_ids required");
  // (no rows: image_ids may be null; the plain element count I * 0 is 0 too)
  return encode_binned(p, image_ids, means2d,
                       radii, depths, nullptr, nullptr, n_isects, n_bin_entries, isect_ids,
                       flatten_ids, tile_offsets, nullptr, workspace, workspace_bytes, stream);
}

extern "C" size_t gs_pack_visible_workspace_size(int64_t n_elements) {
  return n_elements <= 0 ? 256 : align256(8 * (size_t)ceil_div(n_elements, kScanChunk)) + 256;
}

extern "C" int gs_pack_visible(int64_t n_elements, int32_t N, const int32_t* radii,
                               const float* means2d, const float* depths, const float* conics,
                               const float* compensations, int64_t capacity, int32_t* image_ids,
                               int32_t* gaussian_ids, int32_t* p_radii, float* p_means2d,
                               float* p_depths, float* p_conics, float* p_compensations,
                               int64_t* nnz_device, void* workspace, size_t workspace_bytes,
                               gs_stream_t stream) {
  if (n_elements < 0 || N <= 0 || (n_elements % N) != 0 || capacity < 0 || !nnz_device)
    return invalid("pack_visible: bad sizes");
  cudaStream_t s = as_stream(stream);
  if (n_elements == 0) {
    if (cudaMemsetAsync(nnz_device, 0, sizeof(int64_t), s) != cudaSuccess)
      return launch_status("pack_visible");
    return GS_OK;
  }
  if (!radii || !means2d || !depths || !conics ||
      (capacity > 0 && (!image_ids || !gaussian_ids || !p_radii || !p_means2d || !p_depths ||
                        !p_conics || (compensations && !p_compensations))))
    return invalid("pack_visible: missing buffer");
  if (!workspace || workspace_bytes < gs_pack_visible_workspace_size(n_elements)) {
    set_error("pack_visible: workspace of %zu bytes needed",
              gs_pack_visible_workspace_size(n_elements));
    return GS_ERR_WORKSPACE;
  }
  const int64_t nb = ceil_div(n_elements, kScanChunk);
  int64_t* sums = static_cast<int64_t*>(workspace);
  visible_count_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(n_elements, radii, sums);
  scan_sums_kernel<<<1, 1024, 0, s>>>(nb, sums, nnz_device);
  const PackArgs a{n_elements, capacity, N, radii, means2d, depths, conics,
                   compensations, image_ids, gaussian_ids, p_radii, p_means2d, p_depths,
                   p_conics, compensations ? p_compensations : nullptr};
  pack_rows_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(a, sums);
  return launch_status("pack_visible");
}

extern "C" int gs_isect_tile_encode_binned_check(int64_t n_bin_entries, const void* workspace,
                                                 gs_stream_t stream) {
  if (n_bin_entries <= 0) return GS_OK;
  if (!workspace) return invalid("intersect_tile_encode_binned_check: missing workspace");
  // the sort scratch starts the workspace
  return read_sort_error(n_bin_entries, static_cast<const char*>(workspace), as_stream(stream));
}

extern "C" int gs_isect_offset_rows(int64_t n_isects, const int64_t* isect_ids, int32_t I,
                                    int32_t tile_width, int32_t tile_height, int32_t tile_y0,
                                    int32_t tile_y1, int32_t* tile_offsets, gs_stream_t stream) {
  if (I <= 0 || tile_width <= 0 || tile_height <= 0)
    return invalid("intersect_offset expects positive image and tile dimensions.");
  if (n_isects < 0 || n_isects > INT32_MAX) return invalid("intersect_offset: bad n_isects");
  if (tile_y0 < 0 || tile_y1 > tile_height || tile_y1 <= tile_y0)
    return invalid("intersect_offset: bad tile-row window");
  const int T = tile_width * tile_height;
  const int tb = gs_floor_log2_plus_one(T);
  if (!tile_offsets || (n_isects > 0 && !isect_ids)) return invalid("intersect_offset: missing buffer");
  const int rows = tile_y1 - tile_y0;
  offset_kernel<<<grid_for((int64_t)I * rows * tile_width, 256), 256, 0, as_stream(stream)>>>(
      n_isects, isect_ids, I, tile_width, tile_y0, rows, tb, tile_offsets);
  return launch_status("intersect_offset");
}

extern "C" int gs_isect_offset(int64_t n_isects, const int64_t* isect_ids, int32_t I,
                               int32_t tile_width, int32_t tile_height, int32_t* tile_offsets,
                               gs_stream_t stream) {
  return gs_isect_offset_rows(n_isects, isect_ids, I, tile_width, tile_height, 0, tile_height,
                              tile_offsets, stream);
}

// ------------------------------------------------------------ no-alloc sort
// Some callers may not allocate device memory at all while they run -- a host
// engine that plans every device buffer up front and hands plugins only their
// inputs and outputs, or a latency-bound loop where an allocation could fail
// or stall.  For them the sort below takes its scratch from one fixed
// file-scope device array instead of a caller workspace.  The array is part of
// this library's module: every GPU that loads the library holds it until the
// process exits, so it is kept modest and caps the problem size.

#include <mutex>

namespace {
constexpr int64_t kNoAllocMaxIsects = int64_t(1) << 20;  // 1,048,576 intersections
constexpr size_t kNoAllocScratchBytes = size_t(13) << 20;  // 13 MiB
static __device__ __align__(256) unsigned char g_noalloc_sort_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_scratch_ptr[64] = {};  // device address of the array, per device
}  // namespace

extern "C" int gs_isect_sort_noalloc(int64_t n_isects, int32_t key_bits,
                                     const int64_t* isect_ids, const int32_t* flatten_ids,
                                     int64_t* sorted_isect_ids, int32_t* sorted_flatten_ids,
                                     gs_stream_t stream) {
  if (n_isects > kNoAllocMaxIsects) {
    set_error("intersect_tile_sort_noalloc: %lld intersections exceed its fixed scratch "
              "(at most %lld)", (long long)n_isects, (long long)kNoAllocMaxIsects);
    return GS_ERR_INVALID;
  }
  if (n_isects < 0) return invalid("intersect_tile_sort_noalloc: negative size");
  if (sort_layout(n_isects).total > kNoAllocScratchBytes)
    return invalid("intersect_tile_sort_noalloc: scratch layout exceeds the fixed array");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return invalid("intersect_tile_sort_noalloc: no usable current device");
  }
  void* scratch = nullptr;
  {
    // Host code cannot use the array's name as a device address; look the
    // address up once per device, with that device current.
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_sort_scratch);
      if (e != cudaSuccess || p == nullptr) {
        set_error("intersect_tile_sort_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
        return GS_ERR_CUDA;
      }
      g_noalloc_scratch_ptr[dev] = p;
    }
    scratch = g_noalloc_scratch_ptr[dev];
  }
  // Every scratch byte the sort reads is written earlier in the same call
  // (the error word and the per-call region are cleared by gs_isect_sort)
  // (per-tile digit counts, scan block sums, ping-pong key/value buffers), so
  // nothing needs clearing between calls.
  return gs_isect_sort(n_isects, key_bits, isect_ids, flatten_ids, sorted_isect_ids,
                       sorted_flatten_ids, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int gs_isect_sort_noalloc_check(int64_t n_isects, gs_stream_t stream) {
  if (n_isects <= 0) return GS_OK;
  if (n_isects > kNoAllocMaxIsects)
    return invalid("intersect_tile_sort_noalloc_check: more intersections than the sort takes");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return invalid("intersect_tile_sort_noalloc_check: no usable current device");
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    scratch = g_noalloc_scratch_ptr[dev];
  }
  if (!scratch) return GS_OK;  // no sort ran on this device yet
  return read_sort_error(n_isects, static_cast<const char*>(scratch), as_stream(stream));
}

namespace gsb {
namespace {
__global__ void set_u32_kernel(uint32_t* p, uint32_t v) { *p = v; }
}  // namespace
}  // namespace gsb

extern "C" int gs_isect_sort_wait_selftest(int64_t n_isects, const int64_t* isect_ids,
                                           const int32_t* flatten_ids, int64_t* sorted_isect_ids,
                                           int32_t* sorted_flatten_ids, void* workspace,
                                           size_t workspace_bytes, uint32_t spin_limit,
                                           gs_stream_t stream) {
  if (n_isects <= kSortTile || n_isects > 2 * kSortTile)
    return invalid("intersect_sort_wait_selftest: n_isects must be in (4096, 8192]");
  if (spin_limit < 1 || spin_limit > 1024)
    return invalid("intersect_sort_wait_selftest: spin_limit must be in 1..1024");
  if (!isect_ids || !flatten_ids || !sorted_isect_ids || !sorted_flatten_ids)
    return invalid("intersect_sort_wait_selftest: missing buffer");
  const SortLayout L = sort_layout(n_isects);
  if (!workspace || workspace_bytes < L.total) {
    set_error("intersect_sort_wait_selftest: workspace of %zu bytes needed", L.total);
    return GS_ERR_WORKSPACE;
  }
  cudaStream_t s = as_stream(stream);
  char* ws = static_cast<char*>(workspace);
  uint32_t* hist = reinterpret_cast<uint32_t*>(ws + L.hist);
  cudaMemsetAsync(ws + L.err, 0, sizeof(uint32_t), s);
  cudaMemsetAsync(ws + L.hist, 0, L.total - L.hist, s);
  const uint64_t* keys = reinterpret_cast<const uint64_t*>(isect_ids);
  const uint64_t flip = 0ull;
  radix_hist_kernel<<<grid_for(ceil_div(n_isects, 4), 256, 2), 256, 0, s>>>(
      n_isects, keys, 0, 1, flip, nullptr, hist);
  uint32_t* counter = reinterpret_cast<uint32_t*>(ws + L.ctrl);
  // the one CTA claims tile 1: tile 0 never runs, so its state stays unpublished
  set_u32_kernel<<<1, 1, 0, s>>>(counter, 1u);
  PassArgs a{};
  a.n = n_isects;
  a.keys_in = keys;
  a.vals_in = flatten_ids;
  a.keys_out = reinterpret_cast<uint64_t*>(sorted_isect_ids);
  a.vals_out = sorted_flatten_ids;
  a.shift = 0;
  a.flip = flip;
  a.pass = 0;
  a.pass_hist = hist;
  a.tile_counter = counter;
  a.state = reinterpret_cast<uint64_t*>(ws + L.state);
  a.error_word = reinterpret_cast<uint32_t*>(ws + L.err);
  a.spin_limit = spin_limit;
  launch_pass(kKV, kKV, 1, a, s);
  return launch_status("intersect_sort_wait_selftest");
}
