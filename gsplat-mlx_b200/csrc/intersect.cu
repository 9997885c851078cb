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

__global__ void __launch_bounds__(256) count_kernel(int64_t n, const float* __restrict__ means2d,
                                                    const int32_t* __restrict__ radii, int ts,
                                                    int tw, int th,
                                                    int32_t* __restrict__ tiles_per_gauss) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int2 rad = __ldg(reinterpret_cast<const int2*>(radii) + i);
    const float2 m = __ldg(reinterpret_cast<const float2*>(means2d) + i);
    const Rect r = tile_rect(m.x, m.y, rad.x, rad.y, ts, tw, th);
    tiles_per_gauss[i] = (r.y1 - r.y0) * (r.x1 - r.x0);
  }
}

// One warp encodes 32 consecutive Gaussians at a time.  A warp scan of their
// tile counts flattens the 32 runs into one index space j; lane l emits
// entries j = l, l+32, ...: the owner Gaussian of j comes from a search over
// the 32 prefix sums, its k-th tile in row-major order of its rect.  Runs
// start at offsets[i] as in the reference (consecutive runs are adjacent
// when offsets is the scan of the counts, so stores are coalesced); every
// write is bounds-checked like the CPU path (gsplat_intersect.cpp:473).
constexpr int kEncodeThreads = 256;
constexpr int kEncodeWarps = kEncodeThreads / 32;

__global__ void __launch_bounds__(kEncodeThreads) encode_kernel(
    int64_t n, int n_per_image, const float* __restrict__ means2d,
    const int32_t* __restrict__ radii, const float* __restrict__ depths,
    const int32_t* __restrict__ offsets, int ts, int tw, int th, int tile_bits, int64_t n_isects,
    int64_t* __restrict__ isect_ids, int32_t* __restrict__ flatten_ids) {
  __shared__ int s_pref[kEncodeWarps][33];
  __shared__ int s_x0[kEncodeWarps][32], s_y0[kEncodeWarps][32], s_w[kEncodeWarps][32];
  __shared__ int64_t s_off[kEncodeWarps][32], s_base[kEncodeWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t chunks = (n + 31) / 32;
  for (int64_t ch = (int64_t)blockIdx.x * kEncodeWarps + warp; ch < chunks;
       ch += (int64_t)gridDim.x * kEncodeWarps) {
    const int64_t i = ch * 32 + lane;
    int cnt = 0;
    if (i < n) {
      const int2 rad = __ldg(reinterpret_cast<const int2*>(radii) + i);
      if (rad.x > 0 && rad.y > 0) {
        const float2 m = __ldg(reinterpret_cast<const float2*>(means2d) + i);
        const Rect r = tile_rect(m.x, m.y, rad.x, rad.y, ts, tw, th);
        const int w = r.x1 - r.x0;
        cnt = (r.y1 - r.y0) * w;
        if (cnt > 0) {
          s_x0[warp][lane] = r.x0;
          s_y0[warp][lane] = r.y0;
          s_w[warp][lane] = w;
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
    s_pref[warp][lane + 1] = incl;
    if (lane == 0) s_pref[warp][0] = 0;
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    __syncwarp();
    for (int j = lane; j < total; j += 32) {
      // owner: the largest o with s_pref[o] <= j (counts of 0 never own)
      int lo = 0, hi = 31;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_pref[warp][mid] <= j) lo = mid;
        else hi = mid - 1;
      }
      const int o = lo;
      const int k = j - s_pref[warp][o];
      const int w = s_w[warp][o];
      const int dy = k / w;
      const int y = s_y0[warp][o] + dy;
      const int x = s_x0[warp][o] + (k - dy * w);
      const int64_t pos = s_off[warp][o] + k;
      if (pos >= 0 && pos < n_isects) {
        isect_ids[pos] = s_base[warp][o] | ((int64_t)(y * tw + x) << 32);
        flatten_ids[pos] = (int32_t)(ch * 32 + o);
      }
    }
    __syncwarp();
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

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(int64_t n,
                                                                    const int32_t* __restrict__ in,
                                                                    int64_t* __restrict__ sums) {
  __shared__ int64_t s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int64_t acc = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    if (i < n) acc += __ldg(in + i);
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

// May run in place (in == out): every element is read before it is written.
__global__ void __launch_bounds__(kScanThreads) scan_down_kernel(int64_t n, const int32_t* in,
                                                                  const int64_t* __restrict__ sums,
                                                                  int32_t* out) {
  __shared__ int64_t s_warp[32];
  const int64_t base = (int64_t)blockIdx.x * kScanChunk;
  int32_t v[kScanItems];
  int64_t acc = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    v[k] = i < n ? in[i] : 0;
    acc += v[k];
  }
  int64_t total;
  int64_t run = block_exclusive_scan<kScanThreads>(acc, s_warp, &total) + sums[blockIdx.x];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + (int64_t)threadIdx.x * kScanItems + k;
    if (i < n) out[i] = (int32_t)run;
    run += v[k];
  }
}

size_t scan_ws_bytes(int64_t n) {
  const int64_t nb = ceil_div(n < 1 ? 1 : n, kScanChunk);
  return (size_t)((nb * 8 + 255) / 256 * 256);
}

int scan_i32(int64_t n, const int32_t* in, int32_t* out, int64_t* total, void* ws, size_t ws_bytes,
             cudaStream_t s) {
  if (n <= 0) {
    if (total) cudaMemsetAsync(total, 0, sizeof(int64_t), s);
    return launch_status("scan");
  }
  if (!ws || ws_bytes < scan_ws_bytes(n)) {
    set_error("scan: workspace of %zu bytes needed", scan_ws_bytes(n));
    return GS_ERR_WORKSPACE;
  }
  const int64_t nb = ceil_div(n, kScanChunk);
  int64_t* sums = static_cast<int64_t*>(ws);
  scan_reduce_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(n, in, sums);
  scan_sums_kernel<<<1, 1024, 0, s>>>(nb, sums, total);
  scan_down_kernel<<<(unsigned)nb, kScanThreads, 0, s>>>(n, in, sums, out);
  return launch_status("scan");
}

// ------------------------------------------------------------ radix sort

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 16;                          // keys per thread
constexpr int kSortTile = kSortThreads * kSortItems;    // 4096 keys per CTA
constexpr int kWarpSpan = 32 * kSortItems;              // 512 keys per warp
constexpr int kRadix = 256;

__device__ __forceinline__ uint32_t digit_of(uint64_t k, int shift, uint64_t flip) {
  return (uint32_t)(((k ^ flip) >> shift) & 0xFFu);
}

// Per-CTA digit histogram of one pass; counts laid out digit-major
// ([digit][cta]) so that each digit's row can be scanned independently.
__global__ void __launch_bounds__(kSortThreads) radix_upsweep_kernel(
    int64_t n, const uint64_t* __restrict__ keys, int shift, uint64_t flip, int num_tiles,
    int32_t* __restrict__ counts) {
  __shared__ uint32_t s_hist[kSortWarps][kRadix];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&s_hist[0][0])[i] = 0;
  const int64_t base = (int64_t)blockIdx.x * kSortTile + (int64_t)warp * kWarpSpan;
  uint64_t k[kSortItems];
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {  // all loads in flight before any use
    const int64_t i = base + r * 32 + lane;
    k[r] = i < n ? __ldg(keys + i) : 0ull;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    const int64_t i = base + r * 32 + lane;
    if (i < n) atomicAdd(&s_hist[warp][digit_of(k[r], shift, flip)], 1u);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kRadix; d += kSortThreads) {
    uint32_t c = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) c += s_hist[w][d];
    counts[(int64_t)d * num_tiles + blockIdx.x] = (int32_t)c;
  }
}

// One CTA per digit: exclusive scan of that digit's per-tile counts in
// place (offsets of the digit's keys within the digit) and the digit total.
constexpr int kRowScanThreads = 256;
__global__ void __launch_bounds__(kRowScanThreads) radix_rowscan_kernel(
    int num_tiles, int32_t* __restrict__ counts, int32_t* __restrict__ totals) {
  __shared__ int64_t s_warp[32];
  int32_t* row = counts + (int64_t)blockIdx.x * num_tiles;
  int64_t carry = 0;
  for (int b0 = 0; b0 < num_tiles; b0 += kRowScanThreads * 4) {
    int32_t v[4];
    int64_t acc = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = b0 + threadIdx.x * 4 + k;
      v[k] = i < num_tiles ? row[i] : 0;
      acc += v[k];
    }
    int64_t chunk_total;
    int64_t run = block_exclusive_scan<kRowScanThreads>(acc, s_warp, &chunk_total) + carry;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = b0 + threadIdx.x * 4 + k;
      if (i < num_tiles) row[i] = (int32_t)run;
      run += v[k];
    }
    carry += chunk_total;
  }
  if (threadIdx.x == 0) totals[blockIdx.x] = (int32_t)carry;
}

struct DownSmem {
  uint64_t keys[kSortTile];
  int32_t vals[kSortTile];
  uint32_t hist[kSortWarps][kRadix];  // warp counts -> warp exclusive offsets
  uint32_t digit_start[kRadix];       // CTA-local exclusive prefix over digits
  uint32_t goff[kRadix];              // global offset of each digit for this CTA
  int64_t warp_tot[32];
};

// Stable rank-and-scatter of one pass.  Keys of a warp are processed in
// index order (round r covers keys r*32..r*32+31 of the warp's span), lanes
// in lane order, so ranks respect input order and the sort is stable.  The
// global base of each digit is the exclusive scan of the 256 digit totals
// (done here, redundantly per CTA) plus this CTA's row offset.
__global__ void __launch_bounds__(kSortThreads, 3) radix_downsweep_kernel(
    int64_t n, const uint64_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in,
    uint64_t* __restrict__ keys_out, int32_t* __restrict__ vals_out, int shift, uint64_t flip,
    int num_tiles, const int32_t* __restrict__ offsets, const int32_t* __restrict__ totals) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  DownSmem& sm = *reinterpret_cast<DownSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile_base = (int64_t)blockIdx.x * kSortTile;
  const int64_t base = tile_base + (int64_t)warp * kWarpSpan;
  uint64_t k[kSortItems];
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {  // all loads in flight before ranking
    const int64_t i = base + r * 32 + lane;
    k[r] = i < n ? __ldg(keys_in + i) : 0ull;
  }
  for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&sm.hist[0][0])[i] = 0;
  int64_t unused;
  const int64_t dbase =
      block_exclusive_scan<kSortThreads>(__ldg(totals + threadIdx.x), sm.warp_tot, &unused);
  sm.goff[threadIdx.x] =
      (uint32_t)(dbase + __ldg(offsets + (int64_t)threadIdx.x * num_tiles + blockIdx.x));
  __syncthreads();

  uint32_t rank[kSortItems];
  const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    const bool valid = base + r * 32 + lane < n;
    // Invalid lanes form their own group (digit 256) and count nowhere.
    const uint32_t d = valid ? digit_of(k[r], shift, flip) : (uint32_t)kRadix;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const uint32_t before = __popc(peers & lt_mask);
    const int leader = __ffs(peers) - 1;
    uint32_t cur = 0;
    if (valid) cur = sm.hist[warp][d];
    __syncwarp();
    if (valid && lane == leader) sm.hist[warp][d] = cur + __popc(peers);
    __syncwarp();
    rank[r] = cur + before;
  }
  __syncthreads();
  // Per digit: exclusive offsets over warps, CTA count, then a CTA-wide
  // exclusive scan over digits for the staging layout.
  uint32_t cta_count = 0;
  {
    const int d = threadIdx.x;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
      const uint32_t c = sm.hist[w][d];
      sm.hist[w][d] = cta_count;
      cta_count += c;
    }
  }
  int64_t total;
  const int64_t start = block_exclusive_scan<kSortThreads>(cta_count, sm.warp_tot, &total);
  sm.digit_start[threadIdx.x] = (uint32_t)start;
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    const int64_t i = base + r * 32 + lane;
    if (i < n) {
      const uint32_t d = digit_of(k[r], shift, flip);
      const uint32_t p = sm.digit_start[d] + sm.hist[warp][d] + rank[r];
      sm.keys[p] = k[r];
      sm.vals[p] = __ldg(vals_in + i);
    }
  }
  __syncthreads();
  const int64_t tile_n = (n - tile_base) < kSortTile ? (n - tile_base) : kSortTile;
  for (int i = threadIdx.x; i < tile_n; i += kSortThreads) {
    const uint64_t key = sm.keys[i];
    const uint32_t d = digit_of(key, shift, flip);
    const int64_t dst = (int64_t)sm.goff[d] + (i - (int64_t)sm.digit_start[d]);
    keys_out[dst] = key;
    vals_out[dst] = sm.vals[i];
  }
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

struct SortLayout {
  size_t keys_alt, vals_alt, counts, totals, total;
};

SortLayout sort_layout(int64_t n) {
  SortLayout L;
  const int64_t tiles = ceil_div(n < 1 ? 1 : n, kSortTile);
  const int64_t ncounts = tiles * kRadix;
  L.keys_alt = 0;
  L.vals_alt = L.keys_alt + align256(sizeof(uint64_t) * (size_t)(n < 1 ? 1 : n));
  L.counts = L.vals_alt + align256(sizeof(int32_t) * (size_t)(n < 1 ? 1 : n));
  L.totals = L.counts + align256(sizeof(int32_t) * (size_t)ncounts);
  L.total = L.totals + align256(sizeof(int32_t) * kRadix);
  return L;
}

// ------------------------------------------------------------ offsets

// tile_offsets[o] = lower bound of key(o) = (o / T) << tb | (o % T) in
// isect_ids >> 32: one thread per slot, binary search over the sorted keys,
// as the reference does (gsplat_intersect.cpp:605-641, metal :110-136).
__global__ void __launch_bounds__(256) offset_kernel(int64_t m, const int64_t* __restrict__ ids,
                                                     int I, int T, int tb,
                                                     int32_t* __restrict__ offsets) {
  const int64_t n_off = (int64_t)I * T;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < n_off;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t key = ((o / T) << tb) | (o % T);
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
  count_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
      n, means2d, radii, p->tile_size, p->tile_width, p->tile_height, tiles_per_gauss);
  return launch_status("intersect_tile_count");
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
  encode_kernel<<<grid_for((n + 31) / 32, kEncodeWarps), kEncodeThreads, 0, as_stream(stream)>>>(
      n, p->N, means2d, radii, depths, offsets, p->tile_size, p->tile_width, p->tile_height,
      tile_bits, n_isects, isect_ids, flatten_ids);
  return launch_status("intersect_tile_encode");
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
  uint64_t* alt_k = reinterpret_cast<uint64_t*>(ws + L.keys_alt);
  int32_t* alt_v = reinterpret_cast<int32_t*>(ws + L.vals_alt);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
  int32_t* totals = reinterpret_cast<int32_t*>(ws + L.totals);
  const int tiles = (int)ceil_div(n, kSortTile);
  const int passes = (key_bits + 7) / 8;
  // Signed order: with all 64 bits in play the sign bit is flipped so that
  // an unsigned digit sort orders like the signed int64 comparison.
  const uint64_t flip = key_bits == 64 ? (1ull << 63) : 0ull;
  const int smem = (int)sizeof(DownSmem);
  cudaFuncSetAttribute(radix_downsweep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const uint64_t* src_k = reinterpret_cast<const uint64_t*>(isect_ids);
  const int32_t* src_v = flatten_ids;
  for (int pass = 0; pass < passes; ++pass) {
    // Choose destinations so that the last pass lands in the output.
    const bool to_out = ((passes - 1 - pass) % 2) == 0;
    uint64_t* dst_k = to_out ? reinterpret_cast<uint64_t*>(sorted_isect_ids) : alt_k;
    int32_t* dst_v = to_out ? sorted_flatten_ids : alt_v;
    const int shift = pass * 8;
    radix_upsweep_kernel<<<tiles, kSortThreads, 0, s>>>(n, src_k, shift, flip, tiles, counts);
    radix_rowscan_kernel<<<kRadix, kRowScanThreads, 0, s>>>(tiles, counts, totals);
    radix_downsweep_kernel<<<tiles, kSortThreads, smem, s>>>(n, src_k, src_v, dst_k, dst_v, shift,
                                                             flip, tiles, counts, totals);
    src_k = dst_k;
    src_v = dst_v;
  }
  return launch_status("intersect_tile_sort");
}

extern "C" int gs_isect_offset(int64_t n_isects, const int64_t* isect_ids, int32_t I,
                               int32_t tile_width, int32_t tile_height, int32_t* tile_offsets,
                               gs_stream_t stream) {
  if (I <= 0 || tile_width <= 0 || tile_height <= 0)
    return invalid("intersect_offset expects positive image and tile dimensions.");
  if (n_isects < 0 || n_isects > INT32_MAX) return invalid("intersect_offset: bad n_isects");
  const int T = tile_width * tile_height;
  const int tb = gs_floor_log2_plus_one(T);
  if (!tile_offsets || (n_isects > 0 && !isect_ids)) return invalid("intersect_offset: missing buffer");
  offset_kernel<<<grid_for((int64_t)I * T, 256), 256, 0, as_stream(stream)>>>(n_isects, isect_ids,
                                                                             I, T, tb, tile_offsets);
  return launch_status("intersect_offset");
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
  // (per-tile digit counts, scan block sums, ping-pong key/value buffers), so
  // nothing needs clearing between calls.
  return gs_isect_sort(n_isects, key_bits, isect_ids, flatten_ids, sorted_isect_ids,
                       sorted_flatten_ids, scratch, kNoAllocScratchBytes, stream);
}
