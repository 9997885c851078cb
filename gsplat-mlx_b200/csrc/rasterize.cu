// Rasterize to pixels (3DGS): front-to-back alpha compositing, forward and
// backward.
//
// Per-pixel semantics: gsplat_rasterize.cpp:249-569 (CPU) ==
// metal/gsplat_rasterize.metal:31-251 -- sigma = 0.5(c0 dx^2 + c2 dy^2) +
// c1 dx dy at the pixel centre, alpha = min(0.99, o e^-sigma), skip when
// sigma < 0 or alpha < 1/255, stop before compositing once T(1-alpha) <=
// 1e-4, last_id = last composited intersection.
//
// B200 mapping: one CTA per (image, tile), one thread per pixel.  The
// tile's intersection range is walked in batches of BLOCK Gaussians staged
// in shared memory (the Metal kernel re-reads device memory per pixel).
// Forward CTAs stop as soon as every pixel of the tile is saturated.  The
// backward walks batches back to front from the CTA's largest last_id; per
// Gaussian, the gradient terms of a warp's 32 pixels are summed with a
// butterfly transpose-reduction (16 shuffles for up to 16 terms), added
// into per-batch shared accumulators, and flushed with one global atomicAdd
// per term per Gaussian per tile (the Metal kernel issues 5-8 global
// atomics per pixel x Gaussian pair).
#include "common.cuh"

namespace gsb {
namespace {

constexpr float kAlphaThreshold = 1.0f / 255.0f;
constexpr float kMaxAlpha = 0.99f;
constexpr float kTransmittanceThreshold = 1.0e-4f;
constexpr float kMinOneMinusAlpha = 1.0e-6f;
constexpr int kMaxChannels = 64;
// last_ids mark of a pixel the forward kernels leave to raster_fix_kernel
// (a real last id is >= 0).
constexpr int32_t kUndecided = -1;

// Exact decisions.  The reference decides with std::exp (glibc expf) on its
// own fp32 sigma: skip when sigma < 0 or o e^-sigma < 1/255, clamp alpha at
// 0.99, stop when T (1 - alpha) <= 1e-4.  Here:
//
// * sigma is the reference's float (gauss_sigma below).
// * The skip and clamp decisions compare sigma with two bounds that depend on
//   the opacity alone (sigma_bounds below): f(sigma) = o (x) e^-sigma, with the
//   exponential correctly rounded and (x) a float multiply, is non-increasing
//   in sigma, so "f >= 1/255" is "sigma <= keep" and "f <= 0.99" is
//   "sigma >= clamp" for two floats found once per Gaussian.  No exponential
//   is evaluated for a decision inside the pixel loops.
// * The stop test sees the fast T (alpha from __expf, T - T alpha with one
//   rounding).  Each pixel carries a bound E on |T_fast - T_reference|: per
//   composited step E becomes E (1 - alpha) + T_prev alpha d + T_next kStepErr,
//   with d = kAlphaErr0 + kAlphaErrS max(keep, 0) bounding the relative alpha
//   error of the Gaussian's pairs, whose sigma is at most its keep bound
//   (__expf is within 2 + floor(1.173 |x|) ulp; the correctly rounded e
//   within half an ulp; the product rounds once; zero for a clamped alpha,
//   which is exact) and kStepErr the three roundings between the two
//   recurrences.  A pixel
//   whose next T lies within E of 1e-4 is marked undecided (last id
//   kUndecided) and recomputed exactly, with the correctly rounded
//   exponential, by raster_fix_kernel after the forward (exact_walk).
constexpr float kAlphaErrS = 1.4e-7f;  // per unit of sigma: 1.173 ulp
constexpr float kAlphaErr0 = 4.2e-7f;  // 2 ulp of __expf, 0.5 of the rounded e, 1 of the product
constexpr float kStepErr = 2.0e-7f;    // three roundings of 2^-24

// e^x correctly rounded to float: CUDA's double exponential (under one
// double ulp of error) rounded once.  glibc's expf, which the reference
// calls, returns the same float on all but 7.7e-5 of the floats in
// [-16, 0] (exhaustive comparison), and there by one ulp, which moves a
// decision only when the product o e^-sigma itself sits on a threshold.
__device__ __forceinline__ float exp_cr(float x) { return __double2float_rn(exp((double)x)); }

__device__ __forceinline__ float next_up(float x) { return nextafterf(x, INFINITY); }
__device__ __forceinline__ float next_down(float x) { return nextafterf(x, -INFINITY); }

// The decision bounds of opacity o: keep = the largest float sigma with
// o (x) CR(e^-sigma) >= 1/255 (-inf when none: the Gaussian is never
// composited), clamp = the smallest float sigma with o (x) CR(e^-sigma) <= 0.99
// (-inf when every sigma >= 0 qualifies: never clamped).  A pair at sigma
// (with sigma >= 0, or -0) is composited iff !(sigma > keep) and has
// alpha = 0.99 iff sigma < clamp, exactly as the reference decides it with
// CR(exp).  NaN or +inf opacities: the reference's std::min(0.99f, NaN)
// yields 0.99, so every pair is composited and clamped (both bounds +inf).
//
// With e_min the smallest float e with o (x) e >= 1/255 and m the midpoint
// between e_min and the float below it, CR(e^-sigma) >= e_min exactly when
// e^-sigma > m (a tie is impossible for the exponential of a float), i.e.
// sigma < -ln m: keep is -ln m rounded down to a float.  The double
// logarithm gives -ln m rounded to nearest; one double exponential tells
// whether that float lies above the root (then the float below is keep).
// The clamp bound is the mirror image with the midpoint above e_max.
__device__ __forceinline__ float root_down(double m) {  // largest float s with e^-s > m
  float s = __double2float_rn(-log(m));
  if (!(exp(-(double)s) > m)) s = next_down(s);
  return s;
}
__device__ __forceinline__ float root_up(double m) {  // smallest float s with e^-s < m
  float s = __double2float_rn(-log(m));
  if (!(exp(-(double)s) < m)) s = next_up(s);
  return s;
}

// The smallest float sigma with CR(e^-sigma) == 0: e^-sigma <= 2^-150 (which
// rounds to zero, ties to even), i.e. sigma >= 150 ln 2 = 103.9720770...
// rounded up.  glibc's expf agrees at this boundary (0 at -S, the smallest
// subnormal one float below).
constexpr float kUnderflowSigma = 0x1.9fe36ap+6f;  // 103.972084

// An opacity of -inf: -inf (x) e is -inf (skipped) while e > 0 and NaN once
// the exponential underflows, which the reference's std::min(0.99f, NaN)
// turns into alpha 0.99.  Its bounds are (-kUnderflowSigma, +inf): a negative
// finite keep bound marks the composited range [kUnderflowSigma, +inf] (see
// keep_range), always clamped.
__device__ __noinline__ float2 sigma_bounds(float o) {
  if (!(o < INFINITY)) return make_float2(INFINITY, INFINITY);
  if (o == -INFINITY) return make_float2(-kUnderflowSigma, INFINITY);
  float2 b = make_float2(-INFINITY, -INFINITY);
  if (!(o > 0.0f)) return b;
  // smallest e with o (x) e >= 1/255
  float e = __fdiv_rn(kAlphaThreshold, o);
  for (int i = 0; i < 8 && __fmul_rn(o, e) < kAlphaThreshold; ++i) e = next_up(e);
  for (int i = 0; i < 8 && e > 0.0f && __fmul_rn(o, next_down(e)) >= kAlphaThreshold; ++i)
    e = next_down(e);
  if (e <= 1.0f) b.x = fmaxf(root_down(0.5 * ((double)e + (double)next_down(e))), 0.0f);
  // largest e with o (x) e <= 0.99
  if (o > kMaxAlpha) {
    e = __fdiv_rn(kMaxAlpha, o);
    for (int i = 0; i < 8 && __fmul_rn(o, e) > kMaxAlpha; ++i) e = next_down(e);
    for (int i = 0; i < 8 && __fmul_rn(o, next_up(e)) <= kMaxAlpha; ++i) e = next_up(e);
    if (e < 1.0f) b.y = fmaxf(root_up(0.5 * ((double)e + (double)next_up(e))), 0.0f);
  }
  return b;
}

// The stop decision of the fast path for a pixel whose fast T after this
// step is next_T, E its error bound: 0 continue, 1 stop, 2 undecided
// (within E of 1e-4: recompute the pixel exactly).
__device__ __forceinline__ int stop_decision(float next_T, float E) {
  if (next_T > fmaf(E, 1.0625f, kTransmittanceThreshold + 1.0e-12f)) return 0;
  return next_T > fmaf(E, -1.0625f, kTransmittanceThreshold - 1.0e-12f) ? 2 : 1;
}

// E after a step from Tr with alpha (vis = alpha Tr, oma = 1 - alpha); a
// clamped alpha (exactly 0.99) adds no alpha error.
// d: the relative alpha error bound of the Gaussian, alpha_err(keep) (its
// composited pairs have sigma <= keep).
__device__ __forceinline__ float step_bound(float E, float vis, float oma, float next_T,
                                            float d, bool clamped) {
  return fmaf(E, oma, fmaf(vis, clamped ? 0.0f : d, next_T * kStepErr));
}

// The relative error bound of the fast alpha of a Gaussian with keep bound sk.
__device__ __forceinline__ float alpha_err(float sk) {
  return fmaf(fmaxf(sk, 0.0f), kAlphaErrS, kAlphaErr0);
}

// The fast path's alpha of a composited pair: exactly 0.99 when clamped,
// else o __expf(-sigma) (within the alpha error of step_bound).
__device__ __forceinline__ float fast_alpha(float sigma, float o, bool clamped) {
  return clamped ? kMaxAlpha : fminf(kMaxAlpha, __fmul_rn(o, __expf(-sigma)));
}

// The reference's sigma = 0.5f * (c0 * dx * dx + c2 * dy * dy) + c1 * dx * dy
// (gsplat_rasterize.cpp:333-334, 474-475), evaluated in its order with one
// IEEE rounding per operation (explicit intrinsics, which the compiler does
// not contract), so that every kernel here gets the reference's float.
// c0 dx and c2 dy are returned for reuse by the backward.
struct Sigma {
  float cdx, cdy, s;
};

__device__ __forceinline__ Sigma gauss_sigma(float dx, float dy, float c0, float c1, float c2) {
  Sigma r;
  r.cdx = __fmul_rn(c0, dx);
  r.cdy = __fmul_rn(c2, dy);
  const float q = __fadd_rn(__fmul_rn(r.cdx, dx), __fmul_rn(r.cdy, dy));
  r.s = __fadd_rn(__fmul_rn(0.5f, q), __fmul_rn(__fmul_rn(c1, dx), dy));
  return r;
}

// The sigma range [lo, hi] in which an entry's pairs are composited, from
// its keep bound: [0, keep] (keep >= 0, or -inf: never), or for the -inf
// opacity marker (a negative finite keep, -kUnderflowSigma) [-keep, +inf].
// Worked out once per entry, outside the pixel loops.
struct Range {
  float lo, hi;
};
__device__ __forceinline__ Range keep_range(float keep) {
  const bool under = keep < 0.0f && keep > -INFINITY;
  return Range{under ? -keep : 0.0f, under ? INFINITY : keep};
}

// Composited (reference: !(sigma < 0 || alpha < 1/255)) for the entry's
// range; a NaN sigma is composited, as the reference's min(0.99, NaN) is
// 0.99.
__device__ __forceinline__ bool composited(float sigma, Range r) {
  return !(sigma < r.lo) && !(sigma > r.hi);
}

struct RArgs {
  int I, N, CH, W, H, ts, tw, th;
  int ty0, rows;  // tile rows [ty0, ty0 + rows) are rendered (all: 0, th)
  int opac_shared;  // opacities / v_opacities are [N]: entry g reads g mod N
  int64_t n_isects;
  const float* means2d;
  const float* conics;
  const float* colors;
  const float* opacities;
  const float* backgrounds;
  const uint8_t* masks;
  const int32_t* tile_offsets;
  const int32_t* flatten_ids;
  const float2* sbounds;  // per opacity entry: (keep, clamp) of sigma_bounds; null: computed
  const int32_t* tile_order;  // CTA b renders slot tile_order[b]; null: slot b
  int32_t* tile_cost;  // fwd, optional: per slot, the list entries its pixels walk
};

// The forward's record of a tile's cost for the backward's schedule: the
// number of list entries the backward walks for the tile, max over its
// pixels of (min(end - 1, last id) - start + 1), with an undecided pixel
// counted as the whole list.  `my` is the thread's max of min(end - 1,
// last id) (-1: no pixel); every thread of the CTA calls this.
__device__ __forceinline__ void record_tile_cost(const RArgs& a, int64_t slot, int start, int my,
                                                 int* s_cost) {
  if (!a.tile_cost) return;
  __syncthreads();  // s_cost's initial value is visible to every warp
  my = __reduce_max_sync(0xffffffffu, my);
  if ((threadIdx.x & 31) == 0) atomicMax(s_cost, my);
  __syncthreads();
  if (threadIdx.x == 0) a.tile_cost[slot] = max(0, *s_cost - start + 1);
}

// Index of entry g's opacity (and opacity gradient).
// With shared opacities entry g reads g mod N.  The lists of a tile of
// image i hold the elements i N .. i N + N - 1 (the encode's flatten ids), so
// g - i N is that remainder without a 64-bit division; other ids take the
// division.
__device__ __forceinline__ int64_t opac_index(const RArgs& a, int64_t g, int image) {
  if (!a.opac_shared) return g;
  const int64_t r = g - (int64_t)image * a.N;
  return (uint64_t)r < (uint64_t)a.N ? r : g % a.N;
}

// (keep, clamp) sigma bounds of entry g (of a tile of `image`) with opacity o.
__device__ __forceinline__ float2 entry_bounds(const RArgs& a, int64_t g, int image, float o) {
  return a.sbounds ? __ldg(a.sbounds + opac_index(a, g, image)) : sigma_bounds(o);
}

// The CTA's tile: `slot` indexes tile_offsets ([I, rows, tw]), `mask` the
// masks ([I, th, tw]).
struct TileIdx {
  int64_t slot, mask;
  int image, tile_x, tile_y;
};

__device__ __forceinline__ TileIdx tile_of(const RArgs& a) {
  TileIdx t;
  t.slot = a.tile_order ? __ldg(a.tile_order + blockIdx.x) : (int)blockIdx.x;
  const int64_t per = (int64_t)a.rows * a.tw;
  t.image = (int)(t.slot / per);
  const int loc = (int)(t.slot - (int64_t)t.image * per);
  const int ly = loc / a.tw;
  t.tile_x = loc - ly * a.tw;
  t.tile_y = a.ty0 + ly;
  t.mask = ((int64_t)t.image * a.th + t.tile_y) * a.tw + t.tile_x;
  return t;
}

__device__ __forceinline__ void tile_range(const RArgs& a, int64_t slot, int& start, int& end) {
  const int64_t n_slots = (int64_t)a.I * a.rows * a.tw;
  start = __ldg(a.tile_offsets + slot);
  end = (slot + 1 == n_slots) ? (int)a.n_isects : __ldg(a.tile_offsets + slot + 1);
}

// The CTA recomputes the pixel `pix` of `image`, centred at (px, py), whose
// tile list is [start, end), exactly as the reference does
// (gsplat_rasterize.cpp:320-357), and writes its outputs: the reference's
// sigma, its decisions (sigma bounds), alpha from the correctly rounded
// exponential, and T (1 - alpha), alpha T and the colour sums with one
// rounding per operation in list order.  Per chunk of kWalk entries (one
// per thread; the next chunk's loads are issued before this one is folded)
// the composited entries are compacted in list order into shared memory
// with their colours, thread 0 folds them into T in order (stopping where
// the reference stops) together with the colour sums (with a runtime
// channel count, thread c sums channel c and c + kWalk afterwards).  The longest walk bounds the fix-up
// kernel's time, so a walk gets every thread of the CTA.
constexpr int kWalk = 256;

struct WalkSmem {
  __align__(16) float al[kWalk + 4];      // alpha of the kept entries, in list order
  int g[kWalk];                           // their Gaussian
  __align__(16) int ix[kWalk + 4];        // their list index
  float vis[kWalk];                       // alpha T of the folded ones
  __align__(16) float col[kWalk + 4][4];  // their colours (CH in 1..4)
  int wcnt[kWalk / 32];  // kept entries per warp
  float T;
  int cur, nfold, stop;
};

template <int CH>
__device__ __forceinline__ void exact_walk(const RArgs& a, int start, int end, int image,
                                           int64_t pix,
                                        float px, float py, WalkSmem& w, float* render_colors,
                                        float* render_alphas, int32_t* last_ids) {
  const int ch = CH > 0 ? CH : a.CH;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __syncthreads();  // every thread has read the previous walk's final T
  if (tid == 0) {
    w.T = 1.0f;
    w.cur = 0;
    w.stop = 0;
  }
  float acc0 = 0.0f, acc1 = 0.0f;  // CH == 0: channels tid and tid + kWalk (<= 64)
  float acc[CH > 0 ? CH : 1];       // CH > 0: thread 0's colour sums
#pragma unroll
  for (int c = 0; c < (CH > 0 ? CH : 1); ++c) acc[c] = 0.0f;
  int g = 0;
  float2 m = make_float2(0.f, 0.f), sb = make_float2(0.f, 0.f);
  float c0 = 0.f, c1 = 0.f, c2 = 0.f, o = 0.f;
  float4 cl = make_float4(0.f, 0.f, 0.f, 0.f);  // CH > 0: the entry's colour
  auto load = [&](int cb) {
    const int idx = cb + tid;
    if (idx < end) {
      g = __ldg(a.flatten_ids + idx);
      m = __ldg(reinterpret_cast<const float2*>(a.means2d) + g);
      const float* con = a.conics + (int64_t)g * 3;
      c0 = __ldg(con);
      c1 = __ldg(con + 1);
      c2 = __ldg(con + 2);
      o = __ldg(a.opacities + opac_index(a, g, image));
      if (a.sbounds) sb = __ldg(a.sbounds + opac_index(a, g, image));
      if (CH > 0) {
        const float* cp = a.colors + (int64_t)g * ch;
        cl.x = __ldg(cp);
        if (CH > 1) cl.y = __ldg(cp + 1);
        if (CH > 2) cl.z = __ldg(cp + 2);
        if (CH > 3) cl.w = __ldg(cp + 3);
      }
    }
  };
  load(start);
  for (int cb = start; cb < end; cb += kWalk) {
    const int idx = cb + tid;
    bool take = false;
    float al = 0.0f;
    const int gk = g;
    const float4 clk = cl;
    if (idx < end) {
      const float sigma = gauss_sigma(__fsub_rn(m.x, px), __fsub_rn(m.y, py), c0, c1, c2).s;
      if (!a.sbounds) sb = sigma_bounds(o);
      take = composited(sigma, keep_range(sb.x));
      if (take) al = sigma < sb.y ? kMaxAlpha : fminf(kMaxAlpha, __fmul_rn(o, exp_cr(-sigma)));
    }
    if (cb + kWalk < end) load(cb + kWalk);  // in flight during the fold
    const unsigned bal = __ballot_sync(0xffffffffu, take);
    if (lane == 0) w.wcnt[warp] = __popc(bal);
    __syncthreads();
    int base = 0, cnt = 0;
#pragma unroll
    for (int i = 0; i < kWalk / 32; ++i) {
      const int c = w.wcnt[i];
      base += i < warp ? c : 0;
      cnt += c;
    }
    if (take) {
      const int slot = base + __popc(bal & ((1u << lane) - 1u));
      w.al[slot] = al;
      w.g[slot] = gk;
      w.ix[slot] = idx;
      if (CH > 0) *reinterpret_cast<float4*>(w.col[slot]) = clk;
    }
    __syncthreads();
    if (tid == 0) {
      // T and, with CH > 0, the colour sums (thread 0 keeps them in acc[])
      // four entries per round from vector loads, so that the shared
      // memory reads do not sit on the T recurrence
      float T = w.T;
      int k = 0, cur = w.cur;
      bool stop = false;
      for (int k4 = 0; k4 < cnt && !stop; k4 += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(w.al + k4);
        const int4 i4 = *reinterpret_cast<const int4*>(w.ix + k4);
        float4 col4[4];
        if (CH > 0) {
#pragma unroll
          for (int j = 0; j < 4; ++j) col4[j] = *reinterpret_cast<const float4*>(w.col[k4 + j]);
        }
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
        const int iv[4] = {i4.x, i4.y, i4.z, i4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (k4 + j >= cnt || stop) break;
          const float nT = __fmul_rn(T, __fsub_rn(1.0f, av[j]));
          if (nT <= kTransmittanceThreshold) {
            stop = true;
            break;
          }
          const float vis = __fmul_rn(av[j], T);
          if (CH > 0) {
            const float cc[4] = {col4[j].x, col4[j].y, col4[j].z, col4[j].w};
#pragma unroll
            for (int c = 0; c < (CH > 0 ? CH : 1); ++c)
              acc[c] = __fadd_rn(acc[c], __fmul_rn(cc[c], vis));
          } else {
            w.vis[k4 + j] = vis;
          }
          cur = iv[j];
          T = nT;
          k = k4 + j + 1;
        }
      }
      if (stop) w.stop = 1;
      w.T = T;
      w.cur = cur;
      w.nfold = k;
    }
    __syncthreads();
    const int nf = w.nfold;
    if (CH == 0) {
      for (int k = 0; k < nf; ++k) {
        const float vis = w.vis[k];
        const int64_t gq = w.g[k];
        if (tid < ch) acc0 = __fadd_rn(acc0, __fmul_rn(__ldg(a.colors + gq * ch + tid), vis));
        if (tid + kWalk < ch)
          acc1 = __fadd_rn(acc1, __fmul_rn(__ldg(a.colors + gq * ch + tid + kWalk), vis));
      }
    }
    const bool stop = w.stop != 0;
    __syncthreads();  // the arrays are refilled by the next chunk
    if (stop) break;
  }
  const float T = w.T;
  if (CH > 0) {
    if (tid == 0) {
#pragma unroll
      for (int c = 0; c < (CH > 0 ? CH : 1); ++c) {
        const float bg = a.backgrounds ? __ldg(a.backgrounds + image * ch + c) : 0.0f;
        render_colors[pix * ch + c] = __fadd_rn(acc[c], __fmul_rn(T, bg));
      }
    }
  } else {
    for (int j = 0; j < 2; ++j) {
      const int c = tid + j * kWalk;
      if (c < ch) {
        const float bg = a.backgrounds ? __ldg(a.backgrounds + image * ch + c) : 0.0f;
        render_colors[pix * ch + c] = __fadd_rn(j ? acc1 : acc0, __fmul_rn(T, bg));
      }
    }
  }
  if (tid == 0) {
    render_alphas[pix] = __fsub_rn(1.0f, T);
    last_ids[pix] = w.cur;
  }
  __syncthreads();  // w serves the next pixel
}

// ------------------------------------------------------------------ forward
// CH > 0: channel count known at compile time (colours staged in smem and
// accumulated in registers); CH == 0: runtime channel count up to 64.
template <int CH>
__global__ void raster_fwd_kernel(RArgs a, float* __restrict__ render_colors,
                                  float* __restrict__ render_alphas,
                                  int32_t* __restrict__ last_ids) {
  extern __shared__ float smem[];
  const int BLOCK = blockDim.x;
  const int ch = CH > 0 ? CH : a.CH;
  float2* s_xy = reinterpret_cast<float2*>(smem);
  float4* s_co = reinterpret_cast<float4*>(smem + 2 * BLOCK);  // conic xyz, opacity
  float2* s_sb = reinterpret_cast<float2*>(smem + 6 * BLOCK);  // sigma bounds
  float* s_col = smem + 8 * BLOCK;                              // [BLOCK][ch]

  __shared__ int s_cost;
  const TileIdx ti = tile_of(a);
  const int image = ti.image, tile_x = ti.tile_x, tile_y = ti.tile_y;
  const int tid = threadIdx.x;
  const int ly = tid / a.ts, lx = tid - ly * a.ts;
  const int x = tile_x * a.ts + lx, y = tile_y * a.ts + ly;
  const bool inside = tid < a.ts * a.ts && x < a.W && y < a.H;
  const int64_t pix = ((int64_t)image * a.H + y) * a.W + x;

  if (a.masks && !a.masks[ti.mask]) {
    if (inside) {
      for (int c = 0; c < ch; ++c)
        render_colors[pix * ch + c] = a.backgrounds ? __ldg(a.backgrounds + image * ch + c) : 0.0f;
      render_alphas[pix] = 0.0f;
      last_ids[pix] = 0;
    }
    if (a.tile_cost && tid == 0) a.tile_cost[ti.slot] = 0;
    return;
  }
  if (tid == 0) s_cost = -1;
  int start, end;
  tile_range(a, ti.slot, start, end);
  const float px = (float)x + 0.5f, py = (float)y + 0.5f;
  float Tr = 1.0f;
  int cur = 0;
  bool done = !inside, unsure = false;
  float E = 0.0f;  // bound on |Tr - the reference's T|
  float acc[CH > 0 ? CH : 1];
#pragma unroll
  for (int c = 0; c < (CH > 0 ? CH : 1); ++c) acc[c] = 0.0f;
  if (CH == 0 && inside)
    for (int c = 0; c < ch; ++c) render_colors[pix * ch + c] = 0.0f;

  for (int b0 = start; b0 < end; b0 += BLOCK) {
    if (__syncthreads_count(!done) == 0) break;
    const int idx = b0 + tid;
    if (idx < end) {
      const int g = __ldg(a.flatten_ids + idx);
      const float o = __ldg(a.opacities + opac_index(a, g, image));
      s_xy[tid] = __ldg(reinterpret_cast<const float2*>(a.means2d) + g);
      s_co[tid] = make_float4(__ldg(a.conics + (int64_t)g * 3), __ldg(a.conics + (int64_t)g * 3 + 1),
                              __ldg(a.conics + (int64_t)g * 3 + 2), o);
      s_sb[tid] = entry_bounds(a, g, image, o);
      for (int c = 0; c < ch; ++c) s_col[tid * ch + c] = __ldg(a.colors + (int64_t)g * ch + c);
    }
    __syncthreads();
    const int cnt = min(BLOCK, end - b0);
    for (int j = 0; j < cnt && !done; ++j) {
      const float2 m = s_xy[j];
      const float4 co = s_co[j];
      const float2 sb = s_sb[j];
      const float dx = m.x - px, dy = m.y - py;
      const float sigma = gauss_sigma(dx, dy, co.x, co.y, co.z).s;
      if (!composited(sigma, keep_range(sb.x))) continue;
      const bool clamped = !(sigma >= sb.y);  // o e^-sigma > 0.99 (or NaN)
      const float alpha = fast_alpha(sigma, co.w, clamped);
      const float vis = alpha * Tr;
      const float next_T = __fmaf_rn(-alpha, Tr, Tr);
      const float nE = step_bound(E, vis, 1.0f - alpha, next_T, alpha_err(sb.x), clamped);
      if (const int st = stop_decision(next_T, nE)) {
        unsure = st == 2;
        done = true;
        break;
      }
      E = nE;
      if (CH > 0) {
#pragma unroll
        for (int c = 0; c < (CH > 0 ? CH : 1); ++c) acc[c] += s_col[j * (CH > 0 ? CH : 1) + c] * vis;
      } else {
        for (int c = 0; c < ch; ++c) render_colors[pix * ch + c] += s_col[j * ch + c] * vis;
      }
      cur = b0 + j;
      Tr = next_T;
    }
  }
  if (inside && !unsure) {
    render_alphas[pix] = 1.0f - Tr;
    if (CH > 0) {
#pragma unroll
      for (int c = 0; c < (CH > 0 ? CH : 1); ++c) {
        const float bg = a.backgrounds ? __ldg(a.backgrounds + image * CH + c) : 0.0f;
        render_colors[pix * CH + c] = acc[c] + Tr * bg;
      }
    } else {
      for (int c = 0; c < ch; ++c) {
        const float bg = a.backgrounds ? __ldg(a.backgrounds + image * ch + c) : 0.0f;
        render_colors[pix * ch + c] += Tr * bg;
      }
    }
    last_ids[pix] = cur;
  }
  // a pixel whose stop decision fell within the error bound is left to
  // raster_fix_kernel
  if (inside && unsure) last_ids[pix] = kUndecided;
  record_tile_cost(a, ti.slot, start, inside ? (unsure ? end - 1 : min(end - 1, cur)) : -1,
                   &s_cost);
}

// Recomputes exactly the pixels that the forward kernel left undecided
// (last_ids == kUndecided).  The CTAs scan the rendered rows in row-major
// order, one pixel per thread (so that the few undecided pixels land in
// different CTAs and are walked at once), and walk each undecided pixel they
// find with all their threads
// (exact_walk).  Kept out of the forward kernels: the walk code there took
// registers from the compositing loop.
constexpr int kFixPixels = kWalk;

template <int CH>
__global__ void __launch_bounds__(kWalk) raster_fix_kernel(RArgs a,
                                                           float* __restrict__ render_colors,
                                                           float* __restrict__ render_alphas,
                                                           int32_t* __restrict__ last_ids) {
  __shared__ WalkSmem w;
  __shared__ int64_t s_list[kFixPixels];
  __shared__ int s_n;
  const int tid = threadIdx.x;
  // the rendered rows: those of tile rows [ty0, ty0 + rows)
  const int y0 = a.ty0 * a.ts, y1 = min(a.H, (a.ty0 + a.rows) * a.ts);
  const int64_t per_image = (int64_t)(y1 - y0) * a.W;
  const int64_t total = (int64_t)a.I * per_image;
  if (tid == 0) s_n = 0;
  __syncthreads();
  const int64_t p0 = (int64_t)blockIdx.x * kFixPixels;
  const bool all_rows = y0 == 0 && y1 == a.H;  // then pixel p of the scan is pixel p
  for (int k = tid; k < kFixPixels; k += kWalk) {
    const int64_t p = p0 + k;
    if (p >= total) break;
    int64_t pix = p;
    if (!all_rows) {
      const int64_t image = p / per_image, r = p - image * per_image;
      pix = (image * a.H + y0) * a.W + r;
    }
    if (__ldg(last_ids + pix) == kUndecided) s_list[atomicAdd(&s_n, 1)] = pix;
  }
  __syncthreads();
  const int n = s_n;
  for (int u = 0; u < n; ++u) {
    const int64_t pix = s_list[u];
    const int64_t image = pix / ((int64_t)a.H * a.W);
    const int rem = (int)(pix - image * a.H * a.W);
    const int y = rem / a.W, x = rem - y * a.W;
    const int tx = x / a.ts, ty = y / a.ts;
    const int64_t slot = ((int64_t)image * a.rows + (ty - a.ty0)) * a.tw + tx;
    int start, end;
    tile_range(a, slot, start, end);
    exact_walk<CH>(a, start, end, (int)image, pix, (float)x + 0.5f, (float)y + 0.5f, w,
                   render_colors, render_alphas, last_ids);
  }
}

// CTAs of raster_fix_kernel.
inline unsigned fix_grid(const RArgs& a) {
  const int y0 = a.ty0 * a.ts, y1 = a.H < (a.ty0 + a.rows) * a.ts ? a.H : (a.ty0 + a.rows) * a.ts;
  const int64_t total = (int64_t)a.I * (y1 - y0) * a.W;
  return (unsigned)(total > 0 ? ceil_div(total, kFixPixels) : 1);
}

// The fix-up pass after a forward kernel.  (A variant that visited only the
// tiles the forward flagged, one CTA walking all of a tile's undecided
// pixels, was slower: the walks, not the scan, set this kernel's time, and
// the pixel-row CTAs spread them wider.)
template <int CH>
void launch_fix(const RArgs& a, float* rc, float* ra, int32_t* li, cudaStream_t s) {
  raster_fix_kernel<CH><<<fix_grid(a), kWalk, 0, s>>>(a, rc, ra, li);
}

// ------------------------------------------------------------------ backward

// Sum NV (<= 16) per-lane values over the warp.  After the call, lane l
// with (l & 1) == 0 holds the warp total of value index red_index(l).
template <int NV>
__device__ __forceinline__ float butterfly_reduce(float (&v)[16], int lane) {
  static_assert(NV <= 16, "at most 16 values");
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool hi = lane & 16;
    const float send = hi ? v[i] : v[i + 8];
    const float keep = hi ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool hi = lane & 8;
    const float send = hi ? v[i] : v[i + 4];
    const float keep = hi ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool hi = lane & 4;
    const float send = hi ? v[i] : v[i + 2];
    const float keep = hi ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool hi = lane & 2;
    const float send = hi ? v[0] : v[1];
    const float keep = hi ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return v[0];
}

__device__ __forceinline__ int red_index(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

// The same for the first 8 values (9 shuffles); afterwards lane l with
// (l & 3) == 0 holds the warp total of value red_index8(l).  v[8..15] are
// left untouched.
__device__ __forceinline__ float butterfly_reduce8(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool hi = lane & 16;
    const float send = hi ? v[i] : v[i + 4];
    const float keep = hi ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool hi = lane & 8;
    const float send = hi ? v[i] : v[i + 2];
    const float keep = hi ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const bool hi = lane & 4;
    const float send = hi ? v[0] : v[1];
    const float keep = hi ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return v[0];
}

__device__ __forceinline__ int red_index8(int lane) {
  return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
}

// Gradient terms per Gaussian: [0,1] v_xy, [2,3,4] v_conic, [5] v_opacity,
// [6,7] |v_xy| (absgrad), [8..8+CH) v_colors.  With CH <= 4 everything fits
// the 16-term butterfly; larger channel counts reduce colours separately.
template <int CH>
__global__ void raster_bwd_kernel(RArgs a, const float* __restrict__ render_alphas,
                                  const int32_t* __restrict__ last_ids,
                                  const float* __restrict__ v_render_colors,
                                  const float* __restrict__ v_render_alphas, int absgrad,
                                  float* __restrict__ v_means2d_abs, float* __restrict__ v_means2d,
                                  float* __restrict__ v_conics, float* __restrict__ v_colors,
                                  float* __restrict__ v_opacities,
                                  float* __restrict__ v_backgrounds) {
  extern __shared__ float smem[];
  constexpr int CHS = CH > 0 ? CH : 1;
  const int BLOCK = blockDim.x;
  const int ch = CH > 0 ? CH : a.CH;
  const int NT = 8 + ch;  // gradient terms per Gaussian
  float2* s_xy = reinterpret_cast<float2*>(smem);
  float4* s_co = reinterpret_cast<float4*>(smem + 2 * BLOCK);
  float2* s_sb = reinterpret_cast<float2*>(smem + 6 * BLOCK);  // sigma bounds
  float* s_col = smem + 8 * BLOCK;         // [BLOCK][ch]
  float* s_acc = s_col + BLOCK * ch;       // [BLOCK][NT]
  __shared__ int s_last;
  __shared__ float s_bg[kMaxChannels];

  const TileIdx ti = tile_of(a);
  const int image = ti.image, tile_x = ti.tile_x, tile_y = ti.tile_y;
  const int tid = threadIdx.x, lane = tid & 31;
  const int ly = tid / a.ts, lx = tid - ly * a.ts;
  const int x = tile_x * a.ts + lx, y = tile_y * a.ts + ly;
  const bool inside = tid < a.ts * a.ts && x < a.W && y < a.H;
  const int64_t pix = ((int64_t)image * a.H + y) * a.W + x;

  if (a.masks && !a.masks[ti.mask]) return;
  int start, end;
  tile_range(a, ti.slot, start, end);

  const float px = (float)x + 0.5f, py = (float)y + 0.5f;
  const float T_final = inside ? 1.0f - __ldg(render_alphas + pix) : 1.0f;
  float Tr = T_final;
  const int my_last = inside ? min(end - 1, __ldg(last_ids + pix)) : -1;
  const float v_ra = inside ? __ldg(v_render_alphas + pix) : 0.0f;
  float v_rc[CHS];
  float buf[CHS];
  float v_rc_dyn[CH > 0 ? 1 : kMaxChannels];
  float buf_dyn[CH > 0 ? 1 : kMaxChannels];
  if (CH > 0) {
#pragma unroll
    for (int c = 0; c < CHS; ++c) {
      v_rc[c] = inside ? __ldg(v_render_colors + pix * CHS + c) : 0.0f;
      buf[c] = 0.0f;
    }
  } else {
    for (int c = 0; c < ch; ++c) {
      v_rc_dyn[c] = inside ? __ldg(v_render_colors + pix * ch + c) : 0.0f;
      buf_dyn[c] = 0.0f;
    }
  }
  // v_backgrounds += T_final * v_render_colors, reduced over the CTA.
  if (tid < ch) s_bg[tid] = 0.0f;
  if (tid == 0) s_last = -1;
  __syncthreads();
  if (v_backgrounds) {
    for (int c = 0; c < ch; ++c) {
      const float v = warp_sum(inside ? T_final * (CH > 0 ? v_rc[c < CHS ? c : 0] : v_rc_dyn[c]) : 0.0f);
      if (lane == 0) atomicAdd(&s_bg[c], v);
    }
  }
  // Background dot product used by every v_alpha of this pixel.
  float bg_dot = 0.0f;
  if (a.backgrounds) {
    for (int c = 0; c < ch; ++c)
      bg_dot += __ldg(a.backgrounds + image * ch + c) * (CH > 0 ? v_rc[c < CHS ? c : 0] : v_rc_dyn[c]);
  }
  if (inside) atomicMax(&s_last, my_last);
  __syncthreads();
  if (v_backgrounds && tid < ch && s_bg[tid] != 0.0f)
    atomicAdd(v_backgrounds + image * ch + tid, s_bg[tid]);
  const int cta_last = s_last;

  for (int b_end = cta_last + 1; b_end > start; b_end -= BLOCK) {
    const int b0 = max(start, b_end - BLOCK);
    const int cnt = b_end - b0;
    __syncthreads();
    if (tid < cnt) {
      const int g = __ldg(a.flatten_ids + b0 + tid);
      const float o = __ldg(a.opacities + opac_index(a, g, image));
      s_xy[tid] = __ldg(reinterpret_cast<const float2*>(a.means2d) + g);
      s_co[tid] = make_float4(__ldg(a.conics + (int64_t)g * 3), __ldg(a.conics + (int64_t)g * 3 + 1),
                              __ldg(a.conics + (int64_t)g * 3 + 2), o);
      s_sb[tid] = entry_bounds(a, g, image, o);
      for (int c = 0; c < ch; ++c) s_col[tid * ch + c] = __ldg(a.colors + (int64_t)g * ch + c);
    }
    for (int i = tid; i < cnt * NT; i += BLOCK) s_acc[i] = 0.0f;
    __syncthreads();
    for (int j = cnt - 1; j >= 0; --j) {
      const int idx = b0 + j;
      bool valid = idx <= my_last;
      float vis = 0.0f, alpha = 0.0f, dx = 0.0f, dy = 0.0f;
      bool clamped = false;
      const float2 m = s_xy[j];
      const float4 co = s_co[j];
      if (valid) {
        const float2 sb = s_sb[j];
        dx = m.x - px;
        dy = m.y - py;
        const float sigma = gauss_sigma(dx, dy, co.x, co.y, co.z).s;
        valid = composited(sigma, keep_range(sb.x));
        clamped = !(sigma >= sb.y);  // the reference's !(o * vis <= 0.99)
        vis = __expf(-sigma);
        alpha = clamped ? kMaxAlpha : fminf(kMaxAlpha, __fmul_rn(co.w, vis));
      }
      if (!__any_sync(0xffffffffu, valid)) continue;
      float g[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) g[i] = 0.0f;
      float gdyn_scale = 0.0f;  // fac, for the runtime-channel colour terms
      if (valid) {
        const float ra = 1.0f / fmaxf(kMinOneMinusAlpha, 1.0f - alpha);
        Tr *= ra;
        const float fac = alpha * Tr;
        float v_alpha = 0.0f;
        if (CH > 0) {
#pragma unroll
          for (int c = 0; c < CHS; ++c) {
            const float col = s_col[j * CHS + c];
            g[8 + c] = fac * v_rc[c];
            v_alpha += (col * Tr - buf[c] * ra) * v_rc[c];
            buf[c] += col * fac;
          }
        } else {
          gdyn_scale = fac;
          for (int c = 0; c < ch; ++c) {
            const float col = s_col[j * ch + c];
            v_alpha += (col * Tr - buf_dyn[c] * ra) * v_rc_dyn[c];
            buf_dyn[c] += col * fac;
          }
        }
        v_alpha += T_final * ra * v_ra;
        if (a.backgrounds) v_alpha += -T_final * ra * bg_dot;
        if (!clamped) {
          const float v_sigma = -co.w * vis * v_alpha;
          const float vx = v_sigma * (co.x * dx + co.y * dy);
          const float vy = v_sigma * (co.y * dx + co.z * dy);
          g[0] = vx;
          g[1] = vy;
          g[2] = 0.5f * v_sigma * dx * dx;
          g[3] = v_sigma * dx * dy;
          g[4] = 0.5f * v_sigma * dy * dy;
          g[5] = vis * v_alpha;
          g[6] = fabsf(vx);
          g[7] = fabsf(vy);
        }
      }
      const float r = butterfly_reduce<16>(g, lane);
      const int ri = red_index(lane);
      const int nfix = CH > 0 ? 8 + CHS : 8;
      if ((lane & 1) == 0 && ri < nfix && r != 0.0f) atomicAdd(&s_acc[j * NT + ri], r);
      if (CH == 0) {
        for (int c = 0; c < ch; ++c) {
          const float v = warp_sum(valid ? gdyn_scale * v_rc_dyn[c] : 0.0f);
          if (lane == 0 && v != 0.0f) atomicAdd(&s_acc[j * NT + 8 + c], v);
        }
      }
    }
    __syncthreads();
    // Flush this batch: one global atomic per non-zero term.
    for (int i = tid; i < cnt * NT; i += BLOCK) {
      const float v = s_acc[i];
      if (v == 0.0f) continue;
      const int j = i / NT, k = i - j * NT;
      const int64_t gg = __ldg(a.flatten_ids + b0 + j);
      if (k < 2) atomicAdd(v_means2d + gg * 2 + k, v);
      else if (k < 5) atomicAdd(v_conics + gg * 3 + (k - 2), v);
      else if (k == 5) atomicAdd(v_opacities + opac_index(a, gg, image), v);
      else if (k < 8) {
        if (absgrad) atomicAdd(v_means2d_abs + gg * 2 + (k - 6), v);
      } else atomicAdd(v_colors + gg * ch + (k - 8), v);
    }
  }
}

// ------------------------------------------------------------------ 16x16 tiles
// The common 16x16 tile runs on 256 / P threads, each owning P pixels of one
// column: thread t has pixels (t % 16, t / 16 + q * 16 / P), q < P.  Per
// staged Gaussian the shared loads, the loop control and -- in the backward
// -- the warp reduction are shared by 32 P pixels per warp.  Gaussians are
// staged packed: a = (mean x, mean y, conic0, conic1), b = (conic2, opacity,
// col0, col1), c = (col2, col3), in batches of one per thread.  Per-pixel
// arithmetic is unchanged.
// P pixels per thread (256 / P threads per tile): P = 4 when the grid has
// enough tiles to fill every SM many times over; P = 1 for small grids,
// where a tile's CTA must bring more warps of its own to hide latency.
constexpr int kT16Pixels = 4;
constexpr int kT16SmallPixels = 1;

// Stage the batch [b0, b0 + 128) of the tile's intersection list: thread t
// loads entry b0 + t, tests it against the tile, and the kept entries are
// compacted in list order into the packed shared arrays.  Returns the
// number kept.  Entries: a = (mean x, mean y, conic0, conic1),
// b = (conic2, opacity, col0, col1), c = (col2, col3), d = (upper end of
// the composited sigma range, clamp bound), its lower end, the
// intersection index and the Gaussian id.
template <int CH, int THREADS>
__device__ __forceinline__ int stage16(const RArgs& a, int image, int b0, int end, float x0,
                                       float y0,
                                       float4* sa, float4* sb, float2* sc, float2* sd,
                                       float* slo, int* sidx,
                                       int* sgid, int* swcnt) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int idx = b0 + tid;
  bool keep = false;
  int g = 0;
  if (idx < end) {
    g = __ldg(a.flatten_ids + idx);
    const float2 m = __ldg(reinterpret_cast<const float2*>(a.means2d) + g);
    const float* con = a.conics + (int64_t)g * 3;
    keep = tile_may_hit(m.x, m.y, __ldg(con), __ldg(con + 1), __ldg(con + 2),
                        __ldg(a.opacities + opac_index(a, g, image)), x0, y0);
  }
  const unsigned bal = __ballot_sync(0xffffffffu, keep);
  if (lane == 0) swcnt[warp] = __popc(bal);
  __syncthreads();
  int base = 0, cnt = 0;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) {
    const int c = swcnt[w];
    base += w < warp ? c : 0;
    cnt += c;
  }
  if (keep) {
    // the record is re-read (L1 hits) rather than held across the barrier
    const int slot = base + __popc(bal & ((1u << lane) - 1u));
    const float2 m = __ldg(reinterpret_cast<const float2*>(a.means2d) + g);
    const float* con = a.conics + (int64_t)g * 3;
    const float* col = a.colors + (int64_t)g * CH;
    float cc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int c = 0; c < CH; ++c) cc[c] = __ldg(col + c);
    const float o = __ldg(a.opacities + opac_index(a, g, image));
    sa[slot] = make_float4(m.x, m.y, __ldg(con), __ldg(con + 1));
    sb[slot] = make_float4(__ldg(con + 2), o, cc[0], cc[1]);
    sc[slot] = make_float2(cc[2], cc[3]);
    // the composited range's upper end and the clamp bound; the lower end
    // apart (0 but for the -inf opacity marker)
    const float2 bnd = entry_bounds(a, g, image, o);
    const Range rg = keep_range(bnd.x);
    sd[slot] = make_float2(rg.hi, bnd.y);
    slo[slot] = rg.lo;
    sidx[slot] = idx;
    if (sgid) sgid[slot] = g;
  }
  __syncthreads();
  return cnt;
}

// Returns 0 while the pixel goes on, 1 once it stopped, 2 when its stop
// decision is left to the exact walk.
template <int CH>
__device__ __forceinline__ int composite16(float dx, float dy, const float4& A, const float4& B,
                                           float2 sb, Range r, float dg, const float* col,
                                           float& Tr,
                                           float& E, float* acc, int& cur, int idx) {
  const float sigma = gauss_sigma(dx, dy, A.z, A.w, B.x).s;
  if (!composited(sigma, r)) return 0;
  const bool clamped = !(sigma >= sb.y);  // o e^-sigma > 0.99 (or NaN)
  const float alpha = fast_alpha(sigma, B.y, clamped);
  const float vis = alpha * Tr;
  const float next_T = __fmaf_rn(-alpha, Tr, Tr);
  const float nE = step_bound(E, vis, 1.0f - alpha, next_T, dg, clamped);
  if (const int st = stop_decision(next_T, nE)) return st;
  E = nE;
#pragma unroll
  for (int c = 0; c < CH; ++c) acc[c] += col[c] * vis;
  cur = idx;
  Tr = next_T;
  return 0;
}

// Both 16x16 kernels are capped at 64 registers (16 CTAs of 64 threads per
// SM at P = 4): a few bytes of spill outside the Gaussian loop, ~2% faster
// than the 71-72 registers (14 CTAs) the compiler picks on its own.
template <int CH, int P>
__global__ void __launch_bounds__(256 / P, 4 * P) raster_fwd16_kernel(
    RArgs a, float* __restrict__ render_colors, float* __restrict__ render_alphas,
    int32_t* __restrict__ last_ids) {
  constexpr int THREADS = 256 / P, RS = 16 / P;  // threads, row stride of a thread's pixels
  __shared__ float4 s_a[THREADS];
  __shared__ float4 s_b[THREADS];
  __shared__ float2 s_c[THREADS];
  __shared__ float2 s_d[THREADS];
  __shared__ float s_lo[THREADS];
  __shared__ int s_idx[THREADS];
  __shared__ int s_wcnt[THREADS / 32];
  __shared__ int s_cost;
  const TileIdx ti = tile_of(a);
  const int image = ti.image, tile_x = ti.tile_x, tile_y = ti.tile_y;
  const int tid = threadIdx.x;
  const int x = tile_x * 16 + (tid & 15);
  const int ybase = tile_y * 16 + (tid >> 4);
  bool in[P];
#pragma unroll
  for (int q = 0; q < P; ++q) in[q] = x < a.W && ybase + q * RS < a.H;
  const int64_t pix0 = ((int64_t)image * a.H + ybase) * a.W + x;

  if (a.masks && !a.masks[ti.mask]) {
#pragma unroll
    for (int q = 0; q < P; ++q) {
      if (!in[q]) continue;
      const int64_t pix = pix0 + (int64_t)q * RS * a.W;
#pragma unroll
      for (int c = 0; c < CH; ++c)
        render_colors[pix * CH + c] = a.backgrounds ? __ldg(a.backgrounds + image * CH + c) : 0.0f;
      render_alphas[pix] = 0.0f;
      last_ids[pix] = 0;
    }
    if (a.tile_cost && tid == 0) a.tile_cost[ti.slot] = 0;
    return;
  }
  if (tid == 0) s_cost = -1;
  int start, end;
  tile_range(a, ti.slot, start, end);
  const float px = (float)x + 0.5f;
  float py[P], Tr[P], tb[P], acc[P][CH];
  int cur[P];
  unsigned dn = 0u, uns = 0u;  // bit q: pixel q stopped / left to the exact walk
#pragma unroll
  for (int q = 0; q < P; ++q) {
    py[q] = (float)(ybase + q * RS) + 0.5f;
    Tr[q] = 1.0f;
    tb[q] = 0.0f;
    cur[q] = 0;
    dn |= in[q] ? 0u : 1u << q;
#pragma unroll
    for (int c = 0; c < CH; ++c) acc[q][c] = 0.0f;
  }
  auto all_done = [&]() { return dn == (1u << P) - 1u; };

  for (int b0 = start; b0 < end; b0 += THREADS) {
    if (__syncthreads_count(!all_done()) == 0) break;
    const int cnt = stage16<CH, THREADS>(a, image, b0, end, tile_x * 16 + 0.5f, tile_y * 16 + 0.5f, s_a,
                                         s_b, s_c, s_d, s_lo, s_idx, nullptr, s_wcnt);
    for (int j = 0; j < cnt; ++j) {
      if (all_done()) break;
      const float4 A = s_a[j];
      const float4 B = s_b[j];
      const float2 sb = s_d[j];
      float col[4] = {B.z, B.w, 0.0f, 0.0f};
      if (CH > 2) {
        const float2 C = s_c[j];
        col[2] = C.x;
        col[3] = C.y;
      }
      const float dx = A.x - px;
      const int idx = s_idx[j];
      const float dg = alpha_err(sb.x);
      const Range r{s_lo[j], sb.x};
#pragma unroll
      for (int q = 0; q < P; ++q)
        if (!(dn >> q & 1u)) {
          const int st = composite16<CH>(dx, A.y - py[q], A, B, sb, r, dg, col, Tr[q], tb[q],
                                         acc[q], cur[q], idx);
          if (st) {
            dn |= 1u << q;
            if (st == 2) uns |= 1u << q;
          }
        }
    }
  }
#pragma unroll
  for (int q = 0; q < P; ++q) {
    if (!in[q] || (uns >> q & 1u)) continue;
    const int64_t pix = pix0 + (int64_t)q * RS * a.W;
    render_alphas[pix] = 1.0f - Tr[q];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const float bg = a.backgrounds ? __ldg(a.backgrounds + image * CH + c) : 0.0f;
      render_colors[pix * CH + c] = acc[q][c] + Tr[q] * bg;
    }
    last_ids[pix] = cur[q];
  }
  // pixels whose stop decision fell within the error bound are left to
  // raster_fix_kernel
  int my = -1;
#pragma unroll
  for (int q = 0; q < P; ++q) {
    if (uns >> q & 1u) last_ids[pix0 + (int64_t)q * RS * a.W] = kUndecided;
    if (in[q]) my = max(my, (uns >> q & 1u) ? end - 1 : min(end - 1, cur[q]));
  }
  record_tile_cost(a, ti.slot, start, my, &s_cost);
}

// Reverse step of one pixel for one Gaussian (gsplat_rasterize.cpp:503-562);
// adds the pixel's contributions to the Gaussian's gradient terms g[]:
// [0,1] v_xy, [2,3,4] v_conic (terms 2 and 4 doubled, halved once at the
// flush), [5] v_opacity, then with ABS [6,7] |v_xy| and [8..8+CH)
// v_colors, without ABS [6..6+CH) v_colors.
//
// The reference's per-channel terms are folded into scalars per pixel:
//   v_alpha = sum_c (col_c T - buf_c ra) vrc_c + ra T_final (v_ra - bg.vrc)
//           = T (col.vrc) + ra (K - bufdot),
// with K = T_final (v_ra - bg.vrc) fixed per pixel and bufdot = buf.vrc
// advanced by fac (col.vrc) -- the same sums in fewer operations.
// 1 / (1 - alpha) uses the fast reciprocal (2 ulp; alpha <= 0.99 keeps its
// argument in [0.01, 1]).
template <int CH, bool ABS>
__device__ __forceinline__ bool backward16(bool in_range, float dx, float dy, const float4& A,
                                           const float4& B, float2 sb, Range r, const float* col,
                                           float& Tr, float& bufdot, float K, const float* v_rc,
                                           float* g) {
  if (!in_range) return false;
  const Sigma sg = gauss_sigma(dx, dy, A.z, A.w, B.x);
  if (!composited(sg.s, r)) return false;
  const bool clamped = !(sg.s >= sb.y);  // the reference's !(o * vis <= 0.99)
  const float vis = __expf(-sg.s);
  const float ov = __fmul_rn(B.y, vis);
  const float alpha = clamped ? kMaxAlpha : fminf(kMaxAlpha, ov);
  // alpha <= 0.99, so 1 - alpha >= 0.01 and the reference's max(1e-6, .)
  // never binds
  const float ra = __fdividef(1.0f, 1.0f - alpha);
  Tr *= ra;
  const float fac = alpha * Tr;
  float cdot = col[0] * v_rc[0];
#pragma unroll
  for (int c = 1; c < CH; ++c) cdot = fmaf(col[c], v_rc[c], cdot);
#pragma unroll
  for (int c = 0; c < CH; ++c) g[(ABS ? 8 : 6) + c] = fmaf(fac, v_rc[c], g[(ABS ? 8 : 6) + c]);
  const float v_alpha = fmaf(Tr, cdot, ra * (K - bufdot));
  bufdot = fmaf(fac, cdot, bufdot);
  if (!clamped) {
    const float v_sigma = -ov * v_alpha;
    const float vsdx = v_sigma * dx, vsdy = v_sigma * dy;
    const float vx = fmaf(A.w, vsdy, v_sigma * sg.cdx);   // v_sigma (c0 dx + c1 dy)
    const float vy = fmaf(A.w, vsdx, v_sigma * sg.cdy);   // v_sigma (c1 dx + c2 dy)
    g[0] += vx;
    g[1] += vy;
    g[2] = fmaf(vsdx, dx, g[2]);  // halved at the flush (exact: a power of two)
    g[3] = fmaf(vsdx, dy, g[3]);
    g[4] = fmaf(vsdy, dy, g[4]);  // halved at the flush
    g[5] = fmaf(vis, v_alpha, g[5]);
    if (ABS) {
      g[6] += fabsf(vx);
      g[7] += fabsf(vy);
    }
  }
  return true;
}

template <int CH, bool ABS, int P>
__global__ void __launch_bounds__(256 / P, 4 * P) raster_bwd16_kernel(
    RArgs a, const float* __restrict__ render_alphas, const int32_t* __restrict__ last_ids,
    const float* __restrict__ v_render_colors, const float* __restrict__ v_render_alphas,
    int absgrad, float* __restrict__ v_means2d_abs, float* __restrict__ v_means2d,
    float* __restrict__ v_conics, float* __restrict__ v_colors, float* __restrict__ v_opacities,
    float* __restrict__ v_backgrounds) {
  constexpr int THREADS = 256 / P, RS = 16 / P;  // threads, row stride of a thread's pixels
  constexpr int CB = ABS ? 8 : 6;  // index of the first colour term
  constexpr int NT = CB + CH;      // gradient terms per Gaussian
  __shared__ float4 s_a[THREADS];
  __shared__ float4 s_b[THREADS];
  __shared__ float2 s_c[THREADS];
  __shared__ float2 s_d[THREADS];
  __shared__ float s_lo[THREADS];
  __shared__ int s_idx[THREADS];
  __shared__ int s_gid[THREADS];
  __shared__ int s_wcnt[THREADS / 32];
  __shared__ float s_acc[THREADS * NT];
  __shared__ int s_last;
  __shared__ float s_bg[4];
  const TileIdx ti = tile_of(a);
  const int image = ti.image, tile_x = ti.tile_x, tile_y = ti.tile_y;
  const int tid = threadIdx.x, lane = tid & 31;
  const int x = tile_x * 16 + (tid & 15);
  const int ybase = tile_y * 16 + (tid >> 4);
  if (a.masks && !a.masks[ti.mask]) return;
  int start, end;
  tile_range(a, ti.slot, start, end);
  const float px = (float)x + 0.5f;
  // per pixel: centre row, transmittance, last id, K = T_final (v_ra - bg.vrc),
  // bufdot, colour cotangent
  float py[P], Tr[P], K[P], bufdot[P], vrc[P][CH];
  int last[P];
  bool in[P];
  int my_last = -1;
  float bgsum[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) bgsum[c] = 0.0f;
#pragma unroll
  for (int q = 0; q < P; ++q) {
    const int y = ybase + q * RS;
    in[q] = x < a.W && y < a.H;
    const int64_t pix = ((int64_t)image * a.H + y) * a.W + x;
    py[q] = (float)y + 0.5f;
    const float Tf = in[q] ? 1.0f - __ldg(render_alphas + pix) : 1.0f;
    Tr[q] = Tf;
    last[q] = in[q] ? min(end - 1, __ldg(last_ids + pix)) : -1;
    my_last = max(my_last, last[q]);
    const float vra = in[q] ? __ldg(v_render_alphas + pix) : 0.0f;
    float bgd = 0.0f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      vrc[q][c] = in[q] ? __ldg(v_render_colors + pix * CH + c) : 0.0f;
      if (a.backgrounds) bgd += __ldg(a.backgrounds + image * CH + c) * vrc[q][c];
      bgsum[c] += in[q] ? Tf * vrc[q][c] : 0.0f;
    }
    K[q] = Tf * (vra - bgd);
    bufdot[q] = 0.0f;
  }
  if (tid < 4) s_bg[tid] = 0.0f;
  if (tid == 0) s_last = -1;
  __syncthreads();
  if (v_backgrounds) {
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const float v = warp_sum(bgsum[c]);
      if (lane == 0) atomicAdd(&s_bg[c], v);
    }
  }
  if (my_last >= 0) atomicMax(&s_last, my_last);
  __syncthreads();
  if (v_backgrounds && tid < CH && s_bg[tid] != 0.0f)
    atomicAdd(v_backgrounds + image * CH + tid, s_bg[tid]);
  const int cta_last = s_last;

  for (int b_end = cta_last + 1; b_end > start; b_end -= THREADS) {
    const int b0 = max(start, b_end - THREADS);
    __syncthreads();
    const int cnt = stage16<CH, THREADS>(a, image, b0, b_end, tile_x * 16 + 0.5f, tile_y * 16 + 0.5f,
                                         s_a, s_b, s_c, s_d, s_lo, s_idx, s_gid, s_wcnt);
    for (int i = tid; i < cnt * NT; i += THREADS) s_acc[i] = 0.0f;
    __syncthreads();
    for (int j = cnt - 1; j >= 0; --j) {
      const int idx = s_idx[j];
      const float4 A = s_a[j];
      const float4 B = s_b[j];
      float col[4] = {B.z, B.w, 0.0f, 0.0f};
      if (CH > 2) {
        const float2 C = s_c[j];
        col[2] = C.x;
        col[3] = C.y;
      }
      float g[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) g[i] = 0.0f;
      const float dx = A.x - px;
      const float2 sb = s_d[j];
      const Range r{s_lo[j], sb.x};
      bool any = false;
#pragma unroll
      for (int q = 0; q < P; ++q)
        any |= backward16<CH, ABS>(idx <= last[q], dx, A.y - py[q], A, B, sb, r, col, Tr[q],
                                   bufdot[q], K[q], vrc[q], g);
      const unsigned active = __ballot_sync(0xffffffffu, any);
      if (!active) continue;
      if (__popc(active) <= 2) {
        // Sparse warp: its one or two contributing lanes add directly.
        if (any) {
#pragma unroll
          for (int k = 0; k < NT; ++k)
            if (g[k] != 0.0f) atomicAdd(&s_acc[j * NT + k], g[k]);
        }
      } else if (NT <= 10) {
        // terms 0..7 by the 8-value butterfly, the rest (<= 2) by warp sums
        const float r = butterfly_reduce8(g, lane);
        const int ri = red_index8(lane);
        if ((lane & 3) == 0 && ri < NT && r != 0.0f) atomicAdd(&s_acc[j * NT + ri], r);
#pragma unroll
        for (int k = 8; k < NT; ++k) {
          const float v = warp_sum(g[k]);
          if (lane == 0 && v != 0.0f) atomicAdd(&s_acc[j * NT + k], v);
        }
      } else {
        const float r = butterfly_reduce<16>(g, lane);
        const int ri = red_index(lane);
        if ((lane & 1) == 0 && ri < NT && r != 0.0f) atomicAdd(&s_acc[j * NT + ri], r);
      }
    }
    __syncthreads();
    for (int i = tid; i < cnt * NT; i += THREADS) {
      const float v = s_acc[i];
      if (v == 0.0f) continue;
      const int j = i / NT, k = i - j * NT;
      const int64_t gg = s_gid[j];
      if (k < 2) atomicAdd(v_means2d + gg * 2 + k, v);
      else if (k < 5) atomicAdd(v_conics + gg * 3 + (k - 2), k == 3 ? v : 0.5f * v);
      else if (k == 5) atomicAdd(v_opacities + opac_index(a, gg, image), v);
      else if (k < CB) atomicAdd(v_means2d_abs + gg * 2 + (k - 6), v);  // ABS only
      else atomicAdd(v_colors + gg * CH + (k - CB), v);
    }
  }
}

// Bounds of every opacity; with radii ([cameras, n, 2]) only of the
// Gaussians some camera sees (no intersection lists the others).
__global__ void sigma_bounds_kernel(int64_t n, const float* __restrict__ opacities,
                                    const int2* __restrict__ radii, int cameras,
                                    float2* __restrict__ bounds) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (radii) {
      bool seen = false;
      for (int c = 0; c < cameras && !seen; ++c) {
        const int2 r = __ldg(radii + (int64_t)c * n + i);
        seen = r.x > 0 && r.y > 0;
      }
      if (!seen) continue;
    }
    bounds[i] = sigma_bounds(__ldg(opacities + i));
  }
}

int smem_bytes(int block, int ch, bool bwd) {
  return (int)sizeof(float) * (block * (8 + ch) + (bwd ? block * (8 + ch) : 0));
}

// Fewer tiles than 8 per SM: the four-pixel kernels' two-warp CTAs would
// leave most schedulers without a warp to switch to.
inline bool small_grid(int64_t tiles) { return tiles < 8 * (int64_t)sm_count(); }

template <int CH>
int launch_fwd(const RArgs& a, int block, float* rc, float* ra, int32_t* li, cudaStream_t s) {
  if (CH > 0 && a.ts == 16) {
    constexpr int C1 = CH > 0 ? CH : 1;
    const int64_t tiles = (int64_t)a.I * a.rows * a.tw;
    if (small_grid(tiles))
      raster_fwd16_kernel<C1, kT16SmallPixels><<<(unsigned)tiles, 256 / kT16SmallPixels, 0, s>>>(
          a, rc, ra, li);
    else
      raster_fwd16_kernel<C1, kT16Pixels><<<(unsigned)tiles, 256 / kT16Pixels, 0, s>>>(a, rc, ra,
                                                                                        li);
    launch_fix<C1>(a, rc, ra, li, s);
    return launch_status("rasterize_fwd");
  }
  const int smem = smem_bytes(block, a.CH, false);
  cudaFuncSetAttribute(raster_fwd_kernel<CH>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int64_t tiles = (int64_t)a.I * a.rows * a.tw;
  raster_fwd_kernel<CH><<<(unsigned)tiles, block, smem, s>>>(a, rc, ra, li);
  launch_fix<CH>(a, rc, ra, li, s);
  return launch_status("rasterize_fwd");
}

template <int CH>
int launch_bwd(const RArgs& a, int block, const float* ra, const int32_t* li, const float* vrc,
               const float* vra, int absgrad, float* vabs, float* vm, float* vc, float* vcol,
               float* vop, float* vbg, cudaStream_t s) {
  if (CH > 0 && a.ts == 16) {
    constexpr int C1 = CH > 0 ? CH : 1;
    const int64_t tiles = (int64_t)a.I * a.rows * a.tw;
    const unsigned grid = (unsigned)tiles;
    constexpr int PS = kT16SmallPixels, PL = kT16Pixels;
    if (small_grid(tiles) && absgrad)
      raster_bwd16_kernel<C1, true, PS><<<grid, 256 / PS, 0, s>>>(a, ra, li, vrc, vra, absgrad,
                                                                  vabs, vm, vc, vcol, vop, vbg);
    else if (small_grid(tiles))
      raster_bwd16_kernel<C1, false, PS><<<grid, 256 / PS, 0, s>>>(a, ra, li, vrc, vra, absgrad,
                                                                   vabs, vm, vc, vcol, vop, vbg);
    else if (absgrad)
      raster_bwd16_kernel<C1, true, PL><<<grid, 256 / PL, 0, s>>>(a, ra, li, vrc, vra, absgrad,
                                                                  vabs, vm, vc, vcol, vop, vbg);
    else
      raster_bwd16_kernel<C1, false, PL><<<grid, 256 / PL, 0, s>>>(a, ra, li, vrc, vra, absgrad,
                                                                   vabs, vm, vc, vcol, vop, vbg);
    return launch_status("rasterize_bwd");
  }
  const int smem = smem_bytes(block, a.CH, true);
  cudaFuncSetAttribute(raster_bwd_kernel<CH>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int64_t tiles = (int64_t)a.I * a.rows * a.tw;
  raster_bwd_kernel<CH><<<(unsigned)tiles, block, smem, s>>>(a, ra, li, vrc, vra, absgrad, vabs, vm,
                                                             vc, vcol, vop, vbg);
  return launch_status("rasterize_bwd");
}

int check_raster(const gs_raster_params* p) {
  if (!p) return invalid("rasterize: params missing");
  if (p->I <= 0 || p->N < 0 || p->channels <= 0 || p->image_width < 0 || p->image_height < 0 ||
      p->n_isects < 0)
    return invalid("rasterize: bad params");
  if (p->tile_size <= 0 || p->tile_size > 32)
    return invalid("rasterize: tile_size must be in 1..32");
  if (p->tile_width <= 0 || p->tile_height <= 0) return invalid("rasterize: bad tile grid");
  if ((int64_t)p->tile_width * p->tile_size < p->image_width ||
      (int64_t)p->tile_height * p->tile_size < p->image_height)
    return invalid("rasterize: tile grid does not cover the image");
  if (p->n_isects > INT32_MAX) {
    set_error("rasterize: more than 2^31 intersections");
    return GS_ERR_OVERFLOW;
  }
  if ((int64_t)p->I * p->tile_width * p->tile_height > INT32_MAX)
    return invalid("rasterize: too many tiles");
  if (p->tile_y1 > p->tile_y0 && (p->tile_y0 < 0 || p->tile_y1 > p->tile_height))
    return invalid("rasterize: bad tile-row window");
  return GS_OK;
}

RArgs make_args(const gs_raster_params* p, const float* means2d, const float* conics,
                const float* colors, const float* opacities, const float* backgrounds,
                const uint8_t* masks, const int32_t* tile_offsets, const int32_t* flatten_ids) {
  int ty0 = 0, rows = p->tile_height;
  if (p->tile_y1 > p->tile_y0) {
    ty0 = p->tile_y0;
    rows = p->tile_y1 - p->tile_y0;
  }
  return RArgs{p->I, p->N, p->channels, p->image_width, p->image_height, p->tile_size,
               p->tile_width, p->tile_height, ty0, rows, p->shared_opacities ? 1 : 0,
               p->n_isects, means2d, conics, colors,
               opacities,
               p->use_backgrounds ? backgrounds : nullptr, p->use_masks ? masks : nullptr,
               tile_offsets, flatten_ids,
               reinterpret_cast<const float2*>(p->sigma_bounds), p->tile_order, p->tile_cost};
}

// Schedule of the rasterizer's CTAs: the slots in descending order of their
// intersection-list length, bucketed at 1/8-octave steps (bucket = 8 floor
// log2 len + the next three bits of len).  The hardware hands CTAs to SMs
// in blockIdx order, so the longest tiles start first and the short ones
// fill in behind them (longest-processing-time-first), instead of a long
// tile that happens to come last running alone on an otherwise idle GPU.
// One CTA: a shared histogram of the buckets, its scan, a scatter.  The
// order inside a bucket is that of the shared atomics; it changes no
// output, only which SM renders which tile when.
constexpr int kOrderThreads = 1024;
constexpr int kOrderBuckets = 256;

__device__ __forceinline__ int length_bucket(int len) {
  if (len <= 0) return 0;
  const int lz = 31 - __clz(len);
  const int frac = lz >= 3 ? (len >> (lz - 3)) & 7 : (len << (3 - lz)) & 7;
  return min(kOrderBuckets - 1, lz * 8 + frac + 1);
}

__device__ __forceinline__ int slot_cost(const RArgs& a, const int32_t* cost, int t) {
  if (cost) return __ldg(cost + t);
  int start, end;
  tile_range(a, t, start, end);
  return end - start;
}

// Slots whose buckets the kernel keeps in shared memory between its passes
// (more are recomputed in the second pass).
constexpr int kOrderKeep = 32768;

// Whether a rasterizer call follows its tile_order: grids of more tiles than
// kOrderKeep (about 14 waves of the 16x16 kernels) keep slot order -- their
// last wave is a small share of the work, and one CTA would take longer to
// order them than the balance gains.
inline bool scheduled(const RArgs& a) {
  return a.tile_order && (int64_t)a.I * a.rows * a.tw <= kOrderKeep;
}
constexpr int kOrderUnroll = 4;

__global__ void __launch_bounds__(kOrderThreads) tile_order_kernel(RArgs a,
                                                                  const int32_t* __restrict__ cost,
                                                                  int32_t* __restrict__ order) {
  __shared__ int hist[kOrderBuckets];
  __shared__ uint8_t s_bucket[kOrderKeep];
  const int n_slots = a.I * a.rows * a.tw;
  const bool keep = n_slots <= kOrderKeep;
  for (int i = threadIdx.x; i < kOrderBuckets; i += kOrderThreads) hist[i] = 0;
  __syncthreads();
  for (int t0 = threadIdx.x; t0 < n_slots; t0 += kOrderUnroll * kOrderThreads) {
    int b[kOrderUnroll];
#pragma unroll
    for (int u = 0; u < kOrderUnroll; ++u) {  // the loads of every slot in flight first
      const int t = t0 + u * kOrderThreads;
      b[u] = t < n_slots ? slot_cost(a, cost, t) : -1;
    }
#pragma unroll
    for (int u = 0; u < kOrderUnroll; ++u) {
      const int t = t0 + u * kOrderThreads;
      if (t >= n_slots) break;
      const int bk = length_bucket(b[u]);
      if (keep) s_bucket[t] = (uint8_t)bk;
      atomicAdd(&hist[kOrderBuckets - 1 - bk], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // exclusive scan of the 256 counts by one warp, 8 per lane
    const int lane = threadIdx.x;
    int v[8], sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      v[k] = hist[lane * 8 + k];
      sum += v[k];
    }
    int incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += u;
    }
    int run = incl - sum;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      hist[lane * 8 + k] = run;
      run += v[k];
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < n_slots; t += kOrderThreads) {
    const int bk = keep ? (int)s_bucket[t] : length_bucket(slot_cost(a, cost, t));
    order[atomicAdd(&hist[kOrderBuckets - 1 - bk], 1)] = t;
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gs_rasterize_fwd(const gs_raster_params* p, const float* means2d,
                                const float* conics, const float* colors, const float* opacities,
                                const float* backgrounds, const uint8_t* masks,
                                const int32_t* tile_offsets, const int32_t* flatten_ids,
                                float* render_colors, float* render_alphas, int32_t* last_ids,
                                gs_stream_t stream) {
  if (int rc = check_raster(p)) return rc;
  if (p->channels > kMaxChannels) return invalid("rasterize: at most 64 channels");
  if ((int64_t)p->image_width * p->image_height == 0) return GS_OK;
  if (!render_colors || !render_alphas || !last_ids || !tile_offsets)
    return invalid("rasterize_fwd: missing output buffer");
  if (p->n_isects > 0 && (!means2d || !conics || !colors || !opacities || !flatten_ids))
    return invalid("rasterize_fwd: missing input buffer");
  if ((p->use_backgrounds && !backgrounds) || (p->use_masks && !masks))
    return invalid("rasterize_fwd: missing backgrounds/masks");
  if (reinterpret_cast<uintptr_t>(means2d) % 8) return invalid("rasterize_fwd: means2d must be 8-byte aligned");
  if (reinterpret_cast<uintptr_t>(p->sigma_bounds) % 8)
    return invalid("rasterize_fwd: sigma_bounds must be 8-byte aligned");
  RArgs a = make_args(p, means2d, conics, colors, opacities, backgrounds, masks, tile_offsets,
                      flatten_ids);
  const int block = ((p->tile_size * p->tile_size + 31) / 32) * 32;
  cudaStream_t s = as_stream(stream);
  // the schedule: longest tile lists first
  if (!scheduled(a)) a.tile_order = nullptr;
  if (a.tile_order) tile_order_kernel<<<1, kOrderThreads, 0, s>>>(a, nullptr, p->tile_order);
  switch (p->channels) {
    case 1: return launch_fwd<1>(a, block, render_colors, render_alphas, last_ids, s);
    case 2: return launch_fwd<2>(a, block, render_colors, render_alphas, last_ids, s);
    case 3: return launch_fwd<3>(a, block, render_colors, render_alphas, last_ids, s);
    case 4: return launch_fwd<4>(a, block, render_colors, render_alphas, last_ids, s);
    default: return launch_fwd<0>(a, block, render_colors, render_alphas, last_ids, s);
  }
}

extern "C" int gs_rasterize_bwd(const gs_raster_params* p, const float* means2d,
                                const float* conics, const float* colors, const float* opacities,
                                const float* backgrounds, const uint8_t* masks,
                                const int32_t* tile_offsets, const int32_t* flatten_ids,
                                const float* render_alphas, const int32_t* last_ids,
                                const float* v_render_colors, const float* v_render_alphas,
                                float* v_means2d_abs, float* v_means2d, float* v_conics,
                                float* v_colors, float* v_opacities, float* v_backgrounds,
                                gs_stream_t stream) {
  if (int rc = check_raster(p)) return rc;
  if (p->channels > kMaxChannels) return invalid("rasterize_bwd: at most 64 channels");
  if (!v_means2d || !v_conics || !v_colors || !v_opacities)
    return invalid("rasterize_bwd: missing gradient buffer");
  if (p->absgrad && !v_means2d_abs) return invalid("rasterize_bwd: v_means2d_abs missing");
  if ((p->use_backgrounds && (!backgrounds || !v_backgrounds)) || (p->use_masks && !masks))
    return invalid("rasterize_bwd: missing backgrounds/masks");
  cudaStream_t s = as_stream(stream);
  const int64_t nG = (int64_t)p->I * p->N;
  const size_t f = sizeof(float);
  if (nG > 0 && !p->accumulate) {
    if (cudaMemsetAsync(v_means2d, 0, f * 2 * nG, s) || cudaMemsetAsync(v_conics, 0, f * 3 * nG, s) ||
        cudaMemsetAsync(v_colors, 0, f * p->channels * nG, s) ||
        cudaMemsetAsync(v_opacities, 0, f * (p->shared_opacities ? (int64_t)p->N : nG), s) ||
        (p->absgrad && cudaMemsetAsync(v_means2d_abs, 0, f * 2 * nG, s)))
      return launch_status("rasterize_bwd: zero gradients");
  }
  if (p->use_backgrounds && !p->accumulate &&
      cudaMemsetAsync(v_backgrounds, 0, f * p->I * p->channels, s))
    return launch_status("rasterize_bwd: zero v_backgrounds");
  if ((int64_t)p->image_width * p->image_height == 0) return launch_status("rasterize_bwd");
  if (!tile_offsets || !render_alphas || !last_ids || !v_render_colors || !v_render_alphas)
    return invalid("rasterize_bwd: missing input buffer");
  if (p->n_isects > 0 && (!means2d || !conics || !colors || !opacities || !flatten_ids))
    return invalid("rasterize_bwd: missing input buffer");
  if (reinterpret_cast<uintptr_t>(means2d) % 8) return invalid("rasterize_bwd: means2d must be 8-byte aligned");
  if (reinterpret_cast<uintptr_t>(p->sigma_bounds) % 8)
    return invalid("rasterize_bwd: sigma_bounds must be 8-byte aligned");
  RArgs a = make_args(p, means2d, conics, colors, opacities, backgrounds, masks, tile_offsets,
                      flatten_ids);
  const int block = ((p->tile_size * p->tile_size + 31) / 32) * 32;
  float* vbg = p->use_backgrounds ? v_backgrounds : nullptr;
  // the schedule: costliest tiles (by the forward's record, else by list
  // length) first
  if (!scheduled(a)) a.tile_order = nullptr;
  if (a.tile_order) tile_order_kernel<<<1, kOrderThreads, 0, s>>>(a, p->tile_cost, p->tile_order);
  switch (p->channels) {
    case 1: return launch_bwd<1>(a, block, render_alphas, last_ids, v_render_colors, v_render_alphas, p->absgrad, v_means2d_abs, v_means2d, v_conics, v_colors, v_opacities, vbg, s);
    case 2: return launch_bwd<2>(a, block, render_alphas, last_ids, v_render_colors, v_render_alphas, p->absgrad, v_means2d_abs, v_means2d, v_conics, v_colors, v_opacities, vbg, s);
    case 3: return launch_bwd<3>(a, block, render_alphas, last_ids, v_render_colors, v_render_alphas, p->absgrad, v_means2d_abs, v_means2d, v_conics, v_colors, v_opacities, vbg, s);
    case 4: return launch_bwd<4>(a, block, render_alphas, last_ids, v_render_colors, v_render_alphas, p->absgrad, v_means2d_abs, v_means2d, v_conics, v_colors, v_opacities, vbg, s);
    default: return launch_bwd<0>(a, block, render_alphas, last_ids, v_render_colors, v_render_alphas, p->absgrad, v_means2d_abs, v_means2d, v_conics, v_colors, v_opacities, vbg, s);
  }
}

extern "C" int gs_raster_tile_order(const gs_raster_params* p, const int32_t* tile_offsets,
                                    const int32_t* tile_cost, int32_t* tile_order,
                                    gs_stream_t stream) {
  if (int rc = check_raster(p)) return rc;
  if (!tile_order || (!tile_offsets && !tile_cost))
    return invalid("raster_tile_order: missing buffer");
  gs_raster_params q = *p;
  q.tile_order = nullptr;
  q.tile_cost = nullptr;
  const RArgs a = make_args(&q, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                            tile_offsets, nullptr);
  tile_order_kernel<<<1, kOrderThreads, 0, as_stream(stream)>>>(a, tile_cost, tile_order);
  return launch_status("raster_tile_order");
}

extern "C" int gs_rasterize_sigma_bounds(int64_t n, const float* opacities,
                                         const int32_t* radii, int32_t cameras, float* bounds,
                                         gs_stream_t stream) {
  if (n < 0 || (radii && cameras <= 0)) return invalid("rasterize_sigma_bounds: bad sizes");
  if (n == 0) return GS_OK;
  if (!opacities || !bounds) return invalid("rasterize_sigma_bounds: missing buffer");
  if (reinterpret_cast<uintptr_t>(bounds) % 8 || reinterpret_cast<uintptr_t>(radii) % 8)
    return invalid("rasterize_sigma_bounds: bounds and radii must be 8-byte aligned");
  sigma_bounds_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
      n, opacities, reinterpret_cast<const int2*>(radii), cameras,
      reinterpret_cast<float2*>(bounds));
  return launch_status("rasterize_sigma_bounds");
}
