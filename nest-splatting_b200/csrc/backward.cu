// backward.cu -- gradients of the mode-0 surfel render with respect to the
// surfels (mean, scale, rotation, opacity) and the hash-grid table.
//
// Restates the reference's backward for render_mode 0, kernel_type 0, level > 0:
//   renderCUDAsurfelBackward (backward.cu:445-2052): per pixel, back to front
//   from the last contributor, T recovered by division (:914), the colour term
//   through the re-queried hash features (:934-980, :1786-1797), auxiliary
//   terms (depth, alpha, normal, median depth, distortion, :1799-1852), the
//   Gaussian kernel (:1854-1914), homotrans (:1921-1953) and transform / mean2D
//   grads (:1956-2045), opacity (:2048);
//   query_feature<true> (hashgrid.h:106-299): table-gradient scatter and dL/dxyz;
//   preprocessCUDA backward (:2216-2273) with compute_transmat_aabb (:2056-2214).
//
// Design (one CTA of kThreads = 16 x kRows threads per band of kRows rows of a
// 16x16 tile, one thread per pixel, warp w on band rows 2w, 2w+1):
//   * the tile's list is walked back to front only up to the largest last
//     contributor of the band's pixels; batches of kThreads records are
//     gathered into shared memory in reverse order;
//   * phase A: a warp-synchronous walk (all lanes at one record) recomputes the
//     forward's decisions, divides T by (1 - alpha) and queues each contributing
//     sample (hit point in [0,1]^3, alpha T, levels, record, T);
//   * phase B: the warp's samples, compacted into one list, are processed one
//     per lane: per level the 8 corners are loaded, the feature is dotted with
//     the pixel's dL/dcolor (the colour term needs only that scalar), the
//     table gradient is scattered with float2 vector atomics and dL/d(hit) is
//     formed from the corner differences;
//   * phase C: each lane replays its own samples in order with the reference's
//     recursions (colour, depth, alpha, normal, distortion) and adds each
//     sample's per-surfel gradients to the surfel's accumulators in global
//     memory with four (rho2d branch: five) float4 reductions. Per-record
//     shared-memory float atomics cost a third of the kernel here (measured);
//     vector reductions resolve in L2 and a surfel's ~30 samples rarely collide.
// The transform gradient is folded into dL/dM = P dL/dT^T + dL/dhomotrans per
// sample (P = world2ndc * ndc2pix is one matrix per camera), so a record carries
// 18 accumulators instead of 25; the preprocess-backward kernel then turns dL/dM,
// the mean2D and normal gradients into mean, scale and quaternion gradients.
#include "hashgrid.cuh"
#include "kernels.cuh"

namespace ns {
namespace {

// A tile is split into bands of kRows rows, one CTA each: a CTA's barriers
// then hold only its band's two warps, which wait less for one another than a
// whole tile's eight, and the band walks its list only up to its own largest
// last contributor. Measured on the config-4 step (median backward): 16x16
// CTAs with 256-record batches 17.24 ms, 16x8 with 128 17.0, 16x4 with 64
// 16.55 and with 8-deep queues 16.40, 16x2 with 64 17.3-17.7.
constexpr int kRows = 4;                   // tile rows per CTA
constexpr int kBands = kTile / kRows;      // CTAs per tile
constexpr int kThreads = kTile * kRows;    // one thread per pixel of the band
constexpr int kWarps = kThreads / 32;
constexpr int kBatch = 64;        // records per batch (gathered back to front)
static_assert(kTile % kRows == 0 && kRows % 2 == 0, "bands of whole warps (two rows each)");
static_assert(kBatch <= 256, "a sample's record index is one byte");
constexpr int kQueue = 8;       // queued samples per pixel between drains
static_assert(kQueue <= 8, "a list entry holds the queue slot in three bits");
constexpr int kGradWords = 20;  // per-surfel accumulator words (18 used), 80 bytes
// Table-gradient aggregation on levels below this resolution (cells per axis):
// float atomics 512, fixed-point atomics (two 64-bit adds per corner, dearer
// than one float2 reduction) 1024. Measured on the config-4 step (median
// backward, ms, float / fixed point): 128: 16.42 / 25.34, 256: 16.15 / 23.1,
// 512: 16.13-16.18 / 22.0, 1024: 16.34-16.39 / 21.7, every level: 16.78 / 21.9.
constexpr float kAggScaleFloat = 512.f;
constexpr float kAggScaleFixed = 1024.f;

// Accumulator words of one surfel (80 bytes, five float4 groups; the last group
// is non-zero only for samples of the rho2d branch and for the shape gradient of
// the splat kernels 1-3).
enum : int {
  kGM = 0,          // dL/dM columns 0..2 (rows 0..2): L0, L1, mean -> words 0..8
  kGTuz = 9,        // dL/dT[0].z, dL/dT[1].z: the densification statistic
  kGTvz = 10,
  kGOpacity = 11,
  kGNormal = 12,    // dL/dnormal (view space) x, y, z
  kGGradSum = 15,
  kGMean2D = 16,    // dL/dmean2D x, y (rho2d branch)
  kGShape = 18,     // dL/dshape (splat kernels 1-3)
};

// Fixed-point unit of the deterministic table gradient: 2^32 units per
// 2^ceil(log2 gmax), gmax = max |dL/dcolor|. A sample's contribution to a table
// entry is w * alpha * T * dL/dcolor with w, alpha * T <= 1, so it stays below
// 2^32 units, a warp's aggregated sum below 2^37, and an entry's sum fits in 63
// bits while fewer than 2^31 maximal contributions land on it. Integer addition
// is associative, so the sums do not depend on the order of the atomics.
// Returns 0 for a non-finite gmax (the finish kernel then writes NaN).
__device__ __forceinline__ float fixed_point_scale(uint32_t gmax_bits) {
  const float g = __uint_as_float(gmax_bits);
  if (!(g <= 3.0e38f)) return 0.0f;
  if (g == 0.0f) return 1.0f;
  int e;
  frexpf(g, &e);  // g < 2^e
  return ldexpf(1.0f, 32 - max(e, -90));
}

// a * b - c * d with one rounding error at most (Kahan's difference of products
// with fused multiply-adds): the z rows of the transform gradient that feed the
// densification statistic subtract nearly equal products.
__device__ __forceinline__ float dop(float a, float b, float c, float d) {
  const float w = c * d;
  const float e = fmaf(-c, d, w);
  const float f = fmaf(a, b, -w);
  return f + e;
}

// Per-pixel constants of phase C, parked in shared memory while phase B runs
// (they are not needed there, and the registers they would hold go to phase
// B's loads in flight).
enum : int {
  kPxD = 0, kPxD2, kPxA, kPxDepth, kPxAccum, kPxReg, kPxMed, kPxN0, kPxN1, kPxN2, kPxAbs, kPxMedC,
  kPxWords
};

struct BwSmem {
  float4 rec[kBatch][kRecordFloat4];    // records of the batch, back to front
  float g[kThreads * kAccStride];       // dL/dcolor per pixel (acc_pair layout)
  float4 samp[kQueue][kThreads];        // (hit in [0,1]^3, alpha T) -> (f, dL/dhit)
  float Ts[kQueue][kThreads];           // T at the sample
  uint8_t jj[kQueue][kThreads];         // record of the sample
  uint8_t lvl[kQueue][kThreads];        // levels to query
  uint8_t item[kWarps][kQueue * 32];    // per warp: samples in k-major order, (k << 5) | lane
  uint32_t ids[kBatch];
  uint32_t wmax[kWarps];
  float pix[kPxWords][kThreads];        // per-pixel constants of phase C
  float Pm[9];                          // P[k][r], k = T column, r = 0..2
  float cam[3];                         // camera centre in world space
  LevelConst lv[kMaxLevels];
};

// Render modes 4 / 12 / 14 in the backward (backward.cu:987-1033, 1425-1606):
// the factor of the hash features in this sample (0 with `query` false: the
// mode does not read the grid here).
__device__ __forceinline__ float mode_hash_factor(const BackwardParams& p, uint32_t id, bool& query) {
  const int base = p.render_mode & 0xFF;
  const int pg = 2 * p.hybrid_levels;
  query = p.L > 0;
  if (base == 0 || (base >= 8 && base <= 10)) {  // level 0; modes 8-10 query in phase C
    query = false;
    return 0.0f;
  }
  if (base == 4 || base == 11) return 1.0f;
  if (base == 6) return 0.5f;
  if (base == 7) return 1.0f - __ldg(p.gauss + (size_t)id * (2 * p.total_levels + 1) + 2 * p.total_levels);
  if (base == 12) return 1.0f - __ldg(p.gauss + (size_t)id * (2 * p.total_levels + 1) + 2 * p.total_levels);
  const float wgt = __ldg(p.gauss + (size_t)id * (pg + 1) + pg);
  query = query && wgt > 1e-6f;
  return query ? wgt : 0.0f;
}

// The per-surfel side of a sample in modes 4 / 12 / 14: adds the gradients of
// the surfel's row (coarse channels aT g, mode 12's fine channels wgt aT g, the
// blend weight's aT (sum_fine row g - hdot) for 12 and aT hdot for 14) and
// returns feat . dL/dcolor for the colour recursion, hdot being the hash
// features' dot product with dL/dcolor (phase B). The reference's cases 12 and
// 14 leave the feature array of that recursion unwritten; this uses the
// forward's features.
__device__ __forceinline__ float mode_backward(const BackwardParams& p, uint32_t id, float aT, float hdot,
                                               const float* g, int t) {
  const int base = p.render_mode & 0xFF;
  // mode 11 (backward.cu:1372-1424): the hash levels only; its SH rows get no gradient
  if (base == 11) return hdot;
  const int pg = 2 * p.hybrid_levels, hd = 2 * (int)p.L, td = 2 * p.total_levels;
  auto gc = [&](int c) {
    const float2 v = *acc_pair(const_cast<float*>(g), t, c >> 1);
    return (c & 1) ? v.y : v.x;
  };
  const size_t stride = (base == 0 || base == 6) ? (size_t)p.C
                        : base == 4                ? (size_t)pg
                        : (base == 7 || base == 12) ? (size_t)td + 1
                                                    : (size_t)pg + 1;
  const float* row = p.gauss + (size_t)id * stride;
  float* drow = p.dL_dcolors + (size_t)id * stride;
  if (base == 0 || base == 6) {
    // level 0: per-surfel colours, dL/drow = aT dL/dC. Mode 6: feat = 0.5 row +
    // 0.5 hash on the hash levels' channels, dL/drow = 0.5 aT dL/dC there (the
    // derivative of the forward; the reference's case 6 backward reads a row
    // of 2 L LD values with a per-channel mask that its forward does not have,
    // backward.cu:1041-1106).
    const int n = base == 0 ? p.C : min(hd, p.C);
    const float sc = base == 0 ? 1.0f : 0.5f;
    float gdot = 0.0f;
    for (int c = 0; c < n; c++) {
      const float gv = gc(c);
      gdot += __ldg(row + c) * gv;
      atomicAdd(drow + c, sc * (aT * gv));
    }
    return base == 0 ? gdot : 0.5f * gdot + 0.5f * hdot;
  }
  if (base == 7) {
    // adaptive_add (backward.cu:1108-1190): dL/drow = wgt aT dL/dC; the weight
    // slot gets the reference's d_gamma = aT (row - hash) . dL/dC wgt (1 - wgt)
    // (the gradient of the pre-sigmoid parameter, as the reference returns it)
    const float wgt = __ldg(row + td);
    float gdot = 0.0f;
    for (int c = 0; c < td; c++) {
      const float gv = gc(c);
      gdot += __ldg(row + c) * gv;
      atomicAdd(drow + c, wgt * (aT * gv));
    }
    atomicAdd(drow + td, aT * (gdot - hdot) * (wgt * (1.0f - wgt)));
    return wgt * gdot + (1.0f - wgt) * hdot;
  }
  float f = 0.0f;
  for (int c = 0; c < pg; c++) {
    const float gv = gc(c);
    f += __ldg(row + c) * gv;
    atomicAdd(drow + c, aT * gv);
  }
  if (base == 4) return f + hdot;
  if (base == 12) {
    const float wgt = __ldg(row + td);
    float gdot = 0.0f;
    if (p.L > 0) {
      for (int c = pg; c < pg + hd; c++) {
        const float gv = gc(c);
        gdot += __ldg(row + c) * gv;
        atomicAdd(drow + c, wgt * (aT * gv));
      }
    }
    atomicAdd(drow + td, aT * (gdot - hdot));
    return f + wgt * gdot + (1.0f - wgt) * hdot;
  }
  const float wgt = __ldg(row + pg);
  const bool query = p.L > 0 && wgt > 1e-6f;
  atomicAdd(drow + pg, query ? aT * hdot : 0.0f);
  return query ? f + wgt * hdot : f;
}

// Render modes 8 / 9 / 10 in the backward (backward.cu:1191-1371), one sample:
// the single 3-wide hash level is looked up here, at the hit point `in`
// (phase B skips these modes). Adds the row gradients to dL_dcolors and the
// table gradient, writes dL/d(hit) in grid units (as phase B's d0..d2) to d,
// and returns feat . dL/dcolor for the colour recursion (the forward's
// features: the reference's cases leave that array unwritten). As the
// reference computes them, the row and table gradients carry alpha T twice
// (grad_feat = aT dL/dC, times aT again in each case).
template <typename TableT, bool kFixed>
__device__ __forceinline__ float sh_hybrid_backward(const BackwardParams& p, const LevelConst& lv0, uint32_t id,
                                                    float aT, float in0, float in1, float in2, bool q,
                                                    float half_shift, const float* g_sm, int t, uint32_t pid,
                                                    float fscale, float (&d)[3]) {
  const int base = p.render_mode & 0xFF, dec = p.hybrid_levels;
  const size_t HW = (size_t)p.H * p.W;
  auto gv = [&](int c) {
    if (c < kAccStride) {
      const float2 v = *acc_pair(const_cast<float*>(g_sm), t, c >> 1);
      return (c & 1) ? v.y : v.x;
    }
    return p.dL_dcolor[(size_t)c * HW + pid];
  };
  float h[3] = {0.f, 0.f, 0.f}, f[3] = {0.f, 0.f, 0.f}, dv[3] = {1.f, 1.f, 1.f}, cv[8][3];
  uint32_t idx[8];
  if (q) lookup_rows3<TableT>(lv0, p.table, in0, in1, in2, half_shift, p.interp, f, dv, idx, cv, h);
  const size_t width = base == 9 ? 48 : 3;
  const float* row = p.gauss + (size_t)id * width;
  float* drow = p.dL_dcolors + (size_t)id * width;
  float hg[3] = {0.f, 0.f, 0.f}, fdot = 0.f;
  if (base == 9) {
    for (int c = 0; c < 48; c++) {
      const float gc = gv(c);
      float v = __ldg(row + c);
      if ((c & 15) == 0) {
        const float hc = h[c >> 4];
        v = dec == 2 ? hc : (dec != 1 ? v + hc : v);
        hg[c >> 4] = aT * (aT * gc);
      }
      fdot += v * gc;
      if (dec != 2) atomicAdd(drow + c, aT * (aT * gc));
    }
  } else {
#pragma unroll
    for (int c = 0; c < 3; c++) {
      const float gc = gv(c), rv = __ldg(row + c);
      if (base == 8) {
        const float gr = fmaxf(0.0f, fminf(1.0f, rv + 0.5f));
        const float hr = 1.0f / (1.0f + expf(-h[c]));
        const float sum = gr + hr;
        fdot += (dec == 2 ? hr : dec == 1 ? gr : fmaxf(0.0f, fminf(1.0f, sum))) * gc;
        const float gpc = (sum >= 0.0f && sum <= 1.0f) ? aT * gc : 0.0f;
        const float va = rv + 0.5f;
        if (dec != 2) atomicAdd(drow + c, aT * ((va >= 0.0f && va <= 1.0f) ? gpc : 0.0f));
        hg[c] = aT * gpc * hr * (1.0f - hr);
      } else {
        const float comb = dec == 2 ? h[c] : dec == 1 ? rv : rv + h[c];
        const float sg = 1.0f / (1.0f + expf(-comb));
        fdot += sg * gc;
        const float gcomb = aT * gc * sg * (1.0f - sg);
        if (dec != 2) atomicAdd(drow + c, aT * gcomb);
        hg[c] = aT * gcomb;
      }
    }
  }
  d[0] = d[1] = d[2] = 0.0f;
  if (!q) return fdot;
  const float wx[2] = {1 - f[0], f[0]}, wy[2] = {1 - f[1], f[1]}, wz[2] = {1 - f[2], f[2]};
  // table gradient (hashgrid.h:184-190), one row of three per corner
#pragma unroll
  for (int c = 0; c < 8; c++) {
    const float w = (wx[c & 1] * wy[(c >> 1) & 1]) * wz[c >> 2];
    const size_t e = 3 * ((size_t)lv0.row0 + idx[c]);
#pragma unroll
    for (int ch = 0; ch < 3; ch++) {
      if (kFixed) atomicAdd(p.dL_dtable_fixed + e + ch, (unsigned long long)llrintf(w * hg[ch] * fscale));
      else atomicAdd(p.dL_dtable + e + ch, w * hg[ch]);
    }
  }
  // dL/d(hit): the 4 edges along each axis weighted by the other two axes'
  // corner weights (hashgrid.h:231-297), dotted with the hash gradient
  float ex = 0.f, ey = 0.f, ez = 0.f;
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const int b0 = e & 1, b1 = e >> 1;
#pragma unroll
    for (int ch = 0; ch < 3; ch++) {
      ex += (wy[b0] * wz[b1]) * (hg[ch] * (cv[1 + 2 * b0 + 4 * b1][ch] - cv[2 * b0 + 4 * b1][ch]));
      ey += (wx[b0] * wz[b1]) * (hg[ch] * (cv[b0 + 2 + 4 * b1][ch] - cv[b0 + 4 * b1][ch]));
      ez += (wx[b0] * wy[b1]) * (hg[ch] * (cv[b0 + 2 * b1 + 4][ch] - cv[b0 + 2 * b1][ch]));
    }
  }
  d[0] = ex * lv0.scale * dv[0];
  d[1] = ey * lv0.scale * dv[1];
  d[2] = ez * lv0.scale * dv[2];
  return fdot;
}

// kVariant 0: the Gaussian splat kernel in mode 0 (the hot loop free of the
// rest); 1: the splat kernels 1-3 (p.kernel_type), the render modes 4, 6, 7,
// 12, 14 and level 0 (p.render_mode); 2: also the spherical-harmonic hybrids,
// modes 8-11, whose per-sample lookup would otherwise take registers from
// variant 1's loop. kFixed: the table gradient goes to p.dL_dtable_fixed in
// fixed point (deterministic mode).
template <typename TableT, int kVariant, bool kFixed>
__global__ void __launch_bounds__(kThreads, 2 * kBands) blend_backward_kernel(const BackwardParams p) {
  constexpr bool kAnyKernel = kVariant != 0;
  constexpr bool kSH = kVariant == 2;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BwSmem& S = *reinterpret_cast<BwSmem*>(smem_raw);

  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int gx = div_up(p.W, kTile);
  const int slot = (int)blockIdx.x / kBands, band = (int)blockIdx.x % kBands;
  const int tile = p.tile_order ? (int)p.tile_order[slot] : slot;  // heaviest first
  const int tx = tile % gx, ty = tile / gx;
  const uint32_t px = tx * kTile + (t & (kTile - 1));
  const uint32_t py = ty * kTile + band * kRows + (t >> 4);
  const bool inside = px < (uint32_t)p.W && py < (uint32_t)p.H;
  const uint32_t pid = py * p.W + px;
  const float pxf = (float)px, pyf = (float)py;
  const size_t HW = (size_t)p.H * p.W;
  const float half_shift = p.align_corners ? 0.0f : 0.5f;
  const uint32_t L = p.L;
  const float vmin = p.gridrange[0], vmax = p.gridrange[1];
  const float fscale = kFixed ? fixed_point_scale(*p.grad_max_bits) : 0.0f;
  const int hoff = kAnyKernel ? hash_level_offset(p.render_mode, p.hybrid_levels) : 0;  // level of hash level 0

  if (t < (int)L) S.lv[t] = make_level<TableT>(p.table, p.offsets, p.S, p.Hres, p.align_corners, t);
  if (t < 9) {
    // P = world2ndc * ndc2pix (backward.cu:2106-2119), with the W, H of the
    // preprocess backward; column k (k = 0, 1, 2) pairs with T[k].
    const int k = t / 3, r = t % 3;
    const float* pm = p.projmatrix;
    const float n0 = k == 0 ? float(p.Wq) / 2.0f : 0.f;
    const float n1 = k == 1 ? float(p.Hq) / 2.0f : 0.f;
    const float n3 = k == 0 ? float(p.Wq - 1) / 2.0f : (k == 1 ? float(p.Hq - 1) / 2.0f : 1.f);
    S.Pm[t] = ((pm[4 * r + 0] * n0 + pm[4 * r + 1] * n1) + pm[4 * r + 2] * 0.f) + pm[4 * r + 3] * n3;
  }

  if (t >= 32 && t < 35) {
    // Camera centre o = -A^T b of the rigid view transform v = A x + b.
    const float* vm = p.viewmatrix;
    const int j = t - 32;
    S.cam[j] = -(vm[4 * j + 0] * vm[12] + vm[4 * j + 1] * vm[13] + vm[4 * j + 2] * vm[14]);
  }

  // Per-pixel state (backward.cu:560-630).
  float T = 0.f, final_D = 0.f, final_D2 = 0.f;
  uint32_t lc = 0;
  int median_c = 0;
  float dL_ddepth = 0.f, dL_daccum = 0.f, dL_dreg = 0.f, dL_dmed = 0.f;
  float dn0 = 0.f, dn1 = 0.f, dn2 = 0.f, gabs = 0.f;
  if (inside) {
    T = p.final_T[pid];
    final_D = p.final_T[pid + HW];
    final_D2 = p.final_T[pid + 2 * HW];
    lc = p.n_contrib[pid];
    median_c = (int)p.n_contrib[pid + HW];
    const float* go = p.dL_dothers + pid;
    dL_ddepth = go[0 * HW];
    dL_daccum = go[1 * HW];
    dn0 = go[2 * HW];
    dn1 = go[3 * HW];
    dn2 = go[4 * HW];
    dL_dmed = go[5 * HW];
    dL_dreg = go[6 * HW];
  }
  for (int l = 0; l < kAccStride / 2; l++) {
    float2 v = make_float2(0.f, 0.f);
    if (inside && 2 * l < p.C) v.x = p.dL_dcolor[(size_t)(2 * l) * HW + pid];
    if (inside && 2 * l + 1 < p.C) v.y = p.dL_dcolor[(size_t)(2 * l + 1) * HW + pid];
    gabs += fabsf(v.x) + fabsf(v.y);
    *acc_pair(S.g, t, l) = v;
  }
  if (inside)  // mode 9's channels past the shared copy
    for (int c = kAccStride; c < p.C; c++) gabs += fabsf(p.dL_dcolor[(size_t)c * HW + pid]);
  {
    float* px = &S.pix[0][t];
    px[kPxD * kThreads] = final_D;
    px[kPxD2 * kThreads] = final_D2;
    px[kPxA * kThreads] = 1 - T;
    px[kPxDepth * kThreads] = dL_ddepth;
    px[kPxAccum * kThreads] = dL_daccum;
    px[kPxReg * kThreads] = dL_dreg;
    px[kPxMed * kThreads] = dL_dmed;
    px[kPxN0 * kThreads] = dn0;
    px[kPxN1 * kThreads] = dn1;
    px[kPxN2 * kThreads] = dn2;
    px[kPxAbs * kThreads] = gabs;
    px[kPxMedC * kThreads] = __int_as_float(median_c);
  }
  {
    const uint32_t m = __reduce_max_sync(0xffffffffu, lc);
    if (lane == 0) S.wmax[wid] = m;
  }
  __syncthreads();
  uint32_t maxlc = 0;
#pragma unroll
  for (int w = 0; w < kWarps; w++) maxlc = max(maxlc, S.wmax[w]);
  const uint2 range = p.ranges[tile];
  const int total = (int)maxlc;
  const int rounds = div_up(total, kBatch);

  // Back-to-front recursions of the reference (scalar colour term: the
  // feature vector only enters through f = feat . dL/dcolor).
  float last_alpha = 0.f, acc_f = 0.f, last_f = 0.f;
  float last_depth = 0.f, acc_depth = 0.f, acc_alpha = 0.f, last_dL_dT = 0.f;
  float ln0 = 0.f, ln1 = 0.f, ln2 = 0.f, an0 = 0.f, an1 = 0.f, an2 = 0.f;

  for (int r = 0; r < rounds; r++) {
    const int hi = total - r * kBatch;
    const int lo = max(0, hi - kBatch);
    const int todo = hi - lo;
#pragma unroll
    for (int i = t; i < kBatch; i += kThreads) {
      if (i < todo) {
        const uint32_t id = p.point_list[range.x + hi - 1 - i];
        S.ids[i] = id;
        const float4* src = reinterpret_cast<const float4*>(p.records + id);
#pragma unroll
        for (int q = 0; q < kRecordFloat4; q++) {
          const unsigned dst = (unsigned)__cvta_generic_to_shared(&S.rec[i][q]);
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src + q));
        }
      }
    }
    asm volatile("cp.async.commit_group;");
    asm volatile("cp.async.wait_group 0;");
    __syncthreads();

    // Record j is list position hi-1-j; this pixel takes part from j >= jstart.
    const int jstart = hi - (int)lc;
    int j = max(0, __reduce_min_sync(0xffffffffu, jstart));
    while (j < todo) {
      // ---------------- phase A: decisions, T, queue.
      int cnt = 0;
      while (j < todo) {
        if (__any_sync(0xffffffffu, cnt == kQueue)) break;
        const int jj = j++;
        const float4 box = S.rec[jj][0];
        const bool cand =
            jj >= jstart && !(pxf < box.x || pxf > box.y || pyf < box.z || pyf > box.w);
        if (!__any_sync(0xffffffffu, cand)) continue;
        if (!cand) continue;
        const float4 q0 = S.rec[jj][1], q1 = S.rec[jj][2], q2 = S.rec[jj][3];
        const float3 Tu = f3(q0.x, q0.y, q0.z), Tv = f3(q0.w, q1.x, q1.y), Tw = f3(q1.z, q1.w, q2.x);
        const float3 kk = pxf * Tw - Tu;
        const float3 ll = pyf * Tw - Tv;
        const float3 pp = cross3(kk, ll);
        const float dx = q2.y - pxf, dy = q2.z - pyf;
        const float rho2d = kFilterInvSquare * (dx * dx + dy * dy);
        const float rho_cut = S.rec[jj][7].y;
        if (pp.x * pp.x + pp.y * pp.y > rho_cut * (pp.z * pp.z) && rho2d > rho_cut) continue;
        if (pp.z == 0.0f) continue;
        const float sx = pp.x / pp.z, sy = pp.y / pp.z;
        const float rho3d = sx * sx + sy * sy;
        const float rho = fminf(rho3d, rho2d);
        const bool on_plane = rho3d <= rho2d;
        const float depth = on_plane ? (sx * Tw.x + sy * Tw.y) + Tw.z : Tw.z;
        if (depth < kNear) continue;
        float G;
        if (!kAnyKernel || p.kernel_type == 0) {
          const float power = -0.5f * rho;
          if (power > 0.0f) continue;
          G = expf(power);
          if (p.beta > 0.0f) {
            const float demon = (float)(1.0 + (double)p.beta * G);
            G = (float)((1.0 + (double)p.beta) * G / demon);
          }
        } else {
          // Splat kernels 1-3 (backward.cu:765-803), as the forward evaluates them.
          const float shape = S.rec[jj][7].w;
          if (p.kernel_type == 1) {
            if (rho >= 1.0f) continue;
            G = powf(1.0f - rho, shape);
          } else if (p.kernel_type == 2) {
            const float power = -0.5f * rho;
            if (power > 0.0f) continue;
            G = expf(power);
            if (shape > 0.0f) G = (1.0f + shape) * G / (1.0f + shape * G);
          } else {
            const float power = -0.5f * powf(fmaxf(rho, 1e-8f), 0.5f * shape);
            if (power > 0.0f) continue;
            G = expf(power);
          }
        }
        const float alpha = fminf(0.99f, q2.w * G);
        if (alpha < 1.0f / 255.0f) continue;
        T = T / (1.f - alpha);

        const float4 q4 = S.rec[jj][5], q5 = S.rec[jj][6], q6 = S.rec[jj][7];
        float3 xyz;
        if (on_plane) {
          xyz = f3(sx * q4.x + sy * q4.w + q5.z, sx * q4.y + sy * q5.x + q5.w,
                   sx * q4.z + sy * q5.y + q6.x);
        } else {
          xyz = f3(q5.z, q5.w, q6.x);
        }
        const uint32_t apl = __float_as_uint(S.rec[jj][4].w);
        float in0, in1, in2;
        bool oob = false;
        if (!p.contract) {
          const float inv = 1.0f / (vmax - vmin);
          in0 = (xyz.x - vmin) * inv;
          in1 = (xyz.y - vmin) * inv;
          in2 = (xyz.z - vmin) * inv;
          oob = in0 < 0 || in0 > 1 || in1 < 0 || in1 > 1 || in2 < 0 || in2 > 1;
        } else {
          const float vmid = (vmax + vmin) * 0.5f;
          const float inv = 1.0f / ((vmax - vmin) * 0.5f);
          in0 = (xyz.x - vmid) * inv;
          in1 = (xyz.y - vmid) * inv;
          in2 = (xyz.z - vmid) * inv;
          const float nrm = sqrtf(in0 * in0 + in1 * in1 + in2 * in2);
          const float inv_n = 1.0f / nrm;
          const float st = (nrm <= 1.0f) ? 1.0f : (2.0f - inv_n) * inv_n;
          in0 = (st * in0 + 2.0f) * 0.25f;
          in1 = (st * in1 + 2.0f) * 0.25f;
          in2 = (st * in2 + 2.0f) * 0.25f;
        }
        float hw = alpha * T;  // weight of this sample's hash features
        bool query = true;
        if (kAnyKernel && uses_surfel_rows(p.render_mode, p.L)) hw *= mode_hash_factor(p, S.ids[jj], query);
        S.samp[cnt][t] = make_float4(in0, in1, in2, hw);
        S.lvl[cnt][t] = (uint8_t)((oob || !query) ? 0u : min(apl, L));
        S.jj[cnt][t] = (uint8_t)jj;
        S.Ts[cnt][t] = T;
        cnt++;
      }

      const int kmax = __reduce_max_sync(0xffffffffu, cnt);
      if (kmax == 0) continue;
      // ---------------- phase B: lookups, table-gradient scatter, dL/dhit.
      const int pbase = wid * 32;
      const uint32_t lt = lane_mask_lt();
      int nitems = 0;
#pragma unroll
      for (int k = 0; k < kQueue; k++) {
        const uint32_t m = __ballot_sync(0xffffffffu, cnt > k);
        if (cnt > k) S.item[wid][nitems + __popc(m & lt)] = (uint8_t)((k << 5) | lane);
        nitems += __popc(m);
      }
      __syncwarp();
      // One list entry per lane per step; levels in a warp-uniform loop so that
      // the table-gradient scatter can be aggregated across the warp.
      for (int base = 0; base < nitems; base += 32) {
        const int ii = base + lane;
        const bool has = ii < nitems;
        int pp = pbase, k = 0;
        float4 sm = make_float4(0.f, 0.f, 0.f, 0.f);
        uint32_t nl = 0;
        if (has) {
          const uint32_t tb = S.item[wid][ii];
          pp = pbase + (int)(tb & 31u);
          k = (int)(tb >> 5);
          sm = S.samp[k][pp];
          nl = S.lvl[k][pp];
        }
        const uint32_t nlmax = __reduce_max_sync(0xffffffffu, nl);
        const float aT = sm.w;
        const float pin[3] = {sm.x, sm.y, sm.z};
        float fdot = 0.f, d0 = 0.f, d1 = 0.f, d2 = 0.f;
        for (uint32_t l = 0; l < nlmax; l++) {
          const bool on = l < nl;
          const LevelConst lcst = S.lv[l];
          uint32_t gc[3] = {0u, 0u, 0u}, idx[8];
          float f[3], dv[3];
#pragma unroll
          for (int d = 0; d < 3; d++) {
            const float pos = pin[d] * lcst.scale + half_shift;
            const float fl = floorf(pos);
            gc[d] = (uint32_t)fl;
            f[d] = pos - fl;
            if (p.interp == 1) {
              dv[d] = 6 * f[d] * (1.0f - f[d]);
              f[d] = f[d] * f[d] * (3.0f - 2.0f * f[d]);
            } else {
              dv[d] = 1.0f;
            }
          }
          Corner8<TableT> cv;
          float2 v[8];
          float2 gl = make_float2(0.f, 0.f);
          if (on) {
            corner_rows(lcst, gc, idx);
#pragma unroll
            for (int c = 0; c < 8; c++) cv.load(lcst.base, c, idx[c]);
            gl = *acc_pair(S.g, pp, hoff + (int)l);
            const float2 grad = make_float2(aT * gl.x, aT * gl.y);
            const float wx[2] = {1 - f[0], f[0]}, wy[2] = {1 - f[1], f[1]}, wz[2] = {1 - f[2], f[2]};
            float2 feat = make_float2(0.f, 0.f);
#pragma unroll
            for (int c = 0; c < 8; c++) {
              const float w = (wx[c & 1] * wy[(c >> 1) & 1]) * wz[c >> 2];
              const float2 cvv = cv.get(c);
              feat.x += w * cvv.x;
              feat.y += w * cvv.y;
              v[c] = make_float2(w * grad.x, w * grad.y);
            }
            fdot += gl.x * feat.x + gl.y * feat.y;
            // d feat / d hit_d: the 4 edges along axis d weighted by the other two
            // axes' corner weights (hashgrid.h:231-283), dotted with grad.
            float ex = 0.f, ey = 0.f, ez = 0.f;
#pragma unroll
            for (int e = 0; e < 4; e++) {
              // x edges: corners (0|1) + 2 by + 4 bz, e = by + 2 bz
              const int by = e & 1, bz = e >> 1;
              const float2 a0 = cv.get(2 * by + 4 * bz), a1 = cv.get(1 + 2 * by + 4 * bz);
              ex += (wy[by] * wz[bz]) * (grad.x * (a1.x - a0.x) + grad.y * (a1.y - a0.y));
              // y edges: corners bx + (0|2) + 4 bz, e = bx + 2 bz
              const int bx = e & 1;
              const float2 b0 = cv.get(bx + 4 * bz), b1 = cv.get(bx + 2 + 4 * bz);
              ey += (wx[bx] * wz[bz]) * (grad.x * (b1.x - b0.x) + grad.y * (b1.y - b0.y));
              // z edges: corners bx + 2 by + (0|4), e = bx + 2 by
              const int by2 = e >> 1;
              const float2 c0 = cv.get(bx + 2 * by2), c1 = cv.get(bx + 2 * by2 + 4);
              ez += (wx[bx] * wy[by2]) * (grad.x * (c1.x - c0.x) + grad.y * (c1.y - c0.y));
            }
            d0 += ex * lcst.scale * dv[0];
            d1 += ey * lcst.scale * dv[1];
            d2 += ez * lcst.scale * dv[2];
          } else {
#pragma unroll
            for (int c = 0; c < 8; c++) v[c] = make_float2(0.f, 0.f);
          }
          // Table-gradient scatter (hashgrid.h:184-190), aggregated per cell:
          // lanes in the same cell of this level form a list (each lane links to
          // the next lane of its cell), pointer jumping sums every list into its
          // first lane, which alone issues the cell's 8 float2 atomics. At the
          // coarse levels a warp's 32 samples share a few cells, and unaggregated
          // atomics there serialise on a few hundred table rows.
          const uint32_t act = __ballot_sync(0xffffffffu, on);
          int nxt = -1;
          bool head = true;
          // Coarser levels only (fewer than kAggScale* cells per axis): finer
          // cells are rarely shared by a warp's samples and their atomics do not
          // contend, so the grouping would cost more than it saves.
          if (on && lcst.scale < (kFixed ? kAggScaleFixed : kAggScaleFloat)) {
            head = false;
            const unsigned long long key =
                (unsigned long long)gc[0] | ((unsigned long long)gc[1] << 21) | ((unsigned long long)gc[2] << 42);
            const uint32_t grp = __match_any_sync(act, key);
            const uint32_t after = grp & ~((2u << lane) - 1u);
            nxt = after ? __ffs(after) - 1 : -1;
            head = (grp & ((1u << lane) - 1u)) == 0u;
          }
          while (__any_sync(0xffffffffu, nxt >= 0)) {
            const int src = nxt >= 0 ? nxt : lane;
#pragma unroll
            for (int c = 0; c < 8; c++) {
              const float vx = __shfl_sync(0xffffffffu, v[c].x, src);
              const float vy = __shfl_sync(0xffffffffu, v[c].y, src);
              if (nxt >= 0) {
                v[c].x += vx;
                v[c].y += vy;
              }
            }
            const int nn = __shfl_sync(0xffffffffu, nxt, src);
            nxt = nxt >= 0 ? nn : -1;
          }
          if (on && head) {
            if (kFixed) {
              unsigned long long* dfx = p.dL_dtable_fixed + 2 * (size_t)lcst.row0;
#pragma unroll
              for (int c = 0; c < 8; c++) {
                atomicAdd(dfx + 2 * (size_t)idx[c], (unsigned long long)llrintf(v[c].x * fscale));
                atomicAdd(dfx + 2 * (size_t)idx[c] + 1, (unsigned long long)llrintf(v[c].y * fscale));
              }
            } else {
              float2* dtab = reinterpret_cast<float2*>(p.dL_dtable) + lcst.row0;
#pragma unroll
              for (int c = 0; c < 8; c++) atomicAdd(dtab + idx[c], v[c]);
            }
          }
        }
        if (has) S.samp[k][pp] = make_float4(fdot, d0, d1, d2);
      }
      __syncwarp();

      // ---------------- phase C: this lane's samples, back to front.
      const volatile float* pxv = &S.pix[0][t];
      const float final_D = pxv[kPxD * kThreads], final_D2 = pxv[kPxD2 * kThreads];
      const float final_A = pxv[kPxA * kThreads], dL_ddepth = pxv[kPxDepth * kThreads];
      const float dL_daccum = pxv[kPxAccum * kThreads], dL_dreg = pxv[kPxReg * kThreads];
      const float dL_dmed = pxv[kPxMed * kThreads];
      const float dn0 = pxv[kPxN0 * kThreads], dn1 = pxv[kPxN1 * kThreads], dn2 = pxv[kPxN2 * kThreads];
      const float gabs = pxv[kPxAbs * kThreads];
      const int median_c = __float_as_int(pxv[kPxMedC * kThreads]);
      const volatile float* pmv = S.Pm;
      const float P00 = pmv[0], P01 = pmv[1], P02 = pmv[2];
      const float P10 = pmv[3], P11 = pmv[4], P12 = pmv[5];
      const float P20 = pmv[6], P21 = pmv[7], P22 = pmv[8];
      for (int k = 0; k < cnt; k++) {
        const int jj = S.jj[k][t];
        const float Ti = S.Ts[k][t];
        float4 res = S.samp[k][t];
        const float4 q0 = S.rec[jj][1], q1 = S.rec[jj][2], q2 = S.rec[jj][3];
        const float4 q3 = S.rec[jj][4], q4 = S.rec[jj][5], q5 = S.rec[jj][6], q6 = S.rec[jj][7];
        const float3 Tu = f3(q0.x, q0.y, q0.z), Tv = f3(q0.w, q1.x, q1.y), Tw = f3(q1.z, q1.w, q2.x);
        const float3 kk = pxf * Tw - Tu;
        const float3 ll = pyf * Tw - Tv;
        const float3 pp = cross3(kk, ll);
        const float dx = q2.y - pxf, dy = q2.z - pyf;
        const float rho2d = kFilterInvSquare * (dx * dx + dy * dy);
        const float sx = pp.x / pp.z, sy = pp.y / pp.z;
        const float rho3d = sx * sx + sy * sy;
        const float rho = fminf(rho3d, rho2d);
        const bool on_plane = rho3d <= rho2d;
        const float c_d = on_plane ? (sx * Tw.x + sy * Tw.y) + Tw.z : Tw.z;
        float G, demon = 1.0f;
        float shape = 0.f, G_raw = 0.f, base = 0.f, pow_term = 0.f, rho_safe = 0.f;
        if (!kAnyKernel || p.kernel_type == 0) {
          G = expf(-0.5f * rho);
          if (p.beta > 0.0f) {
            demon = (float)(1.0 + (double)p.beta * G);
            G = (float)((1.0 + (double)p.beta) * G / demon);
          }
        } else {
          shape = q6.w;
          if (p.kernel_type == 1) {
            base = 1.0f - rho;
            G = powf(base, shape);
          } else if (p.kernel_type == 2) {
            G_raw = expf(-0.5f * rho);
            G = G_raw;
            if (shape > 0.0f) {
              demon = 1.0f + shape * G_raw;
              G = (1.0f + shape) * G_raw / demon;
            }
          } else {
            rho_safe = fmaxf(rho, 1e-8f);
            pow_term = powf(rho_safe, 0.5f * shape);
            G = expf(-0.5f * pow_term);
          }
        }
        const float opa = q2.w;
        const float alpha = fminf(0.99f, opa * G);
        const float aT = alpha * Ti;
        float3 xyz;
        if (on_plane) {
          xyz = f3(sx * q4.x + sy * q4.w + q5.z, sx * q4.y + sy * q5.x + q5.w,
                   sx * q4.z + sy * q5.y + q6.x);
        } else {
          xyz = f3(q5.z, q5.w, q6.x);
        }

        // Colour term (:1786-1797) with the scalar recursion.
        acc_f = last_alpha * last_f + (1.f - last_alpha) * acc_f;
        float fsc;
        const int mbase = p.render_mode & 0xFF;
        if (kSH && mbase >= 8 && mbase <= 10) {
          // modes 8-10: the one 3-wide level is looked up here (query_feature's
          // mapping of the hit point, hashgrid.h:63-114, without contraction
          // for these modes' tables as for the others)
          float i0, i1, i2;
          bool oob = false;
          if (!p.contract) {
            const float inv = 1.0f / (vmax - vmin);
            i0 = (xyz.x - vmin) * inv;
            i1 = (xyz.y - vmin) * inv;
            i2 = (xyz.z - vmin) * inv;
            oob = i0 < 0 || i0 > 1 || i1 < 0 || i1 > 1 || i2 < 0 || i2 > 1;
          } else {
            const float vmid = (vmax + vmin) * 0.5f;
            const float inv = 1.0f / ((vmax - vmin) * 0.5f);
            i0 = (xyz.x - vmid) * inv;
            i1 = (xyz.y - vmid) * inv;
            i2 = (xyz.z - vmid) * inv;
            const float nrm = sqrtf(i0 * i0 + i1 * i1 + i2 * i2);
            const float inv_n = 1.0f / nrm;
            const float st = (nrm <= 1.0f) ? 1.0f : (2.0f - inv_n) * inv_n;
            i0 = (st * i0 + 2.0f) * 0.25f;
            i1 = (st * i1 + 2.0f) * 0.25f;
            i2 = (st * i2 + 2.0f) * 0.25f;
          }
          const bool q = p.L > 0 && p.hybrid_levels != 1 && !oob && __float_as_uint(q3.w) >= 1u;
          float dh[3];
          fsc = sh_hybrid_backward<TableT, kFixed>(p, S.lv[0], S.ids[jj], aT, i0, i1, i2, q, half_shift, S.g, t,
                                                   pid, fscale, dh);
          res.y = dh[0];
          res.z = dh[1];
          res.w = dh[2];
        } else {
          fsc = (kAnyKernel && uses_surfel_rows(p.render_mode, p.L)) ? mode_backward(p, S.ids[jj], aT, res.x, S.g, t)
                                                                     : res.x;
        }
        last_f = fsc;
        float dL_dalpha = fsc - acc_f;

        // Auxiliary maps (:1799-1852).
        float dL_dz = 0.0f;
        const float m_d = kFar / (kFar - kNear) * (1 - kNear / c_d);
        const float dmd_dd = (kFar * kNear) / ((kFar - kNear) * c_d * c_d);
        const int position = hi - 1 - jj;
        if (position == median_c - 1) dL_dz += dL_dmed;
        const float dL_dweight = (final_D2 + m_d * m_d * final_A - 2 * m_d * final_D) * dL_dreg;
        dL_dalpha += dL_dweight - last_dL_dT;
        last_dL_dT = dL_dweight * alpha + (1 - alpha) * last_dL_dT;
        const float dL_dmd = 2.0f * (Ti * alpha) * (m_d * final_A - final_D) * dL_dreg;
        dL_dz += dL_dmd * dmd_dd;
        acc_depth = last_alpha * last_depth + (1.f - last_alpha) * acc_depth;
        last_depth = c_d;
        dL_dalpha += (c_d - acc_depth) * dL_ddepth;
        acc_alpha = last_alpha + (1.f - last_alpha) * acc_alpha;
        dL_dalpha += (1 - acc_alpha) * dL_daccum;
        an0 = last_alpha * ln0 + (1.f - last_alpha) * an0;
        an1 = last_alpha * ln1 + (1.f - last_alpha) * an1;
        an2 = last_alpha * ln2 + (1.f - last_alpha) * an2;
        ln0 = q3.x;
        ln1 = q3.y;
        ln2 = q3.z;
        dL_dalpha += (q3.x - an0) * dn0 + (q3.y - an1) * dn1 + (q3.z - an2) * dn2;
        dL_dalpha *= Ti;
        last_alpha = alpha;

        float dL_dG = opa * dL_dalpha;
        // dL/dshape and the kernel's dG/drho factor (backward.cu:1862-1914, :1960-2038).
        float dG_factor = -G, dshape = 0.f;
        if (!kAnyKernel || p.kernel_type == 0) {
          if (p.beta > 0.0f) dL_dG *= (float)((1.0 + (double)p.beta) / ((double)demon * demon));
        } else if (p.kernel_type == 1) {
          if (base > 1e-7f) dshape = dL_dalpha * opa * G * logf(base);
          dG_factor = base > 1e-7f ? -shape * G / base : 0.0f;
        } else if (p.kernel_type == 2) {
          if (shape > 0.0f) {
            dL_dG *= (1.0f + shape) / (demon * demon);
            dshape = dL_dalpha * opa * (G_raw * (1.0f - G_raw) / (demon * demon));
          }
          dG_factor = -G_raw;
        } else {
          dshape = dL_dalpha * opa * (-0.25f * G * pow_term * logf(rho_safe));
          dG_factor = -0.5f * shape * G * pow_term / rho_safe;
        }
        dL_dz += aT * dL_ddepth;

        // dL/dxyz from the hit-point gradient (query_feature's grad_scale).
        float gscale;
        if (!p.contract) {
          gscale = 1.0f / (vmax - vmin);
        } else {
          const float vmid = (vmax + vmin) * 0.5f;
          const float inv = 1.0f / ((vmax - vmin) * 0.5f);
          const float i0 = (xyz.x - vmid) * inv, i1 = (xyz.y - vmid) * inv, i2 = (xyz.z - vmid) * inv;
          const float nrm = sqrtf(i0 * i0 + i1 * i1 + i2 * i2);
          const float inv_n = 1.0f / nrm;
          const float st = (nrm <= 1.0f) ? 1.0f : (2.0f - inv_n) * inv_n;
          gscale = inv * st * 0.25f;
        }
        const float gx_ = res.y * gscale, gy_ = res.z * gscale, gz_ = res.w * gscale;

        // Transform, homotrans and mean2D gradients (:1921-2045).
        float3 dTu = f3(0.f, 0.f, 0.f), dTv = dTu, dTw = dTu;
        float h0x = 0.f, h0y = 0.f, h0z = 0.f, h1x = 0.f, h1y = 0.f, h1z = 0.f;
        float h2x = gx_, h2y = gy_, h2z = gz_;
        float dmx = 0.f, dmy = 0.f, tuz = 0.f, tvz = 0.f;
        if (on_plane) {
          const float du = gx_ * q4.x + gy_ * q4.y + gz_ * q4.z;
          const float dv = gx_ * q4.w + gy_ * q5.x + gz_ * q5.y;
          float dsx = dL_dG * dG_factor * sx + dL_dz * Tw.x;
          float dsy = dL_dG * dG_factor * sy + dL_dz * Tw.y;
          if (!p.ray_hit) {
            // The reference's form: the hit point's gradient enters both the
            // homotrans columns and, through (du, dv), the splat coordinates.
            h0x = gx_ * sx;
            h0y = gy_ * sx;
            h0z = gz_ * sx;
            h1x = gx_ * sy;
            h1y = gy_ * sy;
            h1z = gz_ * sy;
            dsx += du;
            dsy += dv;
          }
          const float dsx_pz = dsx / pp.z;
          const float dsy_pz = dsy / pp.z;
          const float3 dp = f3(dsx_pz, dsy_pz, -(dsx_pz * sx + dsy_pz * sy));
          const float3 dk = cross3(ll, dp);
          const float3 dl = cross3(dp, kk);
          dTu = f3(-dk.x, -dk.y, -dk.z);
          dTv = f3(-dl.x, -dl.y, -dl.z);
          dTw = f3(pxf * dk.x + pyf * dl.x + dL_dz * sx, pxf * dk.y + pyf * dl.y + dL_dz * sy,
                   pxf * dk.z + pyf * dl.z + dL_dz * 1.0f);
          tuz = -dop(ll.x, dp.y, ll.y, dp.x);
          tvz = -dop(dp.x, kk.y, dp.y, kk.x);
          if (p.ray_hit) {
            // The same hit-point gradient, well conditioned: the hit point is
            // the pixel ray's intersection with the surfel plane, so only the
            // plane's motion along the ray moves it. With n = L0 x L1 and the
            // ray r = xyz - camera, a = (g.r)/(r.n) and c = a (p - xyz):
            // dL/dp += a n, dL/dL0 += L1 x c, dL/dL1 += c x L0. In exact
            // arithmetic this equals the reference's homotrans + splat-coordinate
            // terms, whose large in-plane parts cancel; here they never form.
            const float3 su = f3(q4.x, q4.y, q4.z), sv = f3(q4.w, q5.x, q5.y);
            const float3 nrm = cross3(su, sv);
            const float3 ray = f3(xyz.x - S.cam[0], xyz.y - S.cam[1], xyz.z - S.cam[2]);
            const float a = (gx_ * ray.x + gy_ * ray.y + gz_ * ray.z) /
                            (ray.x * nrm.x + ray.y * nrm.y + ray.z * nrm.z);
            const float3 c = f3(-a * (sx * su.x + sy * sv.x), -a * (sx * su.y + sy * sv.y),
                                -a * (sx * su.z + sy * sv.z));
            const float3 c0 = cross3(sv, c), c1 = cross3(c, su);
            h0x = c0.x;
            h0y = c0.y;
            h0z = c0.z;
            h1x = c1.x;
            h1y = c1.y;
            h1z = c1.z;
            h2x = a * nrm.x;
            h2y = a * nrm.y;
            h2z = a * nrm.z;
            // The densification statistic keeps the reference's definition
            // (dL/dT[0].z, dL/dT[1].z including the (du, dv) path).
            const float hx = du / pp.z, hy = dv / pp.z;
            tuz -= dop(ll.x, hy, ll.y, hx);
            tvz -= dop(hx, kk.y, hy, kk.x);
          }
        } else {
          const float dG_factor_2d = dG_factor * kFilterInvSquare;
          dmx = dL_dG * (dG_factor_2d * dx);
          dmy = dL_dG * (dG_factor_2d * dy);
          dTw.z = dL_dz;
        }
        // dL/dM column c = sum_k P[k] dL/dT[k][c] + dL/dhomotrans column c; with
        // precomputed transforms (p.raw_T) dL/dT itself, columns Tu, Tv, Tw (the
        // homotrans gradient has no destination there, as in the reference).
        float4* ga = reinterpret_cast<float4*>(p.accum + (size_t)S.ids[jj] * kGradWords);
        if (p.raw_T) {
          atomicAdd(ga + 0, make_float4(dTu.x, dTu.y, dTu.z, dTv.x));
          atomicAdd(ga + 1, make_float4(dTv.y, dTv.z, dTw.x, dTw.y));
          atomicAdd(ga + 2, make_float4(dTw.z, tuz, tvz, G * dL_dalpha));
        } else {
          atomicAdd(ga + 0, make_float4(P00 * dTu.x + P10 * dTv.x + P20 * dTw.x + h0x,
                                        P01 * dTu.x + P11 * dTv.x + P21 * dTw.x + h0y,
                                        P02 * dTu.x + P12 * dTv.x + P22 * dTw.x + h0z,
                                        P00 * dTu.y + P10 * dTv.y + P20 * dTw.y + h1x));
          atomicAdd(ga + 1, make_float4(P01 * dTu.y + P11 * dTv.y + P21 * dTw.y + h1y,
                                        P02 * dTu.y + P12 * dTv.y + P22 * dTw.y + h1z,
                                        P00 * dTu.z + P10 * dTv.z + P20 * dTw.z + h2x,
                                        P01 * dTu.z + P11 * dTv.z + P21 * dTw.z + h2y));
          atomicAdd(ga + 2, make_float4(P02 * dTu.z + P12 * dTv.z + P22 * dTw.z + h2z, tuz, tvz,
                                        G * dL_dalpha));
        }
        // level 0 adds nothing to the densification sum (backward.cu:833-849)
        const float gsum = (kAnyKernel && p.render_mode == 0 && p.L == 0) ? 0.f : aT * gabs;
        atomicAdd(ga + 3, make_float4(aT * dn0, aT * dn1, aT * dn2, gsum));
        if (!on_plane || dshape != 0.f) atomicAdd(ga + 4, make_float4(dmx, dmy, dshape, 0.f));
      }
      __syncwarp();
    }
    __syncthreads();  // every warp is done with this batch before S.rec is refilled
  }
}

// preprocessCUDA backward (backward.cu:2216-2273) + compute_transmat_aabb
// (:2056-2214) from the folded accumulators: the mean2D gradient goes through
// the compute_aabb centre with t = (9, 9, -1) (:2143) into dL/dT and then dL/dM;
// the normal gradient through the normalisation (:2177-2190), the transposed view
// rotation and the camera-facing sign (:2194-2199); dL/dM, the normal and the
// scales give the rotation (quat_to_rotmat_vjp, auxiliary.h:243-287), scale and
// mean gradients; dL/dmean2D returned is the densification statistic (:2268-2272).
// The transform is rebuilt with scale_modifier 1, as the reference does.
__global__ void __launch_bounds__(256)
preprocess_backward_kernel(int P, const float* __restrict__ means3D, const float* __restrict__ scales,
                           const float* __restrict__ rotations, const int32_t* __restrict__ radii,
                           const float* __restrict__ viewmatrix, const float* __restrict__ projmatrix,
                           int Wq, int Hq, const float* __restrict__ accum, const float* __restrict__ Ts,
                           ns_raster_grads_out o) {
  __shared__ float vm[16], Pm[3][4];
  if (threadIdx.x < 16) vm[threadIdx.x] = viewmatrix[threadIdx.x];
  if (threadIdx.x >= 32 && threadIdx.x < 44) {
    const int c = (threadIdx.x - 32) / 4, r = (threadIdx.x - 32) % 4;
    const float* pm = projmatrix;
    const float n0 = c == 0 ? float(Wq) / 2.0f : 0.f;
    const float n1 = c == 1 ? float(Hq) / 2.0f : 0.f;
    const float n3 = c == 0 ? float(Wq - 1) / 2.0f : (c == 1 ? float(Hq - 1) / 2.0f : 1.f);
    Pm[c][r] = ((pm[4 * r + 0] * n0 + pm[4 * r + 1] * n1) + pm[4 * r + 2] * 0.f) + pm[4 * r + 3] * n3;
  }
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  float* dmean = o.dL_dmeans3D + 3 * (size_t)i;
  float* dscale = o.dL_dscales + 2 * (size_t)i;
  float* drot = o.dL_drots + 4 * (size_t)i;
  float* dm2 = o.dL_dmean2D + 3 * (size_t)i;
  if (!(radii[i] > 0)) {
    dmean[0] = dmean[1] = dmean[2] = 0.f;
    dscale[0] = dscale[1] = 0.f;
    drot[0] = drot[1] = drot[2] = drot[3] = 0.f;
    dm2[0] = dm2[1] = dm2[2] = 0.f;
    o.dL_dopacity[i] = 0.f;
    o.dL_gradsum[i] = 0.f;
    if (o.dL_dshapes) o.dL_dshapes[i] = 0.f;
    if (Ts)
      for (int k = 0; k < 9; k++) o.dL_dtransmat_precomp[9 * (size_t)i + k] = 0.f;
    return;
  }
  const float4* a4 = reinterpret_cast<const float4*>(accum + (size_t)i * kGradWords);
  float a[kGradWords];
#pragma unroll
  for (int q = 0; q < kGradWords / 4; q++) {
    const float4 v = a4[q];
    a[4 * q] = v.x;
    a[4 * q + 1] = v.y;
    a[4 * q + 2] = v.z;
    a[4 * q + 3] = v.w;
  }
  if (Ts) {
    // Precomputed transforms (backward.cu:2082-2088, 2128-2158): the render
    // pass's dL/dT plus, where the centre moved, the compute_aabb term (t = (9,
    // 9, -1)), written as the transforms' gradient; nothing reaches the mean,
    // scales or rotations; the densification statistic reads the updated dL/dT.
    float T[3][3], dT[3][3];
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
      for (int r = 0; r < 3; r++) {
        T[c][r] = Ts[9 * (size_t)i + 3 * c + r];
        dT[c][r] = a[kGM + 3 * c + r];
      }
    const float gx = a[kGMean2D], gy = a[kGMean2D + 1];
    if (gx != 0.f || gy != 0.f) {
      const float tv[3] = {9.0f, 9.0f, -1.0f};
      const float d = tv[0] * (T[2][0] * T[2][0]) + tv[1] * (T[2][1] * T[2][1]) + tv[2] * (T[2][2] * T[2][2]);
      const float id = 1.0f / d;
      float dL_df_dot = 0.f, add2[3];
#pragma unroll
      for (int r = 0; r < 3; r++) {
        const float fv = tv[r] * id;
        dT[0][r] += gx * fv * T[2][r];
        dT[1][r] += gy * fv * T[2][r];
        add2[r] = gx * fv * T[0][r] + gy * fv * T[1][r];
        dL_df_dot += (gx * T[0][r] * T[2][r] + gy * T[1][r] * T[2][r]) * fv;
      }
      const float dL_dd = (float)((double)dL_df_dot * (-1.0 / (double)d));
#pragma unroll
      for (int r = 0; r < 3; r++) dT[2][r] += add2[r] + dL_dd * (tv[r] * T[2][r] * 2.0f);
    }
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
      for (int r = 0; r < 3; r++) o.dL_dtransmat_precomp[9 * (size_t)i + 3 * c + r] = dT[c][r];
    dmean[0] = dmean[1] = dmean[2] = 0.f;
    dscale[0] = dscale[1] = 0.f;
    drot[0] = drot[1] = drot[2] = drot[3] = 0.f;
    const float depth = T[2][2];
    dm2[0] = (float)((double)(dT[0][2] * depth) * 0.5 * (double)Wq);
    dm2[1] = (float)((double)(dT[1][2] * depth) * 0.5 * (double)Hq);
    dm2[2] = 0.f;
    o.dL_dopacity[i] = a[kGOpacity];
    o.dL_gradsum[i] = a[kGGradSum];
    if (o.dL_dshapes) o.dL_dshapes[i] = a[kGShape];
    return;
  }
  const float3 pm_ = f3(means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]);
  const float4 q = make_float4(rotations[4 * i], rotations[4 * i + 1], rotations[4 * i + 2],
                               rotations[4 * i + 3]);
  const float sx = scales[2 * i], sy = scales[2 * i + 1];
  const float qs = rsqrtf(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
  const float w = q.x * qs, x = q.y * qs, y = q.z * qs, z = q.w * qs;
  const float3 R0 = f3(1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z), 2.f * (x * z - w * y));
  const float3 R1 = f3(2.f * (x * y - w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x));
  const float3 R2 = f3(2.f * (x * z + w * y), 2.f * (y * z - w * x), 1.f - 2.f * (x * x + y * y));

  float dM[3][3];
#pragma unroll
  for (int c = 0; c < 3; c++)
#pragma unroll
    for (int r = 0; r < 3; r++) dM[c][r] = a[kGM + 3 * c + r];

  const float gmx = a[kGMean2D], gmy = a[kGMean2D + 1];
  if (gmx != 0.f || gmy != 0.f) {
    // T = transpose(M) * P, M = [(L0,0), (L1,0), (p,1)]; T[c] = (L0.P[c], L1.P[c], p.P[c] + P[c][3]).
    const float3 L0 = sx * R0, L1 = sy * R1;
    float3 T[3];
#pragma unroll
    for (int c = 0; c < 3; c++) {
      T[c] = f3(L0.x * Pm[c][0] + L0.y * Pm[c][1] + L0.z * Pm[c][2],
                L1.x * Pm[c][0] + L1.y * Pm[c][1] + L1.z * Pm[c][2],
                pm_.x * Pm[c][0] + pm_.y * Pm[c][1] + pm_.z * Pm[c][2] + Pm[c][3]);
    }
    const float tv[3] = {9.0f, 9.0f, -1.0f};
    const float d = tv[0] * (T[2].x * T[2].x) + tv[1] * (T[2].y * T[2].y) + tv[2] * (T[2].z * T[2].z);
    const float id = 1.0f / d;
    const float fv[3] = {tv[0] * id, tv[1] * id, tv[2] * id};
    const float t0[3] = {T[0].x, T[0].y, T[0].z}, t1[3] = {T[1].x, T[1].y, T[1].z};
    const float t2[3] = {T[2].x, T[2].y, T[2].z};
    float dT[3][3];
    float dL_df_dot = 0.f;
#pragma unroll
    for (int r = 0; r < 3; r++) {
      dT[0][r] = gmx * fv[r] * t2[r];
      dT[1][r] = gmy * fv[r] * t2[r];
      dT[2][r] = gmx * fv[r] * t0[r] + gmy * fv[r] * t1[r];
      dL_df_dot += (gmx * t0[r] * t2[r] + gmy * t1[r] * t2[r]) * fv[r];
    }
    const float dL_dd = (float)((double)dL_df_dot * (-1.0 / (double)d));
#pragma unroll
    for (int r = 0; r < 3; r++) dT[2][r] += dL_dd * (tv[r] * t2[r] * 2.0f);
    // dL/dM += P * dT^T
#pragma unroll
    for (int c = 0; c < 3; c++)
#pragma unroll
      for (int r = 0; r < 3; r++)
        dM[c][r] += Pm[0][r] * dT[0][c] + Pm[1][r] * dT[1][c] + Pm[2][r] * dT[2][c];
  }

  // Normal: normalisation backprop, transposed view rotation, facing sign.
  const float3 n = f3(vm[0] * R2.x + vm[4] * R2.y + vm[8] * R2.z,
                      vm[1] * R2.x + vm[5] * R2.y + vm[9] * R2.z,
                      vm[2] * R2.x + vm[6] * R2.y + vm[10] * R2.z);
  const float gnx = a[kGNormal], gny = a[kGNormal + 1], gnz = a[kGNormal + 2];
  const float nlen = sqrtf(n.x * n.x + n.y * n.y + n.z * n.z);
  float gux = 0.f, guy = 0.f, guz = 0.f;
  if (nlen > 1e-7f) {
    const float dgn = gnx * n.x + gny * n.y + gnz * n.z;
    gux = (gnx - dgn * n.x / nlen) / nlen;
    guy = (gny - dgn * n.y / nlen) / nlen;
    guz = (gnz - dgn * n.z / nlen) / nlen;
  }
  float3 dtn = f3(vm[0] * gux + vm[1] * guy + vm[2] * guz, vm[4] * gux + vm[5] * guy + vm[6] * guz,
                  vm[8] * gux + vm[9] * guy + vm[10] * guz);
  const float3 pv = f3(vm[0] * pm_.x + vm[4] * pm_.y + vm[8] * pm_.z + vm[12],
                       vm[1] * pm_.x + vm[5] * pm_.y + vm[9] * pm_.z + vm[13],
                       vm[2] * pm_.x + vm[6] * pm_.y + vm[10] * pm_.z + vm[14]);
  const float cosv = -((pv.x * n.x + pv.y * n.y) + pv.z * n.z);
  if (!(cosv > 0)) dtn = f3(-dtn.x, -dtn.y, -dtn.z);

  const float v[3][3] = {{sx * dM[0][0], sx * dM[0][1], sx * dM[0][2]},
                         {sy * dM[1][0], sy * dM[1][1], sy * dM[1][2]},
                         {dtn.x, dtn.y, dtn.z}};
  drot[0] = 2.f * (x * (v[1][2] - v[2][1]) + y * (v[2][0] - v[0][2]) + z * (v[0][1] - v[1][0]));
  drot[1] = 2.f * (-2.f * x * (v[1][1] + v[2][2]) + y * (v[0][1] + v[1][0]) + z * (v[0][2] + v[2][0]) +
                   w * (v[1][2] - v[2][1]));
  drot[2] = 2.f * (x * (v[0][1] + v[1][0]) - 2.f * y * (v[0][0] + v[2][2]) + z * (v[1][2] + v[2][1]) +
                   w * (v[2][0] - v[0][2]));
  drot[3] = 2.f * (x * (v[0][2] + v[2][0]) + y * (v[1][2] + v[2][1]) - 2.f * z * (v[0][0] + v[1][1]) +
                   w * (v[0][1] - v[1][0]));
  dscale[0] = dM[0][0] * R0.x + dM[0][1] * R0.y + dM[0][2] * R0.z;
  dscale[1] = dM[1][0] * R1.x + dM[1][1] * R1.y + dM[1][2] * R1.z;
  dmean[0] = dM[2][0];
  dmean[1] = dM[2][1];
  dmean[2] = dM[2][2];
  // Densification statistic with depth = Tw.z = p . P[2] + P[2][3].
  const float depth = pm_.x * Pm[2][0] + pm_.y * Pm[2][1] + pm_.z * Pm[2][2] + Pm[2][3];
  dm2[0] = (float)((double)(a[kGTuz] * depth) * 0.5 * (double)Wq);
  dm2[1] = (float)((double)(a[kGTvz] * depth) * 0.5 * (double)Hq);
  dm2[2] = 0.f;
  o.dL_dopacity[i] = a[kGOpacity];
  o.dL_gradsum[i] = a[kGGradSum];
  if (o.dL_dshapes) o.dL_dshapes[i] = a[kGShape];
}

// max |g| over n floats as float bits, by atomicMax on the bit patterns (their
// order is the order of the non-negative values; NaN sorts above +inf).
// n4: float4 groups read vectorised (0 when g is not 16-byte aligned).
__global__ void __launch_bounds__(256) grad_abs_max_kernel(const float* __restrict__ g, size_t n,
                                                           size_t n4, uint32_t* __restrict__ out) {
  uint32_t m = 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = g4[i];
    m = max(m, max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
                   max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu)));
  }
  for (size_t i = 4 * n4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    m = max(m, __float_as_uint(g[i]) & 0x7fffffffu);
  m = __reduce_max_sync(0xffffffffu, m);
  if ((threadIdx.x & 31) == 0 && m != 0) atomicMax(out, m);
}

// Fixed point -> float: one rounding of the exact sum (a power-of-two scale).
__global__ void __launch_bounds__(256) table_fixed_finish_kernel(const unsigned long long* __restrict__ fx,
                                                                 size_t n, const uint32_t* __restrict__ gmax,
                                                                 float* __restrict__ out) {
  const float scale = fixed_point_scale(*gmax);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = scale != 0.0f ? (float)((double)(long long)fx[i] / (double)scale) : __int_as_float(0x7fc00000);
}

template <typename TableT, int kVariant, bool kFixed>
int launch_backward3(const BackwardParams& p, int tiles, cudaStream_t stream) {
  const int smem = (int)sizeof(BwSmem);
  NS_CUDA_TRY(cudaFuncSetAttribute(blend_backward_kernel<TableT, kVariant, kFixed>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  blend_backward_kernel<TableT, kVariant, kFixed><<<tiles * kBands, kThreads, smem, stream>>>(p);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

template <typename TableT, int kVariant>
int launch_backward(const BackwardParams& p, int tiles, cudaStream_t stream) {
  return p.dL_dtable_fixed ? launch_backward3<TableT, kVariant, true>(p, tiles, stream)
                           : launch_backward3<TableT, kVariant, false>(p, tiles, stream);
}

}  // namespace

size_t backward_accum_bytes(int64_t P) { return (size_t)max64(P, 1) * kGradWords * sizeof(float); }

int table_grad_max_launch(const float* dL_dcolor, size_t n, uint32_t* gmax, cudaStream_t stream) {
  NS_CUDA_TRY(cudaMemsetAsync(gmax, 0, sizeof(uint32_t), stream));
  if (n == 0) return NS_OK;
  const int blocks = (int)min64((int64_t)div_up64((int64_t)(n / 4 + 1), 256), 148 * 8);
  const size_t n4 = (reinterpret_cast<uintptr_t>(dL_dcolor) & 15u) ? 0 : n / 4;
  grad_abs_max_kernel<<<blocks, 256, 0, stream>>>(dL_dcolor, n, n4, gmax);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int table_grad_finish_launch(const unsigned long long* fx, size_t n, const uint32_t* gmax, float* out,
                             cudaStream_t stream) {
  if (n == 0) return NS_OK;
  const int blocks = (int)min64((int64_t)div_up64((int64_t)n, 256), 148 * 16);
  table_fixed_finish_kernel<<<blocks, 256, 0, stream>>>(fx, n, gmax, out);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int blend_backward_launch(const BackwardParams& p, int fp16, cudaStream_t stream) {
  const int base = p.render_mode & 0xFF;
  if (p.C <= 0) return NS_ERR_UNSUPPORTED;
  if (base >= 8 && base <= 10) {
    if (p.LD != 3 || p.L > 1 || p.C != (base == 9 ? 48 : 3)) return NS_ERR_UNSUPPORTED;
  } else {
    if (p.LD != 2 || p.C > kAccStride) return NS_ERR_UNSUPPORTED;
    const int hoff = hash_level_offset(p.render_mode, p.hybrid_levels);
    if (hoff < 0 || (int64_t)hoff + p.L > (uint32_t)(p.C / p.LD) || p.L > (uint32_t)kMaxLevels)
      return NS_ERR_UNSUPPORTED;
  }
  if ((p.render_mode >> 8) != 0) return NS_ERR_UNSUPPORTED;  // training rules only
  const int tiles = div_up(p.W, kTile) * div_up(p.H, kTile);
  if (tiles == 0) return NS_OK;
  if (base >= 8 && base <= 11)
    return fp16 ? launch_backward<__half, 2>(p, tiles, stream) : launch_backward<float, 2>(p, tiles, stream);
  if (p.kernel_type != 0 || uses_surfel_rows(p.render_mode, p.L))
    return fp16 ? launch_backward<__half, 1>(p, tiles, stream) : launch_backward<float, 1>(p, tiles, stream);
  return fp16 ? launch_backward<__half, 0>(p, tiles, stream) : launch_backward<float, 0>(p, tiles, stream);
}

int preprocess_backward_launch(int P, const float* means3D, const float* scales,
                               const float* rotations, const int32_t* radii, const float* vm,
                               const float* pm, int Wq, int Hq, const float* accum, const float* Ts,
                               const ns_raster_grads_out& o, cudaStream_t stream) {
  if (P <= 0) return NS_OK;
  preprocess_backward_kernel<<<div_up(P, 256), 256, 0, stream>>>(P, means3D, scales, rotations,
                                                                  radii, vm, pm, Wq, Hq, accum, Ts, o);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
