// render.cu -- per-pixel blend of depth-sorted surfels with the multiresolution
// hash-grid texture lookup (render_mode 0 of the reference).
//
// Restates forward.cu:639-2049 of the reference's diff-surfel-rasterization for
// render_mode 0, kernel_type 0 (Gaussian), level > 0:
//   intersection (:839-858), alpha / termination (:903-939), auxiliary maps
//   (:941-959), hit point from homotrans (:1099-1109), hash query (:1127-1145 ->
//   hashgrid.h:53-212), feature compositing (:1914-1916), level colour
//   (:1945-1957), transmittance record (:1961-1964), outputs (:2008-2048).
//
// One CTA of 128 threads per band of eight rows of a 16x16 tile (two CTAs per
// tile), one thread per pixel; warp w owns band rows 2w and 2w+1. The tile's
// surfel records stream through a ring of two 32-record slots in shared memory
// (cp.async, completion on an mbarrier per slot); the last warp to finish a
// batch refills its slot, so warps never meet at a CTA barrier and drift up to
// one batch apart. A band whose pixels are all done leaves and frees its SM
// slot for the next band. Each warp alternates, on its own 32 pixels, between
// two phases:
//
//   Phase A (intersect). The warp walks the batch in the reference's
//   front-to-back order, all lanes at the same position (a warp-uniform skip
//   when no lane is inside the surfel's alpha >= 1/255 box; a division-free
//   pre-test per lane before the reference arithmetic). It applies the
//   reference's decision rules exactly (alpha >= 1/255, T * (1 - alpha) >=
//   1e-4, depth >= near, max_intersections), keeps the auxiliary maps in
//   registers and appends each blended sample (hit point mapped to [0,1]^3,
//   weight, number of levels to query) to its pixel's queue in shared memory.
//   The warp stops when one of its queues is full; queues carry over between
//   batches.
//
//   Phase B (hash lookups). The warp's queued samples are compacted into one
//   k-major list (every pixel's sample k, then k+1, ...) so all 32 lanes look up
//   real samples; neighbouring pixels' k-th samples usually hit nearby points,
//   so their corner loads coalesce at the coarse levels. Levels run in a
//   warp-uniform outer loop (the dense/hashed choice is a uniform branch), four
//   levels of one list entry (four lookups) in flight per lane, so the list and
//   the owners' queues are walked once per four levels. Each pixel's owner lane
//   adds its results in queue order, the reference's per-pixel order: straight
//   from its own registers for a queue slot that every pixel of the warp fills
//   (that chunk of the list has lane = pixel), otherwise from a staging area,
//   while the next chunk's corner loads are in flight.
//
// The hash table is read as fp16 (or fp32) pairs through the read-only path;
// at 16 levels x 2^19 x 2 fp16 it is 32 MB and stays resident in the 126 MB L2.
#include "hashgrid.cuh"
#include "kernels.cuh"

namespace ns {
namespace {

// Measured on the config-2 frame (blend, CUDA events; same images): 16 rows
// with four slots 5.034 ms, 8 rows with four 5.27, 8 rows with two 4.922
// (kept), 4 rows with two 5.52, with four 6.48. Four 8-row CTAs of 47.7 KB per
// SM keep the 16 warps and the ~60 KB of L1 of two 97 KB 16-row CTAs; the
// four-slot 8-row ring and the 4-row bands take L1 down to ~28 KB.
constexpr int kRows = 8;               // tile rows per CTA
constexpr int kBands = kTile / kRows;  // CTAs per tile
constexpr int kThreads = kTile * kRows;  // one pixel per thread
constexpr int kQueue = 8;              // queued samples per pixel between drains
constexpr int kWarps = kThreads / 32;
constexpr int kBatch = 32;             // surfel records per ring slot
constexpr int kSlots = 2;              // ring slots (batches in flight), a power of two
constexpr int kChunk = 32;             // compacted samples looked up per warp step (1 per lane)
static_assert(kTile % kRows == 0 && kRows % 2 == 0, "bands of whole warps (two rows each)");
static_assert((kSlots & (kSlots - 1)) == 0 && kBatch % 32 == 0, "ring slot index and fill shape");
constexpr int kMaxChannels = 32;

struct BlendSmem {
  float4 rec[kSlots][kBatch][kRecordFloat4];  // ring of surfel-record batches
  float4 samp[kQueue][kThreads];        // (hit point in [0,1]^3, weight)
  uint8_t lvl[kQueue][kThreads];        // levels to query for the sample (0: none)
  uint8_t item[kWarps][kQueue * 32];    // per warp: queued samples in k-major order, (k << 5) | lane
  uint8_t pos[kQueue][kThreads];        // position of a pixel's k-th sample in its warp's list
  float4 res[2][kWarps][kChunk];        // lookups of the current chunk: levels l, l+1 | l+2, l+3 per entry
                                        // (two arrays, so a lane's stores and reads are 16-byte
                                        // strided: no shared-memory bank conflicts)
  float acc[kThreads * kAccStride];     // feature accumulators, see acc_pair()
  LevelConst lv[kMaxLevels];
  uint64_t full[kSlots];                // slot filled (32 cp.async arrivals per fill)
  int used[kSlots];                     // warps done with the slot's current batch
  int ndone;                            // warps whose pixels are all done
};

// Render modes 4 / 6 / 7 / 12-14 and level 0 (forward.cu:1093-1096,
// 1218-1377, 1593-1790): adds this sample's per-surfel features, weighted by
// w, to the pixel's accumulators and returns the factor of the hash features
// (0: the mode does not query the grid).
// Mode 4 (cat): features [0, hybrid LD), hash levels after them. Mode 12
// (adaptive_cat, rows of total LD + 1 with the blend weight last): coarse
// channels from the surfel, fine channels wgt * surfel + (1 - wgt) * hash; with
// the inference flag all channels from the surfel when wgt >= 0.9, else coarse
// from the surfel and fine from the grid. Mode 14 (adaptive_zero, rows of
// hybrid LD + 1): coarse from the surfel, fine wgt * hash (training: wgt > 1e-6;
// inference: wgt >= 0.1, else zeros). Mode 13 (adaptive_cat_fast, mode 12's
// rows, :964-1091): with the inference flag all channels from the surfel when
// wgt > 0.5, else coarse from the surfel and fine from the grid; without it
// coarse wgt * surfel and fine as mode 12.
__device__ __forceinline__ float mode_features(const RenderParams& p, uint32_t id, float w, float* acc,
                                               int t) {
  const int base = p.render_mode & 0xFF;
  const bool infer = ((p.render_mode >> 8) & 1) != 0;
  const int pg = 2 * p.hybrid_levels, hd = 2 * (int)p.L;
  auto add = [&](const float* g, int c0, int c1, float scale) {
    for (int c = c0; c < c1 && c < p.C; c += 2) {
      float2* a = acc_pair(acc, t, c >> 1);
      a->x += __ldg(g + c) * scale;
      if (c + 1 < p.C) a->y += __ldg(g + c + 1) * scale;
    }
  };
  if (base == 4) {
    add(p.gauss + (size_t)id * pg, 0, pg, w);
    return p.L > 0 ? 1.0f : 0.0f;
  }
  if (base == 13) {
    const int td = 2 * p.total_levels;
    const float* g = p.gauss + (size_t)id * (td + 1);
    const float wgt = __ldg(g + td);
    if (infer && wgt > 0.5f) {
      add(g, 0, td, w);
      return 0.0f;
    }
    add(g, 0, pg, infer ? w : wgt * w);
    if (p.L == 0) return 0.0f;
    if (infer) return 1.0f;
    add(g, pg, pg + hd, wgt * w);
    return 1.0f - wgt;
  }
  if (base == 12) {
    const int td = 2 * p.total_levels;
    const float* g = p.gauss + (size_t)id * (td + 1);
    const float wgt = __ldg(g + td);
    if (infer && wgt >= 0.9f) {
      add(g, 0, td, w);
      return 0.0f;
    }
    add(g, 0, pg, w);
    if (p.L == 0) return 0.0f;
    if (infer) return 1.0f;
    add(g, pg, pg + hd, wgt * w);
    return 1.0f - wgt;
  }
  if (base == 6) {
    // adaptive (forward.cu:1283-1325): rows of C channels, feat = 0.5 row +
    // 0.5 hash over the L hash levels' channels
    add(p.gauss + (size_t)id * p.C, 0, min(hd, p.C), 0.5f * w);
    return p.L > 0 ? 0.5f : 0.0f;
  }
  if (base == 7) {
    // adaptive_add (:1326-1377): rows of total LD + 1, feat = wgt row +
    // (1 - wgt) hash, the hash levels' channels from 0
    const int td = 2 * p.total_levels;
    const float* g = p.gauss + (size_t)id * (td + 1);
    const float wgt = __ldg(g + td);
    add(g, 0, td, wgt * w);
    return p.L > 0 ? 1.0f - wgt : 0.0f;
  }
  if (base == 0) {
    // level 0 (:1093-1096): per-surfel colours of C channels, no hash query
    add(p.gauss + (size_t)id * p.C, 0, p.C, w);
    return 0.0f;
  }
  const float* g = p.gauss + (size_t)id * (pg + 1);  // base == 14
  const float wgt = __ldg(g + pg);
  add(g, 0, pg, w);
  return (p.L > 0 && (infer ? wgt >= 0.1f : wgt > 1e-6f)) ? wgt : 0.0f;
}

// Render modes 8 (hybrid_SH), 9 (hybrid_SH_post) and 10 (hybrid_SH_raw),
// forward.cu:1378-1526: the sample's feature from the surfel's row (3 raw SH
// colours; 48 SH coefficients for 9) and one 3-wide hash level queried here,
// at the hit point (no phase-B lookup). p.hybrid_levels holds the level
// word's decompose flag (0 both parts, 1 the surfel only, 2 the grid only).
// Mode 9's channels from kMaxChannels on are accumulated in out_color itself
// (the pixel's own words, zeroed at the kernel's start).
template <typename TableT>
__device__ __forceinline__ void sh_hybrid_features(const RenderParams& p, const LevelConst& lv0, uint32_t id,
                                                   float w, float in0, float in1, float in2, bool oob,
                                                   uint32_t apl, float half_shift, float* acc, int t,
                                                   uint32_t pid) {
  const int base = p.render_mode & 0xFF, dec = p.hybrid_levels;
  float h[3] = {0.f, 0.f, 0.f};
  if (p.L > 0 && dec != 1 && !oob && apl >= 1) {
    float f[3], dv[3], cv[8][3];
    uint32_t idx[8];
    lookup_rows3<TableT>(lv0, p.table, in0, in1, in2, half_shift, p.interp, f, dv, idx, cv, h);
  }
  auto add = [&](int c, float v) {
    if (c < kMaxChannels) {
      float2* a = acc_pair(acc, t, c >> 1);
      if (c & 1) a->y += v * w;
      else a->x += v * w;
    } else {
      p.out_color[(size_t)c * p.H * p.W + pid] += v * w;
    }
  };
  if (base == 9) {
    const float* g = p.gauss + (size_t)id * 48;
    for (int c = 0; c < 48; c++) {
      float v = __ldg(g + c);
      if ((c & 15) == 0) {
        const float hc = h[c >> 4];
        v = dec == 2 ? hc : (dec != 1 ? v + hc : v);
      }
      add(c, v);
    }
    return;
  }
  const float* g = p.gauss + (size_t)id * 3;
#pragma unroll
  for (int c = 0; c < 3; c++) {
    const float gv = __ldg(g + c);
    float v;
    if (base == 8) {
      const float gr = fmaxf(0.0f, fminf(1.0f, gv + 0.5f));
      const float hr = 1.0f / (1.0f + expf(-h[c]));
      v = dec == 2 ? hr : dec == 1 ? gr : fmaxf(0.0f, fminf(1.0f, gr + hr));
    } else {
      const float comb = dec == 2 ? h[c] : dec == 1 ? gv : gv + h[c];
      v = 1.0f / (1.0f + expf(-comb));
    }
    add(c, v);
  }
}

// Render mode 11 (residual_hybrid), forward.cu:1918-1943: the surfel's degree-3
// spherical-harmonic colour along the unit direction from its centre to the
// hit point, its 48 coefficients read interleaved (coefficient k of channel c
// at 3 k + c), 0.5 added to the DC term, clamped at 0 (eval_sh_inline,
// :76-155), weighted by w into the three accumulators after the C hash
// channels. The basis constants are the standard real SH normalisations.
__device__ __forceinline__ void residual_sh(const RenderParams& p, uint32_t id, float3 xyz, float3 pk, float w,
                                            float* acc, int t) {
  constexpr float C0 = 0.28209479177387814f, C1 = 0.4886025119029199f;
  constexpr float C2a = 1.0925484305920792f, C2b = -1.0925484305920792f, C2c = 0.31539156525252005f,
                  C2d = -1.0925484305920792f, C2e = 0.5462742152960396f;
  constexpr float C3a = -0.5900435899266435f, C3b = 2.890611442640554f, C3c = -0.4570457994644658f,
                  C3d = 0.3731763325901154f, C3e = -0.4570457994644658f, C3f = 1.445305721320277f,
                  C3g = -0.5900435899266435f;
  float dx = xyz.x - pk.x, dy = xyz.y - pk.y, dz = xyz.z - pk.z;
  const float inv = rsqrtf(dx * dx + dy * dy + dz * dz);
  const float x = dx * inv, y = dy * inv, z = dz * inv;
  const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
  const float* sh = p.gauss + (size_t)id * 48;
#pragma unroll
  for (int c = 0; c < 3; c++) {
    auto k = [&](int i) { return __ldg(sh + 3 * i + c); };
    float r = C0 * k(0) + 0.5f;
    r = r - C1 * y * k(1) + C1 * z * k(2) - C1 * x * k(3);
    r = r + C2a * xy * k(4) + C2b * yz * k(5) + C2c * (2.0f * zz - xx - yy) * k(6) + C2d * xz * k(7) +
        C2e * (xx - yy) * k(8);
    r = r + C3a * y * (3.0f * xx - yy) * k(9) + C3b * xy * z * k(10) + C3c * y * (4.0f * zz - xx - yy) * k(11) +
        C3d * z * (2.0f * zz - 3.0f * xx - 3.0f * yy) * k(12) + C3e * x * (4.0f * zz - xx - yy) * k(13) +
        C3f * z * (xx - yy) * k(14) + C3g * x * (xx - 3.0f * yy) * k(15);
    r = fmaxf(r, 0.0f);
    const int ch = p.C + c;
    float2* a = acc_pair(acc, t, ch >> 1);
    if (ch & 1) a->y += w * r;
    else a->x += w * r;
  }
}

// kVariant 0: the Gaussian splat kernel in mode 0 (the hot loop free of the
// rest); 1: the splat kernels 1-3 (p.kernel_type), the render modes 4, 6, 7,
// 12-14 and level 0 (p.render_mode); 2: also the spherical-harmonic hybrids,
// modes 8-11, whose per-sample lookup and SH evaluation would otherwise take
// registers from variant 1's loop.
template <typename TableT, int kVariant>
__global__ void __launch_bounds__(kThreads, 2 * kBands) blend_kernel(const RenderParams p) {
  constexpr bool kGeneral = kVariant != 0;
  constexpr bool kSH = kVariant == 2;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BlendSmem& S = *reinterpret_cast<BlendSmem*>(smem_raw);

  const int t = threadIdx.x;
  const int gx = div_up(p.W, kTile);
  const int slot = (int)blockIdx.x / kBands, band = (int)blockIdx.x % kBands;
  const int tile = p.tile_order ? (int)p.tile_order[slot] : slot;  // heaviest first
  const int tx = tile % gx, ty = tile / gx;
  const uint32_t px = tx * kTile + (t & (kTile - 1));
  const uint32_t py = ty * kTile + band * kRows + (t >> 4);
  const bool inside = px < (uint32_t)p.W && py < (uint32_t)p.H;
  const uint32_t pid = py * p.W + px;
  const float pxf = (float)px, pyf = (float)py;
  const float half_shift = p.align_corners ? 0.0f : 0.5f;
  const uint32_t L = p.L;

  if (t < (int)L) S.lv[t] = make_level<TableT>(p.table, p.offsets, p.S, p.Hres, p.align_corners, t);
  for (int c = 0; c < kAccStride; c++) S.acc[t * kAccStride + c] = 0.f;  // only this thread's row
  if (kSH && inside)  // mode 9: channels past the shared accumulators add up in out_color
    for (int c = kMaxChannels; c < p.C; c++) p.out_color[(size_t)c * p.H * p.W + pid] = 0.0f;
  if (t < kSlots) {
    mbar_init_shared(&S.full[t], 32);
    S.used[t] = 0;
  }
  if (t == 0) S.ndone = 0;

  const uint2 range = p.ranges[tile];
  const int total = (int)(range.y - range.x);
  const int rounds = div_up(total, kBatch);
  const float vmin = p.gridrange[0], vmax = p.gridrange[1];
  const int hoff = kGeneral ? hash_level_offset(p.render_mode, p.hybrid_levels) : 0;  // level of hash level 0

  float T = 1.0f;
  uint32_t contributor = 0, last_contributor = 0, render_number = 0;
  float N0 = 0, N1 = 0, N2 = 0, D = 0, M1 = 0, M2 = 0, distortion = 0, median_depth = 0;
  float median_contributor = -1;
  float pos0 = 0, pos1 = 0, pos2 = 0, vis0 = 0, vis1 = 0;
  bool done = !inside;

  // Record ring: slot s holds batch b (b % kSlots == s). Warp w fills batches
  // w, w + kWarps, ... below kSlots; after that the last warp to finish batch b
  // refills its slot with batch b + kSlots, so warps drift up to kSlots - 1
  // batches apart instead of meeting at a CTA barrier per batch. Each lane of
  // the filling warp copies one record and arrives on full[s] when its copies
  // have landed.
  const int lane = t & 31, wid = t >> 5, pbase = wid * 32;
  auto fetch = [&](int b) {
    const int s = b & (kSlots - 1);
#pragma unroll
    for (int h = 0; h < kBatch / 32; h++) {
      const int jj = h * 32 + lane;
      const int k = b * kBatch + jj;
      if (k < total) {
        const uint32_t id = p.point_list[range.x + k];
        const float4* src = reinterpret_cast<const float4*>(p.records + id);
#pragma unroll
        for (int q = 0; q < kRecordFloat4; q++) {
          const unsigned dst = (unsigned)__cvta_generic_to_shared(&S.rec[s][jj][q]);
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src + q));
        }
      }
    }
    cp_async_arrive(&S.full[s]);
  };

  int cnt = 0;  // this pixel's queued samples (kept across batches)
  // Phase B: the warp's queued hash lookups (see the file comment); empties
  // every queue of the warp.
  auto drain = [&]() {
    if (!__any_sync(0xffffffffu, cnt > 0)) return;
    // Compact the warp's queued samples into one k-major list (sample k of
    // every pixel that has one, then k+1, ...), so all 32 lanes look up real
    // samples; neighbouring pixels' k-th samples stay adjacent (coalescing).
    const uint32_t lt = lane_mask_lt();
    int nitems = 0;
    int nfull = 0;  // leading queue slots that every pixel of the warp fills
#pragma unroll
    for (int k = 0; k < kQueue; k++) {
      const uint32_t m = __ballot_sync(0xffffffffu, cnt > k);
      if (cnt > k) {
        const int ps = nitems + __popc(m & lt);
        S.item[wid][ps] = (uint8_t)((k << 5) | lane);
        S.pos[k][t] = (uint8_t)ps;
      }
      if (nfull == k && m == 0xffffffffu) nfull++;
      nitems += __popc(m);
    }
    __syncwarp();
    // Four levels per pass, 32 list entries (one per lane) per step: four
    // lookups in flight per lane. Each pixel's owner lane then adds its own
    // results from the step, in sample order.
    for (uint32_t l = 0; l < L; l += 4) {
      const uint32_t nl = min(4u, L - l);
      float2 c[4];
      float2* ap[4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        ap[q] = acc_pair(S.acc, t, hoff + (int)(l + min((uint32_t)q, nl - 1)));
        c[q] = (uint32_t)q < nl ? *ap[q] : make_float2(0.f, 0.f);
      }
      int nk = 0;
      // The owners add chunk ch - 32's staged results while chunk ch's corner
      // loads are in flight; the last staged chunk is added after the loop.
      bool staged = false;
      auto owners = [&](int chp) {
        while (nk < cnt) {
          const int ps = S.pos[nk][t];
          if (ps >= chp + kChunk) break;
          const float4 r01 = S.res[0][wid][ps - chp];
          const float4 r23 = S.res[1][wid][ps - chp];
          const uint32_t mk = S.lvl[nk][t];
          const float w = S.samp[nk][t].w;
          const float2 ww = make_float2(w, w);
          if (l < mk) c[0] = __ffma2_rn(make_float2(r01.x, r01.y), ww, c[0]);
          if (l + 1 < mk && nl > 1) c[1] = __ffma2_rn(make_float2(r01.z, r01.w), ww, c[1]);
          if (l + 2 < mk && nl > 2) c[2] = __ffma2_rn(make_float2(r23.x, r23.y), ww, c[2]);
          if (l + 3 < mk && nl > 3) c[3] = __ffma2_rn(make_float2(r23.z, r23.w), ww, c[3]);
          nk++;
        }
      };
      for (int ch = 0; ch < nitems; ch += kChunk) {
        float4 sa = make_float4(0.f, 0.f, 0.f, 0.f);
        uint32_t ma = 0;
        const int ia = ch + lane;
        if (ia < nitems) {
          const uint32_t tb = S.item[wid][ia];
          const int pp = pbase + (int)(tb & 31u), k = (int)(tb >> 5);
          sa = S.samp[k][pp];
          ma = S.lvl[k][pp];
        }
        float f[4][3];
        Corner8<TableT> v[4];
        bool u[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          u[q] = (uint32_t)q < nl && l + q < ma;
          if (u[q]) lookup_issue<TableT>(S.lv[l + q], p.table, sa, half_shift, p.interp, f[q], v[q]);
        }
        if (staged) {
          owners(ch - kChunk);
          __syncwarp();
          staged = false;
        }
        float2 r[4];
#pragma unroll
        for (int q = 0; q < 4; q++) r[q] = u[q] ? lookup_finish<TableT>(f[q], v[q]) : make_float2(0.f, 0.f);
        if (ch < kChunk * nfull) {
          const float2 ww = make_float2(sa.w, sa.w);
#pragma unroll
          for (int q = 0; q < 4; q++)
            if (u[q]) c[q] = __ffma2_rn(r[q], ww, c[q]);
          nk++;
          continue;
        }
        S.res[0][wid][lane] = make_float4(r[0].x, r[0].y, r[1].x, r[1].y);
        S.res[1][wid][lane] = make_float4(r[2].x, r[2].y, r[3].x, r[3].y);
        __syncwarp();
        staged = true;
      }
      if (staged) {
        owners(((nitems - 1) / kChunk) * kChunk);
        __syncwarp();
      }
#pragma unroll
      for (int q = 0; q < 4; q++)
        if ((uint32_t)q < nl) *ap[q] = c[q];
    }
    __syncwarp();
    cnt = 0;
  };

  __syncthreads();  // level table, accumulators and ring barriers are initialised
  for (int b0 = wid; b0 < kSlots && b0 < rounds; b0 += kWarps) fetch(b0);
  bool wdone = !__any_sync(0xffffffffu, !done);
  if (wdone && lane == 0) atomicAdd(&S.ndone, 1);
  for (int b = 0; b < rounds; b++) {
    const int s = b & (kSlots - 1);
    // Wait for batch b (gives up when every warp of the tile is done).
    const int ws = mbar_wait_parity(&S.full[s], (uint32_t)(b / kSlots) & 1u, p.spin_limit, &S.ndone, kWarps);
    if (ws <= 0) {
      if (ws < 0) set_error(p.err, kErrSpinTimeout);
      break;
    }
    if (!wdone) {
      const int todo = min(kBatch, total - b * kBatch);
      int j = 0;
      while (true) {
        // ---------------- phase A: intersect, composite aux maps, queue samples.
        // Warp-synchronous walk: all lanes share `j`; votes only at the loop head.
        while (j < todo) {
          const bool active = !done;
          if (!__any_sync(0xffffffffu, active)) break;
          if (__any_sync(0xffffffffu, cnt == kQueue)) break;
          const int jj = j++;
          if (active) contributor++;
          // Outside the surfel's alpha >= 1/255 box the reference would reach
          // `alpha < 1/255 -> continue` (or an earlier continue): skip the math,
          // for the whole warp when no lane is inside.
          const float4 box = S.rec[s][jj][0];
          const bool cand = active && !(pxf < box.x || pxf > box.y || pyf < box.z || pyf > box.w);
          if (!__any_sync(0xffffffffu, cand)) continue;
          if (!cand) continue;
          const float4 q0 = S.rec[s][jj][1], q1 = S.rec[s][jj][2], q2 = S.rec[s][jj][3];
          const float3 Tu = f3(q0.x, q0.y, q0.z), Tv = f3(q0.w, q1.x, q1.y), Tw = f3(q1.z, q1.w, q2.x);
          const float3 kk = pxf * Tw - Tu;
          const float3 ll = pyf * Tw - Tv;
          const float3 pp = cross3(kk, ll);
          const float dx = q2.y - pxf, dy = q2.z - pyf;
          const float rho2d = kFilterInvSquare * (dx * dx + dy * dy);
          // Division-free pre-test: rho3d = |p.xy|^2 / p.z^2 and rho2d both above the
          // surfel's (margined) alpha cutoff means alpha < 1/255 on the reference path.
          const float rho_cut = S.rec[s][jj][7].y;
          if (pp.x * pp.x + pp.y * pp.y > rho_cut * (pp.z * pp.z) && rho2d > rho_cut) continue;
          if (pp.z == 0.0f) continue;
          const float sx = pp.x / pp.z, sy = pp.y / pp.z;
          const float rho3d = sx * sx + sy * sy;
          const float rho = fminf(rho3d, rho2d);
          const bool on_plane = rho3d <= rho2d;
          const float depth = on_plane ? (sx * Tw.x + sy * Tw.y) + Tw.z : Tw.z;
          if (depth < kNear) continue;
          float G;
          if (!kGeneral || p.kernel_type == 0) {
            const float power = -0.5f * rho;
            if (power > 0.0f) continue;
            G = expf(power);
            if (p.beta > 0.0f) G = (float)((1.0 + (double)p.beta) * G / (1.0 + (double)p.beta * G));
          } else {
            // The other splat kernels of forward.cu:864-902, with the record's shape.
            const float shape = S.rec[s][jj][7].w;
            if (p.kernel_type == 1) {  // beta kernel: (1 - rho)^shape inside the unit circle
              if (rho >= 1.0f) continue;
              G = powf(1.0f - rho, shape);
            } else if (p.kernel_type == 2) {  // flex: per-surfel beta
              const float power = -0.5f * rho;
              if (power > 0.0f) continue;
              G = expf(power);
              if (shape > 0.0f) G = (1.0f + shape) * G / (1.0f + shape * G);
            } else {  // general: exp(-0.5 rho^(shape / 2))
              const float power = -0.5f * powf(fmaxf(rho, 1e-8f), 0.5f * shape);
              if (power > 0.0f) continue;
              G = expf(power);
            }
          }
          const float alpha = fminf(0.99f, q2.w * G);
          if (alpha < 1.0f / 255.0f) continue;
          const float test_T = T * (1 - alpha);
          if (test_T < 0.0001f) {
            done = true;
            continue;
          }
          const float w = alpha * T;
          render_number++;
          if (p.max_intersections > 0 && render_number >= p.max_intersections) done = true;

          const float A = 1 - T;
          const float m = kFar / (kFar - kNear) * (1 - kNear / depth);
          distortion += (m * m * A + M2 - 2 * m * M1) * w;
          D += depth * w;
          M1 += m * w;
          M2 += m * m * w;
          if (T > 0.5f) {
            median_depth = depth;
            median_contributor = (float)contributor;
          }
          const float4 q3 = S.rec[s][jj][4];
          N0 += q3.x * w;
          N1 += q3.y * w;
          N2 += q3.z * w;

          const float4 q4 = S.rec[s][jj][5], q5 = S.rec[s][jj][6], q6 = S.rec[s][jj][7];
          float3 xyz;
          if (on_plane) {
            xyz = f3(sx * q4.x + sy * q4.w + q5.z, sx * q4.y + sy * q5.x + q5.w,
                     sx * q4.z + sy * q5.y + q6.x);
          } else {
            xyz = f3(q5.z, q5.w, q6.x);
          }
          // Mode 13 (forward.cu:964-1091) skips the hit point of its fast path
          // and, for every sample, the level colours, the transmittance record
          // and the last-contributor update.
          const bool m13 = kGeneral && (p.render_mode & 0xFF) == 13;
          const bool fast13 = m13 && (p.render_mode >> 8) != 0 &&
                              __ldg(p.gauss + (size_t)__float_as_uint(q6.z) * (2 * p.total_levels + 1) +
                                    2 * p.total_levels) > 0.5f;
          // Level 0 (forward.cu:1093-1096) adds the per-surfel colours only: no
          // position, no level colour, nothing queued for the hash grid.
          const bool lvl0 = kGeneral && p.render_mode == 0 && L == 0;
          if (!fast13 && !lvl0) {
            pos0 += w * xyz.x;
            pos1 += w * xyz.y;
            pos2 += w * xyz.z;
          }

          // query_feature's mapping of the hit point to [0,1]^3 (hashgrid.h:63-114).
          const uint32_t apl = __float_as_uint(q3.w);
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
          float hw = w;  // weight of this sample's hash features (0: nothing to look up)
          if (kGeneral && uses_surfel_rows(p.render_mode, p.L)) {
            const int base = p.render_mode & 0xFF;
            const uint32_t sid = __float_as_uint(q6.z);
            if (kSH && base >= 8 && base <= 10) {
              sh_hybrid_features<TableT>(p, S.lv[0], sid, w, in0, in1, in2, oob, apl, half_shift, S.acc, t, pid);
              hw = 0.0f;
            } else if (kSH && base == 11) {
              residual_sh(p, sid, xyz, f3(q5.z, q5.w, q6.x), w, S.acc, t);
            } else {
              hw = w * mode_features(p, sid, w, S.acc, t);
            }
          }
          if (!lvl0 && !(kGeneral && hw == 0.0f)) {
            S.samp[cnt][t] = make_float4(in0, in1, in2, hw);
            S.lvl[cnt][t] = (uint8_t)((oob || hw == 0.0f) ? 0u : min(apl, L));
            cnt++;
          }

          if (m13) {
            T = test_T;
            continue;
          }
          float ac0, ac1;
          if (apl <= 4) {
            ac0 = (float)((apl - 2) * 0.5);
            ac1 = 1.0f;
          } else {
            ac0 = 1.0f;
            ac1 = (float)(1.0 - (apl - 4) * 0.5);
          }
          if (!lvl0) {
            vis0 += ac0 * w;
            vis1 += ac1 * w;
          }
          if (p.record_transmittance) {
            const uint32_t id = __float_as_uint(S.rec[s][jj][7].z);  // the record's surfel index
            atomicAdd(p.cover_pixels + id, 1.0f);
            atomicAdd(p.trans_avg + id, T);
          }
          T = test_T;
          last_contributor = contributor;
        }

        // ---------------- phase B: this warp's hash lookups, when a queue is
        // full or the warp's pixels are all done (queues carry over between
        // batches). Each lane reads only its own queue and accumulator row.
        const bool qfull = __any_sync(0xffffffffu, cnt == kQueue);
        const bool alldone = !__any_sync(0xffffffffu, !done);
        if (qfull || alldone) drain();
        if (j >= todo || alldone) {
          wdone = alldone;
          break;
        }
      }
      if (wdone && lane == 0) atomicAdd(&S.ndone, 1);
    }
    // Release slot s; the last warp out refills it.
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&S.used[s], 1) == kWarps - 1;
      if (last) S.used[s] = 0;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last && b + kSlots < rounds && *(volatile int*)&S.ndone < kWarps) fetch(b + kSlots);
    if (wdone && *(volatile int*)&S.ndone == kWarps) break;
  }
  if (__any_sync(0xffffffffu, cnt > 0)) drain();
  asm volatile("cp.async.wait_all;" ::: "memory");

  if (inside) {
    const size_t HW = (size_t)p.H * p.W;
    p.final_T[pid] = T;
    p.final_T[pid + HW] = M1;
    p.final_T[pid + 2 * HW] = M2;
    p.n_contrib[pid] = last_contributor;
    p.n_contrib[pid + HW] = (uint32_t)median_contributor;  // -1 saturates to 0
    for (int c = 0; c < min(p.C, kMaxChannels); c++) {
      const float2 pr = *acc_pair(S.acc, t, c >> 1);
      p.out_color[c * HW + pid] = (c & 1) ? pr.y : pr.x;
    }
    float* o = p.out_others + pid;
    o[0 * HW] = D;
    o[1 * HW] = 1 - T;
    o[2 * HW] = N0;
    o[3 * HW] = N1;
    o[4 * HW] = N2;
    o[5 * HW] = median_depth;
    o[6 * HW] = distortion;
    o[7 * HW] = (float)render_number;
    o[8 * HW] = pos0;
    o[9 * HW] = pos1;
    o[10 * HW] = pos2;
    o[11 * HW] = vis0;
    o[12 * HW] = vis1;
    o[13 * HW] = 0.0f;
    if (kSH && (p.render_mode & 0xFF) == 11) {
      // mode 11's SH colour (forward.cu:2039-2045): out_others has 17 channels
#pragma unroll
      for (int c = 0; c < 3; c++) {
        const float2 pr = *acc_pair(S.acc, t, (p.C + c) >> 1);
        o[(14 + c) * HW] = ((p.C + c) & 1) ? pr.y : pr.x;
      }
    }
  }
}

template <typename TableT, int kVariant>
int launch_blend(const RenderParams& p, int tiles, cudaStream_t stream) {
  const int smem = (int)sizeof(BlendSmem);
  NS_CUDA_TRY(cudaFuncSetAttribute(blend_kernel<TableT, kVariant>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   smem));
  blend_kernel<TableT, kVariant><<<tiles * kBands, kThreads, smem, stream>>>(p);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace

// Supported: level_dim 2, up to 16 levels, up to 32 channels (C >= 2 L), fp16 or
// fp32 table; modes 8-10: one 3-wide level, C = 3 (48 for mode 9); mode 11: C + 3
// <= 32 (its SH colour takes three accumulators). Other shapes report
// NS_ERR_UNSUPPORTED (the reference prints and renders nothing for shapes it was
// not compiled for).
int render_launch(const RenderParams& p, int fp16, cudaStream_t stream) {
  const int base = p.render_mode & 0xFF;
  if (p.C <= 0) return NS_ERR_UNSUPPORTED;
  if (base >= 8 && base <= 10) {
    if (p.LD != 3 || p.L > 1 || p.C != (base == 9 ? 48 : 3)) return NS_ERR_UNSUPPORTED;
  } else {
    if (p.LD != 2 || p.C > kMaxChannels) return NS_ERR_UNSUPPORTED;
    if (base == 11 && p.C + 3 > kMaxChannels) return NS_ERR_UNSUPPORTED;
    const int hoff = hash_level_offset(p.render_mode, p.hybrid_levels);
    if (hoff < 0 || (int64_t)hoff + p.L > (uint32_t)(p.C / p.LD) || p.L > (uint32_t)kMaxLevels)
      return NS_ERR_UNSUPPORTED;
  }
  const int tiles = div_up(p.W, kTile) * div_up(p.H, kTile);
  if (tiles == 0) return NS_OK;
  if (base >= 8 && base <= 11)
    return fp16 ? launch_blend<__half, 2>(p, tiles, stream) : launch_blend<float, 2>(p, tiles, stream);
  if (p.kernel_type != 0 || uses_surfel_rows(p.render_mode, p.L))
    return fp16 ? launch_blend<__half, 1>(p, tiles, stream) : launch_blend<float, 1>(p, tiles, stream);
  return fp16 ? launch_blend<__half, 0>(p, tiles, stream) : launch_blend<float, 0>(p, tiles, stream);
}

}  // namespace ns
