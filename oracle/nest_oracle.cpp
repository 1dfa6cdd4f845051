// nest_oracle.cpp -- CPU restatement of nest-splatting's mode-0 forward rasterizer.
//
// TEST INFRASTRUCTURE ONLY. Nothing in the product links or calls this file:
// tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
// use it as the checker. The CUDA library in nest-splatting_b200/csrc is the
// product and never falls back to this code.
//
// Parity status: the reference rasterizer cannot be built in this image (its
// glm submodule is empty and glm is not installed), so this restatement is
// pinned by known-answer tests (dense/hash grid indices, a single surfel facing
// the camera, early termination on an opaque stack, one-hot RVQ decode) and,
// for the camera and homotrans inputs, by golden vectors produced by importing
// the reference's own Python utilities (tests/golden/make_golden.py).
//
// Every function cites the reference code it restates; paths are relative to
// submodules/diff-surfel-rasterization/ unless noted.
#include "oracle_math.h"

using namespace oracle;

// The feature vector of one blended sample in render modes 4, 12, 14: the
// per-surfel features of `gauss` (row id) and, where the mode asks for it, the
// L hash levels queried at the hit point (query() fills hf[0, L * LD)).
template <class Q>
void mode_feature(float* feat, int C, int LD, int render_mode, int hybrid_levels, int total_levels,
                  uint32_t L, const float* gauss, int id, float* hf, Q query) {
  const int base = render_mode & 0xFF;
  const bool infer = ((render_mode >> 8) & 1) != 0;
  const int pg = hybrid_levels * LD;
  const int hd = (int)L * LD;
  for (int c = 0; c < C; c++) feat[c] = 0.0f;
  if (base == 4) {  // :1218-1282
    const float* g = gauss + (size_t)id * pg;
    for (int i = 0; i < pg; i++) feat[i] = g[i];
    if (L > 0) {
      query();
      for (int i = 0; i < hd && pg + i < C; i++) feat[pg + i] = hf[i];
    }
  } else if (base == 12) {  // :1593-1700
    const int td = total_levels * LD;
    const float* g = gauss + (size_t)id * (td + 1);
    const float wgt = g[td];
    if (infer && wgt >= 0.9f) {
      for (int i = 0; i < td && i < C; i++) feat[i] = g[i];
    } else {
      for (int i = 0; i < pg; i++) feat[i] = g[i];
      if (L > 0) {
        query();
        for (int i = 0; i < hd && pg + i < C; i++)
          feat[pg + i] = infer ? hf[i] : wgt * g[pg + i] + (1.0f - wgt) * hf[i];
      }
    }
  } else if (base == 13) {  // :964-1091
    const int td = total_levels * LD;
    const float* g = gauss + (size_t)id * (td + 1);
    const float wgt = g[td];
    if (infer && wgt > 0.5f) {
      for (int i = 0; i < td && i < C; i++) feat[i] = g[i];
    } else if (infer) {
      for (int i = 0; i < pg && i < C; i++) feat[i] = g[i];
      if (L > 0) {
        query();
        for (int i = 0; i < hd && pg + i < C; i++) feat[pg + i] = hf[i];
      }
    } else {
      for (int i = 0; i < pg && i < C; i++) feat[i] = g[i] * wgt;
      if (L > 0) {
        query();
        for (int i = 0; i < hd && pg + i < C; i++) feat[pg + i] = wgt * g[pg + i] + (1.0f - wgt) * hf[i];
      }
    }
  } else if (base == 6) {  // :1283-1325: rows of C, uniform blend with the hash levels
    const float* g = gauss + (size_t)id * C;
    if (L > 0) query();
    for (int i = 0; i < hd && i < C; i++) feat[i] = 0.5f * g[i] + 0.5f * (L > 0 ? hf[i] : 0.0f);
  } else if (base == 7) {  // :1326-1377: rows of total LD + 1, weight last
    const int td = total_levels * LD;
    const float* g = gauss + (size_t)id * (td + 1);
    const float wgt = g[td];
    if (L > 0) query();
    for (int i = 0; i < td && i < C; i++)
      feat[i] = wgt * g[i] + (1.0f - wgt) * (L > 0 && i < hd ? hf[i] : 0.0f);
  } else if (base == 14) {  // :1701-1790
    const float* g = gauss + (size_t)id * (pg + 1);
    const float wgt = g[pg];
    for (int i = 0; i < pg && i < C; i++) feat[i] = g[i];
    if (L > 0 && (infer ? wgt >= 0.1f : wgt > 1e-6f)) {
      query();
      for (int i = 0; i < hd && pg + i < C; i++) feat[pg + i] = wgt * hf[i];
    }
  }
}

extern "C" {

// forward.cu:237-290 (compute_transmat), 294-320 (compute_aabb), 323-441
// (preprocessCUDA, colour path skipped: mode 0 never reads it), auxiliary.h:190-215
// (in_frustum). Per surfel outputs use the reference layouts:
//   means2D [P,2], depths [P], transMat [P,9] (Tu, Tv, Tw), normal_opacity [P,4],
//   radii [P] int32, tiles_touched [P] uint32.
// Ts: NULL, or precomputed transforms [P, 9] (columns Tu, Tv, Tw; the
// reference's transMat_precomp, forward.cu:366-380), whose normal is the view
// axis (0, 0, 1) before the camera-facing flip; scales and rotations are then
// not read.
static void preprocess_impl(int P, const float* means3D, const float* scales, float mod,
                            const float* rotations, const float* opacities, const float* viewmatrix,
                            const float* projmatrix, int W, int H, int* radii, float* means2D,
                            float* depths, float* transMat, float* normal_opacity,
                            uint32_t* tiles_touched, const float* Ts) {
  const int gx = (W + kBlock - 1) / kBlock, gy = (H + kBlock - 1) / kBlock;
#pragma omp parallel for schedule(static)
  for (int i = 0; i < P; i++) {
    radii[i] = 0;
    tiles_touched[i] = 0;
    F3 p = {means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]};
    F3 pv = xform_point4x3(p, viewmatrix);
    if (pv.z <= 0.2f) continue;
    F3 Tu, Tv, Tw, n;
    if (Ts) {
      const float* t = Ts + 9 * (size_t)i;
      Tu = {t[0], t[1], t[2]};
      Tv = {t[3], t[4], t[5]};
      Tw = {t[6], t[7], t[8]};
      n = {0.f, 0.f, 1.f};
    } else {
    F3 R[3];
    quat_to_cols(rotations + 4 * i, R);
    F3 L0 = scl(mod * scales[2 * i], R[0]);
    F3 L1 = scl(mod * scales[2 * i + 1], R[1]);
    F3 L2 = R[2];
    // h_r = projmatrix applied to basis r (homogeneous); T column c row r.
    float basis[3][4] = {{L0.x, L0.y, L0.z, 0.f}, {L1.x, L1.y, L1.z, 0.f}, {p.x, p.y, p.z, 1.f}};
    float Q[4][3];
    for (int c = 0; c < 4; c++)
      for (int r = 0; r < 3; r++)
        Q[c][r] = basis[r][0] * projmatrix[c] + basis[r][1] * projmatrix[4 + c] +
                  basis[r][2] * projmatrix[8 + c] + basis[r][3] * projmatrix[12 + c];
    const float hw = float(W) / 2.0f, hh = float(H) / 2.0f;
    const float cw = float(W - 1) / 2.0f, ch = float(H - 1) / 2.0f;
    float* tu = &Tu.x; float* tv = &Tv.x; float* tw = &Tw.x;
    for (int r = 0; r < 3; r++) {
      tu[r] = Q[0][r] * hw + Q[3][r] * cw;
      tv[r] = Q[1][r] * hh + Q[3][r] * ch;
      tw[r] = Q[3][r];
    }
    n = xform_vec4x3(L2, viewmatrix);
    float nl = std::sqrt(n.x * n.x + n.y * n.y + n.z * n.z);
    if (nl > 1e-7f) { n.x /= nl; n.y /= nl; n.z /= nl; }
    }
    float cosv = -(pv.x * n.x + pv.y * n.y + pv.z * n.z);
    if (cosv == 0) continue;
    float mult = cosv > 0 ? 1.f : -1.f;
    n = scl(mult, n);
    const float cutoff = 4.0f;
    // glm: t = (c^2, c^2, -1); d = dot(t, Tw*Tw); f = (1/d) t; p = (dot(f, Tu*Tw), dot(f, Tv*Tw))
    const float t0 = cutoff * cutoff;
    float d = t0 * (Tw.x * Tw.x) + t0 * (Tw.y * Tw.y) + -1.0f * (Tw.z * Tw.z);
    if (d == 0.0f) continue;
    F3 f = {(1 / d) * t0, (1 / d) * t0, (1 / d) * -1.0f};
    float ppx = f.x * (Tu.x * Tw.x) + f.y * (Tu.y * Tw.y) + f.z * (Tu.z * Tw.z);
    float ppy = f.x * (Tv.x * Tw.x) + f.y * (Tv.y * Tw.y) + f.z * (Tv.z * Tw.z);
    float h0x = ppx * ppx - (f.x * (Tu.x * Tu.x) + f.y * (Tu.y * Tu.y) + f.z * (Tu.z * Tu.z));
    float h0y = ppy * ppy - (f.x * (Tv.x * Tv.x) + f.y * (Tv.y * Tv.y) + f.z * (Tv.z * Tv.z));
    float ex = std::sqrt(std::max(1e-4f, h0x));
    float ey = std::sqrt(std::max(1e-4f, h0y));
    float radius = std::ceil(std::max(std::max(ex, ey), cutoff * kFilterSize));
    int x0, y0, x1, y1;
    get_rect(ppx, ppy, (int)radius, gx, gy, x0, y0, x1, y1);
    if ((x1 - x0) * (y1 - y0) == 0) continue;
    depths[i] = pv.z;
    radii[i] = (int)radius;
    means2D[2 * i] = ppx;
    means2D[2 * i + 1] = ppy;
    float* T = transMat + 9 * i;
    T[0] = Tu.x; T[1] = Tu.y; T[2] = Tu.z;
    T[3] = Tv.x; T[4] = Tv.y; T[5] = Tv.z;
    T[6] = Tw.x; T[7] = Tw.y; T[8] = Tw.z;
    normal_opacity[4 * i] = n.x;
    normal_opacity[4 * i + 1] = n.y;
    normal_opacity[4 * i + 2] = n.z;
    normal_opacity[4 * i + 3] = opacities[i];
    tiles_touched[i] = (uint32_t)((y1 - y0) * (x1 - x0));
  }
}

void oracle_preprocess(int P, const float* means3D, const float* scales, float mod,
                       const float* rotations, const float* opacities, const float* viewmatrix,
                       const float* projmatrix, int W, int H, int* radii, float* means2D,
                       float* depths, float* transMat, float* normal_opacity,
                       uint32_t* tiles_touched) {
  preprocess_impl(P, means3D, scales, mod, rotations, opacities, viewmatrix, projmatrix, W, H, radii, means2D,
                  depths, transMat, normal_opacity, tiles_touched, nullptr);
}

// The same with precomputed transforms Ts [P, 9] (transMat_precomp).
void oracle_preprocess_precomp(int P, const float* means3D, const float* Ts, const float* opacities,
                               const float* viewmatrix, const float* projmatrix, int W, int H, int* radii,
                               float* means2D, float* depths, float* transMat, float* normal_opacity,
                               uint32_t* tiles_touched) {
  preprocess_impl(P, means3D, nullptr, 1.0f, nullptr, opacities, viewmatrix, projmatrix, W, H, radii, means2D,
                  depths, transMat, normal_opacity, tiles_touched, Ts);
}

// rasterizer_impl.cu:70-111 (duplicateWithKeys), 381-386 (stable radix sort on
// [tile | depth bits]), 173-195 (identifyTileRanges). Returns the instance
// count; writes at most `cap` pairs (returns -count when cap is too small).
// ranges has 2*tiles entries, [start, end) per tile, zero for empty tiles.
int64_t oracle_bin(int P, const float* means2D, const float* depths, const int* radii, int W,
                   int H, uint64_t* keys, uint32_t* vals, int64_t cap, uint32_t* ranges) {
  const int gx = (W + kBlock - 1) / kBlock, gy = (H + kBlock - 1) / kBlock;
  std::vector<std::pair<uint64_t, uint32_t>> inst;
  for (int i = 0; i < P; i++) {
    if (radii[i] <= 0) continue;
    int x0, y0, x1, y1;
    get_rect(means2D[2 * i], means2D[2 * i + 1], radii[i], gx, gy, x0, y0, x1, y1);
    uint32_t dbits;
    std::memcpy(&dbits, &depths[i], 4);
    for (int y = y0; y < y1; y++)
      for (int x = x0; x < x1; x++)
        inst.push_back({((uint64_t)(uint32_t)(y * gx + x) << 32) | dbits, (uint32_t)i});
  }
#ifdef _OPENMP
  __gnu_parallel::stable_sort(inst.begin(), inst.end(),
#else
  std::stable_sort(inst.begin(), inst.end(),
#endif
                   [](const std::pair<uint64_t, uint32_t>& a, const std::pair<uint64_t, uint32_t>& b) {
                     return a.first < b.first;
                   });
  int64_t n = (int64_t)inst.size();
  std::memset(ranges, 0, sizeof(uint32_t) * 2 * (size_t)gx * gy);
  if (n > cap) return -n;
  for (int64_t k = 0; k < n; k++) {
    keys[k] = inst[k].first;
    vals[k] = inst[k].second;
    uint32_t t = (uint32_t)(inst[k].first >> 32);
    if (k == 0) ranges[2 * t] = 0;
    else {
      uint32_t pt = (uint32_t)(inst[k - 1].first >> 32);
      if (pt != t) { ranges[2 * pt + 1] = (uint32_t)k; ranges[2 * t] = (uint32_t)k; }
    }
    if (k == n - 1) ranges[2 * t + 1] = (uint32_t)n;
  }
  return n;
}

// forward.cu:639-2049, render_mode 0 with level > 0, kernel_type 0 (Gaussian) or
// the beta / flex / general kernels of :864-902 (kernel_type 1-3, shapes[P]):
// ray/surfel intersection (:839-858), alpha and termination (:903-939),
// auxiliary maps (:941-959), hit point and hash query (:1099-1145, 1914-1916),
// level visualisation colour (:1945-1957), transmittance record (:1961-1964),
// outputs (:2008-2048). homotrans is [P,16] row-major (general_utils.py:101-113).
// table is fp32 [sum_l T_l, LD]; offsets int32 [L+1].
// render_mode (base | inference flag << 8): 0, or the modes that combine
// per-surfel features `gauss` (colors_precomp) with the hash grid's L levels at
// channel hybrid_levels * LD: 4 cat (:1218-1282), 12 adaptive_cat (:1593-1700),
// 13 adaptive_cat_fast (:964-1091), 14 adaptive_zero (:1701-1790); see
// mode_feature(). Mode 13 leaves out the hit point of its fast path and, for
// every sample, the level colours, the transmittance record and the
// last-contributor update (its `continue` at :1088-1090).
void oracle_render(int W, int H, const uint32_t* ranges, const uint32_t* point_list,
                   const float* means2D, const float* transMat, const float* normal_opacity,
                   const float* homotrans, const float* ap_level, const float* table,
                   const int* offsets, const float* gridrange, int C, int LD, uint32_t L,
                   float S, uint32_t Hres, int align_corners, uint32_t interp, int contract,
                   float beta, uint32_t max_intersections, int record_transmittance,
                   float* out_color, float* out_others, float* final_T, uint32_t* n_contrib,
                   float* cover_pixels, float* trans_avg, int row_stride, int kernel_type,
                   const float* shapes, int render_mode, int hybrid_levels, int total_levels,
                   const float* gauss) {
  const int gx = (W + kBlock - 1) / kBlock, gy = (H + kBlock - 1) / kBlock;
  const size_t HW = (size_t)H * W;
  const float vmin = gridrange[0], vmax = gridrange[1];
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < gx * gy; tile++) {
    std::vector<float> Cacc(C), feat(C > 0 ? C : 1), hf(16 * LD);
    const int tx = tile % gx, ty = tile / gx;
    if (row_stride > 1 && ty % row_stride != 0) continue;
    const uint32_t r0 = ranges[2 * tile], r1 = ranges[2 * tile + 1];
    for (int py = ty * kBlock; py < std::min(H, (ty + 1) * kBlock); py++) {
      for (int px = tx * kBlock; px < std::min(W, (tx + 1) * kBlock); px++) {
        const size_t pid = (size_t)py * W + px;
        const float pxf = (float)px, pyf = (float)py;
        float T = 1.0f;
        uint32_t contributor = 0, last_contributor = 0, render_number = 0;
        std::fill(Cacc.begin(), Cacc.end(), 0.f);
        float N[3] = {0, 0, 0}, D = 0, M1 = 0, M2 = 0, distortion = 0, median_depth = 0;
        float median_contributor = -1;
        float pos[3] = {0, 0, 0}, vis[3] = {0, 0, 0}, sh_rgb[3] = {0, 0, 0};
        bool done = false;
        for (uint32_t k = r0; k < r1 && !done; k++) {
          contributor++;
          const uint32_t id = point_list[k];
          const float* Tm = transMat + 9 * (size_t)id;
          F3 Tu = {Tm[0], Tm[1], Tm[2]}, Tv = {Tm[3], Tm[4], Tm[5]}, Tw = {Tm[6], Tm[7], Tm[8]};
          F3 kk = sub(scl((float)px, Tw), Tu);
          F3 ll = sub(scl((float)py, Tw), Tv);
          F3 p = crs(kk, ll);
          if (p.z == 0.0f) continue;
          float sx = p.x / p.z, sy = p.y / p.z;
          float rho3d = sx * sx + sy * sy;
          float dx = means2D[2 * id] - pxf, dy = means2D[2 * id + 1] - pyf;
          float rho2d = kFilterInvSquare * (dx * dx + dy * dy);
          float rho = std::min(rho3d, rho2d);
          float depth = (rho3d <= rho2d) ? (sx * Tw.x + sy * Tw.y) + Tw.z : Tw.z;
          if (depth < kNear) continue;
          const float* no = normal_opacity + 4 * (size_t)id;
          float G;
          if (kernel_type == 1) {
            if (rho >= 1.0f) continue;
            G = powf(1.0f - rho, shapes[id]);
          } else if (kernel_type == 2) {
            float power = -0.5f * rho;
            if (power > 0.0f) continue;
            G = std::exp(power);
            const float b = shapes[id];
            if (b > 0.0f) G = (1.0f + b) * G / (1.0f + b * G);
          } else if (kernel_type == 3) {
            const float pt = powf(std::max(rho, 1e-8f), 0.5f * shapes[id]);
            float power = -0.5f * pt;
            if (power > 0.0f) continue;
            G = std::exp(power);
          } else {
            float power = -0.5f * rho;
            if (power > 0.0f) continue;
            G = std::exp(power);
            if (beta > 0.0) G = (float)((1.0 + beta) * G / (1.0 + beta * G));
          }
          float alpha = std::min(0.99f, no[3] * G);
          if (alpha < 1.0f / 255.0f) continue;
          float test_T = T * (1 - alpha);
          if (test_T < 0.0001f) { done = true; continue; }
          float w = alpha * T;
          render_number++;
          if (max_intersections > 0 && render_number >= max_intersections) done = true;
          float A = 1 - T;
          float m = kFar / (kFar - kNear) * (1 - kNear / depth);
          distortion += (m * m * A + M2 - 2 * m * M1) * w;
          D += depth * w;
          M1 += m * w;
          M2 += m * m * w;
          if (T > 0.5f) { median_depth = depth; median_contributor = (float)contributor; }
          for (int c = 0; c < 3; c++) N[c] += no[c] * w;
          const float* h = homotrans + 16 * (size_t)id;
          F3 pk = {h[3], h[7], h[11]};
          F3 xyz;
          if (rho3d <= rho2d) {
            xyz = {sx * h[0] + sy * h[1] + pk.x, sx * h[4] + sy * h[5] + pk.y,
                   sx * h[8] + sy * h[9] + pk.z};
          } else {
            xyz = pk;
          }
          const bool m13 = (render_mode & 0xFF) == 13;
          const bool fast13 = m13 && ((render_mode >> 8) & 1) &&
                              gauss[(size_t)id * (total_levels * LD + 1) + total_levels * LD] > 0.5f;
          // level 0 (forward.cu:1093-1096): the per-surfel colours only; no hit
          // point, position or level colour
          const bool lvl0 = render_mode == 0 && L == 0;
          if (lvl0) {
            for (int c = 0; c < C; c++) Cacc[c] += gauss[(size_t)id * C + c] * w;
            if (record_transmittance) {
#pragma omp atomic
              cover_pixels[id] += 1.0f;
#pragma omp atomic
              trans_avg[id] += T;
            }
            T = test_T;
            last_contributor = contributor;
            continue;
          }
          if (!fast13) {
            pos[0] += w * xyz.x;
            pos[1] += w * xyz.y;
            pos[2] += w * xyz.z;
          }
          uint32_t apl = (uint32_t)std::floor(ap_level[id]);
          const int base = render_mode & 0xFF;
          if (base == 0 || base == 11) {
            // mode 11 (residual_hybrid, forward.cu:1527-1592): the L hash levels
            // from channel 0, as mode 0; its SH colour is accumulated below
            query_feature(feat.data(), C, LD, xyz, vmin, vmax, offsets, apl, table, L, S, Hres,
                          align_corners != 0, interp, contract != 0);
          } else if (base >= 8 && base <= 10) {
            // one 3-wide hash level (query_feature<false, 3, 3> with level 1)
            const int decompose = hybrid_levels;
            float h[3] = {0.f, 0.f, 0.f};
            if (L > 0 && decompose != 1)
              query_feature(h, 3, 3, xyz, vmin, vmax, offsets, apl, table, 1, S, Hres,
                            align_corners != 0, interp, contract != 0);
            sh_hybrid_feature(base, decompose, gauss + (size_t)id * (base == 9 ? 48 : 3), h, feat.data());
          } else {
            auto query = [&]() {
              query_feature(hf.data(), (int)L * LD, LD, xyz, vmin, vmax, offsets, apl, table, L, S,
                            Hres, align_corners != 0, interp, contract != 0);
            };
            mode_feature(feat.data(), C, LD, render_mode, hybrid_levels, total_levels, L, gauss, id,
                         hf.data(), query);
          }
          for (int c = 0; c < C; c++) Cacc[c] += feat[c] * w;
          if (base == 11) {
            // forward.cu:1918-1943: the surfel's degree-3 SH (48 coefficients read
            // interleaved) along the direction from its centre to the hit point
            F3 dir = {xyz.x - pk.x, xyz.y - pk.y, xyz.z - pk.z};
            const float inv_len = 1.0f / std::sqrt(dir.x * dir.x + dir.y * dir.y + dir.z * dir.z);
            dir = {dir.x * inv_len, dir.y * inv_len, dir.z * inv_len};
            float rgb[3];
            eval_sh_interleaved(3, gauss + (size_t)id * 48, dir, rgb);
            for (int c = 0; c < 3; c++) sh_rgb[c] += w * rgb[c];
          }
          if (m13) {
            T = T * (1 - alpha);
            continue;
          }
          float apc[3] = {0, 0, 0};
          if (apl <= 4) { apc[0] = (float)((apl - 2) * 0.5); apc[1] = 1.0f; }
          else { apc[0] = 1.0f; apc[1] = (float)(1.0 - (apl - 4) * 0.5); }
          for (int c = 0; c < 3; c++) vis[c] += apc[c] * w;
          if (record_transmittance) {
#pragma omp atomic
            cover_pixels[id] += 1.0f;
#pragma omp atomic
            trans_avg[id] += T;
          }
          T = test_T;
          last_contributor = contributor;
        }
        final_T[pid] = T;
        final_T[pid + HW] = M1;
        final_T[pid + 2 * HW] = M2;
        n_contrib[pid] = last_contributor;
        // float -> uint32 of -1 saturates to 0 on the device (cvt.rzi.u32.f32).
        n_contrib[pid + HW] = median_contributor < 0 ? 0u : (uint32_t)median_contributor;
        for (int c = 0; c < C; c++) out_color[c * HW + pid] = Cacc[c];
        out_others[pid + 0 * HW] = D;
        out_others[pid + 1 * HW] = 1 - T;
        for (int c = 0; c < 3; c++) out_others[pid + (2 + c) * HW] = N[c];
        out_others[pid + 5 * HW] = median_depth;
        out_others[pid + 6 * HW] = distortion;
        out_others[pid + 7 * HW] = (float)render_number;
        for (int c = 0; c < 3; c++) out_others[pid + (8 + c) * HW] = pos[c];
        for (int c = 0; c < 3; c++) out_others[pid + (11 + c) * HW] = vis[c];
        // mode 11: channels 14-16 (forward.cu:2039-2045; out_others has 17 channels)
        if ((render_mode & 0xFF) == 11)
          for (int c = 0; c < 3; c++) out_others[pid + (14 + c) * HW] = sh_rgb[c];
      }
    }
  }
  (void)kOthers;
}

// SH colours of P surfels (forward.cu:414-423 with computeColorFromSH, :21-74):
// shs [P, M, 3], campos [3]; rgb [P, 3] (clamped at 0).
void oracle_sh_color(int P, int deg, int M, const float* means3D, const float* campos, const float* shs,
                     float* rgb) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < P; i++) {
    F3 d = {means3D[3 * i] - campos[0], means3D[3 * i + 1] - campos[1], means3D[3 * i + 2] - campos[2]};
    const float len = std::sqrt(d.x * d.x + d.y * d.y + d.z * d.z);
    d = {d.x / len, d.y / len, d.z / len};
    bool clamped[3];
    sh_color(deg, shs + (size_t)i * M * 3, d, rgb + 3 * (size_t)i, clamped);
  }
}

// Hash-grid lookup of a batch of points (hashgrid.h:53-212), exported for the
// known-answer tests of grid_index and the trilinear gather.
// level_exp2: NULL, or [L] values of exp2f(l S) to use instead of the host's.
void oracle_query(int n, const float* xyz, const uint32_t* ap_level, const float* table,
                  const int* offsets, float vmin, float vmax, int C, int LD, uint32_t L, float S,
                  uint32_t Hres, int align_corners, uint32_t interp, int contract,
                  const float* level_exp2, float* out) {
  for (int i = 0; i < n; i++) {
    F3 p = {xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2]};
    query_feature(out + (size_t)i * C, C, LD, p, vmin, vmax, offsets, ap_level[i], table, L, S,
                  Hres, align_corners != 0, interp, contract != 0, level_exp2);
  }
}

uint32_t oracle_grid_index(int align_corners, uint32_t hashmap_size, uint32_t res, uint32_t x,
                           uint32_t y, uint32_t z) {
  uint32_t g[3] = {x, y, z};
  return grid_index(align_corners != 0, hashmap_size, res, g);
}

// RVQ decode (benchmark config 0 definition; the reference has no RVQ code):
// out[n,:] = sum over stages k = 0..K-1 of codebooks[k, idx[n,k], :], accumulated
// in fp32 starting from +0.0 in stage order.
void oracle_rvq_decode(int64_t n, int K, int E, int Dm, const uint8_t* idx, const float* cb,
                       float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) {
    float* o = out + i * Dm;
    for (int d = 0; d < Dm; d++) o[d] = 0.0f;
    for (int k = 0; k < K; k++) {
      const float* row = cb + ((size_t)k * E + idx[i * K + k]) * Dm;
      for (int d = 0; d < Dm; d++) o[d] += row[d];
    }
  }
}

// Threads of the OpenMP regions from now on (n <= 0: leave unchanged); a
// launcher's OMP_NUM_THREADS=1 would otherwise pin the CPU baseline to one core.
void oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int oracle_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
