// oracle_math.h -- helpers shared by the CPU oracle's forward and backward
// restatements (TEST INFRASTRUCTURE ONLY; see nest_oracle.cpp).
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#include <parallel/algorithm>
#endif


namespace oracle {

inline constexpr int kBlock = 16;           // cuda_rasterizer/config.h:17-18
inline constexpr float kNear = 0.2f;        // cuda_rasterizer/auxiliary.h:42
inline constexpr float kFar = 100.0f;       // cuda_rasterizer/auxiliary.h:43
inline constexpr float kFilterSize = 0.707106f;     // auxiliary.h:44
inline constexpr float kFilterInvSquare = 2.0f;     // auxiliary.h:45
inline constexpr int kOthers = 14;          // rasterize_points.cu:159 (3+3+1+1+3+3)

struct F3 { float x, y, z; };
inline F3 sub(F3 a, F3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
inline F3 scl(float f, F3 a) { return {f * a.x, f * a.y, f * a.z}; }
inline F3 crs(F3 a, F3 b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}

// auxiliary.h:84-92 (column-major 4x4, row-vector convention of the torch tensor)
inline F3 xform_point4x3(F3 p, const float* m) {
  return {m[0] * p.x + m[4] * p.y + m[8] * p.z + m[12],
          m[1] * p.x + m[5] * p.y + m[9] * p.z + m[13],
          m[2] * p.x + m[6] * p.y + m[10] * p.z + m[14]};
}
// auxiliary.h:105-113
inline F3 xform_vec4x3(F3 p, const float* m) {
  return {m[0] * p.x + m[4] * p.y + m[8] * p.z,
          m[1] * p.x + m[5] * p.y + m[9] * p.z,
          m[2] * p.x + m[6] * p.y + m[10] * p.z};
}

// auxiliary.h:218-240: unit-quaternion (w,x,y,z stored as x,y,z,w fields) to a
// rotation matrix. Returned as three columns.
inline void quat_to_cols(const float* q, F3 col[3]) {
  float s = 1.0f / std::sqrt(q[3] * q[3] + q[0] * q[0] + q[1] * q[1] + q[2] * q[2]);
  float w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
  col[0] = {1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z), 2.f * (x * z - w * y)};
  col[1] = {2.f * (x * y - w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x)};
  col[2] = {2.f * (x * z + w * y), 2.f * (y * z - w * x), 1.f - 2.f * (x * x + y * y)};
}

// auxiliary.h:72-82
inline void get_rect(float px, float py, int r, int gx, int gy, int& x0, int& y0, int& x1, int& y1) {
  auto clampi = [](int v, int hi) { return std::min(hi, std::max(0, v)); };
  x0 = clampi((int)((px - r) / kBlock), gx);
  y0 = clampi((int)((py - r) / kBlock), gy);
  x1 = clampi((int)((px + r + kBlock - 1) / kBlock), gx);
  y1 = clampi((int)((py + r + kBlock - 1) / kBlock), gy);
}

// hashgrid.h:7-20 (D = 3)
inline uint32_t fast_hash3(const uint32_t g[3]) {
  return (g[0] * 1u) ^ (g[1] * 2654435761u) ^ (g[2] * 805459861u);
}

// hashgrid.h:22-40 with C = LD (the channel offset is applied by the caller).
inline uint32_t grid_index(bool align_corners, uint32_t hashmap_size, uint32_t res, const uint32_t g[3]) {
  uint32_t stride = 1, index = 0;
  for (uint32_t d = 0; d < 3 && stride <= hashmap_size; d++) {
    index += g[d] * stride;
    stride *= align_corners ? res : (res + 1);
  }
  if (stride > hashmap_size) index = fast_hash3(g);
  return index % hashmap_size;
}

// exp2f(l * S) of hashgrid.h:128 (the level scale is exp2f(l S) H - 1). The
// host's exp2f and the device's may differ in the last place (CUDA documents
// up to 2 ulp for exp2f); level_exp2, when given, supplies the device's value
// per level so a check can take that difference out.
inline float level_exp2(uint32_t l, float S, const float* level_exp2) {
  return level_exp2 ? level_exp2[l] : std::exp2(l * S);
}

// hashgrid.h:53-212 (forward only, BW = false). feat has room for C channels.
inline void query_feature(float* feat, int C, int LD, F3 xyz, float vmin, float vmax, const int* offsets,
                   uint32_t ap_level, const float* table, uint32_t L, float S, uint32_t Hres,
                   bool align_corners, uint32_t interp, bool contract,
                   const float* lexp2 = nullptr) {
  float in[3];
  bool oob = false;
  if (!contract) {
    float inv = 1.0f / (vmax - vmin);
    in[0] = (xyz.x - vmin) * inv;
    in[1] = (xyz.y - vmin) * inv;
    in[2] = (xyz.z - vmin) * inv;
    oob = in[0] < 0 || in[0] > 1 || in[1] < 0 || in[1] > 1 || in[2] < 0 || in[2] > 1;
  } else {
    float vmid = (vmax + vmin) * 0.5f;
    float inv = 1.0f / ((vmax - vmin) * 0.5f);
    in[0] = (xyz.x - vmid) * inv;
    in[1] = (xyz.y - vmid) * inv;
    in[2] = (xyz.z - vmid) * inv;
    float norm = std::sqrt(in[0] * in[0] + in[1] * in[1] + in[2] * in[2]);
    float inv_norm = 1.0f / norm;
    float st = (norm <= 1.0f) ? 1.0f : (2.0f - inv_norm) * inv_norm;
    for (int d = 0; d < 3; d++) in[d] = (st * in[d] + 2.0f) * 0.25f;
  }
  uint32_t max_level = std::min(ap_level, L);
  for (int c = 0; c < C; c++) feat[c] = 0.f;
  if (oob) return;
  for (uint32_t lv = 0; lv < max_level; lv++) {
    uint32_t hsize = (uint32_t)(offsets[lv + 1] - offsets[lv]);
    float scale = level_exp2(lv, S, lexp2) * Hres - 1.0f;
    uint32_t res = (uint32_t)std::ceil(scale) + 1;
    const float* grid = table + (size_t)(uint32_t)offsets[lv] * LD;
    float pos[3];
    uint32_t pg[3];
    for (int d = 0; d < 3; d++) {
      // nvcc contracts the reference's `inputs[d] * scale + 0.5f` (and the
      // corner sums below) into fused multiply-adds; std::fma does the same.
      pos[d] = std::fma(in[d], scale, align_corners ? 0.0f : 0.5f);
      pg[d] = (uint32_t)std::floor(pos[d]);
      pos[d] -= (float)pg[d];
      if (interp == 1) pos[d] = pos[d] * pos[d] * (3.0f - 2.0f * pos[d]);
    }
    float r[16] = {0};
    for (uint32_t c = 0; c < 8; c++) {
      float w = 1;
      uint32_t g[3];
      for (int d = 0; d < 3; d++) {
        if ((c & (1u << d)) == 0) { w *= 1 - pos[d]; g[d] = pg[d]; }
        else { w *= pos[d]; g[d] = pg[d] + 1; }
      }
      uint32_t idx = grid_index(align_corners, hsize, res, g) * LD;
      for (int ch = 0; ch < LD; ch++) r[ch] = std::fma(w, grid[idx + ch], r[ch]);
    }
    for (int ch = 0; ch < LD; ch++) feat[lv * LD + ch] = r[ch];
  }
}

// Real spherical-harmonic basis up to degree 3 (the standard normalisation
// constants of the 3D Gaussian splatting SH colour model), evaluated as the
// reference's eval_sh_inline (forward.cu:76-155) does for render mode 11: the
// 48 coefficients are read interleaved (coefficient k of channel c at 3 k + c),
// 0.5 is added to the DC term and the result is clamped at 0.
inline void eval_sh_interleaved(int deg, const float* sh, F3 dir, float* out) {
  const float C0 = 0.28209479177387814f, C1 = 0.4886025119029199f;
  const float C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                       -1.0925484305920792f, 0.5462742152960396f};
  const float C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                       0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                       -0.5900435899266435f};
  for (int c = 0; c < 3; c++) out[c] = C0 * sh[c] + 0.5f;
  if (deg > 0) {
    const float x = dir.x, y = dir.y, z = dir.z;
    for (int c = 0; c < 3; c++)
      out[c] = out[c] - C1 * y * sh[3 + c] + C1 * z * sh[6 + c] - C1 * x * sh[9 + c];
    if (deg > 1) {
      const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
      for (int c = 0; c < 3; c++)
        out[c] = out[c] + C2[0] * xy * sh[12 + c] + C2[1] * yz * sh[15 + c] +
                 C2[2] * (2.0f * zz - xx - yy) * sh[18 + c] + C2[3] * xz * sh[21 + c] +
                 C2[4] * (xx - yy) * sh[24 + c];
      if (deg > 2) {
        for (int c = 0; c < 3; c++)
          out[c] = out[c] + C3[0] * y * (3.0f * xx - yy) * sh[27 + c] + C3[1] * xy * z * sh[30 + c] +
                   C3[2] * y * (4.0f * zz - xx - yy) * sh[33 + c] +
                   C3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy) * sh[36 + c] +
                   C3[4] * x * (4.0f * zz - xx - yy) * sh[39 + c] + C3[5] * z * (xx - yy) * sh[42 + c] +
                   C3[6] * x * (xx - 3.0f * yy) * sh[45 + c];
      }
    }
  }
  for (int c = 0; c < 3; c++) out[c] = std::fmax(out[c], 0.0f);
}

// The 3D Gaussian splatting SH colour of a surfel (forward.cu:21-74,
// computeColorFromSH): sh holds M coefficients as RGB triples (coefficient k
// at 3 k), dir the unit direction from the camera centre to the mean; degree
// deg <= 3 terms, + 0.5, clamped at 0 (clamped[c]: the sum was negative).
inline void sh_color(int deg, const float* sh, F3 dir, float* out, bool* clamped) {
  const float C0 = 0.28209479177387814f, C1 = 0.4886025119029199f;
  const float C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                       -1.0925484305920792f, 0.5462742152960396f};
  const float C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                       0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                       -0.5900435899266435f};
  const float x = dir.x, y = dir.y, z = dir.z;
  const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
  for (int c = 0; c < 3; c++) {
    auto k = [&](int i) { return sh[3 * i + c]; };
    float r = C0 * k(0);
    if (deg > 0) {
      r = r - C1 * y * k(1) + C1 * z * k(2) - C1 * x * k(3);
      if (deg > 1) {
        r = r + C2[0] * xy * k(4) + C2[1] * yz * k(5) + C2[2] * (2.0f * zz - xx - yy) * k(6) +
            C2[3] * xz * k(7) + C2[4] * (xx - yy) * k(8);
        if (deg > 2)
          r = r + C3[0] * y * (3.0f * xx - yy) * k(9) + C3[1] * xy * z * k(10) +
              C3[2] * y * (4.0f * zz - xx - yy) * k(11) + C3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy) * k(12) +
              C3[4] * x * (4.0f * zz - xx - yy) * k(13) + C3[5] * z * (xx - yy) * k(14) +
              C3[6] * x * (xx - 3.0f * yy) * k(15);
      }
    }
    r += 0.5f;
    clamped[c] = r < 0;
    out[c] = std::fmax(r, 0.0f);
  }
}

// Render modes 8 (hybrid_SH), 9 (hybrid_SH_post) and 10 (hybrid_SH_raw),
// forward.cu:1378-1526: the sample's feature from the surfel's row `g` (3 raw
// SH colours; 48 SH coefficients for mode 9) and h, the single-level, 3-wide
// hash value at the hit point (zero when not queried). decompose: 0 both
// parts, 1 the surfel only, 2 the grid only. Writes C = 3 (48) channels.
inline void sh_hybrid_feature(int base, int decompose, const float* g, const float h[3], float* feat) {
  if (base == 8) {
    for (int c = 0; c < 3; c++) {
      const float gr = std::fmax(0.0f, std::fmin(1.0f, g[c] + 0.5f));
      const float hr = 1.0f / (1.0f + std::exp(-h[c]));
      feat[c] = decompose == 2 ? hr : decompose == 1 ? gr : std::fmax(0.0f, std::fmin(1.0f, gr + hr));
    }
  } else if (base == 10) {
    for (int c = 0; c < 3; c++) {
      const float comb = decompose == 2 ? h[c] : decompose == 1 ? g[c] : g[c] + h[c];
      feat[c] = 1.0f / (1.0f + std::exp(-comb));
    }
  } else {
    for (int i = 0; i < 48; i++) feat[i] = g[i];
    for (int c = 0; c < 3; c++) {
      if (decompose == 2) feat[16 * c] = h[c];
      else if (decompose != 1) feat[16 * c] += h[c];
    }
  }
}

}  // namespace oracle
