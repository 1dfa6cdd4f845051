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

}  // namespace oracle
