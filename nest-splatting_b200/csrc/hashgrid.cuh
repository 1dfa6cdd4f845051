// hashgrid.cuh -- per-level constants and corner loads of the multiresolution
// hash grid, shared by the forward blend and the backward kernels.
//
// Restates hashgrid.h:7-40 (fast_hash, get_grid_index) and :128-131 (per-level
// scale, resolution and table slice) of the reference's rasterizer.
#pragma once

#include "common.cuh"

namespace ns {

constexpr int kMaxLevels = 16;
constexpr int kAccStride = 32;  // floats per pixel row of the per-pixel channel arrays

// Channels (2l, 2l+1) of pixel p: float2 pair (l ^ (p & 15)) of the pixel's row,
// so that threads reading one channel of consecutive pixels hit distinct banks.
__device__ __forceinline__ float2* acc_pair(float* acc, int p, int l) {
  return reinterpret_cast<float2*>(acc + p * kAccStride + 2 * (l ^ (p & 15)));
}

__device__ __forceinline__ uint32_t lane_mask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}


// Constants of one hash level (hashgrid.h:128-131 and the dense/hash choice of
// get_grid_index, :22-40), computed with the device's exp2f as the reference does.
struct LevelConst {
  const void* base; // the level's first table row
  float scale;
  uint32_t row0;    // first table row of the level
  uint32_t mask;    // hsize-1 for a power-of-two size, ~0 otherwise
  uint32_t hsize;   // rows in the level
  uint32_t s1, s2;  // dense strides of y and z
  uint32_t dense;   // 1: dense index, 0: hashed
  uint32_t modulo;  // 1: size not a power of two, use %
};

template <typename TableT>
__device__ LevelConst make_level(const void* table, const int32_t* offsets, float S, uint32_t Hres,
                                  int align_corners, int l) {
  LevelConst lc{};
  const uint32_t hsize = (uint32_t)(offsets[l + 1] - offsets[l]);
  const float scale = exp2f(l * S) * Hres - 1.0f;
  const uint32_t res = (uint32_t)ceilf(scale) + 1;
  const uint32_t R = align_corners ? res : res + 1;
  uint32_t stride = 1, s1 = 0, s2 = 0;
  int used = 0;
  for (int d = 0; d < 3 && stride <= hsize; d++) {
    if (d == 1) s1 = stride;
    if (d == 2) s2 = stride;
    stride *= R;
    used++;
  }
  lc.scale = scale;
  lc.row0 = (uint32_t)offsets[l];
  lc.base = static_cast<const TableT*>(table) + 2 * (size_t)lc.row0;  // LD = 2 per row
  lc.hsize = hsize;
  lc.dense = (stride <= hsize && used == 3) ? 1u : 0u;
  lc.s1 = s1;
  lc.s2 = s2;
  // index % hashmap_size applies to dense levels too (with align_corners the
  // top corner of a dense level can pass R^3 - 1).
  const bool pow2 = hsize != 0 && (hsize & (hsize - 1)) == 0;
  lc.mask = pow2 ? hsize - 1 : 0xffffffffu;
  lc.modulo = pow2 ? 0u : 1u;
  return lc;
}

template <typename TableT>
struct Corner8;
template <>
struct Corner8<__half> {
  __half2 v[8];
  __device__ float2 get(int c) const { return __half22float2(v[c]); }
  __device__ void load(const void* t, int c, uint32_t row) {
    v[c] = __ldg(reinterpret_cast<const __half2*>(t) + row);
  }
};
template <>
struct Corner8<float> {
  float2 v[8];
  __device__ float2 get(int c) const { return v[c]; }
  __device__ void load(const void* t, int c, uint32_t row) {
    v[c] = __ldg(reinterpret_cast<const float2*>(t) + row);
  }
};

// Table rows (relative to the level's first row) of the 8 corners of cell g;
// corner c takes +1 along x, y, z for bits 0, 1, 2 of c (hashgrid.h:153-170).
// Dense levels index x + y s1 + z s2; hashed levels (x * 1) ^ (y * 2654435761) ^
// (z * 805459861), with the (y, z) terms formed once; both modulo the level size.
__device__ __forceinline__ void corner_rows(const LevelConst& lc, const uint32_t (&g)[3],
                                            uint32_t (&idx)[8]) {
  if (lc.dense) {
    const uint32_t base = g[0] + g[1] * lc.s1 + g[2] * lc.s2;
#pragma unroll
    for (int c = 0; c < 8; c++)
      idx[c] = base + (c & 1) + ((c >> 1) & 1 ? lc.s1 : 0u) + ((c >> 2) & 1 ? lc.s2 : 0u);
    if (lc.modulo) {
#pragma unroll
      for (int c = 0; c < 8; c++) idx[c] %= lc.hsize;
    } else {
#pragma unroll
      for (int c = 0; c < 8; c++) idx[c] &= lc.mask;
    }
    return;
  }
  const uint32_t hy0 = g[1] * 2654435761u, hy1 = (g[1] + 1) * 2654435761u;
  const uint32_t hz0 = g[2] * 805459861u, hz1 = (g[2] + 1) * 805459861u;
  uint32_t hyz[4] = {hy0 ^ hz0, hy1 ^ hz0, hy0 ^ hz1, hy1 ^ hz1};
  if (lc.modulo) {
#pragma unroll
    for (int c = 0; c < 8; c++) idx[c] = ((g[0] + (c & 1)) ^ hyz[c >> 1]) % lc.hsize;
  } else {
    // (x ^ h) & m == (x & m) ^ (h & m): six masks instead of eight.
#pragma unroll
    for (int e = 0; e < 4; e++) hyz[e] &= lc.mask;
    const uint32_t x0 = g[0] & lc.mask, x1 = (g[0] + 1) & lc.mask;
#pragma unroll
    for (int c = 0; c < 8; c++) idx[c] = ((c & 1) ? x1 : x0) ^ hyz[c >> 1];
  }
}

// Trilinear lookup of one level at a point of [0,1]^3 (hashgrid.h:140-193),
// split so that two lookups' loads are in flight together: lookup_issue()
// finds the cell and issues the 8 corner loads; lookup_finish() weights corner
// c by ((wx * wy) * wz) and accumulates corners in order c = 0..7.
template <typename TableT>
__device__ __forceinline__ void lookup_issue(const LevelConst& lc, const void* table, float4 in,
                                             float half_shift, uint32_t interp, float (&f)[3],
                                             Corner8<TableT>& cv) {
  uint32_t g[3];
  const float pin[3] = {in.x, in.y, in.z};
#pragma unroll
  for (int d = 0; d < 3; d++) {
    const float pos = pin[d] * lc.scale + half_shift;
    const float fl = floorf(pos);  // pos in (0, 2^24): the integer converts exactly
    g[d] = (uint32_t)fl;
    f[d] = pos - fl;
    if (interp == 1) f[d] = f[d] * f[d] * (3.0f - 2.0f * f[d]);
  }
  uint32_t idx[8];
  corner_rows(lc, g, idx);
#pragma unroll
  for (int c = 0; c < 8; c++) cv.load(lc.base, c, idx[c]);
}

// Corner weights ((wx * wy) * wz) and the weighted sum in packed fp32
// (__fmul2_rn / __ffma2_rn round each lane like the scalar operations).
template <typename TableT>
__device__ __forceinline__ float2 lookup_finish(const float (&f)[3], const Corner8<TableT>& cv) {
  const float2 wx = make_float2(1 - f[0], f[0]);
  const float2 wxy0 = __fmul2_rn(wx, make_float2(1 - f[1], 1 - f[1]));  // corners 0, 1
  const float2 wxy1 = __fmul2_rn(wx, make_float2(f[1], f[1]));          // corners 2, 3
  const float2 z0 = make_float2(1 - f[2], 1 - f[2]), z1 = make_float2(f[2], f[2]);
  const float2 w01 = __fmul2_rn(wxy0, z0), w23 = __fmul2_rn(wxy1, z0);
  const float2 w45 = __fmul2_rn(wxy0, z1), w67 = __fmul2_rn(wxy1, z1);
  const float w[8] = {w01.x, w01.y, w23.x, w23.y, w45.x, w45.y, w67.x, w67.y};
  float2 r = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 8; c++) r = __ffma2_rn(make_float2(w[c], w[c]), cv.get(c), r);
  return r;
}

// One 3-wide level (render modes 8-10 query one level of a table with three
// channels per row, query_feature<.., 3, 3>, hashgrid.h:53-212). Finds the cell
// of the point `in` of [0,1]^3, loads its 8 corner rows into cv and returns the
// trilinear value in r (corner c weighted ((wx * wy) * wz), accumulated in
// order c = 0..7). f: the cell fractions (smoothstep applied with interp 1),
// dv: their derivatives, idx: the corner rows relative to the level.
template <typename TableT>
__device__ __forceinline__ float ld_table(const TableT* t, size_t i);
template <>
__device__ __forceinline__ float ld_table<float>(const float* t, size_t i) {
  return __ldg(t + i);
}
template <>
__device__ __forceinline__ float ld_table<__half>(const __half* t, size_t i) {
  return __half2float(__ldg(t + i));
}

template <typename TableT>
__device__ __forceinline__ void lookup_rows3(const LevelConst& lc, const void* table, float in0, float in1,
                                             float in2, float half_shift, uint32_t interp, float (&f)[3],
                                             float (&dv)[3], uint32_t (&idx)[8], float (&cv)[8][3],
                                             float (&r)[3]) {
  uint32_t g[3];
  const float pin[3] = {in0, in1, in2};
#pragma unroll
  for (int d = 0; d < 3; d++) {
    const float pos = pin[d] * lc.scale + half_shift;
    const float fl = floorf(pos);
    g[d] = (uint32_t)fl;
    f[d] = pos - fl;
    if (interp == 1) {
      dv[d] = 6 * f[d] * (1.0f - f[d]);
      f[d] = f[d] * f[d] * (3.0f - 2.0f * f[d]);
    } else {
      dv[d] = 1.0f;
    }
  }
  corner_rows(lc, g, idx);
  const TableT* base = static_cast<const TableT*>(table) + 3 * (size_t)lc.row0;
#pragma unroll
  for (int c = 0; c < 8; c++)
#pragma unroll
    for (int ch = 0; ch < 3; ch++) cv[c][ch] = ld_table<TableT>(base, 3 * (size_t)idx[c] + ch);
  const float wx[2] = {1 - f[0], f[0]}, wy[2] = {1 - f[1], f[1]}, wz[2] = {1 - f[2], f[2]};
  r[0] = r[1] = r[2] = 0.0f;
#pragma unroll
  for (int c = 0; c < 8; c++) {
    const float w = (wx[c & 1] * wy[(c >> 1) & 1]) * wz[c >> 2];
#pragma unroll
    for (int ch = 0; ch < 3; ch++) r[ch] = fmaf(w, cv[c][ch], r[ch]);
  }
}

}  // namespace ns
