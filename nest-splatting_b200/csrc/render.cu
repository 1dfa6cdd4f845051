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
// One CTA of 256 threads per 16x16 tile, one thread per pixel. Each round a
// batch of up to 256 surfel records (128-byte records written by preprocess)
// is gathered into shared memory, double-buffered with cp.async so the next
// batch streams in while the current one is blended. The hash table is read
// as fp16 (or fp32) pairs through the read-only path; it is small enough
// (32 MB at 16 levels x 2^19 x 2 fp16) to stay resident in the 126 MB L2.
// Per-level parameters (scale, resolution, dense/hash, mask) are computed once
// per CTA, with the device's own exp2f, exactly as the reference does per
// sample.
#include "kernels.cuh"

namespace ns {

constexpr int kMaxLevels = 16;

struct LevelParams {
  float scale[kMaxLevels];
  uint32_t offset[kMaxLevels];  // row offset of the level in the table
  uint32_t hsize[kMaxLevels];
  uint32_t mask[kMaxLevels];    // hsize-1 when hsize is a power of two, else 0
  uint32_t stride1[kMaxLevels]; // dense strides (0 in stride1 marks a hashed level)
  uint32_t stride2[kMaxLevels];
};


namespace {

constexpr int kRenderThreads = kTilePixels;

template <typename TableT, int LD>
struct TableLoad;
template <>
struct TableLoad<__half, 2> {
  __device__ static float2 get(const void* t, uint32_t row) {
    const __half2 h = __ldg(reinterpret_cast<const __half2*>(t) + row);
    return __half22float2(h);
  }
};
template <>
struct TableLoad<float, 2> {
  __device__ static float2 get(const void* t, uint32_t row) {
    return __ldg(reinterpret_cast<const float2*>(t) + row);
  }
};

// Level setup (hashgrid.h:128-131 and the dense/hash choice of :22-40).
__device__ void setup_levels(const RenderParams& p, LevelParams& lp) {
  const int lv = threadIdx.x;
  if (lv < (int)p.L && lv < kMaxLevels) {
    const uint32_t hsize = (uint32_t)(p.offsets[lv + 1] - p.offsets[lv]);
    const float scale = exp2f(lv * p.S) * p.Hres - 1.0f;
    const uint32_t res = (uint32_t)ceilf(scale) + 1;
    const uint32_t R = p.align_corners ? res : res + 1;
    uint32_t stride = 1, s1 = 0, s2 = 0;
    int used = 0;
    for (int d = 0; d < 3 && stride <= hsize; d++) {
      if (d == 1) s1 = stride;
      if (d == 2) s2 = stride;
      stride *= R;
      used++;
    }
    lp.scale[lv] = scale;
    lp.offset[lv] = (uint32_t)p.offsets[lv];
    lp.hsize[lv] = hsize;
    lp.mask[lv] = (hsize & (hsize - 1)) == 0 ? hsize - 1 : 0;
    const bool dense = stride <= hsize && used == 3;
    lp.stride1[lv] = dense ? s1 : 0;
    lp.stride2[lv] = dense ? s2 : 0;
  }
}

// Trilinear lookup of one level; returns the LD=2 features (hashgrid.h:140-193).
template <typename TableT>
__device__ __forceinline__ float2 level_lookup(const LevelParams& lp, int lv, const float in[3],
                                               const void* table, bool align_corners,
                                               uint32_t interp) {
  const float scale = lp.scale[lv];
  float pos[3];
  uint32_t g[3];
#pragma unroll
  for (int d = 0; d < 3; d++) {
    pos[d] = in[d] * scale + (align_corners ? 0.0f : 0.5f);
    g[d] = (uint32_t)floorf(pos[d]);
    pos[d] -= (float)g[d];
    if (interp == 1) pos[d] = pos[d] * pos[d] * (3.0f - 2.0f * pos[d]);
  }
  const uint32_t hsize = lp.hsize[lv], mask = lp.mask[lv];
  const uint32_t s1 = lp.stride1[lv], s2 = lp.stride2[lv];
  const uint32_t base_row = lp.offset[lv];
  float rx = 0.f, ry = 0.f;
#pragma unroll
  for (uint32_t c = 0; c < 8; c++) {
    const uint32_t bx = c & 1u, by = (c >> 1) & 1u, bz = (c >> 2) & 1u;
    const float w = ((bx ? pos[0] : 1 - pos[0]) * (by ? pos[1] : 1 - pos[1])) *
                    (bz ? pos[2] : 1 - pos[2]);
    const uint32_t x = g[0] + bx, y = g[1] + by, z = g[2] + bz;
    uint32_t idx;
    if (s1 != 0) idx = x + y * s1 + z * s2;
    else idx = x ^ (y * 2654435761u) ^ (z * 805459861u);
    idx = mask ? (idx & mask) : (idx % hsize);
    const float2 v = TableLoad<TableT, 2>::get(table, base_row + idx);
    rx += w * v.x;
    ry += w * v.y;
  }
  return make_float2(rx, ry);
}

template <typename TableT, int C>
__global__ void __launch_bounds__(kRenderThreads, 2)
render_kernel(const RenderParams p) {
  constexpr int LD = 2;
  constexpr int kLevelsMax = C / LD;
  static_assert(kLevelsMax <= kMaxLevels, "at most 16 levels");
  extern __shared__ float4 s_dyn[];
  float4 (*s_rec)[kRenderThreads][kRecordFloat4] =
      reinterpret_cast<float4 (*)[kRenderThreads][kRecordFloat4]>(s_dyn);
  __shared__ LevelParams lp;

  setup_levels(p, lp);

  const int gx = div_up(p.W, kTile);
  const int tile = blockIdx.x;
  const int tx = tile % gx, ty = tile / gx;
  const int t = threadIdx.x;
  const uint32_t px = tx * kTile + (t & (kTile - 1));
  const uint32_t py = ty * kTile + (t >> 4);
  const bool inside = px < (uint32_t)p.W && py < (uint32_t)p.H;
  const uint32_t pid = py * p.W + px;
  const float pxf = (float)px, pyf = (float)py;

  const uint2 range = p.ranges[tile];
  const int total = (int)(range.y - range.x);
  const int rounds = div_up(total, kRenderThreads);

  const float vmin = p.gridrange[0], vmax = p.gridrange[1];
  const uint32_t L = p.L;

  float T = 1.0f;
  uint32_t contributor = 0, last_contributor = 0, render_number = 0;
  float Cacc[C];
#pragma unroll
  for (int c = 0; c < C; c++) Cacc[c] = 0.f;
  float N0 = 0, N1 = 0, N2 = 0, D = 0, M1 = 0, M2 = 0, distortion = 0, median_depth = 0;
  float median_contributor = -1;
  float pos0 = 0, pos1 = 0, pos2 = 0, vis0 = 0, vis1 = 0, vis2 = 0;
  bool done = !inside;

  auto fetch = [&](int round, int buf) {
    const int k = round * kRenderThreads + t;
    if (k < total) {
      const uint32_t id = p.point_list[range.x + k];
      const float4* src = reinterpret_cast<const float4*>(p.records + id);
#pragma unroll
      for (int q = 0; q < kRecordFloat4; q++) {
        const unsigned dst = (unsigned)__cvta_generic_to_shared(&s_rec[buf][t][q]);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src + q));
      }
    }
    asm volatile("cp.async.commit_group;");
  };

  if (rounds > 0) fetch(0, 0);
  for (int r = 0; r < rounds; r++) {
    const int buf = r & 1;
    asm volatile("cp.async.wait_group 0;");
    // End when the whole tile is done (forward.cu:791-796). The barrier also
    // guarantees every thread has finished reading buffer buf^1 before the
    // next batch is copied into it.
    const int num_done = __syncthreads_count(done);
    if (num_done == kRenderThreads) break;
    if (r + 1 < rounds) fetch(r + 1, buf ^ 1);

    const int todo = min(kRenderThreads, total - r * kRenderThreads);
    for (int j = 0; !done && j < todo; j++) {
      contributor++;
      const float4 q0 = s_rec[buf][j][0], q1 = s_rec[buf][j][1], q2 = s_rec[buf][j][2];
      const float3 Tu = f3(q0.x, q0.y, q0.z), Tv = f3(q0.w, q1.x, q1.y), Tw = f3(q1.z, q1.w, q2.x);
      const float3 kk = pxf * Tw - Tu;
      const float3 ll = pyf * Tw - Tv;
      const float3 pp = cross3(kk, ll);
      if (pp.z == 0.0f) continue;
      const float sx = pp.x / pp.z, sy = pp.y / pp.z;
      const float rho3d = sx * sx + sy * sy;
      const float dx = q2.y - pxf, dy = q2.z - pyf;
      const float rho2d = kFilterInvSquare * (dx * dx + dy * dy);
      const float rho = fminf(rho3d, rho2d);
      const bool surf = rho3d <= rho2d;
      const float depth = surf ? (sx * Tw.x + sy * Tw.y) + Tw.z : Tw.z;
      if (depth < kNear) continue;
      const float power = -0.5f * rho;
      if (power > 0.0f) continue;
      float G = expf(power);
      if (p.beta > 0.0f) G = (float)((1.0 + (double)p.beta) * G / (1.0 + (double)p.beta * G));
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
      const float4 q3 = s_rec[buf][j][3];
      N0 += q3.x * w;
      N1 += q3.y * w;
      N2 += q3.z * w;

      const float4 q4 = s_rec[buf][j][4], q5 = s_rec[buf][j][5], q6 = s_rec[buf][j][6];
      float3 xyz;
      if (surf) {
        xyz = f3(sx * q4.x + sy * q4.w + q5.z, sx * q4.y + sy * q5.x + q5.w,
                 sx * q4.z + sy * q5.y + q6.x);
      } else {
        xyz = f3(q5.z, q5.w, q6.x);
      }
      pos0 += w * xyz.x;
      pos1 += w * xyz.y;
      pos2 += w * xyz.z;

      const uint32_t apl = __float_as_uint(q3.w);
      // query_feature (hashgrid.h:53-212): box map to [0,1]^3 or contraction.
      float in[3];
      bool oob = false;
      if (!p.contract) {
        const float inv = 1.0f / (vmax - vmin);
        in[0] = (xyz.x - vmin) * inv;
        in[1] = (xyz.y - vmin) * inv;
        in[2] = (xyz.z - vmin) * inv;
        oob = in[0] < 0 || in[0] > 1 || in[1] < 0 || in[1] > 1 || in[2] < 0 || in[2] > 1;
      } else {
        const float vmid = (vmax + vmin) * 0.5f;
        const float inv = 1.0f / ((vmax - vmin) * 0.5f);
        in[0] = (xyz.x - vmid) * inv;
        in[1] = (xyz.y - vmid) * inv;
        in[2] = (xyz.z - vmid) * inv;
        const float nrm = sqrtf(in[0] * in[0] + in[1] * in[1] + in[2] * in[2]);
        const float inv_n = 1.0f / nrm;
        const float st = (nrm <= 1.0f) ? 1.0f : (2.0f - inv_n) * inv_n;
#pragma unroll
        for (int d = 0; d < 3; d++) in[d] = (st * in[d] + 2.0f) * 0.25f;
      }
      if (!oob) {
        const uint32_t max_level = min(apl, L);
#pragma unroll
        for (int lv = 0; lv < kLevelsMax; lv++) {
          if ((uint32_t)lv < max_level) {
            const float2 f = level_lookup<TableT>(lp, lv, in, p.table, p.align_corners != 0,
                                                  p.interp);
            Cacc[2 * lv] += f.x * w;
            Cacc[2 * lv + 1] += f.y * w;
          }
        }
      }
      float ac0, ac1;
      if (apl <= 4) {
        ac0 = (float)((apl - 2) * 0.5);
        ac1 = 1.0f;
      } else {
        ac0 = 1.0f;
        ac1 = (float)(1.0 - (apl - 4) * 0.5);
      }
      vis0 += ac0 * w;
      vis1 += ac1 * w;
      if (p.record_transmittance) {
        const uint32_t id = p.point_list[range.x + r * kRenderThreads + j];
        atomicAdd(p.cover_pixels + id, 1.0f);
        atomicAdd(p.trans_avg + id, T);
      }
      T = test_T;
      last_contributor = contributor;
    }
  }
  asm volatile("cp.async.wait_group 0;");

  if (inside) {
    const size_t HW = (size_t)p.H * p.W;
    p.final_T[pid] = T;
    p.final_T[pid + HW] = M1;
    p.final_T[pid + 2 * HW] = M2;
    p.n_contrib[pid] = last_contributor;
    p.n_contrib[pid + HW] = (uint32_t)median_contributor;  // -1 saturates to 0
#pragma unroll
    for (int c = 0; c < C; c++) p.out_color[c * HW + pid] = Cacc[c];
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
    o[13 * HW] = vis2;
  }
}

constexpr size_t kRenderSmem = sizeof(float4) * 2 * kRenderThreads * kRecordFloat4;

template <typename TableT, int C>
int launch_render(const RenderParams& p, int tiles, cudaStream_t stream) {
  NS_CUDA_TRY(cudaFuncSetAttribute(render_kernel<TableT, C>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRenderSmem));
  render_kernel<TableT, C><<<tiles, kRenderThreads, kRenderSmem, stream>>>(p);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace

// Supported: LD == 2 with C in {4, 8, 16, 24, 32} (C = L*LD channels), fp16 or
// fp32 table. Other shapes report NS_ERR_UNSUPPORTED (the reference prints and
// renders nothing for shapes it was not built for).
int render_launch(const RenderParams& p, int fp16, cudaStream_t stream) {
  if (p.LD != 2) return NS_ERR_UNSUPPORTED;
  if (p.L > (uint32_t)(p.C / p.LD) || p.L > (uint32_t)kMaxLevels) return NS_ERR_UNSUPPORTED;
  const int tiles = div_up(p.W, kTile) * div_up(p.H, kTile);
  if (tiles == 0) return NS_OK;
#define NS_RENDER_CASE(CC)                                                  \
  case CC:                                                                  \
    return fp16 ? launch_render<__half, CC>(p, tiles, stream)               \
                : launch_render<float, CC>(p, tiles, stream);
  switch (p.C) {
    NS_RENDER_CASE(4)
    NS_RENDER_CASE(8)
    NS_RENDER_CASE(16)
    NS_RENDER_CASE(24)
    NS_RENDER_CASE(32)
    default:
      return NS_ERR_UNSUPPORTED;
  }
#undef NS_RENDER_CASE
}

}  // namespace ns
