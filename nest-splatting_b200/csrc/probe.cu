// probe.cu -- the gather roofline of the blend kernel: how fast this GPU can
// serve hash-grid lookups from an L2-resident table when nothing else runs.
//
// The blend kernel's hash lookups are 8 scattered 4-byte loads each (the
// corners of one cell of one level; the two x-neighbours of a corner pair
// usually share a 128-byte line, the four (y, z) pairs land on unrelated
// lines at the hashed levels). Neither the HBM copy peak nor a streaming L2
// bandwidth is a fair ceiling for that access pattern, so bench.py measures
// one here: every thread performs lookups at pseudo-random points of the
// table's hashed levels with the blend's own level constants, corner
// indexing and loads (hashgrid.cuh), four lookups in flight, at full
// occupancy, and sums the corners so that no load is dead. The figure is
// corner bytes per second (lookups x 8 x the table's row size).
//
// Two point patterns. spacing = 0: every lane an independent random point
// and level (no two lanes share a line at the hashed levels). spacing > 0:
// the blend's pattern and order: a warp's lanes hold 8 samples each, the hit
// points of a 16 x 2 pixel strip (spacing = the distance between neighbouring
// pixels' hit points, in grid units) on 8 surfels stacked along the view
// direction (4 spacings apart), looked up level by level in an outer loop
// (two samples x two levels in flight, as the blend's phase B), then the next
// strip. lookups_per_thread must then be a multiple of 8 x levels.
//
// It is a measurement tool, not part of the render path.
#include "hashgrid.cuh"
#include "kernels.cuh"

namespace ns {
namespace {

constexpr int kProbeThreads = 256;

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

template <typename TableT>
__global__ void __launch_bounds__(kProbeThreads) gather_probe_kernel(const void* __restrict__ table,
                                                                    const int32_t* __restrict__ offsets,
                                                                    uint32_t level0, uint32_t levels, float S,
                                                                    uint32_t H, uint32_t lookups, float spacing,
                                                                    float* __restrict__ sink) {
  __shared__ LevelConst lv[kMaxLevels];
  if (threadIdx.x < levels) lv[threadIdx.x] = make_level<TableT>(table, offsets, S, H, 0, level0 + threadIdx.x);
  __syncthreads();
  const uint32_t tid = blockIdx.x * kProbeThreads + threadIdx.x;
  float2 acc = make_float2(0.f, 0.f);
  if (spacing <= 0.f) {
    // every lane its own random point and level
    for (uint32_t j = 0; j < lookups; j += 4) {
      float f[4][3];
      Corner8<TableT> cv[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const uint32_t h = mix32(tid * 0x9e3779b9u + (j + u) * 0x85ebca6bu);
        const float4 p = make_float4((mix32(h ^ 1u) >> 8) * 0x1p-24f, (mix32(h ^ 2u) >> 8) * 0x1p-24f,
                                     (mix32(h ^ 3u) >> 8) * 0x1p-24f, 0.f);
        lookup_issue<TableT>(lv[h % levels], table, p, 0.5f, 0, f[u], cv[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float2 r = lookup_finish<TableT>(f[u], cv[u]);
        acc.x += r.x;
        acc.y += r.y;
      }
    }
  } else {
    // The blend's order: a warp holds kQ samples per lane (lane (i, j) of a
    // 16 x 2 pixel strip on a surfel plane, sample k one surfel further along
    // the view direction), and runs the levels in an outer loop over all of
    // them, two samples x two levels in flight; then a new strip.
    constexpr int kQ = 8;
    const uint32_t lane = threadIdx.x & 31u, wid = tid >> 5;
    const float li = (float)(lane & 15u), lj = (float)(lane >> 4);
    const uint32_t per_drain = kQ * levels;
    for (uint32_t d = 0; d * per_drain < lookups; d++) {
      const uint32_t h = mix32(wid * 0x9e3779b9u + d * 0x85ebca6bu);
      const float a = (mix32(h ^ 4u) >> 8) * 0x1p-24f * 6.2831853f;
      const float b = (mix32(h ^ 5u) >> 8) * 0x1p-24f * 3.1415927f;
      const float3 uu = make_float3(cosf(a), sinf(a), 0.f);
      const float3 vv = make_float3(-sinf(a) * cosf(b), cosf(a) * cosf(b), sinf(b));
      const float3 ww = make_float3(uu.y * vv.z - uu.z * vv.y, uu.z * vv.x - uu.x * vv.z, uu.x * vv.y - uu.y * vv.x);
      const float3 p0 = make_float3((mix32(h ^ 1u) >> 8) * 0x1p-24f * 0.8f + 0.1f,
                                    (mix32(h ^ 2u) >> 8) * 0x1p-24f * 0.8f + 0.1f,
                                    (mix32(h ^ 3u) >> 8) * 0x1p-24f * 0.8f + 0.1f);
      const float3 pl = make_float3(p0.x + spacing * (li * uu.x + lj * vv.x), p0.y + spacing * (li * uu.y + lj * vv.y),
                                    p0.z + spacing * (li * uu.z + lj * vv.z));
      const float dz = 4.0f * spacing;  // surfel spacing along the ray
      for (uint32_t l = 0; l < levels; l += 2) {
        const LevelConst& l0 = lv[l];
        const LevelConst& l1 = lv[l + 1 < levels ? l + 1 : l];
        for (int k = 0; k < kQ; k += 2) {
          float f[4][3];
          Corner8<TableT> cv[4];
#pragma unroll
          for (int u = 0; u < 2; u++) {
            const float t = (float)(k + u) * dz;
            const float4 p = make_float4(pl.x + t * ww.x, pl.y + t * ww.y, pl.z + t * ww.z, 0.f);
            lookup_issue<TableT>(l0, table, p, 0.5f, 0, f[2 * u], cv[2 * u]);
            lookup_issue<TableT>(l1, table, p, 0.5f, 0, f[2 * u + 1], cv[2 * u + 1]);
          }
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const float2 r = lookup_finish<TableT>(f[u], cv[u]);
            acc.x += r.x;
            acc.y += r.y;
          }
        }
      }
    }
  }
  sink[tid] = acc.x + acc.y;
}

}  // namespace
}  // namespace ns

extern "C" int ns_gather_probe(const void* table, int32_t table_fp16, const int32_t* offsets, uint32_t level0,
                               uint32_t levels, float S, uint32_t H, uint32_t lookups_per_thread, float spacing,
                               int32_t blocks, float* sink, void* stream_) {
  using namespace ns;
  if (!table || !offsets || !sink || levels == 0 || levels > (uint32_t)kMaxLevels || blocks <= 0 ||
      lookups_per_thread == 0 || (lookups_per_thread & 3u) != 0 || !(spacing >= 0.f) ||
      (spacing > 0.f && lookups_per_thread % (8u * levels) != 0))
    return NS_ERR_INVALID;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (table_fp16)
    gather_probe_kernel<__half><<<blocks, kProbeThreads, 0, stream>>>(table, offsets, level0, levels, S, H,
                                                                      lookups_per_thread, spacing, sink);
  else
    gather_probe_kernel<float><<<blocks, kProbeThreads, 0, stream>>>(table, offsets, level0, levels, S, H,
                                                                     lookups_per_thread, spacing, sink);
  NS_LAUNCH_CHECK();
  return NS_OK;
}
