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
// (the hashed levels' worst case: no two lanes share a line). spacing > 0:
// the blend's pattern, where the 32 lanes of a warp look up the hit points of
// a 16 x 2 pixel strip on one surfel: a random point and a random plane per
// warp and lookup, lane (i, j) at point + spacing (i u + j v), with spacing
// the distance between neighbouring pixels' hit points in grid units.
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
  const uint32_t lane = threadIdx.x & 31u;
  // per-lookup seed: the thread's own, or (coherent pattern) its warp's
  const uint32_t sid = spacing > 0.f ? tid >> 5 : tid;
  const float li = (float)(lane & 15u), lj = (float)(lane >> 4);
  float2 acc = make_float2(0.f, 0.f);
  for (uint32_t j = 0; j < lookups; j += 4) {
    float f[4][3];
    Corner8<TableT> cv[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const uint32_t h = mix32(sid * 0x9e3779b9u + (j + u) * 0x85ebca6bu);
      const LevelConst& lc = lv[h % levels];
      float4 p = make_float4((mix32(h ^ 1u) >> 8) * 0x1p-24f, (mix32(h ^ 2u) >> 8) * 0x1p-24f,
                             (mix32(h ^ 3u) >> 8) * 0x1p-24f, 0.f);
      if (spacing > 0.f) {
        // a plane through the point: two directions from the hash, lanes on a 16 x 2 grid
        const float a = (mix32(h ^ 4u) >> 8) * 0x1p-24f * 6.2831853f;
        const float b = (mix32(h ^ 5u) >> 8) * 0x1p-24f * 3.1415927f;
        const float3 uu = make_float3(cosf(a), sinf(a), 0.f);
        const float3 vv = make_float3(-sinf(a) * cosf(b), cosf(a) * cosf(b), sinf(b));
        p.x = fminf(fmaxf(p.x * 0.9f + 0.05f + spacing * (li * uu.x + lj * vv.x), 0.f), 1.f);
        p.y = fminf(fmaxf(p.y * 0.9f + 0.05f + spacing * (li * uu.y + lj * vv.y), 0.f), 1.f);
        p.z = fminf(fmaxf(p.z * 0.9f + 0.05f + spacing * (li * uu.z + lj * vv.z), 0.f), 1.f);
      }
      lookup_issue<TableT>(lc, table, p, 0.5f, 0, f[u], cv[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const float2 r = lookup_finish<TableT>(f[u], cv[u]);
      acc.x += r.x;
      acc.y += r.y;
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
      lookups_per_thread == 0 || (lookups_per_thread & 3u) != 0 || !(spacing >= 0.f))
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
