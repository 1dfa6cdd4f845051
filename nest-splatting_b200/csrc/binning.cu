// binning.cu -- surfel/tile instance generation and per-tile ranges.
//
// Restates rasterizer_impl.cu:355-396 of the reference -- the prefix sum of the
// per-surfel tile counts, duplicateWithKeys (:70-111) and identifyTileRanges
// (:173-195) -- with the sort split in two (sorting is in sort.cu):
//   1. the surfels are sorted by the float bits of their view depth (stable,
//      so equal depths keep surfel-index order; surfels that touch no tile
//      sort last);
//   2. instances are generated in that depth order with key = tile id,
//      value = surfel index;
//   3. a stable sort on the tile id (13 bits at 4346 tiles: 2 digit passes).
// Within a tile this gives (depth, surfel index) order: exactly the order of
// the reference's stable sort on key = (tile << 32) | depth bits over
// instances generated in surfel-index order, for a third of the sort traffic
// (2 passes over the instances instead of 6, plus 4 over the surfels).
//
// The tile rectangle of a surfel is the one preprocess computed from its
// alpha >= 1/255 footprint, a subset of the reference's 4-sigma rectangle that
// holds every pixel the surfel can be blended into (see preprocess.cu).
#include "common.cuh"

namespace ns {
namespace {

constexpr int kScanThreads = 1024;

// Exclusive scan of nb per-CTA totals (one CTA). Writes the instance total.
__global__ void __launch_bounds__(kScanThreads)
scan_block_sums_kernel(const uint32_t* __restrict__ sums, uint32_t* __restrict__ prefix, int nb,
                       int64_t* __restrict__ total) {
  __shared__ uint32_t warp_tot[kScanThreads / 32];
  __shared__ uint64_t carry_s;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  if (t == 0) carry_s = 0;
  __syncthreads();
  for (int base = 0; base < nb; base += kScanThreads) {
    const int i = base + t;
    const uint32_t v = i < nb ? sums[i] : 0u;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[w] = x;
    __syncthreads();
    uint32_t add = 0;
    for (int k = 0; k < w; k++) add += warp_tot[k];
    const uint64_t carry = carry_s;
    if (i < nb) prefix[i] = (uint32_t)(carry + x - v + add);
    __syncthreads();
    if (t == kScanThreads - 1) carry_s = carry + x + add;
    __syncthreads();
  }
  if (t == 0) *total = (int64_t)carry_s;
}

constexpr int kDupThreads = 256;  // depth-sorted surfels per CTA
constexpr int kDupStage = 4096;   // instances staged in shared memory per CTA (48 KB)

// CTA-local inclusive scan of one value per thread; returns the CTA total.
__device__ __forceinline__ uint32_t cta_scan(uint32_t v, uint32_t& incl, uint32_t* warp_tot) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[w] = x;
  __syncthreads();
  uint32_t add = 0, tot = 0;
#pragma unroll
  for (int k = 0; k < kDupThreads / 32; k++) {
    if (k < w) add += warp_tot[k];
    tot += warp_tot[k];
  }
  incl = x + add;
  return tot;
}

// Tile counts of kDupThreads consecutive depth-sorted surfels, per CTA.
__global__ void __launch_bounds__(kDupThreads)
sorted_block_totals_kernel(int P, const uint32_t* __restrict__ order,
                           const uint32_t* __restrict__ tiles, uint32_t* __restrict__ sums) {
  __shared__ uint32_t warp_tot[kDupThreads / 32];
  const int k = blockIdx.x * kDupThreads + threadIdx.x;
  const uint32_t v = k < P ? tiles[order[k]] : 0u;
  uint32_t incl;
  const uint32_t tot = cta_scan(v, incl, warp_tot);
  if (threadIdx.x == 0) sums[blockIdx.x] = tot;
}

// duplicateWithKeys over the surfels in depth order: surfel order[k] emits
// (tile, surfel) for every tile of its rectangle, row-major. A CTA's surfels
// emit one contiguous run of instances, assembled in shared memory and written
// out with consecutive threads on consecutive instances. Instances past
// kDupStage (surfels with very large footprints) are written directly.
__global__ void __launch_bounds__(kDupThreads)
duplicate_keys_kernel(int P, const uint32_t* __restrict__ order, const BinInfo* __restrict__ bin,
                      const uint32_t* __restrict__ tiles, const uint32_t* __restrict__ block_prefix,
                      int gx, uint32_t* __restrict__ keys, uint32_t* __restrict__ vals,
                      int64_t capacity, uint32_t* __restrict__ err, int64_t* __restrict__ count) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint32_t* sk = reinterpret_cast<uint32_t*>(smem_raw);
  uint32_t* sv = reinterpret_cast<uint32_t*>(sk + kDupStage);
  __shared__ uint32_t warp_tot[kDupThreads / 32];
  const int k = blockIdx.x * kDupThreads + threadIdx.x;
  const uint32_t i = k < P ? order[k] : 0u;
  const uint32_t n = k < P ? tiles[i] : 0u;
  uint32_t incl;
  const int64_t total = (int64_t)cta_scan(n, incl, warp_tot);
  const int64_t base = (int64_t)block_prefix[blockIdx.x];
  if (base + total > capacity) {  // uniform over the CTA
    // Overflow: flag it and zero the instance count, so that the sort and the
    // ranges that read the count on the device (device-count mode) see no
    // instances instead of the unwritten part of the buffers.
    if (threadIdx.x == 0) {
      set_error(err, kErrCapacity);
      *count = 0;
    }
    return;
  }
  if (n) {
    const BinInfo b = bin[i];
    int64_t off = (int64_t)(incl - n);
    for (int y = b.y0; y < b.y1; y++) {
      for (int x = b.x0; x < b.x1; x++) {
        const uint32_t key = (uint32_t)(y * gx + x);
        if (off < kDupStage) {
          sk[off] = key;
          sv[off] = i;
        } else {
          keys[base + off] = key;
          vals[base + off] = i;
        }
        off++;
      }
    }
  }
  __syncthreads();
  const int staged = (int)min64(total, kDupStage);
  for (int j = threadIdx.x; j < staged; j += kDupThreads) {
    keys[base + j] = sk[j];
    vals[base + j] = sv[j];
  }
}

__global__ void identify_ranges_kernel(const uint32_t* __restrict__ keys,
                                       const int64_t* __restrict__ count_dev, int64_t count_host,
                                       int64_t capacity, uint2* __restrict__ ranges) {
  int64_t n = count_dev ? min(*count_dev, capacity) : count_host;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t cur = (uint32_t)keys[idx];
    if (idx == 0) {
      ranges[cur].x = 0;
    } else {
      const uint32_t prev = (uint32_t)keys[idx - 1];
      if (cur != prev) {
        ranges[prev].y = (uint32_t)idx;
        ranges[cur].x = (uint32_t)idx;
      }
    }
    if (idx == n - 1) ranges[cur].y = (uint32_t)n;
  }
}

// Launch order of the per-tile kernels: tiles by descending instance count
// (the blend's and the backward's work per tile grows with it), so the
// heaviest tiles start first and the grid's tail is made of light ones. At
// config 2 half the tiles are empty and the busiest hold ~7,600 instances; in
// row-major order the last heavy tiles start late and stretch the tail (a
// list-scheduling model of the 296 resident CTAs puts it at 8% of the launch).
// One CTA: a counting sort on kOrderBuckets descending buckets of the count
// (log-spaced, so the order is exact enough for scheduling); the order inside
// a bucket follows atomics and does not affect any output (tiles are
// independent).
constexpr int kOrderThreads = 1024;
constexpr int kOrderBuckets = 64;

__device__ __forceinline__ int order_bucket(uint32_t n) {
  // 0 for the heaviest: 4 buckets per power of two from 2^15 down, last = empty
  if (n == 0) return kOrderBuckets - 1;
  const int lz = __clz(n);                                 // 31 - floor(log2 n)
  const uint32_t rest = lz == 31 ? 0u : n << (lz + 1);      // bits below the leading one
  const int frac = (int)(rest >> 30);                       // their top two
  const int b = (lz - 16) * 4 + (3 - frac);       // n >= 2^15 -> bucket <= 0
  return b < 0 ? 0 : (b > kOrderBuckets - 2 ? kOrderBuckets - 2 : b);
}

__global__ void __launch_bounds__(kOrderThreads) tile_order_kernel(const uint2* __restrict__ ranges, int tiles,
                                                                   uint32_t* __restrict__ order) {
  __shared__ uint32_t cnt[kOrderBuckets];
  if (threadIdx.x < kOrderBuckets) cnt[threadIdx.x] = 0;
  __syncthreads();
  for (int t = threadIdx.x; t < tiles; t += kOrderThreads) {
    const uint2 r = ranges[t];
    atomicAdd(&cnt[order_bucket(r.y - r.x)], 1u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t run = 0;
    for (int b = 0; b < kOrderBuckets; b++) {
      const uint32_t c = cnt[b];
      cnt[b] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < tiles; t += kOrderThreads) {
    const uint2 r = ranges[t];
    order[atomicAdd(&cnt[order_bucket(r.y - r.x)], 1u)] = (uint32_t)t;
  }
}

}  // namespace

int tile_order_launch(const uint2* ranges, int tiles, uint32_t* order, cudaStream_t stream) {
  if (tiles <= 0) return NS_OK;
  tile_order_kernel<<<1, kOrderThreads, 0, stream>>>(ranges, tiles, order);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int scan_block_sums_launch(const uint32_t* sums, uint32_t* prefix, int nb, int64_t* total,
                           cudaStream_t stream) {
  scan_block_sums_kernel<<<1, kScanThreads, 0, stream>>>(sums, prefix, nb, total);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int duplicate_keys_launch(int P, const uint32_t* order, const BinInfo* bin, const uint32_t* tiles,
                          uint32_t* sorted_sums, uint32_t* sorted_prefix, int64_t* total, int gx,
                          uint32_t* keys, uint32_t* vals, int64_t capacity, uint32_t* err,
                          cudaStream_t stream) {
  if (P <= 0) return NS_OK;
  const int nb = div_up(P, kDupThreads);
  sorted_block_totals_kernel<<<nb, kDupThreads, 0, stream>>>(P, order, tiles, sorted_sums);
  NS_LAUNCH_CHECK();
  int rc = scan_block_sums_launch(sorted_sums, sorted_prefix, nb, total, stream);
  if (rc) return rc;
  const int smem = kDupStage * (int)(2 * sizeof(uint32_t));
  NS_CUDA_TRY(cudaFuncSetAttribute(duplicate_keys_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  duplicate_keys_kernel<<<nb, kDupThreads, smem, stream>>>(P, order, bin, tiles, sorted_prefix, gx,
                                                           keys, vals, capacity, err, total);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int identify_ranges_launch(const uint32_t* keys, const int64_t* count_dev, int64_t count_host,
                           int64_t capacity, uint2* ranges, int tiles, int sms,
                           cudaStream_t stream) {
  NS_CUDA_TRY(cudaMemsetAsync(ranges, 0, sizeof(uint2) * (size_t)tiles, stream));
  const int64_t n = count_dev ? capacity : count_host;
  if (n <= 0) return NS_OK;
  const int blocks = (int)min64(div_up64(n, 256), (int64_t)sms * 8);
  identify_ranges_kernel<<<blocks, 256, 0, stream>>>(keys, count_dev, count_host, capacity, ranges);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
