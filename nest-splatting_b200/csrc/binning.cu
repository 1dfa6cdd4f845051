// binning.cu -- surfel/tile instance generation and per-tile ranges.
//
// Restates rasterizer_impl.cu:355-396 of the reference: the prefix sum of the
// per-surfel tile counts (here a scan of the per-CTA totals that preprocess
// already produced), duplicateWithKeys (:70-111) emitting
// key = (tile << 32) | float bits of view depth, value = surfel index, and
// identifyTileRanges (:173-195). Sorting is in sort.cu.
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

constexpr int kDupThreads = 256;  // = the preprocess CTA size (one CTA's surfels per CTA here)
constexpr int kDupStage = 4096;   // instances staged in shared memory per CTA (48 KB)

// A CTA's surfels emit one contiguous run of instances (their offsets come from
// the preprocess CTA's scan), so the run is assembled in shared memory and
// written out with consecutive threads on consecutive instances: per-surfel
// writes of a few scattered 12-byte records kept the store queue full.
// Instances past kDupStage (surfels with very large footprints) are written
// directly.
__global__ void __launch_bounds__(kDupThreads)
duplicate_keys_kernel(int P, const BinInfo* __restrict__ bin,
                      const uint32_t* __restrict__ excl_local,
                      const uint32_t* __restrict__ block_prefix,
                      const uint32_t* __restrict__ block_sums, int gx,
                      uint64_t* __restrict__ keys, uint32_t* __restrict__ vals, int64_t capacity,
                      uint32_t* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* sk = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* sv = reinterpret_cast<uint32_t*>(sk + kDupStage);
  const int cta = blockIdx.x;
  const int i = cta * kDupThreads + threadIdx.x;
  const int64_t base = (int64_t)block_prefix[cta];
  const int64_t total = (int64_t)block_sums[cta];
  if (base + total > capacity) {  // uniform over the CTA
    if (threadIdx.x == 0) set_error(err, kErrCapacity);
    return;
  }
  if (i < P) {
    const BinInfo b = bin[i];
    const int x0 = b.x0, y0 = b.y0, x1 = b.x1, y1 = b.y1;
    if (x1 > x0 && y1 > y0) {
      int64_t off = (int64_t)excl_local[i];
      const uint64_t dbits = (uint64_t)__float_as_uint(b.depth);
      for (int y = y0; y < y1; y++) {
        for (int x = x0; x < x1; x++) {
          const uint64_t key = ((uint64_t)(uint32_t)(y * gx + x) << 32) | dbits;
          if (off < kDupStage) {
            sk[off] = key;
            sv[off] = (uint32_t)i;
          } else {
            keys[base + off] = key;
            vals[base + off] = (uint32_t)i;
          }
          off++;
        }
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

__global__ void identify_ranges_kernel(const uint64_t* __restrict__ keys,
                                       const int64_t* __restrict__ count_dev, int64_t count_host,
                                       int64_t capacity, uint2* __restrict__ ranges) {
  int64_t n = count_dev ? min(*count_dev, capacity) : count_host;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t cur = (uint32_t)(keys[idx] >> 32);
    if (idx == 0) {
      ranges[cur].x = 0;
    } else {
      const uint32_t prev = (uint32_t)(keys[idx - 1] >> 32);
      if (cur != prev) {
        ranges[prev].y = (uint32_t)idx;
        ranges[cur].x = (uint32_t)idx;
      }
    }
    if (idx == n - 1) ranges[cur].y = (uint32_t)n;
  }
}

}  // namespace

int scan_block_sums_launch(const uint32_t* sums, uint32_t* prefix, int nb, int64_t* total,
                           cudaStream_t stream) {
  scan_block_sums_kernel<<<1, kScanThreads, 0, stream>>>(sums, prefix, nb, total);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int duplicate_keys_launch(int P, int block_size, const BinInfo* bin, const uint32_t* excl_local,
                          const uint32_t* block_prefix, const uint32_t* block_sums, int gx,
                          int gy, uint64_t* keys, uint32_t* vals, int64_t capacity, uint32_t* err,
                          cudaStream_t stream) {
  if (P <= 0) return NS_OK;
  if (block_size != kDupThreads) return NS_ERR_UNSUPPORTED;  // offsets are per preprocess CTA
  (void)gy;
  const int smem = kDupStage * (int)(sizeof(uint64_t) + sizeof(uint32_t));
  NS_CUDA_TRY(cudaFuncSetAttribute(duplicate_keys_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  duplicate_keys_kernel<<<div_up(P, kDupThreads), kDupThreads, smem, stream>>>(
      P, bin, excl_local, block_prefix, block_sums, gx, keys, vals, capacity, err);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int identify_ranges_launch(const uint64_t* keys, const int64_t* count_dev, int64_t count_host,
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
