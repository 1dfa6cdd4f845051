// sort.cu -- in-house onesweep LSD radix sort of (u64 key, u32 value) pairs.
//
// Replaces cub::DeviceRadixSort::SortPairs as the reference calls it
// (cuda_rasterizer/rasterizer_impl.cu:381-386): a stable sort on bits
// [0, end_bit) of a key | tile id | float bits of view depth |.
//
// Structure (single-pass "onesweep" digit passes with decoupled look-back):
//   1. upfront histogram: one read of the keys builds the 256-bin histogram
//      of every 8-bit digit position at once;
//   2. bucket bases: exclusive scan of each histogram;
//   3. one kernel per digit pass. A CTA takes the next 4096-key tile from an
//      atomic counter (so tiles start in order and every look-back target is
//      already resident), ranks its keys stably with warp match-any, publishes
//      its per-digit counts, resolves its global per-digit offsets by looking
//      back over earlier tiles' published words, and scatters through shared
//      memory so global writes come out in digit runs.
// Stability: within a tile keys are ranked in (warp, item, lane) order, which
// is the input order of the warp-striped layout; tiles are prefixed in order.
// Every wait on another CTA's word is bounded (kSpinLimit); running out sets an
// error bit and the pass continues, so a fault elsewhere cannot hang the GPU.
#include "common.cuh"

namespace ns {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 16;
constexpr int kSortTile = kSortThreads * kSortItems;  // 4096 keys per CTA
constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;
constexpr int kMaxPasses = 8;
constexpr uint32_t kFlagAggregate = 1u << 30;
constexpr uint32_t kFlagPrefix = 2u << 30;
constexpr uint32_t kFlagMask = 3u << 30;
constexpr uint32_t kValueMask = ~kFlagMask;

// Layout of the temp buffer (all u32).
struct SortTemp {
  uint32_t* hist;      // [kMaxPasses][256]
  uint32_t* tile_ctr;  // [kMaxPasses]
  uint32_t* err;       // [1]
  uint32_t* status;    // [kMaxPasses][tiles][256]
};

__host__ __device__ inline int64_t sort_tiles(int64_t n) { return div_up64(n, kSortTile); }

__host__ inline size_t sort_temp_words(int64_t n) {
  return (size_t)kMaxPasses * kRadix + kMaxPasses + 1 + 1 /*pad*/ +
         (size_t)kMaxPasses * (size_t)max64(1, sort_tiles(n)) * kRadix;
}

__host__ inline SortTemp carve(void* temp, int64_t n) {
  SortTemp t;
  uint32_t* p = reinterpret_cast<uint32_t*>(temp);
  t.hist = p;
  t.tile_ctr = p + kMaxPasses * kRadix;
  t.err = t.tile_ctr + kMaxPasses;
  t.status = t.err + 2;
  (void)n;
  return t;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ uint32_t load_volatile(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Histogram of every digit position in one pass over the keys.
__global__ void __launch_bounds__(256) upfront_histogram_kernel(const uint64_t* __restrict__ keys,
                                                                int64_t n, int passes,
                                                                uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[kMaxPasses][kRadix];
  for (int i = threadIdx.x; i < kMaxPasses * kRadix; i += blockDim.x) (&h[0][0])[i] = 0;
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t k = keys[i];
    for (int p = 0; p < passes; p++) atomicAdd(&h[p][(k >> (p * kRadixBits)) & (kRadix - 1)], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRadix; i += blockDim.x) {
    uint32_t v = (&h[0][0])[i];
    if (v) atomicAdd(hist + i, v);
  }
}

// In place: hist[p][d] -> exclusive prefix over d (the bucket base of digit d).
__global__ void bucket_scan_kernel(uint32_t* __restrict__ hist, int passes) {
  __shared__ uint32_t warp_tot[kRadix / 32];
  const int p = blockIdx.x;
  if (p >= passes) return;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  uint32_t v = hist[p * kRadix + t];
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[w] = x;
  __syncthreads();
  uint32_t add = 0;
  for (int i = 0; i < w; i++) add += warp_tot[i];
  hist[p * kRadix + t] = x - v + add;
}

struct PassSmem {
  uint32_t warp_hist[kSortWarps][kRadix];
  uint32_t digit_excl[kRadix];
  uint32_t global_base[kRadix];
  uint32_t warp_tot[kSortWarps];
  uint32_t tile;
  uint64_t keys[kSortTile];
  uint32_t vals[kSortTile];
};

__global__ void __launch_bounds__(kSortThreads)
onesweep_pass_kernel(const uint64_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                     uint64_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, int64_t n,
                     int shift, const uint32_t* __restrict__ bucket_base, uint32_t* status,
                     uint32_t* tile_ctr, uint32_t* err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PassSmem& S = *reinterpret_cast<PassSmem*>(smem_raw);
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;

  if (t == 0) S.tile = atomicAdd(tile_ctr, 1u);
  for (int i = lane; i < kRadix; i += 32) S.warp_hist[w][i] = 0;
  __syncthreads();
  const uint32_t tile = S.tile;
  const int64_t tile_base = (int64_t)tile * kSortTile;

  uint64_t key[kSortItems];
  uint32_t val[kSortItems];
  uint32_t rank[kSortItems];
#pragma unroll
  for (int k = 0; k < kSortItems; k++) {
    const int64_t i = tile_base + w * (kSortItems * 32) + k * 32 + lane;
    if (i < n) {
      key[k] = keys_in[i];
      val[k] = vals_in[i];
    } else {
      key[k] = ~0ull;  // digit 255: ranks after every valid key of the tile
      val[k] = 0;
    }
  }
  const uint32_t lt = lanemask_lt();
#pragma unroll
  for (int k = 0; k < kSortItems; k++) {
    const uint32_t d = (uint32_t)(key[k] >> shift) & (kRadix - 1);
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const uint32_t before = __popc(peers & lt);
    const uint32_t prior = S.warp_hist[w][d];
    __syncwarp();
    if (before == 0) S.warp_hist[w][d] = prior + __popc(peers);
    __syncwarp();
    rank[k] = prior + before;
  }
  __syncthreads();

  // Thread t owns digit t: per-warp exclusive offsets and the tile's count.
  uint32_t run = 0;
#pragma unroll
  for (int ww = 0; ww < kSortWarps; ww++) {
    const uint32_t c = S.warp_hist[ww][t];
    S.warp_hist[ww][t] = run;
    run += c;
  }
  const uint32_t count = run;
  uint32_t* my_status = status + (size_t)tile * kRadix + t;
  if (tile == 0) {
    atomicExch(my_status, kFlagPrefix | count);
  } else {
    atomicExch(my_status, kFlagAggregate | count);
  }

  // Block-wide exclusive scan of the per-digit counts.
  {
    uint32_t x = count;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) S.warp_tot[w] = x;
    __syncthreads();
    uint32_t add = 0;
    for (int i = 0; i < w; i++) add += S.warp_tot[i];
    S.digit_excl[t] = x - count + add;
  }

  // Decoupled look-back for digit t.
  uint32_t prefix = 0;
  if (tile > 0) {
    int64_t j = (int64_t)tile - 1;
    bool ok = true;
    while (j >= 0) {
      const uint32_t* p = status + (size_t)j * kRadix + t;
      uint32_t s = load_volatile(p);
      uint32_t spins = 0;
      while ((s & kFlagMask) == 0 && ++spins < kSpinLimit) s = load_volatile(p);
      if ((s & kFlagMask) == 0) {
        ok = false;
        break;
      }
      prefix += s & kValueMask;
      if ((s & kFlagMask) == kFlagPrefix) break;
      --j;
    }
    if (!ok) set_error(err, kErrLookbackTimeout);
    atomicExch(my_status, kFlagPrefix | ((prefix + count) & kValueMask));
  }
  S.global_base[t] = bucket_base[t] + prefix;
  __syncthreads();

  // Scatter into shared memory in digit order.
#pragma unroll
  for (int k = 0; k < kSortItems; k++) {
    const uint32_t d = (uint32_t)(key[k] >> shift) & (kRadix - 1);
    const uint32_t pos = S.digit_excl[d] + S.warp_hist[w][d] + rank[k];
    S.keys[pos] = key[k];
    S.vals[pos] = val[k];
  }
  __syncthreads();

  const int valid = (int)min64(kSortTile, n - tile_base);
  for (int i = t; i < valid; i += kSortThreads) {
    const uint64_t k = S.keys[i];
    const uint32_t d = (uint32_t)(k >> shift) & (kRadix - 1);
    const uint32_t dst = S.global_base[d] + (uint32_t)i - S.digit_excl[d];
    // dst < n whenever the look-back completed; the guard keeps a timed-out
    // look-back (error bit set) from writing out of bounds.
    if ((int64_t)dst < n) {
      keys_out[dst] = k;
      vals_out[dst] = S.vals[i];
    }
  }
}

}  // namespace

size_t radix_sort_temp_bytes(int64_t n) { return sort_temp_words(n) * sizeof(uint32_t); }

// Sorts n pairs on bits [0, end_bit). keys_in/vals_in are read only; the result
// lands in keys_out/vals_out, with keys_alt/vals_alt used as the second buffer.
int radix_sort_launch(const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                      uint32_t* vals_out, uint64_t* keys_alt, uint32_t* vals_alt, int64_t n,
                      int end_bit, void* temp, size_t temp_bytes, cudaStream_t stream) {
  if (n < 0 || end_bit < 0 || end_bit > 64) return NS_ERR_INVALID;
  if (n >= (int64_t)kValueMask) return NS_ERR_UNSUPPORTED;
  if (temp_bytes < radix_sort_temp_bytes(n)) return NS_ERR_SCRATCH;
  if (n == 0) return NS_OK;
  int passes = div_up(max(end_bit, 1), kRadixBits);
  SortTemp T = carve(temp, n);
  const int64_t tiles = sort_tiles(n);
  NS_CUDA_TRY(cudaMemsetAsync(temp, 0,
                              ((size_t)kMaxPasses * kRadix + kMaxPasses + 2 +
                               (size_t)passes * tiles * kRadix) * sizeof(uint32_t),
                              stream));
  int dev = 0, sms = 0;
  NS_CUDA_TRY(cudaGetDevice(&dev));
  NS_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int hblocks = (int)min64(div_up64(n, 256 * 8), (int64_t)sms * 4);
  upfront_histogram_kernel<<<max(1, hblocks), 256, 0, stream>>>(keys_in, n, passes, T.hist);
  NS_LAUNCH_CHECK();
  bucket_scan_kernel<<<passes, kRadix, 0, stream>>>(T.hist, passes);
  NS_LAUNCH_CHECK();
  const size_t smem = sizeof(PassSmem);
  NS_CUDA_TRY(cudaFuncSetAttribute(onesweep_pass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem));
  // Ping-pong so that the last pass writes keys_out/vals_out.
  const uint64_t* kin = keys_in;
  const uint32_t* vin = vals_in;
  for (int p = 0; p < passes; p++) {
    const bool to_out = ((passes - 1 - p) % 2) == 0;
    uint64_t* kout = to_out ? keys_out : keys_alt;
    uint32_t* vout = to_out ? vals_out : vals_alt;
    onesweep_pass_kernel<<<(unsigned)tiles, kSortThreads, smem, stream>>>(
        kin, vin, kout, vout, n, p * kRadixBits, T.hist + p * kRadix,
        T.status + (size_t)p * tiles * kRadix, T.tile_ctr + p, T.err);
    NS_LAUNCH_CHECK();
    kin = kout;
    vin = vout;
  }
  return NS_OK;
}

// Address of the sort's device error word inside temp (for status reads).
uint32_t* radix_sort_error_word(void* temp) { return carve(temp, 0).err; }

}  // namespace ns
