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
// Every wait on another CTA's word is bounded (wait_word with the launch's poll
// limit, ns_set_wait_limit); running out sets an
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
  uint32_t* count;     // [kMaxPasses][256]
  uint32_t* nz;        // [kMaxPasses]
  uint32_t* tile_ctr;  // [kMaxPasses]
  uint32_t* err;       // [1]
  uint32_t* status;    // [kMaxPasses][tiles][256]
};

__host__ __device__ inline int64_t sort_tiles(int64_t n) { return div_up64(n, kSortTile); }

__host__ inline size_t sort_temp_words(int64_t n) {
  return (size_t)2 * kMaxPasses * kRadix + 2 * kMaxPasses + 1 + 1 /*pad*/ +
         (size_t)kMaxPasses * (size_t)max64(1, sort_tiles(n)) * kRadix;
}

__host__ inline SortTemp carve(void* temp, int64_t n) {
  SortTemp t;
  uint32_t* p = reinterpret_cast<uint32_t*>(temp);
  t.hist = p;
  t.count = p + kMaxPasses * kRadix;
  t.nz = t.count + kMaxPasses * kRadix;
  t.tile_ctr = t.nz + kMaxPasses;
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


// Histogram of every digit position in one pass over the keys. Each warp
// counts into its own shared-memory histogram (keys with few distinct digits
// would otherwise serialise all the CTA's atomics on a few words).
constexpr int kHistThreads = 256;
template <typename KeyT>
__global__ void __launch_bounds__(kHistThreads) upfront_histogram_kernel(const KeyT* __restrict__ keys,
                                                                         int64_t n, const int64_t* n_dev,
                                                                         int passes,
                                                                         uint32_t* __restrict__ hist) {
  extern __shared__ uint32_t hw[];  // [warps][passes][kRadix]
  if (n_dev) n = min(*n_dev, n);  // device-side count, at most the launch capacity
  const int w = threadIdx.x >> 5;
  const int words = (kHistThreads / 32) * passes * kRadix;
  for (int i = threadIdx.x; i < words; i += blockDim.x) hw[i] = 0;
  __syncthreads();
  uint32_t* h = hw + w * passes * kRadix;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t k = (uint64_t)keys[i];
    for (int p = 0; p < passes; p++) atomicAdd(&h[p * kRadix + ((k >> (p * kRadixBits)) & (kRadix - 1))], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRadix; i += blockDim.x) {
    uint32_t v = 0;
    for (int ww = 0; ww < kHistThreads / 32; ww++) v += hw[ww * passes * kRadix + i];
    if (v) atomicAdd(hist + i, v);
  }
}

// In place: hist[p][d] -> exclusive prefix over d (the bucket base of digit d);
// the digit counts are kept in cnt[p][d], the number of digits that occur in
// nz[p].
__global__ void bucket_scan_kernel(uint32_t* __restrict__ hist, uint32_t* __restrict__ cnt,
                                   uint32_t* __restrict__ nz, int passes) {
  __shared__ uint32_t warp_tot[kRadix / 32];
  const int p = blockIdx.x;
  if (p >= passes) return;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  uint32_t v = hist[p * kRadix + t];
  cnt[p * kRadix + t] = v;
  {
    const uint32_t m = __ballot_sync(0xffffffffu, v != 0);
    if (lane == 0) atomicAdd(nz + p, (uint32_t)__popc(m));
  }
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

template <typename KeyT>
struct PassSmem {
  uint32_t warp_hist[kSortWarps][kRadix];
  uint32_t digit_excl[kRadix];
  uint32_t global_base[kRadix];
  uint32_t warp_tot[kSortWarps];
  uint32_t tile;
  KeyT keys[kSortTile];
  uint32_t vals[kSortTile];
};

// Lanes of the warp whose 8-bit digit equals this lane's: eight ballots, one
// per digit bit (the warp multi-split of a radix pass).
__device__ __forceinline__ uint32_t equal_digit_lanes(uint32_t d) {
  uint32_t eq = 0xffffffffu;
#pragma unroll
  for (int b = 0; b < kRadixBits; b++) {
    const uint32_t bit = (d >> b) & 1u;
    const uint32_t bal = __ballot_sync(0xffffffffu, bit);
    eq &= bit ? bal : ~bal;
  }
  return eq;
}

template <typename KeyT>
__global__ void __launch_bounds__(kSortThreads)
onesweep_pass_kernel(const KeyT* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                     KeyT* __restrict__ keys_out, uint32_t* __restrict__ vals_out, int64_t n,
                     const int64_t* n_dev, int shift, const uint32_t* __restrict__ bucket_base,
                     const uint32_t* __restrict__ bucket_count, const uint32_t* __restrict__ nz_digits,
                     uint32_t* status, uint32_t* tile_ctr, uint32_t* err, uint32_t spin_limit) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PassSmem<KeyT>& S = *reinterpret_cast<PassSmem<KeyT>*>(smem_raw);
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;

  if (t == 0) S.tile = atomicAdd(tile_ctr, 1u);
  for (int i = lane; i < kRadix; i += 32) S.warp_hist[w][i] = 0;
  __syncthreads();
  const uint32_t tile = S.tile;
  // Device-side count: the grid covers the capacity; tiles past the count
  // leave at once (tiles are numbered in launch order, and a tile only looks
  // back at lower tiles, so no tile waits for one that left).
  if (n_dev) n = min(*n_dev, n);
  if ((int64_t)tile >= sort_tiles(n)) return;
  const int64_t tile_base = (int64_t)tile * kSortTile;

  KeyT key[kSortItems];
  uint32_t val[kSortItems];
  uint32_t rank[kSortItems];
#pragma unroll
  for (int k = 0; k < kSortItems; k++) {
    const int64_t i = tile_base + w * (kSortItems * 32) + k * 32 + lane;
    if (i < n) {
      key[k] = keys_in[i];
      val[k] = vals_in[i];
    } else {
      key[k] = (KeyT)~(KeyT)0;  // digit 255: ranks after every valid key of the tile
      val[k] = 0;
    }
  }
  const uint32_t lt = lanemask_lt();
  // match-any is cheap when a warp's keys share few digits, the ballots when
  // they are spread: choose by the number of digits the pass has (uniform).
  const bool spread = *nz_digits > 32u;
#pragma unroll
  for (int k = 0; k < kSortItems; k++) {
    const uint32_t d = (uint32_t)(key[k] >> shift) & (kRadix - 1);
    const uint32_t peers = spread ? equal_digit_lanes(d) : __match_any_sync(0xffffffffu, d);
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

  // Decoupled look-back for digit t (none for a digit no key of the pass has).
  uint32_t prefix = 0;
  if (tile > 0 && bucket_count[t] != 0) {
    int64_t j = (int64_t)tile - 1;
    bool ok = true;
    while (j >= 0) {
      const uint32_t s = wait_word(status + (size_t)j * kRadix + t, kFlagMask, spin_limit);
      if (s == 0u) {
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
    const KeyT k = S.keys[i];
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

template <typename KeyT>
int radix_sort_impl(const KeyT* keys_in, const uint32_t* vals_in, KeyT* keys_out, uint32_t* vals_out,
                    KeyT* keys_alt, uint32_t* vals_alt, int64_t n, int end_bit, void* temp,
                    size_t temp_bytes, cudaStream_t stream, const int64_t* n_dev) {
  if (n < 0 || end_bit < 0 || end_bit > (int)(8 * sizeof(KeyT))) return NS_ERR_INVALID;
  if (n >= (int64_t)kValueMask) return NS_ERR_UNSUPPORTED;
  if (temp_bytes < sort_temp_words(n) * sizeof(uint32_t)) return NS_ERR_SCRATCH;
  if (n == 0) return NS_OK;
  int passes = div_up(max(end_bit, 1), kRadixBits);
  SortTemp T = carve(temp, n);
  const int64_t tiles = sort_tiles(n);
  NS_CUDA_TRY(cudaMemsetAsync(temp, 0,
                              ((size_t)2 * kMaxPasses * kRadix + 2 * kMaxPasses + 2 +
                               (size_t)passes * tiles * kRadix) * sizeof(uint32_t),
                              stream));
  int dev = 0, sms = 0;
  NS_CUDA_TRY(cudaGetDevice(&dev));
  NS_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int hblocks = (int)min64(div_up64(n, 256 * 8), (int64_t)sms * 4);
  const size_t hsmem = (size_t)(kHistThreads / 32) * passes * kRadix * sizeof(uint32_t);
  if (hsmem > 48 * 1024)
    NS_CUDA_TRY(cudaFuncSetAttribute(upfront_histogram_kernel<KeyT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hsmem));
  upfront_histogram_kernel<KeyT><<<max(1, hblocks), kHistThreads, hsmem, stream>>>(keys_in, n, n_dev,
                                                                                  passes, T.hist);
  NS_LAUNCH_CHECK();
  bucket_scan_kernel<<<passes, kRadix, 0, stream>>>(T.hist, T.count, T.nz, passes);
  NS_LAUNCH_CHECK();
  const size_t smem = sizeof(PassSmem<KeyT>);
  NS_CUDA_TRY(cudaFuncSetAttribute(onesweep_pass_kernel<KeyT>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  // Ping-pong so that the last pass writes keys_out/vals_out.
  const KeyT* kin = keys_in;
  const uint32_t* vin = vals_in;
  for (int p = 0; p < passes; p++) {
    const bool to_out = ((passes - 1 - p) % 2) == 0;
    KeyT* kout = to_out ? keys_out : keys_alt;
    uint32_t* vout = to_out ? vals_out : vals_alt;
    onesweep_pass_kernel<KeyT><<<(unsigned)tiles, kSortThreads, smem, stream>>>(
        kin, vin, kout, vout, n, n_dev, p * kRadixBits, T.hist + p * kRadix, T.count + p * kRadix,
        T.nz + p, T.status + (size_t)p * tiles * kRadix, T.tile_ctr + p, T.err, ns_host::wait_limit());
    NS_LAUNCH_CHECK();
    kin = kout;
    vin = vout;
  }
  return NS_OK;
}

}  // namespace

size_t radix_sort_temp_bytes(int64_t n) { return sort_temp_words(n) * sizeof(uint32_t); }

// Sorts n pairs on bits [0, end_bit). keys_in/vals_in are read only; the result
// lands in keys_out/vals_out, with keys_alt/vals_alt used as the second buffer.
int radix_sort_launch(const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                      uint32_t* vals_out, uint64_t* keys_alt, uint32_t* vals_alt, int64_t n,
                      int end_bit, void* temp, size_t temp_bytes, cudaStream_t stream) {
  return radix_sort_impl<uint64_t>(keys_in, vals_in, keys_out, vals_out, keys_alt, vals_alt, n,
                                   end_bit, temp, temp_bytes, stream, nullptr);
}

// The same for 32-bit keys (end_bit <= 32): two thirds of the traffic per pass.
// n_dev (optional): the number of pairs as a device value, at most n; the
// launches are sized by n and read the count on the device (no host sync).
int radix_sort32_launch(const uint32_t* keys_in, const uint32_t* vals_in, uint32_t* keys_out,
                        uint32_t* vals_out, uint32_t* keys_alt, uint32_t* vals_alt, int64_t n,
                        int end_bit, void* temp, size_t temp_bytes, cudaStream_t stream,
                        const int64_t* n_dev) {
  return radix_sort_impl<uint32_t>(keys_in, vals_in, keys_out, vals_out, keys_alt, vals_alt, n,
                                   end_bit, temp, temp_bytes, stream, n_dev);
}

// Address of the sort's device error word inside temp (for status reads).
uint32_t* radix_sort_error_word(void* temp) { return carve(temp, 0).err; }

}  // namespace ns
