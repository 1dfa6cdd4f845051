// rvq.cu -- residual-vector-quantised attribute decode.
//
// out[n, d] = sum_{k=0..K-1} codebooks[k, idx[n,k], d], accumulated in fp32 from
// +0.0 in stage order k = 0, 1, ... (the reference repository
// has no RVQ code, so this is new scope with a bit-exact contract).
//
// Shared-memory kernel (the fast path). The whole codebook of the benchmark
// shape (6 x 256 x 59 fp32 = 354 KB) does not fit one SM's 227 KB of shared
// memory, so the dimension axis is split in two halves of 32 columns and each
// CTA holds all stages of one half (6 x 256 x 32 x 4 = 192 KB). CTAs are
// persistent (one per SM) and walk 1024-surfel chunks. The codebook half and
// the chunks' index bytes arrive by cp.async; index bytes run three chunks
// ahead of the decode (a chunk decodes in about a microsecond, less than one
// DRAM round trip, so a single chunk of look-ahead left the kernel waiting on
// its index stream). Index bytes are packed to one u64 per surfel in shared
// memory so the stage indices of a surfel cost one broadcast read.
//
// Bound: HBM (6 B of indices read + 4*dims B written per surfel); the shared
// memory gather (6 x 128 B per surfel-half) runs at about the same time, so
// the two overlap.
#include "common.cuh"

namespace ns {
namespace {

constexpr int kRvqThreads = 512;
constexpr int kRvqChunk = 1024;  // surfels per chunk (two per thread for index packing)
constexpr int kHalfCols = 32;
constexpr int kIdxStages = 3;    // index chunks in flight

// Raw index bytes of one chunk as 4-byte words, for K stages.
template <int K>
__host__ __device__ constexpr int kIdxWordsK() { return (kRvqChunk * K + 3) / 4; }

__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src, int src_bytes) {
  const unsigned dst = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(gmem_src),
               "r"(src_bytes));
}

// Streams the raw index bytes of chunk `ch` (cnt surfels x K bytes, contiguous
// in global memory at a 4-byte aligned offset) into `raw` with 4-byte cp.async;
// the tail word is zero-filled past the end of the array.
__device__ __forceinline__ void fetch_indices(const uint8_t* __restrict__ idx, int64_t n, int K,
                                              int64_t ch, int64_t nchunks, uint32_t* raw) {
  if (ch < nchunks) {
    const int64_t first = ch * kRvqChunk;
    const int cnt = (int)min64(kRvqChunk, n - first);
    const int bytes = cnt * K;
    const uint8_t* src = idx + first * K;
    for (int w = threadIdx.x; w * 4 < bytes; w += kRvqThreads)
      cp_async4(raw + w, src + 4 * w, min(4, bytes - 4 * w));
  }
  asm volatile("cp.async.commit_group;");
}

// Shared-memory decode. Template on the stage count K (fully unrolled).
// Codebook half layout in shared memory, permuted per lane: entry (k, e) is 32
// floats where lane j of an 8-lane group finds its columns col0 + j + 8q
// (q = 0..3) at [j*4 + q], so one 128-bit load gives a lane its four columns.
// A warp decodes four surfels per step (one 8-lane group each); stores of a
// step are 8 consecutive floats per surfel and column block (full sectors).
template <int K>
__global__ void __launch_bounds__(kRvqThreads, 1)
rvq_decode_smem_kernel(const uint8_t* __restrict__ idx, const float* __restrict__ cb,
                       float* __restrict__ out, int64_t n, int E, int D) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* cb_s = reinterpret_cast<float*>(smem_raw);                                  // [K*E][32]
  uint32_t* raw = reinterpret_cast<uint32_t*>(cb_s + (size_t)K * E * kHalfCols);     // [stages][words]
  uint2* idx_s = reinterpret_cast<uint2*>(raw + kIdxStages * kIdxWordsK<K>());       // [chunk]

  const int half = blockIdx.y;
  const int col0 = half * kHalfCols;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  // Stage this half of every codeword, permuted (columns past D zero-filled).
  const int rows = K * E;
  for (int i = tid; i < rows * kHalfCols; i += kRvqThreads) {
    const int r = i >> 5, jq = i & 31;           // destination slot j*4 + q
    const int c = col0 + (jq >> 2) + 8 * (jq & 3);
    const float* src = cb + (size_t)r * D + (c < D ? c : 0);
    cp_async4(cb_s + i, src, c < D ? 4 : 0);
  }
  asm volatile("cp.async.commit_group;");

  const int64_t nchunks = div_up64(n, kRvqChunk);
  int64_t chunk = blockIdx.x;
  int buf = 0;
  constexpr int kWords = kIdxWordsK<K>();
#pragma unroll
  for (int st = 0; st < kIdxStages; st++)
    fetch_indices(idx, n, K, chunk + (int64_t)st * gridDim.x, nchunks, raw + st * kWords);

  const int grp = lane >> 3;  // surfel of the step
  const int j = lane & 7;     // column block of the lane
  const float4* cb4 = reinterpret_cast<const float4*>(cb_s);
  const bool check_e = E < 256;

  for (; chunk < nchunks; chunk += gridDim.x, buf = (buf + 1 == kIdxStages) ? 0 : buf + 1) {
    // The oldest of the kIdxStages groups in flight (this chunk's bytes; the
    // first time also the codebook) is complete.
    asm volatile("cp.async.wait_group %0;" ::"n"(kIdxStages - 1));
    __syncthreads();  // ... for every thread; the previous chunk's decode is done
    const int64_t base = chunk * kRvqChunk;
    const int cnt = (int)min64(kRvqChunk, n - base);
#pragma unroll
    for (int h = 0; h < (kRvqChunk + kRvqThreads - 1) / kRvqThreads; h++) {  // surfel's K index bytes
      const int sl = tid + h * kRvqThreads;
      const uint8_t* b = reinterpret_cast<const uint8_t*>(raw + buf * kWords) + sl * K;
      uint32_t lo = 0, hi = 0;
      if (sl < cnt) {
#pragma unroll
        for (int k = 0; k < K; k++) {
          if (k < 4) lo |= (uint32_t)b[k] << (8 * k);
          else hi |= (uint32_t)b[k] << (8 * (k - 4));
        }
      }
      idx_s[sl] = make_uint2(lo, hi);
    }
    __syncthreads();  // packed indices visible; raw[buf] free for the chunk kIdxStages ahead
    fetch_indices(idx, n, K, chunk + (int64_t)kIdxStages * gridDim.x, nchunks, raw + buf * kWords);
    constexpr int kWarpsPerCta = kRvqThreads / 32;
    constexpr int kPerWarp = kRvqChunk / kWarpsPerCta;  // surfels per warp per chunk
#pragma unroll 2
    for (int step = 0; step < kPerWarp / 4; step++) {
      const int s = warp * kPerWarp + step * 4 + grp;
      if (s < cnt) {
        const uint2 ix = idx_s[s];
        float2 a01 = make_float2(0.0f, 0.0f), a23 = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < K; k++) {
          const uint32_t e = ((k < 4 ? ix.x : ix.y) >> (8 * (k & 3))) & 0xffu;
          if (check_e && e >= (uint32_t)E) continue;  // outside the codebook: contributes nothing
          const float4 v = cb4[(k * E + (int)e) * 8 + j];
          a01 = __fadd2_rn(a01, make_float2(v.x, v.y));
          a23 = __fadd2_rn(a23, make_float2(v.z, v.w));
        }
        float* o = out + (base + s) * D + col0 + j;
        const float a[4] = {a01.x, a01.y, a23.x, a23.y};
#pragma unroll
        for (int q = 0; q < 4; q++)
          if (col0 + j + 8 * q < D) o[8 * q] = a[q];
      }
    }
  }
  asm volatile("cp.async.wait_group 0;");
}

template <int K>
int launch_rvq_smem(const uint8_t* idx, const float* cb, float* out, int64_t n, int E, int D,
                    size_t smem, int sms, cudaStream_t stream) {
  NS_CUDA_TRY(cudaFuncSetAttribute(rvq_decode_smem_kernel<K>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int halves = D > kHalfCols ? 2 : 1;
  const int64_t nchunks = div_up64(n, kRvqChunk);
  const int gx = (int)min64(nchunks, (int64_t)max(1, sms / halves));
  rvq_decode_smem_kernel<K><<<dim3(gx, halves), kRvqThreads, smem, stream>>>(idx, cb, out, n, E, D);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

// General shape: one thread per output value, codebook rows read through L1/L2.
__global__ void rvq_decode_gather_kernel(const uint8_t* __restrict__ idx,
                                         const float* __restrict__ cb, float* __restrict__ out,
                                         int64_t n, int K, int E, int D) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = n * D;
  for (; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t s = i / D;
    int d = (int)(i - s * D);
    float acc = 0.0f;
    for (int k = 0; k < K; k++) {
      const int e = idx[s * K + k];
      if (e < E) acc += __ldg(cb + ((size_t)k * E + e) * D + d);
    }
    out[i] = acc;
  }
}

}  // namespace

int rvq_decode_launch(const uint8_t* idx, const float* cb, float* out, int64_t n, int K, int E,
                      int D, cudaStream_t stream) {
  if (n < 0 || K <= 0 || K > 8 || E <= 0 || E > 256 || D <= 0 || D > 64) return NS_ERR_UNSUPPORTED;
  if (n == 0) return NS_OK;
  if (!idx || !cb || !out) return NS_ERR_INVALID;
  const size_t smem = (size_t)K * E * kHalfCols * sizeof(float) +
                      kIdxStages * (size_t)((kRvqChunk * K + 3) / 4) * sizeof(uint32_t) +
                      kRvqChunk * sizeof(uint2);
  int dev = 0, sms = 0, max_smem = 0;
  NS_CUDA_TRY(cudaGetDevice(&dev));
  NS_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  NS_CUDA_TRY(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  // The shared-memory kernel copies index bytes in 4-byte words and codebook
  // entries as floats: both arrays must be 4-byte aligned.
  const bool aligned = ((uintptr_t)idx % 4 == 0) && ((uintptr_t)cb % 4 == 0);
  if (smem <= (size_t)max_smem && aligned) {
    switch (K) {
      case 1: return launch_rvq_smem<1>(idx, cb, out, n, E, D, smem, sms, stream);
      case 2: return launch_rvq_smem<2>(idx, cb, out, n, E, D, smem, sms, stream);
      case 3: return launch_rvq_smem<3>(idx, cb, out, n, E, D, smem, sms, stream);
      case 4: return launch_rvq_smem<4>(idx, cb, out, n, E, D, smem, sms, stream);
      case 5: return launch_rvq_smem<5>(idx, cb, out, n, E, D, smem, sms, stream);
      case 6: return launch_rvq_smem<6>(idx, cb, out, n, E, D, smem, sms, stream);
      case 7: return launch_rvq_smem<7>(idx, cb, out, n, E, D, smem, sms, stream);
      default: return launch_rvq_smem<8>(idx, cb, out, n, E, D, smem, sms, stream);
    }
  } else {
    int64_t total = n * D;
    int blocks = (int)min64(div_up64(total, 256), (int64_t)sms * 16);
    rvq_decode_gather_kernel<<<blocks, 256, 0, stream>>>(idx, cb, out, n, K, E, D);
  }
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
