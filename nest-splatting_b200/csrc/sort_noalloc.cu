// sort_noalloc.cu -- the radix sort for callers that cannot allocate device memory.
//
// Some hosts own every byte of device memory themselves: a renderer plugin
// that runs inside an engine's frame with a fixed memory budget, a serving
// runtime that hands kernels slices of one pre-sized arena, or a binding from
// a language without a CUDA allocator. Such callers can pass their inputs and
// outputs but cannot obtain the sort's ping-pong buffers and look-back state
// with cudaMalloc. ns_radix_sort_pairs_noalloc keeps that state in a
// file-scope device array instead, sized for at most kNoAllocMaxPairs pairs.
//
// Costs and limits (stated in include/nest_b200.h as well):
//   * the array (kNoAllocBytes, about 14 MB) exists on every GPU that loads the
//     library, from load until process exit;
//   * all calls share it: two calls whose kernels overlap on the GPU (other
//     streams, other host threads) race and corrupt each other's results, so
//     callers must serialise them (one stream is enough);
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress for that device; make that first call before any
//     stream capture. The address is cached per device together with the
//     identity of the device's current CUDA context: after a context reset
//     (cudaDeviceReset, a primary context released and retained again) the
//     next call looks it up again, so a reloaded module is never addressed
//     through a stale pointer;
//   * the sort's bounded look-back waits record a timeout in an error word
//     inside the array, which this entry point does not read back (that would
//     cost a stream synchronisation per call): it reports argument and launch
//     errors only. A look-back wait runs out only on a GPU that has stopped
//     making progress; the sorted output is then undefined.
#include <cuda.h>

#include <mutex>

#include "kernels.cuh"

namespace ns {
namespace {

constexpr int64_t kNoAllocMaxPairs = int64_t(1) << 20;
// keys_alt (8 B) + vals_alt (4 B) per pair, then the sort's temp words.
constexpr size_t kAltKeysBytes = size_t(kNoAllocMaxPairs) * sizeof(uint64_t);
constexpr size_t kAltValsBytes = size_t(kNoAllocMaxPairs) * sizeof(uint32_t);
// histograms + digit counts (2 x 8 x 256), digits-present and tile counters
// (2 x 8), error word, pad, look-back words of 8 passes x 256 tiles x 256
// digits (radix_sort_temp_bytes(kNoAllocMaxPairs)).
constexpr size_t kTempBytesMax =
    (size_t(2) * 8 * 256 + 2 * 8 + 2 + size_t(8) * 256 * 256) * sizeof(uint32_t);
constexpr size_t kNoAllocBytes = kAltKeysBytes + kAltValsBytes + kTempBytesMax;

__device__ __align__(256) unsigned char g_sort_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_addr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};  // context id the address belongs to

// Unique id of the calling thread's current context (cuCtxGetId: ids are never
// reused within a process), through the runtime's driver entry points so the
// library needs no link against libcuda. 0 when unavailable.
unsigned long long current_context_id() {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(f);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of g_sort_scratch on the current device, looked up once per
// device and context (without a context id, on every call).
int scratch_address(void** out) {
  int dev = 0;
  NS_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return NS_ERR_UNSUPPORTED;
  // Id 0: no context is current on this thread yet (the runtime makes the
  // device's primary context current on its first call that needs one, e.g.
  // the lookup below) or the driver lacks cuCtxGetId.
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_scratch_addr[dev] || ctx == 0 || g_scratch_ctx[dev] != ctx) {
    void* ptr = nullptr;
    NS_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_sort_scratch));
    g_scratch_addr[dev] = ptr;
    g_scratch_ctx[dev] = ctx ? ctx : current_context_id();
  }
  *out = g_scratch_addr[dev];
  return NS_OK;
}

}  // namespace
}  // namespace ns

extern "C" int ns_radix_sort_pairs_noalloc(const uint64_t* keys_in, const uint32_t* vals_in,
                                           uint64_t* keys_out, uint32_t* vals_out, int64_t n,
                                           int32_t end_bit, void* stream) {
  using namespace ns;
  if (n < 0 || end_bit < 0 || end_bit > 64) return NS_ERR_INVALID;  // as ns_radix_sort_pairs
  if (n > kNoAllocMaxPairs) return NS_ERR_CAPACITY;
  if (n > 0 && (!keys_in || !vals_in || !keys_out || !vals_out)) return NS_ERR_INVALID;
  if (n == 0) return NS_OK;
  if (radix_sort_temp_bytes(n) > kTempBytesMax) return NS_ERR_CAPACITY;
  void* base = nullptr;
  const int rc = scratch_address(&base);
  if (rc) return rc;
  unsigned char* b = static_cast<unsigned char*>(base);
  uint64_t* keys_alt = reinterpret_cast<uint64_t*>(b);
  uint32_t* vals_alt = reinterpret_cast<uint32_t*>(b + kAltKeysBytes);
  void* temp = b + kAltKeysBytes + kAltValsBytes;
  // radix_sort_launch zeroes the histogram, tile-counter and look-back words it
  // uses (cudaMemsetAsync on `temp`) before its first kernel; the ping-pong
  // buffers are fully written before they are read.
  return radix_sort_launch(keys_in, vals_in, keys_out, vals_out, keys_alt, vals_alt, n, end_bit,
                           temp, kTempBytesMax, reinterpret_cast<cudaStream_t>(stream));
}
