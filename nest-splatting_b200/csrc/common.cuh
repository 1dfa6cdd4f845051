// common.cuh -- shared constants, small vector math and error plumbing for the
// sm_100a kernels of the nest-splatting render path.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nest_b200.h"

namespace ns {

// Tile geometry and rasterizer constants (cuda_rasterizer/config.h:17-18,
// auxiliary.h:42-45 of the reference).
constexpr int kTile = 16;
constexpr float kNear = 0.2f;
constexpr float kFar = 100.0f;
constexpr float kFilterSize = 0.707106f;
constexpr float kFilterInvSquare = 2.0f;
constexpr int kOtherChannels = 14;

// Device error word bits (written by kernels, read by ns_read_device_status).
constexpr uint32_t kErrLookbackTimeout = 1u;
constexpr uint32_t kErrCapacity = 2u;
constexpr uint32_t kErrSpinTimeout = 4u;

// Default bound on the polls of any wait in these kernels (ns_set_wait_limit
// changes it for later launches; the launchers pass the current value to the
// kernels). A wait that runs out records an error bit and continues, so no
// kernel can hang the GPU.
constexpr uint32_t kSpinLimit = 1u << 22;

// Per-surfel render record: 8 float4 = 128 bytes, one L2 line, written by the
// preprocess kernel and gathered by the blend kernel.
//   q0 = (x0, x1, y0, y1): pixel box outside which the surfel's alpha < 1/255
//   q1 = (Tu.x, Tu.y, Tu.z, Tv.x)      q2 = (Tv.y, Tv.z, Tw.x, Tw.y)
//   q3 = (Tw.z, xy.x, xy.y, opacity)    q4 = (n.x, n.y, n.z, ap_level bits)
//   q5 = (SuTu.x, SuTu.y, SuTu.z, SvTv.x)  q6 = (SvTv.y, SvTv.z, pk.x, pk.y)
//   q7 = (pk.z, rho_cut, surfel index bits, 0): rho_cut bounds min(rho3d, rho2d)
//        where alpha >= 1/255
struct alignas(16) SurfelRecord {
  float4 q[8];
};
constexpr int kRecordFloat4 = 8;  // float4 words the blend kernel reads

// Binning info per surfel: the tile rectangle [x0, x1) x [y0, y1) that receives
// instances (empty for culled surfels) and the view depth of the sort key.
struct alignas(16) BinInfo {
  int16_t x0, y0, x1, y1;
  float depth;
  uint32_t pad;
};

__host__ __device__ inline int div_up(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t div_up64(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ inline int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

__device__ __forceinline__ float3 f3(float x, float y, float z) { return make_float3(x, y, z); }
__device__ __forceinline__ float3 operator-(float3 a, float3 b) {
  return make_float3(a.x - b.x, a.y - b.y, a.z - b.z);
}
__device__ __forceinline__ float3 operator*(float f, float3 a) {
  return make_float3(f * a.x, f * a.y, f * a.z);
}
__device__ __forceinline__ float3 cross3(float3 a, float3 b) {
  return make_float3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}

// Tile rectangle of a screen-space disc (auxiliary.h:72-82).
__device__ __forceinline__ void tile_rect(float px, float py, int r, int gx, int gy, int& x0,
                                          int& y0, int& x1, int& y1) {
  x0 = min(gx, max(0, (int)((px - r) / kTile)));
  y0 = min(gy, max(0, (int)((py - r) / kTile)));
  x1 = min(gx, max(0, (int)((px + r + kTile - 1) / kTile)));
  y1 = min(gy, max(0, (int)((py + r + kTile - 1) / kTile)));
}

__device__ __forceinline__ void set_error(uint32_t* err, uint32_t bit) {
  if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Bounded wait on a global word that another CTA publishes: polls *p until
// (value & mask) != 0 and returns the value, or returns 0 after `limit` polls
// (the caller records the timeout in its error word).
__device__ __forceinline__ uint32_t wait_word(const uint32_t* p, uint32_t mask, uint32_t limit) {
  uint32_t v = ld_volatile_u32(p);
  for (uint32_t spins = 0; (v & mask) == 0 && spins < limit; spins++) v = ld_volatile_u32(p);
  return (v & mask) ? v : 0u;
}

// Bounded wait on a shared-memory mbarrier for the completion of the phase
// with parity `parity`. Returns 1 when it completed, 0 when *stop (if given)
// reached `stop_at` first, -1 when `limit` polls ran out.
__device__ __forceinline__ int mbar_wait_parity(const uint64_t* bar, uint32_t parity, uint32_t limit,
                                                const int* stop = nullptr, int stop_at = 0) {
  const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
  for (uint32_t spins = 0; spins < limit; spins++) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return 1;
    if (stop && *(const volatile int*)stop == stop_at) return 0;
  }
  return -1;
}

__device__ __forceinline__ void mbar_init_shared(uint64_t* bar, uint32_t count) {
  const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}

// Arrive on `bar` once all cp.async copies this thread issued so far have landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(a) : "memory");
}

}  // namespace ns

// Host-side helpers shared by the .cu files (defined in capi.cu).
namespace ns_host {
int record_cuda(cudaError_t e);  // stores e as the last CUDA error, returns NS_ERR_CUDA
void count_launch();             // one more kernel launched by this library
uint32_t wait_limit();           // poll bound passed to the kernels' waits (ns_set_wait_limit)
}

#define NS_CUDA_TRY(expr)                                       \
  do {                                                          \
    cudaError_t _e = (expr);                                    \
    if (_e != cudaSuccess) return ns_host::record_cuda(_e);     \
  } while (0)

#define NS_LAUNCH_CHECK()                                       \
  do {                                                          \
    ns_host::count_launch();                                    \
    cudaError_t _e = cudaGetLastError();                        \
    if (_e != cudaSuccess) return ns_host::record_cuda(_e);     \
  } while (0)
