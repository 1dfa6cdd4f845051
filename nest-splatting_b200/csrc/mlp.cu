// mlp.cu -- the per-pixel colour MLP on tensor cores.
//
// Restates INGP.get_color (hash_encoder/modules.py:587-594) for the baseline
// branch of render() (gaussian_renderer/__init__.py:1005-1015): a bias-free
// tiny-cuda-nn "MLP" 32 -> 64 -> 64 -> 3 with ReLU hidden layers, fp16
// operands, and a sigmoid on the (fp16) network output, then x (alpha > 0) and
// the optional background term (:1020-1021).
//
// Numerics: inputs and weights fp16, fp32 accumulation, each layer's output
// rounded to fp16 (the next layer's operand and the network output dtype).
//
// Tensor-core mapping: mma.sync m16n8k16 (f16 x f16 -> f32). A warp owns 16
// pixels; layer l's fp32 accumulator fragments are rounded to f16x2 in place
// and become the A fragments of layer l+1 without touching shared memory. The
// weights live in shared memory with padded rows (conflict-free fragment
// loads). The MLP is 14.3 kFLOP per pixel: it is a small share of a frame.
#include "common.cuh"

namespace ns {
namespace {

constexpr int kIn = 32, kHid = 64, kOut = 8;  // output padded to one n-tile
constexpr int kW1Stride = kIn + 8;            // halves per padded row
constexpr int kW2Stride = kHid + 8;
constexpr int kMlpWarps = 4;

struct MlpSmem {
  __half w1[kHid * kW1Stride];
  __half w2[kHid * kW2Stride];
  __half w3[kOut * kW2Stride];
};

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t lds32(const __half* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

__device__ void load_weights(MlpSmem& S, const uint16_t* __restrict__ w) {
  const __half* W = reinterpret_cast<const __half*>(w);
  for (int i = threadIdx.x; i < kHid * kIn; i += blockDim.x)
    S.w1[(i / kIn) * kW1Stride + (i % kIn)] = W[i];
  const __half* W2 = W + kHid * kIn;
  for (int i = threadIdx.x; i < kHid * kHid; i += blockDim.x)
    S.w2[(i / kHid) * kW2Stride + (i % kHid)] = W2[i];
  const __half* W3 = W2 + kHid * kHid;
  for (int i = threadIdx.x; i < kOut * kHid; i += blockDim.x) {
    const int r = i / kHid;
    S.w3[r * kW2Stride + (i % kHid)] = r < 3 ? W3[i] : __float2half(0.f);
  }
}

// MLP of 16 pixels held by one warp. a_in: layer-1 A fragments (2 k-steps).
// Returns the output fragment (cols 0..7 of rows g and g+8; cols 0..2 valid),
// already rounded through fp16.
__device__ __forceinline__ void mlp16(const MlpSmem& S, const uint32_t (&a_in)[2][4],
                                      float (&y)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  // Layer 1: [16 x 32] x [32 x 64]
  float h1[8][4];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    h1[j][0] = h1[j][1] = h1[j][2] = h1[j][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 2; s++) {
      const __half* wr = S.w1 + (8 * j + g) * kW1Stride + 16 * s + 2 * tig;
      mma16816(h1[j], a_in[s], lds32(wr), lds32(wr + 8));
    }
  }
  uint32_t a2[4][4];
#pragma unroll
  for (int s = 0; s < 4; s++) {
    a2[s][0] = pack_half2(fmaxf(h1[2 * s][0], 0.f), fmaxf(h1[2 * s][1], 0.f));
    a2[s][1] = pack_half2(fmaxf(h1[2 * s][2], 0.f), fmaxf(h1[2 * s][3], 0.f));
    a2[s][2] = pack_half2(fmaxf(h1[2 * s + 1][0], 0.f), fmaxf(h1[2 * s + 1][1], 0.f));
    a2[s][3] = pack_half2(fmaxf(h1[2 * s + 1][2], 0.f), fmaxf(h1[2 * s + 1][3], 0.f));
  }
  // Layer 2: [16 x 64] x [64 x 64]
  float h2[8][4];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    h2[j][0] = h2[j][1] = h2[j][2] = h2[j][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; s++) {
      const __half* wr = S.w2 + (8 * j + g) * kW2Stride + 16 * s + 2 * tig;
      mma16816(h2[j], a2[s], lds32(wr), lds32(wr + 8));
    }
  }
  uint32_t a3[4][4];
#pragma unroll
  for (int s = 0; s < 4; s++) {
    a3[s][0] = pack_half2(fmaxf(h2[2 * s][0], 0.f), fmaxf(h2[2 * s][1], 0.f));
    a3[s][1] = pack_half2(fmaxf(h2[2 * s][2], 0.f), fmaxf(h2[2 * s][3], 0.f));
    a3[s][2] = pack_half2(fmaxf(h2[2 * s + 1][0], 0.f), fmaxf(h2[2 * s + 1][1], 0.f));
    a3[s][3] = pack_half2(fmaxf(h2[2 * s + 1][2], 0.f), fmaxf(h2[2 * s + 1][3], 0.f));
  }
  // Layer 3: [16 x 64] x [64 x 8]
  y[0] = y[1] = y[2] = y[3] = 0.f;
#pragma unroll
  for (int s = 0; s < 4; s++) {
    const __half* wr = S.w3 + g * kW2Stride + 16 * s + 2 * tig;
    mma16816(y, a3[s], lds32(wr), lds32(wr + 8));
  }
#pragma unroll
  for (int i = 0; i < 4; i++) y[i] = __half2float(__float2half_rn(y[i]));
}

__device__ __forceinline__ float sigmoidf(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void __launch_bounds__(kMlpWarps * 32)
mlp_kernel(const float* __restrict__ feat, int64_t npix, const uint16_t* __restrict__ weights,
           const float* __restrict__ alpha, float bg0, float bg1, float bg2, int use_bg,
           float* __restrict__ rgb) {
  __shared__ MlpSmem S;
  load_weights(S, weights);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tig = lane & 3;
  const int64_t ntiles = div_up64(npix, 16);
  for (int64_t tile = (int64_t)blockIdx.x * kMlpWarps + warp; tile < ntiles;
       tile += (int64_t)gridDim.x * kMlpWarps) {
    const int64_t p0 = tile * 16 + g, p1 = p0 + 8;
    const bool v0 = p0 < npix, v1 = p1 < npix;
    uint32_t a[2][4];
#pragma unroll
    for (int s = 0; s < 2; s++) {
      const int c = 16 * s + 2 * tig;
      auto ld = [&](int ch, int64_t px, bool v) { return v ? __ldg(feat + ch * npix + px) : 0.f; };
      a[s][0] = pack_half2(ld(c, p0, v0), ld(c + 1, p0, v0));
      a[s][1] = pack_half2(ld(c, p1, v1), ld(c + 1, p1, v1));
      a[s][2] = pack_half2(ld(c + 8, p0, v0), ld(c + 9, p0, v0));
      a[s][3] = pack_half2(ld(c + 8, p1, v1), ld(c + 9, p1, v1));
    }
    float y[4];
    mlp16(S, a, y);
    // y[0..1]: row g cols 2tig, 2tig+1; y[2..3]: row g+8.
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int64_t px = r ? p1 : p0;
      if (!(r ? v1 : v0)) continue;
      const float a_px = alpha ? alpha[px] : 1.0f;
#pragma unroll
      for (int cc = 0; cc < 2; cc++) {
        const int col = 2 * tig + cc;
        if (col >= 3) continue;
        float v = sigmoidf(y[2 * r + cc]);
        if (alpha && !(a_px > 0.f)) v = 0.f;
        if (use_bg) v += (1.0f - a_px) * (col == 0 ? bg0 : col == 1 ? bg1 : bg2);
        rgb[col * npix + px] = v;
      }
    }
  }
}

}  // namespace

int mlp_launch(const float* feat, int in_dims, int64_t npix, const uint16_t* weights, int hidden,
               int out_dims, const float* alpha, const float* bg_host, float* rgb,
               cudaStream_t stream) {
  if (in_dims != kIn || hidden != kHid || out_dims != 3) return NS_ERR_UNSUPPORTED;
  if (npix < 0) return NS_ERR_INVALID;
  if (npix == 0) return NS_OK;
  if (!feat || !weights || !rgb) return NS_ERR_INVALID;
  int use_bg = 0;
  float b0 = 0, b1 = 0, b2 = 0;
  if (bg_host) {
    b0 = bg_host[0];
    b1 = bg_host[1];
    b2 = bg_host[2];
    use_bg = (b0 + b1 + b2) > 0.f;
  }
  if (use_bg && !alpha) return NS_ERR_INVALID;
  int dev = 0, sms = 0;
  NS_CUDA_TRY(cudaGetDevice(&dev));
  NS_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t ntiles = div_up64(npix, 16);
  const int blocks = (int)min64(div_up64(ntiles, kMlpWarps), (int64_t)sms * 8);
  mlp_kernel<<<blocks, kMlpWarps * 32, 0, stream>>>(feat, npix, weights, alpha, b0, b1, b2, use_bg,
                                                    rgb);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
