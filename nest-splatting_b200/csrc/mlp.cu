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
// Forward: tcgen05.mma on 128-pixel tiles with the accumulators in TMEM
// (mlp_tc.cuh). Backward: mma.sync (m16n8k16 fp16 for the recomputed forward,
// m16n8k8 TF32 for the gradients), a warp per 16 pixels, weights in shared
// memory with padded rows (conflict-free fragment loads). The MLP is 14.3
// kFLOP per pixel: it is a small share of a frame.
#include "common.cuh"

namespace ns {
namespace {

constexpr int kIn = 32, kHid = 64, kOut = 8;  // output padded to one n-tile
constexpr int kW1Stride = kIn + 8;            // halves per padded row
constexpr int kW2Stride = kHid + 8;

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

__device__ __forceinline__ float sigmoidf(float x) { return 1.0f / (1.0f + expf(-x)); }

#include "mlp_tc.cuh"

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
  NS_CUDA_TRY(cudaFuncSetAttribute(mlp_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBytes));
  const int blocks = (int)min64(div_up64(npix, kTcThreads), (int64_t)sms * 4);
  mlp_tc_kernel<<<blocks, kTcThreads, kTcSmemBytes, stream>>>(feat, npix, weights, alpha, b0, b1, b2, use_bg,
                                                              rgb);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

// ---------------------------------------------------------------------------
// Backward of the colour MLP (the training step's d loss / d features and
// d loss / d weights), fused: per 16-pixel warp tile the forward is recomputed
// with the forward's roundings (fp16 operands, fp32 accumulation, each
// layer rounded to fp16, ReLU masks kept as bits), then
//   dz3 = g * (alpha > 0) * s (1 - s)           s = sigmoid(z3), 3 outputs
//   dz2 = (dz3 W3) * (z2 > 0),  dz1 = (dz2 W2) * (z1 > 0),  dfeat = dz1 W1
// on TF32 tensor cores (mma.sync m16n8k8, fp32 accumulation; the fp16 weights
// and activations are exact in TF32, dz is rounded to TF32). The weight
// gradients dW3 = dz3^T a2, dW2 = dz2^T a1, dW1 = dz1^T x are GEMMs over the
// pixels: each 64-pixel block's dz and activations are staged in shared memory
// and every warp accumulates its 16-row slice of dW1 / dW2 (and two n-tiles of
// dW3) in registers across all blocks of the CTA, added to the global
// gradients once per CTA. The fp16 roundings are treated as identity in the
// backward, as autograd through .half() does.
namespace {

constexpr int kBwWarps = 4;
constexpr int kBwPix = 16 * kBwWarps;  // pixels per block
constexpr int kDzStride = 68;          // floats per staged dz row (conflict-free A loads)
constexpr int kAhStride = 72;          // halves per staged activation row
constexpr int kXhStride = 40;          // halves per staged input row
constexpr int kD3Stride = 12;          // floats per staged dz3 row

struct MlpBwSmem {
  MlpSmem w;
  float dz2[kBwPix * kDzStride];
  float dz1[kBwPix * kDzStride];
  float dz3[kBwPix * kD3Stride];
  __half a1[kBwPix * kAhStride];
  __half a2[kBwPix * kAhStride];
  __half xh[kBwPix * kXhStride];
};

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ uint32_t h2tf(__half h) { return __float_as_uint(__half2float(h)); }

__device__ __forceinline__ void mma1688(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kBwWarps * 32)
mlp_backward_kernel(const float* __restrict__ feat, int64_t npix, const uint16_t* __restrict__ weights,
                    const float* __restrict__ alpha, const float* __restrict__ grgb,
                    float* __restrict__ dfeat, float* __restrict__ dW) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  MlpBwSmem& S = *reinterpret_cast<MlpBwSmem*>(smem_raw);
  load_weights(S.w, weights);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tig = lane & 3;
  const int r0 = 16 * warp + g, r1 = r0 + 8;  // this thread's rows of the block

  // Weight-gradient accumulators: dW2 rows 16w..16w+15 (8 n-tiles), dW1 rows
  // 16w..16w+15 (4 n-tiles), dW3 rows 0..15 (valid 0..2) n-tiles 2w, 2w+1.
  float gw2[8][4], gw1[4][4], gw3[2][4];
#pragma unroll
  for (int j = 0; j < 8; j++) gw2[j][0] = gw2[j][1] = gw2[j][2] = gw2[j][3] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++) gw1[j][0] = gw1[j][1] = gw1[j][2] = gw1[j][3] = 0.f;
#pragma unroll
  for (int j = 0; j < 2; j++) gw3[j][0] = gw3[j][1] = gw3[j][2] = gw3[j][3] = 0.f;

  const int64_t nblocks = div_up64(npix, kBwPix);
  for (int64_t blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
    const int64_t p0 = blk * kBwPix + r0, p1 = blk * kBwPix + r1;
    const bool v0 = p0 < npix, v1 = p1 < npix;
    // ---- forward recompute (the forward's layers and roundings), keeping ReLU masks and staging a1, a2, x.
    uint32_t a[2][4];
#pragma unroll
    for (int s = 0; s < 2; s++) {
      const int c = 16 * s + 2 * tig;
      auto ld = [&](int ch, int64_t px, bool v) { return v ? __ldg(feat + ch * npix + px) : 0.f; };
      a[s][0] = pack_half2(ld(c, p0, v0), ld(c + 1, p0, v0));
      a[s][1] = pack_half2(ld(c, p1, v1), ld(c + 1, p1, v1));
      a[s][2] = pack_half2(ld(c + 8, p0, v0), ld(c + 9, p0, v0));
      a[s][3] = pack_half2(ld(c + 8, p1, v1), ld(c + 9, p1, v1));
      *reinterpret_cast<uint32_t*>(S.xh + r0 * kXhStride + c) = a[s][0];
      *reinterpret_cast<uint32_t*>(S.xh + r1 * kXhStride + c) = a[s][1];
      *reinterpret_cast<uint32_t*>(S.xh + r0 * kXhStride + c + 8) = a[s][2];
      *reinterpret_cast<uint32_t*>(S.xh + r1 * kXhStride + c + 8) = a[s][3];
    }
    uint32_t m1 = 0, m2 = 0;  // ReLU masks, bit 4j + e for element e of n-tile j
    uint32_t a2f[4][4];
    {
      float h[8][4];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        h[j][0] = h[j][1] = h[j][2] = h[j][3] = 0.f;
#pragma unroll
        for (int s = 0; s < 2; s++) {
          const __half* wr = S.w.w1 + (8 * j + g) * kW1Stride + 16 * s + 2 * tig;
          mma16816(h[j], a[s], lds32(wr), lds32(wr + 8));
        }
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int c = 8 * j + 2 * tig;
        const __half2 lo = __floats2half2_rn(fmaxf(h[j][0], 0.f), fmaxf(h[j][1], 0.f));
        const __half2 hi = __floats2half2_rn(fmaxf(h[j][2], 0.f), fmaxf(h[j][3], 0.f));
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (__half2float(__float2half_rn(h[j][e])) > 0.f) m1 |= 1u << (4 * j + e);
        *reinterpret_cast<__half2*>(S.a1 + r0 * kAhStride + c) = lo;
        *reinterpret_cast<__half2*>(S.a1 + r1 * kAhStride + c) = hi;
        const int s = j >> 1;
        if ((j & 1) == 0) {
          a2f[s][0] = *reinterpret_cast<const uint32_t*>(&lo);
          a2f[s][1] = *reinterpret_cast<const uint32_t*>(&hi);
        } else {
          a2f[s][2] = *reinterpret_cast<const uint32_t*>(&lo);
          a2f[s][3] = *reinterpret_cast<const uint32_t*>(&hi);
        }
      }
    }
    uint32_t a3f[4][4];
    {
      float h[8][4];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        h[j][0] = h[j][1] = h[j][2] = h[j][3] = 0.f;
#pragma unroll
        for (int s = 0; s < 4; s++) {
          const __half* wr = S.w.w2 + (8 * j + g) * kW2Stride + 16 * s + 2 * tig;
          mma16816(h[j], a2f[s], lds32(wr), lds32(wr + 8));
        }
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int c = 8 * j + 2 * tig;
        const __half2 lo = __floats2half2_rn(fmaxf(h[j][0], 0.f), fmaxf(h[j][1], 0.f));
        const __half2 hi = __floats2half2_rn(fmaxf(h[j][2], 0.f), fmaxf(h[j][3], 0.f));
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (__half2float(__float2half_rn(h[j][e])) > 0.f) m2 |= 1u << (4 * j + e);
        *reinterpret_cast<__half2*>(S.a2 + r0 * kAhStride + c) = lo;
        *reinterpret_cast<__half2*>(S.a2 + r1 * kAhStride + c) = hi;
        const int s = j >> 1;
        if ((j & 1) == 0) {
          a3f[s][0] = *reinterpret_cast<const uint32_t*>(&lo);
          a3f[s][1] = *reinterpret_cast<const uint32_t*>(&hi);
        } else {
          a3f[s][2] = *reinterpret_cast<const uint32_t*>(&lo);
          a3f[s][3] = *reinterpret_cast<const uint32_t*>(&hi);
        }
      }
    }
    float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 4; s++) {
      const __half* wr = S.w.w3 + g * kW2Stride + 16 * s + 2 * tig;
      mma16816(y, a3f[s], lds32(wr), lds32(wr + 8));
    }
    // ---- dz3 (rows r0 / r1, cols 2tig, 2tig+1; outputs 0..2), staged for da2 and dW3.
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int64_t px = r ? p1 : p0;
      const bool v = r ? v1 : v0;
      const bool on = v && (!alpha || alpha[px] > 0.f);
#pragma unroll
      for (int cc = 0; cc < 2; cc++) {
        const int col = 2 * tig + cc;
        float d = 0.f;
        if (on && col < 3) {
          const float z = __half2float(__float2half_rn(y[2 * r + cc]));
          const float sg = sigmoidf(z);
          d = grgb[col * npix + px] * (sg * (1.0f - sg));
        }
        S.dz3[(r ? r1 : r0) * kD3Stride + col] = d;
      }
    }
    __syncwarp();
    // ---- dz2 = (dz3 W3) * (z2 > 0): K = 8 (rows 3..7 of W3 are zero).
    {
      uint32_t af[4];
      af[0] = to_tf32(S.dz3[r0 * kD3Stride + tig]);
      af[1] = to_tf32(S.dz3[r1 * kD3Stride + tig]);
      af[2] = to_tf32(S.dz3[r0 * kD3Stride + tig + 4]);
      af[3] = to_tf32(S.dz3[r1 * kD3Stride + tig + 4]);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t b0 = h2tf(S.w.w3[tig * kW2Stride + 8 * j + g]);
        const uint32_t b1 = h2tf(S.w.w3[(tig + 4) * kW2Stride + 8 * j + g]);
        mma1688(d, af, b0, b1);
        const int c = 8 * j + 2 * tig;
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (!((m2 >> (4 * j + e)) & 1u)) d[e] = 0.f;
        S.dz2[r0 * kDzStride + c] = d[0];
        S.dz2[r0 * kDzStride + c + 1] = d[1];
        S.dz2[r1 * kDzStride + c] = d[2];
        S.dz2[r1 * kDzStride + c + 1] = d[3];
      }
    }
    __syncwarp();
    // ---- dz1 = (dz2 W2) * (z1 > 0): K = 64.
    {
      float d[8][4];
#pragma unroll
      for (int j = 0; j < 8; j++) d[j][0] = d[j][1] = d[j][2] = d[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        uint32_t af[4];
        af[0] = to_tf32(S.dz2[r0 * kDzStride + 8 * ks + tig]);
        af[1] = to_tf32(S.dz2[r1 * kDzStride + 8 * ks + tig]);
        af[2] = to_tf32(S.dz2[r0 * kDzStride + 8 * ks + tig + 4]);
        af[3] = to_tf32(S.dz2[r1 * kDzStride + 8 * ks + tig + 4]);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const uint32_t b0 = h2tf(S.w.w2[(8 * ks + tig) * kW2Stride + 8 * j + g]);
          const uint32_t b1 = h2tf(S.w.w2[(8 * ks + tig + 4) * kW2Stride + 8 * j + g]);
          mma1688(d[j], af, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int c = 8 * j + 2 * tig;
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (!((m1 >> (4 * j + e)) & 1u)) d[j][e] = 0.f;
        S.dz1[r0 * kDzStride + c] = d[j][0];
        S.dz1[r0 * kDzStride + c + 1] = d[j][1];
        S.dz1[r1 * kDzStride + c] = d[j][2];
        S.dz1[r1 * kDzStride + c + 1] = d[j][3];
      }
    }
    __syncwarp();
    // ---- dfeat = dz1 W1: K = 64, N = 32.
    {
      float d[4][4];
#pragma unroll
      for (int j = 0; j < 4; j++) d[j][0] = d[j][1] = d[j][2] = d[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        uint32_t af[4];
        af[0] = to_tf32(S.dz1[r0 * kDzStride + 8 * ks + tig]);
        af[1] = to_tf32(S.dz1[r1 * kDzStride + 8 * ks + tig]);
        af[2] = to_tf32(S.dz1[r0 * kDzStride + 8 * ks + tig + 4]);
        af[3] = to_tf32(S.dz1[r1 * kDzStride + 8 * ks + tig + 4]);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const uint32_t b0 = h2tf(S.w.w1[(8 * ks + tig) * kW1Stride + 8 * j + g]);
          const uint32_t b1 = h2tf(S.w.w1[(8 * ks + tig + 4) * kW1Stride + 8 * j + g]);
          mma1688(d[j], af, b0, b1);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int c = 8 * j + 2 * tig;
        if (v0) {
          dfeat[c * npix + p0] = d[j][0];
          dfeat[(c + 1) * npix + p0] = d[j][1];
        }
        if (v1) {
          dfeat[c * npix + p1] = d[j][2];
          dfeat[(c + 1) * npix + p1] = d[j][3];
        }
      }
    }
    __syncthreads();  // the block's dz and activations are staged
    // ---- weight gradients over the block's 64 pixels (K = pixels).
#pragma unroll
    for (int ks = 0; ks < kBwPix / 8; ks++) {
      const int q0 = 8 * ks + tig, q1 = q0 + 4;  // pixel rows of the k-step
      uint32_t af[4];
      // dW2 slice: A = dz2^T rows 16w + (g, g+8)
      af[0] = to_tf32(S.dz2[q0 * kDzStride + 16 * warp + g]);
      af[1] = to_tf32(S.dz2[q0 * kDzStride + 16 * warp + g + 8]);
      af[2] = to_tf32(S.dz2[q1 * kDzStride + 16 * warp + g]);
      af[3] = to_tf32(S.dz2[q1 * kDzStride + 16 * warp + g + 8]);
#pragma unroll
      for (int j = 0; j < 8; j++)
        mma1688(gw2[j], af, h2tf(S.a1[q0 * kAhStride + 8 * j + g]),
                h2tf(S.a1[q1 * kAhStride + 8 * j + g]));
      af[0] = to_tf32(S.dz1[q0 * kDzStride + 16 * warp + g]);
      af[1] = to_tf32(S.dz1[q0 * kDzStride + 16 * warp + g + 8]);
      af[2] = to_tf32(S.dz1[q1 * kDzStride + 16 * warp + g]);
      af[3] = to_tf32(S.dz1[q1 * kDzStride + 16 * warp + g + 8]);
#pragma unroll
      for (int j = 0; j < 4; j++)
        mma1688(gw1[j], af, h2tf(S.xh[q0 * kXhStride + 8 * j + g]),
                h2tf(S.xh[q1 * kXhStride + 8 * j + g]));
      // dW3: A = dz3^T rows 0..15 (columns 8..15 of dz3 do not exist: zero)
      af[0] = to_tf32(S.dz3[q0 * kD3Stride + g]);
      af[1] = 0u;
      af[2] = to_tf32(S.dz3[q1 * kD3Stride + g]);
      af[3] = 0u;
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const int n0 = 8 * (2 * warp + j) + g;
        mma1688(gw3[j], af, h2tf(S.a2[q0 * kAhStride + n0]), h2tf(S.a2[q1 * kAhStride + n0]));
      }
    }
    __syncthreads();  // before the next block overwrites the staging
  }
  // ---- add this CTA's weight gradients (dW laid out as the packed weights).
  float* dW1 = dW;
  float* dW2 = dW + kHid * kIn;
  float* dW3 = dW2 + kHid * kHid;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int row = 16 * warp + g, col = 8 * j + 2 * tig;
    atomicAdd(dW2 + row * kHid + col, gw2[j][0]);
    atomicAdd(dW2 + row * kHid + col + 1, gw2[j][1]);
    atomicAdd(dW2 + (row + 8) * kHid + col, gw2[j][2]);
    atomicAdd(dW2 + (row + 8) * kHid + col + 1, gw2[j][3]);
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int row = 16 * warp + g, col = 8 * j + 2 * tig;
    atomicAdd(dW1 + row * kIn + col, gw1[j][0]);
    atomicAdd(dW1 + row * kIn + col + 1, gw1[j][1]);
    atomicAdd(dW1 + (row + 8) * kIn + col, gw1[j][2]);
    atomicAdd(dW1 + (row + 8) * kIn + col + 1, gw1[j][3]);
  }
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int col = 8 * (2 * warp + j) + 2 * tig;
    if (g < 3) {  // rows g (< 3 valid); rows g + 8 are padding
      atomicAdd(dW3 + g * kHid + col, gw3[j][0]);
      atomicAdd(dW3 + g * kHid + col + 1, gw3[j][1]);
    }
  }
}

}  // namespace

int mlp_backward_launch(const float* feat, int in_dims, int64_t npix, const uint16_t* weights,
                        int hidden, int out_dims, const float* alpha, const float* grgb,
                        float* dfeat, float* dW, cudaStream_t stream) {
  if (in_dims != kIn || hidden != kHid || out_dims != 3) return NS_ERR_UNSUPPORTED;
  if (npix < 0) return NS_ERR_INVALID;
  if (!weights || !dW) return NS_ERR_INVALID;
  const size_t wcount = (size_t)kHid * kIn + (size_t)kHid * kHid + 3 * (size_t)kHid;
  NS_CUDA_TRY(cudaMemsetAsync(dW, 0, wcount * sizeof(float), stream));
  if (npix == 0) return NS_OK;
  if (!feat || !grgb || !dfeat) return NS_ERR_INVALID;
  int dev = 0, sms = 0;
  NS_CUDA_TRY(cudaGetDevice(&dev));
  NS_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int smem = (int)sizeof(MlpBwSmem);
  NS_CUDA_TRY(cudaFuncSetAttribute(mlp_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   smem));
  const int64_t nblocks = div_up64(npix, kBwPix);
  const int grid = (int)min64(nblocks, (int64_t)sms * 2);
  mlp_backward_kernel<<<grid, kBwWarps * 32, smem, stream>>>(feat, npix, weights, alpha, grgb,
                                                            dfeat, dW);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
