// sh.cu -- view-dependent surfel colours from spherical harmonics, for the
// rasterizer's level-0 path when it is given SH coefficients instead of
// precomputed colours (the reference's warm-up renders, before the hash grid).
//
// Restates computeColorFromSH (forward.cu:21-74, called by preprocessCUDA at
// :414-423) and its backward (backward.cu:21-140 with dnormvdv,
// auxiliary.h:133-143, called by the preprocess backward at :2266-2267): the
// degree-`deg` real SH basis (the standard normalisation constants of the 3D
// Gaussian splatting colour model) along the unit direction from the camera
// centre to the surfel's mean, + 0.5, clamped at 0; the gradient is cut where
// the clamp acted and reaches the mean through the direction's normalisation.
// The coefficients are M RGB triples per surfel (coefficient k at 3 k).
//
// One thread per surfel; each reads its own 3 M coefficients (a 192-byte row
// for M = 16, whole L2 lines). The backward recomputes the clamp instead of
// storing it.
#include "kernels.cuh"

namespace ns {
namespace {

constexpr float kC0 = 0.28209479177387814f, kC1 = 0.4886025119029199f;
__constant__ float kC2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                             -1.0925484305920792f, 0.5462742152960396f};
__constant__ float kC3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                             0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                             -0.5900435899266435f};

__device__ __forceinline__ float3 view_dir(const float* __restrict__ means, const float* __restrict__ campos,
                                           int i, float3& d0) {
  d0 = f3(means[3 * i] - campos[0], means[3 * i + 1] - campos[1], means[3 * i + 2] - campos[2]);
  const float len = sqrtf(d0.x * d0.x + d0.y * d0.y + d0.z * d0.z);
  return f3(d0.x / len, d0.y / len, d0.z / len);
}

// The colour channel c of one surfel before the clamp (forward.cu:30-66, + 0.5).
__device__ __forceinline__ float sh_channel(int deg, const float* __restrict__ sh, float3 d, int c) {
  auto k = [&](int i) { return __ldg(sh + 3 * i + c); };
  const float x = d.x, y = d.y, z = d.z;
  float r = kC0 * k(0);
  if (deg > 0) {
    r = r - kC1 * y * k(1) + kC1 * z * k(2) - kC1 * x * k(3);
    if (deg > 1) {
      const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
      r = r + kC2[0] * xy * k(4) + kC2[1] * yz * k(5) + kC2[2] * (2.0f * zz - xx - yy) * k(6) +
          kC2[3] * xz * k(7) + kC2[4] * (xx - yy) * k(8);
      if (deg > 2)
        r = r + kC3[0] * y * (3.0f * xx - yy) * k(9) + kC3[1] * xy * z * k(10) +
            kC3[2] * y * (4.0f * zz - xx - yy) * k(11) + kC3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy) * k(12) +
            kC3[4] * x * (4.0f * zz - xx - yy) * k(13) + kC3[5] * z * (xx - yy) * k(14) +
            kC3[6] * x * (xx - 3.0f * yy) * k(15);
    }
  }
  return r + 0.5f;
}

__global__ void __launch_bounds__(256) sh_color_kernel(int P, int deg, int M, const float* __restrict__ means,
                                                       const float* __restrict__ campos,
                                                       const float* __restrict__ shs, float* __restrict__ rgb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  float3 d0;
  const float3 d = view_dir(means, campos, i, d0);
  const float* sh = shs + (size_t)i * M * 3;
#pragma unroll
  for (int c = 0; c < 3; c++) rgb[3 * (size_t)i + c] = fmaxf(sh_channel(deg, sh, d, c), 0.0f);
}

__global__ void __launch_bounds__(256)
    sh_color_backward_kernel(int P, int deg, int M, const float* __restrict__ means, const float* __restrict__ campos,
                             const float* __restrict__ shs, const int32_t* __restrict__ radii,
                             const float* __restrict__ dL_drgb, float* __restrict__ dL_dshs,
                             float* __restrict__ dL_dmeans) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  float* dsh = dL_dshs + (size_t)i * M * 3;
  if (!(radii[i] > 0)) {
    for (int j = 0; j < 3 * M; j++) dsh[j] = 0.0f;
    return;
  }
  float3 d0;
  const float3 d = view_dir(means, campos, i, d0);
  const float* sh = shs + (size_t)i * M * 3;
  float g[3];
#pragma unroll
  for (int c = 0; c < 3; c++) g[c] = sh_channel(deg, sh, d, c) < 0.0f ? 0.0f : dL_drgb[3 * (size_t)i + c];
  for (int j = 0; j < 3 * M; j++) dsh[j] = 0.0f;
  auto put = [&](int k, float b) {
#pragma unroll
    for (int c = 0; c < 3; c++) dsh[3 * k + c] = b * g[c];
  };
  auto s = [&](int k, int c) { return __ldg(sh + 3 * k + c); };
  const float x = d.x, y = d.y, z = d.z;
  float dx[3] = {0.f, 0.f, 0.f}, dy[3] = {0.f, 0.f, 0.f}, dz[3] = {0.f, 0.f, 0.f};
  put(0, kC0);
  if (deg > 0) {
    put(1, -kC1 * y);
    put(2, kC1 * z);
    put(3, -kC1 * x);
#pragma unroll
    for (int c = 0; c < 3; c++) {
      dx[c] = -kC1 * s(3, c);
      dy[c] = -kC1 * s(1, c);
      dz[c] = kC1 * s(2, c);
    }
    if (deg > 1) {
      const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
      put(4, kC2[0] * xy);
      put(5, kC2[1] * yz);
      put(6, kC2[2] * (2.f * zz - xx - yy));
      put(7, kC2[3] * xz);
      put(8, kC2[4] * (xx - yy));
#pragma unroll
      for (int c = 0; c < 3; c++) {
        dx[c] += kC2[0] * y * s(4, c) + kC2[2] * 2.f * -x * s(6, c) + kC2[3] * z * s(7, c) +
                 kC2[4] * 2.f * x * s(8, c);
        dy[c] += kC2[0] * x * s(4, c) + kC2[1] * z * s(5, c) + kC2[2] * 2.f * -y * s(6, c) +
                 kC2[4] * 2.f * -y * s(8, c);
        dz[c] += kC2[1] * y * s(5, c) + kC2[2] * 2.f * 2.f * z * s(6, c) + kC2[3] * x * s(7, c);
      }
      if (deg > 2) {
        put(9, kC3[0] * y * (3.f * xx - yy));
        put(10, kC3[1] * xy * z);
        put(11, kC3[2] * y * (4.f * zz - xx - yy));
        put(12, kC3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy));
        put(13, kC3[4] * x * (4.f * zz - xx - yy));
        put(14, kC3[5] * z * (xx - yy));
        put(15, kC3[6] * x * (xx - 3.f * yy));
#pragma unroll
        for (int c = 0; c < 3; c++) {
          dx[c] += kC3[0] * s(9, c) * 3.f * 2.f * xy + kC3[1] * s(10, c) * yz + kC3[2] * s(11, c) * -2.f * xy +
                   kC3[3] * s(12, c) * -3.f * 2.f * xz + kC3[4] * s(13, c) * (-3.f * xx + 4.f * zz - yy) +
                   kC3[5] * s(14, c) * 2.f * xz + kC3[6] * s(15, c) * 3.f * (xx - yy);
          dy[c] += kC3[0] * s(9, c) * 3.f * (xx - yy) + kC3[1] * s(10, c) * xz +
                   kC3[2] * s(11, c) * (-3.f * yy + 4.f * zz - xx) + kC3[3] * s(12, c) * -3.f * 2.f * yz +
                   kC3[4] * s(13, c) * -2.f * xy + kC3[5] * s(14, c) * -2.f * yz +
                   kC3[6] * s(15, c) * -3.f * 2.f * xy;
          dz[c] += kC3[1] * s(10, c) * xy + kC3[2] * s(11, c) * 4.f * 2.f * yz +
                   kC3[3] * s(12, c) * 3.f * (2.f * zz - xx - yy) + kC3[4] * s(13, c) * 4.f * 2.f * xz +
                   kC3[5] * s(14, c) * (xx - yy);
        }
      }
    }
  }
  // dL/d(unit direction), then through the normalisation to the mean.
  const float ddx = dx[0] * g[0] + dx[1] * g[1] + dx[2] * g[2];
  const float ddy = dy[0] * g[0] + dy[1] * g[1] + dy[2] * g[2];
  const float ddz = dz[0] * g[0] + dz[1] * g[1] + dz[2] * g[2];
  const float sum2 = d0.x * d0.x + d0.y * d0.y + d0.z * d0.z;
  const float inv32 = 1.0f / sqrtf(sum2 * sum2 * sum2);
  float* dm = dL_dmeans + 3 * (size_t)i;
  dm[0] += ((sum2 - d0.x * d0.x) * ddx - d0.y * d0.x * ddy - d0.z * d0.x * ddz) * inv32;
  dm[1] += (-d0.x * d0.y * ddx + (sum2 - d0.y * d0.y) * ddy - d0.z * d0.y * ddz) * inv32;
  dm[2] += (-d0.x * d0.z * ddx - d0.y * d0.z * ddy + (sum2 - d0.z * d0.z) * ddz) * inv32;
}

}  // namespace

int sh_color_launch(int P, int deg, int M, const float* means, const float* campos, const float* shs, float* rgb,
                    cudaStream_t stream) {
  if (P <= 0) return NS_OK;
  sh_color_kernel<<<div_up(P, 256), 256, 0, stream>>>(P, deg, M, means, campos, shs, rgb);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int sh_color_backward_launch(int P, int deg, int M, const float* means, const float* campos, const float* shs,
                             const int32_t* radii, const float* dL_drgb, float* dL_dshs, float* dL_dmeans,
                             cudaStream_t stream) {
  if (P <= 0) return NS_OK;
  sh_color_backward_kernel<<<div_up(P, 256), 256, 0, stream>>>(P, deg, M, means, campos, shs, radii, dL_drgb,
                                                                dL_dshs, dL_dmeans);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
