// normals.cu -- the allmap decode of a rendered frame (the render_pkg maps) and
// the depth-normal consistency term of training (config 4): pseudo surface
// normal from the expected depth and the per-pixel normal error, forward and
// backward.
//
// Restates, per pixel, the reference's torch code:
//   gaussian_renderer/__init__.py:763-797 (depth_ratio 0): alpha = allmap[1];
//     rend_normal = view-space normal rotated to world (x @ W[:3,:3]^T);
//     expected depth = nan_to_num(allmap[0] / alpha, 0, 0);
//     surf_normal = depth_to_normal(expected depth) * alpha.detach();
//   utils/point_utils.py:10-30, 48-60: points = depth * ray_d + ray_o; interior
//     normal = normalize(cross(p[y+1,x] - p[y-1,x], p[y,x+1] - p[y,x-1])), zero on
//     the one-pixel border;
//   train.py:674-675: normal_error = 1 - sum_c rend_normal * surf_normal.
// The per-pixel rays are given (computed once per camera by the host). Pixels
// whose D / alpha is not finite (alpha == 0: no surfel contributed) take depth
// 0 as nan_to_num gives, and pass no gradient to D or alpha (torch's autograd
// yields 0 / 0 there, which the rasterizer backward never reads: such pixels
// have no contributors).
#include <cfloat>

#include "kernels.cuh"

namespace ns {
namespace {

constexpr int kNormThreads = 256;

struct V3f {
  float x, y, z;
};
__device__ __forceinline__ V3f v3(float x, float y, float z) { return {x, y, z}; }
__device__ __forceinline__ V3f vsub3(V3f a, V3f b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
__device__ __forceinline__ V3f vcross(V3f a, V3f b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
__device__ __forceinline__ float vdot(V3f a, V3f b) { return a.x * b.x + a.y * b.y + a.z * b.z; }

// Expected depth of pixel q: torch.nan_to_num(D / alpha, 0, 0) maps NaN and
// +inf to 0 and -inf to the lowest finite float.
__device__ __forceinline__ float expected_depth(const float* __restrict__ allmap, size_t HW, size_t q) {
  const float d = allmap[q] / allmap[HW + q];
  if (isfinite(d)) return d;
  return (isinf(d) && d < 0.0f) ? -FLT_MAX : 0.0f;
}
__device__ __forceinline__ V3f world_point(const float* __restrict__ allmap, const float* __restrict__ rays_d,
                                           const float* __restrict__ ray_o, size_t HW, size_t q) {
  const float d = expected_depth(allmap, HW, q);
  return v3(d * rays_d[3 * q] + ray_o[0], d * rays_d[3 * q + 1] + ray_o[1], d * rays_d[3 * q + 2] + ray_o[2]);
}

// World-space rendered normal: the view-space allmap normal times W[:3,:3]^T
// as a row vector (viewmatrix column-major: element (i, j) at vm[4 i + j]).
__device__ __forceinline__ V3f world_normal(const float* __restrict__ allmap, const float* __restrict__ vm,
                                            size_t HW, size_t p) {
  const float a = allmap[2 * HW + p], b = allmap[3 * HW + p], c = allmap[4 * HW + p];
  return v3(a * vm[0] + b * vm[1] + c * vm[2], a * vm[4] + b * vm[5] + c * vm[6],
            a * vm[8] + b * vm[9] + c * vm[10]);
}

// Unnormalised stencil normal m = dx x dy of interior pixel (x, y).
__device__ __forceinline__ void stencil(const float* __restrict__ allmap, const float* __restrict__ rays_d,
                                        const float* __restrict__ ray_o, int W, size_t HW, int x, int y,
                                        V3f& dx, V3f& dy) {
  const size_t up = (size_t)(y + 1) * W + x, dn = (size_t)(y - 1) * W + x;
  const size_t rt = (size_t)y * W + x + 1, lf = (size_t)y * W + x - 1;
  dx = vsub3(world_point(allmap, rays_d, ray_o, HW, up), world_point(allmap, rays_d, ray_o, HW, dn));
  dy = vsub3(world_point(allmap, rays_d, ray_o, HW, rt), world_point(allmap, rays_d, ray_o, HW, lf));
}

__global__ void __launch_bounds__(kNormThreads)
normal_error_kernel(const float* __restrict__ allmap, const float* __restrict__ vm,
                    const float* __restrict__ rays_d, const float* __restrict__ ray_o, int W, int H,
                    float* __restrict__ err) {
  const int64_t p = (int64_t)blockIdx.x * kNormThreads + threadIdx.x;
  const size_t HW = (size_t)W * H;
  if (p >= (int64_t)HW) return;
  const int x = (int)(p % W), y = (int)(p / W);
  float e = 1.0f;
  if (x > 0 && x < W - 1 && y > 0 && y < H - 1) {
    V3f dx, dy;
    stencil(allmap, rays_d, ray_o, W, HW, x, y, dx, dy);
    const V3f m = vcross(dx, dy);
    const float inv = 1.0f / fmaxf(sqrtf(vdot(m, m)), 1e-12f);  // F.normalize, eps 1e-12
    const float alpha = allmap[HW + p];
    const V3f sn = v3(m.x * inv * alpha, m.y * inv * alpha, m.z * inv * alpha);
    e = 1.0f - vdot(world_normal(allmap, vm, HW, p), sn);
  }
  err[p] = e;
}

// Backward, step 1 (per pixel p, upstream g = d loss / d err[p]): the rendered
// normal's gradient (allmap channels 2-4) and the stencil gradients d dx, d dy.
__global__ void __launch_bounds__(kNormThreads)
normal_error_bw1_kernel(const float* __restrict__ allmap, const float* __restrict__ vm,
                        const float* __restrict__ rays_d, const float* __restrict__ ray_o, int W,
                        int H, const float* __restrict__ derr, int64_t derr_stride,
                        float* __restrict__ dallmap, float* __restrict__ dstencil) {
  const int64_t p = (int64_t)blockIdx.x * kNormThreads + threadIdx.x;
  const size_t HW = (size_t)W * H;
  if (p >= (int64_t)HW) return;
  const int x = (int)(p % W), y = (int)(p / W);
  const float g = derr[p * derr_stride];
  V3f ddx = v3(0.f, 0.f, 0.f), ddy = ddx, drn = ddx;
  if (x > 0 && x < W - 1 && y > 0 && y < H - 1) {
    V3f dx, dy;
    stencil(allmap, rays_d, ray_o, W, HW, x, y, dx, dy);
    const V3f m = vcross(dx, dy);
    const float len = sqrtf(vdot(m, m));
    const float inv = 1.0f / fmaxf(len, 1e-12f);
    const V3f nh = v3(m.x * inv, m.y * inv, m.z * inv);
    const float alpha = allmap[HW + p];
    const V3f rn = world_normal(allmap, vm, HW, p);
    // err = 1 - rn . (nh * alpha): d rn = -g * nh * alpha; d nh = -g * rn * alpha.
    drn = v3(-g * nh.x * alpha, -g * nh.y * alpha, -g * nh.z * alpha);
    const V3f dnh = v3(-g * rn.x * alpha, -g * rn.y * alpha, -g * rn.z * alpha);
    // nh = m / max(|m|, eps): d m = (d nh - nh (nh . d nh)) / |m| above eps, d nh / eps below.
    V3f dm;
    if (len > 1e-12f) {
      const float pr = vdot(nh, dnh);
      dm = v3((dnh.x - nh.x * pr) * inv, (dnh.y - nh.y * pr) * inv, (dnh.z - nh.z * pr) * inv);
    } else {
      dm = v3(dnh.x * inv, dnh.y * inv, dnh.z * inv);
    }
    // m = dx x dy: d dx = dy x dm, d dy = dm x dx.
    ddx = vcross(dy, dm);
    ddy = vcross(dm, dx);
  }
  // rn = rows of W[:3,:3] applied to the view normal: d view = W[:3,:3]^T-weighted sum.
  dallmap[2 * HW + p] = drn.x * vm[0] + drn.y * vm[4] + drn.z * vm[8];
  dallmap[3 * HW + p] = drn.x * vm[1] + drn.y * vm[5] + drn.z * vm[9];
  dallmap[4 * HW + p] = drn.x * vm[2] + drn.y * vm[6] + drn.z * vm[10];
  float* s = dstencil + p;
  s[0 * HW] = ddx.x;
  s[1 * HW] = ddx.y;
  s[2 * HW] = ddx.z;
  s[3 * HW] = ddy.x;
  s[4 * HW] = ddy.y;
  s[5 * HW] = ddy.z;
}

// Backward, step 2 (per pixel q): gather the stencil gradients of the four
// neighbours that read q's point (dx of (x, y-1) adds it, dx of (x, y+1)
// subtracts it; dy of (x-1, y) adds, dy of (x+1, y) subtracts), then
// point -> expected depth -> allmap channels 0 (D) and 1 (alpha).
__global__ void __launch_bounds__(kNormThreads)
normal_error_bw2_kernel(const float* __restrict__ allmap, const float* __restrict__ rays_d, int W,
                        int H, const float* __restrict__ dstencil, float* __restrict__ dallmap) {
  const int64_t q = (int64_t)blockIdx.x * kNormThreads + threadIdx.x;
  const size_t HW = (size_t)W * H;
  if (q >= (int64_t)HW) return;
  const int x = (int)(q % W), y = (int)(q / W);
  float gx = 0.f, gy = 0.f, gz = 0.f;
  if (y - 1 >= 0) {  // pixel (x, y-1): its dx = p[y] - p[y-2]
    const size_t n = q - W;
    gx += dstencil[0 * HW + n], gy += dstencil[1 * HW + n], gz += dstencil[2 * HW + n];
  }
  if (y + 1 < H) {  // pixel (x, y+1): its dx = p[y+2] - p[y]
    const size_t n = q + W;
    gx -= dstencil[0 * HW + n], gy -= dstencil[1 * HW + n], gz -= dstencil[2 * HW + n];
  }
  if (x - 1 >= 0) {  // pixel (x-1, y): its dy = p[x] - p[x-2]
    const size_t n = q - 1;
    gx += dstencil[3 * HW + n], gy += dstencil[4 * HW + n], gz += dstencil[5 * HW + n];
  }
  if (x + 1 < W) {  // pixel (x+1, y): its dy = p[x+2] - p[x]
    const size_t n = q + 1;
    gx -= dstencil[3 * HW + n], gy -= dstencil[4 * HW + n], gz -= dstencil[5 * HW + n];
  }
  // point = depth * ray_d + ray_o; depth = D / alpha where finite.
  const float ddepth = gx * rays_d[3 * q] + gy * rays_d[3 * q + 1] + gz * rays_d[3 * q + 2];
  const float D = allmap[q], a = allmap[HW + q];
  const float depth = D / a;
  float dD = 0.f, da = 0.f;
  if (isfinite(depth)) {
    dD = ddepth / a;
    da = -ddepth * depth / a;
  }
  dallmap[q] = dD;
  dallmap[HW + q] = da;
}

// nan_to_num(x, 0, 0) of torch: NaN and +inf to 0, -inf to the lowest finite float.
__device__ __forceinline__ float nan_to_num0(float v) {
  if (isfinite(v)) return v;
  return (isinf(v) && v < 0.0f) ? -FLT_MAX : 0.0f;
}

// Surface depth of pixel q (gaussian_renderer/__init__.py:770-786):
// expected * (1 - ratio) + ratio * median.
__device__ __forceinline__ float surf_depth_at(const float* __restrict__ allmap, size_t HW, size_t q,
                                               float one_minus_ratio, float ratio) {
  const float e = expected_depth(allmap, HW, q);
  const float m = nan_to_num0(allmap[5 * HW + q]);
  return e * one_minus_ratio + ratio * m;
}

// The render_pkg maps of one frame from its allmap (gaussian_renderer/__init__.py
// :763-797 and :1035-1045): out channels 0-2 rend_normal (world), 3
// depth_expected, 4 depth_median, 5 surf_depth, 6-8 surf_normal
// (= depth_to_normal(surf_depth) * alpha, zero on the image border).
__global__ void __launch_bounds__(kNormThreads)
allmap_decode_kernel(const float* __restrict__ allmap, const float* __restrict__ vm,
                     const float* __restrict__ rays_d, const float* __restrict__ ray_o, int W, int H,
                     float one_minus_ratio, float ratio, float* __restrict__ out) {
  const int64_t p = (int64_t)blockIdx.x * kNormThreads + threadIdx.x;
  const size_t HW = (size_t)W * H;
  if (p >= (int64_t)HW) return;
  const int x = (int)(p % W), y = (int)(p / W);
  const V3f rn = world_normal(allmap, vm, HW, p);
  out[0 * HW + p] = rn.x;
  out[1 * HW + p] = rn.y;
  out[2 * HW + p] = rn.z;
  out[3 * HW + p] = expected_depth(allmap, HW, p);
  out[4 * HW + p] = nan_to_num0(allmap[5 * HW + p]);
  out[5 * HW + p] = surf_depth_at(allmap, HW, p, one_minus_ratio, ratio);
  V3f sn = v3(0.f, 0.f, 0.f);
  if (x > 0 && x < W - 1 && y > 0 && y < H - 1) {
    auto point = [&](size_t q) {
      const float d = surf_depth_at(allmap, HW, q, one_minus_ratio, ratio);
      return v3(d * rays_d[3 * q] + ray_o[0], d * rays_d[3 * q + 1] + ray_o[1],
                d * rays_d[3 * q + 2] + ray_o[2]);
    };
    const V3f dx = vsub3(point((size_t)(y + 1) * W + x), point((size_t)(y - 1) * W + x));
    const V3f dy = vsub3(point((size_t)y * W + x + 1), point((size_t)y * W + x - 1));
    const V3f m = vcross(dx, dy);
    const float inv = 1.0f / fmaxf(sqrtf(vdot(m, m)), 1e-12f);
    const float alpha = allmap[HW + p];
    sn = v3(m.x * inv * alpha, m.y * inv * alpha, m.z * inv * alpha);
  }
  out[6 * HW + p] = sn.x;
  out[7 * HW + p] = sn.y;
  out[8 * HW + p] = sn.z;
}

}  // namespace

int allmap_decode_launch(const float* allmap, const float* vm, const float* rays_d,
                         const float* ray_o, int W, int H, float depth_ratio, float* out,
                         cudaStream_t stream) {
  const int64_t HW = (int64_t)W * H;
  if (HW <= 0) return NS_OK;
  allmap_decode_kernel<<<(unsigned)div_up64(HW, kNormThreads), kNormThreads, 0, stream>>>(
      allmap, vm, rays_d, ray_o, W, H, 1.0f - depth_ratio, depth_ratio, out);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int normal_error_launch(const float* allmap, const float* vm, const float* rays_d,
                        const float* ray_o, int W, int H, float* err, cudaStream_t stream) {
  const int64_t HW = (int64_t)W * H;
  if (HW <= 0) return NS_OK;
  normal_error_kernel<<<(unsigned)div_up64(HW, kNormThreads), kNormThreads, 0, stream>>>(
      allmap, vm, rays_d, ray_o, W, H, err);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int normal_error_backward_launch(const float* allmap, const float* vm, const float* rays_d,
                                 const float* ray_o, int W, int H, const float* derr,
                                 int64_t derr_stride, float* dallmap, float* dstencil,
                                 cudaStream_t stream) {
  const int64_t HW = (int64_t)W * H;
  if (HW <= 0) return NS_OK;
  const unsigned blocks = (unsigned)div_up64(HW, kNormThreads);
  normal_error_bw1_kernel<<<blocks, kNormThreads, 0, stream>>>(
      allmap, vm, rays_d, ray_o, W, H, derr, derr_stride, dallmap, dstencil);
  NS_LAUNCH_CHECK();
  normal_error_bw2_kernel<<<blocks, kNormThreads, 0, stream>>>(allmap, rays_d, W, H, dstencil,
                                                               dallmap);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
