// gridencode.cu -- the multiresolution hash-grid encoding as a standalone op:
// the reference's gridencoder extension (gridencoder/src/gridencoder.cu) on
// the lookup code of the blend kernel.
//
// ns_grid_encode_forward restates kernel_grid (gridencoder.cu:88-242): per
// point and level, the trilinear lookup of the level's table slice (outputs
// [L, B, 2]) and, optionally, d output / d input (dy_dx [B, L, 3, 2]).
// ns_grid_encode_backward restates kernel_grid_backward (:246-338: the table
// gradient, one float2 atomic per corner) and kernel_input_backward (:341-367:
// dL/dx from dy_dx). The lookup is lookup_issue / lookup_finish of
// hashgrid.cuh, the same code the blend kernel runs per blended sample, so a
// check of these entry points against the reference's kernels checks the
// blend's lookups too. The rasterizer's query_feature (hashgrid.h:53-299) runs
// the same per-level arithmetic.
//
// Layout: one thread per (point, level), CTAs of 256 points of one level
// (blockIdx.y = level), as the reference launches it: a CTA's lookups share one
// level's table slice, consecutive threads write consecutive float2 outputs.
#include "hashgrid.cuh"
#include "kernels.cuh"

namespace ns {
namespace {

constexpr int kGridThreads = 256;

__device__ __forceinline__ bool outside_unit_box(const float* x) {
  return x[0] < 0 || x[0] > 1 || x[1] < 0 || x[1] > 1 || x[2] < 0 || x[2] > 1;
}

// Position of the point in the level's grid: cell g, fraction f (smoothstep
// applied for interp 1) and the derivative of f (gridencoder.cu:145-158).
__device__ __forceinline__ void cell_of(const LevelConst& lc, const float* x, float shift,
                                        uint32_t interp, uint32_t (&g)[3], float (&f)[3],
                                        float (&df)[3]) {
#pragma unroll
  for (int d = 0; d < 3; d++) {
    const float pos = x[d] * lc.scale + shift;
    const float fl = floorf(pos);
    g[d] = (uint32_t)fl;
    f[d] = pos - fl;
    if (interp == 1) {
      df[d] = 6 * f[d] * (1.0f - f[d]);
      f[d] = f[d] * f[d] * (3.0f - 2.0f * f[d]);
    } else {
      df[d] = 1.0f;
    }
  }
}

template <typename TableT>
__global__ void __launch_bounds__(kGridThreads) grid_forward_kernel(
    const float* __restrict__ inputs, const void* __restrict__ table, const int32_t* __restrict__ offsets,
    float* __restrict__ outputs, uint32_t B, uint32_t L, float S, uint32_t H, float* __restrict__ dy_dx,
    int align_corners, uint32_t interp) {
  const uint32_t b = blockIdx.x * kGridThreads + threadIdx.x;
  if (b >= B) return;
  const int l = blockIdx.y;
  const float x[3] = {inputs[3 * (size_t)b], inputs[3 * (size_t)b + 1], inputs[3 * (size_t)b + 2]};
  float2* out = reinterpret_cast<float2*>(outputs) + (size_t)l * B + b;
  float2* dyd = dy_dx ? reinterpret_cast<float2*>(dy_dx) + ((size_t)b * L + l) * 3 : nullptr;
  if (outside_unit_box(x)) {
    *out = make_float2(0.f, 0.f);
    if (dyd)
      for (int d = 0; d < 3; d++) dyd[d] = make_float2(0.f, 0.f);
    return;
  }
  const LevelConst lc = make_level<TableT>(table, offsets, S, H, align_corners, l);
  const float shift = align_corners ? 0.0f : 0.5f;
  float f[3];
  Corner8<TableT> cv;
  lookup_issue<TableT>(lc, table, make_float4(x[0], x[1], x[2], 0.f), shift, interp, f, cv);
  *out = lookup_finish<TableT>(f, cv);
  if (!dyd) return;
  // d out / d x_gd (gridencoder.cu:203-240): the 4 edges along gd, weighted by
  // scale and the other two axes' corner weights (in axis order), times the
  // smoothstep derivative.
  uint32_t g[3];
  float ff[3], df[3];
  cell_of(lc, x, shift, interp, g, ff, df);
#pragma unroll
  for (int gd = 0; gd < 3; gd++) {
    const int da = gd == 0 ? 1 : 0, db = gd == 2 ? 1 : 2;  // the other two axes, in order
    float2 rg = make_float2(0.f, 0.f);
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int ba = e & 1, bb = e >> 1;
      float w = lc.scale;
      w *= ba ? ff[da] : 1 - ff[da];
      w *= bb ? ff[db] : 1 - ff[db];
      const int c0 = (ba << da) | (bb << db);  // corner with bit gd clear
      const float2 lo = cv.get(c0), hi = cv.get(c0 | (1 << gd));
      rg.x = fmaf(w * (hi.x - lo.x), df[gd], rg.x);
      rg.y = fmaf(w * (hi.y - lo.y), df[gd], rg.y);
    }
    dyd[gd] = rg;
  }
}

template <typename TableT>
__global__ void __launch_bounds__(kGridThreads) grid_backward_kernel(
    const float* __restrict__ grad, const float* __restrict__ inputs, const void* __restrict__ table,
    const int32_t* __restrict__ offsets, float* __restrict__ grad_table, uint32_t B, float S, uint32_t H,
    int align_corners, uint32_t interp) {
  const uint32_t b = blockIdx.x * kGridThreads + threadIdx.x;
  if (b >= B) return;
  const int l = blockIdx.y;
  const float x[3] = {inputs[3 * (size_t)b], inputs[3 * (size_t)b + 1], inputs[3 * (size_t)b + 2]};
  if (outside_unit_box(x)) return;  // no gradient (gridencoder.cu:272-276)
  const LevelConst lc = make_level<TableT>(table, offsets, S, H, align_corners, l);
  uint32_t g[3], idx[8];
  float f[3], df[3];
  cell_of(lc, x, align_corners ? 0.0f : 0.5f, interp, g, f, df);
  corner_rows(lc, g, idx);
  const float2 gr = reinterpret_cast<const float2*>(grad)[(size_t)l * B + b];
  float2* dt = reinterpret_cast<float2*>(grad_table) + lc.row0;
#pragma unroll
  for (int c = 0; c < 8; c++) {
    const float w = ((c & 1 ? f[0] : 1 - f[0]) * (c & 2 ? f[1] : 1 - f[1])) * (c & 4 ? f[2] : 1 - f[2]);
    atomicAdd(dt + idx[c], make_float2(w * gr.x, w * gr.y));
  }
}

// dL/dx[b, d] = sum over levels, then channels, of grad[l, b, ch] * dy_dx[b, l, d, ch].
__global__ void __launch_bounds__(kGridThreads) grid_input_backward_kernel(
    const float* __restrict__ grad, const float* __restrict__ dy_dx, float* __restrict__ grad_inputs,
    uint32_t B, uint32_t L) {
  const uint32_t t = blockIdx.x * kGridThreads + threadIdx.x;
  if (t >= B * 3) return;
  const uint32_t b = t / 3, d = t - b * 3;
  float r = 0.f;
  for (uint32_t l = 0; l < L; l++) {
    const float2 gr = reinterpret_cast<const float2*>(grad)[(size_t)l * B + b];
    const float2 dy = reinterpret_cast<const float2*>(dy_dx)[((size_t)b * L + l) * 3 + d];
    r = fmaf(gr.x, dy.x, r);
    r = fmaf(gr.y, dy.y, r);
  }
  grad_inputs[t] = r;
}

int check_shape(uint32_t D, uint32_t C, uint32_t L, uint32_t gridtype) {
  if (D != 3 || C != 2 || gridtype != 0) return NS_ERR_UNSUPPORTED;
  if (L == 0 || L > 65535) return NS_ERR_INVALID;
  return NS_OK;
}

}  // namespace
}  // namespace ns

extern "C" int ns_grid_encode_forward(const float* inputs, const void* embeddings, int32_t embeddings_fp16,
                                      const int32_t* offsets, float* outputs, uint32_t B, uint32_t D,
                                      uint32_t C, uint32_t L, float S, uint32_t H, float* dy_dx,
                                      uint32_t gridtype, int32_t align_corners, uint32_t interp,
                                      void* stream_) {
  using namespace ns;
  int rc = check_shape(D, C, L, gridtype);
  if (rc) return rc;
  if (B == 0) return NS_OK;
  if (!inputs || !embeddings || !offsets || !outputs || interp > 1 || B > (1u << 31) / 3)
    return NS_ERR_INVALID;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const dim3 grid((B + kGridThreads - 1) / kGridThreads, L);
  if (embeddings_fp16)
    grid_forward_kernel<__half><<<grid, kGridThreads, 0, stream>>>(inputs, embeddings, offsets, outputs, B, L, S,
                                                                   H, dy_dx, align_corners, interp);
  else
    grid_forward_kernel<float><<<grid, kGridThreads, 0, stream>>>(inputs, embeddings, offsets, outputs, B, L, S,
                                                                  H, dy_dx, align_corners, interp);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

extern "C" int ns_grid_encode_backward(const float* grad, const float* inputs, const void* embeddings,
                                       int32_t embeddings_fp16, const int32_t* offsets, float* grad_embeddings,
                                       uint32_t B, uint32_t D, uint32_t C, uint32_t L, float S, uint32_t H,
                                       const float* dy_dx, float* grad_inputs, uint32_t gridtype,
                                       int32_t align_corners, uint32_t interp, void* stream_) {
  using namespace ns;
  int rc = check_shape(D, C, L, gridtype);
  if (rc) return rc;
  if (B == 0) return NS_OK;
  if (!grad || !inputs || !embeddings || !offsets || !grad_embeddings || interp > 1 || B > (1u << 31) / 3)
    return NS_ERR_INVALID;
  if (grad_inputs && !dy_dx) return NS_ERR_INVALID;  // dL/dx is formed from the forward's dy_dx
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const dim3 grid((B + kGridThreads - 1) / kGridThreads, L);
  if (embeddings_fp16)
    grid_backward_kernel<__half><<<grid, kGridThreads, 0, stream>>>(grad, inputs, embeddings, offsets,
                                                                    grad_embeddings, B, S, H, align_corners,
                                                                    interp);
  else
    grid_backward_kernel<float><<<grid, kGridThreads, 0, stream>>>(grad, inputs, embeddings, offsets,
                                                                   grad_embeddings, B, S, H, align_corners,
                                                                   interp);
  NS_LAUNCH_CHECK();
  if (grad_inputs) {
    grid_input_backward_kernel<<<(B * 3 + kGridThreads - 1) / kGridThreads, kGridThreads, 0, stream>>>(
        grad, dy_dx, grad_inputs, B, L);
    NS_LAUNCH_CHECK();
  }
  return NS_OK;
}
