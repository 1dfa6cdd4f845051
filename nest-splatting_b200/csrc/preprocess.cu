// preprocess.cu -- per-surfel preprocess: cull, splat-to-pixel transform, normal,
// screen bounding box, tile count, and the 128-byte render record.
//
// Restates forward.cu:323-441 (preprocessCUDA), :237-290 (compute_transmat),
// :294-320 (compute_aabb) and auxiliary.h:190-240 (in_frustum, quat_to_rotmat)
// of the reference's diff-surfel-rasterization, for render_mode 0. The SH colour
// evaluation of preprocessCUDA is not done: mode 0 never reads it.
//
// Two attribute sources share one body:
//   * ApiAttrs: activated tensors as the rasterizer API receives them, plus the
//     optional homotrans [P,16] (general_utils.py:101-113 build_H);
//   * MixAttrs: the fused RVQ frame, raw = base + mix * decoded[:, 0:10], then the
//     activations of gaussian_model.py:231-281 (exp scale, normalised quaternion,
//     sigmoid opacity) and build_H, computed here instead of in torch.
// The block also writes each surfel's exclusive tile offset within its CTA and
// the CTA total, so binning needs only a tiny scan of per-CTA totals.
#include "common.cuh"

namespace ns {
namespace {

constexpr int kPreThreads = 256;

struct SurfelIn {
  float3 p;      // mean
  float2 s;      // activated scale (before scale_modifier)
  float4 q;      // rotation quaternion (w, x, y, z) as given to quat_to_rotmat
  float opacity;
  float3 su, sv, pk;  // homotrans columns 0, 1 and translation
  float ap;
  float shape;        // kernel parameter (kernel types 1-3)
  bool given_T;       // precomputed transform (Tu, Tv, Tw below), scale / rotation unused
  float3 Tu, Tv, Tw;
};

struct ApiAttrs {
  const float* means3D;
  const float* scales;
  const float* rotations;
  const float* opacities;
  const float* homotrans;
  const float* ap_level;
  const float* shapes;
  const float* transmats;  // [P, 9] precomputed transforms, or NULL (then scales / rotations are read)
  __device__ SurfelIn load(int i) const {
    SurfelIn a;
    a.shape = shapes ? shapes[i] : 0.0f;
    a.p = f3(means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]);
    a.given_T = transmats != nullptr;
    if (a.given_T) {
      const float* t = transmats + 9 * (size_t)i;
      a.Tu = f3(t[0], t[1], t[2]);
      a.Tv = f3(t[3], t[4], t[5]);
      a.Tw = f3(t[6], t[7], t[8]);
      a.s = make_float2(0.f, 0.f);
      a.q = make_float4(1.f, 0.f, 0.f, 0.f);
    } else {
      a.s = make_float2(scales[2 * i], scales[2 * i + 1]);
      a.q = make_float4(rotations[4 * i], rotations[4 * i + 1], rotations[4 * i + 2], rotations[4 * i + 3]);
    }
    a.opacity = opacities[i];
    if (homotrans) {
      const float* h = homotrans + 16 * (size_t)i;
      a.su = f3(h[0], h[4], h[8]);
      a.sv = f3(h[1], h[5], h[9]);
      a.pk = f3(h[3], h[7], h[11]);
    } else {
      // build_rotation (general_utils.py:78-99) on the given quaternion, then
      // build_H: columns 0/1 of R scaled by the two scales, translation = mean.
      const float nrm = sqrtf(a.q.x * a.q.x + a.q.y * a.q.y + a.q.z * a.q.z + a.q.w * a.q.w);
      const float r = a.q.x / nrm, x = a.q.y / nrm, y = a.q.z / nrm, z = a.q.w / nrm;
      a.su = f3((1 - 2 * (y * y + z * z)) * a.s.x, (2 * (x * y + r * z)) * a.s.x,
                (2 * (x * z - r * y)) * a.s.x);
      a.sv = f3((2 * (x * y - r * z)) * a.s.y, (1 - 2 * (x * x + z * z)) * a.s.y,
                (2 * (y * z + r * x)) * a.s.y);
      a.pk = a.p;
    }
    a.ap = ap_level ? ap_level[i] : 1e9f;
    return a;
  }
};

struct MixAttrs {
  const float* base;     // [P,10]
  const float* decoded;  // [P,dims]
  int dims;
  float mix;
  const float* ap_level;
  __device__ SurfelIn load(int i) const {
    const float* b = base + 10 * (size_t)i;
    const float* d = decoded + (size_t)dims * i;
    float raw[10];
    SurfelIn a;
    a.shape = 0.0f;
    a.given_T = false;
#pragma unroll
    for (int k = 0; k < 10; k++) raw[k] = b[k] + mix * d[k];
    a.p = f3(raw[0], raw[1], raw[2]);
    a.s = make_float2(expf(raw[3]), expf(raw[4]));
    // torch.nn.functional.normalize: q / max(|q|, 1e-12)
    const float qn = fmaxf(sqrtf(raw[5] * raw[5] + raw[6] * raw[6] + raw[7] * raw[7] +
                                 raw[8] * raw[8]), 1e-12f);
    a.q = make_float4(raw[5] / qn, raw[6] / qn, raw[7] / qn, raw[8] / qn);
    a.opacity = 1.0f / (1.0f + expf(-raw[9]));
    // build_rotation on the raw quaternion (it normalises again) and build_H.
    const float nrm = sqrtf(raw[5] * raw[5] + raw[6] * raw[6] + raw[7] * raw[7] + raw[8] * raw[8]);
    const float r = raw[5] / nrm, x = raw[6] / nrm, y = raw[7] / nrm, z = raw[8] / nrm;
    a.su = f3((1 - 2 * (y * y + z * z)) * a.s.x, (2 * (x * y + r * z)) * a.s.x,
              (2 * (x * z - r * y)) * a.s.x);
    a.sv = f3((2 * (x * y - r * z)) * a.s.y, (1 - 2 * (x * x + z * z)) * a.s.y,
              (2 * (y * z + r * x)) * a.s.y);
    a.pk = a.p;
    a.ap = ap_level ? ap_level[i] : 1e9f;
    return a;
  }
};

struct PreOut {
  SurfelRecord* records;
  BinInfo* bin;
  int32_t* radii;
  uint32_t* tiles;       // tiles touched
  uint32_t* depth_keys;  // float bits of the view depth (all ones when no tile is touched)
  uint32_t* depth_vals;  // surfel index
  uint32_t* block_sums;  // per-CTA total of the tile counts
};

// Squared radius rho (in the units of the blend kernel's rho = min(rho3d, rho2d))
// beyond which alpha = min(0.99, o * G(rho)) < 1/255 (forward.cu:864-919):
//   kernel 0: G = exp(-rho/2), or for beta > 0 (1+beta) G / (1 + beta G);
//   kernel 1: G = (1 - rho)^shape on rho < 1;   kernel 2: as 0 with beta = shape;
//   kernel 3: G = exp(-0.5 max(rho, 1e-8)^(shape/2)).
// Returns false when no rho reaches 1/255; rho_cut = +inf when G does not fall
// with rho (kernel 3 with shape <= 0). A relative margin keeps the bound
// conservative under float rounding.
__device__ __forceinline__ bool alpha_cutoff(float o, float beta, int kernel_type, float shape,
                                             float& rho_cut) {
  if (!(o > 0.0f)) return false;
  const double a = 1.0 / (255.0 * (double)o);  // G needed
  if (kernel_type == 1) {
    if (!(shape > 0.0f)) {  // G >= 1 everywhere on rho < 1
      rho_cut = 1.0f;
      return true;
    }
    if (a > 1.001) return false;
    const double rc = 1.0 - pow(a < 1.0 ? a : 1.0, 1.0 / (double)shape);
    rho_cut = (float)fmin(rc * 1.002 + 1e-3, 1.0);
    return true;
  }
  if (kernel_type == 3) {
    if (!(shape > 0.0f)) {
      rho_cut = __int_as_float(0x7f800000);  // +inf
      return true;
    }
    if (a > 1.001) return false;
    const double lg = a >= 1.0 ? 0.0 : -2.0 * log(a);  // rho^(shape/2) <= 2 ln(255 o)
    const double rc = pow(lg, 2.0 / (double)shape);
    rho_cut = (float)(rc * 1.002 + 1e-3);
    return true;
  }
  if (kernel_type == 2) beta = shape > 0.0f ? shape : 0.0f;
  if (a > 1.001) return false;
  double g = a;
  if (beta > 0.0f) g = a / (1.0 + beta - beta * a);  // invert G' = (1+b) G / (1 + b G)
  const double rc = g >= 1.0 ? 0.0 : -2.0 * log(g);
  rho_cut = (float)(rc * 1.002 + 1e-3);
  return true;
}

// Returns the number of tiles that receive instances (0 when culled) and fills
// the record, the binning info and the reference's radius.
__device__ __forceinline__ uint32_t preprocess_one(const SurfelIn& a, float mod, float beta,
                                                   int kernel_type, const float* vm, const float* pm,
                                                   int W, int H, int gx, int gy, SurfelRecord& rec,
                                                   BinInfo& bi, int& radius_out) {
  // in_frustum: view-space depth must exceed 0.2 (auxiliary.h:190-215).
  const float3 pv = f3(vm[0] * a.p.x + vm[4] * a.p.y + vm[8] * a.p.z + vm[12],
                       vm[1] * a.p.x + vm[5] * a.p.y + vm[9] * a.p.z + vm[13],
                       vm[2] * a.p.x + vm[6] * a.p.y + vm[10] * a.p.z + vm[14]);
  if (pv.z <= 0.2f) return 0;

  float3 Tu, Tv, Tw, n;
  if (a.given_T) {
    // precomputed transform (forward.cu:366-380): the normal is the view axis
    Tu = a.Tu;
    Tv = a.Tv;
    Tw = a.Tw;
    n = f3(0.f, 0.f, 1.f);
  } else {
  // quat_to_rotmat (rsqrt-normalised) -> L = R * diag(mod*s.x, mod*s.y, 1).
  const float qs = rsqrtf(a.q.w * a.q.w + a.q.x * a.q.x + a.q.y * a.q.y + a.q.z * a.q.z);
  const float w = a.q.x * qs, x = a.q.y * qs, y = a.q.z * qs, z = a.q.w * qs;
  const float sx = mod * a.s.x, sy = mod * a.s.y;
  const float3 L0 = sx * f3(1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z), 2.f * (x * z - w * y));
  const float3 L1 = sy * f3(2.f * (x * y - w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x));
  const float3 L2 = f3(2.f * (x * z + w * y), 2.f * (y * z - w * x), 1.f - 2.f * (x * x + y * y));

  // T = splat2world^T * world2ndc * ndc2pix: row r of the 3x4 homogeneous
  // projections of the basis (L0, 0), (L1, 0), (p, 1).
  const float b[3][4] = {{L0.x, L0.y, L0.z, 0.f}, {L1.x, L1.y, L1.z, 0.f}, {a.p.x, a.p.y, a.p.z, 1.f}};
  float Q[4][3];
#pragma unroll
  for (int c = 0; c < 4; c++)
#pragma unroll
    for (int r = 0; r < 3; r++)
      Q[c][r] = b[r][0] * pm[c] + b[r][1] * pm[4 + c] + b[r][2] * pm[8 + c] + b[r][3] * pm[12 + c];
  const float hw = float(W) / 2.0f, hh = float(H) / 2.0f;
  const float cw = float(W - 1) / 2.0f, ch = float(H - 1) / 2.0f;
  Tu = f3(Q[0][0] * hw + Q[3][0] * cw, Q[0][1] * hw + Q[3][1] * cw, Q[0][2] * hw + Q[3][2] * cw);
  Tv = f3(Q[1][0] * hh + Q[3][0] * ch, Q[1][1] * hh + Q[3][1] * ch, Q[1][2] * hh + Q[3][2] * ch);
  Tw = f3(Q[3][0], Q[3][1], Q[3][2]);

  // View-space normal (normalised), flipped to face the camera below.
  n = f3(vm[0] * L2.x + vm[4] * L2.y + vm[8] * L2.z,
         vm[1] * L2.x + vm[5] * L2.y + vm[9] * L2.z,
         vm[2] * L2.x + vm[6] * L2.y + vm[10] * L2.z);
  const float nl = sqrtf(n.x * n.x + n.y * n.y + n.z * n.z);
  if (nl > 1e-7f) {
    n.x /= nl;
    n.y /= nl;
    n.z /= nl;
  }
  }
  const float cosv = -(pv.x * n.x + pv.y * n.y + pv.z * n.z);
  if (cosv == 0) return 0;
  const float mult = cosv > 0 ? 1.f : -1.f;
  n = mult * n;

  // compute_aabb with cutoff 4.
  const float cutoff = 4.0f;
  const float t0 = cutoff * cutoff;
  const float d = t0 * (Tw.x * Tw.x) + t0 * (Tw.y * Tw.y) + -1.0f * (Tw.z * Tw.z);
  if (d == 0.0f) return 0;
  const float inv_d = 1 / d;
  const float3 f = f3(inv_d * t0, inv_d * t0, inv_d * -1.0f);
  const float ppx = f.x * (Tu.x * Tw.x) + f.y * (Tu.y * Tw.y) + f.z * (Tu.z * Tw.z);
  const float ppy = f.x * (Tv.x * Tw.x) + f.y * (Tv.y * Tw.y) + f.z * (Tv.z * Tw.z);
  const float h0x = ppx * ppx - (f.x * (Tu.x * Tu.x) + f.y * (Tu.y * Tu.y) + f.z * (Tu.z * Tu.z));
  const float h0y = ppy * ppy - (f.x * (Tv.x * Tv.x) + f.y * (Tv.y * Tv.y) + f.z * (Tv.z * Tv.z));
  const float ex = sqrtf(fmaxf(1e-4f, h0x)), ey = sqrtf(fmaxf(1e-4f, h0y));
  const float radius = ceilf(fmaxf(fmaxf(ex, ey), cutoff * kFilterSize));
  int x0, y0, x1, y1;
  tile_rect(ppx, ppy, (int)radius, gx, gy, x0, y0, x1, y1);
  if ((x1 - x0) * (y1 - y0) == 0) return 0;
  radius_out = (int)radius;

  // Tight footprint: a pixel can only blend this surfel where
  // min(rho3d, rho2d) <= rho_cut, i.e. inside the ellipse rho3d <= rho_cut (its
  // screen box is compute_aabb's formula at cutoff sqrt(rho_cut)) or inside the
  // disc rho2d = 2 |xy - pixel|^2 <= rho_cut. Tiles outside that box would only
  // ever see alpha < 1/255 and are not emitted; the pixel box is also kept in
  // the record so the blend kernel skips pixels outside it.
  float rho_cut = 0.f;
  float bx0 = 1.f, bx1 = 0.f, by0 = 1.f, by1 = 0.f;  // empty
  uint32_t tiles = 0;
  int tx0 = x0, tx1 = x0, ty0 = y0, ty1 = y0;
  if (alpha_cutoff(a.opacity, beta, kernel_type, a.shape, rho_cut)) {
    const bool bounded = isfinite(rho_cut);
    // The disc u^2 + v^2 <= rho_cut of the splat plane projects to an ellipse
    // when the whole disc lies in front of the camera: w = Tw.x u + Tw.y v + Tw.z
    // > 0 on it, i.e. dc < 0 (with a relative margin against near-degenerate
    // conics). Otherwise its image is unbounded and the reference rectangle stays.
    const float dc = rho_cut * (Tw.x * Tw.x) + rho_cut * (Tw.y * Tw.y) - (Tw.z * Tw.z);
    float ex0, ex1, ey0, ey1;
    bool ok = bounded && dc < -1e-4f * (Tw.z * Tw.z);
    if (ok) {
      const float idc = 1.0f / dc;
      const float3 fc = f3(idc * rho_cut, idc * rho_cut, -idc);
      const float cx = fc.x * (Tu.x * Tw.x) + fc.y * (Tu.y * Tw.y) + fc.z * (Tu.z * Tw.z);
      const float cy = fc.x * (Tv.x * Tw.x) + fc.y * (Tv.y * Tw.y) + fc.z * (Tv.z * Tw.z);
      const float hx2 = cx * cx - (fc.x * (Tu.x * Tu.x) + fc.y * (Tu.y * Tu.y) + fc.z * (Tu.z * Tu.z));
      const float hy2 = cy * cy - (fc.x * (Tv.x * Tv.x) + fc.y * (Tv.y * Tv.y) + fc.z * (Tv.z * Tv.z));
      ok = hx2 >= 0.0f && hy2 >= 0.0f && isfinite(cx) && isfinite(cy);
      if (ok) {
        const float hx = sqrtf(hx2) * 1.01f + 1.0f, hy = sqrtf(hy2) * 1.01f + 1.0f;
        ex0 = cx - hx;
        ex1 = cx + hx;
        ey0 = cy - hy;
        ey1 = cy + hy;
      }
    }
    if (!ok) {  // not an ellipse at this cutoff: keep the reference rectangle
      ex0 = (float)(x0 * kTile);
      ex1 = (float)(x1 * kTile - 1);
      ey0 = (float)(y0 * kTile);
      ey1 = (float)(y1 * kTile - 1);
    }
    const float r2 = bounded ? sqrtf(0.5f * rho_cut) * 1.01f + 1.0f : 0.0f;
    bx0 = fmaxf(fminf(ex0, ppx - r2), -1.0f);
    bx1 = fminf(fmaxf(ex1, ppx + r2), (float)W);
    by0 = fmaxf(fminf(ey0, ppy - r2), -1.0f);
    by1 = fminf(fmaxf(ey1, ppy + r2), (float)H);
    if (bx0 <= bx1 && by0 <= by1) {
      tx0 = max(x0, (int)floorf(fmaxf(bx0, 0.f) / kTile));
      tx1 = min(x1, (int)floorf(bx1 / kTile) + 1);
      ty0 = max(y0, (int)floorf(fmaxf(by0, 0.f) / kTile));
      ty1 = min(y1, (int)floorf(by1 / kTile) + 1);
      if (tx1 > tx0 && ty1 > ty0) tiles = (uint32_t)((tx1 - tx0) * (ty1 - ty0));
    }
  }
  if (tiles == 0) tx1 = tx0, ty1 = ty0;

  const uint32_t ap_bits = (uint32_t)floorf(fminf(a.ap, 4.0e9f));
  rec.q[0] = make_float4(bx0, bx1, by0, by1);
  rec.q[1] = make_float4(Tu.x, Tu.y, Tu.z, Tv.x);
  rec.q[2] = make_float4(Tv.y, Tv.z, Tw.x, Tw.y);
  rec.q[3] = make_float4(Tw.z, ppx, ppy, a.opacity);
  rec.q[4] = make_float4(n.x, n.y, n.z, __uint_as_float(ap_bits));
  rec.q[5] = make_float4(a.su.x, a.su.y, a.su.z, a.sv.x);
  rec.q[6] = make_float4(a.sv.y, a.sv.z, a.pk.x, a.pk.y);
  rec.q[7] = make_float4(a.pk.z, rho_cut, 0.f, a.shape);
  bi.x0 = (int16_t)tx0;
  bi.x1 = (int16_t)tx1;
  bi.y0 = (int16_t)ty0;
  bi.y1 = (int16_t)ty1;
  bi.depth = pv.z;
  bi.pad = 0;
  return tiles;
}

template <class Attrs>
__global__ void __launch_bounds__(kPreThreads)
preprocess_kernel(int P, Attrs attrs, float mod, float beta, int kernel_type,
                  const float* __restrict__ viewmatrix, const float* __restrict__ projmatrix, int W,
                  int H, PreOut out) {
  __shared__ float vm[16], pm[16];
  __shared__ uint32_t warp_sums[kPreThreads / 32];
  if (threadIdx.x < 16) vm[threadIdx.x] = viewmatrix[threadIdx.x];
  else if (threadIdx.x < 32) pm[threadIdx.x - 16] = projmatrix[threadIdx.x - 16];
  __syncthreads();
  const int gx = div_up(W, kTile), gy = div_up(H, kTile);
  const int i = blockIdx.x * kPreThreads + threadIdx.x;
  uint32_t tiles = 0;
  if (i < P) {
    SurfelRecord rec;
    BinInfo bi;
    bi.x0 = bi.x1 = bi.y0 = bi.y1 = 0;
    bi.depth = 0.f;
    bi.pad = 0;
    int radius = 0;
    const SurfelIn a = attrs.load(i);
    tiles = preprocess_one(a, mod, beta, kernel_type, vm, pm, W, H, gx, gy, rec, bi, radius);
    rec.q[7].z = __uint_as_float((uint32_t)i);
    if (tiles) {
      float4* dst = reinterpret_cast<float4*>(out.records + i);
#pragma unroll
      for (int k = 0; k < 8; k++) dst[k] = rec.q[k];
    }
    out.bin[i] = bi;
    out.radii[i] = radius;
    out.tiles[i] = tiles;
    out.depth_keys[i] = tiles ? __float_as_uint(bi.depth) : 0xffffffffu;
    out.depth_vals[i] = (uint32_t)i;
  }
  // CTA total of the tile counts (the instance count is their sum).
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = tiles;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[w] = x;
  __syncthreads();
  uint32_t add = 0;
  for (int k = 0; k < w; k++) add += warp_sums[k];
  if (threadIdx.x == kPreThreads - 1) out.block_sums[blockIdx.x] = x + add;
}

__global__ void mark_visible_kernel(int P, const float* __restrict__ means3D,
                                    const float* __restrict__ vm, uint8_t* __restrict__ present) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  const float x = means3D[3 * i], y = means3D[3 * i + 1], z = means3D[3 * i + 2];
  const float vz = vm[2] * x + vm[6] * y + vm[10] * z + vm[14];
  present[i] = vz <= 0.2f ? 0 : 1;
}

}  // namespace

int preprocess_blocks(int P) { return div_up(max(P, 1), kPreThreads); }
int preprocess_block_size() { return kPreThreads; }

int preprocess_api_launch(int P, const ns_surfels& s, float mod, float beta, int kernel_type,
                          const float* vm,
                          const float* pm, int W, int H, SurfelRecord* records, BinInfo* bin,
                          int32_t* radii, uint32_t* tiles, uint32_t* depth_keys,
                          uint32_t* depth_vals, uint32_t* block_sums, cudaStream_t stream) {
  ApiAttrs a{s.means3D, s.scales, s.rotations, s.opacities, s.homotrans, s.ap_level, s.shapes, s.transmat_precomp};
  PreOut o{records, bin, radii, tiles, depth_keys, depth_vals, block_sums};
  preprocess_kernel<ApiAttrs><<<preprocess_blocks(P), kPreThreads, 0, stream>>>(
      P, a, mod, beta, kernel_type, vm, pm, W, H, o);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int preprocess_mix_launch(int P, const float* base, const float* decoded, int dims, float mix,
                          const float* ap_level, float mod, float beta, const float* vm,
                          const float* pm, int W, int H, SurfelRecord* records, BinInfo* bin,
                          int32_t* radii, uint32_t* tiles, uint32_t* depth_keys,
                          uint32_t* depth_vals, uint32_t* block_sums, cudaStream_t stream) {
  MixAttrs a{base, decoded, dims, mix, ap_level};
  PreOut o{records, bin, radii, tiles, depth_keys, depth_vals, block_sums};
  preprocess_kernel<MixAttrs><<<preprocess_blocks(P), kPreThreads, 0, stream>>>(
      P, a, mod, beta, 0, vm, pm, W, H, o);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

int mark_visible_launch(int P, const float* means3D, const float* vm, uint8_t* present,
                        cudaStream_t stream) {
  if (P <= 0) return NS_OK;
  mark_visible_kernel<<<div_up(P, 256), 256, 0, stream>>>(P, means3D, vm, present);
  NS_LAUNCH_CHECK();
  return NS_OK;
}

}  // namespace ns
