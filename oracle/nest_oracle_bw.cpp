// nest_oracle_bw.cpp -- CPU restatement of the mode-0 backward pass of
// nest-splatting's surfel rasterizer.
//
// TEST INFRASTRUCTURE ONLY (the same rules as nest_oracle.cpp): tests/ use it as
// the checker of the CUDA backward; the product never links or calls it.
//
// Parity status: the reference backward cannot be run here (the rasterizer does
// not build without glm), so this restatement is pinned in
// tests/test_oracle_backward.py against float64 autograd of an independent
// torch model of the forward pass. The model carries, explicitly, the places
// where the reference's backward is not the derivative of its forward (listed
// there and in the comments below), so every other term is checked as a true
// gradient.
//
// Paths are relative to submodules/diff-surfel-rasterization/.
#include "oracle_math.h"

using namespace oracle;

namespace {

inline void atomic_add(float* p, float v) {
#pragma omp atomic
  *p += v;
}

// hashgrid.h:53-299 with BW = true, D = 3: the forward lookup, the table
// gradient scatter (:184-190: dL_dgrid[index + ch] += w * grad_feat[level LD + ch])
// and dL/dxyz from the finite differences of the 4 edges along each axis
// (:212-299). grad_scale is the box-map slope, or for contract the slope of the
// inner region times the radial scale (the reference's approximation of the
// contraction Jacobian, :66-97).
void query_feature_bw(float* feat, int C, int LD, F3 xyz, float vmin, float vmax,
                      const int* offsets, uint32_t ap_level, const float* table, uint32_t L,
                      float S, uint32_t Hres, bool align_corners, uint32_t interp, bool contract,
                      const float* grad_feat, float* dL_dtable, float dL_dxyz[3]) {
  float in[3];
  bool oob = false;
  float grad_scale = 0.0f;
  if (!contract) {
    float inv = 1.0f / (vmax - vmin);
    in[0] = (xyz.x - vmin) * inv;
    in[1] = (xyz.y - vmin) * inv;
    in[2] = (xyz.z - vmin) * inv;
    grad_scale = inv;
    oob = in[0] < 0 || in[0] > 1 || in[1] < 0 || in[1] > 1 || in[2] < 0 || in[2] > 1;
  } else {
    float vmid = (vmax + vmin) * 0.5f;
    float inv = 1.0f / ((vmax - vmin) * 0.5f);
    in[0] = (xyz.x - vmid) * inv;
    in[1] = (xyz.y - vmid) * inv;
    in[2] = (xyz.z - vmid) * inv;
    float norm = std::sqrt(in[0] * in[0] + in[1] * in[1] + in[2] * in[2]);
    float inv_norm = 1.0f / norm;
    float st = (norm <= 1.0f) ? 1.0f : (2.0f - inv_norm) * inv_norm;
    for (int d = 0; d < 3; d++) in[d] = (st * in[d] + 2.0f) * 0.25f;
    grad_scale = inv * st * 0.25f;
  }
  const uint32_t max_level = std::min(ap_level, L);
  for (int c = 0; c < C; c++) feat[c] = 0.f;
  for (int d = 0; d < 3; d++) dL_dxyz[d] = 0.f;
  if (oob) return;
  std::vector<float> dy_dx((size_t)3 * C, 0.f);
  for (uint32_t lv = 0; lv < max_level; lv++) {
    const uint32_t hsize = (uint32_t)(offsets[lv + 1] - offsets[lv]);
    const float scale = std::exp2(lv * S) * Hres - 1.0f;
    const uint32_t res = (uint32_t)std::ceil(scale) + 1;
    const float* grid = table + (size_t)(uint32_t)offsets[lv] * LD;
    float* dgrid = dL_dtable + (size_t)(uint32_t)offsets[lv] * LD;
    const float* gl = grad_feat + lv * LD;
    float pos[3], deriv[3];
    uint32_t pg[3];
    for (int d = 0; d < 3; d++) {
      pos[d] = in[d] * scale + (align_corners ? 0.0f : 0.5f);
      pg[d] = (uint32_t)std::floor(pos[d]);
      pos[d] -= (float)pg[d];
      if (interp == 1) {
        deriv[d] = 6 * pos[d] * (1.0f - pos[d]);
        pos[d] = pos[d] * pos[d] * (3.0f - 2.0f * pos[d]);
      } else {
        deriv[d] = 1.0f;
      }
    }
    float r[16] = {0};
    for (uint32_t c = 0; c < 8; c++) {
      float w = 1;
      uint32_t g[3];
      for (int d = 0; d < 3; d++) {
        if ((c & (1u << d)) == 0) { w *= 1 - pos[d]; g[d] = pg[d]; }
        else { w *= pos[d]; g[d] = pg[d] + 1; }
      }
      const uint32_t idx = grid_index(align_corners, hsize, res, g) * LD;
      for (int ch = 0; ch < LD; ch++) r[ch] += w * grid[idx + ch];
      for (int ch = 0; ch < LD; ch++) atomic_add(&dgrid[idx + ch], w * gl[ch]);
    }
    for (int ch = 0; ch < LD; ch++) feat[lv * LD + ch] = r[ch];
    // hashgrid.h:231-283: d feat / d in_gd from the 4 edges along axis gd.
    for (int gd = 0; gd < 3; gd++) {
      float rg[16] = {0};
      for (uint32_t e = 0; e < 4; e++) {
        float w = scale * grad_scale;
        uint32_t g[3];
        for (int nd = 0; nd < 2; nd++) {
          const int d = (nd >= gd) ? nd + 1 : nd;
          if ((e & (1u << nd)) == 0) { w *= 1 - pos[d]; g[d] = pg[d]; }
          else { w *= pos[d]; g[d] = pg[d] + 1; }
        }
        g[gd] = pg[gd];
        const uint32_t il = grid_index(align_corners, hsize, res, g) * LD;
        g[gd] = pg[gd] + 1;
        const uint32_t ir = grid_index(align_corners, hsize, res, g) * LD;
        for (int ch = 0; ch < LD; ch++) rg[ch] += w * (grid[ir + ch] - grid[il + ch]) * deriv[gd];
      }
      for (int ch = 0; ch < LD; ch++) dy_dx[(size_t)gd * C + lv * LD + ch] = rg[ch];
    }
  }
  // hashgrid.h:285-297
  for (int d = 0; d < 3; d++) {
    float acc = 0;
    for (uint32_t lv = 0; lv < max_level; lv++)
      for (int ch = 0; ch < LD; ch++)
        acc += grad_feat[lv * LD + ch] * dy_dx[(size_t)d * C + lv * LD + ch];
    dL_dxyz[d] = acc;
  }
}

// glm::dot of two 3-vectors: the products summed left to right.
inline float dot3(F3 a, F3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline F3 add3(F3 a, F3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
inline F3 mul3(F3 a, F3 b) { return {a.x * b.x, a.y * b.y, a.z * b.z}; }

}  // namespace

extern "C" {

// backward.cu:445-2052, renderCUDAsurfelBackward<C> for render_mode 0,
// kernel_type 0, level > 0, homotrans given. Per pixel, the tile list is walked
// back to front from the last contributor; T is recovered by dividing by
// (1 - alpha) (:914); the colour term uses the hash features re-queried at the
// hit point (:934-980, :1786-1797), the auxiliary terms follow :1799-1852, the
// kernel/homotrans/transform grads :1854-2045 and opacity :2048.
//
// Places where the reference's backward is not the derivative of its forward,
// kept as they are:
//   * beta > 0: the ray/surfel term uses dG_factor = -G with G after the beta
//     transform (:1957-1982) and the transform's denominator is rounded to
//     float (:909-912);
//   * the 0.99 clamp on alpha is not differentiated.
// Gradient outputs are accumulated (+=), as with the reference's zeroed
// buffers: dL_dtable [rows, LD], dL_dtransMat [P,9], dL_dhomoMat [P,9],
// dL_dmean2D [P,3], dL_dnormal [P,3], dL_dopacity [P], dL_gradsum [P].
void oracle_render_backward(int W, int H, const uint32_t* ranges, const uint32_t* point_list,
                            const float* means2D, const float* transMat,
                            const float* normal_opacity, const float* homotrans,
                            const float* ap_level, const float* table, const int* offsets,
                            const float* gridrange, int C, int LD, uint32_t L, float S,
                            uint32_t Hres, int align_corners, uint32_t interp, int contract,
                            float beta, const float* final_T, const uint32_t* n_contrib,
                            const float* dL_dout_color, const float* dL_dout_others,
                            float* dL_dtable, float* dL_dtransMat, float* dL_dhomoMat,
                            float* dL_dmean2D, float* dL_dnormal, float* dL_dopacity,
                            float* dL_gradsum) {
  const int gx = (W + kBlock - 1) / kBlock, gy = (H + kBlock - 1) / kBlock;
  const size_t HW = (size_t)H * W;
  const float vmin = gridrange[0], vmax = gridrange[1];
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < gx * gy; tile++) {
    std::vector<float> dL_dpixel(C), accum_rec(C), last_color(C), grad_feat(C), feat(C);
    const int tx = tile % gx, ty = tile / gx;
    const uint32_t r0 = ranges[2 * tile], r1 = ranges[2 * tile + 1];
    for (int py = ty * kBlock; py < std::min(H, (ty + 1) * kBlock); py++) {
      for (int px = tx * kBlock; px < std::min(W, (tx + 1) * kBlock); px++) {
        const size_t pid = (size_t)py * W + px;
        const float pxf = (float)px, pyf = (float)py;
        const float T_final = final_T[pid];
        float T = T_final;
        uint32_t contributor = r1 - r0;
        const uint32_t last_contributor = n_contrib[pid];
        const int median_contributor = (int)n_contrib[pid + HW];
        const float dL_ddepth = dL_dout_others[0 * HW + pid];
        const float dL_daccum = dL_dout_others[1 * HW + pid];
        const float dL_dreg = dL_dout_others[6 * HW + pid];
        float dL_dnormal2D[3];
        for (int i = 0; i < 3; i++) dL_dnormal2D[i] = dL_dout_others[(2 + i) * HW + pid];
        const float dL_dmedian_depth = dL_dout_others[5 * HW + pid];
        float last_depth = 0, last_normal[3] = {0, 0, 0};
        float accum_depth_rec = 0, accum_alpha_rec = 0, accum_normal_rec[3] = {0, 0, 0};
        const float final_D = final_T[pid + HW];
        const float final_D2 = final_T[pid + 2 * HW];
        const float final_A = 1 - T_final;
        float last_dL_dT = 0;
        for (int c = 0; c < C; c++) {
          dL_dpixel[c] = dL_dout_color[c * HW + pid];
          accum_rec[c] = 0.f;
          last_color[c] = 0.f;
        }
        float last_alpha = 0;
        for (uint32_t k = r1; k-- > r0;) {
          contributor--;
          if (contributor >= last_contributor) continue;
          const uint32_t id = point_list[k];
          const float* Tm = transMat + 9 * (size_t)id;
          const F3 Tu = {Tm[0], Tm[1], Tm[2]}, Tv = {Tm[3], Tm[4], Tm[5]}, Tw = {Tm[6], Tm[7], Tm[8]};
          const F3 kk = sub(scl(pxf, Tw), Tu);
          const F3 ll = sub(scl(pyf, Tw), Tv);
          const F3 p = crs(kk, ll);
          if (p.z == 0.0f) continue;
          const float sx = p.x / p.z, sy = p.y / p.z;
          const float rho3d = sx * sx + sy * sy;
          const float dx = means2D[2 * id] - pxf, dy = means2D[2 * id + 1] - pyf;
          const float rho2d = kFilterInvSquare * (dx * dx + dy * dy);
          const float rho = std::min(rho3d, rho2d);
          const float c_d = (rho3d <= rho2d) ? (sx * Tw.x + sy * Tw.y) + Tw.z : Tw.z;
          if (c_d < kNear) continue;
          const float* no = normal_opacity + 4 * (size_t)id;
          const float normal[3] = {no[0], no[1], no[2]};
          const float opa = no[3];
          const float power = -0.5f * rho;
          if (power > 0.0f) continue;
          float G = std::exp(power);
          float demon = 1.0f;
          if (beta > 0.0) {
            demon = (float)(1.0 + beta * G);
            G = (float)((1.0 + beta) * G / demon);
          }
          const float alpha = std::min(0.99f, opa * G);
          if (alpha < 1.0f / 255.0f) continue;

          T = T / (1.f - alpha);
          const float dchannel_dcolor = alpha * T;
          float dL_dalpha = 0.0f;

          // Hit point and hash features (:934-980).
          const float* h = homotrans + 16 * (size_t)id;
          const F3 sutu = {h[0], h[4], h[8]}, svtv = {h[1], h[5], h[9]}, pk = {h[3], h[7], h[11]};
          F3 xyz;
          if (rho3d <= rho2d) {
            xyz = {sx * sutu.x + sy * svtv.x + pk.x, sx * sutu.y + sy * svtv.y + pk.y,
                   sx * sutu.z + sy * svtv.z + pk.z};
          } else {
            xyz = pk;
          }
          float sum_grad = 0.0f;
          for (int c = 0; c < C; c++) {
            grad_feat[c] = dchannel_dcolor * dL_dpixel[c];
            sum_grad += std::fabs(grad_feat[c]);
          }
          atomic_add(&dL_gradsum[id], sum_grad);
          const uint32_t apl = (uint32_t)std::floor(ap_level[id]);
          float dL_dxyz[3];
          query_feature_bw(feat.data(), C, LD, xyz, vmin, vmax, offsets, apl, table, L, S, Hres,
                           align_corners != 0, interp, contract != 0, grad_feat.data(), dL_dtable,
                           dL_dxyz);
          for (int c = 0; c < C; c++) {
            accum_rec[c] = last_alpha * last_color[c] + (1.f - last_alpha) * accum_rec[c];
            last_color[c] = feat[c];
            dL_dalpha += (feat[c] - accum_rec[c]) * dL_dpixel[c];
          }

          // Auxiliary maps (:1799-1852).
          float dL_dz = 0.0f;
          float dL_dweight = 0;
          const float m_d = kFar / (kFar - kNear) * (1 - kNear / c_d);
          const float dmd_dd = (kFar * kNear) / ((kFar - kNear) * c_d * c_d);
          if ((int)contributor == median_contributor - 1) dL_dz += dL_dmedian_depth;
          dL_dweight += (final_D2 + m_d * m_d * final_A - 2 * m_d * final_D) * dL_dreg;
          dL_dalpha += dL_dweight - last_dL_dT;
          last_dL_dT = dL_dweight * alpha + (1 - alpha) * last_dL_dT;
          const float dL_dmd = 2.0f * (T * alpha) * (m_d * final_A - final_D) * dL_dreg;
          dL_dz += dL_dmd * dmd_dd;
          accum_depth_rec = last_alpha * last_depth + (1.f - last_alpha) * accum_depth_rec;
          last_depth = c_d;
          dL_dalpha += (c_d - accum_depth_rec) * dL_ddepth;
          accum_alpha_rec = (float)(last_alpha * 1.0 + (1.f - last_alpha) * accum_alpha_rec);
          dL_dalpha += (1 - accum_alpha_rec) * dL_daccum;
          for (int c = 0; c < 3; c++) {
            accum_normal_rec[c] = last_alpha * last_normal[c] + (1.f - last_alpha) * accum_normal_rec[c];
            last_normal[c] = normal[c];
            dL_dalpha += (normal[c] - accum_normal_rec[c]) * dL_dnormal2D[c];
            atomic_add(&dL_dnormal[id * 3 + c], alpha * T * dL_dnormal2D[c]);
          }
          dL_dalpha *= T;
          last_alpha = alpha;

          float dL_dG = opa * dL_dalpha;
          if (beta > 0.0) {
            const float dG_dg = (float)((1.0 + beta) / (demon * demon));
            dL_dG *= dG_dg;
          }
          dL_dz += alpha * T * dL_ddepth;

          // homotrans grads (:1921-1953).
          float dL_du = 0.0f, dL_dv = 0.0f;
          float* hm = dL_dhomoMat + (size_t)id * 9;
          if (rho3d <= rho2d) {
            dL_du = dL_dxyz[0] * sutu.x + dL_dxyz[1] * sutu.y + dL_dxyz[2] * sutu.z;
            dL_dv = dL_dxyz[0] * svtv.x + dL_dxyz[1] * svtv.y + dL_dxyz[2] * svtv.z;
            atomic_add(&hm[0], dL_dxyz[0] * sx);
            atomic_add(&hm[1], dL_dxyz[1] * sx);
            atomic_add(&hm[2], dL_dxyz[2] * sx);
            atomic_add(&hm[3], dL_dxyz[0] * sy);
            atomic_add(&hm[4], dL_dxyz[1] * sy);
            atomic_add(&hm[5], dL_dxyz[2] * sy);
          }
          atomic_add(&hm[6], dL_dxyz[0]);
          atomic_add(&hm[7], dL_dxyz[1]);
          atomic_add(&hm[8], dL_dxyz[2]);

          float* tm = dL_dtransMat + (size_t)id * 9;
          if (rho3d <= rho2d) {
            // :1956-2017, Gaussian kernel: dG_factor = -G.
            const float dG_factor = -G;
            float dsx = dL_dG * dG_factor * sx + dL_dz * Tw.x;
            float dsy = dL_dG * dG_factor * sy + dL_dz * Tw.y;
            dsx += dL_du;
            dsy += dL_dv;
            const float dsx_pz = dsx / p.z;
            const float dsy_pz = dsy / p.z;
            const F3 dL_dp = {dsx_pz, dsy_pz, -(dsx_pz * sx + dsy_pz * sy)};
            const F3 dL_dk = crs(ll, dL_dp);
            const F3 dL_dl = crs(dL_dp, kk);
            atomic_add(&tm[0], -dL_dk.x);
            atomic_add(&tm[1], -dL_dk.y);
            atomic_add(&tm[2], -dL_dk.z);
            atomic_add(&tm[3], -dL_dl.x);
            atomic_add(&tm[4], -dL_dl.y);
            atomic_add(&tm[5], -dL_dl.z);
            atomic_add(&tm[6], pxf * dL_dk.x + pyf * dL_dl.x + dL_dz * sx);
            atomic_add(&tm[7], pxf * dL_dk.y + pyf * dL_dl.y + dL_dz * sy);
            atomic_add(&tm[8], pxf * dL_dk.z + pyf * dL_dl.z + dL_dz * 1.0f);
          } else {
            // :2018-2045
            const float dG_factor_2d = -G * kFilterInvSquare;
            const float dG_ddelx = dG_factor_2d * dx;
            const float dG_ddely = dG_factor_2d * dy;
            atomic_add(&dL_dmean2D[(size_t)id * 3 + 0], dL_dG * dG_ddelx);
            atomic_add(&dL_dmean2D[(size_t)id * 3 + 1], dL_dG * dG_ddely);
            atomic_add(&tm[8], dL_dz);
          }
          atomic_add(&dL_dopacity[id], G * dL_dalpha);
        }
      }
    }
  }
}

// backward.cu:2216-2273 (preprocessCUDA, backward) and :2056-2214
// (compute_transmat_aabb) for surfels with radii > 0, scales and rotations given.
// As in the reference, the transform is rebuilt with scale_modifier 1 (:2090),
// the mean2D gradient is pushed into T through the compute_aabb centre with a
// cutoff of 3 (t = (9, 9, -1), :2143) while the forward uses 4, and dL_dmean2D
// is then overwritten by the densification statistic (:2270-2272) computed with
// W = int(focal_x * tan_fovx * 2).
// transMat [P,9] is the forward pass's transform (with scale_modifier).
// In: dL_dmean2D [P,3] (render pass values; overwritten), dL_dnormal [P,3],
// dL_dtransMat [P,9], dL_dhomoMat [P,9]. Out: dL_dmeans3D [P,3], dL_dscales
// [P,2], dL_drots [P,4] (written only for radii > 0).
void oracle_preprocess_backward(int P, const float* means3D, const float* scales,
                                const float* rotations, const int* radii,
                                const float* transMat, const float* viewmatrix, const float* projmatrix, int width,
                                int height, float tanfovx, float tanfovy, float* dL_dmean2D,
                                const float* dL_dnormal, const float* dL_dtransMat,
                                const float* dL_dhomoMat, float* dL_dmeans3D, float* dL_dscales,
                                float* dL_drots) {
  const float focal_x = width / (2.0f * tanfovx);
  const float focal_y = height / (2.0f * tanfovy);
  const int W = int(focal_x * tanfovx * 2);
  const int H = int(focal_y * tanfovy * 2);
  const float* pm = projmatrix;
  const float* vm = viewmatrix;
#pragma omp parallel for schedule(static)
  for (int i = 0; i < P; i++) {
    if (!(radii[i] > 0)) continue;
    const F3 p = {means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]};
    const float* q = rotations + 4 * i;
    const float sx = scales[2 * i], sy = scales[2 * i + 1];
    F3 R[3];
    quat_to_cols(q, R);
    const F3 L0 = scl(sx, R[0]), L1 = scl(sy, R[1]), L2 = R[2];
    // P = world2ndc * ndc2pix as glm mat3x4: column c, rows 0..3.
    const float n[3][4] = {{float(W) / 2.0f, 0.f, 0.f, float(W - 1) / 2.0f},
                           {0.f, float(H) / 2.0f, 0.f, float(H - 1) / 2.0f},
                           {0.f, 0.f, 0.f, 1.f}};
    float Pm[3][4];
    for (int c = 0; c < 3; c++)
      for (int r = 0; r < 4; r++)
        Pm[c][r] = ((pm[4 * r + 0] * n[c][0] + pm[4 * r + 1] * n[c][1]) + pm[4 * r + 2] * n[c][2]) +
                   pm[4 * r + 3] * n[c][3];
    // T = transpose(M) * P, M columns (L0,0), (L1,0), (p,1); T[c][i] = M[i] . P[c].
    const float Mc[3][4] = {{L0.x, L0.y, L0.z, 0.f}, {L1.x, L1.y, L1.z, 0.f}, {p.x, p.y, p.z, 1.f}};
    F3 T[3];
    for (int c = 0; c < 3; c++) {
      float t[3];
      for (int r = 0; r < 3; r++)
        t[r] = ((Mc[r][0] * Pm[c][0] + Mc[r][1] * Pm[c][1]) + Mc[r][2] * Pm[c][2]) + Mc[r][3] * Pm[c][3];
      T[c] = {t[0], t[1], t[2]};
    }
    const F3 normal = xform_vec4x3(L2, vm);

    F3 dT[3];
    for (int c = 0; c < 3; c++)
      dT[c] = {dL_dtransMat[9 * i + 3 * c], dL_dtransMat[9 * i + 3 * c + 1], dL_dtransMat[9 * i + 3 * c + 2]};
    const float gmx = dL_dmean2D[3 * i], gmy = dL_dmean2D[3 * i + 1];
    if (gmx != 0 || gmy != 0) {
      const F3 t_vec = {9.0f, 9.0f, -1.0f};
      const float d = dot3(t_vec, mul3(T[2], T[2]));
      const F3 f_vec = scl(1.0f / d, t_vec);
      const F3 dT0 = mul3(scl(gmx, f_vec), T[2]);
      const F3 dT1 = mul3(scl(gmy, f_vec), T[2]);
      F3 dT3 = add3(mul3(scl(gmx, f_vec), T[0]), mul3(scl(gmy, f_vec), T[1]));
      const F3 dL_df = add3(mul3(scl(gmx, T[0]), T[2]), mul3(scl(gmy, T[1]), T[2]));
      const float dL_dd = (float)(dot3(dL_df, f_vec) * (-1.0 / d));
      const F3 dd_dT3 = scl(2.0f, mul3(t_vec, T[2]));
      dT3 = add3(dT3, scl(dL_dd, dd_dT3));
      dT[0] = add3(dT[0], dT0);
      dT[1] = add3(dT[1], dT1);
      dT[2] = add3(dT[2], dT3);
    }
    // dL_dM = P * transpose(dL_dT) + dL_dhomo: column c = sum_k P[k] dL_dT[k][c].
    float dM[3][4];
    for (int c = 0; c < 3; c++) {
      const float g[3] = {(&dT[0].x)[c], (&dT[1].x)[c], (&dT[2].x)[c]};
      for (int r = 0; r < 4; r++)
        dM[c][r] = (Pm[0][r] * g[0] + Pm[1][r] * g[1]) + Pm[2][r] * g[2];
    }
    for (int c = 0; c < 3; c++)
      for (int r = 0; r < 3; r++) dM[c][r] += dL_dhomoMat[9 * i + 3 * c + r];

    // Normal: normalisation backprop as written at :2177-2190, view transform
    // transposed, and the camera-facing flip (DUAL_VISIABLE, :2194-2199).
    const F3 gn = {dL_dnormal[3 * i], dL_dnormal[3 * i + 1], dL_dnormal[3 * i + 2]};
    const float nlen = std::sqrt(normal.x * normal.x + normal.y * normal.y + normal.z * normal.z);
    F3 gu = {0.f, 0.f, 0.f};
    if (nlen > 1e-7f) {
      const float dgn = gn.x * normal.x + gn.y * normal.y + gn.z * normal.z;
      gu.x = (gn.x - dgn * normal.x / nlen) / nlen;
      gu.y = (gn.y - dgn * normal.y / nlen) / nlen;
      gu.z = (gn.z - dgn * normal.z / nlen) / nlen;
    }
    F3 dtn = {vm[0] * gu.x + vm[1] * gu.y + vm[2] * gu.z, vm[4] * gu.x + vm[5] * gu.y + vm[6] * gu.z,
              vm[8] * gu.x + vm[9] * gu.y + vm[10] * gu.z};
    const F3 pv = xform_point4x3(p, vm);
    const float cosv = -((pv.x * normal.x + pv.y * normal.y) + pv.z * normal.z);
    const float mult = cosv > 0 ? 1.f : -1.f;
    dtn = scl(mult, dtn);

    const F3 dRS0 = {dM[0][0], dM[0][1], dM[0][2]}, dRS1 = {dM[1][0], dM[1][1], dM[1][2]};
    const F3 dR0 = scl(sx, dRS0), dR1 = scl(sy, dRS1), dR2 = dtn;
    // auxiliary.h:243-287 quat_to_rotmat_vjp; v_R[c][r] = column c, row r.
    const float s = 1.0f / std::sqrt(q[3] * q[3] + q[0] * q[0] + q[1] * q[1] + q[2] * q[2]);
    const float w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    const float v[3][3] = {{dR0.x, dR0.y, dR0.z}, {dR1.x, dR1.y, dR1.z}, {dR2.x, dR2.y, dR2.z}};
    float* dq = dL_drots + 4 * i;
    dq[0] = 2.f * (x * (v[1][2] - v[2][1]) + y * (v[2][0] - v[0][2]) + z * (v[0][1] - v[1][0]));
    dq[1] = 2.f * (-2.f * x * (v[1][1] + v[2][2]) + y * (v[0][1] + v[1][0]) +
                   z * (v[0][2] + v[2][0]) + w * (v[1][2] - v[2][1]));
    dq[2] = 2.f * (x * (v[0][1] + v[1][0]) - 2.f * y * (v[0][0] + v[2][2]) +
                   z * (v[1][2] + v[2][1]) + w * (v[2][0] - v[0][2]));
    dq[3] = 2.f * (x * (v[0][2] + v[2][0]) + y * (v[1][2] + v[2][1]) -
                   2.f * z * (v[0][0] + v[1][1]) + w * (v[0][1] - v[1][0]));
    dL_dscales[2 * i] = dot3(dRS0, R[0]);
    dL_dscales[2 * i + 1] = dot3(dRS1, R[1]);
    dL_dmeans3D[3 * i] = dM[2][0];
    dL_dmeans3D[3 * i + 1] = dM[2][1];
    dL_dmeans3D[3 * i + 2] = dM[2][2];

    // Densification statistic (:2268-2272), depth = Tw.z of the forward transform.
    const float depth = transMat[9 * i + 8];
    dL_dmean2D[3 * i] = (float)((double)(dL_dtransMat[9 * i + 2] * depth) * 0.5 * (double)(float)W);
    dL_dmean2D[3 * i + 1] = (float)((double)(dL_dtransMat[9 * i + 5] * depth) * 0.5 * (double)(float)H);
  }
}

}  // extern "C"
