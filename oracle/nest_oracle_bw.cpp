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

template <typename R>
inline void atomic_add(R* p, R v) {
#pragma omp atomic
  *p += v;
}

// 3-vector in the working precision R (float: the reference's arithmetic;
// double: the same formulas without float cancellation, for conditioning checks).
template <typename R>
struct V3 {
  R x, y, z;
};
template <typename R>
inline V3<R> vsub(V3<R> a, V3<R> b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
template <typename R>
inline V3<R> vscl(R f, V3<R> a) { return {f * a.x, f * a.y, f * a.z}; }
template <typename R>
inline V3<R> vcrs(V3<R> a, V3<R> b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}

// hashgrid.h:53-299 with BW = true, D = 3: the forward lookup, the table
// gradient scatter (:184-190: dL_dgrid[index + ch] += w * grad_feat[level LD + ch])
// and dL/dxyz from the finite differences of the 4 edges along each axis
// (:212-299). grad_scale is the box-map slope, or for contract the slope of the
// inner region times the radial scale (the reference's approximation of the
// contraction Jacobian, :66-97).
template <typename R>
void query_feature_bw(R* feat, int C, int LD, V3<R> xyz, R vmin, R vmax, const int* offsets,
                      uint32_t ap_level, const float* table, uint32_t L, float S, uint32_t Hres,
                      bool align_corners, uint32_t interp, bool contract, const R* grad_feat,
                      R* dL_dtable, R dL_dxyz[3], const float* lexp2 = nullptr) {
  R in[3];
  bool oob = false;
  R grad_scale = 0;
  if (!contract) {
    R inv = R(1) / (vmax - vmin);
    in[0] = (xyz.x - vmin) * inv;
    in[1] = (xyz.y - vmin) * inv;
    in[2] = (xyz.z - vmin) * inv;
    grad_scale = inv;
    oob = in[0] < 0 || in[0] > 1 || in[1] < 0 || in[1] > 1 || in[2] < 0 || in[2] > 1;
  } else {
    R vmid = (vmax + vmin) * R(0.5);
    R inv = R(1) / ((vmax - vmin) * R(0.5));
    in[0] = (xyz.x - vmid) * inv;
    in[1] = (xyz.y - vmid) * inv;
    in[2] = (xyz.z - vmid) * inv;
    R norm = std::sqrt(in[0] * in[0] + in[1] * in[1] + in[2] * in[2]);
    R inv_norm = R(1) / norm;
    R st = (norm <= R(1)) ? R(1) : (R(2) - inv_norm) * inv_norm;
    for (int d = 0; d < 3; d++) in[d] = (st * in[d] + R(2)) * R(0.25);
    grad_scale = inv * st * R(0.25);
  }
  const uint32_t max_level = std::min(ap_level, L);
  for (int c = 0; c < C; c++) feat[c] = 0;
  for (int d = 0; d < 3; d++) dL_dxyz[d] = 0;
  if (oob) return;
  std::vector<R> dy_dx((size_t)3 * C, R(0));
  for (uint32_t lv = 0; lv < max_level; lv++) {
    const uint32_t hsize = (uint32_t)(offsets[lv + 1] - offsets[lv]);
    const float scale_f = level_exp2(lv, S, lexp2) * Hres - 1.0f;  // the level scale as the reference forms it
    const R scale = scale_f;
    const uint32_t res = (uint32_t)std::ceil(scale_f) + 1;
    const float* grid = table + (size_t)(uint32_t)offsets[lv] * LD;
    R* dgrid = dL_dtable + (size_t)(uint32_t)offsets[lv] * LD;
    const R* gl = grad_feat + lv * LD;
    R pos[3], deriv[3];
    uint32_t pg[3];
    for (int d = 0; d < 3; d++) {
      pos[d] = std::fma(in[d], scale, align_corners ? R(0) : R(0.5));  // contracted as nvcc does
      pg[d] = (uint32_t)std::floor(pos[d]);
      pos[d] -= (R)pg[d];
      if (interp == 1) {
        deriv[d] = 6 * pos[d] * (R(1) - pos[d]);
        pos[d] = pos[d] * pos[d] * (R(3) - R(2) * pos[d]);
      } else {
        deriv[d] = R(1);
      }
    }
    R r[16] = {0};
    for (uint32_t c = 0; c < 8; c++) {
      R w = 1;
      uint32_t g[3];
      for (int d = 0; d < 3; d++) {
        if ((c & (1u << d)) == 0) { w *= 1 - pos[d]; g[d] = pg[d]; }
        else { w *= pos[d]; g[d] = pg[d] + 1; }
      }
      const uint32_t idx = grid_index(align_corners, hsize, res, g) * LD;
      for (int ch = 0; ch < LD; ch++) r[ch] = std::fma(w, (R)grid[idx + ch], r[ch]);
      for (int ch = 0; ch < LD; ch++) atomic_add<R>(&dgrid[idx + ch], w * gl[ch]);
    }
    for (int ch = 0; ch < LD; ch++) feat[lv * LD + ch] = r[ch];
    // hashgrid.h:231-283: d feat / d in_gd from the 4 edges along axis gd.
    for (int gd = 0; gd < 3; gd++) {
      R rg[16] = {0};
      for (uint32_t e = 0; e < 4; e++) {
        R w = scale * grad_scale;
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
        for (int ch = 0; ch < LD; ch++)
          rg[ch] = std::fma(w * ((R)grid[ir + ch] - (R)grid[il + ch]), deriv[gd], rg[ch]);
      }
      for (int ch = 0; ch < LD; ch++) dy_dx[(size_t)gd * C + lv * LD + ch] = rg[ch];
    }
  }
  // hashgrid.h:285-297
  for (int d = 0; d < 3; d++) {
    R acc = 0;
    for (uint32_t lv = 0; lv < max_level; lv++)
      for (int ch = 0; ch < LD; ch++)
        acc = std::fma(grad_feat[lv * LD + ch], dy_dx[(size_t)d * C + lv * LD + ch], acc);
    dL_dxyz[d] = acc;
  }
}

// glm::dot of two 3-vectors: the products summed left to right.
template <typename R>
inline R dot3(V3<R> a, V3<R> b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
template <typename R>
inline V3<R> add3(V3<R> a, V3<R> b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
template <typename R>
inline V3<R> mul3(V3<R> a, V3<R> b) { return {a.x * b.x, a.y * b.y, a.z * b.z}; }



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
template <typename R>
void render_backward(int W, int H, const uint32_t* ranges, const uint32_t* point_list,
                     const float* means2D, const float* transMat, const float* normal_opacity,
                     const float* homotrans, const float* ap_level, const float* table,
                     const int* offsets, const float* gridrange, int C, int LD, uint32_t L, float S,
                     uint32_t Hres, int align_corners, uint32_t interp, int contract, float beta,
                     const float* final_T, const uint32_t* n_contrib, const float* dL_dout_color,
                     const float* dL_dout_others, R* dL_dtable, R* dL_dtransMat, R* dL_dhomoMat,
                     R* dL_dmean2D, R* dL_dnormal, R* dL_dopacity, R* dL_gradsum, int kernel_type,
                     const float* shapes, R* dL_dshapes, int render_mode, int hybrid_levels,
                     int total_levels, const float* gauss, R* dL_dcolors, int row_stride) {
  using V = V3<R>;
  const int base_mode = render_mode & 0xFF;
  const int pg = hybrid_levels * LD, hd = (int)L * LD, td = total_levels * LD;
  const int gx = (W + kBlock - 1) / kBlock, gy = (H + kBlock - 1) / kBlock;
  const size_t HW = (size_t)H * W;
  const R vmin = gridrange[0], vmax = gridrange[1];
#pragma omp parallel for schedule(dynamic, 1)
  for (int tile = 0; tile < gx * gy; tile++) {
    std::vector<R> dL_dpixel(C), accum_rec(C), last_color(C), grad_feat(C), feat(C);
    std::vector<R> hfeat(hd > 0 ? hd : 1), grad_hash(hd > 0 ? hd : 1);
    const int tx = tile % gx, ty = tile / gx;
    // row_stride > 1: only tile rows ty % row_stride == 0 (a bounded sample; the
    // caller's upstream gradient is zero on the others)
    if (row_stride > 1 && ty % row_stride != 0) continue;
    const uint32_t r0 = ranges[2 * tile], r1 = ranges[2 * tile + 1];
    for (int py = ty * kBlock; py < std::min(H, (ty + 1) * kBlock); py++) {
      for (int px = tx * kBlock; px < std::min(W, (tx + 1) * kBlock); px++) {
        const size_t pid = (size_t)py * W + px;
        const R pxf = (R)px, pyf = (R)py;
        const R T_final = final_T[pid];
        R T = T_final;
        uint32_t contributor = r1 - r0;
        const uint32_t last_contributor = n_contrib[pid];
        const int median_contributor = (int)n_contrib[pid + HW];
        const R dL_ddepth = dL_dout_others[0 * HW + pid];
        const R dL_daccum = dL_dout_others[1 * HW + pid];
        const R dL_dreg = dL_dout_others[6 * HW + pid];
        R dL_dnormal2D[3];
        for (int i = 0; i < 3; i++) dL_dnormal2D[i] = dL_dout_others[(2 + i) * HW + pid];
        const R dL_dmedian_depth = dL_dout_others[5 * HW + pid];
        R last_depth = 0, last_normal[3] = {0, 0, 0};
        R accum_depth_rec = 0, accum_alpha_rec = 0, accum_normal_rec[3] = {0, 0, 0};
        const R final_D = final_T[pid + HW];
        const R final_D2 = final_T[pid + 2 * HW];
        const R final_A = 1 - T_final;
        R last_dL_dT = 0;
        for (int c = 0; c < C; c++) {
          dL_dpixel[c] = dL_dout_color[c * HW + pid];
          accum_rec[c] = 0;
          last_color[c] = 0;
        }
        R last_alpha = 0;
        for (uint32_t k = r1; k-- > r0;) {
          contributor--;
          if (contributor >= last_contributor) continue;
          const uint32_t id = point_list[k];
          const float* Tm = transMat + 9 * (size_t)id;
          const V Tu = {Tm[0], Tm[1], Tm[2]}, Tv = {Tm[3], Tm[4], Tm[5]}, Tw = {Tm[6], Tm[7], Tm[8]};
          const V kk = vsub(vscl(pxf, Tw), Tu);
          const V ll = vsub(vscl(pyf, Tw), Tv);
          const V p = vcrs(kk, ll);
          if (p.z == 0) continue;
          const R sx = p.x / p.z, sy = p.y / p.z;
          const R rho3d = sx * sx + sy * sy;
          const R dx = (R)means2D[2 * id] - pxf, dy = (R)means2D[2 * id + 1] - pyf;
          const R rho2d = R(kFilterInvSquare) * (dx * dx + dy * dy);
          const R rho = std::min(rho3d, rho2d);
          const R c_d = (rho3d <= rho2d) ? (sx * Tw.x + sy * Tw.y) + Tw.z : Tw.z;
          if (c_d < R(kNear)) continue;
          const float* no = normal_opacity + 4 * (size_t)id;
          const R normal[3] = {no[0], no[1], no[2]};
          const R opa = no[3];
          // Splat kernels (backward.cu:765-818): Gaussian (+ beta), beta, flex, general.
          const R shape = kernel_type != 0 ? (R)shapes[id] : R(0);
          R G, G_raw = 0, base = 0, pow_term = 0, rho_safe = 0;
          R demon = 1;
          if (kernel_type == 1) {
            if (rho >= R(1)) continue;
            base = R(1) - rho;
            G = std::pow(base, shape);
          } else if (kernel_type == 2) {
            const R power = R(-0.5) * rho;
            if (power > 0) continue;
            G_raw = std::exp(power);
            G = G_raw;
            if (shape > 0) {
              demon = R(1) + shape * G_raw;
              G = (R(1) + shape) * G_raw / demon;
            }
          } else if (kernel_type == 3) {
            rho_safe = std::max(rho, R(1e-8f));
            pow_term = std::pow(rho_safe, R(0.5) * shape);
            const R power = R(-0.5) * pow_term;
            if (power > 0) continue;
            G = std::exp(power);
          } else {
            const R power = R(-0.5) * rho;
            if (power > 0) continue;
            G = std::exp(power);
            if (beta > 0.0) {
              demon = (R)(1.0 + beta * G);
              G = (R)((1.0 + beta) * G / demon);
            }
          }
          const R alpha = std::min(R(0.99f), opa * G);
          if (alpha < R(1.0f / 255.0f)) continue;

          T = T / (R(1) - alpha);
          const R dchannel_dcolor = alpha * T;
          R dL_dalpha = 0;

          // Hit point and hash features (:934-980).
          const float* h = homotrans + 16 * (size_t)id;
          const V sutu = {h[0], h[4], h[8]}, svtv = {h[1], h[5], h[9]}, pk = {h[3], h[7], h[11]};
          V xyz;
          if (rho3d <= rho2d) {
            xyz = {sx * sutu.x + sy * svtv.x + pk.x, sx * sutu.y + sy * svtv.y + pk.y,
                   sx * sutu.z + sy * svtv.z + pk.z};
          } else {
            xyz = pk;
          }
          R sum_grad = 0;
          for (int c = 0; c < C; c++) {
            grad_feat[c] = dchannel_dcolor * dL_dpixel[c];
            sum_grad += std::fabs(grad_feat[c]);
          }
          const uint32_t apl = (uint32_t)std::floor(ap_level[id]);
          R dL_dxyz[3];
          const bool lvl0 = base_mode == 0 && L == 0;
          // level 0 (backward.cu:833-849): the per-surfel colours' gradient only,
          // no densification sum, no hit-point gradient
          if (!lvl0) atomic_add<R>(&dL_gradsum[id], sum_grad);
          if (lvl0) {
            dL_dxyz[0] = dL_dxyz[1] = dL_dxyz[2] = 0;
            for (int c = 0; c < C; c++) {
              feat[c] = gauss[(size_t)id * C + c];
              atomic_add<R>(&dL_dcolors[(size_t)id * C + c], grad_feat[c]);
            }
          } else if (base_mode == 0 || base_mode == 11) {
            // mode 11 (backward.cu:1372-1424): the hash levels from channel 0 as in
            // mode 0; its SH colour (out_others 14-16) has no gradient here
            query_feature_bw<R>(feat.data(), C, LD, xyz, vmin, vmax, offsets, apl, table, L, S, Hres,
                             align_corners != 0, interp, contract != 0, grad_feat.data(), dL_dtable,
                             dL_dxyz);
          } else if (base_mode >= 8 && base_mode <= 10) {
            // Modes 8 / 9 / 10 (backward.cu:1191-1371), one 3-wide hash level. As
            // the reference computes them, the row and table gradients carry alpha T
            // twice: grad_feat already holds alpha T dL/dC and each case multiplies
            // by alpha T again. The colour term below uses the forward's features
            // (the reference's cases leave `feat` unwritten).
            const int decompose = hybrid_levels;
            const size_t row = (size_t)id * (base_mode == 9 ? 48 : 3);
            const float* g = gauss + row;
            const bool q = L > 0 && decompose != 1;
            R h[3] = {0, 0, 0}, zero[3] = {0, 0, 0}, hgrad[3] = {0, 0, 0}, scratch[3];
            if (q)
              query_feature_bw<R>(h, 3, 3, xyz, vmin, vmax, offsets, apl, table, 1, S, Hres,
                                  align_corners != 0, interp, contract != 0, zero, dL_dtable, scratch);
            const R aT = dchannel_dcolor;
            if (base_mode == 8) {
              for (int c = 0; c < 3; c++) {
                const R gr = std::max(R(0), std::min(R(1), R(g[c]) + R(0.5f)));
                const R hr = R(1) / (R(1) + std::exp(-h[c]));
                const R sum = gr + hr;
                feat[c] = decompose == 2 ? hr : decompose == 1 ? gr : std::max(R(0), std::min(R(1), sum));
                const R gpc = (sum >= 0 && sum <= 1) ? grad_feat[c] : R(0);
                const R v = R(g[c]) + R(0.5f);
                if (decompose != 2) atomic_add<R>(&dL_dcolors[row + c], aT * ((v >= 0 && v <= 1) ? gpc : R(0)));
                hgrad[c] = aT * gpc * hr * (R(1) - hr);
              }
            } else if (base_mode == 10) {
              for (int c = 0; c < 3; c++) {
                const R comb = decompose == 2 ? h[c] : decompose == 1 ? R(g[c]) : R(g[c]) + h[c];
                const R sg = R(1) / (R(1) + std::exp(-comb));
                feat[c] = sg;
                const R gc = grad_feat[c] * sg * (R(1) - sg);
                if (decompose != 2) atomic_add<R>(&dL_dcolors[row + c], aT * gc);
                hgrad[c] = aT * gc;
              }
            } else {
              for (int i = 0; i < 48; i++) {
                feat[i] = g[i];
                if (decompose != 2) atomic_add<R>(&dL_dcolors[row + i], aT * grad_feat[i]);
              }
              for (int c = 0; c < 3; c++) {
                if (decompose == 2) feat[16 * c] = h[c];
                else if (decompose != 1) feat[16 * c] += h[c];
                hgrad[c] = aT * grad_feat[16 * c];
              }
            }
            dL_dxyz[0] = dL_dxyz[1] = dL_dxyz[2] = 0;
            if (q)
              query_feature_bw<R>(scratch, 3, 3, xyz, vmin, vmax, offsets, apl, table, 1, S, Hres,
                                  align_corners != 0, interp, contract != 0, hgrad, dL_dtable, dL_dxyz);
          } else {
            // Render modes 4 / 12 / 14 (backward.cu:987-1033, 1425-1606): the hash
            // levels see the fine channels' gradient times the mode's factor b; the
            // per-surfel rows get theirs in dL_dcolors (blend weight last). The
            // colour term of dL/dalpha below uses the forward's feature vector: the
            // reference's cases 12 and 14 leave `feat` unwritten there.
            R b = 1;
            bool query = L > 0;
            const float* g = nullptr;
            R wgt = 0;
            size_t row = 0;
            if (base_mode == 4) {
              row = (size_t)id * pg;
              g = gauss + row;
            } else if (base_mode == 6) {  // rows of C, hash factor 1/2
              row = (size_t)id * C;
              g = gauss + row;
              b = R(0.5);
            } else if (base_mode == 7) {  // rows of total LD + 1, hash factor 1 - wgt
              row = (size_t)id * (td + 1);
              g = gauss + row;
              wgt = g[td];
              b = R(1) - wgt;
            } else if (base_mode == 12) {
              row = (size_t)id * (td + 1);
              g = gauss + row;
              wgt = g[td];
              b = R(1) - wgt;
            } else {
              row = (size_t)id * (pg + 1);
              g = gauss + row;
              wgt = g[pg];
              b = wgt;
              query = query && wgt > R(1e-6f);
            }
            for (int i = 0; i < hd; i++) grad_hash[i] = b * grad_feat[pg + i];
            dL_dxyz[0] = dL_dxyz[1] = dL_dxyz[2] = 0;
            std::fill(hfeat.begin(), hfeat.end(), R(0));
            if (query)
              query_feature_bw<R>(hfeat.data(), hd, LD, xyz, vmin, vmax, offsets, apl, table, L, S,
                                  Hres, align_corners != 0, interp, contract != 0, grad_hash.data(),
                                  dL_dtable, dL_dxyz);
            std::fill(feat.begin(), feat.end(), R(0));
            for (int c = 0; c < pg; c++) {
              feat[c] = g[c];
              atomic_add<R>(&dL_dcolors[row + c], grad_feat[c]);
            }
            if (base_mode == 4) {
              for (int i = 0; i < hd; i++) feat[pg + i] = hfeat[i];
            } else if (base_mode == 6) {
              // the derivative of the forward (feat = (row + hash) / 2 on the hash
              // levels' channels); the reference's case 6 backward reads a row of
              // 2 L LD values with a per-channel mask its forward does not have
              for (int i = 0; i < hd && i < C; i++) {
                feat[i] = R(0.5) * R(g[i]) + R(0.5) * hfeat[i];
                atomic_add<R>(&dL_dcolors[row + i], R(0.5) * grad_feat[i]);
              }
            } else if (base_mode == 7) {
              // backward.cu:1108-1190: the weight slot gets d_gamma = (row - hash) .
              // grad_feat * wgt (1 - wgt), the pre-sigmoid parameter's gradient
              R dw = 0;
              for (int i = 0; i < td && i < C; i++) {
                const R hv = (L > 0 && i < hd) ? hfeat[i] : R(0);
                feat[i] = wgt * R(g[i]) + (R(1) - wgt) * hv;
                atomic_add<R>(&dL_dcolors[row + i], wgt * grad_feat[i]);
                dw += grad_feat[i] * (R(g[i]) - hv);
              }
              atomic_add<R>(&dL_dcolors[row + td], dw * wgt * (R(1) - wgt));
            } else if (base_mode == 12) {
              R dw = 0;
              if (L > 0) {
                for (int i = 0; i < hd; i++) {
                  feat[pg + i] = wgt * R(g[pg + i]) + (R(1) - wgt) * hfeat[i];
                  atomic_add<R>(&dL_dcolors[row + pg + i], wgt * grad_feat[pg + i]);
                  dw += (R(g[pg + i]) - hfeat[i]) * grad_feat[pg + i];
                }
              }
              atomic_add<R>(&dL_dcolors[row + td], dw);
            } else {
              R dw = 0;
              if (query) {
                for (int i = 0; i < hd; i++) {
                  feat[pg + i] = wgt * hfeat[i];
                  dw += hfeat[i] * grad_feat[pg + i];
                }
              }
              atomic_add<R>(&dL_dcolors[row + pg], dw);
            }
          }
          for (int c = 0; c < C; c++) {
            accum_rec[c] = last_alpha * last_color[c] + (R(1) - last_alpha) * accum_rec[c];
            last_color[c] = feat[c];
            dL_dalpha += (feat[c] - accum_rec[c]) * dL_dpixel[c];
          }

          // Auxiliary maps (:1799-1852).
          R dL_dz = 0;
          R dL_dweight = 0;
          const R m_d = R(kFar) / (R(kFar) - R(kNear)) * (1 - R(kNear) / c_d);
          const R dmd_dd = (R(kFar) * R(kNear)) / ((R(kFar) - R(kNear)) * c_d * c_d);
          if ((int)contributor == median_contributor - 1) dL_dz += dL_dmedian_depth;
          dL_dweight += (final_D2 + m_d * m_d * final_A - 2 * m_d * final_D) * dL_dreg;
          dL_dalpha += dL_dweight - last_dL_dT;
          last_dL_dT = dL_dweight * alpha + (1 - alpha) * last_dL_dT;
          const R dL_dmd = R(2) * (T * alpha) * (m_d * final_A - final_D) * dL_dreg;
          dL_dz += dL_dmd * dmd_dd;
          accum_depth_rec = last_alpha * last_depth + (R(1) - last_alpha) * accum_depth_rec;
          last_depth = c_d;
          dL_dalpha += (c_d - accum_depth_rec) * dL_ddepth;
          accum_alpha_rec = (R)(last_alpha * 1.0 + (R(1) - last_alpha) * accum_alpha_rec);
          dL_dalpha += (1 - accum_alpha_rec) * dL_daccum;
          for (int c = 0; c < 3; c++) {
            accum_normal_rec[c] = last_alpha * last_normal[c] + (R(1) - last_alpha) * accum_normal_rec[c];
            last_normal[c] = normal[c];
            dL_dalpha += (normal[c] - accum_normal_rec[c]) * dL_dnormal2D[c];
            atomic_add<R>(&dL_dnormal[id * 3 + c], alpha * T * dL_dnormal2D[c]);
          }
          dL_dalpha *= T;
          last_alpha = alpha;

          R dL_dG = opa * dL_dalpha;
          // dL/dshape and the kernel's dG/drho (backward.cu:1864-2040).
          R dG_factor = -G;
          if (kernel_type == 1) {
            if (base > R(1e-7f)) atomic_add<R>(&dL_dshapes[id], dL_dalpha * opa * G * std::log(base));
            dG_factor = base > R(1e-7f) ? -shape * G / base : R(0);
          } else if (kernel_type == 2) {
            if (shape > 0) {
              dL_dG *= (R(1) + shape) / (demon * demon);
              atomic_add<R>(&dL_dshapes[id], dL_dalpha * opa * (G_raw * (R(1) - G_raw) / (demon * demon)));
            }
            dG_factor = -G_raw;
          } else if (kernel_type == 3) {
            atomic_add<R>(&dL_dshapes[id], dL_dalpha * opa * (R(-0.25) * G * pow_term * std::log(rho_safe)));
            dG_factor = R(-0.5) * shape * G * pow_term / rho_safe;
          } else if (beta > 0.0) {
            const R dG_dg = (R)((1.0 + beta) / (demon * demon));
            dL_dG *= dG_dg;
          }
          dL_dz += alpha * T * dL_ddepth;

          // homotrans grads (:1921-1953).
          R dL_du = 0, dL_dv = 0;
          R* hm = dL_dhomoMat + (size_t)id * 9;
          if (rho3d <= rho2d) {
            dL_du = dL_dxyz[0] * sutu.x + dL_dxyz[1] * sutu.y + dL_dxyz[2] * sutu.z;
            dL_dv = dL_dxyz[0] * svtv.x + dL_dxyz[1] * svtv.y + dL_dxyz[2] * svtv.z;
            atomic_add<R>(&hm[0], dL_dxyz[0] * sx);
            atomic_add<R>(&hm[1], dL_dxyz[1] * sx);
            atomic_add<R>(&hm[2], dL_dxyz[2] * sx);
            atomic_add<R>(&hm[3], dL_dxyz[0] * sy);
            atomic_add<R>(&hm[4], dL_dxyz[1] * sy);
            atomic_add<R>(&hm[5], dL_dxyz[2] * sy);
          }
          atomic_add<R>(&hm[6], dL_dxyz[0]);
          atomic_add<R>(&hm[7], dL_dxyz[1]);
          atomic_add<R>(&hm[8], dL_dxyz[2]);

          R* tm = dL_dtransMat + (size_t)id * 9;
          if (rho3d <= rho2d) {
            // :1956-2017 (dG_factor per kernel above; -G for the Gaussian).
            R dsx = dL_dG * dG_factor * sx + dL_dz * Tw.x;
            R dsy = dL_dG * dG_factor * sy + dL_dz * Tw.y;
            dsx += dL_du;
            dsy += dL_dv;
            const R dsx_pz = dsx / p.z;
            const R dsy_pz = dsy / p.z;
            const V dL_dp = {dsx_pz, dsy_pz, -(dsx_pz * sx + dsy_pz * sy)};
            const V dL_dk = vcrs(ll, dL_dp);
            const V dL_dl = vcrs(dL_dp, kk);
            atomic_add<R>(&tm[0], -dL_dk.x);
            atomic_add<R>(&tm[1], -dL_dk.y);
            atomic_add<R>(&tm[2], -dL_dk.z);
            atomic_add<R>(&tm[3], -dL_dl.x);
            atomic_add<R>(&tm[4], -dL_dl.y);
            atomic_add<R>(&tm[5], -dL_dl.z);
            atomic_add<R>(&tm[6], pxf * dL_dk.x + pyf * dL_dl.x + dL_dz * sx);
            atomic_add<R>(&tm[7], pxf * dL_dk.y + pyf * dL_dl.y + dL_dz * sy);
            atomic_add<R>(&tm[8], pxf * dL_dk.z + pyf * dL_dl.z + dL_dz * R(1));
          } else {
            // :2018-2045
            const R dG_factor_2d = dG_factor * R(kFilterInvSquare);
            const R dG_ddelx = dG_factor_2d * dx;
            const R dG_ddely = dG_factor_2d * dy;
            atomic_add<R>(&dL_dmean2D[(size_t)id * 3 + 0], dL_dG * dG_ddelx);
            atomic_add<R>(&dL_dmean2D[(size_t)id * 3 + 1], dL_dG * dG_ddely);
            atomic_add<R>(&tm[8], dL_dz);
          }
          atomic_add<R>(&dL_dopacity[id], G * dL_dalpha);
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
template <typename R>
void preprocess_backward(int P, const float* means3D, const float* scales, const float* rotations,
                         const int* radii, const float* transMat, const float* viewmatrix,
                         const float* projmatrix, int width, int height, float tanfovx,
                         float tanfovy, R* dL_dmean2D, const R* dL_dnormal, const R* dL_dtransMat,
                         const R* dL_dhomoMat, R* dL_dmeans3D, R* dL_dscales, R* dL_drots,
                         R* dL_dTs = nullptr) {
  using V = V3<R>;
  const float focal_x = width / (2.0f * tanfovx);
  const float focal_y = height / (2.0f * tanfovy);
  const int W = int(focal_x * tanfovx * 2);
  const int H = int(focal_y * tanfovy * 2);
  const float* pm = projmatrix;
  const float* vm = viewmatrix;
#pragma omp parallel for schedule(static)
  for (int i = 0; i < P; i++) {
    if (!(radii[i] > 0)) continue;
    if (dL_dTs) {
      // Precomputed transforms (scales == NULL, backward.cu:2082-2088, 2128-2158):
      // the render-pass dL/dT plus the centre's mean2D term, written back as the
      // transforms' gradient; nothing reaches means, scales or rotations; the
      // densification statistic reads the updated dL/dT.
      V T[3], dT[3];
      for (int c = 0; c < 3; c++) {
        T[c] = {transMat[9 * i + 3 * c], transMat[9 * i + 3 * c + 1], transMat[9 * i + 3 * c + 2]};
        dT[c] = {dL_dtransMat[9 * i + 3 * c], dL_dtransMat[9 * i + 3 * c + 1], dL_dtransMat[9 * i + 3 * c + 2]};
      }
      const R gmx = dL_dmean2D[3 * i], gmy = dL_dmean2D[3 * i + 1];
      if (gmx != 0 || gmy != 0) {
        const V t_vec = {9, 9, -1};
        const R d = dot3(t_vec, mul3(T[2], T[2]));
        const V f_vec = vscl(R(1) / d, t_vec);
        const V dT0 = mul3(vscl(gmx, f_vec), T[2]);
        const V dT1 = mul3(vscl(gmy, f_vec), T[2]);
        V dT3 = add3(mul3(vscl(gmx, f_vec), T[0]), mul3(vscl(gmy, f_vec), T[1]));
        const V dL_df = add3(mul3(vscl(gmx, T[0]), T[2]), mul3(vscl(gmy, T[1]), T[2]));
        const R dL_dd = (R)(dot3(dL_df, f_vec) * (-1.0 / d));
        dT3 = add3(dT3, vscl(dL_dd, vscl(R(2), mul3(t_vec, T[2]))));
        dT[0] = add3(dT[0], dT0);
        dT[1] = add3(dT[1], dT1);
        dT[2] = add3(dT[2], dT3);
      }
      for (int c = 0; c < 3; c++) {
        dL_dTs[9 * i + 3 * c] = dT[c].x;
        dL_dTs[9 * i + 3 * c + 1] = dT[c].y;
        dL_dTs[9 * i + 3 * c + 2] = dT[c].z;
      }
      for (int k = 0; k < 3; k++) dL_dmeans3D[3 * i + k] = 0;
      for (int k = 0; k < 2; k++) dL_dscales[2 * i + k] = 0;
      for (int k = 0; k < 4; k++) dL_drots[4 * i + k] = 0;
      const R depth = transMat[9 * i + 8];
      dL_dmean2D[3 * i] = (R)((double)(dT[0].z * depth) * 0.5 * (double)(float)W);
      dL_dmean2D[3 * i + 1] = (R)((double)(dT[1].z * depth) * 0.5 * (double)(float)H);
      continue;
    }
    const V p = {means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]};
    const float* qf = rotations + 4 * i;
    const R q[4] = {qf[0], qf[1], qf[2], qf[3]};
    const R sx = scales[2 * i], sy = scales[2 * i + 1];
    // auxiliary.h:218-240 quat_to_rotmat (normalised), as three columns.
    const R s = R(1) / std::sqrt(q[3] * q[3] + q[0] * q[0] + q[1] * q[1] + q[2] * q[2]);
    const R w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    const V Rc[3] = {{R(1) - R(2) * (y * y + z * z), R(2) * (x * y + w * z), R(2) * (x * z - w * y)},
                     {R(2) * (x * y - w * z), R(1) - R(2) * (x * x + z * z), R(2) * (y * z + w * x)},
                     {R(2) * (x * z + w * y), R(2) * (y * z - w * x), R(1) - R(2) * (x * x + y * y)}};
    const V L0 = vscl(sx, Rc[0]), L1 = vscl(sy, Rc[1]), L2 = Rc[2];
    // P = world2ndc * ndc2pix as glm mat3x4: column c, rows 0..3.
    const R n[3][4] = {{R(float(W) / 2.0f), 0, 0, R(float(W - 1) / 2.0f)},
                       {0, R(float(H) / 2.0f), 0, R(float(H - 1) / 2.0f)},
                       {0, 0, 0, 1}};
    R Pm[3][4];
    for (int c = 0; c < 3; c++)
      for (int r = 0; r < 4; r++)
        Pm[c][r] = (((R)pm[4 * r + 0] * n[c][0] + (R)pm[4 * r + 1] * n[c][1]) + (R)pm[4 * r + 2] * n[c][2]) +
                   (R)pm[4 * r + 3] * n[c][3];
    // T = transpose(M) * P, M columns (L0,0), (L1,0), (p,1); T[c][i] = M[i] . P[c].
    const R Mc[3][4] = {{L0.x, L0.y, L0.z, 0}, {L1.x, L1.y, L1.z, 0}, {p.x, p.y, p.z, 1}};
    V T[3];
    for (int c = 0; c < 3; c++) {
      R t[3];
      for (int r = 0; r < 3; r++)
        t[r] = ((Mc[r][0] * Pm[c][0] + Mc[r][1] * Pm[c][1]) + Mc[r][2] * Pm[c][2]) + Mc[r][3] * Pm[c][3];
      T[c] = {t[0], t[1], t[2]};
    }
    // auxiliary.h:105-113 transformVec4x3
    const V normal = {(R)vm[0] * L2.x + (R)vm[4] * L2.y + (R)vm[8] * L2.z,
                      (R)vm[1] * L2.x + (R)vm[5] * L2.y + (R)vm[9] * L2.z,
                      (R)vm[2] * L2.x + (R)vm[6] * L2.y + (R)vm[10] * L2.z};

    V dT[3];
    for (int c = 0; c < 3; c++)
      dT[c] = {dL_dtransMat[9 * i + 3 * c], dL_dtransMat[9 * i + 3 * c + 1], dL_dtransMat[9 * i + 3 * c + 2]};
    const R gmx = dL_dmean2D[3 * i], gmy = dL_dmean2D[3 * i + 1];
    if (gmx != 0 || gmy != 0) {
      const V t_vec = {9, 9, -1};
      const R d = dot3(t_vec, mul3(T[2], T[2]));
      const V f_vec = vscl(R(1) / d, t_vec);
      const V dT0 = mul3(vscl(gmx, f_vec), T[2]);
      const V dT1 = mul3(vscl(gmy, f_vec), T[2]);
      V dT3 = add3(mul3(vscl(gmx, f_vec), T[0]), mul3(vscl(gmy, f_vec), T[1]));
      const V dL_df = add3(mul3(vscl(gmx, T[0]), T[2]), mul3(vscl(gmy, T[1]), T[2]));
      const R dL_dd = (R)(dot3(dL_df, f_vec) * (-1.0 / d));
      const V dd_dT3 = vscl(R(2), mul3(t_vec, T[2]));
      dT3 = add3(dT3, vscl(dL_dd, dd_dT3));
      dT[0] = add3(dT[0], dT0);
      dT[1] = add3(dT[1], dT1);
      dT[2] = add3(dT[2], dT3);
    }
    // dL_dM = P * transpose(dL_dT) + dL_dhomo: column c = sum_k P[k] dL_dT[k][c].
    R dM[3][4];
    for (int c = 0; c < 3; c++) {
      const R g[3] = {(&dT[0].x)[c], (&dT[1].x)[c], (&dT[2].x)[c]};
      for (int r = 0; r < 4; r++)
        dM[c][r] = (Pm[0][r] * g[0] + Pm[1][r] * g[1]) + Pm[2][r] * g[2];
    }
    for (int c = 0; c < 3; c++)
      for (int r = 0; r < 3; r++) dM[c][r] += dL_dhomoMat[9 * i + 3 * c + r];

    // Normal: normalisation backprop as written at :2177-2190, view transform
    // transposed, and the camera-facing flip (DUAL_VISIABLE, :2194-2199).
    const V gn = {dL_dnormal[3 * i], dL_dnormal[3 * i + 1], dL_dnormal[3 * i + 2]};
    const R nlen = std::sqrt(normal.x * normal.x + normal.y * normal.y + normal.z * normal.z);
    V gu = {0, 0, 0};
    if (nlen > R(1e-7f)) {
      const R dgn = gn.x * normal.x + gn.y * normal.y + gn.z * normal.z;
      gu.x = (gn.x - dgn * normal.x / nlen) / nlen;
      gu.y = (gn.y - dgn * normal.y / nlen) / nlen;
      gu.z = (gn.z - dgn * normal.z / nlen) / nlen;
    }
    V dtn = {(R)vm[0] * gu.x + (R)vm[1] * gu.y + (R)vm[2] * gu.z,
             (R)vm[4] * gu.x + (R)vm[5] * gu.y + (R)vm[6] * gu.z,
             (R)vm[8] * gu.x + (R)vm[9] * gu.y + (R)vm[10] * gu.z};
    // auxiliary.h:84-92 transformPoint4x3
    const V pv = {(R)vm[0] * p.x + (R)vm[4] * p.y + (R)vm[8] * p.z + (R)vm[12],
                  (R)vm[1] * p.x + (R)vm[5] * p.y + (R)vm[9] * p.z + (R)vm[13],
                  (R)vm[2] * p.x + (R)vm[6] * p.y + (R)vm[10] * p.z + (R)vm[14]};
    const R cosv = -((pv.x * normal.x + pv.y * normal.y) + pv.z * normal.z);
    const R mult = cosv > 0 ? R(1) : R(-1);
    dtn = vscl(mult, dtn);

    const V dRS0 = {dM[0][0], dM[0][1], dM[0][2]}, dRS1 = {dM[1][0], dM[1][1], dM[1][2]};
    const V dR0 = vscl(sx, dRS0), dR1 = vscl(sy, dRS1), dR2 = dtn;
    // auxiliary.h:243-287 quat_to_rotmat_vjp; v_R[c][r] = column c, row r.
    const R v[3][3] = {{dR0.x, dR0.y, dR0.z}, {dR1.x, dR1.y, dR1.z}, {dR2.x, dR2.y, dR2.z}};
    R* dq = dL_drots + 4 * i;
    dq[0] = R(2) * (x * (v[1][2] - v[2][1]) + y * (v[2][0] - v[0][2]) + z * (v[0][1] - v[1][0]));
    dq[1] = R(2) * (R(-2) * x * (v[1][1] + v[2][2]) + y * (v[0][1] + v[1][0]) +
                    z * (v[0][2] + v[2][0]) + w * (v[1][2] - v[2][1]));
    dq[2] = R(2) * (x * (v[0][1] + v[1][0]) - R(2) * y * (v[0][0] + v[2][2]) +
                    z * (v[1][2] + v[2][1]) + w * (v[2][0] - v[0][2]));
    dq[3] = R(2) * (x * (v[0][2] + v[2][0]) + y * (v[1][2] + v[2][1]) -
                    R(2) * z * (v[0][0] + v[1][1]) + w * (v[0][1] - v[1][0]));
    dL_dscales[2 * i] = dot3(dRS0, Rc[0]);
    dL_dscales[2 * i + 1] = dot3(dRS1, Rc[1]);
    dL_dmeans3D[3 * i] = dM[2][0];
    dL_dmeans3D[3 * i + 1] = dM[2][1];
    dL_dmeans3D[3 * i + 2] = dM[2][2];

    // Densification statistic (:2268-2272), depth = Tw.z of the forward transform.
    const R depth = transMat[9 * i + 8];
    dL_dmean2D[3 * i] = (R)((double)(dL_dtransMat[9 * i + 2] * depth) * 0.5 * (double)(float)W);
    dL_dmean2D[3 * i + 1] = (R)((double)(dL_dtransMat[9 * i + 5] * depth) * 0.5 * (double)(float)H);
  }
}

}  // namespace

// backward.cu:21-140 (computeColorFromSH backward) for one surfel: dL/dsh
// (written, M RGB triples) and the view-direction part of dL/dmean (added),
// with the direction's normalisation through dnormvdv (auxiliary.h:133-143);
// the colour gradient is cut where the forward clamped.
template <typename R>
void sh_color_backward(int deg, int M, const float* sh, V3<R> pos, V3<R> campos, const R dL_drgb_in[3],
                       R* dL_dsh, R dL_dmean[3]) {
  const R C0 = R(0.28209479177387814f), C1 = R(0.4886025119029199f);
  const R C2[5] = {R(1.0925484305920792f), R(-1.0925484305920792f), R(0.31539156525252005f),
                   R(-1.0925484305920792f), R(0.5462742152960396f)};
  const R C3[7] = {R(-0.5900435899266435f), R(2.890611442640554f), R(-0.4570457994644658f),
                   R(0.3731763325901154f), R(-0.4570457994644658f), R(1.445305721320277f),
                   R(-0.5900435899266435f)};
  const V3<R> d0 = {pos.x - campos.x, pos.y - campos.y, pos.z - campos.z};
  const R len = std::sqrt(d0.x * d0.x + d0.y * d0.y + d0.z * d0.z);
  const R x = d0.x / len, y = d0.y / len, z = d0.z / len;
  // clamp of the forward, recomputed
  float rgbf[3];
  bool clamped[3];
  oracle::sh_color(deg, sh, F3{(float)x, (float)y, (float)z}, rgbf, clamped);
  R g[3];
  for (int c = 0; c < 3; c++) g[c] = clamped[c] ? R(0) : dL_drgb_in[c];
  for (int i = 0; i < 3 * M; i++) dL_dsh[i] = 0;
  auto k = [&](int i, int c) { return (R)sh[3 * i + c]; };
  R dx[3] = {0, 0, 0}, dy[3] = {0, 0, 0}, dz[3] = {0, 0, 0};
  auto put = [&](int i, R b) { for (int c = 0; c < 3; c++) dL_dsh[3 * i + c] = b * g[c]; };
  put(0, C0);
  if (deg > 0) {
    put(1, -C1 * y);
    put(2, C1 * z);
    put(3, -C1 * x);
    for (int c = 0; c < 3; c++) {
      dx[c] = -C1 * k(3, c);
      dy[c] = -C1 * k(1, c);
      dz[c] = C1 * k(2, c);
    }
    if (deg > 1) {
      const R xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
      put(4, C2[0] * xy);
      put(5, C2[1] * yz);
      put(6, C2[2] * (R(2) * zz - xx - yy));
      put(7, C2[3] * xz);
      put(8, C2[4] * (xx - yy));
      for (int c = 0; c < 3; c++) {
        dx[c] += C2[0] * y * k(4, c) + C2[2] * R(2) * -x * k(6, c) + C2[3] * z * k(7, c) + C2[4] * R(2) * x * k(8, c);
        dy[c] += C2[0] * x * k(4, c) + C2[1] * z * k(5, c) + C2[2] * R(2) * -y * k(6, c) + C2[4] * R(2) * -y * k(8, c);
        dz[c] += C2[1] * y * k(5, c) + C2[2] * R(2) * R(2) * z * k(6, c) + C2[3] * x * k(7, c);
      }
      if (deg > 2) {
        put(9, C3[0] * y * (R(3) * xx - yy));
        put(10, C3[1] * xy * z);
        put(11, C3[2] * y * (R(4) * zz - xx - yy));
        put(12, C3[3] * z * (R(2) * zz - R(3) * xx - R(3) * yy));
        put(13, C3[4] * x * (R(4) * zz - xx - yy));
        put(14, C3[5] * z * (xx - yy));
        put(15, C3[6] * x * (xx - R(3) * yy));
        for (int c = 0; c < 3; c++) {
          dx[c] += C3[0] * k(9, c) * R(3) * R(2) * xy + C3[1] * k(10, c) * yz + C3[2] * k(11, c) * R(-2) * xy +
                   C3[3] * k(12, c) * R(-3) * R(2) * xz + C3[4] * k(13, c) * (R(-3) * xx + R(4) * zz - yy) +
                   C3[5] * k(14, c) * R(2) * xz + C3[6] * k(15, c) * R(3) * (xx - yy);
          dy[c] += C3[0] * k(9, c) * R(3) * (xx - yy) + C3[1] * k(10, c) * xz +
                   C3[2] * k(11, c) * (R(-3) * yy + R(4) * zz - xx) + C3[3] * k(12, c) * R(-3) * R(2) * yz +
                   C3[4] * k(13, c) * R(-2) * xy + C3[5] * k(14, c) * R(-2) * yz + C3[6] * k(15, c) * R(-3) * R(2) * xy;
          dz[c] += C3[1] * k(10, c) * xy + C3[2] * k(11, c) * R(4) * R(2) * yz +
                   C3[3] * k(12, c) * R(3) * (R(2) * zz - xx - yy) + C3[4] * k(13, c) * R(4) * R(2) * xz +
                   C3[5] * k(14, c) * (xx - yy);
        }
      }
    }
  }
  const R ddx = dx[0] * g[0] + dx[1] * g[1] + dx[2] * g[2];
  const R ddy = dy[0] * g[0] + dy[1] * g[1] + dy[2] * g[2];
  const R ddz = dz[0] * g[0] + dz[1] * g[1] + dz[2] * g[2];
  const R sum2 = d0.x * d0.x + d0.y * d0.y + d0.z * d0.z;
  const R inv32 = R(1) / std::sqrt(sum2 * sum2 * sum2);
  dL_dmean[0] += ((sum2 - d0.x * d0.x) * ddx - d0.y * d0.x * ddy - d0.z * d0.x * ddz) * inv32;
  dL_dmean[1] += (-d0.x * d0.y * ddx + (sum2 - d0.y * d0.y) * ddy - d0.z * d0.y * ddz) * inv32;
  dL_dmean[2] += (-d0.x * d0.z * ddx - d0.y * d0.z * ddy + (sum2 - d0.z * d0.z) * ddz) * inv32;
}

template <typename R>
void sh_color_backward_all(int P, int deg, int M, const float* means3D, const float* campos, const float* shs,
                           const int* radii, const R* dL_drgb, R* dL_dshs, R* dL_dmeans) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < P; i++) {
    R* dsh = dL_dshs + (size_t)i * M * 3;
    if (!(radii[i] > 0)) {
      for (int j = 0; j < 3 * M; j++) dsh[j] = 0;
      continue;
    }
    const V3<R> pos = {means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]};
    const V3<R> cp = {campos[0], campos[1], campos[2]};
    sh_color_backward<R>(deg, M, shs + (size_t)i * M * 3, pos, cp, dL_drgb + 3 * (size_t)i, dsh,
                         dL_dmeans + 3 * (size_t)i);
  }
}

extern "C" {

// SH colour backward of P surfels (preprocess backward, backward.cu:2267 with
// computeColorFromSH, :21-140): dL_dshs [P, M, 3] written (zero where radii <=
// 0), dL_dmeans [P, 3] added to.
void oracle_sh_color_backward(int P, int deg, int M, const float* means3D, const float* campos, const float* shs,
                              const int* radii, const float* dL_drgb, float* dL_dshs, float* dL_dmeans) {
  sh_color_backward_all<float>(P, deg, M, means3D, campos, shs, radii, dL_drgb, dL_dshs, dL_dmeans);
}
void oracle_sh_color_backward_f64(int P, int deg, int M, const float* means3D, const float* campos,
                                  const float* shs, const int* radii, const double* dL_drgb, double* dL_dshs,
                                  double* dL_dmeans) {
  sh_color_backward_all<double>(P, deg, M, means3D, campos, shs, radii, dL_drgb, dL_dshs, dL_dmeans);
}

// Working precision float: the reference's arithmetic, the parity checker.
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
                            float* dL_gradsum, int kernel_type, const float* shapes,
                            float* dL_dshapes, int render_mode, int hybrid_levels,
                            int total_levels, const float* gauss, float* dL_dcolors,
                            int row_stride) {
  render_backward<float>(W, H, ranges, point_list, means2D, transMat, normal_opacity, homotrans,
                         ap_level, table, offsets, gridrange, C, LD, L, S, Hres, align_corners,
                         interp, contract, beta, final_T, n_contrib, dL_dout_color, dL_dout_others,
                         dL_dtable, dL_dtransMat, dL_dhomoMat, dL_dmean2D, dL_dnormal, dL_dopacity,
                         dL_gradsum, kernel_type, shapes, dL_dshapes, render_mode, hybrid_levels,
                         total_levels, gauss, dL_dcolors, row_stride);
}

// Working precision double: the same formulas and decisions, without float
// rounding; measures how far any float32 evaluation (the reference's, this
// file's float instance, the CUDA kernels) sits from its exact value.
void oracle_render_backward_f64(int W, int H, const uint32_t* ranges, const uint32_t* point_list,
                                const float* means2D, const float* transMat,
                                const float* normal_opacity, const float* homotrans,
                                const float* ap_level, const float* table, const int* offsets,
                                const float* gridrange, int C, int LD, uint32_t L, float S,
                                uint32_t Hres, int align_corners, uint32_t interp, int contract,
                                float beta, const float* final_T, const uint32_t* n_contrib,
                                const float* dL_dout_color, const float* dL_dout_others,
                                double* dL_dtable, double* dL_dtransMat, double* dL_dhomoMat,
                                double* dL_dmean2D, double* dL_dnormal, double* dL_dopacity,
                                double* dL_gradsum, int kernel_type, const float* shapes,
                                double* dL_dshapes, int render_mode, int hybrid_levels,
                                int total_levels, const float* gauss, double* dL_dcolors,
                                int row_stride) {
  render_backward<double>(W, H, ranges, point_list, means2D, transMat, normal_opacity, homotrans,
                          ap_level, table, offsets, gridrange, C, LD, L, S, Hres, align_corners,
                          interp, contract, beta, final_T, n_contrib, dL_dout_color,
                          dL_dout_others, dL_dtable, dL_dtransMat, dL_dhomoMat, dL_dmean2D,
                          dL_dnormal, dL_dopacity, dL_gradsum, kernel_type, shapes, dL_dshapes,
                          render_mode, hybrid_levels, total_levels, gauss, dL_dcolors, row_stride);
}

void oracle_preprocess_backward(int P, const float* means3D, const float* scales,
                                const float* rotations, const int* radii, const float* transMat,
                                const float* viewmatrix, const float* projmatrix, int width,
                                int height, float tanfovx, float tanfovy, float* dL_dmean2D,
                                const float* dL_dnormal, const float* dL_dtransMat,
                                const float* dL_dhomoMat, float* dL_dmeans3D, float* dL_dscales,
                                float* dL_drots) {
  preprocess_backward<float>(P, means3D, scales, rotations, radii, transMat, viewmatrix, projmatrix,
                             width, height, tanfovx, tanfovy, dL_dmean2D, dL_dnormal, dL_dtransMat,
                             dL_dhomoMat, dL_dmeans3D, dL_dscales, dL_drots);
}

// Precomputed transforms: dL_dTs [P, 9] written (transMat = the forward's
// transforms, i.e. the given ones); means, scales and rotations get zeros.
void oracle_preprocess_backward_precomp(int P, const int* radii, const float* transMat, int width, int height,
                                        float tanfovx, float tanfovy, float* dL_dmean2D,
                                        const float* dL_dtransMat, float* dL_dTs, float* dL_dmeans3D,
                                        float* dL_dscales, float* dL_drots) {
  preprocess_backward<float>(P, nullptr, nullptr, nullptr, radii, transMat, nullptr, nullptr, width, height,
                             tanfovx, tanfovy, dL_dmean2D, nullptr, dL_dtransMat, nullptr, dL_dmeans3D,
                             dL_dscales, dL_drots, dL_dTs);
}
void oracle_preprocess_backward_precomp_f64(int P, const int* radii, const float* transMat, int width,
                                            int height, float tanfovx, float tanfovy, double* dL_dmean2D,
                                            const double* dL_dtransMat, double* dL_dTs, double* dL_dmeans3D,
                                            double* dL_dscales, double* dL_drots) {
  preprocess_backward<double>(P, nullptr, nullptr, nullptr, radii, transMat, nullptr, nullptr, width, height,
                              tanfovx, tanfovy, dL_dmean2D, nullptr, dL_dtransMat, nullptr, dL_dmeans3D,
                              dL_dscales, dL_drots, dL_dTs);
}

void oracle_preprocess_backward_f64(int P, const float* means3D, const float* scales,
                                    const float* rotations, const int* radii,
                                    const float* transMat, const float* viewmatrix,
                                    const float* projmatrix, int width, int height, float tanfovx,
                                    float tanfovy, double* dL_dmean2D, const double* dL_dnormal,
                                    const double* dL_dtransMat, const double* dL_dhomoMat,
                                    double* dL_dmeans3D, double* dL_dscales, double* dL_drots) {
  preprocess_backward<double>(P, means3D, scales, rotations, radii, transMat, viewmatrix,
                              projmatrix, width, height, tanfovx, tanfovy, dL_dmean2D, dL_dnormal,
                              dL_dtransMat, dL_dhomoMat, dL_dmeans3D, dL_dscales, dL_drots);
}

// Per-point query_feature<true> (hashgrid.h:106-299) with a given upstream
// gradient: grad_feat [n, C] in, table gradient accumulated into dL_dtable
// ([rows, LD], caller-zeroed) and dL/dxyz [n, 3] out. Serial (the table
// gradient's float additions in point order). level_exp2 as oracle_query.
void oracle_query_backward(int n, const float* xyz, const uint32_t* ap_level, const float* table,
                           const int* offsets, float vmin, float vmax, int C, int LD, uint32_t L,
                           float S, uint32_t Hres, int align_corners, uint32_t interp, int contract,
                           const float* level_exp2, const float* grad_feat, float* dL_dtable,
                           float* dL_dxyz) {
  std::vector<float> feat((size_t)C);
  for (int i = 0; i < n; i++) {
    const V3<float> p{xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2]};
    query_feature_bw<float>(feat.data(), C, LD, p, vmin, vmax, offsets, ap_level[i], table, L, S,
                            Hres, align_corners != 0, interp, contract != 0,
                            grad_feat + (size_t)i * C, dL_dtable, dL_dxyz + 3 * (size_t)i,
                            level_exp2);
  }
}

}  // extern "C"
