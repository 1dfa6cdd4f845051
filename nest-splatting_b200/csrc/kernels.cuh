// kernels.cuh -- internal launch interfaces shared by the .cu files of
// libnest_b200.so (not part of the public C-ABI).
#pragma once

#include "common.cuh"

namespace ns {
// The render modes that put the hash levels after hybrid_levels per-surfel
// levels (4 cat, 12-14 adaptive_cat / _fast / adaptive_zero); in modes 6 and 7
// (adaptive, adaptive_add) the hash levels start at channel 0, as in mode 0.
__host__ __device__ inline int hash_level_offset(int render_mode, int hybrid_levels) {
  const int base = render_mode & 0xFF;
  return (base == 4 || base == 12 || base == 13 || base == 14) ? hybrid_levels : 0;
}
// Samples read per-surfel rows (colors_precomp) in every mode but 0, and in
// mode 0 with no hash level (level 0: per-surfel colours, forward.cu:1093-1096).
__host__ __device__ inline bool uses_surfel_rows(int render_mode, uint32_t levels) {
  return render_mode != 0 || levels == 0;
}

struct RenderParams {
  int W, H;
  int C, LD;
  uint32_t L;
  float S;
  uint32_t Hres;
  int align_corners;
  uint32_t interp;
  int contract;
  float beta;
  int kernel_type;  // 0 Gaussian, 1 beta, 2 flex, 3 general (record word q7.w = shape)
  // Render modes 4 / 12 / 14 (render_mode = base | inference flag << 8): the
  // per-surfel features `gauss` (colors_precomp rows) fill channels from 0 and
  // the L hash levels land at level hybrid_levels (channel hybrid_levels * LD).
  int render_mode;
  int hybrid_levels;
  int total_levels;
  const float* gauss;
  uint32_t max_intersections;
  int record_transmittance;
  const uint2* ranges;
  const uint32_t* tile_order;  // blockIdx.x -> tile (heaviest first), or NULL: row-major
  const uint32_t* point_list;
  const SurfelRecord* records;
  const void* table;
  const int32_t* offsets;
  const float* gridrange;
  float* out_color;
  float* out_others;
  float* final_T;
  uint32_t* n_contrib;
  float* cover_pixels;
  float* trans_avg;
  uint32_t* err;  // device status word (kErr* bits)
  uint32_t spin_limit;  // poll bound of the record-ring waits
};
struct BackwardParams {
  int W, H;
  int C, LD;
  uint32_t L;
  float S;
  uint32_t Hres;
  int align_corners;
  uint32_t interp;
  int contract;
  float beta;
  int kernel_type;            // splat kernel 0-3; 1-3 read the shape in record word 31
  int render_mode;            // 0, or 4 / 12 / 14 (training rules) as in RenderParams
  int hybrid_levels;
  int total_levels;
  const float* gauss;         // per-surfel rows of the render modes
  float* dL_dcolors;          // their gradient (same layout), accumulated
  int Wq, Hq;                 // image size as the reference's preprocess backward recomputes it
  const float* projmatrix;
  const float* viewmatrix;
  int ray_hit;                // 1: hit-point gradient in the ray/plane form (see backward.cu)
  int raw_T;                  // 1: precomputed transforms, accumulate dL/dT itself (not folded into dL/dM)
  const uint2* ranges;
  const uint32_t* tile_order;  // blockIdx.x -> tile (heaviest first), or NULL: row-major
  const uint32_t* point_list;
  const SurfelRecord* records;
  const void* table;
  const int32_t* offsets;
  const float* gridrange;
  const float* final_T;
  const uint32_t* n_contrib;
  const float* dL_dcolor;
  const float* dL_dothers;
  float* dL_dtable;
  unsigned long long* dL_dtable_fixed;  // non-null: fixed-point table gradient (deterministic)
  const uint32_t* grad_max_bits;        // max |dL/dcolor| as float bits (deterministic)
  float* accum;
};
size_t backward_accum_bytes(int64_t P);
// SH colours of the level-0 path (sh.cu): rgb [P, 3] from shs [P, M, 3]; the
// backward writes dL_dshs and adds to dL_dmeans (surfels with radii > 0).
int sh_color_launch(int P, int deg, int M, const float* means, const float* campos, const float* shs, float* rgb,
                    cudaStream_t stream);
int sh_color_backward_launch(int P, int deg, int M, const float* means, const float* campos, const float* shs,
                             const int32_t* radii, const float* dL_drgb, float* dL_dshs, float* dL_dmeans,
                             cudaStream_t stream);
int table_grad_max_launch(const float* dL_dcolor, size_t n, uint32_t* gmax, cudaStream_t stream);
int table_grad_finish_launch(const unsigned long long* fx, size_t n, const uint32_t* gmax, float* out,
                             cudaStream_t stream);
int blend_backward_launch(const BackwardParams& p, int fp16, cudaStream_t stream);
int preprocess_backward_launch(int P, const float* means3D, const float* scales,
                               const float* rotations, const int32_t* radii, const float* vm,
                               const float* pm, int Wq, int Hq, const float* accum, const float* Ts,
                               const ns_raster_grads_out& o, cudaStream_t stream);
int rvq_decode_launch(const uint8_t*, const float*, float*, int64_t, int, int, int, cudaStream_t);
int wait_selftest_launch(const uint32_t* flag, uint32_t* err, cudaStream_t stream);
int tile_order_launch(const uint2* ranges, int tiles, uint32_t* order, cudaStream_t stream);
int preprocess_blocks(int P);
int preprocess_block_size();
int preprocess_api_launch(int P, const ns_surfels& s, float mod, float beta, int kernel_type,
                          const float* vm,
                          const float* pm, int W, int H, SurfelRecord* records, BinInfo* bin,
                          int32_t* radii, uint32_t* tiles, uint32_t* depth_keys,
                          uint32_t* depth_vals, uint32_t* block_sums, cudaStream_t stream);
int preprocess_mix_launch(int P, const float* base, const float* decoded, int dims, float mix,
                          const float* ap_level, float mod, float beta, const float* vm,
                          const float* pm, int W, int H, SurfelRecord* records, BinInfo* bin,
                          int32_t* radii, uint32_t* tiles, uint32_t* depth_keys,
                          uint32_t* depth_vals, uint32_t* block_sums, cudaStream_t stream);
int mark_visible_launch(int P, const float* means3D, const float* vm, uint8_t* present,
                        cudaStream_t stream);
int scan_block_sums_launch(const uint32_t* sums, uint32_t* prefix, int nb, int64_t* total,
                           cudaStream_t stream);
int duplicate_keys_launch(int P, const uint32_t* order, const BinInfo* bin, const uint32_t* tiles,
                          uint32_t* sorted_sums, uint32_t* sorted_prefix, int64_t* total, int gx,
                          uint32_t* keys, uint32_t* vals, int64_t capacity, uint32_t* err,
                          cudaStream_t stream);
int identify_ranges_launch(const uint32_t* keys, const int64_t* count_dev, int64_t count_host,
                           int64_t capacity, uint2* ranges, int tiles, int sms,
                           cudaStream_t stream);
size_t radix_sort_temp_bytes(int64_t n);
int radix_sort_launch(const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                      uint32_t* vals_out, uint64_t* keys_alt, uint32_t* vals_alt, int64_t n,
                      int end_bit, void* temp, size_t temp_bytes, cudaStream_t stream);
int radix_sort32_launch(const uint32_t* keys_in, const uint32_t* vals_in, uint32_t* keys_out,
                        uint32_t* vals_out, uint32_t* keys_alt, uint32_t* vals_alt, int64_t n,
                        int end_bit, void* temp, size_t temp_bytes, cudaStream_t stream,
                        const int64_t* n_dev = nullptr);
uint32_t* radix_sort_error_word(void* temp);
int render_launch(const RenderParams& p, int fp16, cudaStream_t stream);
int mlp_launch(const float* feat, int in_dims, int64_t npix, const uint16_t* weights, int hidden,
               int out_dims, const float* alpha, const float* bg_host, float* rgb,
               cudaStream_t stream);
int mlp_backward_launch(const float* feat, int in_dims, int64_t npix, const uint16_t* weights,
                        int hidden, int out_dims, const float* alpha, const float* grgb,
                        float* dfeat, float* dW, cudaStream_t stream);
int allmap_decode_launch(const float* allmap, const float* vm, const float* rays_d,
                         const float* ray_o, int W, int H, float depth_ratio, float* out,
                         cudaStream_t stream);
int normal_error_launch(const float* allmap, const float* vm, const float* rays_d,
                        const float* ray_o, int W, int H, float* err, cudaStream_t stream);
int normal_error_backward_launch(const float* allmap, const float* vm, const float* rays_d,
                                 const float* ray_o, int W, int H, const float* derr,
                                 int64_t derr_stride, float* dallmap, float* dstencil,
                                 cudaStream_t stream);
}  // namespace ns
