/*
 * nest_b200.h -- C-ABI of the B200-native (sm_100a) nest-splatting render path.
 *
 * Plain pointers and sizes only: every buffer is caller-owned device memory
 * unless a parameter says "host". No entry point allocates device memory, none
 * throws, none traps: each returns an ns_status code. Kernels are enqueued on
 * the caller's stream (a cudaStream_t passed as void*; NULL = legacy default).
 *
 * Reference interfaces replaced (paths inside NilKel/nest-splatting):
 *   ns_rasterize_forward  <- RasterizeGaussiansCUDA
 *                            submodules/diff-surfel-rasterization/rasterize_points.cu:39-242
 *                            and CudaRasterizer::Rasterizer::forward
 *                            .../cuda_rasterizer/rasterizer_impl.cu:255-440 (render_mode
 *                            0, 4, 12-14; forward.cu:639-2049)
 *   ns_mark_visible       <- markVisible, rasterize_points.cu:452-471 and
 *                            rasterizer_impl.cu:54-66,198-210
 *   ns_mlp_forward        <- INGP.rgb_decode / get_color, hash_encoder/modules.py:587-602
 *                            (tiny-cuda-nn "MLP", no biases, sigmoid on the output)
 *   ns_rvq_decode         <- no reference counterpart: the RVQ attribute decode of
 *                            the benchmark config-0 definition (new scope)
 *   ns_render_frame       <- gaussian_renderer/__init__.py:render() baseline branch
 *                            (:178-213, 694-797, 905-1021) fused with an RVQ attribute
 *                            decode: decode -> activate -> rasterize -> MLP -> mask/bg
 *   ns_radix_sort_pairs   <- cub::DeviceRadixSort::SortPairs as called at
 *                            rasterizer_impl.cu:381-386 (stable, bits [0, end_bit))
 *   ns_rasterize_backward <- RasterizeGaussiansBackwardCUDA, rasterize_points.cu:244-450,
 *                            and CudaRasterizer::Rasterizer::backward,
 *                            rasterizer_impl.cu:444-592 (BACKWARD::render,
 *                            backward.cu:445-2052; BACKWARD::preprocess, :2216-2273)
 *   ns_mlp_backward       <- tiny-cuda-nn's backward of the same MLP (autograd of
 *                            INGP.get_color in the training step, train.py:651)
 *   ns_allmap_decode      <- the render_pkg maps of gaussian_renderer/__init__.py
 *                            :763-797,1035-1045 (rend_normal, depth_expected,
 *                            depth_median, surf_depth, surf_normal)
 *   ns_normal_error       <- the depth-normal term of the 2DGS training loss:
 *                            gaussian_renderer/__init__.py:763-792 (allmap decode,
 *                            depth_ratio 0), utils/point_utils.py:10-30,48-60
 *                            (depths_to_points, depth_to_normal), train.py:674-675
 *   ns_normal_error_backward <- torch autograd of the same expressions
 *   ns_grid_encode_forward   <- grid_encode_forward, gridencoder/src/gridencoder.h:9 and
 *                               gridencoder.cu:450-473 (kernel_grid, :88-242)
 *   ns_grid_encode_backward  <- grid_encode_backward, gridencoder/src/gridencoder.h:10 and
 *                               gridencoder.cu:475-505 (kernel_grid_backward, :246-338;
 *                               kernel_input_backward, :341-367)
 */
#ifndef NEST_B200_H_
#define NEST_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ns_status {
  NS_OK = 0,
  NS_ERR_INVALID = 1,      /* a pointer, size or shape argument is invalid */
  NS_ERR_UNSUPPORTED = 2,  /* channel / level-dim combination or mode not built */
  NS_ERR_CAPACITY = 3,     /* binning scratch too small: *num_rendered holds the need */
  NS_ERR_CUDA = 4,         /* a CUDA runtime call failed (see ns_last_cuda_error) */
  NS_ERR_SCRATCH = 5,      /* a scratch buffer is smaller than ns_*_scratch_bytes() */
  NS_ERR_DEVICE = 6        /* a kernel recorded an error word (bounded wait ran out,
                              instance count above capacity in device-count mode) */
} ns_status;

const char* ns_status_string(int status);
/* Number of kernels this library has launched in the calling process. */
uint64_t ns_kernel_launches(void);
/* cudaError_t of the last failing CUDA call made by this library (0 if none). */
int ns_last_cuda_error(void);
int ns_version(void);

/* ------------------------------------------------------------------ settings */

/* Mirrors GaussianRasterizationSettings + HashGridSettings
 * (diff_surfel_rasterization/__init__.py:277-302). */
typedef struct ns_raster_settings {
  int32_t image_height;
  int32_t image_width;
  float tanfovx;
  float tanfovy;
  float scale_modifier;
  const float* viewmatrix; /* device [16], world_view_transform (row-vector layout) */
  const float* projmatrix; /* device [16], full_proj_transform */
  float beta;              /* kernel sharpening; 0 = plain Gaussian */
  int32_t if_contract;     /* scene contraction in the hash lookup */
  int32_t record_transmittance;
  uint32_t max_intersections; /* 0 = no limit */
  int32_t prefiltered;
  /* HashGridSettings */
  uint32_t levels;            /* L (active levels) */
  float level_scale_log2;     /* S = log2(per_level_scale) */
  uint32_t base_resolution;   /* H */
  int32_t align_corners;
  uint32_t interpolation;     /* 0 linear, 1 smoothstep */
  uint32_t channels;          /* C = shape_dims[2], output feature channels */
  uint32_t level_dim;         /* LD = features.size(1) */
  int32_t table_fp16;         /* 1: features are fp16, 0: fp32 */
  /* Splat kernel (forward.cu:864-919): 0 Gaussian (with beta above), 1 beta
   * kernel alpha = o (1 - rho)^shape for rho < 1, 2 flex (per-surfel beta =
   * shape), 3 general G = exp(-0.5 rho^(shape / 2)); 1-3 read ns_surfels.shapes.
   * ns_render_frame takes kernel 0. */
  int32_t kernel_type;
  /* Backward only. 1: the hash-table gradient is reduced in 64-bit fixed point
   * (2^32 / 2^ceil(log2 max|dL_dout_color|) units), so it is bit-identical from
   * run to run; needs ns_backward_scratch_bytes_deterministic. 0: float atomics,
   * whose summation order varies, as in the reference. */
  int32_t deterministic;
  /* Render mode (forward.cu:964-1824; base | inference flag << 8): 0 baseline
   * hash grid (levels 0: per-surfel colours); 4 cat: per-surfel features
   * (hybrid_levels levels) then the hash grid's `levels` levels; 6 adaptive
   * and 7 adaptive_add: per-surfel rows blended with the hash levels; 12
   * adaptive_cat, 13 adaptive_cat_fast and 14 adaptive_zero: per-surfel
   * features blended with the hash levels by a per-surfel weight (flag 256:
   * inference rules). hybrid_levels / total_levels: the reference's level
   * encoding (total << 16 | active << 8 | hybrid) split out; `levels` is the
   * number of hash levels queried. 8 hybrid_SH, 9 hybrid_SH_post, 10
   * hybrid_SH_raw (:1378-1526): one hash level of level_dim 3, channels 3 (48
   * for mode 9), the level word decompose << 24 | SH degree << 16 | 1 << 8 split
   * as hybrid_levels = decompose flag (0 both parts, 1 the surfel only, 2 the
   * grid only), total_levels = SH degree, levels = 1. 11 residual_hybrid
   * (:1527-1592): the hash levels from channel 0 (channels + 3 <= 32) and the
   * rows' degree-3 SH colour in out_others channels 14-16. The dual-grid modes
   * 1-3 and 5 report NS_ERR_UNSUPPORTED. ns_rasterize_backward takes every
   * built mode but 13 without the inference flag (training rules; the
   * reference has no mode-13 backward); ns_render_frame takes 0. */
  int32_t render_mode;
  uint32_t hybrid_levels;
  uint32_t total_levels;
  /* SH colours (forward.cu:414-423, computeColorFromSH :21-74): with render_mode
   * 0, levels 0, channels 3, ns_surfels.colors_precomp NULL and ns_surfels.shs
   * set, the surfels' colours are their degree-sh_degree (0-3) SH along the
   * unit direction from campos (device [3], the camera centre) to the mean,
   * + 0.5, clamped at 0; the backward returns dL/dshs and adds the colour's
   * part of dL/dmeans3D. */
  int32_t sh_degree;
  const float* campos;
} ns_raster_settings;

/* Per-surfel inputs of the rasterizer. */
typedef struct ns_surfels {
  int32_t P;
  const float* means3D;   /* [P,3] */
  const float* scales;    /* [P,2] activated (exp) scales */
  const float* rotations; /* [P,4] unit quaternions (w,x,y,z) */
  const float* opacities; /* [P] activated opacity */
  const float* homotrans; /* [P,16] build_H output, or NULL: computed from the above */
  const float* ap_level;  /* [P] appearance level, or NULL: all levels */
  const void* features;   /* hash table [sum_l T_l, LD], fp32 or fp16 */
  const int32_t* offsets; /* [L+1] int32 level offsets (rows) */
  const float* gridrange; /* [2] = (vmin, vmax) */
  const float* shapes;    /* [P] per-surfel kernel parameter for kernel_type 1-3, else NULL */
  const float* colors_precomp; /* render modes other than 0, and level 0: per-surfel
                                  rows (the reference's colors_precomp): mode 4
                                  [P, hybrid LD], 6 and level 0 [P, C], 7 and 12 / 13
                                  [P, total LD + 1], 14 [P, hybrid LD + 1] (blend
                                  weight last), 8 / 10 [P, 3] raw SH colours, 9 and
                                  11 [P, 48] SH coefficients (mode 11 reads them
                                  interleaved, coefficient k of channel c at 3 k + c,
                                  as the reference's kernel does); else NULL */
  const float* shs;       /* [P, sh_coeffs, 3] SH coefficients (RGB triples per
                             coefficient), read for the level-0 SH colours, else NULL */
  int32_t sh_coeffs;      /* M >= (sh_degree + 1)^2 */
  const float* transmat_precomp; /* [P, 9] precomputed splat-to-pixel transforms (columns
                             Tu, Tv, Tw; the reference's transMat_precomp /
                             cov3D_precomp, forward.cu:366-380), else NULL: with
                             them scales and rotations may be NULL, homotrans is
                             required, the normal is the view axis and the
                             backward writes dL_dtransmat_precomp instead of mean,
                             scale and rotation gradients (zeros) */
} ns_surfels;

/* Outputs (caller-owned, device). cover_pixels / trans_avg may be NULL when
 * record_transmittance is 0; they are accumulated into (zero them first). */
typedef struct ns_raster_outputs {
  float* out_color;   /* [C,H,W] composited features */
  float* out_others;  /* [14,H,W] depth, alpha, normal(3), median depth, distortion,
                         count, position(3), level colour(3); [17,H,W] in render
                         mode 11, whose SH colour fills channels 14-16 (the
                         reference writes them past its 14-channel buffer,
                         rasterize_points.cu:159-163, forward.cu:2039-2045) */
  int32_t* radii;     /* [P] */
  float* cover_pixels;/* [P] or NULL */
  float* trans_avg;   /* [P] or NULL */
} ns_raster_outputs;

/* ----------------------------------------------------------- scratch sizes */

/* Per-surfel state kept between forward and backward (the reference geomBuffer). */
size_t ns_geometry_scratch_bytes(int32_t P);
/* Per-image state (the reference imgBuffer): tile ranges, final T, contributor counts. */
size_t ns_image_scratch_bytes(int32_t width, int32_t height);
/* Key/value sort state for up to max_instances surfel/tile pairs (the binningBuffer). */
size_t ns_binning_scratch_bytes(int64_t max_instances);

/* ------------------------------------------------------------- rasterizer */

#define NS_FLAG_DEVICE_COUNT 1 /* do not read the instance count back to the host;
                                  size the sort by the binning capacity instead.
                                  Overflow is reported as NS_ERR_DEVICE by
                                  ns_read_device_status. */

/* Forward rasterization: render_mode 0 (baseline hash grid; levels 0: per-surfel
 * colours) or 4 / 6-14 (settings->render_mode), splat kernel settings->kernel_type.
 * geom/image/binning are scratch buffers of at least the ns_*_scratch_bytes size.
 * num_rendered (host, may be NULL): number of surfel/tile instances. Without
 * NS_FLAG_DEVICE_COUNT the call synchronises the stream once to read it and
 * returns NS_ERR_CAPACITY (nothing rendered) when binning is too small. */
int ns_rasterize_forward(const ns_raster_settings* settings, const ns_surfels* surfels,
                         const ns_raster_outputs* outputs, void* geom, size_t geom_bytes,
                         void* binning, size_t binning_bytes, void* image, size_t image_bytes,
                         int64_t* num_rendered, int flags, void* stream);

/* Gradients arriving at the forward outputs. */
typedef struct ns_raster_grads_in {
  const float* dL_dout_color;   /* [channels, H, W] */
  const float* dL_dout_others;  /* [14, H, W] (or mode 11's 17); channels 0-6 carry
                                   gradient (depth, alpha, normal x3, median depth,
                                   distortion) */
  const int32_t* radii;         /* [P] as written by the forward call */
} ns_raster_grads_in;

/* Gradients produced by the backward pass (every pointer required). Per-surfel
 * arrays are written for all P surfels (zero where radii <= 0); dL_dtable is
 * zeroed by the call and then accumulated. */
typedef struct ns_raster_grads_out {
  float* dL_dmeans3D;   /* [P,3] */
  float* dL_dmean2D;    /* [P,3] screen-space densification statistic (the
                           reference's means2D gradient, backward.cu:2268-2272) */
  float* dL_dopacity;   /* [P] */
  float* dL_dscales;    /* [P,2] */
  float* dL_drots;      /* [P,4] */
  float* dL_dtable;     /* [table_rows, level_dim] fp32, for an fp16 or fp32 table */
  int64_t table_rows;   /* rows of dL_dtable (offsets[levels]) */
  float* dL_gradsum;    /* [P] sum over samples of alpha*T*|dL/dcolor|_1 (the
                           reference's dL_gradsum, returned in ap_level's slot) */
  float* dL_dshapes;    /* [P] or NULL: gradient of the splat kernel's shape
                           (kernel_type 1-3, backward.cu:1864-1909) */
  float* dL_dcolors_precomp; /* render modes other than 0, and level 0: gradient of
                           the per-surfel rows (ns_surfels.colors_precomp layout,
                           blend weight included; backward.cu:987-1033,
                           1108-1606; modes 8-10 with alpha T applied twice as the
                           reference's cases 8-10 compute it; zero in mode 11,
                           whose SH colour has no gradient), else NULL */
  float* dL_dshs;       /* [P, sh_coeffs, 3] with the SH colours (written, zero
                           where radii <= 0; backward.cu:21-140), else NULL */
  float* dL_dtransmat_precomp; /* [P, 9] with ns_surfels.transmat_precomp (written;
                           the render pass's dL/dT plus the centre's term,
                           backward.cu:2128-2158), else NULL */
} ns_raster_grads_out;

/* Scratch of the backward pass: per-surfel gradient accumulators. */
size_t ns_backward_scratch_bytes(int32_t P);
/* Scratch of the backward pass with settings->deterministic = 1: the per-surfel
 * accumulators, the fixed-point table gradient and its scale. */
size_t ns_backward_scratch_bytes_deterministic(int32_t P, int64_t table_rows, int32_t level_dim);

/* Backward rasterization (every built render_mode but 13 and the inference
 * flag; kernel_type 0-3). settings,
 * surfels, geom, binning and image must be those of the forward call whose outputs the gradients refer to
 * (the scratch buffers unchanged since). homotrans, when given to the forward,
 * is treated as build_H(rotations, scales, means3D): its gradient is folded into
 * the mean, scale and rotation gradients, as the reference does. The transform
 * is rebuilt with scale_modifier 1 and rotations are differentiated as given
 * (no normalisation), also as in the reference. */
int ns_rasterize_backward(const ns_raster_settings* settings, const ns_surfels* surfels,
                          const ns_raster_grads_in* grads_in, const ns_raster_grads_out* grads_out,
                          const void* geom, size_t geom_bytes, const void* binning,
                          size_t binning_bytes, const void* image, size_t image_bytes,
                          int64_t num_rendered, void* scratch, size_t scratch_bytes, void* stream);

/* Copies what a forward call left in its scratch buffers into caller buffers
 * (device; any output may be NULL), for inspection and tests. The reference
 * keeps the same state in its binningBuffer / geomBuffer / imgBuffer
 * (rasterizer_impl.cu:212-251, BinningState::point_list, ImageState::ranges):
 *   point_list [num_rendered] u32  surfel ids, per tile in (tile, depth) order
 *   ranges     [tiles, 2] u32      [start, end) of each tile in point_list
 *   tile_rects [P, 4] i16          x0, y0, x1, y1: the tiles that received the
 *                                  surfel (the reference's getRect rectangle cut
 *                                  to the surfel's alpha >= 1/255 box)
 *   depths     [P] f32             view-space depth of the sort key
 *   pixel_boxes [P, 4] f32         x0, x1, y0, y1 pixel box outside which the
 *                                  surfel's alpha < 1/255 (valid where the tile
 *                                  rectangle is non-empty)
 *   means2D    [P, 2] f32          the screen centre of the tile rectangle
 *                                  (compute_aabb's point_image; same validity)
 * num_rendered is the forward's instance count. Asynchronous on `stream`. */
int ns_read_binning(const void* geom, size_t geom_bytes, int32_t P, const void* binning,
                    size_t binning_bytes, const void* image, size_t image_bytes, int32_t width,
                    int32_t height, int64_t num_rendered, uint32_t* point_list, uint32_t* ranges,
                    int16_t* tile_rects, float* depths, float* pixel_boxes, float* means2D,
                    void* stream);

/* Poll bound of every bounded device wait in this library's kernels (the
 * radix sort's look-back on earlier tiles, the blend's record ring): a wait
 * that polls `spins` times without success records an error bit (reported by
 * ns_read_device_status, or lost where no status word is read) and the kernel
 * finishes. 0 restores the default 2^22. Applies to launches made after the
 * call, in the whole process; returns the previous bound. */
uint32_t ns_set_wait_limit(uint32_t spins);

/* Self-test of that wait path (no reference counterpart): one thread waits,
 * with the current bound and the sort's wait code, for the device word *flag
 * to become non-zero; if the bound runs out it records the timeout in the
 * error word of the geometry scratch `geom` (sized for P surfels), which
 * ns_read_device_status then reports as NS_ERR_DEVICE. Nothing traps. */
int ns_wait_selftest(const uint32_t* flag, void* geom, int32_t P, void* stream);

/* Reads (and clears) the device error word of a geometry scratch buffer; syncs. */
int ns_read_device_status(void* geom, int32_t P, void* stream);

/* Frustum visibility (view-space z > 0.2) per point: present[P] (bytes, 0/1). */
int ns_mark_visible(int32_t P, const float* means3D, const float* viewmatrix,
                    const float* projmatrix, uint8_t* present, void* stream);

/* ------------------------------------------------------------------ MLP */

/* Bias-free MLP in fp16 with fp32 accumulation: feat [in_dims, npix] (channel-major,
 * fp32) -> rgb [3, npix] = sigmoid(W3 relu(W2 relu(W1 x))) [:3]. weights: fp16
 * row-major [out,in] matrices packed back to back (W1 [hidden,in], W2 [hidden,hidden],
 * W3 [out_dims,hidden]). alpha (optional, [npix]): rgb is zeroed where alpha <= 0;
 * bg (optional, host [3]): rgb += (1-alpha) bg when bg sums > 0.
 * Supported: in_dims 32, hidden 64, two hidden layers, out_dims 3. */
int ns_mlp_forward(const float* feat, int32_t in_dims, int64_t npix, const uint16_t* weights,
                   int32_t hidden, int32_t out_dims, const float* alpha, const float* bg_host,
                   float* rgb, void* stream);

/* Backward of ns_mlp_forward (without the background term) given dL_drgb
 * [3, npix] fp32: dL_dfeat [in_dims, npix] fp32 and dL_dweights fp32 in the
 * packed-weight layout (W1 [hidden, in_dims], W2 [hidden, hidden], W3 [3,
 * hidden]; overwritten). The forward is recomputed exactly as ns_mlp_forward
 * computes it; the backward runs on TF32 tensor cores with fp32 accumulation,
 * treating the fp16 roundings as identity. alpha may be NULL (no mask). */
int ns_mlp_backward(const float* feat, int32_t in_dims, int64_t npix, const uint16_t* weights,
                    int32_t hidden, int32_t out_dims, const float* alpha, const float* dL_drgb,
                    float* dL_dfeat, float* dL_dweights, void* stream);

/* ------------------------------------------------------------------ RVQ */

/* out[n, d] = sum_{k=0..stages-1} codebooks[k, idx[n,k], d], fp32, stage order.
 * idx u8 [n, stages]; codebooks fp32 [stages, entries, dims]; out fp32 [n, dims].
 * Supported: entries <= 256, dims <= 64, stages <= 8. Bit-exact. */
int ns_rvq_decode(const uint8_t* idx, const float* codebooks, float* out, int64_t n,
                  int32_t stages, int32_t entries, int32_t dims, void* stream);

/* ------------------------------------------------------------------ sort */

/* Stable LSD radix sort of (key u64, value u32) pairs on bits [0, end_bit).
 * keys_alt / vals_alt are ping-pong buffers of n elements; the sorted result is
 * written to keys_out / vals_out. temp: ns_radix_sort_temp_bytes(n) bytes. */
size_t ns_radix_sort_temp_bytes(int64_t n);
int ns_radix_sort_pairs(const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                        uint32_t* vals_out, uint64_t* keys_alt, uint32_t* vals_alt, int64_t n,
                        int32_t end_bit, void* temp, size_t temp_bytes, void* stream);

/* Allocation-free variant of ns_radix_sort_pairs, for callers that cannot
 * allocate device memory (a plugin inside a host renderer with a fixed memory
 * budget, a runtime that hands out slices of its own arena, a language binding
 * without a CUDA allocator). It has no counterpart in the reference. The
 * ping-pong buffers and look-back state live in a file-scope device array sized
 * for at most 1,048,576 pairs (about 14 MB, held on every GPU that loads the
 * library until process exit); larger n returns NS_ERR_CAPACITY. All calls share
 * that array: calls whose kernels overlap on the GPU (other streams or host
 * threads) race, so serialise them. The first call on a device looks up the
 * array's address for that device (cudaGetSymbolAddress); make it before any
 * stream capture. The address is cached per device and CUDA context, so the
 * first call after a context reset (cudaDeviceReset) looks it up again. Same
 * result and argument checks as ns_radix_sort_pairs, except that device-side
 * errors (a look-back wait that ran out of its bound, which only a GPU that has
 * stopped making progress produces) are not reported: the call returns
 * argument and launch errors only, and the output is then undefined. */
int ns_radix_sort_pairs_noalloc(const uint64_t* keys_in, const uint32_t* vals_in,
                                uint64_t* keys_out, uint32_t* vals_out, int64_t n,
                                int32_t end_bit, void* stream);

/* ------------------------------------------------------------ fused frame */

/* One frame of the RVQ-driven render: decode -> attribute mix + activation ->
 * preprocess -> bin/sort -> blend + hash -> MLP (fused) -> mask/background.
 * Attributes: raw[n] = base[n, 0:10] + mix * decoded[n, 0:10] with the decoded
 * row layout mean(3) log-scale(2) quaternion(4) opacity-logit(1) SH(48) tex(1);
 * scale = exp(raw), rotation = normalize(raw), opacity = sigmoid(raw). */
#define NS_FLAG_SKIP_DECODE 2  /* ns_render_frame: `decoded` already holds the decoded
                                  attributes (e.g. all-gathered from other ranks) */
#define NS_FRAME_STAGES 5      /* decode, preprocess, binning, blend, mlp */

typedef struct ns_frame_inputs {
  int32_t P;
  const uint8_t* rvq_idx;     /* [P, stages] */
  const float* codebooks;     /* [stages, entries, dims] */
  int32_t stages, entries, dims;
  const float* base;          /* [P, 10] raw base attributes */
  float mix;                  /* weight of the decoded attributes */
  float* decoded;             /* [P, dims] output of the decode stage (caller-owned) */
  const float* ap_level;      /* [P] or NULL */
  const void* features;       /* hash table */
  const int32_t* offsets;
  const float* gridrange;
  const uint16_t* mlp_weights;/* fp16, as ns_mlp_forward */
  int32_t mlp_hidden;
  const float* bg_host;       /* host [3] */
  void* const* stage_events;  /* NULL, or 2*NS_FRAME_STAGES cudaEvent_t recorded on the
                                 stream before/after each stage (for stage timing) */
} ns_frame_inputs;

typedef struct ns_frame_outputs {
  float* rgb;        /* [3,H,W] */
  float* out_color;  /* [C,H,W] features */
  float* out_others; /* [14,H,W] */
  int32_t* radii;    /* [P] */
} ns_frame_outputs;

int ns_render_frame(const ns_raster_settings* settings, const ns_frame_inputs* inputs,
                    const ns_frame_outputs* outputs, void* geom, size_t geom_bytes,
                    void* binning, size_t binning_bytes, void* image, size_t image_bytes,
                    int64_t* num_rendered, int flags, void* stream);

/* --------------------------------------------------------- allmap decode */

/* The per-frame maps the reference's render() derives from the allmap
 * (allmap = out_others: 0 depth*w, 1 alpha, 2-4 view-space normal, 5 median
 * depth), in one pass. maps fp32 [9, H, W]: 0-2 rend_normal (R^T n_view),
 * 3 depth_expected (nan_to_num(D / alpha)), 4 depth_median (nan_to_num),
 * 5 surf_depth = expected * (1 - depth_ratio) + depth_ratio * median,
 * 6-8 surf_normal = normalize(cross(P(x, y+1) - P(x, y-1), P(x+1, y) - P(x-1, y)))
 * * alpha with P = surf_depth * rays_d + ray_o (zero on the border). Inputs as
 * ns_normal_error. rend_alpha, rend_dist and gaussian_num are allmap channels
 * 1, 6 and 7 as they are. */
int ns_allmap_decode(const float* allmap, const float* viewmatrix, const float* rays_d,
                     const float* ray_o, int32_t width, int32_t height, float depth_ratio,
                     float* maps, void* stream);

/* --------------------------------------------------------- normal error */

/* Per-pixel depth-normal consistency error of the training loss, with the
 * allmap decode fused in (allmap = out_others of the rasterizer, channels
 * 0 = accumulated depth D, 1 = alpha, 2-4 = view-space normal):
 *   depth(q)  = D(q) / alpha(q), non-finite -> 0 (+inf, NaN) or -FLT_MAX (-inf)
 *   P(q)      = depth(q) * rays_d[q] + ray_o                        (world point)
 *   surf(p)   = normalize(cross(P(x, y+1) - P(x, y-1), P(x+1, y) - P(x-1, y))) * alpha(p)
 *               (eps 1e-12; zero on the one-pixel image border)
 *   rend(p)   = R^T n_view(p), R = viewmatrix[:3,:3] (world-to-view rotation)
 *   err[p]    = 1 - <rend(p), surf(p)>
 * allmap fp32 [>=5, H, W]; viewmatrix fp32 [16] (device, the rasterizer's
 * layout); rays_d fp32 [H*W, 3] (device: per-pixel ray direction, pixel y*W + x,
 * as utils/point_utils.py:10-30 builds it); ray_o fp32 [3] (device); err fp32
 * [H, W]. */
int ns_normal_error(const float* allmap, const float* viewmatrix, const float* rays_d,
                    const float* ray_o, int32_t width, int32_t height, float* err, void* stream);

/* Scratch of ns_normal_error_backward: 6 floats per pixel. */
size_t ns_normal_error_scratch_bytes(int32_t width, int32_t height);

/* dL_dallmap[0:5] = d L / d allmap[0:5] given dL_derr (fp32, pixel p at
 * dL_derr[p * derr_stride]; stride 0 broadcasts one value, e.g. the gradient
 * of a mean). Channels 5 and up of dL_dallmap are not written. alpha enters
 * through the depth only (surf uses alpha detached, as the reference does);
 * pixels whose depth is not finite pass no gradient to D or alpha. */
int ns_normal_error_backward(const float* allmap, const float* viewmatrix, const float* rays_d,
                             const float* ray_o, int32_t width, int32_t height,
                             const float* dL_derr, int64_t derr_stride, float* dL_dallmap,
                             void* scratch, size_t scratch_bytes, void* stream);

/* ------------------------------------------------------ hash-grid encoding */

/* The multiresolution hash-grid encoding as a standalone op, with the
 * reference gridencoder's arguments (gridencoder.h:9-10; B points, D = 3
 * dims, C = 2 features per level, L levels, S = log2(per-level scale), H base
 * resolution, gridtype 0 = hash; interp 0 linear / 1 smoothstep). The lookup is
 * the blend kernel's (the rasterizer's per-level query_feature arithmetic).
 *   inputs     fp32 [B, 3] in [0, 1]; points outside give zeros / no gradient
 *   embeddings [offsets[L], 2], fp16 (embeddings_fp16 = 1) or fp32
 *   offsets    int32 [L + 1] level row offsets
 *   outputs    fp32 [L, B, 2] (also for an fp16 table: computed in fp32, where
 *              the reference's fp16 path accumulates in half precision)
 *   dy_dx      fp32 [B, L * 3 * 2] or NULL: d output / d input
 * Supported: D 3, C 2, gridtype 0 (others NS_ERR_UNSUPPORTED). */
int ns_grid_encode_forward(const float* inputs, const void* embeddings, int32_t embeddings_fp16,
                           const int32_t* offsets, float* outputs, uint32_t B, uint32_t D, uint32_t C,
                           uint32_t L, float S, uint32_t H, float* dy_dx, uint32_t gridtype,
                           int32_t align_corners, uint32_t interp, void* stream);

/* Backward of ns_grid_encode_forward for grad fp32 [L, B, 2]: grad_embeddings
 * fp32 [offsets[L], 2] is accumulated into (zero it first, as the reference's
 * caller does) with float atomics; grad_inputs fp32 [B, 3] (or NULL) is
 * formed from dy_dx, which must then be the forward's dy_dx. */
int ns_grid_encode_backward(const float* grad, const float* inputs, const void* embeddings,
                            int32_t embeddings_fp16, const int32_t* offsets, float* grad_embeddings,
                            uint32_t B, uint32_t D, uint32_t C, uint32_t L, float S, uint32_t H,
                            const float* dy_dx, float* grad_inputs, uint32_t gridtype,
                            int32_t align_corners, uint32_t interp, void* stream);

/* ------------------------------------------------------------ measurement */

/* Gather roofline probe (no reference counterpart; a measurement tool, not
 * part of the render path): blocks x 256 threads each perform
 * lookups_per_thread (a multiple of 4) hash-grid lookups at pseudo-random
 * points of levels [level0, level0 + levels) of `table`, with the blend
 * kernel's lookup code, and write one float per thread to sink (blocks * 256
 * floats). spacing = 0: independent points and levels per lane; spacing > 0:
 * the blend's pattern (a warp's 32 lanes as a 16 x 2 pixel strip of that
 * spacing in grid units on 8 stacked surfels, levels in an outer loop;
 * lookups_per_thread a multiple of 8 * levels). Corner bytes read = blocks *
 * 256 * lookups_per_thread * 8 * row bytes (4 for an fp16 pair table). */
int ns_gather_probe(const void* table, int32_t table_fp16, const int32_t* offsets, uint32_t level0,
                    uint32_t levels, float S, uint32_t H, uint32_t lookups_per_thread, float spacing,
                    int32_t blocks, float* sink, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NEST_B200_H_ */
