// capi.cu -- the extern "C" entry points of libnest_b200.so (declared in
// include/nest_b200.h), scratch-buffer carving and the frame pipeline.
//
// The pipeline mirrors CudaRasterizer::Rasterizer::forward
// (rasterizer_impl.cu:255-440): preprocess -> prefix sum -> instance count ->
// duplicate keys -> radix sort -> tile ranges -> blend. Differences by design:
// buffers are caller-owned (no resize functors), the prefix sum reuses the
// per-CTA totals computed by preprocess, the sort is the in-house onesweep sort
// and, in NS_FLAG_DEVICE_COUNT mode, the instance count never returns to the host.
#include <atomic>
#include <cstdio>
#include <cstring>

#include "kernels.cuh"


namespace ns_host {
static thread_local int g_last_cuda_error = 0;
static std::atomic<uint64_t> g_launches{0};
static std::atomic<uint32_t> g_wait_limit{ns::kSpinLimit};
uint32_t wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }
int record_cuda(cudaError_t e) {
  g_last_cuda_error = (int)e;
  return NS_ERR_CUDA;
}
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace ns_host

namespace {

using namespace ns;

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

// Bump allocator over a caller buffer (a null base only measures).
struct Carver {
  char* base;
  size_t off = 0;
  template <typename T>
  T* take(size_t count) {
    off = align_up(off);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += sizeof(T) * count;
    return p;
  }
};

struct GeomState {
  SurfelRecord* records;
  BinInfo* bin;
  uint32_t* tiles;
  uint32_t* block_sums;    // per preprocess CTA: tile-count totals
  uint32_t* block_prefix;
  int64_t* count;          // instance total
  uint32_t* err;
  // Depth sort of the surfels (binning step 1) and the per-CTA totals of the
  // tile counts in depth order.
  uint32_t* depth_keys;
  uint32_t* depth_keys_alt;
  uint32_t* depth_keys_sorted;
  uint32_t* depth_vals;
  uint32_t* depth_vals_alt;
  uint32_t* depth_vals_sorted;  // surfel indices in depth order
  uint32_t* sorted_sums;
  uint32_t* sorted_prefix;
  float* rgb;  // [P, 3] SH colours of the level-0 SH path
  void* depth_sort_temp;
  size_t depth_sort_temp_bytes;
};

GeomState carve_geom(void* base, int P, size_t* used) {
  Carver c{reinterpret_cast<char*>(base)};
  GeomState g;
  const int nb = preprocess_blocks(P);
  g.records = c.take<SurfelRecord>((size_t)max(P, 1));
  g.bin = c.take<BinInfo>((size_t)max(P, 1));
  g.tiles = c.take<uint32_t>((size_t)max(P, 1));
  g.block_sums = c.take<uint32_t>((size_t)nb);
  g.block_prefix = c.take<uint32_t>((size_t)nb);
  g.count = c.take<int64_t>(1);
  g.err = c.take<uint32_t>(4);
  const size_t np = (size_t)max(P, 1);
  g.depth_keys = c.take<uint32_t>(np);
  g.depth_keys_alt = c.take<uint32_t>(np);
  g.depth_keys_sorted = c.take<uint32_t>(np);
  g.depth_vals = c.take<uint32_t>(np);
  g.depth_vals_alt = c.take<uint32_t>(np);
  g.depth_vals_sorted = c.take<uint32_t>(np);
  g.sorted_sums = c.take<uint32_t>((size_t)nb);
  g.sorted_prefix = c.take<uint32_t>((size_t)nb);
  g.rgb = c.take<float>(3 * np);
  g.depth_sort_temp_bytes = radix_sort_temp_bytes(P);
  g.depth_sort_temp = c.take<char>(g.depth_sort_temp_bytes);
  if (used) *used = align_up(c.off);
  return g;
}

struct ImageState {
  uint2* ranges;
  uint32_t* order;  // tiles, heaviest first (launch order of the per-tile kernels)
  float* final_T;
  uint32_t* n_contrib;
};

ImageState carve_image(void* base, int W, int H, size_t* used) {
  Carver c{reinterpret_cast<char*>(base)};
  ImageState s;
  const size_t tiles = (size_t)div_up(W, kTile) * div_up(H, kTile);
  const size_t HW = (size_t)W * H;
  s.ranges = c.take<uint2>((size_t)max64(tiles, 1));
  s.order = c.take<uint32_t>((size_t)max64(tiles, 1));
  s.final_T = c.take<float>((size_t)max64(3 * HW, 1));
  s.n_contrib = c.take<uint32_t>((size_t)max64(2 * HW, 1));
  if (used) *used = align_up(c.off);
  return s;
}

struct BinState {
  uint32_t* keys_unsorted;  // tile ids
  uint32_t* keys_alt;
  uint32_t* keys_sorted;
  uint32_t* vals_unsorted;
  uint32_t* vals_alt;
  uint32_t* vals_sorted;
  void* sort_temp;
  size_t sort_temp_bytes;
};

BinState carve_bin(void* base, int64_t cap, size_t* used) {
  Carver c{reinterpret_cast<char*>(base)};
  BinState b;
  const size_t n = (size_t)max64(cap, 1);
  b.keys_unsorted = c.take<uint32_t>(n);
  b.keys_alt = c.take<uint32_t>(n);
  b.keys_sorted = c.take<uint32_t>(n);
  b.vals_unsorted = c.take<uint32_t>(n);
  b.vals_alt = c.take<uint32_t>(n);
  b.vals_sorted = c.take<uint32_t>(n);
  b.sort_temp_bytes = radix_sort_temp_bytes(cap);
  b.sort_temp = c.take<char>(b.sort_temp_bytes);
  if (used) *used = align_up(c.off);
  return b;
}

size_t bin_bytes(int64_t cap) {
  size_t u = 0;
  carve_bin(nullptr, cap, &u);
  return u;
}

// Largest instance capacity whose binning layout fits in `bytes`.
int64_t bin_capacity(size_t bytes) {
  if (bytes < bin_bytes(0)) return -1;
  int64_t lo = 0, hi = 1;
  while (bin_bytes(hi) <= bytes && hi < ((int64_t)1 << 40)) hi <<= 1;
  while (hi - lo > 1) {
    const int64_t mid = lo + (hi - lo) / 2;
    if (bin_bytes(mid) <= bytes) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Next-highest bit of the MSB (rasterizer_impl.cu:35-50).
uint32_t higher_msb(uint32_t n) {
  uint32_t msb = sizeof(n) * 4;
  uint32_t step = msb;
  while (step > 1) {
    step /= 2;
    if (n >> msb) msb += step;
    else msb -= step;
  }
  if (n >> msb) msb++;
  return msb;
}

int num_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return sms;
}

int validate_settings(const ns_raster_settings* s) {
  if (!s) return NS_ERR_INVALID;
  if (s->image_width <= 0 || s->image_height <= 0) return NS_ERR_INVALID;
  if (!s->viewmatrix || !s->projmatrix) return NS_ERR_INVALID;
  // levels == 0 in mode 0: per-surfel colours (colors_precomp, C channels)
  if (s->level_dim == 0 || s->channels == 0) return NS_ERR_INVALID;
  if (s->levels * s->level_dim > s->channels) return NS_ERR_INVALID;
  if (s->kernel_type < 0 || s->kernel_type > 3) return NS_ERR_UNSUPPORTED;
  const int base = s->render_mode & 0xFF, flag = s->render_mode >> 8;
  if (base == 1 || base == 2 || base == 3 || base == 5 || base > 14) return NS_ERR_UNSUPPORTED;
  if (flag > 1 || (flag && base != 12 && base != 13 && base != 14)) return NS_ERR_UNSUPPORTED;
  if (base >= 8 && base <= 10) {
    // one 3-wide hash level; hybrid_levels carries the decompose flag
    if (s->level_dim != 3 || s->levels > 1 || s->hybrid_levels > 2) return NS_ERR_INVALID;
    if (s->channels != (base == 9 ? 48u : 3u)) return NS_ERR_INVALID;
  } else if (base == 11) {
    // hash levels from channel 0; three more accumulators hold the SH colour
    if (s->channels + 3 > 32) return NS_ERR_INVALID;
  } else if (base != 0) {
    if (s->hybrid_levels > 16 || s->total_levels > 16) return NS_ERR_INVALID;
    // modes 6 and 7 have no per-surfel levels before the hash levels
    if ((base == 6 || base == 7) && s->hybrid_levels != 0) return NS_ERR_INVALID;
    if ((s->hybrid_levels + s->levels) * s->level_dim > s->channels) return NS_ERR_INVALID;
    if ((base == 7 || base == 12 || base == 13) && s->total_levels * s->level_dim > s->channels)
      return NS_ERR_INVALID;
    if (base == 7 && s->levels > s->total_levels) return NS_ERR_INVALID;
  }
  return NS_OK;
}

// The level-0 SH path (forward.cu:414-423): mode 0 without hash levels, no
// precomputed colours, SH coefficients given.
bool sh_colours(const ns_raster_settings* s, const ns_surfels* f) {
  return s->render_mode == 0 && s->levels == 0 && !f->colors_precomp && f->shs;
}
int validate_sh(const ns_raster_settings* s, const ns_surfels* f) {
  if (s->channels != 3 || s->sh_degree < 0 || s->sh_degree > 3 || !s->campos) return NS_ERR_INVALID;
  if (f->sh_coeffs < (s->sh_degree + 1) * (s->sh_degree + 1)) return NS_ERR_INVALID;
  return NS_OK;
}

// Binning + blend shared by the API forward and the fused frame.
int bin_and_render(const ns_raster_settings* st, int P, const GeomState& g, const ImageState& im,
                   void* binning, size_t binning_bytes, const void* features,
                   const int32_t* offsets, const float* gridrange, float* out_color,
                   float* out_others, float* cover_pixels, float* trans_avg, const float* gauss,
                   int64_t* num_rendered, int flags, cudaStream_t stream,
                   void* const* ev = nullptr) {
  const int W = st->image_width, H = st->image_height;
  const int gx = div_up(W, kTile), gy = div_up(H, kTile);
  const int tiles = gx * gy;
  const int nb = preprocess_blocks(P);
  int rc = scan_block_sums_launch(g.block_sums, g.block_prefix, nb, g.count, stream);
  if (rc) return rc;
  const int64_t cap = bin_capacity(binning_bytes);
  if (cap < 0) return NS_ERR_SCRATCH;
  const bool device_count = (flags & NS_FLAG_DEVICE_COUNT) != 0;
  // Binning step 1, the depth sort of the surfels, runs while the host waits
  // for the instance count.
  rc = radix_sort32_launch(g.depth_keys, g.depth_vals, g.depth_keys_sorted, g.depth_vals_sorted,
                         g.depth_keys_alt, g.depth_vals_alt, P, 32, g.depth_sort_temp,
                         g.depth_sort_temp_bytes, stream);
  if (rc) return rc;
  int64_t count = cap;  // device-count mode: the tile sort and ranges are sized by the capacity
  if (!device_count) {
    NS_CUDA_TRY(cudaMemcpyAsync(&count, g.count, sizeof(int64_t), cudaMemcpyDeviceToHost, stream));
    NS_CUDA_TRY(cudaStreamSynchronize(stream));
    if (num_rendered) *num_rendered = count;
    if (count > cap) return NS_ERR_CAPACITY;
  } else if (num_rendered) {
    *num_rendered = -1;  // on the device only (g.count); overflow sets the device error word
  }
  BinState b = carve_bin(binning, cap, nullptr);
  rc = duplicate_keys_launch(P, g.depth_vals_sorted, g.bin, g.tiles, g.sorted_sums,
                             g.sorted_prefix, g.count, gx, b.keys_unsorted, b.vals_unsorted, cap,
                             g.err, stream);
  if (rc) return rc;
  const int end_bit = (int)higher_msb((uint32_t)tiles);
  rc = radix_sort32_launch(b.keys_unsorted, b.vals_unsorted, b.keys_sorted, b.vals_sorted, b.keys_alt,
                         b.vals_alt, count, end_bit, b.sort_temp, b.sort_temp_bytes, stream,
                         device_count ? g.count : nullptr);
  if (rc) return rc;
  rc = identify_ranges_launch(b.keys_sorted, device_count ? g.count : nullptr, count, cap, im.ranges,
                              tiles, num_sms(), stream);
  if (rc) return rc;
  rc = tile_order_launch(im.ranges, tiles, im.order, stream);
  if (rc) return rc;
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[5], stream));
  RenderParams rp;
  rp.W = W;
  rp.H = H;
  rp.C = (int)st->channels;
  rp.LD = (int)st->level_dim;
  rp.L = st->levels;
  rp.S = st->level_scale_log2;
  rp.Hres = st->base_resolution;
  rp.align_corners = st->align_corners;
  rp.interp = st->interpolation;
  rp.contract = st->if_contract;
  rp.beta = st->beta;
  rp.kernel_type = st->kernel_type;
  rp.render_mode = st->render_mode;
  rp.hybrid_levels = (int)st->hybrid_levels;
  rp.total_levels = (int)st->total_levels;
  rp.gauss = gauss;
  rp.max_intersections = st->max_intersections;
  rp.record_transmittance = st->record_transmittance;
  rp.ranges = im.ranges;
  rp.tile_order = im.order;
  rp.point_list = b.vals_sorted;
  rp.records = g.records;
  rp.table = features;
  rp.offsets = offsets;
  rp.gridrange = gridrange;
  rp.out_color = out_color;
  rp.out_others = out_others;
  rp.final_T = im.final_T;
  rp.n_contrib = im.n_contrib;
  rp.cover_pixels = cover_pixels;
  rp.trans_avg = trans_avg;
  rp.err = g.err;
  rp.spin_limit = ns_host::wait_limit();
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[6], stream));
  rc = render_launch(rp, st->table_fp16, stream);
  if (rc) return rc;
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[7], stream));
  return NS_OK;
}

}  // namespace

extern "C" {

const char* ns_status_string(int status) {
  switch (status) {
    case NS_OK: return "ok";
    case NS_ERR_INVALID: return "invalid argument";
    case NS_ERR_UNSUPPORTED: return "unsupported shape or mode";
    case NS_ERR_CAPACITY: return "binning scratch too small for the instance count";
    case NS_ERR_CUDA: return "CUDA runtime error";
    case NS_ERR_SCRATCH: return "scratch buffer too small";
    case NS_ERR_DEVICE: return "a kernel recorded an error";
    default: return "unknown status";
  }
}

int ns_last_cuda_error(void) { return ns_host::g_last_cuda_error; }

uint32_t ns_set_wait_limit(uint32_t spins) {
  return ns_host::g_wait_limit.exchange(spins ? spins : ns::kSpinLimit);
}
uint64_t ns_kernel_launches(void) { return ns_host::g_launches.load(); }
int ns_version(void) { return 1; }

size_t ns_geometry_scratch_bytes(int32_t P) {
  size_t u = 0;
  carve_geom(nullptr, P, &u);
  return u;
}
size_t ns_image_scratch_bytes(int32_t width, int32_t height) {
  size_t u = 0;
  carve_image(nullptr, width, height, &u);
  return u;
}
size_t ns_binning_scratch_bytes(int64_t max_instances) { return bin_bytes(max_instances); }

int ns_rasterize_forward(const ns_raster_settings* settings, const ns_surfels* surfels,
                         const ns_raster_outputs* outputs, void* geom, size_t geom_bytes,
                         void* binning, size_t binning_bytes, void* image, size_t image_bytes,
                         int64_t* num_rendered, int flags, void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  int rc = validate_settings(settings);
  if (rc) return rc;
  if (!surfels || !outputs) return NS_ERR_INVALID;
  const int P = surfels->P;
  if (P < 0) return NS_ERR_INVALID;
  if (num_rendered) *num_rendered = 0;
  if (P == 0) return NS_OK;
  // precomputed transforms replace scales and rotations, and need the homotrans
  // that places the hit point (transMat_precomp, forward.cu:366-380)
  const bool given_T = surfels->transmat_precomp != nullptr;
  if (!surfels->means3D || (!given_T && (!surfels->scales || !surfels->rotations)) ||
      (given_T && !surfels->homotrans) || !surfels->opacities || !surfels->features || !surfels->offsets ||
      !surfels->gridrange)
    return NS_ERR_INVALID;
  if (!outputs->out_color || !outputs->out_others || !outputs->radii) return NS_ERR_INVALID;
  if (settings->kernel_type != 0 && P > 0 && !surfels->shapes) return NS_ERR_INVALID;
  const bool shc = sh_colours(settings, surfels);
  if (shc && (rc = validate_sh(settings, surfels))) return rc;
  if (uses_surfel_rows(settings->render_mode, settings->levels) && P > 0 && !surfels->colors_precomp && !shc)
    return NS_ERR_INVALID;
  if (settings->record_transmittance && (!outputs->cover_pixels || !outputs->trans_avg))
    return NS_ERR_INVALID;
  const int fbase = settings->render_mode & 0xFF;
  if (settings->level_dim != ((fbase >= 8 && fbase <= 10) ? 3u : 2u)) return NS_ERR_UNSUPPORTED;
  if (geom_bytes < ns_geometry_scratch_bytes(P)) return NS_ERR_SCRATCH;
  if (image_bytes < ns_image_scratch_bytes(settings->image_width, settings->image_height))
    return NS_ERR_SCRATCH;
  GeomState g = carve_geom(geom, P, nullptr);
  ImageState im = carve_image(image, settings->image_width, settings->image_height, nullptr);
  NS_CUDA_TRY(cudaMemsetAsync(g.err, 0, sizeof(uint32_t), stream));
  rc = preprocess_api_launch(P, *surfels, settings->scale_modifier, settings->beta,
                             settings->kernel_type, settings->viewmatrix,
                             settings->projmatrix, settings->image_width, settings->image_height,
                             g.records, g.bin, outputs->radii, g.tiles, g.depth_keys, g.depth_vals,
                             g.block_sums, stream);
  if (rc) return rc;
  if (shc) {
    rc = sh_color_launch(P, settings->sh_degree, surfels->sh_coeffs, surfels->means3D, settings->campos,
                         surfels->shs, g.rgb, stream);
    if (rc) return rc;
  }
  return bin_and_render(settings, P, g, im, binning, binning_bytes, surfels->features,
                        surfels->offsets, surfels->gridrange, outputs->out_color,
                        outputs->out_others, outputs->cover_pixels, outputs->trans_avg,
                        shc ? g.rgb : surfels->colors_precomp, num_rendered, flags, stream);
}

int ns_read_binning(const void* geom, size_t geom_bytes, int32_t P, const void* binning,
                    size_t binning_bytes, const void* image, size_t image_bytes, int32_t width,
                    int32_t height, int64_t num_rendered, uint32_t* point_list, uint32_t* ranges,
                    int16_t* tile_rects, float* depths, float* pixel_boxes, float* means2D,
                    void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (P < 0 || width <= 0 || height <= 0 || num_rendered < 0) return NS_ERR_INVALID;
  if (!geom || !image || (num_rendered > 0 && point_list && !binning)) return NS_ERR_INVALID;
  if (geom_bytes < ns_geometry_scratch_bytes(P) || image_bytes < ns_image_scratch_bytes(width, height))
    return NS_ERR_SCRATCH;
  GeomState g = carve_geom(const_cast<void*>(geom), P, nullptr);
  ImageState im = carve_image(const_cast<void*>(image), width, height, nullptr);
  if (point_list && num_rendered > 0) {
    const int64_t cap = bin_capacity(binning_bytes);
    if (cap < 0 || num_rendered > cap) return NS_ERR_SCRATCH;
    BinState b = carve_bin(const_cast<void*>(binning), cap, nullptr);
    NS_CUDA_TRY(cudaMemcpyAsync(point_list, b.vals_sorted, (size_t)num_rendered * sizeof(uint32_t),
                                cudaMemcpyDeviceToDevice, stream));
  }
  if (ranges) {
    const size_t tiles = (size_t)div_up(width, kTile) * div_up(height, kTile);
    NS_CUDA_TRY(cudaMemcpyAsync(ranges, im.ranges, tiles * sizeof(uint2), cudaMemcpyDeviceToDevice, stream));
  }
  if (P == 0) return NS_OK;
  // Strided copies out of the 16-byte BinInfo and 128-byte SurfelRecord arrays.
  if (tile_rects)
    NS_CUDA_TRY(cudaMemcpy2DAsync(tile_rects, 4 * sizeof(int16_t), g.bin, sizeof(BinInfo),
                                  4 * sizeof(int16_t), (size_t)P, cudaMemcpyDeviceToDevice, stream));
  if (depths)
    NS_CUDA_TRY(cudaMemcpy2DAsync(depths, sizeof(float), reinterpret_cast<const char*>(g.bin) + 8,
                                  sizeof(BinInfo), sizeof(float), (size_t)P, cudaMemcpyDeviceToDevice,
                                  stream));
  if (pixel_boxes)
    NS_CUDA_TRY(cudaMemcpy2DAsync(pixel_boxes, sizeof(float4), g.records, sizeof(SurfelRecord),
                                  sizeof(float4), (size_t)P, cudaMemcpyDeviceToDevice, stream));
  if (means2D)  // record words 13, 14 (q3.y, q3.z)
    NS_CUDA_TRY(cudaMemcpy2DAsync(means2D, 2 * sizeof(float), reinterpret_cast<const char*>(g.records) + 52,
                                  sizeof(SurfelRecord), 2 * sizeof(float), (size_t)P,
                                  cudaMemcpyDeviceToDevice, stream));
  return NS_OK;
}

size_t ns_backward_scratch_bytes(int32_t P) {
  // the per-surfel accumulators, then dL/drgb of the level-0 SH path
  return align_up(backward_accum_bytes(P)) + align_up((size_t)max64(P, 1) * 3 * sizeof(float));
}

size_t ns_backward_scratch_bytes_deterministic(int32_t P, int64_t table_rows, int32_t level_dim) {
  const int64_t entries = max64(table_rows, 0) * max64(level_dim, 0);
  return ns_backward_scratch_bytes(P) + align_up((size_t)entries * sizeof(unsigned long long)) +
         align_up(sizeof(uint32_t));
}

int ns_rasterize_backward(const ns_raster_settings* settings, const ns_surfels* surfels,
                          const ns_raster_grads_in* gi, const ns_raster_grads_out* go,
                          const void* geom, size_t geom_bytes, const void* binning,
                          size_t binning_bytes, const void* image, size_t image_bytes,
                          int64_t num_rendered, void* scratch, size_t scratch_bytes,
                          void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  int rc = validate_settings(settings);
  if (rc) return rc;
  // training rules only (the reference has no mode-13 backward)
  if ((settings->render_mode >> 8) != 0 || (settings->render_mode & 0xFF) == 13) return NS_ERR_UNSUPPORTED;
  if (!surfels || !gi || !go) return NS_ERR_INVALID;
  const int P = surfels->P;
  if (P < 0 || num_rendered < 0) return NS_ERR_INVALID;
  if (settings->kernel_type != 0 && P > 0 && (!surfels->shapes || !go->dL_dshapes))
    return NS_ERR_INVALID;
  const int base_mode = settings->render_mode & 0xFF;
  const bool rows = uses_surfel_rows(settings->render_mode, settings->levels);
  const bool shc = sh_colours(settings, surfels);
  if (shc && ((rc = validate_sh(settings, surfels)) || (P > 0 && !go->dL_dshs))) return rc ? rc : NS_ERR_INVALID;
  if (rows && !shc && P > 0 && (!surfels->colors_precomp || !go->dL_dcolors_precomp)) return NS_ERR_INVALID;
  // row length of colors_precomp: level 0 and mode 6 C, mode 4 hybrid LD,
  // modes 7 / 12 total LD + 1, mode 14 hybrid LD + 1, modes 8 / 10 3, modes 9 / 11 48
  const size_t mode_stride = !rows                              ? 0
                             : (base_mode == 0 || base_mode == 6) ? (size_t)settings->channels
                             : base_mode == 4 ? (size_t)settings->hybrid_levels * settings->level_dim
                             : (base_mode == 8 || base_mode == 10) ? 3
                             : (base_mode == 9 || base_mode == 11) ? 48
                             : (base_mode == 7 || base_mode == 12)
                                 ? (size_t)settings->total_levels * settings->level_dim + 1
                                 : (size_t)settings->hybrid_levels * settings->level_dim + 1;
  if (settings->level_dim != ((base_mode >= 8 && base_mode <= 10) ? 3u : 2u)) return NS_ERR_UNSUPPORTED;
  if (!go->dL_dmeans3D || !go->dL_dmean2D || !go->dL_dopacity || !go->dL_dscales ||
      !go->dL_drots || !go->dL_dtable || !go->dL_gradsum || go->table_rows < 0)
    return NS_ERR_INVALID;
  const bool det = settings->deterministic != 0;
  if (go->table_rows > 0)
    NS_CUDA_TRY(cudaMemsetAsync(go->dL_dtable, 0,
                                (size_t)go->table_rows * settings->level_dim * sizeof(float), stream));
  if (P == 0) return NS_OK;
  const bool given_T = surfels->transmat_precomp != nullptr;
  if (!surfels->means3D || (!given_T && (!surfels->scales || !surfels->rotations)) ||
      (given_T && (!surfels->homotrans || !go->dL_dtransmat_precomp)) || !surfels->features ||
      !surfels->offsets || !surfels->gridrange)
    return NS_ERR_INVALID;
  if (!gi->dL_dout_color || !gi->dL_dout_others || !gi->radii) return NS_ERR_INVALID;
  if (!geom || !binning || !image || !scratch) return NS_ERR_INVALID;
  if (geom_bytes < ns_geometry_scratch_bytes(P)) return NS_ERR_SCRATCH;
  if (image_bytes < ns_image_scratch_bytes(settings->image_width, settings->image_height))
    return NS_ERR_SCRATCH;
  if (scratch_bytes < (det ? ns_backward_scratch_bytes_deterministic(P, go->table_rows, settings->level_dim)
                           : ns_backward_scratch_bytes(P)))
    return NS_ERR_SCRATCH;
  const int64_t cap = bin_capacity(binning_bytes);
  if (cap < 0 || num_rendered > cap) return NS_ERR_SCRATCH;
  const int W = settings->image_width, H = settings->image_height;
  GeomState g = carve_geom(const_cast<void*>(geom), P, nullptr);
  ImageState im = carve_image(const_cast<void*>(image), W, H, nullptr);
  BinState b = carve_bin(const_cast<void*>(binning), cap, nullptr);
  float* accum = static_cast<float*>(scratch);
  NS_CUDA_TRY(cudaMemsetAsync(accum, 0, backward_accum_bytes(P), stream));
  const size_t table_entries = (size_t)go->table_rows * settings->level_dim;
  unsigned long long* table_fixed = nullptr;
  uint32_t* grad_max = nullptr;
  if (det) {
    unsigned char* base = static_cast<unsigned char*>(scratch) + ns_backward_scratch_bytes(P);
    table_fixed = reinterpret_cast<unsigned long long*>(base);
    grad_max = reinterpret_cast<uint32_t*>(base + align_up(table_entries * sizeof(unsigned long long)));
    NS_CUDA_TRY(cudaMemsetAsync(table_fixed, 0, table_entries * sizeof(unsigned long long), stream));
    rc = table_grad_max_launch(gi->dL_dout_color,
                               (size_t)settings->channels * (size_t)settings->image_width *
                                   (size_t)settings->image_height,
                               grad_max, stream);
    if (rc) return rc;
  }
  // W and H as preprocessCUDA's backward recomputes them from the focal length
  // (backward.cu:2247-2248, focal from rasterizer_impl.cu:508-509), in float.
  const float focal_x = (float)W / (2.0f * settings->tanfovx);
  const float focal_y = (float)H / (2.0f * settings->tanfovy);
  volatile float wx = focal_x * settings->tanfovx, wy = focal_y * settings->tanfovy;
  const int Wq = (int)(wx * 2.0f), Hq = (int)(wy * 2.0f);
  BackwardParams bp;
  bp.W = W;
  bp.H = H;
  bp.C = (int)settings->channels;
  bp.LD = (int)settings->level_dim;
  bp.L = settings->levels;
  bp.S = settings->level_scale_log2;
  bp.Hres = settings->base_resolution;
  bp.align_corners = settings->align_corners;
  bp.interp = settings->interpolation;
  bp.contract = settings->if_contract;
  bp.beta = settings->beta;
  bp.kernel_type = settings->kernel_type;
  bp.render_mode = settings->render_mode;
  bp.hybrid_levels = (int)settings->hybrid_levels;
  bp.total_levels = (int)settings->total_levels;
  // SH path: the colours' gradient goes to scratch, then through the SH backward
  float* drgb = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) +
                                         align_up(backward_accum_bytes(P)));
  bp.gauss = shc ? g.rgb : surfels->colors_precomp;
  bp.dL_dcolors = shc ? drgb : go->dL_dcolors_precomp;
  if (rows)
    NS_CUDA_TRY(cudaMemsetAsync(bp.dL_dcolors, 0, (size_t)P * mode_stride * sizeof(float), stream));
  bp.Wq = Wq;
  bp.Hq = Hq;
  bp.projmatrix = settings->projmatrix;
  bp.viewmatrix = settings->viewmatrix;
  // The ray/plane form of the hit-point gradient equals the reference's form
  // when the blended transform and the preprocess backward's rebuilt transform
  // are the same matrix: scale_modifier 1 and the same image size.
  bp.ray_hit = (!given_T && settings->scale_modifier == 1.0f && Wq == W && Hq == H) ? 1 : 0;
  bp.raw_T = given_T ? 1 : 0;
  bp.ranges = im.ranges;
  bp.tile_order = im.order;
  bp.point_list = b.vals_sorted;
  bp.records = g.records;
  bp.table = surfels->features;
  bp.offsets = surfels->offsets;
  bp.gridrange = surfels->gridrange;
  bp.final_T = im.final_T;
  bp.n_contrib = im.n_contrib;
  bp.dL_dcolor = gi->dL_dout_color;
  bp.dL_dothers = gi->dL_dout_others;
  bp.dL_dtable = go->dL_dtable;
  bp.dL_dtable_fixed = table_fixed;
  bp.grad_max_bits = grad_max;
  bp.accum = accum;
  rc = blend_backward_launch(bp, settings->table_fp16, stream);
  if (rc) return rc;
  if (det) {
    rc = table_grad_finish_launch(table_fixed, table_entries, grad_max, go->dL_dtable, stream);
    if (rc) return rc;
  }
  rc = preprocess_backward_launch(P, surfels->means3D, surfels->scales, surfels->rotations, gi->radii,
                                  settings->viewmatrix, settings->projmatrix, Wq, Hq, accum,
                                  surfels->transmat_precomp, *go, stream);
  if (rc || !shc) return rc;
  // computeColorFromSH's backward after the mean gradient is written (it adds to it)
  return sh_color_backward_launch(P, settings->sh_degree, surfels->sh_coeffs, surfels->means3D, settings->campos,
                                  surfels->shs, gi->radii, drgb, go->dL_dshs, go->dL_dmeans3D, stream);
}

int ns_read_device_status(void* geom, int32_t P, void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!geom || P < 0) return NS_ERR_INVALID;
  GeomState g = carve_geom(geom, P, nullptr);
  uint32_t err = 0;
  NS_CUDA_TRY(cudaMemcpyAsync(&err, g.err, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream));
  NS_CUDA_TRY(cudaMemsetAsync(g.err, 0, sizeof(uint32_t), stream));
  NS_CUDA_TRY(cudaStreamSynchronize(stream));
  return err ? NS_ERR_DEVICE : NS_OK;
}

int ns_wait_selftest(const uint32_t* flag, void* geom, int32_t P, void* stream) {
  if (!flag || !geom || P < 0) return NS_ERR_INVALID;
  GeomState g = carve_geom(geom, P, nullptr);
  return wait_selftest_launch(flag, g.err, reinterpret_cast<cudaStream_t>(stream));
}

int ns_mark_visible(int32_t P, const float* means3D, const float* viewmatrix,
                    const float* projmatrix, uint8_t* present, void* stream) {
  if (P < 0) return NS_ERR_INVALID;
  if (P == 0) return NS_OK;
  if (!means3D || !viewmatrix || !projmatrix || !present) return NS_ERR_INVALID;
  return mark_visible_launch(P, means3D, viewmatrix, present,
                             reinterpret_cast<cudaStream_t>(stream));
}

int ns_mlp_forward(const float* feat, int32_t in_dims, int64_t npix, const uint16_t* weights,
                   int32_t hidden, int32_t out_dims, const float* alpha, const float* bg_host,
                   float* rgb, void* stream) {
  return mlp_launch(feat, in_dims, npix, weights, hidden, out_dims, alpha, bg_host, rgb,
                    reinterpret_cast<cudaStream_t>(stream));
}

int ns_allmap_decode(const float* allmap, const float* viewmatrix, const float* rays_d,
                     const float* ray_o, int32_t width, int32_t height, float depth_ratio,
                     float* maps, void* stream) {
  if (width < 0 || height < 0) return NS_ERR_INVALID;
  if ((int64_t)width * height == 0) return NS_OK;
  if (!allmap || !viewmatrix || !rays_d || !ray_o || !maps) return NS_ERR_INVALID;
  return allmap_decode_launch(allmap, viewmatrix, rays_d, ray_o, width, height, depth_ratio, maps,
                              reinterpret_cast<cudaStream_t>(stream));
}

int ns_normal_error(const float* allmap, const float* viewmatrix, const float* rays_d,
                    const float* ray_o, int32_t width, int32_t height, float* err, void* stream) {
  if (width < 0 || height < 0) return NS_ERR_INVALID;
  if ((int64_t)width * height == 0) return NS_OK;
  if (!allmap || !viewmatrix || !rays_d || !ray_o || !err) return NS_ERR_INVALID;
  return normal_error_launch(allmap, viewmatrix, rays_d, ray_o, width, height, err,
                             reinterpret_cast<cudaStream_t>(stream));
}

size_t ns_normal_error_scratch_bytes(int32_t width, int32_t height) {
  if (width <= 0 || height <= 0) return 0;
  return align_up((size_t)width * (size_t)height * 6 * sizeof(float));
}

int ns_normal_error_backward(const float* allmap, const float* viewmatrix, const float* rays_d,
                             const float* ray_o, int32_t width, int32_t height,
                             const float* dL_derr, int64_t derr_stride, float* dL_dallmap,
                             void* scratch, size_t scratch_bytes, void* stream) {
  if (width < 0 || height < 0 || derr_stride < 0) return NS_ERR_INVALID;
  if ((int64_t)width * height == 0) return NS_OK;
  if (!allmap || !viewmatrix || !rays_d || !ray_o || !dL_derr || !dL_dallmap || !scratch)
    return NS_ERR_INVALID;
  if (scratch_bytes < ns_normal_error_scratch_bytes(width, height)) return NS_ERR_SCRATCH;
  return normal_error_backward_launch(allmap, viewmatrix, rays_d, ray_o, width, height, dL_derr,
                                      derr_stride, dL_dallmap, static_cast<float*>(scratch),
                                      reinterpret_cast<cudaStream_t>(stream));
}

int ns_mlp_backward(const float* feat, int32_t in_dims, int64_t npix, const uint16_t* weights,
                    int32_t hidden, int32_t out_dims, const float* alpha, const float* dL_drgb,
                    float* dL_dfeat, float* dL_dweights, void* stream) {
  return mlp_backward_launch(feat, in_dims, npix, weights, hidden, out_dims, alpha, dL_drgb,
                             dL_dfeat, dL_dweights, reinterpret_cast<cudaStream_t>(stream));
}

int ns_rvq_decode(const uint8_t* idx, const float* codebooks, float* out, int64_t n,
                  int32_t stages, int32_t entries, int32_t dims, void* stream) {
  return rvq_decode_launch(idx, codebooks, out, n, stages, entries, dims,
                           reinterpret_cast<cudaStream_t>(stream));
}

size_t ns_radix_sort_temp_bytes(int64_t n) { return radix_sort_temp_bytes(n); }

int ns_radix_sort_pairs(const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                        uint32_t* vals_out, uint64_t* keys_alt, uint32_t* vals_alt, int64_t n,
                        int32_t end_bit, void* temp, size_t temp_bytes, void* stream) {
  if (n > 0 && (!keys_in || !vals_in || !keys_out || !vals_out || !keys_alt || !vals_alt || !temp))
    return NS_ERR_INVALID;
  if (keys_in == keys_alt || vals_in == vals_alt) return NS_ERR_INVALID;
  return radix_sort_launch(keys_in, vals_in, keys_out, vals_out, keys_alt, vals_alt, n, end_bit,
                           temp, temp_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int ns_render_frame(const ns_raster_settings* settings, const ns_frame_inputs* in,
                    const ns_frame_outputs* out, void* geom, size_t geom_bytes, void* binning,
                    size_t binning_bytes, void* image, size_t image_bytes,
                    int64_t* num_rendered, int flags, void* stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  int rc = validate_settings(settings);
  if (settings && (settings->kernel_type != 0 || settings->render_mode != 0 || settings->levels == 0))
    return NS_ERR_UNSUPPORTED;  // the frame renders the hash grid (no per-surfel colours)
  if (rc) return rc;
  if (!in || !out) return NS_ERR_INVALID;
  const int P = in->P;
  if (P < 0) return NS_ERR_INVALID;
  if (num_rendered) *num_rendered = 0;
  if (!in->rvq_idx || !in->codebooks || !in->base || !in->decoded || !in->features ||
      !in->offsets || !in->gridrange || !in->mlp_weights)
    return NS_ERR_INVALID;
  if (!out->rgb || !out->out_color || !out->out_others || !out->radii) return NS_ERR_INVALID;
  if (in->dims < 10) return NS_ERR_INVALID;
  if (settings->level_dim != 2 || settings->channels != 32) return NS_ERR_UNSUPPORTED;
  if (settings->record_transmittance) return NS_ERR_UNSUPPORTED;
  if (geom_bytes < ns_geometry_scratch_bytes(P)) return NS_ERR_SCRATCH;
  if (image_bytes < ns_image_scratch_bytes(settings->image_width, settings->image_height))
    return NS_ERR_SCRATCH;
  const int W = settings->image_width, H = settings->image_height;
  GeomState g = carve_geom(geom, P, nullptr);
  ImageState im = carve_image(image, W, H, nullptr);
  void* const* ev = in->stage_events;
  NS_CUDA_TRY(cudaMemsetAsync(g.err, 0, sizeof(uint32_t), stream));
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[0], stream));
  if (!(flags & NS_FLAG_SKIP_DECODE)) {
    rc = rvq_decode_launch(in->rvq_idx, in->codebooks, in->decoded, P, in->stages, in->entries,
                           in->dims, stream);
    if (rc) return rc;
  }
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[1], stream));
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[2], stream));
  rc = preprocess_mix_launch(P, in->base, in->decoded, in->dims, in->mix, in->ap_level,
                             settings->scale_modifier, settings->beta, settings->viewmatrix,
                             settings->projmatrix,
                             W, H, g.records, g.bin, out->radii, g.tiles, g.depth_keys,
                             g.depth_vals, g.block_sums, stream);
  if (rc) return rc;
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[3], stream));
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[4], stream));
  rc = bin_and_render(settings, P, g, im, binning, binning_bytes, in->features, in->offsets,
                      in->gridrange, out->out_color, out->out_others, nullptr, nullptr, nullptr,
                      num_rendered, flags & ~NS_FLAG_SKIP_DECODE, stream, ev);
  if (rc) return rc;
  const size_t HW = (size_t)W * H;
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[8], stream));
  rc = mlp_launch(out->out_color, (int)settings->channels, (int64_t)HW, in->mlp_weights,
                  in->mlp_hidden, 3, out->out_others + HW, in->bg_host, out->rgb, stream);
  if (rc) return rc;
  if (ev) NS_CUDA_TRY(cudaEventRecord((cudaEvent_t)ev[9], stream));
  return NS_OK;
}

}  // extern "C"
