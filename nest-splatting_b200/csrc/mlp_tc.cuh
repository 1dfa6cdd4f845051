// Colour MLP forward on the 5th-generation tensor cores (tcgen05, accumulators
// in TMEM). Included by mlp.cu inside its anonymous namespace.
//
// A CTA of 128 threads runs 128-pixel tiles (thread t = pixel row t of the
// MMA's M = 128): each thread converts its pixel's 32 fp32 features to fp16 and
// writes them as row t of A1 in shared memory; one thread issues the layer's
// tcgen05.mma (fp16 x fp16 -> fp32 in TMEM) and commits it to an mbarrier; each
// thread reads its row back from TMEM (tcgen05.ld), applies ReLU, rounds to
// fp16 and writes the next layer's A row. Operands use the no-swizzle K-major
// canonical layout: 8-row x 16-byte core matrices, LBO = 128 B between the two
// K halves of an MMA, SBO = (K / 8) x 128 B between 8-row groups. The next
// tile's features are loaded into registers while a tile's layers run. The
// roundings are those of the mma.sync path (fp16 operands, fp32 accumulation,
// each layer rounded to fp16), and the images it gives are the same.
//
// TMEM: 128 columns per CTA, allocated once and freed at the end by warp 0; the
// 48 KB of shared memory a CTA asks for keeps at most 4 CTAs (512 columns) on
// an SM, so an allocation never waits for another CTA.
constexpr int kTcThreads = 128;
constexpr int kTcCols = 128;        // TMEM columns: D1 / D3 at 0, D2 at 64
constexpr int kTcSmemBytes = 49152; // at most 4 CTAs per SM (4 x 128 TMEM columns)

struct TcSmem {
  uint16_t w1[64 * 32];   // B of layer 1: N = 64, K = 32
  uint16_t w2[64 * 64];   // B of layer 2: N = 64, K = 64
  uint16_t w3[16 * 64];   // B of layer 3: N = 16 (rows 3..15 zero), K = 64
  uint16_t a1[128 * 32];  // A of layer 1
  uint16_t a2[128 * 64];  // A of layers 2 and 3
  uint64_t bar;
  uint32_t tbase;
};
static_assert(sizeof(TcSmem) <= kTcSmemBytes, "shared-memory budget");

// Half offset of element (r, k) in a K-major canonical matrix with K columns.
__device__ __forceinline__ int canon(int r, int k, int K) {
  return (((r >> 3) * (K >> 3) + (k >> 3)) * 8 + (r & 7)) * 8 + (k & 7);
}

// Shared-memory matrix descriptor for K-step s (16 columns) of a canonical
// K-major matrix at `base` with K columns (no swizzle, version 1).
__device__ __forceinline__ uint64_t tc_desc(const uint16_t* base, int s, int K) {
  const uint32_t start = (uint32_t)__cvta_generic_to_shared(base) + (uint32_t)s * 256u;
  const uint64_t lbo = 128u, sbo = (uint64_t)(K >> 3) * 128u;
  return (uint64_t)((start >> 4) & 0x3fffu) | ((lbo >> 4) << 16) | ((sbo >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: D fp32, A and B fp16, both K-major.
__host__ __device__ constexpr uint32_t tc_idesc(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, int acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   (unsigned)__cvta_generic_to_shared(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 4; i++) v[i] = __uint_as_float(r[i]);
}

// ReLU, fp16 rounding and the write of 32 columns (k0 .. k0+31) of row r of a
// canonical K-major matrix with K columns.
__device__ __forceinline__ void tc_store_row(uint16_t* m, int r, int k0, int K, const float (&v)[32], bool relu) {
#pragma unroll
  for (int c = 0; c < 4; c++) {
    uint32_t h[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float x0 = v[8 * c + 2 * j], x1 = v[8 * c + 2 * j + 1];
      if (relu) {
        x0 = fmaxf(x0, 0.f);
        x1 = fmaxf(x1, 0.f);
      }
      h[j] = pack_half2(x0, x1);
    }
    *reinterpret_cast<uint4*>(m + canon(r, k0 + 8 * c, K)) = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

__device__ __forceinline__ void tc_sync_before() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__global__ void __launch_bounds__(kTcThreads, 4)
mlp_tc_kernel(const float* __restrict__ feat, int64_t npix, const uint16_t* __restrict__ weights,
              const float* __restrict__ alpha, float bg0, float bg1, float bg2, int use_bg,
              float* __restrict__ rgb) {
  extern __shared__ __align__(128) unsigned char tc_smem_raw[];
  TcSmem& S = *reinterpret_cast<TcSmem*>(tc_smem_raw);
  const int t = threadIdx.x, w = t >> 5;

  // Weights into the canonical layouts (layer 3 padded to 16 rows with zeros).
  for (int i = t; i < 64 * 32; i += kTcThreads) S.w1[canon(i / 32, i % 32, 32)] = weights[i];
  for (int i = t; i < 64 * 64; i += kTcThreads) S.w2[canon(i / 64, i % 64, 64)] = weights[64 * 32 + i];
  for (int i = t; i < 16 * 64; i += kTcThreads)
    S.w3[canon(i / 64, i % 64, 64)] = i < 3 * 64 ? weights[64 * 32 + 64 * 64 + i] : (uint16_t)0;
  if (w == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(&S.tbase)),
                 "r"(kTcCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (t == 0) {
    mbar_init_shared(&S.bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_sync_before();
  const uint32_t tmem = S.tbase;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * w) << 16);
  constexpr uint32_t kId64 = tc_idesc(128, 64), kId16 = tc_idesc(128, 16);
  const int64_t ntiles = div_up64(npix, kTcThreads);
  uint32_t phase = 0;
  // An MMA always completes; the poll bound only keeps the wait finite (a
  // second bounded wait before TMEM or the operands are reused).
  auto wait_mma = [&]() {
    if (mbar_wait_parity(&S.bar, phase, kSpinLimit) <= 0) mbar_wait_parity(&S.bar, phase, kSpinLimit);
    phase ^= 1u;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  };

  // The next tile's features are loaded while this tile's layers run.
  float nf[32];
  auto load_features = [&](int64_t tl) {
    const int64_t q = tl * kTcThreads + t;
    const bool v = tl < ntiles && q < npix;
#pragma unroll
    for (int c = 0; c < 32; c++) nf[c] = v ? __ldg(feat + (int64_t)c * npix + q) : 0.f;
  };
  load_features(blockIdx.x);
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t px = tile * kTcThreads + t;
    const bool valid = px < npix;
    tc_store_row(S.a1, t, 0, 32, nf, false);
    load_features(tile + gridDim.x);
    tc_sync_before();
    if (t == 0) {
#pragma unroll
      for (int s = 0; s < 2; s++) tc_mma(tmem, tc_desc(S.a1, s, 32), tc_desc(S.w1, s, 32), kId64, s);
      tc_commit(&S.bar);
    }
    wait_mma();
    {
      float v[32];
      tc_ld32(lane_base + 0, v);
      tc_store_row(S.a2, t, 0, 64, v, true);
      tc_ld32(lane_base + 32, v);
      tc_store_row(S.a2, t, 32, 64, v, true);
    }
    tc_sync_before();
    if (t == 0) {
#pragma unroll
      for (int s = 0; s < 4; s++) tc_mma(tmem + 64, tc_desc(S.a2, s, 64), tc_desc(S.w2, s, 64), kId64, s);
      tc_commit(&S.bar);
    }
    wait_mma();
    {
      float v[32];
      tc_ld32(lane_base + 64, v);
      tc_store_row(S.a2, t, 0, 64, v, true);
      tc_ld32(lane_base + 96, v);
      tc_store_row(S.a2, t, 32, 64, v, true);
    }
    tc_sync_before();
    if (t == 0) {
#pragma unroll
      for (int s = 0; s < 4; s++) tc_mma(tmem, tc_desc(S.a2, s, 64), tc_desc(S.w3, s, 64), kId16, s);
      tc_commit(&S.bar);
    }
    wait_mma();
    float y[4];
    tc_ld4(lane_base + 0, y);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    if (valid) {
      const float a_px = alpha ? alpha[px] : 1.0f;
#pragma unroll
      for (int col = 0; col < 3; col++) {
        float v = sigmoidf(__half2float(__float2half_rn(y[col])));
        if (alpha && !(a_px > 0.f)) v = 0.f;
        if (use_bg) v += (1.0f - a_px) * (col == 0 ? bg0 : col == 1 ? bg1 : bg2);
        rgb[col * npix + px] = v;
      }
    }
  }
  __syncthreads();
  if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols));
}
