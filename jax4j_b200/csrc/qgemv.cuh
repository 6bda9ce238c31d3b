// Batched dequant-GEMV kernel (included by quant.cu inside namespace j4b::<anonymous>).
//
// One CTA of 16 warps per SM. A CTA owns one 1024-column K range ("split") of a run of 16-row tiles. For
// each tile, the K range's quant bytes and scale bytes are contiguous in the repacked layout, so
// one elected thread streams them into a ring of shared-memory stages with 1-D TMA bulk copies
// (cp.async.bulk, completion counted on an mbarrier); the eight warps decode their 128-column
// slice from shared memory into fp16 mma.m16n8k16 fragments, multiply them by the x fragments
// they keep in registers for the whole run, and fold the per-block scales in fp32. Warp partials
// of a tile are summed through shared memory; the K splits of a tile group are combined by the
// last CTA of the group to finish (one arrival counter per group, partials in the weight's
// scratch), which also applies `add`.
//
// Launches use programmatic dependent launch: the weight prefetch of one GEMV overlaps the tail
// of the kernel before it (see the comment at the prefetch).
//
// Every mbarrier wait is bounded in time (0.2 s): on timeout the CTA records an error code in the weight's
// status word, waits (bounded) for its copies in flight, and returns.

constexpr int kGemvThreads = 512;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// 1-D bulk copy global -> this CTA's own shared memory (one destination CTA), 16-byte aligned,
// size % 16 == 0, for weight bytes that one launch reads exactly once: the copy carries an L2
// evict-first policy, so the streamed weights do not push x, y and the split-K partials (read
// again within the launch, or by the next one) out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_load_1d_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                   uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
  return mbar_wait_timed(smem_u32(bar), phase);
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue early /
// wait until the previous kernel's writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same with a zero accumulator input: starts a chain without zeroing registers first.
__device__ __forceinline__ void mma16816_z(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                           uint32_t a3, uint32_t b0, uint32_t b1) {
  const float z = 0.0f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ uint32_t rotr(uint32_t v, int s) { return __funnelshift_r(v, v, s); }
__device__ __forceinline__ uint32_t lop_or(uint32_t v, uint32_t mask, uint32_t bias) {
  return (v & mask) | bias;
}
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
// Q8_0: 4 bytes (a0..a3 or a4..a7) -> two half2 holding the exact integer codes.
__device__ __forceinline__ void q8_pairs(uint32_t w, uint32_t& p0, uint32_t& p1) {
  const uint32_t kBias = 0x64806480u;  // half2(1152, 1152): 1024 + the 0x80 code offset
  p0 = h2sub(__byte_perm(w, 0x64646464u, 0x4140), kBias);
  p1 = h2sub(__byte_perm(w, 0x64646464u, 0x4342), kBias);
}
// 4-bit: one word -> four half2 of (1 + q/16).
__device__ __forceinline__ void q4_pairs(uint32_t w, uint32_t (&a)[4]) {
  const uint32_t kMask = 0x03C003C0u, kOne = 0x3C003C00u;
  a[0] = lop_or(w, kMask, kOne);
  a[1] = lop_or(rotr(w, 4), kMask, kOne);
  a[2] = lop_or(rotr(w, 8), kMask, kOne);
  a[3] = lop_or(rotr(w, 12), kMask, kOne);
}
// 2-bit: one word -> eight half2 of (1 + c/4); pairs 0..3 are k-step 0, 4..7 k-step 1.
__device__ __forceinline__ uint32_t q2_pair(uint32_t w, int p) {
  return lop_or(rotr(w, 2 * p), 0x03000300u, 0x3C003C00u);
}
// 6-bit (Q6_K): the low-nibble word of k-step ks and the group's high-crumb word -> four half2
// holding the exact integers q - 32: pair p's nibbles go to bits 0..3 / 16..19 and its crumbs to
// bits 4..5 / 20..21 of half2(1024, 1024), then 1056 = 1024 + 32 is subtracted.
__device__ __forceinline__ void q6_pairs(uint32_t nw, uint32_t cw, int ks, uint32_t (&a)[4]) {
  const uint32_t kBias = 0x64206420u;  // half2(1056, 1056)
#pragma unroll
  for (int p = 0; p < 4; p++) {
    const uint32_t v = (rotr(nw, 6 + 4 * p) & 0x000F000Fu) | (rotr(cw, 4 + 2 * (4 * ks + p)) & 0x00300030u);
    a[p] = h2sub(v | 0x64006400u, kBias);
  }
}
// Q6_K sub-block scale j (0..7) of the half super-block held in two words, as a float.
__device__ __forceinline__ float q6_scale(uint2 s, int j) {
  return (float)(int8_t)(((j < 4 ? s.x : s.y) >> (8 * (j & 3))) & 0xFF);
}

// Bytes of one tile chunk, and the tiles per bulk copy: as many as two stages, the staged x and
// the warp-partial buffer leave room for in shared memory (a copy of 35-147 KB; bulk-copy
// throughput grows with the copy size, and more tiles per stage means fewer barriers and more
// independent mma chains per warp).
template <int QT>
struct GemvTraits {
  static constexpr int kQ = QT == J4B_Q8_0 ? 512 : (QT == J4B_Q2_0 ? 128 : (QT == J4B_Q6_K ? 384 : 256));
  static constexpr int kM = QT == J4B_Q2_0 ? 8 : (QT == J4B_Q6_K ? 36 : 32);
  static constexpr int kChunk = 32 * (kQ + kM);  // bytes of one full tile chunk
  static constexpr int kStages = 2;
};
template <int QT, int NT>
constexpr int kTilesPerCopy = QT == J4B_Q8_0   ? (NT == 1 ? 4 : 2)
                              : QT == J4B_Q2_0 ? 8
                              : QT == J4B_Q6_K ? (NT == 1 ? 6 : 2)
                                               : (NT == 1 ? 8 : 4);

struct GemvArgs {
  const uint8_t* data;
  Layout L;
  int64_t rows, cols, kpad, rt;
  const float* x;
  const float* add;
  float* y;
  int batch;  // batch rows handled by this launch (<= 8 * NT)
  int ksplit;
  int tiles_per_cta;
  int cluster;         // 1: the ksplit CTAs of a tile group form a cluster and fold through DSMEM
  float* partials;     // [ksplit][rt][256] (global split-K fold only)
  unsigned* arrivals;  // one counter per tile group
  int* status;         // nonzero after a bounded wait gave up
  // All-gather over peer memory (nranks > 1): this rank's rows of y go straight into every
  // rank's gathered buffer, [batch][rows * nranks] flagged words in the parity half selected by
  // the local step counter (see gather_store).
  int nranks, rank;
  unsigned long long* peer_y[kMaxPeerRanks];
  const unsigned* step;
  int64_t half_words;
};

// Where this launch's outputs go in the gathered buffers: the parity half's offset and the flag
// of this step (step + 1). Read after the dependency wait.
struct GatherSlot {
  int64_t off = 0;
  unsigned flag = 0;
};
__device__ __forceinline__ GatherSlot gather_slot(const GemvArgs& a) {
  GatherSlot g;
  if (a.nranks > 1) {
    const unsigned st = *a.step;
    g.off = (int64_t)(st & 1u) * a.half_words;
    g.flag = st + 1u;
  }
  return g;
}

// Stores one output, locally or into every rank's gathered buffer.
__device__ __forceinline__ void store_y(const GemvArgs& a, const GatherSlot& gs, int bcol, int64_t r, float v) {
  if (a.nranks <= 1) {
    a.y[(int64_t)bcol * a.rows + r] = v;
    return;
  }
  const int64_t idx = gs.off + (int64_t)bcol * (a.rows * a.nranks) + (int64_t)a.rank * a.rows + r;
  for (int p = 0; p < a.nranks; ++p) gather_store(a.peer_y[p] + idx, v, gs.flag);
}

constexpr int kXStride = 1024 + 4;  // floats per staged x row (padding spreads the banks)

// Shared memory: [stages | warp partials | staged x | stage barriers | (cluster mode) this CTA's
// per-tile totals]. The cluster fold reuses the bytes from offset 0 as the leader's landing area.
template <int QT, int NT>
__host__ __device__ constexpr int gemv_smem_base() {
  return GemvTraits<QT>::kStages * kTilesPerCopy<QT, NT> * GemvTraits<QT>::kChunk +
         kTilesPerCopy<QT, NT> * 8 * NT * 128 * 4 + 8 * NT * kXStride * 4 +
         GemvTraits<QT>::kStages * 8 + 16;
}

// x block sums per warp chunk (Q8_0 and Q6_K multiply exact signed codes and need none)
template <int QT>
constexpr int kXBlocks = (QT == J4B_Q2_0 || QT == J4B_Q6_K) ? 1 : 4;

// One warp's contribution to one 16-row tile: its 128-column slice of the tile's chunk (quants at
// sq, scales at sm) times the x fragments, accumulated into acc (C-fragment layout: rows g and
// g+8, batch columns 2t and 2t+1 of each n-tile). Per 32-column block, the hi and lo halves of x
// run through one accumulator chain that starts with a zero-C mma (four mma deep, no zeroing and
// no hi + lo add), and the block scale and the code-offset term are two fmas per output.
template <int QT, int NT>
__device__ __forceinline__ void tile_compute(const uint8_t* __restrict__ sq,
                                             const uint8_t* __restrict__ sm, int warp, int lane,  // warp = K chunk 0..7
                                             const uint32_t (&bh)[NT][8][2],
                                             const uint32_t (&bl)[NT][8][2],
                                             const float (&xblk)[NT][kXBlocks<QT>][2],
                                             float (&acc)[NT][4]) {
  const int g = lane >> 2, t = lane & 3;
  // c[n] = W_block . x over k-steps j0 and j0 + 1 (hi and lo), fresh chain per block
  auto block_mma = [&](float (&c)[NT][4], const uint32_t (&a)[2][4], int j0) {
#pragma unroll
    for (int n = 0; n < NT; n++) {
      mma16816_z(c[n], a[0][0], a[0][1], a[0][2], a[0][3], bh[n][j0][0], bh[n][j0][1]);
      mma16816(c[n], a[0][0], a[0][1], a[0][2], a[0][3], bl[n][j0][0], bl[n][j0][1]);
      mma16816(c[n], a[1][0], a[1][1], a[1][2], a[1][3], bh[n][j0 + 1][0], bh[n][j0 + 1][1]);
      mma16816(c[n], a[1][0], a[1][1], a[1][2], a[1][3], bl[n][j0 + 1][0], bl[n][j0 + 1][1]);
    }
  };
  if constexpr (QT == J4B_Q8_0) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint4 line = *reinterpret_cast<const uint4*>(sq + (warp * 4 + q) * 512 + lane * 16);
      const uint32_t sc = *reinterpret_cast<const uint32_t*>(sm + (warp * 4 + q) * 32 + g * 4);
      uint32_t a[2][4];
      q8_pairs(line.x, a[0][0], a[0][1]);
      q8_pairs(line.y, a[0][2], a[0][3]);
      q8_pairs(line.z, a[1][0], a[1][1]);
      q8_pairs(line.w, a[1][2], a[1][3]);
      float c[NT][4];
      block_mma(c, a, 2 * q);
      const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc));
#pragma unroll
      for (int n = 0; n < NT; n++) {
        acc[n][0] = fmaf(d.x, c[n][0], acc[n][0]);
        acc[n][1] = fmaf(d.x, c[n][1], acc[n][1]);
        acc[n][2] = fmaf(d.y, c[n][2], acc[n][2]);
        acc[n][3] = fmaf(d.y, c[n][3], acc[n][3]);
      }
    }
  } else if constexpr (QT == J4B_Q4_0) {
    const uint4 l0 = *reinterpret_cast<const uint4*>(sq + warp * 1024 + lane * 16);
    const uint4 l1 = *reinterpret_cast<const uint4*>(sq + warp * 1024 + 512 + lane * 16);
    const uint32_t wv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint32_t sc = *reinterpret_cast<const uint32_t*>(sm + (warp * 4 + q) * 32 + g * 4);
      uint32_t a[2][4];
      q4_pairs(wv[2 * q], a[0]);
      q4_pairs(wv[2 * q + 1], a[1]);
      float c[NT][4];
      block_mma(c, a, 2 * q);
      // sum w x = d (16 C' - 24 X), C' = sum (1 + q/16) x
      const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc));
      const float c0 = 16.f * d.x, c1 = 16.f * d.y, x0 = -24.f * d.x, x1 = -24.f * d.y;
#pragma unroll
      for (int n = 0; n < NT; n++) {
        acc[n][0] = fmaf(x0, xblk[n][q][0], fmaf(c0, c[n][0], acc[n][0]));
        acc[n][1] = fmaf(x0, xblk[n][q][1], fmaf(c0, c[n][1], acc[n][1]));
        acc[n][2] = fmaf(x1, xblk[n][q][0], fmaf(c1, c[n][2], acc[n][2]));
        acc[n][3] = fmaf(x1, xblk[n][q][1], fmaf(c1, c[n][3], acc[n][3]));
      }
    }
  } else if constexpr (QT == J4B_Q2_0) {
    const uint4 line = *reinterpret_cast<const uint4*>(sq + warp * 512 + lane * 16);
    const uint32_t sc = *reinterpret_cast<const uint32_t*>(sm + warp * 32 + g * 4);
    const uint32_t wv[4] = {line.x, line.y, line.z, line.w};
    float c[NT][4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      uint32_t a[2][4];
#pragma unroll
      for (int ks = 0; ks < 2; ks++)
#pragma unroll
        for (int p = 0; p < 4; p++) a[ks][p] = q2_pair(wv[q], 4 * ks + p);
      if (q == 0) {
        block_mma(c, a, 0);
      } else {
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
          for (int ks = 0; ks < 2; ks++) {
            mma16816(c[n], a[ks][0], a[ks][1], a[ks][2], a[ks][3], bh[n][2 * q + ks][0], bh[n][2 * q + ks][1]);
            mma16816(c[n], a[ks][0], a[ks][1], a[ks][2], a[ks][3], bl[n][2 * q + ks][0], bl[n][2 * q + ks][1]);
          }
      }
    }
    // sum w x = d (4 C' - 5 X), C' = sum (1 + c/4) x
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc));
    const float c0 = 4.f * d.x, c1 = 4.f * d.y, x0 = -5.f * d.x, x1 = -5.f * d.y;
#pragma unroll
    for (int n = 0; n < NT; n++) {
      acc[n][0] = fmaf(x0, xblk[n][0][0], fmaf(c0, c[n][0], acc[n][0]));
      acc[n][1] = fmaf(x0, xblk[n][0][1], fmaf(c0, c[n][1], acc[n][1]));
      acc[n][2] = fmaf(x1, xblk[n][0][0], fmaf(c1, c[n][2], acc[n][2]));
      acc[n][3] = fmaf(x1, xblk[n][0][1], fmaf(c1, c[n][3], acc[n][3]));
    }
  } else if constexpr (QT == J4B_Q6_K) {
    // warp w holds half (w & 1) of super-block w / 2 of the CTA's K range; one scale d * sc per
    // 16-column k-step, so each k-step is its own hi + lo chain of exact signed codes
    const int h = warp & 1;
    const uint8_t* lp = sq + warp * 1536 + lane * 48;
    const uint4 n0 = *reinterpret_cast<const uint4*>(lp);
    const uint4 n1 = *reinterpret_cast<const uint4*>(lp + 16);
    const uint4 cr = *reinterpret_cast<const uint4*>(lp + 32);
    const uint8_t* mp = sm + (warp >> 1) * 288;
    const uint2 s0 = *reinterpret_cast<const uint2*>(mp + (2 * g) * 16 + 8 * h);
    const uint2 s1 = *reinterpret_cast<const uint2*>(mp + (2 * g + 1) * 16 + 8 * h);
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(mp + 256 + 4 * g));
    const uint32_t wv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
    const uint32_t cv[4] = {cr.x, cr.y, cr.z, cr.w};
#pragma unroll
    for (int j = 0; j < 8; j++) {
      uint32_t a[4];
      q6_pairs(wv[j], cv[j >> 1], j & 1, a);
      const float f0 = d.x * q6_scale(s0, j), f1 = d.y * q6_scale(s1, j);
#pragma unroll
      for (int n = 0; n < NT; n++) {
        float c[4];
        mma16816_z(c, a[0], a[1], a[2], a[3], bh[n][j][0], bh[n][j][1]);
        mma16816(c, a[0], a[1], a[2], a[3], bl[n][j][0], bl[n][j][1]);
        acc[n][0] = fmaf(f0, c[0], acc[n][0]);
        acc[n][1] = fmaf(f0, c[1], acc[n][1]);
        acc[n][2] = fmaf(f1, c[2], acc[n][2]);
        acc[n][3] = fmaf(f1, c[3], acc[n][3]);
      }
    }
  } else {  // Q4_K: warp w holds half (w & 1) of super-block w / 2 of the CTA's K range
    const int h = warp & 1;
    const uint4 l0 = *reinterpret_cast<const uint4*>(sq + warp * 1024 + lane * 32);
    const uint4 l1 = *reinterpret_cast<const uint4*>(sq + warp * 1024 + lane * 32 + 16);
    const uint8_t* mp = sm + (warp >> 1) * 256 + g * 32;
    const uint4 mm[2] = {*reinterpret_cast<const uint4*>(mp), *reinterpret_cast<const uint4*>(mp + 16)};
    // Lane t decodes sub-block 4h+t for rows g and g+8: coefficients 16 d sc and
    // -(16 d sc + dmin m); the four lanes of the group then exchange them.
    float cs[2], cx[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const uint32_t w0 = mm[r].x, w1 = mm[r].y, w2 = mm[r].z, w3 = mm[r].w;
      const float d = __half2float(__ushort_as_half((uint16_t)(w0 & 0xFFFF)));
      const float dmin = __half2float(__ushort_as_half((uint16_t)(w0 >> 16)));
      const int j = 4 * h + t;
      int sc, mn;
      if (j < 4) {
        sc = (w1 >> (8 * j)) & 63;
        mn = (w2 >> (8 * j)) & 63;
      } else {
        const int jj = j - 4;
        const uint32_t qj4 = (w3 >> (8 * jj)) & 0xFF;  // q[j+4]
        sc = (qj4 & 0xF) | (((w1 >> (8 * jj + 6)) & 3) << 4);
        mn = (qj4 >> 4) | (((w2 >> (8 * jj + 6)) & 3) << 4);
      }
      const float ds = d * (float)sc;
      cs[r] = 16.f * ds;
      cx[r] = -fmaf(16.f, ds, dmin * (float)mn);
    }
    const uint32_t wv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      uint32_t a[2][4];
      q4_pairs(wv[2 * q], a[0]);
      q4_pairs(wv[2 * q + 1], a[1]);
      float c[NT][4];
      block_mma(c, a, 2 * q);
      const int src = (lane & ~3) | q;
      const float s0 = __shfl_sync(0xffffffffu, cs[0], src);
      const float s1 = __shfl_sync(0xffffffffu, cs[1], src);
      const float z0 = __shfl_sync(0xffffffffu, cx[0], src);
      const float z1 = __shfl_sync(0xffffffffu, cx[1], src);
#pragma unroll
      for (int n = 0; n < NT; n++) {
        acc[n][0] = fmaf(z0, xblk[n][q][0], fmaf(s0, c[n][0], acc[n][0]));
        acc[n][1] = fmaf(z0, xblk[n][q][1], fmaf(s0, c[n][1], acc[n][1]));
        acc[n][2] = fmaf(z1, xblk[n][q][0], fmaf(s1, c[n][2], acc[n][2]));
        acc[n][3] = fmaf(z1, xblk[n][q][1], fmaf(s1, c[n][3], acc[n][3]));
      }
    }
  }
}

// Batch <= 4: the B fragment carries x's fp16 hi part of batch b in n-column 2b and its lo part
// in column 2b+1, so one mma covers both halves and lane (g, t) reads batch t of rows g and
// g + 8 as c0 + c1 and c2 + c3. acc[0] is row g, acc[1] row g + 8.
template <int QT>
__device__ __forceinline__ void tile_compute_pk(const uint8_t* __restrict__ sq,
                                                const uint8_t* __restrict__ sm, int warp, int lane,
                                                const uint32_t (&bp)[8][2],
                                                const float (&xblk)[kXBlocks<QT>],
                                                float (&acc)[2]) {
  const int g = lane >> 2, t = lane & 3;
  if constexpr (QT == J4B_Q8_0) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint4 line = *reinterpret_cast<const uint4*>(sq + (warp * 4 + q) * 512 + lane * 16);
      const uint32_t sc = *reinterpret_cast<const uint32_t*>(sm + (warp * 4 + q) * 32 + g * 4);
      float c[4];
      uint32_t a0, a1, a2, a3;
      q8_pairs(line.x, a0, a1);
      q8_pairs(line.y, a2, a3);
      mma16816_z(c, a0, a1, a2, a3, bp[2 * q][0], bp[2 * q][1]);
      q8_pairs(line.z, a0, a1);
      q8_pairs(line.w, a2, a3);
      mma16816(c, a0, a1, a2, a3, bp[2 * q + 1][0], bp[2 * q + 1][1]);
      const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc));
      acc[0] = fmaf(d.x, c[0] + c[1], acc[0]);
      acc[1] = fmaf(d.y, c[2] + c[3], acc[1]);
    }
  } else if constexpr (QT == J4B_Q4_0) {
    const uint4 l0 = *reinterpret_cast<const uint4*>(sq + warp * 1024 + lane * 16);
    const uint4 l1 = *reinterpret_cast<const uint4*>(sq + warp * 1024 + 512 + lane * 16);
    const uint32_t wv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint32_t sc = *reinterpret_cast<const uint32_t*>(sm + (warp * 4 + q) * 32 + g * 4);
      float c[4];
      uint32_t av[4];
      q4_pairs(wv[2 * q], av);
      mma16816_z(c, av[0], av[1], av[2], av[3], bp[2 * q][0], bp[2 * q][1]);
      q4_pairs(wv[2 * q + 1], av);
      mma16816(c, av[0], av[1], av[2], av[3], bp[2 * q + 1][0], bp[2 * q + 1][1]);
      const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc));
      acc[0] += d.x * fmaf(16.f, c[0] + c[1], -24.f * xblk[q]);
      acc[1] += d.y * fmaf(16.f, c[2] + c[3], -24.f * xblk[q]);
    }
  } else if constexpr (QT == J4B_Q2_0) {
    const uint4 line = *reinterpret_cast<const uint4*>(sq + warp * 512 + lane * 16);
    const uint32_t sc = *reinterpret_cast<const uint32_t*>(sm + warp * 32 + g * 4);
    const uint32_t wv[4] = {line.x, line.y, line.z, line.w};
    float c[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
#pragma unroll
      for (int ks = 0; ks < 2; ks++) {
        const uint32_t a0 = q2_pair(wv[q], 4 * ks), a1 = q2_pair(wv[q], 4 * ks + 1);
        const uint32_t a2 = q2_pair(wv[q], 4 * ks + 2), a3 = q2_pair(wv[q], 4 * ks + 3);
        const int j = 2 * q + ks;
        if (j == 0) mma16816_z(c, a0, a1, a2, a3, bp[j][0], bp[j][1]);
        else mma16816(c, a0, a1, a2, a3, bp[j][0], bp[j][1]);
      }
    }
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc));
    acc[0] += d.x * fmaf(4.f, c[0] + c[1], -5.f * xblk[0]);
    acc[1] += d.y * fmaf(4.f, c[2] + c[3], -5.f * xblk[0]);
  } else if constexpr (QT == J4B_Q6_K) {  // as in tile_compute
    const int h = warp & 1;
    const uint8_t* lp = sq + warp * 1536 + lane * 48;
    const uint4 n0 = *reinterpret_cast<const uint4*>(lp);
    const uint4 n1 = *reinterpret_cast<const uint4*>(lp + 16);
    const uint4 cr = *reinterpret_cast<const uint4*>(lp + 32);
    const uint8_t* mp = sm + (warp >> 1) * 288;
    const uint2 s0 = *reinterpret_cast<const uint2*>(mp + (2 * g) * 16 + 8 * h);
    const uint2 s1 = *reinterpret_cast<const uint2*>(mp + (2 * g + 1) * 16 + 8 * h);
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(mp + 256 + 4 * g));
    const uint32_t wv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
    const uint32_t cv[4] = {cr.x, cr.y, cr.z, cr.w};
#pragma unroll
    for (int j = 0; j < 8; j++) {
      uint32_t a[4];
      q6_pairs(wv[j], cv[j >> 1], j & 1, a);
      float c[4];
      mma16816_z(c, a[0], a[1], a[2], a[3], bp[j][0], bp[j][1]);
      acc[0] = fmaf(d.x * q6_scale(s0, j), c[0] + c[1], acc[0]);
      acc[1] = fmaf(d.y * q6_scale(s1, j), c[2] + c[3], acc[1]);
    }
  } else {  // Q4_K, as in tile_compute
    const int h = warp & 1;
    const uint4 l0 = *reinterpret_cast<const uint4*>(sq + warp * 1024 + lane * 32);
    const uint4 l1 = *reinterpret_cast<const uint4*>(sq + warp * 1024 + lane * 32 + 16);
    const uint8_t* mp = sm + (warp >> 1) * 256 + g * 32;
    const uint4 mm[2] = {*reinterpret_cast<const uint4*>(mp), *reinterpret_cast<const uint4*>(mp + 16)};
    float cs[2], cx[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const uint32_t w0 = mm[r].x, w1 = mm[r].y, w2 = mm[r].z, w3 = mm[r].w;
      const float d = __half2float(__ushort_as_half((uint16_t)(w0 & 0xFFFF)));
      const float dmin = __half2float(__ushort_as_half((uint16_t)(w0 >> 16)));
      const int j = 4 * h + t;
      int sc, mn;
      if (j < 4) {
        sc = (w1 >> (8 * j)) & 63;
        mn = (w2 >> (8 * j)) & 63;
      } else {
        const int jj = j - 4;
        const uint32_t qj4 = (w3 >> (8 * jj)) & 0xFF;
        sc = (qj4 & 0xF) | (((w1 >> (8 * jj + 6)) & 3) << 4);
        mn = (qj4 >> 4) | (((w2 >> (8 * jj + 6)) & 3) << 4);
      }
      const float ds = d * (float)sc;
      cs[r] = 16.f * ds;
      cx[r] = -fmaf(16.f, ds, dmin * (float)mn);
    }
    const uint32_t wv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      float c[4];
      uint32_t av[4];
      q4_pairs(wv[2 * q], av);
      mma16816_z(c, av[0], av[1], av[2], av[3], bp[2 * q][0], bp[2 * q][1]);
      q4_pairs(wv[2 * q + 1], av);
      mma16816(c, av[0], av[1], av[2], av[3], bp[2 * q + 1][0], bp[2 * q + 1][1]);
      const int src = (lane & ~3) | q;
      const float s0 = __shfl_sync(0xffffffffu, cs[0], src);
      const float s1 = __shfl_sync(0xffffffffu, cs[1], src);
      const float z0 = __shfl_sync(0xffffffffu, cx[0], src);
      const float z1 = __shfl_sync(0xffffffffu, cx[1], src);
      acc[0] += fmaf(s0, c[0] + c[1], z0 * xblk[q]);
      acc[1] += fmaf(s1, c[2] + c[3], z1 * xblk[q]);
    }
  }
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Full cluster barrier with release/acquire ordering of shared::cluster accesses.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store to the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ void st_cluster_f32(const void* local, uint32_t rank, float v) {
  uint32_t raddr;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(raddr) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(raddr), "f"(v) : "memory");
}

// Output element v (0 .. NT*128) of a tile's 16 x (8 NT) block -> (row in tile, batch column).
__device__ __forceinline__ void out_coord(int v, int& row, int& bcol) {
  const int nc = v >> 5, ln = v & 31, n = nc >> 2, c = nc & 3;
  row = (ln >> 2) + 8 * (c >> 1);
  bcol = 8 * n + 2 * (ln & 3) + (c & 1);
}

// Output element v (0 .. 64) of a tile in the packed (batch <= 4) layout.
__device__ __forceinline__ void out_coord_pk(int v, int& row, int& bcol) {
  row = ((v & 31) >> 2) + 8 * (v >> 5);
  bcol = v & 3;
}

// Inverse maps: the element index v of (row in tile, batch column). The epilogues walk outputs
// row-fastest with them, so a warp's stores to y are 128 contiguous bytes (over NVLink too).
__device__ __forceinline__ int out_index(int row, int bcol) {
  const int n = bcol >> 3, t = (bcol & 7) >> 1, c = 2 * (row >> 3) + (bcol & 1);
  return 32 * (4 * n + c) + 4 * (row & 7) + t;
}
__device__ __forceinline__ int out_index_pk(int row, int bcol) { return 32 * (row >> 3) + 4 * (row & 7) + bcol; }

template <int QT, int NT, bool PK>
__global__ void __launch_bounds__(kGemvThreads, 1) qgemv_kernel(GemvArgs a) {
  using T = GemvTraits<QT>;
  constexpr int kStages = T::kStages, kM = kTilesPerCopy<QT, NT>;
  constexpr int kStageBytes = kM * T::kChunk;
  constexpr int kVals = PK ? 64 : NT * 128;  // outputs of one tile
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stage_base = smem;
  float* red = reinterpret_cast<float*>(smem + kStages * kStageBytes);  // [kM][8 chunks][kVals]
  float* xstage = red + kM * 8 * kVals;                                  // [8 NT][kXStride]
  uint64_t* full = reinterpret_cast<uint64_t*>(xstage + 8 * NT * kXStride);
  float* mine = reinterpret_cast<float*>(smem + gemv_smem_base<QT, NT>());  // cluster mode only
  __shared__ int last_flag;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  GatherSlot gslot;  // where outputs go when all-gathered; read after the dependency wait
  // 16 warps: warp w works on the 128-column chunk w % 8 of the CTA's K range, for the tiles of
  // each stage whose index has the parity w / 8.
  const int chunk = warp & 7, sub = warp >> 3;
  const int g = lane >> 2, t = lane & 3;
  const int split = blockIdx.x % a.ksplit;
  const int group = blockIdx.x / a.ksplit;
  const int64_t tile0 = (int64_t)group * a.tiles_per_cta;
  const int64_t tile1 = min(tile0 + a.tiles_per_cta, a.rt);
  const int ntiles = (int)(tile1 - tile0);
  const int ncopies = (ntiles + kM - 1) / kM;
  const int64_t kc0 = (int64_t)split * 1024;
  const int64_t k0 = kc0 + chunk * 128;  // this warp's 128-column chunk
  const bool active = k0 < a.kpad;
  const int groups_here = a.L.groups_in_split(split);
  const uint32_t chunk_bytes = (uint32_t)a.L.chunk_bytes(split);  // one tile of this split
  const uint32_t meta_off = (uint32_t)(groups_here * T::kQ);

  // copy c brings tiles [c*kM, min((c+1)*kM, ntiles)) into stage c % kStages
  auto issue = [&](int c) {
    const int first = c * kM, count = min(kM, ntiles - first);
    const uint32_t bytes = (uint32_t)count * chunk_bytes;
    uint64_t* bar = &full[c % kStages];
    mbar_expect_tx(bar, bytes);
    tma_load_1d_stream(stage_base + (c % kStages) * kStageBytes,
                       a.data + a.L.chunk_offset(split, tile0 + first), bytes, bar, l2_evict_first_policy());
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Weights are immutable once uploaded, so they stream in before this kernel waits on the one
  // before it in the stream; x, add, y and the split-K scratch are touched only after the wait.
  int issued = 0;  // copies thread 0 has issued (only thread 0 tracks it)
  if (threadIdx.x == 0)
    for (; issued < kStages && issued < ncopies; issued++) issue(issued);
  pdl_launch_dependents();
  pdl_wait();
  gslot = gather_slot(a);

  // ---- x: the CTA's 1024-column slice of every batch row, staged once in shared memory with
  // coalesced 128-bit loads (columns past K and rows past the batch are zeros) ----
  {
    constexpr int kPer = 8 * NT * 256 / kGemvThreads;  // float4s per thread
    float4 v[kPer];
#pragma unroll
    for (int u = 0; u < kPer; u++) {  // all loads first: one round trip, not kPer
      const int idx = threadIdx.x + u * kGemvThreads, b = idx >> 8, c4 = idx & 255;
      const int64_t k = kc0 + 4 * c4;
      const bool ok = b < a.batch && k < a.cols;
      v[u] = __ldg(reinterpret_cast<const float4*>(a.x + (ok ? (int64_t)b * a.cols + k : 0)));
      if (!ok) v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kPer; u++) {
      const int idx = threadIdx.x + u * kGemvThreads, b = idx >> 8, c4 = idx & 255;
      *reinterpret_cast<float4*>(xstage + b * kXStride + 4 * c4) = v[u];
    }
  }
  __syncthreads();
  // ---- x fragments of this warp's 128-column chunk: hi/lo fp16, per n-tile and k-step ----
  // (packed: lane group g holds batch g / 2, its hi part for even g and lo part for odd g)
  constexpr int NTF = PK ? 1 : NT;
  uint32_t bh[NTF][8][2], bl[PK ? 1 : NT][8][2];
  float xs[NTF][8];
#pragma unroll
  for (int n = 0; n < NTF; n++) {
    const int xrow = PK ? (g >> 1) : 8 * n + g;
    const float* xr = xstage + xrow * kXStride + chunk * 128 + 2 * t;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float2 p0 = *reinterpret_cast<const float2*>(xr + 16 * j);
      const float2 p1 = *reinterpret_cast<const float2*>(xr + 16 * j + 8);
      const float v[4] = {p0.x, p0.y, p1.x, p1.y};
      __half2 h0 = __floats2half2_rn(v[0], v[1]);
      __half2 h1 = __floats2half2_rn(v[2], v[3]);
      const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
      __half2 l0 = __floats2half2_rn(v[0] - f0.x, v[1] - f0.y);
      __half2 l1 = __floats2half2_rn(v[2] - f1.x, v[3] - f1.y);
      const float2 g0 = __half22float2(l0), g1 = __half22float2(l1);
      if constexpr (PK) {
        const bool lo = g & 1;
        bh[n][j][0] = lo ? *reinterpret_cast<uint32_t*>(&l0) : *reinterpret_cast<uint32_t*>(&h0);
        bh[n][j][1] = lo ? *reinterpret_cast<uint32_t*>(&l1) : *reinterpret_cast<uint32_t*>(&h1);
        xs[n][j] = lo ? (g0.x + g0.y) + (g1.x + g1.y) : (f0.x + f0.y) + (f1.x + f1.y);
      } else {
        bh[n][j][0] = *reinterpret_cast<uint32_t*>(&h0);
        bh[n][j][1] = *reinterpret_cast<uint32_t*>(&h1);
        bl[n][j][0] = *reinterpret_cast<uint32_t*>(&l0);
        bl[n][j][1] = *reinterpret_cast<uint32_t*>(&l1);
        xs[n][j] = (f0.x + g0.x) + (f0.y + g0.y) + (f1.x + g1.x) + (f1.y + g1.y);
      }
    }
  }
  // Block sums of x for the output columns this lane holds (batch 2t, 2t+1 of each n-tile;
  // packed: batch t, the sum of its hi and lo column sums).
  constexpr int kXB = kXBlocks<QT>;
  float xblk[NT][kXB][2] = {};
  float xblkp[kXB] = {};
  if constexpr (QT != J4B_Q8_0 && QT != J4B_Q6_K) {
#pragma unroll
    for (int n = 0; n < NTF; n++) {
#pragma unroll
      for (int q = 0; q < kXB; q++) {
        float s = 0.f;
        constexpr int kSteps = 8 / kXB;
#pragma unroll
        for (int j = 0; j < kSteps; j++) s += xs[n][q * kSteps + j];
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        const float s0 = __shfl_sync(0xffffffffu, s, 4 * (2 * t));
        const float s1 = __shfl_sync(0xffffffffu, s, 4 * (2 * t + 1));
        if constexpr (PK) {
          xblkp[q] = s0 + s1;
        } else {
          xblk[n][q][0] = s0;
          xblk[n][q][1] = s1;
        }
      }
    }
  }

  bool failed = false;
  int consumed = 0;  // copies fully consumed
  for (int c = 0; c < ncopies; c++) {
    const int s = c % kStages;
    const int count = min(kM, ntiles - c * kM);
    if (!mbar_wait_bounded(&full[s], (uint32_t)((c / kStages) & 1))) failed = true;
    constexpr int kMine = kM / 2;  // tiles of the stage this warp computes: sub, sub + 2, ...
    if constexpr (PK) {
      float acc[kMine][2] = {};
      if (active && !failed) {
        const uint8_t* st = stage_base + s * kStageBytes;
#pragma unroll
        for (int jj = 0; jj < kMine; jj++) {
          const int j = sub + 2 * jj;
          tile_compute_pk<QT>(st + j * chunk_bytes, st + j * chunk_bytes + meta_off, chunk, lane, bh[0], xblkp, acc[jj]);
        }
      }
#pragma unroll
      for (int jj = 0; jj < kMine; jj++)
#pragma unroll
        for (int cc = 0; cc < 2; cc++) red[((sub + 2 * jj) * 8 + chunk) * kVals + cc * 32 + lane] = acc[jj][cc];
    } else {
      float acc[kMine][NT][4] = {};
      if (active && !failed) {
        const uint8_t* st = stage_base + s * kStageBytes;
        // tiles past `count` read stale stage bytes and are discarded
#pragma unroll
        for (int jj = 0; jj < kMine; jj++) {
          const int j = sub + 2 * jj;
          tile_compute<QT, NT>(st + j * chunk_bytes, st + j * chunk_bytes + meta_off, chunk, lane, bh, bl, xblk, acc[jj]);
        }
      }
#pragma unroll
      for (int jj = 0; jj < kMine; jj++)
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
          for (int cc = 0; cc < 4; cc++)
            red[((sub + 2 * jj) * 8 + chunk) * kVals + (n * 4 + cc) * 32 + lane] = acc[jj][n][cc];
    }
    if (__syncthreads_or(failed)) {
      failed = true;
      break;
    }
    consumed = c + 1;
    if (threadIdx.x == 0 && c + kStages < ncopies) {
      fence_proxy_async();  // generic-proxy reads of stage s happen before the async refill
      issue(c + kStages);
      issued++;
    }
    for (int idx = threadIdx.x; idx < count * kVals; idx += kGemvThreads) {
      const int j = idx / kVals, v = idx % kVals;
      float total = 0.f;
#pragma unroll
      for (int w = 0; w < 8; w++) total += red[(j * 8 + w) * kVals + v];
      const int64_t tile = tile0 + c * kM + j;
      if (a.ksplit == 1) {
        int row, bcol;
        if (PK) out_coord_pk(v, row, bcol); else out_coord(v, row, bcol);
        const int64_t r = tile * 16 + row;
        if (r < a.rows && bcol < a.batch) {
          if (a.add) total += a.add[(int64_t)bcol * a.rows + r];
          store_y(a, gslot, bcol, r, total);
        }
      } else if (a.cluster) {
        mine[(c * kM + j) * kVals + v] = total;
      } else {
        a.partials[((int64_t)split * a.rt + tile) * 256 + v] = total;
      }
    }
    __syncthreads();  // red is rewritten by the next stage
  }

  if (failed) {
    // Let copies still in flight land before the CTA's shared memory is reused or released.
    if (threadIdx.x == 0) {
      atomicExch(a.status, 1);
      for (int cc = consumed; cc < issued; cc++)  // bounded wait for each copy still in flight
        mbar_wait_bounded(&full[cc % kStages], (uint32_t)((cc / kStages) & 1));
    }
    __syncthreads();
    if (!a.cluster) return;  // cluster members still take both cluster barriers below
  }

  if (a.cluster) {
    // Split-K fold inside the cluster: every CTA is past its main loop (barrier 1), CTAs 1.. push
    // their per-tile totals into CTA 0's shared memory from offset 0, where its stages were
    // (barrier 2), and CTA 0 adds them in split order, so the result is deterministic.
    const uint32_t rank = cluster_ctarank();
    const int nv = ntiles * kVals;
    float* landing = reinterpret_cast<float*>(smem);  // [ksplit - 1][nv] in CTA 0
    cluster_sync();
    if (rank != 0)
      for (int i = threadIdx.x; i < nv; i += kGemvThreads)
        st_cluster_f32(landing + (rank - 1) * nv + i, 0, mine[i]);
    cluster_sync();
    if (rank == 0 && !failed) {
      const int nr = ntiles * 16;  // rows of this tile group, walked fastest
      for (int j = threadIdx.x; j < a.batch * nr; j += kGemvThreads) {
        const int bcol = j / nr, rr = j % nr;
        const int i = (rr >> 4) * kVals + (PK ? out_index_pk(rr & 15, bcol) : out_index(rr & 15, bcol));
        float total = mine[i];
        for (int sp = 1; sp < a.ksplit; sp++) total += landing[(sp - 1) * nv + i];
        const int64_t r = tile0 * 16 + rr;
        if (r < a.rows) {
          if (a.add) total += a.add[(int64_t)bcol * a.rows + r];
          store_y(a, gslot, bcol, r, total);
        }
      }
    }
    return;
  }

  if (a.ksplit > 1) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_flag = atomicAdd(a.arrivals + group, 1u) == (unsigned)(a.ksplit - 1);
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    // The last CTA of the group folds the K splits in split order (deterministic), walking the
    // outputs row-fastest; four outputs per thread per pass keep their loads in flight together.
    const int nr = ntiles * 16;
    const int nout = a.batch * nr;
    for (int j0 = threadIdx.x; j0 < nout; j0 += 4 * kGemvThreads) {
      float tot[4] = {0.f, 0.f, 0.f, 0.f};
      int64_t off[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int j = min(j0 + u * kGemvThreads, nout - 1);
        const int bcol = j / nr, rr = j % nr;
        off[u] = (tile0 + (rr >> 4)) * 256 + (PK ? out_index_pk(rr & 15, bcol) : out_index(rr & 15, bcol));
      }
      for (int sp = 0; sp < a.ksplit; sp++) {
#pragma unroll
        for (int u = 0; u < 4; u++) tot[u] += __ldcg(a.partials + (int64_t)sp * a.rt * 256 + off[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int j = j0 + u * kGemvThreads;
        if (j >= nout) break;
        const int bcol = j / nr, rr = j % nr;
        const int64_t r = tile0 * 16 + rr;
        if (r < a.rows) {
          float v = tot[u];
          if (a.add) v += a.add[(int64_t)bcol * a.rows + r];
          store_y(a, gslot, bcol, r, v);
        }
      }
    }
    if (threadIdx.x == 0) a.arrivals[group] = 0u;
  }
}

template <int QT, int NT, bool PK>
cudaError_t launch_gemv(const j4b_qweight* w, const float* x, const float* add, float* y,
                        int batch, int sms, cudaStream_t stream, const GemvPeers* peers,
                        unsigned* grid_out, bool pdl) {
  // Largest dynamic shared memory a CTA may request: the device's opt-in limit minus the
  // kernel's static shared memory (set once per instantiation).
  static int64_t kMaxSmem = -1;
  constexpr int base = gemv_smem_base<QT, NT>();
  constexpr int kVals = PK ? 64 : NT * 128;
  if (kMaxSmem < 0) {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, qgemv_kernel<QT, NT, PK>);
    if (e != cudaSuccess) return e;
    const int64_t lim = (int64_t)optin - (int64_t)fa.sharedSizeBytes;
    if (lim < base) return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(qgemv_kernel<QT, NT, PK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lim);
    if (e != cudaSuccess) return e;
    kMaxSmem = lim;
  }
  GemvArgs a;
  a.data = w->data;
  a.L = layout_of(w);
  a.rows = w->rows;
  a.cols = w->cols;
  a.kpad = w->kpad;
  a.rt = w->rt;
  a.x = x;
  a.add = add;
  a.y = y;
  a.batch = batch;
  a.ksplit = w->ksplit;
  a.partials = w->partials;
  a.arrivals = w->arrivals;
  a.status = w->status;
  a.nranks = 1;
  a.rank = 0;
  a.step = nullptr;
  a.half_words = 0;
  for (int p = 0; p < kMaxPeerRanks; ++p) a.peer_y[p] = nullptr;
  if (peers) {
    a.nranks = peers->nranks;
    a.rank = peers->rank;
    a.step = peers->step;
    a.half_words = peers->half_words;
    for (int p = 0; p < peers->nranks; ++p) a.peer_y[p] = peers->y[p];
  }
  // One 16-warp CTA per SM: as many tile groups as fit next to the K splits, tiles shared out
  // evenly.
  int64_t groups_fit = std::max<int64_t>(1, (int64_t)sms / w->ksplit);
  int64_t tiles = (w->rt + groups_fit - 1) / groups_fit;
  int64_t groups = (w->rt + tiles - 1) / tiles;
  // Cluster split-K fold when the splits fit one portable cluster, the per-tile totals fit next
  // to the base layout, the landing area fits below them, and every cluster is co-resident.
  int64_t smem = base;
  a.cluster = 0;
  if (w->ksplit >= 2 && w->ksplit <= 8) {
    const int64_t need = base + tiles * kVals * 4;
    const int64_t landing = (w->ksplit - 1) * tiles * kVals * 4;
    if (need <= kMaxSmem && landing <= base) {
      cudaLaunchConfig_t occ = {};
      occ.gridDim = dim3((unsigned)(groups * w->ksplit));
      occ.blockDim = dim3(kGemvThreads);
      occ.dynamicSmemBytes = (size_t)need;
      cudaLaunchAttribute ca[1];
      ca[0].id = cudaLaunchAttributeClusterDimension;
      ca[0].val.clusterDim.x = (unsigned)w->ksplit;
      ca[0].val.clusterDim.y = 1;
      ca[0].val.clusterDim.z = 1;
      occ.attrs = ca;
      occ.numAttrs = 1;
      int max_clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&max_clusters, qgemv_kernel<QT, NT, PK>, &occ) == cudaSuccess &&
          max_clusters >= 1) {
        if (groups > max_clusters) {  // keep one wave
          tiles = (w->rt + max_clusters - 1) / max_clusters;
          groups = (w->rt + tiles - 1) / tiles;
        }
        const int64_t need2 = base + tiles * kVals * 4;
        if (need2 <= kMaxSmem && (w->ksplit - 1) * tiles * kVals * 4 <= base) {
          a.cluster = 1;
          smem = need2;
        }
      } else {
        cudaGetLastError();
      }
    }
  }
  a.tiles_per_cta = (int)tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(groups * w->ksplit));
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a.cluster ? (unsigned)w->ksplit : 1u;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.cluster ? 2 : 1;
  if (grid_out) *grid_out = cfg.gridDim.x;
  return cudaLaunchKernelEx(&cfg, qgemv_kernel<QT, NT, PK>, a);
}

#include "qgemv_stream.cuh"

template <int QT>
cudaError_t gemv_dispatch(const j4b_qweight* w, const float* x, const float* add, float* y,
                          int batch, int sms, cudaStream_t stream, const GemvPeers* peers = nullptr,
                          unsigned* grid_out = nullptr) {
  const bool pdl = !w->fresh;
  const_cast<j4b_qweight*>(w)->fresh = false;
  if (batch <= 4) return launch_gemv_stream<QT, true, 15>(w, x, add, y, batch, sms, stream, peers, grid_out, pdl);
  if (batch <= 8) return launch_gemv_stream<QT, false, 15>(w, x, add, y, batch, sms, stream, peers, grid_out, pdl);
  return launch_gemv_stream<QT, false, 15, 2>(w, x, add, y, batch, sms, stream, peers, grid_out, pdl);
}
