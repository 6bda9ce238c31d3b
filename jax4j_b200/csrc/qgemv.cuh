// Shared pieces of the batched dequant-GEMV (included by quant.cu inside namespace
// j4b::<anonymous>): bulk-copy and mbarrier helpers, the exact fp16 decoders of the quant codes,
// the per-warp tile decoders tile_compute / tile_compute_pk (one warp's 16-row x 128-column chunk
// of a tile times the x fragments, block scales folded in fp32), the launch arguments and the
// output store (local, or into every rank's gathered buffer over peer memory). The kernel itself,
// a producer-warp bulk-copy ring feeding compute warps that own whole tiles, is
// qgemv_stream.cuh.

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

// Bytes of one tile's quant and scale bytes in one 1024-column split (16 rows).
template <int QT>
struct GemvTraits {
  static constexpr int kQ = QT == J4B_Q8_0 ? 512 : (QT == J4B_Q2_0 ? 128 : (QT == J4B_Q6_K ? 384 : 256));
  static constexpr int kM = QT == J4B_Q2_0 ? 8 : (QT == J4B_Q6_K ? 36 : 32);
  static constexpr int kChunk = 32 * (kQ + kM);  // bytes of one full tile chunk
};

struct GemvArgs {
  const uint8_t* data;
  Layout L;
  int64_t rows, cols, kpad, rt;
  const float* x;
  const float* add;
  float* y;
  int batch;  // batch rows handled by this launch (<= 8 * NT)
  int ksplit;
  float* partials;     // [ksplit][rt][256] split-K partials
  unsigned* arrivals;  // one counter per tile group
  int* status;         // nonzero after a bounded wait gave up
  // All-gather over peer memory (nranks > 1): this rank's rows of y go straight into every
  // rank's gathered buffer, [batch][rows * nranks] flagged words in the parity half selected by
  // the local step counter (see gather_store).
  int nranks, rank;
  unsigned long long* peer_y[kMaxPeerRanks];
  unsigned* step;       // the channel's step counter, advanced by the launch's last warp
  unsigned* done;       // finished-warp counter of the channel
  int64_t half_words;
  float* gout;          // the gathered output the warps copy into, [batch][rows * nranks]
  int64_t gathered;     // its floats
  int* pstatus;         // the peer group's status word
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
