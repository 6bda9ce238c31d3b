// Prefill projection y [m, rows] = x [m, cols] . W^T with W's block dequantisation fused into the
// tcgen05 pipeline (included by quant.cu inside namespace j4b::<anonymous>, after Layout).
//
// The quantised weight never exists as a bf16 matrix in HBM: decode warps turn its repacked
// fragment-layout bytes (plus the per-row block scales) into the 128-byte-swizzled bf16 operand
// tile in shared memory, k-block by k-block, right before the tensor cores read it. W is the
// MMA's M = 128 operand and the activations its N operand: for long inputs a CTA holds two
// accumulators of 256 tokens (the whole TMEM), so every decoded weight element feeds 2 x 512
// FLOPs; the tile's accumulator D[w row][token] lives in TMEM and the epilogue writes it
// transposed, y[token][w row], with warp-coalesced stores.
//
// Warps of one CTA (one 128 x BN output tile):
//   warp 0     one thread streams the x tile's 64-wide K slices with 2-D TMA loads;
//   warp 1     allocates the TMEM accumulator; one thread issues tcgen05.mma per 16-wide K step and
//              releases each stage with tcgen05.commit;
//   warps 2-5  epilogue: tcgen05.ld of TMEM lanes 32 (w % 4) .. + 31 (= W rows), 8 tokens at a
//              time, stores to y;
//   warps 6..  decoders (4 when two CTAs share an SM, else 8): each decodes one or two 16-row tiles of every k-block,
//              loading the next k-block's bytes before writing the current one; each writes its
//              part of the stage, fences the generic-proxy writes for the async proxy the tensor
//              core reads through, and arrives on the stage's `full_a` barrier.
// Values are those of the bit-exact gather (d * code in float; the Q4_K d*sc*q - dmin*m with one
// rounding instead of two), rounded to bf16 (mode 1) or split into bf16 hi + lo (fp32-accurate mode: the product is
// hi.hi + hi.lo + lo.hi, with x split the same way). Every mbarrier wait is bounded; a wait that
// gives up records an error in the weight's status word.

constexpr int kQgBM = 128, kQgBK = 64;
// decode warps: 4 (two 16-row tiles each) when two CTAs share an SM, 8 (one tile each) when a CTA
// holds the SM alone, so an SM always runs eight decoders
template <int TERMS, int N, int NH>
constexpr int qg_decode_warps();
template <int TERMS, int N, int NH>
constexpr int qg_threads() { return (6 + qg_decode_warps<TERMS, N, NH>()) * 32; }

// N tokens per MMA, NH accumulators of N columns each per CTA (NH = 2, N = 256: 512 tokens in bf16
// mode, the whole TMEM, one CTA per SM; N = 64: decode-time batches).
// Two rings of the same depth: A (the decoded weight tile, written by the decoders) and B (the
// activation tiles, TMA). Measured on the 16384 x 14336 x 4096 bf16 prefill projection (2 x 256
// tokens, two 64 KB B stages: 2.12 ms, tensor pipe 44% busy, shared-memory pipes ~32% busy):
// a third B stage (224 KB, no room left for the decoders' prefetch ring) 2.22 ms; 2 x 192 tokens
// with three 48 KB B stages 2.39 ms.
template <int TERMS, int N, int NH>
constexpr int qg_stages() { return (TERMS == 1 && N * NH <= 256) ? 2 : (TERMS == 3 && N * NH <= 128 ? 3 : 2); }
template <int TERMS, int N, int NH>
constexpr int qg_stages_a() { return qg_stages<TERMS, N, NH>(); }
template <int TERMS, int N, int NH>
constexpr int qg_stages_b() { return qg_stages<TERMS, N, NH>(); }
// TMEM columns allocated for NH accumulators of N columns (a power of two, at least 32)
template <int N, int NH>
constexpr uint32_t qg_tmem_cols() {
  return N * NH <= 32 ? 32u : N * NH <= 64 ? 64u : N * NH <= 128 ? 128u : N * NH <= 256 ? 256u : 512u;
}
constexpr uint32_t kQgABytes = kQgBM * kQgBK * 2;  // one 128 x 64 bf16 tile
template <int N, int NH>
constexpr uint32_t qg_b_bytes() { return (uint32_t)(NH * N) * kQgBK * 2; }
// A stage: A hi (| A lo); B stage: B hi (| B lo), a B part holding the NH token boxes in a row
template <int TERMS>
constexpr uint32_t qg_a_stage_bytes() { return (TERMS == 3 ? 2u : 1u) * kQgABytes; }
template <int TERMS, int N, int NH>
constexpr uint32_t qg_b_stage_bytes() { return (TERMS == 3 ? 2u : 1u) * qg_b_bytes<N, NH>(); }
template <int TERMS, int N, int NH>
constexpr uint32_t qg_ring_bytes() {
  return qg_stages_a<TERMS, N, NH>() * qg_a_stage_bytes<TERMS>() +
         qg_stages_b<TERMS, N, NH>() * qg_b_stage_bytes<TERMS, N, NH>();
}
template <int TERMS, int N, int NH>
constexpr int qg_min_blocks() { return (TERMS == 1 && N * NH <= 256) ? 2 : 1; }
template <int TERMS, int N, int NH>
constexpr int qg_decode_warps() { return qg_min_blocks<TERMS, N, NH>() == 2 ? 4 : 8; }

// Decoder prefetch. A decoder's loads of its tiles' code and scale bytes come from L2/HBM and take
// longer than one k-block of MMAs, so with one CTA per SM they go through a per-lane shared-memory
// ring filled by cp.async, kQgPre k-blocks deep (48 bytes per lane, tile and k-block); a
// configuration whose rings leave no room (two CTAs per SM) keeps one k-block of prefetch in
// registers (depth 0 here).
constexpr uint32_t kQgSlot = 48;  // bytes per lane per tile per k-block
template <int TERMS, int N, int NH>
constexpr uint32_t qg_pre_bytes(int depth) {
  return (uint32_t)depth * 8u * 32u * kQgSlot;  // 8 row tiles per CTA, whatever the decoder split
}
template <int TERMS, int N, int NH>
constexpr int qg_pre_depth() {
  constexpr uint32_t kMax = 232448 - 1024 - 256;  // opt-in shared memory per block, minus slack
  if (qg_min_blocks<TERMS, N, NH>() != 1) return 0;
  return qg_ring_bytes<TERMS, N, NH>() + qg_pre_bytes<TERMS, N, NH>(4) <= kMax   ? 4
         : qg_ring_bytes<TERMS, N, NH>() + qg_pre_bytes<TERMS, N, NH>(3) <= kMax ? 3
         : qg_ring_bytes<TERMS, N, NH>() + qg_pre_bytes<TERMS, N, NH>(2) <= kMax ? 2
                                                                                 : 0;
}

struct QgArgs {
  const uint8_t* data;
  Layout L;
  int64_t rows, cols;
  int m, kp;
  int splits, kb_per;  // K splits and 64-column k-blocks per split
  float* y;            // [m, rows]; with splits > 1 the partials [splits][m][rows]
  const float* add;    // added to y (splits == 1 only; else the fold adds it)
  int* status;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

// One lane's bytes of one 16-row tile for one 64-column k-block (two 32-column groups).
struct QgBytes {
  uint4 q0, q1;  // quants: Q8_0 one line per group; 4-bit formats q0 only (words: g0 ks0, g0 ks1, g1 ks0, g1 ks1)
  uint4 s0, s1;  // scales: Q8_0/Q4_0 s0.x / s0.y = (d row g | d row g+8) of the two groups; Q4_K the
                 // 16 GGUF header bytes of rows g (s0) and g + 8 (s1)
};

template <int QT>
__device__ __forceinline__ void qg_load(const QgArgs& a, int64_t tile, int kb, int lane, QgBytes& b) {
  const int g = lane >> 2;
  const int64_t G = 2 * (int64_t)kb;
  const int64_t s = G / 32;
  const int gl = (int)(G % 32);
  if (tile >= a.L.rt) {
    b.q0 = b.q1 = b.s0 = b.s1 = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint8_t* base = a.data + a.L.chunk_offset(s, tile);
  const int64_t meta = (int64_t)a.L.groups_in_split(s) * GemvTraits<QT>::kQ;
  if constexpr (QT == J4B_Q8_0) {
    b.q0 = __ldg(reinterpret_cast<const uint4*>(base + gl * 512 + lane * 16));
    b.q1 = __ldg(reinterpret_cast<const uint4*>(base + (gl + 1) * 512 + lane * 16));
    b.s0.x = __ldg(reinterpret_cast<const uint32_t*>(base + meta + gl * 32 + g * 4));
    b.s0.y = __ldg(reinterpret_cast<const uint32_t*>(base + meta + (gl + 1) * 32 + g * 4));
  } else if constexpr (QT == J4B_Q4_0) {
    b.q0 = __ldg(reinterpret_cast<const uint4*>(base + (gl / 2) * 512 + lane * 16));
    b.s0.x = __ldg(reinterpret_cast<const uint32_t*>(base + meta + gl * 32 + g * 4));
    b.s0.y = __ldg(reinterpret_cast<const uint32_t*>(base + meta + (gl + 1) * 32 + g * 4));
  } else {  // Q4_K
    b.q0 = __ldg(reinterpret_cast<const uint4*>(base + (gl / 4) * 1024 + lane * 32 + (gl % 4) * 8));
    const uint8_t* mp = base + meta + (gl / 8) * 256 + (g * 2) * 16;
    b.s0 = __ldg(reinterpret_cast<const uint4*>(mp));
    b.s1 = __ldg(reinterpret_cast<const uint4*>(mp + 16));
  }
}

// The same bytes as qg_load, copied asynchronously into the lane's 48-byte slot at shared address
// `slot`: [0, 16) the first code line, [16, 32) the second (Q8_0) or the rows' Q4_K headers of
// row g, [32, 48) Q4_K row g + 8's headers, or the two group scale words (Q8_0, Q4_0). A tile past
// the matrix gets zeros (plain stores, read back by the same lane).
template <int QT>
__device__ __forceinline__ void qg_copy(const QgArgs& a, int64_t tile, int kb, int lane, uint8_t* slot_ptr) {
  const int g = lane >> 2;
  const int64_t G = 2 * (int64_t)kb;
  const int64_t s = G / 32;
  const int gl = (int)(G % 32);
  if (tile >= a.L.rt) {
    uint4* z = reinterpret_cast<uint4*>(slot_ptr);
    z[0] = z[1] = z[2] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint32_t slot = (uint32_t)__cvta_generic_to_shared(slot_ptr);
  const uint8_t* base = a.data + a.L.chunk_offset(s, tile);
  const int64_t meta = (int64_t)a.L.groups_in_split(s) * GemvTraits<QT>::kQ;
  if constexpr (QT == J4B_Q8_0) {
    cp_async16(slot, base + gl * 512 + lane * 16);
    cp_async16(slot + 16, base + (gl + 1) * 512 + lane * 16);
    cp_async4(slot + 32, base + meta + gl * 32 + g * 4);
    cp_async4(slot + 36, base + meta + (gl + 1) * 32 + g * 4);
  } else if constexpr (QT == J4B_Q4_0) {
    cp_async16(slot, base + (gl / 2) * 512 + lane * 16);
    cp_async4(slot + 32, base + meta + gl * 32 + g * 4);
    cp_async4(slot + 36, base + meta + (gl + 1) * 32 + g * 4);
  } else {  // Q4_K
    cp_async16(slot, base + (gl / 4) * 1024 + lane * 32 + (gl % 4) * 8);
    const uint8_t* mp = base + meta + (gl / 8) * 256 + (g * 2) * 16;
    cp_async16(slot + 16, mp);
    cp_async16(slot + 32, mp + 16);
  }
}
template <int QT>
__device__ __forceinline__ void qg_read_slot(const uint8_t* slot, QgBytes& b) {
  const uint4* v = reinterpret_cast<const uint4*>(slot);
  b.q0 = v[0];
  if constexpr (QT == J4B_Q4_K) {
    b.s0 = v[1];
    b.s1 = v[2];
  } else {
    b.q1 = v[1];
    b.s0 = v[2];
  }
}

// Q4_K: d * sc_j and dmin * m_j of sub-block j from a row's 16 header bytes (the GGUF 6-bit pairs).
__device__ __forceinline__ void q4k_row_scales(const uint4& h, int j, float& d1, float& m1) {
  const float d = __half2float(__ushort_as_half((uint16_t)(h.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
  int sc, mn;
  if (j < 4) {
    sc = (h.y >> (8 * j)) & 63;
    mn = (h.z >> (8 * j)) & 63;
  } else {
    const int jj = j - 4;
    const uint32_t qj4 = (h.w >> (8 * jj)) & 0xFF;
    sc = (qj4 & 0xF) | (((h.y >> (8 * jj + 6)) & 3) << 4);
    mn = (qj4 >> 4) | (((h.z >> (8 * jj + 6)) & 3) << 4);
  }
  d1 = __fmul_rn(d, (float)sc);
  m1 = __fmul_rn(dmin, (float)mn);
}

__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// Writes one lane's 32 decoded elements of one 16-row tile (tile rows from r0, a multiple of 16,
// in the A operand). Codes become floats without conversions: a 4-bit code masked into the
// mantissa of 2^23 (bits 6..9) is 2^23 + 64 q, so one subtraction gives 64 q exactly and one fma
// with d / 64 (exact: a power-of-two scale) gives d q - offset rounded once; a Q8_0 byte placed
// under 2^23's exponent gives 2^23 + (code + 128).
template <int QT, int TERMS>
__device__ __forceinline__ void qg_store(const QgBytes& b, int kb, int lane, uint8_t* a_hi, uint8_t* a_lo, int r0) {
  const int g = lane >> 2, t = lane & 3;
  float mul[2][2], off[2][2];  // value = fma(code_term, mul, off) per [group][row g / g + 8]
#pragma unroll
  for (int gg = 0; gg < 2; gg++) {
    if constexpr (QT == J4B_Q4_K) {
      const int j = (2 * kb) % 8 + gg;
      float d1, m1;
      q4k_row_scales(b.s0, j, d1, m1);
      mul[gg][0] = d1 * (1.f / 64.f);
      off[gg][0] = -m1;
      q4k_row_scales(b.s1, j, d1, m1);
      mul[gg][1] = d1 * (1.f / 64.f);
      off[gg][1] = -m1;
    } else {
      const uint32_t w = gg ? b.s0.y : b.s0.x;
      const float d0 = __half2float(__ushort_as_half((uint16_t)(w & 0xFFFF)));
      const float d8 = __half2float(__ushort_as_half((uint16_t)(w >> 16)));
      if constexpr (QT == J4B_Q4_0) {
        mul[gg][0] = d0 * (1.f / 64.f);
        off[gg][0] = -8.f * d0;
        mul[gg][1] = d8 * (1.f / 64.f);
        off[gg][1] = -8.f * d8;
      } else {
        mul[gg][0] = d0;
        mul[gg][1] = d8;
        off[gg][0] = off[gg][1] = 0.f;
      }
    }
  }
  const uint32_t q4[4] = {b.q0.x, b.q0.y, b.q0.z, b.q0.w};
  const uint32_t q8[2][4] = {{b.q0.x, b.q0.y, b.q0.z, b.q0.w}, {b.q1.x, b.q1.y, b.q1.z, b.q1.w}};
  const float kMagic = 8388608.f;  // 2^23
  // row r0 + g + 8 which: 1024-byte row group (r0 >> 3) + which, row g inside it; the 16-byte
  // chunk index of column col is col >> 3, XORed with the row's g (the 128-byte swizzle)
  const uint32_t row_base = (uint32_t)((r0 >> 3) * 1024 + g * 128 + 4 * t);
#pragma unroll
  for (int gg = 0; gg < 2; gg++)
#pragma unroll
    for (int ks = 0; ks < 2; ks++)
#pragma unroll
      for (int i = 0; i < 4; i++) {  // element pair (2i, 2i + 1) of the k-step's A fragment
        const int which = i & 1;
        float v0, v1;
        if constexpr (QT == J4B_Q8_0) {
          const uint32_t w = q8[gg][2 * ks + (i >> 1)];
          const int sh = 2 * (i & 1);  // byte index of the pair's first code
          const float c0 = __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7650 + sh)) - (kMagic + 128.f);
          const float c1 = __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7651 + sh)) - (kMagic + 128.f);
          v0 = c0 * mul[gg][which];
          v1 = c1 * mul[gg][which];
        } else {
          const uint32_t w = q4[2 * gg + ks];
          const float c0 = __int_as_float((int)((rotr(w, 4 * i) & 0x3C0u) | 0x4B000000u)) - kMagic;        // 64 q
          const float c1 = __int_as_float((int)((rotr(w, 4 * i + 16) & 0x3C0u) | 0x4B000000u)) - kMagic;   // 64 q
          v0 = fmaf(c0, mul[gg][which], off[gg][which]);
          v1 = fmaf(c1, mul[gg][which], off[gg][which]);
        }
        const int chunk = ((4 * gg + 2 * ks + (i >> 1)) ^ g) & 7;
        const uint32_t o = row_base + which * 1024 + (chunk << 4);
        const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
        *reinterpret_cast<uint32_t*>(a_hi + o) = bf16x2_bits(h);
        if constexpr (TERMS == 3) {
          const float2 hf = __bfloat1622float2(h);
          *reinterpret_cast<uint32_t*>(a_lo + o) = bf16x2_bits(__floats2bfloat162_rn(v0 - hf.x, v1 - hf.y));
        }
      }
}

template <int QT, int TERMS, int N, int NH>
__global__ void __launch_bounds__(qg_threads<TERMS, N, NH>(), qg_min_blocks<TERMS, N, NH>())
    qgemm_fused_kernel(const __grid_constant__ CUtensorMap x_hi, const __grid_constant__ CUtensorMap x_lo, QgArgs p) {
  constexpr int kN = N;                // tokens per MMA
  constexpr int kBN = NH * kN;         // tokens per tile (TMEM columns)
  constexpr int kSA = qg_stages_a<TERMS, N, NH>();
  constexpr int kSB = qg_stages_b<TERMS, N, NH>();
  constexpr uint32_t kAStage = qg_a_stage_bytes<TERMS>();
  constexpr uint32_t kBStage = qg_b_stage_bytes<TERMS, N, NH>();
  constexpr uint32_t kB = qg_b_bytes<N, NH>();
  constexpr uint32_t kBox = (uint32_t)kN * kQgBK * 2;  // one token box
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + qg_ring_bytes<TERMS, N, NH>());
  uint64_t* empty_a = full_a + kSA;
  uint64_t* full_b = empty_a + kSA;
  uint64_t* empty_b = full_b + kSB;
  uint64_t* acc_full = empty_b + kSB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tile order: W-row tiles fastest, then K splits, then token tiles
  const int n_tiles = (int)((p.rows + kQgBM - 1) / kQgBM);
  const int n_tile = (int)(blockIdx.x % n_tiles);
  const int split = (int)((blockIdx.x / n_tiles) % p.splits);
  const int t_tile = (int)(blockIdx.x / n_tiles / p.splits);
  const int64_t w0 = (int64_t)n_tile * kQgBM;
  const int tok0 = t_tile * kBN;
  const int kb0 = split * p.kb_per;
  const int nk = min(p.kp / kQgBK - kb0, p.kb_per);  // k-blocks of this CTA, from kb0
  float* out = p.y + (int64_t)split * p.m * p.rows;
  auto stage_a = [&](int s, int lo) { return smem + s * kAStage + (lo ? kQgABytes : 0); };
  auto stage_b = [&](int s, int lo) { return smem + kSA * kAStage + s * kBStage + (lo ? kB : 0); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSA; ++s) {
      bar_init(&full_a[s], qg_decode_warps<TERMS, N, NH>());
      bar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < kSB; ++s) {
      bar_init(&full_b[s], 1);
      bar_init(&empty_b[s], 1);
    }
    bar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                 "r"(qg_tmem_cols<N, NH>()));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {  // x tiles
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kSB, use = kb / kSB;
        if (use > 0 && !bar_wait(&empty_b[s], (uint32_t)((use - 1) & 1))) ok = false;
        bar_expect_tx(&full_b[s], kBStage);
        const int kx = (kb0 + kb) * kQgBK;
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          tma_tile(stage_b(s, 0) + h * kBox, &x_hi, kx, tok0 + h * kN, &full_b[s]);
          if (TERMS == 3) tma_tile(stage_b(s, 1) + h * kBox, &x_lo, kx, tok0 + h * kN, &full_b[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issue
      constexpr uint32_t idesc = idesc_bf16(kQgBM, kN);
      for (int kb = 0; kb < nk; ++kb) {
        const int sa = kb % kSA, sb = kb % kSB;
        if (!bar_wait(&full_a[sa], (uint32_t)((kb / kSA) & 1))) ok = false;
        if (!bar_wait(&full_b[sb], (uint32_t)((kb / kSB) & 1))) ok = false;
        tc_fence_after();
        const uint32_t ah = saddr(stage_a(sa, 0)), bh = saddr(stage_b(sb, 0));
        const uint32_t al = saddr(stage_a(sa, 1)), bl = saddr(stage_b(sb, 1));
#pragma unroll
        for (int k = 0; k < kQgBK / 16; ++k) {  // 16 bf16 = 32 bytes along the swizzled row
          const uint64_t dah = kmajor_sw128(ah + k * 32);
#pragma unroll
          for (int h = 0; h < NH; ++h) {  // accumulator h: TMEM columns [h N, (h + 1) N)
            const uint32_t acc = tmem + (uint32_t)(h * kN);
            const uint64_t dbh = kmajor_sw128(bh + h * kBox + k * 32);
            umma_bf16(acc, dah, dbh, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            if (TERMS == 3) {
              umma_bf16(acc, dah, kmajor_sw128(bl + h * kBox + k * 32), idesc, 1u);
              umma_bf16(acc, kmajor_sw128(al + k * 32), dbh, idesc, 1u);
            }
          }
        }
        umma_commit(&empty_a[sa]);  // the stages are free once these MMAs have read them
        umma_commit(&empty_b[sb]);
      }
      umma_commit(acc_full);
    }
  } else if (warp < 6) {
    // epilogue: TMEM lane = W row (warp w reads lanes 32 (w % 4) .. + 31), column = token
    const int quarter = warp & 3;
    const int64_t row = w0 + quarter * 32 + lane;
    if (!bar_wait(acc_full, 0)) ok = false;
    tc_fence_after();
    const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < kBN; c += 8) {
      uint32_t v[8];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
          : "r"(taddr + (uint32_t)c));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row < p.rows) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int tok = tok0 + c + u;
          if (tok < p.m) {
            const int64_t o = (int64_t)tok * p.rows + row;
            out[o] = p.add ? __uint_as_float(v[u]) + p.add[o] : __uint_as_float(v[u]);
          }
        }
      }
    }
  } else {
    // decoders: warp d owns row tiles [kT d, kT (d + 1)) of the 128-row A tile
    constexpr int kT = 8 / qg_decode_warps<TERMS, N, NH>();
    constexpr int kPre = qg_pre_depth<TERMS, N, NH>();
    const int d = warp - 6;
    const int64_t tile0 = w0 / 16 + kT * d;
    QgBytes cur[kT], nxt[kT];
    // the lane's slot of tile i for k-block kb in the prefetch ring (after both operand rings)
    uint8_t* pre = smem + qg_ring_bytes<TERMS, N, NH>() + 256;
    auto slot = [&](int kb, int i) {
      return pre + ((uint32_t)(kb % (kPre > 0 ? kPre : 1)) * 8u + (uint32_t)(kT * d + i)) * (32u * kQgSlot) +
             (uint32_t)lane * kQgSlot;
    };
    if constexpr (kPre > 0) {
      for (int j = 0; j < kPre - 1; ++j) {
        if (j < nk)
#pragma unroll
          for (int i = 0; i < kT; ++i) qg_copy<QT>(p, tile0 + i, kb0 + j, lane, slot(j, i));
        cp_async_commit();
      }
    } else {
#pragma unroll
      for (int i = 0; i < kT; ++i) qg_load<QT>(p, tile0 + i, kb0, lane, cur[i]);
    }
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kSA, use = kb / kSA;
      if constexpr (kPre > 0) {
        const int ahead = kb + kPre - 1;  // refills the slot read one iteration ago
        if (ahead < nk)
#pragma unroll
          for (int i = 0; i < kT; ++i) qg_copy<QT>(p, tile0 + i, kb0 + ahead, lane, slot(ahead, i));
        cp_async_commit();
        cp_async_wait<kPre - 1>();  // k-block kb's copies have landed
#pragma unroll
        for (int i = 0; i < kT; ++i) qg_read_slot<QT>(slot(kb, i), cur[i]);
      } else if (kb + 1 < nk) {
#pragma unroll
        for (int i = 0; i < kT; ++i) qg_load<QT>(p, tile0 + i, kb0 + kb + 1, lane, nxt[i]);
      }
      if (use > 0 && !bar_wait(&empty_a[s], (uint32_t)((use - 1) & 1))) ok = false;
      uint8_t* ahi = stage_a(s, 0);
      uint8_t* alo = stage_a(s, 1);
#pragma unroll
      for (int i = 0; i < kT; ++i) qg_store<QT, TERMS>(cur[i], kb0 + kb, lane, ahi, alo, 16 * (kT * d + i));
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
      __syncwarp();
      if (lane == 0) bar_arrive(&full_a[s]);
      if constexpr (kPre == 0) {
#pragma unroll
        for (int i = 0; i < kT; ++i) cur[i] = nxt[i];
      }
    }
    if constexpr (kPre > 0) cp_async_wait<0>();  // nothing in flight into shared memory at exit
  }
  if (!ok) atomicExch(p.status, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(qg_tmem_cols<N, NH>()));
  }
}

// y[i] = sum over splits of part[sp][i], in split order (+ add[i]).
__global__ void qgemm_fold_kernel(const float* __restrict__ part, int splits, int64_t n, const float* __restrict__ add,
                                  float* __restrict__ y) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int sp = 0; sp < splits; ++sp) v += __ldcg(part + sp * n + i);
    if (add) v += add[i];
    y[i] = v;
  }
}

template <int QT, int TERMS, int N, int NH>
cudaError_t launch_qgemm_fused(const j4b_qweight* w, const CUtensorMap& xh, const CUtensorMap& xl, int m, int kp,
                               int splits, int kb_per, float* out, const float* add, cudaStream_t stream) {
  constexpr int kBN = NH * N;
  const size_t smem = (size_t)qg_ring_bytes<TERMS, N, NH>() + 1024 + 256 +
                     qg_pre_bytes<TERMS, N, NH>(qg_pre_depth<TERMS, N, NH>());
  static bool attr_set[kMaxDevices] = {};
  if (w->dev < 0 || w->dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_set[w->dev]) {
    cudaError_t e = cudaFuncSetAttribute(qgemm_fused_kernel<QT, TERMS, N, NH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_set[w->dev] = true;
  }
  const int nk = kp / kQgBK;
  QgArgs p;
  p.data = w->data;
  p.L = layout_of(w);
  p.rows = w->rows;
  p.cols = w->cols;
  p.m = m;
  p.kp = kp;
  p.kb_per = kb_per;
  p.splits = splits;
  if (splits < 1 || kb_per < 1 || (int64_t)(splits - 1) * kb_per >= nk) return cudaErrorInvalidValue;
  p.y = out;
  p.add = p.splits == 1 ? add : nullptr;
  p.status = w->status;
  const int64_t tiles = ((w->rows + kQgBM - 1) / kQgBM) * p.splits * (((int64_t)m + kBN - 1) / kBN);
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  qgemm_fused_kernel<QT, TERMS, N, NH><<<(unsigned)tiles, qg_threads<TERMS, N, NH>(), smem, stream>>>(xh, xl, p);
  return cudaGetLastError();
}
