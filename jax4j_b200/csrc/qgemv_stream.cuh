// Streaming dequant-GEMV for batch <= 16 (included by qgemv.cuh, inside namespace
// j4b::<anonymous>; it reuses that file's fragment decoders tile_compute / tile_compute_pk and
// its bulk-copy and mbarrier helpers). Batch <= 4 packs x's hi and lo halves into one 8-column
// n-tile; 5..8 use one n-tile per half; 9..16 two n-tiles (NT = 2).
//
// Shape of one launch: one CTA per SM (15 compute warps + 1 producer warp, the whole SM's shared
// memory for a deep ring; a half-SM variant with 8 compute warps, so that two launches' CTAs
// co-reside, measured slower). A CTA owns one 1024-column K range ("split") of a contiguous run
// of 16-row tiles:
//   - the last warp is the producer: one elected lane streams the run's tile chunks (contiguous in the
//     split-major layout) into a ring of shared-memory stages with 1-D bulk copies, each stage
//     completing on its `full` mbarrier; it refills a stage once the warps that read it have
//     arrived on its `empty` mbarrier. A run that fits the ring is issued whole before the
//     dependency wait (weights are immutable once uploaded); of a longer run, about 48 KB, and
//     the rest once x is staged.
//   - the compute warps first turn x's 1024-column slice into fp16 hi/lo mma fragments in shared
//     memory (one 128-column chunk of one n-tile per warp, round-robin), then each warp takes
//     whole tiles round-robin and walks the tile's 8 chunks itself, so a tile's partial sum over
//     the split never leaves the warp's registers: no block barrier and no cross-warp reduction
//     in the main loop.
//   - split-K: a warp stores its tile's partial into the weight's scratch, and the warp whose
//     arrival completes the tile's counter adds the splits in split order (deterministic) and
//     writes y (+ add); with one split the warp writes y directly.
// Every mbarrier wait is bounded (j4b_wait.cuh); on a timeout the CTA records an error in the
// weight's status word, lets every copy still in flight land, and returns.

// NW compute warps + 1 producer warp. NW = 8: at most half an SM (112 KB of shared memory), so
// two launches' CTAs co-reside; NW = 15: one CTA per SM with a deeper ring, 512 threads, so the
// compiler may give each thread 128 registers (17 warps cap it at 96 and the two-n-tile decode
// spills).
template <int NW>
constexpr int stream_threads() { return (NW + 1) * 32; }
template <int NW>
constexpr int stream_smem_budget() { return NW <= 8 ? 112 * 1024 : 220 * 1024; }

template <int QT>
constexpr bool stream_needs_xblk() {
  return QT != J4B_Q8_0 && QT != J4B_Q6_K;
}
// Tile chunks per ring stage: copies of ~9-18 KB.
template <int QT>
constexpr int stream_tiles_per_stage() {
  return GemvTraits<QT>::kChunk <= 5000 ? 4 : (GemvTraits<QT>::kChunk <= 10000 ? 2 : 1);
}
// Shared-memory bytes of one 128-column chunk's x fragments: packed (batch <= 4) 4 x 16 bytes
// per lane of B fragments (+ 16 bytes of x block sums), unpacked 8 x 16 bytes (hi, lo of each
// k-step) (+ 32 bytes of block sums).
// Batch 9..16 (NT = 2, unpacked only): the 8-column n-tile's block repeated for batch rows 8..15.
template <int QT>
constexpr int stream_frag_ntile() { return 4096 + (stream_needs_xblk<QT>() ? 1024 : 0); }
template <int QT, bool PK, int NT = 1>
constexpr int stream_frag_chunk() {
  return PK ? 2048 + (stream_needs_xblk<QT>() ? 512 : 0) : NT * stream_frag_ntile<QT>();
}
template <int QT, bool PK, int NW, int NT = 1>
constexpr int stream_stages() {
  constexpr int stage = stream_tiles_per_stage<QT>() * GemvTraits<QT>::kChunk;
  constexpr int r = (stream_smem_budget<NW>() - 8 * stream_frag_chunk<QT, PK, NT>() - 512) / stage;
  return r > 16 ? 16 : r;
}
// ring | x fragments | full[R] | empty[R] mbarriers | seq[R] stage numbers
template <int QT, bool PK, int NW, int NT = 1>
constexpr int stream_smem_bytes() {
  return stream_stages<QT, PK, NW, NT>() * stream_tiles_per_stage<QT>() * GemvTraits<QT>::kChunk +
         8 * stream_frag_chunk<QT, PK, NT>() + 2 * 8 * stream_stages<QT, PK, NW, NT>() +
         4 * stream_stages<QT, PK, NW, NT>();
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Barrier 1 over the compute warps only (the producer warp never takes it).
template <int NW>
__device__ __forceinline__ void compute_warps_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory");
}
// Barrier 2: the compute warps arrive once x is staged; the producer waits on it before it issues
// the stages after the first ones. Global loads queue behind the SM's bulk copies in flight, so
// x (read only after the dependency wait) would otherwise land behind the whole ring.
template <int NW>
__device__ __forceinline__ void x_staged_arrive() {
  asm volatile("bar.arrive 2, %0;" ::"n"((NW + 1) * 32) : "memory");
}
template <int NW>
__device__ __forceinline__ void x_staged_wait() {
  asm volatile("bar.sync 2, %0;" ::"n"((NW + 1) * 32) : "memory");
}
// Stages issued before the dependency wait when the CTA's run is longer than the ring: about
// 48 KB, what the SM's share of HBM bandwidth brings in while the previous kernel drains; the
// rest waits for x, which the refills need anyway. A run that fits the ring is issued whole
// before the wait (measured: Q8_0 4096 x 4096 at batch 8, 7 tiles per CTA, 8.2 us per call whole
// against 9.0 us with 48 KB; Q4_K 14336 x 4096 at batch 1, 24 tiles per CTA, 14.9 us with 48 KB
// against 16.5 us with the whole ring).
template <int QT, bool PK, int NW, int NT>
constexpr int stream_pre_stages() {
  constexpr int stage = stream_tiles_per_stage<QT>() * GemvTraits<QT>::kChunk;
  constexpr int r = stream_stages<QT, PK, NW, NT>();
  constexpr int p = 49152 / stage;
  return p < 1 ? 1 : (p > r ? r : p);
}
template <int QT, bool PK, int NW, int NT>
__device__ __forceinline__ int stream_pre_ring(int nstages) {
  return nstages <= stream_stages<QT, PK, NW, NT>() ? stream_stages<QT, PK, NW, NT>()
                                                    : stream_pre_stages<QT, PK, NW, NT>();
}
// Waits (bounded) until the producer has issued stage `st` into its slot: only then is the slot's
// `full` barrier on the phase of that stage, so its parity identifies the stage. (A warp can reach
// a slot while the slot's previous stage is still in flight; the parity of that earlier phase
// would otherwise read as complete.)
__device__ __forceinline__ bool wait_issued(const volatile int* seq, int st) {
  if (*seq == st) return true;
  const uint64_t t0 = global_ns();
  while (*seq != st)
    if (global_ns() - t0 > kWaitNs) return false;
  return true;
}

// Counts one arrival at a split-K counter with acquire-release semantics at GPU scope: the
// arriving warp's partial stores (ordered before it by __syncwarp) are released with it, and the
// last arrival acquires every other split's partials; one atomic in place of fence + atomic.
// (A fold by a designated split that waits for the others' release-adds measured slower: Q8_0
// 4096 x 4096 at batch 8, 8.1 against 7.4 us per call; the last arrival never waits.)
__device__ __forceinline__ unsigned arrive_acq_rel(unsigned* ctr) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
  return old;
}

// Converts x's columns [kc0 + 128c, kc0 + 128c + 128) of batch rows row0.. into the fragment
// block at dst (columns past K and rows past the batch are zeros).
template <int QT, bool PK>
__device__ __forceinline__ void stream_prep_x(const GemvArgs& a, int64_t kc0, int c, int lane, uint8_t* dst,
                                              int row0) {
  const int g = lane >> 2, t = lane & 3;
  constexpr int kXB = kXBlocks<QT>;
  const int xrow = row0 + (PK ? (g >> 1) : g);
  const bool row_ok = xrow < a.batch;
  const float* xr = a.x + (int64_t)xrow * a.cols;
  const int64_t kb = kc0 + c * 128 + 2 * t;
  float2 p0[8], p1[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {  // all loads first (cols is a multiple of 32, so k < cols covers k + 9)
    const int64_t k = kb + 16 * j;
    const bool ok = row_ok && k < a.cols;
    p0[j] = ok ? __ldg(reinterpret_cast<const float2*>(xr + k)) : make_float2(0.f, 0.f);
    p1[j] = ok ? __ldg(reinterpret_cast<const float2*>(xr + k + 8)) : make_float2(0.f, 0.f);
  }
  uint32_t hi[8][2], lo[8][2];
  float xs_hi[8], xs_lo[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    __half2 h0 = __floats2half2_rn(p0[j].x, p0[j].y);
    __half2 h1 = __floats2half2_rn(p1[j].x, p1[j].y);
    const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
    __half2 l0 = __floats2half2_rn(p0[j].x - f0.x, p0[j].y - f0.y);
    __half2 l1 = __floats2half2_rn(p1[j].x - f1.x, p1[j].y - f1.y);
    const float2 g0 = __half22float2(l0), g1 = __half22float2(l1);
    hi[j][0] = *reinterpret_cast<uint32_t*>(&h0);
    hi[j][1] = *reinterpret_cast<uint32_t*>(&h1);
    lo[j][0] = *reinterpret_cast<uint32_t*>(&l0);
    lo[j][1] = *reinterpret_cast<uint32_t*>(&l1);
    xs_hi[j] = (f0.x + f0.y) + (f1.x + f1.y);
    xs_lo[j] = (g0.x + g0.y) + (g1.x + g1.y);
  }
  if constexpr (PK) {
    // lane group g carries batch g / 2: its hi part for even g, its lo part for odd g
    const bool odd = g & 1;
#pragma unroll
    for (int jj = 0; jj < 4; jj++) {
      const uint4 v = odd ? make_uint4(lo[2 * jj][0], lo[2 * jj][1], lo[2 * jj + 1][0], lo[2 * jj + 1][1])
                          : make_uint4(hi[2 * jj][0], hi[2 * jj][1], hi[2 * jj + 1][0], hi[2 * jj + 1][1]);
      *reinterpret_cast<uint4*>(dst + (jj * 32 + lane) * 16) = v;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; j++)
      *reinterpret_cast<uint4*>(dst + (j * 32 + lane) * 16) = make_uint4(hi[j][0], hi[j][1], lo[j][0], lo[j][1]);
  }
  if constexpr (stream_needs_xblk<QT>()) {
    // block sums of the represented x (hi + lo) for the output columns this lane holds
    float sums[kXB][2];
#pragma unroll
    for (int q = 0; q < kXB; q++) {
      constexpr int kSteps = 8 / kXB;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kSteps; j++) {
        const int jj = q * kSteps + j;
        s += PK ? ((g & 1) ? xs_lo[jj] : xs_hi[jj]) : xs_hi[jj] + xs_lo[jj];
      }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      sums[q][0] = __shfl_sync(0xffffffffu, s, 4 * (2 * t));
      sums[q][1] = __shfl_sync(0xffffffffu, s, 4 * (2 * t + 1));
    }
    if constexpr (PK) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      float* vp = reinterpret_cast<float*>(&v);
#pragma unroll
      for (int q = 0; q < kXB; q++) vp[q] = sums[q][0] + sums[q][1];  // batch t: hi + lo sums
      *reinterpret_cast<float4*>(dst + 2048 + lane * 16) = v;
    } else {
      float4 v[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
      float* vp = reinterpret_cast<float*>(v);
#pragma unroll
      for (int q = 0; q < kXB; q++) {
        vp[2 * q] = sums[q][0];      // batch 2t
        vp[2 * q + 1] = sums[q][1];  // batch 2t + 1
      }
      *reinterpret_cast<float4*>(dst + 4096 + lane * 16) = v[0];
      *reinterpret_cast<float4*>(dst + 4096 + 512 + lane * 16) = v[1];
    }
  }
}

// All-gather, second half (inside the GEMV, after a warp's tiles): the warp copies its share of
// this rank's gathered half -- every rank's outputs of this step as flagged words -- to the
// output as the flags appear. Each thread issues the loads of up to four word pairs before it
// checks a flag and re-reads only a pair whose flags have not arrived. The launch's last warp to
// finish advances the channel's step counter (every warp read it, in gather_slot, before its own
// arrival) and resets the counter of finished warps. A wait gives up after a second and marks the
// peer group's status word.
template <int NW>
__device__ __forceinline__ void gather_copy(const GemvArgs& a, const GatherSlot& gs, int warp, int lane) {
  const unsigned long long* src = a.peer_y[a.rank] + gs.off;  // 16-byte aligned
  const int64_t nthreads = (int64_t)gridDim.x * NW * 32;
  const int64_t tid = ((int64_t)blockIdx.x * NW + warp) * 32 + lane;
  const unsigned want = gs.flag;
  const uint64_t t0 = global_ns();
  bool timed_out = false;
  if (((uintptr_t)a.gout & 7u) == 0) {
    const int64_t npairs = a.gathered / 2;
    float2* out2 = reinterpret_cast<float2*>(a.gout);
    for (int64_t p0 = tid; p0 < npairs; p0 += nthreads * 4) {
      ulonglong2 w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (p0 + u * nthreads < npairs) w[u] = gather_load2(src + 2 * (p0 + u * nthreads));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t p = p0 + u * nthreads;
        if (p >= npairs) break;
        while (((unsigned)(w[u].x >> 32) != want || (unsigned)(w[u].y >> 32) != want) && !timed_out) {
          if (global_ns() - t0 > kPeerWaitNs) {
            timed_out = true;
          } else {
            __nanosleep(128);  // polls spaced out: warps still on their tiles keep the memory pipes
            w[u] = gather_load2(src + 2 * p);
          }
        }
        out2[p] = make_float2(__uint_as_float((unsigned)w[u].x), __uint_as_float((unsigned)w[u].y));
      }
    }
    if ((a.gathered & 1) && tid == 0) {
      unsigned long long w = gather_load(src + a.gathered - 1);
      while ((unsigned)(w >> 32) != want && !timed_out) {
        if (global_ns() - t0 > kPeerWaitNs) timed_out = true;
        else w = gather_load(src + a.gathered - 1);
      }
      a.gout[a.gathered - 1] = __uint_as_float((unsigned)w);
    }
  } else {
    for (int64_t i = tid; i < a.gathered; i += nthreads) {
      unsigned long long w = gather_load(src + i);
      while ((unsigned)(w >> 32) != want && !timed_out) {
        if (global_ns() - t0 > kPeerWaitNs) timed_out = true;
        else w = gather_load(src + i);
      }
      a.gout[i] = __uint_as_float((unsigned)w);
    }
  }
  if (timed_out) atomicExch(a.pstatus, 1);
  __syncwarp();
  if (lane == 0) {
    __threadfence();
    if (atomicAdd(a.done, 1u) == (unsigned)(gridDim.x * NW - 1)) {
      *a.done = 0u;
      *(volatile unsigned*)a.step = want;  // step + 1
    }
  }
}

// Output element cc of lane (g, t)'s accumulator -> (row in tile, batch column); unpacked element
// cc belongs to n-tile cc / 4 (batch columns 8 (cc / 4) ..).
template <bool PK>
__device__ __forceinline__ void stream_coord(int lane, int cc, int& row, int& bcol) {
  const int g = lane >> 2, t = lane & 3;
  if (PK) {
    row = g + 8 * cc;
    bcol = t;
  } else {
    row = g + 8 * ((cc & 3) >> 1);
    bcol = 8 * (cc >> 2) + 2 * t + (cc & 1);
  }
}

template <int QT, bool PK, int NW, int NT>
__global__ void __launch_bounds__(stream_threads<NW>(), NW == 8 ? 2 : 1) qgemv_stream_kernel(GemvArgs a) {
  using T = GemvTraits<QT>;
  static_assert(NT == 1 || (NT == 2 && !PK), "two n-tiles: unpacked fragments only");
  constexpr int R = stream_stages<QT, PK, NW, NT>();
  constexpr int kU = stream_tiles_per_stage<QT>();
  constexpr int kStage = kU * T::kChunk;
  constexpr int kFrag = stream_frag_chunk<QT, PK, NT>();
  constexpr int kFragN = stream_frag_ntile<QT>();  // one n-tile's part of an unpacked chunk
  constexpr int kNV = PK ? 2 : 4 * NT;  // accumulator floats per lane per tile
  constexpr int kXB = kXBlocks<QT>;
  static_assert(R >= 2, "ring too small");
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* frag = smem + R * kStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(frag + 8 * kFrag);
  uint64_t* empty = full + R;
  volatile int* seq = reinterpret_cast<volatile int*>(empty + R);  // stage last issued per slot

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int split = blockIdx.x % a.ksplit;
  const int ngroups = gridDim.x / a.ksplit;
  const int group = blockIdx.x / a.ksplit;
  const int64_t tile0 = (int64_t)group * a.rt / ngroups;
  const int ntiles = (int)((int64_t)(group + 1) * a.rt / ngroups - tile0);
  const int nstages = (ntiles + kU - 1) / kU;
  const int64_t kc0 = (int64_t)split * 1024;
  const uint32_t chunk_bytes = (uint32_t)a.L.chunk_bytes(split);
  const uint32_t meta_off = (uint32_t)(a.L.groups_in_split(split) * T::kQ);
  const int nchunks = (int)(a.kpad - kc0 >= 1024 ? 8 : (a.kpad - kc0) / 128);

  if (threadIdx.x == 0) {
    for (int s = 0; s < R; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kU);
      seq[s] = -1;
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  int issued = 0;  // stages issued (producer lane 0 only)
  if (warp == NW) {
    // ---------------- producer ----------------
    const uint64_t policy = l2_evict_first_policy();
    auto issue = [&](int st) {
      const int first = st * kU, count = min(kU, ntiles - first);
      const uint32_t bytes = (uint32_t)count * chunk_bytes;
      uint64_t* bar = &full[st % R];
      seq[st % R] = st;
      mbar_expect_tx(bar, bytes);
      tma_load_1d_stream(ring + (st % R) * kStage, a.data + a.L.chunk_offset(split, tile0 + first), bytes, bar,
                         policy);
    };
    const int pre = stream_pre_ring<QT, PK, NW, NT>(nstages);
    if (lane == 0)
      for (; issued < pre && issued < nstages; issued++) issue(issued);
    pdl_launch_dependents();
    pdl_wait();
    x_staged_wait<NW>();
    if (lane == 0) {
      for (; issued < nstages; issued++) {
        const int slot = issued % R;
        if (!mbar_wait_bounded(&empty[slot], (uint32_t)(((issued / R) - 1) & 1))) {
          failed = true;
          break;
        }
        fence_proxy_async();  // the readers' generic-proxy reads of the slot precede the refill
        issue(issued);
      }
    }
  } else {
    // ---------------- compute warps ----------------
    pdl_launch_dependents();
    pdl_wait();
    const GatherSlot gslot = gather_slot(a);  // peer all-gather only
    // the (chunk, n-tile) blocks of x round-robin over the compute warps
    for (int b = warp; b < 8 * NT; b += NW)
      if ((b & 7) < nchunks) stream_prep_x<QT, PK>(a, kc0, b & 7, lane, frag + (b & 7) * kFrag + (b >> 3) * kFragN, 8 * (b >> 3));
    x_staged_arrive<NW>();
    compute_warps_sync<NW>();

    for (int u = warp; u < ntiles; u += NW) {
      const int st = u / kU, slot = st % R;
      if (!failed && !(wait_issued(seq + slot, st) && mbar_wait_bounded(&full[slot], (uint32_t)((st / R) & 1))))
        failed = true;
      failed = __any_sync(0xffffffffu, failed);  // keep the warp's lanes together
      float acc[kNV];
#pragma unroll
      for (int i = 0; i < kNV; i++) acc[i] = 0.f;
      if (!failed) {
        const uint8_t* base = ring + slot * kStage + (u % kU) * chunk_bytes;
#pragma unroll 2
        for (int c = 0; c < nchunks; c++) {
          const uint8_t* fc = frag + c * kFrag;
          if constexpr (PK) {
            uint32_t bp[8][2];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
              const uint4 v = *reinterpret_cast<const uint4*>(fc + (jj * 32 + lane) * 16);
              bp[2 * jj][0] = v.x;
              bp[2 * jj][1] = v.y;
              bp[2 * jj + 1][0] = v.z;
              bp[2 * jj + 1][1] = v.w;
            }
            float xb[kXB];
            if constexpr (stream_needs_xblk<QT>()) {
              const float4 v = *reinterpret_cast<const float4*>(fc + 2048 + lane * 16);
              const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int q = 0; q < kXB; q++) xb[q] = vv[q];
            } else {
#pragma unroll
              for (int q = 0; q < kXB; q++) xb[q] = 0.f;
            }
            float r2[2] = {acc[0], acc[1]};
            tile_compute_pk<QT>(base, base + meta_off, c, lane, bp, xb, r2);
            acc[0] = r2[0];
            acc[1] = r2[1];
          } else {
            uint32_t bh[NT][8][2], bl[NT][8][2];
            float xb[NT][kXB][2];
#pragma unroll
            for (int n = 0; n < NT; n++) {
              const uint8_t* fn = fc + n * kFragN;
#pragma unroll
              for (int j = 0; j < 8; j++) {
                const uint4 v = *reinterpret_cast<const uint4*>(fn + (j * 32 + lane) * 16);
                bh[n][j][0] = v.x;
                bh[n][j][1] = v.y;
                bl[n][j][0] = v.z;
                bl[n][j][1] = v.w;
              }
              if constexpr (stream_needs_xblk<QT>()) {
                const float4 v0 = *reinterpret_cast<const float4*>(fn + 4096 + lane * 16);
                const float4 v1 = *reinterpret_cast<const float4*>(fn + 4096 + 512 + lane * 16);
                const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                for (int q = 0; q < kXB; q++) {
                  xb[n][q][0] = vv[2 * q];
                  xb[n][q][1] = vv[2 * q + 1];
                }
              } else {
#pragma unroll
                for (int q = 0; q < kXB; q++) xb[n][q][0] = xb[n][q][1] = 0.f;
              }
            }
            float r4[NT][4];
#pragma unroll
            for (int n = 0; n < NT; n++)
#pragma unroll
              for (int i = 0; i < 4; i++) r4[n][i] = acc[4 * n + i];
            tile_compute<QT, NT>(base, base + meta_off, c, lane, bh, bl, xb, r4);
#pragma unroll
            for (int n = 0; n < NT; n++)
#pragma unroll
              for (int i = 0; i < 4; i++) acc[4 * n + i] = r4[n][i];
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // this warp is done reading the stage
      if (failed) continue;

      const int64_t tile = tile0 + u;
      if (a.ksplit > 1) {
        float* part = a.partials + ((int64_t)split * a.rt + tile) * 256;
#pragma unroll
        for (int i = 0; i < kNV; i++) __stcg(part + i * 32 + lane, acc[i]);
        __syncwarp();  // every lane's partial store precedes lane 0's release
        unsigned last = 0;
        if (lane == 0) last = arrive_acq_rel(a.arrivals + tile) == (unsigned)(a.ksplit - 1);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __syncwarp();  // lane 0's acquire precedes every lane's loads of the other partials
        // the last arrival adds the splits in split order, four splits' loads in flight at once
        const float* p0 = a.partials + tile * 256 + lane;
        const int64_t sstride = a.rt * 256;
#pragma unroll
        for (int i = 0; i < kNV; i++) acc[i] = 0.f;
        for (int sp0 = 0; sp0 < a.ksplit; sp0 += 4) {
          float v[4][kNV];
#pragma unroll
          for (int s = 0; s < 4; s++)
#pragma unroll
            for (int i = 0; i < kNV; i++)
              v[s][i] = sp0 + s < a.ksplit ? __ldcg(p0 + (sp0 + s) * sstride + i * 32) : 0.f;
#pragma unroll
          for (int s = 0; s < 4; s++)
#pragma unroll
            for (int i = 0; i < kNV; i++)
              if (sp0 + s < a.ksplit) acc[i] += v[s][i];
        }
        if (lane == 0) a.arrivals[tile] = 0u;  // ready for the next launch
      }
#pragma unroll
      for (int i = 0; i < kNV; i++) {
        int row, bcol;
        stream_coord<PK>(lane, i, row, bcol);
        const int64_t r = tile * 16 + row;
        if (r < a.rows && bcol < a.batch) {
          float v = acc[i];
          if (a.add) v += a.add[(int64_t)bcol * a.rows + r];
          store_y(a, gslot, bcol, r, v);
        }
      }
    }
    if (a.nranks > 1) gather_copy<NW>(a, gslot, warp, lane);
  }

  if (__syncthreads_or(failed)) {
    // Let every copy still in flight land before the CTA's shared memory is released.
    if (warp == NW && lane == 0) {
      atomicExch(a.status, 1);
      for (int s = 0; s < R && s < issued; s++) {
        const int last = s + ((issued - 1 - s) / R) * R;  // the last stage issued into slot s
        mbar_wait_bounded(&full[s], (uint32_t)((last / R) & 1));
      }
    }
    __syncthreads();
  }
}

template <int QT, bool PK, int NW, int NT = 1>
cudaError_t launch_gemv_stream(const j4b_qweight* w, const float* x, const float* add, float* y, int batch,
                               int sms, cudaStream_t stream, const GemvPeers* peers, unsigned* grid_out,
                               bool pdl) {
  constexpr int smem = stream_smem_bytes<QT, PK, NW, NT>();
  static bool attr_set[kMaxDevices] = {};  // function attributes are per device context
  if (w->dev < 0 || w->dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_set[w->dev]) {
    cudaError_t e = cudaFuncSetAttribute(qgemv_stream_kernel<QT, PK, NW, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[w->dev] = true;
  }
  GemvArgs a;
  memset(&a, 0, sizeof(a));
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
  if (peers) {
    a.nranks = peers->nranks;
    a.rank = peers->rank;
    a.step = peers->step;
    a.done = peers->done;
    a.half_words = peers->half_words;
    a.gout = peers->out;
    a.gathered = peers->gathered;
    a.pstatus = peers->status;
    for (int p = 0; p < peers->nranks; ++p) a.peer_y[p] = peers->y[p];
  }
  // one CTA per SM: as many tile groups as fit next to the K splits
  const int64_t groups = std::max<int64_t>(1, std::min<int64_t>(w->rt, (int64_t)sms / w->ksplit));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(groups * w->ksplit));
  cfg.blockDim = dim3(stream_threads<NW>());
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (grid_out) *grid_out = cfg.gridDim.x;
  return cudaLaunchKernelEx(&cfg, qgemv_stream_kernel<QT, PK, NW, NT>, a);
}
