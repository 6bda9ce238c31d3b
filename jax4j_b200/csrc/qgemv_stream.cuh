// Streaming dequant-GEMV for batch <= 8 (included by qgemv.cuh, inside namespace
// j4b::<anonymous>; it reuses that file's fragment decoders tile_compute / tile_compute_pk and
// its bulk-copy and mbarrier helpers).
//
// Shape of one launch: one CTA per SM (16 compute warps + 1 producer warp). A CTA owns one
// 1024-column K range ("split") of a contiguous run of 16-row tiles:
//   - the producer warp: one elected lane streams the run's tile chunks (contiguous in the
//     split-major layout) into a ring of shared-memory slots with 1-D bulk copies, each slot's
//     copy completing on its `full` mbarrier, and refills a slot once the tile(s) in it are done
//     (`empty`). The first ring's worth is issued before the dependency wait (weights are
//     immutable once uploaded; the first GEMV after an upload is launched without programmatic
//     dependent launch, so that one waits).
//   - compute warp w takes 128-column chunk c = w % 8 of the split and builds that chunk's x
//     fragments (fp16 hi / lo) in its registers straight from global memory, once; the warps
//     w / 8 = 0 and 1 take alternate tiles. For each tile the eight warps of its stream multiply
//     their chunk in parallel and hand their partial sums over in shared memory; the eighth to
//     arrive (a per-tile counter) adds the eight chunks in chunk order, releases the slot, and
//     finishes the tile. No block barrier in the main loop.
//   - split-K: the finishing warp stores the tile's split partial into the weight's scratch, and
//     the warp whose arrival completes the tile's counter (one acquire-release atomic) adds the
//     splits in split order (deterministic) and writes y (+ add); with one split the finishing
//     warp writes y directly.
// Every mbarrier wait is bounded (j4b_wait.cuh); on a timeout the CTA records an error in the
// weight's status word, lets every copy still in flight land, and returns.

// NW compute warps (a multiple of 8: one warp per 128-column chunk per tile stream) + 1 producer.
template <int NW>
constexpr int stream_threads() { return (NW + 1) * 32; }
template <int NW>
constexpr int stream_smem_budget() { return 220 * 1024; }

template <int QT>
constexpr bool stream_needs_xblk() {
  return QT != J4B_Q8_0 && QT != J4B_Q6_K;
}
// Tile chunks per ring stage: copies of ~9-18 KB.
template <int QT>
constexpr int stream_tiles_per_stage() {
  return GemvTraits<QT>::kChunk <= 5000 ? 4 : (GemvTraits<QT>::kChunk <= 10000 ? 2 : 1);
}
// Shared-memory bytes of one ring slot: its tile chunks, plus for each of them the eight chunk
// partials (kNV floats x 32 lanes each) the tile's warps hand to the warp that adds them.
template <int QT, bool PK>
constexpr int stream_slot_bytes() {
  return stream_tiles_per_stage<QT>() * (GemvTraits<QT>::kChunk + 8 * (PK ? 2 : 4) * 32 * 4);
}
template <int QT, bool PK, int NW>
constexpr int stream_stages() {
  constexpr int r = (stream_smem_budget<NW>() - 1024) / stream_slot_bytes<QT, PK>();
  return r > 16 ? 16 : r;
}
// ring of tile chunks | chunk partials | full[R] | empty[R] mbarriers | seq[R] stage numbers |
// cnt[R * tiles per stage] chunk arrivals
template <int QT, bool PK, int NW>
constexpr int stream_smem_bytes() {
  return stream_stages<QT, PK, NW>() * stream_slot_bytes<QT, PK>() + 2 * 8 * stream_stages<QT, PK, NW>() +
         4 * stream_stages<QT, PK, NW>() + 4 * stream_stages<QT, PK, NW>() * stream_tiles_per_stage<QT>();
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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
__device__ __forceinline__ unsigned arrive_acq_rel(unsigned* ctr) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
  return old;
}

// x fragments of one 128-column chunk (columns [kc0 + 128c, kc0 + 128c + 128) of every batch row,
// zeros past K and past the batch), built in this warp's registers straight from global memory:
// fp16 hi / lo B fragments per k-step and, for the formats whose codes carry an offset, the block
// sums of the represented x (hi + lo) for the output columns this lane holds.
template <int QT, bool PK>
struct StreamX {
  static constexpr int kXB = kXBlocks<QT>;
  uint32_t hi[PK ? 1 : 1][8][2];  // packed: lane group g holds batch g / 2, hi for even g, lo for odd g
  uint32_t lo[PK ? 1 : 1][8][2];  // unpacked only
  float blk[kXB][2];              // unpacked: batch 2t, 2t + 1; packed: [q][0] = batch t
};

template <int QT, bool PK>
__device__ __forceinline__ void stream_x_regs(const GemvArgs& a, int64_t kc0, int c, int lane, StreamX<QT, PK>& X) {
  const int g = lane >> 2, t = lane & 3;
  constexpr int kXB = kXBlocks<QT>;
  const int xrow = PK ? (g >> 1) : g;
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
  float xs_hi[8], xs_lo[8];
  const bool odd = g & 1;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    __half2 h0 = __floats2half2_rn(p0[j].x, p0[j].y);
    __half2 h1 = __floats2half2_rn(p1[j].x, p1[j].y);
    const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
    __half2 l0 = __floats2half2_rn(p0[j].x - f0.x, p0[j].y - f0.y);
    __half2 l1 = __floats2half2_rn(p1[j].x - f1.x, p1[j].y - f1.y);
    const float2 g0 = __half22float2(l0), g1 = __half22float2(l1);
    const uint32_t hw0 = *reinterpret_cast<uint32_t*>(&h0), hw1 = *reinterpret_cast<uint32_t*>(&h1);
    const uint32_t lw0 = *reinterpret_cast<uint32_t*>(&l0), lw1 = *reinterpret_cast<uint32_t*>(&l1);
    if constexpr (PK) {
      X.hi[0][j][0] = odd ? lw0 : hw0;
      X.hi[0][j][1] = odd ? lw1 : hw1;
    } else {
      X.hi[0][j][0] = hw0;
      X.hi[0][j][1] = hw1;
      X.lo[0][j][0] = lw0;
      X.lo[0][j][1] = lw1;
    }
    xs_hi[j] = (f0.x + f0.y) + (f1.x + f1.y);
    xs_lo[j] = (g0.x + g0.y) + (g1.x + g1.y);
  }
#pragma unroll
  for (int q = 0; q < kXB; q++) X.blk[q][0] = X.blk[q][1] = 0.f;
  if constexpr (stream_needs_xblk<QT>()) {
#pragma unroll
    for (int q = 0; q < kXB; q++) {
      constexpr int kSteps = 8 / kXB;
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < kSteps; j++) {
        const int jj = q * kSteps + j;
        sum += PK ? (odd ? xs_lo[jj] : xs_hi[jj]) : xs_hi[jj] + xs_lo[jj];
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      const float s0 = __shfl_sync(0xffffffffu, sum, 4 * (2 * t));
      const float s1 = __shfl_sync(0xffffffffu, sum, 4 * (2 * t + 1));
      if constexpr (PK) {
        X.blk[q][0] = s0 + s1;  // batch t: hi + lo sums
      } else {
        X.blk[q][0] = s0;  // batch 2t
        X.blk[q][1] = s1;  // batch 2t + 1
      }
    }
  }
}

// Output element cc of lane (g, t)'s accumulator -> (row in tile, batch column).
template <bool PK>
__device__ __forceinline__ void stream_coord(int lane, int cc, int& row, int& bcol) {
  const int g = lane >> 2, t = lane & 3;
  if (PK) {
    row = g + 8 * cc;
    bcol = t;
  } else {
    row = g + 8 * (cc >> 1);
    bcol = 2 * t + (cc & 1);
  }
}

template <int QT, bool PK, int NW>
__global__ void __launch_bounds__(stream_threads<NW>(), 1) qgemv_stream_kernel(GemvArgs a) {
  using T = GemvTraits<QT>;
  constexpr int R = stream_stages<QT, PK, NW>();
  constexpr int kU = stream_tiles_per_stage<QT>();
  constexpr int kStage = kU * T::kChunk;
  constexpr int kNV = PK ? 2 : 4;  // accumulator floats per lane per tile
  constexpr int kStreams = NW / 8;  // tile streams: warp w computes chunk w % 8 of stream w / 8's tiles
  static_assert(R >= 2 && NW % 8 == 0, "ring too small");
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  float* part = reinterpret_cast<float*>(smem + R * kStage);  // [R * kU][8 chunks][kNV * 32]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + R * stream_slot_bytes<QT, PK>());
  uint64_t* empty = full + R;
  volatile int* seq = reinterpret_cast<volatile int*>(empty + R);  // stage last issued per slot
  unsigned* cnt = reinterpret_cast<unsigned*>(empty + R) + R;       // chunk arrivals per tile slot

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
      mbar_init(&empty[s], kU);  // one arrival per tile: the warp that adds its chunk partials
      seq[s] = -1;
    }
    for (int s = 0; s < R * kU; s++) cnt[s] = 0u;
    fence_mbar_init();
  }
  __syncthreads();

  bool failed = false;
  int issued = 0;  // stages issued (producer lane 0 only)
  if (warp == NW) {
    // ---------------- producer ----------------
    auto issue = [&](int st) {
      const int first = st * kU, count = min(kU, ntiles - first);
      const uint32_t bytes = (uint32_t)count * chunk_bytes;
      uint64_t* bar = &full[st % R];
      seq[st % R] = st;
      mbar_expect_tx(bar, bytes);
      tma_load_1d(ring + (st % R) * kStage, a.data + a.L.chunk_offset(split, tile0 + first), bytes, bar);
    };
    if (lane == 0)
      for (; issued < R && issued < nstages; issued++) issue(issued);
    pdl_launch_dependents();
    pdl_wait();
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
    const int c = warp & 7, h = warp >> 3;
    const bool active = c < nchunks;
    pdl_launch_dependents();
    pdl_wait();
    int64_t par_off = 0;  // parity half of the gathered buffer (peer all-gather only)
    if (a.nranks > 1) par_off = (int64_t)(*a.step & 1u) * a.half_floats;
    StreamX<QT, PK> X;
    if (active) stream_x_regs<QT, PK>(a, kc0, c, lane, X);

    for (int u = h; u < ntiles; u += kStreams) {
      const int st = u / kU, slot = st % R, ts = slot * kU + u % kU;
      if (!failed && !(wait_issued(seq + slot, st) && mbar_wait_bounded(&full[slot], (uint32_t)((st / R) & 1))))
        failed = true;
      failed = __any_sync(0xffffffffu, failed);  // keep the warp's lanes together
      float acc[kNV];
#pragma unroll
      for (int i = 0; i < kNV; i++) acc[i] = 0.f;
      if (!failed && active) {
        const uint8_t* base = ring + slot * kStage + (u % kU) * chunk_bytes;
        if constexpr (PK) {
          float xb[kXBlocks<QT>];
#pragma unroll
          for (int q = 0; q < kXBlocks<QT>; q++) xb[q] = X.blk[q][0];
          float r2[2] = {0.f, 0.f};
          tile_compute_pk<QT>(base, base + meta_off, c, lane, X.hi[0], xb, r2);
          acc[0] = r2[0];
          acc[1] = r2[1];
        } else {
          float r4[1][4] = {{0.f, 0.f, 0.f, 0.f}};
          float xb[1][kXBlocks<QT>][2];
#pragma unroll
          for (int q = 0; q < kXBlocks<QT>; q++) {
            xb[0][q][0] = X.blk[q][0];
            xb[0][q][1] = X.blk[q][1];
          }
          tile_compute<QT, 1>(base, base + meta_off, c, lane, X.hi, X.lo, xb, r4);
#pragma unroll
          for (int i = 0; i < 4; i++) acc[i] = r4[0][i];
        }
      }
      // hand this chunk's partial over; the eighth warp to arrive adds the chunks in order
      float* pt = part + (int64_t)ts * 8 * kNV * 32;
#pragma unroll
      for (int i = 0; i < kNV; i++) pt[(c * kNV + i) * 32 + lane] = acc[i];
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(cnt + ts, 1u) == 7u;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence_block();
#pragma unroll
      for (int i = 0; i < kNV; i++) {
        float v = 0.f;
#pragma unroll
        for (int cc = 0; cc < 8; cc++) v += pt[(cc * kNV + i) * 32 + lane];
        acc[i] = v;
      }
      __syncwarp();
      if (lane == 0) {
        cnt[ts] = 0u;
        mbar_arrive(&empty[slot]);  // the tile is done with its slot (chunks and partials)
      }
      if (failed) continue;

      const int64_t tile = tile0 + u;
      if (a.ksplit > 1) {
        float* gpart = a.partials + ((int64_t)split * a.rt + tile) * 256;
#pragma unroll
        for (int i = 0; i < kNV; i++) __stcg(gpart + i * 32 + lane, acc[i]);
        __syncwarp();  // every lane's partial store precedes lane 0's release
        unsigned lastk = 0;
        if (lane == 0) lastk = arrive_acq_rel(a.arrivals + tile) == (unsigned)(a.ksplit - 1);
        lastk = __shfl_sync(0xffffffffu, lastk, 0);
        if (!lastk) continue;
        __syncwarp();  // lane 0's acquire precedes every lane's loads of the other partials
        // the last arrival adds the splits in split order, four splits' loads in flight at once
        const float* p0 = a.partials + tile * 256 + lane;
        const int64_t sstride = a.rt * 256;
#pragma unroll
        for (int i = 0; i < kNV; i++) acc[i] = 0.f;
        for (int sp0 = 0; sp0 < a.ksplit; sp0 += 4) {
          float v[4][kNV];
#pragma unroll
          for (int s4 = 0; s4 < 4; s4++)
#pragma unroll
            for (int i = 0; i < kNV; i++)
              v[s4][i] = sp0 + s4 < a.ksplit ? __ldcg(p0 + (sp0 + s4) * sstride + i * 32) : 0.f;
#pragma unroll
          for (int s4 = 0; s4 < 4; s4++)
#pragma unroll
            for (int i = 0; i < kNV; i++)
              if (sp0 + s4 < a.ksplit) acc[i] += v[s4][i];
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
          store_y(a, par_off, bcol, r, v);
        }
      }
    }
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
  signal_peers(a);
}

template <int QT, bool PK, int NW>
cudaError_t launch_gemv_stream(const j4b_qweight* w, const float* x, const float* add, float* y, int batch,
                               int sms, cudaStream_t stream, const GemvPeers* peers, unsigned* grid_out,
                               bool pdl) {
  constexpr int smem = stream_smem_bytes<QT, PK, NW>();
  static bool attr_set[kMaxDevices] = {};  // function attributes are per device context
  if (w->dev < 0 || w->dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_set[w->dev]) {
    cudaError_t e = cudaFuncSetAttribute(qgemv_stream_kernel<QT, PK, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
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
    a.half_floats = peers->half_floats;
    for (int p = 0; p < peers->nranks; ++p) {
      a.peer_y[p] = peers->y[p];
      a.peer_ctr[p] = peers->ctr[p];
    }
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
  return cudaLaunchKernelEx(&cfg, qgemv_stream_kernel<QT, PK, NW>, a);
}
