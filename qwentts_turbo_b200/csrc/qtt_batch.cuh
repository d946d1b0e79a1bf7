// Batched decode on 5th-generation tensor cores (tcgen05). Included by qtt_kernel.cu: it is
// the same translation unit as the batch-1 kernel and uses its grid barrier, attention work
// items, sampler, head masks and stage helpers.
//
// One cooperative launch of qtt_batch_kernel runs one program for B <= 64 utterances: a frame
// of every utterance (MODE_B_FRAME), one context step of the backbone prefill (MODE_B_PREFILL),
// a chunk of one utterance's context (MODE_B_PREFILL_DENSE) or the first group-0 token after the
// prefill (MODE_B_HEAD). The weights are streamed once per program for the whole batch.
//
// The grid is made of thread-block clusters of p.bcl CTAs (4, or 2 when the GPU cannot hold
// enough clusters of 4). Every projection is a GEMM
//     D[tokens x rows] = A[tokens x K] * W[rows x K]^T
// split into 128 / bcl row tiles of N rows, one per cluster, and bcl K slices, one per CTA of the
// cluster (128 CTAs work on every GEMM; the rest of the grid waits at the stage's barrier):
//   * W: the CTA's rows of the tile over its K slice. The producer warp streams them per K step of
//     128 as 2-D TMA boxes of N rows x 64 columns with the 128-byte swizzle (gate/up: a box of N/2
//     gate rows and one of N/2 up rows) into a ring of 4 KB slots (an entry of N / 16 slots per
//     K step) and runs ahead across grid barriers (weights do not depend on activations).
//   * A: the activations of all tokens as two bf16 planes, hi = bf16(v) and lo = bf16(v - hi),
//     written to global memory by the stage that produced them (row = token, plane 1 TBMAX rows
//     below plane 0). After the stage's grid barrier the activation-loader warp streams them with
//     2-D TMA boxes (64 columns x 64 tokens per plane) into a 3-slot ring: one slot per 64-token
//     tile and K step, hi rows 0..63 and lo rows 64..127.
//   * D: one M = 128 tcgen05.mma per K sub-step of 16 reads the whole slot, so TMEM lanes 0..63
//     hold hi.W and lanes 64..127 lo.W of the tile's 64 tokens (fp32, N columns per token tile):
//     ~16 mantissa bits of the activations, close to an fp32 GEMV.
// K-slice exchange: the consumer warps move D to shared memory (the activation ring, idle until
// the next stage's loads), lo lanes first and the hi lanes added, then signal the cluster's other
// CTAs on an mbarrier each; every CTA then sums its share of the tile's outputs over the bcl CTAs'
// partials in rank order, reading them through distributed shared memory, and runs the epilogue:
// the deferred RMSNorm scale and the stage's elementwise work, the next GEMM's A planes. Sums of
// squares for the next RMSNorm are accumulated per token with 64-bit fixed-point atomics (order
// independent), so reruns are bit-identical.
//
// Stages of a code-predictor pass: INPUT (embedding rows -> x, A planes, sums of squares) |
// per layer QKV | attention | O (+ residual) | gate/up | down (+ residual) | NORM | HEAD; a
// frame adds COMBINE (the 16-embedding sum + text row) before the backbone layers and the
// codec head (+ sampler) at the end.

constexpr int KSUB = 64;                  // K elements of one 128-byte swizzle atom row
constexpr int NSUB = 2;                   // atoms per pipeline step
constexpr int KSTEP = KSUB * NSUB;        // K elements per pipeline step
constexpr int BROWS = 128;                // CTAs of a GEMM stage (row tiles x K slices)
constexpr int WSLOT = 4096;               // weight-ring slot; a K step of an N-row tile is N / 16 slots
constexpr int NWSLOT = 30;
constexpr int NWE = 8;                    // weight entries (K steps) in flight
constexpr int APLANE_BYTES = 64 * 128;    // one plane of an activation atom: 64 token rows
constexpr int ASUB_BYTES = 2 * APLANE_BYTES;  // hi plane, then lo plane
constexpr int AS_BYTES = NSUB * ASUB_BYTES;
constexpr int NAS = 3;
constexpr int WRING_BYTES = NWSLOT * WSLOT;
constexpr uint32_t TMEM_COLS = 512;       // up to two 64-token tiles of the widest tile
constexpr int NMAX_B = 192;               // widest tile: 96 gate + 96 up rows (clusters of 4)
// The batched kernel's rings span sm.ring and the two batch-1 scratch areas behind it (sm.xs,
// sm.att), which it does not use.
constexpr int BRING_BYTES = NSLOTS * SLOT_BYTES + NTMAX * INTER * 4 + ATT_STAGE_BYTES;
static_assert(WRING_BYTES + NAS * AS_BYTES <= BRING_BYTES, "batched rings fit the ring region");
static_assert(NMAX_B * 2 * KSTEP <= WRING_BYTES, "a K step of the widest tile fits the weight ring");
static_assert(2 * 64 * NMAX_B * 4 <= NAS * AS_BYTES, "K-slice staging of two token tiles fits the activation ring");
// one token tile, pushed: the own partial plus (cluster - 1) receive slots of up to 64 / cluster + 1
// rows each (cluster 4; cluster 2 halves the widest tile)
static_assert((64 + 3 * (64 / 4 + 1)) * NMAX_B * 4 <= NAS * AS_BYTES, "pushed K-slice slices fit the activation ring");
static_assert((64 + 1 * (64 / 2 + 1)) * (NMAX_B / 2) * 4 <= NAS * AS_BYTES, "pushed K-slice slices fit the activation ring");
static_assert(2 * NMAX_B <= static_cast<int>(TMEM_COLS), "accumulators of two token tiles fit tensor memory");
// mbarriers in sm.bbar (one expected arrival except BB_SREADY: one per CTA of the cluster, and
// BB_RFREE: one per other CTA of the cluster)
enum : int {
  BB_WFULL = 0,                  // weight entry filled (producer expect_tx + TMA bytes)
  BB_WEMPTY = BB_WFULL + NWE,    // weight entry consumed (tcgen05.commit)
  BB_AFULL = BB_WEMPTY + NWE,    // activation slot filled
  BB_AEMPTY = BB_AFULL + NAS,    // activation slot consumed
  BB_ACCFULL = BB_AEMPTY + NAS,  // D complete (tcgen05.commit after the last K step)
  BB_ACCEMPTY,                   // D read by the consumers
  BB_GO,                         // the stage's grid barrier passed: A planes are complete
  BB_DRAIN,                      // every MMA done (exit)
  BB_SREADY,                     // every CTA of the cluster has staged its K-slice partial (pull)
  BB_RFREE,                      // every other CTA of the cluster may receive this CTA's slices (push)
  BB_RCV,                        // the other CTAs' slices of this CTA's items arrived (push)
  BB_N
};
static_assert(BB_N <= 32, "batched mbarriers");

// The batched kernel's grid barrier as a call of its own: its spin loop then keeps its few values
// in registers rather than sharing the caller's register budget. go_next: the coming stage is a
// GEMM, whose activation loads the barrier itself releases (GO) on the CTAs that take part in
// GEMMs, instead of b_gemm_begin after the consumers' CTA barrier.
__device__ __noinline__ bool grid_sync_b(const Params& p, Smem& sm, Cons& cs) {
  uint64_t* go = (cs.go_next && cs.cta() < BROWS_B) ? &sm.bbar[BB_GO] : nullptr;
  cs.go_sent = cs.go_next;
  cs.go_next = 0;
  return grid_sync(p, sm, cs, go);
}

enum BKind : int { BK_QKV = 0, BK_O = 1, BK_GU = 2, BK_D = 3, BK_HEAD = 4 };

// One GEMM stage: kind, global layer index li (backbone l, code predictor n_bb + l), head index
// (0 = codec head, 1 + g = code-predictor head g) and token count.
struct BGemm {
  int kind, li, hidx, T;
};

__device__ __forceinline__ int bg_K(int kind) { return kind == BK_O ? QSZ : kind == BK_D ? INTER : HID; }
__device__ __forceinline__ int bg_abuf(int kind) { return (kind == BK_QKV || kind == BK_GU) ? 0 : 1; }
__device__ __forceinline__ const uint8_t* bmap(const Params& p, int idx) {
  return p.bmaps + static_cast<size_t>(idx) * TMAP_BYTES;
}
__device__ __forceinline__ int bmap_head(const Params& p, int hidx) { return (p.n_bb + p.n_cp) * NLMAPS + hidx; }
__device__ __forceinline__ int bmap_abuf(const Params& p, int buf, bool box128) {
  return (p.n_bb + p.n_cp) * NLMAPS + 1 + NCPHEADS + 2 * buf + (box128 ? 1 : 0);
}
// Output rows of a stage's weight matrix (gate/up: gate + up rows).
__device__ __forceinline__ int bg_rows(const Params& p, const BGemm& g) {
  switch (g.kind) {
    case BK_QKV: return QKV_ROWS;
    case BK_GU: return 2 * INTER;
    case BK_HEAD: return g.hidx == 0 ? p.vocab : p.cp_vocab;
    default: return HID;
  }
}

// Work of a CTA in a GEMM stage: cluster rt (< R = 128 / bcl) takes row tile rt of N rows (gate/up:
// N/2 gate and N/2 up rows of intermediate channels rt * N/2 ...), and its CTA of rank kspl takes K
// steps [ks0, ks1) of slice kspl; clusters rt >= R have no work in GEMM stages.
struct BSplit {
  int rt, R, N, kspl, nk, ks0, ks1;
  bool act;
};
__device__ __forceinline__ BSplit bg_split(const Params& p, const BGemm& g, int cta) {
  BSplit s;
  s.nk = p.bcl;
  s.R = BROWS / p.bcl;
  s.N = bg_rows(p, g) / s.R;
  s.rt = cta / p.bcl;
  s.kspl = cta - s.rt * p.bcl;
  s.act = s.rt < s.R;
  const int nks = bg_K(g.kind) / KSTEP;
  s.ks0 = split_lo(nks, s.nk, s.kspl);
  s.ks1 = split_lo(nks, s.nk, s.kspl + 1);
  return s;
}

// Weight boxes of a CTA tile: one box of N rows per atom (gate/up: a box of N/2 gate rows and one
// of N/2 up rows; the host encodes every tensor map with its stage's box height and checks that
// the head vocabularies split into full tiles). Returns the tensor map and first row of box i.
__device__ __forceinline__ int bg_nbox(int kind) { return kind == BK_GU ? 2 : 1; }
__device__ __forceinline__ void bg_wbox(const Params& p, const BGemm& g, const BSplit& sp, int i, const uint8_t*& map,
                                        int& y) {
  const int base = g.li * NLMAPS;
  switch (g.kind) {
    case BK_QKV: {   // a tile lies inside one of q (2048 rows), k, v (1024 rows each)
      const int r = sp.rt * sp.N;
      const int m = r < QSZ ? 0 : (r < QSZ + KVSZ ? 1 : 2);
      y = r - (m == 0 ? 0 : (m == 1 ? QSZ : QSZ + KVSZ));
      map = bmap(p, base + m);
      break;
    }
    case BK_O: map = bmap(p, base + 3); y = sp.rt * sp.N; break;
    case BK_GU: map = bmap(p, base + 4 + i); y = sp.rt * (sp.N / 2); break;   // channels of the tile
    case BK_D: map = bmap(p, base + 6); y = sp.rt * sp.N; break;
    default: map = bmap(p, bmap_head(p, g.hidx)); y = sp.rt * sp.N; break;
  }
}

// Weight ring: entries (one K step of the CTA's tile, N * 256 bytes = N / 16 slots) are allocated
// in order and never wrap (an entry that does not fit before the end starts at slot 0); the
// producer and the MMA thread walk the same sequence of entry sizes, so both compute the same slot.
struct WRing {
  uint32_t head;
  __device__ __forceinline__ uint32_t alloc(uint32_t n) {
    if (head + n > static_cast<uint32_t>(NWSLOT)) head = 0;
    const uint32_t f = head;
    head += n;
    return f;
  }
};

// Profiling trace (dbg_marks set): marks[(gemm * BKCTAS + cta) * BT_EVENTS + event] = %globaltimer
// for GEMM stages gemm < dbg_marks_len / (BKCTAS * BT_EVENTS) of the launch, every CTA.
enum BTrace : int {
  BT_START = 0,     // consumers: stage start (GO)
  BT_DREADY,        // consumers: D complete
  BT_STAGED,        // consumers: D staged in shared memory, accumulator freed
  BT_PART,          // consumers: cluster signalled
  BT_COUNT,         // consumers: every K slice of the cluster staged
  BT_REDUCED,       // consumers: slices summed, epilogue done
  BT_EPI,           // consumers: epilogue done (barrier arrival)
  BT_BARRIER,       // consumers: barrier passed
  BT_W0,            // MMA: first weight step ready
  BT_A0,            // MMA: first activation slot ready
  BT_MMA_END,       // MMA: last MMA issued
  BT_GO,            // activation loader: GO seen
  BT_A_END,         // activation loader: last box issued
  BT_P0,            // producer: first weight box issued
  BT_P_END,         // producer: last weight box issued
  BT_LAST,          // MMA: the last K step's weights and activations ready
  BT_ALAST,         // activation loader: last step's slot free (loads issued next)
  BT_S0,            // MMA: first step's MMAs and commits issued
  BT_W1,            // MMA: second step's weights ready
  BT_LO_SEEN,       // consumer warp 2: D complete seen
  BT_LO_DONE,       // consumer warp 2: lo lanes staged
  BT_PH0,           // consumers: lo lanes of every warp staged
  BT_HI_DONE,       // consumer warp 0: hi lanes added
  BT_PH1,           // consumers: hi lanes of every warp added
  BT_EVENTS = 24
};
__device__ __forceinline__ void btrace(const Params& p, int gemm, int cta, int G, int ev) {
  if (p.dbg_marks == nullptr) return;
  (void)G;
  const long long i = (static_cast<long long>(gemm) * BKCTAS + cta) * BT_EVENTS + ev;
  if (i < p.dbg_marks_len) p.dbg_marks[i] = globaltimer_ns();
}

// The GEMM stages of the launch's program, in order, by index (one call site for the role
// loops keeps their code compact): a frame is 15 code-predictor passes of n_cp layers x 4 GEMMs +
// a head, then n_bb backbone layers x 4 + the codec head; a prefill step the n_bb layers; the first
// token the codec head.
__device__ __forceinline__ int b_ngemm(const Params& p) {
  if (p.mode == MODE_B_FRAME) return NCPHEADS * (4 * p.n_cp + 1) + 4 * p.n_bb + 1;
  if (p.mode == MODE_B_PREFILL || p.mode == MODE_B_PREFILL_DENSE) return 4 * p.n_bb;
  return 1;
}
__device__ __forceinline__ BGemm b_gemm_at(const Params& p, int i) {
  const int B = p.mode == MODE_B_PREFILL_DENSE ? p.b_ntok : p.nb;   // tokens of the GEMMs
  if (p.mode == MODE_B_FRAME) {
    const int per = 4 * p.n_cp + 1;
    if (i < NCPHEADS * per) {
      const int g = i / per, r = i - g * per;
      if (r == 4 * p.n_cp) return BGemm{BK_HEAD, 0, 1 + g, B};
      return BGemm{r & 3, p.n_bb + (r >> 2), 0, g == 0 ? 2 * B : B};
    }
    i -= NCPHEADS * per;
  } else if (p.mode != MODE_B_PREFILL && p.mode != MODE_B_PREFILL_DENSE) {
    return BGemm{BK_HEAD, 0, 0, B};
  }
  if (i == 4 * p.n_bb) return BGemm{BK_HEAD, 0, 0, B};
  return BGemm{i & 3, i >> 2, 0, B};
}
static_assert(BK_QKV == 0 && BK_O == 1 && BK_GU == 2 && BK_D == 3, "GEMM kinds in layer order");

// Calls f(gemm index, stage) for every GEMM stage of the launch; f returns false to stop.
template <class F>
__device__ void b_walk(const Params& p, F&& f) {
  const int n = b_ngemm(p);
  for (int i = 0; i < n; ++i)
    if (!f(i, b_gemm_at(p, i))) return;
}

// ------------------------------------------------------------------------------------------
// Producer warp (one thread): weight boxes of every GEMM stage into the weight ring, one entry
// (N rows x two 64-column atoms) per K step.
// ------------------------------------------------------------------------------------------
__device__ __noinline__ void b_producer(const Params& p, Smem& sm, int cta, int G) {
  uint8_t* wring = reinterpret_cast<uint8_t*>(sm.ring);
  WRing ring{0u};
  uint32_t e = 0;                 // entries issued
  uint8_t efirst[NWE], en[NWE];   // slot range of the entries in flight
  int* err = p.w.err;
  auto give_up = [&]() {
    if (!*reinterpret_cast<volatile int*>(&sm.abort)) set_error(err, DEV_ERR_EMPTY_TIMEOUT);
  };
  b_walk(p, [&](int gi, const BGemm& g) -> bool {
    const BSplit sp = bg_split(p, g, cta);
    if (!sp.act) return true;
    const int nbox = bg_nbox(g.kind), brows = sp.N / nbox;
    const uint32_t n = static_cast<uint32_t>(sp.N) / 16u;
    bool first = true;
    for (int ks = sp.ks0; ks < sp.ks1; ++ks, ++e) {
      const uint32_t ei = e % NWE;
      // entry e - NWE (same mbarriers) consumed
      if (!mbar_wait(&sm.bbar[BB_WEMPTY + ei], ((e / NWE) & 1u) ^ 1u, &sm.abort)) {
        give_up();
        return false;
      }
      const uint32_t f = ring.alloc(n);
      // the entries still in flight whose slots overlap [f, f + n)
      for (uint32_t k = (e >= NWE ? e - NWE + 1 : 0u); k < e; ++k) {
        const uint32_t ki = k % NWE;
        if (efirst[ki] < f + n && f < static_cast<uint32_t>(efirst[ki]) + en[ki] &&
            !mbar_wait(&sm.bbar[BB_WEMPTY + ki], (k / NWE) & 1u, &sm.abort)) {
          give_up();
          return false;
        }
      }
      efirst[ei] = static_cast<uint8_t>(f);
      en[ei] = static_cast<uint8_t>(n);
      uint8_t* dst = wring + f * WSLOT;
      mbar_arrive_expect_tx(&sm.bbar[BB_WFULL + ei], static_cast<uint32_t>(sp.N * 2 * 128));
      for (int a = 0; a < NSUB; ++a)
        for (int i = 0; i < nbox; ++i) {
          const uint8_t* map;
          int y;
          bg_wbox(p, g, sp, i, map, y);
          if (first) tensormap_acquire(map);   // the host's copy of the map, before its first use
          tma_load_2d(dst + a * (sp.N * 128) + i * (brows * 128), map, ks * KSTEP + a * KSUB, y,
                      &sm.bbar[BB_WFULL + ei]);
        }
      if (first) btrace(p, gi, cta, G, BT_P0);
      first = false;
    }
    btrace(p, gi, cta, G, BT_P_END);
    return true;
  });
  // drain: no box may still be landing in shared memory when the CTA exits
  int zero = 0;
  for (uint32_t i = (e > NWE ? e - NWE : 0u); i < e; ++i)
    mbar_wait(&sm.bbar[BB_WFULL + i % NWE], (i / NWE) & 1u, &zero);
}

// ------------------------------------------------------------------------------------------
// Activation-loader warp (one thread): after each GEMM stage's grid barrier, the A planes of
// every (K step, 64-token tile) into the 3-slot ring.
// ------------------------------------------------------------------------------------------
__device__ __noinline__ void b_aloader(const Params& p, Smem& sm, int cta, int G) {
  uint8_t* aring = reinterpret_cast<uint8_t*>(sm.ring) + WRING_BYTES;
  uint32_t na = 0, n = 0;
  int* err = p.w.err;
  for (int b = 0; b < 2; ++b) tensormap_acquire(bmap(p, bmap_abuf(p, b, false)));
  b_walk(p, [&](int gi, const BGemm& g) -> bool {
    const BSplit sp = bg_split(p, g, cta);
    if (!sp.act) return true;
    const int ntiles = (g.T + 63) >> 6;
    const uint8_t* amap = bmap(p, bmap_abuf(p, bg_abuf(g.kind), false));
    // the consumers arrive on GO after the stage's grid barrier: the A planes are complete, and
    // every CTA of the cluster has read this CTA's staged partials of the previous stage (which
    // share the ring's space)
    if (!mbar_wait(&sm.bbar[BB_GO], n & 1u, &sm.abort)) {
      if (!*reinterpret_cast<volatile int*>(&sm.abort)) set_error(err, DEV_ERR_FULL_TIMEOUT);
      return false;
    }
    ++n;
    btrace(p, gi, cta, G, BT_GO);
    fence_proxy_async_global();
    for (int ks = sp.ks0; ks < sp.ks1; ++ks)
      for (int j = 0; j < ntiles; ++j, ++na) {
        const uint32_t slot = na % NAS, round = na / NAS;
        if (!mbar_wait(&sm.bbar[BB_AEMPTY + slot], (round & 1u) ^ 1u, &sm.abort)) {
          if (!*reinterpret_cast<volatile int*>(&sm.abort)) set_error(err, DEV_ERR_EMPTY_TIMEOUT);
          return false;
        }
        if (ks == sp.ks1 - 1 && j == ntiles - 1) btrace(p, gi, cta, G, BT_ALAST);
        mbar_arrive_expect_tx(&sm.bbar[BB_AFULL + slot], static_cast<uint32_t>(AS_BYTES));
        for (int a = 0; a < NSUB; ++a) {
          uint8_t* dst = aring + slot * AS_BYTES + a * ASUB_BYTES;
          tma_load_2d(dst, amap, ks * KSTEP + a * KSUB, 64 * j, &sm.bbar[BB_AFULL + slot]);
          tma_load_2d(dst + APLANE_BYTES, amap, ks * KSTEP + a * KSUB, TBMAX + 64 * j, &sm.bbar[BB_AFULL + slot]);
        }
      }
    btrace(p, gi, cta, G, BT_A_END);
    return true;
  });
  int zero = 0;
  for (uint32_t i = (na > NAS ? na - NAS : 0u); i < na; ++i)
    mbar_wait(&sm.bbar[BB_AFULL + i % NAS], (i / NAS) & 1u, &zero);
}

// ------------------------------------------------------------------------------------------
// MMA warp (one thread): tcgen05.mma of every GEMM stage.
// ------------------------------------------------------------------------------------------
__device__ __noinline__ void b_mma(const Params& p, Smem& sm, int cta, int G) {
  const uint32_t wbase = smem_u32(sm.ring), abase = wbase + WRING_BYTES;
  const uint32_t tmem = sm.tmem_base;
  WRing ring{0u};
  uint32_t e = 0, ua = 0, n = 0;
  bool any = false;
  int* err = p.w.err;
  auto fail_mma = [&](int code) {
    if (!*reinterpret_cast<volatile int*>(&sm.abort)) {
      set_error(err, code);
      *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    }
  };
  b_walk(p, [&](int gi, const BGemm& g) -> bool {
    const BSplit sp = bg_split(p, g, cta);
    if (!sp.act) return true;
    const int N = sp.N, nks = sp.ks1 - sp.ks0, ntiles = (g.T + 63) >> 6;
    const uint32_t idesc = umma_idesc_bf16(128, N);
    const uint32_t nslots = static_cast<uint32_t>(N) / 16u;
    // the previous stage's consumers have read D
    if (!mbar_wait(&sm.bbar[BB_ACCEMPTY], (n & 1u) ^ 1u, &sm.abort)) {
      fail_mma(DEV_ERR_FULL_TIMEOUT);
      return false;
    }
    tc_fence_after();
    for (int ks = 0; ks < nks; ++ks, ++e) {   // ks: index within this CTA's K slice
      const uint32_t ei = e % NWE;
      const uint32_t ws = wbase + ring.alloc(nslots) * WSLOT;
      if (!mbar_wait(&sm.bbar[BB_WFULL + ei], (e / NWE) & 1u, &sm.abort)) {
        fail_mma(DEV_ERR_FULL_TIMEOUT);
        return false;
      }
      if (ks == 0) btrace(p, gi, cta, G, BT_W0);
      if (ks == 1) btrace(p, gi, cta, G, BT_W1);
      // descriptors built once per step; a K offset adds (bytes >> 4) to the start-address field
      const uint64_t db0 = umma_desc_sw128(ws), db1 = umma_desc_sw128(ws + static_cast<uint32_t>(N) * 128u);
      for (int j = 0; j < ntiles; ++j, ++ua) {
        const uint32_t as = ua % NAS, ar = ua / NAS;
        if (!mbar_wait(&sm.bbar[BB_AFULL + as], ar & 1u, &sm.abort)) {
          fail_mma(DEV_ERR_FULL_TIMEOUT);
          return false;
        }
        if (ks == 0 && j == 0) btrace(p, gi, cta, G, BT_A0);
        if (ks == nks - 1 && j == ntiles - 1) btrace(p, gi, cta, G, BT_LAST);
        tc_fence_after();
        // one M = 128 MMA per K sub-step over the whole slot: hi rows 0..63 -> TMEM lanes 0..63,
        // lo rows 64..127 -> lanes 64..127, the same weights for both
        const uint64_t da = umma_desc_sw128(abase + as * AS_BYTES);
        const uint32_t dt = tmem + static_cast<uint32_t>(j * N);
#pragma unroll
        for (int a = 0; a < NSUB; ++a)
#pragma unroll
          for (int kk = 0; kk < KSUB / 16; ++kk) {   // the first MMA of the slice overwrites D
            const uint64_t dw = (a == 0 ? db0 : db1) + static_cast<uint64_t>((kk * 32) >> 4);
            tc_mma_bf16(dt, da + static_cast<uint64_t>((a * ASUB_BYTES + kk * 32) >> 4), dw, idesc,
                        (ks | a | kk) != 0 ? 1u : 0u);
          }
        any = true;
        tc_commit(&sm.bbar[BB_AEMPTY + as]);
      }
      tc_commit(&sm.bbar[BB_WEMPTY + ei]);
      if (ks == 0) btrace(p, gi, cta, G, BT_S0);
    }
    btrace(p, gi, cta, G, BT_MMA_END);
    tc_commit(&sm.bbar[BB_ACCFULL]);
    ++n;
    return true;
  });
  if (any) {   // every issued MMA done before the accumulator is freed
    int zero = 0;
    tc_commit(&sm.bbar[BB_DRAIN]);
    mbar_wait(&sm.bbar[BB_DRAIN], 0u, &zero);
  }
}

// ------------------------------------------------------------------------------------------
// Consumers
// ------------------------------------------------------------------------------------------
// Per-utterance state of the launch, copied into shared memory at the start.
struct BState {
  int* pos;    // sm.bstate[0 .. 63]
  int* step;   // [64 .. 127]
  int* g0;     // [128 .. 191]
  int* act;    // [192 .. 255]: 1 = this utterance advances in this launch
};
__device__ __forceinline__ BState bstate(Smem& sm) {
  return BState{sm.bstate, sm.bstate + BMAX, sm.bstate + 2 * BMAX, sm.bstate + 3 * BMAX};
}

__device__ __forceinline__ float b_rstd(const unsigned long long* ssq, int t, float eps) {
  const double s = static_cast<double>(static_cast<long long>(__ldcg(ssq + t))) * (1.0 / 4294967296.0);
  return rms_scale(s, HID, eps);
}

// Epilogue items cover EW consecutive output columns of one token.
constexpr int EW = 8;

// hilo_store of EW consecutive columns (col0 a multiple of EW): one 16-byte store per plane.
__device__ __forceinline__ void hilo_store_w(bf16* buf, int t, int col0, const float (&v)[EW]) {
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bf16 h0 = __float2bfloat16_rn(v[2 * i]), h1 = __float2bfloat16_rn(v[2 * i + 1]);
    const bf16 l0 = __float2bfloat16_rn(v[2 * i] - __bfloat162float(h0));
    const bf16 l1 = __float2bfloat16_rn(v[2 * i + 1] - __bfloat162float(h1));
    hi[i] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
    lo[i] = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
  }
  *reinterpret_cast<uint4*>(buf + static_cast<size_t>(t) * ABUF_LD + col0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4*>(buf + static_cast<size_t>(TBMAX + t) * ABUF_LD + col0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}
// EW consecutive fp32 from global (L2) / bf16 weights as fp32.
__device__ __forceinline__ void ldw_f32(const float* src, float (&v)[EW]) {
#pragma unroll
  for (int i = 0; i < EW; i += 4) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(src + i));
    v[i] = a.x; v[i + 1] = a.y; v[i + 2] = a.z; v[i + 3] = a.w;
  }
}
__device__ __forceinline__ void ldw_bf16(const bf16* src, float (&v)[EW]) {
  const uint4 a = *reinterpret_cast<const uint4*>(src);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf16_lo(w[i]);
    v[2 * i + 1] = bf16_hi(w[i]);
  }
}
__device__ __forceinline__ void stw_f32(float* dst, const float (&v)[EW]) {
#pragma unroll
  for (int i = 0; i < EW; i += 4) __stcg(reinterpret_cast<float4*>(dst + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
}

// Inputs of one epilogue item that do not depend on D.
struct EpiSt {
  float a[EW], b[EW];
  float rs;
  bool valid;    // warp-uniform item loops: the lane holds an item of the CTA
  uint4 w4, c4, s4;   // QKV with the q/k norms: norm weights, RoPE cos / sin of the token's position
  void* kv;      // QKV with the K/V write: the token's row in the cache (nullptr: none)
};

// Consumer side of one GEMM stage. Epilogue items are (token t, EW output columns c); the
// callbacks are pre(t, r0, st) (the item's inputs that do not depend on D) and
// run(t, r0, y, y2, st) with y = D[t][EW columns] (gate/up: y = gate, y2 = up) and r0 the first
// output column (row of W; gate/up: intermediate channel).
//   1. release the activation loader (GO);
//   2. wait for D; the consumer warps copy its lo lanes and then add its hi lanes into the K-slice
//      partial in shared memory; D is freed; every CTA of the cluster is told (mbarrier);
//   3. once the cluster's partials are staged, each item sums them in rank order (distributed
//      shared memory), then its epilogue; the grid barrier.
// Steps 1-2 and the barrier are shared code (b_gemm_begin / b_gemm_mid / b_gemm_end): the stage
// kinds differ only in the item callbacks, so the kernel keeps one copy of the pipeline.
struct BStage {
  BSplit sp;
  int gi, N, NO, nci, i0, i1, r0b, T, smask;
  bool gu;
  bool push;         // one token tile: partial slices pushed to their owners by bulk copies
  int ra, rb;        // push: partial rows (tokens) [ra, rb) holding this CTA's items
  uint32_t s_addr;   // shared address of the K-slice partial [tile][64][N] fp32 (swizzled chunks)
  uint32_t r_addr;   // push: receive slots, one per other CTA of the cluster [rb - ra][N] fp32
};

// Partial rows (tokens) holding the epilogue items of cluster rank r: [*ra, *rb). The ranks split
// the tokens, so that all items of a token (a whole head row of QKV) are one CTA's.
__device__ __forceinline__ void b_rows_of(const BStage& S, int r, int& ra, int& rb) {
  ra = split_lo(S.T, S.sp.nk, r);
  rb = split_lo(S.T, S.sp.nk, r + 1);
}

// Partial staging layout: row (token tile j, token t) of N floats holding lo + hi; 16-byte chunk k
// of the row is stored at chunk k ^ (t & smask), so that the lanes of a warp (one token each) hit
// different banks. The hi and lo products are summed here, before the exchange, so that the other
// CTAs of the cluster read one plane: when every SM of the cluster reads at once, distributed
// shared memory moves only ~7 bytes per clock per SM, and the exchange is bound by it.
__device__ __forceinline__ uint32_t b_part_off(const BStage& S, int j, int t, int k) {
  return static_cast<uint32_t>(((j * 64 + t) * S.N + 4 * (k ^ (t & S.smask))) * 4);
}

// Step 1: the stage's tiling (returned by value, so that it stays in registers) and the GO arrival.
__device__ __forceinline__ BStage b_gemm_begin(const Params& p, Smem& sm, Cons& cs, const BGemm& g) {
  BStage S;
  S.sp = bg_split(p, g, cs.cta());
  S.gi = cs.gi;
  cs.gi++;
  S.T = g.T;
  S.N = S.sp.N;
  S.gu = g.kind == BK_GU;
  S.NO = S.gu ? S.N / 2 : S.N;
  S.nci = S.NO / EW;
  S.i0 = S.nci * split_lo(g.T, S.sp.nk, S.sp.kspl);
  S.i1 = S.nci * split_lo(g.T, S.sp.nk, S.sp.kspl + 1);
  S.r0b = S.sp.rt * S.NO;
  S.smask = (S.N / 4) % 8 == 0 ? 7 : 3;
  S.s_addr = smem_u32(sm.ring) + WRING_BYTES;
  S.push = g.T <= 64;
  b_rows_of(S, S.sp.kspl, S.ra, S.rb);
  S.r_addr = S.s_addr + static_cast<uint32_t>(64 * S.N * 4);
  if (S.sp.act) {
    if (p.dbg_marks != nullptr && cs.tid() == 0) btrace(p, S.gi, cs.cta(), cs.G(), BT_START);
    if (cs.tid() == 0) {
      // armed before this CTA frees its receive slots (after its MMAs), so before any slice lands
      if (S.push)
        mbar_arrive_expect_tx(&sm.bbar[BB_RCV], static_cast<uint32_t>((S.sp.nk - 1) * (S.rb - S.ra) * S.N * 4));
      if (!cs.go_sent) mbar_arrive(&sm.bbar[BB_GO]);
    }
  }
  cs.go_sent = 0;
  return S;
}

// Consumer-wide wait for an mbarrier phase: thread 0 polls, the other consumer threads wait at the
// CTA barrier, so that 384 threads do not poll the mbarrier unit while the loader's and the MMA
// thread's mbarriers are busy. Thread 0's acquire and the CTA barrier order the phase's data
// before every consumer's later reads.
__device__ __forceinline__ bool b_cons_wait(const Params& p, Smem& sm, Cons& cs, uint64_t* bar, uint32_t parity,
                                            bool cluster, int code) {
  if (cs.tid() == 0) {
    const bool ok = cluster ? mbar_wait_cluster(bar, parity, &sm.abort) : mbar_wait(bar, parity, &sm.abort);
    if (!ok && !aborted(sm)) fail(p, sm, code);
  }
  named_sync(1, NCT);
  return !aborted(sm);
}

// Step 2 up to the cluster's partials being staged; false on abort.
__device__ __noinline__ bool b_gemm_mid(const Params& p, Smem& sm, Cons& cs, const BStage S, uint32_t gemm_n) {
  const bool tr = p.dbg_marks != nullptr && cs.tid() == 0;
  if (!b_cons_wait(p, sm, cs, &sm.bbar[BB_ACCFULL], gemm_n & 1u, false, DEV_ERR_FULL_TIMEOUT)) return false;
  const bool tr2 = p.dbg_marks != nullptr && cs.tid() == 64;   // warp 2 (lo lanes), lane 0
  if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_DREADY);
  // push: the MMAs have read this CTA's activation ring, where the other CTAs' slices land; the
  // warp barrier orders thread 0's arming of BB_RCV before these arrivals
  if (S.push && cs.warp() == 0) {
    __syncwarp();
    if (cs.tid() < S.sp.nk && cs.tid() != S.sp.kspl)
      mbar_arrive_cluster(mapa_shared(smem_u32(&sm.bbar[BB_RFREE]), static_cast<uint32_t>(cs.tid())));
  }
  if (tr2) btrace(p, S.gi, cs.cta(), cs.G(), BT_LO_SEEN);
  tc_fence_after();
  // D -> partial: TMEM lane quarter q of warp w (w % 4) holds tokens 32 (q & 1) .. of the hi
  // (q < 2) or lo (q >= 2) products. The lo quarters store first, then the hi quarters add (the
  // same order for every element).
  const int ntiles = (S.T + 63) >> 6, nch = S.N / 16;
  const int q = cs.warp() & 3, wq = cs.warp() >> 2;
  uint8_t* sbase = reinterpret_cast<uint8_t*>(sm.ring) + WRING_BYTES;
  for (int phase = 0; phase < 2; ++phase) {
    if ((q >= 2) == (phase == 0)) {
      for (int job = wq; job < ntiles * nch; job += NCW / 4) {
        const int j = job / nch, c = job - j * nch;
        if (64 * j + 32 * (q & 1) < S.T) {   // warp-uniform: tcgen05.ld is a warp-wide instruction
          float v[16];
          tmem_ld16(sm.tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(j * S.N + 16 * c), v);
          const int t = 32 * (q & 1) + cs.lane();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float4* d = reinterpret_cast<float4*>(sbase + b_part_off(S, j, t, 4 * c + i));
            if (phase == 1) {
              const float4 lo = *d;
              *d = make_float4(lo.x + v[4 * i], lo.y + v[4 * i + 1], lo.z + v[4 * i + 2], lo.w + v[4 * i + 3]);
            } else {
              *d = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
          }
        }
      }
    }
    if (tr2 && phase == 0) btrace(p, S.gi, cs.cta(), cs.G(), BT_LO_DONE);
    if (tr && phase == 1) btrace(p, S.gi, cs.cta(), cs.G(), BT_HI_DONE);
    if (phase == 0) named_sync(1, NCT);
    if (tr && phase == 0) btrace(p, S.gi, cs.cta(), cs.G(), BT_PH0);
  }
  tc_fence_before();
  if (S.push) {
    // the partial's generic stores are read by the bulk copies (async proxy) after the CTA barrier
    fence_proxy_async_smem();
    named_sync(1, NCT);
    if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_PH1);
    if (cs.tid() == 0) {
      mbar_arrive(&sm.bbar[BB_ACCEMPTY]);   // D is no longer needed
      if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_STAGED);
    }
    const int d = cs.tid();
    if (d < S.sp.nk && d != S.sp.kspl) {
      // lane d: the rows of rank d's items, into its receive slot of this CTA, once rank d's MMAs
      // are done
      if (!mbar_wait_cluster(&sm.bbar[BB_RFREE], static_cast<uint32_t>(cs.pn) & 1u, &sm.abort)) {
        if (!aborted(sm)) fail(p, sm, DEV_ERR_GRID_TIMEOUT);
      } else {
        int ra, rb;
        b_rows_of(S, d, ra, rb);
        const uint32_t row_bytes = static_cast<uint32_t>(S.N * 4), slot_bytes = static_cast<uint32_t>(rb - ra) * row_bytes;
        const uint32_t sidx = static_cast<uint32_t>(S.sp.kspl < d ? S.sp.kspl : S.sp.kspl - 1);
        if (slot_bytes != 0u)
          bulk_s2cluster(mapa_shared(S.r_addr + sidx * slot_bytes, static_cast<uint32_t>(d)),
                         S.s_addr + static_cast<uint32_t>(ra) * row_bytes, slot_bytes,
                         mapa_shared(smem_u32(&sm.bbar[BB_RCV]), static_cast<uint32_t>(d)));
      }
      if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_PART);
    }
    // the other CTAs' slices of this CTA's items
    if (!b_cons_wait(p, sm, cs, &sm.bbar[BB_RCV], static_cast<uint32_t>(cs.pn) & 1u, true, DEV_ERR_GRID_TIMEOUT))
      return false;
    cs.pn++;
    if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_COUNT);
    return true;
  }
  // pull: the CTA barrier orders every thread's partial stores before the lanes whose release
  // arrivals (cluster scope, cumulative) publish them to the cluster's readers
  named_sync(1, NCT);
  if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_PH1);
  if (cs.tid() < S.sp.nk) {
    if (cs.tid() == 0) {
      mbar_arrive(&sm.bbar[BB_ACCEMPTY]);   // D is no longer needed
      if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_STAGED);
    }
    // lane r signals rank r: the ranks' release arrivals go out together instead of one after
    // another
    mbar_arrive_cluster(mapa_shared(smem_u32(&sm.bbar[BB_SREADY]), static_cast<uint32_t>(cs.tid())));
    if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_PART);
  }
  // every CTA of the cluster has staged its partial of this stage
  if (!b_cons_wait(p, sm, cs, &sm.bbar[BB_SREADY], gemm_n & 1u, true, DEV_ERR_GRID_TIMEOUT)) return false;
  if (tr) btrace(p, S.gi, cs.cta(), cs.G(), BT_COUNT);
  return true;
}

// Partial of the CTA of the cluster at `base` (its cluster address) for chunks k0, k0 + 1 of token
// tt of tile j.
__device__ __forceinline__ void b_part2(const BStage& S, uint32_t base, int j, int tt, int k0, float4 (&a)[2]) {
  a[0] = ld_dsmem_f4(base + b_part_off(S, j, tt, k0));
  a[1] = ld_dsmem_f4(base + b_part_off(S, j, tt, k0 + 1));
}
__device__ __forceinline__ void b_acc8(float (&y)[EW], const float4 (&a)[2]) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    y[4 * i] += a[i].x; y[4 * i + 1] += a[i].y; y[4 * i + 2] += a[i].z; y[4 * i + 3] += a[i].w;
  }
}

// Sum of the cluster's K-slice partials (each lo + hi) of item (t, EW columns from chunk 2c) in
// rank order (y; gate/up: y2 = the matching up columns). NK ranks: every rank's loads are issued
// before the first add, so the item waits for one distributed-shared-memory round trip, not NK.
template <int NK>
__device__ __forceinline__ void b_sum_ranks(const BStage& S, int j, int tt, int k0, float (&y)[EW]) {
  float4 a[NK][2];
#pragma unroll
  for (int r = 0; r < NK; ++r) b_part2(S, mapa_shared(S.s_addr, static_cast<uint32_t>(r)), j, tt, k0, a[r]);
#pragma unroll
  for (int i = 0; i < EW; ++i) y[i] = 0.f;
#pragma unroll
  for (int r = 0; r < NK; ++r) b_acc8(y, a[r]);
}
// The same sum when the slices were pushed: this CTA's own partial and the received slices, all
// in this CTA's shared memory, in rank order.
template <int NK>
__device__ __forceinline__ void b_sum_ranks_pushed(const BStage& S, int t, int k0, float (&y)[EW]) {
  const uint32_t slot = static_cast<uint32_t>((S.rb - S.ra) * S.N * 4);
  const int sw = t & S.smask;
  float4 a[NK][2];
#pragma unroll
  for (int r = 0; r < NK; ++r) {
    const bool own = r == S.sp.kspl;
    const uint32_t base = own ? S.s_addr : S.r_addr + static_cast<uint32_t>(r < S.sp.kspl ? r : r - 1) * slot;
    const int row = own ? t : t - S.ra;
    a[r][0] = ld_smem_f4(base + static_cast<uint32_t>((row * S.N + 4 * (k0 ^ sw)) * 4));
    a[r][1] = ld_smem_f4(base + static_cast<uint32_t>((row * S.N + 4 * ((k0 + 1) ^ sw)) * 4));
  }
#pragma unroll
  for (int i = 0; i < EW; ++i) y[i] = 0.f;
#pragma unroll
  for (int r = 0; r < NK; ++r) b_acc8(y, a[r]);
}

__device__ __forceinline__ void b_reduce_item(const BStage& S, int t, int c, float (&y)[EW], float (&y2)[EW]) {
  const int tt = t & 63, j = t >> 6;
  if (S.push) {
    if (S.sp.nk == 4) {
      b_sum_ranks_pushed<4>(S, t, 2 * c, y);
      if (S.gu) b_sum_ranks_pushed<4>(S, t, S.NO / 4 + 2 * c, y2);
    } else {
      b_sum_ranks_pushed<2>(S, t, 2 * c, y);
      if (S.gu) b_sum_ranks_pushed<2>(S, t, S.NO / 4 + 2 * c, y2);
    }
    return;
  }
  if (S.sp.nk == 4) {
    b_sum_ranks<4>(S, j, tt, 2 * c, y);
    if (S.gu) b_sum_ranks<4>(S, j, tt, S.NO / 4 + 2 * c, y2);
  } else {
    b_sum_ranks<2>(S, j, tt, 2 * c, y);
    if (S.gu) b_sum_ranks<2>(S, j, tt, S.NO / 4 + 2 * c, y2);
  }
}

__device__ __forceinline__ bool b_gemm_end(const Params& p, Smem& sm, Cons& cs, int gi, bool planes) {
  fence_proxy_async_smem();   // the partials alias the activation ring: before the next stage's TMA writes
  if (planes) fence_proxy_async_global();   // the epilogue wrote the next GEMM's operand planes
  if (p.dbg_marks != nullptr && cs.tid() == 0) btrace(p, gi, cs.cta(), cs.G(), BT_EPI);
  const bool ok = grid_sync_b(p, sm, cs);
  if (p.dbg_marks != nullptr && cs.tid() == 0) btrace(p, gi, cs.cta(), cs.G(), BT_BARRIER);
  return ok;
}

// go_after: a GEMM stage follows this one's grid barrier directly.
// UNIFORM: every lane of a warp runs the same trip count (lane l of the warp's 32 consecutive items,
// st.valid false past the CTA's last item), so that run() may shuffle across the lanes of a token.
template <bool UNIFORM = false, class PRE, class RUN>
__device__ __forceinline__ bool b_gemm(const Params& p, Smem& sm, Cons& cs, const BGemm& g, uint32_t& gemm_n, bool go_after,
                                       PRE&& pre, RUN&& run) {
  const BStage S = b_gemm_begin(p, sm, cs, g);
  cs.go_next = go_after ? 1 : 0;
  if (!S.sp.act) return grid_sync_b(p, sm, cs);
  const bool ok = b_gemm_mid(p, sm, cs, S, gemm_n);
  if (ok) {
    for (int ib = S.i0 + (UNIFORM ? (cs.tid() & ~31) : cs.tid()); ib < S.i1; ib += NCT) {
      const int iu = ib + (UNIFORM ? cs.lane() : 0);
      const bool valid = iu < S.i1;
      const int i = valid ? iu : S.i0;   // a stand-in item of this CTA past the end
      const int t = i / S.nci, c = i - t * S.nci, r0 = S.r0b + EW * c;
      // the item's inputs that do not depend on D first: their L2 loads overlap the partials'
      // distributed shared memory loads
      EpiSt st;
      st.valid = valid;
      pre(t, r0, st);
      float y[EW], y2[EW];
      b_reduce_item(S, t, c, y, y2);
      run(t, r0, y, y2, st);
    }
  }
  if (p.dbg_marks != nullptr && cs.tid() == 0) btrace(p, S.gi, cs.cta(), cs.G(), BT_REDUCED);
  const bool ok2 = b_gemm_end(p, sm, cs, S.gi, g.kind == BK_O || g.kind == BK_GU || g.kind == BK_D);
  gemm_n++;
  return ok && ok2;
}

// Sums-of-squares buffer written by the next producing stage (INPUT, O, down); that stage also
// clears the buffer after it, last read two producing stages earlier. The host clears all three
// before every launch.
__device__ __forceinline__ unsigned long long* b_ssq_next(const Params& p, Cons& cs) {
  cs.dk = (cs.dk + 1) % 3;
  unsigned long long* w = p.bw.ssq + cs.dk * TBMAX;
  if (cs.cta() == 0)
    for (int t = cs.tid(); t < TBMAX; t += NCT) __stcg(p.bw.ssq + ((cs.dk + 1) % 3) * TBMAX + t, 0ull);
  return w;
}
__device__ __forceinline__ const unsigned long long* b_ssq_cur(const Params& p, const Cons& cs) {
  return p.bw.ssq + cs.dk * TBMAX;
}
__device__ __forceinline__ void b_ssq_add(unsigned long long* ssq, int t, double ss) {
  atomicAdd(ssq + t, static_cast<unsigned long long>(__double2ll_rn(ss * 4294967296.0)));
}

// End of a stage whose generic-proxy stores (a GEMM operand's hi/lo planes) are read by TMA
// (the async proxy) after the barrier: every writer orders its stores for that proxy first.
__device__ __forceinline__ bool b_sync_planes(const Params& p, Smem& sm, Cons& cs) {
  fence_proxy_async_global();
  fence_proxy_async_smem();   // attention staged rows in the activation ring: before its next TMA writes
  return grid_sync_b(p, sm, cs);
}

// Elementwise stages over T tokens x HID columns: CTA c owns 8-column units
// [split_lo(128, G, c), split_lo(128, G, c + 1)); one thread per (token, unit).
template <class F>
__device__ void b_elementwise(Cons& cs, int T, F&& f) {
  const int u0 = split_lo(HID / 8, cs.G(), cs.cta()), u1 = split_lo(HID / 8, cs.G(), cs.cta() + 1);
  const int nu = u1 - u0;
  for (int e = cs.tid(); e < T * nu; e += NCT) {
    const int t = e / nu, u = u0 + e - t * nu;
    f(t, 8 * u);
  }
}

// INPUT / COMBINE: stack input x (fp32), its A planes scaled by the first layer's input norm
// weights, and its sums of squares. src(t, k0, v[8]) fills 8 consecutive columns.
template <class SRC>
__device__ bool b_input(const Params& p, Smem& sm, Cons& cs, int T, const bf16* norm_w, SRC&& src) {
  unsigned long long* ssq = b_ssq_next(p, cs);
  b_elementwise(cs, T, [&](int t, int k0) {
    float v[8];
    src(t, k0, v);
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      __stcg(p.bw.x + t * HID + k0 + i, v[i]);
      hilo_store(p.bw.abuf[0], t, k0 + i, v[i] * __bfloat162float(norm_w[k0 + i]));
      ss = fma(static_cast<double>(v[i]), static_cast<double>(v[i]), ss);
    }
    b_ssq_add(ssq, t, ss);
  });
  cs.go_next = 1;   // the stack's first QKV follows
  return b_sync_planes(p, sm, cs);
}

// NORM: head input A = bf16(RMSNorm(h)) (lo plane 0) for head tokens i < B taken from stack
// token tmul * i + toff; hstate (backbone): the fp32 normed hidden of each active utterance.
__device__ __noinline__ bool b_norm(const Params& p, Smem& sm, Cons& cs, const float* h, int tmul, int toff, const bf16* w,
                       bool hstate) {
  const unsigned long long* ssq = b_ssq_cur(p, cs);
  const BState bst = bstate(sm);
  b_elementwise(cs, p.nb, [&](int i, int k0) {
    const int t = tmul * i + toff;
    const float rs = b_rstd(ssq, t, p.eps);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float nv = __ldcg(h + t * HID + k0 + j) * rs * __bfloat162float(w[k0 + j]);
      p.bw.abuf[1][static_cast<size_t>(i) * ABUF_LD + k0 + j] = __float2bfloat16_rn(nv);
      p.bw.abuf[1][static_cast<size_t>(TBMAX + i) * ABUF_LD + k0 + j] = __float2bfloat16_rn(0.f);
      if (hstate && bst.act[i]) p.bs[i].st->h[k0 + j] = nv;
    }
  });
  cs.go_next = 1;   // a head follows
  return b_sync_planes(p, sm, cs);
}

// ------------------------------------------------------------------------------------------
// Attention as warp work items. A warp owns one (utterance, KV head, chunk of context
// positions) item; its lanes are WG = 2 position groups of WL = 16 lanes, lane (g, u) holding
// the head dimensions [8u, 8u + 8) of positions g, g + 2, g + 4, ... of the chunk, so one warp
// load reads 2 whole cached rows and a score needs 4 shuffles. Both q heads of the KV head
// (GQA 2:1) are done together; each position group keeps an online softmax, the groups are
// merged with shuffles at the end, and the result is either the output (single chunk) or a
// partial record merged by the head's last chunk to finish (counter), as in flash decoding.
// ------------------------------------------------------------------------------------------
constexpr unsigned WFULL = 0xffffffffu;
constexpr int WD = 8;          // head dimensions per lane
constexpr int WL = HD / WD;    // lanes per position
constexpr int WG = 32 / WL;    // position groups per warp
static_assert(WL == 16 && WG == 2, "warp attention layout");

__device__ __forceinline__ float bf16_at(const uint32_t* w, int i) { return (i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]); }

// q/k RMSNorm (fused_decode_tts.cu:183-197) + RoPE on the dimensions [8u, 8u + 8) in x, with
// the norm weights w4 and the position's cos / sin rows c4 / s4 (bf16, already loaded); the
// rotation partner d +- 64 is in lane u ^ 8 of the same group.
__device__ __forceinline__ void w_norm_rope(float (&x)[WD], uint4 w4, uint4 c4, uint4 s4, float eps, int u) {
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < WD; ++i) ss = fma(static_cast<double>(x[i]), static_cast<double>(x[i]), ss);
#pragma unroll
  for (int o = 1; o < WL; o <<= 1) ss += __shfl_xor_sync(WFULL, ss, o);
  const float rstd = rms_scale(ss, HD, eps);
  const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
  for (int i = 0; i < WD; ++i) x[i] = x[i] * rstd * bf16_at(w, i);
  const uint32_t c[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
  float y[WD];
#pragma unroll
  for (int i = 0; i < WD; ++i) y[i] = __shfl_xor_sync(WFULL, x[i], WL / 2);
#pragma unroll
  for (int i = 0; i < WD; ++i)
    x[i] = u < WL / 2 ? x[i] * bf16_at(c, i) - y[i] * bf16_at(sn, i) : x[i] * bf16_at(c, i) + y[i] * bf16_at(sn, i);
}

// Dimensions [8u, 8u + 8) of cached row j: 4 words of packed bf16 pairs (backbone) or 8 fp32
// words (code predictor).
template <bool CP>
struct WRow {
  uint32_t w[CP ? 8 : 4];
  __device__ __forceinline__ void load(const uint8_t* base, int j, int u) {
    const uint4* r = reinterpret_cast<const uint4*>(base + static_cast<size_t>(j) * HD * (CP ? 4 : 2)) + (CP ? 2 : 1) * u;
#pragma unroll
    for (int i = 0; i < (CP ? 2 : 1); ++i) {
      // code-predictor rows were written by other CTAs earlier in this launch: read through L2
      const uint4 a = CP ? __ldcg(r + i) : __ldcs(r + i);
      w[4 * i] = a.x; w[4 * i + 1] = a.y; w[4 * i + 2] = a.z; w[4 * i + 3] = a.w;
    }
  }
  __device__ __forceinline__ float operator[](int i) const { return CP ? __uint_as_float(w[i]) : bf16_at(w, i); }
};

// Online softmax state of one q head on this lane's dimensions.
struct WSoft {
  float m, l, acc[WD];
  __device__ __forceinline__ void init() {
    m = -INFINITY;
    l = 0.f;
#pragma unroll
    for (int i = 0; i < WD; ++i) acc[i] = 0.f;
  }
  // the P scores s[q] (valid where ok[q]) of one trip with one running-max update
  template <int P, class V>
  __device__ __forceinline__ void add_trip(const float (&s)[P], const bool (&ok)[P], const V (&v)[P]) {
    float mt = -INFINITY;
#pragma unroll
    for (int q = 0; q < P; ++q)
      if (ok[q]) mt = fmaxf(mt, s[q]);
    const float mn = fmaxf(m, mt);
    if (mn == -INFINITY) return;
    const float f = m == -INFINITY ? 0.f : expf(m - mn);
    l *= f;
#pragma unroll
    for (int i = 0; i < WD; ++i) acc[i] *= f;
#pragma unroll
    for (int q = 0; q < P; ++q)
      if (ok[q]) {
        const float e = expf(s[q] - mn);
        l += e;
#pragma unroll
        for (int i = 0; i < WD; ++i) acc[i] = fmaf(e, v[q][i], acc[i]);
      }
    m = mn;
  }
  // merge with another state (m2, l2, a2)
  __device__ __forceinline__ void merge(float m2, float l2, const float (&a2)[WD]) {
    const float mn = fmaxf(m, m2);
    if (mn == -INFINITY) return;
    const float f = m == -INFINITY ? 0.f : expf(m - mn), f2 = m2 == -INFINITY ? 0.f : expf(m2 - mn);
    l = l * f + l2 * f2;
#pragma unroll
    for (int i = 0; i < WD; ++i) acc[i] = acc[i] * f + a2[i] * f2;
    m = mn;
  }
  // merge the position groups of the warp (lanes u and u + 16); every lane takes part
  __device__ __forceinline__ void merge_groups() {
    const float m2 = __shfl_xor_sync(WFULL, m, WL), l2 = __shfl_xor_sync(WFULL, l, WL);
    const float mn = fmaxf(m, m2);
    const float f = m == -INFINITY ? 0.f : expf(m - mn), f2 = m2 == -INFINITY ? 0.f : expf(m2 - mn);
    l = l * f + l2 * f2;
#pragma unroll
    for (int i = 0; i < WD; ++i) acc[i] = acc[i] * f + __shfl_xor_sync(WFULL, acc[i], WL) * f2;
    m = mn;
  }
};

// 8 fp32 from global memory through L2 (rows written by other CTAs in this launch).
__device__ __forceinline__ void ld8_f32(const float* src, float (&v)[WD]) {
  const float4 a = __ldcg(reinterpret_cast<const float4*>(src)), b = __ldcg(reinterpret_cast<const float4*>(src) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Normalised output of q head g (0: a0, 1: a1) on this lane's 8 dimensions as hi/lo planes.
__device__ __forceinline__ void w_out(bf16* hilo, int tok, int col0, const WSoft& a0, const WSoft& a1, int g) {
  const float inv = 1.f / (g == 0 ? a0.l : a1.l);
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float v0 = (g == 0 ? a0.acc[2 * i] : a1.acc[2 * i]) * inv;
    const float v1 = (g == 0 ? a0.acc[2 * i + 1] : a1.acc[2 * i + 1]) * inv;
    const bf16 h0 = __float2bfloat16_rn(v0), h1 = __float2bfloat16_rn(v1);
    const bf16 l0 = __float2bfloat16_rn(v0 - __bfloat162float(h0)), l1 = __float2bfloat16_rn(v1 - __bfloat162float(h1));
    hi[i] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
    lo[i] = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
  }
  *reinterpret_cast<uint4*>(hilo + static_cast<size_t>(tok) * ABUF_LD + col0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4*>(hilo + static_cast<size_t>(TBMAX + tok) * ABUF_LD + col0) =
      make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Backbone items of one token: the cached rows [s0, ce) pass through this warp's WBUF bytes of
// the activation ring (idle between GEMM stages) in sub-chunks of WSC positions, double-buffered
// with cp.async, so that a warp keeps 8 KB of K/V rows in flight instead of the 4 KB its
// registers hold (the stage is bound by bytes in flight from HBM). Group g takes rows g, g + 2,
// g + 4, g + 6 of each sub-chunk, as in the register loop.
constexpr int WSC = 8;                          // positions per sub-chunk
constexpr int WSUB = 2 * WSC * HD * 2;          // K and V rows of one sub-chunk (bf16): 4 KB
constexpr int WBUF = 2 * WSUB;                  // two sub-chunks in flight
static_assert(NCW * WBUF <= NAS * AS_BYTES, "attention staging fits the activation ring");
// Code-predictor items of one token: the warps 0..3 of every CTA take one item each (512 items on
// 132 CTAs) and stage all of its <= 16 cached fp32 rows in 24 KB of the activation ring with one
// round of cp.async.
constexpr int CPWBUF = 24 * 1024;
constexpr int CPW_ROWS = CPWBUF / 2 / (HD * 4);   // 24 rows of K, then 24 of V
static_assert(4 * CPWBUF <= NAS * AS_BYTES && CPW_ROWS >= 16, "code-predictor attention staging fits the activation ring");
__device__ __forceinline__ void w_stage_sub(uint8_t* dst, const uint8_t* kb, const uint8_t* vb, int j0, int n, int lane,
                                            uint64_t pol) {
  const int pieces = n * (HD * 2 / 16);
  const size_t off = static_cast<size_t>(j0) * HD * 2;
  for (int e = lane; e < pieces; e += 32) {
    cp_async16_stream(dst + e * 16, kb + off + e * 16, pol);
    cp_async16_stream(dst + WSUB / 2 + e * 16, vb + off + e * 16, pol);
  }
  cp_async_commit();
}
__device__ __forceinline__ void w_scores4(const float (&q0)[WD], const float (&q1)[WD], const WRow<false> (&kr)[4],
                                          float scale, float (&d0)[4], float (&d1)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    d0[q] = 0.f;
    d1[q] = 0.f;
#pragma unroll
    for (int i = 0; i < WD; ++i) {
      d0[q] = fmaf(q0[i], kr[q][i], d0[q]);
      d1[q] = fmaf(q1[i], kr[q][i], d1[q]);
    }
  }
#pragma unroll
  for (int o = 1; o < WL; o <<= 1)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      d0[q] += __shfl_xor_sync(WFULL, d0[q], o);
      d1[q] += __shfl_xor_sync(WFULL, d1[q], o);
    }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    d0[q] *= scale;
    d1[q] *= scale;
  }
}
// The first two sub-chunks of a backbone item (issued once the item's q/k/v loads have returned).
__device__ __forceinline__ void w_stage_first(const uint8_t* kb, const uint8_t* vb, int s0, int ce, uint8_t* wbuf, int lane) {
  const uint64_t pol = l2_evict_first_policy();
  const int nsc = (ce - s0 + WSC - 1) / WSC;
  if (nsc > 0) w_stage_sub(wbuf, kb, vb, s0, min(WSC, ce - s0), lane, pol);
  if (nsc > 1) w_stage_sub(wbuf + WSUB, kb, vb, s0 + WSC, min(WSC, ce - s0 - WSC), lane, pol);
}
__device__ __forceinline__ void w_loop_staged(const uint8_t* kb, const uint8_t* vb, int s0, int ce, uint8_t* wbuf,
                                              const float (&q0)[WD], const float (&q1)[WD], float scale, int lane,
                                              WSoft& a0, WSoft& a1) {
  const int g = lane / WL, u = lane % WL;
  const uint64_t pol = l2_evict_first_policy();
  const int nsc = (ce - s0 + WSC - 1) / WSC;
  for (int i = 0; i < nsc; ++i) {
    if (i + 1 < nsc)
      cp_async_wait<1>();
    else
      cp_async_wait<0>();
    __syncwarp();   // every lane's copies of sub-chunk i have landed
    const uint8_t* b = wbuf + (i & 1) * WSUB;
    const int n = min(WSC, ce - s0 - i * WSC);
    bool ok[4];
    WRow<false> kr[4], vr[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int r = g + 2 * q;
      ok[q] = r < n;
      const uint4 k4 = *reinterpret_cast<const uint4*>(b + (ok[q] ? r : 0) * HD * 2 + 16 * u);
      const uint4 v4 = *reinterpret_cast<const uint4*>(b + WSUB / 2 + (ok[q] ? r : 0) * HD * 2 + 16 * u);
      kr[q].w[0] = k4.x; kr[q].w[1] = k4.y; kr[q].w[2] = k4.z; kr[q].w[3] = k4.w;
      vr[q].w[0] = v4.x; vr[q].w[1] = v4.y; vr[q].w[2] = v4.z; vr[q].w[3] = v4.w;
    }
    float d0[4], d1[4];
    w_scores4(q0, q1, kr, scale, d0, d1);
    a0.add_trip(d0, ok, vr);
    a1.add_trip(d1, ok, vr);
    __syncwarp();   // sub-chunk i read by every lane before its buffer is refilled
    if (i + 2 < nsc) w_stage_sub(wbuf + (i & 1) * WSUB, kb, vb, s0 + (i + 2) * WSC, min(WSC, ce - s0 - (i + 2) * WSC), lane, pol);
  }
}

// One warp item: tokens t < NT of utterance rows qkv + t * QKV_ROWS at positions p0 + t, KV
// head h, context positions [s0, s1) (chunk c of nch). writer: the item's range ends at the
// tokens' own positions. With p.kv_pre the QKV epilogue has normed q and written the new K/V rows,
// so every position is read from the cache; otherwise the writer item applies the q/k norms and
// RoPE, stores the new rows and takes them from registers.
template <bool CP>
__device__ __noinline__ void watt_item(const Params& p, const Cons& cs, const LayerW* L, const float* qkv, int NT, int p0, int h,
                          uint8_t* kb, uint8_t* vb, bf16* hilo, int tok0, int c, int nch, int s0, int s1,
                          bool writer, float* prt, uint32_t* cnt, uint8_t* wbuf) {
  const int g = cs.lane() / WL, u = cs.lane() % WL;
  // own: the item applies the q/k norms + RoPE and writes the new K/V row itself, then takes that
  // row from registers; with p.kv_pre the QKV epilogue did both, q is normed and every row,
  // the new one included, is read from the cache
  const bool own = writer && !p.kv_pre;
  const int nown = own ? 1 : 0;   // trailing rows of the range taken from registers
  const bool staged = !CP && wbuf != nullptr && NT == 1;
  const bool staged_cp = CP && wbuf != nullptr && NT == 1 && writer && p0 + 1 - nown - s0 <= CPW_ROWS;
  if (staged_cp) {   // cached rows [s0, p0 + 1 - nown), before the item's q loads
    const int pieces = (p0 + 1 - nown - s0) * (HD * 4 / 16);
    const size_t off = static_cast<size_t>(s0) * HD * 4;
    for (int e = cs.lane(); e < pieces; e += 32) {
      cp_async16(wbuf + e * 16, kb + off + e * 16);
      cp_async16(wbuf + CPWBUF / 2 + e * 16, vb + off + e * 16);
    }
    cp_async_commit();
  }
  for (int t = 0; t < NT; ++t) {
    // one round trip: raw q (both heads), k, v, the norm weights and the position's RoPE rows
    const int pos = p0 + t;
    float q0[WD], q1[WD], k[WD], v[WD];
    ld8_f32(qkv + t * QKV_ROWS + (2 * h) * HD + WD * u, q0);
    ld8_f32(qkv + t * QKV_ROWS + (2 * h + 1) * HD + WD * u, q1);
    if (own) {
      ld8_f32(qkv + t * QKV_ROWS + QSZ + h * HD + WD * u, k);
      ld8_f32(qkv + t * QKV_ROWS + QSZ + KVSZ + h * HD + WD * u, v);
    }
    const bool rope = !p.kv_pre;
    const uint4 c4 = rope ? *reinterpret_cast<const uint4*>(p.cos_tab + static_cast<size_t>(pos) * HD + WD * u) : make_uint4(0, 0, 0, 0);
    const uint4 s4 = rope ? *reinterpret_cast<const uint4*>(p.sin_tab + static_cast<size_t>(pos) * HD + WD * u) : make_uint4(0, 0, 0, 0);
    const uint4 wq = rope ? *reinterpret_cast<const uint4*>(L->q_norm + WD * u) : make_uint4(0, 0, 0, 0);
    const uint4 wk = own ? *reinterpret_cast<const uint4*>(L->k_norm + WD * u) : make_uint4(0, 0, 0, 0);
    if (own) {   // the token's new K/V row, read back below like every other row
      w_norm_rope(k, wk, c4, s4, p.eps, u);
      if (g == 0) {
        const size_t row = static_cast<size_t>(pos) * HD + WD * u;
        if (CP) {
          float4* kd = reinterpret_cast<float4*>(reinterpret_cast<float*>(kb) + row);
          float4* vd = reinterpret_cast<float4*>(reinterpret_cast<float*>(vb) + row);
          kd[0] = make_float4(k[0], k[1], k[2], k[3]);
          kd[1] = make_float4(k[4], k[5], k[6], k[7]);
          vd[0] = make_float4(v[0], v[1], v[2], v[3]);
          vd[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
          uint32_t kw[4], vw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            kw[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(k[2 * i]))) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(k[2 * i + 1]))) << 16);
            vw[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i]))) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1]))) << 16);
          }
          *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(kb) + row) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
          *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(vb) + row) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
        }
      }
      __syncwarp();   // the row just stored is read back by the other lanes of this warp
    }
    if (rope) {
      w_norm_rope(q0, wq, c4, s4, p.eps, u);
      w_norm_rope(q1, wq, c4, s4, p.eps, u);
    }
    // Backbone items: the cached rows' copies go out once the item's own loads have returned.
    // Issued earlier, the stage's burst of cache reads (every warp of the grid at once, ~12 MB)
    // holds these L2 loads back by several microseconds. (The code predictor's few cached rows are
    // issued before its loads, at the top of the item.)
    if (t == 0 && staged) w_stage_first(kb, vb, s0, min(s1, p0 + 1) - nown, wbuf, cs.lane());
    WSoft a0, a1;
    a0.init();
    a1.init();
    const int send = min(s1, p0 + t + 1);
    if (staged) {   // one token (frames): staged rows, then this token's own row
      const int ce = send - nown;
      w_loop_staged(kb, vb, s0, ce, wbuf, q0, q1, p.attn_scale, cs.lane(), a0, a1);
      if (own) {   // position send - 1: the row just stored, from registers (bf16 as cached)
        WRow<false> kr[1], vr[1];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          kr[0].w[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(k[2 * i]))) |
                       (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(k[2 * i + 1]))) << 16);
          vr[0].w[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i]))) |
                       (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1]))) << 16);
        }
        bool ok[1] = {g == ((send - 1 - s0) & 1)};
        float d0[1] = {0.f}, d1[1] = {0.f};
#pragma unroll
        for (int i = 0; i < WD; ++i) {
          d0[0] = fmaf(q0[i], kr[0][i], d0[0]);
          d1[0] = fmaf(q1[i], kr[0][i], d1[0]);
        }
#pragma unroll
        for (int o = 1; o < WL; o <<= 1) {
          d0[0] += __shfl_xor_sync(WFULL, d0[0], o);
          d1[0] += __shfl_xor_sync(WFULL, d1[0], o);
        }
        d0[0] *= p.attn_scale;
        d1[0] *= p.attn_scale;
        a0.add_trip(d0, ok, vr);
        a1.add_trip(d1, ok, vr);
      }
    } else if (!staged_cp) {
    constexpr int P = CP ? 2 : 4;   // positions per group per trip: 4 P rows in flight per lane
    for (int j = s0 + g; j - g < send; j += P * WG) {   // every lane runs the same trip count
      bool ok[P];
      WRow<CP> kr[P], vr[P];
#pragma unroll
      for (int q = 0; q < P; ++q) {
        ok[q] = j + q * WG < send;
        kr[q].load(kb, ok[q] ? j + q * WG : s0, u);   // s0: a row that exists, score not used
      }
#pragma unroll
      for (int q = 0; q < P; ++q) vr[q].load(vb, ok[q] ? j + q * WG : s0, u);
      float d0[P], d1[P];
#pragma unroll
      for (int q = 0; q < P; ++q) {
        d0[q] = 0.f;
        d1[q] = 0.f;
#pragma unroll
        for (int i = 0; i < WD; ++i) {
          d0[q] = fmaf(q0[i], kr[q][i], d0[q]);
          d1[q] = fmaf(q1[i], kr[q][i], d1[q]);
        }
      }
#pragma unroll
      for (int o = 1; o < WL; o <<= 1)
#pragma unroll
        for (int q = 0; q < P; ++q) {
          d0[q] += __shfl_xor_sync(WFULL, d0[q], o);
          d1[q] += __shfl_xor_sync(WFULL, d1[q], o);
        }
#pragma unroll
      for (int q = 0; q < P; ++q) {
        d0[q] *= p.attn_scale;
        d1[q] *= p.attn_scale;
      }
      a0.add_trip(d0, ok, vr);
      a1.add_trip(d1, ok, vr);
    }
    } else if (staged_cp) {   // code predictor, one token: staged rows, then (own) the new row
      const int n = p0 + 1 - nown - s0;
      cp_async_wait<0>();
      __syncwarp();   // every lane's copies have landed
      for (int j = g; j - g < n; j += 2 * WG) {   // every lane runs the same trip count
        bool ok[2];
        WRow<true> kr[2], vr[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int r = j + q * WG;
          ok[q] = r < n;
          const uint4* kp = reinterpret_cast<const uint4*>(wbuf + (ok[q] ? r : 0) * HD * 4 + 32 * u);
          const uint4* vp = reinterpret_cast<const uint4*>(wbuf + CPWBUF / 2 + (ok[q] ? r : 0) * HD * 4 + 32 * u);
          const uint4 k0 = kp[0], k1 = kp[1], v0 = vp[0], v1 = vp[1];
          kr[q].w[0] = k0.x; kr[q].w[1] = k0.y; kr[q].w[2] = k0.z; kr[q].w[3] = k0.w;
          kr[q].w[4] = k1.x; kr[q].w[5] = k1.y; kr[q].w[6] = k1.z; kr[q].w[7] = k1.w;
          vr[q].w[0] = v0.x; vr[q].w[1] = v0.y; vr[q].w[2] = v0.z; vr[q].w[3] = v0.w;
          vr[q].w[4] = v1.x; vr[q].w[5] = v1.y; vr[q].w[6] = v1.z; vr[q].w[7] = v1.w;
        }
        float d0[2], d1[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          d0[q] = 0.f;
          d1[q] = 0.f;
#pragma unroll
          for (int i = 0; i < WD; ++i) {
            d0[q] = fmaf(q0[i], kr[q][i], d0[q]);
            d1[q] = fmaf(q1[i], kr[q][i], d1[q]);
          }
        }
#pragma unroll
        for (int o = 1; o < WL; o <<= 1)
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            d0[q] += __shfl_xor_sync(WFULL, d0[q], o);
            d1[q] += __shfl_xor_sync(WFULL, d1[q], o);
          }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          d0[q] *= p.attn_scale;
          d1[q] *= p.attn_scale;
        }
        a0.add_trip(d0, ok, vr);
        a1.add_trip(d1, ok, vr);
      }
      if (own) {   // position p0: the row just stored, from registers (fp32 as cached)
        WRow<true> kr[1], vr[1];
#pragma unroll
        for (int i = 0; i < WD; ++i) {
          kr[0].w[i] = __float_as_uint(k[i]);
          vr[0].w[i] = __float_as_uint(v[i]);
        }
        bool ok[1] = {g == (n & 1)};
        float d0[1] = {0.f}, d1[1] = {0.f};
#pragma unroll
        for (int i = 0; i < WD; ++i) {
          d0[0] = fmaf(q0[i], kr[0][i], d0[0]);
          d1[0] = fmaf(q1[i], kr[0][i], d1[0]);
        }
#pragma unroll
        for (int o = 1; o < WL; o <<= 1) {
          d0[0] += __shfl_xor_sync(WFULL, d0[0], o);
          d1[0] += __shfl_xor_sync(WFULL, d1[0], o);
        }
        d0[0] *= p.attn_scale;
        d1[0] *= p.attn_scale;
        a0.add_trip(d0, ok, vr);
        a1.add_trip(d1, ok, vr);
      }
    }
    a0.merge_groups();
    a1.merge_groups();
    if (nch == 1) {
      if (g < 2) w_out(hilo, tok0 + t, (2 * h + g) * HD + WD * u, a0, a1, g);
      continue;
    }
    // partial record {m, l, -, -, acc[128]} of (token t, q head 2h + g, chunk c)
    if (g < 2) {
      float* rec = prt + ((static_cast<size_t>(t) * NQH + 2 * h + g) * MAX_ATT_CHUNKS + c) * PRT_STRIDE;
      float4* r4 = reinterpret_cast<float4*>(rec + 4 + WD * u);
      if (g == 0) {
        __stcg(r4, make_float4(a0.acc[0], a0.acc[1], a0.acc[2], a0.acc[3]));
        __stcg(r4 + 1, make_float4(a0.acc[4], a0.acc[5], a0.acc[6], a0.acc[7]));
        if (u == 0) __stcg(reinterpret_cast<float2*>(rec), make_float2(a0.m, a0.l));
      } else {
        __stcg(r4, make_float4(a1.acc[0], a1.acc[1], a1.acc[2], a1.acc[3]));
        __stcg(r4 + 1, make_float4(a1.acc[4], a1.acc[5], a1.acc[6], a1.acc[7]));
        if (u == 0) __stcg(reinterpret_cast<float2*>(rec), make_float2(a1.m, a1.l));
      }
    }
    __threadfence();
    __syncwarp();
    uint32_t last = 0;
    if (cs.lane() == 0) last = atomicAdd(cnt, 1u) == static_cast<uint32_t>(nch - 1) ? 1u : 0u;
    last = __shfl_sync(WFULL, last, 0);
    if (!last) continue;
    __threadfence();
    // merge the nch records: group g takes chunks g, g + 2, ... of both heads
    a0.init();
    a1.init();
    // up to 2 chunks per group per round, all their loads issued before the first merge
    for (int cb = g; cb - g < nch; cb += 2 * WG) {
      float2 ml[2][2];
      float a2[2][2][WD];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int cc = min(cb + j * WG, nch - 1);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float* rec = prt + ((static_cast<size_t>(t) * NQH + 2 * h + hh) * MAX_ATT_CHUNKS + cc) * PRT_STRIDE;
          ml[j][hh] = __ldcg(reinterpret_cast<const float2*>(rec));
          ld8_f32(rec + 4 + WD * u, a2[j][hh]);
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j)
        if (cb + j * WG < nch) {
          a0.merge(ml[j][0].x, ml[j][0].y, a2[j][0]);
          a1.merge(ml[j][1].x, ml[j][1].y, a2[j][1]);
        }
    }
    a0.merge_groups();
    a1.merge_groups();
    if (g < 2) w_out(hilo, tok0 + t, (2 * h + g) * HD + WD * u, a0, a1, g);
    if (cs.lane() == 0) atomicExch(cnt, 0u);
  }
}

// Attention of one layer for every utterance, output as the o_proj operand planes. Code
// predictor: one warp item per (utterance, KV head) over its <= 17 positions, 2 tokens in the
// first pass. Backbone: (utterance, KV head, chunk) items, chunk length chosen so that the
// items of all active utterances spread over every consumer warp of the grid.
__device__ __noinline__ bool b_attention(const Params& p, Smem& sm, Cons& cs, int li, bool cp, int pass) {
  const BState bst = bstate(sm);
  const int B = p.nb;
  const int NW = cs.G() * NCW, gw = cs.cta() * NCW + cs.warp();
  if (cp) {
    const int l = li - p.n_bb;
    const LayerW* L = p.cp_layers + l;
    const int NT = pass == 0 ? 2 : 1, p0 = pass == 0 ? 0 : pass + 1;
    // items spread over the CTAs first (warp w of CTA c: item c + G w), so that warps 0..3 of
    // every CTA hold them and each stages its rows in a quarter of the activation ring
    uint8_t* wb = (NT == 1 && cs.warp() < 4)
                      ? reinterpret_cast<uint8_t*>(sm.ring) + WRING_BYTES + cs.warp() * CPWBUF
                      : nullptr;
    for (int item = cs.cta() + cs.G() * cs.warp(); item < B * NKVH; item += NW) {
      const int s = item / NKVH, h = item - s * NKVH;
      const size_t off = (static_cast<size_t>(l) * NKVH + h) * p.cp_max_seq * HD;
      watt_item<true>(p, cs, L, p.bw.qkv + static_cast<size_t>(s * NT) * QKV_ROWS, NT, p0, h,
                      reinterpret_cast<uint8_t*>(static_cast<float*>(sm.bkv[4 * s + 2]) + off),
                      reinterpret_cast<uint8_t*>(static_cast<float*>(sm.bkv[4 * s + 3]) + off),
                      p.bw.abuf[1], s * NT, 0, 1, 0, p0 + NT, true, nullptr, nullptr, wb);
    }
  } else {
    const LayerW* L = p.bb_layers + li;
    // this warp's slice of the activation ring stages the items' cached K/V rows
    uint8_t* wbuf = reinterpret_cast<uint8_t*>(sm.ring) + WRING_BYTES + cs.warp() * WBUF;
    // Items run over "rows": the utterances of a frame / prefill step, or the T context tokens of
    // one utterance in a dense prefill (row v at position p0 + v, all rows sharing its cache).
    const bool dense = p.mode == MODE_B_PREFILL_DENSE;
    const int NV = dense ? p.b_ntok : B, p0d = p.b_step;
    if (dense && !p.kv_pre) {
      // the chunk's new K/V rows first (q/k norm of k + RoPE, bf16), so that every row reads them
      // from the cache after the barrier: item (token t, KV head h). (With p.kv_pre the QKV
      // epilogue has written them.)
      const int g = cs.lane() / WL, u = cs.lane() % WL;
      for (int item = gw; item < NV * NKVH; item += NW) {
        const int t = item / NKVH, h = item - t * NKVH, pos = p0d + t;
        const float* row = p.bw.qkv + static_cast<size_t>(t) * QKV_ROWS;
        float k[WD], v[WD];
        ld8_f32(row + QSZ + h * HD + WD * u, k);
        ld8_f32(row + QSZ + KVSZ + h * HD + WD * u, v);
        const uint4 c4 = *reinterpret_cast<const uint4*>(p.cos_tab + static_cast<size_t>(pos) * HD + WD * u);
        const uint4 s4 = *reinterpret_cast<const uint4*>(p.sin_tab + static_cast<size_t>(pos) * HD + WD * u);
        const uint4 wk = *reinterpret_cast<const uint4*>(L->k_norm + WD * u);
        w_norm_rope(k, wk, c4, s4, p.eps, u);
        if (g == 0) {
          const size_t off = ((static_cast<size_t>(li) * NKVH + h) * p.bb_max_seq + pos) * HD + WD * u;
          uint32_t kw[4], vw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            kw[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(k[2 * i]))) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(k[2 * i + 1]))) << 16);
            vw[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i]))) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1]))) << 16);
          }
          *reinterpret_cast<uint4*>(p.bs[0].k + off) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
          *reinterpret_cast<uint4*>(p.bs[0].v + off) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
        }
      }
      if (!grid_sync_b(p, sm, cs)) return false;
    }
    auto row_len = [&](int v) -> int {   // context length of row v (0: inactive)
      if (dense) return p0d + v + 1;
      return bst.act[v] ? bst.pos[v] + 1 : 0;
    };
    // the plan, computed by warp 0 (lane l: rows l, l + 32, l + 64, l + 96) into sm.bplan: item
    // offset of each row [0, 128), chunks per KV head [128, 256), item count [256]; the chunk
    // length is the smallest (in steps of 1/8) for which every item gets its own warp. The rows'
    // lengths do not change within a launch, so the first backbone layer's plan serves them all.
    int* plan = sm.bplan;
    if (cs.warp() == 0 && !sm.bplan_ok) {
      int Sx[4], nx[4];
      int tot = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int v = cs.lane() + 32 * k;
        Sx[k] = v < NV ? row_len(v) : 0;
        tot += Sx[k];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(WFULL, tot, o);
      int CL = max(16, (tot * NKVH + NW - 1) / NW);
      for (int it = 0; it < 64; ++it) {
        int n = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          nx[k] = Sx[k] ? min(MAX_ATT_CHUNKS, (Sx[k] + CL - 1) / CL) : 0;
          n += nx[k];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(WFULL, n, o);
        if (NKVH * n <= NW) break;
        CL += max(1, CL / 8);
      }
      // exclusive prefix sums of NKVH * chunks over rows 0..127 (four 32-row blocks)
      int base = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        int x = NKVH * nx[k];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(WFULL, x, o);
          if (cs.lane() >= o) x += y;
        }
        plan[cs.lane() + 32 * k] = base + x - NKVH * nx[k];
        plan[128 + cs.lane() + 32 * k] = nx[k];
        base += __shfl_sync(WFULL, x, 31);
      }
      if (cs.lane() == 0) {
        plan[256] = base;
        sm.bplan_ok = 1;
      }
    }
    named_sync(1, NCT);
    const int total = plan[256];
    for (int item = gw; item < total; item += NW) {
      int lo = 0, hi = NV - 1;   // the last row whose offset <= item (binary search)
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (plan[mid] <= item) lo = mid; else hi = mid - 1;
      }
      int v = lo;
      while (plan[128 + v] == 0) --v;   // skip inactive rows sharing the offset
      const int nch = plan[128 + v], idx = item - plan[v];
      const int h = idx / nch, c = idx - h * nch;
      const int S = row_len(v), chunk = (S + nch - 1) / nch;
      const int s0 = c * chunk, s1 = min(S, s0 + chunk);
      const int su = dense ? 0 : v;   // the utterance whose cache the row reads
      const size_t off = (static_cast<size_t>(li) * NKVH + h) * p.bb_max_seq * HD;
      watt_item<false>(p, cs, L, p.bw.qkv + static_cast<size_t>(v) * QKV_ROWS, 1, S - 1, h,
                       reinterpret_cast<uint8_t*>(static_cast<bf16*>(sm.bkv[4 * su]) + off),
                       reinterpret_cast<uint8_t*>(static_cast<bf16*>(sm.bkv[4 * su + 1]) + off),
                       p.bw.abuf[1], v, c, nch, s0, s1, !dense && s1 == S,
                       p.bw.prt + static_cast<size_t>(v) * NQH * MAX_ATT_CHUNKS * PRT_STRIDE,
                       p.bw.att_cnt + v * NKVH + h, wbuf);
    }
  }
  cs.go_next = 1;   // o_proj follows
  return b_sync_planes(p, sm, cs);
}

// One decoder layer of the batch: QKV | attention | O | gate/up | down.
// The four GEMM stages of a layer, each a function of its own: one epilogue's callbacks at a time
// share the register budget, so the item loops run without spilling to local memory.
// QKV with p.kv_pre (clusters of 4: a row tile is one head): the epilogue also applies the q/k
// RMSNorm and RoPE (the 16 items of a token's head row are 16 lanes of one warp, the layout of
// w_norm_rope) and writes the token's new K and V rows into its cache (backbone bf16, code
// predictor fp32), so that the attention items read every row from the cache.
// Row of stack token t: its utterance, position and whether it is decoded (code predictor: pass
// 0 holds two tokens per utterance at positions 0 and 1, pass g the token at position g + 1).
struct BKvRow {
  int s, pos;
  bool on;
};
__device__ __forceinline__ BKvRow b_kv_row(const Params& p, const BState& bst, bool cp, int pass, int T, int t) {
  BKvRow r;
  if (cp) {
    const int NT = T > p.nb ? 2 : 1;
    r.s = t / NT;
    r.pos = pass == 0 ? (t & 1) : pass + 1;
    r.on = true;
  } else if (p.mode == MODE_B_PREFILL_DENSE) {
    r.s = 0;
    r.pos = p.b_step + t;
    r.on = true;
  } else {
    r.s = t;
    r.pos = bst.pos[t];
    r.on = bst.act[t] != 0;
  }
  return r;
}
__device__ __noinline__ bool b_qkv_stage(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, int li, bool cp, int pass, int T) {
  const unsigned long long* ssq = b_ssq_cur(p, cs);
  const float eps = p.eps;
  if (!p.kv_pre)
    return b_gemm(
        p, sm, cs, BGemm{BK_QKV, li, 0, T}, gn, false,
        [&](int t, int r0, EpiSt& st) { st.rs = b_rstd(ssq, t, eps); },
        [&](int t, int r0, const float (&y)[EW], const float (&y2)[EW], const EpiSt& st) {
          float v[EW];
#pragma unroll
          for (int i = 0; i < EW; ++i) v[i] = y[i] * st.rs;
          stw_f32(p.bw.qkv + static_cast<size_t>(t) * QKV_ROWS + r0, v);
        });
  const BState bst = bstate(sm);
  const LayerW* L = cp ? p.cp_layers + (li - p.n_bb) : p.bb_layers + li;
  const bf16* const qn = L->q_norm;   // read once, before the stage's wait for D
  const bf16* const kn = L->k_norm;
  return b_gemm<true>(
      p, sm, cs, BGemm{BK_QKV, li, 0, T}, gn, false,
      [&](int t, int r0, EpiSt& st) {
        st.rs = b_rstd(ssq, t, eps);
        const int sec = r0 / HD, u = (r0 % HD) / WD;   // head row: q 0..15, k 16..23, v 24..31
        const BKvRow kr = b_kv_row(p, bst, cp, pass, T, t);
        const int pos = kr.on ? kr.pos : 0;
        st.w4 = sec < NQH + NKVH ? *reinterpret_cast<const uint4*>((sec < NQH ? qn : kn) + WD * u) : make_uint4(0, 0, 0, 0);
        st.c4 = *reinterpret_cast<const uint4*>(p.cos_tab + static_cast<size_t>(pos) * HD + WD * u);
        st.s4 = *reinterpret_cast<const uint4*>(p.sin_tab + static_cast<size_t>(pos) * HD + WD * u);
        st.kv = nullptr;
        if (sec >= NQH && kr.on && st.valid) {
          const int h = (sec - NQH) % NKVH;
          const bool isv = sec >= NQH + NKVH;
          void* const* base = sm.bkv + 4 * kr.s;   // the utterance's cache addresses (shared memory)
          if (cp) {
            const size_t off = ((static_cast<size_t>(li - p.n_bb) * NKVH + h) * p.cp_max_seq + pos) * HD + WD * u;
            st.kv = static_cast<float*>(base[isv ? 3 : 2]) + off;
          } else {
            const size_t off = ((static_cast<size_t>(li) * NKVH + h) * p.bb_max_seq + pos) * HD + WD * u;
            st.kv = static_cast<bf16*>(base[isv ? 1 : 0]) + off;
          }
        }
      },
      [&](int t, int r0, const float (&y)[EW], const float (&y2)[EW], const EpiSt& st) {
        float v[EW];
#pragma unroll
        for (int i = 0; i < EW; ++i) v[i] = y[i] * st.rs;
        const int sec = r0 / HD, u = (r0 % HD) / WD;
        // warp-uniform: the warp's 32 items are two tokens' rows of the same head
        if (sec < NQH + NKVH) w_norm_rope(v, st.w4, st.c4, st.s4, eps, u);
        if (!st.valid) return;
        if (sec < NQH) {
          stw_f32(p.bw.qkv + static_cast<size_t>(t) * QKV_ROWS + r0, v);
        } else if (st.kv != nullptr) {
          if (cp) {
            float4* d = reinterpret_cast<float4*>(st.kv);
            d[0] = make_float4(v[0], v[1], v[2], v[3]);
            d[1] = make_float4(v[4], v[5], v[6], v[7]);
          } else {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i]))) |
                     (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1]))) << 16);
            *reinterpret_cast<uint4*>(st.kv) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      });
}

// o_proj + residual -> hmid, A planes of gate/up (post-attention norm), sums of squares
__device__ __noinline__ bool b_o_stage(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, int li, int T, const float* hin,
                                       const bf16* post_norm) {
  unsigned long long* ssq = b_ssq_next(p, cs);
  return b_gemm(
      p, sm, cs, BGemm{BK_O, li, 0, T}, gn, true,
      [&](int t, int r0, EpiSt& st) {
        ldw_f32(hin + t * HID + r0, st.a);
        ldw_bf16(post_norm + r0, st.b);
      },
      [&](int t, int r0, const float (&y)[EW], const float (&y2)[EW], const EpiSt& st) {
        double ss = 0.0;
        float v[EW], a[EW];
#pragma unroll
        for (int i = 0; i < EW; ++i) {
          v[i] = y[i] + st.a[i];
          a[i] = v[i] * st.b[i];
          ss = fma(static_cast<double>(v[i]), static_cast<double>(v[i]), ss);
        }
        stw_f32(p.bw.hmid + t * HID + r0, v);
        hilo_store_w(p.bw.abuf[0], t, r0, a);
        b_ssq_add(ssq, t, ss);
      });
}

// gate/up + SiLU (deferred post-attention norm) -> A planes of down
__device__ __noinline__ bool b_gu_stage(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, int li, int T) {
  const unsigned long long* ssq = b_ssq_cur(p, cs);
  const float eps = p.eps;
  return b_gemm(
      p, sm, cs, BGemm{BK_GU, li, 0, T}, gn, true,
      [&](int t, int r0, EpiSt& st) { st.rs = b_rstd(ssq, t, eps); },
      [&](int t, int r0, const float (&y)[EW], const float (&y2)[EW], const EpiSt& st) {
        float m[EW];
#pragma unroll
        for (int i = 0; i < EW; ++i) {
          const float gg = y[i] * st.rs, uu = y2[i] * st.rs;
          m[i] = (gg / (1.0f + expf(-gg))) * uu;
        }
        hilo_store_w(p.bw.abuf[1], t, r0, m);
      });
}

// down + residual -> layer output, A planes of the next layer (its input norm), sums of squares
__device__ __noinline__ bool b_d_stage(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, int li, bool cp, int T,
                                       float* hout, const bf16* next_norm) {
  unsigned long long* ssq = b_ssq_next(p, cs);
  return b_gemm(
      p, sm, cs, BGemm{BK_D, li, 0, T}, gn, next_norm != nullptr,
      [&](int t, int r0, EpiSt& st) {
        ldw_f32(p.bw.hmid + t * HID + r0, st.a);
        if (next_norm) ldw_bf16(next_norm + r0, st.b);
      },
      [&](int t, int r0, const float (&y)[EW], const float (&y2)[EW], const EpiSt& st) {
        double ss = 0.0;
        float v[EW];
#pragma unroll
        for (int i = 0; i < EW; ++i) {
          v[i] = y[i] + st.a[i];
          if (!cp) v[i] = round_bf16(v[i]);
          ss = fma(static_cast<double>(v[i]), static_cast<double>(v[i]), ss);
        }
        stw_f32(hout + t * HID + r0, v);
        if (next_norm) {
          float a[EW];
#pragma unroll
          for (int i = 0; i < EW; ++i) a[i] = v[i] * st.b[i];
          hilo_store_w(p.bw.abuf[0], t, r0, a);
        }
        b_ssq_add(ssq, t, ss);
      });
}

__device__ bool b_layer(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, int li, bool cp, int pass, int T,
                        const float* hin, float* hout, const bf16* next_norm) {
  const LayerW* L = (cp ? p.cp_layers + (li - p.n_bb) : p.bb_layers + li);
  if (!b_qkv_stage(p, sm, cs, gn, li, cp, pass, T)) return false;
  // attention -> A planes of o_proj
  if (!b_attention(p, sm, cs, li, cp, pass)) return false;
  if (!b_o_stage(p, sm, cs, gn, li, T, hin, L->post_norm)) return false;
  if (!b_gu_stage(p, sm, cs, gn, li, T)) return false;
  return b_d_stage(p, sm, cs, gn, li, cp, T, hout, next_norm);
}

// Layers of a stack over T tokens whose input (x, A planes, sums of squares) is ready.
// Returns the buffer holding the last layer's output (nullptr on abort).
__device__ __noinline__ const float* b_stack(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, bool cp, int pass, int T) {
  const int n = cp ? p.n_cp : p.n_bb;
  const LayerW* Ls = cp ? p.cp_layers : p.bb_layers;
  const float* hin = p.bw.x;
  for (int l = 0; l < n; ++l) {
    float* hout = p.bw.hb[l & 1];
    const bf16* nn = l + 1 < n ? Ls[l + 1].in_norm : nullptr;
    if (!b_layer(p, sm, cs, gn, cp ? p.n_bb + l : l, cp, pass, T, hin, hout, nn)) return nullptr;
    hin = hout;
  }
  return hin;
}

// Head GEMM over the NORM stage's A planes: bf16 logits; greedy heads fold the masked argmax of
// each token into amax[slot][t]; sampled heads store the logits for the sampler. The other slot
// is cleared for the next head (two barriers away).
__device__ __noinline__ bool b_head(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, int hidx, const SampleCfg cfg,
                                    int slot) {
  const BState bst = bstate(sm);
  unsigned long long* amax = p.bw.amax + slot * TBMAX;
  if (cs.cta() == 0)
    for (int t = cs.tid(); t < TBMAX; t += NCT) __stcg(p.bw.amax + (slot ^ 1) * TBMAX + t, 0ull);
  float* dbg = hidx > 0 ? p.dbg_cp_logits : (p.mode == MODE_B_FRAME ? p.dbg_g0_logits : nullptr);
  if (cfg.do_sample)   // sampled heads store the bf16 logits; the sampler applies the masks
    return b_gemm(
        p, sm, cs, BGemm{BK_HEAD, 0, hidx, p.nb}, gn, false, [&](int t, int r0, EpiSt& st) {},
        [&](int t, int r0, const float (&y)[EW], const float (&y2)[EW], const EpiSt& st) {
          float lg[EW];
#pragma unroll
          for (int i = 0; i < EW; ++i) lg[i] = round_bf16(y[i]);
          if (dbg != nullptr) {   // parity tests: [B][15][cp_vocab] / [B][vocab]
            float* d = hidx > 0 ? dbg + (static_cast<size_t>(t) * NCPHEADS + hidx - 1) * p.cp_vocab + r0
                                : dbg + static_cast<size_t>(t) * p.vocab + r0;
#pragma unroll
            for (int i = 0; i < EW; ++i) d[i] = lg[i];
          }
          stw_f32(p.bw.logits + static_cast<size_t>(t) * VMAX + r0, lg);
        });
  return b_gemm(
      p, sm, cs, BGemm{BK_HEAD, 0, hidx, p.nb}, gn, false,
      [&](int t, int r0, EpiSt& st) {},
      [&](int t, int r0, const float (&y)[EW], const float (&y2)[EW], const EpiSt& st) {
        SampleCfg c = cfg;
        if (hidx == 0) {
          c.seen = (c.penalty != 1.f) ? p.bs[t].st->seen : nullptr;
          c.mask_eos = (p.mode == MODE_B_HEAD) ? (p.sp.min_new_tokens > 0 ? 1 : 0)
                                               : ((bst.step[t] + 1 < p.sp.min_new_tokens) ? 1 : 0);
        }
        unsigned long long best = 0ull;
#pragma unroll
        for (int i = 0; i < EW; ++i) {
          const int row = r0 + i;
          const float lg = round_bf16(y[i]);
          if (dbg != nullptr) {
            if (hidx > 0)
              dbg[(static_cast<size_t>(t) * NCPHEADS + hidx - 1) * p.cp_vocab + row] = lg;
            else
              dbg[static_cast<size_t>(t) * p.vocab + row] = lg;
          }
          const unsigned long long k = argmax_key(head_mask(c, row, lg), row);
          best = k > best ? k : best;
        }
        if (best != 0ull) atomicMax(amax + t, best);
      });
}

// Token of utterance s from head slot `slot` (greedy) or bw.tok (sampled, column col).
// A token outside the head's vocabulary (an argmax slot no CTA wrote) sets DEV_ERR_BAD_TOKEN and
// reads as 0, so that the embedding rows gathered with it stay inside their tables.
__device__ __forceinline__ int b_token(const Params& p, const SampleCfg& cfg, int slot, int s, int col) {
  int tok;
  if (!cfg.do_sample) {
    const unsigned long long k = __ldcg(p.bw.amax + slot * TBMAX + s);
    tok = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
  } else {
    tok = __ldcg(p.bw.tok + s * NGROUPS + col);
  }
  if (tok < 0 || tok >= cfg.V) {
    set_error(p.w.err, DEV_ERR_BAD_TOKEN);
    tok = 0;
  }
  return tok;
}

// Tokens of a head for every utterance, after its barrier, into bw.tok[s][col]: greedy from the
// packed argmax (CTA 0 copies them; the next stage reads the slot directly), sampled by one CTA
// per utterance followed by a barrier. frame_of: the Philox frame counter is step + frame_of.
__device__ __noinline__ bool b_tokens(const Params& p, Smem& sm, Cons& cs, int hidx, const SampleCfg& cfg, int slot, int frame_of,
                         int col) {
  const BState bst = bstate(sm);
  if (!cfg.do_sample) {
    if (cs.cta() == 0)
      for (int s = cs.tid(); s < p.nb; s += NCT) __stcg(p.bw.tok + s * NGROUPS + col, b_token(p, cfg, slot, s, col));
    return true;
  }
  for (int s = cs.cta(); s < p.nb; s += cs.G()) {
    SampleCfg c = cfg;
    if (hidx == 0) {
      c.seen = (c.penalty != 1.f) ? p.bs[s].st->seen : nullptr;
      c.mask_eos = (p.mode == MODE_B_HEAD) ? (p.sp.min_new_tokens > 0 ? 1 : 0)
                                           : ((bst.step[s] + 1 < p.sp.min_new_tokens) ? 1 : 0);
    }
    Sampling sp = p.sp;
    sp.philox_stream = p.bs[s].philox;
    const int fr = p.mode == MODE_B_HEAD ? 0 : bst.step[s] + frame_of;
    c.u24 = draw_u24(sp, fr, hidx);
    const int tk = sample(p.bw.logits + static_cast<size_t>(s) * VMAX, sm, cs, c);
    if (cs.tid() == 0) __stcg(p.bw.tok + s * NGROUPS + col, tk);
  }
  return grid_sync_b(p, sm, cs);
}

__device__ SampleCfg b_codec_cfg(const Params& p, float penalty) {
  SampleCfg c;
  c.V = p.vocab;
  c.do_sample = p.sp.do_sample;
  c.temperature = p.sp.temperature;
  c.top_k = p.sp.top_k;
  c.top_p = p.sp.top_p;
  c.suppress_from = p.vocab - 1024;
  c.eos = p.sp.eos;
  c.mask_eos = 0;
  c.penalty = penalty;
  c.seen = nullptr;
  c.u24 = 0u;
  return c;
}

// Input of code-predictor pass g (T tokens): [bf16(h), codec_embedding[g0]] for the first pass,
// else the previous head's token's codec embedding g - 1.
__device__ __noinline__ bool b_cp_input(const Params& p, Smem& sm, Cons& cs, int g, int T, int slot, const SampleCfg& cpc) {
  const BState bst = bstate(sm);
  const bf16* w0 = p.cp_layers[0].in_norm;
  if (g == 0) {
    // [bf16(h), codec_embedding[g0]] at positions 0, 1 (generator.py:319-325)
    if (!b_input(p, sm, cs, T, w0, [&](int t, int k0, float (&v)[8]) {
          const int s = t >> 1;
          if (t & 1) {
            const bf16* row = p.codec_emb + static_cast<size_t>(bst.g0[s]) * HID + k0;
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(row[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = round_bf16(__ldcg(p.bs[s].st->h + k0 + i));
          }
        }))
      return false;
  } else {
    // codec embedding g-1 of the previous head's token (generator.py:347-352)
    const bf16* table = p.cp_emb[g - 1];
    const int prev = slot ^ 1;
    if (!b_input(p, sm, cs, T, w0, [&](int t, int k0, float (&v)[8]) {
          const int tk = b_token(p, cpc, prev, t, g);
          const bf16* row = table + static_cast<size_t>(tk) * HID + k0;
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(row[i]);
        }))
      return false;
  }
  return true;
}

// COMBINE of a frame: the 16 codec embeddings of each utterance's codes summed in bf16 + its
// text row (or the pad row); the last code-predictor head's tokens are in argmax slot slot ^ 1.
__device__ __noinline__ bool b_combine(const Params& p, Smem& sm, Cons& cs, int slot, const SampleCfg& cpc) {
  const BState bst = bstate(sm);
  const int B = p.nb;
  if (!b_input(p, sm, cs, B, p.bb_layers[0].in_norm, [&](int s, int k0, float (&v)[8]) {
        const int step = bst.step[s];
        const bf16* extra =
            step < p.bs[s].n_trailing ? p.bs[s].trailing + static_cast<size_t>(step) * HID : p.bs[s].pad;
        // greedy heads publish their tokens in bw.tok without a barrier (CTA 0, for the frame
        // results): the last head's token comes from its argmax slot, complete at its barrier
        int toks[NCPHEADS];
#pragma unroll
        for (int q = 0; q < NCPHEADS - 1; ++q) toks[q] = __ldcg(p.bw.tok + s * NGROUPS + q + 1);
        toks[NCPHEADS - 1] = b_token(p, cpc, slot ^ 1, s, NCPHEADS);
        // the 17 rows' 8 columns as 16-byte loads, all in flight together, then the adds in order
        uint4 e[NCPHEADS + 1];
        e[0] = *reinterpret_cast<const uint4*>(p.codec_emb + static_cast<size_t>(bst.g0[s]) * HID + k0);
#pragma unroll
        for (int q = 0; q < NCPHEADS; ++q)
          e[q + 1] = *reinterpret_cast<const uint4*>(p.cp_emb[q] + static_cast<size_t>(toks[q]) * HID + k0);
        float x[8];   // the caller's text row (no alignment promised beyond bf16)
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = __bfloat162float(extra[k0 + i]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float a = bf16_at(&e[0].x, i);
#pragma unroll
          for (int q = 0; q < NCPHEADS; ++q) a = round_bf16(a + bf16_at(&e[q + 1].x, i));
          v[i] = round_bf16(a + x[i]);
        }
      }))
    return false;
  return true;
}

__device__ bool b_frame(const Params& p, Smem& sm, Cons& cs) {
  const BState bst = bstate(sm);
  const int B = p.nb;
  uint32_t gn = 0;
  if (cs.cta() == 0)
    for (int s = cs.tid(); s < B; s += NCT) {
      if (bst.act[s]) p.bs[s].st->seen[bst.g0[s]] = 1;   // generated_g0.append (generator.py:129)
      else if (ld_volatile_i32(&p.bs[s].st->g0) == p.sp.eos) p.bs[s].st->done = 1;   // generator.py:126
    }
  SampleCfg cpc;
  cpc.V = p.cp_vocab;
  cpc.do_sample = p.sp.cp_do_sample;
  cpc.temperature = p.sp.cp_temperature;
  cpc.top_k = p.sp.cp_top_k;
  cpc.top_p = 1.f;
  cpc.suppress_from = p.cp_vocab;
  cpc.eos = -1;
  cpc.mask_eos = 0;
  cpc.penalty = 1.f;
  cpc.seen = nullptr;
  cpc.u24 = 0u;
  int slot = 0;
  for (int g = 0; g < NCPHEADS; ++g) {
    const int T = g == 0 ? 2 * B : B;
    if (!b_cp_input(p, sm, cs, g, T, slot, cpc)) return false;
    const float* last = b_stack(p, sm, cs, gn, true, g, T);
    if (!last) return false;
    if (!b_norm(p, sm, cs, last, g == 0 ? 2 : 1, g == 0 ? 1 : 0, p.cp_norm, false)) return false;
    if (!b_head(p, sm, cs, gn, 1 + g, cpc, slot)) return false;
    if (!b_tokens(p, sm, cs, 1 + g, cpc, slot, 0, g + 1)) return false;
    slot ^= 1;
  }
  // ---- combine (generator.py:143-149,356-362): sequential bf16 adds + text row
  if (!b_combine(p, sm, cs, slot, cpc)) return false;
  const float* last = b_stack(p, sm, cs, gn, false, 0, B);
  if (!last) return false;
  if (!b_norm(p, sm, cs, last, 1, 0, p.bb_norm, true)) return false;
  const SampleCfg c = b_codec_cfg(p, p.sp.repetition_penalty);
  if (!b_head(p, sm, cs, gn, 0, c, slot)) return false;
  if (!b_tokens(p, sm, cs, 0, c, slot, 1, 0)) return false;
  // ---- frame results: codes, next g0, position, step
  if (cs.cta() == 0)
    for (int s = cs.tid(); s < B; s += NCT) {
      if (!bst.act[s]) continue;
      StreamState* st = p.bs[s].st;
      int32_t* out = p.bs[s].codes + static_cast<size_t>(bst.step[s]) * NGROUPS;
      out[0] = bst.g0[s];
      for (int q = 0; q < NCPHEADS; ++q) out[q + 1] = __ldcg(p.bw.tok + s * NGROUPS + q + 1);
      st->g0 = b_token(p, c, slot, s, 0);
      st->position = bst.pos[s] + 1;
      st->step = bst.step[s] + 1;
    }
  return true;
}

// One context step of the backbone prefill for every utterance with b_step < len.
__device__ bool b_prefill(const Params& p, Smem& sm, Cons& cs) {
  const BState bst = bstate(sm);
  uint32_t gn = 0;
  const int i = p.b_step;
  if (!b_input(p, sm, cs, p.nb, p.bb_layers[0].in_norm, [&](int s, int k0, float (&v)[8]) {
        if (bst.act[s]) {
          const bf16* row = p.bs[s].emb + static_cast<size_t>(i) * HID + k0;
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(row[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = 0.f;
        }
      }))
    return false;
  const float* last = b_stack(p, sm, cs, gn, false, 0, p.nb);
  if (!last) return false;
  // the final norm of each utterance's last context token is its decode state h
  const unsigned long long* ssq = b_ssq_cur(p, cs);
  b_elementwise(cs, p.nb, [&](int s, int k0) {
    if (!bst.act[s] || i != p.bs[s].len - 1) return;
    const float rs = b_rstd(ssq, s, p.eps);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      p.bs[s].st->h[k0 + j] = __ldcg(last + s * HID + k0 + j) * rs * __bfloat162float(p.bb_norm[k0 + j]);
  });
  if (cs.cta() == 0)
    for (int s = cs.tid(); s < p.nb; s += NCT)
      if (bst.act[s]) p.bs[s].st->position = i + 1;
  return true;
}

// Dense prefill of one utterance (bs[0]): context positions [p0, p0 + T) in one program, every
// projection a T-token tensor-core GEMM, the positions' K/V rows written before a causal
// attention over the cache (replaces the reference's PyTorch prefill and KV handoff,
// generator.py:209-225,245-257). After the last chunk the final norm of the last position is
// the decode state h, and the position is the context length.
__device__ bool b_prefill_dense(const Params& p, Smem& sm, Cons& cs) {
  uint32_t gn = 0;
  const int p0 = p.b_step, T = p.b_ntok;
  const bf16* emb = p.bs[0].emb;
  if (!b_input(p, sm, cs, T, p.bb_layers[0].in_norm, [&](int t, int k0, float (&v)[8]) {
        const bf16* row = emb + static_cast<size_t>(p0 + t) * HID + k0;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(row[j]);
      }))
    return false;
  const float* last = b_stack(p, sm, cs, gn, false, 0, T);
  if (!last) return false;
  if (p0 + T == p.bs[0].len) {
    const unsigned long long* ssq = b_ssq_cur(p, cs);
    b_elementwise(cs, 1, [&](int, int k0) {
      const int t = T - 1;
      const float rs = b_rstd(ssq, t, p.eps);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        p.bs[0].st->h[k0 + j] = __ldcg(last + t * HID + k0 + j) * rs * __bfloat162float(p.bb_norm[k0 + j]);
    });
  }
  if (cs.cta() == 0 && cs.tid() == 0) p.bs[0].st->position = p0 + T;
  return true;
}

// First group-0 token of every utterance from its decode state h (generator.py:115-120).
__device__ bool b_first_token(const Params& p, Smem& sm, Cons& cs) {
  uint32_t gn = 0;
  b_elementwise(cs, p.nb, [&](int s, int k0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      p.bw.abuf[1][static_cast<size_t>(s) * ABUF_LD + k0 + j] = __float2bfloat16_rn(__ldcg(p.bs[s].st->h + k0 + j));
      p.bw.abuf[1][static_cast<size_t>(TBMAX + s) * ABUF_LD + k0 + j] = __float2bfloat16_rn(0.f);
    }
  });
  cs.go_next = 1;   // the codec head follows
  if (!grid_sync_b(p, sm, cs)) return false;
  const SampleCfg c = b_codec_cfg(p, 1.f);
  if (!b_head(p, sm, cs, gn, 0, c, 0)) return false;
  if (!b_tokens(p, sm, cs, 0, c, 0, 0, 0)) return false;
  if (cs.cta() == 0)
    for (int s = cs.tid(); s < p.nb; s += NCT) {
      StreamState* st = p.bs[s].st;
      st->g0 = b_token(p, c, 0, s, 0);
      st->step = 0;
      st->done = 0;
    }
  return true;
}

extern "C" __global__ void __launch_bounds__(NTHREADS_B, 1) qtt_batch_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw_b[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw_b);
  const int tid = threadIdx.x, warp = tid >> 5;
  if ((smem_u32(sm.ring) & 1023u) != 0u) {   // 128-byte swizzle atoms need 1024-byte alignment
    if (tid == 0) set_error(p.w.err, DEV_ERR_SMEM_ALIGN);
    return;
  }
  if (tid == 0) {
    for (int i = 0; i < BB_N; ++i)
      mbar_init(&sm.bbar[i], i == BB_SREADY ? static_cast<uint32_t>(p.bcl)
                                            : (i == BB_RFREE ? static_cast<uint32_t>(p.bcl - 1) : 1u));
    sm.abort = 0;
    sm.epoch = 0;
    sm.bplan_ok = 0;
    fence_barrier_init();
  }
  if (warp == NCW + 1) {
    tmem_alloc(&sm.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  // the cluster's mbarriers are initialised before any CTA of the cluster arrives on them
  cluster_sync_all();
  // per-utterance state: position, step, g0, active
  for (int s = tid; s < BMAX; s += NTHREADS_B) {
    int act = 0, pos = 0, step = 0, g0 = 0;
    if (s < p.nb) {
      const StreamState* st = p.bs[s].st;
      pos = ld_volatile_i32(&st->position);
      step = ld_volatile_i32(&st->step);
      g0 = ld_volatile_i32(&st->g0);
      const int done = ld_volatile_i32(&st->done);
      if (p.mode == MODE_B_FRAME)
        act = (!done && g0 != p.sp.eos && g0 >= 0 && g0 < p.vocab && pos >= 0 && pos < p.bb_max_seq &&
               pos < p.rope_rows && step >= 0 && step < p.bs[s].frame_limit)
                  ? 1
                  : 0;
      else if (p.mode == MODE_B_PREFILL)
        act = (p.b_step < p.bs[s].len) ? 1 : 0;
      else
        act = 1;
      if (p.mode == MODE_B_PREFILL || p.mode == MODE_B_PREFILL_DENSE) pos = p.b_step;
      if (g0 < 0 || g0 >= p.vocab) g0 = 0;
    }
    if (s < p.nb) {
      const BStream& b = p.bs[s];
      sm.bkv[4 * s] = b.k;
      sm.bkv[4 * s + 1] = b.v;
      sm.bkv[4 * s + 2] = b.cpk;
      sm.bkv[4 * s + 3] = b.cpv;
    }
    sm.bstate[s] = pos;
    sm.bstate[BMAX + s] = step;
    sm.bstate[2 * BMAX + s] = g0;
    sm.bstate[3 * BMAX + s] = act;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == NCW) {
    if ((tid & 31) == 0) b_producer(p, sm, blockIdx.x, gridDim.x);
    __syncwarp();
  } else if (warp == NCW + 1) {
    if ((tid & 31) == 0) b_mma(p, sm, blockIdx.x, gridDim.x);
    __syncwarp();
  } else if (warp == NCW + 2) {
    if ((tid & 31) == 0) b_aloader(p, sm, blockIdx.x, gridDim.x);
    __syncwarp();
  } else {
    Cons cs;
    cs.slot = 0;
    cs.round = 0;
    cs.bar_target = 0;
    cs.dk = 0;
    cs.gi = 0;
    cs.pn = 0;
    cs.go_next = 0;
    cs.go_sent = 0;
    bool ok;
    if (p.mode == MODE_B_FRAME)
      ok = b_frame(p, sm, cs);
    else if (p.mode == MODE_B_PREFILL)
      ok = b_prefill(p, sm, cs);
    else if (p.mode == MODE_B_PREFILL_DENSE)
      ok = b_prefill_dense(p, sm, cs);
    else
      ok = b_first_token(p, sm, cs);
    if (!ok) *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    tc_fence_before();
  }
  __syncthreads();
  if (warp == NCW + 1) {
    tc_fence_after();
    tmem_dealloc(sm.tmem_base, TMEM_COLS);
  }
  // no CTA leaves while another CTA of its cluster may still read its shared memory
  cluster_sync_all();
}
