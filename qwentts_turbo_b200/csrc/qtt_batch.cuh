// Batched decode on 5th-generation tensor cores (tcgen05). Included by qtt_kernel.cu: it is
// the same translation unit as the batch-1 kernel and uses its grid barrier, attention work
// items, sampler, head masks and stage helpers.
//
// One cooperative launch of qtt_batch_kernel runs one program for B <= 64 utterances: a frame
// of every utterance (MODE_B_FRAME), one context step of the backbone prefill (MODE_B_PREFILL)
// or the first group-0 token after the prefill (MODE_B_HEAD). The weights are streamed once
// per program for the whole batch. Every projection is a GEMM
//     D[tokens x rows] = A[tokens x K] * W[rows x K]^T
//   * W: this CTA's rows of the matrix in blocks of 16. The producer warp streams them as 2-D
//     TMA boxes of 16 rows x 64 columns with the 128-byte swizzle (two per K step of 128) into a
//     4-slot ring and runs ahead across grid barriers (weights do not depend on activations).
//   * A: the activations of all tokens as two bf16 planes, hi = bf16(v) and lo = bf16(v - hi),
//     written to global memory by the stage that produced them (row = token, plane 1 TBMAX rows
//     below plane 0). After the stage's grid barrier the activation-loader warp streams them with
//     2-D TMA boxes (64 columns x 64 tokens per plane; one slot per 64-token tile and K step of
//     128 = two 128-byte swizzle atoms) into a 3-slot ring, independently of the MMA issue.
//   * D: fp32 in tensor memory, N = 16..64 columns. An activation slot holds a 64-token tile's
//     hi plane in rows 0..63 and its lo plane in rows 64..127, so one M = 128 tcgen05.mma per
//     K sub-step of 16 gives D lane t = W hi[t] and lane 64 + t = W lo[t]; the epilogue adds
//     them: D = W (hi + lo), ~16 mantissa bits of the activations, close to an fp32 GEMV.
// The epilogue warps read D with tcgen05.ld (warp 4j + q owns tile j's token lanes 32q..32q+31,
// one thread per token), apply the deferred RMSNorm scale and the stage's elementwise work, and
// write the next GEMM's A planes. Sums of squares for the next RMSNorm are accumulated per token with
// 64-bit fixed-point atomics (order independent).
//
// Stages of a code-predictor pass: INPUT (embedding rows -> x, A planes, sums of squares) |
// per layer QKV | attention | O (+ residual) | gate/up | down (+ residual) | NORM | HEAD; a
// frame adds COMBINE (the 16-embedding sum + text row) before the backbone layers and the
// codec head (+ sampler) at the end.

constexpr int KSUB = 64;                  // K elements of one 128-byte swizzle atom row
constexpr int NSUB = 2;                   // atoms per pipeline step
constexpr int KSTEP = KSUB * NSUB;        // K elements per pipeline step
constexpr int WBOX = 16;                  // weight rows per TMA box
constexpr int WS_BYTES = NSUB * 64 * 128; // weight slot: per atom up to 64 rows of 128 bytes
constexpr int NWS = 4;
constexpr int APLANE_BYTES = 64 * 128;    // one plane of an activation atom: 64 token rows
constexpr int ASUB_BYTES = 2 * APLANE_BYTES;  // hi plane, then lo plane
constexpr int AS_BYTES = NSUB * ASUB_BYTES;
constexpr int NAS = 3;
constexpr int NCHAIN = 1;                 // accumulators per tile
constexpr int DCOLS = 64;                 // tensor-memory columns of one accumulator (N <= 64)
constexpr uint32_t TMEM_COLS = 2 * NCHAIN * DCOLS;   // 2 tiles x 64 columns
constexpr int BATT_SPAN = 96;             // backbone attention: positions per work item (target)
// An M = 128 MMA reads the whole slot: rows 0..63 (hi plane) and 64..127 (lo plane).
static_assert(NWS * WS_BYTES + NAS * AS_BYTES <= NSLOTS * SLOT_BYTES, "batched rings fit the ring region");
constexpr int YLO_STRIDE = DCOLS + 1;     // epilogue staging of the lo lanes: [2 tiles][64 tokens][65]
// mbarriers in sm.bbar (all with one expected arrival)
enum : int {
  BB_WFULL = 0,                  // weight slot filled (producer expect_tx + TMA bytes)
  BB_WEMPTY = BB_WFULL + NWS,    // weight slot consumed (tcgen05.commit)
  BB_AFULL = BB_WEMPTY + NWS,    // activation slot filled
  BB_AEMPTY = BB_AFULL + NAS,    // activation slot consumed
  BB_ACCFULL = BB_AEMPTY + NAS,  // D complete (tcgen05.commit after the last K step)
  BB_ACCEMPTY,                   // D read by the epilogue
  BB_GO,                         // the stage's grid barrier passed: A planes are complete
  BB_DRAIN,                      // every MMA done (exit)
  BB_N
};
static_assert(BB_N <= 32, "batched mbarriers");

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

// Work of a CTA in a GEMM stage. Rows are grouped into row blocks of `nb` blocks of 16 rows
// (gate/up: 16 intermediate columns, i.e. 16 gate + 16 up rows per block), N <= 64 columns of D;
// for o_proj and down the K steps are split too: CTA c < R * nk takes row block
// c / nk and K steps [ks0, ks1) of slice c % nk, and the last CTA of a row block to finish sums
// the slices' partial results (fixed order) and runs the epilogue.
struct BSplit {
  int b0, nb;        // first 16-row block, blocks (0: idle in this stage)
  int rb, kspl, nk;  // row block, K slice, K slices per row block
  int ks0, ks1;      // K steps of this CTA
};
__device__ __forceinline__ BSplit bg_split(const Params& p, const BGemm& g, int cta, int G) {
  int total;
  switch (g.kind) {
    case BK_QKV: total = QKV_ROWS / WBOX; break;
    case BK_GU: total = INTER / WBOX; break;
    case BK_HEAD: total = (g.hidx == 0 ? p.vocab : p.cp_vocab) / WBOX; break;
    default: total = HID / WBOX; break;
  }
  // o_proj and down (1024 rows, K = 2048 / 3072): 16 row blocks of 64 rows, K split over the
  // other CTAs; the rest: ceil(blocks / CTAs) blocks per CTA, no split
  const bool ksplit = g.kind == BK_O || g.kind == BK_D;
  const int bpc = ksplit ? 4 : (total + G - 1) / G;
  const int R = total / bpc;
  const int nks = (g.kind == BK_O ? QSZ : g.kind == BK_D ? INTER : HID) / (KSUB * NSUB);
  int nk = ksplit ? G / R : 1;
  nk = nk < 1 ? 1 : (nk > nks ? nks : nk);
  BSplit s;
  s.nk = nk;
  if (cta < R * nk) {
    s.rb = cta / nk;
    s.kspl = cta - s.rb * nk;
    s.b0 = s.rb * bpc;
    s.nb = bpc;
    s.ks0 = split_lo(nks, nk, s.kspl);
    s.ks1 = split_lo(nks, nk, s.kspl + 1);
  } else {
    s.rb = s.kspl = s.b0 = s.nb = s.ks0 = s.ks1 = 0;
  }
  return s;
}
__device__ __forceinline__ int bg_N(int kind, int nb) { return (kind == BK_GU ? 2 : 1) * WBOX * nb; }

// Tensor map and row of weight box i of a stage (gate/up: boxes 0..nb-1 gate, nb..2nb-1 up).
__device__ __forceinline__ void bg_wbox(const Params& p, const BGemm& g, int b0, int nb, int i, const uint8_t*& map,
                                        int& y) {
  const int base = g.li * NLMAPS;
  switch (g.kind) {
    case BK_QKV: {
      const int r = WBOX * (b0 + i);
      const int m = r < QSZ ? 0 : (r < QSZ + KVSZ ? 1 : 2);
      y = r - (m == 0 ? 0 : (m == 1 ? QSZ : QSZ + KVSZ));
      map = bmap(p, base + m);
      break;
    }
    case BK_O: map = bmap(p, base + 3); y = WBOX * (b0 + i); break;
    case BK_GU:
      if (i < nb) {
        map = bmap(p, base + 4);
        y = WBOX * (b0 + i);
      } else {
        map = bmap(p, base + 5);
        y = WBOX * (b0 + i - nb);
      }
      break;
    case BK_D: map = bmap(p, base + 6); y = WBOX * (b0 + i); break;
    default: map = bmap(p, bmap_head(p, g.hidx)); y = WBOX * (b0 + i); break;
  }
}

// The GEMM stages of the launch's program, in order; f returns false to stop.
template <class F>
__device__ void b_walk(const Params& p, F&& f) {
  const int B = p.nb;
  auto layer = [&](int li, int T) -> bool {
    return f(BGemm{BK_QKV, li, 0, T}) && f(BGemm{BK_O, li, 0, T}) && f(BGemm{BK_GU, li, 0, T}) &&
           f(BGemm{BK_D, li, 0, T});
  };
  if (p.mode == MODE_B_FRAME) {
    for (int g = 0; g < NCPHEADS; ++g) {
      for (int l = 0; l < p.n_cp; ++l)
        if (!layer(p.n_bb + l, g == 0 ? 2 * B : B)) return;
      if (!f(BGemm{BK_HEAD, 0, 1 + g, B})) return;
    }
    for (int l = 0; l < p.n_bb; ++l)
      if (!layer(l, B)) return;
    f(BGemm{BK_HEAD, 0, 0, B});
  } else if (p.mode == MODE_B_PREFILL) {
    for (int l = 0; l < p.n_bb; ++l)
      if (!layer(l, B)) return;
  } else {
    f(BGemm{BK_HEAD, 0, 0, B});
  }
}

// ------------------------------------------------------------------------------------------
// Producer warp (one thread): weight boxes of every GEMM stage into the 8-slot ring.
// ------------------------------------------------------------------------------------------
__device__ void b_producer(const Params& p, Smem& sm, int cta, int G) {
  uint8_t* wring = reinterpret_cast<uint8_t*>(sm.ring);
  uint32_t m = 0;
  int* err = p.w.err;
  b_walk(p, [&](const BGemm& g) -> bool {
    const BSplit sp = bg_split(p, g, cta, G);
    const int b0 = sp.b0, nb = sp.nb;
    if (nb == 0) return true;
    const int N = bg_N(g.kind, nb), nbox = N / WBOX;
    for (int ks = sp.ks0; ks < sp.ks1; ++ks, ++m) {
      const uint32_t slot = m % NWS, round = m / NWS;
      if (!mbar_spin(&sm.bbar[BB_WEMPTY + slot], (round & 1u) ^ 1u, &sm.abort)) {
        if (!*reinterpret_cast<volatile int*>(&sm.abort)) set_error(err, DEV_ERR_EMPTY_TIMEOUT);
        return false;
      }
      mbar_arrive_expect_tx(&sm.bbar[BB_WFULL + slot], static_cast<uint32_t>(NSUB * N * 128));
      for (int i = 0; i < nbox; ++i) {
        const uint8_t* map;
        int y;
        bg_wbox(p, g, b0, nb, i, map, y);
        if (ks == sp.ks0) tensormap_acquire(map);   // the host's copy of the map, before its first use
        for (int a = 0; a < NSUB; ++a)
          tma_load_2d(wring + slot * WS_BYTES + a * (N * 128) + i * (WBOX * 128), map, ks * KSTEP + a * KSUB, y,
                      &sm.bbar[BB_WFULL + slot]);
      }
    }
    return true;
  });
  // drain: no box may still be landing in shared memory when the CTA exits
  int zero = 0;
  for (uint32_t i = (m > NWS ? m - NWS : 0u); i < m; ++i)
    mbar_spin(&sm.bbar[BB_WFULL + i % NWS], (i / NWS) & 1u, &zero);
}

// ------------------------------------------------------------------------------------------
// Activation-loader warp (one thread): after each GEMM stage's grid barrier, the A planes of
// every (K step, 64-token tile) into the 6-slot ring.
// ------------------------------------------------------------------------------------------
__device__ void b_aloader(const Params& p, Smem& sm, int cta, int G) {
  uint8_t* aring = reinterpret_cast<uint8_t*>(sm.ring) + NWS * WS_BYTES;
  uint32_t na = 0, n = 0;
  int* err = p.w.err;
  for (int b = 0; b < 2; ++b) tensormap_acquire(bmap(p, bmap_abuf(p, b, false)));
  b_walk(p, [&](const BGemm& g) -> bool {
    const BSplit sp = bg_split(p, g, cta, G);
    if (sp.nb == 0) return true;
    const int ntiles = (g.T + 63) >> 6;
    const uint8_t* amap = bmap(p, bmap_abuf(p, bg_abuf(g.kind), false));
    // the consumers arrive on GO after the stage's grid barrier: the A planes are complete
    if (!mbar_spin(&sm.bbar[BB_GO], n & 1u, &sm.abort)) {
      if (!*reinterpret_cast<volatile int*>(&sm.abort)) set_error(err, DEV_ERR_FULL_TIMEOUT);
      return false;
    }
    ++n;
    fence_proxy_async_global();
    for (int ks = sp.ks0; ks < sp.ks1; ++ks)
      for (int j = 0; j < ntiles; ++j, ++na) {
        const uint32_t slot = na % NAS, round = na / NAS;
        if (!mbar_spin(&sm.bbar[BB_AEMPTY + slot], (round & 1u) ^ 1u, &sm.abort)) {
          if (!*reinterpret_cast<volatile int*>(&sm.abort)) set_error(err, DEV_ERR_EMPTY_TIMEOUT);
          return false;
        }
        mbar_arrive_expect_tx(&sm.bbar[BB_AFULL + slot], static_cast<uint32_t>(AS_BYTES));
        for (int a = 0; a < NSUB; ++a) {
          uint8_t* dst = aring + slot * AS_BYTES + a * ASUB_BYTES;
          tma_load_2d(dst, amap, ks * KSTEP + a * KSUB, 64 * j, &sm.bbar[BB_AFULL + slot]);
          tma_load_2d(dst + APLANE_BYTES, amap, ks * KSTEP + a * KSUB, TBMAX + 64 * j, &sm.bbar[BB_AFULL + slot]);
        }
      }
    return true;
  });
  int zero = 0;
  for (uint32_t i = (na > NAS ? na - NAS : 0u); i < na; ++i)
    mbar_spin(&sm.bbar[BB_AFULL + i % NAS], (i / NAS) & 1u, &zero);
}

// ------------------------------------------------------------------------------------------
// MMA warp (one thread): tcgen05.mma of every GEMM stage.
// ------------------------------------------------------------------------------------------
__device__ void b_mma(const Params& p, Smem& sm, int cta, int G) {
  const uint32_t wbase = smem_u32(sm.ring), abase = wbase + NWS * WS_BYTES;
  const uint32_t tmem = sm.tmem_base;
  uint32_t m = 0, ua = 0, n = 0;
  bool any = false;
  int* err = p.w.err;
  auto fail_mma = [&](int code) {
    if (!*reinterpret_cast<volatile int*>(&sm.abort)) {
      set_error(err, code);
      *reinterpret_cast<volatile int*>(&sm.abort) = 1;
    }
  };
  b_walk(p, [&](const BGemm& g) -> bool {
    const BSplit sp = bg_split(p, g, cta, G);
    if (sp.nb == 0) return true;
    const int N = bg_N(g.kind, sp.nb), nks = sp.ks1 - sp.ks0, ntiles = (g.T + 63) >> 6;
    const uint32_t idesc = umma_idesc_bf16(128, N);
    // profiling (CTA 0, dbg_marks set), dbg_marks[8192 + 8 n]: accumulator free, first
    // activation slot ready, last MMA issued; the consumers add GO, D ready, epilogue done,
    // barrier passed
    const bool prof = p.dbg_marks != nullptr && cta == 0 && static_cast<int>(8192 + 8 * n + 7) < p.dbg_marks_len;
    unsigned long long tw = 0, ta = 0, t_first = 0;
    long long cyc_fence = 0, cyc_mma = 0, cyc_commit = 0;
    // the previous stage's epilogue has read D
    if (!mbar_spin(&sm.bbar[BB_ACCEMPTY], (n & 1u) ^ 1u, &sm.abort)) {
      fail_mma(DEV_ERR_FULL_TIMEOUT);
      return false;
    }
    tc_fence_after();
    const unsigned long long t_start = prof ? globaltimer_ns() : 0ull;
    for (int ks = 0; ks < nks; ++ks) {   // ks: index within this CTA's K slice
      const uint32_t ws = m % NWS, wr = m / NWS;
      unsigned long long t0 = prof ? globaltimer_ns() : 0ull;
      if (!mbar_spin(&sm.bbar[BB_WFULL + ws], wr & 1u, &sm.abort)) {
        fail_mma(DEV_ERR_FULL_TIMEOUT);
        return false;
      }
      if (prof && ks > 0) tw += globaltimer_ns() - t0;
      const uint32_t wa = wbase + ws * WS_BYTES;
      for (int j = 0; j < ntiles; ++j, ++ua) {
        const uint32_t as = ua % NAS, ar = ua / NAS;
        t0 = prof ? globaltimer_ns() : 0ull;
        if (!mbar_spin(&sm.bbar[BB_AFULL + as], ar & 1u, &sm.abort)) {
          fail_mma(DEV_ERR_FULL_TIMEOUT);
          return false;
        }
        if (prof) {
          if (ks > 0) ta += globaltimer_ns() - t0;
          if (t_first == 0ull) t_first = globaltimer_ns();
        }
        long long c0 = prof ? clock64() : 0;
        tc_fence_after();
        long long c1 = prof ? clock64() : 0;
        const uint32_t aa = abase + as * AS_BYTES;
        // one M = 128 MMA covers both planes: A rows 0..63 = hi, 64..127 = lo of the tile's tokens
        const uint32_t dt = tmem + j * NCHAIN * DCOLS;
#pragma unroll
        for (int a = 0; a < NSUB; ++a)
#pragma unroll
          for (int kk = 0; kk < KSUB / 16; ++kk)   // the first MMA of the slice overwrites D
            tc_mma_bf16(dt, umma_desc_sw128(aa + a * ASUB_BYTES + kk * 32),
                        umma_desc_sw128(wa + a * (N * 128) + kk * 32), idesc, (ks | a | kk) != 0 ? 1u : 0u);
        long long c2 = prof ? clock64() : 0;
        any = true;
        tc_commit(&sm.bbar[BB_AEMPTY + as]);
        long long c3 = prof ? clock64() : 0;
        if (prof) {
          cyc_fence += c1 - c0;
          cyc_mma += c2 - c1;
          cyc_commit += c3 - c2;
        }
      }
      long long c4 = prof ? clock64() : 0;
      tc_commit(&sm.bbar[BB_WEMPTY + ws]);
      if (prof) cyc_commit += clock64() - c4;
      ++m;
    }
    tc_commit(&sm.bbar[BB_ACCFULL]);
    if (prof) {
      p.dbg_marks[8192 + 8 * n + 0] = t_start;
      p.dbg_marks[8192 + 8 * n + 1] = t_first;
      p.dbg_marks[8192 + 8 * n + 2] = globaltimer_ns();
      p.dbg_marks[8192 + 8 * n + 7] = (tw << 32) | (ta & 0xFFFFFFFFull);
      if (static_cast<int>(12288 + 4 * n + 3) < p.dbg_marks_len) {
        p.dbg_marks[12288 + 4 * n + 0] = cyc_fence;
        p.dbg_marks[12288 + 4 * n + 1] = cyc_mma;
        p.dbg_marks[12288 + 4 * n + 2] = cyc_commit;
        p.dbg_marks[12288 + 4 * n + 3] = nks;
      }
    }
    ++n;
    return true;
  });
  if (any) {   // every issued MMA done before the accumulator is freed
    int zero = 0;
    tc_commit(&sm.bbar[BB_DRAIN]);
    mbar_spin(&sm.bbar[BB_DRAIN], 0u, &zero);
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

// Columns [c, c + 16) of D for this thread's token lane.
__device__ __forceinline__ void b_ld16(uint32_t taddr, int c, float (&v)[16]) { tmem_ld16(taddr + c, v); }

// Columns [c, c + 16) of D for token t: hi lanes (chains added) + the lo lanes staged in smem.
// hilo_store of 16 consecutive columns (col0 a multiple of 16): 32-byte stores per plane.
__device__ __forceinline__ void hilo_store16(bf16* buf, int t, int col0, const float (&v)[16]) {
  uint32_t hi[8], lo[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bf16 h0 = __float2bfloat16_rn(v[2 * i]), h1 = __float2bfloat16_rn(v[2 * i + 1]);
    const bf16 l0 = __float2bfloat16_rn(v[2 * i] - __bfloat162float(h0));
    const bf16 l1 = __float2bfloat16_rn(v[2 * i + 1] - __bfloat162float(h1));
    hi[i] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
    lo[i] = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
  }
  uint4* ph = reinterpret_cast<uint4*>(buf + static_cast<size_t>(t) * ABUF_LD + col0);
  uint4* pl = reinterpret_cast<uint4*>(buf + static_cast<size_t>(TBMAX + t) * ABUF_LD + col0);
  ph[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  ph[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
  pl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  pl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
}
// 16 consecutive fp32 from global (L2) / bf16 weights as fp32.
__device__ __forceinline__ void ld16_f32(const float* src, float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(src + i));
    v[i] = a.x; v[i + 1] = a.y; v[i + 2] = a.z; v[i + 3] = a.w;
  }
}
__device__ __forceinline__ void ld16_bf16(const bf16* src, float (&v)[16]) {
  const uint4 a = reinterpret_cast<const uint4*>(src)[0], b = reinterpret_cast<const uint4*>(src)[1];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = bf16_lo(w[i]);
    v[2 * i + 1] = bf16_hi(w[i]);
  }
}
__device__ __forceinline__ void st16_f32(float* dst, const float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i += 4) __stcg(reinterpret_cast<float4*>(dst + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
}

// Columns [c, c + 16) of D for the thread's token. TMEM mode: the hi lanes (chains added) + the
// lo lanes staged in shared memory. Summed mode (K split): the row of the slices' sum.
struct BAcc {
  uint32_t taddr;      // this thread's hi lane, tile base column
  const float* lo;     // staged lo lane row of this token
  const float* y;      // summed row of this token, or nullptr
  __device__ __forceinline__ void ld16(int c, float (&v)[16]) const {
    if (y != nullptr) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = y[c + i];
      return;
    }
    b_ld16(taddr, c, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += lo[c + i];
  }
};

// Consumer side of one GEMM stage: release the activation loader, wait for D, stage the lo
// lanes (warps 2, 3 of each 64-token tile) in shared memory, then on the hi lanes (warps 0, 1 of
// tile 0 and 4, 5 of tile 1, all lanes taking part in the tensor-memory loads):
//   * one K slice: the epilogue epi(t, acc, b0, nb, N) directly;
//   * K split: the slice's partial D rows to global memory; the last CTA of the row block
//     (counter) sums the slices in slice order and runs the epilogue.
// Then free D and the grid barrier.
template <class EPI>
__device__ bool b_gemm(const Params& p, Smem& sm, Cons& cs, const BGemm& g, uint32_t& gemm_n, EPI&& epi) {
  const BSplit sp = bg_split(p, g, cs.cta, cs.G);
  const bool prof = p.dbg_marks != nullptr && cs.cta == 0 && cs.tid == 0 &&
                    static_cast<int>(8192 + 8 * gemm_n + 7) < p.dbg_marks_len;
  if (sp.nb == 0) return grid_sync(p, sm, cs);
  const int N = bg_N(g.kind, sp.nb);
  if (prof) p.dbg_marks[8192 + 8 * gemm_n + 3] = globaltimer_ns();
  if (cs.tid == 0) mbar_arrive(&sm.bbar[BB_GO]);
  bool freed = false;
  if (!mbar_wait(&sm.bbar[BB_ACCFULL], gemm_n & 1u, &sm.abort)) {
    if (!aborted(sm)) fail(p, sm, DEV_ERR_FULL_TIMEOUT);
  } else {
    if (prof) p.dbg_marks[8192 + 8 * gemm_n + 4] = globaltimer_ns();
    tc_fence_after();
    const int q = cs.warp & 3, j = cs.warp >> 2;   // lane quarter, 64-token tile
    float* ylo = sm.xs;                            // [2][64][YLO_STRIDE]
    const uint32_t tq = sm.tmem_base + (static_cast<uint32_t>(32 * q) << 16) + j * NCHAIN * DCOLS;
    if (j < 2 && q >= 2 && 64 * j + 32 * (q - 2) < g.T) {
      float* row = ylo + (j * 64 + 32 * (q - 2) + cs.lane) * YLO_STRIDE;
      for (int c = 0; c < N; c += 16) {
        float v[16];
        b_ld16(tq, c, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) row[c + i] = v[i];
      }
    }
    named_sync(1, NCT);
    const bool mine = j < 2 && q < 2 && 64 * j + 32 * q < g.T;
    const int t = 64 * j + 32 * q + cs.lane;
    const BAcc dacc{tq, ylo + (j * 64 + 32 * q + cs.lane) * YLO_STRIDE, nullptr};
    if (sp.nk == 1) {
      if (mine) epi(t, dacc, sp.b0, sp.nb, N);
      tc_fence_before();
    } else {
      if (mine) {
        float* dst = p.bw.kpart + (static_cast<size_t>(cs.cta) * TBMAX + t) * DCOLS;
        for (int c = 0; c < N; c += 16) {
          float v[16];
          dacc.ld16(c, v);
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            __stcg(reinterpret_cast<float4*>(dst + c + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
        }
      }
      tc_fence_before();
      named_sync(1, NCT);
      if (cs.tid == 0) {
        mbar_arrive(&sm.bbar[BB_ACCEMPTY]);   // D is no longer needed
        __threadfence();
        const uint32_t old = atomicAdd(p.bw.kcnt + sp.rb, 1u);
        const bool last = old == static_cast<uint32_t>(sp.nk - 1);
        if (last) atomicExch(p.bw.kcnt + sp.rb, 0u);
        sm.bcast[0] = last ? 1 : 0;
        __threadfence();
      }
      freed = true;
      named_sync(1, NCT);
      if (sm.bcast[0]) {
        float* y = sm.xs;   // [T][YLO_STRIDE]: the slices' sum (the lo staging is no longer read)
        const float* base = p.bw.kpart + static_cast<size_t>(sp.rb * sp.nk) * TBMAX * DCOLS;
        const int n4 = N / 4;
        for (int e = cs.tid; e < g.T * n4; e += NCT) {
          const int tt = e / n4, c = 4 * (e - tt * n4);
          const float* src = base + static_cast<size_t>(tt) * DCOLS + c;
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int k0 = 0; k0 < sp.nk; k0 += 4) {   // four slices' loads in flight, added in order
            float4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (k0 + k < sp.nk)
                v[k] = __ldcg(reinterpret_cast<const float4*>(src + static_cast<size_t>(k0 + k) * TBMAX * DCOLS));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (k0 + k < sp.nk) {
                a.x += v[k].x; a.y += v[k].y; a.z += v[k].z; a.w += v[k].w;
              }
          }
          float* d = y + tt * YLO_STRIDE + c;
          d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w;
        }
        named_sync(1, NCT);
        if (mine) epi(t, BAcc{0u, nullptr, y + t * YLO_STRIDE}, sp.b0, sp.nb, N);
      }
    }
  }
  named_sync(1, NCT);
  if (prof) p.dbg_marks[8192 + 8 * gemm_n + 5] = globaltimer_ns();
  if (cs.tid == 0 && !freed) mbar_arrive(&sm.bbar[BB_ACCEMPTY]);
  const bool ok = grid_sync(p, sm, cs);
  if (prof) p.dbg_marks[8192 + 8 * gemm_n + 6] = globaltimer_ns();
  gemm_n++;
  return ok;
}

// Sums-of-squares buffer written by the next producing stage (INPUT, O, down); that stage also
// clears the buffer after it, last read two producing stages earlier. The host clears all three
// before every launch.
__device__ __forceinline__ unsigned long long* b_ssq_next(const Params& p, Cons& cs) {
  cs.dk = (cs.dk + 1) % 3;
  unsigned long long* w = p.bw.ssq + cs.dk * TBMAX;
  if (cs.cta == 0)
    for (int t = cs.tid; t < TBMAX; t += NCT) __stcg(p.bw.ssq + ((cs.dk + 1) % 3) * TBMAX + t, 0ull);
  return w;
}
__device__ __forceinline__ const unsigned long long* b_ssq_cur(const Params& p, const Cons& cs) {
  return p.bw.ssq + cs.dk * TBMAX;
}
__device__ __forceinline__ void b_ssq_add(unsigned long long* ssq, int t, double ss) {
  atomicAdd(ssq + t, static_cast<unsigned long long>(__double2ll_rn(ss * 4294967296.0)));
}

// Elementwise stages over T tokens x HID columns: CTA c owns 8-column units
// [split_lo(128, G, c), split_lo(128, G, c + 1)); one thread per (token, unit).
template <class F>
__device__ void b_elementwise(Cons& cs, int T, F&& f) {
  const int u0 = split_lo(HID / 8, cs.G, cs.cta), u1 = split_lo(HID / 8, cs.G, cs.cta + 1);
  const int nu = u1 - u0;
  for (int e = cs.tid; e < T * nu; e += NCT) {
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
  return grid_sync(p, sm, cs);
}

// NORM: head input A = bf16(RMSNorm(h)) (lo plane 0) for head tokens i < B taken from stack
// token tmul * i + toff; hstate (backbone): the fp32 normed hidden of each active utterance.
__device__ bool b_norm(const Params& p, Smem& sm, Cons& cs, const float* h, int tmul, int toff, const bf16* w,
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
  return grid_sync(p, sm, cs);
}

// Attention of one layer for every utterance. Code predictor: one item per (utterance, KV
// head), NT = 2 tokens in the first pass. Backbone: (utterance, KV head, chunk) items over each
// active utterance's own context, combined by the last item of a head.
__device__ bool b_attention(const Params& p, Smem& sm, Cons& cs, int li, bool cp, int pass) {
  const BState bst = bstate(sm);
  const int B = p.nb;
  if (cp) {
    const int l = li - p.n_bb;
    const LayerW* L = p.cp_layers + l;
    const int NT = pass == 0 ? 2 : 1, p0 = pass == 0 ? 0 : pass + 1;
    for (int item = cs.cta; item < B * NKVH; item += cs.G) {
      const int s = item / NKVH, h = item - s * NKVH;
      AttIO io;
      io.qkv = p.bw.qkv + static_cast<size_t>(s * NT) * QKV_ROWS;
      const size_t off = (static_cast<size_t>(l) * NKVH + h) * p.cp_max_seq * HD;
      io.kb = reinterpret_cast<uint8_t*>(p.bs[s].cpk + off);
      io.vb = reinterpret_cast<uint8_t*>(p.bs[s].cpv + off);
      io.out = nullptr;
      io.hilo = p.bw.abuf[1];
      io.tok0 = s * NT;
      io.prt = nullptr;
      io.cnt = nullptr;
      const bool ok = NT == 2 ? att_item<2, true, false>(p, sm, cs, L, io, p0, h, 0, 1, 0, p0 + 2, true)
                              : att_item<1, true, false>(p, sm, cs, L, io, p0, h, 0, 1, 0, p0 + 1, true);
      if (!ok) return false;
    }
  } else {
    const LayerW* L = p.bb_layers + li;
    int total = 0;
    for (int s = 0; s < B; ++s)
      if (bst.act[s]) total += NKVH * min(MAX_ATT_CHUNKS, (bst.pos[s] + 1 + BATT_SPAN - 1) / BATT_SPAN);
    for (int item = cs.cta; item < total; item += cs.G) {
      int idx = item, s = 0, nch = 1;
      for (; s < B; ++s) {
        if (!bst.act[s]) continue;
        nch = min(MAX_ATT_CHUNKS, (bst.pos[s] + 1 + BATT_SPAN - 1) / BATT_SPAN);
        if (idx < NKVH * nch) break;
        idx -= NKVH * nch;
      }
      const int h = idx / nch, c = idx - h * nch;
      const int S = bst.pos[s] + 1, chunk = (S + nch - 1) / nch;
      const int s0 = c * chunk, s1 = min(S, s0 + chunk);
      if (chunk > ATT_CHMAX) {
        fail(p, sm, DEV_ERR_BAD_POSITION);
        return false;
      }
      AttIO io;
      io.qkv = p.bw.qkv + static_cast<size_t>(s) * QKV_ROWS;
      const size_t off = (static_cast<size_t>(li) * NKVH + h) * p.bb_max_seq * HD;
      io.kb = reinterpret_cast<uint8_t*>(p.bs[s].k + off);
      io.vb = reinterpret_cast<uint8_t*>(p.bs[s].v + off);
      io.out = nullptr;
      io.hilo = p.bw.abuf[1];
      io.tok0 = s;
      io.prt = p.bw.prt + static_cast<size_t>(s) * NQH * MAX_ATT_CHUNKS * PRT_STRIDE;
      io.cnt = p.bw.att_cnt + s * NKVH + h;
      if (!att_item<1, false, false>(p, sm, cs, L, io, bst.pos[s], h, c, nch, s0, s1, c == 0)) return false;
    }
  }
  return grid_sync(p, sm, cs);
}

// One decoder layer of the batch: QKV | attention | O | gate/up | down.
__device__ bool b_layer(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, int li, bool cp, int pass, int T,
                        const float* hin, float* hout, const bf16* next_norm) {
  const LayerW* L = (cp ? p.cp_layers + (li - p.n_bb) : p.bb_layers + li);
  const float eps = p.eps;
  // ---- QKV (deferred input norm)
  {
    const unsigned long long* ssq = b_ssq_cur(p, cs);
    if (!b_gemm(p, sm, cs, BGemm{BK_QKV, li, 0, T}, gn, [&](int t, const BAcc& acc, int b0, int nb, int N) {
          const float rs = t < T ? b_rstd(ssq, t, eps) : 0.f;
          for (int c0 = 0; c0 < N; c0 += 16) {
            float v[16];
            acc.ld16(c0, v);
            if (t < T) {
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] *= rs;
              st16_f32(p.bw.qkv + static_cast<size_t>(t) * QKV_ROWS + WBOX * b0 + c0, v);
            }
          }
        }))
      return false;
  }
  // ---- attention -> A planes of o_proj
  if (!b_attention(p, sm, cs, li, cp, pass)) return false;
  // ---- o_proj + residual -> hmid, A planes of gate/up (post-attention norm), sums of squares
  {
    unsigned long long* ssq = b_ssq_next(p, cs);
    if (!b_gemm(p, sm, cs, BGemm{BK_O, li, 0, T}, gn, [&](int t, const BAcc& acc, int b0, int nb, int N) {
          double ss = 0.0;
          for (int c0 = 0; c0 < N; c0 += 16) {
            float v[16];
            acc.ld16(c0, v);
            if (t < T) {
              const int r0 = WBOX * b0 + c0;
              float res[16], wn[16], a[16];
              ld16_f32(hin + t * HID + r0, res);
              ld16_bf16(L->post_norm + r0, wn);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                v[i] += res[i];
                a[i] = v[i] * wn[i];
                ss = fma(static_cast<double>(v[i]), static_cast<double>(v[i]), ss);
              }
              st16_f32(p.bw.hmid + t * HID + r0, v);
              hilo_store16(p.bw.abuf[0], t, r0, a);
            }
          }
          if (t < T) b_ssq_add(ssq, t, ss);
        }))
      return false;
  }
  // ---- gate/up + SiLU (deferred post-attention norm) -> A planes of down
  {
    const unsigned long long* ssq = b_ssq_cur(p, cs);
    if (!b_gemm(p, sm, cs, BGemm{BK_GU, li, 0, T}, gn, [&](int t, const BAcc& acc, int b0, int nb, int N) {
          const float rs = t < T ? b_rstd(ssq, t, eps) : 0.f;
          for (int c0 = 0; c0 < WBOX * nb; c0 += 16) {
            float gv[16], uv[16];
            acc.ld16(c0, gv);
            acc.ld16(WBOX * nb + c0, uv);
            if (t < T) {
              float m[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float gg = gv[i] * rs, uu = uv[i] * rs;
                m[i] = (gg / (1.0f + expf(-gg))) * uu;
              }
              hilo_store16(p.bw.abuf[1], t, WBOX * b0 + c0, m);
            }
          }
        }))
      return false;
  }
  // ---- down + residual -> layer output, A planes of the next layer (its input norm), sums
  {
    unsigned long long* ssq = b_ssq_next(p, cs);
    if (!b_gemm(p, sm, cs, BGemm{BK_D, li, 0, T}, gn, [&](int t, const BAcc& acc, int b0, int nb, int N) {
          double ss = 0.0;
          for (int c0 = 0; c0 < N; c0 += 16) {
            float v[16];
            acc.ld16(c0, v);
            if (t < T) {
              const int r0 = WBOX * b0 + c0;
              float res[16], a[16];
              ld16_f32(p.bw.hmid + t * HID + r0, res);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                v[i] += res[i];
                if (!cp) v[i] = round_bf16(v[i]);
                ss = fma(static_cast<double>(v[i]), static_cast<double>(v[i]), ss);
              }
              st16_f32(hout + t * HID + r0, v);
              if (next_norm) {
                float wn[16];
                ld16_bf16(next_norm + r0, wn);
#pragma unroll
                for (int i = 0; i < 16; ++i) a[i] = v[i] * wn[i];
                hilo_store16(p.bw.abuf[0], t, r0, a);
              }
            }
          }
          if (t < T) b_ssq_add(ssq, t, ss);
        }))
      return false;
  }
  return true;
}

// Layers of a stack over T tokens whose input (x, A planes, sums of squares) is ready.
// Returns the buffer holding the last layer's output (nullptr on abort).
__device__ const float* b_stack(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, bool cp, int pass, int T) {
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
__device__ bool b_head(const Params& p, Smem& sm, Cons& cs, uint32_t& gn, int hidx, const SampleCfg& cfg, int slot) {
  const BState bst = bstate(sm);
  unsigned long long* amax = p.bw.amax + slot * TBMAX;
  if (cs.cta == 0)
    for (int t = cs.tid; t < TBMAX; t += NCT) __stcg(p.bw.amax + (slot ^ 1) * TBMAX + t, 0ull);
  return b_gemm(p, sm, cs, BGemm{BK_HEAD, 0, hidx, p.nb}, gn, [&](int t, const BAcc& acc, int b0, int nb, int N) {
    SampleCfg c = cfg;
    if (t < p.nb && hidx == 0) {
      c.seen = (c.penalty != 1.f) ? p.bs[t].st->seen : nullptr;
      c.mask_eos = (p.mode == MODE_B_HEAD) ? (p.sp.min_new_tokens > 0 ? 1 : 0)
                                           : ((bst.step[t] + 1 < p.sp.min_new_tokens) ? 1 : 0);
    }
    unsigned long long best = 0ull;
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      acc.ld16(c0, v);
      if (t < p.nb) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int row = WBOX * b0 + c0 + i;
          const float lg = round_bf16(v[i]);
          if (hidx > 0 && p.dbg_cp_logits != nullptr)   // parity tests: [B][15][cp_vocab]
            p.dbg_cp_logits[(static_cast<size_t>(t) * NCPHEADS + hidx - 1) * p.cp_vocab + row] = lg;
          if (hidx == 0 && p.dbg_g0_logits != nullptr && p.mode == MODE_B_FRAME)   // [B][vocab]
            p.dbg_g0_logits[static_cast<size_t>(t) * p.vocab + row] = lg;
          if (c.do_sample) {
            __stcg(p.bw.logits + static_cast<size_t>(t) * VMAX + row, lg);
          } else {
            const unsigned long long k = argmax_key(head_mask(c, row, lg), row);
            best = k > best ? k : best;
          }
        }
      }
    }
    if (t < p.nb && !c.do_sample && best != 0ull) atomicMax(amax + t, best);
  });
}

// Token of utterance s from head slot `slot` (greedy) or bw.tok (sampled, column col).
__device__ __forceinline__ int b_token(const Params& p, const SampleCfg& cfg, int slot, int s, int col) {
  if (!cfg.do_sample) {
    const unsigned long long k = __ldcg(p.bw.amax + slot * TBMAX + s);
    return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
  }
  return __ldcg(p.bw.tok + s * NGROUPS + col);
}

// Tokens of a head for every utterance, after its barrier, into bw.tok[s][col]: greedy from the
// packed argmax (CTA 0 copies them; the next stage reads the slot directly), sampled by one CTA
// per utterance followed by a barrier. frame_of: the Philox frame counter is step + frame_of.
__device__ bool b_tokens(const Params& p, Smem& sm, Cons& cs, int hidx, const SampleCfg& cfg, int slot, int frame_of,
                         int col) {
  const BState bst = bstate(sm);
  if (!cfg.do_sample) {
    if (cs.cta == 0)
      for (int s = cs.tid; s < p.nb; s += NCT) __stcg(p.bw.tok + s * NGROUPS + col, b_token(p, cfg, slot, s, col));
    return true;
  }
  for (int s = cs.cta; s < p.nb; s += cs.G) {
    SampleCfg c = cfg;
    if (hidx == 0) {
      c.seen = (c.penalty != 1.f) ? p.bs[s].st->seen : nullptr;
      c.mask_eos = (p.mode == MODE_B_HEAD) ? (p.sp.min_new_tokens > 0 ? 1 : 0)
                                           : ((bst.step[s] + 1 < p.sp.min_new_tokens) ? 1 : 0);
    }
    Sampling sp = p.sp;
    sp.philox_stream = p.sp.philox_stream + s;
    const int fr = p.mode == MODE_B_HEAD ? 0 : bst.step[s] + frame_of;
    c.u24 = draw_u24(sp, fr, hidx);
    const int tk = sample(p.bw.logits + static_cast<size_t>(s) * VMAX, sm, cs, c);
    if (cs.tid == 0) __stcg(p.bw.tok + s * NGROUPS + col, tk);
  }
  return grid_sync(p, sm, cs);
}

__device__ SampleCfg b_codec_cfg(const Params& p, float penalty) {
  SampleCfg c;
  c.V = p.vocab;
  c.do_sample = p.sp.do_sample;
  c.temperature = p.sp.temperature;
  c.top_k = p.sp.top_k;
  c.suppress_from = p.vocab - 1024;
  c.eos = p.sp.eos;
  c.mask_eos = 0;
  c.penalty = penalty;
  c.seen = nullptr;
  c.u24 = 0u;
  return c;
}

__device__ bool b_frame(const Params& p, Smem& sm, Cons& cs) {
  const BState bst = bstate(sm);
  const int B = p.nb;
  uint32_t gn = 0;
  if (cs.cta == 0)
    for (int s = cs.tid; s < B; s += NCT) {
      if (bst.act[s]) p.bs[s].st->seen[bst.g0[s]] = 1;   // generated_g0.append (generator.py:129)
      else if (ld_volatile_i32(&p.bs[s].st->g0) == p.sp.eos) p.bs[s].st->done = 1;   // generator.py:126
    }
  SampleCfg cpc;
  cpc.V = p.cp_vocab;
  cpc.do_sample = p.sp.cp_do_sample;
  cpc.temperature = p.sp.cp_temperature;
  cpc.top_k = p.sp.cp_top_k;
  cpc.suppress_from = p.cp_vocab;
  cpc.eos = -1;
  cpc.mask_eos = 0;
  cpc.penalty = 1.f;
  cpc.seen = nullptr;
  cpc.u24 = 0u;
  int slot = 0;
  for (int g = 0; g < NCPHEADS; ++g) {
    const int T = g == 0 ? 2 * B : B;
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
    const float* last = b_stack(p, sm, cs, gn, true, g, T);
    if (!last) return false;
    if (!b_norm(p, sm, cs, last, g == 0 ? 2 : 1, g == 0 ? 1 : 0, p.cp_norm, false)) return false;
    if (!b_head(p, sm, cs, gn, 1 + g, cpc, slot)) return false;
    if (!b_tokens(p, sm, cs, 1 + g, cpc, slot, 0, g + 1)) return false;
    slot ^= 1;
  }
  // ---- combine (generator.py:143-149,356-362): sequential bf16 adds + text row
  if (!b_input(p, sm, cs, B, p.bb_layers[0].in_norm, [&](int s, int k0, float (&v)[8]) {
        const int step = bst.step[s];
        const bf16* extra =
            step < p.bs[s].n_trailing ? p.bs[s].trailing + static_cast<size_t>(step) * HID : p.bs[s].pad;
        int toks[NCPHEADS];
        for (int q = 0; q < NCPHEADS; ++q) toks[q] = __ldcg(p.bw.tok + s * NGROUPS + q + 1);
#pragma unroll 1
        for (int i = 0; i < 8; ++i) {
          const int k = k0 + i;
          float a = __bfloat162float(p.codec_emb[static_cast<size_t>(bst.g0[s]) * HID + k]);
#pragma unroll 1
          for (int q = 0; q < NCPHEADS; ++q)
            a = round_bf16(a + __bfloat162float(p.cp_emb[q][static_cast<size_t>(toks[q]) * HID + k]));
          v[i] = round_bf16(a + __bfloat162float(extra[k]));
        }
      }))
    return false;
  const float* last = b_stack(p, sm, cs, gn, false, 0, B);
  if (!last) return false;
  if (!b_norm(p, sm, cs, last, 1, 0, p.bb_norm, true)) return false;
  const SampleCfg c = b_codec_cfg(p, p.sp.repetition_penalty);
  if (!b_head(p, sm, cs, gn, 0, c, slot)) return false;
  if (!b_tokens(p, sm, cs, 0, c, slot, 1, 0)) return false;
  // ---- frame results: codes, next g0, position, step
  if (cs.cta == 0)
    for (int s = cs.tid; s < B; s += NCT) {
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
  if (cs.cta == 0)
    for (int s = cs.tid; s < p.nb; s += NCT)
      if (bst.act[s]) p.bs[s].st->position = i + 1;
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
  if (!grid_sync(p, sm, cs)) return false;
  const SampleCfg c = b_codec_cfg(p, 1.f);
  if (!b_head(p, sm, cs, gn, 0, c, 0)) return false;
  if (!b_tokens(p, sm, cs, 0, c, 0, 0, 0)) return false;
  if (cs.cta == 0)
    for (int s = cs.tid; s < p.nb; s += NCT) {
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
    for (int i = 0; i < BB_N; ++i) mbar_init(&sm.bbar[i], 1);
    sm.abort = 0;
    sm.epoch = 0;
    fence_barrier_init();
  }
  if (warp == NCW + 1) {
    tmem_alloc(&sm.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
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
               pos < p.rope_rows && step >= 0 && step < p.max_frames)
                  ? 1
                  : 0;
      else if (p.mode == MODE_B_PREFILL)
        act = (p.b_step < p.bs[s].len) ? 1 : 0;
      else
        act = 1;
      if (p.mode == MODE_B_PREFILL) pos = p.b_step;
      if (g0 < 0 || g0 >= p.vocab) g0 = 0;
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
    cs.cta = blockIdx.x;
    cs.G = gridDim.x;
    cs.tid = tid;
    cs.warp = warp;
    cs.lane = tid & 31;
    cs.dk = 0;
    bool ok;
    if (p.mode == MODE_B_FRAME)
      ok = b_frame(p, sm, cs);
    else if (p.mode == MODE_B_PREFILL)
      ok = b_prefill(p, sm, cs);
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
}
