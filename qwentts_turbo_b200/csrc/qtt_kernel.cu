// Persistent decode kernel for Qwen3-TTS on B200 (sm_100a).
//
// One cooperative launch runs one "program": a whole 12 Hz frame (code-predictor chain of
// 15 weight sweeps + 16-embedding combine + 28-layer backbone step + codec head + group-0
// sampling), or a single backbone / code-predictor decode step (the reference's launchers,
// fused_decode_tts.cu:834-890 and fused_decode_code_predictor.cu:674-730).
//
// Grid: one CTA per SM. Each CTA has
//   * 1 producer warp: walks the same stage schedule as the consumers and streams this CTA's
//     rows of every weight matrix into a 7-slot shared-memory ring with 1-D TMA bulk copies
//     (cp.async.bulk, no multicast). Weights do not depend on activations, so the producer
//     runs ahead across grid barriers and keeps HBM busy while the consumers wait.
//   * 12 consumer warps: GEMV dot products from shared memory (fp32 accumulate), the
//     split-K attention, RMSNorms, sampling, and the grid barriers between dependent stages.
// Row partition: every matrix is split over the CTAs in contiguous row ranges, so a CTA's
// share of a matrix is one contiguous stretch of HBM.
//
// Numerics follow the reference kernels: fp32 accumulation, bf16 backbone hidden between
// layers (fused_decode_tts.cu:541), bf16 backbone KV, fp32 code-predictor hidden and KV
// (fused_decode_code_predictor.cu:553,287-289), bf16 head logits (generator.py:158,351).
#include "qtt_kernel.cuh"
#include "qtt_device.cuh"

namespace qtt {

enum StageKind : int { SK_QKV = 0, SK_O = 1, SK_GU = 2, SK_D = 3, SK_HEAD = 4, SK_GUF = 5 };

struct __align__(128) Smem {
  uint8_t ring[NSLOTS][SLOT_BYTES];
  float xs[NTMAX * INTER];           // stage input vector; attention / sampler scratch
  uint8_t att[ATT_STAGE_BYTES];      // attention: staged K and V rows of one sub-chunk
  float part[MAXPART * NTMAX];       // per-unit partial dot products of the current stage
  float red[4 * NCW];
  double dred[NTMAX * NCW];
  unsigned long long ured[NCW + 1];
  int hist[256];
  uint64_t full[NSLOTS];
  uint64_t empty[NSLOTS];
  int abort;
  int epoch;                         // grid barriers completed by this CTA (producer pacing)
  int free_epoch[NSLOTS];            // epoch during which the consumers freed each slot
  int bcast[4];
  // batched kernel only
  uint64_t bbar[32];                 // pipeline mbarriers
  uint32_t tmem_base;                // tensor-memory address of the accumulator
  int bstate[4 * BMAX];              // per utterance: position, step, g0, active
  int bplan[257];                    // backbone attention plan of the launch (item offsets, chunks, count)
  int bplan_ok;                      // bplan holds the launch's plan
  void* bkv[4 * BMAX];               // per utterance: backbone K, V and code-predictor K, V caches
};

size_t work_bytes() {
  size_t n = 0;
  n += 256;                                             // bar, err, att_cnt
  n += sizeof(float) * 2 * NTMAX * HID;                 // hbuf
  n += sizeof(float) * NTMAX * QKV_ROWS;                // qkv
  n += sizeof(float) * NTMAX * QSZ;                     // attn
  n += sizeof(float) * NTMAX * NQH * MAX_ATT_CHUNKS * PRT_STRIDE;  // prt
  n += sizeof(float) * NTMAX * HID;                     // hmid
  n += sizeof(float) * NTMAX * INTER;                   // mlp
  n += sizeof(float) * VMAX;                            // logits
  n += sizeof(long long) * NHACC * NTMAX * HID;         // hacc
  return n;
}

void work_carve(void* base, Work* w) {
  char* c = static_cast<char*>(base);
  w->bar = reinterpret_cast<uint32_t*>(c);
  w->err = reinterpret_cast<int*>(c + 64);
  w->att_cnt = reinterpret_cast<uint32_t*>(c + 128);
  w->amax = reinterpret_cast<unsigned long long*>(c + 192);
  c += 256;
  w->hbuf = reinterpret_cast<float*>(c); c += sizeof(float) * 2 * NTMAX * HID;
  w->qkv = reinterpret_cast<float*>(c); c += sizeof(float) * NTMAX * QKV_ROWS;
  w->attn = reinterpret_cast<float*>(c); c += sizeof(float) * NTMAX * QSZ;
  w->prt = reinterpret_cast<float*>(c); c += sizeof(float) * NTMAX * NQH * MAX_ATT_CHUNKS * PRT_STRIDE;
  w->hmid = reinterpret_cast<float*>(c); c += sizeof(float) * NTMAX * HID;
  w->mlp = reinterpret_cast<float*>(c); c += sizeof(float) * NTMAX * INTER;
  w->logits = reinterpret_cast<float*>(c); c += sizeof(float) * VMAX;
  w->hacc = reinterpret_cast<long long*>(c);
}

// ------------------------------------------------------------------------------------------
// Stage plans: which rows of which matrix this CTA streams and reduces.
// ------------------------------------------------------------------------------------------
struct Plan {
  int P;            // units per row (K / 1024)
  int nseg;
  int units;        // total units of this CTA in the stage
  int r0, r1;       // logical row range (QKV: of the 4096 fused rows; GU: of the 3072 j)
  const bf16* ptr[3];
  int nun[3];
};

// First row of part c when n rows are split over G parts (n * G < 2^32 for every use here).
__device__ __forceinline__ int split_lo(int n, int G, int c) {
  return static_cast<int>((static_cast<uint32_t>(n) * static_cast<uint32_t>(c)) / static_cast<uint32_t>(G));
}

__device__ __forceinline__ void plan_add(Plan& pl, const bf16* base, int rows) {
  pl.ptr[pl.nseg] = base;
  pl.nun[pl.nseg] = rows * pl.P;
  pl.units += rows * pl.P;
  pl.nseg++;
}

// With lw == nullptr (consumer side) only the shape is computed: the segment pointers are null
// and no layer table is read.
__device__ Plan make_plan(int kind, const LayerW* lw, const bf16* head, int head_rows, int cta, int G) {
  Plan pl;
  pl.nseg = 0;
  pl.units = 0;
  pl.P = 1;
  if (kind == SK_QKV) {
    pl.r0 = split_lo(QKV_ROWS, G, cta);
    pl.r1 = split_lo(QKV_ROWS, G, cta + 1);
    const bf16* mats[3] = {lw ? lw->wq : nullptr, lw ? lw->wk : nullptr, lw ? lw->wv : nullptr};
    const int lo[3] = {0, QSZ, QSZ + KVSZ};
    const int hi[3] = {QSZ, QSZ + KVSZ, QKV_ROWS};
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      const int a = max(pl.r0, lo[m]), b = min(pl.r1, hi[m]);
      if (a < b) plan_add(pl, mats[m] ? mats[m] + static_cast<size_t>(a - lo[m]) * HID : nullptr, b - a);
    }
  } else if (kind == SK_O) {
    pl.P = QSZ / UNIT;
    pl.r0 = split_lo(HID, G, cta);
    pl.r1 = split_lo(HID, G, cta + 1);
    if (pl.r1 > pl.r0) plan_add(pl, lw ? lw->wo + static_cast<size_t>(pl.r0) * QSZ : nullptr, pl.r1 - pl.r0);
  } else if (kind == SK_GU) {
    pl.r0 = split_lo(INTER, G, cta);
    pl.r1 = split_lo(INTER, G, cta + 1);
    if (pl.r1 > pl.r0) {
      plan_add(pl, lw ? lw->wg + static_cast<size_t>(pl.r0) * HID : nullptr, pl.r1 - pl.r0);
      plan_add(pl, lw ? lw->wu + static_cast<size_t>(pl.r0) * HID : nullptr, pl.r1 - pl.r0);
    }
  } else if (kind == SK_GUF) {   // fused MLP stage: intermediate columns in blocks of 8
    pl.r0 = 8 * split_lo(INTER / 8, G, cta);
    pl.r1 = 8 * split_lo(INTER / 8, G, cta + 1);
    if (pl.r1 > pl.r0) {
      plan_add(pl, lw ? lw->wg + static_cast<size_t>(pl.r0) * HID : nullptr, pl.r1 - pl.r0);
      plan_add(pl, lw ? lw->wu + static_cast<size_t>(pl.r0) * HID : nullptr, pl.r1 - pl.r0);
    }
  } else if (kind == SK_D) {
    pl.P = INTER / UNIT;
    pl.r0 = split_lo(HID, G, cta);
    pl.r1 = split_lo(HID, G, cta + 1);
    if (pl.r1 > pl.r0) plan_add(pl, lw ? lw->wd + static_cast<size_t>(pl.r0) * INTER : nullptr, pl.r1 - pl.r0);
  } else {  // SK_HEAD
    pl.r0 = split_lo(head_rows, G, cta);
    pl.r1 = split_lo(head_rows, G, cta + 1);
    if (pl.r1 > pl.r0) plan_add(pl, head + static_cast<size_t>(pl.r0) * HID, pl.r1 - pl.r0);
  }
  return pl;
}

// ------------------------------------------------------------------------------------------
// Producer
// ------------------------------------------------------------------------------------------
struct Prod {
  uint32_t slot, round, issued;
  bool ok;
};

// Waits (bounded) until the consumers complete their next grid barrier after `seen`.
__device__ bool wait_epoch_after(Smem& sm, int seen) {
  volatile int* ep = &sm.epoch;
  volatile int* ab = &sm.abort;
  if (*ep != seen) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (*ep != seen) return true;
    if ((it & 63u) == 63u) {
      if (*ab) return false;
      if (globaltimer_ns() - t0 > QTT_WAIT_NS) return false;
    }
  }
}

// Waits (bounded) until the producer may refill its current slot. A slot freed by the
// consumers is refilled only after the grid barrier that ends the stage in which it was freed,
// so that a stage's refill traffic does not compete with that stage's barrier; the ring holds
// two stages of weights, so the refill still lands in time.
__device__ __forceinline__ bool prod_acquire(Smem& sm, Prod& pr, int* err, bool eager) {
  if (!mbar_wait(&sm.empty[pr.slot], (pr.round & 1u) ^ 1u, &sm.abort) ||
      (!eager && pr.round > 0 &&
       !wait_epoch_after(sm, *reinterpret_cast<volatile int*>(&sm.free_epoch[pr.slot])))) {
    if (!*reinterpret_cast<volatile int*>(&sm.abort)) set_error(err, DEV_ERR_EMPTY_TIMEOUT);
    pr.ok = false;
    return false;
  }
  return true;
}

__device__ __forceinline__ void prod_advance(Prod& pr) {
  pr.issued++;
  if (++pr.slot == NSLOTS) {
    pr.slot = 0;
    pr.round++;
  }
}

__device__ void prod_stage(Smem& sm, Prod& pr, const Plan& pl, int* err, bool eager) {
  for (int u = 0; u < pl.units && pr.ok; u += SLOT_UNITS) {
    const int n = min(SLOT_UNITS, pl.units - u);
    if (!prod_acquire(sm, pr, err, eager)) return;
    mbar_arrive_expect_tx(&sm.full[pr.slot], static_cast<uint32_t>(n * UNIT_BYTES));
    int base = 0;
    for (int s = 0; s < pl.nseg; ++s) {
      const int a = max(u, base), b = min(u + n, base + pl.nun[s]);
      if (a < b)
        bulk_g2s(sm.ring[pr.slot] + (a - u) * UNIT_BYTES, pl.ptr[s] + static_cast<size_t>(a - base) * UNIT,
                 static_cast<uint32_t>((b - a) * UNIT_BYTES), &sm.full[pr.slot]);
      base += pl.nun[s];
    }
    prod_advance(pr);
  }
}

// W_down columns of this CTA's intermediate block for the fused MLP stage: four 2-D boxes
// (256 rows x 24 columns, 12 KB) from the layer's tensor map, two per slot.
__device__ void prod_wd(const void* tmap, Smem& sm, Prod& pr, int cta, int G, int* err, bool eager) {
  const int j0 = 8 * split_lo(INTER / 8, G, cta);
  for (int b = 0; b < WD_BOXES && pr.ok; b += WD_BOXES_PER_SLOT) {
    if (!prod_acquire(sm, pr, err, eager)) return;
    mbar_arrive_expect_tx(&sm.full[pr.slot], static_cast<uint32_t>(WD_BOXES_PER_SLOT * WD_BOX_BYTES));
    for (int k = 0; k < WD_BOXES_PER_SLOT; ++k)
      tma_load_2d(sm.ring[pr.slot] + k * WD_BOX_BYTES, tmap, j0, (b + k) * WD_BOX_ROWS, &sm.full[pr.slot]);
    prod_advance(pr);
  }
}

__device__ __forceinline__ void att_split(int S, int G, int target, int& nch, int& chunk);

// L2 prefetch of the cached backbone K/V rows this CTA's attention item will read in layer
// li (rows written by earlier launches only), issued when the producer reaches the layer.
__device__ void prod_prefetch_attention(const Params& p, int li, int p0, int cta, int G) {
  int nch, chunk;
  att_split(p0 + 1, G, p.att_target, nch, chunk);
  for (int item = cta; item < NKVH * nch; item += G) {
    const int h = item / nch, c = item - h * nch;
    const int s0 = c * chunk, a1 = min(s0 + chunk, p0);
    if (a1 <= s0) continue;
    const size_t off = ((static_cast<size_t>(li) * NKVH + h) * p.bb_max_seq + s0) * HD;
    const uint32_t bytes = static_cast<uint32_t>(a1 - s0) * HD * 2;
    prefetch_l2_bulk(p.bb_k + off, bytes);
    prefetch_l2_bulk(p.bb_v + off, bytes);
  }
}

// Rows [r0, r1) of this CTA's share of its KV head's o_proj columns (code-predictor layers):
// head h = cta / (G/8) owns columns [2h*HD, 2h*HD + 2*HD) of W_o [HID][QSZ].
__device__ __forceinline__ bool oh_rows(int cta, int G, int& h, int& r0, int& r1) {
  const int gph = G / NKVH;
  if (cta >= NKVH * gph) return false;
  h = cta / gph;
  const int i = cta - h * gph;
  r0 = split_lo(HID, gph, i);
  r1 = split_lo(HID, gph, i + 1);
  return r1 > r0;
}

constexpr int OH_ROW_BYTES = 2 * HD * 2;            // 256 bf16 = 512 B
constexpr int OH_ROWS_PER_SLOT = SLOT_BYTES / OH_ROW_BYTES;   // 48

// Streams the CTA's o_proj row pieces (512 B each, stride QSZ) into the ring.
__device__ void prod_oh(const LayerW* lw, Smem& sm, Prod& pr, int cta, int G, int* err, bool eager) {
  int h, r0, r1;
  if (!oh_rows(cta, G, h, r0, r1)) return;
  const int n = r1 - r0;
  for (int u = 0; u < n && pr.ok; u += OH_ROWS_PER_SLOT) {
    const int m = min(OH_ROWS_PER_SLOT, n - u);
    if (!prod_acquire(sm, pr, err, eager)) return;
    mbar_arrive_expect_tx(&sm.full[pr.slot], static_cast<uint32_t>(m * OH_ROW_BYTES));
    for (int k = 0; k < m; ++k)
      bulk_g2s(sm.ring[pr.slot] + k * OH_ROW_BYTES, lw->wo + static_cast<size_t>(r0 + u + k) * QSZ + 2 * h * HD,
               OH_ROW_BYTES, &sm.full[pr.slot]);
    prod_advance(pr);
  }
}

// L1 prefetch of what the consumers of this SM read with plain loads in a layer's prologues:
// the layer's pointer table and its RMSNorm weights (issued a stage or two ahead).
__device__ void prod_prefetch_norms(const LayerW* lw) {
  prefetch_l1(lw);
  prefetch_l1(reinterpret_cast<const uint8_t*>(lw) + sizeof(LayerW) - 1);
  const bf16* v[2] = {lw->in_norm, lw->post_norm};
  for (int i = 0; i < 2; ++i)
    for (int o = 0; o < HID * 2; o += 128) prefetch_l1(reinterpret_cast<const uint8_t*>(v[i]) + o);
  for (int o = 0; o < HD * 2; o += 128) {
    prefetch_l1(reinterpret_cast<const uint8_t*>(lw->q_norm) + o);
    prefetch_l1(reinterpret_cast<const uint8_t*>(lw->k_norm) + o);
  }
}

__device__ void prod_layers(const Params& p, Smem& sm, Prod& pr, const LayerW* L, int n, int cta, int G, int* err,
                            int prefetch_pos, bool cp) {
  const bool eager = (p.flags & FLAG_EAGER_REFILL) != 0;
  const uint8_t* maps = static_cast<const uint8_t*>(cp ? p.cp_wd_map : p.bb_wd_map);
  for (int l = 0; l < n && pr.ok; ++l) {
    prod_prefetch_norms(L + l);
    if (l + 1 == n)
      for (int o = 0; o < HID * 2; o += 128) prefetch_l1(reinterpret_cast<const uint8_t*>(cp ? p.cp_norm : p.bb_norm) + o);
    if (prefetch_pos >= 0) prod_prefetch_attention(p, l, prefetch_pos, cta, G);
    prod_stage(sm, pr, make_plan(SK_QKV, L + l, nullptr, 0, cta, G), err, eager);
    if (cp)
      prod_oh(L + l, sm, pr, cta, G, err, eager);
    else
      prod_stage(sm, pr, make_plan(SK_O, L + l, nullptr, 0, cta, G), err, eager);
    if (maps) {
      prod_stage(sm, pr, make_plan(SK_GUF, L + l, nullptr, 0, cta, G), err, eager);
      prod_wd(maps + l * TMAP_BYTES, sm, pr, cta, G, err, eager);
    } else {
      prod_stage(sm, pr, make_plan(SK_GU, L + l, nullptr, 0, cta, G), err, eager);
      prod_stage(sm, pr, make_plan(SK_D, L + l, nullptr, 0, cta, G), err, eager);
    }
  }
}

__device__ bool frame_skipped(const Params& p) {
  const StreamState* st = p.st;
  const int done = ld_volatile_i32(&st->done);
  const int g0 = ld_volatile_i32(&st->g0);
  return done != 0 || g0 == p.sp.eos;
}

__device__ void producer_main(const Params& p, Smem& sm, int cta, int G) {
  Prod pr{0u, 0u, 0u, true};
  int* err = p.w.err;
  if (p.bb_wd_map != nullptr)
    for (int l = 0; l < p.n_bb; ++l) tensormap_acquire(static_cast<const uint8_t*>(p.bb_wd_map) + l * TMAP_BYTES);
  if (p.cp_wd_map != nullptr)
    for (int l = 0; l < p.n_cp; ++l) tensormap_acquire(static_cast<const uint8_t*>(p.cp_wd_map) + l * TMAP_BYTES);
  if (p.mode == MODE_FRAME) {
    if (!frame_skipped(p)) {
      int pos = ld_volatile_i32(&p.st->position);
      if (pos < 0 || pos >= p.bb_max_seq) pos = -1;   // the consumers report the bad position
      for (int pass = 0; pass < NCPHEADS && pr.ok; ++pass) {
        if (pass + 1 < NCPHEADS) {
          // the next pass reads one row of code-predictor embedding table `pass` (chosen by this
          // pass's token): bring this CTA's slice of the table into L2 while this pass runs
          const int r0 = split_lo(p.cp_vocab, G, cta), r1 = split_lo(p.cp_vocab, G, cta + 1);
          if (r1 > r0)
            prefetch_l2_bulk(p.cp_emb[pass] + static_cast<size_t>(r0) * HID, static_cast<uint32_t>(r1 - r0) * HID * 2);
        }
        prod_layers(p, sm, pr, p.cp_layers, p.n_cp, cta, G, err, -1, true);
        prod_stage(sm, pr, make_plan(SK_HEAD, nullptr, p.cp_head[pass], p.cp_vocab, cta, G), err,
                   (p.flags & FLAG_EAGER_REFILL) != 0);
      }
      prod_layers(p, sm, pr, p.bb_layers, p.n_bb, cta, G, err, pos, false);
      prod_stage(sm, pr, make_plan(SK_HEAD, nullptr, p.codec_head, p.vocab, cta, G), err,
                 (p.flags & FLAG_EAGER_REFILL) != 0);
    }
  } else if (p.mode == MODE_BB_STEP) {
    prod_layers(p, sm, pr, p.bb_layers, p.n_bb, cta, G, err,
                (p.position >= 0 && p.position < p.bb_max_seq) ? p.position : -1, false);
    if (p.flags & FLAG_HEAD_SAMPLE)
      prod_stage(sm, pr, make_plan(SK_HEAD, nullptr, p.codec_head, p.vocab, cta, G), err,
                 (p.flags & FLAG_EAGER_REFILL) != 0);
  } else {
    prod_layers(p, sm, pr, p.cp_layers, p.n_cp, cta, G, err, -1, true);
  }
  // Drain: wait (bounded) for the copies of the last ring's worth of fills so that no bulk
  // copy is still writing shared memory when this CTA exits early.
  const uint32_t inflight = pr.issued < NSLOTS ? pr.issued : NSLOTS;
  uint32_t slot = pr.slot, round = pr.round;
  int zero = 0;
  for (uint32_t i = 0; i < inflight; ++i) {
    if (slot == 0) {
      slot = NSLOTS - 1;
      round--;
    } else {
      slot--;
    }
    mbar_wait(&sm.full[slot], round & 1u, &zero);
  }
}

// ------------------------------------------------------------------------------------------
// Consumers
// ------------------------------------------------------------------------------------------
// A consumer thread's state. Its indices come from special registers (no memory access); only the
// counters below are kept in the struct.
struct Cons {
  uint32_t slot, round, bar_target;
  int dk;   // fused MLP stages completed in this launch (selects the fixed-point output buffer)
  int gi;   // batched kernel: GEMM stages completed in this launch (trace index)
  int pn;   // batched kernel: GEMM stages whose K-slice partials were pushed (mbarrier parity)
  int go_next;   // batched kernel: the coming grid barrier precedes a GEMM stage (release its loads there)
  int go_sent;   // batched kernel: the last grid barrier released the coming GEMM stage's loads
  __device__ __forceinline__ int cta() const { return static_cast<int>(blockIdx.x); }
  __device__ __forceinline__ int G() const { return static_cast<int>(gridDim.x); }
  __device__ __forceinline__ int tid() const { return static_cast<int>(threadIdx.x); }
  __device__ __forceinline__ int warp() const { return static_cast<int>(threadIdx.x) >> 5; }
  __device__ __forceinline__ int lane() const { return static_cast<int>(threadIdx.x) & 31; }
};

// A layer's input or output hidden state in global memory: fp32 (first layer of a stack,
// separate MLP stages) or the fixed-point sum of the fused MLP stage.
struct HIn {
  const float* f;
  const long long* q;
};

__device__ __forceinline__ long long float_to_fix(float v) {
  return __double2ll_rn(static_cast<double>(v) * 4294967296.0);
}
__device__ __forceinline__ float fix_to_float(long long q) {
  return __double2float_rn(static_cast<double>(q) * (1.0 / 4294967296.0));
}
// BB: backbone hidden states are bf16 between layers (fused_decode_tts.cu:541).
template <bool BB>
__device__ __forceinline__ float h_ld(const HIn& h, int i) {
  if (h.q) {
    const float v = fix_to_float(__ldcg(h.q + i));
    return BB ? round_bf16(v) : v;
  }
  return __ldcg(h.f + i);
}
template <bool BB>
__device__ __forceinline__ float4 h_ld4(const HIn& h, int i) {   // i: multiple of 4
  if (h.q) {
    const longlong2 a = __ldcg(reinterpret_cast<const longlong2*>(h.q + i));
    const longlong2 b = __ldcg(reinterpret_cast<const longlong2*>(h.q + i + 2));
    float4 v = make_float4(fix_to_float(a.x), fix_to_float(a.y), fix_to_float(b.x), fix_to_float(b.y));
    if (BB) {
      v.x = round_bf16(v.x);
      v.y = round_bf16(v.y);
      v.z = round_bf16(v.z);
      v.w = round_bf16(v.w);
    }
    return v;
  }
  return __ldcg(reinterpret_cast<const float4*>(h.f + i));
}

__device__ __forceinline__ bool aborted(Smem& sm) { return *reinterpret_cast<volatile int*>(&sm.abort) != 0; }

__device__ __forceinline__ void fail(const Params& p, Smem& sm, int code) {
  set_error(p.w.err, code);
  *reinterpret_cast<volatile int*>(&sm.abort) = 1;
}

// Profiling stamp of CTA 0 for the current stage (no-op unless dbg_marks is set; the batched
// kernel, p.nb > 0, uses dbg_marks for its own trace).
__device__ __forceinline__ void stage_mark(const Params& p, const Cons& cs, int id) {
  if (p.dbg_marks != nullptr && p.nb == 0 && cs.cta() == 0 && cs.tid() == 0) {
    const uint32_t k = cs.bar_target / static_cast<uint32_t>(cs.G());
    if (static_cast<int>(k * 3 + id) < p.dbg_marks_len) p.dbg_marks[k * 3 + id] = globaltimer_ns();
  }
}

// Profiling stamps of CTA 0 inside a stage's RMSNorm prologue (input loaded, norm reduced).
__device__ __forceinline__ void prologue_mark(const Params& p, const Cons& cs, int id) {
  if (p.dbg_marks != nullptr && cs.cta() == 0 && cs.tid() == 0) {
    const uint32_t k = cs.bar_target / static_cast<uint32_t>(cs.G());
    if (static_cast<int>(8 * 1024 + 4 * k + id) < p.dbg_marks_len) p.dbg_marks[8 * 1024 + 4 * k + id] = globaltimer_ns();
  }
}

// Grid-wide barrier over the consumer threads of all CTAs (monotonic counter, bounded). go: an
// mbarrier that thread 0 arrives on as soon as the barrier has passed (the batched kernel's
// activation loader starts the next GEMM stage's loads there).
__device__ __forceinline__ bool grid_sync(const Params& p, Smem& sm, Cons& cs, uint64_t* go = nullptr) {
  named_sync(1, NCT);
  if (cs.tid() == 0) {
    stage_mark(p, cs, 2);
    if (p.dbg_arrivals != nullptr) {
      const int k = static_cast<int>(cs.bar_target / static_cast<uint32_t>(cs.G())) - p.dbg_arr_stage0;
      if (k >= 0 && k < p.dbg_arr_n) p.dbg_arrivals[k * cs.G() + cs.cta()] = globaltimer_ns();
    }
  }
  cs.bar_target += static_cast<uint32_t>(cs.G());
  if (cs.tid() == 0 && !aborted(sm)) {
    // bar.sync above orders this CTA's stores before thread 0; the release add publishes them
    // at gpu scope and the acquire load below orders the other CTAs' stores before ours.
    const bool skip = p.dbg_skip_barrier > 0 && cs.cta() == cs.G() - 1 &&
                      cs.bar_target == static_cast<uint32_t>(p.dbg_skip_barrier) * static_cast<uint32_t>(cs.G());
    if (!skip) red_release_gpu_add(p.w.bar, 1u);
    const uint64_t limit = p.dbg_wait_ns != 0ull ? p.dbg_wait_ns : QTT_WAIT_NS;
    // the spin compares against register copies: the acquire load clobbers memory, so a value
    // read through cs or p would be reloaded from the stack on every iteration
    const uint32_t target = cs.bar_target;
    uint32_t* const bar = p.w.bar;
    const int* const errw = p.w.err;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      const uint32_t v = ld_acquire_gpu(bar);
      if (static_cast<int>(v - target) >= 0) break;
      if ((it & 31u) == 31u) {
        if (ld_volatile_i32(errw) != 0) {
          *reinterpret_cast<volatile int*>(&sm.abort) = 1;
          break;
        }
        if (globaltimer_ns() - t0 > limit) {
          fail(p, sm, DEV_ERR_GRID_TIMEOUT);
          break;
        }
      }
    }
    if (go != nullptr && !aborted(sm)) mbar_arrive(go);
    *reinterpret_cast<volatile int*>(&sm.epoch) = static_cast<int>(cs.bar_target / static_cast<uint32_t>(cs.G()));
    if (p.dbg_timeline != nullptr && cs.cta() == 0) {
      const uint32_t k = cs.bar_target / static_cast<uint32_t>(cs.G());
      if (k < static_cast<uint32_t>(p.dbg_timeline_len)) p.dbg_timeline[k] = globaltimer_ns();
    }
  }
  named_sync(1, NCT);
  return !aborted(sm);
}

// fp64 sum of NT per-thread values over the consumer threads (fixed order, every thread gets
// the same totals). Used for RMSNorm statistics.
template <int NT>
__device__ __forceinline__ void block_sum_d(Smem& sm, Cons& cs, double (&v)[NT]) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const double s = warp_sum_d(v[t]);
    if (cs.lane() == 0) sm.dred[t * NCW + cs.warp()] = s;
  }
  named_sync(1, NCT);
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < NCW; ++w) s += sm.dred[t * NCW + w];
    v[t] = s;
  }
  named_sync(1, NCT);
}

// Sum of NT per-thread values over the consumer threads; every thread gets the same totals.
template <int NT>
__device__ __forceinline__ void block_sum(Smem& sm, Cons& cs, float (&v)[NT]) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const float s = warp_sum(v[t]);
    if (cs.lane() == 0) sm.red[t * NCW + cs.warp()] = s;
  }
  named_sync(1, NCT);
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) s += sm.red[t * NCW + w];
    v[t] = s;
  }
  named_sync(1, NCT);
}

// RMSNorm prologue of a stage: NT vectors of HID floats (from global memory written by other
// CTAs, or from shared memory) are normalised into dst = x * rsqrt(mean(x^2) + eps) * w.
// The activation and the norm weights are loaded in the same round trip; thread t < 256 owns
// elements 4t .. 4t+3 of every token.
// DEFER: dst = x * w only, and each warp's sum of squares goes to sm.dred; the GEMV that
// reads dst applies 1 / rms to its dot products (gemv<NT, true>), which takes the norm's
// block reduction off the path to the GEMV.
template <int NT, bool DEFER>
__device__ void rmsnorm_finish(const Params& p, Smem& sm, Cons& cs, const float4 (&x)[NT], uint2 wv, float eps,
                               float* dst);

template <int NT, bool FROM_SMEM, bool DEFER = false>
__device__ void load_rmsnorm(const Params& p, Smem& sm, Cons& cs, const float* src, const bf16* w, float eps,
                             float* dst) {
  const bool act = cs.tid() < HID / 4;
  float4 x[NT];
  uint2 wv = make_uint2(0u, 0u);
  if (act) {
    wv = *reinterpret_cast<const uint2*>(w + 4 * cs.tid());
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float4* s4 = reinterpret_cast<const float4*>(src + t * HID) + cs.tid();
      x[t] = FROM_SMEM ? *s4 : __ldcg(s4);
    }
  }
  rmsnorm_finish<NT, DEFER>(p, sm, cs, x, wv, eps, dst);
}

// Same, from a layer input in global memory (fp32 or fixed point).
template <int NT, bool BB, bool DEFER = false>
__device__ void load_rmsnorm_h(const Params& p, Smem& sm, Cons& cs, const HIn& h, const bf16* w, float eps,
                               float* dst) {
  float4 x[NT];
  uint2 wv = make_uint2(0u, 0u);
  if (cs.tid() < HID / 4) {
    wv = *reinterpret_cast<const uint2*>(w + 4 * cs.tid());
#pragma unroll
    for (int t = 0; t < NT; ++t) x[t] = h_ld4<BB>(h, t * HID + 4 * cs.tid());
  }
  rmsnorm_finish<NT, DEFER>(p, sm, cs, x, wv, eps, dst);
}

template <int NT, bool DEFER>
__device__ void rmsnorm_finish(const Params& p, Smem& sm, Cons& cs, const float4 (&x)[NT], uint2 wv, float eps,
                               float* dst) {
  const bool act = cs.tid() < HID / 4;
  if constexpr (DEFER) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      double a = 0.0;
      if (act) {
        a = fma(static_cast<double>(x[t].x), static_cast<double>(x[t].x), a);
        a = fma(static_cast<double>(x[t].y), static_cast<double>(x[t].y), a);
        a = fma(static_cast<double>(x[t].z), static_cast<double>(x[t].z), a);
        a = fma(static_cast<double>(x[t].w), static_cast<double>(x[t].w), a);
        const float w0 = bf16_lo(wv.x), w1 = bf16_hi(wv.x), w2 = bf16_lo(wv.y), w3 = bf16_hi(wv.y);
        reinterpret_cast<float4*>(dst + t * HID)[cs.tid()] =
            make_float4(x[t].x * w0, x[t].y * w1, x[t].z * w2, x[t].w * w3);
      }
      a = warp_sum_d(a);
      if (cs.lane() == 0) sm.dred[t * NCW + cs.warp()] = a;
    }
    prologue_mark(p, cs, 0);
    named_sync(1, NCT);
    prologue_mark(p, cs, 3);
  } else {
    double ss[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      double a = 0.0;
      if (act) {
        a = fma(static_cast<double>(x[t].x), static_cast<double>(x[t].x), a);
        a = fma(static_cast<double>(x[t].y), static_cast<double>(x[t].y), a);
        a = fma(static_cast<double>(x[t].z), static_cast<double>(x[t].z), a);
        a = fma(static_cast<double>(x[t].w), static_cast<double>(x[t].w), a);
      }
      ss[t] = a;
    }
    if (p.dbg_marks != nullptr) {
      asm volatile("" ::"d"(ss[0]));
      prologue_mark(p, cs, 0);
    }
    block_sum_d<NT>(sm, cs, ss);
    prologue_mark(p, cs, 1);
    if (act) {
      const float w0 = bf16_lo(wv.x), w1 = bf16_hi(wv.x), w2 = bf16_lo(wv.y), w3 = bf16_hi(wv.y);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float rstd = rms_scale(ss[t], HID, eps);
        float4 o;
        o.x = x[t].x * rstd * w0;
        o.y = x[t].y * rstd * w1;
        o.z = x[t].z * rstd * w2;
        o.w = x[t].w * rstd * w3;
        reinterpret_cast<float4*>(dst + t * HID)[cs.tid()] = o;
      }
    }
    prologue_mark(p, cs, 2);
    named_sync(1, NCT);
    prologue_mark(p, cs, 3);
  }
}

// Copy NT vectors of n floats from global (L2, written by other CTAs) into shared memory.
__device__ __forceinline__ void load_vec(Cons& cs, float* dst, const float* src, int n_total) {
  for (int i = cs.tid() * 4; i < n_total; i += NCT * 4)
    *reinterpret_cast<float4*>(dst + i) = __ldcg(reinterpret_cast<const float4*>(src + i));
}

// GEMV over this CTA's units of one stage: part[u * NT + t] = dot(unit u, x part of u).
// NORM: the input was prepared by a deferred RMSNorm (x * w, sums of squares per warp in
// sm.dred); the dot products are multiplied by 1 / rms of their token.
template <int NT, bool NORM = false>
__device__ bool gemv(const Params& p, const Plan& pl, Smem& sm, Cons& cs, const float* xsrc, int xstride) {
  stage_mark(p, cs, 0);
  if (pl.units > MAXUNITS) {
    fail(p, sm, DEV_ERR_BAD_POSITION);
    return false;
  }
  float* lp = reinterpret_cast<float*>(sm.att);   // [units * NT][LP_STRIDE] lane partials
  uint32_t slot = cs.slot, round = cs.round;   // ring position in registers for the stage
  const int part = cs.warp() % pl.P;
  float xr[NT][32];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const float* xp = xsrc + t * xstride + part * UNIT + 8 * cs.lane();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 a = *reinterpret_cast<const float4*>(xp + 256 * i);
      const float4 b = *reinterpret_cast<const float4*>(xp + 256 * i + 4);
      xr[t][8 * i + 0] = a.x; xr[t][8 * i + 1] = a.y; xr[t][8 * i + 2] = a.z; xr[t][8 * i + 3] = a.w;
      xr[t][8 * i + 4] = b.x; xr[t][8 * i + 5] = b.y; xr[t][8 * i + 6] = b.z; xr[t][8 * i + 7] = b.w;
    }
  }
  // 1 / rms of each token (deferred norm); computed here so that its latency overlaps the loop
  float rs[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    rs[t] = 1.f;
    if (NORM) {
      double a = 0.0;
#pragma unroll
      for (int w = 0; w < NCW; ++w) a += sm.dred[t * NCW + w];
      rs[t] = rms_scale(a, HID, p.eps);
    }
  }
  const bool prof = p.dbg_marks != nullptr && cs.cta() == 0 && cs.tid() == 0;
  unsigned long long waited = 0;
  const uint32_t kst = cs.bar_target / static_cast<uint32_t>(cs.G());
  const bool fine = prof && static_cast<int>(4 * 1024 + 4 * kst + 3) < p.dbg_marks_len;
  if (fine) p.dbg_marks[4 * 1024 + 4 * kst + 0] = globaltimer_ns();
  for (int u0 = 0; u0 < pl.units; u0 += SLOT_UNITS) {
    const int n = min(SLOT_UNITS, pl.units - u0);
    unsigned long long tw = prof ? globaltimer_ns() : 0ull;
    const bool got = mbar_wait(&sm.full[slot], round & 1u, &sm.abort);
    if (prof) waited += globaltimer_ns() - tw;
    if (!got) {
      if (!aborted(sm)) fail(p, sm, DEV_ERR_FULL_TIMEOUT);
    } else if (cs.warp() < n) {
      const uint4* src = reinterpret_cast<const uint4*>(sm.ring[slot] + cs.warp() * UNIT_BYTES);
      // four independent FMA chains (one per 16-byte chunk) keep the dependent chain short
      float ch[NT][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = src[cs.lane() + 32 * i];
        const float w[8] = {bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y),
                            bf16_lo(v.z), bf16_hi(v.z), bf16_lo(v.w), bf16_hi(v.w)};
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float a = w[0] * xr[t][8 * i];
#pragma unroll
          for (int j = 1; j < 8; ++j) a = fmaf(w[j], xr[t][8 * i + j], a);
          ch[t][i] = a;
        }
      }
      // lane partials go to shared memory; the cross-lane sums are done once per stage below
#pragma unroll
      for (int t = 0; t < NT; ++t)
        lp[((u0 + cs.warp()) * NT + t) * LP_STRIDE + cs.lane()] = (ch[t][0] + ch[t][1]) + (ch[t][2] + ch[t][3]);
    }
    __syncwarp();
    if (cs.lane() == 0) {
      *reinterpret_cast<volatile int*>(&sm.free_epoch[slot]) =
          static_cast<int>(cs.bar_target / static_cast<uint32_t>(cs.G()));
      mbar_arrive(&sm.empty[slot]);
    }
    if (++slot == NSLOTS) {
      slot = 0;
      round++;
    }
  }
  cs.slot = slot;
  cs.round = round;
  if (prof) {
    const uint32_t k = cs.bar_target / static_cast<uint32_t>(cs.G());
    if (static_cast<int>(k) < p.dbg_marks_len / 3 - 1024) p.dbg_marks[3 * 1024 + k] = waited;
  }
  if (fine) p.dbg_marks[4 * 1024 + 4 * kst + 1] = globaltimer_ns();
  named_sync(1, NCT);
  if (fine) p.dbg_marks[4 * 1024 + 4 * kst + 2] = globaltimer_ns();
  // one thread per (unit, token): fixed-order pairwise sum of the 32 lane partials
  for (int e = cs.tid(); e < pl.units * NT; e += NCT) {
    const float* row = lp + e * LP_STRIDE;
    float a[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) a[k] = row[k] + row[k + 16];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] += a[k + 8];
#pragma unroll
    for (int k = 0; k < 4; ++k) a[k] += a[k + 4];
    const float v = (a[0] + a[2]) + (a[1] + a[3]);
    sm.part[e] = NORM ? v * ((NT == 1 || (e & 1) == 0) ? rs[0] : rs[NT - 1]) : v;
  }
  named_sync(1, NCT);
  stage_mark(p, cs, 1);
  return !aborted(sm);
}

// ------------------------------------------------------------------------------------------
// Attention: split over (KV head, chunk of positions) work items; the last item of a head to
// finish combines the partial softmaxes (flash-decoding style), so no extra grid barrier.
// Each item stages its q/k/v rows and its cached K/V rows into shared memory with one round
// of cp.async, then works from shared memory; chunks longer than one staging buffer are
// processed in sub-chunks with an online softmax.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void att_split(int S, int G, int target, int& nch, int& chunk) {
  target = target > 0 ? target : ATT_TARGET;
  nch = (S + target - 1) / target;
  const int maxch = min(MAX_ATT_CHUNKS, max(1, G / NKVH));
  nch = min(max(nch, 1), maxch);
  chunk = (S + nch - 1) / nch;
  nch = (S + chunk - 1) / chunk;
}

template <bool CP>
__device__ __forceinline__ void stage_kv_rows(Cons& cs, uint8_t* dst_k, uint8_t* dst_v, const uint8_t* kb,
                                              const uint8_t* vb, int a0, int a1) {
  constexpr int ROWB = HD * (CP ? 4 : 2);
  constexpr int PIECES = ROWB / 16;
  const int n = (a1 - a0) * PIECES;
  for (int e = cs.tid(); e < 2 * n; e += NCT) {
    const int which = e >= n, r = which ? e - n : e;
    const size_t off = static_cast<size_t>(a0) * ROWB + static_cast<size_t>(r) * 16;
    cp_async16((which ? dst_v : dst_k) + static_cast<size_t>(r) * 16, (which ? vb : kb) + off);
  }
}

// One attention work item's inputs and outputs: NT consecutive tokens of one utterance at
// positions p0 .. p0 + NT - 1, one KV head, context positions [s0, s1).
struct AttIO {
  const float* qkv;   // raw q/k/v rows of the item's first token (row stride QKV_ROWS)
  uint8_t* kb;        // the utterance's cached K rows of this (layer, KV head): row s at kb + s * HD * esize
  uint8_t* vb;        // same for V; rows p0 .. p0 + NT - 1 are written by the item's writer
  float* out;         // fp32 output rows of the item's first token (row stride QSZ), or nullptr:
  bf16* hilo;         //   then bf16 hi/lo GEMM operand planes (batched decode), token row tok0 + t
  int tok0;
  float* prt;         // partial records of the item's first token [NT][NQH][MAX_ATT_CHUNKS][PRT_STRIDE]
  uint32_t* cnt;      // last-arriver counter of (utterance, KV head)
};

// v = hi + lo with hi = bf16(v), lo = bf16(v - hi): two bf16 GEMM operands that carry ~16
// mantissa bits, so the tensor-core product stays close to an fp32 GEMV. Plane 0 (rows
// 0..TBMAX-1) holds the hi parts, plane 1 the lo parts; row = token.
__device__ __forceinline__ void hilo_store(bf16* buf, int t, int col, float v) {
  const bf16 hi = __float2bfloat16_rn(v);
  const bf16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
  buf[static_cast<size_t>(t) * ABUF_LD + col] = hi;
  buf[static_cast<size_t>(TBMAX + t) * ABUF_LD + col] = lo;
}

__device__ __forceinline__ void att_store(const AttIO& io, int t, int col, float v) {
  if (io.out != nullptr)
    io.out[t * QSZ + col] = v;
  else
    hilo_store(io.hilo, io.tok0 + t, col, v);
}

// One work item: stage q/k/v and the cached rows, q/k RMSNorm + RoPE, write the new K/V rows
// (writer), scores / softmax / P.V over [s0, s1) in sub-chunks with an online softmax, then
// either the final output (single item per head) or a partial record, the last item of the head
// combining all partials (flash-decoding style). GROUP: output stays in sm.xs.
template <int NT, bool CP, bool GROUP>
__device__ bool att_item(const Params& p, Smem& sm, Cons& cs, const LayerW* L, const AttIO& io, int p0, int h, int c,
                         int nch, int s0, int s1, bool writer) {
  constexpr int ESZ = CP ? 4 : 2;
  constexpr int ROWB = HD * ESZ;
  constexpr int SUB = ATT_STAGE_BYTES / (2 * ROWB);   // 48 bf16 rows or 24 fp32 rows
  constexpr int J = NT * 2;   // (token, q head) pairs
  // shared scratch inside xs
  float* qraw = sm.xs;                  // [NT][4][HD] raw q(2h), q(2h+1), k, v
  float* qr = qraw + NT * 4 * HD;       // [NT][2][HD]
  float* kn = qr + NT * 2 * HD;         // [NT][HD]
  float* vn = kn + NT * HD;             // [NT][HD]
  float* sc = vn + NT * HD;             // [J][SUB]
  float* acc_s = sc + J * SUB;          // [J][HD] running P.V
  float* accg = acc_s + J * HD;         // [3][J][HD]
  float* ml = accg + 3 * J * HD;        // [J][4]: running max, running sum, rescale of this step
  uint8_t* kst = sm.att;
  uint8_t* vst = sm.att + SUB * ROWB;

  // 1. one round trip: raw q/k/v rows of this head + the first sub-chunk of cached rows
  for (int e = cs.tid(); e < NT * 4 * (HD / 4); e += NCT) {
    const int t = e / (4 * HD / 4), r = e - t * (4 * HD / 4), vec = r / (HD / 4), piece = r - vec * (HD / 4);
    const int row0 = vec < 2 ? (2 * h + vec) * HD : (vec == 2 ? QSZ + h * HD : QSZ + KVSZ + h * HD);
    cp_async16(qraw + (t * 4 + vec) * HD + piece * 4, io.qkv + t * QKV_ROWS + row0 + piece * 4);
  }
  {
    const int a1 = min(min(s1, p0), s0 + SUB);
    if (a1 > s0) stage_kv_rows<CP>(cs, kst, vst, io.kb, io.vb, s0, a1);
  }
  for (int j = cs.tid(); j < J * HD; j += NCT) acc_s[j] = 0.f;
  if (cs.tid() < J) {
    ml[cs.tid() * 4 + 0] = -INFINITY;
    ml[cs.tid() * 4 + 1] = 0.f;
  }
  // norm weights and RoPE rows travel with the staged rows (same round trip)
  float nwv[4], cv[4], sv[4];
  if (cs.warp() < NT * 4 && (cs.warp() & 3) < 3) {
    const int pos = p0 + (cs.warp() >> 2);
    const bf16* nw = (cs.warp() & 3) < 2 ? L->q_norm : L->k_norm;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = cs.lane() + 32 * i;
      nwv[i] = __bfloat162float(nw[d]);
      cv[i] = __bfloat162float(p.cos_tab[static_cast<size_t>(pos) * HD + d]);
      sv[i] = __bfloat162float(p.sin_tab[static_cast<size_t>(pos) * HD + d]);
    }
  }
  cp_async_wait_all();
  named_sync(1, NCT);

  // 2. q/k RMSNorm per head (fused_decode_tts.cu:183-197) + RoPE; warp j handles vector j%4
  //    of token j/4 with d = lane + 32 i, so each rotation pair (d, d+64) sits in one lane.
  if (cs.warp() < NT * 4) {
    const int t = cs.warp() >> 2, vec = cs.warp() & 3;
    const float* src = qraw + (t * 4 + vec) * HD;
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = src[cs.lane() + 32 * i];
    if (vec < 3) {
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < 4; ++i) ss = fma(static_cast<double>(x[i]), static_cast<double>(x[i]), ss);
      ss = warp_sum_d(ss);
      const float rstd = rms_scale(ss, HD, p.eps);
      float y[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = x[i] * rstd * nwv[i];
      float o[4];
      o[0] = y[0] * cv[0] - y[2] * sv[0];
      o[1] = y[1] * cv[1] - y[3] * sv[1];
      o[2] = y[2] * cv[2] + y[0] * sv[2];
      o[3] = y[3] * cv[3] + y[1] * sv[3];
      float* dst = vec < 2 ? qr + (t * 2 + vec) * HD : kn + t * HD;
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[cs.lane() + 32 * i] = (vec == 2 && !CP) ? round_bf16(o[i]) : o[i];
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) vn[t * HD + cs.lane() + 32 * i] = CP ? x[i] : round_bf16(x[i]);
    }
  }
  named_sync(1, NCT);

  // 3. item 0 of each head stores the new K/V rows into the cache.
  if (writer) {
    for (int e = cs.tid(); e < NT * HD; e += NCT) {
      const int t = e / HD, d = e - t * HD;
      const size_t off = static_cast<size_t>(p0 + t) * HD + d;
      if (CP) {
        reinterpret_cast<float*>(io.kb)[off] = kn[e];
        reinterpret_cast<float*>(io.vb)[off] = vn[e];
      } else {
        reinterpret_cast<bf16*>(io.kb)[off] = __float2bfloat16_rn(kn[e]);
        reinterpret_cast<bf16*>(io.vb)[off] = __float2bfloat16_rn(vn[e]);
      }
    }
  }

  // 4. sub-chunks of at most SUB positions (one for every chunk up to SUB long)
  for (int sa = s0; sa < s1; sa += SUB) {
    const int sb = min(s1, sa + SUB), len = sb - sa;
    if (sa != s0) {
      const int a1 = min(sb, p0);
      if (a1 > sa) stage_kv_rows<CP>(cs, kst, vst, io.kb, io.vb, sa, a1);
      cp_async_wait_all();
      named_sync(1, NCT);
    }
    // scores: one warp per position, lane holds d = 4 lane .. 4 lane + 3
    for (int s = sa + cs.warp(); s < sb; s += NCW) {
      float k4[4];
      if (s < p0) {
        const uint8_t* row = kst + static_cast<size_t>(s - sa) * ROWB;
        if (CP) {
          const float4 kk = *reinterpret_cast<const float4*>(row + 16 * cs.lane());
          k4[0] = kk.x; k4[1] = kk.y; k4[2] = kk.z; k4[3] = kk.w;
        } else {
          const uint2 kk = *reinterpret_cast<const uint2*>(row + 8 * cs.lane());
          k4[0] = bf16_lo(kk.x); k4[1] = bf16_hi(kk.x); k4[2] = bf16_lo(kk.y); k4[3] = bf16_hi(kk.y);
        }
      } else {
        const float4 kk = *reinterpret_cast<const float4*>(kn + (s - p0) * HD + 4 * cs.lane());
        k4[0] = kk.x; k4[1] = kk.y; k4[2] = kk.z; k4[3] = kk.w;
      }
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const float4 q = *reinterpret_cast<const float4*>(qr + j * HD + 4 * cs.lane());
        float d = q.x * k4[0];
        d = fmaf(q.y, k4[1], d);
        d = fmaf(q.z, k4[2], d);
        d = fmaf(q.w, k4[3], d);
        d = warp_sum(d) * p.attn_scale;
        if (cs.lane() == 0) sc[j * SUB + (s - sa)] = (s <= p0 + (j >> 1)) ? d : -INFINITY;
      }
    }
    named_sync(1, NCT);
    // online softmax statistics: warp j handles (token, q head) j
    if (cs.warp() < J) {
      float* row = sc + cs.warp() * SUB;
      float m = -INFINITY;
      for (int i = cs.lane(); i < len; i += 32) m = fmaxf(m, row[i]);
      m = warp_max(m);
      const float m_old = ml[cs.warp() * 4 + 0];
      const float m_new = fmaxf(m_old, m);
      float l = 0.f;
      for (int i = cs.lane(); i < len; i += 32) {
        const float e = (m_new == -INFINITY) ? 0.f : expf(row[i] - m_new);
        row[i] = e;
        l += e;
      }
      l = warp_sum(l);
      if (cs.lane() == 0) {
        const float rescale = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        ml[cs.warp() * 4 + 0] = m_new;
        ml[cs.warp() * 4 + 1] = ml[cs.warp() * 4 + 1] * rescale + l;
        ml[cs.warp() * 4 + 2] = rescale;
      }
    }
    named_sync(1, NCT);
    // P.V: thread -> (d, position residue g mod 3)
    {
      const int d = cs.tid() & (HD - 1), g = cs.tid() >> 7;
      float acc[J];
#pragma unroll
      for (int j = 0; j < J; ++j) acc[j] = 0.f;
      for (int s = sa + g; s < sb; s += 3) {
        float v;
        if (s < p0) {
          const uint8_t* row = vst + static_cast<size_t>(s - sa) * ROWB;
          v = CP ? reinterpret_cast<const float*>(row)[d]
                 : __bfloat162float(reinterpret_cast<const bf16*>(row)[d]);
        } else {
          v = vn[(s - p0) * HD + d];
        }
#pragma unroll
        for (int j = 0; j < J; ++j) acc[j] = fmaf(sc[j * SUB + (s - sa)], v, acc[j]);
      }
#pragma unroll
      for (int j = 0; j < J; ++j) accg[(g * J + j) * HD + d] = acc[j];
    }
    named_sync(1, NCT);
    for (int e = cs.tid(); e < J * HD; e += NCT) {
      const int j = e / HD, d = e - j * HD;
      const float a = (accg[(0 * J + j) * HD + d] + accg[(1 * J + j) * HD + d]) + accg[(2 * J + j) * HD + d];
      acc_s[e] = acc_s[e] * ml[j * 4 + 2] + a;
    }
    named_sync(1, NCT);
  }


  // 5. publish (or finish directly when the head has a single item).
  if (GROUP) {   // head output stays in shared memory: xs[t][hh * HD + d]
    for (int e = cs.tid(); e < J * HD; e += NCT) {
      const int j = e / HD, d = e - j * HD, t = j >> 1, hh = j & 1;
      sm.xs[t * 2 * HD + hh * HD + d] = acc_s[e] / ml[j * 4 + 1];
    }
    named_sync(1, NCT);
    return true;
  }
  if (nch == 1) {
    for (int e = cs.tid(); e < J * HD; e += NCT) {
      const int j = e / HD, d = e - j * HD, t = j >> 1, hh = j & 1;
      att_store(io, t, (2 * h + hh) * HD + d, acc_s[e] / ml[j * 4 + 1]);
    }
    named_sync(1, NCT);
    return true;
  }
  for (int e = cs.tid(); e < J * PRT_STRIDE; e += NCT) {
    const int j = e / PRT_STRIDE, k = e - j * PRT_STRIDE, t = j >> 1, hh = j & 1;
    const float val = k < 2 ? ml[j * 4 + k] : (k < 4 ? 0.f : acc_s[j * HD + (k - 4)]);
    io.prt[((static_cast<size_t>(t) * NQH + 2 * h + hh) * MAX_ATT_CHUNKS + c) * PRT_STRIDE + k] = val;
  }
  named_sync(1, NCT);
  if (cs.tid() == 0) {
    __threadfence();
    const uint32_t old = atomicAdd(io.cnt, 1u);
    sm.bcast[0] = (old == static_cast<uint32_t>(nch - 1)) ? 1 : 0;
    __threadfence();
  }
  named_sync(1, NCT);
  if (sm.bcast[0]) {
    // combine the nch partials of KV head h in chunk order, staged with one round trip
    const bool staged = J * nch * PRT_STRIDE * 4 <= ATT_STAGE_BYTES;
    float* recs = reinterpret_cast<float*>(sm.att);   // [J][nch][PRT_STRIDE]
    if (staged) {
      const int pieces = nch * PRT_STRIDE / 4;
      for (int e = cs.tid(); e < J * pieces; e += NCT) {
        const int j = e / pieces, r = e - j * pieces, t = j >> 1, hh = j & 1;
        cp_async16(recs + (j * nch) * PRT_STRIDE + r * 4,
                   io.prt + ((static_cast<size_t>(t) * NQH + 2 * h + hh) * MAX_ATT_CHUNKS) * PRT_STRIDE + r * 4);
      }
      cp_async_wait_all();
      named_sync(1, NCT);
    }
    for (int e = cs.tid(); e < J * HD; e += NCT) {
      const int j = e / HD, d = e - j * HD, t = j >> 1, hh = j & 1;
      float M = -INFINITY, Ls = 0.f, O = 0.f;
      if (staged) {
        const float* rec = recs + (j * nch) * PRT_STRIDE;
        for (int cc = 0; cc < nch; ++cc) M = fmaxf(M, rec[cc * PRT_STRIDE]);
        for (int cc = 0; cc < nch; ++cc) {
          const float mc = rec[cc * PRT_STRIDE];
          if (mc == -INFINITY) continue;
          const float wgt = expf(mc - M);
          Ls = fmaf(wgt, rec[cc * PRT_STRIDE + 1], Ls);
          O = fmaf(wgt, rec[cc * PRT_STRIDE + 4 + d], O);
        }
      } else {
        const float* rec = io.prt + ((static_cast<size_t>(t) * NQH + 2 * h + hh) * MAX_ATT_CHUNKS) * PRT_STRIDE;
        for (int cc = 0; cc < nch; ++cc) M = fmaxf(M, __ldcg(rec + cc * PRT_STRIDE));
        for (int cc = 0; cc < nch; ++cc) {
          const float mc = __ldcg(rec + cc * PRT_STRIDE);
          if (mc == -INFINITY) continue;
          const float wgt = expf(mc - M);
          Ls = fmaf(wgt, __ldcg(rec + cc * PRT_STRIDE + 1), Ls);
          O = fmaf(wgt, __ldcg(rec + cc * PRT_STRIDE + 4 + d), O);
        }
      }
      att_store(io, t, (2 * h + hh) * HD + d, O / Ls);
    }
    if (cs.tid() == 0) atomicExch(io.cnt, 0u);
  }
  named_sync(1, NCT);
return true;
}


// GROUP (code predictor): the CTAs are split into 8 groups of G/8, one per KV head; every CTA
// of a group computes that head's whole attention (the context is at most 17 positions) and
// leaves the result in sm.xs[t][2][HD] for the head's o_proj columns; the first CTA of the
// group writes the new K/V rows.
template <int NT, bool CP, bool GROUP>
__device__ bool attention(const Params& p, Smem& sm, Cons& cs, const LayerW* lw, int li, int p0) {
  const int S = p0 + NT;
  int nch, chunk;
  att_split(S, cs.G(), p.att_target, nch, chunk);
  if (GROUP) {
    nch = 1;
    chunk = S;
  } else if (chunk > ATT_CHMAX) {
    fail(p, sm, DEV_ERR_BAD_POSITION);
    return false;
  }
  constexpr int ESZ = CP ? 4 : 2;
  const int max_seq = CP ? p.cp_max_seq : p.bb_max_seq;
  const size_t layer_off = static_cast<size_t>(li) * NKVH * max_seq * HD;
  const int gph = cs.G() / NKVH;
  const int n_items = GROUP ? (cs.cta() < NKVH * gph ? 1 : 0) : NKVH * nch;
  for (int item = GROUP ? 0 : cs.cta(); item < n_items; item += GROUP ? 1 : cs.G()) {
    const int h = GROUP ? cs.cta() / gph : item / nch;
    const int c = GROUP ? 0 : item - h * nch;
    const bool writer = GROUP ? (cs.cta() % gph == 0) : (c == 0);
    const int s0 = c * chunk, s1 = min(S, s0 + chunk);
    AttIO io;
    io.qkv = p.w.qkv;
    io.kb = reinterpret_cast<uint8_t*>(CP ? static_cast<void*>(p.cp_k) : static_cast<void*>(p.bb_k)) +
            (layer_off + static_cast<size_t>(h) * max_seq * HD) * ESZ;
    io.vb = reinterpret_cast<uint8_t*>(CP ? static_cast<void*>(p.cp_v) : static_cast<void*>(p.bb_v)) +
            (layer_off + static_cast<size_t>(h) * max_seq * HD) * ESZ;
    io.out = p.w.attn;
    io.hilo = nullptr;
    io.tok0 = 0;
    io.prt = p.w.prt;
    io.cnt = p.w.att_cnt + h;
    if (!att_item<NT, CP, GROUP>(p, sm, cs, lw, io, p0, h, c, nch, s0, s1, writer)) return false;
  }
  return !aborted(sm);
}

// ------------------------------------------------------------------------------------------
// One decoder layer (fused_decode_tts.cu:764-794 / fused_decode_code_predictor.cu:601-631).
// On entry sm.xs holds the raw layer input of the NT tokens and hin (global) holds the same
// values (written by the previous stage or by CTA 0 before the first barrier).
// ------------------------------------------------------------------------------------------
template <int NT, bool CP>
__device__ bool mlp_tail(const Params& p, Smem& sm, Cons& cs, const LayerW* lw, float* hout_f, HIn& hout);

template <int NT, bool CP>
__device__ bool layer(const Params& p, Smem& sm, Cons& cs, const LayerW* lw, int li, int p0, const HIn& hin,
                      float* hout_f, HIn& hout, bool input_in_smem) {
  // ---- input RMSNorm + QKV
  if (input_in_smem)
    load_rmsnorm<NT, true, true>(p, sm, cs, sm.xs, lw->in_norm, p.eps, sm.xs);
  else
    load_rmsnorm_h<NT, !CP, true>(p, sm, cs, hin, lw->in_norm, p.eps, sm.xs);
  {
    const Plan pl = make_plan(SK_QKV, nullptr, nullptr, 0, cs.cta(), cs.G());
    if (!gemv<NT, true>(p, pl, sm, cs, sm.xs, HID)) return false;
    const int nr = pl.r1 - pl.r0;
    for (int e = cs.tid(); e < NT * nr; e += NCT) {
      const int t = e / nr, r = e - t * nr;
      __stcg(p.w.qkv + t * QKV_ROWS + pl.r0 + r, sm.part[r * NT + t]);
    }
  }
  if (!grid_sync(p, sm, cs)) return false;

  // ---- q/k norm + RoPE + KV write + attention
  if (!attention<NT, CP, false>(p, sm, cs, lw, li, p0)) return false;
  if (!grid_sync(p, sm, cs)) return false;

  // ---- o_proj + residual (the residual rows are fetched with the attention output)
  {
    const Plan pl = make_plan(SK_O, nullptr, nullptr, 0, cs.cta(), cs.G());
    const int nr = pl.r1 - pl.r0;
    float res = 0.f;
    if (cs.tid() < NT * nr) res = h_ld<!CP>(hin, (cs.tid() / nr) * HID + pl.r0 + cs.tid() % nr);
    load_vec(cs, sm.xs, p.w.attn, NT * QSZ);
    named_sync(1, NCT);
    if (!gemv<NT>(p, pl, sm, cs, sm.xs, QSZ)) return false;
    if (cs.tid() < NT * nr) {
      const int t = cs.tid() / nr, r = cs.tid() % nr;
      __stcg(p.w.hmid + t * HID + pl.r0 + r, (sm.part[(2 * r) * NT + t] + sm.part[(2 * r + 1) * NT + t]) + res);
    }
  }
  if (!grid_sync(p, sm, cs)) return false;

  // ---- post-attention RMSNorm, MLP
  load_rmsnorm<NT, false, true>(p, sm, cs, p.w.hmid, lw->post_norm, p.eps, sm.xs);
  return mlp_tail<NT, CP>(p, sm, cs, lw, hout_f, hout);
}

// Fused gate/up + down stage (layers with a W_down tensor map). On entry sm.xs holds the
// post-attention RMSNorm output of the NT tokens and p.w.hmid (rows [d0, d1) of this CTA, as
// split_lo(HID, G, cta)) the residual. This CTA computes the SiLU(gate) * up values of its
// intermediate columns, their down-projection into all HID rows from the W_down boxes in the
// ring, and adds the partials (plus the residual of its own rows) into the fixed-point layer
// output hacc[dk % 3] with 64-bit integer atomics: integer addition is associative, so the
// sum does not depend on the order in which CTAs arrive. It also clears its rows of
// hacc[(dk + 1) % 3], the buffer of the next fused stage (last read two stages before).
template <int NT>
__device__ bool mlp_fused(const Params& p, Smem& sm, Cons& cs, const LayerW* lw, long long*& out) {
  const Plan pl = make_plan(SK_GUF, nullptr, nullptr, 0, cs.cta(), cs.G());
  if (!gemv<NT, true>(p, pl, sm, cs, sm.xs, HID)) return false;
  const int nj = pl.r1 - pl.r0;
  float* mv = sm.xs + NTMAX * HID;   // [NT][WD_BOX_COLS], zero beyond this CTA's columns
  if (cs.tid() < NT * WD_BOX_COLS) {
    const int t = cs.tid() / WD_BOX_COLS, j = cs.tid() - t * WD_BOX_COLS;
    float m = 0.f;
    if (j < nj) {
      const float g = sm.part[j * NT + t], u = sm.part[(nj + j) * NT + t];
      m = (g / (1.0f + expf(-g))) * u;
    }
    mv[t * WD_BOX_COLS + j] = m;
  }
  named_sync(1, NCT);

  uint32_t sl[WD_SLOTS];
  uint32_t slot = cs.slot, round = cs.round;   // ring position in registers for the stage
  bool ok = true;
#pragma unroll
  for (int i = 0; i < WD_SLOTS; ++i) {
    sl[i] = slot;
    if (ok && !mbar_wait(&sm.full[slot], round & 1u, &sm.abort)) {
      if (!aborted(sm)) fail(p, sm, DEV_ERR_FULL_TIMEOUT);
      ok = false;
    }
    if (++slot == NSLOTS) {
      slot = 0;
      round++;
    }
  }
  cs.slot = slot;
  cs.round = round;
  if (p.dbg_marks != nullptr && cs.cta() == 0 && cs.tid() == 0) {   // profiling: W_down boxes ready
    const uint32_t k = cs.bar_target / static_cast<uint32_t>(cs.G());
    if (static_cast<int>(4 * 1024 + 4 * k + 3) < p.dbg_marks_len) p.dbg_marks[4 * 1024 + 4 * k + 3] = globaltimer_ns();
  }
  const int d0 = split_lo(HID, cs.G(), cs.cta()), d1 = split_lo(HID, cs.G(), cs.cta() + 1);
  long long* acc = p.w.hacc + static_cast<size_t>(cs.dk % NHACC) * NTMAX * HID;
  long long* part = reinterpret_cast<long long*>(sm.att);   // [NT][HID] this CTA's fixed-point partials
  if (ok) {
    for (int r = cs.tid(); r < HID; r += NCT) {
      const int box = r / WD_BOX_ROWS;
      const uint8_t* row = sm.ring[box < WD_BOXES_PER_SLOT ? sl[0] : sl[1]] +
                           (box % WD_BOXES_PER_SLOT) * WD_BOX_BYTES + (r % WD_BOX_ROWS) * (WD_BOX_COLS * 2);
      float w[WD_BOX_COLS];
#pragma unroll
      for (int k = 0; k < WD_BOX_COLS / 8; ++k) {
        const uint4 v = reinterpret_cast<const uint4*>(row)[k];
        w[8 * k + 0] = bf16_lo(v.x); w[8 * k + 1] = bf16_hi(v.x);
        w[8 * k + 2] = bf16_lo(v.y); w[8 * k + 3] = bf16_hi(v.y);
        w[8 * k + 4] = bf16_lo(v.z); w[8 * k + 5] = bf16_hi(v.z);
        w[8 * k + 6] = bf16_lo(v.w); w[8 * k + 7] = bf16_hi(v.w);
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float* m = mv + t * WD_BOX_COLS;
        float a0 = w[0] * m[0], a1 = w[1] * m[1];
#pragma unroll
        for (int j = 2; j < WD_BOX_COLS; j += 2) {
          a0 = fmaf(w[j], m[j], a0);
          a1 = fmaf(w[j + 1], m[j + 1], a1);
        }
        long long q = float_to_fix(a0 + a1);
        if (r >= d0 && r < d1) q += float_to_fix(__ldcg(p.w.hmid + t * HID + r));
        part[t * HID + r] = q;
      }
    }
  }
  __syncwarp();
  if (cs.lane() == 0) {
#pragma unroll
    for (int i = 0; i < WD_SLOTS; ++i) {
      *reinterpret_cast<volatile int*>(&sm.free_epoch[sl[i]]) =
          static_cast<int>(cs.bar_target / static_cast<uint32_t>(cs.G()));
      mbar_arrive(&sm.empty[sl[i]]);
    }
  }
  // one TMA bulk reduction adds the CTA's whole partial vector into the layer output
  fence_proxy_async_smem();
  named_sync(1, NCT);
  if (cs.tid() == 0 && ok) {
    fence_proxy_async_global();   // the zeroing of acc (generic stores, earlier stages) first
    bulk_reduce_add_u64(acc, part, static_cast<uint32_t>(NT * HID * sizeof(long long)));
    bulk_commit_and_wait_all();
    fence_proxy_async_global();
  }
  long long* nxt = p.w.hacc + static_cast<size_t>((cs.dk + 1) % NHACC) * NTMAX * HID;
  for (int e = cs.tid(); e < NTMAX * (d1 - d0); e += NCT) {
    const int t = e / (d1 - d0), r = d0 + e % (d1 - d0);
    __stcg(nxt + t * HID + r, 0ll);
  }
  cs.dk++;
  out = acc;
  return !aborted(sm);
}

// MLP half of a layer after its deferred post-attention RMSNorm (x * w in sm.xs, sums of squares
// in sm.dred): the fused stage when the
// stack has W_down tensor maps, else gate/up and down as two stages.
template <int NT, bool CP>
__device__ bool mlp_tail(const Params& p, Smem& sm, Cons& cs, const LayerW* lw, float* hout_f, HIn& hout) {
  if ((CP ? p.cp_wd_map : p.bb_wd_map) != nullptr) {
    long long* acc = nullptr;
    if (!mlp_fused<NT>(p, sm, cs, lw, acc)) return false;
    hout.f = nullptr;
    hout.q = acc;
    return grid_sync(p, sm, cs);
  }
  {
    const Plan pl = make_plan(SK_GU, nullptr, nullptr, 0, cs.cta(), cs.G());
    if (!gemv<NT, true>(p, pl, sm, cs, sm.xs, HID)) return false;
    const int nj = pl.r1 - pl.r0;
    for (int e = cs.tid(); e < NT * nj; e += NCT) {
      const int t = e / nj, j = e - t * nj;
      const float g = sm.part[j * NT + t], u = sm.part[(nj + j) * NT + t];
      __stcg(p.w.mlp + t * INTER + pl.r0 + j, (g / (1.0f + expf(-g))) * u);
    }
  }
  if (!grid_sync(p, sm, cs)) return false;

  // ---- down_proj + residual
  {
    const Plan pl = make_plan(SK_D, nullptr, nullptr, 0, cs.cta(), cs.G());
    const int nr = pl.r1 - pl.r0;
    float res = 0.f;
    if (cs.tid() < NT * nr) res = __ldcg(p.w.hmid + (cs.tid() / nr) * HID + pl.r0 + cs.tid() % nr);
    load_vec(cs, sm.xs, p.w.mlp, NT * INTER);
    named_sync(1, NCT);
    if (!gemv<NT>(p, pl, sm, cs, sm.xs, INTER)) return false;
    if (cs.tid() < NT * nr) {
      const int t = cs.tid() / nr, r = cs.tid() % nr;
      float v = ((sm.part[(3 * r) * NT + t] + sm.part[(3 * r + 1) * NT + t]) + sm.part[(3 * r + 2) * NT + t]) + res;
      if (!CP) v = round_bf16(v);
      __stcg(hout_f + t * HID + pl.r0 + r, v);
    }
  }
  hout.f = hout_f;
  hout.q = nullptr;
  return grid_sync(p, sm, cs);
}

// o_proj of one KV head for the code predictor: this CTA's rows of W_o restricted to the head's
// 2*HD columns (512-byte row pieces in the ring), x = the head's attention output [NT][2*HD] in
// shared memory. Result part[r * NT + t].
template <int NT>
__device__ bool gemv_oh(const Params& p, Smem& sm, Cons& cs, int nrows, const float* x) {
  if (nrows * NT * LP_STRIDE * 4 > ATT_STAGE_BYTES) {
    fail(p, sm, DEV_ERR_BAD_POSITION);
    return false;
  }
  float* lp = reinterpret_cast<float*>(sm.att);
  uint32_t slot = cs.slot, round = cs.round;   // ring position in registers for the stage
  float xr[NT][8];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const float4 a = *reinterpret_cast<const float4*>(x + t * 2 * HD + 8 * cs.lane());
    const float4 b = *reinterpret_cast<const float4*>(x + t * 2 * HD + 8 * cs.lane() + 4);
    xr[t][0] = a.x; xr[t][1] = a.y; xr[t][2] = a.z; xr[t][3] = a.w;
    xr[t][4] = b.x; xr[t][5] = b.y; xr[t][6] = b.z; xr[t][7] = b.w;
  }
  for (int u0 = 0; u0 < nrows; u0 += OH_ROWS_PER_SLOT) {
    const int m = min(OH_ROWS_PER_SLOT, nrows - u0);
    if (!mbar_wait(&sm.full[slot], round & 1u, &sm.abort)) {
      if (!aborted(sm)) fail(p, sm, DEV_ERR_FULL_TIMEOUT);
    } else {
      for (int r = cs.warp(); r < m; r += NCW) {
        const uint4 v = reinterpret_cast<const uint4*>(sm.ring[slot] + r * OH_ROW_BYTES)[cs.lane()];
        const float w[8] = {bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y),
                            bf16_lo(v.z), bf16_hi(v.z), bf16_lo(v.w), bf16_hi(v.w)};
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float a = w[0] * xr[t][0];
#pragma unroll
          for (int j = 1; j < 8; ++j) a = fmaf(w[j], xr[t][j], a);
          lp[((u0 + r) * NT + t) * LP_STRIDE + cs.lane()] = a;
        }
      }
    }
    __syncwarp();
    if (cs.lane() == 0) {
      *reinterpret_cast<volatile int*>(&sm.free_epoch[slot]) =
          static_cast<int>(cs.bar_target / static_cast<uint32_t>(cs.G()));
      mbar_arrive(&sm.empty[slot]);
    }
    if (++slot == NSLOTS) {
      slot = 0;
      round++;
    }
  }
  cs.slot = slot;
  cs.round = round;
  named_sync(1, NCT);
  for (int e = cs.tid(); e < nrows * NT; e += NCT) {
    const float* row = lp + e * LP_STRIDE;
    float a[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) a[k] = row[k] + row[k + 16];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] += a[k + 8];
#pragma unroll
    for (int k = 0; k < 4; ++k) a[k] += a[k + 4];
    sm.part[e] = (a[0] + a[2]) + (a[1] + a[3]);
  }
  named_sync(1, NCT);
  return !aborted(sm);
}

// Code-predictor post-attention prologue: o = (sum over the 8 heads' o_proj partials, in head
// order) + residual, RMSNorm into dst; this CTA's down_proj rows of o are also stored to hmid
// for the down_proj residual.
template <int NT, bool DEFER>
__device__ void load_rmsnorm_oh(const Params& p, Smem& sm, Cons& cs, const float* opart, const HIn& hin,
                                const bf16* w, float eps, float* dst, float* hmid, int d0, int d1) {
  float4 x[NT];
  uint2 wv = make_uint2(0u, 0u);
  if (cs.tid() < HID / 4) {
    wv = *reinterpret_cast<const uint2*>(w + 4 * cs.tid());
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      float4 parts[NKVH];
#pragma unroll
      for (int h = 0; h < NKVH; ++h)
        parts[h] = __ldcg(reinterpret_cast<const float4*>(opart + (h * NTMAX + t) * HID) + cs.tid());
      const float4 r = h_ld4<false>(hin, t * HID + 4 * cs.tid());
      float4 a = parts[0];
#pragma unroll
      for (int h = 1; h < NKVH; ++h) {
        a.x += parts[h].x; a.y += parts[h].y; a.z += parts[h].z; a.w += parts[h].w;
      }
      a.x += r.x; a.y += r.y; a.z += r.z; a.w += r.w;
      x[t] = a;
      const float v4[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int idx = 4 * cs.tid() + k;
        if (idx >= d0 && idx < d1) __stcg(hmid + t * HID + idx, v4[k]);
      }
    }
  }
  rmsnorm_finish<NT, DEFER>(p, sm, cs, x, wv, eps, dst);
}

// One code-predictor layer in four grid-wide stages: QKV | attention + o_proj per KV-head group
// | RMSNorm + gate/up | down (the attention context is at most 17 positions, so each head's
// attention is computed by every CTA of its group instead of being gathered).
template <int NT>
__device__ bool layer_cp(const Params& p, Smem& sm, Cons& cs, const LayerW* lw, int li, int p0, const HIn& hin,
                         float* hout_f, HIn& hout, bool input_in_smem) {
  if (input_in_smem)
    load_rmsnorm<NT, true, true>(p, sm, cs, sm.xs, lw->in_norm, p.eps, sm.xs);
  else
    load_rmsnorm_h<NT, false, true>(p, sm, cs, hin, lw->in_norm, p.eps, sm.xs);
  {
    const Plan pl = make_plan(SK_QKV, nullptr, nullptr, 0, cs.cta(), cs.G());
    if (!gemv<NT, true>(p, pl, sm, cs, sm.xs, HID)) return false;
    const int nr = pl.r1 - pl.r0;
    for (int e = cs.tid(); e < NT * nr; e += NCT) {
      const int t = e / nr, r = e - t * nr;
      __stcg(p.w.qkv + t * QKV_ROWS + pl.r0 + r, sm.part[r * NT + t]);
    }
  }
  if (!grid_sync(p, sm, cs)) return false;

  // ---- attention of this group's KV head + its o_proj columns
  if (!attention<NT, true, true>(p, sm, cs, lw, li, p0)) return false;
  {
    int h, r0, r1;
    if (oh_rows(cs.cta(), cs.G(), h, r0, r1)) {
      const int nr = r1 - r0;
      if (!gemv_oh<NT>(p, sm, cs, nr, sm.xs)) return false;
      for (int e = cs.tid(); e < NT * nr; e += NCT) {
        const int t = e / nr, r = e - t * nr;
        __stcg(p.w.prt + (h * NTMAX + t) * HID + r0 + r, sm.part[r * NT + t]);
      }
    }
  }
  if (!grid_sync(p, sm, cs)) return false;

  // ---- o = sum of head partials + residual; RMSNorm, MLP
  {
    const int d0 = split_lo(HID, cs.G(), cs.cta()), d1 = split_lo(HID, cs.G(), cs.cta() + 1);
    load_rmsnorm_oh<NT, true>(p, sm, cs, p.w.prt, hin, lw->post_norm, p.eps, sm.xs, p.w.hmid, d0, d1);
  }
  return mlp_tail<NT, true>(p, sm, cs, lw, hout_f, hout);
}

// Runs a stack of layers; on return sm.xs holds the final-normed hidden (fp32) of NT tokens.
template <int NT, bool CP>
__device__ bool run_stack(const Params& p, Smem& sm, Cons& cs, int p0, HIn* last = nullptr) {
  const LayerW* L = CP ? p.cp_layers : p.bb_layers;
  const int n = CP ? p.n_cp : p.n_bb;
  // layer input already in sm.xs; CTA 0 publishes it for the o_proj residual.
  float* hb0 = p.w.hbuf;
  float* hb1 = p.w.hbuf + NTMAX * HID;
  if (cs.cta() == 0)
    for (int i = cs.tid(); i < NT * HID; i += NCT) __stcg(hb0 + i, sm.xs[i]);
  HIn h{hb0, nullptr};
  for (int l = 0; l < n; ++l) {
    float* hout_f = (l & 1) ? hb0 : hb1;
    HIn hout{nullptr, nullptr};
    const bool ok = CP ? layer_cp<NT>(p, sm, cs, L + l, l, p0, h, hout_f, hout, l == 0)
                       : layer<NT, CP>(p, sm, cs, L + l, l, p0, h, hout_f, hout, l == 0);
    if (!ok) return false;
    h = hout;
  }
  load_rmsnorm_h<NT, !CP>(p, sm, cs, h, CP ? p.cp_norm : p.bb_norm, p.eps, sm.xs);
  if (last) *last = h;
  return true;
}

struct SampleCfg;
__device__ __forceinline__ float head_mask(const SampleCfg& c, int i, float x);

// Orderable 64-bit key: larger value first, then smaller index (torch.argmax semantics).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(idx));
}

// Head GEMV on token t of sm.xs (bf16-cast hidden, generator.py:158,351) -> bf16 logits in
// global memory, then a grid barrier. Greedy heads (c.do_sample == 0) also apply the masks and
// fold their rows' argmax into a packed atomicMax before the barrier, so every CTA learns the
// token with one 8-byte load; returns the token, -1 when the caller must run the sampler, or -2
// on abort. `call` alternates the two argmax slots.
__device__ int head(const Params& p, Smem& sm, Cons& cs, const bf16* W, int rows, int t, const SampleCfg& c,
                    int call);

// ------------------------------------------------------------------------------------------
// Sampler (generator.py:158-172,178-207), computed redundantly by every CTA so that the
// token is known grid-wide without another barrier. Each consumer thread owns 8 contiguous
// vocabulary entries.
// ------------------------------------------------------------------------------------------
struct SampleCfg {
  int V;
  int do_sample;
  float temperature;
  int top_k;
  int suppress_from;   // ids >= suppress_from are masked, except eos (V = none)
  int eos;
  int mask_eos;
  float penalty;
  const uint8_t* seen; // nullptr = no repetition penalty
  uint32_t u24;
  float top_p;         // nucleus filter (generator.py:196-203); >= 1: off (the code predictor)
};

constexpr int SPT = VMAX / NCT;  // 8 entries per thread

__device__ __forceinline__ uint32_t bf16_key(float v) {
  uint32_t b = __float_as_uint(v) >> 16;
  if (b == 0x8000u) b = 0u;  // -0 == +0
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}

// Find the top-k threshold key: largest key K with count(key >= K) >= k.
__device__ uint32_t radix_threshold(Smem& sm, Cons& cs, const uint32_t (&key)[SPT], int k) {
  uint32_t prefix = 0;
  int need = k;
#pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
    const int shift = pass == 0 ? 8 : 0;
    for (int i = cs.tid(); i < 256; i += NCT) sm.hist[i] = 0;
    named_sync(1, NCT);
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
      if (pass == 0 || (key[j] >> 8) == (prefix >> 8)) atomicAdd(&sm.hist[(key[j] >> shift) & 0xffu], 1);
    }
    named_sync(1, NCT);
    if (cs.warp() == 0) {
      // lane l owns bins [8l, 8l+8); find the bin where the count from the top reaches need
      int c8 = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b) c8 += sm.hist[8 * cs.lane() + b];
      int above = 0;  // count in bins strictly above this lane's range
      int s = c8;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_down_sync(0xffffffffu, s, o);
        if (cs.lane() + o < 32) s += v;
      }
      above = s - c8;  // inclusive suffix minus own
      const bool mine = (above < need) && (s >= need);
      const unsigned ballot = __ballot_sync(0xffffffffu, mine);
      const int src = __ffs(ballot) - 1;
      if (cs.lane() == src) {
        int cnt = above;
        int bin = 8 * cs.lane() + 7;
        for (; bin > 8 * cs.lane(); --bin) {
          if (cnt + sm.hist[bin] >= need) break;
          cnt += sm.hist[bin];
        }
        sm.bcast[1] = bin;
        sm.bcast[2] = need - cnt;
      }
    }
    named_sync(1, NCT);
    const int bin = sm.bcast[1];
    need = sm.bcast[2];
    prefix |= static_cast<uint32_t>(bin) << shift;
    named_sync(1, NCT);
  }
  return prefix;
}

// Nucleus (top-p) filter of generator.py:196-203 on the entries the top-k filter kept: sort
// them by value, descending, ties in index order (a bitonic sort of 4096 keys (bf16 value, index)
// in sm.att), bf16 softmax over the sorted values, running sum in sorted order (fp32, each value
// rounded to bf16 as torch.cumsum on a bf16 tensor), and keep the sorted prefix up to and including
// the first entry whose running sum exceeds bf16(top_p) (the comparison runs in bf16).
constexpr int NSORT = 4096;
static_assert(NSORT * 4 <= ATT_STAGE_BYTES && NSORT >= VMAX, "nucleus sort buffer fits sm.att");
__device__ __noinline__ void nucleus_filter(Smem& sm, Cons& cs, const SampleCfg& c, const float (&v)[SPT],
                                            const uint32_t (&key)[SPT], bool (&kept)[SPT]) {
  uint32_t* sk = reinterpret_cast<uint32_t*>(sm.att);
  const int base = cs.tid() * SPT;
  auto ckey = [&](int j) {   // larger value first, then smaller index; 0 = not a candidate
    return (kept[j] && v[j] != -INFINITY) ? ((key[j] << 16) | (0xFFFFu - static_cast<uint32_t>(base + j))) : 0u;
  };
#pragma unroll
  for (int j = 0; j < SPT; ++j) sk[base + j] = ckey(j);
  for (int i = NCT * SPT + cs.tid(); i < NSORT; i += NCT) sk[i] = 0u;
  named_sync(1, NCT);
  for (int k = 2; k <= NSORT; k <<= 1)
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int i = cs.tid(); i < NSORT; i += NCT) {
        const int l = i ^ jj;
        if (l > i) {
          const uint32_t a = sk[i], b = sk[l];
          // descending order overall: blocks with (i & k) == 0 sort descending
          const bool desc = (i & k) == 0;
          if (desc ? (a < b) : (a > b)) {
            sk[i] = b;
            sk[l] = a;
          }
        }
      }
      named_sync(1, NCT);
    }
  // thread 0: softmax over the sorted candidates and the running sum in sorted order
  if (cs.tid() == 0) {
    auto val = [&](uint32_t k32) {   // the bf16 value of a key
      const uint32_t b = k32 >> 16;
      const uint32_t bits = (b & 0x8000u) ? (b & 0x7fffu) : (~b & 0xffffu);
      return __uint_as_float(bits << 16);
    };
    int n = 0;
    while (n < NSORT && sk[n] != 0u) ++n;
    uint32_t cut = 0u;
    if (n > 0) {
      // bf16 tensors as in the reference: probs = bf16(softmax), cum = bf16(fp32 running sum),
      // compared with bf16(top_p)
      const float mx = val(sk[0]);
      float es = 0.f;
      for (int i = 0; i < n; ++i) es += expf(val(sk[i]) - mx);
      const float tp = round_bf16(c.top_p);
      float cum = 0.f;
      int last = n - 1;
      for (int i = 0; i < n; ++i) {
        cum += round_bf16(__fdiv_rn(expf(val(sk[i]) - mx), es));
        if (round_bf16(cum) > tp) {
          last = i;
          break;
        }
      }
      cut = sk[last];
    }
    sm.bcast[3] = static_cast<int>(cut);
  }
  named_sync(1, NCT);
  const uint32_t cut = static_cast<uint32_t>(sm.bcast[3]);
#pragma unroll
  for (int j = 0; j < SPT; ++j) kept[j] = kept[j] && ckey(j) >= cut && cut != 0u;
  named_sync(1, NCT);
  // sm.att lies in the batched kernel's activation ring, written next by TMA
  fence_proxy_async_smem();
}

__device__ int sample(const float* logits, Smem& sm, Cons& cs, const SampleCfg& c) {
  float v[SPT];
  const int base = cs.tid() * SPT;
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    const int i = base + j;
    float x = -INFINITY;
    if (i < c.V) x = head_mask(c, i, __ldcg(logits + i));
    v[j] = x;
  }
  if (!c.do_sample) {
    // argmax, first index on ties (torch.argmax)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
      if (base + j < c.V && (bi == 0x7fffffff || v[j] > bv)) {
        bv = v[j];
        bi = base + j;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (cs.lane() == 0) {
      sm.red[cs.warp()] = bv;
      sm.red[NCW + cs.warp()] = __int_as_float(bi);
    }
    named_sync(1, NCT);
    float best = sm.red[0];
    int besti = __float_as_int(sm.red[NCW]);
    for (int w = 1; w < NCW; ++w) {
      const float ov = sm.red[w];
      const int oi = __float_as_int(sm.red[NCW + w]);
      if (ov > best || (ov == best && oi < besti)) {
        best = ov;
        besti = oi;
      }
    }
    named_sync(1, NCT);
    return besti;
  }
  // scaled = bf16(l / T)
  uint32_t key[SPT];
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    v[j] = round_bf16(__fdiv_rn(v[j], c.temperature));
    key[j] = (base + j < c.V) ? bf16_key(v[j]) : 0u;
  }
  uint32_t thr = 0;
  if (c.top_k > 0 && c.top_k < c.V) thr = radix_threshold(sm, cs, key, c.top_k);
  bool kept[SPT];
#pragma unroll
  for (int j = 0; j < SPT; ++j) kept[j] = base + j < c.V && key[j] >= thr;
  if (c.top_p < 1.f) nucleus_filter(sm, cs, c, v, key, kept);
  // softmax over kept entries (probabilities rounded to bf16 as torch.softmax on bf16)
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < SPT; ++j)
    if (kept[j]) mx = fmaxf(mx, v[j]);
  mx = warp_max(mx);
  if (cs.lane() == 0) sm.red[cs.warp()] = mx;
  named_sync(1, NCT);
  mx = sm.red[0];
  for (int w = 1; w < NCW; ++w) mx = fmaxf(mx, sm.red[w]);
  named_sync(1, NCT);
  float e[SPT];
  float es[1] = {0.f};
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    e[j] = (kept[j] && v[j] != -INFINITY) ? expf(v[j] - mx) : 0.f;
    es[0] += e[j];
  }
  block_sum<1>(sm, cs, es);
  // exact fixed-point inverse CDF over the bf16 probabilities in vocabulary order
  unsigned long long f[SPT];
  unsigned long long tsum = 0;
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    const float pr = round_bf16(__fdiv_rn(e[j], es[0]));
    f[j] = pr > 0.f ? static_cast<unsigned long long>(ldexp(static_cast<double>(pr), 60)) : 0ull;
    tsum += f[j];
  }
  // block exclusive scan of tsum
  unsigned long long incl = tsum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long n = __shfl_up_sync(0xffffffffu, incl, o);
    if (cs.lane() >= o) incl += n;
  }
  if (cs.lane() == 31) sm.ured[cs.warp()] = incl;
  named_sync(1, NCT);
  unsigned long long wpre = 0, total = 0;
  for (int w = 0; w < NCW; ++w) {
    if (w < cs.warp()) wpre += sm.ured[w];
    total += sm.ured[w];
  }
  named_sync(1, NCT);
  const unsigned long long hi = __umul64hi(static_cast<unsigned long long>(c.u24), total);
  const unsigned long long lo = static_cast<unsigned long long>(c.u24) * total;
  const unsigned long long target = (hi << 40) | (lo >> 24);
  unsigned long long cum = wpre + (incl - tsum);
  float cnt[1] = {0.f};
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    cum += f[j];
    if (base + j < c.V && cum <= target) cnt[0] += 1.f;
  }
  block_sum<1>(sm, cs, cnt);
  const int pick = static_cast<int>(cnt[0]);
  return pick < c.V ? pick : c.V - 1;
}

__device__ __forceinline__ float head_mask(const SampleCfg& c, int i, float x) {
  if (i >= c.suppress_from && i != c.eos) x = -INFINITY;
  if (c.seen != nullptr && __ldcg(c.seen + i)) x = round_bf16(x > 0.f ? __fdiv_rn(x, c.penalty) : x * c.penalty);
  if (c.mask_eos && i == c.eos) x = -INFINITY;
  return x;
}

__device__ int head(const Params& p, Smem& sm, Cons& cs, const bf16* W, int rows, int t, const SampleCfg& c,
                    int call) {
  float* x = sm.xs + t * HID;
  for (int i = cs.tid(); i < HID; i += NCT) x[i] = round_bf16(x[i]);
  named_sync(1, NCT);
  const Plan pl = make_plan(SK_HEAD, nullptr, W, rows, cs.cta(), cs.G());
  if (!gemv<1>(p, pl, sm, cs, x, HID)) return -2;
  const bool greedy = c.do_sample == 0;
  unsigned long long best = 0ull;
  for (int r = cs.tid(); r < pl.r1 - pl.r0; r += NCT) {
    const float lg = round_bf16(sm.part[r]);
    __stcg(p.w.logits + pl.r0 + r, lg);
    if (greedy) {
      const unsigned long long k = argmax_key(head_mask(c, pl.r0 + r, lg), pl.r0 + r);
      best = k > best ? k : best;
    }
  }
  if (greedy) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (cs.lane() == 0) sm.ured[cs.warp()] = best;
    named_sync(1, NCT);
    if (cs.tid() == 0) {
      unsigned long long b = 0ull;
      for (int w = 0; w < NCW; ++w) b = sm.ured[w] > b ? sm.ured[w] : b;
      if (b != 0ull) atomicMax(p.w.amax + (call & 1), b);
    }
  }
  if (!grid_sync(p, sm, cs)) return -2;
  if (!greedy) return -1;
  const unsigned long long k = __ldcg(p.w.amax + (call & 1));
  named_sync(1, NCT);   // every thread has read the slot before it can be reused
  if (cs.cta() == 0 && cs.tid() == 0) p.w.amax[(call + 1) & 1] = 0ull;   // next call's slot
  return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
}

__device__ __forceinline__ uint32_t draw_u24(const Sampling& sp, int frame, int group) {
  const uint4 r = philox4x32_10(make_uint4(static_cast<uint32_t>(frame), static_cast<uint32_t>(group),
                                           static_cast<uint32_t>(sp.philox_stream), 0u),
                                make_uint2(static_cast<uint32_t>(sp.seed), static_cast<uint32_t>(sp.seed >> 32)));
  return r.x >> 8;
}

// Write a bf16 row (as fp32) into NT slot t of sm.xs.
__device__ __forceinline__ void xs_from_bf16(Cons& cs, float* dst, const bf16* src) {
  for (int i = cs.tid(); i < HID; i += NCT) dst[i] = __bfloat162float(src[i]);
}

// ------------------------------------------------------------------------------------------
// Programs
// ------------------------------------------------------------------------------------------
__device__ bool run_frame(const Params& p, Smem& sm, Cons& cs) {
  StreamState* st = p.st;
  const int done = ld_volatile_i32(&st->done);
  const int g0 = ld_volatile_i32(&st->g0);
  const int pos = ld_volatile_i32(&st->position);
  const int step = ld_volatile_i32(&st->step);
  if (done) return true;
  if (g0 == p.sp.eos) {  // generator.py:126
    if (cs.cta() == 0 && cs.tid() == 0) st->done = 1;
    return true;
  }
  if (g0 < 0 || g0 >= p.vocab) {
    fail(p, sm, DEV_ERR_BAD_TOKEN);
    return false;
  }
  if (pos < 0 || pos >= p.bb_max_seq || pos >= p.rope_rows || step >= p.max_frames) {
    fail(p, sm, DEV_ERR_BAD_POSITION);
    return false;
  }
  if (cs.cta() == 0 && cs.tid() == 0) st->seen[g0] = 1;  // generated_g0.append (generator.py:129)

  int toks[NGROUPS];
  toks[0] = g0;
  // ---- code-predictor pass 0: [bf16(h), codec_embedding[g0]] at positions 0, 1
  for (int i = cs.tid(); i < HID; i += NCT) {
    sm.xs[i] = round_bf16(__ldcg(st->h + i));
    sm.xs[HID + i] = __bfloat162float(p.codec_emb[static_cast<size_t>(g0) * HID + i]);
  }
  named_sync(1, NCT);
  if (!run_stack<2, true>(p, sm, cs, 0)) return false;
  for (int g = 0; g < NCPHEADS; ++g) {
    if (g > 0) {
      // pass g: codec embedding g-1 of token g at position g+1 (generator.py:347-352)
      const bf16* row = p.cp_emb[g - 1] + static_cast<size_t>(toks[g]) * HID;
      xs_from_bf16(cs, sm.xs, row);
      named_sync(1, NCT);
      if (!run_stack<1, true>(p, sm, cs, g + 1)) return false;
    }
    SampleCfg c;
    c.V = p.cp_vocab;
    c.do_sample = p.sp.cp_do_sample;
    c.temperature = p.sp.cp_temperature;
    c.top_k = p.sp.cp_top_k;
    c.top_p = 1.f;
    c.suppress_from = p.cp_vocab;
    c.eos = -1;
    c.mask_eos = 0;
    c.penalty = 1.f;
    c.seen = nullptr;
    c.u24 = c.do_sample ? draw_u24(p.sp, step, g + 1) : 0u;
    const int tk = head(p, sm, cs, p.cp_head[g], p.cp_vocab, g == 0 ? 1 : 0, c, g);
    if (tk == -2) return false;
    if (p.dbg_cp_logits && cs.cta() == 0)
      for (int i = cs.tid(); i < p.cp_vocab; i += NCT) p.dbg_cp_logits[g * p.cp_vocab + i] = __ldcg(p.w.logits + i);
    toks[g + 1] = tk >= 0 ? tk : sample(p.w.logits, sm, cs, c);
  }
  // ---- combine (generator.py:143-149,356-362): sequential bf16 adds
  {
    const bf16* extra = step < p.n_trailing ? p.trailing + static_cast<size_t>(step) * HID : p.pad;
    // 8 columns per thread: the 16 table rows as 16-byte loads, all in flight together, then the
    // sequential adds (the caller's text row: bf16 loads, no alignment promised)
    for (int i8 = cs.tid(); i8 < HID / 8; i8 += NCT) {
      const int i0 = 8 * i8;
      uint4 e[NCPHEADS + 1];
      e[0] = *reinterpret_cast<const uint4*>(p.codec_emb + static_cast<size_t>(g0) * HID + i0);
#pragma unroll
      for (int q = 0; q < NCPHEADS; ++q)
        e[q + 1] = *reinterpret_cast<const uint4*>(p.cp_emb[q] + static_cast<size_t>(toks[q + 1]) * HID + i0);
      float x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = __bfloat162float(extra[i0 + i]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t* w0 = &e[0].x;
        float a = (i & 1) ? bf16_hi(w0[i >> 1]) : bf16_lo(w0[i >> 1]);
#pragma unroll
        for (int q = 0; q < NCPHEADS; ++q) {
          const uint32_t* w = &e[q + 1].x;
          a = round_bf16(a + ((i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1])));
        }
        sm.xs[i0 + i] = round_bf16(a + x[i]);
      }
    }
    named_sync(1, NCT);
  }
  // ---- backbone step at position pos
  if (!run_stack<1, false>(p, sm, cs, pos)) return false;
  if (cs.cta() == 0)
    for (int i = cs.tid(); i < HID; i += NCT) __stcg(st->h + i, sm.xs[i]);
  SampleCfg c;
  c.V = p.vocab;
  c.do_sample = p.sp.do_sample;
  c.temperature = p.sp.temperature;
  c.top_k = p.sp.top_k;
  c.top_p = p.sp.top_p;
  c.suppress_from = p.vocab - 1024;
  c.eos = p.sp.eos;
  c.mask_eos = (step + 1 < p.sp.min_new_tokens) ? 1 : 0;
  c.penalty = p.sp.repetition_penalty;
  c.seen = (p.sp.repetition_penalty != 1.f) ? st->seen : nullptr;
  c.u24 = c.do_sample ? draw_u24(p.sp, step + 1, 0) : 0u;
  const int tk = head(p, sm, cs, p.codec_head, p.vocab, 0, c, NCPHEADS);
  if (tk == -2) return false;
  if (p.dbg_g0_logits && cs.cta() == 0)
    for (int i = cs.tid(); i < p.vocab; i += NCT) p.dbg_g0_logits[i] = __ldcg(p.w.logits + i);
  const int g0n = tk >= 0 ? tk : sample(p.w.logits, sm, cs, c);
  if (cs.cta() == 0 && cs.tid() == 0) {
    int32_t* out = p.codes + static_cast<size_t>(step) * NGROUPS;
    for (int g = 0; g < NGROUPS; ++g) out[g] = toks[g];
    st->g0 = g0n;
    st->position = pos + 1;
    st->step = step + 1;
  }
  return true;
}

__device__ bool run_step(const Params& p, Smem& sm, Cons& cs, bool cp) {
  const int pos = p.position;
  const int max_seq = cp ? p.cp_max_seq : p.bb_max_seq;
  if (pos < 0 || pos >= max_seq || pos >= p.rope_rows) {
    fail(p, sm, DEV_ERR_BAD_POSITION);
    return false;
  }
  xs_from_bf16(cs, sm.xs, p.in_emb);
  named_sync(1, NCT);
  HIn last{nullptr, nullptr};
  const bool ok = cp ? run_stack<1, true>(p, sm, cs, pos, &last) : run_stack<1, false>(p, sm, cs, pos, &last);
  if (!ok) return false;
  if (cs.cta() == 0) {
    for (int i = cs.tid(); i < HID; i += NCT) {
      if (p.out_hidden) p.out_hidden[i] = sm.xs[i];
      if (p.out_raw_hidden) p.out_raw_hidden[i] = __float2bfloat16_rn(cp ? h_ld<false>(last, i) : h_ld<true>(last, i));
    }
  }
  if (!cp && (p.flags & FLAG_HEAD_SAMPLE)) {
    // end of prefill: first group-0 token (generator.py:115-120), no repetition history
    StreamState* st = p.st;
    if (cs.cta() == 0)
      for (int i = cs.tid(); i < HID; i += NCT) __stcg(st->h + i, sm.xs[i]);
    SampleCfg c;
    c.V = p.vocab;
    c.do_sample = p.sp.do_sample;
    c.temperature = p.sp.temperature;
    c.top_k = p.sp.top_k;
    c.top_p = p.sp.top_p;
    c.suppress_from = p.vocab - 1024;
    c.eos = p.sp.eos;
    c.mask_eos = p.sp.min_new_tokens > 0 ? 1 : 0;
    c.penalty = 1.f;
    c.seen = nullptr;
    c.u24 = c.do_sample ? draw_u24(p.sp, 0, 0) : 0u;
    const int tk = head(p, sm, cs, p.codec_head, p.vocab, 0, c, 0);
    if (tk == -2) return false;
    const int g0 = tk >= 0 ? tk : sample(p.w.logits, sm, cs, c);
    if (cs.cta() == 0 && cs.tid() == 0) {
      st->g0 = g0;
      st->position = pos + 1;
      st->step = 0;
      st->done = 0;
    }
  }
  return true;
}

// 13 warps over 4 SM sub-partitions: one sub-partition holds 4 warps of its 16K registers,
// so a thread gets at most 128.
extern "C" __global__ void __launch_bounds__(NTHREADS, 1) qtt_decode_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x;
  if ((p.bb_wd_map != nullptr || p.cp_wd_map != nullptr) && (smem_u32(smem_raw) & 127u) != 0u) {
    // 2-D TMA boxes land at 128-byte aligned ring offsets; every CTA leaves before any wait
    if (tid == 0) set_error(p.w.err, DEV_ERR_SMEM_ALIGN);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < NSLOTS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], NCW);
    }
    sm.abort = 0;
    sm.epoch = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const int warp = tid >> 5;
  if (warp == NCW) {
    if ((tid & 31) == 0) producer_main(p, sm, blockIdx.x, gridDim.x);
    return;
  }
  if (p.dbg_timeline != nullptr && blockIdx.x == 0 && tid == 0 && p.dbg_timeline_len > 0)
    p.dbg_timeline[0] = globaltimer_ns();
  if (blockIdx.x == 0 && tid == 0) {   // argmax slots; the first head is several barriers away
    p.w.amax[0] = 0ull;
    p.w.amax[1] = 0ull;
  }
  // attention combine counters (the first attention stage follows a grid barrier): a launch that
  // was abandoned part-way (a bounded wait that timed out) may have left them non-zero
  if (blockIdx.x == 0 && tid < NKVH) p.w.att_cnt[tid] = 0u;
  Cons cs;
  cs.slot = 0;
  cs.round = 0;
  cs.bar_target = 0;
  cs.dk = 0;
  if (p.bb_wd_map != nullptr || p.cp_wd_map != nullptr) {
    // the first fused MLP stage (several barriers away) accumulates into hacc[0]
    const int d0 = split_lo(HID, cs.G(), cs.cta()), d1 = split_lo(HID, cs.G(), cs.cta() + 1);
    for (int e = tid; e < NTMAX * (d1 - d0); e += NCT) {
      const int t = e / (d1 - d0), r = d0 + e % (d1 - d0);
      __stcg(p.w.hacc + t * HID + r, 0ll);
    }
  }
  bool ok;
  if (p.mode == MODE_FRAME)
    ok = run_frame(p, sm, cs);
  else
    ok = run_step(p, sm, cs, p.mode == MODE_CP_STEP);
  if (!ok) *reinterpret_cast<volatile int*>(&sm.abort) = 1;
}

#include "qtt_batch.cuh"

// ------------------------------------------------------------------------------------------
// Host helpers
// ------------------------------------------------------------------------------------------
size_t bwork_bytes() {
  size_t n = 256;
  n += sizeof(unsigned long long) * 5 * TBMAX;                       // ssq, amax
  n += sizeof(uint32_t) * TBMAX * NKVH;                              // att_cnt
  n += sizeof(int32_t) * BMAX * NGROUPS + 256;                       // tok
  n += 2 * sizeof(bf16) * 2 * TBMAX * ABUF_LD;                      // abuf
  n += sizeof(float) * TBMAX * HID * 3;                              // x, hb[2]
  n += sizeof(float) * TBMAX * QKV_ROWS;                             // qkv
  n += sizeof(float) * TBMAX * HID;                                  // hmid
  n += sizeof(float) * BMAX * VMAX;                                  // logits
  n += sizeof(float) * TBMAX * NQH * MAX_ATT_CHUNKS * PRT_STRIDE;   // prt
  return n;
}

void bwork_carve(void* base, BWork* w) {
  char* c = static_cast<char*>(base);
  // ssq and amax first and contiguous: one memset per launch clears both
  w->ssq = reinterpret_cast<unsigned long long*>(c); c += sizeof(unsigned long long) * 3 * TBMAX;
  w->amax = reinterpret_cast<unsigned long long*>(c); c += sizeof(unsigned long long) * 2 * TBMAX;
  w->att_cnt = reinterpret_cast<uint32_t*>(c); c += sizeof(uint32_t) * TBMAX * NKVH;
  w->tok = reinterpret_cast<int32_t*>(c); c += sizeof(int32_t) * BMAX * NGROUPS;
  c = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(c) + 255) & ~static_cast<uintptr_t>(255));
  for (int i = 0; i < 2; ++i) {
    w->abuf[i] = reinterpret_cast<bf16*>(c);
    c += sizeof(bf16) * 2 * TBMAX * ABUF_LD;
  }
  w->x = reinterpret_cast<float*>(c); c += sizeof(float) * TBMAX * HID;
  for (int i = 0; i < 2; ++i) {
    w->hb[i] = reinterpret_cast<float*>(c);
    c += sizeof(float) * TBMAX * HID;
  }
  w->qkv = reinterpret_cast<float*>(c); c += sizeof(float) * TBMAX * QKV_ROWS;
  w->hmid = reinterpret_cast<float*>(c); c += sizeof(float) * TBMAX * HID;
  w->logits = reinterpret_cast<float*>(c); c += sizeof(float) * BMAX * VMAX;
  w->prt = reinterpret_cast<float*>(c);
}

namespace {
// Launch configuration of the batched kernel: clusters of `cluster` CTAs. The launch is not
// cooperative (profilers replay cluster launches only without that attribute); the grid is sized
// from cudaOccupancyMaxActiveClusters so that every CTA is resident at once, which the grid
// barrier needs, and every wait is bounded, so a CTA that could not be placed ends the launch with
// a timeout error rather than a hang.
cudaLaunchConfig_t batch_config(int num_ctas, int cluster, size_t smem_bytes, cudaStream_t stream,
                                cudaLaunchAttribute (&attrs)[1]) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_ctas);
  cfg.blockDim = dim3(NTHREADS_B);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  return cfg;
}
}  // namespace

cudaError_t kernel_setup_b(int device, int* num_ctas, size_t* smem_bytes, int* cluster) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return e;
  const size_t smem = sizeof(Smem);
  e = cudaFuncSetAttribute(qtt_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  for (int c = 4; c >= 2; c /= 2) {
    cudaLaunchAttribute attrs[1];
    cudaLaunchConfig_t cfg = batch_config(c * (sms / c), c, smem, nullptr, attrs);
    int ncl = 0;
    e = cudaOccupancyMaxActiveClusters(&ncl, reinterpret_cast<const void*>(qtt_batch_kernel), &cfg);
    if (e != cudaSuccess) return e;
    int ctas = c * ncl;
    if (ctas > BKCTAS) ctas = (BKCTAS / c) * c;
    if (ctas > sms) ctas = (sms / c) * c;
    if (ctas >= BROWS_B) {
      *num_ctas = ctas;
      *smem_bytes = smem;
      *cluster = c;
      return cudaSuccess;
    }
  }
  return cudaErrorInvalidConfiguration;
}

cudaError_t launch_b(const Params& p, int num_ctas, size_t smem_bytes, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(p.w.bar, 0, sizeof(uint32_t), stream);
  if (e != cudaSuccess) return e;
  // ssq, amax, att_cnt and tok are contiguous at the start of the workspace
  const size_t head = reinterpret_cast<const char*>(p.bw.tok + BMAX * NGROUPS) - reinterpret_cast<const char*>(p.bw.ssq);
  e = cudaMemsetAsync(p.bw.ssq, 0, head, stream);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attrs[1];
  cudaLaunchConfig_t cfg = batch_config(num_ctas, p.bcl, smem_bytes, stream, attrs);
  return cudaLaunchKernelEx(&cfg, qtt_batch_kernel, p);
}

cudaError_t kernel_setup(int device, int* num_ctas, size_t* smem_bytes) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return e;
  const size_t smem = sizeof(Smem);
  e = cudaFuncSetAttribute(qtt_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int sms = 0, coop = 0, per_sm = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device);
  if (e != cudaSuccess) return e;
  if (!coop) return cudaErrorNotSupported;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qtt_decode_kernel, NTHREADS, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  *num_ctas = sms;
  *smem_bytes = smem;
  return cudaSuccess;
}

cudaError_t launch(const Params& p, int num_ctas, size_t smem_bytes, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(p.w.bar, 0, sizeof(uint32_t), stream);
  if (e != cudaSuccess) return e;
  void* args[] = {const_cast<Params*>(&p)};
  return cudaLaunchCooperativeKernel(reinterpret_cast<void*>(qtt_decode_kernel), dim3(num_ctas), dim3(NTHREADS), args,
                                     smem_bytes, stream);
}

}  // namespace qtt
