// Shared definitions between the persistent decode kernel (qtt_kernel.cu) and the
// host-side C-ABI (qtt_api.cu). Model shape constants are compile-time: the engine is
// specialised for the Qwen3-TTS-12Hz-0.6B shape (config.cuh:33-40 in the reference) and
// qtt_engine_create rejects any other qtt_dims.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace qtt {

typedef __nv_bfloat16 bf16;

constexpr int HID = 1024;
constexpr int INTER = 3072;
constexpr int NQH = 16;
constexpr int NKVH = 8;
constexpr int HD = 128;
constexpr int QSZ = NQH * HD;              // 2048
constexpr int KVSZ = NKVH * HD;            // 1024
constexpr int QKV_ROWS = QSZ + 2 * KVSZ;   // 4096
constexpr int NGROUPS = 16;                // codebooks per frame
constexpr int NCPHEADS = NGROUPS - 1;      // 15
constexpr int VMAX = 3072;                 // largest head (codec head)

// Weight streaming: a "unit" is 1024 consecutive bf16 of one weight row (2 KB); a ring slot
// holds 12 units (24 KB) so that rows of 1, 2 or 3 units (K = 1024, 2048, 3072) tile it and
// every consumer warp keeps the same part of the activation vector for a whole stage.
constexpr int UNIT = 1024;
constexpr int UNIT_BYTES = UNIT * 2;
constexpr int SLOT_UNITS = 12;
constexpr int SLOT_BYTES = SLOT_UNITS * UNIT_BYTES;
constexpr int NSLOTS = 7;
constexpr int NCW = 12;                    // consumer warps
constexpr int NCT = NCW * 32;              // consumer threads
constexpr int NTHREADS = NCT + 32;         // + one producer warp
constexpr int NTHREADS_B = NTHREADS + 64;  // batched kernel: + an MMA warp and an activation-loader warp
constexpr int NTMAX = 2;                   // tokens per pass (2 = code-predictor prefill pair)
constexpr int MAXPART = 256;               // partial-sum units per stage per CTA
constexpr int ATT_TARGET = 24;             // attention positions per work item (target)
constexpr int ATT_STAGE_BYTES = 24576;     // shared staging of one K+V sub-chunk
constexpr int ATT_CHMAX = 256;             // attention positions per work item (max)
constexpr int MAX_ATT_CHUNKS = 32;         // attention work items per KV head (max)
constexpr int PRT_STRIDE = HD + 4;         // partial record: m, l, 2 pad, acc[128] (16-byte rows)
constexpr int MAXUNITS = 48;               // weight units per stage per CTA (needs >= 128 CTAs)
constexpr int LP_STRIDE = 33;              // padded row of 32 lane partials
// Fused gate/up + down stage: each CTA owns a block of intermediate columns (multiples of 8,
// at most 24 with >= 128 CTAs) and streams the matching columns of W_down as four 2-D TMA
// boxes of 256 rows x 24 columns; the down-projection partials of all CTAs are summed with
// TMA bulk reductions (cp.reduce.async.bulk .add.u64) of fixed-point values (scale 2^32),
// which makes the sum independent of the order of arrival.
constexpr int WD_BOX_COLS = 24;
constexpr int WD_BOX_ROWS = 256;
constexpr int WD_BOX_BYTES = WD_BOX_COLS * WD_BOX_ROWS * 2;   // 12 KB
constexpr int WD_BOXES = HID / WD_BOX_ROWS;                   // 4
constexpr int WD_BOXES_PER_SLOT = SLOT_BYTES / WD_BOX_BYTES;  // 2
constexpr int WD_SLOTS = WD_BOXES / WD_BOXES_PER_SLOT;        // 2
constexpr int NHACC = 3;                                      // rotating fixed-point layer outputs
constexpr size_t TMAP_BYTES = 128;                            // one CUtensorMap
constexpr int ABUF_LD = INTER;   // row length (elements) of the batched bf16 hi/lo GEMM operand planes

// Same layout as TTSLayerWeights / CPLayerWeights of the reference
// (fused_decode_tts.cu:22-34, fused_decode_code_predictor.cu:30-42).
struct LayerW {
  const bf16* in_norm;
  const bf16* wq;
  const bf16* wk;
  const bf16* wv;
  const bf16* q_norm;
  const bf16* k_norm;
  const bf16* wo;
  const bf16* post_norm;
  const bf16* wg;
  const bf16* wu;
  const bf16* wd;
};

// Per-utterance decode state kept on the device so that frames run back to back with no
// host round trip.
struct StreamState {
  int position;   // next KV position of the backbone
  int step;       // frames produced so far
  int g0;         // group-0 token of the next frame
  int done;       // 1 once group 0 == EOS was reached
  int pad[4];
  float h[HID];   // final-normed backbone hidden of the last step (fp32)
  uint8_t seen[VMAX];  // repetition-penalty history of group-0 tokens
};

struct Sampling {
  int do_sample;
  float temperature;
  int top_k;
  int cp_do_sample;
  float cp_temperature;
  int cp_top_k;
  int min_new_tokens;
  float repetition_penalty;
  int eos;
  int philox_stream;
  unsigned long long seed;
  float top_p;             // nucleus filter of the group-0 sampler (>= 1: off)
};

struct Work {
  uint32_t* bar;       // grid barrier counter (zeroed before every launch)
  int* err;            // first device error code (sticky until the host clears it)
  uint32_t* att_cnt;   // [NKVH] last-arriver counters of the attention combine
  unsigned long long* amax;  // [2] packed (value, first index) greedy argmax of a head
  float* hbuf;         // [2][NTMAX][HID] layer input / output
  float* qkv;          // [NTMAX][QKV_ROWS]
  float* attn;         // [NTMAX][QSZ]
  float* prt;          // [NTMAX][NQH][MAX_ATT_CHUNKS][PRT_STRIDE]
  float* hmid;         // [NTMAX][HID]
  float* mlp;          // [NTMAX][INTER]
  float* logits;       // [VMAX]
  long long* hacc;     // [NHACC][NTMAX][HID] fused-MLP layer outputs, fixed point 2^-32
};

size_t work_bytes();
void work_carve(void* base, Work* w);

// ---- batched decode (qtt_batch_kernel): B utterances advance together, tcgen05 GEMMs
constexpr int BMAX = 64;                  // utterances per batched launch
constexpr int TBMAX = 2 * BMAX;           // tokens per stage (code-predictor first pass: 2 per utterance)
constexpr int NLMAPS = 7;                 // tensor maps per layer: q, k, v, o, gate, up, down
// Per-utterance device pointers of a batched launch.
struct BStream {
  bf16* k;                 // backbone KV [layers][8][max_seq][128] bf16
  bf16* v;
  float* cpk;              // code-predictor KV [5][8][16][128] fp32
  float* cpv;
  StreamState* st;
  int32_t* codes;          // [max_frames][16]
  const bf16* trailing;    // [n_trailing][HID]
  int n_trailing;
  int len;                 // prefill: context length
  const bf16* pad;         // [HID]
  const bf16* emb;         // prefill: context embeddings [len][HID]
  int philox;              // Philox stream of this utterance's draws
  int frame_limit;         // frames: the utterance stops once it has this many (<= max_frames)
};
// Batched scratch (one per engine).
struct BWork {
  bf16* abuf[2];           // [2 planes][TBMAX][ABUF_LD] bf16 GEMM operand: plane 0 = hi, plane 1 = lo
  float* x;                // [TBMAX][HID] stack input (residual of the first layer)
  float* hb[2];            // [TBMAX][HID] layer outputs
  float* qkv;              // [TBMAX][QKV_ROWS]
  float* hmid;             // [TBMAX][HID]
  float* logits;           // [BMAX][VMAX] sampled heads
  float* prt;              // [TBMAX][NQH][MAX_ATT_CHUNKS][PRT_STRIDE]
  uint32_t* att_cnt;       // [TBMAX][NKVH]
  unsigned long long* ssq; // [3][TBMAX] sums of squares for the next RMSNorm, fixed point 2^-32
  unsigned long long* amax;// [2][TBMAX] packed argmax of greedy heads
  int32_t* tok;            // [BMAX][NGROUPS] tokens of the frame
};
// Batched GEMM tiling: 128 CTAs per GEMM stage, as BROWS_B / C row tiles (one per cluster of C
// CTAs) x C K slices (one per CTA of the cluster).
constexpr int BROWS_B = 128;
constexpr int BKCTAS = 160;                // most CTAs a batched launch may have
size_t bwork_bytes();
void bwork_carve(void* base, BWork* w);

enum Mode : int {
  MODE_FRAME = 0, MODE_BB_STEP = 1, MODE_CP_STEP = 2,
  MODE_B_FRAME = 3,        // batched: one frame of every utterance
  MODE_B_PREFILL = 4,      // batched: backbone step b_step of every utterance with b_step < len
  MODE_B_HEAD = 5,         // batched: first group-0 token of every utterance after its prefill
  MODE_B_PREFILL_DENSE = 6,  // one utterance's context positions [b_step, b_step + b_ntok) at once
};
enum Flags : int { FLAG_HEAD_SAMPLE = 1, FLAG_EAGER_REFILL = 2 };

struct Params {
  // model (device pointers)
  const LayerW* bb_layers;
  int n_bb;
  const bf16* bb_norm;
  const bf16* codec_emb;
  const bf16* codec_head;
  int vocab;
  const LayerW* cp_layers;
  int n_cp;
  const bf16* cp_norm;
  const bf16* const* cp_emb;   // device array [15]
  const bf16* const* cp_head;  // device array [15]
  int cp_vocab;
  const bf16* cos_tab;
  const bf16* sin_tab;
  int rope_rows;
  float attn_scale;
  float eps;
  int att_target;          // attention positions per work item (target)
  // optional W_down tensor maps (device arrays of CUtensorMap, one per layer): when set, the
  // stack runs the fused gate/up + down stage; when null, separate gate/up and down stages
  const void* bb_wd_map;
  const void* cp_wd_map;
  // batched decode: tensor maps [(n_bb + n_cp) * 7 layer matrices][codec head, 15 cp heads]
  // [abuf 0 box 64, abuf 0 box 128, abuf 1 box 64, abuf 1 box 128]
  const uint8_t* bmaps;
  int nb;                  // utterances of the batched launch
  int bcl;                 // CTAs per thread-block cluster of the batched launch (4 or 2)
  int kv_pre;              // batched: the QKV epilogue applies the q/k norms + RoPE and writes the new K/V rows
  const BStream* bs;       // [nb]
  BWork bw;
  int b_step;              // MODE_B_PREFILL: context index of this step; DENSE: first position
  int b_ntok;              // MODE_B_PREFILL_DENSE: positions of this launch (<= TBMAX)
  // caches [layer][kv head][max_seq][128]
  bf16* bb_k;
  bf16* bb_v;
  int bb_max_seq;
  float* cp_k;
  float* cp_v;
  int cp_max_seq;
  Work w;
  // launch
  int mode;
  int flags;
  int position;            // step modes
  const bf16* in_emb;      // step modes: input embedding [HID] bf16
  float* out_hidden;       // step modes: final-normed fp32 hidden [HID]
  bf16* out_raw_hidden;    // optional: last layer's bf16 hidden [HID] (reference hidden_buffer)
  // frame mode
  StreamState* st;
  int32_t* codes;          // [max_frames][16]
  int max_frames;
  const bf16* trailing;    // [n_trailing][HID]
  int n_trailing;
  const bf16* pad;         // [HID]
  Sampling sp;
  // optional copies of the raw bf16 head logits of the last frame (parity tests)
  float* dbg_cp_logits;    // [15][cp_vocab]
  float* dbg_g0_logits;    // [vocab]
  // optional %globaltimer stamps (ns) taken by CTA 0 at launch start and after each grid
  // barrier: dbg_timeline[0] = start, dbg_timeline[k] = barrier k (profiling)
  unsigned long long* dbg_timeline;
  int dbg_timeline_len;
  // optional stage breakdown (profiling): CTA 0 stamps [stage][3] = GEMV start, GEMV end,
  // barrier arrival; every CTA stamps its arrival time for stages [arr_stage0, +arr_n)
  unsigned long long* dbg_marks;
  int dbg_marks_len;
  unsigned long long* dbg_arrivals;
  int dbg_arr_stage0;
  int dbg_arr_n;
  // error-path tests: when dbg_skip_barrier = k > 0, the last CTA does not arrive at the launch's
  // k-th grid barrier, and grid-barrier waits give up after dbg_wait_ns (0: QTT_WAIT_NS), so the
  // launch ends with DEV_ERR_GRID_TIMEOUT without a fault or a hang
  int dbg_skip_barrier;
  unsigned long long dbg_wait_ns;
};

// Host side: configure the kernel once per device and report the launch shape.
cudaError_t kernel_setup(int device, int* num_ctas, size_t* smem_bytes);
// Host side: zero the barrier counter and cooperatively launch one program.
cudaError_t launch(const Params& p, int num_ctas, size_t smem_bytes, cudaStream_t stream);
// Batched kernel: the same for qtt_batch_kernel (also clears the sums-of-squares and argmax words),
// launched as clusters of *cluster CTAs: 4 when at least 128 / 4 clusters of 4 fit on the device,
// else 2; num_ctas = cluster x the clusters that fit (at most BKCTAS).
cudaError_t kernel_setup_b(int device, int* num_ctas, size_t* smem_bytes, int* cluster);
cudaError_t launch_b(const Params& p, int num_ctas, size_t smem_bytes, cudaStream_t stream);
// Error code of the last qtt_backbone_step_noalloc on device `dev` (0: none, or the path is
// unused there); clears it. Defined with the fixed scratch in qtt_noalloc.cu.
cudaError_t noalloc_take_error(int dev, int* code);

}  // namespace qtt
