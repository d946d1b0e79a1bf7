// Host side of libqtt: the drop-in launchers and the engine API declared in include/qtt.h.
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include <cuda.h>

#include "../../include/qtt.h"
#include "qtt_kernel.cuh"
#include "qtt_device.cuh"

using qtt::bf16;

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// Tensor map of a bf16 row-major matrix [rows][cols] for the batched GEMMs: boxes of 64 columns
// (128 bytes) x box_rows rows with the 128-byte swizzle that tcgen05 K-major operands use.
bool encode_sw128(const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows, CUtensorMap* out) {
  const EncodeTiledFn fn = encode_tiled();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * sizeof(bf16)};
  const cuuint32_t box[2] = {64u, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of one W_down [HID][INTER] (bf16, row-major) for the fused MLP stage: boxes of
// WD_BOX_ROWS rows x WD_BOX_COLS columns, no swizzle, zero fill beyond the last column.
bool encode_wd_map(const void* wd, CUtensorMap* out) {
  static_assert(sizeof(CUtensorMap) == qtt::TMAP_BYTES, "CUtensorMap size");
  const EncodeTiledFn fn = encode_tiled();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(qtt::INTER), static_cast<cuuint64_t>(qtt::HID)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(qtt::INTER) * sizeof(bf16)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(qtt::WD_BOX_COLS), static_cast<cuuint32_t>(qtt::WD_BOX_ROWS)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(wd), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

thread_local int g_last_status = QTT_OK;

qtt_status from_cuda(cudaError_t e) {
  if (e == cudaSuccess) return QTT_OK;
  if (e == cudaErrorMemoryAllocation) return QTT_ERR_OOM;
  return QTT_ERR_CUDA;
}

qtt_status from_dev(int code) {
  switch (code) {
    case qtt::DEV_OK: return QTT_OK;
    case qtt::DEV_ERR_GRID_TIMEOUT:
    case qtt::DEV_ERR_FULL_TIMEOUT:
    case qtt::DEV_ERR_EMPTY_TIMEOUT:
    case qtt::DEV_ERR_ABORTED: return QTT_ERR_TIMEOUT;
    case qtt::DEV_ERR_BAD_TOKEN: return QTT_ERR_BAD_TOKEN;
    case qtt::DEV_ERR_BAD_POSITION: return QTT_ERR_BAD_POSITION;
    default: return QTT_ERR_DEVICE;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool layer_ok(const TTSLayerWeights& l) {
  const void* ps[11] = {l.input_layernorm_weight, l.q_proj_weight, l.k_proj_weight, l.v_proj_weight,
                        l.q_norm_weight, l.k_norm_weight, l.o_proj_weight, l.post_attn_layernorm_weight,
                        l.gate_proj_weight, l.up_proj_weight, l.down_proj_weight};
  for (const void* p : ps)
    if (p == nullptr || !aligned16(p)) return false;
  return true;
}

// Kernel launch shape per device (kernel_setup is cheap but sets function attributes).
struct DevShape {
  int ctas = 0;
  size_t smem = 0;
};

std::mutex g_mu;
std::map<int, DevShape> g_shapes;

cudaError_t device_shape(int dev, DevShape* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_shapes.find(dev);
  if (it != g_shapes.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  DevShape s;
  cudaError_t e = qtt::kernel_setup(dev, &s.ctas, &s.smem);
  if (e != cudaSuccess) return e;
  g_shapes[dev] = s;
  *out = s;
  return cudaSuccess;
}

// Scratch of the drop-in launchers, one per (device, stream), allocated on first use.
struct CompatWork {
  void* mem = nullptr;
  qtt::Work w{};
};
std::map<std::pair<int, cudaStream_t>, CompatWork> g_compat;

cudaError_t compat_work(int dev, cudaStream_t stream, qtt::Work* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_pair(dev, stream);
  auto it = g_compat.find(key);
  if (it != g_compat.end()) {
    *out = it->second.w;
    return cudaSuccess;
  }
  CompatWork cw;
  cudaError_t e = cudaMalloc(&cw.mem, qtt::work_bytes());
  if (e != cudaSuccess) return e;
  e = cudaMemset(cw.mem, 0, qtt::work_bytes());
  if (e != cudaSuccess) return e;
  qtt::work_carve(cw.mem, &cw.w);
  g_compat[key] = cw;
  *out = cw.w;
  return cudaSuccess;
}

int compat_step(bool cp, const void* input_embedding, const TTSLayerWeights* layer_weights,
                const void* final_norm_weight, const void* cos_table, const void* sin_table, void* k_cache,
                void* v_cache, void* hidden_buffer, void* g_normalized, int num_layers, int position,
                int cache_len, int max_seq_len, float attn_scale, cudaStream_t stream) {
  if (!input_embedding || !layer_weights || !final_norm_weight || !cos_table || !sin_table || !k_cache ||
      !v_cache || !g_normalized || num_layers < 1 || max_seq_len < 1 || position < 0 ||
      position >= max_seq_len || cache_len != position + 1 || !aligned16(input_embedding) ||
      !aligned16(k_cache) || !aligned16(v_cache))
    return QTT_ERR_INVALID_ARG;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return from_cuda(e);
  DevShape shape;
  e = device_shape(dev, &shape);
  if (e != cudaSuccess) return from_cuda(e);
  if (max_seq_len > (shape.ctas / qtt::NKVH) * qtt::ATT_CHMAX || shape.ctas < 128) return QTT_ERR_UNSUPPORTED;
  qtt::Work w;
  e = compat_work(dev, stream, &w);
  if (e != cudaSuccess) return from_cuda(e);
  qtt::Params p;
  std::memset(&p, 0, sizeof(p));
  const qtt::LayerW* layers = reinterpret_cast<const qtt::LayerW*>(layer_weights);
  if (cp) {
    p.cp_layers = layers;
    p.n_cp = num_layers;
    p.cp_norm = static_cast<const bf16*>(final_norm_weight);
    p.cp_k = static_cast<float*>(k_cache);
    p.cp_v = static_cast<float*>(v_cache);
    p.cp_max_seq = max_seq_len;
    p.mode = qtt::MODE_CP_STEP;
  } else {
    p.bb_layers = layers;
    p.n_bb = num_layers;
    p.bb_norm = static_cast<const bf16*>(final_norm_weight);
    p.bb_k = static_cast<bf16*>(k_cache);
    p.bb_v = static_cast<bf16*>(v_cache);
    p.bb_max_seq = max_seq_len;
    p.out_raw_hidden = static_cast<bf16*>(hidden_buffer);
    p.mode = qtt::MODE_BB_STEP;
  }
  p.cos_tab = static_cast<const bf16*>(cos_table);
  p.sin_tab = static_cast<const bf16*>(sin_table);
  p.rope_rows = max_seq_len;  // the reference builds [max_seq_len, 128] tables
  p.attn_scale = attn_scale;
  p.eps = 1e-6f;
  p.w = w;
  p.position = position;
  p.in_emb = static_cast<const bf16*>(input_embedding);
  p.out_hidden = static_cast<float*>(g_normalized);
  return from_cuda(qtt::launch(p, shape.ctas, shape.smem, stream));
}

}  // namespace

// ==========================================================================================
// Drop-in launchers
// ==========================================================================================
extern "C" void launch_tts_decode_with_embedding(const void* input_embedding, const TTSLayerWeights* layer_weights,
                                                 const void* final_norm_weight, const void* cos_table,
                                                 const void* sin_table, void* k_cache, void* v_cache,
                                                 void* hidden_buffer, void*, void*, void*, void*, void*, void*,
                                                 void*, void* g_normalized, int num_layers, int position,
                                                 int cache_len, int max_seq_len, float attn_scale,
                                                 cudaStream_t stream) {
  g_last_status = compat_step(false, input_embedding, layer_weights, final_norm_weight, cos_table, sin_table,
                              k_cache, v_cache, hidden_buffer, g_normalized, num_layers, position, cache_len,
                              max_seq_len, attn_scale, stream);
}

extern "C" void launch_tts_decode(int input_token_id, const void* embed_weight, const TTSLayerWeights* layer_weights,
                                  const void* final_norm_weight, const void* cos_table, const void* sin_table,
                                  void* k_cache, void* v_cache, void* hidden_buffer, void*, void*, void*, void*,
                                  void*, void*, void*, void* g_normalized, int num_layers, int position,
                                  int cache_len, int max_seq_len, float attn_scale, cudaStream_t stream) {
  if (!embed_weight || input_token_id < 0) {
    g_last_status = QTT_ERR_INVALID_ARG;
    return;
  }
  const void* emb = static_cast<const bf16*>(embed_weight) + static_cast<size_t>(input_token_id) * qtt::HID;
  g_last_status = compat_step(false, emb, layer_weights, final_norm_weight, cos_table, sin_table, k_cache, v_cache,
                              hidden_buffer, g_normalized, num_layers, position, cache_len, max_seq_len,
                              attn_scale, stream);
}

extern "C" void launch_cp_decode_with_embedding(const void* input_embedding, const CPLayerWeights* layer_weights,
                                                const void* final_norm_weight, const void* cos_table,
                                                const void* sin_table, void* k_cache, void* v_cache, void*, void*,
                                                void*, void*, void*, void*, void*, void*, void* g_normalized,
                                                int num_layers, int position, int cache_len, int max_seq_len,
                                                float attn_scale, cudaStream_t stream) {
  g_last_status = compat_step(true, input_embedding, layer_weights, final_norm_weight, cos_table, sin_table,
                              k_cache, v_cache, nullptr, g_normalized, num_layers, position, cache_len,
                              max_seq_len, attn_scale, stream);
}

extern "C" int qtt_last_launch_status(void) { return g_last_status; }

#ifndef QTT_BUILD_ID
#define QTT_BUILD_ID "unstamped"
#endif
extern "C" const char* qtt_build_id(void) { return QTT_BUILD_ID; }

extern "C" int qtt_stream_check(cudaStream_t stream) {
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return from_cuda(e);
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return from_cuda(e);
  // steps of qtt_backbone_step_noalloc keep their error word in the library's fixed scratch
  int noalloc_code = 0;
  e = qtt::noalloc_take_error(dev, &noalloc_code);
  if (e != cudaSuccess) return from_cuda(e);
  qtt::Work w;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_compat.find(std::make_pair(dev, stream));
    if (it == g_compat.end()) return from_dev(noalloc_code);
    w = it->second.w;
  }
  int code = 0;
  e = cudaMemcpy(&code, w.err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return from_cuda(e);
  if (code != 0) {
    const int zero = 0;
    cudaMemcpy(w.err, &zero, sizeof(int), cudaMemcpyHostToDevice);
  }
  return from_dev(code != 0 ? code : noalloc_code);
}

// ==========================================================================================
// Engine
// ==========================================================================================
struct StreamBufs {
  bf16* k = nullptr;
  bf16* v = nullptr;
  qtt::StreamState* st = nullptr;
  int32_t* codes = nullptr;
  int philox = -1;        // qtt_set_stream_params: own Philox stream (-1: the launch's default)
  int frame_limit = 0;    // > 0: frame limit, 0: max_frames, < 0: parked
};

struct qtt_engine {
  // batched decode resources (allocated on the first batched call)
  std::vector<TTSLayerWeights> h_bb, h_cp;   // host copies of the layer tables
  const void* h_codec_head = nullptr;
  const void* h_cp_head[qtt::NCPHEADS] = {};
  DevShape bshape;
  int bcl = 0;               // CTAs per cluster of the batched kernel
  int dbg_kv_in_attention = 0;   // test hook: the batched attention stage writes the K/V rows
  bool b_ready = false;
  void* d_bwork = nullptr;
  void* d_bmaps = nullptr;
  qtt::BStream* d_bs = nullptr;
  float* d_cpkv = nullptr;
  qtt::StreamState** d_stptr = nullptr;   // qtt_batch_states: state pointers, gathered words, pinned copy
  int32_t** d_codeptr = nullptr;          // qtt_batch_last_codes: each stream's code buffer
  int32_t* d_states = nullptr;
  int32_t* h_states = nullptr;
  std::vector<qtt::BStream> h_bs;
  float* b_dbg_cp = nullptr;   // batched debug logits [B][15][cp_vocab], [B][vocab]
  float* b_dbg_g0 = nullptr;
  int device = 0;
  DevShape shape;
  qtt_dims dims{};
  int max_streams = 0, max_seq = 0, max_frames = 0;
  qtt::LayerW* d_bb = nullptr;
  qtt::LayerW* d_cp = nullptr;
  const bf16** d_cp_emb = nullptr;
  const bf16** d_cp_head = nullptr;
  void* d_maps = nullptr;   // W_down tensor maps: [backbone layers] then [cp layers]
  void* d_work = nullptr;
  float* cp_k = nullptr;
  float* cp_v = nullptr;
  qtt::Params base{};
  std::vector<StreamBufs> streams;
};

namespace {
constexpr int kCpMaxSeq = 16;  // code-predictor positions per frame: 0..15

qtt_status set_device(const qtt_engine* e) { return from_cuda(cudaSetDevice(e->device)); }

qtt_status check_sampling(const qtt_sampling* sp, const qtt_engine* e) {
  if (!sp) return QTT_ERR_INVALID_ARG;
  if (!(sp->top_p >= 0.f)) return QTT_ERR_INVALID_ARG;   // NaN or negative
  if (sp->do_sample && !(sp->temperature > 0.f)) return QTT_ERR_INVALID_ARG;
  if (sp->cp_do_sample && !(sp->cp_temperature > 0.f)) return QTT_ERR_INVALID_ARG;
  if (!(sp->repetition_penalty > 0.f)) return QTT_ERR_INVALID_ARG;
  if (sp->eos_token_id < 0 || sp->eos_token_id >= e->dims.vocab) return QTT_ERR_INVALID_ARG;
  return QTT_OK;
}

qtt::Sampling to_dev(const qtt_sampling* sp) {
  qtt::Sampling s{};
  s.do_sample = sp->do_sample;
  s.temperature = sp->temperature;
  s.top_k = sp->top_k;
  s.cp_do_sample = sp->cp_do_sample;
  s.cp_temperature = sp->cp_temperature;
  s.cp_top_k = sp->cp_top_k;
  s.min_new_tokens = sp->min_new_tokens;
  s.repetition_penalty = sp->repetition_penalty;
  s.eos = sp->eos_token_id;
  s.philox_stream = sp->philox_stream;
  s.seed = sp->seed;
  s.top_p = sp->top_p;
  return s;
}

void engine_free(qtt_engine* e) {
  for (auto& s : e->streams) {
    cudaFree(s.k);
    cudaFree(s.v);
    cudaFree(s.st);
    cudaFree(s.codes);
  }
  cudaFree(e->d_bb);
  cudaFree(e->d_cp);
  cudaFree(e->d_cp_emb);
  cudaFree(e->d_cp_head);
  cudaFree(e->d_maps);
  cudaFree(e->d_bwork);
  cudaFree(e->d_bmaps);
  cudaFree(e->d_bs);
  cudaFree(e->d_cpkv);
  cudaFree(e->d_stptr);
  cudaFree(e->d_codeptr);
  cudaFree(e->d_states);
  cudaFreeHost(e->h_states);
  cudaFree(e->d_work);
  cudaFree(e->cp_k);
  cudaFree(e->cp_v);
  delete e;
}

__global__ void kv_f32_to_bf16(const float* __restrict__ src, bf16* __restrict__ dst, int rows, int len,
                               int max_seq) {
  const size_t n = static_cast<size_t>(rows) * len * qtt::HD;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / (static_cast<size_t>(len) * qtt::HD);
    const size_t rem = i - row * len * qtt::HD;
    dst[row * static_cast<size_t>(max_seq) * qtt::HD + rem] = __float2bfloat16_rn(src[i]);
  }
}

}  // namespace

extern "C" const char* qtt_status_string(qtt_status s) {
  switch (s) {
    case QTT_OK: return "ok";
    case QTT_ERR_INVALID_ARG: return "invalid argument";
    case QTT_ERR_CUDA: return "CUDA error";
    case QTT_ERR_OOM: return "out of device memory";
    case QTT_ERR_TIMEOUT: return "device wait timed out";
    case QTT_ERR_UNSUPPORTED: return "unsupported shape or option";
    case QTT_ERR_BAD_TOKEN: return "token id out of range";
    case QTT_ERR_BAD_POSITION: return "position beyond the KV cache";
    case QTT_ERR_DEVICE: return "device error";
  }
  return "unknown status";
}

extern "C" qtt_status qtt_engine_create(const qtt_weights* w, const qtt_dims* d, int device, int max_streams,
                                        int max_seq, int max_frames, qtt_engine** out) {
  if (!w || !d || !out || max_streams < 1 || max_seq < 1 || max_frames < 1) return QTT_ERR_INVALID_ARG;
  *out = nullptr;
  if (d->hidden != qtt::HID || d->intermediate != qtt::INTER || d->n_q_heads != qtt::NQH ||
      d->n_kv_heads != qtt::NKVH || d->head_dim != qtt::HD || d->n_groups != qtt::NGROUPS ||
      d->vocab < 1025 || d->vocab > qtt::VMAX || d->cp_vocab < 1 || d->cp_vocab > qtt::VMAX ||
      d->backbone_layers < 1 || d->cp_layers < 1)
    return QTT_ERR_UNSUPPORTED;
  if (!w->backbone_layers || !w->cp_layers || !w->backbone_norm || !w->codec_embedding || !w->codec_head ||
      !w->cp_norm || !w->rope_cos || !w->rope_sin || w->rope_rows < 1)
    return QTT_ERR_INVALID_ARG;
  if (!aligned16(w->codec_embedding) || !aligned16(w->codec_head)) return QTT_ERR_INVALID_ARG;
  for (int i = 0; i < d->backbone_layers; ++i)
    if (!layer_ok(w->backbone_layers[i])) return QTT_ERR_INVALID_ARG;
  for (int i = 0; i < d->cp_layers; ++i)
    if (!layer_ok(w->cp_layers[i])) return QTT_ERR_INVALID_ARG;
  for (int g = 0; g < qtt::NCPHEADS; ++g)
    if (!w->cp_codec_embedding[g] || !w->cp_lm_head[g] || !aligned16(w->cp_lm_head[g]) ||
        !aligned16(w->cp_codec_embedding[g]))
      return QTT_ERR_INVALID_ARG;

  qtt_engine* e = new qtt_engine();
  e->device = device;
  e->dims = *d;
  e->max_streams = max_streams;
  e->max_seq = max_seq;
  e->max_frames = max_frames;
  cudaError_t ce = cudaSetDevice(device);
  if (ce == cudaSuccess) ce = device_shape(device, &e->shape);
  if (ce != cudaSuccess) {
    delete e;
    return from_cuda(ce);
  }
  if (max_seq > (e->shape.ctas / qtt::NKVH) * qtt::ATT_CHMAX || e->shape.ctas < 128) {
    delete e;
    return QTT_ERR_UNSUPPORTED;
  }
  const size_t lw = sizeof(qtt::LayerW);
#define QTT_TRY(x)              \
  do {                          \
    ce = (x);                   \
    if (ce != cudaSuccess) {    \
      engine_free(e);           \
      return from_cuda(ce);     \
    }                           \
  } while (0)
  QTT_TRY(cudaMalloc(&e->d_bb, lw * d->backbone_layers));
  QTT_TRY(cudaMemcpy(e->d_bb, w->backbone_layers, lw * d->backbone_layers, cudaMemcpyHostToDevice));
  QTT_TRY(cudaMalloc(&e->d_cp, lw * d->cp_layers));
  QTT_TRY(cudaMemcpy(e->d_cp, w->cp_layers, lw * d->cp_layers, cudaMemcpyHostToDevice));
  QTT_TRY(cudaMalloc(reinterpret_cast<void**>(&e->d_cp_emb), sizeof(void*) * qtt::NCPHEADS));
  QTT_TRY(cudaMemcpy(e->d_cp_emb, w->cp_codec_embedding, sizeof(void*) * qtt::NCPHEADS, cudaMemcpyHostToDevice));
  QTT_TRY(cudaMalloc(reinterpret_cast<void**>(&e->d_cp_head), sizeof(void*) * qtt::NCPHEADS));
  QTT_TRY(cudaMemcpy(e->d_cp_head, w->cp_lm_head, sizeof(void*) * qtt::NCPHEADS, cudaMemcpyHostToDevice));
  // Fused gate/up + down stage: one W_down tensor map per layer (QTT_FUSED_MLP=0 selects the
  // two-stage MLP, for comparison).
  bool fused_mlp = true;
  if (const char* v = std::getenv("QTT_FUSED_MLP")) fused_mlp = std::atoi(v) != 0;
  if (fused_mlp) {
    const int nl = d->backbone_layers + d->cp_layers;
    std::vector<CUtensorMap> maps(nl);
    for (int i = 0; i < nl && fused_mlp; ++i) {
      const void* wd = i < d->backbone_layers ? w->backbone_layers[i].down_proj_weight
                                              : w->cp_layers[i - d->backbone_layers].down_proj_weight;
      fused_mlp = encode_wd_map(wd, &maps[i]);
    }
    if (fused_mlp) {
      QTT_TRY(cudaMalloc(&e->d_maps, qtt::TMAP_BYTES * nl));
      QTT_TRY(cudaMemcpy(e->d_maps, maps.data(), qtt::TMAP_BYTES * nl, cudaMemcpyHostToDevice));
    }
  }
  QTT_TRY(cudaMalloc(&e->d_work, qtt::work_bytes()));
  QTT_TRY(cudaMemset(e->d_work, 0, qtt::work_bytes()));
  const size_t cp_kv = sizeof(float) * d->cp_layers * qtt::NKVH * kCpMaxSeq * qtt::HD;
  QTT_TRY(cudaMalloc(&e->cp_k, cp_kv));
  QTT_TRY(cudaMalloc(&e->cp_v, cp_kv));
  QTT_TRY(cudaMemset(e->cp_k, 0, cp_kv));
  QTT_TRY(cudaMemset(e->cp_v, 0, cp_kv));
  const size_t kv = sizeof(bf16) * static_cast<size_t>(d->backbone_layers) * qtt::NKVH * max_seq * qtt::HD;
  e->streams.resize(max_streams);
  for (auto& s : e->streams) {
    QTT_TRY(cudaMalloc(&s.k, kv));
    QTT_TRY(cudaMalloc(&s.v, kv));
    QTT_TRY(cudaMalloc(&s.st, sizeof(qtt::StreamState)));
    QTT_TRY(cudaMalloc(&s.codes, sizeof(int32_t) * qtt::NGROUPS * max_frames));
    QTT_TRY(cudaMemset(s.k, 0, kv));
    QTT_TRY(cudaMemset(s.v, 0, kv));
    QTT_TRY(cudaMemset(s.st, 0, sizeof(qtt::StreamState)));
    QTT_TRY(cudaMemset(s.codes, 0, sizeof(int32_t) * qtt::NGROUPS * max_frames));
  }
#undef QTT_TRY
  e->h_bb.assign(w->backbone_layers, w->backbone_layers + d->backbone_layers);
  e->h_cp.assign(reinterpret_cast<const TTSLayerWeights*>(w->cp_layers),
                 reinterpret_cast<const TTSLayerWeights*>(w->cp_layers) + d->cp_layers);
  e->h_codec_head = w->codec_head;
  for (int g = 0; g < qtt::NCPHEADS; ++g) e->h_cp_head[g] = w->cp_lm_head[g];
  qtt::Params& p = e->base;
  std::memset(&p, 0, sizeof(p));
  p.bb_layers = e->d_bb;
  p.n_bb = d->backbone_layers;
  p.bb_norm = static_cast<const bf16*>(w->backbone_norm);
  p.codec_emb = static_cast<const bf16*>(w->codec_embedding);
  p.codec_head = static_cast<const bf16*>(w->codec_head);
  p.vocab = d->vocab;
  p.cp_layers = e->d_cp;
  p.n_cp = d->cp_layers;
  p.cp_norm = static_cast<const bf16*>(w->cp_norm);
  p.cp_emb = e->d_cp_emb;
  p.cp_head = e->d_cp_head;
  p.cp_vocab = d->cp_vocab;
  p.cos_tab = static_cast<const bf16*>(w->rope_cos);
  p.sin_tab = static_cast<const bf16*>(w->rope_sin);
  p.rope_rows = w->rope_rows;
  p.attn_scale = d->attn_scale;
  p.eps = d->rms_eps;
  p.att_target = qtt::ATT_TARGET;
  if (const char* v = std::getenv("QTT_ATT_TARGET")) {   // tuning knob: attention positions per item
    const int t = std::atoi(v);
    if (t >= 8 && t <= qtt::ATT_CHMAX) p.att_target = t;
  }
  if (e->d_maps) {
    p.bb_wd_map = e->d_maps;
    p.cp_wd_map = static_cast<const uint8_t*>(e->d_maps) + qtt::TMAP_BYTES * d->backbone_layers;
  }
  p.bb_max_seq = max_seq;
  p.cp_k = e->cp_k;
  p.cp_v = e->cp_v;
  p.cp_max_seq = kCpMaxSeq;
  qtt::work_carve(e->d_work, &p.w);
  p.max_frames = max_frames;
  *out = e;
  return QTT_OK;
}

extern "C" qtt_status qtt_engine_destroy(qtt_engine* e) {
  if (!e) return QTT_ERR_INVALID_ARG;
  cudaSetDevice(e->device);
  cudaDeviceSynchronize();
  engine_free(e);
  return QTT_OK;
}

extern "C" int qtt_engine_num_ctas(const qtt_engine* e) { return e ? e->shape.ctas : 0; }

#define QTT_STREAM_CHECK(e, s) \
  if (!(e) || (s) < 0 || (s) >= (e)->max_streams) return QTT_ERR_INVALID_ARG

extern "C" qtt_status qtt_reset(qtt_engine* e, int s, cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  const size_t kv = sizeof(bf16) * static_cast<size_t>(e->dims.backbone_layers) * qtt::NKVH * e->max_seq * qtt::HD;
  StreamBufs& b = e->streams[s];
  cudaError_t ce = cudaMemsetAsync(b.k, 0, kv, stream);
  if (ce == cudaSuccess) ce = cudaMemsetAsync(b.v, 0, kv, stream);
  if (ce == cudaSuccess) ce = cudaMemsetAsync(b.st, 0, sizeof(qtt::StreamState), stream);
  return from_cuda(ce);
}

extern "C" qtt_status qtt_set_kv(qtt_engine* e, int s, const void* k, const void* v, int len, int dtype,
                                 cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  if (!k || !v || len < 0 || len > e->max_seq || (dtype != 0 && dtype != 1)) return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK || len == 0) return r;
  StreamBufs& b = e->streams[s];
  const int rows = e->dims.backbone_layers * qtt::NKVH;
  cudaError_t ce;
  if (dtype == 0) {
    const size_t w = static_cast<size_t>(len) * qtt::HD * sizeof(bf16);
    const size_t dp = static_cast<size_t>(e->max_seq) * qtt::HD * sizeof(bf16);
    ce = cudaMemcpy2DAsync(b.k, dp, k, w, w, rows, cudaMemcpyDeviceToDevice, stream);
    if (ce == cudaSuccess) ce = cudaMemcpy2DAsync(b.v, dp, v, w, w, rows, cudaMemcpyDeviceToDevice, stream);
  } else {
    kv_f32_to_bf16<<<592, 256, 0, stream>>>(static_cast<const float*>(k), b.k, rows, len, e->max_seq);
    kv_f32_to_bf16<<<592, 256, 0, stream>>>(static_cast<const float*>(v), b.v, rows, len, e->max_seq);
    ce = cudaGetLastError();
  }
  return from_cuda(ce);
}

extern "C" qtt_status qtt_get_kv(qtt_engine* e, int s, void** k, void** v, int* max_seq) {
  QTT_STREAM_CHECK(e, s);
  if (k) *k = e->streams[s].k;
  if (v) *v = e->streams[s].v;
  if (max_seq) *max_seq = e->max_seq;
  return QTT_OK;
}

extern "C" qtt_status qtt_set_position(qtt_engine* e, int s, int position, cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  if (position < 0 || position > e->max_seq) return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  // pinned-free path: a tiny kernel-free memcpy of a host int must outlive the call, so
  // copy synchronously with respect to the host.
  cudaError_t ce = cudaStreamSynchronize(stream);
  if (ce == cudaSuccess)
    ce = cudaMemcpy(&e->streams[s].st->position, &position, sizeof(int), cudaMemcpyHostToDevice);
  return from_cuda(ce);
}

extern "C" qtt_status qtt_get_state(qtt_engine* e, int s, int* position, int* frames, int* g0, int* done,
                                    cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  cudaError_t ce = cudaStreamSynchronize(stream);
  int hdr[4] = {0, 0, 0, 0};
  if (ce == cudaSuccess) ce = cudaMemcpy(hdr, e->streams[s].st, sizeof(hdr), cudaMemcpyDeviceToHost);
  if (ce != cudaSuccess) return from_cuda(ce);
  if (position) *position = hdr[0];
  if (frames) *frames = hdr[1];
  if (g0) *g0 = hdr[2];
  if (done) *done = hdr[3];
  return QTT_OK;
}

extern "C" qtt_status qtt_backbone_step(qtt_engine* e, int s, const void* emb, int position, float* out_hidden,
                                        cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  if (!emb || !aligned16(emb) || position < 0 || position >= e->max_seq || position >= e->base.rope_rows)
    return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  qtt::Params p = e->base;
  p.mode = qtt::MODE_BB_STEP;
  p.bb_k = e->streams[s].k;
  p.bb_v = e->streams[s].v;
  p.st = e->streams[s].st;
  p.position = position;
  p.in_emb = static_cast<const bf16*>(emb);
  p.out_hidden = out_hidden;
  return from_cuda(qtt::launch(p, e->shape.ctas, e->shape.smem, stream));
}

extern "C" qtt_status qtt_prefill(qtt_engine* e, int s, const void* embeds, int len, const qtt_sampling* sp,
                                  cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  if (!embeds || !aligned16(embeds) || len < 1 || len >= e->max_seq || len > e->base.rope_rows)
    return QTT_ERR_INVALID_ARG;
  qtt_status r = check_sampling(sp, e);
  if (r != QTT_OK) return r;
  r = qtt_reset(e, s, stream);
  if (r != QTT_OK) return r;
  qtt::Params p = e->base;
  p.mode = qtt::MODE_BB_STEP;
  p.bb_k = e->streams[s].k;
  p.bb_v = e->streams[s].v;
  p.st = e->streams[s].st;
  p.codes = e->streams[s].codes;
  p.sp = to_dev(sp);
  for (int i = 0; i < len; ++i) {
    p.position = i;
    p.in_emb = static_cast<const bf16*>(embeds) + static_cast<size_t>(i) * qtt::HID;
    p.flags = (e->base.flags & qtt::FLAG_EAGER_REFILL) | ((i == len - 1) ? qtt::FLAG_HEAD_SAMPLE : 0);
    cudaError_t ce = qtt::launch(p, e->shape.ctas, e->shape.smem, stream);
    if (ce != cudaSuccess) return from_cuda(ce);
  }
  return QTT_OK;
}

extern "C" qtt_status qtt_frames(qtt_engine* e, int s, int n_frames, const void* trailing, int n_trailing,
                                 const void* pad, const qtt_sampling* sp, cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  if (n_frames < 0 || !pad || n_trailing < 0 || (n_trailing > 0 && !trailing)) return QTT_ERR_INVALID_ARG;
  qtt_status r = check_sampling(sp, e);
  if (r != QTT_OK) return r;
  r = set_device(e);
  if (r != QTT_OK) return r;
  qtt::Params p = e->base;
  p.mode = qtt::MODE_FRAME;
  p.bb_k = e->streams[s].k;
  p.bb_v = e->streams[s].v;
  p.st = e->streams[s].st;
  p.codes = e->streams[s].codes;
  p.trailing = static_cast<const bf16*>(trailing);
  p.n_trailing = n_trailing;
  p.pad = static_cast<const bf16*>(pad);
  p.sp = to_dev(sp);
  for (int i = 0; i < n_frames; ++i) {
    cudaError_t ce = qtt::launch(p, e->shape.ctas, e->shape.smem, stream);
    if (ce != cudaSuccess) return from_cuda(ce);
  }
  return QTT_OK;
}

// ------------------------------------------------------------------------------------------
// Batched decode
// ------------------------------------------------------------------------------------------
namespace {

constexpr size_t kCpKvFloats = static_cast<size_t>(qtt::NKVH) * kCpMaxSeq * qtt::HD;   // per layer

// Kernel attributes, scratch, per-utterance code-predictor KV and the tensor maps of every
// weight matrix, once per engine.
qtt_status ensure_batch(qtt_engine* e) {
  if (e->b_ready) return QTT_OK;
  cudaError_t ce = qtt::kernel_setup_b(e->device, &e->bshape.ctas, &e->bshape.smem, &e->bcl);
  if (ce == cudaErrorInvalidConfiguration) return QTT_ERR_UNSUPPORTED;   // too few clusters fit
  if (ce != cudaSuccess) return from_cuda(ce);
  const int nbb = e->dims.backbone_layers, ncp = e->dims.cp_layers;
  const int h0 = (nbb + ncp) * qtt::NLMAPS;
  const int nmaps = h0 + 1 + qtt::NCPHEADS + 4;
  std::vector<CUtensorMap> maps(nmaps);
  bool ok = true;
  // every stage splits its rows into R = 128 / cluster tiles: one box of a tile's N rows per
  // 64-column atom (gate/up: a box of N/2 gate rows and one of N/2 up rows)
  const uint32_t R = qtt::BROWS_B / e->bcl;
  auto layer_maps = [&](const TTSLayerWeights& L, CUtensorMap* m) {
    const uint32_t nq = qtt::QKV_ROWS / R, no = qtt::HID / R, ngu = 2 * qtt::INTER / R, nd = qtt::HID / R;
    ok = ok && encode_sw128(L.q_proj_weight, qtt::QSZ, qtt::HID, nq, m + 0);
    ok = ok && encode_sw128(L.k_proj_weight, qtt::KVSZ, qtt::HID, nq, m + 1);
    ok = ok && encode_sw128(L.v_proj_weight, qtt::KVSZ, qtt::HID, nq, m + 2);
    ok = ok && encode_sw128(L.o_proj_weight, qtt::HID, qtt::QSZ, no, m + 3);
    ok = ok && encode_sw128(L.gate_proj_weight, qtt::INTER, qtt::HID, ngu / 2, m + 4);
    ok = ok && encode_sw128(L.up_proj_weight, qtt::INTER, qtt::HID, ngu / 2, m + 5);
    ok = ok && encode_sw128(L.down_proj_weight, qtt::HID, qtt::INTER, nd, m + 6);
  };
  // the heads split into R full tiles whose row counts the M = 128 MMA takes (multiples of 16)
  if (e->dims.vocab % (16 * R) != 0 || e->dims.cp_vocab % (16 * R) != 0) return QTT_ERR_UNSUPPORTED;
  for (int l = 0; l < nbb; ++l) layer_maps(e->h_bb[l], maps.data() + l * qtt::NLMAPS);
  for (int l = 0; l < ncp; ++l) layer_maps(e->h_cp[l], maps.data() + (nbb + l) * qtt::NLMAPS);
  ok = ok && encode_sw128(e->h_codec_head, e->dims.vocab, qtt::HID, e->dims.vocab / R, &maps[h0]);
  for (int g = 0; g < qtt::NCPHEADS; ++g)
    ok = ok && encode_sw128(e->h_cp_head[g], e->dims.cp_vocab, qtt::HID, e->dims.cp_vocab / R, &maps[h0 + 1 + g]);
  if (!ok) return QTT_ERR_UNSUPPORTED;
  ce = cudaMalloc(&e->d_bwork, qtt::bwork_bytes());
  if (ce == cudaSuccess) ce = cudaMemset(e->d_bwork, 0, qtt::bwork_bytes());
  if (ce != cudaSuccess) return from_cuda(ce);
  qtt::BWork bw;
  qtt::bwork_carve(e->d_bwork, &bw);
  for (int b = 0; b < 2; ++b)
    if (!encode_sw128(bw.abuf[b], 2 * qtt::TBMAX, qtt::ABUF_LD, 64, &maps[h0 + 1 + qtt::NCPHEADS + 2 * b]) ||
        !encode_sw128(bw.abuf[b], 2 * qtt::TBMAX, qtt::ABUF_LD, 128, &maps[h0 + 1 + qtt::NCPHEADS + 2 * b + 1]))
      return QTT_ERR_UNSUPPORTED;
  ce = cudaMalloc(&e->d_bmaps, qtt::TMAP_BYTES * nmaps);
  if (ce == cudaSuccess) ce = cudaMemcpy(e->d_bmaps, maps.data(), qtt::TMAP_BYTES * nmaps, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMalloc(reinterpret_cast<void**>(&e->d_bs), sizeof(qtt::BStream) * e->max_streams);
  const size_t cpkv = 2 * kCpKvFloats * ncp * e->max_streams;
  if (ce == cudaSuccess) ce = cudaMalloc(reinterpret_cast<void**>(&e->d_cpkv), sizeof(float) * cpkv);
  if (ce == cudaSuccess) ce = cudaMemset(e->d_cpkv, 0, sizeof(float) * cpkv);
  std::vector<qtt::StreamState*> stp(e->max_streams);
  for (int s = 0; s < e->max_streams; ++s) stp[s] = e->streams[s].st;
  if (ce == cudaSuccess) ce = cudaMalloc(reinterpret_cast<void**>(&e->d_stptr), sizeof(void*) * e->max_streams);
  if (ce == cudaSuccess)
    ce = cudaMemcpy(e->d_stptr, stp.data(), sizeof(void*) * e->max_streams, cudaMemcpyHostToDevice);
  std::vector<int32_t*> cdp(e->max_streams);
  for (int s = 0; s < e->max_streams; ++s) cdp[s] = e->streams[s].codes;
  if (ce == cudaSuccess) ce = cudaMalloc(reinterpret_cast<void**>(&e->d_codeptr), sizeof(void*) * e->max_streams);
  if (ce == cudaSuccess)
    ce = cudaMemcpy(e->d_codeptr, cdp.data(), sizeof(void*) * e->max_streams, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMalloc(reinterpret_cast<void**>(&e->d_states), sizeof(int32_t) * 4 * e->max_streams);
  if (ce == cudaSuccess) ce = cudaMallocHost(reinterpret_cast<void**>(&e->h_states), sizeof(int32_t) * 4 * e->max_streams);
  if (ce != cudaSuccess) return from_cuda(ce);
  e->h_bs.assign(e->max_streams, qtt::BStream{});
  for (int s = 0; s < e->max_streams; ++s) {
    qtt::BStream& b = e->h_bs[s];
    b.k = e->streams[s].k;
    b.v = e->streams[s].v;
    b.cpk = e->d_cpkv + 2 * kCpKvFloats * ncp * s;
    b.cpv = b.cpk + kCpKvFloats * ncp;
    b.st = e->streams[s].st;
    b.codes = e->streams[s].codes;
  }
  e->b_ready = true;
  return QTT_OK;
}

qtt::Params batch_params(qtt_engine* e, int B, const qtt_sampling* sp) {
  qtt::Params p = e->base;
  p.bmaps = static_cast<const uint8_t*>(e->d_bmaps);
  p.nb = B;
  p.bcl = e->bcl;
  // a QKV row tile is one head (N = 128) with clusters of 4
  p.kv_pre = (e->bcl == 4 && !e->dbg_kv_in_attention) ? 1 : 0;
  p.bs = e->d_bs;
  qtt::bwork_carve(e->d_bwork, &p.bw);
  p.sp = to_dev(sp);
  p.bb_wd_map = nullptr;
  p.cp_wd_map = nullptr;
  p.dbg_cp_logits = e->b_dbg_cp;
  p.dbg_g0_logits = e->b_dbg_g0;
  p.dbg_skip_barrier = 0;   // the barrier-fault test hook applies to the batch-1 kernel only
  p.dbg_wait_ns = 0ull;
  return p;   // the stage timeline, profile marks and barrier arrivals, if set, are kept
}

// Draw stream and frame limit of engine stream s for a batched launch (qtt_set_stream_params).
void stream_params(const qtt_engine* e, int s, int default_philox, qtt::BStream& b) {
  const StreamBufs& sb = e->streams[s];
  b.philox = sb.philox >= 0 ? sb.philox : default_philox;
  b.frame_limit = sb.frame_limit < 0 ? 0 : (sb.frame_limit > 0 && sb.frame_limit < e->max_frames ? sb.frame_limit
                                                                                                  : e->max_frames);
}

__global__ void batch_states_kernel(qtt::StreamState* const* st, int B, int32_t* out) {
  for (int i = threadIdx.x; i < 4 * B; i += blockDim.x) {
    const qtt::StreamState* x = st[i >> 2];
    const int f = i & 3;
    out[i] = f == 0 ? x->position : f == 1 ? x->step : f == 2 ? x->g0 : x->done;
  }
}

qtt_status batch_check(qtt_engine* e, int B, const qtt_sampling* sp) {
  if (!e || B < 1 || B > e->max_streams || B > qtt::BMAX) return QTT_ERR_INVALID_ARG;
  qtt_status r = check_sampling(sp, e);
  if (r != QTT_OK) return r;
  r = set_device(e);
  if (r != QTT_OK) return r;
  return ensure_batch(e);
}

}  // namespace

extern "C" qtt_status qtt_batch_prefill(qtt_engine* e, int B, const void* const* embeds, const int* lens,
                                        const qtt_sampling* sp, cudaStream_t stream) {
  qtt_status r = batch_check(e, B, sp);
  if (r != QTT_OK) return r;
  if (!embeds || !lens) return QTT_ERR_INVALID_ARG;
  int maxlen = 0;
  for (int s = 0; s < B; ++s) {
    if (!embeds[s] || !aligned16(embeds[s]) || lens[s] < 1 || lens[s] >= e->max_seq || lens[s] > e->base.rope_rows)
      return QTT_ERR_INVALID_ARG;
    maxlen = lens[s] > maxlen ? lens[s] : maxlen;
  }
  for (int s = 0; s < B; ++s) {
    r = qtt_reset(e, s, stream);
    if (r != QTT_OK) return r;
    qtt::BStream& b = e->h_bs[s];
    b.trailing = nullptr;
    b.n_trailing = 0;
    b.pad = nullptr;
    b.len = lens[s];
    b.emb = static_cast<const bf16*>(embeds[s]);
    stream_params(e, s, sp->philox_stream + s, b);
  }
  // pageable source: the copy is staged before the call returns
  cudaError_t ce = cudaMemcpyAsync(e->d_bs, e->h_bs.data(), sizeof(qtt::BStream) * B, cudaMemcpyHostToDevice, stream);
  if (ce != cudaSuccess) return from_cuda(ce);
  qtt::Params p = batch_params(e, B, sp);
  p.mode = qtt::MODE_B_PREFILL;
  for (int i = 0; i < maxlen; ++i) {
    p.b_step = i;
    ce = qtt::launch_b(p, e->bshape.ctas, e->bshape.smem, stream);
    if (ce != cudaSuccess) return from_cuda(ce);
  }
  p.mode = qtt::MODE_B_HEAD;
  return from_cuda(qtt::launch_b(p, e->bshape.ctas, e->bshape.smem, stream));
}

extern "C" qtt_status qtt_prefill_tc(qtt_engine* e, int s, const void* embeds, int len, const qtt_sampling* sp,
                                     cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  if (!embeds || !aligned16(embeds) || len < 1 || len >= e->max_seq || len > e->base.rope_rows)
    return QTT_ERR_INVALID_ARG;
  qtt_status r = batch_check(e, 1, sp);
  if (r != QTT_OK) return r;
  r = qtt_reset(e, s, stream);
  if (r != QTT_OK) return r;
  // the launch's utterance 0 is stream s
  qtt::BStream b = e->h_bs[s];
  b.trailing = nullptr;
  b.n_trailing = 0;
  b.pad = nullptr;
  b.len = len;
  b.emb = static_cast<const bf16*>(embeds);
  stream_params(e, s, sp->philox_stream, b);
  // pageable source: the copy is staged before the call returns
  cudaError_t ce = cudaMemcpyAsync(e->d_bs, &b, sizeof(qtt::BStream), cudaMemcpyHostToDevice, stream);
  if (ce != cudaSuccess) return from_cuda(ce);
  qtt::Params p = batch_params(e, 1, sp);
  p.mode = qtt::MODE_B_PREFILL_DENSE;
  for (int p0 = 0; p0 < len; p0 += qtt::TBMAX) {
    p.b_step = p0;
    p.b_ntok = len - p0 < qtt::TBMAX ? len - p0 : qtt::TBMAX;
    ce = qtt::launch_b(p, e->bshape.ctas, e->bshape.smem, stream);
    if (ce != cudaSuccess) return from_cuda(ce);
  }
  p.mode = qtt::MODE_B_HEAD;
  return from_cuda(qtt::launch_b(p, e->bshape.ctas, e->bshape.smem, stream));
}

extern "C" qtt_status qtt_batch_frames(qtt_engine* e, int B, int n_frames, const void* const* trailing,
                                       const int* n_trailing, const void* const* pad, const qtt_sampling* sp,
                                       cudaStream_t stream) {
  qtt_status r = batch_check(e, B, sp);
  if (r != QTT_OK) return r;
  if (n_frames < 0 || !pad || !n_trailing) return QTT_ERR_INVALID_ARG;
  for (int s = 0; s < B; ++s)
    if (!pad[s] || n_trailing[s] < 0 || (n_trailing[s] > 0 && (!trailing || !trailing[s]))) return QTT_ERR_INVALID_ARG;
  for (int s = 0; s < B; ++s) {
    qtt::BStream& b = e->h_bs[s];
    b.trailing = n_trailing[s] > 0 ? static_cast<const bf16*>(trailing[s]) : nullptr;
    b.n_trailing = n_trailing[s];
    b.pad = static_cast<const bf16*>(pad[s]);
    b.emb = nullptr;
    b.len = 0;
    stream_params(e, s, sp->philox_stream + s, b);
  }
  cudaError_t ce = cudaMemcpyAsync(e->d_bs, e->h_bs.data(), sizeof(qtt::BStream) * B, cudaMemcpyHostToDevice, stream);
  if (ce != cudaSuccess) return from_cuda(ce);
  qtt::Params p = batch_params(e, B, sp);
  p.mode = qtt::MODE_B_FRAME;
  for (int i = 0; i < n_frames; ++i) {
    ce = qtt::launch_b(p, e->bshape.ctas, e->bshape.smem, stream);
    if (ce != cudaSuccess) return from_cuda(ce);
  }
  return QTT_OK;
}

extern "C" qtt_status qtt_set_stream_params(qtt_engine* e, int s, int philox_stream, int frame_limit) {
  QTT_STREAM_CHECK(e, s);
  if (philox_stream < -1) return QTT_ERR_INVALID_ARG;
  e->streams[s].philox = philox_stream;
  e->streams[s].frame_limit = frame_limit;
  return QTT_OK;
}

extern "C" qtt_status qtt_batch_states(qtt_engine* e, int B, int32_t* out, cudaStream_t stream) {
  if (!e || !out || B < 1 || B > e->max_streams) return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  r = ensure_batch(e);
  if (r != QTT_OK) return r;
  batch_states_kernel<<<1, 256, 0, stream>>>(e->d_stptr, B, e->d_states);
  cudaError_t ce = cudaGetLastError();
  if (ce == cudaSuccess)
    ce = cudaMemcpyAsync(e->h_states, e->d_states, sizeof(int32_t) * 4 * B, cudaMemcpyDeviceToHost, stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(stream);
  if (ce != cudaSuccess) return from_cuda(ce);
  std::memcpy(out, e->h_states, sizeof(int32_t) * 4 * B);
  return QTT_OK;
}

// Row s of out: the 16 codes of stream s's latest frame (frame step - 1), or -1 without one.
__global__ void batch_last_codes_kernel(qtt::StreamState* const* st, int32_t* const* codes, int B, int32_t* out) {
  for (int i = threadIdx.x; i < qtt::NGROUPS * B; i += blockDim.x) {
    const int s = i / qtt::NGROUPS, g = i - s * qtt::NGROUPS;
    const int step = st[s]->step;
    out[i] = step > 0 ? codes[s][(step - 1) * qtt::NGROUPS + g] : -1;
  }
}

extern "C" qtt_status qtt_batch_last_codes(qtt_engine* e, int B, int32_t* out, cudaStream_t stream) {
  if (!e || !out || B < 1 || B > e->max_streams) return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  r = ensure_batch(e);
  if (r != QTT_OK) return r;
  batch_last_codes_kernel<<<1, 256, 0, stream>>>(e->d_stptr, e->d_codeptr, B, out);
  return from_cuda(cudaGetLastError());
}

extern "C" qtt_status qtt_batch_set_debug_outputs(qtt_engine* e, float* cp_logits, float* g0_logits) {
  if (!e) return QTT_ERR_INVALID_ARG;
  e->b_dbg_cp = cp_logits;
  e->b_dbg_g0 = g0_logits;
  return QTT_OK;
}

extern "C" qtt_status qtt_batch_debug_buffers(qtt_engine* e, void** ptrs, int n) {
  if (!e || !ptrs || n < 1) return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  r = ensure_batch(e);
  if (r != QTT_OK) return r;
  qtt::BWork bw;
  qtt::bwork_carve(e->d_bwork, &bw);
  void* all[9] = {bw.abuf[0], bw.abuf[1], bw.logits, bw.tok, bw.x, bw.hb[0], bw.hb[1], bw.hmid, bw.qkv};
  for (int i = 0; i < n && i < 9; ++i) ptrs[i] = all[i];
  return QTT_OK;
}

extern "C" qtt_status qtt_codes_ptr(qtt_engine* e, int s, int32_t** codes) {
  QTT_STREAM_CHECK(e, s);
  if (!codes) return QTT_ERR_INVALID_ARG;
  *codes = e->streams[s].codes;
  return QTT_OK;
}

extern "C" qtt_status qtt_cp_step(qtt_engine* e, const void* emb, int position, float* out_hidden,
                                  cudaStream_t stream) {
  if (!e || !emb || !aligned16(emb) || position < 0 || position >= kCpMaxSeq || position >= e->base.rope_rows)
    return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  qtt::Params p = e->base;
  p.mode = qtt::MODE_CP_STEP;
  p.position = position;
  p.in_emb = static_cast<const bf16*>(emb);
  p.out_hidden = out_hidden;
  return from_cuda(qtt::launch(p, e->shape.ctas, e->shape.smem, stream));
}

namespace {
__global__ void set_decode_state_kernel(qtt::StreamState* st, const float* h, int g0, int position) {
  for (int i = threadIdx.x; i < qtt::HID; i += blockDim.x) st->h[i] = h[i];
  for (int i = threadIdx.x; i < qtt::VMAX; i += blockDim.x) st->seen[i] = 0;
  if (threadIdx.x == 0) {
    st->position = position;
    st->step = 0;
    st->g0 = g0;
    st->done = 0;
  }
}
__global__ void get_hidden_kernel(const qtt::StreamState* st, float* out) {
  for (int i = threadIdx.x; i < qtt::HID; i += blockDim.x) out[i] = st->h[i];
}
}  // namespace

extern "C" qtt_status qtt_set_decode_state(qtt_engine* e, int s, const float* h, int g0, int position,
                                           cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  if (!h || g0 < 0 || g0 >= e->dims.vocab || position < 0 || position >= e->max_seq) return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  set_decode_state_kernel<<<1, 256, 0, stream>>>(e->streams[s].st, h, g0, position);
  return from_cuda(cudaGetLastError());
}

extern "C" qtt_status qtt_get_hidden(qtt_engine* e, int s, float* out, cudaStream_t stream) {
  QTT_STREAM_CHECK(e, s);
  if (!out) return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  get_hidden_kernel<<<1, 256, 0, stream>>>(e->streams[s].st, out);
  return from_cuda(cudaGetLastError());
}

extern "C" qtt_status qtt_set_debug_outputs(qtt_engine* e, float* cp_logits, float* g0_logits) {
  if (!e) return QTT_ERR_INVALID_ARG;
  e->base.dbg_cp_logits = cp_logits;
  e->base.dbg_g0_logits = g0_logits;
  return QTT_OK;
}

extern "C" qtt_status qtt_set_debug_timeline(qtt_engine* e, unsigned long long* stamps, int n) {
  if (!e || n < 0 || (n > 0 && !stamps)) return QTT_ERR_INVALID_ARG;
  e->base.dbg_timeline = n > 0 ? stamps : nullptr;
  e->base.dbg_timeline_len = n;
  return QTT_OK;
}

extern "C" qtt_status qtt_set_debug_profile(qtt_engine* e, unsigned long long* marks, int n_marks,
                                            unsigned long long* arrivals, int arrival_stage0, int arrival_stages) {
  if (!e || n_marks < 0 || arrival_stages < 0) return QTT_ERR_INVALID_ARG;
  e->base.dbg_marks = n_marks > 0 ? marks : nullptr;
  e->base.dbg_marks_len = n_marks;
  e->base.dbg_arrivals = arrival_stages > 0 ? arrivals : nullptr;
  e->base.dbg_arr_stage0 = arrival_stage0;
  e->base.dbg_arr_n = arrival_stages;
  return QTT_OK;
}

extern "C" qtt_status qtt_set_debug_barrier_fault(qtt_engine* e, int barrier, unsigned long long wait_ns) {
  if (!e || barrier < 0) return QTT_ERR_INVALID_ARG;
  e->base.dbg_skip_barrier = barrier;
  e->base.dbg_wait_ns = wait_ns;
  return QTT_OK;
}

extern "C" qtt_status qtt_set_debug_kv_in_attention(qtt_engine* e, int on) {
  if (!e) return QTT_ERR_INVALID_ARG;
  e->dbg_kv_in_attention = on ? 1 : 0;
  return QTT_OK;
}

extern "C" qtt_status qtt_set_refill_policy(qtt_engine* e, int eager) {
  if (!e) return QTT_ERR_INVALID_ARG;
  e->base.flags = eager ? (e->base.flags | qtt::FLAG_EAGER_REFILL) : (e->base.flags & ~qtt::FLAG_EAGER_REFILL);
  return QTT_OK;
}

extern "C" qtt_status qtt_check(qtt_engine* e, cudaStream_t stream) {
  if (!e) return QTT_ERR_INVALID_ARG;
  qtt_status r = set_device(e);
  if (r != QTT_OK) return r;
  cudaError_t ce = cudaStreamSynchronize(stream);
  if (ce != cudaSuccess) return from_cuda(ce);
  int code = 0;
  ce = cudaMemcpy(&code, e->base.w.err, sizeof(int), cudaMemcpyDeviceToHost);
  if (ce != cudaSuccess) return from_cuda(ce);
  if (code != 0) {
    const int zero = 0;
    cudaMemcpy(e->base.w.err, &zero, sizeof(int), cudaMemcpyHostToDevice);
  }
  return from_dev(code);
}
