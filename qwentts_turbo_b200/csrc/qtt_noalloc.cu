// Backbone decode step that allocates no device memory (qtt_backbone_step_noalloc).
//
// Who needs it: callers that must not allocate device memory while decoding - a speech
// service that reserves its whole device memory budget at start-up and treats any later
// allocation as a failure (a cudaMalloc in the middle of streaming audio can stall or run out
// of memory), or a host framework whose caching allocator owns the device memory so that a
// library-side cudaMalloc would bypass and fragment it. The drop-in launcher
// launch_tts_decode_with_embedding allocates its scratch with cudaMalloc on the first call on
// each (device, stream); this entry point never allocates.
//
// Where the scratch lives: a file-scope __device__ array (below) of kNoAllocScratchBytes. The
// array is part of the library's device image, so every GPU that loads libqtt.so holds it
// until the process exits. Under lazy module loading (CUDA_MODULE_LOADING=LAZY, the default
// since CUDA 12.2) the driver places the array in device memory only when it is first used:
// the first call on each device, which takes its address. That first call is therefore a
// one-time driver allocation; make it at start-up (a warm-up step) and before any stream
// capture. In host code the array's name is only a host-side stand-in, never a device
// address: the device address comes from cudaGetSymbolAddress, taken once per device on the
// first call with that device current, and is passed to the kernel.
//
// Sharing: every call on a device uses the same array, which keeps the last call's contents.
// The barrier counter, the error word and the attention combine counters are cleared before
// every launch. Calls whose executions overlap on the GPU (different streams, no ordering
// between them) race on the array; order them on one stream. The return value covers the
// argument checks and the launch; a device-side error of the step (a bounded wait that timed
// out) is kept in the array's error word and returned, then cleared, by qtt_stream_check().
#include <cstring>
#include <map>
#include <mutex>

#include "../../include/qtt.h"
#include "qtt_device.cuh"
#include "qtt_kernel.cuh"

namespace {

// Same layout as qtt::work_carve (barrier / error / combine counters, per-token activations
// for up to NTMAX tokens, MAX_ATT_CHUNKS attention partial records per query head, and the
// fixed-point layer outputs of the fused MLP stage).
constexpr size_t kNoAllocScratchBytes =
    256 + sizeof(float) * (2 * qtt::NTMAX * qtt::HID + qtt::NTMAX * qtt::QKV_ROWS + qtt::NTMAX * qtt::QSZ +
                           qtt::NTMAX * qtt::NQH * qtt::MAX_ATT_CHUNKS * qtt::PRT_STRIDE + qtt::NTMAX * qtt::HID +
                           qtt::NTMAX * qtt::INTER + qtt::VMAX) +
    sizeof(long long) * qtt::NHACC * qtt::NTMAX * qtt::HID;

// Largest cache length one step supports: at most (CTAs / 8) attention work items per KV head,
// each over at most ATT_CHMAX positions, and never more than the scratch's MAX_ATT_CHUNKS
// partial records per head.
constexpr int kNoAllocMaxSeq = qtt::MAX_ATT_CHUNKS * qtt::ATT_CHMAX;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct DeviceSetup {
  void* scratch = nullptr;
  int ctas = 0;
  size_t smem = 0;
};
std::mutex g_mu;
std::map<int, DeviceSetup> g_setup;

// Once per device, with that device current: kernel attributes and the scratch's device address.
qtt_status device_setup(int dev, DeviceSetup* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_setup.find(dev);
  if (it != g_setup.end()) {
    *out = it->second;
    return QTT_OK;
  }
  DeviceSetup s;
  if (qtt::kernel_setup(dev, &s.ctas, &s.smem) != cudaSuccess) return QTT_ERR_CUDA;
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return QTT_ERR_CUDA;
  s.scratch = ptr;
  g_setup[dev] = s;
  *out = s;
  return QTT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace qtt {
// Device error code left in the fixed scratch by the last no-alloc step on `dev` (0 when the
// path was never used there), then cleared. The caller has synchronised the step's stream.
// Copies to and from a __device__ symbol allocate nothing.
cudaError_t noalloc_take_error(int dev, int* code) {
  *code = 0;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_setup.find(dev);
    if (it == g_setup.end()) return cudaSuccess;
    scratch = it->second.scratch;
  }
  Work w;
  work_carve(scratch, &w);
  const size_t off = static_cast<size_t>(reinterpret_cast<char*>(w.err) - static_cast<char*>(scratch));
  cudaError_t e = cudaMemcpyFromSymbol(code, g_noalloc_scratch, sizeof(int), off, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess || *code == 0) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof(int), off, cudaMemcpyHostToDevice);
}
}  // namespace qtt

extern "C" qtt_status qtt_backbone_step_noalloc(const void* input_embedding, const TTSLayerWeights* layer_weights,
                                                const void* final_norm_weight, const void* cos_table,
                                                const void* sin_table, void* k_cache, void* v_cache,
                                                void* hidden_buffer, void* g_normalized, int num_layers,
                                                int position, int max_seq_len, float attn_scale,
                                                cudaStream_t stream) {
  if (!input_embedding || !layer_weights || !final_norm_weight || !cos_table || !sin_table || !k_cache ||
      !v_cache || !g_normalized || num_layers < 1 || max_seq_len < 1 || position < 0 || position >= max_seq_len ||
      !aligned16(input_embedding) || !aligned16(k_cache) || !aligned16(v_cache))
    return QTT_ERR_INVALID_ARG;
  if (max_seq_len > kNoAllocMaxSeq) return QTT_ERR_UNSUPPORTED;   // beyond the scratch's capacity
  if (qtt::work_bytes() > kNoAllocScratchBytes) return QTT_ERR_UNSUPPORTED;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QTT_ERR_CUDA;
  DeviceSetup ds;
  qtt_status st = device_setup(dev, &ds);
  if (st != QTT_OK) return st;
  // the persistent kernel's per-stage weight shares assume at least 128 CTAs (one per SM)
  if (ds.ctas < 128 || max_seq_len > (ds.ctas / qtt::NKVH) * qtt::ATT_CHMAX) return QTT_ERR_UNSUPPORTED;
  qtt::Params p;
  std::memset(&p, 0, sizeof(p));
  qtt::work_carve(ds.scratch, &p.w);
  // The array keeps the previous call's contents: clear the error word and the attention
  // combine counters (the barrier counter is cleared by qtt::launch).
  if (cudaMemsetAsync(p.w.err, 0, sizeof(int), stream) != cudaSuccess) return QTT_ERR_CUDA;
  if (cudaMemsetAsync(p.w.att_cnt, 0, sizeof(uint32_t) * qtt::NKVH, stream) != cudaSuccess) return QTT_ERR_CUDA;
  p.bb_layers = reinterpret_cast<const qtt::LayerW*>(layer_weights);
  p.n_bb = num_layers;
  p.bb_norm = static_cast<const qtt::bf16*>(final_norm_weight);
  p.bb_k = static_cast<qtt::bf16*>(k_cache);
  p.bb_v = static_cast<qtt::bf16*>(v_cache);
  p.bb_max_seq = max_seq_len;
  p.out_raw_hidden = static_cast<qtt::bf16*>(hidden_buffer);
  p.mode = qtt::MODE_BB_STEP;
  p.cos_tab = static_cast<const qtt::bf16*>(cos_table);
  p.sin_tab = static_cast<const qtt::bf16*>(sin_table);
  p.rope_rows = max_seq_len;
  p.attn_scale = attn_scale;
  p.eps = 1e-6f;
  p.position = position;
  p.in_emb = static_cast<const qtt::bf16*>(input_embedding);
  p.out_hidden = static_cast<float*>(g_normalized);
  return qtt::launch(p, ds.ctas, ds.smem, stream) == cudaSuccess ? QTT_OK : QTT_ERR_CUDA;
}
