/*
 * qtt.h - C ABI of the B200 (sm_100a) Qwen3-TTS decode engine (libqtt.so).
 *
 * Two layers of entry points:
 *
 * 1. Drop-in launchers with the exact names, arguments and void return of the reference's
 *    extern "C" functions (hamza1brh/qwenTTS-turbo, qwentts_turbo/csrc/). A binding that
 *    compiled the reference .cu files can link this library instead, unchanged. They run
 *    the sm_100a persistent kernel on the caller's weights, caches and stream. Because the
 *    reference returns void, the status of the calling thread's last launch is available
 *    from qtt_last_launch_status().
 *
 * 2. The engine API (qtt_engine_*): owns per-utterance KV caches and device-side decode
 *    state so that whole frames (code-predictor chain + combine + backbone step + sampling)
 *    run back to back on the device with no host round trip. Every call returns qtt_status.
 *
 * All pointers passed to the library are DEVICE pointers unless stated otherwise. Weight
 * matrices are row-major bf16 [out_features, in_features], 16-byte aligned.
 */
#ifndef QTT_H_
#define QTT_H_

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------
 * Reference weight-pointer structs. Same member order and layout as
 * TTSLayerWeights (fused_decode_tts.cu:22-34) and CPLayerWeights
 * (fused_decode_code_predictor.cu:30-42).
 * ---------------------------------------------------------------------------------------- */
typedef struct TTSLayerWeights {
  const void* input_layernorm_weight;
  const void* q_proj_weight;
  const void* k_proj_weight;
  const void* v_proj_weight;
  const void* q_norm_weight;
  const void* k_norm_weight;
  const void* o_proj_weight;
  const void* post_attn_layernorm_weight;
  const void* gate_proj_weight;
  const void* up_proj_weight;
  const void* down_proj_weight;
} TTSLayerWeights;

typedef TTSLayerWeights CPLayerWeights;

/* ------------------------------------------------------------------------------------------
 * 1. Drop-in launchers
 * ---------------------------------------------------------------------------------------- */

/* Replaces launch_tts_decode_with_embedding (fused_decode_tts.cu:834-890).
 * One 28-layer backbone decode step of a bf16 embedding [1024] at `position`.
 * layer_weights: DEVICE array of num_layers structs. k_cache/v_cache: bf16
 * [num_layers][8][max_seq_len][128]; the step writes row `position` and attends over
 * [0, cache_len), cache_len must equal position + 1. Outputs: g_normalized fp32 [1024]
 * (final RMSNorm), hidden_buffer bf16 [1024] (last layer output). The remaining g_* scratch
 * arguments are accepted for ABI compatibility and not used; the library keeps its own
 * scratch per (device, stream), allocated on the first call on that stream. */
void launch_tts_decode_with_embedding(const void* input_embedding, const TTSLayerWeights* layer_weights,
                                      const void* final_norm_weight, const void* cos_table,
                                      const void* sin_table, void* k_cache, void* v_cache,
                                      void* hidden_buffer, void* g_activations, void* g_residual, void* g_q,
                                      void* g_k, void* g_v, void* g_attn_out, void* g_mlp_intermediate,
                                      void* g_normalized, int num_layers, int position, int cache_len,
                                      int max_seq_len, float attn_scale, cudaStream_t stream);

/* Replaces launch_tts_decode (fused_decode_tts.cu:664-722): the same step with the input
 * taken from row input_token_id of embed_weight [vocab][1024]. */
void launch_tts_decode(int input_token_id, const void* embed_weight, const TTSLayerWeights* layer_weights,
                       const void* final_norm_weight, const void* cos_table, const void* sin_table,
                       void* k_cache, void* v_cache, void* hidden_buffer, void* g_activations,
                       void* g_residual, void* g_q, void* g_k, void* g_v, void* g_attn_out,
                       void* g_mlp_intermediate, void* g_normalized, int num_layers, int position,
                       int cache_len, int max_seq_len, float attn_scale, cudaStream_t stream);

/* Replaces launch_cp_decode_with_embedding (fused_decode_code_predictor.cu:674-730).
 * One code-predictor decode step: bf16 input [1024], fp32 hidden state between layers,
 * fp32 k_cache/v_cache [num_layers][8][max_seq_len][128]. Output g_normalized fp32 [1024]. */
void launch_cp_decode_with_embedding(const void* input_embedding, const CPLayerWeights* layer_weights,
                                     const void* final_norm_weight, const void* cos_table, const void* sin_table,
                                     void* k_cache, void* v_cache, void* hidden_buffer, void* g_activations,
                                     void* g_residual, void* g_q, void* g_k, void* g_v, void* g_attn_out,
                                     void* g_mlp_intermediate, void* g_normalized, int num_layers,
                                     int position, int cache_len, int max_seq_len, float attn_scale,
                                     cudaStream_t stream);

/* Status (qtt_status) of the calling thread's last drop-in launch: argument checks and the
 * launch itself. Device-side errors (timeouts) are reported by qtt_stream_check(). */
int qtt_last_launch_status(void);

/* Identifies the sources the library was built from: 16 hex digits of a SHA-256 over
 * csrc/*.cu, csrc/*.cuh and this header, stamped at build time (no counterpart in the
 * reference). A host can compare it with the hash of the sources it ships. */
const char* qtt_build_id(void);

/* Synchronises `stream` and returns the device error recorded by drop-in launches on it and by
 * qtt_backbone_step_noalloc on the current device (then clears them). */
int qtt_stream_check(cudaStream_t stream);

/* ------------------------------------------------------------------------------------------
 * 2. Engine API
 * ---------------------------------------------------------------------------------------- */
typedef enum qtt_status {
  QTT_OK = 0,
  QTT_ERR_INVALID_ARG = 1,
  QTT_ERR_CUDA = 2,
  QTT_ERR_OOM = 3,
  QTT_ERR_TIMEOUT = 4,      /* a bounded device wait expired; the launch was abandoned */
  QTT_ERR_UNSUPPORTED = 5,  /* shape or option this build does not implement */
  QTT_ERR_BAD_TOKEN = 6,
  QTT_ERR_BAD_POSITION = 7,
  QTT_ERR_DEVICE = 8
} qtt_status;

/* No counterpart in the reference. The backbone decode step of
 * launch_tts_decode_with_embedding for callers that must not allocate device memory while
 * decoding (a service that reserves its whole memory budget at start-up, or a host whose caching
 * allocator owns the device memory): the scratch lives in a fixed 684 KB device array inside the
 * library instead of a per-stream cudaMalloc. Same arguments as the drop-in launcher minus the
 * unused g_* scratch pointers and cache_len (= position + 1). The first call on a device takes
 * the array's device address (cudaGetSymbolAddress) with that device current; with lazy module
 * loading (the CUDA default) that is also when the driver places the array in device memory, a
 * one-time allocation: make the first call at start-up as a warm-up, before any stream capture.
 * Calls share the array: calls that overlap on the GPU race, so keep them on one stream.
 * max_seq_len above 8192 (or above what the device's CTA count supports), or a GPU with fewer
 * than 128 SMs, returns QTT_ERR_UNSUPPORTED. Returns the status of the argument checks and the
 * launch; a device-side error of the step (a bounded wait that timed out) is returned by
 * qtt_stream_check(stream). */
qtt_status qtt_backbone_step_noalloc(const void* input_embedding, const TTSLayerWeights* layer_weights,
                                     const void* final_norm_weight, const void* cos_table,
                                     const void* sin_table, void* k_cache, void* v_cache, void* hidden_buffer,
                                     void* g_normalized, int num_layers, int position, int max_seq_len,
                                     float attn_scale, cudaStream_t stream);

typedef struct qtt_engine qtt_engine;

/* Model shape; must equal the compiled-in Qwen3-TTS-12Hz-0.6B shape
 * (config.cuh:33-40 of the reference). */
typedef struct qtt_dims {
  int hidden;           /* 1024 */
  int intermediate;     /* 3072 */
  int n_q_heads;        /* 16 */
  int n_kv_heads;       /* 8 */
  int head_dim;         /* 128 */
  int vocab;            /* 3072 */
  int cp_vocab;         /* 2048 */
  int n_groups;         /* 16 */
  int backbone_layers;  /* 28 (any >= 1 accepted) */
  int cp_layers;        /* 5 (any >= 1 accepted) */
  float rms_eps;        /* 1e-6 */
  float attn_scale;     /* 1/sqrt(head_dim) */
} qtt_dims;

/* Device pointers of all weights. The engine borrows them (no copy): keep them alive and
 * unchanged until qtt_engine_destroy. Layer arrays are HOST arrays of structs. */
typedef struct qtt_weights {
  const TTSLayerWeights* backbone_layers;  /* [backbone_layers] */
  const void* backbone_norm;               /* [1024] */
  const void* codec_embedding;             /* [vocab][1024] */
  const void* codec_head;                  /* [vocab][1024] */
  const CPLayerWeights* cp_layers;         /* [cp_layers] */
  const void* cp_norm;                     /* [1024] */
  const void* cp_codec_embedding[15];      /* [cp_vocab][1024] each */
  const void* cp_lm_head[15];              /* [cp_vocab][1024] each */
  const void* rope_cos;                    /* bf16 [rope_rows][128] */
  const void* rope_sin;                    /* bf16 [rope_rows][128] */
  int rope_rows;
} qtt_weights;

/* Sampling options of NativeTTSGenerator.generate (generator.py:77-81). Draws are
 * Philox4x32-10 keyed by `seed`, counter (frame, group, philox_stream, 0). top_p < 1 applies the
 * nucleus filter to group 0 after top-k (generator.py:196-203; the code predictor samples with
 * top_p = 1 as in generator.py:332,352); NaN or negative top_p is an invalid argument. */
typedef struct qtt_sampling {
  int do_sample;
  float temperature;
  int top_k;
  float top_p;
  int cp_do_sample;
  float cp_temperature;
  int cp_top_k;
  int min_new_tokens;
  float repetition_penalty;
  int eos_token_id;
  int philox_stream;
  uint64_t seed;
} qtt_sampling;

const char* qtt_status_string(qtt_status s);

/* Creates an engine on `device` for up to max_streams independent utterances, each with a
 * backbone KV cache of max_seq positions and a code buffer of max_frames frames. */
qtt_status qtt_engine_create(const qtt_weights* w, const qtt_dims* d, int device, int max_streams, int max_seq,
                             int max_frames, qtt_engine** out);
qtt_status qtt_engine_destroy(qtt_engine* e);
/* Number of CTAs of the persistent kernel (one per SM). */
int qtt_engine_num_ctas(const qtt_engine* e);

/* Zero the stream's KV cache and decode state (MegakernelTTSDecoder::reset,
 * megakernel_backbone.py:269-273). */
qtt_status qtt_reset(qtt_engine* e, int s, cudaStream_t stream);
/* Copy k/v [backbone_layers][8][len][128] (dtype 0 = bf16, 1 = fp32, cast to bf16) into
 * positions [0, len) of the cache (set_kv_cache, megakernel_backbone.py:285-294). */
qtt_status qtt_set_kv(qtt_engine* e, int s, const void* k, const void* v, int len, int dtype, cudaStream_t stream);
/* Device pointers of the stream's bf16 caches [L][8][max_seq][128] (get_k_cache/get_v_cache). */
qtt_status qtt_get_kv(qtt_engine* e, int s, void** k, void** v, int* max_seq);
qtt_status qtt_set_position(qtt_engine* e, int s, int position, cudaStream_t stream);
/* Reads the device state (synchronises `stream`). Any pointer may be NULL. */
qtt_status qtt_get_state(qtt_engine* e, int s, int* position, int* frames, int* g0, int* done, cudaStream_t stream);

/* One backbone decode step of emb [1024] bf16 at `position` (decode_step_with_embedding,
 * megakernel_backbone.py:230-267). out_hidden: fp32 [1024] final-normed, may be NULL. */
qtt_status qtt_backbone_step(qtt_engine* e, int s, const void* emb, int position, float* out_hidden,
                             cudaStream_t stream);
/* Context prefill: resets the stream, runs the backbone over embeds [len][1024] bf16 and
 * samples the first group-0 token (generator.py:104-120). */
qtt_status qtt_prefill(qtt_engine* e, int s, const void* embeds, int len, const qtt_sampling* sp,
                       cudaStream_t stream);
/* n_frames iterations of the frame loop (generator.py:125-174) on the device: the frame
 * uses trailing row `frame` while frame < n_trailing, else pad. Codes land in the stream's
 * code buffer [max_frames][16]; frames after EOS are no-ops. */
qtt_status qtt_frames(qtt_engine* e, int s, int n_frames, const void* trailing, int n_trailing, const void* pad,
                      const qtt_sampling* sp, cudaStream_t stream);
/* KV handoff (generator.py:245-257 + 115-120): after qtt_set_kv, start decoding at
 * `position` from the final-normed hidden h (fp32 [1024], device) with group-0 token g0.
 * Clears the frame counter, the EOS flag and the repetition history. */
qtt_status qtt_set_decode_state(qtt_engine* e, int s, const float* h, int g0, int position, cudaStream_t stream);
/* Copies the stream's last final-normed backbone hidden (fp32 [1024]) to `out` (device). */
qtt_status qtt_get_hidden(qtt_engine* e, int s, float* out, cudaStream_t stream);
/* Device pointer of the stream's code buffer int32 [max_frames][16]. */
qtt_status qtt_codes_ptr(qtt_engine* e, int s, int32_t** codes);

/* Tensor-core prefill of utterance s: the same result as qtt_prefill (KV cache rows of the
 * context, decode state h, first group-0 token; the stream's state reset first), but the context
 * is processed in chunks of up to 128 positions per launch, every projection a dense tcgen05 GEMM
 * over the chunk and a causal attention per position. Replaces the reference's PyTorch prefill and
 * KV handoff (generator.py:209-225,245-257); qtt_prefill is the token-by-token
 * counterpart of the reference's megakernel loop. Needs the batched path's conditions (see
 * qtt_batch_prefill). */
qtt_status qtt_prefill_tc(qtt_engine* e, int s, const void* embeds, int len, const qtt_sampling* sampling,
                          cudaStream_t stream);

/* Batched decode (no counterpart in the reference, which decodes one utterance at a time:
 * generator.py:77-176 is the per-utterance loop these replace for B utterances). Streams
 * 0..B-1 of the engine (B <= 64 and <= max_streams) advance together: every launch streams the
 * weights once for the whole batch and runs the projections on tcgen05 tensor cores.
 * qtt_batch_prefill: resets the streams, decodes each utterance's context (embeds[s]: device
 * bf16 [lens[s]][1024]) and samples its first group-0 token (as qtt_prefill per stream).
 * qtt_batch_frames: n_frames frames of every stream that has not reached EOS (as qtt_frames per
 * stream; trailing[s] device bf16 [n_trailing[s]][1024] or NULL when n_trailing[s] == 0,
 * pad[s] device bf16 [1024]). Sampling draws of stream s use Philox stream sp->philox_stream + s
 * unless qtt_set_stream_params gave the stream its own.
 * The pointer and length arrays are host arrays of B entries. */
qtt_status qtt_batch_prefill(qtt_engine* e, int B, const void* const* embeds, const int* lens,
                             const qtt_sampling* sp, cudaStream_t stream);
qtt_status qtt_batch_frames(qtt_engine* e, int B, int n_frames, const void* const* trailing, const int* n_trailing,
                            const void* const* pad, const qtt_sampling* sp, cudaStream_t stream);
/* Continuous batching (no counterpart in the reference, whose generate() call takes one
 * utterance, its max_new_tokens and torch's global generator: generator.py:77-127). Settings of
 * stream s for the batched launches and qtt_prefill_tc that follow, kept across resets:
 * philox_stream >= 0 is the Philox stream of all the stream's draws (-1: the default above, and
 * sp->philox_stream in qtt_prefill_tc), so an utterance's codes do not depend on the stream it
 * runs in; frame_limit > 0 stops the stream after that many frames (as max_new_tokens),
 * 0 = max_frames, < 0 parks it (no frames until set again). */
qtt_status qtt_set_stream_params(qtt_engine* e, int s, int philox_stream, int frame_limit);
/* States of streams 0..B-1 with one device->host copy: out[4 * s + 0..3] = position, frames,
 * group-0 token of the next frame, done (EOS reached). Host array of 4 * B ints; synchronizes
 * `stream`. */
qtt_status qtt_batch_states(qtt_engine* e, int B, int32_t* out, cudaStream_t stream);
/* The codes of the latest frame of streams 0..B-1 in one device buffer (no counterpart in the
 * reference, whose generate() returns the codes of one utterance at its end): out is device int32
 * [B][16], row s = stream s's most recent frame (its 16 groups), or -1s if the stream has no frame
 * yet. One small kernel on `stream`, asynchronous, so that a serving loop reads a whole batched
 * frame with one device-to-host copy instead of one per utterance. */
qtt_status qtt_batch_last_codes(qtt_engine* e, int B, int32_t* out, cudaStream_t stream);
/* Diagnostics of the batched path (parity tests): the first n of its scratch device pointers,
 * in this order: GEMM operand planes 0 and 1 (bf16 [2][128][3072] each: plane 0 = hi, plane 1 =
 * lo, row = token), sampled-head logits (fp32 [64][3072]), frame tokens (int32 [64][16]), stack
 * input, layer outputs 0 and 1, post-attention residual (fp32 [128][1024] each), q/k/v
 * (fp32 [128][4096]). */
qtt_status qtt_batch_debug_buffers(qtt_engine* e, void** ptrs, int n);
/* Parity tests: when set, batched frames also write every head's bf16-valued logits, fp32
 * [B][15][cp_vocab] for the code-predictor heads and [B][vocab] for the codec head (NULL: off). */
qtt_status qtt_batch_set_debug_outputs(qtt_engine* e, float* cp_logits, float* g0_logits);
/* One code-predictor decode step on the engine's own fp32 CP cache (position < 16). */
qtt_status qtt_cp_step(qtt_engine* e, const void* emb, int position, float* out_hidden, cudaStream_t stream);
/* Test hook: when non-NULL, each frame copies its raw bf16 head logits (as fp32) into
 * cp_logits [15][cp_vocab] and g0_logits [vocab]. Pass NULLs to turn it off. */
qtt_status qtt_set_debug_outputs(qtt_engine* e, float* cp_logits, float* g0_logits);
/* Profiling hook: when n > 0, each launch writes %globaltimer (ns) into stamps[0] at start
 * and stamps[k] after its k-th grid barrier (k < n). Pass n = 0 to turn it off. */
qtt_status qtt_set_debug_timeline(qtt_engine* e, unsigned long long* stamps, int n);
/* Profiling hook: CTA 0 stamps marks[3 k + {0,1,2}] = start of the k-th stage's GEMV, its
 * end, and the barrier arrival; every CTA stamps arrivals[(k - arrival_stage0) * num_ctas +
 * cta] for stages k in [arrival_stage0, arrival_stage0 + arrival_stages). Zeros turn it off. */
qtt_status qtt_set_debug_profile(qtt_engine* e, unsigned long long* marks, int n_marks,
                                 unsigned long long* arrivals, int arrival_stage0, int arrival_stages);
/* Error-path test hook (no counterpart in the reference): when barrier = k > 0, the batch-1
 * launches that follow (qtt_frames, qtt_prefill, qtt_backbone_step, qtt_cp_step) lose one
 * arrival at their k-th grid barrier (the last CTA does not arrive), and every
 * grid-barrier wait gives up after wait_ns nanoseconds (0: the built-in 2 s). Such a launch ends
 * early with the error word set; qtt_check then returns QTT_ERR_TIMEOUT and the engine stays
 * usable. barrier = 0 turns it off. */
qtt_status qtt_set_debug_barrier_fault(qtt_engine* e, int barrier, unsigned long long wait_ns);
/* Test hook (no counterpart in the reference): on = 1 makes the batched launches that follow apply
 * the q/k norms and RoPE and write the new K/V rows in their attention stage, the path of GPUs
 * whose thread-block clusters hold 2 CTAs, instead of in the QKV GEMM's epilogue (the default
 * wherever a cluster holds 4 CTAs, a QKV row tile then being one whole head). 0 turns it off. */
qtt_status qtt_set_debug_kv_in_attention(qtt_engine* e, int on);
/* Weight-ring refill policy of the persistent kernel: 0 (default) refills a freed slot only
 * after the consumers' next grid barrier, keeping refill traffic out of the barrier; 1 refills
 * as soon as a slot is free. */
qtt_status qtt_set_refill_policy(qtt_engine* e, int eager);
/* Synchronises `stream` and converts the engine's device error word into a status. */
qtt_status qtt_check(qtt_engine* e, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QTT_H_ */
