/*
 * magpie_tts_rt_b200 -- B200 (sm_100a) implementation of MagpieTTS-RT's
 * per-frame Local AR + sampling hot path, behind the reference's C ABI.
 *
 * Five groups of entry points:
 *
 * 1. The plugin-library ABI the runtime dlopen()s
 *    (reference: include/magpie_tts_rt/magpie_tts_rt_plugin.h:70-152,
 *    exported symbols cmake/magpie_tts_rt_plugins.map): mtt_plugin_get_api_v1
 *    and mtt_plugin_get_main_device_position_class_table_v1, with
 *    byte-identical structs and status codes.
 *
 * 2. The plugin kernel launchers (reference: plugins/local_ar_plugins.hpp:29-55,
 *    src/runtime/synthesis_kernels.hpp launch_finalize_local_step), as
 *    extern "C" functions with the same arguments, the same 0 / -1 return
 *    convention (-1 for a null pointer or a failed launch), stream-ordered,
 *    no host synchronisation, all buffers caller-owned device memory.  C++
 *    callers also get inline forwarders under the reference's names in
 *    namespace magpie_tts_rt::plugins (bottom of this header).
 *
 * 3. The batched frame entry (new; no single reference counterpart): one call
 *    runs the whole 16-position Local AR frame, sampling, EOS and the
 *    next-frame embedding sum for N independent sessions ("streams") held as
 *    structure-of-arrays device state.  It replaces, for N sessions at once,
 *    the reference's per-session Local AR graph launch plus
 *    launch_finalize_local_step (src/runtime/synthesis_pipeline.cpp:511-569).
 *
 * 4. The alignment controller (reference: src/runtime/alignment_kernel.hpp
 *    launch_alignment_controller), per utterance with the reference's
 *    arguments, and batched over sessions together with the Local AR EOS
 *    inputs (forbid_eos, unfinished, the finished latch) that the reference
 *    prepares on the host before every Local AR step.
 *
 * 5. The Main Decoder one-step (reference:
 *    tools/export/main_decoder_wrapper.py MainDecoderStepWrapper), batched
 *    over sessions: the decoder position between two Local AR frames.
 *
 * Streams (`void* stream`) are cudaStream_t values; NULL is the legacy
 * default stream.
 */
#ifndef MAGPIE_TTS_RT_B200_H_
#define MAGPIE_TTS_RT_B200_H_

#include <stddef.h>
#include <stdint.h>
#ifndef __cplusplus
#include <stdbool.h>
#endif

#if defined(__GNUC__) || defined(__clang__)
#define MTT_B200_API __attribute__((visibility("default")))
#else
#define MTT_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* 1. Plugin-library ABI v1 (byte-compatible with magpie_tts_rt_plugin.h)    */
/* ------------------------------------------------------------------------ */

#ifndef MAGPIE_TTS_RT_MAGPIE_TTS_RT_PLUGIN_H_
#define MTT_PLUGIN_ABI_VERSION_1 UINT32_C(1)
#define MTT_PLUGIN_CREATOR_COUNT_V1 UINT32_C(5)
#define MTT_PLUGIN_CREATOR_NAME_CAPACITY UINT32_C(64)
#define MTT_PLUGIN_CREATOR_VERSION_CAPACITY UINT32_C(16)
#define MTT_PLUGIN_NAMESPACE_CAPACITY UINT32_C(64)

typedef int32_t mtt_plugin_status_t;

#define MTT_PLUGIN_STATUS_OK INT32_C(0)
#define MTT_PLUGIN_STATUS_ALREADY_REGISTERED INT32_C(1)
#define MTT_PLUGIN_STATUS_INVALID_ARGUMENT INT32_C(2)
#define MTT_PLUGIN_STATUS_ABI_MISMATCH INT32_C(3)
#define MTT_PLUGIN_STATUS_REGISTRY_UNAVAILABLE INT32_C(4)
#define MTT_PLUGIN_STATUS_REGISTRATION_CONFLICT INT32_C(5)
#define MTT_PLUGIN_STATUS_REGISTRATION_FAILED INT32_C(6)
#define MTT_PLUGIN_STATUS_NOT_READY INT32_C(7)
#define MTT_PLUGIN_STATUS_CLASS_TABLE_CONFLICT INT32_C(8)

#define MTT_MAIN_DEVICE_POSITION_CLASS_COUNT_V1 UINT32_C(21)
#define MTT_MAIN_DEVICE_POSITION_K_COUNT_V1 UINT32_C(249)
#define MTT_MAIN_DEVICE_POSITION_FUNCTION_NAME_CAPACITY UINT32_C(256)

typedef struct mtt_plugin_creator_v1 {
  uint32_t struct_size;
  uint32_t abi_version;
  char name[MTT_PLUGIN_CREATOR_NAME_CAPACITY];
  char version[MTT_PLUGIN_CREATOR_VERSION_CAPACITY];
  char plugin_namespace[MTT_PLUGIN_NAMESPACE_CAPACITY];
} mtt_plugin_creator_v1_t;

typedef mtt_plugin_status_t (*mtt_plugin_register_v1_fn)(void);

typedef struct mtt_plugin_api_v1 {
  uint32_t struct_size;
  uint32_t abi_version;
  uint32_t creator_count;
  uint32_t reserved_0;
  mtt_plugin_creator_v1_t creators[MTT_PLUGIN_CREATOR_COUNT_V1];
  mtt_plugin_register_v1_fn register_plugins;
  uint64_t reserved[4];
} mtt_plugin_api_v1_t;

typedef struct mtt_main_device_position_class_v1 {
  uint32_t struct_size;
  uint32_t abi_version;
  uint32_t operation;
  uint32_t class_index;
  uint32_t parameter_transport;
  uint32_t block_x;
  uint32_t block_y;
  uint32_t block_z;
  uint32_t shared_memory_bytes;
  uint32_t reserved_0;
  uint64_t parameter_offset;
  uint64_t parameter_size;
  char function_name[MTT_MAIN_DEVICE_POSITION_FUNCTION_NAME_CAPACITY];
  uint64_t reserved[4];
} mtt_main_device_position_class_v1_t;

typedef struct mtt_main_device_position_k_v1 {
  uint32_t struct_size;
  uint32_t abi_version;
  int32_t active_k;
  int32_t qk_class_index;
  uint32_t qk_grid_x;
  uint32_t qk_grid_y;
  uint32_t qk_grid_z;
  int32_t pv_class_index;
  uint32_t pv_grid_x;
  uint32_t pv_grid_y;
  uint32_t pv_grid_z;
  uint32_t reserved_0;
  uint64_t reserved[4];
} mtt_main_device_position_k_v1_t;

typedef struct mtt_main_device_position_class_table_v1 {
  uint32_t struct_size;
  uint32_t abi_version;
  uint32_t class_count;
  uint32_t k_count;
  mtt_main_device_position_class_v1_t classes[MTT_MAIN_DEVICE_POSITION_CLASS_COUNT_V1];
  mtt_main_device_position_k_v1_t k_records[MTT_MAIN_DEVICE_POSITION_K_COUNT_V1];
  uint64_t reserved[4];
} mtt_main_device_position_class_table_v1_t;
#endif /* MAGPIE_TTS_RT_MAGPIE_TTS_RT_PLUGIN_H_ */

/*
 * Replaces mtt_plugin_get_api_v1 (plugins/local_ar_plugins.cu:4858-4900).
 * The caller pre-fills struct_size and abi_version; NULL -> INVALID_ARGUMENT,
 * mismatch -> ABI_MISMATCH.  Fills the five creator descriptors in the
 * reference's order and names (MagpieLocalARSampling, MagpieLocalAREos,
 * MagpieLayerNorm, MagpieGeluTanh, MagpieSoftmax; version "1", namespace
 * "magpie_tts_rt").  register_plugins returns REGISTRY_UNAVAILABLE in builds
 * without TensorRT (this build), else the reference's registration statuses.
 */
MTT_B200_API mtt_plugin_status_t mtt_plugin_get_api_v1(mtt_plugin_api_v1_t* api);

/*
 * Replaces mtt_plugin_get_main_device_position_class_table_v1
 * (plugins/local_ar_plugins.cu:4083-4104,4908-4913).  The Main Decoder mode-8
 * bank is outside this library's path, so the table never becomes ready:
 * NULL -> INVALID_ARGUMENT, wrong struct_size/abi_version -> ABI_MISMATCH,
 * otherwise NOT_READY.
 */
MTT_B200_API mtt_plugin_status_t mtt_plugin_get_main_device_position_class_table_v1(
    mtt_main_device_position_class_table_v1_t* table);

/* ------------------------------------------------------------------------ */
/* 2. Plugin kernel launchers                                                */
/* ------------------------------------------------------------------------ */

/*
 * Replaces launch_local_ar_sampling (plugins/local_ar_plugins.hpp:29-41).
 * One Local AR position for one session: logits [2][2024] bf16 (conditional
 * row, unconditional row); unfinished / finished / forbid_eos [1] bool;
 * rng_seed [1] int64 in [0, 2^32); rng_counter [1] int64; embedding table
 * [2024][768] bf16.  Writes sampled_token [1] int64, next_embedding [2][768]
 * bf16 (the chosen row, duplicated for both CFG rows), updated_rng_counter [1]
 * (counter + 1 when the counter is valid) and invalid_rows [1] int32.
 * CFG 2.5, temperature 0.6, inclusive top-80, Philox-4x32-10 Gumbel.
 */
MTT_B200_API int mtt_b200_launch_local_ar_sampling(
    const void* logits_bf16, const bool* unfinished, const bool* finished, const bool* forbid_eos,
    const int64_t* rng_seed, const int64_t* rng_counter, const void* embedding_weight_bf16,
    int64_t* sampled_token, void* next_embedding_bf16, int64_t* updated_rng_counter,
    int32_t* invalid_rows, void* stream);

/* Replaces local_ar_eos_workspace_size (plugins/local_ar_plugins.hpp:43):
 * the same byte count, so callers size their buffers identically. */
MTT_B200_API size_t mtt_b200_local_ar_eos_workspace_size(void);

/*
 * Replaces launch_local_ar_eos (plugins/local_ar_plugins.hpp:45-55).
 * decoder_hidden [2][768] bf16, codec_tokens [1][8][2] int64, flags [1] bool,
 * final projection weight [32384][768] bf16 and bias [32384] bf16, caller
 * workspace of mtt_b200_local_ar_eos_workspace_size() bytes (256-byte
 * aligned).  Writes end_frame_index [1] int32 in {-1, 0, 1}.
 */
MTT_B200_API int mtt_b200_launch_local_ar_eos(
    const void* decoder_hidden_bf16, const int64_t* codec_tokens, const bool* unfinished,
    const bool* finished, const bool* forbid_eos, const void* final_weight_bf16,
    const void* final_bias_bf16, void* workspace, int32_t* end_frame_index, void* stream);

/*
 * Replaces launch_finalize_local_step (src/runtime/synthesis_kernels.cu:177-214):
 * copies the step's [8][2] codec tokens into the [8][8] batch aggregate at
 * frame_offset (0, 2, 4 or 6), copies the canonical invalid / EOS outputs
 * into the step slots, commits updated_rng_counter into rng_counter and
 * latches generation_finished when end_frame_index is 0 or 1.  Returns 0, or
 * -1 for a null pointer, a bad frame_offset or a failed launch.
 */
MTT_B200_API int mtt_b200_launch_finalize_local_step(
    const int64_t* step_codec_tokens, int64_t* aggregate_codec_tokens, uint32_t frame_offset,
    const int32_t* canonical_invalid_rows, const int32_t* canonical_end_frame_index,
    int32_t* step_invalid_rows, int32_t* step_end_frame_index, const int64_t* updated_rng_counter,
    int64_t* rng_counter, bool* generation_finished, void* stream);

/*
 * Replace the kernels behind the MagpieLayerNorm, MagpieGeluTanh and
 * MagpieSoftmax (mode 0) plugins: launch_layer_norm / launch_gelu_tanh /
 * launch_softmax (plugins/local_ar_plugins.hpp:57-76,
 * plugins/local_ar_plugins.cu:4218-4356).  bf16 in and out, stream-ordered,
 * return 0, or -1 for a null pointer, a size out of range or a failed launch.
 *   layer_norm: rows of width 768, 1 <= row_count <= 1024, no bias, eps 1e-5;
 *   gelu_tanh:  1 <= element_count <= 3072 * 512;
 *   softmax:    batch_count >= 1 rows of 1 <= element_count <= 512.
 */
MTT_B200_API int mtt_b200_launch_layer_norm(const void* input_bf16, const void* weight_bf16, void* output_bf16,
                                            int32_t row_count, void* stream);
MTT_B200_API int mtt_b200_launch_gelu_tanh(const void* input_bf16, void* output_bf16, size_t element_count,
                                           void* stream);
MTT_B200_API int mtt_b200_launch_softmax(const void* input_bf16, void* output_bf16, int32_t batch_count,
                                         int32_t element_count, void* stream);

/* ------------------------------------------------------------------------ */
/* 3. Batched Local AR frame                                                 */
/* ------------------------------------------------------------------------ */

#define MTT_B200_STATUS_OK 0
#define MTT_B200_STATUS_INVALID_ARGUMENT -1
#define MTT_B200_STATUS_CUDA_ERROR -2
#define MTT_B200_STATUS_UNSUPPORTED -3

/* Model shape: head width is always 64; the in-projection 768 -> d_model
 * exists iff d_model != 768 (magpietts.py:1347-1352). */
typedef struct mtt_b200_local_ar_shape {
  int32_t d_model;
  int32_t n_layers;
  int32_t n_heads;
  int32_t d_ffn;
} mtt_b200_local_ar_shape_t;

/* Device pointers, bf16, PyTorch [out][in] layout.  in_proj_* are NULL when
 * d_model == 768.  final_* may be NULL when EOS evaluation is never enabled
 * (every stream unfinished, finished or forbid_eos on every frame). */
typedef struct mtt_b200_local_ar_weights {
  const void* in_proj_w; /* [d][768] */
  const void* in_proj_b; /* [d] */
  const void* pos;       /* [>=16][d] learnable position table */
  const void* ln_self;   /* [L][d] */
  const void* qkv;       /* [L][3d][d]: q rows, k rows, v rows */
  const void* o;         /* [L][d][d] */
  const void* ln_ff;     /* [L][d] */
  const void* ffn1;      /* [L][F][d] */
  const void* ffn2;      /* [L][d][F] */
  const void* head_w;    /* [16][2024][d] */
  const void* head_b;    /* [16][2024] */
  const void* emb;       /* [16][2024][768] audio embedding tables */
  const void* final_w;   /* [32384][768] Main Decoder final projection (EOS) */
  const void* final_b;   /* [32384] */
  /* Optional [16][2024][d] bf16: the in-projection folded into the embedding
   * tables, emb_proj[p][v] = bf16(W_in table_p[v] + b_in), made once by
   * mtt_b200_launch_fold_in_projection.  When present, positions 1..15 read
   * their in-projected input row from it instead of multiplying the gathered
   * 768-wide row by W_in (same rounding points: f32 accumulation, one bf16
   * rounding, then the position add).  NULL: multiply at every position. */
  const void* emb_proj;
} mtt_b200_local_ar_weights_t;

/* Bytes of the folded table for a shape (0 for identity in-projections). */
MTT_B200_API size_t mtt_b200_fold_in_projection_bytes(const mtt_b200_local_ar_shape_t* shape);

/* Computes emb_proj (see above) from weights->emb, in_proj_w, in_proj_b into
 * `out` (mtt_b200_fold_in_projection_bytes bytes, 16-byte aligned).  A one-time
 * weight transform, run when the weights are loaded.  Returns MTT_B200_STATUS_*. */
MTT_B200_API int mtt_b200_launch_fold_in_projection(const mtt_b200_local_ar_shape_t* shape,
                                                   const mtt_b200_local_ar_weights_t* weights, void* out,
                                                   void* stream);

/* Frame implementations.  For the shape d_model 256, 4 heads, FFN 1024,
 * 1 layer these fused single-launch kernels exist: FUSED_CLUSTER spreads a
 * 16-row tile (8 sessions with CFG, 16 without) over a 16-CTA thread-block
 * cluster (lowest latency per tile, at most a few clusters on the device at
 * once); FUSED_TILE runs 8 sessions in one CTA with their KV cache in tensor
 * memory; FUSED_PAIR runs 16 sessions on a 2-CTA cluster, each CTA streaming
 * half of every weight matrix; SPLIT_1 / _2 / _4 / _8 run 8 sessions on a
 * cluster of 1, 2, 4 or 8 CTAs (SPLIT_2X32: 16 sessions on 2 CTAs), each
 * streaming that fraction of every weight
 * matrix, with the GEMMs on tcgen05 tensor cores (accumulators and the KV
 * cache in tensor memory).  AUTO picks FUSED_CLUSTER while the batch's tiles
 * fit in one wave of its clusters, then SPLIT_8 and _4 while theirs do
 * (fewer sessions per GPU: more CTAs per session, shorter frames), then QUAD
 * and SPLIT_2 while theirs do, then FUSED_PAIR while its 16-session tiles fit
 * in one wave, then FUSED_TILE, and the phase kernels for other shapes. */
#define MTT_B200_FRAME_PATH_AUTO 0
#define MTT_B200_FRAME_PATH_PHASE_KERNELS 1
#define MTT_B200_FRAME_PATH_FUSED_CLUSTER 2
#define MTT_B200_FRAME_PATH_FUSED_TILE 3
#define MTT_B200_FRAME_PATH_FUSED_PAIR 4
#define MTT_B200_FRAME_PATH_SPLIT_1 5
#define MTT_B200_FRAME_PATH_SPLIT_2 6
#define MTT_B200_FRAME_PATH_SPLIT_4 7
#define MTT_B200_FRAME_PATH_SPLIT_8 8
#define MTT_B200_FRAME_PATH_SPLIT_2X32 9
/* QUAD: 16 sessions (32 rows) on a 4-CTA cluster, one attention head per CTA
 * (its key/value cache in tensor memory), each CTA streaming a quarter of
 * FFN and head weights, tcgen05 GEMMs on 32-row tiles (benchmark shape). */
#define MTT_B200_FRAME_PATH_QUAD 10
/* OCTO: 16 sessions (32 rows) on an 8-CTA cluster, two CTAs per attention
 * head, each CTA streaming an eighth of the FFN and head weights (benchmark
 * shape); for batches whose 8-session tiles outnumber the 8-CTA clusters
 * that fit at once. */
#define MTT_B200_FRAME_PATH_OCTO 11

/* Sampling configuration; the reference's values are 80 / 0.6 / 2.5 with CFG
 * and top-k.  argmax != 0 selects greedy decoding (no RNG, counter unchanged;
 * magpietts_fused_sampling.py:136-197).  cfg == 0 runs one row per stream.
 * path: MTT_B200_FRAME_PATH_*; requesting the fused path where it cannot run
 * returns MTT_B200_STATUS_UNSUPPORTED. */
typedef struct mtt_b200_sampling_config {
  int32_t top_k;
  float temperature;
  float cfg_scale;
  int32_t argmax;
  int32_t cfg;
  int32_t path;
} mtt_b200_sampling_config_t;

/*
 * Structure-of-arrays session state for n_streams independent sessions
 * (device pointers).  Stream s owns CFG rows 2s (conditional) and 2s+1
 * (unconditional), its own seed (its session's seed: row 0 of a one-row
 * application batch) and its own RNG counter.
 */
typedef struct mtt_b200_stream_batch {
  int32_t n_streams;
  int32_t reserved_0;
  const void* decoder_hidden;  /* [n][rows][768] bf16, rows = 2 (cfg) or 1 */
  const bool* unfinished;      /* [n] */
  const bool* finished;        /* [n] */
  const bool* forbid_eos;      /* [n] */
  const bool* active;          /* [n] or NULL: inactive streams are skipped, outputs untouched */
  const int64_t* rng_seed;     /* [n] */
  int64_t* rng_counter;        /* [n] in/out: +16 per frame while valid (argmax: unchanged) */
  int64_t* codec_tokens;       /* [n][8][2] out, position p = frame*8 + codebook */
  int32_t* invalid_rows;       /* [n] out: 0 valid, else invalid (max over positions) */
  int32_t* end_frame_index;    /* [n] out: -1, 0 or 1 */
  void* next_embedding;        /* [n][768] bf16 out: sum_p table_p[tok_p] / 16 */
  /* Optional (NULL in production): */
  const int64_t* forced_tokens; /* [n][16]: next-position inputs replace the sampled
                                   tokens (teacher forcing, for parity checks) */
  void* logits_out;             /* [n][16][rows][2024] bf16 per-position logits */
  /* Folding launch_finalize_local_step (src/runtime/synthesis_kernels.cu:53-86)
   * into the frame call (zero-initialised: the [n][8][2] layout, no latch): */
  int32_t codec_frames_stride;  /* codec_tokens is [n][8][stride]; 0 means 2.  8 writes the
                                   steady emission aggregate [n][8][8] directly */
  int32_t codec_frame_offset;   /* this frame's two frames go to columns offset, offset + 1
                                   (0, 2, 4, 6 for the aggregate); even, offset + 2 <= stride */
  bool* finished_latch;         /* [n] or NULL: set to true where end_frame_index is 0 or 1
                                   (may alias `finished`; it is written after the frame read it) */
  int32_t* codec_frames;        /* [n] or NULL: for sessions not finished on entry, the audio
                                   frames of the aggregate so far -- offset + 2, or offset +
                                   end_frame_index at the EOS frame (the EOS frame is not audio;
                                   src/runtime/eos_contract.hpp:14-30): the F of the NanoCodec
                                   [1][8][F] route after the emission batch's last frame */
  /* Optional: the EOS projection of these sessions' decoder_hidden, already
   * computed by the Main Decoder step that produced it
   * (mtt_b200_main_decoder_batch_t.eos_projection, [n][32] 32-bit words).
   * The frame then skips its own projection and decides EOS from it. */
  const void* eos_projection;
} mtt_b200_stream_batch_t;

/* Device workspace bytes for launching up to max_streams streams. */
MTT_B200_API size_t mtt_b200_local_ar_frame_workspace_size(const mtt_b200_local_ar_shape_t* shape,
                                                          int32_t max_streams, int32_t cfg);

/*
 * One Local AR frame (16 positions) for a batch of streams, stream-ordered.
 * workspace: >= mtt_b200_local_ar_frame_workspace_size(shape, n_streams, cfg)
 * bytes, 256-byte aligned, caller-owned; contents need not be preserved
 * between calls.  Returns MTT_B200_STATUS_*.  Data-plane failures (non-finite
 * logits, no candidate, bad seed/counter, overlapping flags) are reported
 * in-band through invalid_rows, as in the reference.
 */
MTT_B200_API int mtt_b200_launch_local_ar_frame(const mtt_b200_local_ar_shape_t* shape,
                                               const mtt_b200_local_ar_weights_t* weights,
                                               const mtt_b200_sampling_config_t* sampling,
                                               const mtt_b200_stream_batch_t* batch, void* workspace,
                                               size_t workspace_bytes, void* stream);

/*
 * Allocation-free variant of mtt_b200_launch_local_ar_frame (no counterpart
 * in the reference).  For callers that cannot call cudaMalloc where frames
 * run: a TensorRT plugin's enqueue(), code being captured into a CUDA graph,
 * a real-time synthesis thread that must not stall on an allocation.  The
 * scratch memory is a device array of MTT_B200_STATIC_FRAME_WORKSPACE_BYTES
 * (2 MiB) inside this library (held by every GPU that loads it, until exit)
 * instead of a caller workspace.  A batch fits when
 * mtt_b200_local_ar_frame_workspace_size(shape, n_streams, cfg) is at most
 * that size: with CFG up to 40 sessions of the benchmark shape (d=256,
 * 1 layer, FFN 1024) or 7 of the d=768 2-layer shape (74 and 14 without
 * CFG).  A larger batch is rejected with
 * MTT_B200_STATUS_STATIC_WORKSPACE_TOO_SMALL and nothing is launched.  The
 * first call on a device (that device current) resolves the array's device
 * address; make it before any stream capture.  All calls share the array:
 * calls whose kernels overlap on the GPU race.  Other arguments and results
 * are those of mtt_b200_launch_local_ar_frame.
 */
#define MTT_B200_STATIC_FRAME_WORKSPACE_BYTES ((size_t)2 << 20)
#define MTT_B200_STATUS_STATIC_WORKSPACE_TOO_SMALL -4
MTT_B200_API int mtt_b200_launch_local_ar_frame_static_workspace(const mtt_b200_local_ar_shape_t* shape,
                                                                const mtt_b200_local_ar_weights_t* weights,
                                                                const mtt_b200_sampling_config_t* sampling,
                                                                const mtt_b200_stream_batch_t* batch,
                                                                void* stream);

/* The path (MTT_B200_FRAME_PATH_PHASE_KERNELS, _FUSED_CLUSTER, _FUSED_TILE,
 * _FUSED_PAIR, _SPLIT_1 / _2 / _4 / _8 or _QUAD) that mtt_b200_launch_local_ar_frame takes for this shape,
 * configuration and batch size on the current device, or
 * MTT_B200_STATUS_UNSUPPORTED. */
MTT_B200_API int32_t mtt_b200_local_ar_frame_path(const mtt_b200_local_ar_shape_t* shape,
                                                  const mtt_b200_sampling_config_t* sampling, int32_t n_streams);

/* Thread-block clusters of a fused frame path (MTT_B200_FRAME_PATH_FUSED_CLUSTER,
 * _FUSED_TILE (1-CTA clusters), _FUSED_PAIR, _SPLIT_1 / _2 / _4 / _8, _QUAD) that
 * the current device runs at once, each holding one tile of the batch; 0 when
 * the path cannot run here.  AUTO compares the batch's tiles with these. */
MTT_B200_API int32_t mtt_b200_local_ar_frame_path_clusters(int32_t path);

/* Number of kernels mtt_b200_launch_local_ar_frame enqueues for this shape,
 * configuration and batch on the current device (for launch accounting). */
MTT_B200_API int32_t mtt_b200_local_ar_frame_launch_count(const mtt_b200_local_ar_shape_t* shape,
                                                          const mtt_b200_sampling_config_t* sampling,
                                                          int32_t n_streams);

/* ------------------------------------------------------------------------ */
/* 4. Alignment controller and the Local AR's EOS inputs                     */
/* ------------------------------------------------------------------------ */

/* Layout-identical to AlignmentKernelContract (src/runtime/alignment_kernel.hpp:9-15). */
typedef struct mtt_b200_alignment_contract {
  uint32_t text_length;
  uint32_t ignored_terminal_tokens;
  uint32_t short_text_no_prior_max_tokens;
  uint32_t lookahead;
  uint32_t sink_threshold;
} mtt_b200_alignment_contract_t;

/*
 * Replaces launch_alignment_controller (src/runtime/alignment_kernel.hpp:
 * 20-29, alignment_kernel.cu:158-184): one utterance, all pointers device
 * pointers.  alignment_scores [2][T] bf16 (only the conditional row 0 is
 * read), counters [T] uint32 and last_attended [1] uint32 (state, updated),
 * next_prior [2][1][T] bf16, attended_token_index [1] int64, unfinished_text
 * [1] bool, invalid_state [1] int32.  Picks the attended token as the
 * left-most maximum of row 0 over the search window, counts the visit, writes
 * unfinished = attended < T - ignored_terminal_tokens and the next prior
 * (0.1, with 1.0 at the history / attended / look-ahead tokens past the last
 * sink, or on every token for short texts).  Data-plane errors are in-band:
 * invalid_state = 1 for a rejected contract (nothing else written), a
 * non-finite score anywhere in row 0 or a counter overflow (state advanced,
 * prior not written).  Returns the launch's cudaError_t value (0 on
 * success; cudaErrorInvalidValue for a NULL pointer), stream-ordered, no
 * host synchronisation.
 */
MTT_B200_API int mtt_b200_launch_alignment_controller(
    const void* alignment_scores_bf16, const mtt_b200_alignment_contract_t* contract, uint32_t* counters,
    uint32_t* last_attended, void* next_prior_bf16, int64_t* attended_token_index, bool* unfinished_text,
    int32_t* invalid_state, void* stream);

/*
 * The same controller for n_sessions utterances in one launch (new; the
 * reference runs one launch per session), plus the Local AR inputs the
 * reference's pipeline prepares around it on the host, so that one decoder
 * step is [Main Decoder] -> this -> mtt_b200_launch_local_ar_frame with no
 * host copy in between:
 *   forbid_eos[s] = decoder_steps[s] < 2, then decoder_steps[s] += 1
 *     (synthesis_pipeline.cpp:525-569, generated_decoder_steps_);
 *   finished[s] |= end_frame_index[s] in {0, 1}, the previous frame's result
 *     (the latch of launch_finalize_local_step, synthesis_kernels.cu:79-84;
 *     initialise end_frame_index to -1);
 *   unfinished[s] = the controller's unfinished_text.
 * Point forbid_eos / unfinished / finished at the frame batch's arrays.
 * Row layout: session s's score and prior rows at s * 2 * token_stride
 * (conditional) and + token_stride (unconditional), its counters at
 * s * token_stride; token_stride >= every text_length (a longer text is
 * rejected in-band).  Inactive sessions (active[s] false) are untouched.
 * decoder_steps / forbid_eos and end_frame_index / finished are optional
 * pairs (both NULL or both set).  Returns MTT_B200_STATUS_*.
 */
typedef struct mtt_b200_alignment_batch {
  int32_t n_sessions;
  uint32_t token_stride;
  uint32_t ignored_terminal_tokens;
  uint32_t short_text_no_prior_max_tokens;
  uint32_t lookahead;
  uint32_t sink_threshold;
  const uint32_t* text_length;    /* [n] */
  const bool* active;             /* [n] or NULL */
  const void* alignment_scores;   /* [n][2][token_stride] bf16 */
  uint32_t* counters;             /* [n][token_stride] in/out */
  uint32_t* last_attended;        /* [n] in/out */
  void* next_prior;               /* [n][2][token_stride] bf16 out */
  int64_t* attended_token_index;  /* [n] out */
  bool* unfinished;               /* [n] out */
  int32_t* invalid_state;         /* [n] out */
  int64_t* decoder_steps;         /* [n] in/out, or NULL */
  bool* forbid_eos;               /* [n] out, or NULL */
  const int32_t* end_frame_index; /* [n] in, or NULL */
  bool* finished;                 /* [n] in/out, or NULL */
} mtt_b200_alignment_batch_t;

MTT_B200_API int mtt_b200_launch_alignment_batch(const mtt_b200_alignment_batch_t* batch, void* stream);

/* ------------------------------------------------------------------------ */
/* 5. Main Decoder one-step                                                  */
/* ------------------------------------------------------------------------ */

/* Device pointers, bf16, PyTorch [out][in] layout, layer-major
 * (tools/export/main_decoder_wrapper.py:778-911; accepted shape 12 layers,
 * width 768, 12 self-attention heads of 64, one 128-wide cross-attention
 * head, FFN 3072 of kernel-one convolutions). */
typedef struct mtt_b200_main_decoder_weights {
  const void* pos;      /* [pos_rows][768] learnable position embeddings */
  const void* ln_self;  /* [L][768] */
  const void* qkv;      /* [L][2304][768]: q, k, v rows (12 heads x 64 each) */
  const void* o;        /* [L][768][768] */
  const void* ln_xq;    /* [L][768] cross-attention query norm */
  const void* xq;       /* [L][128][768] */
  const void* xo;       /* [L][768][128] */
  const void* ln_ff;    /* [L][768] */
  const void* ffn1;     /* [L][3072][768] */
  const void* ffn2;     /* [L][768][3072] */
  const void* norm_out; /* [768] */
  int32_t n_layers;     /* >= 10 (alignment layers 4, 5, 8, 9; prior layers 2..10) */
  int32_t pos_rows;     /* >= cache_capacity */
  /* Optional (for eos_projection): the final projection [16 x 2024][768] and
   * its bias [16 x 2024], bf16, as in mtt_b200_local_ar_weights_t. */
  const void* final_w;
  const void* final_b;
} mtt_b200_main_decoder_weights_t;

/* Structure-of-arrays state of n sessions (device pointers).  Rows 2s and
 * 2s + 1 are session s's conditional and unconditional rows.  S =
 * token_stride (a multiple of 8, <= 512, >= every text length). */
typedef struct mtt_b200_main_decoder_batch {
  int32_t n_sessions;
  int32_t cache_capacity;      /* positions per session cache (the reference: 467) */
  int32_t token_stride;        /* S */
  int32_t reserved_0;
  const void* embedded;        /* [n][768] bf16: the codec-token embedding sum
                                  (the Local AR frame's next_embedding) */
  const int64_t* position;     /* [n] absolute position this step writes, in [0, cache_capacity) */
  const uint32_t* text_length; /* [n] text tokens T, 1 <= T <= S */
  const bool* active;          /* [n] or NULL: inactive sessions are skipped, their outputs untouched */
  void* self_k;                /* [n][L][2][12][cache_capacity][64] bf16, in/out */
  void* self_v;                /* same */
  bool* self_mask;             /* [n][2][cache_capacity] key mask, in/out (one for all layers) */
  const void* cross_k;         /* [n][L][2][S][128] bf16 text keys (prefill output) */
  const void* cross_v;         /* same */
  const bool* cond_mask;       /* [n][2][S] condition mask */
  const void* prior;           /* [n][2][S] bf16 attention prior (the alignment gate's next_prior) */
  void* hidden;                /* [n][2][768] bf16 out: the Local AR frame's decoder_hidden */
  void* alignment;             /* [n][2][S] bf16 out: the alignment gate's scores */
  int32_t* status;             /* [n] out: 0; 1 for a position or text length out of range
                                  (nothing written for the session); 2 when a cache copy did
                                  not complete within its bounded wait (outputs unreliable) */
  /* Optional [n][32] 32-bit words out (NULL: not computed): the Local AR's EOS
   * projection of the hidden state this step produces (the Main Decoder
   * final projection's guided logits reduced per position,
   * plugins/local_ar_plugins.cu:1372-1432), computed right after the last
   * layer on the tensor cores for every session: words [0, 16) the largest
   * guided code logit of positions 0..15 as order-preserving keys, words
   * [16, 32) the guided EOS logits (f32).  Pass it to the frame as
   * mtt_b200_stream_batch_t.eos_projection.  Needs weights final_w / final_b. */
  void* eos_projection;
  float eos_cfg_scale;         /* CFG scale of the guided logits (the reference: 2.5) */
  int32_t reserved_1;
} mtt_b200_main_decoder_batch_t;

/* Workspace bytes for up to max_sessions sessions (0 for bad arguments). */
MTT_B200_API size_t mtt_b200_main_decoder_workspace_size(int32_t max_sessions, int32_t token_stride);

/*
 * One Main Decoder position for every session (replaces one
 * MainDecoderStepWrapper engine launch per session,
 * src/runtime/synthesis_pipeline.cpp:572-648): writes each session's new
 * key / value at its position and sets its key mask there, and produces the
 * decoder hidden state and the alignment scores.  Stream-ordered; the layer
 * GEMMs run on this library's tcgen05 kernel (the first call on a device
 * sets its shared-memory opt-in there: make that call before any stream
 * capture).  workspace: >=
 * mtt_b200_main_decoder_workspace_size bytes, 256-byte aligned.  Returns
 * MTT_B200_STATUS_*.
 */
MTT_B200_API int mtt_b200_launch_main_decoder_step(const mtt_b200_main_decoder_weights_t* weights,
                                                   const mtt_b200_main_decoder_batch_t* batch, void* workspace,
                                                   size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* 6. Per-GPU session engine (the host side of the per-step loop)            */
/* ------------------------------------------------------------------------ */

/*
 * Replaces, for up to max_sessions sessions on one GPU, the reference's
 * per-session step sequence of SynthesisPipeline::run_local
 * (src/runtime/synthesis_pipeline.cpp:511-569: a D2D copy of `unfinished`, an
 * H2D copy of forbid_eos, the Local AR graph launch, finalize_local_step) and
 * the per-session CUDA graphs of SessionResources
 * (src/runtime/session_resources.cpp:661-684).  The engine owns every
 * session's structure-of-arrays state on the device (RNG seed and counter,
 * alignment counters and prior, EOS flags, codec tokens, decoder cache when
 * with_decoder) and its own CUDA stream; one step is one replay of a CUDA
 * graph captured on the engine's second step (the first runs the same
 * launches one by one):
 *   [Main Decoder step -> ]alignment gate -> Local AR frame[ -> position + 1]
 * for every open session, with no host copy inside.  Sessions are opened and
 * closed between steps by slot; a closed slot is skipped by every kernel.
 * Weights are caller-owned device memory that must outlive the engine.
 * Every function returns MTT_B200_STATUS_*; the engine is not thread-safe
 * (one host thread drives one engine, as one request thread drives one
 * reference session).
 */
typedef struct mtt_b200_session_engine mtt_b200_session_engine_t;

typedef struct mtt_b200_session_engine_config {
  int32_t max_sessions;
  int32_t token_stride;      /* text tokens per row: a multiple of 8, <= 512 */
  int32_t with_decoder;      /* 1: each step starts with the Main Decoder step */
  int32_t cache_capacity;    /* decoder positions per session (with_decoder) */
  /* the alignment contract (src/runtime/alignment_kernel.hpp:9-15) */
  uint32_t ignored_terminal_tokens;
  uint32_t short_text_no_prior_max_tokens;
  uint32_t lookahead;
  uint32_t sink_threshold;
  mtt_b200_local_ar_shape_t shape;
  mtt_b200_local_ar_weights_t local_ar;    /* device pointers (final_w / final_b for EOS) */
  mtt_b200_sampling_config_t sampling;
  mtt_b200_main_decoder_weights_t decoder; /* with_decoder */
  /* Optional caller-owned device buffers (NULL: the engine allocates them):
   * decoder_hidden [n][rows][768] bf16 (rows 2 with CFG), alignment_scores
   * [n][2][S] bf16, next_embedding [n][768] bf16; 16-byte aligned. */
  void* decoder_hidden;
  void* alignment_scores;
  void* next_embedding;
} mtt_b200_session_engine_config_t;

/* Device buffers of the engine, for the caller to fill or read on the
 * engine's stream (sessions in slot order; rows 2s / 2s + 1). */
typedef struct mtt_b200_session_engine_buffers {
  void* stream;                 /* cudaStream_t of the engine */
  void* decoder_hidden;         /* [n][2][768] bf16: the frame's input (written by the decoder
                                   step with with_decoder, else by the caller before each step) */
  void* alignment_scores;       /* [n][2][S] bf16: the gate's input (likewise) */
  void* next_embedding;         /* [n][768] bf16: the frame's embedding sum (the decoder's next input) */
  int64_t* codec_tokens;        /* [n][8][2] int64: the last step's tokens */
  int32_t* end_frame_index;     /* [n] */
  int32_t* invalid_rows;        /* [n] */
  int64_t* rng_counter;         /* [n] */
  bool* finished;               /* [n] */
  int64_t* position;            /* [n] decoder positions (with_decoder) */
  int32_t* decoder_status;      /* [n] (with_decoder) */
} mtt_b200_session_engine_buffers_t;

MTT_B200_API int mtt_b200_session_engine_create(const mtt_b200_session_engine_config_t* config,
                                                mtt_b200_session_engine_t** engine);
MTT_B200_API void mtt_b200_session_engine_destroy(mtt_b200_session_engine_t* engine);
MTT_B200_API int mtt_b200_session_engine_buffers(const mtt_b200_session_engine_t* engine,
                                                 mtt_b200_session_engine_buffers_t* buffers);

/* Opens session `slot` (its state reset on the engine's stream): seed in
 * [0, 2^32) (row 0 of a one-row request, docs/c-abi.md random_seed), text
 * length 1..token_stride.  With the decoder: cross_k / cross_v [L][2][T][128]
 * bf16 and cond_mask [2][T] bool (device pointers, the prefill's outputs; T =
 * text_length) are copied into the slot, initial_embedding [768] bf16 (or
 * NULL for zeros) is its first decoder input, its cache starts empty at
 * position 0. */
MTT_B200_API int mtt_b200_session_engine_open(mtt_b200_session_engine_t* engine, int32_t slot, int64_t seed,
                                              uint32_t text_length, const void* cross_k, const void* cross_v,
                                              const bool* cond_mask, const void* initial_embedding);
MTT_B200_API int mtt_b200_session_engine_close(mtt_b200_session_engine_t* engine, int32_t slot);

/* One step for every open session, enqueued on the engine's stream. */
MTT_B200_API int mtt_b200_session_engine_step(mtt_b200_session_engine_t* engine);

/* Copies the last step's codec tokens [n][8][2], end-frame indices [n] and
 * invalid flags [n] of slots [0, n) to host memory (any pointer may be NULL)
 * and waits for the engine's stream. */
MTT_B200_API int mtt_b200_session_engine_collect(mtt_b200_session_engine_t* engine, int32_t n,
                                                 int64_t* codec_tokens, int32_t* end_frame_index,
                                                 int32_t* invalid_rows);

/* ------------------------------------------------------------------------ */
/* Test hooks (no reference counterpart beyond launch_test_clamped_gumbel,   */
/* plugins/local_ar_plugins.hpp:171-175)                                      */
/* ------------------------------------------------------------------------ */

/* gumbel[i] = -log(-log(clamp(uniform[i], 6e-8, 0.99999994))) on the device. */
MTT_B200_API int mtt_b200_launch_test_clamped_gumbel(const float* uniform, float* gumbel, size_t count,
                                                     void* stream);
/* out[i] = the device's correctly rounded natural log of x[i]. */
MTT_B200_API int mtt_b200_launch_test_log(const float* x, float* out, size_t count, void* stream);

/* The projection GEMM of the Main Decoder step on its own (for numerics tests
 * and timing): Y[rows][n] = bf16(X[rows][k] W[n][k]^T) with f32 accumulation
 * on the tcgen05 kernel; gelu != 0 applies GELU-tanh to the bf16-rounded
 * product; splits > 1 splits K and writes the f32 partial sums to
 * partial[splits][rows][n] instead of Y (Y untouched).  n a multiple of 128,
 * k of 64 * splits; X, W, Y, partial 16-byte aligned device pointers.
 * Returns MTT_B200_STATUS_*. */
/* Measurement hooks (no reference counterpart).  cycles[c] of CTA c, 0 when
 * a bounded wait gave up.
 * umma_cycles: SM cycles for n_mma (a multiple of 16) back-to-back
 *   tcgen05.mma kind::f16 of M = 128, N = n (16..256, multiple of 16), K = 16
 *   into `accumulators` (a power of two, accumulators * n <= 512) TMEM
 *   accumulators, on `ctas` CTAs.
 * dsmem_cycles: SM cycles for `rounds` rounds in which every CTA of an 8-CTA
 *   cluster bulk-copies bytes_per_peer (16..16384, multiple of 16) of its
 *   shared memory into each of its 7 peers', on `clusters` clusters. */
MTT_B200_API int mtt_b200_test_umma_cycles(int32_t n, int32_t accumulators, int32_t n_mma, int32_t ctas,
                                           uint64_t* cycles, void* stream);
MTT_B200_API int mtt_b200_test_dsmem_cycles(int32_t bytes_per_peer, int32_t rounds, int32_t clusters,
                                            uint64_t* cycles, void* stream);

/* Trace hook: while `stamps` is non-null, every frame launched on the fused
 * cluster path or the quad path records, from CTA 0 of its first cluster,
 * the SM clock at 16 points of each position into stamps[16 * p + i], then
 * stamps[256..259] = clock and global timer (ns) at the frame's start and end.
 * Fused cluster path, i: 0 position start; 1 x ready; 2 q|k|v and partial
 * scores; 3 their round; 4 attention; 5 its round; 6 o-projection; 7 its
 * round; 8 LN2 + FFN1; 9 FFN2 partials; 10 their round; 11 FFN2 sum round;
 * 12 head; 13 logits round; 14 sampling; 15 token round.  Quad path, i:
 * 0 position start; 1 LN1 rows ready; 2 q|k|v; 3 attention; 4 its round;
 * 5 o-projection and its round; 6 LN2; 7 FFN1; 8 FFN2 partials sent; 9 their
 * round; 10 x'' and its round; 11 head; 12 values round; 13 sampling;
 * 14 token round; 15 next rows and their LN1.  `stamps` is a device buffer of
 * 260 entries; null turns the hook off.  Process-wide; for measurement only. */
MTT_B200_API int mtt_b200_test_frame_trace(uint64_t* stamps);

MTT_B200_API int mtt_b200_launch_test_gemm(const void* x_bf16, const void* w_bf16, void* y_bf16, int32_t rows,
                                           int32_t n, int32_t k, int32_t gelu, int32_t splits, float* partial,
                                           void* stream);

#ifdef __cplusplus
} /* extern "C" */

/* C++ forwarders under the reference's names (plugins/local_ar_plugins.hpp). */
#if defined(__CUDACC__) || defined(CUDART_VERSION) || defined(__CUDA_RUNTIME_API_H__)
#include <cstddef>
#include <cstdint>
namespace magpie_tts_rt::plugins {
[[nodiscard]] inline int launch_local_ar_sampling(
    const void* logits_bf16, const bool* unfinished, const bool* finished, const bool* forbid_eos,
    const std::int64_t* rng_seed, const std::int64_t* rng_counter, const void* embedding_weight_bf16,
    std::int64_t* sampled_token, void* next_embedding_bf16, std::int64_t* updated_rng_counter,
    std::int32_t* invalid_rows, cudaStream_t stream) noexcept {
  return mtt_b200_launch_local_ar_sampling(logits_bf16, unfinished, finished, forbid_eos, rng_seed,
                                           rng_counter, embedding_weight_bf16, sampled_token,
                                           next_embedding_bf16, updated_rng_counter, invalid_rows,
                                           static_cast<void*>(stream));
}
[[nodiscard]] inline std::size_t local_ar_eos_workspace_size() noexcept {
  return mtt_b200_local_ar_eos_workspace_size();
}
[[nodiscard]] inline int launch_local_ar_eos(const void* decoder_hidden_bf16, const std::int64_t* codec_tokens,
                                             const bool* unfinished, const bool* finished,
                                             const bool* forbid_eos, const void* final_weight_bf16,
                                             const void* final_bias_bf16, void* workspace,
                                             std::int32_t* end_frame_index, cudaStream_t stream) noexcept {
  return mtt_b200_launch_local_ar_eos(decoder_hidden_bf16, codec_tokens, unfinished, finished, forbid_eos,
                                      final_weight_bf16, final_bias_bf16, workspace, end_frame_index,
                                      static_cast<void*>(stream));
}
[[nodiscard]] inline int launch_layer_norm(const void* input_bf16, const void* weight_bf16, void* output_bf16,
                                           std::int32_t row_count, cudaStream_t stream) noexcept {
  return mtt_b200_launch_layer_norm(input_bf16, weight_bf16, output_bf16, row_count, static_cast<void*>(stream));
}
[[nodiscard]] inline int launch_gelu_tanh(const void* input_bf16, void* output_bf16, std::size_t element_count,
                                          cudaStream_t stream) noexcept {
  return mtt_b200_launch_gelu_tanh(input_bf16, output_bf16, element_count, static_cast<void*>(stream));
}
[[nodiscard]] inline int launch_softmax(const void* input_bf16, void* output_bf16, std::int32_t batch_count,
                                        std::int32_t element_count, cudaStream_t stream) noexcept {
  return mtt_b200_launch_softmax(input_bf16, output_bf16, batch_count, element_count, static_cast<void*>(stream));
}
}  // namespace magpie_tts_rt::plugins
#endif
#endif /* __cplusplus */

#endif /* MAGPIE_TTS_RT_B200_H_ */
