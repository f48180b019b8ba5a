// Per-GPU session engine: the C++ host side of the per-step loop (the C ABI
// in section 6 of include/magpie_tts_rt_b200.h).
//
// The reference drives one session per request thread: every decoder step it
// copies `unfinished` device to device and uploads forbid_eos from pageable
// host memory, launches the session's Local AR CUDA graph, then
// launch_finalize_local_step (src/runtime/synthesis_pipeline.cpp:511-569;
// graphs captured per session, src/runtime/session_resources.cpp:661-684).
// Here one engine per GPU holds the state of all its sessions as
// structure-of-arrays device buffers and runs one step for all of them as one
// CUDA graph on its own stream:
//   [Main Decoder step ->] alignment gate -> Local AR frame [-> position + 1]
// The gate produces the frame's unfinished / forbid_eos / finished inputs on
// the device, the frame folds finalize_local_step, and the decoder's hidden
// state, alignment scores, prior and embedding sum are shared buffers, so no
// step copies anything between host and device.  Opening or closing a
// session writes its slot with one small kernel on the same stream; the
// graph reads the slot's `active` flag, so it never needs to be re-captured.
#include <cuda_runtime.h>

#include <cstring>
#include <new>
#include <vector>

#include "../../include/magpie_tts_rt_b200.h"
#include "common.cuh"

namespace {

constexpr int kEmbedW = 768;
constexpr int kDecLayersMin = 10;
constexpr int kSelfHeads = 12;
constexpr int kSelfDim = 64;
constexpr int kCrossDim = 128;

using bf16 = __nv_bfloat16;

// Slot state at open: RNG, flags, outputs, alignment state, prior (ones), and
// with the decoder the position, empty cache mask, text mask and first input.
struct OpenArgs {
  int slot, S, cap, with_decoder;
  int64_t seed;
  uint32_t text_length;
  const bf16* initial_embedding;
};

struct Slots {
  int n, S, cap, L;
  bool *active, *unfinished, *finished, *forbid;
  int64_t *seed, *counter, *codec, *attended, *steps, *position;
  int32_t *invalid, *end, *invalid_state, *status;
  uint32_t *text_length, *counters, *last_attended;
  bf16 *prior, *embedding;
  bool *self_mask, *cond_mask;
};

__global__ void open_slot_kernel(Slots st, OpenArgs a) {
  const int s = a.slot;
  const int t = threadIdx.x;
  if (t == 0) {
    st.active[s] = true;
    st.unfinished[s] = true;
    st.finished[s] = false;
    st.forbid[s] = true;
    st.seed[s] = a.seed;
    st.counter[s] = 0;
    st.invalid[s] = 0;
    st.end[s] = -1;
    st.text_length[s] = a.text_length;
    st.last_attended[s] = 1;
    st.attended[s] = 0;
    st.invalid_state[s] = 0;
    st.steps[s] = 0;
    if (a.with_decoder) {
      st.position[s] = 0;
      st.status[s] = 0;
    }
  }
  for (int i = t; i < 16; i += blockDim.x) st.codec[static_cast<int64_t>(s) * 16 + i] = 0;
  for (int i = t; i < a.S; i += blockDim.x) st.counters[static_cast<int64_t>(s) * a.S + i] = 0;
  for (int i = t; i < 2 * a.S; i += blockDim.x) st.prior[static_cast<int64_t>(s) * 2 * a.S + i] = __float2bfloat16(1.0f);
  for (int i = t; i < kEmbedW; i += blockDim.x) {
    st.embedding[static_cast<int64_t>(s) * kEmbedW + i] =
        a.initial_embedding != nullptr ? a.initial_embedding[i] : __float2bfloat16(0.0f);
  }
  if (a.with_decoder) {
    for (int i = t; i < 2 * a.cap; i += blockDim.x) st.self_mask[static_cast<int64_t>(s) * 2 * a.cap + i] = false;
    for (int i = t; i < 2 * a.S; i += blockDim.x) st.cond_mask[static_cast<int64_t>(s) * 2 * a.S + i] = false;
  }
}

__global__ void close_slot_kernel(bool* active, int slot) { active[slot] = false; }

// The decoder's next position for every open session (the step graph's last node).
__global__ void advance_positions_kernel(int64_t* position, const bool* active, int n) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < n && active[s]) position[s] += 1;
}

}  // namespace

struct mtt_b200_session_engine {
  mtt_b200_session_engine_config_t cfg{};
  int device = -1;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocations;
  Slots slots{};
  mtt_b200_stream_batch_t frame{};
  mtt_b200_alignment_batch_t gate{};
  mtt_b200_main_decoder_batch_t dec{};
  mtt_b200_local_ar_weights_t lw{};
  void* frame_ws = nullptr;
  size_t frame_ws_bytes = 0;
  void* dec_ws = nullptr;
  size_t dec_ws_bytes = 0;
  int steps_done = 0;
  cudaGraphExec_t graph = nullptr;

  template <typename T>
  T* alloc(size_t count) {
    void* p = nullptr;
    if (cudaMalloc(&p, count * sizeof(T)) != cudaSuccess) return nullptr;
    allocations.push_back(p);
    if (cudaMemsetAsync(p, 0, count * sizeof(T), stream) != cudaSuccess) return nullptr;
    return static_cast<T*>(p);
  }

  // One step's launches on `stream` (eagerly, or while it is being captured).
  int enqueue_step() {
    if (cfg.with_decoder) {
      const int rc = mtt_b200_launch_main_decoder_step(&cfg.decoder, &dec, dec_ws, dec_ws_bytes, stream);
      if (rc != MTT_B200_STATUS_OK) return rc;
    }
    int rc = mtt_b200_launch_alignment_batch(&gate, stream);
    if (rc != MTT_B200_STATUS_OK) return rc;
    rc = mtt_b200_launch_local_ar_frame(&cfg.shape, &lw, &cfg.sampling, &frame, frame_ws, frame_ws_bytes, stream);
    if (rc != MTT_B200_STATUS_OK) return rc;
    if (cfg.with_decoder) {
      advance_positions_kernel<<<(slots.n + 255) / 256, 256, 0, stream>>>(slots.position, slots.active, slots.n);
      if (cudaGetLastError() != cudaSuccess) return MTT_B200_STATUS_CUDA_ERROR;
    }
    return MTT_B200_STATUS_OK;
  }

  ~mtt_b200_session_engine() {
    int previous = -1;
    cudaGetDevice(&previous);
    if (device >= 0) cudaSetDevice(device);
    if (stream != nullptr) cudaStreamSynchronize(stream);
    if (graph != nullptr) cudaGraphExecDestroy(graph);
    for (void* p : allocations) cudaFree(p);
    if (stream != nullptr) cudaStreamDestroy(stream);
    if (previous >= 0) cudaSetDevice(previous);
  }
};

namespace {

bool config_ok(const mtt_b200_session_engine_config_t* c) {
  if (c == nullptr || c->max_sessions <= 0 || c->token_stride <= 0 || c->token_stride > 512 ||
      c->token_stride % 8 != 0 || c->lookahead == 0 || c->sink_threshold == 0) {
    return false;
  }
  if (c->with_decoder && (c->cache_capacity <= 0 || c->decoder.n_layers < kDecLayersMin ||
                          c->decoder.pos_rows < c->cache_capacity)) {
    return false;
  }
  return true;
}

}  // namespace

extern "C" MTT_B200_API int mtt_b200_session_engine_create(const mtt_b200_session_engine_config_t* config,
                                                          mtt_b200_session_engine_t** engine) {
  if (engine == nullptr) return MTT_B200_STATUS_INVALID_ARGUMENT;
  *engine = nullptr;
  if (!config_ok(config)) return MTT_B200_STATUS_INVALID_ARGUMENT;
  auto* e = new (std::nothrow) mtt_b200_session_engine();
  if (e == nullptr) return MTT_B200_STATUS_CUDA_ERROR;
  e->cfg = *config;
  const int n = config->max_sessions, S = config->token_stride;
  auto fail = [&](int rc) {
    delete e;
    return rc;
  };
  if (cudaGetDevice(&e->device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    return fail(MTT_B200_STATUS_CUDA_ERROR);
  }
  const int rows = config->sampling.cfg ? 2 : 1;
  Slots& st = e->slots;
  st.n = n;
  st.S = S;
  st.cap = config->with_decoder ? config->cache_capacity : 0;
  st.L = config->with_decoder ? config->decoder.n_layers : 0;
  bf16* hidden = config->decoder_hidden != nullptr ? static_cast<bf16*>(config->decoder_hidden)
                                                   : e->alloc<bf16>(static_cast<size_t>(n) * rows * kEmbedW);
  bf16* scores = config->alignment_scores != nullptr ? static_cast<bf16*>(config->alignment_scores)
                                                     : e->alloc<bf16>(static_cast<size_t>(n) * 2 * S);
  st.active = e->alloc<bool>(n);
  st.unfinished = e->alloc<bool>(n);
  st.finished = e->alloc<bool>(n);
  st.forbid = e->alloc<bool>(n);
  st.seed = e->alloc<int64_t>(n);
  st.counter = e->alloc<int64_t>(n);
  st.codec = e->alloc<int64_t>(static_cast<size_t>(n) * 16);
  st.attended = e->alloc<int64_t>(n);
  st.steps = e->alloc<int64_t>(n);
  st.invalid = e->alloc<int32_t>(n);
  st.end = e->alloc<int32_t>(n);
  st.invalid_state = e->alloc<int32_t>(n);
  st.text_length = e->alloc<uint32_t>(n);
  st.counters = e->alloc<uint32_t>(static_cast<size_t>(n) * S);
  st.last_attended = e->alloc<uint32_t>(n);
  st.prior = e->alloc<bf16>(static_cast<size_t>(n) * 2 * S);
  st.embedding = config->next_embedding != nullptr ? static_cast<bf16*>(config->next_embedding)
                                                   : e->alloc<bf16>(static_cast<size_t>(n) * kEmbedW);
  if (!hidden || !scores || !st.active || !st.unfinished || !st.finished || !st.forbid || !st.seed || !st.counter ||
      !st.codec || !st.attended || !st.steps || !st.invalid || !st.end || !st.invalid_state || !st.text_length ||
      !st.counters || !st.last_attended || !st.prior || !st.embedding ||
      cudaMemsetAsync(st.end, 0xff, static_cast<size_t>(n) * sizeof(int32_t), e->stream) != cudaSuccess) {  // -1: no EOS
    return fail(MTT_B200_STATUS_CUDA_ERROR);
  }
  // Local AR weights: fold the in-projection into the embedding tables once
  e->lw = config->local_ar;
  if (config->shape.d_model != kEmbedW && e->lw.emb_proj == nullptr) {
    const size_t fold = mtt_b200_fold_in_projection_bytes(&config->shape);
    void* table = e->alloc<unsigned char>(fold);
    if (table == nullptr || mtt_b200_launch_fold_in_projection(&config->shape, &e->lw, table, e->stream) !=
                                MTT_B200_STATUS_OK) {
      return fail(MTT_B200_STATUS_CUDA_ERROR);
    }
    e->lw.emb_proj = table;
  }
  e->frame_ws_bytes = mtt_b200_local_ar_frame_workspace_size(&config->shape, n, config->sampling.cfg);
  e->frame_ws = e->alloc<unsigned char>(e->frame_ws_bytes);
  if (e->frame_ws_bytes == 0 || e->frame_ws == nullptr) return fail(MTT_B200_STATUS_INVALID_ARGUMENT);
  // the frame batch
  mtt_b200_stream_batch_t& f = e->frame;
  f.n_streams = n;
  f.decoder_hidden = hidden;
  f.unfinished = st.unfinished;
  f.finished = st.finished;
  f.forbid_eos = st.forbid;
  f.active = st.active;
  f.rng_seed = st.seed;
  f.rng_counter = st.counter;
  f.codec_tokens = st.codec;
  f.invalid_rows = st.invalid;
  f.end_frame_index = st.end;
  f.next_embedding = st.embedding;
  f.finished_latch = st.finished;
  // the alignment gate, writing the frame's EOS inputs
  mtt_b200_alignment_batch_t& g = e->gate;
  g.n_sessions = n;
  g.token_stride = static_cast<uint32_t>(S);
  g.ignored_terminal_tokens = config->ignored_terminal_tokens;
  g.short_text_no_prior_max_tokens = config->short_text_no_prior_max_tokens;
  g.lookahead = config->lookahead;
  g.sink_threshold = config->sink_threshold;
  g.text_length = st.text_length;
  g.active = st.active;
  g.alignment_scores = scores;
  g.counters = st.counters;
  g.last_attended = st.last_attended;
  g.next_prior = st.prior;
  g.attended_token_index = st.attended;
  g.unfinished = st.unfinished;
  g.invalid_state = st.invalid_state;
  g.decoder_steps = st.steps;
  g.forbid_eos = st.forbid;
  g.end_frame_index = st.end;
  g.finished = st.finished;
  if (config->with_decoder) {
    const size_t L = static_cast<size_t>(config->decoder.n_layers), cap = static_cast<size_t>(config->cache_capacity);
    st.position = e->alloc<int64_t>(n);
    st.status = e->alloc<int32_t>(n);
    st.self_mask = e->alloc<bool>(static_cast<size_t>(n) * 2 * cap);
    st.cond_mask = e->alloc<bool>(static_cast<size_t>(n) * 2 * S);
    bf16* self_k = e->alloc<bf16>(static_cast<size_t>(n) * L * 2 * kSelfHeads * cap * kSelfDim);
    bf16* self_v = e->alloc<bf16>(static_cast<size_t>(n) * L * 2 * kSelfHeads * cap * kSelfDim);
    bf16* cross_k = e->alloc<bf16>(static_cast<size_t>(n) * L * 2 * S * kCrossDim);
    bf16* cross_v = e->alloc<bf16>(static_cast<size_t>(n) * L * 2 * S * kCrossDim);
    e->dec_ws_bytes = mtt_b200_main_decoder_workspace_size(n, S);
    e->dec_ws = e->alloc<unsigned char>(e->dec_ws_bytes);
    if (!st.position || !st.status || !st.self_mask || !st.cond_mask || !self_k || !self_v || !cross_k || !cross_v ||
        e->dec_ws == nullptr) {
      return fail(MTT_B200_STATUS_CUDA_ERROR);
    }
    mtt_b200_main_decoder_batch_t& d = e->dec;
    d.n_sessions = n;
    d.cache_capacity = config->cache_capacity;
    d.token_stride = S;
    d.embedded = st.embedding;  // the frame's embedding sum is the next decoder input
    d.position = st.position;
    d.text_length = st.text_length;
    d.active = st.active;
    d.self_k = self_k;
    d.self_v = self_v;
    d.self_mask = st.self_mask;
    d.cross_k = cross_k;
    d.cross_v = cross_v;
    d.cond_mask = st.cond_mask;
    d.prior = st.prior;          // the gate's next prior
    d.hidden = hidden;           // the frame's input
    d.alignment = scores;        // the gate's input
    d.status = st.status;
    d.eos_cfg_scale = config->sampling.cfg_scale;
  }
  if (cudaStreamSynchronize(e->stream) != cudaSuccess) return fail(MTT_B200_STATUS_CUDA_ERROR);
  *engine = e;
  return MTT_B200_STATUS_OK;
}

extern "C" MTT_B200_API void mtt_b200_session_engine_destroy(mtt_b200_session_engine_t* engine) { delete engine; }

extern "C" MTT_B200_API int mtt_b200_session_engine_buffers(const mtt_b200_session_engine_t* e,
                                                           mtt_b200_session_engine_buffers_t* b) {
  if (e == nullptr || b == nullptr) return MTT_B200_STATUS_INVALID_ARGUMENT;
  b->stream = e->stream;
  b->decoder_hidden = const_cast<void*>(e->frame.decoder_hidden);
  b->alignment_scores = const_cast<void*>(e->gate.alignment_scores);
  b->next_embedding = e->frame.next_embedding;
  b->codec_tokens = e->slots.codec;
  b->end_frame_index = e->slots.end;
  b->invalid_rows = e->slots.invalid;
  b->rng_counter = e->slots.counter;
  b->finished = e->slots.finished;
  b->position = e->slots.position;
  b->decoder_status = e->slots.status;
  return MTT_B200_STATUS_OK;
}

extern "C" MTT_B200_API int mtt_b200_session_engine_open(mtt_b200_session_engine_t* e, int32_t slot, int64_t seed,
                                                        uint32_t text_length, const void* cross_k,
                                                        const void* cross_v, const bool* cond_mask,
                                                        const void* initial_embedding) {
  if (e == nullptr || slot < 0 || slot >= e->slots.n || text_length < 1 ||
      text_length > static_cast<uint32_t>(e->slots.S)) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  const bool dec = e->cfg.with_decoder != 0;
  if (dec && (cross_k == nullptr || cross_v == nullptr || cond_mask == nullptr)) return MTT_B200_STATUS_INVALID_ARGUMENT;
  OpenArgs a{slot, e->slots.S, e->slots.cap, dec ? 1 : 0, seed, text_length,
             static_cast<const bf16*>(initial_embedding)};
  open_slot_kernel<<<1, 256, 0, e->stream>>>(e->slots, a);
  if (cudaGetLastError() != cudaSuccess) return MTT_B200_STATUS_CUDA_ERROR;
  if (dec) {
    // the prefill's [L][2][T][128] text keys / values into the slot's [L][2][S][128]
    const size_t row = static_cast<size_t>(text_length) * kCrossDim * sizeof(bf16);
    const size_t pitch = static_cast<size_t>(e->slots.S) * kCrossDim * sizeof(bf16);
    const size_t slot_elems = static_cast<size_t>(e->slots.L) * 2 * e->slots.S * kCrossDim;
    bf16* dk = static_cast<bf16*>(const_cast<void*>(e->dec.cross_k)) + slot_elems * slot;
    bf16* dv = static_cast<bf16*>(const_cast<void*>(e->dec.cross_v)) + slot_elems * slot;
    bool* dm = e->slots.cond_mask + static_cast<size_t>(2) * e->slots.S * slot;
    if (cudaMemcpy2DAsync(dk, pitch, cross_k, row, row, 2 * e->slots.L, cudaMemcpyDeviceToDevice, e->stream) !=
            cudaSuccess ||
        cudaMemcpy2DAsync(dv, pitch, cross_v, row, row, 2 * e->slots.L, cudaMemcpyDeviceToDevice, e->stream) !=
            cudaSuccess ||
        cudaMemcpy2DAsync(dm, e->slots.S, cond_mask, text_length, text_length, 2, cudaMemcpyDeviceToDevice,
                          e->stream) != cudaSuccess) {
      return MTT_B200_STATUS_CUDA_ERROR;
    }
  }
  return MTT_B200_STATUS_OK;
}

extern "C" MTT_B200_API int mtt_b200_session_engine_close(mtt_b200_session_engine_t* e, int32_t slot) {
  if (e == nullptr || slot < 0 || slot >= e->slots.n) return MTT_B200_STATUS_INVALID_ARGUMENT;
  close_slot_kernel<<<1, 1, 0, e->stream>>>(e->slots.active, slot);
  return cudaGetLastError() == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
}

extern "C" MTT_B200_API int mtt_b200_session_engine_step(mtt_b200_session_engine_t* e) {
  if (e == nullptr) return MTT_B200_STATUS_INVALID_ARGUMENT;
  int rc = MTT_B200_STATUS_OK;
  if (e->graph != nullptr) {
    return cudaGraphLaunch(e->graph, e->stream) == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
  }
  if (e->steps_done == 0) {
    // the first step runs eagerly: it makes the libraries' one-time set-up
    // (kernel attributes per device) outside any capture
    rc = e->enqueue_step();
  } else {
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      return MTT_B200_STATUS_CUDA_ERROR;
    }
    rc = e->enqueue_step();
    const cudaError_t end = cudaStreamEndCapture(e->stream, &g);
    if (rc != MTT_B200_STATUS_OK || end != cudaSuccess || g == nullptr) {
      if (g != nullptr) cudaGraphDestroy(g);
      cudaGetLastError();
      return rc != MTT_B200_STATUS_OK ? rc : MTT_B200_STATUS_CUDA_ERROR;
    }
    const cudaError_t inst = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    if (inst != cudaSuccess) {
      e->graph = nullptr;
      return MTT_B200_STATUS_CUDA_ERROR;
    }
    rc = cudaGraphLaunch(e->graph, e->stream) == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
  }
  if (rc == MTT_B200_STATUS_OK) ++e->steps_done;
  return rc;
}

extern "C" MTT_B200_API int mtt_b200_session_engine_collect(mtt_b200_session_engine_t* e, int32_t n,
                                                           int64_t* codec_tokens, int32_t* end_frame_index,
                                                           int32_t* invalid_rows) {
  if (e == nullptr || n < 0 || n > e->slots.n) return MTT_B200_STATUS_INVALID_ARGUMENT;
  const size_t nn = static_cast<size_t>(n);
  if ((codec_tokens != nullptr && cudaMemcpyAsync(codec_tokens, e->slots.codec, nn * 16 * sizeof(int64_t),
                                                  cudaMemcpyDeviceToHost, e->stream) != cudaSuccess) ||
      (end_frame_index != nullptr && cudaMemcpyAsync(end_frame_index, e->slots.end, nn * sizeof(int32_t),
                                                     cudaMemcpyDeviceToHost, e->stream) != cudaSuccess) ||
      (invalid_rows != nullptr && cudaMemcpyAsync(invalid_rows, e->slots.invalid, nn * sizeof(int32_t),
                                                  cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)) {
    return MTT_B200_STATUS_CUDA_ERROR;
  }
  return cudaStreamSynchronize(e->stream) == cudaSuccess ? MTT_B200_STATUS_OK : MTT_B200_STATUS_CUDA_ERROR;
}
