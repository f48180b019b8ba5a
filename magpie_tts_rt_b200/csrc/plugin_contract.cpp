// The five plugins' contracts (plugin_contract.hpp).  Shapes and types follow
// the reference's onShapeChange / supportsFormatCombination checks
// (plugins/local_ar_plugins.cu:1497-1600 shape predicates, :1849-1960
// sampling, :2053-2148 EOS, :2200-2560 LayerNorm / GeluTanh, :3410-3880
// Softmax); enqueue calls this library's launchers.
#include "plugin_contract.hpp"

#include <cstring>
#include <initializer_list>

#include "../../include/magpie_tts_rt_b200.h"

namespace mtt {
namespace plugin {
namespace {

constexpr int64_t kVocab = 2024;
constexpr int64_t kEmbed = 768;
constexpr int64_t kPositions = 16;
constexpr int64_t kCodebooks = 8;
constexpr int64_t kFrames = 2;
constexpr int64_t kFfnWidth = 3072;     // the accepted model's FFN width
constexpr int64_t kHeads = 12;          // its attention heads
constexpr int64_t kMaxText = 512;
constexpr int64_t kDecoderRows = 2;     // CFG pair
constexpr int64_t kPrefill = 218;
constexpr int64_t kCacheCapacity = 467;
constexpr int64_t kCrossHeads = 1;

bool dims_are(const Dims& d, std::initializer_list<int64_t> want) {
  if (d.nb != static_cast<int32_t>(want.size())) return false;
  int i = 0;
  for (const int64_t w : want) {
    if (d.d[i++] != w) return false;
  }
  return true;
}

Dims make_dims(std::initializer_list<int64_t> v) {
  Dims d;
  d.nb = static_cast<int32_t>(v.size());
  int i = 0;
  for (const int64_t x : v) d.d[i++] = x;
  return d;
}

OutputShape constant(std::initializer_list<int64_t> v) {
  OutputShape s;
  s.dims = make_dims(v);
  return s;
}

OutputShape like_input(int i) {
  OutputShape s;
  s.like = i;
  return s;
}

bool in_range(int64_t v, int64_t lo, int64_t hi) { return v >= lo && v <= hi; }

// ---------------------------------------------------------------------------

class Sampling final : public Contract {
 public:
  const char* name() const override { return "MagpieLocalARSampling"; }
  int inputs() const override { return 7; }
  int outputs() const override { return 4; }
  DType type(int p) const override {
    static constexpr DType t[11] = {DType::kBF16,  DType::kBool,  DType::kBool, DType::kBool,
                                    DType::kInt64, DType::kInt64, DType::kBF16, DType::kInt64,
                                    DType::kBF16,  DType::kInt64, DType::kInt32};
    return p >= 0 && p < 11 ? t[p] : DType::kOther;
  }
  bool shapes_ok(const Dims* in, int n) const override {
    return n == 7 && dims_are(in[0], {2, kVocab}) && dims_are(in[1], {1}) && dims_are(in[2], {1}) &&
           dims_are(in[3], {1}) && dims_are(in[4], {1}) && dims_are(in[5], {1}) && dims_are(in[6], {kVocab, kEmbed});
  }
  OutputShape output_shape(int o) const override {
    return o == 1 ? constant({2, kEmbed}) : constant({1});
  }
  int32_t enqueue(const Dims*, const void* const* in, void* const* out, void*, void* stream) const override {
    return mtt_b200_launch_local_ar_sampling(
        in[0], static_cast<const bool*>(in[1]), static_cast<const bool*>(in[2]), static_cast<const bool*>(in[3]),
        static_cast<const int64_t*>(in[4]), static_cast<const int64_t*>(in[5]), in[6], static_cast<int64_t*>(out[0]),
        out[1], static_cast<int64_t*>(out[2]), static_cast<int32_t*>(out[3]), stream);
  }
};

class Eos final : public Contract {
 public:
  const char* name() const override { return "MagpieLocalAREos"; }
  int inputs() const override { return 7; }
  int outputs() const override { return 1; }
  DType type(int p) const override {
    static constexpr DType t[8] = {DType::kBF16, DType::kInt64, DType::kBool, DType::kBool,
                                   DType::kBool, DType::kBF16,  DType::kBF16, DType::kInt32};
    return p >= 0 && p < 8 ? t[p] : DType::kOther;
  }
  bool shapes_ok(const Dims* in, int n) const override {
    return n == 7 && dims_are(in[0], {2, kEmbed}) && dims_are(in[1], {1, kCodebooks, kFrames}) &&
           dims_are(in[2], {1}) && dims_are(in[3], {1}) && dims_are(in[4], {1}) &&
           dims_are(in[5], {kPositions * kVocab, kEmbed}) && dims_are(in[6], {kPositions * kVocab});
  }
  OutputShape output_shape(int) const override { return constant({1}); }
  size_t workspace_bytes() const override { return mtt_b200_local_ar_eos_workspace_size(); }
  int32_t enqueue(const Dims*, const void* const* in, void* const* out, void* ws, void* stream) const override {
    return mtt_b200_launch_local_ar_eos(in[0], static_cast<const int64_t*>(in[1]), static_cast<const bool*>(in[2]),
                                        static_cast<const bool*>(in[3]), static_cast<const bool*>(in[4]), in[5], in[6],
                                        ws, static_cast<int32_t*>(out[0]), stream);
  }
};

// LayerNorm over rows of 768: the Local AR's [2, 1, 768], the text encoder's
// [1, T, 768] and the Main Decoder prefill's [2, T, 768], T <= 512.
class LayerNorm final : public Contract {
 public:
  const char* name() const override { return "MagpieLayerNorm"; }
  int inputs() const override { return 2; }
  int outputs() const override { return 1; }
  DType type(int p) const override { return p >= 0 && p < 3 ? DType::kBF16 : DType::kOther; }
  static bool input_ok(const Dims& d) {
    if (d.nb != 3 || d.d[2] != kEmbed) return false;
    return (d.d[0] == 2 && d.d[1] == 1) || (d.d[0] == 1 && in_range(d.d[1], 1, kMaxText)) ||
           (d.d[0] == kDecoderRows && in_range(d.d[1], 1, kMaxText));
  }
  bool shapes_ok(const Dims* in, int n) const override {
    return n == 2 && input_ok(in[0]) && dims_are(in[1], {kEmbed});
  }
  OutputShape output_shape(int) const override { return like_input(0); }
  int32_t enqueue(const Dims* dims, const void* const* in, void* const* out, void*, void* stream) const override {
    if (dims == nullptr || !input_ok(dims[0])) return -1;
    return mtt_b200_launch_layer_norm(in[0], in[1], out[0], static_cast<int32_t>(dims[0].d[0] * dims[0].d[1]), stream);
  }
};

// GELU-tanh on [rows, 3072, T] activations: the Local AR's [2, 3072, 1], the
// text encoder's [1, 3072, T <= 512], the decoder prefill's [2, 3072, T <= 218].
class GeluTanh final : public Contract {
 public:
  const char* name() const override { return "MagpieGeluTanh"; }
  int inputs() const override { return 1; }
  int outputs() const override { return 1; }
  DType type(int p) const override { return p >= 0 && p < 2 ? DType::kBF16 : DType::kOther; }
  static bool input_ok(const Dims& d) {
    if (d.nb != 3 || d.d[1] != kFfnWidth) return false;
    return (d.d[0] == 2 && d.d[2] == 1) || (d.d[0] == 1 && in_range(d.d[2], 1, kMaxText)) ||
           (d.d[0] == kDecoderRows && in_range(d.d[2], 1, kPrefill));
  }
  bool shapes_ok(const Dims* in, int n) const override { return n == 1 && input_ok(in[0]); }
  OutputShape output_shape(int) const override { return like_input(0); }
  int32_t enqueue(const Dims* dims, const void* const* in, void* const* out, void*, void* stream) const override {
    if (dims == nullptr || !input_ok(dims[0])) return -1;
    const size_t count = static_cast<size_t>(dims[0].d[0] * dims[0].d[1] * dims[0].d[2]);
    return mtt_b200_launch_gelu_tanh(in[0], out[0], count, stream);
  }
};

// Softmax mode 0 over the last dimension of [B, H, Q, K] attention scores:
// the Local AR's [2, 12, 1, K <= 16], the text encoder's [1, 12, T, T], the
// decoder prefill's self [2, 12, 218, 218] / cross [2, 1, 218, K] and step
// self [2, 12, 1, 219..467] / cross [2, 1, 1, K] shapes, K <= 512.
class Softmax final : public Contract {
 public:
  const char* name() const override { return "MagpieSoftmax"; }
  int inputs() const override { return 1; }
  int outputs() const override { return 1; }
  DType type(int p) const override { return p >= 0 && p < 2 ? DType::kBF16 : DType::kOther; }
  static bool input_ok(const Dims& d) {
    if (d.nb != 4 || !in_range(d.d[3], 1, kMaxText)) return false;
    const bool local = d.d[0] == kDecoderRows && d.d[1] == kHeads && d.d[2] == 1 && d.d[3] <= kPositions;
    const bool text = d.d[0] == 1 && d.d[1] == kHeads && d.d[2] == d.d[3];
    const bool prefill_self = d.d[0] == kDecoderRows && d.d[1] == kHeads && d.d[2] == kPrefill && d.d[3] == kPrefill;
    const bool prefill_cross = d.d[0] == kDecoderRows && d.d[1] == kCrossHeads && d.d[2] == kPrefill;
    const bool step_self = d.d[0] == kDecoderRows && d.d[1] == kHeads && d.d[2] == 1 &&
                           in_range(d.d[3], kPrefill + 1, kCacheCapacity);
    const bool step_cross = d.d[0] == kDecoderRows && d.d[1] == kCrossHeads && d.d[2] == 1;
    return local || text || prefill_self || prefill_cross || step_self || step_cross;
  }
  bool shapes_ok(const Dims* in, int n) const override { return n == 1 && input_ok(in[0]); }
  OutputShape output_shape(int) const override { return like_input(0); }
  int32_t enqueue(const Dims* dims, const void* const* in, void* const* out, void*, void* stream) const override {
    if (dims == nullptr || !input_ok(dims[0])) return -1;
    const int64_t rows = dims[0].d[0] * dims[0].d[1] * dims[0].d[2];
    return mtt_b200_launch_softmax(in[0], out[0], static_cast<int32_t>(rows), static_cast<int32_t>(dims[0].d[3]),
                                   stream);
  }
};

const Sampling g_sampling;
const Eos g_eos;
const LayerNorm g_layer_norm;
const GeluTanh g_gelu;
const Softmax g_softmax;
const Contract* const g_contracts[] = {&g_sampling, &g_eos, &g_layer_norm, &g_gelu, &g_softmax};

}  // namespace

int contract_count() { return static_cast<int>(sizeof(g_contracts) / sizeof(g_contracts[0])); }

const Contract* contract_at(int i) { return i >= 0 && i < contract_count() ? g_contracts[i] : nullptr; }

const Contract* find_contract(const char* name) {
  if (name == nullptr) return nullptr;
  for (const Contract* c : g_contracts) {
    if (std::strcmp(c->name(), name) == 0) return c;
  }
  return nullptr;
}

bool fields_ok(const Contract* c, const Field* fields, int n_fields) {
  if (c == nullptr || n_fields < 0 || (n_fields > 0 && fields == nullptr)) return false;
  if (c != &g_softmax) return n_fields == 0;
  // MagpieSoftmax: optional "mode" and "layer_index", each once, int32 x 1
  int32_t mode = 0, layer_index = -1;
  bool mode_seen = false, layer_seen = false;
  if (n_fields > 2) return false;
  for (int i = 0; i < n_fields; ++i) {
    const Field& f = fields[i];
    if (f.name == nullptr || !f.int32_type || f.length != 1 || f.data == nullptr) return false;
    int32_t v;
    std::memcpy(&v, f.data, sizeof(v));
    if (std::strcmp(f.name, "mode") == 0 && !mode_seen) {
      mode = v;
      mode_seen = true;
    } else if (std::strcmp(f.name, "layer_index") == 0 && !layer_seen) {
      layer_index = v;
      layer_seen = true;
    } else {
      return false;
    }
  }
  return mode == 0 && layer_index == -1;
}

}  // namespace plugin
}  // namespace mtt
