// The five TensorRT plugins' tensor contracts, independent of TensorRT.
//
// The reference registers five IPluginV3 creators (MagpieLocalARSampling,
// MagpieLocalAREos, MagpieLayerNorm, MagpieGeluTanh, MagpieSoftmax; version
// "1", namespace "magpie_tts_rt"; plugins/local_ar_plugins.cu:1805-2180,
// 2200-2560, 3410-3880) whose I/O contract is fixed by the exported engines
// (docs/engine-contracts.md:186-316).  Here each plugin's contract is data:
// input and output element types, the accepted input shapes (the
// onShapeChange checks), the output shapes (constants or an input's shape),
// the workspace size, and the enqueue as a call of this library's launcher.
// trt_plugins.cpp wraps one generic IPluginV3 class around this table when
// TensorRT's headers are present; the table itself is compiled everywhere and
// tested on the CPU.
#pragma once

#include <cstddef>
#include <cstdint>

namespace mtt {
namespace plugin {

// Element types (mapped one by one from nvinfer1::DataType in the TensorRT
// layer; the numeric values are this file's own).
enum class DType : int32_t { kFloat, kHalf, kBF16, kInt8, kInt32, kInt64, kBool, kUInt8, kOther };

constexpr int kMaxDims = 8;
constexpr int kMaxTensors = 16;

struct Dims {
  int32_t nb = 0;
  int64_t d[kMaxDims] = {};
};

// An output shape: the dims of input `like` (like >= 0) or the constant dims.
struct OutputShape {
  int like = -1;
  Dims dims;
};

class Contract {
 public:
  virtual ~Contract() = default;
  virtual const char* name() const = 0;
  virtual int inputs() const = 0;
  virtual int outputs() const = 0;
  // Type of tensor `position` (inputs first, then outputs); every tensor is
  // linear (row-major, no vectorised format).
  virtual DType type(int position) const = 0;
  // The accepted input shapes (onShapeChange); false rejects the binding.
  virtual bool shapes_ok(const Dims* in, int n_in) const = 0;
  virtual OutputShape output_shape(int o) const = 0;
  virtual size_t workspace_bytes() const { return 0; }
  // Runs the plugin on device buffers, stream-ordered; 0 or -1 (a null
  // pointer, a shape outside the contract or a failed launch).
  virtual int32_t enqueue(const Dims* in_dims, const void* const* in, void* const* out, void* workspace,
                          void* stream) const = 0;

  // supportsFormatCombination: the type at `position` and a linear format.
  bool supports(int position, DType t, bool linear, int n_in, int n_out) const {
    if (n_in != inputs() || n_out != outputs() || position < 0 || position >= n_in + n_out) return false;
    return linear && t == type(position);
  }
};

// Plugin fields: the four fixed-contract plugins take none; MagpieSoftmax
// takes "mode" and "layer_index" (int32, one element each).  Mode 0 (the
// plain row softmax) is this library's; the reference's Main Decoder modes
// 1..8 belong to its decoder engines, which this library replaces by
// mtt_b200_launch_main_decoder_step, so a creator asked for them refuses.
struct Field {
  const char* name;
  const void* data;
  int32_t length;
  bool int32_type;
};

// The contracts in the reference's creator order.
int contract_count();
const Contract* contract_at(int i);
const Contract* find_contract(const char* name);

// Validates a creator's fields for `c` (createPlugin): true when the plugin
// can be created.
bool fields_ok(const Contract* c, const Field* fields, int n_fields);

constexpr const char* kVersion = "1";
constexpr const char* kNamespace = "magpie_tts_rt";

}  // namespace plugin
}  // namespace mtt
