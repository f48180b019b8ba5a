// TensorRT IPluginV3 layer over the plugin contracts (plugin_contract.hpp).
//
// Compiled when TensorRT's headers are available (a build defines
// MTT_B200_WITH_TENSORRT after finding NvInfer.h); without them this file is
// empty and the plugin ABI's register_plugins reports REGISTRY_UNAVAILABLE.
//
// One plugin class serves all five creators: every IPluginV3OneCore /
// OneBuild / OneRuntime method asks the plugin's Contract (names, tensor
// types and shapes, workspace, enqueue), so the five plugins differ only in
// their table entries.  Plugins are stateless: clone() and attachToContext()
// return a fresh plugin over the same contract (the reference's ownership
// rule, docs/engine-contracts.md:247-250).  The creators and the
// registration statuses follow plugins/local_ar_plugins.cu:3880-4104:
// ALREADY_REGISTERED when these five creators are the registered ones,
// REGISTRATION_CONFLICT when any creator of these names is already there (or
// appears while registering), REGISTRATION_FAILED when the registry refuses
// one; a failed registration takes back the creators it had added.
#if defined(MTT_B200_WITH_TENSORRT)

#include <NvInfer.h>

#include <array>
#include <cstring>
#include <mutex>
#include <new>

#include "../../include/magpie_tts_rt_b200.h"
#include "plugin_contract.hpp"

namespace mtt {
namespace plugin {
namespace {

DType to_dtype(nvinfer1::DataType t) {
  switch (t) {
    case nvinfer1::DataType::kFLOAT: return DType::kFloat;
    case nvinfer1::DataType::kHALF: return DType::kHalf;
    case nvinfer1::DataType::kBF16: return DType::kBF16;
    case nvinfer1::DataType::kINT8: return DType::kInt8;
    case nvinfer1::DataType::kINT32: return DType::kInt32;
    case nvinfer1::DataType::kINT64: return DType::kInt64;
    case nvinfer1::DataType::kBOOL: return DType::kBool;
    case nvinfer1::DataType::kUINT8: return DType::kUInt8;
    default: return DType::kOther;
  }
}

bool from_dtype(DType t, nvinfer1::DataType* out) {
  switch (t) {
    case DType::kFloat: *out = nvinfer1::DataType::kFLOAT; return true;
    case DType::kHalf: *out = nvinfer1::DataType::kHALF; return true;
    case DType::kBF16: *out = nvinfer1::DataType::kBF16; return true;
    case DType::kInt8: *out = nvinfer1::DataType::kINT8; return true;
    case DType::kInt32: *out = nvinfer1::DataType::kINT32; return true;
    case DType::kInt64: *out = nvinfer1::DataType::kINT64; return true;
    case DType::kBool: *out = nvinfer1::DataType::kBOOL; return true;
    case DType::kUInt8: *out = nvinfer1::DataType::kUINT8; return true;
    default: return false;
  }
}

bool to_dims(const nvinfer1::Dims& in, Dims* out) {
  if (in.nbDims < 0 || in.nbDims > kMaxDims) return false;
  out->nb = in.nbDims;
  for (int i = 0; i < in.nbDims; ++i) out->d[i] = in.d[i];
  return true;
}

class ContractPlugin final : public nvinfer1::IPluginV3,
                             public nvinfer1::IPluginV3OneCore,
                             public nvinfer1::IPluginV3OneBuild,
                             public nvinfer1::IPluginV3OneRuntime {
 public:
  explicit ContractPlugin(const Contract* c) : c_(c) {}

  nvinfer1::IPluginCapability* getCapabilityInterface(nvinfer1::PluginCapabilityType type) noexcept override {
    switch (type) {
      case nvinfer1::PluginCapabilityType::kCORE: return static_cast<nvinfer1::IPluginV3OneCore*>(this);
      case nvinfer1::PluginCapabilityType::kBUILD: return static_cast<nvinfer1::IPluginV3OneBuild*>(this);
      case nvinfer1::PluginCapabilityType::kRUNTIME: return static_cast<nvinfer1::IPluginV3OneRuntime*>(this);
      default: return nullptr;
    }
  }
  nvinfer1::IPluginV3* clone() noexcept override { return new (std::nothrow) ContractPlugin(c_); }

  // core
  const char* getPluginName() const noexcept override { return c_->name(); }
  const char* getPluginVersion() const noexcept override { return kVersion; }
  const char* getPluginNamespace() const noexcept override { return kNamespace; }

  // build
  int32_t getNbOutputs() const noexcept override { return c_->outputs(); }
  int32_t configurePlugin(const nvinfer1::DynamicPluginTensorDesc*, int32_t n_in,
                          const nvinfer1::DynamicPluginTensorDesc*, int32_t n_out) noexcept override {
    return n_in == c_->inputs() && n_out == c_->outputs() ? 0 : -1;
  }
  bool supportsFormatCombination(int32_t pos, const nvinfer1::DynamicPluginTensorDesc* io, int32_t n_in,
                                 int32_t n_out) noexcept override {
    if (io == nullptr || pos < 0 || pos >= n_in + n_out) return false;
    return c_->supports(pos, to_dtype(io[pos].desc.type), io[pos].desc.format == nvinfer1::TensorFormat::kLINEAR,
                        n_in, n_out);
  }
  int32_t getOutputDataTypes(nvinfer1::DataType* out, int32_t n_out, const nvinfer1::DataType*,
                             int32_t n_in) const noexcept override {
    if (out == nullptr || n_in != c_->inputs() || n_out != c_->outputs()) return -1;
    for (int32_t o = 0; o < n_out; ++o) {
      if (!from_dtype(c_->type(c_->inputs() + o), &out[o])) return -1;
    }
    return 0;
  }
  int32_t getOutputShapes(const nvinfer1::DimsExprs* in, int32_t n_in, const nvinfer1::DimsExprs*,
                          int32_t n_shape_in, nvinfer1::DimsExprs* out, int32_t n_out,
                          nvinfer1::IExprBuilder& exprs) noexcept override {
    if (in == nullptr || out == nullptr || n_in != c_->inputs() || n_shape_in != 0 || n_out != c_->outputs()) {
      return -1;
    }
    for (int32_t o = 0; o < n_out; ++o) {
      const OutputShape s = c_->output_shape(o);
      if (s.like >= 0) {
        out[o] = in[s.like];
        continue;
      }
      out[o].nbDims = s.dims.nb;
      for (int i = 0; i < s.dims.nb; ++i) out[o].d[i] = exprs.constant(s.dims.d[i]);
    }
    return 0;
  }
  size_t getWorkspaceSize(const nvinfer1::DynamicPluginTensorDesc*, int32_t, const nvinfer1::DynamicPluginTensorDesc*,
                          int32_t) const noexcept override {
    return c_->workspace_bytes();
  }

  // runtime
  int32_t onShapeChange(const nvinfer1::PluginTensorDesc* in, int32_t n_in, const nvinfer1::PluginTensorDesc*,
                        int32_t n_out) noexcept override {
    if (in == nullptr || n_in != c_->inputs() || n_out != c_->outputs() || n_in > kMaxTensors) return -1;
    std::array<Dims, kMaxTensors> dims{};
    for (int32_t i = 0; i < n_in; ++i) {
      if (!to_dims(in[i].dims, &dims[i])) return -1;
    }
    return c_->shapes_ok(dims.data(), n_in) ? 0 : -1;
  }
  int32_t enqueue(const nvinfer1::PluginTensorDesc* in_desc, const nvinfer1::PluginTensorDesc*,
                  const void* const* inputs, void* const* outputs, void* workspace,
                  cudaStream_t stream) noexcept override {
    if (in_desc == nullptr || inputs == nullptr || outputs == nullptr || c_->inputs() > kMaxTensors) return -1;
    std::array<Dims, kMaxTensors> dims{};
    for (int i = 0; i < c_->inputs(); ++i) {
      if (!to_dims(in_desc[i].dims, &dims[i])) return -1;
    }
    return c_->enqueue(dims.data(), inputs, outputs, workspace, static_cast<void*>(stream));
  }
  nvinfer1::IPluginV3* attachToContext(nvinfer1::IPluginResourceContext*) noexcept override { return clone(); }
  const nvinfer1::PluginFieldCollection* getFieldsToSerialize() noexcept override { return &no_fields_; }

 private:
  const Contract* c_;
  nvinfer1::PluginFieldCollection no_fields_{0, nullptr};
};

class ContractCreator final : public nvinfer1::IPluginCreatorV3One {
 public:
  explicit ContractCreator(const Contract* c) : c_(c) {
    if (std::strcmp(c->name(), "MagpieSoftmax") == 0) {  // advertises its two optional fields
      advertised_[0] = nvinfer1::PluginField{"mode", nullptr, nvinfer1::PluginFieldType::kINT32, 1};
      advertised_[1] = nvinfer1::PluginField{"layer_index", nullptr, nvinfer1::PluginFieldType::kINT32, 1};
      names_ = nvinfer1::PluginFieldCollection{2, advertised_.data()};
    }
  }
  const char* getPluginName() const noexcept override { return c_->name(); }
  const char* getPluginVersion() const noexcept override { return kVersion; }
  const char* getPluginNamespace() const noexcept override { return kNamespace; }
  const nvinfer1::PluginFieldCollection* getFieldNames() noexcept override { return &names_; }
  nvinfer1::IPluginV3* createPlugin(const char*, const nvinfer1::PluginFieldCollection* fields,
                                    nvinfer1::TensorRTPhase) noexcept override {
    if (fields == nullptr || fields->nbFields < 0 || fields->nbFields > 2 ||
        (fields->nbFields > 0 && fields->fields == nullptr)) {
      return nullptr;
    }
    std::array<Field, 2> f{};
    for (int32_t i = 0; i < fields->nbFields; ++i) {
      const nvinfer1::PluginField& pf = fields->fields[i];
      f[i] = Field{pf.name, pf.data, pf.length, pf.type == nvinfer1::PluginFieldType::kINT32};
    }
    if (!fields_ok(c_, f.data(), fields->nbFields)) return nullptr;
    return new (std::nothrow) ContractPlugin(c_);
  }

 private:
  const Contract* c_;
  std::array<nvinfer1::PluginField, 2> advertised_{};
  nvinfer1::PluginFieldCollection names_{0, nullptr};
};

// The five creators (registered by address: they live as long as the library).
constexpr int kCreators = 5;
ContractCreator& creator(int i) {
  static ContractCreator c0(contract_at(0)), c1(contract_at(1)), c2(contract_at(2)), c3(contract_at(3)),
      c4(contract_at(4));
  static ContractCreator* const all[kCreators] = {&c0, &c1, &c2, &c3, &c4};
  return *all[i];
}

std::mutex g_registration;

}  // namespace

mtt_plugin_status_t register_tensorrt_plugins() noexcept {
  const std::lock_guard<std::mutex> lock(g_registration);
  nvinfer1::IPluginRegistry* registry = ::getPluginRegistry();
  if (registry == nullptr) return MTT_PLUGIN_STATUS_REGISTRY_UNAVAILABLE;
  int ours = 0, present = 0;
  for (int i = 0; i < kCreators; ++i) {
    ContractCreator& c = creator(i);
    nvinfer1::IPluginCreatorInterface* found = registry->getCreator(c.getPluginName(), kVersion, kNamespace);
    present += found != nullptr;
    ours += found == static_cast<nvinfer1::IPluginCreatorInterface*>(&c);
  }
  if (ours == kCreators) return MTT_PLUGIN_STATUS_ALREADY_REGISTERED;
  if (present != 0) return MTT_PLUGIN_STATUS_REGISTRATION_CONFLICT;
  for (int i = 0; i < kCreators; ++i) {
    if (registry->registerCreator(creator(i), kNamespace)) continue;
    const bool taken = registry->getCreator(creator(i).getPluginName(), kVersion, kNamespace) != nullptr;
    for (int j = 0; j < i; ++j) registry->deregisterCreator(creator(j));  // take back this call's creators
    return taken ? MTT_PLUGIN_STATUS_REGISTRATION_CONFLICT : MTT_PLUGIN_STATUS_REGISTRATION_FAILED;
  }
  return MTT_PLUGIN_STATUS_OK;
}

}  // namespace plugin
}  // namespace mtt

#endif  // MTT_B200_WITH_TENSORRT
