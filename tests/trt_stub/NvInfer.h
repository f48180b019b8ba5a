// Stand-in for TensorRT's NvInfer.h, for compiling and exercising
// magpie_tts_rt_b200/csrc/trt_plugins.cpp on a machine without TensorRT.
// It declares only the part of the nvinfer1 plugin interface that file uses,
// with the names and signatures of TensorRT 10's IPluginV3 API as the
// reference plugin library uses them (plugins/local_ar_plugins.cu); the test
// program supplies the registry and the expression builder.  Not a TensorRT
// header: a build against TensorRT uses the real one.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime_api.h>

namespace nvinfer1 {

using AsciiChar = char;

enum class DataType : int32_t { kFLOAT, kHALF, kINT8, kINT32, kBOOL, kUINT8, kFP8, kBF16, kINT64, kINT4, kFP4 };
enum class TensorFormat : int32_t { kLINEAR, kCHW2, kHWC8, kCHW4, kCHW16, kCHW32 };
using PluginFormat = TensorFormat;

struct Dims64 {
  static constexpr int32_t MAX_DIMS = 8;
  int32_t nbDims;
  int64_t d[MAX_DIMS];
};
using Dims = Dims64;

class IDimensionExpr {
 public:
  virtual ~IDimensionExpr() = default;
};

class IExprBuilder {
 public:
  virtual ~IExprBuilder() = default;
  virtual const IDimensionExpr* constant(int64_t value) noexcept = 0;
};

struct DimsExprs {
  int32_t nbDims;
  const IDimensionExpr* d[Dims::MAX_DIMS];
};

struct PluginTensorDesc {
  Dims dims;
  DataType type;
  TensorFormat format;
  float scale;
};

struct DynamicPluginTensorDesc {
  PluginTensorDesc desc;
  Dims min;
  Dims max;
  Dims opt;
};

enum class PluginFieldType : int32_t { kFLOAT16, kFLOAT32, kFLOAT64, kINT8, kINT16, kINT32, kCHAR, kDIMS, kUNKNOWN };

struct PluginField {
  const AsciiChar* name;
  const void* data;
  PluginFieldType type;
  int32_t length;
};

struct PluginFieldCollection {
  int32_t nbFields;
  const PluginField* fields;
};

enum class PluginCapabilityType : int32_t { kCORE, kBUILD, kRUNTIME };
enum class TensorRTPhase : int32_t { kBUILD, kRUNTIME };

class IPluginCapability {
 public:
  virtual ~IPluginCapability() = default;
};

class IPluginResourceContext {
 public:
  virtual ~IPluginResourceContext() = default;
};

class IPluginV3 {
 public:
  virtual ~IPluginV3() = default;
  virtual IPluginCapability* getCapabilityInterface(PluginCapabilityType type) noexcept = 0;
  virtual IPluginV3* clone() noexcept = 0;
};

class IPluginV3OneCore : public IPluginCapability {
 public:
  virtual const AsciiChar* getPluginName() const noexcept = 0;
  virtual const AsciiChar* getPluginVersion() const noexcept = 0;
  virtual const AsciiChar* getPluginNamespace() const noexcept = 0;
};

class IPluginV3OneBuild : public IPluginCapability {
 public:
  virtual int32_t configurePlugin(const DynamicPluginTensorDesc* in, int32_t nbInputs,
                                  const DynamicPluginTensorDesc* out, int32_t nbOutputs) noexcept = 0;
  virtual int32_t getOutputDataTypes(DataType* outputTypes, int32_t nbOutputs, const DataType* inputTypes,
                                     int32_t nbInputs) const noexcept = 0;
  virtual int32_t getOutputShapes(const DimsExprs* inputs, int32_t nbInputs, const DimsExprs* shapeInputs,
                                  int32_t nbShapeInputs, DimsExprs* outputs, int32_t nbOutputs,
                                  IExprBuilder& exprBuilder) noexcept = 0;
  virtual bool supportsFormatCombination(int32_t pos, const DynamicPluginTensorDesc* inOut, int32_t nbInputs,
                                         int32_t nbOutputs) noexcept = 0;
  virtual int32_t getNbOutputs() const noexcept = 0;
  virtual size_t getWorkspaceSize(const DynamicPluginTensorDesc* inputs, int32_t nbInputs,
                                  const DynamicPluginTensorDesc* outputs, int32_t nbOutputs) const noexcept {
    return 0;
  }
};

class IPluginV3OneRuntime : public IPluginCapability {
 public:
  virtual int32_t onShapeChange(const PluginTensorDesc* in, int32_t nbInputs, const PluginTensorDesc* out,
                                int32_t nbOutputs) noexcept = 0;
  virtual int32_t enqueue(const PluginTensorDesc* inputDesc, const PluginTensorDesc* outputDesc,
                          const void* const* inputs, void* const* outputs, void* workspace,
                          cudaStream_t stream) noexcept = 0;
  virtual IPluginV3* attachToContext(IPluginResourceContext* context) noexcept = 0;
  virtual const PluginFieldCollection* getFieldsToSerialize() noexcept = 0;
};

class IPluginCreatorInterface {
 public:
  virtual ~IPluginCreatorInterface() = default;
};

class IPluginCreatorV3One : public IPluginCreatorInterface {
 public:
  virtual IPluginV3* createPlugin(const AsciiChar* name, const PluginFieldCollection* fc,
                                  TensorRTPhase phase) noexcept = 0;
  virtual const PluginFieldCollection* getFieldNames() noexcept = 0;
  virtual const AsciiChar* getPluginName() const noexcept = 0;
  virtual const AsciiChar* getPluginVersion() const noexcept = 0;
  virtual const AsciiChar* getPluginNamespace() const noexcept = 0;
};

class IPluginRegistry {
 public:
  virtual ~IPluginRegistry() = default;
  virtual bool registerCreator(IPluginCreatorInterface& creator, const AsciiChar* pluginNamespace) noexcept = 0;
  virtual IPluginCreatorInterface* getCreator(const AsciiChar* pluginName, const AsciiChar* pluginVersion,
                                              const AsciiChar* pluginNamespace = "") noexcept = 0;
  virtual bool deregisterCreator(const IPluginCreatorInterface& creator) noexcept = 0;
};

}  // namespace nvinfer1

extern "C" nvinfer1::IPluginRegistry* getPluginRegistry() noexcept;
