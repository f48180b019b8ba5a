// Plugin-library ABI v1 (the symbols the runtime's model loader dlopen()s).
//
// Replaces mtt_plugin_get_api_v1 / mtt_plugin_get_main_device_position_class_table_v1
// (plugins/local_ar_plugins.cu:4083-4104,4858-4913).  The struct layouts,
// status codes, creator order, names, version and namespace are part of the
// contract and are therefore the same as the reference's
// (include/magpie_tts_rt/magpie_tts_rt_plugin.h, docs/engine-contracts.md:247-250).
//
// register_plugins registers the five IPluginV3 creators of trt_plugins.cpp
// (one generic plugin over the contracts of plugin_contract.cpp) into
// TensorRT's process-wide registry when the library is built against
// TensorRT (MTT_B200_WITH_TENSORRT); otherwise it reports that no plugin
// registry is available, and the kernels behind the five creators are
// reached directly through the mtt_b200_launch_* C functions.
#include <cstring>

#include "../../include/magpie_tts_rt_b200.h"

namespace {

constexpr char kPluginVersion[] = "1";
constexpr char kPluginNamespace[] = "magpie_tts_rt";
constexpr const char* kCreatorNames[MTT_PLUGIN_CREATOR_COUNT_V1] = {
    "MagpieLocalARSampling", "MagpieLocalAREos", "MagpieLayerNorm", "MagpieGeluTanh", "MagpieSoftmax",
};

#if defined(MTT_B200_WITH_TENSORRT)
}  // namespace
namespace mtt {
namespace plugin {
mtt_plugin_status_t register_tensorrt_plugins() noexcept;
}  // namespace plugin
}  // namespace mtt
namespace {
mtt_plugin_status_t register_plugins_entry() { return mtt::plugin::register_tensorrt_plugins(); }
#else
mtt_plugin_status_t register_plugins_entry() { return MTT_PLUGIN_STATUS_REGISTRY_UNAVAILABLE; }
#endif

void fill_creator(mtt_plugin_creator_v1_t& creator, const char* name) {
  creator.struct_size = sizeof(creator);
  creator.abi_version = MTT_PLUGIN_ABI_VERSION_1;
  std::strncpy(creator.name, name, MTT_PLUGIN_CREATOR_NAME_CAPACITY - 1U);
  std::strncpy(creator.version, kPluginVersion, MTT_PLUGIN_CREATOR_VERSION_CAPACITY - 1U);
  std::strncpy(creator.plugin_namespace, kPluginNamespace, MTT_PLUGIN_NAMESPACE_CAPACITY - 1U);
}

}  // namespace

extern "C" MTT_B200_API mtt_plugin_status_t mtt_plugin_get_api_v1(mtt_plugin_api_v1_t* api) {
  if (api == nullptr) return MTT_PLUGIN_STATUS_INVALID_ARGUMENT;
  if (api->struct_size != sizeof(mtt_plugin_api_v1_t) || api->abi_version != MTT_PLUGIN_ABI_VERSION_1) {
    return MTT_PLUGIN_STATUS_ABI_MISMATCH;
  }
  mtt_plugin_api_v1_t populated{};
  populated.struct_size = sizeof(populated);
  populated.abi_version = MTT_PLUGIN_ABI_VERSION_1;
  populated.creator_count = MTT_PLUGIN_CREATOR_COUNT_V1;
  populated.register_plugins = &register_plugins_entry;
  for (unsigned i = 0; i < MTT_PLUGIN_CREATOR_COUNT_V1; ++i) fill_creator(populated.creators[i], kCreatorNames[i]);
  *api = populated;
  return MTT_PLUGIN_STATUS_OK;
}

extern "C" MTT_B200_API mtt_plugin_status_t mtt_plugin_get_main_device_position_class_table_v1(
    mtt_main_device_position_class_table_v1_t* table) {
  if (table == nullptr) return MTT_PLUGIN_STATUS_INVALID_ARGUMENT;
  if (table->struct_size != sizeof(*table) || table->abi_version != MTT_PLUGIN_ABI_VERSION_1) {
    return MTT_PLUGIN_STATUS_ABI_MISMATCH;
  }
  return MTT_PLUGIN_STATUS_NOT_READY;
}
