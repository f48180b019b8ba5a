// CPU test of the TensorRT plugin layer (magpie_tts_rt_b200/csrc/
// trt_plugins.cpp over plugin_contract.cpp), built against the stand-in
// header tests/trt_stub/NvInfer.h with this program's fake plugin registry and
// expression builder.  It checks the five creators (order, names, version,
// namespace, fields), every plugin's I/O contract as TensorRT would query it,
// and the registration statuses of the plugin ABI's register_plugins.  The
// launchers are called only with null buffers (their -1 path), so no GPU is
// needed; with --gpu each plugin's enqueue also runs on device buffers and
// must give bit for bit what a direct call of its launcher gives.  Prints "OK"
// and exits 0, or names the failed checks.
#include <NvInfer.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "magpie_tts_rt_b200.h"

namespace {

int g_failures = 0;
#define CHECK(cond)                                                    \
  do {                                                                 \
    if (!(cond)) {                                                     \
      std::printf("FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);    \
      ++g_failures;                                                    \
    }                                                                  \
  } while (0)

// --- fakes ------------------------------------------------------------------

struct ConstExpr final : nvinfer1::IDimensionExpr {
  explicit ConstExpr(int64_t v) : value(v) {}
  int64_t value;
};

struct Builder final : nvinfer1::IExprBuilder {
  std::vector<std::unique_ptr<ConstExpr>> made;
  const nvinfer1::IDimensionExpr* constant(int64_t v) noexcept override {
    made.push_back(std::make_unique<ConstExpr>(v));
    return made.back().get();
  }
};

int64_t value_of(const nvinfer1::IDimensionExpr* e) { return static_cast<const ConstExpr*>(e)->value; }

struct Registry final : nvinfer1::IPluginRegistry {
  std::map<std::string, nvinfer1::IPluginCreatorInterface*> by_name;
  int refuse_at = -1;      // registerCreator call index that fails
  bool foreign_on_refusal = false;
  int calls = 0;
  static std::string key(const char* n, const char* v, const char* ns) {
    return std::string(n) + "/" + v + "/" + ns;
  }
  bool registerCreator(nvinfer1::IPluginCreatorInterface& c, const char* ns) noexcept override {
    auto* v3 = static_cast<nvinfer1::IPluginCreatorV3One*>(&c);
    const std::string k = key(v3->getPluginName(), v3->getPluginVersion(), ns);
    if (calls++ == refuse_at) {
      if (foreign_on_refusal) by_name[k] = &foreign;
      return false;
    }
    if (by_name.count(k)) return false;
    by_name[k] = &c;
    return true;
  }
  nvinfer1::IPluginCreatorInterface* getCreator(const char* n, const char* v, const char* ns) noexcept override {
    auto it = by_name.find(key(n, v, ns));
    return it == by_name.end() ? nullptr : it->second;
  }
  bool deregisterCreator(const nvinfer1::IPluginCreatorInterface& c) noexcept override {
    for (auto it = by_name.begin(); it != by_name.end(); ++it) {
      if (it->second == &c) {
        by_name.erase(it);
        return true;
      }
    }
    return false;
  }
  struct Foreign final : nvinfer1::IPluginCreatorInterface {} foreign;
};

Registry* g_registry = nullptr;

}  // namespace

extern "C" nvinfer1::IPluginRegistry* getPluginRegistry() noexcept { return g_registry; }

namespace {

nvinfer1::Dims dims(std::initializer_list<int64_t> v) {
  nvinfer1::Dims d{};
  d.nbDims = static_cast<int32_t>(v.size());
  int i = 0;
  for (int64_t x : v) d.d[i++] = x;
  return d;
}

mtt_plugin_status_t register_via_abi() {
  mtt_plugin_api_v1_t api{};
  api.struct_size = sizeof(api);
  api.abi_version = MTT_PLUGIN_ABI_VERSION_1;
  if (mtt_plugin_get_api_v1(&api) != MTT_PLUGIN_STATUS_OK || api.register_plugins == nullptr) return -100;
  return api.register_plugins();
}

struct Spec {
  const char* name;
  std::vector<nvinfer1::DataType> types;  // inputs then outputs
  int n_in;
  std::vector<nvinfer1::Dims> good;       // an accepted input binding
  std::vector<nvinfer1::Dims> bad;        // a rejected one
};

using DT = nvinfer1::DataType;

std::vector<Spec> specs() {
  const int64_t V = 2024, E = 768;
  return {
      {"MagpieLocalARSampling",
       {DT::kBF16, DT::kBOOL, DT::kBOOL, DT::kBOOL, DT::kINT64, DT::kINT64, DT::kBF16, DT::kINT64, DT::kBF16,
        DT::kINT64, DT::kINT32},
       7,
       {dims({2, V}), dims({1}), dims({1}), dims({1}), dims({1}), dims({1}), dims({V, E})},
       {dims({2, V}), dims({1}), dims({1}), dims({1}), dims({1}), dims({2}), dims({V, E})}},
      {"MagpieLocalAREos",
       {DT::kBF16, DT::kINT64, DT::kBOOL, DT::kBOOL, DT::kBOOL, DT::kBF16, DT::kBF16, DT::kINT32},
       7,
       {dims({2, E}), dims({1, 8, 2}), dims({1}), dims({1}), dims({1}), dims({16 * V, E}), dims({16 * V})},
       {dims({2, E}), dims({1, 8, 2}), dims({1}), dims({1}), dims({1}), dims({16 * V, E}), dims({16 * V, 1})}},
      {"MagpieLayerNorm", {DT::kBF16, DT::kBF16, DT::kBF16}, 2, {dims({1, 300, E}), dims({E})},
       {dims({1, 513, E}), dims({E})}},
      {"MagpieGeluTanh", {DT::kBF16, DT::kBF16}, 1, {dims({2, 3072, 1})}, {dims({2, 3072, 219})}},
      {"MagpieSoftmax", {DT::kBF16, DT::kBF16}, 1, {dims({2, 12, 1, 300})}, {dims({2, 12, 1, 468})}},
  };
}

void check_plugin(nvinfer1::IPluginCreatorV3One* creator, const Spec& s) {
  nvinfer1::PluginFieldCollection none{0, nullptr};
  std::unique_ptr<nvinfer1::IPluginV3> plugin(creator->createPlugin("p", &none, nvinfer1::TensorRTPhase::kBUILD));
  CHECK(plugin != nullptr);
  if (!plugin) return;
  auto* core = static_cast<nvinfer1::IPluginV3OneCore*>(plugin->getCapabilityInterface(nvinfer1::PluginCapabilityType::kCORE));
  auto* build = static_cast<nvinfer1::IPluginV3OneBuild*>(plugin->getCapabilityInterface(nvinfer1::PluginCapabilityType::kBUILD));
  auto* run = static_cast<nvinfer1::IPluginV3OneRuntime*>(plugin->getCapabilityInterface(nvinfer1::PluginCapabilityType::kRUNTIME));
  CHECK(core && build && run);
  CHECK(plugin->getCapabilityInterface(static_cast<nvinfer1::PluginCapabilityType>(7)) == nullptr);
  CHECK(std::strcmp(core->getPluginName(), s.name) == 0);
  CHECK(std::strcmp(core->getPluginVersion(), "1") == 0);
  CHECK(std::strcmp(core->getPluginNamespace(), "magpie_tts_rt") == 0);
  const int n_in = s.n_in, n_out = static_cast<int>(s.types.size()) - s.n_in;
  CHECK(build->getNbOutputs() == n_out);
  std::vector<nvinfer1::DynamicPluginTensorDesc> io(s.types.size());
  CHECK(build->configurePlugin(io.data(), n_in, io.data() + n_in, n_out) == 0);
  CHECK(build->configurePlugin(io.data(), n_in + 1, io.data() + n_in, n_out) == -1);
  // formats: the contract type, linear only; another type or format refused
  for (int p = 0; p < static_cast<int>(s.types.size()); ++p) {
    io[p].desc.type = s.types[p];
    io[p].desc.format = nvinfer1::TensorFormat::kLINEAR;
    CHECK(build->supportsFormatCombination(p, io.data(), n_in, n_out));
    io[p].desc.type = s.types[p] == DT::kFLOAT ? DT::kHALF : DT::kFLOAT;
    CHECK(!build->supportsFormatCombination(p, io.data(), n_in, n_out));
    io[p].desc.type = s.types[p];
    io[p].desc.format = nvinfer1::TensorFormat::kHWC8;
    CHECK(!build->supportsFormatCombination(p, io.data(), n_in, n_out));
    io[p].desc.format = nvinfer1::TensorFormat::kLINEAR;
  }
  CHECK(!build->supportsFormatCombination(n_in + n_out, io.data(), n_in, n_out));
  std::vector<DT> out_types(n_out);
  CHECK(build->getOutputDataTypes(out_types.data(), n_out, s.types.data(), n_in) == 0);
  for (int o = 0; o < n_out; ++o) CHECK(out_types[o] == s.types[n_in + o]);
  // output shapes
  Builder b;
  std::vector<nvinfer1::DimsExprs> in_exprs(n_in), out_exprs(n_out);
  for (int i = 0; i < n_in; ++i) {
    in_exprs[i].nbDims = s.good[i].nbDims;
    for (int k = 0; k < s.good[i].nbDims; ++k) in_exprs[i].d[k] = b.constant(s.good[i].d[k]);
  }
  CHECK(build->getOutputShapes(in_exprs.data(), n_in, nullptr, 0, out_exprs.data(), n_out, b) == 0);
  if (std::strcmp(s.name, "MagpieLocalARSampling") == 0) {
    CHECK(out_exprs[0].nbDims == 1 && value_of(out_exprs[0].d[0]) == 1);
    CHECK(out_exprs[1].nbDims == 2 && value_of(out_exprs[1].d[0]) == 2 && value_of(out_exprs[1].d[1]) == 768);
    CHECK(out_exprs[3].nbDims == 1 && value_of(out_exprs[3].d[0]) == 1);
  } else if (std::strcmp(s.name, "MagpieLocalAREos") == 0) {
    CHECK(out_exprs[0].nbDims == 1 && value_of(out_exprs[0].d[0]) == 1);
  } else {  // the output has the input's shape
    CHECK(out_exprs[0].nbDims == in_exprs[0].nbDims);
    for (int k = 0; k < in_exprs[0].nbDims; ++k) CHECK(out_exprs[0].d[k] == in_exprs[0].d[k]);
  }
  const size_t ws = build->getWorkspaceSize(io.data(), n_in, io.data() + n_in, n_out);
  CHECK(ws == (std::strcmp(s.name, "MagpieLocalAREos") == 0 ? mtt_b200_local_ar_eos_workspace_size() : 0));
  // shapes at runtime
  std::vector<nvinfer1::PluginTensorDesc> in_desc(n_in), out_desc(n_out);
  for (int i = 0; i < n_in; ++i) in_desc[i].dims = s.good[i];
  CHECK(run->onShapeChange(in_desc.data(), n_in, out_desc.data(), n_out) == 0);
  std::vector<nvinfer1::PluginTensorDesc> bad_desc(n_in);
  for (int i = 0; i < n_in; ++i) bad_desc[i].dims = s.bad[i];
  CHECK(run->onShapeChange(bad_desc.data(), n_in, out_desc.data(), n_out) == -1);
  // enqueue with no buffers: the launcher's argument check (-1), no device work
  std::vector<const void*> in_ptr(n_in, nullptr);
  std::vector<void*> out_ptr(n_out, nullptr);
  CHECK(run->enqueue(in_desc.data(), out_desc.data(), in_ptr.data(), out_ptr.data(), nullptr, nullptr) == -1);
  // stateless copies
  std::unique_ptr<nvinfer1::IPluginV3> copy(plugin->clone());
  std::unique_ptr<nvinfer1::IPluginV3> attached(run->attachToContext(nullptr));
  CHECK(copy && attached);
  CHECK(run->getFieldsToSerialize() != nullptr && run->getFieldsToSerialize()->nbFields == 0);
}

// --gpu: each plugin's enqueue on device buffers must give exactly what the
// launcher it dispatches to gives for the same inputs (input order, output
// order, the shape-derived sizes).
bool gpu_matches(nvinfer1::IPluginCreatorV3One* creator, const Spec& s, uint32_t seed) {
  nvinfer1::PluginFieldCollection none{0, nullptr};
  std::unique_ptr<nvinfer1::IPluginV3> plugin(creator->createPlugin("g", &none, nvinfer1::TensorRTPhase::kRUNTIME));
  auto* run = static_cast<nvinfer1::IPluginV3OneRuntime*>(plugin->getCapabilityInterface(nvinfer1::PluginCapabilityType::kRUNTIME));
  const int n_in = s.n_in, n_out = static_cast<int>(s.types.size()) - n_in;
  auto elem = [](DT t) { return t == DT::kBF16 ? 2 : (t == DT::kBOOL ? 1 : (t == DT::kINT32 ? 4 : 8)); };
  auto count = [](const nvinfer1::Dims& d) { int64_t c = 1; for (int k = 0; k < d.nbDims; ++k) c *= d.d[k]; return c; };
  std::vector<nvinfer1::Dims> out_dims(n_out);
  const bool fixed = std::strcmp(s.name, "MagpieLocalARSampling") == 0 || std::strcmp(s.name, "MagpieLocalAREos") == 0;
  for (int o = 0; o < n_out; ++o) out_dims[o] = fixed ? (o == 1 ? dims({2, 768}) : dims({1})) : s.good[0];
  std::vector<void*> in_buf(n_in), out_a(n_out), out_b(n_out);
  std::vector<size_t> out_bytes(n_out);
  uint32_t x = seed;
  for (int i = 0; i < n_in; ++i) {
    const size_t bytes = static_cast<size_t>(count(s.good[i])) * elem(s.types[i]);
    std::vector<uint8_t> h(bytes);
    for (size_t k = 0; k < bytes; ++k) {
      x = x * 1664525u + 1013904223u;
      h[k] = static_cast<uint8_t>(x >> 24);
    }
    if (s.types[i] == DT::kBOOL) for (auto& v : h) v &= 1;
    if (s.types[i] == DT::kBF16)  // finite values: clear the top exponent bits
      for (size_t k = 1; k < bytes; k += 2) h[k] &= 0x3f;
    if (s.types[i] == DT::kINT64) for (size_t k = 0; k < bytes; ++k) h[k] = (k % 8 == 0) ? h[k] & 0x7f : 0;
    if (std::strcmp(s.name, "MagpieLocalARSampling") == 0 && i == 1) h[0] = 1, h.resize(1);  // unfinished
    if (std::strcmp(s.name, "MagpieLocalARSampling") == 0 && (i == 2 || i == 3)) h[0] = 0;
    cudaMalloc(&in_buf[i], bytes);
    cudaMemcpy(in_buf[i], h.data(), bytes, cudaMemcpyHostToDevice);
  }
  for (int o = 0; o < n_out; ++o) {
    out_bytes[o] = static_cast<size_t>(count(out_dims[o])) * elem(s.types[n_in + o]);
    cudaMalloc(&out_a[o], out_bytes[o]);
    cudaMalloc(&out_b[o], out_bytes[o]);
    cudaMemset(out_a[o], 0x5a, out_bytes[o]);
    cudaMemset(out_b[o], 0x5a, out_bytes[o]);
  }
  void* ws = nullptr;
  const size_t ws_bytes = mtt_b200_local_ar_eos_workspace_size();
  cudaMalloc(&ws, ws_bytes);
  std::vector<nvinfer1::PluginTensorDesc> in_desc(n_in), out_desc(n_out);
  for (int i = 0; i < n_in; ++i) in_desc[i].dims = s.good[i];
  int rc_plugin = run->enqueue(in_desc.data(), out_desc.data(), in_buf.data(), out_a.data(), ws, nullptr);
  int rc_direct = -7;
  auto I = [&](int i) { return in_buf[i]; };
  if (std::strcmp(s.name, "MagpieLocalARSampling") == 0) {
    rc_direct = mtt_b200_launch_local_ar_sampling(I(0), (const bool*)I(1), (const bool*)I(2), (const bool*)I(3),
                                                  (const int64_t*)I(4), (const int64_t*)I(5), I(6), (int64_t*)out_b[0],
                                                  out_b[1], (int64_t*)out_b[2], (int32_t*)out_b[3], nullptr);
  } else if (std::strcmp(s.name, "MagpieLocalAREos") == 0) {
    rc_direct = mtt_b200_launch_local_ar_eos(I(0), (const int64_t*)I(1), (const bool*)I(2), (const bool*)I(3),
                                             (const bool*)I(4), I(5), I(6), ws, (int32_t*)out_b[0], nullptr);
  } else if (std::strcmp(s.name, "MagpieLayerNorm") == 0) {
    rc_direct = mtt_b200_launch_layer_norm(I(0), I(1), out_b[0], (int32_t)(s.good[0].d[0] * s.good[0].d[1]), nullptr);
  } else if (std::strcmp(s.name, "MagpieGeluTanh") == 0) {
    rc_direct = mtt_b200_launch_gelu_tanh(I(0), out_b[0], (size_t)count(s.good[0]), nullptr);
  } else {
    rc_direct = mtt_b200_launch_softmax(I(0), out_b[0], (int32_t)(count(s.good[0]) / s.good[0].d[3]),
                                        (int32_t)s.good[0].d[3], nullptr);
  }
  bool same = rc_plugin == 0 && rc_direct == 0 && cudaDeviceSynchronize() == cudaSuccess;
  for (int o = 0; o < n_out && same; ++o) {
    std::vector<uint8_t> a(out_bytes[o]), b(out_bytes[o]);
    cudaMemcpy(a.data(), out_a[o], out_bytes[o], cudaMemcpyDeviceToHost);
    cudaMemcpy(b.data(), out_b[o], out_bytes[o], cudaMemcpyDeviceToHost);
    same = a == b;
  }
  for (void* p : in_buf) cudaFree(p);
  for (int o = 0; o < n_out; ++o) { cudaFree(out_a[o]); cudaFree(out_b[o]); }
  cudaFree(ws);
  return same;
}

}  // namespace

int main(int argc, char** argv) {
  const bool gpu = argc > 1 && std::strcmp(argv[1], "--gpu") == 0;
  const char* order[] = {"MagpieLocalARSampling", "MagpieLocalAREos", "MagpieLayerNorm", "MagpieGeluTanh",
                         "MagpieSoftmax"};
  // no registry
  g_registry = nullptr;
  CHECK(register_via_abi() == MTT_PLUGIN_STATUS_REGISTRY_UNAVAILABLE);

  // register, then again
  Registry reg;
  g_registry = &reg;
  CHECK(register_via_abi() == MTT_PLUGIN_STATUS_OK);
  CHECK(reg.by_name.size() == 5);
  CHECK(register_via_abi() == MTT_PLUGIN_STATUS_ALREADY_REGISTERED);
  std::vector<nvinfer1::IPluginCreatorV3One*> creators;
  for (const char* n : order) {
    auto* c = static_cast<nvinfer1::IPluginCreatorV3One*>(reg.getCreator(n, "1", "magpie_tts_rt"));
    CHECK(c != nullptr);
    creators.push_back(c);
  }
  for (size_t i = 0; i < creators.size(); ++i) {
    if (!creators[i]) continue;
    CHECK(std::strcmp(creators[i]->getPluginName(), order[i]) == 0);
    CHECK(std::strcmp(creators[i]->getPluginVersion(), "1") == 0);
    CHECK(std::strcmp(creators[i]->getPluginNamespace(), "magpie_tts_rt") == 0);
    CHECK(creators[i]->getFieldNames()->nbFields == (i == 4 ? 2 : 0));
  }

  // fields: none for the fixed contracts; MagpieSoftmax takes mode 0 (and layer_index -1)
  const int32_t zero = 0, one = 1, minus_one = -1, three = 3;
  nvinfer1::PluginField mode0{"mode", &zero, nvinfer1::PluginFieldType::kINT32, 1};
  nvinfer1::PluginField mode1{"mode", &one, nvinfer1::PluginFieldType::kINT32, 1};
  nvinfer1::PluginField layer_m1{"layer_index", &minus_one, nvinfer1::PluginFieldType::kINT32, 1};
  nvinfer1::PluginField layer3{"layer_index", &three, nvinfer1::PluginFieldType::kINT32, 1};
  nvinfer1::PluginField mode0_f{"mode", &zero, nvinfer1::PluginFieldType::kFLOAT32, 1};
  auto make = [&](int c, std::vector<nvinfer1::PluginField> f) {
    nvinfer1::PluginFieldCollection fc{static_cast<int32_t>(f.size()), f.data()};
    std::unique_ptr<nvinfer1::IPluginV3> p(creators[c]->createPlugin("x", &fc, nvinfer1::TensorRTPhase::kRUNTIME));
    return p != nullptr;
  };
  CHECK(!make(0, {mode0}));
  CHECK(make(4, {}));
  CHECK(make(4, {mode0}));
  CHECK(make(4, {mode0, layer_m1}));
  CHECK(!make(4, {mode1}));         // a Main Decoder bank mode: not this library's
  CHECK(!make(4, {mode0, layer3}));
  CHECK(!make(4, {mode0_f}));
  CHECK(!make(4, {mode0, mode0}));
  CHECK(creators[2]->createPlugin("x", nullptr, nvinfer1::TensorRTPhase::kBUILD) == nullptr);

  // every plugin's contract
  const std::vector<Spec> all = specs();
  for (size_t i = 0; i < all.size(); ++i) {
    if (creators[i]) check_plugin(creators[i], all[i]);
  }
  if (gpu) {
    for (size_t i = 0; i < all.size(); ++i) {
      if (creators[i]) CHECK(gpu_matches(creators[i], all[i], 17u + static_cast<uint32_t>(i)));
    }
  }

  // a foreign creator under one of the names: conflict, nothing registered
  Registry foreign;
  foreign.by_name[Registry::key("MagpieGeluTanh", "1", "magpie_tts_rt")] = &foreign.foreign;
  g_registry = &foreign;
  CHECK(register_via_abi() == MTT_PLUGIN_STATUS_REGISTRATION_CONFLICT);
  CHECK(foreign.by_name.size() == 1);

  // the registry refuses the third creator: failure, the first two taken back
  Registry refusing;
  refusing.refuse_at = 2;
  g_registry = &refusing;
  CHECK(register_via_abi() == MTT_PLUGIN_STATUS_REGISTRATION_FAILED);
  CHECK(refusing.by_name.empty());

  // another library registers the fourth name meanwhile: conflict, taken back
  Registry racing;
  racing.refuse_at = 3;
  racing.foreign_on_refusal = true;
  g_registry = &racing;
  CHECK(register_via_abi() == MTT_PLUGIN_STATUS_REGISTRATION_CONFLICT);
  CHECK(racing.by_name.size() == 1);

  g_registry = nullptr;
  if (g_failures == 0) std::printf("OK\n");
  return g_failures == 0 ? 0 : 1;
}
