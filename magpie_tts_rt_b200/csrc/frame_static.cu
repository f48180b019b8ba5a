// Allocation-free entry to the batched Local AR frame.
//
// Some callers cannot call cudaMalloc on the path that runs a frame: a
// TensorRT plugin's enqueue() may only use the workspace the engine hands it;
// code being recorded into a CUDA graph must not allocate (global-mode stream
// capture rejects it); and a real-time synthesis thread cannot afford an
// allocation that may synchronise the device or take unbounded time.  This
// entry point gives them the frame without a caller-provided workspace: the
// scratch memory is a file-scope device array of fixed size
// (kStaticFrameWorkspaceBytes, 2 MiB) that every GPU which loads the library
// holds until the process exits.
//
// Set-up: on its first call on a device (that device current) the entry point
// resolves the array's device address with cudaGetSymbolAddress and caches
// it; make that first call before any stream capture begins.  The host-side
// name of the array is only a stand-in and is never passed to a kernel.
//
// Every call shares the one array and it keeps the last call's contents.  The
// frame initialises everything it reads from the workspace (stream list,
// counters, flags, caches) at its start, so nothing has to be cleared between
// calls; two calls whose kernels overlap on the GPU (different streams without
// ordering, or different host threads) race on the array.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/magpie_tts_rt_b200.h"

namespace {

constexpr size_t kStaticFrameWorkspaceBytes = MTT_B200_STATIC_FRAME_WORKSPACE_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_frame_workspace[kStaticFrameWorkspaceBytes];

std::mutex g_setup_mutex;
void* g_device_address[kMaxDevices] = {};

}  // namespace

extern "C" MTT_B200_API int mtt_b200_launch_local_ar_frame_static_workspace(
    const mtt_b200_local_ar_shape_t* shape, const mtt_b200_local_ar_weights_t* weights,
    const mtt_b200_sampling_config_t* sampling, const mtt_b200_stream_batch_t* batch, void* stream) {
  if (shape == nullptr || weights == nullptr || sampling == nullptr || batch == nullptr) {
    return MTT_B200_STATUS_INVALID_ARGUMENT;
  }
  const size_t needed = mtt_b200_local_ar_frame_workspace_size(shape, batch->n_streams, sampling->cfg);
  if (needed == 0) return MTT_B200_STATUS_INVALID_ARGUMENT;
  if (needed > kStaticFrameWorkspaceBytes) return MTT_B200_STATUS_STATIC_WORKSPACE_TOO_SMALL;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return MTT_B200_STATUS_CUDA_ERROR;
  if (device < 0 || device >= kMaxDevices) return MTT_B200_STATUS_UNSUPPORTED;
  void* workspace = nullptr;
  {
    const std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_device_address[device] == nullptr) {
      void* address = nullptr;
      if (cudaGetSymbolAddress(&address, g_static_frame_workspace) != cudaSuccess || address == nullptr) {
        return MTT_B200_STATUS_CUDA_ERROR;
      }
      g_device_address[device] = address;
    }
    workspace = g_device_address[device];
  }
  return mtt_b200_launch_local_ar_frame(shape, weights, sampling, batch, workspace, kStaticFrameWorkspaceBytes,
                                        stream);
}
