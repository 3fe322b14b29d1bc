// iSTFT entry point that allocates no device memory.
//
// Some callers of this library cannot call cudaMalloc when they separate
// audio: a host running the provider on a real-time audio thread (a plugin's
// process callback, for instance) must not make a call that can block for an
// unbounded time or synchronise the device, and an embedding application that
// fixes its GPU memory budget when it loads the library cannot have the
// footprint grow later.  vocalarc_b200_stage_istft sizes its frame scratch on
// first use with cudaMalloc; this variant runs the same two kernels with the
// scratch in a fixed array declared below, which every GPU that loads the
// library holds (kNoAllocScratchBytes) until the process exits.
#include <cstdio>
#include <mutex>

#include "vab_internal.h"
#include "vocalarc_b200.h"

namespace vab {
bool provider_view(native_gpu* g, int* device, cudaStream_t* stream, const float** window, const float2** twiddle);
bool provider_launched(native_gpu* g, cudaError_t e, const char* what);
}

namespace {

// 32 MiB: windowed frames of up to 2048 (segment x frame) pairs, both
// channels, 2048 samples each -- one 881,559-sample chunk (1,722 frames).
constexpr long long kNoAllocMaxFrames = 2048;
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(kNoAllocMaxFrames) * 2 * vab::kNfft * sizeof(float);

static __device__ __align__(256) float g_istft_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
float* g_scratch_address[kMaxDevices] = {nullptr};

// Device address of g_istft_scratch on `device` (which must be current).
// In host code the symbol name is only a host-side stand-in for the array, so
// the address is looked up once per device and then reused.
float* scratch_for(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_address[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_istft_scratch);
    if (e != cudaSuccess) {
      fprintf(stderr, "vocalarc-b200: cudaGetSymbolAddress(istft scratch) failed on device %d: %s\n", device,
              cudaGetErrorString(e));
      return nullptr;
    }
    g_scratch_address[device] = static_cast<float*>(ptr);
  }
  return g_scratch_address[device];
}

}  // namespace

extern "C" int vocalarc_b200_stage_istft_noalloc(native_gpu* gpu, const float* spec, const float* mask, int segments,
                                                  int length, float* audio) {
  int device = 0;
  cudaStream_t stream = nullptr;
  const float* window = nullptr;
  const float2* twiddle = nullptr;
  if (!vab::provider_view(gpu, &device, &stream, &window, &twiddle) || segments <= 0 || length <= 0 ||
      spec == nullptr || mask == nullptr || audio == nullptr)
    return 0;
  const long long frames = length / vab::kHop + 1;
  if (static_cast<long long>(segments) * frames > kNoAllocMaxFrames) {
    fprintf(stderr,
            "vocalarc-b200: istft_noalloc: %d segment(s) x %lld frames exceeds the fixed scratch of %lld frames "
            "(%zu bytes); split the call or use vocalarc_b200_stage_istft\n",
            segments, frames, kNoAllocMaxFrames, kNoAllocScratchBytes);
    return 0;
  }
  if (cudaSetDevice(device) != cudaSuccess) return 0;
  float* scratch = scratch_for(device);
  if (scratch == nullptr) return 0;
  // Every frame slot that the overlap-add reads is written first by the frame
  // kernel, so nothing in the scratch has to start at zero.
  // The launches are checked, counted and traced like the provider's own: a
  // launch error disables the provider (later calls return 0).
  if (!vab::provider_launched(gpu,
                              vab::launch_istft_frames(spec, mask, segments, static_cast<int>(frames), window, twiddle,
                                                       scratch, stream),
                              "istft"))
    return 0;
  return vab::provider_launched(
             gpu, vab::launch_overlap_add(scratch, segments, static_cast<int>(frames), length, window, audio, stream),
             "overlap-add")
             ? 1
             : 0;
}
