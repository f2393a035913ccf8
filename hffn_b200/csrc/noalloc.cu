// hffn_forward_noalloc: the CUDA-core forward with its hidden-activation scratch in a fixed device array of this
// library, for callers that can hand the library only their input and output buffers and cannot allocate device
// memory (see include/hffn_b200.h for who they are).
//
// The scratch lives in `g_noalloc_scratch`, a file-scope __device__ array of kNoAllocScratchBytes (16 MiB) that every
// GPU loading this library holds until the process exits. Host code cannot use the array's name as a device address
// (on the host it names a host-side stand-in), so the first call on each device, with that device current, asks the
// runtime for the device address with cudaGetSymbolAddress and caches it; later calls reuse it. The cached address
// belongs to the device's primary context (the one the CUDA runtime and torch use): it stays valid while that context
// lives, not across cudaDeviceReset, and not for a caller that makes its own context current.
#include <mutex>

#include "common.cuh"

namespace hffn {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

int launch_up(int dtype, int mode, const void* x, const int32_t* off, const int16_t* idx, const void* w,
              const void* b, void* act, float* z, int d, int H, int64_t n, cudaStream_t s,
              const int16_t* next_idx = nullptr, const void* next_val = nullptr, int64_t next_nnz = 0);
int launch_down(int dtype, int mode, const void* act, const int32_t* off, const int16_t* hid, const void* v,
                const void* bias, void* y, int d, int H, int64_t n, cudaStream_t s);
int64_t max_staged_rows();
int check_shape(int dtype, int32_t d, int32_t H, int64_t n);   // abi.cu: the argument checks of hffn_forward
int check_layer(const hffn_layer* L);

static std::mutex g_scratch_mutex;
static void* g_scratch_address[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up on the first call per device).
static int scratch_address(void** out) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) {
    set_error("noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return HFFN_ERR_CUDA;
  }
  if (device < 0 || device >= kMaxDevices) {
    set_error("noalloc: device %d beyond the %d devices this entry tracks", device, kMaxDevices);
    return HFFN_ERR_ARGUMENT;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[device] == nullptr) {
    void* address = nullptr;
    e = cudaGetSymbolAddress(&address, g_noalloc_scratch);
    if (e != cudaSuccess || address == nullptr) {
      set_error("noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return HFFN_ERR_CUDA;
    }
    g_scratch_address[device] = address;
  }
  *out = g_scratch_address[device];
  return HFFN_OK;
}

}  // namespace hffn

using namespace hffn;

extern "C" {

int64_t hffn_forward_noalloc_max_bytes(void) { return (int64_t)kNoAllocScratchBytes; }

int hffn_forward_noalloc(int dtype, const hffn_layer* layer, const void* x, void* y, int64_t n, void* stream) {
  // the same refusals as hffn_forward (layer arrays, edge-count range, dtype, dimensions, token range)
  HFFN_TRY(check_layer(layer));
  HFFN_TRY(check_shape(dtype, layer->d_model, layer->d_ff, n));
  HFFN_REQUIRE(x && y, "null pointer argument");
  const int32_t d = layer->d_model, H = layer->d_ff;
  const int64_t elem = dtype == HFFN_F32 ? 4 : 2;
  HFFN_REQUIRE(n <= (int64_t)(kNoAllocScratchBytes / (elem * H)),
               "noalloc: d_ff x n x %lld bytes = %lld exceeds the %lld-byte scratch (at most %lld tokens for d_ff %d)",
               (long long)elem, (long long)(elem * H * n), (long long)kNoAllocScratchBytes,
               (long long)(kNoAllocScratchBytes / (elem * H)), H);
  const int up = hffn_up_mode(n, d), down = hffn_down_mode(n, H);
  HFFN_REQUIRE(up == HFFN_UP_COOP || d <= max_staged_rows(), "d_model %d exceeds the staged tile", d);
  HFFN_REQUIRE(down == HFFN_DOWN_COOP || H <= max_staged_rows(), "d_ff %d exceeds the staged tile", H);
  HFFN_TRY(bind_stream_device(stream));
  void* act = nullptr;
  HFFN_TRY(scratch_address(&act));
  // The up kernel writes every entry of act [d_ff, n] before the down kernel reads it: nothing needs clearing.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  HFFN_TRY(launch_up(dtype, up, x, layer->up_offsets, layer->up_idx, layer->up_val, layer->b_up, act, nullptr, d, H, n,
                     s));
  return launch_down(dtype, down, act, layer->out_offsets, layer->out_hidden, layer->out_val, layer->b_down, y, d, H, n,
                     s);
}

}  // extern "C"
