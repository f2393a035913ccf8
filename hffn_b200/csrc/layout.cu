// Device-side layout build of one layer: the output-major down edges (the reference's HFFNLayer.from_hidden_major,
// runtime/gpu/nvidia/common/kernels/hffn_cuda/runtime.py:55-67) and the two transposed supports of the training step
// (transposed_supports, runtime/gpu/nvidia/ffn/training/train_runtime.py:39-56), equal bit for bit to the host's
// stable sorts, so that a model loaded onto the GPU needs no host argsort.
//
// Each is a stable counting sort of a 16-bit key (an output feature, an input feature, a hidden neuron):
//   1 histogram: the slots are cut into B <= 256 chunks of consecutive slots; one CTA counts the keys of its chunk in
//     shared memory -> counts[b][k];
//   2 scan: per key, the chunks' counts in chunk order (the exclusive prefix is the key's first position among the
//     chunks before b), then the keys' totals in key order (the offsets array of the sorted layout);
//   3 ranks: one warp per chunk walks its slots in order, 32 at a time: slots of one key within the 32 are ranked by
//     __match_any_sync and the lane order, and a per-key counter in shared memory (offsets[k] + the chunks before b)
//     gives their positions. Position = offsets[k] + slots of key k before it in slot order: the stable order.
// Then gathers: the sorted position's source slot, its owner row (the neuron or output of the slot), its value.
// Keys outside [0, K) are skipped and counted in the caller's flag (no out-of-range access): a layer that passed
// hffn_validate_layout never sets it.
#include <algorithm>

#include "common.cuh"

namespace hffn {
namespace lay {

constexpr int kChunks = 256;
constexpr int kThreads = 512;

// owner[e] = r for every slot e of row r (offsets [rows + 1]); one warp per row. Slots outside [0, n) are skipped and
// flagged.
__global__ void owner_kernel(const int32_t* __restrict__ off, int rows, int64_t n, int16_t* __restrict__ owner,
                             int32_t* flag) {
  const int lane = threadIdx.x & 31;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += (gridDim.x * blockDim.x) >> 5) {
    const int begin = off[r], end = off[r + 1];
    if (lane == 0 && (begin < 0 || end > n || begin > end)) atomicOr(flag, 1);
    const int64_t stop = (int64_t)end < n ? (int64_t)end : n;
    for (int64_t e = max(begin, 0) + lane; e < stop; e += 32) owner[e] = (int16_t)r;
  }
}

__device__ __forceinline__ bool key_ok(int k, int K, int32_t* flag) {
  if (k >= 0 && k < K) return true;
  atomicOr(flag, 1);
  return false;
}

// counts[b][k] for the chunk b = blockIdx.x of `keys` (chunk slots [b C, min((b + 1) C, n))).
__global__ void histogram_kernel(const int16_t* __restrict__ keys, int64_t n, int64_t chunk, int K,
                                 int32_t* __restrict__ counts, int32_t* flag) {
  extern __shared__ int32_t hist[];
  for (int k = threadIdx.x; k < K; k += blockDim.x) hist[k] = 0;
  __syncthreads();
  const int64_t lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const int k = keys[i];
    if (key_ok(k, K, flag)) atomicAdd(&hist[k], 1);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < K; k += blockDim.x) counts[(int64_t)blockIdx.x * K + k] = hist[k];
}

// Per key: counts[b][k] -> the exclusive prefix over the chunks b; totals[k] = the key's count.
__global__ void column_scan_kernel(int32_t* __restrict__ counts, int chunks, int K, int32_t* __restrict__ totals) {
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < K; k += gridDim.x * blockDim.x) {
    int32_t running = 0;
    for (int b = 0; b < chunks; ++b) {
      const int32_t c = counts[(int64_t)b * K + k];
      counts[(int64_t)b * K + k] = running;
      running += c;
    }
    totals[k] = running;
  }
}

// offsets[0] = 0, offsets[k + 1] = offsets[k] + totals[k]: one CTA, chunked block scan.
__global__ void key_scan_kernel(const int32_t* __restrict__ totals, int K, int32_t* __restrict__ offsets) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) {
    carry = 0;
    offsets[0] = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  for (int base = 0; base < K; base += blockDim.x) {
    const int k = base + threadIdx.x;
    int32_t v = k < K ? totals[k] : 0;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {             // inclusive scan within the warp
      const int32_t u = __shfl_up_sync(0xffffffffu, v, s);
      if (lane >= s) v += u;
    }
    if (lane == 31) warp_sums[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int32_t w = lane < warps ? warp_sums[lane] : 0;
#pragma unroll
      for (int s = 1; s < 32; s <<= 1) {
        const int32_t u = __shfl_up_sync(0xffffffffu, w, s);
        if (lane >= s) w += u;
      }
      if (lane < warps) warp_sums[lane] = w;       // inclusive prefix of the warps' sums
    }
    __syncthreads();
    const int32_t before = carry + (warp > 0 ? warp_sums[warp - 1] : 0);
    if (k < K) offsets[k + 1] = before + v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = before + v;
    __syncthreads();
  }
}

// One warp per chunk: the sorted position of every slot of the chunk, in slot order; perm[position] = slot.
__global__ void rank_kernel(const int16_t* __restrict__ keys, int64_t n, int64_t chunk, int K,
                            const int32_t* __restrict__ base, const int32_t* __restrict__ offsets,
                            int32_t* __restrict__ perm) {
  extern __shared__ int32_t next[];               // per key: the next position of that key in this chunk
  const int b = blockIdx.x;
  for (int k = threadIdx.x; k < K; k += blockDim.x) next[k] = offsets[k] + base[(int64_t)b * K + k];
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  const int64_t lo = b * chunk, hi = min(n, lo + chunk);
  for (int64_t i0 = lo; i0 < hi; i0 += 32) {
    const int64_t i = i0 + lane;
    const bool live = i < hi;
    int k = live ? keys[i] : -1;
    if (k >= K) k = -1;                           // out of range: counted by the histogram, skipped here
    const unsigned same = __match_any_sync(0xffffffffu, k);
    const int rank = __popc(same & ((1u << lane) - 1));
    const int32_t first = k >= 0 ? next[k] : 0;
    __syncwarp();
    if (k >= 0) {
      perm[first + rank] = (int32_t)i;
      if (rank == __popc(same) - 1) next[k] = first + rank + 1;   // the key's last lane advances its counter
    }
    __syncwarp();
  }
}

// dst_owner[p] = owner[perm[p]] (int16), and optionally dst_pos[p] = perm[p] (int32) and dst_val[p] = val[perm[p]].
template <typename T>
__global__ void gather_kernel(const int32_t* __restrict__ perm, int64_t n, const int16_t* __restrict__ owner,
                              const T* __restrict__ val, int16_t* __restrict__ dst_owner, int32_t* __restrict__ dst_pos,
                              T* __restrict__ dst_val) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x) {
    const int32_t i = perm[p];
    if (i < 0 || i >= n) continue;                // a position no valid slot filled (the flag is set)
    if (dst_owner) dst_owner[p] = owner[i];
    if (dst_pos) dst_pos[p] = i;
    if (dst_val) dst_val[p] = val[i];
  }
}

struct Work {
  int32_t* perm;      // [max nnz]
  int16_t* owner;     // [max nnz] (two: the hidden-major owners, then the output-major owners)
  int16_t* owner2;
  int32_t* counts;    // [kChunks][max keys]
  int32_t* totals;    // [max keys]
};

inline int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

inline int64_t workspace(int K, int64_t nnz) {
  return align256(4 * nnz) + 2 * align256(2 * nnz) + align256((int64_t)4 * kChunks * K) + align256(4 * (int64_t)K);
}

inline Work carve(void* work, int K, int64_t nnz) {
  char* p = static_cast<char*>(work);
  Work w;
  w.perm = reinterpret_cast<int32_t*>(p);
  p += align256(4 * nnz);
  w.owner = reinterpret_cast<int16_t*>(p);
  p += align256(2 * nnz);
  w.owner2 = reinterpret_cast<int16_t*>(p);
  p += align256(2 * nnz);
  w.counts = reinterpret_cast<int32_t*>(p);
  p += align256((int64_t)4 * kChunks * K);
  w.totals = reinterpret_cast<int32_t*>(p);
  return w;
}

// The stable counting sort of `keys` (n slots, keys in [0, K)): offsets [K + 1] and w.perm.
static int sort(const int16_t* keys, int64_t n, int K, int32_t* offsets, const Work& w, int32_t* flag, cudaStream_t s) {
  const int chunks = (int)std::max<int64_t>(1, std::min<int64_t>(kChunks, ceil_div(n, 4096)));
  const int64_t chunk = std::max<int64_t>(1, ceil_div(n, chunks));
  const size_t smem = (size_t)K * 4;
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(histogram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  histogram_kernel<<<chunks, kThreads, smem, s>>>(keys, n, chunk, K, w.counts, flag);
  column_scan_kernel<<<(unsigned)ceil_div(K, 256), 256, 0, s>>>(w.counts, chunks, K, w.totals);
  key_scan_kernel<<<1, 1024, 0, s>>>(w.totals, K, offsets);
  if (n > 0) rank_kernel<<<chunks, 256, smem, s>>>(keys, n, chunk, K, w.counts, offsets, w.perm);
  return launch_status("layout sort");
}

static unsigned grid_for(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), 4 * 148)); }

}  // namespace lay
}  // namespace hffn

using namespace hffn;

extern "C" {

int64_t hffn_build_layout_workspace(int32_t d_model, int32_t d_ff, int64_t nnz_up, int64_t nnz_down) {
  if (d_model < 1 || d_ff < 1 || nnz_up < 0 || nnz_down < 0) return -1;
  return lay::workspace(std::max(d_model, d_ff), std::max(nnz_up, nnz_down));
}

int hffn_build_out_major(int dtype, int32_t d_model, int32_t d_ff, const int32_t* down_offsets,
                         const int16_t* down_idx, const void* down_val, int64_t nnz_down, int32_t* out_offsets,
                         int16_t* out_hidden, void* out_val, void* work, int32_t* flag, void* stream) {
  HFFN_REQUIRE(dtype == HFFN_F32 || dtype == HFFN_BF16, "unknown dtype %d", dtype);
  HFFN_REQUIRE(d_model >= 1 && d_model <= 32767 && d_ff >= 1 && d_ff <= 32767, "d_model %d / d_ff %d out of range",
               d_model, d_ff);
  HFFN_REQUIRE(nnz_down >= 0 && nnz_down < (int64_t(1) << 31), "edge count out of the int32 offset range");
  HFFN_REQUIRE(down_offsets && down_idx && down_val && out_offsets && out_hidden && out_val && work && flag,
               "null pointer argument");
  HFFN_TRY(bind_stream_device(stream));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const lay::Work w = lay::carve(work, std::max(d_model, d_ff), nnz_down);
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) {
    set_error("hffn_build_out_major: %s", cudaGetErrorString(e));
    return HFFN_ERR_CUDA;
  }
  lay::owner_kernel<<<(unsigned)ceil_div(d_ff, lay::kThreads / 32), lay::kThreads, 0, s>>>(down_offsets, d_ff,
                                                                                         nnz_down, w.owner, flag);
  HFFN_TRY(lay::sort(down_idx, nnz_down, d_model, out_offsets, w, flag, s));
  if (dtype == HFFN_F32)
    lay::gather_kernel<float><<<lay::grid_for(nnz_down), 256, 0, s>>>(
        w.perm, nnz_down, w.owner, static_cast<const float*>(down_val), out_hidden, nullptr, static_cast<float*>(out_val));
  else
    lay::gather_kernel<__nv_bfloat16><<<lay::grid_for(nnz_down), 256, 0, s>>>(
        w.perm, nnz_down, w.owner, static_cast<const __nv_bfloat16*>(down_val), out_hidden, nullptr,
        static_cast<__nv_bfloat16*>(out_val));
  return launch_status("hffn_build_out_major");
}

int hffn_build_supports(int32_t d_model, int32_t d_ff, const int32_t* up_offsets, const int16_t* up_idx,
                        int64_t nnz_up, const int32_t* out_offsets, const int16_t* out_hidden, int64_t nnz_down,
                        int32_t* in_offsets, int32_t* in_pos, int16_t* in_hidden, int32_t* hid_offsets,
                        int32_t* hid_pos, int16_t* hid_output, void* work, int32_t* flag, void* stream) {
  HFFN_REQUIRE(d_model >= 1 && d_model <= 32767 && d_ff >= 1 && d_ff <= 32767, "d_model %d / d_ff %d out of range",
               d_model, d_ff);
  HFFN_REQUIRE(nnz_up >= 0 && nnz_down >= 0 && nnz_up < (int64_t(1) << 31) && nnz_down < (int64_t(1) << 31),
               "edge counts out of the int32 offset range");
  HFFN_REQUIRE(up_offsets && up_idx && out_offsets && out_hidden && work && flag, "null pointer argument");
  HFFN_REQUIRE(in_offsets && in_pos && in_hidden && hid_offsets && hid_pos && hid_output, "null pointer argument");
  HFFN_TRY(bind_stream_device(stream));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const lay::Work w = lay::carve(work, std::max(d_model, d_ff), std::max(nnz_up, nnz_down));
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) {
    set_error("hffn_build_supports: %s", cudaGetErrorString(e));
    return HFFN_ERR_CUDA;
  }
  // up slots input-major (stable by input): their positions and owner neurons
  lay::owner_kernel<<<(unsigned)ceil_div(d_ff, lay::kThreads / 32), lay::kThreads, 0, s>>>(up_offsets, d_ff, nnz_up,
                                                                                         w.owner, flag);
  HFFN_TRY(lay::sort(up_idx, nnz_up, d_model, in_offsets, w, flag, s));
  lay::gather_kernel<float><<<lay::grid_for(nnz_up), 256, 0, s>>>(w.perm, nnz_up, w.owner, nullptr, in_hidden, in_pos,
                                                                     nullptr);
  // down edges hidden-major (stable by neuron over the output-major order): their positions and outputs
  lay::owner_kernel<<<(unsigned)ceil_div(d_model, lay::kThreads / 32), lay::kThreads, 0, s>>>(out_offsets, d_model,
                                                                                             nnz_down, w.owner2, flag);
  HFFN_TRY(lay::sort(out_hidden, nnz_down, d_ff, hid_offsets, w, flag, s));
  lay::gather_kernel<float><<<lay::grid_for(nnz_down), 256, 0, s>>>(w.perm, nnz_down, w.owner2, nullptr, hid_output,
                                                                       hid_pos, nullptr);
  return launch_status("hffn_build_supports");
}

}  // extern "C"
