// HFFN forward on the CUDA cores: fused up projection + bias + exact GELU (+ optional z store), then the down
// projection by output owners. Both read their gathered operand from a token tile staged in shared memory.
//
// Every hidden value and every output is written by one thread; the sums have a fixed order that depends on
// neither the grid nor the launch order (no atomic): the same bits on every call.
//   up    z[r, t] = b_up[r] + sum over the slots e of r, in slot order, of up_val[e] * x[t, up_idx[e]]
//         (coop: 32 lane-strided partial sums reduced by the xor tree, then added to the bias)
//   down  y[t, o] = (sum over the edges q of o, in output-major order, of out_val[q] * act[out_hidden[q], t]) + b_down[o]
// The reference's kernels (runtime/gpu/nvidia/common/kernels/hffn_cuda/kernels.py:102-191) read the gathered rows
// from L2 without staging; here a CTA stages one token tile of x (up) or of act (down), transposed to
// [feature][tile + 1] so that both the staging stores and the gathered loads are free of bank conflicts, and its
// warps walk the compact index/value streams against it.
#include <algorithm>

#include "common.cuh"

namespace hffn {

constexpr int kCoopThreads = 256;   // 8 warps, one neuron (or output) per warp
constexpr int kTileThreads = 512;   // 16 warps
constexpr int kSmemBudget = 200 * 1024;
constexpr int kTargetCtas = 4 * 148;  // four waves of one CTA per SM

// ---------------------------------------------------------------------------------------------------------------
// up

// Warp per neuron; the lanes stride its slots and keep one partial sum per token of a chunk of NT tokens; the
// chunks run in turn, so any n is accepted (the policy uses it for n <= 8).
template <typename T, int NT, bool kStoreZ>
__global__ void __launch_bounds__(kCoopThreads)
up_coop_kernel(const T* __restrict__ x, const int32_t* __restrict__ off, const int16_t* __restrict__ idx,
               const T* __restrict__ w, const T* __restrict__ b, T* __restrict__ act, float* __restrict__ z,
               int d, int H, int n) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (kCoopThreads / 32) + (threadIdx.x >> 5);
  if (r >= H) return;
  const int begin = off[r], end = off[r + 1];
  const float bias = to_f(b[r]);
  for (int t0 = 0; t0 < n; t0 += NT) {
    const T* xc = x + (int64_t)t0 * d;
    const int m = min(NT, n - t0);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    for (int e = begin + lane; e < end; e += 32) {
      const int i = idx[e];
      const float wv = to_f(w[e]);
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < m) acc[t] += wv * to_f(ldg(xc + (int64_t)t * d + i));
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float s = warp_sum(acc[t]);
      if (lane == t && t < m) {
        const float zz = bias + s;
        const int64_t at = (int64_t)r * n + t0 + t;
        if (kStoreZ) z[at] = zz;
        act[at] = from_f<T>(gelu(zz));
      }
    }
  }
}

// Token tile of TT tokens; a warp holds 32 / TT neurons, lane = (neuron of the warp, token of the tile).
template <typename T, int TT, bool kStoreZ>
__global__ void __launch_bounds__(kTileThreads)
up_tile_kernel(const T* __restrict__ x, const int32_t* __restrict__ off, const int16_t* __restrict__ idx,
               const T* __restrict__ w, const T* __restrict__ b, T* __restrict__ act, float* __restrict__ z,
               int d, int H, int n, int neurons_per_cta) {
  extern __shared__ float xs[];   // [d][TT + 1]
  constexpr int S = TT + 1, G = 32 / TT;
  const int t0 = blockIdx.y * TT;
  for (int k = threadIdx.x; k < TT * d; k += kTileThreads) {
    const int tt = k / d, i = k - tt * d;
    const int t = t0 + tt;
    xs[i * S + tt] = t < n ? to_f(x[(int64_t)t * d + i]) : 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TT, tt = lane - sub * TT;
  const int t = t0 + tt;
  const float* col = xs + tt;
  const int r_end = min(H, (blockIdx.x + 1) * neurons_per_cta);
  for (int r = blockIdx.x * neurons_per_cta + warp * G + sub; r < r_end; r += (kTileThreads / 32) * G) {
    int e = off[r];
    const int end = off[r + 1];
    float acc = to_f(b[r]);
    for (; e + 4 <= end; e += 4) {
      const int i0 = idx[e], i1 = idx[e + 1], i2 = idx[e + 2], i3 = idx[e + 3];
      const float w0 = to_f(w[e]), w1 = to_f(w[e + 1]), w2 = to_f(w[e + 2]), w3 = to_f(w[e + 3]);
      const float x0 = col[i0 * S], x1 = col[i1 * S], x2 = col[i2 * S], x3 = col[i3 * S];
      acc += w0 * x0;
      acc += w1 * x1;
      acc += w2 * x2;
      acc += w3 * x3;
    }
    for (; e < end; ++e) acc += to_f(w[e]) * col[idx[e] * S];
    if (t < n) {
      if (kStoreZ) z[(int64_t)r * n + t] = acc;
      act[(int64_t)r * n + t] = from_f<T>(gelu(acc));
    }
  }
}

// Decode form of the cooperative mode (n <= 8 tokens, the decode calls): HBM-bound on the compact index and value
// streams, so each lane streams 8 consecutive slots per load (16-byte index loads, 16- or 32-byte value loads) and
// the rows it gathers come from shared memory (up: x staged as [feature][NT] floats, one or two vector reads per
// slot) or from one vector load (down: the act row of a hidden neuron, n contiguous values). A row's slots before
// its first multiple of 8 and after its last run one per lane. Each sum still has a fixed order (per lane: its head
// slot, its tail slot, its chunks in order; then the xor tree; down: then the warps of the output in order).
constexpr int kDecodeThreads = 256;
constexpr int kDecodeWarps = kDecodeThreads / 32;
constexpr int kDecodeSplit = 4;        // warps per output in the down kernel

__device__ __forceinline__ void load_idx8(const int16_t* p, int (&i)[8]) {
  const int4 raw = __ldg(reinterpret_cast<const int4*>(p));
  const int words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    i[2 * k] = (int)(int16_t)(words[k] & 0xffff);
    i[2 * k + 1] = (int)(int16_t)((uint32_t)words[k] >> 16);
  }
}

__device__ __forceinline__ void load_val8(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p + 4));
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void load_val8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = __uint_as_float(words[k] << 16);
    v[2 * k + 1] = __uint_as_float(words[k] & 0xffff0000u);
  }
}

// NT floats of a shared-memory row (row start aligned to NT * 4 bytes).
template <int NT>
__device__ __forceinline__ void load_row_smem(const float* p, float (&r)[NT]) {
  if constexpr (NT >= 4) {
#pragma unroll
    for (int k = 0; k < NT; k += 4) {
      const float4 a = *reinterpret_cast<const float4*>(p + k);
      r[k] = a.x; r[k + 1] = a.y; r[k + 2] = a.z; r[k + 3] = a.w;
    }
  } else if constexpr (NT == 2) {
    const float2 a = *reinterpret_cast<const float2*>(p);
    r[0] = a.x; r[1] = a.y;
  } else {
    r[0] = *p;
  }
}

// The same for a row staged in bfloat16 (the bf16 runtimes: x is bf16, so staging it as is loses nothing): 16-byte
// rows at NT = 8, one load per slot, consecutive rows in distinct bank groups. Element k is the low half of its
// 32-bit word; the conversion is exact.
template <int NT>
__device__ __forceinline__ void load_row_smem(const __nv_bfloat16* p, float (&r)[NT]) {
  if constexpr (NT == 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      r[2 * k] = __uint_as_float(words[k] << 16);
      r[2 * k + 1] = __uint_as_float(words[k] & 0xffff0000u);
    }
  } else if constexpr (NT == 4) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    r[0] = __uint_as_float(raw.x << 16); r[1] = __uint_as_float(raw.x & 0xffff0000u);
    r[2] = __uint_as_float(raw.y << 16); r[3] = __uint_as_float(raw.y & 0xffff0000u);
  } else if constexpr (NT == 2) {
    const uint32_t raw = *reinterpret_cast<const uint32_t*>(p);
    r[0] = __uint_as_float(raw << 16); r[1] = __uint_as_float(raw & 0xffff0000u);
  } else {
    r[0] = __bfloat162float(*p);
  }
}

// The n <= NT values of a global row (hidden-major act: row start aligned to n * sizeof(T) bytes); vector loads when
// the row fills the tile (n == NT), else one load per value.
template <typename T, int NT>
__device__ __forceinline__ void load_row_global(const T* p, int n, float (&r)[NT]) {
  if (n == NT) {
    if constexpr (sizeof(T) == 4 && NT >= 4) {
#pragma unroll
      for (int k = 0; k < NT; k += 4) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p) + k / 4);
        r[k] = a.x; r[k + 1] = a.y; r[k + 2] = a.z; r[k + 3] = a.w;
      }
      return;
    } else if constexpr (sizeof(T) == 2 && NT == 8) {
      float v[8];
      load_val8(reinterpret_cast<const __nv_bfloat16*>(p), v);
#pragma unroll
      for (int k = 0; k < 8; ++k) r[k] = v[k];
      return;
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) r[t] = t < n ? to_f(ldg(p + t)) : 0.f;
}

template <typename T, int NT, bool kStoreZ>
__global__ void __launch_bounds__(kDecodeThreads)
up_decode_kernel(const T* __restrict__ x, const int32_t* __restrict__ off, const int16_t* __restrict__ idx,
                 const T* __restrict__ w, const T* __restrict__ b, T* __restrict__ act, float* __restrict__ z,
                 int d, int H, int n) {
  extern __shared__ __align__(16) unsigned char xs_raw[];
  T* xs = reinterpret_cast<T*>(xs_raw);       // [d][NT] in the storage type, zero past n
  // staged in batches of 8 elements per thread: the 8 loads first (in flight together), then the 8 stores
  const int total = NT * d;
  for (int k0 = 0; k0 < total; k0 += 8 * kDecodeThreads) {
    T v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int k = k0 + u * kDecodeThreads + (int)threadIdx.x;
      const int t = k / d, i = k - t * d;
      v[u] = k < total && t < n ? x[(int64_t)t * d + i] : from_f<T>(0.f);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int k = k0 + u * kDecodeThreads + (int)threadIdx.x;
      const int t = k / d, i = k - t * d;
      if (k < total) xs[i * NT + t] = v[u];
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = blockIdx.x * kDecodeWarps + warp; r < H; r += gridDim.x * kDecodeWarps) {
    const int begin = off[r], end = off[r + 1];
    const int body = min(end, (begin + 7) & ~7);
    const int body_end = max(body, end & ~7);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    auto one = [&](int e) {
      const float wv = to_f(w[e]);
      float rv[NT];
      load_row_smem<NT>(xs + (int)idx[e] * NT, rv);
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] += wv * rv[t];
    };
    if (begin + lane < body) one(begin + lane);
    if (body_end + lane < end) one(body_end + lane);
#pragma unroll 2
    for (int c = body + 8 * lane; c < body_end; c += 256) {
      int iv[8];
      float wv[8];
      load_idx8(idx + c, iv);
      load_val8(w + c, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float rv[NT];
        load_row_smem<NT>(xs + iv[j] * NT, rv);
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] += wv[j] * rv[t];
      }
    }
    const float bias = to_f(b[r]);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float sum = warp_sum(acc[t]);
      if (lane == t && t < n) {
        const float zz = bias + sum;
        const int64_t at = (int64_t)r * n + t;
        if (kStoreZ) z[at] = zz;
        act[at] = from_f<T>(gelu(zz));
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// down

// Warp per output; the lanes stride its edges, one partial sum per token of a chunk of NT tokens, chunks in turn.
template <typename T, int NT>
__global__ void __launch_bounds__(kCoopThreads)
down_coop_kernel(const T* __restrict__ act, const int32_t* __restrict__ off, const int16_t* __restrict__ hid,
                 const T* __restrict__ v, const T* __restrict__ bias, T* __restrict__ y, int d, int n) {
  const int lane = threadIdx.x & 31;
  const int o = blockIdx.x * (kCoopThreads / 32) + (threadIdx.x >> 5);
  if (o >= d) return;
  const int begin = off[o], end = off[o + 1];
  const float bo = to_f(bias[o]);
  for (int t0 = 0; t0 < n; t0 += NT) {
    const int m = min(NT, n - t0);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    for (int q = begin + lane; q < end; q += 32) {
      const T* row = act + (int64_t)hid[q] * n + t0;
      const float vv = to_f(v[q]);
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < m) acc[t] += vv * to_f(ldg(row + t));
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float s = warp_sum(acc[t]);
      if (lane == t && t < m) y[(int64_t)(t0 + t) * d + o] = from_f<T>(s + bo);
    }
  }
}

// Decode form of the down projection: kDecodeSplit warps per output share its edges (chunks of 8 dealt round-robin
// over the group's lanes), reduce them with the xor tree, and the output's first warp adds the warps' partial sums in
// warp order, then the bias.
template <typename T, int NT>
__global__ void __launch_bounds__(kDecodeThreads)
down_decode_kernel(const T* __restrict__ act, const int32_t* __restrict__ off, const int16_t* __restrict__ hid,
                   const T* __restrict__ v, const T* __restrict__ bias, T* __restrict__ y, int d, int n) {
  constexpr int kGroups = kDecodeWarps / kDecodeSplit;      // outputs per pass of a CTA
  __shared__ float part[kDecodeWarps][NT];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int group = warp / kDecodeSplit, member = warp - group * kDecodeSplit;
  const int glane = member * 32 + lane;
  for (int o0 = blockIdx.x * kGroups; o0 < d; o0 += gridDim.x * kGroups) {   // uniform over the CTA
    const int o = o0 + group;
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    if (o < d) {
      const int begin = off[o], end = off[o + 1];
      const int body = min(end, (begin + 7) & ~7);
      const int body_end = max(body, end & ~7);
      auto one = [&](int q) {
        const float vv = to_f(v[q]);
        float rv[NT];
        load_row_global<T, NT>(act + (int64_t)hid[q] * n, n, rv);
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] += vv * rv[t];
      };
      if (begin + glane < body) one(begin + glane);
      if (body_end + glane < end) one(body_end + glane);
#pragma unroll 2
      for (int c = body + 8 * glane; c < body_end; c += 8 * 32 * kDecodeSplit) {
        int hv[8];
        float vv[8];
        load_idx8(hid + c, hv);
        load_val8(v + c, vv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float rv[NT];
          load_row_global<T, NT>(act + (int64_t)hv[j] * n, n, rv);
#pragma unroll
          for (int t = 0; t < NT; ++t) acc[t] += vv[j] * rv[t];
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float sum = warp_sum(acc[t]);
      if (lane == 0) part[warp][t] = sum;
    }
    __syncthreads();
    if (o < d && member == 0 && lane < NT && lane < n) {
      float sum = 0.f;
#pragma unroll
      for (int m = 0; m < kDecodeSplit; ++m) sum += part[group * kDecodeSplit + m][lane];
      y[(int64_t)lane * d + o] = from_f<T>(sum + to_f(bias[o]));
    }
    __syncthreads();
  }
}

template <typename T, int TT>
__global__ void __launch_bounds__(kTileThreads)
down_tile_kernel(const T* __restrict__ act, const int32_t* __restrict__ off, const int16_t* __restrict__ hid,
                 const T* __restrict__ v, const T* __restrict__ bias, T* __restrict__ y, int d, int H, int n,
                 int outputs_per_cta) {
  extern __shared__ float hs[];   // [H][TT + 1]
  constexpr int S = TT + 1, G = 32 / TT;
  const int t0 = blockIdx.y * TT;
  for (int k = threadIdx.x; k < TT * H; k += kTileThreads) {
    const int r = k / TT, tt = k - r * TT;
    const int t = t0 + tt;
    hs[r * S + tt] = t < n ? to_f(act[(int64_t)r * n + t]) : 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TT, tt = lane - sub * TT;
  const int t = t0 + tt;
  const float* col = hs + tt;
  const int o_end = min(d, (blockIdx.x + 1) * outputs_per_cta);
  for (int o = blockIdx.x * outputs_per_cta + warp * G + sub; o < o_end; o += (kTileThreads / 32) * G) {
    int q = off[o];
    const int end = off[o + 1];
    float acc = 0.f;
    for (; q + 4 <= end; q += 4) {
      const int h0 = hid[q], h1 = hid[q + 1], h2 = hid[q + 2], h3 = hid[q + 3];
      const float v0 = to_f(v[q]), v1 = to_f(v[q + 1]), v2 = to_f(v[q + 2]), v3 = to_f(v[q + 3]);
      const float a0 = col[h0 * S], a1 = col[h1 * S], a2 = col[h2 * S], a3 = col[h3 * S];
      acc += v0 * a0;
      acc += v1 * a1;
      acc += v2 * a2;
      acc += v3 * a3;
    }
    for (; q < end; ++q) acc += to_f(v[q]) * col[hid[q] * S];
    if (t < n) y[(int64_t)t * d + o] = from_f<T>(acc + to_f(bias[o]));
  }
}

// ---------------------------------------------------------------------------------------------------------------
// tile choice and launchers

// Largest token tile TT in {32, 16, 8, 4, 2, 1} whose [rows][TT + 1] float32 staging fits the budget, capped by the
// next power of two of n; `half` asks for half of it (the "lane" / "tiled" modes).
static int tile_tokens(int64_t rows, int64_t n, bool half) {
  int tt = 32;
  while (tt > 1 && rows * (tt + 1) * 4 > kSmemBudget) tt >>= 1;
  int cap = 1;
  while (cap < n && cap < 32) cap <<= 1;
  tt = tt < cap ? tt : cap;
  if (half && tt > 1) tt >>= 1;
  return tt;
}

static int units_per_cta(int units, int64_t tiles, int per_pass) {
  int64_t blocks = (kTargetCtas + tiles - 1) / tiles;
  int64_t max_blocks = ceil_div(units, per_pass);
  if (blocks > max_blocks) blocks = max_blocks;
  if (blocks < 1) blocks = 1;
  return (int)ceil_div(units, blocks);
}

bool up_fits(int64_t d) { return d * 2 * 4 <= kSmemBudget; }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T, bool kZ>
static int launch_up_t(int mode, const T* x, const int32_t* off, const int16_t* idx, const T* w, const T* b, T* act,
                       float* z, int d, int H, int64_t n, cudaStream_t s) {
  if (mode == HFFN_UP_COOP && n <= 8 && aligned16(idx) && aligned16(w) && (int64_t)d * 8 * 4 <= kSmemBudget) {
    const int nn = (int)n;
    // one neuron per warp, every CTA resident at once (x staged in <= 64 KB per CTA for the decode shapes)
    const int grid = (int)std::min<int64_t>(ceil_div(H, kDecodeWarps), 8 * 148);
    auto run = [&](auto kernel, int nt) {
      const size_t smem = (size_t)d * nt * sizeof(T);
      if (smem > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      kernel<<<grid, kDecodeThreads, smem, s>>>(x, off, idx, w, b, act, z, d, H, nn);
    };
    if (n <= 1) run(up_decode_kernel<T, 1, kZ>, 1);
    else if (n <= 2) run(up_decode_kernel<T, 2, kZ>, 2);
    else if (n <= 4) run(up_decode_kernel<T, 4, kZ>, 4);
    else run(up_decode_kernel<T, 8, kZ>, 8);
    return launch_status("up_decode");
  }
  if (mode == HFFN_UP_COOP) {
    dim3 grid((unsigned)ceil_div(H, kCoopThreads / 32));
    const int nn = (int)n;
    if (n <= 1) up_coop_kernel<T, 1, kZ><<<grid, kCoopThreads, 0, s>>>(x, off, idx, w, b, act, z, d, H, nn);
    else if (n <= 2) up_coop_kernel<T, 2, kZ><<<grid, kCoopThreads, 0, s>>>(x, off, idx, w, b, act, z, d, H, nn);
    else if (n <= 4) up_coop_kernel<T, 4, kZ><<<grid, kCoopThreads, 0, s>>>(x, off, idx, w, b, act, z, d, H, nn);
    else up_coop_kernel<T, 8, kZ><<<grid, kCoopThreads, 0, s>>>(x, off, idx, w, b, act, z, d, H, nn);
    return launch_status("up_coop");
  }
  const int tt = tile_tokens(d, n, mode == HFFN_UP_LANE);
  const int64_t tiles = ceil_div(n, tt);
  const int per_pass = (kTileThreads / 32) * (32 / tt);
  const int npc = units_per_cta(H, tiles, per_pass);
  dim3 grid((unsigned)ceil_div(H, npc), (unsigned)tiles);
  const size_t smem = (size_t)d * (tt + 1) * 4;
  const int nn = (int)n;
#define HFFN_UP_TILE_CASE(TTV)                                                                                   \
  case TTV: {                                                                                                    \
    auto k = up_tile_kernel<T, TTV, kZ>;                                                                         \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                            \
    k<<<grid, kTileThreads, smem, s>>>(x, off, idx, w, b, act, z, d, H, nn, npc);                                \
    break;                                                                                                       \
  }
  switch (tt) {
    HFFN_UP_TILE_CASE(32)
    HFFN_UP_TILE_CASE(16)
    HFFN_UP_TILE_CASE(8)
    HFFN_UP_TILE_CASE(4)
    HFFN_UP_TILE_CASE(2)
    HFFN_UP_TILE_CASE(1)
  }
#undef HFFN_UP_TILE_CASE
  return launch_status("up_tile");
}

template <typename T>
static int launch_down_t(int mode, const T* act, const int32_t* off, const int16_t* hid, const T* v, const T* bias,
                         T* y, int d, int H, int64_t n, cudaStream_t s) {
  const int nn = (int)n;
  if (mode == HFFN_DOWN_COOP && n <= 8 && aligned16(hid) && aligned16(v) && aligned16(act)) {
    const int grid = (int)std::min<int64_t>(ceil_div(d, kDecodeWarps / kDecodeSplit), 4 * 148);
    if (n <= 1) down_decode_kernel<T, 1><<<grid, kDecodeThreads, 0, s>>>(act, off, hid, v, bias, y, d, nn);
    else if (n <= 2) down_decode_kernel<T, 2><<<grid, kDecodeThreads, 0, s>>>(act, off, hid, v, bias, y, d, nn);
    else if (n <= 4) down_decode_kernel<T, 4><<<grid, kDecodeThreads, 0, s>>>(act, off, hid, v, bias, y, d, nn);
    else down_decode_kernel<T, 8><<<grid, kDecodeThreads, 0, s>>>(act, off, hid, v, bias, y, d, nn);
    return launch_status("down_decode");
  }
  if (mode == HFFN_DOWN_COOP) {
    dim3 grid((unsigned)ceil_div(d, kCoopThreads / 32));
    if (n <= 1) down_coop_kernel<T, 1><<<grid, kCoopThreads, 0, s>>>(act, off, hid, v, bias, y, d, nn);
    else if (n <= 2) down_coop_kernel<T, 2><<<grid, kCoopThreads, 0, s>>>(act, off, hid, v, bias, y, d, nn);
    else if (n <= 4) down_coop_kernel<T, 4><<<grid, kCoopThreads, 0, s>>>(act, off, hid, v, bias, y, d, nn);
    else down_coop_kernel<T, 8><<<grid, kCoopThreads, 0, s>>>(act, off, hid, v, bias, y, d, nn);
    return launch_status("down_coop");
  }
  const int tt = tile_tokens(H, n, mode == HFFN_DOWN_TILED);
  const int64_t tiles = ceil_div(n, tt);
  const int per_pass = (kTileThreads / 32) * (32 / tt);
  const int opc = units_per_cta(d, tiles, per_pass);
  dim3 grid((unsigned)ceil_div(d, opc), (unsigned)tiles);
  const size_t smem = (size_t)H * (tt + 1) * 4;
#define HFFN_DOWN_TILE_CASE(TTV)                                                                                 \
  case TTV: {                                                                                                    \
    auto k = down_tile_kernel<T, TTV>;                                                                           \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                            \
    k<<<grid, kTileThreads, smem, s>>>(act, off, hid, v, bias, y, d, H, nn, opc);                                \
    break;                                                                                                       \
  }
  switch (tt) {
    HFFN_DOWN_TILE_CASE(32)
    HFFN_DOWN_TILE_CASE(16)
    HFFN_DOWN_TILE_CASE(8)
    HFFN_DOWN_TILE_CASE(4)
    HFFN_DOWN_TILE_CASE(2)
    HFFN_DOWN_TILE_CASE(1)
  }
#undef HFFN_DOWN_TILE_CASE
  return launch_status("down_tile");
}

int launch_up_decode(int dtype, const void* x, const int32_t* off, const int16_t* idx, const void* w, const void* b,
                     void* act, float* z, int d, int H, int64_t n, cudaStream_t s, const int16_t* next_idx,
                     const void* next_val, int64_t next_nnz);
int launch_down_decode(int dtype, const void* act, const int32_t* off, const int16_t* hid, const void* v,
                       const void* bias, void* y, int d, int H, int64_t n, cudaStream_t s);

int launch_up(int dtype, int mode, const void* x, const int32_t* off, const int16_t* idx, const void* w,
              const void* b, void* act, float* z, int d, int H, int64_t n, cudaStream_t s, const int16_t* next_idx,
              const void* next_val, int64_t next_nnz) {
  if (mode == HFFN_UP_COOP && n <= 8) {     // the decode kernels (decode.cu) when the shape fits them
    const int status = launch_up_decode(dtype, x, off, idx, w, b, act, z, d, H, n, s, next_idx, next_val, next_nnz);
    if (status != kNotApplicable) return status;
  }
  if (dtype == HFFN_F32) {
    auto f = z ? launch_up_t<float, true> : launch_up_t<float, false>;
    return f(mode, (const float*)x, off, idx, (const float*)w, (const float*)b, (float*)act, z, d, H, n, s);
  }
  using B = __nv_bfloat16;
  auto f = z ? launch_up_t<B, true> : launch_up_t<B, false>;
  return f(mode, (const B*)x, off, idx, (const B*)w, (const B*)b, (B*)act, z, d, H, n, s);
}

int launch_down(int dtype, int mode, const void* act, const int32_t* off, const int16_t* hid, const void* v,
                const void* bias, void* y, int d, int H, int64_t n, cudaStream_t s) {
  if (mode == HFFN_DOWN_COOP && n <= 8) {
    const int status = launch_down_decode(dtype, act, off, hid, v, bias, y, d, H, n, s);
    if (status != kNotApplicable) return status;
  }
  if (dtype == HFFN_F32)
    return launch_down_t<float>(mode, (const float*)act, off, hid, (const float*)v, (const float*)bias, (float*)y, d,
                                H, n, s);
  using B = __nv_bfloat16;
  return launch_down_t<B>(mode, (const B*)act, off, hid, (const B*)v, (const B*)bias, (B*)y, d, H, n, s);
}

// Largest d_model / d_ff whose smallest staging tile ([rows][2] float32) fits shared memory.
int64_t max_staged_rows() { return kSmemBudget / (2 * 4); }

}  // namespace hffn
