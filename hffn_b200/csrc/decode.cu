// Decode kernels of the forward: the cooperative mode at n <= 8 tokens per call (the decode steps of a language model,
// one call per layer). A call streams the layer's compact index / value arrays once (C4 bf16: 8.4 MB per projection)
// and does 2 n FLOPs per slot: HBM-bound in principle. Measured on B200 (ncu and per-phase %globaltimer stamps of an
// instrumented copy), a plain design is bound instead by shared-memory wavefronts of the random-row gathers and by
// barrier-separated passes with too little independent work per warp. Design:
//
//  - one CTA per SM, persistent over a contiguous range of output rows (neurons for up, output features for down);
//  - prologue, before griddepcontrol.wait (launched with programmatic dependent launch, the kernel starts while its
//    predecessor still runs): the CTA's slice of its own compact arrays is copied into shared memory by TMA bulk
//    copies (cp.async.bulk, completion counted on an mbarrier) when it fits, else sent to L2
//    (cp.async.bulk.prefetch.L2); the up kernel of a layer also sends a slice of the down projection's arrays to L2.
//    The compact arrays are constants of the layer; only the gathered table (x or act) is written by the predecessor.
//    The wait on the copies is bounded (2 s of %globaltimer): on expiry the CTA records code 301 in the decode error
//    flag (hffn_decode_error), waits (bounded) for its copies and returns;
//  - the gathered table is staged once per CTA after griddepcontrol.wait, [row][plane][copy] in 16-byte units (a
//    plane holds 8 bf16 or 4 float tokens of a row), read at L2 (ld.global.cg: the predecessor wrote it), replicated
//    COPIES times: lane L of a quarter-warp reads copy L mod COPIES; with 8 copies (up: x of 1024 features, 128 KB)
//    the eight 16-byte gathers of a quarter-warp always fall in distinct bank groups;
//  - warps walk rows independently: a row owned by one warp is reduced by its xor tree and stored by its lanes, with
//    no CTA-wide barrier; a row shared by `split` warps (few rows per CTA: the down projection) is combined through
//    shared memory under a named barrier of just those warps. 8 consecutive slots per lane per 16-byte index load
//    (from shared memory, or from L2 where the prologue put them); products accumulated in pairs by the packed
//    fma.rn.f32x2; a fixed summation order: per lane its head slot, its tail slot, its
//    chunks in order; the xor tree; the warps of a row in warp order. The same bits on every call.
//   up    act[r, t] = gelu(b_up[r] + sum of up_val[e] x[t, up_idx[e]] over the slots e of neuron r)  (z optional)
//   down  y[t, o] = (sum of out_val[q] act[out_hidden[q], t] over the edges q of output o) + b_down[o]
#include <algorithm>
#include <atomic>
#include <type_traits>

#include "common.cuh"

namespace hffn {
namespace dec {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxDevices = 64;
constexpr size_t kBudget = 132 * 1024;   // table copies + warp partials of one CTA
constexpr size_t kTotal = 200 * 1024;    // with the edge buffer (one CTA per SM)
constexpr int kMaxRowsPerCta = 256;
// shared memory after the table: warp partials [2][kWarps][8] floats, the CTA's offsets, the mbarrier and the staging
// record, then the edge buffer
constexpr size_t kPartBytes = 2 * kWarps * 8 * 4, kOffsBytes = ((kMaxRowsPerCta + 1) * 4 + 15) / 16 * 16;
constexpr size_t kHeaderBytes = kPartBytes + kOffsBytes + 64;
constexpr int kErrDecodeTimeout = 301;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ int g_decode_error;           // first error code recorded by a decode kernel (0: none)

struct Params {
  const void* src;      // up: x [n, rows_in] token-major; down: act [rows_in, n] hidden-major
  const int32_t* off;   // [rows_out + 1]
  const int16_t* idx;   // table row of each slot
  const void* val;      // value of each slot
  const void* bias;     // [rows_out]
  void* out;            // up: act [rows_out, n]; down: y [n, rows_out]
  float* z;             // up, optional: z [rows_out, n]
  const void* hint[2];  // optional: two more arrays the next kernel streams (the down projection's), prefetched
  int64_t hint_bytes[2];
  int rows_in, rows_out, n, copies, split;
  int buffer;           // bytes of the edge buffer after the table and the partials (0: none)
  int vector_src;       // down: act rows are whole 16-byte units (n fills the planes, 16-byte aligned base)
};

// The CTA's slots in shared memory: elements [i0, i1) of idx at byte 0 of the buffer, [v0, v1) of val at val_at
// (i1 = v1 = 0: none, the kernel reads its slots from global memory).
struct Staged {
  int i0, i1, v0, v1, val_at;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of parity `parity`; false once kWaitLimitNs have passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - start > kWaitLimitNs) return false;
  return true;
}

// Bytes [0, size) of global `src` into shared `dst`, completion counted on `bar` (both 16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t size, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(size), "r"(smem_u32(bar))
               : "memory");
}

// The 16-byte aligned interior of bytes [lo, hi) of an array with a 16-byte aligned base, prefetched into L2.
__device__ __forceinline__ void prefetch_l2(const void* base, int64_t lo, int64_t hi) {
  const int64_t a = (lo + 15) & ~int64_t(15), b = hi & ~int64_t(15);
  for (int64_t p = a; p < b; p += int64_t(1) << 20) {
    const uint32_t size = (uint32_t)min(b - p, int64_t(1) << 20);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const char*>(base) + p), "r"(size)
                 : "memory");
  }
}

__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void wait_for_predecessor() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Barrier of the `count` threads of one row group (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void group_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <typename T> struct Unit;
template <> struct Unit<__nv_bfloat16> {
  static constexpr int kTokens = 8;
  __device__ static __forceinline__ uint32_t bits(const __nv_bfloat16* p) {
    return __ldcg(reinterpret_cast<const unsigned short*>(p));
  }
  __device__ static __forceinline__ void unpack(const uint4 u, float* r) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      r[2 * k] = __uint_as_float(w[k] << 16);
      r[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  }
  __device__ static __forceinline__ uint4 pack(const uint32_t (&v)[8]) {
    return make_uint4(v[0] | (v[1] << 16), v[2] | (v[3] << 16), v[4] | (v[5] << 16), v[6] | (v[7] << 16));
  }
};
template <> struct Unit<float> {
  static constexpr int kTokens = 4;
  __device__ static __forceinline__ uint32_t bits(const float* p) { return __float_as_uint(__ldcg(p)); }
  __device__ static __forceinline__ void unpack(const uint4 u, float* r) {
    r[0] = __uint_as_float(u.x); r[1] = __uint_as_float(u.y); r[2] = __uint_as_float(u.z); r[3] = __uint_as_float(u.w);
  }
  __device__ static __forceinline__ uint4 pack(const uint32_t (&v)[4]) { return make_uint4(v[0], v[1], v[2], v[3]); }
};

// The 16-byte unit (row, plane) of the table: tokens plane * TPP + k, zero past n.
template <typename T, bool kUp>
__device__ __forceinline__ uint4 load_unit(const Params& p, int row, int plane) {
  constexpr int TPP = Unit<T>::kTokens;
  const T* src = static_cast<const T*>(p.src);
  if (!kUp && p.vector_src) return __ldcg(reinterpret_cast<const uint4*>(src + (int64_t)row * p.n + plane * TPP));
  uint32_t v[TPP];
#pragma unroll
  for (int k = 0; k < TPP; ++k) {
    const int t = plane * TPP + k;
    v[k] = 0u;
    if (t < p.n) v[k] = Unit<T>::bits(kUp ? src + (int64_t)t * p.rows_in + row : src + (int64_t)row * p.n + t);
  }
  return Unit<T>::pack(v);
}

// Pairs of float32 in one 64-bit register, multiplied and added by the packed fma.rn.f32x2 of sm_100: per element the
// same fused multiply-add, rounded once, as a scalar FFMA (the same bits), at half the instruction count.
using f32x2 = unsigned long long;

__device__ __forceinline__ f32x2 pair_bits(uint32_t lo, uint32_t hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}

__device__ __forceinline__ void fma2(f32x2& acc, f32x2 a, f32x2 b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

__device__ __forceinline__ float pair_lo(f32x2 v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float pair_hi(f32x2 v) { return __uint_as_float((uint32_t)(v >> 32)); }

// acc[k] += w * (tokens 2k, 2k + 1) of the 16-byte unit u (bf16: 8 tokens, 4 pairs; float: 4 tokens, 2 pairs).
__device__ __forceinline__ void fma_unit(f32x2* acc, f32x2 w2, uint4 u, __nv_bfloat16*) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) fma2(acc[k], w2, pair_bits(w[k] << 16, w[k] & 0xffff0000u));
}
__device__ __forceinline__ void fma_unit(f32x2* acc, f32x2 w2, uint4 u, float*) {
  fma2(acc[0], w2, pair_bits(u.x, u.y));
  fma2(acc[1], w2, pair_bits(u.z, u.w));
}

// acc += w * row `row` of the table (copy `copy`), all its planes.
template <typename T, int PLANES, int COPIES>
__device__ __forceinline__ void fma_row(f32x2* acc, float w, const uint4* table, int row, int copy) {
  const f32x2 w2 = pair_bits(__float_as_uint(w), __float_as_uint(w));
#pragma unroll
  for (int plane = 0; plane < PLANES; ++plane)
    fma_unit(acc + plane * (Unit<T>::kTokens / 2), w2, table[((size_t)row * PLANES + plane) * COPIES + copy],
             static_cast<T*>(nullptr));
}

// 8 slots from 16-byte aligned shared or global memory (the compact arrays: constants while a kernel runs).
__device__ __forceinline__ void load_idx8(const int16_t* p, int (&i)[8]) {
  const int4 raw = *reinterpret_cast<const int4*>(p);
  const int words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    i[2 * k] = (int)(int16_t)(words[k] & 0xffff);
    i[2 * k + 1] = (int)(int16_t)((uint32_t)words[k] >> 16);
  }
}

__device__ __forceinline__ void load_val8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void load_val8(const __nv_bfloat16* p, float (&v)[8]) {
  Unit<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(p), v);
}

template <typename T, int PLANES, int COPIES, bool kUp, bool kStoreZ>
__global__ void __launch_bounds__(kThreads, 1) gather_kernel(const Params p) {
  constexpr int NT = Unit<T>::kTokens * PLANES;
  constexpr int E = (int)sizeof(T);
  extern __shared__ __align__(16) unsigned char smem[];
  const size_t table_bytes = (size_t)p.rows_in * PLANES * COPIES * 16;
  uint4* table = reinterpret_cast<uint4*>(smem);                                   // [rows_in][PLANES][COPIES]
  float* part = reinterpret_cast<float*>(smem + table_bytes);                      // [2][kWarps][NT]
  int32_t* offs = reinterpret_cast<int32_t*>(smem + table_bytes + kPartBytes);     // off[r0 .. r1]
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + table_bytes + kPartBytes + kOffsBytes);
  Staged* staged = reinterpret_cast<Staged*>(bar + 2);
  unsigned char* buffer = smem + table_bytes + kHeaderBytes;
  const T* val = static_cast<const T*>(p.val);

  const int r0 = (int)((int64_t)p.rows_out * blockIdx.x / gridDim.x);
  const int r1 = (int)((int64_t)p.rows_out * (blockIdx.x + 1) / gridDim.x);
  for (int r = threadIdx.x; r <= r1 - r0; r += kThreads) offs[r] = __ldg(p.off + r0 + r);
  if (threadIdx.x == 0) {
    Staged st{0, 0, 0, 0, 0};
    if (r1 > r0) {
      const int64_t e0 = __ldg(p.off + r0), e1 = __ldg(p.off + r1), nnz = __ldg(p.off + p.rows_out);
      const int64_t ia = (2 * e0) & ~int64_t(15), ib = min((2 * e1 + 15) & ~int64_t(15), (2 * nnz) & ~int64_t(15));
      const int64_t va = (E * e0) & ~int64_t(15), vb = min((E * e1 + 15) & ~int64_t(15), (E * nnz) & ~int64_t(15));
      if (ib > ia && vb > va && (ib - ia) + (vb - va) <= p.buffer) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        st = Staged{(int)(ia / 2), (int)(ib / 2), (int)(va / E), (int)(vb / E), (int)(ib - ia)};
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                     "r"((uint32_t)((ib - ia) + (vb - va)))
                     : "memory");
        bulk_copy(buffer, reinterpret_cast<const char*>(p.idx) + ia, (uint32_t)(ib - ia), bar);
        bulk_copy(buffer + st.val_at, static_cast<const char*>(p.val) + va, (uint32_t)(vb - va), bar);
      } else {
        prefetch_l2(p.idx, e0 * 2, e1 * 2);
        prefetch_l2(p.val, e0 * E, e1 * E);
      }
    }
    *staged = st;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (p.hint[h] != nullptr)
        prefetch_l2(p.hint[h], p.hint_bytes[h] * blockIdx.x / gridDim.x, p.hint_bytes[h] * (blockIdx.x + 1) / gridDim.x);
  }
  allow_dependents();
  wait_for_predecessor();   // the table (x or act) is written by the preceding kernel
  if (r1 <= r0) return;

  for (int u = threadIdx.x; u < p.rows_in * PLANES; u += kThreads) {
    const int row = PLANES == 1 ? u : u >> 1, plane = PLANES == 1 ? 0 : u & 1;
    const uint4 v = load_unit<T, kUp>(p, row, plane);
    uint4* line = table + (size_t)u * COPIES;
#pragma unroll
    for (int c = 0; c < COPIES; ++c) line[(c + threadIdx.x) & (COPIES - 1)] = v;
  }
  __syncthreads();
  const Staged st = *staged;
  if (st.i1 > 0) {                     // the CTA's slots are on their way into shared memory
    const bool failed = !mbar_wait(bar, 0);
    if (__syncthreads_or(failed)) {
      if (threadIdx.x == 0) {
        atomicCAS(&g_decode_error, 0, kErrDecodeTimeout);
        mbar_wait(bar, 0);             // the copies land in this CTA's shared memory: let them finish (bounded)
      }
      return;
    }
  }
  const int16_t* sidx = reinterpret_cast<const int16_t*>(buffer) - st.i0;   // indexed by slot
  const T* sval = reinterpret_cast<const T*>(buffer + st.val_at) - st.v0;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int copy = lane & (COPIES - 1);
  const int split = p.split, per_pass = kWarps / split;
  const int group = warp / split, member = warp - group * split;
  const int glane = member * 32 + lane, stride = 8 * 32 * split;
  // the rows, with the slots read from the shared-memory copy (kStaged) or from global memory (L2); in the staged
  // walk a slot past the copied range (the last bytes of an array whose end is not 16-byte aligned) is read from
  // global memory
  auto walk = [&](auto staged_tag) {
    constexpr bool kStaged = decltype(staged_tag)::value;
    int pass = 0;
    for (int row = r0 + group; row - group < r1; row += per_pass, ++pass) {   // uniform over the group's warps
      f32x2 acc[NT / 2];
#pragma unroll
      for (int k = 0; k < NT / 2; ++k) acc[k] = 0ull;
      if (row < r1) {
        const int begin = offs[row - r0], end = offs[row + 1 - r0];
        const int body = min(end, (begin + 7) & ~7);
        const int body_end = max(body, end & ~7);
        auto one = [&](int e) {
          int id;
          float w;
          if (kStaged && e < st.i1) id = sidx[e];
          else id = p.idx[e];
          if (kStaged && e < st.v1) w = to_f(sval[e]);
          else w = to_f(val[e]);
          fma_row<T, PLANES, COPIES>(acc, w, table, id, copy);
        };
        if (begin + glane < body) one(begin + glane);
        if (body_end + glane < end) one(body_end + glane);
#pragma unroll 2
        for (int c = body + 8 * glane; c < body_end; c += stride) {
          int iv[8];
          float wv[8];
          if (kStaged && c + 8 <= st.i1) load_idx8(sidx + c, iv);
          else load_idx8(p.idx + c, iv);
          if (kStaged && c + 8 <= st.v1) load_val8(sval + c, wv);
          else load_val8(val + c, wv);
#pragma unroll
          for (int j = 0; j < 8; ++j) fma_row<T, PLANES, COPIES>(acc, wv[j], table, iv[j], copy);
        }
      }
      float sum[NT];
#pragma unroll
      for (int k = 0; k < NT / 2; ++k) {
        sum[2 * k] = warp_sum(pair_lo(acc[k]));
        sum[2 * k + 1] = warp_sum(pair_hi(acc[k]));
      }
      float mine = sum[0];                         // lane t < NT keeps the sum of token t
#pragma unroll
      for (int t = 1; t < NT; ++t) mine = lane == t ? sum[t] : mine;
      if (split > 1) {   // the row's warps in warp order, through shared memory (two buffers: alternate passes)
        float* slot = part + (size_t)(pass & 1) * kWarps * NT;
        if (lane < NT) slot[warp * NT + lane] = mine;
        group_barrier(1 + group, 32 * split);
        if (member == 0 && lane < NT) {
          mine = 0.f;
          for (int m = 0; m < split; ++m) mine += slot[(group * split + m) * NT + lane];
        }
      }
      if (row < r1 && member == 0 && lane < p.n) {   // lane t stores token t
        const float bias = to_f(static_cast<const T*>(p.bias)[row]);
        if constexpr (kUp) {
          const float zz = bias + mine;
          const int64_t at = (int64_t)row * p.n + lane;
          if constexpr (kStoreZ) p.z[at] = zz;
          static_cast<T*>(p.out)[at] = from_f<T>(gelu(zz));
        } else {
          static_cast<T*>(p.out)[(int64_t)lane * p.rows_out + row] = from_f<T>(mine + bias);
        }
      }
    }
  };
  if (st.i1 > 0) walk(std::true_type{});
  else walk(std::false_type{});
}

static int sm_count(int device) {   // device < kMaxDevices (checked by the caller)
  static std::atomic<int> counts[kMaxDevices];
  int c = counts[device].load(std::memory_order_relaxed);
  if (c == 0) {
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || c <= 0) c = 148;
    counts[device].store(c, std::memory_order_relaxed);
  }
  return c;
}

template <typename T, int PLANES, int COPIES, bool kUp, bool kZ>
static int launch(const Params& p, int grid, int device, cudaStream_t s, const char* what) {
  static std::atomic<uint64_t> opted_in{0};   // devices on which this kernel's shared-memory opt-in is set
  auto kernel = gather_kernel<T, PLANES, COPIES, kUp, kZ>;
  const size_t smem = (size_t)p.rows_in * PLANES * COPIES * 16 + kHeaderBytes + p.buffer;
  const uint64_t bit = uint64_t(1) << device;
  cudaError_t e = cudaSuccess;
  if (smem > 48 * 1024 && !(opted_in.load(std::memory_order_relaxed) & bit)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTotal);
    if (e != cudaSuccess) {
      set_error("%s: %s", what, cudaGetErrorString(e));
      return HFFN_ERR_CUDA;
    }
    opted_in.fetch_or(bit, std::memory_order_relaxed);
  }
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3((unsigned)grid);
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = smem;
  config.stream = s;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  e = cudaLaunchKernelEx(&config, kernel, p);
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return HFFN_ERR_CUDA;
  }
  return HFFN_OK;
}

// Largest power-of-two copy count (<= max_copies) whose table fits the budget; 0 if one copy does not fit.
static int copies_for(int rows_in, int planes, int max_copies) {
  for (int c = max_copies; c >= 1; c >>= 1)
    if ((size_t)rows_in * planes * c * 16 + kHeaderBytes <= kBudget) return c;
  return 0;
}

// Warps per row: a power of two, as many as the CTA's share of rows leaves idle warps for.
static int split_for(int rows_out, int grid) {
  const int rows_per_cta = (rows_out + grid - 1) / grid;
  int split = 1;
  while (split < kWarps && rows_per_cta * split * 2 <= kWarps) split <<= 1;
  return split;
}

template <typename T, int PLANES, bool kUp, bool kZ>
static int run(Params p, int max_copies, cudaStream_t s, const char* what) {
  const int copies = copies_for(p.rows_in, PLANES, max_copies);
  if (copies == 0) return kNotApplicable;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return kNotApplicable;
  const int grid = std::min(sm_count(device), p.rows_out);
  if ((p.rows_out + grid - 1) / grid > kMaxRowsPerCta) return kNotApplicable;
  p.copies = copies;
  p.split = split_for(p.rows_out, grid);
  const size_t fixed = (size_t)p.rows_in * PLANES * copies * 16 + kHeaderBytes;
  p.buffer = fixed < kTotal ? (int)((kTotal - fixed) & ~size_t(15)) : 0;
  switch (copies) {
    case 8: return launch<T, PLANES, 8, kUp, kZ>(p, grid, device, s, what);
    case 4: return launch<T, PLANES, 4, kUp, kZ>(p, grid, device, s, what);
    case 2: return launch<T, PLANES, 2, kUp, kZ>(p, grid, device, s, what);
    default: return launch<T, PLANES, 1, kUp, kZ>(p, grid, device, s, what);
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace dec

// The decode forms, tried by the cooperative mode at n <= 8: HFFN_OK / HFFN_ERR_CUDA when launched, kNotApplicable
// when the shape or the alignment does not fit them (the caller then runs its general cooperative kernels).
// `next_idx` / `next_val` (optional, `next_nnz` slots): the down projection's arrays, which the up kernel prefetches
// into L2 for the down kernel that follows it.
int launch_up_decode(int dtype, const void* x, const int32_t* off, const int16_t* idx, const void* w, const void* b,
                     void* act, float* z, int d, int H, int64_t n, cudaStream_t s, const int16_t* next_idx,
                     const void* next_val, int64_t next_nnz) {
  if (n < 1 || n > 8 || !dec::aligned16(idx) || !dec::aligned16(w)) return kNotApplicable;
  const int64_t elem = dtype == HFFN_F32 ? 4 : 2;
  const bool hint = next_idx != nullptr && next_val != nullptr && dec::aligned16(next_idx) && dec::aligned16(next_val);
  dec::Params p{x, off, idx, w, b, act, z, {hint ? next_idx : nullptr, hint ? next_val : nullptr},
                {2 * next_nnz, elem * next_nnz}, d, H, (int)n, 1, 1, 0, 0};
  if (dtype == HFFN_F32) {
    if (n <= 4) return z ? dec::run<float, 1, true, true>(p, 8, s, "up_decode")
                         : dec::run<float, 1, true, false>(p, 8, s, "up_decode");
    return z ? dec::run<float, 2, true, true>(p, 8, s, "up_decode") : dec::run<float, 2, true, false>(p, 8, s, "up_decode");
  }
  if (z) return kNotApplicable;
  return dec::run<__nv_bfloat16, 1, true, false>(p, 8, s, "up_decode");
}

int launch_down_decode(int dtype, const void* act, const int32_t* off, const int16_t* hid, const void* v,
                       const void* bias, void* y, int d, int H, int64_t n, cudaStream_t s) {
  if (n < 1 || n > 8 || !dec::aligned16(hid) || !dec::aligned16(v)) return kNotApplicable;
  const int elem = dtype == HFFN_F32 ? 4 : 2;
  const int tokens_per_unit = 16 / elem;
  const bool vector = dec::aligned16(act) && (n == tokens_per_unit || n == 2 * tokens_per_unit);
  dec::Params p{act, off, hid, v, bias, y, nullptr, {nullptr, nullptr}, {0, 0}, H, d, (int)n, 1, 1, 0,
                vector ? 1 : 0};
  if (dtype == HFFN_F32) {
    if (n <= 4) return dec::run<float, 1, false, false>(p, 1, s, "down_decode");
    return dec::run<float, 2, false, false>(p, 1, s, "down_decode");
  }
  return dec::run<__nv_bfloat16, 1, false, false>(p, 1, s, "down_decode");
}

}  // namespace hffn

extern "C" int hffn_decode_error(int32_t* value, int clear) {
  if (value == nullptr) {
    hffn::set_error("null pointer argument");
    return HFFN_ERR_ARGUMENT;
  }
  cudaError_t e = cudaMemcpyFromSymbol(value, hffn::dec::g_decode_error, sizeof(int32_t));
  if (e == cudaSuccess && clear) {
    const int32_t zero = 0;
    e = cudaMemcpyToSymbol(hffn::dec::g_decode_error, &zero, sizeof(int32_t));
  }
  if (e != cudaSuccess) {
    hffn::set_error("hffn_decode_error: %s", cudaGetErrorString(e));
    return HFFN_ERR_CUDA;
  }
  return HFFN_OK;
}
