// Decode kernels of the forward: the cooperative mode at n <= 8 tokens per call (the decode steps of a language model,
// one call per layer). A call moves the layer's compact index / value streams once (C4 bf16: 8.4 MB per projection)
// and does 2 x n FLOPs per slot, so it is bound by HBM in principle. What bounds a plain kernel in practice is latency:
// a warp that walks its rows' slots with vector loads keeps 32 bytes per lane in flight, far from the megabytes HBM
// needs in flight to stream at full rate. Design:
//
//  - one CTA per SM, persistent over a contiguous range of output rows (neurons for up, output features for down),
//    whose slots are contiguous in the compact arrays;
//  - the CTA's slot range is cut into row-aligned windows of at most `window` slots; two windows are in flight at a
//    time in two shared-memory slots, each moved by one TMA bulk copy per array (cp.async.bulk, completion counted on
//    an mbarrier). Both are issued at kernel start, before griddepcontrol.wait, and the rest of the CTA's range is
//    sent to L2 (cp.async.bulk.prefetch.L2): the compact arrays are constants of the layer, only the gathered table
//    (x or act) is written by the preceding kernel. Launched with programmatic dependent launch, a kernel starts
//    while its predecessor still computes (shared memory is budgeted so that an up CTA and a down CTA fit one SM),
//    so one projection's stream overlaps the other's compute;
//  - the gathered table is staged once per CTA after griddepcontrol.wait, [row][plane][copy] in 16-byte units (a
//    plane holds 8 bf16 or 4 float tokens of a row), read at L2 (the predecessor wrote it); replicated when shared
//    memory allows: lane L of a quarter-warp reads copy L mod COPIES, which spreads its random rows over more bank
//    groups (8 copies: never a conflict);
//  - a row's slots are walked by `split` warps (a power of two picked per window), 8 consecutive slots per lane per
//    16-byte load from the window's slot; each warp sums its lanes with the xor tree and the row's warps are added in
//    warp order: a fixed summation order, the same bits on every call;
//  - every wait is bounded (2 s of %globaltimer): on expiry the CTA records kErrDecodeTimeout in the library's decode
//    error flag (hffn_decode_error), waits (bounded) for its copies in flight and returns.
//   up    act[r, t] = gelu(b_up[r] + sum of up_val[e] x[t, up_idx[e]] over the slots e of neuron r)  (z optional)
//   down  y[t, o] = (sum of out_val[q] act[out_hidden[q], t] over the edges q of output o) + b_down[o]
#include <algorithm>
#include <atomic>

#include "common.cuh"

namespace hffn {
namespace dec {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxDevices = 64;
constexpr int kMaxRowsPerCta = 256;          // off slice staged per CTA: rows_out <= 256 x SMs
constexpr size_t kUpBudget = 92 * 1024;      // an up CTA and a down CTA together stay within one SM's shared memory
constexpr size_t kDownBudget = 126 * 1024;
constexpr size_t kMinBuffer = 16 * 1024;     // smallest slot buffer worth the staging
constexpr int kErrDecodeTimeout = 301;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ int g_decode_error;               // first error code recorded by a decode kernel (0: none)

struct Params {
  const void* src;      // up: x [n, rows_in] token-major; down: act [rows_in, n] hidden-major
  const int32_t* off;   // [rows_out + 1]
  const int16_t* idx;   // table row of each slot
  const void* val;      // value of each slot
  const void* bias;     // [rows_out]
  void* out;            // up: act [rows_out, n]; down: y [n, rows_out]
  float* z;             // up, optional: z [rows_out, n]
  int rows_in, rows_out, n, copies;
  int buffer;           // bytes of the window buffer (a multiple of 32)
  int vector_src;       // down: act rows are whole 16-byte units (n fills the planes, 16-byte aligned base)
};

// One window of the CTA's rows, written by the producer thread before its copies. Elements [i0, i1) of idx and
// [v0, v1) of val are in shared memory at byte offsets idx_at and val_at of the buffer (i1 <= i0: none; those
// elements are read from global memory).
struct Window {
  int ra, rb;           // rows [ra, rb); ra == rb: no rows left
  int i0, i1, v0, v1;
  int idx_at, val_at;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
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

// The 16-byte unit (row, plane) of the table: tokens plane * TPP + k, zero past n. Read at L2 (ld.global.cg): the
// table was written by the preceding kernel, which may still have been running when this CTA started.
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

template <typename T, int PLANES>
__device__ __forceinline__ void load_row(const uint4* table, int copies, int row, int copy,
                                         float (&r)[Unit<T>::kTokens * PLANES]) {
#pragma unroll
  for (int plane = 0; plane < PLANES; ++plane)
    Unit<T>::unpack(table[((size_t)row * PLANES + plane) * copies + copy], r + plane * Unit<T>::kTokens);
}

__device__ __forceinline__ void unpack_idx8(const int4 raw, int (&i)[8]) {
  const int words[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    i[2 * k] = (int)(int16_t)(words[k] & 0xffff);
    i[2 * k + 1] = (int)(int16_t)((uint32_t)words[k] >> 16);
  }
}

// 8 values from 16-byte aligned memory (shared or global).
__device__ __forceinline__ void load_val8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load_val8(const __nv_bfloat16* p, float (&v)[8]) {
  Unit<__nv_bfloat16>::unpack(*reinterpret_cast<const uint4*>(p), v);
}

// Shared-memory layout of a CTA (byte offsets; every part 16-byte aligned).
struct Layout {
  size_t table, buffer, offs, part, windows, bars, total;
};

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

template <int PLANES>
__host__ __device__ inline Layout layout(int rows_in, int copies, int buffer) {
  Layout l;
  l.table = 0;
  l.buffer = align16((size_t)rows_in * PLANES * copies * 16);
  l.offs = l.buffer + (size_t)buffer;
  l.part = l.offs + align16((size_t)(kMaxRowsPerCta + 1) * 4);
  l.windows = l.part + (size_t)kWarps * 8 * 4;
  l.bars = l.windows + align16(2 * sizeof(Window));
  l.total = l.bars + 2 * 8;
  return l;
}

// Bytes a window of elements [e0, e1) takes in the buffer: each array's 16-byte aligned cover of the range.
__device__ __forceinline__ int64_t window_bytes(int64_t e0, int64_t e1, int elem) {
  return (((2 * e1 + 15) & ~int64_t(15)) - ((2 * e0) & ~int64_t(15))) +
         (((elem * e1 + 15) & ~int64_t(15)) - ((elem * e0) & ~int64_t(15)));
}

template <typename T, int PLANES, bool kUp, bool kStoreZ>
__global__ void __launch_bounds__(kThreads, 2) window_kernel(const Params p) {
  constexpr int NT = Unit<T>::kTokens * PLANES;
  constexpr int E = (int)sizeof(T);
  extern __shared__ __align__(16) unsigned char smem[];
  const Layout L = layout<PLANES>(p.rows_in, p.copies, p.buffer);
  uint4* table = reinterpret_cast<uint4*>(smem + L.table);
  unsigned char* buffer = smem + L.buffer;
  int32_t* offs = reinterpret_cast<int32_t*>(smem + L.offs);
  float* part = reinterpret_cast<float*>(smem + L.part);
  Window* windows = reinterpret_cast<Window*>(smem + L.windows);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);

  const int r0 = (int)((int64_t)p.rows_out * blockIdx.x / gridDim.x);
  const int r1 = (int)((int64_t)p.rows_out * (blockIdx.x + 1) / gridDim.x);
  for (int r = threadIdx.x; r <= r1 - r0; r += kThreads) offs[r] = __ldg(p.off + r0 + r);
  if (threadIdx.x == 0) {
    mbar_init(&bars[0]);
    mbar_init(&bars[1]);
  }
  __syncthreads();

  // Producer (thread 0). The CTA's whole range is one window in the whole buffer when it fits; otherwise row-aligned
  // windows of at most half the buffer alternate between its two halves (slot s at s x buffer / 2), two in flight.
  // issue(s) stages the next window from row `next` into slot s and always arrives once on the slot's barrier.
  const int64_t nnz = __ldg(p.off + p.rows_out);
  const bool whole = window_bytes(offs[0], offs[r1 - r0], E) <= p.buffer;
  const int capacity = whole ? p.buffer : p.buffer / 2;
  int next = r0;
  auto issue = [&](int s) {
    Window w{next, next, 0, 0, 0, 0, 0, 0};
    int rb = next;
    while (rb < r1 && window_bytes(offs[next - r0], offs[rb + 1 - r0], E) <= capacity) ++rb;
    if (rb == next && next < r1) rb = next + 1;            // a row larger than a slot: read from global memory
    w.rb = rb;
    uint32_t bytes = 0;
    const int64_t e0 = offs[next - r0], e1 = offs[rb - r0];
    if (rb > next && window_bytes(e0, e1, E) <= capacity) {
      const int64_t ia = (2 * e0) & ~int64_t(15), ib = min((2 * e1 + 15) & ~int64_t(15), (2 * nnz) & ~int64_t(15));
      const int64_t va = (E * e0) & ~int64_t(15), vb = min((E * e1 + 15) & ~int64_t(15), (E * nnz) & ~int64_t(15));
      const int at = whole ? 0 : s * capacity;
      w.idx_at = at;
      w.val_at = at + (int)max(int64_t(0), ib - ia);
      w.i0 = (int)(ia / 2);
      w.i1 = (int)(max(ia, ib) / 2);
      w.v0 = (int)(va / E);
      w.v1 = (int)(max(va, vb) / E);
      // the slot's previous contents were read through the generic proxy: order those reads before the async copies
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bytes = (uint32_t)(max(int64_t(0), ib - ia) + max(int64_t(0), vb - va));
      windows[s] = w;
      mbar_arrive_expect(&bars[s], bytes);
      if (ib > ia) bulk_copy(buffer + w.idx_at, reinterpret_cast<const char*>(p.idx) + ia, (uint32_t)(ib - ia), &bars[s]);
      if (vb > va)
        bulk_copy(buffer + w.val_at, static_cast<const char*>(p.val) + va, (uint32_t)(vb - va), &bars[s]);
    } else {
      windows[s] = w;
      mbar_arrive_expect(&bars[s], 0);
    }
    next = rb;
  };
  if (threadIdx.x == 0) {
    issue(0);
    if (!whole) issue(1);
    if (next < r1) {                                        // the rest of the CTA's range: on its way to L2
      prefetch_l2(p.idx, 2 * (int64_t)offs[next - r0], 2 * (int64_t)offs[r1 - r0]);
      prefetch_l2(p.val, E * (int64_t)offs[next - r0], E * (int64_t)offs[r1 - r0]);
    }
  }
  allow_dependents();
  wait_for_predecessor();   // the table (x or act) is written by the preceding kernel

  if (r1 > r0) {
    const int units = p.rows_in * PLANES;
    for (int u = threadIdx.x; u < units; u += kThreads) {
      const int row = PLANES == 1 ? u : u >> 1, plane = PLANES == 1 ? 0 : u & 1;
      const uint4 v = load_unit<T, kUp>(p, row, plane);
      uint4* line = table + (size_t)u * p.copies;
      for (int c = 0; c < p.copies; ++c) line[(c + threadIdx.x) & (p.copies - 1)] = v;
    }
  }
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int copy = lane & (p.copies - 1);
  const T* val = static_cast<const T*>(p.val);
  const int slots = whole ? 1 : 2;
  bool failed = false;
  for (int k = 0; r1 > r0; ++k) {
    const int s = k % slots;
    failed = !mbar_wait(&bars[s], (k / slots) & 1);
    if (__syncthreads_or(failed)) {
      failed = true;
      break;
    }
    const Window w = windows[s];
    if (w.ra >= w.rb) break;
    const int16_t* sidx = reinterpret_cast<const int16_t*>(buffer + w.idx_at) - w.i0;   // indexed by element
    const T* sval = reinterpret_cast<const T*>(buffer + w.val_at) - w.v0;
    const int rows = w.rb - w.ra;
    int split = 1;
    while (split < kWarps && rows * split * 2 <= kWarps) split <<= 1;
    const int per_pass = kWarps / split;
    const int group = warp / split, member = warp - group * split;
    const int glane = member * 32 + lane, stride = 8 * 32 * split;
    for (int base = w.ra; base < w.rb; base += per_pass) {   // uniform over the CTA
      const int row = base + group;
      float acc[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = 0.f;
      if (row < w.rb) {
        const int begin = offs[row - r0], end = offs[row + 1 - r0];
        const int body = min(end, (begin + 7) & ~7);
        const int body_end = max(body, end & ~7);
        auto one = [&](int e) {
          const int id = e >= w.i0 && e < w.i1 ? sidx[e] : (int)__ldg(p.idx + e);
          const float wv = to_f(e >= w.v0 && e < w.v1 ? sval[e] : val[e]);
          float r[NT];
          load_row<T, PLANES>(table, p.copies, id, copy, r);
#pragma unroll
          for (int t = 0; t < NT; ++t) acc[t] += wv * r[t];
        };
        if (begin + glane < body) one(begin + glane);
        if (body_end + glane < end) one(body_end + glane);
#pragma unroll 2
        for (int c = body + 8 * glane; c < body_end; c += stride) {
          int iv[8];
          float wv[8];
          unpack_idx8(c + 8 <= w.i1 ? *reinterpret_cast<const int4*>(sidx + c)
                                    : __ldg(reinterpret_cast<const int4*>(p.idx + c)), iv);
          load_val8(c + 8 <= w.v1 ? sval + c : val + c, wv);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float r[NT];
            load_row<T, PLANES>(table, p.copies, iv[j], copy, r);
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] += wv[j] * r[t];
          }
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0) part[warp * NT + t] = v;
      }
      __syncthreads();
      if (row < w.rb && member == 0 && lane < p.n) {
        float v = 0.f;
        for (int m = 0; m < split; ++m) v += part[(group * split + m) * NT + lane];
        const float bias = to_f(static_cast<const T*>(p.bias)[row]);
        if constexpr (kUp) {
          const float zz = bias + v;
          const int64_t at = (int64_t)row * p.n + lane;
          if constexpr (kStoreZ) p.z[at] = zz;
          static_cast<T*>(p.out)[at] = from_f<T>(gelu(zz));
        } else {
          static_cast<T*>(p.out)[(int64_t)lane * p.rows_out + row] = from_f<T>(v + bias);
        }
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) issue(s);                          // every thread is done with slot s
  }
  if (failed && threadIdx.x == 0) {
    atomicCAS(&g_decode_error, 0, kErrDecodeTimeout);
    // copies of this CTA still in flight land in its shared memory: wait for them (bounded) before the CTA retires
    for (int s = 0; s < 2; ++s)
      for (int parity = 0; parity < 2; ++parity) mbar_wait(&bars[s], parity);
  }
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

template <typename T, int PLANES, bool kUp, bool kZ>
static int launch(const Params& p, size_t smem, int grid, int device, cudaStream_t s, const char* what) {
  static std::atomic<uint64_t> opted_in{0};   // devices on which this kernel's shared-memory opt-in is set
  auto kernel = window_kernel<T, PLANES, kUp, kZ>;
  const uint64_t bit = uint64_t(1) << device;
  cudaError_t e = cudaSuccess;
  if (!(opted_in.load(std::memory_order_relaxed) & bit)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
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

// Shape the launch (grid, table copies, window buffer) within the budget and run it; kNotApplicable when it does not
// fit. The largest copy count (up to max_copies) that leaves at least kMinBuffer; the buffer takes the rest of the
// budget. Each CTA stages its whole share as one window when it fits the buffer (C4: up 57 KB of a 58 KB buffer with
// two copies of x; down 57 KB of a 60 KB buffer beside act), else row-aligned windows of half the buffer.
template <typename T, int PLANES, bool kUp, bool kZ>
static int plan_and_launch(Params p, size_t budget, int max_copies, cudaStream_t s, const char* what) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return kNotApplicable;
  const int grid = std::min(sm_count(device), p.rows_out);
  if ((p.rows_out + grid - 1) / grid > kMaxRowsPerCta) return kNotApplicable;
  for (int copies = max_copies; copies >= 1; copies >>= 1) {
    const size_t fixed = layout<PLANES>(p.rows_in, copies, 0).total;
    if (fixed + kMinBuffer > budget) continue;
    p.copies = copies;
    p.buffer = (int)((budget - fixed) & ~size_t(31));
    return launch<T, PLANES, kUp, kZ>(p, layout<PLANES>(p.rows_in, copies, p.buffer).total, grid, device, s, what);
  }
  return kNotApplicable;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace dec

// The decode forms, tried by the cooperative mode at n <= 8: HFFN_OK / HFFN_ERR_CUDA when launched, kNotApplicable
// when the shape or the alignment does not fit them (the caller then runs its general cooperative kernels).
int launch_up_decode(int dtype, const void* x, const int32_t* off, const int16_t* idx, const void* w, const void* b,
                     void* act, float* z, int d, int H, int64_t n, cudaStream_t s) {
  if (n < 1 || n > 8 || !dec::aligned16(idx) || !dec::aligned16(w)) return kNotApplicable;
  dec::Params p{x, off, idx, w, b, act, z, d, H, (int)n, 1, 0, 0};
  constexpr size_t B = dec::kUpBudget;
  if (dtype == HFFN_F32) {
    if (n <= 4)
      return z ? dec::plan_and_launch<float, 1, true, true>(p, B, 2, s, "up_decode")
               : dec::plan_and_launch<float, 1, true, false>(p, B, 2, s, "up_decode");
    return z ? dec::plan_and_launch<float, 2, true, true>(p, B, 2, s, "up_decode")
             : dec::plan_and_launch<float, 2, true, false>(p, B, 2, s, "up_decode");
  }
  if (z) return kNotApplicable;
  return dec::plan_and_launch<__nv_bfloat16, 1, true, false>(p, B, 2, s, "up_decode");
}

int launch_down_decode(int dtype, const void* act, const int32_t* off, const int16_t* hid, const void* v,
                       const void* bias, void* y, int d, int H, int64_t n, cudaStream_t s) {
  if (n < 1 || n > 8 || !dec::aligned16(hid) || !dec::aligned16(v)) return kNotApplicable;
  const int elem = dtype == HFFN_F32 ? 4 : 2;
  const int tokens_per_unit = 16 / elem;
  const bool vector = dec::aligned16(act) && (n == tokens_per_unit || n == 2 * tokens_per_unit);
  dec::Params p{act, off, hid, v, bias, y, nullptr, H, d, (int)n, 1, 0, vector ? 1 : 0};
  constexpr size_t B = dec::kDownBudget;
  if (dtype == HFFN_F32) {
    if (n <= 4) return dec::plan_and_launch<float, 1, false, false>(p, B, 1, s, "down_decode");
    return dec::plan_and_launch<float, 2, false, false>(p, B, 1, s, "down_decode");
  }
  return dec::plan_and_launch<__nv_bfloat16, 1, false, false>(p, B, 1, s, "down_decode");
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
