// HFFN forward on the 5th-generation tensor cores (tcgen05, TMEM accumulators, TMA operand staging), for supports
// dense enough that a masked dense tile beats the gather path: W_up and W_down are materialised once as dense
// matrices with zeros off the support ("densified"), and the layer becomes two GEMMs with fused epilogues:
//   up    Z[r, t] = sum_i W_up[r, i] x[t, i]       epilogue: + b_up[r], exact GELU, (z store), act store
//   down  Y[o, t] = sum_r W_down[o, r] act[t, r]   epilogue: + b_down[o], y store (token-major)
// Both are D[M = features, N = tokens] = A[M, K] * B[N, K]^T with A and B K-major; the accumulator tile is
// 128 features x BN tokens in TMEM (lane = feature, column = token).
//
// Precision. bfloat16 storage: one bf16 MMA (kind::f16, fp32 accumulate). float32 storage: the 3xTF32 split
// (a published method: Ootomo & Yokota 2022, and CUTLASS's "3xTF32" fast-accurate GEMM): every operand v is stored as
// two tf32 values hi = rna_tf32(v), lo = rna_tf32(v - hi), and a*b is computed as hi*hi + hi*lo + lo*hi (the lo*lo term,
// ~2^-22 relative, is dropped), with fp32 accumulation in TMEM: products carry ~2^-21 relative error instead of tf32's
// 2^-11. The conversions are the PTX instruction cvt.rna.tf32.f32.
//
// float32 storage, fp16x3 format (the float32 forward's default): the same three-product split with fp16 parts, which
// carry the same 11-bit significand as tf32 but run at the f16 MMA rate (twice tf32's) and take half the bytes. fp16's
// 5-bit exponent is met by power-of-two scales that leave every product exact: each weight row r is stored scaled by
// 2^e_r (its largest |value| into [2^14, 2^15)), each token's x row by 2^e_t likewise, and each token's act row by a
// power of two that maps a bound of |act| below 2^15 (|gelu(z)| <= max(|z|, 0.17), |z| <= max_r ||W_up[r]||_1 max|x_t|
// + max|b_up|). The epilogues multiply the accumulator by 2^-(e_r + e_t) before the bias. An element far below its
// row's largest loses significand bits to fp16's subnormal range only where its error is below 2^-40 of that row's
// largest, far under float32's own rounding of the dot product.
//
// float32 accumulation runs in K chunks of 128 values (48 MMAs) into fresh TMEM accumulators that the epilogue adds
// into float32 registers with round-to-nearest: the accumulation bias of the tensor core stays bounded by one chunk.
//
// Kernel shape: persistent, one CTA per SM: warp 0 issues the TMA loads (lane 0 arms each stage, then one box per
// lane), warp 1 owns the TMEM allocation and issues the MMAs (one elected thread), EW = 8 or 16 epilogue warps
// follow (one TMEM lane = one feature row per thread, EW / 4 warps per lane quarter splitting the token columns).
// Two accumulator buffers in TMEM let the epilogue of one tile overlap the MMAs of the next. Shared-memory stages are
// recycled through mbarriers (full: TMA -> MMA, empty: MMA commit -> TMA); every wait
// is bounded by a 2 s timer after which the kernel records an error code, stops issuing work, waits (bounded) for its
// own copies in flight, frees its TMEM and returns. No TMA multicast is used.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <atomic>
#include <climits>

#include "common.cuh"

namespace hffn {
namespace tc {

// warp 0 TMA, warp 1 MMA, then EW epilogue warps (EW / 4 per TMEM lane quarter, splitting the token columns)
__host__ __device__ constexpr int threads_for(int ew) { return 64 + 32 * ew; }
constexpr int BM = 128;                  // features per tile (TMEM lanes)
constexpr uint64_t kWaitNs = 2000000000ull;

// kUp: + b_up, GELU, act (and z) stores. kDown: + bias (optional), y store. kDownMse: + b_down, y store, the MSE
// gradient gy = scale (y - target) as tf32 hi/lo, per-thread partial sums of (y - target)^2 and of gy per output.
// kGradHidden: gz = acc * gelu'(z) as tf32 hi/lo, per-thread partial sums of gz per neuron. kSampled: the weight
// gradient sampled at the support entries of each row (CSR, columns ascending), stored and / or applied by AdamW, the
// dense operand refreshed with the new value.
// kDownPeer: as kDown, the value of token t stored into the buffer of the rank that owns t (peer memory over NVLink):
// peers[t / tokens_per_owner] + (t % tokens_per_owner) * M + row.
// kUpT: kUp of the training step, which also stores act^T (the feature-major copy).
enum Epilogue { kUp = 0, kDown = 1, kDownMse = 2, kGradHidden = 3, kSampled = 4, kDownPeer = 5, kUpT = 6 };

constexpr int kMaxPeers = 8;

// error codes written to the kernel's error flag
constexpr int kErrTimeoutProducer = 101, kErrTimeoutMma = 102, kErrTimeoutEpilogue = 103;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// Wait for the phase of parity `parity` to complete; false after the time limit (or once another role has aborted).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - start > limit_ns) return false;
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c_inner, int c_row) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c_inner), "r"(c_row)
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile in the swizzle layout TMA writes for rows of RB bytes
// (RB = 128: 128-byte swizzle, layout type 2; RB = 64: 64-byte swizzle, layout type 4): 8-row groups 8 x RB bytes
// apart (stride byte offset), descriptor version 1.
template <int RB>
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  static_assert(RB == 128 || RB == 64, "row bytes");
  constexpr uint64_t layout = RB == 128 ? 2 : 4;
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)((8 * RB) >> 4) << 32) |
         ((uint64_t)1 << 46) | (layout << 61);
}

// Shared-memory matrix descriptor of an MN-major 32-bit (tf32) operand. The only MN-major layout of tf32 operands is the
// 128-byte swizzle with 32-byte atomicity (layout type 1): atoms of 128 bytes of MN (32 elements) x 4 K rows, the
// 32-byte granules of a row XORed with the row index mod 4 (TMA's CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B writes it).
// Blocks of 32 MN elements x BK K rows: MN blocks `lbo` bytes apart (leading byte offset), 4-row K groups 512 bytes
// apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t addr, uint32_t lbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) | ((uint64_t)(512 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)1 << 61);
}

// Instruction descriptor: fp32 accumulator, A/B format (tf32 = 2, bf16 = 1), A/B major (0 K, 1 MN), N = bn, M = 128.
__host__ __device__ constexpr uint32_t instr_desc(int fmt, int bn, bool a_mn = false, bool b_mn = false) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

template <bool kBf16>
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  if constexpr (kBf16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
  }
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 TMEM lanes x 32 consecutive 32-bit columns: register j of lane l = column (taddr.col + j) of lane (taddr.lane + l).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ float tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}

struct EpilogueArgs {
  const void* bias;   // [M] of the storage type (NULL: none)
  void* out_hi;       // kUp: act (hi part for fp32) [N, M]; kDown / kDownMse: y [N, M]; kGradHidden: gz hi [N, M]
  void* out_lo;       // kUp fp32: act lo part; kGradHidden: gz lo
  float* z;           // kUp fp32, optional: pre-activations [N, M]
  // kDownMse
  const float* target;   // [N, M]
  float* gy_hi;          // [N, M]
  float* gy_lo;
  float scale;           // 2 / (N_total M)
  float* loss_partial;   // [num_n * parts, M]
  float* col_partial;    // kDownMse / kGradHidden: [num_n * parts, M] partial sums of gy / gz per row
  // kGradHidden
  const float* z_in;     // [N, M] pre-activations of the forward
  // kUpT / kDownMse / kGradHidden (float32): feature-major copies [M, t_ld] of the tf32 hi / lo outputs (act, gy,
  // gz), the K-major operands of the sampled weight-gradient GEMMs (t_ld: a multiple of 4 >= N)
  float* t_hi;
  float* t_lo;
  int64_t t_ld;
  // kSampled: the support of each row as a bitmask over the N columns (32-column words, mask_ld words per row) and,
  // per word, the compact index of the row's first support entry at or after the word's first column; compact
  // values / gradient / moments
  const uint32_t* mask;
  const int32_t* first;
  int64_t mask_ld;
  float* value;
  float* grad;           // NULL: not stored
  float* m;
  float* v;
  float* dense_hi;       // [M, N] refreshed with the updated value (tf32 hi / lo)
  float* dense_lo;
  int adam;              // apply AdamW
  hffn_adamw_step step;
  // kDownPeer
  void* peers[kMaxPeers];
  int64_t tokens_per_owner;
  int64_t rows;          // M
  // fp16x3 (kUp, kDown): the accumulator of (row, token t) is scaled back by row_inv[row] times the token's inverse
  // scale; kUp stores act 2^a_t as fp16 hi / lo parts into out_hi / out_lo. The token scales sit in the token's
  // packet: tok_tab + t tok_stride holds {x_inv, act_mul = 2^a_t, act_inv = 2^-a_t} (kUp reads the first two, kDown
  // the third).
  const float* row_inv;
  const float* tok_tab;
  int64_t tok_stride;
};

// One value of the output tile: bias added, then (up) GELU and the stores of act (float32: tf32 hi and lo parts) and
// of z, or (down) the store of y. Out of line: the epilogue calls it once per value, and an inlined copy per value
// of an unrolled tile overflows the instruction cache.
template <bool kBf16, int EPI>
__device__ __forceinline__ float2 emit_one(const EpilogueArgs* e, int64_t at, float s, float& hi, float& lo) {
  if constexpr (EPI == kUp || EPI == kUpT) {
    if (!kBf16 && e->z) e->z[at] = s;
    const float h = gelu(s);
    if constexpr (kBf16) {
      reinterpret_cast<__nv_bfloat16*>(e->out_hi)[at] = __float2bfloat16_rn(h);
    } else {
      hi = tf32_rna(h);
      lo = tf32_rna(h - hi);
      reinterpret_cast<float*>(e->out_hi)[at] = hi;
      reinterpret_cast<float*>(e->out_lo)[at] = lo;
    }
    return make_float2(0.f, 0.f);
  } else if constexpr (EPI == kDown) {
    if constexpr (kBf16) reinterpret_cast<__nv_bfloat16*>(e->out_hi)[at] = __float2bfloat16_rn(s);
    else reinterpret_cast<float*>(e->out_hi)[at] = s;
    return make_float2(0.f, 0.f);
  } else if constexpr (EPI == kDownPeer) {
    const int64_t t = at / e->rows, row = at - t * e->rows;
    const int64_t owner = t / e->tokens_per_owner, local = t - owner * e->tokens_per_owner;
    const int64_t dst = local * e->rows + row;
    if constexpr (kBf16) reinterpret_cast<__nv_bfloat16*>(e->peers[owner])[dst] = __float2bfloat16_rn(s);
    else reinterpret_cast<float*>(e->peers[owner])[dst] = s;
    return make_float2(0.f, 0.f);
  } else if constexpr (EPI == kDownMse) {
    reinterpret_cast<float*>(e->out_hi)[at] = s;
    const float diff = s - e->target[at];
    const float g = e->scale * diff;
    hi = tf32_rna(g);
    lo = tf32_rna(g - hi);
    e->gy_hi[at] = hi;
    e->gy_lo[at] = lo;
    return make_float2(diff * diff, g);
  } else {   // kGradHidden
    const float g = s * gelu_grad(e->z_in[at]);
    hi = tf32_rna(g);
    lo = tf32_rna(g - hi);
    reinterpret_cast<float*>(e->out_hi)[at] = hi;
    reinterpret_cast<float*>(e->out_lo)[at] = lo;
    return make_float2(0.f, g);
  }
}

// Four values of one output row (tokens t0 .. t0 + 3 at `stride` apart, `count` of them valid): bias added, then
// the epilogue's stores; returns the partial sums it contributes (loss, column sum). The four values are independent,
// so their chains interleave. Out of line (emit4) where a thread holds 128 values (an inlined copy per value of the
// unrolled tile overflows the instruction cache), inlined (emit4_inline) where it holds at most 64 (measured faster:
// no call, no registers saved around it).
template <bool kBf16, int EPI>
__device__ __forceinline__ float2 emit4_inline(const EpilogueArgs* e, int64_t at, int64_t stride, int count,
                                               float bias, float v0, float v1, float v2, float v3) {
  float2 acc = make_float2(0.f, 0.f), r;
  float hi, lo;
  if (count >= 4) {
    r = emit_one<kBf16, EPI>(e, at, v0 + bias, hi, lo); acc.x += r.x; acc.y += r.y;
    r = emit_one<kBf16, EPI>(e, at + stride, v1 + bias, hi, lo); acc.x += r.x; acc.y += r.y;
    r = emit_one<kBf16, EPI>(e, at + 2 * stride, v2 + bias, hi, lo); acc.x += r.x; acc.y += r.y;
    r = emit_one<kBf16, EPI>(e, at + 3 * stride, v3 + bias, hi, lo); acc.x += r.x; acc.y += r.y;
    return acc;
  }
  if (count > 0) { r = emit_one<kBf16, EPI>(e, at, v0 + bias, hi, lo); acc.x += r.x; acc.y += r.y; }
  if (count > 1) { r = emit_one<kBf16, EPI>(e, at + stride, v1 + bias, hi, lo); acc.x += r.x; acc.y += r.y; }
  if (count > 2) { r = emit_one<kBf16, EPI>(e, at + 2 * stride, v2 + bias, hi, lo); acc.x += r.x; acc.y += r.y; }
  return acc;
}

// The same for the training epilogues that also store feature-major copies (kUpT, kDownMse, kGradHidden): the four
// values of row `row`, tokens t0 .. t0 + 3 (t0 a multiple of 4), and their tf32 hi / lo parts into the copies as one
// 16-byte store each.
template <bool kBf16, int EPI>
__device__ __forceinline__ float2 emit4t_inline(const EpilogueArgs* e, int row, int t0, int M, int N, float bias,
                                                float v0, float v1, float v2, float v3) {
  const int64_t at = (int64_t)t0 * M + row;
  const int count = N - t0;
  const float v[4] = {v0, v1, v2, v3};
  float h[4] = {0.f, 0.f, 0.f, 0.f}, l[4] = {0.f, 0.f, 0.f, 0.f};
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (count >= 4 || j < count) {
      const float2 r = emit_one<kBf16, EPI>(e, at + (int64_t)j * M, v[j] + bias, h[j], l[j]);
      acc.x += r.x;
      acc.y += r.y;
    }
  float* th = e->t_hi + (int64_t)row * e->t_ld + t0;
  float* tl = e->t_lo + (int64_t)row * e->t_ld + t0;
  if (count >= 4) {
    *reinterpret_cast<float4*>(th) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(tl) = make_float4(l[0], l[1], l[2], l[3]);
  } else {
    for (int j = 0; j < count; ++j) {
      th[j] = h[j];
      tl[j] = l[j];
    }
  }
  return acc;
}

template <bool kBf16, int EPI>
__device__ __noinline__ float2 emit4(const EpilogueArgs* e, int64_t at, int64_t stride, int count, float bias,
                                     float v0, float v1, float v2, float v3) {
  return emit4_inline<kBf16, EPI>(e, at, stride, count, bias, v0, v1, v2, v3);
}

template <bool kBf16, int EPI>
__device__ __noinline__ float2 emit4t(const EpilogueArgs* e, int row, int t0, int M, int N, float bias, float v0,
                                      float v1, float v2, float v3) {
  return emit4t_inline<kBf16, EPI>(e, row, t0, M, N, bias, v0, v1, v2, v3);
}

// The emitter of an epilogue: with or without the feature-major copies, out of line or inlined by the number of
// values per epilogue thread.
template <bool kBf16, int EPI, int HALF>
__device__ __forceinline__ float2 emit4_at(const EpilogueArgs* e, int row, int t0, int M, int N, float bias, float v0,
                                           float v1, float v2, float v3) {
  constexpr bool kCopies = !kBf16 && (EPI == kUpT || EPI == kDownMse || EPI == kGradHidden);
  if constexpr (kCopies) {
    if constexpr (HALF <= 64) return emit4t_inline<kBf16, EPI>(e, row, t0, M, N, bias, v0, v1, v2, v3);
    else return emit4t<kBf16, EPI>(e, row, t0, M, N, bias, v0, v1, v2, v3);
  } else {
    const int64_t at = (int64_t)t0 * M + row;
    if constexpr (HALF <= 64) return emit4_inline<kBf16, EPI>(e, at, M, N - t0, bias, v0, v1, v2, v3);
    else return emit4<kBf16, EPI>(e, at, M, N - t0, bias, v0, v1, v2, v3);
  }
}

// fp16x3: one value of the output tile, token t: the accumulator scaled back by row_inv tok_inv[t] (powers of two: exact,
// so a fused multiply-add rounds once like the separate add), + bias; then (up) z, GELU and act 2^e_t split into fp16
// hi / lo, or (down) the y store.
template <int EPI>
__device__ __forceinline__ void emit_f16_one(const EpilogueArgs* e, int64_t at, float acc, float row_inv, float tok_inv,
                                             float act_mul, float bias) {
  const float s = acc * row_inv * tok_inv + bias;
  if constexpr (EPI == kUp) {
    if (e->z != nullptr) e->z[at] = s;
    const float h = gelu(s) * act_mul;
    const __half hi = __float2half_rn(h);
    reinterpret_cast<__half*>(e->out_hi)[at] = hi;
    reinterpret_cast<__half*>(e->out_lo)[at] = __float2half_rn(h - __half2float(hi));
  } else {
    static_assert(EPI == kDown, "fp16x3 epilogues: up and down");
    reinterpret_cast<float*>(e->out_hi)[at] = s;
  }
}

// fp16x3: the scales of token t from its packet (written by the split kernel, read-only here): up GEMMs {x_inv,
// act_mul} (one 8-byte load), down GEMMs {act_inv, unused}.
template <int EPI>
__device__ __forceinline__ float2 token_scales(const EpilogueArgs* e, int t) {
  const float* p = e->tok_tab + (int64_t)t * e->tok_stride;
  if constexpr (EPI == kUp || EPI == kUpT) return __ldg(reinterpret_cast<const float2*>(p));
  else return make_float2(__ldg(p + 2), 0.f);
}

// fp16x3 training epilogues: four values of one output row, tokens t0 .. t0 + 3 (t0 a multiple of 4; N - t0 of them
// valid when fewer than four), their token scales sa (the B operand's inverse scale) and sb (act_mul). kUpT: z, act
// 2^a_t as fp16 hi / lo token-major (the down GEMM's operand; the same values as the forward's up epilogue) and act as
// tf32 hi / lo into the feature-major copies (the weight-gradient GEMM's operand); kDownMse: y, the MSE gradient gy as
// tf32 hi / lo token-major and feature-major, and the partial sums (loss, column sum); kGradHidden: gz = acc gelu'(z)
// as tf32 hi / lo token-major and feature-major, and the column sum. Out of line: a thread holds up to 128 values.
template <int EPI>
__device__ __noinline__ float2 emit4t_f16(const EpilogueArgs* e, int row, int t0, int M, int N, float row_inv,
                                          float bias, float4 v, float4 sa, float4 sb) {
  static_assert(EPI == kUpT || EPI == kDownMse || EPI == kGradHidden, "fp16x3 training epilogues");
  const int count = N - t0;
  const float vv[4] = {v.x, v.y, v.z, v.w}, a[4] = {sa.x, sa.y, sa.z, sa.w}, b[4] = {sb.x, sb.y, sb.z, sb.w};
  float h[4] = {0.f, 0.f, 0.f, 0.f}, l[4] = {0.f, 0.f, 0.f, 0.f};
  float2 acc = make_float2(0.f, 0.f);
  int64_t at = (int64_t)t0 * M + row;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (count >= 4 || j < count) {
      const float s = vv[j] * row_inv * a[j] + bias;
      if constexpr (EPI == kUpT) {
        if (e->z != nullptr) e->z[at] = s;
        const float g = gelu(s);
        const float scaled = g * b[j];
        const __half hh = __float2half_rn(scaled);
        reinterpret_cast<__half*>(e->out_hi)[at] = hh;
        reinterpret_cast<__half*>(e->out_lo)[at] = __float2half_rn(scaled - __half2float(hh));
        h[j] = tf32_rna(g);
        l[j] = tf32_rna(g - h[j]);
      } else if constexpr (EPI == kGradHidden) {
        const float g = s * gelu_grad(e->z_in[at]);
        h[j] = tf32_rna(g);
        l[j] = tf32_rna(g - h[j]);
        reinterpret_cast<float*>(e->out_hi)[at] = h[j];
        reinterpret_cast<float*>(e->out_lo)[at] = l[j];
        acc.y += g;
      } else {
        reinterpret_cast<float*>(e->out_hi)[at] = s;
        const float diff = s - e->target[at];
        const float g = e->scale * diff;
        h[j] = tf32_rna(g);
        l[j] = tf32_rna(g - h[j]);
        e->gy_hi[at] = h[j];
        e->gy_lo[at] = l[j];
        acc.x += diff * diff;
        acc.y += g;
      }
    }
    at += M;
  }
  float* th = e->t_hi + (int64_t)row * e->t_ld + t0;
  float* tl = e->t_lo + (int64_t)row * e->t_ld + t0;
  if (count >= 4) {
    *reinterpret_cast<float4*>(th) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(tl) = make_float4(l[0], l[1], l[2], l[3]);
  } else {
    for (int j = 0; j < count; ++j) {
      th[j] = h[j];
      tl[j] = l[j];
    }
  }
  return acc;
}

// fp16x3: the values of one output row over the thread's HALF token columns n0 .. n0 + HALF - 1 (sum: the chunk sums),
// in groups of four tokens, the token scales read as float4 from the warp's shared-memory table (tab: the first scale
// of the warp's columns; the second HALF floats further).
template <int EPI, int HALF>
__device__ __forceinline__ void emit_row_f16(const EpilogueArgs* e, const float* tab, int row, int n0, int M, int N,
                                             float row_inv, float bias, const float (&sum)[HALF]) {
  const int count = N - n0 < HALF ? N - n0 : HALF;
  int64_t at = (int64_t)n0 * M + row;
#pragma unroll
  for (int g = 0; g < HALF / 4; ++g) {
    const float4 a = *reinterpret_cast<const float4*>(tab + 4 * g);
    const float4 b = EPI == kUp ? *reinterpret_cast<const float4*>(tab + HALF + 4 * g) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float sa[4] = {a.x, a.y, a.z, a.w}, sb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (4 * g + j < count) emit_f16_one<EPI>(e, at + j * (int64_t)M, sum[4 * g + j], row_inv, sa[j], sb[j], bias);
    at += 4 * (int64_t)M;
  }
}

// The support entries of one row among four consecutive columns (nib: which are on the support; q: the compact index of
// the first of them; g0 .. g3: the gradients of the four columns): each gradient stored and / or applied by AdamW
// (PyTorch's fused order) and, with dense_hi != NULL, the dense operand's entry refreshed with the new value as tf32
// hi / lo. The loads of all four are issued before their arithmetic: a thread walks its own row, so its loads do not
// coalesce with its warp's, and four independent ones in flight hide more of their latency than one (measured).
__device__ __noinline__ void sampled_entries4(const EpilogueArgs* e, int q, uint32_t nib, int64_t dense_at, float g0,
                                              float g1, float g2, float g3) {
  const float g[4] = {g0, g1, g2, g3};
  int qs[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) qs[j] = q + __popc(nib & ((1u << j) - 1u));
  if (e->grad)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if ((nib >> j) & 1u) e->grad[qs[j]] = g[j];
  if (!e->adam) return;
  const hffn_adamw_step& st = e->step;
  float p[4] = {0.f, 0.f, 0.f, 0.f}, m[4] = {0.f, 0.f, 0.f, 0.f}, v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if ((nib >> j) & 1u) {
      p[j] = e->value[qs[j]];
      m[j] = e->m[qs[j]];
      v[j] = e->v[qs[j]];
    }
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if ((nib >> j) & 1u) {
      float pj = p[j];
      pj -= st.lr_decay * pj;
      const float mi = st.beta1 * m[j] + st.one_minus_beta1 * g[j];
      const float vi = st.beta2 * v[j] + st.one_minus_beta2 * g[j] * g[j];
      e->m[qs[j]] = mi;
      e->v[qs[j]] = vi;
      pj -= st.step_size * mi / (sqrtf(vi) / st.bias2_sqrt + st.eps);
      e->value[qs[j]] = pj;
      if (e->dense_hi != nullptr) {
        const float hi = tf32_rna(pj);
        e->dense_hi[dense_at + j] = hi;
        e->dense_lo[dense_at + j] = tf32_rna(pj - hi);
      }
    }
}

// Shared memory: [stages][A parts][128 rows x RB bytes] then [stages][B parts][BN rows x RB bytes], 1024-aligned, the
// barriers, then (fp16x3) each epilogue warp's table of token scales for its columns, [2][HALF] floats per warp (8 BN
// floats in all).
template <bool kBf16, int BN, int STAGES, int RB, bool kF16 = false>
struct Layout {
  static constexpr int kParts = kBf16 ? 1 : 2;
  static constexpr int kA = BM * RB;
  static constexpr int kB = BN * RB;
  static constexpr int kStageBytes = kParts * (kA + kB);
  static constexpr int kOperandBytes = STAGES * kStageBytes;
  static constexpr int kBarrierBytes = 8 * (2 * STAGES + 5) + 16;
  static constexpr int kTokOffset = kOperandBytes + (kBarrierBytes + 15) / 16 * 16;
  static constexpr int kTokBytes = kF16 ? 8 * BN * 4 : 0;
  static constexpr int kTotal = 1024 + kTokOffset + kTokBytes;
  static constexpr int kTmemCols = 2 * BN;
};

template <bool kBf16, int BN, int STAGES, int EPI, int KCHUNK, int RB, int EW, bool A_MN, bool B_MN, bool kF16>
__global__ void __launch_bounds__(threads_for(EW), 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a_hi, const __grid_constant__ CUtensorMap map_a_lo,
               const __grid_constant__ CUtensorMap map_b_hi, const __grid_constant__ CUtensorMap map_b_lo, int M,
               int N, int K, const __grid_constant__ EpilogueArgs epi, int* err) {
  using L = Layout<kBf16, BN, STAGES, RB, kF16>;
  constexpr int kRowBytes = RB;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_base = smem;
  uint8_t* b_base = smem + STAGES * L::kParts * L::kA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOperandBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN, num_tiles = num_m * num_n;
  static_assert(!(kBf16 && kF16), "fp16x3 operands are a float32 format");
  static_assert(!kF16 || KCHUNK > 0, "fp16x3 accumulates in chunks");
  constexpr int kElem = kBf16 || kF16 ? 2 : 4;
  const int num_kb = (K * kElem + kRowBytes - 1) / kRowBytes;
  const int k_elems = kRowBytes / kElem;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * EW);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    prefetch_map(&map_a_hi);
    prefetch_map(&map_b_hi);
    if (!kBf16) {
      prefetch_map(&map_a_lo);
      prefetch_map(&map_b_lo);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(L::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch (no-ops in a plain launch): the next kernel of the stream may be scheduled onto SMs
  // this grid leaves (its prologue overlaps this grid's last tiles); this grid reads its predecessor's outputs only
  // after the predecessor has completed.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // Lane 0 waits for a free stage and arms its barrier; then the stage's boxes are issued one per lane (an MN-major
    // operand takes one box per 32-element MN block: up to 24 boxes a stage, which one thread issues too slowly to
    // keep the MMAs fed).
    constexpr int kBoxA = A_MN ? BM / 32 : 1, kBoxB = B_MN ? BN / 32 : 1;
    constexpr int kBoxes = (kBoxA + kBoxB) * (kBf16 ? 1 : 2);
    static_assert(kBoxes <= 32, "one box per lane");
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed = 0;   // bit s: stage s has been armed at least once
    uint32_t armed_parity = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int m0 = (tile % num_m) * BM, n0 = (tile / num_m) * BN;
      for (int kb = 0; kb < num_kb; ++kb) {
        int got = 1;
        if (lane == 0) {
          got = mbar_wait(&empty[stage], phase ^ 1, abort_flag, kWaitNs) ? 1 : 0;
          if (got) {
            mbar_expect_tx(&full[stage], L::kStageBytes);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
        }
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        __syncwarp();
        if (lane < kBoxes) {
          const int kc = kb * k_elems;
          int box = lane;
          const bool lo = !kBf16 && box >= kBoxA + kBoxB;
          if (lo) box -= kBoxA + kBoxB;
          const bool is_a = box < kBoxA;
          const int blk = is_a ? box : box - kBoxA;
          const bool mn = is_a ? A_MN : B_MN;
          const CUtensorMap* map = is_a ? (lo ? &map_a_lo : &map_a_hi) : (lo ? &map_b_lo : &map_b_hi);
          uint8_t* dst = is_a ? a_base + stage * L::kParts * L::kA + (lo ? L::kA : 0)
                              : b_base + stage * L::kParts * L::kB + (lo ? L::kB : 0);
          // K-major: one box (K extent x rows); MN-major: one box (32 MN x K extent) per 32-element MN block
          if (!mn) tma_load_2d(dst, map, &full[stage], kc, is_a ? m0 : n0);
          else tma_load_2d(dst + blk * (k_elems * 128), map, &full[stage], (is_a ? m0 : n0) + 32 * blk, kc);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (lane == 0) {
      if (!ok) {
        atomicCAS(err, 0, kErrTimeoutProducer);
        *abort_flag = 1;
      }
      // wait (bounded) until every armed stage's last load has landed, so no copy is in flight at exit
      for (int s = 0; s < STAGES; ++s)
        if (armed & (1u << s)) {
          const uint64_t start = global_ns();
          while (!mbar_try_wait(&full[s], (armed_parity >> s) & 1u) && global_ns() - start < kWaitNs) {
          }
        }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The K loop of a tile runs in chunks of chunk_kb k-blocks, each into a fresh accumulator buffer that the
    // epilogue drains (float32: the chunk sums are added in registers with round-to-nearest; see the epilogue).
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(kBf16 ? 1 : (kF16 ? 0 : 2), BN, A_MN, B_MN);
      const uint32_t mn_lbo = (uint32_t)(k_elems * 128);    // bytes between 32-element MN blocks of a stage
      const int chunk_kb = KCHUNK > 0 ? KCHUNK : num_kb;
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kc = 0; kc < num_kb && ok; kc += chunk_kb) {
          const int kend = kc + chunk_kb < num_kb ? kc + chunk_kb : num_kb;
          if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, kWaitNs)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t d_tmem = tmem_base + acc * BN;
          for (int kb = kc; kb < kend; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag, kWaitNs)) {
              ok = false;
              break;
            }
            fence_after();
            const uint32_t a = smem_u32(a_base + stage * L::kParts * L::kA);
            const uint32_t b = smem_u32(b_base + stage * L::kParts * L::kB);
#pragma unroll
            for (int k = 0; k < kRowBytes / 32; ++k) {
              const uint32_t acc_in = (kb != kc || k != 0) ? 1u : 0u;
              const uint64_t ah = A_MN ? smem_desc_mn(a + 1024 * k, mn_lbo) : smem_desc<RB>(a + 32 * k);
              const uint64_t bh = B_MN ? smem_desc_mn(b + 1024 * k, mn_lbo) : smem_desc<RB>(b + 32 * k);
              mma<kBf16 || kF16>(d_tmem, ah, bh, idesc, acc_in);
              if (!kBf16) {
                const uint64_t al = A_MN ? smem_desc_mn(a + L::kA + 1024 * k, mn_lbo) : smem_desc<RB>(a + L::kA + 32 * k);
                const uint64_t bl = B_MN ? smem_desc_mn(b + L::kB + 1024 * k, mn_lbo) : smem_desc<RB>(b + L::kB + 32 * k);
                mma<kBf16 || kF16>(d_tmem, ah, bl, idesc, 1);
                mma<kBf16 || kF16>(d_tmem, al, bh, idesc, 1);
              }
            }
            mma_commit(&empty[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          mma_commit(&tfull[acc]);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
      if (!ok) {
        atomicCAS(err, 0, kErrTimeoutMma);
        *abort_flag = 1;
      }
      // every MMA issued by this thread has completed before the TMEM is freed (bounded wait)
      mma_commit(done);
      const uint64_t start = global_ns();
      while (!mbar_try_wait(done, 0) && global_ns() - start < kWaitNs) {
      }
    }
  } else {
    // ---------------- epilogue: warps 2 .. EW + 1; TMEM lane quarter = warp % 4, column part = (warp - 2) / 4 ----------
    constexpr int PARTS = EW / 4;
    constexpr int HALF = BN / PARTS;
    static_assert(HALF % 32 == 0, "column part of an epilogue warp");
    const EpilogueArgs* e = &epi;
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16) + half * HALF;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int m0 = (tile % num_m) * BM, n_blk = tile / num_m, n0 = n_blk * BN + half * HALF;
      const int row = m0 + quarter * 32 + lane;
      // fp16x3: the token scales of this warp's columns, read once per tile from the packets (one token per lane)
      // into the warp's own shared-memory table ([first scale][HALF], [second scale][HALF]) and read back as float4 by
      // the emit; the warp alone writes and reads it, so it needs no barrier beyond the warp's own
      float* tok_tab = nullptr;
      if constexpr (kF16) {
        tok_tab = reinterpret_cast<float*>(smem + L::kTokOffset) + (warp - 2) * 2 * HALF;
        __syncwarp();
#pragma unroll
        for (int c = 0; c < HALF / 32; ++c) {
          const int t = n0 + c * 32 + lane;
          const float2 v = t < N ? token_scales<EPI>(e, t) : make_float2(0.f, 0.f);
          tok_tab[c * 32 + lane] = v.x;
          tok_tab[HALF + c * 32 + lane] = v.y;
        }
        __syncwarp();
      }
      float bias = 0.f;
      if (row < M && e->bias != nullptr) {
        if constexpr (kBf16) bias = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(e->bias)[row]);
        else bias = reinterpret_cast<const float*>(e->bias)[row];
      }
      float row_inv = 1.f;
      if constexpr (kF16)
        if (row < M) row_inv = e->row_inv[row];
      float2 partial = make_float2(0.f, 0.f);
      if constexpr (KCHUNK > 0) {
        // chunk partials summed in registers, chunk after chunk, round-to-nearest
        float sum[HALF];
#pragma unroll
        for (int i = 0; i < HALF; ++i) sum[i] = 0.f;
        for (int kc = 0; kc < num_kb; kc += KCHUNK) {
          if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, kWaitNs)) {
            ok = false;
            break;
          }
          fence_after();
#pragma unroll
          for (int c = 0; c < HALF / 32; ++c) {
            float v[32];
            tmem_ld32(lane_base + acc * BN + c * 32, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) sum[c * 32 + j] += v[j];
          }
          fence_before();
          mbar_arrive(&tempty[acc]);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (EPI == kSampled) {
          // the support entries of this row within columns [n0, n0 + HALF): the row's bitmask words for these
          // columns and the compact index of the first of them (independent loads, no search)
          if (row < M) {
            static_assert(HALF % 32 == 0, "whole mask words");
            const int64_t word0 = (int64_t)row * e->mask_ld + (n0 >> 5);
            uint32_t bits[HALF / 32];
#pragma unroll
            for (int c = 0; c < HALF / 32; ++c) bits[c] = e->mask[word0 + c];
            int q = e->first[word0];
            const int64_t dense_row = (int64_t)row * N;
#pragma unroll
            for (int g4 = 0; g4 < HALF / 4; ++g4) {
              const uint32_t nib = (bits[g4 >> 3] >> ((g4 & 7) * 4)) & 0xFu;
              if (nib) {
                sampled_entries4(e, q, nib, dense_row + n0 + 4 * g4, sum[4 * g4], sum[4 * g4 + 1], sum[4 * g4 + 2],
                                 sum[4 * g4 + 3]);
                q += __popc(nib);
              }
            }
          }
        } else if (row < M) {
          if constexpr (kF16 && (EPI == kUpT || EPI == kDownMse || EPI == kGradHidden)) {
#pragma unroll
            for (int g = 0; g < HALF / 4; ++g)
              if (n0 + 4 * g < N) {
                const float4 sa = *reinterpret_cast<const float4*>(tok_tab + 4 * g);
                const float4 sb = *reinterpret_cast<const float4*>(tok_tab + HALF + 4 * g);
                const float2 r = emit4t_f16<EPI>(e, row, n0 + 4 * g, M, N, row_inv, bias,
                                                 make_float4(sum[4 * g], sum[4 * g + 1], sum[4 * g + 2], sum[4 * g + 3]),
                                                 sa, sb);
                partial.x += r.x;
                partial.y += r.y;
              }
          } else if constexpr (kF16) {
            emit_row_f16<EPI, HALF>(e, tok_tab, row, n0, M, N, row_inv, bias, sum);
          } else {
#pragma unroll
            for (int i = 0; i < HALF; i += 4)
              if (n0 + i < N) {
                const float2 r = emit4_at<kBf16, EPI, HALF>(e, row, n0 + i, M, N, bias, sum[i], sum[i + 1],
                                                            sum[i + 2], sum[i + 3]);
                partial.x += r.x;
                partial.y += r.y;
              }
          }
        }
      } else {
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, kWaitNs)) {
          ok = false;
          break;
        }
        fence_after();
        for (int c = 0; c < HALF / 32; ++c) {
          float v[32];
          tmem_ld32(lane_base + acc * BN + c * 32, v);
          if (row < M) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const int t = n0 + c * 32 + j;
              if (t < N) {
                const float2 r = emit4_at<kBf16, EPI, HALF>(e, row, t, M, N, bias, v[j], v[j + 1], v[j + 2],
                                                            v[j + 3]);
                partial.x += r.x;
                partial.y += r.y;
              }
            }
          }
        }
        fence_before();
        mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if constexpr (EPI == kDownMse || EPI == kGradHidden) {
        // one partial per (token block, column part, row): summed in a fixed order by the reduction kernel
        if (row < M) {
          const int64_t at = (int64_t)(n_blk * PARTS + half) * M + row;
          e->col_partial[at] = partial.y;
          if constexpr (EPI == kDownMse) e->loss_partial[at] = partial.x;
        }
      }
    }
    if (!ok) {
      atomicCAS(err, 0, kErrTimeoutEpilogue);
      *abort_flag = 1;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(L::kTmemCols));
  }
}

// ---------------------------------------------------------------------------------------------------------------
// operand preparation: densify a compact CSR-by-row layout, split float32 into tf32 hi/lo

__global__ void densify_kernel(const int32_t* __restrict__ off, const int16_t* __restrict__ idx,
                               const void* __restrict__ val, int rows, int cols, int bf16, void* hi, void* lo) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int64_t base = (int64_t)warp * cols;
  for (int e = off[warp] + lane; e < off[warp + 1]; e += 32) {
    const int c = idx[e];
    if (bf16) {
      reinterpret_cast<__nv_bfloat16*>(hi)[base + c] = reinterpret_cast<const __nv_bfloat16*>(val)[e];
    } else {
      const float v = reinterpret_cast<const float*>(val)[e];
      const float h = tf32_rna(v);
      reinterpret_cast<float*>(hi)[base + c] = h;
      reinterpret_cast<float*>(lo)[base + c] = tf32_rna(v - h);
    }
  }
}

__global__ void split_kernel(const float4* __restrict__ x, float4* __restrict__ hi, float4* __restrict__ lo,
                             int64_t count4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = x[i];
    float4 h, l;
    h.x = tf32_rna(v.x); l.x = tf32_rna(v.x - h.x);
    h.y = tf32_rna(v.y); l.y = tf32_rna(v.y - h.y);
    h.z = tf32_rna(v.z); l.z = tf32_rna(v.z - h.z);
    h.w = tf32_rna(v.w); l.w = tf32_rna(v.w - h.w);
    hi[i] = h;
    lo[i] = l;
  }
}

// x [n, d] -> feature-major tf32 parts x_hi^T, x_lo^T [d, ld] (ld >= n): 32 x 32 tiles through shared memory, reads
// and writes coalesced.
__global__ void split_transpose_kernel(const float* __restrict__ x, int64_t n, int d, float* __restrict__ hi,
                                       float* __restrict__ lo, int64_t ld) {
  __shared__ float tile[32][33];
  const int64_t t0 = (int64_t)blockIdx.x * 32;
  const int f0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t t = t0 + r;
    const int f = f0 + threadIdx.x;
    tile[r][threadIdx.x] = t < n && f < d ? x[t * d + f] : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int f = f0 + r;
    const int64_t t = t0 + threadIdx.x;
    if (f < d && t < n) {
      const float v = tile[threadIdx.x][r];
      const float h = tf32_rna(v);
      hi[(int64_t)f * ld + t] = h;
      lo[(int64_t)f * ld + t] = tf32_rna(v - h);
    }
  }
}

// fp16x3 scales. 2^e as a float (e in [-126, 127]).
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

// The exponent e that maps the largest magnitude m of a row into [2^14, 2^15) (m = f 2^k, f in [0.5, 1): e = 15 - k),
// clamped to [-63, 63] so that the product of two scales stays a normal float; 0 for an all-zero row.
__device__ __forceinline__ int row_exponent(float m) {
  if (!(m > 0.f)) return 0;
  const int k = (int)((__float_as_uint(m) >> 23) & 0xFF) - 126;
  const int e = 15 - k;
  return e < -63 ? -63 : (e > 63 ? 63 : e);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_add(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// fp16x3 operands of a CSR-by-row support [rows, cols] (zeroed beforehand): one warp per row; the row's values scaled by
// 2^e (row_exponent of its largest |value|) and split into fp16 hi / lo at their dense positions, inv[row] = 2^-e; with
// `bound`, bound[0] = the largest row L1 norm and bound[1] = the largest |bias| (atomicMax on the bits of non-negative
// floats, which order as integers).
__global__ void densify_f16_kernel(const int32_t* __restrict__ off, const int16_t* __restrict__ idx,
                                   const float* __restrict__ val, const float* __restrict__ bias, int rows, int cols,
                                   __half* __restrict__ hi, __half* __restrict__ lo, float* __restrict__ inv,
                                   float* bound) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int begin = off[row], end = off[row + 1];
  float m = 0.f, l1 = 0.f;
  for (int q = begin + lane; q < end; q += 32) {
    const float a = fabsf(val[q]);
    m = fmaxf(m, a);
    l1 += a;
  }
  m = warp_max(m);
  l1 = warp_add(l1);
  const int e = row_exponent(m);
  if (lane == 0) {
    inv[row] = exp2i(-e);
    if (bound != nullptr) {
      atomicMax(reinterpret_cast<int*>(bound), __float_as_int(l1));
      if (bias != nullptr) atomicMax(reinterpret_cast<int*>(bound) + 1, __float_as_int(fabsf(bias[row])));
    }
  }
  const float scale = exp2i(e);
  const int64_t base = (int64_t)row * cols;
  for (int q = begin + lane; q < end; q += 32) {
    const float v = val[q] * scale;
    const __half h = __float2half_rn(v);
    hi[base + idx[q]] = h;
    lo[base + idx[q]] = __float2half_rn(v - __half2float(h));
  }
}

// fp16x3 token packets: token t's row of x as fp16 parts and its scales, one row of packet_halves(d) halves: the hi
// part at 0, the lo part at part_halves(d), then float32 {x_inv = 2^-e_t, act_mul = 2^a_t, act_inv = 2^-a_t, 0} at
// 2 part_halves(d); each piece starts on a 64-byte boundary (a part holds d halves rounded up to 32: the TMA rows of
// the GEMMs then cover whole 32-byte sectors; with 16-byte offsets a 64-byte row read touched three sectors and the up
// GEMM ran 15 % slower, measured). Packets of several ranks' tokens concatenate into one batch (the neuron-sharded
// forward gathers them as they are); the GEMMs read the parts through tensor maps with the packet stride.
__host__ __device__ constexpr int64_t part_halves(int64_t d) { return (d + 31) / 32 * 32; }
__host__ __device__ constexpr int64_t packet_halves(int64_t d) { return 2 * part_halves(d) + 32; }

// The split: one warp per token row t of x [n, d] (d a multiple of 8, x 16-byte aligned). e_t = row_exponent of
// max |x_t|; a_t = row_exponent of the bound max(bound[0] max|x_t| + bound[1], 0.17) of |act_t| (|z| <=
// ||W_up[r]||_1 max|x_t| + |b_up[r]|, and |gelu(z)| <= max(|z|, 0.17)): act 2^a_t stays below 2^15, half of fp16's
// largest finite value, which leaves room for the rounding of the bound and of z.
__global__ void split_f16_kernel(const float* __restrict__ x, int64_t n, int d, const float* __restrict__ bound,
                                 __half* __restrict__ packets) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // the up GEMM's prologue may overlap this kernel
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  const float4* row = reinterpret_cast<const float4*>(x + t * d);
  const int d4 = d >> 2;
  float m = 0.f;
  for (int i = lane; i < d4; i += 32) {
    const float4 v = row[i];
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  m = warp_max(m);
  const int e = row_exponent(m);
  const float scale = exp2i(e);
  __half* packet = packets + t * packet_halves(d);
  uint2* h_row = reinterpret_cast<uint2*>(packet);
  uint2* l_row = reinterpret_cast<uint2*>(packet + part_halves(d));
  for (int i = lane; i < d4; i += 32) {
    const float4 v = row[i];
    const float s[4] = {v.x * scale, v.y * scale, v.z * scale, v.w * scale};
    __half h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = __float2half_rn(s[j]);
      l[j] = __float2half_rn(s[j] - __half2float(h[j]));
    }
    uint2 ph, pl;
    ph.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
    ph.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
    pl.x = (uint32_t)__half_as_ushort(l[0]) | ((uint32_t)__half_as_ushort(l[1]) << 16);
    pl.y = (uint32_t)__half_as_ushort(l[2]) | ((uint32_t)__half_as_ushort(l[3]) << 16);
    h_row[i] = ph;
    l_row[i] = pl;
  }
  if (lane == 0) {
    const int a = row_exponent(fmaxf(bound[0] * m + bound[1], 0.17f));
    *reinterpret_cast<float4*>(packet + 2 * part_halves(d)) = make_float4(exp2i(-e), exp2i(a), exp2i(-a), 0.f);
  }
}

// fp16x3 packets of a float32 operand held as tf32 hi / lo pairs [n, K] (the training step's gy and gz, the B operands of
// its backward GEMMs): one warp per token row, v = hi + lo scaled by 2^e_t (row_exponent of its largest |v|) and split
// into fp16 hi / lo, the table {0, 0, 2^-e_t, 0} (the down-type epilogues read the third entry).
__global__ void split_pair_f16_kernel(const float* __restrict__ hi, const float* __restrict__ lo, int64_t n, int K,
                                      __half* __restrict__ packets) {
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  const float4* rh = reinterpret_cast<const float4*>(hi + t * K);
  const float4* rl = reinterpret_cast<const float4*>(lo + t * K);
  const int k4 = K >> 2;
  float m = 0.f;
  for (int i = lane; i < k4; i += 32) {
    const float4 a = rh[i], b = rl[i];
    m = fmaxf(m, fmaxf(fmaxf(fabsf(a.x + b.x), fabsf(a.y + b.y)), fmaxf(fabsf(a.z + b.z), fabsf(a.w + b.w))));
  }
  m = warp_max(m);
  const int e = row_exponent(m);
  const float scale = exp2i(e);
  __half* packet = packets + t * packet_halves(K);
  uint2* h_row = reinterpret_cast<uint2*>(packet);
  uint2* l_row = reinterpret_cast<uint2*>(packet + part_halves(K));
  for (int i = lane; i < k4; i += 32) {
    const float4 a = rh[i], b = rl[i];
    const float sv[4] = {(a.x + b.x) * scale, (a.y + b.y) * scale, (a.z + b.z) * scale, (a.w + b.w) * scale};
    __half h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = __float2half_rn(sv[j]);
      l[j] = __float2half_rn(sv[j] - __half2float(h[j]));
    }
    uint2 ph, pl;
    ph.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
    ph.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
    pl.x = (uint32_t)__half_as_ushort(l[0]) | ((uint32_t)__half_as_ushort(l[1]) << 16);
    pl.y = (uint32_t)__half_as_ushort(l[2]) | ((uint32_t)__half_as_ushort(l[3]) << 16);
    h_row[i] = ph;
    l_row[i] = pl;
  }
  if (lane == 0) *reinterpret_cast<float4*>(packet + 2 * part_halves(K)) = make_float4(0.f, 0.f, exp2i(-e), 0.f);
}

// The transposed fp16x3 operand of a dense fp16x3 matrix [R, C] (hi, lo, per-row inverse scales; R and C multiples of
// 32), in two passes. colmax: the largest |w| of each column (atomicMax on the bits of non-negative floats; zeroed
// before). transpose: 32 x 32 tiles through shared memory, w = (hi + lo) row_inv of the source written as the row
// c of the result, scaled by 2^e_c (row_exponent of the column's largest) and split into fp16 hi / lo, inv[c] = 2^-e_c.
__global__ void colmax_f16_kernel(const __half* __restrict__ hi, const __half* __restrict__ lo,
                                  const float* __restrict__ row_inv, int R, int C, int rows_per_block,
                                  unsigned* __restrict__ colmax) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(R, r0 + rows_per_block);
  float m = 0.f;
  for (int r = r0; r < r1; ++r) {
    const int64_t at = (int64_t)r * C + c;
    m = fmaxf(m, fabsf((__half2float(hi[at]) + __half2float(lo[at])) * row_inv[r]));
  }
  atomicMax(colmax + c, __float_as_uint(m));
}

__global__ void transpose_f16_kernel(const __half* __restrict__ hi, const __half* __restrict__ lo,
                                     const float* __restrict__ row_inv, int R, int C,
                                     const unsigned* __restrict__ colmax, __half* __restrict__ out_hi,
                                     __half* __restrict__ out_lo, float* __restrict__ out_inv) {
  __shared__ float tile[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t at = (int64_t)(r0 + i) * C + c0 + threadIdx.x;
    tile[i][threadIdx.x] = (__half2float(hi[at]) + __half2float(lo[at])) * row_inv[r0 + i];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i;
    const int e = row_exponent(__uint_as_float(colmax[c]));
    const float v = tile[threadIdx.x][i] * exp2i(e);
    const __half h = __float2half_rn(v);
    const int64_t at = (int64_t)c * R + r0 + threadIdx.x;
    out_hi[at] = h;
    out_lo[at] = __float2half_rn(v - __half2float(h));
    if (blockIdx.y == 0 && threadIdx.x == 0) out_inv[c] = exp2i(-e);
  }
}

// The support of each row (CSR: offsets [rows + 1], columns) as a bitmask over 32-column words (ld words per row,
// zero past the last column) and, per word, the compact index of the row's first entry at or after the word's first
// column. One warp per row, the row's mask assembled in shared memory (ld <= kMaxMaskWords).
constexpr int kMaskWarps = 4, kMaxMaskWords = 1024;
__global__ void support_tables_kernel(const int32_t* __restrict__ off, const int16_t* __restrict__ cols, int rows,
                                      int ld, uint32_t* __restrict__ mask, int32_t* __restrict__ first) {
  extern __shared__ uint32_t words[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kMaskWarps + warp;
  if (row >= rows) return;
  uint32_t* w = words + warp * ld;
  for (int k = lane; k < ld; k += 32) w[k] = 0u;
  __syncwarp();
  const int begin = off[row], end = off[row + 1];
  for (int q = begin + lane; q < end; q += 32) {
    const int c = cols[q];
    atomicOr(&w[c >> 5], 1u << (c & 31));
  }
  __syncwarp();
  int base = begin;
  for (int k0 = 0; k0 < ld; k0 += 32) {
    const int k = k0 + lane;
    const uint32_t word = k < ld ? w[k] : 0u;
    const int count = __popc(word);
    int inclusive = count;
#pragma unroll
    for (int step = 1; step < 32; step <<= 1) {
      const int other = __shfl_up_sync(0xffffffffu, inclusive, step);
      if (lane >= step) inclusive += other;
    }
    if (k < ld) {
      mask[(int64_t)row * ld + k] = word;
      first[(int64_t)row * ld + k] = base + inclusive - count;
    }
    base += __shfl_sync(0xffffffffu, inclusive, 31);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Element types of the operands: float32 (tf32 parts), bfloat16, fp16 (fp16x3 parts).
enum Elem { kElemF32 = 0, kElemBf16 = 1, kElemF16 = 2 };

// [rows, k] K-major operand, box = (row_bytes bytes of K) x box_rows, 128- or 64-byte swizzle, zero fill outside.
static int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int elem_type, int box_rows,
                    int row_bytes, int64_t ld = 0) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled unavailable");
    return HFFN_ERR_CUDA;
  }
  const int elem = elem_type == kElemF32 ? 4 : 2;
  const CUtensorMapDataType type = elem_type == kElemF32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : elem_type == kElemBf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)((ld > 0 ? ld : k) * elem)};
  cuuint32_t box[2] = {(cuuint32_t)(row_bytes / elem), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for a [%lld, %lld] operand", (int)r, (long long)rows, (long long)k);
    return HFFN_ERR_CUDA;
  }
  return HFFN_OK;
}

// CTA cap of the persistent GEMMs (0: one CTA per SM). Leaving SMs free lets collectives (NCCL kernels) run
// alongside a GEMM instead of after it.
static std::atomic<int> g_max_ctas{0};

static int sm_count() {
  static int count = 0;
  if (count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
    if (count <= 0) count = 148;
  }
  const int cap = g_max_ctas.load();
  return cap > 0 && cap < count ? cap : count;
}

// An MN-major float32 operand whose element (mn, k) sits at base + k * ld + mn: boxes of 32 MN elements x k_box K rows,
// 128-byte swizzle with 32-byte atomicity (the layout the MMA reads for MN-major tf32). Zero fill outside.
static int make_map_mn(CUtensorMap* map, const void* base, int64_t mn, int64_t k, int64_t ld, int k_box) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled unavailable");
    return HFFN_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)mn, (cuuint64_t)k};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {32, (cuuint32_t)k_box};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for an MN-major [%lld, %lld] operand", (int)r, (long long)mn,
              (long long)k);
    return HFFN_ERR_CUDA;
  }
  return HFFN_OK;
}

// D[M, N] = A[M, K] B[N, K]^T. K-major operands are [rows, K] with K contiguous; an MN-major operand A (B) is stored
// [K, M] ([K, N]), its leading dimension lda (ldb) elements.
// pdl: launched with programmatic stream serialization, so that its CTAs may start (and run the prologue up to
// griddepcontrol.wait) while the previous kernel of the stream finishes; the previous kernel must be one whose
// outputs are all this GEMM waits for (the forward's chain: split -> up GEMM -> down GEMM).
template <bool kBf16, int BN, int STAGES, int EPI, int KCHUNK, int RB, int EW, bool A_MN = false, bool B_MN = false,
          bool kF16 = false>
static int launch_gemm(const void* a_hi, const void* a_lo, const void* b_hi, const void* b_lo, int M, int N, int K,
                       const EpilogueArgs& epi, int* err, cudaStream_t s, int64_t lda = 0, int64_t ldb = 0,
                       bool pdl = false) {
  using L = Layout<kBf16, BN, STAGES, RB, kF16>;
  static_assert(!((kBf16 || kF16) && (A_MN || B_MN)), "MN-major operands are tf32 parts only");
  constexpr int kElemType = kBf16 ? kElemBf16 : (kF16 ? kElemF16 : kElemF32);
  constexpr int k_box = RB / 4;
  CUtensorMap ma_hi, ma_lo, mb_hi, mb_lo;
  auto map = [&](CUtensorMap* m, const void* base, int rows, int box_rows, bool mn, int64_t ld) {
    return mn ? make_map_mn(m, base, rows, K, ld, k_box) : make_map(m, base, rows, K, kElemType, box_rows, RB, ld);
  };
  HFFN_TRY(map(&ma_hi, a_hi, M, BM, A_MN, lda));
  HFFN_TRY(map(&mb_hi, b_hi, N, BN, B_MN, ldb));
  if (!kBf16) {
    HFFN_TRY(map(&ma_lo, a_lo, M, BM, A_MN, lda));
    HFFN_TRY(map(&mb_lo, b_lo, N, BN, B_MN, ldb));
  } else {
    ma_lo = ma_hi;
    mb_lo = mb_hi;
  }
  auto kernel = tc_gemm_kernel<kBf16, BN, STAGES, EPI, KCHUNK, RB, EW, A_MN, B_MN, kF16>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    configured = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  if (!pdl) {
    kernel<<<grid, threads_for(EW), L::kTotal, s>>>(ma_hi, ma_lo, mb_hi, mb_lo, M, N, K, epi, err);
    return launch_status("tc_gemm");
  }
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3((unsigned)grid);
  config.blockDim = dim3((unsigned)threads_for(EW));
  config.dynamicSmemBytes = L::kTotal;
  config.stream = s;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  cudaLaunchKernelEx(&config, kernel, ma_hi, ma_lo, mb_hi, mb_lo, M, N, K, epi, err);
  return launch_status("tc_gemm");
}

// Token width of the forward GEMMs' tiles (g_tile_tokens 256, 128 or 64 forces one). Measured on B200 over the layer
// shapes of the single-GPU and neuron-sharded forwards (float32 and bfloat16, one call or token chunks), the 256-wide
// tile was fastest wherever it gives the persistent grid a tile for at least half of the SMs (C2's down GEMM: 128 tiles
// of 256 took 80 us, 256 tiles of 128 took 116 us): a narrower tile reloads the whole 128 x K weight tile per token
// block. A GEMM with fewer 256-wide tiles than that (a small batch: C1's 256 tokens make 16 up tiles and 4 down
// tiles) takes 128, or 64 if 128 still leaves more than half of the SMs idle (C1: 78 -> 46 us per forward).
static std::atomic<int> g_tile_tokens{0};

static int pick_tile_tokens(int M, int N) {
  const int forced = g_tile_tokens.load();
  if (forced == 64 || forced == 128 || forced == 256) return forced;
  const int64_t m_tiles = (M + BM - 1) / BM, sms = sm_count();
  if (2 * m_tiles * ((N + 255) / 256) >= sms) return 256;
  if (2 * m_tiles * ((N + 127) / 128) >= sms) return 128;
  return 64;
}

// float32 accumulation: the tensor cores' fp32 accumulation in TMEM is not round-to-nearest at every add (measured
// here: results biased toward zero by ~1e-5 relative over ~400 MMAs), so the K loop runs in chunks of kFp32Chunk
// k-blocks (128 K values, 48 MMAs) into fresh accumulators whose values the epilogue adds in float32 registers. 128
// values measured faster than 64 (8 % on the C2 forward, 2.5 % on the C3 training step), the error well inside the
// float32 bar.
constexpr int kFp32Chunk = 8;

// One forward GEMM at the tile width pick_tile_tokens gives (float32: 64-byte rows; bfloat16: 128-byte rows; 8
// epilogue warps at width 64, where 16 would split 64 columns too finely).
// pdl: programmatic dependent launch, for a GEMM whose predecessor in the stream is the GEMM that wrote its operand (the
// down GEMM after the up GEMM of the same forward).
template <bool kBf16, int EPI>
static int launch_forward_gemm(const void* a_hi, const void* a_lo, const void* b_hi, const void* b_lo, int M, int N,
                               int K, const EpilogueArgs& epi, int* err, cudaStream_t s, bool pdl = false) {
  constexpr int kChunk = kBf16 ? 0 : kFp32Chunk;
  constexpr int kRow = kBf16 ? 128 : 64;
  // float32 up: 16 warps (its tail epilogue, GELU and the tf32 split of 128 x 256 values, would otherwise stall the
  // MMAs; measured 0.212 ms against 0.238 ms with 8 at C2); float32 down: 8 (16 measured slower)
  constexpr int kWarps = kBf16 || EPI == kUp ? 16 : 8;
  switch (pick_tile_tokens(M, N)) {
    case 64:
      return launch_gemm<kBf16, 64, 6, EPI, kChunk, kRow, 8>(a_hi, a_lo, b_hi, b_lo, M, N, K, epi, err, s, 0, 0, pdl);
    case 128:
      return launch_gemm<kBf16, 128, 5, EPI, kChunk, kRow, kWarps>(a_hi, a_lo, b_hi, b_lo, M, N, K, epi, err, s, 0, 0,
                                                                   pdl);
    default:
      return launch_gemm<kBf16, 256, 4, EPI, kChunk, kRow, kWarps>(a_hi, a_lo, b_hi, b_lo, M, N, K, epi, err, s, 0, 0,
                                                                   pdl);
  }
}

// fp16x3 accumulation chunks: up 8 k-blocks (256 K values, 48 MMAs: the MMA count of a 3xTF32 chunk, so the same bound
// on the accumulation bias; two chunks let the MMAs run a quarter of a C2 tile ahead of the GELU epilogue), down 4
// (128 K values: its epilogue is light, and shorter chunks keep its error below the up's).
template <int EPI>
constexpr int f16_chunk() { return EPI == kUp || EPI == kUpT ? 8 : 4; }

// One fp16x3 forward GEMM (ldb: the row stride of B in elements, 0: K; pdl: launched with programmatic dependent
// launch, its predecessor in the stream being the kernel that wrote its operands): 64-byte rows of fp16 (32 K values a stage, 48 KB: A hi / lo + B hi / lo), the tile widths
// and stage counts of the 3xTF32 GEMMs, 16 epilogue warps for up (GELU and the split), 8 for down.
template <int EPI>
static int launch_forward_gemm_f16(const void* a_hi, const void* a_lo, const void* b_hi, const void* b_lo, int M, int N,
                                   int K, const EpilogueArgs& epi, int* err, cudaStream_t s, int64_t ldb, bool pdl) {
  constexpr int kWarps = EPI == kUp ? 16 : 8;
  constexpr int kChunk = f16_chunk<EPI>();
  switch (pick_tile_tokens(M, N)) {
    case 64:
      return launch_gemm<false, 64, 6, EPI, kChunk, 64, 8, false, false, true>(a_hi, a_lo, b_hi, b_lo, M, N, K, epi,
                                                                               err, s, 0, ldb, pdl);
    case 128:
      return launch_gemm<false, 128, 5, EPI, kChunk, 64, kWarps, false, false, true>(a_hi, a_lo, b_hi, b_lo, M, N, K,
                                                                                    epi, err, s, 0, ldb, pdl);
    default:
      return launch_gemm<false, 256, 4, EPI, kChunk, 64, kWarps, false, false, true>(a_hi, a_lo, b_hi, b_lo, M, N, K,
                                                                                    epi, err, s, 0, ldb, pdl);
  }
}

// The fp16x3 forward's workspace: the token packets [n, packet_halves(d)] and the act parts [n, H] (fp16 hi, lo), each
// piece 256-byte aligned.
struct F16Work {
  __half *packets, *act_hi, *act_lo;
};

static int64_t f16_work(int64_t d, int64_t H, int64_t n, F16Work* w, uint8_t* base) {
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += (bytes + 255) / 256 * 256;
    return p;
  };
  F16Work dummy;
  F16Work* t = w ? w : &dummy;
  t->packets = reinterpret_cast<__half*>(take(2 * n * packet_halves(d)));
  t->act_hi = reinterpret_cast<__half*>(take(2 * n * H));
  t->act_lo = reinterpret_cast<__half*>(take(2 * n * H));
  return off;
}

// The up GEMM from packets (pdl: its predecessor in the stream is the split kernel that wrote them).
static int up_from_packets(const __half* packets, const hffn_dense_f16x3* D, const float* b, float* z, __half* act_hi,
                           __half* act_lo, int* err, int d, int H, int64_t n, bool pdl, cudaStream_t s) {
  const int64_t stride = packet_halves(d);
  EpilogueArgs up{};
  up.bias = b;
  up.out_hi = act_hi;
  up.out_lo = act_lo;
  up.z = z;
  up.row_inv = D->up_scale;
  up.tok_tab = reinterpret_cast<const float*>(packets + 2 * part_halves(d));
  up.tok_stride = stride / 2;
  return launch_forward_gemm_f16<kUp>(D->up_hi, D->up_lo, packets, packets + part_halves(d), H, (int)n, d, up, err, s,
                                      stride, pdl);
}

static int down_from_packets(const __half* packets, const __half* act_hi, const __half* act_lo,
                             const hffn_dense_f16x3* D, const float* b, float* y, int* err, int d, int H, int64_t n,
                             cudaStream_t s) {
  EpilogueArgs dn{};
  dn.bias = b;
  dn.out_hi = y;
  dn.row_inv = D->down_scale;
  dn.tok_tab = reinterpret_cast<const float*>(packets + 2 * part_halves(d));
  dn.tok_stride = packet_halves(d) / 2;
  return launch_forward_gemm_f16<kDown>(D->down_hi, D->down_lo, act_hi, act_lo, d, (int)n, H, dn, err, s, 0, true);
}

}  // namespace tc

int64_t tc_f16_workspace(int d, int H, int64_t n) { return tc::f16_work(d, H, n, nullptr, nullptr); }

int64_t tc_f16_packet_bytes(int d) { return 2 * tc::packet_halves(d); }

// x [n, d] float32 -> token packets [n, packet_halves(d)].
int tc_split_f16(const float* x, const hffn_dense_f16x3* D, void* packets, int d, int64_t n, cudaStream_t s) {
  tc::split_f16_kernel<<<(unsigned)ceil_div(n * 32, 256), 256, 0, s>>>(x, n, d, D->up_bound,
                                                                     reinterpret_cast<__half*>(packets));
  return launch_status("tc_split_f16");
}

// fp16x3 up: x [n, d] float32 -> packets and act parts in `work` (z: float32 [n, H] token-major, or NULL).
int tc_up_f16(const float* x, const hffn_dense_f16x3* D, const float* b, float* z, void* work, int* err, int d, int H,
              int64_t n, cudaStream_t s) {
  tc::F16Work w;
  tc::f16_work(d, H, n, &w, reinterpret_cast<uint8_t*>(work));
  HFFN_TRY(tc_split_f16(x, D, w.packets, d, n, s));
  return tc::up_from_packets(w.packets, D, b, z, w.act_hi, w.act_lo, err, d, H, n, true, s);
}

// fp16x3 down: the packets and act parts of tc_up_f16 in `work` -> y [n, d] float32.
int tc_down_f16(const void* work, const hffn_dense_f16x3* D, const float* b, float* y, int* err, int d, int H,
                int64_t n, cudaStream_t s) {
  tc::F16Work w;
  tc::f16_work(d, H, n, &w, reinterpret_cast<uint8_t*>(const_cast<void*>(work)));
  return tc::down_from_packets(w.packets, w.act_hi, w.act_lo, D, b, y, err, d, H, n, s);
}

// fp16x3 forward of n tokens from packets made by tc_split_f16 (possibly on other ranks and gathered): the up GEMM
// (a plain launch: its predecessor in the stream need not be the split) and the down GEMM, act parts in `work`.
int tc_forward_f16_packets(const void* packets, const hffn_dense_f16x3* D, const float* b_up, const float* b_down,
                           float* y, float* z, void* work, int* err, int d, int H, int64_t n, cudaStream_t s) {
  tc::F16Work w;
  tc::f16_work(d, H, n, &w, reinterpret_cast<uint8_t*>(work));
  const __half* p = reinterpret_cast<const __half*>(packets);
  HFFN_TRY(tc::up_from_packets(p, D, b_up, z, w.act_hi, w.act_lo, err, d, H, n, false, s));
  return tc::down_from_packets(p, w.act_hi, w.act_lo, D, b_down, y, err, d, H, n, s);
}

int tc_densify_f16(const int32_t* off, const int16_t* idx, const float* val, const float* bias, int rows, int cols,
                   void* hi, void* lo, float* scale, float* bound, cudaStream_t s) {
  const size_t bytes = (size_t)rows * cols * 2;
  if (cudaMemsetAsync(hi, 0, bytes, s) != cudaSuccess || cudaMemsetAsync(lo, 0, bytes, s) != cudaSuccess ||
      (bound != nullptr && cudaMemsetAsync(bound, 0, 2 * sizeof(float), s) != cudaSuccess))
    return launch_status("densify memset");
  const int blocks = (int)ceil_div((int64_t)rows * 32, 256);
  tc::densify_f16_kernel<<<blocks, 256, 0, s>>>(off, idx, val, bias, rows, cols, reinterpret_cast<__half*>(hi),
                                                reinterpret_cast<__half*>(lo), scale, bound);
  return launch_status("densify f16x3");
}

// Tile shapes: float32 (3xTF32) 128 x 256 tiles, stages of 16 K values (64-byte rows, 48 KB: A hi/lo + B hi/lo), 4
// stages, 16 epilogue warps for up and 8 for down; bfloat16 128 x 256 tiles, stages of 64 K values (128-byte rows,
// 48 KB), 4 stages, 16 epilogue warps.
// up: x [n, d] -> act [n, H] token-major (fp32: the split x_hi / x_lo [n, d] go to x_split, act as hi / lo parts).
int tc_up(int dtype, const void* x, const void* w_hi, const void* w_lo, const void* b, void* act_hi, void* act_lo,
          float* z, void* x_split, int* err, int d, int H, int64_t n, cudaStream_t s) {
  const int nn = (int)n;
  if (dtype == HFFN_BF16) {
    tc::EpilogueArgs up{};
    up.bias = b;
    up.out_hi = act_hi;
    return tc::launch_forward_gemm<true, tc::kUp>(w_hi, nullptr, x, nullptr, H, nn, d, up, err, s);
  }
  float* x_hi = reinterpret_cast<float*>(x_split);
  float* x_lo = x_hi + (int64_t)n * d;
  const int64_t count4 = (int64_t)n * d / 4;
  const int blocks = (int)std::min<int64_t>(std::max<int64_t>(ceil_div(count4, 256), 1), 148 * 8);
  tc::split_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(x_hi),
                                          reinterpret_cast<float4*>(x_lo), count4);
  HFFN_TRY(launch_status("tc_split"));
  tc::EpilogueArgs up{};
  up.bias = b;
  up.out_hi = act_hi;
  up.out_lo = act_lo;
  up.z = z;
  return tc::launch_forward_gemm<false, tc::kUp>(w_hi, w_lo, x_hi, x_lo, H, nn, d, up, err, s);
}

// down: act [n, H] token-major -> y [n, d].
// pdl: the caller's previous launch on s is the up GEMM that wrote act (tc_forward).
int tc_down(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo, const void* b,
            void* y, int* err, int d, int H, int64_t n, cudaStream_t s, bool pdl) {
  const int nn = (int)n;
  tc::EpilogueArgs dn{};
  dn.bias = b;
  dn.out_hi = y;
  if (dtype == HFFN_BF16)
    return tc::launch_forward_gemm<true, tc::kDown>(w_hi, nullptr, act_hi, nullptr, d, nn, H, dn, err, s, pdl);
  return tc::launch_forward_gemm<false, tc::kDown>(w_hi, w_lo, act_hi, act_lo, d, nn, H, dn, err, s, pdl);
}

// Workspace of the whole forward: fp32 [x_hi, x_lo (n d each), act_hi, act_lo (n H each)] floats; bf16 act [n, H].
int tc_forward(int dtype, const hffn_layer* L, const void* up_hi, const void* up_lo, const void* down_hi,
               const void* down_lo, const void* x, void* y, float* z, void* work, int* err, int64_t n,
               cudaStream_t s) {
  const int d = L->d_model, H = L->d_ff;
  if (dtype == HFFN_BF16) {
    HFFN_TRY(tc_up(dtype, x, up_hi, nullptr, L->b_up, work, nullptr, nullptr, nullptr, err, d, H, n, s));
    return tc_down(dtype, work, nullptr, down_hi, nullptr, L->b_down, y, err, d, H, n, s, true);
  }
  float* x_split = reinterpret_cast<float*>(work);
  float* act_hi = x_split + 2 * n * d;
  float* act_lo = act_hi + n * H;
  HFFN_TRY(tc_up(dtype, x, up_hi, up_lo, L->b_up, act_hi, act_lo, z, x_split, err, d, H, n, s));
  return tc_down(dtype, act_hi, act_lo, down_hi, down_lo, L->b_down, y, err, d, H, n, s, true);
}

// ---------------------------------------------------------------------------------------------------------------
// training step on the tensor cores (float32, 3xTF32, chunked accumulation)

namespace tc {

// Fixed-order sums of the per-(token block, column part) partials: the bias gradients (then stored and / or applied
// by AdamW) and, in block 0 of the loss launch, the loss.
__global__ void bias_reduce_kernel(const float* __restrict__ partial, int rows, int count, hffn_param p, int adam,
                                   hffn_adamw_step st) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  float g = 0.f;
  for (int j = 0; j < rows; ++j) g += partial[(int64_t)j * count + i];
  if (p.grad) p.grad[i] = g;
  if (!adam) return;
  float v = p.value[i];
  v -= st.lr_decay * v;
  const float mi = st.beta1 * p.m[i] + st.one_minus_beta1 * g;
  const float vi = st.beta2 * p.v[i] + st.one_minus_beta2 * g * g;
  p.m[i] = mi;
  p.v[i] = vi;
  p.value[i] = v - st.step_size * mi / (sqrtf(vi) / st.bias2_sqrt + st.eps);
}

// The loss in two fixed-order levels (the same bits whatever the launch timing): block b sums its contiguous chunk of
// the partials (each thread a strided share, then the threads' sums in thread order) into block_sums[b]; one block then
// sums the block sums in block order. One block over all the partials took 112 us at C3 (262 k partials).
constexpr int kLossBlocks = 148;
__global__ void loss_blocks_kernel(const float* __restrict__ partial, int64_t count, double* __restrict__ block_sums) {
  __shared__ double red[256];
  const int64_t chunk = (count + gridDim.x - 1) / gridDim.x;
  const int64_t begin = (int64_t)blockIdx.x * chunk, end = begin + chunk < count ? begin + chunk : count;
  double acc = 0.0;
  for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) acc += partial[i];
  red[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int k = 0; k < (int)blockDim.x; ++k) sum += red[k];
    block_sums[blockIdx.x] = sum;
  }
}

__global__ void loss_reduce_kernel(const double* __restrict__ block_sums, int blocks, double inv, float* loss) {
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int k = 0; k < blocks; ++k) sum += block_sums[k];
    *loss = (float)(sum * inv);
  }
}

// Training GEMMs: 256-token tiles. The per-(token block, column part) partial sums of the down + MSE GEMM (8
// epilogue warps: 2 column parts) and of the gelu' GEMM (16 warps: 4 column parts, its tail epilogue being the
// heavier) are reduced in a fixed order afterwards.
constexpr int kTrainBN = 256, kTrainPartsDown = 2, kTrainPartsUp = 4;
// fp16x3: the up and down + MSE GEMMs run 16 epilogue warps (their epilogues, with the feature-major copies, took
// longer than their MMAs at the f16 rate with 8): the down + MSE GEMM's partials come in 4 column parts
constexpr int kTrainPartsDownF16 = 4;

// The training step's workspace: token-major operands [n, features], their feature-major copies [features, t_ld]
// (the K-major operands of the two weight-gradient GEMMs), the partial sums, and the support tables of both
// supports (bitmask words and first indices, mask_ld words per row: whole 256-column tiles).
struct TrainWork {
  float *x_hi, *x_lo, *z, *act_hi, *act_lo, *gy_hi, *gy_lo, *gz_hi, *gz_lo, *loss_p, *dn_p, *up_p, *loss_blocks;
  float *xt_hi, *xt_lo, *actt_hi, *actt_lo, *gyt_hi, *gyt_lo, *gzt_hi, *gzt_lo;
  uint32_t *dn_mask, *up_mask;
  int32_t *dn_first, *up_first;
  int64_t t_ld, dn_ld, up_ld;
  // fp16x3 backward GEMMs: W_down^T [H, d] and W_up^T [d, H] as fp16 hi / lo with their rows' inverse scales, and the
  // column maxima of the transposes
  __half *dnt_hi, *dnt_lo, *upt_hi, *upt_lo;
  float *dnt_inv, *upt_inv;
  unsigned *colmax_dn, *colmax_up;
};

static int64_t mask_words(int64_t cols) { return (cols + kTrainBN - 1) / kTrainBN * (kTrainBN / 32); }

static int64_t train_floats(int64_t d, int64_t H, int64_t n, TrainWork* w, float* base) {
  const int64_t blocks = (n + kTrainBN - 1) / kTrainBN;
  int64_t off = 0;
  auto take = [&](float** slot, int64_t count) {
    if (w) *slot = base + off;
    off += (count + 63) / 64 * 64;   // 256-byte aligned pieces
  };
  TrainWork dummy;
  TrainWork* t = w ? w : &dummy;
  take(&t->x_hi, n * d);
  take(&t->x_lo, n * d);
  take(&t->z, n * H);
  take(&t->act_hi, n * H);
  take(&t->act_lo, n * H);
  take(&t->gy_hi, n * d);
  take(&t->gy_lo, n * d);
  take(&t->gz_hi, n * H);
  take(&t->gz_lo, n * H);
  take(&t->loss_p, kTrainPartsDownF16 * blocks * d);
  take(&t->dn_p, kTrainPartsDownF16 * blocks * d);
  take(&t->up_p, kTrainPartsUp * blocks * H);
  take(&t->loss_blocks, 2 * kLossBlocks);                      // doubles
  t->t_ld = (n + 3) / 4 * 4;
  take(&t->xt_hi, d * t->t_ld);
  take(&t->xt_lo, d * t->t_ld);
  take(&t->actt_hi, H * t->t_ld);
  take(&t->actt_lo, H * t->t_ld);
  take(&t->gyt_hi, d * t->t_ld);
  take(&t->gyt_lo, d * t->t_ld);
  take(&t->gzt_hi, H * t->t_ld);
  take(&t->gzt_lo, H * t->t_ld);
  // down support: rows d (outputs) over H columns; up support: rows H (neurons) over d columns
  t->dn_ld = mask_words(H);
  t->up_ld = mask_words(d);
  float* tables[4];
  take(&tables[0], d * t->dn_ld);
  take(&tables[1], d * t->dn_ld);
  take(&tables[2], H * t->up_ld);
  take(&tables[3], H * t->up_ld);
  t->dn_mask = reinterpret_cast<uint32_t*>(tables[0]);
  t->dn_first = reinterpret_cast<int32_t*>(tables[1]);
  t->up_mask = reinterpret_cast<uint32_t*>(tables[2]);
  t->up_first = reinterpret_cast<int32_t*>(tables[3]);
  float* parts[4] = {};
  for (int k = 0; k < 4; ++k) take(&parts[k], d * H / 2);     // d H halves each
  t->dnt_hi = reinterpret_cast<__half*>(parts[0]);
  t->dnt_lo = reinterpret_cast<__half*>(parts[1]);
  t->upt_hi = reinterpret_cast<__half*>(parts[2]);
  t->upt_lo = reinterpret_cast<__half*>(parts[3]);
  take(&t->dnt_inv, H);
  take(&t->upt_inv, d);
  float* maxima[2] = {};
  take(&maxima[0], H);
  take(&maxima[1], d);
  t->colmax_dn = reinterpret_cast<unsigned*>(maxima[0]);
  t->colmax_up = reinterpret_cast<unsigned*>(maxima[1]);
  return off;
}

static int build_support_tables(const int32_t* off, const int16_t* cols, int rows, int64_t ld, uint32_t* mask,
                                int32_t* first, cudaStream_t s) {
  if (ld > kMaxMaskWords) {
    set_error("support tables: %lld mask words per row above %d", (long long)ld, kMaxMaskWords);
    return HFFN_ERR_ARGUMENT;
  }
  const size_t smem = (size_t)kMaskWarps * ld * sizeof(uint32_t);
  support_tables_kernel<<<(rows + kMaskWarps - 1) / kMaskWarps, 32 * kMaskWarps, smem, s>>>(off, cols, rows, (int)ld,
                                                                                            mask, first);
  return launch_status("support tables");
}

}  // namespace tc

int64_t tc_train_workspace(const hffn_layer* L, int64_t n) {
  return 4 * tc::train_floats(L->d_model, L->d_ff, n, nullptr, nullptr);
}

// D16 != NULL: four GEMMs run in the fp16x3 format: the up GEMM and the down + MSE GEMM on D16 (fp16x3 operands of
// the current values) and the token packets of x (in the workspace of x's tf32 parts), their act operand the fp16 hi /
// lo pair (in the workspace of act's tf32 pairs); W_down^T gy and W_up^T gz on the transposes of D16 (built here) and
// the token packets of gy and gz (over the x and act workspaces, dead by then). The two sampled weight-gradient GEMMs
// stay on the tf32 copies (bound by their AdamW epilogue, measured: in fp16x3 the packing of their operands cost more
// than their MMAs saved), and the dense tf32 pairs, which this step then does not read, are not refreshed (the caller
// rebuilds them when it next needs them).
int tc_train_step(const hffn_layer* L, const void* up_hi, const void* up_lo, const void* down_hi, const void* down_lo,
                  const hffn_dense_f16x3* D16, const float* x, const float* target, float* y, float* gx,
                  const hffn_train_params* P, const hffn_adamw_step* opt, float* loss, void* work, int* err, int64_t n,
                  int64_t n_total, cudaStream_t s) {
  using namespace tc;
  const int d = L->d_model, H = L->d_ff, nn = (int)n;
  TrainWork w;
  train_floats(d, H, n, &w, reinterpret_cast<float*>(work));
  const int blocks = (int)((n + kTrainBN - 1) / kTrainBN);
  const int rows_dn = (D16 != nullptr ? kTrainPartsDownF16 : kTrainPartsDown) * blocks, rows_up = kTrainPartsUp * blocks;
  const int adam = opt != nullptr;
  const hffn_adamw_step st = opt ? *opt : hffn_adamw_step{};
  float* dense_up_hi = const_cast<float*>(reinterpret_cast<const float*>(up_hi));
  float* dense_up_lo = const_cast<float*>(reinterpret_cast<const float*>(up_lo));
  float* dense_dn_hi = const_cast<float*>(reinterpret_cast<const float*>(down_hi));
  float* dense_dn_lo = const_cast<float*>(reinterpret_cast<const float*>(down_lo));

  // x -> tf32 hi / lo (3xTF32 up GEMM) or token packets (fp16x3), over the same workspace
  __half* packets = reinterpret_cast<__half*>(w.x_hi);
  __half* act16_hi = reinterpret_cast<__half*>(w.act_hi);
  __half* act16_lo = act16_hi + n * H;
  if (D16 != nullptr) {
    if ((int64_t)((reinterpret_cast<uint8_t*>(w.z) - reinterpret_cast<uint8_t*>(w.x_hi))) < 2 * n * packet_halves(d) ||
        (int64_t)((reinterpret_cast<uint8_t*>(w.gy_hi) - reinterpret_cast<uint8_t*>(w.act_hi))) <
            2 * n * packet_halves(H)) {
      set_error("training step: the token packets do not fit the workspace (d_model %d, d_ff %d)", d, H);
      return HFFN_ERR_ARGUMENT;
    }
    split_f16_kernel<<<(unsigned)ceil_div(n * 32, 256), 256, 0, s>>>(x, n, d, D16->up_bound, packets);
    HFFN_TRY(launch_status("tc_split_f16"));
  } else {
    const int64_t count4 = n * d / 4;
    split_kernel<<<(int)std::min<int64_t>(std::max<int64_t>(ceil_div(count4, 256), 1), 148 * 8), 256, 0, s>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(w.x_hi), reinterpret_cast<float4*>(w.x_lo),
        count4);
    HFFN_TRY(launch_status("tc_split"));
  }
  split_transpose_kernel<<<dim3((unsigned)ceil_div(n, 32), (unsigned)ceil_div(d, 32)), dim3(32, 8), 0, s>>>(
      x, n, d, w.xt_hi, w.xt_lo, w.t_ld);
  HFFN_TRY(launch_status("tc_split_transpose"));
  HFFN_TRY(build_support_tables(L->out_offsets, L->out_hidden, d, w.dn_ld, w.dn_mask, w.dn_first, s));
  HFFN_TRY(build_support_tables(L->up_offsets, L->up_idx, H, w.up_ld, w.up_mask, w.up_first, s));
  if (D16 != nullptr) {
    // W_down^T [H, d] and W_up^T [d, H] in fp16x3, from the step's fp16x3 operands: the backward GEMMs' A operands,
    // K-major
    if (cudaMemsetAsync(w.colmax_dn, 0, (size_t)H * 4, s) != cudaSuccess ||
        cudaMemsetAsync(w.colmax_up, 0, (size_t)d * 4, s) != cudaSuccess)
      return launch_status("colmax memset");
    constexpr int kRowsPerBlock = 64;
    colmax_f16_kernel<<<dim3((unsigned)ceil_div(H, 256), (unsigned)ceil_div(d, kRowsPerBlock)), 256, 0, s>>>(
        reinterpret_cast<const __half*>(D16->down_hi), reinterpret_cast<const __half*>(D16->down_lo), D16->down_scale,
        d, H, kRowsPerBlock, w.colmax_dn);
    colmax_f16_kernel<<<dim3((unsigned)ceil_div(d, 256), (unsigned)ceil_div(H, kRowsPerBlock)), 256, 0, s>>>(
        reinterpret_cast<const __half*>(D16->up_hi), reinterpret_cast<const __half*>(D16->up_lo), D16->up_scale, H, d,
        kRowsPerBlock, w.colmax_up);
    HFFN_TRY(launch_status("colmax_f16"));
    transpose_f16_kernel<<<dim3((unsigned)(H / 32), (unsigned)(d / 32)), dim3(32, 8), 0, s>>>(
        reinterpret_cast<const __half*>(D16->down_hi), reinterpret_cast<const __half*>(D16->down_lo), D16->down_scale,
        d, H, w.colmax_dn, w.dnt_hi, w.dnt_lo, w.dnt_inv);
    transpose_f16_kernel<<<dim3((unsigned)(d / 32), (unsigned)(H / 32)), dim3(32, 8), 0, s>>>(
        reinterpret_cast<const __half*>(D16->up_hi), reinterpret_cast<const __half*>(D16->up_lo), D16->up_scale, H, d,
        w.colmax_up, w.upt_hi, w.upt_lo, w.upt_inv);
    HFFN_TRY(launch_status("transpose_f16"));
  }
  // 1. up: z, act = gelu(z) (+ act^T)                             D[H, n] = W_up[H, d] x[n, d]^T
  EpilogueArgs e1{};
  e1.bias = L->b_up;
  e1.out_hi = w.act_hi;
  e1.out_lo = w.act_lo;
  e1.z = w.z;
  e1.t_hi = w.actt_hi;
  e1.t_lo = w.actt_lo;
  e1.t_ld = w.t_ld;
  if (D16 != nullptr) {
    e1.out_hi = act16_hi;
    e1.out_lo = act16_lo;
    e1.row_inv = D16->up_scale;
    e1.tok_tab = reinterpret_cast<const float*>(packets + 2 * part_halves(d));
    e1.tok_stride = packet_halves(d) / 2;
    HFFN_TRY((launch_gemm<false, kTrainBN, 4, kUpT, f16_chunk<kUpT>(), 64, 16, false, false, true>(
        D16->up_hi, D16->up_lo, packets, packets + part_halves(d), H, nn, d, e1, err, s, 0, packet_halves(d))));
  } else {
    HFFN_TRY((launch_gemm<false, kTrainBN, 4, kUpT, kFp32Chunk, 64, 8>(up_hi, up_lo, w.x_hi, w.x_lo, H, nn, d, e1, err,
                                                                       s)));
  }
  // 2. down + MSE: y, gy = 2 (y - target) / (n_total d) (+ gy^T)  D[d, n] = W_down[d, H] act[n, H]^T
  EpilogueArgs e2{};
  e2.bias = L->b_down;
  e2.out_hi = y;
  e2.target = target;
  e2.gy_hi = w.gy_hi;
  e2.gy_lo = w.gy_lo;
  e2.scale = (float)(2.0 / ((double)n_total * d));
  e2.loss_partial = w.loss_p;
  e2.col_partial = w.dn_p;
  e2.t_hi = w.gyt_hi;
  e2.t_lo = w.gyt_lo;
  e2.t_ld = w.t_ld;
  if (D16 != nullptr) {
    e2.row_inv = D16->down_scale;
    e2.tok_tab = reinterpret_cast<const float*>(packets + 2 * part_halves(d));
    e2.tok_stride = packet_halves(d) / 2;
    HFFN_TRY((launch_gemm<false, kTrainBN, 4, kDownMse, f16_chunk<kDownMse>(), 64, 16, false, false, true>(
        D16->down_hi, D16->down_lo, act16_hi, act16_lo, d, nn, H, e2, err, s)));
  } else {
    HFFN_TRY((launch_gemm<false, kTrainBN, 4, kDownMse, kFp32Chunk, 64, 8>(down_hi, down_lo, w.act_hi, w.act_lo, d,
                                                                            nn, H, e2, err, s)));
  }
  // 3. gz = (W_down^T gy) * gelu'(z) (+ gz^T)                      D[H, n] = W_down^T[H, d] gy[n, d]^T
  EpilogueArgs e3{};
  e3.out_hi = w.gz_hi;
  e3.out_lo = w.gz_lo;
  e3.z_in = w.z;
  e3.col_partial = w.up_p;
  e3.t_hi = w.gzt_hi;
  e3.t_lo = w.gzt_lo;
  e3.t_ld = w.t_ld;
  if (D16 != nullptr) {
    // gy into token packets over the x packets' workspace (read for the last time by the down GEMM)
    __half* gy_pk = packets;
    split_pair_f16_kernel<<<(unsigned)ceil_div(n * 32, 256), 256, 0, s>>>(w.gy_hi, w.gy_lo, n, d, gy_pk);
    HFFN_TRY(launch_status("tc_split_pair gy"));
    e3.row_inv = w.dnt_inv;
    e3.tok_tab = reinterpret_cast<const float*>(gy_pk + 2 * part_halves(d));
    e3.tok_stride = packet_halves(d) / 2;
    HFFN_TRY((launch_gemm<false, kTrainBN, 4, kGradHidden, f16_chunk<kGradHidden>(), 64, 16, false, false, true>(
        w.dnt_hi, w.dnt_lo, gy_pk, gy_pk + part_halves(d), H, nn, d, e3, err, s, 0, packet_halves(d))));
  } else {
    HFFN_TRY((launch_gemm<false, kTrainBN, 4, kGradHidden, kFp32Chunk, 64, 16, true, false>(
        down_hi, down_lo, w.gy_hi, w.gy_lo, H, nn, d, e3, err, s, H, 0)));
  }
  // 4. gx = W_up^T gz                                              D[d, n] = W_up^T[d, H] gz[n, H]^T
  EpilogueArgs e4{};
  e4.out_hi = gx;
  if (D16 != nullptr) {
    // gz into token packets over the act parts' workspace (read for the last time by the down GEMM)
    __half* gz_pk = act16_hi;
    split_pair_f16_kernel<<<(unsigned)ceil_div(n * 32, 256), 256, 0, s>>>(w.gz_hi, w.gz_lo, n, H, gz_pk);
    HFFN_TRY(launch_status("tc_split_pair gz"));
    e4.row_inv = w.upt_inv;
    e4.tok_tab = reinterpret_cast<const float*>(gz_pk + 2 * part_halves(H));
    e4.tok_stride = packet_halves(H) / 2;
    HFFN_TRY((launch_gemm<false, kTrainBN, 4, kDown, f16_chunk<kDown>(), 64, 8, false, false, true>(
        w.upt_hi, w.upt_lo, gz_pk, gz_pk + part_halves(H), d, nn, H, e4, err, s, 0, packet_halves(H))));
  } else {
    HFFN_TRY((launch_gemm<false, kTrainBN, 4, kDown, kFp32Chunk, 64, 8, true, false>(up_hi, up_lo, w.gz_hi, w.gz_lo, d,
                                                                                      nn, H, e4, err, s, d, 0)));
  }
  // 5. g_down sampled on the output-major support, AdamW, W_down refreshed   D[d, H] = gy^T[d, n] act^T[H, n]^T
  //    (both operands K-major: the feature-major copies)
  EpilogueArgs e5{};
  e5.mask = w.dn_mask;
  e5.first = w.dn_first;
  e5.mask_ld = w.dn_ld;
  e5.value = P->out_val.value;
  e5.grad = P->out_val.grad;
  e5.m = P->out_val.m;
  e5.v = P->out_val.v;
  e5.dense_hi = D16 != nullptr ? nullptr : dense_dn_hi;    // the fp16x3 step reads no tf32 pair: no refresh
  e5.dense_lo = D16 != nullptr ? nullptr : dense_dn_lo;
  e5.adam = adam;
  e5.step = st;
  HFFN_TRY((launch_gemm<false, kTrainBN, 4, kSampled, kFp32Chunk, 64, 8, false, false>(
      w.gyt_hi, w.gyt_lo, w.actt_hi, w.actt_lo, d, H, nn, e5, err, s, w.t_ld, w.t_ld)));
  // 6. g_up sampled on the hidden-major support, AdamW, W_up refreshed        D[H, d] = gz^T[H, n] x^T[d, n]^T
  EpilogueArgs e6{};
  e6.mask = w.up_mask;
  e6.first = w.up_first;
  e6.mask_ld = w.up_ld;
  e6.value = P->up_val.value;
  e6.grad = P->up_val.grad;
  e6.m = P->up_val.m;
  e6.v = P->up_val.v;
  e6.dense_hi = D16 != nullptr ? nullptr : dense_up_hi;
  e6.dense_lo = D16 != nullptr ? nullptr : dense_up_lo;
  e6.adam = adam;
  e6.step = st;
  HFFN_TRY((launch_gemm<false, kTrainBN, 4, kSampled, kFp32Chunk, 64, 8, false, false>(
      w.gzt_hi, w.gzt_lo, w.xt_hi, w.xt_lo, H, d, nn, e6, err, s, w.t_ld, w.t_ld)));
  // 7. biases and loss
  bias_reduce_kernel<<<(d + 255) / 256, 256, 0, s>>>(w.dn_p, rows_dn, d, P->b_down, adam, st);
  HFFN_TRY(launch_status("bias_reduce down"));
  bias_reduce_kernel<<<(H + 255) / 256, 256, 0, s>>>(w.up_p, rows_up, H, P->b_up, adam, st);
  HFFN_TRY(launch_status("bias_reduce up"));
  loss_blocks_kernel<<<kLossBlocks, 256, 0, s>>>(w.loss_p, (int64_t)rows_dn * d,
                                                 reinterpret_cast<double*>(w.loss_blocks));
  HFFN_TRY(launch_status("loss_blocks"));
  loss_reduce_kernel<<<1, 32, 0, s>>>(reinterpret_cast<const double*>(w.loss_blocks), kLossBlocks,
                                      1.0 / ((double)n * d), loss);
  return launch_status("loss_reduce");
}

// D^T [N, M] = (A B^T)^T for the operand layouts of the training GEMMs: A [M, K] K-major or stored [K, M] (MN-major,
// leading dimension lda), B likewise; float32 3xTF32 hi / lo parts, plain y-store epilogue. A test entry of the GEMM
// engine itself.
int tc_gemm_f32(int a_mn, int b_mn, const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                float* d, int M, int N, int K, int64_t lda, int64_t ldb, int* err, cudaStream_t s) {
  using namespace tc;
  EpilogueArgs e{};
  e.out_hi = d;
  if (!a_mn && !b_mn)
    return launch_gemm<false, kTrainBN, 4, kDown, kFp32Chunk, 64, 8, false, false>(a_hi, a_lo, b_hi, b_lo, M, N, K, e,
                                                                                   err, s, lda, ldb);
  if (a_mn && !b_mn)
    return launch_gemm<false, kTrainBN, 4, kDown, kFp32Chunk, 64, 8, true, false>(a_hi, a_lo, b_hi, b_lo, M, N, K, e,
                                                                                  err, s, lda, ldb);
  if (!a_mn && b_mn)
    return launch_gemm<false, kTrainBN, 4, kDown, kFp32Chunk, 64, 8, false, true>(a_hi, a_lo, b_hi, b_lo, M, N, K, e,
                                                                                  err, s, lda, ldb);
  return launch_gemm<false, kTrainBN, 4, kDown, kFp32Chunk, 64, 8, true, true>(a_hi, a_lo, b_hi, b_lo, M, N, K, e, err,
                                                                               s, lda, ldb);
}

// down with the outputs routed to their owners' buffers (the neuron-sharded forward's reduction target).
int tc_down_peer(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo, const void* b,
                 void* const* peers, int world, int64_t tokens_per_owner, int* err, int d, int H, int64_t n,
                 cudaStream_t s) {
  tc::EpilogueArgs dn{};
  dn.bias = b;
  for (int p = 0; p < world && p < tc::kMaxPeers; ++p) dn.peers[p] = peers[p];
  dn.tokens_per_owner = tokens_per_owner;
  dn.rows = d;
  const int nn = (int)n;
  if (dtype == HFFN_BF16)
    return tc::launch_forward_gemm<true, tc::kDownPeer>(w_hi, nullptr, act_hi, nullptr, d, nn, H, dn, err, s);
  return tc::launch_forward_gemm<false, tc::kDownPeer>(w_hi, w_lo, act_hi, act_lo, d, nn, H, dn, err, s);
}

// out[i] = slots[0][i] + slots[1][i] + ... in slot order (float32 accumulation).
template <typename T>
__global__ void sum_slots_kernel(const T* __restrict__ slots, int count, int64_t elems, T* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < elems; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = to_f(slots[i]);
    for (int k = 1; k < count; ++k) acc += to_f(slots[(int64_t)k * elems + i]);
    out[i] = from_f<T>(acc);
  }
}

int tc_sum_slots(int dtype, const void* slots, int count, int64_t elems, void* out, cudaStream_t s) {
  const int blocks = (int)std::min<int64_t>(std::max<int64_t>(ceil_div(elems, 256), 1), 148 * 16);
  if (dtype == HFFN_BF16)
    sum_slots_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(slots), count, elems,
                                                          reinterpret_cast<__nv_bfloat16*>(out));
  else
    sum_slots_kernel<float><<<blocks, 256, 0, s>>>(reinterpret_cast<const float*>(slots), count, elems,
                                                  reinterpret_cast<float*>(out));
  return launch_status("sum_slots");
}

void tc_set_max_ctas(int max_ctas) { tc::g_max_ctas.store(max_ctas > 0 ? max_ctas : 0); }

void tc_set_tile_tokens(int tokens) { tc::g_tile_tokens.store(tokens); }

int64_t tc_forward_workspace(int dtype, const hffn_layer* L, int64_t n) {
  if (dtype == HFFN_BF16) return n * L->d_ff * 2;
  return 4 * (2 * n * L->d_model + 2 * n * L->d_ff);
}

int tc_densify(int dtype, const int32_t* off, const int16_t* idx, const void* val, int rows, int cols, void* hi,
               void* lo, cudaStream_t s) {
  const size_t bytes = (size_t)rows * cols * (dtype == HFFN_BF16 ? 2 : 4);
  if (cudaMemsetAsync(hi, 0, bytes, s) != cudaSuccess) return launch_status("densify memset");
  if (dtype != HFFN_BF16 && cudaMemsetAsync(lo, 0, bytes, s) != cudaSuccess) return launch_status("densify memset");
  const int blocks = (int)ceil_div((int64_t)rows * 32, 256);
  tc::densify_kernel<<<blocks, 256, 0, s>>>(off, idx, val, rows, cols, dtype == HFFN_BF16, hi, lo);
  return launch_status("densify");
}

}  // namespace hffn
