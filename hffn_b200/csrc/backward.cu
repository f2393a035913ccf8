// HFFN backward and compact AdamW on the CUDA cores (float32), with the AdamW update fused into the kernel that
// completes each gradient entry.
//
// Quantities (the reference's kernels_train.py:38-56, runtime/gpu/nvidia/ffn/training):
//   gz[r, t]   = (sum over the down edges of r, hidden-major order, of out_val * gy[t, o]) * gelu'(z[r, t])
//   gx[t, i]   = sum over the up slots of input i, input-major order (hidden ascending), of up_val * gz[r, t]
//   g_down[q]  = sum_t gy[t, o_q] h[r_q, t],   gb_down[o] = sum_t gy[t, o]       (output-major edge order)
//   g_up[e]    = sum_t gz[r_e, t] x[t, i_e],   gb_up[r]   = sum_t gz[r, t]       (hidden-major slot order)
// Token sums of the weight gradients: the tokens are cut into G <= 16 groups of consecutive tokens; a warp owns one
// (row, group), lane l adds the tokens l, l + 32, ... of the group in ascending order and the xor tree reduces the
// lanes (group partial P_g); the entry is ((P_0 + P_1) + P_2) + ..., summed by one thread. The order depends on n
// only, not on the grid or the launch order: the same bits on every call.
// The value arrays are read by gz and gx before the AdamW update writes them: gz and gx run first.
#include "common.cuh"

namespace hffn {

constexpr int kThreads = 512;
constexpr int kSmemBudget = 200 * 1024;
constexpr int kTargetCtas = 4 * 148;
constexpr int kMaxGroups = 16;
constexpr int kGroupMinTokens = 256;

// ---------------------------------------------------------------------------------------------------------------
// AdamW in the order of PyTorch's fused AdamW (kernels_train.py:246-258):
//   p -= lr*wd*p; m = b1 m + (1 - b1) g; v = b2 v + (1 - b2) g g; p -= step_size * m / (sqrt(v) / bias2_sqrt + eps)
__device__ __forceinline__ void adamw_entry(float* p, float* m, float* v, int64_t i, float g,
                                            const hffn_adamw_step& s) {
  float pi = p[i];
  pi -= s.lr_decay * pi;
  const float mi = s.beta1 * m[i] + s.one_minus_beta1 * g;
  const float vi = s.beta2 * v[i] + s.one_minus_beta2 * g * g;
  m[i] = mi;
  v[i] = vi;
  p[i] = pi - s.step_size * mi / (sqrtf(vi) / s.bias2_sqrt + s.eps);
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, int64_t count, hffn_adamw_step s) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    adamw_entry(p, m, v, i, g[i], s);
}

// ---------------------------------------------------------------------------------------------------------------
// transposes [rows, cols] -> [cols, rows] through a 32 x 33 tile

__global__ void transpose_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t rows, int64_t cols) {
  __shared__ float tile[32][33];
  const int64_t c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t r = r0 + k, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[k][threadIdx.x] = src[r * cols + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t c = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[c * rows + r] = tile[threadIdx.x][k];
  }
}

static int transpose(const float* src, float* dst, int64_t rows, int64_t cols, cudaStream_t s) {
  dim3 grid((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, s>>>(src, dst, rows, cols);
  return launch_status("transpose");
}

// ---------------------------------------------------------------------------------------------------------------
// gz: hidden owners over a token tile of gy staged [d][TT + 1]; the weights are out_val read through hid_pos.

template <int TT>
__global__ void __launch_bounds__(kThreads)
grad_hidden_kernel(const float* __restrict__ gy, const float* __restrict__ z, const int32_t* __restrict__ hoff,
                   const int32_t* __restrict__ hpos, const int16_t* __restrict__ hout, const float* __restrict__ v,
                   float* __restrict__ gz, int d, int H, int n, int neurons_per_cta) {
  extern __shared__ float gs[];
  constexpr int S = TT + 1, G = 32 / TT;
  const int t0 = blockIdx.y * TT;
  for (int k = threadIdx.x; k < TT * d; k += kThreads) {
    const int tt = k / d, i = k - tt * d;
    const int t = t0 + tt;
    gs[i * S + tt] = t < n ? gy[(int64_t)t * d + i] : 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TT, tt = lane - sub * TT;
  const int t = t0 + tt;
  const float* col = gs + tt;
  const int r_end = min(H, (blockIdx.x + 1) * neurons_per_cta);
  for (int r = blockIdx.x * neurons_per_cta + warp * G + sub; r < r_end; r += (kThreads / 32) * G) {
    int j = hoff[r];
    const int end = hoff[r + 1];
    float acc = 0.f;
    for (; j + 4 <= end; j += 4) {
      const int o0 = hout[j], o1 = hout[j + 1], o2 = hout[j + 2], o3 = hout[j + 3];
      const float w0 = v[hpos[j]], w1 = v[hpos[j + 1]], w2 = v[hpos[j + 2]], w3 = v[hpos[j + 3]];
      const float a0 = col[o0 * S], a1 = col[o1 * S], a2 = col[o2 * S], a3 = col[o3 * S];
      acc += w0 * a0;
      acc += w1 * a1;
      acc += w2 * a2;
      acc += w3 * a3;
    }
    for (; j < end; ++j) acc += v[hpos[j]] * col[hout[j] * S];
    if (t < n) {
      const int64_t at = (int64_t)r * n + t;
      gz[at] = acc * gelu_grad(z[at]);
    }
  }
}

// gx: input owners over a token tile of gz staged [H][TT + 1]; the weights are up_val read through in_pos.
template <int TT>
__global__ void __launch_bounds__(kThreads)
grad_x_kernel(const float* __restrict__ gz, const int32_t* __restrict__ ioff, const int32_t* __restrict__ ipos,
              const int16_t* __restrict__ ihid, const float* __restrict__ w, float* __restrict__ gx, int d, int H,
              int n, int inputs_per_cta) {
  extern __shared__ float gs[];
  constexpr int S = TT + 1, G = 32 / TT;
  const int t0 = blockIdx.y * TT;
  for (int k = threadIdx.x; k < TT * H; k += kThreads) {
    const int r = k / TT, tt = k - r * TT;
    const int t = t0 + tt;
    gs[r * S + tt] = t < n ? gz[(int64_t)r * n + t] : 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / TT, tt = lane - sub * TT;
  const int t = t0 + tt;
  const float* col = gs + tt;
  const int i_end = min(d, (blockIdx.x + 1) * inputs_per_cta);
  for (int i = blockIdx.x * inputs_per_cta + warp * G + sub; i < i_end; i += (kThreads / 32) * G) {
    int j = ioff[i];
    const int end = ioff[i + 1];
    float acc = 0.f;
    for (; j + 4 <= end; j += 4) {
      const int r0 = ihid[j], r1 = ihid[j + 1], r2 = ihid[j + 2], r3 = ihid[j + 3];
      const float w0 = w[ipos[j]], w1 = w[ipos[j + 1]], w2 = w[ipos[j + 2]], w3 = w[ipos[j + 3]];
      const float a0 = col[r0 * S], a1 = col[r1 * S], a2 = col[r2 * S], a3 = col[r3 * S];
      acc += w0 * a0;
      acc += w1 * a1;
      acc += w2 * a2;
      acc += w3 * a3;
    }
    for (; j < end; ++j) acc += w[ipos[j]] * col[ihid[j] * S];
    if (t < n) gx[(int64_t)t * d + i] = acc;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Sampled products: warp per (owner row, token group). own [rows][n], partner [*][n] feature-/hidden-major.
// Writes, per group g, the partial of each slot at out[g * stride + slot] and of the owner at
// out_bias[g * stride + row]; with one group and `adamw` set, applies AdamW to the entry instead.

struct SddmmTarget {
  float* g;        // gradient (or partial column base)
  float* gb;
  float *p, *m, *v;        // AdamW state of the values (fused, one group)
  float *pb, *mb, *vb;     // AdamW state of the biases
};

__global__ void __launch_bounds__(kThreads)
sddmm_kernel(const float* __restrict__ own, const float* __restrict__ partner, const int32_t* __restrict__ off,
             const int16_t* __restrict__ pidx, int rows, int n, int group_tokens, int64_t stride, SddmmTarget out,
             int fused, hffn_adamw_step s) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int g = blockIdx.y;
  const int tb = g * group_tokens, te = min(n, tb + group_tokens);
  const float* orow = own + (int64_t)row * n;
  const int64_t part = (int64_t)g * stride;
  float partial = 0.f;
  for (int t = tb + lane; t < te; t += 32) partial += orow[t];
  float total = warp_sum(partial);
  if (lane == 0) {
    if (fused) {
      if (out.gb) out.gb[row] = total;
      adamw_entry(out.pb, out.mb, out.vb, row, total, s);
    } else {
      out.gb[part + row] = total;
    }
  }
  const int end = off[row + 1];
  for (int q = off[row]; q < end; ++q) {
    const float* prow = partner + (int64_t)pidx[q] * n;
    partial = 0.f;
    for (int t = tb + lane; t < te; t += 32) partial += orow[t] * prow[t];
    total = warp_sum(partial);
    if (lane == 0) {
      if (fused) {
        if (out.g) out.g[q] = total;
        adamw_entry(out.p, out.m, out.v, q, total, s);
      } else {
        out.g[part + q] = total;
      }
    }
  }
}

// Fixed-order sum of the group partials ws[g][j], g ascending, then store and / or AdamW, one thread per column.
// Columns: [0, c1) g_down, [c1, c2) gb_down, [c2, c3) g_up, [c3, c4) gb_up.
struct ReduceTarget {
  hffn_param down, b_down, up, b_up;
};

__global__ void reduce_groups_kernel(const float* __restrict__ ws, int64_t stride, int groups, int64_t c1, int64_t c2,
                                     int64_t c3, int64_t c4, ReduceTarget t, int fused, hffn_adamw_step s) {
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < c4; j += (int64_t)gridDim.x * blockDim.x) {
    float sum = ws[j];
    for (int g = 1; g < groups; ++g) sum += ws[(int64_t)g * stride + j];
    const hffn_param* p;
    int64_t i;
    if (j < c1) { p = &t.down; i = j; }
    else if (j < c2) { p = &t.b_down; i = j - c1; }
    else if (j < c3) { p = &t.up; i = j - c2; }
    else { p = &t.b_up; i = j - c3; }
    if (p->grad) p->grad[i] = sum;
    if (fused) adamw_entry(p->value, p->m, p->v, i, sum, s);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// MSE: gy = 2 (y - t) / (n d); per-block partial sums of (y - t)^2 in double, then one block sums them in order.

__global__ void mse_kernel(const float* __restrict__ y, const float* __restrict__ target, float* __restrict__ gy,
                           int64_t count, float scale, double* __restrict__ partials) {
  __shared__ double red[kThreads / 32];
  double acc = 0.0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const float diff = y[i] - target[i];
    gy[i] = scale * diff;
    acc += (double)diff * diff;
  }
  for (int sft = 16; sft > 0; sft >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, sft);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) sum += red[w];
    partials[blockIdx.x] = sum;
  }
}

__global__ void mse_finish_kernel(const double* __restrict__ partials, int count, double inv, float* __restrict__ loss) {
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int b = 0; b < count; ++b) sum += partials[b];
    *loss = (float)(sum * inv);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// layout validation

__global__ void validate_kernel(const int32_t* __restrict__ off, int64_t count, int64_t nnz,
                                const int16_t* __restrict__ idx, int bound, int32_t* __restrict__ flag) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k <= count; k += stride) {
    const int32_t o = off[k];
    bool bad = o < 0 || o > nnz || (k == 0 && o != 0) || (k == count && o != nnz) || (k < count && off[k + 1] < o);
    if (bad) *flag = 1;
  }
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nnz; e += stride) {
    const int i = idx[e];
    if (i < 0 || i >= bound) *flag = 1;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// launchers

static int tile_tokens(int64_t rows, int64_t n) {
  int tt = 32;
  while (tt > 1 && rows * (tt + 1) * 4 > kSmemBudget) tt >>= 1;
  int cap = 1;
  while (cap < n && cap < 32) cap <<= 1;
  return tt < cap ? tt : cap;
}

static int units_per_cta(int units, int64_t tiles, int per_pass) {
  int64_t blocks = (kTargetCtas + tiles - 1) / tiles;
  int64_t max_blocks = ceil_div(units, per_pass);
  if (blocks > max_blocks) blocks = max_blocks;
  if (blocks < 1) blocks = 1;
  return (int)ceil_div(units, blocks);
}

int backward_groups(int64_t n, int* group_tokens) {
  int64_t gt = ceil_div(n, kMaxGroups);
  if (gt < kGroupMinTokens) gt = kGroupMinTokens;
  gt = ceil_div(gt, 32) * 32;
  if (group_tokens) *group_tokens = (int)gt;
  return (int)ceil_div(n, gt);
}

static int launch_grad_hidden(const float* gy, const float* z, const hffn_supports* S, const float* out_val,
                              float* gz, int d, int H, int64_t n, cudaStream_t s) {
  const int tt = tile_tokens(d, n);
  const int64_t tiles = ceil_div(n, tt);
  const int per = units_per_cta(H, tiles, (kThreads / 32) * (32 / tt));
  dim3 grid((unsigned)ceil_div(H, per), (unsigned)tiles);
  const size_t smem = (size_t)d * (tt + 1) * 4;
#define CASE(TTV)                                                                                                \
  case TTV: {                                                                                                    \
    auto k = grad_hidden_kernel<TTV>;                                                                            \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                            \
    k<<<grid, kThreads, smem, s>>>(gy, z, S->hid_offsets, S->hid_pos, S->hid_output, out_val, gz, d, H, (int)n,  \
                                   per);                                                                         \
    break;                                                                                                       \
  }
  switch (tt) { CASE(32) CASE(16) CASE(8) CASE(4) CASE(2) CASE(1) }
#undef CASE
  return launch_status("grad_hidden");
}

static int launch_grad_x(const float* gz, const hffn_supports* S, const float* up_val, float* gx, int d, int H,
                         int64_t n, cudaStream_t s) {
  const int tt = tile_tokens(H, n);
  const int64_t tiles = ceil_div(n, tt);
  const int per = units_per_cta(d, tiles, (kThreads / 32) * (32 / tt));
  dim3 grid((unsigned)ceil_div(d, per), (unsigned)tiles);
  const size_t smem = (size_t)H * (tt + 1) * 4;
#define CASE(TTV)                                                                                                \
  case TTV: {                                                                                                    \
    auto k = grad_x_kernel<TTV>;                                                                                 \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                            \
    k<<<grid, kThreads, smem, s>>>(gz, S->in_offsets, S->in_pos, S->in_hidden, up_val, gx, d, H, (int)n, per);   \
    break;                                                                                                       \
  }
  switch (tt) { CASE(32) CASE(16) CASE(8) CASE(4) CASE(2) CASE(1) }
#undef CASE
  return launch_status("grad_x");
}

int64_t backward_workspace(const hffn_layer* L, int64_t n) {
  const int groups = backward_groups(n, nullptr);
  const int64_t stride = L->nnz_down + L->d_model + L->nnz_up + L->d_ff;
  return 2 * (int64_t)L->d_model * n + (groups > 1 ? groups * stride : 0);
}

int launch_backward(const hffn_layer* L, const hffn_supports* S, const float* x, const float* gy, const float* z,
                    const float* act, float* gz, float* gx, const hffn_train_params* P, const hffn_adamw_step* opt,
                    float* work, int64_t n, cudaStream_t s) {
  const int d = L->d_model, H = L->d_ff;
  float* x_t = work;
  float* gy_t = work + (int64_t)d * n;
  float* partials = gy_t + (int64_t)d * n;
  int group_tokens = 0;
  const int groups = backward_groups(n, &group_tokens);
  const int64_t c1 = L->nnz_down, c2 = c1 + d, c3 = c2 + L->nnz_up, c4 = c3 + H;
  const hffn_adamw_step step = opt ? *opt : hffn_adamw_step{};
  const int fused = opt != nullptr;

  HFFN_TRY(transpose(x, x_t, n, d, s));
  HFFN_TRY(transpose(gy, gy_t, n, d, s));
  // gz and gx read out_val and up_val before any update
  HFFN_TRY(launch_grad_hidden(gy, z, S, (const float*)L->out_val, gz, d, H, n, s));
  HFFN_TRY(launch_grad_x(gz, S, (const float*)L->up_val, gx, d, H, n, s));

  const bool direct = groups == 1;
  SddmmTarget down{}, up{};
  if (direct) {
    down = {P->out_val.grad, P->b_down.grad, P->out_val.value, P->out_val.m, P->out_val.v,
            P->b_down.value, P->b_down.m, P->b_down.v};
    up = {P->up_val.grad, P->b_up.grad, P->up_val.value, P->up_val.m, P->up_val.v,
          P->b_up.value, P->b_up.m, P->b_up.v};
  } else {
    down.g = partials;
    down.gb = partials + c1;
    up.g = partials + c2;
    up.gb = partials + c3;
  }
  const int64_t stride = direct ? 0 : c4;
  const int sddmm_fused = direct && fused;
  dim3 gd((unsigned)ceil_div(d, kThreads / 32), (unsigned)groups);
  sddmm_kernel<<<gd, kThreads, 0, s>>>(gy_t, act, L->out_offsets, L->out_hidden, d, (int)n, group_tokens, stride,
                                       down, sddmm_fused, step);
  HFFN_TRY(launch_status("grad_down"));
  dim3 gu((unsigned)ceil_div(H, kThreads / 32), (unsigned)groups);
  sddmm_kernel<<<gu, kThreads, 0, s>>>(gz, x_t, L->up_offsets, L->up_idx, H, (int)n, group_tokens, stride, up,
                                       sddmm_fused, step);
  HFFN_TRY(launch_status("grad_up"));
  if (!direct) {
    ReduceTarget t{P->out_val, P->b_down, P->up_val, P->b_up};
    const int64_t blocks = std::min<int64_t>(ceil_div(c4, 256), 148 * 16);
    reduce_groups_kernel<<<(unsigned)blocks, 256, 0, s>>>(partials, c4, groups, c1, c2, c3, c4, t, fused, step);
    HFFN_TRY(launch_status("reduce_groups"));
  }
  return HFFN_OK;
}

int launch_adamw(const hffn_param* P, const hffn_adamw_step* step, cudaStream_t s) {
  const int64_t blocks = std::min<int64_t>(ceil_div(P->count, 256), 148 * 16);
  if (blocks == 0) return HFFN_OK;
  adamw_kernel<<<(unsigned)blocks, 256, 0, s>>>(P->value, P->grad, P->m, P->v, P->count, *step);
  return launch_status("adamw");
}

int launch_mse(const float* y, const float* target, float* gy, float* loss, int64_t n, int d, float* work,
               cudaStream_t s) {
  const int64_t count = n * d;
  const int blocks = (int)std::min<int64_t>(std::max<int64_t>(ceil_div(count, kThreads * 8), 1), 512);
  double* partials = reinterpret_cast<double*>(work);
  mse_kernel<<<blocks, kThreads, 0, s>>>(y, target, gy, count, 2.0f / (float)count, partials);
  HFFN_TRY(launch_status("mse"));
  mse_finish_kernel<<<1, 32, 0, s>>>(partials, blocks, 1.0 / (double)count, loss);
  return launch_status("mse_finish");
}

int launch_validate(const hffn_layer* L, int32_t* flag, cudaStream_t s) {
  if (cudaMemsetAsync(flag, 0, sizeof(int32_t), s) != cudaSuccess) return launch_status("validate memset");
  validate_kernel<<<148, 256, 0, s>>>(L->up_offsets, L->d_ff, L->nnz_up, L->up_idx, L->d_model, flag);
  HFFN_TRY(launch_status("validate up"));
  validate_kernel<<<148, 256, 0, s>>>(L->out_offsets, L->d_model, L->nnz_down, L->out_hidden, L->d_ff, flag);
  return launch_status("validate down");
}

}  // namespace hffn
