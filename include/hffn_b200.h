/* HFFN fixed-support sparse FFN on B200 (sm_100a): the C ABI of libhffn_b200.so.
 *
 * One layer is y = W_down gelu(W_up x + b_up) + b_down stored per hidden neuron (compact supports, int16 indices,
 * int32 offsets, float32 or bfloat16 values). No dense weight, mask, gradient or moment exists behind this ABI.
 *
 * Conventions of every entry:
 *  - arguments are raw device pointers, sizes and a cudaStream_t passed as void* (NULL: the legacy default stream);
 *  - the device of `stream` is made current for the call; launches are queued on `stream` and the host is never
 *    synchronised; nothing is allocated: the caller passes every buffer, workspaces included;
 *  - the return value is a status (HFFN_OK = 0); hffn_last_error() gives the message of the calling thread's last
 *    failure. Argument errors are detected before any launch.
 * Layouts: x, y, gy, gx token-major [n, d_model]; the hidden activations act (h), z and gz hidden-major [d_ff, n]
 * (element r * n + t), as the reference runtime holds them (runtime/gpu/nvidia/ffn/training/kernels_train.py:9-11).
 */
#ifndef HFFN_B200_H
#define HFFN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define HFFN_OK 0
#define HFFN_ERR_ARGUMENT 1    /* bad shape, pointer, mode or range: nothing was launched */
#define HFFN_ERR_CUDA 2        /* a CUDA call or launch failed */
#define HFFN_ERR_LAYOUT 3      /* hffn_validate_layout found an invalid offset or index */

/* Storage types of x, the values, the biases, act and y (arithmetic is float32 in both). */
#define HFFN_F32 0
#define HFFN_BF16 1

/* Kernel modes, the names of the reference runtime (runtime/gpu/nvidia/common/kernels/hffn_cuda/runtime.py:22-38).
 * up:   coop = warp per neuron reducing its slots over the lanes, for tiny n;
 *       lane = token tile of 16 per neuron, x staged in shared memory;   tile = token tile of 32 per neuron.
 * down: coop = warp per output reducing its edges over the lanes, for tiny n;
 *       tiled = output owner over a 4-token tile of act staged in shared memory; blocked = 8-token tile.
 * AUTO picks by n and the shape (hffn_up_mode / hffn_down_mode). */
#define HFFN_MODE_AUTO (-1)
#define HFFN_UP_COOP 0
#define HFFN_UP_LANE 1
#define HFFN_UP_TILE 2
#define HFFN_DOWN_COOP 0
#define HFFN_DOWN_TILED 1
#define HFFN_DOWN_BLOCKED 2

/* The kernel arrays of one layer (HFFNLayer, runtime.py:41-53): up slots hidden-major, down edges output-major.
 * Value pointers are float* or __nv_bfloat16* per the call's dtype. */
typedef struct hffn_layer {
  int32_t d_model, d_ff;
  int64_t nnz_up, nnz_down;
  const void* b_up;            /* [d_ff] */
  const int32_t* up_offsets;   /* [d_ff + 1] */
  const int16_t* up_idx;       /* [nnz_up] input feature of each slot */
  const void* up_val;          /* [nnz_up] */
  const void* b_down;          /* [d_model] */
  const int32_t* out_offsets;  /* [d_model + 1] */
  const int16_t* out_hidden;   /* [nnz_down] hidden neuron of each edge */
  const void* out_val;         /* [nnz_down] */
} hffn_layer;

/* Transposed supports of the backward, positions into the arrays above (transposed_supports,
 * runtime/gpu/nvidia/ffn/training/train_runtime.py:39-56). */
typedef struct hffn_supports {
  const int32_t* in_offsets;   /* [d_model + 1] */
  const int32_t* in_pos;       /* [nnz_up] position of each slot in up_* (input-major, hidden ascending) */
  const int16_t* in_hidden;    /* [nnz_up] */
  const int32_t* hid_offsets;  /* [d_ff + 1] */
  const int32_t* hid_pos;      /* [nnz_down] position of each edge in out_* (hidden-major, output ascending) */
  const int16_t* hid_output;   /* [nnz_down] */
} hffn_supports;

/* One compact float32 parameter array with its gradient and AdamW moments, all of `count` entries. */
typedef struct hffn_param {
  float* value;
  float* grad;   /* may be NULL in the fused backward + AdamW: the gradient is then never stored */
  float* m;
  float* v;
  int64_t count;
} hffn_param;

typedef struct hffn_train_params {
  hffn_param up_val, b_up, out_val, b_down;
} hffn_train_params;

/* The step scalars of one AdamW update, computed in float64 on the host and passed as float32
 * (runtime/gpu/nvidia/ffn/training/train_runtime.py:195-207):
 * lr_decay = lr * wd, step_size = lr / (1 - beta1^k), bias2_sqrt = sqrt(1 - beta2^k). */
typedef struct hffn_adamw_step {
  float lr_decay, beta1, one_minus_beta1, beta2, one_minus_beta2, step_size, bias2_sqrt, eps;
} hffn_adamw_step;

const char* hffn_version(void);
const char* hffn_last_error(void);

/* Policy of the reference runtime's up_mode / down_mode (runtime.py:29-38), on this build's kernels. */
int hffn_up_mode(int64_t n, int32_t d_model);
int hffn_down_mode(int64_t n, int32_t d_ff);

/* Up projection + bias + exact GELU, optional float32 pre-activation store.
 * Replaces the up_coop / up_lane / up_tile (and _z) kernels (runtime/gpu/nvidia/common/kernels/hffn_cuda/
 * kernels.py:102-143). act[r * n + t] = gelu(z), z[r * n + t] = b[r] + sum_e w[e] x[t, idx[e]] if z != NULL. */
int hffn_up(int dtype, int mode, const void* x, const int32_t* up_offsets, const int16_t* up_idx, const void* up_val,
            const void* b_up, void* act, float* z, int32_t d_model, int32_t d_ff, int64_t n, void* stream);

/* Down projection, output owners: y[t, o] = sum over the edges of o of out_val * act[hid, t] + b_down[o].
 * Replaces down_coop / down_tiled / down_blocked (kernels.py:145-191). */
int hffn_down(int dtype, int mode, const void* act, const int32_t* out_offsets, const int16_t* out_hidden,
              const void* out_val, const void* b_down, void* y, int32_t d_model, int32_t d_ff, int64_t n, void* stream);

/* Whole forward of one layer: up then down. Replaces HFFNRuntime._launch (runtime.py:134-163).
 * act: [d_ff, n] workspace of the dtype; z: NULL or float32 [d_ff, n]. */
int hffn_forward(int dtype, const hffn_layer* layer, const void* x, void* y, void* act, float* z, int64_t n,
                 int up_mode, int down_mode, void* stream);

/* Float32 entries of the workspace hffn_backward needs for n tokens. */
int64_t hffn_backward_workspace(const hffn_layer* layer, int64_t n);

/* Backward of the last forward (z, act of that forward), float32. Computes gz [d_ff, n], gx [n, d_model] and the
 * four compact gradients. With adamw == NULL the gradients are written to params->*.grad (the reference's backward,
 * runtime/gpu/nvidia/ffn/training/train_runtime.py:163-193). With adamw != NULL each gradient entry is applied by
 * AdamW as soon as it is complete (the reference's backward followed by adamw, train_runtime.py:195-214) and stored
 * only where params->*.grad != NULL. params->*.value must be the layer's up_val, b_up, out_val, b_down. */
int hffn_backward(const hffn_layer* layer, const hffn_supports* supports, const float* x, const float* gy,
                  const float* z, const float* act, float* gz, float* gx, const hffn_train_params* params,
                  const hffn_adamw_step* adamw, float* work, int64_t n, void* stream);

/* AdamW on one compact array from its stored gradient. Replaces the adamw kernel (kernels_train.py:246-258). */
int hffn_adamw(const hffn_param* param, const hffn_adamw_step* step, void* stream);

/* MSE loss of the training benchmark (no counterpart in the reference, whose step takes gy from the caller):
 * gy = 2 (y - target) / (n d_model); *loss = mean((y - target)^2), float32 on the device. work: 1024 floats. */
int hffn_mse(const float* y, const float* target, float* gy, float* loss, int64_t n, int32_t d_model, float* work,
             void* stream);

/* The error flag of the decode kernels (the cooperative mode at n <= 8 of hffn_up / hffn_down / hffn_forward, which
 * copy their slots into shared memory by TMA bulk copies): 0, or the code of the first bounded wait that expired
 * (301), on the current device. Synchronous; clear != 0 resets it. No counterpart in the reference (whose kernels
 * do not wait). */
int hffn_decode_error(int32_t* value, int clear);

/* Device-side check of a layer's arrays (offsets from 0 to nnz, non-decreasing, indices in range): sets *flag
 * (device int32, cleared by the call) to 1 if any array is invalid. The export reader's checks
 * (runtime/common/pythia/hffn_pythia/export.py:37-45) on device-resident arrays. */
int hffn_validate_layout(const hffn_layer* layer, int32_t* flag, void* stream);

/* Device-side layout build (no host sort): bytes of the workspace of hffn_build_out_major / hffn_build_supports. */
int64_t hffn_build_layout_workspace(int32_t d_model, int32_t d_ff, int64_t nnz_up, int64_t nnz_down);

/* The down edges of one layer in output-major order from its hidden-major storage: out_offsets [d_model + 1] (edges
 * per output, prefix-summed), out_hidden [nnz_down] (the neuron of each edge) and out_val [nnz_down] (its value, in
 * the storage type `dtype`), by a stable counting sort of down_idx on the device: the edges of one output keep
 * ascending neuron order. Equal bit for bit to the host form, HFFNLayer.from_hidden_major
 * (runtime/gpu/nvidia/common/kernels/hffn_cuda/runtime.py:55-67). *flag (device int32) is set to 1 if an offset or
 * an index is out of range (those entries are skipped; the outputs are then undefined). */
int hffn_build_out_major(int dtype, int32_t d_model, int32_t d_ff, const int32_t* down_offsets,
                         const int16_t* down_idx, const void* down_val, int64_t nnz_down, int32_t* out_offsets,
                         int16_t* out_hidden, void* out_val, void* work, int32_t* flag, void* stream);

/* The transposed supports of the training step on the device: up slots input-major (in_offsets [d_model + 1], in_pos
 * [nnz_up] positions into the up arrays, in_hidden [nnz_up] their neurons) and down edges hidden-major (hid_offsets
 * [d_ff + 1], hid_pos [nnz_down] positions into the output-major arrays, hid_output [nnz_down] their outputs), by
 * stable counting sorts: equal bit for bit to transposed_supports (runtime/gpu/nvidia/ffn/training/
 * train_runtime.py:39-56). *flag as for hffn_build_out_major. */
int hffn_build_supports(int32_t d_model, int32_t d_ff, const int32_t* up_offsets, const int16_t* up_idx,
                        int64_t nnz_up, const int32_t* out_offsets, const int16_t* out_hidden, int64_t nnz_down,
                        int32_t* in_offsets, int32_t* in_pos, int16_t* in_hidden, int32_t* hid_offsets,
                        int32_t* hid_pos, int16_t* hid_output, void* work, int32_t* flag, void* stream);

/* Dense tensor-core operands of one layer, built by hffn_densify: W_up [d_ff, d_model] and W_down [d_model, d_ff] with
 * zeros off the support. float32: the tf32 hi and lo parts of the 3xTF32 split; bfloat16: hi only (lo NULL). */
typedef struct hffn_dense {
  void* up_hi;
  void* up_lo;
  void* down_hi;
  void* down_lo;
} hffn_dense;

/* Materialise the dense [rows, cols] matrix of a CSR-by-row support (up: rows = d_ff over up_offsets / up_idx /
 * up_val; down: rows = d_model over out_offsets / out_hidden / out_val). The reference has no dense path: this is the
 * "support densified at high density" layout of the tensor-core forward, built once per layer. */
int hffn_densify(int dtype, const int32_t* offsets, const int16_t* idx, const void* val, int32_t rows, int32_t cols,
                 void* hi, void* lo, void* stream);

/* The up projection on the tensor cores (same function as hffn_up; replaces the up_* kernels, kernels.py:102-143):
 * act = gelu(W_up x + b_up), TOKEN-major [n, d_ff]. float32: x is split into tf32 hi/lo parts in x_split
 * (2 n d_model floats) and act is written as its hi (act_hi) and lo (act_lo) parts; z NULL or float32 [n, d_ff].
 * bfloat16: w_lo, act_lo, x_split and z NULL. err: device int32 set non-zero if a wait timed out. */
int hffn_up_tc(int dtype, const void* x, const void* w_hi, const void* w_lo, const void* b_up, void* act_hi,
               void* act_lo, float* z, void* x_split, int32_t* err, int32_t d_model, int32_t d_ff, int64_t n,
               void* stream);

/* The down projection on the tensor cores (same function as hffn_down; replaces the down_* kernels,
 * kernels.py:145-191): y = W_down act + b_down from the token-major act of hffn_up_tc. */
int hffn_down_tc(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo,
                 const void* b_down, void* y, int32_t* err, int32_t d_model, int32_t d_ff, int64_t n, void* stream);

/* Bytes of the workspace hffn_forward_tc needs for n tokens. */
int64_t hffn_forward_tc_workspace(int dtype, const hffn_layer* layer, int64_t n);

/* The forward on the tcgen05 tensor cores, the same function as hffn_forward (it replaces HFFNRuntime._launch,
 * runtime.py:134-163, for large n): up GEMM with a bias + GELU epilogue, then down GEMM with a bias epilogue.
 * y [n, d_model]; z NULL or float32 [n, d_ff] TOKEN-major; work: hffn_forward_tc_workspace bytes;
 * err: device int32, set non-zero by a kernel whose wait timed out (never cleared by the call). */
int hffn_forward_tc(int dtype, const hffn_layer* layer, const hffn_dense* dense, const void* x, void* y, float* z,
                    void* work, int32_t* err, int64_t n, void* stream);

/* Dense tensor-core operands of one float32 layer in the fp16x3 format, built by hffn_densify_f16x3: W_up [d_ff,
 * d_model] and W_down [d_model, d_ff], zeros off the support, each row r scaled by a power of two 2^e_r (its largest
 * |value| into [2^14, 2^15)) and stored as fp16 parts hi = rn(w 2^e_r), lo = rn(w 2^e_r - hi); up_scale [d_ff] and
 * down_scale [d_model] hold 2^-e_r; up_bound [2] = {max_r sum_k |W_up[r, k]|, max_r |b_up[r]|} (the bound of |z| the
 * activations' scales derive from). A product of fp16 parts is exact and each part holds tf32's 11-bit significand, so
 * the forward computes the 3xTF32 split's three products (hi hi + hi lo + lo hi) at the f16 tensor-core rate. */
typedef struct hffn_dense_f16x3 {
  void* up_hi;
  void* up_lo;
  float* up_scale;
  void* down_hi;
  void* down_lo;
  float* down_scale;
  float* up_bound;
} hffn_dense_f16x3;

/* Build one projection's fp16x3 operands from its CSR-by-row support (up: rows = d_ff over up_offsets / up_idx /
 * up_val with bias = b_up and bound = the up_bound of the struct; down: rows = d_model over out_offsets / out_hidden /
 * out_val, bias and bound NULL). hi, lo: fp16 [rows, cols]; scale: float32 [rows]. */
int hffn_densify_f16x3(const int32_t* offsets, const int16_t* idx, const float* val, const float* bias, int32_t rows,
                       int32_t cols, void* hi, void* lo, float* scale, float* bound, void* stream);

/* Bytes of the workspace of the fp16x3 forward for n tokens. */
int64_t hffn_forward_f16x3_workspace(const hffn_layer* layer, int64_t n);

/* The float32 forward on the tcgen05 tensor cores in the fp16x3 format (the same function as hffn_forward and
 * hffn_forward_tc, which it replaces for float32 layers, runtime.py:134-163): x split per token into scaled fp16
 * parts, the up GEMM with a scale + bias + GELU epilogue that stores act as scaled fp16 parts, the down GEMM with a
 * scale + bias epilogue. y [n, d_model]; z NULL or float32 [n, d_ff] TOKEN-major; work:
 * hffn_forward_f16x3_workspace bytes; err as for hffn_forward_tc. */
int hffn_forward_f16x3(const hffn_layer* layer, const hffn_dense_f16x3* dense, const float* x, float* y, float* z,
                       void* work, int32_t* err, int64_t n, void* stream);

/* The two halves of hffn_forward_f16x3, for callers that run them apart (the benchmark's per-kernel timing):
 * hffn_up_f16x3 leaves the token packets and act in `work` for hffn_down_f16x3 over the same n. */
int hffn_up_f16x3(const float* x, const hffn_dense_f16x3* dense, const float* b_up, float* z, void* work, int32_t* err,
                  int32_t d_model, int32_t d_ff, int64_t n, void* stream);
int hffn_down_f16x3(const void* work, const hffn_dense_f16x3* dense, const float* b_down, float* y, int32_t* err,
                    int32_t d_model, int32_t d_ff, int64_t n, void* stream);

/* Token packets of the fp16x3 forward: per token, hffn_f16x3_packet_bytes(d_model) = 4 D + 64 bytes (D = d_model
 * rounded up to 32), the x row scaled by a power of two 2^e_t (its largest |value| into [2^14, 2^15)) as fp16 hi and
 * lo parts of D halves each (the first d_model used), then float32 {2^-e_t, 2^a_t, 2^-a_t, 0} and 48 bytes of padding
 * (a_t: the scale of the token's activations, from dense->up_bound; every piece 64-byte aligned). The
 * packets of several ranks' tokens concatenate into one batch, so the neuron-sharded forward splits each rank's own
 * tokens once and gathers the packets instead of gathering x and splitting the whole gathered batch on every rank. */
int64_t hffn_f16x3_packet_bytes(int32_t d_model);

/* x [n, d_model] float32 -> packets [n] (16-byte aligned). */
int hffn_split_f16x3(const float* x, const hffn_dense_f16x3* dense, void* packets, int32_t d_model, int32_t d_ff,
                     int64_t n, void* stream);

/* hffn_forward_f16x3 from the packets of its n tokens (work: hffn_forward_f16x3_workspace bytes). */
int hffn_forward_f16x3_packets(const hffn_layer* layer, const hffn_dense_f16x3* dense, const void* packets, float* y,
                               float* z, void* work, int32_t* err, int64_t n, void* stream);

/* The tensor-core down projection of a rank's neuron shard, fused with the reduction's transfer: the partial output of
 * token t is stored directly into the receive buffer of the rank that owns t (peer memory over NVLink, plain stores,
 * no collective call): peer_y[t / tokens_per_owner] + (t % tokens_per_owner) * d_model. n = world x tokens_per_owner;
 * peer_y: `world` device addresses (host array). Replaces the reduce-scatter of the partial outputs (no reference
 * counterpart: the reference has no multi-GPU path). */
int hffn_down_tc_peer(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo,
                      const void* b_down, const uint64_t* peer_y, int32_t world, int64_t tokens_per_owner,
                      int32_t* err, int32_t d_model, int32_t d_ff, int64_t n, void* stream);

/* out[i] = slots[0][i] + ... + slots[count - 1][i] in slot order (float32 accumulation): the owner's sum of the partial
 * outputs its peers stored. */
int hffn_sum_slots(int dtype, const void* slots, int32_t count, int64_t elems, void* out, void* stream);

/* The neuron-sharded forward over a stream of batches, exchanged through NVLink peer memory (no reference
 * counterpart: the reference runs one GPU). Buffers come from the caller (symmetric memory mapped on every rank);
 * positions j = 0 .. world - 1 name rank (rank + j) % world. Per batch of n tokens: gather[b] [world n, d] holds the
 * gathered batch (rows [0, n) this rank's, staged from the caller's input; rows of position j pulled from
 * gather_peer[b][j]); the shard runs over it; its partial outputs go to slot_peer[s][j] (this rank's slot in the
 * receive buffer of position j) from partial[b] by copy engines, or, with partial == NULL, from the down GEMM's
 * epilogue; slots[s] [world, n, d] receives the peers' partials and is summed in rank order into the output. The
 * signal pads (uint32 [world], zeroed on every rank before the first run) carry the barrier between iterations. */
typedef struct hffn_peer_config {
  int32_t world;
  int32_t rank;
  int64_t tokens;                 /* n: tokens per rank per batch */
  int32_t dtype;
  void* gather[2];
  uint64_t gather_peer[2][8];
  void* slots[3];
  uint64_t slot_peer[3][8];
  void* partial[2];               /* both NULL: delivery by the down GEMM's epilogue */
  uint32_t* signal;
  uint64_t signal_peer[8];
  void* work;                     /* hffn_forward_tc_workspace(world n) bytes */
} hffn_peer_config;

/* A pipeline over the rank's shard (layer: its compact arrays; dense: its densified operands). err: the device error
 * flag its kernels set (201: a barrier wait ran out: a peer is dead or late). */
int hffn_peer_pipeline_create(const hffn_peer_config* config, const hffn_layer* layer, const hffn_dense* dense,
                              int32_t* err, void** pipeline);

/* outs[k] [n, d] = the layer's output for this rank's batch xs[k] [n, d], k < count; every rank calls with the same
 * count, on a stream of the pipeline's device. Iteration k stages batch k, waits for the pulls of batch k - 1 and the
 * deliveries of batch k - 3, passes the barrier, pulls batch k, runs the shard over batch k - 1, delivers its
 * partials and sums batch k - 3. A run that fails part-way leaves the pipeline unusable (its later runs are refused:
 * the ranks' barriers may be out of step); destroy it and create a new one on every rank. */
int hffn_peer_pipeline_run(void* pipeline, const void* const* xs, void* const* outs, int32_t count, void* stream);

int hffn_peer_pipeline_destroy(void* pipeline);

/* One barrier over the signal pads: writes epoch into this rank's slot of every peer's pad, then waits until every
 * peer's slot of signal holds at least epoch, for at most timeout_ns (then err = 201 and the kernel returns). */
int hffn_peer_barrier(uint32_t* signal, const uint64_t* signal_peer, int32_t world, int32_t rank, uint32_t epoch,
                      int64_t timeout_ns, int32_t* err, void* stream);

/* Cap on the CTAs of the persistent tensor-core GEMMs, process-wide (0: one per SM, the default). A tuning knob with
 * no reference counterpart: the neuron-sharded forward leaves a few SMs to the NCCL kernels so that its collectives
 * run alongside the GEMMs. */
int hffn_set_tc_max_ctas(int32_t max_ctas);

/* Token width of the forward GEMMs' tiles, process-wide: 0 (the default: 256, or 128 / 64 for a GEMM whose 256-wide
 * tiles would leave more than half of the SMs idle) or a forced 256, 128 or 64. A tuning knob with no reference
 * counterpart. */
int hffn_set_tc_tile_tokens(int32_t tokens);

/* The GEMM engine of the tensor-core path alone (a test entry; no reference counterpart): out [n, m] = (A B^T)^T with
 * A [m, k] (a_mn = 0: K contiguous) or stored [k, m] (a_mn = 1, leading dimension lda), B [n, k] or stored [k, n]
 * (ldb), float32 operands as tf32 hi / lo parts (3xTF32). */
int hffn_gemm_tc_f32(int a_mn, int b_mn, const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                     float* out, int32_t m, int32_t n, int32_t k, int64_t lda, int64_t ldb, int32_t* err, void* stream);

/* Bytes of the workspace hffn_train_step_tc needs for n tokens. */
int64_t hffn_train_step_tc_workspace(const hffn_layer* layer, int64_t n);

/* One MSE training step on the tcgen05 tensor cores (float32): forward, loss, backward and AdamW, the
 * tensor-core form of HFFNTrainRuntime.step (runtime/gpu/nvidia/ffn/training/train_runtime.py:209-214) with the
 * training benchmark's MSE loss. Six GEMMs over the dense operands (up; down with the MSE gradient in its epilogue;
 * W_down^T gy with gelu'; W_up^T gz; gy^T act and gz^T x sampled on the supports). With adamw != NULL every gradient
 * entry is applied by AdamW in the epilogue that completes it and the dense operands are refreshed in place (so
 * they stay consistent with the compact values); gradients are stored where params->*.grad != NULL. With
 * adamw == NULL the gradients are stored and nothing is updated (data parallelism: exchange, then hffn_adamw and
 * hffn_densify). gy = 2 (y - target) / (n_total d_model); *loss = mean((y - target)^2) over this call's n tokens.
 * Requires d_model and d_ff multiples of 32 and, for the sampled update, the up slots of each neuron in ascending
 * input order (the output-major down edges always are). x, target, y, gx token-major [n, d_model]. The GEMMs run on
 * the 3xTF32 pairs of `dense`, except with dense16 != NULL (fp16x3 operands of the same, current values, from
 * hffn_densify_f16x3) four of them run in the fp16x3 format at the f16 rate: up, down + MSE, W_down^T gy and W_up^T gz
 * (on transposes of dense16 built by the step); the sampled weight-gradient GEMMs stay on tf32 copies of the
 * activations and gradients, and the dense tf32 pairs are then NOT refreshed (rebuild them with hffn_densify before
 * using them again; dense16 must be rebuilt after every applied step in any case). */
int hffn_train_step_tc(const hffn_layer* layer, const hffn_dense* dense, const hffn_dense_f16x3* dense16,
                       const float* x, const float* target, float* y, float* gx, const hffn_train_params* params,
                       const hffn_adamw_step* adamw, float* loss, void* work, int32_t* err, int64_t n, int64_t n_total,
                       void* stream);

/* Forward that allocates nothing and needs no workspace from the caller. No counterpart in the reference.
 * Some callers can hand this library only their input and output buffers: a plugin whose host framework owns every
 * device allocation and exposes no allocator, or a caller that must not call cudaMalloc on its path (it can
 * synchronise the device). This entry runs the same CUDA-core kernels as hffn_forward under its policy and keeps the
 * hidden activations in a 16 MiB array that the library holds on every GPU that loads it, until the process exits.
 * Limit: d_ff x n x sizeof(storage) <= hffn_forward_noalloc_max_bytes() (16 MiB); larger calls return
 * HFFN_ERR_ARGUMENT before any launch. The first call on a device looks up the array's device address with that
 * device current; make that first call before any stream capture. The address is cached per device ordinal and
 * belongs to the device's primary context (the runtime's and torch's): it is valid while that context lives, not
 * after cudaDeviceReset and not under a context the caller created and made current. Every call uses the same
 * array: calls that overlap on the GPU (other streams, other host threads) race on it. */
int64_t hffn_forward_noalloc_max_bytes(void);
int hffn_forward_noalloc(int dtype, const hffn_layer* layer, const void* x, void* y, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HFFN_B200_H */
