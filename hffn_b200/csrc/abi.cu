// The extern "C" entries of libhffn_b200.so (declared in include/hffn_b200.h): argument checks, device binding and
// dispatch to the kernels. Nothing here allocates device memory or synchronises the host.
#include <cstring>

#include "common.cuh"

namespace hffn {

int launch_up(int dtype, int mode, const void* x, const int32_t* off, const int16_t* idx, const void* w,
              const void* b, void* act, float* z, int d, int H, int64_t n, cudaStream_t s,
              const int16_t* next_idx = nullptr, const void* next_val = nullptr, int64_t next_nnz = 0);
int launch_down(int dtype, int mode, const void* act, const int32_t* off, const int16_t* hid, const void* v,
                const void* bias, void* y, int d, int H, int64_t n, cudaStream_t s);
int64_t max_staged_rows();
int64_t backward_workspace(const hffn_layer* L, int64_t n);
int launch_backward(const hffn_layer* L, const hffn_supports* S, const float* x, const float* gy, const float* z,
                    const float* act, float* gz, float* gx, const hffn_train_params* P, const hffn_adamw_step* opt,
                    float* work, int64_t n, cudaStream_t s);
int launch_adamw(const hffn_param* P, const hffn_adamw_step* step, cudaStream_t s);
int launch_mse(const float* y, const float* target, float* gy, float* loss, int64_t n, int d, float* work,
               cudaStream_t s);
int launch_validate(const hffn_layer* L, int32_t* flag, cudaStream_t s);
int tc_forward(int dtype, const hffn_layer* L, const void* up_hi, const void* up_lo, const void* down_hi,
               const void* down_lo, const void* x, void* y, float* z, void* work, int* err, int64_t n,
               cudaStream_t s);
int64_t tc_forward_workspace(int dtype, const hffn_layer* L, int64_t n);
int tc_up(int dtype, const void* x, const void* w_hi, const void* w_lo, const void* b, void* act_hi, void* act_lo,
          float* z, void* x_split, int* err, int d, int H, int64_t n, cudaStream_t s);
int64_t tc_train_workspace(const hffn_layer* L, int64_t n);
void tc_set_max_ctas(int max_ctas);
void tc_set_tile_tokens(int tokens);
int tc_down_peer(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo, const void* b,
                 void* const* peers, int world, int64_t tokens_per_owner, int* err, int d, int H, int64_t n,
                 cudaStream_t s);
int tc_sum_slots(int dtype, const void* slots, int count, int64_t elems, void* out, cudaStream_t s);
int tc_gemm_f32(int a_mn, int b_mn, const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                float* d, int M, int N, int K, int64_t lda, int64_t ldb, int* err, cudaStream_t s);
int tc_train_step(const hffn_layer* L, const void* up_hi, const void* up_lo, const void* down_hi, const void* down_lo,
                  const hffn_dense_f16x3* D16,
                  const float* x, const float* target, float* y, float* gx, const hffn_train_params* P,
                  const hffn_adamw_step* opt, float* loss, void* work, int* err, int64_t n, int64_t n_total,
                  cudaStream_t s);
int tc_down(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo, const void* b,
            void* y, int* err, int d, int H, int64_t n, cudaStream_t s, bool pdl = false);
int tc_densify(int dtype, const int32_t* off, const int16_t* idx, const void* val, int rows, int cols, void* hi,
               void* lo, cudaStream_t s);
int64_t tc_f16_workspace(int d, int H, int64_t n);
int64_t tc_f16_packet_bytes(int d);
int tc_split_f16(const float* x, const hffn_dense_f16x3* D, void* packets, int d, int64_t n, cudaStream_t s);
int tc_forward_f16_packets(const void* packets, const hffn_dense_f16x3* D, const float* b_up, const float* b_down,
                           float* y, float* z, void* work, int* err, int d, int H, int64_t n, cudaStream_t s);
int tc_up_f16(const float* x, const hffn_dense_f16x3* D, const float* b, float* z, void* work, int* err, int d, int H,
              int64_t n, cudaStream_t s);
int tc_down_f16(const void* work, const hffn_dense_f16x3* D, const float* b, float* y, int* err, int d, int H,
                int64_t n, cudaStream_t s);
int tc_densify_f16(const int32_t* off, const int16_t* idx, const float* val, const float* bias, int rows, int cols,
                   void* hi, void* lo, float* scale, float* bound, cudaStream_t s);

static thread_local char g_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
}

const char* last_error() { return g_error; }

// Token counts: every kernel indexes tokens with 32-bit ints and act with 64-bit offsets.
constexpr int64_t kMaxTokens = int64_t(1) << 30;
constexpr int kCoopMaxTokens = 8;

int check_shape(int dtype, int32_t d, int32_t H, int64_t n) {
  HFFN_REQUIRE(dtype == HFFN_F32 || dtype == HFFN_BF16, "unknown dtype %d", dtype);
  HFFN_REQUIRE(d >= 1 && d <= 32767 && H >= 1 && H <= 32767, "d_model %d / d_ff %d out of range [1, 32767]", d, H);
  HFFN_REQUIRE(n >= 1 && n <= kMaxTokens, "token count %lld out of range", (long long)n);
  return HFFN_OK;
}

static int resolve_up(int mode, int64_t n, int32_t d) {
  if (mode == HFFN_MODE_AUTO) return hffn_up_mode(n, d);
  return mode;
}

static int resolve_down(int mode, int64_t n, int32_t H) {
  if (mode == HFFN_MODE_AUTO) return hffn_down_mode(n, H);
  return mode;
}

int check_layer(const hffn_layer* L) {
  HFFN_REQUIRE(L != nullptr, "null layer");
  HFFN_REQUIRE(L->b_up && L->up_offsets && L->up_idx && L->up_val && L->b_down && L->out_offsets && L->out_hidden &&
                   L->out_val,
               "null layer array");
  HFFN_REQUIRE(L->nnz_up >= 0 && L->nnz_down >= 0 && L->nnz_up < (int64_t(1) << 31) &&
                   L->nnz_down < (int64_t(1) << 31),
               "edge counts out of the int32 offset range");
  return HFFN_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace hffn

using namespace hffn;

extern "C" {

const char* hffn_version(void) { return "hffn_b200 0.1 sm_100a"; }

const char* hffn_last_error(void) { return last_error(); }

int hffn_up_mode(int64_t n, int32_t d_model) {
  (void)d_model;
  return n <= kCoopMaxTokens ? HFFN_UP_COOP : HFFN_UP_TILE;
}

int hffn_down_mode(int64_t n, int32_t d_ff) {
  (void)d_ff;
  return n <= kCoopMaxTokens ? HFFN_DOWN_COOP : HFFN_DOWN_BLOCKED;
}

// hffn_up, and the up half of hffn_forward, whose decode kernel also prefetches the down arrays (next_*) into L2.
static int up_call(int dtype, int mode, const void* x, const int32_t* up_offsets, const int16_t* up_idx,
                   const void* up_val, const void* b_up, void* act, float* z, int32_t d_model, int32_t d_ff, int64_t n,
                   void* stream, const int16_t* next_idx, const void* next_val, int64_t next_nnz) {
  HFFN_TRY(check_shape(dtype, d_model, d_ff, n));
  HFFN_REQUIRE(x && up_offsets && up_idx && up_val && b_up && act, "null pointer argument");
  HFFN_REQUIRE(z == nullptr || dtype == HFFN_F32, "z is stored by the float32 path only");
  mode = resolve_up(mode, n, d_model);
  HFFN_REQUIRE(mode == HFFN_UP_COOP || mode == HFFN_UP_LANE || mode == HFFN_UP_TILE, "unknown up mode %d", mode);
  HFFN_REQUIRE(mode == HFFN_UP_COOP || d_model <= max_staged_rows(), "d_model %d exceeds the staged tile", d_model);
  HFFN_TRY(bind_stream_device(stream));
  return launch_up(dtype, mode, x, up_offsets, up_idx, up_val, b_up, act, z, d_model, d_ff, n,
                   static_cast<cudaStream_t>(stream), next_idx, next_val, next_nnz);
}

int hffn_up(int dtype, int mode, const void* x, const int32_t* up_offsets, const int16_t* up_idx, const void* up_val,
            const void* b_up, void* act, float* z, int32_t d_model, int32_t d_ff, int64_t n, void* stream) {
  return up_call(dtype, mode, x, up_offsets, up_idx, up_val, b_up, act, z, d_model, d_ff, n, stream, nullptr,
                 nullptr, 0);
}

int hffn_down(int dtype, int mode, const void* act, const int32_t* out_offsets, const int16_t* out_hidden,
              const void* out_val, const void* b_down, void* y, int32_t d_model, int32_t d_ff, int64_t n,
              void* stream) {
  HFFN_TRY(check_shape(dtype, d_model, d_ff, n));
  HFFN_REQUIRE(act && out_offsets && out_hidden && out_val && b_down && y, "null pointer argument");
  mode = resolve_down(mode, n, d_ff);
  HFFN_REQUIRE(mode == HFFN_DOWN_COOP || mode == HFFN_DOWN_TILED || mode == HFFN_DOWN_BLOCKED,
               "unknown down mode %d", mode);
  HFFN_REQUIRE(mode == HFFN_DOWN_COOP || d_ff <= max_staged_rows(), "d_ff %d exceeds the staged tile", d_ff);
  HFFN_TRY(bind_stream_device(stream));
  return launch_down(dtype, mode, act, out_offsets, out_hidden, out_val, b_down, y, d_model, d_ff, n,
                     static_cast<cudaStream_t>(stream));
}

int hffn_forward(int dtype, const hffn_layer* layer, const void* x, void* y, void* act, float* z, int64_t n,
                 int up_mode, int down_mode, void* stream) {
  HFFN_TRY(check_layer(layer));
  HFFN_TRY(up_call(dtype, up_mode, x, layer->up_offsets, layer->up_idx, layer->up_val, layer->b_up, act, z,
                   layer->d_model, layer->d_ff, n, stream, layer->out_hidden, layer->out_val, layer->nnz_down));
  return hffn_down(dtype, down_mode, act, layer->out_offsets, layer->out_hidden, layer->out_val, layer->b_down, y,
                   layer->d_model, layer->d_ff, n, stream);
}

int64_t hffn_backward_workspace(const hffn_layer* layer, int64_t n) {
  if (layer == nullptr || n < 1) return -1;
  return backward_workspace(layer, n);
}

static int check_param(const hffn_param& p, int64_t count, bool need_grad, bool need_state, const char* name) {
  HFFN_REQUIRE(p.count == count, "%s: count %lld, expected %lld", name, (long long)p.count, (long long)count);
  HFFN_REQUIRE(!need_grad || p.grad, "%s: null gradient", name);
  HFFN_REQUIRE(!need_state || (p.value && p.m && p.v), "%s: null value or moment", name);
  return HFFN_OK;
}

int hffn_backward(const hffn_layer* layer, const hffn_supports* supports, const float* x, const float* gy,
                  const float* z, const float* act, float* gz, float* gx, const hffn_train_params* params,
                  const hffn_adamw_step* adamw, float* work, int64_t n, void* stream) {
  HFFN_TRY(check_layer(layer));
  HFFN_TRY(check_shape(HFFN_F32, layer->d_model, layer->d_ff, n));
  HFFN_REQUIRE(supports && supports->in_offsets && supports->in_pos && supports->in_hidden && supports->hid_offsets &&
                   supports->hid_pos && supports->hid_output,
               "null support array");
  HFFN_REQUIRE(x && gy && z && act && gz && gx && params && work, "null pointer argument");
  HFFN_REQUIRE(layer->d_model <= max_staged_rows() && layer->d_ff <= max_staged_rows(), "shape exceeds the staged tile");
  const bool fused = adamw != nullptr;
  HFFN_TRY(check_param(params->up_val, layer->nnz_up, !fused, fused, "up_val"));
  HFFN_TRY(check_param(params->b_up, layer->d_ff, !fused, fused, "b_up"));
  HFFN_TRY(check_param(params->out_val, layer->nnz_down, !fused, fused, "out_val"));
  HFFN_TRY(check_param(params->b_down, layer->d_model, !fused, fused, "b_down"));
  HFFN_REQUIRE(!fused || (params->up_val.value == layer->up_val && params->b_up.value == layer->b_up &&
                          params->out_val.value == layer->out_val && params->b_down.value == layer->b_down),
               "fused AdamW: the parameter values must be the layer's arrays");
  HFFN_TRY(bind_stream_device(stream));
  return launch_backward(layer, supports, x, gy, z, act, gz, gx, params, adamw, work, n,
                         static_cast<cudaStream_t>(stream));
}

int hffn_adamw(const hffn_param* param, const hffn_adamw_step* step, void* stream) {
  HFFN_REQUIRE(param && step, "null pointer argument");
  HFFN_REQUIRE(param->count >= 0, "negative count");
  HFFN_REQUIRE(param->count == 0 || (param->value && param->grad && param->m && param->v), "null array");
  HFFN_TRY(bind_stream_device(stream));
  return launch_adamw(param, step, static_cast<cudaStream_t>(stream));
}

int hffn_mse(const float* y, const float* target, float* gy, float* loss, int64_t n, int32_t d_model, float* work,
             void* stream) {
  HFFN_REQUIRE(y && target && gy && loss && work, "null pointer argument");
  HFFN_REQUIRE(n >= 1 && d_model >= 1, "empty shape");
  HFFN_TRY(bind_stream_device(stream));
  return launch_mse(y, target, gy, loss, n, d_model, work, static_cast<cudaStream_t>(stream));
}

int hffn_validate_layout(const hffn_layer* layer, int32_t* flag, void* stream) {
  HFFN_TRY(check_layer(layer));
  HFFN_REQUIRE(flag != nullptr, "null flag");
  HFFN_TRY(bind_stream_device(stream));
  return launch_validate(layer, flag, static_cast<cudaStream_t>(stream));
}

int hffn_densify(int dtype, const int32_t* offsets, const int16_t* idx, const void* val, int32_t rows, int32_t cols,
                 void* hi, void* lo, void* stream) {
  HFFN_REQUIRE(dtype == HFFN_F32 || dtype == HFFN_BF16, "unknown dtype %d", dtype);
  HFFN_REQUIRE(rows >= 1 && cols >= 1 && rows <= 32767 && cols <= 32767, "dense shape out of range");
  HFFN_REQUIRE(offsets && idx && val && hi && (dtype == HFFN_BF16 || lo), "null pointer argument");
  HFFN_TRY(bind_stream_device(stream));
  return tc_densify(dtype, offsets, idx, val, rows, cols, hi, lo, static_cast<cudaStream_t>(stream));
}

int64_t hffn_forward_tc_workspace(int dtype, const hffn_layer* layer, int64_t n) {
  if (layer == nullptr || n < 1 || (dtype != HFFN_F32 && dtype != HFFN_BF16)) return -1;
  return tc_forward_workspace(dtype, layer, n);
}

int hffn_forward_tc(int dtype, const hffn_layer* layer, const hffn_dense* dense, const void* x, void* y, float* z,
                    void* work, int32_t* err, int64_t n, void* stream) {
  HFFN_TRY(check_layer(layer));
  HFFN_TRY(check_shape(dtype, layer->d_model, layer->d_ff, n));
  HFFN_REQUIRE(n <= (int64_t(1) << 31) - 1, "token count beyond 2^31 - 1");
  HFFN_REQUIRE(layer->d_model % 8 == 0 && layer->d_ff % 8 == 0, "tensor-core path: d_model and d_ff multiples of 8");
  HFFN_REQUIRE(dense && dense->up_hi && dense->down_hi && (dtype == HFFN_BF16 || (dense->up_lo && dense->down_lo)),
               "null dense operand");
  HFFN_REQUIRE(x && y && work && err, "null pointer argument");
  HFFN_REQUIRE(z == nullptr || dtype == HFFN_F32, "z is stored by the float32 path only");
  HFFN_REQUIRE(aligned16(x) && aligned16(work) && aligned16(dense->up_hi) && aligned16(dense->down_hi) &&
                   (dtype == HFFN_BF16 || (aligned16(dense->up_lo) && aligned16(dense->down_lo))),
               "tensor-core operands must be 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  return tc_forward(dtype, layer, dense->up_hi, dense->up_lo, dense->down_hi, dense->down_lo, x, y, z, work, err, n,
                    static_cast<cudaStream_t>(stream));
}

static int check_tc(int dtype, int32_t d_model, int32_t d_ff, int64_t n) {
  HFFN_TRY(check_shape(dtype, d_model, d_ff, n));
  HFFN_REQUIRE(n <= (int64_t(1) << 31) - 1, "token count beyond 2^31 - 1");
  HFFN_REQUIRE(d_model % 8 == 0 && d_ff % 8 == 0, "tensor-core path: d_model and d_ff multiples of 8");
  return HFFN_OK;
}

int hffn_densify_f16x3(const int32_t* offsets, const int16_t* idx, const float* val, const float* bias, int32_t rows,
                       int32_t cols, void* hi, void* lo, float* scale, float* bound, void* stream) {
  HFFN_REQUIRE(rows >= 1 && cols >= 1 && rows <= 32767 && cols <= 32767, "dense shape out of range");
  HFFN_REQUIRE(offsets && idx && val && hi && lo && scale, "null pointer argument");
  HFFN_REQUIRE(bias == nullptr || bound != nullptr, "a bias needs the bound it feeds");
  HFFN_TRY(bind_stream_device(stream));
  return tc_densify_f16(offsets, idx, val, bias, rows, cols, hi, lo, scale, bound, static_cast<cudaStream_t>(stream));
}

int64_t hffn_forward_f16x3_workspace(const hffn_layer* layer, int64_t n) {
  if (layer == nullptr || n < 1) return -1;
  return tc_f16_workspace(layer->d_model, layer->d_ff, n);
}

static int check_dense_f16(const hffn_dense_f16x3* D, bool up, bool down) {
  HFFN_REQUIRE(D != nullptr, "null dense operands");
  HFFN_REQUIRE(!up || (D->up_hi && D->up_lo && D->up_scale && D->up_bound), "null up operand");
  HFFN_REQUIRE(!down || (D->down_hi && D->down_lo && D->down_scale), "null down operand");
  HFFN_REQUIRE((!up || (aligned16(D->up_hi) && aligned16(D->up_lo))) &&
                   (!down || (aligned16(D->down_hi) && aligned16(D->down_lo))),
               "tensor-core operands must be 16-byte aligned");
  return HFFN_OK;
}

int hffn_up_f16x3(const float* x, const hffn_dense_f16x3* dense, const float* b_up, float* z, void* work, int32_t* err,
                  int32_t d_model, int32_t d_ff, int64_t n, void* stream) {
  HFFN_TRY(check_tc(HFFN_F32, d_model, d_ff, n));
  HFFN_TRY(check_dense_f16(dense, true, false));
  HFFN_REQUIRE(x && b_up && work && err, "null pointer argument");
  HFFN_REQUIRE(aligned16(x) && aligned16(work), "x and work must be 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  return tc_up_f16(x, dense, b_up, z, work, err, d_model, d_ff, n, static_cast<cudaStream_t>(stream));
}

int hffn_down_f16x3(const void* work, const hffn_dense_f16x3* dense, const float* b_down, float* y, int32_t* err,
                    int32_t d_model, int32_t d_ff, int64_t n, void* stream) {
  HFFN_TRY(check_tc(HFFN_F32, d_model, d_ff, n));
  HFFN_TRY(check_dense_f16(dense, false, true));
  HFFN_REQUIRE(work && b_down && y && err, "null pointer argument");
  HFFN_REQUIRE(aligned16(work), "work must be 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  return tc_down_f16(work, dense, b_down, y, err, d_model, d_ff, n, static_cast<cudaStream_t>(stream));
}

int64_t hffn_f16x3_packet_bytes(int32_t d_model) {
  if (d_model < 1) return -1;
  return tc_f16_packet_bytes(d_model);
}

int hffn_split_f16x3(const float* x, const hffn_dense_f16x3* dense, void* packets, int32_t d_model, int32_t d_ff,
                     int64_t n, void* stream) {
  HFFN_TRY(check_tc(HFFN_F32, d_model, d_ff, n));
  HFFN_REQUIRE(dense != nullptr && dense->up_bound != nullptr, "null up bound");
  HFFN_REQUIRE(x && packets, "null pointer argument");
  HFFN_REQUIRE(aligned16(x) && aligned16(packets), "x and packets must be 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  return tc_split_f16(x, dense, packets, d_model, n, static_cast<cudaStream_t>(stream));
}

int hffn_forward_f16x3_packets(const hffn_layer* layer, const hffn_dense_f16x3* dense, const void* packets, float* y,
                               float* z, void* work, int32_t* err, int64_t n, void* stream) {
  HFFN_TRY(check_layer(layer));
  HFFN_TRY(check_tc(HFFN_F32, layer->d_model, layer->d_ff, n));
  HFFN_TRY(check_dense_f16(dense, true, true));
  HFFN_REQUIRE(packets && y && work && err, "null pointer argument");
  HFFN_REQUIRE(aligned16(packets) && aligned16(work), "packets and work must be 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  return tc_forward_f16_packets(packets, dense, static_cast<const float*>(layer->b_up),
                                static_cast<const float*>(layer->b_down), y, z, work, err, layer->d_model, layer->d_ff,
                                n, static_cast<cudaStream_t>(stream));
}

int hffn_forward_f16x3(const hffn_layer* layer, const hffn_dense_f16x3* dense, const float* x, float* y, float* z,
                       void* work, int32_t* err, int64_t n, void* stream) {
  HFFN_TRY(check_layer(layer));
  HFFN_TRY(check_tc(HFFN_F32, layer->d_model, layer->d_ff, n));
  HFFN_TRY(check_dense_f16(dense, true, true));
  HFFN_REQUIRE(x && y && work && err, "null pointer argument");
  HFFN_REQUIRE(aligned16(x) && aligned16(work), "x and work must be 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  HFFN_TRY(tc_up_f16(x, dense, static_cast<const float*>(layer->b_up), z, work, err, layer->d_model, layer->d_ff, n,
                     s));
  return tc_down_f16(work, dense, static_cast<const float*>(layer->b_down), y, err, layer->d_model, layer->d_ff, n, s);
}

int hffn_up_tc(int dtype, const void* x, const void* w_hi, const void* w_lo, const void* b_up, void* act_hi,
               void* act_lo, float* z, void* x_split, int32_t* err, int32_t d_model, int32_t d_ff, int64_t n,
               void* stream) {
  HFFN_TRY(check_tc(dtype, d_model, d_ff, n));
  const bool f32 = dtype == HFFN_F32;
  HFFN_REQUIRE(x && w_hi && b_up && act_hi && err && (!f32 || (w_lo && act_lo && x_split)), "null pointer argument");
  HFFN_REQUIRE(z == nullptr || f32, "z is stored by the float32 path only");
  HFFN_REQUIRE(aligned16(x) && aligned16(w_hi) && (!f32 || (aligned16(w_lo) && aligned16(x_split))),
               "tensor-core operands must be 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  return tc_up(dtype, x, w_hi, w_lo, b_up, act_hi, act_lo, z, x_split, err, d_model, d_ff, n,
               static_cast<cudaStream_t>(stream));
}

int hffn_down_tc(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo,
                 const void* b_down, void* y, int32_t* err, int32_t d_model, int32_t d_ff, int64_t n, void* stream) {
  HFFN_TRY(check_tc(dtype, d_model, d_ff, n));
  const bool f32 = dtype == HFFN_F32;
  HFFN_REQUIRE(act_hi && w_hi && b_down && y && err && (!f32 || (act_lo && w_lo)), "null pointer argument");
  HFFN_REQUIRE(aligned16(act_hi) && aligned16(w_hi) && (!f32 || (aligned16(act_lo) && aligned16(w_lo))),
               "tensor-core operands must be 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  return tc_down(dtype, act_hi, act_lo, w_hi, w_lo, b_down, y, err, d_model, d_ff, n,
                 static_cast<cudaStream_t>(stream));
}

int hffn_down_tc_peer(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo,
                      const void* b_down, const uint64_t* peer_y, int32_t world, int64_t tokens_per_owner,
                      int32_t* err, int32_t d_model, int32_t d_ff, int64_t n, void* stream) {
  HFFN_TRY(check_tc(dtype, d_model, d_ff, n));
  const bool f32 = dtype == HFFN_F32;
  HFFN_REQUIRE(act_hi && w_hi && b_down && peer_y && err && (!f32 || (act_lo && w_lo)), "null pointer argument");
  HFFN_REQUIRE(world >= 1 && world <= 8, "world %d outside [1, 8]", world);
  HFFN_REQUIRE(tokens_per_owner >= 1 && n == (int64_t)world * tokens_per_owner, "n must be world x tokens_per_owner");
  void* peers[8] = {};
  for (int p = 0; p < world; ++p) {
    HFFN_REQUIRE(peer_y[p] != 0, "null peer buffer %d", p);
    peers[p] = reinterpret_cast<void*>(peer_y[p]);
  }
  HFFN_TRY(bind_stream_device(stream));
  return tc_down_peer(dtype, act_hi, act_lo, w_hi, w_lo, b_down, peers, world, tokens_per_owner, err, d_model, d_ff,
                      n, static_cast<cudaStream_t>(stream));
}

int hffn_sum_slots(int dtype, const void* slots, int32_t count, int64_t elems, void* out, void* stream) {
  HFFN_REQUIRE(dtype == HFFN_F32 || dtype == HFFN_BF16, "unknown dtype %d", dtype);
  HFFN_REQUIRE(slots && out && count >= 1 && elems >= 0, "bad argument");
  HFFN_TRY(bind_stream_device(stream));
  return tc_sum_slots(dtype, slots, count, elems, out, static_cast<cudaStream_t>(stream));
}

int hffn_set_tc_max_ctas(int32_t max_ctas) {
  HFFN_REQUIRE(max_ctas >= 0, "negative CTA cap");
  tc_set_max_ctas(max_ctas);
  return HFFN_OK;
}

int hffn_set_tc_tile_tokens(int32_t tokens) {
  HFFN_REQUIRE(tokens == 0 || tokens == 64 || tokens == 128 || tokens == 256, "tile tokens %d not in {0, 64, 128, 256}",
               tokens);
  tc_set_tile_tokens(tokens);
  return HFFN_OK;
}

int hffn_gemm_tc_f32(int a_mn, int b_mn, const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                     float* d, int32_t m, int32_t n, int32_t k, int64_t lda, int64_t ldb, int32_t* err, void* stream) {
  HFFN_REQUIRE(a_hi && a_lo && b_hi && b_lo && d && err, "null pointer argument");
  HFFN_REQUIRE(m >= 1 && n >= 1 && k >= 1, "empty GEMM");
  HFFN_REQUIRE(k % 4 == 0 && (!a_mn || (m % 32 == 0 && lda >= m && lda % 4 == 0)) &&
                   (!b_mn || (n % 32 == 0 && ldb >= n && ldb % 4 == 0)),
               "GEMM shape: K a multiple of 4, MN-major extents multiples of 32");
  HFFN_REQUIRE(aligned16(a_hi) && aligned16(a_lo) && aligned16(b_hi) && aligned16(b_lo), "operands 16-byte aligned");
  HFFN_TRY(bind_stream_device(stream));
  return tc_gemm_f32(a_mn, b_mn, a_hi, a_lo, b_hi, b_lo, d, m, n, k, lda, ldb, err, static_cast<cudaStream_t>(stream));
}

int64_t hffn_train_step_tc_workspace(const hffn_layer* layer, int64_t n) {
  if (layer == nullptr || n < 1) return -1;
  return tc_train_workspace(layer, n);
}

int hffn_train_step_tc(const hffn_layer* layer, const hffn_dense* dense, const hffn_dense_f16x3* dense16,
                       const float* x, const float* target, float* y, float* gx, const hffn_train_params* params,
                       const hffn_adamw_step* adamw, float* loss, void* work, int32_t* err, int64_t n, int64_t n_total,
                       void* stream) {
  HFFN_TRY(check_layer(layer));
  HFFN_TRY(check_tc(HFFN_F32, layer->d_model, layer->d_ff, n));
  HFFN_REQUIRE(layer->d_model % 32 == 0 && layer->d_ff % 32 == 0,
               "tensor-core training: d_model and d_ff multiples of 32");
  HFFN_REQUIRE(n_total >= n, "n_total below n");
  HFFN_REQUIRE(dense && dense->up_hi && dense->up_lo && dense->down_hi && dense->down_lo, "null dense operand");
  if (dense16 != nullptr) HFFN_TRY(check_dense_f16(dense16, true, true));
  HFFN_REQUIRE(x && target && y && gx && params && loss && work && err, "null pointer argument");
  HFFN_REQUIRE(aligned16(x) && aligned16(work), "x and the workspace must be 16-byte aligned");
  const bool fused = adamw != nullptr;
  HFFN_TRY(check_param(params->up_val, layer->nnz_up, !fused, fused, "up_val"));
  HFFN_TRY(check_param(params->b_up, layer->d_ff, !fused, fused, "b_up"));
  HFFN_TRY(check_param(params->out_val, layer->nnz_down, !fused, fused, "out_val"));
  HFFN_TRY(check_param(params->b_down, layer->d_model, !fused, fused, "b_down"));
  HFFN_REQUIRE(params->up_val.value == layer->up_val && params->out_val.value == layer->out_val &&
                   params->b_up.value == layer->b_up && params->b_down.value == layer->b_down,
               "the parameter values must be the layer's arrays");
  HFFN_TRY(bind_stream_device(stream));
  return tc_train_step(layer, dense->up_hi, dense->up_lo, dense->down_hi, dense->down_lo, dense16, x, target, y, gx,
                       params, adamw, loss, work, err, n, n_total, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
