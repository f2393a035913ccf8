// The neuron-sharded forward over a stream of batches, exchanged through NVLink peer memory: the native issue loop of
// the pipeline (copy-engine gathers and deliveries, the shard's tensor-core GEMMs, the slot sums) and the
// signal-pad barrier between its iterations.
//
// Each rank holds a neuron shard. Batch k of every rank is staged into that rank's gather buffer, pulled by copy
// engines into every other rank's gather buffer (position j of a gathered batch: the tokens of rank (rank + j) %
// world), run through the shard (one up + down call over world x n tokens), and its partial outputs are delivered
// into the owners' receive slots (copy engines from a local buffer, or the down GEMM's epilogue storing into the peer
// slots); each owner sums its slots in rank order. Iteration k stages batch k, waits for the pulls of batch k - 1 and
// the deliveries of batch k - 3, passes the barrier, starts the pulls of batch k, runs batch k - 1, starts its
// deliveries and sums batch k - 3: gathers and deliveries run on the copy engines while the GEMMs run on the SMs.
// Gather and partial buffers are double-buffered, slots triple-buffered; the barrier orders every reuse (a buffer is
// rewritten only after every rank passed the barrier that follows its last reader).
//
// The barrier: every rank writes the barrier's epoch into its slot of every peer's signal pad (system-scope release
// store) and waits until every peer's slot of its own pad holds at least the epoch (polled with back-off, then an
// acquire fence), for at most timeout_ns, after which it records kErrBarrierTimeout and returns: a dead or late peer
// ends the wait with an error status, never a hang. Only ranks on distinct GPUs wait on one another.
#include <cuda_runtime.h>

#include "common.cuh"

namespace hffn {

int tc_up(int dtype, const void* x, const void* w_hi, const void* w_lo, const void* b, void* act_hi, void* act_lo,
          float* z, void* x_split, int* err, int d, int H, int64_t n, cudaStream_t s);
int tc_down(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo, const void* b,
            void* y, int* err, int d, int H, int64_t n, cudaStream_t s, bool pdl = false);
int tc_down_peer(int dtype, const void* act_hi, const void* act_lo, const void* w_hi, const void* w_lo, const void* b,
                 void* const* peers, int world, int64_t tokens_per_owner, int* err, int d, int H, int64_t n,
                 cudaStream_t s);
int tc_sum_slots(int dtype, const void* slots, int count, int64_t elems, void* out, cudaStream_t s);

namespace {

constexpr int kErrBarrierTimeout = 201;
constexpr int kMaxWorld = 8;
constexpr int64_t kBarrierTimeoutNs = 2000000000ll;

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PeerSignals {
  uint32_t* own;                  // this rank's pad [world]: slot p written by rank p
  uint32_t* peer[kMaxWorld];      // rank p's pad (absolute rank order)
};

// One warp: lane p signals rank p and waits for rank p's signal (lanes >= world and the own lane idle).
__global__ void barrier_kernel(PeerSignals sig, int world, int rank, uint32_t epoch, int64_t timeout_ns, int* err) {
  const int p = threadIdx.x;
  if (p >= world || p == rank) return;
  __threadfence_system();                      // this rank's earlier writes before the signal
  store_release_sys(sig.peer[p] + rank, epoch);
  // poll with relaxed loads and a short back-off (no stream of system-scope fences), then one acquire fence
  const uint64_t start = now_ns();
  while ((int32_t)(load_relaxed_sys(sig.own + p) - epoch) < 0) {
    if ((int64_t)(now_ns() - start) > timeout_ns) {
      atomicCAS(err, 0, kErrBarrierTimeout);
      return;
    }
    __nanosleep(256);
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

}  // namespace

struct PeerPipeline {
  hffn_peer_config cfg;
  hffn_layer layer;
  hffn_dense dense;
  int* err;
  int device;
  int64_t elem;
  uint32_t epoch = 0;
  bool failed = false;     // a run stopped part-way: the ranks' barrier epochs may differ, the pipeline is unusable
  cudaStream_t pull[kMaxWorld] = {}, push[kMaxWorld] = {};
  cudaEvent_t pulled[2][kMaxWorld] = {}, delivered[3][kMaxWorld] = {};
  cudaEvent_t barrier_done = nullptr, computed = nullptr;

  ~PeerPipeline() {
    for (int j = 0; j < kMaxWorld; ++j) {
      if (pull[j]) cudaStreamDestroy(pull[j]);
      if (push[j]) cudaStreamDestroy(push[j]);
      for (int b = 0; b < 2; ++b)
        if (pulled[b][j]) cudaEventDestroy(pulled[b][j]);
      for (int b = 0; b < 3; ++b)
        if (delivered[b][j]) cudaEventDestroy(delivered[b][j]);
    }
    if (barrier_done) cudaEventDestroy(barrier_done);
    if (computed) cudaEventDestroy(computed);
  }

  int barrier(cudaStream_t s, int64_t timeout_ns) {
    PeerSignals sig{};
    sig.own = cfg.signal;
    for (int j = 0; j < cfg.world; ++j)
      sig.peer[(cfg.rank + j) % cfg.world] = reinterpret_cast<uint32_t*>(cfg.signal_peer[j]);
    barrier_kernel<<<1, 32, 0, s>>>(sig, cfg.world, cfg.rank, ++epoch, timeout_ns, err);
    return launch_status("peer barrier");
  }

  // up + down of the shard over the gathered batch in gather[b]; partial outputs into partial[b] (copy delivery) or
  // straight into the owners' slots of `slot` (store delivery)
  int shard(int b, int slot, cudaStream_t s) {
    const int64_t m = (int64_t)cfg.world * cfg.tokens;
    const int d = layer.d_model, H = layer.d_ff;
    char* work = static_cast<char*>(cfg.work);
    void *x_split = nullptr, *act_hi = work, *act_lo = nullptr;
    if (cfg.dtype == HFFN_F32) {
      x_split = work;
      act_hi = work + 2 * m * d * 4;
      act_lo = static_cast<char*>(act_hi) + m * H * 4;
    }
    HFFN_TRY(tc_up(cfg.dtype, cfg.gather[b], dense.up_hi, dense.up_lo, layer.b_up, act_hi, act_lo, nullptr, x_split,
                   err, d, H, m, s));
    if (cfg.partial[0] != nullptr)
      return tc_down(cfg.dtype, act_hi, act_lo, dense.down_hi, dense.down_lo, layer.b_down, cfg.partial[b], err, d, H,
                     m, s);
    void* targets[kMaxWorld] = {};
    for (int j = 0; j < cfg.world; ++j) targets[j] = reinterpret_cast<void*>(cfg.slot_peer[slot][j]);
    return tc_down_peer(cfg.dtype, act_hi, act_lo, dense.down_hi, dense.down_lo, layer.b_down, targets, cfg.world,
                        cfg.tokens, err, d, H, m, s);
  }

  int run(const void* const* xs, void* const* outs, int count, cudaStream_t s) {
    const int w = cfg.world;
    const int64_t n = cfg.tokens, d = layer.d_model, batch = n * d * elem;
    const bool copy_delivery = cfg.partial[0] != nullptr;
    auto check = [](cudaError_t e, const char* what) {
      if (e == cudaSuccess) return HFFN_OK;
      set_error("peer pipeline %s: %s", what, cudaGetErrorString(e));
      return HFFN_ERR_CUDA;
    };
    for (int k = 0; k < count + 3; ++k) {
      const int g = k % 2;
      if (k < count)
        HFFN_TRY(check(cudaMemcpyAsync(cfg.gather[g], xs[k], batch, cudaMemcpyDeviceToDevice, s), "stage"));
      if (k >= 1 && k <= count)
        for (int j = 1; j < w; ++j) HFFN_TRY(check(cudaStreamWaitEvent(s, pulled[(k - 1) % 2][j], 0), "wait pulls"));
      if (k >= 3)
        for (int j = 0; j < w; ++j)
          HFFN_TRY(check(cudaStreamWaitEvent(s, delivered[(k - 3) % 3][j], 0), "wait deliveries"));
      HFFN_TRY(barrier(s, kBarrierTimeoutNs));
      HFFN_TRY(check(cudaEventRecord(barrier_done, s), "record"));
      if (k < count)
        for (int j = 1; j < w; ++j) {
          HFFN_TRY(check(cudaStreamWaitEvent(pull[j], barrier_done, 0), "pull wait"));
          HFFN_TRY(check(cudaMemcpyAsync(static_cast<char*>(cfg.gather[g]) + j * batch,
                                         reinterpret_cast<const void*>(cfg.gather_peer[g][j]), batch,
                                         cudaMemcpyDeviceToDevice, pull[j]),
                         "pull"));
          HFFN_TRY(check(cudaEventRecord(pulled[g][j], pull[j]), "record pull"));
        }
      if (k >= 1 && k <= count) {
        const int b = (k - 1) % 2, slot = (k - 1) % 3;
        HFFN_TRY(shard(b, slot, s));
        if (!copy_delivery) {
          for (int j = 0; j < w; ++j) HFFN_TRY(check(cudaEventRecord(delivered[slot][j], s), "record delivery"));
        } else {
          HFFN_TRY(check(cudaEventRecord(computed, s), "record compute"));
          for (int j = 0; j < w; ++j) {
            HFFN_TRY(check(cudaStreamWaitEvent(push[j], computed, 0), "push wait"));
            HFFN_TRY(check(cudaMemcpyAsync(reinterpret_cast<void*>(cfg.slot_peer[slot][j]),
                                           static_cast<const char*>(cfg.partial[b]) + j * batch, batch,
                                           cudaMemcpyDeviceToDevice, push[j]),
                           "deliver"));
            HFFN_TRY(check(cudaEventRecord(delivered[slot][j], push[j]), "record delivery"));
          }
        }
      }
      if (k >= 3) HFFN_TRY(tc_sum_slots(cfg.dtype, cfg.slots[(k - 3) % 3], w, n * d, outs[k - 3], s));
    }
    return HFFN_OK;
  }
};

static int create_pipeline(const hffn_peer_config* cfg, const hffn_layer* layer, const hffn_dense* dense, int* err,
                           PeerPipeline** out) {
  PeerPipeline* p = new PeerPipeline();
  p->cfg = *cfg;
  p->layer = *layer;
  p->dense = *dense;
  p->err = err;
  p->elem = cfg->dtype == HFFN_BF16 ? 2 : 4;
  cudaGetDevice(&p->device);
  bool ok = true;
  for (int j = 0; j < cfg->world && ok; ++j) {
    ok = cudaStreamCreateWithFlags(&p->pull[j], cudaStreamNonBlocking) == cudaSuccess &&
         cudaStreamCreateWithFlags(&p->push[j], cudaStreamNonBlocking) == cudaSuccess;
    for (int b = 0; b < 2 && ok; ++b)
      ok = cudaEventCreateWithFlags(&p->pulled[b][j], cudaEventDisableTiming) == cudaSuccess;
    for (int b = 0; b < 3 && ok; ++b)
      ok = cudaEventCreateWithFlags(&p->delivered[b][j], cudaEventDisableTiming) == cudaSuccess;
  }
  ok = ok && cudaEventCreateWithFlags(&p->barrier_done, cudaEventDisableTiming) == cudaSuccess &&
       cudaEventCreateWithFlags(&p->computed, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    delete p;
    set_error("peer pipeline: stream or event creation failed");
    return HFFN_ERR_CUDA;
  }
  *out = p;
  return HFFN_OK;
}

int peer_barrier_once(uint32_t* own, const uint64_t* peers, int world, int rank, uint32_t epoch, int64_t timeout_ns,
                      int* err, cudaStream_t s) {
  PeerSignals sig{};
  sig.own = own;
  for (int p = 0; p < world; ++p) sig.peer[p] = reinterpret_cast<uint32_t*>(peers[p]);
  barrier_kernel<<<1, 32, 0, s>>>(sig, world, rank, epoch, timeout_ns, err);
  return launch_status("peer barrier");
}

}  // namespace hffn

using namespace hffn;

extern "C" {

int hffn_peer_pipeline_create(const hffn_peer_config* cfg, const hffn_layer* layer, const hffn_dense* dense,
                              int32_t* err, void** handle) {
  HFFN_REQUIRE(cfg && layer && dense && err && handle, "null argument");
  HFFN_REQUIRE(cfg->world >= 1 && cfg->world <= kMaxWorld && cfg->rank >= 0 && cfg->rank < cfg->world,
               "world %d / rank %d", cfg->world, cfg->rank);
  HFFN_REQUIRE(cfg->dtype == HFFN_F32 || cfg->dtype == HFFN_BF16, "unknown dtype %d", cfg->dtype);
  HFFN_REQUIRE(cfg->tokens >= 1 && (int64_t)cfg->world * cfg->tokens < (1ll << 31), "tokens %lld",
               (long long)cfg->tokens);
  HFFN_REQUIRE(layer->d_model % 8 == 0 && layer->d_ff % 8 == 0, "tensor-core shapes: d_model and d_ff multiples of 8");
  HFFN_REQUIRE(dense->up_hi && dense->down_hi && (cfg->dtype == HFFN_BF16 || (dense->up_lo && dense->down_lo)),
               "dense operands missing");
  HFFN_REQUIRE(cfg->work && cfg->signal, "workspace or signal pad missing");
  for (int b = 0; b < 2; ++b) HFFN_REQUIRE(cfg->gather[b] != nullptr, "gather buffer %d missing", b);
  for (int b = 0; b < 3; ++b) HFFN_REQUIRE(cfg->slots[b] != nullptr, "slot buffer %d missing", b);
  HFFN_REQUIRE((cfg->partial[0] == nullptr) == (cfg->partial[1] == nullptr), "partial buffers: both or none");
  for (int j = 0; j < cfg->world; ++j) {
    HFFN_REQUIRE(cfg->signal_peer[j] != 0, "signal pad of position %d missing", j);
    for (int b = 0; b < 2; ++b) HFFN_REQUIRE(cfg->gather_peer[b][j] != 0, "gather buffer %d of position %d", b, j);
    for (int b = 0; b < 3; ++b) HFFN_REQUIRE(cfg->slot_peer[b][j] != 0, "slot %d of position %d", b, j);
  }
  PeerPipeline* p = nullptr;
  HFFN_TRY(create_pipeline(cfg, layer, dense, err, &p));
  *handle = p;
  return HFFN_OK;
}

int hffn_peer_pipeline_run(void* handle, const void* const* xs, void* const* outs, int32_t count, void* stream) {
  HFFN_REQUIRE(handle != nullptr, "null pipeline");
  HFFN_REQUIRE(count >= 0 && (count == 0 || (xs && outs)), "batches");
  for (int k = 0; k < count; ++k) HFFN_REQUIRE(xs[k] && outs[k], "batch %d: null pointer", k);
  PeerPipeline* p = static_cast<PeerPipeline*>(handle);
  if (p->failed) {
    set_error("peer pipeline: an earlier run failed part-way (the ranks' barriers are out of step); recreate it");
    return HFFN_ERR_CUDA;
  }
  HFFN_TRY(bind_stream_device(stream));
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device != p->device) {
    set_error("peer pipeline: created on device %d, run on a stream of device %d", p->device, device);
    return HFFN_ERR_ARGUMENT;
  }
  const int status = p->run(xs, outs, count, static_cast<cudaStream_t>(stream));
  if (status != HFFN_OK) p->failed = true;
  return status;
}

int hffn_peer_pipeline_destroy(void* handle) {
  delete static_cast<PeerPipeline*>(handle);
  return HFFN_OK;
}

int hffn_peer_barrier(uint32_t* signal, const uint64_t* signal_peer, int32_t world, int32_t rank, uint32_t epoch,
                      int64_t timeout_ns, int32_t* err, void* stream) {
  HFFN_REQUIRE(signal && signal_peer && err, "null argument");
  HFFN_REQUIRE(world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world, "world %d / rank %d", world, rank);
  HFFN_REQUIRE(timeout_ns > 0 && timeout_ns <= 60ll * 1000000000ll, "timeout %lld ns outside (0, 60 s]",
               (long long)timeout_ns);
  for (int p = 0; p < world; ++p) HFFN_REQUIRE(p == rank || signal_peer[p] != 0, "signal pad of rank %d missing", p);
  HFFN_TRY(bind_stream_device(stream));
  return peer_barrier_once(signal, signal_peer, world, rank, epoch, timeout_ns, err, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
