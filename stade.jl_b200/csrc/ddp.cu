// Data-parallel epilogue over NCCL (NVLink / NVSwitch inside one box).
//
// Replaces the MPI functions `ddpgen_` emits (src/STADE.jl:17595-17696):
//   reset_accum! / reset_reduced! / reset_local!  -> stade_ddp_zero
//   allreduce_accum!(bufs..., n_local, comm)      -> stade_ddp_allreduce_sum
//   allreduce_reduced!(bufs..., comm)             -> stade_ddp_allreduce_sum
//   check_replicas(bufs..., comm)                 -> stade_ddp_check_replicas
// The generated code issues one blocking MPI.Allreduce! per buffer
// (src/STADE.jl:17629-17645). Here all buffers of a call travel as ONE
// contiguous bucket in one NCCL group together with the sample count: in
// place when the caller's buffers are already laid out back to back,
// otherwise packed into a persistent per-communicator bucket by one gather
// kernel and scattered back by another.
//
// Failure handling: the communicator is created non-blocking; every wait on
// NCCL or on the stream polls with a deadline and aborts the communicator
// when it runs out (STADE_ETIMEDOUT), so a rank that never joins ends the
// call with an error instead of a hang.
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"
#include "halo.cuh"

struct stade_comm {
  ncclComm_t nccl = nullptr;
  int rank = 0, size = 1, device = 0;
  int timeout_ms = 60000;
  void* bucket = nullptr;
  size_t bucket_bytes = 0;
  double* sums = nullptr;     // device, 2 * kMaxBufs checksums (+ min/max results)
  int64_t* count = nullptr;   // device, the sample count
  double* host_sums = nullptr;  // pinned
  int64_t* host_count = nullptr;
  bool broken = false;
  // halo exchanges run on a side stream so the owner's interior work overlaps
  cudaStream_t side = nullptr;
  cudaEvent_t ev_ready = nullptr, ev_halo = nullptr;
};

namespace stade {
namespace {

constexpr int kMaxBufs = 32;

stade_status nccl_fail(ncclResult_t r, const char* what) {
  return fail(STADE_ENCCL, "%s failed: %s", what, ncclGetErrorString(r));
}

using Clock = std::chrono::steady_clock;

// Poll pacing: the first polls spin (issuing usually completes within a few
// microseconds and a sleep would hold the host thread, and with it the
// launches queued behind the call, for the sleep's whole length), later ones
// sleep.
inline void poll_pause(int& polls) {
  if (++polls > 2000) std::this_thread::sleep_for(std::chrono::microseconds(20));
}

// Waits until the non-blocking communicator has finished issuing the last
// call (ncclInProgress -> ncclSuccess), bounded by the deadline.
stade_status wait_issue(stade_comm* c, Clock::time_point deadline, const char* what) {
  int polls = 0;
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = ncclCommGetAsyncError(c->nccl, &st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommGetAsyncError");
    if (st == ncclSuccess) return STADE_OK;
    if (st != ncclInProgress) {
      c->broken = true;
      ncclCommAbort(c->nccl);
      c->nccl = nullptr;
      return nccl_fail(st, what);
    }
    if (Clock::now() > deadline) {
      c->broken = true;
      ncclCommAbort(c->nccl);
      c->nccl = nullptr;
      return fail(STADE_ETIMEDOUT, "%s: peers did not respond within the timeout", what);
    }
    poll_pause(polls);
  }
}

// Waits for the stream to drain while watching the communicator for errors.
stade_status wait_stream(stade_comm* c, cudaStream_t s, Clock::time_point deadline,
                         const char* what) {
  int polls = 0;
  for (;;) {
    cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return STADE_OK;
    if (q != cudaErrorNotReady) return cuda_fail(q, what, __FILE__, __LINE__);
    ncclResult_t st = ncclSuccess;
    ncclCommGetAsyncError(c->nccl, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      c->broken = true;
      ncclCommAbort(c->nccl);
      c->nccl = nullptr;
      return nccl_fail(st, what);
    }
    if (Clock::now() > deadline) {
      c->broken = true;
      ncclCommAbort(c->nccl);
      c->nccl = nullptr;
      return fail(STADE_ETIMEDOUT, "%s: collective did not complete within the timeout", what);
    }
    poll_pause(polls);
  }
}

struct Segs {
  void* ptr[kMaxBufs];
  int64_t off[kMaxBufs + 1];
  int n;
};

// Gathers (pack = 1) or scatters (pack = 0) buffers to / from the bucket.
template <class T>
__global__ void bucket_copy_kernel(Segs sg, T* __restrict__ bucket, int pack) {
  const int64_t total = sg.off[sg.n];
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int i = 0;
    while (e >= sg.off[i + 1]) ++i;
    T* p = static_cast<T*>(sg.ptr[i]) + (e - sg.off[i]);
    if (pack) bucket[e] = *p;
    else *p = bucket[e];
  }
}

// Per buffer: sum and sum of abs in Float64, one block per buffer, fixed order.
template <class T>
__global__ void checksum_kernel(Segs sg, double* __restrict__ out) {
  __shared__ double red[32];
  const int i = blockIdx.x;
  const T* p = static_cast<const T*>(sg.ptr[i]);
  const int64_t n = sg.off[i + 1] - sg.off[i];
  double s1 = 0.0, s2 = 0.0;
  for (int64_t e = threadIdx.x; e < n; e += blockDim.x) {
    const double v = (double)p[e];
    s1 += v;
    s2 += fabs(v);
  }
  s1 = block_sum(s1, red);
  s2 = block_sum(s2, red);
  if (threadIdx.x == 0) {
    out[2 * i] = s1;
    out[2 * i + 1] = s2;
  }
}

stade_status build_segs(void* const* bufs, const int64_t* counts, int nbuf, Segs* sg,
                        bool* contiguous, size_t es) {
  STADE_REQUIRE(nbuf >= 0 && nbuf <= kMaxBufs, "ddp: %d buffers (at most %d)", nbuf, kMaxBufs);
  STADE_REQUIRE(nbuf == 0 || (bufs && counts), "ddp: null buffer list");
  sg->n = nbuf;
  sg->off[0] = 0;
  *contiguous = true;
  for (int i = 0; i < nbuf; ++i) {
    STADE_REQUIRE(counts[i] >= 0, "ddp: negative count for buffer %d", i);
    STADE_REQUIRE(counts[i] == 0 || bufs[i], "ddp: null buffer %d", i);
    sg->ptr[i] = bufs[i];
    sg->off[i + 1] = sg->off[i] + counts[i];
    if (i > 0 && static_cast<char*>(bufs[i - 1]) + counts[i - 1] * es != static_cast<char*>(bufs[i]))
      *contiguous = false;
  }
  return STADE_OK;
}

stade_status ensure_bucket(stade_comm* c, size_t bytes) {
  if (c->bucket_bytes >= bytes) return STADE_OK;
  if (c->bucket) STADE_CUDA(cudaFree(c->bucket));
  c->bucket = nullptr;
  STADE_CUDA(cudaMalloc(&c->bucket, bytes));
  c->bucket_bytes = bytes;
  return STADE_OK;
}

}  // namespace

stade_status halo_begin(stade_comm* c, const double* first_row, const double* last_row,
                        double* top_halo, double* bottom_halo, int64_t count, cudaStream_t s) {
  if (c == nullptr || c->size == 1) {
    // one slab holds the whole periodic grid: its halos are its own edge rows
    STADE_CUDA(cudaMemcpyAsync(top_halo, last_row, count * sizeof(double),
                               cudaMemcpyDeviceToDevice, s));
    STADE_CUDA(cudaMemcpyAsync(bottom_halo, first_row, count * sizeof(double),
                               cudaMemcpyDeviceToDevice, s));
    return STADE_OK;
  }
  STADE_REQUIRE(c->nccl, "halo exchange: communicator is aborted");
  if (!c->side) {
    STADE_CUDA(cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking));
    STADE_CUDA(cudaEventCreateWithFlags(&c->ev_ready, cudaEventDisableTiming));
    STADE_CUDA(cudaEventCreateWithFlags(&c->ev_halo, cudaEventDisableTiming));
  }
  STADE_CUDA(cudaEventRecord(c->ev_ready, s));
  STADE_CUDA(cudaStreamWaitEvent(c->side, c->ev_ready, 0));
  const int prev = (c->rank + c->size - 1) % c->size;
  const int next = (c->rank + 1) % c->size;
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  // With two ranks both neighbours are the same peer and NCCL pairs the
  // sends and receives between two ranks in issue order: the last row goes
  // out first and the top halo is received first, so each receive meets the
  // row it stands for.
  ncclResult_t r = ncclGroupStart();
  if (r == ncclSuccess) r = ncclSend(last_row, (size_t)count, ncclFloat64, next, c->nccl, c->side);
  if (r == ncclSuccess || r == ncclInProgress)
    r = ncclSend(first_row, (size_t)count, ncclFloat64, prev, c->nccl, c->side);
  if (r == ncclSuccess || r == ncclInProgress)
    r = ncclRecv(top_halo, (size_t)count, ncclFloat64, prev, c->nccl, c->side);
  if (r == ncclSuccess || r == ncclInProgress)
    r = ncclRecv(bottom_halo, (size_t)count, ncclFloat64, next, c->nccl, c->side);
  ncclResult_t r2 = ncclGroupEnd();
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclSend/ncclRecv (halo)");
  if (r2 != ncclSuccess && r2 != ncclInProgress) return nccl_fail(r2, "ncclGroupEnd (halo)");
  stade_status st = wait_issue(c, deadline, "halo exchange");
  if (st != STADE_OK) return st;
  STADE_CUDA(cudaEventRecord(c->ev_halo, c->side));
  return STADE_OK;
}

stade_status halo_end(stade_comm* c, cudaStream_t s) {
  if (c == nullptr || c->size == 1) return STADE_OK;
  STADE_CUDA(cudaStreamWaitEvent(s, c->ev_halo, 0));
  return STADE_OK;
}

stade_status comm_allreduce_f64(stade_comm* c, double* buf, int64_t count, cudaStream_t s) {
  if (c == nullptr || c->size == 1) return STADE_OK;
  STADE_REQUIRE(c->nccl, "allreduce: communicator is aborted");
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  ncclResult_t r = ncclAllReduce(buf, buf, (size_t)count, ncclFloat64, ncclSum, c->nccl, s);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclAllReduce");
  return wait_issue(c, deadline, "ncclAllReduce");
}

stade_status comm_wait_stream(stade_comm* c, cudaStream_t s) {
  if (c == nullptr || c->size == 1) {
    STADE_CUDA(cudaStreamSynchronize(s));
    return STADE_OK;
  }
  STADE_REQUIRE(c->nccl, "wait: communicator is aborted");
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  return wait_stream(c, s, deadline, "stream wait");
}

int comm_size(const stade_comm* c) { return c ? c->size : 1; }

}  // namespace stade

using namespace stade;

extern "C" {

stade_status stade_comm_unique_id(unsigned char id_out[128]) {
  STADE_REQUIRE(id_out, "stade_comm_unique_id: null output");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id_out, &id, 128);
  return STADE_OK;
}

stade_status stade_comm_init(const unsigned char id[128], int nranks, int rank, int timeout_ms,
                             stade_comm** comm_out) {
  STADE_REQUIRE(id && comm_out, "stade_comm_init: null argument");
  STADE_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "stade_comm_init: bad rank %d of %d",
                rank, nranks);
  *comm_out = nullptr;
  auto* c = new stade_comm();
  c->rank = rank;
  c->size = nranks;
  c->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  cudaError_t ce = cudaGetDevice(&c->device);
  if (ce != cudaSuccess) { delete c; return cuda_fail(ce, "cudaGetDevice", __FILE__, __LINE__); }
  ncclUniqueId uid;
  std::memcpy(&uid, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&c->nccl, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  stade_status st = wait_issue(c, deadline, "ncclCommInitRankConfig");
  if (st != STADE_OK) { delete c; return st; }
  ce = cudaMalloc(&c->sums, sizeof(double) * 6 * kMaxBufs);
  if (ce == cudaSuccess) ce = cudaMalloc(&c->count, sizeof(int64_t) * 2);
  if (ce == cudaSuccess) ce = cudaMallocHost(&c->host_sums, sizeof(double) * 6 * kMaxBufs);
  if (ce == cudaSuccess) ce = cudaMallocHost(&c->host_count, sizeof(int64_t) * 2);
  if (ce != cudaSuccess) {
    stade_comm_destroy(c);
    return cuda_fail(ce, "cudaMalloc (communicator state)", __FILE__, __LINE__);
  }
  *comm_out = c;
  return STADE_OK;
}

stade_status stade_comm_destroy(stade_comm* c) {
  if (!c) return STADE_OK;
  if (c->nccl) {
    if (c->broken) ncclCommAbort(c->nccl);
    else ncclCommDestroy(c->nccl);
  }
  if (c->side) {
    cudaStreamSynchronize(c->side);
    cudaStreamDestroy(c->side);
  }
  if (c->ev_ready) cudaEventDestroy(c->ev_ready);
  if (c->ev_halo) cudaEventDestroy(c->ev_halo);
  if (c->bucket) cudaFree(c->bucket);
  if (c->sums) cudaFree(c->sums);
  if (c->count) cudaFree(c->count);
  if (c->host_sums) cudaFreeHost(c->host_sums);
  if (c->host_count) cudaFreeHost(c->host_count);
  delete c;
  return STADE_OK;
}

int stade_comm_rank(const stade_comm* c) { return c ? c->rank : -1; }
int stade_comm_size(const stade_comm* c) { return c ? c->size : 0; }

stade_status stade_ddp_allreduce_sum(stade_comm* c, void* const* bufs, const int64_t* counts,
                                     int nbuf, int dtype, int64_t n_local, int64_t* n_global,
                                     const stade_opts* opts) {
  STADE_REQUIRE(c && c->nccl, "ddp_allreduce_sum: communicator is null or aborted");
  STADE_REQUIRE(dtype == STADE_F32 || dtype == STADE_F64, "ddp_allreduce_sum: bad dtype");
  const size_t es = dtype == STADE_F32 ? 4 : 8;
  Segs sg;
  bool contiguous = false;
  stade_status st = build_segs(bufs, counts, nbuf, &sg, &contiguous, es);
  if (st != STADE_OK) return st;
  cudaStream_t s = stream_of(opts);
  PhaseScope ph("allreduce", s);
  const int64_t total = sg.off[nbuf];
  void* data = nbuf > 0 ? bufs[0] : nullptr;
  if (total > 0 && !contiguous) {
    st = ensure_bucket(c, (size_t)total * es);
    if (st != STADE_OK) return st;
    data = c->bucket;
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 1184);
    if (dtype == STADE_F32) bucket_copy_kernel<float><<<blocks, 256, 0, s>>>(sg, (float*)data, 1);
    else bucket_copy_kernel<double><<<blocks, 256, 0, s>>>(sg, (double*)data, 1);
    STADE_CHECK_LAUNCH();
  }
  if (n_global) {
    c->host_count[0] = n_local;
    STADE_CUDA(cudaMemcpyAsync(c->count, c->host_count, sizeof(int64_t), cudaMemcpyHostToDevice, s));
  }
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  ncclResult_t r = ncclGroupStart();
  if (r != ncclSuccess) return nccl_fail(r, "ncclGroupStart");
  if (total > 0)
    r = ncclAllReduce(data, data, (size_t)total, dtype == STADE_F32 ? ncclFloat32 : ncclFloat64,
                      ncclSum, c->nccl, s);
  if ((r == ncclSuccess || r == ncclInProgress) && n_global)
    r = ncclAllReduce(c->count, c->count, 1, ncclInt64, ncclSum, c->nccl, s);
  ncclResult_t r2 = ncclGroupEnd();
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclAllReduce");
  if (r2 != ncclSuccess && r2 != ncclInProgress) return nccl_fail(r2, "ncclGroupEnd");
  st = wait_issue(c, deadline, "ncclAllReduce");
  if (st != STADE_OK) return st;
  if (total > 0 && !contiguous) {
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 1184);
    if (dtype == STADE_F32) bucket_copy_kernel<float><<<blocks, 256, 0, s>>>(sg, (float*)data, 0);
    else bucket_copy_kernel<double><<<blocks, 256, 0, s>>>(sg, (double*)data, 0);
    STADE_CHECK_LAUNCH();
  }
  if (n_global) {
    STADE_CUDA(cudaMemcpyAsync(c->host_count, c->count, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    st = wait_stream(c, s, deadline, "ddp_allreduce_sum");
    if (st != STADE_OK) return st;
    *n_global = c->host_count[0];
  }
  return STADE_OK;
}

stade_status stade_ddp_check_replicas(stade_comm* c, const void* const* bufs, const int64_t* counts,
                                      int nbuf, int dtype, uint64_t* bad_mask,
                                      const stade_opts* opts) {
  STADE_REQUIRE(c && c->nccl, "ddp_check_replicas: communicator is null or aborted");
  STADE_REQUIRE(dtype == STADE_F32 || dtype == STADE_F64, "ddp_check_replicas: bad dtype");
  Segs sg;
  bool contiguous = false;
  stade_status st = build_segs(const_cast<void* const*>(bufs), counts, nbuf, &sg, &contiguous,
                               dtype == STADE_F32 ? 4 : 8);
  if (st != STADE_OK) return st;
  if (bad_mask) *bad_mask = 0;
  if (nbuf == 0) return STADE_OK;
  cudaStream_t s = stream_of(opts);
  double* sums = c->sums;              // [2 nbuf] local
  double* mins = sums + 2 * kMaxBufs;  // [2 nbuf]
  double* maxs = sums + 4 * kMaxBufs;  // [2 nbuf]
  if (dtype == STADE_F32) checksum_kernel<float><<<nbuf, 256, 0, s>>>(sg, sums);
  else checksum_kernel<double><<<nbuf, 256, 0, s>>>(sg, sums);
  STADE_CHECK_LAUNCH();
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  ncclResult_t r = ncclGroupStart();
  if (r == ncclSuccess) r = ncclAllReduce(sums, mins, 2 * nbuf, ncclFloat64, ncclMin, c->nccl, s);
  if (r == ncclSuccess || r == ncclInProgress)
    r = ncclAllReduce(sums, maxs, 2 * nbuf, ncclFloat64, ncclMax, c->nccl, s);
  ncclResult_t r2 = ncclGroupEnd();
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclAllReduce(min/max)");
  if (r2 != ncclSuccess && r2 != ncclInProgress) return nccl_fail(r2, "ncclGroupEnd");
  st = wait_issue(c, deadline, "check_replicas");
  if (st != STADE_OK) return st;
  STADE_CUDA(cudaMemcpyAsync(c->host_sums, mins, sizeof(double) * 4 * kMaxBufs,
                             cudaMemcpyDeviceToHost, s));
  st = wait_stream(c, s, deadline, "check_replicas");
  if (st != STADE_OK) return st;
  uint64_t mask = 0;
  const double* hmin = c->host_sums;
  const double* hmax = c->host_sums + 2 * kMaxBufs;
  for (int i = 0; i < nbuf; ++i) {
    const bool agree = hmin[2 * i] == hmax[2 * i] && hmin[2 * i + 1] == hmax[2 * i + 1];
    if (!agree) mask |= (uint64_t(1) << i);
  }
  if (bad_mask) *bad_mask = mask;
  if (mask) return fail(STADE_EREPLICA, "check_replicas: buffers differ across ranks (mask 0x%llx)",
                        (unsigned long long)mask);
  return STADE_OK;
}

// ---- generated epilogue names of mlp2_ce (adjoint mode) -------------------
stade_status stade_mlp2_ce_b_reset_accum_f32(float* w1b, float* b1b, float* w2b, float* b2b,
                                             int64_t n_i, int64_t n_h, int64_t n_o,
                                             const stade_opts* opts) {
  void* bufs[4] = {w1b, b1b, w2b, b2b};
  const int64_t counts[4] = {n_i * n_h, n_h, n_h * n_o, n_o};
  return stade_ddp_zero(bufs, counts, 4, STADE_F32, opts);
}
stade_status stade_mlp2_ce_b_reset_reduced_f32(float* loss, const stade_opts* opts) {
  void* bufs[1] = {loss};
  const int64_t counts[1] = {1};
  return stade_ddp_zero(bufs, counts, 1, STADE_F32, opts);
}
stade_status stade_mlp2_ce_b_reset_local_f32(float* xb, float* yb, float* hb, float* zb, float* pb,
                                             int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o,
                                             const stade_opts* opts) {
  void* bufs[5] = {xb, yb, hb, zb, pb};
  const int64_t counts[5] = {n_s * n_i, n_s * n_o, n_s * n_h, n_s * n_o, n_s * n_o};
  return stade_ddp_zero(bufs, counts, 5, STADE_F32, opts);
}
stade_status stade_mlp2_ce_b_allreduce_accum_f32(float* w1b, float* b1b, float* w2b, float* b2b,
                                                 int64_t n_i, int64_t n_h, int64_t n_o,
                                                 int64_t n_local, stade_comm* comm,
                                                 int64_t* n_global, const stade_opts* opts) {
  void* bufs[4] = {w1b, b1b, w2b, b2b};
  const int64_t counts[4] = {n_i * n_h, n_h, n_h * n_o, n_o};
  return stade_ddp_allreduce_sum(comm, bufs, counts, 4, STADE_F32, n_local, n_global, opts);
}
stade_status stade_mlp2_ce_b_allreduce_reduced_f32(float* loss, stade_comm* comm,
                                                   const stade_opts* opts) {
  void* bufs[1] = {loss};
  const int64_t counts[1] = {1};
  return stade_ddp_allreduce_sum(comm, bufs, counts, 1, STADE_F32, 0, nullptr, opts);
}
stade_status stade_mlp2_ce_b_check_replicas_f32(const float* w1, const float* b1, const float* w2,
                                                const float* b2, const float* lossb, int64_t n_i,
                                                int64_t n_h, int64_t n_o, stade_comm* comm,
                                                uint64_t* bad_mask, const stade_opts* opts) {
  const void* bufs[5] = {w1, b1, w2, b2, lossb};
  const int64_t counts[5] = {n_i * n_h, n_h, n_h * n_o, n_o, 1};
  return stade_ddp_check_replicas(comm, bufs, counts, 5, STADE_F32, bad_mask, opts);
}


// ---- conv1d_relu_mse in adjoint mode, per_sample = [:x, :t] ------------------
// roles: :accum wb   :reduced loss   :local xb tb zb rb   :shared w   :seed lossb
stade_status stade_conv1d_relu_mse_b_reset_accum_f32(float* wb, int64_t n_o, int64_t n_c,
                                                     int64_t n_k, const stade_opts* opts) {
  void* bufs[1] = {wb};
  const int64_t counts[1] = {n_o * n_c * n_k};
  return stade_ddp_zero(bufs, counts, 1, STADE_F32, opts);
}
stade_status stade_conv1d_relu_mse_b_reset_reduced_f32(float* loss, const stade_opts* opts) {
  void* bufs[1] = {loss};
  const int64_t counts[1] = {1};
  return stade_ddp_zero(bufs, counts, 1, STADE_F32, opts);
}
stade_status stade_conv1d_relu_mse_b_reset_local_f32(float* xb, float* tb, float* zb, float* rb,
                                                     int64_t n_b, int64_t n_c, int64_t n_l,
                                                     int64_t n_o, int64_t n_k,
                                                     const stade_opts* opts) {
  const int64_t nt = n_b * n_o * (n_l - n_k + 1);
  STADE_REQUIRE(n_l >= n_k, "conv1d_relu_mse_b_reset_local: n_l < n_k");
  void* bufs[4] = {xb, tb, zb, rb};
  const int64_t counts[4] = {n_b * n_c * n_l, nt, nt, nt};
  return stade_ddp_zero(bufs, counts, 4, STADE_F32, opts);
}
stade_status stade_conv1d_relu_mse_b_allreduce_accum_f32(float* wb, int64_t n_o, int64_t n_c,
                                                         int64_t n_k, int64_t n_local,
                                                         stade_comm* comm, int64_t* n_global,
                                                         const stade_opts* opts) {
  void* bufs[1] = {wb};
  const int64_t counts[1] = {n_o * n_c * n_k};
  return stade_ddp_allreduce_sum(comm, bufs, counts, 1, STADE_F32, n_local, n_global, opts);
}
stade_status stade_conv1d_relu_mse_b_allreduce_reduced_f32(float* loss, stade_comm* comm,
                                                           const stade_opts* opts) {
  void* bufs[1] = {loss};
  const int64_t counts[1] = {1};
  return stade_ddp_allreduce_sum(comm, bufs, counts, 1, STADE_F32, 0, nullptr, opts);
}
stade_status stade_conv1d_relu_mse_b_check_replicas_f32(const float* w, const float* lossb,
                                                        int64_t n_o, int64_t n_c, int64_t n_k,
                                                        stade_comm* comm, uint64_t* bad_mask,
                                                        const stade_opts* opts) {
  const void* bufs[2] = {w, lossb};
  const int64_t counts[2] = {n_o * n_c * n_k, 1};
  return stade_ddp_check_replicas(comm, bufs, counts, 2, STADE_F32, bad_mask, opts);
}

// ---- mlp2_ce in hvp mode (the _hv names), per_sample = [:x, :y] --------------
// roles: :accum w1b b1b w2b b2b w1bd b1bd w2bd b2bd   :reduced loss lossd
//        :local xb yb hb zb pb xbd ybd hbd zbd pbd    :shared w1 b1 w2 b2 w1d b1d w2d b2d
//        :seed lossb lossbd
stade_status stade_mlp2_ce_hv_reset_accum_f64(double* w1b, double* b1b, double* w2b, double* b2b,
                                              double* w1bd, double* b1bd, double* w2bd,
                                              double* b2bd, int64_t n_i, int64_t n_h, int64_t n_o,
                                              const stade_opts* opts) {
  void* bufs[8] = {w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd};
  const int64_t counts[8] = {n_i * n_h, n_h, n_h * n_o, n_o, n_i * n_h, n_h, n_h * n_o, n_o};
  return stade_ddp_zero(bufs, counts, 8, STADE_F64, opts);
}
stade_status stade_mlp2_ce_hv_reset_reduced_f64(double* loss, double* lossd,
                                                const stade_opts* opts) {
  void* bufs[2] = {loss, lossd};
  const int64_t counts[2] = {1, 1};
  return stade_ddp_zero(bufs, counts, 2, STADE_F64, opts);
}
stade_status stade_mlp2_ce_hv_reset_local_f64(double* xb, double* yb, double* hb, double* zb,
                                              double* pb, double* xbd, double* ybd, double* hbd,
                                              double* zbd, double* pbd, int64_t n_s, int64_t n_i,
                                              int64_t n_h, int64_t n_o, const stade_opts* opts) {
  void* bufs[10] = {xb, yb, hb, zb, pb, xbd, ybd, hbd, zbd, pbd};
  const int64_t counts[10] = {n_s * n_i, n_s * n_o, n_s * n_h, n_s * n_o, n_s * n_o,
                              n_s * n_i, n_s * n_o, n_s * n_h, n_s * n_o, n_s * n_o};
  return stade_ddp_zero(bufs, counts, 10, STADE_F64, opts);
}
stade_status stade_mlp2_ce_hv_allreduce_accum_f64(double* w1b, double* b1b, double* w2b,
                                                  double* b2b, double* w1bd, double* b1bd,
                                                  double* w2bd, double* b2bd, int64_t n_i,
                                                  int64_t n_h, int64_t n_o, int64_t n_local,
                                                  stade_comm* comm, int64_t* n_global,
                                                  const stade_opts* opts) {
  void* bufs[8] = {w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd};
  const int64_t counts[8] = {n_i * n_h, n_h, n_h * n_o, n_o, n_i * n_h, n_h, n_h * n_o, n_o};
  return stade_ddp_allreduce_sum(comm, bufs, counts, 8, STADE_F64, n_local, n_global, opts);
}
stade_status stade_mlp2_ce_hv_allreduce_reduced_f64(double* loss, double* lossd, stade_comm* comm,
                                                    const stade_opts* opts) {
  void* bufs[2] = {loss, lossd};
  const int64_t counts[2] = {1, 1};
  return stade_ddp_allreduce_sum(comm, bufs, counts, 2, STADE_F64, 0, nullptr, opts);
}
stade_status stade_mlp2_ce_hv_check_replicas_f64(const double* w1, const double* b1,
                                                 const double* w2, const double* b2,
                                                 const double* w1d, const double* b1d,
                                                 const double* w2d, const double* b2d,
                                                 const double* lossb, const double* lossbd,
                                                 int64_t n_i, int64_t n_h, int64_t n_o,
                                                 stade_comm* comm, uint64_t* bad_mask,
                                                 const stade_opts* opts) {
  const void* bufs[10] = {w1, b1, w2, b2, w1d, b1d, w2d, b2d, lossb, lossbd};
  const int64_t counts[10] = {n_i * n_h, n_h, n_h * n_o, n_o, n_i * n_h, n_h, n_h * n_o, n_o, 1, 1};
  return stade_ddp_check_replicas(comm, bufs, counts, 10, STADE_F64, bad_mask, opts);
}

}  // extern "C"
