// Library state behind the C ABI: error text, launch counting, the cached
// per-device workspace, and the buffer-zeroing entry point of the epilogue.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace stade {

namespace {
thread_local std::string g_last_error;
thread_local int g_launches = 0;

struct CachedWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_ws_mutex;
std::vector<CachedWorkspace> g_ws;  // indexed by device ordinal
}  // namespace

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

stade_status fail(stade_status code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

stade_status cuda_fail(cudaError_t e, const char* what, const char* file, int line) {
  return fail(STADE_ECUDA, "%s failed at %s:%d: %s (%s)", what, file, line, cudaGetErrorName(e),
              cudaGetErrorString(e));
}

void count_launch() { ++g_launches; }

namespace {
struct PhaseRec {
  std::string name;
  cudaEvent_t a, b;
};
thread_local bool g_prof = false;
thread_local std::vector<PhaseRec> g_recs;      // recorded, not yet read
thread_local std::vector<cudaEvent_t> g_pool;   // reusable events
thread_local std::vector<std::string> g_open;   // names of open phases
thread_local std::vector<cudaEvent_t> g_open_ev;

cudaEvent_t take_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}
}  // namespace

bool profile_on() { return g_prof; }

void phase_begin(const char* name, cudaStream_t s) {
  cudaEvent_t e = take_event();
  cudaEventRecord(e, s);
  g_open.push_back(name);
  g_open_ev.push_back(e);
}

void phase_end(cudaStream_t s) {
  if (g_open.empty()) return;
  cudaEvent_t e = take_event();
  cudaEventRecord(e, s);
  g_recs.push_back(PhaseRec{g_open.back(), g_open_ev.back(), e});
  g_open.pop_back();
  g_open_ev.pop_back();
}

stade_status get_workspace(const stade_opts* o, size_t bytes, void** p) {
  *p = nullptr;
  if (bytes == 0) return STADE_OK;
  if (o && o->workspace) {
    if (o->workspace_bytes < bytes)
      return fail(STADE_EINVAL, "workspace too small: %zu bytes given, %zu needed",
                  o->workspace_bytes, bytes);
    if ((reinterpret_cast<uintptr_t>(o->workspace) & 255u) != 0)
      return fail(STADE_EINVAL, "workspace must be 256-byte aligned");
    *p = o->workspace;
    return STADE_OK;
  }
  int dev = 0;
  STADE_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  if ((int)g_ws.size() <= dev) g_ws.resize(dev + 1);
  CachedWorkspace& w = g_ws[dev];
  if (w.bytes < bytes) {
    // Growth happens once per size class; a caller that must not allocate
    // passes its own workspace instead.
    if (w.ptr) {
      STADE_CUDA(cudaDeviceSynchronize());
      STADE_CUDA(cudaFree(w.ptr));
      w.ptr = nullptr;
      w.bytes = 0;
    }
    STADE_CUDA(cudaMalloc(&w.ptr, bytes));
    w.bytes = bytes;
  }
  *p = w.ptr;
  return STADE_OK;
}

}  // namespace stade

extern "C" {

const char* stade_last_error(void) { return stade::g_last_error.c_str(); }
const char* stade_version(void) { return "libstade_b200 0.1 (sm_100a)"; }
int stade_kernel_launches(void) { return stade::g_launches; }
void stade_reset_kernel_launches(void) { stade::g_launches = 0; }

size_t stade_workspace_cached_bytes(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(stade::g_ws_mutex);
  return dev < (int)stade::g_ws.size() ? stade::g_ws[dev].bytes : 0;
}

void stade_profile_enable(int on) { stade::g_prof = on != 0; }

// Sums the recorded phases by name (in first-seen order) into names / ms /
// counts (up to max entries), waits for their events, and clears the record.
// Returns the number of distinct phases.
int stade_profile_read(char* names, int name_len, double* ms, int* counts, int max) {
  using namespace stade;
  std::vector<std::string> order;
  std::vector<double> tot;
  std::vector<int> cnt;
  for (auto& r : g_recs) {
    cudaEventSynchronize(r.b);
    float t = 0.f;
    cudaEventElapsedTime(&t, r.a, r.b);
    size_t i = 0;
    for (; i < order.size(); ++i)
      if (order[i] == r.name) break;
    if (i == order.size()) {
      order.push_back(r.name);
      tot.push_back(0.0);
      cnt.push_back(0);
    }
    tot[i] += t;
    cnt[i] += 1;
    g_pool.push_back(r.a);
    g_pool.push_back(r.b);
  }
  g_recs.clear();
  const int n = (int)order.size();
  for (int i = 0; i < n && i < max; ++i) {
    if (names && name_len > 0) {
      std::strncpy(names + (size_t)i * name_len, order[i].c_str(), name_len - 1);
      names[(size_t)i * name_len + name_len - 1] = 0;
    }
    if (ms) ms[i] = tot[i];
    if (counts) counts[i] = cnt[i];
  }
  return n;
}

stade_status stade_ddp_zero(void* const* bufs, const int64_t* counts, int nbuf, int dtype,
                            const stade_opts* opts) {
  STADE_REQUIRE(nbuf >= 0 && (nbuf == 0 || (bufs && counts)), "stade_ddp_zero: bad buffer list");
  STADE_REQUIRE(dtype == STADE_F32 || dtype == STADE_F64, "stade_ddp_zero: bad dtype %d", dtype);
  const size_t es = dtype == STADE_F32 ? 4 : 8;
  cudaStream_t s = stade::stream_of(opts);
  stade::PhaseScope ph("reset", s);
  // buffers that follow each other in memory are cleared by one memset
  char* run = nullptr;
  size_t run_bytes = 0;
  for (int i = 0; i < nbuf; ++i) {
    STADE_REQUIRE(counts[i] >= 0, "stade_ddp_zero: negative count for buffer %d", i);
    if (counts[i] == 0) continue;
    STADE_REQUIRE(bufs[i] != nullptr, "stade_ddp_zero: null buffer %d", i);
    char* p = static_cast<char*>(bufs[i]);
    const size_t bytes = (size_t)counts[i] * es;
    if (run && run + run_bytes == p) {
      run_bytes += bytes;
      continue;
    }
    if (run) STADE_CUDA(cudaMemsetAsync(run, 0, run_bytes, s));
    run = p;
    run_bytes = bytes;
  }
  if (run) STADE_CUDA(cudaMemsetAsync(run, 0, run_bytes, s));
  return STADE_OK;
}

}  // extern "C"
