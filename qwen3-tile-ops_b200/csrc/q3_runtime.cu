// Library-wide runtime state: launch counter and the benchmark timing hook.
#include <atomic>
#include <mutex>
#include <string.h>

#include "q3_common.cuh"

namespace {
std::atomic<uint64_t> g_launches{0};

struct Timer {
  std::mutex mu;
  int family = q3h::TIMER_NONE;
  void *const *start = nullptr;
  void *const *stop = nullptr;
  int capacity = 0;
  int used = 0;
  bool open = false;   // a begin without its end
};
Timer g_timer;
}  // namespace

namespace q3h {

// under stream capture a plain cudaEventRecord only adds a dependency; the
// external flag makes it an event-record node of the graph
static void record(void *ev, cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(s, &cs);
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(static_cast<cudaEvent_t>(ev), s, cudaEventRecordExternal);
  else
    cudaEventRecord(static_cast<cudaEvent_t>(ev), s);
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void timer_begin(int family, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_timer.mu);
  if (g_timer.family != family || g_timer.used >= g_timer.capacity) return;
  record(g_timer.start[g_timer.used], s);
  g_timer.open = true;
}

void timer_end(int family, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_timer.mu);
  if (g_timer.family != family || !g_timer.open) return;
  record(g_timer.stop[g_timer.used], s);
  g_timer.open = false;
  ++g_timer.used;
}

}  // namespace q3h

extern "C" uint64_t q3_launch_count(void) { return g_launches.load(); }

extern "C" int q3_timer_attach(const char *family, void *const *start_events,
                               void *const *stop_events, int capacity) {
  if (!family || !start_events || !stop_events || capacity <= 0) return Q3_ERR_NULL;
  int fam = q3h::TIMER_NONE;
  if (!strcmp(family, "attention")) fam = q3h::TIMER_ATTENTION;
  else if (!strcmp(family, "gemm")) fam = q3h::TIMER_GEMM;
  else if (!strcmp(family, "exchange")) fam = q3h::TIMER_EXCHANGE;
  else return Q3_ERR_SHAPE;
  std::lock_guard<std::mutex> lk(g_timer.mu);
  g_timer.family = fam;
  g_timer.start = start_events;
  g_timer.stop = stop_events;
  g_timer.capacity = capacity;
  g_timer.used = 0;
  g_timer.open = false;
  return Q3_OK;
}

extern "C" int q3_timer_detach(void) {
  std::lock_guard<std::mutex> lk(g_timer.mu);
  const int used = g_timer.used;
  g_timer.family = q3h::TIMER_NONE;
  g_timer.start = g_timer.stop = nullptr;
  g_timer.capacity = g_timer.used = 0;
  return used;
}
