// Unified-memory migration counters without nsys: CUPTI's unified-memory
// activity records collected in-process.
//
// The reference measures UVM/HMM migration by wrapping a run in `nsys profile`,
// exporting SQLite and summing, over the feature matrix's address range, the
// host-to-device and device-to-host migration bytes and the GPU page faults
// (run/profile_spmm_migration.py:303-461, reported at :571-575). nsys is not
// available here; CUPTI, which nsys itself reads, is. This library enables the
// CUPTI_ACTIVITY_KIND_UNIFIED_MEMORY_COUNTER records (bytes HtoD/DtoH, GPU and
// CPU page faults, thrashing, throttling, remote maps), keeps a compact copy of
// every record as CUPTI hands over its buffers, and sums them on request over
// an address range and a time window with the reference's rules:
//   * a migration counts when [address, address + bytes) overlaps the range and
//     its [start, end) overlaps the window;
//   * a GPU page-fault record counts its `value` (page-fault groups of one page)
//     when its address lies in the range and its [start, end) overlaps the window.
// It is a separate shared library (libgnnb200_umprof.so) so that the aggregation
// library itself never depends on CUPTI.
#include <cupti.h>
#include <dlfcn.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gnn_b200_umprof.h"

namespace {

struct Record {
  uint64_t value, start, end, address;
  uint32_t kind;
};

std::mutex g_mu;
std::vector<Record> g_records;
uint64_t g_dropped = 0;
bool g_registered = false;
bool g_enabled = false;
size_t g_kinds = 0;  // counter kinds enabled: a prefix of kKinds
thread_local std::string g_error;

constexpr size_t kBufferBytes = 8u << 20;

int fail(int status, const std::string& msg) {
  g_error = msg;
  return status;
}

int cupti_fail(CUptiResult r, const char* what) {
  const char* s = nullptr;
  cuptiGetResultString(r, &s);
  return fail(GNN_ERR_CUDA, std::string(what) + ": " + (s ? s : "CUPTI error"));
}

void CUPTIAPI buffer_requested(uint8_t** buffer, size_t* size, size_t* max_records) {
  void* p = nullptr;
  if (posix_memalign(&p, 8, kBufferBytes) != 0) p = nullptr;
  *buffer = static_cast<uint8_t*>(p);
  *size = p ? kBufferBytes : 0;
  *max_records = 0;
}

void CUPTIAPI buffer_completed(CUcontext ctx, uint32_t stream_id, uint8_t* buffer, size_t /*size*/,
                               size_t valid) {
  std::vector<Record> local;
  CUpti_Activity* rec = nullptr;
  while (buffer != nullptr && cuptiActivityGetNextRecord(buffer, valid, &rec) == CUPTI_SUCCESS) {
    if (rec->kind != CUPTI_ACTIVITY_KIND_UNIFIED_MEMORY_COUNTER) continue;
    const auto* u = reinterpret_cast<const CUpti_ActivityUnifiedMemoryCounter3*>(rec);
    local.push_back(Record{u->value, u->start, u->end, u->address, static_cast<uint32_t>(u->counterKind)});
  }
  size_t dropped = 0;
  if (buffer != nullptr) cuptiActivityGetNumDroppedRecords(ctx, stream_id, &dropped);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    g_records.insert(g_records.end(), local.begin(), local.end());
    g_dropped += dropped;
  }
  free(buffer);
}

const CUpti_ActivityUnifiedMemoryCounterKind kKinds[] = {
    CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_BYTES_TRANSFER_HTOD,
    CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_BYTES_TRANSFER_DTOH,
    CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_GPU_PAGE_FAULT,
    CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_CPU_PAGE_FAULT_COUNT,
    CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_THRASHING,
    CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_THROTTLING,
    CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_REMOTE_MAP,
};

bool overlaps_window(const Record& r, uint64_t t0, uint64_t t1) {
  if (t0 == 0 && t1 == 0) return true;
  const uint64_t end = std::max(r.end, r.start);
  return r.start < t1 && end > t0;
}

// CUPTI enables the unified-memory counters only once the driver API is
// initialised (cuptiActivityEnable answers CUPTI_ERROR_NOT_READY before).
// cuInit creates no context; it is looked up at run time so that this library
// has no link-time dependency on the driver.
int init_driver() {
  void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) return fail(GNN_ERR_DEVICE, "libcuda.so.1 not found: no NVIDIA driver");
  using InitFn = int (*)(unsigned int);
  auto init = reinterpret_cast<InitFn>(dlsym(h, "cuInit"));
  if (init == nullptr) return fail(GNN_ERR_DEVICE, "cuInit not found in libcuda.so.1");
  const int rc = init(0);
  if (rc != 0) return fail(GNN_ERR_DEVICE, "cuInit failed with driver error " + std::to_string(rc));
  return GNN_OK;
}

}  // namespace

extern "C" int gnn_um_profiler_start(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_enabled) {
    g_error.clear();
    return GNN_OK;
  }
  // The unified-memory counters come from the driver's UVM tools interface
  // (/dev/nvidia-uvm-tools). Where that node is absent or closed (containers
  // often do not map it) CUPTI's enable fails in several ways and was seen to
  // crash the process, so it is not attempted at all.
  if (access("/dev/nvidia-uvm-tools", R_OK | W_OK) != 0) {
    return fail(GNN_ERR_UNSUPPORTED,
                "unified-memory counters need /dev/nvidia-uvm-tools, which this system does not provide");
  }
  const int drc = init_driver();
  if (drc != GNN_OK) return drc;
  CUptiResult r;
  if (!g_registered) {
    r = cuptiActivityRegisterCallbacks(buffer_requested, buffer_completed);
    if (r != CUPTI_SUCCESS) return cupti_fail(r, "cuptiActivityRegisterCallbacks");
    g_registered = true;
  }
  // One attempt with the three kinds the migration report needs; no retries
  // with other settings after a failure.
  constexpr size_t nk = 3;  // HtoD bytes, DtoH bytes, GPU page faults
  CUpti_ActivityUnifiedMemoryCounterConfig cfg[nk];
  std::memset(cfg, 0, sizeof(cfg));
  for (size_t i = 0; i < nk; ++i) {
    cfg[i].scope = CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_SCOPE_PROCESS_SINGLE_DEVICE;
    cfg[i].kind = kKinds[i];
    cfg[i].deviceId = 0;
    cfg[i].enable = 1;
  }
  r = cuptiActivityConfigureUnifiedMemoryCounter(cfg, static_cast<uint32_t>(nk));
  if (r == CUPTI_SUCCESS) r = cuptiActivityEnable(CUPTI_ACTIVITY_KIND_UNIFIED_MEMORY_COUNTER);
  const CUptiResult last = r;
  if (r == CUPTI_SUCCESS) g_kinds = nk;
  if (r != CUPTI_SUCCESS) return cupti_fail(last, "enabling CUPTI unified-memory counters");
  g_enabled = true;
  g_error.clear();
  return GNN_OK;
}

extern "C" int gnn_um_profiler_flush(void) {
  const CUptiResult r = cuptiActivityFlushAll(CUPTI_ACTIVITY_FLAG_FLUSH_FORCED);
  if (r != CUPTI_SUCCESS) return cupti_fail(r, "cuptiActivityFlushAll");
  g_error.clear();
  return GNN_OK;
}

extern "C" int gnn_um_profiler_stop(void) {
  bool was = false;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    was = g_enabled;
  }
  if (!was) {
    g_error.clear();
    return GNN_OK;
  }
  CUptiResult r = cuptiActivityFlushAll(CUPTI_ACTIVITY_FLAG_FLUSH_FORCED);
  if (r != CUPTI_SUCCESS) return cupti_fail(r, "cuptiActivityFlushAll");
  r = cuptiActivityDisable(CUPTI_ACTIVITY_KIND_UNIFIED_MEMORY_COUNTER);
  if (r != CUPTI_SUCCESS) return cupti_fail(r, "cuptiActivityDisable(UNIFIED_MEMORY_COUNTER)");
  std::lock_guard<std::mutex> lk(g_mu);
  g_enabled = false;
  g_error.clear();
  return GNN_OK;
}

extern "C" int gnn_um_profiler_clear(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_records.clear();
  g_dropped = 0;
  g_error.clear();
  return GNN_OK;
}

extern "C" uint64_t gnn_um_profiler_timestamp(void) {
  uint64_t t = 0;
  if (cuptiGetTimestamp(&t) != CUPTI_SUCCESS) return 0;
  return t;
}

extern "C" int gnn_um_profiler_totals(uint64_t range_begin, uint64_t range_end, uint64_t t_begin, uint64_t t_end,
                                      gnn_um_totals* out) {
  if (out == nullptr) return fail(GNN_ERR_NULL_POINTER, "out must not be NULL");
  if (range_end < range_begin) return fail(GNN_ERR_INVALID_ARGUMENT, "range_end must be >= range_begin");
  if (t_end < t_begin) return fail(GNN_ERR_INVALID_ARGUMENT, "t_end must be >= t_begin");
  const bool all = range_begin == 0 && range_end == 0;
  gnn_um_totals s;
  std::memset(&s, 0, sizeof(s));
  std::lock_guard<std::mutex> lk(g_mu);
  for (const Record& r : g_records) {
    if (!overlaps_window(r, t_begin, t_end)) continue;
    const bool bytes_kind = r.kind == CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_BYTES_TRANSFER_HTOD ||
                            r.kind == CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_BYTES_TRANSFER_DTOH ||
                            r.kind == CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_THRASHING ||
                            r.kind == CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_REMOTE_MAP;
    bool in_range = all;
    if (!all) {
      in_range = bytes_kind ? (r.address < range_end && r.address + r.value > range_begin)
                            : (r.address >= range_begin && r.address < range_end);
    }
    if (!in_range) continue;
    switch (r.kind) {
      case CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_BYTES_TRANSFER_HTOD: s.htod_bytes += double(r.value); break;
      case CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_BYTES_TRANSFER_DTOH: s.dtoh_bytes += double(r.value); break;
      case CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_GPU_PAGE_FAULT: s.gpu_page_faults += double(r.value); break;
      case CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_CPU_PAGE_FAULT_COUNT: s.cpu_page_faults += 1.0; break;
      case CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_THRASHING: s.thrashing_bytes += double(r.value); break;
      case CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_THROTTLING: s.throttling_events += 1.0; break;
      case CUPTI_ACTIVITY_UNIFIED_MEMORY_COUNTER_KIND_REMOTE_MAP: s.remote_map_bytes += double(r.value); break;
      default: break;
    }
    s.records += 1;
  }
  s.dropped_records = g_dropped;
  *out = s;
  g_error.clear();
  return GNN_OK;
}

extern "C" int gnn_um_profiler_enabled_kinds(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  return static_cast<int>(g_kinds);
}

extern "C" const char* gnn_um_profiler_last_error(void) { return g_error.c_str(); }
