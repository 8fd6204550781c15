// Library-level C ABI: version, thread-local error text, tuning knobs.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace gnnb200 {

namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
std::atomic<uint64_t> g_launches{0};
}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

Config& config() {
  static Config cfg;
  return cfg;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;
  }
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int v = g_sm_count[dev];
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
      cudaGetLastError();
      v = 148;
    }
    g_sm_count[dev] = v;
  }
  return v;
}

}  // namespace gnnb200

using namespace gnnb200;

extern "C" int gnn_version(void) { return 0 * 10000 + 1 * 100 + 0; }

extern "C" uint64_t gnn_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" const char* gnn_last_error(void) { return g_last_error.c_str(); }

extern "C" const char* gnn_status_string(int status) {
  switch (status) {
    case GNN_OK: return "ok";
    case GNN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case GNN_ERR_NULL_POINTER: return "null pointer";
    case GNN_ERR_UNSUPPORTED: return "unsupported";
    case GNN_ERR_CUDA: return "cuda error";
    case GNN_ERR_TIMEOUT: return "timeout";
    case GNN_ERR_DEVICE: return "device error";
    case GNN_ERR_WORKSPACE: return "workspace error";
    default: return "unknown status";
  }
}

extern "C" int gnn_config_set_int(const char* name, int64_t value) {
  GNN_REQUIRE(name != nullptr, GNN_ERR_NULL_POINTER, "config name must not be NULL");
  if (std::strcmp(name, "spmm.long_row_threshold") == 0) {
    GNN_REQUIRE(value >= 0, GNN_ERR_INVALID_ARGUMENT, "spmm.long_row_threshold must be >= 0");
    config().long_row_threshold.store(value);
  } else if (std::strcmp(name, "spmm.long_row_warps") == 0) {
    GNN_REQUIRE(value >= 4 && value <= 16, GNN_ERR_INVALID_ARGUMENT,
                "spmm.long_row_warps must be in [4, 16]");
    config().long_row_warps.store(value);
  } else if (std::strcmp(name, "spmm.kernel") == 0) {
    GNN_REQUIRE(value >= 0 && value <= 2, GNN_ERR_INVALID_ARGUMENT, "spmm.kernel must be 0, 1 or 2");
    config().spmm_kernel.store(value);
  } else if (std::strcmp(name, "gemm.stages") == 0) {
    GNN_REQUIRE(value == 0 || (value >= 2 && value <= 8), GNN_ERR_INVALID_ARGUMENT,
                "gemm.stages must be 0 (automatic) or in [2, 8]");
    config().gemm_stages.store(value);
  } else if (std::strcmp(name, "spmm.schedule") == 0) {
    GNN_REQUIRE(value >= 0 && value <= 3, GNN_ERR_INVALID_ARGUMENT,
                "spmm.schedule must be 0 (id order), 1 (windowed degree order), 2 (global degree order) or "
                "3 (automatic)");
    config().spmm_schedule.store(value);
  } else if (std::strcmp(name, "spmm.schedule_window") == 0) {
    GNN_REQUIRE(value >= 1024 && value <= (int64_t(1) << 30), GNN_ERR_INVALID_ARGUMENT,
                "spmm.schedule_window must be in [1024, 2^30]");
    config().spmm_schedule_window.store(value);
  } else {
    return fail(GNN_ERR_INVALID_ARGUMENT, std::string("unknown config key: ") + name);
  }
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_config_get_int(const char* name, int64_t* value) {
  GNN_REQUIRE(name != nullptr && value != nullptr, GNN_ERR_NULL_POINTER, "name and value must not be NULL");
  if (std::strcmp(name, "spmm.long_row_threshold") == 0) {
    *value = config().long_row_threshold.load();
  } else if (std::strcmp(name, "spmm.long_row_warps") == 0) {
    *value = config().long_row_warps.load();
  } else if (std::strcmp(name, "spmm.kernel") == 0) {
    *value = config().spmm_kernel.load();
  } else if (std::strcmp(name, "gemm.stages") == 0) {
    *value = config().gemm_stages.load();
  } else if (std::strcmp(name, "spmm.schedule") == 0) {
    *value = config().spmm_schedule.load();
  } else if (std::strcmp(name, "spmm.schedule_window") == 0) {
    *value = config().spmm_schedule_window.load();
  } else {
    return fail(GNN_ERR_INVALID_ARGUMENT, std::string("unknown config key: ") + name);
  }
  clear_error();
  return GNN_OK;
}
