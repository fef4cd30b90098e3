// C-ABI error reporting and device queries shared by every kernel file.
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace tb {

static thread_local char g_last_error[512] = "";

static std::atomic<long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return set_error(TB_ELAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return TB_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("TESTT_B200_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}

static TimeoutReader g_readers[16];
static int g_n_readers = 0;

int register_timeout_reader(TimeoutReader reader) {
  if (g_n_readers < 16) g_readers[g_n_readers++] = reader;
  return g_n_readers;
}

}  // namespace tb

extern "C" const char *tb_last_error(void) { return tb::g_last_error; }

extern "C" int tb_wait_timeouts(int32_t device, uint32_t *count) {
  if (count == nullptr) return tb::set_error(TB_EINVAL, "wait_timeouts: count is required");
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return tb::check_launch("wait_timeouts");
  if (device >= 0 && cudaSetDevice(device) != cudaSuccess) return tb::check_launch("wait_timeouts");
  uint32_t total = 0;
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < tb::g_n_readers && e == cudaSuccess; ++i) {
    unsigned int c = 0;
    e = tb::g_readers[i](&c);
    total += c;
  }
  if (device >= 0) cudaSetDevice(prev);
  if (e != cudaSuccess)
    return tb::set_error(TB_ELAUNCH, "wait_timeouts: %s", cudaGetErrorString(e));
  *count = total;
  return TB_OK;
}

extern "C" int64_t tb_launch_count(void) { return tb::g_launches.load(std::memory_order_relaxed); }

extern "C" int tb_version(void) { return (0 << 16) | (1 << 8) | 0; }
