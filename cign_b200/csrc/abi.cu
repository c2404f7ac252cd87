// Library-wide pieces of the C ABI: version, thread-local error text, device
// properties cache.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "common.cuh"

namespace cign {

namespace {
thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
std::mutex g_sm_mutex;
int g_sm_count[64] = {0};
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  if (g_sm_count[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess ||
        v <= 0)
      v = 148;
    g_sm_count[dev] = v;
  }
  return g_sm_count[dev];
}

int build_segments(const int32_t* ptr_dev, int64_t rows, int seg_len, SegList* out) {
  *out = SegList();
  out->seg_len = seg_len;
  if (rows <= 0) return CIGN_OK;
  std::vector<int32_t> ptr(static_cast<size_t>(rows) + 1);
  CIGN_CHECK_CUDA(cudaMemcpy(ptr.data(), ptr_dev, ptr.size() * sizeof(int32_t),
                             cudaMemcpyDeviceToHost),
                  "plan: copy row pointers");
  std::vector<std::pair<int32_t, int32_t>> heavy;  // (length, row)
  // light rows bucketed by length (counting sort: longest first, ties in row order)
  std::vector<int64_t> bucket(static_cast<size_t>(seg_len) + 2, 0);
  int32_t max_len = 0;
  for (int64_t r = 0; r < rows; ++r) {
    const int32_t len = ptr[r + 1] - ptr[r];
    max_len = std::max(max_len, len);
    if (len > seg_len) heavy.emplace_back(len, static_cast<int32_t>(r));
    else ++bucket[static_cast<size_t>(seg_len - len) + 1];
  }
  out->max_len = max_len;
  for (size_t b = 1; b < bucket.size(); ++b) bucket[b] += bucket[b - 1];
  const int64_t n_light = bucket.back();
  std::vector<int32_t> light(static_cast<size_t>(n_light));
  for (int64_t r = 0; r < rows; ++r) {
    const int32_t len = ptr[r + 1] - ptr[r];
    if (len <= seg_len) light[static_cast<size_t>(bucket[static_cast<size_t>(seg_len - len)]++)] =
        static_cast<int32_t>(r);
  }
  std::stable_sort(heavy.begin(), heavy.end(),
                   [](const std::pair<int32_t, int32_t>& a,
                      const std::pair<int32_t, int32_t>& b) { return a.first > b.first; });
  std::vector<int32_t> srow, sbeg, send, hrow, hfirst;
  for (const auto& hr : heavy) {
    const int32_t r = hr.second;
    hrow.push_back(r);
    hfirst.push_back(static_cast<int32_t>(srow.size()));
    for (int32_t b = ptr[r]; b < ptr[r + 1]; b += seg_len) {
      srow.push_back(r);
      sbeg.push_back(b);
      send.push_back(std::min(b + seg_len, ptr[r + 1]));
    }
  }
  hfirst.push_back(static_cast<int32_t>(srow.size()));
  const int64_t n_seg = static_cast<int64_t>(srow.size());
  const int64_t n_heavy = static_cast<int64_t>(hrow.size());
  std::vector<int32_t> host;
  host.reserve(3 * n_seg + 2 * n_heavy + 1 + n_light);
  host.insert(host.end(), srow.begin(), srow.end());
  host.insert(host.end(), sbeg.begin(), sbeg.end());
  host.insert(host.end(), send.begin(), send.end());
  host.insert(host.end(), hrow.begin(), hrow.end());
  host.insert(host.end(), hfirst.begin(), hfirst.end());
  host.insert(host.end(), light.begin(), light.end());
  int32_t* d = nullptr;
  CIGN_CHECK_CUDA(cudaMalloc(&d, host.size() * sizeof(int32_t)), "plan: cudaMalloc segments");
  cudaError_t e = cudaMemcpy(d, host.data(), host.size() * sizeof(int32_t), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return set_error(CIGN_ERR_CUDA, "plan: copy segments: %s", cudaGetErrorString(e));
  }
  out->buf = d;
  out->n_seg = n_seg;
  out->n_heavy = n_heavy;
  out->n_light = n_light;
  return CIGN_OK;
}

void free_segments(SegList* s) {
  if (s->buf) cudaFree(s->buf);
  *s = SegList();
}

}  // namespace cign

extern "C" {

int cign_version(void) { return 1; }

const char* cign_last_error(void) { return cign::g_last_error.c_str(); }

uint64_t cign_kernel_launches(void) {
  return cign::g_launches.load(std::memory_order_relaxed);
}

}  // extern "C"
