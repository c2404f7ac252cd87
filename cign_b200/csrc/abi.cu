// Library-wide pieces of the C ABI: version, thread-local error text, device
// properties cache.
#include <algorithm>
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

int build_heavy_list(const int32_t* ptr_dev, int64_t rows, int threshold,
                     int32_t** heavy_out, int64_t* n_out,
                     int32_t* max_len_out) {
  *heavy_out = nullptr;
  *n_out = 0;
  *max_len_out = 0;
  std::vector<int32_t> ptr(static_cast<size_t>(rows) + 1);
  CIGN_CHECK_CUDA(cudaMemcpy(ptr.data(), ptr_dev, ptr.size() * sizeof(int32_t),
                             cudaMemcpyDeviceToHost),
                  "plan: copy row pointers");
  std::vector<std::pair<int32_t, int32_t>> heavy;  // (length, row)
  int32_t max_len = 0;
  for (int64_t r = 0; r < rows; ++r) {
    const int32_t len = ptr[r + 1] - ptr[r];
    max_len = std::max(max_len, len);
    if (len > threshold) heavy.emplace_back(len, static_cast<int32_t>(r));
  }
  std::stable_sort(heavy.begin(), heavy.end(),
                   [](const std::pair<int32_t, int32_t>& a,
                      const std::pair<int32_t, int32_t>& b) {
                     return a.first > b.first;
                   });
  *max_len_out = max_len;
  if (heavy.empty()) return CIGN_OK;
  std::vector<int32_t> rows_h(heavy.size());
  for (size_t i = 0; i < heavy.size(); ++i) rows_h[i] = heavy[i].second;
  int32_t* d = nullptr;
  CIGN_CHECK_CUDA(cudaMalloc(&d, rows_h.size() * sizeof(int32_t)),
                  "plan: cudaMalloc heavy list");
  cudaError_t e = cudaMemcpy(d, rows_h.data(), rows_h.size() * sizeof(int32_t),
                             cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return set_error(CIGN_ERR_CUDA, "plan: copy heavy list: %s",
                     cudaGetErrorString(e));
  }
  *heavy_out = d;
  *n_out = static_cast<int64_t>(rows_h.size());
  return CIGN_OK;
}

}  // namespace cign

extern "C" {

int cign_version(void) { return 1; }

const char* cign_last_error(void) { return cign::g_last_error.c_str(); }

}  // extern "C"
