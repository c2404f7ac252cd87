// Halo exchange over peer memory (NVLink P2P stores) for the row-partitioned
// path: each rank writes the rows its peers need straight into the peers'
// halo buffers, which are mapped into its address space with CUDA IPC.
//
// One launch of halo_push_kernel covers every peer: flat row k of the send
// list belongs to the peer p with peer_begin[p] <= k < peer_begin[p+1]; the
// row src[idx[k]] (or src[k] when idx is NULL) is copied with 16-byte
// stores, one warp per row, to peer_dst[p] + (k - peer_begin[p]) * F.
// The stores are plain st.global to peer addresses (no multicast); the
// caller orders the copies against the peers' reads with a collective
// issued after the launch on the same stream.
//
// cign_halo_push_copy moves the same rows with the copy engines instead of
// SM stores: the send rows are gathered into a local staging buffer and
// each peer's block goes over NVLink as one cudaMemcpyAsync, so the
// transfer takes no SM time from the kernels it overlaps.  The peers are
// served in turn from `first_peer` (rank + 1 on the caller's side), so the
// ranks' copies form a permutation instead of all targeting one peer.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace cign {
namespace {

constexpr int kPushThreads = 256;

// Warp j copies send-list row order[j] (row j without an order): an order
// that interleaves the peers keeps every peer's inbound links busy at once
// instead of all ranks storing into the same peer first.
__global__ void __launch_bounds__(kPushThreads)
halo_push_kernel(int n_peers, const float* __restrict__ src, int64_t F,
                 const int64_t* __restrict__ idx, const int64_t* __restrict__ peer_begin,
                 float* const* __restrict__ peer_dst, int64_t total,
                 const int64_t* __restrict__ order) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kPushThreads / 32);
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * (kPushThreads / 32) + (threadIdx.x >> 5);
       j < total; j += warps) {
    const int64_t k = order != nullptr ? order[j] : j;
    int p = 0;
    while (p + 1 < n_peers && peer_begin[p + 1] <= k) ++p;  // few peers: linear scan
    const int64_t row = idx != nullptr ? idx[k] : k;
    const float4* s4 = reinterpret_cast<const float4*>(src + row * F);
    float4* d4 = reinterpret_cast<float4*>(peer_dst[p] + (k - peer_begin[p]) * F);
    for (int64_t q = lane; q < F / 4; q += 32) d4[q] = __ldg(s4 + q);
  }
}

// Gathers the send rows into a contiguous staging buffer in this GPU's own
// memory (warp per row, 16-byte copies), so that each peer's share is one
// contiguous block the copy engine can move.
__global__ void __launch_bounds__(kPushThreads)
halo_gather_kernel(const float* __restrict__ src, int64_t F, const int64_t* __restrict__ idx,
                   int64_t total, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kPushThreads / 32);
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * (kPushThreads / 32) + (threadIdx.x >> 5);
       k < total; k += warps) {
    const float4* s4 = reinterpret_cast<const float4*>(src + idx[k] * F);
    float4* d4 = reinterpret_cast<float4*>(out + k * F);
    for (int64_t q = lane; q < F / 4; q += 32) d4[q] = __ldg(s4 + q);
  }
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_device_alloc(size_t bytes, void** ptr) {
  CIGN_REQUIRE(ptr != nullptr, CIGN_ERR_NULL_POINTER, "device_alloc: ptr is NULL");
  *ptr = nullptr;
  if (bytes == 0) return CIGN_OK;
  CIGN_CHECK_CUDA(cudaMalloc(ptr, bytes), "device_alloc: cudaMalloc");
  return CIGN_OK;
}

int cign_device_free(void* ptr) {
  if (ptr != nullptr) CIGN_CHECK_CUDA(cudaFree(ptr), "device_free: cudaFree");
  return CIGN_OK;
}

int cign_ipc_handle(const void* ptr, void* handle) {
  CIGN_REQUIRE(ptr != nullptr && handle != nullptr, CIGN_ERR_NULL_POINTER,
               "ipc_handle: NULL argument");
  cudaIpcMemHandle_t h;
  CIGN_CHECK_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "ipc_handle");
  static_assert(sizeof(h) == CIGN_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return CIGN_OK;
}

int cign_ipc_open(const void* handle, void** ptr) {
  CIGN_REQUIRE(ptr != nullptr && handle != nullptr, CIGN_ERR_NULL_POINTER,
               "ipc_open: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  CIGN_CHECK_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc_open");
  return CIGN_OK;
}

int cign_ipc_close(void* ptr) {
  if (ptr != nullptr) CIGN_CHECK_CUDA(cudaIpcCloseMemHandle(ptr), "ipc_close");
  return CIGN_OK;
}

int cign_halo_push(int32_t n_peers, const float* src, int64_t F, const int64_t* idx,
                   const int64_t* peer_begin, float* const* peer_dst, int64_t total,
                   const int64_t* order, cign_stream_t stream) {
  CIGN_REQUIRE(n_peers >= 1 && F > 0 && total >= 0, CIGN_ERR_INVALID_ARGUMENT,
               "halo_push: bad sizes");
  if (total == 0) return CIGN_OK;
  CIGN_REQUIRE(src != nullptr && peer_begin != nullptr && peer_dst != nullptr,
               CIGN_ERR_NULL_POINTER, "halo_push: NULL argument");
  CIGN_REQUIRE(F % 4 == 0 && aligned16(src), CIGN_ERR_ALIGNMENT,
               "halo_push: rows must be float4-aligned (F %% 4 == 0)");
  const int64_t blocks = std::min<int64_t>((total + 7) / 8, 4 * 148 * 8);
  halo_push_kernel<<<static_cast<unsigned>(blocks), kPushThreads, 0,
                     static_cast<cudaStream_t>(stream)>>>(n_peers, src, F, idx, peer_begin,
                                                          peer_dst, total, order);
  CIGN_CHECK_LAUNCH("halo_push_kernel");
  return CIGN_OK;
}

int cign_halo_push_copy(int32_t n_peers, const float* src, int64_t F, const int64_t* idx,
                        const int64_t* peer_begin_host, float* const* peer_dst_host,
                        int64_t total, float* staging, int32_t first_peer,
                        cign_stream_t stream) {
  CIGN_REQUIRE(n_peers >= 1 && F > 0 && total >= 0, CIGN_ERR_INVALID_ARGUMENT,
               "halo_push_copy: bad sizes");
  if (total == 0) return CIGN_OK;
  CIGN_REQUIRE(src != nullptr && peer_begin_host != nullptr && peer_dst_host != nullptr,
               CIGN_ERR_NULL_POINTER, "halo_push_copy: NULL argument");
  CIGN_REQUIRE(peer_begin_host[0] == 0 && peer_begin_host[n_peers] == total,
               CIGN_ERR_INVALID_ARGUMENT, "halo_push_copy: peer_begin must run from 0 to total");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float* rows = src;
  if (idx != nullptr) {
    CIGN_REQUIRE(staging != nullptr, CIGN_ERR_NULL_POINTER,
                 "halo_push_copy: a gathered push needs a staging buffer of total * F floats");
    CIGN_REQUIRE(F % 4 == 0 && aligned16(src) && aligned16(staging), CIGN_ERR_ALIGNMENT,
                 "halo_push_copy: rows must be float4-aligned (F %% 4 == 0)");
    const int64_t blocks = std::min<int64_t>((total + 7) / 8, 4 * 148 * 8);
    halo_gather_kernel<<<static_cast<unsigned>(blocks), kPushThreads, 0, s>>>(src, F, idx, total,
                                                                              staging);
    CIGN_CHECK_LAUNCH("halo_gather_kernel");
    rows = staging;
  }
  CIGN_REQUIRE(first_peer >= 0 && first_peer < n_peers, CIGN_ERR_INVALID_ARGUMENT,
               "halo_push_copy: first_peer out of range");
  for (int i = 0; i < n_peers; ++i) {  // peers in turn from first_peer
    const int p = (first_peer + i) % n_peers;
    const int64_t b = peer_begin_host[p], e = peer_begin_host[p + 1];
    CIGN_REQUIRE(b <= e, CIGN_ERR_INVALID_ARGUMENT, "halo_push_copy: peer_begin not sorted");
    if (e == b) continue;
    CIGN_REQUIRE(peer_dst_host[p] != nullptr, CIGN_ERR_NULL_POINTER,
                 "halo_push_copy: NULL destination for peer %d", p);
    CIGN_CHECK_CUDA(cudaMemcpyAsync(peer_dst_host[p], rows + b * F,
                                    static_cast<size_t>(e - b) * F * sizeof(float),
                                    cudaMemcpyDeviceToDevice, s),
                    "halo_push_copy: cudaMemcpyAsync");
  }
  return CIGN_OK;
}

}  // extern "C"
