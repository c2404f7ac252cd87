// Device-side dropout seed streams, for training steps captured in a CUDA
// graph.  The eager Python wrappers draw one seed per dropout call from two
// host counters (collapsed_gat.py:201-211 and fused_block_ops.py:46-50):
//   GAT call c:          (base + 0x9E3779B97F4A7C15 * (c + 1)) mod 2^63
//   block-op call c, t:  (base + 0x9E3779B97F4A7C15 * (c + 1)
//                              + 0xD2B74407B1CE6E93 * t) mod 2^63
// (t = 1 dropout-LayerNorm, t = 2 gamma residual).  Here the two counters
// live in device memory and one launch fills a table of the seeds of every
// dropout call of the next step (slot i: stream kind[i], tag[i], offset[i]
// within the step), then advances the counters by the step's call counts.
// The kernels of the step read their seed from the table (seed_ptr).
#include "common.cuh"

namespace cign {
namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kTagMul = 0xD2B74407B1CE6E93ull;
constexpr uint64_t kMask63 = (1ull << 63) - 1;

__global__ void seed_table_kernel(uint64_t base, int n_slots, const int32_t* __restrict__ layout,
                                  int64_t* __restrict__ counters, int32_t n_gat, int32_t n_block,
                                  uint64_t* __restrict__ table) {
  for (int i = threadIdx.x; i < n_slots; i += blockDim.x) {
    const int kind = layout[3 * i], tag = layout[3 * i + 1], off = layout[3 * i + 2];
    const uint64_t call = static_cast<uint64_t>(counters[kind]) + static_cast<uint64_t>(off) + 1;
    uint64_t s = base + kGolden * call;
    if (kind == 1) s += kTagMul * static_cast<uint64_t>(tag);
    table[i] = s & kMask63;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    counters[0] += n_gat;
    counters[1] += n_block;
  }
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_seed_table_step(uint64_t base, int32_t n_slots, const int32_t* layout, int64_t* counters,
                         int32_t n_gat, int32_t n_block, uint64_t* table, cign_stream_t stream) {
  CIGN_REQUIRE(n_slots >= 0 && n_slots <= 4096 && n_gat >= 0 && n_block >= 0,
               CIGN_ERR_INVALID_ARGUMENT, "seed_table_step: bad counts");
  CIGN_REQUIRE(counters != nullptr && (n_slots == 0 || (layout != nullptr && table != nullptr)),
               CIGN_ERR_NULL_POINTER, "seed_table_step: NULL argument");
  seed_table_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      base & kMask63, n_slots, layout, counters, n_gat, n_block, table);
  CIGN_CHECK_LAUNCH("seed_table_kernel");
  return CIGN_OK;
}

}  // extern "C"
