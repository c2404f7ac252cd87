// Clifford pack + proj linear layer as one tcgen05 GEMM (TF32, fp32 accumulate):
//
//   out[n, :] = G[n, :] @ W^T + bias,   G = pack(H_norm, C_norm, P_1..P_K, alpha)
//
// for the production pack switches (interaction "new", outer none, alpha
// weighting "old": G[n, k*2D + d] = a_k W_k[d], G[n, k*2D + D + d] = a_k D_k[d];
// generic_engine/model_cign.py:869-876 followed by the block's proj,
// model_cign.py:927-929).  The reference materialises G [N, 2KD] in HBM and runs a
// separate cuBLAS GEMM on it; here G is produced tile by tile straight into
// shared memory as the MMA's A operand and never round-trips through HBM
// (optionally it is also written out once, for the proj weight gradient).
// The pack is evaluated with the hardware exponential (values within ~1e-6
// relative of cign_pack_fwd's), since it only feeds TF32 products and the
// TF32-tolerance weight gradient.
//
// One CTA owns 128 node rows and the whole output width (Dout <= 512 fp32
// accumulator columns of tensor memory).  Warp roles:
//   warp 0      one lane streams W k-blocks into a shared-memory ring with
//               cp.async.bulk (no multicast): W is re-laid out once per call
//               (pack_proj_prepare_w) into the MMA's 128-byte-swizzled K-major
//               tile order, so each k-block is one contiguous copy;
//   warp 1      allocates tensor memory; one lane issues tcgen05.mma
//               (kind::tf32, M=128, N<=256 per instruction) and releases ring
//               slots with tcgen05.commit;
//   warps 2-17  (4 threads per row, 8 channels each) read H/C/P rows with
//               16-byte loads, evaluate the pack for 32 channels x K hops,
//               round to TF32 and store the A tiles in the swizzled layout;
//               afterwards they drain the accumulator (tcgen05.ld), add the
//               bias and store the output rows.
// Every wait on an mbarrier is bounded (kWaitLimit polls, or earlier once
// another role gave up); on expiry the CTA records kStatusTimeout in the
// status word, stops producing, lets issued copies and MMAs complete
// (bounded waits) and frees its tensor memory before it exits.
#include <algorithm>

#include "common.cuh"
#include "pack_math.cuh"

namespace cign {
namespace {

constexpr int kPPThreads = 576;      // 18 warps
constexpr int kPPProducers = 512;    // warps 2..17
constexpr int kPPRows = 128;         // rows per CTA (MMA M)
constexpr int kPPBK = 32;            // fp32 k-elements per k-block (128 bytes per row)
constexpr int kPPAStages = 3;
constexpr int kPPMaxK = 8;
constexpr uint32_t kATileBytes = kPPRows * kPPBK * 4;  // 16 KB
constexpr size_t kPPSmemBudget = 208 * 1024;

struct PPtrs { const float* p[kPPMaxK]; };

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                   dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, both K-major; accumulate selects +=.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive once on `bar` when every tcgen05 op issued so far by this thread is done
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::
                   "r"(bar)
               : "memory");
}
// this warp's 32 TMEM lanes x 32 consecutive 32-bit columns starting at taddr
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte
// swizzle layout: rows of 128 bytes (32 fp32), groups of 8 rows 1024 bytes
// apart (stride byte offset), tile base 1024-byte aligned; the k-offset
// inside the 128-byte row is added to the start address.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address, 16 B units
  d |= static_cast<uint64_t>(1) << 16;                           // leading offset (unused)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;                   // stride offset: 8-row group
  d |= static_cast<uint64_t>(1) << 46;                           // descriptor version
  d |= static_cast<uint64_t>(2) << 61;                           // 128-byte swizzle
  return d;
}
// Instruction descriptor: TF32 x TF32 -> F32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t tf32_idesc(uint32_t n) {
  return (1u << 4)          // D format F32
         | (2u << 7)        // A format TF32
         | (2u << 10)       // B format TF32
         | ((n >> 3) << 17) // N / 8
         | ((128u >> 4) << 24);  // M / 16
}
// byte offset of element (row, col) of a [rows x 32] fp32 K-major tile in the
// 128-byte swizzle layout (16-byte chunk index XOR row within the 8-row group)
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t col) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + ((((col >> 2) ^ (row & 7u)) & 7u) << 4) +
         (col & 3u) * 4u;
}

// The production interaction ("new", outer none) with the SiLU from the
// hardware exponential and fast division: the values feed a TF32 product
// (operands rounded to 2^-11 relative), so their ~1e-6 relative error is
// immaterial, and the shorter dependency chain keeps the few producer warps
// per scheduler ahead of the tensor core.
__device__ __forceinline__ void interact_fwd_fast(float bhr, float brh, float& D, float& W) {
  const float sym = 0.5f * (bhr + brh);
  D = __fdividef(sym, 1.0f + __expf(-sym));
  W = 0.5f * (bhr - brh);
}

// wait on `bar` for `parity`, bounded; gives up early once *abort is set
__device__ __forceinline__ bool pp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  for (unsigned i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort) return false;
  }
  return false;
}
__device__ __forceinline__ void pp_fail(volatile int* abort, int* status) {
  *abort = 1;
  atomicExch(status, kStatusTimeout);
}

// W [dout, kdim] row-major -> per 32-column k-block, a [dout x 32] tile in the
// 128-byte swizzle layout, values rounded to TF32.
__global__ void pack_proj_prepare_w(const float* __restrict__ w, int64_t dout, int64_t kdim,
                                    float* __restrict__ wt) {
  const int64_t chunks = dout * kdim / 4;  // float4 chunks
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < chunks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / (kdim / 4);
    const int64_t c = (i % (kdim / 4)) * 4;
    const int64_t kb = c / kPPBK;
    float4 v = __ldg(reinterpret_cast<const float4*>(w + n * kdim + c));
    v.x = to_tf32(v.x);
    v.y = to_tf32(v.y);
    v.z = to_tf32(v.z);
    v.w = to_tf32(v.w);
    char* tile = reinterpret_cast<char*>(wt) + static_cast<size_t>(kb) * dout * 128;
    *reinterpret_cast<float4*>(tile + sw128_offset(static_cast<uint32_t>(n),
                                                   static_cast<uint32_t>(c % kPPBK))) = v;
  }
}

// W ring entries hold one 256-row chunk of a k-block (32 KB at 32 columns):
// finer than whole k-blocks (Dout x 128 B), so more of W is in flight.
constexpr int kPPChunkRows = 256;
constexpr uint32_t kBEntryBytes = kPPChunkRows * kPPBK * 4;  // 32 KB

__global__ void __launch_bounds__(kPPThreads, 1)
pack_proj_kernel(int64_t n, int64_t D, int K, int64_t dout, const float* __restrict__ H,
                 const float* __restrict__ C, PPtrs P, int64_t ldp,
                 const float* __restrict__ alpha, const float* __restrict__ wt,
                 const float* __restrict__ bias, float* __restrict__ out,
                 float* __restrict__ g_out, int b_stages, uint32_t tmem_cols,
                 int* __restrict__ status) {
  extern __shared__ __align__(1024) unsigned char pp_smem_raw[];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;
  __shared__ const float* hop_ptr_sh[kPPMaxK];
  // 1024-byte aligned operand rings (the swizzle pattern is address based)
  const uint32_t raw = smem_u32(pp_smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* base_ptr = pp_smem_raw + (base - raw);
  const uint32_t a_ring = base;
  const uint32_t b_ring = a_ring + kPPAStages * kATileBytes;
  const uint32_t bars = b_ring + b_stages * kBEntryBytes;
  auto a_full = [&](int s) { return bars + 8u * s; };
  auto a_empty = [&](int s) { return bars + 8u * (kPPAStages + s); };
  auto b_full = [&](int s) { return bars + 8u * (2 * kPPAStages + s); };
  auto b_empty = [&](int s) { return bars + 8u * (2 * kPPAStages + b_stages + s); };
  const uint32_t acc_full = bars + 8u * (2 * kPPAStages + 2 * b_stages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kPPRows;
  const int64_t kdim = 2 * K * D;
  const int n_db = static_cast<int>(D / kPPBK);
  const int n_blocks = n_db * K * 2;  // k-blocks in production order (db, hop, half)
  const int n_chunks = static_cast<int>((dout + kPPChunkRows - 1) / kPPChunkRows);
  volatile int* abort = &abort_sh;

#pragma unroll
  for (int i = 0; i < kPPMaxK; ++i)
    if (threadIdx.x == i) hop_ptr_sh[i] = P.p[i];
  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < kPPAStages; ++s) {
      mbar_init(a_full(s), kPPProducers);
      mbar_init(a_empty(s), 1);
    }
    for (int s = 0; s < b_stages; ++s) {
      mbar_init(b_full(s), 1);
      mbar_init(b_empty(s), 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_base_sh), tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ------------------------------------------------ W chunk stream
    if (lane == 0) {
      const int n_entries = n_blocks * n_chunks;
      int issued = 0;
      for (int e = 0; e < n_entries; ++e) {
        const int s = e % b_stages;
        const int u = e / b_stages;
        if (u > 0 && !pp_wait(b_empty(s), (u - 1) & 1, abort)) {
          pp_fail(abort, status);
          break;
        }
        if (*abort) break;
        const int b = e / n_chunks;
        const int c = e % n_chunks;
        const int db = b / (2 * K);
        const int hop = (b / 2) % K;
        const int half = b & 1;
        const int64_t kb = (static_cast<int64_t>(hop) * 2 * D + half * D) / kPPBK + db;
        const int64_t r0 = static_cast<int64_t>(c) * kPPChunkRows;
        const uint32_t bytes =
            static_cast<uint32_t>((dout - r0 < kPPChunkRows ? dout - r0 : kPPChunkRows) * 128);
        mbar_expect_tx(b_full(s), bytes);
        bulk_g2s(b_ring + s * kBEntryBytes, wt + (kb * dout + r0) * kPPBK, bytes, b_full(s));
        ++issued;
      }
      // let the last copy of every slot land before the CTA can exit (a
      // plain bounded wait: it must not give up early on abort)
      for (int e = max(0, issued - b_stages); e < issued; ++e)
        mbar_wait(b_full(e % b_stages), (e / b_stages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issue
    if (lane == 0) {
      bool ok = true;
      for (int b = 0; b < n_blocks && ok; ++b) {
        const int sa = b % kPPAStages, ua = b / kPPAStages;
        if (!pp_wait(a_full(sa), ua & 1, abort)) {
          pp_fail(abort, status);
          break;
        }
        const uint32_t a_addr = a_ring + sa * kATileBytes;
        for (int c = 0; c < n_chunks; ++c) {
          const int e = b * n_chunks + c;
          const int sb = e % b_stages, ub = e / b_stages;
          if (!pp_wait(b_full(sb), ub & 1, abort)) {
            pp_fail(abort, status);
            ok = false;
            break;
          }
          tc_fence_after();
          const int64_t n0 = static_cast<int64_t>(c) * kPPChunkRows;
          const uint32_t nn = static_cast<uint32_t>(dout - n0 < kPPChunkRows ? dout - n0
                                                                             : kPPChunkRows);
          const uint32_t idesc = tf32_idesc(nn);
          const uint32_t b_addr = b_ring + sb * kBEntryBytes;
#pragma unroll
          for (int kk = 0; kk < kPPBK / 8; ++kk) {
            umma_tf32(tmem + static_cast<uint32_t>(n0), sw128_kmajor_desc(a_addr + kk * 32),
                      sw128_kmajor_desc(b_addr + kk * 32), idesc, (b > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(b_empty(sb));
        }
        if (ok) umma_commit(a_empty(sa));
      }
      umma_commit(acc_full);
      // every MMA issued above completes before tensor memory is freed
      if (!mbar_wait(acc_full, 0)) pp_fail(abort, status);
    }
  } else {
    // ------------------------------------------------ pack producers
    // Steps walk (d-block, hop); the next step's P rows are loaded while the
    // current step is evaluated and stored.
    const int t = threadIdx.x - 64;
    const int r = t >> 2;          // tile row
    const int hf = t & 3;          // which 8 of the 32 channels
    const int64_t row = row0 + r;
    const bool valid = row < n;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    const int n_steps = n_db * K;
    float4 h4[2], c4[2], th[2], tc[2];
    float a;
    auto load_hc = [&](int db, float4 (&hh)[2], float4 (&cc)[2]) {
      const int64_t d0 = static_cast<int64_t>(db) * kPPBK + hf * 8;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        hh[q] = valid ? __ldg(reinterpret_cast<const float4*>(H + row * D + d0) + q) : zero;
        cc[q] = valid ? __ldg(reinterpret_cast<const float4*>(C + row * D + d0) + q) : zero;
      }
    };
    auto load_p = [&](int db, int hop, float4 (&pth)[2], float4 (&ptc)[2], float& pa) {
      const int64_t d0 = static_cast<int64_t>(db) * kPPBK + hf * 8;
      const float* prow = hop_ptr_sh[hop] + row * ldp;
      pa = valid ? __ldg(alpha + row * K + hop) : 0.0f;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        pth[q] = valid ? __ldg(reinterpret_cast<const float4*>(prow + d0) + q) : zero;
        ptc[q] = valid ? __ldg(reinterpret_cast<const float4*>(prow + D + d0) + q) : zero;
      }
    };
    load_hc(0, h4, c4);
    load_p(0, 0, th, tc, a);
    for (int step = 0; step < n_steps && !*abort; ++step) {
      const int db = step / K;
      const int hop = step % K;
      float4 nth[2], ntc[2];
      float na = 0.0f;
      const bool more = step + 1 < n_steps;
      const bool new_db = more && (step + 1) % K == 0;
      if (more) load_p((step + 1) / K, (step + 1) % K, nth, ntc, na);
      const int64_t d0 = static_cast<int64_t>(db) * kPPBK + hf * 8;
      // both A slots of this step (W half, D half) must be free
      const int b0 = step * 2;
      const int s0 = b0 % kPPAStages, s1 = (b0 + 1) % kPPAStages;
      const int u0 = b0 / kPPAStages, u1 = (b0 + 1) / kPPAStages;
      if ((u0 > 0 && !pp_wait(a_empty(s0), (u0 - 1) & 1, abort)) ||
          (u1 > 0 && !pp_wait(a_empty(s1), (u1 - 1) & 1, abort))) {
        pp_fail(abort, status);
        break;
      }
      unsigned char* tile0 = base_ptr + s0 * kATileBytes;
      unsigned char* tile1 = base_ptr + s1 * kATileBytes;
      float* g = (g_out != nullptr && valid)
                     ? g_out + row * kdim + static_cast<int64_t>(hop) * 2 * D + d0
                     : nullptr;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float4 wv, dv;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float Dv, Wv;
          interact_fwd_fast(vel(h4[q], j) * vel(tc[q], j), vel(c4[q], j) * vel(th[q], j), Dv,
                            Wv);
          vel(wv, j) = a * Wv;
          vel(dv, j) = a * Dv;
        }
        if (g != nullptr) {
          reinterpret_cast<float4*>(g)[q] = wv;
          reinterpret_cast<float4*>(g + D)[q] = dv;
        }
        const uint32_t off = sw128_offset(r, hf * 8 + q * 4);
        *reinterpret_cast<float4*>(tile0 + off) =
            make_float4(to_tf32(wv.x), to_tf32(wv.y), to_tf32(wv.z), to_tf32(wv.w));
        *reinterpret_cast<float4*>(tile1 + off) =
            make_float4(to_tf32(dv.x), to_tf32(dv.y), to_tf32(dv.z), to_tf32(dv.w));
      }
      fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
      mbar_arrive(a_full(s0));
      mbar_arrive(a_full(s1));
      if (more) {
        // H/C rows of the next d-block go into the registers just freed
        if (new_db) load_hc(db + 1, h4, c4);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          th[q] = nth[q];
          tc[q] = ntc[q];
        }
        a = na;
      }
    }
    // ------------------------------------------------ epilogue
    const bool ok = pp_wait(acc_full, 0, abort);
    if (!ok) pp_fail(abort, status);
    tc_fence_after();
    // warp-uniform decision: tcgen05.ld is a .sync.aligned warp instruction
    if (__all_sync(kFullMask, ok && !*abort)) {
      const int q = warp & 3;                  // TMEM lane quarter of this warp
      const int cg = (warp - 2) >> 2;          // column group 0..3 (warps 2-5, 6-9, ...)
      const int64_t orow = row0 + q * 32 + lane;
      for (int64_t c0 = cg * 32; c0 < dout; c0 += 128) {
        uint32_t v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c0), v);
        tmem_ld_wait();
        if (orow < n) {
          float* o = out + orow * dout + c0;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 f;
            f.x = __uint_as_float(v[j + 0]) + __ldg(bias + c0 + j + 0);
            f.y = __uint_as_float(v[j + 1]) + __ldg(bias + c0 + j + 1);
            f.z = __uint_as_float(v[j + 2]) + __ldg(bias + c0 + j + 2);
            f.w = __uint_as_float(v[j + 3]) + __ldg(bias + c0 + j + 3);
            *reinterpret_cast<float4*>(o + j) = f;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

size_t pp_wt_bytes(int64_t dout, int64_t kdim) {
  return (static_cast<size_t>(dout) * kdim * 4 + 1023) / 1024 * 1024;
}
int pp_b_stages() {
  const size_t room = kPPSmemBudget - kPPAStages * kATileBytes;
  return static_cast<int>(std::min<size_t>(8, room / kBEntryBytes));
}
size_t pp_smem_bytes(int b_stages) {
  return 1024 /* alignment slack */ + kPPAStages * kATileBytes +
         static_cast<size_t>(b_stages) * kBEntryBytes + 8 * (2 * kPPAStages + 2 * b_stages + 1);
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

size_t cign_pack_proj_workspace_bytes(int64_t d, int32_t k, int64_t dout) {
  if (d <= 0 || k <= 0 || dout <= 0) return 0;
  return pp_wt_bytes(dout, 2 * k * d) + 256;
}

int cign_pack_proj_gemm_tf32(int64_t n, int64_t d, int32_t k, int64_t dout, const float* h,
                             const float* c, const float* const* p, int64_t ldp,
                             const float* alpha, const float* w, const float* bias, float* out,
                             float* g_out, void* ws, size_t ws_bytes, cign_stream_t stream) {
  CIGN_REQUIRE(n >= 0 && d >= 1 && dout >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "pack_proj: bad sizes");
  CIGN_REQUIRE(k >= 1 && k <= kPPMaxK, CIGN_ERR_UNSUPPORTED,
               "pack_proj: hop count must be in [1, %d]", kPPMaxK);
  CIGN_REQUIRE(d % kPPBK == 0, CIGN_ERR_UNSUPPORTED, "pack_proj: D must be a multiple of 32");
  CIGN_REQUIRE(dout % 32 == 0 && dout <= 512, CIGN_ERR_UNSUPPORTED,
               "pack_proj: Dout must be a multiple of 32 and <= 512");
  CIGN_REQUIRE(ldp >= 2 * d && ldp % 4 == 0, CIGN_ERR_INVALID_ARGUMENT,
               "pack_proj: ldp must be >= 2D and a multiple of 4");
  CIGN_REQUIRE(p != nullptr && w != nullptr && bias != nullptr && ws != nullptr,
               CIGN_ERR_NULL_POINTER, "pack_proj: NULL argument");
  const int64_t kdim = 2 * static_cast<int64_t>(k) * d;
  const size_t need = cign_pack_proj_workspace_bytes(d, k, dout);
  CIGN_REQUIRE(ws_bytes >= need, CIGN_ERR_INVALID_ARGUMENT,
               "pack_proj: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  CIGN_REQUIRE(aligned16(ws) && aligned16(w), CIGN_ERR_ALIGNMENT,
               "pack_proj: W and ws must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* wt = static_cast<float*>(ws);
  int* status = reinterpret_cast<int*>(static_cast<char*>(ws) + pp_wt_bytes(dout, kdim));
  CIGN_CHECK_CUDA(cudaMemsetAsync(status, 0, sizeof(int), s), "pack_proj: reset status");
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(h != nullptr && c != nullptr && alpha != nullptr && out != nullptr,
               CIGN_ERR_NULL_POINTER, "pack_proj: NULL argument");
  CIGN_REQUIRE(aligned16(h) && aligned16(c) && aligned16(out) &&
                   (g_out == nullptr || aligned16(g_out)),
               CIGN_ERR_ALIGNMENT, "pack_proj: H, C, out, G must be 16-byte aligned");
  PPtrs P{};
  for (int i = 0; i < k; ++i) {
    CIGN_REQUIRE(p[i] != nullptr, CIGN_ERR_NULL_POINTER, "pack_proj: P[%d] is NULL", i);
    CIGN_REQUIRE(aligned16(p[i]), CIGN_ERR_ALIGNMENT, "pack_proj: P[%d] must be 16-byte aligned",
                 i);
    P.p[i] = p[i];
  }
  {
    const int64_t chunks = dout * kdim / 4;
    const int blocks = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, 4 * 148));
    pack_proj_prepare_w<<<blocks, 256, 0, s>>>(w, dout, kdim, wt);
    CIGN_CHECK_LAUNCH("pack_proj_prepare_w");
  }
  const int b_stages = pp_b_stages();
  const size_t smem = pp_smem_bytes(b_stages);
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(dout)) cols <<= 1;
  {
    // raise the kernel's dynamic shared-memory limit once per device (to the
    // largest size any Dout needs), outside any later stream capture
    static int configured[64] = {0};
    int dev = 0;
    CIGN_CHECK_CUDA(cudaGetDevice(&dev), "pack_proj: device");
    if (dev < 0 || dev >= 64 || !configured[dev]) {
      CIGN_CHECK_CUDA(cudaFuncSetAttribute(pack_proj_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kPPSmemBudget + 16 * 1024)),
                      "pack_proj: smem attribute");
      if (dev >= 0 && dev < 64) configured[dev] = 1;
    }
  }
  CIGN_REQUIRE(smem <= kPPSmemBudget + 16 * 1024, CIGN_ERR_UNSUPPORTED,
               "pack_proj: shared memory plan too large");
  const int64_t grid = (n + kPPRows - 1) / kPPRows;
  CIGN_REQUIRE(grid < (1ll << 31), CIGN_ERR_UNSUPPORTED, "pack_proj: too many rows");
  pack_proj_kernel<<<static_cast<unsigned>(grid), kPPThreads, smem, s>>>(
      n, d, k, dout, h, c, P, ldp, alpha, wt, bias, out, g_out, b_stages, cols, status);
  CIGN_CHECK_LAUNCH("pack_proj_kernel");
  return CIGN_OK;
}

int cign_pack_proj_status(const void* ws, int64_t d, int32_t k, int64_t dout,
                          cign_stream_t stream) {
  CIGN_REQUIRE(ws != nullptr, CIGN_ERR_NULL_POINTER, "pack_proj_status: ws is NULL");
  const int* status = reinterpret_cast<const int*>(static_cast<const char*>(ws) +
                                                   pp_wt_bytes(dout, 2 * k * d));
  int v = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CIGN_CHECK_CUDA(cudaMemcpyAsync(&v, status, sizeof(int), cudaMemcpyDeviceToHost, s),
                  "pack_proj_status: copy");
  CIGN_CHECK_CUDA(cudaStreamSynchronize(s), "pack_proj_status: sync");
  CIGN_REQUIRE(v == 0, CIGN_ERR_TIMEOUT, "pack_proj: a device-side wait expired");
  return CIGN_OK;
}

}  // extern "C"
