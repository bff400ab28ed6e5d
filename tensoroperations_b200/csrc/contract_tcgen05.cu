// contract_tcgen05.cu -- the permuted multilevel contraction chain on the
// 5th-generation tensor cores (tcgen05 + TMEM + TMA), fp32 accurate.
//
//   T[a,b,c,d] = sum_{e,f} A[a,e,c,f] * B[f,b,e,d]        (step 1, 2 E^6 flops)
//   R[a,d]     = sum_{b,c} T[a,b,c,d] * C[c,b]             (step 2, fused)
// every extent E (32, 64 or 128), row-major tensors.  This is the chain the
// reference expresses with ContractionNodes over permuted operands
// (benchmarks/permuted_contraction/bench_permuted_contraction.cpp,
// benchmarks/multilevel_contraction/bench_multilevel_contraction.cpp; its
// evaluator permutes operands in scratch, include/TensorOperations/Permute.hpp:127-228).
//
// Step 1 is one dense GEMM once the labels are grouped: M = (a,c), N = (b,d),
// K = (e,f).  Both operands enter the tensor core K-major, 128B-swizzled:
//   A tile: a 4-D TMA box {f:32, c, a, e:1} of A in place (A viewed as dims
//           (f, c, a, e)): rows (a,c) of 32 K-values = 128 B;
//   B tile: rows (b,d) of 32 K-values from B' = B regrouped as [b][d][e][f]
//           (a 2-D box over (K, N)).  B's own layout has K outermost, so the
//           split pre-pass writes it regrouped (E x E tile transposes through
//           shared memory); the TF32 MMA did not accept B in N-major order
//           with the plain 128-byte swizzle.
// fp32 accuracy from three TF32 products: a = a_hi + a_lo with a_hi = a rounded
// to TF32 (exactly representable, so the tensor core reads it unchanged) and
// a_lo = a - a_hi (exact in fp32); T ~ A_hi B_hi + A_hi B_lo + A_lo B_hi, the
// dropped A_lo B_lo term being about 2^-22 relative.  Two pre-pass kernels
// write the four split operands into the caller's workspace.
//
// CTA: 10 warps.  warp 0 lane 0 issues TMA into a 2-stage ring (full/empty
// mbarriers); warp 1 owns the TMEM allocation (512 columns: two 128 x 256
// fp32 accumulators) and lane 0 issues tcgen05.mma (M=128, N=256, K=8,
// kind::tf32) and tcgen05.commit.  K is processed in chunks of 512 values,
// alternating between the two accumulators; warps 2-9 (the epilogue, one row
// x 128 columns per thread) drain each finished chunk into IEEE fp32 registers
// while the next chunk accumulates.  The tensor core's own fp32 accumulation
// is not rounded like IEEE additions and its error grows with the number of
// accumulated products (measured: 2.9e-5 relative at K = 4096 in one
// accumulator); chunking bounds it independently of E.  At the end each
// thread multiplies its row (a, c) by C[c, b], the rows are summed over c
// through shared memory into R[a, d] (atomicAdd; R is zeroed first), and
// optionally the T tile is stored (for checks).  Every wait is
// bounded; on a timeout the kernel records TO_ERR_TIMEOUT in the device status
// word, waits (bounded) for its own copies in flight, frees its TMEM and
// returns.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "common.hpp"
#include "sm100_primitives.cuh"

namespace to_b200 {
// This file's device status word (device symbols are per translation unit);
// to_device_status() reads it together with the SEM kernels' word.
__device__ int g_chain_status = 0;
}

namespace to_b200 {
namespace {

constexpr int kTileM = 128, kTileN = 256, kTileK = 32, kStages = 2;
constexpr int kEpilogueWarps = 8;
constexpr int kThreads = 64 + 32 * kEpilogueWarps;
constexpr int kChunkIters = 16;  // K-iterations (of 32) per TMEM accumulation chunk
constexpr uint32_t kABytes = kTileM * kTileK * 4;  // 16 KB
constexpr uint32_t kBBytes = kTileN * kTileK * 4;  // 32 KB
constexpr uint32_t kStageBytes = 2 * kABytes + 2 * kBBytes;  // A_hi, A_lo, B_hi, B_lo
constexpr uint32_t kSmemBytes = 1024 + kStages * kStageBytes + 1024;
constexpr long long kMaxPolls = 1ll << 24;

struct ChainArgs {
  const float* C;   // [E][E]  C[c][b]
  float* R;         // [E][E]  R[a][d]
  float* T;         // optional [E][E][E][E] T[a][b][c][d]
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor, 128B swizzle, sm100 version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t((saddr >> 4) & 0x3FFFu)) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor: D f32, A/B tf32, both K-major, N=256, M=128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (0u << 15) | (0u << 16) |
                            (uint32_t(kTileN >> 3) << 17) | (uint32_t(kTileM >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_one(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity) {
  for (long long i = 0; i < kMaxPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

#define TO_TMEM_LD_X32(taddr, r)                                                               \
  asm volatile(                                                                                \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13," \
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"   \
      "tcgen05.wait::ld.sync.aligned;"                                                         \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),    \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),             \
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),          \
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),          \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),          \
        "=r"(r[31])                                                                            \
      : "r"(taddr)                                                                             \
      : "memory")

template <int E>
__global__ void __launch_bounds__(kThreads, 1)
    chain_tcgen05_kernel(const __grid_constant__ CUtensorMap mAhi, const __grid_constant__ CUtensorMap mAlo,
                         const __grid_constant__ CUtensorMap mBhi, const __grid_constant__ CUtensorMap mBlo,
                         const ChainArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned tiles (128B swizzle atoms)
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* tiles = base;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2] a chunk's accumulator is complete
  uint64_t* acc_empty = acc_full + 2;    // [2] the epilogue has drained it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int a_per_tile = kTileM / E;   // a-values in the M tile (M = a * E + c)
  constexpr int k_iters = E * (E / 32);    // K = E^2 in steps of 32
  constexpr int nchunks = k_iters / kChunkIters;
  static_assert(k_iters % kChunkIters == 0, "whole chunks");
  const int m_tile = blockIdx.y, n_tile = blockIdx.x;
  const int a0 = m_tile * a_per_tile;
  const int b0 = n_tile * (kTileN / E);  // N = b * E + d

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], kEpilogueWarps);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(uint32_t(2 * kTileN)) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- producer ----
    int issued = 0;
    bool ok = true;
    for (int it = 0; it < k_iters && ok; ++it) {
      const int s = it % kStages, n = it / kStages;
      if (n > 0 && !wait_bounded(&empty[s], (n - 1) & 1)) {
        ok = false;
        break;
      }
      if (*reinterpret_cast<volatile int*>(abort_flag)) break;
      unsigned char* st = tiles + s * kStageBytes;
      const int e = it / (E / 32), f0 = (it % (E / 32)) * 32;
      mbar_arrive_expect_tx(&full[s], kStageBytes);
      // A view (f, c, a, e); B' view (K = (e,f), N = (b,d))
      tma_load_4d(st, &mAhi, f0, 0, a0, e, &full[s]);
      tma_load_4d(st + kABytes, &mAlo, f0, 0, a0, e, &full[s]);
      tma_load_2d(st + 2 * kABytes, &mBhi, it * 32, n_tile * kTileN, &full[s]);
      tma_load_2d(st + 2 * kABytes + kBBytes, &mBlo, it * 32, n_tile * kTileN, &full[s]);
      issued = it + 1;
    }
    if (!ok) {
      atomicExch(&g_chain_status, int(TO_ERR_TIMEOUT));
      atomicExch(abort_flag, 1);
    }
    // copies still in flight land before the CTA exits
    for (int it = (issued > kStages ? issued - kStages : 0); it < issued; ++it)
      wait_bounded(&full[it % kStages], (it / kStages) & 1);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: chunk ch accumulates into TMEM columns [ (ch%2)*256, +256 ) ----
    bool ok = true;
    for (int ch = 0; ch < nchunks && ok; ++ch) {
      const int j = ch & 1;
      if (ch >= 2 && !wait_bounded(&acc_empty[j], ((ch >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t dacc = tmem + uint32_t(j * kTileN);
      for (int ci = 0; ci < kChunkIters; ++ci) {
        const int it = ch * kChunkIters + ci;
        const int s = it % kStages, n = it / kStages;
        if (!wait_bounded(&full[s], n & 1) || *reinterpret_cast<volatile int*>(abort_flag)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t st = smem_u32(tiles + s * kStageBytes);
        const uint32_t sAhi = st, sAlo = st + kABytes, sBhi = st + 2 * kABytes,
                       sBlo = st + 2 * kABytes + kBBytes;
#pragma unroll
        for (int k = 0; k < kTileK / 8; ++k) {
          // K-major: 8 tf32 = 32 B per step inside each 128 B row; 8-row
          // groups 1 KB apart.
          const uint64_t dAhi = umma_desc(sAhi + 32 * k, 16, 1024);
          const uint64_t dAlo = umma_desc(sAlo + 32 * k, 16, 1024);
          const uint64_t dBhi = umma_desc(sBhi + 32 * k, 16, 1024);
          const uint64_t dBlo = umma_desc(sBlo + 32 * k, 16, 1024);
          umma_tf32(dacc, dAlo, dBhi, (ci > 0 || k > 0) ? 1u : 0u);
          umma_tf32(dacc, dAhi, dBlo, 1u);
          umma_tf32(dacc, dAhi, dBhi, 1u);
        }
        umma_commit(&empty[s]);  // frees the stage when these MMAs have read it
      }
      umma_commit(&acc_full[j]);  // this chunk's partial sums are complete
    }
    if (!ok) {
      atomicExch(&g_chain_status, int(TO_ERR_TIMEOUT));
      atomicExch(abort_flag, 1);
    }
  } else if (warp >= 2) {
    // ---- epilogue: thread = accumulator row (a, c) x 128 of the 256 columns.
    // Each finished chunk is added into registers in IEEE fp32, so the tensor
    // core never sums more than kChunkIters * 32 K-values. ----
    const int ew = warp - 2;           // 0..7
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int h = ew >> 2;             // column half
    const int row = q * 32 + lane;     // M index inside the tile
    const int al = row / E, c = row - al * E;
    float acc[kTileN / 2];
#pragma unroll
    for (int x = 0; x < kTileN / 2; ++x) acc[x] = 0.f;
    bool live = true;
    for (int ch = 0; ch < nchunks; ++ch) {
      const int j = ch & 1;
      const bool ok = live && wait_bounded(&acc_full[j], (ch >> 1) & 1);
      if (!ok || *reinterpret_cast<volatile int*>(abort_flag)) {
        if (live) atomicExch(&g_chain_status, int(TO_ERR_TIMEOUT));
        live = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int part = 0; part < 4; ++part) {
        uint32_t r[32];
        // load and wait in one statement: the registers exist only once the
        // asynchronous load has completed
        TO_TMEM_LD_X32(tmem + (uint32_t(q * 32) << 16) + uint32_t(j * kTileN + h * 128 + part * 32), r);
#pragma unroll
        for (int x = 0; x < 32; ++x) acc[part * 32 + x] += __uint_as_float(r[x]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_one(&acc_empty[j]);
    }
    // T tile rows (optional) and R = sum over b of T * C[c, b]
    const int col0 = h * 128;  // N index of acc[0]
    if (live && args.T) {
#pragma unroll
      for (int x = 0; x < 128; ++x) {
        const int n = col0 + x, bl = n / E, d = n - bl * E;
        args.T[((size_t(a0 + al) * E + (b0 + bl)) * E + c) * E + d] = acc[x];
      }
    }
    // this half holds kFold b-values; fold them into slots d = 0..E-1
    constexpr int kFold = 128 / E;
#pragma unroll
    for (int g = 0; g < kFold; ++g) {
      const float cb = __ldg(args.C + size_t(c) * E + (b0 + h * kFold + g));
#pragma unroll
      for (int d = 0; d < E; ++d) acc[g * E + d] *= cb;
    }
#pragma unroll
    for (int g = 1; g < kFold; ++g)
#pragma unroll
      for (int d = 0; d < E; ++d) acc[d] += acc[g * E + d];
    asm volatile("bar.sync 1, 256;" ::: "memory");  // every epilogue thread is past the chunk loop
    // red[h][row][E]: each half's row sums, rotated by row to spread banks
    float* red = reinterpret_cast<float*>(tiles);
#pragma unroll
    for (int d = 0; d < E; ++d) red[(size_t(h) * kTileM + row) * E + ((d + row) % E)] = acc[d];
    asm volatile("bar.sync 1, 256;" ::: "memory");
    // (al2, d) pairs: a_per_tile * E = 128 of them
    const int t = threadIdx.x - 64;
    if (live && t < kTileM) {
      const int al2 = t / E, d = t - al2 * E;
      float sum = 0.f;
      for (int hh = 0; hh < 2; ++hh)
        for (int cc = 0; cc < E; ++cc) {
          const int rr = al2 * E + cc;
          sum += red[(size_t(hh) * kTileM + rr) * E + ((d + rr) % E)];
        }
      atomicAdd(args.R + size_t(a0 + al2) * E + d, sum);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(uint32_t(2 * kTileN)) : "memory");
}

// ---- the general contraction as one GEMM: C[m][n] = sum_k A[m][k] B[n][k] ----
// The same producer / MMA issuer / epilogue roles as the chain kernel, on
// operands already grouped K-major and split into TF32 hi/lo (the caller -- the
// frontend's contraction lowering -- packs them): A [Mp][Kp], B [Np][Kp], C
// [Mp][Np] row-major, Mp a multiple of 128, Np of 256, Kp of 32.  K runs in
// chunks of kChunkIters steps alternating between the two TMEM accumulators,
// the last chunk possibly shorter; each finished chunk is added in IEEE fp32.
// One CTA per work unit (one CTA fits an SM).  Units [0, full_tiles) are whole
// 128 x 256 tiles, stored; when the tiles do not fill the last wave of SMs,
// each remaining tile is split in K between `split` (= 2) CTAs that add their
// halves into C, zeroed by the host beforehand -- the last wave then takes
// half as long.  Two contributions to a zero keep the sum independent of
// their order.
struct GemmArgs {
  float* C;
  long long ldc;
  int k_iters;     // K-iterations (of 32) of a whole tile
  int tiles_n;     // tiles along N
  int full_tiles;  // units that are whole tiles
  int split;       // K-parts of each remaining tile (1 or 2)
};

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap mAhi, const __grid_constant__ CUtensorMap mAlo,
                        const __grid_constant__ CUtensorMap mBhi, const __grid_constant__ CUtensorMap mBlo,
                        const GemmArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* tiles = base;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int tile = static_cast<int>(blockIdx.x), k_begin = 0, k_end = args.k_iters;
  bool partial = false;
  if (tile >= args.full_tiles) {
    const int r = tile - args.full_tiles, part = r % args.split;
    tile = args.full_tiles + r / args.split;
    k_begin = static_cast<int>(static_cast<long long>(args.k_iters) * part / args.split);
    k_end = static_cast<int>(static_cast<long long>(args.k_iters) * (part + 1) / args.split);
    partial = args.split > 1;
  }
  const int k_iters = k_end - k_begin;
  const int nchunks = (k_iters + kChunkIters - 1) / kChunkIters;
  const int m_tile = tile / args.tiles_n, n_tile = tile % args.tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], kEpilogueWarps);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(uint32_t(2 * kTileN)) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- producer ----
    int issued = 0;
    bool ok = true;
    for (int it = 0; it < k_iters && ok; ++it) {
      const int s = it % kStages, n = it / kStages;
      if (n > 0 && !wait_bounded(&empty[s], (n - 1) & 1)) {
        ok = false;
        break;
      }
      if (*reinterpret_cast<volatile int*>(abort_flag)) break;
      unsigned char* st = tiles + s * kStageBytes;
      mbar_arrive_expect_tx(&full[s], kStageBytes);
      const int kx = (k_begin + it) * kTileK;
      tma_load_2d(st, &mAhi, kx, m_tile * kTileM, &full[s]);
      tma_load_2d(st + kABytes, &mAlo, kx, m_tile * kTileM, &full[s]);
      tma_load_2d(st + 2 * kABytes, &mBhi, kx, n_tile * kTileN, &full[s]);
      tma_load_2d(st + 2 * kABytes + kBBytes, &mBlo, kx, n_tile * kTileN, &full[s]);
      issued = it + 1;
    }
    if (!ok) {
      atomicExch(&g_chain_status, int(TO_ERR_TIMEOUT));
      atomicExch(abort_flag, 1);
    }
    for (int it = (issued > kStages ? issued - kStages : 0); it < issued; ++it)
      wait_bounded(&full[it % kStages], (it / kStages) & 1);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    bool ok = true;
    for (int ch = 0; ch < nchunks && ok; ++ch) {
      const int j = ch & 1;
      if (ch >= 2 && !wait_bounded(&acc_empty[j], ((ch >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t dacc = tmem + uint32_t(j * kTileN);
      const int iters = (k_iters - ch * kChunkIters) < kChunkIters ? (k_iters - ch * kChunkIters)
                                                                    : kChunkIters;
      for (int ci = 0; ci < iters; ++ci) {
        const int it = ch * kChunkIters + ci;
        const int s = it % kStages, n = it / kStages;
        if (!wait_bounded(&full[s], n & 1) || *reinterpret_cast<volatile int*>(abort_flag)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t st = smem_u32(tiles + s * kStageBytes);
        const uint32_t sAhi = st, sAlo = st + kABytes, sBhi = st + 2 * kABytes,
                       sBlo = st + 2 * kABytes + kBBytes;
#pragma unroll
        for (int k = 0; k < kTileK / 8; ++k) {
          const uint64_t dAhi = umma_desc(sAhi + 32 * k, 16, 1024);
          const uint64_t dAlo = umma_desc(sAlo + 32 * k, 16, 1024);
          const uint64_t dBhi = umma_desc(sBhi + 32 * k, 16, 1024);
          const uint64_t dBlo = umma_desc(sBlo + 32 * k, 16, 1024);
          umma_tf32(dacc, dAlo, dBhi, (ci > 0 || k > 0) ? 1u : 0u);
          umma_tf32(dacc, dAhi, dBlo, 1u);
          umma_tf32(dacc, dAhi, dBhi, 1u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(&acc_full[j]);
    }
    if (!ok) {
      atomicExch(&g_chain_status, int(TO_ERR_TIMEOUT));
      atomicExch(abort_flag, 1);
    }
  } else if (warp >= 2) {
    // ---- epilogue: thread = tile row x 128 of the 256 columns ----
    const int ew = warp - 2;
    const int q = warp & 3;
    const int h = ew >> 2;
    const int row = q * 32 + lane;
    float acc[kTileN / 2];
#pragma unroll
    for (int x = 0; x < kTileN / 2; ++x) acc[x] = 0.f;
    bool live = true;
    for (int ch = 0; ch < nchunks; ++ch) {
      const int j = ch & 1;
      const bool ok = live && wait_bounded(&acc_full[j], (ch >> 1) & 1);
      if (!ok || *reinterpret_cast<volatile int*>(abort_flag)) {
        if (live) atomicExch(&g_chain_status, int(TO_ERR_TIMEOUT));
        live = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int part = 0; part < 4; ++part) {
        uint32_t r[32];
        TO_TMEM_LD_X32(tmem + (uint32_t(q * 32) << 16) + uint32_t(j * kTileN + h * 128 + part * 32), r);
#pragma unroll
        for (int x = 0; x < 32; ++x) acc[part * 32 + x] += __uint_as_float(r[x]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_one(&acc_empty[j]);
    }
    if (live) {
      float4* out = reinterpret_cast<float4*>(args.C + (size_t(m_tile) * kTileM + row) * args.ldc +
                                              size_t(n_tile) * kTileN + h * 128);
      if (partial) {
#pragma unroll
        for (int x = 0; x < 32; ++x)
          atomicAdd(out + x, make_float4(acc[4 * x], acc[4 * x + 1], acc[4 * x + 2], acc[4 * x + 3]));
      } else {
#pragma unroll
        for (int x = 0; x < 32; ++x)
          out[x] = make_float4(acc[4 * x], acc[4 * x + 1], acc[4 * x + 2], acc[4 * x + 3]);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(uint32_t(2 * kTileN)) : "memory");
}

// hi = x rounded to TF32 (low 13 mantissa bits zero), lo = x - hi (exact).
__global__ void tf32_split_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float v = x[i];
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
    const float hv = __uint_as_float(h);
    hi[i] = hv;
    lo[i] = v - hv;
  }
}

// B[f][b][e][d] -> B'[b][d][e][f] (hi and lo): for each (b, e) an E x E
// transpose of (f, d), through a 32 x 33 shared tile.
__global__ void tf32_split_regroup_b_kernel(const float* __restrict__ B, float* __restrict__ hi,
                                            float* __restrict__ lo, int E) {
  __shared__ float tile[32][33];
  const int nt = E / 32;
  int blk = blockIdx.x;
  const int ft = blk % nt; blk /= nt;
  const int dt = blk % nt; blk /= nt;
  const int e = blk % E;
  const int b = blk / E;
  const size_t E2 = size_t(E) * E, E3 = E2 * E;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int f = ft * 32 + r, d = dt * 32 + threadIdx.x;
    tile[r][threadIdx.x] = B[f * E3 + b * E2 + size_t(e) * E + d];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int d = dt * 32 + r, f = ft * 32 + threadIdx.x;
    const float v = tile[threadIdx.x][r];
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
    const size_t o = b * E3 + d * E2 + size_t(e) * E + f;
    hi[o] = __uint_as_float(h);
    lo[o] = v - __uint_as_float(h);
  }
}

// ---- host: tensor maps through the driver entry point ---------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn(int* st) {
  static std::once_flag once;
  static EncodeTiled fn = nullptr;
  static int status = TO_OK;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p) {
      cudaGetLastError();
      status = set_error(TO_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
      return;
    }
    fn = reinterpret_cast<EncodeTiled>(p);
  });
  *st = status;
  return fn;
}

int make_map(EncodeTiled enc, CUtensorMap* m, const void* ptr, int rank, const cuuint64_t* dims,
             const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void*>(ptr), dims,
                         strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TO_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return ok();
}

template <int E>
int launch_chain(dim3 grid, const CUtensorMap& a, const CUtensorMap& al, const CUtensorMap& b,
                 const CUtensorMap& bl, const ChainArgs& args, cudaStream_t s) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(chain_tcgen05_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kSmemBytes));
  });
  TO_CUDA_TRY(attr);
  chain_tcgen05_kernel<E><<<grid, kThreads, kSmemBytes, s>>>(a, al, b, bl, args);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // namespace

int chain_device_status(int reset, int* value) {
  int v = 0;
  TO_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_chain_status, sizeof(int)));
  if (reset && v) {
    const int z = 0;
    TO_CUDA_TRY(cudaMemcpyToSymbol(g_chain_status, &z, sizeof(int)));
  }
  *value = v;
  return ok();
}

}  // namespace to_b200

using namespace to_b200;

extern "C" {

size_t to_chain_workspace_bytes(int32_t E) {
  if (E != 32 && E != 64 && E != 128) return 0;
  const size_t n = size_t(E) * E * E * E;
  return 4 * n * sizeof(float);
}

int to_chain_f32(int32_t E, const float* A, const float* B, const float* C, float* R, float* T,
                 void* workspace, size_t workspace_bytes, void* stream) {
  if (E != 32 && E != 64 && E != 128)
    return set_error(TO_ERR_UNSUPPORTED, "to_chain_f32: extent %d (built: 32, 64, 128)", E);
  if (!A || !B || !C || !R || !workspace)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_chain_f32: null pointer");
  if (workspace_bytes < to_chain_workspace_bytes(E))
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_chain_f32: workspace %zu < %zu bytes",
                     workspace_bytes, to_chain_workspace_bytes(E));
  const void* p16[] = {A, B, workspace};
  for (const void* p : p16)
    if (!aligned(p, 16)) return set_error(TO_ERR_ALIGNMENT, "to_chain_f32: operands must be 16-byte aligned");
  if (!aligned(R, 4) || !aligned(C, 4) || (T && !aligned(T, 4)))
    return set_error(TO_ERR_ALIGNMENT, "to_chain_f32: misaligned output");
  int st = TO_OK;
  EncodeTiled enc = encode_fn(&st);
  if (!enc) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long n = (long long)E * E * E * E;
  float* ws = static_cast<float*>(workspace);
  float *Ahi = ws, *Alo = ws + n, *Bhi = ws + 2 * n, *Blo = ws + 3 * n;
  int dev = 0;
  const int sms = device_sm_count(&dev);
  if (sms <= 0) return -sms;
  tf32_split_kernel<<<4 * sms, 256, 0, s>>>(A, Ahi, Alo, n);
  tf32_split_regroup_b_kernel<<<unsigned(E * E * (E / 32) * (E / 32)), dim3(32, 8), 0, s>>>(
      B, Bhi, Blo, E);
  TO_CUDA_TRY(cudaGetLastError());
  TO_CUDA_TRY(cudaMemsetAsync(R, 0, sizeof(float) * E * E, s));

  const cuuint64_t e = cuuint64_t(E), fb = 4;
  // A[a][e][c][f] viewed as (f, c, a, e)
  const cuuint64_t adims[4] = {e, e, e, e};
  const cuuint64_t astr[3] = {e * fb, e * e * e * fb, e * e * fb};
  const cuuint32_t abox[4] = {32, cuuint32_t(E), cuuint32_t(kTileM / E), 1};
  // B'[b][d][e][f] viewed as (K = (e,f), N = (b,d))
  const cuuint64_t bdims[2] = {e * e, e * e};
  const cuuint64_t bstr[1] = {e * e * fb};
  const cuuint32_t bbox[2] = {32, cuuint32_t(kTileN)};
  CUtensorMap mAhi, mAlo, mBhi, mBlo;
  if ((st = make_map(enc, &mAhi, Ahi, 4, adims, astr, abox))) return st;
  if ((st = make_map(enc, &mAlo, Alo, 4, adims, astr, abox))) return st;
  if ((st = make_map(enc, &mBhi, Bhi, 2, bdims, bstr, bbox))) return st;
  if ((st = make_map(enc, &mBlo, Blo, 2, bdims, bstr, bbox))) return st;

  ChainArgs args{C, R, T};
  const dim3 grid(unsigned(E * E / kTileN), unsigned(E * E / kTileM));
  if (E == 32) st = launch_chain<32>(grid, mAhi, mAlo, mBhi, mBlo, args, s);
  else if (E == 64) st = launch_chain<64>(grid, mAhi, mAlo, mBhi, mBlo, args, s);
  else st = launch_chain<128>(grid, mAhi, mAlo, mBhi, mBlo, args, s);
  if (st) return st;
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

double to_chain_flops(int32_t E) {
  const double e = E;
  return 2.0 * e * e * e * e * e * e + 2.0 * e * e * e * e;
}

int to_gemm_tf32x3(int64_t Mp, int64_t Np, int64_t Kp, const float* Ahi, const float* Alo,
                   const float* Bhi, const float* Blo, float* C, void* stream) {
  if (Mp <= 0 || Np <= 0 || Kp <= 0 || Mp % kTileM || Np % kTileN || Kp % kTileK)
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "to_gemm_tf32x3: sizes %lld x %lld x %lld must be positive multiples of "
                     "128 x 256 x 32", (long long)Mp, (long long)Np, (long long)Kp);
  if ((Mp / kTileM) * (Np / kTileN) > (1ll << 30) || Kp / kTileK > (1ll << 30))
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_gemm_tf32x3: M x N or K too large");
  const void* ptrs[] = {Ahi, Alo, Bhi, Blo, C};
  for (const void* p : ptrs) {
    if (!p) return set_error(TO_ERR_INVALID_ARGUMENT, "to_gemm_tf32x3: null pointer");
    if (!aligned(p, 16)) return set_error(TO_ERR_ALIGNMENT, "to_gemm_tf32x3: operands must be 16-byte aligned");
  }
  int st = TO_OK;
  EncodeTiled enc = encode_fn(&st);
  if (!enc) return st;
  const cuuint64_t fb = 4;
  const cuuint64_t adims[2] = {cuuint64_t(Kp), cuuint64_t(Mp)};
  const cuuint64_t astr[1] = {cuuint64_t(Kp) * fb};
  const cuuint32_t abox[2] = {cuuint32_t(kTileK), cuuint32_t(kTileM)};
  const cuuint64_t bdims[2] = {cuuint64_t(Kp), cuuint64_t(Np)};
  const cuuint32_t bbox[2] = {cuuint32_t(kTileK), cuuint32_t(kTileN)};
  CUtensorMap mAhi, mAlo, mBhi, mBlo;
  if ((st = make_map(enc, &mAhi, Ahi, 2, adims, astr, abox))) return st;
  if ((st = make_map(enc, &mAlo, Alo, 2, adims, astr, abox))) return st;
  if ((st = make_map(enc, &mBhi, Bhi, 2, bdims, astr, bbox))) return st;
  if ((st = make_map(enc, &mBlo, Blo, 2, bdims, astr, bbox))) return st;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(gemm_tcgen05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kSmemBytes));
  });
  TO_CUDA_TRY(attr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long tiles_n = Np / kTileN, tiles = (Mp / kTileM) * tiles_n;
  const int k_iters = static_cast<int>(Kp / kTileK);
  int dev = 0;
  const int sms = device_sm_count(&dev);
  const long long tail = sms > 0 ? tiles % sms : 0;
  GemmArgs args{C, (long long)Np, k_iters, static_cast<int>(tiles_n), static_cast<int>(tiles), 1};
  if (tail > 0 && 2 * tail <= sms && k_iters >= 2) {
    // split the partial last wave in K; zero the rows of tiles it adds into
    args.split = 2;
    args.full_tiles = static_cast<int>(tiles - tail);
    const long long row0 = (args.full_tiles / tiles_n) * kTileM;
    TO_CUDA_TRY(cudaMemsetAsync(C + row0 * Np, 0, size_t((Mp - row0) * Np) * sizeof(float), s));
  }
  const long long units = args.full_tiles + (tiles - args.full_tiles) * args.split;
  gemm_tcgen05_kernel<<<unsigned(units), kThreads, kSmemBytes, s>>>(mAhi, mAlo, mBhi, mBlo, args);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // extern "C"
