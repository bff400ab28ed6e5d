// sem3d_elastic_v3.cuh -- f32 fused SEM 3D elastic kernel, third design.
//
// Thread (le, j, i) owns the k-column of element le, as in the other two
// kernels.  What changed, and why (measured on the 32^3 mesh with ncu):
//
//  * u gathers are software-pipelined.  The ibool indices and the gathered
//    u of batch b+G are loaded while batch b runs its divergence phase, so no
//    warp waits a dependent L2/HBM round trip (ibool -> u) at the top of a
//    batch -- that wait was 38% of all stall cycles in the TMA-only design.
//  * Shared-memory operands of the contractions are stored as point-pair
//    blocks: for the k-pair (k0, k1) a thread's block holds, per component c,
//    the float2 (x(k0), x(k1)): components 0 and 1 in one float4 array and
//    component 2 in a float2 array (no padding -- shared-memory wavefronts
//    are the limiting resource).  One LDS.128 + one LDS.64 then feed packed
//    f32x2 FMAs for two points at once with no register shuffles; the
//    operator coefficients are held as duplicated float2 pairs built once
//    per phase.  The odd last k of NGLL 5 uses float2 + float arrays with
//    scalar FMAs.
//  * The 12 per-point arrays of a batch move global -> shared with one bulk
//    copy each (cp.async.bulk, L2::evict_first: the data is read exactly once)
//    after an L2 bulk prefetch two batches ahead.  ibool is not staged: it is
//    read by the gather pipeline.
//
// Shared memory per CTA (EB elements, NT = 25 EB threads): stage 12 EB 500 B,
// u / F^xi / F^eta blocks 3 x (2 x 24 + 12) B x NT, H and Hw.
#pragma once

#include <cstdint>
#include <type_traits>

#include "sem3d_elastic.cuh"
#include "sem3d_elastic_tma.cuh"
#include "sm100_primitives.cuh"

namespace to_b200 {

template <int N, int EB, bool ASM>
struct Sem3dV3Layout {
  static constexpr int NN = N * N, P = NN * N, NT = EB * NN, EP = EB * P;
  static constexpr int NP = N / 2;        // k-pairs
  static constexpr bool ODD = (N % 2) == 1;
  static constexpr int kStaged = kNumPointArrays + (ASM ? 0 : 3);
  static constexpr size_t kHeader = 128;
  static constexpr size_t kStageBytes = size_t(kStaged) * EP * 4;
  // one "block set" per quantity: for each k-pair a float4 (c0, c1 pairs) and a
  // float2 (c2 pair) per thread; for the odd k a float2 (c0, c1) and a float (c2)
  static constexpr size_t kPairA = size_t(NT) * NP * 16, kPairB = size_t(NT) * NP * 8;
  static constexpr size_t kSingA = ODD ? size_t(NT) * 8 : 0, kSingB = ODD ? size_t(NT) * 4 : 0;
  static constexpr size_t kBlockSetBytes = (kPairA + kPairB + kSingA + kSingB + 15) & ~size_t(15);
  static constexpr size_t kOpsBytes = size_t(2) * NN * 4;
  static constexpr size_t kTotal = kHeader + kStageBytes + 3 * kBlockSetBytes + kOpsBytes;
};

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

template <int N, int EB, int MINB, bool ASM>
__global__ void __launch_bounds__(EB* N* N, MINB)
    sem3d_elastic_v3_kernel(const __grid_constant__ Sem3dArgs<float, N> a) {
  using LY = Sem3dV3Layout<N, EB, ASM>;
  constexpr int NN = LY::NN, P = LY::P, NT = LY::NT, EP = LY::EP, NP = LY::NP;
  constexpr bool ODD = LY::ODD;
  constexpr int kStaged = LY::kStaged;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);
  float* stage = reinterpret_cast<float*>(smem_raw + LY::kHeader);
  unsigned char* blocks = smem_raw + LY::kHeader + LY::kStageBytes;
  // block sets: 0 = u, 1 = F^xi, 2 = F^eta
  struct BlockSet {
    float4* pa;  // [NP][NT]  (c0(k0), c0(k1), c1(k0), c1(k1))
    float2* pb;  // [NP][NT]  (c2(k0), c2(k1))
    float2* sa;  // [NT]      (c0, c1) of the odd k
    float* sb;   // [NT]      c2 of the odd k
  };
  auto block_set = [&](int q) {
    unsigned char* p = blocks + size_t(q) * LY::kBlockSetBytes;
    return BlockSet{reinterpret_cast<float4*>(p), reinterpret_cast<float2*>(p + LY::kPairA),
                    reinterpret_cast<float2*>(p + LY::kPairA + LY::kPairB),
                    reinterpret_cast<float*>(p + LY::kPairA + LY::kPairB + LY::kSingA)};
  };
  const BlockSet BU = block_set(0), BX = block_set(1), BE = block_set(2);
  float* sops = reinterpret_cast<float*>(blocks + 3 * LY::kBlockSetBytes);

  const int tid = threadIdx.x;
  const int le = tid / NN;
  const int ji = tid - le * NN;
  const int j = ji / N;
  const int i = ji - j * N;
  const int row = le * NN + j * N;  // thread index of (le, j, 0)
  const int col = le * NN + i;      // thread index of (le, 0, i)
  const int spt = le * P + ji;

  const long long nbatch = (a.nelem + EB - 1) / EB;
  const long long G = gridDim.x;
  const uint64_t pol_stream = l2_policy_evict_first();

  auto batch_words = [&](long long bb) {
    const long long e0 = bb * EB;
    const long long ne = (a.nelem - e0 < EB) ? (a.nelem - e0) : EB;
    return ne * P;
  };
  auto issue_stage = [&](long long bb) {
    const long long e0 = bb * EB;
    const uint32_t bytes = static_cast<uint32_t>(batch_words(bb) * 4) & ~15u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(bar, kStaged * bytes);
#pragma unroll
    for (int q = 0; q < kNumPointArrays; ++q)
      bulk_g2s_hint(stage + size_t(q) * EP, a.m[q] + e0 * P, bytes, bar, pol_stream);
    if (!ASM) {
#pragma unroll
      for (int c = 0; c < 3; ++c)
        bulk_g2s_hint(stage + size_t(kNumPointArrays + c) * EP, a.u[c] + e0 * P, bytes, bar,
                      pol_stream);
    }
  };
  auto prefetch_batch = [&](long long bb) {
    if (bb >= nbatch) return;
    const long long e0 = bb * EB;
    const uint32_t bytes = static_cast<uint32_t>(batch_words(bb) * 4);
#pragma unroll
    for (int q = 0; q < kNumPointArrays; ++q) l2_prefetch_bulk(a.m[q] + e0 * P, bytes);
    if (ASM)
      l2_prefetch_bulk(a.ibool + e0 * P, bytes);
    else
#pragma unroll
      for (int c = 0; c < 3; ++c) l2_prefetch_bulk(a.u[c] + e0 * P, bytes);
  };

  for (int t = tid; t < 2 * NN; t += NT)
    sops[t] = t < NN ? (&a.ops.H[0][0])[t] : (&a.ops.Hw[0][0])[t - NN];
  const long long b0 = blockIdx.x;
  if (tid == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0 && b0 < nbatch) {
    issue_stage(b0);
    prefetch_batch(b0 + G);
  }

  const float wi = a.ops.w[i];
  const float wj = a.ops.w[j];
  const float wij = wi * wj;
  uint32_t parity = 0;

  // gather pipeline registers: ibool and u of the NEXT batch to run
  int node_n[N];
  float uc_n[3][N];
  auto gather = [&](long long bb) {
    const long long e = bb * EB + le;
    const bool v = (bb < nbatch) && (e < a.nelem);
    const long long base = e * P + ji;
#pragma unroll
    for (int k = 0; k < N; ++k) node_n[k] = v ? __ldg(a.ibool + base + k * NN) : 0;
#pragma unroll
    for (int k = 0; k < N; ++k)
#pragma unroll
      for (int c = 0; c < 3; ++c) uc_n[c][k] = v ? __ldg(a.u[c] + node_n[k]) : 0.f;
  };
  if (ASM) gather(b0);

  for (long long b = b0; b < nbatch; b += G) {
    if (tid == 0) prefetch_batch(b + 2 * G);
    const long long e0 = b * EB;
    const long long e = e0 + le;
    const bool valid = e < a.nelem;

    // ---- A: u of this batch (registers from the gather pipeline) -> blocks ----
    int node[N];
    float2 dgp[3][NP > 0 ? NP : 1];
    float dgs[3];
    if (ASM) {
#pragma unroll
      for (int k = 0; k < N; ++k) node[k] = node_n[k];
    } else {
      // element-local u is part of the stage: wait for it first
#pragma unroll
      for (int k = 0; k < N; ++k) node[k] = 0;
    }
    const bool ok = mbar_wait_bounded(bar, parity, kMbarMaxPolls);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicExch(&g_to_device_status, int(TO_ERR_TIMEOUT));
      mbar_wait_bounded(bar, parity, kMbarMaxPolls);
      return;
    }
    parity ^= 1u;
    {
      // tail of the launch: words past the last 16-byte boundary of each run
      const long long words = batch_words(b);
      const long long bw = ((words * 4) & ~15ll) / 4;
      if (bw < words) {
        for (int t = tid; t < kStaged * 4; t += NT) {
          const int q = t >> 2;
          const long long x = bw + (t & 3);
          if (x < words)
            stage[size_t(q) * EP + x] =
                q < kNumPointArrays ? a.m[q][e0 * P + x] : a.u[q - kNumPointArrays][e0 * P + x];
        }
        __syncthreads();
      }
    }
    {
      float uc[3][N];
#pragma unroll
      for (int k = 0; k < N; ++k)
#pragma unroll
        for (int c = 0; c < 3; ++c)
          uc[c][k] = ASM ? uc_n[c][k]
                         : (valid ? stage[size_t(kNumPointArrays + c) * EP + spt + k * NN] : 0.f);
#pragma unroll
      for (int kp = 0; kp < NP; ++kp) {
        const int k0 = 2 * kp, k1 = k0 + 1;
        BU.pa[kp * NT + tid] = make_float4(uc[0][k0], uc[0][k1], uc[1][k0], uc[1][k1]);
        BU.pb[kp * NT + tid] = f2(uc[2][k0], uc[2][k1]);
      }
      if (ODD) {
        BU.sa[tid] = f2(uc[0][N - 1], uc[1][N - 1]);
        BU.sb[tid] = uc[2][N - 1];
      }
#pragma unroll
      for (int c = 0; c < 3; ++c) {
#pragma unroll
        for (int kp = 0; kp < NP; ++kp) {
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int p = 0; p < N; ++p) {
            s0 += a.ops.H[2 * kp][p] * uc[c][p];
            s1 += a.ops.H[2 * kp + 1][p] * uc[c][p];
          }
          dgp[c][kp] = f2(s0, s1);
        }
        if (ODD) {
          float s = 0.f;
#pragma unroll
          for (int p = 0; p < N; ++p) s += a.ops.H[N - 1][p] * uc[c][p];
          dgs[c] = s;
        }
      }
    }
    __syncthreads();

    // ---- B: gradients + Integrand9 ----
    float Fg[3][N];
    {
      float2 HiHi[N], HjHj[N];
#pragma unroll
      for (int p = 0; p < N; ++p) {
        const float hi = sops[i * N + p], hj = sops[j * N + p];
        HiHi[p] = f2(hi, hi);
        HjHj[p] = f2(hj, hj);
      }
#pragma unroll
      for (int kp = 0; kp < NP; ++kp) {
        const int k0 = 2 * kp, k1 = k0 + 1;
        float2 gx[3] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
        float2 ge[3] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
        for (int p = 0; p < N; ++p) {
          const float4 xl = BU.pa[kp * NT + row + p];
          const float2 xh = BU.pb[kp * NT + row + p];
          const float4 yl = BU.pa[kp * NT + col + p * N];
          const float2 yh = BU.pb[kp * NT + col + p * N];
          gx[0] = ffma2(HiHi[p], f2(xl.x, xl.y), gx[0]);
          gx[1] = ffma2(HiHi[p], f2(xl.z, xl.w), gx[1]);
          gx[2] = ffma2(HiHi[p], xh, gx[2]);
          ge[0] = ffma2(HjHj[p], f2(yl.x, yl.y), ge[0]);
          ge[1] = ffma2(HjHj[p], f2(yl.z, yl.w), ge[1]);
          ge[2] = ffma2(HjHj[p], yh, ge[2]);
        }
        V2<float> dxi[3], det[3], dgm[3], J[3][3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          dxi[c] = {gx[c]};
          det[c] = {ge[c]};
          dgm[c] = {dgp[c][kp]};
        }
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
          for (int d = 0; d < 3; ++d) {
            const float* q = stage + size_t(kXIX + 3 * r + d) * EP + spt;
            J[r][d] = mk2(q[k0 * NN], q[k1 * NN]);
          }
        const float* qj = stage + size_t(kJAC) * EP + spt;
        const float* ql = stage + size_t(kL2M) * EP + spt;
        const float* qm = stage + size_t(kMU) * EP + spt;
        V2<float> F[3][3];
        integrand9_lanes<V2<float>, float>(dxi, det, dgm, J, mk2(ql[k0 * NN], ql[k1 * NN]),
                                           mk2(qm[k0 * NN], qm[k1 * NN]),
                                           mk2(qj[k0 * NN], qj[k1 * NN]), F);
        BX.pa[kp * NT + tid] = make_float4(F[0][0].v.x, F[0][0].v.y, F[0][1].v.x, F[0][1].v.y);
        BX.pb[kp * NT + tid] = F[0][2].v;
        BE.pa[kp * NT + tid] = make_float4(F[1][0].v.x, F[1][0].v.y, F[1][1].v.x, F[1][1].v.y);
        BE.pb[kp * NT + tid] = F[1][2].v;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          Fg[c][k0] = F[2][c].v.x;
          Fg[c][k1] = F[2][c].v.y;
        }
      }
      if (ODD) {
        constexpr int k = N - 1;
        float gx[3] = {0.f, 0.f, 0.f}, ge[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < N; ++p) {
          const float2 x = BU.sa[row + p];
          const float x2 = BU.sb[row + p];
          const float2 y = BU.sa[col + p * N];
          const float y2 = BU.sb[col + p * N];
          gx[0] += HiHi[p].x * x.x;
          gx[1] += HiHi[p].x * x.y;
          gx[2] += HiHi[p].x * x2;
          ge[0] += HjHj[p].x * y.x;
          ge[1] += HjHj[p].x * y.y;
          ge[2] += HjHj[p].x * y2;
        }
        float J[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
          for (int d = 0; d < 3; ++d) J[r][d] = stage[size_t(kXIX + 3 * r + d) * EP + spt + k * NN];
        float F[3][3];
        integrand9_lanes<float, float>(gx, ge, dgs, J, stage[size_t(kL2M) * EP + spt + k * NN],
                                       stage[size_t(kMU) * EP + spt + k * NN],
                                       stage[size_t(kJAC) * EP + spt + k * NN], F);
        BX.sa[tid] = f2(F[0][0], F[0][1]);
        BX.sb[tid] = F[0][2];
        BE.sa[tid] = f2(F[1][0], F[1][1]);
        BE.sb[tid] = F[1][2];
#pragma unroll
        for (int c = 0; c < 3; ++c) Fg[c][k] = F[2][c];
      }
    }
    __syncthreads();  // stage reads and flux writes of this batch are done

    if (tid == 0 && b + G < nbatch) issue_stage(b + G);
    if (ASM) gather(b + G);  // lands while the divergences run

    // ---- C: divergences + WeightedSum, then scatter-add / store ----
    {
      float2 WiWi[N], WjWj[N];
#pragma unroll
      for (int q = 0; q < N; ++q) {
        const float xi = sops[NN + q * N + i], xj = sops[NN + q * N + j];
        WiWi[q] = f2(xi, xi);
        WjWj[q] = f2(xj, xj);
      }
      const long long obase = e * P + ji;
#pragma unroll
      for (int kp = 0; kp < NP; ++kp) {
        const int k0 = 2 * kp, k1 = k0 + 1;
        float2 tx[3] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
        float2 te[3] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
        for (int q = 0; q < N; ++q) {
          const float4 xl = BX.pa[kp * NT + row + q];
          const float2 xh = BX.pb[kp * NT + row + q];
          const float4 yl = BE.pa[kp * NT + col + q * N];
          const float2 yh = BE.pb[kp * NT + col + q * N];
          tx[0] = ffma2(WiWi[q], f2(xl.x, xl.y), tx[0]);
          tx[1] = ffma2(WiWi[q], f2(xl.z, xl.w), tx[1]);
          tx[2] = ffma2(WiWi[q], xh, tx[2]);
          te[0] = ffma2(WjWj[q], f2(yl.x, yl.y), te[0]);
          te[1] = ffma2(WjWj[q], f2(yl.z, yl.w), te[1]);
          te[2] = ffma2(WjWj[q], yh, te[2]);
        }
        const float2 wjk = f2(wj * a.ops.w[k0], wj * a.ops.w[k1]);
        const float2 wik = f2(wi * a.ops.w[k0], wi * a.ops.w[k1]);
        const float2 wijv = f2(wij, wij);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          float g0 = 0.f, g1 = 0.f;
#pragma unroll
          for (int q = 0; q < N; ++q) {
            g0 += a.ops.Hw[q][k0] * Fg[c][q];
            g1 += a.ops.Hw[q][k1] * Fg[c][q];
          }
          const float2 fc = ffma2(wijv, f2(g0, g1), ffma2(wik, te[c], __fmul2_rn(wjk, tx[c])));
          if (valid) {
            if (ASM) {
              atomicAdd(a.f[c] + node[k0], fc.x);
              atomicAdd(a.f[c] + node[k1], fc.y);
            } else {
              a.f[c][obase + k0 * NN] = fc.x;
              a.f[c][obase + k1 * NN] = fc.y;
            }
          }
        }
      }
      if (ODD) {
        constexpr int k = N - 1;
        float tx[3] = {0.f, 0.f, 0.f}, te[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < N; ++q) {
          const float2 x = BX.sa[row + q];
          const float x2 = BX.sb[row + q];
          const float2 y = BE.sa[col + q * N];
          const float y2 = BE.sb[col + q * N];
          tx[0] += WiWi[q].x * x.x;
          tx[1] += WiWi[q].x * x.y;
          tx[2] += WiWi[q].x * x2;
          te[0] += WjWj[q].x * y.x;
          te[1] += WjWj[q].x * y.y;
          te[2] += WjWj[q].x * y2;
        }
        const float wjk = wj * a.ops.w[k], wik = wi * a.ops.w[k];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          float g = 0.f;
#pragma unroll
          for (int q = 0; q < N; ++q) g += a.ops.Hw[q][k] * Fg[c][q];
          const float fc = wij * g + (wik * te[c] + wjk * tx[c]);
          if (valid) {
            if (ASM)
              atomicAdd(a.f[c] + node[k], fc);
            else
              a.f[c][obase + k * NN] = fc;
          }
        }
      }
    }
    __syncthreads();  // blocks are rewritten by the next batch
  }
}

}  // namespace to_b200
