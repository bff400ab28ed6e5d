// sem3d_elastic_tma.cuh -- the TMA-staged fused SEM 3D elastic kernel (sm_100a).
//
// Same pipeline and thread mapping as sem3d_elastic.cuh (thread (le, j, i)
// owns the k-column of element le), with the data movement redesigned:
//
//  * every per-point array of a batch of EB elements (12 metric/material
//    arrays, plus ibool or the element-local u) is ONE contiguous run of
//    EB*N^3 values in global memory; one elected thread moves each run into
//    shared memory with a 1D bulk copy (cp.async.bulk, no multicast) that
//    completes on an mbarrier, so the compute threads read it with plain LDS
//    at compile-time offsets -- no address arithmetic, no registers held for
//    loads in flight;
//  * the runs of the batch two steps ahead are prefetched into L2 with
//    cp.async.bulk.prefetch.L2, which keeps the HBM stream independent of the
//    compute phases; the bulk copy of the next batch is issued as soon as the
//    current batch's metric reads are done (after the gradient/Integrand9
//    phase) and lands from L2 during the divergence phase;
//  * points are processed in k-pairs (k, k+1) with packed f32x2 FMAs
//    (__ffma2_rn and friends) for the contractions and the whole Integrand9
//    physics, the odd last k with scalar instructions;
//  * every mbarrier wait is bounded; a CTA whose data never arrives records
//    TO_ERR_TIMEOUT in the device status word and leaves.
//
// Requirements (checked on the host, else the LDG kernel runs): every staged
// array 16-byte aligned and EB a multiple of 4 (so each batch starts on a
// 16-byte boundary: 4 elements * 125 floats = 2000 bytes).
#pragma once

#include <cstdint>
#include <type_traits>

#include "sem3d_elastic.cuh"
#include "sm100_primitives.cuh"

namespace to_b200 {

// The including translation unit defines the device status word
// `__device__ int g_to_device_status` (0 ok, else a to_status code) before
// including this header.

template <typename T, int L>
struct LaneT {
  using type = V2<T>;
};
template <typename T>
struct LaneT<T, 1> {
  using type = T;
};

template <typename T>
__device__ __forceinline__ T splat(T x, T*) {
  return x;
}
template <typename T>
__device__ __forceinline__ V2<T> splat(T x, V2<T>*) {
  return mk2(x, x);
}
template <typename V, typename T>
__device__ __forceinline__ V splat_as(T x) {
  return splat(x, static_cast<V*>(nullptr));
}

// Load lane values: L == 2 -> (p0[0], p1[0]) as a pair; L == 1 -> p0[0].
template <int L, typename T>
__device__ __forceinline__ typename LaneT<T, L>::type ld_lanes(const T* p0, const T* p1) {
  if constexpr (L == 2)
    return mk2(p0[0], p1[0]);
  else
    return p0[0];
}

// Integrand9 on L lanes (bench_sem3d_levelgraph.cpp:126-154, 214-231):
// ds = chain_rule(dxi, det, dgm, J); sigma = mu (ds + ds^T) + (l2m - 2 mu) tr I;
// F[r][c] = jac * sum_d sigma[c][d] J[r][d].
template <typename V, typename T>
__device__ __forceinline__ void integrand9_lanes(const V dxi[3], const V det[3], const V dgm[3],
                                                 const V J[3][3], V l2m, V mu, V jac,
                                                 V F[3][3]) {
  V ds[3][3];
#pragma unroll
  for (int c = 0; c < 3; ++c)
#pragma unroll
    for (int d = 0; d < 3; ++d)
      ds[c][d] = fma2(dgm[c], J[2][d], fma2(det[c], J[1][d], mul2(dxi[c], J[0][d])));
  const V lambda = fma2(mu, splat_as<V>(T(-2)), l2m);
  const V tr = add2(add2(ds[0][0], ds[1][1]), ds[2][2]);
  const V lt = mul2(lambda, tr);
  V s[3][3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    s[c][c] = fma2(mu, add2(ds[c][c], ds[c][c]), lt);
#pragma unroll
    for (int d = c + 1; d < 3; ++d) {
      s[c][d] = mul2(mu, add2(ds[c][d], ds[d][c]));
      s[d][c] = s[c][d];
    }
  }
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      F[r][c] = mul2(jac, fma2(s[c][2], J[r][2], fma2(s[c][1], J[r][1], mul2(s[c][0], J[r][0]))));
}

template <typename T, int N, int EB, bool ASM>
struct Sem3dTmaLayout {
  static constexpr int NN = N * N, P = NN * N, NT = EB * NN, EP = EB * P;
  static constexpr int kStaged = kNumPointArrays + (ASM ? 1 : 3);
  static constexpr size_t kHeader = 128;  // mbarrier + padding
  static constexpr size_t kStageBytes = size_t(kStaged) * EP * sizeof(T);
  static constexpr size_t kSuBytes = size_t(3) * N * NT * sizeof(T);
  static constexpr size_t kSfBytes = size_t(6) * N * NT * sizeof(T);
  static constexpr size_t kOpsBytes = size_t(2) * NN * sizeof(T);
  static constexpr size_t kTotal = kHeader + kStageBytes + kSuBytes + kSfBytes + kOpsBytes;
};

constexpr uint32_t kMbarMaxPolls = 1u << 22;

template <typename T, int N, int EB, int MINB, bool ASM>
__global__ void __launch_bounds__(EB* N* N, MINB)
    sem3d_elastic_tma_kernel(const __grid_constant__ Sem3dArgs<T, N> a) {
  using LY = Sem3dTmaLayout<T, N, EB, ASM>;
  constexpr int NN = LY::NN, P = LY::P, NT = LY::NT, EP = LY::EP;
  constexpr int kStaged = LY::kStaged;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);
  T* stage = reinterpret_cast<T*>(smem_raw + LY::kHeader);  // [kStaged][EP]
  T* su = stage + size_t(kStaged) * EP;                      // [3][N][NT]
  T* sF = su + 3 * N * NT;                                   // [6][N][NT]
  T* sops = sF + 6 * N * NT;                                 // [H N*N][Hw N*N]
  const int32_t* stage_ib = reinterpret_cast<const int32_t*>(stage + size_t(kNumPointArrays) * EP);

  const int tid = threadIdx.x;
  const int le = tid / NN;
  const int ji = tid - le * NN;
  const int j = ji / N;
  const int i = ji - j * N;
  const int row = le * NN + j * N;
  const int col = le * NN + i;
  const int spt = le * P + ji;  // this thread's point (k = 0) inside a staged array

  const long long nbatch = (a.nelem + EB - 1) / EB;
  const long long G = gridDim.x;

  // One elected thread moves batch `bb` into the stage (or does nothing past the end).
  auto issue_stage = [&](long long bb) {
    const long long e0 = bb * EB;
    const long long ne = (a.nelem - e0 < EB) ? (a.nelem - e0) : EB;
    const uint32_t bytes = static_cast<uint32_t>(ne * P * (long long)sizeof(T)) & ~15u;
    const uint32_t ibytes = static_cast<uint32_t>(ne * P * 4ll) & ~15u;
    const uint32_t total = kNumPointArrays * bytes + (ASM ? ibytes : 3 * bytes);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(bar, total);
#pragma unroll
    for (int q = 0; q < kNumPointArrays; ++q)
      bulk_g2s(stage + size_t(q) * EP, a.m[q] + e0 * P, bytes, bar);
    if (ASM) {
      bulk_g2s(stage + size_t(kNumPointArrays) * EP, a.ibool + e0 * P, ibytes, bar);
    } else {
#pragma unroll
      for (int c = 0; c < 3; ++c)
        bulk_g2s(stage + size_t(kNumPointArrays + c) * EP, a.u[c] + e0 * P, bytes, bar);
    }
  };
  auto prefetch_batch = [&](long long bb) {
    if (bb >= nbatch) return;
    const long long e0 = bb * EB;
    const long long ne = (a.nelem - e0 < EB) ? (a.nelem - e0) : EB;
    const uint32_t bytes = static_cast<uint32_t>(ne * P * (long long)sizeof(T));
#pragma unroll
    for (int q = 0; q < kNumPointArrays; ++q) l2_prefetch_bulk(a.m[q] + e0 * P, bytes);
    if (ASM)
      l2_prefetch_bulk(a.ibool + e0 * P, static_cast<uint32_t>(ne * P * 4ll));
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

  const T wi = a.ops.w[i];
  const T wj = a.ops.w[j];
  const T wij = wi * wj;
  uint32_t parity = 0;

  for (long long b = b0; b < nbatch; b += G) {
    if (tid == 0) prefetch_batch(b + 2 * G);
    const long long e0 = b * EB;
    const long long e = e0 + le;
    const bool valid = e < a.nelem;

    // ---- wait for the stage (bounded); agree CTA-wide on the outcome ----
    const bool ok = mbar_wait_bounded(bar, parity, kMbarMaxPolls);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicExch(&g_to_device_status, int(TO_ERR_TIMEOUT));
      // bounded wait for the copies still in flight before the CTA leaves
      mbar_wait_bounded(bar, parity, kMbarMaxPolls);
      return;
    }
    parity ^= 1u;
    // Tail of the launch: values past the last 16-byte boundary of a run
    // (at most 3 per array) are not moved by the bulk copy; load them here.
    {
      const long long ne = (a.nelem - e0 < EB) ? (a.nelem - e0) : EB;
      const int words = static_cast<int>(ne * P);
      const int bw = static_cast<int>(((ne * P * (long long)sizeof(T)) & ~15ll) / (long long)sizeof(T));
      const int iw = static_cast<int>(((ne * P * 4ll) & ~15ll) / 4);
      if (bw < words || (ASM && iw < words)) {
        for (int t = tid; t < kStaged * 4; t += NT) {
          const int q = t >> 2, w = t & 3;
          if (q < kNumPointArrays) {
            const int x = bw + w;
            if (x < words) stage[size_t(q) * EP + x] = a.m[q][e0 * P + x];
          } else if (ASM) {
            const int x = iw + w;
            if (x < words)
              const_cast<int32_t*>(stage_ib)[x] = a.ibool[e0 * P + x];
          } else {
            const int c = q - kNumPointArrays, x = bw + w;
            if (x < words) stage[size_t(q) * EP + x] = a.u[c][e0 * P + x];
          }
        }
        __syncthreads();
      }
    }

    // ---- stage u: gather through ibool (assembled) or read the staged run ----
    int node[N];
    T dg[3][N];  // gamma-direction gradients, from the thread's own column
    {
      T uc[3][N];
#pragma unroll
      for (int k = 0; k < N; ++k) {
        if (ASM) {
          node[k] = valid ? stage_ib[spt + k * NN] : 0;
#pragma unroll
          for (int c = 0; c < 3; ++c) uc[c][k] = valid ? __ldg(a.u[c] + node[k]) : T(0);
        } else {
          node[k] = 0;
#pragma unroll
          for (int c = 0; c < 3; ++c)
            uc[c][k] = valid ? stage[size_t(kNumPointArrays + c) * EP + spt + k * NN] : T(0);
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) su[(c * N + k) * NT + tid] = uc[c][k];
      }
#pragma unroll
      for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int k = 0; k < N; ++k) {
          T s = T(0);
#pragma unroll
          for (int p = 0; p < N; ++p) s += a.ops.H[k][p] * uc[c][p];
          dg[c][k] = s;
        }
    }
    __syncthreads();

    // ---- gradients + Integrand9 on k-pairs (packed) and the odd last k ----
    T Fg[3][N];
    {
      T Hi[N], Hj[N];
#pragma unroll
      for (int p = 0; p < N; ++p) {
        Hi[p] = sops[i * N + p];
        Hj[p] = sops[j * N + p];
      }
      auto point_block = [&](auto lanes_tag, int k0) {
        constexpr int L = decltype(lanes_tag)::value;
        using V = typename LaneT<T, L>::type;
        const int k1 = (L == 2) ? k0 + 1 : k0;
        V dxi[3], det[3], dgm[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          const T* s0 = su + (c * N + k0) * NT;
          const T* s1 = su + (c * N + k1) * NT;
          V ax = splat_as<V>(T(0)), ae = splat_as<V>(T(0));
#pragma unroll
          for (int p = 0; p < N; ++p) {
            ax = fma2(splat_as<V>(Hi[p]), ld_lanes<L>(s0 + row + p, s1 + row + p), ax);
            ae = fma2(splat_as<V>(Hj[p]), ld_lanes<L>(s0 + col + p * N, s1 + col + p * N), ae);
          }
          dxi[c] = ax;
          det[c] = ae;
          if constexpr (L == 2)
            dgm[c] = mk2(dg[c][k0], dg[c][k1]);
          else
            dgm[c] = dg[c][k0];
        }
        V J[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
          for (int d = 0; d < 3; ++d) {
            const T* q = stage + size_t(kXIX + 3 * r + d) * EP + spt;
            J[r][d] = ld_lanes<L>(q + k0 * NN, q + k1 * NN);
          }
        const T* qj = stage + size_t(kJAC) * EP + spt;
        const T* ql = stage + size_t(kL2M) * EP + spt;
        const T* qm = stage + size_t(kMU) * EP + spt;
        const V jac = ld_lanes<L>(qj + k0 * NN, qj + k1 * NN);
        const V l2m = ld_lanes<L>(ql + k0 * NN, ql + k1 * NN);
        const V mu = ld_lanes<L>(qm + k0 * NN, qm + k1 * NN);
        V F[3][3];
        integrand9_lanes<V, T>(dxi, det, dgm, J, l2m, mu, jac, F);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          if constexpr (L == 2) {
            sF[(c * N + k0) * NT + tid] = F[0][c].v.x;
            sF[(c * N + k1) * NT + tid] = F[0][c].v.y;
            sF[((3 + c) * N + k0) * NT + tid] = F[1][c].v.x;
            sF[((3 + c) * N + k1) * NT + tid] = F[1][c].v.y;
            Fg[c][k0] = F[2][c].v.x;
            Fg[c][k1] = F[2][c].v.y;
          } else {
            sF[(c * N + k0) * NT + tid] = F[0][c];
            sF[((3 + c) * N + k0) * NT + tid] = F[1][c];
            Fg[c][k0] = F[2][c];
          }
        }
      };
#pragma unroll
      for (int kp = 0; kp < N / 2; ++kp) point_block(std::integral_constant<int, 2>{}, 2 * kp);
      if constexpr (N % 2 == 1) point_block(std::integral_constant<int, 1>{}, N - 1);
    }
    __syncthreads();  // stage metric reads and sF writes done

    // the stage is free: move the next batch in while the divergences run
    if (tid == 0 && b + G < nbatch) issue_stage(b + G);

    // ---- divergences + WeightedSum on k-pairs, then store / scatter-add ----
    {
      T Wi[N], Wj[N];
#pragma unroll
      for (int q = 0; q < N; ++q) {
        Wi[q] = sops[NN + q * N + i];
        Wj[q] = sops[NN + q * N + j];
      }
      auto point_block = [&](auto lanes_tag, int k0) {
        constexpr int L = decltype(lanes_tag)::value;
        using V = typename LaneT<T, L>::type;
        const int k1 = (L == 2) ? k0 + 1 : k0;
        V wjk, wik;
        if constexpr (L == 2) {
          wjk = mk2(wj * a.ops.w[k0], wj * a.ops.w[k1]);
          wik = mk2(wi * a.ops.w[k0], wi * a.ops.w[k1]);
        } else {
          wjk = wj * a.ops.w[k0];
          wik = wi * a.ops.w[k0];
        }
        const V wijv = splat_as<V>(wij);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          const T* x0 = sF + (c * N + k0) * NT;
          const T* x1 = sF + (c * N + k1) * NT;
          const T* y0 = sF + ((3 + c) * N + k0) * NT;
          const T* y1 = sF + ((3 + c) * N + k1) * NT;
          V tx = splat_as<V>(T(0)), te = splat_as<V>(T(0));
#pragma unroll
          for (int q = 0; q < N; ++q) {
            tx = fma2(splat_as<V>(Wi[q]), ld_lanes<L>(x0 + row + q, x1 + row + q), tx);
            te = fma2(splat_as<V>(Wj[q]), ld_lanes<L>(y0 + col + q * N, y1 + col + q * N), te);
          }
          T tg0 = T(0), tg1 = T(0);
#pragma unroll
          for (int q = 0; q < N; ++q) {
            tg0 += a.ops.Hw[q][k0] * Fg[c][q];
            if (L == 2) tg1 += a.ops.Hw[q][k1] * Fg[c][q];
          }
          V tg;
          if constexpr (L == 2)
            tg = mk2(tg0, tg1);
          else
            tg = tg0;
          const V fc = fma2(wijv, tg, fma2(wik, te, mul2(wjk, tx)));
          T f0, f1 = T(0);
          if constexpr (L == 2) {
            f0 = fc.v.x;
            f1 = fc.v.y;
          } else {
            f0 = fc;
          }
          if (valid) {
            if (ASM) {
              atomicAdd(a.f[c] + node[k0], f0);
              if (L == 2) atomicAdd(a.f[c] + node[k1], f1);
            } else {
              const long long base = e * P + ji;
              a.f[c][base + k0 * NN] = f0;
              if (L == 2) a.f[c][base + k1 * NN] = f1;
            }
          }
        }
      };
#pragma unroll
      for (int kp = 0; kp < N / 2; ++kp) point_block(std::integral_constant<int, 2>{}, 2 * kp);
      if constexpr (N % 2 == 1) point_block(std::integral_constant<int, 1>{}, N - 1);
    }
    __syncthreads();  // su / sF are rewritten by the next batch
  }
}

}  // namespace to_b200
