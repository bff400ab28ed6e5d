// sem3d_elastic_lo.cuh -- line-owner SEM 3D elastic kernel for any (T, N)
// whose per-point geometry does not fit a shared-memory stage: the fp64 NGLL-8
// configuration (12 arrays x 512 points x 8 B = 49 KB per element).
//
// Same ownership as the f32 NGLL-5 line-owner kernel (sem3d_elastic_v5.cuh):
// thread (le, a, b) is the k-column owner of (j=a, i=b) (u gather, gamma
// contractions in registers, Integrand9, scatter), the xi-row owner of
// (k=b, j=a) and the eta-row owner of (k=a, i=b); exchange buffers X and E are
// k-major with k-strides chosen so that every access of every phase is
// conflict-free for 4- and 8-byte words (NGLL 8: NT + 1 and NT + 8, checked
// exhaustively for EB = 1, 2, 4), and each value overwrites its input in place.
// Differences: the 12 per-point arrays are read straight from global memory by
// the column owner (at fixed k consecutive threads read consecutive words), the
// next batch's arrays are prefetched into L2 by bulk prefetches, and the ibool /
// u gathers of the next batch are pipelined only when they fit the register
// budget (f32 NGLL 5 would; fp64 NGLL 8 does not).  (A variant that parked
// the fp64 gamma values in a third shared region to raise occupancy measured
// slower -- 71.4 vs 66.6 ms per 128^3 power step -- and is kept disabled.)
#pragma once

#include <cstdint>

#include "sem3d_elastic.cuh"
#include "sm100_primitives.cuh"

namespace to_b200 {

template <typename T, int N, int EB>
struct Sem3dLoLayout {
  static constexpr int NN = N * N, P = NN * N, NT = EB * NN;
  static_assert(N == 8 && (EB == 1 || EB == 2 || EB == 4), "strides searched for NGLL 8, EB 1/2/4");
  static constexpr int SKX = NT + 1;
  static constexpr int SKE = NT + 8;
  static constexpr size_t kXBytes = (size_t(3) * N * SKX * sizeof(T) + 15) & ~size_t(15);
  static constexpr size_t kEBytes = (size_t(3) * N * SKE * sizeof(T) + 15) & ~size_t(15);
  // G: gamma-gradients (A -> B2) and gamma-fluxes (B2 -> C2) at the thread's
  // own column positions, out of the register file when T is 8 bytes
  static constexpr bool kParkG = false;  // measured: parking fp64 values here was slower
  static constexpr size_t kGBytes = kParkG ? (size_t(3) * N * NT * sizeof(T) + 15) & ~size_t(15) : 0;
  static constexpr size_t kTotal = kXBytes + kEBytes + kGBytes;
  static constexpr bool kPipe = sizeof(T) * 3 * N <= 64;  // gather pipeline registers
};

template <typename T, int N, int EB, int MINB, bool ASM>
__global__ void __launch_bounds__(EB * N * N, MINB)
    sem3d_elastic_lo_kernel(const __grid_constant__ Sem3dArgs<T, N> a) {
  using LY = Sem3dLoLayout<T, N, EB>;
  constexpr int NN = LY::NN, P = LY::P, NT = LY::NT;
  constexpr int SKX = LY::SKX, SKE = LY::SKE;
  constexpr int CX = N * SKX, CE = N * SKE;
  constexpr bool PIPE = ASM && LY::kPipe;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* RX = reinterpret_cast<T*>(smem_raw);
  T* RE = reinterpret_cast<T*>(smem_raw + LY::kXBytes);
  T* RG = reinterpret_cast<T*>(smem_raw + LY::kXBytes + LY::kEBytes);  // [3][N][NT]
  constexpr bool PARK = LY::kParkG;

  const int tid = threadIdx.x;
  const int le = tid / NN;
  const int ab = tid - le * NN;
  const int ra = ab / N;
  const int rb = ab - ra * N;
  const int lx = rb * SKX + le * NN + ra * N;  // xi-row (k=b, j=a): + i
  const int ly = ra * SKE + le * NN + rb;      // eta-row (k=a, i=b): + N j

  const long long nbatch = (a.nelem + EB - 1) / EB;
  const long long G = gridDim.x;

  auto prefetch_batch = [&](long long bb) {
    if (bb >= nbatch) return;
    const long long e0 = bb * EB;
    const long long ne = (a.nelem - e0 < EB) ? (a.nelem - e0) : EB;
    const uint32_t bytes = static_cast<uint32_t>(ne * P * sizeof(T)) & ~15u;
    if (!a.prefetch || bytes == 0) return;
#pragma unroll
    for (int q = 0; q < kNumPointArrays; ++q) l2_prefetch_bulk(a.m[q] + e0 * P, bytes);
    if (ASM)
      l2_prefetch_bulk(a.ibool + e0 * P, static_cast<uint32_t>(ne * P * 4) & ~15u);
    else
#pragma unroll
      for (int c = 0; c < 3; ++c) l2_prefetch_bulk(a.u[c] + e0 * P, bytes);
  };

  const T wi = a.ops.w[rb];
  const T wj = a.ops.w[ra];
  const T wij = wi * wj;

  int node_n[PIPE ? N : 1];
  T uc_n[PIPE ? 3 : 1][PIPE ? N : 1];
  auto gather = [&](long long bb) {
    if constexpr (PIPE) {
      const long long e = bb * EB + le;
      const bool v = (bb < nbatch) && (e < a.nelem);
      const long long base = e * P + ab;
#pragma unroll
      for (int k = 0; k < N; ++k) node_n[k] = v ? __ldg(a.ibool + base + k * NN) : 0;
      const bool uscaled = ASM && a.u_norm2 != nullptr;
      const double usf = uscaled ? sem_u_factor(a.u_norm2) : 1.0;
#pragma unroll
      for (int k = 0; k < N; ++k)
#pragma unroll
        for (int c = 0; c < 3; ++c)
          uc_n[c][k] = v ? sem_u_scaled(__ldg(a.u[c] + node_n[k]), usf, uscaled) : T(0);
    }
  };
  if (tid == 0) prefetch_batch(blockIdx.x);
  if (PIPE) gather(blockIdx.x);

  for (long long b = blockIdx.x; b < nbatch; b += G) {
    if (tid == 0) prefetch_batch(b + G);
    const long long e = b * EB + le;
    const bool valid = e < a.nelem;
    const long long base = e * P + ab;  // point (k=0, j=a, i=b): + k*NN

    // ---- A: column u -> X, E; gamma-gradients in registers ----
    int node[N];
    T dgm[3][PARK ? 1 : N];
    {
      T uc[3][N];
      if constexpr (PIPE) {
#pragma unroll
        for (int k = 0; k < N; ++k) {
          node[k] = node_n[k];
#pragma unroll
          for (int c = 0; c < 3; ++c) uc[c][k] = uc_n[c][k];
        }
      } else if constexpr (ASM) {
#pragma unroll
        for (int k = 0; k < N; ++k) node[k] = valid ? __ldg(a.ibool + base + k * NN) : 0;
        const bool uscaled = a.u_norm2 != nullptr;
        const double usf = uscaled ? sem_u_factor(a.u_norm2) : 1.0;
#pragma unroll
        for (int k = 0; k < N; ++k)
#pragma unroll
          for (int c = 0; c < 3; ++c)
            uc[c][k] = valid ? sem_u_scaled(__ldg(a.u[c] + node[k]), usf, uscaled) : T(0);
      } else {
#pragma unroll
        for (int k = 0; k < N; ++k) {
          node[k] = 0;
#pragma unroll
          for (int c = 0; c < 3; ++c) uc[c][k] = valid ? __ldcs(a.u[c] + base + k * NN) : T(0);
        }
      }
#pragma unroll
      for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int k = 0; k < N; ++k) {
          RX[c * CX + k * SKX + tid] = uc[c][k];
          RE[c * CE + k * SKE + tid] = uc[c][k];
        }
#pragma unroll
      for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int k = 0; k < N; ++k) {
          T s = T(0);
#pragma unroll
          for (int p = 0; p < N; ++p) s = fma(a.ops.H[k][p], uc[c][p], s);
          if constexpr (PARK)
            RG[(c * N + k) * NT + tid] = s;
          else
            dgm[c][PARK ? 0 : k] = s;
        }
    }
    __syncthreads();

    // ---- B1: row owners -> xi- and eta-gradients of their rows (in place) ----
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      T v[N], w[N];
#pragma unroll
      for (int p = 0; p < N; ++p) {
        v[p] = RX[c * CX + lx + p];
        w[p] = RE[c * CE + ly + p * N];
      }
#pragma unroll
      for (int o = 0; o < N; ++o) {
        T sx = T(0), se = T(0);
#pragma unroll
        for (int p = 0; p < N; ++p) {
          sx = fma(a.ops.H[o][p], v[p], sx);
          se = fma(a.ops.H[o][p], w[p], se);
        }
        RX[c * CX + lx + o] = sx;
        RE[c * CE + ly + o * N] = se;
      }
    }
    __syncthreads();

    // ---- B2: column Integrand9, geometry straight from global memory ----
    T Fg[3][PARK ? 1 : N];
#pragma unroll
    for (int k = 0; k < N; ++k) {
      const long long pidx = base + k * NN;
      T J[3][3], jac = T(0), l2m = T(0), mu = T(0);
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int d = 0; d < 3; ++d) J[r][d] = valid ? __ldcs(a.m[kXIX + 3 * r + d] + pidx) : T(0);
      if (valid) {
        jac = __ldcs(a.m[kJAC] + pidx);
        l2m = __ldcs(a.m[kL2M] + pidx);
        mu = __ldcs(a.m[kMU] + pidx);
      }
      T dxi[3], det[3], dg[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        dxi[c] = RX[c * CX + k * SKX + tid];
        det[c] = RE[c * CE + k * SKE + tid];
        dg[c] = PARK ? RG[(c * N + k) * NT + tid] : dgm[c][PARK ? 0 : k];
      }
      T F[3][3];
      sem_integrand9(dxi, det, dg, J, l2m, mu, jac, F);
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        RX[c * CX + k * SKX + tid] = F[0][c];
        RE[c * CE + k * SKE + tid] = F[1][c];
        if constexpr (PARK)
          RG[(c * N + k) * NT + tid] = F[2][c];  // in place of this point's gamma-gradient
        else
          Fg[c][PARK ? 0 : k] = F[2][c];
      }
    }
    __syncthreads();
    if (PIPE) gather(b + G);

    // ---- C1: row owners -> xi- and eta-divergences (in place) ----
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      T v[N], w[N];
#pragma unroll
      for (int q = 0; q < N; ++q) {
        v[q] = RX[c * CX + lx + q];
        w[q] = RE[c * CE + ly + q * N];
      }
#pragma unroll
      for (int o = 0; o < N; ++o) {
        T sx = T(0), se = T(0);
#pragma unroll
        for (int q = 0; q < N; ++q) {
          sx = fma(a.ops.Hw[q][o], v[q], sx);
          se = fma(a.ops.Hw[q][o], w[q], se);
        }
        RX[c * CX + lx + o] = sx;
        RE[c * CE + ly + o * N] = se;
      }
    }
    __syncthreads();

    // ---- C2: column WeightedSum -> scatter-add / store ----
#pragma unroll
    for (int k = 0; k < N; ++k) {
      const T wjk = wj * a.ops.w[k], wik = wi * a.ops.w[k];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        T g = T(0);
#pragma unroll
        for (int q = 0; q < N; ++q)
          g = fma(a.ops.Hw[q][k], PARK ? RG[(c * N + q) * NT + tid] : Fg[c][PARK ? 0 : q], g);
        const T tx = RX[c * CX + k * SKX + tid];
        const T te = RE[c * CE + k * SKE + tid];
        const T fc = fma(wij, g, fma(wik, te, wjk * tx));
        if (valid) {
          if (ASM)
            atomicAdd(a.f[c] + node[k], fc);
          else
            a.f[c][base + k * NN] = fc;
        }
      }
    }
    // next batch's A writes the column positions this thread just read (its
    // own) and B1 reads rows only after the next barrier
  }
}

}  // namespace to_b200
