// sem3d_elastic.cuh -- device side of the fused SEM 3D isotropic-elastic
// stiffness operator (the LevelGraph SEM3D pipeline of the reference,
// benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp:247-351), written for
// sm_100a as ONE kernel that keeps every intermediate on chip.
//
// Thread mapping ("k-column"): a CTA processes EB elements per batch with
// EB*N*N threads; thread (le, j, i) owns the N points (k = 0..N-1, j, i) of
// element le.  Consequences:
//   * every per-point array access at fixed k is 25 consecutive words per
//     element across consecutive threads -> coalesced streaming loads;
//   * the gamma-direction contractions (sum over k) need only the thread's own
//     column, so they run from registers against the operator coefficients in
//     the kernel-parameter constant bank (compile-time indices);
//   * the xi / eta contractions read the neighbours' columns from shared
//     memory laid out [quantity][k][thread]: at fixed k every thread writes
//     word (k*NT + tid), and the row / column reads hit distinct banks.
// Per batch: gather u (through ibool) -> smem; barrier; per k: 9 gradients,
// chain rule + stress + 9 fluxes (Integrand9); xi/eta fluxes -> smem, gamma
// fluxes stay in registers; barrier; per k: 9 divergences + weighted sum
// (WeightedSum) -> store or scatter-add.  The next batch's per-point arrays are
// prefetched into L2 with cp.async.bulk.prefetch so HBM streaming does not
// depend on how many loads the threads keep in flight.
#pragma once

#include <cstdint>

namespace to_b200 {

template <typename T, int N>
struct Sem3dOps {
  T H[N][N];   // H(i,p): d/dxi at node i from node p
  T Hw[N][N];  // Hw(q,i): weighted transpose, summed over q
  T w[N];      // GLL weights
};

// Per-point array order inside Sem3dArgs::m.  J[r][d] = m[3r+d].
enum : int { kXIX = 0, kJAC = 9, kL2M = 10, kMU = 11, kNumPointArrays = 12 };

template <typename T, int N>
struct Sem3dArgs {
  const T* u[3];
  T* f[3];
  const int32_t* ibool;
  const T* m[kNumPointArrays];
  long long nelem;
  int prefetch;  // 1 if every streamed array is 16-byte aligned
  Sem3dOps<T, N> ops;
  // assembled mode, optional: every gathered u value is multiplied by
  // 1 / sqrt(*u_norm2) (computed and applied in double, as to_scale3 does)
  const double* u_norm2;
};

// The factor of Sem3dArgs::u_norm2 (1 without it).
__device__ __forceinline__ double sem_u_factor(const double* u_norm2) {
  return u_norm2 ? 1.0 / sqrt(*u_norm2) : 1.0;
}
// x times the factor, rounded once to T (x itself when there is no factor).
template <typename T>
__device__ __forceinline__ T sem_u_scaled(T x, double s, bool scaled) {
  return scaled ? static_cast<T>(static_cast<double>(x) * s) : x;
}

// Issue an L2 bulk prefetch of `bytes` (rounded down to 16) at `p`.
__device__ __forceinline__ void l2_prefetch(const void* p, long long bytes) {
  unsigned int b = static_cast<unsigned int>(bytes) & ~15u;
  if (b == 0) return;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(b)
               : "memory");
}

// The reference's shared physics, restated (bench_sem3d_levelgraph.cpp:126-154):
// ds[c][d] = dxi[c] J[0][d] + det[c] J[1][d] + dgm[c] J[2][d];
// sigma = mu (ds + ds^T) + (l2m - 2 mu) tr(ds) I;  F^r_c = jac sum_d sigma[c][d] J[r][d].
template <typename T>
__device__ __forceinline__ void sem_integrand9(const T dxi[3], const T det[3],
                                               const T dgm[3], const T J[3][3],
                                               T l2m, T mu, T jac, T F[3][3]) {
  T ds[3][3];
#pragma unroll
  for (int c = 0; c < 3; ++c)
#pragma unroll
    for (int d = 0; d < 3; ++d)
      ds[c][d] = dxi[c] * J[0][d] + det[c] * J[1][d] + dgm[c] * J[2][d];
  const T lambda = l2m - T(2) * mu;
  const T tr = ds[0][0] + ds[1][1] + ds[2][2];
  T s[3][3];
#pragma unroll
  for (int c = 0; c < 3; ++c)
#pragma unroll
    for (int d = 0; d < 3; ++d) s[c][d] = mu * (ds[c][d] + ds[d][c]);
#pragma unroll
  for (int c = 0; c < 3; ++c) s[c][c] += lambda * tr;
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c)
      F[r][c] = jac * (s[c][0] * J[r][0] + s[c][1] * J[r][1] + s[c][2] * J[r][2]);
}

template <typename T, int N, int EB, bool ASSEMBLED>
__global__ void __launch_bounds__(EB* N* N, 1)
    sem3d_elastic_kernel(const __grid_constant__ Sem3dArgs<T, N> a) {
  constexpr int NN = N * N;
  constexpr int P = N * N * N;
  constexpr int NT = EB * NN;  // threads per CTA = points per k-slice of a batch
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* su = reinterpret_cast<T*>(smem_raw);  // [3][N][NT]   u_c(k, thread)
  T* sF = su + 3 * N * NT;                 // [6][N][NT]   F^xi_c, F^eta_c

  const int tid = threadIdx.x;
  const int le = tid / NN;
  const int ji = tid - le * NN;
  const int j = ji / N;
  const int i = ji - j * N;
  const int row = le * NN + j * N;  // start of (le, ., j, .) row inside a k-slice
  const int col = le * NN + i;      // start of (le, ., ., i) column inside a k-slice

  // The gamma-direction coefficients are indexed with compile-time (k, p) and
  // stay in the kernel-parameter constant bank.  The xi / eta rows depend on
  // the thread's (i, j); they are re-read from shared memory at the start of
  // each phase so only the rows that phase needs occupy registers.
  T* sops = sF + 6 * N * NT;  // [H: N*N][Hw: N*N]
  int* snode = reinterpret_cast<int*>(sops + 2 * NN);  // [N][NT] global node ids
  for (int t = tid; t < 2 * NN; t += NT) sops[t] = t < NN ? (&a.ops.H[0][0])[t] : (&a.ops.Hw[0][0])[t - NN];
  const T wi = a.ops.w[i];
  const T wj = a.ops.w[j];
  const T wij = wi * wj;
  __syncthreads();

  const long long nbatch = (a.nelem + EB - 1) / EB;
  for (long long b = blockIdx.x; b < nbatch; b += gridDim.x) {
    if (a.prefetch && tid == 0) {
      const long long nb = b + gridDim.x;
      if (nb < nbatch) {
        const long long e0 = nb * EB;
        const long long ne = (a.nelem - e0 < EB) ? (a.nelem - e0) : EB;
        const long long off = e0 * P;
        const long long bytes = ne * P * (long long)sizeof(T);
#pragma unroll
        for (int q = 0; q < kNumPointArrays; ++q) l2_prefetch(a.m[q] + off, bytes);
        if (ASSEMBLED) {
          l2_prefetch(a.ibool + off, ne * P * 4);
        } else {
#pragma unroll
          for (int c = 0; c < 3; ++c) l2_prefetch(a.u[c] + off, bytes);
        }
      }
    }

    const long long e = b * EB + le;
    const bool valid = e < a.nelem;
    const long long base = e * P + ji;  // point (k=0, j, i); +k*NN per level

    // ---- stage u: gather (assembled) or stream (element-local) ----
    const bool uscaled = ASSEMBLED && a.u_norm2 != nullptr;
    const double usf = uscaled ? sem_u_factor(a.u_norm2) : 1.0;
    T uc[3][N];
#pragma unroll
    for (int k = 0; k < N; ++k) {
      if (ASSEMBLED) {
        const int node = valid ? __ldg(a.ibool + base + k * NN) : 0;
        snode[k * NT + tid] = node;
#pragma unroll
        for (int c = 0; c < 3; ++c)
          uc[c][k] = valid ? sem_u_scaled(__ldg(a.u[c] + node), usf, uscaled) : T(0);
      } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
          uc[c][k] = valid ? __ldg(a.u[c] + base + k * NN) : T(0);
      }
#pragma unroll
      for (int c = 0; c < 3; ++c) su[(c * N + k) * NT + tid] = uc[c][k];
    }
    __syncthreads();

    // ---- gradients + Integrand9, one point of the column at a time ----
    T Hi[N], Hj[N];
#pragma unroll
    for (int p = 0; p < N; ++p) {
      Hi[p] = sops[i * N + p];
      Hj[p] = sops[j * N + p];
    }
    T Fg[3][N];
#pragma unroll
    for (int k = 0; k < N; ++k) {
      T dxi[3], det[3], dgm[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const T* s = su + (c * N + k) * NT;
        T ax = T(0), ae = T(0), ag = T(0);
#pragma unroll
        for (int p = 0; p < N; ++p) {
          ax += Hi[p] * s[row + p];
          ae += Hj[p] * s[col + p * N];
          ag += a.ops.H[k][p] * uc[c][p];
        }
        dxi[c] = ax;
        det[c] = ae;
        dgm[c] = ag;
      }
      T J[3][3], jac = T(0), l2m = T(0), mu = T(0);
      const long long pidx = base + k * NN;
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int d = 0; d < 3; ++d) J[r][d] = valid ? __ldg(a.m[kXIX + 3 * r + d] + pidx) : T(0);
      if (valid) {
        jac = __ldg(a.m[kJAC] + pidx);
        l2m = __ldg(a.m[kL2M] + pidx);
        mu = __ldg(a.m[kMU] + pidx);
      }
      T F[3][3];
      sem_integrand9(dxi, det, dgm, J, l2m, mu, jac, F);
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        sF[(c * N + k) * NT + tid] = F[0][c];
        sF[((3 + c) * N + k) * NT + tid] = F[1][c];
        Fg[c][k] = F[2][c];
      }
    }
    __syncthreads();

    // ---- divergences + WeightedSum, then store / scatter-add ----
    T Wi[N], Wj[N];
#pragma unroll
    for (int q = 0; q < N; ++q) {
      Wi[q] = sops[NN + q * N + i];
      Wj[q] = sops[NN + q * N + j];
    }
#pragma unroll
    for (int k = 0; k < N; ++k) {
      const T wk = a.ops.w[k];
      const T wjk = wj * wk;
      const T wik = wi * wk;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const T* sx = sF + (c * N + k) * NT;
        const T* se = sF + ((3 + c) * N + k) * NT;
        T tx = T(0), te = T(0), tg = T(0);
#pragma unroll
        for (int q = 0; q < N; ++q) {
          tx += Wi[q] * sx[row + q];
          te += Wj[q] * se[col + q * N];
          tg += a.ops.Hw[q][k] * Fg[c][q];
        }
        const T fc = wjk * tx + wik * te + wij * tg;
        if (valid) {
          if (ASSEMBLED)
            atomicAdd(a.f[c] + snode[k * NT + tid], fc);
          else
            a.f[c][base + k * NN] = fc;
        }
      }
    }
    __syncthreads();  // su / sF are rewritten by the next batch
  }
}

}  // namespace to_b200
