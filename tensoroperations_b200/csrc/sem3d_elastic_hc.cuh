// sem3d_elastic_hc.cuh -- "half-column" line-owner SEM 3D elastic kernel for
// NGLL 8 (f64: config 5; f32: the reference's N=8 element-local size).
//
// The NGLL-8 line-owner kernel (sem3d_elastic_lo.cuh) gives each thread a
// whole k-column (8 points) and both a xi-row and an eta-row; in fp64 that is
// 255 registers and 8 resident warps per SM, and the kernel stalls on the
// global loads of the per-point geometry.  Here each column has TWO owners,
// one per half (points k = 4h .. 4h+3), and each thread owns ONE line:
//
//   thread (le, r), r = 0..127:  h = bit 5 of r (warp-uniform),
//                                column c = (r & 31) | (r >> 6) << 5,
//                                j = c / 8, i = c % 8;
//   column-half owner  (le, j, i, h): gathers u, evaluates Integrand9 and
//                      scatters f at its four points;
//   line owner         h = 0: the xi-row (k = i, j);  h = 1: the eta-row
//                      (k = j, i) -- each warp takes one branch, so the two
//                      roles never diverge inside a warp.
//
// The gamma contractions need the whole column: the column halves meet in a
// third shared buffer G (u in A, the gamma-fluxes in B2), read during the
// phases in which G is read-only (B1: gamma-gradients, C1: gamma-divergences),
// so the batch keeps four barriers.  X and E keep the line-owner kernel's
// k-major layout and conflict-free strides (the same lanes meet the same
// words); G is [3][8][NT], one word per point.
#pragma once

#include <cstdint>

#include "sem3d_elastic.cuh"
#include "sem3d_elastic_lo.cuh"
#include "sm100_primitives.cuh"

namespace to_b200 {

template <typename T, int EB>
struct Sem3dHcLayout {
  using LO = Sem3dLoLayout<T, 8, EB>;
  static constexpr int N = 8, NN = 64, P = 512, NT = EB * NN, THREADS = 2 * NT;
  static constexpr int SKX = LO::SKX, SKE = LO::SKE;
  static constexpr size_t kXBytes = LO::kXBytes;
  static constexpr size_t kEBytes = LO::kEBytes;
  static constexpr size_t kGBytes = (size_t(3) * N * NT * sizeof(T) + 15) & ~size_t(15);
  static constexpr size_t kTotal = kXBytes + kEBytes + kGBytes;
};

// PIPE: the next point's geometry is loaded before the current point is
// computed, so its twelve loads are in flight during that point's physics and
// ahead of its shared-memory stores (which the compiler may not move loads
// through generic pointers across).
// SCALE: u is read times 1 / sqrt(*a.u_norm2) (assembled); thread 0 computes
// the factor once into shared memory, so the batches only add a broadcast
// load and one multiply per gathered value.
// IBPIPE (assembled): the node ids of this thread's points in its NEXT batch are
// loaded during phases C1 and C2, so phase A's u gathers issue at once instead
// of after an ibool round trip.
template <typename T, int EB, int MINB, bool ASM, bool PIPE = false, bool SCALE = false,
          bool IBPIPE = false, bool UPIPE = false, bool GEARLY = false>
__global__ void __launch_bounds__(EB * 128, MINB)
    sem3d_elastic_hc_kernel(const __grid_constant__ Sem3dArgs<T, 8> a) {
  using LY = Sem3dHcLayout<T, EB>;
  constexpr int N = 8, H = 4, NN = 64, P = 512, NT = LY::NT;
  constexpr int SKX = LY::SKX, SKE = LY::SKE;
  constexpr int CX = N * SKX, CE = N * SKE;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* RX = reinterpret_cast<T*>(smem_raw);
  T* RE = reinterpret_cast<T*>(smem_raw + LY::kXBytes);
  T* RG = reinterpret_cast<T*>(smem_raw + LY::kXBytes + LY::kEBytes);  // [3][N][NT]

  const int tid = threadIdx.x;
  const int le = tid >> 7;
  const int r = tid & 127;
  const int h = (r >> 5) & 1;
  const int col = (r & 31) | ((r >> 6) << 5);
  const int ra = col >> 3;  // j of the column; the xi-row's j; the eta-row's k
  const int rb = col & 7;   // i of the column; the xi-row's k; the eta-row's i
  const int cw = le * NN + col;                // the column's word at each k
  const int lx = rb * SKX + le * NN + ra * N;  // xi-row (k=rb, j=ra): + i
  const int ly = ra * SKE + le * NN + rb;      // eta-row (k=ra, i=rb): + N j
  const int k0 = H * h;

  const long long nbatch = (a.nelem + EB - 1) / EB;
  const long long G = gridDim.x;

  // a.prefetch: how many of this CTA's batches ahead the L2 prefetch runs (0:
  // none, the default -- see launch_hc)
  const int pf_dist = a.prefetch;
  auto prefetch_batch = [&](long long bb) {
    if (bb >= nbatch) return;
    const long long e0 = bb * EB;
    const long long ne = (a.nelem - e0 < EB) ? (a.nelem - e0) : EB;
    const uint32_t bytes = static_cast<uint32_t>(ne * P * sizeof(T)) & ~15u;
    if (!pf_dist || bytes == 0) return;
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
  __shared__ double s_ufac;
  if constexpr (SCALE) {
    if (tid == 0) s_ufac = sem_u_factor(a.u_norm2);
    __syncthreads();
  }
  if (tid == 0)
    for (int d = 0; d < pf_dist; ++d) prefetch_batch(blockIdx.x + d * G);
  int node_n[IBPIPE ? H : 1];
  auto load_nodes = [&](long long bb) {
    if constexpr (IBPIPE) {
      const long long en = bb * EB + le;
      const bool vn = bb < nbatch && en < a.nelem;
#pragma unroll
      for (int kk = 0; kk < H; ++kk) node_n[kk] = vn ? __ldg(a.ibool + en * P + col + (k0 + kk) * NN) : 0;
    }
  };
  load_nodes(blockIdx.x);
  // UPIPE (with IBPIPE): the next batch's u values gathered at the start of C2
  T uc_n[UPIPE ? 3 : 1][UPIPE ? H : 1];
  auto gather_u = [&](long long bb) {
    if constexpr (UPIPE) {
      const long long en = bb * EB + le;
      const bool vn = bb < nbatch && en < a.nelem;
#pragma unroll
      for (int kk = 0; kk < H; ++kk)
#pragma unroll
        for (int c = 0; c < 3; ++c)
          uc_n[c][kk] = vn ? sem_u_scaled(__ldg(a.u[c] + node_n[kk]), SCALE ? s_ufac : 1.0, SCALE)
                           : T(0);
    }
  };
  gather_u(blockIdx.x);

  for (long long b = blockIdx.x; b < nbatch; b += G) {
    if (tid == 0) prefetch_batch(b + pf_dist * G);
    const long long e = b * EB + le;
    const bool valid = e < a.nelem;
    const long long base = e * P + col;  // point (k=0, j, i): + k*NN

    // ---- A: the column half's u -> X, E, G ----
    int node[H];
    {
      T uc[3][H];
#pragma unroll
      for (int kk = 0; kk < H; ++kk) {
        const long long pidx = base + (k0 + kk) * NN;
        if constexpr (ASM && IBPIPE) {
          node[kk] = node_n[kk];
        } else if constexpr (ASM) {
          node[kk] = valid ? __ldg(a.ibool + pidx) : 0;
        } else {
          node[kk] = 0;
        }
      }
#pragma unroll
      for (int kk = 0; kk < H; ++kk)
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          if constexpr (ASM && UPIPE)
            uc[c][kk] = uc_n[c][kk];
          else if constexpr (ASM)
            uc[c][kk] = valid ? sem_u_scaled(__ldg(a.u[c] + node[kk]), SCALE ? s_ufac : 1.0, SCALE)
                              : T(0);
          else
            uc[c][kk] = valid ? __ldcs(a.u[c] + base + (k0 + kk) * NN) : T(0);
        }
#pragma unroll
      for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int kk = 0; kk < H; ++kk) {
          const int k = k0 + kk;
          RX[c * CX + k * SKX + cw] = uc[c][kk];
          RE[c * CE + k * SKE + cw] = uc[c][kk];
          RG[(c * N + k) * NT + cw] = uc[c][kk];
        }
    }
    __syncthreads();

    T Jn[3][3], jacn = T(0), l2mn = T(0), mun = T(0);  // the next point's (PIPE)
    auto load_geom = [&](int kk, T (&Jd)[3][3], T& jd, T& ld, T& md) {
      const long long pidx = base + (k0 + kk) * NN;
#pragma unroll
      for (int rr = 0; rr < 3; ++rr)
#pragma unroll
        for (int d = 0; d < 3; ++d) Jd[rr][d] = valid ? __ldcs(a.m[kXIX + 3 * rr + d] + pidx) : T(0);
      if (valid) {
        jd = __ldcs(a.m[kJAC] + pidx);
        ld = __ldcs(a.m[kL2M] + pidx);
        md = __ldcs(a.m[kMU] + pidx);
      }
    };
    // GEARLY: the first point's geometry requested now, in flight during B1
    if constexpr (PIPE && GEARLY) load_geom(0, Jn, jacn, l2mn, mun);

    // ---- B1: the line's gradients (in place); the half-column's gamma-gradients from G ----
    T dgm[3][H];
    if (h == 0) {
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        T v[N];
#pragma unroll
        for (int p = 0; p < N; ++p) v[p] = RX[c * CX + lx + p];
#pragma unroll
        for (int o = 0; o < N; ++o) {
          T s = T(0);
#pragma unroll
          for (int p = 0; p < N; ++p) s = fma(a.ops.H[o][p], v[p], s);
          RX[c * CX + lx + o] = s;
        }
      }
    } else {
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        T v[N];
#pragma unroll
        for (int p = 0; p < N; ++p) v[p] = RE[c * CE + ly + p * N];
#pragma unroll
        for (int o = 0; o < N; ++o) {
          T s = T(0);
#pragma unroll
          for (int p = 0; p < N; ++p) s = fma(a.ops.H[o][p], v[p], s);
          RE[c * CE + ly + o * N] = s;
        }
      }
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      T v[N];
#pragma unroll
      for (int p = 0; p < N; ++p) v[p] = RG[(c * N + p) * NT + cw];
#pragma unroll
      for (int kk = 0; kk < H; ++kk) {
        T s = T(0);
#pragma unroll
        for (int p = 0; p < N; ++p) s = fma(a.ops.H[k0 + kk][p], v[p], s);
        dgm[c][kk] = s;
      }
    }
    __syncthreads();

    // ---- B2: Integrand9 at the half-column's points; geometry from global ----
    if constexpr (PIPE && !GEARLY) load_geom(0, Jn, jacn, l2mn, mun);
#pragma unroll
    for (int kk = 0; kk < H; ++kk) {
      const int k = k0 + kk;
      T J[3][3], jac = T(0), l2m = T(0), mu = T(0);
      if constexpr (PIPE) {
#pragma unroll
        for (int rr = 0; rr < 3; ++rr)
#pragma unroll
          for (int d = 0; d < 3; ++d) J[rr][d] = Jn[rr][d];
        jac = jacn;
        l2m = l2mn;
        mu = mun;
        if (kk + 1 < H) load_geom(kk + 1, Jn, jacn, l2mn, mun);
      } else {
        load_geom(kk, J, jac, l2m, mu);
      }
      T dxi[3], det[3], dg[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        dxi[c] = RX[c * CX + k * SKX + cw];
        det[c] = RE[c * CE + k * SKE + cw];
        dg[c] = dgm[c][kk];
      }
      T F[3][3];
      sem_integrand9(dxi, det, dg, J, l2m, mu, jac, F);
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        RX[c * CX + k * SKX + cw] = F[0][c];
        RE[c * CE + k * SKE + cw] = F[1][c];
        RG[(c * N + k) * NT + cw] = F[2][c];
      }
    }
    __syncthreads();
    load_nodes(b + G);  // in flight during C1 and C2

    // ---- C1: the line's divergences (in place); the half-column's gamma-divergences from G ----
    if (h == 0) {
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        T v[N];
#pragma unroll
        for (int q = 0; q < N; ++q) v[q] = RX[c * CX + lx + q];
#pragma unroll
        for (int o = 0; o < N; ++o) {
          T s = T(0);
#pragma unroll
          for (int q = 0; q < N; ++q) s = fma(a.ops.Hw[q][o], v[q], s);
          RX[c * CX + lx + o] = s;
        }
      }
    } else {
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        T v[N];
#pragma unroll
        for (int q = 0; q < N; ++q) v[q] = RE[c * CE + ly + q * N];
#pragma unroll
        for (int o = 0; o < N; ++o) {
          T s = T(0);
#pragma unroll
          for (int q = 0; q < N; ++q) s = fma(a.ops.Hw[q][o], v[q], s);
          RE[c * CE + ly + o * N] = s;
        }
      }
    }
    T gdv[3][H];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      T v[N];
#pragma unroll
      for (int q = 0; q < N; ++q) v[q] = RG[(c * N + q) * NT + cw];
#pragma unroll
      for (int kk = 0; kk < H; ++kk) {
        T s = T(0);
#pragma unroll
        for (int q = 0; q < N; ++q) s = fma(a.ops.Hw[q][k0 + kk], v[q], s);
        gdv[c][kk] = s;
      }
    }
    __syncthreads();
    gather_u(b + G);  // in flight during C2

    // ---- C2: WeightedSum at the half-column's points -> scatter-add / store ----
#pragma unroll
    for (int kk = 0; kk < H; ++kk) {
      const int k = k0 + kk;
      const T wjk = wj * a.ops.w[k], wik = wi * a.ops.w[k];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const T tx = RX[c * CX + k * SKX + cw];
        const T te = RE[c * CE + k * SKE + cw];
        const T fc = fma(wij, gdv[c][kk], fma(wik, te, wjk * tx));
        if (valid) {
          if (ASM)
            atomicAdd(a.f[c] + node[kk], fc);
          else
            a.f[c][base + k * NN] = fc;
        }
      }
    }
    // the next batch's A overwrites X, E and G only at this thread's own
    // column points, which no other thread reads before the next barrier
  }
}

}  // namespace to_b200
