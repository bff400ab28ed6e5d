// sem_oracle.cpp -- CPU ORACLE for the fused SEM stiffness path.
//
// TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library, the
// C++ frontend) links, loads or calls this file; tests/, __graft_entry__.smoke()
// and bench.py's cpu_baseline / --impl reference legs use it as the checker and
// as the timed CPU port.
//
// What it restates (Rohit-Kakodkar/TensorOperations, paths inside that repo):
//   * the shared physics chain_rule / compute_stress / project / metric_at,
//     benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp:126-172, in the
//     same operation order (float arithmetic for the f32 entry points);
//   * the host reference loop reference(), same file :600-663: gradients summed
//     over p = 0..N-1, then one fused divergence + weighting sum over q;
//   * the 2D acoustic and batched-GEMM configurations have no reference
//     counterpart and are restated from their definitions.
//   * the assembled (ibool) mode has no counterpart in the reference (its SEM
//     programs are element-local, bench_sem_stiffness.cpp:8-11): the element
//     kernel is the one above, gather/scatter follow the numbering.
// Pinning: the element-local f32 entry point is compared bit-for-bit with the
// reference's own reference() compiled from its source (oracle/ref_pin.cpp,
// built into oracle/_ref/ when the reference tree is present) on the
// reference's own fill(); see tests/test_oracle_cpu.py.
//
// Built twice from this one source: -O2 -ffp-contract=off (parity oracle,
// libsem_oracle.so) and -O3 -fopenmp (CPU baseline, libsem_cpu.so).
#include <cstdint>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

template <typename T>
struct Mat3 {
  T m[3][3];
};

// bench_sem3d_levelgraph.cpp:126-133
template <typename T>
Mat3<T> chain_rule(const T dxi[3], const T det[3], const T dgm[3], const Mat3<T>& J) {
  Mat3<T> ds{};
  for (int c = 0; c < 3; ++c)
    for (int d = 0; d < 3; ++d)
      ds.m[c][d] = dxi[c] * J.m[0][d] + det[c] * J.m[1][d] + dgm[c] * J.m[2][d];
  return ds;
}

// bench_sem3d_levelgraph.cpp:135-144
template <typename T>
Mat3<T> compute_stress(const Mat3<T>& ds, T l2m, T mu) {
  const T lambda = l2m - T(2) * mu;
  const T tr = ds.m[0][0] + ds.m[1][1] + ds.m[2][2];
  Mat3<T> s{};
  for (int c = 0; c < 3; ++c)
    for (int d = 0; d < 3; ++d) s.m[c][d] = mu * (ds.m[c][d] + ds.m[d][c]);
  for (int c = 0; c < 3; ++c) s.m[c][c] += lambda * tr;
  return s;
}

// bench_sem3d_levelgraph.cpp:146-154
template <typename T>
void project(const Mat3<T>& sig, const T dref[3], T jac, T f[3]) {
  for (int c = 0; c < 3; ++c)
    f[c] = jac * (sig.m[c][0] * dref[0] + sig.m[c][1] * dref[1] + sig.m[c][2] * dref[2]);
}

// One element, element-local input ue[c][P] and output fe[c][P], per-point
// arrays already offset to the element.  bench_sem3d_levelgraph.cpp:624-661.
template <typename T>
void element_operator(int N, const T* const ue[3], const T* const m[12], int64_t e0,
                      const T* H, const T* Hw, const T* w, T* const fe[3], T* F) {
  const int NN = N * N, P = NN * N;
  auto at = [&](int k, int j, int i) { return (k * N + j) * N + i; };
  auto fidx = [&](int s, int k, int j, int i) { return s * P + at(k, j, i); };
  for (int k = 0; k < N; ++k)
    for (int j = 0; j < N; ++j)
      for (int i = 0; i < N; ++i) {
        T dxi[3] = {0, 0, 0}, det[3] = {0, 0, 0}, dgm[3] = {0, 0, 0};
        for (int p = 0; p < N; ++p) {
          for (int c = 0; c < 3; ++c) {
            dxi[c] += H[i * N + p] * ue[c][at(k, j, p)];
            det[c] += H[j * N + p] * ue[c][at(k, p, i)];
            dgm[c] += H[k * N + p] * ue[c][at(p, j, i)];
          }
        }
        const int64_t pt = e0 + at(k, j, i);
        Mat3<T> J;
        for (int r = 0; r < 3; ++r)
          for (int d = 0; d < 3; ++d) J.m[r][d] = m[3 * r + d][pt];
        const Mat3<T> sig = compute_stress(chain_rule(dxi, det, dgm, J), m[10][pt], m[11][pt]);
        for (int dir = 0; dir < 3; ++dir) {
          T f[3];
          project(sig, J.m[dir], m[9][pt], f);
          for (int c = 0; c < 3; ++c) F[fidx(3 * dir + c, k, j, i)] = f[c];
        }
      }
  for (int k = 0; k < N; ++k)
    for (int j = 0; j < N; ++j)
      for (int i = 0; i < N; ++i) {
        T acc[3] = {0, 0, 0};
        for (int q = 0; q < N; ++q)
          for (int c = 0; c < 3; ++c)
            acc[c] += w[j] * w[k] * Hw[q * N + i] * F[fidx(0 + c, k, j, q)] +
                      w[i] * w[k] * Hw[q * N + j] * F[fidx(3 + c, k, q, i)] +
                      w[i] * w[j] * Hw[q * N + k] * F[fidx(6 + c, q, j, i)];
        for (int c = 0; c < 3; ++c) fe[c][at(k, j, i)] = acc[c];
      }
}

template <typename T>
void sem3d_local(int64_t E, int N, const T* const u[3], const T* const m[12], const T* H,
                 const T* Hw, const T* w, T* const f[3]) {
  const int P = N * N * N;
  std::vector<T> F(9 * P);
  for (int64_t e = 0; e < E; ++e) {
    const T* ue[3] = {u[0] + e * P, u[1] + e * P, u[2] + e * P};
    T* fe[3] = {f[0] + e * P, f[1] + e * P, f[2] + e * P};
    element_operator(N, ue, m, e * P, H, Hw, w, fe, F.data());
  }
}

template <typename T>
void sem3d_assembled(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                     const T* const u[3], const T* const m[12], const T* H, const T* Hw,
                     const T* w, T* const f[3]) {
  const int P = N * N * N;
  for (int c = 0; c < 3; ++c) std::memset(f[c], 0, sizeof(T) * nglob);
  std::vector<T> F(9 * P), ub(3 * P), fb(3 * P);
  for (int64_t e = 0; e < E; ++e) {
    const int32_t* ib = ibool + e * P;
    for (int c = 0; c < 3; ++c)
      for (int p = 0; p < P; ++p) ub[c * P + p] = u[c][ib[p]];
    const T* ue[3] = {&ub[0], &ub[P], &ub[2 * P]};
    T* fe[3] = {&fb[0], &fb[P], &fb[2 * P]};
    element_operator(N, ue, m, e * P, H, Hw, w, fe, F.data());
    for (int c = 0; c < 3; ++c)
      for (int p = 0; p < P; ++p) f[c][ib[p]] += fb[c * P + p];
  }
}

// Element-parallel assembled operator: elements of one colour share no node,
// so each colour is a parallel loop with a race-free scatter.
template <typename T>
void sem3d_assembled_omp(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                         const T* const u[3], const T* const m[12], const T* H, const T* Hw,
                         const T* w, T* const f[3], int ncolours, const int64_t* colour_start,
                         const int64_t* colour_elems) {
  const int P = N * N * N;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < nglob; ++g)
    for (int c = 0; c < 3; ++c) f[c][g] = T(0);
  for (int col = 0; col < ncolours; ++col) {
    const int64_t b = colour_start[col], en = colour_start[col + 1];
#pragma omp parallel
    {
      std::vector<T> F(9 * P), ub(3 * P), fb(3 * P);
#pragma omp for schedule(static)
      for (int64_t x = b; x < en; ++x) {
        const int64_t e = colour_elems[x];
        const int32_t* ib = ibool + e * P;
        for (int c = 0; c < 3; ++c)
          for (int p = 0; p < P; ++p) ub[c * P + p] = u[c][ib[p]];
        const T* ue[3] = {&ub[0], &ub[P], &ub[2 * P]};
        T* fe[3] = {&fb[0], &fb[P], &fb[2 * P]};
        element_operator(N, ue, m, e * P, H, Hw, w, fe, F.data());
        for (int c = 0; c < 3; ++c)
          for (int p = 0; p < P; ++p) f[c][ib[p]] += fb[c * P + p];
      }
    }
  }
}

}  // namespace

// 2D elastic P-SV, element-local, the reference's host loop restated
// (benchmarks/sem_stiffness/bench_sem_stiffness.cpp:1335-1385, compute_stress
// :319-331): gradients with sums over p in order, chain rule, stress,
// integrands, then divergences with sums over q in order and the weighted sum.
// m = {xix, xiz, gamx, gamz, jac, l2m, mu}; arrays [E][j][i].
template <typename T>
void sem2d_local(int64_t E, int N, const T* const* u, const T* const* m, const T* H,
                 const T* Hw, const T* w, T* const* f) {
  const int P = N * N;
  std::vector<T> Fx0(P), Fg0(P), Fx1(P), Fg1(P);
  for (int64_t e = 0; e < E; ++e) {
    const T* U0 = u[0] + e * P;
    const T* U1 = u[1] + e * P;
    for (int j = 0; j < N; ++j)
      for (int i = 0; i < N; ++i) {
        T a0 = 0, a1 = 0, g0 = 0, g1 = 0;
        for (int p = 0; p < N; ++p) {
          a0 += H[i * N + p] * U0[j * N + p];
          a1 += H[i * N + p] * U1[j * N + p];
          g0 += H[j * N + p] * U0[p * N + i];
          g1 += H[j * N + p] * U1[p * N + i];
        }
        const int64_t q = e * P + j * N + i;
        const T ax = m[0][q], az = m[1][q], px = m[2][q], pz = m[3][q];
        const T jac = m[4][q], l2m = m[5][q], mu = m[6][q];
        const T ds00 = a0 * ax + g0 * px, ds01 = a0 * az + g0 * pz;
        const T ds10 = a1 * ax + g1 * px, ds11 = a1 * az + g1 * pz;
        const T lambda = l2m - T(2) * mu;
        const T s00 = l2m * ds00 + lambda * ds11;
        const T s11 = lambda * ds00 + l2m * ds11;
        const T s01 = mu * (ds01 + ds10);
        const T s10 = s01;
        Fx0[j * N + i] = jac * (s00 * ax + s01 * az);
        Fg0[j * N + i] = jac * (s00 * px + s01 * pz);
        Fx1[j * N + i] = jac * (s10 * ax + s11 * az);
        Fg1[j * N + i] = jac * (s10 * px + s11 * pz);
      }
    for (int j = 0; j < N; ++j)
      for (int i = 0; i < N; ++i) {
        T s0 = 0, s1 = 0, t0 = 0, t1 = 0;
        for (int q = 0; q < N; ++q) {
          s0 += Hw[q * N + i] * Fx0[j * N + q];
          s1 += Hw[q * N + i] * Fx1[j * N + q];
          t0 += Hw[q * N + j] * Fg0[q * N + i];
          t1 += Hw[q * N + j] * Fg1[q * N + i];
        }
        f[0][e * P + j * N + i] = w[j] * s0 + w[i] * t0;
        f[1][e * P + j * N + i] = w[j] * s1 + w[i] * t1;
      }
  }
}

// 2D acoustic, assembled (the first configuration's operator; no reference
// kernel exists -- same definition as to_sem2d_acoustic_apply).
// m = {xix, xiz, gamx, gamz, jac, rho}.
template <typename T>
void sem2d_acoustic(int64_t E, int N, int64_t nglob, const int32_t* ibool, const T* u,
                    const T* const* m, const T* H, const T* Hw, const T* w, T* f) {
  const int P = N * N;
  std::vector<T> ul(P), Fx(P), Fg(P);
  for (int64_t g = 0; g < nglob; ++g) f[g] = T(0);
  for (int64_t e = 0; e < E; ++e) {
    for (int p = 0; p < P; ++p) ul[p] = u[ibool[e * P + p]];
    for (int j = 0; j < N; ++j)
      for (int i = 0; i < N; ++i) {
        T dxi = 0, dgm = 0;
        for (int p = 0; p < N; ++p) {
          dxi += H[i * N + p] * ul[j * N + p];
          dgm += H[j * N + p] * ul[p * N + i];
        }
        const int64_t q = e * P + j * N + i;
        const T xix = m[0][q], xiz = m[1][q], gx = m[2][q], gz = m[3][q];
        const T s = m[4][q] / m[5][q];
        const T dudx = dxi * xix + dgm * gx, dudz = dxi * xiz + dgm * gz;
        Fx[j * N + i] = s * (dudx * xix + dudz * xiz);
        Fg[j * N + i] = s * (dudx * gx + dudz * gz);
      }
    for (int j = 0; j < N; ++j)
      for (int i = 0; i < N; ++i) {
        T tx = 0, tg = 0;
        for (int q = 0; q < N; ++q) {
          tx += Hw[q * N + i] * Fx[j * N + q];
          tg += Hw[q * N + j] * Fg[q * N + i];
        }
        f[ibool[e * P + j * N + i]] += w[j] * tx + w[i] * tg;
      }
  }
}

extern "C" {

void oracle_sem2d_acoustic_f64(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                               const double* u, const double* const* m, const double* H,
                               const double* Hw, const double* w, double* f) {
  sem2d_acoustic<double>(E, N, nglob, ibool, u, m, H, Hw, w, f);
}
void oracle_sem2d_acoustic_f32(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                               const float* u, const float* const* m, const float* H,
                               const float* Hw, const float* w, float* f) {
  sem2d_acoustic<float>(E, N, nglob, ibool, u, m, H, Hw, w, f);
}

void oracle_sem2d_local_f32(int64_t E, int N, const float* const* u, const float* const* m,
                            const float* H, const float* Hw, const float* w, float* const* f) {
  sem2d_local<float>(E, N, u, m, H, Hw, w, f);
}
void oracle_sem2d_local_f64(int64_t E, int N, const double* const* u, const double* const* m,
                            const double* H, const double* Hw, const double* w, double* const* f) {
  sem2d_local<double>(E, N, u, m, H, Hw, w, f);
}


int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// Thread count of the OpenMP CPU port, set explicitly: launchers such as
// torch.distributed.run export OMP_NUM_THREADS=1 to every rank, which would
// otherwise time the port on one core.
void oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

void oracle_sem3d_local_f32(int64_t E, int N, const float* const* u, const float* const* m,
                            const float* H, const float* Hw, const float* w, float* const* f) {
  sem3d_local<float>(E, N, u, m, H, Hw, w, f);
}
void oracle_sem3d_local_f64(int64_t E, int N, const double* const* u, const double* const* m,
                            const double* H, const double* Hw, const double* w,
                            double* const* f) {
  sem3d_local<double>(E, N, u, m, H, Hw, w, f);
}
void oracle_sem3d_assembled_f32(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                                const float* const* u, const float* const* m, const float* H,
                                const float* Hw, const float* w, float* const* f) {
  sem3d_assembled<float>(E, N, nglob, ibool, u, m, H, Hw, w, f);
}
void oracle_sem3d_assembled_f64(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                                const double* const* u, const double* const* m, const double* H,
                                const double* Hw, const double* w, double* const* f) {
  sem3d_assembled<double>(E, N, nglob, ibool, u, m, H, Hw, w, f);
}

// Greedy element colouring: no two elements of one colour share a node.
// Returns the number of colours and writes colour[E].
int oracle_colour_elements(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                           int32_t* colour) {
  const int P = N * N * N;
  std::vector<uint64_t> used(nglob, 0);  // bit c set: node touched by colour c
  int ncol = 0;
  for (int64_t e = 0; e < E; ++e) {
    uint64_t mask = 0;
    const int32_t* ib = ibool + e * P;
    for (int p = 0; p < P; ++p) mask |= used[ib[p]];
    int c = 0;
    while (c < 64 && (mask >> c) & 1ull) ++c;
    if (c == 64) return -1;
    colour[e] = c;
    if (c + 1 > ncol) ncol = c + 1;
    for (int p = 0; p < P; ++p) used[ib[p]] |= (1ull << c);
  }
  return ncol;
}

void oracle_sem3d_assembled_omp_f32(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                                    const float* const* u, const float* const* m,
                                    const float* H, const float* Hw, const float* w,
                                    float* const* f, int ncolours, const int64_t* colour_start,
                                    const int64_t* colour_elems) {
  sem3d_assembled_omp<float>(E, N, nglob, ibool, u, m, H, Hw, w, f, ncolours, colour_start,
                             colour_elems);
}
void oracle_sem3d_assembled_omp_f64(int64_t E, int N, int64_t nglob, const int32_t* ibool,
                                    const double* const* u, const double* const* m,
                                    const double* H, const double* Hw, const double* w,
                                    double* const* f, int ncolours,
                                    const int64_t* colour_start, const int64_t* colour_elems) {
  sem3d_assembled_omp<double>(E, N, nglob, ibool, u, m, H, Hw, w, f, ncolours, colour_start,
                              colour_elems);
}

}  // extern "C"
