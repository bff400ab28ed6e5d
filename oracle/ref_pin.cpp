// ref_pin.cpp -- exposes the reference's own host-side SEM 3D code to the tests.
//
// TEST INFRASTRUCTURE ONLY (see oracle/build_ref.py).  This translation unit
// compiles the reference benchmark source
//   benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp
// from where it lies, host-only, against this repository's Kokkos subset and
// frontend headers, and exports two of its functions through a C ABI:
//   fill()       the deterministic sin() inputs              (:588-598)
//   reference()  the host reference loop of the SEM operator (:600-663)
// so tests can pin the CPU oracle (oracle/sem_oracle.cpp) bit for bit against
// the reference's own code on the reference's own inputs.  The reference's
// main() is renamed so this file can define the exported entry points.
#define main reference_bench_sem3d_main
#include BENCH_SEM3D_SOURCE
#undef main

#include <cstring>

namespace {
void copy_out(const V4& v, int E, float* out) {
  std::memcpy(out, v.data(), sizeof(float) * std::size_t(E) * cfg::N * cfg::N * cfg::N);
}
V4 wrap_in(const float* src, int E, const char* name) {
  V4 v(name, E);
  std::memcpy(v.data(), src, sizeof(float) * std::size_t(E) * cfg::N * cfg::N * cfg::N);
  return v;
}
}  // namespace

extern "C" {

// The 15 element-local inputs in the reference's fill order
// u0 u1 u2 xix xiy xiz etx ety etz gmx gmy gmz l2m mu jac (seeds 0..14).
int ref_sem3d_fill(int E, float* const* out15) {
  for (int s = 0; s < 15; ++s) {
    V4 v("fill", E);
    fill(v, E, s);
    copy_out(v, E, out15[s]);
  }
  return cfg::N;
}

// The reference host loop on caller-given inputs (same order as above) and
// operators H[N][N], Hw[N][N], w[N]; writes r0, r1, r2 [E][N][N][N].
void ref_sem3d_reference(int E, const float* const* in15, const float* H, const float* Hw,
                         const float* w, float* r0, float* r1, float* r2) {
  Fields d;
  V4* dst[15] = {&d.u0, &d.u1, &d.u2, &d.xix, &d.xiy, &d.xiz, &d.etx, &d.ety,
                 &d.etz, &d.gmx, &d.gmy, &d.gmz, &d.l2m, &d.mu, &d.jac};
  for (int s = 0; s < 15; ++s) *dst[s] = wrap_in(in15[s], E, "in");
  d.H = V2("H", cfg::N, cfg::N);
  d.Hw = V2("Hw", cfg::N, cfg::N);
  std::memcpy(d.H.data(), H, sizeof(float) * cfg::N * cfg::N);
  std::memcpy(d.Hw.data(), Hw, sizeof(float) * cfg::N * cfg::N);
  Kokkos::View<float*, Kokkos::LayoutRight> wv("w", cfg::N);
  std::memcpy(wv.data(), w, sizeof(float) * cfg::N);
  d.w = wv;
  V4H h0("r0", E), h1("r1", E), h2("r2", E);
  reference(d, E, h0, h1, h2);
  copy_out(h0, E, r0);
  copy_out(h1, E, r1);
  copy_out(h2, E, r2);
}

}  // extern "C"
