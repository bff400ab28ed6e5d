// ref_pin2d.cpp -- exposes the reference's own host-side SEM 2D code to the tests.
//
// TEST INFRASTRUCTURE ONLY (see oracle/build_ref.py).  This translation unit
// compiles the reference benchmark source
//   benchmarks/sem_stiffness/bench_sem_stiffness.cpp
// from where it lies, host-only, against this repository's Kokkos subset and
// frontend headers, and exports three of its functions through a C ABI:
//   fill_field()      the deterministic integer-pattern inputs  (:1306-1313)
//   fill_operators()  H, Hw and the weights w                   (:1318-1329)
//   host_reference()  the host loop of the 2D P-SV operator     (:1335-1385)
// so tests can pin the CPU oracle's 2D restatement (oracle/sem_oracle.cpp,
// sem2d_local) bit for bit against the reference's own code.  The reference's
// main() is renamed so this file can define the exported entry points.
#define main reference_bench_sem2d_main
#include BENCH_SEM2D_SOURCE
#undef main

#include <cstring>

namespace {
constexpr std::size_t kPts = std::size_t(cfg::N) * cfg::N;
}  // namespace

extern "C" {

int ref_sem2d_ngll(void) { return cfg::N; }

// The nine element-local inputs in the reference's salt order
// u0 u1 xix xiz gx gz l2m mu jac (salts 0..8), then H[N][N], Hw[N][N], w[N].
int ref_sem2d_fill(int E, float* const* out9, float* H, float* Hw, float* w) {
  for (int s = 0; s < 9; ++s) {
    V3 v("fill", E, cfg::N, cfg::N);
    fill_field(v, E, s);
    std::memcpy(out9[s], v.data(), sizeof(float) * E * kPts);
  }
  V2 h("H", cfg::N, cfg::N), hw("Hw", cfg::N, cfg::N);
  Kokkos::Array<float, cfg::N> wa{};
  fill_operators(h, hw, wa);
  std::memcpy(H, h.data(), sizeof(float) * kPts);
  std::memcpy(Hw, hw.data(), sizeof(float) * kPts);
  for (int a = 0; a < cfg::N; ++a) w[a] = wa[a];
  return cfg::N;
}

// The reference host loop on caller-given inputs (order as above); writes
// f0, f1 [E][N][N].
void ref_sem2d_reference(int E, const float* const* in9, const float* H, const float* Hw,
                         const float* w, float* f0, float* f1) {
  V3 v[9];
  for (int s = 0; s < 9; ++s) {
    v[s] = V3("in", E, cfg::N, cfg::N);
    std::memcpy(v[s].data(), in9[s], sizeof(float) * E * kPts);
  }
  V2 h("H", cfg::N, cfg::N), hw("Hw", cfg::N, cfg::N);
  std::memcpy(h.data(), H, sizeof(float) * kPts);
  std::memcpy(hw.data(), Hw, sizeof(float) * kPts);
  Kokkos::Array<float, cfg::N> wa{};
  for (int a = 0; a < cfg::N; ++a) wa[a] = w[a];
  V3H r0("r0", E, cfg::N, cfg::N), r1("r1", E, cfg::N, cfg::N);
  host_reference(v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8], h, hw, wa, r0, r1, E);
  std::memcpy(f0, r0.data(), sizeof(float) * E * kPts);
  std::memcpy(f1, r1.data(), sizeof(float) * E * kPts);
}

}  // extern "C"
