// kokkos_subset_gpu.cpp -- exercises the Kokkos subset on the GPU, one step at
// a time (each step prints before it runs), and checks the results.  Built by
// tests/cpp/build.py, run by tests/test_frontend_gpu.py.
#include <Kokkos_Core.hpp>

#include <cstdio>

#define STEP(msg) std::printf("step: %s\n", msg), std::fflush(stdout)

using V4 = Kokkos::View<float* [5][5][5], Kokkos::LayoutRight>;
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;
using V1c = Kokkos::View<const float*, Kokkos::LayoutRight>;

int main(int argc, char* argv[]) {
  int fails = 0;
  STEP("initialize");
  Kokkos::initialize(argc, argv);
  {
    const int E = 7;
    STEP("allocate V4");
    V4 a("a", E);
    STEP("mirror + host fill");
    auto h = Kokkos::create_mirror_view(a);
    static_assert(std::is_same_v<decltype(h)::memory_space, Kokkos::HostSpace>);
    for (int e = 0; e < E; ++e)
      for (int k = 0; k < 5; ++k)
        for (int j = 0; j < 5; ++j)
          for (int i = 0; i < 5; ++i) h(e, k, j, i) = 1000.f * e + 100.f * k + 10.f * j + i;
    STEP("deep_copy H2D");
    Kokkos::deep_copy(a, h);
    STEP("range parallel_for");
    V4 b("b", E);
    Kokkos::parallel_for(
        "scale", E * 125, KOKKOS_LAMBDA(const int n) { b.data()[n] = 2.f * a.data()[n]; });
    STEP("team parallel_for with scratch");
    V4 c("c", E);
    using member_t = Kokkos::TeamPolicy<>::member_type;
    using SE = Kokkos::View<float* [5][5][5], Kokkos::DefaultExecutionSpace::scratch_memory_space,
                            Kokkos::MemoryUnmanaged>;
    const std::size_t bytes = SE::shmem_size(1);
    Kokkos::parallel_for(
        "team", Kokkos::TeamPolicy<>(E, 64).set_scratch_size(0, Kokkos::PerTeam(bytes)),
        KOKKOS_LAMBDA(const member_t& t) {
          SE s(t.team_scratch(0), 1);
          const int e = t.league_rank();
          Kokkos::parallel_for(Kokkos::TeamVectorRange(t, 125), [&](int n) {
            s.data()[n] = b(e, n / 25, (n / 5) % 5, n % 5);
          });
          t.team_barrier();
          Kokkos::parallel_for(Kokkos::TeamVectorRange(t, 125), [&](int n) {
            c(e, n / 25, (n / 5) % 5, n % 5) = s.data()[124 - n] + 1.f;
          });
        });
    STEP("fence + mirror_and_copy D2H");
    Kokkos::fence();
    auto hc = Kokkos::create_mirror_view_and_copy(Kokkos::HostSpace{}, c);
    for (int e = 0; e < E; ++e)
      for (int n = 0; n < 125; ++n) {
        const int m = 124 - n;
        const float want =
            2.f * (1000.f * e + 100.f * (m / 25) + 10.f * ((m / 5) % 5) + m % 5) + 1.f;
        if (hc(e, n / 25, (n / 5) % 5, n % 5) != want) ++fails;
      }
    STEP("const view conversion + deep_copy scalar");
    Kokkos::View<float*, Kokkos::LayoutRight> w("w", 5);
    Kokkos::deep_copy(w, 3.5f);
    V1c wc = w;
    auto hw = Kokkos::create_mirror_view_and_copy(Kokkos::HostSpace{}, wc);
    for (int i = 0; i < 5; ++i)
      if (hw(i) != 3.5f) ++fails;
    STEP("2D view extents");
    V2 m("m", 3, 4);
    if (m.extent(0) != 3 || m.extent(1) != 4 || a.extent(0) != 7 || a.extent(3) != 5) ++fails;
  }
  STEP("finalize");
  Kokkos::finalize();
  std::printf("kokkos subset: %s (%d failures)\n", fails ? "FAIL" : "PASS", fails);
  return fails ? 1 : 0;
}
