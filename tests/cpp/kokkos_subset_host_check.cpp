// kokkos_subset_host_check.cpp -- TEST ONLY: host (Serial) checks of the Kokkos
// subset the reference programs compile against (tensoroperations_b200/include/
// Kokkos_Core.hpp).  Built with g++ and run by tests/test_frontend_cpu.py.
//   * TeamPolicy::set_scratch_size sets the request IN PLACE (the reference's
//     multilevel/team contraction benchmarks call it as a statement), and a
//     team that carves exactly that many bytes of scratch views gets distinct,
//     in-bounds regions;
//   * a scratch request past the policy's size (larger than the whole region,
//     or than what is left of it) hands out no pointer: the team stops and
//     the status word that fence() checks is set;
//   * LayoutLeft views: first index fastest, strides, mirrors keep the layout;
//   * MDRangePolicy<Rank<N>> visits every point of the box exactly once.
#include <Kokkos_Core.hpp>

#include <cstdio>
#include <vector>

#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::printf("FAILED %s at line %d\n", #c, __LINE__);         \
      return 1;                                                    \
    }                                                              \
  } while (0)

int main() {
  Kokkos::initialize();
  {
    // ---- scratch sizing through a policy set by statement ----
    using Scratch2 = Kokkos::View<float**, Kokkos::DefaultExecutionSpace::scratch_memory_space,
                                  Kokkos::MemoryTraits<Kokkos::Unmanaged>>;
    const std::size_t bytes = Scratch2::shmem_size(3, 5) + Scratch2::shmem_size(7, 2) +
                              Scratch2::shmem_size(1, 1);
    Kokkos::TeamPolicy<> policy(4, Kokkos::AUTO);
    policy.set_scratch_size(0, Kokkos::PerTeam(bytes));
    CHECK(policy.scratch_size(0) == bytes);
    const auto chained = Kokkos::TeamPolicy<>(2, 1).set_scratch_size(0, Kokkos::PerTeam(64));
    CHECK(chained.scratch_size(0) == 64);
    std::vector<int> ok(4, 0);
    Kokkos::parallel_for("carve", policy, [&](const Kokkos::TeamPolicy<>::member_type& t) {
      Scratch2 a(t.team_scratch(0), 3, 5), b(t.team_scratch(0), 7, 2), c(t.team_scratch(0), 1, 1);
      const char* lo = static_cast<const char*>(static_cast<const void*>(a.data()));
      const bool in = a.data() && b.data() && c.data() &&
                      static_cast<const char*>(static_cast<const void*>(c.data())) + 4 <= lo + bytes &&
                      a.data() + 15 <= b.data() && b.data() + 14 <= c.data();
      for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 5; ++j) a(i, j) = float(i * 5 + j);
      ok[t.league_rank()] = in && a(2, 4) == 14.f;
    });
    for (int r = 0; r < 4; ++r) CHECK(ok[r] == 1);
    CHECK(Kokkos::Impl::take_scratch_status() == 0);

    // ---- a request past the policy's size never gets a pointer ----
    // (one view larger than the whole region, and one that only overflows
    // what is left): the team stops at the request, the status word is set,
    // and no view of the team was handed memory outside its region
    for (const std::size_t first : {std::size_t(0), bytes - 16}) {
      std::vector<int> reached(3, 0);
      Kokkos::TeamPolicy<> small(3, 1);
      small.set_scratch_size(0, Kokkos::PerTeam(bytes));
      Kokkos::parallel_for("overflow", small, [&](const Kokkos::TeamPolicy<>::member_type& t) {
        if (first) Scratch2 pre(t.team_scratch(0), 1, first / 4);
        Scratch2 big(t.team_scratch(0), 64, 64);  // 16 KiB > bytes
        reached[t.league_rank()] = big.data() ? 1 : 2;
      });
      for (int r = 0; r < 3; ++r) CHECK(reached[r] == 0);
      CHECK(Kokkos::Impl::take_scratch_status() == 1);
      CHECK(Kokkos::Impl::take_scratch_status() == 0);
    }

    // ---- LayoutLeft ----
    Kokkos::View<float**, Kokkos::LayoutLeft, Kokkos::HostSpace> L("L", 3, 4);
    CHECK(L.stride(0) == 1 && L.stride(1) == 3);
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 4; ++j) L(i, j) = float(10 * i + j);
    CHECK(L.data()[1] == 10.f && L.data()[3] == 1.f);  // (1,0) then (0,1)
    auto M = Kokkos::create_mirror_view(L);
    static_assert(std::is_same_v<decltype(M)::array_layout, Kokkos::LayoutLeft>);
    Kokkos::View<float* [2][3], Kokkos::LayoutLeft, Kokkos::HostSpace> S("S", 4);
    CHECK(S.stride(0) == 1 && S.stride(1) == 4 && S.stride(2) == 8);
    S(3, 1, 2) = 7.f;
    CHECK(S.data()[3 + 4 * 1 + 8 * 2] == 7.f);

    // ---- MDRangePolicy ----
    std::vector<int> seen(2 * 3 * 4, 0);
    Kokkos::parallel_for("md", Kokkos::MDRangePolicy<Kokkos::Rank<3>>({1, 0, 2}, {3, 3, 6}),
                         [&](int a, int b, int c) { seen[((a - 1) * 3 + b) * 4 + (c - 2)] += 1; });
    for (int v : seen) CHECK(v == 1);
  }
  Kokkos::finalize();
  std::printf("kokkos subset host ok\n");
  return 0;
}
