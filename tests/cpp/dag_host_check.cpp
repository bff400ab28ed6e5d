// dag_host_check.cpp -- TEST ONLY: the flat-DAG route (make_dag / add /
// as<> / multi-output combine / outputs) lowered by b200/Dag.hpp and run
// through the generic device evaluator compiled as HOST code, one thread per
// CTA, exactly as level_kernel_host_check.cpp does for the level route.
//
// The graph has the shape of the reference's DAG SEM program
// (benchmarks/sem_stiffness_3d/bench_sem_stiffness_3d.cpp:251-472): nine
// gradients that contract INPUT nodes directly (so every input operand is
// staged by the lowering), three three-output combines that read all nine
// gradients under different label assignments, nine divergences, three
// weighted sums -- with functors of this test's own.  Checked:
//   * the plan: 6 levels (stage 2-D operators | stage 4-D fields | gradients |
//     combines | divergences | sums), 57 slots, the grid = the last node's
//     blocked labels; and the self-staging form (5 levels);
//   * values against a direct loop in BOTH forms;
//   * values against a direct loop, with a partial last element tile;
//   * index_consistent() and the scratch accounting on the host.
// Built and run by tests/test_frontend_cpu.py under AddressSanitizer/UBSan.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#define __device__
#define __forceinline__ inline
#define __global__
#define __launch_bounds__(x)
#define __shared__
#define __align__(n) __attribute__((aligned(n)))
struct EmuDim { unsigned x = 0, y = 0, z = 0; };
inline EmuDim threadIdx, blockIdx, blockDim{1, 1, 1}, gridDim;
inline void __syncthreads() {}
#include <Kokkos_Core.hpp>
#include <TensorOperations/DagGraph.hpp>
#include <TensorOperations/Tiling.hpp>
namespace TensorOperations::b200 { alignas(16) unsigned char lg_smem[1 << 20]; }
#include <TensorOperations/b200/LevelKernel.cuh>

using namespace TensorOperations;
using ES = Kokkos::DefaultExecutionSpace;
constexpr int N = 5;
constexpr int TE = 2;
using V4 = Kokkos::View<float* [N][N][N], Kokkos::LayoutRight>;
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;

using T2 = StaticTile<N, N>;
using TE4 = StaticTile<TE, N, N, N>;   // (e, z, y, x)
using TQ4 = StaticTile<N, TE, N, N>;   // (q, e, ., .)
using Grad = Tile<T2, TE4, TQ4>;
using Div = Tile<T2, TQ4, TE4>;
using Comb = CombineTile<TQ4, TQ4, TQ4, TQ4, TQ4, TQ4, TQ4, TQ4, TQ4, TQ4>;
using Sum = CombineTile<TE4, TE4, TE4, TE4>;

// Three outputs from nine gradients; `s` is a captured per-point field read at
// the GLOBAL coordinate the evaluator passes (axis roles given by `Dir`).
template <int Dir>
struct Mix {
  V4 s;
  Kokkos::Array<float, 3> operator()(int q, int e, int a, int b, float x0, float x1, float x2,
                                     float y0, float y1, float y2, float z0, float z1,
                                     float z2) const {
    int z, y, x;
    if (Dir == 0) { z = a; y = b; x = q; }
    if (Dir == 1) { z = a; y = q; x = b; }
    if (Dir == 2) { z = q; y = a; x = b; }
    const float m = s(e, z, y, x);
    return {m * x0 + y1 - 0.5f * z2, x1 - m * y0 + 0.25f * z1,
            0.75f * x2 + y2 * z0 + static_cast<float>(Dir) * m};
  }
};
struct WSum {
  float operator()(int, int k, int j, int i, float a, float b, float c) const {
    return (1.f + 0.1f * k) * a + (1.f + 0.01f * j) * b + (1.f + 0.001f * i) * c;
  }
};

template <int Dummy>
auto build_graph(V2 H, V2 Hw, V4 u0, V4 u1, V4 u2, V4 sc) {
  auto gx = [&](V4 u) {
    return make_contraction_node<'q', 'e', 'k', 'j'>(make_input_node(make_handle<'q', 'p'>(H)),
                                                     make_input_node(make_handle<'e', 'k', 'j', 'p'>(u)));
  };
  auto ge = [&](V4 u) {
    return make_contraction_node<'q', 'e', 'k', 'i'>(make_input_node(make_handle<'q', 'p'>(H)),
                                                     make_input_node(make_handle<'e', 'k', 'p', 'i'>(u)));
  };
  auto gg = [&](V4 u) {
    return make_contraction_node<'q', 'e', 'j', 'i'>(make_input_node(make_handle<'q', 'p'>(H)),
                                                     make_input_node(make_handle<'e', 'p', 'j', 'i'>(u)));
  };
  auto [d0, x0] = make_dag<float, ES>().add(gx(u0), Grad{});
  auto [d1, x1] = d0.add(gx(u1), Grad{});
  auto [d2, x2] = d1.add(gx(u2), Grad{});
  auto [d3, y0] = d2.add(ge(u0), Grad{});
  auto [d4, y1] = d3.add(ge(u1), Grad{});
  auto [d5, y2] = d4.add(ge(u2), Grad{});
  auto [d6, z0] = d5.add(gg(u0), Grad{});
  auto [d7, z1] = d6.add(gg(u1), Grad{});
  auto [d8, z2] = d7.add(gg(u2), Grad{});
  // x* is (new-x, e, z, y), y* is (new-y, e, z, x), z* is (new-z, e, y, x)
  auto [d9, a0, a1, a2] = d8.add(
      make_combine_node<'q', 'e', 'k', 'j'>(
          x0.template as<'q', 'e', 'k', 'j'>(), x1.template as<'q', 'e', 'k', 'j'>(),
          x2.template as<'q', 'e', 'k', 'j'>(), y0.template as<'j', 'e', 'k', 'q'>(),
          y1.template as<'j', 'e', 'k', 'q'>(), y2.template as<'j', 'e', 'k', 'q'>(),
          z0.template as<'k', 'e', 'j', 'q'>(), z1.template as<'k', 'e', 'j', 'q'>(),
          z2.template as<'k', 'e', 'j', 'q'>(), Mix<0>{sc}),
      Comb{});
  auto [d10, b0, b1, b2] = d9.add(
      make_combine_node<'q', 'e', 'k', 'i'>(
          x0.template as<'i', 'e', 'k', 'q'>(), x1.template as<'i', 'e', 'k', 'q'>(),
          x2.template as<'i', 'e', 'k', 'q'>(), y0.template as<'q', 'e', 'k', 'i'>(),
          y1.template as<'q', 'e', 'k', 'i'>(), y2.template as<'q', 'e', 'k', 'i'>(),
          z0.template as<'k', 'e', 'q', 'i'>(), z1.template as<'k', 'e', 'q', 'i'>(),
          z2.template as<'k', 'e', 'q', 'i'>(), Mix<1>{sc}),
      Comb{});
  auto [d11, c0, c1, c2] = d10.add(
      make_combine_node<'q', 'e', 'j', 'i'>(
          x0.template as<'i', 'e', 'q', 'j'>(), x1.template as<'i', 'e', 'q', 'j'>(),
          x2.template as<'i', 'e', 'q', 'j'>(), y0.template as<'j', 'e', 'q', 'i'>(),
          y1.template as<'j', 'e', 'q', 'i'>(), y2.template as<'j', 'e', 'q', 'i'>(),
          z0.template as<'q', 'e', 'j', 'i'>(), z1.template as<'q', 'e', 'j', 'i'>(),
          z2.template as<'q', 'e', 'j', 'i'>(), Mix<2>{sc}),
      Comb{});
  auto dx = [&](auto f) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(make_input_node(make_handle<'q', 'i'>(Hw)),
                                                     f.template as<'q', 'e', 'k', 'j'>());
  };
  auto de = [&](auto f) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(make_input_node(make_handle<'q', 'j'>(Hw)),
                                                     f.template as<'q', 'e', 'k', 'i'>());
  };
  auto dg = [&](auto f) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(make_input_node(make_handle<'q', 'k'>(Hw)),
                                                     f.template as<'q', 'e', 'j', 'i'>());
  };
  auto [d12, t0] = d11.add(dx(a0), Div{});
  auto [d13, t1] = d12.add(dx(a1), Div{});
  auto [d14, t2] = d13.add(dx(a2), Div{});
  auto [d15, t3] = d14.add(de(b0), Div{});
  auto [d16, t4] = d15.add(de(b1), Div{});
  auto [d17, t5] = d16.add(de(b2), Div{});
  auto [d18, t6] = d17.add(dg(c0), Div{});
  auto [d19, t7] = d18.add(dg(c1), Div{});
  auto [d20, t8] = d19.add(dg(c2), Div{});
  // a divergence stores freeA ++ freeB: (i,e,k,j), (j,e,k,i), (k,e,j,i)
  auto sum = [&](auto tx, auto te, auto tg) {
    return make_combine_node<'e', 'k', 'j', 'i'>(tx.template as<'i', 'e', 'k', 'j'>(),
                                                 te.template as<'j', 'e', 'k', 'i'>(),
                                                 tg.template as<'k', 'e', 'j', 'i'>(), WSum{});
  };
  auto [d21, r0] = d20.add(sum(t0, t3, t6), Sum{});
  auto [d22, r1] = d21.add(sum(t1, t4, t7), Sum{});
  auto [d23, r2] = d22.add(sum(t2, t5, t8), Sum{});
  return std::make_tuple(d23, r0, r1, r2);
}

using Built = decltype(build_graph<0>(V2(), V2(), V4(), V4(), V4(), V4()));
using Dag = std::tuple_element_t<0, Built>;
using Low = typename Dag::lowering;
static_assert(Dag::N == 24);
static_assert(Low::NS == 27, "9 gradients stage H and a field, 9 divergences stage Hw");
static_assert(Low::num_levels == 6,
              "stage 2-D | stage 4-D | gradients | combines | divergences | sums");
static_assert(Low::num_dag_slots == 30, "24 nodes, three of them with three outputs");
static_assert(b200::Algebra<typename Low::levels_t>::num_slots == 57, "30 node slots + 27 stages");
static_assert(LevelPlan<typename Low::levels_t>::num_levels == 6);
static_assert(tuple_size_v<tuple_element_t<0, typename Low::levels_t>> == 18);
static_assert(tuple_size_v<tuple_element_t<1, typename Low::levels_t>> == 9);
static_assert(tuple_size_v<tuple_element_t<2, typename Low::levels_t>> == 9);
static_assert(tuple_size_v<tuple_element_t<3, typename Low::levels_t>> == 3);
static_assert(tuple_size_v<tuple_element_t<4, typename Low::levels_t>> == 9);
static_assert(tuple_size_v<tuple_element_t<5, typename Low::levels_t>> == 3);
// the form a launch takes when a contracted label spans several tiles: the
// gradients (H x u) stage their own operands
using LowK = typename Dag::lowering_ktiled;
static_assert(LowK::NS == 9 && LowK::num_levels == 5);
static_assert(b200::Algebra<typename LowK::levels_t>::num_slots == 57,
              "30 node slots + 9 stages + 2 operand tiles per gradient");
static_assert(b200::member_traits<tuple_element_t<0, tuple_element_t<1, typename LowK::levels_t>>>::kind == 3);
using GS = b200::GridSpec<typename Low::label_tiles_t, typename Low::levels_t>;
static_assert(GS::rank == 4 && GS::labels[0] == 'e', "the grid is the last node's labels");
static_assert(Low::label_tiles_t::tile('e') == TE && !Low::label_tiles_t::is_gridded('q'));

int main(int argc, char** argv) {
  const int E = argc > 1 ? std::atoi(argv[1]) : 5;
  V2 H("H", N, N), Hw("Hw", N, N);
  V4 u0("u0", E), u1("u1", E), u2("u2", E), sc("sc", E), f0("f0", E), f1("f1", E), f2("f2", E);
  for (int a = 0; a < N; ++a)
    for (int b = 0; b < N; ++b) {
      H(a, b) = 0.1f * a - 0.2f * b + (a == b);
      Hw(a, b) = 0.3f * b + 0.05f * a * b - 0.1f;
    }
  for (int n = 0; n < E * N * N * N; ++n) {
    u0.data()[n] = std::sin(0.1f * n);
    u1.data()[n] = std::cos(0.07f * n);
    u2.data()[n] = 0.01f * (n % 97);
    sc.data()[n] = 1.f + 0.001f * n;
  }
  auto [dag, r0, r1, r2] = build_graph<0>(H, Hw, u0, u1, u2, sc);
  if (!dag.index_consistent()) {
    std::printf("index_consistent false\n");
    return 1;
  }
  const auto outs = dag.outputs(r0, r1, r2);
  std::printf("pools %zu scratch %zu unpooled %zu\n", decltype(outs)::num_pools, outs.scratch_bytes(),
              dag.scratch_bytes());
  if (outs.slot_bytes() > dag.slot_bytes() || outs.operand_bytes() > dag.operand_bytes() ||
      outs.launch_scratch_bytes() == 0)
    return 1;

  if (dag.needs_contracted_tiles()) return 1;
  auto emulate = [&]<class L>(L) {
    constexpr std::size_t S0 = L::level_slot(decltype(r0)::slot_index);
    constexpr std::size_t S1 = L::level_slot(decltype(r1)::slot_index);
    constexpr std::size_t S2 = L::level_slot(decltype(r2)::slot_index);
    using GK = b200::GraphKernel<float, typename L::label_tiles_t, typename L::levels_t, S0, S1, S2>;
    static_assert(GK::GR == 4);
    b200::GridRuntime<GK::GR> grid{};
    grid.ntiles[0] = (E + TE - 1) / TE;
    grid.ntiles[1] = grid.ntiles[2] = grid.ntiles[3] = 1;
    const auto levels = L::make_levels(dag.nodes);
    DeviceTuple<V4, V4, V4> views(f0, f1, f2);
    for (unsigned bx = 0; bx < static_cast<unsigned>(grid.ntiles[0]); ++bx) {
      blockIdx.x = bx;
      GK::run(levels, grid, views);
    }
  };
  const int form = argc > 2 ? std::atoi(argv[2]) : 0;
  if (form == 0)
    emulate(Low{});
  else
    emulate(LowK{});

  // direct loop
  V4* us[3] = {&u0, &u1, &u2};
  auto grad = [&](int c, int dir, int e, int z, int y, int x) {
    double s = 0;
    for (int p = 0; p < N; ++p) {
      if (dir == 0) s += H(x, p) * (*us[c])(e, z, y, p);
      if (dir == 1) s += H(y, p) * (*us[c])(e, z, p, x);
      if (dir == 2) s += H(z, p) * (*us[c])(e, p, y, x);
    }
    return static_cast<float>(s);
  };
  auto mix = [&](int dir, int e, int z, int y, int x) {
    float g[9];
    for (int c = 0; c < 3; ++c)
      for (int d = 0; d < 3; ++d) g[3 * d + c] = grad(c, d, e, z, y, x);
    const float m = sc(e, z, y, x);
    Kokkos::Array<float, 3> r{{m * g[0] + g[4] - 0.5f * g[8], g[1] - m * g[3] + 0.25f * g[7],
                               0.75f * g[2] + g[5] * g[6] + static_cast<float>(dir) * m}};
    return r;
  };
  double worst = 0, scale = 1e-30;
  for (int e = 0; e < E; ++e)
    for (int k = 0; k < N; ++k)
      for (int j = 0; j < N; ++j)
        for (int i = 0; i < N; ++i)
          for (int c = 0; c < 3; ++c) {
            double tx = 0, te = 0, tg = 0;
            for (int q = 0; q < N; ++q) {
              tx += Hw(q, i) * mix(0, e, k, j, q)[c];
              te += Hw(q, j) * mix(1, e, k, q, i)[c];
              tg += Hw(q, k) * mix(2, e, q, j, i)[c];
            }
            const double want = (1.0 + 0.1 * k) * tx + (1.0 + 0.01 * j) * te + (1.0 + 0.001 * i) * tg;
            const V4& f = c == 0 ? f0 : (c == 1 ? f1 : f2);
            worst = std::fmax(worst, std::fabs(f(e, k, j, i) - want));
            scale = std::fmax(scale, std::fabs(want));
          }
  std::printf("max abs error %.3e (scale %.3e)\n", worst, scale);
  return worst / scale < 1e-5 ? 0 : 1;
}
