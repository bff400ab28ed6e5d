// tree_host_check.cpp -- TEST ONLY: the tree route (make_graph().ops(node),
// a nested Tile / CombineTile bundle, Graph::execute) lowered by b200/Tree.hpp
// onto the flat DAG and the level plan, run through the generic device
// evaluator compiled as HOST code (one thread per CTA), against direct loops.
//
// Case 1 has the shape of the reference's 2D tree program
// (benchmarks/sem_stiffness/bench_sem_stiffness.cpp:502-549): a root combine of
// two divergence contractions, each contracting a nested combine of four
// gradient contractions on INPUT nodes -- declared in the consumer's order, so
// the combine reads them through their storage permutation.  Case 2 is a
// contraction chain R = (A . B) . C given as a flat pre-order list of
// Tile<A,B,C> bundles (reference Graph.hpp:316-327), with a contraction hook
// and an input hook.  Case 3 contracts two labels that span several (ragged)
// tiles, with a hook that must act once per element.  All with partial last
// tiles.  Built and run by tests/test_frontend_cpu.py under ASan/UBSan.
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
#include <TensorOperations/Evaluator.hpp>
#include <TensorOperations/Graph.hpp>
#include <TensorOperations/Tiling.hpp>
namespace TensorOperations::b200 { alignas(16) unsigned char lg_smem[1 << 20]; }
#include <TensorOperations/b200/LevelKernel.cuh>

using namespace TensorOperations;
using ES = Kokkos::DefaultExecutionSpace;
constexpr int N = 4;
constexpr int TE = 3;
using V3 = Kokkos::View<float* [N][N], Kokkos::LayoutRight>;
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;

using TH = StaticTile<N, N>;
using TEJI = StaticTile<TE, N, N>;  // (e, ., .)
using TQEJ = StaticTile<N, TE, N>;  // (., e, .)
using BGrad = Tile<TH, TEJI, TQEJ>;
using CombF = CombineTile<TQEJ, BGrad, BGrad, BGrad, BGrad>;
using BDiv = Tile<TH, CombF, TEJI>;
using CombR = CombineTile<TEJI, BDiv, BDiv>;

struct Flux {
  V3 s;
  int dir;
  float operator()(int q, int e, int j, float a0, float a1, float g0, float g1) const {
    const float m = dir == 0 ? s(e, j, q) : s(e, q, j);
    return m * a0 - 0.5f * a1 + g0 * g1 + 0.25f * static_cast<float>(dir);
  }
};
struct Sum2 {
  float operator()(int, int j, int i, float t1, float t2) const {
    return (1.f + 0.1f * j) * t1 + (1.f - 0.05f * i) * t2;
  }
};

template <class Map, class Levels, std::size_t... R, class Views>
void emulate(const Levels& levels, int ntiles_e, const Views& views, int grid_rank) {
  using GK = b200::GraphKernel<float, Map, Levels, R...>;
  b200::GridRuntime<GK::GR> grid{};
  for (int g = 0; g < GK::GR; ++g) grid.ntiles[g] = 1;
  grid.ntiles[0] = ntiles_e;
  if (GK::GR != grid_rank) std::printf("unexpected grid rank %d\n", GK::GR);
  for (unsigned bx = 0; bx < static_cast<unsigned>(ntiles_e); ++bx) {
    blockIdx.x = bx;
    GK::run(levels, grid, views);
  }
}

int main(int argc, char** argv) {
  const int E = argc > 1 ? std::atoi(argv[1]) : 5;
  int bad = 0;
  // ---- case 1: the 2D-shaped tree -------------------------------------------
  {
    V2 H("H", N, N), Hw("Hw", N, N);
    V3 u0("u0", E), u1("u1", E), sc("sc", E), out("out", E);
    for (int a = 0; a < N; ++a)
      for (int b = 0; b < N; ++b) {
        H(a, b) = 0.2f * a - 0.3f * b + (a == b);
        Hw(a, b) = 0.1f * (a + 1) * (b - 1.5f);
      }
    for (int n = 0; n < E * N * N; ++n) {
      u0.data()[n] = std::sin(0.3f * n);
      u1.data()[n] = std::cos(0.11f * n);
      sc.data()[n] = 1.f + 0.01f * n;
    }
    auto grad_x = [&](V3 u) {  // (q, e, j): contracts x
      return make_contraction_node<'q', 'e', 'j'>(make_input_node(make_handle<'q', 'p'>(H)),
                                                  make_input_node(make_handle<'e', 'j', 'p'>(u)));
    };
    auto grad_z = [&](V3 u) {  // declared (j, e, q): contracts z, read as the combine's (q, e, j)
      return make_contraction_node<'j', 'e', 'q'>(make_input_node(make_handle<'j', 'p'>(H)),
                                                  make_input_node(make_handle<'e', 'p', 'q'>(u)));
    };
    auto F0 = make_combine_node<'q', 'e', 'j'>(grad_x(u0), grad_x(u1), grad_z(u0), grad_z(u1),
                                               Flux{sc, 0});
    auto grad_x1 = [&](V3 u) {  // declared (i, e, q)
      return make_contraction_node<'i', 'e', 'q'>(make_input_node(make_handle<'i', 'p'>(H)),
                                                  make_input_node(make_handle<'e', 'q', 'p'>(u)));
    };
    auto grad_z1 = [&](V3 u) {  // (q, e, i)
      return make_contraction_node<'q', 'e', 'i'>(make_input_node(make_handle<'q', 'p'>(H)),
                                                  make_input_node(make_handle<'e', 'p', 'i'>(u)));
    };
    auto F1 = make_combine_node<'q', 'e', 'i'>(grad_x1(u0), grad_x1(u1), grad_z1(u0), grad_z1(u1),
                                               Flux{sc, 1});
    auto root = make_combine_node<'e', 'j', 'i'>(
        make_contraction_node<'e', 'j', 'i'>(make_input_node(make_handle<'q', 'i'>(Hw)), F0),
        make_contraction_node<'e', 'j', 'i'>(make_input_node(make_handle<'q', 'j'>(Hw)), F1),
        Sum2{});
    auto [g1, h] = make_graph().ops(root);
    (void)h;
    const CombR spec = make_combine_tile(TEJI{}, BDiv{}, BDiv{});
    using Node = decltype(root);
    using TT = b200::tree_types<Node, CombR>;
    using Dag = typename TT::dag_t;
    using Low = typename Dag::lowering;
    static_assert(Dag::N == 13, "8 gradients + 2 fluxes + 2 divergences + the root");
    static_assert(Low::num_levels == 6,
                  "stage H/Hw | stage u | gradients | fluxes | divergences | root");
    const auto dag = b200::TreeLowering<float, ES>::dag_of<CombR>(root);
    if (!dag.index_consistent()) {
      std::printf("tree: index_consistent false\n");
      return 1;
    }
    std::printf("tree scratch %zu\n", Evaluator<TeamPolicyTag<ES>, Node, CombR>::scratch_size_per_team(spec));
    constexpr std::size_t S = Low::level_slot(Dag::num_slots() - 1);
    emulate<typename Low::label_tiles_t, typename Low::levels_t, S>(
        Low::make_levels(dag.nodes), (E + TE - 1) / TE, DeviceTuple<V3>(out), 3);
    double worst = 0, scale = 1e-30;
    auto gx = [&](V3 u, int e, int j, int x) {
      double s = 0;
      for (int p = 0; p < N; ++p) s += H(x, p) * u(e, j, p);
      return static_cast<float>(s);
    };
    auto gz = [&](V3 u, int e, int z, int i) {
      double s = 0;
      for (int p = 0; p < N; ++p) s += H(z, p) * u(e, p, i);
      return static_cast<float>(s);
    };
    for (int e = 0; e < E; ++e)
      for (int j = 0; j < N; ++j)
        for (int i = 0; i < N; ++i) {
          double t1 = 0, t2 = 0;
          for (int q = 0; q < N; ++q) {
            // F0 at (x = q, z = j); F1 at (x = i, z = q)
            const float f0 = Flux{sc, 0}(q, e, j, gx(u0, e, j, q), gx(u1, e, j, q), gz(u0, e, j, q),
                                         gz(u1, e, j, q));
            const float f1 = Flux{sc, 1}(q, e, i, gx(u0, e, q, i), gx(u1, e, q, i), gz(u0, e, q, i),
                                         gz(u1, e, q, i));
            t1 += Hw(q, i) * f0;
            t2 += Hw(q, j) * f1;
          }
          const double want = (1.0 + 0.1 * j) * t1 + (1.0 - 0.05 * i) * t2;
          worst = std::fmax(worst, std::fabs(out(e, j, i) - want));
          scale = std::fmax(scale, std::fabs(want));
        }
    std::printf("tree max abs error %.3e (scale %.3e)\n", worst, scale);
    if (!(worst / scale < 1e-5)) bad = 1;
  }
  // ---- case 2: a contraction chain with a flat pre-order tile list ------------
  {
    constexpr int K = 5;
    using V3d = Kokkos::View<float***, Kokkos::LayoutRight>;
    V3d A("A", E, N, K), B("B", K, N, N), C("C", N, N, N), R("R", E, N, N);
    for (int n = 0; n < E * N * K; ++n) A.data()[n] = std::sin(0.05f * n + 1.f);
    for (int n = 0; n < K * N * N; ++n) B.data()[n] = std::cos(0.13f * n);
    for (int n = 0; n < N * N * N; ++n) C.data()[n] = 0.01f * (n % 17) - 0.05f;
    // T(e, a, b, c) = sum_k A(e, a, k) B(k, b, c), then the contraction hook
    // T += 0.01 (a + 1) c at its global, declared-order coordinates; C passes
    // through an input hook C *= 1 + 0.1 d when staged
    auto T = make_contraction_node<'e', 'a', 'b', 'c'>(
        make_input_node(make_handle<'e', 'a', 'k'>(A)), make_input_node(make_handle<'k', 'b', 'c'>(B)),
        [](int, int a, int, int c, float& v) { v += 0.01f * static_cast<float>((a + 1) * c); });
    // R(e, a, d) = sum_{b,c} T(e,a,b,c) C(b,c,d)
    auto Rn = make_contraction_node<'e', 'a', 'd'>(
        T, make_input_node(make_handle<'b', 'c', 'd'>(C),
                           [](int, int, int d, float& v) { v *= 1.f + 0.1f * static_cast<float>(d); }));
    using BT = Tile<StaticTile<TE, N, K>, StaticTile<K, N, N>, StaticTile<TE, N, N, N>>;
    using BR = Tile<StaticTile<TE, N, N, N>, StaticTile<N, N, N>, StaticTile<TE, N, N>>;
    using Spec = typename b200::assembled_tile<0, decltype(Rn), std::tuple<BR, BT>>::type;
    static_assert(std::is_same_v<typename Spec::a_type, BT>, "the chain's A operand gets bundle 1");
    auto [g1, h] = make_graph().ops(Rn);
    (void)g1;
    (void)h;
    using TT = b200::tree_types<decltype(Rn), Spec>;
    using Dag = typename TT::dag_t;
    using Low = typename Dag::lowering;
    const auto dag = b200::TreeLowering<float, ES>::dag_of<Spec>(Rn);
    if (!dag.index_consistent()) {
      std::printf("chain: index_consistent false\n");
      return 1;
    }
    constexpr std::size_t S = Low::level_slot(Dag::num_slots() - 1);
    emulate<typename Low::label_tiles_t, typename Low::levels_t, S>(
        Low::make_levels(dag.nodes), (E + TE - 1) / TE, DeviceTuple<V3d>(R), 3);
    double worst = 0, scale = 1e-30;
    for (int e = 0; e < E; ++e)
      for (int a = 0; a < N; ++a)
        for (int d = 0; d < N; ++d) {
          double want = 0;
          for (int b = 0; b < N; ++b)
            for (int c = 0; c < N; ++c) {
              double t = 0;
              for (int k = 0; k < K; ++k) t += A(e, a, k) * B(k, b, c);
              t += 0.01 * (a + 1) * c;
              want += static_cast<float>(t) * (C(b, c, d) * (1.0 + 0.1 * d));
            }
          worst = std::fmax(worst, std::fabs(R(e, a, d) - want));
          scale = std::fmax(scale, std::fabs(want));
        }
    std::printf("chain max abs error %.3e (scale %.3e)\n", worst, scale);
    if (!(worst / scale < 1e-5)) bad = 1;
  }
  // ---- case 3: contracted labels spanning several tiles (ragged) -----------
  {
    constexpr int J = 6, K = 7, TI = 4, TL = 3, TJ = 4, TK = 3;
    const int I = E + 2, L = 5;
    using V3d = Kokkos::View<float***, Kokkos::LayoutRight>;
    using V2d = Kokkos::View<float**, Kokkos::LayoutRight>;
    V3d A("A", J, I, K), B("B", J, K, L);
    V2d Cm("C", L, I);
    for (int n = 0; n < J * I * K; ++n) A.data()[n] = std::sin(0.37f * n);
    for (int n = 0; n < J * K * L; ++n) B.data()[n] = std::cos(0.23f * n + 0.5f);
    // C[l, i] = sum_{j,k} A[j,i,k] B[j,k,l] + 1 (a hook applied once per element)
    auto Cn = make_contraction_node<'l', 'i'>(make_input_node(make_handle<'j', 'i', 'k'>(A)),
                                              make_input_node(make_handle<'j', 'k', 'l'>(B)),
                                              [](int, int, float& v) { v += 1.f; });
    using Spec = Tile<StaticTile<TJ, TI, TK>, StaticTile<TJ, TK, TL>, StaticTile<TL, TI>>;
    auto [g1, h] = make_graph().ops(Cn);
    (void)g1;
    (void)h;
    using TT = b200::tree_types<decltype(Cn), Spec>;
    using Dag = typename TT::dag_t;
    using Low = typename Dag::lowering_ktiled;
    static_assert(Low::num_levels == 1 && Low::NS == 0, "one self-staging contraction");
    const auto dag = b200::TreeLowering<float, ES>::dag_of<Spec>(Cn);
    if (!dag.needs_contracted_tiles()) {
      std::printf("ktiles: the contracted labels should span several tiles\n");
      return 1;
    }
    if (!dag.index_consistent()) {
      std::printf("ktiles: index_consistent false\n");
      return 1;
    }
    using GK = b200::GraphKernel<float, typename Low::label_tiles_t, typename Low::levels_t,
                                 Low::level_slot(Dag::num_slots() - 1)>;
    // grid over (i, l): canonical storage (i, l) -- freeA ++ freeB
    b200::GridRuntime<GK::GR> grid{};
    static_assert(GK::GR == 2);
    using GS = typename GK::GS;
    const int ext[2] = {GS::labels[0] == 'i' ? I : L, GS::labels[1] == 'i' ? I : L};
    const int til[2] = {GS::labels[0] == 'i' ? TI : TL, GS::labels[1] == 'i' ? TI : TL};
    grid.ntiles[0] = (ext[0] + til[0] - 1) / til[0];
    grid.ntiles[1] = (ext[1] + til[1] - 1) / til[1];
    const auto levels = Low::make_levels(dag.nodes);
    DeviceTuple<V2d> views(Cm);
    for (unsigned bx = 0; bx < static_cast<unsigned>(grid.ntiles[0] * grid.ntiles[1]); ++bx) {
      blockIdx.x = bx;
      GK::run(levels, grid, views);
    }
    double worst = 0, scale = 1e-30;
    for (int l = 0; l < L; ++l)
      for (int i = 0; i < I; ++i) {
        double want = 1.0;
        for (int j = 0; j < J; ++j)
          for (int k = 0; k < K; ++k) want += double(A(j, i, k)) * B(j, k, l);
        worst = std::fmax(worst, std::fabs(Cm(l, i) - want));
        scale = std::fmax(scale, std::fabs(want));
      }
    std::printf("ktiles max abs error %.3e (scale %.3e)\n", worst, scale);
    if (!(worst / scale < 1e-5)) bad = 1;
  }
  return bad;
}
