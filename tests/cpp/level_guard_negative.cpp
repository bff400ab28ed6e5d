// level_guard_negative.cpp -- level graphs that MUST NOT compile.
//
// Each case builds, through the public factories, a graph one of the planner's
// guards forbids and names its LevelPlan; tests/test_frontend_cpu.py compiles
// every case with -DNEG_CASE=<n> and requires the build to fail with THAT
// guard's own diagnostic (the same wording the reference's
// tests/negative/level_guard_negative.cpp and labeltiles_guard_negative.cpp
// pin).  Case 0 is the control and must compile.
//   1  a level mixing a contraction and a combine           (HOMOGENEOUS)
//   2  contraction members whose SA disagree                (ONE iteration space)
//   3  combine members whose output tiles disagree          (ONE iteration space)
//   4  a member reading a slot its own level produces       (ITS OWN LEVEL)
//   5  staged members of different rank                     (ONE iteration space)
//   6  a label named twice in the LabelTiles map            (at most once)
//   7  a node carrying a label the map does not name        (must appear)
#include <Kokkos_Core.hpp>
#include <TensorOperations/LevelGraph.hpp>

#ifndef NEG_CASE
#error "define NEG_CASE"
#endif

using namespace TensorOperations;
using ES = Kokkos::DefaultExecutionSpace;
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;
using V4 = Kokkos::View<float****, Kokkos::LayoutRight>;

constexpr int kN = 5, kTE = 4, kOdd = 7;
using Map = LabelTiles<LabelTile<'e', kTE>, LabelWhole<'q', kN>, LabelWhole<'r', kOdd>,
                       LabelWhole<'a', kN>, LabelWhole<'b', kN>, LabelWhole<'c', kN>>;

struct Id4 {
  KOKKOS_FUNCTION float operator()(int, int, int, int, float v) const { return v; }
};
struct Id2 {
  KOKKOS_FUNCTION float operator()(int, int, float v) const { return v; }
};

template <class G>
void plan_of(const G&) {
  using Plan = LevelPlan<typename G::levels_type>;
  (void)sizeof(Plan);
}

int main() {
  V2 H("H", kN, kN), R("R", kOdd, kN);
  V4 U("U", 8, kN, kN, kN);
#if NEG_CASE == 6
  using Bad = LabelTiles<LabelTile<'e', kTE>, LabelWhole<'a', kN>, LabelWhole<'e', kN>>;
  auto g0 = make_level_graph<float, ES>(Bad{});
  auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'e', 'a'>(H))));
  plan_of(g1);
#elif NEG_CASE == 7
  using Small = LabelTiles<LabelTile<'e', kTE>, LabelWhole<'a', kN>>;
  auto g0 = make_level_graph<float, ES>(Small{});
  auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(H))));
  plan_of(g1);
#else
  auto g0 = make_level_graph<float, ES>(Map{});
  auto [g1a, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(H))));
  auto [g1, r] = g1a.add(make_stage_node(make_input_node(make_handle<'r', 'a'>(R))));
  auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(U))));
  auto ga = make_contraction_node<'q', 'e', 'b', 'c'>(h, u);
  auto gb = make_contraction_node<'q', 'e', 'a', 'c'>(h.as<'q', 'b'>(), u);
#if NEG_CASE == 0
  auto [g3, sa, sb] = g2.add(ga, gb);
  auto [g4, c0, c1] = g3.add(make_combine_node<'q', 'e', 'b', 'c'>(sa, Id4{}),
                             make_combine_node<'q', 'e', 'a', 'c'>(sb, Id4{}));
  plan_of(g4);
#elif NEG_CASE == 1
  auto [g3, sa] = g2.add(ga);
  auto [g4, x, y] = g3.add(make_contraction_node<'q', 'e', 'b', 'c'>(h, u),
                           make_combine_node<'q', 'e', 'b', 'c'>(sa, Id4{}));
  plan_of(g4);
#elif NEG_CASE == 2
  auto gr = make_contraction_node<'r', 'e', 'b', 'c'>(r, u);
  auto [g3, sa, sr] = g2.add(ga, gr);
  plan_of(g3);
#elif NEG_CASE == 3
  auto [g3, sa] = g2.add(ga);
  auto [g4, p] = g3.add(make_contraction_node<'q', 'r'>(h, r));
  auto [g5, c4, c2] = g4.add(make_combine_node<'q', 'e', 'b', 'c'>(sa, Id4{}),
                             make_combine_node<'q', 'r'>(p, Id2{}));
  plan_of(g5);
#elif NEG_CASE == 4
  // A handle to slot 3 (the member about to be added at level 3) obtained from
  // a twin graph, then read by that very level.
  auto [twin, own] = g2.add(ga);
  auto [g3, self] = g2.add(make_combine_node<'q', 'e', 'b', 'c'>(own, Id4{}));
  (void)twin;
  plan_of(g3);
#elif NEG_CASE == 5
  auto [g3, x, y] = g2.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(H))),
                           make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(U))));
  plan_of(g3);
#endif
#endif
  return 0;
}
