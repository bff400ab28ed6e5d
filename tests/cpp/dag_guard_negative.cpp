// dag_guard_negative.cpp -- each NEG_CASE builds a flat DAG that one of the
// DagGraph diagnostics forbids; NEG_CASE=0 is the legal control graph.
// Compiled with -fsyntax-only by tests/test_frontend_cpu.py, which checks that
// exactly the expected diagnostic fires.
#include <Kokkos_Core.hpp>
#include <TensorOperations/DagGraph.hpp>
#include <TensorOperations/Tiling.hpp>

using namespace TensorOperations;
using ES = Kokkos::DefaultExecutionSpace;
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;
using V3 = Kokkos::View<float***, Kokkos::LayoutRight>;

using TA = StaticTile<4, 4>;       // (q, p)
using TB = StaticTile<2, 4, 4>;    // (e, y, p)
using TC = StaticTile<4, 2, 4>;    // (q, e, y)
using TCe = StaticTile<2, 4, 4>;   // (e, y, q) declared order

#ifndef NEG_CASE
#define NEG_CASE 0
#endif

bool control(V2 A, V3 B) {
  auto c = make_contraction_node<'q', 'e', 'y'>(make_input_node(make_handle<'q', 'p'>(A)),
                                                make_input_node(make_handle<'e', 'y', 'p'>(B)));
#if NEG_CASE == 1
  // a contraction's tile must be a Tile<A, B, C> bundle
  auto [g0, h] = make_dag<float, ES>().add(c, TC{});
#elif NEG_CASE == 3
  // the declared output tile disagrees with what the operands imply
  auto [g0, h] = make_dag<float, ES>().add(c, Tile<TA, TB, StaticTile<4, 2, 2>>{});
#else
  auto [g0, h] = make_dag<float, ES>().add(c, Tile<TA, TB, TC>{});
#endif
  auto sq = KOKKOS_LAMBDA(int, int, int, float v) { return v * v; };
#if NEG_CASE == 2
  // a handle of ANOTHER graph (slot 5 of a graph that has one slot)
  b200::DagSlotHandle<5, float, ES, Labels<'q', 'e', 'y'>, TC> stray{};
  auto [g1, r] = g0.add(make_combine_node<'q', 'e', 'y'>(stray.template as<'q', 'e', 'y'>(), sq), TC{});
#elif NEG_CASE == 4
  // a handle operand named with a tile its producer was not given
  auto [g1, r] = g0.add(make_combine_node<'q', 'e', 'y'>(h.template as<'q', 'e', 'y'>(), sq),
                        StaticTile<4, 1, 4>{});
#elif NEG_CASE == 3
  auto [g1, r] = g0.add(make_combine_node<'q', 'e', 'y'>(h.template as<'q', 'e', 'y'>(), sq),
                        StaticTile<4, 2, 2>{});
#else
  auto [g1, r] = g0.add(make_combine_node<'q', 'e', 'y'>(h.template as<'q', 'e', 'y'>(), sq), TC{});
#endif
  (void)r;
  return g1.index_consistent();
}
