// frontend_static.cpp -- compile-time checks of the level-graph planner.
//
// Mostly static_asserts, compiled by g++ (host only) in tests/test_frontend_cpu.py.
// It restates, in this repository's own code, the claims the reference pins in
// tests/test_level_graph.cpp (slot algebra with mixed arities, tile derivation,
// declared-order storage) and benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp
// (the SEM3D plan: 6 levels, 35 slots, 19 pools).
#include <Kokkos_Core.hpp>
#include <TensorOperations/LevelGraph.hpp>

#include <cstdio>

using namespace TensorOperations;
using ES = Kokkos::DefaultExecutionSpace;

// ---- 1. slot algebra over mixed arities -------------------------------------
template <int N>
struct Multi {
  static constexpr int NumOut = N;
};
struct Single {};
using Lv0 = DeviceTuple<Single, Single, Single>;
using Lv1 = DeviceTuple<Multi<3>, Single>;
using Lv2 = DeviceTuple<Multi<2>>;
using Synth = DeviceTuple<Lv0, Lv1, Lv2>;
using Alg = b200::Algebra<Synth>;
static_assert(Alg::total_members == 6);
static_assert(Alg::num_slots == 9, "3 + 4 + 2 slots");
static_assert(Alg::level_base(0) == 0 && Alg::level_base(1) == 3 && Alg::level_base(2) == 7);
static_assert(Alg::member_base(1, 0) == 3);
static_assert(Alg::member_base(1, 1) == 6, "member 1 of level 1 starts 3 slots in (arity 3)");
static_assert(Alg::member_base(2, 0) == 7);
static_assert(Alg::slot_level(5) == 1 && Alg::slot_member(5) == 0,
              "a middle slot of a 3-output member belongs to that member");
static_assert(Alg::slot_level(6) == 1 && Alg::slot_member(6) == 1);
static_assert(Alg::slot_level(8) == 2 && Alg::slot_member(8) == 0);
static_assert(b200::Algebra<DeviceTuple<>>::num_slots == 0);

// ---- 2. tile derivation and declared order through the public factories -----
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;
using V4 = Kokkos::View<float****, Kokkos::LayoutRight>;
constexpr int kQ = 7, kA = 3, kB = 4, kC = 5, kTE = 2;
using MapD = LabelTiles<LabelWhole<'q', kQ>, LabelWhole<'a', kA>, LabelWhole<'b', kB>,
                        LabelWhole<'c', kC>, LabelTile<'e', kTE>>;

template <int Dummy>
auto declared_graph() {
  V2 H("H", kQ, kA);
  V4 U("U", 8, kA, kB, kC);
  auto g0 = make_level_graph<float, ES>(MapD{});
  auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(H))));
  auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(U))));
  auto c = make_contraction_node<'e', 'b', 'q', 'c'>(h, u);  // canonical (q, e, b, c)
  auto [g3, s] = g2.add(c);
  return std::make_tuple(g3, c, s);
}
using DG = decltype(declared_graph<0>());
using Cnx = std::tuple_element_t<1, DG>;
using CnxSlot = std::tuple_element_t<2, DG>;
static_assert(std::is_same_v<b200::member_traits<Cnx>::tile, StaticTile<kQ, kTE, kB, kC>>,
              "canonical tile: freeA (q) then freeB (e, b, c)");
static_assert(std::is_same_v<typename CnxSlot::modes_seq, Labels<'e', 'b', 'q', 'c'>>,
              "the handle carries the DECLARED labels");
static_assert(b200::to_array_int<typename CnxSlot::decl_to_storage_seq>() ==
                  std::array<int, 4>{1, 2, 0, 3},
              "declared axis -> canonical storage axis");
static_assert(b200::operand_label_stride<CnxSlot>('q') == kTE * kB * kC);
static_assert(b200::operand_label_stride<CnxSlot>('c') == 1);
static_assert(CnxSlot::SlotIdx == 2, "stage H, stage U, then the contraction");
using Relab = decltype(std::declval<CnxSlot>().template as<'b', 'q', 'e', 'c'>());
static_assert(b200::operand_label_stride<Relab>('b') == kB * kC &&
                  b200::operand_label_stride<Relab>('q') == kC &&
                  b200::operand_label_stride<Relab>('e') == kTE * kB * kC,
              "as<>() renames positions: position 0 (declared e, now named b) is still "
              "canonical axis 1, position 2 (declared q, now named e) canonical axis 0");

// ---- 3. the SEM3D plan (the reference program's static_asserts) -------------
using V4s = Kokkos::View<float* [5][5][5], Kokkos::LayoutRight>;
template <int TE>
using GMap = LabelTiles<LabelTile<'e', TE>, LabelWhole<'k', 5>, LabelWhole<'j', 5>,
                        LabelWhole<'i', 5>, LabelWhole<'p', 5>, LabelWhole<'r', 5>>;
struct Integrand {
  KOKKOS_FUNCTION Kokkos::Array<float, 9> operator()(int, int, int, int, float a, float b,
                                                     float c, float d, float e, float f, float g,
                                                     float h, float i) const {
    return {a, b, c, d, e, f, g, h, i};
  }
};
struct WSum {
  KOKKOS_FUNCTION float operator()(int, int, int, int, float a, float b, float c) const {
    return a + b + c;
  }
};

template <int TE>
auto sem3d_graph(int E) {
  V2 H("H", 5, 5), Hw("Hw", 5, 5);
  V4s u0("u0", E), u1("u1", E), u2("u2", E);
  auto g0 = make_level_graph<float, ES>(GMap<TE>{});
  auto [g1, h, hw] = g0.add(make_stage_node(make_input_node(make_handle<'r', 'p'>(H))),
                            make_stage_node(make_input_node(make_handle<'p', 'r'>(Hw))));
  auto [g2, a, b, c] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'k', 'j', 'i'>(u0))),
                              make_stage_node(make_input_node(make_handle<'e', 'k', 'j', 'i'>(u1))),
                              make_stage_node(make_input_node(make_handle<'e', 'k', 'j', 'i'>(u2))));
  auto gx = [&](auto x) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(h.template as<'i', 'p'>(),
                                                     x.template as<'e', 'k', 'j', 'p'>());
  };
  auto ge = [&](auto x) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(h.template as<'j', 'p'>(),
                                                     x.template as<'e', 'k', 'p', 'i'>());
  };
  auto gg = [&](auto x) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(h.template as<'k', 'p'>(),
                                                     x.template as<'e', 'p', 'j', 'i'>());
  };
  auto [g3, x0, x1, x2, e0, e1, e2, y0, y1, y2] =
      g2.add(gx(a), gx(b), gx(c), ge(a), ge(b), ge(c), gg(a), gg(b), gg(c));
  auto [g4, f0, f1, f2, f3, f4, f5, f6, f7, f8] = g3.add(
      make_combine_node<'e', 'k', 'j', 'i'>(x0, x1, x2, e0, e1, e2, y0, y1, y2, Integrand{}));
  auto dx = [&](auto f) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(hw.template as<'p', 'i'>(),
                                                     f.template as<'e', 'k', 'j', 'p'>());
  };
  auto de = [&](auto f) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(hw.template as<'p', 'j'>(),
                                                     f.template as<'e', 'k', 'p', 'i'>());
  };
  auto dg = [&](auto f) {
    return make_contraction_node<'e', 'k', 'j', 'i'>(hw.template as<'p', 'k'>(),
                                                     f.template as<'e', 'p', 'j', 'i'>());
  };
  auto [g5, t0, t1, t2, t3, t4, t5, t6, t7, t8] =
      g4.add(dx(f0), dx(f1), dx(f2), de(f3), de(f4), de(f5), dg(f6), dg(f7), dg(f8));
  auto [g6, r0, r1, r2] = g5.add(make_combine_node<'e', 'k', 'j', 'i'>(t0, t3, t6, WSum{}),
                                 make_combine_node<'e', 'k', 'j', 'i'>(t1, t4, t7, WSum{}),
                                 make_combine_node<'e', 'k', 'j', 'i'>(t2, t5, t8, WSum{}));
  using Plan = LevelPlan<typename decltype(g6)::levels_type>;
  static_assert(Plan::num_levels == 6);
  static_assert(Plan::num_slots == 2 + 3 + 9 + 9 + 9 + 3);
  static_assert(Plan::num_members == 2 + 3 + 9 + 1 + 9 + 3);
  static_assert(decltype(g6.outputs(r0, r1, r2))::num_pools == 19,
                "19 = Hw + 9 gradients + 9 integrands, the widest overlap, which left-edge "
                "colouring attains");
  return g6.outputs(r0, r1, r2);
}

int main() {
  int rc = 0;
  const auto o1 = sem3d_graph<1>(4);
  const auto o8 = sem3d_graph<8>(16);
  std::printf("sem3d TE=1 pooled %zu B unpooled %zu B; TE=8 pooled %zu B; pools %zu; "
              "index_consistent %d\n",
              o1.scratch_bytes(), o1.slot_bytes(), o8.scratch_bytes(),
              decltype(o1)::num_pools, int(o1.graph.index_consistent()));
  if (!(o1.scratch_bytes() < o1.slot_bytes())) rc = 1;
  if (!o1.graph.index_consistent()) rc = 1;
  return rc;
}
