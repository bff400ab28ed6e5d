// TileSpec.hpp -- per-node tile bundles of the flat-DAG route.
//
// Public surface as the reference (include/TensorOperations/Tiling.hpp:
// Tile<TileA, TileB, TileC> :985-990, output_tile :1000-1014, CombineTile
// :1039-1050):
//   Tile<TA, TB, TC>          a contraction's tiles: A's and B's in their own
//                             label order, the output's in its DECLARED order;
//   CombineTile<Out, Ops...>  a combine's output tile plus one tile per operand
//                             (an operand's tile in that operand's label order);
//   a plain StaticTile        a combine's output tile, every operand staged in
//                             the output's order.
// On the tree route (Graph::execute) the bundles nest like the expression: an
// operand that is itself a node carries that node's bundle (a Tile<...> for a
// contraction, a CombineTile<...> for a combine) in place of its plain tile.
// Only static extents exist on this route: every tile is a compile-time
// constant of the device evaluator.
#pragma once

#include <tuple>

#include <TensorOperations/b200/Labels.hpp>

namespace TensorOperations {

template <typename TileA, typename TileB, typename TileC>
struct Tile {
  using a_type = TileA;
  using b_type = TileB;
  using c_type = TileC;
  TileA a{};
  TileB b{};
  TileC c{};
};

template <typename OutTile, typename... OpTiles>
struct CombineTile {
  using out_type = OutTile;
  using op_types = std::tuple<OpTiles...>;
  static constexpr int rank = OutTile::rank;
  static constexpr bool is_static = true;
  static constexpr int num_ops = static_cast<int>(sizeof...(OpTiles));
  OutTile out{};
  KOKKOS_INLINE_FUNCTION static constexpr int extent(int i) { return OutTile::extent(i); }
};

// make_combine_tile(out, op_tiles...) -- the bundle for a combine whose
// operands are nested nodes (reference Tiling.hpp:1070-1074).
template <typename OutTile, typename... OpTiles>
constexpr CombineTile<OutTile, OpTiles...> make_combine_tile(const OutTile&, const OpTiles&...) {
  return CombineTile<OutTile, OpTiles...>{};
}

template <typename TileA, typename TileB, typename TileC>
KOKKOS_INLINE_FUNCTION constexpr TileC output_tile(const Tile<TileA, TileB, TileC>&) noexcept {
  return TileC{};
}
template <int... E>
KOKKOS_INLINE_FUNCTION constexpr StaticTile<E...> output_tile(StaticTile<E...> t) noexcept {
  return t;
}
template <typename OutTile, typename... OpTiles>
KOKKOS_INLINE_FUNCTION constexpr OutTile output_tile(const CombineTile<OutTile, OpTiles...>&) noexcept {
  return OutTile{};
}

namespace b200 {
template <class T>
struct is_contraction_tile : std::false_type {};
template <class A, class B, class C>
struct is_contraction_tile<Tile<A, B, C>> : std::true_type {};
template <class T>
struct is_combine_tile : std::false_type {};
template <class O, class... Ops>
struct is_combine_tile<CombineTile<O, Ops...>> : std::true_type {};

// The output tile of a combine's tile spec (a CombineTile or a plain tile).
template <class T, bool = is_combine_tile<T>::value>
struct combine_out_tile {
  using type = T;
};
template <class T>
struct combine_out_tile<T, true> {
  using type = typename T::out_type;
};
}  // namespace b200

}  // namespace TensorOperations
