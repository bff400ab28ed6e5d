// LabelTiles.hpp -- one tile extent per label for a whole level graph.
//
// Public surface as in the reference (include/TensorOperations/LabelTiles.hpp:32-63,
// 108-121, 211-212): LabelTile<L, E> marks a BLOCKED label (a grid mode, one
// team per tile), LabelWhole<L, E> a label whose single tile spans the axis;
// LabelTiles<...> is the map; tile_from_labels_t<Map, Labels> is the tile a
// node with those labels gets.  The two map guards carry the reference's
// diagnostics (a duplicated label, a label missing from the map).
#pragma once

#include <TensorOperations/b200/Labels.hpp>

namespace TensorOperations {

template <int32_t Label, int Extent>
struct LabelTile {
  static constexpr int32_t label = Label;
  static constexpr int extent = Extent;
  static constexpr bool gridded = true;
  static_assert(Extent > 0, "LabelTile: a tile extent must be positive");
};

template <int32_t Label, int Extent>
struct LabelWhole {
  static constexpr int32_t label = Label;
  static constexpr int extent = Extent;
  static constexpr bool gridded = false;
  static_assert(Extent > 0, "LabelWhole: an extent must be positive");
};

template <typename... Entries>
struct LabelTiles {
  static constexpr std::size_t size = sizeof...(Entries);
  static constexpr std::array<int32_t, sizeof...(Entries)> labels{Entries::label...};
  static constexpr std::array<int, sizeof...(Entries)> extents{Entries::extent...};
  static constexpr std::array<bool, sizeof...(Entries)> gridded{Entries::gridded...};

  static constexpr bool distinct() { return b200::all_distinct(labels); }
  // Tile of a label, -1 if the label is not in the map.
  static constexpr int tile(int32_t l) {
    const int i = b200::index_of(labels, l);
    return i < 0 ? -1 : extents[i];
  }
  static constexpr bool is_gridded(int32_t l) {
    const int i = b200::index_of(labels, l);
    return i >= 0 && gridded[i];
  }
};

namespace Impl {
template <typename LT, typename ModesSeq>
struct TileFromLabels;
template <typename LT, int32_t... Modes>
struct TileFromLabels<LT, std::integer_sequence<int32_t, Modes...>> {
  static_assert(LT::distinct(), "LabelTiles: a label may appear at most once in the map");
  static_assert(((LT::tile(Modes) > 0) && ...),
                "LabelTiles: every label a node carries must appear in the graph's tile "
                "map -- an absent label has no tile extent to give, and defaulting one "
                "would silently change the iteration space");
  using type = StaticTile<LT::tile(Modes)...>;
};
}  // namespace Impl

template <typename LT, typename ModesSeq>
using tile_from_labels_t = typename Impl::TileFromLabels<LT, ModesSeq>::type;

template <typename LT>
using label_seq_t = b200::array_seq_t<LT::labels>;

template <typename LT>
using grid_tile_t = tile_from_labels_t<LT, label_seq_t<LT>>;

}  // namespace TensorOperations
