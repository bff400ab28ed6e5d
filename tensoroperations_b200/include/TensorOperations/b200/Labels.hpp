// Labels.hpp -- compile-time label algebra for the B200 frontend.
//
// A label is an int32_t (usually a character literal); a tensor's labels are a
// std::integer_sequence<int32_t, ...> in axis order.  Everything here is
// constexpr over small fixed arrays so that plans, permutations and strides
// are constants in device code.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <type_traits>
#include <utility>

#include <Kokkos_Core.hpp>

namespace TensorOperations {

template <int32_t... L>
using Labels = std::integer_sequence<int32_t, L...>;

namespace b200 {

template <class Seq>
struct seq_info;
template <int32_t... L>
struct seq_info<std::integer_sequence<int32_t, L...>> {
  static constexpr std::size_t size = sizeof...(L);
  static constexpr std::array<int32_t, sizeof...(L)> arr{L...};
};

template <class Seq>
constexpr auto to_array() {
  return seq_info<Seq>::arr;
}

template <std::size_t N>
constexpr int index_of(const std::array<int32_t, N>& a, int32_t l) {
  for (std::size_t i = 0; i < N; ++i)
    if (a[i] == l) return static_cast<int>(i);
  return -1;
}

template <std::size_t N>
constexpr bool all_distinct(const std::array<int32_t, N>& a) {
  for (std::size_t i = 0; i < N; ++i)
    for (std::size_t j = 0; j < i; ++j)
      if (a[i] == a[j]) return false;
  return true;
}

template <class A, class B>
constexpr bool same_label_set() {
  constexpr auto a = to_array<A>();
  constexpr auto b = to_array<B>();
  if constexpr (a.size() != b.size()) {
    return false;
  } else {
    for (std::size_t i = 0; i < a.size(); ++i)
      if (index_of(b, a[i]) < 0) return false;
    return true;
  }
}

// Labels of A that are not in B, in A's order.
template <class A, class B>
struct minus_labels {
  static constexpr auto a = to_array<A>();
  static constexpr auto b = to_array<B>();
  static constexpr std::size_t count() {
    std::size_t n = 0;
    for (std::size_t i = 0; i < a.size(); ++i)
      if (index_of(b, a[i]) < 0) ++n;
    return n;
  }
  static constexpr auto values() {
    std::array<int32_t, count()> out{};
    std::size_t n = 0;
    for (std::size_t i = 0; i < a.size(); ++i)
      if (index_of(b, a[i]) < 0) out[n++] = a[i];
    return out;
  }
};
// Labels of A that are also in B, in A's order.
template <class A, class B>
struct common_labels {
  static constexpr auto a = to_array<A>();
  static constexpr auto b = to_array<B>();
  static constexpr std::size_t count() {
    std::size_t n = 0;
    for (std::size_t i = 0; i < a.size(); ++i)
      if (index_of(b, a[i]) >= 0) ++n;
    return n;
  }
  static constexpr auto values() {
    std::array<int32_t, count()> out{};
    std::size_t n = 0;
    for (std::size_t i = 0; i < a.size(); ++i)
      if (index_of(b, a[i]) >= 0) out[n++] = a[i];
    return out;
  }
};

// constexpr std::array -> integer_sequence
template <auto Arr, class Idx = std::make_index_sequence<Arr.size()>>
struct array_seq;
template <auto Arr, std::size_t... I>
struct array_seq<Arr, std::index_sequence<I...>> {
  using type = std::integer_sequence<int32_t, static_cast<int32_t>(Arr[I])...>;
};
template <auto Arr>
using array_seq_t = typename array_seq<Arr>::type;

template <class A, class B>
struct concat_seq;
template <int32_t... X, int32_t... Y>
struct concat_seq<std::integer_sequence<int32_t, X...>, std::integer_sequence<int32_t, Y...>> {
  using type = std::integer_sequence<int32_t, X..., Y...>;
};

// Position in `To` of each label of `From` (From and To: same label set).
template <class From, class To>
constexpr auto label_positions() {
  constexpr auto f = to_array<From>();
  constexpr auto t = to_array<To>();
  std::array<int, f.size()> out{};
  for (std::size_t i = 0; i < f.size(); ++i) out[i] = index_of(t, f[i]);
  return out;
}

template <class Seq>
using labels_array_t = decltype(to_array<Seq>());

// int sequences (axis permutations)
template <class Seq>
struct iseq_info;
template <int... P>
struct iseq_info<std::integer_sequence<int, P...>> {
  static constexpr std::array<int, sizeof...(P)> arr{P...};
};
template <class Seq>
constexpr auto to_array_int() {
  return iseq_info<Seq>::arr;
}
template <auto Arr, class Idx = std::make_index_sequence<Arr.size()>>
struct array_iseq;
template <auto Arr, std::size_t... I>
struct array_iseq<Arr, std::index_sequence<I...>> {
  using type = std::integer_sequence<int, static_cast<int>(Arr[I])...>;
};
template <auto Arr>
using array_iseq_t = typename array_iseq<Arr>::type;

}  // namespace b200

// ---------------------------------------------------------------------------
// Static tiles: one compile-time extent per axis.
// ---------------------------------------------------------------------------
template <int... E>
struct StaticTile {
  static constexpr int rank = static_cast<int>(sizeof...(E));
  static constexpr int num_elements = (E * ... * 1);
  static constexpr std::array<int, sizeof...(E)> extents{E...};
  KOKKOS_INLINE_FUNCTION static constexpr int extent(int d) {
    constexpr int e[] = {E..., 0};
    return e[d];
  }
};

namespace b200 {
template <class T>
struct is_static_tile : std::false_type {};
template <int... E>
struct is_static_tile<StaticTile<E...>> : std::true_type {};

template <auto Arr, class Idx = std::make_index_sequence<Arr.size()>>
struct array_tile;
template <auto Arr, std::size_t... I>
struct array_tile<Arr, std::index_sequence<I...>> {
  using type = StaticTile<static_cast<int>(Arr[I])...>;
};
template <auto Arr>
using array_tile_t = typename array_tile<Arr>::type;

// Row-major strides of a static tile.
template <class Tile>
constexpr auto tile_strides() {
  std::array<int, Tile::rank> s{};
  int acc = 1;
  for (int d = Tile::rank - 1; d >= 0; --d) {
    s[d] = acc;
    acc *= Tile::extents[d];
  }
  return s;
}
}  // namespace b200

}  // namespace TensorOperations
