// Plan.hpp -- everything the level graph knows before anything runs.
//
// Semantics follow the reference's LevelPlan (include/TensorOperations/LevelPlan.hpp):
//   * slots are numbered level by level, member by member, output by output
//     (a multi-output combine advances the cursor by its arity);
//   * liveness is on the LEVEL timeline with closed ranges: a slot is live from
//     the level that writes it to the last level that reads it, a root until
//     after the last level (the root store) -- members of one level run
//     interleaved, so ranking them inside a level would be unsound;
//   * slots whose ranges do not overlap share a pool; pools are assigned by
//     left-edge colouring in slot order, which is optimal for interval graphs;
//   * three level guards: homogeneous non-empty levels, one iteration space
//     per level, no member reading its own level's output.
// The implementation is this library's: one constexpr table per graph type.
#pragma once

#include <TensorOperations/LabelTiles.hpp>
#include <TensorOperations/b200/Nodes.hpp>

namespace TensorOperations {
namespace b200 {

// Tile extent of label l in a slot operand (its declared axes renamed by as<>()).
template <class X>
constexpr int operand_label_extent(int32_t l) {
  constexpr auto lab = to_array<typename X::modes_seq>();
  constexpr auto perm = to_array_int<typename X::decl_to_storage_seq>();
  using ST = typename X::storage_tile;
  const int d = index_of(lab, l);
  return d < 0 ? -1 : ST::extents[perm[d]];
}
// Storage stride (elements) of label l in a slot operand, -1 if absent.
template <class X>
constexpr int operand_label_stride(int32_t l) {
  constexpr auto lab = to_array<typename X::modes_seq>();
  constexpr auto perm = to_array_int<typename X::decl_to_storage_seq>();
  constexpr auto st = tile_strides<typename X::storage_tile>();
  const int d = index_of(lab, l);
  return d < 0 ? -1 : st[perm[d]];
}

template <class Node, class Tag = typename Node::node_tag>
struct member_traits;

template <class Node>
struct member_traits<Node, StagedTag> {
  static_assert(!std::is_void_v<typename Node::tile_type>,
                "level graph: a stage member's tile is resolved by LevelGraph::add");
  static constexpr int kind = 0;
  static constexpr int num_out = 1;
  static constexpr int rank = Node::Rank;
  using storage_labels = typename Node::modes_seq;
  using decl_labels = storage_labels;
  using tile = typename Node::tile_type;
  static constexpr auto decl_to_storage = [] {
    std::array<int, Node::Rank> p{};
    for (int d = 0; d < Node::Rank; ++d) p[d] = d;
    return p;
  }();
  static constexpr std::array<std::size_t, 0> reads{};
};

template <class Node>
struct member_traits<Node, ContractionTag> {
  using A = typename Node::node_a_type;
  using B = typename Node::node_b_type;
  static_assert(is_slot_v<A> && is_slot_v<B>,
                "level graph: contraction operands must be handles returned by "
                "LevelGraph::add (slots)");
  static constexpr int kind = 1;
  static constexpr int num_out = 1;
  static constexpr int rank = Node::Rank;
  using storage_labels = typename Node::canon_seq;
  using decl_labels = typename Node::decl_seq;
  static constexpr auto extents = [] {
    std::array<int, Node::Rank> e{};
    for (int d = 0; d < Node::FreeA; ++d) e[d] = operand_label_extent<A>(Node::freeA[d]);
    for (int d = 0; d < Node::FreeB; ++d)
      e[Node::FreeA + d] = operand_label_extent<B>(Node::freeB[d]);
    return e;
  }();
  using tile = array_tile_t<extents>;
  static constexpr auto decl_to_storage =
      label_positions<typename Node::decl_seq, typename Node::canon_seq>();
  static constexpr std::array<std::size_t, 2> reads{A::SlotIdx, B::SlotIdx};
  static constexpr int sa = [] {
    int s = 1;
    for (int d = 0; d < Node::FreeA; ++d) s *= extents[d];
    return s;
  }();
  static constexpr int sb = [] {
    int s = 1;
    for (int d = 0; d < Node::FreeB; ++d) s *= extents[Node::FreeA + d];
    return s;
  }();
  static constexpr int sk = [] {
    int s = 1;
    for (int d = 0; d < Node::NumContracted; ++d) {
      const int ea = operand_label_extent<A>(Node::contracted[d]);
      const int eb = operand_label_extent<B>(Node::contracted[d]);
      s *= ea;
      if (ea != eb) return -1;
    }
    return s;
  }();
  static_assert(sk > 0,
                "level graph: a contracted label has different tile extents in A and B");
};

template <class Node>
struct member_traits<Node, CombineTag> {
  using Ops = typename Node::ops_tuple_t;
  using Op0 = tuple_element_t<0, Ops>;
  template <std::size_t... K>
  static constexpr bool all_slots(std::index_sequence<K...>) {
    return (is_slot_v<tuple_element_t<K, Ops>> && ...);
  }
  static_assert(all_slots(std::make_index_sequence<Node::NumOps>{}),
                "level graph: combine operands must be handles returned by LevelGraph::add "
                "(slots)");
  static constexpr int kind = 2;
  static constexpr int num_out = Node::NumOut;
  static constexpr int rank = Node::Rank;
  using storage_labels = typename Node::modes_seq;
  using decl_labels = storage_labels;
  static constexpr auto extents = [] {
    constexpr auto o = to_array<typename Node::modes_seq>();
    std::array<int, Node::Rank> e{};
    for (int d = 0; d < Node::Rank; ++d) e[d] = operand_label_extent<Op0>(o[d]);
    return e;
  }();
  using tile = array_tile_t<extents>;
  static constexpr auto decl_to_storage = [] {
    std::array<int, Node::Rank> p{};
    for (int d = 0; d < Node::Rank; ++d) p[d] = d;
    return p;
  }();
  template <std::size_t... K>
  static constexpr std::array<std::size_t, sizeof...(K)> reads_of(std::index_sequence<K...>) {
    return {tuple_element_t<K, Ops>::SlotIdx...};
  }
  static constexpr auto reads = reads_of(std::make_index_sequence<Node::NumOps>{});
  template <std::size_t... K>
  static constexpr bool tiles_agree(std::index_sequence<K...>) {
    constexpr auto o = to_array<typename Node::modes_seq>();
    for (int d = 0; d < Node::Rank; ++d)
      if (((operand_label_extent<tuple_element_t<K, Ops>>(o[d]) != extents[d]) || ...))
        return false;
    return true;
  }
  static_assert(tiles_agree(std::make_index_sequence<Node::NumOps>{}),
                "combine node: operand tiles must match on every mode");
};

// A staged contraction (kind 3): a contraction of two INPUT operands whose
// member stages both operand tiles itself, once per tile of the contracted
// labels, and accumulates (reference Team.hpp Spec 4: the contracted modes may
// be tiled).  Its three slots are the output and the two operand tiles; it
// reads no slot of any other member.
template <class Node>
struct member_traits<Node, StagedContractionTag> {
  using C = typename Node::contraction_type;
  using CT = member_traits<C, ContractionTag>;
  static constexpr int kind = 3;
  static constexpr int num_out = 3;
  static constexpr int rank = CT::rank;
  using storage_labels = typename CT::storage_labels;
  using decl_labels = typename CT::decl_labels;
  using tile = typename CT::tile;
  static constexpr auto decl_to_storage = CT::decl_to_storage;
  static constexpr std::array<std::size_t, 0> reads{};
  static constexpr int sa = CT::sa, sb = CT::sb, sk = CT::sk;
  static constexpr std::size_t out_elems(std::size_t o) {
    return o == 0 ? std::size_t(tile::num_elements)
                  : (o == 1 ? std::size_t(C::node_a_type::storage_tile::num_elements)
                            : std::size_t(C::node_b_type::storage_tile::num_elements));
  }
};

// Elements of output o of a member (every output of other kinds has the
// member's tile).
template <class Node>
constexpr std::size_t member_out_elems(std::size_t o) {
  using MT = member_traits<Node>;
  if constexpr (requires { MT::out_elems(o); })
    return MT::out_elems(o);
  else
    return static_cast<std::size_t>(MT::tile::num_elements);
}

template <class Node>
constexpr int output_arity() {
  if constexpr (requires { Node::NumOut; })
    return Node::NumOut;
  else
    return 1;
}

// Slots a member occupies in the level plan: its outputs, plus the two
// operand tiles of a staged contraction.
template <class Node>
constexpr int member_slots() {
  if constexpr (requires { typename Node::node_tag; }) {
    if constexpr (std::is_same_v<typename Node::node_tag, StagedContractionTag>) return 3;
  }
  return output_arity<Node>();
}

// ---------------------------------------------------------------------------
// Slot algebra over a level list.
// ---------------------------------------------------------------------------
template <class Levels>
struct Algebra {
  static constexpr std::size_t NL = tuple_size_v<Levels>;

  template <std::size_t... L>
  static constexpr std::array<std::size_t, sizeof...(L)> counts(std::index_sequence<L...>) {
    return {tuple_size_v<tuple_element_t<L, Levels>>...};
  }
  static constexpr auto member_counts = counts(std::make_index_sequence<NL>{});

  static constexpr std::size_t total_members = [] {
    std::size_t n = 0;
    for (std::size_t c : member_counts) n += c;
    return n;
  }();

  template <class Lvl, std::size_t... M>
  static constexpr std::array<std::size_t, sizeof...(M)> level_arities(std::index_sequence<M...>) {
    return {static_cast<std::size_t>(member_slots<tuple_element_t<M, Lvl>>())...};
  }
  template <std::size_t L>
  static constexpr auto arities_of() {
    using Lvl = tuple_element_t<L, Levels>;
    return level_arities<Lvl>(std::make_index_sequence<tuple_size_v<Lvl>>{});
  }
  template <std::size_t... L>
  static constexpr std::array<std::size_t, total_members> flat(std::index_sequence<L...>) {
    std::array<std::size_t, total_members> out{};
    std::size_t pos = 0;
    ((
         [&] {
           for (std::size_t a : arities_of<L>()) out[pos++] = a;
         }()),
     ...);
    return out;
  }
  static constexpr auto flat_arities = flat(std::make_index_sequence<NL>{});

  static constexpr std::size_t num_slots = [] {
    std::size_t n = 0;
    for (std::size_t a : flat_arities) n += a;
    return n;
  }();

  static constexpr std::size_t member_offset(std::size_t l) {
    std::size_t o = 0;
    for (std::size_t i = 0; i < l; ++i) o += member_counts[i];
    return o;
  }
  static constexpr std::size_t level_base(std::size_t l) {
    std::size_t o = 0, m = 0;
    for (std::size_t i = 0; i < l; ++i)
      for (std::size_t k = 0; k < member_counts[i]; ++k) o += flat_arities[m++];
    return o;
  }
  static constexpr std::size_t member_base(std::size_t l, std::size_t m) {
    std::size_t o = level_base(l);
    const std::size_t f = member_offset(l);
    for (std::size_t k = 0; k < m; ++k) o += flat_arities[f + k];
    return o;
  }
  static constexpr std::size_t slot_level(std::size_t s) {
    for (std::size_t l = 0; l < NL; ++l)
      if (s < level_base(l + 1)) return l;
    return NL;
  }
  static constexpr std::size_t slot_member(std::size_t s) {
    const std::size_t l = slot_level(s);
    if (l >= NL) return 0;
    std::size_t end = level_base(l);
    const std::size_t f = member_offset(l);
    for (std::size_t m = 0; m < member_counts[l]; ++m) {
      end += flat_arities[f + m];
      if (s < end) return m;
    }
    return member_counts[l];
  }
};

template <class Levels, std::size_t S>
struct slot_member_node {
  using Alg = Algebra<Levels>;
  static constexpr std::size_t L = Alg::slot_level(S);
  static constexpr std::size_t M = Alg::slot_member(S);
  using type = tuple_element_t<M, tuple_element_t<L, Levels>>;
  static constexpr std::size_t out = S - Alg::member_base(L, M);
};

// ---------------------------------------------------------------------------
// Liveness on the level timeline and left-edge pooling.
// ---------------------------------------------------------------------------
template <class Levels, std::size_t... Roots>
struct Pooling {
  using Alg = Algebra<Levels>;
  static constexpr std::size_t NS = Alg::num_slots;
  static constexpr std::size_t NL = Alg::NL;

  template <std::size_t L, std::size_t... M>
  static constexpr void note_level(std::array<std::size_t, NS>& last, std::index_sequence<M...>) {
    ((
         [&] {
           for (std::size_t s : member_traits<tuple_element_t<M, tuple_element_t<L, Levels>>>::reads)
             if (s + 1 <= NS && last[s] + 1 <= L) last[s] = L;
         }()),
     ...);
  }
  template <std::size_t... L>
  static constexpr void note_all(std::array<std::size_t, NS>& last, std::index_sequence<L...>) {
    (note_level<L>(last, std::make_index_sequence<tuple_size_v<tuple_element_t<L, Levels>>>{}), ...);
  }

  static constexpr auto def = [] {
    std::array<std::size_t, NS> d{};
    for (std::size_t s = 0; s < NS; ++s) d[s] = Alg::slot_level(s);
    return d;
  }();
  static constexpr auto last = [] {
    std::array<std::size_t, NS> l = def;
    note_all(l, std::make_index_sequence<NL>{});
    const std::size_t roots[] = {Roots..., NS};
    for (std::size_t r : roots)
      if (r < NS) l[r] = NL;  // read by the root store after every level
    return l;
  }();
  // pool[s]: left-edge colouring over [def, last] closed intervals, slot order.
  static constexpr auto pool = [] {
    std::array<int, NS> p{};
    std::array<std::size_t, NS + 1> busy_until{};
    int npools = 0;
    for (std::size_t s = 0; s < NS; ++s) {
      int chosen = -1;
      for (int q = 0; q < npools; ++q)
        if (busy_until[q] < def[s]) {
          chosen = q;
          break;
        }
      if (chosen < 0) chosen = npools++;
      p[s] = chosen;
      busy_until[chosen] = last[s];
    }
    return p;
  }();
  static constexpr std::size_t num_pools = [] {
    std::size_t n = 0;
    for (int q : pool)
      if (static_cast<std::size_t>(q) + 1 > n) n = q + 1;
    return n;
  }();
};

// Bytes of one slot's tile, padded to 16.
template <class V, class Levels, std::size_t S>
constexpr std::size_t slot_tile_bytes() {
  using SN = slot_member_node<Levels, S>;
  const std::size_t b = member_out_elems<typename SN::type>(SN::out) * sizeof(V);
  return (b + 15) & ~std::size_t(15);
}

template <class V, class Levels, std::size_t... Roots>
struct Layout {
  using P = Pooling<Levels, Roots...>;
  static constexpr std::size_t NS = P::NS;
  template <std::size_t... S>
  static constexpr std::array<std::size_t, sizeof...(S)> bytes_of(std::index_sequence<S...>) {
    return {slot_tile_bytes<V, Levels, S>()...};
  }
  static constexpr std::array<std::size_t, NS> slot_bytes = bytes_of(std::make_index_sequence<NS>{});
  static constexpr std::size_t num_pools = P::num_pools;
  static constexpr auto pool_bytes = [] {
    std::array<std::size_t, NS + 1> pb{};
    for (std::size_t s = 0; s < NS; ++s)
      if (slot_bytes[s] > pb[P::pool[s]]) pb[P::pool[s]] = slot_bytes[s];
    return pb;
  }();
  static constexpr auto pool_offset = [] {
    std::array<std::size_t, NS + 1> po{};
    std::size_t acc = 0;
    for (std::size_t q = 0; q < num_pools; ++q) {
      po[q] = acc;
      acc += pool_bytes[q];
    }
    po[num_pools] = acc;
    return po;
  }();
  static constexpr std::size_t scratch_bytes = pool_offset[num_pools];
  static constexpr std::size_t unpooled_bytes = [] {
    std::size_t t = 0;
    for (std::size_t b : slot_bytes) t += b;
    return t;
  }();
  static constexpr std::size_t slot_offset(std::size_t s) { return pool_offset[P::pool[s]]; }
};

// ---------------------------------------------------------------------------
// Level predicates (the guards' bodies).
// ---------------------------------------------------------------------------
template <class Lvl, std::size_t... M>
constexpr bool level_homogeneous_impl(std::index_sequence<M...>) {
  if constexpr (sizeof...(M) == 0) {
    return false;
  } else {
    constexpr int k0 = member_traits<tuple_element_t<0, Lvl>>::kind;
    return ((member_traits<tuple_element_t<M, Lvl>>::kind == k0) && ...);
  }
}
template <class Lvl>
constexpr bool level_homogeneous() {
  return level_homogeneous_impl<Lvl>(std::make_index_sequence<tuple_size_v<Lvl>>{});
}

template <class Lvl, std::size_t... M>
constexpr bool level_space_agrees_impl(std::index_sequence<M...>) {
  using T0 = member_traits<tuple_element_t<0, Lvl>>;
  if constexpr (T0::kind == 1 || T0::kind == 3) {
    return ((member_traits<tuple_element_t<M, Lvl>>::sa == T0::sa &&
             member_traits<tuple_element_t<M, Lvl>>::sb == T0::sb) &&
            ...);
  } else {
    return (std::is_same_v<typename member_traits<tuple_element_t<M, Lvl>>::tile,
                           typename T0::tile> &&
            ...);
  }
}
template <class Lvl>
constexpr bool level_space_agrees() {
  if constexpr (!level_homogeneous<Lvl>())
    return true;  // the homogeneity guard reports that defect alone
  else
    return level_space_agrees_impl<Lvl>(std::make_index_sequence<tuple_size_v<Lvl>>{});
}

template <class Levels, std::size_t L, std::size_t... M>
constexpr bool level_reads_earlier_impl(std::index_sequence<M...>) {
  constexpr std::size_t base = Algebra<Levels>::level_base(L);
  bool ok = true;
  ((
       [&] {
         for (std::size_t s : member_traits<tuple_element_t<M, tuple_element_t<L, Levels>>>::reads)
           if (s + 1 > base) ok = false;
       }()),
   ...);
  return ok;
}

template <class Levels, std::size_t... L>
constexpr bool all_homogeneous(std::index_sequence<L...>) {
  return (level_homogeneous<tuple_element_t<L, Levels>>() && ...);
}
template <class Levels, std::size_t... L>
constexpr bool all_spaces(std::index_sequence<L...>) {
  return (level_space_agrees<tuple_element_t<L, Levels>>() && ...);
}
template <class Levels, std::size_t... L>
constexpr bool all_reads_earlier(std::index_sequence<L...>) {
  return (level_reads_earlier_impl<Levels, L>(
              std::make_index_sequence<tuple_size_v<tuple_element_t<L, Levels>>>{}) &&
          ...);
}

// Grid labels of a graph: the map's blocked labels that some stage member carries.
template <class LT, class Levels>
struct GridSpec {
  template <class Node>
  static constexpr bool member_carries(int32_t l) {
    if constexpr (member_traits<Node>::kind == 0) {
      return index_of(to_array<typename Node::modes_seq>(), l) >= 0;
    } else if constexpr (member_traits<Node>::kind == 3) {
      // the free labels of a staged contraction's operands (its contracted
      // labels are looped over, not gridded)
      using C = typename Node::contraction_type;
      return index_of(C::freeA, l) >= 0 || index_of(C::freeB, l) >= 0;
    } else {
      return false;
    }
  }
  template <class Lvl, std::size_t... M>
  static constexpr bool level_carries(int32_t l, std::index_sequence<M...>) {
    return (member_carries<tuple_element_t<M, Lvl>>(l) || ...);
  }
  template <std::size_t... L>
  static constexpr bool carried(int32_t l, std::index_sequence<L...>) {
    return (level_carries<tuple_element_t<L, Levels>>(
                l, std::make_index_sequence<tuple_size_v<tuple_element_t<L, Levels>>>{}) ||
            ...);
  }
  static constexpr int rank = [] {
    int n = 0;
    for (std::size_t i = 0; i < LT::size; ++i)
      if (LT::gridded[i] && carried(LT::labels[i], std::make_index_sequence<tuple_size_v<Levels>>{}))
        ++n;
    return n;
  }();
  static constexpr auto labels = [] {
    std::array<int32_t, rank> out{};
    int n = 0;
    for (std::size_t i = 0; i < LT::size; ++i)
      if (LT::gridded[i] && carried(LT::labels[i], std::make_index_sequence<tuple_size_v<Levels>>{}))
        out[n++] = LT::labels[i];
    return out;
  }();
  static constexpr int grid_slot(int32_t l) { return index_of(labels, l); }
};

}  // namespace b200

// ---------------------------------------------------------------------------
// LevelPlan: the static checks, instantiated by naming the type.
// ---------------------------------------------------------------------------
template <typename LevelsT>
struct LevelPlan {
  using levels_type = LevelsT;
  using Alg = b200::Algebra<LevelsT>;
  static constexpr std::size_t num_levels = tuple_size_v<LevelsT>;
  static constexpr std::size_t num_slots = Alg::num_slots;
  static constexpr std::size_t num_members = Alg::total_members;

  static_assert(b200::all_homogeneous<LevelsT>(std::make_index_sequence<num_levels>{}),
                "level graph: a level must be NON-EMPTY and HOMOGENEOUS -- every member a "
                "contraction, every member a combine, or every member a stage. The decodes "
                "are different objects, so a mixed level computes both and banks neither");
  static_assert(b200::all_spaces<LevelsT>(std::make_index_sequence<num_levels>{}),
                "level graph: every member of a level must share ONE iteration space -- "
                "contraction members must agree on SA and SB (separately, not on their "
                "product), combine and STAGED members on their whole output tile layout. For "
                "a staged level this is what makes fusing its copies into one range sound");
  static_assert(b200::all_reads_earlier<LevelsT>(std::make_index_sequence<num_levels>{}),
                "level graph: a member may not read a slot ITS OWN LEVEL produces -- a level's "
                "members run concurrently, so a sibling's output is a cross-thread hazard, not "
                "an operand");
};

}  // namespace TensorOperations
