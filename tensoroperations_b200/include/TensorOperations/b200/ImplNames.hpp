// ImplNames.hpp -- the reference's internal plan names that its own unit tests
// reach for, spelled over this build's plan code so those tests compile
// unmodified (reference tests/test_level_graph.cpp, test_level_liveness.cpp,
// test_label_tiles.cpp).  Nothing here computes anything new: every name reads
// the slot algebra (b200::Algebra), the level liveness (b200::Pooling), the
// member traits or the label map this build's LevelGraph already uses.
//
//   reference name (LevelGraph.hpp / LevelPlan.hpp / LabelTiles.hpp /
//   DagGraph.hpp)                       here
//   SlotView<V, ES, Tile>               a placeholder view type: value, space, tile
//   make_slot_node_seq<I, Modes>(v, s)  SlotNode over slot I, declared = storage
//   member_out_tile_t<M>                member_traits<M>::tile (storage order)
//   Impl::lg_total_members_v / lg_num_slots_v / lg_level_slots_v /
//     lg_level_base_v / lg_member_base_v / lg_slot_level_v / lg_slot_member_v
//                                       Algebra<Levels>
//   Impl::lg_pool_of_slot / lg_pool_count   Pooling<Levels, Roots...>
//   Impl::lg_member_sa_v / lg_member_sb_v   member_traits<M>::sa / sb
//   Impl::lg_level_homogeneous_v / lg_level_space_agrees_v / lg_levels_reads_v
//                                       the three level guards' predicates
//   Impl::lg_max_operand_slot_v<M>      the largest slot M reads (-1: none)
//   Impl::lg_member_decl_tile<M>        M's tile in its declared label order
//   Impl::lg_resolve_member(_t)         resolve_member (a stage's tile from the map)
//   Impl::canonC_modes_seq_t<R, A, B>   freeA in A's order ++ freeB in B's order
//   Impl::label_tile_v / label_tiles_distinct_v   LabelTiles::tile / distinct
//   Impl::permA_seq_t / permB_seq_t / permC_seq_t / inverse_perm_seq_t /
//     is_identity_seq / operand_stageable_v   the contraction's operand
//                                       permutations (test_graph.cpp)
//   Impl::label_perm_seq_t / same_label_set / produces_own_scratch_v /
//     fusable_operand_v / operand_relabelable_v   the combine's operand rules
//                                       (test_combine_node.cpp)
//   Impl::dag_num_slots / dag_operand_slot / dag_pool_of_slot / dag_pool_count
//                                       slot liveness on a flat node list (below)
#pragma once

#include <array>
#include <cstddef>
#include <type_traits>

#include <TensorOperations/LabelTiles.hpp>
#include <TensorOperations/b200/Plan.hpp>
#include <TensorOperations/b200/TileSpec.hpp>

namespace TensorOperations {

template <typename Value, typename ExecSpace, typename Tile>
struct SlotView {
  using value_type = Value;
  using execution_space = ExecSpace;
  using tile_type = Tile;
};

// A slot node over slot I whose declared labels are its storage order.
template <std::size_t I, typename ModesSeq, typename Value, typename ExecSpace, typename Tile>
auto make_slot_node_seq(SlotView<Value, ExecSpace, Tile>,
                        Kokkos::Array<int, ModesSeq::size()> shape) {
  return SlotNode<Value, ExecSpace, I, ModesSeq, Tile,
                  std::make_integer_sequence<int, static_cast<int>(ModesSeq::size())>>{shape};
}

template <typename Member>
using member_out_tile_t = typename b200::member_traits<Member>::tile;

namespace Impl {

template <typename Levels>
inline constexpr std::size_t lg_total_members_v = b200::Algebra<Levels>::total_members;
template <typename Levels>
inline constexpr std::size_t lg_num_slots_v = b200::Algebra<Levels>::num_slots;
template <typename Levels, std::size_t L>
inline constexpr std::size_t lg_level_base_v = b200::Algebra<Levels>::level_base(L);
template <typename Levels, std::size_t L>
inline constexpr std::size_t lg_level_slots_v =
    b200::Algebra<Levels>::level_base(L + 1) - b200::Algebra<Levels>::level_base(L);
template <typename Levels, std::size_t L, std::size_t M>
inline constexpr std::size_t lg_member_base_v = b200::Algebra<Levels>::member_base(L, M);
template <typename Levels, std::size_t S>
inline constexpr std::size_t lg_slot_level_v = b200::Algebra<Levels>::slot_level(S);
template <typename Levels, std::size_t S>
inline constexpr std::size_t lg_slot_member_v = b200::Algebra<Levels>::slot_member(S);

template <typename Levels, std::size_t... Roots>
constexpr auto lg_pool_of_slot() {
  return b200::Pooling<Levels, Roots...>::pool;
}
template <typename Levels, std::size_t... Roots>
constexpr std::size_t lg_pool_count() {
  return b200::Pooling<Levels, Roots...>::num_pools;
}

template <typename Member>
inline constexpr int lg_member_sa_v = b200::member_traits<Member>::sa;
template <typename Member>
inline constexpr int lg_member_sb_v = b200::member_traits<Member>::sb;

template <typename Level>
inline constexpr bool lg_level_homogeneous_v = b200::level_homogeneous<Level>();
template <typename Level>
inline constexpr bool lg_level_space_agrees_v = b200::level_space_agrees<Level>();
template <typename Levels>
inline constexpr bool lg_levels_reads_v =
    b200::all_reads_earlier<Levels>(std::make_index_sequence<tuple_size_v<Levels>>{});

template <typename Member>
inline constexpr int lg_max_operand_slot_v = [] {
  int m = -1;
  for (std::size_t s : b200::member_traits<Member>::reads)
    if (static_cast<int>(s) > m) m = static_cast<int>(s);
  return m;
}();

template <typename Member>
struct lg_member_decl_tile {
  using MT = b200::member_traits<Member>;
  template <std::size_t... D>
  static auto make(std::index_sequence<D...>)
      -> StaticTile<MT::tile::extents[MT::decl_to_storage[D]]...>;
  using type = decltype(make(std::make_index_sequence<static_cast<std::size_t>(MT::rank)>{}));
};

template <typename LT, typename Raw>
using lg_resolve_member = b200::resolve_member<LT, Raw>;
template <typename LT, typename Raw>
using lg_resolve_member_t = typename b200::resolve_member<LT, Raw>::type;

template <int Rank, typename A, typename B>
using canonC_modes_seq_t =
    typename b200::concat_seq<b200::array_seq_t<b200::minus_labels<A, B>::values()>,
                              b200::array_seq_t<b200::minus_labels<B, A>::values()>>::type;

// Operand permutations of a contraction, gather convention (perm[c] = the
// user axis that becomes canonical axis c): canonical A = freeA ++ contracted
// (both in A's order), canonical B = contracted (A's order) ++ freeB, canonical
// C = freeA ++ freeB.  This build reads operands through these permutations
// instead of permuting them in scratch; the names serve the reference's plan
// checks (reference Permute.hpp).
namespace perm_detail {
template <class Seq, class Labs>
struct positions;
template <class Seq, int32_t... L>
struct positions<Seq, std::integer_sequence<int32_t, L...>> {
  using type = std::integer_sequence<int, b200::index_of(b200::to_array<Seq>(), L)...>;
};
template <class A, class B>
using canon_a_t =
    typename b200::concat_seq<b200::array_seq_t<b200::minus_labels<A, B>::values()>,
                              b200::array_seq_t<b200::common_labels<A, B>::values()>>::type;
template <class A, class B>
using canon_b_t =
    typename b200::concat_seq<b200::array_seq_t<b200::common_labels<A, B>::values()>,
                              b200::array_seq_t<b200::minus_labels<B, A>::values()>>::type;
template <class Perm>
struct inverse_of;
template <int... P>
struct inverse_of<std::integer_sequence<int, P...>> {
  static constexpr std::size_t n = sizeof...(P);
  static constexpr std::array<int, n> inv = [] {
    std::array<int, n> r{};
    const int p[] = {P..., 0};
    for (std::size_t j = 0; j < n; ++j) r[static_cast<std::size_t>(p[j])] = static_cast<int>(j);
    return r;
  }();
  template <std::size_t... I>
  static auto make(std::index_sequence<I...>) -> std::integer_sequence<int, inv[I]...>;
  using type = decltype(make(std::make_index_sequence<n>{}));
};
template <class S>
struct out_tile {
  using type = S;
};
template <class A, class B, class C>
struct out_tile<Tile<A, B, C>> {
  using type = C;
};
template <class O, class... Ops>
struct out_tile<CombineTile<O, Ops...>> {
  using type = O;
};
template <class Op>
constexpr bool hooked() {
  if constexpr (requires { typename Op::hook_type; })
    return !std::is_same_v<typename Op::hook_type, NoHook>;
  else
    return false;
}
}  // namespace perm_detail

// A combine gathers each operand into its output order: perm[o] = the operand
// axis carrying output label o (reference Permute.hpp label_perm).
template <typename OutSeq, typename OpSeq>
using label_perm_seq_t = typename perm_detail::positions<OpSeq, OutSeq>::type;

template <typename A, typename B>
constexpr bool same_label_set() {
  return b200::same_label_set<A, B>();
}

// A contraction or combine hands its output back in scratch it owns; an input
// is the user's tensor.  Both kinds are legal operands.
template <typename Op>
inline constexpr bool produces_own_scratch_v =
    std::is_same_v<typename Op::node_tag, ContractionTag> ||
    std::is_same_v<typename Op::node_tag, CombineTag>;
template <typename Op>
inline constexpr bool fusable_operand_v =
    std::is_same_v<typename Op::node_tag, InputTag> || produces_own_scratch_v<Op>;

template <typename A, typename B>
using permA_seq_t = typename perm_detail::positions<A, perm_detail::canon_a_t<A, B>>::type;
template <typename A, typename B>
using permB_seq_t = typename perm_detail::positions<B, perm_detail::canon_b_t<A, B>>::type;
template <int Rank, typename A, typename B, typename Out>
using permC_seq_t = typename perm_detail::positions<Out, canonC_modes_seq_t<Rank, A, B>>::type;
template <typename Perm>
using inverse_perm_seq_t = typename perm_detail::inverse_of<Perm>::type;

template <int... P>
constexpr bool is_identity_seq(std::integer_sequence<int, P...>) {
  int i = 0;
  return ((P == i++) && ...);
}

// The reference evaluator's staging rule for a permuted operand: a fused
// (node) operand is reordered inside its own output tile, so the permutation
// must map that tile's extents onto themselves; an input is copied into a
// fresh buffer and always qualifies.  (This build reads a fused operand
// through its storage permutation and has no such restriction; the predicate
// is kept for the reference's plan checks.)
template <typename Operand, typename TileSpec, typename Perm>
inline constexpr bool operand_stageable_v = [] {
  if constexpr (std::is_same_v<typename Operand::node_tag, InputTag>) {
    return true;
  } else {
    using T = typename perm_detail::out_tile<TileSpec>::type;
    constexpr auto p = b200::to_array_int<Perm>();
    for (std::size_t i = 0; i < p.size(); ++i)
      if (T::extents[static_cast<std::size_t>(p[i])] != T::extents[i]) return false;
    return true;
  }
}();

// The reference combine evaluator's relabel rule: a permuted operand that
// produces its own scratch and carries no hook is read through a relabel
// instead of being reordered (an input is never relabelled, an unpermuted
// operand is passed through).  This build reads every operand through its
// permutation; the predicate is kept for the reference's plan checks.
template <typename Operand, typename Perm>
inline constexpr bool operand_relabelable_v =
    produces_own_scratch_v<Operand> && !perm_detail::hooked<Operand>() &&
    !is_identity_seq(Perm{});

template <typename LT, int32_t L>
inline constexpr int label_tile_v = LT::tile(L);
template <typename LT>
inline constexpr bool label_tiles_distinct_v = LT::distinct();

// ---- slot liveness on a flat node list (a DagGraph's nodes, in add order) ----
// Node k defines slots [base(k), base(k) + arity); a slot lives from its node
// to the last node that reads it (closed), a root to one past the last node;
// slots take pools by left-edge colouring in slot order.
template <typename Node>
constexpr std::size_t dag_operand_slot() {
  return Node::SlotIdx;
}

namespace dag_detail {
constexpr std::size_t kNone = ~std::size_t(0);
template <typename Op>
constexpr std::size_t slot_of() {
  if constexpr (requires { Op::SlotIdx; })
    return Op::SlotIdx;
  else if constexpr (requires { Op::slot_index; })
    return Op::slot_index;
  else
    return kNone;
}
// The slots node K reads (kNone where an operand is not a slot).
template <typename Node>
constexpr auto reads_of() {
  using Tag = typename Node::node_tag;
  if constexpr (std::is_same_v<Tag, ContractionTag>) {
    return std::array<std::size_t, 2>{slot_of<typename Node::node_a_type>(),
                                      slot_of<typename Node::node_b_type>()};
  } else if constexpr (std::is_same_v<Tag, StagedTag>) {
    return std::array<std::size_t, 1>{slot_of<typename Node::operand_type>()};
  } else if constexpr (std::is_same_v<Tag, CombineTag>) {
    return [&]<std::size_t... K>(std::index_sequence<K...>) {
      return std::array<std::size_t, sizeof...(K)>{
          slot_of<std::decay_t<decltype(std::declval<Node>().operands.template get<K>())>>()...};
    }(std::make_index_sequence<static_cast<std::size_t>(Node::NumOps)>{});
  } else {
    return std::array<std::size_t, 0>{};
  }
}
}  // namespace dag_detail

template <typename Nodes>
constexpr std::size_t dag_num_slots() {
  return [&]<std::size_t... K>(std::index_sequence<K...>) {
    return (std::size_t{0} + ... +
            static_cast<std::size_t>(b200::output_arity<tuple_element_t<K, Nodes>>()));
  }(std::make_index_sequence<tuple_size_v<Nodes>>{});
}

template <typename Nodes, std::size_t... Roots>
constexpr auto dag_pool_of_slot() {
  constexpr std::size_t NN = tuple_size_v<Nodes>;
  constexpr std::size_t NS = dag_num_slots<Nodes>();
  std::array<std::size_t, NS> def{}, last{};
  [&]<std::size_t... K>(std::index_sequence<K...>) {
    std::size_t s = 0;
    ((
         [&] {
           for (int o = 0; o < b200::output_arity<tuple_element_t<K, Nodes>>(); ++o, ++s)
             def[s] = last[s] = K;
         }()),
     ...);
    ((
         [&] {
           for (std::size_t r : dag_detail::reads_of<tuple_element_t<K, Nodes>>())
             if (r < NS && last[r] < K) last[r] = K;
         }()),
     ...);
  }(std::make_index_sequence<NN>{});
  const std::size_t roots[] = {Roots..., NS};
  for (std::size_t r : roots)
    if (r < NS) last[r] = NN;
  std::array<int, NS> pool{};
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
    pool[s] = chosen;
    busy_until[chosen] = last[s];
  }
  return pool;
}
template <typename Nodes, std::size_t... Roots>
constexpr std::size_t dag_pool_count() {
  std::size_t n = 0;
  for (int q : dag_pool_of_slot<Nodes, Roots...>())
    if (static_cast<std::size_t>(q) + 1 > n) n = static_cast<std::size_t>(q) + 1;
  return n;
}

}  // namespace Impl
}  // namespace TensorOperations
