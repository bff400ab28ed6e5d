// Dag.hpp -- DagGraph: a flat, topologically ordered node list whose operands
// NAME earlier results, lowered onto the level plan and the level evaluator.
//
// Public surface as the reference (include/TensorOperations/DagGraph.hpp:
// make_dag :1006-1011, DagGraph::add :846-851 returning the new graph and one
// handle per output, outputs :854-857, slot_bytes / pooled_slot_bytes /
// operand_bytes / arena_bytes / scratch_bytes / index_consistent :866-918,
// DagOutputs::{team_size, slot_bytes, operand_bytes, scratch_bytes, num_pools,
// execute} :781-815).  Semantics kept:
//   * every node is evaluated ONCE per team, however many later nodes name it;
//   * a handle's as<>() renames the slot's axes positionally in STORAGE order
//     (a contraction stores canonical freeA ++ freeB, a combine its output
//     order), so naming a buffer twice with different labels moves no data;
//   * a multi-output combine (fn returning Kokkos::Array<V, M>) yields M
//     handles that share one evaluation;
//   * the LAST node fixes the team decomposition: its output tile is the grid,
//     and every other node's tile is gathered from it by label.  A node mode the
//     grid node carries must be tiled identically; any other mode must fit in
//     one tile (index_consistent(), checked before every launch).
//
// Lowering (this build's own).  add() only records nodes and tiles; execute()
// turns the DAG into a level plan at compile time and launches the same device
// evaluator as the level-graph route (LevelKernel.cuh):
//   1. every input operand of a node becomes a STAGE item (the tile the node's
//      Tile<A,B,C> or CombineTile names, copied on chip) -- except, when a
//      contracted label of a contraction of two inputs spans several tiles at
//      run time, that contraction becomes one self-staging member, which copies
//      its operand tiles once per contracted tile and accumulates;
//   2. items get a depth -- stages 0, a node one more than the deepest item it
//      reads -- and the items of one depth are grouped into levels by kind and
//      iteration space (stages by tile, contractions by SA x SB, combines by
//      output tile), in definition order.  A level never reads its own
//      results, so the level guards hold by construction;
//   3. slots are renumbered level by level (member, output) and every operand
//      is rebound to its new slot; liveness pooling, scratch layout and the
//      launch are the level graph's.
// For the reference's SEM 3D program (24 nodes) this gives six levels: stage
// H and Hw, stage u, 9 gradients, 3 three-output integrands, 9 divergences,
// 3 weighted sums (five, with the gradients self-staging, where a contracted
// label spans several tiles).
//
// Restrictions, each a compile-time diagnostic: nodes are contractions or
// combines; operands are input nodes or handles of this graph; tiles are
// static; a label staged twice has one tile extent.  A contracted label of a
// contraction that reads a handle must fit in one tile (checked at launch).
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <tuple>

#include <TensorOperations/LabelTiles.hpp>
#include <TensorOperations/b200/Graph.hpp>
#include <TensorOperations/b200/TileSpec.hpp>

namespace TensorOperations {
namespace b200 {

template <class... T>
struct TypeList {};
template <class L, class U>
struct tl_append;
template <class... T, class U>
struct tl_append<TypeList<T...>, U> {
  using type = TypeList<T..., U>;
};
template <std::size_t I, class L>
struct tl_at;
template <std::size_t I, class... T>
struct tl_at<I, TypeList<T...>> {
  using type = std::tuple_element_t<I, std::tuple<T...>>;
};

inline constexpr int kDagMaxRank = 8;
inline constexpr int kDagMaxOps = 32;

template <class N>
inline constexpr bool dag_is_contraction_v = std::is_same_v<typename N::node_tag, ContractionTag>;
template <class N>
inline constexpr bool dag_is_combine_v = std::is_same_v<typename N::node_tag, CombineTag>;
template <class N>
inline constexpr bool dag_is_input_v = std::is_same_v<typename N::node_tag, InputTag>;

// Operand P of a node.
template <class Node, std::size_t P, bool = dag_is_contraction_v<Node>>
struct dag_op {
  using type = std::conditional_t<P == 0, typename Node::node_a_type, typename Node::node_b_type>;
  static const type& get(const Node& n) {
    if constexpr (P == 0)
      return n.node_a;
    else
      return n.node_b;
  }
};
template <class Node, std::size_t P>
struct dag_op<Node, P, false> {
  using type = tuple_element_t<P, typename Node::ops_tuple_t>;
  static const type& get(const Node& n) { return n.operands.template get<P>(); }
};

template <class Node>
constexpr std::size_t dag_num_ops() {
  if constexpr (dag_is_contraction_v<Node>)
    return 2;
  else
    return static_cast<std::size_t>(Node::NumOps);
}

template <class Node>
struct dag_storage_labels {
  using type = typename Node::modes_seq;  // combine: its output order
};
template <class Node>
  requires dag_is_contraction_v<Node>
struct dag_storage_labels<Node> {
  using type = typename Node::canon_seq;
};
template <class Node>
using dag_storage_labels_t = typename dag_storage_labels<Node>::type;

// Tile of operand P (in that operand's label order) named by the node's spec.
template <class Node, class TS, std::size_t P>
constexpr auto dag_operand_tile() {
  using Op = typename dag_op<Node, P>::type;
  constexpr int R = Op::Rank;
  std::array<int, R> t{};
  if constexpr (dag_is_contraction_v<Node>) {
    static_assert(is_contraction_tile<TS>::value,
                  "DagGraph::add: a contraction node's tile must be Tile<TileA, TileB, TileC>");
    using T = std::conditional_t<P == 0, typename TS::a_type, typename TS::b_type>;
    static_assert(T::rank == R, "DagGraph::add: an operand tile's rank differs from its operand's");
    for (int d = 0; d < R; ++d) t[d] = T::extents[d];
  } else {
    using O = typename combine_out_tile<TS>::type;
    static_assert(O::rank == Node::Rank,
                  "DagGraph::add: a combine node's output tile rank differs from its rank");
    constexpr auto out = to_array<typename Node::modes_seq>();
    constexpr auto lab = to_array<typename Op::modes_seq>();
    for (int d = 0; d < R; ++d) t[d] = O::extents[index_of(out, lab[d])];
  }
  return t;
}

// The node's output tile in STORAGE order.
template <class Node, class TS>
constexpr auto dag_storage_tile() {
  std::array<int, Node::Rank> t{};
  if constexpr (dag_is_contraction_v<Node>) {
    static_assert(is_contraction_tile<TS>::value,
                  "DagGraph::add: a contraction node's tile must be Tile<TileA, TileB, TileC>");
    using C = typename TS::c_type;
    static_assert(C::rank == Node::Rank,
                  "DagGraph::add: Tile<A, B, C>'s output tile rank differs from the node's rank");
    constexpr auto canon = to_array<typename Node::canon_seq>();
    constexpr auto decl = to_array<typename Node::decl_seq>();
    for (int i = 0; i < Node::Rank; ++i) t[i] = C::extents[index_of(decl, canon[i])];
  } else {
    using O = typename combine_out_tile<TS>::type;
    static_assert(O::rank == Node::Rank,
                  "DagGraph::add: a combine node's output tile rank differs from its rank");
    for (int i = 0; i < Node::Rank; ++i) t[i] = O::extents[i];
  }
  return t;
}

// The output tile the operands imply (the level planner's derivation), in
// storage order; it must equal the tile the spec names.
template <class Node, class TS>
constexpr auto dag_implied_tile() {
  std::array<int, Node::Rank> t{};
  if constexpr (dag_is_contraction_v<Node>) {
    constexpr auto ta = dag_operand_tile<Node, TS, 0>();
    constexpr auto tb = dag_operand_tile<Node, TS, 1>();
    constexpr auto la = to_array<typename Node::AL>();
    constexpr auto lb = to_array<typename Node::BL>();
    for (int d = 0; d < Node::FreeA; ++d) t[d] = ta[index_of(la, Node::freeA[d])];
    for (int d = 0; d < Node::FreeB; ++d) t[Node::FreeA + d] = tb[index_of(lb, Node::freeB[d])];
  } else {
    constexpr auto t0 = dag_operand_tile<Node, TS, 0>();
    constexpr auto out = to_array<typename Node::modes_seq>();
    constexpr auto l0 = to_array<typename dag_op<Node, 0>::type::modes_seq>();
    for (int d = 0; d < Node::Rank; ++d) t[d] = t0[index_of(l0, out[d])];
  }
  return t;
}

// Checks made when a node is added: operands are inputs or slots, a slot
// operand's tile is the one its producer was given, contracted labels agree.
template <class Node, class TS>
constexpr bool dag_operand_tiles_agree() {
  bool ok = true;
  [&]<std::size_t... P>(std::index_sequence<P...>) {
    (
        [&] {
          using Op = typename dag_op<Node, P>::type;
          if constexpr (is_slot_v<Op>) {
            constexpr auto named = dag_operand_tile<Node, TS, P>();
            constexpr auto held = operand_tile_by_axis<Op>();
            for (int d = 0; d < Op::Rank; ++d)
              if (named[d] != held[d]) ok = false;
          }
        }(),
        ...);
  }(std::make_index_sequence<dag_num_ops<Node>()>{});
  return ok;
}
template <class Node, class TS>
constexpr bool dag_contracted_tiles_agree() {
  if constexpr (dag_is_contraction_v<Node>) {
    constexpr auto ta = dag_operand_tile<Node, TS, 0>();
    constexpr auto tb = dag_operand_tile<Node, TS, 1>();
    constexpr auto la = to_array<typename Node::AL>();
    constexpr auto lb = to_array<typename Node::BL>();
    for (int d = 0; d < Node::NumContracted; ++d)
      if (ta[index_of(la, Node::contracted[d])] != tb[index_of(lb, Node::contracted[d])])
        return false;
  }
  return true;
}
template <class Node>
constexpr bool dag_operands_supported() {
  bool ok = true;
  [&]<std::size_t... P>(std::index_sequence<P...>) {
    ((ok = ok && (dag_is_input_v<typename dag_op<Node, P>::type> ||
                  is_slot_v<typename dag_op<Node, P>::type>)),
     ...);
  }(std::make_index_sequence<dag_num_ops<Node>()>{});
  return ok;
}

// A DAG handle: one output of one node, named by its flat DAG slot.
template <std::size_t Slot, class V, class ES, class StorageLabels, class StorageTile>
struct DagSlotHandle {
  static constexpr std::size_t slot_index = Slot;
  static constexpr int Rank = static_cast<int>(StorageLabels::size());
  using value_type = V;
  using storage_labels = StorageLabels;
  using storage_tile = StorageTile;
  Kokkos::Array<int, Rank> shape_;  // storage order

  Kokkos::Array<int, Rank> shape() const { return shape_; }

  template <int32_t... Modes>
  auto as() const {
    static_assert(static_cast<int>(sizeof...(Modes)) == Rank,
                  "DagGraph handle as(): one label per axis of the slot");
    static_assert(all_distinct(std::array<int32_t, sizeof...(Modes)>{Modes...}),
                  "DagGraph handle as(): labels must be distinct");
    return SlotNode<V, ES, Slot, Labels<Modes...>, StorageTile,
                    std::make_integer_sequence<int, Rank>>{shape_};
  }
};

template <class Arr, std::size_t... I>
constexpr bool arrays_equal(const Arr& a, const Arr& b, std::index_sequence<I...>) {
  return ((a[I] == b[I]) && ...);
}

// ---------------------------------------------------------------------------
// The lowering of one graph type.
// ---------------------------------------------------------------------------
// SelfStage: contractions of two inputs become self-staging members (kind 3)
// that loop over the tiles of their contracted labels; otherwise their
// operands are stage items like any other input.  A launch takes the second
// form whenever every contracted label fits its tile (the common case, and
// the cheaper kernel) and the first only when one does not.
template <class V, class ES, class NodesT, class TilesL, bool SelfStage = false>
struct DagLowering {
  static constexpr std::size_t NK = tuple_size_v<NodesT>;
  static_assert(NK > 0, "DagGraph::execute: the graph has no nodes");
  template <std::size_t K>
  using node_t = tuple_element_t<K, NodesT>;
  template <std::size_t K>
  using spec_t = typename tl_at<K, TilesL>::type;

  // ---- per-node facts --------------------------------------------------------
  struct NodeRow {
    int kind = 0;  // 1 contraction, 2 combine, 3 contraction of two inputs (staged by itself)
    int arity = 1;
    int nops = 0;
    int rank = 0;
    bool input[kDagMaxOps] = {};
    std::size_t slot[kDagMaxOps] = {};
    int sa = 0, sb = 0;
    int32_t lab[kDagMaxRank] = {};  // storage labels
    int tile[kDagMaxRank] = {};     // storage tile
  };
  template <std::size_t K>
  static constexpr NodeRow node_row() {
    using N = node_t<K>;
    static_assert(dag_num_ops<N>() <= static_cast<std::size_t>(kDagMaxOps),
                  "DagGraph: too many operands in one node for this build");
    static_assert(N::Rank <= kDagMaxRank, "DagGraph: node rank above this build's maximum (8)");
    NodeRow r{};
    r.kind = dag_is_combine_v<N> ? 2 : 1;
    if constexpr (SelfStage && dag_is_contraction_v<N>) {
      if constexpr (dag_is_input_v<typename N::node_a_type> && dag_is_input_v<typename N::node_b_type>)
        r.kind = 3;
    }
    r.arity = output_arity<N>();
    r.nops = static_cast<int>(dag_num_ops<N>());
    r.rank = N::Rank;
    [&]<std::size_t... P>(std::index_sequence<P...>) {
      (
          [&] {
            using Op = typename dag_op<N, P>::type;
            r.input[P] = dag_is_input_v<Op>;
            if constexpr (is_slot_v<Op>) r.slot[P] = Op::SlotIdx;
          }(),
          ...);
    }(std::make_index_sequence<dag_num_ops<N>()>{});
    constexpr auto st = dag_storage_tile<N, spec_t<K>>();
    constexpr auto sl = to_array<dag_storage_labels_t<N>>();
    for (int d = 0; d < N::Rank; ++d) {
      r.lab[d] = sl[d];
      r.tile[d] = st[d];
    }
    if constexpr (dag_is_contraction_v<N>) {
      constexpr auto t = dag_implied_tile<N, spec_t<K>>();
      r.sa = 1;
      r.sb = 1;
      for (int d = 0; d < N::FreeA; ++d) r.sa *= t[d];
      for (int d = 0; d < N::FreeB; ++d) r.sb *= t[N::FreeA + d];
    }
    return r;
  }
  template <std::size_t... K>
  static constexpr std::array<NodeRow, NK> node_rows(std::index_sequence<K...>) {
    return {node_row<K>()...};
  }
  static constexpr std::array<NodeRow, NK> rows = node_rows(std::make_index_sequence<NK>{});

  static constexpr std::array<std::size_t, NK + 1> dag_base = [] {
    std::array<std::size_t, NK + 1> b{};
    for (std::size_t k = 0; k < NK; ++k) b[k + 1] = b[k] + static_cast<std::size_t>(rows[k].arity);
    return b;
  }();
  static constexpr std::size_t num_dag_slots = dag_base[NK];

  static constexpr std::size_t owner(std::size_t s) {
    for (std::size_t k = 0; k < NK; ++k)
      if (s >= dag_base[k] && s < dag_base[k + 1]) return k;
    return NK;
  }

  // every slot operand names an earlier node of THIS graph
  static constexpr bool reads_earlier = [] {
    for (std::size_t k = 0; k < NK; ++k)
      for (int p = 0; p < rows[k].nops; ++p)
        if (!rows[k].input[p] && !(rows[k].slot[p] < dag_base[k])) return false;
    return true;
  }();
  static_assert(reads_earlier,
                "DagGraph: an operand names a slot that no earlier node of this graph produced "
                "(a handle from another graph, or a node reading itself)");

  // ---- stage items -------------------------------------------------------------
  struct StageRef {
    std::size_t node = 0, pos = 0;
  };
  // (a contraction of two inputs stages its operands itself: no stage items)
  static constexpr std::size_t NS = [] {
    std::size_t n = 0;
    for (std::size_t k = 0; k < NK; ++k)
      for (int p = 0; p < rows[k].nops; ++p)
        if (rows[k].input[p] && rows[k].kind != 3) ++n;
    return n;
  }();
  static constexpr std::array<StageRef, NS> stages = [] {
    std::array<StageRef, NS> s{};
    std::size_t n = 0;
    for (std::size_t k = 0; k < NK; ++k)
      for (int p = 0; p < rows[k].nops; ++p)
        if (rows[k].input[p] && rows[k].kind != 3) s[n++] = StageRef{k, static_cast<std::size_t>(p)};
    return s;
  }();
  static constexpr std::size_t stage_of(std::size_t k, std::size_t p) {
    for (std::size_t s = 0; s < NS; ++s)
      if (stages[s].node == k && stages[s].pos == p) return s;
    return NS;
  }

  struct StageRow {
    int rank = 0;
    int32_t lab[kDagMaxRank] = {};
    int tile[kDagMaxRank] = {};
  };
  template <std::size_t S>
  static constexpr StageRow stage_row() {
    constexpr StageRef ref = stages[S];
    using N = node_t<ref.node>;
    using Op = typename dag_op<N, ref.pos>::type;
    static_assert(Op::Rank <= kDagMaxRank, "DagGraph: input rank above this build's maximum (8)");
    constexpr auto t = dag_operand_tile<N, spec_t<ref.node>, ref.pos>();
    constexpr auto l = to_array<typename Op::modes_seq>();
    StageRow r{};
    r.rank = Op::Rank;
    for (int d = 0; d < Op::Rank; ++d) {
      r.lab[d] = l[d];
      r.tile[d] = t[d];
    }
    return r;
  }
  template <std::size_t... S>
  static constexpr std::array<StageRow, NS> stage_rows(std::index_sequence<S...>) {
    return {stage_row<S>()...};
  }
  static constexpr std::array<StageRow, NS> srows = stage_rows(std::make_index_sequence<NS>{});

  // ---- items, depths, levels -------------------------------------------------
  static constexpr std::size_t NI = NS + NK;
  using Sig = std::array<int, 2 + kDagMaxRank>;

  static constexpr std::array<int, NK> depth = [] {
    std::array<int, NK> d{};
    for (std::size_t k = 0; k < NK; ++k) {
      int m = 0;
      for (int p = 0; p < rows[k].nops; ++p)
        if (!rows[k].input[p]) {
          const std::size_t o = owner(rows[k].slot[p]);
          if (o < k && d[o] > m) m = d[o];
        }
      d[k] = m + 1;
    }
    return d;
  }();
  static constexpr int item_depth(std::size_t i) { return i < NS ? 0 : depth[i - NS]; }
  // slots of the lowered member: a self-staging contraction also holds its
  // two operand tiles
  static constexpr int item_arity(std::size_t i) {
    return i < NS ? 1 : (rows[i - NS].kind == 3 ? 3 : rows[i - NS].arity);
  }
  static constexpr Sig item_sig(std::size_t i) {
    Sig s{};
    if (i < NS) {
      s[0] = 0;
      s[1] = srows[i].rank;
      for (int d = 0; d < srows[i].rank; ++d) s[2 + d] = srows[i].tile[d];
    } else {
      const NodeRow& r = rows[i - NS];
      s[0] = r.kind;
      if (r.kind == 1 || r.kind == 3) {
        s[1] = r.sa;
        s[2] = r.sb;
      } else {
        s[1] = r.rank;
        for (int d = 0; d < r.rank; ++d) s[2 + d] = r.tile[d];
      }
    }
    return s;
  }

  struct Plan {
    std::size_t nl = 0;
    std::array<std::size_t, NI> level{}, member{}, level_size{}, level_first{}, order{}, slot_base{};
  };
  static constexpr Plan plan = [] {
    Plan p{};
    std::array<Sig, NI> lsig{};
    int maxd = 0;
    for (std::size_t i = 0; i < NI; ++i)
      if (item_depth(i) > maxd) maxd = item_depth(i);
    for (int d = 0; d <= maxd; ++d) {
      const std::size_t first = p.nl;
      for (std::size_t i = 0; i < NI; ++i) {
        if (item_depth(i) != d) continue;
        const Sig s = item_sig(i);
        std::size_t L = p.nl;
        for (std::size_t l = first; l < p.nl; ++l)
          if (lsig[l] == s) {
            L = l;
            break;
          }
        if (L == p.nl) lsig[p.nl++] = s;
        p.level[i] = L;
        p.member[i] = p.level_size[L]++;
      }
    }
    std::size_t n = 0;
    for (std::size_t L = 0; L < p.nl; ++L) {
      p.level_first[L] = n;
      for (std::size_t m = 0; m < p.level_size[L]; ++m)
        for (std::size_t i = 0; i < NI; ++i)
          if (p.level[i] == L && p.member[i] == m) p.order[n++] = i;
    }
    std::size_t s = 0;
    for (std::size_t q = 0; q < NI; ++q) {
      p.slot_base[p.order[q]] = s;
      s += static_cast<std::size_t>(item_arity(p.order[q]));
    }
    return p;
  }();
  static constexpr std::size_t num_levels = plan.nl;

  // Slot of the lowered plan that holds DAG slot s.
  static constexpr std::size_t level_slot(std::size_t s) {
    const std::size_t k = owner(s);
    return plan.slot_base[NS + k] + (s - dag_base[k]);
  }

  // ---- lowered member types ------------------------------------------------------
  template <std::size_t K, std::size_t P, class Op = typename dag_op<node_t<K>, P>::type,
            bool = dag_is_input_v<Op>>
  struct lowered_op {
    static constexpr auto t = dag_operand_tile<node_t<K>, spec_t<K>, P>();
    using type = SlotNode<V, ES, plan.slot_base[stage_of(K, P)], typename Op::modes_seq,
                          array_tile_t<t>, std::make_integer_sequence<int, Op::Rank>>;
  };
  template <std::size_t K, std::size_t P, class Op>
  struct lowered_op<K, P, Op, false> {
    using type = SlotNode<V, ES, level_slot(Op::SlotIdx), typename Op::modes_seq,
                          typename Op::storage_tile, typename Op::decl_to_storage_seq>;
  };
  template <std::size_t K, std::size_t P>
  using lowered_op_t = typename lowered_op<K, P>::type;

  template <std::size_t K, std::size_t P>
  static lowered_op_t<K, P> lower_op(const typename dag_op<node_t<K>, P>::type& op) {
    return lowered_op_t<K, P>{op.shape()};
  }

  template <std::size_t K, class N = node_t<K>, bool = dag_is_contraction_v<N>>
  struct lowered_node {
    using type = NodeHandle<ContractionTag, lowered_op_t<K, 0>, lowered_op_t<K, 1>,
                            typename N::decl_seq, typename N::value_type, typename N::exec_space,
                            typename N::hook_type>;
    static type make(const N& n) {
      return type{lower_op<K, 0>(n.node_a), lower_op<K, 1>(n.node_b), n.shape_, n.hook_op};
    }
  };
  template <std::size_t K, class N>
  struct lowered_node<K, N, false> {
    template <std::size_t... P>
    static auto type_of(std::index_sequence<P...>)
        -> NodeHandle<CombineTag, typename N::combine_type, typename N::modes_seq,
                      typename N::value_type, typename N::exec_space,
                      std::integral_constant<int, N::NumOut>, lowered_op_t<K, P>...>;
    using type = decltype(type_of(std::make_index_sequence<dag_num_ops<N>()>{}));
    static type make(const N& n) {
      return [&]<std::size_t... P>(std::index_sequence<P...>) {
        return type{n.fn,
                    typename type::ops_tuple_t(lower_op<K, P>(n.operands.template get<P>())...),
                    n.shape_};
      }(std::make_index_sequence<dag_num_ops<N>()>{});
    }
  };

  template <std::size_t I, bool = (I < NS)>
  struct member {
    static constexpr StageRef ref = stages[I];
    using N = node_t<ref.node>;
    using Op = typename dag_op<N, ref.pos>::type;
    static constexpr auto t = dag_operand_tile<N, spec_t<ref.node>, ref.pos>();
    using type = NodeHandle<StagedTag, Op, typename Op::modes_seq, array_tile_t<t>>;
    static type make(const NodesT& nodes) {
      return type{dag_op<N, ref.pos>::get(nodes.template get<ref.node>())};
    }
  };
  // A contraction of two inputs: one member that stages both operand tiles
  // into its own slots base+1 and base+2, once per contracted tile.
  template <std::size_t K, class N = node_t<K>>
  struct staged_node {
    static constexpr std::size_t base = plan.slot_base[NS + K];
    using InA = typename N::node_a_type;
    using InB = typename N::node_b_type;
    static constexpr auto ta = dag_operand_tile<N, spec_t<K>, 0>();
    static constexpr auto tb = dag_operand_tile<N, spec_t<K>, 1>();
    using SA = SlotNode<V, ES, base + 1, typename InA::modes_seq, array_tile_t<ta>,
                        std::make_integer_sequence<int, InA::Rank>>;
    using SB = SlotNode<V, ES, base + 2, typename InB::modes_seq, array_tile_t<tb>,
                        std::make_integer_sequence<int, InB::Rank>>;
    using Cs = NodeHandle<ContractionTag, SA, SB, typename N::decl_seq, typename N::value_type,
                          typename N::exec_space, typename N::hook_type>;
    using type = NodeHandle<StagedContractionTag, InA, InB, Cs>;
    static type make(const N& n) {
      return type{n.node_a, n.node_b, Cs{SA{n.node_a.shape()}, SB{n.node_b.shape()}, n.shape_, n.hook_op}};
    }
  };

  template <std::size_t I, bool = (rows[I - NS].kind == 3)>
  struct node_member {
    using type = typename lowered_node<I - NS>::type;
    static type make(const NodesT& nodes) {
      return lowered_node<I - NS>::make(nodes.template get<I - NS>());
    }
  };
  template <std::size_t I>
  struct node_member<I, true> {
    using type = typename staged_node<I - NS>::type;
    static type make(const NodesT& nodes) {
      return staged_node<I - NS>::make(nodes.template get<I - NS>());
    }
  };
  template <std::size_t I>
  struct member<I, false> : node_member<I> {};

  template <std::size_t L, std::size_t... M>
  static auto level_type_of(std::index_sequence<M...>)
      -> DeviceTuple<typename member<plan.order[plan.level_first[L] + M]>::type...>;
  template <std::size_t L>
  using level_t = decltype(level_type_of<L>(std::make_index_sequence<plan.level_size[L]>{}));
  template <std::size_t... L>
  static auto levels_type_of(std::index_sequence<L...>) -> DeviceTuple<level_t<L>...>;
  using levels_t = decltype(levels_type_of(std::make_index_sequence<num_levels>{}));

  template <std::size_t L>
  static level_t<L> make_level(const NodesT& nodes) {
    return [&]<std::size_t... M>(std::index_sequence<M...>) {
      return level_t<L>(member<plan.order[plan.level_first[L] + M]>::make(nodes)...);
    }(std::make_index_sequence<plan.level_size[L]>{});
  }
  static levels_t make_levels(const NodesT& nodes) {
    return [&]<std::size_t... L>(std::index_sequence<L...>) {
      return levels_t(make_level<L>(nodes)...);
    }(std::make_index_sequence<num_levels>{});
  }

  // ---- the label map ----------------------------------------------------------------
  // The grid node's labels are blocked with its tile; every other staged
  // label is whole, with the one tile every stage gives it.
  using GridNode = node_t<NK - 1>;
  static constexpr auto root_labels = to_array<dag_storage_labels_t<GridNode>>();
  static constexpr int root_rank = GridNode::Rank;
  static constexpr auto root_tile = dag_storage_tile<GridNode, spec_t<NK - 1>>();

  // Labels every staged tile carries: the stage items', and the FREE labels of
  // the self-staging contractions' operands (their contracted labels are
  // looped over, so they are in neither the grid nor the whole-label checks).
  struct StagedLabels {
    std::size_t n = 0;
    std::array<int32_t, kDagMaxRank * 2 * (NS + NK) + 1> lab{};
    std::array<int, kDagMaxRank * 2 * (NS + NK) + 1> tile{};
  };
  template <std::size_t K>
  static constexpr void note_staged_node(StagedLabels& m) {
    using N = node_t<K>;
    if constexpr (SelfStage && dag_is_contraction_v<N>) {
      if constexpr (dag_is_input_v<typename N::node_a_type> && dag_is_input_v<typename N::node_b_type>) {
        constexpr auto ta = dag_operand_tile<N, spec_t<K>, 0>();
        constexpr auto tb = dag_operand_tile<N, spec_t<K>, 1>();
        constexpr auto la = to_array<typename N::AL>();
        constexpr auto lb = to_array<typename N::BL>();
        for (std::size_t d = 0; d < la.size(); ++d)
          if (index_of(N::contracted, la[d]) < 0) {
            m.lab[m.n] = la[d];
            m.tile[m.n++] = ta[d];
          }
        for (std::size_t d = 0; d < lb.size(); ++d)
          if (index_of(N::contracted, lb[d]) < 0) {
            m.lab[m.n] = lb[d];
            m.tile[m.n++] = tb[d];
          }
      }
    }
  }
  static constexpr StagedLabels staged_labels = [] {
    StagedLabels m{};
    for (std::size_t s = 0; s < NS; ++s)
      for (int d = 0; d < srows[s].rank; ++d) {
        m.lab[m.n] = srows[s].lab[d];
        m.tile[m.n++] = srows[s].tile[d];
      }
    [&]<std::size_t... K>(std::index_sequence<K...>) {
      (note_staged_node<K>(m), ...);
    }(std::make_index_sequence<NK>{});
    return m;
  }();

  struct LabelMap {
    std::size_t n = 0;
    std::array<int32_t, kDagMaxRank * 2 * (NS + NK + 1)> lab{};
    std::array<int, kDagMaxRank * 2 * (NS + NK + 1)> ext{};
    std::array<bool, kDagMaxRank * 2 * (NS + NK + 1)> grid{};
    bool consistent = true;
  };
  static constexpr LabelMap label_map = [] {
    LabelMap m{};
    for (int d = 0; d < root_rank; ++d) {
      m.lab[m.n] = root_labels[d];
      m.ext[m.n] = root_tile[d];
      m.grid[m.n] = true;
      ++m.n;
    }
    for (std::size_t q = 0; q < staged_labels.n; ++q) {
      const int32_t l = staged_labels.lab[q];
      std::size_t i = 0;
      while (i < m.n && m.lab[i] != l) ++i;
      if (i < m.n) {
        if (m.ext[i] != staged_labels.tile[q]) m.consistent = false;
      } else {
        m.lab[m.n] = l;
        m.ext[m.n] = staged_labels.tile[q];
        m.grid[m.n] = false;
        ++m.n;
      }
    }
    return m;
  }();
  static_assert(label_map.consistent,
                "DagGraph: a label is staged with two different tile extents, or a staged "
                "label the last (grid) node carries is tiled differently from it -- every "
                "shared mode must be tiled identically in node and grid node");

  // Every node mode the grid node carries has the grid node's tile extent
  // (the static half of index_consistent()).
  static constexpr bool nodes_tiled_like_root = [] {
    for (std::size_t k = 0; k < NK; ++k)
      for (int d = 0; d < rows[k].rank; ++d)
        for (int g = 0; g < root_rank; ++g)
          if (rows[k].lab[d] == root_labels[g] && rows[k].tile[d] != root_tile[g]) return false;
    return true;
  }();

  template <std::size_t... I>
  static auto label_tiles_of(std::index_sequence<I...>)
      -> LabelTiles<std::conditional_t<label_map.grid[I], LabelTile<label_map.lab[I], label_map.ext[I]>,
                                       LabelWhole<label_map.lab[I], label_map.ext[I]>>...>;
  using label_tiles_t = decltype(label_tiles_of(std::make_index_sequence<label_map.n>{}));

  using graph_t = LevelGraph<V, ES, label_tiles_t, levels_t>;

  // grid-node labels that no stage carries (the level grid cannot see them)
  static constexpr std::array<bool, root_rank> root_label_staged = [] {
    std::array<bool, root_rank> f{};
    for (int d = 0; d < root_rank; ++d)
      for (std::size_t q = 0; q < staged_labels.n; ++q)
        if (staged_labels.lab[q] == root_labels[d]) f[d] = true;
    return f;
  }();
};

}  // namespace b200
}  // namespace TensorOperations
