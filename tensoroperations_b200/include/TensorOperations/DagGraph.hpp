// DagGraph.hpp -- make_dag / DagGraph / DagOutputs (B200 frontend).
//
// Public surface as the reference (include/TensorOperations/DagGraph.hpp:
// DagOutputs :781-815, DagGraph :823-1005, make_dag :1006-1011):
//
//   auto [g0, grad]      = make_dag<float>().add(contraction, Tile<TA, TB, TC>{});
//   auto [g1, f0, f1]    = g0.add(two_output_combine(grad.as<...>()), CombineTile<...>{});
//   g1.outputs(f0, f1).team_size(128).execute(TeamPolicyTag<>{}, view0, view1);
//
// add() returns the new graph followed by one handle per output, so definition
// order is the topological order.  execute() lowers the graph onto the level
// plan (b200/Dag.hpp) and launches one kernel; it returns the league size.
// Where the reference asserts (index_consistent) or traps, this build throws
// TensorOperations::LevelGraphError with a one-line reason.
//
// Scratch accounting.  The numbers are the reference's account of the DAG
// (reference DagGraph.hpp: DagGraph::slot_bytes / operand_bytes /
// pooled_slot_bytes / arena_bytes, DagOutputs::slot_bytes / operand_bytes /
// num_pools): DagGraph::slot_bytes() / operand_bytes() are the un-pooled bounds
// (one tile per node output / per staged operand); DagOutputs::slot_bytes() and
// num_pools pool the node outputs by live range on the node timeline (a root
// lives past the last node), and DagOutputs::operand_bytes() is the largest
// single node's operand staging.  What a launch here requests is the lowered
// level plan's store, where staged inputs are slots pooled with everything
// else: DagOutputs::launch_scratch_bytes().
#pragma once

#include <TensorOperations/LabelTiles.hpp>
#include <TensorOperations/LevelGraph.hpp>
#include <TensorOperations/Tiling.hpp>
#include <TensorOperations/b200/Dag.hpp>
#if defined(__CUDACC__)
#include <TensorOperations/b200/SemFusedDag.hpp>
#endif
#include <TensorOperations/b200/TcContract.hpp>

namespace TensorOperations {

template <typename Dag, std::size_t... Roots>
struct DagOutputs;

template <typename ValueType, typename ExecSpace, typename NodesT, typename TilesL>
struct DagGraph {
  static constexpr std::size_t N = tuple_size_v<NodesT>;
  using value_type = ValueType;
  using exec_space = ExecSpace;
  using nodes_type = NodesT;
  using tiles_type = TilesL;

  NodesT nodes;

  template <typename Node, typename TileSpec>
  auto add(const Node& node, const TileSpec&) const {
    static_assert(b200::dag_is_contraction_v<Node> || b200::dag_is_combine_v<Node>,
                  "DagGraph::add: a node is a contraction or a combine (an input is an operand "
                  "of the nodes that read it)");
    static_assert(b200::dag_operands_supported<Node>(),
                  "DagGraph::add: every operand must be an input node or a handle returned by "
                  "DagGraph::add (as<>() of it)");
    static_assert(b200::dag_operand_tiles_agree<Node, TileSpec>(),
                  "DagGraph::add: a handle operand's tile in this node's tile spec differs "
                  "from the tile its producer was given");
    static_assert(b200::dag_contracted_tiles_agree<Node, TileSpec>(),
                  "DagGraph::add: a contracted label has different tile extents in A and B");
    constexpr auto named = b200::dag_storage_tile<Node, TileSpec>();
    constexpr auto implied = b200::dag_implied_tile<Node, TileSpec>();
    static_assert(b200::arrays_equal(named, implied, std::make_index_sequence<Node::Rank>{}),
                  "DagGraph::add: the node's output tile differs from the tile its operands' "
                  "tiles give it");
    constexpr std::size_t M = static_cast<std::size_t>(b200::output_arity<Node>());
    return add_impl<Node, TileSpec>(node, std::make_index_sequence<M>{});
  }

  // Designate graph outputs; the order matches the views given to execute().
  template <typename... Handles>
  auto outputs(const Handles&...) const {
    return DagOutputs<DagGraph, Handles::slot_index...>{*this};
  }

  // Un-pooled bounds, as the reference reports them: one storage tile per
  // node output, and one tile per staged input operand.
  std::size_t slot_bytes() const { return unpooled_slot_bytes(); }
  std::size_t operand_bytes() const { return unpooled_operand_bytes(); }
  std::size_t scratch_bytes() const { return slot_bytes() + operand_bytes(); }

  static constexpr std::size_t unpooled_slot_bytes() {
    return slot_bytes_impl(std::make_index_sequence<N>{});
  }
  static constexpr std::size_t unpooled_operand_bytes() {
    using Low = lowering;
    std::size_t b = 0;
    for (std::size_t s = 0; s < Low::NS; ++s) {
      std::size_t e = 1;
      for (int d = 0; d < Low::srows[s].rank; ++d) e *= static_cast<std::size_t>(Low::srows[s].tile[d]);
      b += round16(e * sizeof(ValueType));
    }
    return b;
  }
  // The largest single node's operand staging (no two nodes' staged operands
  // are live together).
  std::size_t arena_bytes() const { return max_node_operand_bytes(); }
  std::size_t arena_elems() const { return (arena_bytes() + sizeof(ValueType) - 1) / sizeof(ValueType); }

  static constexpr std::size_t max_node_operand_bytes() {
    using Low = lowering;
    std::array<std::size_t, N + 1> per{};
    for (std::size_t s = 0; s < Low::NS; ++s) {
      std::size_t e = 1;
      for (int d = 0; d < Low::srows[s].rank; ++d) e *= static_cast<std::size_t>(Low::srows[s].tile[d]);
      per[Low::stages[s].node] += round16(e * sizeof(ValueType));
    }
    std::size_t m = 0;
    for (std::size_t b : per)
      if (b > m) m = b;
    return m;
  }

  // The node-output slots pooled by live range for these roots: the sum of the
  // pools' largest slots.
  template <std::size_t... Roots>
  std::size_t pooled_slot_bytes() const {
    return node_pooled_slot_bytes<Roots...>();
  }
  template <std::size_t... Roots>
  static constexpr std::size_t node_pooled_slot_bytes() {
    constexpr std::size_t NSL = num_slots();
    constexpr auto pool = Impl::dag_pool_of_slot<NodesT, Roots...>();
    constexpr auto sz = slot_sizes(std::make_index_sequence<N>{});
    std::array<std::size_t, NSL + 1> pmax{};
    for (std::size_t s = 0; s < NSL; ++s) {
      const auto q = static_cast<std::size_t>(pool[s]);
      if (sz[s] > pmax[q]) pmax[q] = sz[s];
    }
    std::size_t b = 0;
    for (std::size_t x : pmax) b += x;
    return b;
  }

  // The store the launch requests: the lowered level plan's, pooled by
  // liveness for these roots (staged inputs included).
  template <std::size_t... Roots>
  std::size_t launch_scratch_bytes() const {
    using Low = lowering;
    return b200::Layout<ValueType, typename Low::levels_t, Low::level_slot(Roots)...>::scratch_bytes;
  }

  // The reference's precondition for gathering every node's tile index from
  // the grid node's by label: a mode the grid (last) node carries is tiled
  // identically and has the same extent there; any other mode has one tile.
  bool index_consistent() const {
    using Low = lowering;
    if constexpr (!Low::nodes_tiled_like_root) return false;
    const auto gshape = nodes.template get<N - 1>().shape();
    bool ok = true;
    for_each_node([&]<std::size_t K>(const auto& node) {
      constexpr auto& r = Low::rows[K];
      const auto sh = node.shape();
      for (int d = 0; d < r.rank; ++d) {
        int g = -1;
        for (int q = 0; q < Low::root_rank; ++q)
          if (Low::root_labels[q] == r.lab[d]) g = q;
        if (g >= 0) {
          if (sh[d] != gshape[g]) ok = false;
        } else if (sh[d] > r.tile[d]) {
          ok = false;
        }
      }
    });
    // a grid-node mode no input carries cannot be gridded by the level plan
    for (int q = 0; q < Low::root_rank; ++q)
      if (!Low::root_label_staged[q] && gshape[q] > Low::root_tile[q]) ok = false;
    return ok;
  }

  template <typename ES, std::size_t... Roots, typename... ViewTs>
  int launch(int team_size, const ViewTs&... views) const {
    static_assert(sizeof...(Roots) == sizeof...(ViewTs),
                  "DagGraph::execute needs one view per designated output");
    static_assert(std::is_same_v<ES, ExecSpace>,
                  "DagGraph::execute policy tag must match the graph's execution space");
    using ViewT = std::tuple_element_t<0, std::tuple<ViewTs...>>;
    static_assert((std::is_same_v<ViewT, ViewTs> && ...),
                  "DagGraph::execute: output views must share one type");
    if (!index_consistent())
      throw LevelGraphError(
          TO_ERR_INVALID_ARGUMENT,
          "DagGraph: a node's mode is either tiled differently from the grid node's or is "
          "multi-tiled and absent from it, so its tile index cannot be gathered from the grid "
          "node's. Retile so every shared mode matches and every unshared mode has one tile.");
#if defined(__CUDACC__)
    // the spectral-element stiffness shape: one fused line-owner kernel that
    // calls this graph's combine functors (b200/SemFusedDag.hpp)
    if constexpr (b200::SemDagShape<NodesT, Roots...>::ok) {
      cudaError_t fe = cudaSuccess;
      const int league = b200::sem_fused_dag_launch<ValueType, NodesT, Roots...>(nodes, &fe, views...);
      if (league >= 0) {
        if (fe != cudaSuccess)
          throw LevelGraphError(TO_ERR_CUDA, std::string("DagGraph fused launch: ") + cudaGetErrorString(fe));
        return league;
      }
    }
#endif
    if constexpr (b200::tc_candidate<NodesT, ValueType>() && sizeof...(ViewTs) == 1) {
      // one large fp32 contraction of two inputs: a GEMM on the tensor cores
      const int league = b200::tc_try_contract(nodes.template get<0>(), views...);
      if (league >= 0) return league;
    }
    if (needs_contracted_tiles()) {
      using Low = lowering_ktiled;
      const typename Low::graph_t g{Low::make_levels(nodes)};
      return g.template launch<ES, Low::level_slot(Roots)...>(team_size, views...);
    }
    using Low = lowering;
    const typename Low::graph_t g{Low::make_levels(nodes)};
    return g.template launch<ES, Low::level_slot(Roots)...>(team_size, views...);
  }

  using lowering = b200::DagLowering<ValueType, ExecSpace, NodesT, TilesL, false>;
  using lowering_ktiled = b200::DagLowering<ValueType, ExecSpace, NodesT, TilesL, true>;

  // True when a contraction of two inputs has a contracted label longer than
  // its tile: the launch then loops over the contracted tiles.
  bool needs_contracted_tiles() const {
    bool need = false;
    for_each_node([&]<std::size_t K>(const auto& node) {
      using Node = std::decay_t<decltype(node)>;
      if constexpr (b200::dag_is_contraction_v<Node>) {
        if constexpr (b200::dag_is_input_v<typename Node::node_a_type> &&
                      b200::dag_is_input_v<typename Node::node_b_type>) {
          using TS = typename b200::tl_at<K, TilesL>::type;
          constexpr auto ta = b200::dag_operand_tile<Node, TS, 0>();
          constexpr auto la = b200::to_array<typename Node::AL>();
          const auto sh = node.node_a.shape();
          for (std::size_t c = 0; c < Node::contracted.size(); ++c) {
            const int d = b200::index_of(la, Node::contracted[c]);
            if (sh[d] > ta[d]) need = true;
          }
        }
      }
    });
    return need;
  }

  // Slots of the flat DAG (one per node output).
  static constexpr std::size_t num_slots() {
    return [&]<std::size_t... K>(std::index_sequence<K...>) {
      return (std::size_t{0} + ... +
              static_cast<std::size_t>(b200::output_arity<tuple_element_t<K, NodesT>>()));
    }(std::make_index_sequence<N>{});
  }

 private:
  static constexpr std::size_t round16(std::size_t b) { return (b + 15) & ~std::size_t(15); }

  template <typename Node, typename TileSpec, std::size_t... Ms>
  auto add_impl(const Node& node, std::index_sequence<Ms...>) const {
    using NewNodes = decltype(tuple_append(nodes, node));
    using NewTiles = typename b200::tl_append<TilesL, TileSpec>::type;
    constexpr std::size_t Base = num_slots();
    constexpr auto st = b200::dag_storage_tile<Node, TileSpec>();
    using SL = b200::dag_storage_labels_t<Node>;
    using ST = b200::array_tile_t<st>;
    const auto shape = node.shape();
    return std::make_tuple(DagGraph<ValueType, ExecSpace, NewNodes, NewTiles>{tuple_append(nodes, node)},
                           b200::DagSlotHandle<Base + Ms, ValueType, ExecSpace, SL, ST>{shape}...);
  }

  // Bytes of each node-output slot, in slot order.
  template <std::size_t... K>
  static constexpr auto slot_sizes(std::index_sequence<K...>) {
    std::array<std::size_t, num_slots() + 1> out{};
    std::size_t s = 0;
    ((
         [&] {
           using Node = tuple_element_t<K, NodesT>;
           constexpr auto st =
               b200::dag_storage_tile<Node, typename b200::tl_at<K, TilesL>::type>();
           std::size_t e = 1;
           for (int d = 0; d < Node::Rank; ++d) e *= static_cast<std::size_t>(st[d]);
           for (int o = 0; o < b200::output_arity<Node>(); ++o) out[s++] = round16(e * sizeof(ValueType));
         }()),
     ...);
    return out;
  }

  template <std::size_t... K>
  static constexpr std::size_t slot_bytes_impl(std::index_sequence<K...>) {
    return (std::size_t{0} + ... +
            [&] {
              using Node = tuple_element_t<K, NodesT>;
              constexpr auto st =
                  b200::dag_storage_tile<Node, typename b200::tl_at<K, TilesL>::type>();
              std::size_t e = 1;
              for (int d = 0; d < Node::Rank; ++d) e *= static_cast<std::size_t>(st[d]);
              return static_cast<std::size_t>(b200::output_arity<Node>()) *
                     round16(e * sizeof(ValueType));
            }());
  }

  template <typename F>
  void for_each_node(F&& f) const {
    [&]<std::size_t... K>(std::index_sequence<K...>) {
      (f.template operator()<K>(nodes.template get<K>()), ...);
    }(std::make_index_sequence<N>{});
  }
};

template <typename Dag, std::size_t... Roots>
struct DagOutputs {
  Dag dag;
  int team = -1;  // threads per team; <= 0 picks a size from the tile

  DagOutputs team_size(int n) const { return {dag, n}; }

  std::size_t slot_bytes() const { return dag.template pooled_slot_bytes<Roots...>(); }
  std::size_t operand_bytes() const { return dag.arena_bytes(); }
  std::size_t scratch_bytes() const { return slot_bytes() + operand_bytes(); }
  // What a launch requests (the lowered level plan's pooled store).
  std::size_t launch_scratch_bytes() const { return dag.template launch_scratch_bytes<Roots...>(); }

  static constexpr std::size_t num_pools =
      Impl::dag_pool_count<typename Dag::nodes_type, Roots...>();

  template <typename ES, TensorLike... Ts>
  int execute(const TeamPolicyTag<ES>&, const Ts&... ts) const {
    return dag.template launch<ES, Roots...>(team, ts...);
  }
};

template <typename ValueType, typename ExecSpace = Kokkos::DefaultExecutionSpace>
auto make_dag() {
  return DagGraph<ValueType, ExecSpace, DeviceTuple<>, b200::TypeList<>>{DeviceTuple<>{}};
}

}  // namespace TensorOperations
