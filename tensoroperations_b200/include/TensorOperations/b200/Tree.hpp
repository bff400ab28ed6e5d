// Tree.hpp -- the tree route: make_graph().ops(nodes...) / Graph::execute with
// a nested tile bundle, lowered onto the flat DAG and from there onto the level
// plan and the level evaluator.
//
// Public surface as the reference (include/TensorOperations/Graph.hpp:
// Graph::ops :283-293 returning the new graph and one handle per output,
// execute(TeamPolicyTag, tile, views...) :295-310 -- one launch per output
// node, the league sizes summed --, the flat tile-list execute :316-327 whose
// Tile<A,B,C> bundles are taken in pre-order, make_graph :337; Evaluator<
// TeamPolicyTag, Node, Tile>::scratch_size_per_team, Evaluator.hpp:452).
//
// A tree nests its operands: a contraction's A or B, or a combine's operand,
// may itself be a contraction or a combine, and the tile bundle nests the same
// way (Tile<A,B,C> for a contraction, CombineTile<Out, Ops...> for a combine,
// the plain tile for an input).  Lowering walks the tree in post-order and adds
// every inner node to a DagGraph with its own bundle; a nested node becomes a
// slot operand of its parent, read under the labels it was DECLARED with (a
// contraction's declared order, through its storage permutation).  A subtree
// reached twice in a tree is two subtrees, so it is evaluated twice, as in the
// reference; sharing is what the DagGraph route is for.
#pragma once

#include <mutex>
#include <tuple>
#include <vector>

#include <TensorOperations/b200/Dag.hpp>
#include <TensorOperations/b200/TcContract.hpp>

namespace TensorOperations {

template <typename ValueType, typename ExecSpace, typename NodesT, typename TilesL>
struct DagGraph;
template <typename Dag, std::size_t... Roots>
struct DagOutputs;

namespace b200 {

// The plain tile of a bundle: what the node's parent sees as its operand tile.
template <class S>
struct plain_tile {
  using type = S;
};
template <class A, class B, class C>
struct plain_tile<Tile<A, B, C>> {
  using type = C;
};
template <class O, class... Ops>
struct plain_tile<CombineTile<O, Ops...>> {
  using type = O;
};

// The bundle of operand M of a combine: its own entry of a CombineTile, else
// the output tile (an input operand staged in the output's order).
template <class Spec, std::size_t M, bool = is_combine_tile<Spec>::value>
struct combine_op_spec {
  using type = typename combine_out_tile<Spec>::type;
};
template <class Spec, std::size_t M>
struct combine_op_spec<Spec, M, true> {
  using ops = typename Spec::op_types;
  using type = typename std::conditional_t<(M < std::tuple_size_v<ops>),
                                           std::tuple_element<M < std::tuple_size_v<ops> ? M : 0, ops>,
                                           std::type_identity<typename Spec::out_type>>::type;
};

// The operand a parent reads for a node lowered into slot `Slot` with bundle
// TS: its declared labels over its storage tile.
template <class V, class ES, std::size_t Slot, class Node, class TS>
auto declared_operand(const Node& node) {
  constexpr auto st = dag_storage_tile<Node, TS>();
  using STile = array_tile_t<st>;
  if constexpr (dag_is_contraction_v<Node>) {
    constexpr auto perm = label_positions<typename Node::decl_seq, typename Node::canon_seq>();
    using Op = SlotNode<V, ES, Slot, typename Node::decl_seq, STile, array_iseq_t<perm>>;
    const auto sh = node.shape();  // canonical
    Kokkos::Array<int, Node::Rank> decl{};
    for (int d = 0; d < Node::Rank; ++d) decl[d] = sh[perm[d]];
    return Op{decl};
  } else {
    static_assert(Node::NumOut == 1,
                  "Graph: a multi-output combine cannot be an operand of another node on the "
                  "tree route (name its outputs through DagGraph instead)");
    using Op = SlotNode<V, ES, Slot, typename Node::modes_seq, STile,
                        std::make_integer_sequence<int, Node::Rank>>;
    return Op{node.shape()};
  }
}

template <class V, class ES>
struct TreeLowering {
  // Lower `node` (bundle Spec) into `dag`; returns (new dag, the operand a
  // parent reads: the input node itself, or a slot operand).
  template <class Spec, class Dag, class Node>
  static auto run(const Dag& dag, const Node& node) {
    if constexpr (dag_is_input_v<Node>) {
      return std::make_tuple(dag, node);
    } else if constexpr (dag_is_contraction_v<Node>) {
      static_assert(is_contraction_tile<Spec>::value,
                    "Graph::execute: a contraction node's tile must be a Tile<TileA, TileB, "
                    "TileC> bundle");
      const auto ra = run<typename Spec::a_type>(dag, node.node_a);
      const auto rb = run<typename Spec::b_type>(std::get<0>(ra), node.node_b);
      using A = std::decay_t<decltype(std::get<1>(ra))>;
      using B = std::decay_t<decltype(std::get<1>(rb))>;
      using C = NodeHandle<ContractionTag, A, B, typename Node::decl_seq, typename Node::value_type,
                           typename Node::exec_space, typename Node::hook_type>;
      const C c{std::get<1>(ra), std::get<1>(rb), node.shape_, node.hook_op};
      using TS = Tile<typename plain_tile<typename Spec::a_type>::type,
                      typename plain_tile<typename Spec::b_type>::type, typename Spec::c_type>;
      return finish(std::get<0>(rb), c, TS{});
    } else {
      static_assert(dag_is_combine_v<Node>,
                    "Graph::execute: a node is an input, a contraction or a combine");
      return run_combine<Spec, 0>(dag, node);
    }
  }

  template <class Spec, std::size_t M, class Dag, class Node, class... Done>
  static auto run_combine(const Dag& dag, const Node& node, const Done&... done) {
    if constexpr (M == static_cast<std::size_t>(Node::NumOps)) {
      using C = NodeHandle<CombineTag, typename Node::combine_type, typename Node::modes_seq,
                           typename Node::value_type, typename Node::exec_space,
                           std::integral_constant<int, Node::NumOut>, Done...>;
      const C c{node.fn, DeviceTuple<Done...>(done...), node.shape_};
      return finish(dag, c, typename combine_out_tile<Spec>::type{});
    } else {
      const auto r = run<typename combine_op_spec<Spec, M>::type>(
          dag, node.operands.template get<M>());
      return run_combine<Spec, M + 1>(std::get<0>(r), node, done..., std::get<1>(r));
    }
  }

  template <class Dag, class Node, class TS>
  static auto finish(const Dag& dag, const Node& node, const TS& ts) {
    const auto added = dag.add(node, ts);
    constexpr std::size_t slot = std::decay_t<decltype(std::get<1>(added))>::slot_index;
    if constexpr (output_arity<Node>() == 1)
      return std::make_tuple(std::get<0>(added), declared_operand<V, ES, slot, Node, TS>(node));
    else
      return std::make_tuple(std::get<0>(added), 0);  // a multi-output root: no operand
  }

  // The DAG of one output node: the root is the last node added.
  template <class Spec, class Node>
  static auto dag_of(const Node& node) {
    return std::get<0>(run<Spec>(make_dag_empty(), node));
  }
  static auto make_dag_empty() {
    return DagGraph<V, ES, DeviceTuple<>, TypeList<>>{DeviceTuple<>{}};
  }
};

// ---- materialised intermediates --------------------------------------------
// A tree whose nested contraction is read by a parent that contracts one of
// its labels over several tiles cannot run as one fused launch: the level plan
// would have to recompute the child once per contracted tile (reference
// Evaluator.hpp re-evaluates the sub-tree per tile).  Such a tree runs in
// steps instead: each non-input operand of the root is evaluated on its own,
// with its own bundle, into a device buffer in its declared label order, and
// the root then runs as a contraction of two inputs -- the self-staging member
// or the tensor-core GEMM.  Results are the same sums in another order.  A
// fusible tree also runs in steps when its root alone is a large tensor-core
// GEMM (tc_steps_pay): the fused launch would do the root's contraction on
// the CUDA cores.

// Device buffers for those intermediates: kept and reused across launches and
// never handed back to the driver (a cudaFree would synchronise the device on
// every execute).  A buffer belongs to the memory it was allocated in -- the
// host, or one CUDA device -- and is only handed out again for that same
// memory, so a process that runs the frontend on several GPUs never gets one
// device's buffer on another.  Reuse is stream-ordered: the frontend launches
// every evaluation on the default stream.
class IntermediateLease {
 public:
  IntermediateLease() = default;
  IntermediateLease(const IntermediateLease&) = delete;
  IntermediateLease& operator=(const IntermediateLease&) = delete;
  ~IntermediateLease() {
    if (idx_ == kNone) return;
    std::lock_guard<std::mutex> lk(mu());
    pool()[idx_].busy = false;
  }

  // The smallest idle buffer of at least `bytes` in that memory (the host, or
  // the current CUDA device), else a new one.
  void* acquire(std::size_t bytes, bool device) {
    int where = kHost;
#ifdef KOKKOS_ENABLE_CUDA
    if (device) {
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        throw LevelGraphError(TO_ERR_CUDA, "intermediate buffer: no usable current device");
      }
      where = dev;
    }
#endif
    std::lock_guard<std::mutex> lk(mu());
    auto& p = pool();
    std::size_t best = kNone;
    for (std::size_t i = 0; i < p.size(); ++i)
      if (!p[i].busy && p[i].where == where && p[i].bytes >= bytes &&
          (best == kNone || p[i].bytes < p[best].bytes))
        best = i;
    if (best == kNone) {
      p.push_back({Kokkos::Impl::alloc_bytes(bytes, device, "TensorOperations intermediate"), bytes,
                   where, false});
      best = p.size() - 1;
    }
    p[best].busy = true;
    idx_ = best;
    return p[best].ptr;
  }

 private:
  struct Buf {
    void* ptr;
    std::size_t bytes;
    int where;  // kHost, or the CUDA device ordinal
    bool busy;
  };
  static constexpr std::size_t kNone = ~std::size_t(0);
  static constexpr int kHost = -1;
  static std::vector<Buf>& pool() {
    static auto* v = new std::vector<Buf>;  // intentionally never destroyed
    return *v;
  }
  static std::mutex& mu() {
    static auto* m = new std::mutex;
    return *m;
  }
  std::size_t idx_ = kNone;
};

template <class V, int R>
struct ptr_rank {
  using type = typename ptr_rank<V, R - 1>::type*;
};
template <class V>
struct ptr_rank<V, 0> {
  using type = V;
};
template <class V, int R>
using intermediate_view_t =
    Kokkos::View<typename ptr_rank<V, R>::type, Kokkos::LayoutRight, Kokkos::MemoryUnmanaged>;

template <class Node>
constexpr bool has_nested_operand() {
  if constexpr (dag_is_contraction_v<Node>)
    return !dag_is_input_v<typename Node::node_a_type> || !dag_is_input_v<typename Node::node_b_type>;
  else
    return false;
}

// Evaluate operand `node` (bundle Spec) into a leased buffer and return an
// input node over it under the node's declared labels; an input node is
// returned as it is.
template <class Spec, class Node>
auto materialize(const Node& node, IntermediateLease& lease);

// The handle of output M of a multi-output root (its index among the outputs).
template <std::size_t M>
struct OutputHandle : std::integral_constant<std::size_t, M> {
  static constexpr std::size_t OutputIndex = M;
};

// Roots of the lowered tree: the root node's slots, the last ones of the DAG.
template <class Dag, class Seq>
struct tree_outputs;
template <class Dag, std::size_t... M>
struct tree_outputs<Dag, std::index_sequence<M...>> {
  static constexpr std::size_t NS = Dag::num_slots();
  static constexpr std::size_t arity = sizeof...(M);
  using type = DagOutputs<Dag, (NS - arity + M)...>;
};
template <class Node, class Spec>
struct tree_types {
  using V = typename Node::value_type;
  using ES = typename Node::exec_space;
  using dag_t = decltype(TreeLowering<V, ES>::template dag_of<Spec>(std::declval<const Node&>()));
  using outputs_t = typename tree_outputs<
      dag_t, std::make_index_sequence<static_cast<std::size_t>(output_arity<Node>())>>::type;
};

// ---- the flat tile list (pre-order Tile<A,B,C> bundles of a contraction chain)
template <class Node>
constexpr std::size_t count_contractions() {
  if constexpr (dag_is_contraction_v<Node>)
    return 1 + count_contractions<typename Node::node_a_type>() +
           count_contractions<typename Node::node_b_type>();
  else
    return 0;
}
template <std::size_t Offset, class Node, class Tuple>
struct assembled_tile;
template <std::size_t Offset, class Op, class Leaf, class Tuple>
struct assembled_operand {
  static_assert(dag_is_input_v<Op> || dag_is_contraction_v<Op>,
                "flat tile list: a non-contraction operand must be an input node; a fused "
                "combine operand needs its own nested bundle (make_combine_tile) and the "
                "execute overload taking one assembled tile");
  using type = Leaf;
};
template <std::size_t Offset, class Op, class Leaf, class Tuple>
  requires dag_is_contraction_v<Op>
struct assembled_operand<Offset, Op, Leaf, Tuple> {
  using type = typename assembled_tile<Offset, Op, Tuple>::type;
  static_assert(std::is_same_v<Leaf, typename type::c_type>,
                "flat tile list: a parent's operand tile must equal the fused sub-contraction's "
                "output tile (bundle.c)");
};
template <std::size_t Offset, class Node, class Tuple>
struct assembled_tile {
  static_assert(dag_is_contraction_v<Node>, "flat tile list: the output node must be a contraction");
  static_assert(Offset < std::tuple_size_v<Tuple>,
                "flat tile list: fewer Tile<A,B,C> bundles than contraction nodes");
  using bundle = std::tuple_element_t<Offset, Tuple>;
  static constexpr std::size_t offB = Offset + 1 + count_contractions<typename Node::node_a_type>();
  using type = Tile<typename assembled_operand<Offset + 1, typename Node::node_a_type,
                                               typename bundle::a_type, Tuple>::type,
                    typename assembled_operand<offB, typename Node::node_b_type,
                                               typename bundle::b_type, Tuple>::type,
                    typename bundle::c_type>;
};

}  // namespace b200

// ---------------------------------------------------------------------------
// Graph: the tree builder.  OutputTuple holds the nodes of the last ops().
// ---------------------------------------------------------------------------
template <typename OutputTuple = std::tuple<>>
struct Graph {
  OutputTuple outputs{};

  // Register output nodes; returns {new graph, one handle per output}: the node
  // itself for a single-output node (usable as an operand downstream), its
  // output index for each output of a multi-output combine.
  template <typename... Nodes>
  auto ops(const Nodes&... nodes) const {
    using G = Graph<std::tuple<Nodes...>>;
    return std::tuple_cat(std::make_tuple(G{std::make_tuple(nodes...)}), handles_of(nodes)...);
  }

  // One launch per output node, every node with the same bundle; one view per
  // output (the sum of the nodes' output arities).  Returns the summed league.
  template <typename ES, typename Spec, TensorLike... Ts>
  int execute(const TeamPolicyTag<ES>&, const Spec&, const Ts&... ts) const {
    constexpr std::size_t N = std::tuple_size_v<OutputTuple>;
    static_assert(total_arity(std::make_index_sequence<N>{}) == static_cast<int>(sizeof...(Ts)),
                  "execute needs one view per output (sum of output arities)");
    const auto views = std::tie(ts...);
    int league = 0;
    [&]<std::size_t... I>(std::index_sequence<I...>) {
      ((league += run_output<I, Spec>(views)), ...);
    }(std::make_index_sequence<N>{});
    return league;
  }

  // The flat tile-list form of a contraction chain: one Tile<A,B,C> per
  // contraction node in pre-order (node, A subtree, B subtree); single output.
  template <typename ES, typename... Bundles, TensorLike... Ts>
  int execute(const TeamPolicyTag<ES>& tag, const std::tuple<Bundles...>&, const Ts&... ts) const {
    static_assert(std::tuple_size_v<OutputTuple> == 1,
                  "flat tile-list execute supports a single output node");
    static_assert(sizeof...(Ts) == 1, "exactly one output view is required");
    using Node = std::tuple_element_t<0, OutputTuple>;
    using Spec = typename b200::assembled_tile<0, Node, std::tuple<Bundles...>>::type;
    return execute(tag, Spec{}, ts...);
  }

 private:
  template <typename Node>
  static auto handles_of(const Node& n) {
    constexpr int M = b200::output_arity<Node>();
    if constexpr (M == 1)
      return std::make_tuple(n);
    else
      return [&]<std::size_t... Ms>(std::index_sequence<Ms...>) {
        return std::make_tuple(b200::OutputHandle<Ms>{}...);
      }(std::make_index_sequence<static_cast<std::size_t>(M)>{});
  }

  template <std::size_t... I>
  static constexpr int total_arity(std::index_sequence<I...>) {
    return (0 + ... + b200::output_arity<std::tuple_element_t<I, OutputTuple>>());
  }
  template <std::size_t I>
  static constexpr int view_offset() {
    int o = 0;
    [&]<std::size_t... K>(std::index_sequence<K...>) {
      ((o += b200::output_arity<std::tuple_element_t<K, OutputTuple>>()), ...);
    }(std::make_index_sequence<I>{});
    return o;
  }

  template <typename Spec, typename Node, typename Out>
  static int run_in_steps(const Node& node, const Out& out);

  template <std::size_t I, typename Spec, typename Views>
  int run_output(const Views& views) const {
    using Node = std::tuple_element_t<I, OutputTuple>;
    using V = typename Node::value_type;
    using ES = typename Node::exec_space;
    using TT = b200::tree_types<Node, Spec>;
    const auto dag = b200::TreeLowering<V, ES>::template dag_of<Spec>(std::get<I>(outputs));
    const typename TT::outputs_t outs{dag};
    constexpr int off = view_offset<I>();
    if constexpr (b200::has_nested_operand<Node>()) {
      // run in steps when a nested contraction is read over several contracted
      // tiles, or when the root alone is a large tensor-core GEMM
      if (!dag.index_consistent() || b200::tc_steps_pay(std::get<I>(outputs)))
        return run_in_steps<Spec>(std::get<I>(outputs), std::get<off>(views));
    }
    return [&]<std::size_t... K>(std::index_sequence<K...>) {
      return outs.execute(TeamPolicyTag<ES>{}, std::get<off + K>(views)...);
    }(std::make_index_sequence<static_cast<std::size_t>(b200::output_arity<Node>())>{});
  }
};

inline Graph<> make_graph() { return {}; }

namespace b200 {
template <class Spec, class Node>
auto materialize(const Node& node, IntermediateLease& lease) {
  if constexpr (dag_is_input_v<Node>) {
    (void)lease;
    return node;
  } else {
    using V = typename Node::value_type;
    using ES = typename Node::exec_space;
    constexpr int R = Node::Rank;
    using DeclSeq = std::conditional_t<dag_is_contraction_v<Node>, typename Node::decl_seq,
                                       typename Node::modes_seq>;
    static_assert(output_arity<Node>() == 1,
                  "Graph: a multi-output combine cannot be an operand of another node on the "
                  "tree route (name its outputs through DagGraph instead)");
    const auto sh = node.shape();
    std::array<std::size_t, R> ext{};
    for (int d = 0; d < R; ++d) {
      if constexpr (dag_is_contraction_v<Node>) {
        constexpr auto perm = label_positions<typename Node::decl_seq, typename Node::canon_seq>();
        ext[d] = static_cast<std::size_t>(sh[perm[d]]);
      } else {
        ext[d] = static_cast<std::size_t>(sh[d]);
      }
    }
    std::size_t elems = 1;
    for (int d = 0; d < R; ++d) elems *= ext[d];
    using TV = intermediate_view_t<V, R>;
    constexpr bool dev = !std::is_same_v<typename TV::memory_space, Kokkos::HostSpace>;
    V* p = static_cast<V*>(lease.acquire(elems * sizeof(V), dev));
    const TV t = [&]<std::size_t... D>(std::index_sequence<D...>) {
      return TV(p, ext[D]...);
    }(std::make_index_sequence<R>{});
    const auto step = std::get<0>(make_graph().ops(node));
    step.execute(TeamPolicyTag<ES>{}, Spec{}, t);
    return make_input_node(TensorHandle<TV, DeclSeq>{t});
  }
}
}  // namespace b200

template <typename OutputTuple>
template <typename Spec, typename Node, typename Out>
int Graph<OutputTuple>::run_in_steps(const Node& node, const Out& out) {
  using V = typename Node::value_type;
  using ES = typename Node::exec_space;
  b200::IntermediateLease la, lb;
  const auto a = b200::materialize<typename Spec::a_type>(node.node_a, la);
  const auto b = b200::materialize<typename Spec::b_type>(node.node_b, lb);
  using A = std::decay_t<decltype(a)>;
  using B = std::decay_t<decltype(b)>;
  using C = NodeHandle<ContractionTag, A, B, typename Node::decl_seq, V, ES, typename Node::hook_type>;
  const C root{a, b, node.shape_, node.hook_op};
  using TS = Tile<typename b200::plain_tile<typename Spec::a_type>::type,
                  typename b200::plain_tile<typename Spec::b_type>::type, typename Spec::c_type>;
  return std::get<0>(make_graph().ops(root)).execute(TeamPolicyTag<ES>{}, TS{}, out);
}

// Evaluator<TeamPolicyTag<ES>, Node, Spec>::scratch_size_per_team: the scratch
// of `Node` under bundle `Spec` as the reference sizes a tree (reference
// Evaluator.hpp:452): every node's output tile plus every staged operand tile,
// nothing shared -- the same un-pooled sum DagGraph::scratch_bytes() gives the
// tree's DAG spelling.  The launch itself requests the liveness-pooled store,
// which is never larger (pooled_scratch_size_per_team).
template <typename Policy, typename Node, typename Spec>
struct Evaluator;
template <typename ES, typename Node, typename Spec>
struct Evaluator<TeamPolicyTag<ES>, Node, Spec> {
  using dag_t = typename b200::tree_types<Node, Spec>::dag_t;
  using outputs_t = typename b200::tree_types<Node, Spec>::outputs_t;
  static std::size_t scratch_size_per_team(const Spec&) {
    return dag_t::unpooled_slot_bytes() + dag_t::unpooled_operand_bytes();
  }
  static std::size_t pooled_scratch_size_per_team(const Spec&) {
    return pooled_of(static_cast<outputs_t*>(nullptr));
  }

 private:
  template <typename Dag, std::size_t... R>
  static std::size_t pooled_of(DagOutputs<Dag, R...>*) {
    using Low = typename Dag::lowering;
    return b200::Layout<typename Dag::value_type, typename Low::levels_t,
                        Low::level_slot(R)...>::scratch_bytes;
  }
};

}  // namespace TensorOperations
