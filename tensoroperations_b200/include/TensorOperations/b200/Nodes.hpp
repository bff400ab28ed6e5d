// Nodes.hpp -- labelled operands and expression nodes of the level-graph API.
//
// Public factories keep the reference's names, argument order and meaning
// (include/TensorOperations/TensorHandle.hpp:28-32, NodeHandle.hpp:258-322,
// 366-443, 491-610):
//   make_handle<labels...>(view)              a tensor with one label per axis
//   make_input_node(handle)                   an input operand
//   make_stage_node(input)                    "copy this tile on chip"
//   make_contraction_node<out...>(a, b)       C{out} = sum over shared labels of A*B
//   make_combine_node<out...>(ops..., fn)     pointwise fn(coords..., values...)
//   slot.as<labels...>()                      positional relabel of a slot handle
// The node types are this library's own: each carries what the planner and
// the device evaluator need as compile-time constants (labels, the storage
// tile, the declared-to-storage axis map) and nothing else.
//
// Storage conventions (the reference's): a contraction STORES its result in
// canonical order freeA ++ freeB and is DECLARED (read, rooted) in the order
// its output labels name; a combine stores in its output-label order; a stage
// stores in its operand's label order.
#pragma once

#include <cassert>
#include <tuple>

#include <TensorOperations/b200/Labels.hpp>

namespace TensorOperations {

struct InputTag {};
struct IntermTag {};
struct ContractionTag {};
struct CombineTag {};
struct SlotTag {};
struct StagedTag {};
struct StagedContractionTag {};
struct NoHook {};

// ---------------------------------------------------------------------------
// DeviceTuple: a heterogeneous tuple usable in device code.
// ---------------------------------------------------------------------------
// Layout note.  Tuples of nodes travel to the device as kernel parameters, so
// the device pass must place every member at the bytes the host compiler
// wrote.  With an empty `[[no_unique_address]]` member inside a node, nvcc's
// device pass placed the members that follow such a node at other offsets
// than the host compiler (same sizeof; the kernel read a View's extent where
// the host had written its data pointer).  Every type here is therefore built
// from plain members only: the tuple by composition (a head and a tail
// member), nodes without `[[no_unique_address]]`.
namespace b200 {
template <class... T>
struct TupleStore {};
template <class H, class... R>
struct TupleStore<H, R...> {
  H head;
  TupleStore<R...> tail;
};
template <class H>
struct TupleStore<H> {
  H head;
};

template <std::size_t I, class S>
KOKKOS_INLINE_FUNCTION constexpr const auto& store_get(const S& s) {
  if constexpr (I == 0)
    return s.head;
  else
    return store_get<I - 1>(s.tail);
}
template <std::size_t I, class S>
KOKKOS_INLINE_FUNCTION constexpr auto& store_get(S& s) {
  if constexpr (I == 0)
    return s.head;
  else
    return store_get<I - 1>(s.tail);
}
template <class H, class... R>
KOKKOS_INLINE_FUNCTION constexpr TupleStore<H, R...> store_make(const H& h, const R&... r) {
  if constexpr (sizeof...(R) == 0)
    return TupleStore<H>{h};
  else
    return TupleStore<H, R...>{h, store_make(r...)};
}
}  // namespace b200

template <class... T>
struct DeviceTuple {
  static constexpr std::size_t size = sizeof...(T);
  b200::TupleStore<T...> store;

  DeviceTuple() = default;
  template <class... U, class = std::enable_if_t<sizeof...(U) == sizeof...(T) && (sizeof...(T) > 0)>>
  KOKKOS_INLINE_FUNCTION explicit DeviceTuple(const U&... v)
      : store(b200::store_make<T...>(static_cast<const T&>(v)...)) {}

  template <std::size_t I>
  KOKKOS_INLINE_FUNCTION const auto& get() const {
    return b200::store_get<I>(store);
  }
  template <std::size_t I>
  KOKKOS_INLINE_FUNCTION auto& get() {
    return b200::store_get<I>(store);
  }
};

// Free get<I>(tuple), as the reference's DeviceTuple offers.
template <std::size_t I, class... T>
KOKKOS_INLINE_FUNCTION constexpr const auto& get(const DeviceTuple<T...>& t) {
  return t.template get<I>();
}
template <std::size_t I, class... T>
KOKKOS_INLINE_FUNCTION constexpr auto& get(DeviceTuple<T...>& t) {
  return t.template get<I>();
}

template <class Tup>
struct tuple_size;
template <class... T>
struct tuple_size<DeviceTuple<T...>> : std::integral_constant<std::size_t, sizeof...(T)> {};
template <class Tup>
inline constexpr std::size_t tuple_size_v = tuple_size<std::remove_cv_t<Tup>>::value;

template <std::size_t I, class Tup>
struct tuple_element;
template <std::size_t I, class... T>
struct tuple_element<I, DeviceTuple<T...>> {
  using type = std::tuple_element_t<I, std::tuple<T...>>;
};
template <std::size_t I, class Tup>
using tuple_element_t = typename tuple_element<I, std::remove_cv_t<Tup>>::type;

namespace b200 {
template <class... T, class U, std::size_t... I>
KOKKOS_INLINE_FUNCTION DeviceTuple<T..., U> append_impl(const DeviceTuple<T...>& t, const U& u,
                                                       std::index_sequence<I...>) {
  return DeviceTuple<T..., U>(t.template get<I>()..., u);
}
}  // namespace b200
template <class... T, class U>
KOKKOS_INLINE_FUNCTION DeviceTuple<T..., U> tuple_append(const DeviceTuple<T...>& t, const U& u) {
  return b200::append_impl(t, u, std::index_sequence_for<T...>{});
}

// ---------------------------------------------------------------------------
// TensorHandle / make_handle
// ---------------------------------------------------------------------------
template <typename T>
concept TensorLike = requires(T t) {
  requires(static_cast<int>(T::rank) >= 0);
  { t.extent(0) } -> std::convertible_to<std::size_t>;
  t.data();
};

template <TensorLike T, typename ModesSeq>
struct TensorHandle {
  static constexpr int Rank = static_cast<int>(T::rank);
  static_assert(static_cast<int>(ModesSeq::size()) == Rank,
                "TensorHandle: number of mode labels must equal tensor rank");
  static_assert(b200::all_distinct(b200::to_array<ModesSeq>()),
                "TensorHandle: mode labels must be pairwise distinct");
  using modes_seq = ModesSeq;
  using tensor_type = T;
  T tensor;
  KOKKOS_INLINE_FUNCTION std::size_t extent(int d) const { return tensor.extent(d); }
  template <class... I>
  KOKKOS_INLINE_FUNCTION decltype(auto) operator()(I... idx) const {
    return tensor(idx...);
  }
};

template <int32_t... Modes, TensorLike T>
auto make_handle(T base) {
  return TensorHandle<T, Labels<Modes...>>{base};
}

// ---------------------------------------------------------------------------
// Node kinds
// ---------------------------------------------------------------------------
template <typename Tag, typename... Args>
struct NodeHandle;

namespace b200 {
template <class T, class = void>
struct value_of {
  using type = void;
};
template <class T>
struct value_of<T, std::void_t<typename T::value_type>> {
  using type = std::remove_const_t<typename T::value_type>;
};
template <class T, class = void>
struct exec_of {
  using type = Kokkos::DefaultExecutionSpace;
};
template <class T>
struct exec_of<T, std::void_t<typename T::execution_space>> {
  using type = typename T::execution_space;
};
}  // namespace b200

namespace b200 {
// Hooks: op(i_0, ..., i_{Rank-1}, value&) applied in place to every element of
// a node's tile at its global coordinates (reference NodeHandle.hpp:258-266,
// Evaluator.hpp:59-77).
template <int N, typename... Acc>
struct ints_tuple {
  using type = typename ints_tuple<N - 1, int, Acc...>::type;
};
template <typename... Acc>
struct ints_tuple<0, Acc...> {
  using type = std::tuple<Acc...>;
};
template <typename Op, typename V, typename Tup>
struct hook_invocable;
template <typename Op, typename V, typename... Is>
struct hook_invocable<Op, V, std::tuple<Is...>> : std::is_invocable<const Op&, Is..., V&> {};
template <typename Op, int Rank, typename V>
constexpr bool hook_like() {
  if constexpr (std::is_same_v<Op, NoHook>)
    return true;
  else if constexpr (std::is_void_v<V>)
    return false;
  else
    return hook_invocable<Op, V, typename ints_tuple<Rank>::type>::value;
}
}  // namespace b200

// Input: a labelled tensor.
template <typename T, typename ModesSeq, typename HookOp>
struct NodeHandle<InputTag, T, ModesSeq, HookOp> {
  using node_tag = InputTag;
  using tensor_type = T;
  using value_type = typename b200::value_of<T>::type;
  using exec_space = typename b200::exec_of<T>::type;
  using modes_seq = ModesSeq;
  static constexpr int Rank = static_cast<int>(ModesSeq::size());
  TensorHandle<T, ModesSeq> handle;
  HookOp hook_op;  // a plain member: see the layout note above DeviceTuple

  KOKKOS_INLINE_FUNCTION Kokkos::Array<int, Rank> shape() const {
    Kokkos::Array<int, Rank> s{};
    for (int i = 0; i < Rank; ++i) s[i] = static_cast<int>(handle.tensor.extent(i));
    return s;
  }
};

template <typename T, typename ModesSeq, typename HookOp = NoHook>
auto make_input_node(TensorHandle<T, ModesSeq> h, HookOp hook = {}) {
  static_assert(b200::hook_like<HookOp, static_cast<int>(ModesSeq::size()),
                                typename b200::value_of<T>::type>(),
                "input hook must be callable as op(i_0, ..., i_{Rank-1}, value_type&)");
  return NodeHandle<InputTag, T, ModesSeq, HookOp>{h, hook};
}

// Intermediate: a view the evaluator owns, named as a node (reference
// NodeHandle.hpp IntermTag, make_interm_node).  This build's evaluators keep
// intermediates in slots, so the node only carries its storage and tag.
template <typename Storage>
struct NodeHandle<IntermTag, Storage> {
  using node_tag = IntermTag;
  using storage_type = Storage;
  Storage storage;
};

template <typename Storage>
auto make_interm_node(Storage s) {
  return NodeHandle<IntermTag, Storage>{s};
}

// Stage: a tile of an input copied on chip.  Tile is void until the graph
// resolves it from its label map (LevelGraph::add).
template <typename Operand, typename ModesSeq, typename Tile>
struct NodeHandle<StagedTag, Operand, ModesSeq, Tile> {
  using node_tag = StagedTag;
  using operand_type = Operand;
  using tile_type = Tile;
  using value_type = typename Operand::value_type;
  using exec_space = typename Operand::exec_space;
  using modes_seq = ModesSeq;
  static constexpr int Rank = Operand::Rank;
  static_assert(static_cast<int>(ModesSeq::size()) == Rank, "staged node: one label per axis");
  static_assert(b200::all_distinct(b200::to_array<ModesSeq>()),
                "staged node: labels must be distinct");
  Operand operand_;

  KOKKOS_INLINE_FUNCTION Kokkos::Array<int, Rank> shape() const { return operand_.shape(); }

  template <int32_t... Modes>
  auto as() const {
    return NodeHandle<StagedTag, Operand, Labels<Modes...>, void>{operand_};
  }
};

template <typename Operand>
auto make_stage_node(Operand op) {
  static_assert(std::is_same_v<typename Operand::node_tag, InputTag> ||
                    std::is_same_v<typename Operand::node_tag, SlotTag>,
                "make_stage_node: the operand must be an input node (or, in a DAG, a slot)");
  return NodeHandle<StagedTag, Operand, typename Operand::modes_seq, void>{op};
}

// Slot: a labelled read-only view of a buffer produced by a level member.
//   SlotIdx       the slot's index in the graph's flat slot space
//   ModesSeq      the current names of the DECLARED axes (renamed by as<>())
//   StorageTile   the tile in STORAGE order
//   DeclToStore   storage axis of each declared axis
template <typename Value, typename ExecSpace, std::size_t SlotIdx_, typename ModesSeq,
          typename StorageTile, typename DeclToStore>
struct NodeHandle<SlotTag, Value, ExecSpace, std::integral_constant<std::size_t, SlotIdx_>,
                  ModesSeq, StorageTile, DeclToStore> {
  using node_tag = SlotTag;
  using value_type = Value;
  using exec_space = ExecSpace;
  using modes_seq = ModesSeq;
  using storage_tile = StorageTile;
  using decl_to_storage_seq = DeclToStore;
  static constexpr std::size_t SlotIdx = SlotIdx_;
  static constexpr int Rank = static_cast<int>(ModesSeq::size());
  Kokkos::Array<int, Rank> shape_;  // the producer's full extents, declared order

  KOKKOS_INLINE_FUNCTION Kokkos::Array<int, Rank> shape() const { return shape_; }

  template <int32_t... Modes>
  auto as() const {
    static_assert(static_cast<int>(sizeof...(Modes)) == Rank, "slot node as(): one label per axis");
    static_assert(b200::all_distinct(std::array<int32_t, sizeof...(Modes)>{Modes...}),
                  "slot node as(): labels must be distinct");
    return NodeHandle<SlotTag, Value, ExecSpace, std::integral_constant<std::size_t, SlotIdx_>,
                      Labels<Modes...>, StorageTile, DeclToStore>{shape_};
  }
};

template <typename Value, typename ExecSpace, std::size_t Idx, typename ModesSeq,
          typename StorageTile, typename DeclToStore>
using SlotNode = NodeHandle<SlotTag, Value, ExecSpace, std::integral_constant<std::size_t, Idx>,
                            ModesSeq, StorageTile, DeclToStore>;

// ---------------------------------------------------------------------------
// Operand introspection used by the contraction / combine factories.
// ---------------------------------------------------------------------------
namespace b200 {

template <class Node>
inline constexpr bool is_slot_v = std::is_same_v<typename Node::node_tag, SlotTag>;

// Tile extent of each declared axis of an operand (slot operands only carry
// tiles; level-graph operands are always slots).
template <class Node>
constexpr auto operand_tile_by_axis() {
  static_assert(is_slot_v<Node>,
                "level graph: contraction and combine operands must be handles returned "
                "by LevelGraph::add (slots)");
  using ST = typename Node::storage_tile;
  constexpr auto perm = to_array_int<typename Node::decl_to_storage_seq>();
  std::array<int, Node::Rank> out{};
  for (int d = 0; d < Node::Rank; ++d) out[d] = ST::extents[perm[d]];
  return out;
}

}  // namespace b200

// ---------------------------------------------------------------------------
// Contraction
// ---------------------------------------------------------------------------
template <typename NodeA, typename NodeB, typename OutSeq, typename Scalar, typename ExecSpace,
          typename HookOp>
struct NodeHandle<ContractionTag, NodeA, NodeB, OutSeq, Scalar, ExecSpace, HookOp> {
  using node_tag = ContractionTag;
  using node_a_type = NodeA;
  using node_b_type = NodeB;
  using value_type = Scalar;
  using exec_space = ExecSpace;
  using hook_type = HookOp;
  using AL = typename NodeA::modes_seq;
  using BL = typename NodeB::modes_seq;
  static constexpr auto freeA = b200::minus_labels<AL, BL>::values();
  static constexpr auto freeB = b200::minus_labels<BL, AL>::values();
  static constexpr auto contracted = b200::common_labels<AL, BL>::values();
  static constexpr int FreeA = static_cast<int>(freeA.size());
  static constexpr int FreeB = static_cast<int>(freeB.size());
  static constexpr int NumContracted = static_cast<int>(contracted.size());
  static constexpr int Rank = FreeA + FreeB;
  static constexpr int NumOut = 1;
  // canonical (storage) labels freeA ++ freeB, and the user's declared order
  using canon_seq = typename b200::concat_seq<b200::array_seq_t<freeA>, b200::array_seq_t<freeB>>::type;
  using modes_seq = canon_seq;
  using decl_seq = OutSeq;

  NodeA node_a;
  NodeB node_b;
  Kokkos::Array<int, Rank> shape_;  // canonical order
  HookOp hook_op;  // op(i_0.., i_{Rank-1}, value&) on every output element, declared order

  KOKKOS_INLINE_FUNCTION Kokkos::Array<int, Rank> shape() const { return shape_; }
};

namespace b200 {
template <class A, class B, class Out>
constexpr bool valid_contraction() {
  constexpr auto a = to_array<A>();
  constexpr auto b = to_array<B>();
  constexpr auto o = to_array<Out>();
  if (!all_distinct(o)) return false;
  std::size_t nfree = 0;
  for (std::size_t i = 0; i < a.size(); ++i)
    if (index_of(b, a[i]) < 0) ++nfree;
  for (std::size_t i = 0; i < b.size(); ++i)
    if (index_of(a, b[i]) < 0) ++nfree;
  if (nfree != o.size()) return false;
  for (std::size_t i = 0; i < o.size(); ++i) {
    const bool ina = index_of(a, o[i]) >= 0, inb = index_of(b, o[i]) >= 0;
    if (ina == inb) return false;  // in both (contracted) or in neither
  }
  return true;
}
}  // namespace b200

// A staged contraction: a contraction of two input operands as one level
// member that stages the operand tiles itself (one pass per tile of the
// contracted labels).  Built by the DAG lowering, never by user code.
//   InA, InB      the input nodes
//   Contraction   the contraction over slot operands naming the member's own
//                 operand slots (output slot base+1: A's tile, base+2: B's)
template <typename InA, typename InB, typename Contraction>
struct NodeHandle<StagedContractionTag, InA, InB, Contraction> {
  using node_tag = StagedContractionTag;
  using input_a_type = InA;
  using input_b_type = InB;
  using contraction_type = Contraction;
  using value_type = typename Contraction::value_type;
  using exec_space = typename Contraction::exec_space;
  using hook_type = typename Contraction::hook_type;
  using modes_seq = typename Contraction::modes_seq;
  using decl_seq = typename Contraction::decl_seq;
  using canon_seq = typename Contraction::canon_seq;
  static constexpr int Rank = Contraction::Rank;
  static constexpr int NumOut = 1;
  InA in_a;
  InB in_b;
  Contraction c;

  KOKKOS_INLINE_FUNCTION Kokkos::Array<int, Rank> shape() const { return c.shape(); }
};

namespace Impl {
template <typename Scalar, typename ExecSpace, int32_t... OutModes, typename NodeA, typename NodeB,
          typename HookOp>
auto make_contraction_node_impl(NodeA a, NodeB b, HookOp hook) {
  using AL = typename NodeA::modes_seq;
  using BL = typename NodeB::modes_seq;
  using OutSeq = Labels<OutModes...>;
  static_assert(b200::valid_contraction<AL, BL, OutSeq>(),
                "each output mode must appear in exactly one input tensor, output modes "
                "must be pairwise distinct, and the output rank must equal the number "
                "of free modes");
  using Node = NodeHandle<ContractionTag, NodeA, NodeB, OutSeq, Scalar, ExecSpace, HookOp>;
  static_assert(b200::hook_like<HookOp, Node::Rank, Scalar>(),
                "contraction hook must be callable as op(i_0, ..., i_{Rank-1}, value_type&)");
  constexpr auto al = b200::to_array<AL>();
  constexpr auto bl = b200::to_array<BL>();
  const auto as = a.shape();
  const auto bs = b.shape();
  for (std::size_t i = 0; i < Node::contracted.size(); ++i) {
    [[maybe_unused]] const int ea = as[b200::index_of(al, Node::contracted[i])];
    [[maybe_unused]] const int eb = bs[b200::index_of(bl, Node::contracted[i])];
    assert(ea == eb && "contracted mode extents must match between A and B");
  }
  Kokkos::Array<int, Node::Rank> shape{};
  for (int i = 0; i < Node::FreeA; ++i) shape[i] = as[b200::index_of(al, Node::freeA[i])];
  for (int i = 0; i < Node::FreeB; ++i) shape[Node::FreeA + i] = bs[b200::index_of(bl, Node::freeB[i])];
  return Node{a, b, shape, hook};
}
}  // namespace Impl

template <int32_t... OutModes, typename NodeA, typename NodeB, typename HookOp = NoHook>
auto make_contraction_node(NodeA a, NodeB b, HookOp hook = {}) {
  return Impl::make_contraction_node_impl<typename NodeA::value_type,
                                          Kokkos::DefaultExecutionSpace, OutModes...>(a, b, hook);
}
template <typename Scalar, typename ExecSpace = Kokkos::DefaultExecutionSpace, int32_t... OutModes,
          typename NodeA, typename NodeB, typename HookOp = NoHook>
auto make_contraction_node(NodeA a, NodeB b, HookOp hook = {}) {
  return Impl::make_contraction_node_impl<Scalar, ExecSpace, OutModes...>(a, b, hook);
}

// ---------------------------------------------------------------------------
// Combine
// ---------------------------------------------------------------------------
namespace b200 {
template <typename Fn, typename V, std::size_t... Is, std::size_t... Ks>
auto combine_ret(std::index_sequence<Is...>, std::index_sequence<Ks...>)
    -> decltype(std::declval<const Fn&>()((void(Is), 0)..., (void(Ks), std::declval<V>())...));

template <typename Fn, int Rank, int N, typename V>
struct CombineLikeImpl {
  template <class SI, class SK>
  static auto probe(SI is, SK ks) -> decltype((void)combine_ret<Fn, V>(is, ks), std::true_type{});
  static std::false_type probe(...);
  static constexpr bool value =
      decltype(probe(std::make_index_sequence<Rank>{}, std::make_index_sequence<N>{}))::value;
};
template <typename Fn, int Rank, int N, typename V>
using combine_ret_t = decltype(combine_ret<Fn, V>(std::make_index_sequence<Rank>{},
                                                  std::make_index_sequence<N>{}));
template <class R>
struct combine_out {
  static constexpr int num = 1;
  using elem = R;
};
template <class U, std::size_t M>
struct combine_out<Kokkos::Array<U, M>> {
  static constexpr int num = static_cast<int>(M);
  using elem = U;
};
}  // namespace b200

template <typename Fn, int Rank, int N, typename V>
concept CombineLike = b200::CombineLikeImpl<Fn, Rank, N, V>::value;

template <typename CombineFn, typename OutSeq, typename Scalar, typename ExecSpace, int NumOut_,
          typename... Ops>
struct NodeHandle<CombineTag, CombineFn, OutSeq, Scalar, ExecSpace,
                  std::integral_constant<int, NumOut_>, Ops...> {
  using node_tag = CombineTag;
  using combine_type = CombineFn;
  using value_type = Scalar;
  using exec_space = ExecSpace;
  using modes_seq = OutSeq;
  using decl_seq = OutSeq;
  using ops_tuple_t = DeviceTuple<Ops...>;
  static constexpr int Rank = static_cast<int>(OutSeq::size());
  static constexpr int NumOps = static_cast<int>(sizeof...(Ops));
  static constexpr int NumOut = NumOut_;
  CombineFn fn;  // a plain member: see the layout note above DeviceTuple
  ops_tuple_t operands;
  Kokkos::Array<int, Rank> shape_;

  KOKKOS_INLINE_FUNCTION Kokkos::Array<int, Rank> shape() const { return shape_; }
};

namespace Impl {
template <typename OutSeq, typename Op>
Kokkos::Array<int, OutSeq::size()> gathered_shape(const Op& op) {
  constexpr auto o = b200::to_array<OutSeq>();
  constexpr auto l = b200::to_array<typename Op::modes_seq>();
  const auto s = op.shape();
  Kokkos::Array<int, OutSeq::size()> out{};
  for (std::size_t i = 0; i < o.size(); ++i) out[i] = s[b200::index_of(l, o[i])];
  return out;
}

template <typename Scalar, typename ExecSpace, int32_t... OutModes, typename Fn, typename... Ops>
auto make_combine_node_impl(Fn fn, Ops... ops) {
  constexpr int Rank = static_cast<int>(sizeof...(OutModes));
  constexpr int N = static_cast<int>(sizeof...(Ops));
  using OutSeq = Labels<OutModes...>;
  static_assert(N >= 1, "combine node needs at least one operand");
  static_assert(((static_cast<int>(Ops::Rank) == Rank) && ...),
                "combine node: every operand and the output must have equal rank");
  static_assert(b200::all_distinct(b200::to_array<OutSeq>()),
                "combine node: output labels must be pairwise distinct");
  static_assert((b200::same_label_set<typename Ops::modes_seq, OutSeq>() && ...),
                "combine node: each operand's label set must equal the output label set "
                "(a pointwise op reduces no mode)");
  static_assert(CombineLike<Fn, Rank, N, Scalar>,
                "combine fn must be const-callable as "
                "fn(i_0, ..., i_{Rank-1}, v_0, ..., v_{N-1}) -> value_type "
                "(the evaluator invokes it through a const kernel capture)");
  using Info = b200::combine_out<b200::combine_ret_t<Fn, Rank, N, Scalar>>;
  static_assert(std::is_convertible_v<typename Info::elem, Scalar>,
                "combine fn output element type must be convertible to the operand scalar "
                "(multi-output combine is homogeneous)");
  const std::array<Kokkos::Array<int, Rank>, N> shapes{gathered_shape<OutSeq>(ops)...};
  for (int k = 1; k < N; ++k)
    for (int i = 0; i < Rank; ++i)
      assert(shapes[k][i] == shapes[0][i] &&
             "combine node: operand extents must match on every mode");
  using Node = NodeHandle<CombineTag, Fn, OutSeq, Scalar, ExecSpace,
                          std::integral_constant<int, Info::num>, Ops...>;
  return Node{fn, DeviceTuple<Ops...>(ops...), shapes[0]};
}

template <typename Scalar, typename ExecSpace, int32_t... OutModes, typename Tuple, std::size_t... Is>
auto combine_from_args(Tuple args, std::index_sequence<Is...>) {
  return make_combine_node_impl<Scalar, ExecSpace, OutModes...>(std::get<sizeof...(Is)>(args),
                                                               std::get<Is>(args)...);
}
}  // namespace Impl

template <int32_t... OutModes, typename... Args>
auto make_combine_node(Args... args) {
  static_assert(sizeof...(Args) >= 2,
                "make_combine_node needs at least one operand and a combine fn");
  using First = std::tuple_element_t<0, std::tuple<Args...>>;
  return Impl::combine_from_args<typename First::value_type, Kokkos::DefaultExecutionSpace,
                                 OutModes...>(std::tuple<Args...>(args...),
                                              std::make_index_sequence<sizeof...(Args) - 1>{});
}
template <typename Scalar, typename ExecSpace = Kokkos::DefaultExecutionSpace, int32_t... OutModes,
          typename... Args>
auto make_combine_node(Args... args) {
  static_assert(sizeof...(Args) >= 2,
                "make_combine_node needs at least one operand and a combine fn");
  return Impl::combine_from_args<Scalar, ExecSpace, OutModes...>(
      std::tuple<Args...>(args...), std::make_index_sequence<sizeof...(Args) - 1>{});
}

}  // namespace TensorOperations
