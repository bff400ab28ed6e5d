// LevelKernel.cuh -- the generic level-graph evaluator for sm_100a.
//
// One CTA per grid tile (the product of the blocked labels' tile counts); the
// CTA's dynamic shared memory holds the graph's pooled slots at compile-time
// offsets.  Levels run in order, separated by one __syncthreads each:
//   stage        every member copies its input tile (global -> slot) in ONE
//                loop over the shared tile layout, so all loads are in flight
//                together (reference: LevelGraph.hpp:346-365);
//   contraction  items (a, b) of SA x SB; each member accumulates
//                sum_k A[a,k] B[k,b] over the contracted labels with every
//                stride a compile-time constant (reference: Team2.hpp:229-317);
//   staged contraction
//                a contraction of two inputs that stages its own operand
//                tiles, one pass per tile of the contracted labels, and
//                accumulates (reference Team.hpp Spec 4 with tiled K);
//   combine      for every output coordinate, gather the operands through
//                their label permutations and call fn at the GLOBAL coordinate
//                (reference: Team2.hpp:431-544);
// then every root slot is written to its output view in declared order,
// traversing the destination contiguously (reference: LevelGraph.hpp:397-426).
// Coordinates past the end of a tensor (a partial last tile) are never read,
// written or handed to a combine fn.
#pragma once

#include <TensorOperations/b200/Plan.hpp>

namespace TensorOperations {
namespace b200 {

template <int GR>
struct GridRuntime {
  int ntiles[GR > 0 ? GR : 1];
};

// Calls f(std::integral_constant<int, D>{}) for D = 0 .. N-1: per-axis loops
// in device code are compile-time folds, so every label, extent and stride
// they touch is a constant and no host table is read at run time.
template <int N, class F>
__device__ __forceinline__ void static_for(F&& f) {
  [&]<int... D>(std::integer_sequence<int, D...>) {
    (f(std::integral_constant<int, D>{}), ...);
  }(std::make_integer_sequence<int, N>{});
}

// Origin of label L in the tile this CTA owns.
template <class GS, class LT, int32_t L>
__device__ __forceinline__ int label_origin(const int* tile_idx) {
  constexpr int g = GS::grid_slot(L);
  if constexpr (g < 0) {
    return 0;
  } else {
    constexpr int t = LT::tile(L);
    return tile_idx[g] * t;
  }
}

template <class Tile>
__device__ __forceinline__ void decode_tile(int t, int* c) {
  static_for<Tile::rank>([&](auto dc) {
    constexpr int d = Tile::rank - 1 - decltype(dc)::value;
    constexpr int e = Tile::extents[d];
    c[d] = t % e;
    t /= e;
  });
}

template <class View, std::size_t... I>
__device__ __forceinline__ auto& view_at(const View& v, const long long* g, std::index_sequence<I...>) {
  return v(g[I]...);
}

template <class Op, class C, class V, std::size_t... I>
__device__ __forceinline__ void call_hook(const Op& op, const C* g, V& v, std::index_sequence<I...>) {
  op(static_cast<int>(g[I])..., v);
}

template <class V, class Lay, std::size_t S>
__device__ __forceinline__ V* slot_ptr(unsigned char* smem) {
  constexpr std::size_t off = Lay::slot_offset(S);
  return reinterpret_cast<V*>(smem + off);
}

// ---- stage ---------------------------------------------------------------
template <class V, class Lay, class GS, class LT, class Levels, std::size_t L, std::size_t M>
__device__ __forceinline__ void stage_one(const tuple_element_t<M, tuple_element_t<L, Levels>>& node,
                                          const int* c, int t, const int* tile_idx,
                                          unsigned char* smem) {
  using Node = tuple_element_t<M, tuple_element_t<L, Levels>>;
  constexpr std::size_t S = Algebra<Levels>::member_base(L, M);
  constexpr int R = Node::Rank;
  constexpr auto lab = to_array<typename Node::modes_seq>();
  const auto& view = node.operand_.handle.tensor;
  long long g[R > 0 ? R : 1];
  bool in = true;
  static_for<R>([&](auto dc) {
    constexpr int d = decltype(dc)::value;
    constexpr int32_t l = lab[d];
    g[d] = label_origin<GS, LT, l>(tile_idx) + c[d];
    in = in && g[d] < static_cast<long long>(view.extent(d));
  });
  V* out = slot_ptr<V, Lay, S>(smem);
  V v = in ? static_cast<V>(view_at(view, g, std::make_index_sequence<R>{})) : V(0);
  using Hook = decltype(node.operand_.hook_op);
  if constexpr (!std::is_same_v<Hook, NoHook>) {
    if (in) call_hook(node.operand_.hook_op, g, v, std::make_index_sequence<R>{});
  }
  out[t] = v;
}

template <class V, class Lay, class GS, class LT, class Levels, std::size_t L, std::size_t... M>
__device__ void run_stage_level(const tuple_element_t<L, Levels>& lvl, const int* tile_idx,
                                unsigned char* smem, std::index_sequence<M...>) {
  using Tile = typename member_traits<tuple_element_t<0, tuple_element_t<L, Levels>>>::tile;
  for (int t = threadIdx.x; t < Tile::num_elements; t += blockDim.x) {
    int c[Tile::rank > 0 ? Tile::rank : 1];
    decode_tile<Tile>(t, c);
    (stage_one<V, Lay, GS, LT, Levels, L, M>(lvl.template get<M>(), c, t, tile_idx, smem), ...);
  }
}

// ---- contraction -----------------------------------------------------------
// Offsets of a flat index decoded over a list of labels (row-major in the
// list's order) into a slot operand X.
template <class X, auto Labs>
__device__ __forceinline__ int label_offset(int idx) {
  constexpr int n = static_cast<int>(Labs.size());
  int off = 0;
  static_for<n>([&](auto dc) {
    constexpr int d = n - 1 - decltype(dc)::value;
    constexpr int e = operand_label_extent<X>(Labs[d]);
    constexpr int st = operand_label_stride<X>(Labs[d]);
    off += (idx % e) * st;
    idx /= e;
  });
  return off;
}
// The same decode for the contracted labels, extents taken from A.
template <class A, class X, auto Labs>
__device__ __forceinline__ int label_offset_extents_of(int idx) {
  constexpr int n = static_cast<int>(Labs.size());
  int off = 0;
  static_for<n>([&](auto dc) {
    constexpr int d = n - 1 - decltype(dc)::value;
    constexpr int e = operand_label_extent<A>(Labs[d]);
    constexpr int st = operand_label_stride<X>(Labs[d]);
    off += (idx % e) * st;
    idx /= e;
  });
  return off;
}

// One output element t = (a, b) of contraction node Cn into slot SOut:
// sum_k A[a,k] B[k,b] (added to the slot's value when `accumulate`), then the
// node's hook when `hook` (the last pass).
template <class V, class Lay, class GS, class LT, class Cn, std::size_t SOut>
__device__ __forceinline__ void contract_core(const Cn& node, const int* tile_idx,
                                              unsigned char* smem, int a, int b, int t,
                                              bool accumulate, bool hook) {
  using A = typename Cn::node_a_type;
  using B = typename Cn::node_b_type;
  using MT = member_traits<Cn, ContractionTag>;
  constexpr auto freeA = Cn::freeA;
  constexpr auto freeB = Cn::freeB;
  constexpr auto cont = Cn::contracted;
  constexpr int SK = MT::sk;
  const V* pa = slot_ptr<V, Lay, A::SlotIdx>(smem) + label_offset<A, freeA>(a);
  const V* pb = slot_ptr<V, Lay, B::SlotIdx>(smem) + label_offset<B, freeB>(b);
  V* out = slot_ptr<V, Lay, SOut>(smem);
  V acc = accumulate ? out[t] : V(0);
  if constexpr (SK <= 64) {
    static_for<SK>([&](auto kc) {
      constexpr int k = decltype(kc)::value;
      acc += pa[label_offset_extents_of<A, A, cont>(k)] * pb[label_offset_extents_of<A, B, cont>(k)];
    });
  } else {
#pragma unroll 8
    for (int k = 0; k < SK; ++k)
      acc += pa[label_offset_extents_of<A, A, cont>(k)] * pb[label_offset_extents_of<A, B, cont>(k)];
  }
  if constexpr (!std::is_same_v<typename Cn::hook_type, NoHook>) {
    if (hook) {
      // the element's global coordinates in the node's DECLARED order
      constexpr int R = Cn::Rank;
      using STile = typename MT::tile;
      constexpr auto decl = to_array<typename MT::decl_labels>();
      constexpr auto perm = MT::decl_to_storage;
      int c[R > 0 ? R : 1];
      decode_tile<STile>(t, c);
      long long g[R > 0 ? R : 1];
      bool in = true;
      const auto shape = node.shape();  // canonical
      static_for<R>([&](auto dc) {
        constexpr int d = decltype(dc)::value;
        constexpr int32_t l = decl[d];
        g[d] = label_origin<GS, LT, l>(tile_idx) + c[perm[d]];
        in = in && g[d] < shape[perm[d]];
      });
      if (in) call_hook(node.hook_op, g, acc, std::make_index_sequence<R>{});
    }
  } else {
    (void)hook;
    (void)tile_idx;
  }
  out[t] = acc;
}

template <class V, class Lay, class GS, class LT, class Levels, std::size_t L, std::size_t M>
__device__ __forceinline__ void contract_one(const tuple_element_t<M, tuple_element_t<L, Levels>>& node,
                                             const int* tile_idx, unsigned char* smem, int a, int b,
                                             int t) {
  constexpr std::size_t SC = Algebra<Levels>::member_base(L, M);
  contract_core<V, Lay, GS, LT, tuple_element_t<M, tuple_element_t<L, Levels>>, SC>(
      node, tile_idx, smem, a, b, t, false, true);
}

template <class V, class Lay, class GS, class LT, class Levels, std::size_t L, std::size_t... M>
__device__ void run_contraction_level(const tuple_element_t<L, Levels>& lvl, const int* tile_idx,
                                      unsigned char* smem, std::index_sequence<M...>) {
  using MT0 = member_traits<tuple_element_t<0, tuple_element_t<L, Levels>>>;
  constexpr int SA = MT0::sa, SB = MT0::sb;
  for (int t = threadIdx.x; t < SA * SB; t += blockDim.x) {
    const int a = t / SB;
    const int b = t - a * SB;
    (contract_one<V, Lay, GS, LT, Levels, L, M>(lvl.template get<M>(), tile_idx, smem, a, b, t), ...);
  }
}

// ---- staged contraction ------------------------------------------------------
// Tiles of the contracted labels (row-major over them in the node's contracted
// order), from operand A's extents; at least one.
template <class Node>
__device__ __forceinline__ int sc_num_ktiles(const Node& node) {
  using C = typename Node::contraction_type;
  using SA = typename C::node_a_type;
  constexpr auto la = to_array<typename Node::input_a_type::modes_seq>();
  int n = 1;
  static_for<C::NumContracted>([&](auto ic) {
    constexpr int d = index_of(la, C::contracted[decltype(ic)::value]);
    constexpr int tile = SA::storage_tile::extents[d];
    const int e = static_cast<int>(node.in_a.handle.tensor.extent(d));
    n *= (e + tile - 1) / tile;
  });
  return n > 0 ? n : 1;
}

// Element t of operand `in` (an input node) into its tile slot SlotOp for
// contracted tile kidx: contracted labels at that tile, free labels at the
// team's grid tile.
template <class V, class Lay, class GS, class LT, class C, class In, class SlotOp>
__device__ __forceinline__ void sc_stage_elem(const In& in, const int* kidx, const int* tile_idx,
                                              unsigned char* smem, int t) {
  using Tile = typename SlotOp::storage_tile;
  constexpr int R = In::Rank;
  constexpr auto lab = to_array<typename In::modes_seq>();
  const auto& view = in.handle.tensor;
  int c[R > 0 ? R : 1];
  decode_tile<Tile>(t, c);
  long long g[R > 0 ? R : 1];
  bool inr = true;
  static_for<R>([&](auto dc) {
    constexpr int d = decltype(dc)::value;
    constexpr int32_t l = lab[d];
    constexpr int ci = index_of(C::contracted, l);
    long long o;
    if constexpr (ci >= 0)
      o = static_cast<long long>(kidx[ci]) * Tile::extents[d];
    else
      o = label_origin<GS, LT, l>(tile_idx);
    g[d] = o + c[d];
    inr = inr && g[d] < static_cast<long long>(view.extent(d));
  });
  V v = inr ? static_cast<V>(view_at(view, g, std::make_index_sequence<R>{})) : V(0);
  using Hook = decltype(in.hook_op);
  if constexpr (!std::is_same_v<Hook, NoHook>) {
    if (inr) call_hook(in.hook_op, g, v, std::make_index_sequence<R>{});
  }
  slot_ptr<V, Lay, SlotOp::SlotIdx>(smem)[t] = v;
}

template <class Node>
__device__ __forceinline__ void sc_kidx(const Node& node, int kt, int* kidx) {
  using C = typename Node::contraction_type;
  using SA = typename C::node_a_type;
  constexpr auto la = to_array<typename Node::input_a_type::modes_seq>();
  static_for<C::NumContracted>([&](auto icr) {
    constexpr int i = C::NumContracted - 1 - decltype(icr)::value;
    constexpr int d = index_of(la, C::contracted[i]);
    constexpr int tile = SA::storage_tile::extents[d];
    const int e = static_cast<int>(node.in_a.handle.tensor.extent(d));
    const int n = e > 0 ? (e + tile - 1) / tile : 1;
    kidx[i] = kt % n;
    kt /= n;
  });
}

template <class Node>
constexpr int sc_tile_elems() {
  using C = typename Node::contraction_type;
  constexpr int a = C::node_a_type::storage_tile::num_elements;
  constexpr int b = C::node_b_type::storage_tile::num_elements;
  return a > b ? a : b;
}
template <class Lvl, std::size_t... M>
constexpr int sc_level_tile_elems(std::index_sequence<M...>) {
  int m = 0;
  ((m = sc_tile_elems<tuple_element_t<M, Lvl>>() > m ? sc_tile_elems<tuple_element_t<M, Lvl>>() : m),
   ...);
  return m;
}
template <class Lvl, std::size_t... M>
constexpr int sc_level_max_contracted(std::index_sequence<M...>) {
  int m = 1;
  ((m = tuple_element_t<M, Lvl>::contraction_type::NumContracted > m
            ? tuple_element_t<M, Lvl>::contraction_type::NumContracted
            : m),
   ...);
  return m;
}

// One pass of a staged-contraction level: every member whose contracted tile
// kt exists stages both operand tiles in ONE loop over the level's widest
// tile (all loads in flight together, as in a stage level), then accumulates.
// SINGLE: every member has one contracted tile (kt = 0, nothing to add to,
// the hook applies) -- the common case, compiled without the loop's
// run-time indices.
template <bool SINGLE, class V, class Lay, class GS, class LT, class Levels, std::size_t L,
          std::size_t... M>
__device__ __forceinline__ void sc_pass(const tuple_element_t<L, Levels>& lvl, const int* tile_idx,
                                        unsigned char* smem, int kt, const int* nk,
                                        std::index_sequence<M...>) {
  using Lvl = tuple_element_t<L, Levels>;
  using MT0 = member_traits<tuple_element_t<0, Lvl>>;
  constexpr int SA = MT0::sa, SB = MT0::sb;
  constexpr int NM = sizeof...(M);
  constexpr int TMAX = sc_level_tile_elems<Lvl>(std::index_sequence<M...>{});
  constexpr int MC = sc_level_max_contracted<Lvl>(std::index_sequence<M...>{});
  int kidx[NM][MC];
  if constexpr (SINGLE) {
    for (int m = 0; m < NM; ++m)
      for (int c = 0; c < MC; ++c) kidx[m][c] = 0;
  } else {
    (sc_kidx(lvl.template get<M>(), kt, kidx[M]), ...);
  }
  for (int t = threadIdx.x; t < TMAX; t += blockDim.x) {
    (
        [&] {
          using Node = tuple_element_t<M, Lvl>;
          using C = typename Node::contraction_type;
          if (SINGLE || kt < nk[M]) {
            const Node& node = lvl.template get<M>();
            if (t < C::node_a_type::storage_tile::num_elements)
              sc_stage_elem<V, Lay, GS, LT, C, typename Node::input_a_type, typename C::node_a_type>(
                  node.in_a, kidx[M], tile_idx, smem, t);
            if (t < C::node_b_type::storage_tile::num_elements)
              sc_stage_elem<V, Lay, GS, LT, C, typename Node::input_b_type, typename C::node_b_type>(
                  node.in_b, kidx[M], tile_idx, smem, t);
          }
        }(),
        ...);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < SA * SB; t += blockDim.x) {
    const int a = t / SB;
    const int b = t - a * SB;
    (
        [&] {
          using Node = tuple_element_t<M, Lvl>;
          constexpr std::size_t S = Algebra<Levels>::member_base(L, M);
          if constexpr (SINGLE) {
            contract_core<V, Lay, GS, LT, typename Node::contraction_type, S>(
                lvl.template get<M>().c, tile_idx, smem, a, b, t, false, true);
          } else {
            if (kt < nk[M])
              contract_core<V, Lay, GS, LT, typename Node::contraction_type, S>(
                  lvl.template get<M>().c, tile_idx, smem, a, b, t, kt > 0, kt == nk[M] - 1);
          }
        }(),
        ...);
  }
}

template <class V, class Lay, class GS, class LT, class Levels, std::size_t L, std::size_t... M>
__device__ void run_sc_level(const tuple_element_t<L, Levels>& lvl, const int* tile_idx,
                             unsigned char* smem, std::index_sequence<M...>) {
  constexpr int NM = sizeof...(M);
  const int nk[NM] = {sc_num_ktiles(lvl.template get<M>())...};
  int NK = 1;
  for (int m = 0; m < NM; ++m) NK = nk[m] > NK ? nk[m] : NK;
  if (NK == 1) {
    sc_pass<true, V, Lay, GS, LT, Levels, L>(lvl, tile_idx, smem, 0, nk, std::index_sequence<M...>{});
    return;
  }
  for (int kt = 0; kt < NK; ++kt) {
    sc_pass<false, V, Lay, GS, LT, Levels, L>(lvl, tile_idx, smem, kt, nk, std::index_sequence<M...>{});
    if (kt + 1 < NK) __syncthreads();  // the next pass overwrites the operand tiles
  }
}

// ---- combine ---------------------------------------------------------------
template <class Fn, class V, std::size_t... I, std::size_t... K>
__device__ __forceinline__ auto call_combine(const Fn& fn, const int* gc, const V* vals,
                                             std::index_sequence<I...>, std::index_sequence<K...>) {
  return fn(gc[I]..., vals[K]...);
}

template <class V, class Lay, class Levels, class Node, std::size_t K>
__device__ __forceinline__ V combine_operand(unsigned char* smem, const int* c) {
  using Op = tuple_element_t<K, typename Node::ops_tuple_t>;
  constexpr auto o = to_array<typename Node::modes_seq>();
  int off = 0;
  static_for<Node::Rank>([&](auto dc) {
    constexpr int d = decltype(dc)::value;
    constexpr int st = operand_label_stride<Op>(o[d]);
    off += c[d] * st;
  });
  return slot_ptr<V, Lay, Op::SlotIdx>(smem)[off];
}

template <class V, class Lay, class GS, class LT, class Levels, std::size_t L, std::size_t M,
          std::size_t... K>
__device__ __forceinline__ void combine_one(const tuple_element_t<M, tuple_element_t<L, Levels>>& node,
                                            const int* c, int t, const int* tile_idx,
                                            unsigned char* smem, std::index_sequence<K...>) {
  using Node = tuple_element_t<M, tuple_element_t<L, Levels>>;
  constexpr std::size_t S = Algebra<Levels>::member_base(L, M);
  constexpr int R = Node::Rank;
  constexpr auto o = to_array<typename Node::modes_seq>();
  int gc[R > 0 ? R : 1];
  bool in = true;
  const auto shape = node.shape();
  static_for<R>([&](auto dc) {
    constexpr int d = decltype(dc)::value;
    constexpr int32_t l = o[d];
    gc[d] = label_origin<GS, LT, l>(tile_idx) + c[d];
    in = in && gc[d] < shape[d];
  });
  if constexpr (Node::NumOut == 1) {
    V r = V(0);
    if (in) {
      const V vals[sizeof...(K)] = {combine_operand<V, Lay, Levels, Node, K>(smem, c)...};
      r = static_cast<V>(call_combine(node.fn, gc, vals, std::make_index_sequence<R>{},
                                      std::make_index_sequence<sizeof...(K)>{}));
    }
    slot_ptr<V, Lay, S>(smem)[t] = r;
  } else {
    if (in) {
      const V vals[sizeof...(K)] = {combine_operand<V, Lay, Levels, Node, K>(smem, c)...};
      const auto r = call_combine(node.fn, gc, vals, std::make_index_sequence<R>{},
                                  std::make_index_sequence<sizeof...(K)>{});
      [&]<std::size_t... O>(std::index_sequence<O...>) {
        ((slot_ptr<V, Lay, S + O>(smem)[t] = static_cast<V>(r[O])), ...);
      }(std::make_index_sequence<Node::NumOut>{});
    } else {
      [&]<std::size_t... O>(std::index_sequence<O...>) {
        ((slot_ptr<V, Lay, S + O>(smem)[t] = V(0)), ...);
      }(std::make_index_sequence<Node::NumOut>{});
    }
  }
}

template <class V, class Lay, class GS, class LT, class Levels, std::size_t L, std::size_t... M>
__device__ void run_combine_level(const tuple_element_t<L, Levels>& lvl, const int* tile_idx,
                                  unsigned char* smem, std::index_sequence<M...>) {
  using Tile = typename member_traits<tuple_element_t<0, tuple_element_t<L, Levels>>>::tile;
  for (int t = threadIdx.x; t < Tile::num_elements; t += blockDim.x) {
    int c[Tile::rank > 0 ? Tile::rank : 1];
    decode_tile<Tile>(t, c);
    (combine_one<V, Lay, GS, LT, Levels, L, M>(
         lvl.template get<M>(), c, t, tile_idx, smem,
         std::make_index_sequence<tuple_element_t<M, tuple_element_t<L, Levels>>::NumOps>{}),
     ...);
  }
}

// ---- levels and roots ---------------------------------------------------------
template <class V, class Lay, class GS, class LT, class Levels, std::size_t L>
__device__ __forceinline__ void run_level(const Levels& levels, const int* tile_idx,
                                          unsigned char* smem) {
  using Lvl = tuple_element_t<L, Levels>;
  constexpr int kind = member_traits<tuple_element_t<0, Lvl>>::kind;
  using Ms = std::make_index_sequence<tuple_size_v<Lvl>>;
  if constexpr (kind == 0)
    run_stage_level<V, Lay, GS, LT, Levels, L>(levels.template get<L>(), tile_idx, smem, Ms{});
  else if constexpr (kind == 1)
    run_contraction_level<V, Lay, GS, LT, Levels, L>(levels.template get<L>(), tile_idx, smem, Ms{});
  else if constexpr (kind == 3)
    run_sc_level<V, Lay, GS, LT, Levels, L>(levels.template get<L>(), tile_idx, smem, Ms{});
  else
    run_combine_level<V, Lay, GS, LT, Levels, L>(levels.template get<L>(), tile_idx, smem, Ms{});
  __syncthreads();
}

template <class V, class Lay, class GS, class LT, class Levels, std::size_t S, class View>
__device__ __forceinline__ void store_root(const View& view, const int* tile_idx,
                                           unsigned char* smem) {
  using SN = slot_member_node<Levels, S>;
  using MT = member_traits<typename SN::type>;
  constexpr int R = MT::rank;
  constexpr auto decl = to_array<typename MT::decl_labels>();
  constexpr auto perm = MT::decl_to_storage;
  using STile = typename MT::tile;
  constexpr auto sstride = tile_strides<STile>();
  // declared-order tile extents (no local captured: every value is a constant)
  constexpr auto dext = [] {
    std::array<int, R> e{};
    for (int d = 0; d < R; ++d) e[d] = STile::extents[MT::decl_to_storage[d]];
    return e;
  }();
  using DTile = array_tile_t<dext>;
  const V* src = slot_ptr<V, Lay, S>(smem);
  for (int t = threadIdx.x; t < DTile::num_elements; t += blockDim.x) {
    int c[R > 0 ? R : 1];
    decode_tile<DTile>(t, c);
    long long g[R > 0 ? R : 1];
    int off = 0;
    bool in = true;
    static_for<R>([&](auto dc) {
      constexpr int d = decltype(dc)::value;
      constexpr int st = sstride[perm[d]];
      constexpr int32_t l = decl[d];
      off += c[d] * st;
      g[d] = label_origin<GS, LT, l>(tile_idx) + c[d];
      in = in && g[d] < static_cast<long long>(view.extent(d));
    });
    if (in) view_at(view, g, std::make_index_sequence<R>{}) = src[off];
  }
}

template <class V, class Lay, class GS, class LT, class Levels, class Views, std::size_t... R,
          std::size_t... S>
__device__ __forceinline__ void store_roots(const Views& views, const int* tile_idx,
                                            unsigned char* smem, std::index_sequence<R...>,
                                            std::index_sequence<S...>) {
  (store_root<V, Lay, GS, LT, Levels, S>(views.template get<R>(), tile_idx, smem), ...);
}

template <class V, class LT, class Levels, std::size_t... Roots>
struct GraphKernel {
  using GS = GridSpec<LT, Levels>;
  using Lay = Layout<V, Levels, Roots...>;
  static constexpr int GR = GS::rank;

  template <class Views>
  __device__ static void run(const Levels& levels, const GridRuntime<GR>& grid, const Views& views) {
    extern __shared__ __align__(16) unsigned char lg_smem[];
    int tile_idx[GR > 0 ? GR : 1];
    int r = static_cast<int>(blockIdx.x);
#pragma unroll
    for (int d = GR - 1; d >= 0; --d) {
      tile_idx[d] = r % grid.ntiles[d];
      r /= grid.ntiles[d];
    }
    [&]<std::size_t... L>(std::index_sequence<L...>) {
      (run_level<V, Lay, GS, LT, Levels, L>(levels, tile_idx, lg_smem), ...);
    }(std::make_index_sequence<tuple_size_v<Levels>>{});
    store_roots<V, Lay, GS, LT, Levels>(views, tile_idx, lg_smem,
                                        std::make_index_sequence<sizeof...(Roots)>{},
                                        std::index_sequence<Roots...>{});
  }
};

template <class V, class LT, class Levels, class Views, std::size_t... Roots>
__global__ void __launch_bounds__(1024)
    level_graph_kernel(const Levels levels, const GridRuntime<GridSpec<LT, Levels>::rank> grid,
                       const Views views) {
  GraphKernel<V, LT, Levels, Roots...>::run(levels, grid, views);
}

}  // namespace b200
}  // namespace TensorOperations
