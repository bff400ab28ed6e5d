// Graph.hpp -- LevelGraph / LevelOutputs: building a level graph, lowering its
// plan through the C ABI and launching the device evaluator.
//
// Public surface as the reference (include/TensorOperations/LevelGraph.hpp:
// make_level_graph :799-804, LevelGraph::add :685-691, outputs :693-696,
// index_consistent, scratch_bytes / slot_bytes :701-711, LevelOutputs
// team_size / scratch_bytes / slot_bytes / num_pools / execute :648-671).
// execute() returns the league size.  Errors a launch can only detect at run
// time (a whole label longer than its tile, scratch above the device limit,
// a CUDA failure) throw TensorOperations::LevelGraphError with the library's
// one-line reason.
#pragma once

#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include <tensoroperations_b200.h>

#include <TensorOperations/b200/Plan.hpp>
#if defined(__CUDACC__)
#include <TensorOperations/b200/LevelKernel.cuh>
#include <TensorOperations/b200/SemFused.cuh>
#endif

namespace TensorOperations {

template <typename ES = Kokkos::DefaultExecutionSpace>
struct TeamPolicyTag {
  using execution_space = ES;
};
template <typename ES = Kokkos::DefaultExecutionSpace>
struct TeamPolicyTag2 {
  using execution_space = ES;
};

struct LevelGraphError : std::runtime_error {
  int status;
  LevelGraphError(int st, const std::string& what) : std::runtime_error(what), status(st) {}
};

namespace b200 {

template <class LT, class M, class Tag = typename M::node_tag>
struct resolve_member {
  using type = M;
  static const M& get(const M& m) { return m; }
};
template <class LT, class M>
struct resolve_member<LT, M, StagedTag> {
  static_assert(std::is_same_v<typename M::operand_type::node_tag, InputTag>,
                "level graph: a stage member copies an input node into scratch");
  using type = NodeHandle<StagedTag, typename M::operand_type, typename M::modes_seq,
                          tile_from_labels_t<LT, typename M::modes_seq>>;
  static type get(const M& m) { return type{m.operand_}; }
};

// The handle of output O of member (L, M), typed from the member alone.
template <class V, class ES, class Levels, std::size_t L, std::size_t M, std::size_t O, class Member>
auto member_handle(const Member& m) {
  using MT = member_traits<Member>;
  constexpr std::size_t base = Algebra<Levels>::member_base(L, M);
  using Perm = array_iseq_t<MT::decl_to_storage>;
  using H = SlotNode<V, ES, base + O, typename MT::decl_labels, typename MT::tile, Perm>;
  const auto storage_shape = m.shape();
  Kokkos::Array<int, MT::rank> decl{};
  for (int d = 0; d < MT::rank; ++d) decl[d] = storage_shape[MT::decl_to_storage[d]];
  return H{decl};
}

}  // namespace b200

template <typename Graph, std::size_t... Roots>
struct LevelOutputs;

template <typename ValueType, typename ExecSpace, typename LabelTilesT, typename LevelsT>
struct LevelGraph {
  using value_type = ValueType;
  using exec_space = ExecSpace;
  using label_tiles_type = LabelTilesT;
  using levels_type = LevelsT;
  static constexpr std::size_t num_levels = tuple_size_v<LevelsT>;

  LevelsT levels;

  template <typename... Members>
  auto add(const Members&... members) const {
    static_assert(sizeof...(Members) > 0,
                  "level graph: a level must be NON-EMPTY and HOMOGENEOUS");
    using Level = DeviceTuple<typename b200::resolve_member<LabelTilesT, Members>::type...>;
    const Level level(b200::resolve_member<LabelTilesT, Members>::get(members)...);
    using NewLevels = decltype(tuple_append(levels, level));
    using G = LevelGraph<ValueType, ExecSpace, LabelTilesT, NewLevels>;
    const G g{tuple_append(levels, level)};
    return add_handles<NewLevels>(g, level, std::index_sequence_for<Members...>{});
  }

  template <typename... Handles>
  auto outputs(const Handles&...) const {
    return LevelOutputs<LevelGraph, Handles::SlotIdx...>{*this};
  }

  template <typename RootsSeq>
  std::size_t scratch_bytes() const {
    return scratch_bytes_impl(RootsSeq{});
  }
  std::size_t slot_bytes() const { return b200::Layout<ValueType, LevelsT>::unpooled_bytes; }

  // Every member's tile agrees with the grid: blocked labels carry exactly the
  // map's tile; every other label has one tile covering its whole extent.
  bool index_consistent() const {
    bool ok = true;
    for_each_member([&](const auto& m) {
      using Node = std::decay_t<decltype(m)>;
      using MT = b200::member_traits<Node>;
      constexpr auto lab = b200::to_array<typename MT::storage_labels>();
      const auto sh = m.shape();
      for (int d = 0; d < MT::rank; ++d) {
        const int tile = MT::tile::extents[d];
        if (LabelTilesT::is_gridded(lab[d])) {
          if (tile != LabelTilesT::tile(lab[d])) ok = false;
        } else if (sh[d] > tile) {
          ok = false;
        }
      }
    });
    return ok;
  }

  template <typename ES, std::size_t... Roots, typename... ViewTs>
  int launch(int team_size, const ViewTs&... views) const {
    static_assert(sizeof...(Roots) == sizeof...(ViewTs),
                  "LevelGraph::execute needs one view per designated output");
    static_assert(std::is_same_v<ES, ExecSpace>,
                  "LevelGraph::execute policy tag must match the graph's execution space");
    using Plan = LevelPlan<LevelsT>;
    static_assert(Plan::num_members > 0, "LevelGraph::execute: the graph has no members");
    using Lay = b200::Layout<ValueType, LevelsT, Roots...>;
    using GS = GridSpecOf;
    static_assert(GS::rank > 0,
                  "level graph: at least one label must be blocked (LabelTile) -- with every "
                  "label declared LabelWhole the whole problem is one team, which is a tile "
                  "map that forgot to block an axis");
    check_root_views<Roots...>(views...);

    // grid extents and whole-label checks from the staged inputs
    std::array<long long, GS::rank> gext{};
    std::array<bool, GS::rank> seen{};
    std::vector<long long> wext;
    std::vector<int> wtile;
    // one staged label: a grid extent, or a whole label that must fit its tile
    auto note_label = [&](int32_t l, long long extent, int tile) {
      const int g = GS::grid_slot(l);
      if (g < 0) {
        wext.push_back(extent);
        wtile.push_back(tile);
      } else {
        if (seen[g] && gext[g] != extent)
          throw LevelGraphError(TO_ERR_INVALID_ARGUMENT,
                                "grid: two inputs disagree on a label's extent");
        gext[g] = extent;
        seen[g] = true;
      }
    };
    for_each_member([&](const auto& m) {
      using Node = std::decay_t<decltype(m)>;
      if constexpr (b200::member_traits<Node>::kind == 0) {
        constexpr auto lab = b200::to_array<typename Node::modes_seq>();
        const auto sh = m.shape();
        for (int d = 0; d < Node::Rank; ++d) note_label(lab[d], sh[d], LabelTilesT::tile(lab[d]));
      } else if constexpr (b200::member_traits<Node>::kind == 3) {
        // the free labels of both operands; contracted labels are looped over
        using C = typename Node::contraction_type;
        auto note_operand = [&](const auto& in, auto slot_tag) {
          using In = std::decay_t<decltype(in)>;
          using SlotOp = typename decltype(slot_tag)::type;
          constexpr auto lab = b200::to_array<typename In::modes_seq>();
          const auto sh = in.shape();
          for (int d = 0; d < In::Rank; ++d)
            if (b200::index_of(C::contracted, lab[d]) < 0)
              note_label(lab[d], sh[d], SlotOp::storage_tile::extents[d]);
        };
        note_operand(m.in_a, std::type_identity<typename C::node_a_type>{});
        note_operand(m.in_b, std::type_identity<typename C::node_b_type>{});
      }
    });
    std::array<int, GS::rank> gtile{};
    for (int g = 0; g < GS::rank; ++g) gtile[g] = LabelTilesT::tile(GS::labels[g]);

    // lower the compile-time plan through the C ABI
    using Alg = b200::Algebra<LevelsT>;
    using Pool = b200::Pooling<LevelsT, Roots...>;
    constexpr std::size_t NS = Alg::num_slots;
    std::array<int32_t, num_levels> lkind{}, lmem{};
    std::array<int64_t, num_levels> lspace{};
    level_tables(lkind, lmem, lspace, std::make_index_sequence<num_levels>{});
    std::array<int32_t, NS> sdef{}, slast{}, spool{};
    std::array<int64_t, NS> sbytes{};
    for (std::size_t s = 0; s < NS; ++s) {
      sdef[s] = static_cast<int32_t>(Pool::def[s]);
      slast[s] = static_cast<int32_t>(Pool::last[s]);
      spool[s] = Pool::pool[s];
      sbytes[s] = static_cast<int64_t>(Lay::slot_bytes[s]);
    }
    std::array<int64_t, NS + 1> poff{};
    for (std::size_t q = 0; q <= Lay::num_pools; ++q) poff[q] = static_cast<int64_t>(Lay::pool_offset[q]);
    std::array<int64_t, GS::rank> gext64{};
    for (int g = 0; g < GS::rank; ++g) gext64[g] = gext[g];
    to_level_plan_desc desc{};
    desc.value_bytes = sizeof(ValueType);
    desc.num_levels = static_cast<int32_t>(num_levels);
    desc.num_slots = static_cast<int32_t>(NS);
    desc.num_pools = static_cast<int32_t>(Lay::num_pools);
    desc.level_kind = lkind.data();
    desc.level_members = lmem.data();
    desc.level_space = lspace.data();
    desc.slot_def = sdef.data();
    desc.slot_last = slast.data();
    desc.slot_pool = spool.data();
    desc.slot_bytes = sbytes.data();
    desc.pool_offset = poff.data();
    desc.grid_rank = GS::rank;
    desc.grid_extent = gext64.data();
    desc.grid_tile = gtile.data();
    desc.num_whole = static_cast<int32_t>(wext.size());
    std::vector<int64_t> wext64(wext.begin(), wext.end());
    desc.whole_extent = wext64.data();
    desc.whole_tile = wtile.data();
    desc.team_size = team_size;
#if defined(__CUDACC__)
    to_level_launch ln{};
    if (int st = to_level_plan_lower(&desc, 1, &ln)) throw LevelGraphError(st, to_last_error());
    b200::GridRuntime<GS::rank> grid{};
    for (int g = 0; g < GS::rank; ++g)
      grid.ntiles[g] = static_cast<int>((gext[g] + gtile[g] - 1) / gtile[g]);
    using Views = DeviceTuple<ViewTs...>;
    const Views vt(views...);
    if (ln.league == 0) return 0;
    // the spectral-element stiffness shape: one fused line-owner kernel that
    // calls this graph's combine functors (SemFused.cuh)
    if constexpr (GS::rank == 1) {
      cudaError_t fe = cudaSuccess;
      if (b200::sem_fused_launch<ValueType, LabelTilesT, LevelsT, Views, Roots...>(levels, vt,
                                                                                  gext[0], &fe)) {
        if (fe != cudaSuccess)
          throw LevelGraphError(TO_ERR_CUDA,
                                std::string("level graph fused launch: ") + cudaGetErrorString(fe));
        return static_cast<int>(ln.league);
      }
    }
    auto kernel = b200::level_graph_kernel<ValueType, LabelTilesT, LevelsT, Views, Roots...>;
    if (ln.scratch_bytes > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(ln.scratch_bytes));
      if (e != cudaSuccess) throw LevelGraphError(TO_ERR_CUDA, cudaGetErrorString(e));
    }
    kernel<<<static_cast<unsigned>(ln.league), ln.team, static_cast<size_t>(ln.scratch_bytes)>>>(
        levels, grid, vt);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
      throw LevelGraphError(TO_ERR_CUDA, std::string("level graph launch: ") + cudaGetErrorString(e));
    return static_cast<int>(ln.league);
#else
    to_level_launch ln{};
    if (int st = to_level_plan_lower(&desc, 0, &ln)) throw LevelGraphError(st, to_last_error());
    throw LevelGraphError(TO_ERR_UNSUPPORTED,
                          "LevelGraph::execute runs on the GPU only: compile this translation "
                          "unit with nvcc for sm_100a");
#endif
  }

  using GridSpecOf = b200::GridSpec<LabelTilesT, LevelsT>;

 private:
  template <std::size_t... R>
  static std::size_t scratch_bytes_impl(std::index_sequence<R...>) {
    return b200::Layout<ValueType, LevelsT, R...>::scratch_bytes;
  }

  template <typename NewLevels, typename G, typename Level, std::size_t... Ms>
  static auto add_handles(const G& g, const Level& level, std::index_sequence<Ms...>) {
    constexpr std::size_t L = num_levels;
    return std::tuple_cat(std::make_tuple(g),
                          member_handles<NewLevels, L, Ms>(level.template get<Ms>())...);
  }
  template <typename NewLevels, std::size_t L, std::size_t M, typename Member>
  static auto member_handles(const Member& m) {
    return [&]<std::size_t... O>(std::index_sequence<O...>) {
      return std::make_tuple(
          b200::member_handle<ValueType, ExecSpace, NewLevels, L, M, O>(m)...);
    }(std::make_index_sequence<b200::member_traits<Member>::num_out>{});
  }

  template <typename F>
  void for_each_member(F&& f) const {
    [&]<std::size_t... L>(std::index_sequence<L...>) {
      (
          [&] {
            const auto& lvl = levels.template get<L>();
            [&]<std::size_t... M>(std::index_sequence<M...>) {
              (f(lvl.template get<M>()), ...);
            }(std::make_index_sequence<tuple_size_v<tuple_element_t<L, LevelsT>>>{});
          }(),
          ...);
    }(std::make_index_sequence<num_levels>{});
  }

  template <std::size_t... L>
  static void level_tables(std::array<int32_t, num_levels>& kind,
                           std::array<int32_t, num_levels>& mem,
                           std::array<int64_t, num_levels>& space, std::index_sequence<L...>) {
    ((
         [&] {
           using Lvl = tuple_element_t<L, LevelsT>;
           using MT = b200::member_traits<tuple_element_t<0, Lvl>>;
           kind[L] = MT::kind;
           mem[L] = static_cast<int32_t>(tuple_size_v<Lvl>);
           if constexpr (MT::kind == 1 || MT::kind == 3)
             space[L] = static_cast<int64_t>(MT::sa) * MT::sb;
           else
             space[L] = MT::tile::num_elements;
         }()),
     ...);
  }

  template <std::size_t... Roots, typename... ViewTs>
  static void check_root_views(const ViewTs&...) {
    static_assert(((b200::member_traits<typename b200::slot_member_node<LevelsT, Roots>::type>::rank ==
                    static_cast<int>(ViewTs::rank)) &&
                   ...),
                  "LevelGraph::execute: each output view's rank must equal its root's rank");
  }
};

template <typename Graph, std::size_t... Roots>
struct LevelOutputs {
  Graph graph;
  int team = -1;

  LevelOutputs team_size(int n) const { return {graph, n}; }

  using roots_seq = std::index_sequence<Roots...>;

  std::size_t scratch_bytes() const {
    return b200::Layout<typename Graph::value_type, typename Graph::levels_type, Roots...>::scratch_bytes;
  }
  std::size_t slot_bytes() const { return graph.slot_bytes(); }

  static constexpr std::size_t num_pools =
      b200::Pooling<typename Graph::levels_type, Roots...>::num_pools;

  template <typename ES, typename... Ts>
  int execute(const TeamPolicyTag2<ES>&, const Ts&... views) const {
    return graph.template launch<ES, Roots...>(team, views...);
  }
};

template <typename ValueType, typename ExecSpace = Kokkos::DefaultExecutionSpace,
          typename LabelTilesT>
auto make_level_graph(LabelTilesT) {
  return LevelGraph<ValueType, ExecSpace, LabelTilesT, DeviceTuple<>>{DeviceTuple<>{}};
}

}  // namespace TensorOperations

#include <TensorOperations/b200/ImplNames.hpp>
