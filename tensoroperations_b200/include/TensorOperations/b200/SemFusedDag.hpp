// SemFusedDag.hpp -- a DagGraph with the spectral-element stiffness shape runs
// as the same fused line-owner kernel as its LevelGraph spelling
// (SemFused.cuh), calling the DAG's own combine functors, instead of being
// lowered to the generic level evaluator.
#pragma once

#include <TensorOperations/b200/Dag.hpp>
#include <TensorOperations/b200/SemFused.cuh>

namespace TensorOperations {
namespace b200 {

// An input node without a hook.
template <class A>
struct sem_plain_input : std::false_type {};
template <class T, class M>
struct sem_plain_input<NodeHandle<InputTag, T, M, NoHook>> : std::true_type {};

// ---- the same operator spelled as a DagGraph ----------------------------------
// The reference's library_sem3d (benchmarks/sem_stiffness_3d/
// bench_sem_stiffness_3d.cpp:263-472, built through include/TensorOperations/
// DagGraph.hpp:846-851): nine gradient contractions of two INPUT nodes (an
// N x N operator and a field view), integrand combines reading all nine
// gradients (one per flux direction, three outputs each, or one with nine),
// nine divergence contractions of an input operator with one integrand output,
// three combines of three divergences as the roots -- in any topological order.
// A DAG handle's as<>() renames the slot's STORAGE axes (a contraction stores
// canonical freeA ++ freeB, a combine its output order), so every slot gets a
// map from storage position to physical axis (0 the element, 1..3 the field
// views' k, j, i), propagated node by node; a combine's operands must agree on
// which physical axis each label names, and its output labels then fix the
// order in which its functor receives the coordinates.
template <class NodesT, std::size_t... Roots>
struct SemDagShape {
  static constexpr int N = 5;
  static constexpr std::size_t NK = tuple_size_v<NodesT>;
  template <std::size_t K>
  using node_t = tuple_element_t<K, NodesT>;

  template <std::size_t K>
  static constexpr std::size_t arity() {
    return static_cast<std::size_t>(output_arity<node_t<K>>());
  }
  static constexpr auto base = [] {
    std::array<std::size_t, NK + 1> b{};
    [&]<std::size_t... K>(std::index_sequence<K...>) {
      ((b[K + 1] = b[K] + arity<K>()), ...);
    }(std::make_index_sequence<NK>{});
    return b;
  }();
  static constexpr std::size_t NS = base[NK];

  struct State {
    SemTables t{};
    bool ok = true;
    int kind_of_slot[NS > 0 ? NS : 1] = {};  // 1 gradient, 2 integrand output, 3 divergence, 4 sum
    int index_of_slot[NS > 0 ? NS : 1] = {};  // member index of that kind (integrand: c*9 + o)
    int pmap[NS > 0 ? NS : 1][4] = {};
    int ng = 0, ni = 0, nd = 0, nsum = 0, nint_out = 0;
    int per_axis_g[4] = {}, per_axis_d[4] = {};
    bool used_i[3][9] = {}, used_d[9] = {};
  };
  static constexpr void fail(State& st, int why) {
    st.ok = false;
    if (!st.t.why) st.t.why = why;
  }

  // The operator input (rank 2, N x N labels whole) and its orientation.
  template <class A>
  static constexpr bool operator_input() {
    if constexpr (!sem_plain_input<A>::value)
      return false;
    else
      return A::Rank == 2;
  }

  template <std::size_t K>
  static constexpr void node(State& st) {
    using Nd = node_t<K>;
    if constexpr (dag_is_contraction_v<Nd>) {
      using A = typename Nd::node_a_type;
      using B = typename Nd::node_b_type;
      if constexpr (!operator_input<A>() || Nd::NumContracted != 1 || Nd::Rank != 4 ||
                    !std::is_same_v<typename Nd::hook_type, NoHook> || B::Rank != 4) {
        fail(st, 30);
      } else {
        constexpr auto al = to_array<typename A::modes_seq>();
        constexpr auto bl = to_array<typename B::modes_seq>();
        const int32_t c = Nd::contracted[0];
        const int pa = index_of(al, c), pb = index_of(bl, c);
        if (pa < 0 || pb < 0) {
          fail(st, 31);
          return;
        }
        int bmap[4] = {0, 1, 2, 3};  // an input field: its view dimensions are physical
        bool grad = false;
        int src_slot = -1;
        if constexpr (dag_is_input_v<B>) {
          if constexpr (!sem_plain_input<B>::value) {
            fail(st, 32);
            return;
          }
          grad = true;
        } else if constexpr (is_slot_v<B>) {
          src_slot = static_cast<int>(B::SlotIdx);
          if (src_slot >= static_cast<int>(NS) || st.kind_of_slot[src_slot] != 2) {
            fail(st, 33);
            return;
          }
          for (int d = 0; d < 4; ++d) bmap[d] = st.pmap[src_slot][d];
        } else {
          fail(st, 34);
          return;
        }
        const int ax = bmap[pb];
        if (ax < 1) {
          fail(st, 35);  // never along the element axis
          return;
        }
        const std::size_t slot = base[K];
        st.pmap[slot][0] = ax;  // storage: the operator's free label, then B's others
        for (int d = 0, w = 1; d < 4; ++d)
          if (d != pb) st.pmap[slot][w++] = bmap[d];
        if (grad) {
          const int m = st.ng++;
          if (m >= 9) {
            fail(st, 36);
            return;
          }
          const int f = st.per_axis_g[ax]++;
          if (f >= 3) {
            fail(st, 37);
            return;
          }
          st.t.g_comp[m] = f;
          st.t.g_axis[m] = ax;
          st.t.g_op[m] = m;
          st.t.g_tr[m] = pa == 0 ? 1 : 0;
          st.t.g_of[f][ax] = m;
          st.t.g_node[m] = static_cast<int>(K);
          st.kind_of_slot[slot] = 1;
          st.index_of_slot[slot] = m;
        } else {
          const int m = st.nd++;
          if (m >= 9) {
            fail(st, 38);
            return;
          }
          const int cc = st.index_of_slot[src_slot] / 9, o = st.index_of_slot[src_slot] % 9;
          if (st.used_i[cc][o]) {
            fail(st, 39);
            return;
          }
          st.used_i[cc][o] = true;
          st.t.i_out_div[cc][o] = m;
          const int sl = st.per_axis_d[ax]++;
          if (sl >= 3) {
            fail(st, 40);
            return;
          }
          st.t.d_axis[m] = ax;
          st.t.d_slot[m] = sl;
          st.t.d_at[ax][sl] = m;
          st.t.d_op[m] = 9 + m;
          st.t.d_tr[m] = pa == 0 ? 1 : 0;
          st.t.d_node[m] = static_cast<int>(K);
          st.kind_of_slot[slot] = 3;
          st.index_of_slot[slot] = m;
        }
      }
    } else if constexpr (dag_is_combine_v<Nd>) {
      if constexpr (Nd::Rank != 4) {
        fail(st, 41);
      } else {
        // the physical axis of every label the operands name
        int32_t lab[8] = {};
        int phys[8] = {};
        int nl = 0;
        int first_kind = -1;
        int idx[9] = {};
        [&]<std::size_t... P>(std::index_sequence<P...>) {
          (
              [&] {
                using Op = tuple_element_t<P, typename Nd::ops_tuple_t>;
                if constexpr (!is_slot_v<Op> || Op::Rank != 4) {
                  fail(st, 42);
                } else {
                  const int sl = static_cast<int>(Op::SlotIdx);
                  if (sl >= static_cast<int>(NS)) {
                    fail(st, 43);
                    return;
                  }
                  const int kd = st.kind_of_slot[sl];
                  if (first_kind < 0) first_kind = kd;
                  if (kd != first_kind || (kd != 1 && kd != 3)) {
                    fail(st, 44);
                    return;
                  }
                  if (P < 9) idx[P] = st.index_of_slot[sl];
                  constexpr auto ol = to_array<typename Op::modes_seq>();
                  for (int d = 0; d < 4; ++d) {
                    int found = -1;
                    for (int q = 0; q < nl; ++q)
                      if (lab[q] == ol[d]) found = q;
                    if (found < 0) {
                      lab[nl] = ol[d];
                      phys[nl++] = st.pmap[sl][d];
                    } else if (phys[found] != st.pmap[sl][d]) {
                      fail(st, 45);  // a label naming two physical axes
                    }
                  }
                }
              }(),
              ...);
        }(std::make_index_sequence<static_cast<std::size_t>(Nd::NumOps)>{});
        constexpr auto co = to_array<typename Nd::modes_seq>();
        int coord[4] = {-1, -1, -1, -1};
        bool seen[4] = {};
        for (int t = 0; t < 4; ++t) {
          for (int q = 0; q < nl; ++q)
            if (lab[q] == co[t]) coord[t] = phys[q];
          if (coord[t] < 0 || seen[coord[t]]) {
            fail(st, 46);
            return;
          }
          seen[coord[t]] = true;
        }
        if (first_kind == 1 && Nd::NumOps == 9) {  // an integrand
          const int cc = st.ni++;
          if (cc >= 3) {
            fail(st, 47);
            return;
          }
          st.t.i_nout[cc] = Nd::NumOut;
          st.nint_out += Nd::NumOut;
          for (int q = 0; q < 9; ++q) st.t.i_in[cc][q] = idx[q];
          for (int t = 0; t < 4; ++t) st.t.i_coord[cc][t] = coord[t];
          st.t.i_node[cc] = static_cast<int>(K);
          for (int o = 0; o < Nd::NumOut; ++o) {
            st.kind_of_slot[base[K] + o] = 2;
            st.index_of_slot[base[K] + o] = cc * 9 + o;
            for (int t = 0; t < 4; ++t) st.pmap[base[K] + o][t] = coord[t];
          }
        } else if (first_kind == 3 && Nd::NumOps == 3 && Nd::NumOut == 1) {  // a root sum
          const int r = st.nsum++;
          if (r >= 3) {
            fail(st, 48);
            return;
          }
          for (int q = 0; q < 3; ++q) {
            if (st.used_d[idx[q]]) fail(st, 49);
            st.used_d[idx[q]] = true;
            st.t.s_in[r][q] = idx[q];
          }
          for (int t = 0; t < 4; ++t) st.t.s_coord[r][t] = coord[t];
          constexpr std::array<std::size_t, sizeof...(Roots)> roots{Roots...};
          int pos = -1;
          for (std::size_t i = 0; i < roots.size(); ++i)
            if (roots[i] == base[K]) pos = static_cast<int>(i);
          if (pos < 0) fail(st, 50);
          st.t.s_root[r] = pos;
          st.t.s_node[r] = static_cast<int>(K);
          st.kind_of_slot[base[K]] = 4;
        } else {
          fail(st, 51);
        }
      }
    } else {
      fail(st, 52);
    }
  }

  static constexpr SemTables analyze() {
    State st{};
    if constexpr (sizeof...(Roots) != 3 || NK < 22 || NK > 24) {
      st.t.why = 29;
      return st.t;
    } else {
      [&]<std::size_t... K>(std::index_sequence<K...>) {
        (node<K>(st), ...);
      }(std::make_index_sequence<NK>{});
      if (st.ng != 9 || st.nd != 9 || st.nsum != 3 || st.nint_out != 9) fail(st, 53);
      for (int a = 1; a < 4; ++a)
        if (st.per_axis_g[a] != 3 || st.per_axis_d[a] != 3) fail(st, 54);
      for (int c = 0; c < st.ni; ++c)
        for (int o = 0; o < st.t.i_nout[c]; ++o)
          if (!st.used_i[c][o]) fail(st, 55);
      // the integrands must read every gradient exactly once (each of them)
      for (int c = 0; c < st.ni; ++c) {
        bool seen[9] = {};
        for (int q = 0; q < 9; ++q) {
          if (seen[st.t.i_in[c][q]]) fail(st, 56);
          seen[st.t.i_in[c][q]] = true;
        }
      }
      st.t.nops = 18;
      st.t.nint = st.ni;
      st.t.ok = st.ok;
      return st.t;
    }
  }

  static constexpr SemTables tables = analyze();
  static constexpr bool ok = tables.ok;
};


// Fused launch of a DagGraph: returns its league (batches of eight elements),
// or -1 when this graph / these views do not qualify (the caller then lowers
// it to the generic evaluator).  Besides the
// compile-time shape: the three gradients the shape assigns to one field read
// one view (same data, extents and strides), fields are (E, 5, 5, 5), the
// eighteen operators dense row-major 5 x 5, the roots (E, 5, 5, 5) in their
// combines' coordinate order.  Throws nothing; CUDA errors come back in *err.
template <class V, class NodesT, std::size_t... Roots, class... ViewTs>
int sem_fused_dag_launch(const NodesT& nodes, cudaError_t* err, const ViewTs&... views) {
  using Pat = SemDagShape<NodesT, Roots...>;
  *err = cudaSuccess;
  if constexpr (!Pat::ok || sizeof...(ViewTs) != 3 ||
                !(std::is_same_v<V, float> || std::is_same_v<V, double>)) {
    return -1;
  } else {
    if (!sem_fused_enabled()) return -1;
    constexpr const SemTables& T = Pat::tables;
    const auto& u0 = nodes.template get<T.g_node[T.g_of[0][1]]>().node_b.handle.tensor;
    const long long nelem = static_cast<long long>(u0.extent(0));
    bool ok = nelem > 0;
    [&]<std::size_t... C>(std::index_sequence<C...>) {
      (
          [&] {
            const auto& a = nodes.template get<T.g_node[T.g_of[C][1]]>().node_b.handle.tensor;
            const auto& b = nodes.template get<T.g_node[T.g_of[C][2]]>().node_b.handle.tensor;
            const auto& c = nodes.template get<T.g_node[T.g_of[C][3]]>().node_b.handle.tensor;
            ok = ok && a.data() == b.data() && a.data() == c.data();
            for (int d = 0; d < 4; ++d) {
              const long long want = d == 0 ? nelem : 5;
              ok = ok && static_cast<long long>(a.extent(d)) == want &&
                   static_cast<long long>(b.extent(d)) == want &&
                   static_cast<long long>(c.extent(d)) == want && a.stride(d) == b.stride(d) &&
                   a.stride(d) == c.stride(d);
            }
          }(),
          ...);
    }(std::make_index_sequence<3>{});
    SemOpPtrs<V> ops{};
    [&]<std::size_t... M>(std::index_sequence<M...>) {
      (
          [&] {
            const auto& g = nodes.template get<T.g_node[M]>().node_a.handle.tensor;
            const auto& d = nodes.template get<T.d_node[M]>().node_a.handle.tensor;
            ok = ok && sem_dense_operator<V>(g) && sem_dense_operator<V>(d);
            ops.p[M] = reinterpret_cast<const V*>(g.data());
            ops.p[9 + M] = reinterpret_cast<const V*>(d.data());
          }(),
          ...);
    }(std::make_index_sequence<9>{});
    using ViewsT = DeviceTuple<ViewTs...>;
    const ViewsT vt(views...);
    ok = ok && sem_roots_fit<Pat>(vt, nelem);
    if (!ok) return -1;
    auto field = [&]<std::size_t C>(std::integral_constant<std::size_t, C>) -> const auto& {
      return nodes.template get<T.g_node[T.g_of[C][1]]>().node_b.handle.tensor;
    };
    using FieldsT = DeviceTuple<std::decay_t<decltype(field(std::integral_constant<std::size_t, 0>{}))>,
                                std::decay_t<decltype(field(std::integral_constant<std::size_t, 1>{}))>,
                                std::decay_t<decltype(field(std::integral_constant<std::size_t, 2>{}))>>;
    const FieldsT fields(field(std::integral_constant<std::size_t, 0>{}),
                         field(std::integral_constant<std::size_t, 1>{}),
                         field(std::integral_constant<std::size_t, 2>{}));
    const auto ints = [&]<std::size_t... C>(std::index_sequence<C...>) {
      return DeviceTuple<std::decay_t<decltype(nodes.template get<T.i_node[C]>().fn)>...>(
          nodes.template get<T.i_node[C]>().fn...);
    }(std::make_index_sequence<static_cast<std::size_t>(T.nint)>{});
    const auto sums = [&]<std::size_t... R>(std::index_sequence<R...>) {
      return DeviceTuple<std::decay_t<decltype(nodes.template get<T.s_node[R]>().fn)>...>(
          nodes.template get<T.s_node[R]>().fn...);
    }(std::make_index_sequence<3>{});
    const SemFusedSource<FieldsT, std::decay_t<decltype(ints)>, std::decay_t<decltype(sums)>> src{
        fields, ints, sums};
    *err = sem_fused_run<V, Pat>(src, vt, nelem, ops, T.nops);
    return static_cast<int>((nelem + SemFusedLayout::EB - 1) / SemFusedLayout::EB);
  }
}

}  // namespace b200
}  // namespace TensorOperations
