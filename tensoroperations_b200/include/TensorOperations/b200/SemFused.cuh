// SemFused.cuh -- a LevelGraph with the spectral-element stiffness shape runs as
// ONE fused line-owner kernel that calls the user's own combine functors,
// instead of the generic level evaluator (LevelKernel.cuh).
//
// The shape (the reference's levelgraph_sem3d, benchmarks/sem_stiffness_3d/
// bench_sem3d_levelgraph.cpp:247-351, built through include/TensorOperations/
// LevelGraph.hpp:685-691):
//   level 0  two stages of N x N operators (any labels, whole extents N)
//   level 1  three stages of rank-4 fields u_c with labels F = (fe, f1, f2, f3):
//            fe the one blocked label, f1..f3 whole labels of extent N
//   level 2  nine contractions G_m = sum_p Op(x_a, p) u_c(x with x_a -> p): one
//            operator slot, one field slot renamed along one axis a of f1..f3;
//            output declared F.  Every (field, axis) pair exactly once.
//   level 3  one combine of the nine gradients (operands labelled F) with nine
//            outputs, called at the GLOBAL coordinate (e, x1, x2, x3)
//   level 4  nine contractions of the operator slots with the combine's
//            outputs, each output read once, three along each axis
//   level 5  three combines of three level-4 slots each, the graph's roots
// Everything else keeps the generic evaluator.  The recognition is a
// compile-time walk of the level types (SemShape<...>::tables); the launch
// selects the fused kernel when `ok` holds, the value type is float or double,
// the whole labels are exactly N = 5 long and the operator views are dense
// row-major N x N.  TO_LEVELGRAPH_FUSED=0 in the environment keeps the generic
// evaluator (the tests compare the two).
//
// Kernel: a CTA takes batches of 8 elements with 200 threads; thread
// (le, a, b) is at once the column owner of element le's points (k = 0..4,
// j = a, i = b), the owner of the x3-line (k = b, j = a) and of the x2-line
// (k = a, i = b), as in the library's line-owner kernel (csrc/
// sem3d_elastic_v5.cuh): contractions along x1 run in registers, along x3 and
// x2 through two shared buffers with conflict-free strides, values updated in
// place.  The operators sit in constant memory (copied from the level-0 views
// before the launch), so every coefficient is an immediate operand.  The
// combine functors are inlined at each point with its global coordinate; the
// fields they read themselves (the reference's metric and material arrays)
// come straight from global memory with coalesced loads.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>

#include <TensorOperations/b200/Plan.hpp>

namespace TensorOperations {
namespace b200 {

// ---- the recognised shape ----------------------------------------------------

struct SemTables {
  bool ok = false;
  int why = 0;  // first failed check (0: none), for diagnosing a graph that is not recognised
  // gradient member m (level 2): field index, axis (1..3 in F), operator slot
  // (0/1 of level 0), transposed (Op(o,p) = S[p][o] instead of S[o][p])
  int g_comp[9] = {}, g_axis[9] = {}, g_op[9] = {}, g_tr[9] = {};
  int g_of[3][4] = {};  // [field][axis] -> gradient member
  int c_in[9] = {};     // combine operand q -> gradient member
  // divergence member m (level 4): combine output read, axis, operator, transposed,
  // and its position among the members of its axis (0..2)
  int d_src[9] = {}, d_axis[9] = {}, d_op[9] = {}, d_tr[9] = {}, d_slot[9] = {};
  int d_of_src[9] = {};  // combine output o -> divergence member
  int d_at[4][3] = {};   // [axis][slot] -> divergence member
  int s_in[3][3] = {};   // final combine r, operand q -> divergence member
  int s_root[3] = {};    // final combine r -> position of its slot in Roots
  // The kernel reads the tables below, which both spellings fill.  Physical
  // axes: 0 the element, 1..3 the field views' other dimensions (k, j, i).
  int nops = 0;          // operators in constant memory; gradient m uses g_op[m],
                         // divergence m uses d_op[m]
  int nint = 0;          // integrand combines (the nine gradients in, nine fluxes out)
  int i_in[3][9] = {};   // integrand c, operand q -> gradient member
  int i_nout[3] = {};    // integrand c: outputs
  int i_out_div[3][9] = {};  // integrand c, output o -> divergence member
  int i_coord[3][4] = {};    // integrand c: physical axis of its functor coordinate t
  int s_coord[3][4] = {};    // final combine r: the same for its coordinates (and root view)
  int g_node[9] = {}, i_node[3] = {}, d_node[9] = {}, s_node[3] = {};  // DAG node indices
};

template <class A>
constexpr bool identity_perm() {
  constexpr auto p = to_array_int<typename A::decl_to_storage_seq>();
  for (std::size_t d = 0; d < p.size(); ++d)
    if (p[d] != static_cast<int>(d)) return false;
  return true;
}

template <class Seq, std::size_t NF>
constexpr bool labels_equal(const std::array<int32_t, NF>& f) {
  constexpr auto s = to_array<Seq>();
  if (s.size() != NF) return false;
  for (std::size_t d = 0; d < NF; ++d)
    if (s[d] != f[d]) return false;
  return true;
}

// One contraction member of level 2 or 4: operator slot x field slot along one
// axis of the frame F, output declared F.
struct SemContraction {
  bool ok = false;
  std::size_t a_slot = 0, b_slot = 0;
  int axis = 0, tr = 0;
};

template <class C>
constexpr SemContraction sem_contraction(const std::array<int32_t, 4>& F) {
  SemContraction r{};
  if constexpr (member_traits<C>::kind != 1) {
    return r;
  } else if constexpr (C::NumContracted != 1 ||
                       !std::is_same_v<typename C::hook_type, NoHook>) {
    return r;
  } else {
    using A = typename C::node_a_type;
    using B = typename C::node_b_type;
    if constexpr (A::Rank != 2 || B::Rank != 4 || C::Rank != 4) {
      return r;
    } else {
      constexpr auto al = to_array<typename A::modes_seq>();
      constexpr auto bl = to_array<typename B::modes_seq>();
      constexpr auto out = to_array<typename C::decl_seq>();
      const int32_t c = C::contracted[0];
      const int pa = index_of(al, c);
      const int ax = index_of(bl, c);
      if (pa < 0 || ax < 1) return r;
      const int32_t fa = al[1 - pa];
      for (int q = 0; q < 4; ++q) {
        if (q == ax) {
          if (out[q] != fa) return r;
        } else if (out[q] != bl[q]) {
          return r;
        }
        if (out[q] != F[q]) return r;  // the output keeps the frame's labels
      }
      if (!identity_perm<A>() || !identity_perm<B>()) return r;
      r.a_slot = A::SlotIdx;
      r.b_slot = B::SlotIdx;
      r.axis = ax;
      r.tr = pa == 0 ? 1 : 0;
      r.ok = true;
      return r;
    }
  }
}

template <class LT, class Levels, std::size_t... Roots>
struct SemShape {
  static constexpr int N = 5;
  using Alg = Algebra<Levels>;

  template <std::size_t L, std::size_t M>
  using mem_t = tuple_element_t<M, tuple_element_t<L, Levels>>;

  static constexpr bool level_sizes() {
    if constexpr (tuple_size_v<Levels> != 6) {
      return false;
    } else {
      constexpr std::array<std::size_t, 6> want{2, 3, 9, 1, 9, 3};
      constexpr std::array<int, 6> kind{0, 0, 1, 2, 1, 2};
      for (std::size_t l = 0; l < 6; ++l)
        if (Alg::member_counts[l] != want[l]) return false;
      bool k = true;
      [&]<std::size_t... L>(std::index_sequence<L...>) {
        ((k = k && member_traits<mem_t<L, 0>>::kind == kind[L]), ...);
      }(std::make_index_sequence<6>{});
      return k && sizeof...(Roots) == 3;
    }
  }

  using Frame = std::array<int32_t, 4>;
  static constexpr void fail(SemTables& t, bool& ok, int why) {
    ok = false;
    if (!t.why) t.why = why;
  }

  template <std::size_t M>
  static constexpr void op_stage(SemTables& t, bool& ok) {
    using S = mem_t<0, M>;
    if constexpr (S::Rank != 2) {
      fail(t, ok, 2);
    } else {
      constexpr auto l = to_array<typename S::modes_seq>();
      for (int d = 0; d < 2; ++d)
        if (LT::is_gridded(l[d]) || LT::tile(l[d]) != N) fail(t, ok, 3);
    }
  }

  template <std::size_t M>
  static constexpr void field_stage(SemTables& t, bool& ok, const Frame& F) {
    if (!labels_equal<typename mem_t<1, M>::modes_seq>(F)) fail(t, ok, 4);
  }

  template <std::size_t M>
  static constexpr void gradient(SemTables& t, bool& ok, const Frame& F, bool (&seen)[3][4]) {
    const std::size_t op0 = Alg::member_base(0, 0), op1 = Alg::member_base(0, 1);
    const std::size_t u0 = Alg::member_base(1, 0);
    const SemContraction c = sem_contraction<mem_t<2, M>>(F);
    if (!c.ok || (c.a_slot != op0 && c.a_slot != op1) || c.b_slot < u0 || c.b_slot >= u0 + 3) {
      fail(t, ok, 5);
      return;
    }
    const int comp = static_cast<int>(c.b_slot - u0);
    t.g_comp[M] = comp;
    t.g_axis[M] = c.axis;
    t.g_op[M] = c.a_slot == op0 ? 0 : 1;
    t.g_tr[M] = c.tr;
    if (seen[comp][c.axis]) fail(t, ok, 6);
    seen[comp][c.axis] = true;
    t.g_of[comp][c.axis] = static_cast<int>(M);
  }

  template <std::size_t Q>
  static constexpr void combine_operand(SemTables& t, bool& ok, const Frame& F, bool (&used)[9]) {
    using Op = tuple_element_t<Q, typename mem_t<3, 0>::ops_tuple_t>;
    if (!labels_equal<typename Op::modes_seq>(F)) fail(t, ok, 9);
    const std::size_t g0 = Alg::member_base(2, 0);
    const std::size_t slot = Op::SlotIdx;
    if (slot < g0 || slot >= g0 + 9 || used[slot - g0]) {
      fail(t, ok, 10);
      return;
    }
    used[slot - g0] = true;
    t.c_in[Q] = static_cast<int>(slot - g0);
  }

  template <std::size_t M>
  static constexpr void divergence(SemTables& t, bool& ok, const Frame& F, bool (&used)[9],
                                   int (&per_axis)[4]) {
    const std::size_t op0 = Alg::member_base(0, 0), op1 = Alg::member_base(0, 1);
    const std::size_t f0 = Alg::member_base(3, 0);
    const SemContraction c = sem_contraction<mem_t<4, M>>(F);
    if (!c.ok || (c.a_slot != op0 && c.a_slot != op1) || c.b_slot < f0 || c.b_slot >= f0 + 9 ||
        used[c.b_slot - f0]) {
      fail(t, ok, 11);
      return;
    }
    const int src = static_cast<int>(c.b_slot - f0);
    used[src] = true;
    t.d_src[M] = src;
    t.d_axis[M] = c.axis;
    t.d_op[M] = c.a_slot == op0 ? 0 : 1;
    t.d_tr[M] = c.tr;
    if (per_axis[c.axis] >= 3) {
      fail(t, ok, 12);
      return;
    }
    t.d_slot[M] = per_axis[c.axis];
    t.d_at[c.axis][per_axis[c.axis]] = static_cast<int>(M);
    ++per_axis[c.axis];
    t.d_of_src[src] = static_cast<int>(M);
  }

  template <std::size_t R, std::size_t Q>
  static constexpr void sum_operand(SemTables& t, bool& ok, const Frame& F, bool (&used)[9]) {
    using Op = tuple_element_t<Q, typename mem_t<5, R>::ops_tuple_t>;
    if (!labels_equal<typename Op::modes_seq>(F)) fail(t, ok, 15);
    const std::size_t d0 = Alg::member_base(4, 0);
    const std::size_t slot = Op::SlotIdx;
    if (slot < d0 || slot >= d0 + 9 || used[slot - d0]) {
      fail(t, ok, 16);
      return;
    }
    used[slot - d0] = true;
    t.s_in[R][Q] = static_cast<int>(slot - d0);
  }

  template <std::size_t R>
  static constexpr void sum_member(SemTables& t, bool& ok, const Frame& F, bool (&used)[9]) {
    using S = mem_t<5, R>;
    if constexpr (S::NumOps != 3 || S::NumOut != 1 || S::Rank != 4) {
      fail(t, ok, 13);
    } else {
      if (!labels_equal<typename S::modes_seq>(F)) fail(t, ok, 14);
      sum_operand<R, 0>(t, ok, F, used);
      sum_operand<R, 1>(t, ok, F, used);
      sum_operand<R, 2>(t, ok, F, used);
      constexpr std::array<std::size_t, sizeof...(Roots)> roots{Roots...};
      const std::size_t slot = Alg::member_base(5, R);
      int pos = -1;
      for (std::size_t i = 0; i < roots.size(); ++i)
        if (roots[i] == slot) pos = static_cast<int>(i);
      if (pos < 0) fail(t, ok, 17);
      t.s_root[R] = pos;
    }
  }

  template <std::size_t... I>
  static constexpr void walk(SemTables& t, bool& ok, const Frame& F, std::index_sequence<I...>) {
    op_stage<0>(t, ok);
    op_stage<1>(t, ok);
    field_stage<0>(t, ok, F);
    field_stage<1>(t, ok, F);
    field_stage<2>(t, ok, F);
    bool seen[3][4] = {};
    (gradient<I>(t, ok, F, seen), ...);
    using Cb = mem_t<3, 0>;
    if constexpr (Cb::NumOps != 9 || Cb::NumOut != 9 || Cb::Rank != 4) {
      fail(t, ok, 7);
    } else {
      if (!labels_equal<typename Cb::modes_seq>(F)) fail(t, ok, 8);
      bool used[9] = {};
      (combine_operand<I>(t, ok, F, used), ...);
    }
    bool used_f[9] = {};
    int per_axis[4] = {};
    (divergence<I>(t, ok, F, used_f, per_axis), ...);
    bool used_d[9] = {};
    sum_member<0>(t, ok, F, used_d);
    sum_member<1>(t, ok, F, used_d);
    sum_member<2>(t, ok, F, used_d);
    for (int a = 1; a < 4; ++a)
      if (per_axis[a] != 3) fail(t, ok, 18);
  }

  static constexpr SemTables analyze() {
    SemTables t{};
    if constexpr (!level_sizes()) {
      t.why = 1;
      return t;
    } else {
      using U0 = mem_t<1, 0>;  // the frame: the first field stage's labels
      if constexpr (U0::Rank != 4) {
        t.why = 1;
        return t;
      } else {
        constexpr auto Fa = to_array<typename U0::modes_seq>();
        const Frame F{Fa[0], Fa[1], Fa[2], Fa[3]};
        bool ok = LT::is_gridded(F[0]);
        if (!ok) t.why = 100;
        for (int d = 1; d < 4; ++d)
          if (LT::is_gridded(F[d]) || LT::tile(F[d]) != N) fail(t, ok, 100);
        walk(t, ok, F, std::make_index_sequence<9>{});
        t.nops = 2;
        t.nint = 1;
        t.i_nout[0] = 9;
        for (int q = 0; q < 9; ++q) {
          t.i_in[0][q] = t.c_in[q];
          t.i_out_div[0][q] = t.d_of_src[q];
        }
        for (int d = 0; d < 4; ++d) {
          t.i_coord[0][d] = d;
          for (int r = 0; r < 3; ++r) t.s_coord[r][d] = d;
        }
        t.ok = ok;
        return t;
      }
    }
  }

  static constexpr SemTables tables = analyze();
  static constexpr bool ok = tables.ok;
};

// ---- the kernel ----------------------------------------------------------------

// The operators of the running launch, [op][o][p], row-major: two for a
// LevelGraph (its level-0 stages), eighteen for a DagGraph (gradient m uses
// operator m, divergence m operator 9 + m).  Per translation unit; gathered by
// sem_fused_gather_ops into the staging array and copied here by the launch,
// stream-ordered before the kernel.
inline constexpr int kSemFusedMaxOps = 18;
static __constant__ float sem_fused_ops_f32[kSemFusedMaxOps][5][5];
static __constant__ double sem_fused_ops_f64[kSemFusedMaxOps][5][5];
static __device__ float sem_fused_stage_f32[kSemFusedMaxOps * 25];
static __device__ double sem_fused_stage_f64[kSemFusedMaxOps * 25];

template <class V>
struct SemOpPtrs {
  const V* p[kSemFusedMaxOps];
};

template <class V>
__global__ void sem_fused_gather_ops(const SemOpPtrs<V> ops, int nops) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= nops * 25) return;
  if constexpr (std::is_same_v<V, float>)
    sem_fused_stage_f32[t] = ops.p[t / 25][t % 25];
  else
    sem_fused_stage_f64[t] = ops.p[t / 25][t % 25];
}

// What the kernel reads besides the operators: the three field views (indexed
// by the physical axes element, k, j, i), the integrand combine functors and
// the three root combine functors -- copied out of the graph so the kernel's
// parameters hold nothing else.
template <class Fields, class Ints, class Sums>
struct SemFusedSource {
  Fields fields;
  Ints ints;
  Sums sums;
};

// Coefficient Op(o, p) of operator OP, transposed when TR: every index is a
// compile-time constant once the loops are unrolled, so it is an immediate
// constant-bank operand.
template <class V, int OP, int TR>
__device__ __forceinline__ V sem_op(int o, int p) {
  if constexpr (std::is_same_v<V, float>)
    return TR ? sem_fused_ops_f32[OP][p][o] : sem_fused_ops_f32[OP][o][p];
  else
    return TR ? sem_fused_ops_f64[OP][p][o] : sem_fused_ops_f64[OP][o][p];
}

struct SemFusedLayout {
  static constexpr int N = 5, NN = 25, EB = 8, NT = EB * NN;
  static constexpr int SKX = NT + 25, SKE = NT + 29;  // conflict-free k-strides (32-bit words)
  static constexpr int CX = N * SKX, CE = N * SKE;
  template <class V>
  static constexpr std::size_t bytes() {
    return sizeof(V) * (3 * CX + 3 * CE);
  }
};

// out[o] = sum_p Op(o, p) in[p] for o, p < 5.
template <class V, int OP, int TR>
__device__ __forceinline__ void sem_line(const V* in, V* out) {
#pragma unroll
  for (int o = 0; o < 5; ++o) {
    V s = V(0);
#pragma unroll
    for (int p = 0; p < 5; ++p) s = fma(sem_op<V, OP, TR>(o, p), in[p], s);
    out[o] = s;
  }
}

// Every table lookup below happens at compile time (static_for indices and
// constexpr locals); a run-time index into the tables would put them in local
// memory.
#ifndef TO_SEM_FUSED_ZBUF
#define TO_SEM_FUSED_ZBUF 1
#endif
// Resident CTAs per SM the kernel is compiled for (its register budget): one
// integrand (56 registers, a few bytes of spills) 5 -- 1.788 vs 1.816 ms for the
// reference's LevelGraph program at E=786,432 --, three integrands (113
// registers; 80 at 3 CTAs spill 164 bytes) 2.  TO_SEM_FUSED_MIN_BLOCKS
// overrides both.
#ifdef TO_SEM_FUSED_MIN_BLOCKS
template <class Pat>
constexpr int sem_fused_min_blocks() {
  return TO_SEM_FUSED_MIN_BLOCKS;
}
#else
template <class Pat>
constexpr int sem_fused_min_blocks() {
  return Pat::tables.nint == 1 ? 5 : (TO_SEM_FUSED_ZBUF ? 3 : 2);
}
#endif
// Several integrands: the column's x1 gradients and fluxes live in a third
// shared buffer Z ([3][N][NT], the column owner's own words) instead of 30
// registers, so the kernel fits 3 CTAs per SM at 80 registers without spills
// (the reference's DagGraph program 2.979 vs 3.079 ms with them in registers
// and the fields read ahead).  TO_SEM_FUSED_ZBUF=0 keeps them in registers.
// One integrand keeps them in registers: with the buffer the reference's
// LevelGraph program took 2.79 ms instead of 1.79 ms.
template <class Pat>
constexpr bool sem_fused_zbuf() {
  return TO_SEM_FUSED_ZBUF != 0 && Pat::tables.nint > 1;
}
// Whether the kernel reads the next batch's fields ahead: on for several
// integrands with x1 data in registers (128 registers, no spills; the
// reference's DagGraph program 3.08 vs 3.11 ms), off with the Z buffer (it
// would spill at 80 registers) and for one integrand (it would spill 40 bytes
// at 56).
// TO_SEM_FUSED_U_PIPE = 0 / 1 forces it off / on for every spelling.
#ifdef TO_SEM_FUSED_U_PIPE
template <class Pat>
constexpr bool sem_fused_u_pipe() {
  return TO_SEM_FUSED_U_PIPE != 0;
}
#else
template <class Pat>
constexpr bool sem_fused_u_pipe() {
  return Pat::tables.nint > 1 && !sem_fused_zbuf<Pat>();
}
#endif
// Points per group of functor calls in phase B2.
#ifndef TO_SEM_FUSED_B2_GROUP
#define TO_SEM_FUSED_B2_GROUP 1
#endif

// Integrand combine C at one point: its coordinates in its own label order,
// its nine gradient operands in its own operand order.
template <class Pat, int C, class Fn, class V, std::size_t... Q>
__device__ __forceinline__ auto sem_call_integrand(const Fn& fn, const int (&P)[4], const V (&g)[9],
                                                   std::index_sequence<Q...>) {
  constexpr int c0 = Pat::tables.i_coord[C][0], c1 = Pat::tables.i_coord[C][1];
  constexpr int c2 = Pat::tables.i_coord[C][2], c3 = Pat::tables.i_coord[C][3];
  constexpr int q[9] = {Pat::tables.i_in[C][Q]...};
  return fn(P[c0], P[c1], P[c2], P[c3], g[q[Q]]...);
}

template <class V, class Pat, class Src, class Views>
__global__ void __launch_bounds__(SemFusedLayout::NT, sem_fused_min_blocks<Pat>())
    sem_fused_kernel(const Src src, const Views views, long long nelem) {
  using LY = SemFusedLayout;
  constexpr int N = LY::N, NN = LY::NN, EB = LY::EB, NT = LY::NT;
  constexpr int SKX = LY::SKX, SKE = LY::SKE, CX = LY::CX, CE = LY::CE;
  extern __shared__ __align__(16) unsigned char sem_smem[];
  V* X = reinterpret_cast<V*>(sem_smem);  // [3][N][SKX]: rows along x3 (i)
  V* E = X + 3 * CX;                      // [3][N][SKE]: rows along x2 (j)
  constexpr bool kZ = sem_fused_zbuf<Pat>();
  V* Z = E + 3 * CE;                      // kZ: [3][N][NT], x1 data of the columns

  const int tid = threadIdx.x;
  const int le = tid / NN;
  const int ab = tid - le * NN;
  const int ra = ab / N;        // column j / x3-line j / x2-line k
  const int rb = ab - ra * N;   // column i / x3-line k / x2-line i
  const int lx = rb * SKX + le * NN + ra * N;  // x3-line (k = rb, j = ra): + i
  const int ly = ra * SKE + le * NN + rb;      // x2-line (k = ra, i = rb): + N j

  // kUPipe: the next batch's column of the three fields is read during C1 and
  // C2 of this one, so phase A waits on no global load
  constexpr bool kUPipe = sem_fused_u_pipe<Pat>();
  V un[kUPipe ? 3 : 1][kUPipe ? N : 1];
  auto load_u = [&](long long bb) {
    if constexpr (kUPipe) {
      const long long en = bb * EB + le;
      const bool vn = en < nelem;
      const int eni = vn ? static_cast<int>(en) : 0;
      static_for<3>([&](auto cc) {
        constexpr int c = decltype(cc)::value;
        const auto& u = src.fields.template get<c>();
#pragma unroll
        for (int k = 0; k < N; ++k) un[c][k] = vn ? static_cast<V>(u(eni, k, ra, rb)) : V(0);
      });
    }
  };
  load_u(blockIdx.x);
  for (long long b = blockIdx.x; b * EB < nelem; b += gridDim.x) {
    const long long e = b * EB + le;
    const bool valid = e < nelem;
    const int ei = valid ? static_cast<int>(e) : 0;

    // ---- A: the column's fields -> X, E; gradients along x1 in registers ----
    V dg[kZ ? 1 : 3][kZ ? 1 : N];
    static_for<3>([&](auto cc) {
      constexpr int c = decltype(cc)::value;
      const auto& u = src.fields.template get<c>();
      V uc[N];
#pragma unroll
      for (int k = 0; k < N; ++k) {
        if constexpr (kUPipe)
          uc[k] = un[c][k];
        else
          uc[k] = valid ? static_cast<V>(u(ei, k, ra, rb)) : V(0);
      }
#pragma unroll
      for (int k = 0; k < N; ++k) {
        X[c * CX + k * SKX + tid] = uc[k];
        E[c * CE + k * SKE + tid] = uc[k];
      }
      constexpr int m = Pat::tables.g_of[c][1];
      if constexpr (kZ) {
        V gl[N];
        sem_line<V, Pat::tables.g_op[m], Pat::tables.g_tr[m]>(uc, gl);
#pragma unroll
        for (int k = 0; k < N; ++k) Z[(c * N + k) * NT + tid] = gl[k];
      } else {
        sem_line<V, Pat::tables.g_op[m], Pat::tables.g_tr[m]>(uc, dg[c]);
      }
    });
    __syncthreads();

    // ---- B1: gradients along x3 (X rows) and x2 (E rows), in place ----
    static_for<3>([&](auto cc) {
      constexpr int c = decltype(cc)::value;
      constexpr int mx = Pat::tables.g_of[c][3], me = Pat::tables.g_of[c][2];
      V v[N], w[N], ov[N], ow[N];
#pragma unroll
      for (int p = 0; p < N; ++p) {
        v[p] = X[c * CX + lx + p];
        w[p] = E[c * CE + ly + p * N];
      }
      sem_line<V, Pat::tables.g_op[mx], Pat::tables.g_tr[mx]>(v, ov);
      sem_line<V, Pat::tables.g_op[me], Pat::tables.g_tr[me]>(w, ow);
#pragma unroll
      for (int o = 0; o < N; ++o) {
        X[c * CX + lx + o] = ov[o];
        E[c * CE + ly + o * N] = ow[o];
      }
    });
    __syncthreads();

    // ---- B2: the integrand combines at every point of the column ----
    // All nine gradients of a point are read before any flux is stored (the
    // fluxes go to the same places, and every integrand reads all nine).
    // Points go in groups of TO_SEM_FUSED_B2_GROUP: every functor call of the
    // group is made before any flux is stored, so the functors' own global
    // loads (through generic pointers, which the compiler may not move across
    // a shared-memory store) of the whole group are in flight together.
    V Fg[kZ ? 1 : 3][kZ ? 1 : N];
    constexpr int KG = TO_SEM_FUSED_B2_GROUP;
    static_for<(N + KG - 1) / KG>([&](auto gg) {
      constexpr int k0 = decltype(gg)::value * KG;
      constexpr int nk = (N - k0 < KG) ? (N - k0) : KG;
      V F[nk][9];  // [point][divergence member]
      // flux of divergence member md at point k -> its slot
      auto store_flux = [&](auto mdc, auto kc, V value) {
        constexpr int md = decltype(mdc)::value, k = decltype(kc)::value;
        constexpr int ax = Pat::tables.d_axis[md], sl = Pat::tables.d_slot[md];
        if constexpr (ax == 3)
          X[sl * CX + k * SKX + tid] = value;
        else if constexpr (ax == 2)
          E[sl * CE + k * SKE + tid] = value;
        else if constexpr (kZ)
          Z[(sl * N + k) * NT + tid] = value;
        else
          Fg[sl][k] = value;
      };
      static_for<nk>([&](auto kk) {
        constexpr int k = k0 + decltype(kk)::value;
        V g[9];  // [gradient member]
        static_for<9>([&](auto mm) {
          constexpr int m = decltype(mm)::value;
          constexpr int comp = Pat::tables.g_comp[m], ax = Pat::tables.g_axis[m];
          if constexpr (ax == 3)
            g[m] = X[comp * CX + k * SKX + tid];
          else if constexpr (ax == 2)
            g[m] = E[comp * CE + k * SKE + tid];
          else
            g[m] = kZ ? Z[(comp * N + k) * NT + tid] : dg[kZ ? 0 : comp][kZ ? 0 : k];
        });
        const int P[4] = {ei, k, ra, rb};
        static_for<Pat::tables.nint>([&](auto ci) {
          constexpr int c = decltype(ci)::value;
          constexpr int nout = Pat::tables.i_nout[c];
          if (valid) {
            const auto r = sem_call_integrand<Pat, c>(src.ints.template get<c>(), P, g,
                                                      std::make_index_sequence<9>{});
            static_for<nout>([&](auto oo) {
              constexpr int o = decltype(oo)::value;
              constexpr int md = Pat::tables.i_out_div[c][o];
              F[decltype(kk)::value][md] = static_cast<V>(r[o]);
            });
          } else {
            static_for<nout>([&](auto oo) {
              constexpr int o = decltype(oo)::value;
              constexpr int md = Pat::tables.i_out_div[c][o];
              F[decltype(kk)::value][md] = V(0);
            });
          }
        });
      });
      static_for<nk>([&](auto kk) {
        constexpr int k = k0 + decltype(kk)::value;
        static_for<9>([&](auto mm) {
          store_flux(mm, std::integral_constant<int, k>{}, F[decltype(kk)::value][decltype(mm)::value]);
        });
      });
    });
    __syncthreads();

    load_u(b + gridDim.x);  // in flight during C1 and C2

    // ---- C1: divergences along x3 and x2, in place ----
    static_for<3>([&](auto ss) {
      constexpr int sl = decltype(ss)::value;
      constexpr int mx = Pat::tables.d_at[3][sl], me = Pat::tables.d_at[2][sl];
      V v[N], w[N], ov[N], ow[N];
#pragma unroll
      for (int q = 0; q < N; ++q) {
        v[q] = X[sl * CX + lx + q];
        w[q] = E[sl * CE + ly + q * N];
      }
      sem_line<V, Pat::tables.d_op[mx], Pat::tables.d_tr[mx]>(v, ov);
      sem_line<V, Pat::tables.d_op[me], Pat::tables.d_tr[me]>(w, ow);
#pragma unroll
      for (int o = 0; o < N; ++o) {
        X[sl * CX + lx + o] = ov[o];
        E[sl * CE + ly + o * N] = ow[o];
      }
    });
    __syncthreads();

    // ---- C2: divergences along x1, the three root combines, the roots ----
    V tgc[3][N];
    static_for<3>([&](auto ss) {
      constexpr int sl = decltype(ss)::value;
      constexpr int m = Pat::tables.d_at[1][sl];
      if constexpr (kZ) {
        V fz[N];
#pragma unroll
        for (int q = 0; q < N; ++q) fz[q] = Z[(sl * N + q) * NT + tid];
        sem_line<V, Pat::tables.d_op[m], Pat::tables.d_tr[m]>(fz, tgc[sl]);
      } else {
        sem_line<V, Pat::tables.d_op[m], Pat::tables.d_tr[m]>(Fg[sl], tgc[sl]);
      }
    });
#pragma unroll
    for (int k = 0; k < N; ++k) {
      const int P[4] = {ei, k, ra, rb};
      static_for<3>([&](auto rr) {
        constexpr int R = decltype(rr)::value;
        constexpr int s0 = Pat::tables.s_coord[R][0], s1 = Pat::tables.s_coord[R][1];
        constexpr int s2 = Pat::tables.s_coord[R][2], s3 = Pat::tables.s_coord[R][3];
        V t3[3];
        static_for<3>([&](auto qq) {
          constexpr int q = decltype(qq)::value;
          constexpr int md = Pat::tables.s_in[R][q];
          constexpr int ax = Pat::tables.d_axis[md], sl = Pat::tables.d_slot[md];
          if constexpr (ax == 3)
            t3[q] = X[sl * CX + k * SKX + tid];
          else if constexpr (ax == 2)
            t3[q] = E[sl * CE + k * SKE + tid];
          else
            t3[q] = tgc[sl][k];
        });
        if (valid) {
          const V r = static_cast<V>(
              src.sums.template get<R>()(P[s0], P[s1], P[s2], P[s3], t3[0], t3[1], t3[2]));
          views.template get<Pat::tables.s_root[R]>()(P[s0], P[s1], P[s2], P[s3]) = r;
        }
      });
    }
    __syncthreads();  // the next batch overwrites X and E
  }
}

// Fused launches made by this process (the tests check which route ran).
inline long long& sem_fused_launch_count() {
  static long long n = 0;
  return n;
}

// The launch both spellings share, once the graph and its views qualify:
// gathers the operators into constant memory and launches the fused kernel on
// the legacy default stream, one CTA per batch up to the resident limit.
// Returns the CUDA status.
template <class V, class Pat, class Src, class Views>
cudaError_t sem_fused_run(const Src& src, const Views& views, long long nelem,
                          const SemOpPtrs<V>& ops, int nops) {
  using LY = SemFusedLayout;
  constexpr std::size_t smem =
      LY::bytes<V>() + (sem_fused_zbuf<Pat>() ? sizeof(V) * 3 * LY::N * LY::NT : 0);
  auto kernel = sem_fused_kernel<V, Pat, Src, Views>;
  int dev = 0, sms = 0, nb = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return err;
  if (smem > 48 * 1024 &&
      (err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem))) != cudaSuccess)
    return err;
  if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, LY::NT, smem)) != cudaSuccess)
    return err;
  sem_fused_gather_ops<V><<<(nops * 25 + 127) / 128, 128, 0, 0>>>(ops, nops);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  void* stage = nullptr;
  if constexpr (std::is_same_v<V, float>) {
    if ((err = cudaGetSymbolAddress(&stage, sem_fused_stage_f32)) != cudaSuccess) return err;
    err = cudaMemcpyToSymbolAsync(sem_fused_ops_f32, stage, nops * 25 * sizeof(V), 0,
                                  cudaMemcpyDeviceToDevice, 0);
  } else {
    if ((err = cudaGetSymbolAddress(&stage, sem_fused_stage_f64)) != cudaSuccess) return err;
    err = cudaMemcpyToSymbolAsync(sem_fused_ops_f64, stage, nops * 25 * sizeof(V), 0,
                                  cudaMemcpyDeviceToDevice, 0);
  }
  if (err != cudaSuccess) return err;
  const long long nbatch = (nelem + LY::EB - 1) / LY::EB;
  const long long cap = static_cast<long long>(sms) * (nb > 0 ? nb : 1);
  const int grid = static_cast<int>(nbatch < cap ? nbatch : cap);
  kernel<<<grid, LY::NT, smem, 0>>>(src, views, nelem);
  err = cudaGetLastError();
  if (err == cudaSuccess) ++sem_fused_launch_count();
  return err;
}

inline bool sem_fused_enabled() {
  static const bool enabled = [] {
    const char* e = std::getenv("TO_LEVELGRAPH_FUSED");
    return !(e && std::strcmp(e, "0") == 0);
  }();
  return enabled;
}

// A dense row-major 5 x 5 view of V (its data is copied into the constant bank
// as V, so another element type keeps the generic evaluator, which converts).
template <class V, class H>
bool sem_dense_operator(const H& h) {
  if constexpr (!std::is_same_v<typename value_of<H>::type, V>)
    return false;
  else
    return h.extent(0) == 5 && h.extent(1) == 5 && h.stride(0) == 5 && h.stride(1) == 1;
}

// Root view R of extents (nelem, 5, 5, 5) in physical order, permuted by the
// root combine's coordinate order sc.
template <class F>
bool sem_root_extents(const F& f, const int (&sc)[4], long long nelem) {
  bool ok = true;
  for (int t = 0; t < 4; ++t) {
    const long long want = sc[t] == 0 ? nelem : 5;
    ok = ok && static_cast<long long>(f.extent(t)) == want;
  }
  return ok;
}

// Every root view: root combine r writes view s_root[r] in its own coordinate order.
template <class Pat, class Views>
bool sem_roots_fit(const Views& views, long long nelem) {
  return [&]<std::size_t... R>(std::index_sequence<R...>) {
    return (sem_root_extents(views.template get<Pat::tables.s_root[R]>(), Pat::tables.s_coord[R], nelem) &&
            ...);
  }(std::make_index_sequence<3>{});
}

// Fused launch of a LevelGraph, or false when this graph / these views do not
// qualify (the caller then runs the generic evaluator).  Throws nothing; CUDA
// errors come back as the status in *err.
template <class V, class LT, class Levels, class Views, std::size_t... Roots>
bool sem_fused_launch(const Levels& levels, const Views& views, long long nelem, cudaError_t* err) {
  using Pat = SemShape<LT, Levels, Roots...>;
  *err = cudaSuccess;
  if constexpr (!Pat::ok || !(std::is_same_v<V, float> || std::is_same_v<V, double>)) {
    return false;
  } else {
    if (!sem_fused_enabled()) return false;
    // every field and root: whole labels exactly 5; operators dense row-major 5 x 5
    bool shapes = true;
    const auto& lv1 = levels.template get<1>();
    [&]<std::size_t... C>(std::index_sequence<C...>) {
      (
          [&] {
            const auto& u = lv1.template get<C>().operand_.handle.tensor;
            shapes = shapes && static_cast<long long>(u.extent(0)) == nelem;
            for (int d = 1; d < 4; ++d) shapes = shapes && u.extent(d) == 5;
          }(),
          ...);
    }(std::make_index_sequence<3>{});
    shapes = shapes && sem_roots_fit<Pat>(views, nelem);
    SemOpPtrs<V> ops{};
    [&]<std::size_t... S>(std::index_sequence<S...>) {
      (
          [&] {
            const auto& h = levels.template get<0>().template get<S>().operand_.handle.tensor;
            shapes = shapes && sem_dense_operator<V>(h);
            ops.p[S] = reinterpret_cast<const V*>(h.data());
          }(),
          ...);
    }(std::make_index_sequence<2>{});
    if (!shapes || nelem <= 0) return false;
    const auto& lv3 = levels.template get<3>();
    const auto& lv5 = levels.template get<5>();
    using FieldsT = DeviceTuple<std::decay_t<decltype(lv1.template get<0>().operand_.handle.tensor)>,
                                std::decay_t<decltype(lv1.template get<1>().operand_.handle.tensor)>,
                                std::decay_t<decltype(lv1.template get<2>().operand_.handle.tensor)>>;
    using IntsT = DeviceTuple<std::decay_t<decltype(lv3.template get<0>().fn)>>;
    using SumsT = DeviceTuple<std::decay_t<decltype(lv5.template get<0>().fn)>,
                              std::decay_t<decltype(lv5.template get<1>().fn)>,
                              std::decay_t<decltype(lv5.template get<2>().fn)>>;
    const SemFusedSource<FieldsT, IntsT, SumsT> src{
        FieldsT(lv1.template get<0>().operand_.handle.tensor, lv1.template get<1>().operand_.handle.tensor,
                lv1.template get<2>().operand_.handle.tensor),
        IntsT(lv3.template get<0>().fn),
        SumsT(lv5.template get<0>().fn, lv5.template get<1>().fn, lv5.template get<2>().fn)};
    *err = sem_fused_run<V, Pat>(src, views, nelem, ops, Pat::tables.nops);
    return true;
  }
}

}  // namespace b200
}  // namespace TensorOperations
