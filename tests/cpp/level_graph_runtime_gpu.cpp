// level_graph_runtime_gpu.cpp -- LevelGraph runtime scenarios on the GPU.
//
// Each scenario builds a small graph through the public API, runs it with
// execute(TeamPolicyTag2<ES>{}, ...) and compares every output element with a
// host loop in double precision (max abs error < 1e-4, or 1e-3 where the
// values include coordinate terms of order 1e3).  The scenarios are the ones
// the reference pins in tests/test_level_graph.cpp:330-778: a single
// contraction, a fused three-member gradient level relabelling one staged
// operand, a combine over a contraction, a two-output combine, a contraction
// rooted in a non-canonical declared order, a combine reading that slot in a
// third order, a contraction reading a declared-order slot, and a combine fn
// receiving GLOBAL coordinates.  Extents are pairwise distinct and the
// permutations are 3-cycles so a transposed index cannot pass.
#include <Kokkos_Core.hpp>
#include <TensorOperations/LevelGraph.hpp>

#include <cmath>
#include <cstdio>

using namespace TensorOperations;
using ES = Kokkos::DefaultExecutionSpace;
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;
using V4 = Kokkos::View<float****, Kokkos::LayoutRight>;

static int g_fail = 0;
static void report(const char* name, double err, double tol) {
  const bool ok = err < tol;
  if (!ok) ++g_fail;
  std::printf("%-44s max err %.3e  %s\n", name, err, ok ? "PASS" : "FAIL");
  std::fflush(stdout);
}

// ---- fills (closed form, distinct per tensor) ----
static float hv(int q, int a) { return 0.25f + 0.13f * q - 0.21f * a + 0.03f * q * a; }
static float wv(int p, int q) { return 0.55f - 0.09f * p + 0.17f * q; }
static float uv(int e, int a, int b, int c) {
  return 0.6f - 0.11f * e + 0.08f * a - 0.06f * b + 0.19f * c + 0.015f * (e + b) * (c + 1);
}

template <int Q, int A, int B, int C, int E>
struct Data {
  V2 H{"H", Q, A};
  V4 U{"U", E, A, B, C};
  Data() {
    auto h = Kokkos::create_mirror_view(H);
    auto u = Kokkos::create_mirror_view(U);
    for (int q = 0; q < Q; ++q)
      for (int a = 0; a < A; ++a) h(q, a) = hv(q, a);
    for (int e = 0; e < E; ++e)
      for (int a = 0; a < A; ++a)
        for (int b = 0; b < B; ++b)
          for (int c = 0; c < C; ++c) u(e, a, b, c) = uv(e, a, b, c);
    Kokkos::deep_copy(H, h);
    Kokkos::deep_copy(U, u);
  }
  static double g(int q, int e, int b, int c) {  // sum_a H[q,a] U[e,a,b,c]
    double s = 0;
    for (int a = 0; a < A; ++a) s += double(hv(q, a)) * uv(e, a, b, c);
    return s;
  }
};

struct Scale {
  KOKKOS_FUNCTION float operator()(int, int, int, int, float x) const { return 2.0f * x + 0.5f; }
};
struct Dup {
  KOKKOS_FUNCTION Kokkos::Array<float, 2> operator()(int, int, int, int, float x) const {
    return {2.0f * x, 3.0f * x};
  }
};
struct Probe {  // sees (e, b, q, c) global coordinates
  KOKKOS_FUNCTION float operator()(int e, int b, int q, int c, float x) const {
    return x + 1000.0f * e + 10.0f * b + 1.0f * q + 0.5f * c;
  }
};

template <int TE>
void scenarios_same_extents() {
  constexpr int N = 5, E = 8;
  using Map = LabelTiles<LabelWhole<'q', N>, LabelWhole<'a', N>, LabelTile<'e', TE>,
                         LabelWhole<'b', N>, LabelWhole<'c', N>>;
  Data<N, N, N, N, E> d;
  using D = Data<N, N, N, N, E>;
  auto host = [](const V4& v) { return Kokkos::create_mirror_view_and_copy(Kokkos::HostSpace{}, v); };
  {  // single contraction
    V4 C("C", N, E, N, N);
    auto g0 = make_level_graph<float, ES>(Map{});
    auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(d.H))));
    auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(d.U))));
    auto [g3, ca] = g2.add(make_contraction_node<'q', 'e', 'b', 'c'>(h, u));
    g3.outputs(ca).execute(TeamPolicyTag2<ES>{}, C);
    Kokkos::fence();
    auto Ch = host(C);
    double err = 0;
    for (int q = 0; q < N; ++q)
      for (int e = 0; e < E; ++e)
        for (int b = 0; b < N; ++b)
          for (int c = 0; c < N; ++c) err = std::fmax(err, std::fabs(D::g(q, e, b, c) - Ch(q, e, b, c)));
    report("single contraction", err, 1e-4);
  }
  {  // three-member gradient level: one staged H relabelled per direction
    V4 A("A", N, E, N, N), B("B", N, E, N, N), C("C", N, E, N, N);
    auto g0 = make_level_graph<float, ES>(Map{});
    auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(d.H))));
    auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(d.U))));
    auto [g3, ha, hb, hc] = g2.add(make_contraction_node<'q', 'e', 'b', 'c'>(h, u),
                                   make_contraction_node<'q', 'e', 'a', 'c'>(h.template as<'q', 'b'>(), u),
                                   make_contraction_node<'q', 'e', 'a', 'b'>(h.template as<'q', 'c'>(), u));
    g3.outputs(ha, hb, hc).team_size(64).execute(TeamPolicyTag2<ES>{}, A, B, C);
    Kokkos::fence();
    auto Ah = host(A), Bh = host(B), Chh = host(C);
    double ea = 0, eb = 0, ec = 0;
    for (int q = 0; q < N; ++q)
      for (int e = 0; e < E; ++e)
        for (int m = 0; m < N; ++m)
          for (int n = 0; n < N; ++n) {
            double ra = 0, rb = 0, rc = 0;
            for (int k = 0; k < N; ++k) {
              ra += double(hv(q, k)) * uv(e, k, m, n);
              rb += double(hv(q, k)) * uv(e, m, k, n);
              rc += double(hv(q, k)) * uv(e, m, n, k);
            }
            ea = std::fmax(ea, std::fabs(ra - Ah(q, e, m, n)));
            eb = std::fmax(eb, std::fabs(rb - Bh(q, e, m, n)));
            ec = std::fmax(ec, std::fabs(rc - Chh(q, e, m, n)));
          }
    report("fused gradient level (3 members)", std::fmax(ea, std::fmax(eb, ec)), 1e-4);
  }
  {  // combine over a contraction, and a two-output combine
    V4 P("P", N, E, N, N), O0("O0", N, E, N, N), O1("O1", N, E, N, N);
    auto g0 = make_level_graph<float, ES>(Map{});
    auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(d.H))));
    auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(d.U))));
    auto [g3, ca] = g2.add(make_contraction_node<'q', 'e', 'b', 'c'>(h, u));
    auto [g4, pa] = g3.add(make_combine_node<'q', 'e', 'b', 'c'>(ca, Scale{}));
    g4.outputs(pa).execute(TeamPolicyTag2<ES>{}, P);
    auto [g4b, o0, o1] = g3.add(make_combine_node<'q', 'e', 'b', 'c'>(ca, Dup{}));
    g4b.outputs(o0, o1).execute(TeamPolicyTag2<ES>{}, O0, O1);
    Kokkos::fence();
    auto Ph = host(P), H0 = host(O0), H1 = host(O1);
    double ep = 0, e0 = 0, e1 = 0;
    for (int q = 0; q < N; ++q)
      for (int e = 0; e < E; ++e)
        for (int b = 0; b < N; ++b)
          for (int c = 0; c < N; ++c) {
            const double g = D::g(q, e, b, c);
            ep = std::fmax(ep, std::fabs(2 * g + 0.5 - Ph(q, e, b, c)));
            e0 = std::fmax(e0, std::fabs(2 * g - H0(q, e, b, c)));
            e1 = std::fmax(e1, std::fabs(3 * g - H1(q, e, b, c)));
          }
    report("combine over contraction", ep, 1e-4);
    report("two-output combine", std::fmax(e0, e1), 1e-4);
  }
}

template <int TE>
void scenarios_declared_order() {
  constexpr int Q = 7, A = 3, B = 4, C = 5, P = 6, E = 8;
  using Map = LabelTiles<LabelWhole<'q', Q>, LabelWhole<'a', A>, LabelWhole<'b', B>,
                         LabelWhole<'c', C>, LabelTile<'e', TE>, LabelWhole<'p', P>>;
  Data<Q, A, B, C, E> d;
  using D = Data<Q, A, B, C, E>;
  auto host = [](const V4& v) { return Kokkos::create_mirror_view_and_copy(Kokkos::HostSpace{}, v); };
  {  // contraction declared (e, b, q, c) -- a 3-cycle of the canonical (q, e, b, c)
    V4 O("O", E, B, Q, C);
    auto g0 = make_level_graph<float, ES>(Map{});
    auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(d.H))));
    auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(d.U))));
    auto [g3, ca] = g2.add(make_contraction_node<'e', 'b', 'q', 'c'>(h, u));
    g3.outputs(ca).execute(TeamPolicyTag2<ES>{}, O);
    Kokkos::fence();
    auto Oh = host(O);
    double err = 0;
    for (int e = 0; e < E; ++e)
      for (int b = 0; b < B; ++b)
        for (int q = 0; q < Q; ++q)
          for (int c = 0; c < C; ++c) err = std::fmax(err, std::fabs(D::g(q, e, b, c) - Oh(e, b, q, c)));
    report("declared-order contraction root", err, 1e-4);
  }
  {  // combine reads the declared slot in a third order (q, c, e, b)
    V4 O("O", Q, C, E, B);
    auto g0 = make_level_graph<float, ES>(Map{});
    auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(d.H))));
    auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(d.U))));
    auto [g3, ca] = g2.add(make_contraction_node<'e', 'b', 'q', 'c'>(h, u));
    auto [g4, pa] = g3.add(make_combine_node<'q', 'c', 'e', 'b'>(ca, Scale{}));
    g4.outputs(pa).execute(TeamPolicyTag2<ES>{}, O);
    Kokkos::fence();
    auto Oh = host(O);
    double err = 0;
    for (int q = 0; q < Q; ++q)
      for (int c = 0; c < C; ++c)
        for (int e = 0; e < E; ++e)
          for (int b = 0; b < B; ++b)
            err = std::fmax(err, std::fabs(2 * D::g(q, e, b, c) + 0.5 - Oh(q, c, e, b)));
    report("combine over declared-order slot", err, 1e-4);
  }
  {  // a contraction reads the declared slot, and declares its own output non-canonically
    V2 W("W", P, Q);
    auto Wh = Kokkos::create_mirror_view(W);
    for (int p = 0; p < P; ++p)
      for (int q = 0; q < Q; ++q) Wh(p, q) = wv(p, q);
    Kokkos::deep_copy(W, Wh);
    V4 O("O", E, B, P, C);
    auto g0 = make_level_graph<float, ES>(Map{});
    auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(d.H))));
    auto [g2, w] = g1.add(make_stage_node(make_input_node(make_handle<'p', 'q'>(W))));
    auto [g3, u] = g2.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(d.U))));
    auto [g4, ca] = g3.add(make_contraction_node<'e', 'b', 'q', 'c'>(h, u));
    auto [g5, cb] = g4.add(make_contraction_node<'e', 'b', 'p', 'c'>(w, ca));
    g5.outputs(cb).execute(TeamPolicyTag2<ES>{}, O);
    Kokkos::fence();
    auto Oh = host(O);
    double err = 0;
    for (int e = 0; e < E; ++e)
      for (int b = 0; b < B; ++b)
        for (int p = 0; p < P; ++p)
          for (int c = 0; c < C; ++c) {
            double ref = 0;
            for (int q = 0; q < Q; ++q) ref += double(wv(p, q)) * D::g(q, e, b, c);
            err = std::fmax(err, std::fabs(ref - Oh(e, b, p, c)));
          }
    report("contraction over declared-order slot", err, 1e-4);
  }
  {  // the combine fn sees GLOBAL coordinates (4 tiles along e)
    V4 O("O", E, B, Q, C);
    auto g0 = make_level_graph<float, ES>(Map{});
    auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(d.H))));
    auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(d.U))));
    auto [g3, ca] = g2.add(make_contraction_node<'e', 'b', 'q', 'c'>(h, u));
    auto [g4, pa] = g3.add(make_combine_node<'e', 'b', 'q', 'c'>(ca, Probe{}));
    const int league = g4.outputs(pa).execute(TeamPolicyTag2<ES>{}, O);
    Kokkos::fence();
    auto Oh = host(O);
    double err = 0;
    for (int e = 0; e < E; ++e)
      for (int b = 0; b < B; ++b)
        for (int q = 0; q < Q; ++q)
          for (int c = 0; c < C; ++c)
            err = std::fmax(err, std::fabs(D::g(q, e, b, c) + 1000.0 * e + 10.0 * b + q + 0.5 * c -
                                           Oh(e, b, q, c)));
    report("combine fn sees global coordinates", err, 1e-3);
    if (league != (E + TE - 1) / TE) {
      ++g_fail;
      std::printf("league %d != %d FAIL\n", league, (E + TE - 1) / TE);
    }
  }
}

// Kernel-parameter layout: the device must read every member of a nested
// DeviceTuple (the form levels, operands and root views travel in) at the
// same bytes the host wrote.  Each value read on the device is compared with
// the host's.
struct Tag3 {
  int a;
  double b;
};
template <class T>
__global__ void tuple_layout_kernel(const T t, long long* out) {
  out[0] = (long long)t.template get<0>().template get<0>().data();
  out[1] = (long long)t.template get<1>().template get<0>().data();
  out[2] = (long long)t.template get<1>().template get<0>().extent(3);
  out[3] = t.template get<2>().template get<0>();
  out[4] = (long long)t.template get<2>().template get<1>().b;
  out[5] = (long long)t.template get<2>().template get<2>().data();
  out[6] = (long long)t.template get<2>().template get<2>().extent(1);
  out[7] = (long long)sizeof(T);
}

void kernel_parameter_layout() {
  V2 a("a", 3, 4), c("c", 5, 6);
  V4 b("b", 2, 3, 4, 7);
  using T = DeviceTuple<DeviceTuple<V2>, DeviceTuple<V4>, DeviceTuple<int, Tag3, V2>>;
  const T t(DeviceTuple<V2>(a), DeviceTuple<V4>(b), DeviceTuple<int, Tag3, V2>(11, Tag3{1, 42.0}, c));
  long long* d = nullptr;
  cudaMalloc(&d, 8 * sizeof(long long));
  cudaMemset(d, 0, 8 * sizeof(long long));
  tuple_layout_kernel<T><<<1, 1>>>(t, d);
  long long got[8] = {};
  cudaMemcpy(got, d, sizeof(got), cudaMemcpyDeviceToHost);
  cudaFree(d);
  const long long want[8] = {(long long)a.data(), (long long)b.data(), 7, 11, 42,
                             (long long)c.data(), 6, (long long)sizeof(T)};
  int bad = 0;
  for (int i = 0; i < 8; ++i) bad += got[i] != want[i];
  report("kernel parameter layout (nested DeviceTuple)", bad, 0.5);
}

// The same check on a real level tuple (stage, contraction and combine
// members): the device reads the staged View and the members' shapes.
template <class Lv>
__global__ void level_layout_kernel(const Lv levels, long long* out) {
  const auto& u = levels.template get<1>().template get<0>().operand_.handle.tensor;
  out[0] = (long long)levels.template get<0>().template get<0>().operand_.handle.tensor.data();
  out[1] = (long long)u.data();
  out[2] = (long long)u.extent(0);
  out[3] = levels.template get<2>().template get<0>().shape()[1];
  out[4] = levels.template get<3>().template get<0>().shape()[1];
  out[5] = (long long)sizeof(Lv);
}

void level_tuple_layout() {
  constexpr int N = 5, E = 9;
  using Map = LabelTiles<LabelWhole<'q', N>, LabelWhole<'a', N>, LabelTile<'e', 2>,
                         LabelWhole<'b', N>, LabelWhole<'c', N>>;
  V2 H("H", N, N);
  V4 U("U", E, N, N, N);
  auto g0 = make_level_graph<float, ES>(Map{});
  auto [g1, h] = g0.add(make_stage_node(make_input_node(make_handle<'q', 'a'>(H))));
  auto [g2, u] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'a', 'b', 'c'>(U))));
  auto [g3, ca] = g2.add(make_contraction_node<'q', 'e', 'b', 'c'>(h, u));
  auto [g4, pa] = g3.add(make_combine_node<'q', 'e', 'b', 'c'>(ca, Scale{}));
  using Lv = typename decltype(g4)::levels_type;
  long long* d = nullptr;
  cudaMalloc(&d, 6 * sizeof(long long));
  cudaMemset(d, 0, 6 * sizeof(long long));
  level_layout_kernel<Lv><<<1, 1>>>(g4.levels, d);
  long long got[6] = {};
  cudaMemcpy(got, d, sizeof(got), cudaMemcpyDeviceToHost);
  cudaFree(d);
  const long long want[6] = {(long long)H.data(), (long long)U.data(), E, E, E, (long long)sizeof(Lv)};
  int bad = 0;
  for (int i = 0; i < 6; ++i) bad += got[i] != want[i];
  report("kernel parameter layout (level tuple)", bad, 0.5);
}

int main(int argc, char* argv[]) {
  Kokkos::initialize(argc, argv);
  kernel_parameter_layout();
  level_tuple_layout();
  if (g_fail) {  // operands would be read from the wrong bytes: run nothing else
    Kokkos::finalize();
    std::printf("level graph runtime: FAIL (kernel parameter layout)\n");
    return 1;
  }
  scenarios_same_extents<2>();
  scenarios_same_extents<3>();  // 8 elements in tiles of 3: a partial last tile
  scenarios_declared_order<2>();
  scenarios_declared_order<3>();
  Kokkos::finalize();
  std::printf("level graph runtime: %s (%d failures)\n", g_fail ? "FAIL" : "PASS", g_fail);
  return g_fail ? 1 : 0;
}
