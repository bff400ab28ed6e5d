// tc_contract_gpu.cpp -- TEST ONLY (GPU): a large fp32 contraction of two
// inputs through the public API, which the frontend runs as a tensor-core GEMM
// (b200/TcContract.hpp: pack -> to_gemm_tf32x3 -> unpack), against a float64
// host loop.  Permuted operands and output, contracted labels spanning several
// bundle tiles, an input hook and a contraction hook, ragged sizes:
//   C[l, i] = h( sum_{j,k} A[j, i, k] * g(B[k, j, l]) )
// through the tree route (make_graph().ops) and the DAG route (make_dag), plus
// a small case (M < 128) that stays on the level evaluator; and chains whose
// intermediate is contracted over one (fused), three (run in steps, the root a
// self-staging contraction) and four (in steps, the root on the tensor cores)
// tiles; and a fusible chain whose root is large enough for the tensor cores
// (in steps with them, fused without); and the permuted rank-4 chain of the
// chain benchmark (config 4) at extent 32.  Prints one line
// per case with the relative error and the league execute() returned (the
// GEMM's tile count on the tensor-core path; the grid on the level path).
// Run by tests/test_frontend_gpu.py, with and without
// TO_FRONTEND_TENSOR_CORES=0.
#include <Kokkos_Core.hpp>
#include <TensorOperations/DagGraph.hpp>
#include <TensorOperations/Graph.hpp>
#include <TensorOperations/Tiling.hpp>

#include <cmath>
#include <cstdio>
#include <vector>

using namespace TensorOperations;
using ES = Kokkos::DefaultExecutionSpace;
using V3 = Kokkos::View<float***, Kokkos::LayoutRight>;
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;

struct InHook {
  KOKKOS_FUNCTION void operator()(int k, int, int l, float& v) const { v *= 1.f + 0.01f * ((k + l) % 5); }
};
struct OutHook {
  KOKKOS_FUNCTION void operator()(int l, int i, float& v) const { v += 0.001f * l - 0.002f * i; }
};

using Bundle = Tile<StaticTile<4, 32, 4>, StaticTile<4, 4, 32>, StaticTile<32, 32>>;

static double run_case(int I, int L, int J, int K, int route, int* league_out) {
  V3 A("A", J, I, K), B("B", K, J, L);
  V2 C("C", L, I);
  auto hA = Kokkos::create_mirror_view(A);
  auto hB = Kokkos::create_mirror_view(B);
  for (int j = 0; j < J; ++j)
    for (int i = 0; i < I; ++i)
      for (int k = 0; k < K; ++k) hA(j, i, k) = std::sin(0.013f * i + 0.7f * j - 0.3f * k);
  for (int k = 0; k < K; ++k)
    for (int j = 0; j < J; ++j)
      for (int l = 0; l < L; ++l) hB(k, j, l) = std::cos(0.021f * l - 0.4f * j + 0.9f * k);
  Kokkos::deep_copy(A, hA);
  Kokkos::deep_copy(B, hB);
  auto node = make_contraction_node<'l', 'i'>(make_input_node(make_handle<'j', 'i', 'k'>(A)),
                                              make_input_node(make_handle<'k', 'j', 'l'>(B), InHook{}),
                                              OutHook{});
  int league = 0;
  if (route == 0) {
    auto [g1, h] = make_graph().ops(node);
    (void)h;
    league = g1.execute(TeamPolicyTag<ES>{}, Bundle{}, C);
  } else {
    auto [g, h] = make_dag<float, ES>().add(node, Bundle{});
    league = g.outputs(h).execute(TeamPolicyTag<ES>{}, C);
  }
  Kokkos::fence();
  *league_out = league;
  auto hC = Kokkos::create_mirror_view_and_copy(Kokkos::HostSpace{}, C);
  double num = 0, den = 0;
  for (int l = 0; l < L; ++l)
    for (int i = 0; i < I; ++i) {
      double s = 0;
      for (int j = 0; j < J; ++j)
        for (int k = 0; k < K; ++k) {
          float b = hB(k, j, l);
          InHook{}(k, j, l, b);
          s += double(hA(j, i, k)) * double(b);
        }
      const double want = s + (0.001 * l - 0.002 * i);  // OutHook in float64
      num += (hC(l, i) - want) * (hC(l, i) - want);
      den += want * want;
    }
  return std::sqrt(num / den);
}

// A chain whose intermediate is contracted over several tiles, run in steps
// (the intermediate evaluated into a buffer, then the root):
//   M[j, i] = m( sum_k A[i, k] B[k, j] ),  E[l, i] = sum_j M[j, i] D[j, l]
struct MidHook {
  KOKKOS_FUNCTION void operator()(int j, int i, float& v) const { v = v * 0.5f + 0.001f * (j - i); }
};
using TopBundle = Tile<StaticTile<32, 32>, StaticTile<32, 32>, StaticTile<32, 32>>;
using MidBundle = Tile<StaticTile<32, 16>, StaticTile<16, 32>, StaticTile<32, 32>>;

static double run_chain(int I, int L, int J, int K, int* league_out) {
  V2 A("A", I, K), B("B", K, J), D("D", J, L), E("E", L, I);
  auto hA = Kokkos::create_mirror_view(A);
  auto hB = Kokkos::create_mirror_view(B);
  auto hD = Kokkos::create_mirror_view(D);
  for (int i = 0; i < I; ++i)
    for (int k = 0; k < K; ++k) hA(i, k) = std::sin(0.017f * i - 0.5f * k);
  for (int k = 0; k < K; ++k)
    for (int j = 0; j < J; ++j) hB(k, j) = std::cos(0.3f * k + 0.023f * j);
  for (int j = 0; j < J; ++j)
    for (int l = 0; l < L; ++l) hD(j, l) = std::sin(0.011f * l + 0.031f * j + 0.2f);
  Kokkos::deep_copy(A, hA);
  Kokkos::deep_copy(B, hB);
  Kokkos::deep_copy(D, hD);
  auto M = make_contraction_node<'j', 'i'>(make_input_node(make_handle<'i', 'k'>(A)),
                                           make_input_node(make_handle<'k', 'j'>(B)), MidHook{});
  auto root = make_contraction_node<'l', 'i'>(M, make_input_node(make_handle<'j', 'l'>(D)));
  auto [g, h] = make_graph().ops(root);
  (void)h;
  *league_out = g.execute(TeamPolicyTag<ES>{}, std::make_tuple(TopBundle{}, MidBundle{}), E);
  Kokkos::fence();
  auto hE = Kokkos::create_mirror_view_and_copy(Kokkos::HostSpace{}, E);
  std::vector<double> mid(static_cast<std::size_t>(J) * I);
  for (int j = 0; j < J; ++j)
    for (int i = 0; i < I; ++i) {
      double s = 0;
      for (int k = 0; k < K; ++k) s += double(hA(i, k)) * double(hB(k, j));
      mid[static_cast<std::size_t>(j) * I + i] = s * 0.5 + 0.001 * (j - i);
    }
  double num = 0, den = 0;
  for (int l = 0; l < L; ++l)
    for (int i = 0; i < I; ++i) {
      double s = 0;
      for (int j = 0; j < J; ++j) s += mid[static_cast<std::size_t>(j) * I + i] * double(hD(j, l));
      num += (hE(l, i) - s) * (hE(l, i) - s);
      den += s * s;
    }
  return std::sqrt(num / den);
}

// The permuted multilevel chain of the chain benchmark, through the public
// tree API with rank-4 permuted operands:
//   T[a, b, c, d] = sum_{e,f} A[a, e, c, f] B[f, b, e, d],
//   R[a, d]       = sum_{b,c} T[a, b, c, d] C[c, b]
// T's contracted labels b, c span four tiles, so the tree runs in steps: T on
// the tensor cores (M = (a, c), N = (b, d), K = (e, f)), then R as a
// self-staging contraction.
using V4 = Kokkos::View<float****, Kokkos::LayoutRight>;
using TBundle = Tile<StaticTile<4, 8, 8, 8>, StaticTile<8, 8, 8, 4>, StaticTile<4, 8, 8, 4>>;
using RBundle = Tile<StaticTile<4, 8, 8, 4>, StaticTile<8, 8>, StaticTile<4, 4>>;

static double run_config4(int n, int* league_out) {
  V4 A("A", n, n, n, n), B("B", n, n, n, n);
  V2 C("C", n, n), R("R", n, n);
  auto hA = Kokkos::create_mirror_view(A);
  auto hB = Kokkos::create_mirror_view(B);
  auto hC = Kokkos::create_mirror_view(C);
  for (int a = 0; a < n; ++a)
    for (int e = 0; e < n; ++e)
      for (int c = 0; c < n; ++c)
        for (int f = 0; f < n; ++f) hA(a, e, c, f) = std::sin(0.37f * a + 0.11f * e - 0.23f * c + 0.05f * f);
  for (int f = 0; f < n; ++f)
    for (int b = 0; b < n; ++b)
      for (int e = 0; e < n; ++e)
        for (int d = 0; d < n; ++d) hB(f, b, e, d) = std::cos(0.13f * f - 0.29f * b + 0.07f * e + 0.41f * d);
  for (int c = 0; c < n; ++c)
    for (int b = 0; b < n; ++b) hC(c, b) = std::sin(0.19f * c - 0.31f * b + 0.5f);
  Kokkos::deep_copy(A, hA);
  Kokkos::deep_copy(B, hB);
  Kokkos::deep_copy(C, hC);
  auto T = make_contraction_node<'a', 'b', 'c', 'd'>(make_input_node(make_handle<'a', 'e', 'c', 'f'>(A)),
                                                     make_input_node(make_handle<'f', 'b', 'e', 'd'>(B)));
  auto root = make_contraction_node<'a', 'd'>(T, make_input_node(make_handle<'c', 'b'>(C)));
  auto [g, h] = make_graph().ops(root);
  (void)h;
  *league_out = g.execute(TeamPolicyTag<ES>{}, std::make_tuple(RBundle{}, TBundle{}), R);
  Kokkos::fence();
  auto hR = Kokkos::create_mirror_view_and_copy(Kokkos::HostSpace{}, R);
  // float64: W[a, c, b, d] = sum_{e,f} A B, then R = sum_{b,c} W C
  std::vector<double> W(static_cast<std::size_t>(n) * n * n * n, 0.0);
  for (int a = 0; a < n; ++a)
    for (int c = 0; c < n; ++c)
      for (int e = 0; e < n; ++e)
        for (int f = 0; f < n; ++f) {
          const double x = hA(a, e, c, f);
          for (int b = 0; b < n; ++b)
            for (int d = 0; d < n; ++d)
              W[((static_cast<std::size_t>(a) * n + c) * n + b) * n + d] += x * double(hB(f, b, e, d));
        }
  double num = 0, den = 0;
  for (int a = 0; a < n; ++a)
    for (int d = 0; d < n; ++d) {
      double s = 0;
      for (int b = 0; b < n; ++b)
        for (int c = 0; c < n; ++c)
          s += W[((static_cast<std::size_t>(a) * n + c) * n + b) * n + d] * double(hC(c, b));
      num += (hR(a, d) - s) * (hR(a, d) - s);
      den += s * s;
    }
  return std::sqrt(num / den);
}

int main(int argc, char* argv[]) {
  Kokkos::initialize(argc, argv);
  int rc = 0;
  {
    struct Case {
      const char* name;
      int I, L, J, K, route;
    } cases[] = {{"tree_large", 300, 260, 7, 9, 0},
                 {"dag_large", 300, 260, 7, 9, 1},
                 {"tree_square", 512, 512, 16, 16, 0},
                 {"dag_small", 100, 90, 5, 6, 1}};
    for (const Case& c : cases) {
      int league = 0;
      const double err = run_case(c.I, c.L, c.J, c.K, c.route, &league);
      std::printf("case %s err %.3e league %d\n", c.name, err, league);
      if (!(err <= 1e-5)) rc = 1;
    }
    struct Chain {
      const char* name;
      int I, L, J, K;
    } chains[] = {{"chain_one_tile", 96, 64, 32, 16},
                  {"chain_three_tiles", 96, 64, 96, 16},
                  {"chain_large", 384, 320, 128, 16},
                  {"chain_large_one_tile", 2048, 2048, 32, 16}};
    for (const Chain& c : chains) {
      int league = 0;
      const double err = run_chain(c.I, c.L, c.J, c.K, &league);
      std::printf("case %s err %.3e league %d\n", c.name, err, league);
      if (!(err <= 1e-5)) rc = 1;
    }
    {
      int league = 0;
      const double err = run_config4(32, &league);
      std::printf("case config4_n32 err %.3e league %d\n", err, league);
      if (!(err <= 1e-5)) rc = 1;
    }
  }
  Kokkos::finalize();
  return rc;
}
