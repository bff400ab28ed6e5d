// level_kernel_host_check.cpp -- TEST ONLY: the generic level-graph device
// evaluator (TensorOperations/b200/LevelKernel.cuh) compiled as HOST code, one
// thread per CTA, so its index arithmetic (stage, contraction, combine and
// root-store offsets, partial last tiles) can be checked on a CPU under
// AddressSanitizer / UBSan against a direct loop.  The CUDA keywords are
// defined away below; __syncthreads() is a no-op because with one thread per
// CTA every level loop finishes before the next begins.  Built and run by
// tests/test_frontend_cpu.py.  The product has no host execution path.
#include <cstdio>
#include <cmath>
#include <cstdlib>
#define __device__
#define __forceinline__ inline
#define __global__
#define __launch_bounds__(x)
#define __shared__
#define __align__(n) __attribute__((aligned(n)))
struct EmuDim { unsigned x = 0, y = 0, z = 0; };
inline EmuDim threadIdx, blockIdx, blockDim{1, 1, 1}, gridDim;
inline void __syncthreads() {}
#include <Kokkos_Core.hpp>
#include <TensorOperations/LevelGraph.hpp>
namespace TensorOperations::b200 { alignas(16) unsigned char lg_smem[1 << 20]; }
#include <TensorOperations/b200/LevelKernel.cuh>
using namespace TensorOperations;
using ES = Kokkos::DefaultExecutionSpace;
using V4 = Kokkos::View<float* [5][5][5], Kokkos::LayoutRight>;
using V2 = Kokkos::View<float**, Kokkos::LayoutRight>;
using GMap = LabelTiles<LabelTile<'e', 2>, LabelWhole<'k', 5>, LabelWhole<'j', 5>,
                        LabelWhole<'i', 5>, LabelWhole<'p', 5>, LabelWhole<'r', 5>>;
struct F9 {
  V4 s;
  Kokkos::Array<float, 9> operator()(int e, int k, int j, int i, float a, float b, float c, float d,
                                     float f, float g, float h, float x, float y) const {
    const float m = s(e, k, j, i);
    return {m * a, b, c + m, d, f, g, h, x, y};
  }
};
struct WS {
  float operator()(int, int, int, int, float a, float b, float c) const { return a + 2 * b + 3 * c; }
};
int main(int argc, char** argv) {
  const int E = argc > 1 ? std::atoi(argv[1]) : 5;
  V2 H("H", 5, 5), Hw("Hw", 5, 5);
  V4 u0("u0", E), u1("u1", E), u2("u2", E), sc("sc", E), f0("f0", E), f1("f1", E), f2("f2", E);
  for (int a = 0; a < 5; ++a) for (int b = 0; b < 5; ++b) { H(a, b) = 0.1f * a - 0.2f * b + (a == b); Hw(a, b) = 0.3f * b + 0.05f * a * b; }
  for (int n = 0; n < E * 125; ++n) { u0.data()[n] = std::sin(0.1f * n); u1.data()[n] = std::cos(0.07f * n); u2.data()[n] = 0.01f * n; sc.data()[n] = 1.f + 0.001f * n; }
  auto g0 = make_level_graph<float, ES>(GMap{});
  auto [g1, h, hw] = g0.add(make_stage_node(make_input_node(make_handle<'r', 'p'>(H))),
                            make_stage_node(make_input_node(make_handle<'p', 'r'>(Hw))));
  auto [g2, a, b, c] = g1.add(make_stage_node(make_input_node(make_handle<'e', 'k', 'j', 'i'>(u0))),
                              make_stage_node(make_input_node(make_handle<'e', 'k', 'j', 'i'>(u1))),
                              make_stage_node(make_input_node(make_handle<'e', 'k', 'j', 'i'>(u2))));
  auto gx = [&](auto x) { return make_contraction_node<'e', 'k', 'j', 'i'>(h.template as<'i', 'p'>(), x.template as<'e', 'k', 'j', 'p'>()); };
  auto ge = [&](auto x) { return make_contraction_node<'e', 'k', 'j', 'i'>(h.template as<'j', 'p'>(), x.template as<'e', 'k', 'p', 'i'>()); };
  auto gg = [&](auto x) { return make_contraction_node<'e', 'k', 'j', 'i'>(h.template as<'k', 'p'>(), x.template as<'e', 'p', 'j', 'i'>()); };
  auto [g3, x0, x1, x2, e0, e1, e2, y0, y1, y2] = g2.add(gx(a), gx(b), gx(c), ge(a), ge(b), ge(c), gg(a), gg(b), gg(c));
  auto [g4, q0, q1, q2, q3, q4, q5, q6, q7, q8] = g3.add(make_combine_node<'e', 'k', 'j', 'i'>(x0, x1, x2, e0, e1, e2, y0, y1, y2, F9{sc}));
  auto dx = [&](auto f) { return make_contraction_node<'e', 'k', 'j', 'i'>(hw.template as<'p', 'i'>(), f.template as<'e', 'k', 'j', 'p'>()); };
  auto de = [&](auto f) { return make_contraction_node<'e', 'k', 'j', 'i'>(hw.template as<'p', 'j'>(), f.template as<'e', 'k', 'p', 'i'>()); };
  auto dg = [&](auto f) { return make_contraction_node<'e', 'k', 'j', 'i'>(hw.template as<'p', 'k'>(), f.template as<'e', 'p', 'j', 'i'>()); };
  auto [g5, t0, t1, t2, t3, t4, t5, t6, t7, t8] = g4.add(dx(q0), dx(q1), dx(q2), de(q3), de(q4), de(q5), dg(q6), dg(q7), dg(q8));
  auto [g6, r0, r1, r2] = g5.add(make_combine_node<'e', 'k', 'j', 'i'>(t0, t3, t6, WS{}),
                                 make_combine_node<'e', 'k', 'j', 'i'>(t1, t4, t7, WS{}),
                                 make_combine_node<'e', 'k', 'j', 'i'>(t2, t5, t8, WS{}));
  using Levels = typename decltype(g6)::levels_type;
  using GK = b200::GraphKernel<float, GMap, Levels, decltype(r0)::SlotIdx, decltype(r1)::SlotIdx, decltype(r2)::SlotIdx>;
  b200::GridRuntime<GK::GR> grid{};
  grid.ntiles[0] = (E + 1) / 2;
  DeviceTuple<V4, V4, V4> views(f0, f1, f2);
  std::printf("scratch %zu\n", GK::Lay::scratch_bytes);
  for (unsigned bx = 0; bx < (unsigned)grid.ntiles[0]; ++bx) { blockIdx.x = bx; GK::run(g6.levels, grid, views); }
  // direct reference
  double worst = 0;
  for (int e = 0; e < E; ++e) for (int k = 0; k < 5; ++k) for (int j = 0; j < 5; ++j) for (int i = 0; i < 5; ++i) {
    V4* us[3] = {&u0, &u1, &u2};
    auto grad = [&](int c, int dir, int e2, int k2, int j2, int i2) {
      double s = 0; for (int p = 0; p < 5; ++p) {
        if (dir == 0) s += H(i2, p) * (*us[c])(e2, k2, j2, p);
        if (dir == 1) s += H(j2, p) * (*us[c])(e2, k2, p, i2);
        if (dir == 2) s += H(k2, p) * (*us[c])(e2, p, j2, i2); }
      return s; };
    auto Fv = [&](int o, int e2, int k2, int j2, int i2) {
      double g[9]; for (int d = 0; d < 3; ++d) for (int c = 0; c < 3; ++c) g[3 * d + c] = grad(c, d, e2, k2, j2, i2);
      const double m = sc(e2, k2, j2, i2);
      double r[9] = {m * g[0], g[1], g[2] + m, g[3], g[4], g[5], g[6], g[7], g[8]}; return r[o]; };
    double out[3];
    for (int c = 0; c < 3; ++c) {
      double tx = 0, te = 0, tg = 0;
      for (int p = 0; p < 5; ++p) { tx += Hw(p, i) * Fv(c, e, k, j, p); te += Hw(p, j) * Fv(3 + c, e, k, p, i); tg += Hw(p, k) * Fv(6 + c, e, p, j, i); }
      out[c] = tx + 2 * te + 3 * tg;
    }
    worst = std::fmax(worst, std::fabs(out[0] - f0(e, k, j, i)));
    worst = std::fmax(worst, std::fabs(out[1] - f1(e, k, j, i)));
    worst = std::fmax(worst, std::fabs(out[2] - f2(e, k, j, i)));
  }
  std::printf("max abs error %.3e\n", worst);
  return worst < 1e-3 ? 0 : 1;
}
