// sem3d_elastic_v5.cuh -- f32 fused SEM 3D elastic kernel, "line owner" design.
//
// Measured on the point-pair kernel: the SM's L1 / shared-memory pipe was the
// limiter (about 630 wavefronts per element against about 710 cycles), and
// most shared-memory traffic was the xi / eta contractions: every thread of
// an i-row read the same five neighbours and produced one output, so each
// row was read five times.  Here every thread holds three roles at once:
//
//   column owner   (le, j=a, i=b), the N points k = 0..N-1: gathers u,
//                  contracts along k in registers (gamma), evaluates the
//                  Integrand9 physics at its points, scatters f;
//   xi-line owner  (le, k=b, j=a), the N points i = 0..N-1: reads the row
//                  once and produces all N xi-derivatives (and later all N
//                  xi-divergences) of that row;
//   eta-line owner (le, k=a, i=b): the same along j.
//
// A thread's lane is t = le*25 + a*5 + b.  Shared buffers keep one word per
// point, k-major: word (k*SK + le*25 + j*5 + i).  The k-stride SK is
// 25*EB + 25 for the buffers the xi-lines read or write and 25*EB + 29 for
// the eta-side ones (129 and 101 for EB = 4); with these strides every access
// of every phase -- a column at fixed k (consecutive words), a xi-row at fixed
// i, an eta-row at fixed j -- touches 32 distinct banks (checked exhaustively
// for EB = 4, 8, 12, 16), so u is written twice, once in each layout.  Per thread and batch of 5 points:
// 120 shared stores + 120 exchange loads + 60 geometry loads, all
// conflict-free.
//
// Phases per batch (4 barriers), all in two buffers X (xi side) and E (eta
// side), each value overwriting its input in place -- a row's words are read
// and written only by its line owner, a column's only by its column owner:
//   A  column: u -> X, E; gamma-gradients in registers
//   B1 lines:  X rows -> xi-gradients (in place), E rows -> eta-gradients
//   B2 column: gradients + gamma -> Integrand9 (geometry from the staged
//              arrays) -> F^xi into X, F^eta into E (in place); gamma fluxes
//              stay in registers
//   C1 lines:  F rows -> xi- / eta-divergences (in place)
//   C2 column: divergences + gamma-divergence -> WeightedSum -> scatter-add /
//              store
// Two buffers instead of four keep a CTA of 8 elements at about 74 KB of
// shared memory, so three CTAs (600 threads) fit on an SM.
// The 12 per-point arrays stream global -> shared with bulk copies (as in the
// point-pair kernel) and the next batch's ibool / u gathers are in flight
// during C1 / C2.
#pragma once

#include <cstdint>

#include "sem3d_elastic.cuh"
#include "sem3d_elastic_tma.cuh"
#include "sm100_primitives.cuh"

namespace to_b200 {

template <int EB, bool ASM>
struct Sem3dV5Layout {
  static constexpr int N = 5, NN = 25, P = 125, NT = EB * NN, EP = EB * P;
  // k-strides of the xi- and eta-side buffers: the smallest strides >= NT with
  // every access pattern conflict-free for this batch size (exhaustive search)
  static_assert(EB == 4 || EB == 8 || EB == 12 || EB == 16, "strides searched for EB 4/8/12/16");
  static constexpr int SKX = EB == 4 ? 129 : NT + 25;
  static constexpr int SKE = EB == 4 ? 101 : NT + 29;
  static constexpr int kStaged = kNumPointArrays + (ASM ? 0 : 3);
  static constexpr size_t kHeader = 128;
  static constexpr size_t kStageBytes = size_t(kStaged) * EP * 4;
  static constexpr size_t kXBytes = (size_t(3) * N * SKX * 4 + 15) & ~size_t(15);
  static constexpr size_t kEBytes = (size_t(3) * N * SKE * 4 + 15) & ~size_t(15);
  static constexpr size_t kTotal = kHeader + kStageBytes + kXBytes + kEBytes;
};

// Up to two element ranges processed in order, batch by batch, with the
// batches handed out by a device-wide ticket counter instead of the static
// grid stride (option kV5Ranges).  Batches never straddle a range: the last
// batch of a range may hold fewer than EB elements.  The z-slab operator uses
// it to scatter the two element layers next to its neighbours in one launch
// and to run the interior so that CTAs which start late (their SM was busy
// with the exchange) simply take fewer batches.
struct Sem3dV5Ranges {
  long long first[2];            // first element of each range
  long long count[2];            // elements of each range (count[1] = 0: one range)
  long long nb[2];               // batches of each range
  unsigned long long* ticket;    // zeroed before the launch; one ticket per batch fetch
};

// The kernel's parameters: the common arguments plus the operators splatted
// into f32 pairs, so a packed FMA takes both lanes' coefficient from one
// 64-bit constant.
struct Sem3dV5Args {
  Sem3dArgs<float, 5> a;
  float2 H2[5][5];   // (H(i,p), H(i,p))
  float2 Hw2[5][5];  // (Hw(q,i), Hw(q,i))
  Sem3dV5Ranges rg;  // used with kV5Ranges only
};

// Options of the line-owner kernel (OPT bit mask):
//   kV5Packed    the contractions in packed f32x2 FMAs: each line owner pairs
//                its xi and eta rows, each column owner pairs components 0
//                and 1 (element-local NGLL 5 at E=786,432: 1.491 vs 1.518 ms;
//                assembled 64^3: unchanged).
// (Waiting for the staged geometry just before B2 instead of before A, so the
// bulk copies also overlap A and B1, measured 0.597 vs 0.592 ms and was
// removed.)
//   kV5Ranges    the element ranges of Sem3dV5Args::rg with ticketed batches.
//   kV5WarpAgg   warp-aggregated scatter-add (assembled): the point (le, j, i=4, k)
//                and (le+1, j, i=0, k) of x-adjacent elements are one node; when
//                the two owners sit in one warp (lanes 21 apart) and ibool gives
//                them the same node, the i=4 owner adds its partner's
//                contribution (one shuffle per component) and only it issues the
//                atomic.  Opt-in (TO_SEM3D_WARP_AGG=1): it removes about 6 % of
//                the atomics but the shuffles cost more of the L1 pipe than they
//                save (64^3, interleaved: 0.550 vs 0.497 ms).
enum : int { kV5Packed = 2, kV5Ranges = 4, kV5WarpAgg = 8 };

// IL: assembled u and f interleaved per node (x, y, z, unused) -- one 128-bit
// gather and one 128-bit atomicAdd per point instead of three of each.
template <int EB, int MINB, bool ASM, bool IL = false, int OPT = kV5Packed>
__global__ void __launch_bounds__(EB * 25, MINB)
    sem3d_elastic_v5_kernel(const __grid_constant__ Sem3dV5Args args) {
  const Sem3dArgs<float, 5>& a = args.a;
  constexpr bool kPk = (OPT & kV5Packed) != 0;
  constexpr bool kRg = (OPT & kV5Ranges) != 0;
  constexpr bool kAgg = ASM && (OPT & kV5WarpAgg) != 0;
  using LY = Sem3dV5Layout<EB, ASM>;
  constexpr int N = 5, NN = 25, P = 125, NT = LY::NT, EP = LY::EP;
  constexpr int SKX = LY::SKX, SKE = LY::SKE;
  constexpr int CX = N * SKX, CE = N * SKE;  // component strides
  constexpr int kStaged = LY::kStaged;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);
  float* stage = reinterpret_cast<float*>(smem_raw + LY::kHeader);
  float* RX = reinterpret_cast<float*>(smem_raw + LY::kHeader + LY::kStageBytes);  // xi side
  float* RE = RX + LY::kXBytes / 4;                                               // eta side
  float* RDX = RX;  // the same words, named by what they hold in B1 / C1 outputs
  float* RDE = RE;

  const int tid = threadIdx.x;
  const int le = tid / NN;
  const int ab = tid - le * NN;
  const int ra = ab / N;  // column j / xi-line j / eta-line k
  const int rb = ab - ra * N;  // column i / xi-line k / eta-line i
  const int lx = rb * SKX + le * NN + ra * N;  // xi-line (k=b, j=a): + i
  const int ly = ra * SKE + le * NN + rb;      // eta-line (k=a, i=b): + 5 j
  const int spt = le * P + ab;                  // staged point (k=0, j=a, i=b): + k*NN

  const long long nbatch = kRg ? args.rg.nb[0] + args.rg.nb[1] : (a.nelem + EB - 1) / EB;
  const long long G = gridDim.x;
  const uint64_t pol_stream = l2_policy_evict_first();

  // batch bb -> its first element and element count
  auto batch_first = [&](long long bb) -> long long {
    if constexpr (kRg) {
      return bb < args.rg.nb[0] ? args.rg.first[0] + bb * EB
                                : args.rg.first[1] + (bb - args.rg.nb[0]) * EB;
    } else {
      return bb * EB;
    }
  };
  auto batch_elems = [&](long long bb) -> long long {
    long long end;
    if constexpr (kRg)
      end = bb < args.rg.nb[0] ? args.rg.first[0] + args.rg.count[0]
                               : args.rg.first[1] + args.rg.count[1];
    else
      end = a.nelem;
    const long long e0 = batch_first(bb);
    return (end - e0 < EB) ? (end - e0) : EB;
  };
  auto batch_words = [&](long long bb) { return batch_elems(bb) * P; };
  auto issue_stage = [&](long long bb) {
    const long long e0 = batch_first(bb);
    const uint32_t bytes = static_cast<uint32_t>(batch_words(bb) * 4) & ~15u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(bar, kStaged * bytes);
#pragma unroll
    for (int q = 0; q < kNumPointArrays; ++q)
      bulk_g2s_hint(stage + size_t(q) * EP, a.m[q] + e0 * P, bytes, bar, pol_stream);
    if (!ASM) {
#pragma unroll
      for (int c = 0; c < 3; ++c)
        bulk_g2s_hint(stage + size_t(kNumPointArrays + c) * EP, a.u[c] + e0 * P, bytes, bar,
                      pol_stream);
    }
  };
  auto prefetch_batch = [&](long long bb) {
    if (kRg || bb >= nbatch) return;  // ticketed batches are not known ahead
    const long long e0 = batch_first(bb);
    const uint32_t bytes = static_cast<uint32_t>(batch_words(bb) * 4);
#pragma unroll
    for (int q = 0; q < kNumPointArrays; ++q) l2_prefetch_bulk(a.m[q] + e0 * P, bytes);
    if (ASM)
      l2_prefetch_bulk(a.ibool + e0 * P, bytes);
    else
#pragma unroll
      for (int c = 0; c < 3; ++c) l2_prefetch_bulk(a.u[c] + e0 * P, bytes);
  };

  // ticketed batches: thread 0 draws the next ticket and leaves it here
  long long* next_ticket = reinterpret_cast<long long*>(smem_raw + 64);
  if (tid == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (kRg) *next_ticket = static_cast<long long>(atomicAdd(args.rg.ticket, 1ull));
  }
  __syncthreads();
  const long long b0 = kRg ? *next_ticket : static_cast<long long>(blockIdx.x);
  if (tid == 0 && b0 < nbatch) {
    issue_stage(b0);
    prefetch_batch(b0 + G);
  }

  const float wi = a.ops.w[rb];
  const float wj = a.ops.w[ra];
  const float wij = wi * wj;
  uint32_t parity = 0;

  // gather pipeline registers: ibool and u of the NEXT batch to run
  int node_n[N];
  float uc_n[3][N];
  auto gather = [&](long long bb) {
    const bool v = (bb < nbatch) && (le < batch_elems(bb));
    const long long e = v ? batch_first(bb) + le : 0;
    const long long base = e * P + ab;
#pragma unroll
    for (int k = 0; k < N; ++k) node_n[k] = v ? __ldg(a.ibool + base + k * NN) : 0;
    if constexpr (IL) {
      const float4* u4 = reinterpret_cast<const float4*>(a.u[0]);
#pragma unroll
      for (int k = 0; k < N; ++k) {
        const float4 x = v ? __ldg(u4 + node_n[k]) : make_float4(0.f, 0.f, 0.f, 0.f);
        uc_n[0][k] = x.x;
        uc_n[1][k] = x.y;
        uc_n[2][k] = x.z;
      }
    } else {
#pragma unroll
      for (int k = 0; k < N; ++k)
#pragma unroll
        for (int c = 0; c < 3; ++c) uc_n[c][k] = v ? __ldg(a.u[c] + node_n[k]) : 0.f;
    }
  };
  if (ASM) gather(b0);

  for (long long b = b0, bnext = 0; b < nbatch; b = bnext) {
    if (tid == 0) prefetch_batch(b + 2 * G);
    const long long e0 = batch_first(b);
    const long long e = e0 + le;
    const bool valid = le < batch_elems(b);

    int node[N];
#pragma unroll
    for (int k = 0; k < N; ++k) node[k] = ASM ? node_n[k] : 0;
    // Wait for this batch's staged arrays (bounded; on a timeout every thread
    // leaves together after the copies have landed or the second wait ends).
    const bool ok = mbar_wait_bounded(bar, parity, kMbarMaxPolls);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicExch(&g_to_device_status, int(TO_ERR_TIMEOUT));
      mbar_wait_bounded(bar, parity, kMbarMaxPolls);
      return;
    }
    parity ^= 1u;
    {
      // tail of the launch: words past the last 16-byte boundary of each run
      const long long words = batch_words(b);
      const long long bw = ((words * 4) & ~15ll) / 4;
      if (bw < words) {
        for (int t = tid; t < kStaged * 4; t += NT) {
          const int q = t >> 2;
          const long long x = bw + (t & 3);
          if (x < words)
            stage[size_t(q) * EP + x] =
                q < kNumPointArrays ? a.m[q][e0 * P + x] : a.u[q - kNumPointArrays][e0 * P + x];
        }
        __syncthreads();
      }
    }

    // ---- A: column u -> UX, UE; gamma-gradients in registers ----
    float dgm[3][N];
    {
      float uc[3][N];
#pragma unroll
      for (int k = 0; k < N; ++k)
#pragma unroll
        for (int c = 0; c < 3; ++c)
          uc[c][k] = ASM ? uc_n[c][k]
                         : (valid ? stage[size_t(kNumPointArrays + c) * EP + spt + k * NN] : 0.f);
#pragma unroll
      for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int k = 0; k < N; ++k) {
          RX[c * CX + k * SKX + tid] = uc[c][k];
          RE[c * CE + k * SKE + tid] = uc[c][k];
        }
      if constexpr (kPk) {
#pragma unroll
        for (int k = 0; k < N; ++k) {
          float2 s01 = make_float2(0.f, 0.f);
          float s2 = 0.f;
#pragma unroll
          for (int p = 0; p < N; ++p) {
            s01 = __ffma2_rn(args.H2[k][p], make_float2(uc[0][p], uc[1][p]), s01);
            s2 = fmaf(a.ops.H[k][p], uc[2][p], s2);
          }
          dgm[0][k] = s01.x;
          dgm[1][k] = s01.y;
          dgm[2][k] = s2;
        }
      } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
          for (int k = 0; k < N; ++k) {
            float s = 0.f;
#pragma unroll
            for (int p = 0; p < N; ++p) s = fmaf(a.ops.H[k][p], uc[c][p], s);
            dgm[c][k] = s;
          }
      }
    }
    __syncthreads();

    // ---- B1: line owners -> xi- and eta-gradients of their rows ----
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float v[N], w[N];
#pragma unroll
      for (int p = 0; p < N; ++p) {
        v[p] = RX[c * CX + lx + p];
        w[p] = RE[c * CE + ly + p * N];
      }
#pragma unroll
      for (int o = 0; o < N; ++o) {
        float sx = 0.f, se = 0.f;
        if constexpr (kPk) {
          float2 s = make_float2(0.f, 0.f);
#pragma unroll
          for (int p = 0; p < N; ++p) s = __ffma2_rn(args.H2[o][p], make_float2(v[p], w[p]), s);
          sx = s.x;
          se = s.y;
        } else {
#pragma unroll
          for (int p = 0; p < N; ++p) {
            sx = fmaf(a.ops.H[o][p], v[p], sx);
            se = fmaf(a.ops.H[o][p], w[p], se);
          }
        }
        RDX[c * CX + lx + o] = sx;
        RDE[c * CE + ly + o * N] = se;
      }
    }
    __syncthreads();

    // ---- B2: column Integrand9 (k-pairs in packed lanes) -> FX, FE ----
    float Fg[3][N];
    {
      // the staged geometry of point k of this column: J[r][d], jac, l2m, mu
      auto geom = [&](int k, float (&J)[3][3], float& jac, float& l2m, float& mu) {
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
          for (int d = 0; d < 3; ++d) J[r][d] = stage[size_t(kXIX + 3 * r + d) * EP + spt + k * NN];
        jac = stage[size_t(kJAC) * EP + spt + k * NN];
        l2m = stage[size_t(kL2M) * EP + spt + k * NN];
        mu = stage[size_t(kMU) * EP + spt + k * NN];
      };
      auto point_pair = [&](int k0, int k1) {
        V2<float> dxi[3], det[3], dg[3], J[3][3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          dxi[c] = mk2(RDX[c * CX + k0 * SKX + tid], RDX[c * CX + k1 * SKX + tid]);
          det[c] = mk2(RDE[c * CE + k0 * SKE + tid], RDE[c * CE + k1 * SKE + tid]);
          dg[c] = mk2(dgm[c][k0], dgm[c][k1]);
        }
        float J0[3][3], J1[3][3], jac0, jac1, l2m0, l2m1, mu0, mu1;
        geom(k0, J0, jac0, l2m0, mu0);
        geom(k1, J1, jac1, l2m1, mu1);
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
          for (int d = 0; d < 3; ++d) J[r][d] = mk2(J0[r][d], J1[r][d]);
        V2<float> F[3][3];
        integrand9_lanes<V2<float>, float>(dxi, det, dg, J, mk2(l2m0, l2m1), mk2(mu0, mu1),
                                           mk2(jac0, jac1), F);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          RX[c * CX + k0 * SKX + tid] = F[0][c].v.x;
          RX[c * CX + k1 * SKX + tid] = F[0][c].v.y;
          RE[c * CE + k0 * SKE + tid] = F[1][c].v.x;
          RE[c * CE + k1 * SKE + tid] = F[1][c].v.y;
          Fg[c][k0] = F[2][c].v.x;
          Fg[c][k1] = F[2][c].v.y;
        }
      };
      point_pair(0, 1);
      point_pair(2, 3);
      {
        constexpr int k = N - 1;
        float dxi[3], det[3], dg[3], J[3][3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          dxi[c] = RDX[c * CX + k * SKX + tid];
          det[c] = RDE[c * CE + k * SKE + tid];
          dg[c] = dgm[c][k];
        }
        float jac, l2m, mu;
        geom(k, J, jac, l2m, mu);
        float F[3][3];
        integrand9_lanes<float, float>(dxi, det, dg, J, l2m, mu, jac, F);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          RX[c * CX + k * SKX + tid] = F[0][c];
          RE[c * CE + k * SKE + tid] = F[1][c];
          Fg[c][k] = F[2][c];
        }
      }
    }
    if (kRg && tid == 0) *next_ticket = static_cast<long long>(atomicAdd(args.rg.ticket, 1ull));
    __syncthreads();  // stage reads and flux writes of this batch are done

    bnext = kRg ? *next_ticket : b + G;
    if (tid == 0 && bnext < nbatch) issue_stage(bnext);
    if (ASM) gather(bnext);  // lands while the divergences run

    // ---- C1: line owners -> xi- and eta-divergences of their rows ----
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float v[N], w[N];
#pragma unroll
      for (int q = 0; q < N; ++q) {
        v[q] = RX[c * CX + lx + q];
        w[q] = RE[c * CE + ly + q * N];
      }
#pragma unroll
      for (int o = 0; o < N; ++o) {
        float sx = 0.f, se = 0.f;
        if constexpr (kPk) {
          float2 s = make_float2(0.f, 0.f);
#pragma unroll
          for (int q = 0; q < N; ++q) s = __ffma2_rn(args.Hw2[q][o], make_float2(v[q], w[q]), s);
          sx = s.x;
          se = s.y;
        } else {
#pragma unroll
          for (int q = 0; q < N; ++q) {
            sx = fmaf(a.ops.Hw[q][o], v[q], sx);
            se = fmaf(a.ops.Hw[q][o], w[q], se);
          }
        }
        RDX[c * CX + lx + o] = sx;
        RDE[c * CE + ly + o * N] = se;
      }
    }
    __syncthreads();

    // ---- C2: column WeightedSum -> scatter-add / store ----
    {
      const long long obase = e * P + ab;
#pragma unroll
      for (int k = 0; k < N; ++k) {
        const float wjk = wj * a.ops.w[k], wik = wi * a.ops.w[k];
        float fc[3];
        float gg[3];
        if constexpr (kPk) {
          float2 g01 = make_float2(0.f, 0.f);
          float g2 = 0.f;
#pragma unroll
          for (int q = 0; q < N; ++q) {
            g01 = __ffma2_rn(args.Hw2[q][k], make_float2(Fg[0][q], Fg[1][q]), g01);
            g2 = fmaf(a.ops.Hw[q][k], Fg[2][q], g2);
          }
          gg[0] = g01.x;
          gg[1] = g01.y;
          gg[2] = g2;
        } else {
#pragma unroll
          for (int c = 0; c < 3; ++c) {
            float g = 0.f;
#pragma unroll
            for (int q = 0; q < N; ++q) g = fmaf(a.ops.Hw[q][k], Fg[c][q], g);
            gg[c] = g;
          }
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          const float g = gg[c];
          const float tx = RDX[c * CX + k * SKX + tid];
          const float te = RDE[c * CE + k * SKE + tid];
          fc[c] = fmaf(wij, g, fmaf(wik, te, wjk * tx));
        }
        bool issue = valid;
        if constexpr (kAgg) {
          // x-face partners: lane + 21 holds (le+1, j, 0) when this is (le, j, 4);
          // they are combined only when ibool gives them the same node (any mesh)
          const int lane = tid & 31;
          const unsigned mask = __activemask();
          float pv[3];
#pragma unroll
          for (int c = 0; c < 3; ++c) pv[c] = __shfl_down_sync(mask, fc[c], 21);
          const int pnode = __shfl_down_sync(mask, node[k], 21);  // partner's node
          const int onode = __shfl_up_sync(mask, node[k], 21);    // owner's node
          const bool owner = rb == N - 1 && lane + 21 < 32 && tid + 21 < NT &&
                             le + 1 < batch_elems(b) && pnode == node[k];
          if (owner) {
#pragma unroll
            for (int c = 0; c < 3; ++c) fc[c] += pv[c];
          }
          if (rb == 0 && le >= 1 && lane >= 21 && onode == node[k])
            issue = false;  // the owner (lane - 21) adds it
        }
        if (issue) {
          if (ASM && IL) {
            atomicAdd(reinterpret_cast<float4*>(a.f[0]) + node[k],
                      make_float4(fc[0], fc[1], fc[2], 0.f));
          } else {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
              if (ASM)
                atomicAdd(a.f[c] + node[k], fc[c]);
              else
                a.f[c][obase + k * NN] = fc[c];
            }
          }
        }
      }
    }
  }
}

}  // namespace to_b200
