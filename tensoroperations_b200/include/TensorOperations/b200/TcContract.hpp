// TcContract.hpp -- a graph that is one large fp32 contraction of two inputs,
// run as a dense GEMM on the tensor cores (tcgen05) instead of the level
// evaluator.
//
// The reference evaluates such a contraction with its team GEMM over permuted
// operand tiles (include/TensorOperations/Evaluator/Team.hpp:318-927,
// Permute.hpp:127-228).  Here, when the DAG (or the tree lowered to it) is a
// single contraction node whose operands are both input nodes, the value type
// is float and the problem is big enough to fill the tensor-core tiles
// (M = prod of A's free extents >= 128, N = prod of B's free extents >= 128,
// K = prod of the contracted extents >= 32), execute() runs three kernels:
//   pack      A -> [Mp][Kp] and B -> [Np][Kp], K-major (rows in the canonical
//             free-label order, columns in the node's contracted-label order),
//             each value split into TF32 hi and lo parts (+ the input's hook),
//             zero padding to multiples of 128 / 256 / 32;
//   GEMM      to_gemm_tf32x3 (C ABI): three TF32 products per K step
//             accumulated in TMEM, drained in fp32;
//   unpack    C -> the output view in the node's DECLARED order (+ the
//             contraction's hook at its global coordinates).
// The tile bundle the caller gave (a hint for the level evaluator) is not
// needed.  The packed operands live in one device buffer this header keeps
// for the process and grows on demand (the only allocation on this route).
// TO_FRONTEND_TENSOR_CORES=0 in the environment keeps every graph on the level
// evaluator (used by the tests to compare the two).
#pragma once

#include <array>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <TensorOperations/b200/Dag.hpp>

namespace TensorOperations {
namespace b200 {

// Is this DAG (node list type) one contraction of two inputs, in float?
template <class NodesT, class V>
constexpr bool tc_candidate() {
  if constexpr (tuple_size_v<NodesT> != 1 || !std::is_same_v<V, float>) {
    return false;
  } else {
    using N = tuple_element_t<0, NodesT>;
    if constexpr (!dag_is_contraction_v<N>)
      return false;
    else
      return dag_is_input_v<typename N::node_a_type> && dag_is_input_v<typename N::node_b_type> &&
             N::NumContracted > 0 && N::FreeA > 0 && N::FreeB > 0;
  }
}

inline bool tc_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("TO_FRONTEND_TENSOR_CORES");
    return !(e && std::strcmp(e, "0") == 0);
  }();
  return on;
}

// Product of an input's extents along labels `labs`.
template <class In, std::size_t NL>
long long tc_extent_product(const In& in, const std::array<int32_t, NL>& labs) {
  constexpr auto lab = to_array<typename In::modes_seq>();
  long long p = 1;
  for (std::size_t i = 0; i < NL; ++i) p *= static_cast<long long>(in.handle.tensor.extent(index_of(lab, labs[i])));
  return p;
}

// The same over any node's shape (an input's or a nested node's storage order).
template <class Nd, std::size_t NL>
long long tc_shape_product(const Nd& nd, const std::array<int32_t, NL>& labs) {
  constexpr auto lab = to_array<typename Nd::modes_seq>();
  const auto sh = nd.shape();
  long long p = 1;
  for (std::size_t i = 0; i < NL; ++i) p *= static_cast<long long>(sh[index_of(lab, labs[i])]);
  return p;
}

// True when fp32 contraction `node` is large enough for the tensor-core GEMM
// (M, N >= 128, K >= 32).  A tree whose root qualifies evaluates its nested
// operands first, so that the root can take that path.
template <class Node>
bool tc_sized(const Node& node) {
  if constexpr (!std::is_same_v<typename Node::value_type, float> || Node::NumContracted == 0 ||
                Node::FreeA == 0 || Node::FreeB == 0) {
    return false;
  } else {
    return tc_enabled() && tc_shape_product(node.node_a, Node::freeA) >= 128 &&
           tc_shape_product(node.node_b, Node::freeB) >= 128 &&
           tc_shape_product(node.node_a, Node::contracted) >= 32;
  }
}

// True when a fusible tree should still run in steps so that its root takes
// the tensor-core GEMM: the root is tc_sized and has at least 2^27 multiply-
// adds.  Measured on the reference's multilevel chain (root M = N = n, K = 32):
// at n = 1024 the fused launch is faster (2.8 vs 1.8 TFLOP/s; three small
// launches), at 2048 and 4096 the steps are (5.5 vs 4.7, 8.9 vs 5.7).
template <class Node>
bool tc_steps_pay(const Node& node) {
  if (!tc_sized(node)) return false;
  return tc_shape_product(node.node_a, Node::freeA) * tc_shape_product(node.node_b, Node::freeB) *
             tc_shape_product(node.node_a, Node::contracted) >=
         (1LL << 27);
}

#if defined(__CUDACC__)

// Decode `idx` row-major over labels `labs` (last fastest), extents read from
// the input's view; writes the coordinate of each label into c[].
template <class In, class LabSeq>
__device__ __forceinline__ void tc_decode(const In& in, long long idx, long long* c) {
  constexpr auto lab = to_array<typename In::modes_seq>();
  constexpr auto Labs = to_array<LabSeq>();
  constexpr int n = static_cast<int>(Labs.size());
  static_for<n>([&](auto ic) {
    constexpr int i = n - 1 - decltype(ic)::value;
    constexpr int d = index_of(lab, Labs[i]);
    const long long e = static_cast<long long>(in.handle.tensor.extent(d));
    c[i] = idx % e;
    idx /= e;
  });
}

// The operand on side 0 (A: rows = freeA) or 1 (B: rows = freeB); columns
// are the contracted labels in the node's order.  (A kernel's template
// arguments are the node type and the side only: the stub generator cannot
// spell class-type constant arguments.)
template <class Node, int Side>
struct tc_side {
  using In = typename Node::node_a_type;
  using Rows = array_seq_t<Node::freeA>;
};
template <class Node>
struct tc_side<Node, 1> {
  using In = typename Node::node_b_type;
  using Rows = array_seq_t<Node::freeB>;
};

template <class Node, int Side>
__global__ void tc_pack_kernel(const typename tc_side<Node, Side>::In in, float* __restrict__ hi,
                               float* __restrict__ lo, long long rows, long long cols, long long Kp,
                               long long total) {
  using In = typename tc_side<Node, Side>::In;
  using RowSeq = typename tc_side<Node, Side>::Rows;
  using ColSeq = array_seq_t<Node::contracted>;
  constexpr auto lab = to_array<typename In::modes_seq>();
  constexpr auto RowLabs = to_array<RowSeq>();
  constexpr auto ColLabs = to_array<ColSeq>();
  constexpr int R = In::Rank;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long r = t / Kp, k = t - r * Kp;
    float v = 0.f;
    if (r < rows && k < cols) {
      long long rc[RowLabs.size() > 0 ? RowLabs.size() : 1];
      long long kc[ColLabs.size() > 0 ? ColLabs.size() : 1];
      tc_decode<In, RowSeq>(in, r, rc);
      tc_decode<In, ColSeq>(in, k, kc);
      long long g[R > 0 ? R : 1];
      static_for<R>([&](auto dc) {
        constexpr int d = decltype(dc)::value;
        constexpr int ri = index_of(RowLabs, lab[d]);
        constexpr int ci = index_of(ColLabs, lab[d]);
        if constexpr (ri >= 0)
          g[d] = rc[ri];
        else
          g[d] = kc[ci];
      });
      v = static_cast<float>(view_at(in.handle.tensor, g, std::make_index_sequence<R>{}));
      if constexpr (!std::is_same_v<decltype(in.hook_op), NoHook>)
        call_hook(in.hook_op, g, v, std::make_index_sequence<R>{});
    }
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
    const float hv = __uint_as_float(h);
    hi[t] = hv;
    lo[t] = v - hv;
  }
}

// One thread per output element, in the output view's storage order (so the
// writes are coalesced whatever the declared order); it reads its value from
// the packed C.
template <class Node, class View>
__global__ void tc_unpack_kernel(const Node node, const View out, const float* __restrict__ C,
                                 long long ldc) {
  using A = typename Node::node_a_type;
  using B = typename Node::node_b_type;
  constexpr int R = Node::Rank;
  constexpr auto perm = label_positions<typename Node::decl_seq, typename Node::canon_seq>();
  constexpr bool left = std::is_same_v<typename View::array_layout, Kokkos::LayoutLeft>;
  // canonical extents (freeA ++ freeB) from the operands, and the declared ones
  long long cext[R > 0 ? R : 1];
  {
    constexpr auto la = to_array<typename A::modes_seq>();
    constexpr auto lb = to_array<typename B::modes_seq>();
    constexpr auto fa = Node::freeA;
    constexpr auto fb = Node::freeB;
    static_for<Node::FreeA>([&](auto dc) {
      constexpr int d = decltype(dc)::value;
      cext[d] = static_cast<long long>(node.node_a.handle.tensor.extent(index_of(la, fa[d])));
    });
    static_for<Node::FreeB>([&](auto dc) {
      constexpr int d = decltype(dc)::value;
      cext[Node::FreeA + d] = static_cast<long long>(node.node_b.handle.tensor.extent(index_of(lb, fb[d])));
    });
  }
  long long dext[R > 0 ? R : 1];
  long long total = 1;
  for (int d = 0; d < R; ++d) {
    const long long e = static_cast<long long>(out.extent(d));
    dext[d] = cext[perm[d]] < e ? cext[perm[d]] : e;  // write what fits
    total *= dext[d];
  }
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    long long g[R > 0 ? R : 1];
    long long x = t;
    if constexpr (left) {
      for (int d = 0; d < R; ++d) {
        g[d] = x % dext[d];
        x /= dext[d];
      }
    } else {
      for (int d = R - 1; d >= 0; --d) {
        g[d] = x % dext[d];
        x /= dext[d];
      }
    }
    long long cc[R > 0 ? R : 1];
    for (int d = 0; d < R; ++d) cc[perm[d]] = g[d];
    long long m = 0, n = 0;
    for (int d = 0; d < Node::FreeA; ++d) m = m * cext[d] + cc[d];
    for (int d = Node::FreeA; d < R; ++d) n = n * cext[d] + cc[d];
    float v = C[m * ldc + n];
    if constexpr (!std::is_same_v<typename Node::hook_type, NoHook>)
      call_hook(node.hook_op, g, v, std::make_index_sequence<R>{});
    view_at(out, g, std::make_index_sequence<R>{}) = v;
  }
}

// The packed operands and the GEMM output: one buffer per CUDA device, kept
// for the process and grown when a larger contraction needs it.  The current
// device picks the buffer, so a process that runs the frontend on several GPUs
// never hands one device's memory to another.  Reuse is stream-ordered: the
// frontend launches every evaluation on the default stream.
inline float* tc_workspace(std::size_t floats) {
  struct Slot {
    float* ptr = nullptr;
    std::size_t cap = 0;
  };
  static std::mutex mu;
  static Slot slots[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    throw LevelGraphError(TO_ERR_CUDA, "tensor-core contraction: no usable current device");
  }
  std::lock_guard<std::mutex> lock(mu);
  Slot& s = slots[dev];
  if (floats > s.cap) {
    if (s.ptr) cudaFree(s.ptr);
    s.ptr = nullptr;
    s.cap = 0;
    if (cudaMalloc(&s.ptr, floats * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      throw LevelGraphError(TO_ERR_CUDA, "tensor-core contraction: workspace allocation failed");
    }
    s.cap = floats;
  }
  return s.ptr;
}

// Runs the contraction on the tensor cores when it is large enough; returns
// the number of GEMM tiles, or -1 to leave it to the level evaluator.
template <class Node, class View>
int tc_try_contract(const Node& node, const View& out) {
  if (!tc_enabled()) return -1;
  const long long M = tc_extent_product(node.node_a, Node::freeA);
  const long long Nn = tc_extent_product(node.node_b, Node::freeB);
  const long long K = tc_extent_product(node.node_a, Node::contracted);
  if (M < 128 || Nn < 128 || K < 32) return -1;
  if (tc_extent_product(node.node_b, Node::contracted) != K)
    throw LevelGraphError(TO_ERR_INVALID_ARGUMENT,
                          "contraction: the contracted extents of A and B differ");
  const long long Mp = (M + 127) / 128 * 128, Np = (Nn + 255) / 256 * 256, Kp = (K + 31) / 32 * 32;
  if (Mp / 128 > 65535) return -1;
  float* ws = tc_workspace(static_cast<std::size_t>(2 * Mp * Kp + 2 * Np * Kp + Mp * Np));
  float *Ahi = ws, *Alo = Ahi + Mp * Kp, *Bhi = Alo + Mp * Kp, *Blo = Bhi + Np * Kp, *C = Blo + Np * Kp;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned blocks = static_cast<unsigned>(sms > 0 ? 8 * sms : 1024);
  tc_pack_kernel<Node, 0><<<blocks, 256>>>(node.node_a, Ahi, Alo, M, K, Kp, Mp * Kp);
  tc_pack_kernel<Node, 1><<<blocks, 256>>>(node.node_b, Bhi, Blo, Nn, K, Kp, Np * Kp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    throw LevelGraphError(TO_ERR_CUDA, std::string("tensor-core contraction: pack: ") + cudaGetErrorString(e));
  if (int st = to_gemm_tf32x3(Mp, Np, Kp, Ahi, Alo, Bhi, Blo, C, nullptr))
    throw LevelGraphError(st, to_last_error());
  tc_unpack_kernel<Node, View><<<blocks, 256>>>(node, out, C, Np);
  e = cudaGetLastError();
  if (e != cudaSuccess)
    throw LevelGraphError(TO_ERR_CUDA, std::string("tensor-core contraction: unpack: ") + cudaGetErrorString(e));
  return static_cast<int>((Mp / 128) * (Np / 256));
}

#else

template <class Node, class View>
int tc_try_contract(const Node&, const View&) {
  return -1;
}

#endif

}  // namespace b200
}  // namespace TensorOperations
