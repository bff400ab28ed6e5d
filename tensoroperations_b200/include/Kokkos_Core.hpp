// Kokkos_Core.hpp -- the subset of the Kokkos API that TensorOperations
// programs name, implemented directly on the CUDA runtime (device side, when
// the translation unit is compiled by nvcc) and on plain C++ (host side).
//
// Kokkos itself is not a dependency of this project.  This header exists so
// that a program written against the reference library -- which includes
// <Kokkos_Core.hpp> and declares its tensors as Kokkos::View -- compiles
// unchanged against the B200 frontend.  What it provides:
//
//   Views       View<DataType, Props...> with LayoutRight or LayoutLeft, mixed static and
//               dynamic extents ("float*[5][5][5]", "float****"), HostSpace /
//               CudaSpace / team-scratch memory, managed (reference counted,
//               zero-initialised) or unmanaged; create_mirror_view[_and_copy],
//               deep_copy, host_mirror_type.
//   Execution   Cuda (default when compiled by nvcc) and Serial spaces;
//               parallel_for over RangePolicy, MDRangePolicy<Rank<N>> and
//               TeamPolicy; TeamVectorRange /
//               TeamThreadRange / ThreadVectorRange; team_barrier, team_scratch;
//               fence, Timer, initialize / finalize, abort, Array.
//
// A team is a CUDA thread block, a league rank a block index, team scratch the
// block's dynamic shared memory.  Device-side abort() prints and does not trap.
#pragma once

#include <atomic>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <string>
#include <type_traits>
#include <utility>

#if defined(__CUDACC__)
#include <cuda_runtime.h>
#define KOKKOS_ENABLE_CUDA 1
#define KOKKOS_FUNCTION __host__ __device__
#define KOKKOS_INLINE_FUNCTION __host__ __device__ inline
#define KOKKOS_FORCEINLINE_FUNCTION __host__ __device__ __forceinline__
#define KOKKOS_LAMBDA [=] __host__ __device__
#define KOKKOS_CLASS_LAMBDA [=, *this] __host__ __device__
#else
#define KOKKOS_FUNCTION
#define KOKKOS_INLINE_FUNCTION inline
#define KOKKOS_FORCEINLINE_FUNCTION inline
#define KOKKOS_LAMBDA [=]
#define KOKKOS_CLASS_LAMBDA [=, *this]
#endif

#if defined(__CUDA_ARCH__)
#define TO_KOKKOS_DEVICE_PASS 1
#endif

namespace Kokkos {

// ---------------------------------------------------------------------------
// Spaces
// ---------------------------------------------------------------------------
struct Serial;
struct HostSpace {
  using memory_space = HostSpace;
  using execution_space = Serial;
  static constexpr const char* name() { return "HostSpace"; }
};

template <class ExecSpace>
struct ScratchMemorySpace;

struct Serial {
  using execution_space = Serial;
  using memory_space = HostSpace;
  using scratch_memory_space = ScratchMemorySpace<Serial>;
  using size_type = std::size_t;
  static constexpr const char* name() { return "Serial"; }
  void fence(const char* = nullptr) const {}
  static int concurrency() { return 1; }
};

#ifdef KOKKOS_ENABLE_CUDA
struct Cuda;
struct CudaSpace {
  using memory_space = CudaSpace;
  using execution_space = Cuda;
  static constexpr const char* name() { return "CudaSpace"; }
};
struct Cuda {
  using execution_space = Cuda;
  using memory_space = CudaSpace;
  using scratch_memory_space = ScratchMemorySpace<Cuda>;
  using size_type = std::size_t;
  static constexpr const char* name() { return "Cuda"; }
  void fence(const char* = nullptr) const;
  static int concurrency() { return 148 * 2048; }
};
using DefaultExecutionSpace = Cuda;
#else
using DefaultExecutionSpace = Serial;
#endif
using DefaultHostExecutionSpace = Serial;

template <class ExecSpace, class MemSpace>
struct SpaceAccessibility {
  static constexpr bool accessible =
      std::is_same_v<typename ExecSpace::memory_space, HostSpace> ==
      std::is_same_v<typename MemSpace::memory_space, HostSpace>;
  static constexpr bool assignable = accessible;
};

struct LayoutRight {};
struct LayoutLeft {};
struct Unmanaged {};
template <class... T>
struct MemoryTraits {};
using MemoryUnmanaged = MemoryTraits<Unmanaged>;

// ---------------------------------------------------------------------------
// Array
// ---------------------------------------------------------------------------
template <class T, std::size_t N>
struct Array {
  T m_data[N > 0 ? N : 1];
  using value_type = T;
  KOKKOS_INLINE_FUNCTION T& operator[](std::size_t i) { return m_data[i]; }
  KOKKOS_INLINE_FUNCTION const T& operator[](std::size_t i) const { return m_data[i]; }
  KOKKOS_INLINE_FUNCTION static constexpr std::size_t size() { return N; }
  KOKKOS_INLINE_FUNCTION T* data() { return m_data; }
  KOKKOS_INLINE_FUNCTION const T* data() const { return m_data; }
};

// ---------------------------------------------------------------------------
// Host services
// ---------------------------------------------------------------------------
namespace Impl {
inline bool& initialized_flag() {
  static bool f = false;
  return f;
}
}  // namespace Impl

namespace Impl {
// Status word of team scratch overflows: set by a team whose scratch requests
// go past the size set on its policy (that team stops before it uses any of
// the memory), read and cleared by fence() / finalize(), which then abort as
// Kokkos::abort would.  CUDA builds keep it in mapped pinned host memory, so
// a kernel writes it and the host reads it after synchronising; without
// mapped memory the word is null and only the device message remains.
inline int* scratch_status() {
#ifdef KOKKOS_ENABLE_CUDA
  static int* word = [] {
    void* h = nullptr;
    if (cudaHostAlloc(&h, sizeof(int), cudaHostAllocMapped) != cudaSuccess) {
      cudaGetLastError();
      return static_cast<int*>(nullptr);
    }
    *static_cast<volatile int*>(h) = 0;
    return static_cast<int*>(h);
  }();
  return word;
#else
  static int word = 0;
  return &word;
#endif
}

// Returns and clears the status word (1 after an overflow, else 0).
inline int take_scratch_status() {
  int* w = scratch_status();
  if (!w) return 0;
  const int v = *static_cast<volatile int*>(w);
  *static_cast<volatile int*>(w) = 0;
  return v;
}

inline void check_scratch_status(const char* where) {
  if (take_scratch_status()) {
    std::fprintf(stderr,
                 "Kokkos::%s: a team scratch request exceeded the size set on its policy; "
                 "the team stopped before using the memory, so results are incomplete\n",
                 where);
    std::abort();
  }
}

// Thrown on the host to stop a team whose scratch request overflowed.
struct ScratchOverflow {};
}  // namespace Impl

inline void initialize() {
#ifdef KOKKOS_ENABLE_CUDA
  cudaFree(nullptr);  // create the primary context
#endif
  Impl::initialized_flag() = true;
}
inline void initialize(int& argc, char* argv[]) {
  (void)argc;
  (void)argv;
#ifdef KOKKOS_ENABLE_CUDA
  cudaFree(nullptr);
#endif
  Impl::initialized_flag() = true;
}
inline void finalize() {
#ifdef KOKKOS_ENABLE_CUDA
  cudaDeviceSynchronize();
#endif
  Impl::initialized_flag() = false;
  Impl::check_scratch_status("finalize");
}
inline bool is_initialized() { return Impl::initialized_flag(); }


inline void fence(const char* = nullptr) {
#ifdef KOKKOS_ENABLE_CUDA
  cudaDeviceSynchronize();
#endif
  Impl::check_scratch_status("fence");
}
#ifdef KOKKOS_ENABLE_CUDA
inline void Cuda::fence(const char*) const {
  cudaDeviceSynchronize();
  Impl::check_scratch_status("Cuda::fence");
}
#endif

KOKKOS_INLINE_FUNCTION void abort(const char* msg) {
#if defined(TO_KOKKOS_DEVICE_PASS)
  printf("Kokkos::abort (device): %s\n", msg);
#else
  std::fprintf(stderr, "Kokkos::abort: %s\n", msg);
  std::abort();
#endif
}

class Timer {
  std::chrono::steady_clock::time_point t0_ = std::chrono::steady_clock::now();

 public:
  void reset() { t0_ = std::chrono::steady_clock::now(); }
  double seconds() const {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0_).count();
  }
};

// ---------------------------------------------------------------------------
// Team scratch: a per-thread bump allocator over the block's shared memory.
// Every thread of a team constructs its scratch Views in the same order, so
// every copy of the cursor hands out the same addresses.
// ---------------------------------------------------------------------------
template <class ExecSpace>
struct ScratchMemorySpace {
  using memory_space = ScratchMemorySpace<ExecSpace>;
  using execution_space = ExecSpace;
  static constexpr std::size_t align = 16;
  char* base_ = nullptr;
  std::size_t size_ = 0;
  mutable std::size_t used_ = 0;
  int* status_ = nullptr;  // Impl::scratch_status(), or null

  ScratchMemorySpace() = default;
  KOKKOS_INLINE_FUNCTION ScratchMemorySpace(void* base, std::size_t size, int* status = nullptr)
      : base_(static_cast<char*>(base)), size_(size), used_(0), status_(status) {}
  // A request past the size set on the policy never gets a pointer: the
  // status word is set and the team stops right there -- on the device every
  // thread of the team exits (they all make the same requests in the same
  // order), on the host the team's functor is unwound -- so no view of an
  // under-sized policy reaches outside the team's memory.  fence() then
  // reports the overflow and aborts.
  KOKKOS_INLINE_FUNCTION void* get_shmem(std::size_t bytes) const {
    const std::size_t b = (bytes + align - 1) & ~(align - 1);
    if (used_ + b > size_) {
#if defined(TO_KOKKOS_DEVICE_PASS)
      if (status_) {
        *static_cast<volatile int*>(status_) = 1;
        __threadfence_system();
      }
      if (threadIdx.x == 0)
        printf("Kokkos: team scratch request of %llu bytes exceeds the %llu left of the size set "
               "on the policy; team %d stops\n",
               static_cast<unsigned long long>(b), static_cast<unsigned long long>(size_ - used_),
               static_cast<int>(blockIdx.x));
      asm volatile("exit;");
      return nullptr;  // not reached
#else
      if (status_) *status_ = 1;
      throw Impl::ScratchOverflow{};
#endif
    }
    void* p = base_ + used_;
    used_ += b;
    return p;
  }
  KOKKOS_INLINE_FUNCTION static std::size_t round(std::size_t bytes) {
    return (bytes + align - 1) & ~(align - 1);
  }
};

// ---------------------------------------------------------------------------
// View
// ---------------------------------------------------------------------------
namespace Impl {

template <class X>
struct PtrDepth {
  static constexpr int n = 0;
  using base = X;
};
template <class X>
struct PtrDepth<X*> {
  static constexpr int n = 1 + PtrDepth<X>::n;
  using base = typename PtrDepth<X>::base;
};

template <class DataType>
struct DataAnalysis {
  using no_arr = std::remove_all_extents_t<DataType>;
  static constexpr int rank_static = static_cast<int>(std::rank_v<DataType>);
  static constexpr int rank_dynamic = PtrDepth<no_arr>::n;
  static constexpr int rank = rank_dynamic + rank_static;
  using value_type = typename PtrDepth<no_arr>::base;

};

template <class T>
struct is_layout : std::bool_constant<std::is_same_v<T, LayoutRight> ||
                                      std::is_same_v<T, LayoutLeft>> {};
template <class T>
struct is_memory_traits : std::false_type {};
template <class... T>
struct is_memory_traits<MemoryTraits<T...>> : std::true_type {};

template <class T, class = void>
struct has_exec_space : std::false_type {};
template <class T>
struct has_exec_space<T, std::void_t<typename T::execution_space>> : std::true_type {};

// Memory space named by a View property, or void.
template <class P, class = void>
struct MemSpaceOf {
  using type = void;
};
template <class P>
struct MemSpaceOf<P, std::void_t<typename P::memory_space>> {
  using type = typename P::memory_space;
};

template <class... Props>
struct PropsAnalysis {
  template <class Acc, class... Rest>
  struct first_non_void {
    using type = Acc;
  };
  template <class Acc, class H, class... Rest>
  struct first_non_void<Acc, H, Rest...> {
    using type = typename first_non_void<std::conditional_t<std::is_void_v<Acc>, H, Acc>,
                                         Rest...>::type;
  };
  using named = typename first_non_void<void, typename MemSpaceOf<Props>::type...>::type;
  using memory_space =
      std::conditional_t<std::is_void_v<named>, DefaultExecutionSpace::memory_space, named>;
  static constexpr bool unmanaged = (is_memory_traits<Props>::value || ...);
  static constexpr bool layout_left = (std::is_same_v<Props, LayoutLeft> || ...);
};

template <class M>
struct is_scratch : std::false_type {};
template <class E>
struct is_scratch<ScratchMemorySpace<E>> : std::true_type {};

struct ControlBlock {
  std::atomic<int> refs{1};
  void* ptr = nullptr;
  bool device = false;
  std::string label;
};

inline void* alloc_bytes(std::size_t bytes, bool device, const char* label) {
  if (bytes == 0) bytes = 1;
  void* p = nullptr;
#ifdef KOKKOS_ENABLE_CUDA
  if (device) {
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
      std::fprintf(stderr, "Kokkos::View '%s': cudaMalloc(%zu) failed\n", label, bytes);
      std::abort();
    }
    cudaMemset(p, 0, bytes);
    return p;
  }
#else
  (void)device;
#endif
  p = std::calloc(1, bytes);
  if (!p) {
    std::fprintf(stderr, "Kokkos::View '%s': host allocation of %zu bytes failed\n", label,
                 bytes);
    std::abort();
  }
  return p;
}

inline void free_bytes(void* p, bool device) {
#ifdef KOKKOS_ENABLE_CUDA
  if (device) {
    cudaFree(p);
    return;
  }
#else
  (void)device;
#endif
  std::free(p);
}

}  // namespace Impl

template <class DataType, class... Props>
class View {
  using DA = Impl::DataAnalysis<DataType>;
  using PA = Impl::PropsAnalysis<Props...>;
  static constexpr bool kLeft = PA::layout_left;

 public:
  using data_type = DataType;
  using value_type = typename DA::value_type;
  using const_value_type = std::add_const_t<value_type>;
  using non_const_value_type = std::remove_const_t<value_type>;
  using pointer_type = value_type*;
  using reference_type = value_type&;
  using array_layout = std::conditional_t<kLeft, LayoutLeft, LayoutRight>;
  using memory_space = typename PA::memory_space;
  using execution_space = typename memory_space::execution_space;
  using device_type = View;
  using size_type = std::size_t;
  static constexpr int rank = DA::rank;
  static constexpr int rank_dynamic = DA::rank_dynamic;
  static constexpr bool is_scratch = Impl::is_scratch<memory_space>::value;
  static constexpr bool managed = !PA::unmanaged && !is_scratch;
  using non_const_data_type = std::remove_const_t<DataType>;
  using host_mirror_type =
      std::conditional_t<std::is_same_v<memory_space, HostSpace>, View<DataType, Props...>,
                         View<non_const_data_type, array_layout, HostSpace>>;
  using HostMirror = host_mirror_type;

 private:
  pointer_type data_ = nullptr;
  std::size_t dyn_[rank_dynamic > 0 ? rank_dynamic : 1] = {};
  Impl::ControlBlock* cb_ = nullptr;

  KOKKOS_INLINE_FUNCTION void retain() const {
#if !defined(TO_KOKKOS_DEVICE_PASS)
    if (cb_) cb_->refs.fetch_add(1, std::memory_order_relaxed);
#endif
  }
  KOKKOS_INLINE_FUNCTION void release() {
#if !defined(TO_KOKKOS_DEVICE_PASS)
    if (cb_ && cb_->refs.fetch_sub(1, std::memory_order_acq_rel) == 1) {
      Impl::free_bytes(cb_->ptr, cb_->device);
      delete cb_;
    }
#endif
    cb_ = nullptr;
  }

  template <class... N>
  void set_extents(N... n) {
    static_assert(sizeof...(N) <= rank_dynamic || sizeof...(N) == rank,
                  "View: give one extent per dynamic rank (or one per rank)");
    const std::size_t e[] = {static_cast<std::size_t>(n)..., 0};
    for (int d = 0; d < rank_dynamic; ++d) dyn_[d] = d < int(sizeof...(N)) ? e[d] : 0;
  }

 public:
  KOKKOS_INLINE_FUNCTION View() {}
  KOKKOS_INLINE_FUNCTION View(const View& o) : data_(o.data_), cb_(o.cb_) {
    for (int d = 0; d < rank_dynamic; ++d) dyn_[d] = o.dyn_[d];
    retain();
  }
  KOKKOS_INLINE_FUNCTION View(View&& o) : data_(o.data_), cb_(o.cb_) {
    for (int d = 0; d < rank_dynamic; ++d) dyn_[d] = o.dyn_[d];
    o.cb_ = nullptr;
  }
  KOKKOS_INLINE_FUNCTION View& operator=(const View& o) {
    if (this != &o) {
      o.retain();
      release();
      data_ = o.data_;
      cb_ = o.cb_;
      for (int d = 0; d < rank_dynamic; ++d) dyn_[d] = o.dyn_[d];
    }
    return *this;
  }
  KOKKOS_INLINE_FUNCTION ~View() { release(); }

  // non-const -> const conversion
  template <class D2, class... P2,
            class = std::enable_if_t<!std::is_same_v<View<D2, P2...>, View> &&
                                     std::is_same_v<typename View<D2, P2...>::non_const_value_type,
                                                    non_const_value_type> &&
                                     View<D2, P2...>::rank == rank>>
  KOKKOS_INLINE_FUNCTION View(const View<D2, P2...>& o) : data_(o.data()), cb_(o.impl_cb()) {
    for (int d = 0; d < rank_dynamic; ++d) dyn_[d] = o.extent(d);
    retain();
  }

  // Managed allocation: View("label", n0, n1, ...) -- one extent per dynamic rank.
  template <class... N, class = std::enable_if_t<(std::is_integral_v<N> && ...)>>
  explicit View(const std::string& label, N... n) {
    static_assert(managed, "View(label, ...) allocates; this View type is unmanaged");
    set_extents(n...);
    const bool dev = !std::is_same_v<memory_space, HostSpace>;
    cb_ = new Impl::ControlBlock;
    cb_->device = dev;
    cb_->label = label;
    cb_->ptr = Impl::alloc_bytes(span() * sizeof(value_type), dev, label.c_str());
    data_ = static_cast<pointer_type>(cb_->ptr);
  }
  template <class... N, class = std::enable_if_t<(std::is_integral_v<N> && ...)>>
  explicit View(const char* label, N... n) : View(std::string(label), n...) {}

  // Unmanaged wrap of existing memory.
  template <class... N, class = std::enable_if_t<(std::is_integral_v<N> && ...)>>
  KOKKOS_INLINE_FUNCTION View(pointer_type p, N... n) : data_(p) {
    const std::size_t e[] = {static_cast<std::size_t>(n)..., 0};
    for (int d = 0; d < rank_dynamic; ++d) dyn_[d] = d < int(sizeof...(N)) ? e[d] : 0;
  }

  // Team-scratch allocation: View(member.team_scratch(0), n0, ...).
  template <class E, class... N, class = std::enable_if_t<(std::is_integral_v<N> && ...)>>
  KOKKOS_INLINE_FUNCTION View(const ScratchMemorySpace<E>& space, N... n) {
    const std::size_t e[] = {static_cast<std::size_t>(n)..., 0};
    for (int d = 0; d < rank_dynamic; ++d) dyn_[d] = d < int(sizeof...(N)) ? e[d] : 0;
    data_ = static_cast<pointer_type>(space.get_shmem(span() * sizeof(value_type)));
  }

  template <std::size_t... I>
  KOKKOS_INLINE_FUNCTION static constexpr std::size_t static_extent_impl(int s,
                                                                         std::index_sequence<I...>) {
    std::size_t r = 0;
    ((s == static_cast<int>(I) ? (r = std::extent_v<DataType, I>, 0) : 0), ...);
    return r;
  }
  // extent of the s-th static (bracketed) dimension
  KOKKOS_INLINE_FUNCTION static constexpr std::size_t static_extent(int s) {
    return static_extent_impl(s, std::make_index_sequence<DA::rank_static>{});
  }

  template <class... N>
  KOKKOS_INLINE_FUNCTION static std::size_t shmem_size(N... n) {
    const std::size_t e[] = {static_cast<std::size_t>(n)..., 0};
    std::size_t total = 1;
    for (int d = 0; d < rank; ++d)
      total *= d < rank_dynamic ? (d < int(sizeof...(N)) ? e[d] : 0) : static_extent(d - rank_dynamic);
    return ScratchMemorySpace<DefaultExecutionSpace>::round(total * sizeof(value_type));
  }

  KOKKOS_INLINE_FUNCTION constexpr std::size_t extent(int d) const {
    return d < rank_dynamic ? dyn_[d] : static_extent(d - rank_dynamic);
  }
  KOKKOS_INLINE_FUNCTION constexpr int extent_int(int d) const {
    return static_cast<int>(extent(d));
  }
  KOKKOS_INLINE_FUNCTION std::size_t stride(int d) const {
    std::size_t s = 1;
    if constexpr (kLeft) {
      for (int q = 0; q < d; ++q) s *= extent(q);
    } else {
      for (int q = rank - 1; q > d; --q) s *= extent(q);
    }
    return s;
  }
  KOKKOS_INLINE_FUNCTION std::size_t size() const {
    std::size_t s = 1;
    for (int d = 0; d < rank; ++d) s *= extent(d);
    return s;
  }
  KOKKOS_INLINE_FUNCTION std::size_t span() const { return size(); }
  KOKKOS_INLINE_FUNCTION pointer_type data() const { return data_; }
  KOKKOS_INLINE_FUNCTION bool is_allocated() const { return data_ != nullptr; }
  KOKKOS_INLINE_FUNCTION Impl::ControlBlock* impl_cb() const { return cb_; }
  std::string label() const { return cb_ ? cb_->label : std::string(); }
  int use_count() const { return cb_ ? cb_->refs.load() : 0; }

  template <class... I>
  KOKKOS_FORCEINLINE_FUNCTION reference_type operator()(I... idx) const {
    static_assert(sizeof...(I) == rank || (rank == 0 && sizeof...(I) == 0),
                  "View: one index per rank");
    std::size_t off = 0;
    if constexpr (kLeft) {
      // first index fastest: fold from the last index down
      const std::size_t ix[] = {static_cast<std::size_t>(idx)..., 0};
      for (int d = rank - 1; d >= 0; --d) off = off * extent(d) + ix[d];
    } else {
      int d = 0;
      ((off = off * extent(d++) + static_cast<std::size_t>(idx)), ...);
    }
    return data_[off];
  }
  KOKKOS_FORCEINLINE_FUNCTION reference_type operator[](std::size_t i) const { return data_[i]; }
};

template <class V>
using host_mirror_t = typename V::host_mirror_type;

// ---------------------------------------------------------------------------
// deep_copy / mirrors
// ---------------------------------------------------------------------------
template <class D1, class... P1, class D2, class... P2>
void deep_copy(const View<D1, P1...>& dst, const View<D2, P2...>& src) {
  using T1 = typename View<D1, P1...>::non_const_value_type;
  using T2 = typename View<D2, P2...>::non_const_value_type;
  static_assert(std::is_same_v<T1, T2>, "deep_copy: value types differ");
  static_assert(std::is_same_v<typename View<D1, P1...>::array_layout,
                               typename View<D2, P2...>::array_layout> ||
                    View<D1, P1...>::rank <= 1,
                "deep_copy: this Kokkos subset copies between views of one layout");
  if (dst.span() != src.span()) {
    std::fprintf(stderr, "Kokkos::deep_copy: extents differ (%zu vs %zu)\n", dst.span(),
                 src.span());
    std::abort();
  }
  if (dst.data() == src.data()) return;
  const std::size_t bytes = dst.span() * sizeof(T1);
#ifdef KOKKOS_ENABLE_CUDA
  cudaDeviceSynchronize();
  cudaMemcpy(const_cast<T1*>(dst.data()), src.data(), bytes, cudaMemcpyDefault);
#else
  std::memcpy(const_cast<T1*>(dst.data()), src.data(), bytes);
#endif
}

#ifdef KOKKOS_ENABLE_CUDA
namespace Impl {
template <class T>
__global__ void fill_kernel(T* p, std::size_t n, T v) {
  for (std::size_t i = blockIdx.x * std::size_t(blockDim.x) + threadIdx.x; i < n;
       i += std::size_t(gridDim.x) * blockDim.x)
    p[i] = v;
}
}  // namespace Impl
#endif

template <class D, class... P>
void deep_copy(const View<D, P...>& dst, typename View<D, P...>::const_value_type& value) {
  using V = View<D, P...>;
  using T = typename V::non_const_value_type;
  T* p = const_cast<T*>(dst.data());
  const std::size_t n = dst.span();
#ifdef KOKKOS_ENABLE_CUDA
  if (!std::is_same_v<typename V::memory_space, HostSpace>) {
    if (n) Impl::fill_kernel<T><<<(n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096, 256>>>(p, n, value);
    cudaDeviceSynchronize();
    return;
  }
#endif
  for (std::size_t i = 0; i < n; ++i) p[i] = value;
}

template <class D, class... P>
auto create_mirror_view(const View<D, P...>& v) {
  using V = View<D, P...>;
  using M = typename V::host_mirror_type;
  if constexpr (std::is_same_v<M, V>) {
    return v;
  } else {
    M m;
    if constexpr (V::rank_dynamic == 0)
      m = M(v.label() + "_mirror");
    else
      m = [&]<std::size_t... Is>(std::index_sequence<Is...>) {
        return M(v.label() + "_mirror", v.extent(Is)...);
      }(std::make_index_sequence<V::rank_dynamic>{});
    return m;
  }
}
template <class D, class... P>
auto create_mirror(const View<D, P...>& v) {
  using V = View<D, P...>;
  using M = typename V::host_mirror_type;
  if constexpr (V::rank_dynamic == 0)
    return M(v.label() + "_mirror");
  else
    return [&]<std::size_t... Is>(std::index_sequence<Is...>) {
      return M(v.label() + "_mirror", v.extent(Is)...);
    }(std::make_index_sequence<V::rank_dynamic>{});
}
template <class D, class... P>
auto create_mirror_view_and_copy(const HostSpace&, const View<D, P...>& v) {
  auto m = create_mirror_view(v);
  if (m.data() != v.data()) deep_copy(m, v);
  return m;
}

// ---------------------------------------------------------------------------
// Policies and team members
// ---------------------------------------------------------------------------
struct AUTO_t {};
inline constexpr AUTO_t AUTO{};
struct ParallelForTag {};

struct PerTeamValue {
  std::size_t value;
};
struct PerThreadValue {
  std::size_t value;
};
inline PerTeamValue PerTeam(std::size_t b) { return {b}; }
inline PerThreadValue PerThread(std::size_t b) { return {b}; }

template <class... Props>
struct PolicyExec {
  template <class Acc, class... R>
  struct pick {
    using type = Acc;
  };
  template <class Acc, class H, class... R>
  struct pick<Acc, H, R...> {
    static constexpr bool is_es =
        std::is_same_v<H, Serial>
#ifdef KOKKOS_ENABLE_CUDA
        || std::is_same_v<H, Cuda>
#endif
        ;
    using type = std::conditional_t<std::is_void_v<Acc> && is_es, H,
                                    typename pick<Acc, R...>::type>;
  };
  using named = typename pick<void, Props...>::type;
  using type = std::conditional_t<std::is_void_v<named>, DefaultExecutionSpace, named>;
};

template <class ExecSpace>
class TeamMember {
 public:
  using execution_space = ExecSpace;
  using scratch_memory_space = ScratchMemorySpace<ExecSpace>;

 private:
  int league_rank_, league_size_, team_rank_, team_size_;
  scratch_memory_space scratch_;

 public:
  KOKKOS_INLINE_FUNCTION TeamMember(int lr, int ls, int tr, int ts, void* smem, std::size_t bytes,
                                    int* status = nullptr)
      : league_rank_(lr), league_size_(ls), team_rank_(tr), team_size_(ts),
        scratch_(smem, bytes, status) {}
  KOKKOS_INLINE_FUNCTION int league_rank() const { return league_rank_; }
  KOKKOS_INLINE_FUNCTION int league_size() const { return league_size_; }
  KOKKOS_INLINE_FUNCTION int team_rank() const { return team_rank_; }
  KOKKOS_INLINE_FUNCTION int team_size() const { return team_size_; }
  KOKKOS_INLINE_FUNCTION const scratch_memory_space& team_scratch(int = 0) const { return scratch_; }
  KOKKOS_INLINE_FUNCTION const scratch_memory_space& team_shmem() const { return scratch_; }
  KOKKOS_INLINE_FUNCTION void team_barrier() const {
#if defined(TO_KOKKOS_DEVICE_PASS)
    __syncthreads();
#endif
  }
};

template <class... Props>
class TeamPolicy {
 public:
  using execution_space = typename PolicyExec<Props...>::type;
  using member_type = TeamMember<execution_space>;

 private:
  int league_ = 0, team_ = -1;
  std::size_t scratch_[2] = {0, 0};

 public:
  TeamPolicy() = default;
  TeamPolicy(int league, int team) : league_(league), team_(team) {}
  TeamPolicy(int league, AUTO_t) : league_(league), team_(-1) {}
  TeamPolicy(int league, int team, int) : league_(league), team_(team) {}
  TeamPolicy(int league, AUTO_t, int) : league_(league), team_(-1) {}
  TeamPolicy(const execution_space&, int league, int team) : league_(league), team_(team) {}
  TeamPolicy(const execution_space&, int league, AUTO_t) : league_(league), team_(-1) {}
  // Sets the request in place and returns the policy, as Kokkos does: both
  // `policy.set_scratch_size(0, PerTeam(b));` and a chained call on a
  // temporary reach the launch.
  TeamPolicy& set_scratch_size(int level, PerTeamValue v) {
    scratch_[level ? 1 : 0] = v.value;
    return *this;
  }
  TeamPolicy& set_scratch_size(int level, PerTeamValue v, PerThreadValue) {
    return set_scratch_size(level, v);
  }
  int league_size() const { return league_; }
  int team_size() const { return team_; }
  // The team size parallel_for launches with AUTO (128 threads): the shim
  // does not size teams from occupancy.
  template <class F>
  int team_size_recommended(const F&, ParallelForTag) const {
    return team_ > 0 ? team_ : 128;
  }
  template <class F>
  int team_size_max(const F&, ParallelForTag) const {
    return 1024;
  }
  bool auto_team() const { return team_ <= 0; }
  std::size_t scratch_size(int level) const { return scratch_[level ? 1 : 0]; }
};

template <class... Props>
class RangePolicy {
 public:
  using execution_space = typename PolicyExec<Props...>::type;
  std::int64_t begin_ = 0, end_ = 0;
  RangePolicy(std::int64_t b, std::int64_t e) : begin_(b), end_(e) {}
  RangePolicy(const execution_space&, std::int64_t b, std::int64_t e) : begin_(b), end_(e) {}
};

// MDRangePolicy<Rank<N>>: the box [lo, hi) of an N-dimensional index space.
// The iteration-order and tiling arguments of Kokkos are accepted and ignored:
// every point is visited exactly once, the last index fastest.
enum class Iterate { Default, Left, Right };
template <unsigned N, Iterate Outer = Iterate::Default, Iterate Inner = Iterate::Default>
struct Rank {
  static constexpr unsigned rank = N;
};

namespace Impl {
template <class T>
struct rank_of_prop : std::integral_constant<unsigned, 0> {};
template <unsigned N, Iterate O, Iterate I>
struct rank_of_prop<Rank<N, O, I>> : std::integral_constant<unsigned, N> {};
}  // namespace Impl

template <class... Props>
class MDRangePolicy {
 public:
  using execution_space = typename PolicyExec<Props...>::type;
  static constexpr int rank = static_cast<int>((Impl::rank_of_prop<Props>::value + ... + 0u));
  static_assert(rank >= 1 && rank <= 6, "MDRangePolicy: give Kokkos::Rank<N> with 1 <= N <= 6");
  Array<std::int64_t, rank> lo{}, hi{};

  MDRangePolicy(std::initializer_list<std::int64_t> b, std::initializer_list<std::int64_t> e,
                std::initializer_list<std::int64_t> = {}) {
    assign(b, e);
  }
  MDRangePolicy(const execution_space&, std::initializer_list<std::int64_t> b,
                std::initializer_list<std::int64_t> e, std::initializer_list<std::int64_t> = {}) {
    assign(b, e);
  }
  template <class I>
  MDRangePolicy(const Array<I, rank>& b, const Array<I, rank>& e) {
    for (int d = 0; d < rank; ++d) {
      lo[d] = static_cast<std::int64_t>(b[d]);
      hi[d] = static_cast<std::int64_t>(e[d]);
    }
  }
  std::int64_t size() const {
    std::int64_t n = 1;
    for (int d = 0; d < rank; ++d) n *= hi[d] > lo[d] ? hi[d] - lo[d] : 0;
    return n;
  }

 private:
  void assign(std::initializer_list<std::int64_t> b, std::initializer_list<std::int64_t> e) {
    if (static_cast<int>(b.size()) != rank || static_cast<int>(e.size()) != rank) {
      std::fprintf(stderr, "Kokkos::MDRangePolicy: give %d lower and %d upper bounds\n", rank, rank);
      std::abort();
    }
    int d = 0;
    for (std::int64_t v : b) lo[d++] = v;
    d = 0;
    for (std::int64_t v : e) hi[d++] = v;
  }
};

namespace Impl {
// Point `flat` of the box, the last index fastest, handed to f as N indices.
template <int N, class F, std::size_t... D>
KOKKOS_INLINE_FUNCTION void md_call(const F& f, const Array<std::int64_t, N>& lo,
                                    const Array<std::int64_t, N>& ext, std::int64_t flat,
                                    std::index_sequence<D...>) {
  std::int64_t idx[N];
  for (int d = N - 1; d >= 0; --d) {
    idx[d] = lo[d] + flat % ext[d];
    flat /= ext[d];
  }
  f(idx[D]...);
}
}  // namespace Impl

template <class Member>
struct TeamRange {
  const Member& member;
  int begin, end;
};
template <class Member>
struct VectorRange {
  const Member& member;
  int begin, end;
};

template <class Member>
KOKKOS_INLINE_FUNCTION TeamRange<Member> TeamVectorRange(const Member& m, int n) {
  return {m, 0, n};
}
template <class Member>
KOKKOS_INLINE_FUNCTION TeamRange<Member> TeamVectorRange(const Member& m, int b, int e) {
  return {m, b, e};
}
template <class Member>
KOKKOS_INLINE_FUNCTION TeamRange<Member> TeamThreadRange(const Member& m, int n) {
  return {m, 0, n};
}
template <class Member>
KOKKOS_INLINE_FUNCTION TeamRange<Member> TeamThreadRange(const Member& m, int b, int e) {
  return {m, b, e};
}
template <class Member>
KOKKOS_INLINE_FUNCTION VectorRange<Member> ThreadVectorRange(const Member& m, int n) {
  return {m, 0, n};
}
template <class Member>
KOKKOS_INLINE_FUNCTION VectorRange<Member> ThreadVectorRange(const Member& m, int b, int e) {
  return {m, b, e};
}

// Nested ranges: the team's threads split the range; a vector range is the
// calling thread's own loop (vector length 1).
template <class Member, class F>
KOKKOS_INLINE_FUNCTION void parallel_for(const TeamRange<Member>& r, const F& f) {
  for (int i = r.begin + r.member.team_rank(); i < r.end; i += r.member.team_size()) f(i);
}
template <class Member, class F>
KOKKOS_INLINE_FUNCTION void parallel_for(const VectorRange<Member>& r, const F& f) {
  for (int i = r.begin; i < r.end; ++i) f(i);
}

namespace Impl {
#ifdef KOKKOS_ENABLE_CUDA
template <class F>
__global__ void team_kernel(const F f, std::size_t scratch_bytes, int* status) {
  extern __shared__ __align__(16) unsigned char team_smem[];
  TeamMember<Cuda> m(static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x),
                     static_cast<int>(threadIdx.x), static_cast<int>(blockDim.x), team_smem,
                     scratch_bytes, status);
  f(m);
}
template <class F>
__global__ void range_kernel(const F f, std::int64_t begin, std::int64_t end) {
  for (std::int64_t i = begin + blockIdx.x * std::int64_t(blockDim.x) + threadIdx.x; i < end;
       i += std::int64_t(gridDim.x) * blockDim.x)
    f(i);
}
inline void check_launch(const char* label) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    std::fprintf(stderr, "Kokkos::parallel_for('%s'): %s\n", label ? label : "",
                 cudaGetErrorString(e));
    std::abort();
  }
}
#endif
}  // namespace Impl

template <class F, class... Props>
void parallel_for(const char* label, const TeamPolicy<Props...>& p, const F& f) {
  using ES = typename TeamPolicy<Props...>::execution_space;
  const std::size_t bytes = p.scratch_size(0) + p.scratch_size(1);
#ifdef KOKKOS_ENABLE_CUDA
  if constexpr (std::is_same_v<ES, Cuda>) {
    const int team = p.auto_team() ? 128 : p.team_size();
    if (p.league_size() <= 0) return;
    if (bytes > 48 * 1024)
      cudaFuncSetAttribute(Impl::team_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes));
    Impl::team_kernel<F><<<p.league_size(), team, bytes>>>(f, bytes, Impl::scratch_status());
    Impl::check_launch(label);
  } else
#endif
  {
    (void)label;
    void* buf = bytes ? std::malloc(bytes) : nullptr;
    for (int lr = 0; lr < p.league_size(); ++lr) {
      TeamMember<Serial> m(lr, p.league_size(), 0, 1, buf, bytes, Impl::scratch_status());
      try {
        f(m);
      } catch (const Impl::ScratchOverflow&) {
        // this team stopped at its over-sized request; the status word says so
      }
    }
    std::free(buf);
  }
}
template <class F, class... Props>
void parallel_for(const TeamPolicy<Props...>& p, const F& f) {
  parallel_for("", p, f);
}

template <class F, class... Props>
void parallel_for(const char* label, const RangePolicy<Props...>& p, const F& f) {
  using ES = typename RangePolicy<Props...>::execution_space;
#ifdef KOKKOS_ENABLE_CUDA
  if constexpr (std::is_same_v<ES, Cuda>) {
    const std::int64_t n = p.end_ - p.begin_;
    if (n <= 0) return;
    const std::int64_t blocks = (n + 255) / 256;
    Impl::range_kernel<F><<<static_cast<unsigned>(blocks < 65535 * 8 ? blocks : 65535 * 8), 256>>>(
        f, p.begin_, p.end_);
    Impl::check_launch(label);
  } else
#endif
  {
    (void)label;
    for (std::int64_t i = p.begin_; i < p.end_; ++i) f(i);
  }
}
template <class F, class... Props>
void parallel_for(const RangePolicy<Props...>& p, const F& f) {
  parallel_for("", p, f);
}
#ifdef KOKKOS_ENABLE_CUDA
namespace Impl {
template <int N, class F>
__global__ void md_range_kernel(const F f, const Array<std::int64_t, N> lo,
                                const Array<std::int64_t, N> ext, std::int64_t total) {
  for (std::int64_t i = blockIdx.x * std::int64_t(blockDim.x) + threadIdx.x; i < total;
       i += std::int64_t(gridDim.x) * blockDim.x)
    md_call<N>(f, lo, ext, i, std::make_index_sequence<N>{});
}
}  // namespace Impl
#endif

template <class F, class... Props>
void parallel_for(const char* label, const MDRangePolicy<Props...>& p, const F& f) {
  using P = MDRangePolicy<Props...>;
  using ES = typename P::execution_space;
  constexpr int N = P::rank;
  const std::int64_t total = p.size();
  if (total <= 0) return;
  Array<std::int64_t, N> ext{};
  for (int d = 0; d < N; ++d) ext[d] = p.hi[d] - p.lo[d];
#ifdef KOKKOS_ENABLE_CUDA
  if constexpr (std::is_same_v<ES, Cuda>) {
    const std::int64_t blocks = (total + 255) / 256;
    Impl::md_range_kernel<N, F><<<static_cast<unsigned>(blocks < 65535 * 8 ? blocks : 65535 * 8), 256>>>(
        f, p.lo, ext, total);
    Impl::check_launch(label);
  } else
#endif
  {
    (void)label;
    for (std::int64_t i = 0; i < total; ++i)
      Impl::md_call<N>(f, p.lo, ext, i, std::make_index_sequence<N>{});
  }
}
template <class F, class... Props>
void parallel_for(const MDRangePolicy<Props...>& p, const F& f) {
  parallel_for("", p, f);
}

template <class F, class I, class = std::enable_if_t<std::is_integral_v<I>>>
void parallel_for(const char* label, I n, const F& f) {
  parallel_for(label, RangePolicy<>(0, static_cast<std::int64_t>(n)), f);
}
template <class F, class I, class = std::enable_if_t<std::is_integral_v<I>>>
void parallel_for(I n, const F& f) {
  parallel_for("", RangePolicy<>(0, static_cast<std::int64_t>(n)), f);
}

}  // namespace Kokkos
