// sem3d_vector.cu -- field reductions and rescaling for repeated applications
// (u <- K u / ||K u||, the steady-state loop of the large fp64 configuration).
//
// sum of squares, two passes, deterministic:
//   pass 1: block b sums the squares of values [b*kChunk, (b+1)*kChunk) of the
//           component-major sequence x_0[first..first+n) ++ x_1[...] ++ x_2[...]
//           in a fixed order (per-thread strided sums, then a fixed tree) and
//           writes partial[b] (the workspace);
//   pass 2: one block adds the partials in a fixed order into *result.
// The chunk size is fixed, so the grouping -- and the rounding -- depends
// only on n, never on the GPU's SM count: the same inputs give the same bits
// on any device.  Accumulation is in double for every dtype.
#include <mutex>

#include "common.hpp"

namespace to_b200 {

constexpr int kSumThreads = 256;
constexpr long long kSumChunk = 131072;  // values per block of pass 1

template <typename T>
struct Fields3 {
  const T* x[3];
};

__device__ __forceinline__ double block_sum_fixed(double v, double* red) {
  // fixed-order tree: warp shuffles, then warp 0 over the warp sums
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  double s = 0.0;
  if (w == 0) {
    s = l < (kSumThreads / 32) ? red[l] : 0.0;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  }
  return s;  // valid in thread 0
}

template <typename T>
__global__ void __launch_bounds__(kSumThreads)
    sumsq_partial_kernel(Fields3<T> f, long long first, long long n, double* __restrict__ partial) {
  __shared__ double red[kSumThreads / 32];
  const long long total = 3 * n;
  const long long c0 = static_cast<long long>(blockIdx.x) * kSumChunk;
  const long long c1 = c0 + kSumChunk < total ? c0 + kSumChunk : total;
  // The chunk meets at most three components, each a contiguous run walked
  // without a division per value.  In each run, thread tid takes the values
  // t = s0' + 256 j (s0' its first index there, j = 0, 1, ...) into
  // accumulator j % 4 -- four loads in flight -- and the four are added in a
  // fixed order at the end: the grouping depends on n, first and the chunk
  // only.
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  for (int c = static_cast<int>(c0 / n); c < 3 && static_cast<long long>(c) * n < c1; ++c) {
    const long long s0 = c0 > c * n ? c0 : c * n;  // run [s0, s1) of component c
    const long long s1 = c1 < (c + 1) * n ? c1 : (c + 1) * n;
    long long t = s0 + ((static_cast<long long>(threadIdx.x) - (s0 - c0)) % kSumThreads +
                        kSumThreads) % kSumThreads;
    const T* x = f.x[c] + first - c * n;
    for (; t + 3 * kSumThreads < s1; t += 4 * kSumThreads) {
      const double v0 = static_cast<double>(x[t]);
      const double v1 = static_cast<double>(x[t + kSumThreads]);
      const double v2 = static_cast<double>(x[t + 2 * kSumThreads]);
      const double v3 = static_cast<double>(x[t + 3 * kSumThreads]);
      acc[0] = fma(v0, v0, acc[0]);
      acc[1] = fma(v1, v1, acc[1]);
      acc[2] = fma(v2, v2, acc[2]);
      acc[3] = fma(v3, v3, acc[3]);
    }
    if (t < s1) {
      const double v = static_cast<double>(x[t]);
      acc[0] = fma(v, v, acc[0]);
    }
    if (t + kSumThreads < s1) {
      const double v = static_cast<double>(x[t + kSumThreads]);
      acc[1] = fma(v, v, acc[1]);
    }
    if (t + 2 * kSumThreads < s1) {
      const double v = static_cast<double>(x[t + 2 * kSumThreads]);
      acc[2] = fma(v, v, acc[2]);
    }
  }
  const double s = block_sum_fixed((acc[0] + acc[1]) + (acc[2] + acc[3]), red);
  if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

__global__ void __launch_bounds__(kSumThreads)
    sumsq_final_kernel(const double* __restrict__ partial, int nb, double* __restrict__ result) {
  __shared__ double red[kSumThreads / 32];
  double acc = 0.0;
  for (int b = threadIdx.x; b < nb; b += kSumThreads) acc += partial[b];
  const double s = block_sum_fixed(acc, red);
  if (threadIdx.x == 0) *result = s;
}

template <typename T>
__global__ void scale3_kernel(Fields3<T> x, T* y0, T* y1, T* y2, long long n,
                              const double* __restrict__ sumsq) {
  const double inv = 1.0 / sqrt(*sumsq);
  const long long total = 3 * n;
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(t / n);
    const long long k = t - c * n;
    T* y = c == 0 ? y0 : (c == 1 ? y1 : y2);
    y[k] = static_cast<T>(static_cast<double>(x.x[c][k]) * inv);
  }
}

long long sumsq_blocks(long long n) { return (3 * n + kSumChunk - 1) / kSumChunk; }

template <typename T>
int sumsq_launch(const void* const x[3], long long first, long long n, double* result,
                 double* partial, cudaStream_t s) {
  Fields3<T> f;
  for (int c = 0; c < 3; ++c) {
    if (!x[c]) return set_error(TO_ERR_INVALID_ARGUMENT, "sumsq: null x[%d]", c);
    if (!aligned(x[c], sizeof(T))) return set_error(TO_ERR_ALIGNMENT, "sumsq: x[%d] misaligned", c);
    f.x[c] = static_cast<const T*>(x[c]);
  }
  const long long nb = sumsq_blocks(n);
  if (nb > 0) sumsq_partial_kernel<T><<<static_cast<unsigned>(nb), kSumThreads, 0, s>>>(f, first, n, partial);
  sumsq_final_kernel<<<1, kSumThreads, 0, s>>>(partial, static_cast<int>(nb), result);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

// Shared argument checks and dispatch of the sum of squares; `partial` must
// hold sumsq_blocks(n) doubles.
int sumsq_common(int32_t dtype, const void* const x[3], int64_t first, int64_t n, double* result,
                 double* partial, cudaStream_t s, const char* who) {
  if (!x || !result || !partial) return set_error(TO_ERR_INVALID_ARGUMENT, "%s: null", who);
  if (first < 0 || n < 0) return set_error(TO_ERR_INVALID_ARGUMENT, "%s: bad range", who);
  if (!aligned(result, 8) || !aligned(partial, 8))
    return set_error(TO_ERR_ALIGNMENT, "%s: result / workspace not 8-byte aligned", who);
  if (sumsq_blocks(n) > 2147483647ll) return set_error(TO_ERR_INVALID_ARGUMENT, "%s: n too large", who);
  if (dtype == TO_F32) return sumsq_launch<float>(x, first, n, result, partial, s);
  if (dtype == TO_F64) return sumsq_launch<double>(x, first, n, result, partial, s);
  return set_error(TO_ERR_INVALID_ARGUMENT, "%s: dtype %d", who, dtype);
}

// ---- the allocation-free variant ----------------------------------------------
// Block partials of to_sumsq3_noalloc live in this file-scope array: 32768
// doubles (256 KiB), held by every GPU that loads the library until the
// process exits.  One partial covers kSumChunk values, so one call handles at
// most 32768 * 131072 values, i.e. n <= kNoAllocMaxN per component.
constexpr long long kNoAllocMaxPartials = 32768;
constexpr long long kNoAllocMaxN = kNoAllocMaxPartials * kSumChunk / 3;
static __device__ __align__(256) double g_noalloc_partials[kNoAllocMaxPartials];

// Device address of g_noalloc_partials, looked up once per device and CUDA
// context.  In host code the array's name only stands in for the symbol, so
// the address comes from cudaGetSymbolAddress with that device current.  The
// cache remembers the context it was filled in (through the driver's
// cuCtxGetCurrent, reached without linking the driver library): a caller that
// makes its own context current, or a cudaDeviceReset that replaced the
// primary context, gets a fresh lookup instead of a stale address.
using CtxGetCurrentFn = int (*)(void**);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      f = nullptr;
    }
    return reinterpret_cast<CtxGetCurrentFn>(f);
  }();
  return fn;
}

double* noalloc_partials(int* status) {
  static std::mutex mu;
  static double* ptr[64] = {};
  static void* ctx_of[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *status = cuda_fail(e, "to_sumsq3_noalloc: cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    *status = set_error(TO_ERR_UNSUPPORTED, "to_sumsq3_noalloc: device id %d >= 64", dev);
    return nullptr;
  }
  auto current_ctx = [] {
    void* c = nullptr;
    if (CtxGetCurrentFn f = ctx_get_current())
      if (f(&c) != 0) c = nullptr;
    return c;
  };
  void* ctx = current_ctx();  // null until the runtime has made a context current
  std::lock_guard<std::mutex> lock(mu);
  if (!ptr[dev] || ctx == nullptr || ctx_of[dev] != ctx) {
    double* p = nullptr;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_partials);
    if (e != cudaSuccess) {
      *status = cuda_fail(e, "to_sumsq3_noalloc: cudaGetSymbolAddress");
      return nullptr;
    }
    ptr[dev] = p;
    ctx_of[dev] = ctx ? ctx : current_ctx();  // the lookup made the primary context current
  }
  *status = TO_OK;
  return ptr[dev];
}

}  // namespace to_b200

using namespace to_b200;

extern "C" {

size_t to_sumsq3_workspace_bytes(int64_t n) {
  return n < 0 ? 0 : static_cast<size_t>(sumsq_blocks(n)) * sizeof(double);
}

int to_sumsq3(int32_t dtype, const void* const x[3], int64_t first, int64_t n, double* result,
              void* workspace, size_t workspace_bytes, void* stream) {
  if (n >= 0 && workspace_bytes < to_sumsq3_workspace_bytes(n))
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "to_sumsq3: workspace of %zu bytes, %zu needed for n = %lld", workspace_bytes,
                     to_sumsq3_workspace_bytes(n), static_cast<long long>(n));
  return sumsq_common(dtype, x, first, n, result, static_cast<double*>(workspace),
                      static_cast<cudaStream_t>(stream), "to_sumsq3");
}

int to_sumsq3_noalloc(int32_t dtype, const void* const x[3], int64_t first, int64_t n,
                      double* result, void* stream) {
  if (n > kNoAllocMaxN)
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "to_sumsq3_noalloc: n = %lld values per component exceeds this entry "
                     "point's fixed scratch (at most %lld); use to_sumsq3 with a workspace",
                     static_cast<long long>(n), kNoAllocMaxN);
  if (!x || !result || first < 0 || n < 0)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sumsq3_noalloc: bad argument");
  int st = TO_OK;
  double* partial = noalloc_partials(&st);
  if (!partial) return st;
  return sumsq_common(dtype, x, first, n, result, partial, static_cast<cudaStream_t>(stream),
                      "to_sumsq3_noalloc");
}

int64_t to_sumsq3_noalloc_max_n(void) { return kNoAllocMaxN; }

int to_scale3(int32_t dtype, void* const y[3], const void* const x[3], int64_t n,
              const double* sumsq, void* stream) {
  if (!y || !x || !sumsq || n < 0) return set_error(TO_ERR_INVALID_ARGUMENT, "to_scale3: bad argument");
  if (n == 0) return ok();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0;
  const int sms = device_sm_count(&dev);
  if (sms <= 0) return -sms;
  const long long want = (3 * n + 255) / 256;
  const int grid = static_cast<int>(want < 8ll * sms ? want : 8ll * sms);
  for (int c = 0; c < 3; ++c)
    if (!x[c] || !y[c]) return set_error(TO_ERR_INVALID_ARGUMENT, "to_scale3: null component");
  if (dtype == TO_F32) {
    Fields3<float> f{{static_cast<const float*>(x[0]), static_cast<const float*>(x[1]),
                      static_cast<const float*>(x[2])}};
    scale3_kernel<float><<<grid, 256, 0, s>>>(f, static_cast<float*>(y[0]), static_cast<float*>(y[1]),
                                              static_cast<float*>(y[2]), n, sumsq);
  } else if (dtype == TO_F64) {
    Fields3<double> f{{static_cast<const double*>(x[0]), static_cast<const double*>(x[1]),
                       static_cast<const double*>(x[2])}};
    scale3_kernel<double><<<grid, 256, 0, s>>>(f, static_cast<double*>(y[0]), static_cast<double*>(y[1]),
                                               static_cast<double*>(y[2]), n, sumsq);
  } else {
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_scale3: dtype %d", dtype);
  }
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // extern "C"
