// batched_gemm.cu -- batched small GEMM with a shared left operand:
//   C[b][i][j] = sum_k A[i][k] * B[b][k][j]      (A: M x K, B[b]: K x N)
// the shape of one gradient contraction of the SEM operator, batched over
// elements (the reference's analogue: benchmarks/sem_stiffness/bench_sem_stiffness.cpp:884-896).
// HBM-bound (1.25 flop/byte in f32 at M=K=5, N=25): one thread per output
// column (b, j) reads its K inputs B[b][:, j] (consecutive threads, consecutive
// words), keeps A in the kernel-parameter bank and writes its M outputs; the
// sums run over k in order with fused multiply-adds.  Grid-stride over the
// batch so any batch size uses every SM.
#include "common.hpp"

namespace to_b200 {
namespace {

constexpr int kMaxMK = 16;

template <typename T>
struct SmallA {
  T a[kMaxMK * kMaxMK];
};

template <typename T, int M, int K>
__global__ void __launch_bounds__(256) batched_small_gemm_kernel(const __grid_constant__ SmallA<T> A,
                                                                 const T* __restrict__ B,
                                                                 T* __restrict__ C, long long batch,
                                                                 int N) {
  const long long total = batch * N;
  for (long long t = blockIdx.x * 256ll + threadIdx.x; t < total; t += gridDim.x * 256ll) {
    const long long b = t / N;
    const int j = static_cast<int>(t - b * N);
    const T* bp = B + b * K * N + j;
    T x[K];
#pragma unroll
    for (int k = 0; k < K; ++k) x[k] = __ldcs(bp + k * N);  // streamed once
    T* cp = C + b * M * N + j;
#pragma unroll
    for (int i = 0; i < M; ++i) {
      T s = T(0);
#pragma unroll
      for (int k = 0; k < K; ++k) s = fma(A.a[i * K + k], x[k], s);
      __stcs(cp + i * N, s);
    }
  }
}

template <typename T, int M, int K>
int launch(const double* A, const void* B, void* C, long long batch, int N, cudaStream_t s) {
  SmallA<T> a;
  for (int i = 0; i < M * K; ++i) a.a[i] = static_cast<T>(A[i]);
  int dev = 0;
  const int sms = device_sm_count(&dev);
  if (sms <= 0) return -sms;
  const long long want = (batch * N + 255) / 256;
  const long long cap = 16ll * sms;
  const int grid = static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
  batched_small_gemm_kernel<T, M, K><<<grid, 256, 0, s>>>(a, static_cast<const T*>(B),
                                                          static_cast<T*>(C), batch, N);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // namespace
}  // namespace to_b200

using namespace to_b200;

extern "C" int to_batched_small_gemm(int32_t dtype, int32_t M, int32_t K, int32_t N, int64_t batch,
                                     const double* A, const void* B, void* C, void* stream) {
  if (!A || !B || !C || batch < 0 || N <= 0)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_batched_small_gemm: bad argument");
  if (batch == 0) return ok();
  const size_t vb = dtype == TO_F64 ? 8 : 4;
  if (!aligned(B, vb) || !aligned(C, vb))
    return set_error(TO_ERR_ALIGNMENT, "to_batched_small_gemm: B / C misaligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // built shapes: the SEM operator's (M, K) = (N_gll, N_gll) for N_gll 5 and 8
  if (M == 5 && K == 5) {
    if (dtype == TO_F32) return launch<float, 5, 5>(A, B, C, batch, N, s);
    if (dtype == TO_F64) return launch<double, 5, 5>(A, B, C, batch, N, s);
  } else if (M == 8 && K == 8) {
    if (dtype == TO_F32) return launch<float, 8, 8>(A, B, C, batch, N, s);
    if (dtype == TO_F64) return launch<double, 8, 8>(A, B, C, batch, N, s);
  }
  return set_error(TO_ERR_UNSUPPORTED, "to_batched_small_gemm: (M, K, dtype) = (%d, %d, %d) not built",
                   M, K, dtype);
}
