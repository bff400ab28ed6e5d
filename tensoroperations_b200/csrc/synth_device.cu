// synth_device.cu -- the seeded synthetic inputs generated on the device, for
// problems too large to stage through host memory (the 142 GB fp64 NGLL-8
// configuration).  Same sequence as the host fill: element m of a stream is
// derived from splitmix64(seed, m) only.  Uniform values are bit-identical to
// the host's (the arithmetic is written without contraction); normal values
// use the device's log / cos and may differ from the host's in the last bits.
#include <cmath>

#include "common.hpp"

namespace to_b200 {
namespace {

__device__ __forceinline__ uint64_t splitmix64_dev(uint64_t seed, uint64_t m) {
  uint64_t z = seed + (m + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

template <typename T>
__global__ void synth_fill_kernel(T* dst, long long first, long long n, uint64_t seed, int dist,
                                  double a, double b, double add) {
  const double inv53 = 1.0 / 9007199254740992.0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const uint64_t m = static_cast<uint64_t>(first + i);
    double v;
    if (dist == 0) {
      const double u = __dmul_rn(static_cast<double>(splitmix64_dev(seed, m) >> 11), inv53);
      v = __dadd_rn(a, __dmul_rn(__dsub_rn(b, a), u));
    } else {
      const uint64_t m2 = 2 * m;
      const double u1 = __dmul_rn(__dadd_rn(static_cast<double>(splitmix64_dev(seed, m2) >> 11), 1.0), inv53);
      const double u2 = __dmul_rn(static_cast<double>(splitmix64_dev(seed, m2 + 1) >> 11), inv53);
      v = a + b * sqrt(-2.0 * log(u1)) * cos(2.0 * 3.141592653589793 * u2);
    }
    dst[i] = static_cast<T>(__dadd_rn(v, add));
  }
}

template <typename T>
__global__ void axpy2_kernel(T* y, const T* x, long long n) {  // y += 2 x
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = y[i] + T(2) * x[i];
}

__global__ void structured_ibool_kernel(int nex, int ney, int nez, int N, int32_t* ib, long long total) {
  const int n1 = N - 1;
  const long long nx = (long long)nex * n1 + 1, ny = (long long)ney * n1 + 1;
  const int P = N * N * N;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long e = t / P;
    const int p = static_cast<int>(t - e * P);
    const int k = p / (N * N), j = (p / N) % N, i = p % N;
    const long long ex = e % nex, ey = (e / nex) % ney, ez = e / ((long long)nex * ney);
    ib[t] = static_cast<int32_t>(((ez * n1 + k) * ny + ey * n1 + j) * nx + ex * n1 + i);
  }
}

int grid_of(long long n) {
  int dev = 0;
  const int sms = device_sm_count(&dev);
  const long long want = (n + 255) / 256;
  const long long cap = 8ll * (sms > 0 ? sms : 148);
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace
}  // namespace to_b200

using namespace to_b200;

extern "C" {

int to_synth_fill_device(void* dst, int32_t dtype, int64_t first, int64_t n, uint64_t seed,
                         int32_t dist, double a, double b, double add, void* stream) {
  if (!dst || n < 0 || first < 0 || (dist != 0 && dist != 1))
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_synth_fill_device: bad argument");
  if (n == 0) return ok();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TO_F32)
    synth_fill_kernel<float><<<grid_of(n), 256, 0, s>>>(static_cast<float*>(dst), first, n, seed, dist, a, b, add);
  else if (dtype == TO_F64)
    synth_fill_kernel<double><<<grid_of(n), 256, 0, s>>>(static_cast<double*>(dst), first, n, seed, dist, a, b, add);
  else
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_synth_fill_device: dtype %d", dtype);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

int to_axpy2_device(void* y, const void* x, int32_t dtype, int64_t n, void* stream) {
  if (!y || !x || n < 0) return set_error(TO_ERR_INVALID_ARGUMENT, "to_axpy2_device: bad argument");
  if (n == 0) return ok();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TO_F32)
    axpy2_kernel<float><<<grid_of(n), 256, 0, s>>>(static_cast<float*>(y), static_cast<const float*>(x), n);
  else if (dtype == TO_F64)
    axpy2_kernel<double><<<grid_of(n), 256, 0, s>>>(static_cast<double*>(y), static_cast<const double*>(x), n);
  else
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_axpy2_device: dtype %d", dtype);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

int to_mesh_structured_ibool_device(int32_t nex, int32_t ney, int32_t nez, int32_t ngll,
                                    int32_t* ibool, void* stream) {
  if (!ibool || nex <= 0 || ney <= 0 || nez <= 0 || ngll < 2 || ngll > 16)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_mesh_structured_ibool_device: bad argument");
  const long long n1 = ngll - 1;
  const long long nglob = ((long long)nex * n1 + 1) * ((long long)ney * n1 + 1) * ((long long)nez * n1 + 1);
  if (nglob > 2147483647ll)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_mesh_structured_ibool_device: %lld nodes exceed int32", nglob);
  const long long total = (long long)nex * ney * nez * ngll * ngll * ngll;
  structured_ibool_kernel<<<grid_of(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      nex, ney, nez, ngll, ibool, total);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // extern "C"
