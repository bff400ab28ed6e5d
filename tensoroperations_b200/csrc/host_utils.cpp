// host_utils.cpp -- library-level C-ABI entry points that need no GPU:
// status text, structured mesh numbering, GLL operators, seeded synthetic fill.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.hpp"

namespace to_b200 {

namespace {
thread_local std::string g_last_error;
}

int set_error(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int device_sm_count(int* device_out) {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return -cuda_fail(e, "cudaGetDevice");
  }
  if (device_out) *device_out = dev;
  std::lock_guard<std::mutex> lock(mu);
  if (dev < static_cast<int>(cache.size()) && cache[dev] > 0) return cache[dev];
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return -cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
  if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
  cache[dev] = sms;
  return sms;
}

// splitmix64: the m-th output of the stream seeded with `seed`.
static inline uint64_t splitmix64_at(uint64_t seed, uint64_t m) {
  uint64_t z = seed + (m + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace to_b200

using namespace to_b200;

extern "C" {

int to_abi_version(void) { return TO_ABI_VERSION; }

const char* to_status_string(int status) {
  switch (status) {
    case TO_OK: return "TO_OK";
    case TO_ERR_INVALID_ARGUMENT: return "TO_ERR_INVALID_ARGUMENT";
    case TO_ERR_UNSUPPORTED: return "TO_ERR_UNSUPPORTED";
    case TO_ERR_CUDA: return "TO_ERR_CUDA";
    case TO_ERR_SCRATCH: return "TO_ERR_SCRATCH";
    case TO_ERR_ALIGNMENT: return "TO_ERR_ALIGNMENT";
    case TO_ERR_TIMEOUT: return "TO_ERR_TIMEOUT";
    case TO_ERR_COMM: return "TO_ERR_COMM";
    case TO_ERR_NO_DEVICE: return "TO_ERR_NO_DEVICE";
    case TO_ERR_GRID: return "TO_ERR_GRID";
    default: return "TO_ERR_UNKNOWN";
  }
}

const char* to_last_error(void) { return g_last_error.c_str(); }

int to_device_sm_count(void) {
  const int n = device_sm_count(nullptr);
  return n;
}

int to_mesh_structured_ibool(int32_t nex, int32_t ney, int32_t nez, int32_t ngll,
                             int32_t* ibool) {
  if (nex <= 0 || ney <= 0 || nez <= 0 || ngll < 2 || !ibool)
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "to_mesh_structured_ibool: bad mesh %d x %d x %d, ngll %d or null ibool",
                     nex, ney, nez, ngll);
  const int64_t n1 = ngll - 1;
  const int64_t nx = nex * n1 + 1, ny = ney * n1 + 1, nz = nez * n1 + 1;
  if (nx * ny * nz > INT32_MAX)
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "to_mesh_structured_ibool: %lld global nodes overflow int32",
                     static_cast<long long>(nx * ny * nz));
  const int64_t N = ngll, P = N * N * N;
  const int64_t nelem = static_cast<int64_t>(nex) * ney * nez;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < nelem; ++e) {
    const int64_t ex = e % nex, ey = (e / nex) % ney, ez = e / (static_cast<int64_t>(nex) * ney);
    int32_t* out = ibool + e * P;
    for (int64_t k = 0; k < N; ++k)
      for (int64_t j = 0; j < N; ++j)
        for (int64_t i = 0; i < N; ++i)
          out[(k * N + j) * N + i] = static_cast<int32_t>(
              ((ez * n1 + k) * ny + ey * n1 + j) * nx + ex * n1 + i);
  }
  return ok();
}

int to_gll_operators(int32_t ngll, double* nodes, double* weights, double* hprime,
                     double* hprimewgll) {
  if (ngll < 2 || ngll > 16)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_gll_operators: ngll %d outside [2,16]",
                     ngll);
  const int N = ngll, n = N - 1;
  // Legendre-Gauss-Lobatto nodes: Newton iteration on (1-x^2) P_n'(x) from the
  // Chebyshev-Gauss-Lobatto points, using the three-term Legendre recurrence.
  std::vector<double> x(N), Pn(N), Pn1(N);
  for (int i = 0; i < N; ++i) x[i] = -std::cos(M_PI * i / n);
  for (int it = 0; it < 100; ++it) {
    double delta = 0.0;
    for (int i = 0; i < N; ++i) {
      double p0 = 1.0, p1 = x[i];
      for (int k = 2; k <= n; ++k) {
        const double p2 = ((2.0 * k - 1.0) * x[i] * p1 - (k - 1.0) * p0) / k;
        p0 = p1;
        p1 = p2;
      }
      // p1 = P_n(x), p0 = P_{n-1}(x)
      const double xn = x[i] - (x[i] * p1 - p0) / (N * p1);
      delta = std::fmax(delta, std::fabs(xn - x[i]));
      x[i] = xn;
      Pn[i] = p1;
    }
    if (delta < 1e-16) break;
  }
  for (int i = 0; i < N; ++i) {  // final P_n at converged nodes
    double p0 = 1.0, p1 = x[i];
    for (int k = 2; k <= n; ++k) {
      const double p2 = ((2.0 * k - 1.0) * x[i] * p1 - (k - 1.0) * p0) / k;
      p0 = p1;
      p1 = p2;
    }
    Pn[i] = p1;
  }
  std::vector<double> w(N), D(N * N);
  for (int i = 0; i < N; ++i) w[i] = 2.0 / (static_cast<double>(n) * N * Pn[i] * Pn[i]);
  // Lagrange derivative at the nodes: D(i,p) = l_p'(x_i).
  for (int i = 0; i < N; ++i)
    for (int p = 0; p < N; ++p) {
      if (i != p)
        D[i * N + p] = Pn[i] / (Pn[p] * (x[i] - x[p]));
      else if (i == 0)
        D[i * N + p] = -0.25 * n * N;
      else if (i == n)
        D[i * N + p] = 0.25 * n * N;
      else
        D[i * N + p] = 0.0;
    }
  if (nodes) std::memcpy(nodes, x.data(), sizeof(double) * N);
  if (weights) std::memcpy(weights, w.data(), sizeof(double) * N);
  if (hprime) std::memcpy(hprime, D.data(), sizeof(double) * N * N);
  if (hprimewgll)
    for (int q = 0; q < N; ++q)
      for (int i = 0; i < N; ++i) hprimewgll[q * N + i] = D[q * N + i] * w[q];
  return ok();
}

int to_synth_fill_at(void* dst, int32_t dtype, int64_t first, int64_t n, uint64_t seed,
                     int32_t dist, double a, double b) {
  if (!dst || n < 0 || first < 0 || (dtype != TO_F32 && dtype != TO_F64) ||
      (dist != 0 && dist != 1))
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_synth_fill_at: bad argument");
  const double inv53 = 1.0 / 9007199254740992.0;  // 2^-53
  float* df = static_cast<float*>(dst);
  double* dd = static_cast<double*>(dst);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t m = static_cast<uint64_t>(first + i);
    double v;
    if (dist == 0) {
      const double u = static_cast<double>(splitmix64_at(seed, m) >> 11) * inv53;
      v = a + (b - a) * u;
    } else {
      const uint64_t m2 = 2 * m;
      const double u1 = (static_cast<double>(splitmix64_at(seed, m2) >> 11) + 1.0) * inv53;
      const double u2 = static_cast<double>(splitmix64_at(seed, m2 + 1) >> 11) * inv53;
      v = a + b * std::sqrt(-2.0 * std::log(u1)) * std::cos(2.0 * M_PI * u2);
    }
    if (dtype == TO_F32)
      df[i] = static_cast<float>(v);
    else
      dd[i] = v;
  }
  return ok();
}

int to_synth_fill(void* dst, int32_t dtype, int64_t n, uint64_t seed, int32_t dist,
                  double a, double b) {
  return to_synth_fill_at(dst, dtype, 0, n, seed, dist, a, b);
}

}  // extern "C"
