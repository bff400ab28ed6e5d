// sem3d_slab.cu -- interface-plane kernels of the z-slab (multi-GPU) operator.
//
// A rank owns a contiguous z-range of elements and the node planes that range
// touches; its first and last node planes are shared with the neighbouring
// ranks.  After the rank's elements have scattered into its f, the shared
// planes hold partial sums: each rank packs its planes (3 components, one
// contiguous nx*ny range each), exchanges them with the neighbour, and adds
// the neighbour's partial sums in.  Both kernels are single grid-stride
// passes over 3 x plane values (HBM-bound, a few microseconds).
#include "common.hpp"

namespace to_b200 {
namespace {

template <typename T>
struct Planes3 {
  T* f[3];
};

template <typename T>
__global__ void halo_pack_kernel(Planes3<T> src, int64_t offset, int64_t n, T* __restrict__ buf) {
  const int64_t total = 3 * n;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(t / n);
    buf[t] = src.f[c][offset + (t - c * n)];
  }
}

template <typename T>
__global__ void halo_accumulate_kernel(Planes3<T> dst, int64_t offset, int64_t n,
                                       const T* __restrict__ buf) {
  const int64_t total = 3 * n;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(t / n);
    dst.f[c][offset + (t - c * n)] += buf[t];
  }
}

template <typename T>
__global__ void flat_accumulate_kernel(T* __restrict__ dst, const T* __restrict__ buf, int64_t n) {
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < n;
       t += int64_t(gridDim.x) * blockDim.x)
    dst[t] += buf[t];
}

// u4[i] = (u0[i], u1[i], u2[i], 0) and back: the interleaved node layout
// (one 16-byte node per point gather / scatter) from and to one array per
// component.
__global__ void interleave_kernel(float4* __restrict__ out, const float* __restrict__ x,
                                  const float* __restrict__ y, const float* __restrict__ z,
                                  int64_t n) {
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < n;
       t += int64_t(gridDim.x) * blockDim.x)
    out[t] = make_float4(x[t], y[t], z[t], 0.f);
}

__global__ void deinterleave_kernel(float* __restrict__ x, float* __restrict__ y,
                                    float* __restrict__ z, const float4* __restrict__ in, int64_t n) {
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < n;
       t += int64_t(gridDim.x) * blockDim.x) {
    const float4 v = in[t];
    x[t] = v.x;
    y[t] = v.y;
    z[t] = v.z;
  }
}

int grid_for(int64_t total) {
  int dev = 0;
  const int sms = device_sm_count(&dev);
  const int64_t want = (total + 255) / 256;
  const int64_t cap = sms > 0 ? 4ll * sms : 592;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

template <typename T>
int launch_pack(void* const f[3], int64_t offset, int64_t n, void* buf, cudaStream_t s, bool pack) {
  Planes3<T> p;
  for (int c = 0; c < 3; ++c) {
    if (!f[c]) return set_error(TO_ERR_INVALID_ARGUMENT, "halo: null f[%d]", c);
    if (!aligned(f[c], sizeof(T))) return set_error(TO_ERR_ALIGNMENT, "halo: f[%d] misaligned", c);
    p.f[c] = static_cast<T*>(f[c]);
  }
  if (!aligned(buf, sizeof(T))) return set_error(TO_ERR_ALIGNMENT, "halo: buffer misaligned");
  const int grid = grid_for(3 * n);
  if (pack)
    halo_pack_kernel<T><<<grid, 256, 0, s>>>(p, offset, n, static_cast<T*>(buf));
  else
    halo_accumulate_kernel<T><<<grid, 256, 0, s>>>(p, offset, n, static_cast<const T*>(buf));
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

int halo_common(int32_t dtype, void* const f[3], int64_t offset, int64_t n, const void* buf,
                void* stream, bool pack, const char* who) {
  if (!f || !buf) return set_error(TO_ERR_INVALID_ARGUMENT, "%s: null", who);
  if (offset < 0 || n < 0) return set_error(TO_ERR_INVALID_ARGUMENT, "%s: bad range", who);
  if (n == 0) return ok();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* b = const_cast<void*>(buf);
  if (dtype == TO_F32) return launch_pack<float>(f, offset, n, b, s, pack);
  if (dtype == TO_F64) return launch_pack<double>(f, offset, n, b, s, pack);
  return set_error(TO_ERR_INVALID_ARGUMENT, "%s: dtype %d", who, dtype);
}

}  // namespace

// dst[t] += buf[t] for t < n (one contiguous range; the interleaved layout's
// shared plane is 4 * plane_nodes consecutive values).
int flat_accumulate(int32_t dtype, void* dst, const void* buf, int64_t n, cudaStream_t s) {
  if (!dst || !buf || n < 0) return set_error(TO_ERR_INVALID_ARGUMENT, "flat accumulate: bad argument");
  if (n == 0) return ok();
  const int grid = grid_for(n);
  if (dtype == TO_F32)
    flat_accumulate_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(dst),
                                                       static_cast<const float*>(buf), n);
  else
    flat_accumulate_kernel<double><<<grid, 256, 0, s>>>(static_cast<double*>(dst),
                                                        static_cast<const double*>(buf), n);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // namespace to_b200

using namespace to_b200;

extern "C" {

int to_sem3d_halo_pack(int32_t dtype, void* const f[3], int64_t offset, int64_t n, void* buf,
                       void* stream) {
  return halo_common(dtype, f, offset, n, buf, stream, true, "to_sem3d_halo_pack");
}

int to_sem3d_halo_accumulate(int32_t dtype, void* const f[3], int64_t offset, int64_t n,
                             const void* buf, void* stream) {
  return halo_common(dtype, f, offset, n, buf, stream, false, "to_sem3d_halo_accumulate");
}

int to_nodes_interleave(const float* const x[3], float* out, int64_t n, void* stream) {
  if (!x || !x[0] || !x[1] || !x[2] || !out || n < 0)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_nodes_interleave: bad argument");
  if (!aligned(out, 16)) return set_error(TO_ERR_ALIGNMENT, "to_nodes_interleave: out not 16-byte aligned");
  if (n == 0) return ok();
  interleave_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<float4*>(out), x[0], x[1], x[2], n);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

int to_nodes_deinterleave(const float* in, float* const x[3], int64_t n, void* stream) {
  if (!x || !x[0] || !x[1] || !x[2] || !in || n < 0)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_nodes_deinterleave: bad argument");
  if (!aligned(in, 16)) return set_error(TO_ERR_ALIGNMENT, "to_nodes_deinterleave: in not 16-byte aligned");
  if (n == 0) return ok();
  deinterleave_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x[0], x[1], x[2], reinterpret_cast<const float4*>(in), n);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // extern "C"
