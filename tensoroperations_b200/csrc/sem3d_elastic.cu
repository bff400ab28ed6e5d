// sem3d_elastic.cu -- C-ABI plan / launch for the fused SEM 3D elastic operator.
#include <cstring>
#include <mutex>
#include <new>
#include <type_traits>

#include <cstdlib>

#include "common.hpp"
#include "sem3d_elastic.cuh"

namespace to_b200 {
__device__ int g_to_device_status = 0;
}

#include "sem3d_elastic_tma.cuh"
#include "sem3d_elastic_v3.cuh"
#include "sem3d_elastic_v5.cuh"
#include "sem3d_elastic_lo.cuh"
#include "sem3d_elastic_hc.cuh"

struct to_sem3d_plan {
  to_sem3d_desc desc;
  double H[16 * 16];
  double Hw[16 * 16];
  double w[16];
};

namespace to_b200 {
namespace {

// Elements per CTA batch for each instantiation: EB * N^2 threads per CTA.
template <typename T, int N>
struct Sem3dConfig;
template <>
struct Sem3dConfig<float, 5> {
  static constexpr int EB = 32;  // 800 threads, 25 warps
};
template <>
struct Sem3dConfig<double, 5> {
  static constexpr int EB = 16;  // 400 threads
};
template <>
struct Sem3dConfig<float, 8> {
  static constexpr int EB = 4;  // 256 threads
};
template <>
struct Sem3dConfig<double, 8> {
  static constexpr int EB = 2;  // 128 threads
};

template <typename T, int N>
size_t sem3d_smem_bytes() {
  constexpr int EB = Sem3dConfig<T, N>::EB;
  return sizeof(T) * (9ull * N * EB * N * N + 2ull * N * N) + 4ull * N * EB * N * N;
}

// Per-kernel launch state, configured once per device: the shared-memory
// opt-in and the number of resident CTAs per SM.
struct KernelSlot {
  std::mutex mu;
  unsigned long long configured = 0;  // bit per device id (< 64)
  int blocks_per_sm[64] = {0};
};

template <typename Kernel>
int configure(KernelSlot& slot, Kernel kernel, int dev, int threads, size_t smem, int* nb_out) {
  if (dev >= 64) return set_error(TO_ERR_UNSUPPORTED, "device id %d >= 64", dev);
  std::lock_guard<std::mutex> lock(slot.mu);
  if (!(slot.configured & (1ull << dev))) {
    int optin = 0;
    TO_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (smem > static_cast<size_t>(optin))
      return set_error(TO_ERR_SCRATCH, "kernel needs %zu B of shared memory, device allows %d",
                       smem, optin);
    TO_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    int nb = 0;
    TO_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, threads, smem));
    if (nb <= 0)
      return set_error(TO_ERR_SCRATCH, "kernel (%d threads, %zu B shared) cannot be resident",
                       threads, smem);
    slot.blocks_per_sm[dev] = nb;
    slot.configured |= (1ull << dev);
  }
  *nb_out = slot.blocks_per_sm[dev];
  return TO_OK;
}

template <typename T, int N>
Sem3dArgs<T, N> make_args(const to_sem3d_plan* plan, const to_sem3d_fields* fl) {
  Sem3dArgs<T, N> a;
  std::memset(&a, 0, sizeof(a));
  for (int c = 0; c < 3; ++c) {
    a.u[c] = static_cast<const T*>(fl->u[c]);
    a.f[c] = static_cast<T*>(fl->f[c]);
  }
  a.ibool = fl->ibool;
  a.u_norm2 = plan->desc.assembled ? fl->u_norm2 : nullptr;
  const void* m[kNumPointArrays] = {fl->xix,  fl->xiy,  fl->xiz,  fl->etax,
                                    fl->etay, fl->etaz, fl->gamx, fl->gamy,
                                    fl->gamz, fl->jac,  fl->l2m,  fl->mu};
  for (int q = 0; q < kNumPointArrays; ++q) a.m[q] = static_cast<const T*>(m[q]);
  a.nelem = plan->desc.nelem;
  for (int i = 0; i < N; ++i) {
    a.ops.w[i] = static_cast<T>(plan->w[i]);
    for (int p = 0; p < N; ++p) {
      a.ops.H[i][p] = static_cast<T>(plan->H[i * N + p]);
      a.ops.Hw[i][p] = static_cast<T>(plan->Hw[i * N + p]);
    }
  }
  return a;
}

// Every array the TMA kernel stages is 16-byte aligned.
bool staged_arrays_aligned(const to_sem3d_fields* fl, bool assembled) {
  const void* m[] = {fl->xix, fl->xiy, fl->xiz, fl->etax, fl->etay, fl->etaz,
                     fl->gamx, fl->gamy, fl->gamz, fl->jac, fl->l2m, fl->mu};
  for (const void* p : m)
    if (!aligned(p, 16)) return false;
  if (assembled) return aligned(fl->ibool, 16);
  for (int c = 0; c < 3; ++c)
    if (!aligned(fl->u[c], 16)) return false;
  return true;
}

// The register-streaming kernel (any 4-byte alignment).
template <typename T, int N, bool ASM>
int launch_ldg(const to_sem3d_plan* plan, const to_sem3d_fields* fl, cudaStream_t stream,
               int dev, int sms) {
  constexpr int EB = Sem3dConfig<T, N>::EB;
  constexpr int NT = EB * N * N;
  const size_t smem = sem3d_smem_bytes<T, N>();
  auto kernel = sem3d_elastic_kernel<T, N, EB, ASM>;
  static KernelSlot slot;
  int nb = 0;
  if (int st = configure(slot, kernel, dev, NT, smem, &nb)) return st;
  Sem3dArgs<T, N> a = make_args<T, N>(plan, fl);
  bool pf = ASM ? aligned(fl->ibool, 16) : true;
  for (int q = 0; q < kNumPointArrays; ++q) pf = pf && aligned(a.m[q], 16);
  if (!ASM)
    for (int c = 0; c < 3; ++c) pf = pf && aligned(fl->u[c], 16);
  a.prefetch = pf ? 1 : 0;
  const long long nbatch = (plan->desc.nelem + EB - 1) / EB;
  const long long cap = static_cast<long long>(sms) * nb;
  const int grid = static_cast<int>(nbatch < cap ? nbatch : cap);
  kernel<<<grid, NT, smem, stream>>>(a);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

// The TMA-staged kernel (all staged arrays 16-byte aligned).
template <typename T, int N, int EB, int MINB, bool ASM>
int launch_tma(const to_sem3d_plan* plan, const to_sem3d_fields* fl, cudaStream_t stream,
               int dev, int sms) {
  constexpr int NT = EB * N * N;
  const size_t smem = Sem3dTmaLayout<T, N, EB, ASM>::kTotal;
  auto kernel = sem3d_elastic_tma_kernel<T, N, EB, MINB, ASM>;
  static KernelSlot slot;
  int nb = 0;
  if (int st = configure(slot, kernel, dev, NT, smem, &nb)) return st;
  Sem3dArgs<T, N> a = make_args<T, N>(plan, fl);
  a.prefetch = 1;
  const long long nbatch = (plan->desc.nelem + EB - 1) / EB;
  const long long cap = static_cast<long long>(sms) * nb;
  const int grid = static_cast<int>(nbatch < cap ? nbatch : cap);
  kernel<<<grid, NT, smem, stream>>>(a);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

// The point-pair / gather-pipelined kernel (f32, staged arrays 16-byte aligned).
template <int N, int EB, int MINB, bool ASM>
int launch_v3(const to_sem3d_plan* plan, const to_sem3d_fields* fl, cudaStream_t stream,
              int dev, int sms) {
  constexpr int NT = EB * N * N;
  const size_t smem = Sem3dV3Layout<N, EB, ASM>::kTotal;
  auto kernel = sem3d_elastic_v3_kernel<N, EB, MINB, ASM>;
  static KernelSlot slot;
  int nb = 0;
  if (int st = configure(slot, kernel, dev, NT, smem, &nb)) return st;
  Sem3dArgs<float, N> a = make_args<float, N>(plan, fl);
  a.prefetch = 1;
  const long long nbatch = (plan->desc.nelem + EB - 1) / EB;
  const long long cap = static_cast<long long>(sms) * nb;
  const int grid = static_cast<int>(nbatch < cap ? nbatch : cap);
  kernel<<<grid, NT, smem, stream>>>(a);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

// The line-owner kernel (f32 NGLL 5, staged arrays 16-byte aligned).
template <int EB, int MINB, bool ASM, bool IL = false, int OPT = kV5Packed>
int launch_v5(const to_sem3d_plan* plan, const to_sem3d_fields* fl, cudaStream_t stream,
              int dev, int sms) {
  constexpr int NT = EB * 25;
  const size_t smem = Sem3dV5Layout<EB, ASM>::kTotal;
  auto kernel = sem3d_elastic_v5_kernel<EB, MINB, ASM, IL, OPT>;
  static KernelSlot slot;
  int nb = 0;
  if (int st = configure(slot, kernel, dev, NT, smem, &nb)) return st;
  Sem3dV5Args a{};
  a.a = make_args<float, 5>(plan, fl);
  a.a.prefetch = 1;
  for (int i = 0; i < 5; ++i)
    for (int p = 0; p < 5; ++p) {
      a.H2[i][p] = make_float2(a.a.ops.H[i][p], a.a.ops.H[i][p]);
      a.Hw2[i][p] = make_float2(a.a.ops.Hw[i][p], a.a.ops.Hw[i][p]);
    }
  const long long nbatch = (plan->desc.nelem + EB - 1) / EB;
  const long long cap = static_cast<long long>(sms) * nb;
  const int grid = static_cast<int>(nbatch < cap ? nbatch : cap);
  kernel<<<grid, NT, smem, stream>>>(a);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

// The line-owner kernel over up to two element ranges with ticketed batches
// (f32 NGLL 5, assembled, either node layout; the z-slab operator's launches).
template <bool IL, int OPT = kV5Packed | kV5Ranges>
int launch_v5_ranges(const to_sem3d_plan* plan, const to_sem3d_fields* fl, const int64_t first[2],
                     const int64_t count[2], unsigned long long* ticket, cudaStream_t stream,
                     int dev, int sms) {
  constexpr int EB = 8, NT = EB * 25;
  const size_t smem = Sem3dV5Layout<EB, true>::kTotal;
  auto kernel = sem3d_elastic_v5_kernel<EB, 3, true, IL, OPT>;
  static KernelSlot slot;
  int nb = 0;
  if (int st = configure(slot, kernel, dev, NT, smem, &nb)) return st;
  Sem3dV5Args a{};
  a.a = make_args<float, 5>(plan, fl);
  a.a.prefetch = 1;
  for (int i = 0; i < 5; ++i)
    for (int p = 0; p < 5; ++p) {
      a.H2[i][p] = make_float2(a.a.ops.H[i][p], a.a.ops.H[i][p]);
      a.Hw2[i][p] = make_float2(a.a.ops.Hw[i][p], a.a.ops.Hw[i][p]);
    }
  long long total = 0;
  for (int r = 0; r < 2; ++r) {
    a.rg.first[r] = first[r];
    a.rg.count[r] = count[r];
    a.rg.nb[r] = (count[r] + EB - 1) / EB;
    total += a.rg.nb[r];
  }
  a.rg.ticket = ticket;
  if (total == 0) return ok();
  const long long cap = static_cast<long long>(sms) * nb;
  const int grid = static_cast<int>(total < cap ? total : cap);
  kernel<<<grid, NT, smem, stream>>>(a);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

// The line-owner kernel with geometry from global memory (NGLL 8).
template <typename T, int N, int EB, int MINB, bool ASM>
int launch_lo(const to_sem3d_plan* plan, const to_sem3d_fields* fl, cudaStream_t stream,
              int dev, int sms) {
  constexpr int NT = EB * N * N;
  const size_t smem = Sem3dLoLayout<T, N, EB>::kTotal;
  auto kernel = sem3d_elastic_lo_kernel<T, N, EB, MINB, ASM>;
  static KernelSlot slot;
  int nb = 0;
  if (int st = configure(slot, kernel, dev, NT, smem, &nb)) return st;
  Sem3dArgs<T, N> a = make_args<T, N>(plan, fl);
  a.prefetch = staged_arrays_aligned(fl, ASM) ? 1 : 0;
  const long long nbatch = (plan->desc.nelem + EB - 1) / EB;
  const long long cap = static_cast<long long>(sms) * nb;
  const int grid = static_cast<int>(nbatch < cap ? nbatch : cap);
  kernel<<<grid, NT, smem, stream>>>(a);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

// The half-column line-owner kernel (NGLL 8): two owners per column.
template <typename T, int EB, int MINB, bool ASM, bool PIPE = false, bool IBPIPE = false,
          bool UPIPE = false, bool GEARLY = false>
int launch_hc(const to_sem3d_plan* plan, const to_sem3d_fields* fl, cudaStream_t stream,
              int dev, int sms) {
  constexpr int NT = EB * 128;
  const size_t smem = Sem3dHcLayout<T, EB>::kTotal;
  Sem3dArgs<T, 8> a = make_args<T, 8>(plan, fl);
  // L2 bulk prefetch of this CTA's next batches (TO_SEM3D_HC_PREFETCH batches
  // ahead, 0..3): off by default -- 128^3 f64 power step 48.5 ms without it,
  // 50.4 ms one batch ahead, 56.2 ms two (evict-first hints changed nothing)
  static const int distance = [] {
    const char* e = std::getenv("TO_SEM3D_HC_PREFETCH");
    const int d = e ? std::atoi(e) : 0;
    return d < 0 ? 0 : (d > 3 ? 3 : d);
  }();
  a.prefetch = staged_arrays_aligned(fl, ASM) ? distance : 0;
  auto go = [&](auto kernel, KernelSlot& slot) -> int {
    int nb = 0;
    if (int st = configure(slot, kernel, dev, NT, smem, &nb)) return st;
    const long long nbatch = (plan->desc.nelem + EB - 1) / EB;
    const long long cap = static_cast<long long>(sms) * nb;
    const int grid = static_cast<int>(nbatch < cap ? nbatch : cap);
    kernel<<<grid, NT, smem, stream>>>(a);
    TO_CUDA_TRY(cudaGetLastError());
    return ok();
  };
  static KernelSlot slot, slot_scaled;
  if (ASM && a.u_norm2)
    return go(sem3d_elastic_hc_kernel<T, EB, MINB, ASM, PIPE, true, IBPIPE, UPIPE, GEARLY>,
              slot_scaled);
  return go(sem3d_elastic_hc_kernel<T, EB, MINB, ASM, PIPE, false, IBPIPE, UPIPE, GEARLY>, slot);
}

// Kernel variant for f32 NGLL 5 (TO_SEM3D_VARIANT; default 5):
//   0 point-pair pipelined kernel, 8 elements x 2 CTAs/SM
//   1 TMA-staged kernel, 8 elements x 2 CTAs/SM
//   2 register-streaming kernel
//   3 point-pair pipelined kernel, 4 elements x 4 CTAs/SM
//   4 point-pair pipelined kernel, 16 elements x 1 CTA/SM
//   5 line-owner kernel, 8 elements x 3 CTAs/SM
//   6 line-owner kernel, 4 elements x 5 CTAs/SM
//   7 line-owner kernel with scalar (unpacked) contractions
int sem3d_f32_variant() {
  static const int v = [] {
    const char* e = std::getenv("TO_SEM3D_VARIANT");
    return e ? std::atoi(e) : 5;
  }();
  return v;
}

// Warp-aggregated scatter-add in the ticketed launches (TO_SEM3D_WARP_AGG=1).
bool sem3d_warp_agg() {
  static const bool on = [] {
    const char* e = std::getenv("TO_SEM3D_WARP_AGG");
    return e && std::atoi(e) != 0;
  }();
  return on;
}

template <typename T, int N, bool ASM>
int launch_sem3d(const to_sem3d_plan* plan, const to_sem3d_fields* fl, cudaStream_t stream) {
  int dev = 0;
  const int sms = device_sm_count(&dev);
  if (sms <= 0) return -sms;
  if constexpr (std::is_same_v<T, float> && N == 5 && ASM) {
    // u_norm2 (a power iteration's deferred normalisation) is read by the
    // NGLL-8 kernels and the generic one, not by the NGLL-5 line-owner kernel
    if (fl->u_norm2) {
      if (plan->desc.node_layout == 1)
        return set_error(TO_ERR_UNSUPPORTED, "to_sem3d_apply: u_norm2 with interleaved nodes");
      return launch_ldg<T, N, ASM>(plan, fl, stream, dev, sms);
    }
    if (plan->desc.node_layout == 1) {
      if (!staged_arrays_aligned(fl, ASM))
        return set_error(TO_ERR_ALIGNMENT,
                         "to_sem3d_apply: interleaved nodes need 16-byte aligned per-point arrays");
      return launch_v5<8, 3, true, true>(plan, fl, stream, dev, sms);
    }
  }
  if constexpr (std::is_same_v<T, float> && N == 5) {
    const int v = sem3d_f32_variant();
    if (v != 2 && staged_arrays_aligned(fl, ASM)) {
      if (v == 1) return launch_tma<T, N, 8, 2, ASM>(plan, fl, stream, dev, sms);
      if (v == 3) return launch_v3<N, 4, 4, ASM>(plan, fl, stream, dev, sms);
      if (v == 4) return launch_v3<N, 16, 1, ASM>(plan, fl, stream, dev, sms);
      if (v == 6) return launch_v5<4, ASM ? 5 : 4, ASM>(plan, fl, stream, dev, sms);
      if (v == 0) return launch_v3<N, 8, 2, ASM>(plan, fl, stream, dev, sms);
      if (v == 7) return launch_v5<8, ASM ? 3 : 2, ASM, false, 0>(plan, fl, stream, dev, sms);
      return launch_v5<8, ASM ? 3 : 2, ASM>(plan, fl, stream, dev, sms);
    }
  }
  if constexpr (N == 8) {
    // NGLL 8: fp64 takes the half-column kernel (2 owners per column, 16
    // resident warps per SM: 59.5 vs 66.6 ms per 128^3 power step), fp32 the
    // whole-column one (the half-column kernel measured 1.91 vs 1.59 ms at
    // E=196,608); TO_SEM3D_VARIANT 10 / 12 force one or the other, 2 the
    // streaming kernel
    // (the half-column kernel loads the next point's geometry ahead: 58.7 vs
    // 60.3 ms per 128^3 power step; TO_SEM3D_VARIANT 14 keeps per-point loads)
    const int v = sem3d_f32_variant();
    if (v == 14)
      return launch_hc<T, 2, sizeof(T) == 8 ? 2 : 3, ASM, false>(plan, fl, stream, dev, sms);
    // fp64 assembled: the next batch's node ids loaded during C1 and its u
    // gathered during C2, so phase A waits on no global load (per 128^3 power
    // step: 49.3 ms with both in phase A -- TO_SEM3D_VARIANT 13 --, 47.3-47.9 ms
    // with the node ids ahead -- 17 --, 46.0-46.1 ms with both)
    if (ASM && sizeof(T) == 8 && v == 17)
      return launch_hc<T, 2, 2, ASM, true, true>(plan, fl, stream, dev, sms);
    // ... and the first point's geometry requested before B1 (43.5-43.6 vs
    // 43.9-44.0 ms on one box; TO_SEM3D_VARIANT 18 requests it at B2)
    if (ASM && sizeof(T) == 8 && v == 18)
      return launch_hc<T, 2, 2, ASM, true, true, true>(plan, fl, stream, dev, sms);
    if (ASM && sizeof(T) == 8 && v != 2 && v != 10 && v != 12 && v != 13 && v != 14)
      return launch_hc<T, 2, 2, ASM, true, true, true, true>(plan, fl, stream, dev, sms);
    if (v == 10 || v == 13 || (sizeof(T) == 8 && v != 2 && v != 12))
      return launch_hc<T, 2, sizeof(T) == 8 ? 2 : 3, ASM, true>(plan, fl, stream, dev, sms);
    if (v != 2)
      return launch_lo<T, N, 2, sizeof(T) == 8 ? 2 : 3, ASM>(plan, fl, stream, dev, sms);
  }
  return launch_ldg<T, N, ASM>(plan, fl, stream, dev, sms);
}

template <typename T, int N>
int apply_typed(const to_sem3d_plan* plan, const to_sem3d_fields* fl, int accumulate,
                cudaStream_t stream) {
  const size_t al = sizeof(T);
  const bool il = plan->desc.node_layout == 1;
  const void* ptrs[] = {fl->u[0], fl->u[1], fl->u[2], fl->f[0], fl->f[1], fl->f[2],
                        fl->xix,  fl->xiy,  fl->xiz,  fl->etax, fl->etay, fl->etaz,
                        fl->gamx, fl->gamy, fl->gamz, fl->jac,  fl->l2m,  fl->mu};
  for (int q = 0; q < 18; ++q) {
    const void* p = ptrs[q];
    if (il && (q == 1 || q == 2 || q == 4 || q == 5)) continue;  // one interleaved array
    if (!p) return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_apply: null field pointer");
    const size_t need = (il && (q == 0 || q == 3)) ? 16 : al;
    if (!aligned(p, need))
      return set_error(TO_ERR_ALIGNMENT, "to_sem3d_apply: field pointer %p not %zu-byte aligned",
                       p, need);
  }
  if (fl->u_norm2 && !plan->desc.assembled)
    return set_error(TO_ERR_UNSUPPORTED, "to_sem3d_apply: u_norm2 needs assembled mode");
  if (fl->u_norm2 && !aligned(fl->u_norm2, 8))
    return set_error(TO_ERR_ALIGNMENT, "to_sem3d_apply: u_norm2 not 8-byte aligned");
  if (plan->desc.assembled) {
    if (!fl->ibool)
      return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_apply: assembled mode needs ibool");
    if (!aligned(fl->ibool, 4))
      return set_error(TO_ERR_ALIGNMENT, "to_sem3d_apply: ibool not 4-byte aligned");
    if (!accumulate) {
      if (il)
        TO_CUDA_TRY(cudaMemsetAsync(fl->f[0], 0, sizeof(T) * 4 * plan->desc.nglob, stream));
      else
        for (int c = 0; c < 3; ++c)
          TO_CUDA_TRY(cudaMemsetAsync(fl->f[c], 0, sizeof(T) * plan->desc.nglob, stream));
    }
    return launch_sem3d<T, N, true>(plan, fl, stream);
  }
  return launch_sem3d<T, N, false>(plan, fl, stream);
}

// Every built (dtype, NGLL) pair.
int apply_dispatch(const to_sem3d_plan* plan, const to_sem3d_fields* fl, int accumulate,
                   cudaStream_t s, const char* who) {
  const to_sem3d_desc& d = plan->desc;
  if (d.ngll == 5 && d.dtype == TO_F32) return apply_typed<float, 5>(plan, fl, accumulate, s);
  if (d.ngll == 5 && d.dtype == TO_F64) return apply_typed<double, 5>(plan, fl, accumulate, s);
  if (d.ngll == 8 && d.dtype == TO_F32) return apply_typed<float, 8>(plan, fl, accumulate, s);
  if (d.ngll == 8 && d.dtype == TO_F64) return apply_typed<double, 8>(plan, fl, accumulate, s);
  return set_error(TO_ERR_UNSUPPORTED, "%s: ngll %d dtype %d not built", who, d.ngll, d.dtype);
}

}  // namespace

// Element ranges [first[r], first[r] + count[r]) of the plan's elements (r = 0, 1;
// a zero count skips a range), scattered into f without zeroing it.  f32 NGLL 5
// assembled plans with 16-byte aligned per-point arrays run as ONE launch of the
// line-owner kernel with ticketed batches (`ticket` must be zero on `stream`
// when the launch starts); other plans run to_sem3d_apply_elements per range.
const to_sem3d_desc* sem3d_plan_desc(const to_sem3d_plan* plan) { return &plan->desc; }

int sem3d_apply_ranges(const to_sem3d_plan* plan, const to_sem3d_fields* fl,
                       const int64_t first[2], const int64_t count[2],
                       unsigned long long* ticket, cudaStream_t stream) {
  const to_sem3d_desc& d = plan->desc;
  for (int r = 0; r < 2; ++r)
    if (first[r] < 0 || count[r] < 0 || first[r] > d.nelem || count[r] > d.nelem - first[r])
      return set_error(TO_ERR_INVALID_ARGUMENT, "sem3d ranges: range %d outside the plan", r);
  // bulk copies need every batch's per-point rows 16-byte aligned: element
  // e starts at e * 500 bytes, so each range must start at a multiple of 4
  bool starts4 = true;
  for (int r = 0; r < 2; ++r)
    if (count[r] && first[r] % 4 != 0) starts4 = false;
  const bool il = d.node_layout == 1;
  if (fl->u_norm2 && il)
    return set_error(TO_ERR_UNSUPPORTED, "sem3d ranges: u_norm2 with interleaved nodes");
  const bool fast = !fl->u_norm2 && d.dtype == TO_F32 && d.ngll == 5 && d.assembled &&
                    ticket != nullptr && (il || sem3d_f32_variant() == 5) && starts4 &&
                    staged_arrays_aligned(fl, true) && aligned(ticket, 8);
  if (il && !fast)
    return set_error(TO_ERR_ALIGNMENT,
                     "sem3d ranges: interleaved nodes need 16-byte aligned per-point arrays and "
                     "ranges starting at multiples of 4 elements");
  if (fast) {
    int dev = 0;
    const int sms = device_sm_count(&dev);
    if (sms <= 0) return -sms;
    for (int q = 0; q < 6; ++q) {
      if (il && q % 3 != 0) continue;  // one interleaved array each
      if (!(q < 3 ? fl->u[q] : fl->f[q - 3]))
        return set_error(TO_ERR_INVALID_ARGUMENT, "sem3d ranges: null u / f");
    }
    if (il && (!aligned(fl->u[0], 16) || !aligned(fl->f[0], 16)))
      return set_error(TO_ERR_ALIGNMENT, "sem3d ranges: interleaved u / f not 16-byte aligned");
    if (!fl->ibool) return set_error(TO_ERR_INVALID_ARGUMENT, "sem3d ranges: null ibool");
    if (sem3d_warp_agg()) {
      constexpr int kAggOpt = kV5Packed | kV5Ranges | kV5WarpAgg;
      if (il) return launch_v5_ranges<true, kAggOpt>(plan, fl, first, count, ticket, stream, dev, sms);
      return launch_v5_ranges<false, kAggOpt>(plan, fl, first, count, ticket, stream, dev, sms);
    }
    if (il) return launch_v5_ranges<true>(plan, fl, first, count, ticket, stream, dev, sms);
    return launch_v5_ranges<false>(plan, fl, first, count, ticket, stream, dev, sms);
  }
  for (int r = 0; r < 2; ++r)
    if (count[r])
      if (int st = to_sem3d_apply_elements(plan, fl, first[r], count[r], stream)) return st;
  return ok();
}

}  // namespace to_b200

using namespace to_b200;

extern "C" {

int to_sem3d_plan_create(const to_sem3d_desc* desc, to_sem3d_plan** plan) {
  if (!desc || !plan) return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_plan_create: null");
  *plan = nullptr;
  if (desc->dtype != TO_F32 && desc->dtype != TO_F64)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_plan_create: dtype %d", desc->dtype);
  if (desc->ngll < 2 || desc->ngll > 16)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_plan_create: ngll %d", desc->ngll);
  const bool built = (desc->ngll == 5 || desc->ngll == 8);
  if (!built)
    return set_error(TO_ERR_UNSUPPORTED, "to_sem3d_plan_create: ngll %d (%s) not built",
                     desc->ngll, desc->dtype == TO_F32 ? "f32" : "f64");
  if (desc->nelem < 0)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_plan_create: nelem %lld < 0",
                     static_cast<long long>(desc->nelem));
  if (desc->node_layout != 0 &&
      !(desc->node_layout == 1 && desc->assembled && desc->dtype == TO_F32 && desc->ngll == 5))
    return set_error(TO_ERR_UNSUPPORTED,
                     "to_sem3d_plan_create: node_layout %d (interleaved nodes: assembled f32 NGLL 5)",
                     desc->node_layout);
  if (desc->assembled && (desc->nglob <= 0 || desc->nglob > INT32_MAX))
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "to_sem3d_plan_create: assembled mode needs 0 < nglob <= INT32_MAX");
  if (!desc->hprime || !desc->hprimewgll || !desc->wgll)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_plan_create: null operator array");
  to_sem3d_plan* p = new (std::nothrow) to_sem3d_plan;
  if (!p) return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_plan_create: out of host memory");
  std::memset(p, 0, sizeof(*p));
  p->desc = *desc;
  p->desc.hprime = p->H;
  p->desc.hprimewgll = p->Hw;
  p->desc.wgll = p->w;
  const int N = desc->ngll;
  std::memcpy(p->H, desc->hprime, sizeof(double) * N * N);
  std::memcpy(p->Hw, desc->hprimewgll, sizeof(double) * N * N);
  std::memcpy(p->w, desc->wgll, sizeof(double) * N);
  *plan = p;
  return ok();
}

int to_sem3d_plan_destroy(to_sem3d_plan* plan) {
  delete plan;
  return ok();
}

int to_sem3d_apply(const to_sem3d_plan* plan, const to_sem3d_fields* fields,
                   int32_t accumulate, void* stream) {
  if (!plan || !fields) return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_apply: null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const to_sem3d_desc& d = plan->desc;
  if (d.nelem == 0) return ok();
  return apply_dispatch(plan, fields, accumulate, s, "to_sem3d_apply");
}

int to_sem3d_apply_elements(const to_sem3d_plan* plan, const to_sem3d_fields* fields,
                            int64_t first, int64_t count, void* stream) {
  if (!plan || !fields) return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_apply_elements: null");
  const to_sem3d_desc& d = plan->desc;
  if (first < 0 || count < 0 || first > d.nelem || count > d.nelem - first)
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "to_sem3d_apply_elements: range [%lld, %lld) outside [0, %lld)",
                     static_cast<long long>(first), static_cast<long long>(first + count),
                     static_cast<long long>(d.nelem));
  if (count == 0) return ok();
  // The same operator on the sub-batch: every per-element array (and, in
  // element-local mode, u and f) starts `first` elements in; assembled u and f
  // stay global.  The sub-plan never zeroes f.
  to_sem3d_plan sub = *plan;
  sub.desc.nelem = count;
  to_sem3d_fields fl = *fields;
  const size_t P = static_cast<size_t>(d.ngll) * d.ngll * d.ngll;
  const size_t vb = d.dtype == TO_F64 ? 8 : 4;
  const size_t off = static_cast<size_t>(first) * P;
  auto shift = [&](const void* p, size_t bytes) -> const void* {
    return p ? static_cast<const char*>(p) + off * bytes : p;
  };
  fl.xix = shift(fl.xix, vb);   fl.xiy = shift(fl.xiy, vb);   fl.xiz = shift(fl.xiz, vb);
  fl.etax = shift(fl.etax, vb); fl.etay = shift(fl.etay, vb); fl.etaz = shift(fl.etaz, vb);
  fl.gamx = shift(fl.gamx, vb); fl.gamy = shift(fl.gamy, vb); fl.gamz = shift(fl.gamz, vb);
  fl.jac = shift(fl.jac, vb);   fl.l2m = shift(fl.l2m, vb);   fl.mu = shift(fl.mu, vb);
  if (d.assembled) {
    fl.ibool = static_cast<const int32_t*>(shift(fl.ibool, 4));
  } else {
    for (int c = 0; c < 3; ++c) {
      fl.u[c] = shift(fl.u[c], vb);
      fl.f[c] = const_cast<void*>(shift(fl.f[c], vb));
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return apply_dispatch(&sub, &fl, 1, s, "to_sem3d_apply_elements");
}

int to_device_status(int32_t reset) {
  int v = 0;
  TO_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_to_device_status, sizeof(int)));
  if (reset && v) {
    const int z = 0;
    TO_CUDA_TRY(cudaMemcpyToSymbol(g_to_device_status, &z, sizeof(int)));
  }
  int w = 0;
  if (int st = chain_device_status(reset, &w)) return st;
  if (!v) v = w;
  if (v) return set_error(v, "a kernel reported %s", to_status_string(v));
  return ok();
}

double to_sem3d_algorithmic_bytes(const to_sem3d_plan* plan) {
  if (!plan) return 0.0;
  const to_sem3d_desc& d = plan->desc;
  const double s = d.dtype == TO_F64 ? 8.0 : 4.0;
  const double P = static_cast<double>(d.ngll) * d.ngll * d.ngll;
  const double E = static_cast<double>(d.nelem);
  if (d.assembled) return E * P * (12.0 * s + 4.0) + static_cast<double>(d.nglob) * 3.0 * s * 2.0;
  return E * P * (12.0 * s + 3.0 * s * 2.0);
}

double to_sem3d_flops(const to_sem3d_plan* plan) {
  if (!plan) return 0.0;
  const to_sem3d_desc& d = plan->desc;
  const double P = static_cast<double>(d.ngll) * d.ngll * d.ngll;
  return static_cast<double>(d.nelem) * P * (36.0 * d.ngll + 159.0);
}

}  // extern "C"
