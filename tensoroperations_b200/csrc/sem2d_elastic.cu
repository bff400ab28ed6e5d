// sem2d_elastic.cu -- 2D elastic P-SV spectral-element stiffness, NGLL 8, f32,
// element-local: the operator of the reference's 2D benchmark
// (benchmarks/sem_stiffness/bench_sem_stiffness.cpp: physics :319-357,
// host loop :1335-1385):
//   a_c = sum_p H(i,p) u_c(j,p)      g_c = sum_p H(j,p) u_c(p,i)
//   ds = [[a0 ax + g0 px, a0 az + g0 pz], [a1 ax + g1 px, a1 az + g1 pz]]
//   sigma: s00 = l2m ds00 + lam ds11, s11 = lam ds00 + l2m ds11,
//          s01 = s10 = mu (ds01 + ds10), lam = l2m - 2 mu
//   Fx_c = J (s_c0 ax + s_c1 az),  Fg_c = J (s_c0 px + s_c1 pz)
//   f_c(j,i) = w_j sum_q Hw(q,i) Fx_c(j,q) + w_i sum_q Hw(q,j) Fg_c(q,i)
// Arrays are [E][j][i] (i fastest), one per quantity, like the reference's
// View<float*[8][8], LayoutRight>.
//
// Mapping: one thread per element ROW (8 threads per element), so a warp holds
// four whole elements and every exchange is warp-local (__syncwarp only).
//   * a row of 8 floats is 32 B: each thread moves its row of every array with
//     two 128-bit loads / stores, consecutive threads consecutive rows;
//   * xi contractions (along i) and the xi divergence run in registers;
//   * gamma contractions: the row owner writes its row to the warp's shared
//     buffer, the thread then acts as COLUMN owner (column = its row index),
//     reads that column once, produces all 8 outputs of the column and writes
//     them back in place; the row owner reads its row of results.  Rows are
//     12 floats apart (128-bit row accesses of 8 lanes hit distinct banks) and
//     element slots 200 floats apart (= 8 mod 32: column accesses of the
//     warp's four elements hit 32 distinct banks).
#include "common.hpp"

namespace to_b200 {
namespace {

constexpr int kN = 8;
constexpr int kElemsPerWarp = 4;
constexpr int kWarps = 8;                    // 256 threads, 32 elements per CTA batch
constexpr int kRow = 12;                     // floats between rows in the exchange buffer
constexpr int kComp = kN * kRow;             // 96 floats per component
constexpr int kSlot = 2 * kComp + 8;         // 200 floats per element slot

struct Sem2dArgs {
  const float* u[2];
  float* f[2];
  const float* m[7];  // xix, xiz, gamx, gamz, jac, l2m, mu
  long long nelem;
  float H[kN][kN];
  float Hw[kN][kN];
  float w[kN];
};

__device__ __forceinline__ void load_row(const float* p, float (&r)[kN]) {
  const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
  r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w;
  r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
}

__device__ __forceinline__ void sts_row(float* p, const float (&r)[kN]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(r[0], r[1], r[2], r[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(r[4], r[5], r[6], r[7]);
}
__device__ __forceinline__ void lds_row(const float* p, float (&r)[kN]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w;
  r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
}

__device__ __forceinline__ void store_row(float* p, const float (&r)[kN]) {
  __stcs(reinterpret_cast<float4*>(p), make_float4(r[0], r[1], r[2], r[3]));
  __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(r[4], r[5], r[6], r[7]));
}

__global__ void __launch_bounds__(kWarps * 32) sem2d_elastic_kernel(const __grid_constant__ Sem2dArgs a) {
  __shared__ __align__(16) float sbuf[kWarps][kElemsPerWarp * kSlot];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int le = lane >> 3;   // element of the warp
  const int r = lane & 7;     // row j as row owner, column i as column owner
  float* slot = &sbuf[warp][le * kSlot];
  const long long groups = (a.nelem + kElemsPerWarp - 1) / kElemsPerWarp;
  const long long gw = static_cast<long long>(gridDim.x) * kWarps;

  for (long long g = static_cast<long long>(blockIdx.x) * kWarps + warp; g < groups; g += gw) {
    const long long e = g * kElemsPerWarp + le;
    const bool valid = e < a.nelem;
    const long long row0 = (e * kN + r) * kN;  // word of (e, j=r, i=0)

    // ---- u rows, xi-gradients in registers ----
    float u[2][kN];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      if (valid) {
        load_row(a.u[c] + row0, u[c]);
      } else {
#pragma unroll
        for (int i = 0; i < kN; ++i) u[c][i] = 0.f;
      }
    }
    float ax[2][kN];
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int i = 0; i < kN; ++i) {
        float s = 0.f;
#pragma unroll
        for (int p = 0; p < kN; ++p) s = fmaf(a.H[i][p], u[c][p], s);
        ax[c][i] = s;
      }
    // ---- gamma-gradients through the column owners ----
#pragma unroll
    for (int c = 0; c < 2; ++c) sts_row(slot + c * kComp + r * kRow, u[c]);
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float col[kN];
#pragma unroll
      for (int p = 0; p < kN; ++p) col[p] = slot[c * kComp + p * kRow + r];
#pragma unroll
      for (int j = 0; j < kN; ++j) {
        float s = 0.f;
#pragma unroll
        for (int p = 0; p < kN; ++p) s = fmaf(a.H[j][p], col[p], s);
        slot[c * kComp + j * kRow + r] = s;  // in place: this column is only ours
      }
    }
    __syncwarp();
    float gm[2][kN];
#pragma unroll
    for (int c = 0; c < 2; ++c) lds_row(slot + c * kComp + r * kRow, gm[c]);
    __syncwarp();

    // ---- chain rule, stress, integrands: Fx in registers, Fg to the buffer ----
    float geo[7][kN];
#pragma unroll
    for (int q = 0; q < 7; ++q) {
      if (valid) {
        load_row(a.m[q] + row0, geo[q]);
      } else {
#pragma unroll
        for (int i = 0; i < kN; ++i) geo[q][i] = 0.f;
      }
    }
    float fx[2][kN], fg[2][kN];
#pragma unroll
    for (int i = 0; i < kN; ++i) {
      const float xix = geo[0][i], xiz = geo[1][i], gx = geo[2][i], gz = geo[3][i];
      const float jac = geo[4][i], l2m = geo[5][i], mu = geo[6][i];
      const float ds00 = ax[0][i] * xix + gm[0][i] * gx;
      const float ds01 = ax[0][i] * xiz + gm[0][i] * gz;
      const float ds10 = ax[1][i] * xix + gm[1][i] * gx;
      const float ds11 = ax[1][i] * xiz + gm[1][i] * gz;
      const float lam = l2m - 2.0f * mu;
      const float s00 = l2m * ds00 + lam * ds11;
      const float s11 = lam * ds00 + l2m * ds11;
      const float s01 = mu * (ds01 + ds10);
      fx[0][i] = jac * (s00 * xix + s01 * xiz);
      fx[1][i] = jac * (s01 * xix + s11 * xiz);
      fg[0][i] = jac * (s00 * gx + s01 * gz);
      fg[1][i] = jac * (s01 * gx + s11 * gz);
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) sts_row(slot + c * kComp + r * kRow, fg[c]);
    __syncwarp();
    // ---- gamma-divergences through the column owners ----
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float col[kN];
#pragma unroll
      for (int q = 0; q < kN; ++q) col[q] = slot[c * kComp + q * kRow + r];
#pragma unroll
      for (int j = 0; j < kN; ++j) {
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < kN; ++q) s = fmaf(a.Hw[q][j], col[q], s);
        slot[c * kComp + j * kRow + r] = s;
      }
    }
    __syncwarp();
    // ---- xi-divergences in registers, weighted sum, store ----
    const float wj = a.w[r];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float out[kN], tg[kN];
      lds_row(slot + c * kComp + r * kRow, tg);
#pragma unroll
      for (int i = 0; i < kN; ++i) {
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < kN; ++q) s = fmaf(a.Hw[q][i], fx[c][q], s);
        out[i] = wj * s + a.w[i] * tg[i];
      }
      if (valid) store_row(a.f[c] + row0, out);
    }
    __syncwarp();  // the buffer is rewritten by the next group
  }
}

}  // namespace
}  // namespace to_b200

using namespace to_b200;

extern "C" int to_sem2d_elastic_local(int32_t ngll, int64_t nelem, const double* hprime,
                                      const double* hprimewgll, const double* wgll,
                                      const to_sem2d_fields* fl, void* stream) {
  if (!fl || !hprime || !hprimewgll || !wgll || nelem < 0)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem2d_elastic_local: bad argument");
  if (ngll != kN)
    return set_error(TO_ERR_UNSUPPORTED, "to_sem2d_elastic_local: ngll %d (built: 8)", ngll);
  if (nelem == 0) return ok();
  Sem2dArgs a;
  const void* ptrs[] = {fl->u[0], fl->u[1], fl->f[0], fl->f[1], fl->xix, fl->xiz,
                        fl->gamx, fl->gamz, fl->jac, fl->l2m, fl->mu};
  for (const void* p : ptrs) {
    if (!p) return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem2d_elastic_local: null field");
    if (!aligned(p, 16))
      return set_error(TO_ERR_ALIGNMENT, "to_sem2d_elastic_local: fields must be 16-byte aligned");
  }
  for (int c = 0; c < 2; ++c) {
    a.u[c] = static_cast<const float*>(fl->u[c]);
    a.f[c] = static_cast<float*>(fl->f[c]);
  }
  const void* m[7] = {fl->xix, fl->xiz, fl->gamx, fl->gamz, fl->jac, fl->l2m, fl->mu};
  for (int q = 0; q < 7; ++q) a.m[q] = static_cast<const float*>(m[q]);
  a.nelem = nelem;
  for (int i = 0; i < kN; ++i) {
    a.w[i] = static_cast<float>(wgll[i]);
    for (int p = 0; p < kN; ++p) {
      a.H[i][p] = static_cast<float>(hprime[i * kN + p]);
      a.Hw[i][p] = static_cast<float>(hprimewgll[i * kN + p]);
    }
  }
  int dev = 0;
  const int sms = device_sm_count(&dev);
  if (sms <= 0) return -sms;
  const long long groups = (nelem + kElemsPerWarp - 1) / kElemsPerWarp;
  const long long want = (groups + kWarps - 1) / kWarps;
  const long long cap = 8ll * sms;
  const int grid = static_cast<int>(want < cap ? want : cap);
  sem2d_elastic_kernel<<<grid, kWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}
