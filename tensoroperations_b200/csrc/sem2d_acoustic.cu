// sem2d_acoustic.cu -- 2D acoustic (scalar) spectral-element stiffness,
// assembled through ibool.  The reference has no acoustic kernel (its 2D
// benchmark is elastic P-SV); this is the configuration's operator:
//   dxi = sum_p H(i,p) u(j,p),  dgm = sum_p H(j,p) u(p,i)      (u gathered)
//   du/dx = dxi xix + dgm gamx,  du/dz = dxi xiz + dgm gamz
//   Fx = jac / rho (du/dx xix + du/dz xiz),  Fg = jac / rho (du/dx gamx + du/dz gamz)
//   f(ibool(j,i)) += w_j sum_q Hw(q,i) Fx(j,q) + w_i sum_q Hw(q,j) Fg(q,i)
// Per-point arrays [E][j][i]; u and f [nglob].  The problem of the
// configuration (128 x 128 quads, NGLL 5, fp64: 29 MB) is launch-bound on a
// B200, so the kernel is the plain form: one thread per point, EB elements
// per CTA, the element's u / fluxes in shared memory between two barriers.
#include "common.hpp"

namespace to_b200 {
namespace {

template <typename T, int N>
struct Ac2dArgs {
  const T* u;
  T* f;
  const int32_t* ibool;
  const T* m[6];  // xix, xiz, gamx, gamz, jac, rho
  long long nelem;
  T H[N][N], Hw[N][N], w[N];
};

template <typename T, int N, int EB>
__global__ void __launch_bounds__(EB * N * N) sem2d_acoustic_kernel(const __grid_constant__ Ac2dArgs<T, N> a) {
  constexpr int NN = N * N;
  __shared__ T su[EB][NN], sfx[EB][NN], sfg[EB][NN];
  const int t = threadIdx.x, le = t / NN, ji = t - le * NN, j = ji / N, i = ji - j * N;
  const long long nb = (a.nelem + EB - 1) / EB;
  for (long long b = blockIdx.x; b < nb; b += gridDim.x) {
    const long long e = b * EB + le;
    const bool valid = e < a.nelem;
    const long long pt = e * NN + ji;
    const int node = valid ? __ldg(a.ibool + pt) : 0;
    su[le][ji] = valid ? __ldg(a.u + node) : T(0);
    __syncthreads();
    T dxi = 0, dgm = 0;
#pragma unroll
    for (int p = 0; p < N; ++p) {
      dxi = fma(a.H[i][p], su[le][j * N + p], dxi);
      dgm = fma(a.H[j][p], su[le][p * N + i], dgm);
    }
    T xix = 0, xiz = 0, gx = 0, gz = 0, jac = 0, rho = 1;
    if (valid) {
      xix = __ldg(a.m[0] + pt); xiz = __ldg(a.m[1] + pt);
      gx = __ldg(a.m[2] + pt);  gz = __ldg(a.m[3] + pt);
      jac = __ldg(a.m[4] + pt); rho = __ldg(a.m[5] + pt);
    }
    const T dudx = dxi * xix + dgm * gx, dudz = dxi * xiz + dgm * gz;
    const T s = jac / rho;
    sfx[le][ji] = s * (dudx * xix + dudz * xiz);
    sfg[le][ji] = s * (dudx * gx + dudz * gz);
    __syncthreads();
    T tx = 0, tg = 0;
#pragma unroll
    for (int q = 0; q < N; ++q) {
      tx = fma(a.Hw[q][i], sfx[le][j * N + q], tx);
      tg = fma(a.Hw[q][j], sfg[le][q * N + i], tg);
    }
    if (valid) atomicAdd(a.f + node, a.w[j] * tx + a.w[i] * tg);
    __syncthreads();
  }
}

template <typename T, int N>
int launch(const to_sem2d_acoustic_desc* d, const to_sem2d_acoustic_fields* fl, int accumulate,
           cudaStream_t s) {
  constexpr int EB = 8;
  Ac2dArgs<T, N> a;
  a.u = static_cast<const T*>(fl->u);
  a.f = static_cast<T*>(fl->f);
  a.ibool = fl->ibool;
  const void* m[6] = {fl->xix, fl->xiz, fl->gamx, fl->gamz, fl->jac, fl->rho};
  for (int q = 0; q < 6; ++q) a.m[q] = static_cast<const T*>(m[q]);
  a.nelem = d->nelem;
  for (int i = 0; i < N; ++i) {
    a.w[i] = static_cast<T>(d->wgll[i]);
    for (int p = 0; p < N; ++p) {
      a.H[i][p] = static_cast<T>(d->hprime[i * N + p]);
      a.Hw[i][p] = static_cast<T>(d->hprimewgll[i * N + p]);
    }
  }
  if (!accumulate) TO_CUDA_TRY(cudaMemsetAsync(fl->f, 0, sizeof(T) * d->nglob, s));
  if (d->nelem == 0) return ok();
  int dev = 0;
  const int sms = device_sm_count(&dev);
  if (sms <= 0) return -sms;
  const long long want = (d->nelem + EB - 1) / EB;
  const long long cap = 16ll * sms;
  sem2d_acoustic_kernel<T, N, EB><<<static_cast<int>(want < cap ? want : cap), EB * N * N, 0, s>>>(a);
  TO_CUDA_TRY(cudaGetLastError());
  return ok();
}

}  // namespace
}  // namespace to_b200

using namespace to_b200;

extern "C" int to_sem2d_acoustic_apply(const to_sem2d_acoustic_desc* d,
                                       const to_sem2d_acoustic_fields* fl, int32_t accumulate,
                                       void* stream) {
  if (!d || !fl || !d->hprime || !d->hprimewgll || !d->wgll || d->nelem < 0 || d->nglob <= 0)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem2d_acoustic_apply: bad argument");
  const void* ptrs[] = {fl->u, fl->f, fl->ibool, fl->xix, fl->xiz, fl->gamx, fl->gamz, fl->jac, fl->rho};
  for (const void* p : ptrs)
    if (!p) return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem2d_acoustic_apply: null field");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (d->ngll == 5 && d->dtype == TO_F64) return launch<double, 5>(d, fl, accumulate, s);
  if (d->ngll == 5 && d->dtype == TO_F32) return launch<float, 5>(d, fl, accumulate, s);
  return set_error(TO_ERR_UNSUPPORTED, "to_sem2d_acoustic_apply: ngll %d dtype %d (built: 5)", d->ngll,
                   d->dtype);
}
