// sem3d_mgpu.cu -- the z-slab (multi-GPU) SEM 3D operator behind one C-ABI call.
//
// A rank owns a contiguous range of element layers and every node plane they
// touch; its first and last node planes are shared with the neighbouring
// ranks.  One application (to_sem3d_elastic_mgpu):
//
//   compute stream   zero f and the ticket counters
//                    scatter the element layers next to a neighbour: both
//                      layers in ONE launch of the line-owner kernel
//                    record "boundary done"
//                    scatter the interior layers: one launch, batches handed
//                      out by a ticket counter
//                    wait for "exchange done"
//   comm stream      wait for "boundary done"
//                    one NCCL group: send this rank's shared planes straight
//                      from f (each component's plane is one contiguous node
//                      range) and receive the neighbour's into `recv`
//                    add the received partial sums into f's shared planes
//                    record "exchange done"
//
// The interior launch keeps every SM slot it can get for its whole run, so
// the exchange's kernels (NCCL's, then the add) can only start on a slot the
// interior has not taken.  With the comm stream at a higher priority than the
// compute stream those kernels are dispatched first when the boundary launch
// drains; the interior CTAs that could not start meanwhile start when the
// exchange releases its slots and, because batches come from the ticket
// counter, simply take fewer of them -- no CTA is left holding a fixed share
// at the end.  Interior layers touch no shared plane, so the add overlaps them.
//
// NCCL is reached through the process's own libnccl.so.2 (looked up at run
// time, the library already loaded by the caller first), so the communicator
// the caller passes and the calls made on it come from one NCCL.  The
// reference is single-GPU (one Kokkos execution space); this partition is this
// build's own.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.hpp"

namespace to_b200 {

int sem3d_apply_ranges(const to_sem3d_plan* plan, const to_sem3d_fields* fl,
                       const int64_t first[2], const int64_t count[2],
                       unsigned long long* ticket, cudaStream_t stream);
const to_sem3d_desc* sem3d_plan_desc(const to_sem3d_plan* plan);
int flat_accumulate(int32_t dtype, void* dst, const void* buf, int64_t n, cudaStream_t s);

namespace {

struct NcclApi {
  bool loaded = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

template <typename F>
bool bind(void* h, const char* name, F& fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

// The NCCL of this process: the libnccl.so.2 already loaded (by torch, or by
// a program linked against NCCL), else the first one the loader finds.
const NcclApi* nccl_api(int* status) {
  static std::mutex mu;
  static NcclApi api;
  static bool tried = false;
  std::lock_guard<std::mutex> lock(mu);
  if (!tried) {
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      api.loaded = bind(h, "ncclGetUniqueId", api.GetUniqueId) &&
                   bind(h, "ncclCommInitRank", api.CommInitRank) &&
                   bind(h, "ncclCommDestroy", api.CommDestroy) &&
                   bind(h, "ncclGroupStart", api.GroupStart) && bind(h, "ncclGroupEnd", api.GroupEnd) &&
                   bind(h, "ncclSend", api.Send) && bind(h, "ncclRecv", api.Recv) &&
                   bind(h, "ncclAllReduce", api.AllReduce) &&
                   bind(h, "ncclGetErrorString", api.GetErrorString);
    }
  }
  if (!api.loaded) {
    *status = set_error(TO_ERR_COMM, "NCCL (libnccl.so.2) could not be loaded");
    return nullptr;
  }
  *status = TO_OK;
  return &api;
}

int nccl_fail(const NcclApi* api, ncclResult_t r, const char* what) {
  return set_error(TO_ERR_COMM, "%s: %s", what, api->GetErrorString(r));
}

#define TO_NCCL_TRY(api, expr)                                   \
  do {                                                           \
    ncclResult_t to_r_ = (expr);                                 \
    if (to_r_ != ncclSuccess) return nccl_fail(api, to_r_, #expr); \
  } while (0)

// Two events per (host thread, device) order the streams inside one call;
// each call re-records them after the previous call's waits were enqueued.
struct CallEvents {
  cudaEvent_t bnd = nullptr, done = nullptr;
};

int call_events(int dev, CallEvents** out) {
  thread_local CallEvents ev[64];
  if (dev < 0 || dev >= 64) return set_error(TO_ERR_UNSUPPORTED, "device id %d >= 64", dev);
  CallEvents& e = ev[dev];
  if (!e.bnd) {
    TO_CUDA_TRY(cudaEventCreateWithFlags(&e.bnd, cudaEventDisableTiming));
    TO_CUDA_TRY(cudaEventCreateWithFlags(&e.done, cudaEventDisableTiming));
  }
  *out = &e;
  return ok();
}

}  // namespace
}  // namespace to_b200

using namespace to_b200;

extern "C" {

int to_nccl_unique_id(void* id) {
  if (!id) return set_error(TO_ERR_INVALID_ARGUMENT, "to_nccl_unique_id: null");
  int st = TO_OK;
  const NcclApi* api = nccl_api(&st);
  if (!api) return st;
  ncclUniqueId u;
  TO_NCCL_TRY(api, api->GetUniqueId(&u));
  static_assert(sizeof(ncclUniqueId) == TO_NCCL_UNIQUE_ID_BYTES, "NCCL unique id size");
  std::memcpy(id, &u, sizeof(u));
  return ok();
}

int to_nccl_comm_init(int32_t nranks, int32_t rank, const void* id, ncclComm_t* comm) {
  if (!id || !comm || nranks < 1 || rank < 0 || rank >= nranks)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_nccl_comm_init: bad argument");
  *comm = nullptr;
  int st = TO_OK;
  const NcclApi* api = nccl_api(&st);
  if (!api) return st;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  TO_NCCL_TRY(api, api->CommInitRank(comm, nranks, u, rank));
  return ok();
}

int to_nccl_comm_destroy(ncclComm_t comm) {
  if (!comm) return ok();
  int st = TO_OK;
  const NcclApi* api = nccl_api(&st);
  if (!api) return st;
  TO_NCCL_TRY(api, api->CommDestroy(comm));
  return ok();
}

int to_nccl_allreduce_sum_f64(double* x, int64_t n, ncclComm_t comm, void* stream) {
  if (!x || !comm || n < 0) return set_error(TO_ERR_INVALID_ARGUMENT, "to_nccl_allreduce_sum_f64: bad argument");
  if (n == 0) return ok();
  int st = TO_OK;
  const NcclApi* api = nccl_api(&st);
  if (!api) return st;
  TO_NCCL_TRY(api, api->AllReduce(x, x, static_cast<size_t>(n), ncclFloat64, ncclSum, comm,
                                  static_cast<cudaStream_t>(stream)));
  return ok();
}

size_t to_slab_sync_bytes(void) { return 256; }

int to_sem3d_elastic_mgpu(const to_sem3d_plan* plan, const to_sem3d_fields* fields,
                          const to_slab* slab, ncclComm_t comm, void* compute_stream,
                          void* comm_stream) {
  if (!plan || !fields || !slab)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu: null argument");
  const to_sem3d_desc& d = *sem3d_plan_desc(plan);
  if (!d.assembled)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu: the plan must be assembled");
  const bool il = d.node_layout == 1;  // u[0], f[0]: [nglob][4] floats
  const bool lo = slab->prev >= 0, hi = slab->next >= 0;
  const int64_t L = slab->layer_elems, plane = slab->plane_nodes;
  if (L <= 0 || plane <= 0 || d.nelem % L != 0 || d.nelem < L)
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "to_sem3d_elastic_mgpu: %lld elements are not whole layers of %lld",
                     static_cast<long long>(d.nelem), static_cast<long long>(L));
  if (2 * plane > d.nglob)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu: plane of %lld nodes > nglob / 2",
                     static_cast<long long>(plane));
  if ((lo || hi) && !comm)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu: neighbours but no communicator");
  if ((lo && !slab->recv[0]) || (hi && !slab->recv[1]) || !slab->sync)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu: null recv / sync buffer");
  if (!aligned(slab->sync, 16))
    return set_error(TO_ERR_ALIGNMENT, "to_sem3d_elastic_mgpu: sync buffer not 16-byte aligned");
  for (int c = 0; c < (il ? 1 : 3); ++c)
    if (!fields->f[c] || !fields->u[c])
      return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu: null u / f component");
  cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
  cudaStream_t xs = static_cast<cudaStream_t>(comm_stream);
  const size_t vb = d.dtype == TO_F64 ? 8 : 4;
  const ncclDataType_t nt = d.dtype == TO_F64 ? ncclFloat64 : ncclFloat32;

  const NcclApi* api = nullptr;
  CallEvents* ev = nullptr;
  if (lo || hi) {
    int st = TO_OK;
    api = nccl_api(&st);
    if (!api) return st;
    int dev = 0;
    TO_CUDA_TRY(cudaGetDevice(&dev));
    if (int s2 = call_events(dev, &ev)) return s2;
  }

  // ---- compute stream: zero f and the tickets, boundary layers ----
  if (!slab->f_is_zero) {
    if (il)
      TO_CUDA_TRY(cudaMemsetAsync(fields->f[0], 0, 4 * vb * d.nglob, cs));
    else
      for (int c = 0; c < 3; ++c) TO_CUDA_TRY(cudaMemsetAsync(fields->f[c], 0, vb * d.nglob, cs));
  }
  auto* tickets = static_cast<unsigned long long*>(slab->sync);
  TO_CUDA_TRY(cudaMemsetAsync(tickets, 0, 2 * sizeof(unsigned long long), cs));
  int64_t bfirst[2] = {0, 0}, bcount[2] = {0, 0};
  int nb = 0;
  if (lo) {
    bfirst[nb] = 0;
    bcount[nb++] = L;
  }
  if (hi && !(lo && d.nelem == L)) {  // one layer touching both planes is scattered once
    bfirst[nb] = d.nelem - L;
    bcount[nb++] = L;
  }
  if (nb)
    if (int st = sem3d_apply_ranges(plan, fields, bfirst, bcount, tickets, cs)) return st;

  // ---- comm stream: exchange the shared planes, add the neighbours' sums ----
  if (lo || hi) {
    TO_CUDA_TRY(cudaEventRecord(ev->bnd, cs));
    TO_CUDA_TRY(cudaStreamWaitEvent(xs, ev->bnd, 0));
    const int64_t off[2] = {0, d.nglob - plane};
    const int peer[2] = {slab->prev, slab->next};
    TO_NCCL_TRY(api, api->GroupStart());
    for (int side = 0; side < 2; ++side) {
      if (peer[side] < 0) continue;
      if (il) {  // the plane is 4 * plane consecutive values of f[0]
        const char* src = static_cast<const char*>(fields->f[0]) + 4 * vb * off[side];
        ncclResult_t r = api->Send(src, static_cast<size_t>(4 * plane), nt, peer[side], comm, xs);
        if (r == ncclSuccess)
          r = api->Recv(slab->recv[side], static_cast<size_t>(4 * plane), nt, peer[side], comm, xs);
        if (r != ncclSuccess) {
          api->GroupEnd();
          return nccl_fail(api, r, "to_sem3d_elastic_mgpu: ncclSend / ncclRecv");
        }
        continue;
      }
      for (int c = 0; c < 3; ++c) {
        const char* src = static_cast<const char*>(fields->f[c]) + vb * off[side];
        char* dst = static_cast<char*>(slab->recv[side]) + vb * c * plane;
        ncclResult_t r = api->Send(src, static_cast<size_t>(plane), nt, peer[side], comm, xs);
        if (r == ncclSuccess)
          r = api->Recv(dst, static_cast<size_t>(plane), nt, peer[side], comm, xs);
        if (r != ncclSuccess) {
          api->GroupEnd();
          return nccl_fail(api, r, "to_sem3d_elastic_mgpu: ncclSend / ncclRecv");
        }
      }
    }
    TO_NCCL_TRY(api, api->GroupEnd());
    for (int side = 0; side < 2; ++side) {
      if (peer[side] < 0) continue;
      int st;
      if (il)
        st = flat_accumulate(d.dtype, static_cast<char*>(fields->f[0]) + 4 * vb * off[side],
                             slab->recv[side], 4 * plane, xs);
      else
        st = to_sem3d_halo_accumulate(d.dtype, fields->f, off[side], plane, slab->recv[side], xs);
      if (st) return st;
    }
    TO_CUDA_TRY(cudaEventRecord(ev->done, xs));
  }

  // ---- compute stream: interior layers, then wait for the exchange ----
  const int64_t i0 = lo ? L : 0, i1 = hi ? d.nelem - L : d.nelem;
  if (i1 > i0) {
    const int64_t ifirst[2] = {i0, 0}, icount[2] = {i1 - i0, 0};
    if (int st = sem3d_apply_ranges(plan, fields, ifirst, icount, tickets + 1, cs)) return st;
  }
  if (lo || hi) TO_CUDA_TRY(cudaStreamWaitEvent(cs, ev->done, 0));
  return ok();
}

int to_sem3d_elastic_mgpu_host(const to_sem3d_plan* plan, const to_sem3d_fields* fields,
                               const to_slab* slab, ncclComm_t comm, const to_host_nodes* host,
                               void* compute_stream, void* comm_stream) {
  if (!plan || !fields || !slab || !host)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu_host: null argument");
  const to_sem3d_desc& d = *sem3d_plan_desc(plan);
  const bool il = d.node_layout == 1;
  const size_t vb = d.dtype == TO_F64 ? 8 : 4;
  const size_t bytes = vb * static_cast<size_t>(d.nglob);
  for (int c = 0; c < 3; ++c) {
    if (!host->u[c] || !host->f[c])
      return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu_host: null host array");
    if (il && !host->stage[c])
      return set_error(TO_ERR_INVALID_ARGUMENT,
                       "to_sem3d_elastic_mgpu_host: interleaved nodes need three stage arrays");
  }
  if (!fields->u[0] || !fields->f[0])
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_sem3d_elastic_mgpu_host: null device u / f");
  cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
  // copy in (and interleave)
  for (int c = 0; c < 3; ++c) {
    void* dst = il ? host->stage[c] : const_cast<void*>(fields->u[c]);
    TO_CUDA_TRY(cudaMemcpyAsync(dst, host->u[c], bytes, cudaMemcpyHostToDevice, cs));
  }
  if (il) {
    const float* x[3] = {static_cast<const float*>(host->stage[0]),
                         static_cast<const float*>(host->stage[1]),
                         static_cast<const float*>(host->stage[2])};
    if (int st = to_nodes_interleave(x, static_cast<float*>(const_cast<void*>(fields->u[0])),
                                     d.nglob, cs))
      return st;
  }
  if (int st = to_sem3d_elastic_mgpu(plan, fields, slab, comm, compute_stream, comm_stream))
    return st;
  // (de-interleave and) copy out
  if (il) {
    float* x[3] = {static_cast<float*>(host->stage[0]), static_cast<float*>(host->stage[1]),
                   static_cast<float*>(host->stage[2])};
    if (int st = to_nodes_deinterleave(static_cast<const float*>(fields->f[0]), x, d.nglob, cs))
      return st;
  }
  for (int c = 0; c < 3; ++c) {
    const void* src = il ? host->stage[c] : fields->f[c];
    TO_CUDA_TRY(cudaMemcpyAsync(host->f[c], src, bytes, cudaMemcpyDeviceToHost, cs));
  }
  return ok();
}

}  // extern "C"
