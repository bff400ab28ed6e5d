/*
 * tensoroperations_b200.h -- C ABI of the B200 (sm_100a) evaluator for the
 * fused spectral-element stiffness path of TensorOperations.
 *
 * Everything here is plain C: pointers, sizes and integer status codes.  No
 * call traps or aborts; every failure comes back as a non-zero `to_status`
 * and `to_last_error()` holds a one-line reason for the calling thread.
 * Device pointers are CUDA device addresses of the current device; `stream`
 * arguments are `cudaStream_t` values passed as `void*` (NULL = legacy
 * default stream).  Nothing in a launch entry point allocates device memory.
 *
 * The reference interface each entry point replaces is cited as
 * path:line inside Rohit-Kakodkar/TensorOperations.
 */
#ifndef TENSOROPERATIONS_B200_H_
#define TENSOROPERATIONS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TO_ABI_VERSION 2

typedef enum to_status {
  TO_OK = 0,
  TO_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, bad enum          */
  TO_ERR_UNSUPPORTED = 2,      /* dtype / NGLL combination not built        */
  TO_ERR_CUDA = 3,             /* a CUDA runtime call failed                */
  TO_ERR_SCRATCH = 4,          /* shared-memory request above device limit  */
  TO_ERR_ALIGNMENT = 5,        /* a pointer is not aligned as required      */
  TO_ERR_TIMEOUT = 6,          /* a bounded device-side wait gave up        */
  TO_ERR_COMM = 7,             /* a collective / peer exchange failed       */
  TO_ERR_NO_DEVICE = 8,        /* no CUDA device visible                    */
  TO_ERR_GRID = 9              /* a LabelWhole label longer than its tile   */
} to_status;

typedef enum to_dtype { TO_F32 = 0, TO_F64 = 1 } to_dtype;

/* ---------------------------------------------------------------------- */
/* Library                                                                 */
/* ---------------------------------------------------------------------- */

/* ABI version of the loaded library (compare with TO_ABI_VERSION). */
int to_abi_version(void);

/* Static text for a status code. */
const char* to_status_string(int status);

/* Detail of the last failure on the calling thread ("" if none). */
const char* to_last_error(void);

/* Number of SMs of the current device, or a negative to_status. */
int to_device_sm_count(void);

/* Device status word of the current device: TO_OK, or the status a kernel
 * recorded instead of trapping (TO_ERR_TIMEOUT when a bounded wait gave up).
 * Synchronous (reads device memory).  reset != 0 clears it. */
int to_device_status(int32_t reset);

/* ---------------------------------------------------------------------- */
/* Mesh and operators (host utilities)                                     */
/* ---------------------------------------------------------------------- */

/*
 * Structured shared-node numbering of an nex x ney x nez hexahedral mesh with
 * NGLL points per direction.  Element e = (ez*ney + ey)*nex + ex; node
 *   ibool[e][k][j][i] = ((ez*(N-1)+k)*ny + ey*(N-1)+j)*nx + ex*(N-1)+i,
 * nx = nex*(N-1)+1 (same for y, z).  `ibool` is a HOST buffer of
 * nex*ney*nez*N^3 int32.  The reference has no global numbering: its SEM
 * programs are element-local (benchmarks/sem_stiffness/bench_sem_stiffness.cpp:8-11,
 * benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp:104-105); this
 * defines the one the assembled mode uses.
 */
int to_mesh_structured_ibool(int32_t nex, int32_t ney, int32_t nez,
                             int32_t ngll, int32_t* ibool);

/*
 * GLL nodes, weights, derivative matrix H(i,p) = l_p'(x_i) and the weighted
 * transpose Hw(q,i) = H(q,i) * w(q) (hprimewgll), all HOST double arrays
 * (nodes/weights [N], hprime/hprimewgll [N][N]).  Any pointer may be NULL.
 * 2 <= ngll <= 16.
 */
int to_gll_operators(int32_t ngll, double* nodes, double* weights,
                     double* hprime, double* hprimewgll);

/*
 * Seeded synthetic fill of a HOST buffer: dst[n] of `dtype`.  Element m gets
 * a value derived from splitmix64(seed, m) only, so any slice can be
 * generated independently and identically anywhere.
 *   dist 0: Uniform[a, b)      dist 1: Normal(mean a, stddev b)
 */
int to_synth_fill(void* dst, int32_t dtype, int64_t n, uint64_t seed,
                  int32_t dist, double a, double b);

/* The slice [first, first + n) of the same sequence: dst[i] is element
 * first + i of to_synth_fill's output (how a z-slab rank generates exactly its
 * part of a global problem). */
int to_synth_fill_at(void* dst, int32_t dtype, int64_t first, int64_t n, uint64_t seed,
                     int32_t dist, double a, double b);

/* The same generators on the DEVICE, for problems too large for host memory:
 * dst[i] = (element first + i of the sequence) + add, converted to dtype, and
 * the structured numbering written to a device int32 buffer.  Uniform values
 * equal the host's bit for bit; normal values use the device's log / cos.
 * to_axpy2_device: y += 2 x (l2m = lambda + 2 mu in place).  Asynchronous. */
int to_synth_fill_device(void* dst, int32_t dtype, int64_t first, int64_t n, uint64_t seed,
                         int32_t dist, double a, double b, double add, void* stream);
int to_axpy2_device(void* y, const void* x, int32_t dtype, int64_t n, void* stream);
int to_mesh_structured_ibool_device(int32_t nex, int32_t ney, int32_t nez, int32_t ngll,
                                    int32_t* ibool, void* stream);

/* ---------------------------------------------------------------------- */
/* SEM 3D isotropic-elastic stiffness operator                             */
/* ---------------------------------------------------------------------- */
/*
 * One application f = K u of the pipeline the reference builds as a
 * LevelGraph in benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp:247-351
 * (stage H,Hw | stage u | 9 gradient contractions | 1 nine-output combine
 * Integrand9 | 9 divergence contractions | 3 WeightedSum combines) and
 * launches through LevelOutputs::execute (include/TensorOperations/LevelGraph.hpp:664-667):
 *
 *   grad    dxi_c = sum_p H(i,p) u_c(k,j,p)   (and eta over j, gamma over k)
 *   stress  ds = chain_rule(dxi,deta,dgam,J); sigma = mu(ds+ds^T)+lambda tr(ds) I,
 *           lambda = l2m - 2 mu
 *   flux    F^r_c = jac * sum_d sigma[c][d] J[r][d]
 *   div     t^xi_c = sum_q Hw(q,i) F^xi_c(k,j,q)  (eta over j, gamma over k)
 *   force   f_c = w_j w_k t^xi_c + w_i w_k t^eta_c + w_i w_j t^gam_c
 *
 * Per-point arrays are [E][k][j][i] (i fastest), one array per quantity, as the
 * reference's Kokkos::View<T*[N][N][N], LayoutRight> fields.
 * Element-local mode (ibool == NULL): u_c and f_c are [E][N][N][N] and f is
 * overwritten.  Assembled mode: u_c and f_c are [nglob] and f_c[ibool[...]]
 * receives the scatter-add of every element's contribution; with
 * accumulate == 0 f is zeroed first (stream-ordered memset), else added to.
 */
typedef struct to_sem3d_desc {
  int32_t dtype;            /* TO_F32 or TO_F64                              */
  int32_t ngll;             /* N: 5 or 8 (f32 and f64 each)                  */
  int64_t nelem;            /* E                                              */
  int64_t nglob;            /* assembled: number of global nodes; else 0     */
  int32_t assembled;        /* 1 = through ibool, 0 = element-local          */
  int32_t node_layout;      /* assembled u, f: 0 = one [nglob] array per
                               component; 1 = interleaved [nglob][4] floats
                               (x, y, z, unused) in u[0] / f[0], 16-byte
                               aligned (f32, NGLL 5 only): one 128-bit gather
                               and one 128-bit scatter-add per point         */
  const double* hprime;     /* HOST [N][N]  H(i,p)   (reference d.H)          */
  const double* hprimewgll; /* HOST [N][N]  Hw(q,i)  (reference d.Hw)         */
  const double* wgll;       /* HOST [N]     w        (reference d.w)           */
} to_sem3d_desc;

typedef struct to_sem3d_fields {
  const void* u[3];         /* displacement components                       */
  void* f[3];               /* force components (output)                     */
  const int32_t* ibool;     /* [E][N][N][N] global node ids (assembled mode) */
  /* inverse Jacobian J[r][d] = d(xi_r)/d(x_d), then jac, l2m, mu            */
  const void* xix;  const void* xiy;  const void* xiz;
  const void* etax; const void* etay; const void* etaz;
  const void* gamx; const void* gamy; const void* gamz;
  const void* jac;  const void* l2m;  const void* mu;
  /* Assembled mode, optional (NULL: none): DEVICE double; every gathered u
   * value is read as u * (1 / sqrt(*u_norm2)), the product taken in double
   * and rounded once -- what to_scale3 writes, so a power iteration can keep
   * the unnormalised K u and fold the normalisation into the next
   * application (one pass over u and f less per step).  Appended last: a
   * zero-initialised struct has none. */
  const double* u_norm2;
} to_sem3d_fields;

typedef struct to_sem3d_plan to_sem3d_plan;

/* Validate a description and capture the operators.  Host only. */
int to_sem3d_plan_create(const to_sem3d_desc* desc, to_sem3d_plan** plan);
int to_sem3d_plan_destroy(to_sem3d_plan* plan);

/* Launch one application on `stream` (asynchronous).  Device pointers in
 * `fields` must be 4-byte (f32) or 8-byte (f64) aligned; all per-point arrays
 * hold E*N^3 values. */
int to_sem3d_apply(const to_sem3d_plan* plan, const to_sem3d_fields* fields,
                   int32_t accumulate, void* stream);

/* The contribution of elements [first, first + count) of the plan only,
 * ADDED to f (never zeroed): `fields` describes the whole batch exactly as for
 * to_sem3d_apply.  Lets a caller order element ranges -- a z-slab rank
 * computes the element layers next to its neighbours first, starts the
 * interface exchange, then computes the interior.  The reference launches
 * its whole league at once (include/TensorOperations/LevelGraph.hpp:576-628);
 * this is the same operator on a sub-range. */
int to_sem3d_apply_elements(const to_sem3d_plan* plan, const to_sem3d_fields* fields,
                            int64_t first, int64_t count, void* stream);

/* Algorithmic HBM bytes of one application of `plan` (the roofline numerator:
 * every per-point array read once, ibool read once, u read and f written once
 * per global node in assembled mode, per point in element-local mode). */
double to_sem3d_algorithmic_bytes(const to_sem3d_plan* plan);

/* Useful floating-point operations of one application (36N+159 per point). */
double to_sem3d_flops(const to_sem3d_plan* plan);

/* ---------------------------------------------------------------------- */
/* Z-slab interface planes (multi-GPU assembled mode)                      */
/* ---------------------------------------------------------------------- */
/*
 * A rank of a z-slab partition owns a contiguous range of element layers
 * and every node plane they touch; its first and last planes are shared with
 * the neighbouring ranks and hold partial sums after the rank's own scatter.
 * With the structured numbering a node plane is one contiguous range
 * [offset, offset + n) of each component (n = nx*ny).
 *   pack:        buf[c*n + i]      = f[c][offset + i]      (c = 0..2)
 *   accumulate:  f[c][offset + i] += buf[c*n + i]
 * `f` is a HOST array of 3 device pointers; `buf` is device memory of 3*n
 * values.  Both launch one kernel on `stream`.  The reference is single-GPU;
 * these are the two local steps around the neighbour exchange (NCCL
 * send/recv of `buf`).
 */
int to_sem3d_halo_pack(int32_t dtype, void* const f[3], int64_t offset, int64_t n,
                       void* buf, void* stream);
int to_sem3d_halo_accumulate(int32_t dtype, void* const f[3], int64_t offset, int64_t n,
                             const void* buf, void* stream);

/* Node layouts (f32): out[i] = (x[0][i], x[1][i], x[2][i], 0) for i < n, the
 * interleaved [nglob][4] layout of node_layout 1, from one array per component,
 * and back (x[c][i] = in[i].c).  `x` is a HOST array of 3 device pointers;
 * the interleaved array is 16-byte aligned.  One kernel on `stream`.  No
 * counterpart in the reference (it has no assembled fields). */
int to_nodes_interleave(const float* const x[3], float* out, int64_t n, void* stream);
int to_nodes_deinterleave(const float* in, float* const x[3], int64_t n, void* stream);


/* ---------------------------------------------------------------------- */
/* Z-slab operator over NCCL (one rank per GPU)                            */
/* ---------------------------------------------------------------------- */
/*
 * NCCL's communicator handle: the same typedef as nccl.h's, so a caller that
 * includes nccl.h passes its own ncclComm_t unchanged.
 */
typedef struct ncclComm* ncclComm_t;

#define TO_NCCL_UNIQUE_ID_BYTES 128

/*
 * One rank's z-slab of a structured mesh split in element layers across the
 * ranks of `comm`.  The rank's plan covers its elements (whole layers of
 * layer_elems elements, ordered layer by layer) and the nodes they touch;
 * its first node plane is shared with rank `prev` and its last with rank
 * `next` (-1: no neighbour on that side).  With the structured numbering each
 * plane is one contiguous range of plane_nodes nodes per component: nodes
 * [0, plane_nodes) and [nglob - plane_nodes, nglob).
 */
typedef struct to_slab {
  int32_t prev;          /* rank below in `comm`, or -1                      */
  int32_t next;          /* rank above in `comm`, or -1                      */
  int64_t layer_elems;   /* elements per element layer (nex * ney)           */
  int64_t plane_nodes;   /* nodes per node plane                             */
  void* recv[2];         /* device buffers of 3 * plane_nodes values (4 *
                            plane_nodes with interleaved nodes): the partial
                            sums received from prev ([0]) / next ([1])       */
  void* sync;            /* device buffer of to_slab_sync_bytes() bytes,
                            16-byte aligned (batch tickets of the launches)  */
  int32_t f_is_zero;     /* 0: the call zeroes f first (on compute_stream);
                            1: the caller has already zeroed f in stream order
                            (lets a caller time the operator without the fill) */
} to_slab;

/*
 * f = K u on this rank's slab, with the shared planes summed across the
 * neighbours, so every copy of a shared node holds the full sum and f equals
 * the slice of the single-mesh result for this rank's nodes.  Either node
 * layout of the plan: one array per component, or interleaved (u[0], f[0]
 * [nglob][4]; each shared plane then travels as one contiguous range).
 * The reference evaluates the whole mesh in one Kokkos launch on one device
 * (include/TensorOperations/LevelGraph.hpp:576-628, bench_sem3d_levelgraph.cpp
 * :247-351); this is the same operator partitioned over ranks.
 *   compute_stream: zero f (unless slab->f_is_zero); the element layers next
 *     to a neighbour (one launch); the interior layers (one launch, batches
 *     handed out by a ticket counter); then it waits for the exchange.
 *   comm_stream: after the boundary layers, one NCCL group sends this rank's
 *     shared planes (read in place from f) and receives the neighbours' into
 *     `recv`, then adds them into f's shared planes -- overlapped with the
 *     interior, which touches no shared plane.  Give comm_stream a higher
 *     priority than compute_stream (cudaStreamCreateWithPriority) so its
 *     kernels are dispatched ahead of the interior's batches.
 * Every rank must make the same sequence of calls.  Asynchronous; returns
 * TO_ERR_COMM if NCCL cannot be loaded or a call fails.  Nothing is allocated.
 */
size_t to_slab_sync_bytes(void);
int to_sem3d_elastic_mgpu(const to_sem3d_plan* plan, const to_sem3d_fields* fields,
                          const to_slab* slab, ncclComm_t comm, void* compute_stream,
                          void* comm_stream);

/*
 * The same call with u and f in HOST memory, one array per component (pinned
 * memory for asynchronous copies): on compute_stream it copies u in (and,
 * with interleaved nodes, converts it into fields->u[0] through host->stage),
 * applies the operator as to_sem3d_elastic_mgpu, and copies f out (converting
 * from fields->f[0] through host->stage).  fields->u / f are the device
 * buffers the operator uses; `stage` holds three device arrays of nglob values
 * (interleaved plans only; NULL otherwise).  Two calls on two streams with
 * two sets of device buffers overlap one call's copy-out with the next one's
 * copy-in.  The end-to-end path a caller with host data takes.
 */
typedef struct to_host_nodes {
  const void* u[3];      /* HOST: nglob values per component, read            */
  void* f[3];            /* HOST: nglob values per component, written         */
  void* stage[3];        /* DEVICE: nglob values each (interleaved plans)     */
} to_host_nodes;
int to_sem3d_elastic_mgpu_host(const to_sem3d_plan* plan, const to_sem3d_fields* fields,
                               const to_slab* slab, ncclComm_t comm, const to_host_nodes* host,
                               void* compute_stream, void* comm_stream);

/* NCCL set-up for callers without their own: rank 0 makes an id (bytes
 * TO_NCCL_UNIQUE_ID_BYTES), every rank receives it by its own means and
 * creates its communicator (the current device is the rank's GPU).  These and
 * to_nccl_allreduce_sum_f64 (in-place sum of n doubles across the ranks, on
 * `stream`) call the process's libnccl.so.2. */
int to_nccl_unique_id(void* id);
int to_nccl_comm_init(int32_t nranks, int32_t rank, const void* id, ncclComm_t* comm);
int to_nccl_comm_destroy(ncclComm_t comm);
int to_nccl_allreduce_sum_f64(double* x, int64_t n, ncclComm_t comm, void* stream);

/* ---------------------------------------------------------------------- */
/* Field reductions (repeated applications u <- K u / ||K u||)             */
/* ---------------------------------------------------------------------- */
/*
 * Sum of squares of three device arrays over [first, first + n):
 *   *result = sum_c sum_i x[c][first + i]^2        (accumulated in double)
 * `x` is a HOST array of 3 device pointers, `result` one device double.  Two
 * kernels on `stream`; the grouping of the sum is fixed by n alone (blocks of
 * 131072 values, then a fixed-order pass over the block partials), so the
 * result is bitwise the same on every device.  `workspace` is device memory
 * of at least to_sumsq3_workspace_bytes(n) bytes holding the block partials;
 * nothing in it needs to be initialised.  For a z-slab rank, [first, first+n)
 * is the nodes it owns: a shared interface plane is counted by the lower rank
 * only.  The reference's benchmark has no norm; this is the configuration's
 * steady-state loop.
 */
size_t to_sumsq3_workspace_bytes(int64_t n);
int to_sumsq3(int32_t dtype, const void* const x[3], int64_t first, int64_t n, double* result,
              void* workspace, size_t workspace_bytes, void* stream);

/* to_sumsq3 without a workspace argument, for callers that may not allocate
 * device memory: for example a solver step running inside an application
 * that owns the GPU's memory through its own pool (a cudaMalloc of ours
 * would fail or bypass its accounting), or a loop that must not stall the
 * device the way cudaFree does.  No counterpart in the reference.
 *   - The block partials live in one fixed array inside the library (256 KiB
 *     per GPU, kept until the process exits); nothing is allocated per call.
 *   - The first call on a device looks up that array's device address (with
 *     the device current); make that first call before any stream capture.
 *     The address is remembered per device and CUDA context: a call in
 *     another context (the caller's own, or a new primary context after
 *     cudaDeviceReset) looks it up again, so it too should come before any
 *     capture in that context.
 *   - n per component is limited to to_sumsq3_noalloc_max_n()
 *     (1,431,655,765); a larger n is rejected with TO_ERR_INVALID_ARGUMENT
 *     before anything is launched.
 *   - Every call shares the array and it keeps the last call's partials.
 *     Nothing in it needs to start at zero (a call writes every partial it
 *     later reads), but calls whose kernels overlap on the GPU -- on
 *     different streams, or from different host threads -- race on it and
 *     give wrong sums.  Order such calls on one stream.
 * Same result, bit for bit, as to_sumsq3 on the same inputs. */
int to_sumsq3_noalloc(int32_t dtype, const void* const x[3], int64_t first, int64_t n,
                      double* result, void* stream);
int64_t to_sumsq3_noalloc_max_n(void);

/* y[c][i] = x[c][i] / sqrt(*sumsq) for i < n (sumsq read on the device, so no
 * host synchronisation); y may equal x. */
int to_scale3(int32_t dtype, void* const y[3], const void* const x[3], int64_t n,
              const double* sumsq, void* stream);

/* ---------------------------------------------------------------------- */
/* SEM 2D elastic P-SV stiffness operator (element-local)                  */
/* ---------------------------------------------------------------------- */
/*
 * The operator of the reference's 2D benchmark
 * (benchmarks/sem_stiffness/bench_sem_stiffness.cpp: physics :319-357, host
 * loop :1335-1385), f32, NGLL 8, two components, element-local:
 *   a_c = sum_p H(i,p) u_c(j,p),  g_c = sum_p H(j,p) u_c(p,i)
 *   ds = grad u through (xix, xiz, gamx, gamz); sigma = isotropic P-SV stress
 *   Fx_c = jac (s_c0 xix + s_c1 xiz),  Fg_c = jac (s_c0 gamx + s_c1 gamz)
 *   f_c(j,i) = w_j sum_q Hw(q,i) Fx_c(j,q) + w_i sum_q Hw(q,j) Fg_c(q,i)
 * Per-point arrays [E][j][i] (i fastest), 16-byte aligned device pointers.
 * H, Hw, w: HOST doubles ([8][8], [8][8], [8]).  f is overwritten.
 */
typedef struct to_sem2d_fields {
  const void* u[2];
  void* f[2];
  const void* xix; const void* xiz; const void* gamx; const void* gamz;
  const void* jac; const void* l2m; const void* mu;
} to_sem2d_fields;

int to_sem2d_elastic_local(int32_t ngll, int64_t nelem, const double* hprime,
                           const double* hprimewgll, const double* wgll,
                           const to_sem2d_fields* fields, void* stream);

/* ---------------------------------------------------------------------- */
/* SEM 2D acoustic stiffness operator (assembled)                          */
/* ---------------------------------------------------------------------- */
/*
 * The scalar (acoustic) 2D operator of the first benchmark configuration;
 * the reference has no acoustic kernel, so this is the configuration's own
 * definition:
 *   dxi = sum_p H(i,p) u(j,p),  dgm = sum_p H(j,p) u(p,i)   (u gathered by ibool)
 *   du/dx = dxi xix + dgm gamx,  du/dz = dxi xiz + dgm gamz
 *   Fx = jac/rho (du/dx xix + du/dz xiz),  Fg = jac/rho (du/dx gamx + du/dz gamz)
 *   f(ibool(j,i)) += w_j sum_q Hw(q,i) Fx(j,q) + w_i sum_q Hw(q,j) Fg(q,i)
 * Per-point arrays [E][j][i]; u, f [nglob]; with accumulate == 0 f is zeroed
 * first.  NGLL 5, f64 or f32.  (kappa belongs to the mass matrix, not here.)
 */
typedef struct to_sem2d_acoustic_desc {
  int32_t dtype; int32_t ngll; int64_t nelem; int64_t nglob;
  const double* hprime; const double* hprimewgll; const double* wgll;  /* HOST */
} to_sem2d_acoustic_desc;
typedef struct to_sem2d_acoustic_fields {
  const void* u; void* f; const int32_t* ibool;
  const void* xix; const void* xiz; const void* gamx; const void* gamz;
  const void* jac; const void* rho;
} to_sem2d_acoustic_fields;
int to_sem2d_acoustic_apply(const to_sem2d_acoustic_desc* desc,
                            const to_sem2d_acoustic_fields* fields, int32_t accumulate,
                            void* stream);

/* ---------------------------------------------------------------------- */
/* Batched small GEMM with a shared left operand                           */
/* ---------------------------------------------------------------------- */
/*
 *   C[b][i][j] = sum_k A[i][k] * B[b][k][j],  b < batch, i < M, k < K, j < N
 * A: HOST double [M][K] (shared by every batch entry, converted to dtype);
 * B: device [batch][K][N], C: device [batch][M][N], row-major, dtype TO_F32
 * or TO_F64.  Built for (M, K) = (5, 5) and (8, 8), any N.  The batched form
 * of one gradient contraction of the SEM operator (the reference's analogue:
 * benchmarks/sem_stiffness/bench_sem_stiffness.cpp:884-896).  One kernel on
 * `stream`.
 */
int to_batched_small_gemm(int32_t dtype, int32_t M, int32_t K, int32_t N, int64_t batch,
                          const double* A, const void* B, void* C, void* stream);

/* ---------------------------------------------------------------------- */
/* Permuted multilevel contraction chain on the tensor cores               */
/* ---------------------------------------------------------------------- */
/*
 *   T[a,b,c,d] = sum_{e,f} A[a,e,c,f] * B[f,b,e,d]
 *   R[a,d]     = sum_{b,c} T[a,b,c,d] * C[c,b]
 * All six extents equal E (32, 64 or 128); row-major fp32 tensors in device
 * memory (A, B and the workspace 16-byte aligned).  The chain the reference
 * builds from ContractionNodes over permuted operands
 * (benchmarks/permuted_contraction/bench_permuted_contraction.cpp,
 * benchmarks/multilevel_contraction/bench_multilevel_contraction.cpp).  Step 1
 * runs on tcgen05 (TF32 x3 split, fp32 accumulation in TMEM) with TMA reading
 * the permuted operands in place; step 2 is fused into its epilogue, so T
 * never reaches memory unless `T` is non-NULL (then it is also stored, for
 * checking).  R is overwritten.  `workspace` holds the split operands:
 * to_chain_workspace_bytes(E) bytes.  Asynchronous on `stream`.
 */
size_t to_chain_workspace_bytes(int32_t E);
int to_chain_f32(int32_t E, const float* A, const float* B, const float* C, float* R, float* T,
                 void* workspace, size_t workspace_bytes, void* stream);
/* Useful flops of one chain: 2 E^6 + 2 E^4. */
double to_chain_flops(int32_t E);

/* One contraction as a dense GEMM on the tensor cores:
 *   C[m][n] = sum_k A[m][k] * B[n][k]
 * with both operands K-major and given split into TF32 parts, A = Ahi + Alo
 * and B = Bhi + Blo elementwise (hi = the value rounded to TF32, lo = the
 * exact remainder); the product is formed from three TF32 products (the lo*lo
 * term, about 2^-22 relative, is dropped) accumulated in fp32.  This is the
 * path the frontend lowers a large contraction of two inputs to (the
 * reference's team contraction evaluator, include/TensorOperations/Evaluator/
 * Team.hpp:318-927, with its permuted operands, Permute.hpp:127-228, packed
 * by the frontend).  Mp, Np, Kp must be positive multiples of 128, 256 and
 * 32 (pad with zeros); A* are [Mp][Kp], B* [Np][Kp], C [Mp][Np], row-major
 * fp32 in device memory, 16-byte aligned.  C is overwritten (when the tiles
 * leave the last wave of SMs less than half full, those tiles are split in K
 * between two CTAs that add into rows of C zeroed first on `stream`).
 * Asynchronous on `stream`; allocates nothing. */
int to_gemm_tf32x3(int64_t Mp, int64_t Np, int64_t Kp, const float* Ahi, const float* Alo,
                   const float* Bhi, const float* Blo, float* C, void* stream);

/* ---------------------------------------------------------------------- */
/* Level-graph lowering                                                    */
/* ---------------------------------------------------------------------- */
/*
 * The header-only C++ frontend (make_level_graph / add / outputs / execute)
 * plans a level graph at compile time -- slots, level-timeline liveness,
 * pooled scratch, tiles -- and lowers the plan to this descriptor before every
 * launch (the reference launches from LevelGraph::launch / lg_execute,
 * include/TensorOperations/LevelGraph.hpp:576-628,718-733).  The library
 * re-checks the plan independently and returns the launch shape:
 *   - every pair of slots sharing a pool has disjoint live ranges and every
 *     pool is large enough for its slots (else TO_ERR_INVALID_ARGUMENT);
 *   - a label declared whole on a staged input is not longer than its tile
 *     (TO_ERR_GRID; the reference aborts, LevelGraph.hpp:519-522);
 *   - league = product over blocked labels of ceil(extent / tile);
 *   - team: the requested size (1..1024) or, when <= 0, the smallest multiple
 *     of 32 covering the widest level, clamped to [64, 512];
 *   - with query_device != 0, the scratch must fit the current device's
 *     opt-in shared memory per block (TO_ERR_SCRATCH).
 * Host only apart from the optional device-attribute query.
 */
typedef struct to_level_plan_desc {
  int32_t value_bytes;          /* sizeof(value type)                          */
  int32_t num_levels;
  int32_t num_slots;
  int32_t num_pools;
  const int32_t* level_kind;    /* [num_levels] 0 stage, 1 contraction, 2 combine,
                                   3 contraction staging its own operand tiles */
  const int32_t* level_members; /* [num_levels]                                */
  const int64_t* level_space;   /* [num_levels] items of the level's one loop  */
  const int32_t* slot_def;      /* [num_slots] level that writes the slot      */
  const int32_t* slot_last;     /* [num_slots] last level reading it (roots: num_levels) */
  const int32_t* slot_pool;     /* [num_slots]                                 */
  const int64_t* slot_bytes;    /* [num_slots]                                 */
  const int64_t* pool_offset;   /* [num_pools + 1] byte offsets, then the total */
  int32_t grid_rank;            /* number of blocked labels carried by stages  */
  int32_t num_whole;            /* whole-label checks                          */
  const int64_t* grid_extent;   /* [grid_rank] global extent per blocked label */
  const int32_t* grid_tile;     /* [grid_rank]                                 */
  const int64_t* whole_extent;  /* [num_whole] staged extent along a whole label */
  const int32_t* whole_tile;    /* [num_whole]                                 */
  int32_t team_size;            /* <= 0: automatic                             */
  int32_t reserved0;
} to_level_plan_desc;

typedef struct to_level_launch {
  int64_t league;         /* CTAs (one per grid tile)                          */
  int64_t scratch_bytes;  /* dynamic shared memory per CTA                     */
  int32_t team;           /* threads per CTA                                   */
  int32_t reserved0;
} to_level_launch;

int to_level_plan_lower(const to_level_plan_desc* desc, int32_t query_device,
                        to_level_launch* out);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* TENSOROPERATIONS_B200_H_ */
