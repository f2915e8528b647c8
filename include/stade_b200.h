/*
 * stade_b200.h -- C ABI of libstade_b200.so, a B200 (sm_100a) execution backend
 * for the derivative code that STADE.jl generates.
 *
 * Every adjoint entry point below replaces one host function `<k>_b_cuda` that
 * STADE's CUDA port emits (`cgen_emit`, src/STADE.jl:12062-12111, named by
 * `cgen_host_fname`, src/STADE.jl:12018) for the adjoint `<k>_b` of a primal
 * kernel `<k>` (`agen_fname`, src/STADE.jl:3442), or the HVP `<k>_hv`
 * (`hvp_fname`, src/STADE.jl:6806).
 *
 * Argument order is the generated one (`agen_signature_args`,
 * src/STADE.jl:3455-3465): every primal argument in order, each float argument
 * (array or scalar) immediately followed by its adjoint, integer arguments
 * once, then stack (tape) arrays. HVP entry points append one (tangent,
 * adjoint-of-tangent) pair per float argument (src/STADE.jl:6751-6758).
 * A trailing `const stade_opts*` carries the stream and the workspace.
 *
 * Conventions
 *  - Arrays are DEVICE pointers to caller-owned memory in the flat layout the
 *    primal indexes by hand (row-major `(i - 1) * n + j` in 1-based Julia terms;
 *    element [i][j] at offset i * n + j here).
 *  - The kernels run the forward sweep (primal outputs and scratch are left
 *    with their forward values, `loss` is accumulated), ADD into every adjoint
 *    output, and leave every consumed intermediate adjoint at zero, exactly as
 *    the generated sweep does (`__oldb_N = vb; vb = 0.0`,
 *    `agen_backward_assign`, src/STADE.jl:6605). An intermediate adjoint that
 *    is non-zero on entry acts as a seed, as in the generated code.
 *  - A scalar float argument's adjoint, which the generated Julia returns by
 *    value (`emit_return_scalars`, src/STADE.jl:2072), is an in/out pointer:
 *    its entry value is the starting value and the sweep adds to it. It is a
 *    device pointer unless `opts->flags` has STADE_HOST_SCALARS, in which case
 *    it is a host pointer and the call synchronises its stream.
 *  - Calls are stream-ordered and asynchronous. Nothing on the hot path
 *    allocates device memory when the caller passes a workspace of at least
 *    the queried size; with `opts->workspace == NULL` the library uses a
 *    per-device cached buffer that it grows (once) on first use.
 *  - No floating-point atomics are used on any result path: cross-block sums
 *    run in a fixed order, so repeated calls give bit-identical results.
 *  - Every function returns a stade_status; stade_last_error() gives text.
 */
#ifndef STADE_B200_H
#define STADE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int stade_status;
#define STADE_OK         0
#define STADE_EINVAL     1  /* bad shape, null pointer, size overflow       */
#define STADE_ECUDA      2  /* a CUDA runtime call failed                    */
#define STADE_ENCCL      3  /* an NCCL call failed                           */
#define STADE_ETIMEDOUT  4  /* a bounded wait ran out (device or host side) */
#define STADE_ENOTSUP    5  /* shape outside what the kernels support        */
#define STADE_EREPLICA   6  /* check_replicas: buffers differ across ranks   */

#define STADE_HOST_SCALARS  0x1u  /* scalar adjoint out-params are host pointers */

typedef struct stade_opts {
  void*    stream;          /* cudaStream_t; NULL = the legacy default stream     */
  void*    workspace;       /* device scratch; NULL = library-managed cache       */
  size_t   workspace_bytes; /* size of `workspace` in bytes                       */
  uint32_t flags;           /* STADE_HOST_SCALARS                                 */
} stade_opts;

/* Library state ------------------------------------------------------------ */
const char* stade_last_error(void);          /* thread-local message of the last failure */
const char* stade_version(void);
int         stade_kernel_launches(void);     /* kernels this thread launched since the last reset */
void        stade_reset_kernel_launches(void);
/* Bytes of the library-managed workspace cache on the current device (0 when
 * no entry point has needed one there: every call so far passed its own
 * workspace or needed none). */
size_t      stade_workspace_cached_bytes(void);
/* Phase profiler (tracing): when enabled, entry points bracket each phase
 * with CUDA events on their stream; stade_profile_read waits for them and
 * sums device milliseconds per phase name (names: max entries of name_len
 * bytes each). Returns the number of distinct phases recorded. */
/* Sticky device-side error word of the kernels with bounded waits (the
 * tensor-core pipeline): 0 = none; nonzero = a wait ran out and the results of
 * that call are invalid. Reading it waits for the device and clears it. */
int         stade_device_error(void);
/* Check of the device-side wait guard (no counterpart in the reference, whose
 * kernels have no bounded waits): one kernel waits on an mbarrier nothing
 * ever arrives on, with the tensor-core kernels' own wait loop limited to
 * wait_cycles SM clock cycles (1000 .. ~4e9, the kernels' own limit); the wait
 * gives up, sets the device error word and the kernel returns. Synchronises
 * the stream. Returns STADE_ETIMEDOUT when the guard worked; afterwards
 * stade_device_error() reads nonzero (and clears it), and the context stays
 * usable. */
stade_status stade_check_bounded_wait(int64_t wait_cycles, const stade_opts* opts);
void        stade_profile_enable(int on);
int         stade_profile_read(char* names, int name_len, double* ms, int* counts, int max);

/* ---------------------------------------------------------------------------
 * C1  affine_ls: y = W x + b per sample, loss += 0.5 sum (y - t)^2.
 * Replaces `affine_ls_b_cuda(loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb,
 * n_s, n_o, n_i)`; generated-code pattern of test/val-corpus/affine_loss_b.jl:5-23
 * and test/val-corpus/matvec_loss_b.jl:5-27.
 * w: n_o x n_i, b: n_o, x: n_s x n_i, t, y: n_s x n_o (Float64).
 * ------------------------------------------------------------------------- */
size_t stade_affine_ls_b_f64_workspace(int64_t n_s, int64_t n_o, int64_t n_i);
stade_status stade_affine_ls_b_f64(double* loss, const double* lossb,
                                   const double* w, double* wb,
                                   const double* b, double* bb,
                                   const double* x, double* xb,
                                   const double* t, double* tb,
                                   double* y, double* yb,
                                   int64_t n_s, int64_t n_o, int64_t n_i,
                                   const stade_opts* opts);

/* Allocation-free variant of stade_affine_ls_b_f64. It has no counterpart in
 * the reference. For callers that cannot allocate device memory where they
 * run the sweep (all device memory handed to their own pool, a fixed memory
 * plan, a thread that must not block on cudaMalloc) and cannot size and pass
 * a workspace: the per-block partial sums live in a fixed 4 MiB array in the
 * library's own device memory, held by every GPU that loads the library until
 * the process exits. The call makes no cudaMalloc, cudaFree or other
 * allocating call; opts->workspace is ignored. Every call looks up the
 * array's device address on the current device (cudaGetSymbolAddress, a query
 * that allocates nothing), so a cudaDeviceReset between calls is harmless; the
 * first call on a device also loads the library's device code there, so make
 * that first call before any stream capture. Sizes whose
 * partial sums exceed the array (stade_affine_ls_b_f64_noalloc_max_scratch()
 * bytes; the full 1024 x 64 x 32 configuration needs 2.03 MiB) return
 * STADE_EINVAL. All calls share the one array: calls that overlap on the GPU
 * (different streams, no ordering between them) race on it. Results equal
 * those of stade_affine_ls_b_f64. */
size_t stade_affine_ls_b_f64_noalloc_max_scratch(void);
stade_status stade_affine_ls_b_f64_noalloc(double* loss, const double* lossb,
                                           const double* w, double* wb,
                                           const double* b, double* bb,
                                           const double* x, double* xb,
                                           const double* t, double* tb,
                                           double* y, double* yb,
                                           int64_t n_s, int64_t n_o, int64_t n_i,
                                           const stade_opts* opts);

/* ---------------------------------------------------------------------------
 * C2  mlp2_ce: h = tanh(x W1 + b1), z = h W2 + b2, softmax cross-entropy
 * against y, one sample per row. Float32 (STADE's precision conversion,
 * `cgen_convert_precision`, src/STADE.jl:15351). Replaces
 * `mlp2_ce_b_cuda(loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2,
 * b2b, h, hb, z, zb, p, pb, n_s, n_i, n_h, n_o)`; pattern of
 * test/val-corpus/mlp1d_b.jl:5-78 and the softmax of
 * test/val-corpus/transformer_b.jl:615-667.
 * x: n_s x n_i, y, z, p: n_s x n_o, w1: n_i x n_h, w2: n_h x n_o, h: n_s x n_h.
 * Supported: n_o <= 32.
 * ------------------------------------------------------------------------- */
size_t stade_mlp2_ce_b_f32_workspace(int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o);
stade_status stade_mlp2_ce_b_f32(float* loss, const float* lossb,
                                 const float* x, float* xb,
                                 const float* y, float* yb,
                                 const float* w1, float* w1b,
                                 const float* b1, float* b1b,
                                 const float* w2, float* w2b,
                                 const float* b2, float* b2b,
                                 float* h, float* hb,
                                 float* z, float* zb,
                                 float* p, float* pb,
                                 int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o,
                                 const stade_opts* opts);

/* ---------------------------------------------------------------------------
 * C3  heat2d: n_step explicit steps of the periodic 5-point heat equation on
 * an n x n grid, u <- u + alpha (sum of 4 neighbours - 4 u), then
 * loss += sum u^2. Replaces `heat2d_b_cuda(loss, lossb, u, ub, un, unb, alpha,
 * alphab, n, n_step, u_stack)` and `initstacks_heat2d_b(n, n_step)`; time loop
 * and tape of test/val-corpus/advection_b.jl:1-37, scatter adjoint of
 * test/val-corpus/stencil_loss_b.jl:12-21.
 * u_stack holds n_step * n * n values; slot ((idx - 1) + (i_t - 1) n^2) + 1
 * (thread loop fastest, as the generated tape index) receives the state u
 * before step i_t overwrites it. On exit u holds the initial state again
 * (restored from the tape), un the final state, unb is zero, ub holds the
 * gradient, *alphab is increased by dloss/dalpha.
 * ------------------------------------------------------------------------- */
int64_t stade_initstacks_heat2d_b(int64_t n, int64_t n_step);  /* u_stack length (elements) */
size_t  stade_heat2d_b_f64_workspace(int64_t n, int64_t n_step);
stade_status stade_heat2d_b_f64(double* loss, const double* lossb,
                                double* u, double* ub,
                                double* un, double* unb,
                                double alpha, double* alphab,
                                int64_t n, int64_t n_step,
                                double* u_stack,
                                const stade_opts* opts);

/* ---------------------------------------------------------------------------
 * C4  conv1d_relu_mse: valid 1-D convolution over channels, ReLU, mean squared
 * error against t. Float32. Replaces `conv1d_relu_mse_b_cuda(loss, lossb, x,
 * xb, w, wb, t, tb, z, zb, r, rb, n_b, n_c, n_l, n_o, n_k)`; pattern of
 * test/val-corpus/selfrace_conv_b.jl:5-35 (valid convolution adjoint) and the
 * max partial of der_partials_maxmin (src/STADE.jl:1489).
 * x: n_b x n_c x n_l, w: n_o x n_c x n_k, t, z, r: n_b x n_o x (n_l - n_k + 1).
 * ------------------------------------------------------------------------- */
size_t stade_conv1d_relu_mse_b_f32_workspace(int64_t n_b, int64_t n_c, int64_t n_l,
                                             int64_t n_o, int64_t n_k);
stade_status stade_conv1d_relu_mse_b_f32(float* loss, const float* lossb,
                                         const float* x, float* xb,
                                         const float* w, float* wb,
                                         const float* t, float* tb,
                                         float* z, float* zb,
                                         float* r, float* rb,
                                         int64_t n_b, int64_t n_c, int64_t n_l,
                                         int64_t n_o, int64_t n_k,
                                         const stade_opts* opts);

/* ---------------------------------------------------------------------------
 * C5  mlp2_ce_hv: forward-over-reverse Hessian-vector product of mlp2_ce in
 * Float64. Replaces `mlp2_ce_hv_cuda(...)` with the argument layout of
 * `hvp_emit` (src/STADE.jl:6751-6758; exemplar test/val-corpus/mlp1d_hv.jl):
 * the adjoint list, then one (tangent, adjoint-of-tangent) pair per float
 * argument in primal order.
 * ------------------------------------------------------------------------- */
size_t stade_mlp2_ce_hv_f64_workspace(int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o);
stade_status stade_mlp2_ce_hv_f64(double* loss, const double* lossb,
                                  const double* x, double* xb,
                                  const double* y, double* yb,
                                  const double* w1, double* w1b,
                                  const double* b1, double* b1b,
                                  const double* w2, double* w2b,
                                  const double* b2, double* b2b,
                                  double* h, double* hb,
                                  double* z, double* zb,
                                  double* p, double* pb,
                                  int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o,
                                  double* lossd, const double* lossbd,
                                  const double* xd, double* xbd,
                                  const double* yd, double* ybd,
                                  const double* w1d, double* w1bd,
                                  const double* b1d, double* b1bd,
                                  const double* w2d, double* w2bd,
                                  const double* b2d, double* b2bd,
                                  double* hd, double* hbd,
                                  double* zd, double* zbd,
                                  double* pd, double* pbd,
                                  const stade_opts* opts);

/* ---------------------------------------------------------------------------
 * Tangent (forward-mode) sweeps `<k>_d`. Replace the functions
 * `stade_tangent_file` writes (tgen_emit, src/STADE.jl:3271-3279): one sweep
 * in primal order, every active statement preceded by its tangent line.
 * Arguments in tgen_signature_args order (src/STADE.jl:3306-3316): each float
 * argument followed by its `d` shadow, integer sizes once. Scratch arrays and
 * their shadows are overwritten; loss and lossd accumulate. No scalar argument
 * of these primals is reassigned, so nothing is returned (a scalar's tangent,
 * alphad, is passed by value).
 * ------------------------------------------------------------------------- */
size_t stade_affine_ls_d_f64_workspace(int64_t n_s, int64_t n_o, int64_t n_i);
stade_status stade_affine_ls_d_f64(double* loss, double* lossd,
                                   const double* w, const double* wd,
                                   const double* b, const double* bd,
                                   const double* x, const double* xd,
                                   const double* t, const double* td,
                                   double* y, double* yd,
                                   int64_t n_s, int64_t n_o, int64_t n_i,
                                   const stade_opts* opts);
size_t stade_mlp2_ce_d_f32_workspace(int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o);
size_t stade_mlp2_ce_d_f64_workspace(int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o);
stade_status stade_mlp2_ce_d_f32(float* loss, float* lossd, const float* x, const float* xd,
                                 const float* y, const float* yd, const float* w1,
                                 const float* w1d, const float* b1, const float* b1d,
                                 const float* w2, const float* w2d, const float* b2,
                                 const float* b2d, float* h, float* hd, float* z, float* zd,
                                 float* p, float* pd, int64_t n_s, int64_t n_i, int64_t n_h,
                                 int64_t n_o, const stade_opts* opts);
stade_status stade_mlp2_ce_d_f64(double* loss, double* lossd, const double* x, const double* xd,
                                 const double* y, const double* yd, const double* w1,
                                 const double* w1d, const double* b1, const double* b1d,
                                 const double* w2, const double* w2d, const double* b2,
                                 const double* b2d, double* h, double* hd, double* z,
                                 double* zd, double* p, double* pd, int64_t n_s, int64_t n_i,
                                 int64_t n_h, int64_t n_o, const stade_opts* opts);
size_t stade_heat2d_d_f64_workspace(int64_t n, int64_t n_step);
/* On exit u == un and ud == und hold the final state and its tangent, as the
 * generated copy loop leaves them. */
stade_status stade_heat2d_d_f64(double* loss, double* lossd, double* u, double* ud,
                                double* un, double* und, double alpha, double alphad,
                                int64_t n, int64_t n_step, const stade_opts* opts);
size_t stade_conv1d_relu_mse_d_f32_workspace(int64_t n_b, int64_t n_c, int64_t n_l,
                                             int64_t n_o, int64_t n_k);
stade_status stade_conv1d_relu_mse_d_f32(float* loss, float* lossd,
                                         const float* x, const float* xd,
                                         const float* w, const float* wd,
                                         const float* t, const float* td,
                                         float* z, float* zd, float* r, float* rd,
                                         int64_t n_b, int64_t n_c, int64_t n_l,
                                         int64_t n_o, int64_t n_k, const stade_opts* opts);

/* ---------------------------------------------------------------------------
 * Data-parallel epilogue (replaces the MPI functions `ddpgen_` emits,
 * src/STADE.jl:17595-17696). One communicator per GPU, one process per GPU.
 * ------------------------------------------------------------------------- */
typedef struct stade_comm stade_comm;

#define STADE_F32 0
#define STADE_F64 1

/* 128 opaque bytes made on one rank and broadcast by the caller (MPI, a
 * torch.distributed store, a file) before stade_comm_init on every rank. */
stade_status stade_comm_unique_id(unsigned char id_out[128]);
/* Collective over `nranks` processes; binds the current CUDA device. Fails
 * with STADE_ETIMEDOUT when the peers do not all join within timeout_ms. */
stade_status stade_comm_init(const unsigned char id[128], int nranks, int rank,
                             int timeout_ms, stade_comm** comm_out);
stade_status stade_comm_destroy(stade_comm* comm);
int          stade_comm_rank(const stade_comm* comm);
int          stade_comm_size(const stade_comm* comm);

/* `fill!(b, 0.0)` for every buffer (ddpgen_fill_fn, src/STADE.jl:17589-17597). */
stade_status stade_ddp_zero(void* const* bufs, const int64_t* counts, int nbuf,
                            int dtype, const stade_opts* opts);
/* `MPI.Allreduce!(b, +, comm)` for every buffer plus the global sample count
 * (ddpgen_allreduce_accum_expr, src/STADE.jl:17629-17645), as ONE collective
 * over one contiguous bucket. *n_global is a host pointer. */
stade_status stade_ddp_allreduce_sum(stade_comm* comm, void* const* bufs,
                                     const int64_t* counts, int nbuf, int dtype,
                                     int64_t n_local, int64_t* n_global,
                                     const stade_opts* opts);
/* The two checksums per buffer (sum, sum of abs) compared by min against max
 * across ranks (ddpgen_check_expr, src/STADE.jl:17665-17696). Returns
 * STADE_EREPLICA and sets bit i of *bad_mask (host) when buffer i differs. */
stade_status stade_ddp_check_replicas(stade_comm* comm, const void* const* bufs,
                                      const int64_t* counts, int nbuf, int dtype,
                                      uint64_t* bad_mask, const stade_opts* opts);

/* The generated epilogue functions of mlp2_ce in adjoint mode with
 * per_sample = [:x, :y] (roles by ddpgen_roles, src/STADE.jl:17404):
 *   :accum  w1b b1b w2b b2b       :reduced loss       :seed lossb
 *   :local  xb yb hb zb pb        :shared  w1 b1 w2 b2                    */
stade_status stade_mlp2_ce_b_reset_accum_f32(float* w1b, float* b1b, float* w2b, float* b2b,
                                             int64_t n_i, int64_t n_h, int64_t n_o,
                                             const stade_opts* opts);
stade_status stade_mlp2_ce_b_reset_reduced_f32(float* loss, const stade_opts* opts);
stade_status stade_mlp2_ce_b_reset_local_f32(float* xb, float* yb, float* hb, float* zb, float* pb,
                                             int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o,
                                             const stade_opts* opts);
stade_status stade_mlp2_ce_b_allreduce_accum_f32(float* w1b, float* b1b, float* w2b, float* b2b,
                                                 int64_t n_i, int64_t n_h, int64_t n_o,
                                                 int64_t n_local, stade_comm* comm,
                                                 int64_t* n_global, const stade_opts* opts);
stade_status stade_mlp2_ce_b_allreduce_reduced_f32(float* loss, stade_comm* comm,
                                                   const stade_opts* opts);
stade_status stade_mlp2_ce_b_check_replicas_f32(const float* w1, const float* b1,
                                                const float* w2, const float* b2,
                                                const float* lossb,
                                                int64_t n_i, int64_t n_h, int64_t n_o,
                                                stade_comm* comm, uint64_t* bad_mask,
                                                const stade_opts* opts);

/* The generated epilogue functions of conv1d_relu_mse in adjoint mode with
 * per_sample = [:x, :t] (`conv1d_relu_mse_b_reset_accum!` ...
 * `conv1d_relu_mse_b_check_replicas`, ddpgen_fname src/STADE.jl:17578-17582;
 * roles by ddpgen_roles, src/STADE.jl:17404):
 *   :accum  wb                    :reduced loss       :seed lossb
 *   :local  xb tb zb rb           :shared  w
 * The mean loss (1 / (n_b n_o n_lo) inside the primal) makes a rank's loss
 * seed and summed loss carry its own batch's count: scale lossb by
 * n_local / n_global before the sweep and the summed loss by the same factor
 * after (exact for power-of-two rank counts). */
stade_status stade_conv1d_relu_mse_b_reset_accum_f32(float* wb, int64_t n_o, int64_t n_c,
                                                     int64_t n_k, const stade_opts* opts);
stade_status stade_conv1d_relu_mse_b_reset_reduced_f32(float* loss, const stade_opts* opts);
stade_status stade_conv1d_relu_mse_b_reset_local_f32(float* xb, float* tb, float* zb, float* rb,
                                                     int64_t n_b, int64_t n_c, int64_t n_l,
                                                     int64_t n_o, int64_t n_k,
                                                     const stade_opts* opts);
stade_status stade_conv1d_relu_mse_b_allreduce_accum_f32(float* wb, int64_t n_o, int64_t n_c,
                                                         int64_t n_k, int64_t n_local,
                                                         stade_comm* comm, int64_t* n_global,
                                                         const stade_opts* opts);
stade_status stade_conv1d_relu_mse_b_allreduce_reduced_f32(float* loss, stade_comm* comm,
                                                           const stade_opts* opts);
stade_status stade_conv1d_relu_mse_b_check_replicas_f32(const float* w, const float* lossb,
                                                        int64_t n_o, int64_t n_c, int64_t n_k,
                                                        stade_comm* comm, uint64_t* bad_mask,
                                                        const stade_opts* opts);

/* The generated epilogue functions of mlp2_ce in hvp mode, with the `_hv`
 * suffix ddpgen_mode_suffix gives that mode (`mlp2_ce_hv_reset_accum!` ...,
 * src/STADE.jl:17578-17582), per_sample = [:x, :y]:
 *   :accum   w1b b1b w2b b2b w1bd b1bd w2bd b2bd     :reduced loss lossd
 *   :local   xb yb hb zb pb xbd ybd hbd zbd pbd      :seed    lossb lossbd
 *   :shared  w1 b1 w2 b2 w1d b1d w2d b2d
 * allreduce_accum sums all eight :accum buffers in one NCCL bucket. */
stade_status stade_mlp2_ce_hv_reset_accum_f64(double* w1b, double* b1b, double* w2b, double* b2b,
                                              double* w1bd, double* b1bd, double* w2bd,
                                              double* b2bd, int64_t n_i, int64_t n_h, int64_t n_o,
                                              const stade_opts* opts);
stade_status stade_mlp2_ce_hv_reset_reduced_f64(double* loss, double* lossd,
                                                const stade_opts* opts);
stade_status stade_mlp2_ce_hv_reset_local_f64(double* xb, double* yb, double* hb, double* zb,
                                              double* pb, double* xbd, double* ybd, double* hbd,
                                              double* zbd, double* pbd, int64_t n_s, int64_t n_i,
                                              int64_t n_h, int64_t n_o, const stade_opts* opts);
stade_status stade_mlp2_ce_hv_allreduce_accum_f64(double* w1b, double* b1b, double* w2b,
                                                  double* b2b, double* w1bd, double* b1bd,
                                                  double* w2bd, double* b2bd, int64_t n_i,
                                                  int64_t n_h, int64_t n_o, int64_t n_local,
                                                  stade_comm* comm, int64_t* n_global,
                                                  const stade_opts* opts);
stade_status stade_mlp2_ce_hv_allreduce_reduced_f64(double* loss, double* lossd, stade_comm* comm,
                                                    const stade_opts* opts);
stade_status stade_mlp2_ce_hv_check_replicas_f64(const double* w1, const double* b1,
                                                 const double* w2, const double* b2,
                                                 const double* w1d, const double* b1d,
                                                 const double* w2d, const double* b2d,
                                                 const double* lossb, const double* lossbd,
                                                 int64_t n_i, int64_t n_h, int64_t n_o,
                                                 stade_comm* comm, uint64_t* bad_mask,
                                                 const stade_opts* opts);

/* ---------------------------------------------------------------------------
 * C3 over several GPUs: heat2d_b on row slabs. No reference counterpart (the
 * reference parallelises only over samples, ddpgen_); this is the domain
 * decomposition the configuration's grid needs across GPUs. Rank r of the
 * communicator owns `rows` consecutive grid rows directly below rank r-1's
 * (rank 0's top neighbour is the last rank: the grid is periodic); the
 * slabs' rows add up to n. u, ub, un, unb are this rank's rows (rows x n,
 * row-major, 16-byte aligned) with the meaning they have in
 * stade_heat2d_b_f64; *loss and *alphab receive the sums over ALL slabs on
 * every rank. u_stack holds stade_initstacks_heat2d_b_slab(n, n_step, rows)
 * values: per step one state with a halo row above and below. Per step and
 * per sweep direction one 8 n-byte row goes to each neighbour over NCCL,
 * overlapped with the slab's interior rows. comm == NULL is allowed when
 * rows == n (one slab holds the grid). With STADE_HOST_SCALARS the call
 * waits for the stream, bounded by the communicator's timeout; otherwise it
 * returns with the work queued.
 * ------------------------------------------------------------------------- */
int64_t stade_initstacks_heat2d_b_slab(int64_t n, int64_t n_step, int64_t rows);
size_t  stade_heat2d_b_f64_slab_workspace(int64_t n, int64_t n_step, int64_t rows);
stade_status stade_heat2d_b_f64_slab(double* loss, const double* lossb,
                                     double* u, double* ub,
                                     double* un, double* unb,
                                     double alpha, double* alphab,
                                     int64_t n, int64_t n_step,
                                     double* u_stack, int64_t rows,
                                     stade_comm* comm, const stade_opts* opts);

/* ---------------------------------------------------------------------------
 * Synthetic inputs (host side). Seed = FNV-1a-64 of a name, the scheme of
 * `val_stable_seed` (src/STADE.jl:16619-16626); draws from xoshiro256**
 * split into independent 2^20-element chunks; normals by the Box-Muller
 * cosine branch of `val_normal` (src/STADE.jl:16628-16638).
 * ------------------------------------------------------------------------- */
uint64_t stade_fnv1a64(const char* s);
void stade_fill_normal_f64(double* out, int64_t n, uint64_t seed, double mean, double std);
void stade_fill_normal_f32(float* out, int64_t n, uint64_t seed, double mean, double std);
void stade_fill_uniform_f64(double* out, int64_t n, uint64_t seed, double lo, double hi);
void stade_fill_uniform_f32(float* out, int64_t n, uint64_t seed, double lo, double hi);
/* one-hot rows of width n_o, class drawn uniformly per row */
void stade_fill_onehot_f32(float* out, int64_t n_rows, int64_t n_o, uint64_t seed);
void stade_fill_onehot_f64(double* out, int64_t n_rows, int64_t n_o, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif /* STADE_B200_H */
