/*
 * sla_b200.h -- C ABI of libsla_b200.so, the sm_100a (B200) iterative-solve
 * hot path behind torch-sla's `pytorch` backend.
 *
 * Conventions
 *   - Every pointer argument named as "device" is CUDA device memory owned by
 *     the caller (the Python layer allocates it through PyTorch's caching
 *     allocator). The library never frees caller memory and never calls
 *     cudaMalloc on the solve path: scratch space is a caller-provided
 *     workspace whose size is returned by the matching *_workspace() query.
 *   - All work is enqueued on the caller's stream (`sla_stream_t` is a
 *     cudaStream_t). Functions that must return a host value produced on the
 *     device (coalesced nnz, iteration counts) synchronise that stream.
 *   - Return value: 0 = OK; > 0 = numerical outcome (not converged,
 *     breakdown); < 0 = error (invalid argument, CUDA/NCCL error, timeout).
 *   - dtype codes: SLA_F32 (float) and SLA_F64 (double). Index arrays are
 *     int32 (local problem sizes stay below 2^31), COO inputs are int64 as in
 *     torch-sla.
 *
 * Each entry point cites the torch-sla function whose work it replaces
 * (paths relative to the torch-sla source tree).
 */
#ifndef SLA_B200_H
#define SLA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *sla_stream_t; /* identical to cudaStream_t */

enum { SLA_F32 = 0, SLA_F64 = 1 };

enum {
  SLA_OK = 0,
  SLA_NOT_CONVERGED = 1,   /* maxiter reached (torch-sla warns)            */
  SLA_BREAKDOWN = 2,       /* BiCGStab rho / t.t / omega guard fired        */
  SLA_ERR_INVALID = -1,    /* bad argument (sizes, dtype, null pointer)     */
  SLA_ERR_CUDA = -2,       /* a CUDA runtime call failed                    */
  SLA_ERR_NCCL = -3,       /* an NCCL call failed                           */
  SLA_ERR_TIMEOUT = -4,    /* a bounded device-side wait gave up            */
  SLA_ERR_UNSUPPORTED = -5,/* shape outside the supported envelope          */
  SLA_ERR_WORKSPACE = -6,  /* workspace smaller than *_workspace() asked,
                              or not 16-byte aligned                        */
  SLA_ERR_INDEX = -7       /* a COO index lies outside the matrix shape     */
};

/* Jacobi rules: how a diagonal d turns into the inverse used by M^{-1}. */
enum {
  SLA_JACOBI_EPS = 0,     /* 1/d, d := 1 where |d| < 100*eps(dtype)
                             (backends/pytorch_backend.py:221-235)          */
  SLA_JACOBI_CLAMP = 1,   /* 1/max(d, 1e-30)  (distributed/solve.py:95-115) */
  SLA_JACOBI_NONZERO = 2  /* |d| > 0 ? 1/d : 1 (pytorch_backend.py:2611-2614)*/
};

/* Solver path selection for sla_pcg (flags argument). */
enum {
  SLA_PCG_AUTO = 0,        /* small systems: the cluster kernel when the system
                              fits one thread-block cluster, else the persistent
                              kernel; larger systems streamed                     */
  SLA_PCG_STREAMED = 1,    /* three kernels per iteration                         */
  SLA_PCG_PERSISTENT = 2,  /* one cooperative launch for the whole solve          */
  SLA_PCG_CLUSTER = 3      /* one thread-block cluster for the whole solve (the
                              vectors and a diagonal-offset view in distributed
                              shared memory); SLA_ERR_UNSUPPORTED when it does
                              not fit                                             */
};

/* SELL-32 (SELL-C-sigma with C = 32, sigma = 1) matrix view. Slice s holds
 * 32 consecutive row slots; entry j of slot l sits at
 * slice_ptr[s] + 32*j + l. Padding entries have col == -1.
 *
 * Diagonal-offset views (n_diags > 0): every row's columns lie on the
 * n_diags diagonals diag_offsets[0] < ... < diag_offsets[n_diags-1]; the
 * layout is uniform (width n_diags), entry j of a slot belongs to column
 * row + diag_offsets[j] and `col` is not stored (NULL). Entries whose
 * diagonal the row does not use, or whose column falls outside
 * [0, n_cols), hold value 0 and are skipped. The summation order of a row
 * (ascending column) is the same as in the explicit layout. */
#define SLA_MAX_DIAGS 32
typedef struct {
  int64_t n_slots;           /* row slots covered by this view               */
  int64_t n_slices;          /* ceil(n_slots / 32)                           */
  const int32_t *slice_ptr;  /* device [n_slices + 1]                        */
  const int32_t *col;        /* device [slice_ptr[n_slices]]                 */
  const void *val;           /* device, same length, dtype T                 */
  const int32_t *row_ids;    /* device [n_slots] row of each slot, or NULL
                                when slot i is row i                          */
  int32_t max_width;         /* widest slice (entries per slot)              */
  int32_t uniform_width;     /* W when every slice has width W (then
                                slice_ptr[s] == 32*W*s), else 0               */
  int64_t n_cols;            /* columns of the matrix (diagonal-offset views) */
  int64_t row_base;          /* row_ids == NULL: slot i is row row_base + i   */
  int32_t n_diags;           /* > 0: diagonal-offset view, 5, 7 or 27          */
  int32_t diag_offsets[SLA_MAX_DIAGS]; /* ascending, first n_diags used     */
} sla_sell_t;

typedef struct {
  int64_t iterations;        /* torch-sla's iteration count convention       */
  double residual;           /* recursive residual norm at exit              */
  int32_t status;            /* SLA_OK / SLA_NOT_CONVERGED / SLA_BREAKDOWN    */
  int32_t reason;            /* solver-specific detail, 0 if none            */
} sla_solve_info_t;

/* ------------------------------------------------------------------ misc */
/* Version of this interface; 2 since sla_sell_t carries n_cols, row_base
 * and the diagonal offsets, 3 since sla_pcg_mixed, 4 since
 * sla_p2p_profile_read (and one-rank peer-memory plans), 5 since
 * sla_spmv_rows_csr. _lib.py refuses a
 * library with another. */
#define SLA_ABI_VERSION 5
int sla_abi_version(void);
const char *sla_status_string(int status);
/* Kernels this library has launched in this process (all devices). */
int64_t sla_kernel_launch_count(void);
/* Per-kernel-class device time (ms) and launch count gathered while
 * sampling is on; class 0 is the SpMV-bearing kernel of the running solver. */
int sla_profile_enable(int enable, int sample_every);
int sla_profile_read(int kernel_class, double *total_ms, int64_t *launches);

/* ------------------------------------------------------------ COO -> CSR */
/* Replaces CachedSparseMatrix.__init__'s sparse_coo_tensor(...).to_sparse_csr()
 * (backends/pytorch_backend.py:114-152) and the int32 CSR of shard_matvec
 * (distributed/matvec.py:271-294): sorts by (row, col), sums duplicates in
 * input order, emits int32 CSR. Optional outputs: src_index[t] = input
 * position of the t-th sorted entry, seg_ptr[e] = first sorted position of
 * CSR entry e (seg_ptr has nnz_out + 1 entries). Synchronises `stream`. */
int sla_csr_build_workspace(int64_t n_rows, int64_t nnz, size_t *bytes);
int sla_csr_build(int dtype, const int64_t *row, const int64_t *col,
                  const void *val, int64_t nnz, int64_t n_rows, int64_t n_cols,
                  int32_t *rowptr, int32_t *colind, void *vals,
                  int64_t *src_index, int32_t *seg_ptr, int64_t *nnz_out,
                  void *workspace, size_t workspace_bytes, sla_stream_t stream);

/* ------------------------------------------------------------- SELL-32 */
/* Layout of a SELL-32 view over the CSR rows listed in row_ids (or rows
 * 0..n_slots-1), every slice padded to at least min_width entries per slot
 * (min_width = the widest row gives a uniform-width layout). Writes
 * slice_ptr and returns the padded entry count and the widest slice. */
int sla_sell_layout_workspace(int64_t n_slots, size_t *bytes);
int sla_sell_layout(const int32_t *rowptr, const int32_t *row_ids,
                    int64_t n_slots, int32_t min_width, int32_t *slice_ptr,
                    int64_t *padded_out, int32_t *max_width_out,
                    void *workspace, size_t workspace_bytes,
                    sla_stream_t stream);
int sla_sell_fill(int dtype, const int32_t *rowptr, const int32_t *colind,
                  const void *vals, const int32_t *row_ids, int64_t n_slots,
                  const int32_t *slice_ptr, int32_t *sell_col, void *sell_val,
                  sla_stream_t stream);
/* SELL-32-sigma row order (no counterpart in torch-sla, whose CSR SpMV
 * serves any pattern, pytorch_backend.py:154-161): order[t] lists the rows
 * of the view (row_ids, or 0..n_slots-1 when row_ids is NULL) with each
 * window of sigma consecutive entries sorted by decreasing row length, equal
 * lengths kept in ascending order, and every full window rotated by
 * (window index mod sigma/32) slices so that the widest slices of
 * successive windows fall on different slice positions. Passed as the row_ids of
 * sla_sell_layout / sla_sell_fill it groups rows of similar length into each
 * 32-row slice, so irregular patterns pad less. sigma is a power of two in
 * [32, 4096]. The solver and SpMV kernels accept such a view for the whole
 * matrix: its row_ids must be a permutation of 0..n-1. */
int sla_sell_sigma_order(const int32_t *rowptr, const int32_t *row_ids,
                         int64_t n_slots, int32_t sigma, int32_t *order,
                         sla_stream_t stream);

/* Distinct diagonal offsets (col - row) of the CSR rows listed in row_ids
 * (or rows 0..n_slots-1). Writes up to SLA_MAX_DIAGS ascending offsets to
 * the host array offsets_out and their count to *count_out; *count_out = -1
 * when the rows use more than SLA_MAX_DIAGS diagonals. Synchronises the
 * stream. */
int sla_sell_diag_probe_workspace(size_t *bytes);
int sla_sell_diag_probe(const int32_t *rowptr, const int32_t *colind,
                        const int32_t *row_ids, int64_t n_slots,
                        int32_t *offsets_out, int32_t *count_out,
                        void *workspace, size_t workspace_bytes,
                        sla_stream_t stream);
/* Values of a diagonal-offset view (see sla_sell_t): sell_val holds
 * ceil(n_slots/32)*32*n_diags entries and is fully written (0 where a row
 * has no entry on a diagonal). Every CSR entry of the listed rows must lie
 * on one of the n_diags ascending host-side offsets (SLA_ERR_INVALID
 * otherwise). Workspace as for the probe. Synchronises the stream. */
/* Position of every CSR entry of rows 0..n_rows-1 in the diagonal-offset
 * view with the given ascending host-side offsets:
 * (row/32)*32*n_diags + 32*j + row%32. SLA_ERR_INVALID when an entry lies on
 * none of them. Workspace as for the probe. Synchronises the stream. */
int sla_sell_diag_positions(const int32_t *rowptr, const int32_t *colind,
                            int64_t n_rows, const int32_t *offsets,
                            int32_t n_diags, int64_t *pos, void *workspace,
                            size_t workspace_bytes, sla_stream_t stream);
int sla_sell_diag_fill(int dtype, const int32_t *rowptr, const int32_t *colind,
                       const void *vals, const int32_t *row_ids, int64_t n_slots,
                       const int32_t *offsets, int32_t n_diags, void *sell_val,
                       void *workspace, size_t workspace_bytes,
                       sla_stream_t stream);

/* Inverse diagonal for Jacobi (pytorch_backend.py:167-174, 221-235;
 * distributed/solve.py:95-115). Rows without a stored diagonal use d = 0. */
int sla_jacobi_inverse(int dtype, const int32_t *rowptr, const int32_t *colind,
                       const void *vals, int64_t n_rows, int rule, void *dinv,
                       sla_stream_t stream);

/* ---------------------------------------------------------------- SpMV */
/* y[row] = sum_j A[row, j] x[j] for every slot of A (torch.mv in
 * CachedSparseMatrix.matvec, pytorch_backend.py:154-161; SparseTensor @ x,
 * sparse_tensor/matmul.py:10-85). */
int sla_spmv(int dtype, const sla_sell_t *A, const void *x, void *y,
             sla_stream_t stream);
/* y[r] = sum over CSR row r for the n_rows rows listed in `rows` (int32 CSR
 * of sla_csr_build), one warp per row: lane l sums entries l, l+32, ... in
 * ascending order, then the 32 lane sums are combined in a fixed butterfly
 * order. With sla_spmv over a SELL view of the remaining rows it forms the
 * hybrid SpMV of irregular patterns, whose long rows would otherwise keep one
 * lane of a slice busy while the rest of the grid idles. No counterpart in
 * torch-sla (its CSR torch.mv serves any pattern, pytorch_backend.py:154-161);
 * a long row's sum is ordered differently from a sequential one (agrees to
 * rounding). */
int sla_spmv_rows_csr(int dtype, const int32_t *rowptr, const int32_t *colind,
                      const void *vals, const int32_t *rows, int64_t n_rows,
                      const void *x, void *y, sla_stream_t stream);

/* g[k] = -sum_c a[row[k]*K + c] * b[col[k]*K + c] for every COO entry k,
 * repeated for `batch` independent problems laid out back to back: the
 * adjoint's value gradient (linear_solve.py:321-323,
 * batch_solve.py:138). a has n_a*K entries per problem, b has n_b*K. */
int sla_coo_value_grad(int dtype, const int64_t *row, const int64_t *col,
                       int64_t nnz, const void *a, const void *b,
                       int64_t n_a, int64_t n_b, int64_t K, int64_t batch,
                       void *g, sla_stream_t stream);

/* ------------------------------------------------------------- Krylov */
/* Jacobi-PCG / CG with torch-sla's stopping rule: stop at the start of
 * iteration i when (r,r) < max(atol, rtol*||b||)^2, iterations = i
 * (pcg_solve_optimized, pytorch_backend.py:1262-1362). dinv == NULL selects
 * preconditioner='none'. x holds the initial guess when x_is_guess != 0.
 * A covers all n rows: row_base 0, and row_ids NULL (slot i is row i) or a
 * permutation of 0..n-1 (a SELL-32-sigma order, sla_sell_sigma_order); the
 * same holds for sla_bicgstab and sla_pcg_mixed. */
int sla_pcg_workspace(int dtype, int64_t n, size_t *bytes);
int sla_pcg(int dtype, const sla_sell_t *A, const void *dinv, const void *b,
            void *x, int x_is_guess, double atol, double rtol,
            int64_t maxiter, int flags, void *workspace,
            size_t workspace_bytes, sla_solve_info_t *info,
            sla_stream_t stream);

/* Allocation-free variant of sla_pcg. It has no counterpart in torch-sla: it
 * exists for callers that cannot allocate device memory at solve time -- a
 * host application whose device memory is owned by another framework's pool,
 * a plugin that must not call cudaMalloc (which can synchronise the device
 * and fail under memory pressure), or a C/Fortran code with no allocator of
 * its own. Its scratch vectors live in one file-scope device array of
 * SLA_PCG_NOALLOC_SCRATCH_BYTES (16 MiB), held on every GPU that loads the
 * library until the process exits; that fits n <= 500,000 rows in float64
 * (1,000,000 in float32) on a 148-SM B200. Larger n returns
 * SLA_ERR_UNSUPPORTED. The caller still provides A, dinv, b and x. Each
 * call resolves the array's device address on the current device
 * (cudaGetSymbolAddress), so make the first call on a device before any
 * stream capture. The call blocks the host until the solve has finished (it
 * reads the convergence flag back every 8 iterations on the streamed path
 * and the final state at the end). All calls share the one array: calls that
 * overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller. No cudaMalloc/cudaFree or other allocating
 * routine is called. */
#define SLA_PCG_NOALLOC_SCRATCH_BYTES (16u << 20)
int sla_pcg_noalloc(int dtype, const sla_sell_t *A, const void *dinv,
                    const void *b, void *x, int x_is_guess, double atol,
                    double rtol, int64_t maxiter, int flags,
                    sla_solve_info_t *info, sla_stream_t stream);

/* Mixed-precision PCG: pytorch_solve's float32 + mixed_precision branch
 * (pytorch_backend.py:2278-2285) into pcg_solve_mixed_precision
 * (:1176-1255). A is a float32 view; Ap = (double)(A (float)p) with float32
 * accumulation; x (float64, [n]) and every vector, dot and update are
 * float64; b is float32 or float64 (b_dtype). No start-of-iteration test:
 * iteration i stops when ||r|| < max(atol, rtol*||b||) (||b|| = 0 counts
 * as 1) after its r update, iterations = i + 1. p'Ap <= 0 stops before the
 * update with SLA_BREAKDOWN (reason 5), iterations = i, the residual of the
 * previous update and *pap_out = p'Ap (pap_out may be NULL). */
enum {
  SLA_MIXED_M_F32_NONE = 0,   /* z = (double)(float)r: 'none' run in float32
                                 (pytorch_solve's M_f64 wrapper, :2281-2283) */
  SLA_MIXED_M_F32_JACOBI = 1, /* z = (double)(dinv * (float)r), dinv float32 */
  SLA_MIXED_M_F64_JACOBI = 2, /* z = dinv * r, dinv float64 (the default of
                                 pcg_solve_mixed_precision, :1211-1216)      */
  SLA_MIXED_M_F64_NONE = 3    /* z = r                                        */
};
int sla_pcg_mixed_workspace(int64_t n, size_t *bytes);
int sla_pcg_mixed(const sla_sell_t *A, int precond, const void *dinv,
                  int b_dtype, const void *b, double *x, int x_is_guess,
                  double atol, double rtol, int64_t maxiter, void *workspace,
                  size_t workspace_bytes, sla_solve_info_t *info,
                  double *pap_out, sla_stream_t stream);

/* Jacobi-PBiCGStab with torch-sla's half-step / full-step stopping tests and
 * 1e-30 breakdown guards (pbicgstab_solve, pytorch_backend.py:1508-1596). */
int sla_bicgstab_workspace(int dtype, int64_t n, size_t *bytes);
int sla_bicgstab(int dtype, const sla_sell_t *A, const void *dinv,
                 const void *b, void *x, int x_is_guess, double atol,
                 double rtol, int64_t maxiter, void *workspace,
                 size_t workspace_bytes, sla_solve_info_t *info,
                 sla_stream_t stream);

/* B Jacobi-PCG solves sharing one CSR pattern, values interleaved
 * [nnz][B] (batched_cg_same_pattern, pytorch_backend.py:2575-2638): stops
 * when every ||R_b|| <= max(atol, rtol*||b_b||). b and x are [B][n]. */
int sla_batched_values(int dtype, const void *val_batch, int64_t batch,
                       int64_t nnz_coo, const int64_t *src_index,
                       const int32_t *seg_ptr, int64_t nnz_csr, void *out,
                       sla_stream_t stream);
/* The same values placed in the order of a diagonal-offset view of the
 * pattern: out ([n_out][B], zero-filled first) receives member b's value of
 * CSR entry e at (pos[e] * B + b); pos from sla_sell_diag_positions. */
int sla_batched_values_at(int dtype, const void *val_batch, int64_t batch,
                          int64_t nnz_coo, const int64_t *src_index,
                          const int32_t *seg_ptr, int64_t nnz_csr,
                          const int64_t *pos, int64_t n_out, void *out,
                          sla_stream_t stream);
int sla_batched_cg_workspace(int dtype, int64_t n, int64_t batch,
                             size_t *bytes);
int sla_batched_cg(int dtype, const int32_t *rowptr, const int32_t *colind,
                   const void *vals_interleaved, int64_t n, int64_t batch,
                   const void *b, void *x, double atol, double rtol,
                   int64_t maxiter, void *workspace, size_t workspace_bytes,
                   sla_solve_info_t *info, sla_stream_t stream);
/* The same solve on a diagonal-offset view of the pattern (5, 7 or 27
 * diagonals, square, no row ids; the view's own values are not used) with
 * values in that view's order (sla_batched_values_at): no column or
 * row-pointer loads in the SpMV. */
int sla_batched_cg_diag(int dtype, const sla_sell_t *A, const void *vals_diag,
                        int64_t batch, const void *b, void *x, double atol,
                        double rtol, int64_t maxiter, void *workspace,
                        size_t workspace_bytes, sla_solve_info_t *info,
                        sla_stream_t stream);

/* CG on K right-hand sides of one CSR matrix (batched_pcg_solve,
 * pytorch_backend.py:2352-2504; pytorch_solve with a 2-D b). b and x are
 * [n][K] row-major (x holds the guess when x_is_guess != 0); dinv [n] or
 * NULL. Convergence is tested every `check_every` iterations (50 in
 * torch-sla); iters_out / converged_out (host, K entries, may be NULL)
 * receive the per-column iteration counts and flags. */
int sla_multi_rhs_cg_workspace(int dtype, int64_t n, int64_t k, size_t *bytes);
int sla_multi_rhs_cg(int dtype, const int32_t *rowptr, const int32_t *colind,
                     const void *vals, int64_t n, int64_t k, const void *dinv,
                     const void *b, void *x, int x_is_guess, double atol,
                     double rtol, int64_t maxiter, int64_t check_every,
                     int64_t *iters_out, int32_t *converged_out,
                     void *workspace, size_t workspace_bytes,
                     sla_solve_info_t *info, sla_stream_t stream);
/* The same solve with the matrix given as a diagonal-offset SELL view
 * (n_diags 5, 7 or 27, square, no row ids): no column or row-pointer loads
 * in the SpMV. Same results as sla_multi_rhs_cg on the same matrix up to
 * the sign of zero sums. Views with offsets (-a,-b,-1,0,1,b,a) or
 * (-b,-1,0,1,b) and K a multiple of 16 bytes' worth of values stage each
 * tile of P in shared memory with bulk copies; a copy that never completes
 * within the bounded wait stops the solve with SLA_ERR_TIMEOUT (info->reason
 * 4). */
int sla_multi_rhs_cg_diag(int dtype, const sla_sell_t *A, int64_t k,
                          const void *dinv, const void *b, void *x,
                          int x_is_guess, double atol, double rtol,
                          int64_t maxiter, int64_t check_every,
                          int64_t *iters_out, int32_t *converged_out,
                          void *workspace, size_t workspace_bytes,
                          sla_solve_info_t *info, sla_stream_t stream);

/* -------------------------------------------------- row-sharded (NCCL) */
/* Opaque NCCL communicator management (one process per GPU). */
int sla_comm_unique_id(unsigned char id[128]);
int sla_comm_init(void **comm, int nranks, const unsigned char id[128],
                  int rank);
int sla_comm_destroy(void *comm);

/* Halo plan of one rank (partition.py:317-423 send/recv maps). Local vector
 * layout is [owned | halo]; neighbours ascend by rank id. */
typedef struct {
  int32_t n_neighbors;
  const int32_t *neighbor_rank;  /* host [n_neighbors]                        */
  const int64_t *send_offset;    /* host [n_neighbors + 1] into send_index    */
  const int64_t *recv_offset;    /* host [n_neighbors + 1] into the recv buf  */
  const int32_t *send_index;     /* device: owned local rows to send          */
  const int32_t *halo_src;       /* device [n_halo]: recv-buffer position of
                                    halo slot h, or NULL when identity        */
  int64_t n_owned;
  int64_t n_halo;
} sla_halo_plan_t;

/* halo_exchange (distributed/matvec.py:26-93): fills x_local[n_owned:]. */
int sla_halo_exchange(void *comm, const sla_halo_plan_t *plan, int dtype,
                      void *x_local, void *sendbuf, void *recvbuf,
                      sla_stream_t stream);
/* shard_matvec (distributed/matvec.py:235-303): y_owned = A_local x_local,
 * halo exchange overlapped with the interior rows. x_local has n_owned +
 * n_halo entries; its halo part is overwritten. */
int sla_shard_spmv(void *comm, const sla_halo_plan_t *plan, int dtype,
                   const sla_sell_t *A_interior, const sla_sell_t *A_boundary,
                   void *x_local, void *y_owned, void *sendbuf, void *recvbuf,
                   sla_stream_t stream);
/* reverse_halo_exchange (distributed/matvec.py:96-170): the halo slots of
 * w_local are sent to their owners, which add them onto the owned slots they
 * sent in the forward exchange, neighbour by neighbour in ascending order.
 * sendbuf holds n_halo values, recvbuf the plan's total send count. */
int sla_reverse_halo_exchange(void *comm, const sla_halo_plan_t *plan,
                              int dtype, void *w_local, void *sendbuf,
                              void *recvbuf, sla_stream_t stream);
/* shard_rmatvec (distributed/matvec.py:306-348): w_local = A_local^T y over
 * AT, the SELL view of the local transpose (rows: the n_owned + n_halo local
 * ids; columns: owned), then the reverse halo exchange. The owned part of
 * w_local is the owned slice of A^T y. */
int sla_shard_rmatvec(void *comm, const sla_halo_plan_t *plan, int dtype,
                      const sla_sell_t *AT, const void *y_owned, void *w_local,
                      void *sendbuf, void *recvbuf, sla_stream_t stream);
/* cg_shard / bicgstab_shard (distributed/solve.py:279-436): stopping test
 * every `check_every` iterations, one fused allreduce per reduction point. */
int sla_shard_krylov_workspace(int dtype, int64_t n_owned, int64_t n_halo,
                               int64_t n_send, size_t *bytes);
int sla_shard_cg(void *comm_halo, void *comm_reduce,
                 const sla_halo_plan_t *plan, int dtype,
                 const sla_sell_t *A_interior, const sla_sell_t *A_boundary,
                 const void *dinv, const void *b, void *x, double atol,
                 double rtol, int64_t maxiter, int64_t check_every,
                 void *workspace, size_t workspace_bytes,
                 sla_solve_info_t *info, sla_stream_t stream);
int sla_shard_bicgstab(void *comm_halo, void *comm_reduce,
                       const sla_halo_plan_t *plan, int dtype,
                       const sla_sell_t *A_interior,
                       const sla_sell_t *A_boundary, const void *dinv,
                       const void *b, void *x, double atol, double rtol,
                       int64_t maxiter, int64_t check_every, void *workspace,
                       size_t workspace_bytes, sla_solve_info_t *info,
                       sla_stream_t stream);

/* Peer-memory shard CG (single node, 1..8 ranks; the same algorithm and
 * stopping rule as sla_shard_cg, distributed/solve.py:279-350). Halo values
 * and dot products are stored by the solver kernels directly into the other
 * GPUs' memory through CUDA IPC mappings, so an iteration is two kernel
 * launches and no NCCL call.
 * sla_p2p_create is collective over `comm` (NCCL is used once to trade the
 * IPC handles and agree): it maps every rank's exchange buffer and returns
 * *p2p_out = NULL with SLA_OK on every rank when any rank cannot (more than
 * 8 ranks, peer mapping refused, a halo permutation in the plan). One rank
 * maps nothing and runs the same kernels, its cross-rank sums covering
 * itself. The handle
 * owns its device buffer; sla_p2p_destroy is collective (it waits until
 * every rank is past its last remote store). Every cross-GPU wait inside the
 * kernels is bounded; a peer that stops answering ends the solve with
 * SLA_ERR_TIMEOUT. The ranks must call the solver the same number of times
 * with the same arguments, as with sla_shard_cg. */
int sla_p2p_create(void *comm, const sla_halo_plan_t *plan, int dtype, void **p2p_out);
int sla_p2p_destroy(void *p2p);
/* Instrumentation of the peer-memory CG (no counterpart in torch-sla): while
 * profiling is on (sla_profile_enable), the solver kernels add GPU-timer
 * nanoseconds into per-plan slots, copied to out[0..n_out) (zeros past the
 * 7 slots) and cleared when reset != 0: 0 halo send (K_P, summed over
 * blocks), 1 halo-arrival wait (K_A, summed over blocks), 2 cross-rank
 * (p,Ap) sum (K_A last block), 3 cross-rank (r,r),(r,z) sum (K_B last
 * block), 4 K_A blocks summed over launches, 5 K_A launches, 6 K_P blocks
 * summed over launches. Synchronises the device. */
int sla_p2p_profile_read(void *p2p, int reset, unsigned long long *out, int n_out);
int sla_shard_cg_p2p(void *p2p, const sla_halo_plan_t *plan, int dtype,
                     const sla_sell_t *A_interior, const sla_sell_t *A_boundary,
                     const void *dinv, const void *b, void *x, double atol,
                     double rtol, int64_t maxiter, int64_t check_every,
                     void *workspace, size_t workspace_bytes,
                     sla_solve_info_t *info, sla_stream_t stream);
/* Peer-memory twin of sla_shard_bicgstab (distributed/solve.py:356-436,
 * including the reference's reuse of the SpMV output buffer): three kernel
 * launches and three cross-rank sums per iteration, no NCCL call. */
int sla_shard_bicgstab_p2p(void *p2p, const sla_halo_plan_t *plan, int dtype,
                           const sla_sell_t *A_interior,
                           const sla_sell_t *A_boundary, const void *dinv,
                           const void *b, void *x, double atol, double rtol,
                           int64_t maxiter, int64_t check_every, void *workspace,
                           size_t workspace_bytes, sla_solve_info_t *info,
                           sla_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SLA_B200_H */
