/*
 * appt_spgemm.h -- C ABI of the B200 adaptive SpGEMM engine (libappt_spgemm.so).
 *
 * Two layers are exported with C linkage (plain pointers and sizes, no C++ or torch types):
 *
 *  1. Reference-compatible entry points. Same names, argument order, argument meaning and
 *     error convention as the reference's include/spgemm.h and include/mempool.h
 *     (XUE77565/APPT-Spgemm-Challenge). A caller that bound the reference through an FFI
 *     (ctypes, cgo, JNI, N-API) binds these. The same functions are also exported with C++
 *     linkage (mangled names) so the reference's own driver src/main.cu links against this
 *     library unchanged.
 *
 *  2. Native entry points (appt_*): int64 sizes, explicit status codes, device- or host-resident
 *     operands, CUDA stream, optional per-phase statistics.
 *
 * Matrices are CSR with int32 row_ptr/col_idx and fp64 values, columns sorted ascending in every
 * row (the reference's layout). Results keep structural zeros (a column reached by a product is
 * stored even if its sum is exactly 0), matching every reference method.
 */
#ifndef APPT_SPGEMM_H
#define APPT_SPGEMM_H

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------
 * Layer 1: reference-compatible entry points.
 *
 * A_buffer is a host buffer [row_ptr (A_rows+1) int32 | col_idx (A_nnz) int32 |
 * pad to 8 | val (A_nnz) fp64] with col_idx starting right after row_ptr (the reference's
 * read_matrix_market layout, src/matrix_utils.cu:142-145).
 * On success *C_buffer_out is a host buffer [row_ptr (C_rows+1) int32 | pad to 8 |
 * col_idx (C_nnz) int32 | pad to 8 | val (C_nnz) fp64] (src/main.cu:185-193) allocated with
 * pinned_d2h_alloc; release it with pinned_free.
 * On failure *C_nnz = -1 and *C_buffer_out = NULL (spgemm_kernel_hash.cu:1009,1038). Unlike
 * the reference, CUDA errors do not exit the process; the message is in appt_last_error().
 * C_nnz is also -1 when nnz(C) does not fit in int32 (use appt_spgemm for such products).
 * ---------------------------------------------------------------------------------------- */

/* C = A*A, adaptive per-bin tiers. Replaces spgemm_self_product_adaptive (spgemm.h:104-106,
 * src/spgemm_adaptive.cu:49-100). */
void spgemm_self_product_adaptive(void *A_buffer, int A_rows, int A_cols, int A_nnz,
                                  void **C_buffer_out, int *C_rows, int *C_cols, int *C_nnz);
/* C = A*A, hash tiers (window tier for rows beyond shared memory, so it never overflows).
 * Replaces spgemm_self_product_hash (spgemm.h:99-100, src/spgemm_kernel_hash.cu:1111-1114). */
void spgemm_self_product_hash(void *A_buffer, int A_rows, int A_cols, int A_nnz,
                              void **C_buffer_out, int *C_rows, int *C_cols, int *C_nnz);
/* C = A*A, k-way merge tier. Replaces spgemm_self_product_merge3 (spgemm.h:93-94,
 * src/spgemm_merge.cu:935-938). */
void spgemm_self_product_merge3(void *A_buffer, int A_rows, int A_cols, int A_nnz,
                                void **C_buffer_out, int *C_rows, int *C_cols, int *C_nnz);
/* C = A*A, expand-sort-compress baseline. Replaces spgemm_self_product_manual (spgemm.h:78-79,
 * src/spgemm_kernel_manual.cu:272-437). */
void spgemm_self_product_manual(void *A_buffer, int A_rows, int A_cols, int A_nnz,
                                void **C_buffer_out, int *C_rows, int *C_cols, int *C_nnz);
/* Upper triangle (j >= i) of A*A^T. Replace spgemm_att_hash / spgemm_att_merge3 /
 * spgemm_att_adaptive (spgemm.h:62-73). As in the reference, *C_cols is reported as A_cols
 * (src/spgemm_kernel_hash.cu:1103); the true column count is A_rows. */
void spgemm_att_hash(void *A_buffer, int A_rows, int A_cols, int A_nnz, void **C_buffer_out,
                     int *C_rows, int *C_cols, int *C_nnz);
void spgemm_att_merge3(void *A_buffer, int A_rows, int A_cols, int A_nnz, void **C_buffer_out,
                       int *C_rows, int *C_cols, int *C_nnz);
void spgemm_att_adaptive(void *A_buffer, int A_rows, int A_cols, int A_nnz, void **C_buffer_out,
                         int *C_rows, int *C_cols, int *C_nnz);
/* Full C = A*A^T (C_cols = A_rows). Replaces spgemm_transpose_product (spgemm.h:58-60), which
 * the reference computes with cuSPARSE (src/spgemm_kernel_cusparse.cu:216). */
void spgemm_transpose_product(void *A_buffer, int A_rows, int A_cols, int A_nnz,
                              void **C_buffer_out, int *C_rows, int *C_cols, int *C_nnz);

/* Device CSR -> CSC of A (= CSR of A^T), rows of the result sorted. Replaces build_csc
 * (spgemm.h:111-115, src/spgemm_kernel_formulations.cu:69-120). Same contract as the
 * reference: the column count is taken to be A_rows; outputs are cudaMalloc'ed and the caller
 * cudaFree's them. Returns nothing, as the reference; on error the outputs are NULL. */
void build_csc(const int *d_row_ptr, const int *d_col_idx, const double *d_val, int A_rows,
               int A_nnz, int **col_ptr_out, int **row_idx_out, double **val_out);

/* Matrix files for the reference's driver: read_matrix_market / write_matrix_market,
 * print_matrix_info and verify_csr_matrices of src/matrix_utils.cu (include/spgemm.h:44-52) are
 * exported with the reference's C++ linkage, so src/main.cu links without matrix_utils.cu. The
 * reader also takes binary CSR files (8-byte magic "APPTCSR1", int64 rows/cols/nnz, int32
 * row_ptr, int32 col_idx, fp64 val) with no parsing, and parses MatrixMarket text in one pass;
 * the buffer layout and allocation (pinned when g_use_mempool, else malloc; release with
 * host_free) are the reference's. These are the same functions with C linkage; a name ending in
 * ".bin" makes the writer produce the binary form. */
bool appt_read_matrix_file(const char *filename, void **buffer_out, int **row_ptr_out,
                           int **col_idx_out, double **val_out, int *rows, int *cols, int *nnz);
bool appt_write_matrix_file(const char *filename, const int *row_ptr, const int *col_idx,
                            const double *val, int rows, int cols, int nnz);

/* METHOD environment gating. Replaces should_run_method (spgemm.h:108,
 * src/spgemm_adaptive.cu:9-20). */
bool should_run_method(const char *key);

/* Pinned host arena and device arena. Replace include/mempool.h:28-76 (src/mempool.cu).
 * g_use_mempool / g_use_dev_pool select the pooled paths (mempool.h:28-30). Differences:
 * an arena that is too small grows instead of exiting, and the device arena is a CUDA
 * stream-ordered memory pool rather than one fixed cudaMalloc. */
extern bool g_use_mempool;
extern bool g_use_dev_pool;
bool mempool_init(size_t cap_bytes);
void mempool_destroy(void);
int pinned_d2h_alloc(void **out, size_t bytes); /* returns a cudaError_t value */
void pinned_free(void *p);
void host_free(void *p);
void dev_pool_reset(void);
void *dev_alloc(size_t bytes);
void dev_free(void *p);
size_t mempool_cap(void);
size_t mempool_used(void);
size_t dev_pool_used(void);

/* ------------------------------------------------------------------------------------------
 * Layer 2: native API.
 * ---------------------------------------------------------------------------------------- */
#define APPT_OK 0
#define APPT_ERR_INVALID (-1)   /* bad argument */
#define APPT_ERR_CUDA (-2)      /* CUDA runtime error */
#define APPT_ERR_OOM (-3)       /* device or host allocation failed */
#define APPT_ERR_DEVICE (-4)    /* a kernel reported an internal capacity/bound error */
#define APPT_ERR_TOO_LARGE (-5) /* result not representable in the requested format */
#define APPT_ERR_NO_DEVICE (-6) /* no CUDA device */

#define APPT_OP_AB 0        /* C = A * B (B = A when B is NULL) */
#define APPT_OP_AAT 1       /* C = A * A^T, full */
#define APPT_OP_AAT_UPPER 2 /* C = upper triangle (j >= i) of A * A^T */
#define APPT_OP_AB_UPPER 3  /* C = entries j >= i + row_base of A * B (row blocks of A*A^T when
                               B = A^T is passed explicitly, e.g. one shard per GPU) */

#define APPT_METHOD_ADAPTIVE 0
#define APPT_METHOD_HASH 1
#define APPT_METHOD_MERGE 2
#define APPT_METHOD_ESC 3

#define APPT_MEM_HOST 0
#define APPT_MEM_DEVICE 1

typedef struct appt_csr {
  int64_t rows, cols, nnz;
  const int32_t *row_ptr; /* rows + 1 entries, absolute offsets into col_idx / val */
  const int32_t *col_idx;
  const double *val;
} appt_csr;

typedef struct appt_csr_out {
  int64_t rows, cols, nnz;
  int64_t *row_ptr; /* rows + 1 entries, row_ptr[0] = 0 */
  int32_t *col_idx;
  double *val;
  int32_t mem;      /* APPT_MEM_HOST or APPT_MEM_DEVICE */
  int32_t device;
  void *opaque;     /* owning handle; release with appt_free_out */
} appt_csr_out;

#define APPT_NUM_BINS 32
typedef struct appt_stats {
  int64_t products;                 /* intermediate products; flops = 2 * products */
  int64_t c_nnz;
  int64_t bin_rows[APPT_NUM_BINS];  /* rows per numeric tier */
  double ms_total;                  /* device time of the call (CUDA events) when timing != 0 */
  double ms_phase[8];               /* h2d, transpose, analyze, symbolic, scan, numeric, d2h, other */
  int64_t kernel_launches;          /* kernels this call launched */
  int32_t method_used;
  int32_t pad;
} appt_stats;

typedef struct appt_options {
  int32_t op;       /* APPT_OP_* */
  int32_t method;   /* APPT_METHOD_* */
  int32_t in_mem;   /* where A and B live (APPT_MEM_*) */
  int32_t out_mem;  /* where C is returned (APPT_MEM_*) */
  int64_t row_base; /* global index of A's first row (upper-triangle filter on row blocks) */
  void *stream;     /* cudaStream_t; NULL = the library's stream for the device */
  int32_t device;   /* CUDA device ordinal */
  int32_t timing;   /* nonzero: record per-phase CUDA events into stats */
  int32_t b_mem;    /* where B lives: APPT_B_AS_A (0, where in_mem says), APPT_B_HOST or
                       APPT_B_DEVICE -- e.g. a host row block of A against a device-resident B */
  int32_t reserved; /* 0 */
} appt_options;

#define APPT_B_AS_A 0
#define APPT_B_HOST 1
#define APPT_B_DEVICE 2

/* Fill *opt with defaults: AB, adaptive, host in/out, device 0, row_base 0, no timing. */
void appt_default_options(appt_options *opt);

/* C = op(A, B). Operands are read where opt->in_mem says; C is returned where opt->out_mem
 * says and must be released with appt_free_out. stats may be NULL. */
int appt_spgemm(const appt_csr *A, const appt_csr *B, const appt_options *opt, appt_csr_out *C,
                appt_stats *stats);
int appt_free_out(appt_csr_out *C);

/* CSR of A^T (rows sorted), device- or host-resident per in_mem/out_mem of opt. */
int appt_transpose(const appt_csr *A, const appt_options *opt, appt_csr_out *AT);

/* CSR of A^T written into caller-provided buffers in the operand format (int32 row_ptr):
 * t_row_ptr has A->cols + 1 entries, t_col_idx / t_val A->nnz. Buffers are device or host per
 * opt->in_mem (A and the outputs live in the same space). Counterpart of build_csc with an
 * explicit column count and caller-owned outputs. */
int appt_transpose_into(const appt_csr *A, const appt_options *opt, int32_t *t_row_ptr,
                        int32_t *t_col_idx, double *t_val);

/* Intermediate products per row of A*B (B = A when NULL); out has A->rows entries, host. */
int appt_row_products(const appt_csr *A, const appt_csr *B, const appt_options *opt,
                      int64_t *out);

/* The reference's per-row output-size estimate (its hash-path sizing, est array): exact
 * products count when nnz(A) < 100000, else the 128-partition MinHash estimate x1.5 snapped
 * to {<=16} U {32, 64, ..., 16384} -- or, with EST_METHOD=hll in the environment as in the
 * reference (src/spgemm_kernel_hash.cu:862), the HyperLogLog estimate. att != 0 uses B = A^T.
 * out has A->rows entries, host. Replaces the est computation of hash_product
 * (src/spgemm_kernel_hash.cu:855-912). */
int appt_estimate_row_nnz(const appt_csr *A, int32_t att, const appt_options *opt,
                          int32_t *out);

#define APPT_EST_DEFAULT 0   /* the reference's selection (EST_METHOD) */
#define APPT_EST_MINHASH 1   /* mh_construct_kernel / mh_merge_kernel, src/spgemm_kernel_hash.cu:257-369 */
#define APPT_EST_HLL 2       /* hll_construct_kernel / hll_merge_kernel, src/spgemm_kernel_hash.cu:94-240 */
/* appt_estimate_row_nnz with an explicit estimator (APPT_EST_*). */
int appt_estimate_row_nnz_with(const appt_csr *A, int32_t att, int32_t estimator,
                               const appt_options *opt, int32_t *out);

/* The reference dispatcher's score (src/spgemm_adaptive.cu:67-72) for a host row_ptr; the
 * reference picks its hash path when the score is negative. */
double appt_reference_score(const int32_t *row_ptr, int64_t rows, int64_t nnz);

/* C = A * B (B = A when NULL) for device-resident A and B, written into device buffers the
 * caller owns, without allocating any memory: for callers that cannot call cudaMalloc during the
 * multiply (a framework whose allocator owns the device heap, code where allocation is
 * forbidden, loops that pre-size every buffer). No counterpart in the reference.
 * C_row_ptr: A->rows + 1 int64; C_col_idx / C_val: room for C_capacity entries. Fills
 * C_row_ptr and *C_nnz_out; returns APPT_ERR_TOO_LARGE before the numeric phase when nnz(C) >
 * C_capacity (size the buffers and call again). Temporaries live in one fixed 64 MiB device
 * array owned by the library (present on every GPU that loads it, until exit), which limits A
 * to about 2.2 million rows (larger A: APPT_ERR_TOO_LARGE with a message). The first call on a
 * device resolves that array's address. Calls share the array; this function serialises them per device and waits for its own GPU work: every call
 * blocks its host thread (nnz(C) is read back mid-call and the stream is synchronised before it
 * returns). */
int appt_spgemm_noalloc(const appt_csr *A, const appt_csr *B, int64_t *C_row_ptr,
                        int32_t *C_col_idx, double *C_val, int64_t C_capacity,
                        int64_t *C_nnz_out, void *stream);

/* ------------------------------------------------------------------------------------------
 * Multi-GPU: one process per GPU, rows of A sharded across the ranks, B replicated.
 *
 * The reference runs on one GPU (src/main.cu:44 selects device 0); these entry points are the
 * row-sharded scaling of appt_spgemm. Rows of C are independent: each rank computes a contiguous
 * block of rows (balanced by intermediate products) against a B that every rank holds. NCCL over
 * NVLink carries only the replication of B and, per product, an all-gather of the ranks'
 * nnz(C block) that gives every block its offset in the global C; C stays sharded. NCCL is
 * loaded at run time (libnccl.so.2) by the first of these calls; waits on the other ranks are
 * bounded by APPT_COMM_TIMEOUT_S seconds (default 300), after which the communicator is aborted
 * and the call fails. Calls marked "collective" must be made by every rank, in the same order.
 * ---------------------------------------------------------------------------------------- */
#define APPT_COMM_ID_BYTES 128
typedef struct appt_comm appt_comm;

/* A fresh communicator id (APPT_COMM_ID_BYTES bytes, an NCCL unique id). One rank creates it and
 * sends the bytes to the others over any host channel. */
int appt_comm_unique_id(void *id);
/* Joins the nranks-rank communicator named by id as `rank`, using CUDA device `device`.
 * Collective. */
int appt_comm_init(const void *id, int nranks, int rank, int device, appt_comm **out);
int appt_comm_destroy(appt_comm *comm);
/* Replicates a device-resident CSR from `root` to every rank: on the root M is read; on the other
 * ranks the library allocates device arrays, fills them and stores them (and the sizes) in *M --
 * release those with appt_comm_free_csr. *ms (may be NULL) receives the transfer's device time
 * on this rank. Collective. */
int appt_comm_broadcast_csr(appt_comm *comm, int root, appt_csr *M, double *ms);
int appt_comm_free_csr(appt_comm *comm, appt_csr *M);
/* Contiguous row bounds bounds[0 .. parts] (bounds[0] = 0, bounds[parts] = rows) that split the
 * per-row intermediate products as evenly as contiguous blocks allow (each cut at the prefix
 * nearest to r/parts of the total). Host only. */
int appt_split_rows(const int64_t *row_products, int64_t rows, int parts, int64_t *bounds);
/* The row split of C = A * B (B = A when NULL; both device-resident on `root`, may be NULL
 * elsewhere) over the communicator's ranks: products counted on the root's GPU, bounds
 * (nranks + 1 entries) broadcast to every rank. Collective. */
int appt_comm_row_split(appt_comm *comm, int root, const appt_csr *A, const appt_csr *B,
                        int64_t *bounds);
/* This rank's block of C = op(A, B): A_block holds rows [opt->row_base, opt->row_base +
 * A_block->rows) of A (where opt->in_mem says), B the whole of B (opt->b_mem may place it on the
 * device while A_block is on the host). The C block is returned as by appt_spgemm;
 * block_offsets[0 .. nranks] receives every rank's first entry in the global C (the last is
 * nnz(C)). The nnz all-gather is posted as soon as this rank's nnz is known and overlaps its
 * numeric phase. A rank whose call fails still takes part (and the others then fail with
 * APPT_ERR_DEVICE). Collective. */
int appt_comm_spgemm(appt_comm *comm, const appt_csr *A_block, const appt_csr *B,
                     const appt_options *opt, appt_csr_out *C_block, int64_t *block_offsets,
                     appt_stats *stats);

const char *appt_last_error(void);
int appt_device_count(void);
/* Device memory that the library keeps cached for later calls (freed temporaries and released
 * results stay in its stream-ordered pools) is returned to the driver. Waits for the device's
 * library stream first. */
int appt_release_cached(int device);
int64_t appt_kernel_launches(void); /* kernels launched by this process so far */
const char *appt_version(void);

#ifdef __cplusplus
}
#endif

#endif /* APPT_SPGEMM_H */
