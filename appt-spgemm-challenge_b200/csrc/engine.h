// Internal C++ interface of the engine (host side). The C ABI (capi.cu) and the C++-linkage
// spgemm.h compatibility layer (compat_cxx.cpp) are thin wrappers over these functions.
#pragma once
#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>

namespace appt {

// Status codes (same values as the APPT_* macros of include/appt_spgemm.h).
enum Status : int {
  kOk = 0,
  kErrInvalid = -1,
  kErrCuda = -2,
  kErrOom = -3,
  kErrDevice = -4,
  kErrTooLarge = -5,
  kErrNoDevice = -6,
};

enum Op : int { kOpAB = 0, kOpAAT = 1, kOpAATUpper = 2, kOpABUpper = 3 };

struct MatView {          // CSR operand; pointers are host or device per the call
  long long rows = 0, cols = 0, nnz = 0;
  const int* rp = nullptr;
  const int* ci = nullptr;
  const double* val = nullptr;
};

struct MatOut {           // CSR result with int64 row pointers
  long long rows = 0, cols = 0, nnz = 0;
  long long* rp = nullptr;
  int* ci = nullptr;
  double* val = nullptr;
  int mem = 0;            // 0 host, 1 device
  int device = 0;
  int alloc_kind = 0;     // how the storage was obtained (see engine.cu)
  void* base = nullptr;   // owning pointer
};

struct CallStats {
  long long products = 0;
  long long c_nnz = 0;
  long long bin_rows[32] = {0};
  double ms_total = 0.0;
  double ms_phase[8] = {0};   // h2d, transpose, analyze, symbolic, scan, numeric, d2h, other
  long long launches = 0;
  int method_used = 0;
};

struct CallOptions {
  int op = kOpAB;
  int method = 0;
  int in_mem = 0;
  int out_mem = 0;
  long long row_base = 0;
  void* stream = nullptr;
  int device = 0;
  int timing = 0;
  int b_mem = 0;          // where B lives: 0 as in_mem, 1 host, 2 device
  // called with nnz(C) once it is known, before the numeric phase (multi-GPU nnz exchange)
  const std::function<int(long long)>* on_nnz = nullptr;
  // prefix of the per-phase lines printed when APPT_PROF=1 ("[<tag>] <phase> <ms> ms")
  const char* prof_tag = "appt-prof";
};

// Main entry: C = op(A, B). B may be null (B = A).
int spgemm(const MatView& A, const MatView* B, const CallOptions& opt, MatOut* C,
           CallStats* stats);
int free_out(MatOut* C);
int transpose(const MatView& A, const CallOptions& opt, MatOut* AT);
int transpose_into(const MatView& A, const CallOptions& opt, int* t_rp, int* t_ci, double* t_val);
int row_products(const MatView& A, const MatView* B, const CallOptions& opt, long long* out);
// estimator: 0 = the reference's default selection (EST_METHOD=hll picks HyperLogLog, else
// MinHash), 1 = MinHash, 2 = HyperLogLog
int estimate_row_nnz(const MatView& A, int att, int estimator, const CallOptions& opt, int* out);
double reference_score(const int* row_ptr, long long rows, long long nnz);
// Returns the device's cached pool memory (freed temporaries and results) to the driver.
int release_cached(int device);

// spgemm.h-compatible flow: host buffer in the reference layout in, pinned host buffer in the
// reference's C layout out. `att_quirk_cols` reports C_cols = A_cols as the reference's att_*.
void compat_call(void* A_buffer, int A_rows, int A_cols, int A_nnz, void** C_buffer_out,
                 int* C_rows, int* C_cols, int* C_nnz, int op, int method, const char* tag,
                 bool att_quirk_cols);
void compat_build_csc(const int* d_row_ptr, const int* d_col_idx, const double* d_val, int A_rows,
                      int A_nnz, int** col_ptr_out, int** row_idx_out, double** val_out);
bool compat_should_run_method(const char* key);

// Pools (reference mempool.h semantics).
extern bool g_mempool_on;
extern bool g_devpool_on;
bool pool_init(size_t cap_bytes);
void pool_destroy();
int pinned_alloc_reset(void** out, size_t bytes);   // returns a cudaError_t value
void pinned_release(void* p);
void host_release(void* p);
void devarena_reset();
void* devarena_alloc(size_t bytes);
void devarena_free(void* p);
size_t host_arena_cap();
size_t host_arena_used();
size_t devarena_used();

// Multi-GPU (dist.cu): one communicator per process and GPU, NCCL loaded at run time.
struct Comm;
int comm_unique_id(void* id);
int comm_init(const void* id, int nranks, int rank, int device, Comm** out);
int comm_destroy(Comm* c);
// Replicates a device CSR from `root`; non-root ranks get library-allocated arrays in *M
// (*allocated = true).
int comm_broadcast_csr(Comm* c, int root, MatView* M, bool* allocated, double* ms);
int comm_row_split(Comm* c, int root, const MatView* A, const MatView* B, long long* bounds);
// This rank's block of C; offsets[0 .. nranks] receives the ranks' first global entries.
int comm_spgemm(Comm* c, const MatView& A, const MatView* B, CallOptions opt, MatOut* C,
                long long* offsets, CallStats* st);
// Prefix-balanced contiguous split of rows by their products count (host).
int split_rows(const long long* products, long long rows, int parts, long long* bounds);

void set_error(const std::string& msg);
const char* last_error();
int device_count();
long long kernel_launches();
void note_launches(long long n);

}  // namespace appt

// Opaque communicator handle of the C ABI (include/appt_spgemm.h).
struct appt_comm {
  appt::Comm* c;
};
