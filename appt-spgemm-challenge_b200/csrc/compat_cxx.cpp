// C++-linkage definitions of the reference's include/spgemm.h and include/mempool.h entry
// points, so that the reference's unmodified driver (src/main.cu, compiled with its own
// headers) links against libappt_spgemm.so in place of the reference's kernel objects.
//
// Mapping of the reference functions (spgemm.h:51-125) onto this engine:
//   spgemm_self_product_adaptive / _hash / _merge3 / _manual -> adaptive / hash / merge / ESC
//   spgemm_att_adaptive / _hash / _merge3                   -> upper(A*A^T), C_cols = A_cols
//   spgemm_transpose_product (cuSPARSE in the reference)      -> full A*A^T, adaptive
//   spgemm_transpose_product_manual (all-pairs in the ref.)   -> full A*A^T, ESC
//   spgemm_self_product (cuSPARSE in the reference)           -> A*A, adaptive
//   spgemm_self_product_merge / _merge2 (serial/warp merges)  -> A*A, merge
//   spgemm_self_product_outer / _colwise / _inner (ESC forms) -> A*A, ESC
// The cuSPARSE, all-pairs and formulation variants are outside this engine's scope; they are
// provided only so that the driver links, and return the same C as the mapped method.
#include <cuda_runtime_api.h>
#include <cstddef>
#include "engine.h"

extern bool g_use_mempool;    // defined in capi.cu (global variables are not name-mangled)
extern bool g_use_dev_pool;

namespace {
inline void flags() {
  appt::g_mempool_on = g_use_mempool;
  appt::g_devpool_on = g_use_dev_pool;
}
inline void call(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc, int* Cn, int op,
                 int method, const char* tag, bool quirk) {
  flags();
  appt::compat_call(A, r, c, n, Co, Cr, Cc, Cn, op, method, tag, quirk);
}
}  // namespace

void spgemm_self_product(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc, int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 0, "cu-prof", false);
}
void spgemm_transpose_product(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                              int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAAT, 0, "aat-prof", false);
}
void spgemm_att_hash(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc, int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAATUpper, 1, "atth-prof", true);
}
void spgemm_att_merge3(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc, int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAATUpper, 2, "attm-prof", true);
}
void spgemm_att_adaptive(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc, int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAATUpper, 0, "atta-prof", true);
}
void spgemm_transpose_product_manual(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                                     int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAAT, 3, "aat-esc-prof", false);
}
void spgemm_self_product_manual(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                                int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 3, "esc-prof", false);
}
void spgemm_self_product_merge(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                               int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 2, "merge-prof", false);
}
void spgemm_self_product_merge2(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                                int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 2, "mrg2-prof", false);
}
void spgemm_self_product_merge3(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                                int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 2, "mrg3-prof", false);
}
void spgemm_self_product_hash(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                              int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 1, "hash-prof", false);
}
void spgemm_self_product_adaptive(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                                  int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 0, "adapt-prof", false);
}
void spgemm_self_product_outer(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                               int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 3, "outer-prof", false);
}
void spgemm_self_product_colwise(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                                 int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 3, "colwise-prof", false);
}
void spgemm_self_product_inner(void* A, int r, int c, int n, void** Co, int* Cr, int* Cc,
                               int* Cn) {
  call(A, r, c, n, Co, Cr, Cc, Cn, appt::kOpAB, 3, "inner-prof", false);
}
bool should_run_method(const char* key) { return appt::compat_should_run_method(key); }
void build_csc(const int* rp, const int* ci, const double* v, int rows, int nnz, int** cp,
               int** ri, double** vo) {
  appt::compat_build_csc(rp, ci, v, rows, nnz, cp, ri, vo);
}

bool mempool_init(size_t cap_bytes) {
  flags();
  return appt::pool_init(cap_bytes);
}
void mempool_destroy() { appt::pool_destroy(); }
cudaError_t pinned_d2h_alloc(void** out, size_t bytes) {
  flags();
  return (cudaError_t)appt::pinned_alloc_reset(out, bytes);
}
void pinned_free(void* p) {
  flags();
  appt::pinned_release(p);
}
void host_free(void* p) {
  flags();
  appt::host_release(p);
}
void dev_pool_reset() {
  flags();
  appt::devarena_reset();
}
void* dev_alloc(size_t bytes) {
  flags();
  return appt::devarena_alloc(bytes);
}
void dev_free(void* p) {
  flags();
  appt::devarena_free(p);
}
size_t mempool_cap() { return appt::host_arena_cap(); }
size_t mempool_used() { return appt::host_arena_used(); }
size_t dev_pool_used() { return appt::devarena_used(); }
