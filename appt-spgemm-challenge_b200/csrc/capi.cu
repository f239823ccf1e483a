// C-linkage exports declared in include/appt_spgemm.h.
#include <cstring>
#include "../../include/appt_spgemm.h"
#include "engine.h"

using appt::CallOptions;
using appt::CallStats;
using appt::MatOut;
using appt::MatView;

namespace {

MatView view_of(const appt_csr* a) {
  MatView v;
  v.rows = a->rows;
  v.cols = a->cols;
  v.nnz = a->nnz;
  v.rp = a->row_ptr;
  v.ci = a->col_idx;
  v.val = a->val;
  return v;
}

CallOptions opts_of(const appt_options* o) {
  CallOptions c;
  if (o) {
    c.op = o->op;
    c.method = o->method;
    c.in_mem = o->in_mem;
    c.out_mem = o->out_mem;
    c.row_base = o->row_base;
    c.stream = o->stream;
    c.device = o->device;
    c.timing = o->timing;
    c.b_mem = o->b_mem;
  }
  return c;
}

// The public appt_csr_out mirrors MatOut's first fields; the owning details travel in a small
// heap record behind `opaque`.
struct OutRecord {
  MatOut m;
};

void export_out(const MatOut& m, appt_csr_out* C) {
  C->rows = m.rows;
  C->cols = m.cols;
  C->nnz = m.nnz;
  C->row_ptr = reinterpret_cast<int64_t*>(m.rp);
  C->col_idx = m.ci;
  C->val = m.val;
  C->mem = m.mem ? APPT_MEM_DEVICE : APPT_MEM_HOST;
  C->device = m.device;
  C->opaque = new OutRecord{m};
}

}  // namespace

static void export_stats(const CallStats& st, appt_stats* stats) {
  if (!stats) return;
  std::memset(stats, 0, sizeof(*stats));
  stats->products = st.products;
  stats->c_nnz = st.c_nnz;
  for (int i = 0; i < APPT_NUM_BINS; ++i) stats->bin_rows[i] = st.bin_rows[i];
  stats->ms_total = st.ms_total;
  for (int i = 0; i < 8; ++i) stats->ms_phase[i] = st.ms_phase[i];
  stats->kernel_launches = st.launches;
  stats->method_used = st.method_used;
}


extern "C" {

bool g_use_mempool = false;
bool g_use_dev_pool = false;

static void sync_pool_flags() {
  appt::g_mempool_on = g_use_mempool;
  appt::g_devpool_on = g_use_dev_pool;
}

void spgemm_self_product_adaptive(void* A_buffer, int A_rows, int A_cols, int A_nnz,
                                  void** C_buffer_out, int* C_rows, int* C_cols, int* C_nnz) {
  sync_pool_flags();
  appt::compat_call(A_buffer, A_rows, A_cols, A_nnz, C_buffer_out, C_rows, C_cols, C_nnz,
                    appt::kOpAB, 0, "adapt-prof", false);
}
void spgemm_self_product_hash(void* A_buffer, int A_rows, int A_cols, int A_nnz,
                              void** C_buffer_out, int* C_rows, int* C_cols, int* C_nnz) {
  sync_pool_flags();
  appt::compat_call(A_buffer, A_rows, A_cols, A_nnz, C_buffer_out, C_rows, C_cols, C_nnz,
                    appt::kOpAB, 1, "hash-prof", false);
}
void spgemm_self_product_merge3(void* A_buffer, int A_rows, int A_cols, int A_nnz,
                                void** C_buffer_out, int* C_rows, int* C_cols, int* C_nnz) {
  sync_pool_flags();
  appt::compat_call(A_buffer, A_rows, A_cols, A_nnz, C_buffer_out, C_rows, C_cols, C_nnz,
                    appt::kOpAB, 2, "mrg3-prof", false);
}
void spgemm_self_product_manual(void* A_buffer, int A_rows, int A_cols, int A_nnz,
                                void** C_buffer_out, int* C_rows, int* C_cols, int* C_nnz) {
  sync_pool_flags();
  appt::compat_call(A_buffer, A_rows, A_cols, A_nnz, C_buffer_out, C_rows, C_cols, C_nnz,
                    appt::kOpAB, 3, "esc-prof", false);
}
void spgemm_att_hash(void* A_buffer, int A_rows, int A_cols, int A_nnz, void** C_buffer_out,
                     int* C_rows, int* C_cols, int* C_nnz) {
  sync_pool_flags();
  appt::compat_call(A_buffer, A_rows, A_cols, A_nnz, C_buffer_out, C_rows, C_cols, C_nnz,
                    appt::kOpAATUpper, 1, "atth-prof", true);
}
void spgemm_att_merge3(void* A_buffer, int A_rows, int A_cols, int A_nnz, void** C_buffer_out,
                       int* C_rows, int* C_cols, int* C_nnz) {
  sync_pool_flags();
  appt::compat_call(A_buffer, A_rows, A_cols, A_nnz, C_buffer_out, C_rows, C_cols, C_nnz,
                    appt::kOpAATUpper, 2, "attm-prof", true);
}
void spgemm_att_adaptive(void* A_buffer, int A_rows, int A_cols, int A_nnz, void** C_buffer_out,
                         int* C_rows, int* C_cols, int* C_nnz) {
  sync_pool_flags();
  appt::compat_call(A_buffer, A_rows, A_cols, A_nnz, C_buffer_out, C_rows, C_cols, C_nnz,
                    appt::kOpAATUpper, 0, "atta-prof", true);
}
void spgemm_transpose_product(void* A_buffer, int A_rows, int A_cols, int A_nnz,
                              void** C_buffer_out, int* C_rows, int* C_cols, int* C_nnz) {
  sync_pool_flags();
  appt::compat_call(A_buffer, A_rows, A_cols, A_nnz, C_buffer_out, C_rows, C_cols, C_nnz,
                    appt::kOpAAT, 0, "aat-prof", false);
}

void build_csc(const int* d_row_ptr, const int* d_col_idx, const double* d_val, int A_rows,
               int A_nnz, int** col_ptr_out, int** row_idx_out, double** val_out) {
  appt::compat_build_csc(d_row_ptr, d_col_idx, d_val, A_rows, A_nnz, col_ptr_out, row_idx_out,
                         val_out);
}

bool should_run_method(const char* key) { return appt::compat_should_run_method(key); }

bool mempool_init(size_t cap_bytes) {
  sync_pool_flags();
  return appt::pool_init(cap_bytes);
}
void mempool_destroy(void) { appt::pool_destroy(); }
int pinned_d2h_alloc(void** out, size_t bytes) {
  sync_pool_flags();
  return appt::pinned_alloc_reset(out, bytes);
}
void pinned_free(void* p) {
  sync_pool_flags();
  appt::pinned_release(p);
}
void host_free(void* p) {
  sync_pool_flags();
  appt::host_release(p);
}
void dev_pool_reset(void) {
  sync_pool_flags();
  appt::devarena_reset();
}
void* dev_alloc(size_t bytes) {
  sync_pool_flags();
  return appt::devarena_alloc(bytes);
}
void dev_free(void* p) {
  sync_pool_flags();
  appt::devarena_free(p);
}
size_t mempool_cap(void) { return appt::host_arena_cap(); }
size_t mempool_used(void) { return appt::host_arena_used(); }
size_t dev_pool_used(void) { return appt::devarena_used(); }

void appt_default_options(appt_options* opt) {
  if (!opt) return;
  std::memset(opt, 0, sizeof(*opt));
  opt->op = APPT_OP_AB;
  opt->method = APPT_METHOD_ADAPTIVE;
  opt->in_mem = APPT_MEM_HOST;
  opt->out_mem = APPT_MEM_HOST;
}

int appt_spgemm(const appt_csr* A, const appt_csr* B, const appt_options* opt, appt_csr_out* C,
                appt_stats* stats) {
  if (!A || !C) {
    appt::set_error("null argument");
    return APPT_ERR_INVALID;
  }
  std::memset(C, 0, sizeof(*C));
  appt_options def;
  appt_default_options(&def);
  const CallOptions o = opts_of(opt ? opt : &def);
  MatView a = view_of(A);
  MatView b;
  if (B) b = view_of(B);
  MatOut m;
  CallStats st;
  const int rc = appt::spgemm(a, B ? &b : nullptr, o, &m, &st);
  export_stats(st, stats);
  if (rc != APPT_OK) return rc;
  export_out(m, C);
  return APPT_OK;
}

int appt_comm_spgemm(appt_comm* comm, const appt_csr* A_block, const appt_csr* B,
                     const appt_options* opt, appt_csr_out* C_block, int64_t* block_offsets,
                     appt_stats* stats) {
  if (!comm || !A_block || !C_block || !block_offsets) {
    appt::set_error("null argument");
    return APPT_ERR_INVALID;
  }
  std::memset(C_block, 0, sizeof(*C_block));
  appt_options def;
  appt_default_options(&def);
  const CallOptions o = opts_of(opt ? opt : &def);
  MatView a = view_of(A_block);
  MatView b;
  if (B) b = view_of(B);
  MatOut m;
  CallStats st;
  const int rc = appt::comm_spgemm(comm->c, a, B ? &b : nullptr, o, &m,
                                   reinterpret_cast<long long*>(block_offsets), &st);
  export_stats(st, stats);
  if (rc != APPT_OK) return rc;
  export_out(m, C_block);
  return APPT_OK;
}

int appt_free_out(appt_csr_out* C) {
  if (!C) return APPT_ERR_INVALID;
  if (C->opaque) {
    OutRecord* r = static_cast<OutRecord*>(C->opaque);
    appt::free_out(&r->m);
    delete r;
  }
  std::memset(C, 0, sizeof(*C));
  return APPT_OK;
}

int appt_transpose(const appt_csr* A, const appt_options* opt, appt_csr_out* AT) {
  if (!A || !AT) return APPT_ERR_INVALID;
  std::memset(AT, 0, sizeof(*AT));
  appt_options def;
  appt_default_options(&def);
  MatOut m;
  const int rc = appt::transpose(view_of(A), opts_of(opt ? opt : &def), &m);
  if (rc != APPT_OK) return rc;
  export_out(m, AT);
  return APPT_OK;
}

int appt_transpose_into(const appt_csr* A, const appt_options* opt, int32_t* t_row_ptr,
                        int32_t* t_col_idx, double* t_val) {
  if (!A) return APPT_ERR_INVALID;
  appt_options def;
  appt_default_options(&def);
  return appt::transpose_into(view_of(A), opts_of(opt ? opt : &def), t_row_ptr, t_col_idx, t_val);
}

int appt_row_products(const appt_csr* A, const appt_csr* B, const appt_options* opt,
                      int64_t* out) {
  if (!A || !out) return APPT_ERR_INVALID;
  appt_options def;
  appt_default_options(&def);
  MatView b;
  if (B) b = view_of(B);
  return appt::row_products(view_of(A), B ? &b : nullptr, opts_of(opt ? opt : &def),
                            reinterpret_cast<long long*>(out));
}

int appt_estimate_row_nnz(const appt_csr* A, int32_t att, const appt_options* opt,
                          int32_t* out) {
  if (!A || !out) return APPT_ERR_INVALID;
  appt_options def;
  appt_default_options(&def);
  return appt::estimate_row_nnz(view_of(A), att, 0, opts_of(opt ? opt : &def), out);
}

int appt_estimate_row_nnz_with(const appt_csr* A, int32_t att, int32_t estimator,
                               const appt_options* opt, int32_t* out) {
  if (!A || !out) return APPT_ERR_INVALID;
  appt_options def;
  appt_default_options(&def);
  return appt::estimate_row_nnz(view_of(A), att, estimator, opts_of(opt ? opt : &def), out);
}

double appt_reference_score(const int32_t* row_ptr, int64_t rows, int64_t nnz) {
  if (!row_ptr) return 0.0;
  return appt::reference_score(row_ptr, rows, nnz);
}

const char* appt_last_error(void) { return appt::last_error(); }
int appt_device_count(void) { return appt::device_count(); }
int appt_release_cached(int device) { return appt::release_cached(device); }
int64_t appt_kernel_launches(void) { return appt::kernel_launches(); }
const char* appt_version(void) { return "appt-spgemm-b200 0.1 (sm_100a)"; }

}  // extern "C"
