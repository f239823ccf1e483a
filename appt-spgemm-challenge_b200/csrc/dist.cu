// Row-sharded multi-GPU SpGEMM: one process per GPU, NCCL over NVLink for the data plane.
//
// The reference is single-GPU (src/main.cu:44 selects device 0). Rows of C are independent, so
// the product scales by giving each rank a contiguous block of A's rows, balanced by their
// intermediate-product count (prefix split), against a B (or A^T) that every GPU holds. NCCL
// carries exactly two things: the replication of B (broadcasts from one root) and, per product,
// an all-gather of each rank's nnz(C block), from which every rank learns where its block
// starts in the global C. C stays sharded. Nothing else crosses GPUs.
//
// The nnz all-gather is posted on the communicator's own stream from inside the pipeline, right
// after the mid-pipeline synchronisation that learns nnz(C block), so it overlaps the numeric
// phase: a rank waits for the exchange only at the end of its call, by which time every other
// rank has normally passed its own mid-point.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2) when the first communicator is created;
// the rest of the library does not depend on it. Every host wait on a collective is bounded
// (APPT_COMM_TIMEOUT_S, default 300 s): on expiry the communicator is aborted, which ends the
// outstanding NCCL kernels, and the call fails.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "../../include/appt_spgemm.h"
#include "engine.h"

namespace appt {
namespace {

// NCCL entry points used here, resolved from the shared library.
struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

bool load_nccl() {
  std::lock_guard<std::mutex> g(g_nccl_mu);
  if (g_nccl.handle) return true;
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  void* h = nullptr;
  for (const char* n : names)
    if ((h = dlopen(n, RTLD_NOW | RTLD_GLOBAL))) break;
  if (!h) {
    set_error(std::string("NCCL not found (dlopen libnccl.so.2): ") + dlerror());
    return false;
  }
  NcclApi a;
  a.handle = h;
  bool ok = true;
  auto sym = [&](auto& fn, const char* name) {
    fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
    if (!fn) ok = false;
  };
  sym(a.get_unique_id, "ncclGetUniqueId");
  sym(a.comm_init_rank, "ncclCommInitRank");
  sym(a.comm_destroy, "ncclCommDestroy");
  sym(a.comm_abort, "ncclCommAbort");
  sym(a.comm_get_async_error, "ncclCommGetAsyncError");
  sym(a.broadcast, "ncclBroadcast");
  sym(a.all_gather, "ncclAllGather");
  sym(a.group_start, "ncclGroupStart");
  sym(a.group_end, "ncclGroupEnd");
  sym(a.error_string, "ncclGetErrorString");
  if (!ok) {
    set_error("libnccl.so.2 lacks an expected entry point");
    dlclose(h);
    return false;
  }
  g_nccl = a;
  return true;
}

int nccl_fail(ncclResult_t r, const char* what) {
  set_error(std::string(what) + ": " + (g_nccl.error_string ? g_nccl.error_string(r) : "NCCL"));
  return kErrCuda;
}

double timeout_s() {
  const char* e = std::getenv("APPT_COMM_TIMEOUT_S");
  const double v = e ? std::atof(e) : 0.0;
  return v > 0.0 ? v : 300.0;
}

}  // namespace

struct Comm {
  ncclComm_t nc = nullptr;
  int nranks = 0, rank = 0, device = 0;
  cudaStream_t s = nullptr;
  cudaEvent_t done = nullptr;
  long long* h_buf = nullptr;   // pinned: [0] value sent, [1 ..] values received / broadcast
  long long* d_buf = nullptr;   // device: same layout
  int cap = 0;                  // int64 slots of h_buf / d_buf
  bool broken = false;
  std::mutex mu;
};

// Host polling of a pending exchange spins (yielding the core) for this long before it falls back
// to 20 us sleeps: a Linux sleep of 20 us returns after 60 us or more, and a rank that wakes late
// starts its next product late, which the other ranks then wait for at their next exchange.
#ifndef APPT_COMM_SPIN_US
#define APPT_COMM_SPIN_US 2000
#endif

// Waits for `done` on the host, polling, for at most timeout_s(); aborts the communicator on
// expiry or on an asynchronous NCCL error (that ends its pending kernels).
static int wait_bounded(Comm* c, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  const double limit = timeout_s();
  for (;;) {
    const cudaError_t e = cudaEventQuery(c->done);
    if (e == cudaSuccess) return kOk;
    if (e != cudaErrorNotReady) {
      set_error(std::string(what) + ": " + cudaGetErrorString(e));
      return kErrCuda;
    }
    ncclResult_t ae = ncclSuccess;
    g_nccl.comm_get_async_error(c->nc, &ae);
    const double el =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if ((ae != ncclSuccess && ae != ncclInProgress) || el > limit) {
      g_nccl.comm_abort(c->nc);
      c->nc = nullptr;
      c->broken = true;
      set_error(std::string(what) + (el > limit ? ": timed out waiting for the other ranks"
                                                : ": NCCL reported an asynchronous error") +
                "; the communicator was aborted");
      return kErrCuda;
    }
    if (el * 1e6 < APPT_COMM_SPIN_US)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

#define CKC(call)                                                                     \
  do {                                                                                \
    cudaError_t e_ = (call);                                                          \
    if (e_ != cudaSuccess) {                                                          \
      set_error(std::string(#call) + ": " + cudaGetErrorString(e_));                  \
      return kErrCuda;                                                                \
    }                                                                                 \
  } while (0)

#define CKN(call, what)                                                               \
  do {                                                                                \
    ncclResult_t r_ = (call);                                                         \
    if (r_ != ncclSuccess) return nccl_fail(r_, what);                                \
  } while (0)

int comm_unique_id(void* id) {
  if (!id) {
    set_error("null id buffer");
    return kErrInvalid;
  }
  if (!load_nccl()) return kErrInvalid;
  ncclUniqueId u;
  CKN(g_nccl.get_unique_id(&u), "ncclGetUniqueId");
  std::memcpy(id, &u, sizeof(u));
  return kOk;
}

int comm_init(const void* id, int nranks, int rank, int device, Comm** out) {
  if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks || device < 0) {
    set_error("appt_comm_init: invalid argument");
    return kErrInvalid;
  }
  *out = nullptr;
  if (!load_nccl()) return kErrInvalid;
  const int n = device_count();
  if (n == 0) {
    set_error("no CUDA device");
    return kErrNoDevice;
  }
  if (device >= n) {
    set_error("appt_comm_init: device ordinal beyond the device count");
    return kErrInvalid;
  }
  CKC(cudaSetDevice(device));
  Comm* c = new Comm;
  c->nranks = nranks;
  c->rank = rank;
  c->device = device;
  c->cap = nranks + 8 > 64 ? nranks + 8 : 64;
  int rc = kOk;
  auto fail = [&](int code) {
    if (c->s) cudaStreamDestroy(c->s);
    if (c->done) cudaEventDestroy(c->done);
    if (c->h_buf) cudaFreeHost(c->h_buf);
    if (c->d_buf) cudaFree(c->d_buf);
    delete c;
    return code;
  };
  if (cudaStreamCreateWithFlags(&c->s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming) != cudaSuccess ||
      cudaMallocHost((void**)&c->h_buf, sizeof(long long) * (size_t)c->cap) != cudaSuccess ||
      cudaMalloc((void**)&c->d_buf, sizeof(long long) * (size_t)c->cap) != cudaSuccess) {
    set_error(std::string("appt_comm_init: ") + cudaGetErrorString(cudaGetLastError()));
    return fail(kErrCuda);
  }
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  const ncclResult_t r = g_nccl.comm_init_rank(&c->nc, nranks, u, rank);
  if (r != ncclSuccess) {
    rc = nccl_fail(r, "ncclCommInitRank");
    return fail(rc);
  }
  *out = c;
  return kOk;
}

int comm_destroy(Comm* c) {
  if (!c) return kOk;
  cudaSetDevice(c->device);
  if (c->s) cudaStreamSynchronize(c->s);
  if (c->nc) g_nccl.comm_destroy(c->nc);
  if (c->s) cudaStreamDestroy(c->s);
  if (c->done) cudaEventDestroy(c->done);
  if (c->h_buf) cudaFreeHost(c->h_buf);
  if (c->d_buf) cudaFree(c->d_buf);
  delete c;
  return kOk;
}

static int check_live(Comm* c) {
  if (!c) {
    set_error("null communicator");
    return kErrInvalid;
  }
  if (c->broken || !c->nc) {
    set_error("the communicator was aborted by an earlier failure; create a new one");
    return kErrCuda;
  }
  return kOk;
}

// Broadcast of `count` int64 values from root through the pinned/device staging buffers; on
// return h_buf[1 .. count] holds them on every rank.
static int bcast_small(Comm* c, int root, int count) {
  CKC(cudaMemcpyAsync(c->d_buf + 1, c->h_buf + 1, sizeof(long long) * (size_t)count,
                      cudaMemcpyHostToDevice, c->s));
  CKN(g_nccl.broadcast(c->d_buf + 1, c->d_buf + 1, (size_t)count, ncclInt64, root, c->nc, c->s),
      "ncclBroadcast");
  CKC(cudaMemcpyAsync(c->h_buf + 1, c->d_buf + 1, sizeof(long long) * (size_t)count,
                      cudaMemcpyDeviceToHost, c->s));
  CKC(cudaEventRecord(c->done, c->s));
  return wait_bounded(c, "broadcast");
}

int comm_broadcast_csr(Comm* c, int root, MatView* M, bool* allocated, double* ms) {
  int rc = check_live(c);
  if (rc) return rc;
  if (!M || root < 0 || root >= c->nranks) {
    set_error("appt_comm_broadcast_csr: invalid argument");
    return kErrInvalid;
  }
  std::lock_guard<std::mutex> lk(c->mu);
  CKC(cudaSetDevice(c->device));
  *allocated = false;
  if (c->rank == root) {
    c->h_buf[1] = M->rows;
    c->h_buf[2] = M->cols;
    c->h_buf[3] = M->nnz;
  }
  rc = bcast_small(c, root, 3);
  if (rc) return rc;
  const long long rows = c->h_buf[1], cols = c->h_buf[2], nnz = c->h_buf[3];
  if (rows < 0 || cols < 0 || nnz < 0 || rows >= (1ll << 31) - 1 || nnz >= (1ll << 31) - 1) {
    set_error("appt_comm_broadcast_csr: sizes out of range");
    return kErrInvalid;
  }
  int* rp = const_cast<int*>(M->rp);
  int* ci = const_cast<int*>(M->ci);
  double* val = const_cast<double*>(M->val);
  if (c->rank != root) {
    rp = nullptr;
    ci = nullptr;
    val = nullptr;
    if (cudaMalloc((void**)&rp, sizeof(int) * (size_t)(rows + 1)) != cudaSuccess ||
        cudaMalloc((void**)&ci, sizeof(int) * (size_t)(nnz > 0 ? nnz : 1)) != cudaSuccess ||
        cudaMalloc((void**)&val, sizeof(double) * (size_t)(nnz > 0 ? nnz : 1)) != cudaSuccess) {
      cudaGetLastError();
      cudaFree(rp);
      cudaFree(ci);
      cudaFree(val);
      set_error("appt_comm_broadcast_csr: device allocation failed");
      // the root still sends: receive into nothing is impossible, so abort the communicator
      g_nccl.comm_abort(c->nc);
      c->nc = nullptr;
      c->broken = true;
      return kErrOom;
    }
  }
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  CKC(cudaEventCreate(&t0));
  CKC(cudaEventCreate(&t1));
  CKC(cudaEventRecord(t0, c->s));
  CKN(g_nccl.group_start(), "ncclGroupStart");
  CKN(g_nccl.broadcast(rp, rp, (size_t)(rows + 1), ncclInt32, root, c->nc, c->s), "ncclBroadcast");
  if (nnz > 0) {
    CKN(g_nccl.broadcast(ci, ci, (size_t)nnz, ncclInt32, root, c->nc, c->s), "ncclBroadcast");
    CKN(g_nccl.broadcast(val, val, (size_t)nnz, ncclFloat64, root, c->nc, c->s),
        "ncclBroadcast");
  }
  CKN(g_nccl.group_end(), "ncclGroupEnd");
  CKC(cudaEventRecord(t1, c->s));
  CKC(cudaEventRecord(c->done, c->s));
  rc = wait_bounded(c, "broadcast of B");
  float el = 0.f;
  if (rc == kOk) cudaEventElapsedTime(&el, t0, t1);
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  if (ms) *ms = el;
  if (c->rank != root) {
    if (rc) {
      cudaFree(rp);
      cudaFree(ci);
      cudaFree(val);
      return rc;
    }
    M->rows = rows;
    M->cols = cols;
    M->nnz = nnz;
    M->rp = rp;
    M->ci = ci;
    M->val = val;
    *allocated = true;
  }
  return rc;
}

int comm_row_split(Comm* c, int root, const MatView* A, const MatView* B, long long* bounds) {
  int rc = check_live(c);
  if (rc) return rc;
  if (!bounds || root < 0 || root >= c->nranks || (c->rank == root && !A)) {
    set_error("appt_comm_row_split: invalid argument");
    return kErrInvalid;
  }
  const int n = c->nranks;
  std::vector<long long> b(n + 1, 0);
  int local = kOk;
  if (c->rank == root) {   // row products of op(A, B) on this device, then the prefix split
    CallOptions o;
    o.in_mem = 1;
    o.device = c->device;
    std::vector<long long> p((size_t)A->rows);
    local = row_products(*A, B, o, p.data());
    if (local == kOk) local = split_rows(p.data(), A->rows, n, b.data());
    if (local != kOk) std::fill(b.begin(), b.end(), -1ll);   // the others learn of the failure
  }
  std::lock_guard<std::mutex> lk(c->mu);
  CKC(cudaSetDevice(c->device));
  for (int r = 0; r <= n; ++r) c->h_buf[1 + r] = b[(size_t)r];
  rc = bcast_small(c, root, n + 1);
  if (rc) return rc;
  for (int r = 0; r <= n; ++r) bounds[r] = c->h_buf[1 + r];
  if (local) return local;
  if (bounds[0] < 0) {
    set_error("appt_comm_row_split: the root rank failed to compute the split");
    return kErrInvalid;
  }
  return kOk;
}

// Posts this rank's nnz (or -1 for a failed call) to the all-gather on the comm stream.
static int post_nnz(Comm* c, long long nnz) {
  c->h_buf[0] = nnz;
  CKC(cudaMemcpyAsync(c->d_buf, c->h_buf, sizeof(long long), cudaMemcpyHostToDevice, c->s));
  CKN(g_nccl.all_gather(c->d_buf, c->d_buf + 1, 1, ncclInt64, c->nc, c->s), "ncclAllGather");
  CKC(cudaMemcpyAsync(c->h_buf + 1, c->d_buf + 1, sizeof(long long) * (size_t)c->nranks,
                      cudaMemcpyDeviceToHost, c->s));
  CKC(cudaEventRecord(c->done, c->s));
  return kOk;
}

int comm_spgemm(Comm* c, const MatView& A, const MatView* B, CallOptions opt, MatOut* C,
                long long* offsets, CallStats* st) {
  int rc = check_live(c);
  if (rc) return rc;
  if (!offsets || !C) {
    set_error("appt_comm_spgemm: null argument");
    return kErrInvalid;
  }
  std::lock_guard<std::mutex> lk(c->mu);
  opt.device = c->device;
  using clk = std::chrono::steady_clock;
  const clk::time_point t0 = clk::now();
  clk::time_point t_post = t0;
  bool posted = false;
  int post_rc = kOk;
  const std::function<int(long long)> hook = [&](long long nnz) {
    posted = true;
    post_rc = post_nnz(c, nnz);
    t_post = clk::now();
    return post_rc;
  };
  opt.on_nnz = &hook;
  rc = spgemm(A, B, opt, C, st);
  const clk::time_point t_pipe = clk::now();
  // every rank takes part in the exchange, failed or not, so that no rank waits for ever
  if (!posted) post_rc = post_nnz(c, -1);
  if (post_rc) {
    if (rc == kOk) free_out(C);
    return post_rc;
  }
  const bool ready = cudaEventQuery(c->done) == cudaSuccess;
  const int wrc = wait_bounded(c, "nnz exchange");
  if (wrc) {
    if (rc == kOk) free_out(C);
    return wrc;
  }
  const char* pe = std::getenv("APPT_PROF");
  if (pe && std::atoi(pe) >= 2) {
    auto us = [&](clk::time_point t) {
      return std::chrono::duration<double, std::micro>(t - t0).count();
    };
    fprintf(stderr,
            "[%s-host] rank %d/%d: exchange posted %.1f us, call returned %.1f us, exchange "
            "%s, done %.1f us\n",
            opt.prof_tag, c->rank, c->nranks, us(t_post), us(t_pipe),
            ready ? "already complete" : "waited for", us(clk::now()));
  }
  offsets[0] = 0;
  bool peer_failed = false;
  for (int r = 0; r < c->nranks; ++r) {
    const long long v = c->h_buf[1 + r];
    if (v < 0) peer_failed = true;
    offsets[r + 1] = offsets[r] + (v > 0 ? v : 0);
  }
  if (rc == kOk && peer_failed) {
    free_out(C);
    set_error("appt_comm_spgemm: another rank's block failed");
    return kErrDevice;
  }
  return rc;
}

int split_rows(const long long* products, long long rows, int parts, long long* bounds) {
  if (!bounds || parts < 1 || rows < 0 || (rows > 0 && !products)) {
    set_error("appt_split_rows: invalid argument");
    return kErrInvalid;
  }
  std::vector<long long> cum((size_t)rows + 1, 0);
  for (long long i = 0; i < rows; ++i) {
    if (products[i] < 0) {
      set_error("appt_split_rows: negative products count");
      return kErrInvalid;
    }
    cum[(size_t)i + 1] = cum[(size_t)i] + products[i];
  }
  const long long total = cum[(size_t)rows];
  bounds[0] = 0;
  for (int r = 1; r < parts; ++r) {
    // the cut whose prefix is nearest to r/parts of the total (ties to the earlier cut)
    const long double target = (long double)total * r / parts;
    long long lo = 0, hi = rows;   // first index with cum >= target
    while (lo < hi) {
      const long long mid = (lo + hi) / 2;
      if ((long double)cum[(size_t)mid] < target) lo = mid + 1; else hi = mid;
    }
    long long b = lo;
    if (b > 0 && target - (long double)cum[(size_t)b - 1] <= (long double)cum[(size_t)b] - target)
      --b;
    if (b < bounds[r - 1]) b = bounds[r - 1];
    bounds[r] = b;
  }
  bounds[parts] = rows;
  return kOk;
}

}  // namespace appt

// ---------------------------------------------------------------------------------- C ABI
namespace {
appt::MatView view_of_csr(const appt_csr* a) {
  appt::MatView v;
  v.rows = a->rows;
  v.cols = a->cols;
  v.nnz = a->nnz;
  v.rp = a->row_ptr;
  v.ci = a->col_idx;
  v.val = a->val;
  return v;
}
}  // namespace

extern "C" {

int appt_comm_unique_id(void* id) { return appt::comm_unique_id(id); }

int appt_comm_init(const void* id, int nranks, int rank, int device, appt_comm** out) {
  if (!out) {
    appt::set_error("null output");
    return APPT_ERR_INVALID;
  }
  *out = nullptr;
  appt::Comm* c = nullptr;
  const int rc = appt::comm_init(id, nranks, rank, device, &c);
  if (rc) return rc;
  *out = new appt_comm{c};
  return APPT_OK;
}

int appt_comm_destroy(appt_comm* comm) {
  if (!comm) return APPT_OK;
  const int rc = appt::comm_destroy(comm->c);
  delete comm;
  return rc;
}

int appt_comm_broadcast_csr(appt_comm* comm, int root, appt_csr* M, double* ms) {
  if (!comm || !M) {
    appt::set_error("null argument");
    return APPT_ERR_INVALID;
  }
  appt::MatView v = view_of_csr(M);
  bool allocated = false;
  const int rc = appt::comm_broadcast_csr(comm->c, root, &v, &allocated, ms);
  if (rc == APPT_OK && allocated) {
    M->rows = v.rows;
    M->cols = v.cols;
    M->nnz = v.nnz;
    M->row_ptr = v.rp;
    M->col_idx = v.ci;
    M->val = v.val;
  }
  return rc;
}

int appt_comm_free_csr(appt_comm* comm, appt_csr* M) {
  if (!comm || !M) return APPT_ERR_INVALID;
  cudaSetDevice(comm->c->device);
  cudaFree(const_cast<int32_t*>(M->row_ptr));
  cudaFree(const_cast<int32_t*>(M->col_idx));
  cudaFree(const_cast<double*>(M->val));
  std::memset(M, 0, sizeof(*M));
  return APPT_OK;
}

int appt_split_rows(const int64_t* row_products, int64_t rows, int parts, int64_t* bounds) {
  return appt::split_rows(reinterpret_cast<const long long*>(row_products), rows, parts,
                          reinterpret_cast<long long*>(bounds));
}

int appt_comm_row_split(appt_comm* comm, int root, const appt_csr* A, const appt_csr* B,
                        int64_t* bounds) {
  if (!comm) {
    appt::set_error("null communicator");
    return APPT_ERR_INVALID;
  }
  appt::MatView a, b;
  if (A) a = view_of_csr(A);
  if (B) b = view_of_csr(B);
  return appt::comm_row_split(comm->c, root, A ? &a : nullptr, B ? &b : nullptr,
                              reinterpret_cast<long long*>(bounds));
}

}  // extern "C"
