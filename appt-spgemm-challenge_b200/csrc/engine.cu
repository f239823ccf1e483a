// Host pipeline of the engine: operand staging, transpose for A*A^T, the analyze -> symbolic ->
// scan -> numeric sequence, the ESC baseline flow, pools, error handling and phase timing.
//
// Reference counterparts: hash_product (spgemm_kernel_hash.cu:813-1109), merge3_product
// (spgemm_merge.cu:760-933), spgemm_self_product_manual (spgemm_kernel_manual.cu:272-437) and
// the pools of src/mempool.cu. Differences that matter to callers:
//   * one host synchronisation inside the pipeline (to size C), instead of one per phase;
//   * all temporaries come from a CUDA stream-ordered memory pool (release threshold raised, so
//     steady-state calls do no driver allocation);
//   * every failure returns a status instead of exiting the process.
#include <cuda_runtime.h>
#include <algorithm>
#include <chrono>
#include <functional>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "engine.h"
#include "kernels.cuh"

namespace appt {

// ------------------------------------------------------------------ errors and counters
static thread_local std::string t_last_error;
void set_error(const std::string& m) { t_last_error = m; }
const char* last_error() { return t_last_error.c_str(); }

static std::atomic<long long> g_launches{0};
long long kernel_launches() { return g_launches.load(); }
void note_launches(long long n) { g_launches += n; }

#define CK(call)                                                                          \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess) {                                                              \
      set_error(std::string(#call) + ": " + cudaGetErrorString(e_));                      \
      return e_ == cudaErrorMemoryAllocation ? kErrOom : kErrCuda;                        \
    }                                                                                     \
  } while (0)

static bool env_flag(const char* k) {
  const char* e = std::getenv(k);
  return e && *e && std::atoi(e) > 0;
}

int device_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// ------------------------------------------------------------------ per-device context
struct DeviceCtx {
  int device = -1;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t copy_stream = nullptr;   // device-to-host copies that overlap the numeric phase
  cudaMemPool_t pool = nullptr;        // per-call temporaries
  cudaMemPool_t pool_big = nullptr;    // allocations of 64 MiB and more (C, large scratch): kept
                                       // apart so small temporaries never split their blocks
  char* stage = nullptr;       // pinned host staging for small device->host reads
  char* stage_dev = nullptr;   // the same memory as the device addresses it (readback kernels)
  // bitmap handoff arena (symbolic -> numeric rank tier), allocated on first use and kept: calls
  // on a device are serialised by `mu` and each ends with its work complete
  unsigned* harena = nullptr;
  bool harena_tried = false;
  // side streams: the per-bin kernels of one phase run concurrently (the small bins' kernels and
  // the tails of the large ones overlap instead of queueing behind each other)
  static constexpr int kSide = 3;
  cudaStream_t side[kSide] = {};
  cudaEvent_t ev_fork = nullptr;
  cudaEvent_t ev_join[kSide] = {};
  // events reused by every call (calls on a device are serialised by `mu`): phase timing events
  // (created on demand, kept), and the ordering events of host operands and host results
  std::vector<cudaEvent_t> ev_timing;
  static constexpr int kSinkEvents = 9;   // kSinkBlocks + 1
  cudaEvent_t ev_sink[kSinkEvents] = {};
  cudaEvent_t ev_staged[2] = {};           // operand allocations ordered before their copies
  cudaEvent_t ev_values = nullptr;         // host operands' values in place
  std::mutex mu;
  bool ok = false;
};

// Fans the launches of one phase out over `s` and the context's side streams: fork() makes the
// side streams wait for the work queued on `s` so far, at(j) is the stream of launch j, join()
// makes `s` wait for everything launched on the side streams.
struct Fan {
  DeviceCtx* ctx;
  cudaStream_t s;
  cudaError_t fork() {
    cudaError_t e = cudaEventRecord(ctx->ev_fork, s);
    for (int j = 0; j < DeviceCtx::kSide && e == cudaSuccess; ++j)
      e = cudaStreamWaitEvent(ctx->side[j], ctx->ev_fork, 0);
    return e;
  }
  cudaStream_t at(int j) const {
    const int l = j % (DeviceCtx::kSide + 1);
    return l == 0 ? s : ctx->side[l - 1];
  }
  cudaError_t join() {
    cudaError_t e = cudaSuccess;
    for (int j = 0; j < DeviceCtx::kSide && e == cudaSuccess; ++j) {
      e = cudaEventRecord(ctx->ev_join[j], ctx->side[j]);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ctx->ev_join[j], 0);
    }
    return e;
  }
};

static DeviceCtx g_ctx[64];
static std::mutex g_ctx_mu;

static int get_ctx(int device, DeviceCtx** out) {
  if (device < 0 || device >= 64) {
    set_error("device ordinal out of range");
    return kErrInvalid;
  }
  std::lock_guard<std::mutex> g(g_ctx_mu);
  DeviceCtx& c = g_ctx[device];
  if (!c.ok) {
    const int n = device_count();
    if (n == 0) {
      set_error("no CUDA device");
      return kErrNoDevice;
    }
    if (device >= n) {
      set_error("device ordinal beyond the device count");
      return kErrInvalid;
    }
    CK(cudaSetDevice(device));
    CK(cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, device));
    CK(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&c.copy_stream, cudaStreamNonBlocking));
    for (int j = 0; j < DeviceCtx::kSide; ++j) {
      CK(cudaStreamCreateWithFlags(&c.side[j], cudaStreamNonBlocking));
      CK(cudaEventCreateWithFlags(&c.ev_join[j], cudaEventDisableTiming));
    }
    CK(cudaEventCreateWithFlags(&c.ev_fork, cudaEventDisableTiming));
    for (int k = 0; k < DeviceCtx::kSinkEvents; ++k)
      CK(cudaEventCreateWithFlags(&c.ev_sink[k], cudaEventDisableTiming));
    for (int k = 0; k < 2; ++k) CK(cudaEventCreateWithFlags(&c.ev_staged[k], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&c.ev_values, cudaEventDisableTiming));
    cudaMemPoolProps props;
    std::memset(&props, 0, sizeof(props));
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    CK(cudaMemPoolCreate(&c.pool, &props));
    CK(cudaMemPoolCreate(&c.pool_big, &props));
    unsigned long long thr = ~0ull;
    CK(cudaMemPoolSetAttribute(c.pool, cudaMemPoolAttrReleaseThreshold, &thr));
    CK(cudaMemPoolSetAttribute(c.pool_big, cudaMemPoolAttrReleaseThreshold, &thr));
    CK(cudaMallocHost((void**)&c.stage, 4096));
    CK(cudaHostGetDevicePointer((void**)&c.stage_dev, c.stage, 0));
    c.device = device;
    c.ok = true;
  }
  *out = &c;
  return kOk;
}

// Lays several arrays out in one allocation (256-byte aligned): a first pass with base == nullptr
// only adds up the bytes, a second pass over a block of that size hands out the pointers.
struct Carver {
  char* base = nullptr;
  size_t off = 0;
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += (count ? count : 1) * sizeof(T);
    return p;
  }
};

// Stream-ordered scratch allocations freed when the object goes out of scope, unless detached.
struct Scratch {
  DeviceCtx* ctx;
  cudaStream_t s;
  std::vector<void*> ptrs;
  std::vector<std::vector<int>> host_keep;   // host staging copies alive until the call ends
  bool failed = false;
  Scratch(DeviceCtx* c, cudaStream_t st) : ctx(c), s(st) {}
  // One allocation for the arrays `layout(Carver&)` takes (called twice: sizes, then pointers).
  template <typename F>
  bool carve(F&& layout) {
    Carver sizes;
    layout(sizes);
    char* base = get<char>(sizes.off, true);   // per-call arrays: never beside C in the big pool
    if (!base) return false;
    Carver c;
    c.base = base;
    layout(c);
    return true;
  }
  template <typename T>
  T* get(size_t count, bool small_pool = false) {
    size_t bytes = count * sizeof(T);
    if (bytes == 0) bytes = 256;
    void* p = nullptr;
    cudaMemPool_t pool = !small_pool && bytes >= (size_t(64) << 20) ? ctx->pool_big : ctx->pool;
    if (cudaMallocFromPoolAsync(&p, bytes, pool, s) != cudaSuccess) {
      cudaGetLastError();
      failed = true;
      return nullptr;
    }
    ptrs.push_back(p);
    return reinterpret_cast<T*>(p);
  }
  void detach(void* p) {
    for (auto& q : ptrs)
      if (q == p) q = nullptr;
  }
  ~Scratch() {
    for (void* p : ptrs)
      if (p) cudaFreeAsync(p, s);
  }
};

// ------------------------------------------------------------------ phase timing
struct PhaseTimer {
  bool on = false;
  cudaStream_t s = nullptr;
  std::vector<cudaEvent_t>* pool = nullptr;   // the device's reusable timing events
  size_t used = 0;
  struct Mark {
    int phase;
    cudaEvent_t a, b;
  };
  std::vector<Mark> marks;
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  int cur = -1;
  cudaEvent_t cur_a = nullptr;
  cudaEvent_t take() {
    if (used == pool->size()) {
      cudaEvent_t e = nullptr;
      cudaEventCreate(&e);
      pool->push_back(e);
    }
    return (*pool)[used++];
  }
  void start(bool enable, cudaStream_t st, std::vector<cudaEvent_t>* events) {
    on = enable;
    s = st;
    pool = events;
    used = 0;
    if (!on) return;
    t0 = take();
    t1 = take();
    cudaEventRecord(t0, s);
  }
  void begin(int phase) {
    if (!on) return;
    end();
    cur = phase;
    cur_a = take();
    cudaEventRecord(cur_a, s);
  }
  void end() {
    if (!on || cur < 0) return;
    cudaEvent_t b = take();
    cudaEventRecord(b, s);
    marks.push_back({cur, cur_a, b});
    cur = -1;
  }
  void finish(CallStats* st) {
    if (!on) return;
    end();
    cudaEventRecord(t1, s);
    cudaEventSynchronize(t1);
    float ms = 0.f;
    if (st) {
      cudaEventElapsedTime(&ms, t0, t1);
      st->ms_total = ms;
      for (int i = 0; i < 8; ++i) st->ms_phase[i] = 0.0;
      for (auto& m : marks) {
        cudaEventElapsedTime(&ms, m.a, m.b);
        st->ms_phase[m.phase] += ms;
      }
    }
    marks.clear();
    used = 0;   // the events go back to the device's pool
    on = false;
  }
  ~PhaseTimer() {
    if (on) finish(nullptr);
  }
};

enum Phase { kPhH2D = 0, kPhTranspose, kPhAnalyze, kPhSymbolic, kPhScan, kPhNumeric, kPhD2H, kPhOther };
static const char* kPhaseNames[8] = {"h2d", "transpose", "analyze", "symbolic",
                                     "scan", "numeric",   "d2h",     "other"};

// ------------------------------------------------------------------ host timeline
// With APPT_PROF=2 the host-side moments of a call are recorded (microseconds since the call
// began) and printed with the phase lines: where the host waits at the synchronisations and how
// long it takes to issue the work around them.
struct HostMarks {
  bool on = false;
  std::chrono::steady_clock::time_point t0;
  std::vector<std::pair<const char*, double>> marks;
  void start(bool enable) {
    on = enable;
    marks.clear();
    if (on) t0 = std::chrono::steady_clock::now();
  }
  void mark(const char* what) {
    if (!on) return;
    marks.push_back({what, std::chrono::duration<double, std::micro>(
                               std::chrono::steady_clock::now() - t0).count()});
  }
};
static thread_local HostMarks t_marks;

// ------------------------------------------------------------------ device pipeline
// Called once per pipeline run with nnz(C), right after the mid-pipeline synchronisation that
// learns it and before the numeric phase (multi-GPU calls post their nnz exchange from here).
using NnzHook = std::function<int(long long)>;

static int notify_nnz(const NnzHook* hook, long long nnz) { return hook ? (*hook)(nnz) : kOk; }

constexpr int kSinkBlocks = 8;   // row blocks of the numeric phase when C goes to the host

// Host destination of C. With a sink, the numeric phase runs in row blocks and the copies of a
// finished block go out on the copy stream while the next block computes; `alloc` is called
// once nnz(C) is known and returns the host arrays (exactly one of rp32 / rp64 set).
struct HostDst {
  int* rp32 = nullptr;
  long long* rp64 = nullptr;
  int* ci = nullptr;
  double* val = nullptr;
};
struct HostSink {
  std::function<bool(long long nnz, HostDst* d)> alloc;
  bool done = false;   // the pipeline filled the destination
  long long nnz = 0;
  long long cols = 0;
};

struct DevC {            // device-resident result, allocations owned by the pool
  long long rows = 0, cols = 0, nnz = 0;
  long long* rp = nullptr;
  int* ci = nullptr;
  double* val = nullptr;
};

static int lanes_per_row(long long nnz, long long rows) {
  return analyze_lanes_per_row(nnz, rows);
}

static int esc_device(DeviceCtx* ctx, Csr A, Csr B, long long a_nnz, int upper, int row_base,
                      cudaStream_t s, Scratch& sc, PhaseTimer& tm, DevC* C, CallStats* st,
                      const NnzHook* on_nnz) {
  const int m = A.rows;
  const int sms = ctx->num_sms;
  long long* flop = sc.get<long long>(m);
  int* lo = sc.get<int>(m);
  int* hi = sc.get<int>(m);
  uint8_t* key = sc.get<uint8_t>(m);
  int* row_nnz = sc.get<int>(m);
  long long* foff = sc.get<long long>((size_t)m + 1);
  long long* crp = sc.get<long long>((size_t)m + 1);
  long long* scs = sc.get<long long>(scan_scratch_elems(m));
  AnalyzeStats* gst = sc.get<AnalyzeStats>(1);
  int* err = sc.get<int>(4);
  if (sc.failed) {
    set_error("device pool allocation failed");
    return kErrOom;
  }
  CK(cudaMemsetAsync(gst, 0, sizeof(AnalyzeStats), s));
  CK(cudaMemsetAsync(err, 0, sizeof(int) * 4, s));
  tm.begin(kPhAnalyze);
  launch_analyze(A, B, upper, row_base, kMethodEsc, lanes_per_row(a_nnz, m), flop, lo, hi, key,
                 row_nnz, gst, err, sms, s);
  note_launches(m > 0 ? 2 : 0);
  note_launches(scan_exclusive(flop, foff, m, scs, s));
  CK(cudaMemcpyAsync(ctx->stage, foff + m, 8, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(ctx->stage + 64, gst, sizeof(AnalyzeStats), cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(ctx->stage + 128, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  long long P;
  std::memcpy(&P, ctx->stage, 8);
  AnalyzeStats hst;
  std::memcpy(&hst, ctx->stage + 64, sizeof(hst));
  int herr = 0;
  std::memcpy(&herr, ctx->stage + 128, sizeof(int));
  if (herr & kErrBounds) {
    set_error("operand index out of range (A column >= B rows)");
    return kErrInvalid;
  }
  if (st) st->products = (long long)hst.total_flop;
  int* keys = sc.get<int>(P);
  double* vals = sc.get<double>(P);
  int* keys_alt = sc.get<int>(P);
  double* vals_alt = sc.get<double>(P);
  void* sss = sc.get<char>(segsort_scratch_bytes(m));
  if (sc.failed) {
    set_error("device pool allocation failed (ESC needs 24 bytes per intermediate product)");
    return kErrOom;
  }
  tm.begin(kPhNumeric);
  launch_esc_expand(A, B, upper, row_base, foff, keys, vals, sms, s);
  segsort(keys, vals, keys_alt, vals_alt, foff, m, sss, sms, s);
  launch_esc_count(m, foff, keys, row_nnz, sms, s);
  note_launches(m > 0 ? 13 : 0);
  tm.begin(kPhScan);
  note_launches(scan_exclusive(row_nnz, crp, m, scs, s));
  CK(cudaMemcpyAsync(ctx->stage, crp + m, 8, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  long long nnz;
  std::memcpy(&nnz, ctx->stage, 8);
  const int hrc = notify_nnz(on_nnz, nnz);
  if (hrc) return hrc;
  int* cci = sc.get<int>(nnz);
  double* cval = sc.get<double>(nnz);
  if (sc.failed) {
    set_error("device pool allocation failed for C");
    return kErrOom;
  }
  tm.begin(kPhNumeric);
  launch_esc_compress(m, foff, keys, vals, crp, cci, cval, sms, s);
  note_launches(m > 0 ? 1 : 0);
  tm.end();
  CK(cudaStreamSynchronize(s));   // the call returns with C complete, like the other methods
  sc.detach(crp);
  sc.detach(cci);
  sc.detach(cval);
  C->rows = m;
  C->cols = B.cols;
  C->nnz = nnz;
  C->rp = crp;
  C->ci = cci;
  C->val = cval;
  if (st) {
    st->c_nnz = nnz;
    st->method_used = kMethodEsc;
  }
  return kOk;
}

// Small problems: one unbinned symbolic pass and one rank-tier launch over all rows, a handful of
// launches instead of the binned pipeline's dozens. *fallback is set (nothing computed) when a
// row does not fit; the caller then runs the general pipeline. The row limit is measured: a
// 2^17-row block of the 64^3 stencil or of a banded matrix runs 10-13 % faster here than binned,
// a whole 2^18-row stencil 4 % slower.
#ifndef APPT_SMALL_ROWS
#define APPT_SMALL_ROWS 131072
#endif
constexpr long long kSmallRows = APPT_SMALL_ROWS;
constexpr long long kSmallNnz = 32 * kSmallRows;

static int small_device(DeviceCtx* ctx, Csr A, Csr B, long long a_nnz, int upper, int row_base,
                        cudaStream_t s, Scratch& sc, PhaseTimer& tm, DevC* C, CallStats* st,
                        bool* fallback, cudaEvent_t vals_ready, const NnzHook* on_nnz) {
  *fallback = false;
  const int m = A.rows;
  const int sms = ctx->num_sms;
  int *lo, *hi, *row_nnz, *err;
  long long *boff, *scs;
  unsigned long long* tflop;
  sc.carve([&](Carver& c) {   // err and tflop first: one memset clears both
    err = c.take<int>(4);
    tflop = c.take<unsigned long long>(1);
    lo = c.take<int>(m);
    hi = c.take<int>(m);
    row_nnz = c.take<int>(m);
    boff = c.take<long long>(2);
    scs = c.take<long long>(scan_scratch_elems(m));
  });
  long long* crp = sc.get<long long>((size_t)m + 1);   // handed to the caller with C
  if (sc.failed) {
    set_error("device pool allocation failed");
    return kErrOom;
  }
  CK(cudaMemsetAsync(err, 0, (char*)(tflop + 1) - (char*)err, s));
  const int gidx = group_index(a_nnz, m);   // B rows' average length taken from A's
  tm.begin(kPhSymbolic);
  launch_symbolic_small(A, B, upper, row_base, gidx, lo, hi, row_nnz, boff, tflop, err, sms, s);
  note_launches(1);
  tm.begin(kPhScan);
  note_launches(scan_exclusive(row_nnz, crp, m, scs, s));
  char* stg = ctx->stage;
  Readback rb;   // one kernel writes the values into the pinned stage
  const int o_nnz = rb.add(crp + m, 8), o_flop = rb.add(tflop, 8), o_err = rb.add(err, 8);
  launch_readback(rb, ctx->stage_dev, s);
  note_launches(1);
  t_marks.mark("issued up to the mid sync");
  CK(cudaStreamSynchronize(s));
  t_marks.mark("mid sync returned");
  long long nnz;
  int herr;
  unsigned long long hflop;
  int max_need = 0;   // err[1]: the largest per-row rank-tier budget
  std::memcpy(&nnz, stg + o_nnz, 8);
  std::memcpy(&herr, stg + o_err, sizeof(int));
  std::memcpy(&max_need, stg + o_err + 4, sizeof(int));
  std::memcpy(&hflop, stg + o_flop, 8);
  if (herr & kErrBounds) {
    set_error("operand index out of range (A column >= B rows)");
    return kErrInvalid;
  }
  if (herr & kErrSmallFallback) {
    *fallback = true;
    return kOk;
  }
  if (herr) {
    set_error("symbolic phase reported device error bits " + std::to_string(herr));
    return kErrDevice;
  }
  const int hrc = notify_nnz(on_nnz, nnz);
  if (hrc) return hrc;
  int* cci = sc.get<int>(nnz);
  double* cval = sc.get<double>(nnz);
  if (sc.failed) {
    set_error("device pool allocation failed for C (" + std::to_string(nnz) + " entries)");
    return kErrOom;
  }
  tm.begin(kPhNumeric);
  if (vals_ready) CK(cudaStreamWaitEvent(s, vals_ready, 0));
  launch_numeric_rank_all(boff, m, gidx, max_need, A, B, lo, hi, crp, cci, cval, err, sms, s);
  note_launches(1);
  tm.end();
  CK(cudaMemcpyAsync(stg + 8, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  t_marks.mark("numeric issued");
  CK(cudaStreamSynchronize(s));
  t_marks.mark("final sync returned");
  std::memcpy(&herr, stg + 8, sizeof(int));
  if (herr) {
    set_error("numeric phase reported device error bits " + std::to_string(herr));
    return kErrDevice;
  }
  sc.detach(crp);
  sc.detach(cci);
  sc.detach(cval);
  C->rows = m;
  C->cols = B.cols;
  C->nnz = nnz;
  C->rp = crp;
  C->ci = cci;
  C->val = cval;
  if (st) {
    st->products = (long long)hflop;
    st->c_nnz = nnz;
    st->method_used = kMethodAdaptive;
    const int tier = max_need <= 2304 ? kNumRank2K : max_need <= 4608 ? kNumRank4K : kNumRank8K;
    st->bin_rows[tier + gidx] = m;
  }
  return kOk;
}

// vals_ready (may be null): event after which A's and B's values are in place; kernels that
// read values wait for it.
static int multiply_device(DeviceCtx* ctx, Csr A, Csr B, long long a_nnz, long long b_nnz,
                           int upper, int row_base, int method, cudaStream_t s, Scratch& sc,
                           PhaseTimer& tm, DevC* C, CallStats* st, HostSink* sink,
                           cudaEvent_t vals_ready, const NnzHook* on_nnz) {
  if (method == kMethodEsc) {
    if (vals_ready) CK(cudaStreamWaitEvent(s, vals_ready, 0));
    return esc_device(ctx, A, B, a_nnz, upper, row_base, s, sc, tm, C, st, on_nnz);
  }
  if (method == kMethodAdaptive && A.rows > 0 && A.rows <= kSmallRows && a_nnz <= kSmallNnz &&
      !env_flag("APPT_NO_SMALL_PATH")) {
    bool fallback = false;
    const int rc = small_device(ctx, A, B, a_nnz, upper, row_base, s, sc, tm, C, st, &fallback,
                                vals_ready, on_nnz);
    if (rc != kOk || !fallback) return rc;
  }
  const int m = A.rows;
  const int sms = ctx->num_sms;
  constexpr int kSymMergeBin = kNumSymBins;
  const int nsb = kNumSymBins + 1;
  long long *flop, *boff_sym, *boff_num, *scs;
  int *lo, *hi, *row_nnz, *hslot, *rows_sym, *rows_num, *err;
  uint8_t *symkey, *numkey;
  unsigned long long* htop;
  AnalyzeStats* gst;
  void* pscr;
  sc.carve([&](Carver& c) {   // the three zero-initialised ones first: one memset clears them
    gst = c.take<AnalyzeStats>(1);
    err = c.take<int>(4);
    htop = c.take<unsigned long long>(1);
    flop = c.take<long long>(m);
    lo = c.take<int>(m);
    hi = c.take<int>(m);
    symkey = c.take<uint8_t>(m);
    numkey = c.take<uint8_t>(m);
    row_nnz = c.take<int>(m);
    hslot = c.take<int>(m);
    rows_sym = c.take<int>(m);
    rows_num = c.take<int>(m);
    boff_sym = c.take<long long>(kMaxBins + 1);
    boff_num = c.take<long long>(kMaxBins + 1);
    scs = c.take<long long>(scan_scratch_elems(m));
    pscr = c.take<char>(partition_scratch_bytes(m, kMaxBins));
  });
  long long* crp = sc.get<long long>((size_t)m + 1);   // handed to the caller with C
  if (sc.failed) {
    set_error("device pool allocation failed");
    return kErrOom;
  }
  CK(cudaMemsetAsync(gst, 0, (char*)(htop + 1) - (char*)gst, s));
  CK(cudaMemsetAsync(hslot, 0xff, sizeof(int) * (size_t)m, s));

  // arena for the bitmaps the symbolic bitmap tier hands to the numeric rank tier (rows that
  // find it full rebuild their bitmaps in the numeric phase)
  if (!ctx->harena_tried) {
    ctx->harena_tried = true;
    if (cudaMalloc((void**)&ctx->harena, sizeof(unsigned) * (size_t)kHandoffArenaWords) !=
        cudaSuccess) {
      cudaGetLastError();
      ctx->harena = nullptr;
    }
  }
  RowBitmaps handoff;
  if (ctx->harena && m > 0) {
    handoff.slot = hslot;
    handoff.data = ctx->harena;
    handoff.top = htop;
    handoff.capacity = kHandoffArenaWords;
    // a smaller usable capacity (tests of the arena-full fallback)
    if (const char* e = std::getenv("APPT_HANDOFF_WORDS")) {
      const long long w = std::atoll(e);
      if (w >= 0 && w < handoff.capacity) handoff.capacity = w;
    }
  }

  tm.begin(kPhAnalyze);
  launch_analyze(A, B, upper, row_base, method, lanes_per_row(a_nnz, m), flop, lo, hi, symkey,
                 row_nnz, gst, err, sms, s);
  note_launches(m > 0 ? 2 : 0);   // analyze (short rows, long rows)
  note_launches(partition_rows(symkey, m, nsb, rows_sym, boff_sym, pscr, s));

  tm.begin(kPhSymbolic);
  // bitmaps of B's dense rows for the CTA symbolic tier, when B is wide enough for that tier
  DenseRows dense;
  if (m > 0 && B.cols > kDenseRowsMinCols && b_nnz >= kDenseRowsMinAvg * B.rows) {
    const long long stride = ((long long)B.cols + 31) / 32 + 1;
    long long max_rows = b_nnz * 32 / B.cols;   // rows with >= B.cols / 32 entries
    if (max_rows > kDenseRowsMaxWords / (2 * stride)) max_rows = kDenseRowsMaxWords / (2 * stride);
    if (max_rows > 0) {
      int* did = sc.get<int>(B.rows);
      int* dlist = sc.get<int>(max_rows);
      unsigned* dbits = sc.get<unsigned>((size_t)max_rows * stride);
      unsigned* dpre = sc.get<unsigned>((size_t)max_rows * stride);
      int* dcnt = sc.get<int>(1);
      if (sc.failed) {
        set_error("device pool allocation failed");
        return kErrOom;
      }
      CK(cudaMemsetAsync(dcnt, 0, sizeof(int), s));
      note_launches(
          build_dense_rows(B, did, dlist, dbits, dpre, stride, (int)max_rows, dcnt, sms, s));
      dense.id = did;
      dense.bits = dbits;
      dense.pre = dpre;
      dense.stride = stride;
    }
  }
  if (m > 0) {
    Fan fan{ctx, s};
    CK(fan.fork());
    for (int b = 0; b < kNumSymBins; ++b)
      launch_symbolic(b, rows_sym, boff_sym, A, B, upper, row_base, lo, hi, flop, row_nnz, handoff,
                      dense, err + 3, err, sms, fan.at(b));
    CK(fan.join());
    note_launches(kNumSymBins);
    if (method == kMethodMerge) {
      launch_merge_count(rows_sym, boff_sym, kSymMergeBin, A, B, upper, row_base, row_nnz, err,
                         sms, s);
      note_launches(1);
    }
  }

  tm.begin(kPhScan);
  note_launches(scan_exclusive(row_nnz, crp, m, scs, s));
  launch_classify_numeric(A, m, method, flop, lo, hi, row_nnz, numkey, sms, s);
  note_launches(m > 0 ? 1 : 0);
  note_launches(partition_rows(numkey, m, kNumNumBins, rows_num, boff_num, pscr, s));
  // with a host sink the numeric phase runs in K row blocks (rows [k*m/K, (k+1)*m/K)), each
  // bin's share of a block located by binary search in its ascending row list
  const int K = (sink && m >= 4096) ? kSinkBlocks : 1;
  long long* bsub = nullptr;
  // row counters of the CTA tiers (which take rows dynamically): one per block and bin
  int* nctr = sc.get<int>((size_t)K * kNumNumBins);
  if (sc.failed) {
    set_error("device pool allocation failed");
    return kErrOom;
  }
  CK(cudaMemsetAsync(nctr, 0, sizeof(int) * (size_t)K * kNumNumBins, s));
  if (K > 1) {
    bsub = sc.get<long long>((size_t)kNumNumBins * (K + 1));
    if (sc.failed) {
      set_error("device pool allocation failed");
      return kErrOom;
    }
    block_bin_bounds(rows_num, boff_num, kNumNumBins, m, K, bsub, s);
    note_launches(1);
  }

  // the one mid-pipeline synchronisation: C's size, the numeric bin sizes (and the blocks' first
  // entries in C)
  // (one kernel writes them into the pinned stage)
  char* stg = ctx->stage;
  Readback rb;
  const int o_nnz = rb.add(crp + m, 8);
  const int o_boff = rb.add(boff_num, 8 * (kNumNumBins + 1));
  const int o_gst = rb.add(gst, sizeof(AnalyzeStats));
  const int o_err = rb.add(err, 4);
  int o_cs[kSinkBlocks + 1] = {0};
  for (int k = 1; k < K; ++k) o_cs[k] = rb.add(crp + (long long)k * m / K, 8);
  launch_readback(rb, ctx->stage_dev, s);
  note_launches(1);
  t_marks.mark("issued up to the mid sync");
  CK(cudaStreamSynchronize(s));
  t_marks.mark("mid sync returned");
  long long nnz;
  long long boff[kNumNumBins + 1];
  AnalyzeStats hst;
  int herr;
  std::memcpy(&nnz, stg + o_nnz, 8);
  std::memcpy(boff, stg + o_boff, sizeof(boff));
  std::memcpy(&hst, stg + o_gst, sizeof(hst));
  std::memcpy(&herr, stg + o_err, sizeof(int));
  if (herr & kErrBounds) {
    set_error("operand index out of range (A column >= B rows)");
    return kErrInvalid;
  }
  if (herr) {
    set_error("symbolic phase reported device error bits " + std::to_string(herr));
    return kErrDevice;
  }
  if (st) {
    st->products = (long long)hst.total_flop;
    for (int b = 0; b < kNumNumBins && b < 32; ++b) st->bin_rows[b] = boff[b + 1] - boff[b];
  }
  {
    const int hrc = notify_nnz(on_nnz, nnz);
    if (hrc) return hrc;
  }
  long long cstart[kSinkBlocks + 1];
  cstart[0] = 0;
  for (int k = 1; k < K; ++k) std::memcpy(&cstart[k], stg + o_cs[k], 8);
  cstart[K] = nnz;
  int* cci = sc.get<int>(nnz);
  double* cval = sc.get<double>(nnz);
  if (sc.failed) {
    set_error("device pool allocation failed for C (" + std::to_string(nnz) + " entries)");
    return kErrOom;
  }
  HostDst hd;
  cudaStream_t cs = ctx->copy_stream;
  cudaEvent_t evs[kSinkBlocks + 1];
  if (sink) {
    if (!sink->alloc(nnz, &hd)) {
      set_error("host allocation failed for C");
      return kErrOom;
    }
    for (int k = 0; k <= K; ++k) evs[k] = ctx->ev_sink[k];
    // row pointers first (converted to int32 for the reference layout)
    if (hd.rp32) {
      int* rp32 = sc.get<int>((size_t)m + 1);
      if (!rp32) {
        set_error("device pool allocation failed");
        return kErrOom;
      }
      narrow_rowptr(crp, rp32, (long long)m + 1, s);
      note_launches(1);
      CK(cudaEventRecord(evs[K], s));
      CK(cudaStreamWaitEvent(cs, evs[K], 0));
      CK(cudaMemcpyAsync(hd.rp32, rp32, sizeof(int) * ((size_t)m + 1), cudaMemcpyDeviceToHost,
                         cs));
    } else {
      CK(cudaEventRecord(evs[K], s));
      CK(cudaStreamWaitEvent(cs, evs[K], 0));
      CK(cudaMemcpyAsync(hd.rp64, crp, sizeof(long long) * ((size_t)m + 1),
                         cudaMemcpyDeviceToHost, cs));
    }
  }

  tm.begin(kPhNumeric);
  if (vals_ready) CK(cudaStreamWaitEvent(s, vals_ready, 0));
  for (int k = 0; k < K; ++k) {
    Fan fan{ctx, s};
    CK(fan.fork());
    int nl = 0;
    for (int b = 0; b < kNumNumBins; ++b) {
      const long long nr_all = boff[b + 1] - boff[b];
      if (nr_all <= 0) continue;
      // bin offsets of this block: bo[b], bo[b + 1] are the block's share of bin b
      const long long* bo = K > 1 ? bsub + (size_t)b * K + k : boff_num;
      const long long nr = K > 1 ? nr_all / K + 1 : nr_all;   // grid sizing only
      int* ctr = nctr + (size_t)k * kNumNumBins + b;
      const cudaStream_t bs = fan.at(nl++);
      if (b == kNumMerge)
        launch_merge_numeric(rows_num, bo, b, nr, A, B, upper, row_base, crp, cci, cval, err, sms,
                             bs);
      else
        launch_numeric(b, rows_num, bo, nr, A, B, upper, row_base, lo, hi, flop, handoff, dense,
                       crp, cci, cval, ctr, err, sms, bs);
      note_launches(1);
    }
    CK(fan.join());
    if (sink) {
      const long long e0 = cstart[k], e1 = cstart[k + 1];
      CK(cudaEventRecord(evs[k], s));
      CK(cudaStreamWaitEvent(cs, evs[k], 0));
      if (e1 > e0) {
        CK(cudaMemcpyAsync(hd.ci + e0, cci + e0, sizeof(int) * (size_t)(e1 - e0),
                           cudaMemcpyDeviceToHost, cs));
        CK(cudaMemcpyAsync(hd.val + e0, cval + e0, sizeof(double) * (size_t)(e1 - e0),
                           cudaMemcpyDeviceToHost, cs));
      }
    }
  }
  tm.end();
  if (sink) {
    CK(cudaStreamSynchronize(cs));
    sink->done = true;
    sink->nnz = nnz;
  }
  CK(cudaMemcpyAsync(stg + 512, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  t_marks.mark("numeric issued");
  CK(cudaStreamSynchronize(s));
  t_marks.mark("final sync returned");
  std::memcpy(&herr, stg + 512, sizeof(int));
  if (herr) {
    set_error("numeric phase reported device error bits " + std::to_string(herr));
    return kErrDevice;
  }
  sc.detach(crp);
  sc.detach(cci);
  sc.detach(cval);
  C->rows = m;
  C->cols = B.cols;
  C->nnz = nnz;
  C->rp = crp;
  C->ci = cci;
  C->val = cval;
  if (st) {
    st->c_nnz = nnz;
    st->method_used = method;
  }
  return kOk;
}

// ------------------------------------------------------------------ operand staging
// Copies a host operand into pool memory on `s`; with `vs` the values go on that stream instead
// (after an event that orders them behind the allocation on `s`), so that the index-only phases
// (analyze, symbolic) overlap their copy -- the caller must make `s` wait for `vs` before any
// kernel reads the values.
static int stage_operand(const MatView& M, Scratch& sc, cudaStream_t s, Csr* out,
                         cudaStream_t vs = nullptr, cudaEvent_t order_ev = nullptr) {
  int* rp = sc.get<int>((size_t)M.rows + 1);
  int* ci = sc.get<int>((size_t)M.nnz);
  double* val = sc.get<double>((size_t)M.nnz);
  if (sc.failed) {
    set_error("device pool allocation failed for an operand");
    return kErrOom;
  }
  // A host row block (row_ptr[0] != 0) is staged from col_idx + row_ptr[0] with its row pointers
  // rebased to 0, so the device copy holds exactly the block's entries.
  const int rp0 = M.rp[0];
  if (rp0 == 0) {
    CK(cudaMemcpyAsync(rp, M.rp, sizeof(int) * ((size_t)M.rows + 1), cudaMemcpyHostToDevice, s));
  } else {
    sc.host_keep.emplace_back((size_t)M.rows + 1);
    std::vector<int>& rb = sc.host_keep.back();
    for (long long i = 0; i <= M.rows; ++i) rb[(size_t)i] = M.rp[i] - rp0;
    CK(cudaMemcpyAsync(rp, rb.data(), sizeof(int) * rb.size(), cudaMemcpyHostToDevice, s));
  }
  if (M.nnz > 0) {
    CK(cudaMemcpyAsync(ci, M.ci + rp0, sizeof(int) * (size_t)M.nnz, cudaMemcpyHostToDevice, s));
    if (vs) {   // the values' stream waits for the allocation made on `s`
      CK(cudaEventRecord(order_ev, s));
      CK(cudaStreamWaitEvent(vs, order_ev, 0));
    }
    CK(cudaMemcpyAsync(val, M.val + rp0, sizeof(double) * (size_t)M.nnz, cudaMemcpyHostToDevice,
                       vs ? vs : s));
  }
  out->rp = rp;
  out->ci = ci;
  out->val = val;
  out->rows = (int)M.rows;
  out->cols = (int)M.cols;
  return kOk;
}

static int check_view(const MatView& M, int in_mem, const char* name) {
  if (M.rows < 0 || M.cols < 0 || M.nnz < 0 || M.rows >= (1ll << 31) - 1 ||
      M.cols >= (1ll << 31) - 1 || M.nnz >= (1ll << 31) - 1) {
    set_error(std::string(name) + ": sizes must be non-negative and below 2^31 - 1");
    return kErrInvalid;
  }
  if (!M.rp || (M.nnz > 0 && (!M.ci || !M.val))) {
    set_error(std::string(name) + ": null pointer");
    return kErrInvalid;
  }
  if (in_mem == 0) {
    if (M.rp[M.rows] - M.rp[0] != M.nnz) {
      set_error(std::string(name) + ": row_ptr[rows] - row_ptr[0] != nnz");
      return kErrInvalid;
    }
  }
  return kOk;
}

static int do_transpose(DeviceCtx* ctx, Csr A, long long nnz, Scratch& sc, cudaStream_t s,
                        Csr* AT, bool detach) {
  int* trp = sc.get<int>((size_t)A.cols + 1);
  int* tci = sc.get<int>((size_t)nnz);
  double* tval = sc.get<double>((size_t)nnz);
  void* tscr = sc.get<char>(transpose_scratch_bytes(A.rows, A.cols, nnz));
  if (sc.failed) {
    set_error("device pool allocation failed for the transpose");
    return kErrOom;
  }
  launch_transpose(A, nnz, trp, tci, tval, tscr, ctx->num_sms, s);
  note_launches(16);
  AT->rp = trp;
  AT->ci = tci;
  AT->val = tval;
  AT->rows = A.cols;
  AT->cols = A.rows;
  if (detach) {
    sc.detach(trp);
    sc.detach(tci);
    sc.detach(tval);
  }
  return kOk;
}

static bool prof_env() { return env_flag("APPT_PROF"); }
static int prof_level() {
  const char* e = std::getenv("APPT_PROF");
  return e && *e ? std::atoi(e) : 0;
}

// Per-phase device times in the reference's HashProf line format (include/hash_prof.h:9-28:
// "[<tag>] <phase, left-aligned in 16> <ms, %7.3f> ms", then "[<tag>] TOTAL(GPU) ..."), on
// stderr, so the reference's scripts/compare_methods.py computes TOTAL(GPU) - h2d - d2h from it.
static void print_prof(const char* tag, const CallStats& st) {
  for (int p = 0; p < 8; ++p)
    if (st.ms_phase[p] > 0.0) fprintf(stderr, "[%s] %-16s %7.3f ms\n", tag, kPhaseNames[p], st.ms_phase[p]);
  fprintf(stderr, "[%s] TOTAL(GPU)      %7.3f ms\n", tag, st.ms_total);
  for (auto& m : t_marks.marks) fprintf(stderr, "[%s-host] %9.1f us  %s\n", tag, m.second, m.first);
}

// Core call. Returns C in device memory (pool allocations) in *dc.
static int run(const MatView& A, const MatView* B, const CallOptions& opt, DeviceCtx* ctx,
               cudaStream_t s, Scratch& sc, PhaseTimer& tm, DevC* dc, CallStats* st,
               HostSink* sink) {
  int rc = check_view(A, opt.in_mem, "A");
  if (rc) return rc;
  const bool ab = opt.op == kOpAB || opt.op == kOpABUpper;
  if (opt.b_mem < 0 || opt.b_mem > 2) {
    set_error("bad b_mem");
    return kErrInvalid;
  }
  // where B lives: with A unless b_mem says otherwise (a host row block of A against a B that is
  // already resident on the device, as in multi-GPU calls)
  const int b_in = opt.b_mem == 0 ? opt.in_mem : (opt.b_mem == 1 ? 0 : 1);
  if (B && ab) {
    rc = check_view(*B, b_in, "B");
    if (rc) return rc;
  }
  Csr dA{}, dB{};
  tm.begin(kPhH2D);
  // host operands of the binned pipeline: values copied on the copy stream while the index-only
  // phases run; `vals` orders them before the numeric phase (and before anything is freed)
  struct ValuesReady {
    cudaStream_t s = nullptr;
    cudaEvent_t ev = nullptr;
    void wait() {   // make `s` wait for the values; idempotent
      if (ev) {
        cudaStreamWaitEvent(s, ev, 0);
        cudaEventSynchronize(ev);   // host buffers stay untouched once this returns
        ev = nullptr;               // (the event belongs to the device context)
      }
    }
    ~ValuesReady() { wait(); }
  } vals;
  const bool defer = opt.in_mem == 0 && ab && opt.method != kMethodEsc;
  cudaStream_t vs = defer ? ctx->copy_stream : nullptr;
  if (opt.in_mem == 0) {
    rc = stage_operand(A, sc, s, &dA, vs, ctx->ev_staged[0]);
    if (rc) return rc;
  } else {
    dA = Csr{A.rp, A.ci, A.val, (int)A.rows, (int)A.cols};
  }
  long long b_nnz = A.nnz;
  if (ab) {
    if (B) {
      if (A.cols != B->rows) {
        set_error("A.cols != B.rows");
        return kErrInvalid;
      }
      b_nnz = B->nnz;
      if (b_in == 0) {
        rc = stage_operand(*B, sc, s, &dB, vs, ctx->ev_staged[1]);
        if (rc) return rc;
      } else {
        dB = Csr{B->rp, B->ci, B->val, (int)B->rows, (int)B->cols};
      }
    } else {
      if (A.rows != A.cols) {
        set_error("C = A*A needs a square A");
        return kErrInvalid;
      }
      dB = dA;
    }
  } else {
    tm.begin(kPhTranspose);
    rc = do_transpose(ctx, dA, A.nnz, sc, s, &dB, false);
    if (rc) return rc;
    b_nnz = A.nnz;
  }
  if (A.rows + opt.row_base >= (1ll << 31) || opt.row_base < 0) {
    set_error("row_base + rows exceeds int32");
    return kErrInvalid;
  }
  const int upper = (opt.op == kOpAATUpper || opt.op == kOpABUpper) ? 1 : 0;
  if (defer) {
    vals.s = s;
    vals.ev = ctx->ev_values;
    CK(cudaEventRecord(vals.ev, vs));
  }
  return multiply_device(ctx, dA, dB, A.nnz, b_nnz, upper, (int)opt.row_base, opt.method, s, sc,
                         tm, dc, st, sink, vals.ev, opt.on_nnz);
}

// Pinned host blocks for results returned in host memory: a block released by free_out is kept
// for the next result that fits (pinning hundreds of MB costs far more than the copy into it);
// at most kPinnedCacheBytes stay cached.
static std::mutex g_pin_mu;
static std::vector<std::pair<void*, size_t>> g_pin_free;
static size_t g_pin_cached = 0;
static constexpr size_t kPinnedCacheBytes = size_t(16) << 30;
static std::vector<std::pair<void*, size_t>> g_pin_live;

static void* pinned_take(size_t bytes) {
  {
    std::lock_guard<std::mutex> g(g_pin_mu);
    int best = -1;
    for (size_t k = 0; k < g_pin_free.size(); ++k)
      if (g_pin_free[k].second >= bytes &&
          (best < 0 || g_pin_free[k].second < g_pin_free[(size_t)best].second))
        best = (int)k;
    if (best >= 0) {
      auto blk = g_pin_free[(size_t)best];
      g_pin_free.erase(g_pin_free.begin() + best);
      g_pin_cached -= blk.second;
      g_pin_live.push_back(blk);
      return blk.first;
    }
  }
  void* h = nullptr;
  if (cudaMallocHost(&h, bytes) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> g(g_pin_mu);
  g_pin_live.push_back({h, bytes});
  return h;
}

static void pinned_give_back(void* h) {
  std::lock_guard<std::mutex> g(g_pin_mu);
  size_t bytes = 0;
  for (size_t k = 0; k < g_pin_live.size(); ++k)
    if (g_pin_live[k].first == h) {
      bytes = g_pin_live[k].second;
      g_pin_live.erase(g_pin_live.begin() + (long)k);
      break;
    }
  if (bytes == 0 || g_pin_cached + bytes > kPinnedCacheBytes) {
    cudaFreeHost(h);
    return;
  }
  g_pin_free.push_back({h, bytes});
  g_pin_cached += bytes;
}

// C = op(A, B) into a host destination chosen by `sink` once nnz(C) is known. The adaptive
// pipelines fill it block by block while computing; the ESC pipeline copies at the end.
static int spgemm_to_host(const MatView& A, const MatView* B, const CallOptions& opt,
                          HostSink* sink, CallStats* st) {
  if (opt.op < 0 || opt.op > 3 || opt.method < 0 || opt.method > 3) {
    set_error("bad op or method");
    return kErrInvalid;
  }
  DeviceCtx* ctx = nullptr;
  int rc = get_ctx(opt.device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  CK(cudaSetDevice(opt.device));
  cudaStream_t s = opt.stream ? (cudaStream_t)opt.stream : ctx->stream;
  const long long launches0 = kernel_launches();
  CallStats local;
  CallStats* stp = st ? st : &local;
  *stp = CallStats();
  PhaseTimer tm;
  tm.start(opt.timing != 0 || prof_env(), s, &ctx->ev_timing);
  t_marks.start(prof_level() >= 2);
  DevC dc;
  {
    Scratch sc(ctx, s);
    rc = run(A, B, opt, ctx, s, sc, tm, &dc, stp, sink);
    if (rc == kOk && !sink->done) {
      tm.begin(kPhD2H);
      HostDst d;
      if (!sink->alloc(dc.nnz, &d)) {
        set_error("host allocation failed for C");
        rc = kErrOom;
      } else {
        if (d.rp32) {
          int* rp32 = sc.get<int>((size_t)dc.rows + 1);
          if (rp32) {
            narrow_rowptr(dc.rp, rp32, dc.rows + 1, s);
            note_launches(1);
            cudaMemcpyAsync(d.rp32, rp32, sizeof(int) * ((size_t)dc.rows + 1),
                            cudaMemcpyDeviceToHost, s);
          } else {
            rc = kErrOom;
          }
        } else {
          cudaMemcpyAsync(d.rp64, dc.rp, sizeof(long long) * ((size_t)dc.rows + 1),
                          cudaMemcpyDeviceToHost, s);
        }
        if (dc.nnz > 0) {
          cudaMemcpyAsync(d.ci, dc.ci, sizeof(int) * (size_t)dc.nnz, cudaMemcpyDeviceToHost, s);
          cudaMemcpyAsync(d.val, dc.val, sizeof(double) * (size_t)dc.nnz, cudaMemcpyDeviceToHost,
                          s);
        }
        sink->done = true;
        sink->nnz = dc.nnz;
      }
    }
    tm.end();
    if (dc.rp) {
      cudaFreeAsync(dc.rp, s);
      cudaFreeAsync(dc.ci, s);
      cudaFreeAsync(dc.val, s);
    }
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess && rc == kOk) {
      set_error(std::string("D2H of C: ") + cudaGetErrorString(e));
      rc = kErrCuda;
    }
    tm.finish(stp);   // before the scratch frees are queued (the stream is idle here)
  }
  stp->launches = kernel_launches() - launches0;
  sink->cols = dc.cols;
  if (rc == kOk) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      set_error(std::string("launch error: ") + cudaGetErrorString(e));
      rc = kErrCuda;
    }
  }
  t_marks.mark("call returns");
  if (prof_env() && rc == kOk) print_prof(opt.prof_tag, *stp);
  return rc;
}

int spgemm(const MatView& A, const MatView* B, const CallOptions& opt, MatOut* C,
           CallStats* st) {
  if (!C) {
    set_error("null output");
    return kErrInvalid;
  }
  std::memset((void*)C, 0, sizeof(*C));
  if (opt.out_mem == 0) {
    // host result: one pinned block [int64 row_ptr | col_idx | val] owned by the caller
    // (appt_free_out)
    void* block = nullptr;
    int kind = 0;
    const long long rows = A.rows;
    HostSink sink;
    sink.alloc = [&](long long nnz, HostDst* d) -> bool {
      const size_t bytes = sizeof(long long) * ((size_t)rows + 1) + sizeof(int) * (size_t)nnz +
                           sizeof(double) * (size_t)nnz + 64;
      kind = 2;
      block = pinned_take(bytes);
      if (!block) {
        block = std::malloc(bytes);
        kind = 3;
      }
      if (!block) return false;
      char* p = (char*)block;
      d->rp64 = (long long*)p;
      p += sizeof(long long) * ((size_t)rows + 1);
      d->ci = (int*)p;
      d->val = (double*)(((uintptr_t)p + sizeof(int) * (size_t)nnz + 7) & ~(uintptr_t)7);
      return true;
    };
    const int rc = spgemm_to_host(A, B, opt, &sink, st);
    if (rc != kOk) {
      if (block) {
        if (kind == 2) pinned_give_back(block);
        else std::free(block);
      }
      return rc;
    }
    char* p = (char*)block;
    C->rows = rows;
    C->cols = sink.cols;
    C->nnz = sink.nnz;
    C->rp = (long long*)p;
    p += sizeof(long long) * ((size_t)rows + 1);
    C->ci = (int*)p;
    C->val = (double*)(((uintptr_t)p + sizeof(int) * (size_t)sink.nnz + 7) & ~(uintptr_t)7);
    C->mem = 0;
    C->device = opt.device;
    C->alloc_kind = kind;
    C->base = block;
    return kOk;
  }
  if (opt.op < 0 || opt.op > 3 || opt.method < 0 || opt.method > 3) {
    set_error("bad op or method");
    return kErrInvalid;
  }
  DeviceCtx* ctx = nullptr;
  int rc = get_ctx(opt.device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  CK(cudaSetDevice(opt.device));
  cudaStream_t s = opt.stream ? (cudaStream_t)opt.stream : ctx->stream;
  const long long launches0 = kernel_launches();
  CallStats local;
  CallStats* stp = st ? st : &local;
  *stp = CallStats();
  PhaseTimer tm;
  tm.start(opt.timing != 0 || prof_env(), s, &ctx->ev_timing);
  t_marks.start(prof_level() >= 2);
  DevC dc;
  {
    Scratch sc(ctx, s);
    rc = run(A, B, opt, ctx, s, sc, tm, &dc, stp, nullptr);
    if (rc == kOk) {
      C->rp = dc.rp;
      C->ci = dc.ci;
      C->val = dc.val;
      C->mem = 1;
      C->alloc_kind = 1;
      C->base = (void*)s;   // stream the pool allocations are ordered on
    } else if (dc.rp) {
      cudaFreeAsync(dc.rp, s);
      cudaFreeAsync(dc.ci, s);
      cudaFreeAsync(dc.val, s);
    }
    // before the scratch frees are queued: the pipeline ended with a synchronisation, so the
    // closing event completes at once instead of one more round trip behind the frees
    tm.finish(stp);
  }
  stp->launches = kernel_launches() - launches0;
  if (rc == kOk) {
    C->rows = dc.rows;
    C->cols = dc.cols;
    C->nnz = dc.nnz;
    C->device = opt.device;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      set_error(std::string("launch error: ") + cudaGetErrorString(e));
      free_out(C);
      return kErrCuda;
    }
  }
  t_marks.mark("call returns");
  if (prof_env() && rc == kOk) print_prof(opt.prof_tag, *stp);
  return rc;
}

int free_out(MatOut* C) {
  if (!C) return kErrInvalid;
  switch (C->alloc_kind) {
    case 1:
      cudaSetDevice(C->device);
      cudaFreeAsync(C->rp, (cudaStream_t)C->base);
      cudaFreeAsync(C->ci, (cudaStream_t)C->base);
      cudaFreeAsync(C->val, (cudaStream_t)C->base);
      break;
    case 2:
      pinned_give_back(C->base);
      break;
    case 3:
      std::free(C->base);
      break;
    case 4:   // separate device allocations (transpose output)
      cudaSetDevice(C->device);
      cudaFree(C->rp);
      cudaFree(C->ci);
      cudaFree(C->val);
      break;
    default:
      break;
  }
  std::memset((void*)C, 0, sizeof(*C));
  return kOk;
}

// ------------------------------------------------------------------ transpose / analysis APIs
int transpose(const MatView& A, const CallOptions& opt, MatOut* AT) {
  if (!AT) return kErrInvalid;
  std::memset((void*)AT, 0, sizeof(*AT));
  int rc = check_view(A, opt.in_mem, "A");
  if (rc) return rc;
  DeviceCtx* ctx = nullptr;
  rc = get_ctx(opt.device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  CK(cudaSetDevice(opt.device));
  cudaStream_t s = opt.stream ? (cudaStream_t)opt.stream : ctx->stream;
  Scratch sc(ctx, s);
  Csr dA{};
  if (opt.in_mem == 0) {
    rc = stage_operand(A, sc, s, &dA);
    if (rc) return rc;
  } else {
    dA = Csr{A.rp, A.ci, A.val, (int)A.rows, (int)A.cols};
  }
  Csr T{};
  rc = do_transpose(ctx, dA, A.nnz, sc, s, &T, true);
  if (rc) return rc;
  // widen row pointers to int64 for the output format
  long long* rp64 = nullptr;
  CK(cudaMalloc(&rp64, sizeof(long long) * ((size_t)A.cols + 1)));
  {
    std::vector<int> tmp;   // small: cols + 1 entries
    tmp.resize((size_t)A.cols + 1);
    CK(cudaMemcpyAsync(tmp.data(), T.rp, sizeof(int) * tmp.size(), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    std::vector<long long> t64(tmp.begin(), tmp.end());
    CK(cudaMemcpy(rp64, t64.data(), sizeof(long long) * t64.size(), cudaMemcpyHostToDevice));
  }
  int* ci = nullptr;
  double* val = nullptr;
  CK(cudaMalloc(&ci, sizeof(int) * ((size_t)A.nnz + 1)));
  CK(cudaMalloc(&val, sizeof(double) * ((size_t)A.nnz + 1)));
  CK(cudaMemcpyAsync(ci, T.ci, sizeof(int) * (size_t)A.nnz, cudaMemcpyDeviceToDevice, s));
  CK(cudaMemcpyAsync(val, T.val, sizeof(double) * (size_t)A.nnz, cudaMemcpyDeviceToDevice, s));
  cudaFreeAsync((void*)T.rp, s);
  cudaFreeAsync((void*)T.ci, s);
  cudaFreeAsync((void*)T.val, s);
  CK(cudaStreamSynchronize(s));
  AT->rows = A.cols;
  AT->cols = A.rows;
  AT->nnz = A.nnz;
  AT->device = opt.device;
  if (opt.out_mem == 1) {
    AT->rp = rp64;
    AT->ci = ci;
    AT->val = val;
    AT->mem = 1;
    AT->alloc_kind = 4;
    return kOk;
  }
  const size_t bytes = sizeof(long long) * ((size_t)A.cols + 1) + (sizeof(int) + sizeof(double)) * (size_t)A.nnz + 16;
  char* h = (char*)std::malloc(bytes);
  if (!h) {
    cudaFree(rp64);
    cudaFree(ci);
    cudaFree(val);
    set_error("host allocation failed");
    return kErrOom;
  }
  AT->rp = (long long*)h;
  AT->val = (double*)(h + sizeof(long long) * ((size_t)A.cols + 1));
  AT->ci = (int*)(AT->val + A.nnz);
  CK(cudaMemcpy(AT->rp, rp64, sizeof(long long) * ((size_t)A.cols + 1), cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(AT->ci, ci, sizeof(int) * (size_t)A.nnz, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(AT->val, val, sizeof(double) * (size_t)A.nnz, cudaMemcpyDeviceToHost));
  cudaFree(rp64);
  cudaFree(ci);
  cudaFree(val);
  AT->mem = 0;
  AT->alloc_kind = 3;
  AT->base = h;
  return kOk;
}

int transpose_into(const MatView& A, const CallOptions& opt, int* t_rp, int* t_ci,
                   double* t_val) {
  if (!t_rp || (A.nnz > 0 && (!t_ci || !t_val))) {
    set_error("appt_transpose_into: null output buffer");
    return kErrInvalid;
  }
  int rc = check_view(A, opt.in_mem, "A");
  if (rc) return rc;
  DeviceCtx* ctx = nullptr;
  rc = get_ctx(opt.device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  CK(cudaSetDevice(opt.device));
  cudaStream_t s = opt.stream ? (cudaStream_t)opt.stream : ctx->stream;
  Scratch sc(ctx, s);
  Csr dA{};
  if (opt.in_mem == 0) {
    rc = stage_operand(A, sc, s, &dA);
    if (rc) return rc;
  } else {
    dA = Csr{A.rp, A.ci, A.val, (int)A.rows, (int)A.cols};
  }
  Csr T{};
  rc = do_transpose(ctx, dA, A.nnz, sc, s, &T, false);
  if (rc) return rc;
  const cudaMemcpyKind kind = opt.in_mem == 0 ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  CK(cudaMemcpyAsync(t_rp, T.rp, sizeof(int) * ((size_t)A.cols + 1), kind, s));
  if (A.nnz > 0) {
    CK(cudaMemcpyAsync(t_ci, T.ci, sizeof(int) * (size_t)A.nnz, kind, s));
    CK(cudaMemcpyAsync(t_val, T.val, sizeof(double) * (size_t)A.nnz, kind, s));
  }
  CK(cudaStreamSynchronize(s));
  return kOk;
}

int row_products(const MatView& A, const MatView* B, const CallOptions& opt, long long* out) {
  int rc = check_view(A, opt.in_mem, "A");
  if (rc) return rc;
  DeviceCtx* ctx = nullptr;
  rc = get_ctx(opt.device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  CK(cudaSetDevice(opt.device));
  cudaStream_t s = opt.stream ? (cudaStream_t)opt.stream : ctx->stream;
  Scratch sc(ctx, s);
  Csr dA{}, dB{};
  if (opt.in_mem == 0) {
    rc = stage_operand(A, sc, s, &dA);
    if (rc) return rc;
    if (B) {
      rc = stage_operand(*B, sc, s, &dB);
      if (rc) return rc;
    } else {
      dB = dA;
    }
  } else {
    dA = Csr{A.rp, A.ci, A.val, (int)A.rows, (int)A.cols};
    dB = B ? Csr{B->rp, B->ci, B->val, (int)B->rows, (int)B->cols} : dA;
  }
  const int m = (int)A.rows;
  long long* flop = sc.get<long long>(m);
  int* lo = sc.get<int>(m);
  int* hi = sc.get<int>(m);
  uint8_t* key = sc.get<uint8_t>(m);
  int* rn = sc.get<int>(m);
  AnalyzeStats* gst = sc.get<AnalyzeStats>(1);
  if (sc.failed) return kErrOom;
  CK(cudaMemsetAsync(gst, 0, sizeof(AnalyzeStats), s));
  launch_analyze(dA, dB, 0, 0, kMethodAdaptive, lanes_per_row(A.nnz, A.rows), flop, lo, hi, key,
                 rn, gst, nullptr, ctx->num_sms, s);
  note_launches(m > 0 ? 2 : 0);
  if (m > 0) CK(cudaMemcpyAsync(out, flop, sizeof(long long) * (size_t)m, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  return kOk;
}

int estimate_row_nnz(const MatView& A, int att, int estimator, const CallOptions& opt, int* out) {
  if (estimator == 0) {
    const char* e = std::getenv("EST_METHOD");
    estimator = (e && std::strcmp(e, "hll") == 0) ? 2 : 1;
  }
  if (estimator != 1 && estimator != 2) {
    set_error("unknown estimator");
    return kErrInvalid;
  }
  int rc = check_view(A, opt.in_mem, "A");
  if (rc) return rc;
  DeviceCtx* ctx = nullptr;
  rc = get_ctx(opt.device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  CK(cudaSetDevice(opt.device));
  cudaStream_t s = opt.stream ? (cudaStream_t)opt.stream : ctx->stream;
  Scratch sc(ctx, s);
  Csr dA{}, dB{};
  if (opt.in_mem == 0) {
    rc = stage_operand(A, sc, s, &dA);
    if (rc) return rc;
  } else {
    dA = Csr{A.rp, A.ci, A.val, (int)A.rows, (int)A.cols};
  }
  if (att) {
    rc = do_transpose(ctx, dA, A.nnz, sc, s, &dB, false);
    if (rc) return rc;
  } else {
    dB = dA;
  }
  const int m = (int)A.rows;
  int* est = sc.get<int>(m);
  if (sc.failed) return kErrOom;
  if (A.nnz < 100000) {
    launch_flop_count_i32(dA, dB, est, s);
    note_launches(m > 0 ? 1 : 0);
  } else if (estimator == 2) {
    unsigned char* regs = sc.get<unsigned char>((size_t)dB.rows * 128);
    if (sc.failed) return kErrOom;
    launch_hll_estimate(dA, dB, regs, est, ctx->num_sms, s);
    note_launches(2);
  } else {
    unsigned* sketch = sc.get<unsigned>((size_t)dB.rows * 128);
    if (sc.failed) return kErrOom;
    launch_minhash_estimate(dA, dB, sketch, est, ctx->num_sms, s);
    note_launches(2);
  }
  if (m > 0) CK(cudaMemcpyAsync(out, est, sizeof(int) * (size_t)m, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  return kOk;
}

int release_cached(int device) {
  DeviceCtx* ctx = nullptr;
  int rc = get_ctx(device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  CK(cudaSetDevice(device));
  CK(cudaStreamSynchronize(ctx->stream));
  CK(cudaMemPoolTrimTo(ctx->pool, 0));
  CK(cudaMemPoolTrimTo(ctx->pool_big, 0));
  return kOk;
}

double reference_score(const int* row_ptr, long long rows, long long nnz) {
  int max_row = 0;
  for (long long i = 0; i < rows; ++i) max_row = std::max(max_row, row_ptr[i + 1] - row_ptr[i]);
  const double avg = rows > 0 ? (double)nnz / (double)rows : 0.0;
  const double skew = avg > 0.0 ? (double)max_row / avg : 0.0;
  const double fp = (double)nnz * (double)nnz / (double)std::max<long long>(rows, 1);
  const double lfp = std::log10(std::max(fp, 1.0));
  const double ln = std::log10((double)rows);
  const double lmr = std::log10((double)std::max(max_row, 1));
  const double lsk = std::log10(std::max(skew, 1.0));
  return -0.4259 * lfp - 0.4215 * ln - 0.6441 * lmr - 0.6420 * lsk + 5.4297;
}

// ------------------------------------------------------------------ pools (mempool.h semantics)
bool g_mempool_on = false;
bool g_devpool_on = false;
static char* g_hbase = nullptr;
static size_t g_hcap = 0, g_hoff = 0;
static std::vector<std::pair<void*, size_t>> g_dev_live;
static size_t g_dev_used = 0;
static std::mutex g_pool_mu;

static size_t env_mb(const char* k, size_t def_mb) {
  const char* e = std::getenv(k);
  if (e && *e) {
    long v = std::atol(e);
    if (v > 0) return (size_t)v << 20;
  }
  return def_mb << 20;
}

bool pool_init(size_t cap_bytes) {
  std::lock_guard<std::mutex> g(g_pool_mu);
  if (!g_mempool_on) return true;
  if (cap_bytes == 0) cap_bytes = env_mb("MP_HOST_MB", 256);
  if (g_hbase && g_hcap >= cap_bytes) return true;
  if (g_hbase) cudaFreeHost(g_hbase);
  g_hbase = nullptr;
  g_hcap = g_hoff = 0;
  if (cudaMallocHost((void**)&g_hbase, cap_bytes) != cudaSuccess) {
    cudaGetLastError();
    g_hbase = nullptr;
    set_error("cudaMallocHost of the pinned arena failed");
    return false;
  }
  g_hcap = cap_bytes;
  return true;
}

void pool_destroy() {
  std::lock_guard<std::mutex> g(g_pool_mu);
  if (g_hbase) cudaFreeHost(g_hbase);
  g_hbase = nullptr;
  g_hcap = g_hoff = 0;
  for (auto& p : g_dev_live) cudaFreeAsync(p.first, 0);
  g_dev_live.clear();
  g_dev_used = 0;
}

int pinned_alloc_reset(void** out, size_t bytes) {
  if (!out) return (int)cudaErrorInvalidValue;
  if (!g_mempool_on) return (int)cudaMallocHost(out, bytes ? bytes : 1);
  std::lock_guard<std::mutex> g(g_pool_mu);
  if (bytes == 0) bytes = 1;
  if (!g_hbase || bytes > g_hcap) {
    // grow (the previous C is dead by contract: each call resets the arena)
    size_t cap = std::max(bytes + (bytes >> 3), env_mb("MP_HOST_MB", 256));
    if (g_hbase) cudaFreeHost(g_hbase);
    g_hbase = nullptr;
    g_hcap = 0;
    cudaError_t e = cudaMallocHost((void**)&g_hbase, cap);
    if (e != cudaSuccess) {
      g_hbase = nullptr;
      return (int)e;
    }
    g_hcap = cap;
  }
  g_hoff = bytes;
  *out = g_hbase;
  return 0;
}

void pinned_release(void* p) {
  if (!p) return;
  if (!g_mempool_on) cudaFreeHost(p);
}

void host_release(void* p) {
  if (!p) return;
  if (g_mempool_on) cudaFreeHost(p);
  else std::free(p);
}

void devarena_reset() {
  std::lock_guard<std::mutex> g(g_pool_mu);
  if (!g_devpool_on) return;
  for (auto& p : g_dev_live) cudaFreeAsync(p.first, 0);
  g_dev_live.clear();
  g_dev_used = 0;
}

void* devarena_alloc(size_t bytes) {
  if (bytes == 0) bytes = 1;
  if (!g_devpool_on) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
      cudaGetLastError();
      set_error("cudaMalloc failed in dev_alloc");
      return nullptr;
    }
    return p;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceCtx* ctx = nullptr;
  if (get_ctx(dev, &ctx)) return nullptr;
  void* p = nullptr;
  if (cudaMallocFromPoolAsync(&p, bytes, ctx->pool, 0) != cudaSuccess) {
    cudaGetLastError();
    set_error("device pool allocation failed in dev_alloc");
    return nullptr;
  }
  std::lock_guard<std::mutex> g(g_pool_mu);
  g_dev_live.push_back({p, bytes});
  g_dev_used += bytes;
  return p;
}

void devarena_free(void* p) {
  if (!p) return;
  if (!g_devpool_on) cudaFree(p);
}

size_t host_arena_cap() { return g_hcap; }
size_t host_arena_used() { return g_hoff; }
size_t devarena_used() { return g_dev_used; }

// ------------------------------------------------------------------ spgemm.h compatible flow
static inline size_t align8(size_t x) { return (x + 7) & ~(size_t)7; }

void compat_call(void* A_buffer, int A_rows, int A_cols, int A_nnz, void** C_buffer_out,
                 int* C_rows, int* C_cols, int* C_nnz, int op, int method, const char* tag,
                 bool att_quirk_cols) {
  if (C_buffer_out) *C_buffer_out = nullptr;
  if (C_nnz) *C_nnz = -1;
  if (C_rows) *C_rows = A_rows;
  if (C_cols) *C_cols = (op == kOpAB || att_quirk_cols) ? A_cols : A_rows;
  if (!A_buffer || !C_buffer_out || !C_rows || !C_cols || !C_nnz || A_rows < 0 || A_nnz < 0) {
    set_error("invalid argument");
    return;
  }
  // The adaptive entry reports its choice on stdout as the reference does
  // (src/spgemm_adaptive.cu:85, "[adapt] n=.. maxrow=.. skew=.. -> hash|merge3 (why)"); the
  // per-row tiers here are all hash-family, so the line names hash and the phase lines that
  // follow carry the reference hash path's tag, which is what the reference's scripts expect.
  if ((env_flag("APPT_VERBOSE") || prof_env()) && method == kMethodAdaptive && A_rows > 0) {
    const int* rp = (const int*)A_buffer;
    int max_row = 0;
    for (int i = 0; i < A_rows; ++i) max_row = std::max(max_row, rp[i + 1] - rp[i]);
    const double avg = (double)A_nnz / (double)A_rows;
    const double sc = reference_score(rp, A_rows, A_nnz);
    printf("[adapt] n=%d maxrow=%d skew=%.1f \u2192 hash (per-row tiers; reference rule: %s, "
           "score=%.2f)\n", A_rows, max_row, avg > 0 ? max_row / avg : 0.0,
           sc < 0 ? "hash" : "merge3", sc);
    fflush(stdout);
  }
  MatView A;
  A.rows = A_rows;
  A.cols = A_cols;
  A.nnz = A_nnz;
  A.rp = (const int*)A_buffer;
  A.ci = A.rp + (size_t)A_rows + 1;
  A.val = (const double*)((const char*)A_buffer + align8((size_t)(A_rows + 1) * 4 + (size_t)A_nnz * 4));
  CallOptions opt;
  opt.op = op;
  opt.method = method;
  opt.in_mem = 0;
  opt.out_mem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  opt.device = dev;
  const bool prof = prof_env();
  opt.timing = prof ? 1 : 0;
  // the reference's adaptive entry profiles under its hash path's tag
  opt.prof_tag = std::strcmp(tag, "adapt-prof") == 0 ? "hash-prof" : tag;
  // C goes straight into the reference's output layout in the pinned arena
  // [int32 row_ptr | pad8 | col_idx | pad8 | val], written while the numeric phase runs
  void* buf = nullptr;
  bool too_big = false;
  HostSink sink;
  sink.alloc = [&](long long nnz, HostDst* d) -> bool {
    if (nnz > 0x7fffffffll) {
      too_big = true;
      return false;
    }
    const size_t rp_al = align8((size_t)(A_rows + 1) * 4);
    const size_t ci_al = align8((size_t)nnz * 4);
    if (pinned_alloc_reset(&buf, rp_al + ci_al + (size_t)nnz * 8) != 0 || !buf) {
      buf = nullptr;
      return false;
    }
    d->rp32 = (int*)buf;
    d->ci = (int*)((char*)buf + rp_al);
    d->val = (double*)((char*)buf + rp_al + ci_al);
    return true;
  };
  CallStats st;
  const int rc = spgemm_to_host(A, nullptr, opt, &sink, &st);
  if (rc != kOk) {
    if (too_big) set_error("nnz(C) exceeds int32; use appt_spgemm");
    fprintf(stderr, "[appt] %s failed: %s\n", tag, last_error());
    if (buf) pinned_release(buf);
    return;
  }
  *C_buffer_out = buf;
  *C_nnz = (int)sink.nnz;
}

void compat_build_csc(const int* d_row_ptr, const int* d_col_idx, const double* d_val, int A_rows,
                      int A_nnz, int** col_ptr_out, int** row_idx_out, double** val_out) {
  if (col_ptr_out) *col_ptr_out = nullptr;
  if (row_idx_out) *row_idx_out = nullptr;
  if (val_out) *val_out = nullptr;
  if (!col_ptr_out || !row_idx_out || !val_out || A_rows < 0 || A_nnz < 0) return;
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceCtx* ctx = nullptr;
  if (get_ctx(dev, &ctx)) return;
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaStream_t s = ctx->stream;
  int *cp = nullptr, *ri = nullptr;
  double* v = nullptr;
  if (cudaMalloc(&cp, sizeof(int) * ((size_t)A_rows + 1)) != cudaSuccess ||
      cudaMalloc(&ri, sizeof(int) * ((size_t)A_nnz + 1)) != cudaSuccess ||
      cudaMalloc(&v, sizeof(double) * ((size_t)A_nnz + 1)) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(cp);
    cudaFree(ri);
    cudaFree(v);
    set_error("cudaMalloc failed in build_csc");
    return;
  }
  {
    Scratch sc(ctx, s);
    void* tscr = sc.get<char>(transpose_scratch_bytes(A_rows, A_rows, A_nnz));
    if (sc.failed) {
      cudaFree(cp);
      cudaFree(ri);
      cudaFree(v);
      set_error("pool allocation failed in build_csc");
      return;
    }
    Csr A{d_row_ptr, d_col_idx, d_val, A_rows, A_rows};
    launch_transpose(A, A_nnz, cp, ri, v, tscr, ctx->num_sms, s);
    note_launches(16);
  }
  if (cudaStreamSynchronize(s) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(cp);
    cudaFree(ri);
    cudaFree(v);
    set_error("build_csc failed");
    return;
  }
  *col_ptr_out = cp;
  *row_idx_out = ri;
  *val_out = v;
}

bool compat_should_run_method(const char* key) {
  const char* m = std::getenv("METHOD");
  if (!m || !*m || !std::strcmp(m, "all")) return true;
  if (!key) return false;
  for (int i = 0;; ++i) {
    char a = m[i], b = key[i];
    if (a >= 'A' && a <= 'Z') a += 32;
    if (b >= 'A' && b <= 'Z') b += 32;
    if (a != b) return false;
    if (a == 0) return true;
  }
}

}  // namespace appt
