// appt_spgemm_noalloc: C = A*B for device-resident operands, written into buffers the caller
// owns, without allocating any memory.
//
// Who needs this: callers that must not call cudaMalloc (or any other allocator) from inside
// the multiply -- for example a framework whose caching allocator owns the whole device heap,
// code running inside a region where the CUDA allocator is forbidden, or real-time loops that
// pre-size every buffer at start-up. Everything the pipeline needs beyond the caller's inputs
// and outputs lives in one fixed, file-scope device array (kNoAllocScratchBytes, 64 MiB). The
// array exists on every GPU where this library is loaded, for the life of the process.
//
// Protocol: the caller passes C_row_ptr (rows + 1 int64) and C_col_idx / C_val with room for
// C_capacity entries. The call always fills C_row_ptr and *C_nnz_out; when nnz(C) exceeds
// C_capacity it returns APPT_ERR_TOO_LARGE before the numeric phase, so the caller can size its
// buffers and call again. A has at most noalloc_max_rows() rows (the scratch holds about 30
// bytes per row of A); larger A is rejected with APPT_ERR_TOO_LARGE and a message.
//
// The first call on a device looks up the device address of the scratch array
// (cudaGetSymbolAddress, with that device current) and caches it. Every call uses the same array and leaves its contents there; everything
// a call relies on being zero it clears itself. Calls whose GPU work overlapped would race on the
// array: this function serialises its callers per device on the host and returns only after its
// own GPU work has finished, so calls made through it do not overlap. Each call blocks its host
// thread: it reads nnz(C) back in the middle (a stream synchronisation) and synchronises the
// stream again before it returns.
// This entry point has no counterpart in the reference.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/appt_spgemm.h"
#include "engine.h"
#include "kernels.cuh"

namespace appt {
namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu[64];
void* g_noalloc_ptr[64] = {nullptr};

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Byte layout of the scratch for an A with m rows (all offsets 256-byte aligned).
struct Layout {
  size_t flop, lo, hi, symkey, numkey, row_nnz, rows_sym, rows_num, boff_sym, boff_num, stats, err,
      scan, part, total;
};

Layout layout_for(long long m) {
  Layout L{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += align256(bytes ? bytes : 1);
    return at;
  };
  L.flop = take(8 * (size_t)m);
  L.lo = take(4 * (size_t)m);
  L.hi = take(4 * (size_t)m);
  L.symkey = take((size_t)m);
  L.numkey = take((size_t)m);
  L.row_nnz = take(4 * (size_t)m);
  L.rows_sym = take(4 * (size_t)m);
  L.rows_num = take(4 * (size_t)m);
  L.boff_sym = take(8 * (kMaxBins + 1));
  L.boff_num = take(8 * (kMaxBins + 1));
  L.stats = take(sizeof(AnalyzeStats));
  L.err = take((4 + kMaxBins) * sizeof(int));   // error word, counters (symbolic CTA tier at
                                                 // [3], numeric CTA tiers at [4 + bin])
  L.scan = take(8 * scan_scratch_elems(m));
  L.part = take(partition_scratch_bytes((int)m, kMaxBins));
  L.total = o;
  return L;
}

}  // namespace

long long noalloc_max_rows() {
  long long lo = 0, hi = 1ll << 31;
  while (lo < hi) {   // largest m whose layout fits the array
    const long long mid = (lo + hi + 1) / 2;
    if (layout_for(mid).total <= kNoAllocScratchBytes) lo = mid; else hi = mid - 1;
  }
  return lo;
}

int spgemm_noalloc(const MatView& A, const MatView* Bp, long long* crp, int* cci, double* cval,
                   long long capacity, long long* nnz_out, void* stream) {
  if (nnz_out) *nnz_out = -1;
  if (!crp || !nnz_out || capacity < 0 || (capacity > 0 && (!cci || !cval))) {
    set_error("appt_spgemm_noalloc: null output buffer or negative capacity");
    return kErrInvalid;
  }
  // every size is narrowed to int32 for the kernels: reject what does not fit
  auto fits = [](long long x) { return x >= 0 && x < (1ll << 31) - 1; };
  if (!fits(A.rows) || !fits(A.cols) || !fits(A.nnz) || !A.rp ||
      (A.nnz > 0 && (!A.ci || !A.val))) {
    set_error("appt_spgemm_noalloc: invalid A (sizes must lie in [0, 2^31 - 1), pointers set)");
    return kErrInvalid;
  }
  const MatView B = Bp ? *Bp : A;
  if (!Bp && A.rows != A.cols) {
    set_error("appt_spgemm_noalloc: C = A*A needs a square A");
    return kErrInvalid;
  }
  if (!fits(B.rows) || !fits(B.cols) || !fits(B.nnz) || !B.rp ||
      (B.nnz > 0 && (!B.ci || !B.val))) {
    set_error("appt_spgemm_noalloc: invalid B (sizes must lie in [0, 2^31 - 1), pointers set)");
    return kErrInvalid;
  }
  if (A.cols != B.rows) {
    set_error("appt_spgemm_noalloc: A.cols != B.rows");
    return kErrInvalid;
  }
  const long long max_rows = noalloc_max_rows();
  if (A.rows > max_rows) {
    set_error("appt_spgemm_noalloc: A has " + std::to_string(A.rows) +
              " rows; the fixed scratch array (64 MiB) holds at most " +
              std::to_string(max_rows) + " rows");
    return kErrTooLarge;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_error(std::string("appt_spgemm_noalloc: no current device: ") + cudaGetErrorString(e));
    return e == cudaSuccess ? kErrInvalid : kErrNoDevice;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu[dev]);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error(std::string("appt_spgemm_noalloc: cudaGetSymbolAddress: ") +
                cudaGetErrorString(e));
      return kErrCuda;
    }
    g_noalloc_ptr[dev] = p;
  }
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) {
    set_error(std::string("appt_spgemm_noalloc: ") + cudaGetErrorString(e));
    return kErrCuda;
  }
  cudaStream_t s = (cudaStream_t)stream;
  const int m = (int)A.rows;
  const Layout L = layout_for(m);
  char* base = (char*)g_noalloc_ptr[dev];
  long long* flop = (long long*)(base + L.flop);
  int* lo = (int*)(base + L.lo);
  int* hi = (int*)(base + L.hi);
  uint8_t* symkey = (uint8_t*)(base + L.symkey);
  uint8_t* numkey = (uint8_t*)(base + L.numkey);
  int* row_nnz = (int*)(base + L.row_nnz);
  int* rows_sym = (int*)(base + L.rows_sym);
  int* rows_num = (int*)(base + L.rows_num);
  long long* boff_sym = (long long*)(base + L.boff_sym);
  long long* boff_num = (long long*)(base + L.boff_num);
  AnalyzeStats* gst = (AnalyzeStats*)(base + L.stats);
  int* err = (int*)(base + L.err);
  long long* scs = (long long*)(base + L.scan);
  void* pscr = base + L.part;
  const Csr dA{A.rp, A.ci, A.val, (int)A.rows, (int)A.cols};
  const Csr dB{B.rp, B.ci, B.val, (int)B.rows, (int)B.cols};

  // the previous call's contents stay in the array: clear what must start at zero
  cudaMemsetAsync(gst, 0, sizeof(AnalyzeStats), s);
  cudaMemsetAsync(err, 0, (4 + kMaxBins) * sizeof(int), s);
  const int lpr = analyze_lanes_per_row(A.nnz, m);
  launch_analyze(dA, dB, 0, 0, kMethodAdaptive, lpr, flop, lo, hi, symkey, row_nnz, gst, err, sms,
                 s);
  long long launched = m > 0 ? 3 : 0;   // analyze (two kernels), classify
  launched += partition_rows(symkey, m, kNumSymBins + 1, rows_sym, boff_sym, pscr, s);
  if (m > 0)
    for (int b = 0; b < kNumSymBins; ++b)
      launch_symbolic(b, rows_sym, boff_sym, dA, dB, 0, 0, lo, hi, flop, row_nnz, RowBitmaps{},
                      DenseRows{}, err + 3, err, sms, s);
  if (m > 0) launched += kNumSymBins;
  launched += scan_exclusive(row_nnz, crp, m, scs, s);
  launch_classify_numeric(dA, m, kMethodAdaptive, flop, lo, hi, row_nnz, numkey, sms, s);
  launched += partition_rows(numkey, m, kNumNumBins, rows_num, boff_num, pscr, s);
  note_launches(launched);
  // A launch that failed left the array holding the previous call's row counts and bin lists:
  // stop before anything is read back from it.
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("appt_spgemm_noalloc: launch failed: ") + cudaGetErrorString(e));
    return kErrCuda;
  }

  long long nnz = 0;
  long long boff[kNumNumBins + 1];
  int herr = 0;
  e = cudaMemcpyAsync(&nnz, crp + m, sizeof(long long), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(boff, boff_num, sizeof(boff), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_error(std::string("appt_spgemm_noalloc: ") + cudaGetErrorString(e));
    return kErrCuda;
  }
  if (herr & kErrBounds) {
    set_error("appt_spgemm_noalloc: operand index out of range (A column >= B rows)");
    return kErrInvalid;
  }
  if (herr) {
    set_error("appt_spgemm_noalloc: symbolic phase reported device error bits " +
              std::to_string(herr));
    return kErrDevice;
  }
  *nnz_out = nnz;
  if (nnz > capacity) {
    set_error("appt_spgemm_noalloc: nnz(C) = " + std::to_string(nnz) +
              " exceeds the capacity of C_col_idx / C_val (" + std::to_string(capacity) +
              "); C_row_ptr and *C_nnz_out are filled");
    return kErrTooLarge;
  }
  for (int b = 0; b < kNumNumBins; ++b) {
    const long long nr = boff[b + 1] - boff[b];
    if (nr <= 0) continue;
    launch_numeric(b, rows_num, boff_num, nr, dA, dB, 0, 0, lo, hi, flop, RowBitmaps{},
                   DenseRows{}, crp, cci, cval, err + 4 + b, err, sms, s);
    note_launches(1);
  }
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_error(std::string("appt_spgemm_noalloc: ") + cudaGetErrorString(e));
    return kErrCuda;
  }
  if (herr) {
    set_error("appt_spgemm_noalloc: numeric phase reported device error bits " +
              std::to_string(herr));
    return kErrDevice;
  }
  return kOk;
}

}  // namespace appt

extern "C" int appt_spgemm_noalloc(const appt_csr* A, const appt_csr* B, int64_t* C_row_ptr,
                                   int32_t* C_col_idx, double* C_val, int64_t C_capacity,
                                   int64_t* C_nnz_out, void* stream) {
  if (!A) {
    appt::set_error("appt_spgemm_noalloc: null A");
    return APPT_ERR_INVALID;
  }
  appt::MatView a, b;
  a.rows = A->rows;
  a.cols = A->cols;
  a.nnz = A->nnz;
  a.rp = A->row_ptr;
  a.ci = A->col_idx;
  a.val = A->val;
  if (B) {
    b.rows = B->rows;
    b.cols = B->cols;
    b.nnz = B->nnz;
    b.rp = B->row_ptr;
    b.ci = B->col_idx;
    b.val = B->val;
  }
  return appt::spgemm_noalloc(a, B ? &b : nullptr, reinterpret_cast<long long*>(C_row_ptr),
                              C_col_idx, C_val, C_capacity,
                              reinterpret_cast<long long*>(C_nnz_out), stream);
}
