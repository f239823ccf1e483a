// Host-side launchers for the engine's kernels. Every launcher is asynchronous on `s`.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "common.cuh"

namespace appt {

constexpr int kMaxBins = 32;

// Capacities shared by the classifier and the kernels.
constexpr int kWindowCols = 16384;      // CTA window tier: window scale of the classifier's cost
                                        // model (the kernel itself walks 8192-column windows)
constexpr int kWindowSplit = 1536;      // CTA window tier: per-row table of B-row window bounds
constexpr int kHashBlockSlots = 8192;   // CTA hash tier: table slots (rows with nnz <= slots/2)
constexpr int kSymBlockWords = 32768;   // CTA symbolic bitmap window: 2^20 columns
constexpr int kMergeMaxLists = 256;     // merge tier: rows with more A entries use other tiers
constexpr int kRankMaxBudget = 9216;    // largest per-warp shared budget of the rank tier (bytes)

// Column bitmaps that the symbolic bitmap tier hands to the rank tier of the numeric phase, so
// that the numeric phase need not walk the products twice. The bitmaps live in one arena of
// `capacity` words; each warp of the symbolic kernel takes chunks of it with one atomic on `top`
// and places its rows' bitmaps there (logical word order). slot[i] = first word of row i's bitmap
// / 32, or -1 (no bitmap: the arena was full, the row does not qualify, or it ran in another
// tier). Only rows that could fit the rank tier and whose products outweigh their bitmap
// (handoff_pays) are handed off. data == nullptr: no handoff at all.
struct RowBitmaps {
  int* slot = nullptr;
  unsigned* data = nullptr;
  unsigned long long* top = nullptr;
  long long capacity = 0;
};

constexpr int kHandoffChunkWords = 16384;          // arena words a warp takes at a time
constexpr long long kHandoffArenaWords = 1ll << 28;  // arena size (1 GiB)

__host__ __device__ __forceinline__ bool handoff_fits_rank(int bitmap_words) {
  return 6ll * bitmap_words + 20 <= kRankMaxBudget;
}

// The handoff replaces the numeric phase's pass over the row's products (about flop / 32 warp
// steps of loads and shared atomics) by a copy of the row's W bitmap words (about W / 32
// coalesced steps, written once by the symbolic phase); it pays unless the span is much wider
// than the products.
__host__ __device__ __forceinline__ bool handoff_pays(long long flop, long long words) {
  return 3 * flop >= words;
}

// B rows kept a second time as column bitmaps -- rows with at least one entry per 32 columns of
// B -- so that the CTA walks OR whole words of a window from them instead of one bit per entry.
// id == nullptr: none.
// Each kept row also has the exclusive popcount prefix of its words, so the entries of a column
// range are found in O(1): rank(c) = pre[c / 32] + popc(bits[c / 32] & below(c % 32)). Rows are
// `stride` = ceil(B.cols / 32) + 1 words apart (the extra word makes rank(B.cols) valid).
struct DenseRows {
  const int* id = nullptr;          // [B.rows] index of the row's bitmap, -1 when it has none
  const unsigned* bits = nullptr;   // [rows kept][stride]
  const unsigned* pre = nullptr;    // [rows kept][stride]
  long long stride = 0;
};

// The CTA tiers with window spans beyond the warp tiers' 4096 words use them, so they are built
// only when B is that wide, and only when B's rows average enough entries for some row to
// qualify often enough to pay for the build.
constexpr long long kDenseRowsMinCols = 32ll * 4096;
constexpr long long kDenseRowsMinAvg = 64;
constexpr long long kDenseRowsMaxWords = 1ll << 27;   // 512 MB of bitmaps and prefixes at most

// Lane groups of the warp walks (walk.cuh): a row whose B rows average <= 8 entries is walked by
// 4 groups of 8 lanes, <= 16 by 2 groups of 16, longer by the whole warp. Tiers that walk
// k-sequentially come in one bin per group count (index 0, 1, 2 for G = 1, 2, 4).
__host__ __device__ __forceinline__ int group_index(long long flop, long long rowlen) {
  const long long avg = rowlen > 0 ? flop / rowlen : 32;
  return avg <= 8 ? 2 : avg <= 16 ? 1 : 0;
}

// ---- symbolic bins (chosen per row from products count and column span) ----
enum SymBin : int {
  kSymBmS = 0,     // warp per row, bitmap over the span, <= 256 words   (k-sequential), x3 G
  kSymBmM = 3,     //                                      <= 1024 words
  kSymBmL = 6,     //                                      <= 4096 words
  kSymHashS = 9,   // warp per row, key hash of 256 / 1024 / 4096 slots (wide spans)
  kSymHashM,
  kSymHashL,
  kSymBlock,       // CTA per row, 2^20-column bitmap windows (any row)
  kNumSymBins      // (index kNumSymBins itself is the merge-count bin of the merge method)
};

// ---- numeric bins (chosen per row from exact nnz, products count and span) ----
enum NumBin : int {
  kNumRank2K = 0,  // warp per row, bitmap-rank accumulator in 2 / 4 / 8 KB of shared memory,
  kNumRank4K = 3,  // each x3 lane-group counts
  kNumRank8K = 6,
  kNumHash64 = 9,  // warp per row, hash tables of 64 .. 1024 slots + in-smem sort
  kNumHash128,
  kNumHash256,
  kNumHash512,
  kNumHash1024,
  kNumHashBlock,   // CTA per row, 8192-slot table
  kNumWindow,      // CTA per row, dense windows of 16384 columns (long rows, >= 1 entry / 4 cols)
  kNumBlockRank,   // CTA per row, bitmap rank over 2^20-column windows, sums in C (long rows)
  kNumMerge,       // warp per row, k-way merge of the row's B rows (merge method)
  kNumNumBins
};

// Method selector shared by the C-ABI and the dispatcher.
enum Method : int {
  kMethodAdaptive = 0,   // per-row choice (rank / hash / window)
  kMethodHash = 1,       // hash tiers only (window tier for rows beyond smem)
  kMethodMerge = 2,      // k-way merge tier for every row
  kMethodEsc = 3,        // expand - sort - compress baseline
};

struct AnalyzeStats {          // device-side global statistics (atomics)
  unsigned long long total_flop;
  unsigned long long max_flop;
  unsigned long long max_span;
  unsigned long long pad;
};

// util.cu
// Raises the dynamic shared-memory limit of kernel `kern` to `bytes` on the current device.
// The attribute belongs to the device that is current when it is set, so it is applied once
// per (kernel, device) -- and again if a launch asks for more -- under a mutex (callers on
// several host threads or devices are safe).
void smem_opt_in(const void* kern, size_t bytes);
size_t scan_scratch_elems(long long n);
// scans and partitions return the number of kernels they launched
int scan_exclusive(const int* in, long long* out, long long n, long long* scratch, cudaStream_t s);
int scan_exclusive(const long long* in, long long* out, long long n, long long* scratch,
                    cudaStream_t s);
size_t partition_scratch_bytes(int m, int nb);
int partition_rows(const uint8_t* key, int m, int nb, int* out_rows, long long* bin_off,
                    void* scratch, cudaStream_t s);
void narrow_rowptr(const long long* in, int* out, long long n, cudaStream_t s);
// Per-bin positions of the K row blocks [k*m/K, (k+1)*m/K) in the bins' row lists:
// sub[b * (K + 1) + k], k = 0 .. K.
void block_bin_bounds(const int* rows, const long long* bin_off, int nb, long long m, int K,
                      long long* sub, cudaStream_t s);
void iota(int* out, int n, cudaStream_t s);
// Small device values read back at a synchronisation point: one kernel copies them (4-byte
// words, sources 4-byte aligned) into a pinned host buffer, in list order, instead of one
// device-to-host copy per value.
struct Readback {
  static constexpr int kMax = 16;
  const void* src[kMax];
  int words[kMax];
  int n = 0;
  // appends `bytes` (a multiple of 4) from src; returns the byte offset in the host buffer
  int add(const void* p, int bytes) {
    int off = 0;
    for (int i = 0; i < n; ++i) off += 4 * words[i];
    src[n] = p;
    words[n] = bytes / 4;
    ++n;
    return off;
  }
};
void launch_readback(const Readback& r, void* pinned_dst, cudaStream_t s);

// analyze.cu
// Lanes per row of the analysis of short rows (rows beyond 32 x that many entries take a CTA).
inline int analyze_lanes_per_row(long long nnz, long long rows) {
  const double avg = rows > 0 ? (double)nnz / (double)rows : 0.0;
  if (avg <= 32) return 4;
  if (avg <= 64) return 8;
  if (avg <= 128) return 16;
  return 32;
}
// Launches two kernels (short rows by lane groups, long rows by CTAs).
void launch_analyze(Csr A, Csr B, int upper, int row_base, int method, int lanes_per_row,
                    long long* flop, int* lo, int* hi, uint8_t* symkey, int* row_nnz,
                    AnalyzeStats* stats, int* err, int num_sms, cudaStream_t s);
void launch_classify_numeric(Csr A, int m, int method, const long long* flop, const int* lo,
                             const int* hi, const int* row_nnz, uint8_t* numkey, int num_sms,
                             cudaStream_t s);

// symbolic.cu
// row_counter: a zeroed int (the CTA tier takes rows from it dynamically)
void launch_symbolic(int bin, const int* rows, const long long* bin_off, Csr A, Csr B, int upper,
                     int row_base, const int* lo, const int* hi, const long long* flop,
                     int* row_nnz, RowBitmaps handoff, DenseRows dense, int* row_counter,
                     int* err, int num_sms, cudaStream_t s);
// Bitmaps and prefixes of B's dense rows (at most max_rows of them; counter: a zeroed int).
// Returns the number of kernels launched.
int build_dense_rows(Csr B, int* id, int* list, unsigned* bits, unsigned* pre, long long stride,
                     int max_rows, int* counter, int num_sms, cudaStream_t s);

// Small problems (symbolic.cu / numeric.cu): one unbinned symbolic pass over all rows, then the
// 9 KB rank tier over all rows; kErrSmallFallback means some row does not fit (run the general
// pipeline instead). bin_off: 2 int64, set to {0, m} by the symbolic pass.
void launch_symbolic_small(Csr A, Csr B, int upper, int row_base, int gidx, int* lo, int* hi,
                           int* row_nnz, long long* bin_off, unsigned long long* total_flop,
                           int* err, int num_sms, cudaStream_t s);
// max_need: the largest per-row rank-tier budget in bytes (the symbolic pass leaves it in err[1]);
// the launch uses the smallest budget (2304, 4608 or 9216 bytes per warp) that covers it.
void launch_numeric_rank_all(const long long* bin_off, long long m, int gidx, int max_need,
                             Csr A, Csr B, const int* lo, const int* hi, const long long* crp,
                             int* cci, double* cval, int* err, int num_sms, cudaStream_t s);

// numeric.cu
// row_counter: a zeroed int (the CTA tiers take rows from it dynamically)
void launch_numeric(int bin, const int* rows, const long long* bin_off, long long nrows_host,
                    Csr A, Csr B, int upper, int row_base, const int* lo, const int* hi,
                    const long long* flop, RowBitmaps handoff, DenseRows dense,
                    const long long* crp, int* cci, double* cval, int* row_counter, int* err,
                    int num_sms, cudaStream_t s);

// merge.cu
void launch_merge_count(const int* rows, const long long* bin_off, int bin, Csr A, Csr B,
                        int upper, int row_base, int* row_nnz, int* err, int num_sms,
                        cudaStream_t s);
void launch_merge_numeric(const int* rows, const long long* bin_off, int bin, long long nrows,
                          Csr A, Csr B, int upper, int row_base, const long long* crp, int* cci,
                          double* cval, int* err, int num_sms, cudaStream_t s);

// segsort.cu
size_t segsort_scratch_bytes(int nseg);
void segsort(int* keys, double* vals, int* keys_alt, double* vals_alt, const long long* off,
             int nseg, void* scratch, int num_sms, cudaStream_t s);

// esc_transpose.cu
void launch_esc_expand(Csr A, Csr B, int upper, int row_base, const long long* foff, int* keys,
                       double* vals, int num_sms, cudaStream_t s);
void launch_esc_count(int m, const long long* foff, const int* keys, int* row_nnz, int num_sms,
                      cudaStream_t s);
void launch_esc_compress(int m, const long long* foff, const int* keys, const double* vals,
                         const long long* crp, int* cci, double* cval, int num_sms,
                         cudaStream_t s);
size_t transpose_scratch_bytes(int rows, int cols, long long nnz);
void launch_transpose(Csr A, long long nnz, int* t_rp, int* t_ci, double* t_val, void* scratch,
                      int num_sms, cudaStream_t s);

// minhash.cu
void launch_minhash_estimate(Csr A, Csr B, unsigned* sketch, int* est, int num_sms,
                             cudaStream_t s);
void launch_hll_estimate(Csr A, Csr B, unsigned char* regs, int* est, int num_sms,
                         cudaStream_t s);
void launch_flop_count_i32(Csr A, Csr B, int* out, cudaStream_t s);

}  // namespace appt
