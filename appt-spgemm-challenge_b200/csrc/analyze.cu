// Row analysis: exact intermediate-product count per row, the row's reachable column span,
// and the symbolic / numeric bin of every row.
//
// Reference counterparts: count_intermediates_kernel / count_intermediates_par_kernel
// (spgemm_kernel_manual.cu:121-133, spgemm_kernel_hash.cu:33-55) for the product count and
// compute_bucket_kernel (spgemm_kernel_hash.cu:725-740) for the bin choice. The reference bins
// by a sketch estimate; here the symbolic phase is exact, so bins use the exact products count
// (an upper bound on distinct columns) and the column span [lo, hi] -- the first and last
// column of every B row the A row reaches (B rows are sorted, so two loads per A entry).
#include <climits>
#include "common.cuh"
#include "kernels.cuh"
#include "walk.cuh"

namespace appt {

namespace {

constexpr int kAnThreads = 256;

__device__ __forceinline__ int sym_bin_of(long long flop, long long span, long long rowlen) {
  if (flop == 0 || span <= 0) return 255;
  const long long W = span <= (1ll << 20) ? bitmap_words(span) : 1ll << 40;
  if (W <= 4096 && W <= 8 * flop + 64) {       // bitmap: clearing/counting W words pays off
    if (W <= 256) return kSymBmS + group_index(flop, rowlen);
    if (W <= 1024) return kSymBmM + group_index(flop, rowlen);
    return kSymBmL + group_index(flop, rowlen);
  }
  if (flop <= (1ll << 26)) {
    if (2 * flop <= 256) return kSymHashS;
    if (2 * flop <= 1024) return kSymHashM;
    if (2 * flop <= 4096) return kSymHashL;
  }
  return kSymBlock;
}

// Outputs of one analysed row: products count, span, symbolic bin (255: nothing to compute).
__device__ __forceinline__ void finish_row(long long row, int upper, int row_base, int method,
                                           long long f, int lo, int hi, int bad, int rowlen,
                                           long long* flop, int* lo_out, int* hi_out,
                                           uint8_t* symkey, int* row_nnz, int* err,
                                           long long* span_out) {
  const int ig = (int)row + row_base;
  if (upper && lo < ig) lo = ig;
  const long long span = (hi >= lo) ? (long long)hi - lo + 1 : 0;
  flop[row] = f;
  lo_out[row] = lo;
  hi_out[row] = hi;
  int key;
  if (bad) {
    key = 255;
    set_error(err, kErrBounds);
  } else if (method == kMethodMerge && rowlen <= kMergeMaxLists) {
    key = (f > 0 && span > 0) ? kNumSymBins : 255;   // the merge-count bin
  } else {
    key = sym_bin_of(f, span, rowlen);
  }
  symkey[row] = (uint8_t)key;
  if (key == 255) row_nnz[row] = 0;
  *span_out = span;
}

// Products count and span contributions of entries [p0, re) of a row, every `step`-th entry.
__device__ __forceinline__ void scan_entries(const Csr& A, const Csr& B, int p0, int re, int step,
                                             long long& f, int& lo, int& hi, int& bad) {
#pragma unroll 4
  for (int p = p0; p < re; p += step) {
    const int k = A.ci[p];
    if ((unsigned)k >= (unsigned)B.rows) {   // column outside B: flag, never dereference
      bad = 1;
      continue;
    }
    const int b0 = B.rp[k], b1 = B.rp[k + 1];
    if (b1 > b0) {
      f += b1 - b0;
      lo = min(lo, B.ci[b0]);
      hi = max(hi, B.ci[b1 - 1]);
    }
  }
}

// LPR lanes cooperate on one row; 32/LPR rows per warp per step. Rows longer than 32 * LPR
// entries are left to analyze_long_kernel (a CTA per row), so that one long row does not hold
// its warp for thousands of dependent steps.
template <int LPR>
__global__ void __launch_bounds__(kAnThreads) analyze_kernel(Csr A, Csr B, int upper, int row_base,
                                                             int method, long long* flop, int* lo_out,
                                                             int* hi_out, uint8_t* symkey,
                                                             int* row_nnz,
                                                             AnalyzeStats* stats, int* err) {
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR, grp = lane / LPR;
  const long long warps_total = (long long)gridDim.x * (kAnThreads / 32);
  const long long gw = (long long)blockIdx.x * (kAnThreads / 32) + (threadIdx.x >> 5);
  const int m = A.rows;
  unsigned long long my_flop_sum = 0, my_flop_max = 0, my_span_max = 0;
  for (long long base = gw * RPW; base < m; base += warps_total * RPW) {
    const long long row = base + grp;
    long long f = 0;
    int lo = INT_MAX, hi = -1;
    int bad = 0;
    int rowlen = 0;
    bool valid = row < m;
    if (valid) {
      const int rs = A.rp[row], re = A.rp[row + 1];
      rowlen = re - rs;
      if (rowlen > 32 * LPR)
        valid = false;   // a long row
      else
        scan_entries(A, B, rs + sub, re, LPR, f, lo, hi, bad);
    }
#pragma unroll
    for (int o = 1; o < LPR; o <<= 1) {
      f += __shfl_xor_sync(kFull, f, o);
      bad |= __shfl_xor_sync(kFull, bad, o);
      lo = min(lo, __shfl_xor_sync(kFull, lo, o));
      hi = max(hi, __shfl_xor_sync(kFull, hi, o));
    }
    if (valid && sub == 0) {
      long long span;
      finish_row(row, upper, row_base, method, f, lo, hi, bad, rowlen, flop, lo_out, hi_out,
                 symkey, row_nnz, err, &span);
      my_flop_sum += (unsigned long long)f;
      my_flop_max = max(my_flop_max, (unsigned long long)f);
      my_span_max = max(my_span_max, (unsigned long long)span);
    }
  }
  // block reduce of the statistics, one atomic per block
  __shared__ unsigned long long red[3][kAnThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    my_flop_sum += __shfl_xor_sync(kFull, my_flop_sum, o);
    my_flop_max = max(my_flop_max, __shfl_xor_sync(kFull, my_flop_max, o));
    my_span_max = max(my_span_max, __shfl_xor_sync(kFull, my_span_max, o));
  }
  if (lane == 0) {
    red[0][threadIdx.x >> 5] = my_flop_sum;
    red[1][threadIdx.x >> 5] = my_flop_max;
    red[2][threadIdx.x >> 5] = my_span_max;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s = 0, mf = 0, ms = 0;
    for (int w = 0; w < kAnThreads / 32; ++w) {
      s += red[0][w];
      mf = max(mf, red[1][w]);
      ms = max(ms, red[2][w]);
    }
    if (s) atomicAdd(&stats->total_flop, s);
    if (mf) atomicMax(&stats->max_flop, mf);
    if (ms) atomicMax(&stats->max_span, ms);
  }
}

// The rows analyze_kernel<LPR> leaves (more than `min_len` entries): each CTA checks a chunk of
// kAnThreads rows, lists its long ones in shared memory and walks each with all its threads.
__global__ void __launch_bounds__(kAnThreads) analyze_long_kernel(
    Csr A, Csr B, int upper, int row_base, int method, int min_len, long long* flop,
    int* lo_out, int* hi_out, uint8_t* symkey, int* row_nnz, AnalyzeStats* stats, int* err) {
  __shared__ int s_list[kAnThreads];
  __shared__ int s_n;
  __shared__ long long s_f[kAnThreads / 32];
  __shared__ int s_lo[kAnThreads / 32], s_hi[kAnThreads / 32], s_bad[kAnThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m = A.rows;
  for (long long c0 = (long long)blockIdx.x * kAnThreads; c0 < m;
       c0 += (long long)gridDim.x * kAnThreads) {
    if (tid == 0) s_n = 0;
    __syncthreads();
    const long long row = c0 + tid;
    if (row < m && A.rp[row + 1] - A.rp[row] > min_len) s_list[atomicAdd(&s_n, 1)] = (int)row;
    __syncthreads();
    const int n = s_n;
    for (int t = 0; t < n; ++t) {
      const int r = s_list[t];
      const int rs = A.rp[r], re = A.rp[r + 1];
      long long f = 0;
      int lo = INT_MAX, hi = -1, bad = 0;
      scan_entries(A, B, rs + tid, re, kAnThreads, f, lo, hi, bad);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        f += __shfl_xor_sync(kFull, f, o);
        bad |= __shfl_xor_sync(kFull, bad, o);
        lo = min(lo, __shfl_xor_sync(kFull, lo, o));
        hi = max(hi, __shfl_xor_sync(kFull, hi, o));
      }
      if (lane == 0) {
        s_f[warp] = f;
        s_lo[warp] = lo;
        s_hi[warp] = hi;
        s_bad[warp] = bad;
      }
      __syncthreads();
      if (tid == 0) {
        for (int w = 1; w < kAnThreads / 32; ++w) {
          f += s_f[w];
          lo = min(lo, s_lo[w]);
          hi = max(hi, s_hi[w]);
          bad |= s_bad[w];
        }
        long long span;
        finish_row(r, upper, row_base, method, f, lo, hi, bad, re - rs, flop, lo_out, hi_out,
                   symkey, row_nnz, err, &span);
        if (f) atomicAdd(&stats->total_flop, (unsigned long long)f);
        atomicMax(&stats->max_flop, (unsigned long long)f);
        atomicMax(&stats->max_span, (unsigned long long)span);
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ int num_bin_of(int method, long long nnz, long long flop, long long span,
                                          int rowlen) {
  if (nnz == 0) return 255;
  if (method == kMethodMerge && rowlen <= kMergeMaxLists) return kNumMerge;
  if (method == kMethodAdaptive) {
    // bitmap, prefix, sums and columns (plus one spare slot)
    const long long bytes = span <= 65536 ? 6ll * bitmap_words(span) + 10 * (nnz + 1) : 1ll << 40;
    if (bytes <= 2304) return kNumRank2K + group_index(flop, rowlen);
    if (bytes <= 4608) return kNumRank4K + group_index(flop, rowlen);
    if (bytes <= 9216) return kNumRank8K + group_index(flop, rowlen);
    // dense rows: windows of kWindowCols columns -- when the span needs several windows, only if
    // the binary searches that restrict every B row to every window stay small next to the
    // products
    if (nnz > 512 && span <= 4 * nnz &&
        (span <= kWindowCols ||
         (long long)rowlen * ((span + kWindowCols - 1) / kWindowCols) * 64 <= flop))
      return kNumWindow;
    if (nnz > kHashBlockSlots / 2) return kNumBlockRank;
  }
  if (nnz <= 32) return kNumHash64;
  if (nnz <= 64) return kNumHash128;
  if (nnz <= 128) return kNumHash256;
  if (nnz <= 256) return kNumHash512;
  if (nnz <= 512) return kNumHash1024;
  if (nnz <= kHashBlockSlots / 2) return kNumHashBlock;
  return kNumWindow;
}

__global__ void classify_numeric_kernel(Csr A, int m, int method, const long long* flop,
                                        const int* lo, const int* hi, const int* row_nnz,
                                        uint8_t* numkey) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  long long span = (hi[i] >= lo[i]) ? (long long)hi[i] - lo[i] + 1 : 0;
  numkey[i] = (uint8_t)num_bin_of(method, row_nnz[i], flop[i], span, A.rp[i + 1] - A.rp[i]);
}

}  // namespace

void launch_analyze(Csr A, Csr B, int upper, int row_base, int method, int lanes_per_row,
                    long long* flop, int* lo, int* hi, uint8_t* symkey, int* row_nnz,
                    AnalyzeStats* stats, int* err, int num_sms, cudaStream_t s) {
  const int m = A.rows;
  if (m <= 0) return;
  const int lpr = lanes_per_row;
  const long long rows_per_block = (long long)(kAnThreads / 32) * (32 / lpr);
  long long blocks = (m + rows_per_block - 1) / rows_per_block;
  long long cap = (long long)num_sms * 16;
  if (blocks > cap) blocks = cap;
  // rows beyond 32 * lpr entries: a CTA each
  long long lblocks = (m + kAnThreads - 1) / kAnThreads;
  if (lblocks > (long long)num_sms * 8) lblocks = (long long)num_sms * 8;
  analyze_long_kernel<<<(unsigned)lblocks, kAnThreads, 0, s>>>(A, B, upper, row_base, method,
                                                               32 * lpr, flop, lo, hi, symkey,
                                                               row_nnz, stats, err);
  switch (lpr) {
    case 4:
      analyze_kernel<4><<<(unsigned)blocks, kAnThreads, 0, s>>>(A, B, upper, row_base, method, flop,
                                                              lo, hi, symkey, row_nnz, stats, err);
      break;
    case 8:
      analyze_kernel<8><<<(unsigned)blocks, kAnThreads, 0, s>>>(A, B, upper, row_base, method, flop,
                                                              lo, hi, symkey, row_nnz, stats, err);
      break;
    case 16:
      analyze_kernel<16><<<(unsigned)blocks, kAnThreads, 0, s>>>(A, B, upper, row_base, method,
                                                               flop, lo, hi, symkey, row_nnz, stats,
                                                               err);
      break;
    default:
      analyze_kernel<32><<<(unsigned)blocks, kAnThreads, 0, s>>>(A, B, upper, row_base, method,
                                                               flop, lo, hi, symkey, row_nnz, stats,
                                                               err);
      break;
  }
}

void launch_classify_numeric(Csr A, int m, int method, const long long* flop, const int* lo,
                             const int* hi, const int* row_nnz, uint8_t* numkey, int num_sms,
                             cudaStream_t s) {
  (void)num_sms;
  if (m <= 0) return;
  classify_numeric_kernel<<<(m + 255) / 256, 256, 0, s>>>(A, m, method, flop, lo, hi, row_nnz,
                                                          numkey);
}

}  // namespace appt
