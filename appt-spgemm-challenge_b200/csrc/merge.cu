// Merge tier: warp per row k-way merge of the (sorted) B rows that the A row selects. The output
// comes out in column order, so no table and no sort are needed; duplicates of a column are
// summed with a warp reduction as they are popped.
//
// Reference counterpart: merge3 (bucket_flop_kernel + bucket_merge_flop_kernel +
// bucket_compact_kernel, spgemm_merge.cu:649-757, host merge3_product :760-933). The reference
// splits each row's column domain into K=5 buckets with one warp each and writes into a
// products-sized gapped buffer that a compaction pass then copies into C; it keeps the per-list
// cursors in shared memory sized by the longest A row, which fails beyond 227 KB. Here the
// symbolic count (count mode of this kernel) gives exact offsets, the numeric mode writes C in
// place, and rows with more than kMergeMaxLists A entries are routed to the window tier by the
// host (documented behaviour of the merge method).
//
// Lists are held as (cursor, end, head column) triples in shared memory; each lane owns the
// lists t = lane, lane + 32, ... of its row.
#include <climits>
#include "common.cuh"
#include "kernels.cuh"

namespace appt {

namespace {

template <bool NUMERIC, int WPB>
__global__ void __launch_bounds__(WPB * 32) merge_kernel(const int* rows, const long long* bin_off,
                                                         int bin, Csr A, Csr B, int upper,
                                                         int row_base, const long long* crp,
                                                         int* row_nnz, int* cci, double* cval,
                                                         int* err) {
  extern __shared__ __align__(16) unsigned char mg_smem[];
  constexpr int LISTS = kMergeMaxLists;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int* cur = reinterpret_cast<int*>(mg_smem) + warp * 3 * LISTS;
  int* end = cur + LISTS;
  int* head = end + LISTS;
  const long long b0 = bin_off[bin];
  const long long nrows = bin_off[bin + 1] - b0;
  for (long long r = (long long)blockIdx.x * WPB + warp; r < nrows;
       r += (long long)gridDim.x * WPB) {
    const int i = rows[b0 + r];
    const int ig = i + row_base;
    const int rs = A.rp[i], re = A.rp[i + 1];
    const int nk = re - rs;
    if (nk > LISTS) {
      if (lane == 0) set_error(err, kErrCapacity);
      continue;
    }
    for (int t = lane; t < nk; t += 32) {
      const int k = A.ci[rs + t];
      int bs = B.rp[k];
      const int be = B.rp[k + 1];
      if (upper) bs = lower_bound_col(B.ci, bs, be, ig);
      cur[t] = bs;
      end[t] = be;
      head[t] = bs < be ? B.ci[bs] : INT_MAX;
    }
    __syncwarp();
    long long c0 = 0, n = 0;
    if (NUMERIC) {
      c0 = crp[i];
      n = crp[i + 1] - c0;
    }
    int out = 0;
    // every iteration pops one distinct column; bounded by the products of the row
    for (;;) {
      int mymin = INT_MAX;
      for (int t = lane; t < nk; t += 32) mymin = min(mymin, head[t]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mymin = min(mymin, __shfl_xor_sync(kFull, mymin, o));
      if (mymin == INT_MAX) break;
      double s = 0.0;
      for (int t = lane; t < nk; t += 32) {
        if (head[t] == mymin) {
          const int q = cur[t];
          if (NUMERIC) s += A.val[rs + t] * B.val[q];
          const int q1 = q + 1;
          cur[t] = q1;
          head[t] = q1 < end[t] ? B.ci[q1] : INT_MAX;
        }
      }
      if (NUMERIC) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
        if (lane == 0 && out < n) {
          cci[c0 + out] = mymin;
          cval[c0 + out] = s;
        }
      }
      ++out;
      __syncwarp();
    }
    if (lane == 0) {
      if (NUMERIC) {
        if (out != n) set_error(err, kErrCapacity);
      } else {
        row_nnz[i] = out;
      }
    }
    __syncwarp();
  }
}

template <bool NUMERIC>
void run_merge(const int* rows, const long long* bin_off, int bin, long long nrows_host, Csr A,
               Csr B, int upper, int row_base, const long long* crp, int* row_nnz, int* cci,
               double* cval, int* err, int num_sms, cudaStream_t s) {
  constexpr int WPB = 4;
  const size_t smem = (size_t)WPB * 3 * kMergeMaxLists * sizeof(int);
  auto kern = merge_kernel<NUMERIC, WPB>;
  smem_opt_in((const void*)kern, smem);
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, WPB * 32, smem);
  if (occ < 1) occ = 1;
  long long grid = (long long)num_sms * occ;
  if (nrows_host >= 0) {
    long long want = (nrows_host + WPB - 1) / WPB;
    if (want < grid) grid = want < 1 ? 1 : want;
  }
  kern<<<(unsigned)grid, WPB * 32, smem, s>>>(rows, bin_off, bin, A, B, upper, row_base, crp,
                                              row_nnz, cci, cval, err);
}

}  // namespace

void launch_merge_count(const int* rows, const long long* bin_off, int bin, Csr A, Csr B,
                        int upper, int row_base, int* row_nnz, int* err, int num_sms,
                        cudaStream_t s) {
  run_merge<false>(rows, bin_off, bin, -1, A, B, upper, row_base, nullptr, row_nnz, nullptr,
                   nullptr, err, num_sms, s);
}

void launch_merge_numeric(const int* rows, const long long* bin_off, int bin, long long nrows,
                          Csr A, Csr B, int upper, int row_base, const long long* crp, int* cci,
                          double* cval, int* err, int num_sms, cudaStream_t s) {
  if (nrows <= 0) return;
  run_merge<true>(rows, bin_off, bin, nrows, A, B, upper, row_base, crp, nullptr, cci, cval, err,
                  num_sms, s);
}

}  // namespace appt
