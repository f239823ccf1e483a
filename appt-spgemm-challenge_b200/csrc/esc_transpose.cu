// ESC baseline (expand - sort - compress) and the device transpose used by the A*A^T path.
//
// ESC reference counterpart: spgemm_self_product_manual with count_intermediates_kernel,
// expand_intermediates_kernel, thrust sort_by_key / reduce_by_key and finalize_csr_kernel
// (spgemm_kernel_manual.cu:121-173, 272-437). Here the expansion lands at exact per-row offsets
// (prefix of the products count) in product order, each row's segment is sorted stably by
// column, and the compress step sums equal columns in expansion order -- one write of C.
//
// Transpose reference counterpart: build_csc (spgemm_kernel_formulations.cu:36-120): column
// count, scan, atomic scatter, then a global sort by (col << 32 | row). Here the scatter is
// followed by a per-column stable sort by row index (segsort), so the rows of A^T come out
// sorted without 64-bit keys. Column pointers are sized by A's column count (the reference
// sizes them by A's row count, which is only valid when cols <= rows).
#include <climits>
#include "common.cuh"
#include "kernels.cuh"

namespace appt {

namespace {

constexpr int kEscWPB = 8;

__global__ void __launch_bounds__(kEscWPB * 32) esc_expand_kernel(Csr A, Csr B, int upper,
                                                                  int row_base,
                                                                  const long long* foff, int* keys,
                                                                  double* vals) {
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * kEscWPB;
  for (long long i = (long long)blockIdx.x * kEscWPB + (threadIdx.x >> 5); i < A.rows; i += nw) {
    const int ig = (int)i + row_base;
    const int rs = A.rp[i], re = A.rp[i + 1];
    long long o = foff[i];
    for (int base = rs; base < re; base += 32) {
      const int p = base + lane;
      const bool v = p < re;
      const int k = v ? A.ci[p] : 0;
      const int bs = v ? B.rp[k] : 0;
      const int len = v ? B.rp[k + 1] - bs : 0;
      const double a = v ? A.val[p] : 0.0;
      const int incl = warp_incl_scan(len);
      const int excl = incl - len;
      const int total = __shfl_sync(kFull, incl, 31);
      for (int t0 = 0; t0 < total; t0 += 32) {
        const int t = t0 + lane;
        const int L = warp_owner(excl, t);
        const int bsL = __shfl_sync(kFull, bs, L), exL = __shfl_sync(kFull, excl, L);
        const double aL = __shfl_sync(kFull, a, L);
        if (t < total) {
          const int q = bsL + t - exL;
          int j = B.ci[q];
          if (upper && j < ig) j = INT_MAX;   // filtered products sort to the end of the row
          keys[o + t] = j;
          vals[o + t] = aL * B.val[q];
        }
      }
      o += total;
    }
  }
}

template <bool WRITE>
__global__ void __launch_bounds__(kEscWPB * 32) esc_reduce_kernel(int m, const long long* foff,
                                                                  const int* keys,
                                                                  const double* vals,
                                                                  int* row_nnz,
                                                                  const long long* crp, int* cci,
                                                                  double* cval) {
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * kEscWPB;
  for (long long i = (long long)blockIdx.x * kEscWPB + (threadIdx.x >> 5); i < m; i += nw) {
    const long long f0 = foff[i], f1 = foff[i + 1];
    const long long c0 = WRITE ? crp[i] : 0;
    int running = 0;
    for (long long base = f0; base < f1; base += 32) {
      const long long t = base + lane;
      const bool valid = t < f1;
      const int key = valid ? keys[t] : INT_MAX;
      const int prev = (valid && t > f0) ? keys[t - 1] : -1;
      const bool head = valid && key != INT_MAX && key != prev;
      const unsigned bal = __ballot_sync(kFull, head);
      if (WRITE && head) {
        double s = vals[t];
        long long u = t + 1;
        while (u < f1 && keys[u] == key) {
          s += vals[u];
          ++u;
        }
        const long long dst = c0 + running + __popc(bal & lanemask_lt());
        cci[dst] = key;
        cval[dst] = s;
      }
      running += __popc(bal);
    }
    if (!WRITE && lane == 0) row_nnz[i] = running;
  }
}

// ------------------------------------------------------------------ transpose
// Entries whose column is outside [0, cols) are dropped here; the product's analysis pass
// reports them as an invalid operand.
__global__ void tr_count_kernel(const int* ci, long long nnz, int cols, int* cnt) {
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p < nnz && (unsigned)ci[p] < (unsigned)cols) atomicAdd(&cnt[ci[p]], 1);
}

__global__ void tr_scatter_kernel(Csr A, unsigned long long* cursor, int* t_ci, double* t_val) {
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long i = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < A.rows;
       i += nw) {
    const int rs = A.rp[i], re = A.rp[i + 1];
    for (int p = rs + lane; p < re; p += 32) {
      if ((unsigned)A.ci[p] >= (unsigned)A.cols) continue;
      const unsigned long long pos = atomicAdd(&cursor[A.ci[p]], 1ull);
      t_ci[pos] = (int)i;
      t_val[pos] = A.val[p];
    }
  }
}

}  // namespace

size_t segsort_scratch_bytes(int nseg);
void segsort(int* keys, double* vals, int* keys_alt, double* vals_alt, const long long* off,
             int nseg, void* scratch, int num_sms, cudaStream_t s);

void launch_esc_expand(Csr A, Csr B, int upper, int row_base, const long long* foff, int* keys,
                       double* vals, int num_sms, cudaStream_t s) {
  if (A.rows <= 0) return;
  long long blocks = (A.rows + kEscWPB - 1) / kEscWPB;
  if (blocks > (long long)num_sms * 8) blocks = (long long)num_sms * 8;
  esc_expand_kernel<<<(unsigned)blocks, kEscWPB * 32, 0, s>>>(A, B, upper, row_base, foff, keys,
                                                               vals);
}

void launch_esc_count(int m, const long long* foff, const int* keys, int* row_nnz, int num_sms,
                      cudaStream_t s) {
  if (m <= 0) return;
  long long blocks = (m + kEscWPB - 1) / kEscWPB;
  if (blocks > (long long)num_sms * 8) blocks = (long long)num_sms * 8;
  esc_reduce_kernel<false><<<(unsigned)blocks, kEscWPB * 32, 0, s>>>(m, foff, keys, nullptr,
                                                                     row_nnz, nullptr, nullptr,
                                                                     nullptr);
}

void launch_esc_compress(int m, const long long* foff, const int* keys, const double* vals,
                         const long long* crp, int* cci, double* cval, int num_sms,
                         cudaStream_t s) {
  if (m <= 0) return;
  long long blocks = (m + kEscWPB - 1) / kEscWPB;
  if (blocks > (long long)num_sms * 8) blocks = (long long)num_sms * 8;
  esc_reduce_kernel<true><<<(unsigned)blocks, kEscWPB * 32, 0, s>>>(m, foff, keys, vals, nullptr,
                                                                    crp, cci, cval);
}

size_t transpose_scratch_bytes(int rows, int cols, long long nnz) {
  (void)rows;
  size_t b = 0;
  b += ((size_t)cols * sizeof(int) + 255) & ~(size_t)255;                   // counts
  b += ((size_t)(cols + 1) * sizeof(long long) + 255) & ~(size_t)255;       // offsets
  b += ((size_t)cols * sizeof(long long) + 255) & ~(size_t)255;             // cursors
  b += ((size_t)nnz * sizeof(int) + 255) & ~(size_t)255;                    // alt keys
  b += ((size_t)nnz * sizeof(double) + 255) & ~(size_t)255;                 // alt vals
  b += (scan_scratch_elems(cols) * sizeof(long long) + 255) & ~(size_t)255;
  b += segsort_scratch_bytes(cols) + 256;
  return b;
}

void launch_transpose(Csr A, long long nnz, int* t_rp, int* t_ci, double* t_val, void* scratch,
                      int num_sms, cudaStream_t s) {
  const int n = A.cols;
  char* p = (char*)scratch;
  auto take = [&](size_t bytes) {
    char* r = p;
    p += (bytes + 255) & ~(size_t)255;
    return r;
  };
  int* cnt = (int*)take((size_t)n * sizeof(int));
  long long* off = (long long*)take((size_t)(n + 1) * sizeof(long long));
  unsigned long long* cursor = (unsigned long long*)take((size_t)n * sizeof(long long));
  int* alt_k = (int*)take((size_t)nnz * sizeof(int));
  double* alt_v = (double*)take((size_t)nnz * sizeof(double));
  long long* sc = (long long*)take(scan_scratch_elems(n) * sizeof(long long));
  void* ss = take(segsort_scratch_bytes(n));
  cudaMemsetAsync(cnt, 0, (size_t)n * sizeof(int), s);
  if (nnz > 0)
    tr_count_kernel<<<(unsigned)((nnz + 255) / 256), 256, 0, s>>>(A.ci, nnz, n, cnt);
  scan_exclusive(cnt, off, n, sc, s);
  narrow_rowptr(off, t_rp, (long long)n + 1, s);
  cudaMemcpyAsync(cursor, off, (size_t)n * sizeof(long long), cudaMemcpyDeviceToDevice, s);
  if (A.rows > 0) {
    long long blocks = (A.rows + 7) / 8;
    if (blocks > (long long)num_sms * 16) blocks = (long long)num_sms * 16;
    tr_scatter_kernel<<<(unsigned)blocks, 256, 0, s>>>(A, cursor, t_ci, t_val);
  }
  segsort(t_ci, t_val, alt_k, alt_v, off, n, ss, num_sms, s);
}

}  // namespace appt
