// Shared device-side definitions for the B200 adaptive SpGEMM engine.
//
// Conventions (all kernels):
//   * Operand CSR matrices (A and B) keep the reference's int32 row_ptr/col_idx and fp64
//     values (include/spgemm.h:55-106 of the reference: `int` indices, `double` values).
//   * C uses an int64 row_ptr internally so that nnz(C) > 2^31 (R-MAT 2^20 class inputs)
//     is representable; the spgemm.h-compatible wrappers narrow it back to int32.
//   * Every loop that waits or probes is bounded; a kernel that hits a bound sets a bit in a
//     device error word and returns instead of spinning.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace appt {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;
constexpr unsigned kEmptyKey = 0xffffffffu;   // empty hash slot (column ids are < 2^31)

// Device error bits (OR-ed into a device int; read back by the host at sync points).
enum DeviceError : int {
  kErrTableFull = 1,      // a hash probe sequence exceeded the table size
  kErrCapacity = 2,       // a row was routed to a kernel whose capacity it exceeds
  kErrBounds = 4,         // an index check failed (write skipped)
  kErrSpin = 8,           // a bounded wait gave up
  kErrSmallFallback = 16, // the small-problem path cannot take this input (not an error)
};

// Read-only CSR view used by kernels. `rp` values are absolute offsets into ci/val.
struct Csr {
  const int32_t* rp;
  const int32_t* ci;
  const double* val;
  int32_t rows;
  int32_t cols;
};

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Inclusive warp scan of an int.
__device__ __forceinline__ int warp_incl_scan(int x) {
  const int lane = lane_id();
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(kFull, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

__device__ __forceinline__ long long warp_sum_ll(long long x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
  return x;
}

__device__ __forceinline__ int warp_sum(int x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
  return x;
}

// Fibonacci hashing: the high bits of j * 2^32/phi. Using the high bits matters for
// stencil-like column sets (columns that differ by multiples of a power of two would all
// collide under a low-bit mask).
__device__ __forceinline__ unsigned hash_slot(unsigned j, int log2_size) {
  return (j * 2654435769u) >> (32 - log2_size);
}

__host__ __device__ __forceinline__ int ilog2_ceil(long long x) {
  int l = 0;
  while ((1ll << l) < x) ++l;
  return l;
}

// Within a warp, find for product index t (0 <= t < total) the lane L whose segment
// [excl_L, excl_L + len_L) contains t. `excl` is the exclusive prefix of segment lengths
// held one per lane (non-decreasing across lanes). Must be called by all 32 lanes.
__device__ __forceinline__ int warp_owner(int excl, int t) {
  int L = 0;
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1) {
    int e = __shfl_sync(kFull, excl, L + step);
    if (e <= t) L += step;
  }
  return L;
}

// First position in ci[lo, hi) whose value is >= v (B rows are sorted by column).
__device__ __forceinline__ int lower_bound_col(const int32_t* ci, int lo, int hi, int v) {
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (ci[mid] < v) lo = mid + 1; else hi = mid;
  }
  return lo;
}


// Block-wide exclusive scan of one int64 per thread. `buf` needs NT/32 + 1 entries of shared
// memory. Returns the exclusive prefix; *total receives the block sum. Contains barriers: all
// threads of the block must call it.
template <int NT>
__device__ __forceinline__ long long block_excl_scan_ll(long long x, long long* buf,
                                                        long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  long long incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    long long y = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) buf[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    long long w = (lane < NT / 32) ? buf[lane] : 0;
    long long wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      long long y = __shfl_up_sync(kFull, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < NT / 32) buf[lane] = wi - w;
    if (lane == NT / 32 - 1) buf[NT / 32] = wi;
  }
  __syncthreads();
  const long long res = buf[warp] + incl - x;
  if (total) *total = buf[NT / 32];
  __syncthreads();
  return res;
}

// Index (0-based) of the r-th set bit of m (r < popc(m)).
__device__ __forceinline__ int nth_set_bit(unsigned m, int r) {
  int pos = 0;
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const int c = __popc(m & ((1u << w) - 1u));
    if (r >= c) {
      r -= c;
      m >>= w;
      pos += w;
    }
  }
  return pos;
}

// Index (0-based) of the r-th set bit of a 64-bit word (r < popcll(m)).
__device__ __forceinline__ int nth_set_bit64(unsigned long long m, int r) {
  const unsigned lo = (unsigned)m;
  const int c = __popc(lo);
  return r < c ? nth_set_bit(lo, r) : 32 + nth_set_bit((unsigned)(m >> 32), r - c);
}

// Largest index L in [0, n) with a[L] <= t for a non-decreasing array.
template <typename T>
__device__ __forceinline__ int search_le(const T* a, int n, long long t) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if ((long long)a[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void set_error(int* err, int code) {
  if (err) atomicOr(err, code);
}

}  // namespace appt
