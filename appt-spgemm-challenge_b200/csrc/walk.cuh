// Row walks: visiting the products a_ik * b_kj of one row of C with one warp.
//
// k-sequential order: A entries k ascending, and for each k the entries j of row k of B
// ascending -- the reference's (and the CPU oracle's) summation order. The 32 lanes cover one
// row of B per step (lane q takes entries q, q + 32, ...), so within a step every lane holds a
// different column and per-column updates need no atomics; a __syncwarp() between steps orders
// updates of the same column exactly as the sequential algorithm does.
//
// The A entries are loaded 32 at a time (one per lane) with their B row bounds, and the next two
// rows of B are prefetched while the current one is processed. Whether any row of B in the chunk
// is longer than a warp is decided once per chunk, so the common step is branch-free apart from
// predicated loads and updates.
#pragma once
#include "common.cuh"

namespace appt {

// Product in the reference's rounding: no fused multiply-add, so a*b then + rounds twice,
// as the sequential CPU algorithm does.
__device__ __forceinline__ double mul_add_rn(double acc, double a, double b) {
  return __dadd_rn(acc, __dmul_rn(a, b));
}

// Generic k-sequential walk: calls f(j, b_kj, a_ik) for every product of the row (lanes
// without a product in a step do not call f).
template <bool WITH_VAL, typename F>
__device__ __forceinline__ void walk_row_k_sequential(const Csr& A, const Csr& B, int rs, int re,
                                                      F&& f) {
  const int lane = threadIdx.x & 31;
  for (int base = rs; base < re; base += 32) {
    const int p = base + lane;
    const bool v = p < re;
    const int k = v ? A.ci[p] : 0;
    const int bs = v ? B.rp[k] : 0;
    const int len = v ? B.rp[k + 1] - bs : 0;
    const double a = (WITH_VAL && v) ? A.val[p] : 0.0;
    const int cnt = (re - base) < 32 ? (re - base) : 32;
    const bool any_long = __any_sync(kFull, len > 32);
    int j0 = -1, j1 = -1;
    double x0 = 0.0, x1 = 0.0;
    {
      const int b0 = __shfl_sync(kFull, bs, 0), l0 = __shfl_sync(kFull, len, 0);
      const int b1 = __shfl_sync(kFull, bs, 1);
      int l1 = __shfl_sync(kFull, len, 1);
      l1 = cnt > 1 ? l1 : 0;
      if (lane < l0) {
        j0 = __ldg(B.ci + b0 + lane);
        if (WITH_VAL) x0 = __ldg(B.val + b0 + lane);
      }
      if (lane < l1) {
        j1 = __ldg(B.ci + b1 + lane);
        if (WITH_VAL) x1 = __ldg(B.val + b1 + lane);
      }
    }
    for (int t = 0; t < cnt; ++t) {
      const int t2 = (t + 2) & 31;
      const int b2 = __shfl_sync(kFull, bs, t2);
      int l2 = __shfl_sync(kFull, len, t2);
      l2 = (t + 2 < cnt) ? l2 : 0;
      int j2 = -1;
      double x2 = 0.0;
      if (lane < l2) {
        j2 = __ldg(B.ci + b2 + lane);
        if (WITH_VAL) x2 = __ldg(B.val + b2 + lane);
      }
      const double at = WITH_VAL ? __shfl_sync(kFull, a, t) : 0.0;
      if (j0 >= 0) f(j0, x0, at);
      if (any_long) {
        const int lt = __shfl_sync(kFull, len, t), bt = __shfl_sync(kFull, bs, t);
        for (int q = 32 + lane; q < lt; q += 32) {
          const int j = __ldg(B.ci + bt + q);
          const double x = WITH_VAL ? __ldg(B.val + bt + q) : 0.0;
          f(j, x, at);
        }
      }
      __syncwarp();
      j0 = j1;
      x0 = x1;
      j1 = j2;
      x1 = x2;
    }
  }
}

// Presence bitmap of a row over [lo, lo + span): bit (j - lo) for every product column
// j >= jmin. Order-free (commutative ORs), so no step ordering is needed. Returns true if a
// column fell outside the span (a B row that is not sorted or lies outside [lo, hi]).
__device__ __forceinline__ bool fill_row_bitmap(const Csr& A, const Csr& B, int rs, int re,
                                                int lo, unsigned span, int jmin, unsigned* bm32) {
  const int lane = threadIdx.x & 31;
  bool bad = false;
  for (int base = rs; base < re; base += 32) {
    const int p = base + lane;
    const bool v = p < re;
    const int k = v ? A.ci[p] : 0;
    const int bs = v ? B.rp[k] : 0;
    const int len = v ? B.rp[k + 1] - bs : 0;
    const int cnt = (re - base) < 32 ? (re - base) : 32;
    const bool any_long = __any_sync(kFull, len > 32);
    int j0 = -1, j1 = -1;
    {
      const int b0 = __shfl_sync(kFull, bs, 0), l0 = __shfl_sync(kFull, len, 0);
      const int b1 = __shfl_sync(kFull, bs, 1);
      int l1 = __shfl_sync(kFull, len, 1);
      l1 = cnt > 1 ? l1 : 0;
      if (lane < l0) j0 = __ldg(B.ci + b0 + lane);
      if (lane < l1) j1 = __ldg(B.ci + b1 + lane);
    }
    for (int t = 0; t < cnt; ++t) {
      const int t2 = (t + 2) & 31;
      const int b2 = __shfl_sync(kFull, bs, t2);
      int l2 = __shfl_sync(kFull, len, t2);
      l2 = (t + 2 < cnt) ? l2 : 0;
      const int j2 = (lane < l2) ? __ldg(B.ci + b2 + lane) : -1;
      const unsigned off = (unsigned)(j0 - lo);
      if (j0 >= jmin) {
        if (off < span) atomicOr(bm32 + (off >> 5), 1u << (off & 31));
        else bad = true;
      }
      if (any_long) {
        const int lt = __shfl_sync(kFull, len, t), bt = __shfl_sync(kFull, bs, t);
        for (int q = 32 + lane; q < lt; q += 32) {
          const int j = __ldg(B.ci + bt + q);
          const unsigned o = (unsigned)(j - lo);
          if (j >= jmin) {
            if (o < span) atomicOr(bm32 + (o >> 5), 1u << (o & 31));
            else bad = true;
          }
        }
      }
      j0 = j1;
      j1 = j2;
    }
  }
  return bad;
}

// Exclusive popcount prefix of W 64-bit bitmap words into 16-bit entries; returns the total.
// Lane l owns a contiguous range of words, so one warp scan covers the whole bitmap.
__device__ __forceinline__ int bitmap_prefix64(const unsigned long long* bm, int W,
                                               unsigned short* pre) {
  const int lane = threadIdx.x & 31;
  const int per = (W + 31) >> 5;
  const int w0 = lane * per;
  const int w1 = (w0 + per < W) ? w0 + per : W;
  int s = 0;
  for (int w = w0; w < w1; ++w) s += __popcll(bm[w]);
  const int incl = warp_incl_scan(s);
  int run = incl - s;
  for (int w = w0; w < w1; ++w) {
    pre[w] = (unsigned short)run;
    run += __popcll(bm[w]);
  }
  return __shfl_sync(kFull, incl, 31);
}

// Rank accumulation (the numeric pass of the rank tier): every product a_ik * b_kj is added to
// acc[rank of j], where rank = pre[w] + popcount(bitmap[w] below j); col[rank] records j.
// k-sequential, so sums form in the reference's order.
__device__ __forceinline__ void accumulate_row_ranked(const Csr& A, const Csr& B, int rs, int re,
                                                      int lo, unsigned span, int jmin,
                                                      const unsigned long long* bm,
                                                      const unsigned short* pre, double* acc,
                                                      int* col) {
  const int lane = threadIdx.x & 31;
  for (int base = rs; base < re; base += 32) {
    const int p = base + lane;
    const bool v = p < re;
    const int k = v ? A.ci[p] : 0;
    const int bs = v ? B.rp[k] : 0;
    const int len = v ? B.rp[k + 1] - bs : 0;
    const double a = v ? A.val[p] : 0.0;
    const int cnt = (re - base) < 32 ? (re - base) : 32;
    const bool any_long = __any_sync(kFull, len > 32);
    int j0 = -1, j1 = -1;
    double x0 = 0.0, x1 = 0.0;
    {
      const int b0 = __shfl_sync(kFull, bs, 0), l0 = __shfl_sync(kFull, len, 0);
      const int b1 = __shfl_sync(kFull, bs, 1);
      int l1 = __shfl_sync(kFull, len, 1);
      l1 = cnt > 1 ? l1 : 0;
      if (lane < l0) {
        j0 = __ldg(B.ci + b0 + lane);
        x0 = __ldg(B.val + b0 + lane);
      }
      if (lane < l1) {
        j1 = __ldg(B.ci + b1 + lane);
        x1 = __ldg(B.val + b1 + lane);
      }
    }
    for (int t = 0; t < cnt; ++t) {
      const int t2 = (t + 2) & 31;
      const int b2 = __shfl_sync(kFull, bs, t2);
      int l2 = __shfl_sync(kFull, len, t2);
      l2 = (t + 2 < cnt) ? l2 : 0;
      int j2 = -1;
      double x2 = 0.0;
      if (lane < l2) {
        j2 = __ldg(B.ci + b2 + lane);
        x2 = __ldg(B.val + b2 + lane);
      }
      const double at = __shfl_sync(kFull, a, t);
      const unsigned off = (unsigned)(j0 - lo);
      if (j0 >= jmin && off < span) {
        const unsigned w = off >> 6;
        const int pos = pre[w] + __popcll(bm[w] & ((1ull << (off & 63)) - 1ull));
        acc[pos] = mul_add_rn(acc[pos], at, x0);
        col[pos] = j0;
      }
      if (any_long) {
        const int lt = __shfl_sync(kFull, len, t), bt = __shfl_sync(kFull, bs, t);
        for (int q = 32 + lane; q < lt; q += 32) {
          const int j = __ldg(B.ci + bt + q);
          const unsigned o = (unsigned)(j - lo);
          if (j >= jmin && o < span) {
            const unsigned w = o >> 6;
            const int pos = pre[w] + __popcll(bm[w] & ((1ull << (o & 63)) - 1ull));
            acc[pos] = mul_add_rn(acc[pos], at, __ldg(B.val + bt + q));
            col[pos] = j;
          }
        }
      }
      __syncwarp();
      j0 = j1;
      x0 = x1;
      j1 = j2;
      x1 = x2;
    }
  }
}

}  // namespace appt
