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

// ---------------------------------------------------------------------------------------------
// Grouped walks for rows whose B rows are short. The warp is split into G groups of L = 32 / G
// lanes; in step s group g takes A entry t = s * G + g of the current chunk and its lanes cover
// that row of B (lane q of the group takes entries q, q + L, ...). Loads and rank computations
// are shared by all groups; updates that must be ordered are applied group by group (G
// sub-phases, each ended by __syncwarp), which keeps every column's contributions k-ascending.

template <int G>
__device__ __forceinline__ void load_group_entry(const Csr& B, int bs, int len, int cnt, int s,
                                                 int grp, int sub, int& j, double* x) {
  constexpr int L = 32 / G;
  const int t = s * G + grp;
  const int bt = __shfl_sync(kFull, bs, t & 31);
  int lt = __shfl_sync(kFull, len, t & 31);
  lt = t < cnt ? lt : 0;
  j = -1;
  if (sub < lt) {
    j = __ldg(B.ci + bt + sub);
    if (x) *x = __ldg(B.val + bt + sub);
  }
  (void)L;
}

// Bitmap fill with G groups (order-free).
template <int G>
__device__ __forceinline__ bool fill_row_bitmap_g(const Csr& A, const Csr& B, int rs, int re,
                                                  int lo, unsigned span, int jmin, unsigned* bm32) {
  constexpr int L = 32 / G;
  const int lane = threadIdx.x & 31, grp = lane / L, sub = lane % L;
  bool bad = false;
  for (int base = rs; base < re; base += 32) {
    const int p = base + lane;
    const bool v = p < re;
    const int k = v ? A.ci[p] : 0;
    const int bs = v ? B.rp[k] : 0;
    const int len = v ? B.rp[k + 1] - bs : 0;
    const int cnt = (re - base) < 32 ? (re - base) : 32;
    const bool any_long = __any_sync(kFull, len > L);
    const int steps = (cnt + G - 1) / G;
    int j0, j1, j2;
    load_group_entry<G>(B, bs, len, cnt, 0, grp, sub, j0, nullptr);
    load_group_entry<G>(B, bs, len, cnt, 1, grp, sub, j1, nullptr);
    for (int s = 0; s < steps; ++s) {
      load_group_entry<G>(B, bs, len, cnt, s + 2, grp, sub, j2, nullptr);
      const unsigned off = (unsigned)(j0 - lo);
      if (j0 >= jmin) {
        if (off < span) atomicOr(bm32 + (off >> 5), 1u << (off & 31));
        else bad = true;
      }
      if (any_long) {
        const int t = s * G + grp;
        const int bt = __shfl_sync(kFull, bs, t & 31);
        int lt = __shfl_sync(kFull, len, t & 31);
        lt = t < cnt ? lt : 0;
        for (int q = L + sub; q < lt; q += L) {
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

// Exclusive popcount prefix of W 32-bit bitmap words into 16-bit entries; returns the total.
__device__ __forceinline__ int bitmap_prefix32(const unsigned* bm, int W, unsigned short* pre) {
  const int lane = threadIdx.x & 31;
  const int per = (W + 31) >> 5;
  const int w0 = lane * per;
  const int w1 = (w0 + per < W) ? w0 + per : W;
  int s = 0;
  for (int w = w0; w < w1; ++w) s += __popc(bm[w]);
  const int incl = warp_incl_scan(s);
  int run = incl - s;
  for (int w = w0; w < w1; ++w) {
    pre[w] = (unsigned short)run;
    run += __popc(bm[w]);
  }
  return __shfl_sync(kFull, incl, 31);
}

// Ranked accumulation with G groups: acc[rank(j)] += a_ik * b_kj and coff[rank(j)] = j - lo,
// with rank(j) = pre[w] + popc(bm[w] below j) over 32-bit words. Sums form k-ascending.
template <int G>
__device__ __forceinline__ void accumulate_row_ranked_g(const Csr& A, const Csr& B, int rs, int re,
                                                        int lo, unsigned span, int jmin,
                                                        const unsigned* bm,
                                                        const unsigned short* pre, double* acc,
                                                        unsigned short* coff) {
  constexpr int L = 32 / G;
  const int lane = threadIdx.x & 31, grp = lane / L, sub = lane % L;
  for (int base = rs; base < re; base += 32) {
    const int p = base + lane;
    const bool v = p < re;
    const int k = v ? A.ci[p] : 0;
    const int bs = v ? B.rp[k] : 0;
    const int len = v ? B.rp[k + 1] - bs : 0;
    const double a = v ? A.val[p] : 0.0;
    const int cnt = (re - base) < 32 ? (re - base) : 32;
    const bool any_long = __any_sync(kFull, len > L);
    const int steps = (cnt + G - 1) / G;
    int j0, j1, j2;
    double x0, x1, x2;
    load_group_entry<G>(B, bs, len, cnt, 0, grp, sub, j0, &x0);
    load_group_entry<G>(B, bs, len, cnt, 1, grp, sub, j1, &x1);
    for (int s = 0; s < steps; ++s) {
      load_group_entry<G>(B, bs, len, cnt, s + 2, grp, sub, j2, &x2);
      const int t = s * G + grp;
      const double at = __shfl_sync(kFull, a, t & 31);
      const unsigned off = (unsigned)(j0 - lo);
      const bool ok = j0 >= jmin && off < span;
      int pos = 0;
      if (ok) pos = pre[off >> 5] + __popc(bm[off >> 5] & ((1u << (off & 31)) - 1u));
      int lt = 0, bt = 0;
      if (any_long) {
        bt = __shfl_sync(kFull, bs, t & 31);
        lt = __shfl_sync(kFull, len, t & 31);
        lt = t < cnt ? lt : 0;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        if (grp == g) {
          if (ok) {
            acc[pos] = mul_add_rn(acc[pos], at, x0);
            coff[pos] = (unsigned short)off;
          }
          if (any_long) {
            for (int q = L + sub; q < lt; q += L) {
              const int j = __ldg(B.ci + bt + q);
              const unsigned o = (unsigned)(j - lo);
              if (j >= jmin && o < span) {
                const int ps = pre[o >> 5] + __popc(bm[o >> 5] & ((1u << (o & 31)) - 1u));
                acc[ps] = mul_add_rn(acc[ps], at, __ldg(B.val + bt + q));
                coff[ps] = (unsigned short)o;
              }
            }
          }
        }
        __syncwarp();
      }
      j0 = j1;
      x0 = x1;
      j1 = j2;
      x1 = x2;
    }
  }
}

}  // namespace appt
