// k-sequential product walk for one row per warp.
//
// Visits the products a_ik * b_kj of row i in the reference order: A entries k ascending,
// and for each k the entries j of row k of B ascending. The 32 lanes of the warp cover one
// row of B at a time (lane q takes entry q, q + 32, ...), so within one step every lane holds a
// different column j -- per-column updates need no atomics -- and a __syncwarp() separates
// consecutive rows of B, which orders updates of the same column across steps exactly as the
// sequential algorithm does.
//
// The A entries are loaded 32 at a time (one per lane) together with the B row bounds, and the
// next B row's first 32 (j, b_kj) pairs are prefetched while the current one is processed, so
// each step waits on one memory round trip at most.
#pragma once
#include "common.cuh"

namespace appt {

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
    // pipeline: the (j, b_kj) pairs of the next two rows of B are loaded ahead; j = -1 marks
    // a lane without an entry
    int j0 = -1, j1 = -1;
    double x0 = 0.0, x1 = 0.0;
    {
      const int b0 = __shfl_sync(kFull, bs, 0), l0 = __shfl_sync(kFull, len, 0);
      const int b1 = __shfl_sync(kFull, bs, 1);
      const int l1 = cnt > 1 ? __shfl_sync(kFull, len, 1) : 0;
      if (lane < l0) {
        j0 = B.ci[b0 + lane];
        if (WITH_VAL) x0 = B.val[b0 + lane];
      }
      if (lane < l1) {
        j1 = B.ci[b1 + lane];
        if (WITH_VAL) x1 = B.val[b1 + lane];
      }
    }
    for (int t = 0; t < cnt; ++t) {
      const int t2 = (t + 2) & 31;
      const int b2 = __shfl_sync(kFull, bs, t2);
      const int l2 = (t + 2 < cnt) ? __shfl_sync(kFull, len, t2) : 0;
      int j2 = -1;
      double x2 = 0.0;
      if (lane < l2) {
        j2 = B.ci[b2 + lane];
        if (WITH_VAL) x2 = B.val[b2 + lane];
      }
      const double at = WITH_VAL ? __shfl_sync(kFull, a, t) : 0.0;
      if (j0 >= 0) f(j0, x0, at);
      const int lt = __shfl_sync(kFull, len, t);
      if (lt > 32) {                      // rows of B longer than a warp (warp-uniform branch)
        const int bt = __shfl_sync(kFull, bs, t);
        for (int q = 32 + lane; q < lt; q += 32) {
          const int j = B.ci[bt + q];
          const double x = WITH_VAL ? B.val[bt + q] : 0.0;
          f(j, x, at);
        }
      }
      __syncwarp();
      j0 = j1; x0 = x1;
      j1 = j2; x1 = x2;
    }
  }
}

// Product in the reference's rounding: no fused multiply-add, so a*b then + rounds twice,
// as the sequential CPU algorithm does.
__device__ __forceinline__ double mul_add_rn(double acc, double a, double b) {
  return __dadd_rn(acc, __dmul_rn(a, b));
}

}  // namespace appt
