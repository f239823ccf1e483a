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
    int bs_c = __shfl_sync(kFull, bs, 0);
    int len_c = __shfl_sync(kFull, len, 0);
    double a_c = WITH_VAL ? __shfl_sync(kFull, a, 0) : 0.0;
    int j_c = (lane < len_c) ? B.ci[bs_c + lane] : 0;
    double x_c = (WITH_VAL && lane < len_c) ? B.val[bs_c + lane] : 0.0;
    for (int t = 0; t < cnt; ++t) {
      const int tn = (t + 1) & 31;
      const int bs_n = __shfl_sync(kFull, bs, tn);
      const int len_n = (t + 1 < cnt) ? __shfl_sync(kFull, len, tn) : 0;
      const double a_n = WITH_VAL ? __shfl_sync(kFull, a, tn) : 0.0;
      int j_n = 0;
      double x_n = 0.0;
      if (lane < len_n) {
        j_n = B.ci[bs_n + lane];
        if (WITH_VAL) x_n = B.val[bs_n + lane];
      }
      if (lane < len_c) f(j_c, x_c, a_c);
      for (int q = 32 + lane; q < len_c; q += 32) {   // rows of B longer than a warp
        const int j = B.ci[bs_c + q];
        const double x = WITH_VAL ? B.val[bs_c + q] : 0.0;
        f(j, x, a_c);
      }
      __syncwarp();
      bs_c = bs_n;
      len_c = len_n;
      a_c = a_n;
      j_c = j_n;
      x_c = x_n;
    }
  }
}

// Product in the reference's rounding: no fused multiply-add, so a*b then + rounds twice,
// as the sequential CPU algorithm does.
__device__ __forceinline__ double mul_add_rn(double acc, double a, double b) {
  return __dadd_rn(acc, __dmul_rn(a, b));
}

}  // namespace appt
