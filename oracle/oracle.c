/*
 * CPU oracle for the adaptive SpGEMM path -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may load
 * this library, and only as the checker or the timed CPU baseline; the engine never calls it.
 *
 * What it restates (reference = XUE77565/APPT-Spgemm-Challenge):
 *  - the products of C = A*B row by row: every a_ik * b_kj for k in row i of A and j in row k
 *    of B, structural zeros kept, columns strictly ascending per row -- the output contract of
 *    every reference method (count_intermediates_kernel / expand_intermediates_kernel,
 *    src/spgemm_kernel_manual.cu:121-159; merge semantics src/spgemm_merge.cu:682-739; sorted
 *    check src/spgemm_kernel_hash.cu:803-809);
 *  - the upper-triangle filter of the A*A^T entry points (j >= i; src/spgemm_kernel_hash.cu:406,
 *    src/spgemm_merge.cu:731);
 *  - the device transpose build_csc (CSR -> CSC with rows sorted inside each column,
 *    src/spgemm_kernel_formulations.cu:69-120), here as a stable counting sort;
 *  - the MinHash output-size estimate (murmur_hash3, mh_construct_kernel, mh_merge_kernel,
 *    src/spgemm_kernel_hash.cu:78-90, 257-369) including its floating-point summation order;
 *  - the products-count estimate used below 100000 nonzeros (count_intermediates_par_kernel,
 *    src/spgemm_kernel_hash.cu:33-55, 853-858).
 * Sums run in k-then-q order (row k of A ascending, then row k of B ascending) with no
 * fused multiply-add (compiled with -ffp-contract=off), starting from 0.0.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void oracle_set_threads(int n) { g_threads = n; }

int oracle_num_threads(void) {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_row_products(int64_t m, const int32_t *arp, const int32_t *aci, const int32_t *brp,
                         int64_t *out) {
  int nt = oracle_num_threads();
  (void)nt;
#pragma omp parallel for schedule(static) num_threads(nt)
  for (int64_t i = 0; i < m; ++i) {
    int64_t s = 0;
    for (int32_t p = arp[i]; p < arp[i + 1]; ++p) s += brp[aci[p] + 1] - brp[aci[p]];
    out[i] = s;
  }
}

int64_t oracle_symbolic(int64_t m, int64_t ncols, const int32_t *arp, const int32_t *aci,
                        const int32_t *brp, const int32_t *bci, int upper, int64_t row_base,
                        int64_t *row_nnz) {
  int64_t total = 0;
  int nt = oracle_num_threads();
#pragma omp parallel num_threads(nt) reduction(+ : total)
  {
    int64_t *mark = (int64_t *)malloc(sizeof(int64_t) * (size_t)(ncols > 0 ? ncols : 1));
    for (int64_t j = 0; j < ncols; ++j) mark[j] = -1;
#pragma omp for schedule(dynamic, 256)
    for (int64_t i = 0; i < m; ++i) {
      const int64_t ig = i + row_base;
      int64_t cnt = 0;
      for (int32_t p = arp[i]; p < arp[i + 1]; ++p) {
        const int32_t k = aci[p];
        for (int32_t q = brp[k]; q < brp[k + 1]; ++q) {
          const int32_t j = bci[q];
          if (upper && j < ig) continue;
          if (mark[j] != i) {
            mark[j] = i;
            ++cnt;
          }
        }
      }
      row_nnz[i] = cnt;
      total += cnt;
    }
    free(mark);
  }
  return total;
}

/* Per-row structure invariants of C for products too large to hold on the host: the exact
 * number of distinct columns (as oracle_symbolic) and the sum of those distinct column ids. A
 * matching (count, sum) pair per row is a size-independent check of the row's column set.
 * Same product enumeration as oracle_symbolic (src/spgemm_kernel_manual.cu:121-159). */
void oracle_symbolic_sums(int64_t m, int64_t ncols, const int32_t *arp, const int32_t *aci,
                          const int32_t *brp, const int32_t *bci, int upper, int64_t row_base,
                          int64_t *row_nnz, int64_t *row_colsum) {
  int nt = oracle_num_threads();
#pragma omp parallel num_threads(nt)
  {
    int64_t *mark = (int64_t *)malloc(sizeof(int64_t) * (size_t)(ncols > 0 ? ncols : 1));
    for (int64_t j = 0; j < ncols; ++j) mark[j] = -1;
#pragma omp for schedule(dynamic, 64)
    for (int64_t i = 0; i < m; ++i) {
      const int64_t ig = i + row_base;
      int64_t cnt = 0, sum = 0;
      for (int32_t p = arp[i]; p < arp[i + 1]; ++p) {
        const int32_t k = aci[p];
        for (int32_t q = brp[k]; q < brp[k + 1]; ++q) {
          const int32_t j = bci[q];
          if (upper && j < ig) continue;
          if (mark[j] != i) {
            mark[j] = i;
            ++cnt;
            sum += j;
          }
        }
      }
      row_nnz[i] = cnt;
      row_colsum[i] = sum;
    }
    free(mark);
  }
}

typedef struct {
  int32_t col;
  double val;
} entry_t;

static int cmp_entry(const void *a, const void *b) {
  const int32_t x = ((const entry_t *)a)->col, y = ((const entry_t *)b)->col;
  return (x > y) - (x < y);
}

static void sort_entries(entry_t *e, int64_t n) {
  if (n < 24) {
    for (int64_t i = 1; i < n; ++i) {
      entry_t t = e[i];
      int64_t j = i - 1;
      while (j >= 0 && e[j].col > t.col) {
        e[j + 1] = e[j];
        --j;
      }
      e[j + 1] = t;
    }
  } else {
    qsort(e, (size_t)n, sizeof(entry_t), cmp_entry);
  }
}

/* Fills cci/cval at the offsets crp (exclusive prefix of the symbolic counts). Returns 0, or -1
 * if a row's count disagrees with crp. */
int oracle_numeric(int64_t m, int64_t ncols, const int32_t *arp, const int32_t *aci,
                   const double *aval, const int32_t *brp, const int32_t *bci, const double *bval,
                   int upper, int64_t row_base, const int64_t *crp, int32_t *cci, double *cval) {
  int bad = 0;
  int nt = oracle_num_threads();
#pragma omp parallel num_threads(nt) reduction(| : bad)
  {
    int64_t *mark = (int64_t *)malloc(sizeof(int64_t) * (size_t)(ncols > 0 ? ncols : 1));
    int64_t *slot = (int64_t *)malloc(sizeof(int64_t) * (size_t)(ncols > 0 ? ncols : 1));
    for (int64_t j = 0; j < ncols; ++j) mark[j] = -1;
    int64_t cap = 1024;
    entry_t *buf = (entry_t *)malloc(sizeof(entry_t) * (size_t)cap);
#pragma omp for schedule(dynamic, 256)
    for (int64_t i = 0; i < m; ++i) {
      const int64_t ig = i + row_base;
      const int64_t want = crp[i + 1] - crp[i];
      if (want > cap) {
        cap = want;
        buf = (entry_t *)realloc(buf, sizeof(entry_t) * (size_t)cap);
      }
      int64_t cnt = 0;
      for (int32_t p = arp[i]; p < arp[i + 1]; ++p) {
        const int32_t k = aci[p];
        const double a = aval[p];
        for (int32_t q = brp[k]; q < brp[k + 1]; ++q) {
          const int32_t j = bci[q];
          if (upper && j < ig) continue;
          const double v = a * bval[q];
          if (mark[j] != i) {
            mark[j] = i;
            if (cnt >= want) {
              bad = 1;
              continue;
            }
            slot[j] = cnt;
            buf[cnt].col = j;
            buf[cnt].val = 0.0 + v;
            ++cnt;
          } else {
            buf[slot[j]].val += v;
          }
        }
      }
      if (cnt != want) bad = 1;
      sort_entries(buf, cnt);
      for (int64_t t = 0; t < cnt; ++t) {
        cci[crp[i] + t] = buf[t].col;
        cval[crp[i] + t] = buf[t].val;
      }
    }
    free(mark);
    free(slot);
    free(buf);
  }
  return bad ? -1 : 0;
}

/* CSR (m x n) -> CSR of the transpose (n x m); rows of the result ascending (stable). */
void oracle_transpose(int64_t m, int64_t n, const int32_t *arp, const int32_t *aci,
                      const double *aval, int32_t *trp, int32_t *tci, double *tval) {
  int64_t *cnt = (int64_t *)calloc((size_t)n + 1, sizeof(int64_t));
  for (int64_t p = arp[0]; p < arp[m]; ++p) cnt[aci[p] + 1]++;
  for (int64_t c = 0; c < n; ++c) cnt[c + 1] += cnt[c];
  for (int64_t c = 0; c <= n; ++c) trp[c] = (int32_t)cnt[c];
  for (int64_t i = 0; i < m; ++i) {
    for (int32_t p = arp[i]; p < arp[i + 1]; ++p) {
      const int64_t pos = cnt[aci[p]]++;
      tci[pos] = (int32_t)i;
      tval[pos] = aval[p];
    }
  }
  free(cnt);
}

/* ---- output-size estimate of the reference's hash path ---- */
static uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

uint32_t oracle_murmur3(uint32_t key) {
  uint32_t h = 1234u;
  uint32_t k = key * 0xcc9e2d51u;
  k = rotl32(k, 15);
  k *= 0x1b873593u;
  h ^= k;
  h = rotl32(h, 13);
  h = h * 5u + 0xe6546b64u;
  h ^= 4u;
  h ^= h >> 16;
  h *= 0x85ebca6bu;
  h ^= h >> 13;
  h *= 0xc2b2ae35u;
  h ^= h >> 16;
  return h;
}

void oracle_minhash_sketch(int64_t nb, const int32_t *brp, const int32_t *bci, uint32_t *sketch) {
  int nt = oracle_num_threads();
#pragma omp parallel for schedule(static) num_threads(nt)
  for (int64_t r = 0; r < nb; ++r) {
    uint32_t *s = sketch + r * 128;
    for (int t = 0; t < 128; ++t) s[t] = 0xffffffffu;
    for (int32_t p = brp[r]; p < brp[r + 1]; ++p) {
      const uint32_t h = oracle_murmur3((uint32_t)bci[p]);
      const uint32_t slot = h & 127u;
      if (h < s[slot]) s[slot] = h;
    }
  }
}

/* HyperLogLog alternative (hll_construct_kernel / hll_merge_kernel,
 * src/spgemm_kernel_hash.cu:94-240; EST_METHOD=hll): 128 one-byte registers per B row
 * (register = low 7 bits of the hash, rank = leading zeros + 1 capped at 26), max-merged per A
 * row; estimate 0.715 * 128 * 128 / sum(2^-reg), or 128 * ln(128 / empty) when registers are
 * empty and the raw estimate is at most 320; x1.5 and the same bin snap as MinHash. The sum is
 * exact in double (powers of two between 2^-26 and 1), so its order is irrelevant. */
static int oracle_clz32(uint32_t x) {
  int n = 0;
  if (x == 0) return 32;
  while (!(x & 0x80000000u)) {
    x <<= 1;
    ++n;
  }
  return n;
}

void oracle_hll_registers(int64_t nb, const int32_t *brp, const int32_t *bci, uint8_t *regs) {
  int nt = oracle_num_threads();
#pragma omp parallel for schedule(static) num_threads(nt)
  for (int64_t r = 0; r < nb; ++r) {
    uint8_t *g = regs + r * 128;
    for (int t = 0; t < 128; ++t) g[t] = 0;
    for (int32_t p = brp[r]; p < brp[r + 1]; ++p) {
      const uint32_t h = oracle_murmur3((uint32_t)bci[p]);
      uint32_t rho = (uint32_t)oracle_clz32(h) + 1u;
      if (rho > 26u) rho = 26u;
      if (rho > g[h & 127u]) g[h & 127u] = (uint8_t)rho;
    }
  }
}

void oracle_hll_merge(int64_t m, const int32_t *arp, const int32_t *aci, const uint8_t *regs,
                      int32_t *est) {
  int nt = oracle_num_threads();
#pragma omp parallel for schedule(static) num_threads(nt)
  for (int64_t i = 0; i < m; ++i) {
    uint8_t mx[128];
    for (int t = 0; t < 128; ++t) mx[t] = 0;
    for (int32_t p = arp[i]; p < arp[i + 1]; ++p) {
      const uint8_t *g = regs + (int64_t)aci[p] * 128;
      for (int t = 0; t < 128; ++t)
        if (g[t] > mx[t]) mx[t] = g[t];
    }
    double z = 0.0;
    int empty = 0;
    for (int t = 0; t < 128; ++t) {
      z += 1.0 / (double)(1ull << mx[t]);
      empty += mx[t] == 0;
    }
    double E = 0.715 * 128.0 * 128.0 / z;
    if (empty != 0 && E <= 2.5 * 128) E = 128.0 * log(128.0 / (double)empty);
    int temp = (int)(E * 1.5);
    if (temp < 1) temp = 1;
    int e;
    if (temp <= 16) {
      e = temp;
    } else {
      int ht = 32;
      while (ht < temp && ht < 16384) ht <<= 1;
      e = ht;
    }
    est[i] = e;
  }
}

/* est per A row from B's sketches: min-merge, then the reference's estimate and bin snap.
 * The sum of 1/min follows the device order: 32 lanes x 4 partitions, then a shuffle-down tree. */
void oracle_minhash_merge(int64_t m, const int32_t *arp, const int32_t *aci,
                          const uint32_t *sketch, int32_t *est) {
  int nt = oracle_num_threads();
#pragma omp parallel for schedule(static) num_threads(nt)
  for (int64_t i = 0; i < m; ++i) {
    uint32_t mn[128];
    for (int t = 0; t < 128; ++t) mn[t] = 0xffffffffu;
    for (int32_t p = arp[i]; p < arp[i + 1]; ++p) {
      const uint32_t *s = sketch + (int64_t)aci[p] * 128;
      for (int t = 0; t < 128; ++t)
        if (s[t] < mn[t]) mn[t] = s[t];
    }
    double part[32];
    int vcnt[32];
    for (int l = 0; l < 32; ++l) {
      double sum = 0.0;
      int V = 0;
      for (int q = 0; q < 4; ++q) {
        const uint32_t x = mn[4 * l + q];
        if (x != 0xffffffffu) {
          sum += 1.0 / (double)x;
          ++V;
        }
      }
      part[l] = sum;
      vcnt[l] = V;
    }
    for (int off = 16; off > 0; off >>= 1) {
      double np_[32];
      int nv[32];
      for (int l = 0; l < 32; ++l) {
        const int src = (l + off < 32) ? l + off : l;
        np_[l] = part[l] + part[src];
        nv[l] = vcnt[l] + vcnt[src];
      }
      memcpy(part, np_, sizeof(part));
      memcpy(vcnt, nv, sizeof(vcnt));
    }
    const double sum_inv = part[0];
    const int V = vcnt[0];
    double E;
    if (V == 0) E = 0.0;
    else if (V < 128) E = 128.0 * log(128.0 / (double)(128 - V));
    else E = 4294967296.0 * sum_inv - 128.0;
    int temp = (int)(E * 1.5);
    if (temp < 1) temp = 1;
    int e;
    if (temp <= 16) {
      e = temp;
    } else {
      int ht = 32;
      while (ht < temp && ht < 16384) ht <<= 1;
      e = ht;
    }
    est[i] = e;
  }
}
