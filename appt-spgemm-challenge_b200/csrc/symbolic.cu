// Symbolic phase: exact number of distinct output columns of every row of C.
//
// Reference counterpart: the per-row distinct count that the reference gets as a side effect of
// hash accumulation (hash_spa_kernel's `cnt`, spgemm_kernel_hash.cu:373-458) or from
// bucket_count_kernel (spgemm_merge.cu:531-571). Here it is a separate, insert-only pass so that
// C can be allocated exactly once and the numeric pass writes every entry to its final place
// (no estimate-sized scratch buffer and no compaction copy).
//
// Two table kinds share one shared-memory budget per warp:
//   * bitmap over the row's column span [lo, hi]  (one atomicOr per product, new bits counted)
//   * open-addressing key hash with Fibonacci slots sized to >= 2 x products (never fills)
// and rows with <= 32 products and <= 32 A entries use warp match in registers (no table).
#include <climits>
#include "common.cuh"
#include "kernels.cuh"
#include "walk.cuh"

namespace appt {

namespace {

template <int WORDS, int WPB>
__global__ void __launch_bounds__(WPB * 32) sym_warp_kernel(const int* rows, const long long* bin_off,
                                                            int bin, Csr A, Csr B, int upper,
                                                            int row_base, const int* lo_arr,
                                                            const int* hi_arr,
                                                            const long long* flop_arr,
                                                            int* row_nnz, int* err) {
  extern __shared__ unsigned sym_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned* tab = sym_smem + warp * WORDS;
  const long long b0 = bin_off[bin];
  const long long nrows = bin_off[bin + 1] - b0;
  for (long long r = (long long)blockIdx.x * WPB + warp; r < nrows;
       r += (long long)gridDim.x * WPB) {
    const int i = rows[b0 + r];
    const int ig = i + row_base;
    const int lo = lo_arr[i], hi = hi_arr[i];
    const long long f = flop_arr[i];
    const int rs = A.rp[i], re = A.rp[i + 1];
    int cnt = 0;
    if (f <= 32 && re - rs <= 32) {
      // register path: at most one product per lane
      const int p = rs + lane;
      const bool v = p < re;
      const int k = v ? A.ci[p] : 0;
      const int bs = v ? B.rp[k] : 0;
      const int len = v ? B.rp[k + 1] - bs : 0;
      const int incl = warp_incl_scan(len);
      const int excl = incl - len;
      const int total = __shfl_sync(kFull, incl, 31);
      const int L = warp_owner(excl, lane);
      const int bsL = __shfl_sync(kFull, bs, L), exL = __shfl_sync(kFull, excl, L);
      int j = -1;
      if (lane < total) {
        j = B.ci[bsL + lane - exL];
        if (upper && j < ig) j = -1;
      }
      const unsigned peers = __match_any_sync(kFull, j);
      const bool lead = (j >= 0) && (lane == __ffs(peers) - 1);
      cnt = __popc(__ballot_sync(kFull, lead));
    } else {
      const long long span = (long long)hi - lo + 1;
      const int words_bm = (int)((span + 31) >> 5);
      const int lg = ilog2_ceil(f * 2 < 32 ? 32 : f * 2);
      const bool bm_ok = span <= 32ll * WORDS;
      const bool h_ok = lg <= 30 && (1 << lg) <= WORDS;
      if (!bm_ok && !h_ok) {
        if (lane == 0) {
          set_error(err, kErrCapacity);
          row_nnz[i] = 0;
        }
        continue;
      }
      const int hslots = h_ok ? (1 << lg) : 0;
      const bool bitmap = bm_ok && (!h_ok || words_bm <= 2 * hslots);
      const int nclear = bitmap ? words_bm : hslots;
      const unsigned fill = bitmap ? 0u : kEmptyKey;
      for (int w = lane; w < nclear; w += 32) tab[w] = fill;
      __syncwarp();
      bool overflow = false;
      for (int base = rs; base < re; base += 32) {
        const int p = base + lane;
        const bool v = p < re;
        const int k = v ? A.ci[p] : 0;
        const int bs = v ? B.rp[k] : 0;
        const int len = v ? B.rp[k + 1] - bs : 0;
        const int incl = warp_incl_scan(len);
        const int excl = incl - len;
        const int total = __shfl_sync(kFull, incl, 31);
        for (int t0 = 0; t0 < total; t0 += 32) {
          const int t = t0 + lane;
          const int L = warp_owner(excl, t);
          const int bsL = __shfl_sync(kFull, bs, L), exL = __shfl_sync(kFull, excl, L);
          if (t < total) {
            const int j = B.ci[bsL + t - exL];
            if (upper && j < ig) continue;
            if (bitmap) {
              const unsigned off = (unsigned)(j - lo);
              if (off >= (unsigned)span) {   // B row not sorted / outside the span
                overflow = true;
                continue;
              }
              const unsigned bit = 1u << (off & 31);
              const unsigned old = atomicOr(&tab[off >> 5], bit);
              cnt += (old & bit) ? 0 : 1;
            } else {
              unsigned s = hash_slot((unsigned)j, lg);
              int probe = 0;
              for (; probe < hslots; ++probe) {
                const unsigned old = atomicCAS(&tab[s], kEmptyKey, (unsigned)j);
                if (old == kEmptyKey) { ++cnt; break; }
                if (old == (unsigned)j) break;
                s = (s + 1) & (unsigned)(hslots - 1);
              }
              if (probe == hslots) overflow = true;
            }
          }
        }
      }
      if (__any_sync(kFull, overflow) && lane == 0) set_error(err, kErrTableFull);
      cnt = warp_sum(cnt);
      __syncwarp();
    }
    if (lane == 0) row_nnz[i] = cnt;
  }
}

// Warp per row, bitmap over [lo, hi] (at most WORDS words), filled with fire-and-forget shared
// OR operations, then counted. G lane groups share the warp (rows whose B rows are short; see
// walk.cuh). Rows that could fit the rank tier and whose products outweigh their bitmap
// (handoff_pays) also copy the finished bitmap out (coalesced, logical word order) into the
// handoff arena, in chunks the warp takes with one atomic each, for the numeric rank tier.
#ifndef APPT_SYM_MIN_BLOCKS
#define APPT_SYM_MIN_BLOCKS 5  // resident 256-thread CTAs per SM the register budget targets
#endif
template <int WORDS, int WPB, int G>
__global__ void __launch_bounds__(WPB * 32, WORDS <= 1024 ? APPT_SYM_MIN_BLOCKS : 3)
    sym_warp_bitmap_kernel(const int* rows, const long long* bin_off, int bin, Csr A, Csr B,
                           int upper, int row_base, const int* lo_arr, const int* hi_arr,
                           const long long* flop_arr, int* row_nnz, RowBitmaps handoff,
                           int* err) {
  extern __shared__ unsigned sym_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned* bm = sym_smem + warp * WORDS;
  const long long b0 = bin_off[bin];
  const long long nrows = bin_off[bin + 1] - b0;
  long long chunk_cur = 0, chunk_end = 0;   // this warp's piece of the handoff arena
  // rows are software-pipelined: the next row's metadata and the id of the row after it are
  // loaded while the current row is processed
  const long long stride = (long long)gridDim.x * WPB;
  long long r = (long long)blockIdx.x * WPB + warp;
  int i_n = r < nrows ? rows[b0 + r] : 0;
  int i_nn = r + stride < nrows ? rows[b0 + r + stride] : 0;
  int lo_n = 0, hi_n = -1, rs_n = 0, re_n = 0;
  long long fl_n = 0;
  if (r < nrows) {
    lo_n = lo_arr[i_n];
    hi_n = hi_arr[i_n];
    rs_n = A.rp[i_n];
    re_n = A.rp[i_n + 1];
    fl_n = flop_arr[i_n];
  }
  for (; r < nrows; r += stride) {
    const int i = i_n, lo = lo_n, rs = rs_n, re = re_n;
    const long long span = (long long)hi_n - lo + 1;
    const long long flop = fl_n;
    i_n = i_nn;
    if (r + stride < nrows) {
      lo_n = lo_arr[i_n];
      hi_n = hi_arr[i_n];
      rs_n = A.rp[i_n];
      re_n = A.rp[i_n + 1];
      fl_n = flop_arr[i_n];
    }
    if (r + 2 * stride < nrows) i_nn = rows[b0 + r + 2 * stride];
    const int W = span <= 32ll * WORDS ? bitmap_words(span) : WORDS + 1;
    if (span <= 0 || W > WORDS) {
      if (lane == 0) {
        set_error(err, kErrCapacity);
        row_nnz[i] = 0;
      }
      continue;
    }
    for (int w = lane; w < W; w += 32) bm[w] = 0u;
    __syncwarp();
    const bool bad = fill_row_bitmap_g<G>(A, B, rs, re, lo, (unsigned)span, bm);
    __syncwarp();
    int cnt = 0;
    for (int w = lane; w < W; w += 32) cnt += __popc(bm[w]);
    cnt = warp_sum(cnt);
    if (__any_sync(kFull, bad) && lane == 0) set_error(err, kErrCapacity);
    if (lane == 0) row_nnz[i] = cnt;
    if (handoff.data && handoff_fits_rank(W) && handoff_pays(flop, W)) {
      if (chunk_cur + W > chunk_end) {
        unsigned long long c = 0;
        if (lane == 0) c = atomicAdd(handoff.top, (unsigned long long)kHandoffChunkWords);
        c = __shfl_sync(kFull, c, 0);
        chunk_cur = (long long)c;
        chunk_end = chunk_cur + kHandoffChunkWords;
        if (chunk_end > handoff.capacity) chunk_end = chunk_cur;   // arena exhausted
      }
      if (chunk_cur + W <= chunk_end) {
        unsigned* out = handoff.data + chunk_cur;
        for (int w = lane; w < W; w += 32) out[w] = bm[swz(w)];
        if (lane == 0) handoff.slot[i] = (int)(chunk_cur >> 5);
        chunk_cur += W;
      }
    }
    __syncwarp();
  }
}

template <int WORDS, int WPB, int G>
void launch_sym_bitmap_g(int bin, const int* rows, const long long* bin_off, Csr A, Csr B,
                         int upper, int row_base, const int* lo, const int* hi,
                         const long long* flop, int* row_nnz, RowBitmaps handoff, int* err,
                         int num_sms, cudaStream_t s) {
  const size_t smem = (size_t)WORDS * WPB * sizeof(unsigned);
  auto kern = sym_warp_bitmap_kernel<WORDS, WPB, G>;
  smem_opt_in((const void*)kern, smem);
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, WPB * 32, smem);
  if (occ < 1) occ = 1;
  kern<<<num_sms * occ, WPB * 32, smem, s>>>(rows, bin_off, bin, A, B, upper, row_base, lo, hi,
                                              flop, row_nnz, handoff, err);
}

// gidx: 0, 1, 2 for G = 1, 2, 4 lane groups.
template <int WORDS, int WPB>
void launch_sym_bitmap(int bin, int gidx, const int* rows, const long long* bin_off, Csr A,
                       Csr B, int upper, int row_base, const int* lo, const int* hi,
                       const long long* flop, int* row_nnz, RowBitmaps handoff, int* err,
                       int num_sms, cudaStream_t s) {
  if (gidx == 2)
    launch_sym_bitmap_g<WORDS, WPB, 4>(bin, rows, bin_off, A, B, upper, row_base, lo, hi, flop,
                                       row_nnz, handoff, err, num_sms, s);
  else if (gidx == 1)
    launch_sym_bitmap_g<WORDS, WPB, 2>(bin, rows, bin_off, A, B, upper, row_base, lo, hi, flop,
                                       row_nnz, handoff, err, num_sms, s);
  else
    launch_sym_bitmap_g<WORDS, WPB, 1>(bin, rows, bin_off, A, B, upper, row_base, lo, hi, flop,
                                       row_nnz, handoff, err, num_sms, s);
}

// CTA per row (rows taken dynamically from a counter). Bitmap windows of WB words (32 * WB
// columns) over [lo, hi]; rows whose span exceeds one window restrict every B row to the window
// by binary search (B rows are sorted). The warps share the products in pieces
// (load_block_chunk, walk.cuh), set bits with fire-and-forget shared OR operations, and the
// window's columns are counted by popcount. B rows kept as bitmaps (`dense`) are ORed in a word
// at a time instead.
template <int NT, int WB>
__global__ void __launch_bounds__(NT, 1) sym_block_kernel(const int* rows, const long long* bin_off,
                                                          int bin, Csr A, Csr B, const int* lo_arr,
                                                          const int* hi_arr, DenseRows dense,
                                                          int* row_nnz, int* row_counter) {
  extern __shared__ __align__(16) unsigned char sym_block_smem[];
  constexpr int NW = NT / 32;
  constexpr long long WCOLS = 32ll * WB;
  unsigned* bm = reinterpret_cast<unsigned*>(sym_block_smem);   // [WB]
  BlockChunk ch;
  ch.a = reinterpret_cast<double*>(bm + WB);                     // [NT] (unused here)
  ch.piece_ex = reinterpret_cast<int*>(ch.a + NT);               // [NT]
  ch.bs = ch.piece_ex + NT;                                      // [NT]
  ch.be = ch.bs + NT;                                            // [NT]
  int* dlist = ch.be + NT;                                       // [NT]
  __shared__ long long sbuf[NW + 1];
  __shared__ long long s_row;
  __shared__ int s_dcount;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long b0 = bin_off[bin];
  const long long nrows = bin_off[bin + 1] - b0;
  for (;;) {
    if (tid == 0) s_row = atomicAdd(row_counter, 1);
    __syncthreads();
    const long long r = s_row;
    if (r >= nrows) break;
    const int i = rows[b0 + r];
    const int lo = lo_arr[i], hi = hi_arr[i];
    const int rs = A.rp[i], re = A.rp[i + 1];
    const bool multi = (long long)hi - lo + 1 > WCOLS;
    long long cnt = 0;
    for (long long w0 = lo; w0 <= hi; w0 += WCOLS) {
      const long long w1 = (w0 + WCOLS < (long long)hi + 1) ? w0 + WCOLS : (long long)hi + 1;
      const unsigned span = (unsigned)(w1 - w0);
      const int W = (int)((span + 31) >> 5);
      for (int w = tid; w < W; w += NT) bm[w] = 0u;
      for (int cb = rs; cb < re; cb += NT) {
        const int cn = (re - cb) < NT ? (re - cb) : NT;
        const int tp = load_block_chunk<NT>(A, B, cb, re, multi, w0, w1, ch, sbuf, dense.id,
                                            dlist, &s_dcount);
        for (int it = warp; it < tp; it += NW) {
          const int L = search_le(ch.piece_ex, cn, it);
          const int q0 = ch.bs[L] + (it - ch.piece_ex[L]) * kPiece;
          const int q1 = (q0 + kPiece < ch.be[L]) ? q0 + kPiece : ch.be[L];
          for (int q = q0 + lane; q < q1; q += 128) {
            PieceRound pr;
            load_piece_round<false>(B, q, q1, w0, pr);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              red_or_shared_if(pr.off[u] < span, bm + (pr.off[u] >> 5), 1u << (pr.off[u] & 31));
          }
        }
        __syncthreads();
        if (dense.id && s_dcount > 0) {   // block-uniform
          or_dense_rows<NT>(bm, W, span, w0, dense, ch, dlist, s_dcount);
          __syncthreads();
        }
      }
      int c = 0;
      for (int w = tid; w < W; w += NT) c += __popc(bm[w]);
      long long tot;
      block_excl_scan_ll<NT>(c, sbuf, &tot);
      cnt += tot;
    }
    if (tid == 0) row_nnz[i] = (int)(cnt < 0x7fffffffll ? cnt : 0x7fffffffll);
    __syncthreads();
  }
}

template <int WORDS, int WPB>
void launch_sym_warp(int bin, const int* rows, const long long* bin_off, Csr A, Csr B, int upper,
                     int row_base, const int* lo, const int* hi, const long long* flop,
                     int* row_nnz, int* err, int num_sms, cudaStream_t s) {
  const size_t smem = (size_t)WORDS * WPB * sizeof(unsigned);
  auto kern = sym_warp_kernel<WORDS, WPB>;
  smem_opt_in((const void*)kern, smem);
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, WPB * 32, smem);
  if (occ < 1) occ = 1;
  kern<<<num_sms * occ, WPB * 32, smem, s>>>(rows, bin_off, bin, A, B, upper, row_base, lo, hi,
                                              flop, row_nnz, err);
}

// Small problems: warp per row over every row of A (no binning) computes the row's column span
// and exact count in one pass with a bitmap of at most WORDS words, writes lo / hi for the rank
// tier, and sets kErrSmallFallback (row_nnz 0) for a row whose bitmap or rank-tier layout would
// not fit, after which the caller runs the general pipeline. Such a row also raises a flag in its
// CTA's shared memory, and the CTA's warps stop at their next row: the pass's results are then
// discarded (the general pipeline's analyze repeats the bounds check). The flag is per CTA on
// purpose: a global stop word polled by every warp on every row queues all those reads at one L2
// slice and slowed the pass even when no row fell back. bin_off receives {0, m}.
template <int WORDS, int WPB, int G>
__global__ void __launch_bounds__(WPB * 32) sym_small_kernel(Csr A, Csr B, int upper,
                                                            int row_base, int* lo_arr,
                                                            int* hi_arr, int* row_nnz,
                                                            long long* bin_off,
                                                            unsigned long long* total_flop,
                                                            int* err) {
  extern __shared__ unsigned sym_smem[];
  __shared__ int cta_stop;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned* bm = sym_smem + warp * WORDS;
  const int m = A.rows;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    bin_off[0] = 0;
    bin_off[1] = m;
  }
  if (threadIdx.x == 0) cta_stop = 0;
  __syncthreads();
  for (long long r = (long long)blockIdx.x * WPB + warp; r < m; r += (long long)gridDim.x * WPB) {
    if (__shfl_sync(kFull, *(volatile int*)&cta_stop, 0)) break;
    const int i = (int)r;
    const int rs = A.rp[i], re = A.rp[i + 1];
    int lo = INT_MAX, hi = -1, bad = 0;
    long long f = 0;
    for (int p = rs + lane; p < re; p += 32) {
      const int k = A.ci[p];
      if ((unsigned)k >= (unsigned)B.rows) {
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
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo = min(lo, __shfl_xor_sync(kFull, lo, o));
      hi = max(hi, __shfl_xor_sync(kFull, hi, o));
      bad |= __shfl_xor_sync(kFull, bad, o);
      f += __shfl_xor_sync(kFull, f, o);
    }
    if (lane == 0 && f) atomicAdd(total_flop, (unsigned long long)f);
    if (upper && lo < i + row_base) lo = i + row_base;
    if (bad) {
      if (lane == 0) {
        set_error(err, kErrBounds);
        row_nnz[i] = 0;
      }
      continue;
    }
    const long long span = (long long)hi - lo + 1;
    if (lane == 0) {
      lo_arr[i] = lo;
      hi_arr[i] = hi;
    }
    if (span <= 0) {
      if (lane == 0) row_nnz[i] = 0;
      continue;
    }
    const int W = span <= 32ll * WORDS ? bitmap_words(span) : WORDS + 1;
    if (W > WORDS || 6ll * W + 20 > kRankMaxBudget) {
      if (lane == 0) {
        set_error(err, kErrSmallFallback);
        *(volatile int*)&cta_stop = 1;
        row_nnz[i] = 0;
      }
      continue;
    }
    for (int w = lane; w < W; w += 32) bm[w] = 0u;
    __syncwarp();
    const bool fbad = fill_row_bitmap_g<G>(A, B, rs, re, lo, (unsigned)span, bm);
    __syncwarp();
    int cnt = 0;
    for (int w = lane; w < W; w += 32) cnt += __popc(bm[w]);
    cnt = warp_sum(cnt);
    if (lane == 0) {
      row_nnz[i] = cnt;
      if (fbad) set_error(err, kErrCapacity);
      const long long need = 6ll * W + 10ll * (cnt + 1);   // the row's rank-tier budget
      if (need > kRankMaxBudget) {
        set_error(err, kErrSmallFallback);
        *(volatile int*)&cta_stop = 1;
      } else {
        atomicMax(err + 1, (int)need);   // the numeric launch picks the smallest budget
      }
    }
    __syncwarp();
  }
}

template <int G>
void run_sym_small(Csr A, Csr B, int upper, int row_base, int* lo, int* hi, int* row_nnz,
                   long long* bin_off, unsigned long long* total_flop, int* err, int num_sms,
                   cudaStream_t s) {
  constexpr int WORDS = 1536, WPB = 8;
  const size_t smem = (size_t)WORDS * WPB * sizeof(unsigned);
  auto kern = sym_small_kernel<WORDS, WPB, G>;
  smem_opt_in((const void*)kern, smem);
  long long blocks = ((long long)A.rows + WPB - 1) / WPB;
  if (blocks > (long long)num_sms * 4) blocks = (long long)num_sms * 4;
  if (blocks < 1) blocks = 1;
  kern<<<(unsigned)blocks, WPB * 32, smem, s>>>(A, B, upper, row_base, lo, hi, row_nnz, bin_off,
                                                total_flop, err);
}

}  // namespace

// ---------------------------------------------------------------------------- dense B rows
__global__ void dense_mark_kernel(Csr B, int* id, int* list, int max_rows, int* counter) {
  const long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (k >= B.rows) return;
  const int len = B.rp[k + 1] - B.rp[k];
  int slot = -1;
  if (len > 0 && 32ll * len >= B.cols) {
    slot = atomicAdd(counter, 1);
    if (slot < max_rows)
      list[slot] = (int)k;
    else
      slot = -1;
  }
  id[k] = slot;
}

__global__ void __launch_bounds__(256) dense_fill_kernel(Csr B, const int* list,
                                                         const int* counter, int max_rows,
                                                         unsigned* bits, unsigned* pre,
                                                         long long stride) {
  __shared__ long long sbuf[256 / 32 + 1];
  const int cnt = *counter < max_rows ? *counter : max_rows;
  const int per = (int)((stride + 255) / 256);   // words per thread in the prefix
  for (int d = blockIdx.x; d < cnt; d += gridDim.x) {
    const int k = list[d];
    unsigned* row = bits + (size_t)d * stride;
    for (long long w = threadIdx.x; w < stride; w += blockDim.x) row[w] = 0u;
    __syncthreads();
    const int e1 = B.rp[k + 1];
    for (int e = B.rp[k] + threadIdx.x; e < e1; e += blockDim.x) {
      const int c = B.ci[e];
      atomicOr(row + (c >> 5), 1u << (c & 31));
    }
    __syncthreads();
    const long long wa = (long long)threadIdx.x * per;
    const long long wb = wa + per < stride ? wa + per : stride;
    long long c = 0;
    for (long long w = wa; w < wb; ++w) c += __popc(row[w]);
    long long tot;
    long long run = block_excl_scan_ll<256>(c, sbuf, &tot);
    unsigned* prow = pre + (size_t)d * stride;
    for (long long w = wa; w < wb; ++w) {
      prow[w] = (unsigned)run;
      run += __popc(row[w]);
    }
    __syncthreads();
  }
}

int build_dense_rows(Csr B, int* id, int* list, unsigned* bits, unsigned* pre, long long stride,
                     int max_rows, int* counter, int num_sms, cudaStream_t s) {
  if (B.rows <= 0 || max_rows <= 0) return 0;
  dense_mark_kernel<<<(unsigned)((B.rows + 255) / 256), 256, 0, s>>>(B, id, list, max_rows,
                                                                      counter);
  const int grid = max_rows < 4 * num_sms ? max_rows : 4 * num_sms;
  dense_fill_kernel<<<grid, 256, 0, s>>>(B, list, counter, max_rows, bits, pre, stride);
  return 2;
}

void launch_symbolic_small(Csr A, Csr B, int upper, int row_base, int gidx, int* lo, int* hi,
                           int* row_nnz, long long* bin_off, unsigned long long* total_flop,
                           int* err, int num_sms, cudaStream_t s) {
  if (gidx == 2)
    run_sym_small<4>(A, B, upper, row_base, lo, hi, row_nnz, bin_off, total_flop, err,
                     num_sms, s);
  else if (gidx == 1)
    run_sym_small<2>(A, B, upper, row_base, lo, hi, row_nnz, bin_off, total_flop, err,
                     num_sms, s);
  else
    run_sym_small<1>(A, B, upper, row_base, lo, hi, row_nnz, bin_off, total_flop, err,
                     num_sms, s);
}

void launch_symbolic(int bin, const int* rows, const long long* bin_off, Csr A, Csr B, int upper,
                     int row_base, const int* lo, const int* hi, const long long* flop,
                     int* row_nnz, RowBitmaps handoff, DenseRows dense, int* row_counter,
                     int* err, int num_sms, cudaStream_t s) {
  if (bin >= kSymBmS && bin < kSymBmM) {
    launch_sym_bitmap<256, 8>(bin, bin - kSymBmS, rows, bin_off, A, B, upper, row_base, lo, hi,
                              flop, row_nnz, handoff, err, num_sms, s);
    return;
  }
  if (bin >= kSymBmM && bin < kSymBmL) {
    launch_sym_bitmap<1024, 8>(bin, bin - kSymBmM, rows, bin_off, A, B, upper, row_base, lo, hi,
                               flop, row_nnz, handoff, err, num_sms, s);
    return;
  }
  if (bin >= kSymBmL && bin < kSymHashS) {
    launch_sym_bitmap<4096, 4>(bin, bin - kSymBmL, rows, bin_off, A, B, upper, row_base, lo, hi,
                               flop, row_nnz, handoff, err, num_sms, s);
    return;
  }
  switch (bin) {
    case kSymHashS:
      launch_sym_warp<256, 8>(bin, rows, bin_off, A, B, upper, row_base, lo, hi, flop, row_nnz,
                              err, num_sms, s);
      break;
    case kSymHashM:
      launch_sym_warp<1024, 8>(bin, rows, bin_off, A, B, upper, row_base, lo, hi, flop, row_nnz,
                               err, num_sms, s);
      break;
    case kSymHashL:
      launch_sym_warp<4096, 4>(bin, rows, bin_off, A, B, upper, row_base, lo, hi, flop, row_nnz,
                               err, num_sms, s);
      break;
    case kSymBlock: {
      constexpr int NT = 1024;
      const size_t smem = (size_t)kSymBlockWords * 4 + (size_t)NT * (8 + 12 + 4);
      auto kern = sym_block_kernel<NT, kSymBlockWords>;
      smem_opt_in((const void*)kern, smem);
      kern<<<num_sms, NT, smem, s>>>(rows, bin_off, bin, A, B, lo, hi, dense, row_nnz,
                                     row_counter);
      break;
    }
    default:
      break;
  }
}

}  // namespace appt
