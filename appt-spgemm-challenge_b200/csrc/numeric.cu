// Numeric phase: accumulate a_ik * b_kj for every row of C and write the row, sorted by column,
// straight to its final place (row offsets come from the exact symbolic count).
//
// Reference counterparts: hash_spa_kernel + hash_ultra_kernel (spgemm_kernel_hash.cu:373-458,
// 573-608) followed by hash_compact_sort_kernel / hash_compact_copy_kernel (:635-674, 773-786).
// The reference accumulates into an estimate-sized scratch buffer and sorts/copies it into C in
// a second pass; here each tier sorts inside shared memory and stores C once.
//
// Tiers (bins chosen by the classifier in analyze.cu):
//   rank    warp per row; bitmap over the row's span + 16-bit popcount prefix gives every
//           column its output position, values accumulate there directly (no table, no sort)
//   hash    warp per row; table of T slots (int key + fp64 value), compaction, warp bitonic sort
//   hashB   CTA per row; 8192-slot table, block bitonic sort
//   window  CTA per row; dense windows of 8192 columns walked over the row's span (heavy rows)
// The warp tiers visit products k-sequentially (walk.cuh) and round like the sequential
// algorithm (no FMA), so their sums are bit-identical to the CPU oracle's; the CTA tiers
// accumulate with shared-memory atomics (order-dependent rounding, within the tolerance).
#include <climits>
#include "common.cuh"
#include "kernels.cuh"
#include "walk.cuh"

namespace appt {

namespace {

// --------------------------------------------------------------------------- warp hash tier
template <int T, int WPB>
__global__ void __launch_bounds__(WPB * 32, 2048 / (WPB * 32) * 3 / 4) num_warp_hash_kernel(
    const int* rows, const long long* bin_off, int bin, Csr A, Csr B, int upper, int row_base,
    const long long* crp, int* cci, double* cval, int* err) {
  extern __shared__ __align__(16) unsigned char num_smem[];
  constexpr int LG = (T == 64) ? 6 : (T == 128) ? 7 : (T == 256) ? 8 : (T == 512) ? 9 : 10;
  static_assert((1 << LG) == T, "table size must be a power of two in [64, 1024]");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double* vals = reinterpret_cast<double*>(num_smem) + warp * T;
  int* keys = reinterpret_cast<int*>(reinterpret_cast<double*>(num_smem) + WPB * T) + warp * T;
  const long long b0 = bin_off[bin];
  const long long nrows = bin_off[bin + 1] - b0;
  for (long long r = (long long)blockIdx.x * WPB + warp; r < nrows;
       r += (long long)gridDim.x * WPB) {
    const int i = rows[b0 + r];
    const int ig = i + row_base;
    const int rs = A.rp[i], re = A.rp[i + 1];
    const long long c0 = crp[i];
    const int n = (int)(crp[i + 1] - c0);
    for (int s = lane; s < T; s += 32) {
      keys[s] = -1;
      vals[s] = 0.0;
    }
    __syncwarp();
    bool overflow = false;
    walk_row_k_sequential<true>(A, B, rs, re, [&](int j, double x, double a) {
      if (upper && j < ig) return;
      unsigned s = hash_slot((unsigned)j, LG);
      int probe = 0;
      for (; probe < T; ++probe) {
        const int old = atomicCAS(&keys[s], -1, j);
        if (old == -1 || old == j) {
          // one lane per column in a step: a plain update, ordered across steps by the walk
          vals[s] = mul_add_rn(vals[s], a, x);
          break;
        }
        s = (s + 1) & (T - 1);
      }
      if (probe == T) overflow = true;
    });
    __syncwarp();
    // compact the occupied slots to the front (reads of a chunk precede its writes)
    int pos = 0;
    for (int c = 0; c < T; c += 32) {
      const int kk = keys[c + lane];
      const double vv = vals[c + lane];
      const bool valid = kk >= 0;
      const unsigned bal = __ballot_sync(kFull, valid);
      __syncwarp();
      if (valid) {
        const int d = pos + __popc(bal & lanemask_lt());
        keys[d] = kk;
        vals[d] = vv;
      }
      pos += __popc(bal);
      __syncwarp();
    }
    int P2 = 1;
    while (P2 < pos) P2 <<= 1;
    for (int x = pos + lane; x < P2; x += 32) keys[x] = INT_MAX;
    __syncwarp();
    for (int kk = 2; kk <= P2; kk <<= 1) {
      for (int jj = kk >> 1; jj > 0; jj >>= 1) {
        for (int x = lane; x < P2; x += 32) {
          const int y = x ^ jj;
          if (y > x) {
            const int kx = keys[x], ky = keys[y];
            const bool up = (x & kk) == 0;
            if ((kx > ky) == up) {
              keys[x] = ky;
              keys[y] = kx;
              const double tv = vals[x];
              vals[x] = vals[y];
              vals[y] = tv;
            }
          }
        }
        __syncwarp();
      }
    }
    const int nw = pos < n ? pos : n;
    const bool any_overflow = __any_sync(kFull, overflow);
    if (lane == 0 && (pos != n || any_overflow)) set_error(err, kErrTableFull);
    for (int t = lane; t < nw; t += 32) {
      cci[c0 + t] = keys[t];
      cval[c0 + t] = vals[t];
    }
    __syncwarp();
  }
}

// --------------------------------------------------------------------------- warp rank tier
// Row layout in the warp's shared budget: bitmap over [lo, hi] in 32-bit words (W words), a
// 16-bit exclusive popcount prefix per word, the fp64 accumulator of the row's nnz entries and
// the 16-bit column offset (j - lo) of every rank, so the finished row is copied out coalesced.
// For the upper-triangle variants lo is already raised to the row's own index.
// The bitmap is rebuilt from the products, after which the output position of column j is
// prefix[w] + popcount(bitmap[w] & below(j)) -- values accumulate directly in output order, so
// the row needs neither a hash table nor a sort. Products are visited k-sequentially (walk.cuh),
// by G lane groups when the row's B rows are short: no atomics on the accumulator, and every sum
// forms in the reference's order.
#ifndef APPT_RANK_MIN_BLOCKS
#define APPT_RANK_MIN_BLOCKS 4  // resident 256-thread CTAs per SM the register budget targets
#endif
template <int BUDGET, int WPB, int G>
__global__ void __launch_bounds__(WPB * 32, BUDGET <= 4608 ? APPT_RANK_MIN_BLOCKS : 7)
    num_warp_rank_kernel(
    const int* rows, const long long* bin_off, int bin, Csr A, Csr B, int upper, int row_base,
    const int* lo_arr, const int* hi_arr, RowBitmaps handoff, const long long* crp, int* cci,
    double* cval, int* err) {
  extern __shared__ __align__(16) unsigned char num_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned char* base = num_smem + (size_t)warp * BUDGET;
  const long long b0 = bin_off[bin];
  const long long nrows = bin_off[bin + 1] - b0;
  for (long long r = (long long)blockIdx.x * WPB + warp; r < nrows;
       r += (long long)gridDim.x * WPB) {
    const int i = rows ? rows[b0 + r] : (int)(b0 + r);   // no row list: every row, in order
    const int lo = lo_arr[i];
    const long long span = (long long)hi_arr[i] - lo + 1;
    const int rs = A.rp[i], re = A.rp[i + 1];
    const long long c0 = crp[i];
    const int n = (int)(crp[i + 1] - c0);
    if (n == 0) continue;   // (only the unbinned small-problem launch passes such rows)
    if (span <= 0 || span > 65536) {
      if (lane == 0) set_error(err, kErrCapacity);
      continue;
    }
    const int W = bitmap_words(span);
    const int acc_off = 6 * W;   // W is a multiple of 32
    if (acc_off + 10 * (n + 1) > BUDGET) {
      if (lane == 0) set_error(err, kErrCapacity);
      continue;
    }
    unsigned* bm = reinterpret_cast<unsigned*>(base);
    unsigned short* pre = reinterpret_cast<unsigned short*>(base + 4 * W);
    double* acc = reinterpret_cast<double*>(base + acc_off);              // n sums + spare
    unsigned short* coff = reinterpret_cast<unsigned short*>(base + acc_off + 8 * (n + 1));
    const unsigned* hbm = nullptr;   // the symbolic phase's bitmap of this row, if handed off
    if (handoff.data) {
      const int hs = handoff.slot[i];
      if (hs >= 0) hbm = handoff.data + 32ll * hs;
    }
    for (int t = lane; t < n; t += 32) acc[t] = 0.0;
    // the first chunk of A entries stays in registers
    int bs, len;
    double a;
    load_chunk(A, B, rs, re, bs, len, &a);
    const int cnt = (re - rs) < 32 ? (re - rs) : 32;
    bool bad = false;
    // 1) presence bitmap of the row's columns: copied in, or built from the products
    if (hbm) {
      for (int w = lane; w < W; w += 32) bm[swz(w)] = __ldg(hbm + w);
      __syncwarp();
    } else {
      for (int w = lane; w < W; w += 32) bm[w] = 0u;
      __syncwarp();
      bad = fill_chunk_bitmap<G>(B, bs, len, cnt, lo, (unsigned)span, bm);
      if (re - rs > 32) bad |= fill_row_bitmap_g<G>(A, B, rs + 32, re, lo, (unsigned)span, bm);
      __syncwarp();
    }
    // 2) exclusive popcount prefix per word
    const int running = bitmap_prefix32(bm, W, pre);
    __syncwarp();
    if (running != n) bad = true;
    // 3) accumulate at the column's rank, k by k; remember the column of every rank
    if (running == n) {
      accumulate_chunk_ranked<G>(B, bs, len, a, cnt, lo, (unsigned)span, n, bm, pre, acc,
                                 coff);
      for (int cb = rs + 32; cb < re; cb += 32) {
        load_chunk(A, B, cb, re, bs, len, &a);
        const int c2 = (re - cb) < 32 ? (re - cb) : 32;
        accumulate_chunk_ranked<G>(B, bs, len, a, c2, lo, (unsigned)span, n, bm, pre, acc,
                                   coff);
      }
      // 4) the row is already in column order: one coalesced copy
      for (int t = lane; t < n; t += 32) {
        cci[c0 + t] = lo + (int)coff[t];
        cval[c0 + t] = acc[t];
      }
    }
    if (__any_sync(kFull, bad) && lane == 0) set_error(err, kErrCapacity);
    __syncwarp();
  }
}

// --------------------------------------------------------------------------- CTA rank tier
// Long rows (more than 4096 entries) whose span is too sparse for dense windows: one CTA per row
// (rows taken dynamically from a counter), the span cut into windows of 32 * MAXW columns. Per
// window: presence bitmap in shared memory, a 16-bit popcount prefix per word relative to the
// owning thread's run of words plus the thread's base, then C's columns are written straight
// from the bitmap (ranks are output positions) with their sums zeroed, and every product is
// added into C at its rank with a global fp64 atomic (the row of C stays in L2 while the CTA
// works on it).
//
template <int NT, int MAXW>
__global__ void __launch_bounds__(NT, 1) num_block_rank_kernel(
    const int* rows, const long long* bin_off, int bin, Csr A, Csr B, const int* lo_arr,
    const int* hi_arr, const long long* crp, int* cci, double* cval, int* row_counter, int* err) {
  extern __shared__ __align__(16) unsigned char num_smem[];
  constexpr int NW = NT / 32;
  constexpr long long WCOLS = 32ll * MAXW;
  unsigned* bm = reinterpret_cast<unsigned*>(num_smem);                   // [MAXW]
  unsigned short* pre = reinterpret_cast<unsigned short*>(bm + MAXW);     // [MAXW]
  unsigned* tbase = reinterpret_cast<unsigned*>(pre + MAXW);              // [NT]
  BlockChunk ch;
  ch.a = reinterpret_cast<double*>(tbase + NT);                           // [NT]
  ch.piece_ex = reinterpret_cast<int*>(ch.a + NT);                        // [NT]
  ch.bs = ch.piece_ex + NT;                                               // [NT]
  ch.be = ch.bs + NT;                                                     // [NT]
  __shared__ long long sbuf[NW + 1];
  __shared__ long long s_row;
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
    const long long c0 = crp[i];
    const long long n = crp[i + 1] - c0;
    const int rs = A.rp[i], re = A.rp[i + 1];
    const bool multi = (long long)hi - lo + 1 > WCOLS;
    long long ob = 0;   // entries emitted by the earlier windows of the row
    for (long long w0 = lo; w0 <= hi; w0 += WCOLS) {
      const long long w1 = (w0 + WCOLS < (long long)hi + 1) ? w0 + WCOLS : (long long)hi + 1;
      const unsigned span = (unsigned)(w1 - w0);
      const int W = (int)((span + 31) >> 5);
      int lp = 0;
      while ((NT << lp) < W) ++lp;   // each thread owns 2^lp consecutive words
      for (int w = tid; w < W; w += NT) bm[w] = 0u;
      // 1) presence bitmap
      for (int cb = rs; cb < re; cb += NT) {
        const int cn = (re - cb) < NT ? (re - cb) : NT;
        const int tp = load_block_chunk<NT>(A, B, cb, re, multi, w0, w1, ch, sbuf);
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
      }
      // 2) ranks: per-thread runs of 2^lp words, 16-bit prefix within the run + run base
      const int wa = tid << lp;
      const int wb = (wa + (1 << lp) < W) ? wa + (1 << lp) : W;
      int c = 0;
      for (int w = wa; w < wb; ++w) c += __popc(bm[w]);
      long long tot;
      const long long ex = block_excl_scan_ll<NT>(c, sbuf, &tot);
      tbase[tid] = (unsigned)ex;
      {
        int run = 0;
        for (int w = wa; w < wb; ++w) {
          pre[w] = (unsigned short)run;
          run += __popc(bm[w]);
        }
      }
      __syncthreads();
      if (ob + tot > n) {   // the symbolic count disagrees: report, write nothing more
        if (tid == 0) set_error(err, kErrCapacity);
        break;
      }
      // 3) columns of C from the bitmap (warp per 32 consecutive words), sums zeroed
      for (int wq = warp * 32; wq < W; wq += NT) {
        const int w = wq + lane;
        unsigned bits = w < W ? bm[w] : 0u;
        long long rk = w < W ? (long long)tbase[w >> lp] + pre[w] : 0;
        while (bits) {
          const int b = __ffs(bits) - 1;
          bits &= bits - 1;
          const long long dst = c0 + ob + rk;
          cci[dst] = (int)(w0 + 32ll * w + b);
          cval[dst] = 0.0;
          ++rk;
        }
      }
      __syncthreads();   // the zeroed sums are visible to the whole block before the atomics
      // 4) every product added at its rank
      for (int cb = rs; cb < re; cb += NT) {
        const int cn = (re - cb) < NT ? (re - cb) : NT;
        const int tp = load_block_chunk<NT>(A, B, cb, re, multi, w0, w1, ch, sbuf);
        for (int it = warp; it < tp; it += NW) {
          const int L = search_le(ch.piece_ex, cn, it);
          const int q0 = ch.bs[L] + (it - ch.piece_ex[L]) * kPiece;
          const int q1 = (q0 + kPiece < ch.be[L]) ? q0 + kPiece : ch.be[L];
          const double a = ch.a[L];
          for (int q = q0 + lane; q < q1; q += 128) {
            PieceRound pr;
            load_piece_round<true>(B, q, q1, w0, pr);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const unsigned off = pr.off[u];
              if (off < span) {
                const unsigned w = off >> 5;
                const long long rk = (long long)tbase[w >> lp] + pre[w] +
                                     __popc(bm[w] & ((1u << (off & 31)) - 1u));
                atomicAdd(cval + c0 + ob + rk, __dmul_rn(a, pr.x[u]));
              }
            }
          }
        }
        __syncthreads();
      }
      ob += tot;
    }
    if (tid == 0 && ob != n) set_error(err, kErrCapacity);
    __syncthreads();
  }
}

// --------------------------------------------------------------------------- CTA hash tier
// Rows with 513 .. T/2 entries whose span suits neither a bitmap nor dense windows: one CTA per
// row (rows taken from a counter), an open-addressing table of the smallest power of two >= 2 x
// the row's exact nnz (at most T slots), filled by the warps sharing the products in pieces
// (load_block_chunk, walk.cuh), then compacted and bitonic-sorted in shared memory.
template <int T, int NT>
__global__ void __launch_bounds__(NT) num_block_hash_kernel(
    const int* rows, const long long* bin_off, int bin, Csr A, Csr B, int upper, int row_base,
    const long long* crp, int* cci, double* cval, int* row_counter, int* err) {
  extern __shared__ __align__(16) unsigned char num_smem[];
  constexpr int NW = NT / 32;
  double* vals = reinterpret_cast<double*>(num_smem);                  // [T]
  int* keys = reinterpret_cast<int*>(vals + T);                        // [T]
  BlockChunk ch;
  ch.a = reinterpret_cast<double*>(keys + T);                          // [NT]
  ch.piece_ex = reinterpret_cast<int*>(ch.a + NT);                     // [NT]
  ch.bs = ch.piece_ex + NT;                                            // [NT]
  ch.be = ch.bs + NT;                                                  // [NT]
  __shared__ long long sbuf[NW + 1];
  __shared__ long long s_row;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long b0 = bin_off[bin];
  const long long nrows = bin_off[bin + 1] - b0;
  for (;;) {
    if (tid == 0) s_row = atomicAdd(row_counter, 1);
    __syncthreads();
    const long long r = s_row;
    if (r >= nrows) break;
    const int i = rows[b0 + r];
    const int lo = upper ? i + row_base : INT_MIN;   // upper-triangle variants drop j < i
    const int rs = A.rp[i], re = A.rp[i + 1];
    const long long c0 = crp[i];
    const int n = (int)(crp[i + 1] - c0);
    int lg = 6;
    while ((1 << lg) < 2 * n && (1 << lg) < T) ++lg;
    const int TR = 1 << lg;
    for (int s = tid; s < TR; s += NT) {
      keys[s] = -1;
      vals[s] = 0.0;
    }
    bool overflow = false;
    for (int cb = rs; cb < re; cb += NT) {
      const int cn = (re - cb) < NT ? (re - cb) : NT;
      const int tp = load_block_chunk<NT>(A, B, cb, re, false, 0, 0, ch, sbuf);
      for (int it = warp; it < tp; it += NW) {
        const int L = search_le(ch.piece_ex, cn, it);
        const int q0 = ch.bs[L] + (it - ch.piece_ex[L]) * kPiece;
        const int q1 = (q0 + kPiece < ch.be[L]) ? q0 + kPiece : ch.be[L];
        const double a = ch.a[L];
        for (int q = q0 + lane; q < q1; q += 32) {
          const int j = __ldg(B.ci + q);
          if (j < lo) continue;
          const double prod = __dmul_rn(a, __ldg(B.val + q));
          unsigned s = hash_slot((unsigned)j, lg);
          int probe = 0;
          for (; probe < TR; ++probe) {
            const int old = atomicCAS(&keys[s], -1, j);
            if (old == -1 || old == j) {
              atomicAdd(&vals[s], prod);
              break;
            }
            s = (s + 1) & (unsigned)(TR - 1);
          }
          if (probe == TR) overflow = true;
        }
      }
      __syncthreads();
    }
    // compaction
    long long pos = 0;
    for (int c = 0; c < TR; c += NT) {
      const int kk = c + tid < TR ? keys[c + tid] : -1;
      const double vv = c + tid < TR ? vals[c + tid] : 0.0;
      long long tot;
      const long long d = block_excl_scan_ll<NT>(kk >= 0 ? 1 : 0, sbuf, &tot);
      if (kk >= 0) {
        keys[pos + d] = kk;
        vals[pos + d] = vv;
      }
      pos += tot;
      __syncthreads();
    }
    int P2 = 1;
    while (P2 < pos) P2 <<= 1;
    for (int x = (int)pos + tid; x < P2; x += NT) keys[x] = INT_MAX;
    __syncthreads();
    // bitonic sort; a stage whose partners lie within one warp's contiguous block of P2 / NW
    // elements runs warp-synchronously, so only the wide stages need block barriers
    const int wb = P2 / (NT / 32);
    for (int kk = 2; kk <= P2; kk <<= 1) {
      for (int jj = kk >> 1; jj > 0; jj >>= 1) {
        const bool in_warp = wb >= 32 && jj < wb;
        if (!in_warp) __syncthreads();
        const int x0 = in_warp ? (tid >> 5) * wb + (tid & 31) : tid;
        const int x1 = in_warp ? ((tid >> 5) + 1) * wb : P2;
        const int dx = in_warp ? 32 : NT;
        for (int x = x0; x < x1; x += dx) {
          const int y = x ^ jj;
          if (y > x) {
            const int kx = keys[x], ky = keys[y];
            const bool up = (x & kk) == 0;
            if ((kx > ky) == up) {
              keys[x] = ky;
              keys[y] = kx;
              const double tv = vals[x];
              vals[x] = vals[y];
              vals[y] = tv;
            }
          }
        }
        if (in_warp) __syncwarp();
        else __syncthreads();
      }
    }
    __syncthreads();
    const int nw = pos < n ? (int)pos : n;
    if (tid == 0 && pos != n) set_error(err, kErrTableFull);
    if (overflow) set_error(err, kErrTableFull);
    for (int t = tid; t < nw; t += NT) {
      cci[c0 + t] = keys[t];
      cval[c0 + t] = vals[t];
    }
    __syncthreads();
  }
}

// --------------------------------------------------------------------------- CTA window tier
// Long, dense rows (at least one entry per four columns of the span, more than 512 entries): one
// CTA per row (rows taken from a counter), the span cut into windows of WC columns. Per window:
// a dense fp64 accumulator and a presence bitmap in shared memory, filled by the warps with
// shared atomics (the warps share the products in pieces, load_block_chunk, walk.cuh; B rows
// are restricted to the window by binary search when the span has several windows), then the
// window's entries are emitted in column order at positions from one block scan of the bitmap
// words' popcounts.
template <int WC, int NT>
__global__ void __launch_bounds__(NT, 1024 / NT) num_block_window_kernel(
    const int* rows, const long long* bin_off, int bin, Csr A, Csr B, const int* lo_arr,
    const int* hi_arr, DenseRows dense, const long long* crp, int* cci, double* cval,
    int* row_counter, int* err) {
  extern __shared__ __align__(16) unsigned char num_smem[];
  constexpr int NW = NT / 32;
  constexpr int WW = WC / 32;
  constexpr int kSplit = kWindowSplit;      // (entry, window boundary) table entries
  constexpr int WPW = (WW + NW - 1) / NW;   // bitmap words per warp in the emit
  constexpr int SUB = WC / NW;              // columns per warp in the dense-row products
  static_assert(WPW <= 32, "one bitmap word per lane when counting a warp's words");
  double* acc = reinterpret_cast<double*>(num_smem);                      // [WC]
  unsigned* bm = reinterpret_cast<unsigned*>(acc + WC);                   // [WW]
  BlockChunk ch;
  ch.a = reinterpret_cast<double*>(bm + WW);                              // [NT]
  ch.piece_ex = reinterpret_cast<int*>(ch.a + NT);                        // [NT]
  ch.bs = ch.piece_ex + NT;                                               // [NT]
  ch.be = ch.bs + NT;                                                     // [NT]
  int* dlist = ch.be + NT;                                                // [NT]
  int* split = dlist + NT;                                                // [kSplit]
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
    const long long c0 = crp[i];
    const long long n = crp[i + 1] - c0;
    const int rs = A.rp[i], re = A.rp[i + 1];
    const bool multi = (long long)hi - lo + 1 > WC;
    // window boundaries of every B row of the row, found once by one binary search per (entry,
    // boundary) pair in parallel, when they fit the table (else every window searches)
    const long long nwin = ((long long)hi - lo + WC) / WC;
    const int T1 = (int)(nwin + 1 < kSplit ? nwin + 1 : kSplit);
    const bool use_split =   // one chunk of A entries (the table is indexed by chunk position)
        multi && re - rs <= NT && (long long)(re - rs) * (nwin + 1) <= kSplit;
    if (use_split) {
      for (int x = tid; x < (re - rs) * T1; x += NT) {
        const int e = x / T1, t = x - e * T1;
        const int k = __ldg(A.ci + rs + e);
        const int rb = __ldg(B.rp + k), rend = __ldg(B.rp + k + 1);
        const long long c = (long long)lo + (long long)t * WC;
        const bool skip = dense.id && __ldg(dense.id + k) >= 0;   // walked by bitmap
        split[x] = skip ? 0 : c > hi ? rend : lower_bound_col(B.ci, rb, rend, (int)c);
      }
      __syncthreads();
    }
    long long ob = 0;
    for (long long w0 = lo; w0 <= hi; w0 += WC) {
      const long long w1 = (w0 + WC < (long long)hi + 1) ? w0 + WC : (long long)hi + 1;
      const unsigned span = (unsigned)(w1 - w0);
      const int words = (int)((span + 31) >> 5);
      const int wt = (int)((w0 - lo) / WC);
      for (int t = tid; t < (int)span; t += NT) acc[t] = 0.0;
      for (int w = tid; w < words; w += NT) bm[w] = 0u;
      for (int cb = rs; cb < re; cb += NT) {
        const int cn = (re - cb) < NT ? (re - cb) : NT;
        const int tp = load_block_chunk<NT>(A, B, cb, re, multi, w0, w1, ch, sbuf, dense.id,
                                            dlist, &s_dcount, use_split ? split : nullptr, wt,
                                            T1);
        for (int it = warp; it < tp; it += NW) {
          const int L = search_le(ch.piece_ex, cn, it);
          const int q0 = ch.bs[L] + (it - ch.piece_ex[L]) * kPiece;
          const int q1 = (q0 + kPiece < ch.be[L]) ? q0 + kPiece : ch.be[L];
          const double a = ch.a[L];
          for (int qb = q0; qb < q1; qb += 128) {   // warp-uniform trip count
            PieceRound pr;
            load_piece_round<true>(B, qb + lane, q1, w0, pr);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (pr.off[u] < span) atomicAdd(acc + pr.off[u], __dmul_rn(a, pr.x[u]));
            or_piece_round(bm, pr, span, true);   // rows of this tier are dense
          }
        }
        __syncthreads();
        const int nd = dense.id ? s_dcount : 0;
        if (nd > 0) {   // block-uniform
          // B rows kept as bitmaps: their bits a word at a time, and their products by column
          // slices -- warp wi owns columns [w0 + wi * SUB, w0 + (wi + 1) * SUB) and adds every
          // listed row's entries there in list order with plain shared-memory updates (no other
          // warp writes those sums)
          or_dense_rows<NT>(bm, words, span, w0, dense, ch, dlist, nd);
          const long long c_lo = w0 + (long long)warp * SUB;
          const long long c_hi = c_lo + SUB < w1 ? c_lo + SUB : w1;
          if (c_lo < c_hi) {
            for (int d0 = 0; d0 < nd; d0 += 32) {
              int s0 = 0, s1 = 0;
              double ad = 0.0;
              if (d0 + lane < nd) {
                const int t = dlist[d0 + lane];
                const int did = ch.be[t];
                s0 = ch.bs[t] + dense_rank(dense, did, c_lo);
                s1 = ch.bs[t] + dense_rank(dense, did, c_hi);
                ad = ch.a[t];
              }
              const int cnt = nd - d0 < 32 ? nd - d0 : 32;
              const int w0i = (int)w0;   // columns of the slice lie in [w0, w1)
              for (int j = 0; j < cnt; ++j) {
                const int q0 = __shfl_sync(0xffffffffu, s0, j);
                const int q1 = __shfl_sync(0xffffffffu, s1, j);
                const double a = __shfl_sync(0xffffffffu, ad, j);
                const int* cp = B.ci + q0 + lane;
                const double* vp = B.val + q0 + lane;
                int q = q0;
                for (; q + 128 <= q1; q += 128, cp += 128, vp += 128) {   // full rounds
                  int c[4];
                  double x[4];
#pragma unroll
                  for (int u = 0; u < 4; ++u) {
                    c[u] = __ldg(cp + 32 * u);
                    x[u] = __ldg(vp + 32 * u);
                  }
#pragma unroll
                  for (int u = 0; u < 4; ++u) {
                    double* p = acc + (c[u] - w0i);
                    *p = fma(a, x[u], *p);
                  }
                }
                if (q < q1) {   // last partial round
                  int c[4];
                  double x[4];
#pragma unroll
                  for (int u = 0; u < 4; ++u) {
                    const bool v = q + lane + 32 * u < q1;
                    c[u] = v ? __ldg(cp + 32 * u) : -1;
                    x[u] = v ? __ldg(vp + 32 * u) : 0.0;
                  }
#pragma unroll
                  for (int u = 0; u < 4; ++u)
                    if (c[u] >= 0) {
                      double* p = acc + (c[u] - w0i);
                      *p = fma(a, x[u], *p);
                    }
                }
                __syncwarp();   // the next row's entries may hit these columns in other lanes
              }
            }
          }
          __syncthreads();
        }
      }
      // emit: warp wi owns words [wi * WPW, (wi + 1) * WPW) and walks them one word at a time,
      // lane b writing bit b, so consecutive lanes store consecutive entries of C
      const int wa = warp * WPW;
      const int wn = words - wa < WPW ? words - wa : WPW;   // may be <= 0
      const unsigned cnt = __reduce_add_sync(0xffffffffu, lane < wn ? __popc(bm[wa + lane]) : 0u);
      long long tot;
      const long long wpos = block_excl_scan_ll<NT>(lane == 0 ? (long long)cnt : 0ll, sbuf, &tot);
      if (ob + tot > n) {
        if (tid == 0) set_error(err, kErrCapacity);
        break;
      }
      long long dst = c0 + ob + __shfl_sync(0xffffffffu, wpos, 0);
      for (int w = wa; w < wa + wn; ++w) {
        const unsigned bits = bm[w];
        if ((bits >> lane) & 1u) {
          const long long d = dst + __popc(bits & ((1u << lane) - 1u));
          cci[d] = (int)(w0 + 32ll * w + lane);
          cval[d] = acc[32 * w + lane];
        }
        dst += __popc(bits);
      }
      __syncthreads();
      ob += tot;
    }
    if (tid == 0 && ob != n) set_error(err, kErrCapacity);
    __syncthreads();
  }
}

template <typename K>
int occupancy_grid(K kern, int threads, size_t smem, int num_sms, long long work_items,
                   int items_per_block) {
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
  if (occ < 1) occ = 1;
  long long want = (work_items + items_per_block - 1) / items_per_block;
  long long cap = (long long)num_sms * occ;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return (int)want;
}

template <int T, int WPB>
void run_warp_hash(int bin, const int* rows, const long long* bin_off, long long nrows, Csr A,
                   Csr B, int upper, int row_base, const long long* crp, int* cci, double* cval,
                   int* err, int num_sms, cudaStream_t s) {
  const size_t smem = (size_t)WPB * T * (sizeof(double) + sizeof(int));
  auto kern = num_warp_hash_kernel<T, WPB>;
  smem_opt_in((const void*)kern, smem);
  const int grid = occupancy_grid(kern, WPB * 32, smem, num_sms, nrows, WPB);
  kern<<<grid, WPB * 32, smem, s>>>(rows, bin_off, bin, A, B, upper, row_base, crp, cci, cval,
                                    err);
}

template <int BUDGET, int WPB, int G>
void run_warp_rank_g(int bin, const int* rows, const long long* bin_off, long long nrows, Csr A,
                     Csr B, int upper, int row_base, const int* lo, const int* hi,
                     const long long* flop, RowBitmaps handoff, const long long* crp, int* cci,
                     double* cval, int* err, int num_sms, cudaStream_t s) {
  const size_t smem = (size_t)WPB * BUDGET;
  auto kern = num_warp_rank_kernel<BUDGET, WPB, G>;
  smem_opt_in((const void*)kern, smem);
  const int grid = occupancy_grid(kern, WPB * 32, smem, num_sms, nrows, WPB);
  kern<<<grid, WPB * 32, smem, s>>>(rows, bin_off, bin, A, B, upper, row_base, lo, hi, handoff,
                                    crp, cci, cval, err);
}

// bin = tier base + group index (0, 1, 2 for G = 1, 2, 4)
template <int BUDGET, int WPB>
void run_warp_rank(int bin, int gidx, const int* rows, const long long* bin_off, long long nrows,
                   Csr A, Csr B, int upper, int row_base, const int* lo, const int* hi,
                   const long long* flop, RowBitmaps handoff, const long long* crp, int* cci,
                   double* cval, int* err, int num_sms, cudaStream_t s) {
  if (gidx == 2)
    run_warp_rank_g<BUDGET, WPB, 4>(bin, rows, bin_off, nrows, A, B, upper, row_base, lo, hi,
                                    flop, handoff, crp, cci, cval, err, num_sms, s);
  else if (gidx == 1)
    run_warp_rank_g<BUDGET, WPB, 2>(bin, rows, bin_off, nrows, A, B, upper, row_base, lo, hi,
                                    flop, handoff, crp, cci, cval, err, num_sms, s);
  else
    run_warp_rank_g<BUDGET, WPB, 1>(bin, rows, bin_off, nrows, A, B, upper, row_base, lo, hi,
                                    flop, handoff, crp, cci, cval, err, num_sms, s);
}

}  // namespace

void launch_numeric_rank_all(const long long* bin_off, long long m, int gidx, int max_need,
                             Csr A, Csr B, const int* lo, const int* hi, const long long* crp,
                             int* cci, double* cval, int* err, int num_sms, cudaStream_t s) {
  // the smallest per-warp budget every row fits (more warps per SM for small rows)
  if (max_need <= 2304)
    run_warp_rank<2304, 8>(0, gidx, nullptr, bin_off, m, A, B, 0, 0, lo, hi, nullptr,
                           RowBitmaps{}, crp, cci, cval, err, num_sms, s);
  else if (max_need <= 4608)
    run_warp_rank<4608, 8>(0, gidx, nullptr, bin_off, m, A, B, 0, 0, lo, hi, nullptr,
                           RowBitmaps{}, crp, cci, cval, err, num_sms, s);
  else
    run_warp_rank<9216, 4>(0, gidx, nullptr, bin_off, m, A, B, 0, 0, lo, hi, nullptr,
                           RowBitmaps{}, crp, cci, cval, err, num_sms, s);
}

void launch_numeric(int bin, const int* rows, const long long* bin_off, long long nrows, Csr A,
                    Csr B, int upper, int row_base, const int* lo, const int* hi,
                    const long long* flop, RowBitmaps handoff, DenseRows dense,
                    const long long* crp, int* cci, double* cval, int* row_counter, int* err,
                    int num_sms, cudaStream_t s) {
  if (nrows <= 0) return;
  if (bin >= kNumRank2K && bin < kNumRank2K + 3) {
    run_warp_rank<2304, 8>(bin, bin - kNumRank2K, rows, bin_off, nrows, A, B, upper, row_base, lo,
                           hi, flop, handoff, crp, cci, cval, err, num_sms, s);
    return;
  }
  if (bin >= kNumRank4K && bin < kNumRank4K + 3) {
    run_warp_rank<4608, 8>(bin, bin - kNumRank4K, rows, bin_off, nrows, A, B, upper, row_base, lo,
                           hi, flop, handoff, crp, cci, cval, err, num_sms, s);
    return;
  }
  if (bin >= kNumRank8K && bin < kNumRank8K + 3) {
    run_warp_rank<9216, 4>(bin, bin - kNumRank8K, rows, bin_off, nrows, A, B, upper, row_base, lo,
                           hi, flop, handoff, crp, cci, cval, err, num_sms, s);
    return;
  }
  switch (bin) {
    case kNumHash64:
      run_warp_hash<64, 8>(bin, rows, bin_off, nrows, A, B, upper, row_base, crp, cci, cval, err,
                           num_sms, s);
      break;
    case kNumHash128:
      run_warp_hash<128, 8>(bin, rows, bin_off, nrows, A, B, upper, row_base, crp, cci, cval, err,
                            num_sms, s);
      break;
    case kNumHash256:
      run_warp_hash<256, 8>(bin, rows, bin_off, nrows, A, B, upper, row_base, crp, cci, cval, err,
                            num_sms, s);
      break;
    case kNumHash512:
      run_warp_hash<512, 8>(bin, rows, bin_off, nrows, A, B, upper, row_base, crp, cci, cval, err,
                            num_sms, s);
      break;
    case kNumHash1024:
      run_warp_hash<1024, 4>(bin, rows, bin_off, nrows, A, B, upper, row_base, crp, cci, cval,
                             err, num_sms, s);
      break;
    case kNumHashBlock: {
      constexpr int NT = 512;
      const size_t smem = (size_t)kHashBlockSlots * (8 + 4) + (size_t)NT * (8 + 8 + 4);
      auto kern = num_block_hash_kernel<kHashBlockSlots, NT>;
      smem_opt_in((const void*)kern, smem);
      const int grid = occupancy_grid(kern, NT, smem, num_sms, nrows, 1);
      kern<<<grid, NT, smem, s>>>(rows, bin_off, bin, A, B, upper, row_base, crp, cci, cval,
                                  row_counter, err);
      break;
    }
    case kNumBlockRank: {
      constexpr int NT = 1024, MAXW = 32768;
      const size_t smem = (size_t)MAXW * 6 + (size_t)NT * (4 + 8 + 12);
      auto kern = num_block_rank_kernel<NT, MAXW>;
      smem_opt_in((const void*)kern, smem);
      const long long grid = nrows < num_sms ? nrows : num_sms;
      kern<<<(unsigned)grid, NT, smem, s>>>(rows, bin_off, bin, A, B, lo, hi, crp, cci, cval,
                                            row_counter, err);
      break;
    }
    case kNumWindow: {
      // two CTAs per SM: one's barriers and L2 waits overlap the other's work
      constexpr int NT = 512, WC = 8192;
      const size_t smem = (size_t)WC * 8 + (size_t)(WC / 32) * 4 + (size_t)NT * (8 + 12 + 4) +
                          (size_t)kWindowSplit * 4;
      auto kern = num_block_window_kernel<WC, NT>;
      smem_opt_in((const void*)kern, smem);
      const long long grid = nrows < 2 * num_sms ? nrows : 2 * num_sms;
      kern<<<(unsigned)grid, NT, smem, s>>>(rows, bin_off, bin, A, B, lo, hi, dense, crp, cci,
                                            cval, row_counter, err);
      break;
    }
    default:
      break;
  }
}

}  // namespace appt
