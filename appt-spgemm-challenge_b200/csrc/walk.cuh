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
#include "kernels.cuh"

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
// Grouped walks for the bitmap tiers. The warp is split into G groups of L = 32 / G lanes; in
// step s group g takes A entry t = s * G + g of the current chunk of 32 A entries and its lanes
// cover that row of B (lane q of the group takes entries q, q + L, ...). The chunk's B row
// bounds and A values sit in registers (one A entry per lane) and are broadcast by shuffles.
// Lanes whose A entry lies past the row end hold an empty B row, so a step needs no bounds
// test against the chunk size. When every B row of the chunk fits its group (the common case),
// the loop body is branch-free: one predicated load per operand and one update.

// Loads the chunk's A entries starting at `base`: B row start, length (0 past the row end) and,
// when `a` is given, the A value.
__device__ __forceinline__ void load_chunk(const Csr& A, const Csr& B, int base, int re, int& bs,
                                           int& len, double* a) {
  const int p = base + (threadIdx.x & 31);
  bs = 0;
  len = 0;
  if (a) *a = 0.0;
  if (p < re) {
    const int k = __ldg(A.ci + p);
    bs = __ldg(B.rp + k);
    len = __ldg(B.rp + k + 1) - bs;
    if (a) *a = __ldg(A.val + p);
  }
}

// OR `bits` into the shared word at `p` when `pred` holds (fire-and-forget, no branch).
__device__ __forceinline__ void red_or_shared_if(bool pred, unsigned* p, unsigned bits) {
  const unsigned a = (unsigned)__cvta_generic_to_shared(p);
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q red.shared.or.b32 [%0], %1;\n\t}"
      :: "r"(a), "r"(bits), "r"((int)pred) : "memory");
}

// Entry `sub` of the B row (bt, lt): its column (lo - 1, i.e. outside every span, when the row is
// shorter) and, when `x` is given, its value. The load address is always valid (entry 0 of B for
// lanes without an entry; B has entries whenever a row reaches these walks), so the load needs
// no branch.
__device__ __forceinline__ int load_b_entry(const Csr& B, int bt, int lt, int sub, int lo,
                                            double* x) {
  const bool v = sub < lt;
  const int idx = v ? bt + sub : 0;
  const int j = __ldg(B.ci + idx);
  if (x) *x = __ldg(B.val + idx);
  return v ? j : lo - 1;
}

// Bitmaps over a row's column span are stored with their 32-bit words permuted within blocks of
// 32 (word w lives at swz(w)), so that words 32 * c apart -- the same bank in a plain layout,
// e.g. the planes of a 3-D stencil -- fall into different banks. The word count is rounded up to
// whole blocks (bitmap_words), which keeps the permutation inside the array.
__host__ __device__ __forceinline__ unsigned swz(unsigned w) { return w ^ ((w >> 5) & 31u); }
__host__ __device__ __forceinline__ int bitmap_words(long long span) {
  return (int)((((span + 31) >> 5) + 31) & ~31ll);
}

// Presence bitmap of the row's columns: bit (j - lo) of logical word (j - lo) / 32 is set for
// every product column j (order-free). The chunk's B row bounds are passed in (one A entry per lane). In the
// common case the column indices of kFillBatch consecutive steps are loaded before any of them
// is applied, so that many loads are in flight per warp; a batch that runs past the chunk wraps
// to entries of the same chunk, which set bits that are set anyway (stopping the last batch at
// the chunk's end measured slower: the early exits break up the batched loads). Returns true if
// a column lies above the span (B rows not sorted); columns below lo are skipped (they are the
// ones the upper-triangle variants drop).
constexpr int kFillBatch = 8;

template <int G>
__device__ __forceinline__ bool fill_chunk_bitmap(const Csr& B, int bs, int len, int cnt, int lo,
                                                  unsigned span, unsigned* bm) {
  constexpr int L = 32 / G;
  const int lane = threadIdx.x & 31, grp = lane / L, sub = lane % L;
  const int hi = lo + (int)span - 1;
  bool bad = false;
  if (!__any_sync(kFull, len > L)) {
    for (int t0 = 0; t0 < cnt; t0 += G * kFillBatch) {
      int jj[kFillBatch];
#pragma unroll
      for (int u = 0; u < kFillBatch; ++u) {
        const int t = (t0 + u * G + grp) & 31;
        jj[u] = load_b_entry(B, __shfl_sync(kFull, bs, t), __shfl_sync(kFull, len, t), sub, lo,
                             nullptr);
      }
#pragma unroll
      for (int u = 0; u < kFillBatch; ++u) {
        const unsigned off = (unsigned)(jj[u] - lo);
        red_or_shared_if(off < span, bm + swz(off >> 5), 1u << (off & 31));
        bad |= jj[u] > hi;
      }
    }
  } else {
    for (int t0 = 0; t0 < cnt; t0 += G) {
      const int t = t0 + grp;
      const int bt = __shfl_sync(kFull, bs, t);
      const int lt = __shfl_sync(kFull, len, t);
      for (int q = sub; q < lt; q += L) {
        const int j = __ldg(B.ci + bt + q);
        const unsigned off = (unsigned)(j - lo);
        red_or_shared_if(off < span, bm + swz(off >> 5), 1u << (off & 31));
        bad |= j > hi;
      }
    }
  }
  return bad;
}

template <int G>
__device__ __forceinline__ bool fill_row_bitmap_g(const Csr& A, const Csr& B, int rs, int re,
                                                  int lo, unsigned span, unsigned* bm) {
  bool bad = false;
  for (int base = rs; base < re; base += 32) {
    int bs, len;
    load_chunk(A, B, base, re, bs, len, nullptr);
    const int cnt = (re - base) < 32 ? (re - base) : 32;
    bad |= fill_chunk_bitmap<G>(B, bs, len, cnt, lo, span, bm);
  }
  return bad;
}

// Exclusive popcount prefix of the W (a multiple of 32) permuted bitmap words, in logical word
// order, into 16-bit entries stored at the same permuted positions (each lane owns a contiguous
// run of logical words); returns the total number of set bits.
__device__ __forceinline__ int bitmap_prefix32(const unsigned* bm, int W, unsigned short* pre) {
  const int lane = threadIdx.x & 31;
  const int per = W >> 5;
  const unsigned w0 = lane * per;
  int s = 0;
  for (int q = 0; q < per; ++q) s += __popc(bm[swz(w0 + q)]);
  const int incl = warp_incl_scan(s);
  int run = incl - s;
  for (int q = 0; q < per; ++q) {
    const unsigned w = swz(w0 + q);
    pre[w] = (unsigned short)run;
    run += __popc(bm[w]);
  }
  return __shfl_sync(kFull, incl, 31);
}

// Rank of span offset `off` among the set bits, or `dummy` (the row's nnz, the spare slot) when
// off is outside the span (word 0 is read instead, so the lookup needs no branch). The result
// never exceeds `dummy`, whatever the bitmap holds.
__device__ __forceinline__ int rank_or(const unsigned* bm, const unsigned short* pre, unsigned off,
                                       unsigned span, int dummy) {
  const bool ok = off < span;
  const unsigned w = ok ? swz(off >> 5) : 0u;
  const int r = (int)pre[w] + __popc(bm[w] & ((1u << (off & 31)) - 1u));
  return ok ? min(r, dummy) : dummy;
}

// Ranked accumulation over one chunk of A entries: acc[rank(j)] += a_ik * b_kj and
// coff[rank(j)] = j - lo for every product with j in the span, k-sequentially (G ordered
// sub-phases per step when G > 1). Lanes without a product in a (sub-)phase update the
// spare slot acc[n] / coff[n] instead, so the step has no branch. In the common case the B
// entries of the next two steps are loaded while the current step is applied.
// Unroll factor of the rank tier's step loop: unrolled three times, the values carried from
// step to step by the two-step prefetch stay in place instead of moving between registers
// (banded 2^22 numeric 7.31 -> 6.40 ms).
#ifndef APPT_RANK_UNROLL
#define APPT_RANK_UNROLL 3
#endif
constexpr int kRankUnroll = APPT_RANK_UNROLL;

template <int G>
__device__ __forceinline__ void accumulate_chunk_ranked(const Csr& B, int bs, int len, double a,
                                                        int cnt, int lo, unsigned span, int n,
                                                        const unsigned* bm,
                                                        const unsigned short* pre, double* acc,
                                                        unsigned short* coff) {
  constexpr int L = 32 / G;
  const int lane = threadIdx.x & 31, grp = lane / L, sub = lane % L;
  if (!__any_sync(kFull, len > L)) {
#ifndef APPT_RANK_PREFETCH2
#define APPT_RANK_PREFETCH2 1
#endif
#if APPT_RANK_PREFETCH2
    // software pipeline: entries loaded two steps ahead, their rank looked up one step ahead
    // (the bitmap is read-only here), so a step's critical path is the accumulator update alone
    double x0, x1;
    const int j0 = load_b_entry(B, __shfl_sync(kFull, bs, grp), __shfl_sync(kFull, len, grp),
                                sub, lo, &x0);
    int j1 = load_b_entry(B, __shfl_sync(kFull, bs, G + grp), __shfl_sync(kFull, len, G + grp),
                          sub, lo, &x1);
    unsigned off0 = (unsigned)(j0 - lo);
    int r0 = rank_or(bm, pre, off0, span, n);
#pragma unroll kRankUnroll
    for (int t0 = 0; t0 < cnt; t0 += G) {
      // entries two steps ahead (a step past the chunk reads a valid row and is discarded)
      const int t2 = (t0 + 2 * G + grp) & 31;
      double x2;
      const int j2 = load_b_entry(B, __shfl_sync(kFull, bs, t2), __shfl_sync(kFull, len, t2),
                                  sub, lo, &x2);
      const unsigned off1 = (unsigned)(j1 - lo);
      const int r1 = rank_or(bm, pre, off1, span, n);
      const double at = __shfl_sync(kFull, a, t0 + grp);
      const double p0 = __dmul_rn(at, x0);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int pos = (G == 1 || grp == g) ? r0 : n;
        acc[pos] = __dadd_rn(acc[pos], p0);
        coff[pos] = (unsigned short)off0;
        __syncwarp();
      }
      off0 = off1;
      r0 = r1;
      x0 = x1;
      j1 = j2;
      x1 = x2;
    }
#else
    // software pipeline: entries and their rank one step ahead
    double x0;
    const int j0 = load_b_entry(B, __shfl_sync(kFull, bs, grp), __shfl_sync(kFull, len, grp),
                                sub, lo, &x0);
    unsigned off0 = (unsigned)(j0 - lo);
    int r0 = rank_or(bm, pre, off0, span, n);
    for (int t0 = 0; t0 < cnt; t0 += G) {
      const int t1 = (t0 + G + grp) & 31;
      double x1;
      const int j1 = load_b_entry(B, __shfl_sync(kFull, bs, t1), __shfl_sync(kFull, len, t1),
                                  sub, lo, &x1);
      const double at = __shfl_sync(kFull, a, t0 + grp);
      const double p0 = __dmul_rn(at, x0);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int pos = (G == 1 || grp == g) ? r0 : n;
        acc[pos] = __dadd_rn(acc[pos], p0);
        coff[pos] = (unsigned short)off0;
        __syncwarp();
      }
      off0 = (unsigned)(j1 - lo);
      r0 = rank_or(bm, pre, off0, span, n);
      x0 = x1;
    }
#endif
  } else {
    for (int t0 = 0; t0 < cnt; t0 += G) {
      const int t = t0 + grp;
      const int bt = __shfl_sync(kFull, bs, t);
      const int lt = __shfl_sync(kFull, len, t);
      const double at = __shfl_sync(kFull, a, t);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        if (G == 1 || grp == g) {
          for (int q = sub; q < lt; q += L) {
            const int j = __ldg(B.ci + bt + q);
            const unsigned off = (unsigned)(j - lo);
            const int pos = rank_or(bm, pre, off, span, n);
            acc[pos] = mul_add_rn(acc[pos], at, __ldg(B.val + bt + q));
            coff[pos] = (unsigned short)off;
          }
        }
        __syncwarp();
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// CTA-wide walks (one CTA per row): the row's A entries are taken NT at a time; each B row (its
// part inside the current column window) is cut into pieces of at most kPiece entries and the
// warps take pieces round-robin (a warp finds its piece's A entry by binary search over the
// piece prefix), so a row made of a few very long B rows keeps every warp busy.
constexpr int kPiece = 256;

struct BlockChunk {   // one chunk of up to NT A entries of a row, in shared memory
  int* piece_ex;      // exclusive prefix of pieces per entry
  int* bs;            // B segment start (inside the window)
  int* be;            // B segment end
  double* a;          // A value
};

// Loads A entries [cb, cb + NT) of the row (segments restricted to [w0, w1) when `multi`, by
// binary search, or read from `split` -- split[e * split_stride + t] is the first entry of
// window t in entry e's B row) and returns the number of pieces. With `dense_id`, entries whose
// B row has a bitmap get no pieces: their chunk indices are listed in dlist[0 .. *dcount), with
// bs = the B row's first entry and be = its bitmap index. Contains barriers.
template <int NT>
__device__ __forceinline__ int load_block_chunk(const Csr& A, const Csr& B, int cb, int re,
                                                bool multi, long long w0, long long w1,
                                                BlockChunk ch, long long* sbuf,
                                                const int* dense_id = nullptr,
                                                int* dlist = nullptr, int* dcount = nullptr,
                                                const int* split = nullptr, int split_t = 0,
                                                int split_stride = 0) {
  const int tid = threadIdx.x;
  const int p = cb + tid;
  int bs = 0, be = 0, did = -1;
  double a = 0.0;
  if (dense_id && tid == 0) *dcount = 0;   // readers of the previous list passed a barrier
  if (p < re) {
    const int k = __ldg(A.ci + p);
    if (dense_id) did = __ldg(dense_id + k);
    bs = __ldg(B.rp + k);
    a = __ldg(A.val + p);
    if (did < 0) {
      be = __ldg(B.rp + k + 1);
      if (multi && split) {
        bs = split[tid * split_stride + split_t];
        be = split[tid * split_stride + split_t + 1];
      } else if (multi) {
        bs = lower_bound_col(B.ci, bs, be, (int)w0);
        be = lower_bound_col(B.ci, bs, be, (int)(w1 > 0x7fffffffll ? 0x7fffffff : w1));
      }
    } else {
      be = did;
    }
  }
  const int pieces = did < 0 ? (be - bs + kPiece - 1) / kPiece : 0;
  long long tot;
  const long long ex = block_excl_scan_ll<NT>(pieces, sbuf, &tot);   // orders the reset above
  if (did >= 0) dlist[atomicAdd(dcount, 1)] = tid;
  ch.piece_ex[tid] = (int)ex;
  ch.bs[tid] = bs;
  ch.be[tid] = be;
  ch.a[tid] = a;
  __syncthreads();
  return (int)tot;
}

// Entries of dense B row `did` with columns below c (0 <= c <= B.cols).
__device__ __forceinline__ int dense_rank(const DenseRows& dense, int did, long long c) {
  const size_t g = (size_t)did * dense.stride + (size_t)(c >> 5);
  const unsigned below = (1u << (c & 31)) - 1u;
  return (int)(__ldg(dense.pre + g) + __popc(__ldg(dense.bits + g) & below));
}

// ORs the words of window [w0, w0 + span) of the listed dense B rows into bm (W words; thread
// per word, plain read-modify-write: no other writer may run concurrently).
template <int NT>
__device__ __forceinline__ void or_dense_rows(unsigned* bm, int W, unsigned span, long long w0,
                                              const DenseRows& dense, const BlockChunk& ch,
                                              const int* dlist, int nd) {
  const long long g0 = w0 >> 5;
  const int sh = (int)(w0 & 31);
  for (int w = threadIdx.x; w < W; w += NT) {
    const long long g = g0 + w;   // g + 1 < stride: the window lies inside B's columns
    unsigned acc = 0u;
    for (int d = 0; d < nd; ++d) {
      const unsigned* row = dense.bits + (size_t)ch.be[dlist[d]] * dense.stride;
      acc |= __funnelshift_r(__ldg(row + g), __ldg(row + g + 1), sh);
    }
    if (w == W - 1 && (span & 31u)) acc &= (1u << (span & 31u)) - 1u;
    bm[w] |= acc;
  }
}

// Entries [q0, q1) of a B row, four rounds of 32 per lane-step with all loads issued before any
// is used: columns (as offsets from the window start w0; entries past q1 get an offset outside
// every window) and, when `x` is given, values.
struct PieceRound {
  unsigned off[4];
  double x[4];
};

template <bool WITH_VAL>
__device__ __forceinline__ void load_piece_round(const Csr& B, int q, int q1, long long w0,
                                                 PieceRound& pr) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int qq = q + 32 * u;
    const bool v = qq < q1;
    const int idx = v ? qq : q1 - 1;   // the piece is not empty: q1 - 1 is always an entry
    const int j = __ldg(B.ci + idx);
    if (WITH_VAL) pr.x[u] = __ldg(B.val + idx);
    pr.off[u] = v ? (unsigned)((long long)j - w0) : 0xffffffffu;
  }
}

// ORs the column bits of one piece round (offsets >= span are skipped) into bm. With `dense`
// (warp-uniform; rows whose B rows are dense) the lanes' bits are first combined per word with
// warp reductions and one lane per word issues the OR, when the round touches at most four words
// -- fewer shared-memory atomics beside the fp64 ones of the dense-window tier; otherwise every
// lane issues its own. All 32 lanes must call.
__device__ __forceinline__ void or_piece_round(unsigned* bm, const PieceRound& pr, unsigned span,
                                               bool dense) {
  const unsigned lane = threadIdx.x & 31;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const unsigned off = pr.off[u];
    const bool v = off < span;
    if (dense) {
      const unsigned w = off >> 5;
      const unsigned wlo = __reduce_min_sync(0xffffffffu, v ? w : 0xffffffffu);
      const unsigned whi = __reduce_max_sync(0xffffffffu, v ? w : 0u);
      if (wlo > whi) continue;   // no lane has an entry in this round
      if (whi - wlo < 4) {
        for (unsigned ww = wlo; ww <= whi; ++ww) {
          const unsigned r =
              __reduce_or_sync(0xffffffffu, (v && w == ww) ? 1u << (off & 31) : 0u);
          red_or_shared_if(lane == 0 && r != 0u, bm + ww, r);
        }
        continue;
      }
    }
    red_or_shared_if(v, bm + (off >> 5), 1u << (off & 31));
  }
}

}  // namespace appt
