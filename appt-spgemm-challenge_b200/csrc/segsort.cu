// Stable segmented sort of (int32 key, fp64 value) pairs, keys >= 0.
//
// Used by the ESC baseline (sort each row's expanded products by column) and by the device
// transpose (sort each column's entries by row). Reference counterparts: the global
// thrust::sort_by_key calls in spgemm_kernel_manual.cu:342-348 (ESC) and
// spgemm_kernel_formulations.cu:102-113 (build_csc), which sort all keys of all rows as
// (row << 32 | col) 64-bit keys. Sorting inside each segment instead needs no 64-bit keys, keeps
// the traffic to one read and one write per pass, and is stable, so equal keys keep their
// expansion order (deterministic sums in the ESC compress step).
//
//   len <= 256   warp per segment, bitonic sort in shared memory
//   len <= 4096  CTA per segment, bitonic sort in shared memory
//   len >  4096  CTA per segment: sorted 4096-chunks, then stable merge-path passes that
//                ping-pong between the data and the alternate buffer
// Ties are broken by the original position (the low 32 bits of the sort word), which is what
// makes the in-smem bitonic sort stable.
#include <climits>
#include "common.cuh"
#include "kernels.cuh"

namespace appt {

namespace {

constexpr int kSegWarpCap = 256;
constexpr int kSegBlockCap = 4096;
constexpr int kSegNT = 512;
constexpr int kSegIPT = 8;

template <bool BLOCK>
__device__ __forceinline__ void sync_group() {
  if (BLOCK) __syncthreads(); else __syncwarp();
}

// Bitonic sort of P2 (power of two) 64-bit words with a carried double, by `nthr` threads with
// thread index `tid` inside the group.
template <bool BLOCK>
__device__ void bitonic_u64(unsigned long long* k, double* v, int P2, int tid, int nthr) {
  for (int kk = 2; kk <= P2; kk <<= 1) {
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      for (int x = tid; x < P2; x += nthr) {
        const int y = x ^ jj;
        if (y > x) {
          const unsigned long long kx = k[x], ky = k[y];
          const bool up = (x & kk) == 0;
          if ((kx > ky) == up) {
            k[x] = ky;
            k[y] = kx;
            const double t = v[x];
            v[x] = v[y];
            v[y] = t;
          }
        }
      }
      sync_group<BLOCK>();
    }
  }
}

template <bool BLOCK>
__device__ void sort_chunk(int* keys, double* vals, long long o0, int len, unsigned long long* sk,
                           double* sv, int tid, int nthr) {
  int P2 = 1;
  while (P2 < len) P2 <<= 1;
  for (int t = tid; t < P2; t += nthr) {
    if (t < len) {
      sk[t] = ((unsigned long long)(unsigned)keys[o0 + t] << 32) | (unsigned)t;
      sv[t] = vals[o0 + t];
    } else {
      sk[t] = ~0ull;
    }
  }
  sync_group<BLOCK>();
  bitonic_u64<BLOCK>(sk, sv, P2, tid, nthr);
  for (int t = tid; t < len; t += nthr) {
    keys[o0 + t] = (int)(sk[t] >> 32);
    vals[o0 + t] = sv[t];
  }
  sync_group<BLOCK>();
}

template <int WPB>
__global__ void __launch_bounds__(WPB * 32) segsort_warp_kernel(int* keys, double* vals,
                                                                const long long* off,
                                                                const int* segs,
                                                                const long long* bin_off,
                                                                int bin) {
  extern __shared__ __align__(16) unsigned char ss_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long* sk = reinterpret_cast<unsigned long long*>(ss_smem) + warp * kSegWarpCap;
  double* sv = reinterpret_cast<double*>(ss_smem + (size_t)WPB * kSegWarpCap * 8) +
               warp * kSegWarpCap;
  const long long b0 = bin_off[bin];
  const long long n = bin_off[bin + 1] - b0;
  for (long long r = (long long)blockIdx.x * WPB + warp; r < n; r += (long long)gridDim.x * WPB) {
    const int sgi = segs[b0 + r];
    const long long o0 = off[sgi];
    const int len = (int)(off[sgi + 1] - o0);
    sort_chunk<false>(keys, vals, o0, len, sk, sv, lane, 32);
  }
}

__global__ void __launch_bounds__(kSegNT) segsort_block_kernel(int* keys, double* vals,
                                                               const long long* off,
                                                               const int* segs,
                                                               const long long* bin_off, int bin) {
  extern __shared__ __align__(16) unsigned char ss_smem[];
  unsigned long long* sk = reinterpret_cast<unsigned long long*>(ss_smem);
  double* sv = reinterpret_cast<double*>(ss_smem + (size_t)kSegBlockCap * 8);
  const long long b0 = bin_off[bin];
  const long long n = bin_off[bin + 1] - b0;
  for (long long r = blockIdx.x; r < n; r += gridDim.x) {
    const int sgi = segs[b0 + r];
    const long long o0 = off[sgi];
    const int len = (int)(off[sgi + 1] - o0);
    sort_chunk<true>(keys, vals, o0, len, sk, sv, threadIdx.x, kSegNT);
  }
}

// Stable merge of a = [a0, a0+na) and b = [b0, b0+nb) (both sorted) into dst[d0 ...].
__device__ void merge_path(const int* k, const double* v, long long a0, long long na, long long b0,
                           long long nb, int* dk, double* dv, long long d0) {
  const long long tot = na + nb;
  for (long long o0 = 0; o0 < tot; o0 += (long long)kSegNT * kSegIPT) {
    long long d = o0 + (long long)threadIdx.x * kSegIPT;
    if (d < tot) {
      long long lo = d > nb ? d - nb : 0, hi = d < na ? d : na;
      while (lo < hi) {
        const long long mid = (lo + hi) >> 1;
        if (k[a0 + mid] <= k[b0 + d - 1 - mid]) lo = mid + 1; else hi = mid;
      }
      long long i = lo, j = d - lo;
      for (int c = 0; c < kSegIPT && d + c < tot; ++c) {
        const bool take_a = i < na && (j >= nb || k[a0 + i] <= k[b0 + j]);
        if (take_a) {
          dk[d0 + d + c] = k[a0 + i];
          dv[d0 + d + c] = v[a0 + i];
          ++i;
        } else {
          dk[d0 + d + c] = k[b0 + j];
          dv[d0 + d + c] = v[b0 + j];
          ++j;
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kSegNT) segsort_large_kernel(int* keys, double* vals,
                                                               int* keys_alt, double* vals_alt,
                                                               const long long* off,
                                                               const int* segs,
                                                               const long long* bin_off, int bin) {
  extern __shared__ __align__(16) unsigned char ss_smem[];
  unsigned long long* sk = reinterpret_cast<unsigned long long*>(ss_smem);
  double* sv = reinterpret_cast<double*>(ss_smem + (size_t)kSegBlockCap * 8);
  const long long b0 = bin_off[bin];
  const long long n = bin_off[bin + 1] - b0;
  for (long long r = blockIdx.x; r < n; r += gridDim.x) {
    const int sgi = segs[b0 + r];
    const long long o0 = off[sgi];
    const long long len = off[sgi + 1] - o0;
    for (long long c = 0; c < len; c += kSegBlockCap) {
      const int cl = (int)((len - c) < kSegBlockCap ? (len - c) : kSegBlockCap);
      sort_chunk<true>(keys, vals, o0 + c, cl, sk, sv, threadIdx.x, kSegNT);
    }
    int* sk_src = keys;
    double* sv_src = vals;
    int* sk_dst = keys_alt;
    double* sv_dst = vals_alt;
    for (long long w = kSegBlockCap; w < len; w <<= 1) {
      for (long long ps = 0; ps < len; ps += 2 * w) {
        const long long a0 = ps, na = (ps + w < len) ? w : len - ps;
        const long long bb = ps + na;
        const long long nb = (bb + w < len) ? w : len - bb;
        merge_path(sk_src + o0, sv_src + o0, a0, na, bb, nb > 0 ? nb : 0, sk_dst + o0,
                   sv_dst + o0, ps);
      }
      __syncthreads();
      int* tk = sk_src; sk_src = sk_dst; sk_dst = tk;
      double* tv = sv_src; sv_src = sv_dst; sv_dst = tv;
    }
    if (sk_src != keys) {
      for (long long t = threadIdx.x; t < len; t += kSegNT) {
        keys[o0 + t] = sk_src[o0 + t];
        vals[o0 + t] = sv_src[o0 + t];
      }
    }
    __syncthreads();
  }
}

__global__ void segsort_classify_kernel(const long long* off, int nseg, uint8_t* cls) {
  int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= nseg) return;
  const long long len = off[s + 1] - off[s];
  cls[s] = (uint8_t)(len <= 1 ? 255 : len <= kSegWarpCap ? 0 : len <= kSegBlockCap ? 1 : 2);
}

}  // namespace

size_t segsort_scratch_bytes(int nseg) {
  return (size_t)nseg + 16 + (size_t)nseg * sizeof(int) + 16 + 8 * sizeof(long long) +
         partition_scratch_bytes(nseg, 3) + 64;
}

void segsort(int* keys, double* vals, int* keys_alt, double* vals_alt, const long long* off,
             int nseg, void* scratch, int num_sms, cudaStream_t s) {
  if (nseg <= 0) return;
  char* p = (char*)scratch;
  uint8_t* cls = (uint8_t*)p;
  p += ((size_t)nseg + 16) & ~(size_t)15;
  int* segs = (int*)p;
  p += (((size_t)nseg * sizeof(int)) + 16) & ~(size_t)15;
  long long* bin_off = (long long*)p;
  p += 8 * sizeof(long long);
  segsort_classify_kernel<<<(nseg + 255) / 256, 256, 0, s>>>(off, nseg, cls);
  partition_rows(cls, nseg, 3, segs, bin_off, p, s);
  {
    constexpr int WPB = 8;
    const size_t smem = (size_t)WPB * kSegWarpCap * 16;
    segsort_warp_kernel<WPB><<<num_sms * 4, WPB * 32, smem, s>>>(keys, vals, off, segs, bin_off,
                                                                 0);
  }
  {
    const size_t smem = (size_t)kSegBlockCap * 16;
    smem_opt_in((const void*)segsort_block_kernel, smem);
    smem_opt_in((const void*)segsort_large_kernel, smem);
    segsort_block_kernel<<<num_sms * 2, kSegNT, smem, s>>>(keys, vals, off, segs, bin_off, 1);
    if (keys_alt && vals_alt)
      segsort_large_kernel<<<num_sms, kSegNT, smem, s>>>(keys, vals, keys_alt, vals_alt, off, segs,
                                                         bin_off, 2);
  }
}

}  // namespace appt
