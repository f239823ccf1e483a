// Device utilities: int64 exclusive scan (reduce-then-scan, no inter-block waits) and a
// stable multi-way row partition (the row binner).
//
// Reference counterparts: the est/row_nnz prefix sums done with thrust::inclusive_scan and the
// single-block Hillis-Steele scan (spgemm_kernel_hash.cu:757-770, 913-924, 1020-1031), and the
// bucket binning compute_bucket_kernel + scatter_rows_kernel (spgemm_kernel_hash.cu:725-752).
// Differences: offsets are int64 (the reference's int totals overflow past 2^31 products),
// and the partition is stable (rows stay ascending inside a bin, which keeps neighbouring
// rows -- which share B rows on banded/stencil inputs -- on neighbouring warps for L2 reuse).
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "kernels.cuh"

namespace appt {

namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

template <int NT>
__device__ long long block_excl_scan(long long x, long long* warp_buf, long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  long long incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    long long y = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_buf[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    long long w = (lane < NT / 32) ? warp_buf[lane] : 0;
    long long wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      long long y = __shfl_up_sync(kFull, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < NT / 32) warp_buf[lane] = wi - w;
    if (lane == NT / 32 - 1) warp_buf[NT / 32] = wi;
  }
  __syncthreads();
  long long res = warp_buf[warp] + incl - x;
  if (total) *total = warp_buf[NT / 32];
  __syncthreads();
  return res;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const T* in, long long n,
                                                                   long long* bsum) {
  __shared__ long long wb[kScanThreads / 32 + 1];
  long long base = (long long)blockIdx.x * kScanTile;
  long long s = 0;
#pragma unroll
  for (int it = 0; it < kScanItems; ++it) {
    long long idx = base + (long long)it * kScanThreads + threadIdx.x;
    if (idx < n) s += (long long)in[idx];
  }
  long long tot;
  block_excl_scan<kScanThreads>(s, wb, &tot);
  if (threadIdx.x == 0) bsum[blockIdx.x] = tot;
}

// Single block: exclusive scan of the per-tile sums, in place; writes the grand total.
__global__ void __launch_bounds__(1024) scan_blocksums_kernel(long long* bsum, long long nb,
                                                              long long* total_out) {
  __shared__ long long wb[1024 / 32 + 1];
  long long carry = 0;
  for (long long base = 0; base < nb; base += 1024) {
    long long idx = base + threadIdx.x;
    long long x = idx < nb ? bsum[idx] : 0;
    long long tot;
    long long ex = block_excl_scan<1024>(x, wb, &tot);
    if (idx < nb) bsum[idx] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0 && total_out) *total_out = carry;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const T* in, long long n,
                                                                  const long long* bsum,
                                                                  long long* out) {
  __shared__ long long wb[kScanThreads / 32 + 1];
  long long base = (long long)blockIdx.x * kScanTile + (long long)threadIdx.x * kScanItems;
  long long v[kScanItems];
  long long s = 0;
#pragma unroll
  for (int it = 0; it < kScanItems; ++it) {
    long long idx = base + it;
    v[it] = idx < n ? (long long)in[idx] : 0;
    s += v[it];
  }
  long long ex = block_excl_scan<kScanThreads>(s, wb, nullptr) + bsum[blockIdx.x];
#pragma unroll
  for (int it = 0; it < kScanItems; ++it) {
    long long idx = base + it;
    if (idx < n) out[idx] = ex;
    ex += v[it];
  }
}

// Inputs of at most kScanSmallMax elements: one 1024-thread block. Each warp owns a contiguous
// segment of n / 32 elements and walks it 32 at a time (coalesced): a first pass sums the
// segment, a scan over the 32 warp sums gives each segment's start, and a second pass writes
// the exclusive prefixes with warp scans; out[n] receives the total. (Runs owned by single
// threads -- strided, uncoalesced loads -- took ~70 us on 32K elements.)
constexpr int kScanSmallThreads = 1024;
constexpr long long kScanSmallMax = 65536;

template <typename T>
__global__ void __launch_bounds__(kScanSmallThreads) scan_small_kernel(const T* in, long long n,
                                                                       long long* out) {
  __shared__ long long wsum[kScanSmallThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = kScanSmallThreads / 32;
  const long long seg = (n + NW - 1) / NW;
  const long long a = (long long)warp * seg;
  const long long b = (a + seg < n) ? a + seg : n;
  long long s = 0;
#pragma unroll 4
  for (long long i = a + lane; i < b; i += 32) s += (long long)in[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if (lane == 0) wsum[warp] = s;
  __syncthreads();
  if (warp == 0) {
    const long long v = wsum[lane];
    long long incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += y;
    }
    wsum[lane] = incl - v;
    if (lane == 31) out[n] = incl;
  }
  __syncthreads();
  long long run = wsum[warp];
#pragma unroll 4
  for (long long base = a; base < b; base += 32) {
    const long long i = base + lane;
    const long long v = i < b ? (long long)in[i] : 0;
    long long incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += y;
    }
    if (i < b) out[i] = run + incl - v;
    run += __shfl_sync(kFull, incl, 31);
  }
}

template <typename T>
int scan_impl(const T* in, long long* out, long long n, long long* scratch, cudaStream_t s) {
  long long nb = (n + kScanTile - 1) / kScanTile;
  if (nb == 0) {
    cudaMemsetAsync(out, 0, sizeof(long long), s);
    return 0;
  }
  if (n <= kScanSmallMax) {
    scan_small_kernel<T><<<1, kScanSmallThreads, 0, s>>>(in, n, out);
    return 1;
  }
  scan_reduce_kernel<T><<<(unsigned)nb, kScanThreads, 0, s>>>(in, n, scratch);
  scan_blocksums_kernel<<<1, 1024, 0, s>>>(scratch, nb, out + n);
  scan_apply_kernel<T><<<(unsigned)nb, kScanThreads, 0, s>>>(in, n, scratch, out);
  return 3;
}

// ---------------------------------------------------------------- stable partition
constexpr int kPartThreads = 256;
constexpr int kPartRounds = 4;
constexpr int kPartTile = kPartThreads * kPartRounds;

__global__ void __launch_bounds__(kPartThreads) part_count_kernel(const uint8_t* key, int m,
                                                                  int nb, int ntiles,
                                                                  int* counts) {
  __shared__ int cnt[kMaxBins];
  if (threadIdx.x < kMaxBins) cnt[threadIdx.x] = 0;
  __syncthreads();
  int base = blockIdx.x * kPartTile;
  for (int r = 0; r < kPartRounds; ++r) {
    int row = base + r * kPartThreads + threadIdx.x;
    if (row < m) {
      int k = key[row];
      if (k < nb) atomicAdd(&cnt[k], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < nb) counts[threadIdx.x * ntiles + blockIdx.x] = cnt[threadIdx.x];
}

__global__ void __launch_bounds__(kPartThreads) part_scatter_kernel(const uint8_t* key, int m,
                                                                    int nb, int ntiles,
                                                                    const long long* offs,
                                                                    int* out_rows) {
  constexpr int NW = kPartThreads / 32;
  __shared__ int wc[NW][kMaxBins];
  __shared__ int running[kMaxBins];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x < kMaxBins) running[threadIdx.x] = 0;
  int base = blockIdx.x * kPartTile;
  for (int r = 0; r < kPartRounds; ++r) {
    for (int t = threadIdx.x; t < NW * kMaxBins; t += kPartThreads) (&wc[0][0])[t] = 0;
    __syncthreads();
    int row = base + r * kPartThreads + threadIdx.x;
    int k = (row < m) ? (int)key[row] : 255;
    unsigned peers = __match_any_sync(kFull, k);
    int rank = __popc(peers & lanemask_lt());
    int leader = __ffs(peers) - 1;
    if (lane == leader && k < nb) wc[warp][k] = __popc(peers);
    __syncthreads();
    if (k < nb) {
      int off = running[k] + rank;
      for (int w = 0; w < warp; ++w) off += wc[w][k];
      long long dst = offs[(long long)k * ntiles + blockIdx.x] + off;
      out_rows[dst] = row;
    }
    __syncthreads();
    if (threadIdx.x < nb) {
      int s = 0;
      for (int w = 0; w < NW; ++w) s += wc[w][threadIdx.x];
      running[threadIdx.x] += s;
    }
    __syncthreads();
  }
}

__global__ void part_binoff_kernel(const long long* offs, int nb, int ntiles, long long* bin_off) {
  int b = threadIdx.x;
  if (b <= nb) bin_off[b] = offs[(long long)b * ntiles];
}

}  // namespace

size_t scan_scratch_elems(long long n) { return (size_t)((n + kScanTile - 1) / kScanTile) + 1; }

int scan_exclusive(const int* in, long long* out, long long n, long long* scratch,
                   cudaStream_t s) {
  return scan_impl<int>(in, out, n, scratch, s);
}
int scan_exclusive(const long long* in, long long* out, long long n, long long* scratch,
                   cudaStream_t s) {
  return scan_impl<long long>(in, out, n, scratch, s);
}

size_t partition_scratch_bytes(int m, int nb) {
  long long ntiles = (m + kPartTile - 1) / kPartTile;
  long long cells = ntiles * nb;
  return sizeof(int) * (size_t)cells + sizeof(long long) * (size_t)(cells + 1) +
         sizeof(long long) * scan_scratch_elems(cells) + 256;
}

int partition_rows(const uint8_t* key, int m, int nb, int* out_rows, long long* bin_off,
                    void* scratch, cudaStream_t s) {
  int ntiles = (m + kPartTile - 1) / kPartTile;
  long long cells = (long long)ntiles * nb;
  char* p = (char*)scratch;
  int* counts = (int*)p;
  p += ((sizeof(int) * cells + 15) / 16) * 16;
  long long* offs = (long long*)p;
  p += sizeof(long long) * (cells + 1);
  long long* sc = (long long*)p;
  if (ntiles == 0) {
    cudaMemsetAsync(bin_off, 0, sizeof(long long) * (nb + 1), s);
    return 0;
  }
  part_count_kernel<<<ntiles, kPartThreads, 0, s>>>(key, m, nb, ntiles, counts);
  const int scan_launches = scan_exclusive(counts, offs, cells, sc, s);
  part_scatter_kernel<<<ntiles, kPartThreads, 0, s>>>(key, m, nb, ntiles, offs, out_rows);
  part_binoff_kernel<<<1, 32, 0, s>>>(offs, nb, ntiles, bin_off);
  return 3 + scan_launches;
}

// ---------------------------------------------------------------- small helpers
namespace {
__global__ void narrow_rowptr_kernel(const long long* in, int* out, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (int)in[i];
}
__global__ void iota_kernel(int* out, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = i;
}
}  // namespace

namespace {
// sub[b * (K + 1) + k] = first position in bin b's row list holding a row >= k * m / K (the
// rows of a bin ascend), so the rows of block k that bin b holds are
// rows[sub[b*(K+1)+k] .. sub[b*(K+1)+k+1]).
__global__ void block_bin_bounds_kernel(const int* rows, const long long* bin_off, int nb,
                                        long long m, int K, long long* sub) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= nb * (K + 1)) return;
  const int b = t / (K + 1), k = t % (K + 1);
  long long lo = bin_off[b], hi = bin_off[b + 1];
  const long long v = (long long)k * m / K;
  while (lo < hi) {
    const long long mid = (lo + hi) >> 1;
    if (rows[mid] < v) lo = mid + 1; else hi = mid;
  }
  sub[t] = lo;
}
}  // namespace

void block_bin_bounds(const int* rows, const long long* bin_off, int nb, long long m, int K,
                      long long* sub, cudaStream_t s) {
  const int n = nb * (K + 1);
  if (n <= 0) return;
  block_bin_bounds_kernel<<<(n + 255) / 256, 256, 0, s>>>(rows, bin_off, nb, m, K, sub);
}

void narrow_rowptr(const long long* in, int* out, long long n, cudaStream_t s) {
  if (n <= 0) return;
  narrow_rowptr_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(in, out, n);
}

void iota(int* out, int n, cudaStream_t s) {
  if (n <= 0) return;
  iota_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, n);
}

namespace {
__global__ void readback_kernel(Readback r, unsigned* dst) {
  int off = 0;
  for (int i = 0; i < r.n; ++i) {
    const unsigned* src = static_cast<const unsigned*>(r.src[i]);
    for (int w = threadIdx.x; w < r.words[i]; w += blockDim.x) dst[off + w] = src[w];
    off += r.words[i];
  }
}
}  // namespace

void launch_readback(const Readback& r, void* pinned_dst, cudaStream_t s) {
  readback_kernel<<<1, 128, 0, s>>>(r, static_cast<unsigned*>(pinned_dst));
}

void smem_opt_in(const void* kern, size_t bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;   // (kernel, device) -> bytes set
  std::lock_guard<std::mutex> g(mu);
  size_t& have = done[{kern, dev}];
  if (have >= bytes) return;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
      cudaSuccess)
    have = bytes;
  else
    cudaGetLastError();   // the launch that follows reports the failure
}

}  // namespace appt
