// Output-size estimators: per-partition MinHash sketch (128 partitions of 32-bit MurmurHash3
// minima) per B row, min-merged over the B rows an A row selects, turned into an estimate of
// the row's distinct output columns.
//
// Reference counterpart: murmur_hash3 + mh_construct_kernel + mh_merge_kernel
// (spgemm_kernel_hash.cu:78-90, 257-369), the reference's default sizing path for A with at
// least 100000 nonzeros; below that it uses the exact products count
// (count_intermediates_par_kernel, :33-55; STREAMLINE_NNZ :65). The estimate and its snapping
// follow the reference exactly: linear counting when some partition is empty, otherwise
// 2^32 * sum(1/min_j) - m; times 1.5; values <= 16 kept, others snapped to a power of two in
// [32, 16384]. The floating-point sum uses the same order as the reference (4 partitions per
// lane, then a shuffle-down tree), so the estimates are reproducible bit for bit.
//
// The engine itself sizes C from an exact symbolic count, so this estimator is exposed through
// the C-ABI (appt_estimate_row_nnz) for callers that want the reference's sizing numbers, and
// for planning (predicting output bytes before the symbolic pass).
#include "common.cuh"
#include "kernels.cuh"

namespace appt {

namespace {

constexpr int kMhParts = 128;
constexpr unsigned kMhEmpty = 0xffffffffu;
constexpr int kMhWPB = 8;

__device__ __forceinline__ unsigned rotl32(unsigned x, int r) { return (x << r) | (x >> (32 - r)); }

// MurmurHash3_x86_32 of one 32-bit key, seed 1234 (the reference's seed).
__device__ __forceinline__ unsigned murmur3_u32(unsigned key) {
  unsigned h = 1234u;
  unsigned k = key * 0xcc9e2d51u;
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

__global__ void __launch_bounds__(kMhWPB * 32) mh_build_kernel(Csr B, unsigned* sketch) {
  __shared__ unsigned sk[kMhWPB][kMhParts];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long nw = (long long)gridDim.x * kMhWPB;
  for (long long r = (long long)blockIdx.x * kMhWPB + warp; r < B.rows; r += nw) {
    for (int t = lane; t < kMhParts; t += 32) sk[warp][t] = kMhEmpty;
    __syncwarp();
    const int rs = B.rp[r], re = B.rp[r + 1];
    for (int p = rs + lane; p < re; p += 32) {
      const unsigned h = murmur3_u32((unsigned)B.ci[p]);
      atomicMin(&sk[warp][h & (kMhParts - 1)], h);
    }
    __syncwarp();
    uint4 v = make_uint4(sk[warp][4 * lane], sk[warp][4 * lane + 1], sk[warp][4 * lane + 2],
                         sk[warp][4 * lane + 3]);
    reinterpret_cast<uint4*>(sketch + (size_t)r * kMhParts)[lane] = v;
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kMhWPB * 32) mh_merge_kernel(Csr A, const unsigned* sketch,
                                                               int* est) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long nw = (long long)gridDim.x * kMhWPB;
  for (long long i = (long long)blockIdx.x * kMhWPB + warp; i < A.rows; i += nw) {
    uint4 m = make_uint4(kMhEmpty, kMhEmpty, kMhEmpty, kMhEmpty);
    const int rs = A.rp[i], re = A.rp[i + 1];
    for (int p = rs; p < re; ++p) {
      const int k = A.ci[p];
      const uint4 v = reinterpret_cast<const uint4*>(sketch + (size_t)k * kMhParts)[lane];
      m.x = min(m.x, v.x);
      m.y = min(m.y, v.y);
      m.z = min(m.z, v.z);
      m.w = min(m.w, v.w);
    }
    double sum_inv = 0.0;
    int V = 0;
    const unsigned mv[4] = {m.x, m.y, m.z, m.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (mv[q] != kMhEmpty) {
        sum_inv += 1.0 / (double)mv[q];
        ++V;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sum_inv += __shfl_down_sync(kFull, sum_inv, off);
      V += __shfl_down_sync(kFull, V, off);
    }
    if (lane == 0) {
      double E;
      if (V == 0) E = 0.0;
      else if (V < kMhParts) E = (double)kMhParts * log((double)kMhParts / (double)(kMhParts - V));
      else E = 4294967296.0 * sum_inv - (double)kMhParts;
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
}

// ---------------------------------------------------------------- HyperLogLog alternative
// Reference counterpart: hll_construct_kernel / hll_merge_kernel (spgemm_kernel_hash.cu:94-240),
// selected there by EST_METHOD=hll. Precision 7: 128 one-byte registers per B row; a column's
// register is the low 7 bits of its MurmurHash3 and its rank the leading-zero count of the hash
// plus one, capped at 26. A row of A takes the register-wise maximum over the B rows it selects;
// the estimate is alpha * m^2 / sum(2^-reg) (alpha = 0.715), or m * ln(m / empty) when some
// register is empty and the raw estimate is at most 2.5 m, then times 1.5 and snapped like the
// MinHash estimate. sum(2^-reg) is a sum of at most 128 powers of two between 2^-26 and 1, which
// double holds exactly, so its order does not matter.
constexpr int kHllM = 128;

__global__ void __launch_bounds__(kMhWPB * 32) hll_build_kernel(Csr B, unsigned char* regs) {
  __shared__ unsigned rk[kMhWPB][kHllM];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long nw = (long long)gridDim.x * kMhWPB;
  for (long long r = (long long)blockIdx.x * kMhWPB + warp; r < B.rows; r += nw) {
    for (int t = lane; t < kHllM; t += 32) rk[warp][t] = 0u;
    __syncwarp();
    const int rs = B.rp[r], re = B.rp[r + 1];
    for (int p = rs + lane; p < re; p += 32) {
      const unsigned h = murmur3_u32((unsigned)B.ci[p]);
      unsigned rho = (unsigned)__clz((int)h) + 1u;
      if (rho > 26u) rho = 26u;
      atomicMax(&rk[warp][h & (kHllM - 1)], rho);
    }
    __syncwarp();
    // four registers per lane, packed into one 32-bit store
    const unsigned packed = rk[warp][4 * lane] | (rk[warp][4 * lane + 1] << 8) |
                            (rk[warp][4 * lane + 2] << 16) | (rk[warp][4 * lane + 3] << 24);
    reinterpret_cast<unsigned*>(regs + (size_t)r * kHllM)[lane] = packed;
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kMhWPB * 32) hll_merge_kernel(Csr A, const unsigned char* regs,
                                                                int* est) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long nw = (long long)gridDim.x * kMhWPB;
  for (long long i = (long long)blockIdx.x * kMhWPB + warp; i < A.rows; i += nw) {
    unsigned m = 0u;
    const int rs = A.rp[i], re = A.rp[i + 1];
    for (int p = rs; p < re; ++p) {
      const int k = A.ci[p];
      m = __vmaxu4(m, reinterpret_cast<const unsigned*>(regs + (size_t)k * kHllM)[lane]);
    }
    double z = 0.0;
    int empty = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const unsigned v = (m >> (8 * q)) & 0xffu;
      z += 1.0 / (double)(1ull << v);
      empty += v == 0u;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      z += __shfl_down_sync(kFull, z, off);
      empty += __shfl_down_sync(kFull, empty, off);
    }
    if (lane == 0) {
      double E = 0.715 * (double)kHllM * (double)kHllM / z;
      if (empty != 0 && E <= 2.5 * kHllM) E = (double)kHllM * log((double)kHllM / (double)empty);
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
}

__global__ void flop_count_kernel(Csr A, Csr B, int* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= A.rows) return;
  long long s = 0;
  for (int p = A.rp[i]; p < A.rp[i + 1]; ++p) {
    const int k = A.ci[p];
    s += B.rp[k + 1] - B.rp[k];
  }
  out[i] = (int)s;
}

}  // namespace

void launch_minhash_estimate(Csr A, Csr B, unsigned* sketch, int* est, int num_sms,
                             cudaStream_t s) {
  if (B.rows > 0) {
    long long blocks = (B.rows + kMhWPB - 1) / kMhWPB;
    if (blocks > (long long)num_sms * 16) blocks = (long long)num_sms * 16;
    mh_build_kernel<<<(unsigned)blocks, kMhWPB * 32, 0, s>>>(B, sketch);
  }
  if (A.rows > 0) {
    long long blocks = (A.rows + kMhWPB - 1) / kMhWPB;
    if (blocks > (long long)num_sms * 16) blocks = (long long)num_sms * 16;
    mh_merge_kernel<<<(unsigned)blocks, kMhWPB * 32, 0, s>>>(A, sketch, est);
  }
}

void launch_hll_estimate(Csr A, Csr B, unsigned char* regs, int* est, int num_sms,
                         cudaStream_t s) {
  if (B.rows > 0) {
    long long blocks = (B.rows + kMhWPB - 1) / kMhWPB;
    if (blocks > (long long)num_sms * 16) blocks = (long long)num_sms * 16;
    hll_build_kernel<<<(unsigned)blocks, kMhWPB * 32, 0, s>>>(B, regs);
  }
  if (A.rows > 0) {
    long long blocks = (A.rows + kMhWPB - 1) / kMhWPB;
    if (blocks > (long long)num_sms * 16) blocks = (long long)num_sms * 16;
    hll_merge_kernel<<<(unsigned)blocks, kMhWPB * 32, 0, s>>>(A, regs, est);
  }
}

void launch_flop_count_i32(Csr A, Csr B, int* out, cudaStream_t s) {
  if (A.rows <= 0) return;
  flop_count_kernel<<<(A.rows + 255) / 256, 256, 0, s>>>(A, B, out);
}

}  // namespace appt
