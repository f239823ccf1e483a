// Driver for the reference's own CUDA build -- TEST AND BENCH INFRASTRUCTURE ONLY.
//
// Linked (by oracle/Makefile) against the unmodified reference sources
// (src/spgemm_adaptive.cu, spgemm_kernel_hash.cu, spgemm_merge.cu, spgemm_kernel_manual.cu,
// spgemm_kernel_formulations.cu, spgemm_kernel_cusparse.cu, mempool.cu) into
// oracle/_ref/ref_spgemm. It calls the reference's public entry points (include/spgemm.h) on a
// binary CSR file, the way the reference's src/main.cu does (pinned input buffer and pinned
// output arena when USE_MEMPOOL is on, warm-up calls, then timed calls), and optionally writes
// the last C to a binary file. Used to generate golden fixtures and as the reference arm of
// bench.py (the reference's GPU path, timed per call through its host-buffer API).
//
// usage: ref_spgemm <method> <in.bin> [--out FILE] [--warmup W] [--repeat N] [--no-mempool]
// method: adaptive | hash | merge3 | manual | att_adaptive | att_hash | att_merge3
#include "spgemm.h"
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace {

bool read_bin(const char* path, void** buf, int* rows, int* cols, int* nnz, bool pinned) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return false;
  char magic[8];
  long long hdr[3];
  if (std::fread(magic, 1, 8, f) != 8 || std::memcmp(magic, "APPTCSR1", 8) != 0 ||
      std::fread(hdr, 8, 3, f) != 3) {
    std::fclose(f);
    return false;
  }
  *rows = (int)hdr[0];
  *cols = (int)hdr[1];
  *nnz = (int)hdr[2];
  const size_t rp_b = (size_t)(*rows + 1) * 4, ci_b = (size_t)(*nnz) * 4;
  const size_t v_off = ALIGN8(rp_b + ci_b);
  const size_t total = v_off + (size_t)(*nnz) * 8;
  void* b = nullptr;
  if (pinned) {
    if (cudaMallocHost(&b, total) != cudaSuccess) b = nullptr;
  } else {
    b = std::malloc(total);
  }
  if (!b) {
    std::fclose(f);
    return false;
  }
  char* c = (char*)b;
  bool ok = std::fread(c, 1, rp_b, f) == rp_b && std::fread(c + rp_b, 1, ci_b, f) == ci_b &&
            std::fread(c + v_off, 1, (size_t)(*nnz) * 8, f) == (size_t)(*nnz) * 8;
  std::fclose(f);
  if (!ok) return false;
  *buf = b;
  return true;
}

bool write_bin(const char* path, const void* cbuf, int rows, int cols, int nnz) {
  FILE* f = std::fopen(path, "wb");
  if (!f) return false;
  const char* c = (const char*)cbuf;
  const size_t rp_al = ALIGN8((size_t)(rows + 1) * 4), ci_al = ALIGN8((size_t)nnz * 4);
  long long hdr[3] = {rows, cols, nnz};
  std::fwrite("APPTCSR1", 1, 8, f);
  std::fwrite(hdr, 8, 3, f);
  std::fwrite(c, 4, (size_t)rows + 1, f);
  std::fwrite(c + rp_al, 4, (size_t)nnz, f);
  std::fwrite(c + rp_al + ci_al, 8, (size_t)nnz, f);
  std::fclose(f);
  return true;
}

typedef void (*entry_t)(void*, int, int, int, void**, int*, int*, int*);

}  // namespace

int main(int argc, char** argv) {
  if (argc < 3) {
    std::fprintf(stderr, "usage: %s <method> <in.bin> [--out F] [--warmup W] [--repeat N] "
                         "[--no-mempool]\n", argv[0]);
    return 2;
  }
  std::string method = argv[1];
  const char* in = argv[2];
  const char* out = nullptr;
  int warmup = 1, repeat = 1;
  bool mempool = true;
  for (int i = 3; i < argc; ++i) {
    if (!std::strcmp(argv[i], "--out") && i + 1 < argc) out = argv[++i];
    else if (!std::strcmp(argv[i], "--warmup") && i + 1 < argc) warmup = std::atoi(argv[++i]);
    else if (!std::strcmp(argv[i], "--repeat") && i + 1 < argc) repeat = std::atoi(argv[++i]);
    else if (!std::strcmp(argv[i], "--no-mempool")) mempool = false;
  }
  entry_t fn = nullptr;
  if (method == "adaptive") fn = spgemm_self_product_adaptive;
  else if (method == "hash") fn = spgemm_self_product_hash;
  else if (method == "merge3") fn = spgemm_self_product_merge3;
  else if (method == "manual") fn = spgemm_self_product_manual;
  else if (method == "att_adaptive") fn = spgemm_att_adaptive;
  else if (method == "att_hash") fn = spgemm_att_hash;
  else if (method == "att_merge3") fn = spgemm_att_merge3;
  if (!fn) {
    std::fprintf(stderr, "unknown method %s\n", method.c_str());
    return 2;
  }
  g_use_mempool = mempool;
  g_use_dev_pool = false;
  cudaFree(0);
  cudaSetDevice(0);
  void* A = nullptr;
  int rows = 0, cols = 0, nnz = 0;
  std::string json;   // printed once at the end: the reference prints its own lines to stdout
  if (!read_bin(in, &A, &rows, &cols, &nnz, mempool)) {
    std::fprintf(stderr, "cannot read %s\n", in);
    return 3;
  }
  // pinned output arena: products * 12 bytes bounds C (as the reference's MP_HOST_MB advice)
  {
    const int* rp = (const int*)A;
    const int* ci = rp + rows + 1;
    long long prod = 0;
    if (method.rfind("att", 0) != 0) {
      for (int p = 0; p < nnz; ++p) prod += rp[ci[p] + 1] - rp[ci[p]];
    } else {
      std::vector<long long> cc((size_t)cols + 1, 0);
      for (int p = 0; p < nnz; ++p) cc[ci[p]]++;
      for (int c = 0; c < cols; ++c) prod += cc[c] * cc[c];
    }
    size_t cap = (size_t)prod * 12 + (size_t)(rows + 1) * 4 + (64u << 20);
    if (mempool && !mempool_init(cap)) {
      std::fprintf(stderr, "mempool_init failed\n");
      return 4;
    }
    json = "{\"products\": " + std::to_string(prod);
  }
  void* C = nullptr;
  int cr = 0, cc = 0, cn = 0;
  for (int w = 0; w < warmup; ++w) {
    C = nullptr;
    fn(A, rows, cols, nnz, &C, &cr, &cc, &cn);
    if (C) pinned_free(C);
  }
  json += ", \"ms\": [";
  for (int r = 0; r < repeat; ++r) {
    C = nullptr;
    auto t0 = std::chrono::steady_clock::now();
    fn(A, rows, cols, nnz, &C, &cr, &cc, &cn);
    auto t1 = std::chrono::steady_clock::now();
    char buf[64];
    std::snprintf(buf, sizeof(buf), "%s%.6f", r ? ", " : "",
                  std::chrono::duration<double, std::milli>(t1 - t0).count());
    json += buf;
    if (r + 1 < repeat && C) pinned_free(C);
  }
  {
    char buf[160];
    std::snprintf(buf, sizeof(buf), "], \"c_rows\": %d, \"c_cols\": %d, \"c_nnz\": %d}", cr, cc, cn);
    json += buf;
  }
  std::fflush(stdout);
  std::printf("\n%s\n", json.c_str());
  std::fflush(stdout);
  if (out && C && cn >= 0) write_bin(out, C, cr, cc, cn);
  if (C) pinned_free(C);
  host_free(A);
  mempool_destroy();
  return cn < 0 ? 5 : 0;
}
