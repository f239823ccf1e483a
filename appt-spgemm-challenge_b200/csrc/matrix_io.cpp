// Matrix file I/O of the reference's driver (src/matrix_utils.cu; declarations in
// include/spgemm.h:44-52): read_matrix_market, write_matrix_market, print_matrix_info and
// verify_csr_matrices, with the same C++-linkage signatures, buffer layout and allocation rules,
// so the reference's src/main.cu links against this library without src/matrix_utils.cu.
//
// read_matrix_market differs in speed, not in result:
//   * a file that starts with the 8 bytes "APPTCSR1" is read as binary CSR (int64 rows, cols,
//     nnz; int32 row_ptr; int32 col_idx; fp64 val) straight into the buffer -- no parsing;
//   * a MatrixMarket text file is read in one block and parsed with std::from_chars (no
//     per-entry fscanf), rows filled by a counting pass instead of one vector per row. The same
//     banner rules as the reference apply: "pattern" gives value 1.0, "complex" keeps the real
//     part, "symmetric" mirrors off-diagonal entries; duplicate entries are kept; each row is
//     sorted by (column, value) pairs, as the reference sorts its (col, val) pairs.
// write_matrix_market writes the reference's text format; a name ending in ".bin" writes the
// binary CSR form instead (exact values, loadable by read_matrix_market).
//
// The A buffer is [row_ptr (rows+1) int32 | col_idx (nnz) int32 | pad to 8 | val (nnz) fp64]
// (src/matrix_utils.cu:120-160), pinned (cudaMallocHost) when g_use_mempool is set, else malloc --
// release it with host_free, as the reference's driver does.
#include <cuda_runtime.h>

#include <algorithm>
#include <charconv>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include "engine.h"

extern "C" bool g_use_mempool;

namespace {

constexpr char kMagic[8] = {'A', 'P', 'P', 'T', 'C', 'S', 'R', '1'};

size_t align8(size_t x) { return (x + 7) & ~(size_t)7; }

void* alloc_buffer(size_t bytes) {
  void* b = nullptr;
  if (g_use_mempool) {
    if (cudaMallocHost(&b, bytes ? bytes : 1) != cudaSuccess) {
      cudaGetLastError();
      std::fprintf(stderr, "cudaMallocHost failed, size = %zu bytes\n", bytes);
      return nullptr;
    }
  } else {
    b = std::malloc(bytes ? bytes : 1);
    if (!b) std::fprintf(stderr, "malloc failed, size = %zu bytes\n", bytes);
  }
  return b;
}

void free_buffer(void* b) {
  if (!b) return;
  if (g_use_mempool) cudaFreeHost(b);
  else std::free(b);
}

struct Out {
  void** buffer;
  int **rp, **ci;
  double** val;
  int *rows, *cols, *nnz;
};

bool publish(const Out& o, void* buf, int rows, int cols, int nnz) {
  char* base = (char*)buf;
  const size_t rp_b = (size_t)(rows + 1) * 4, ci_b = (size_t)nnz * 4;
  *o.buffer = buf;
  *o.rp = (int*)base;
  *o.ci = (int*)(base + rp_b);
  *o.val = (double*)(base + align8(rp_b + ci_b));
  *o.rows = rows;
  *o.cols = cols;
  *o.nnz = nnz;
  return true;
}

bool read_binary(std::FILE* f, const char* name, const Out& o) {
  long long hdr[3];
  if (std::fread(hdr, 8, 3, f) != 3 || hdr[0] < 0 || hdr[1] < 0 || hdr[2] < 0 ||
      hdr[0] >= INT32_MAX || hdr[1] >= INT32_MAX || hdr[2] >= INT32_MAX) {
    std::fprintf(stderr, "%s: bad binary CSR header\n", name);
    return false;
  }
  const int rows = (int)hdr[0], cols = (int)hdr[1], nnz = (int)hdr[2];
  const size_t rp_b = (size_t)(rows + 1) * 4, ci_b = (size_t)nnz * 4;
  const size_t total = align8(rp_b + ci_b) + (size_t)nnz * 8;
  void* buf = alloc_buffer(total);
  if (!buf) return false;
  char* base = (char*)buf;
  const bool ok = std::fread(base, 1, rp_b, f) == rp_b && std::fread(base + rp_b, 1, ci_b, f) == ci_b &&
                  std::fread(base + align8(rp_b + ci_b), 8, (size_t)nnz, f) == (size_t)nnz;
  if (!ok) {
    std::fprintf(stderr, "%s: truncated binary CSR file\n", name);
    free_buffer(buf);
    return false;
  }
  const int* rp = (const int*)base;
  if (rp[0] != 0 || rp[rows] != nnz) {
    std::fprintf(stderr, "%s: row_ptr does not span the entries\n", name);
    free_buffer(buf);
    return false;
  }
  return publish(o, buf, rows, cols, nnz);
}

// Cursor over the text; every parse skips blanks first and fails at the end of the text.
struct Text {
  const char* p;
  const char* end;
  void skip_blank() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\r' || *p == '\n')) ++p;
  }
  template <typename T>
  bool next(T* v) {
    skip_blank();
    auto r = std::from_chars(p, end, *v);
    if (r.ec != std::errc()) return false;
    p = r.ptr;
    return true;
  }
  bool next_double(double* v) {
    skip_blank();
    if (p < end && *p == '+') ++p;   // from_chars does not take a leading '+'
    auto r = std::from_chars(p, end, *v);
    if (r.ec != std::errc()) {
      // out-of-range literals: fall back to strtod on a bounded copy
      char tmp[64];
      const size_t n = std::min<size_t>(63, (size_t)(end - p));
      std::memcpy(tmp, p, n);
      tmp[n] = 0;
      char* e = nullptr;
      *v = std::strtod(tmp, &e);
      if (e == tmp) return false;
      p += e - tmp;
      return true;
    }
    p = r.ptr;
    return true;
  }
  void skip_line() {
    while (p < end && *p != '\n') ++p;
    if (p < end) ++p;
  }
};

bool read_text(std::FILE* f, const char* name, const Out& o) {
  std::fseek(f, 0, SEEK_END);
  const long len = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  if (len <= 0) return false;
  std::string s((size_t)len, '\0');
  if (std::fread(&s[0], 1, (size_t)len, f) != (size_t)len) return false;
  Text t{s.data(), s.data() + s.size()};
  // banner: the first line, case-insensitive keywords (src/matrix_utils.cu:60-66)
  const char* eol = (const char*)std::memchr(t.p, '\n', (size_t)(t.end - t.p));
  std::string banner(t.p, eol ? eol : t.end);
  for (char& ch : banner) ch = (char)std::tolower((unsigned char)ch);
  const bool pattern = banner.find("pattern") != std::string::npos;
  const bool symmetric = banner.find("symmetric") != std::string::npos;
  const bool complex = banner.find("complex") != std::string::npos;
  t.skip_line();
  while (t.p < t.end && *t.p == '%') t.skip_line();
  long long M = 0, N = 0, nz = 0;
  if (!t.next(&M) || !t.next(&N) || !t.next(&nz) || M < 0 || N < 0 || nz < 0 ||
      M >= INT32_MAX || N >= INT32_MAX) {
    std::fprintf(stderr, "%s: bad size line\n", name);
    return false;
  }
  std::vector<int> er, ec;
  std::vector<double> ev;
  const size_t cap = (size_t)nz * (symmetric ? 2 : 1);
  er.reserve(cap);
  ec.reserve(cap);
  ev.reserve(cap);
  for (long long k = 0; k < nz; ++k) {
    long long r = 0, c = 0;
    double v = 1.0, im = 0.0;
    if (!t.next(&r) || !t.next(&c)) return false;
    if (!pattern) {
      if (!t.next_double(&v)) return false;
      if (complex && !t.next_double(&im)) return false;
    }
    if (r < 1 || r > M || c < 1 || c > N) {
      std::fprintf(stderr, "%s: entry %lld outside the matrix\n", name, k + 1);
      return false;
    }
    er.push_back((int)(r - 1));
    ec.push_back((int)(c - 1));
    ev.push_back(v);
    if (symmetric && r != c) {
      er.push_back((int)(c - 1));
      ec.push_back((int)(r - 1));
      ev.push_back(v);
    }
  }
  const size_t nnz = er.size();
  if (nnz >= (size_t)INT32_MAX) {
    std::fprintf(stderr, "%s: too many entries for int32 offsets\n", name);
    return false;
  }
  const size_t rp_b = (size_t)(M + 1) * 4, ci_b = nnz * 4;
  void* buf = alloc_buffer(align8(rp_b + ci_b) + nnz * 8);
  if (!buf) return false;
  char* base = (char*)buf;
  int* rp = (int*)base;
  int* ci = (int*)(base + rp_b);
  double* val = (double*)(base + align8(rp_b + ci_b));
  // counting placement by row, then each unsorted row sorted by (column, value)
  std::vector<int> cnt((size_t)M + 1, 0);
  for (int r : er) ++cnt[(size_t)r + 1];
  std::partial_sum(cnt.begin(), cnt.end(), cnt.begin());
  for (long long i = 0; i <= M; ++i) rp[i] = cnt[(size_t)i];
  std::vector<int> pos(cnt.begin(), cnt.end() - 1);
  for (size_t k = 0; k < nnz; ++k) {
    const int d = pos[(size_t)er[k]]++;
    ci[d] = ec[k];
    val[d] = ev[k];
  }
  std::vector<std::pair<int, double>> row;
  for (long long i = 0; i < M; ++i) {
    const int a = rp[i], b = rp[i + 1];
    bool sorted = true;
    for (int q = a + 1; q < b && sorted; ++q) sorted = ci[q - 1] <= ci[q];
    if (sorted) continue;
    row.assign((size_t)(b - a), {});
    for (int q = a; q < b; ++q) row[(size_t)(q - a)] = {ci[q], val[q]};
    std::sort(row.begin(), row.end());
    for (int q = a; q < b; ++q) {
      ci[q] = row[(size_t)(q - a)].first;
      val[q] = row[(size_t)(q - a)].second;
    }
  }
  return publish(o, buf, (int)M, (int)N, (int)nnz);
}

bool read_any(const char* filename, const Out& o) {
  std::FILE* f = std::fopen(filename, "rb");
  if (!f) {
    std::fprintf(stderr, "Cannot open %s\n", filename);
    return false;
  }
  char magic[8] = {0};
  const size_t got = std::fread(magic, 1, 8, f);
  bool ok;
  if (got == 8 && std::memcmp(magic, kMagic, 8) == 0) {
    ok = read_binary(f, filename, o);
  } else {
    ok = read_text(f, filename, o);
  }
  std::fclose(f);
  return ok;
}

bool ends_with(const char* s, const char* suf) {
  const size_t a = std::strlen(s), b = std::strlen(suf);
  return a >= b && std::strcmp(s + a - b, suf) == 0;
}

}  // namespace

// ---- C++ linkage: the reference driver's declarations (include/spgemm.h:44-52)
bool read_matrix_market(const char* filename, void** buffer_out, int** row_ptr_out,
                        int** col_idx_out, double** val_out, int* rows, int* cols, int* nnz) {
  if (!filename || !buffer_out || !row_ptr_out || !col_idx_out || !val_out || !rows || !cols ||
      !nnz)
    return false;
  return read_any(filename, Out{buffer_out, row_ptr_out, col_idx_out, val_out, rows, cols, nnz});
}

bool write_matrix_market(const char* filename, const int* row_ptr, const int* col_idx,
                         const double* val, int rows, int cols, int nnz) {
  std::FILE* f = std::fopen(filename, ends_with(filename, ".bin") ? "wb" : "w");
  if (!f) {
    std::fprintf(stderr, "Failed to write %s\n", filename);
    return false;
  }
  if (ends_with(filename, ".bin")) {
    const long long hdr[3] = {rows, cols, nnz};
    std::fwrite(kMagic, 1, 8, f);
    std::fwrite(hdr, 8, 3, f);
    std::vector<int> rp((size_t)rows + 1);
    for (int i = 0; i <= rows; ++i) rp[(size_t)i] = row_ptr[i] - row_ptr[0];
    std::fwrite(rp.data(), 4, rp.size(), f);
    std::fwrite(col_idx + row_ptr[0], 4, (size_t)nnz, f);
    std::fwrite(val + row_ptr[0], 8, (size_t)nnz, f);
    std::fclose(f);
    return true;
  }
  // the reference's text form: 1-based "row col value", value with 6 significant digits
  // (ostream default, src/matrix_utils.cu:172-193)
  std::fprintf(f, "%%%%MatrixMarket matrix coordinate real general\n%d %d %d\n", rows, cols, nnz);
  for (int i = 0; i < rows; ++i)
    for (int j = row_ptr[i]; j < row_ptr[i + 1]; ++j)
      std::fprintf(f, "%d %d %g\n", i + 1, col_idx[j] + 1, val[j]);
  std::fclose(f);
  return true;
}

void print_matrix_info(const char* name, int rows, int cols, int nnz) {
  const double sparsity =
      (rows * cols > 0) ? (1.0 - (double)nnz / ((double)rows * cols)) * 100 : 0;
  std::printf("%s: %d × %d, nnz = %d, sparsity = %g%%\n", name, rows, cols, nnz, sparsity);
}

bool verify_csr_matrices(const int* row_ptr1, const int* col_idx1, const double* val1,
                         const int* row_ptr2, const int* col_idx2, const double* val2, int rows,
                         int cols, int nnz1, int nnz2, double tolerance) {
  (void)cols;
  if (nnz1 != nnz2) {
    std::fprintf(stderr, "Verification failed: nnz mismatch (%d vs %d)\n", nnz1, nnz2);
    return false;
  }
  for (int i = 0; i < rows; ++i) {
    const int a1 = row_ptr1[i], b1 = row_ptr1[i + 1], a2 = row_ptr2[i], b2 = row_ptr2[i + 1];
    if (b1 - a1 != b2 - a2) {
      std::fprintf(stderr, "Verification failed: row %d has different nnz (%d vs %d)\n", i,
                   b1 - a1, b2 - a2);
      return false;
    }
    for (int j = a1, k = a2; j < b1; ++j, ++k) {
      if (col_idx1[j] != col_idx2[k]) {
        std::fprintf(stderr, "Verification failed: row %d, col index mismatch (%d vs %d)\n", i,
                     col_idx1[j], col_idx2[k]);
        return false;
      }
      const double diff = std::fabs(val1[j] - val2[k]);
      const double mx = std::max(std::fabs(val1[j]), std::fabs(val2[k]));
      const double rel = mx > 0 ? diff / mx : diff;
      if (rel > tolerance) {
        std::fprintf(stderr,
                     "Verification failed: row %d, col %d, value mismatch (%.6e vs %.6e, "
                     "rel_err=%.6e)\n",
                     i, col_idx1[j], val1[j], val2[k], rel);
        return false;
      }
    }
  }
  return true;
}

// ---- C linkage for FFI callers (include/appt_spgemm.h)
extern "C" bool appt_read_matrix_file(const char* filename, void** buffer_out, int** row_ptr_out,
                                      int** col_idx_out, double** val_out, int* rows, int* cols,
                                      int* nnz) {
  return read_matrix_market(filename, buffer_out, row_ptr_out, col_idx_out, val_out, rows, cols,
                            nnz);
}

extern "C" bool appt_write_matrix_file(const char* filename, const int* row_ptr,
                                       const int* col_idx, const double* val, int rows, int cols,
                                       int nnz) {
  return write_matrix_market(filename, row_ptr, col_idx, val, rows, cols, nnz);
}
