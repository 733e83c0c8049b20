// Matrix Market input and a binary CSR cache: the data format on the input
// side of the SpMV path.
//
// spmvb_read_matrix_market restates the reference's reader
// (src/mtx_io.cpp:40-172): the same banner rules (coordinate matrices,
// real / integer / pattern, general / symmetric; complex, array and
// skew-symmetric refused), comment and blank lines skipped, 1-based indices
// range-checked, pattern entries = 1.0, an off-diagonal symmetric entry
// followed by its mirror, a count check, the CSR assembled by a counting sort
// in file order, then every row sorted by column with std::sort on
// (column, value) pairs compared by column only - the call the reference
// makes, so repeated (row, column) entries end up in the same order. Error
// texts are the reference's ("Matrix Market: <path>: ...").
//
// What differs is the speed: the file is read in one piece and its entry
// lines are parsed by several threads with std::from_chars, each thread a
// contiguous range of lines, the results concatenated in file order. Lines
// past the declared entry count are ignored exactly as the reference's
// sequential loop ignores them (an error there does not count).
#include <algorithm>
#include <cctype>
#include <cmath>
#include <charconv>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../internal.hpp"

using namespace spmvb;

struct spmvb_host_csr_st {
  int32_t m = 0, n = 0;
  int64_t nnz = 0;
  std::vector<int32_t> rowptr, colind;
  std::vector<double> values;
};

namespace {

// 0-based row, 0-based column (top bit set: the mirror of the entry before).
struct Triple {
  int32_t i;
  uint32_t j;
  double v;
};
constexpr uint32_t kMirror = 0x80000000u;

std::string lower(std::string s) {
  for (auto& c : s) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
  return s;
}

spmvb_status mm_fail(const std::string& path, const std::string& msg) {
  return fail(SPMVB_ERR_INVALID_MATRIX, "Matrix Market: " + path + ": " + msg);
}

bool is_space(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\v' || c == '\f' || c == '\r'; }

// Whitespace-separated token, as `istream >> std::string` reads it.
std::string token(const char*& p, const char* e) {
  while (p < e && is_space(*p)) ++p;
  const char* s = p;
  while (p < e && !is_space(*p)) ++p;
  return std::string(s, p);
}

// `istream >> long long`: leading whitespace, an optional sign, digits.
bool parse_ll(const char*& p, const char* e, long long& out) {
  while (p < e && is_space(*p)) ++p;
  const char* q = p;
  bool neg = false;
  if (q < e && (*q == '+' || *q == '-')) neg = *q++ == '-';
  if (q >= e || !std::isdigit(static_cast<unsigned char>(*q))) return false;
  unsigned long long v = 0;
  auto r = std::from_chars(q, e, v);
  if (r.ec != std::errc()) return false;
  if (v > static_cast<unsigned long long>(INT64_MAX) + (neg ? 1ull : 0ull)) return false;
  out = neg ? static_cast<long long>(0 - v) : static_cast<long long>(v);
  p = r.ptr;
  return true;
}

// `istream >> double` for decimal numbers: an optional sign, then digits or a
// point (no inf / nan, which the stream refuses too), correctly rounded. The
// stream's extraction (std::num_get) also takes an 'e' / 'E' after the
// mantissa, with an optional sign and digits, and fails when the collected
// text is not one complete number: "1.5e" and "1.5e+" are errors, not 1.5.
// A value too large for a double fails too; one too small for it is read as
// strtod reads it (zero or a subnormal), as num_get does.
bool parse_double(const char*& p, const char* e, double& out) {
  while (p < e && is_space(*p)) ++p;
  const char* q = p;
  bool neg = false;
  if (q < e && (*q == '+' || *q == '-')) neg = *q++ == '-';
  if (q >= e || !(std::isdigit(static_cast<unsigned char>(*q)) || *q == '.')) return false;
  double v = 0.0;
  auto r = std::from_chars(q, e, v, std::chars_format::general);
  if (r.ec != std::errc() && r.ec != std::errc::result_out_of_range) return false;
  if (r.ptr < e && (*r.ptr == 'e' || *r.ptr == 'E')) return false;  // an exponent without digits
  if (r.ec == std::errc::result_out_of_range) {
    const std::string text(q, r.ptr);
    v = std::strtod(text.c_str(), nullptr);
    if (std::isinf(v)) return false;  // overflow: the stream sets failbit
  }
  out = neg ? -v : v;
  p = r.ptr;
  return true;
}

struct Part {
  std::vector<Triple> tris;
  long long lines = 0;      // entry lines parsed
  bool failed = false;
  std::string message;      // error text (without the path prefix)
};

// Parses the entry lines in [b, e) (b at a line start).
void parse_range(const char* b, const char* e, long long rows, long long cols, bool pattern, bool symmetric,
                 Part& out) {
  const char* p = b;
  while (p < e) {
    const char* nl = static_cast<const char*>(std::memchr(p, '\n', static_cast<size_t>(e - p)));
    const char* le = nl ? nl : e;
    const char* next = nl ? nl + 1 : e;
    if (le == p || *p == '%') {
      p = next;
      continue;
    }
    const char* q = p;
    long long i = 0, j = 0;
    double v = 1.0;
    const char* why = nullptr;
    if (!parse_ll(q, le, i) || !parse_ll(q, le, j))
      why = "malformed entry line: '";
    else if (!pattern && !parse_double(q, le, v))
      why = "expected a value on entry line: '";
    else if (i < 1 || i > rows || j < 1 || j > cols)
      why = "index out of range on entry line: '";
    if (why) {
      out.failed = true;
      out.message = why + std::string(p, le) + "'";
      return;
    }
    out.tris.push_back({static_cast<int32_t>(i - 1), static_cast<uint32_t>(j - 1), v});
    if (symmetric && i != j) out.tris.push_back({static_cast<int32_t>(j - 1), static_cast<uint32_t>(i - 1) | kMirror, v});
    ++out.lines;
    p = next;
  }
}

spmvb_status read_file(const std::string& path, std::string& buf) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return fail(SPMVB_ERR_IO, "Matrix Market: " + path + ": cannot open file");
  std::fseek(f, 0, SEEK_END);
  const long size = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  if (size < 0) {
    std::fclose(f);
    return fail(SPMVB_ERR_IO, path + ": cannot determine the file size");
  }
  buf.resize(static_cast<size_t>(size));
  const size_t got = size ? std::fread(&buf[0], 1, buf.size(), f) : 0;
  std::fclose(f);
  if (got != buf.size()) return fail(SPMVB_ERR_IO, path + ": short read");
  return SPMVB_OK;
}

// One line (without '\n') starting at p; p moves past it. False at the end.
bool next_line(const char*& p, const char* e, const char*& ls, const char*& le) {
  if (p >= e) return false;
  ls = p;
  const char* nl = static_cast<const char*>(std::memchr(p, '\n', static_cast<size_t>(e - p)));
  le = nl ? nl : e;
  p = nl ? nl + 1 : e;
  return true;
}

spmvb_status read_mtx(const std::string& path, int threads, spmvb_host_csr_st& A) {
  std::string buf;
  SPMVB_TRY(read_file(path, buf));
  const char* p = buf.data();
  const char* e = p + buf.size();
  const char *ls, *le;
  if (!next_line(p, e, ls, le)) return mm_fail(path, "empty file");

  // Banner.
  bool pattern = false, symmetric = false;
  {
    const char* q = ls;
    const std::string banner = token(q, le), object = token(q, le), format = token(q, le), field = token(q, le),
                      symmetry = token(q, le);
    if (lower(banner) != "%%matrixmarket") return mm_fail(path, "missing %%MatrixMarket banner");
    if (lower(object) != "matrix") return mm_fail(path, "only 'matrix' objects are supported, got '" + object + "'");
    if (lower(format) != "coordinate")
      return mm_fail(path, "only 'coordinate' format is supported, got '" + format + "'");
    const std::string f = lower(field);
    if (f == "complex") return mm_fail(path, "complex matrices are not supported");
    if (f != "real" && f != "integer" && f != "pattern") return mm_fail(path, "unsupported field type '" + field + "'");
    const std::string sym = lower(symmetry);
    if (sym == "skew-symmetric") return mm_fail(path, "skew-symmetric matrices are not supported");
    if (sym != "general" && sym != "symmetric") return mm_fail(path, "unsupported symmetry '" + symmetry + "'");
    pattern = f == "pattern";
    symmetric = sym == "symmetric";
  }

  // Size line.
  long long rows = 0, cols = 0, entries = 0;
  bool got_size = false;
  while (next_line(p, e, ls, le)) {
    if (le == ls || *ls == '%') continue;
    const char* q = ls;
    if (!parse_ll(q, le, rows) || !parse_ll(q, le, cols) || !parse_ll(q, le, entries))
      return mm_fail(path, "malformed size line: '" + std::string(ls, le) + "'");
    got_size = true;
    break;
  }
  if (!got_size) return mm_fail(path, "missing size line");
  if (rows < 0 || cols < 0 || entries < 0) return mm_fail(path, "negative dimensions in size line");
  if (rows > 2147483647LL || cols > 2147483647LL) return mm_fail(path, "dimensions exceed int32 index range");

  // Entry lines, in contiguous line ranges, one thread each.
  int T = threads > 0 ? threads : static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  const size_t rest = static_cast<size_t>(e - p);
  T = static_cast<int>(std::max<size_t>(1, std::min<size_t>(T, rest / (1 << 20) + 1)));  // >= 1 MiB per thread
  std::vector<const char*> cut(T + 1);
  cut[0] = p;
  cut[T] = e;
  for (int t = 1; t < T; ++t) {
    const char* c = p + rest * t / T;
    c = std::max(c, cut[t - 1]);
    const char* nl = static_cast<const char*>(std::memchr(c, '\n', static_cast<size_t>(e - c)));
    cut[t] = nl ? nl + 1 : e;
  }
  std::vector<Part> parts(T);
  {
    std::vector<std::thread> pool;
    for (int t = 1; t < T; ++t)
      pool.emplace_back(parse_range, cut[t], cut[t + 1], rows, cols, pattern, symmetric, std::ref(parts[t]));
    parse_range(cut[0], cut[1], rows, cols, pattern, symmetric, parts[0]);
    for (auto& th : pool) th.join();
  }
  // Concatenate in file order up to `entries` lines; an error counts only if
  // it comes before the last of them, as in a sequential read.
  std::vector<Triple> tris;
  long long count = 0;
  for (int t = 0; t < T && count < entries; ++t) {
    Part& P = parts[t];
    if (P.lines <= entries - count) {
      tris.insert(tris.end(), P.tris.begin(), P.tris.end());
      count += P.lines;
      // The failing line comes after this part's parsed lines: it matters
      // only if the declared entries are not all read yet.
      if (P.failed && count < entries) return mm_fail(path, P.message);
    } else {
      const long long need = entries - count;  // lines of this part to keep
      long long taken = 0;
      size_t k = 0;
      while (k < P.tris.size() && taken < need) {
        tris.push_back(P.tris[k]);
        ++k;
        if (k < P.tris.size() && (P.tris[k].j & kMirror)) tris.push_back(P.tris[k++]);
        ++taken;
      }
      count += taken;
    }
    P.tris.clear();
    P.tris.shrink_to_fit();
  }
  if (count != entries)
    return mm_fail(path, "expected " + std::to_string(entries) + " entries but found " + std::to_string(count));

  // rowptr holds rows + 1 int32 offsets: with 2^31-1 rows that count is not
  // an int, and the reference's reader fails at this point with the
  // std::vector length error quoted below (its rows + 1 overflows).
  if (rows == 2147483647LL)
    return fail(SPMVB_ERR_INVALID_MATRIX, "Matrix Market: " + path +
                                              ": 2147483647 rows leave no int32 room for rowptr's rows + 1 "
                                              "entries (cannot create std::vector larger than max_size())");

  // CSR: counting sort by row in file order, then each row sorted by column.
  A.m = static_cast<int32_t>(rows);
  A.n = static_cast<int32_t>(cols);
  A.nnz = static_cast<int64_t>(tris.size());
  if (A.nnz > INT32_MAX) return fail(SPMVB_ERR_UNSUPPORTED, "Matrix Market: " + path + ": more than 2^31-1 entries");
  A.rowptr.assign(static_cast<size_t>(A.m) + 1, 0);
  A.colind.resize(tris.size());
  A.values.resize(tris.size());
  for (const auto& t : tris) A.rowptr[t.i + 1]++;
  for (int32_t i = 0; i < A.m; ++i) A.rowptr[i + 1] += A.rowptr[i];
  {
    std::vector<int32_t> cursor(A.rowptr.begin(), A.rowptr.end() - (A.m > 0 ? 1 : 0));
    for (const auto& t : tris) {
      const int32_t pos = cursor[t.i]++;
      A.colind[pos] = static_cast<int32_t>(t.j & ~kMirror);
      A.values[pos] = t.v;
    }
  }
  tris.clear();
  tris.shrink_to_fit();
  // Rows in T nnz-balanced ranges, sorted independently.
  auto sort_rows = [&A](int32_t r0, int32_t r1) {
    std::vector<std::pair<int32_t, double>> row;
    for (int32_t i = r0; i < r1; ++i) {
      const int32_t s = A.rowptr[i], t = A.rowptr[i + 1];
      if (t - s <= 1) continue;
      row.clear();
      for (int32_t q = s; q < t; ++q) row.emplace_back(A.colind[q], A.values[q]);
      std::sort(row.begin(), row.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
      for (int32_t q = s; q < t; ++q) {
        A.colind[q] = row[q - s].first;
        A.values[q] = row[q - s].second;
      }
    }
  };
  std::vector<int32_t> rb(T + 1, A.m);
  rb[0] = 0;
  for (int t = 1; t < T; ++t)
    rb[t] = static_cast<int32_t>(std::lower_bound(A.rowptr.begin(), A.rowptr.end(), A.nnz * t / T) - A.rowptr.begin());
  for (int t = 1; t <= T; ++t) rb[t] = std::min(std::max(rb[t], rb[t - 1]), A.m);
  std::vector<std::thread> pool;
  for (int t = 1; t < T; ++t) pool.emplace_back(sort_rows, rb[t], rb[t + 1]);
  sort_rows(rb[0], rb[1]);
  for (auto& th : pool) th.join();
  return SPMVB_OK;
}

// Binary CSR cache: a 40-byte header, then rowptr, colind, values (f64).
constexpr char kMagic[8] = {'S', 'P', 'M', 'V', 'B', 'C', 'S', 'R'};
struct CacheHeader {
  char magic[8];
  uint32_t version;
  uint32_t value_bytes;
  int32_t m, n;
  int64_t nnz;
  int64_t reserved;
};
static_assert(sizeof(CacheHeader) == 40, "cache header layout");

}  // namespace

extern "C" {

spmvb_status spmvb_read_matrix_market(const char* path, int threads, spmvb_host_csr* out) {
  clear_error();
  if (!path || !out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  auto A = std::make_unique<spmvb_host_csr_st>();
  try {
    SPMVB_TRY(read_mtx(path, threads, *A));
  } catch (const std::bad_alloc&) {
    return fail(SPMVB_ERR_OUT_OF_MEMORY, std::string("Matrix Market: ") + path + ": out of host memory");
  }
  *out = A.release();
  return SPMVB_OK;
}

spmvb_status spmvb_csr_cache_write(const char* path, int32_t m, int32_t n, int64_t nnz, const int32_t* rowptr,
                                   const int32_t* colind, const double* values) {
  clear_error();
  if (!path || !rowptr || (nnz > 0 && (!colind || !values))) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  SPMVB_TRY(spmvb_csr_validate(m, n, nnz, rowptr, colind, nullptr));
  FILE* f = std::fopen(path, "wb");
  if (!f) return fail(SPMVB_ERR_IO, std::string(path) + ": cannot open for writing");
  CacheHeader h{};
  std::memcpy(h.magic, kMagic, 8);
  h.version = 1;
  h.value_bytes = 8;
  h.m = m;
  h.n = n;
  h.nnz = nnz;
  bool ok = std::fwrite(&h, sizeof(h), 1, f) == 1;
  ok = ok && std::fwrite(rowptr, 4, static_cast<size_t>(m) + 1, f) == static_cast<size_t>(m) + 1;
  ok = ok && (nnz == 0 || std::fwrite(colind, 4, static_cast<size_t>(nnz), f) == static_cast<size_t>(nnz));
  ok = ok && (nnz == 0 || std::fwrite(values, 8, static_cast<size_t>(nnz), f) == static_cast<size_t>(nnz));
  ok = (std::fclose(f) == 0) && ok;
  if (!ok) return fail(SPMVB_ERR_IO, std::string(path) + ": write failed");
  return SPMVB_OK;
}

spmvb_status spmvb_csr_cache_read(const char* path, spmvb_host_csr* out) {
  clear_error();
  if (!path || !out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  FILE* f = std::fopen(path, "rb");
  if (!f) return fail(SPMVB_ERR_IO, std::string(path) + ": cannot open file");
  CacheHeader h{};
  if (std::fread(&h, sizeof(h), 1, f) != 1 || std::memcmp(h.magic, kMagic, 8) != 0 || h.version != 1 ||
      h.value_bytes != 8 || h.m < 0 || h.n < 0 || h.nnz < 0 || h.nnz > INT32_MAX) {
    std::fclose(f);
    return fail(SPMVB_ERR_INVALID_MATRIX, std::string(path) + ": not a CSR cache file of this version");
  }
  // The header's sizes must account for the whole file before anything is
  // allocated: a damaged header cannot make the reader claim (and zero) more
  // memory than the file holds.
  const long long expect = static_cast<long long>(sizeof(h)) + (static_cast<long long>(h.m) + 1) * 4 +
                           static_cast<long long>(h.nnz) * 12;
  if (std::fseek(f, 0, SEEK_END) != 0) {
    std::fclose(f);
    return fail(SPMVB_ERR_IO, std::string(path) + ": cannot determine the file size");
  }
  const long long size = std::ftell(f);
  if (size != expect) {
    std::fclose(f);
    return fail(SPMVB_ERR_INVALID_MATRIX, std::string(path) + ": truncated CSR cache file (" +
                                              std::to_string(size) + " bytes, the header describes " +
                                              std::to_string(expect) + ")");
  }
  std::fseek(f, static_cast<long>(sizeof(h)), SEEK_SET);
  auto A = std::make_unique<spmvb_host_csr_st>();
  A->m = h.m;
  A->n = h.n;
  A->nnz = h.nnz;
  try {
    A->rowptr.resize(static_cast<size_t>(h.m) + 1);
    A->colind.resize(static_cast<size_t>(h.nnz));
    A->values.resize(static_cast<size_t>(h.nnz));
  } catch (const std::bad_alloc&) {
    std::fclose(f);
    return fail(SPMVB_ERR_OUT_OF_MEMORY, std::string(path) + ": out of host memory");
  }
  bool ok = std::fread(A->rowptr.data(), 4, A->rowptr.size(), f) == A->rowptr.size();
  ok = ok && std::fread(A->colind.data(), 4, A->colind.size(), f) == A->colind.size();
  ok = ok && std::fread(A->values.data(), 8, A->values.size(), f) == A->values.size();
  std::fclose(f);
  if (!ok) return fail(SPMVB_ERR_INVALID_MATRIX, std::string(path) + ": truncated CSR cache file");
  SPMVB_TRY(spmvb_csr_validate(A->m, A->n, A->nnz, A->rowptr.data(), A->colind.data(), nullptr));
  *out = A.release();
  return SPMVB_OK;
}

spmvb_status spmvb_host_csr_get(spmvb_host_csr A, int32_t* m, int32_t* n, int64_t* nnz, const int32_t** rowptr,
                                const int32_t** colind, const double** values) {
  clear_error();
  if (!A) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null handle");
  if (m) *m = A->m;
  if (n) *n = A->n;
  if (nnz) *nnz = A->nnz;
  if (rowptr) *rowptr = A->rowptr.data();
  if (colind) *colind = A->colind.data();
  if (values) *values = A->values.data();
  return SPMVB_OK;
}

void spmvb_host_csr_free(spmvb_host_csr A) { delete A; }

}  // extern "C"
