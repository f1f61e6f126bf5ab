// lg_mtx.cu — Matrix Market files <-> CSR (host code only).
//
// Reference: src/main.cu:129-244 (export_matrix_market / load_matrix_market:
// fscanf one entry at a time, insertion sort per row, "%.15e" on output, exit()
// on any error).  Here:
//   * read: the whole file in memory, entries parsed with std::from_chars on
//     all host cores (one slice of lines per thread), `general` and
//     `symmetric` / `skew-symmetric` (mirrored entries added), `real`,
//     `integer` and `pattern` (value 1); COO -> CSR by a counting sort on the
//     row, columns sorted inside each row, duplicate entries summed;
//   * write: `coordinate real general` (or `symmetric`, lower triangle only),
//     values in the shortest form that reads back to the same double
//     (std::to_chars), lines formatted on all cores;
//   * errors come back as LG_ERR_INVALID with the line that failed.
#include "../../include/lanczos_b200.h"

#include <algorithm>
#include <charconv>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace lg {
extern thread_local std::string g_last_error;
}

using lg::g_last_error;

struct lg_mtx {
  int nrows = 0, ncols = 0;
  std::vector<int> rowptr, col;
  std::vector<double> val;
};

namespace {

int fail(const std::string& m) {
  g_last_error = "Matrix Market: " + m;
  return LG_ERR_INVALID;
}

bool read_file(const char* path, std::string& out) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return false;
  std::fseek(f, 0, SEEK_END);
  const long sz = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  out.resize(sz > 0 ? (size_t)sz : 0);
  const size_t got = sz > 0 ? std::fread(&out[0], 1, (size_t)sz, f) : 0;
  std::fclose(f);
  return got == out.size();
}

int n_threads() {
  const unsigned h = std::thread::hardware_concurrency();
  return (int)std::max(1u, std::min(h, 64u));
}

const char* skip_ws(const char* p, const char* e) {
  while (p < e && (*p == ' ' || *p == '\t' || *p == '\r')) ++p;
  return p;
}

struct Coo {
  std::vector<int> r, c;
  std::vector<double> v;
  long long bad_line = -1;
};

}  // namespace

extern "C" int lg_mtx_read(const char* path, lg_mtx** out, int* nrows, int* ncols, long long* nnz) {
  if (!path || !out || !nrows || !ncols || !nnz) return fail("null argument");
  *out = nullptr;
  std::string buf;
  if (!read_file(path, buf)) return fail(std::string("cannot read ") + path);
  const char* p = buf.data();
  const char* end = p + buf.size();
  // banner
  const char* eol = (const char*)std::memchr(p, '\n', (size_t)(end - p));
  if (!eol) eol = end;
  std::string banner(p, eol);
  for (char& ch : banner) ch = (char)std::tolower((unsigned char)ch);
  if (banner.rfind("%%matrixmarket", 0) != 0) return fail("missing %%MatrixMarket banner");
  if (banner.find("coordinate") == std::string::npos) return fail("only the coordinate format is supported");
  if (banner.find("complex") != std::string::npos) return fail("complex matrices are not supported");
  const bool pattern = banner.find("pattern") != std::string::npos;
  const bool skew = banner.find("skew-symmetric") != std::string::npos;
  const bool sym = skew || banner.find("symmetric") != std::string::npos || banner.find("hermitian") != std::string::npos;
  p = eol < end ? eol + 1 : end;
  // comments, then the size line
  while (p < end && (*p == '%' || *p == '\n' || *p == '\r')) {
    const char* q = (const char*)std::memchr(p, '\n', (size_t)(end - p));
    p = q ? q + 1 : end;
  }
  long long R = 0, Cc = 0, NZ = 0;
  {
    const char* q = skip_ws(p, end);
    auto r1 = std::from_chars(q, end, R);
    q = skip_ws(r1.ptr, end);
    auto r2 = std::from_chars(q, end, Cc);
    q = skip_ws(r2.ptr, end);
    auto r3 = std::from_chars(q, end, NZ);
    if (r1.ec != std::errc() || r2.ec != std::errc() || r3.ec != std::errc() || R < 1 || Cc < 1 || NZ < 0 ||
        R > 2147483647ll || Cc > 2147483647ll)
      return fail("bad size line");
    const char* nl = (const char*)std::memchr(r3.ptr, '\n', (size_t)(end - r3.ptr));
    p = nl ? nl + 1 : end;
  }
  // line starts of the entries, then parse them on all cores
  std::vector<const char*> lines;
  lines.reserve((size_t)NZ + 1);
  for (const char* q = p; q < end && (long long)lines.size() < NZ;) {
    const char* s = skip_ws(q, end);
    const char* nl = (const char*)std::memchr(q, '\n', (size_t)(end - q));
    if (s < end && *s != '\n' && *s != '%') lines.push_back(q);
    q = nl ? nl + 1 : end;
  }
  if ((long long)lines.size() < NZ) return fail("fewer entries than the size line announces");
  const int T = n_threads();
  std::vector<Coo> parts((size_t)T);
  auto work = [&](int t) {
    const size_t b = lines.size() * (size_t)t / (size_t)T, e = lines.size() * (size_t)(t + 1) / (size_t)T;
    Coo& o = parts[(size_t)t];
    const size_t cap = (e - b) * (sym ? 2 : 1);
    o.r.reserve(cap);
    o.c.reserve(cap);
    o.v.reserve(cap);
    for (size_t i = b; i < e; ++i) {
      const char* q = skip_ws(lines[i], end);
      long long r = 0, c = 0;
      double v = 1.0;
      auto a1 = std::from_chars(q, end, r);
      q = skip_ws(a1.ptr, end);
      auto a2 = std::from_chars(q, end, c);
      bool ok = a1.ec == std::errc() && a2.ec == std::errc() && r >= 1 && r <= R && c >= 1 && c <= Cc;
      if (ok && !pattern) {
        q = skip_ws(a2.ptr, end);
        auto a3 = std::from_chars(q, end, v);
        ok = a3.ec == std::errc();
      }
      if (!ok) {
        o.bad_line = (long long)i;
        return;
      }
      o.r.push_back((int)(r - 1));
      o.c.push_back((int)(c - 1));
      o.v.push_back(v);
      if (sym && r != c) {
        o.r.push_back((int)(c - 1));
        o.c.push_back((int)(r - 1));
        o.v.push_back(skew ? -v : v);
      }
    }
  };
  {
    std::vector<std::thread> th;
    for (int t = 1; t < T; ++t) th.emplace_back(work, t);
    work(0);
    for (auto& x : th) x.join();
  }
  for (const Coo& o : parts)
    if (o.bad_line >= 0) return fail("cannot parse entry " + std::to_string(o.bad_line + 1));
  // COO -> CSR: counting sort on the row, then columns sorted per row,
  // duplicates summed
  lg_mtx* m = new lg_mtx();
  m->nrows = (int)R;
  m->ncols = (int)Cc;
  std::vector<long long> cnt((size_t)R + 1, 0);
  for (const Coo& o : parts)
    for (int r : o.r) ++cnt[(size_t)r + 1];
  for (size_t i = 1; i < cnt.size(); ++i) cnt[i] += cnt[i - 1];
  const long long total = cnt[(size_t)R];
  std::vector<int> tc((size_t)total);
  std::vector<double> tv((size_t)total);
  {
    std::vector<long long> fill(cnt.begin(), cnt.end() - 1);
    for (const Coo& o : parts)
      for (size_t i = 0; i < o.r.size(); ++i) {
        const long long at = fill[(size_t)o.r[i]]++;
        tc[(size_t)at] = o.c[i];
        tv[(size_t)at] = o.v[i];
      }
  }
  parts.clear();
  m->rowptr.assign((size_t)R + 1, 0);
  m->col.reserve((size_t)total);
  m->val.reserve((size_t)total);
  std::vector<std::pair<int, double>> row;
  for (long long r = 0; r < R; ++r) {
    row.clear();
    for (long long k = cnt[(size_t)r]; k < cnt[(size_t)r + 1]; ++k) row.emplace_back(tc[(size_t)k], tv[(size_t)k]);
    std::stable_sort(row.begin(), row.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
    for (size_t k = 0; k < row.size(); ++k) {
      if (!m->col.empty() && (long long)m->col.size() > m->rowptr[(size_t)r] && m->col.back() == row[k].first)
        m->val.back() += row[k].second;
      else {
        m->col.push_back(row[k].first);
        m->val.push_back(row[k].second);
      }
    }
    if ((long long)m->col.size() > 2147483647ll) {
      delete m;
      return fail("more than 2^31 - 1 nonzeros");
    }
    m->rowptr[(size_t)r + 1] = (int)m->col.size();
  }
  *out = m;
  *nrows = m->nrows;
  *ncols = m->ncols;
  *nnz = (long long)m->col.size();
  return LG_OK;
}

extern "C" int lg_mtx_copy(const lg_mtx* m, int* row_ptr, int* col, double* vals) {
  if (!m || !row_ptr || (!m->col.empty() && (!col || !vals))) return fail("null argument");
  std::copy(m->rowptr.begin(), m->rowptr.end(), row_ptr);
  std::copy(m->col.begin(), m->col.end(), col);
  std::copy(m->val.begin(), m->val.end(), vals);
  return LG_OK;
}

extern "C" int lg_mtx_free(lg_mtx* m) {
  delete m;
  return LG_OK;
}

extern "C" int lg_mtx_write(const char* path, int nrows, int ncols, const int* row_ptr, const int* col,
                            const double* vals, int symmetric) {
  if (!path || nrows < 1 || ncols < 1 || !row_ptr || (row_ptr[nrows] > 0 && (!col || !vals)))
    return fail("invalid arguments");
  if (row_ptr[0] != 0) return fail("row_ptr must start at 0");
  for (int i = 0; i < nrows; ++i)
    if (row_ptr[i + 1] < row_ptr[i]) return fail("row_ptr is not monotone");
  if (symmetric && nrows != ncols) return fail("a symmetric file needs a square matrix");
  // rows split over the cores; each slice formats its lines into its own buffer
  const int T = n_threads();
  std::vector<std::string> out((size_t)T);
  std::vector<long long> count((size_t)T, 0);
  std::vector<int> bad((size_t)T, 0);
  auto work = [&](int t) {
    const int rb = (int)((long long)nrows * t / T), re = (int)((long long)nrows * (t + 1) / T);
    std::string& s = out[(size_t)t];
    char line[96];
    for (int r = rb; r < re; ++r)
      for (int k = row_ptr[r]; k < row_ptr[r + 1]; ++k) {
        const int c = col[k];
        if (c < 0 || c >= ncols) {
          bad[(size_t)t] = 1;
          return;
        }
        if (symmetric && c > r) continue;   // lower triangle
        char* q = line;
        q = std::to_chars(q, line + sizeof(line), r + 1).ptr;
        *q++ = ' ';
        q = std::to_chars(q, line + sizeof(line), c + 1).ptr;
        *q++ = ' ';
        q = std::to_chars(q, line + sizeof(line), vals[k]).ptr;   // shortest exact form
        *q++ = '\n';
        s.append(line, (size_t)(q - line));
        ++count[(size_t)t];
      }
  };
  {
    std::vector<std::thread> th;
    for (int t = 1; t < T; ++t) th.emplace_back(work, t);
    work(0);
    for (auto& x : th) x.join();
  }
  for (int b : bad)
    if (b) return fail("column index out of range");
  long long total = 0;
  for (long long c : count) total += c;
  FILE* f = std::fopen(path, "wb");
  if (!f) return fail(std::string("cannot write ") + path);
  std::fprintf(f, "%%%%MatrixMarket matrix coordinate real %s\n%d %d %lld\n", symmetric ? "symmetric" : "general",
               nrows, ncols, total);
  bool ok = true;
  for (const std::string& s : out) ok = ok && std::fwrite(s.data(), 1, s.size(), f) == s.size();
  ok = (std::fclose(f) == 0) && ok;
  return ok ? LG_OK : fail(std::string("write failed: ") + path);
}
