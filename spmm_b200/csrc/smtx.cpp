// .smtx reader / writer, straight to CSR.
//
// Format (smtx_input_to_Dense, src/file_input.cu:135-193):
//   line 1: "M, K, nnz"            fields split on ',' (:141-148)
//   line 2: M + 1 row offsets      split on ' '       (:155-163)
//   rest  : nnz column indices     split on ' '       (:171-180)
// The reference scatters 1.0 into a dense M x K matrix and converts that to
// CSR (src/miscalleneous.cu:29-65), so its effective matrix has, per row, the
// distinct listed columns in ascending order, every value 1.0.  This reader
// builds that CSR directly: columns are sorted per row and, for pattern files,
// repeated columns collapse into one entry.  Optional values live in a sidecar
// "<path>.val" (nnz little-endian float32, in file order), which the reference
// never reads; with values a repeated column is a format error.
#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <vector>

#include "internal.h"

using namespace tca;

namespace {

bool read_file(const char *path, std::vector<char> *buf)
{
    FILE *f = std::fopen(path, "rb");
    if (!f) return false;
    std::fseek(f, 0, SEEK_END);
    long sz = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    buf->resize((size_t)(sz > 0 ? sz : 0) + 1);
    size_t got = sz > 0 ? std::fread(buf->data(), 1, (size_t)sz, f) : 0;
    std::fclose(f);
    buf->resize(got + 1);
    (*buf)[got] = 0;
    return true;
}

struct Cursor {
    const char *p, *end;
    // Next non-negative integer on the current line; false at end of line.
    bool next_on_line(int64_t *v, bool *bad)
    {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\r')) p++;
        if (p >= end || *p == '\n') return false;
        if (*p < '0' || *p > '9') {
            *bad = true;
            return false;
        }
        int64_t x = 0;
        while (p < end && *p >= '0' && *p <= '9') {
            x = x * 10 + (*p - '0');
            if (x > (int64_t)1 << 40) {
                *bad = true;
                return false;
            }
            p++;
        }
        *v = x;
        return true;
    }
    bool next_line()
    {
        while (p < end && *p != '\n') p++;
        if (p < end) {
            p++;
            return true;
        }
        return false;
    }
};

}  // namespace

extern "C" tcaspmm_status tcaspmm_smtx_read(const char *path, tcaspmm_csr *out)
{
    if (!path || !out) return fail(TCASPMM_ERR_INVALID_ARG, "smtx_read: NULL argument");
    std::memset(out, 0, sizeof(*out));
    std::vector<char> buf;
    if (!read_file(path, &buf)) return fail(TCASPMM_ERR_IO, "cannot open %s: %s", path, std::strerror(errno));
    Cursor cur{buf.data(), buf.data() + buf.size() - 1};

    // Header: three integers separated by ',' (whitespace tolerated).
    int64_t hdr[3];
    {
        const char *line_end = cur.p;
        while (line_end < cur.end && *line_end != '\n') line_end++;
        std::string line(cur.p, line_end);
        long long m, k, z;
        char tail;
        int n = std::sscanf(line.c_str(), " %lld , %lld , %lld %c", &m, &k, &z, &tail);
        if (n != 3 || m < 0 || k < 0 || z < 0)
            return fail(TCASPMM_ERR_FORMAT, "%s: header must be \"M, K, nnz\", got \"%.80s\"", path,
                        line.c_str());
        hdr[0] = m;
        hdr[1] = k;
        hdr[2] = z;
        cur.next_line();
    }
    const int64_t M = hdr[0], K = hdr[1], nnz_file = hdr[2];
    if (M > INT32_MAX - 1 || K > INT32_MAX || nnz_file > INT32_MAX)
        return fail(TCASPMM_ERR_UNSUPPORTED, "%s: dimensions above 2^31-1", path);

    std::vector<int64_t> rp;
    rp.reserve(M + 1);
    bool bad = false;
    int64_t v;
    while (cur.next_on_line(&v, &bad)) rp.push_back(v);
    if (bad || (int64_t)rp.size() != M + 1)
        return fail(TCASPMM_ERR_FORMAT, "%s: line 2 must hold %lld row offsets, found %zu%s", path,
                    (long long)(M + 1), rp.size(), bad ? " (bad token)" : "");
    if (rp[0] != 0 || rp[M] != nnz_file)
        return fail(TCASPMM_ERR_FORMAT, "%s: row offsets must run from 0 to nnz=%lld", path,
                    (long long)nnz_file);
    for (int64_t i = 0; i < M; i++)
        if (rp[i + 1] < rp[i]) return fail(TCASPMM_ERR_FORMAT, "%s: row offsets decrease at row %lld", path, (long long)i);
    cur.next_line();

    std::vector<int32_t> col;
    col.reserve(nnz_file);
    for (;;) {
        while (cur.next_on_line(&v, &bad)) {
            if (v >= K)
                return fail(TCASPMM_ERR_FORMAT, "%s: column %lld out of range [0, %lld)", path, (long long)v, (long long)K);
            if ((int64_t)col.size() >= nnz_file)
                return fail(TCASPMM_ERR_FORMAT, "%s: more than nnz=%lld column indices", path, (long long)nnz_file);
            col.push_back((int32_t)v);
        }
        if (bad) return fail(TCASPMM_ERR_FORMAT, "%s: bad column token", path);
        if (!cur.next_line()) break;
    }
    if ((int64_t)col.size() != nnz_file)
        return fail(TCASPMM_ERR_FORMAT, "%s: found %zu column indices, header says %lld", path, col.size(),
                    (long long)nnz_file);

    // Optional values sidecar.
    std::vector<float> val;
    bool has_val = false;
    {
        std::string vpath = std::string(path) + ".val";
        FILE *f = std::fopen(vpath.c_str(), "rb");
        if (f) {
            has_val = true;
            val.resize(nnz_file);
            size_t got = nnz_file ? std::fread(val.data(), sizeof(float), nnz_file, f) : 0;
            int extra = std::fgetc(f);
            std::fclose(f);
            if ((int64_t)got != nnz_file || extra != EOF)
                return fail(TCASPMM_ERR_FORMAT, "%s: expected %lld float32 values", vpath.c_str(), (long long)nnz_file);
        }
    }

    // Sort each row by column; collapse repeats (pattern) or reject them (values).
    std::vector<int64_t> out_rp(M + 1, 0);
    std::vector<int32_t> out_col;
    std::vector<float> out_val;
    out_col.reserve(nnz_file);
    if (has_val) out_val.reserve(nnz_file);
    std::vector<int64_t> perm;
    for (int64_t i = 0; i < M; i++) {
        const int64_t b = rp[i], e = rp[i + 1];
        bool sorted = true;
        for (int64_t j = b + 1; j < e; j++)
            if (col[j] <= col[j - 1]) sorted = false;
        if (sorted) {
            out_col.insert(out_col.end(), col.begin() + b, col.begin() + e);
            if (has_val) out_val.insert(out_val.end(), val.begin() + b, val.begin() + e);
        } else {
            perm.resize(e - b);
            std::iota(perm.begin(), perm.end(), b);
            std::stable_sort(perm.begin(), perm.end(), [&](int64_t x, int64_t y) { return col[x] < col[y]; });
            int32_t last = -1;
            for (int64_t q : perm) {
                if (col[q] == last) {
                    if (has_val)
                        return fail(TCASPMM_ERR_FORMAT, "%s: column %d repeated in row %lld", path, col[q], (long long)i);
                    continue;
                }
                last = col[q];
                out_col.push_back(col[q]);
                if (has_val) out_val.push_back(val[q]);
            }
        }
        out_rp[i + 1] = (int64_t)out_col.size();
    }
    return csr_from_rows(M, K, out_rp, out_col, has_val ? &out_val : nullptr, out);
}

extern "C" tcaspmm_status tcaspmm_smtx_write(const char *path, const tcaspmm_csr *A)
{
    if (!path || !A) return fail(TCASPMM_ERR_INVALID_ARG, "smtx_write: NULL argument");
    tcaspmm_status s = tcaspmm_csr_validate(A);
    if (s != TCASPMM_OK) return s;
    FILE *f = std::fopen(path, "wb");
    if (!f) return fail(TCASPMM_ERR_IO, "cannot create %s: %s", path, std::strerror(errno));
    std::vector<char> line;
    line.reserve(1 << 20);
    char tmp[32];
    auto flush = [&]() {
        if (!line.empty()) std::fwrite(line.data(), 1, line.size(), f);
        line.clear();
    };
    std::fprintf(f, "%lld, %lld, %lld\n", (long long)A->nrow, (long long)A->ncol, (long long)A->nnz);
    for (int64_t i = 0; i <= A->nrow; i++) {
        int n = std::snprintf(tmp, sizeof(tmp), i ? " %lld" : "%lld", (long long)A->row_ptr[i]);
        line.insert(line.end(), tmp, tmp + n);
        if (line.size() > (1 << 20) - 64) flush();
    }
    line.push_back('\n');
    for (int64_t j = 0; j < A->nnz; j++) {
        int n = std::snprintf(tmp, sizeof(tmp), j ? " %d" : "%d", A->col_idx[j]);
        line.insert(line.end(), tmp, tmp + n);
        if (line.size() > (1 << 20) - 64) flush();
    }
    line.push_back('\n');
    flush();
    bool ok = std::fclose(f) == 0;
    std::string vpath = std::string(path) + ".val";
    if (A->val) {
        FILE *g = std::fopen(vpath.c_str(), "wb");
        if (!g) return fail(TCASPMM_ERR_IO, "cannot create %s", vpath.c_str());
        if (A->nnz) ok = ok && std::fwrite(A->val, sizeof(float), A->nnz, g) == (size_t)A->nnz;
        ok = (std::fclose(g) == 0) && ok;
    } else {
        std::remove(vpath.c_str());  // a stale sidecar would attach wrong values
    }
    return ok ? TCASPMM_OK : fail(TCASPMM_ERR_IO, "write to %s failed", path);
}
