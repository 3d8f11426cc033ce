// Matrix Market reader and a binary CSR companion format.
//
// Matrix Market: replaces mtx_input_to_CSR (src/file_input.cu:64-134), which skips
// lines starting with '%', reads "rows cols nnz", then "r c [v]" per entry
// (1-based unless the caller says the file is 0-based, src/file_input.cu:98-102),
// groups entries by row and asserts the entry count.  Here the banner's field
// (real / integer / pattern) and symmetry (general / symmetric /
// skew-symmetric) are honoured (symmetric files list one triangle; the mirror is
// added), columns are sorted within each row and repeated entries are summed,
// so the result is a valid tcaspmm CSR.
//
// Binary CSR (".csrb"): "TCACSR01", int64 nrow, ncol, nnz, flags (bit 0: values
// present), then int64 row offsets [nrow+1], int32 columns [nnz] and, if
// flagged, float32 values [nnz]; all little-endian.  Loads 100M-nonzero graphs in
// the time of a file copy.
#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include "internal.h"

using namespace tca;

namespace {

struct Entry {
    int64_t r, c;
    float v;
};

bool starts_with_ci(const char *s, const char *prefix)
{
    for (; *prefix; ++s, ++prefix)
        if (std::tolower((unsigned char)*s) != *prefix) return false;
    return true;
}

}  // namespace

extern "C" tcaspmm_status tcaspmm_mtx_read(const char *path, int zero_based, tcaspmm_csr *out)
{
    if (!path || !out) return fail(TCASPMM_ERR_INVALID_ARG, "mtx_read: NULL argument");
    std::memset(out, 0, sizeof(*out));
    FILE *f = std::fopen(path, "r");
    if (!f) return fail(TCASPMM_ERR_IO, "cannot open %s: %s", path, std::strerror(errno));
    char line[4096];
    bool pattern = false, symmetric = false, skew = false, have_size = false;
    long long M = 0, K = 0, Z = 0;
    std::vector<Entry> ent;
    tcaspmm_status st = TCASPMM_OK;
    long long lineno = 0;
    while (std::fgets(line, sizeof(line), f)) {
        ++lineno;
        if (line[0] == '%') {
            if (lineno == 1 && starts_with_ci(line, "%%matrixmarket")) {
                std::string b(line);
                for (auto &ch : b) ch = (char)std::tolower((unsigned char)ch);
                if (b.find("coordinate") == std::string::npos || b.find("complex") != std::string::npos) {
                    st = fail(TCASPMM_ERR_UNSUPPORTED, "%s: only real/integer/pattern coordinate matrices", path);
                    break;
                }
                pattern = b.find("pattern") != std::string::npos;
                skew = b.find("skew-symmetric") != std::string::npos;
                symmetric = skew || b.find("symmetric") != std::string::npos || b.find("hermitian") != std::string::npos;
            }
            continue;
        }
        char *p = line;
        while (*p == ' ' || *p == '\t') ++p;
        if (*p == '\n' || *p == '\r' || *p == 0) continue;
        if (!have_size) {
            if (std::sscanf(p, "%lld %lld %lld", &M, &K, &Z) != 3 || M < 0 || K < 0 || Z < 0) {
                st = fail(TCASPMM_ERR_FORMAT, "%s:%lld: size line must be \"rows cols nnz\"", path, lineno);
                break;
            }
            if (M > INT32_MAX - 1 || K > INT32_MAX || Z > INT32_MAX) {
                st = fail(TCASPMM_ERR_UNSUPPORTED, "%s: dimensions above 2^31-1", path);
                break;
            }
            have_size = true;
            ent.reserve((size_t)Z * (symmetric ? 2 : 1));
            continue;
        }
        long long r, c;
        double v = 1.0;
        const int n = std::sscanf(p, "%lld %lld %lf", &r, &c, &v);
        if (n < 2 || (!pattern && n < 3)) {
            st = fail(TCASPMM_ERR_FORMAT, "%s:%lld: bad entry", path, lineno);
            break;
        }
        if (!zero_based) {
            --r;
            --c;
        }
        if (r < 0 || r >= M || c < 0 || c >= K) {
            st = fail(TCASPMM_ERR_FORMAT, "%s:%lld: entry (%lld, %lld) outside %lldx%lld", path, lineno, r, c, M, K);
            break;
        }
        if ((long long)ent.size() >= Z * (symmetric ? 2 : 1)) {
            st = fail(TCASPMM_ERR_FORMAT, "%s: more than nnz=%lld entries", path, Z);
            break;
        }
        ent.push_back(Entry{r, c, (float)v});
        if (symmetric && r != c) {
            if (c >= M || r >= K) {
                st = fail(TCASPMM_ERR_FORMAT, "%s: symmetric matrix must be square", path);
                break;
            }
            ent.push_back(Entry{c, r, skew ? -(float)v : (float)v});
        }
    }
    std::fclose(f);
    if (st != TCASPMM_OK) return st;
    if (!have_size) return fail(TCASPMM_ERR_FORMAT, "%s: no size line", path);
    // The entry count is checked as mtx_input_to_CSR asserts it (src/file_input.cu:114).
    int64_t listed = (int64_t)ent.size();
    if (symmetric) {
        int64_t off = 0;
        for (const Entry &e : ent) off += e.r != e.c;
        listed -= off / 2;
    }
    if (listed != Z) return fail(TCASPMM_ERR_FORMAT, "%s: %lld entries listed, header says %lld", path, (long long)listed, Z);
    std::stable_sort(ent.begin(), ent.end(), [](const Entry &a, const Entry &b) { return a.r != b.r ? a.r < b.r : a.c < b.c; });
    std::vector<int64_t> rp(M + 1, 0);
    std::vector<int32_t> col;
    std::vector<float> val;
    col.reserve(ent.size());
    val.reserve(ent.size());
    for (size_t i = 0; i < ent.size(); ++i) {
        if (i > 0 && ent[i].r == ent[i - 1].r && ent[i].c == ent[i - 1].c) {
            val.back() += ent[i].v;  // repeated entry: summed
            continue;
        }
        col.push_back((int32_t)ent[i].c);
        val.push_back(ent[i].v);
        rp[ent[i].r + 1]++;
    }
    for (int64_t i = 0; i < M; ++i) rp[i + 1] += rp[i];
    return csr_from_rows(M, K, rp, col, pattern ? nullptr : &val, out);
}

extern "C" tcaspmm_status tcaspmm_csrbin_write(const char *path, const tcaspmm_csr *A)
{
    if (!path || !A) return fail(TCASPMM_ERR_INVALID_ARG, "csrbin_write: NULL argument");
    tcaspmm_status s = tcaspmm_csr_validate(A);
    if (s != TCASPMM_OK) return s;
    FILE *f = std::fopen(path, "wb");
    if (!f) return fail(TCASPMM_ERR_IO, "cannot create %s: %s", path, std::strerror(errno));
    const int64_t hdr[4] = {A->nrow, A->ncol, A->nnz, A->val ? 1 : 0};
    bool ok = std::fwrite("TCACSR01", 1, 8, f) == 8 && std::fwrite(hdr, 8, 4, f) == 4 &&
              std::fwrite(A->row_ptr, 8, A->nrow + 1, f) == (size_t)(A->nrow + 1) &&
              (A->nnz == 0 || std::fwrite(A->col_idx, 4, A->nnz, f) == (size_t)A->nnz) &&
              (!A->val || A->nnz == 0 || std::fwrite(A->val, 4, A->nnz, f) == (size_t)A->nnz);
    ok = (std::fclose(f) == 0) && ok;
    return ok ? TCASPMM_OK : fail(TCASPMM_ERR_IO, "write to %s failed", path);
}

extern "C" tcaspmm_status tcaspmm_csrbin_read(const char *path, tcaspmm_csr *out)
{
    if (!path || !out) return fail(TCASPMM_ERR_INVALID_ARG, "csrbin_read: NULL argument");
    std::memset(out, 0, sizeof(*out));
    FILE *f = std::fopen(path, "rb");
    if (!f) return fail(TCASPMM_ERR_IO, "cannot open %s: %s", path, std::strerror(errno));
    char magic[8];
    int64_t hdr[4];
    if (std::fread(magic, 1, 8, f) != 8 || std::memcmp(magic, "TCACSR01", 8) != 0 || std::fread(hdr, 8, 4, f) != 4 ||
        hdr[0] < 0 || hdr[1] < 0 || hdr[2] < 0 || (hdr[3] & ~1LL) != 0) {
        std::fclose(f);
        return fail(TCASPMM_ERR_FORMAT, "%s: not a tcaspmm binary CSR file", path);
    }
    if (hdr[0] > INT32_MAX - 1 || hdr[1] > INT32_MAX || hdr[2] > INT32_MAX) {
        std::fclose(f);
        return fail(TCASPMM_ERR_UNSUPPORTED, "%s: dimensions above 2^31-1", path);
    }
    tcaspmm_status s = tcaspmm_csr_alloc(hdr[0], hdr[1], hdr[2], (int)(hdr[3] & 1), out);
    if (s != TCASPMM_OK) {
        std::fclose(f);
        return s;
    }
    bool ok = std::fread(out->row_ptr, 8, hdr[0] + 1, f) == (size_t)(hdr[0] + 1) &&
              (hdr[2] == 0 || std::fread(out->col_idx, 4, hdr[2], f) == (size_t)hdr[2]) &&
              (!out->val || hdr[2] == 0 || std::fread(out->val, 4, hdr[2], f) == (size_t)hdr[2]) &&
              std::fgetc(f) == EOF;
    std::fclose(f);
    if (!ok) {
        tcaspmm_csr_free(out);
        return fail(TCASPMM_ERR_FORMAT, "%s: truncated or oversized binary CSR", path);
    }
    s = tcaspmm_csr_validate(out);
    if (s != TCASPMM_OK) tcaspmm_csr_free(out);
    return s;
}
