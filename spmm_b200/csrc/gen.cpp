// Seeded synthetic inputs.  Every random value is a pure function of
// (seed, stream, index), so the output does not depend on the thread count.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include <omp.h>

#include "internal.h"

using namespace tca;

namespace {

enum Stream : uint64_t {
    S_DENSE = 1,
    S_KEEP = 2,
    S_VAL = 3,
    S_SCALE = 5,
    S_RMAT = 20,
    S_HUBCOL = 21,
    S_POIS = 22,
    S_COL = 23,
    S_UVAL = 24,
};

// Rows given as (row, col) pairs -> CSR with sorted, distinct columns.
// rows[i] are counted first, then scattered and sorted per row in parallel.
void pairs_to_csr(int64_t n, const std::vector<uint32_t> &r, const std::vector<uint32_t> &c,
                  std::vector<int64_t> *rp, std::vector<int32_t> *col)
{
    const int64_t E = (int64_t)r.size();
    std::vector<int64_t> cnt(n + 1, 0);
    for (int64_t e = 0; e < E; e++) cnt[r[e] + 1]++;
    for (int64_t i = 0; i < n; i++) cnt[i + 1] += cnt[i];
    std::vector<int32_t> tmp(E);
    {
        std::vector<int64_t> pos(cnt.begin(), cnt.end() - 1);
        for (int64_t e = 0; e < E; e++) tmp[pos[r[e]]++] = (int32_t)c[e];
    }
    std::vector<int64_t> uniq(n, 0);
#pragma omp parallel for schedule(dynamic, 1024)
    for (int64_t i = 0; i < n; i++) {
        auto b = tmp.begin() + cnt[i], e = tmp.begin() + cnt[i + 1];
        std::sort(b, e);
        uniq[i] = std::unique(b, e) - b;
    }
    rp->assign(n + 1, 0);
    for (int64_t i = 0; i < n; i++) (*rp)[i + 1] = (*rp)[i] + uniq[i];
    col->resize((*rp)[n]);
#pragma omp parallel for schedule(dynamic, 1024)
    for (int64_t i = 0; i < n; i++)
        std::copy(tmp.begin() + cnt[i], tmp.begin() + cnt[i] + uniq[i], col->begin() + (*rp)[i]);
}

}  // namespace

extern "C" {

tcaspmm_status tcaspmm_gen_dense(int64_t rows, int64_t cols, uint64_t seed, tcaspmm_dtype dt, void *out)
{
    if (rows < 0 || cols < 0 || (!out && rows * cols > 0) || !dtype_valid(dt))
        return fail(TCASPMM_ERR_INVALID_ARG, "gen_dense: bad arguments");
    const int64_t n = rows * cols;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        const float x = (float)rng_normal(seed, S_DENSE, (uint64_t)i);
        if (dtype_fp32(dt))
            ((float *)out)[i] = x;
        else if (dt == TCASPMM_F16)
            ((uint16_t *)out)[i] = float_to_half_bits(x);
        else
            ((uint16_t *)out)[i] = float_to_bf16_bits(x);
    }
    return TCASPMM_OK;
}

tcaspmm_status tcaspmm_gen_uniform(int64_t M, int64_t K, double density, uint64_t seed, tcaspmm_csr *out)
{
    if (!out || M < 0 || K < 0 || !(density >= 0.0 && density <= 1.0))
        return fail(TCASPMM_ERR_INVALID_ARG, "gen_uniform: bad arguments");
    std::vector<int64_t> cnt(M + 1, 0);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; i++) {
        int64_t c = 0;
        for (int64_t k = 0; k < K; k++) c += rng_unit(seed, S_KEEP, (uint64_t)(i * K + k)) < density;
        cnt[i + 1] = c;
    }
    for (int64_t i = 0; i < M; i++) cnt[i + 1] += cnt[i];
    std::vector<int32_t> col(cnt[M]);
    std::vector<float> val(cnt[M]);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; i++) {
        int64_t p = cnt[i];
        for (int64_t k = 0; k < K; k++) {
            const uint64_t idx = (uint64_t)(i * K + k);
            if (rng_unit(seed, S_KEEP, idx) < density) {
                col[p] = (int32_t)k;
                val[p] = (float)rng_normal(seed, S_VAL, idx);
                p++;
            }
        }
    }
    return csr_from_rows(M, K, cnt, col, &val, out);
}

tcaspmm_status tcaspmm_gen_magnitude(int64_t M, int64_t K, double sparsity, uint64_t seed, tcaspmm_csr *out)
{
    if (!out || M < 0 || K < 0 || !(sparsity >= 0.0 && sparsity <= 1.0))
        return fail(TCASPMM_ERR_INVALID_ARG, "gen_magnitude: bad arguments");
    const int64_t n = M * K;
    std::vector<float> w(n);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; i++) {
        const double s = std::exp(0.5 * rng_normal(seed, S_SCALE, (uint64_t)i));
        for (int64_t k = 0; k < K; k++)
            w[i * K + k] = (float)(s * rng_normal(seed, S_VAL, (uint64_t)(i * K + k)));
    }
    int64_t keep = (int64_t)std::llround((1.0 - sparsity) * (double)n);
    if (keep > n) keep = n;
    // Global top-`keep` by |w|; ties at the threshold broken by lower index.
    std::vector<float> mag(n);
    for (int64_t i = 0; i < n; i++) mag[i] = std::fabs(w[i]);
    float thr = INFINITY;
    int64_t above = 0;
    if (keep > 0) {
        std::vector<float> tmp(mag);
        std::nth_element(tmp.begin(), tmp.begin() + (n - keep), tmp.end());
        thr = tmp[n - keep];
        for (int64_t i = 0; i < n; i++) above += mag[i] > thr;
    }
    int64_t ties_left = keep - above;
    std::vector<int64_t> rp(M + 1, 0);
    std::vector<int32_t> col;
    std::vector<float> val;
    col.reserve(keep);
    val.reserve(keep);
    for (int64_t i = 0; i < M; i++) {
        for (int64_t k = 0; k < K; k++) {
            const float m = mag[i * K + k];
            bool take = m > thr;
            if (!take && m == thr && ties_left > 0) {
                take = true;
                ties_left--;
            }
            if (take) {
                col.push_back((int32_t)k);
                val.push_back(w[i * K + k]);
            }
        }
        rp[i + 1] = (int64_t)col.size();
    }
    return csr_from_rows(M, K, rp, col, &val, out);
}

tcaspmm_status tcaspmm_gen_rmat(int scale, int64_t edges, double a, double b, double c, int kind,
                                uint64_t seed, tcaspmm_csr *out)
{
    if (!out || scale < 1 || scale > 30 || edges < 0 || a < 0 || b < 0 || c < 0 || a + b + c > 1.0 ||
        (kind != 0 && kind != 1))
        return fail(TCASPMM_ERR_INVALID_ARG, "gen_rmat: bad arguments");
    const int64_t n = (int64_t)1 << scale;
    const int64_t extra = kind == 0 ? edges + n : 0;  // mirrored edges + self-loops
    std::vector<uint32_t> r(edges + extra), cc(edges + extra);
    const double ab = a + b, abc = a + b + c;
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < edges; e++) {
        uint32_t row = 0, col = 0;
        for (int l = 0; l < scale; l++) {
            const double u = rng_unit(seed, S_RMAT, (uint64_t)e * (uint64_t)scale + (uint64_t)l);
            const uint32_t bit = 1u << (scale - 1 - l);
            if (u < a) {
            } else if (u < ab) {
                col |= bit;
            } else if (u < abc) {
                row |= bit;
            } else {
                row |= bit;
                col |= bit;
            }
        }
        r[e] = row;
        cc[e] = col;
        if (kind == 0) {
            r[edges + e] = col;
            cc[edges + e] = row;
        }
    }
    if (kind == 0)
        for (int64_t i = 0; i < n; i++) {
            r[2 * edges + i] = (uint32_t)i;
            cc[2 * edges + i] = (uint32_t)i;
        }
    std::vector<int64_t> rp;
    std::vector<int32_t> col;
    pairs_to_csr(n, r, cc, &rp, &col);
    r.clear(); r.shrink_to_fit();
    cc.clear(); cc.shrink_to_fit();
    std::vector<float> val(col.size());
    if (kind == 0) {
        std::vector<double> isq(n);
        for (int64_t i = 0; i < n; i++) isq[i] = 1.0 / std::sqrt((double)(rp[i + 1] - rp[i]));
#pragma omp parallel for schedule(dynamic, 4096)
        for (int64_t i = 0; i < n; i++)
            for (int64_t j = rp[i]; j < rp[i + 1]; j++) val[j] = (float)(isq[i] * isq[col[j]]);
    } else {
#pragma omp parallel for schedule(dynamic, 4096)
        for (int64_t i = 0; i < n; i++) {
            const float inv = 1.0f / (float)std::max<int64_t>(1, rp[i + 1] - rp[i]);
            for (int64_t j = rp[i]; j < rp[i + 1]; j++) val[j] = inv;
        }
    }
    return csr_from_rows(n, n, rp, col, &val, out);
}

tcaspmm_status tcaspmm_gen_skew(int64_t n, int64_t hubs, int64_t hub_nnz, double lambda, uint64_t seed,
                                tcaspmm_csr *out)
{
    if (!out || n < 1 || hubs < 0 || hubs > n || hub_nnz < 0 || hub_nnz > n || lambda < 0 || lambda > 64)
        return fail(TCASPMM_ERR_INVALID_ARG, "gen_skew: bad arguments");
    const int64_t stride = hubs ? n / hubs : n + 1;
    auto is_hub = [&](int64_t i) { return hubs && i % stride == 0 && i / stride < hubs; };
    std::vector<int64_t> cnt(n + 1, 0);
    const double el = std::exp(-lambda);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        if (is_hub(i)) {
            cnt[i + 1] = hub_nnz;
            continue;
        }
        // Poisson(lambda) by the product-of-uniforms method (Knuth, TAOCP vol. 2).
        int64_t k = 0;
        double p = rng_unit(seed, S_POIS, (uint64_t)i * 128);
        while (p > el && k < 127) {
            k++;
            p *= rng_unit(seed, S_POIS, (uint64_t)i * 128 + (uint64_t)k);
        }
        cnt[i + 1] = k;
    }
    for (int64_t i = 0; i < n; i++) cnt[i + 1] += cnt[i];
    std::vector<int32_t> col(cnt[n]);
    std::vector<int64_t> fill(n, 0);
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t i = 0; i < n; i++) {
        const int64_t want = cnt[i + 1] - cnt[i];
        if (!want) continue;
        std::vector<int32_t> cs;
        cs.reserve(want + 16);
        uint64_t draw = 0;
        // Draw until `want` distinct columns (hub rows) or take `want` draws
        // deduplicated (ordinary rows, where a repeat is ~1e-7 likely).
        const uint64_t base = (uint64_t)i << 24;
        while ((int64_t)cs.size() < want) {
            const int64_t need = want - (int64_t)cs.size();
            for (int64_t q = 0; q < need; q++)
                cs.push_back((int32_t)(rng_u64(seed, S_COL, base + draw++) % (uint64_t)n));
            std::sort(cs.begin(), cs.end());
            cs.erase(std::unique(cs.begin(), cs.end()), cs.end());
            if (!is_hub(i)) break;
        }
        fill[i] = (int64_t)cs.size();
        std::copy(cs.begin(), cs.end(), col.begin() + cnt[i]);
    }
    // Compact rows that lost a repeated column.
    std::vector<int64_t> rp(n + 1, 0);
    for (int64_t i = 0; i < n; i++) rp[i + 1] = rp[i] + fill[i];
    if (rp[n] != cnt[n]) {
        std::vector<int32_t> c2(rp[n]);
        for (int64_t i = 0; i < n; i++) std::copy(col.begin() + cnt[i], col.begin() + cnt[i] + fill[i], c2.begin() + rp[i]);
        col.swap(c2);
    }
    std::vector<float> val(rp[n]);
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < rp[n]; j++) val[j] = (float)(2.0 * rng_unit(seed, S_UVAL, (uint64_t)j) - 1.0);
    return csr_from_rows(n, n, rp, col, &val, out);
}

}  // extern "C"
