"""Pin the CPU oracle against fixtures made by the reference's own host code
(smtx_input_to_Dense + convert_dense_to_csr + naive_gemm; tests/golden/make_golden.py)."""
import numpy as np

import oracle


def test_oracle_smtx_reader_matches_reference_loader(bundled, bundled_smtx_path):
    M, K, rp, col = oracle.smtx_read(bundled_smtx_path)
    assert (M, K) == (int(bundled["M"]), int(bundled["K"]))
    np.testing.assert_array_equal(rp, bundled["row_ptr"])
    np.testing.assert_array_equal(col, bundled["col"])
    # The reference stores 1.0 for every nonzero (src/file_input.cu:189).
    assert np.all(bundled["val_bits"].view(np.float16) == 1.0)


def test_oracle_integer_known_answer_is_exact(bundled):
    vals = bundled["val_bits"].view(np.float16).astype(np.float32)
    C = oracle.spmm_f64(bundled["row_ptr"], bundled["col"], vals, bundled["B_int"].astype(np.float32))
    # naive_gemm's fp32 sums of small integers are exact, so equality is exact.
    np.testing.assert_array_equal(C, bundled["C_int"].astype(np.float64))


def test_oracle_random_b_matches_reference_gemm(bundled):
    vals = bundled["val_bits"].view(np.float16).astype(np.float32)
    C = oracle.spmm_f64(bundled["row_ptr"], bundled["col"], vals, bundled["B_rand"].astype(np.float32))
    ref = bundled["C_rand"].astype(np.float64)
    assert oracle.rel_l2(C, ref) < 1e-6  # naive_gemm accumulates in fp32
    np.testing.assert_allclose(C, ref, rtol=1e-5, atol=1e-4)


def test_oracle_small_cases_match_reference(small_cases):
    for c in small_cases:
        C = oracle.spmm_f64(c["row_ptr"], c["col"], c["val"].astype(np.float32), c["B"].astype(np.float32))
        assert oracle.rel_l2(C, c["C"]) < 1e-6
        np.testing.assert_allclose(C, c["C"], rtol=1e-4, atol=1e-4)
        # the CSR the reference built is the dense matrix's nonzeros, row-major
        dense = np.zeros((c["M"], c["K"]), np.float16)
        for i in range(c["M"]):
            dense[i, c["col"][c["row_ptr"][i]:c["row_ptr"][i + 1]]] = c["val"][c["row_ptr"][i]:c["row_ptr"][i + 1]]
        np.testing.assert_array_equal(dense, c["dense"])


def test_oracle_f32_loop_close_to_f64(small_cases):
    for c in small_cases:
        args = (c["row_ptr"], c["col"], c["val"].astype(np.float32), c["B"].astype(np.float32))
        assert oracle.rel_l2(oracle.spmm_f32(*args, threads=2), oracle.spmm_f64(*args)) < 1e-6


def test_oracle_row_sample_matches_full(small_cases):
    c = small_cases[0]
    args = (c["row_ptr"], c["col"], c["val"].astype(np.float32), c["B"].astype(np.float32))
    full = oracle.spmm_f32(*args)
    rows = np.array([3, 0, 36, 17])
    np.testing.assert_array_equal(oracle.spmm_f32_rows(rows, *args), full[rows])
