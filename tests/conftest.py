import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs through the C-ABI library")


@pytest.fixture(scope="session")
def bundled():
    return dict(np.load(os.path.join(GOLDEN, "bundled_smtx.npz")))


@pytest.fixture(scope="session")
def small_cases():
    d = np.load(os.path.join(GOLDEN, "small_csr.npz"))
    cases = []
    for t in range(int(d["ncases"])):
        m, k, n = (int(x) for x in d[f"c{t}_shape"])
        cases.append(dict(M=m, K=k, N=n, dense=d[f"c{t}_dense"], row_ptr=d[f"c{t}_row_ptr"], col=d[f"c{t}_col"],
                          val=d[f"c{t}_val_bits"].view(np.float16), B=d[f"c{t}_B"], C=d[f"c{t}_C"]))
    return cases


@pytest.fixture()
def bundled_smtx_path(tmp_path, bundled):
    """The reference's bundled .smtx, byte for byte, written from the fixture."""
    p = tmp_path / "body_decoder_layer_2_ffn_conv1.smtx"
    p.write_bytes(bundled["smtx_text"].tobytes())
    return str(p)
