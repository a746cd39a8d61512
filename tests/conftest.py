import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    # Temporary files of the tests (tmp_path) stay inside the repository tree.
    if not config.option.basetemp:
        config.option.basetemp = os.path.join(ROOT, ".pytest_tmp")
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "needs_ref: needs the reference build in oracle/_ref")
    # The parity tests need the oracle: build it if this tree has not been built yet.
    oracle_so = os.path.join(ROOT, "oracle", "_build", "libmpk_oracle.so")
    if not os.path.exists(oracle_so):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True)


@pytest.fixture(scope="session")
def mpk_lib():
    import mix_precision_kernel_b200 as mpk
    from mix_precision_kernel_b200 import build

    if not os.path.exists(mpk.library_path()):
        build.build()
    return mpk


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    return torch.device("cuda", 0)


@pytest.fixture
def whole_tiles(mpk_lib):
    """Runs a test under the whole-tile GEMM schedule (every D element summed in
    one K order, as the on-chip kernel and any sharding of the same tiles do), and
    restores the previous schedule afterwards."""
    prev = mpk_lib.set_gemm_schedule(mpk_lib.SCHEDULE_TILES)
    yield mpk_lib
    mpk_lib.set_gemm_schedule(prev)
