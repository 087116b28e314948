import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    # GPU tests are selected with `-m gpu` and fail (not skip) without a device.
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
