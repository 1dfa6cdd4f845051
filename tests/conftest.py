"""Test configuration: import paths and the `gpu` marker.

`-m gpu` tests need a CUDA device (a B200) and call the sm_100a library through
its C-ABI; everything else runs on CPU.
"""
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent
for p in (ROOT / "nest-splatting_b200", ROOT, ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); calls libnest_b200.so")
    config.addinivalue_line("markers", "slow: full-size parity case (minutes of oracle time)")
