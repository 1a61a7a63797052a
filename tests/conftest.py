import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")


def pytest_sessionstart(session):
    # The CPython host extensions (_hostpath, _chess; g++, a few seconds) are
    # built when absent or older than their sources, so the CPU tests that
    # import them run in a fresh checkout.
    try:
        from imba_chess_b200.build import build_host

        build_host()
    except Exception:  # the tests that need them report the import error
        pass
