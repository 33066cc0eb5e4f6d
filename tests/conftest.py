import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "granite-speech-4.1-2b-nar-turbo_b200")
for _p in (ROOT, PKG, os.path.dirname(os.path.abspath(__file__))):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def pytest_sessionstart(session):
    # the library is built ahead of time; rebuild only if a source is newer than the .so
    from granite_conv_b200 import build
    if build.needs_build():
        build.build()
